"""Deterministic poker-model parameters by name (shared by the golden generator and the tests).

Every parameter is drawn from a numpy generator seeded by the CRC32 of its name:
weights (2-D) ~ N(0, 1/fan_in), biases and embeddings ~ N(0, 0.05), LayerNorm gains
1 + N(0, 0.05), attention temperatures' theta ~ N(log(expm1(0.5)), 0.1).  The values are
rounded to bf16 and stored back as fp32, so the fp32 reference forward and the bf16 tensor-core
path start from identical weights.
"""

from __future__ import annotations

import math
import zlib

import numpy as np

CONFIG = dict(d_model=128, n_heads=4, layers=2, m_raise=4, k_act=7, max_players=2, class_embedding_dim=8,
              ffn_hidden=256, max_history_tokens=16, folder_beta_rank=2)
RANKS = 4


def _bf16_round(x: np.ndarray) -> np.ndarray:
    bits = x.astype(np.float32).view(np.uint32)
    rounded = (bits + 0x7FFF + ((bits >> 16) & 1)) & 0xFFFF0000
    return rounded.view(np.float32)


def parameter(name: str, shape: tuple[int, ...]) -> np.ndarray:
    rng = np.random.default_rng(zlib.crc32(name.encode()))
    if name.endswith("theta"):
        value = rng.normal(math.log(math.expm1(0.5)), 0.1, shape)
    elif (name.endswith("norm.weight") or ".norm.weight" in name or name.startswith("layer_norms")
          or name.startswith("final_norm")) and name.endswith("weight") and len(shape) == 1:
        value = 1.0 + rng.normal(0.0, 0.05, shape)
    elif len(shape) == 2 and "embedding" not in name and name != "anchor_tokens":
        value = rng.normal(0.0, 1.0 / math.sqrt(shape[1]), shape)
    else:
        value = rng.normal(0.0, 0.05, shape)
    return _bf16_round(np.asarray(value, dtype=np.float32))

# the postflop run has three seats (one folded), so the table holds up to three players
POSTFLOP_CONFIG = dict(CONFIG, max_players=3)


SKETCH_PROBES = 4


def probe(name: str, shape: tuple[int, ...]) -> np.ndarray:
    """Seeded N(0, I) probe vectors [SKETCH_PROBES, numel] of a parameter (float64): the projections of
    its gradient onto them sketch the gradient (each projection's error is about the norm of the
    gradient's error)."""

    rng = np.random.default_rng(zlib.crc32(("probe:" + name).encode()))
    return rng.standard_normal((SKETCH_PROBES, int(np.prod(shape))))
