"""Alias tables and decision log masses against the restatement and the reference's own kernels.

The alias table must be identical entry for entry (float64 thresholds, int32 aliases, the consumed
scaled weights) to both.  The log masses must be bit-identical to the reference kernel (fp32, CUDA
logf, --fmad=false) and within a few ulps of the restatement, whose logf is the C library's.
"""

import time

import numpy as np
import pytest
import torch

import build_ref
import oracle as O

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
REF_ALIAS = build_ref.load("ref_alias_table")
REF_BRANCH = build_ref.load("ref_branching_metadata")


def _scaled(log_weights):
    w = log_weights.double()
    return (torch.exp(w - torch.logsumexp(w, 0)) * w.numel()).contiguous()


CASES = {
    "tiny_underflow": torch.tensor([-1000.0, -3.0, -1.0, 0.0], dtype=torch.float64),
    "linspace_65536": torch.linspace(-40, 0, 65_536, dtype=torch.float64),
    "random_100k": torch.from_numpy(np.random.default_rng(3).normal(0, 3, 100_000)),
    "uniform_4096": torch.zeros(4096, dtype=torch.float64),
    "one": torch.zeros(1, dtype=torch.float64),
    "spiky_777": torch.from_numpy(np.where(np.arange(777) % 50 == 0, 5.0, -2.0)),
}


@pytest.mark.parametrize("name", list(CASES))
def test_alias_table_matches_restatement(name):
    from pbg_b200.branching import build_alias_table

    scaled = _scaled(CASES[name]).to(DEV)
    prob, alias, consumed = O.alias_table(scaled.cpu().numpy())
    p = torch.empty_like(scaled)
    a = torch.empty(scaled.numel(), dtype=torch.int32, device=DEV)
    s = scaled.clone()
    build_alias_table(s, p, a)
    torch.cuda.synchronize()
    assert np.array_equal(p.cpu().numpy(), prob)
    assert np.array_equal(a.cpu().numpy(), alias)
    assert np.array_equal(s.cpu().numpy(), consumed)


@pytest.mark.skipif(REF_ALIAS is None, reason="oracle/_ref alias operator not built")
@pytest.mark.parametrize("name", ["tiny_underflow", "random_100k", "spiky_777"])
def test_alias_table_matches_reference_kernel(name):
    from pbg_b200.branching import build_alias_table

    scaled = _scaled(CASES[name]).to(DEV)
    n = scaled.numel()
    p_ref, a_ref, s_ref = torch.empty_like(scaled), torch.empty(n, dtype=torch.int32, device=DEV), scaled.clone()
    REF_ALIAS.build_alias_table(s_ref, p_ref, a_ref, torch.empty(n, dtype=torch.int64, device=DEV),
                                torch.empty(n, dtype=torch.int64, device=DEV))
    p, a, s = torch.empty_like(scaled), torch.empty(n, dtype=torch.int32, device=DEV), scaled.clone()
    build_alias_table(s, p, a)
    torch.cuda.synchronize()
    assert torch.equal(p, p_ref) and torch.equal(a, a_ref) and torch.equal(s, s_ref)


def test_alias_table_preserves_mass_like_the_reference_test():
    # pbg tests/test_branched_sampled_modes.py:404-425
    from pbg_b200.branching import alias_table

    log_weight = torch.tensor([-1000.0, -3.0, -1.0, 0.0], dtype=torch.float64, device=DEV)
    threshold, alias = alias_table(log_weight)
    observed = threshold / 4
    observed.scatter_add_(0, alias.to(torch.int64), (1 - threshold) / 4)
    torch.testing.assert_close(observed, torch.softmax(log_weight, 0), atol=1.0e-15, rtol=1.0e-12)


def _tree(n, seed, max_depth_chain=False):
    rng = np.random.default_rng(seed)
    parent = np.full(n, -1, np.int32)
    for v in range(1, n):
        if max_depth_chain:
            parent[v] = v - 1 if rng.random() < 0.97 else -1
        elif rng.random() > 0.02:
            parent[v] = rng.integers(max(0, v - 50), v)
    degree = rng.integers(1, 8, n).astype(np.int32)
    return parent, degree


@pytest.mark.parametrize("n,chain", [(1, False), (1000, False), (200_000, False), (3000, True)])
def test_decision_log_mass_matches_restatement(n, chain):
    from pbg_b200.branching import decision_log_mass

    parent, degree = _tree(n, n + int(chain), chain)
    ref, code = O.decision_log_mass(parent, degree)
    failure = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = decision_log_mass(torch.from_numpy(parent).to(DEV), torch.from_numpy(degree).to(DEV), failure)
    assert code == 0 and int(failure.item()) == 0
    # the restatement's logf is the C library's, the kernels' is CUDA's: a few ulps along a path;
    # bit-exactness is checked against the reference's own kernel (same CUDA logf) below
    np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=2e-6, atol=1e-6)


@pytest.mark.parametrize("bad", ["forward_parent", "zero_degree"])
def test_decision_log_mass_reports_first_failure(bad):
    from pbg_b200.branching import decision_log_mass

    parent, degree = _tree(500, 7)
    if bad == "forward_parent":
        parent[300] = 400
        parent[350] = 351
    else:
        degree[parent[200]] = 0
    ref, code = O.decision_log_mass(parent, degree)
    failure = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = decision_log_mass(torch.from_numpy(parent).to(DEV), torch.from_numpy(degree).to(DEV), failure)
    assert int(failure.item()) == code != 0
    good = np.isfinite(ref)  # nodes the sequential loop wrote before it stopped
    np.testing.assert_allclose(out.cpu().numpy()[good], ref[good], rtol=2e-6, atol=1e-6)


@pytest.mark.skipif(REF_BRANCH is None, reason="oracle/_ref branching operator not built")
def test_decision_log_mass_matches_reference_kernel():
    from pbg_b200.branching import decision_log_mass

    parent, degree = _tree(50_000, 11)
    p, d = torch.from_numpy(parent).to(DEV), torch.from_numpy(degree).to(DEV)
    f_ref = torch.zeros(1, dtype=torch.int32, device=DEV)
    ref = REF_BRANCH.decision_log_mass(p, d, f_ref)
    f = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = decision_log_mass(p, d, f)
    torch.cuda.synchronize()
    assert torch.equal(out, ref) and int(f.item()) == int(f_ref.item()) == 0


def _device_us(fn, reps=5):
    fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(reps):
        torch.cuda._sleep(1_000_000)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b) * 1e3)
    return sorted(times)[reps // 2]


@pytest.mark.skipif(REF_ALIAS is None or REF_BRANCH is None, reason="oracle/_ref operators not built")
def test_timing_against_reference_single_thread_kernels():
    from pbg_b200.branching import build_alias_table, decision_log_mass

    n = 65_536
    scaled = _scaled(torch.linspace(-40, 0, n, dtype=torch.float64)).to(DEV)
    p, a = torch.empty_like(scaled), torch.empty(n, dtype=torch.int32, device=DEV)
    small, large = torch.empty(n, dtype=torch.int64, device=DEV), torch.empty(n, dtype=torch.int64, device=DEV)
    ref_us = _device_us(lambda: REF_ALIAS.build_alias_table(scaled.clone(), p, a, small, large))
    ours_us = _device_us(lambda: build_alias_table(scaled.clone(), p, a))
    parent, degree = _tree(200_000, 5)
    pp, dd = torch.from_numpy(parent).to(DEV), torch.from_numpy(degree).to(DEV)
    fail = torch.zeros(1, dtype=torch.int32, device=DEV)
    ref_mass_us = _device_us(lambda: REF_BRANCH.decision_log_mass(pp, dd, fail))
    ours_mass_us = _device_us(lambda: decision_log_mass(pp, dd, fail))
    print(f"\nalias table n={n}: reference {ref_us:.1f} us, pbg_b200 {ours_us:.1f} us")
    print(f"decision log mass n=200000: reference {ref_mass_us:.1f} us, pbg_b200 {ours_mass_us:.1f} us")
    assert ours_us < ref_us and ours_mass_us < ref_mass_us
