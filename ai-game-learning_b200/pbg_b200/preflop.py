"""The preflop class-row policy/value network on this build's kernels.

``PreflopModel.forward`` computes pbg/games/poker/model/preflop.py:472-693
(``PreflopEncoder.forward``) with the shared trunk and readout of
pbg/games/poker/model/shared.py, from the reference's own parameters (a
dict keyed by the two modules' ``state_dict`` names).  Every dense map of the
trunk and readout runs on ``pbg_linear_bf16`` (tcgen05, bf16 operands, fp32
accumulation; K zero-padded to 64 and N to 128 once at bind time), every
LayerNorm on ``pbg_layernorm``, every attention on ``pbg_attention_bf16``.
FamilyFFN's common and static maps become one GEMM over the concatenated
inputs with GELU in its epilogue.  The residual stream stays fp32; the
token assembly (embeddings, the 1- and 6-wide affine maps of the scalars),
the incidence mass reductions (fp32 batched GEMMs, as the reference keeps
them) and the small elementwise steps are torch operations on the device.

In training mode (``FamilyModel.train()``, after ``bind_parameters`` with leaf
tensors) the same forward runs with every native step as an autograd function
of ``pbg_b200.model_train`` (the learner step's backward); embedding rows are
then one-hot products (``lookup``) so that their gradients are GEMMs.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
from torch import Tensor
from torch.nn import functional as F

from ._native import NativeError, call, ptr, rows_ptr, stream
from .model import attention, linear, linear_ex
from .model_train import attention_train, incidence_combine_train, layernorm_train, linear_train, q_scale_of


@dataclass(frozen=True)
class PreflopConfig:
    """The fields of pbg PokerModelConfig (preflop.py:31-54) the forward uses."""

    d_model: int = 256
    n_heads: int = 8
    layers: int = 6
    m_raise: int = 4
    k_act: int = 7
    s_min: float = 0.02
    max_players: int = 9
    class_embedding_dim: int = 32
    ffn_hidden: int | None = None
    max_history_tokens: int = 256
    folder_beta_rank: int = 16
    folder_line_dim: int = 8
    eps: float = 1e-8

    @property
    def hidden(self) -> int:
        return self.ffn_hidden or 4 * self.d_model


def class_geometry(rank_count: int):
    """pbg/games/poker/cards.py DeckGeometry for the preflop network: combo cards, class of each combo,
    class sizes, the orbit-averaged card incidence [classes, cards] and the overlap scalars (preflop.py:234-253)."""

    deck = 4 * rank_count
    first = 52 - deck
    combos = [(i, j) for i in range(deck) for j in range(i + 1, deck)]

    def klass(a, b):
        ra, rb = (a + first) // 4 - (13 - rank_count), (b + first) // 4 - (13 - rank_count)
        high, low = max(ra, rb), min(ra, rb)
        hp, lp = rank_count - 1 - high, rank_count - 1 - low
        suited_or_pair = ra == rb or (a + first) % 4 == (b + first) % 4
        return hp * rank_count + lp if suited_or_pair else lp * rank_count + hp

    classes = rank_count * rank_count
    of_combo = torch.tensor([klass(a, b) for a, b in combos], dtype=torch.long)
    sizes = torch.bincount(of_combo, minlength=classes).to(torch.float32)
    orbit = torch.zeros((classes, deck), dtype=torch.float32)
    cards = torch.tensor(combos, dtype=torch.long)
    orbit.index_put_((of_combo[:, None].expand(-1, 2).reshape(-1), cards.reshape(-1)),
                     torch.ones(cards.numel(), dtype=torch.float32), accumulate=True)
    orbit = orbit / sizes[:, None]
    overlap = orbit @ orbit.T
    within = overlap.diagonal()
    cross = (overlap.sum(1) - within) / (classes - 1)
    return sizes, orbit, torch.stack((within, cross), dim=1)


@dataclass
class PolicyOutput:
    """preflop.py PolicyOutput: raw policy fields, values, and the optional public branching heads."""

    raw: dict
    v: Tensor
    t: Tensor | None = None
    c: Tensor | None = None


class _Binding:
    """Mode shared by a model's maps: ``training`` routes every map through its autograd function."""

    def __init__(self) -> None:
        self.training = False


class _Map:
    """A Linear bound for pbg_linear_bf16: bf16 weight padded to K % 64 == 0 and N % 128 == 0.

    ``source`` returns the map's fp32 (weight [n, k], bias [n] or None) from the model's parameters
    (the concatenation or slice of them for fused maps); in training mode (``binding.training``) the
    map runs as ``model_train.linear_train`` with those tensors as its autograd inputs, the padded bf16
    copy refreshed from them at every call."""

    def __init__(self, weight: Tensor, bias: Tensor | None, device, source=None, binding: _Binding | None = None) -> None:
        n, k = weight.shape
        self.n, self.k = n, k
        self.kp, self.np_ = -(-k // 64) * 64, -(-n // 128) * 128
        w = torch.zeros((self.np_, self.kp), dtype=torch.bfloat16, device=device)
        w[:n, :k] = weight.detach().to(device=device, dtype=torch.bfloat16)
        self.weight = w
        self.bias = None
        if bias is not None:
            b = torch.zeros(self.np_, dtype=torch.float32, device=device)
            b[:n] = bias.detach().to(device=device, dtype=torch.float32)
            self.bias = b
        self.source = source
        self.binding = binding

    def refresh(self, weight: Tensor, bias: Tensor | None) -> None:
        """Copy the fp32 weight / bias into the padded bf16 operand and fp32 bias."""

        self.weight[: self.n, : self.k].copy_(weight.detach())
        if self.bias is not None and bias is not None:
            self.bias[: self.n].copy_(bias.detach())

    def _training(self) -> bool:
        return self.binding is not None and self.binding.training

    def __call__(self, x: Tensor, activation: str | None = None) -> Tensor:
        lead = x.shape[:-1]
        rows = x.reshape(-1, x.shape[-1])
        if rows.shape[1] != self.kp:  # already padded operands (width kp) pass straight through
            rows = _padded(rows, self.kp)
        elif rows.dtype != torch.bfloat16:
            rows = rows.to(torch.bfloat16)
        if self._training():
            return linear_train(self, rows, activation).reshape(*lead, self.n)
        y = linear(rows if rows.is_contiguous() else rows.contiguous(), self.weight, self.bias, activation)
        if self.np_ != self.n:
            y = y[:, : self.n]
        return y.reshape(*lead, self.n)

    def apply(self, rows: Tensor, activation: str | None = None, *, row_scale: Tensor | None = None,
              residual: Tensor | None = None, residual_group: int = 1, out: Tensor | None = None,
              out_dtype: torch.dtype = torch.bfloat16) -> Tensor:
        """The map over a bf16 matrix of width kp (rows contiguous, any row stride) with the fused
        epilogue of ``linear_ex``: per-row scale, fp32 residual, fp32 or bf16 output."""

        if rows.ndim != 2 or rows.shape[1] != self.kp:
            raise NativeError("map operand must be a [rows, padded in] matrix")
        if self.np_ != self.n and (residual is not None or out is not None):
            raise NativeError("a fused residual or output buffer needs an unpadded output width")
        if self._training():
            if out is not None:
                raise NativeError("a map in training mode writes no caller buffer")
            return linear_train(self, rows, activation, row_scale=row_scale, residual=residual,
                                residual_group=residual_group, out_dtype=out_dtype)
        y = linear_ex(rows, self.weight, self.bias, activation, row_scale=row_scale, residual=residual,
                      residual_group=residual_group, out=out, out_dtype=out_dtype)
        return y if self.np_ == self.n else y[:, : self.n]


def _padded(x: Tensor, width: int) -> Tensor:
    """x as a contiguous bf16 matrix zero-padded to ``width`` columns (the map's padded K): one pass
    that converts into the padded buffer, the pad columns filled alone."""

    x = x.reshape(-1, x.shape[-1])
    if x.shape[1] == width:
        return x.to(torch.bfloat16).contiguous()
    if x.requires_grad and torch.is_grad_enabled():  # training: a pad whose backward is a slice, not a copy
        return F.pad(x.to(torch.bfloat16), (0, width - x.shape[1]))
    out = torch.empty((x.shape[0], width), dtype=torch.bfloat16, device=x.device)
    out[:, : x.shape[1]] = x
    out[:, x.shape[1]:] = 0
    return out


def lookup(table: Tensor, index: Tensor) -> Tensor:
    """``table[index]``: rows of an embedding table.  While the table takes a gradient this is the one-hot
    product ``one_hot(index) @ table`` (exact in fp32: one nonzero term per output), so that its backward is
    a GEMM rather than an index scatter serialised over the many repeats of a few table rows."""

    if table.requires_grad and torch.is_grad_enabled():
        rows = F.one_hot(index.reshape(-1), table.shape[0]).to(table.dtype) @ table
        return rows.view(*index.shape, table.shape[1])
    return table[index]


def _affine_rows(affine, feats: Tensor, seat_terms: Tensor, rows_per_seat: int) -> Tensor:
    """affine(feats) + seat_terms broadcast over each seat's rows, in fp32: one map whose epilogue adds
    the per-seat terms (residual row m // rows_per_seat) and writes fp32, where the map's width allows
    it; otherwise the map, then the broadcast addition."""

    lead = feats.shape[:-1]
    if affine.np_ != affine.n:
        return affine(feats).float() + seat_terms[..., None, :]
    rows = _padded(feats, affine.kp)
    terms = seat_terms.reshape(-1, affine.n).float().contiguous()
    return affine.apply(rows, residual=terms, residual_group=rows_per_seat, out_dtype=torch.float32).view(
        *lead, affine.n)


def _cat_maps(first: Tensor, second: Tensor) -> Tensor:
    return torch.cat((first, second), dim=1)


class FamilyModel:
    """The shared trunk and readout (shared.py) bound to this build's kernels; a family adds its tokens.

    ``family`` selects FamilyFFN's static adapter ("pre" or "post", shared.py:19-33).
    """

    family = "pre"

    def __init__(self, cfg: PreflopConfig, rank_count: int, params: dict[str, Tensor], device) -> None:
        if cfg.d_model != cfg.n_heads * 32:
            raise NativeError("this build's attention core takes heads of width 32")
        self.cfg, self.device = cfg, torch.device(device)
        self.rank_count = rank_count
        self.n_cards = 4 * rank_count
        p = {k: v.to(self.device, torch.float32) for k, v in params.items()}
        self.p = p
        self.binding = _Binding()
        self._maps: list[_Map] = []

        def lin(name, bias=True):
            return self._map(p[name + ".weight"], p.get(name + ".bias") if bias else None,
                             lambda: (self.p[name + ".weight"], self.p.get(name + ".bias") if bias else None))

        self._lin = lin
        self.layers = []
        for i in range(cfg.layers):
            inc = f"incidence_residuals.{i}"
            ffn = f"layer_ffns.{i}"
            mha = f"attentions.{i}"
            parts = (f"{inc}.query.weight", f"{inc}.identical.weight", f"{inc}.own.weight")
            halves = (f"{ffn}.common.weight", f"{ffn}.static.{self.family}.weight")
            self.layers.append({
                "source": lin(f"{inc}.source", False),
                # query(n) + identical(other_equal) + own(own_card) as one map over [n | other_equal | own_card]
                "inc_in": self._map(torch.cat([p[n] for n in parts], dim=1), p[f"{inc}.query.bias"],
                                    lambda parts=parts, inc=inc: (torch.cat([self.p[n] for n in parts], dim=1),
                                                                  self.p[f"{inc}.query.bias"])),
                "inc_out": lin(f"{inc}.output"),
                "w_qkv": lin(f"{mha}.w_qkv"),
                "w_o": lin(f"{mha}.w_o"),
                # FamilyFFN (shared.py:19-33): common(x) + static[family](s) as one map over [x, s]
                "ffn_in": self._map(_cat_maps(p[halves[0]], p[halves[1]]), p[f"{ffn}.common.bias"],
                                    lambda halves=halves, ffn=ffn: (_cat_maps(self.p[halves[0]], self.p[halves[1]]),
                                                                    self.p[f"{ffn}.common.bias"])),
                "ffn_out": lin(f"{ffn}.output"),
            })
        self._bind_layer_parameters()

        def ffn(name):
            return (lin(name + ".w1"), lin(name + ".w2"), name)

        self.actor_seat_features = ffn("actor_seat_features")
        self.seat_features = ffn("seat_features")
        self.global_features = ffn("global_features")
        self.type_features = ffn("type_features")
        self.raise_features = ffn("raise_features")
        self.value_features = ffn("value_head.features")
        self.type_head = lin("type_head.affine")
        self.mixture_affine = lin("raise_head.mixture_affine")
        self.allin_affine = lin("raise_head.allin_affine")
        self.value_affine = lin("value_head.affine")
        # PublicBranchingHeads (heads.py:83-104), present when the configuration enables them: one
        # public row per decision, evaluated in fp32 (the cost head is an exponential of its logit)
        self.branching = "branching_heads.public_features.w1.weight" in p
        self._factored: dict = {}

    # ------------------------------------------------------------ parameters and modes
    def _map(self, weight: Tensor, bias: Tensor | None, source) -> _Map:
        m = _Map(weight, bias, self.device, source, self.binding)
        self._maps.append(m)
        return m

    def _bind_layer_parameters(self) -> None:
        """The LayerNorm pairs and head score scales of every layer, from the current parameters."""

        p = self.p
        for i, layer in enumerate(self.layers):
            inc = f"incidence_residuals.{i}"
            layer["ln"] = (p[f"layer_norms.{i}.weight"], p[f"layer_norms.{i}.bias"])
            layer["inc_ln"] = (p[f"{inc}.norm.weight"], p[f"{inc}.norm.bias"])
            layer["theta"] = p[f"attentions.{i}.theta"]
            layer["q_scale"] = q_scale_of(p[f"attentions.{i}.theta"].detach()).contiguous()
        self.final_ln = (p["final_norm.weight"], p["final_norm.bias"])

    def bind_parameters(self, params: dict[str, Tensor]) -> None:
        """Use ``params`` (this model's names, e.g. leaf views of a flat fp32 master) as the parameters."""

        missing = sorted(set(self.p) - set(params))
        if missing:
            raise KeyError(f"parameters missing: {missing[:4]}")
        self.p = {name: params[name] for name in self.p}
        self._bind_layer_parameters()
        self.sync_weights()

    def sync_weights(self) -> None:
        """Refresh every map's bf16 operand and the score scales from the current parameters (after an
        optimizer step, before an inference-mode forward)."""

        with torch.no_grad():
            for m in self._maps:
                if m.source is not None:
                    m.refresh(*m.source())
            for layer in self.layers:
                layer["q_scale"] = q_scale_of(layer["theta"].detach()).contiguous()

    def train(self, mode: bool = True) -> "FamilyModel":
        """Training mode: every native step runs as an autograd function (model_train)."""

        self.binding.training = bool(mode)
        if not mode:
            self.sync_weights()
        return self

    # ------------------------------------------------------------ kernels
    def _ln(self, x: Tensor, gain_bias, out: Tensor | None = None) -> Tensor:
        """LayerNorm -> bf16, into `out` (rows of any stride, e.g. a slice of a wider operand) if given."""

        if self.binding.training:
            if out is not None:
                raise NativeError("a LayerNorm in training mode writes no caller buffer")
            return layernorm_train(x, gain_bias[0], gain_bias[1])
        d = x.shape[-1]
        rows = x.reshape(-1, d).contiguous()
        if out is None:
            out = torch.empty(rows.shape, dtype=torch.bfloat16, device=x.device)
            target, ldy = out, d
        else:
            target, ldy = out, out.stride(-2)
        call("pbg_layernorm", rows.shape[0], d, ptr(rows), int(rows.dtype == torch.bfloat16), ptr(gain_bias[0]),
             ptr(gain_bias[1]), 1e-5, ctypes.c_void_p(target.data_ptr()), 1, ldy, stream(x.device))
        return out.reshape(x.shape)  # a view also for a strided slice (only leading dimensions split)

    def _ffn(self, maps, x: Tensor) -> Tensor:
        return maps[1](maps[0](x, "gelu"))

    def _ffn_factored(self, maps, rows: Tensor, context: Tensor) -> Tensor:
        """primitives.py:62-71 forward_factored: the context projected once per decision."""

        split = rows.shape[-1]
        name = maps[2]
        key = (name, split)
        if key not in self._factored:
            wn, bn = name + ".w1.weight", name + ".w1.bias"
            w1, b1 = self.p[wn], self.p[bn]
            self._factored[key] = (self._map(w1[:, :split], b1, lambda: (self.p[wn][:, :split], self.p[bn])),
                                   self._map(w1[:, split:], None, lambda: (self.p[wn][:, split:], None)))
        row_map, ctx_map = self._factored[key]
        # the context projection is computed once per decision (fp32) and added to each of its rows in the
        # row map's epilogue, GELU fused there too
        batch, count, _ = rows.shape
        ctx = ctx_map.apply(_padded(context, ctx_map.kp), out_dtype=torch.float32)
        hidden = row_map.apply(_padded(rows.reshape(batch * count, -1), row_map.kp), "gelu", residual=ctx,
                               residual_group=count)
        return maps[1](hidden.view(batch, count, -1))

    def _ln_rows(self, x: Tensor, gain_bias, group_rows: int, out: Tensor) -> Tensor:
        """LayerNorm of the first ``group_rows`` tokens of every sequence of ``x`` [B, L, d] (fp32,
        contiguous) into ``out`` [B * group_rows, d] (bf16, rows contiguous, any row stride)."""

        batch, length, d = x.shape
        call("pbg_layernorm_rows", batch * group_rows, d, group_rows, ptr(x), 0, length * d, d, ptr(gain_bias[0]),
             ptr(gain_bias[1]), 1e-5, rows_ptr(out), 1, group_rows * out.stride(0), out.stride(0), stream(x.device))
        return out

    def _incidence(self, layer, x: Tensor, players: int, rows: int, mass: Tensor, incidence: Tensor,
                   identical_scale: Tensor, ffn_operand: Tensor) -> Tensor:
        """incidence.py:30-84 (IncidenceResidual.forward) on the private rows of the residual stream
        ``x`` [B, L, d]: LayerNorm into the staged operand [n | oe | own], the source map with the row
        mass fused as a row scale (fp32 out), the two fp32 card contractions, one combine pass (oe and
        own into the operand, oc as the query map's pre-GELU residual, oc^2 and oc*oe into the
        FamilyFFN operand ``ffn_operand`` [B, L, W]), the query/identical/own map with residual and
        GELU fused, and the output map.  Returns j, bf16 [B * players * rows, d]."""

        batch, length, d = x.shape
        count = batch * players * rows
        operand = torch.empty((count, 3 * d), dtype=torch.bfloat16, device=x.device)
        self._ln_rows(x, layer["inc_ln"], players * rows, operand[:, :d])
        source = layer["source"].apply(operand[:, :d], row_scale=mass, out_dtype=torch.float32)
        # the two fp32 card contractions as batched GEMMs over the [R, d] blocks of every (decision, seat),
        # with no permuted copies: a shared incidence [R, C] (class rows) or one per decision [B, R, C]
        if incidence.dim() == 2:
            blocks = source.view(batch * players, rows, d)
            card_acc = torch.matmul(incidence.t(), blocks)
            card_overlap = torch.matmul(incidence, card_acc)
        else:
            blocks = source.view(batch, players, rows, d)
            card_acc = torch.matmul(incidence.transpose(1, 2)[:, None], blocks)
            card_overlap = torch.matmul(incidence[:, None], card_acc)
        card_overlap = card_overlap.contiguous()
        other_card = torch.empty_like(source)
        width = ffn_operand.shape[-1]
        call("pbg_incidence_combine", batch, players, rows, d, ptr(source), ptr(card_overlap), ptr(identical_scale),
             ptr(operand), 3 * d, d, 2 * d, ptr(other_card), ptr(ffn_operand), length * width, width, 2 * d, 3 * d,
             stream(x.device))
        hidden = layer["inc_in"].apply(operand, "gelu", residual=other_card)
        return layer["inc_out"].apply(hidden)

    def _trunk(self, x: Tensor, players: int, rows_per_seat: int, mass: Tensor, incidence: Tensor,
               identical_scale: Tensor, side: Tensor, key_bias: Tensor, key_mask: Tensor) -> Tensor:
        """The shared layers (preflop.py:614-641 / postflop.py:658-685): incidence residual, LayerNorm,
        biased attention with the residual add fused into the output map, FamilyFFN over
        [LN(x_hat) | j, oc^2, oc*oe | side] with the residual add fused into its output map."""

        if self.binding.training:
            return self._trunk_train(x, players, rows_per_seat, mass, incidence, identical_scale, side, key_bias,
                                     key_mask)
        cfg = self.cfg
        d = cfg.d_model
        batch, length, _ = x.shape
        rows_k = players * rows_per_seat
        # FamilyFFN operand [LN(x_hat) | j | oc^2 | oc*oe | side] in one bf16 buffer, padded to the map's K;
        # the side features (fixed across layers) and the zero rows of non-row tokens are written once
        width = self.layers[0]["ffn_in"].kp if self.layers else 0
        operand = torch.empty((batch, length, width), dtype=torch.bfloat16, device=x.device)
        side_width = side.shape[-1]
        operand[:, :rows_k, 4 * d: 4 * d + side_width] = side.reshape(batch, rows_k, side_width)
        # every layer writes LN(x_hat) into the first d columns of all tokens, and j, oc^2 and oc*oe into
        # the next 3d of the row tokens: what stays zero is filled once, alone
        operand[:, :rows_k, 4 * d + side_width:] = 0
        operand[:, rows_k:, d:] = 0
        mass_rows = mass.reshape(-1).to(torch.float32).contiguous()
        scale_rows = identical_scale.to(torch.float32).contiguous()
        x = x.contiguous()
        flat = operand.view(batch * length, width)
        for layer in self.layers:
            j = self._incidence(layer, x, players, rows_per_seat, mass_rows, incidence, scale_rows, operand)
            call("pbg_scatter_rows_bf16", batch * rows_k, d, rows_k, ptr(j), rows_ptr(flat[:, d: 2 * d]),
                 length * width, width, stream(x.device))
            nx = self._ln(x, layer["ln"])
            qkv = layer["w_qkv"](nx)
            attended = attention(qkv.contiguous(), cfg.n_heads, layer["q_scale"], key_bias, key_mask)
            x_hat = layer["w_o"].apply(attended.view(-1, d), residual=x.view(-1, d), out_dtype=torch.float32)
            self._ln(x_hat, layer["ln"], flat[:, :d])
            hidden = layer["ffn_in"].apply(flat, "gelu")
            x = layer["ffn_out"].apply(hidden, residual=x_hat, out_dtype=torch.float32).view(batch, length, d)
        return x

    def _incidence_train(self, layer, x: Tensor, players: int, rows: int, mass: Tensor, incidence: Tensor,
                         identical_scale: Tensor):
        """``_incidence`` as autograd steps (incidence.py:30-84): the LayerNorm, the source map with the
        row mass as its row scale, the fp32 card contractions, the seat sums (``incidence_combine_train``),
        the query/identical/own map with oc as its pre-GELU residual and the output map.  Returns j
        [B * players * rows, d] and the FamilyFFN features [oc^2 | oc * oe] [B, players * rows, 2d] (bf16)."""

        batch, length, d = x.shape
        count = batch * players * rows
        n = self._ln(x[:, : players * rows].reshape(count, d), layer["inc_ln"])
        source = layer["source"].apply(n, row_scale=mass, out_dtype=torch.float32)
        if incidence.dim() == 2:
            blocks = source.view(batch * players, rows, d)
            card_overlap = torch.matmul(incidence, torch.matmul(incidence.t(), blocks))
        else:
            blocks = source.view(batch, players, rows, d)
            card_overlap = torch.matmul(incidence[:, None], torch.matmul(incidence.transpose(1, 2)[:, None], blocks))
        pair, other_card, features = incidence_combine_train(source.view(batch, players, rows, d),
                                                             card_overlap.reshape(batch, players, rows, d),
                                                             identical_scale)
        hidden = layer["inc_in"].apply(torch.cat((n, pair), -1), "gelu", residual=other_card)
        j = layer["inc_out"].apply(hidden)
        return j, features.view(batch, players * rows, 2 * d)

    def _trunk_train(self, x: Tensor, players: int, rows_per_seat: int, mass: Tensor, incidence: Tensor,
                     identical_scale: Tensor, side: Tensor, key_bias: Tensor, key_mask: Tensor) -> Tensor:
        """``_trunk`` as autograd steps: the same maps, LayerNorms and attention core, the FamilyFFN operand
        assembled by concatenation instead of in place."""

        cfg = self.cfg
        d = cfg.d_model
        batch, length, _ = x.shape
        rows_k = players * rows_per_seat
        side_rows = side.reshape(batch, rows_k, -1).to(torch.bfloat16)
        mass_rows = mass.reshape(-1).detach().to(torch.float32).contiguous()
        # the FamilyFFN operand is assembled at the map's padded width: the columns after
        # [LN(x_hat) | j | oc^2 | oc*oe | side] and the row-only columns of the other tokens are zero
        width = self.layers[0]["ffn_in"].kp if self.layers else 0
        tail = width - 4 * d - side_rows.shape[-1]
        side_rows = torch.cat((side_rows, side_rows.new_zeros((batch, rows_k, tail))), -1) if tail else side_rows
        pad = torch.zeros((batch, length - rows_k, width - d), dtype=torch.bfloat16, device=x.device)
        x = x.contiguous()
        for layer in self.layers:
            j, features = self._incidence_train(layer, x, players, rows_per_seat, mass_rows, incidence,
                                                identical_scale)
            nx = self._ln(x, layer["ln"])
            qkv = layer["w_qkv"](nx)
            attended = attention_train(qkv, cfg.n_heads, q_scale_of(layer["theta"]), key_bias, key_mask)
            x_hat = layer["w_o"].apply(attended.view(-1, d), residual=x.view(-1, d), out_dtype=torch.float32)
            normed = self._ln(x_hat, layer["ln"]).view(batch, length, d)
            extra = torch.cat((torch.cat((j.view(batch, rows_k, d), features, side_rows), -1), pad), 1)
            hidden = layer["ffn_in"].apply(torch.cat((normed, extra), -1).view(batch * length, width), "gelu")
            x = layer["ffn_out"].apply(hidden, residual=x_hat, out_dtype=torch.float32).view(batch, length, d)
        return x

    def _head(self, head: "_Map", x: Tensor) -> Tensor:
        """A final affine head with fp32 output (the fields leave the network in fp32)."""

        lead = x.shape[:-1]
        return head.apply(_padded(x, head.kp), out_dtype=torch.float32).reshape(*lead, head.n)

    def _readout(self, actor_rows: Tensor, private_embedding: Tensor, anchors: Tensor, global_feature: Tensor):
        """shared.py:74-92 readout -> (raw policy fields, value)."""

        cfg = self.cfg
        rows = torch.cat((actor_rows, private_embedding), -1)
        context = torch.cat((anchors.flatten(1), global_feature), -1)
        z_type = self._ffn_factored(self.type_features, rows, context)
        z_raise = self._ffn_factored(self.raise_features, rows, context)
        raw = self._head(self.mixture_affine, z_raise)
        m = cfg.m_raise
        omega = torch.softmax(raw[..., :m], -1)
        mu = torch.sigmoid(raw[..., m:2 * m])
        s = F.softplus(raw[..., 2 * m:]) + cfg.s_min
        iota = torch.sigmoid(self._head(self.allin_affine, z_type)).squeeze(-1)
        value_features = self._ffn_factored(self.value_features, rows, context)
        value = self._head(self.value_affine, value_features).squeeze(-1)
        return {"type_logits": self._head(self.type_head, z_type), "omega": omega, "mu": mu, "s": s,
                "iota": iota}, value

    def _branching(self, global_feature: Tensor, public_mean: Tensor, padded_seats: Tensor):
        """heads.py:83-104 (PublicBranchingHeads) on [global feature, public mean, seat summaries]:
        (trace variance T, subtree cost C), fp32 [B]; (None, None) when the heads are absent."""

        if not self.branching:
            return None, None
        p = self.p

        def ffn(name: str, x: Tensor) -> Tensor:
            hidden = F.gelu(F.linear(x, p[name + ".w1.weight"], p[name + ".w1.bias"]))
            return F.linear(hidden, p[name + ".w2.weight"], p[name + ".w2.bias"])

        public = torch.cat((global_feature, public_mean, padded_seats.flatten(1)), -1).float()
        features = ffn("branching_heads.public_features", public)
        t_logit = F.linear(ffn("branching_heads.t_features", features), p["branching_heads.t_affine.weight"],
                           p["branching_heads.t_affine.bias"]).squeeze(-1)
        c_logit = F.linear(ffn("branching_heads.c_features", features), p["branching_heads.c_affine.weight"],
                           p["branching_heads.c_affine.bias"]).squeeze(-1)
        return torch.sigmoid(t_logit), torch.exp(c_logit.clamp(min=-30.0, max=30.0))


class PreflopModel(FamilyModel):
    """The preflop family (preflop.py): 169 class rows per seat, class geometry, class-row affine."""

    family = "pre"

    def __init__(self, cfg: PreflopConfig, rank_count: int, params: dict[str, Tensor], device) -> None:
        super().__init__(cfg, rank_count, params, device)
        self.class_row_affine = self._lin("class_row_affine")
        self.n_classes = rank_count * rank_count
        sizes, orbit, overlap = class_geometry(rank_count)
        self.class_sizes = sizes.to(self.device)
        self.class_card_geometry = orbit.to(self.device)
        self.class_overlap_scalars = overlap.to(self.device)

    # ------------------------------------------------------------ forward
    def _public_tokens(self, pub, seat_mask: Tensor, relative_seats: Tensor):
        """preflop.py:373-470."""

        p = self.p
        batch, players = seat_mask.shape
        dev = self.device
        groups = [pub["pot"][:, None], pub["stacks"], pub["committed"], pub["street"].float()[:, None],
                  pub["legality_summary"].float(), pub["n_ticks"].float()[:, None],
                  pub["raise_grid_bounds"].float()]
        kinds = [(1, 0), (players, 1), (players, 2), (1, 3), (pub["legality_summary"].shape[1], 4), (1, 5), (2, 6)]
        if pub.get("committed_street") is not None:
            groups.append(pub["committed_street"].float())
            kinds.append((players, 7))
        exact = [pub[k].float()[:, None] for k in ("call_amount", "current_bet", "min_raise_to", "max_raise_to",
                                                  "last_full_raise") if pub.get(k) is not None]
        if exact:
            groups.append(torch.cat(exact, 1))
            kinds.append((len(exact), 8))
        if pub.get("legal_action_mask") is not None:
            groups.append(pub["legal_action_mask"].float())
            kinds.append((pub["legal_action_mask"].shape[1], 9))
        if pub.get("raise_ticks") is not None:
            groups.append(pub["raise_ticks"].float())
            kinds.append((pub["raise_ticks"].shape[1], 10))
        scalars = torch.cat(groups, 1)
        type_ids = torch.cat([torch.full((n,), k, dtype=torch.long, device=dev) for n, k in kinds])
        w = p["public_scalar_affine.weight"][:, 0]
        token = scalars[..., None] * w + p["public_scalar_affine.bias"] + lookup(p["public_type_embedding.weight"], type_ids)
        seat_pos = lookup(p["seat_embedding.weight"], relative_seats)
        rest = scalars.shape[1] - 1 - 2 * players
        zeros = lambda n: torch.zeros((batch, n, self.cfg.d_model), device=dev)  # noqa: E731
        token = token + torch.cat((zeros(1), seat_pos, seat_pos, zeros(rest)), 1)
        valid = torch.cat((torch.ones((batch, 1), dtype=torch.bool, device=dev), seat_mask, seat_mask,
                           torch.ones((batch, rest), dtype=torch.bool, device=dev)), 1)
        h = pub.get("history")
        if h is not None and h["mask"].shape[1]:
            numeric = torch.stack([h[k].float() for k in ("amount", "pot_before", "call_amount", "current_bet",
                                                          "min_raise_to", "max_raise_to")], -1)
            ht = numeric @ p["history_numeric_affine.weight"].T + p["history_numeric_affine.bias"]
            ht = ht + lookup(p["history_action_embedding.weight"], h["action"].clamp(0, 3).long())
            ht = ht + lookup(p["history_street_embedding.weight"], h["street"].clamp(0, 3).long())
            ht = ht + p["history_position_embedding.weight"][: h["mask"].shape[1]][None]
            actor = h["actor"].clamp(0, players - 1).long()
            ht = ht + lookup(p["seat_embedding.weight"], relative_seats.gather(1, actor)) * (h["actor"] >= 0)[..., None]
            token = torch.cat((token, ht), 1)
            valid = torch.cat((valid, h["mask"].bool()), 1)
        mean = (token * valid[..., None]).sum(1) / valid.sum(1, keepdim=True)
        state = p["state_token"] + mean
        return (torch.cat((token, state[:, None]), 1),
                torch.cat((valid, torch.ones((batch, 1), dtype=torch.bool, device=dev)), 1))

    def forward(self, pub: dict, class_ranges: Tensor, class_mask: Tensor | None = None,
                actor_seat: Tensor | None = None, *, selected_private: Tensor | None = None):
        """preflop.py:472-693 -> (raw policy fields, value [B, K]) ([B, 1] with ``selected_private``)."""

        out = self.forward_output(pub, class_ranges, class_mask, actor_seat, selected_private=selected_private)
        return out.raw, out.v

    def forward_output(self, pub: dict, class_ranges: Tensor, class_mask: Tensor | None = None,
                       actor_seat: Tensor | None = None, *, selected_private: Tensor | None = None) -> PolicyOutput:
        """preflop.py:472-693 -> PolicyOutput(raw, v, t, c): every actor class row, or the one class
        ``selected_private`` [B] names (the learner row), and the public branching heads."""

        cfg, p, dev = self.cfg, self.p, self.device
        d, K = cfg.d_model, self.n_classes
        ranges = class_ranges.to(dev, torch.float32)
        batch, players = ranges.shape[:2]
        actor = (pub["to_act"] if actor_seat is None else actor_seat).long()
        seat_mask = pub.get("seat_mask")
        seat_mask = torch.ones((batch, players), dtype=torch.bool, device=dev) if seat_mask is None else seat_mask.bool()
        cmask = torch.ones_like(ranges, dtype=torch.bool) if class_mask is None else class_mask.bool()
        cmask = cmask & seat_mask[:, :, None]
        status = pub.get("status")
        status = torch.zeros((batch, players), dtype=torch.long, device=dev) if status is None else status.long()
        seat_ids = torch.arange(players, device=dev)[None].expand(batch, -1)
        button = pub.get("button")
        relative = torch.remainder(seat_ids - button[:, None].long(), players) if button is not None else seat_ids
        class_emb = p["class_embedding.weight"][None].expand(batch, -1, -1)  # every class row, in class order
        expanded_emb = class_emb[:, None].expand(-1, players, -1, -1)
        size_feature = (self.class_sizes / 12.0)[None, None].expand(batch, players, -1)
        geometry = torch.cat((self.class_card_geometry, self.class_overlap_scalars), -1)
        expanded_geometry = geometry[None, None].expand(batch, players, -1, -1)
        log_range = torch.log(ranges.clamp_min(cfg.eps))
        row_feature = torch.cat((ranges[..., None], log_range[..., None], size_feature[..., None], expanded_emb,
                                 expanded_geometry, torch.ones_like(ranges)[..., None]), -1)
        actor_flag = (torch.arange(players, device=dev)[None] == actor[:, None]).long()
        # each seat's seat, status and actor embeddings, added to its K class rows in the map's epilogue
        seat_terms = (lookup(p["seat_embedding.weight"], relative) + lookup(p["status_embedding.weight"], status)
                      + lookup(p["actor_embedding.weight"], actor_flag))
        row = _affine_rows(self.class_row_affine, row_feature, seat_terms, K)
        row_flat = row.reshape(batch, players * K, d)
        public_token, public_mask = self._public_tokens(pub, seat_mask, relative)
        actor_relative = relative.gather(1, actor[:, None]).squeeze(1)
        anchors = p["anchor_tokens"][None] + lookup(p["anchor_seat_embedding.weight"], actor_relative)[:, None]
        x = torch.cat((row_flat, public_token, anchors), 1)
        length = x.shape[1]
        key_mask = torch.cat((cmask.reshape(batch, players * K), public_mask,
                              torch.ones((batch, cfg.k_act), dtype=torch.bool, device=dev)), 1)
        masked_range = ranges * cmask.float()
        normalized = masked_range / masked_range.sum(-1, keepdim=True).clamp_min(cfg.eps)
        key_bias = torch.cat((torch.log(normalized.clamp_min(cfg.eps)).reshape(batch, players * K),
                              torch.zeros((batch, length - players * K), device=dev)), 1).contiguous()
        side_class = torch.cat((expanded_emb, ranges[..., None], log_range[..., None], expanded_geometry), -1)
        incidence = self.class_card_geometry
        identical_scale = (1.0 / self.class_sizes)[None].expand(batch, -1)

        x = self._trunk(x, players, K, normalized, incidence, identical_scale, side_class, key_bias, key_mask)
        final = self._ln(x, self.final_ln).float()
        final_rows = final[:, : players * K].reshape(batch, players, K, d)
        final_public = final[:, players * K: -cfg.k_act]
        final_anchors = final[:, -cfg.k_act:]
        public_valid = public_mask.float()
        public_mean = (final_public * public_valid[..., None]).sum(1) / public_valid.sum(1, keepdim=True)
        actor_anchor = torch.cat((final_anchors[:, 0], final_anchors[:, 1], final_anchors[:, 2],
                                  final_anchors[:, 3:].mean(1)), -1)
        actor_summary = self._ffn(self.actor_seat_features, actor_anchor).float()
        mass = masked_range.sum(-1)
        pooled = (final_rows * masked_range[..., None]).sum(2) / mass[..., None].clamp_min(cfg.eps)
        seat_meta = torch.stack((mass, status.float() / 2.0, relative.float() / max(cfg.max_players - 1, 1)), -1)
        seat_summary = self._ffn(self.seat_features, torch.cat((pooled, seat_meta), -1)).float()
        selector = torch.arange(players, device=dev)[None] == actor[:, None]
        seat_summary = torch.where(selector[..., None], actor_summary[:, None], seat_summary)
        seat_summary = seat_summary.masked_fill(~seat_mask[..., None], 0.0)
        ordered = torch.zeros_like(seat_summary).scatter(1, relative[..., None].expand(-1, -1, d), seat_summary)
        padded = torch.cat((ordered, torch.zeros((batch, cfg.max_players - players, d), device=dev)), 1)
        global_feature = self._ffn(self.global_features,
                                   torch.cat((public_mean, actor_summary, padded.reshape(batch, -1)), -1)).float()
        actor_rows = final_rows[torch.arange(batch, device=dev), actor]
        if selected_private is not None:
            selected = selected_private.to(dev).long()[:, None, None]
            actor_rows = actor_rows.gather(1, selected.expand(-1, 1, d))
            class_emb = class_emb.gather(1, selected.expand(-1, 1, cfg.class_embedding_dim))
        raw, value = self._readout(actor_rows, class_emb, final_anchors, global_feature)
        t, cost = self._branching(global_feature, public_mean, padded)
        return PolicyOutput(raw, value, t, cost)



def parameter_shapes(cfg: PreflopConfig, rank_count: int) -> dict[str, tuple[int, ...]]:
    """Names and shapes of the parameters PreflopModel binds (SharedPokerParameters, shared.py:36-72,
    and PreflopEncoder, preflop.py:206-233), the state_dict names of the reference modules."""

    d, dc, h = cfg.d_model, cfg.class_embedding_dim, cfg.hidden
    n_cards = 4 * rank_count
    pre = dc + 4 + n_cards
    post = dc + 3 + n_cards + 4 * cfg.folder_beta_rank + 2 * d
    readout = (2 + cfg.k_act) * d + dc
    shapes: dict[str, tuple[int, ...]] = {
        "state_token": (d,), "anchor_tokens": (cfg.k_act, d), "seat_embedding.weight": (cfg.max_players, d),
        "status_embedding.weight": (3, d), "actor_embedding.weight": (2, d),
        "public_scalar_affine.weight": (d, 1), "public_scalar_affine.bias": (d,),
        "public_type_embedding.weight": (13, d), "history_numeric_affine.weight": (d, 6),
        "history_numeric_affine.bias": (d,), "history_action_embedding.weight": (4, d),
        "history_street_embedding.weight": (4, d), "history_position_embedding.weight": (cfg.max_history_tokens, d),
        "anchor_seat_embedding.weight": (cfg.max_players, d),
        "final_norm.weight": (d,), "final_norm.bias": (d,),
        "class_embedding.weight": (rank_count * rank_count, dc),
        "class_row_affine.weight": (d, dc + 4 + n_cards + 2), "class_row_affine.bias": (d,),
        "type_head.affine.weight": (3, d), "type_head.affine.bias": (3,),
        "raise_head.mixture_affine.weight": (3 * cfg.m_raise, d), "raise_head.mixture_affine.bias": (3 * cfg.m_raise,),
        "raise_head.allin_affine.weight": (1, d), "raise_head.allin_affine.bias": (1,),
        "value_head.affine.weight": (1, d), "value_head.affine.bias": (1,),
    }
    for i in range(cfg.layers):
        shapes.update({
            f"layer_norms.{i}.weight": (d,), f"layer_norms.{i}.bias": (d,),
            f"attentions.{i}.theta": (cfg.n_heads,), f"attentions.{i}.w_qkv.weight": (3 * d, d),
            f"attentions.{i}.w_qkv.bias": (3 * d,), f"attentions.{i}.w_o.weight": (d, d),
            f"attentions.{i}.w_o.bias": (d,),
            f"incidence_residuals.{i}.norm.weight": (d,), f"incidence_residuals.{i}.norm.bias": (d,),
            f"incidence_residuals.{i}.source.weight": (d, d), f"incidence_residuals.{i}.query.weight": (d, d),
            f"incidence_residuals.{i}.query.bias": (d,), f"incidence_residuals.{i}.identical.weight": (d, d),
            f"incidence_residuals.{i}.own.weight": (d, d), f"incidence_residuals.{i}.output.weight": (d, d),
            f"incidence_residuals.{i}.output.bias": (d,),
            f"layer_ffns.{i}.common.weight": (h, 4 * d), f"layer_ffns.{i}.common.bias": (h,),
            f"layer_ffns.{i}.static.pre.weight": (h, pre), f"layer_ffns.{i}.static.post.weight": (h, post),
            f"layer_ffns.{i}.output.weight": (d, h), f"layer_ffns.{i}.output.bias": (d,),
        })
    for name, (fan_in, out) in {"actor_seat_features": (4 * d, d), "seat_features": (d + 3, d),
                                "global_features": ((2 + cfg.max_players) * d, d), "type_features": (readout, d),
                                "raise_features": (readout, d), "value_head.features": (readout, d)}.items():
        shapes.update({f"{name}.w1.weight": (h, fan_in), f"{name}.w1.bias": (h,),
                       f"{name}.w2.weight": (out, h), f"{name}.w2.bias": (out,)})
    return shapes


__all__ = ["FamilyModel", "PolicyOutput", "PreflopConfig", "PreflopModel", "class_geometry", "lookup",
           "parameter_shapes"]
