"""numpy/ctypes front end of the CPU oracle (test infrastructure only).

This module is the parity checker for the CUDA library.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline/reference leg
import it.  The shipped path never does, and there is no CPU fallback.

Each wrapper names the reference function (``path:line`` in the pbg
project) that the C restatement in ``pbg_oracle.c`` follows.  Composite
steps that the reference builds from several hooks calls (the rollout
transition, ``pbg/games/poker/queued/hooks.py:1622-1700``) are composed here
from the C primitives in the reference's own order.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass, field, fields

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")

PRIVATE, ROUND, POSTERIOR, ACTION, CHANCE, COMPLETION, LEARNER, ROLE_SELECTION = range(1, 9)
PAD_CARD = 255
LIVE, FOLDED, ALL_IN = 0, 1, 2
FOLD, CHECK_CALL, RAISE_OFFSET = 0, 1, 2


def build() -> str:
    """Compile ``liboracle.so`` with the committed Makefile when missing/stale."""

    src = os.path.join(_HERE, "pbg_oracle.c")
    if (not os.path.exists(_LIB_PATH)) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        cc = "/usr/bin/gcc" if os.path.exists("/usr/bin/gcc") else "gcc"
        subprocess.run(["make", "-C", _HERE, f"CC={cc}", "liboracle.so"], check=True,
                       stdout=subprocess.DEVNULL)
    return _LIB_PATH


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(build())
        _declare(_lib)
    return _lib


class Geom(ctypes.Structure):
    _fields_ = [("players", ctypes.c_int32), ("stack_bb", ctypes.c_float),
                ("rank_count", ctypes.c_int32)]


_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32


class _State(ctypes.Structure):
    _fields_ = [(n, _P) for n in (
        "board", "combo", "button", "street", "to_act", "stacks", "committed",
        "committed_street", "status", "current_bet", "last_full_raise", "pending",
        "can_raise", "terminal")]


class _History(ctypes.Structure):
    _fields_ = [(n, _P) for n in (
        "actor", "street", "action", "amount", "pot_before", "call_amount",
        "current_bet", "min_raise_to", "max_raise_to", "mask")]


def _declare(L: ctypes.CDLL) -> None:
    G = Geom
    S = ctypes.POINTER(_State)
    Hh = ctypes.POINTER(_History)
    sig = {
        "orc_rng_keys": (None, [_I64, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P, _P]),
        "orc_child_path": (None, [_I64, _P, _P, _P]),
        "orc_uniform": (None, [_I64, _P, _P]),
        "orc_categorical": (None, [_I64, _I64, _P, _P, _P, _P, _P]),
        "orc_history_tokens": (_I32, [G]),
        "orc_combo_cards": (None, [G, _I64, _P, _P]),
        "orc_combo_id": (None, [G, _I64, _P, _P, _P]),
        "orc_combo_class": (None, [G, _P]),
        "orc_initial_roots": (None, [G, _I64, _I64, _I64, _I64, _I64, _I64, _P, S]),
        "orc_input_type": (None, [G, _I64, S, _P]),
        "orc_legality": (None, [G, _I64, S, _P]),
        "orc_step_player": (None, [G, _I64, S, _P]),
        "orc_needs_chance": (None, [G, _I64, S, _P]),
        "orc_deal_next_street": (None, [G, _I64, S, _P, _P]),
        "orc_deal_next_street_keyed": (None, [G, _I64, S, _I64, _I64, _P, _P, _I64, _P, _P, _P]),
        "orc_append_player_history": (None, [G, _I64, S, _P, Hh]),
        "orc_append_chance_history": (None, [G, _I64, S, _P, Hh]),
        "orc_sampled_leaf": (None, [G, _I64, S, _P, _P, _P, _P, _P]),
        "orc_hand_value7": (_I64, [_I32, _P]),
        "orc_evaluate_showdowns": (None, [_I32, _I64, _I32, _I32, _P, _P, _P, _P, _P, _P]),
        "orc_rb_complete": (_I32, [_I32, _I64, _I32, _I32, _I32, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
        "orc_policy_probabilities": (None, [_I64, _I32, _I32, _I64, _P, _P, _P, _P, _P, _P, _P]),
        "orc_ppo_categorical": (None, [_I64, _I32, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
        "orc_adam": (_I32, [_I64, _P, _P, _P, _P, _P, _P, _I32, _P]),
        "orc_posterior_sample": (None, [Geom, _I64, _P, _P, _P, _I64, _P, _P, _P, _P, _P, _I64, _I64, _P, _I32,
                                        _P, _P, _P, _P, _P]),
        "orc_alias_table": (None, [_I64, _P, _P, _P]),
        "orc_decision_log_mass": (_I32, [_I64, _P, _P, _P]),
        "orc_layered_targets": (None, [_P, _I32, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I32,
                                       _I32, _I32, _I32, ctypes.c_float, _I32, _I32, _P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def _ptr(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.c_void_p)


def _i64(x, n):
    return np.ascontiguousarray(np.broadcast_to(np.asarray(x, dtype=np.int64), (n,)))


# ---------------------------------------------------------------- geometry


@dataclass(frozen=True)
class Geometry:
    """hooks.py:72-192 (NLHEGeometry)."""

    players: int
    stack_bb: float
    rank_count: int

    @property
    def c(self) -> Geom:
        return Geom(self.players, float(self.stack_bb), self.rank_count)

    @property
    def deck_cards(self) -> int:
        return 4 * self.rank_count

    @property
    def first_card(self) -> int:
        return 52 - self.deck_cards

    @property
    def private_hands(self) -> int:
        return self.deck_cards * (self.deck_cards - 1) // 2

    @property
    def private_classes(self) -> int:
        return self.rank_count ** 2

    @property
    def stack_ticks(self) -> int:
        return round(self.stack_bb * 2)

    @property
    def events(self) -> int:
        return self.stack_ticks + 2

    @property
    def history_tokens(self) -> int:
        return int(lib().orc_history_tokens(self.c))


# ------------------------------------------------------------------- RNG


def rng_keys(*, seed, iteration, root, path, draw, purpose, lane=0, retry_epoch=0, active=None):
    """rollout.py:122-181 (logical_rng_keys) with numpy broadcasting."""

    arrays = np.broadcast_arrays(*(np.asarray(v, dtype=np.int64) for v in (root, path, draw, lane, retry_epoch)))
    shape = arrays[0].shape
    flat = [np.ascontiguousarray(a.reshape(-1)) for a in arrays]
    n = flat[0].size
    act = None
    if active is not None:
        act = np.ascontiguousarray(np.broadcast_to(np.asarray(active, dtype=np.uint8), shape).reshape(-1))
    out = np.empty(n, dtype=np.int64)
    lib().orc_rng_keys(int(seed), int(iteration), int(purpose), n, *map(_ptr, flat), _ptr(act), _ptr(out))
    return out.reshape(shape)


def child_path(path, ordinal):
    """rollout.py:184-202 (child_path_keys)."""

    p, o = np.broadcast_arrays(np.asarray(path, dtype=np.int64), np.asarray(ordinal, dtype=np.int64))
    shape = p.shape
    p = np.ascontiguousarray(p.reshape(-1))
    o = np.ascontiguousarray(o.reshape(-1))
    out = np.empty_like(p)
    lib().orc_child_path(p.size, _ptr(p), _ptr(o), _ptr(out))
    return out.reshape(shape)


def uniform(keys):
    """rollout.py:205-234 (logical_uniform)."""

    k = np.ascontiguousarray(np.asarray(keys, dtype=np.int64).reshape(-1))
    out = np.empty(k.size, dtype=np.float32)
    lib().orc_uniform(k.size, _ptr(k), _ptr(out))
    return out.reshape(np.shape(keys))


def categorical(p, keys, mass=None, with_margin=False):
    """rollout.py:237-267 (logical_categorical); optionally the near-tie margin."""

    p = np.ascontiguousarray(p, dtype=np.float32)
    k = np.ascontiguousarray(keys, dtype=np.int64)
    m = None if mass is None else np.ascontiguousarray(mass, dtype=np.float32)
    out = np.empty(p.shape[0], dtype=np.int64)
    margin = np.empty(p.shape[0], dtype=np.float64)
    lib().orc_categorical(p.shape[0], p.shape[1], _ptr(p), _ptr(k), _ptr(m), _ptr(out), _ptr(margin))
    return (out, margin) if with_margin else out


# ----------------------------------------------------------------- state

_STATE_DTYPES = {
    "board": (np.uint8, 5), "combo": (np.int32, "P"), "button": (np.int32, None),
    "street": (np.int32, None), "to_act": (np.int32, None), "stacks": (np.float32, "P"),
    "committed": (np.float32, "P"), "committed_street": (np.float32, "P"),
    "status": (np.int8, "P"), "current_bet": (np.float32, None),
    "last_full_raise": (np.float32, None), "pending": (np.uint8, "P"),
    "can_raise": (np.uint8, "P"), "terminal": (np.uint8, None),
}


@dataclass
class State:
    """hooks.py:250-326 (PokerState) as numpy SoA columns."""

    board: np.ndarray
    combo: np.ndarray
    button: np.ndarray
    street: np.ndarray
    to_act: np.ndarray
    stacks: np.ndarray
    committed: np.ndarray
    committed_street: np.ndarray
    status: np.ndarray
    current_bet: np.ndarray
    last_full_raise: np.ndarray
    pending: np.ndarray
    can_raise: np.ndarray
    terminal: np.ndarray
    _c: object = field(default=None, repr=False, compare=False)

    @classmethod
    def empty(cls, rows: int, players: int) -> "State":
        cols = {}
        for name, (dt, width) in _STATE_DTYPES.items():
            shape = (rows,) if width is None else (rows, players if width == "P" else width)
            cols[name] = np.zeros(shape, dtype=dt)
        return cls(**cols)

    @property
    def rows(self) -> int:
        return self.button.shape[0]

    def copy(self) -> "State":
        return State(**{n: getattr(self, n).copy() for n in _STATE_DTYPES})

    def cstruct(self):
        for n in _STATE_DTYPES:
            arr = getattr(self, n)
            if not arr.flags["C_CONTIGUOUS"]:
                setattr(self, n, np.ascontiguousarray(arr))
        self._c = _State(*(_ptr(getattr(self, n)) for n in _STATE_DTYPES))
        return ctypes.byref(self._c)

    def columns(self) -> dict[str, np.ndarray]:
        return {n: getattr(self, n) for n in _STATE_DTYPES}


@dataclass
class History:
    """hooks.py:329-339 (PokerHistory) as numpy columns [B, tokens]."""

    actor: np.ndarray
    street: np.ndarray
    action: np.ndarray
    amount: np.ndarray
    pot_before: np.ndarray
    call_amount: np.ndarray
    current_bet: np.ndarray
    min_raise_to: np.ndarray
    max_raise_to: np.ndarray
    mask: np.ndarray
    _c: object = field(default=None, repr=False, compare=False)

    NAMES = ("actor", "street", "action", "amount", "pot_before", "call_amount",
             "current_bet", "min_raise_to", "max_raise_to", "mask")

    @classmethod
    def empty(cls, rows: int, tokens: int) -> "History":
        ints = {n: np.full((rows, tokens), -1, dtype=np.int64) for n in ("actor", "street", "action")}
        floats = {n: np.zeros((rows, tokens), dtype=np.float32)
                  for n in ("amount", "pot_before", "call_amount", "current_bet", "min_raise_to", "max_raise_to")}
        return cls(**ints, **floats, mask=np.zeros((rows, tokens), dtype=np.uint8))

    def cstruct(self):
        self._c = _History(*(_ptr(getattr(self, n)) for n in self.NAMES))
        return ctypes.byref(self._c)

    def columns(self) -> dict[str, np.ndarray]:
        return {n: getattr(self, n) for n in self.NAMES}


class Machine:
    """hooks.py:351-1216 (PokerStateMachine) over the C restatement."""

    def __init__(self, geometry: Geometry) -> None:
        self.g = geometry
        self.L = lib()

    def initial_roots(self, rows, *, seed, iteration, retry_epoch, logical_base=0, lane=0, buttons=None):
        s = State.empty(rows, self.g.players)
        b = None if buttons is None else np.ascontiguousarray(buttons, dtype=np.int32)
        self.L.orc_initial_roots(self.g.c, rows, seed, iteration, retry_epoch, logical_base, lane,
                                 _ptr(b), s.cstruct())
        return s

    def input_type(self, s: State):
        out = np.empty(s.rows, dtype=np.int32)
        self.L.orc_input_type(self.g.c, s.rows, s.cstruct(), _ptr(out))
        return out

    def legality(self, s: State):
        out = np.empty((s.rows, self.g.events), dtype=np.uint8)
        self.L.orc_legality(self.g.c, s.rows, s.cstruct(), _ptr(out))
        return out.astype(bool)

    def step_player(self, s: State, action) -> State:
        n = s.copy()
        a = np.ascontiguousarray(action, dtype=np.int32)
        self.L.orc_step_player(self.g.c, n.rows, n.cstruct(), _ptr(a))
        return n

    def needs_chance(self, s: State):
        out = np.empty(s.rows, dtype=np.uint8)
        self.L.orc_needs_chance(self.g.c, s.rows, s.cstruct(), _ptr(out))
        return out.astype(bool)

    def deal_next_street(self, s: State, keys, active=None) -> State:
        n = s.copy()
        k = np.ascontiguousarray(keys, dtype=np.int64)
        a = None if active is None else np.ascontiguousarray(active, dtype=np.uint8)
        self.L.orc_deal_next_street(self.g.c, n.rows, n.cstruct(), _ptr(k), _ptr(a))
        return n

    def deal_next_street_keyed(self, s: State, *, seed, iteration, root, path, draw,
                               retry_epoch=0, lane=0, active=None) -> State:
        n = s.copy()
        B = n.rows
        r, p, e, l = (_i64(v, B) for v in (root, path, retry_epoch, lane))
        a = None if active is None else np.ascontiguousarray(active, dtype=np.uint8)
        self.L.orc_deal_next_street_keyed(self.g.c, B, n.cstruct(), seed, iteration, _ptr(r), _ptr(p),
                                          draw, _ptr(e), _ptr(l), _ptr(a))
        return n

    def empty_history(self, rows) -> History:
        return History.empty(rows, self.g.history_tokens)

    def append_player_history(self, s: State, action, h: History) -> History:
        h = History(**{n: getattr(h, n).copy() for n in History.NAMES})
        a = np.ascontiguousarray(action, dtype=np.int32)
        self.L.orc_append_player_history(self.g.c, s.rows, s.cstruct(), _ptr(a), h.cstruct())
        return h

    def append_chance_history(self, s: State, active, h: History) -> History:
        h = History(**{n: getattr(h, n).copy() for n in History.NAMES})
        a = np.ascontiguousarray(active, dtype=np.uint8)
        self.L.orc_append_chance_history(self.g.c, s.rows, s.cstruct(), _ptr(a), h.cstruct())
        return h

    def sampled_leaf(self, s: State) -> dict[str, np.ndarray]:
        B, P = s.rows, self.g.players
        out = {
            "leaf_public_state": np.empty((B, 5), np.uint8),
            "leaf_private_profile": np.empty((B, P), np.int32),
            "stratum_level": np.empty((B, P), np.int32),
            "payoff_baseline": np.empty((B, P), np.float32),
            "stratum_amount": np.empty((B, P), np.float32),
        }
        self.L.orc_sampled_leaf(self.g.c, B, s.cstruct(), *(_ptr(v) for v in out.values()))
        return out

    def combo_cards(self, ids):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.empty(ids.shape + (2,), dtype=np.int64)
        self.L.orc_combo_cards(self.g.c, ids.size, _ptr(ids), _ptr(out))
        return out

    def combo_id(self, first, second):
        a = np.ascontiguousarray(first, dtype=np.int64)
        b = np.ascontiguousarray(second, dtype=np.int64)
        out = np.empty(a.shape, dtype=np.int32)
        self.L.orc_combo_id(self.g.c, a.size, _ptr(a), _ptr(b), _ptr(out))
        return out

    def combo_class(self):
        out = np.empty(self.g.private_hands, dtype=np.int32)
        self.L.orc_combo_class(self.g.c, _ptr(out))
        return out


# ------------------------------------------------------------ showdown


def hand_value7(rank_count: int, cards) -> int:
    c = np.ascontiguousarray(cards, dtype=np.int32)
    return int(lib().orc_hand_value7(rank_count, _ptr(c)))


def evaluate_showdowns(rank_count, board_cards, combo_ids, stratum_level, payoff_baseline, stratum_amount):
    """Contract-v2 ``evaluate_showdowns`` restated (hooks.py:2277-2295 call site)."""

    board = np.ascontiguousarray(board_cards, dtype=np.uint8)
    combo = np.ascontiguousarray(combo_ids, dtype=np.int32)
    level = np.ascontiguousarray(stratum_level, dtype=np.int32)
    base = np.ascontiguousarray(payoff_baseline, dtype=np.float32)
    amt = np.ascontiguousarray(stratum_amount, dtype=np.float32)
    B, P = combo.shape
    out = np.empty((B, P), dtype=np.float32)
    lib().orc_evaluate_showdowns(rank_count, B, P, amt.shape[1], _ptr(board), _ptr(combo), _ptr(level),
                                 _ptr(base), _ptr(amt), _ptr(out))
    return out


def rb_complete(rank_count, board_cards, range_weights, stratum_level, payoff_baseline, stratum_amount, n_samples,
                seed, selected_player=None):
    """This build's estimator of the contract-v2 ``complete`` / ``complete_selected`` (hooks.py:2472-2477,
    2512; law core_math.tex:664-684), restated on the host.  Parity with the external evaluator is
    unpinned.  Returns (p_hat, v_hat, n_eff, status): [F,P,H] (or [F,H] with ``selected_player``)."""

    board = np.ascontiguousarray(board_cards, dtype=np.uint8)
    w = np.ascontiguousarray(range_weights, dtype=np.float32)
    F, P, H = w.shape
    level = np.ascontiguousarray(stratum_level, dtype=np.int32)
    base = np.ascontiguousarray(payoff_baseline, dtype=np.float32)
    amt = np.ascontiguousarray(stratum_amount, dtype=np.float32)
    sd = np.ascontiguousarray(seed, dtype=np.int64).reshape(F)
    sel = None if selected_player is None else np.ascontiguousarray(selected_player, dtype=np.int32).reshape(F)
    shape = (F, P, H) if sel is None else (F, H)
    p_hat = np.empty(shape, np.float32)
    v_hat = np.empty(shape, np.float32)
    n_eff = np.empty(F, np.float32)
    status = lib().orc_rb_complete(int(rank_count), F, P, amt.shape[1], int(n_samples), _ptr(board), _ptr(w),
                                   _ptr(level), _ptr(base), _ptr(amt), _ptr(sd), _ptr(sel), _ptr(p_hat),
                                   _ptr(v_hat), _ptr(n_eff))
    return p_hat, v_hat, n_eff, int(status)


# ---------------------------------------------------------------- policy


def policy_probabilities(raw: dict, mask):
    """policy.py:113-204 (PokerPolicyOperator.probabilities).

    ``raw`` fields have prefix [B] or [B, H]; ``mask`` is [B, E] and is
    broadcast over H as in the reference.
    """

    logits = np.asarray(raw["type_logits"], dtype=np.float32)
    prefix = logits.shape[:-1]
    B = prefix[0]
    rows = int(np.prod(prefix))
    per = rows // B
    M = raw["omega"].shape[-1]
    mask = np.ascontiguousarray(mask, dtype=np.uint8)
    E = mask.shape[1]
    T = E - 2
    c = {n: np.ascontiguousarray(np.asarray(raw[n], dtype=np.float32)) for n in ("type_logits", "omega", "mu", "s", "iota")}
    out = np.empty((rows, E), dtype=np.float32)
    lib().orc_policy_probabilities(rows, T, M, per, _ptr(c["type_logits"]), _ptr(c["omega"]), _ptr(c["mu"]),
                                   _ptr(c["s"]), _ptr(c["iota"]), _ptr(mask), _ptr(out))
    return out.reshape(prefix + (E,))


def sample_actor(raw: dict, mask, actor_hand, keys, with_margin=False):
    """policy.py:246-282 (sample_actor): compose for the actor hand only."""

    hand = np.asarray(actor_hand, dtype=np.int64)
    rows = np.arange(hand.size)
    selected = {n: np.asarray(v)[rows, hand] for n, v in raw.items()}
    p = policy_probabilities(selected, mask)
    col, margin = categorical(p, keys, with_margin=True)
    logp = np.log(np.maximum(p[rows, col], np.float32(1e-12))).astype(np.float32)
    out = (col.astype(np.int32), logp)
    return out + (margin,) if with_margin else out


# ------------------------------------------------------------------ loss


def ppo_categorical(logits, mask, action, old_logp, adv, weight, *, clip=0.2, log_cap=np.inf,
                    ent_coef=0.01, scale=1.0, inv_count=None, want_grad=True):
    """Fused categorical PPO objective and d/dlogits (double-precision truth).

    Follows learner.py:2021-2077 with the categorical fixture's log pi and
    entropy (tests/categorical_policy_fixture.py:33-57), weighting each row's
    objective by its decision-mass weight.
    """

    x = np.ascontiguousarray(logits, dtype=np.float32)
    N, A = x.shape
    if inv_count is None:
        inv_count = 1.0 / N
    m = np.ascontiguousarray(mask, dtype=np.uint8)
    a = np.ascontiguousarray(action, dtype=np.int32)
    o = np.ascontiguousarray(old_logp, dtype=np.float32)
    v = np.ascontiguousarray(adv, dtype=np.float32)
    w = np.ascontiguousarray(weight, dtype=np.float32)
    ctl = np.array([clip, log_cap, ent_coef, scale, inv_count], dtype=np.float32)
    d = np.empty((N, A), dtype=np.float32) if want_grad else None
    sums = np.zeros(8, dtype=np.float64)
    lib().orc_ppo_categorical(N, A, _ptr(x), _ptr(m), _ptr(a), _ptr(o), _ptr(v), _ptr(w), _ptr(ctl),
                              _ptr(d), _ptr(sums))
    return d, sums


def ppo_readout(logits, mask, action, old_logp, adv, weight, hidden, **loss_options):
    """The loss gradient above carried through the readout that produced the logits, x = h W^T + b
    (pbg/core/tensor_ops.py:25-38): dW = dlogits^T h and db = sum_r dlogits in float64.
    Returns (dlogits, dW [A, d], db [A], sums)."""

    d, sums = ppo_categorical(logits, mask, action, old_logp, adv, weight, **loss_options)
    d64 = d.astype(np.float64)
    h64 = np.ascontiguousarray(hidden, dtype=np.float64)
    return d, d64.T @ h64, d64.sum(0), sums


def adam(master, grad, first, second, controls, step, decoupled=True):
    """optimization.py:182-233 (adam_transition) for one lane, in place."""

    st = np.array([step], dtype=np.int64)
    norm = np.zeros(1, dtype=np.float64)
    ctl = np.ascontiguousarray(controls, dtype=np.float32)
    applied = lib().orc_adam(master.size, _ptr(master), _ptr(grad), _ptr(first), _ptr(second), _ptr(ctl),
                             _ptr(st), int(decoupled), _ptr(norm))
    return bool(applied), int(st[0]), float(norm[0])


# -------------------------------------------------------- rollout step


def rollout_transition(machine: Machine, s: State, h: History, action, *, seed, iteration,
                       root, path, retry_epoch=0, lane=0):
    """One player transition with its bounded chance closure.

    Follows hooks.py:1656-1700: history append from the pre-action state,
    step_player, then three CHANCE generations (needs_chance → chance
    history → keyed deal at draw=generation) at the row's (root, path).
    Returns the new state, history and the child path (rollout.py:184,
    hooks.py:1870).
    """

    h = machine.append_player_history(s, action, h)
    s = machine.step_player(s, action)
    for generation in range(3):
        active = machine.needs_chance(s)
        h = machine.append_chance_history(s, active, h)
        s = machine.deal_next_street_keyed(s, seed=seed, iteration=iteration, root=root, path=path,
                                           draw=generation, retry_epoch=retry_epoch, lane=lane)
    return s, h, child_path(path, 1)


# ------------------------------------------------------ model input


def direct_model_input(machine: Machine, input_type: str, s: State, log_reach=None, history: History | None = None):
    """hooks.py:531-612 (direct_model_input), with hooks.py:630-648 (_compact_preflop_reach).

    Row layout: public 8+10P | log-reach P*K (pre, class-compact) or P*H (post) | 10 history columns
    of `tokens` | folded summary zeros (post rows of P > 2 tables).
    """

    g = machine.g
    P, D, H, K, first = g.players, g.deck_cards, g.private_hands, g.private_classes, g.first_card
    B = s.rows
    scale = np.float32(g.stack_bb)
    board = s.board.astype(np.float32)
    board = np.where(s.board == PAD_CARD, np.float32(-1.0), (board - np.float32(first)) / np.float32(max(1, D - 1)))
    eye = np.eye(P, dtype=np.float32)
    status = np.eye(3, dtype=np.float32)[s.status.astype(np.int64)].reshape(B, 3 * P)
    public = np.concatenate([
        (s.street.astype(np.float32) / np.float32(3.0))[:, None], board, eye[s.to_act], eye[s.button],
        s.stacks / scale, s.committed / scale, s.committed_street / scale, status,
        s.pending.astype(np.float32), (s.current_bet / scale)[:, None], (s.last_full_raise / scale)[:, None],
        s.can_raise.astype(np.float32)], 1).astype(np.float32)
    cls = machine.combo_class()
    counts = np.bincount(cls, minlength=K).astype(np.float32)
    pre = input_type == "pre"
    if log_reach is None:
        reach = np.broadcast_to(np.log(counts)[None, None], (B, P, K)) if pre else np.zeros((B, P, H), np.float32)
    elif pre:
        exact = np.asarray(log_reach, dtype=np.float32)
        finite = np.isfinite(exact)
        gauge = np.where(finite, exact, -np.inf).max(-1, keepdims=True)
        safe = np.where(np.isfinite(gauge), gauge, np.float32(0.0))
        weight = np.where(finite, np.exp(exact - safe), np.float32(0.0)).astype(np.float32)
        compact = np.zeros((B, P, K), np.float32)
        for k in range(K):
            compact[..., k] = weight[..., cls == k].sum(-1)
        tiny = np.finfo(np.float32).tiny
        reach = np.where(compact > 0, np.log(np.maximum(compact, tiny)) + safe, -np.inf).astype(np.float32)
    else:
        reach = np.asarray(log_reach, dtype=np.float32)
    if history is None:
        history = History.empty(B, g.history_tokens)
    hist = [getattr(history, n).astype(np.float32) for n in History.NAMES]
    parts = [public, reach.reshape(B, -1), *hist]
    if not pre and P > 2:
        width = H + D + D * D + P + P * D + 2
        parts.append(np.zeros((B, width), np.float32))
    return np.concatenate(parts, 1).astype(np.float32)


TARGET_GROUPS = ("work0", "work1", "trace", "cost", "delta", "head_v", "head_t", "head_c",
                 "sigma_v", "sigma_t", "sigma_c", "action_p", "action_a")


def layered_targets(layer_ptr, nodes, children, arenas: dict, conversion, work_cap, head_cap, width, *,
                    n_replica, input_count, output_count, action_partitions, p_train, lam, sampled, branched):
    """pbg/core/csrc/layered_targets.cu:117-411 on host arrays (updated in place).

    ``nodes``: the 12 int32 node columns, ``children``: source_row,
    source_type, path (int32) and multiplier (float32); ``arenas`` maps each
    name of TARGET_GROUPS to a list of float32 arrays (None = absent).
    Returns failure_min (int32 [n_replica]).
    """

    keep = []

    def col(a, dt):
        a = np.ascontiguousarray(a, dtype=dt)
        keep.append(a)
        return a

    lp = col(layer_ptr, np.int32)
    node_cols = [col(a, np.int32) for a in nodes]
    node_tab = col(np.array([a.ctypes.data for a in node_cols], dtype=np.uint64), np.uint64)
    src_row, src_type, path = (col(a, np.int32) for a in children[:3])
    mult = col(children[3], np.float32)
    tables = []
    for name in TARGET_GROUPS:
        group = arenas.get(name) or []
        addresses = []
        for a in group:
            if a is None or a.size == 0:
                addresses.append(0)
            else:
                assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"], name
                addresses.append(a.ctypes.data)
        tables.append(col(np.array(addresses or [0], dtype=np.int64), np.int64))
    table_tab = col(np.array([t.ctypes.data for t in tables], dtype=np.uint64), np.uint64)
    wc, hc, wd = col(work_cap, np.int32), col(head_cap if len(head_cap) else [0], np.int32), col(width, np.int32)
    conv = col(conversion, np.int32)
    failure = np.zeros(n_replica, dtype=np.int32)
    lib().orc_layered_targets(_ptr(lp), len(lp) - 1, _ptr(node_tab), _ptr(src_row), _ptr(src_type), _ptr(path),
                              _ptr(mult), _ptr(table_tab), _ptr(wc), _ptr(hc), _ptr(wd), _ptr(conv), n_replica,
                              input_count, output_count, action_partitions, p_train, int(max(width)),
                              float(lam), int(sampled), int(branched), _ptr(failure))
    return failure


def posterior_sample(geometry_tuple, weights, board, inherited, source, ordinal, active, root, path, seed,
                     iteration, epoch, max_attempts):
    """rb_sampling.py:86-223 on host arrays.  Returns (profile [G,P] int32, attempt_count [G] int32,
    exhausted [G] bool, minimum failing path, per-row margin [G])."""

    players, stack, ranks = geometry_tuple
    w = np.ascontiguousarray(weights, dtype=np.float32)
    B = w.shape[0]
    G = len(source)
    bd = np.ascontiguousarray(board, dtype=np.uint8)
    inh = np.ascontiguousarray(inherited, dtype=np.int32)
    cols = [np.ascontiguousarray(x, dtype=np.int64) for x in (source, ordinal, root, path)]
    act = np.ascontiguousarray(active, dtype=np.uint8)
    ep = np.ascontiguousarray(np.broadcast_to(np.asarray(epoch, dtype=np.int64), (G,)))
    out = np.zeros((G, int(players)), dtype=np.int32)
    count = np.zeros(G, dtype=np.int32)
    exh = np.zeros(G, dtype=np.uint8)
    worst = np.zeros(1, dtype=np.int64)
    margin = np.zeros(G, dtype=np.float64)
    lib().orc_posterior_sample(Geom(int(players), float(stack), int(ranks)), B, _ptr(w), _ptr(bd), _ptr(inh), G,
                               _ptr(cols[0]), _ptr(cols[1]), _ptr(act), _ptr(cols[2]), _ptr(cols[3]), int(seed),
                               int(iteration), _ptr(ep), int(max_attempts), _ptr(out), _ptr(count), _ptr(exh),
                               _ptr(worst), _ptr(margin))
    return out, count, exh.astype(bool), int(worst[0]), margin


def alias_table(scaled):
    """alias_table.cu:11-44 on a float64 vector (not modified); returns (probability, alias, final scaled)."""

    work = np.array(scaled, dtype=np.float64, copy=True)
    n = work.size
    prob = np.empty(n, np.float64)
    alias = np.empty(n, np.int32)
    lib().orc_alias_table(n, _ptr(work), _ptr(prob), _ptr(alias))
    return prob, alias, work


def decision_log_mass(parent, degree):
    """branching_metadata.cu:9-31; returns (log_mass f32 [n] (NaN after a failure), failure code)."""

    p = np.ascontiguousarray(parent, dtype=np.int32)
    d = np.ascontiguousarray(degree, dtype=np.int32)
    out = np.full(p.size, np.nan, np.float32)
    code = lib().orc_decision_log_mass(p.size, _ptr(p), _ptr(d), _ptr(out))
    return out, int(code)
