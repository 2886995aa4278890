"""GPU parity: libpbgb200 (through its C ABI) against the oracle and golden vectors.

Bars: bit-exact for keys, cards, legal masks, chip columns, history and
leaf payloads; sampled actions equal except at documented near-ties (the
threshold within 1e-5 of the row mass of a CDF edge, where a different fp32
summation order legitimately flips the bin -- counted and bounded here);
policy probabilities within the reference's own 1e-6 / 1e-5; fp32 loss
gradients within rtol 1e-5 and bf16 within 2e-2.
"""

import math

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def cuda(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.to(DEV)


def host(t):
    return t.detach().cpu().numpy()


# ------------------------------------------------------------------ RNG


def test_rng_matches_reference_golden(gold):
    from pbg_b200 import rng

    g = gold("rng")
    for i, (seed, iteration, purpose) in enumerate(g["rng_scalars"]):
        keys = rng.logical_rng_keys(seed=int(seed), iteration=int(iteration), purpose=int(purpose),
                                    root=cuda(g["rng_root"][i]), path=cuda(g["rng_path"][i]),
                                    draw=cuda(g["rng_draw"][i]), lane=cuda(g["rng_lane"][i]),
                                    retry_epoch=cuda(g["rng_epoch"][i]),
                                    active=cuda(g["rng_active"][i]).bool())
        np.testing.assert_array_equal(host(keys), g["rng_keys"][i])
        child = rng.child_path_keys(cuda(g["rng_path"][i]), cuda(g["rng_child_ordinal"][i]))
        np.testing.assert_array_equal(host(child), g["rng_child"][i])
    np.testing.assert_array_equal(host(rng.logical_uniform(cuda(g["rng_uniform_keys"]))), g["rng_uniform"])
    sel = host(rng.logical_categorical(cuda(g["cat_prob"]), cuda(g["cat_keys"])))
    ref, margin = O.categorical(g["cat_prob"], g["cat_keys"], with_margin=True)
    np.testing.assert_array_equal(sel, ref)
    endpoint = torch.tensor([((1 << 24) - 1) << 39], dtype=torch.int64, device=DEV)
    assert float(rng.logical_uniform(endpoint)[0]) < 1.0
    assert int(rng.logical_categorical(torch.tensor([[1.0, 0.0]], device=DEV), endpoint)[0]) == 0


def test_rng_is_invariant_to_order_and_subdivision():
    """test_rollout_transactions.py:548-620 properties."""

    from pbg_b200 import rng

    root = torch.tensor([3, 5, 8, 13, 21, 34], dtype=torch.int64, device=DEV)
    path = torch.arange(6, dtype=torch.int64, device=DEV)
    lane = torch.tensor([2, 0, 1, 2, 0, 1], dtype=torch.int64, device=DEV)
    keys = rng.logical_rng_keys(seed=91, iteration=7, root=root, path=path, draw=4, purpose=4, lane=lane)
    order = torch.tensor([4, 1, 5, 0, 3, 2], device=DEV)
    perm = rng.logical_rng_keys(seed=91, iteration=7, root=root[order], path=path[order], draw=4, purpose=4,
                                lane=lane[order])
    rebuilt = torch.empty_like(keys)
    rebuilt[order] = perm
    assert torch.equal(keys, rebuilt)
    split = torch.cat([rng.logical_rng_keys(seed=91, iteration=7, root=root[s], path=path[s], draw=4, purpose=4,
                                            lane=lane[s]) for s in (slice(0, 2), slice(2, 6))])
    assert torch.equal(keys, split)
    assert not torch.equal(keys, rng.logical_rng_keys(seed=91, iteration=7, root=root, path=path, draw=4,
                                                      purpose=5, lane=lane))


# ------------------------------------------------------- state machine

STATE_MAP = {"board_cards": "board", "combo_ids": "combo", "button": "button", "street": "street",
             "to_act": "to_act", "stacks": "stacks", "committed": "committed",
             "committed_street": "committed_street", "status": "status", "current_bet": "current_bet",
             "last_full_raise": "last_full_raise", "pending": "pending", "can_raise": "can_raise",
             "terminal": "terminal"}


def _dev_state(cols, rows=None):
    from pbg_b200.poker import PokerState

    dtypes = {"board_cards": torch.uint8, "combo_ids": torch.int32, "button": torch.int32, "street": torch.int32,
              "to_act": torch.int32, "stacks": torch.float32, "committed": torch.float32,
              "committed_street": torch.float32, "status": torch.int8, "current_bet": torch.float32,
              "last_full_raise": torch.float32, "pending": torch.bool, "can_raise": torch.bool,
              "terminal": torch.bool}
    sel = (lambda v: v) if rows is None else (lambda v: v[rows])
    return PokerState(*(cuda(sel(cols[n])).to(dtypes[n]) for n in STATE_MAP))


@pytest.mark.parametrize("gi", range(7))
def test_state_machine_replays_reference_trajectories(gold, gi):
    from pbg_b200.poker import HISTORY_FIELDS, NLHEGeometry, PokerHistory, PokerStateMachine
    from pbg_b200.rng import child_path_keys

    g = gold("poker")
    tag = f"g{gi}"
    players, stack, ranks = g[f"{tag}_geometry"]
    geometry = NLHEGeometry(int(players), float(stack), int(ranks))
    m = PokerStateMachine(geometry)
    seed, iteration, retry, base, lane, B = (int(x) for x in g[f"{tag}_root_args"])
    s = m.initial_roots(B, seed=seed, iteration=iteration, retry_epoch=retry, logical_base=base, lane=lane,
                        device=DEV)
    for ref, mine in STATE_MAP.items():
        np.testing.assert_array_equal(host(getattr(s, ref)).astype(np.float64),
                                      g[f"{tag}_root_{ref}"].astype(np.float64), err_msg=ref)
    np.testing.assert_array_equal(host(m._combo_class(DEV)), g[f"{tag}_combo_class"])
    cols = {n: g[f"{tag}_root_{n}"].copy() for n in STATE_MAP}
    h = m.empty_history(B, DEV)
    hist = {n: host(getattr(h, n)).copy() for n in HISTORY_FIELDS}
    path = np.zeros(B, dtype=np.int64)
    root = np.arange(base, base + B, dtype=np.int64)
    E = int(g[f"{tag}_mask_events"][0])
    masks = np.unpackbits(g[f"{tag}_masks"], axis=-1)[..., :E].astype(bool)
    for t, action in enumerate(g[f"{tag}_actions"]):
        rows = np.nonzero(action >= 0)[0]
        sub = _dev_state(cols, rows)
        np.testing.assert_array_equal(host(m.legality(sub).mask), masks[t][rows])
        sub_h = PokerHistory(*(cuda(hist[n][rows]) for n in HISTORY_FIELDS))
        act = cuda(action[rows])
        sub_h = m.append_player_history(sub, act, sub_h)
        nxt = m.step_player(sub, act)
        r, p = cuda(root[rows]), cuda(path[rows])
        for generation in range(3):
            active = m.needs_chance(nxt)
            sub_h = m.append_chance_history(nxt, active, sub_h)
            nxt = m.deal_next_street_keyed(nxt, seed=seed, iteration=iteration, root=r, path=p, draw=generation,
                                           retry_epoch=retry, lane=lane)
        for n in STATE_MAP:
            cols[n][rows] = host(getattr(nxt, n))
            np.testing.assert_array_equal(cols[n].astype(np.float64), g[f"{tag}_post_{n}"][t].astype(np.float64),
                                          err_msg=f"step {t} {n}")
        for n in HISTORY_FIELDS:
            hist[n][rows] = host(getattr(sub_h, n))
        path[rows] = host(child_path_keys(p, 1))
    for n in HISTORY_FIELDS:
        np.testing.assert_array_equal(hist[n].astype(np.float64), g[f"{tag}_history_{n}"].astype(np.float64),
                                      err_msg=n)
    leaf = m.sampled_leaf(_dev_state(cols))
    for k, v in leaf.items():
        np.testing.assert_array_equal(host(v), g[f"{tag}_leaf_{k}"], err_msg=k)


def test_explicit_key_deal_and_combo_cards():
    from pbg_b200.poker import NLHEGeometry, PokerStateMachine

    geometry = NLHEGeometry(2, 8.0, 13)
    m = PokerStateMachine(geometry)
    om = O.Machine(O.Geometry(2, 8.0, 13))
    s = m.initial_roots(64, seed=209559, iteration=1, retry_epoch=0, device=DEV)
    os_ = om.initial_roots(64, seed=209559, iteration=1, retry_epoch=0)
    gen = 0
    while not bool(s.terminal.all()):
        if bool(m.needs_chance(s).all()):
            keys = torch.arange(52, dtype=torch.int64, device=DEV)[None].expand(64, -1) + gen * 52 + 1
            s = m.deal_next_street(s, keys.contiguous())
            os_ = om.deal_next_street(os_, host(keys))
            gen += 1
        else:
            a = torch.full((64,), 1, dtype=torch.int32, device=DEV)
            s = m.step_player(s, a)
            os_ = om.step_player(os_, host(a))
    assert gen == 3
    for ref, mine in STATE_MAP.items():
        np.testing.assert_array_equal(host(getattr(s, ref)).astype(np.float64),
                                      getattr(os_, mine).astype(np.float64), err_msg=ref)
    ids = torch.arange(geometry.private_hands, dtype=torch.int32, device=DEV)
    np.testing.assert_array_equal(host(m.combo_cards(ids)), om.combo_cards(host(ids)))


# ------------------------------------------------------------- policy


@pytest.mark.parametrize("name", ["small", "hu8", "hu100", "six50"])
def test_policy_matches_reference_golden(gold, name):
    from pbg_b200.poker import PokerLegality
    from pbg_b200.policy import PokerPolicyOperator

    g = gold("policy")
    raw = {k: cuda(g[f"pol_{name}_{k}"]) for k in ("type_logits", "omega", "mu", "s", "iota")}
    mask = cuda(g[f"pol_{name}_mask"]).bool()
    B, E = mask.shape
    legality = PokerLegality(torch.arange(E, dtype=torch.int32, device=DEV)[None].expand(B, -1).contiguous(), mask)
    op = PokerPolicyOperator()
    prob = host(op.probabilities(raw, legality))
    np.testing.assert_allclose(prob, g[f"pol_{name}_prob"], atol=1e-6, rtol=1e-5)
    sample = op.sample_actor(raw, legality, cuda(g[f"pol_{name}_hand"]), cuda(g[f"pol_{name}_keys"]))
    action = host(sample.action)
    _, _, margin = O.sample_actor({k: g[f"pol_{name}_{k}"] for k in ("type_logits", "omega", "mu", "s", "iota")},
                                  g[f"pol_{name}_mask"], g[f"pol_{name}_hand"], g[f"pol_{name}_keys"],
                                  with_margin=True)
    same = action == g[f"pol_{name}_action"]
    assert np.all(margin[~same] < 1e-5)
    np.testing.assert_allclose(host(sample.selected_log_policy)[same], g[f"pol_{name}_selected"][same],
                               atol=1e-5, rtol=1e-5)
    sel_all = host(op.selected_log_pi(raw, legality, cuda(g[f"pol_{name}_action"])))
    np.testing.assert_allclose(sel_all, g[f"pol_{name}_selected_all"], atol=1e-5, rtol=1e-5)
    entropy, kl = op.policy_reductions(raw, legality, raw)
    np.testing.assert_allclose(host(entropy), g[f"pol_{name}_entropy"], atol=2e-6, rtol=2e-5)
    np.testing.assert_allclose(host(kl), 0.0, atol=2e-7)


# ----------------------------------------------------------- showdown


@pytest.mark.parametrize("ranks,players", [(13, 2), (13, 6), (8, 3), (5, 2), (4, 2), (9, 4)])
def test_showdown_matches_oracle(ranks, players):
    import poker_gpu_evaluator as poker

    rng = np.random.default_rng(ranks * 10 + players)
    B = 3000
    D = 4 * ranks
    first = 52 - D
    geom = O.Geometry(players, 8.0, ranks)
    m = O.Machine(geom)
    deal = np.argsort(rng.random((B, D)), axis=1)[:, : 5 + 2 * players] + first
    board = deal[:, :5].astype(np.uint8)
    hole = deal[:, 5:].reshape(B, players, 2)
    combo = m.combo_id(hole[..., 0], hole[..., 1])
    level = np.where(rng.random((B, players)) < 0.2, -1, 0).astype(np.int32)
    level[:, 0] = 0
    base = -rng.integers(1, 16, (B, players)).astype(np.float32)
    amount = np.zeros((B, players), np.float32)
    amount[:, 0] = -base.sum(1)
    ref = O.evaluate_showdowns(ranks, board, combo, level, base, amount)
    ev = poker.bind(ranks)
    out = ev.evaluate_showdowns(board_cards=cuda(board), combo_ids=cuda(combo), stratum_level=cuda(level),
                                payoff_baseline=cuda(base), stratum_amount=cuda(amount))
    np.testing.assert_array_equal(host(out), ref)
    np.testing.assert_allclose(host(out).sum(1), 0.0, atol=1e-3)
    # hand values directly: every 7-card hand against the brute-force oracle
    from pbg_b200._native import call, ptr, stream
    cards = np.concatenate([board.astype(np.int32), hole[:, 0, :].astype(np.int32)], 1)
    got = torch.empty(B, dtype=torch.int64, device=DEV)
    call("pbg_hand_values", ranks, B, ptr(cuda(cards)), ptr(got), stream())
    want = np.array([O.hand_value7(ranks, c) for c in cards])
    np.testing.assert_array_equal(host(got), want)


# ------------------------------------------------------ fused rollout


@pytest.mark.parametrize("players,ranks,stack", [(2, 13, 100.0), (6, 13, 20.0), (4, 9, 20.5)])
def test_input_type_matches_oracle_along_rollouts(players, ranks, stack):
    """hooks.py:456-462 (input_type: pre 0, post with A contenders A - 1) on every state of seeded
    rollouts, against the oracle's restatement."""

    from pbg_b200.poker import NLHEGeometry
    from pbg_b200.rollout import RolloutStep

    geometry = NLHEGeometry(players, stack, ranks)
    om = O.Machine(O.Geometry(players, stack, ranks))
    B = 2000
    stepper = RolloutStep(geometry, seed=9, iteration=1)
    arena = stepper.roots(B, device=DEV)
    gen = torch.Generator().manual_seed(players + ranks)
    seen = set()
    for _ in range(400):
        got = host(stepper.machine.input_type(arena.state))
        cols = {STATE_MAP[k]: host(getattr(arena.state, k)) for k in STATE_MAP}
        state = O.State(**{k: v.astype(getattr(O.State.empty(1, players), k).dtype) for k, v in cols.items()})
        np.testing.assert_array_equal(got, om.input_type(state))
        seen.update(np.unique(got[~cols["terminal"].astype(bool)]).tolist())
        if bool(arena.state.terminal.all()):
            break
        stepper.step(arena, {k: v.to(DEV) for k, v in _random_raw(gen, (B, 1), 2).items()})
    assert 0 in seen and 1 in seen
    if players > 2:
        assert max(seen) >= 2  # multiway postflop families occur


@pytest.mark.parametrize("players,ranks,stack", [(2, 13, 100.0), (6, 13, 50.0), (3, 4, 8.0)])
def test_rollout_work_list_equals_dense_step(players, ranks, stack):
    """pbg_rollout_step_listed (live hands listed, dense warps) and pbg_rollout_step (one thread per
    row) leave identical arenas after every step of a full rollout."""

    from pbg_b200.poker import NLHEGeometry
    from pbg_b200.rollout import RolloutStep

    geometry = NLHEGeometry(players, stack, ranks)
    B = 3000
    stepper = RolloutStep(geometry, seed=5, iteration=2, work_list=True)
    listed = stepper.roots(B, device=DEV)
    dense = stepper.roots(B, device=DEV)
    dense.worklist = None
    gen = torch.Generator().manual_seed(players)
    for _ in range(400):
        if bool(listed.state.terminal.all()):
            break
        raw = {k: v.to(DEV) for k, v in _random_raw(gen, (B, 1), 2).items()}
        stepper.step(listed, raw)
        stepper.step(dense, raw)
        for name in ("action", "selected_log", "decision", "new_leaf", "root_path", "history_length"):
            assert torch.equal(getattr(listed, name), getattr(dense, name)), name
        for name in STATE_MAP:
            assert torch.equal(getattr(listed.state, name), getattr(dense.state, name)), name
        ended = listed.state.terminal.bool()  # leaf columns are written for the hands that ended
        for k, v in listed.leaf.items():
            assert torch.equal(v[ended], dense.leaf[k][ended]), k
        for k, v in vars(listed.history).items():
            if isinstance(v, torch.Tensor):
                assert torch.equal(v, getattr(dense.history, k)), k
    assert bool(dense.state.terminal.all())


def _random_raw(gen, rows_shape, M):
    t = lambda *s: torch.randn(*s, generator=gen)
    return {
        "type_logits": t(*rows_shape, 3) * 1.5,
        "omega": torch.softmax(t(*rows_shape, M), -1),
        "mu": torch.sigmoid(t(*rows_shape, M)),
        "s": torch.nn.functional.softplus(t(*rows_shape, M)) + 0.02,
        "iota": torch.sigmoid(t(*rows_shape)),
    }


@pytest.mark.parametrize("players,stack,ranks,full_rows", [(2, 8.0, 4, False), (3, 8.0, 4, True),
                                                           (2, 100.0, 13, False), (6, 20.0, 13, True),
                                                           (6, 100.0, 13, False)])
def test_fused_rollout_step_matches_oracle(players, stack, ranks, full_rows):
    from pbg_b200.poker import HISTORY_FIELDS, NLHEGeometry
    from pbg_b200.rollout import RolloutStep

    geometry = NLHEGeometry(players, stack, ranks)
    B = 96 if full_rows and ranks == 13 else (192 if players == 6 else 384)
    seed, iteration, M = 4242 + players, 5, 2
    stepper = RolloutStep(geometry, seed=seed, iteration=iteration)
    arena = stepper.roots(B, device=DEV, retry_epoch=1, logical_base=1000, lane=1)
    om = O.Machine(O.Geometry(players, stack, ranks))
    os_ = om.initial_roots(B, seed=seed, iteration=iteration, retry_epoch=1, logical_base=1000, lane=1)
    oh = om.empty_history(B)
    path = np.zeros(B, np.int64)
    root = np.arange(1000, 1000 + B, dtype=np.int64)
    H = geometry.private_hands
    cls = om.combo_class()
    log_reach = torch.zeros((B, players, H), device=DEV)
    oracle_reach = np.zeros((B, players, H), np.float32)
    gen = torch.Generator().manual_seed(players * 100 + ranks)
    near_ties = 0
    decisions = 0
    for step in range(400):
        active = ~os_.terminal.astype(bool)
        if not active.any():
            break
        rows_shape = (B, H) if full_rows else (B, 1)
        raw = _random_raw(gen, rows_shape, M)
        stepper.step(arena, {k: v.to(DEV) for k, v in raw.items()})
        if full_rows:
            stepper.reach_update(arena, {k: v.to(DEV) for k, v in raw.items()}, log_reach)
        g_action = host(arena.action)
        rows = np.nonzero(active)[0]
        sub = O.State(**{n: np.ascontiguousarray(getattr(os_, n)[rows]) for n in STATE_MAP.values()})
        mask = om.legality(sub)
        actor = sub.to_act
        combo = sub.combo[np.arange(rows.size), actor]
        if full_rows:
            hand = np.where(sub.street == 0, cls[combo], combo)
        else:
            hand = np.zeros(rows.size, np.int64)
        keys = O.rng_keys(seed=seed, iteration=iteration, purpose=O.ACTION, root=root[rows], path=path[rows],
                          draw=0, lane=1, retry_epoch=1)
        raw_np = {k: v.numpy()[rows] for k, v in raw.items()}
        o_action, o_logp, margin = O.sample_actor(raw_np, mask, hand, keys, with_margin=True)
        mismatch = o_action != g_action[rows]
        assert np.all(margin[mismatch] < 1e-5), f"step {step}: non-tie action mismatch"
        near_ties += int(mismatch.sum())
        decisions += rows.size
        action = g_action[rows].astype(np.int32)  # follow the device on near-ties
        assert np.all(g_action[~active] == -1)
        same = ~mismatch
        np.testing.assert_allclose(host(arena.selected_log)[rows][same], o_logp[same], rtol=1e-5, atol=1e-5)
        if full_rows:
            # hooks.py:1641-1703: the actor's reach row gains log pi(action) of every hand
            probs = O.policy_probabilities(raw_np, mask)
            sel = np.log(np.maximum(probs[np.arange(rows.size)[:, None], np.arange(H)[None], action[:, None]],
                                    np.float32(1e-12)))
            pre = sub.street == 0
            sel_hand = np.where(pre[:, None], sel[:, cls], sel)
            oracle_reach[rows, actor] += sel_hand
        sub_h = O.History(**{n: np.ascontiguousarray(getattr(oh, n)[rows]) for n in O.History.NAMES})
        nxt, sub_h, child = O.rollout_transition(om, sub, sub_h, action, seed=seed, iteration=iteration,
                                                 root=root[rows], path=path[rows], retry_epoch=1, lane=1)
        for n in STATE_MAP.values():
            getattr(os_, n)[rows] = getattr(nxt, n)
        for n in O.History.NAMES:
            getattr(oh, n)[rows] = getattr(sub_h, n)
        path[rows] = child
        for ref, mine in STATE_MAP.items():
            np.testing.assert_array_equal(host(getattr(arena.state, ref)).astype(np.float64),
                                          getattr(os_, mine).astype(np.float64), err_msg=f"step {step} {ref}")
        np.testing.assert_array_equal(host(arena.root_path[:, 1]), path)
        if full_rows:
            board = os_.board
            cards = om.combo_cards(np.arange(H))
            conflict = ((board[:, None, :, None] != 255) & (board[:, None, :, None] == cards[None, :, None, :])).any((2, 3))
            oracle_reach = np.where(conflict[:, None, :], -np.inf, oracle_reach).astype(np.float32)
            got = host(log_reach)
            np.testing.assert_array_equal(np.isinf(got), np.isinf(oracle_reach))
            finite = np.isfinite(oracle_reach)
            np.testing.assert_allclose(got[finite], oracle_reach[finite], rtol=1e-5, atol=1e-4)
        new = host(arena.new_leaf).astype(bool)
        ended = new & active
        assert np.array_equal(new[active], os_.terminal[active].astype(bool))
        if ended.any():
            oleaf = om.sampled_leaf(O.State(**{n: np.ascontiguousarray(getattr(os_, n)[ended]) for n in STATE_MAP.values()}))
            for k, v in arena.leaf.items():
                np.testing.assert_array_equal(host(v)[ended], oleaf[k], err_msg=k)
    assert os_.terminal.all()
    for n in HISTORY_FIELDS:
        np.testing.assert_array_equal(host(getattr(arena.history, n)).astype(np.float64),
                                      getattr(oh, n).astype(np.float64), err_msg=n)
    # near-ties are rare; report the rate through the assertion message
    assert near_ties <= max(2, decisions // 1000), f"{near_ties} near-tie flips in {decisions} decisions"


def test_rollout_is_independent_of_batching():
    """Hands addressed by (root, path) evolve identically alone or in a batch."""

    from pbg_b200.poker import NLHEGeometry
    from pbg_b200.rollout import RolloutStep

    geometry = NLHEGeometry(2, 8.0, 4)
    stepper = RolloutStep(geometry, seed=7, iteration=2)
    full = stepper.roots(64, device=DEV, logical_base=0)
    part = stepper.roots(16, device=DEV, logical_base=32)
    gen = torch.Generator().manual_seed(3)
    for _ in range(40):
        raw = _random_raw(gen, (64, 1), 2)
        stepper.step(full, {k: v.to(DEV) for k, v in raw.items()})
        stepper.step(part, {k: v[32:48].to(DEV) for k, v in raw.items()})
    for ref in STATE_MAP:
        assert torch.equal(getattr(full.state, ref)[32:48], getattr(part.state, ref)), ref


# --------------------------------------------------------------- loss


def _loss_inputs(N, A, seed, cap_rows=True):
    rng = np.random.default_rng(seed)
    logits = rng.standard_normal((N, A)).astype(np.float32)
    mask = rng.random((N, A)) < 0.7
    mask[~mask.any(1), 0] = True
    if N > 4:
        mask[1] = False
        mask[1, A - 1] = True  # single legal action
        mask[2] = True
    action = np.array([rng.choice(np.nonzero(m)[0]) for m in mask], dtype=np.int32)
    pert = logits + rng.standard_normal((N, A)).astype(np.float32) * np.float32(0.1)
    if cap_rows:
        pert[: N // 4] += rng.standard_normal((N // 4, A)).astype(np.float32) * np.float32(1.5)
    masked = np.where(mask, pert, -np.inf)
    mx = masked.max(1, keepdims=True)
    lse = np.log(np.exp(masked - mx).sum(1)) + mx[:, 0]
    old = (masked[np.arange(N), action] - lse).astype(np.float32)
    adv = rng.standard_normal(N).astype(np.float32)
    weight = rng.uniform(0.0, 1.0, N).astype(np.float32)
    return logits, mask, action, old, adv, weight


def _boundary_rows(logits, mask, action, old, clip=0.2, log_cap=math.inf, tol=1e-5):
    """Rows whose importance ratio is within `tol` of 1 +- clip or whose log ratio is within `tol` of the cap.

    The clipped objective's gradient jumps there, so an fp32 evaluation and the double-precision oracle can
    land on opposite sides of the edge; those rows are the only ones allowed to differ beyond tolerance.
    """

    x = np.where(mask, logits.astype(np.float64), -np.inf)
    mx = x.max(1, keepdims=True)
    lse = np.log(np.exp(x - mx).sum(1)) + mx[:, 0]
    lr = x[np.arange(len(x)), action] - lse - old.astype(np.float64)
    ratio = np.exp(lr)
    near = (np.abs(ratio - (1 - clip)) < tol) | (np.abs(ratio - (1 + clip)) < tol)
    if math.isfinite(log_cap):
        near |= np.abs(lr - log_cap) < tol
    return near


def _assert_close_except_boundary(got, ref, rows_near, rtol, atol):
    bad = ~np.isclose(got, ref, rtol=rtol, atol=atol)
    bad_rows = bad.any(1) if bad.ndim == 2 else bad
    assert np.all(rows_near[bad_rows]), f"{int((bad_rows & ~rows_near).sum())} rows differ away from a clip edge"
    assert bad_rows.sum() <= max(2, len(bad_rows) // 100000)


@pytest.mark.parametrize("A,cap", [(8, None), (8, 1.5), (3, None), (17, 2.0), (1, None)])
def test_fp32_loss_backward_matches_oracle(A, cap):
    from pbg_b200.loss import LossConfig, fused_ppo_backward

    N = 5000
    logits, mask, action, old, adv, weight = _loss_inputs(N, A, 11 + A)
    cfg = LossConfig(0.2, cap, 0.01)
    d, stats = fused_ppo_backward(cuda(logits), cuda(mask), cuda(action), cuda(old), cuda(adv), cuda(weight), cfg)
    ref_d, ref_s = O.ppo_categorical(logits, mask, action, old, adv, weight,
                                     log_cap=math.inf if cap is None else math.log(cap))
    # absolute floor: the size of one row's gradient terms (coef * |adv| * ratio)
    scale = max(np.abs(ref_d).max(), np.abs(adv).max() / N)
    near = _boundary_rows(logits, mask, action, old, 0.2, math.inf if cap is None else math.log(cap))
    _assert_close_except_boundary(host(d), ref_d, near, rtol=1e-5, atol=1e-5 * scale)
    # sums over N rows: absolute floor of 1e-9 per row
    np.testing.assert_allclose(host(stats)[[0, 1, 2, 3, 6, 7]], ref_s[[0, 1, 2, 3, 6, 7]], rtol=1e-5, atol=1e-9 * N)
    assert abs(host(stats)[4] - ref_s[4]) <= 2 and abs(host(stats)[5] - ref_s[5]) <= 2


def test_loss_matches_reference_autograd_golden(gold):
    from pbg_b200.loss import LossConfig, fused_ppo_backward

    g = gold("loss")
    N = g["loss_logits"].shape[0]
    for ci in (0, 1):
        cap = float(g[f"loss{ci}_cap"][0])
        cfg = LossConfig(0.2, None if math.isinf(cap) else math.exp(cap), 0.01)
        d, stats = fused_ppo_backward(cuda(g["loss_logits"]), cuda(g["loss_mask"]), cuda(g["loss_action"]),
                                      cuda(g["loss_old"]), cuda(g["loss_adv"]), cuda(g["loss_weight"]), cfg)
        np.testing.assert_allclose(host(d) * N, g[f"loss{ci}_grad"], rtol=1e-5, atol=1e-7)
        w = g["loss_weight"].astype(np.float64)
        np.testing.assert_allclose(host(stats)[0], (w * g[f"loss{ci}_row_total"]).sum() / N, rtol=1e-5)


def test_bf16_vector_path_matches_torch_fp32_autograd():
    """The A=8 bf16 kernel against a plain PyTorch fp32 autograd restatement."""

    from pbg_b200.loss import LossConfig, fused_ppo_backward

    N, A = 1 << 16, 8
    logits, mask, action, old, adv, weight = _loss_inputs(N, A, 99)
    x16 = cuda(logits).to(torch.bfloat16)
    d, stats = fused_ppo_backward(x16, cuda(mask), cuda(action), cuda(old), cuda(adv), cuda(weight),
                                  LossConfig(0.2, 2.0, 0.01))
    x = x16.float().clone().requires_grad_()
    m = cuda(mask)
    z = x.masked_fill(~m, -torch.inf)
    lp = torch.log_softmax(z, -1)
    sel = lp.gather(1, cuda(action).long()[:, None])[:, 0]
    # entropy as the categorical fixture writes it (finite logits off the mask)
    finite = torch.where(m, x, torch.zeros_like(x))
    mx = torch.where(m, finite, torch.full_like(x, -torch.inf)).amax(-1, keepdim=True)
    un = torch.where(m, torch.exp(finite - mx), torch.zeros_like(x))
    nz = un.sum(-1, keepdim=True)
    ent = -((un / nz) * torch.where(m, finite - mx - torch.log(nz), torch.zeros_like(x))).sum(-1)
    lr = sel - cuda(old)
    ratio = lr.exp()
    clipped = ratio.clamp(0.8, 1.2)
    a = cuda(adv)
    neg = torch.minimum(lr, torch.full_like(lr, math.log(2.0))).exp()
    pr = torch.where(a < 0, neg, ratio)
    prow = -torch.minimum(pr * a, clipped * a)
    total = (cuda(weight) * (prow - 0.01 * ent)).sum() / N
    total.backward()
    ref = x.grad
    got = d.float()
    scale = ref.abs().max()
    near = _boundary_rows(host(x16.float()), mask, action, old, 0.2, math.log(2.0))
    _assert_close_except_boundary(host(got), host(ref), near, rtol=2e-2, atol=2e-2 * float(scale))
    torch.testing.assert_close(torch.tensor(float(stats[0])), total.detach().cpu().double().float(), rtol=1e-4,
                               atol=1e-6)


def test_loss_edge_shapes():
    from pbg_b200.loss import LossConfig, fused_ppo_backward

    # empty batch: stats are zero, nothing is written
    z = torch.zeros((0, 8), dtype=torch.bfloat16, device=DEV)
    e = torch.zeros(0, device=DEV)
    d, stats = fused_ppo_backward(z, torch.zeros((0, 8), dtype=torch.bool, device=DEV),
                                  torch.zeros(0, dtype=torch.int32, device=DEV), e, e, e, LossConfig(), inv_count=1.0)
    assert float(stats.abs().sum()) == 0.0
    # unaligned rows fall back to the scalar path with identical results
    N = 1001
    logits, mask, action, old, adv, weight = _loss_inputs(N + 1, 8, 5)
    base = cuda(logits).to(torch.bfloat16)
    d_aligned, _ = fused_ppo_backward(base[1:].contiguous(), cuda(mask[1:]), cuda(action[1:]), cuda(old[1:]),
                                      cuda(adv[1:]), cuda(weight[1:]))
    flat = torch.empty((N + 1) * 8 + 1, dtype=torch.bfloat16, device=DEV)
    view = flat[1:1 + N * 8].view(N, 8)
    view.copy_(base[1:])
    d_unaligned, _ = fused_ppo_backward(view, cuda(mask[1:]), cuda(action[1:]), cuda(old[1:]), cuda(adv[1:]),
                                        cuda(weight[1:]))
    # the scalar path rounds differently from the pair path: both meet the bf16 bar
    ref, _ = O.ppo_categorical(base[1:].float().cpu().numpy(), mask[1:], action[1:], old[1:], adv[1:], weight[1:])
    scale = float(np.abs(ref).max())
    for d in (d_aligned, d_unaligned):
        np.testing.assert_allclose(host(d.float()), ref, rtol=2e-2, atol=2e-2 * scale)


# --------------------------------------------------------------- Adam


def test_adam_matches_reference_golden(gold):
    from pbg_b200.optim import FlatAdam

    g = gold("adam")
    c = g["adam_controls"][0]
    opt = FlatAdam(cuda(g["adam_master0"][0]).clone(), lr=float(c[0]), beta1=float(c[1]), beta2=float(c[2]),
                   epsilon=float(c[3]), decay=float(c[4]), clip=float(c[5]), scale=float(c[6]))
    for s in range(3):
        opt.grad.copy_(cuda(g["adam_grad_in"][s][0]))
        report = host(opt.step())
        assert report[0] == 1.0
        np.testing.assert_allclose(host(opt.master), g["adam_master"][s][0], rtol=1e-5, atol=1e-7)
        np.testing.assert_allclose(host(opt.first), g["adam_first"][s][0], rtol=1e-5, atol=1e-9)
        np.testing.assert_allclose(host(opt.second), g["adam_second"][s][0], rtol=1e-4, atol=1e-12)
        np.testing.assert_allclose(host(opt.grad), g["adam_grad_out"][s][0], rtol=1e-5, atol=1e-9)
    # a non-finite gradient leaves the state untouched and zeroes the gradient
    before = opt.master.clone()
    opt.grad.fill_(1.0)
    opt.grad[7] = float("nan")
    report = host(opt.step())
    assert report[0] == 0.0 and torch.equal(opt.master, before) and float(opt.grad.abs().sum()) == 0.0
    assert int(opt.step_count[0]) == 3


def test_adam_vector_and_scalar_apply_agree():
    """Aligned buffers take the four-per-thread apply, a master offset by one element the scalar one."""

    from pbg_b200.optim import FlatAdam

    n = 100_003
    g = torch.Generator(device=DEV).manual_seed(4)
    start = torch.randn(n + 1, generator=g, device=DEV)
    grads = [torch.randn(n, generator=g, device=DEV) * 1e-2 for _ in range(3)]
    aligned = FlatAdam(start[:n].clone(), lr=1e-3, decay=0.01, clip=0.5)
    shifted_storage = torch.zeros(n + 1, device=DEV)
    shifted_storage[1:] = start[:n]
    shifted = FlatAdam(shifted_storage[1:], lr=1e-3, decay=0.01, clip=0.5)
    assert shifted.master.data_ptr() % 16 != 0
    for grad in grads:
        for opt in (aligned, shifted):
            opt.grad.copy_(grad)
            opt.step()
    torch.testing.assert_close(shifted.master, aligned.master, rtol=1e-6, atol=1e-9)
    torch.testing.assert_close(shifted.first, aligned.first, rtol=1e-6, atol=1e-12)
    torch.testing.assert_close(shifted.second, aligned.second, rtol=1e-6, atol=1e-15)


@pytest.mark.parametrize("dtype,N", [(torch.float32, 5000), (torch.bfloat16, 992 * 40 + 77)])
def test_loss_scale_and_global_mass_normaliser(dtype, N):
    """Non-default loss controls: the objective weight x loss scale (training.py:403; here 2.5) and the
    global decision-mass normaliser of the global-Z variant (inv_count = 1 / sum of every rank's weights,
    here the local sum x 3.7 as if three more ranks' mass were added).  Both scale the gradient and the
    totals linearly; checked against the double-precision oracle with the same controls and against the
    default-control launch scaled by hand.  The bf16 size runs the staged bulk kernel."""

    from pbg_b200.loss import LossConfig, fused_ppo_backward

    A = 8
    logits, mask, action, old, adv, weight = _loss_inputs(N, A, 23)
    x = cuda(logits).to(dtype)
    xs = host(x.float())
    scale, inv = 2.5, 1.0 / (3.7 * float(weight.astype(np.float64).sum()))
    cfg = LossConfig(0.2, 1.5, 0.01)
    d, stats = fused_ppo_backward(x, cuda(mask), cuda(action), cuda(old), cuda(adv), cuda(weight), cfg,
                                  scale=scale, inv_count=inv)
    ref_d, ref_s = O.ppo_categorical(xs, mask, action, old, adv, weight, log_cap=math.log(1.5), scale=scale,
                                     inv_count=inv)
    near = _boundary_rows(xs, mask, action, old, 0.2, math.log(1.5))
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    peak = float(np.abs(ref_d).max())
    _assert_close_except_boundary(host(d.float()), ref_d, near, rtol=tol, atol=tol * peak)
    np.testing.assert_allclose(host(stats)[[0, 1, 2]], ref_s[[0, 1, 2]], rtol=10 * tol, atol=1e-9 * N)
    # linearity against the default controls (1 / N, scale 1)
    d1, s1 = fused_ppo_backward(x, cuda(mask), cuda(action), cuda(old), cuda(adv), cuda(weight), cfg)
    factor = scale * inv * N
    ok = np.isclose(host(d.float()), host(d1.float()) * factor, rtol=tol, atol=tol * peak)
    assert ok.mean() > 0.999
    np.testing.assert_allclose(host(stats)[0], host(s1)[0] * factor, rtol=1e-4)


def test_bulk_staged_path_wraps_the_ring_and_handles_the_tail():
    """694,733 rows: 700 full 992-row tiles (several passes of the 4-stage ring per CTA) + 333 tail rows."""

    from pbg_b200.loss import LossConfig, fused_ppo_backward

    N, A = 992 * 700 + 333, 8
    logits, mask, action, old, adv, weight = _loss_inputs(N, A, 17)
    x16 = cuda(logits).to(torch.bfloat16)
    for step in range(2):  # the scratch counter must reset between launches
        d, stats = fused_ppo_backward(x16, cuda(mask), cuda(action), cuda(old), cuda(adv), cuda(weight),
                                      LossConfig(0.2, 2.0, 0.01))
        assert float(stats[7]) == N, "a bulk stage wait timed out"
    ref, ref_s = O.ppo_categorical(host(x16.float()), mask, action, old, adv, weight, log_cap=math.log(2.0))
    scale = float(np.abs(ref).max())
    near = _boundary_rows(host(x16.float()), mask, action, old, 0.2, math.log(2.0))
    _assert_close_except_boundary(host(d.float()), ref, near, rtol=2e-2, atol=2e-2 * scale)
    np.testing.assert_allclose(host(stats)[[0, 1, 2, 3, 6]], ref_s[[0, 1, 2, 3, 6]], rtol=1e-4, atol=1e-9 * N)


def test_bound_loss_launch_and_graph_replay_match_the_call():
    from pbg_b200.loss import FusedPPOBackward, LossConfig

    N, A = 992 * 40 + 7, 8
    logits, mask, action, old, adv, weight = _loss_inputs(N, A, 23)
    args = [cuda(logits).to(torch.bfloat16), cuda(mask), cuda(action), cuda(old), cuda(adv), cuda(weight)]
    op = FusedPPOBackward(N, A, DEV, LossConfig(0.2, None, 0.01))
    ref_d, ref_s = op(*args)
    ref_d, ref_s = ref_d.clone(), ref_s.clone()
    out = torch.empty_like(args[0])
    bound = op.bind(*args, out)
    bound.launch()
    torch.cuda.synchronize()
    assert torch.equal(out, ref_d) and torch.equal(op.stats, ref_s)
    out.zero_()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        bound.launch()
    for _ in range(2):
        op.stats.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, ref_d) and torch.equal(op.stats, ref_s)


@pytest.mark.parametrize("gi", [0, 1, 3, 6])
def test_direct_model_input_matches_reference_golden(gold, gi):
    """hooks.py:531-612 rows: public and history columns exact, the compact preflop reach within 1e-5."""

    from pbg_b200.poker import HISTORY_FIELDS, NLHEGeometry, PokerHistory, PokerStateMachine

    g = gold("model_input")
    p = gold("poker")
    tag = f"mi{gi}"
    players, stack, ranks = g[f"{tag}_geometry"]
    m = PokerStateMachine(NLHEGeometry(int(players), float(stack), int(ranks)))
    cols = {n: g[f"{tag}_state_{n}"] for n in STATE_MAP}
    s = _dev_state(cols)
    B = s.rows
    dtypes = {"actor": torch.int64, "street": torch.int64, "action": torch.int64, "mask": torch.bool}
    h = PokerHistory(*(cuda(p[f"g{gi}_history_{n}"][:B]).to(dtypes.get(n, torch.float32)) for n in HISTORY_FIELDS))
    reach = cuda(g[f"{tag}_reach"])
    post = f"post_{int(players)}"
    np.testing.assert_array_equal(host(m.direct_model_input(post, s)), g[f"{tag}_post_plain"])
    np.testing.assert_array_equal(host(m.direct_model_input(post, s, reach, h)), g[f"{tag}_post_full"])
    for got, want in ((host(m.direct_model_input("pre", s)), g[f"{tag}_pre_plain"]),
                      (host(m.direct_model_input("pre", s, reach, h)), g[f"{tag}_pre_full"])):
        np.testing.assert_array_equal(np.isinf(got), np.isinf(want))
        fin = np.isfinite(want)
        np.testing.assert_allclose(got[fin], want[fin], rtol=1e-5, atol=1e-6)
