"""Family-scheduled rollout with the policy network in the loop (pbg_b200.family_rollout).

Every step groups the live hands by input partition, encodes each family's retained rows, evaluates
QueuedPokerModel on them and runs the fused rollout step on the scattered raw policy rows.  Checks:
the first step samples every hand from the network's own policy at the owner's class row (the
selected log probability equals the composite policy of the model's raw fields, 1e-5); every hand
terminates with chips conserved; the families seen are the partitions the geometry allows; a rerun
with the same seed is identical (keys are addressed by (root, path), not by batching); and every step
matches the CPU oracle given the raw rows the model wrote, with and without chunked family calls.
"""

import math
import os
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))


def _model(geometry, seed=0):
    import model_params
    from pbg_b200.preflop import PreflopConfig
    from pbg_b200.queued_model import QueuedPokerModel, parameter_shapes

    cfg = PreflopConfig(**dict(model_params.CONFIG, max_players=geometry.players,
                               max_history_tokens=geometry.history_tokens))
    names = parameter_shapes(cfg, geometry.rank_count)
    params = {k: torch.from_numpy(model_params.parameter(k, shape)) for k, shape in names.items()}
    return QueuedPokerModel(geometry, cfg, params, DEV)


def _run(geometry, hands, seed):
    from pbg_b200.family_rollout import FamilyRollout

    roll = FamilyRollout(_model(geometry), seed=seed, iteration=2)
    arena, log_reach = roll.roots(hands, device=DEV)
    actions = []
    for _ in range(4 * geometry.player_node_bound):
        if roll.step(arena, log_reach) == 0:
            break
        actions.append(arena.action.clone())
    return roll, arena, log_reach, actions


@pytest.mark.parametrize("players,stack,ranks", [(2, 8.0, 4), (3, 8.0, 4)])
def test_family_rollout_terminates_and_is_deterministic(players, stack, ranks):
    from pbg_b200.poker import NLHEGeometry

    geometry = NLHEGeometry(players, stack, ranks)
    roll, arena, log_reach, actions = _run(geometry, 64, seed=11)
    assert bool(arena.state.terminal.all())
    total = (arena.state.stacks + arena.state.committed).sum(1)
    assert torch.allclose(total, torch.full_like(total, players * stack), atol=1e-4)
    assert "pre" in roll.families and any(k.startswith("post_") for k in roll.families)
    assert set(roll.families) <= {"pre"} | {f"post_{n}" for n in range(2, players + 1)}
    _, arena2, log_reach2, actions2 = _run(geometry, 64, seed=11)
    assert len(actions) == len(actions2) and all(torch.equal(a, b) for a, b in zip(actions, actions2))
    assert torch.equal(log_reach, log_reach2)
    print(f"\n{players}-handed: {len(actions)} steps, families {roll.families}")


def test_first_step_samples_from_the_networks_policy():
    from pbg_b200.family_rollout import FamilyRollout
    from pbg_b200.policy import PokerPolicyOperator
    from pbg_b200.poker import NLHEGeometry

    geometry = NLHEGeometry(2, 8.0, 4)
    model = _model(geometry)
    roll = FamilyRollout(model, seed=5, iteration=1)
    arena, log_reach = roll.roots(48, device=DEV)
    state0 = arena.state.clone()
    history0 = arena.history.clone()
    rows = roll.machine.direct_model_input("pre", state0, log_reach, history0)
    raw = model.rollout_operation("pre", rows, state0.combo_ids, state0.to_act).policy_raw
    legality = roll.machine.legality(state0)
    probs = PokerPolicyOperator().probabilities(raw, legality)             # [B, K, E]
    roll.step(arena, log_reach)
    owner = state0.to_act.long()
    combo = state0.combo_ids.gather(1, owner[:, None]).squeeze(1).long()
    klass = model.combo_class.index_select(0, combo)
    rows_b = torch.arange(48, device=DEV)
    chosen = probs[rows_b, klass, arena.action.long()]
    want = torch.log(chosen.clamp_min(1e-12))
    torch.testing.assert_close(arena.selected_log, want, rtol=1e-5, atol=1e-5)
    assert math.isfinite(float(arena.selected_log.sum()))


STATE_MAP = {"board_cards": "board", "combo_ids": "combo", "button": "button", "street": "street",
             "to_act": "to_act", "stacks": "stacks", "committed": "committed",
             "committed_street": "committed_street", "status": "status", "current_bet": "current_bet",
             "last_full_raise": "last_full_raise", "pending": "pending", "can_raise": "can_raise",
             "terminal": "terminal"}


@pytest.mark.parametrize("max_rows", [None, {"pre": 16, "post": 8}])
def test_family_rollout_matches_oracle_given_the_models_raw_rows(max_rows):
    """Every step against the CPU oracle: the action sampled from the raw rows the model wrote for
    each hand (class row preflop, combo row after; near-tie rule as in the fused-step test) and the
    whole transition (cards, chips, statuses, histories) bit-exact.  With small ``max_rows`` each
    family is evaluated in several chunks, which must not change anything."""

    import numpy as np

    import oracle as O
    from pbg_b200.family_rollout import FamilyRollout
    from pbg_b200.poker import HISTORY_FIELDS, NLHEGeometry

    geometry = NLHEGeometry(2, 8.0, 4)
    B, seed, iteration = 96, 31, 4
    roll = FamilyRollout(_model(geometry), seed=seed, iteration=iteration, max_rows=max_rows)
    arena, log_reach = roll.roots(B, device=DEV)
    om = O.Machine(O.Geometry(2, 8.0, 4))
    os_ = om.initial_roots(B, seed=seed, iteration=iteration, retry_epoch=0)
    oh = om.empty_history(B)
    path = np.zeros(B, np.int64)
    root = np.arange(B, dtype=np.int64)
    cls = om.combo_class()
    host = lambda t: t.detach().cpu().numpy()  # noqa: E731
    decisions = near_ties = 0
    for step in range(4 * geometry.player_node_bound):
        active = ~os_.terminal.astype(bool)
        n = roll.step(arena, log_reach)
        if n == 0:
            break
        assert n == int(active.sum())
        rows = np.nonzero(active)[0]
        sub = O.State(**{m: np.ascontiguousarray(getattr(os_, m)[rows]) for m in STATE_MAP.values()})
        mask = om.legality(sub)
        combo = sub.combo[np.arange(rows.size), sub.to_act]
        hand = np.where(sub.street == 0, cls[combo], combo)
        keys = O.rng_keys(seed=seed, iteration=iteration, purpose=O.ACTION, root=root[rows], path=path[rows], draw=0)
        raw_np = {k: host(v)[rows] for k, v in roll._raw.items()}
        o_action, o_logp, margin = O.sample_actor(raw_np, mask, hand, keys, with_margin=True)
        g_action = host(arena.action)[rows]
        mismatch = o_action != g_action
        assert np.all(margin[mismatch] < 1e-5), f"step {step}: action differs away from a near tie"
        near_ties += int(mismatch.sum())
        decisions += rows.size
        sub_h = O.History(**{m: np.ascontiguousarray(getattr(oh, m)[rows]) for m in O.History.NAMES})
        nxt, sub_h, child = O.rollout_transition(om, sub, sub_h, g_action.astype(np.int32), seed=seed,
                                                 iteration=iteration, root=root[rows], path=path[rows])
        for m in STATE_MAP.values():
            getattr(os_, m)[rows] = getattr(nxt, m)
        for m in O.History.NAMES:
            getattr(oh, m)[rows] = getattr(sub_h, m)
        path[rows] = child
        for ref, mine in STATE_MAP.items():
            np.testing.assert_array_equal(host(getattr(arena.state, ref)).astype(np.float64),
                                          getattr(os_, mine).astype(np.float64), err_msg=f"step {step} {ref}")
    assert os_.terminal.all()
    for m in HISTORY_FIELDS:
        np.testing.assert_array_equal(host(getattr(arena.history, m)).astype(np.float64),
                                      getattr(oh, m).astype(np.float64), err_msg=m)
    assert near_ties <= max(2, decisions // 1000)
