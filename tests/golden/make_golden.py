"""Generate golden vectors by running the pbg reference on CPU.

Usage::

    python tests/golden/make_golden.py --reference <pbg checkout> [--out tests/golden]

The reference (pbustillo05/ai-game-learning) is GPU-only by design: its state
containers refuse non-accelerator tensors.  The pure functions below those
checks are device-agnostic torch, so this script installs three test-only
shims before calling them:

* ``PokerState.validate`` keeps the reference's shape/dtype/range and chip
  conservation checks but accepts CPU tensors (hooks.py:268-326);
* ``PokerLegality.__post_init__`` keeps the legality checks without the
  device test (policy.py:34-52);
* ``PokerStateMachine.initial_roots`` is re-compiled from the reference's own
  source with only its device-type guard removed (hooks.py:369-371);
* ``CollisionConditionedProfileSampler.sample_children`` likewise
  (rb_sampling.py:107-108);
* ``folded._folded_statistics_fp32`` likewise (its board device-type test,
  folded.py:251), and the model runs lift ``tensor_ops._accelerator`` and the
  device test of ``MHA.forward``.

Everything else runs unmodified.  The fixtures are small ``.npz`` files that
the ``-m "not gpu"`` tests use to pin the oracle and the ``-m gpu`` tests use
to pin the CUDA library.
"""

from __future__ import annotations

import argparse
import inspect
import json
import math
import os
import sys
import textwrap
from types import MappingProxyType

import numpy as np


def _install_shims():
    import torch
    from pbg.games.poker.queued import hooks, policy

    def validate(self, geometry):  # hooks.py:268-326 without the device test
        batch, players = self.rows, geometry.players
        expect = {
            "board_cards": (torch.uint8, (batch, 5)), "combo_ids": (torch.int32, (batch, players)),
            "button": (torch.int32, (batch,)), "street": (torch.int32, (batch,)),
            "to_act": (torch.int32, (batch,)), "stacks": (torch.float32, (batch, players)),
            "committed": (torch.float32, (batch, players)),
            "committed_street": (torch.float32, (batch, players)),
            "status": (torch.int8, (batch, players)), "current_bet": (torch.float32, (batch,)),
            "last_full_raise": (torch.float32, (batch,)), "pending": (torch.bool, (batch, players)),
            "can_raise": (torch.bool, (batch, players)), "terminal": (torch.bool, (batch,)),
        }
        for name, (dtype, shape) in expect.items():
            value = getattr(self, name)
            assert value.dtype == dtype and tuple(value.shape) == shape, name
        assert bool((self.stacks >= 0).all())
        total = (self.stacks + self.committed).sum(-1)
        assert bool(((total - players * geometry.stack_bb).abs() <= 1e-5).all())

    hooks.PokerState.validate = validate

    def legality_post_init(self):  # policy.py:34-52 without the device test
        assert self.event_ids.ndim == 2 and self.mask.shape == self.event_ids.shape
        assert bool(self.mask.any(-1).all())

    policy.PokerLegality.__post_init__ = legality_post_init

    source = textwrap.dedent(inspect.getsource(hooks.PokerStateMachine.initial_roots))
    guard = 'if device.type not in ("cuda", "mps"):'
    assert guard in source, "reference initial_roots changed shape"
    source = source.replace(guard, "if False:")
    namespace: dict = {}
    exec(compile(source, hooks.__file__, "exec"), hooks.__dict__, namespace)
    hooks.PokerStateMachine.initial_roots = namespace["initial_roots"]

    from pbg.games.poker.queued import rb_sampling

    source = textwrap.dedent(inspect.getsource(rb_sampling.CollisionConditionedProfileSampler.sample_children))
    guard = 'if device.type != "cuda":'
    assert guard in source, "reference sample_children changed shape"
    source = source.replace(guard, "if False:")
    namespace = {}
    exec(compile(source, rb_sampling.__file__, "exec"), rb_sampling.__dict__, namespace)
    rb_sampling.CollisionConditionedProfileSampler.sample_children = namespace["sample_children"]


STATE_FIELDS = ("board_cards", "combo_ids", "button", "street", "to_act", "stacks", "committed",
                "committed_street", "status", "current_bet", "last_full_raise", "pending",
                "can_raise", "terminal")
HISTORY_FIELDS = ("actor", "street", "action", "amount", "pot_before", "call_amount",
                  "current_bet", "min_raise_to", "max_raise_to", "mask")

GEOMETRIES = [(2, 8.0, 4), (3, 8.0, 4), (6, 8.0, 13), (2, 100.0, 13), (6, 100.0, 13),
              (6, 50.0, 13), (4, 20.5, 9)]


def _np(t):
    return t.detach().cpu().numpy().copy()


def gen_rng(out):
    import torch
    from pbg.core.rollout import (DrawPurpose, child_path_keys, logical_categorical,
                                  logical_rng_keys, logical_uniform)

    rng = np.random.default_rng(20261201)
    n = 64
    cases = []
    for case in range(24):
        seed = int(rng.integers(-2**40, 2**62)) if case % 3 else case
        iteration = int(rng.integers(0, 2**20))
        purpose = int(1 + case % 8)
        root = rng.integers(0, 2**62, n) if case % 2 else rng.integers(0, 4096, n)
        path = np.where(rng.random(n) < 0.3, 0, rng.integers(-2**63, 2**63 - 1, n, dtype=np.int64))
        draw = rng.integers(0, 4096, n)
        lane = rng.integers(0, 8, n)
        epoch = rng.integers(0, 4, n)
        active = rng.random(n) < 0.8
        keys = logical_rng_keys(seed=seed, iteration=iteration, root=torch.from_numpy(root),
                                path=torch.from_numpy(path), draw=torch.from_numpy(draw),
                                purpose=purpose, lane=torch.from_numpy(lane),
                                retry_epoch=torch.from_numpy(epoch),
                                active=torch.from_numpy(active))
        cases.append((seed, iteration, purpose, root, path, draw, lane, epoch, active, _np(keys)))
    out["rng_scalars"] = np.array([[c[0], c[1], c[2]] for c in cases], dtype=np.int64)
    for i, name in enumerate(("root", "path", "draw", "lane", "epoch")):
        out[f"rng_{name}"] = np.stack([c[3 + i] for c in cases]).astype(np.int64)
    out["rng_active"] = np.stack([c[8] for c in cases]).astype(np.uint8)
    out["rng_keys"] = np.stack([c[9] for c in cases])
    ords = rng.integers(1, 1 << 20, (24, n))
    out["rng_child_ordinal"] = ords.astype(np.int64)
    out["rng_child"] = np.stack([
        _np(child_path_keys(torch.from_numpy(out["rng_path"][i]), torch.from_numpy(ords[i])))
        for i in range(24)])
    flat = out["rng_keys"].reshape(-1)
    extra = np.array([0, ((1 << 24) - 1) << 39, (1 << 39) - 1, 1 << 39, 2**63 - 1], dtype=np.int64)
    ukeys = np.concatenate([flat, extra])
    out["rng_uniform_keys"] = ukeys
    out["rng_uniform"] = _np(logical_uniform(torch.from_numpy(ukeys)))
    probs = rng.random((256, 12)).astype(np.float32) * (rng.random((256, 12)) < 0.6)
    probs[:, 3] += 1e-3
    probs = probs / probs.sum(1, keepdims=True)
    ckeys = flat[:256]
    out["cat_prob"] = probs.astype(np.float32)
    out["cat_keys"] = ckeys
    out["cat_selected"] = _np(logical_categorical(torch.from_numpy(probs.astype(np.float32)),
                                                  torch.from_numpy(ckeys)))
    assert DrawPurpose.ACTION == 4


def _state_np(state):
    return {name: _np(getattr(state, name)) for name in STATE_FIELDS}


def _state_from(cols, rows=None):
    import torch
    from pbg.games.poker.queued.hooks import PokerState
    sel = (lambda v: v) if rows is None else (lambda v: v[rows])
    return PokerState(*(torch.from_numpy(np.ascontiguousarray(sel(cols[n]))) for n in STATE_FIELDS))


def gen_poker(out):
    import torch
    from pbg.core.rollout import child_path_keys
    from pbg.games.poker.queued.hooks import NLHEGeometry, PokerHistory, PokerStateMachine

    rng = np.random.default_rng(7)
    for gi, (players, stack, ranks) in enumerate(GEOMETRIES):
        geometry = NLHEGeometry(players, stack, ranks)
        machine = PokerStateMachine(geometry)
        tag = f"g{gi}"
        # roots: two calls with distinct addresses
        seed, iteration, retry, base, lane = 1000 + gi, 3 + gi, gi % 3, 17 * gi, gi % 2
        B = 16 if players == 6 and stack >= 50 else 24
        state = machine.initial_roots(B, seed=seed, iteration=iteration, retry_epoch=retry,
                                      logical_base=base, lane=lane, device="cpu")
        out[f"{tag}_geometry"] = np.array([players, stack, ranks], dtype=np.float64)
        out[f"{tag}_root_args"] = np.array([seed, iteration, retry, base, lane, B], dtype=np.int64)
        for k, v in _state_np(state).items():
            out[f"{tag}_root_{k}"] = v
        # trajectory with random legal actions and keyed chance at (root, path)
        cols = _state_np(state)
        history = machine.empty_history(B, torch.device("cpu"))
        hist = {n: _np(getattr(history, n)) for n in HISTORY_FIELDS}
        path = np.zeros(B, dtype=np.int64)
        root = np.arange(base, base + B, dtype=np.int64)
        actions, masks, posts = [], [], []
        step = 0
        while not cols["terminal"].all():
            active = ~cols["terminal"]
            rows = np.nonzero(active)[0]
            sub = _state_from(cols, rows)
            legality = machine.legality(sub)
            mask = _np(legality.mask)
            chosen = np.full(B, -1, dtype=np.int32)
            for i, r in enumerate(rows):
                legal = np.nonzero(mask[i])[0]
                u = rng.random()
                if u < 0.15 and mask[i, 0]:
                    pick = 0
                elif u < 0.55:
                    pick = 1
                else:
                    raises = legal[legal >= 2]
                    pick = int(rng.choice(raises)) if raises.size else 1
                chosen[r] = pick
            full_mask = np.zeros((B, geometry.stack_ticks + 2), dtype=bool)
            full_mask[rows] = mask
            action = torch.from_numpy(chosen[rows])
            sub_hist = PokerHistory(*(torch.from_numpy(np.ascontiguousarray(hist[n][rows])) for n in HISTORY_FIELDS))
            sub_hist = machine.append_player_history(sub, action, sub_hist)
            nxt = machine.step_player(sub, action)
            sub_root = torch.from_numpy(root[rows])
            sub_path = torch.from_numpy(path[rows])
            for generation in range(3):
                chance_active = machine.needs_chance(nxt)
                sub_hist = machine.append_chance_history(nxt, chance_active, sub_hist)
                nxt = machine.deal_next_street_keyed(nxt, seed=seed, iteration=iteration, root=sub_root,
                                                     path=sub_path, draw=generation,
                                                     retry_epoch=retry, lane=lane)
            new = _state_np(nxt)
            for n in STATE_FIELDS:
                cols[n][rows] = new[n]
            for n in HISTORY_FIELDS:
                hist[n][rows] = _np(getattr(sub_hist, n))
            path[rows] = _np(child_path_keys(sub_path, 1))
            actions.append(chosen)
            masks.append(full_mask)
            posts.append({n: cols[n].copy() for n in STATE_FIELDS})
            step += 1
            assert step < 400
        out[f"{tag}_actions"] = np.stack(actions)
        out[f"{tag}_masks"] = np.packbits(np.stack(masks), axis=-1)
        out[f"{tag}_mask_events"] = np.array([geometry.stack_ticks + 2])
        for n in STATE_FIELDS:
            out[f"{tag}_post_{n}"] = np.stack([p[n] for p in posts])
        for n in HISTORY_FIELDS:
            out[f"{tag}_history_{n}"] = hist[n].astype(np.float32 if hist[n].dtype.kind == "f" else np.int16)
        out[f"{tag}_final_path"] = path
        leaf = machine.sampled_leaf(_state_from(cols))
        for k, v in leaf.items():
            out[f"{tag}_leaf_{k}"] = _np(v)
        out[f"{tag}_combo_class"] = _np(machine._combo_class(torch.device("cpu"))).astype(np.int32)


def gen_known_answers(out):
    """Literal expected states from the reference's own tests, re-derived."""

    import torch
    from pbg.games.poker.queued.hooks import NLHEGeometry, PokerStateMachine

    machine = PokerStateMachine(NLHEGeometry(3, 8.0, 4))
    state = machine.initial_roots(1, seed=71, iteration=0, retry_epoch=0, device="cpu")
    for a in (13, 1, 17):
        state = machine.step_player(state, torch.tensor([a], dtype=torch.int32))
    out["ka_repend_committed_street"] = _np(state.committed_street)
    out["ka_repend_pending"] = _np(state.pending)
    out["ka_repend_can_raise"] = _np(state.can_raise)
    out["ka_repend_to_act"] = _np(state.to_act)
    out["ka_repend_mask"] = _np(machine.legality(state).mask)


def _raw(rng, batch, hands, mixture):
    import torch
    g = torch.Generator().manual_seed(int(rng.integers(0, 2**31)))
    return {
        "type_logits": torch.randn(batch, hands, 3, generator=g) * 1.5,
        "omega": torch.softmax(torch.randn(batch, hands, mixture, generator=g), -1),
        "mu": torch.sigmoid(torch.randn(batch, hands, mixture, generator=g)),
        "s": torch.nn.functional.softplus(torch.randn(batch, hands, mixture, generator=g)) + 0.02,
        "iota": torch.sigmoid(torch.randn(batch, hands, generator=g)),
    }


def gen_policy(out, poker):
    import torch
    from pbg.games.poker.queued.policy import PokerLegality, PokerPolicyOperator

    rng = np.random.default_rng(11)
    op = PokerPolicyOperator()
    cases = [("small", 0, 10, 3, 5), ("hu8", 0, 18, 2, 4), ("hu100", 3, 202, 2, 3), ("six50", 5, 102, 2, 3)]
    for name, gi, E, M, H in cases:
        if name == "small":
            B = 6
            mask = rng.random((B, E)) < 0.6
            mask[:, 1] = True
            mask[1] = False
            mask[1, 1] = True
        else:
            packed = poker[f"g{gi}_masks"]
            masks = np.unpackbits(packed, axis=-1)[..., :E].astype(bool).reshape(-1, E)
            masks = masks[masks.any(1)]
            B = min(48, masks.shape[0])
            mask = masks[rng.choice(masks.shape[0], B, replace=False)]
        raw = _raw(rng, B, H, M)
        ids = torch.arange(E, dtype=torch.int32)[None].expand(B, -1).contiguous()
        legality = PokerLegality(ids, torch.from_numpy(mask))
        prob = op.probabilities(raw, legality)
        out[f"pol_{name}_mask"] = mask.astype(np.uint8)
        for k, v in raw.items():
            out[f"pol_{name}_{k}"] = _np(v)
        out[f"pol_{name}_prob"] = _np(prob)
        hand = torch.from_numpy(rng.integers(0, H, B).astype(np.int32))
        keys = torch.from_numpy(rng.integers(0, 2**63 - 1, B, dtype=np.int64))
        sample = op.sample_actor(raw, legality, hand, keys)
        out[f"pol_{name}_hand"] = _np(hand)
        out[f"pol_{name}_keys"] = _np(keys)
        out[f"pol_{name}_action"] = _np(sample.action)
        out[f"pol_{name}_selected"] = _np(sample.selected_log_policy)
        out[f"pol_{name}_selected_all"] = _np(op.selected_log_pi(raw, legality, sample.action))
        entropy, kl = op.policy_reductions(raw, legality, None)
        out[f"pol_{name}_entropy"] = _np(entropy)


def gen_loss(out):
    import torch
    from pbg.config import EntropyLossConfig, LossConfig, ValueLossConfig
    from pbg.core.contracts import mode_schema
    from pbg.core.learner import LearnerOperation, ModelEvaluation, PolicyEvaluation, SequentialLearnerBatch

    from categorical_policy_fixture import CategoricalPolicyAdapter, PolicyOutput

    adapter = CategoricalPolicyAdapter()
    ids = torch.arange(8)[None]
    rng = np.random.default_rng(5)
    N, A = 160, 8
    logits = rng.standard_normal((N, A)).astype(np.float32)
    mask = rng.random((N, A)) < 0.7
    empty = ~mask.any(1)
    mask[empty, 0] = True
    action = np.array([rng.choice(np.nonzero(m)[0]) for m in mask], dtype=np.int32)
    # old log pi: perturbed logits; spread wide enough that some rows clip
    pert = logits + rng.standard_normal((N, A)).astype(np.float32) * np.float32(0.1)
    pert[: N // 4] += rng.standard_normal((N // 4, A)).astype(np.float32) * np.float32(1.5)
    masked = np.where(mask, pert, -np.inf)
    lse = np.log(np.exp(masked - masked.max(1, keepdims=True)).sum(1)) + masked.max(1)
    old = (masked[np.arange(N), action] - lse).astype(np.float32)
    adv = rng.standard_normal(N).astype(np.float32)
    weight = rng.uniform(0.05, 1.0, N).astype(np.float32)
    caps = [None, 1.5]
    for ci, cap in enumerate(caps):
        per_total = np.zeros(N, dtype=np.float64)
        grads = np.zeros((N, A), dtype=np.float32)
        cfg = LossConfig(policy_clip=0.2, negative_advantage_ratio_cap=cap,
                         value=ValueLossConfig(coefficient=0.0),
                         entropy=EntropyLossConfig(coefficient=0.01))
        for r in range(N):
            x = torch.tensor(logits[r : r + 1], requires_grad=True)
            mrow = torch.from_numpy(mask[r : r + 1])

            def model(input_type, model_input, private, owner, x=x):
                return ModelEvaluation({"logits": x[:, None, :]}, torch.zeros(1, 1))

            def policy(name, mi, raw, act, private, owner, ref, mrow=mrow):
                # the reference's game-neutral categorical fixture
                # (tests/categorical_policy_fixture.py:19-57)
                pout = PolicyOutput(raw["logits"].reshape(1, 1, A).float(), None)
                sel = adapter.log_prob(pout, act.long(), ids, mrow).reshape(1)
                ent = adapter.entropy(pout, ids, mrow).reshape(1)
                return PolicyEvaluation(sel, ent, torch.zeros_like(sel))

            fields = MappingProxyType({
                "model_input": torch.zeros(1, 1), "owner": torch.zeros(1, dtype=torch.int32),
                "sampled_private_state": torch.zeros(1, 2, dtype=torch.int32),
                "action": torch.tensor(action[r : r + 1]),
                "old_log_policy": torch.tensor(old[r : r + 1, None]),
                "old_value": torch.zeros(1, 1), "value_target": torch.zeros(1, 1),
                "advantage_target": torch.tensor(adv[r : r + 1, None]),
            })
            op = LearnerOperation(mode_schema("self_play", "sequential", "sampled"), cfg, model, policy)
            res = op.forward_loss_backward(SequentialLearnerBatch("pre", torch.zeros(1, dtype=torch.int64), fields),
                                           iteration=0, objective_weight=float(weight[r]))
            per_total[r] = float(res.total)
            grads[r] = _np(x.grad)[0]
        out[f"loss{ci}_row_total"] = per_total
        out[f"loss{ci}_grad"] = grads
        out[f"loss{ci}_cap"] = np.array([np.inf if cap is None else math.log(cap)], dtype=np.float64)
    out["loss_logits"] = logits
    out["loss_mask"] = mask.astype(np.uint8)
    out["loss_action"] = action
    out["loss_old"] = old
    out["loss_adv"] = adv
    out["loss_weight"] = weight


def gen_adam(out):
    import torch
    from pbg.core.optimization import adam_transition

    rng = np.random.default_rng(3)
    n = 4096
    master = torch.from_numpy(rng.standard_normal((1, n)).astype(np.float32))
    first = torch.zeros(1, n)
    second = torch.zeros(1, n)
    controls = torch.tensor([[1e-3, 0.9, 0.999, 1e-8, 0.01, 1.0, 128.0, 2.0, 0.5, 2000.0]])
    steps = torch.zeros(1, dtype=torch.int64)
    trackers = torch.zeros(1, dtype=torch.int64)
    out["adam_master0"] = _np(master).copy()
    out["adam_controls"] = _np(controls).copy()
    grads_in, masters, firsts, seconds, grads_out = [], [], [], [], []
    for s in range(3):
        g = torch.from_numpy((rng.standard_normal((1, n)) * (0.05 if s != 1 else 3.0) * 128.0).astype(np.float32))
        grads_in.append(_np(g).copy())
        adam_transition(master, g, first, second, controls, steps, trackers,
                        torch.tensor([False]), torch.tensor([True]), torch.tensor([True]), torch.tensor([False]))
        masters.append(_np(master).copy())
        firsts.append(_np(first).copy())
        seconds.append(_np(second).copy())
        grads_out.append(_np(g).copy())
    out["adam_grad_in"] = np.stack(grads_in)
    out["adam_master"] = np.stack(masters)
    out["adam_first"] = np.stack(firsts)
    out["adam_second"] = np.stack(seconds)
    out["adam_grad_out"] = np.stack(grads_out)


def gen_model_input(out, poker):
    """hooks.py:531-612 (direct_model_input) on trajectory states, with and without reach/history."""

    import torch
    from pbg.games.poker.queued.hooks import NLHEGeometry, PokerHistory, PokerStateMachine

    rng = np.random.default_rng(13)
    for gi in (0, 1, 3, 6):
        players, stack, ranks = poker[f"g{gi}_geometry"]
        geometry = NLHEGeometry(int(players), float(stack), int(ranks))
        machine = PokerStateMachine(geometry)
        tag = f"mi{gi}"
        steps = poker[f"g{gi}_post_board_cards"].shape[0]
        t = min(2, steps - 1)
        cols = {n: poker[f"g{gi}_post_{n}"][t][:8] for n in STATE_FIELDS}
        cols["terminal"] = np.zeros_like(cols["terminal"])
        state = _state_from(cols)
        B, P, H = state.rows, geometry.players, geometry.private_hands
        reach = rng.standard_normal((B, P, H)).astype(np.float32) * 3.0
        reach[rng.random((B, P, H)) < 0.2] = -np.inf
        reach[0, 0, :] = -np.inf  # a seat with no finite reach
        hist = {n: poker[f"g{gi}_history_{n}"][:8] for n in HISTORY_FIELDS}
        history = PokerHistory(*(torch.from_numpy(np.ascontiguousarray(
            hist[n].astype(np.int64) if n in ("actor", "street", "action") else
            (hist[n].astype(bool) if n == "mask" else hist[n].astype(np.float32)))) for n in HISTORY_FIELDS))
        for k, v in cols.items():
            out[f"{tag}_state_{k}"] = v
        out[f"{tag}_geometry"] = np.array([players, stack, ranks])
        out[f"{tag}_reach"] = reach
        out[f"{tag}_pre_plain"] = _np(machine.direct_model_input("pre", state))
        out[f"{tag}_pre_full"] = _np(machine.direct_model_input("pre", state, torch.from_numpy(reach), history))
        post = f"post_{P}"
        out[f"{tag}_post_plain"] = _np(machine.direct_model_input(post, state))
        out[f"{tag}_post_full"] = _np(machine.direct_model_input(post, state, torch.from_numpy(reach), history))


def gen_posterior(out):
    """rb_sampling.py:86-223: collision-conditioned posterior profiles on seeded parents."""

    import torch
    from pbg.games.poker.queued.hooks import NLHEGeometry, PAD_CARD
    from pbg.games.poker.queued.rb_sampling import CollisionConditionedProfileSampler

    cases = [((2, 8.0, 4), 256, "int"), ((3, 8.0, 4), 256, "tensor"), ((6, 100.0, 13), 256, "int"),
             ((4, 20.5, 9), 256, "tensor"), ((4, 8.0, 4), 3, "int"), ((3, 8.0, 4), 1, "tensor")]
    for ci, ((players, stack, ranks), attempts, epoch_kind) in enumerate(cases):
        g = torch.Generator().manual_seed(1000 + ci)
        geometry = NLHEGeometry(players, stack, ranks)
        hands, deck, first = geometry.private_hands, geometry.deck_cards, geometry.first_card
        parents, edges = 12, 48
        weights = torch.rand((parents, players, hands), generator=g)
        weights[torch.rand(weights.shape, generator=g) < 0.3] = 0.0
        if attempts <= 3:  # concentrate mass on a few combos so collisions (and exhaustion) happen
            keep = torch.rand(weights.shape, generator=g) < (6.0 / hands)
            weights = torch.where(keep, weights + 0.1, torch.zeros_like(weights))
            weights[..., 0] += 1.0
        board = torch.full((parents, 5), PAD_CARD, dtype=torch.uint8)
        for b in range(parents):
            shown = [0, 3, 4, 5][b % 4]
            cards = torch.randperm(deck, generator=g)[:shown] + first
            board[b, :shown] = cards.to(torch.uint8)
        # every seat of every parent keeps some board-legal mass (the reference asserts it)
        # every seat of every parent keeps some board-legal mass (the reference asserts it)
        pairs = torch.tensor([(i + first, j + first) for i in range(deck) for j in range(i + 1, deck)])
        for b in range(parents):
            shown = board[b][board[b] != PAD_CARD].long()
            legal = ~((pairs[:, :, None] == shown[None, None, :]).any(-1).any(-1))
            for p in range(players):
                if float((weights[b, p] * legal).sum()) == 0.0:
                    pick = torch.nonzero(legal).flatten()
                    weights[b, p, pick[int(torch.randint(0, pick.numel(), (1,), generator=g))]] = 0.5
        inherited = torch.randint(0, hands, (parents, players), generator=g, dtype=torch.int32)
        source = torch.randint(0, parents, (edges,), generator=g, dtype=torch.int64)
        ordinal = torch.randint(0, 4, (edges,), generator=g, dtype=torch.int64)
        active = torch.rand((edges,), generator=g) < 0.85
        root = torch.randint(0, 2**62, (edges,), generator=g, dtype=torch.int64)
        path = torch.randint(-2**62, 2**62, (edges,), generator=g, dtype=torch.int64)
        # an epoch tensor must broadcast against the [edge, attempt, seat] address grid
        epoch = 3 if epoch_kind == "int" else torch.randint(0, 5, (edges, 1, 1), generator=g, dtype=torch.int64)
        sampler = CollisionConditionedProfileSampler(geometry, max_attempts=attempts)
        seed, iteration = 77 + ci, 5 + ci
        result = sampler.sample_children(range_weights=weights, board_cards=board, inherited_profile=inherited,
                                         source=source, ordinal=ordinal, active=active, root=root, path=path,
                                         seed=seed, iteration=iteration, retry_epoch=epoch)
        obs = sampler.last_observation
        pre = f"c{ci}_"
        out[pre + "geometry"] = np.array([players, stack, ranks], dtype=np.float64)
        out[pre + "max_attempts"] = np.array(attempts)
        out[pre + "seed_iteration"] = np.array([seed, iteration], dtype=np.int64)
        for name, value in (("weights", weights), ("board", board), ("inherited", inherited), ("source", source),
                            ("ordinal", ordinal), ("active", active), ("root", root), ("path", path)):
            out[pre + name] = _np(value)
        out[pre + "epoch"] = (_np(epoch).reshape(edges).astype(np.int64) if torch.is_tensor(epoch)
                              else np.full((edges,), epoch, dtype=np.int64))
        out[pre + "result"] = _np(result)
        out[pre + "attempt_count"] = _np(obs.attempt_count)
        out[pre + "exhausted"] = _np(obs.exhausted)
        out[pre + "minimum_failing"] = np.array(int(obs.minimum_failing_address))
    out["cases"] = np.array(len(cases))


def _gradient_sketch(out, modules, outputs):
    """The reference's own autograd gradient of a seeded loss sum_f <c_f, output_f> (c_f ~ N(0, 1),
    recorded as gcoef_<field>) with respect to every parameter of ``modules``, sketched per parameter
    by its norm (gsk_norm) and its projections onto model_params.probe's vectors (gsk_proj)."""

    import torch

    import model_params

    g = torch.Generator().manual_seed(4242)
    loss = 0.0
    for name, value in outputs.items():
        c = torch.randn(value.shape, generator=g)
        out["gcoef_" + name] = _np(c)
        loss = loss + (c * value).sum()
    params = [(n, q) for m in modules for n, q in m.named_parameters()]
    for _, q in params:
        q.grad = None
    loss.backward()
    names, norms, projections = [], [], []
    for n, q in params:
        grad = torch.zeros_like(q) if q.grad is None else q.grad
        flat = grad.detach().reshape(-1).double().numpy()
        names.append(n)
        norms.append(float(np.linalg.norm(flat)))
        projections.append(model_params.probe(n, tuple(q.shape)) @ flat)
    out["gsk_names"] = np.array(names)
    out["gsk_norm"] = np.array(norms)
    out["gsk_proj"] = np.stack(projections)


def gen_preflop_model(out, config=None, ranks=None, batch=3, tokens=8):
    """preflop.py:472-693 (PreflopEncoder.forward) with shared.py's trunk and readout, fp32 on CPU.

    The reference's accelerator guards (tensor_ops._accelerator, MHA.forward's device check) are
    lifted for this run only; weights come from tests/golden/model_params.py by name.  ``config`` /
    ``ranks`` default to model_params.CONFIG / RANKS; both are recorded in the fixture.
    """

    import inspect
    import textwrap

    import torch
    from pbg.core import tensor_ops
    from pbg.games.poker.cards import DeckGeometry
    from pbg.games.poker.model import primitives
    from pbg.games.poker.model.preflop import (PackedPublicHistory, PokerModelConfig, PokerPublicBatch,
                                               PreflopEncoder, PreflopMasks)
    from pbg.games.poker.model.shared import SharedPokerParameters

    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    import model_params

    tensor_ops._accelerator = lambda value: None
    source = textwrap.dedent(inspect.getsource(primitives.MHA.forward))
    guard = 'if q.device.type not in ("cuda", "mps"):'
    if guard in source:  # (a previous generator in this run may have lifted it already)
        namespace: dict = {}
        exec(compile(source.replace(guard, "if False:"), primitives.__file__, "exec"), primitives.__dict__,
             namespace)
        primitives.MHA.forward = namespace["forward"]

    config = dict(model_params.CONFIG if config is None else config)
    ranks = model_params.RANKS if ranks is None else ranks
    cfg = PokerModelConfig(**config)
    geometry = DeckGeometry(ranks)
    shared = SharedPokerParameters(cfg, geometry.n_cards)
    encoder = PreflopEncoder(cfg, geometry)
    out["config_json"] = np.array(json.dumps(config))
    out["ranks"] = np.array(ranks)
    with torch.no_grad():
        for module in (shared, encoder):
            for name, param in module.named_parameters():
                param.copy_(torch.from_numpy(model_params.parameter(name, tuple(param.shape))))
    g = torch.Generator().manual_seed(2024)
    players = 2
    k = geometry.n_classes
    history = PackedPublicHistory(
        actor=torch.randint(-1, players, (batch, tokens), generator=g),
        street=torch.randint(0, 4, (batch, tokens), generator=g),
        action=torch.randint(0, 4, (batch, tokens), generator=g),
        amount=torch.rand((batch, tokens), generator=g) * 4,
        pot_before=torch.rand((batch, tokens), generator=g) * 6,
        call_amount=torch.rand((batch, tokens), generator=g),
        current_bet=torch.rand((batch, tokens), generator=g) * 2,
        min_raise_to=torch.rand((batch, tokens), generator=g) * 2,
        max_raise_to=torch.rand((batch, tokens), generator=g) * 8,
        mask=torch.rand((batch, tokens), generator=g) < 0.7,
    )
    history.mask[:, 0] = True
    pub = PokerPublicBatch(
        street=torch.zeros(batch, dtype=torch.long),
        board=torch.full((batch, 5), 255, dtype=torch.long),
        pot=torch.rand(batch, generator=g) * 3 + 1.5,
        stacks=torch.rand((batch, players), generator=g) * 8,
        committed=torch.rand((batch, players), generator=g),
        to_act=torch.randint(0, players, (batch,), generator=g),
        legality_summary=torch.rand((batch, 4), generator=g),
        n_ticks=torch.full((batch,), 16.0),
        raise_grid_bounds=torch.rand((batch, 2), generator=g),
        status=torch.randint(0, 3, (batch, players), generator=g),
        seat_mask=torch.ones((batch, players), dtype=torch.bool),
        button=torch.randint(0, players, (batch,), generator=g),
        committed_street=torch.rand((batch, players), generator=g),
        call_amount=torch.rand(batch, generator=g),
        current_bet=torch.rand(batch, generator=g) * 2,
        min_raise_to=torch.rand(batch, generator=g) * 2,
        max_raise_to=torch.rand(batch, generator=g) * 8,
        last_full_raise=torch.ones(batch),
        legal_action_mask=torch.rand((batch, 6), generator=g) < 0.8,
        raise_ticks=torch.rand((batch, 5), generator=g),
        history=history,
    )
    ranges = torch.rand((batch, players, k), generator=g)
    ranges[torch.rand(ranges.shape, generator=g) < 0.25] = 0.0
    class_mask = torch.rand((batch, players, k), generator=g) < 0.9
    masks = PreflopMasks(class_mask=class_mask)
    with torch.no_grad():
        result = encoder(shared, pub, ranges, None, masks)
    for name in ("street", "board", "pot", "stacks", "committed", "to_act", "legality_summary", "n_ticks",
                 "raise_grid_bounds", "status", "seat_mask", "button", "committed_street", "call_amount",
                 "current_bet", "min_raise_to", "max_raise_to", "last_full_raise", "legal_action_mask",
                 "raise_ticks"):
        out["pub_" + name] = _np(getattr(pub, name))
    for name in ("actor", "street", "action", "amount", "pot_before", "call_amount", "current_bet",
                 "min_raise_to", "max_raise_to", "mask"):
        out["hist_" + name] = _np(getattr(history, name))
    out["class_ranges"] = _np(ranges)
    out["class_mask"] = _np(class_mask)
    for name, value in result.raw.items():
        out["raw_" + name] = _np(value)
    out["value"] = _np(result.v)
    spec = []
    for module in (shared, encoder):
        for name, param in module.named_parameters():
            spec.append(name + ":" + ",".join(str(n) for n in param.shape))
    out["param_spec"] = np.array(spec)
    out["class_sizes"] = _np(encoder.class_sizes)
    out["class_card_geometry"] = _np(encoder.class_card_geometry)
    out["class_overlap_scalars"] = _np(encoder.class_overlap_scalars)
    result = encoder(shared, pub, ranges, None, masks)
    _gradient_sketch(out, (shared, encoder), {**result.raw, "value": result.v})


def gen_postflop_model(out, config=None, ranks=None):
    """postflop.py:538-784 (PostflopEncoder.forward) with shared.py's trunk and readout, fp32 on CPU.

    Three seats (one folded, so the folder context is live), a flop or turn board, the compact
    board-compatible combo rows, and evaluator-summary fields of the shapes the encoder reads
    (hand log ratios, beta eigenpairs, folder masses / single-card ratios / line metadata / seats,
    tight-cluster scalar) drawn at random; accelerator guards lifted as for the preflop run.
    """

    import inspect
    import textwrap

    import torch
    from pbg.core import tensor_ops
    from pbg.games.poker.cards import DeckGeometry
    from pbg.games.poker.model import primitives
    from pbg.games.poker.model.postflop import PostflopEncoder, PostflopMasks
    from pbg.games.poker.model.preflop import PackedPublicHistory, PokerModelConfig, PokerPublicBatch
    from pbg.games.poker.model.shared import SharedPokerParameters

    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    import model_params

    tensor_ops._accelerator = lambda value: None
    source = textwrap.dedent(inspect.getsource(primitives.MHA.forward))
    guard = 'if q.device.type not in ("cuda", "mps"):'
    if guard in source:
        namespace: dict = {}
        exec(compile(source.replace(guard, "if False:"), primitives.__file__, "exec"), primitives.__dict__, namespace)
        primitives.MHA.forward = namespace["forward"]

    config = dict(model_params.POSTFLOP_CONFIG if config is None else config)
    ranks = model_params.RANKS if ranks is None else ranks
    cfg = PokerModelConfig(**config)
    geometry = DeckGeometry(ranks)
    shared = SharedPokerParameters(cfg, geometry.n_cards)
    encoder = PostflopEncoder(cfg, geometry)
    out["config_json"] = np.array(json.dumps(config))
    out["ranks"] = np.array(ranks)
    with torch.no_grad():
        for module in (shared, encoder):
            for name, param in module.named_parameters():
                param.copy_(torch.from_numpy(model_params.parameter(name, tuple(param.shape))))
    g = torch.Generator().manual_seed(4048)
    batch, players, tokens, folders = 3, 3, 6, 2
    deck, first, hands = geometry.n_cards, geometry.first_card, geometry.n_hands
    combos = torch.tensor(geometry.combo_cards, dtype=torch.long)
    board = torch.full((batch, 5), -1, dtype=torch.long)
    compat = torch.ones((batch, hands), dtype=torch.bool)
    for b in range(batch):
        shown = [3, 4, 3][b]
        cards = torch.randperm(deck, generator=g)[:shown] + first
        board[b, :shown] = cards
        compat[b] = ~(combos[:, :, None] == cards[None, None, :]).any(-1).any(-1)
    compact_size = int(compat.sum(1).max())
    status = torch.zeros((batch, players), dtype=torch.long)
    status[:, 2] = 1  # seat 2 folded
    to_act = torch.tensor([0, 1, 0])
    history = PackedPublicHistory(
        actor=torch.randint(-1, players, (batch, tokens), generator=g),
        street=torch.randint(0, 4, (batch, tokens), generator=g),
        action=torch.randint(0, 4, (batch, tokens), generator=g),
        amount=torch.rand((batch, tokens), generator=g) * 4,
        pot_before=torch.rand((batch, tokens), generator=g) * 6,
        call_amount=torch.rand((batch, tokens), generator=g),
        current_bet=torch.rand((batch, tokens), generator=g) * 2,
        min_raise_to=torch.rand((batch, tokens), generator=g) * 2,
        max_raise_to=torch.rand((batch, tokens), generator=g) * 8,
        mask=torch.rand((batch, tokens), generator=g) < 0.7,
    )
    history.mask[:, 0] = True
    pub = PokerPublicBatch(
        street=torch.ones(batch, dtype=torch.long), board=board, pot=torch.rand(batch, generator=g) * 3 + 1.5,
        stacks=torch.rand((batch, players), generator=g) * 8, committed=torch.rand((batch, players), generator=g),
        to_act=to_act, legality_summary=torch.rand((batch, 4), generator=g), n_ticks=torch.full((batch,), 16.0),
        raise_grid_bounds=torch.rand((batch, 2), generator=g), status=status,
        seat_mask=torch.ones((batch, players), dtype=torch.bool), button=torch.randint(0, players, (batch,), generator=g),
        committed_street=torch.rand((batch, players), generator=g), call_amount=torch.rand(batch, generator=g),
        current_bet=torch.rand(batch, generator=g), min_raise_to=torch.rand(batch, generator=g),
        max_raise_to=torch.rand(batch, generator=g) * 8, last_full_raise=torch.ones(batch),
        legal_action_mask=torch.rand((batch, 6), generator=g) < 0.8, raise_ticks=torch.rand((batch, 5), generator=g),
        history=history,
    )
    ranges = torch.rand((batch, players, hands), generator=g)
    rank = max(3, cfg.folder_beta_rank)  # the encoder reads folder_beta_rank eigenpairs
    eigvec = torch.randn((batch, deck, rank), generator=g)
    summary = {
        "hand_log_ratio": torch.randn((batch, hands), generator=g) * 0.3,
        "beta_eigenvalue": torch.randn((batch, rank), generator=g),
        "beta_eigenvector": eigvec / eigvec.norm(dim=1, keepdim=True),
        "folder_log_mass": -torch.rand((batch, folders), generator=g),
        "folder_single_card_log_ratio": -torch.rand((batch, folders, deck), generator=g) * 0.5,
        "folder_line_meta": torch.rand((batch, folders, cfg.folder_line_dim), generator=g),
        "folder_mask": torch.tensor([[True, False], [True, True], [True, False]]),
        "folder_seat": torch.full((batch, folders), 2, dtype=torch.long),
        "tight_cluster_scalar": torch.rand(batch, generator=g),
    }
    fold_lines = torch.rand((batch, folders, cfg.folder_line_dim), generator=g)
    masks = PostflopMasks(compatibility=compat, evaluator_summary=summary, fold_line_features=fold_lines,
                          compact_size=compact_size)
    with torch.no_grad():
        result = encoder(shared, pub, ranges, None, masks)
    for name in ("street", "board", "pot", "stacks", "committed", "to_act", "legality_summary", "n_ticks",
                 "raise_grid_bounds", "status", "seat_mask", "button", "committed_street", "call_amount",
                 "current_bet", "min_raise_to", "max_raise_to", "last_full_raise", "legal_action_mask",
                 "raise_ticks"):
        out["pub_" + name] = _np(getattr(pub, name))
    for name in ("actor", "street", "action", "amount", "pot_before", "call_amount", "current_bet",
                 "min_raise_to", "max_raise_to", "mask"):
        out["hist_" + name] = _np(getattr(history, name))
    for name, value in summary.items():
        out["summary_" + name] = _np(value)
    out["combo_ranges"] = _np(ranges)
    out["compatibility"] = _np(compat)
    out["fold_line_features"] = _np(fold_lines)
    out["compact_size"] = np.array(compact_size)
    for name, value in result.raw.items():
        out["raw_" + name] = _np(value)
    out["value"] = _np(result.v)
    spec = []
    for module in (shared, encoder):
        for name, param in module.named_parameters():
            spec.append(name + ":" + ",".join(str(n) for n in param.shape))
    out["param_spec"] = np.array(spec)
    result = encoder(shared, pub, ranges, None, masks)
    _gradient_sketch(out, (shared, encoder), {**result.raw, "value": result.v})


FOLDED_CASES = (
    # (players, stack, ranks, batch, folded seats per row, tight seats per row, board cards per row, line_dim, beta_rank)
    (3, 8.0, 4, 3, ((2,), (1,), (0, 2)), ((2,), (), (0, 2)), (3, 4, 5), 3, 4),
    (4, 8.0, 4, 2, ((1, 2, 3), (0, 2, 3)), ((1, 2, 3), (0, 3)), (3, 5), 0, 16),
    (6, 8.0, 5, 2, ((1, 2, 4, 5), (0, 1, 3)), ((1, 2, 4, 5), (0, 1, 3)), (4, 3), 0, 20),
    (6, 100.0, 13, 1, ((0, 2, 3, 5),), ((0, 2, 3, 5),), (3,), 0, 52),
)


def gen_folded(out):
    """folded.py:235-460 (_folded_statistics_fp32 and its _phi_queries finite-difference queries) on CPU.

    Four geometries (3-, 4- and 6-handed, R4 / R5 / R13) with one to four folded seats, tight-folder
    subsets, flop / turn / river boards, random ranges with zeros, a negative and a non-finite entry;
    the per-query phi and triple terms are recorded from inside the reference call.  The reference's
    one device-type test (folded.py:251) is lifted for this run.
    """

    import torch
    from pbg.games.poker.queued import folded
    from pbg.games.poker.queued.hooks import FOLDED, PAD_CARD, NLHEGeometry, PokerStateMachine

    source = textwrap.dedent(inspect.getsource(folded._folded_statistics_fp32))
    guard = 'board_cards.device.type != "cuda"'
    assert guard in source, "reference folded statistics changed shape"
    namespace: dict = {}
    exec(compile(source.replace(guard, "False"), folded.__file__, "exec"), folded.__dict__, namespace)
    folded._folded_statistics_fp32 = namespace["_folded_statistics_fp32"]
    recorded = []
    original = folded._phi_queries

    def recording(*args, **kwargs):
        result = original(*args, **kwargs)
        recorded.append(result)
        return result

    folded._phi_queries = recording
    g = torch.Generator().manual_seed(5150)
    for index, (players, stack, ranks, batch, folds, tights, shown, line_dim, beta_rank) in enumerate(FOLDED_CASES):
        geometry = NLHEGeometry(players, stack, ranks)
        machine = PokerStateMachine(geometry)
        hands, cards = geometry.private_hands, geometry.deck_cards
        combo = machine.combo_cards(torch.arange(hands, dtype=torch.int32))
        board = torch.full((batch, 5), PAD_CARD, dtype=torch.uint8)
        status = torch.zeros((batch, players), dtype=torch.int8)
        tight = torch.zeros((batch, players), dtype=torch.bool)
        for b in range(batch):
            board[b, : shown[b]] = (torch.randperm(cards, generator=g)[: shown[b]] + geometry.first_card).to(torch.uint8)
            status[b, list(folds[b])] = FOLDED
            tight[b, list(tights[b])] = True
        weights = torch.rand((batch, players, hands), generator=g)
        weights = weights * (torch.rand((batch, players, hands), generator=g) > 0.2)
        weights[0, 0, 3] = -0.5
        weights[0, -1, 5] = float("inf")
        weights[-1, 1, 7] = float("nan")
        line = torch.rand((batch, players, line_dim), generator=g) if line_dim else None
        recorded.clear()
        result = folded.folded_statistics(geometry, board_cards=board, range_weights=weights, status=status,
                                          combo_cards=combo, beta_rank=beta_rank, line_dim=line_dim,
                                          line_metadata=line, tight_mask=tight)
        prefix = f"c{index}_"
        out[prefix + "geometry"] = np.array([players, stack, ranks, beta_rank, line_dim], dtype=np.float64)
        out[prefix + "board_cards"] = _np(board)
        out[prefix + "range_weights"] = _np(weights)
        out[prefix + "status"] = _np(status)
        out[prefix + "tight_mask"] = _np(tight)
        if line is not None:
            out[prefix + "line_metadata"] = _np(line)
        out[prefix + "phi"] = _np(torch.cat([r[0] for r in recorded], 1))
        out[prefix + "triple"] = _np(torch.cat([r[1] for r in recorded], 1))
        for name, value in result.items():
            out[prefix + name] = _np(value)
        if beta_rank == cards:  # the retained-row layout holds the full-rank eigenpairs (hooks.py:1983-1997)
            out[prefix + "packed"] = _np(folded.pack_folded_statistics(geometry, result))
    out["workspace_row_bytes"] = np.array([folded.folded_statistics_workspace_row_bytes(NLHEGeometry(*c[:3]))
                                           for c in FOLDED_CASES] +
                                          [folded.folded_statistics_workspace_row_bytes(NLHEGeometry(6, 128.0, 13))])
    out["family_workspace_row_bytes"] = np.array([folded.sequential_family_workspace_row_bytes(NLHEGeometry(*c[:3]), 4)
                                                  for c in FOLDED_CASES] +
                                                 [folded.sequential_family_workspace_row_bytes(NLHEGeometry(6, 128.0, 13), 4)])
    folded._phi_queries = original


def gen_queued_model(out):
    """queued/model.py:147-452 (QueuedPokerModel: retained model-input rows -> encoders -> outputs) on CPU.

    A 3-handed R4 geometry: player-node states from seeded random-play trajectories, each encoded by
    the reference's own direct_model_input with random log reach (log path probabilities, at most 0)
    and the public history; postflop
    rows with a folded seat carry the reference's packed folded statistics (as hooks.py:1968-2006
    seals them).  The model is the reference QueuedPokerModel with branching heads, weights drawn by
    model_params.parameter from the state_dict names.  Recorded: forward_partition for every
    partition present, and learner_operation on a sampled private state.  Device guards lifted as in
    the encoder runs (state_from_model_input, forward_partition and the folded-statistics board test).
    """

    import inspect
    import textwrap

    import torch
    from pbg.core import tensor_ops
    from pbg.core.rollout import child_path_keys
    from pbg.games.poker.model import primitives
    from pbg.games.poker.model.preflop import PokerModelConfig
    from pbg.games.poker.queued import folded, hooks
    from pbg.games.poker.queued import model as qmodel
    from pbg.games.poker.queued.hooks import FOLDED, NLHEGeometry, PokerHistory, PokerStateMachine

    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    import model_params

    def lift(owner, name, guard, replacement="False", module=None):
        source = textwrap.dedent(inspect.getsource(getattr(owner, name)))
        assert guard in source, f"reference {name} changed shape"
        namespace: dict = {}
        mod = module or inspect.getmodule(owner)
        exec(compile(source.replace(guard, replacement), mod.__file__, "exec"), mod.__dict__, namespace)
        setattr(owner, name, namespace[name])

    tensor_ops._accelerator = lambda value: None
    lift(primitives.MHA, "forward", 'if q.device.type not in ("cuda", "mps"):', "if False:", primitives)
    lift(hooks.PokerStateMachine, "state_from_model_input", 'model_input.device.type not in ("cuda", "mps")', "False",
         hooks)
    lift(qmodel.QueuedPokerModel, "forward_partition", 'model_input.device.type not in ("cuda", "mps")', "False",
         qmodel)
    lift(folded, "_folded_statistics_fp32", 'board_cards.device.type != "cuda"', "False", folded)

    geometry = NLHEGeometry(3, 8.0, 4)
    machine = PokerStateMachine(geometry)
    cfg = PokerModelConfig(**dict(model_params.CONFIG, max_players=3, use_branching_heads=True,
                                  max_history_tokens=geometry.player_node_bound + 3))
    model = qmodel.QueuedPokerModel(geometry, cfg)
    with torch.no_grad():
        for name, param in model.named_parameters():
            param.copy_(torch.from_numpy(model_params.parameter(name, tuple(param.shape))))
    rng = np.random.default_rng(31)
    B, seed, iteration = 48, 77, 5
    state = machine.initial_roots(B, seed=seed, iteration=iteration, retry_epoch=0, device="cpu")
    history = machine.empty_history(B, torch.device("cpu"))
    path = torch.zeros(B, dtype=torch.int64)
    root = torch.arange(B, dtype=torch.int64)
    snaps = []
    for step in range(40):
        active = ~state.terminal
        if not bool(active.any()):
            break
        rows = torch.nonzero(active).flatten()
        sub = hooks.PokerState(*(getattr(state, n)[rows] for n in STATE_FIELDS))
        sub_hist = PokerHistory(*(getattr(history, n)[rows] for n in HISTORY_FIELDS))
        snaps.append((sub, sub_hist))
        mask = machine.legality(sub).mask
        chosen = []
        for i in range(rows.numel()):
            legal = torch.nonzero(mask[i]).flatten().numpy()
            u = rng.random()
            if u < 0.2 and mask[i, 0]:
                chosen.append(0)
            elif u < 0.6:
                chosen.append(1)
            else:
                raises = legal[legal >= 2]
                chosen.append(int(rng.choice(raises)) if raises.size else 1)
        action = torch.tensor(chosen, dtype=torch.int32)
        sub_hist = machine.append_player_history(sub, action, sub_hist)
        nxt = machine.step_player(sub, action)
        for generation in range(3):
            chance = machine.needs_chance(nxt)
            sub_hist = machine.append_chance_history(nxt, chance, sub_hist)
            nxt = machine.deal_next_street_keyed(nxt, seed=seed, iteration=iteration, root=root[rows],
                                                 path=path[rows], draw=generation, retry_epoch=0, lane=0)
        for n in STATE_FIELDS:
            getattr(state, n)[rows] = getattr(nxt, n)
        for n in HISTORY_FIELDS:
            getattr(history, n)[rows] = getattr(sub_hist, n)
        path[rows] = child_path_keys(path[rows], 1)
    groups: dict = {}
    for sub, sub_hist in snaps:
        for i in range(sub.rows):
            if bool(sub.terminal[i]):
                continue
            street = int(sub.street[i])
            live = int((sub.status[i] != FOLDED).sum())
            kind = "pre" if street == 0 else f"post_{live}"
            groups.setdefault(kind, []).append((sub, sub_hist, i))
    out["partitions"] = np.array(sorted(groups))
    learner_outputs: dict = {}
    for kind, items in sorted(groups.items()):
        items = items[:: max(1, len(items) // 12)][:12]
        st = hooks.PokerState(*(torch.stack([getattr(s, n)[i] for s, _, i in items]) for n in STATE_FIELDS))
        hi = PokerHistory(*(torch.stack([getattr(h, n)[i] for _, h, i in items]) for n in HISTORY_FIELDS))
        n, P, H = st.rows, geometry.players, geometry.private_hands
        # log reach as the rollout carries it: log of path probabilities (at most 0), some rows unreachable
        reach = torch.from_numpy(np.log(rng.random((n, P, H)).astype(np.float32) ** 2))
        reach[torch.from_numpy(rng.random((n, P, H)) < 0.15)] = -torch.inf
        rows_in = machine.direct_model_input(kind, st, reach, hi)
        if kind != "pre" and bool((st.status == FOLDED).any()):
            summary = folded.folded_statistics(
                geometry, board_cards=st.board_cards,
                range_weights=torch.exp(reach).masked_fill(~torch.isfinite(reach), 0.0), status=st.status,
                combo_cards=machine.combo_cards(torch.arange(H, dtype=torch.int32)), beta_rank=geometry.deck_cards,
                line_dim=0, tight_mask=hooks.SequentialPokerHooks._tight_folder_mask(
                    type("G", (), {"geometry": geometry})(), hi, st.status))
            rows_in[:, geometry.postflop_base_model_input_width:] = folded.pack_folded_statistics(geometry, summary)
        combos = machine.combo_cards(torch.arange(H, dtype=torch.int32)).to(torch.int64)
        board = st.board_cards.to(torch.int64)
        clash = ((combos[None, :, :, None] == board[:, None, None, :]) & (board != 255)[:, None, None, :]).any(-1).any(-1)
        private = torch.stack([torch.from_numpy(rng.choice(np.nonzero(~clash[r].numpy())[0], P, replace=False))
                               for r in range(n)]).to(torch.int32)
        owner = st.to_act.to(torch.int64)
        with torch.no_grad():
            full = model.forward_partition(kind, rows_in)
            learner = model.learner_operation(kind, rows_in, private, owner)
        tag = "q_" + kind
        out[tag + "_model_input"] = _np(rows_in)
        out[tag + "_private"] = _np(private)
        for name, value in full.policy_raw.items():
            out[tag + "_raw_" + name] = _np(value)
        out[tag + "_value"] = _np(full.value)
        for name, value in full.public_heads.items():
            out[tag + "_head_" + name] = _np(value)
        for name, value in learner.policy_raw.items():
            out[tag + "_lraw_" + name] = _np(value)
        out[tag + "_lvalue"] = _np(learner.value)
        learner = model.learner_operation(kind, rows_in, private, owner)  # with autograd, for the sketch
        learner_outputs.update({f"{kind}__{name}": value for name, value in learner.policy_raw.items()})
        learner_outputs[f"{kind}__value"] = learner.value
    # one seeded loss over the learner rows of every partition: the shared parameters collect the
    # gradient of both networks
    _gradient_sketch(out, (model,), learner_outputs)
    spec = [name + ":" + ",".join(str(x) for x in param.shape) for name, param in model.named_parameters()]
    out["param_spec"] = np.array(spec)
    out["config"] = np.array([cfg.max_history_tokens, cfg.max_players])


def _poker_masks(gi, E):
    with np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "poker.npz")) as data:
        packed = data[f"g{gi}_masks"]
    masks = np.unpackbits(packed, axis=-1)[..., :E].astype(bool).reshape(-1, E)
    return masks[masks.any(1)]


# (name, mask source, E, M, sigma rows, columns (1 = sampled, H = Rao-Blackwell), lanes, branched, reference raw)
POKER_LOSS_CASES = (
    ("s202", 3, 202, 2, 32, 1, 2, False, True),
    ("s10", None, 10, 3, 16, 1, 1, False, False),
    ("rb18", 0, 18, 2, 6, 120, 2, False, True),
    ("br102", 5, 102, 2, 10, 1, 2, True, True),
    ("brrb18", 0, 18, 2, 4, 120, 1, True, False),
)


def gen_poker_loss(out):
    """The poker learner objective and its gradient from the reference's own loss program.

    ``LearnerOperation.forward_loss`` (pbg/core/learner.py:1824-2159) with the
    reference's composite policy (``PokerPolicyOperator.learner``,
    pbg/games/poker/queued/policy.py:284-298) as the policy operation, given a
    model evaluation whose raw fields, value and public heads are leaf tensors;
    ``(total * lane_weight).sum().backward()`` (pbg/core/training.py:403 with
    the objective weight times the loss scale per lane) gives the gradients.
    Cases cover sampled and Rao-Blackwell private estimators, sequential and
    branched (ragged action spans with trace/cost heads) batches, one and two
    lanes with different controls, the clipped and MSE value objectives, the
    negative-advantage log cap, the reference-KL term, and one row whose
    mixture has no fp32 mass on its legal ticks (the uniform fallback).
    """

    import torch
    from pbg.core.contracts import mode_schema
    from pbg.core.learner import (BranchedLearnerBatch, BranchingLossConfig, LearnerOperation, LossConfig,
                                  ModelEvaluation, SequentialLearnerBatch)
    from pbg.games.poker.queued.policy import PokerLegality, PokerPolicyOperator

    BranchedLearnerBatch.__post_init__ = lambda self: None  # learner.py:1127-1150 without the device test
    rng = np.random.default_rng(2024)
    op = PokerPolicyOperator()
    out["cases"] = np.array([c[0] for c in POKER_LOSS_CASES])
    for name, gi, E, M, S, W, lanes, branched, with_ref in POKER_LOSS_CASES:
        if gi is None:
            mask = rng.random((S, E)) < 0.6
            mask[:, 1] = True
            mask[1] = False
            mask[1, 1] = True
        else:
            pool = _poker_masks(gi, E)
            mask = pool[rng.choice(pool.shape[0], S, replace=pool.shape[0] < S)]
        g = torch.Generator().manual_seed(int(rng.integers(0, 2**31)))
        raw = _raw(rng, S, W, M)
        if gi is None:
            # every component far below the legal ticks with a narrow scale: the tick products
            # underflow to zero in fp32, so the raise law is the uniform fallback
            raw["mu"][2] = 0.0
            raw["s"][2] = 0.005
            mask[2] = False
            mask[2, [1, E - 2, E - 1]] = True
        ref_raw = None
        if with_ref:
            ref_raw = {k: v.clone() for k, v in raw.items()}
            ref_raw["type_logits"] = ref_raw["type_logits"] + 0.3 * torch.randn(S, W, 3, generator=g)
            ref_raw["mu"] = (ref_raw["mu"] + 0.1 * torch.randn(S, W, M, generator=g)).clamp(0.0, 1.0)
            ref_raw["iota"] = (ref_raw["iota"] * 0.8).clamp(0.0, 1.0)
        counts = rng.integers(1, 4, S) if branched else np.ones(S, np.int64)
        if branched and lanes > 1:
            # equal action rows per lane
            half = S // lanes
            counts[half:] = counts[:half][::-1]
        A_rows = int(counts.sum())
        ptr = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
        a2s = np.repeat(np.arange(S), counts)
        action = np.array([rng.choice(np.nonzero(mask[s])[0]) for s in a2s], dtype=np.int32)
        legality_sigma = PokerLegality(torch.arange(E, dtype=torch.int32)[None].expand(S, -1).contiguous(),
                                       torch.from_numpy(mask))
        with torch.no_grad():
            p = op.probabilities(raw, legality_sigma)  # [S, W, E]
            cur = torch.log(p[torch.from_numpy(a2s), :, torch.from_numpy(action).long()].clamp_min(1e-12))
        old = (cur + 0.3 * torch.randn(A_rows, W, generator=g)).float()
        far = rng.random(A_rows) < 0.3
        old[torch.from_numpy(far)] += 1.5 * torch.randn(int(far.sum()), W, generator=g)
        adv = torch.randn(A_rows, W, generator=g)
        if W > 1:
            post = torch.rand(A_rows, W, generator=g) * (torch.rand(A_rows, W, generator=g) > 0.3)
        else:
            post = torch.ones(A_rows, 1)
        value = torch.randn(S, W, generator=g)
        old_value = value + 0.3 * torch.randn(S, W, generator=g)
        target = torch.randn(S, W, generator=g)
        controls = torch.tensor([
            [0.2, math.log(1.5), 0.5, 0.2, 0.01, 0.05 if with_ref else 0.0, 0.3 if branched else 0.0,
             0.2 if branched else 0.0, 1.0e-8 if not branched else 1.0e-3, 1.0],
            [0.25, math.inf, 0.7, 0.0, 0.02, 0.1 if with_ref else 0.0, 0.1 if branched else 0.0,
             0.4 if branched else 0.0, 1.0e-8 if not branched else 1.0e-2, 0.0],
        ], dtype=torch.float32)[:lanes]
        lane_weight = torch.tensor([1.6, 0.5], dtype=torch.float32)[:lanes]

        leaves = {k: v.detach().clone().requires_grad_() for k, v in raw.items()}
        value_leaf = value.detach().clone().requires_grad_()
        heads = {}
        sigma = {"model_input": torch.arange(S, dtype=torch.float32)[:, None],
                 "owner": torch.zeros(S, dtype=torch.int32), "old_value": old_value, "value_target": target}
        if W == 1:
            sigma["sampled_private_state"] = torch.zeros(S, 2, dtype=torch.int32)
        if branched:
            sigma["target_degree"] = torch.from_numpy(counts.astype(np.int32))
            trace_pred = (torch.rand(S, generator=g) * 2 + 0.05).requires_grad_()
            cost_pred = (torch.rand(S, generator=g) * 2 + 0.05).requires_grad_()
            heads = {"trace": trace_pred, "cost": cost_pred}
            sigma["trace_target"] = torch.rand(S, generator=g) * 2
            sigma["cost_target"] = torch.rand(S, generator=g) * 2 + 0.01
        action_fields = {"action": torch.from_numpy(action), "old_log_policy": old, "advantage_target": adv,
                         "posterior": post}
        if branched:
            batch = BranchedLearnerBatch("post", torch.arange(S), torch.from_numpy(ptr), torch.arange(A_rows),
                                         MappingProxyType(sigma), MappingProxyType(action_fields))
        else:
            fields = dict(sigma)
            fields.update(action_fields)
            batch = SequentialLearnerBatch("post", torch.arange(S), MappingProxyType(fields))

        def policy(input_type, model_input, raw_rows, act, private, owner, reference):
            rows = model_input[:, 0].long()
            legality = PokerLegality(torch.arange(E, dtype=torch.int32)[None].expand(rows.numel(), -1).contiguous(),
                                     torch.from_numpy(mask)[rows])
            return op.learner(raw_rows, legality, act, private, owner, reference)

        cfg = LossConfig(branching=BranchingLossConfig(0.3, 0.2, 1.0e-3) if branched else None)
        estimator = "sampled" if W == 1 else "rao_blackwell"
        rollout = "branched.fixed" if branched else "sequential"
        learner = LearnerOperation(mode_schema("self_play", rollout, estimator), cfg, None, policy)
        evaluation = ModelEvaluation(leaves, value_leaf, MappingProxyType(heads))
        res = learner.forward_loss(batch, iteration=0, lane_count=lanes, loss_controls=controls,
                                   evaluation=evaluation, reference_raw=ref_raw)
        (res.total * lane_weight).sum().backward()
        pre = f"pl_{name}_"
        for k, v in raw.items():
            out[pre + k] = _np(v)
            out[pre + "grad_" + k] = _np(leaves[k].grad)
            if ref_raw is not None:
                out[pre + "ref_" + k] = _np(ref_raw[k])
        out[pre + "mask"] = mask.astype(np.uint8)
        out[pre + "action_ptr"] = ptr
        out[pre + "action"] = action
        out[pre + "old"] = _np(old)
        out[pre + "adv"] = _np(adv)
        out[pre + "post"] = _np(post)
        out[pre + "value"] = _np(value)
        out[pre + "old_value"] = _np(old_value)
        out[pre + "target"] = _np(target)
        out[pre + "grad_value"] = _np(value_leaf.grad)
        out[pre + "controls"] = _np(controls)
        out[pre + "lane_weight"] = _np(lane_weight)
        out[pre + "meta"] = np.array([E, M, S, W, lanes, A_rows, int(branched), int(with_ref)], np.int64)
        if branched:
            for k in ("trace_target", "cost_target"):
                out[pre + k] = _np(sigma[k])
            out[pre + "trace_pred"] = _np(trace_pred)
            out[pre + "cost_pred"] = _np(cost_pred)
            out[pre + "grad_trace_pred"] = _np(trace_pred.grad)
            out[pre + "grad_cost_pred"] = _np(cost_pred.grad)
        out[pre + "result"] = np.stack([_np(getattr(res, f)) for f in res.__dataclass_fields__], 1)

    # PokerPolicyOperator.learner itself (policy.py:284-298) with autograd: selected log pi, entropy and
    # reference KL of [B, rows] policy rows and the raw-field gradients of a weighted sum of the three.
    for name, gi, E, M, B, rows in (("pl202", 3, 202, 2, 12, 3), ("pl18", 0, 18, 3, 10, 5)):
        pool = _poker_masks(gi, E)
        mask = pool[rng.choice(pool.shape[0], B, replace=False)]
        raw = _raw(rng, B, rows, M)
        ref_raw = {k: v.clone() for k, v in raw.items()}
        ref_raw["type_logits"] = ref_raw["type_logits"] + 0.5
        ref_raw["mu"] = (ref_raw["mu"] * 0.7).clamp(0.0, 1.0)
        leaves = {k: v.detach().clone().requires_grad_() for k, v in raw.items()}
        action = np.array([rng.choice(np.nonzero(m)[0]) for m in mask], dtype=np.int32)
        legality = PokerLegality(torch.arange(E, dtype=torch.int32)[None].expand(B, -1).contiguous(),
                                 torch.from_numpy(mask))
        ev = op.learner(leaves, legality, torch.from_numpy(action), None, None, ref_raw)
        weights = [torch.randn(B, rows, generator=torch.Generator().manual_seed(7 + i)) for i in range(3)]
        (ev.selected_log_policy * weights[0] + ev.entropy * weights[1] + ev.reference_kl * weights[2]).sum().backward()
        pre = f"plr_{name}_"
        out[pre + "mask"] = mask.astype(np.uint8)
        out[pre + "action"] = action
        for k in raw:
            out[pre + k] = _np(raw[k])
            out[pre + "ref_" + k] = _np(ref_raw[k])
            out[pre + "grad_" + k] = _np(leaves[k].grad)
        out[pre + "selected"] = _np(ev.selected_log_policy)
        out[pre + "entropy"] = _np(ev.entropy)
        out[pre + "kl"] = _np(ev.reference_kl)
        out[pre + "weights"] = np.stack([_np(w) for w in weights])


# the cfg2 architecture (d 128, 2 layers, 4 heads, M = 2, class embedding 32, FFN 512)
# and the reference's default network (PokerModelConfig defaults: d 256, 8 heads, 6 layers), at 13 ranks
CFG2_MODEL = dict(d_model=128, n_heads=4, layers=2, m_raise=2, k_act=5, max_players=2, class_embedding_dim=32,
                  ffn_hidden=512, max_history_tokens=110, folder_beta_rank=16)
DEFAULT_MODEL = dict(max_players=2)


def gen_preflop_model_r13(out):
    gen_preflop_model(out, CFG2_MODEL, 13, batch=2, tokens=16)


def gen_preflop_model_default(out):
    gen_preflop_model(out, DEFAULT_MODEL, 13, batch=2, tokens=16)


def gen_postflop_model_r13(out):
    gen_postflop_model(out, dict(CFG2_MODEL, max_players=3), 13)


def gen_postflop_model_default(out):
    gen_postflop_model(out, dict(DEFAULT_MODEL, max_players=3), 13)


GENERATORS = {"posterior": gen_posterior, "preflop_model": gen_preflop_model, "postflop_model": gen_postflop_model,
              "folded": gen_folded, "queued_model": gen_queued_model, "poker_loss": gen_poker_loss,
              "preflop_model_r13": gen_preflop_model_r13, "preflop_model_default": gen_preflop_model_default,
              "postflop_model_r13": gen_postflop_model_r13, "postflop_model_default": gen_postflop_model_default}


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, help="root of a pbg checkout")
    parser.add_argument("--out", default=os.path.dirname(os.path.abspath(__file__)))
    parser.add_argument("--only", default=None, help="comma-separated fixture names to (re)generate")
    args = parser.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))
    sys.path.insert(0, os.path.join(os.path.abspath(args.reference), "tests"))
    import torch
    torch.manual_seed(0)
    _install_shims()
    only = set(args.only.split(",")) if args.only else None
    if only is not None and only <= set(GENERATORS):
        outputs = []
        for name in sorted(only):
            data: dict = {}
            GENERATORS[name](data)
            outputs.append((name, data))
    else:
        rng_out, poker_out, policy_out, loss_out, adam_out, ka_out = {}, {}, {}, {}, {}, {}
        gen_rng(rng_out)
        gen_poker(poker_out)
        gen_known_answers(ka_out)
        gen_policy(policy_out, poker_out)
        gen_loss(loss_out)
        gen_adam(adam_out)
        mi_out, post_out = {}, {}
        gen_model_input(mi_out, poker_out)
        gen_posterior(post_out)
        outputs = (("rng", rng_out), ("poker", poker_out), ("known_answers", ka_out), ("policy", policy_out),
                   ("loss", loss_out), ("adam", adam_out), ("model_input", mi_out), ("posterior", post_out))
        if only is not None:
            outputs = tuple(item for item in outputs if item[0] in only)
    for name, data in outputs:
        np.savez_compressed(os.path.join(args.out, f"{name}.npz"), **data)
        print(name, len(data), os.path.getsize(os.path.join(args.out, f"{name}.npz")))


if __name__ == "__main__":
    main()
