"""QueuedPokerModel (the model entry point of the rollout and the learner) against the reference.

tests/golden/queued_model.npz holds the reference QueuedPokerModel's own outputs (run on CPU by
tests/golden/make_golden.py) for retained model-input rows of a 3-handed R4 geometry, written by the
reference's direct_model_input from seeded random-play states with random log reach and the public
history (postflop rows with a folded seat carry the reference's packed folded statistics), for the
preflop partition and the postflop partitions with two and three live seats; the learner rows pick
a sampled private hand of the acting seat.  Weights: tests/golden/model_params.py by state_dict name
(shared.*, pre_encoder.*, post_encoder.*, with the public branching heads).  This build decodes the
rows, builds the encoder inputs and runs the bf16 tensor-core networks: rtol/atol 2e-2 on every
policy field, value and the trace head, and on the logit of the cost head (an exponential).
"""

import os
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))


def _model(d):
    import model_params
    from pbg_b200.poker import NLHEGeometry
    from pbg_b200.preflop import PreflopConfig
    from pbg_b200.queued_model import QueuedPokerModel

    params = {}
    for item in d["param_spec"]:
        name, dims = str(item).split(":")
        params[name] = torch.from_numpy(model_params.parameter(name, tuple(int(x) for x in dims.split(","))))
    history, players = (int(x) for x in d["config"])
    cfg = PreflopConfig(**dict(model_params.CONFIG, max_players=players, max_history_tokens=history))
    return QueuedPokerModel(NLHEGeometry(3, 8.0, 4), cfg, params, DEV)


@pytest.mark.parametrize("kind", ["pre", "post_2", "post_3"])
def test_queued_model_matches_reference(gold, kind):
    from pbg_b200.checks import input_errors

    d = gold("queued_model")
    assert kind in [str(x) for x in d["partitions"]]
    model = _model(d)
    tag = "q_" + kind
    rows = torch.from_numpy(d[tag + "_model_input"]).to(DEV)
    result = model.forward_partition(kind, rows)
    torch.cuda.synchronize()
    assert input_errors(DEV) == []
    worst = {}
    for name, value in result.policy_raw.items():
        want = torch.from_numpy(d[tag + "_raw_" + name])
        worst[name] = float((value.cpu() - want).abs().max())
        torch.testing.assert_close(value.cpu(), want, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(result.value.cpu(), torch.from_numpy(d[tag + "_value"]), rtol=2e-2, atol=2e-2)
    heads = result.public_heads
    torch.testing.assert_close(heads["trace"].cpu(), torch.from_numpy(d[tag + "_head_trace"]), rtol=2e-2, atol=2e-2)
    # the cost head is exp(logit): the bf16 bar applies to its logit
    torch.testing.assert_close(heads["cost"].log().cpu(), torch.from_numpy(d[tag + "_head_cost"]).log(),
                               rtol=2e-2, atol=2e-2)
    print(f"\n{kind}: max |b200 - reference| {worst}")


@pytest.mark.parametrize("kind", ["pre", "post_2", "post_3"])
def test_queued_learner_operation_matches_reference(gold, kind):
    d = gold("queued_model")
    model = _model(d)
    tag = "q_" + kind
    rows = torch.from_numpy(d[tag + "_model_input"]).to(DEV)
    private = torch.from_numpy(d[tag + "_private"]).to(DEV)
    owner = model._state(kind, rows).to_act.to(torch.int64)
    result = model.learner_operation(kind, rows, private, owner)
    for name, value in result.policy_raw.items():
        torch.testing.assert_close(value.cpu(), torch.from_numpy(d[tag + "_lraw_" + name]), rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(result.value.cpu(), torch.from_numpy(d[tag + "_lvalue"]), rtol=2e-2, atol=2e-2)


def test_state_round_trips_through_the_retained_row(gold):
    # hooks.py:531-612 then 812-881: the state machine's own encoding decodes to the same public state
    from pbg_b200.poker import NLHEGeometry, PokerStateMachine, STATE_FIELDS

    geometry = NLHEGeometry(3, 8.0, 4)
    machine = PokerStateMachine(geometry)
    state = machine.initial_roots(16, seed=3, iteration=1, retry_epoch=0, device=DEV)
    for kind in ("pre", "post_3"):
        rows = machine.direct_model_input(kind, state)
        back = machine.state_from_model_input(kind, rows, state.combo_ids)
        for name in STATE_FIELDS:
            if name != "terminal":
                assert torch.equal(getattr(back, name), getattr(state, name)), (kind, name)
