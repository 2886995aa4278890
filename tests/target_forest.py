"""Seeded topology forests in the layer-plan format of pbg/core/targets.py:244-282.

Test helper: builds node/child columns, per-partition arenas and the
conversion table for the layered-target kernel and its CPU restatement.
Two output partitions (widths 3 and 5) with a class-sum conversion 1 -> 0,
two input partitions bound to outputs 0 and 1.

``reuse=True`` double-buffers work rows the way the reference's layer plan
does (layer l writes arena (l+1)&1 at rows numbered from 0 within the layer,
children come from the layer just below), so a layer overwrites rows that
the layer two below wrote; ``reuse=False`` gives every node its own row.
"""

from __future__ import annotations

import numpy as np

WIDTHS = (3, 5)
CONVERT_1_TO_0 = (0, 0, 1, 2, 2)
INPUT_OUTPUT = (0, 1)


def conversion() -> np.ndarray:
    n, w = len(WIDTHS), max(WIDTHS)
    table = np.full((n, n, w), -1, dtype=np.int32)
    for s in range(n):
        table[s, s, : WIDTHS[s]] = np.arange(WIDTHS[s])
    table[1, 0, : WIDTHS[1]] = CONVERT_1_TO_0
    return table


def _compatible(child_type: int, parent_type: int) -> bool:
    return child_type == parent_type or (child_type == 1 and parent_type == 0)


class PlanRuns:
    """Runs a plan (columns + arenas) through the oracle or the CUDA library."""

    # ------------------------------------------------------------------ runs
    def copy_arenas(self) -> dict:
        return {k: (None if v is None else [None if a is None else a.copy() for a in v]) for k, v in self.arenas.items()}

    def kwargs(self) -> dict:
        return dict(n_replica=self.n_replica, input_count=self.input_count, output_count=self.output_count,
                    action_partitions=self.action_partitions, p_train=self.p_train, lam=self.lam,
                    sampled=self.sampled, branched=self.branched)

    def run_oracle(self, oracle_module, arenas: dict | None = None):
        arenas = self.copy_arenas() if arenas is None else arenas
        failure = oracle_module.layered_targets(self.layer_ptr, self.nodes, self.children, arenas, self.conversion,
                                                self.work_cap, self.head_cap, self.width, **self.kwargs())
        return failure, arenas

    def device_args(self, device, arenas: dict | None = None):
        """Positional arguments of run_layers (both the reference's and pbg_b200's) and the arena tensors."""

        import torch

        arenas = self.copy_arenas() if arenas is None else arenas
        n_in, n_out = self.input_count, self.output_count
        empty = torch.empty(0, dtype=torch.float32, device=device)

        def dev(group, count):
            if group is None:
                return [empty] * count
            return [empty if a is None else torch.from_numpy(a).to(device) for a in group]

        groups = {}
        for name, count in (("work0", n_out), ("work1", n_out), ("trace", n_out), ("cost", n_out), ("delta", n_out),
                            ("head_v", n_in), ("head_t", n_in), ("head_c", n_in),
                            ("sigma_v", self.n_replica * n_in), ("sigma_t", self.n_replica * n_in),
                            ("sigma_c", self.n_replica * n_in),
                            ("action_p", self.n_replica * self.action_partitions),
                            ("action_a", self.n_replica * self.action_partitions)):
            groups[name] = dev(arenas[name], count)
        nodes = [torch.from_numpy(a).to(device) for a in self.nodes]
        children = [torch.from_numpy(a).to(device) for a in self.children]
        args = (torch.from_numpy(self.layer_ptr), nodes, children, groups["work0"], groups["work1"],
                groups["trace"], groups["cost"], groups["delta"], groups["head_v"], groups["head_t"],
                groups["head_c"], groups["sigma_v"], groups["sigma_t"], groups["sigma_c"],
                groups["action_p"], groups["action_a"], torch.from_numpy(self.conversion).flatten().to(device),
                list(self.work_cap), list(self.head_cap), list(self.width), self.n_replica, n_in, n_out,
                self.action_partitions, self.p_train, max(self.width), self.lam, self.sampled, self.branched)
        return args, groups, arenas

    def run_device(self, device, arenas: dict | None = None, runner=None):
        """Run through ``runner`` (default: pbg_b200.targets.run_layers); returns failure, arenas (numpy)."""

        import torch

        if runner is None:
            from pbg_b200.targets import run_layers as runner
        args, groups, arenas = self.device_args(device, arenas)
        failure = runner(*args)
        torch.cuda.synchronize(device)
        out = {}
        for name, group in groups.items():
            if arenas[name] is None:
                out[name] = None
            else:
                out[name] = [None if a is None else t.cpu().numpy() for a, t in zip(arenas[name], group)]
        return failure.cpu().numpy(), out


class Forest(PlanRuns):
    """Plan columns + arenas (numpy, float32/int32) for one seeded forest."""

    def __init__(self, seed: int, *, n_replica: int = 3, p_train: int = 2, sampled: bool = True,
                 branched: bool = False, layers: int = 4, width_per_layer: int = 12, reuse: bool = False,
                 lam: float = 0.5, extra_edges: bool = True) -> None:
        rng = np.random.default_rng(seed)
        self.n_replica, self.p_train, self.sampled, self.branched, self.lam = n_replica, p_train, sampled, branched, lam
        self.input_count, self.output_count = len(INPUT_OUTPUT), len(WIDTHS)
        self.action_partitions = self.output_count if branched else self.input_count
        nodes = []  # dicts
        edges = []  # (source_row, source_type, path, multiplier)
        leaves = []  # (lane, type, row, arena)
        row_next = np.zeros((n_replica, 2, 2), dtype=np.int64)  # per lane, output, arena (unique mode)
        sigma_next = np.zeros((n_replica, self.input_count), dtype=np.int64)
        action_next = np.zeros((n_replica, self.action_partitions), dtype=np.int64)
        head_rows = 7
        layer_nodes: list[list[dict]] = []

        def new_row(lane, t, arena, within):
            if reuse:
                r = within[(lane, t, arena)]
                within[(lane, t, arena)] += 1
                return r
            r = row_next[lane, t, arena]
            row_next[lane, t, arena] += 1
            return int(r)

        pending: list[list[tuple[int, int, int]]] = [[] for _ in range(n_replica)]  # (type, row, arena)
        for layer in range(layers):
            arena = (layer + 1) & 1
            within = {(l, t, a): 0 for l in range(n_replica) for t in range(2) for a in range(2)}
            current = []
            for lane in range(n_replica):
                kids = pending[lane]
                rng.shuffle(kids)
                groups: list[list[tuple[int, int, int]]] = []
                if layer == 0:
                    groups = [[] for _ in range(int(rng.integers(1, width_per_layer + 1)))]
                else:
                    if not kids:
                        continue
                    i = 0
                    while i < len(kids):
                        take = int(rng.integers(1, 4))
                        groups.append(kids[i: i + take])
                        i += take
                next_pending = []
                for group in groups:
                    ptype = 0 if any(k[0] == 0 for k in group) else int(rng.integers(0, 2))
                    if not all(_compatible(k[0], ptype) for k in group):
                        ptype = 0
                    children = list(group)
                    n_leaf = int(rng.integers(1, 4)) if layer == 0 else (int(rng.integers(0, 2)) if not reuse else 0)
                    for _ in range(n_leaf):
                        lt = ptype if ptype == 1 else int(rng.integers(0, 2))
                        la = 0 if reuse else int(rng.integers(0, 2))
                        if reuse:  # layer-0 leaves sit above every node row of arena 0
                            lr = 1000 + sum(1 for x in leaves if x[0] == lane and x[1] == lt)
                        else:
                            lr = new_row(lane, lt, la, within)
                        leaves.append((lane, lt, lr, la))
                        children.append((lt, lr, la))
                    if not children:
                        continue
                    order = rng.permutation(len(children))
                    children = [children[i] for i in order]
                    trained = rng.random() < 0.8
                    input_type = INPUT_OUTPUT.index(ptype) if trained else -1
                    owner = int(rng.integers(-1, p_train)) if trained else -1
                    ntgt = len(children)
                    dest = new_row(lane, ptype, arena, within)
                    node = dict(replica=lane, layer=layer, output_type=ptype, input_type=input_type, owner_slot=owner,
                                target_degree=ntgt, nominal_degree=ntgt + int(rng.integers(0, 3)),
                                destination_row=dest, sigma_head_row=int(rng.integers(0, head_rows)), children=children,
                                extra=int(rng.integers(0, 2)) if extra_edges else 0)
                    if input_type >= 0:
                        node["sigma_target_row"] = int(sigma_next[lane, input_type])
                        sigma_next[lane, input_type] += 1
                        part = ptype if branched else input_type
                        node["action_begin"] = int(action_next[lane, part])
                        action_next[lane, part] += ntgt
                    else:
                        node["sigma_target_row"] = 0
                        node["action_begin"] = 0
                    current.append(node)
                    next_pending.append((ptype, dest, arena))
                pending[lane] = next_pending
            perm = rng.permutation(len(current))
            layer_nodes.append([current[i] for i in perm])

        flat = [n for layer in layer_nodes for n in layer]
        self.layer_ptr = np.cumsum([0] + [len(layer) for layer in layer_nodes]).astype(np.int32)
        cols = {k: [] for k in ("replica", "child_begin", "child_count", "destination_row", "input_type",
                                "output_type", "owner_slot", "nominal_degree", "target_degree", "sigma_head_row",
                                "sigma_target_row", "action_begin")}
        for n in flat:
            cols["child_begin"].append(len(edges))
            for (t, r, a) in n["children"]:
                edges.append((r if a == 0 else -r - 1, t, int(rng.integers(0, 4)), float(rng.uniform(0.0, 1.5))))
            for _ in range(n["extra"]):  # edges past target_degree are never read
                edges.append((-(10 ** 6), 0, 0, float("nan")))
            cols["child_count"].append(len(n["children"]) + n["extra"])
            for k in cols:
                if k not in ("child_begin", "child_count"):
                    cols[k].append(n[k])
        self.nodes = [np.asarray(cols[k], dtype=np.int32) for k in cols]
        self.children = [np.asarray([x[0] for x in edges], dtype=np.int32),
                         np.asarray([x[1] for x in edges], dtype=np.int32),
                         np.asarray([x[2] for x in edges], dtype=np.int32),
                         np.asarray([x[3] for x in edges], dtype=np.float32)]

        max_row = 0
        for n in flat:
            max_row = max(max_row, n["destination_row"])
        for (_, _, r, _) in leaves:
            max_row = max(max_row, r)
        self.work_cap = [int(max_row + 1)] * self.output_count
        self.head_cap = [head_rows] * self.input_count
        self.width = list(WIDTHS)
        self.conversion = conversion()

        def arr(shape, lo=-2.0, hi=2.0):
            return rng.uniform(lo, hi, size=shape).astype(np.float32)

        P, R, cap = p_train, n_replica, self.work_cap[0]
        work0 = [arr((R, cap, 2, P, w)) for w in WIDTHS]
        work1 = [arr((R, cap, 2, P, w)) for w in WIDTHS] if not sampled else None
        # leaves: RB mass >= 0 (some exact zeros with zero moment), moment = mass * value
        for (lane, t, r, a) in leaves:
            if not sampled:
                m = rng.uniform(0.0, 2.0, size=(P, WIDTHS[t])).astype(np.float32)
                m[rng.random(m.shape) < 0.15] = 0.0
                work0[t][lane, r, a] = m
                work1[t][lane, r, a] = (m * rng.uniform(-3, 3, size=m.shape)).astype(np.float32)
        self.leaves = leaves
        self.arenas = {
            "work0": work0,
            "work1": work1,
            "trace": [arr((R, cap, 2, P)) for _ in WIDTHS] if branched else None,
            "cost": [arr((R, cap, 2), 0.0, 3.0) for _ in WIDTHS] if branched else None,
            "delta": [arr((R, cap, 2), -0.5, 0.5) for _ in WIDTHS] if branched else None,
            "head_v": [arr((R, head_rows, WIDTHS[INPUT_OUTPUT[i]])) for i in range(self.input_count)],
            "head_t": [arr((R, head_rows), 0.0, 2.0) for _ in range(self.input_count)] if branched else None,
            "head_c": [arr((R, head_rows), 0.0, 2.0) for _ in range(self.input_count)] if branched else None,
        }
        sv, st, sc = [], [], []
        for lane in range(R):
            for i in range(self.input_count):
                rows = max(int(sigma_next[lane, i]), 1)
                sv.append(np.full((rows, WIDTHS[INPUT_OUTPUT[i]]), np.nan, dtype=np.float32))
                st.append(np.full((rows,), np.nan, dtype=np.float32) if branched else None)
                sc.append(np.full((rows,), np.nan, dtype=np.float32) if branched else None)
        ap, aa = [], []
        for lane in range(R):
            for part in range(self.action_partitions):
                out = part if branched else INPUT_OUTPUT[part]
                rows = max(int(action_next[lane, part]), 1)
                ap.append(np.full((rows, WIDTHS[out]), np.nan, dtype=np.float32) if not sampled else None)
                aa.append(np.full((rows, WIDTHS[out]), np.nan, dtype=np.float32))
        self.arenas.update(sigma_v=sv, sigma_t=st if branched else None, sigma_c=sc if branched else None,
                           action_p=ap if not sampled else None, action_a=aa)



class HandPlan(PlanRuns):
    """An explicit small plan with one output and one input partition (width w).

    ``layers``: lists of node dicts with keys replica, owner, children
    [(row, arena, path, multiplier)], destination_row, sigma_target_row,
    action_begin and optionally input (default 0), nominal, head_row.
    ``leaves``: {(lane, row, arena): (work0 [P, w], work1 [P, w] | None,
    trace [P] | None, cost, delta)}.  ``head``: {(lane, row): (v [w], t, c)}.
    """

    def __init__(self, *, width: int, p_train: int, sampled: bool, branched: bool, lam: float, layers, leaves,
                 head, n_replica: int = 1, cap: int = 8, head_cap: int = 4) -> None:
        self.n_replica, self.p_train, self.sampled, self.branched, self.lam = n_replica, p_train, sampled, branched, lam
        self.input_count = self.output_count = self.action_partitions = 1
        R, P, w = n_replica, p_train, width
        self.width, self.work_cap, self.head_cap = [w], [cap], [head_cap]
        self.conversion = np.arange(w, dtype=np.int32).reshape(1, 1, w)
        flat = [n for layer in layers for n in layer]
        self.layer_ptr = np.cumsum([0] + [len(layer) for layer in layers]).astype(np.int32)
        cols = [[] for _ in range(12)]
        edges = []
        for n in flat:
            values = (n["replica"], len(edges), len(n["children"]), n["destination_row"], n.get("input", 0), 0,
                      n["owner"], n.get("nominal", len(n["children"])), len(n["children"]), n.get("head_row", 0),
                      n["sigma_target_row"], n["action_begin"])
            for c, v in zip(cols, values):
                c.append(v)
            for (r, a, path, mult) in n["children"]:
                edges.append((r if a == 0 else -r - 1, 0, path, mult))
        self.nodes = [np.asarray(c, dtype=np.int32) for c in cols]
        self.children = [np.asarray([e[k] for e in edges], dtype=np.int32) for k in range(3)] + [
            np.asarray([e[3] for e in edges], dtype=np.float32)]
        work0 = np.zeros((R, cap, 2, P, w), np.float32)
        work1 = np.zeros((R, cap, 2, P, w), np.float32)
        trace = np.zeros((R, cap, 2, P), np.float32)
        cost = np.zeros((R, cap, 2), np.float32)
        delta = np.zeros((R, cap, 2), np.float32)
        for (lane, row, arena), (v0, v1, tr, c, d) in leaves.items():
            work0[lane, row, arena] = v0
            if v1 is not None:
                work1[lane, row, arena] = v1
            if tr is not None:
                trace[lane, row, arena] = tr
            cost[lane, row, arena] = c
            delta[lane, row, arena] = d
        hv = np.zeros((R, head_cap, w), np.float32)
        ht = np.zeros((R, head_cap), np.float32)
        hc = np.zeros((R, head_cap), np.float32)
        for (lane, row), (v, t, c) in head.items():
            hv[lane, row], ht[lane, row], hc[lane, row] = v, t, c
        rows = 1 + max(n["sigma_target_row"] for n in flat)
        arows = max(n["action_begin"] + len(n["children"]) for n in flat)
        self.arenas = {
            "work0": [work0], "work1": None if sampled else [work1],
            "trace": [trace] if branched else None, "cost": [cost] if branched else None,
            "delta": [delta] if branched else None, "head_v": [hv],
            "head_t": [ht] if branched else None, "head_c": [hc] if branched else None,
            "sigma_v": [np.full((rows, w), np.nan, np.float32) for _ in range(R)],
            "sigma_t": [np.full((rows,), np.nan, np.float32) for _ in range(R)] if branched else None,
            "sigma_c": [np.full((rows,), np.nan, np.float32) for _ in range(R)] if branched else None,
            "action_p": None if sampled else [np.full((arows, w), np.nan, np.float32) for _ in range(R)],
            "action_a": [np.full((arows, w), np.nan, np.float32) for _ in range(R)],
        }


# ---------------------------------------------------------------- known answers
# The expected values below are the ones pbg's own tests assert for its
# layered-target executor (tests/test_layered_targets.py:1115-1402,
# 1624-1745), restated on hand-built plans: head rows hold old value 2.0,
# old trace 0.25 and old cost 3.0 (tests/test_layered_targets.py:480-499).

OLD_V, OLD_T, OLD_C = 2.0, 0.25, 3.0


def _one_node_plan(*, p_train: int, leaves: int, sampled: bool, branched: bool, lam: float = 0.5, payoff=None,
                   n_replica: int = 1):
    width = 1 if sampled else 2
    leaf_rows = {}
    if sampled:
        pay = (np.arange(1, leaves * p_train + 1, dtype=np.float32).reshape(leaves, p_train)
               if payoff is None else np.asarray(payoff, np.float32))
        for i in range(leaves):
            leaf_rows[(0, i, 0)] = (pay[i].reshape(p_train, 1), None, pay[i] if branched else None, 0.0, 0.0)
        values = pay
    else:
        mass = np.ones((leaves, p_train, 2), np.float32)
        values = np.arange(1, leaves * p_train * 2 + 1, dtype=np.float32).reshape(leaves, p_train, 2)
        for i in range(leaves):
            leaf_rows[(0, i, 0)] = (mass[i], mass[i] * values[i], (mass[i] * values[i]).sum(-1) if branched else None,
                                    0.0, 0.0)
    node = dict(replica=0, owner=0, children=[(i, 0, 1, 1.0) for i in range(leaves)], destination_row=0,
                sigma_target_row=0, action_begin=0, nominal=leaves)
    plan = HandPlan(width=width, p_train=p_train, sampled=sampled, branched=branched, lam=lam, layers=[[node]],
                    leaves=leaf_rows, head={(0, 0): (np.full(width, OLD_V), OLD_T, OLD_C)}, n_replica=n_replica)
    return plan, values


def mode_cases():
    """pbg tests/test_layered_targets.py:1193-1307: all twelve modes, one node."""

    cases = []
    for regime, p_train in (("self_play", 2), ("best_response", 1)):
        for rollout in ("sequential", "branched.fixed", "branched.KKT"):
            for estimator in ("sampled", "rao_blackwell"):
                sampled, branched = estimator == "sampled", rollout != "sequential"
                leaves = 2 if branched else 1
                plan, values = _one_node_plan(p_train=p_train, leaves=leaves, sampled=sampled, branched=branched)

                def check(failure, arenas, values=values, sampled=sampled, branched=branched, leaves=leaves):
                    assert failure.tolist() == [2**31 - 1]
                    sigma = arenas["sigma_v"][0][0]
                    adv = arenas["action_a"][0]
                    owner = values[:, 0]
                    np.testing.assert_allclose(sigma, owner.mean(0).reshape(sigma.shape), rtol=1e-6)
                    for child in range(leaves):
                        base = OLD_V if leaves == 1 else 0.5 * owner[1 - child] + 1.0
                        np.testing.assert_allclose(adv[child], (owner[child] - base).reshape(adv[child].shape),
                                                   rtol=1e-6)
                    if not sampled:
                        assert np.array_equal(arenas["action_p"][0], np.ones_like(arenas["action_p"][0]))
                    if branched:
                        tv = values if sampled else values.sum(-1)
                        expected = ((tv - tv.mean(0, keepdims=True)) ** 2).sum() / (leaves - 1)
                        np.testing.assert_allclose(arenas["sigma_t"][0], [expected], rtol=1e-6)
                        assert arenas["sigma_c"][0].tolist() == [1.0]
                        assert float(arenas["cost"][0][0, 0, 1]) == 2.0
                        assert float(arenas["delta"][0][0, 0, 1]) == 0.0

                cases.append((f"{regime}-{rollout}-{estimator}", plan, check))
    return cases


def _unbalanced(sampled: bool):
    """Root over (leaf, node 1), node 1 over two leaves; lambda = 1 (test_layered_targets.py:1310-1402)."""

    p_train = 2
    if sampled:
        pay = np.array([[2.0, -2.0], [4.0, -4.0], [8.0, -8.0]], np.float32)
        leaf = {(0, i, 0): (pay[i].reshape(2, 1), None, pay[i], 0.0, 0.0) for i in range(3)}
        width = 1
    else:
        vals = np.array([[[2, 2], [2, 2]], [[4, 4], [4, 4]], [[8, 8], [8, 8]]], np.float32)
        leaf = {(0, i, 0): (np.ones((2, 2), np.float32), vals[i], vals[i].sum(-1), 0.0, 0.0) for i in range(3)}
        width = 2
    node1 = dict(replica=0, owner=0, children=[(1, 0, 1, 1.0), (2, 0, 1, 1.0)], destination_row=0,
                 sigma_target_row=1, action_begin=2, nominal=2)
    root = dict(replica=0, owner=0, children=[(0, 0, 1, 1.0), (0, 1, 1, 1.0)], destination_row=3,
                sigma_target_row=0, action_begin=0, nominal=2)
    plan = HandPlan(width=width, p_train=p_train, sampled=sampled, branched=True, lam=1.0, layers=[[node1], [root]],
                    leaves=leaf, head={(0, 0): (np.full(width, OLD_V), OLD_T, OLD_C)})

    def check(failure, arenas):
        assert failure.tolist() == [2**31 - 1]
        sigma = arenas["sigma_v"][0]
        if sampled:
            assert sigma[:, 0].tolist() == [4.0, 6.0]
        else:
            assert sigma.tolist() == [[4.0, 4.0], [6.0, 6.0]]

    return plan, check


def _rb_invalid(bad_mass: float, bad_moment: float):
    """test_layered_targets.py:1153-1190: one RB leaf channel made invalid fails the lane."""

    leaf = {(0, 0, 0): (np.ones((2, 2), np.float32), np.full((2, 2), 2.0, np.float32), None, 0.0, 0.0)}
    leaf[(0, 0, 0)][0][1, 0] = bad_mass
    leaf[(0, 0, 0)][1][1, 0] = bad_moment
    node = dict(replica=0, owner=0, children=[(0, 0, 1, 1.0)], destination_row=0, sigma_target_row=0, action_begin=0)
    plan = HandPlan(width=2, p_train=2, sampled=False, branched=False, lam=0.5, layers=[[node]], leaves=leaf,
                    head={(0, 0): (np.full(2, OLD_V), OLD_T, OLD_C)})

    def check(failure, arenas):
        assert failure.tolist() == [0]

    return plan, check


def _signed_sampled():
    """test_layered_targets.py:1115-1150: a negative sampled return is valid."""

    plan, _ = _one_node_plan(p_train=2, leaves=1, sampled=True, branched=False, payoff=[[-3.0, 3.0]])

    def check(failure, arenas):
        assert failure.tolist() == [2**31 - 1]
        assert arenas["sigma_v"][0][0].tolist() == [-3.0]

    return plan, check


def _failure_isolated():
    """test_layered_targets.py:1624-1668: a NaN return fails lane 1 only."""

    nodes = [dict(replica=lane, owner=0, children=[(0, 0, 1, 1.0)], destination_row=0, sigma_target_row=0,
                  action_begin=0) for lane in (0, 1)]
    leaf = {(0, 0, 0): (np.array([[3.0], [-3.0]], np.float32), None, None, 0.0, 0.0),
            (1, 0, 0): (np.array([[np.nan], [1.0]], np.float32), None, None, 0.0, 0.0)}
    head = {(lane, 0): (np.full(1, OLD_V), OLD_T, OLD_C) for lane in (0, 1)}
    plan = HandPlan(width=1, p_train=2, sampled=True, branched=False, lam=0.5, layers=[nodes], leaves=leaf,
                    head=head, n_replica=2)

    def check(failure, arenas):
        assert failure.tolist() == [2**31 - 1, 1]
        assert arenas["sigma_v"][0][0].tolist() == [3.0]

    return plan, check


def _concentrated_siblings():
    """test_layered_targets.py:1691-1745: sibling sums are direct, not total minus child."""

    pay = np.array([[1.0e8, 0.0], [1.0, 0.0], [-1.0e8, 0.0]], np.float32)
    leaf = {(0, i, 0): (pay[i].reshape(2, 1), None, pay[i], 0.0, 0.0) for i in range(3)}
    node = dict(replica=0, owner=0, children=[(i, 0, 1, 1.0) for i in range(3)], destination_row=0,
                sigma_target_row=0, action_begin=0, nominal=3)
    plan = HandPlan(width=1, p_train=2, sampled=True, branched=True, lam=1.0, layers=[[node]], leaves=leaf,
                    head={(0, 0): (np.full(1, OLD_V), OLD_T, OLD_C)})

    def check(failure, arenas):
        assert float(arenas["action_a"][0][1, 0]) == 1.0

    return plan, check


def known_answer_cases():
    cases = mode_cases()
    for sampled in (True, False):
        cases.append((f"unbalanced-{'sampled' if sampled else 'rb'}", *_unbalanced(sampled)))
    for bad in ((-1.0, -2.0), (0.0, 1.0)):
        cases.append((f"rb-invalid-{bad}", *_rb_invalid(*bad)))
    cases.append(("signed-sampled", *_signed_sampled()))
    cases.append(("failure-isolated", *_failure_isolated()))
    cases.append(("concentrated-siblings", *_concentrated_siblings()))
    return cases
