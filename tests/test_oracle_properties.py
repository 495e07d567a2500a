"""Properties of the numpy oracle that hold independently of the reference fixtures: the
routed forward equals a dense computation masked by the top-k weights, expert
parallelism without a capacity does not change any token's output, and the capacity
cut keeps at most `capacity` rows per expert, the lowest (source rank, token, slot)
first.  Together with the fixture pins they check the oracle from a second side."""
import numpy as np
import pytest

from oracle import moe_oracle as O


def _params(rng, E, d, F, kind):
    if kind == "linear":
        return O.MoEParams(gate=rng.standard_normal((E, d)).astype(np.float32) * 0.3, expert_type="linear",
                           expert_w=(rng.standard_normal((E, d, d)) * 0.1).astype(np.float32))
    w = lambda *s: (rng.standard_normal(s) * 0.1).astype(np.float32)
    return O.MoEParams(gate=rng.standard_normal((E, d)).astype(np.float32) * 0.3, expert_type="swiglu",
                       w1=w(E, F, d), w3=w(E, F, d), w2=w(E, d, F))


def _dense(x, p, k):
    """Every expert on every token, weighted by the router's top-k softmax (0 elsewhere)."""
    idx, w, _ = O.route(x, p.gate, k, p.logit_bias)
    T, E = x.shape[0], p.gate.shape[0]
    gate_w = np.zeros((T, E))
    for j in range(k):
        gate_w[np.arange(T), idx[:, j]] += w[:, j]
    out = np.zeros((T, x.shape[1]))
    for e in range(E):
        if p.expert_type == "linear":
            y = x.astype(np.float64) @ p.expert_w[e].astype(np.float64)
        else:
            xe = x.astype(np.float64)
            g = xe @ p.w1[e].T.astype(np.float64)
            u = xe @ p.w3[e].T.astype(np.float64)
            y = (g / (1 + np.exp(-g)) * u) @ p.w2[e].T.astype(np.float64)
        out += gate_w[:, e:e + 1] * y
    return out


@pytest.mark.parametrize("kind", ["linear", "swiglu"])
@pytest.mark.parametrize("E,k", [(8, 2), (16, 5), (4, 4)])
def test_routed_forward_equals_masked_dense(kind, E, k):
    rng = np.random.default_rng(E * 10 + k)
    d, F, T = 16, 24, 37
    p = _params(rng, E, d, F, kind)
    x = rng.standard_normal((T, d)).astype(np.float32)
    (out,) = O.moe_forward([x], p, k=k, acc=np.float64)
    # fp64 accumulation, output stored as fp32: equal up to the final rounding
    assert np.abs(out - _dense(x, p, k)).max() <= 1e-6 * max(1e-3, np.abs(out).max())


@pytest.mark.parametrize("ws", [2, 4])
def test_expert_parallel_without_capacity_matches_one_rank(ws):
    rng = np.random.default_rng(ws)
    E, d, F, k = 8, 16, 24, 2
    p = _params(rng, E, d, F, "swiglu")
    xs = [rng.standard_normal((T, d)).astype(np.float32) for T in (13, 0, 29, 5)[:ws]]
    outs = O.moe_forward(xs, p, ws=ws, k=k, acc=np.float64)
    for x, o in zip(xs, outs):
        (ref,) = O.moe_forward([x], p, k=k, acc=np.float64)
        assert o.shape == ref.shape
        assert np.abs(o - ref).max(initial=0.0) <= 1e-12


@pytest.mark.parametrize("ws,cap", [(1, 3), (2, 5), (4, 2)])
def test_capacity_keeps_lowest_indices(ws, cap):
    rng = np.random.default_rng(cap)
    E, T, k = 4, 11, 2
    idx = [np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32) for _ in range(ws)]
    plan, kept = O.dispatch_plan(idx, E, ws, cap)
    for e in range(E):
        rows = [tuple(r) for r in plan[e]]
        assert len(rows) == min(cap, sum(int((i == e).sum()) for i in idx))
        allrows = sorted((r, t, j) for r in range(ws) for t in range(T) for j in range(k) if idx[r][t, j] == e)
        assert rows == allrows[:len(rows)]          # the lowest (rank, token, slot) win
