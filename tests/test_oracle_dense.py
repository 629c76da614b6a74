"""The oracle's generic MoEFFN (dense experts, ffn.rs:72-166) against a float64
numpy restatement written from the reference's code: router softmax over all
experts, the k largest probabilities renormalised (ffn.rs:131-149), each
expert's GatedFFN act(gate) clamped then times up, then down (ffn.rs:56-66),
rank-order sum, plus the shared expert over every token (ffn.rs:160-163)."""
import math

import numpy as np
import pytest

import oracle
from gallium_b200 import synth


def _restated(layer, x):
    f = lambda a: synth.bf16_bits_to_f32(a).astype(np.float64)
    rw, G, U, D = f(layer.router_w), f(layer.gate), f(layer.up), f(layer.down)
    lg = x.astype(np.float64) @ rw.T
    p = np.exp(lg - lg.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    c = layer.act_clamp

    def act(g):
        if layer.act_kind == 1:
            a = g / (1 + np.exp(-g))
        elif layer.act_kind == 2:
            a = 0.5 * g * (1 + np.vectorize(math.erf)(g / math.sqrt(2)))
        elif layer.act_kind == 3:
            a = 0.5 * g * (1 + np.tanh(math.sqrt(2 / math.pi) * (g + 0.044715 * g ** 3)))
        else:
            a = np.maximum(g, 0)
        return np.clip(a, -c, c) if c > 0 else a

    out = np.zeros(x.shape, np.float64)
    tops = []
    for t in range(x.shape[0]):
        top = np.argsort(-p[t], kind="stable")[:layer.top_k]
        tops.append(top)
        for e, wt in zip(top, p[t, top] / p[t, top].sum()):
            out[t] += wt * (D[e] @ (act(G[e] @ x[t]) * (U[e] @ x[t])))
        if layer.shared_inter:
            h = act(f(layer.sh_gate) @ x[t]) * (f(layer.sh_up) @ x[t])
            out[t] += f(layer.sh_down) @ h
    return out, np.array(tops)


@pytest.mark.parametrize("act,clamp,shared", [(1, 0.0, 64), (2, 0.0, 0), (3, 2.0, 64),
                                              (4, 0.0, 32), (1, 1.5, 0)])
def test_dense_moe_matches_restatement(act, clamp, shared):
    layer = synth.dense_layer(n_experts=8, hidden=128, inter=96, top_k=3, shared_inter=shared,
                              act_kind=act, act_clamp=clamp, seed=act)
    x = synth.tokens(12, 128, seed=1)
    out, idx, _ = oracle.OracleDense(layer).forward(x)
    want, top = _restated(layer, x)
    assert np.array_equal(idx, top)
    assert np.abs(out - want).max() <= 1e-5 * max(1.0, np.abs(want).max())
