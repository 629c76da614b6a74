"""The oracle's Gemma-4 routed-experts block against a float64 numpy
restatement written from QGemmaMoe::forward (gemma4_q.rs:262-328): router on
rms(x) / sqrt(H) * ffn_gate_inp.scale, softmax, top-k by probability,
weights p / max(sum, 6.1035e-5); experts on pre_ffw_norm_2(x) with the merged
gate_up (gate rows first), GELU (tanh) gating, down, times the expert's output
scale; sum in expert order; post_ffw_norm_2 on the result."""
import math

import numpy as np
import pytest

import oracle
from gallium_b200 import synth


@pytest.mark.parametrize("fmt,H,I,scale", [(1, 256, 96, True), (2, 256, 256, True),
                                          (1, 128, 64, False)])
def test_gemma4_block_matches_restatement(fmt, H, I, scale):
    layer = synth.gemma4_layer(n_experts=8, hidden=H, inter=I, top_k=3, fmt=fmt, seed=fmt,
                               expert_scale=scale)
    x = synth.tokens(9, H, seed=2)
    out, idx, _ = oracle.OracleGemma4(layer).forward(x)
    X = x.astype(np.float64)
    rms = lambda v: v / np.sqrt((v ** 2).mean(-1, keepdims=True) + layer.rms_eps)
    xr = rms(X) * H ** -0.5 * layer.router_scale
    xe = rms(X) * layer.expert_norm
    lg = xr @ layer.router_w.T.astype(np.float64)
    p = np.exp(lg - lg.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    deq = oracle.mxfp4_gguf_dequant if fmt == 1 else oracle.q4k_dequant
    acc = np.zeros_like(X)
    for t in range(9):
        top = np.argsort(-p[t], kind="stable")[:3]
        assert list(top) == list(idx[t])
        wts = p[t, top] / max(p[t, top].sum(), 6.1035e-5)
        for e, wt in sorted(zip(top, wts)):
            gu = deq(layer.gate_up_raw[e], 2 * I * H).reshape(2 * I, H).astype(np.float64)
            dn = deq(layer.down_raw[e], H * I).reshape(H, I).astype(np.float64)
            g, u = gu[:I] @ xe[t], gu[I:] @ xe[t]
            a = 0.5 * g * (1 + np.tanh(math.sqrt(2 / math.pi) * (g + 0.044715 * g ** 3))) * u
            y = dn @ a
            if scale:
                y = y * layer.expert_scale[e]
            acc[t] += y * wt
    want = rms(acc) * layer.output_norm
    assert np.abs(out - want).max() <= 1e-5 * max(1.0, np.abs(want).max())
