"""Gemma-4's routed-experts block (QGemmaMoe, gemma4_q.rs:187-330) on the GPU
against the oracle: expert indices bit for bit, outputs within max-abs 2e-2
and mean-rel 1e-3.  GGUF MXFP4 experts at the 26B-A4B shape (hidden 2816, 128
experts, top-8, expert intermediate 704) and Q4_K experts at a smaller one;
merged gate_up, GELU (tanh) gating, per-expert output scales, the router's and
the experts' input norms and the output norm."""
import numpy as np
import pytest

import oracle
from gallium_b200 import QGemmaMoe, synth

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_REL = 2e-2, 1e-3


@pytest.mark.parametrize("fmt,E,H,I,k,Ts", [
    (1, 128, 2816, 704, 8, (1, 7, 64)),
    (2, 16, 512, 256, 4, (1, 5, 40, 300)),
    (1, 16, 256, 96, 4, (3, 100)),
])
def test_gemma4_block_matches_oracle(fmt, E, H, I, k, Ts):
    import torch

    layer = synth.gemma4_layer(n_experts=E, hidden=H, inter=I, top_k=k, fmt=fmt, seed=E + fmt)
    orc = oracle.OracleGemma4(layer)
    with QGemmaMoe.load(layer, device=0, max_tokens=max(Ts)) as moe:
        for T in Ts:
            x = synth.tokens(T, H, seed=T)
            got = moe.forward(torch.from_numpy(x).cuda()).cpu().numpy()
            want, idx, _ = orc.forward(x)
            err = np.abs(got.astype(np.float64) - want)
            assert err.max() <= MAX_ABS and err.sum() / np.abs(want).sum() <= MEAN_REL, (
                T, err.max())
