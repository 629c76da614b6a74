"""gallium-core's generic MoEFFN (dense experts, ffn.rs:72-166) on the GPU
against the oracle: expert indices bit for bit, outputs within max-abs 2e-2
and mean-rel 1e-3.  Covers the four activations, the clamp of act(gate), the
shared expert, bf16 and f32 weights, and batch sizes from one token to
several hundred (one and several staged chunks per expert)."""
import numpy as np
import pytest

import oracle
from gallium_b200 import MoEFFN, synth

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_REL = 2e-2, 1e-3

CASES = [  # (activation, clamp, shared_inter, bf16)
    (1, 0.0, 64, True), (2, 0.0, 0, True), (3, 2.0, 64, True), (4, 0.0, 32, True),
    (1, 1.5, 96, False),
]


@pytest.mark.parametrize("act,clamp,shared,bf16", CASES)
def test_dense_moe_matches_oracle(act, clamp, shared, bf16):
    import torch

    layer = synth.dense_layer(n_experts=16, hidden=256, inter=192, top_k=4, shared_inter=shared,
                              act_kind=act, act_clamp=clamp, seed=10 + act, bf16=bf16)
    orc = oracle.OracleDense(layer)
    with MoEFFN.load(layer, device=0, max_tokens=300) as moe:
        for T in (1, 5, 37, 300):
            x = synth.tokens(T, 256, seed=T)
            got = moe.forward(torch.from_numpy(x).cuda()).cpu().numpy()
            r = moe.route(torch.from_numpy(x).cuda())
            want, idx, w = orc.forward(x)
            assert np.array_equal(r["idx"].cpu().numpy(), idx), T
            assert np.array_equal(r["w"].cpu().numpy(), w), T
            err = np.abs(got.astype(np.float64) - want)
            assert err.max() <= MAX_ABS and err.sum() / np.abs(want).sum() <= MEAN_REL, (
                T, err.max())


def test_qwen_shaped_dense_layer_decode_and_prefill():
    """A Qwen3-MoE-like layer (hidden 2048, 128 experts, top-8, expert
    intermediate 768, shared expert 512, SiLU, bf16): sampled rows at 1 and
    512 tokens."""
    import torch

    layer = synth.dense_layer(seed=3)
    orc = oracle.OracleDense(layer)
    with MoEFFN.load(layer, device=0, max_tokens=512) as moe:
        for T in (1, 512):
            x = synth.tokens(T, 2048, seed=5)
            got = moe.forward(torch.from_numpy(x).cuda()).cpu().numpy()
            rows = np.arange(T) if T < 16 else np.random.default_rng(0).choice(T, 16, False)
            want, _, _ = orc.forward(x[rows])
            err = np.abs(got[rows].astype(np.float64) - want)
            assert err.max() <= MAX_ABS and err.sum() / np.abs(want).sum() <= MEAN_REL
