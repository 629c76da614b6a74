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


@pytest.mark.parametrize("path", ["cuda_cores", "tensor_cores"])
def test_dense_paths_agree_with_oracle_at_every_batch_size(path):
    """Both dense expert paths forced: the CUDA-core kernel and the bf16
    tensor-core kernel (gate / up rows interleaved, activations as bf16 hi +
    lo), with a shared expert that takes the same path, from 1 token (16-wide
    MMAs) to 300 (full 128-position tiles and ragged ones)."""
    import torch

    layer = synth.dense_layer(n_experts=16, hidden=256, inter=192, top_k=4, shared_inter=128,
                              act_kind=1, seed=21)
    orc = oracle.OracleDense(layer)
    with MoEFFN.load(layer, device=0, max_tokens=300) as moe:
        moe.set_expert_path(path)
        for T in (1, 3, 16, 37, 129, 300):
            x = synth.tokens(T, 256, seed=40 + T)
            got = moe.forward(torch.from_numpy(x).cuda()).cpu().numpy()
            want, _, _ = orc.forward(x)
            err = np.abs(got.astype(np.float64) - want)
            assert err.max() <= MAX_ABS and err.sum() / np.abs(want).sum() <= MEAN_REL, (
                path, T, err.max())


def test_tensor_core_path_needs_bf16_weights():
    from gallium_b200 import GalliumError

    layer = synth.dense_layer(n_experts=8, hidden=128, inter=64, top_k=2, shared_inter=0,
                              seed=2, bf16=False)
    with MoEFFN.load(layer, device=0, max_tokens=4) as moe:
        with pytest.raises(GalliumError):
            moe.set_expert_path("tensor_cores")


@pytest.mark.parametrize("bf16", [True, False])
def test_dense_dequant_returns_the_stored_weights(bf16):
    """gb_moe_dequant_expert on dense experts: the stored gate, up and down
    matrices, widened to f32 exactly (gate and up are kept interleaved on the
    device)."""
    layer = synth.dense_layer(n_experts=4, hidden=128, inter=64, top_k=2, shared_inter=0,
                              seed=8, bf16=bf16)

    def f32(a):
        return synth.bf16_bits_to_f32(a) if bf16 else a

    with MoEFFN.load(layer, device=0, max_tokens=4) as moe:
        for e in range(4):
            for which, want in ((0, layer.gate[e]), (1, layer.up[e]), (2, layer.down[e])):
                got = moe.dequant_expert(which, e).cpu().numpy()
                assert np.array_equal(got, f32(want)), (e, which)
