"""LFM2.5-shaped MoE block with GGML Q4_K experts on the GPU vs the oracle:
hidden 2048, 32 experts, top-4, intermediate 1792, sigmoid router whose
selection bias only steers selection (lfm2moe_q.rs:241-258), SiLU-gated
experts without biases, combine in ascending expert order."""
import numpy as np
import pytest

import oracle
from gallium_b200 import GalliumError, Lfm2QMoEFFN, synth

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_REL = 2e-2, 1e-3


def _cuda(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _parity(got, want, what):
    err = np.abs(np.asarray(got, np.float64) - want)
    max_abs, mean_rel = float(err.max()), float(err.sum() / np.abs(want).sum())
    assert max_abs <= MAX_ABS and mean_rel <= MEAN_REL, (what, max_abs, mean_rel)


@pytest.fixture(scope="module")
def layer():
    lay = synth.lfm2_layer(n_experts=32, seed=0)
    lay.sel_bias[:] = np.random.default_rng(1).normal(0, 0.05, 32).astype(np.float32)
    return lay


@pytest.fixture(scope="module")
def moe(layer):
    m = Lfm2QMoEFFN.load(layer, device=0, max_tokens=64)
    yield m
    m.close()


@pytest.mark.parametrize("expert", [0, 31])
def test_q4k_device_dequant_is_bit_exact(moe, layer, expert):
    H, I = layer.hidden, layer.inter
    g = oracle.q4k_dequant(layer.gate_raw[expert].ravel(), I * H).reshape(I, H)
    u = oracle.q4k_dequant(layer.up_raw[expert].ravel(), I * H).reshape(I, H)
    d = oracle.q4k_dequant(layer.down_raw[expert].ravel(), H * I).reshape(H, I)
    for which, want in ((0, g), (1, u), (2, d)):
        got = moe.dequant_expert(which, expert).cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), which


@pytest.mark.parametrize("T", [1, 5, 64])
def test_sigmoid_routing_is_bit_exact(moe, layer, T):
    x = synth.tokens(T, 2048, seed=T)
    r = moe.route(_cuda(x))
    idx, w = oracle.route_sigmoid_topk(oracle.router_logits(x, layer.router_w), layer.sel_bias, 4)
    counts, offsets, perm, _ = oracle.permute(idx, 32)
    assert np.array_equal(r["idx"].cpu().numpy(), idx)
    assert np.array_equal(r["perm"].cpu().numpy(), perm)
    # same exp, same order: the weights are bit-identical too
    assert np.array_equal(r["w"].cpu().numpy(), w)


# AUTO kernel choice at 32 experts: CUDA cores below 2 rows per expert
# (T = 1, 8), the small-batch tensor-core kernel from there (T = 16, 24, 64)
@pytest.mark.parametrize("T", [1, 8, 16, 24, 64])
def test_lfm2_forward_matches_oracle(moe, layer, T):
    x = synth.tokens(T, 2048, seed=900 + T)
    got = moe.forward(_cuda(x)).cpu().numpy()
    want, _, _ = oracle.OracleLfm2(layer).forward(x)
    _parity(got, want, f"T={T}")


def test_lfm2_full_size_sampled_rows_and_determinism(moe, layer):
    T = 2048
    x = synth.tokens(T, 2048, seed=2048)
    xc = _cuda(x)
    a = moe.forward(xc).cpu().numpy()
    b = moe.forward(xc).cpu().numpy()
    assert np.array_equal(a, b)
    rows = np.random.default_rng(3).choice(T, 16, replace=False)
    want, _, _ = oracle.OracleLfm2(layer).forward(x[rows])
    _parity(a[rows], want, "T=2048 sampled rows")
    # every row against the grouped CPU forward (oracle/cpu_reference.py,
    # checked against the oracle by tests/test_cpu_reference.py)
    from oracle.cpu_reference import CpuReference
    ref = CpuReference(layer)
    try:
        _parity(a, ref.forward(x), "T=2048 every row")
    finally:
        ref.close()


def test_q4k_ragged_rows_are_refused():
    lay = synth.lfm2_layer(n_experts=4, hidden=256, inter=256, top_k=2, seed=1)
    lay.hidden = 200
    with pytest.raises(GalliumError) as ei:
        Lfm2QMoEFFN.load(lay, device=0)
    assert "256-element" in str(ei.value)


@pytest.mark.parametrize("path", ["tensor_cores", "tensor_cores_f16"])
@pytest.mark.parametrize("T", [1, 8, 64, 300])
def test_lfm2_tensor_core_path_matches_oracle(layer, T, path):
    # Two kind::f16 kernels: "tensor_cores" runs the weights as the exact
    # integers sc * q with the super-block scales applied to the partial sums
    # while the batch averages at most 24 rows per expert (T = 1, 8, 64 here)
    # and the f16 hi + lo decode above that (T = 300); "tensor_cores_f16"
    # forces the hi + lo decode.  AUTO takes the tensor cores from 2 rows per
    # expert.
    m = Lfm2QMoEFFN.load(layer, device=0, max_tokens=T)
    try:
        m.set_expert_path(path)
        x = synth.tokens(T, 2048, seed=1300 + T)
        got = m.forward(_cuda(x)).cpu().numpy()
        want, _, _ = oracle.OracleLfm2(layer).forward(x)
        _parity(got, want, f"{path} T={T}")
        m.set_expert_path("cuda_cores")
        cc = m.forward(_cuda(x)).cpu().numpy()
        _parity(got, cc.astype(np.float64), f"{path} vs CUDA cores T={T}")
    finally:
        m.close()


def test_lfm2_small_batch_kernel_splits_a_crowded_expert(layer):
    # every token picks expert 0 (selection bias), so it gets 64 rows: two
    # tiles of 32 in the small-batch kernel while the batch averages 8 rows
    # per expert
    import copy
    lay = copy.deepcopy(layer)
    lay.sel_bias[:] = 0.0
    lay.sel_bias[0] = 30.0
    T = 64
    m = Lfm2QMoEFFN.load(lay, device=0, max_tokens=T)
    try:
        m.set_expert_path("tensor_cores")
        x = synth.tokens(T, 2048, seed=1777)
        got = m.forward(_cuda(x)).cpu().numpy()
        want, idx, _ = oracle.OracleLfm2(lay).forward(x)
        assert (np.asarray(idx) == 0).any(axis=1).all()
        _parity(got, want, "crowded expert")
    finally:
        m.close()
