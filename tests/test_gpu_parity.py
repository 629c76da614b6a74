"""CUDA path vs the CPU oracle, through the C ABI (needs a B200).

Bar (from the path's contract): expert indices and the grouping permutation
bit-exact; outputs within max-abs 2e-2 and mean-rel 1e-3 after f32
accumulation, where mean-rel = sum|gpu - oracle| / sum|oracle|.  Dequantised
weights are compared bit for bit.
"""
import numpy as np
import pytest

import oracle
from gallium_b200 import GalliumError, GptOssQMoEFFN, OssMoEFFN, synth

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_REL = 1e-3


def _torch():
    import torch
    return torch


def assert_parity(got, want, what=""):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape
    assert np.all(np.isfinite(got)), what
    err = np.abs(got - want)
    max_abs = float(err.max()) if err.size else 0.0
    mean_rel = float(err.sum() / max(np.abs(want).sum(), 1e-30))
    assert max_abs <= MAX_ABS and mean_rel <= MEAN_REL, (
        f"{what}: max_abs {max_abs:.3e} (<= {MAX_ABS}), mean_rel {mean_rel:.3e} (<= {MEAN_REL})")
    return max_abs, mean_rel


@pytest.fixture(scope="module")
def layer32():
    return synth.gptoss_layer(n_experts=32, seed=0)


@pytest.fixture(scope="module")
def moe32(layer32):
    m = OssMoEFFN.load(layer32, device=0, max_tokens=64)
    yield m
    m.close()


@pytest.fixture(scope="module")
def layer32_skew():
    return synth.gptoss_layer(n_experts=32, seed=1, skewed=True)


@pytest.fixture(scope="module")
def moe32_skew(layer32_skew):
    m = OssMoEFFN.load(layer32_skew, device=0, max_tokens=64)
    yield m
    m.close()


def _route_oracle(layer, x):
    rw = synth.bf16_bits_to_f32(layer.router_w)
    rb = synth.bf16_bits_to_f32(layer.router_b)
    logits = oracle.router_logits(x, rw, rb)
    idx, w = oracle.route_softmax_topk(logits, layer.top_k)
    counts, offsets, perm, inv = oracle.permute(idx, layer.n_experts)
    return logits, idx, w, counts, offsets, perm


def _cuda(a):
    return _torch().from_numpy(np.ascontiguousarray(a)).cuda()


def _cpu_grouped_forward(layer, x):
    """Every row of a large batch on the CPU: the grouped forward of
    oracle/cpu_reference.py (BLAS GEMMs), which tests/test_cpu_reference.py
    checks against the oracle."""
    from oracle.cpu_reference import CpuReference
    ref = CpuReference(layer)
    try:
        return ref.forward(x)
    finally:
        ref.close()


# ---- decoders ---------------------------------------------------------------

@pytest.mark.parametrize("expert", [0, 17, 31])
def test_device_dequant_is_bit_exact(moe32, layer32, expert):
    gu = oracle.mxfp4_split_dequant(layer32.gu_blocks[expert], layer32.gu_scales[expert])
    dn = oracle.mxfp4_split_dequant(layer32.dn_blocks[expert], layer32.dn_scales[expert])
    for which, want in ((0, gu[0::2]), (1, gu[1::2]), (2, dn)):
        got = moe32.dequant_expert(which, expert).cpu().numpy()
        assert np.array_equal(got.view(np.uint32), np.ascontiguousarray(want).view(np.uint32))


def test_gguf_upload_repacks_to_the_same_values():
    layer = synth.gptoss_layer(n_experts=4, hidden=256, inter=192, seed=6)
    # exercise scale byte 0 (GGUF: 2^-127 per quantized.rs:375-383)
    layer.gu_scales[1, 3, 2] = 0
    gg = synth.gptoss_gguf_from_split(layer)
    m = GptOssQMoEFFN.load(gg, device=0, max_tokens=8)
    try:
        for e in range(4):
            g = oracle.mxfp4_gguf_dequant(gg.gate_raw[e], 192 * 256).reshape(192, 256)
            u = oracle.mxfp4_gguf_dequant(gg.up_raw[e], 192 * 256).reshape(192, 256)
            d = oracle.mxfp4_gguf_dequant(gg.down_raw[e], 256 * 192).reshape(256, 192)
            for which, want in ((0, g), (1, u), (2, d)):
                got = m.dequant_expert(which, e).cpu().numpy()
                assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (e, which)
    finally:
        m.close()


# ---- routing ----------------------------------------------------------------

@pytest.mark.parametrize("T", [1, 3, 8, 64, 512])
def test_routing_is_bit_exact(moe32, layer32, T):
    x = synth.tokens(T, 2880, seed=T)
    r = moe32.route(_cuda(x))
    logits, idx, w, counts, offsets, perm = _route_oracle(layer32, x)
    assert np.array_equal(r["idx"].cpu().numpy(), idx)
    assert np.array_equal(r["counts"].cpu().numpy(), counts)
    assert np.array_equal(r["offsets"].cpu().numpy(), offsets)
    assert np.array_equal(r["perm"].cpu().numpy(), perm)
    # the kernel's exp is the oracle's (correctly rounded) and the sums run in
    # the same order, so the combine weights are bit-identical too
    assert np.array_equal(r["w"].cpu().numpy(), w)


def test_routing_skewed_and_128_experts(moe32_skew, layer32_skew):
    x = synth.tokens(256, 2880, seed=77)
    r = moe32_skew.route(_cuda(x))
    _, idx, w, counts, offsets, perm = _route_oracle(layer32_skew, x)
    assert np.array_equal(r["idx"].cpu().numpy(), idx)
    assert np.array_equal(r["perm"].cpu().numpy(), perm)
    assert counts[0] > counts[-1]  # skew is visible


def _one_hot_router_layer(E, k):
    """A layer whose f32 router weight is the identity on the first E inputs
    and has no bias, so a token's logits are exactly its first E inputs."""
    layer = synth.gptoss_layer(n_experts=E, hidden=64, inter=64, top_k=k, seed=0)
    rw = np.zeros((E, 64), np.float32)
    rw[np.arange(E), np.arange(E)] = 1.0
    layer.router_w, layer.router_b = rw, None
    return layer


def test_routing_near_ties_rank_by_probability():
    """Logits one unit in the last place apart whose softmax probabilities are
    equal (gpt_oss.rs:174-182 sorts probabilities, stably): the lower index
    wins although its logit is the smaller.  One case ties in exp(l - max)
    (the subtraction rounds both to the same value), one only after the
    division by the row sum."""
    import test_router_exp as tre

    for lg in (tre.near_tie_logits(), tre.near_tie_division_logits()):
        E = lg.shape[0]
        layer = _one_hot_router_layer(E, 2)
        x = np.zeros((3, 64), np.float32)
        x[:, :E] = lg
        m = OssMoEFFN.load(layer, device=0, max_tokens=4)
        try:
            r = m.route(_cuda(x))
        finally:
            m.close()
        idx, w = oracle.route_softmax_topk(x[:, :E], 2)
        assert np.array_equal(r["idx"].cpu().numpy(), idx), (lg, r["idx"], idx)
        assert np.array_equal(r["w"].cpu().numpy(), w)
        hi = int(np.argmax(np.where(np.arange(E) == idx[0, 0], -np.inf, lg)))
        assert hi != idx[0, 1] and lg[hi] > lg[idx[0, 1]]  # a logit ranking would differ


def test_routing_ties_take_the_lower_index():
    layer = synth.gptoss_layer(n_experts=8, hidden=64, inter=64, top_k=2, seed=0)
    layer.router_w[:] = 0
    layer.router_b[:] = synth.f32_to_bf16_bits(np.array([0, 1, 1, 0, 1, 0, 0, 0], np.float32))
    m = OssMoEFFN.load(layer, device=0, max_tokens=4)
    try:
        r = m.route(_cuda(synth.tokens(3, 64, seed=1)))
        assert r["idx"].cpu().numpy().tolist() == [[1, 2]] * 3
        np.testing.assert_allclose(r["w"].cpu().numpy(), 0.5)
    finally:
        m.close()


# ---- whole block ------------------------------------------------------------

@pytest.mark.parametrize("T", [1, 8, 64])
def test_forward_matches_oracle_20b_balanced(moe32, layer32, T):
    x = synth.tokens(T, 2880, seed=100 + T)
    got = moe32.forward(_cuda(x)).cpu().numpy()
    want, idx, _ = oracle.OracleMoe(layer32).forward(x)
    assert_parity(got, want, f"T={T}")


@pytest.mark.parametrize("T", [1, 64])
def test_forward_matches_oracle_20b_skewed(moe32_skew, layer32_skew, T):
    x = synth.tokens(T, 2880, seed=200 + T)
    got = moe32_skew.forward(_cuda(x)).cpu().numpy()
    want, _, _ = oracle.OracleMoe(layer32_skew).forward(x)
    assert_parity(got, want, f"skewed T={T}")


def test_forward_matches_oracle_120b_shape():
    layer = synth.gptoss_layer(n_experts=128, seed=0)
    m = OssMoEFFN.load(layer, device=0, max_tokens=32)
    try:
        for T in (1, 32):
            x = synth.tokens(T, 2880, seed=300 + T)
            got = m.forward(_cuda(x)).cpu().numpy()
            want, _, _ = oracle.OracleMoe(layer).forward(x)
            assert_parity(got, want, f"E=128 T={T}")
    finally:
        m.close()


def test_gguf_format_forward_matches_oracle(layer32):
    gg = synth.gptoss_gguf_from_split(layer32)
    m = GptOssQMoEFFN.load(gg, device=0, max_tokens=16)
    try:
        x = synth.tokens(16, 2880, seed=5)
        got = m.forward(_cuda(x)).cpu().numpy()
        want, _, _ = oracle.OracleMoe(layer32, gguf=gg).forward(x)
        assert_parity(got, want, "gguf")
    finally:
        m.close()


def test_host_path_equals_device_path(moe32):
    torch = _torch()
    x = synth.tokens(5, 2880, seed=9)
    dev = moe32.forward(_cuda(x)).cpu().numpy()
    host = moe32.forward(torch.from_numpy(x)).numpy()
    assert np.array_equal(dev, host)


def test_chunked_host_path_equals_device_path(moe32):
    # 4096 tokens through host buffers run as overlapped chunks of 1024,
    # 2048 and 1024; every chunk keeps tiles of 30 or 60 positions (mean rows
    # per expert > 8, one accumulation order), so the result equals the
    # one-launch device forward bit for bit
    torch = _torch()
    x = synth.tokens(4096, 2880, seed=19)
    dev = moe32.forward(_cuda(x)).cpu().numpy()
    host = moe32.forward(torch.from_numpy(x)).numpy()
    assert np.array_equal(dev, host)


def test_batch_shape_and_dtype_contract(moe32):
    torch = _torch()
    x = torch.from_numpy(synth.tokens(6, 2880, seed=10)).cuda()
    flat = moe32.forward(x)
    b = moe32.forward(x.reshape(2, 3, 2880))
    assert b.shape == (2, 3, 2880)
    assert torch.equal(b.reshape(6, 2880), flat)
    xb = x.to(torch.bfloat16)
    ob = moe32.forward(xb)
    assert ob.dtype == torch.bfloat16  # cast back to x's dtype (gpt_oss.rs:230)


def test_zero_tokens_is_a_no_op(moe32):
    torch = _torch()
    out = moe32.forward(torch.empty((0, 2880), device="cuda"))
    assert out.shape == (0, 2880)


def test_wrong_hidden_is_an_error(moe32):
    torch = _torch()
    with pytest.raises(GalliumError):
        moe32.forward(torch.zeros((2, 100), device="cuda"))


def test_misaligned_pointers_are_an_error(moe32):
    # the kernels copy x rows in 16-byte units: a pointer off that grid is
    # refused before any launch
    torch = _torch()
    buf = torch.zeros((4 * 2880 + 4,), device="cuda")
    out = torch.empty((4 * 2880 + 4,), device="cuda")
    with pytest.raises(GalliumError):
        moe32.forward_raw(buf.data_ptr() + 4, 4, out.data_ptr())
    with pytest.raises(GalliumError):
        moe32.forward_raw(buf.data_ptr(), 4, out.data_ptr() + 4)
    moe32.forward_raw(buf.data_ptr(), 4, out.data_ptr())  # aligned: runs
    torch.cuda.synchronize()


# ---- full-size properties (T = 4096, 20B shape) ------------------------------

@pytest.fixture(scope="module")
def big_run(moe32, layer32):
    torch = _torch()
    T = 4096
    x = synth.tokens(T, 2880, seed=4096)
    xc = _cuda(x)
    out1 = moe32.forward(xc)
    out2 = moe32.forward(xc)
    torch.cuda.synchronize()
    return x, xc, out1.cpu().numpy(), out2.cpu().numpy()


def test_full_size_is_deterministic(big_run):
    _, _, a, b = big_run
    assert np.array_equal(a, b)


def test_full_size_routing_bit_exact(moe32, layer32, big_run):
    x, xc, _, _ = big_run
    r = moe32.route(xc)
    _, idx, _, counts, offsets, perm = _route_oracle(layer32, x)
    assert np.array_equal(r["idx"].cpu().numpy(), idx)
    assert np.array_equal(r["perm"].cpu().numpy(), perm)
    assert int(r["counts"].sum()) == 4096 * 4


def test_full_size_sampled_rows_match_oracle(layer32, big_run):
    x, _, out, _ = big_run
    rows = np.random.default_rng(0).choice(4096, 24, replace=False)
    want, _, _ = oracle.OracleMoe(layer32).forward(x[rows])
    assert_parity(out[rows], want, "T=4096 sampled rows")


def test_full_size_rows_do_not_depend_on_the_batch(moe32, big_run):
    torch = _torch()
    _, xc, out, _ = big_run
    part = moe32.forward(xc[1000:1037]).cpu().numpy()
    assert_parity(part, out[1000:1037], "sub-batch vs full batch")


# ---- the 120B-shaped layer at its largest batch (E = 128, T = 8192) ------------

def test_120b_shape_at_8192_tokens():
    """The headline workload's shape: routing and grouping bit-exact on every
    token, sampled rows against the oracle, every row against the grouped
    CPU forward (oracle/cpu_reference.py, itself checked against the oracle),
    two forwards bit-identical."""
    torch = _torch()
    T = 8192
    layer = synth.gptoss_layer(n_experts=128, seed=0)
    x = synth.tokens(T, 2880, seed=8192)
    m = OssMoEFFN.load(layer, device=0, max_tokens=T)
    try:
        xc = _cuda(x)
        out1 = m.forward(xc).cpu().numpy()
        out2 = m.forward(xc).cpu().numpy()
        r = m.route(xc)
        torch.cuda.synchronize()
    finally:
        m.close()
    _, idx, _, counts, _, perm = _route_oracle(layer, x)
    assert np.array_equal(r["idx"].cpu().numpy(), idx)
    assert np.array_equal(r["counts"].cpu().numpy(), counts)
    assert np.array_equal(r["perm"].cpu().numpy(), perm)
    assert np.array_equal(out1, out2)
    rows = np.random.default_rng(1).choice(T, 24, replace=False)
    want, _, _ = oracle.OracleMoe(layer).forward(x[rows])
    assert_parity(out1[rows], want, "E=128 T=8192 sampled rows")
    assert_parity(out1, _cpu_grouped_forward(layer, x), "E=128 T=8192 every row")


def test_skewed_routing_at_4096_tokens(layer32_skew):
    """Zipf-skewed router bias (20B shape): the most popular experts take
    thousands of rows.  Routing bit-exact on every token; sampled rows, half of
    them routed to the most popular expert, against the oracle."""
    T = 4096
    x = synth.tokens(T, 2880, seed=4097)
    m = OssMoEFFN.load(layer32_skew, device=0, max_tokens=T)
    try:
        xc = _cuda(x)
        out = m.forward(xc).cpu().numpy()
        r = m.route(xc)
    finally:
        m.close()
    _, idx, _, counts, _, perm = _route_oracle(layer32_skew, x)
    assert np.array_equal(r["idx"].cpu().numpy(), idx)
    assert np.array_equal(r["counts"].cpu().numpy(), counts)
    assert np.array_equal(r["perm"].cpu().numpy(), perm)
    top = int(np.argmax(counts))
    assert counts[top] > T // 4  # the skew is real
    rng = np.random.default_rng(2)
    hot = rng.choice(np.nonzero((idx == top).any(axis=1))[0], 12, replace=False)
    rows = np.concatenate([hot, rng.choice(T, 12, replace=False)])
    want, _, _ = oracle.OracleMoe(layer32_skew).forward(x[rows])
    assert_parity(out[rows], want, "skewed T=4096 sampled rows")


# ---- tensor-core expert path (tcgen05) ---------------------------------------

# "tensor_cores": block-scaled MMA, MXFP4 weights as stored, E4M3 pieces;
# "tensor_cores_f16": weights decoded to f16 in shared memory, kind::f16.
TC_PATHS = ["tensor_cores", "tensor_cores_f16"]


@pytest.mark.parametrize("path", TC_PATHS)
@pytest.mark.parametrize("T", [1, 8, 64, 300])
def test_tensor_core_path_matches_oracle(moe32, layer32, T, path):
    x = synth.tokens(T, 2880, seed=500 + T)
    want, _, _ = oracle.OracleMoe(layer32).forward(x)
    moe32.set_expert_path(path)
    try:
        got = moe32.forward(_cuda(x)).cpu().numpy()
    finally:
        moe32.set_expert_path("auto")
    assert_parity(got, want, f"{path} T={T}")


@pytest.mark.parametrize("path", TC_PATHS)
def test_tensor_core_and_cuda_core_paths_agree(moe32, path):
    x = _cuda(synth.tokens(200, 2880, seed=42))
    moe32.set_expert_path("cuda_cores")
    a = moe32.forward(x).cpu().numpy()
    moe32.set_expert_path(path)
    b = moe32.forward(x).cpu().numpy()
    moe32.set_expert_path("auto")
    assert_parity(b, a, f"{path} vs cuda cores")


@pytest.mark.parametrize("path", TC_PATHS)
def test_tensor_core_path_skewed_and_gguf(layer32_skew, path):
    gg = synth.gptoss_gguf_from_split(layer32_skew)
    m = GptOssQMoEFFN.load(gg, device=0, max_tokens=256)
    try:
        m.set_expert_path(path)
        x = synth.tokens(256, 2880, seed=8)
        got = m.forward(_cuda(x)).cpu().numpy()
        want, _, _ = oracle.OracleMoe(layer32_skew, gguf=gg).forward(x)
        assert_parity(got, want, f"{path}, skewed, gguf")
    finally:
        m.close()


@pytest.mark.parametrize("path", TC_PATHS)
def test_tensor_core_path_handles_large_and_tiny_activations(moe32, layer32, path):
    # per-row power-of-two scaling keeps f16 hi/lo in range
    x = synth.tokens(64, 2880, seed=77)
    x[0] *= 3.0e4
    x[1] *= 1.0e-5
    want, _, _ = oracle.OracleMoe(layer32).forward(x)
    moe32.set_expert_path(path)
    try:
        got = moe32.forward(_cuda(x)).cpu().numpy()
    finally:
        moe32.set_expert_path("auto")
    assert_parity(got[2:], want[2:], f"{path}, ordinary rows")
    for r in (0, 1):
        err = np.abs(got[r] - want[r])
        assert err.sum() / np.abs(want[r]).sum() <= MEAN_REL, r


@pytest.mark.parametrize("T", [2, 16, 32, 64, 100, 300, 1000])
def test_block_scaled_every_tile_width(moe32, layer32, T):
    # 32 experts, top-4, mean T / 8 rows per expert: the tile holds 2, 4, 8
    # or 16 positions (twice the mean, rounded up to a power of two, while
    # the mean is at most 8), 30 up to a mean of 30, else 60 (T = 1000: two
    # full 60-position tiles and a short one per expert, whose MMAs are only
    # as wide as its rows)
    x = synth.tokens(T, 2880, seed=900 + T)
    want, _, _ = oracle.OracleMoe(layer32).forward(x)
    moe32.set_expert_path("tensor_cores")
    try:
        got = moe32.forward(_cuda(x)).cpu().numpy()
    finally:
        moe32.set_expert_path("auto")
    assert_parity(got, want, f"block-scaled T={T}")


def test_tensor_cores_on_odd_shapes():
    # H, I multiples of 64 but not of 128: partial M tiles on both GEMMs
    layer = synth.gptoss_layer(n_experts=8, hidden=320, inter=192, seed=12)
    m = OssMoEFFN.load(layer, device=0, max_tokens=40)
    try:
        for path in TC_PATHS:
            m.set_expert_path(path)
            x = synth.tokens(37, 320, seed=13)
            got = m.forward(_cuda(x)).cpu().numpy()
            want, _, _ = oracle.OracleMoe(layer).forward(x)
            assert_parity(got, want, f"{path}, H=320 I=192")
    finally:
        m.close()


# ---- forward graphs ---------------------------------------------------------

def test_graph_replay_equals_direct_launches(moe32, layer32):
    # the same buffers three times: launched directly, captured, replayed; new
    # contents of x between calls are read by the replay.  Batches that the
    # fused decode path runs as one launch are never captured (checked last).
    torch = _torch()
    for T in (1, 7, 64):
        xs = [synth.tokens(T, 2880, seed=400 + 10 * T + i) for i in range(3)]
        xd = torch.empty((T, 2880), device="cuda")
        out = torch.empty_like(xd)
        moe32.set_graphs(0)
        direct = []
        for x in xs:
            xd.copy_(torch.from_numpy(x))
            moe32.forward_raw(xd.data_ptr(), T, out.data_ptr())
            torch.cuda.synchronize()
            direct.append(out.cpu().numpy())
        moe32.set_graphs(16)
        c0 = moe32.info()["graph_captures"]
        for i, x in enumerate(xs * 2):
            xd.copy_(torch.from_numpy(x))
            moe32.forward_raw(xd.data_ptr(), T, out.data_ptr())
            moe32.device_status()
            assert np.array_equal(out.cpu().numpy(), direct[i % 3]), f"T={T} call {i}"
        assert moe32.info()["graph_captures"] - c0 == 1
        want, _, _ = oracle.OracleMoe(layer32).forward(xs[2])
        assert_parity(direct[2], want, f"graph T={T}")
    xd = _cuda(synth.tokens(8, 2880, seed=401))
    out = torch.empty_like(xd)
    moe32.set_expert_path("fused_decode")
    try:
        c0 = moe32.info()["graph_captures"]
        first = None
        for _ in range(3):
            moe32.forward_raw(xd.data_ptr(), 8, out.data_ptr())
            moe32.device_status()
            first = out.cpu().numpy() if first is None else first
            assert np.array_equal(out.cpu().numpy(), first)
        assert moe32.info()["graph_captures"] == c0
    finally:
        moe32.set_expert_path("auto")


def test_graph_cache_replaces_the_least_recently_used(moe32):
    torch = _torch()
    moe32.set_graphs(2)
    try:
        xd = _cuda(synth.tokens(16, 2880, seed=77))
        out = torch.empty_like(xd)
        ref = {}
        moe32.set_graphs(0)
        for T in (10, 12, 16):
            moe32.forward_raw(xd.data_ptr(), T, out.data_ptr())
            torch.cuda.synchronize()
            ref[T] = out[:T].cpu().numpy()
        moe32.set_graphs(2)
        c0 = moe32.info()["graph_captures"]
        for T in (10, 10, 12, 12, 16, 16, 10, 10):
            out.zero_()
            moe32.forward_raw(xd.data_ptr(), T, out.data_ptr())
            torch.cuda.synchronize()
            assert np.array_equal(out[:T].cpu().numpy(), ref[T]), f"T={T}"
        # 10, 12, 16 captured; 16 replaced 10, so 10 was seen again and captured again
        assert moe32.info()["graph_captures"] - c0 == 4
    finally:
        moe32.set_graphs(16)


@pytest.mark.parametrize("T", [1, 5, 127, 128, 129])
def test_one_launch_grouping_matches_oracle(layer32_skew, T):
    # up to 512 routing entries the grouping, tile table and activation pieces
    # come from one launch; 129 tokens x top-4 take the separate kernels (the
    # tensor-core path is forced, as AUTO would choose here)
    m = OssMoEFFN.load(layer32_skew, device=0, max_tokens=T)
    m.set_expert_path("tensor_cores")
    try:
        x = synth.tokens(T, 2880, seed=500 + T)
        got = m.forward(_cuda(x)).cpu().numpy()
        want, _, _ = oracle.OracleMoe(layer32_skew).forward(x)
        assert_parity(got, want, f"T={T}")
        # a second forward of other tokens in the same buffers
        x2 = synth.tokens(T, 2880, seed=600 + T)
        got2 = m.forward(_cuda(x2)).cpu().numpy()
        want2, _, _ = oracle.OracleMoe(layer32_skew).forward(x2)
        assert_parity(got2, want2, f"T={T} second")
    finally:
        m.close()
