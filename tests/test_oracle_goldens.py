"""Pins the CPU oracle before it is trusted as the checker.

1. The reference's own MXFP4 GGUF decoder goldens, ported one for one from
   crates/gallium-core/src/quantized.rs:917-1010.
2. Known-answer cases the reference does not pin (safetensors nibble order,
   Q4_K, activation clamps, router tie-break, grouping order), and the Q4_K
   and GGUF MXFP4 decoders against gguf-py 0.19.0 (llama.cpp's Python
   implementation of the GGML formats) on the committed fixture
   tests/golden/ggml_decode_goldens.npz.
3. The whole-block oracle against an independent float64 numpy restatement
   of gpt_oss.rs:166-231 at a small shape.
"""
import os

import numpy as np
import pytest

import oracle
from gallium_b200 import synth

LUT2 = [0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12]  # quantized.rs:370
E2M1 = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0]


# ---- 1. quantized.rs:917-1010 ---------------------------------------------

def test_an_e8m0_byte_of_128_is_unit_scale():  # quantized.rs:921-928
    assert oracle.e8m0_to_f32(128) == 1.0
    assert oracle.e8m0_to_f32(129) == 2.0
    assert oracle.e8m0_to_f32(127) == 0.5


def test_one_block_dequantizes_in_the_documented_nibble_order():  # :930-948
    raw = np.array([128] + [j | (j << 4) for j in range(16)], np.uint8)
    out = oracle.mxfp4_gguf_dequant(raw, 32)
    assert out.shape == (32,)
    for j in range(16):
        assert out[j] == LUT2[j], f"low nibble of byte {j}"
        assert out[j + 16] == LUT2[j], f"high nibble of byte {j}"


def test_every_element_of_a_multi_block_tensor_is_written():  # :950-971
    raw = np.array(([128] + [0x11] * 16) * 3, np.uint8)
    out = oracle.mxfp4_gguf_dequant(raw, 96)
    assert out.shape == (96,)
    assert np.all(out == 1.0)


def test_a_ragged_expert_count_is_an_error_rather_than_a_short_read():  # :973-984
    with pytest.raises(oracle.OracleError):
        oracle.mxfp4_blocks_per_expert(33)
    with pytest.raises(oracle.OracleError):
        oracle.mxfp4_blocks_per_expert(31)
    assert oracle.mxfp4_blocks_per_expert(32) == 1
    assert oracle.mxfp4_blocks_per_expert(128) == 4


def test_the_ragged_expert_error_names_the_count_and_the_block_size():  # :986-993
    with pytest.raises(oracle.OracleError) as ei:
        oracle.mxfp4_blocks_per_expert(100)
    assert "100" in str(ei.value)
    assert "32" in str(ei.value)


def test_negative_codes_and_a_non_unit_scale_survive_dequant():  # :995-1010
    raw = np.array([129] + [0xF7] * 16, np.uint8)
    out = oracle.mxfp4_gguf_dequant(raw, 32)
    for j in range(16):
        assert out[j] == 24.0
        assert out[j + 16] == -24.0


def test_e8m0_small_bytes_are_the_subnormals_of_quantized_rs_375_383():
    assert oracle.e8m0_to_f32(0) == 2.0 ** -128
    assert oracle.e8m0_to_f32(1) == 2.0 ** -127
    assert oracle.e8m0_to_f32(2) == 2.0 ** -126
    assert oracle.e8m0_to_f32(254) == 2.0 ** 126


# ---- 2. known answers the reference does not pin --------------------------

def test_safetensors_nibble_order_golden():
    # gpt_oss.rs:156-159: byte j -> elements 2j (low) and 2j+1 (high).
    blocks = np.full((1, 1, 16), 0x21, np.uint8)
    scales = np.full((1, 1), 127, np.uint8)  # 2^0
    out = oracle.mxfp4_split_dequant(blocks, scales)[0]
    assert np.all(out[0::2] == 0.5) and np.all(out[1::2] == 1.0)
    # every code, both halves, non-unit scale
    blocks = np.array([[[j | ((15 - j) << 4) for j in range(16)]]], np.uint8)
    scales = np.array([[130]], np.uint8)  # 2^3
    out = oracle.mxfp4_split_dequant(blocks, scales)[0]
    for j in range(16):
        assert out[2 * j] == E2M1[j] * 8
        assert out[2 * j + 1] == E2M1[15 - j] * 8


def test_safetensors_scale_zero_is_zero_and_gguf_scale_zero_is_tiny():
    blocks = np.full((1, 1, 16), 0x77, np.uint8)
    out = oracle.mxfp4_split_dequant(blocks, np.zeros((1, 1), np.uint8))[0]
    assert np.all(out == 0.0)
    raw = np.array([0] + [0x77] * 16, np.uint8)
    g = oracle.mxfp4_gguf_dequant(raw, 32)
    assert np.all(g == np.float32(12 * 2.0 ** -128))


def test_split_and_gguf_views_of_a_layer_decode_identically():
    layer = synth.gptoss_layer(n_experts=2, hidden=64, inter=64, seed=3)
    gg = synth.gptoss_gguf_from_split(layer)
    for e in range(2):
        gu = oracle.mxfp4_split_dequant(layer.gu_blocks[e], layer.gu_scales[e])
        g = oracle.mxfp4_gguf_dequant(gg.gate_raw[e], 64 * 64).reshape(64, 64)
        u = oracle.mxfp4_gguf_dequant(gg.up_raw[e], 64 * 64).reshape(64, 64)
        assert np.array_equal(gu[0::2], g)
        assert np.array_equal(gu[1::2], u)


def _f16(v):
    return np.float16(v).view(np.uint16)


def _q4k_numpy(raw, n):
    """Independent restatement of the GGML Q4_K block layout."""
    out = []
    for b in range(n // 256):
        blk = raw[b * 144:(b + 1) * 144]
        d = np.frombuffer(blk[0:2].tobytes(), np.float16)[0].astype(np.float32)
        dm = np.frombuffer(blk[2:4].tobytes(), np.float16)[0].astype(np.float32)
        s = blk[4:16].astype(np.int64)
        q = blk[16:144]
        sc, mn = [], []
        for j in range(8):
            if j < 4:
                sc.append(s[j] & 63)
                mn.append(s[j + 4] & 63)
            else:
                sc.append((s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4))
                mn.append((s[j + 4] >> 4) | ((s[j] >> 6) << 4))
        for c in range(4):
            qq = q[32 * c:32 * c + 32]
            for half, j in ((qq & 0xF, 2 * c), (qq >> 4, 2 * c + 1)):
                dd = np.float32(d * np.float32(sc[j]))
                mm = np.float32(dm * np.float32(mn[j]))
                out.append(dd * half.astype(np.float32) - mm)
    return np.concatenate(out).astype(np.float32)


def test_q4k_decoder_matches_an_independent_restatement():
    rng = np.random.default_rng(7)
    raw = rng.integers(0, 256, 144 * 3, dtype=np.uint8)
    for b in range(3):  # finite, positive d / dmin
        raw[b * 144:b * 144 + 2] = np.frombuffer(_f16(2.0 ** -9 * (b + 1)).tobytes(), np.uint8)
        raw[b * 144 + 2:b * 144 + 4] = np.frombuffer(_f16(2.0 ** -8).tobytes(), np.uint8)
    got = oracle.q4k_dequant(raw, 768)
    want = _q4k_numpy(raw, 768)
    assert np.array_equal(got, want)


def test_q4k_known_answer():
    blk = np.zeros(144, np.uint8)
    blk[0:2] = np.frombuffer(_f16(1.0).tobytes(), np.uint8)   # d
    blk[2:4] = np.frombuffer(_f16(0.5).tobytes(), np.uint8)   # dmin
    blk[4:8] = [1, 2, 3, 4]        # sc0..3
    blk[8:12] = [0, 1, 2, 3]       # m0..3
    blk[12:16] = [0x21, 0x43, 0x65, 0x07]  # sc4..7 low nibbles, m4..7 high nibbles
    blk[16:144] = 0x53              # low nibble 3, high nibble 5
    out = oracle.q4k_dequant(blk, 256)
    sc = [1, 2, 3, 4, 1, 3, 5, 7]
    mn = [0, 1, 2, 3, 2, 4, 6, 0]
    for j in range(8):
        q = 3 if j % 2 == 0 else 5
        assert np.all(out[32 * j:32 * j + 32] == np.float32(sc[j] * q - 0.5 * mn[j])), j


GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden",
                      "ggml_decode_goldens.npz")


def test_q4k_decoder_matches_gguf_py_goldens():
    """Q4_K, pinned bit for bit against gguf-py's decode of the same blocks
    (tests/golden/make_ggml_goldens.py): zero, subnormal, negative and large
    f16 d / dmin included."""
    z = np.load(GOLDEN)
    got = oracle.q4k_dequant(z["q4k_blocks"].reshape(-1), z["q4k_values"].size)
    assert np.array_equal(got.view(np.uint32), z["q4k_values"].view(np.uint32))


def test_gguf_mxfp4_decoder_matches_gguf_py_goldens():
    """GGUF MXFP4 for every E8M0 byte 0..255, bit for bit against gguf-py."""
    z = np.load(GOLDEN)
    with np.errstate(over="ignore"):
        got = oracle.mxfp4_gguf_dequant(z["mxfp4_blocks"].reshape(-1), z["mxfp4_values"].size)
    assert np.array_equal(got.view(np.uint32), z["mxfp4_values"].view(np.uint32))


def test_q4k_ragged_is_an_error():
    with pytest.raises(oracle.OracleError):
        oracle.q4k_dequant(np.zeros(144, np.uint8), 200)


def test_gptoss_activation_clamps():
    lim = 7.0
    sig = lambda v: (np.tanh(np.float32(v) * np.float32(0.851)) + 1) * 0.5
    # gate clamped above only; up clamped to [-7, 7] and shifted by one
    for g, u in [(7.5, 0.0), (7.0, 1.0), (6.999, 7.001), (-20.0, -9.0), (3.0, -7.5), (0.0, 0.0)]:
        gc = min(g, lim)
        uc = min(max(u, -lim), lim)
        want = gc * sig(gc) * (uc + 1)
        assert oracle.act_gptoss(g, u, lim) == pytest.approx(want, rel=1e-6, abs=1e-6)
    assert oracle.act_gptoss(100.0, 100.0, lim) == oracle.act_gptoss(7.0, 7.0, lim)
    assert oracle.act_gptoss(7.0 + 1e-3, 2.0, lim) == oracle.act_gptoss(7.0, 2.0, lim)
    assert oracle.act_gptoss(1.0, -7.0 - 1e-3, lim) == oracle.act_gptoss(1.0, -7.0, lim)
    assert oracle.act_silu(0.0, 5.0) == 0.0
    assert oracle.act_silu(2.0, 3.0) == pytest.approx(2.0 / (1 + np.exp(-2.0)) * 3.0, rel=1e-6)


def test_router_tie_break_prefers_the_lower_index():
    logits = np.array([[1.0, 3.0, 3.0, 2.0, 3.0]], np.float32)
    idx, w = oracle.route_softmax_topk(logits, 3)
    assert idx.tolist() == [[1, 2, 4]]
    assert np.allclose(w, 1.0 / 3.0)
    idx, w = oracle.route_sigmoid_topk(logits, np.zeros(5, np.float32), 2)
    assert idx.tolist() == [[1, 2]]
    # the selection bias steers selection only (lfm2moe_q.rs:246-257)
    idx, w = oracle.route_sigmoid_topk(logits, np.array([0, 0, 0, 5, 0], np.float32), 2)
    assert idx.tolist() == [[3, 1]]
    p = 1 / (1 + np.exp(-np.array([2.0, 3.0])))
    assert np.allclose(w[0], p / p.sum(), rtol=1e-6)


def test_router_logits_fixed_reduction_order():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((3, 96)).astype(np.float32)
    w = rng.standard_normal((5, 96)).astype(np.float32)
    b = rng.standard_normal(5).astype(np.float32)
    got = oracle.router_logits(x, w, b)
    # restate: 32 strided partial sums with FMA (float64 product rounded once),
    # butterfly, bias
    want = np.empty((3, 5), np.float32)
    for t in range(3):
        for e in range(5):
            part = np.zeros(32, np.float32)
            for l in range(32):
                acc = np.float32(0)
                for kk in range(l, 96, 32):
                    acc = np.float32(np.float64(x[t, kk]) * np.float64(w[e, kk]) + np.float64(acc))
                part[l] = acc
            for s in (16, 8, 4, 2, 1):
                part = np.array([part[l] + part[l ^ s] for l in range(32)], np.float32)
            want[t, e] = part[0] + b[e]
    assert np.array_equal(got, want)


def test_grouping_order_is_expert_then_token():
    idx = np.array([[2, 0], [0, 1], [2, 1], [3, 0]], np.int32)
    counts, offsets, perm, inv = oracle.permute(idx, 5)
    assert counts.tolist() == [3, 2, 2, 1, 0]
    assert offsets.tolist() == [0, 3, 5, 7, 8, 8]
    # expert 0: tokens 0 (r1), 1 (r0), 3 (r1); expert 1: 1 (r1), 2 (r1); 2: 0, 2; 3: 3
    assert perm.tolist() == [1, 2, 7, 3, 5, 0, 4, 6]
    for pos, ent in enumerate(perm):
        assert inv[ent] == pos


# ---- 3. whole block vs an independent float64 restatement -----------------

def _numpy_block(layer, x):
    """gpt_oss.rs:166-231 in float64 numpy."""
    H, I, E, k = layer.hidden, layer.inter, layer.n_experts, layer.top_k
    bf = synth.bf16_bits_to_f32

    def deq(blocks, scales):
        lo = np.array(E2M1)[blocks & 0xF]
        hi = np.array(E2M1)[blocks >> 4]
        v = np.empty(blocks.shape[:-1] + (32,))
        v[..., 0::2], v[..., 1::2] = lo, hi
        sc = np.where(scales == 0, 0.0, 2.0 ** (scales.astype(np.float64) - 127))
        v = v * sc[..., None]
        return v.reshape(v.shape[0], -1)

    logits = x.astype(np.float64) @ bf(layer.router_w).astype(np.float64).T + bf(layer.router_b)
    out = np.zeros((x.shape[0], H))
    for t in range(x.shape[0]):
        order = sorted(range(E), key=lambda e: (-logits[t, e], e))[:k]
        ex = np.exp(logits[t, order] - logits[t, order[0]])
        wts = ex / ex.sum()
        for e, wv in zip(order, wts):
            gu = deq(layer.gu_blocks[e], layer.gu_scales[e]) @ x[t] + bf(layer.gu_bias[e])
            g, u = gu[0::2], gu[1::2]
            g = np.minimum(g, 7.0)
            u = np.clip(u, -7.0, 7.0)
            h = g * (1 / (1 + np.exp(-1.702 * g))) * (u + 1)
            y = deq(layer.dn_blocks[e], layer.dn_scales[e]) @ h + bf(layer.dn_bias[e])
            out[t] += wv * y
    return out, logits


@pytest.mark.parametrize("i", [0, 5, 33, 63])
def test_one_hot_input_through_one_expert_by_hand(i):
    # unit scales (E8M0 127), zero biases, x = e_i: gate_up row j is the E2M1
    # value of its code at column i, so the expert's output follows from the
    # code table alone (gpt_oss.rs:189-221)
    layer = synth.gptoss_layer(n_experts=2, hidden=64, inter=32, top_k=1, seed=4)
    layer.gu_scales[:] = 127
    layer.dn_scales[:] = 127
    layer.gu_bias[:] = 0
    layer.dn_bias[:] = 0
    H, I = layer.hidden, layer.inter

    def code(blocks, row, col):
        byte = blocks[row, col // 32, (col % 32) // 2]
        return E2M1[(byte >> 4) if col % 2 else (byte & 0xF)]

    gu = np.array([code(layer.gu_blocks[1], j, i) for j in range(2 * I)])
    g, u = np.minimum(gu[0::2], 7.0), np.clip(gu[1::2], -7.0, 7.0)
    h = g / (1.0 + np.exp(-1.702 * g)) * (u + 1.0)
    w_dn = np.array([[code(layer.dn_blocks[1], r, c) for c in range(I)] for r in range(H)])
    want = w_dn @ h
    x = np.zeros((1, H), np.float32)
    x[0, i] = 1.0
    got = oracle.OracleMoe(layer).expert_ffn(1, x)[0]
    assert np.abs(got - want).max() <= 1e-5 * max(1.0, np.abs(want).max())


@pytest.mark.parametrize("skewed", [False, True])
def test_oracle_block_matches_float64_restatement(skewed):
    layer = synth.gptoss_layer(n_experts=8, hidden=128, inter=96, top_k=2, seed=11, skewed=skewed)
    x = synth.tokens(6, 128, seed=5)
    got, idx, w = oracle.OracleMoe(layer).forward(x)
    want, logits = _numpy_block(layer, x)
    for t in range(6):
        assert idx[t].tolist() == sorted(range(8), key=lambda e: (-logits[t, e], e))[:2]
    err = np.abs(got - want)
    assert err.max() <= 2e-3 * max(1.0, np.abs(want).max())
    assert err.sum() / np.abs(want).sum() < 1e-5


def test_oracle_gguf_view_matches_split():
    layer = synth.gptoss_layer(n_experts=4, hidden=64, inter=64, top_k=2, seed=2)
    gg = synth.gptoss_gguf_from_split(layer)
    x = synth.tokens(5, 64, seed=9)
    a, ia, wa = oracle.OracleMoe(layer).forward(x)
    b, ib, wb = oracle.OracleMoe(layer, gguf=gg).forward(x)
    assert np.array_equal(ia, ib)
    # same values; the GGUF path only changes the combine order (expert ascending)
    assert np.allclose(a, b, rtol=1e-5, atol=1e-4)


# ---- LFM2.5 (Q4_K, sigmoid router, SiLU) vs a float64 restatement ----------

def _numpy_lfm2(layer, x):
    """lfm2moe_q.rs:234-313 in float64 numpy, Q4_K decoded by _q4k_numpy."""
    H, I, E, k = layer.hidden, layer.inter, layer.n_experts, layer.top_k
    logits = x.astype(np.float64) @ layer.router_w.astype(np.float64).T
    p = 1 / (1 + np.exp(-logits))
    out = np.zeros((x.shape[0], H))
    for t in range(x.shape[0]):
        order = sorted(range(E), key=lambda e: (-(p[t, e] + layer.sel_bias[e]), e))[:k]
        wts = p[t, order] / p[t, order].sum()
        # combine in ascending expert order (lfm2moe_q.rs:303-311)
        for e, wv in sorted(zip(order, wts)):
            g = _q4k_numpy(layer.gate_raw[e].ravel(), I * H).reshape(I, H) @ x[t]
            u = _q4k_numpy(layer.up_raw[e].ravel(), I * H).reshape(I, H) @ x[t]
            h = g / (1 + np.exp(-g)) * u
            y = _q4k_numpy(layer.down_raw[e].ravel(), H * I).reshape(H, I) @ h
            out[t] += wv * y
    return out


def test_oracle_lfm2_block_matches_float64_restatement():
    layer = synth.lfm2_layer(n_experts=6, hidden=256, inter=256, top_k=3, seed=5)
    layer.sel_bias[:] = np.array([0, 0.3, 0, 0, -0.2, 0], np.float32)
    x = synth.tokens(4, 256, seed=6)
    got, idx, w = oracle.OracleLfm2(layer).forward(x)
    want = _numpy_lfm2(layer, x)
    err = np.abs(got - want)
    assert err.max() <= 1e-3 * max(1.0, np.abs(want).max())
    assert err.sum() / np.abs(want).sum() < 1e-5
    assert np.allclose(w.sum(axis=1), 1.0, atol=1e-6)
