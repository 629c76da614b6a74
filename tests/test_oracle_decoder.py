"""The decode-stack oracle (oracle/decoder_oracle.py) on the host: the
reference's own mask tests (crates/gallium-core/src/mask.rs:62-129) ported
to the oracle's visibility rule, the YaRN frequencies against an independent
restatement of pos_enc.rs:113-137, the greedy tie rule of sampling.rs:85-92,
the sink softmax, and KV-cache consistency (a prompt in one forward, or
token by token, gives the same logits)."""
import math

import numpy as np

from gallium_b200 import synth
from oracle import decoder_oracle as dor


def test_causal_visibility_matches_the_reference_mask_tests():
    # build_causal_mask(3, 0): row 0 sees [0], row 2 sees 0, 1, 2
    assert list(dor.visible(0, 3, False, 128)) == [True, False, False]
    assert list(dor.visible(2, 3, False, 128)) == [True, True, True]


def test_sliding_window_at_decode_bounds_a_single_query():
    # build_sliding_window_mask(1, 9, 4): positions 6..=9 visible
    row = dor.visible(9, 10, True, 4)
    assert list(np.nonzero(row)[0]) == [6, 7, 8, 9]


def test_sliding_window_inside_the_window_sees_everything():
    # build_sliding_window_mask(1, 3, 8): all four visible
    assert dor.visible(3, 4, True, 8).all()


def test_sliding_window_prefill_rows():
    # build_sliding_window_mask(4, 0, 2)
    assert list(dor.visible(0, 4, True, 2)) == [True, False, False, False]
    assert list(dor.visible(2, 4, True, 2)) == [False, True, True, False]
    assert list(dor.visible(3, 4, True, 2)) == [False, False, True, True]


def test_yarn_frequencies_follow_the_three_bands():
    """GPT-OSS's RoPE (theta 150000, YaRN factor 32 from a 4096 context,
    betas 32 / 1): high-frequency dimensions keep 1/theta^(2i/d), dimensions
    whose wavelength ratio is above high/d are divided by the factor, the
    ones between scaled by 1 / (1 + (factor - 1) t), t = (i - low) / (high - low)."""
    d, theta, factor, ctx = 64, 150000.0, 32.0, 4096
    inv = dor.rope_inv_freq(d, theta, factor, ctx)
    low, high = math.floor(ctx / (32 * 2 * math.pi)), math.floor(ctx / (2 * math.pi))
    assert (low, high) == (20, 651)
    for i in range(d // 2):
        base = 1.0 / theta ** (2.0 * i / d)
        ratio = 2 * math.pi / base / ctx
        if ratio < low / d:
            want = base
        elif ratio > high / d:
            want = base / factor
        else:
            want = base * (1.0 / (1 + (factor - 1) * (i - low) / (high - low)))
        assert inv[i] == want, i
    assert inv[0] == 1.0 and inv[31] == (1.0 / theta ** (62 / 64)) / factor


def test_greedy_takes_the_last_of_equal_maxima():
    lg = np.array([[1.0, 3.0, 3.0, -1.0], [5.0, 5.0, 5.0, 5.0], [0.0, 2.0, 1.0, 2.0]], np.float32)
    assert list(dor.greedy(lg)) == [2, 3, 3]


def test_rms_norm_sums_in_order():
    x = np.array([[3.0, 4.0]], np.float32)
    w = np.array([1.0, 2.0], np.float32)
    got = dor.rms_norm(x, w, 0.0)
    m = np.float32(math.sqrt(12.5))
    assert np.array_equal(got, np.array([[3.0 / m, (4.0 / m) * 2.0]], np.float32))


def _small(seed=0, layers=2):
    return synth.gptoss_decoder(n_layers=layers, hidden=128, n_heads=4, n_kv_heads=2,
                                head_dim=32, vocab=300, n_experts=8, inter=128,
                                sliding_window=4, seed=seed)


def test_sink_softmax_keeps_the_sink_mass_out_of_the_output():
    """With one visible key and its value v, the output is v * p where
    p = 1 / (1 + e^(sink - score)) (gpt_oss_q.rs:92-101)."""
    w = _small()
    o = dor.OracleDecoder(w, max_seq_len=16)
    L = w.layers[0]
    x = np.random.default_rng(1).standard_normal((1, 1, w.hidden)).astype(np.float32)
    xn = dor.rms_norm(x, L.attn_norm, w.rms_eps)
    P = o.lw[0]
    q = o._linear(xn, P["wq"], L.bq)[0, 0].reshape(w.n_heads, w.head_dim)
    k = o._linear(xn, P["wk"], L.bk)[0, 0].reshape(w.n_kv_heads, w.head_dim)
    v = o._linear(xn, P["wv"], L.bv)[0, 0].reshape(w.n_kv_heads, w.head_dim)
    q = dor.rope(q[:, None], o.cos[:1], o.sin[:1])[:, 0]
    k = dor.rope(k[:, None], o.cos[:1], o.sin[:1])[:, 0]
    att = np.empty(w.n_heads * w.head_dim, np.float64)
    for h in range(w.n_heads):
        g = h // (w.n_heads // w.n_kv_heads)
        s = float(np.dot(q[h].astype(np.float64), k[g])) / math.sqrt(w.head_dim)
        p = 1.0 / (1.0 + math.exp(float(L.sinks[h]) - s))
        att[h * w.head_dim:(h + 1) * w.head_dim] = p * v[g]
    want = att @ dor.bf16(L.wo).T.astype(np.float64) + L.bo
    got = o._attention(0, xn, 0)[0, 0]
    assert np.allclose(got, want, rtol=1e-4, atol=1e-5)


def test_prompt_at_once_equals_token_by_token():
    w = _small(seed=3, layers=3)
    toks = np.random.default_rng(2).integers(0, w.vocab, (2, 7))
    a = dor.OracleDecoder(w, max_seq_len=16)
    la = a.forward(toks, 0)
    b = dor.OracleDecoder(w, max_seq_len=16)
    for t in range(7):
        lb = b.forward(toks[:, t:t + 1], t)
    assert np.allclose(la, lb, rtol=1e-4, atol=1e-4)
