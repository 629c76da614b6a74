"""The GPT-OSS decode stack (gb_decoder_*) on the GPU against the numpy
oracle of gpt_oss_q.rs (oracle/decoder_oracle.py): prompt logits within
max-abs 2e-2 / mean-rel 1e-3, and greedy decode giving the oracle's tokens
(the first divergence, if any, only at a near-tie of the oracle's logits).
Covers batch 1 and several sequences in lockstep, sliding-window layers past
their window, the CUDA-core and tensor-core linear layers (16 or more rows),
step-by-step forwards against the replayed decode graph, stage timing, and
the argument checks."""
import numpy as np
import pytest

from gallium_b200 import GalliumError, GptOssQ, _lib, synth
from oracle import decoder_oracle as dor

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_REL = 2e-2, 1e-3


def _weights(seed=0, layers=3):
    return synth.gptoss_decoder(n_layers=layers, hidden=256, n_heads=8, n_kv_heads=2,
                                head_dim=64, vocab=1000, n_experts=8, inter=256,
                                sliding_window=8, seed=seed)


def _close(got, want):
    err = np.abs(got.astype(np.float64) - want)
    return err.max(), err.sum() / np.abs(want).sum()


def _check_tokens(got, want, logits):
    """got / want (steps, B); logits (steps, B, vocab) of the oracle."""
    for b in range(got.shape[1]):
        for s in range(got.shape[0]):
            if got[s, b] != want[s, b]:
                row = logits[s, b]
                gap = abs(float(row[got[s, b]]) - float(row[want[s, b]]))
                assert gap < 5e-3, (b, s, got[s, b], want[s, b], gap)
                break  # the sequences diverge from here


@pytest.mark.parametrize("B,T", [(1, 12), (3, 12), (20, 4)])
def test_prompt_and_greedy_decode_match_the_oracle(B, T):
    import torch

    w = _weights(seed=B)
    steps = 10
    toks = np.random.default_rng(B).integers(0, w.vocab, (B, T)).astype(np.int32)
    orc = dor.OracleDecoder(w, max_seq_len=64)
    want_logits = orc.forward(toks, 0)
    want_first = dor.greedy(want_logits)
    want_toks, want_step_logits = orc.generate(want_first, T, steps)
    with GptOssQ.load(w, device=0, max_batch=B, max_tokens=T, max_seq_len=64) as m:
        got_logits = m.forward(torch.from_numpy(toks).cuda(), 0).cpu().numpy()
        mx, mr = _close(got_logits, want_logits)
        assert mx <= MAX_ABS and mr <= MEAN_REL, (mx, mr)
        first = m.last_next.cpu().numpy()
        assert np.array_equal(first, dor.greedy(got_logits))
        _check_tokens(first[None], want_first[None], want_logits[None])
        got_toks = m.generate(torch.from_numpy(want_first).cuda(), T, steps).cpu().numpy()
        _check_tokens(got_toks, want_toks, want_step_logits)


def test_replayed_steps_equal_step_by_step_forwards():
    """The replayed decode graph against eager forwards of one token."""
    import torch

    w = _weights(seed=7)
    B, T, steps = 2, 9, 6
    toks = np.random.default_rng(9).integers(0, w.vocab, (B, T)).astype(np.int32)
    with GptOssQ.load(w, device=0, max_batch=B, max_tokens=T, max_seq_len=32) as m:
        m.forward(torch.from_numpy(toks).cuda(), 0)
        start = m.last_next.clone()
        g = m.generate(start, T, steps).cpu().numpy()
        m.reset()
        m.forward(torch.from_numpy(toks).cuda(), 0)
        cur = start.reshape(B, 1)
        eager = []
        for s in range(steps):
            m.forward(cur, T + s)
            cur = m.last_next.reshape(B, 1).clone()
            eager.append(cur.reshape(-1).cpu().numpy())
        assert np.array_equal(g, np.stack(eager))
        # a second generate call replays the same captured graph
        m.reset()
        m.forward(torch.from_numpy(toks).cuda(), 0)
        g2 = m.generate(start, T, steps).cpu().numpy()
        assert np.array_equal(g, g2)


def test_stage_times_cover_attention_moe_and_head():
    import torch

    w = _weights(seed=4, layers=2)
    with GptOssQ.load(w, device=0, max_batch=1, max_tokens=4, max_seq_len=32) as m:
        m.set_profiling(True)
        m.forward(torch.zeros((1, 4), dtype=torch.int32).cuda(), 0)
        t = m.stage_times()
        assert t["attention"] > 0 and t["moe"] > 0 and t["head"] > 0


def test_argument_checks():
    import torch

    w = _weights(seed=5, layers=1)
    with GptOssQ.load(w, device=0, max_batch=2, max_tokens=4, max_seq_len=8) as m:
        x = torch.zeros((2, 4), dtype=torch.int32).cuda()
        with pytest.raises(GalliumError) as e:
            m.forward(x, 3)  # nothing cached yet
        assert e.value.status == _lib.GB_ERR_INVALID_ARG
        m.forward(x, 0)
        with pytest.raises(GalliumError):
            m.forward(x[:1], 4)  # the cache holds two sequences
        m.forward(x, 4)
        with pytest.raises(GalliumError):
            m.forward(x[:, :1], 8)  # past max_seq_len
        m.reset()
        bad = torch.full((2, 4), w.vocab, dtype=torch.int32).cuda()
        with pytest.raises(GalliumError) as e:
            m.forward(bad, 0)
        assert e.value.status == _lib.GB_ERR_INVALID_ARG


def test_greedy_token_ties_go_to_the_highest_id():
    """The greedy-token reduction on planted ties: an LM head whose rows are
    all equal gives equal logits, and an all-zero one gives +0 everywhere;
    either way the highest token id wins (sampling.rs:85-92)."""
    import torch

    w = _weights(seed=11, layers=1)
    toks = np.array([[3, 4, 5], [7, 8, 9]], np.int32)
    for head in (np.repeat(w.lm_head[17:18], w.vocab, axis=0), np.zeros_like(w.lm_head)):
        w.lm_head = np.ascontiguousarray(head)
        with GptOssQ.load(w, device=0, max_batch=2, max_tokens=3, max_seq_len=8) as m:
            got = m.forward(torch.from_numpy(toks).cuda(), 0).cpu().numpy()
            assert (got == got[:, :1]).all()
            assert list(m.last_next.cpu().numpy()) == [w.vocab - 1, w.vocab - 1]
