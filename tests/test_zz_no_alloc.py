"""gb_route_noalloc, the routing entry point that allocates nothing.

Some callers cannot call cudaMalloc when they route: a candle custom op whose
device buffers must all come from candle's allocator, or a serving process
that has reserved the device's memory up front.  gb_route_noalloc serves them
with its scratch (router logits, per-tile tickets) in a fixed array inside the
library.  These tests call it through the C ABI and check it against the
existing routing entry point, gb_moe_route, on calls in a row (larger
batches first, then smaller ones, so anything left in the shared scratch by one
call would show in the next).  Both entry points end in the same selection
code and compute the logits in the same order, so indices and weights must be
bit-identical, whichever kernel shape each one picks for a batch (at 2048
tokens gb_route_noalloc runs its 8-token tiles, gb_moe_route its 32-token
tiled kernel).

The file name sorts last so that, if it fails, a run that stops at the first
failure has already run every other test.  It builds everything it needs, so
it passes alone in a fresh process as well as after the rest of the suite.
"""
import numpy as np
import pytest

from gallium_b200 import Lfm2QMoEFFN, OssMoEFFN, _lib, synth

pytestmark = pytest.mark.gpu

# (name, router kind, experts, hidden, token counts of the calls in a row)
CASES = [
    ("softmax-e32", _lib.GB_ROUTER_SOFTMAX_TOPK, 32, 2880, (2048, 100, 37, 3)),
    ("softmax-e128", _lib.GB_ROUTER_SOFTMAX_TOPK, 128, 2880, (512, 300, 7)),
    ("sigmoid-bias-e32", _lib.GB_ROUTER_SIGMOID_TOPK, 32, 2048, (2048, 64, 5)),
    ("sigmoid-nobias-e32", _lib.GB_ROUTER_SIGMOID_TOPK, 32, 2048, (100, 2)),
]
K = 4


def _setup(kind, E, H, T_max, with_bias):
    import torch

    if kind == _lib.GB_ROUTER_SOFTMAX_TOPK:
        layer = synth.gptoss_layer(n_experts=E, hidden=H, inter=64, top_k=K, seed=21)
        moe = OssMoEFFN.load(layer, device=0, max_tokens=T_max)
        rw = torch.from_numpy(synth.bf16_bits_to_f32(layer.router_w)).cuda()
        rb = torch.from_numpy(synth.bf16_bits_to_f32(layer.router_b)).cuda()
        sb = None
    else:
        layer = synth.lfm2_layer(n_experts=E, hidden=H, inter=256, top_k=K, seed=22)
        # a selection bias that changes some selections, or none (zeros)
        layer.sel_bias = (np.random.default_rng(5).normal(0, 0.05, E).astype(np.float32)
                          if with_bias else None)
        moe = Lfm2QMoEFFN.load(layer, device=0, max_tokens=T_max)
        rw = torch.from_numpy(np.ascontiguousarray(layer.router_w, np.float32)).cuda()
        rb = None
        sb = torch.from_numpy(layer.sel_bias).cuda() if with_bias else None
    return moe, rw, rb, sb


def _noalloc(x, rw, rb, sb, T, H, E, kind):
    import torch

    lib = _lib.load_library()
    idx = torch.full((T, K), -1, dtype=torch.int32, device="cuda")
    w = torch.full((T, K), -1.0, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.gb_route_noalloc(x.data_ptr(), rw.data_ptr(),
                                    None if rb is None else rb.data_ptr(),
                                    None if sb is None else sb.data_ptr(), T, H, E, K, kind,
                                    idx.data_ptr(), w.data_ptr(), stream))
    torch.cuda.synchronize()
    return idx, w


@pytest.mark.parametrize("name,kind,E,H,Ts", CASES, ids=[c[0] for c in CASES])
def test_noalloc_routing_matches_gb_moe_route_on_calls_in_a_row(name, kind, E, H, Ts):
    import torch

    moe, rw, rb, sb = _setup(kind, E, H, max(Ts), with_bias=name != "sigmoid-nobias-e32")
    try:
        for i, T in enumerate(Ts):
            x = torch.from_numpy(synth.tokens(T, H, seed=40 + i)).cuda()
            ref = moe.route(x)
            idx, w = _noalloc(x, rw, rb, sb, T, H, E, kind)
            assert torch.equal(idx, ref["idx"]), f"{name} T={T}"
            assert torch.equal(w, ref["w"]), f"{name} T={T}"
    finally:
        moe.close()


def test_noalloc_rejects_batches_beyond_its_scratch():
    import torch

    E, H = 32, 2880
    lib = _lib.load_library()
    T = 65536 // E + 1
    x = torch.zeros((T, H), device="cuda")
    rw = torch.zeros((E, H), device="cuda")
    idx = torch.empty((T, K), dtype=torch.int32, device="cuda")
    w = torch.empty((T, K), device="cuda")
    rc = lib.gb_route_noalloc(x.data_ptr(), rw.data_ptr(), None, None, T, H, E, K,
                              _lib.GB_ROUTER_SOFTMAX_TOPK, idx.data_ptr(), w.data_ptr(), None)
    assert rc == _lib.GB_ERR_INVALID_ARG
    assert "65536" in lib.gb_last_error().decode()
    # an x that does not start on a 16-byte boundary is refused, not read
    rc = lib.gb_route_noalloc(x.data_ptr() + 4, rw.data_ptr(), None, None, 8, H, E, K,
                              _lib.GB_ROUTER_SOFTMAX_TOPK, idx.data_ptr(), w.data_ptr(), None)
    assert rc == _lib.GB_ERR_INVALID_ARG
    assert "16-byte" in lib.gb_last_error().decode()
