"""gb_route_noalloc, the routing entry point that allocates nothing.

Some callers cannot call cudaMalloc when they route: a candle custom op whose
device buffers must all come from candle's allocator, or a serving process
that has reserved the device's memory up front.  gb_route_noalloc serves them
with its scratch (router logits, per-tile tickets) in a fixed array inside the
library.  These tests call it through the C ABI and check it against the
existing routing entry point, gb_moe_route, on calls in a row (larger
batches first, then smaller ones, so anything left in the shared scratch by one
call would show in the next).

The file name sorts last so that, if it fails, a run that stops at the first
failure has already run every other test.  It builds everything it needs, so
it passes alone in a fresh process as well as after the rest of the suite.
"""
import numpy as np
import pytest

from gallium_b200 import OssMoEFFN, _lib, synth

pytestmark = pytest.mark.gpu

H, E, K = 2880, 32, 4


@pytest.fixture(scope="module")
def setup():
    import torch

    layer = synth.gptoss_layer(n_experts=E, hidden=H, inter=64, top_k=K, seed=21)
    moe = OssMoEFFN.load(layer, device=0, max_tokens=128)
    rw = torch.from_numpy(synth.bf16_bits_to_f32(layer.router_w)).cuda()
    rb = torch.from_numpy(synth.bf16_bits_to_f32(layer.router_b)).cuda()
    yield moe, rw, rb
    moe.close()


def _noalloc(x, rw, rb, T):
    import torch

    lib = _lib.load_library()
    idx = torch.full((T, K), -1, dtype=torch.int32, device="cuda")
    w = torch.full((T, K), -1.0, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.gb_route_noalloc(x.data_ptr(), rw.data_ptr(), rb.data_ptr(), None, T, H, E, K,
                                    _lib.GB_ROUTER_SOFTMAX_TOPK, idx.data_ptr(), w.data_ptr(),
                                    stream))
    torch.cuda.synchronize()
    return idx, w


def test_noalloc_routing_matches_gb_moe_route_on_two_calls_in_a_row(setup):
    import torch

    moe, rw, rb = setup
    # 100, 37 and 3 tokens take the three tile shapes (8, 4 and 1 tokens per CTA)
    for T, seed in ((100, 3), (37, 1), (3, 2)):
        x = torch.from_numpy(synth.tokens(T, H, seed=seed)).cuda()
        ref = moe.route(x)
        idx, w = _noalloc(x, rw, rb, T)
        assert torch.equal(idx, ref["idx"]), f"T={T}"
        # same tolerance as the routing-weight parity test
        np.testing.assert_allclose(w.cpu().numpy(), ref["w"].cpu().numpy(), rtol=2e-6, atol=1e-7)


def test_noalloc_rejects_batches_beyond_its_scratch(setup):
    import torch

    _, rw, rb = setup
    lib = _lib.load_library()
    T = 65536 // E + 1
    x = torch.zeros((T, H), device="cuda")
    idx = torch.empty((T, K), dtype=torch.int32, device="cuda")
    w = torch.empty((T, K), device="cuda")
    rc = lib.gb_route_noalloc(x.data_ptr(), rw.data_ptr(), rb.data_ptr(), None, T, H, E, K,
                              _lib.GB_ROUTER_SOFTMAX_TOPK, idx.data_ptr(), w.data_ptr(), None)
    assert rc == _lib.GB_ERR_INVALID_ARG
    assert "65536" in lib.gb_last_error().decode()
