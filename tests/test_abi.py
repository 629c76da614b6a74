"""The C ABI surface, checked without a GPU: the library loads, exports every
function include/gallium_b200.h declares, the ctypes mirrors of the structs
match the C layout, and descriptor validation answers with status codes
(INVALID_ARG / SHAPE / UNSUPPORTED) before any device work."""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

from gallium_b200 import _lib, synth
from gallium_b200._lib import MoeDesc, MoeInfo

HEADER = _lib.HEADER_PATH


def _declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gb_[a-z_0-9]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load_library()
    names = _declared_functions()
    assert len(names) >= 10
    for n in names:
        assert hasattr(lib, n), f"{n} declared in the header but not exported"
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"
    assert lib.gb_abi_version() == 4


def test_struct_layouts_match_the_header(tmp_path):
    fields_d = [f for f, _ in MoeDesc._fields_]
    fields_i = [f for f, _ in MoeInfo._fields_]
    src = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', 'int main(void){']
    src.append('printf("%zu\\n", sizeof(gb_moe_desc));')
    for f in fields_d:
        src.append(f'printf("%zu\\n", offsetof(gb_moe_desc, {f}));')
    src.append('printf("%zu\\n", sizeof(gb_moe_info));')
    for f in fields_i:
        src.append(f'printf("%zu\\n", offsetof(gb_moe_info, {f}));')
    src.append("return 0;}")
    c = tmp_path / "layout.c"
    c.write_text("\n".join(src))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", str(c), "-o", str(exe)], check=True)
    vals = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True,
                                           check=True).stdout.split()]
    want = [ctypes.sizeof(MoeDesc)] + [getattr(MoeDesc, f).offset for f in fields_d]
    want += [ctypes.sizeof(MoeInfo)] + [getattr(MoeInfo, f).offset for f in fields_i]
    assert vals == want


def _desc(**kw):
    d = MoeDesc()
    d.struct_size = ctypes.sizeof(MoeDesc)
    d.hidden, d.inter, d.n_experts, d.top_k = 64, 64, 4, 2
    d.weight_format = _lib.GB_FMT_MXFP4_SPLIT
    d.swiglu_limit = 7.0
    d.ep_size = 1
    d.max_tokens = 4
    for k, v in kw.items():
        setattr(d, k, v)
    return d


def _create(d):
    lib = _lib.load_library()
    h = ctypes.c_void_p()
    rc = lib.gb_moe_create(ctypes.byref(d), ctypes.byref(h))
    return rc, lib.gb_last_error().decode(), h


BUF = np.zeros(1 << 16, np.uint8)
P = BUF.ctypes.data


def _full(**kw):
    base = dict(router_weight=P, gate_up_blocks=P, gate_up_scales=P, down_blocks=P,
                down_scales=P)
    base.update(kw)
    return _desc(**base)


@pytest.mark.parametrize("kw,status,needle", [
    (dict(struct_size=8), _lib.GB_ERR_INVALID_ARG, "struct_size"),
    (dict(hidden=0), _lib.GB_ERR_INVALID_ARG, "shape"),
    (dict(top_k=5), _lib.GB_ERR_INVALID_ARG, "top_k"),
    (dict(top_k=9, n_experts=16), _lib.GB_ERR_INVALID_ARG, "top_k"),
    (dict(router_kind=7), _lib.GB_ERR_INVALID_ARG, "router_kind"),
    (dict(act_kind=7), _lib.GB_ERR_INVALID_ARG, "act_kind"),
    (dict(weight_format=9), _lib.GB_ERR_INVALID_ARG, "weight_format"),
    (dict(router_weight=None), _lib.GB_ERR_INVALID_ARG, "router_weight"),
    (dict(down_scales=None), _lib.GB_ERR_INVALID_ARG, "MXFP4_SPLIT"),
    (dict(hidden=100), _lib.GB_ERR_SHAPE, "100"),
    (dict(inter=48), _lib.GB_ERR_SHAPE, "32-element"),
    (dict(n_experts=300, top_k=2), _lib.GB_ERR_UNSUPPORTED, "256"),
    (dict(weight_format=_lib.GB_FMT_Q4_K, gate_raw=P, up_raw=P, down_raw=P), _lib.GB_ERR_SHAPE,
     "256-element"),
    (dict(weight_format=_lib.GB_FMT_Q4_K), _lib.GB_ERR_INVALID_ARG, "Q4_K needs"),
    (dict(ep_size=2, ep_rank=3), _lib.GB_ERR_INVALID_ARG, "ep_rank"),
    (dict(max_tokens=-1), _lib.GB_ERR_INVALID_ARG, "max_tokens"),
])
def test_create_rejects_bad_descriptors(kw, status, needle):
    rc, msg, h = _create(_full(**kw))
    assert rc == status, msg
    assert needle in msg
    assert not h.value


def test_gguf_format_needs_raw_tensors():
    rc, msg, _ = _create(_desc(router_weight=P, weight_format=_lib.GB_FMT_MXFP4_GGUF))
    assert rc == _lib.GB_ERR_INVALID_ARG and "gate_raw" in msg


def test_null_handle_calls_are_errors_not_crashes():
    lib = _lib.load_library()
    assert lib.gb_moe_forward(None, None, 1, None, None) == _lib.GB_ERR_INVALID_ARG
    assert lib.gb_moe_route(None, None, 1, None, None, None, None, None, None) == \
        _lib.GB_ERR_INVALID_ARG
    assert lib.gb_moe_destroy(None) == _lib.GB_OK
    info = MoeInfo()
    info.struct_size = ctypes.sizeof(MoeInfo)
    assert lib.gb_moe_get_info(None, ctypes.byref(info)) == _lib.GB_ERR_INVALID_ARG


def test_noalloc_routing_checks_arguments_before_any_device_call():
    """gb_route_noalloc refuses bad sizes (and accepts T = 0) before it touches
    the device, so these calls need no GPU; the pointers are never read."""
    lib = _lib.load_library()
    S = _lib.GB_ROUTER_SOFTMAX_TOPK

    def call(T=8, hidden=2880, E=32, k=4, kind=S, ptr=P):
        rc = lib.gb_route_noalloc(ptr, ptr, None, None, T, hidden, E, k, kind, ptr, ptr, None)
        return rc, lib.gb_last_error().decode()

    assert call(T=0)[0] == _lib.GB_OK
    for kw, needle in ((dict(T=-1), "T = -1"), (dict(hidden=100), "multiple of 32"),
                       (dict(hidden=4128), "<= 4096"), (dict(E=0), "n_experts"),
                       (dict(E=300), "n_experts"), (dict(k=9), "top_k"),
                       (dict(E=2, k=3), "top_k"), (dict(kind=7), "router_kind"),
                       (dict(ptr=None), "null"), (dict(T=4097, E=8), "4096"),
                       (dict(T=2049, E=32), "65536"),
                       (dict(ptr=P + 4), "16-byte aligned")):
        rc, msg = call(**kw)
        assert rc == _lib.GB_ERR_INVALID_ARG, (kw, rc, msg)
        assert needle in msg, (kw, msg)


def test_block_refuses_inputs_on_another_gpu():
    """forward / route check the input's device before any kernel sees its
    address (no handle or GPU needed: the check is on the host)."""
    from gallium_b200.moe import MoEBlock

    blk = MoEBlock.__new__(MoEBlock)
    blk.device, blk.hidden = 0, 4

    class OnGpu1:
        is_cuda = True
        device = type("dev", (), {"index": 1})()

    with pytest.raises(_lib.GalliumError) as ei:
        blk._check_device(OnGpu1())
    assert ei.value.status == _lib.GB_ERR_INVALID_ARG and "cuda:1" in str(ei.value)
    import torch
    blk._check_device(torch.zeros(2, 4))  # host tensors go through gb_moe_forward_host


def test_python_errors_carry_status_and_message():
    with pytest.raises(_lib.GalliumError) as ei:
        _lib.check(_create(_full(hidden=100))[0])
    assert ei.value.status == _lib.GB_ERR_SHAPE
    assert "100" in str(ei.value)


def test_gguf_repack_helper_round_trips_values():
    layer = synth.gptoss_layer(n_experts=1, hidden=64, inter=32, seed=4)
    gg = synth.gptoss_gguf_from_split(layer)
    assert gg.gate_raw.shape == (1, 32, 2 * 17)
    assert gg.down_raw.shape == (1, 64, 1 * 17)


def test_decoder_struct_layouts_match_the_header(tmp_path):
    from gallium_b200._lib import DecoderDesc, DecoderLayer
    src = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', 'int main(void){']
    want = []
    for name, cls in (("gb_decoder_layer", DecoderLayer), ("gb_decoder_desc", DecoderDesc)):
        src.append(f'printf("%zu\\n", sizeof({name}));')
        want.append(ctypes.sizeof(cls))
        for f, _ in cls._fields_:
            src.append(f'printf("%zu\\n", offsetof({name}, {f}));')
            want.append(getattr(cls, f).offset)
    src.append("return 0;}")
    c = tmp_path / "dlayout.c"
    c.write_text("\n".join(src))
    exe = tmp_path / "dlayout"
    subprocess.run(["gcc", str(c), "-o", str(exe)], check=True)
    vals = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True,
                                           check=True).stdout.split()]
    assert vals == want


def _decoder_desc(layers=1, **kw):
    """A decoder descriptor whose pointers are all set (to a dummy host
    buffer): validation only, nothing reaches the device."""
    from gallium_b200._lib import DecoderDesc, DecoderLayer
    buf = np.zeros(16, np.float32)
    p = buf.ctypes.data
    moe = _desc()
    L = (DecoderLayer * layers)()
    for i in range(layers):
        for f, _ in DecoderLayer._fields_:
            if f not in ("sliding", "moe"):
                setattr(L[i], f, p)
        L[i].moe = ctypes.pointer(moe)
    d = DecoderDesc()
    d.struct_size = ctypes.sizeof(DecoderDesc)
    d.n_layers, d.hidden, d.n_heads, d.n_kv_heads, d.head_dim = layers, 64, 4, 2, 32
    d.vocab, d.sliding_window, d.max_seq_len, d.max_batch, d.max_tokens = 10, 4, 16, 1, 4
    d.rope_theta, d.rms_eps = 10000.0, 1e-5
    d.embed = d.final_norm = p
    d.layers = L
    for k, v in kw.items():
        setattr(d, k, v)
    return d, (buf, moe, L)


@pytest.mark.parametrize("kw,status,needle", [
    ({"struct_size": 8}, _lib.GB_ERR_INVALID_ARG, "struct_size"),
    ({"n_heads": 3}, _lib.GB_ERR_INVALID_ARG, "multiple"),
    ({"n_heads": 40, "n_kv_heads": 2}, _lib.GB_ERR_INVALID_ARG, "query heads"),
    ({"head_dim": 48}, _lib.GB_ERR_UNSUPPORTED, "head_dim"),
    ({"hidden": 40}, _lib.GB_ERR_INVALID_ARG, "hidden"),
    ({"vocab": 0}, _lib.GB_ERR_INVALID_ARG, "vocab"),
    ({"rope_scaling_factor": 32.0, "rope_orig_ctx": 0}, _lib.GB_ERR_INVALID_ARG, "YaRN"),
    ({"embed": None}, _lib.GB_ERR_INVALID_ARG, "embed"),
])
def test_decoder_create_rejects_bad_descriptors(kw, status, needle):
    lib = _lib.load_library()
    d, keep = _decoder_desc(**kw)
    h = ctypes.c_void_p()
    rc = lib.gb_decoder_create(ctypes.byref(d), ctypes.byref(h))
    assert rc == status, lib.gb_last_error()
    assert needle in lib.gb_last_error().decode()
    assert not h.value


def test_decoder_layer_checks():
    lib = _lib.load_library()
    d, keep = _decoder_desc(layers=2)
    keep[2][1].wk = None
    h = ctypes.c_void_p()
    assert lib.gb_decoder_create(ctypes.byref(d), ctypes.byref(h)) == _lib.GB_ERR_INVALID_ARG
    assert b"layer 1" in lib.gb_last_error()
    d, keep = _decoder_desc(layers=1)
    keep[1].hidden = 128  # the MoE block's hidden differs from the model's
    assert lib.gb_decoder_create(ctypes.byref(d), ctypes.byref(h)) == _lib.GB_ERR_INVALID_ARG
    assert b"hidden" in lib.gb_last_error()


def test_decoder_null_handle_calls_are_errors():
    lib = _lib.load_library()
    assert lib.gb_decoder_forward(None, None, 1, 1, 0, None, None, None) == _lib.GB_ERR_INVALID_ARG
    assert lib.gb_decoder_generate(None, None, 1, 0, 1, None, None) == _lib.GB_ERR_INVALID_ARG
    assert lib.gb_decoder_reset(None) == _lib.GB_ERR_INVALID_ARG
    assert lib.gb_decoder_set_profiling(None, 1) == _lib.GB_ERR_INVALID_ARG
    assert lib.gb_decoder_device_status(None, None) == _lib.GB_ERR_INVALID_ARG
    assert lib.gb_decoder_destroy(None) == _lib.GB_OK
