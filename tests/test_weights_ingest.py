"""Weight ingestion from checkpoint files (safetensors, GGUF) on the host.

Each case writes a small seeded layer in the file layout the reference loads
(gpt_oss.rs:115-142 safetensors names, gpt_oss_q.rs:135-163 and
lfm2moe_q.rs:214-232 GGUF names, GGUF header per quantized.rs:534-617),
reads it back with ``gallium_b200.weights`` and checks that the layer holds
the same bytes and that the oracle gives the same forward.  The error cases
are the ones a real checkpoint can present: wrong magic, truncated data, a
missing tensor, a shape that disagrees with the config, a tensor type the
library cannot take.
"""
import json

import numpy as np
import pytest

from gallium_b200 import synth
from gallium_b200.weights import (GGML_BF16, GGML_F16, GGML_F32, GGML_MXFP4, GGML_Q4_K,
                                  CheckpointError, GgufFile, SafetensorsCheckpoint,
                                  gptoss_layer_from_gguf, gptoss_layer_from_safetensors,
                                  lfm2_layer_from_gguf, write_gguf, write_safetensors)

import oracle


def _st_tensors(layer, i, router_dtype="BF16"):
    ex = f"model.layers.{i}.mlp.experts."
    rt = f"model.layers.{i}.mlp.router."
    rw, rb = layer.router_w, layer.router_b
    if router_dtype == "F32":
        rw, rb = synth.bf16_bits_to_f32(rw), synth.bf16_bits_to_f32(rb)
    return {
        ex + "gate_up_proj_blocks": ("U8", layer.gu_blocks),
        ex + "gate_up_proj_scales": ("U8", layer.gu_scales),
        ex + "gate_up_proj_bias": ("BF16", layer.gu_bias),
        ex + "down_proj_blocks": ("U8", layer.dn_blocks),
        ex + "down_proj_scales": ("U8", layer.dn_scales),
        ex + "down_proj_bias": ("BF16", layer.dn_bias),
        rt + "weight": (router_dtype, rw),
        rt + "bias": (router_dtype, rb),
    }


def _config(layer, n_layers=2):
    return {"hidden_size": layer.hidden, "intermediate_size": layer.inter,
            "num_local_experts": layer.n_experts, "num_experts_per_tok": layer.top_k,
            "num_hidden_layers": n_layers, "swiglu_limit": 7.0}


@pytest.fixture(scope="module")
def small():
    return synth.gptoss_layer(n_experts=8, hidden=128, inter=96, top_k=4, seed=3, skewed=True)


def _same_forward(a, b, gguf_a=None, gguf_b=None, hidden=128, T=9):
    x = synth.tokens(T, hidden, seed=5)
    oa, ia, wa = oracle.OracleMoe(a, gguf=gguf_a).forward(x)
    ob, ib, wb = oracle.OracleMoe(b, gguf=gguf_b).forward(x)
    np.testing.assert_array_equal(ia, ib)
    np.testing.assert_array_equal(wa, wb)
    np.testing.assert_array_equal(oa, ob)


def test_safetensors_sharded_gptoss_layer_round_trip(tmp_path, small):
    # Layer 1's experts in one shard, its router in another, named by an index file.
    t = _st_tensors(small, 1)
    names = sorted(t)
    shard_a = {n: t[n] for n in names if ".experts." in n}
    shard_b = {n: t[n] for n in names if ".router." in n}
    write_safetensors(str(tmp_path / "model-00001.safetensors"), shard_a, {"format": "pt"})
    write_safetensors(str(tmp_path / "model-00002.safetensors"), shard_b)
    wm = {n: "model-00001.safetensors" for n in shard_a}
    wm.update({n: "model-00002.safetensors" for n in shard_b})
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps({"weight_map": wm}))
    (tmp_path / "config.json").write_text(json.dumps(_config(small)))

    ck = SafetensorsCheckpoint.from_index(str(tmp_path / "model.safetensors.index.json"))
    got = gptoss_layer_from_safetensors(ck, str(tmp_path / "config.json"), 1)
    assert (got.hidden, got.inter, got.n_experts, got.top_k, got.swiglu_limit) == (
        small.hidden, small.inter, small.n_experts, small.top_k, 7.0)
    for f in ("router_w", "router_b", "gu_blocks", "gu_scales", "gu_bias", "dn_blocks",
              "dn_scales", "dn_bias"):
        a, b = getattr(got, f), getattr(small, f)
        assert a.dtype == b.dtype and a.shape == b.shape, f
        np.testing.assert_array_equal(a, b, err_msg=f)
    assert isinstance(got.gu_blocks, np.memmap)  # mapped, not copied
    _same_forward(small, got)


def test_moe_layer_listing(tmp_path, small):
    """Which layers of a file carry MoE experts, for loading a whole model."""
    t = dict(_st_tensors(small, 3))
    t.update(_st_tensors(small, 1))
    t["model.layers.2.mlp.gate_proj.weight"] = ("F32", np.zeros((2, 2), np.float32))
    p = str(tmp_path / "m.safetensors")
    write_safetensors(p, t)
    assert SafetensorsCheckpoint(p).moe_layers() == [1, 3]
    md, tensors, _ = _gguf_gptoss(small, 5)
    tensors["blk.0.ffn_gate.weight"] = (GGML_F32, (2, 2), np.zeros((2, 2), np.float32))
    q = str(tmp_path / "m.gguf")
    write_gguf(q, dict(md, **{"gpt-oss.block_count": 6}), tensors)
    assert GgufFile(q).moe_blocks() == [5]


def test_safetensors_f32_router_keeps_f32(tmp_path, small):
    p = str(tmp_path / "m.safetensors")
    write_safetensors(p, _st_tensors(small, 0, router_dtype="F32"))
    got = gptoss_layer_from_safetensors(SafetensorsCheckpoint(p), _config(small), 0)
    assert got.router_w.dtype == np.float32 and got.router_b.dtype == np.float32
    np.testing.assert_array_equal(got.router_w, synth.bf16_bits_to_f32(small.router_w))
    _same_forward(small, got)  # same values, so the same routing and output


def test_safetensors_errors(tmp_path, small):
    t = _st_tensors(small, 0)
    p = str(tmp_path / "m.safetensors")
    write_safetensors(p, t)
    ck = SafetensorsCheckpoint(p)
    with pytest.raises(CheckpointError, match="no tensor"):
        gptoss_layer_from_safetensors(ck, _config(small), 1)  # layer 1 is not in the file
    bad = dict(_config(small), intermediate_size=small.inter * 2)
    with pytest.raises(CheckpointError, match="shape"):
        gptoss_layer_from_safetensors(ck, bad, 0)
    with pytest.raises(CheckpointError, match="outside"):
        gptoss_layer_from_safetensors(ck, _config(small, n_layers=1), 3)
    # Truncated data: the last tensor's bytes run past the end.
    raw = open(p, "rb").read()
    q = str(tmp_path / "cut.safetensors")
    open(q, "wb").write(raw[:-100])
    with pytest.raises(CheckpointError, match="data_offsets"):
        gptoss_layer_from_safetensors(SafetensorsCheckpoint(q), _config(small), 0)
    # A header length beyond the file.
    r = str(tmp_path / "hdr.safetensors")
    open(r, "wb").write((1 << 40).to_bytes(8, "little") + b"{}")
    with pytest.raises(CheckpointError, match="header length"):
        SafetensorsCheckpoint(r)
    # A header entry that is not a tensor record.
    import struct
    h = b'{"w": 5}'
    bad = str(tmp_path / "rec.safetensors")
    open(bad, "wb").write(struct.pack("<Q", len(h)) + h)
    with pytest.raises(CheckpointError, match="not a tensor record"):
        SafetensorsCheckpoint(bad).tensor("w")
    # Missing files and a broken index.
    with pytest.raises(CheckpointError, match="cannot open"):
        SafetensorsCheckpoint(str(tmp_path / "absent.safetensors"))
    with pytest.raises(CheckpointError, match="cannot open"):
        GgufFile(str(tmp_path / "absent.gguf"))
    idx = tmp_path / "model.safetensors.index.json"
    idx.write_text("[1, 2]")
    with pytest.raises(CheckpointError, match="not a safetensors index"):
        SafetensorsCheckpoint.from_index(str(idx))
    idx.write_text('{"weight_map": {}}')
    with pytest.raises(CheckpointError, match="no weight_map"):
        SafetensorsCheckpoint.from_index(str(idx))
    # The same tensor in two shards.
    with pytest.raises(CheckpointError, match="in both"):
        SafetensorsCheckpoint([p, p])
    # Expert blocks stored as F32 instead of U8.
    t2 = dict(t)
    key = "model.layers.0.mlp.experts.down_proj_scales"
    t2[key] = ("F32", small.dn_scales.astype(np.float32))
    s = str(tmp_path / "f32scales.safetensors")
    write_safetensors(s, t2)
    with pytest.raises(CheckpointError, match="expected one of"):
        gptoss_layer_from_safetensors(SafetensorsCheckpoint(s), _config(small), 0)


def _gguf_gptoss(layer, i, n_layers=2, router_type=GGML_F32, alignment=32):
    g = synth.gptoss_gguf_from_split(layer)
    E, H, I = layer.n_experts, layer.hidden, layer.inter
    p = f"blk.{i}."
    rw = synth.bf16_bits_to_f32(layer.router_w)
    if router_type == GGML_F16:
        rw_t = (GGML_F16, (E, H), rw.astype(np.float16))
    elif router_type == GGML_BF16:
        rw_t = (GGML_BF16, (E, H), layer.router_w)
    else:
        rw_t = (GGML_F32, (E, H), rw)
    md = {"general.architecture": "gpt-oss", "gpt-oss.block_count": n_layers,
          "gpt-oss.expert_count": E, "gpt-oss.expert_used_count": layer.top_k,
          "gpt-oss.swiglu_limit": 7.0, "gpt-oss.embedding_length": H,
          "general.name": "synthetic", "gpt-oss.layer_types": ["sliding", "full"],
          "gpt-oss.some_floats": [0.5, 1.5]}
    tensors = {
        "token_embd.weight": (GGML_F32, (4, H), np.zeros((4, H), np.float32)),
        p + "ffn_gate_exps.weight": (GGML_MXFP4, (E, I, H), g.gate_raw),
        p + "ffn_up_exps.weight": (GGML_MXFP4, (E, I, H), g.up_raw),
        p + "ffn_down_exps.weight": (GGML_MXFP4, (E, H, I), g.down_raw),
        p + "ffn_gate_exps.bias": (GGML_F32, (E, I), synth.bf16_bits_to_f32(g.gate_bias)),
        p + "ffn_up_exps.bias": (GGML_F32, (E, I), synth.bf16_bits_to_f32(g.up_bias)),
        p + "ffn_down_exps.bias": (GGML_F32, (E, H), synth.bf16_bits_to_f32(g.down_bias)),
        p + "ffn_gate_inp.weight": rw_t,
        p + "ffn_gate_inp.bias": (GGML_F32, (E,), synth.bf16_bits_to_f32(layer.router_b)),
    }
    return md, tensors, g


@pytest.mark.parametrize("router_type", [GGML_F32, GGML_F16, GGML_BF16])
@pytest.mark.parametrize("alignment", [32, 64])
def test_gguf_gptoss_layer_round_trip(tmp_path, small, router_type, alignment):
    md, tensors, g = _gguf_gptoss(small, 1, router_type=router_type)
    path = str(tmp_path / "m.gguf")
    write_gguf(path, md, tensors, alignment=alignment)
    f = GgufFile(path)
    assert f.version == 3 and f.alignment == alignment and f.architecture == "gpt-oss"
    assert f.metadata["gpt-oss.layer_types"] == ["sliding", "full"]
    assert f.metadata["gpt-oss.some_floats"] == [0.5, 1.5]
    got = gptoss_layer_from_gguf(f, 1)
    b = got.base
    assert (b.hidden, b.inter, b.n_experts, b.top_k, b.swiglu_limit) == (
        small.hidden, small.inter, small.n_experts, small.top_k, 7.0)
    for name in ("gate_raw", "up_raw", "down_raw"):
        np.testing.assert_array_equal(getattr(got, name), getattr(g, name), err_msg=name)
    np.testing.assert_array_equal(got.down_bias, synth.bf16_bits_to_f32(small.dn_bias))
    rw = synth.bf16_bits_to_f32(small.router_w)
    if router_type == GGML_F16:
        rw = rw.astype(np.float16).astype(np.float32)
    np.testing.assert_array_equal(b.router_w, rw)
    if router_type != GGML_F16:  # the f16 router rounds the weights, so routing may differ
        _same_forward(small, b, gguf_a=g, gguf_b=got)


def test_gguf_gptoss_forward_equals_safetensors_forward(tmp_path, small):
    """The GGUF file and the safetensors layer it came from route and compute alike."""
    md, tensors, _ = _gguf_gptoss(small, 0)
    path = str(tmp_path / "m.gguf")
    write_gguf(path, md, tensors)
    got = gptoss_layer_from_gguf(GgufFile(path), 0)
    x = synth.tokens(7, small.hidden, seed=11)
    o1, i1, w1 = oracle.OracleMoe(small).forward(x)
    o2, i2, w2 = oracle.OracleMoe(got.base, gguf=got).forward(x)
    np.testing.assert_array_equal(i1, i2)
    np.testing.assert_array_equal(w1, w2)
    np.testing.assert_allclose(o2, o1, rtol=0, atol=1e-4)


def test_gguf_errors(tmp_path, small):
    md, tensors, _ = _gguf_gptoss(small, 0)
    path = str(tmp_path / "m.gguf")
    write_gguf(path, md, tensors)
    raw = open(path, "rb").read()

    bad = str(tmp_path / "magic.gguf")
    open(bad, "wb").write(b"GGML" + raw[4:])
    with pytest.raises(CheckpointError, match="magic"):
        GgufFile(bad)
    ver = str(tmp_path / "ver.gguf")
    open(ver, "wb").write(raw[:4] + (7).to_bytes(4, "little") + raw[8:])
    with pytest.raises(CheckpointError, match="version"):
        GgufFile(ver)
    head = str(tmp_path / "head.gguf")
    open(head, "wb").write(raw[:200])
    with pytest.raises(CheckpointError, match="past the end"):
        GgufFile(head)
    cut = str(tmp_path / "cut.gguf")
    open(cut, "wb").write(raw[:-64])
    with pytest.raises(CheckpointError, match="past the end of the file"):
        gptoss_layer_from_gguf(GgufFile(cut), 0)

    f = GgufFile(path)
    with pytest.raises(CheckpointError, match="no MoE experts"):
        gptoss_layer_from_gguf(f, 1)
    with pytest.raises(CheckpointError, match="outside"):
        gptoss_layer_from_gguf(f, 5)

    # Experts in a type this library does not take (Q4_K where MXFP4 is expected).
    t2 = dict(tensors)
    E, I, H = small.n_experts, small.inter, small.hidden
    t2["blk.0.ffn_up_exps.weight"] = (GGML_Q4_K, (E, I, 256),
                                      np.zeros((E, I, 144), np.uint8))
    q = str(tmp_path / "q4k.gguf")
    write_gguf(q, md, t2)
    with pytest.raises(CheckpointError, match="MXFP4"):
        gptoss_layer_from_gguf(GgufFile(q), 0)
    # A router in a quantized type (Q8_0 = 8) is refused, not silently dequantised.
    t3 = dict(tensors)
    t3["blk.0.ffn_gate_inp.weight"] = (8, (E, H), np.zeros(E * H // 32 * 34, np.uint8))
    r = str(tmp_path / "q8router.gguf")
    write_gguf(r, md, t3)
    with pytest.raises(CheckpointError, match="GGML type 8"):
        gptoss_layer_from_gguf(GgufFile(r), 0)
    # expert_count that disagrees with the tensors.
    m2 = dict(md)
    m2["gpt-oss.expert_count"] = small.n_experts + 1
    c = str(tmp_path / "count.gguf")
    write_gguf(c, m2, tensors)
    with pytest.raises(CheckpointError, match="expert_count"):
        gptoss_layer_from_gguf(GgufFile(c), 0)


def test_gguf_version1_header(tmp_path):
    """Version-1 files use 32-bit counts, string lengths and dims (quantized.rs:553-584)."""
    import struct

    def s1(x):
        b = x.encode()
        return struct.pack("<I", len(b)) + b

    data = np.arange(6, dtype=np.float32)
    head = struct.pack("<III", 0x46554747, 1, 1) + struct.pack("<I", 1)
    head += s1("general.architecture") + struct.pack("<I", 8) + s1("test")
    head += s1("w") + struct.pack("<I", 2) + struct.pack("<II", 3, 2)  # ne = [3, 2] -> (2, 3)
    head += struct.pack("<IQ", GGML_F32, 0)
    head += b"\0" * (-len(head) % 32)
    p = str(tmp_path / "v1.gguf")
    open(p, "wb").write(head + data.tobytes())
    f = GgufFile(p)
    assert f.version == 1 and f.architecture == "test"
    np.testing.assert_array_equal(f.floats("w", (2, 3)), data.reshape(2, 3))


def test_gguf_container_agrees_with_gguf_py(tmp_path):
    """The GGUF reader and writer against gguf-py (llama.cpp's Python GGUF
    package) in both directions: MXFP4 and Q4_K expert tensors, F32 tensors,
    metadata of several types."""
    gguf = pytest.importorskip("gguf")
    layer = synth.lfm2_layer(n_experts=2, hidden=256, inter=256, top_k=2, seed=9)
    mx = synth.gptoss_gguf_from_split(
        synth.gptoss_layer(n_experts=2, hidden=64, inter=64, top_k=2, seed=9))
    Q4K, MXFP4 = gguf.GGMLQuantizationType.Q4_K, gguf.GGMLQuantizationType.MXFP4

    # gguf-py writes, this module reads.
    a = str(tmp_path / "by_gguf_py.gguf")
    w = gguf.GGUFWriter(a, "lfm2moe")
    w.add_uint32("lfm2moe.expert_count", 2)
    w.add_uint32("lfm2moe.expert_used_count", 2)
    w.add_float32("lfm2moe.rope.freq_base", 1e6)
    w.add_array("lfm2moe.attention.head_count_kv", [0, 8])
    # quantized tensors go in as their bytes; gguf-py derives the element shape
    w.add_tensor("blk.0.ffn_gate_exps.weight", layer.gate_raw, raw_dtype=Q4K)
    w.add_tensor("blk.0.ffn_up_exps.weight", layer.up_raw, raw_dtype=Q4K)
    w.add_tensor("blk.0.ffn_down_exps.weight", layer.down_raw, raw_dtype=Q4K)
    w.add_tensor("blk.0.ffn_gate_inp.weight", layer.router_w)
    w.add_tensor("blk.1.ffn_gate_exps.weight", mx.gate_raw, raw_dtype=MXFP4)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    f = GgufFile(a)
    assert f.architecture == "lfm2moe"
    assert f.metadata["lfm2moe.rope.freq_base"] == np.float32(1e6)
    assert f.metadata["lfm2moe.attention.head_count_kv"] == [0, 8]
    got = lfm2_layer_from_gguf(f, 0)
    for name in ("gate_raw", "up_raw", "down_raw", "router_w"):
        np.testing.assert_array_equal(getattr(got, name), getattr(layer, name), err_msg=name)
    np.testing.assert_array_equal(f.experts("blk.1.ffn_gate_exps.weight", GGML_MXFP4, (2, 64, 64)),
                                  mx.gate_raw)

    # This module writes, gguf-py reads.
    b = str(tmp_path / "by_weights.gguf")
    md, tensors = _gguf_lfm2(layer, 0, lead=0)
    write_gguf(b, md, tensors, alignment=64)
    r = gguf.GGUFReader(b)
    assert r.alignment == 64
    t = {x.name: x for x in r.tensors}
    assert t["blk.0.ffn_gate_exps.weight"].tensor_type == Q4K
    assert [int(v) for v in t["blk.0.ffn_down_exps.weight"].shape] == [256, 256, 2]  # innermost first
    np.testing.assert_array_equal(np.asarray(t["blk.0.ffn_up_exps.weight"].data).reshape(-1),
                                  layer.up_raw.reshape(-1))
    np.testing.assert_array_equal(np.asarray(t["blk.0.ffn_gate_inp.weight"].data).reshape(2, 256),
                                  layer.router_w)
    assert int(r.get_field("lfm2moe.expert_used_count").contents()) == 2


def _gguf_lfm2(layer, i, lead=1):
    E, H, I = layer.n_experts, layer.hidden, layer.inter
    p = f"blk.{i}."
    md = {"general.architecture": "lfm2moe", "lfm2moe.block_count": 3,
          "lfm2moe.expert_count": E, "lfm2moe.expert_used_count": layer.top_k,
          "lfm2moe.leading_dense_block_count": lead,
          "lfm2moe.attention.head_count_kv": [0, 8, 0]}
    tensors = {
        p + "ffn_gate_exps.weight": (GGML_Q4_K, (E, I, H), layer.gate_raw),
        p + "ffn_up_exps.weight": (GGML_Q4_K, (E, I, H), layer.up_raw),
        p + "ffn_down_exps.weight": (GGML_Q4_K, (E, H, I), layer.down_raw),
        p + "ffn_gate_inp.weight": (GGML_F32, (E, H), layer.router_w),
        p + "exp_probs_b.bias": (GGML_F32, (E,), layer.sel_bias),
    }
    return md, tensors


def test_gguf_lfm2_layer_round_trip(tmp_path):
    layer = synth.lfm2_layer(n_experts=8, hidden=256, inter=512, top_k=4, seed=2)
    layer.sel_bias[:] = np.linspace(-0.5, 0.5, 8, dtype=np.float32)
    md, tensors = _gguf_lfm2(layer, 2)
    path = str(tmp_path / "lfm2.gguf")
    write_gguf(path, md, tensors)
    f = GgufFile(path)
    assert f.metadata["lfm2moe.attention.head_count_kv"] == [0, 8, 0]
    got = lfm2_layer_from_gguf(f, 2)
    assert (got.hidden, got.inter, got.n_experts, got.top_k) == (256, 512, 8, 4)
    for name in ("router_w", "sel_bias", "gate_raw", "up_raw", "down_raw"):
        np.testing.assert_array_equal(getattr(got, name), getattr(layer, name), err_msg=name)
    x = synth.tokens(6, 256, seed=1)
    oa, ia, _ = oracle.OracleLfm2(layer).forward(x)
    ob, ib, _ = oracle.OracleLfm2(got).forward(x)
    np.testing.assert_array_equal(ia, ib)
    np.testing.assert_array_equal(oa, ob)
    with pytest.raises(CheckpointError, match="leading dense"):
        lfm2_layer_from_gguf(f, 0)
    # Without exp_probs_b the selection bias is zero.
    t2 = {k: v for k, v in tensors.items() if "exp_probs_b" not in k}
    q = str(tmp_path / "nobias.gguf")
    write_gguf(q, md, t2)
    assert not lfm2_layer_from_gguf(GgufFile(q), 2).sel_bias.any()
    # Real Q4_K_M files hold some expert tensors in Q6_K (type 14): refused by name.
    t3 = dict(tensors)
    E, H, I = 8, 256, 512
    t3["blk.2.ffn_down_exps.weight"] = (14, (E, H, I), np.zeros((E, H, I // 256 * 210), np.uint8))
    r = str(tmp_path / "q6k.gguf")
    write_gguf(r, md, t3)
    with pytest.raises(CheckpointError, match="GGML type 14.*Q4_K"):
        lfm2_layer_from_gguf(GgufFile(r), 2)


def test_block_loaders_accept_ingested_dtypes():
    """The host mirror's dtype handling, without creating a handle: float32
    routers travel as F32, bf16 bits as BF16, and a missing router bias is NULL."""
    from gallium_b200 import _lib
    from gallium_b200.moe import _as_f32, _float_pair

    bits = synth.f32_to_bf16_bits(np.array([1.5, -2.0], np.float32))
    a, b, dt = _float_pair(bits, bits)
    assert dt == _lib.GB_DTYPE_BF16 and a is bits
    a, b, dt = _float_pair(bits, np.array([0.25, 1.0], np.float32))
    assert dt == _lib.GB_DTYPE_F32 and a.dtype == np.float32
    np.testing.assert_array_equal(a, [1.5, -2.0])
    a, b, dt = _float_pair(np.array([3.0], np.float16), None)
    assert dt == _lib.GB_DTYPE_F32 and b is None and a.dtype == np.float32
    assert _as_f32(None) is None


# ---- on the GPU: file-loaded layers through the block loaders ------------------

MAX_ABS = 2e-2
MEAN_REL = 1e-3


def _parity(got, want, what):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape and np.all(np.isfinite(got)), what
    err = np.abs(got - want)
    max_abs = float(err.max())
    mean_rel = float(err.sum() / max(np.abs(want).sum(), 1e-30))
    assert max_abs <= MAX_ABS and mean_rel <= MEAN_REL, (what, max_abs, mean_rel)


def _gpu_forward(block, x):
    import torch
    with block:
        xd = torch.from_numpy(np.ascontiguousarray(x)).to("cuda:0")
        out = block.forward(xd).cpu().numpy()
        idx = block.route(xd)["idx"].cpu().numpy()
    return out, idx


@pytest.mark.gpu
@pytest.mark.parametrize("router_dtype", ["BF16", "F32"])
def test_gpu_safetensors_layer_matches_oracle(tmp_path, router_dtype):
    from gallium_b200 import OssMoEFFN
    layer = synth.gptoss_layer(n_experts=8, hidden=256, inter=256, top_k=4, seed=21)
    p = str(tmp_path / "m.safetensors")
    write_safetensors(p, _st_tensors(layer, 0, router_dtype=router_dtype))
    got_layer = gptoss_layer_from_safetensors(SafetensorsCheckpoint(p), _config(layer), 0)
    x = synth.tokens(40, 256, seed=4)
    out, idx = _gpu_forward(OssMoEFFN.load(got_layer, device=0, max_tokens=40), x)
    want, widx, _ = oracle.OracleMoe(layer).forward(x)
    np.testing.assert_array_equal(idx, widx)
    _parity(out, want, f"safetensors file, {router_dtype} router")
    ref, _ = _gpu_forward(OssMoEFFN.load(layer, device=0, max_tokens=40), x)
    _parity(out, ref, "file-loaded vs in-memory layer")


@pytest.mark.gpu
def test_gpu_gguf_gptoss_layer_matches_oracle(tmp_path):
    from gallium_b200 import GptOssQMoEFFN
    layer = synth.gptoss_layer(n_experts=8, hidden=256, inter=256, top_k=4, seed=22)
    md, tensors, g = _gguf_gptoss(layer, 0)
    path = str(tmp_path / "m.gguf")
    write_gguf(path, md, tensors)
    got = gptoss_layer_from_gguf(GgufFile(path), 0)
    x = synth.tokens(40, 256, seed=6)
    out, idx = _gpu_forward(GptOssQMoEFFN.load(got, device=0, max_tokens=40), x)
    want, widx, _ = oracle.OracleMoe(got.base, gguf=got).forward(x)
    np.testing.assert_array_equal(idx, widx)
    _parity(out, want, "GGUF MXFP4 file")


@pytest.mark.gpu
def test_gpu_gguf_lfm2_layer_matches_oracle(tmp_path):
    from gallium_b200 import Lfm2QMoEFFN
    layer = synth.lfm2_layer(n_experts=4, hidden=256, inter=256, top_k=2, seed=23)
    md, tensors = _gguf_lfm2(layer, 1)
    path = str(tmp_path / "lfm2.gguf")
    write_gguf(path, md, tensors)
    got = lfm2_layer_from_gguf(GgufFile(path), 1)
    x = synth.tokens(24, 256, seed=8)
    out, idx = _gpu_forward(Lfm2QMoEFFN.load(got, device=0, max_tokens=24), x)
    want, widx, _ = oracle.OracleLfm2(layer).forward(x)
    np.testing.assert_array_equal(idx, widx)
    _parity(out, want, "GGUF Q4_K file")


def test_damaged_gguf_files_raise_checkpoint_errors_only(tmp_path, small):
    """Truncations at every 97th byte and 300 single-byte corruptions of the
    header: each file either loads or raises CheckpointError (never another
    exception, never a read outside the file)."""
    md, tensors, _ = _gguf_gptoss(small, 0)
    path = str(tmp_path / "m.gguf")
    write_gguf(path, md, tensors)
    raw = open(path, "rb").read()
    head_len = GgufFile(path).data_offset
    rng = np.random.default_rng(11)
    cases = [raw[:cut] for cut in range(0, len(raw), 97)]
    for _ in range(300):
        b = bytearray(raw)
        b[int(rng.integers(0, head_len))] = int(rng.integers(0, 256))
        cases.append(bytes(b))
    q = str(tmp_path / "damaged.gguf")
    for data in cases:
        open(q, "wb").write(data)
        try:
            gptoss_layer_from_gguf(GgufFile(q), 0)
        except CheckpointError:
            pass


def test_damaged_safetensors_files_raise_checkpoint_errors_only(tmp_path, small):
    """The same for safetensors: truncations and single-byte header damage."""
    path = str(tmp_path / "m.safetensors")
    write_safetensors(path, _st_tensors(small, 0))
    raw = open(path, "rb").read()
    head_len = 8 + int.from_bytes(raw[:8], "little")
    rng = np.random.default_rng(12)
    cases = [raw[:cut] for cut in range(0, len(raw), 89)]
    for _ in range(300):
        b = bytearray(raw)
        b[int(rng.integers(0, head_len))] = int(rng.integers(0, 256))
        cases.append(bytes(b))
    q = str(tmp_path / "damaged.safetensors")
    for data in cases:
        open(q, "wb").write(data)
        try:
            gptoss_layer_from_safetensors(SafetensorsCheckpoint(q), _config(small), 0)
        except CheckpointError:
            pass
