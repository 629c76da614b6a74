"""Weight ingestion: MoE layers read from safetensors and GGUF checkpoint files.

The reference loads its MoE blocks from memory-mapped files and hands the
tensors to the blocks' ``load``:

* safetensors GPT-OSS (``OssMoEFFN::load``, crates/gallium-models/src/gpt_oss.rs:115-142):
  ``model.layers.{i}.mlp.experts.{gate_up,down}_proj_{blocks,scales,bias}`` and
  ``model.layers.{i}.mlp.router.{weight,bias}``, read through candle's
  ``VarBuilder::from_mmaped_safetensors`` (crates/gallium-models/src/loader.rs:13-19,
  gpt_oss.rs:272-273), sizes from the HF ``config.json`` (gpt_oss.rs:56-80);
* GGUF GPT-OSS (``QMoEFFN::load``, crates/gallium-models/src/gpt_oss_q.rs:135-163):
  ``blk.{i}.ffn_{gate,up,down}_exps.weight`` (MXFP4, GGML type 39) and
  ``.bias``, router ``blk.{i}.ffn_gate_inp.{weight,bias}``; metadata keys
  ``{arch}.expert_count``, ``{arch}.expert_used_count``, ``{arch}.swiglu_limit``
  (gpt_oss_q.rs:316-349);
* GGUF LFM2.5 (``QMoEFFN::load``, crates/gallium-models/src/lfm2moe_q.rs:214-232):
  Q4_K (type 12) expert tensors, router ``blk.{i}.ffn_gate_inp.weight`` and the
  selection bias ``blk.{i}.exp_probs_b.bias``; layers below
  ``{arch}.leading_dense_block_count`` are dense (lfm2moe_q.rs:403, 436-440).

The GGUF header is parsed like the reference's tolerant parser
(crates/gallium-core/src/quantized.rs:534-617: versions 1-3, dims stored
innermost first and reversed to row-major, tensor data at the header's end
rounded up to ``general.alignment``, default 32; unknown tensor types are
accepted until a tensor of that type is read).  Tensors are numpy views of an
``np.memmap``, so ``OssMoEFFN.load`` and friends upload straight from the
mapped file without a host copy.

Every problem with the files (a file that cannot be opened, bad magic, a
truncated or damaged header, a tensor outside the file, a missing tensor, a
shape that disagrees with the layer's sizes, a tensor type this library
cannot take) raises ``CheckpointError`` naming the file and tensor.

``write_safetensors`` / ``write_gguf`` produce files in the same formats
(used to build test checkpoints; they are not on the forward path).
"""
from __future__ import annotations

import json
import math
import os
import struct
from typing import Dict, Iterable, List, Optional, Sequence, Tuple, Union

import numpy as np

from .synth import GptOssGgufLayer, GptOssLayer, Lfm2Layer


class CheckpointError(ValueError):
    """A checkpoint file that cannot be read as the requested MoE layer."""


def _file_size(path: str) -> int:
    try:
        return os.path.getsize(path)
    except OSError as e:
        raise CheckpointError(f"{path}: cannot open ({e.strerror})") from None


def _block_indices(names: Iterable[str], prefix: str, suffix: str) -> List[int]:
    out = set()
    for n in names:
        if n.startswith(prefix) and n.endswith(suffix):
            mid = n[len(prefix):len(n) - len(suffix)]
            if mid.isdigit():
                out.add(int(mid))
    return sorted(out)


# ---- safetensors --------------------------------------------------------------

_ST_DTYPES = {
    "BOOL": np.bool_, "U8": np.uint8, "I8": np.int8, "U16": np.uint16, "I16": np.int16,
    "F16": np.float16, "BF16": np.uint16,  # bf16 kept as its uint16 bits
    "U32": np.uint32, "I32": np.int32, "F32": np.float32,
    "U64": np.uint64, "I64": np.int64, "F64": np.float64,
}
_MAX_ST_HEADER = 100 << 20


class SafetensorsFile:
    """One safetensors file: an 8-byte little-endian header length, a JSON
    header {name: {dtype, shape, data_offsets: [begin, end]}} and the data
    bytes, offsets relative to the end of the header."""

    def __init__(self, path: str):
        self.path = path
        size = _file_size(path)
        if size < 8:
            raise CheckpointError(f"{path}: {size} bytes, too short for a safetensors file")
        with open(path, "rb") as f:
            (n,) = struct.unpack("<Q", f.read(8))
            if n > _MAX_ST_HEADER or 8 + n > size:
                raise CheckpointError(f"{path}: header length {n} does not fit the file ({size} B)")
            try:
                header = json.loads(f.read(n).decode("utf-8"))
            except (UnicodeDecodeError, json.JSONDecodeError) as e:
                raise CheckpointError(f"{path}: header is not JSON ({e})") from None
        if not isinstance(header, dict):
            raise CheckpointError(f"{path}: header is not a JSON object")
        self.metadata = header.pop("__metadata__", {}) or {}
        self._base = 8 + n
        self._data_len = size - self._base
        self._infos = header
        self._mm = np.memmap(path, dtype=np.uint8, mode="r") if size > self._base else None

    def names(self) -> List[str]:
        return list(self._infos)

    def __contains__(self, name: str) -> bool:
        return name in self._infos

    def dtype(self, name: str) -> str:
        return self._info(name)["dtype"]

    def _info(self, name: str) -> dict:
        try:
            info = self._infos[name]
        except KeyError:
            raise CheckpointError(f"{self.path}: no tensor {name!r}") from None
        ok = (isinstance(info, dict) and isinstance(info.get("dtype"), str)
              and isinstance(info.get("shape"), list)
              and all(isinstance(d, int) and d >= 0 for d in info["shape"])
              and isinstance(info.get("data_offsets"), list) and len(info["data_offsets"]) == 2
              and all(isinstance(v, int) for v in info["data_offsets"]))
        if not ok:
            raise CheckpointError(f"{self.path}: header entry of {name!r} is not a tensor record "
                                  f"(dtype, shape, data_offsets)")
        return info

    def tensor(self, name: str) -> np.ndarray:
        """The tensor as a read-only numpy view of the mapped file (BF16 as uint16 bits)."""
        info = self._info(name)
        dt = _ST_DTYPES.get(info.get("dtype"))
        if dt is None:
            raise CheckpointError(f"{self.path}: tensor {name!r} has dtype {info.get('dtype')!r}, "
                                  f"not one of {sorted(_ST_DTYPES)}")
        shape = tuple(int(d) for d in info.get("shape", []))
        begin, end = (int(v) for v in info.get("data_offsets", (-1, -1)))
        nbytes = math.prod(shape) * np.dtype(dt).itemsize  # Python ints: no wrap-around
        if not (0 <= begin <= end <= self._data_len) or end - begin != nbytes:
            raise CheckpointError(f"{self.path}: tensor {name!r} data_offsets [{begin}, {end}) do "
                                  f"not hold {shape} {info['dtype']} inside {self._data_len} data "
                                  f"bytes")
        if nbytes == 0:
            return np.zeros(shape, dt)
        return self._mm[self._base + begin:self._base + end].view(dt).reshape(shape)


class SafetensorsCheckpoint:
    """Several safetensors shards seen as one namespace, like candle's
    ``VarBuilder::from_mmaped_safetensors(paths, ...)``.  A tensor name found
    in two shards is an error."""

    def __init__(self, paths: Union[str, Sequence[str]]):
        if isinstance(paths, (str, os.PathLike)):
            paths = [os.fspath(paths)]
        self.files = [SafetensorsFile(p) for p in paths]
        self._where: Dict[str, SafetensorsFile] = {}
        for f in self.files:
            for n in f.names():
                if n in self._where:
                    raise CheckpointError(f"tensor {n!r} is in both {self._where[n].path} and "
                                          f"{f.path}")
                self._where[n] = f

    @classmethod
    def from_index(cls, index_path: str) -> "SafetensorsCheckpoint":
        """Shards named by a ``model.safetensors.index.json`` weight_map."""
        try:
            with open(index_path) as f:
                wm = json.load(f).get("weight_map", {})
        except (OSError, ValueError, AttributeError) as e:
            raise CheckpointError(f"{index_path}: not a safetensors index ({e})") from None
        if not isinstance(wm, dict) or not wm:
            raise CheckpointError(f"{index_path}: no weight_map")
        d = os.path.dirname(os.path.abspath(index_path))
        return cls([os.path.join(d, s) for s in dict.fromkeys(wm.values())])

    def __contains__(self, name: str) -> bool:
        return name in self._where

    def moe_layers(self) -> List[int]:
        """Indices i of the layers whose MoE experts are in the checkpoint
        (``model.layers.{i}.mlp.experts.gate_up_proj_blocks``), ascending."""
        return _block_indices(self._where, "model.layers.", ".mlp.experts.gate_up_proj_blocks")

    def file_of(self, name: str) -> SafetensorsFile:
        try:
            return self._where[name]
        except KeyError:
            raise CheckpointError(f"no tensor {name!r} in "
                                  f"{[f.path for f in self.files]}") from None

    def tensor(self, name: str, shape: Optional[Tuple[int, ...]] = None,
               dtypes: Optional[Iterable[str]] = None) -> np.ndarray:
        f = self.file_of(name)
        if dtypes is not None and f.dtype(name) not in dtypes:
            raise CheckpointError(f"{f.path}: tensor {name!r} is {f.dtype(name)}, "
                                  f"expected one of {sorted(dtypes)}")
        t = f.tensor(name)
        if shape is not None and t.shape != tuple(shape):
            raise CheckpointError(f"{f.path}: tensor {name!r} has shape {t.shape}, "
                                  f"expected {tuple(shape)}")
        return t


def write_safetensors(path: str, tensors: Dict[str, Tuple[str, np.ndarray]],
                      metadata: Optional[Dict[str, str]] = None) -> None:
    """Write {name: (dtype string, array)} as one safetensors file (arrays in
    row-major order; BF16 arrays given as uint16 bits)."""
    header: dict = {}
    if metadata:
        header["__metadata__"] = dict(metadata)
    blobs, off = [], 0
    for name, (dt, a) in tensors.items():
        a = np.ascontiguousarray(a, dtype=_ST_DTYPES[dt])
        b = a.tobytes()
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def _as_int(cfg: dict, key: str, default=None) -> int:
    v = cfg.get(key, default)
    if v is None:
        raise CheckpointError(f"config has no {key!r}")
    return int(v)


def gptoss_layer_from_safetensors(ckpt: SafetensorsCheckpoint, config: Union[dict, str],
                                  layer: int) -> GptOssLayer:
    """MoE block ``layer`` of a safetensors GPT-OSS checkpoint, as ``OssMoEFFN::load``
    reads it (gpt_oss.rs:115-142).  ``config`` is the HF config dict or the
    path of its ``config.json`` (hidden_size, intermediate_size,
    num_local_experts, num_experts_per_tok, swiglu_limit default 7.0,
    gpt_oss.rs:56-80).  Router and expert biases keep their stored dtype:
    BF16 arrive as uint16 bits, F32 as float32 (F16 is widened to float32)."""
    if not isinstance(config, dict):
        with open(config) as f:
            config = json.load(f)
    H = _as_int(config, "hidden_size")
    I = _as_int(config, "intermediate_size")
    E = _as_int(config, "num_local_experts")
    k = _as_int(config, "num_experts_per_tok")
    limit = float(config.get("swiglu_limit", 7.0))
    if H % 32 or I % 32:
        raise CheckpointError(f"hidden {H} and intermediate {I} must be multiples of 32 (MXFP4)")
    n_layers = config.get("num_hidden_layers")
    if n_layers is not None and not 0 <= layer < int(n_layers):
        raise CheckpointError(f"layer {layer} outside 0..{int(n_layers) - 1}")
    ex = f"model.layers.{layer}.mlp.experts."
    rt = f"model.layers.{layer}.mlp.router."
    u8 = ("U8",)
    gu_blocks = ckpt.tensor(ex + "gate_up_proj_blocks", (E, 2 * I, H // 32, 16), u8)
    gu_scales = ckpt.tensor(ex + "gate_up_proj_scales", (E, 2 * I, H // 32), u8)
    gu_bias = _st_float(ckpt, ex + "gate_up_proj_bias", (E, 2 * I))
    dn_blocks = ckpt.tensor(ex + "down_proj_blocks", (E, H, I // 32, 16), u8)
    dn_scales = ckpt.tensor(ex + "down_proj_scales", (E, H, I // 32), u8)
    dn_bias = _st_float(ckpt, ex + "down_proj_bias", (E, H))
    router_w = _st_float(ckpt, rt + "weight", (E, H))
    router_b = _st_float(ckpt, rt + "bias", (E,))
    return GptOssLayer(H, I, E, k, limit, router_w, router_b, gu_blocks, gu_scales, gu_bias,
                       dn_blocks, dn_scales, dn_bias,
                       meta={"source": [f.path for f in ckpt.files], "layer": layer})


def _st_float(ckpt: SafetensorsCheckpoint, name: str, shape) -> np.ndarray:
    t = ckpt.tensor(name, shape, ("BF16", "F32", "F16"))
    return t.astype(np.float32) if t.dtype == np.float16 else t


# ---- GGUF ---------------------------------------------------------------------

GGUF_MAGIC = 0x46554747  # "GGUF" read little-endian
GGML_F32, GGML_F16, GGML_Q4_K, GGML_BF16, GGML_MXFP4 = 0, 1, 12, 30, 39
# (elements per block, bytes per block) of the types this module reads.
_GGML_BLOCKS = {GGML_F32: (1, 4), GGML_F16: (1, 2), GGML_BF16: (1, 2),
                GGML_Q4_K: (256, 144), GGML_MXFP4: (32, 17)}
_GGML_NAMES = {GGML_F32: "F32", GGML_F16: "F16", GGML_Q4_K: "Q4_K", GGML_BF16: "BF16",
               GGML_MXFP4: "MXFP4"}

# GGUF metadata value types: id -> struct format of a scalar.
_GV_SCALARS = {0: "B", 1: "b", 2: "H", 3: "h", 4: "I", 5: "i", 6: "f", 7: "?", 10: "Q",
               11: "q", 12: "d"}
_GV_STRING, _GV_ARRAY = 8, 9


class _Reader:
    def __init__(self, buf, path):
        self.buf, self.pos, self.path = buf, 0, path

    def take(self, n: int) -> bytes:
        if n < 0 or self.pos + n > len(self.buf):
            raise CheckpointError(f"{self.path}: header runs past the end of the file "
                                  f"(offset {self.pos}, {n} more bytes)")
        b = bytes(self.buf[self.pos:self.pos + n])
        self.pos += n
        return b

    def scalar(self, fmt: str):
        return struct.unpack("<" + fmt, self.take(struct.calcsize(fmt)))[0]


class GgufFile:
    """A GGUF file's metadata, tensor table and memory-mapped data."""

    def __init__(self, path: str):
        self.path = path
        size = _file_size(path)
        if size < 16:
            raise CheckpointError(f"{path}: {size} bytes, too short for GGUF")
        self._mm = np.memmap(path, dtype=np.uint8, mode="r")
        r = _Reader(self._mm, path)
        magic = r.scalar("I")
        if magic not in (GGUF_MAGIC, 0x47475546):
            raise CheckpointError(f"{path}: unknown GGUF magic 0x{magic:08x}")
        self.version = r.scalar("I")
        if self.version not in (1, 2, 3):
            raise CheckpointError(f"{path}: unknown GGUF version {self.version}")
        cnt = "I" if self.version == 1 else "Q"
        n_tensors, n_kv = r.scalar(cnt), r.scalar(cnt)
        self.metadata: Dict[str, object] = {}
        for _ in range(n_kv):
            key = self._string(r)
            self.metadata[key] = self._value(r, r.scalar("I"))
        self.tensors: Dict[str, Tuple[Tuple[int, ...], int, int]] = {}
        for _ in range(n_tensors):
            name = self._string(r)
            nd = r.scalar("I")
            if nd > 8:
                raise CheckpointError(f"{path}: tensor {name!r} has {nd} dimensions")
            dims = tuple(int(r.scalar(cnt)) for _ in range(nd))[::-1]  # row-major
            ttype, off = r.scalar("I"), r.scalar("Q")
            self.tensors[name] = (dims, ttype, off)
        align = self.metadata.get("general.alignment", 32)
        if not isinstance(align, int) or align <= 0:
            raise CheckpointError(f"{path}: general.alignment {align!r} is not a positive integer")
        self.alignment = align
        self.data_offset = -(-r.pos // align) * align
        self.size = size

    def _string(self, r: _Reader) -> str:
        n = r.scalar("I" if self.version == 1 else "Q")
        return r.take(n).decode("utf-8", errors="replace")

    def _value(self, r: _Reader, vt: int):
        if vt in _GV_SCALARS:
            return r.scalar(_GV_SCALARS[vt])
        if vt == _GV_STRING:
            return self._string(r)
        if vt == _GV_ARRAY:
            et = r.scalar("I")
            n = r.scalar("I" if self.version == 1 else "Q")
            if et in _GV_SCALARS:  # read scalar arrays in one go
                fmt = _GV_SCALARS[et]
                return list(struct.unpack(f"<{n}{fmt}", r.take(n * struct.calcsize(fmt))))
            return [self._value(r, et) for _ in range(n)]
        raise CheckpointError(f"{self.path}: unknown metadata value type {vt}")

    # -- metadata ---------------------------------------------------------------
    @property
    def architecture(self) -> str:
        a = self.metadata.get("general.architecture")
        if not isinstance(a, str):
            raise CheckpointError(f"{self.path}: no general.architecture")
        return a

    def get_int(self, key: str, default: Optional[int] = None) -> int:
        v = self.metadata.get(key, default)
        if v is None or isinstance(v, (str, list)):
            raise CheckpointError(f"{self.path}: metadata {key!r} missing or not a number")
        return int(v)

    def get_float(self, key: str, default: Optional[float] = None) -> float:
        v = self.metadata.get(key, default)
        if v is None or isinstance(v, (str, list)):
            raise CheckpointError(f"{self.path}: metadata {key!r} missing or not a number")
        return float(v)

    # -- tensors ----------------------------------------------------------------
    def __contains__(self, name: str) -> bool:
        return name in self.tensors

    def moe_blocks(self) -> List[int]:
        """Indices i of the blocks with merged expert tensors
        (``blk.{i}.ffn_gate_exps.weight``), ascending; dense blocks are absent."""
        return _block_indices(self.tensors, "blk.", ".ffn_gate_exps.weight")

    def info(self, name: str) -> Tuple[Tuple[int, ...], int, int]:
        try:
            return self.tensors[name]
        except KeyError:
            raise CheckpointError(f"{self.path}: no tensor {name!r}") from None

    def raw(self, name: str, types: Iterable[int]) -> Tuple[np.ndarray, Tuple[int, ...], int]:
        """(bytes as a uint8 view [rows, bytes per row], row-major dims, type) of
        a tensor whose GGML type is in ``types``."""
        dims, ttype, off = self.info(name)
        types = tuple(types)
        if ttype not in types:
            have = _GGML_NAMES.get(ttype, f"GGML type {ttype}")
            want = ", ".join(_GGML_NAMES[t] for t in types)
            raise CheckpointError(f"{self.path}: tensor {name!r} is {have}; this library takes "
                                  f"{want} here")
        per_block, block_bytes = _GGML_BLOCKS[ttype]
        inner = dims[-1] if dims else 1
        if inner % per_block:
            raise CheckpointError(f"{self.path}: tensor {name!r} rows of {inner} elements are not "
                                  f"whole {_GGML_NAMES[ttype]} blocks of {per_block}")
        row_bytes = inner // per_block * block_bytes
        rows = math.prod(dims[:-1])  # Python ints: no wrap-around on damaged dims
        begin = self.data_offset + off
        end = begin + rows * row_bytes
        if off % self.alignment or end > self.size:
            raise CheckpointError(f"{self.path}: tensor {name!r} at data offset {off} "
                                  f"({rows * row_bytes} B) is misaligned or past the end of the "
                                  f"file")
        return self._mm[begin:end].reshape(rows, row_bytes), dims, ttype

    def floats(self, name: str, shape: Optional[Tuple[int, ...]] = None) -> np.ndarray:
        """An F32 / F16 / BF16 tensor as float32 (F32 is a view of the file;
        F16 and BF16 are widened exactly)."""
        b, dims, ttype = self.raw(name, (GGML_F32, GGML_F16, GGML_BF16))
        if shape is not None and dims != tuple(shape):
            raise CheckpointError(f"{self.path}: tensor {name!r} has shape {dims}, expected "
                                  f"{tuple(shape)}")
        flat = b.reshape(-1)
        if ttype == GGML_F32:
            return flat.view(np.float32).reshape(dims)
        if ttype == GGML_F16:
            return flat.view(np.float16).astype(np.float32).reshape(dims)
        return (flat.view(np.uint16).astype(np.uint32) << 16).view(np.float32).reshape(dims)

    def experts(self, name: str, fmt: int, shape: Tuple[int, int, int]) -> np.ndarray:
        """Merged expert tensor [E, rows, K] of GGML type ``fmt`` as raw block
        bytes [E, rows, bytes per row] (quantized.rs:102-130 slices it per expert)."""
        b, dims, _ = self.raw(name, (fmt,))
        if dims != tuple(shape):
            raise CheckpointError(f"{self.path}: tensor {name!r} has shape {dims}, expected "
                                  f"{tuple(shape)}")
        return b.reshape(shape[0], shape[1], b.shape[1])


def _gv_type(v) -> Tuple[int, object]:
    if isinstance(v, bool):
        return 7, v
    if isinstance(v, int):
        return (4, v) if 0 <= v < 2 ** 32 else (11, v)
    if isinstance(v, float):
        return 6, v
    if isinstance(v, str):
        return _GV_STRING, v
    if isinstance(v, (list, tuple)):
        return _GV_ARRAY, list(v)
    raise TypeError(f"cannot store {type(v).__name__} in GGUF metadata")


def _gv_bytes(vt: int, v) -> bytes:
    if vt in _GV_SCALARS:
        return struct.pack("<" + _GV_SCALARS[vt], v)
    if vt == _GV_STRING:
        b = v.encode()
        return struct.pack("<Q", len(b)) + b
    et = _gv_type(v[0])[0] if v else 4
    return struct.pack("<IQ", et, len(v)) + b"".join(_gv_bytes(et, x) for x in v)


def write_gguf(path: str, metadata: Dict[str, object],
               tensors: Dict[str, Tuple[int, Tuple[int, ...], np.ndarray]],
               alignment: int = 32) -> None:
    """Write a GGUF v3 file.  ``metadata`` values: int (u32, or i64 outside
    u32), float (f32), bool, str, or lists of those.  ``tensors``:
    {name: (GGML type, row-major dims, the tensor's bytes in row-major order)}."""
    md = dict(metadata)
    if alignment != 32:
        md["general.alignment"] = alignment
    out = [struct.pack("<IIQQ", GGUF_MAGIC, 3, len(tensors), len(md))]
    for k, v in md.items():
        vt, v = _gv_type(v)
        out.append(_gv_bytes(_GV_STRING, k) + struct.pack("<I", vt) + _gv_bytes(vt, v))
    blobs, off = [], 0
    for name, (ttype, dims, data) in tensors.items():
        b = np.ascontiguousarray(data).tobytes()
        out.append(_gv_bytes(_GV_STRING, name) + struct.pack("<I", len(dims))
                   + b"".join(struct.pack("<Q", d) for d in dims[::-1])
                   + struct.pack("<IQ", ttype, off))
        pad = -len(b) % alignment
        blobs.append(b + b"\0" * pad)
        off += len(b) + pad
    head = b"".join(out)
    head += b"\0" * (-len(head) % alignment)
    with open(path, "wb") as f:
        f.write(head)
        for b in blobs:
            f.write(b)


def _moe_sizes(g: GgufFile, layer: int) -> Tuple[str, int, int, int]:
    arch = g.architecture
    n_layers = g.metadata.get(f"{arch}.block_count")
    if isinstance(n_layers, int) and not 0 <= layer < n_layers:
        raise CheckpointError(f"{g.path}: layer {layer} outside 0..{n_layers - 1}")
    p = f"blk.{layer}."
    if p + "ffn_gate_exps.weight" not in g:
        raise CheckpointError(f"{g.path}: block {layer} has no MoE experts "
                              f"({p}ffn_gate_exps.weight)")
    dims, _, _ = g.info(p + "ffn_gate_exps.weight")
    if len(dims) != 3:
        raise CheckpointError(f"{g.path}: {p}ffn_gate_exps.weight has shape {dims}, expected "
                              f"[n_expert, n_ff, n_embd]")
    E, I, H = dims
    n_exp = g.metadata.get(f"{arch}.expert_count")
    if isinstance(n_exp, int) and n_exp != E:
        raise CheckpointError(f"{g.path}: {arch}.expert_count {n_exp} but the expert tensors hold "
                              f"{E}")
    return p, E, I, H


def gptoss_layer_from_gguf(g: GgufFile, layer: int) -> GptOssGgufLayer:
    """MoE block ``layer`` of a GGUF GPT-OSS file, as ``QMoEFFN::load`` reads it
    (gpt_oss_q.rs:135-163; top-k and clamp from metadata, defaults 4 and 7.0 as
    gpt_oss_q.rs:344-349).  Experts stay raw MXFP4 blocks; router and biases
    are float32."""
    p, E, I, H = _moe_sizes(g, layer)
    arch = g.architecture
    k = g.get_int(f"{arch}.expert_used_count", 4)
    limit = g.get_float(f"{arch}.swiglu_limit", 7.0)
    gate = g.experts(p + "ffn_gate_exps.weight", GGML_MXFP4, (E, I, H))
    up = g.experts(p + "ffn_up_exps.weight", GGML_MXFP4, (E, I, H))
    down = g.experts(p + "ffn_down_exps.weight", GGML_MXFP4, (E, H, I))
    router_w = g.floats(p + "ffn_gate_inp.weight", (E, H))
    router_b = g.floats(p + "ffn_gate_inp.bias", (E,)) if p + "ffn_gate_inp.bias" in g else None
    gate_b = g.floats(p + "ffn_gate_exps.bias", (E, I))
    up_b = g.floats(p + "ffn_up_exps.bias", (E, I))
    down_b = g.floats(p + "ffn_down_exps.bias", (E, H))
    base = GptOssLayer(H, I, E, k, limit, router_w, router_b, None, None, None, None, None, None,
                       meta={"source": g.path, "layer": layer})
    return GptOssGgufLayer(base, gate, up, down, gate_b, up_b, down_b)


def lfm2_layer_from_gguf(g: GgufFile, layer: int) -> Lfm2Layer:
    """MoE block ``layer`` of a GGUF LFM2.5 file, as ``QMoEFFN::load`` reads it
    (lfm2moe_q.rs:214-232): Q4_K experts, router, selection bias
    ``exp_probs_b.bias`` (zeros when absent).  Dense leading blocks
    (lfm2moe_q.rs:436-440) are refused."""
    arch = g.architecture
    lead = g.get_int(f"{arch}.leading_dense_block_count", 0)
    if layer < lead:
        raise CheckpointError(f"{g.path}: block {layer} is one of the {lead} leading dense blocks")
    p, E, I, H = _moe_sizes(g, layer)
    k = g.get_int(f"{arch}.expert_used_count")
    gate = g.experts(p + "ffn_gate_exps.weight", GGML_Q4_K, (E, I, H))
    up = g.experts(p + "ffn_up_exps.weight", GGML_Q4_K, (E, I, H))
    down = g.experts(p + "ffn_down_exps.weight", GGML_Q4_K, (E, H, I))
    router_w = g.floats(p + "ffn_gate_inp.weight", (E, H))
    if p + "exp_probs_b.bias" in g:
        sel = g.floats(p + "exp_probs_b.bias", (E,))
    else:
        sel = np.zeros(E, np.float32)
    return Lfm2Layer(H, I, E, k, router_w, sel, gate, up, down,
                     meta={"source": g.path, "layer": layer})
