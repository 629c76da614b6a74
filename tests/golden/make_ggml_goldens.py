"""Generate tests/golden/ggml_decode_goldens.npz: GGML block decodes computed by
gguf-py, llama.cpp's Python implementation of the GGML formats (package
``gguf`` 0.19.0, ``gguf.quants.dequantize``).

The reference decodes Q4_K through its dependency candle-core 0.10.2 (git rev
097655a2; called at crates/gallium-core/src/quantized.rs:174-176) and GGUF
MXFP4 (GGML type 39) in its own code (quantized.rs:361-449).  Neither can run
here (no Rust toolchain, candle not vendored), and no reference test pins
Q4_K.  gguf-py is an independent implementation of the same published block
formats, so its outputs pin the oracle's decoders on these inputs:

* Q4_K: 64 seeded 144-byte super-blocks; d and dmin f16 values spread over
  zero, f16 subnormals, negatives and large magnitudes; 6-bit scales / mins
  and 4-bit codes uniform.
* MXFP4 (type 39): 256 seeded 17-byte blocks, block b carrying E8M0 byte b
  (every exponent, including 0 and 1, which decode to subnormals, and 255,
  whose large codes overflow to infinity), codes uniform.

Run from the repository root:  python tests/golden/make_ggml_goldens.py
"""
import os
from importlib.metadata import version

import numpy as np

import gguf
from gguf import quants

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "ggml_decode_goldens.npz")


def q4k_inputs(rng) -> np.ndarray:
    n = 64
    blk = rng.integers(0, 256, (n, 144), dtype=np.uint8)
    d = rng.normal(0.0, 1e-2, n).astype(np.float16)
    dmin = rng.normal(0.0, 1e-2, n).astype(np.float16)
    d[0], dmin[1] = 0, 0                                  # zero scale, zero min
    d[2], dmin[3] = np.float16(6e-8), np.float16(-6e-8)    # f16 subnormals
    d[4], dmin[4] = np.float16(-0.25), np.float16(0.125)   # negative d
    d[5], dmin[5] = np.float16(1000.0), np.float16(-500.0)  # large magnitudes
    blk[:, 0:2] = d.view(np.uint8).reshape(n, 2)
    blk[:, 2:4] = dmin.view(np.uint8).reshape(n, 2)
    return blk


def mxfp4_inputs(rng) -> np.ndarray:
    blk = rng.integers(0, 256, (256, 17), dtype=np.uint8)
    blk[:, 0] = np.arange(256, dtype=np.uint8)
    return blk


def main() -> None:
    rng = np.random.default_rng(20260101)
    q4k = q4k_inputs(rng)
    mx = mxfp4_inputs(rng)
    with np.errstate(over="ignore"):
        q4k_out = quants.dequantize(q4k.reshape(-1), gguf.GGMLQuantizationType.Q4_K)
        mx_out = quants.dequantize(mx.reshape(-1), gguf.GGMLQuantizationType.MXFP4)
    np.savez_compressed(OUT, q4k_blocks=q4k, q4k_values=q4k_out.astype(np.float32).reshape(-1),
                        mxfp4_blocks=mx, mxfp4_values=mx_out.astype(np.float32).reshape(-1),
                        gguf_version=np.array(version("gguf")))
    print(f"wrote {OUT}")


if __name__ == "__main__":
    main()
