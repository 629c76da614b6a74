"""gallium_b200: the rs-gallium MoE FFN block on B200 (sm_100a), behind a C ABI.

Public surface:
  OssMoEFFN, GptOssQMoEFFN, Lfm2QMoEFFN, MoEFFN, QGemmaMoe -- the reference's MoE blocks
  GptOssQ                   -- the GGUF GPT-OSS decode stack around the MoE block
  synth                     -- seeded synthetic layers and inputs
  weights                   -- layers read from safetensors / GGUF checkpoint files
  GalliumError              -- raised for any non-OK gb_status
"""
from ._lib import GalliumError, load_library  # noqa: F401
from .moe import (GptOssQMoEFFN, Lfm2QMoEFFN, MoEBlock, MoEFFN, OssMoEFFN,  # noqa: F401
                  QGemmaMoe, nccl_unique_id)
from .decoder import GptOssQ  # noqa: F401
from . import synth, weights  # noqa: F401
