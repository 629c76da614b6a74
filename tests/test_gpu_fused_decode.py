"""The fused decode path (GB_PATH_FUSED_DECODE: the whole layer in one
cooperative launch, T <= 8)
against the oracle and against the separate tensor-core kernels: expert
indices bit for bit, outputs within max-abs 2e-2 and mean-rel 1e-3, at every
batch size it takes (1-8 tokens), with 32 and 128 experts, safetensors and
GGUF MXFP4 (whose combine runs in expert order).  Repeated forwards are
bit-identical."""
import numpy as np
import pytest

import oracle
from gallium_b200 import GptOssQMoEFFN, OssMoEFFN, synth

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_REL = 2e-2, 1e-3


def _check(got, want):
    err = np.abs(got.astype(np.float64) - want)
    assert err.max() <= MAX_ABS and err.sum() / np.abs(want).sum() <= MEAN_REL, err.max()


@pytest.mark.parametrize("E,gguf", [(32, False), (128, False), (32, True)])
def test_fused_decode_matches_oracle_and_the_tensor_core_path(E, gguf):
    import torch

    layer = synth.gptoss_layer(n_experts=E, seed=E)
    if gguf:
        gl = synth.gptoss_gguf_from_split(layer)
        moe = GptOssQMoEFFN.load(gl, device=0, max_tokens=8)
        orc = oracle.OracleMoe(layer, gguf=gl)
    else:
        moe = OssMoEFFN.load(layer, device=0, max_tokens=8)
        orc = oracle.OracleMoe(layer)
    try:
        for T in range(1, 9):
            x = torch.from_numpy(synth.tokens(T, 2880, seed=100 + T)).cuda()
            moe.set_expert_path("fused_decode")
            fused = moe.forward(x).cpu().numpy()
            again = moe.forward(x).cpu().numpy()
            assert np.array_equal(fused, again), T
            moe.set_expert_path("tensor_cores")
            tc = moe.forward(x).cpu().numpy()
            want, idx, _ = orc.forward(x.cpu().numpy())
            _check(fused, want)
            _check(tc, want)
            assert np.array_equal(moe.route(x)["idx"].cpu().numpy(), idx)
    finally:
        moe.close()
