"""The timed CPU port of the reference's grouped forward (oracle/cpu_reference.py)
against the oracle: same routing, outputs within the path's tolerance.  It is
the CPU baseline bench.py reports, so it must compute the same layer."""
import numpy as np
import pytest

import oracle
from oracle import cpu_reference
from gallium_b200 import synth

MAX_ABS, MEAN_REL = 2e-2, 1e-3


def _check(got, want):
    err = np.abs(got.astype(np.float64) - want)
    assert err.max() <= MAX_ABS and err.sum() / np.abs(want).sum() <= MEAN_REL


@pytest.mark.parametrize("skewed", [False, True])
def test_gptoss_grouped_forward_matches_oracle(skewed, monkeypatch):
    # small chunks so that the busiest experts are split across tasks
    monkeypatch.setattr(cpu_reference, "CHUNK_ROWS", 16)
    layer = synth.gptoss_layer(n_experts=8, hidden=256, inter=192, top_k=4, seed=3,
                               skewed=skewed)
    x = synth.tokens(120, 256, seed=4)
    ref = cpu_reference.CpuReference(layer, n_threads=3)
    try:
        tm = {}
        got = ref.forward(x, tm)
    finally:
        ref.close()
    want, _, _ = oracle.OracleMoe(layer).forward(x)
    _check(got, want)
    assert tm["tasks"] > tm["active_experts"]


def test_lfm2_grouped_forward_matches_oracle():
    layer = synth.lfm2_layer(n_experts=4, hidden=256, inter=256, top_k=2, seed=1)
    x = synth.tokens(50, 256, seed=2)
    ref = cpu_reference.CpuReference(layer, n_threads=2)
    try:
        got = ref.forward(x)
    finally:
        ref.close()
    want, _, _ = oracle.OracleLfm2(layer).forward(x)
    _check(got, want)


@pytest.mark.parametrize("act_kind, clamp, shared", [(1, 0.0, 128), (3, 6.0, 128), (4, 0.0, 0)])
def test_dense_moeffn_grouped_forward_matches_oracle(act_kind, clamp, shared, monkeypatch):
    # gallium-core's generic MoEFFN: dense experts, SiLU / GELU-tanh with a
    # clamp / ReLU, with and without the shared expert; small chunks so that
    # experts and the shared expert are split across tasks
    monkeypatch.setattr(cpu_reference, "CHUNK_ROWS", 16)
    layer = synth.dense_layer(n_experts=8, hidden=256, inter=192, top_k=2,
                              shared_inter=shared, act_kind=act_kind, act_clamp=clamp, seed=5)
    x = synth.tokens(70, 256, seed=6)
    ref = cpu_reference.CpuReference(layer, n_threads=3)
    try:
        got = ref.forward(x)
    finally:
        ref.close()
    want, _, _ = oracle.OracleDense(layer).forward(x)
    _check(got, want)
