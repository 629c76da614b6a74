"""The router's exp (rs-gallium_b200/csrc/exp_f32.h) against the oracle's.

Expert selection ranks softmax (or sigmoid) probabilities and breaks exact
ties by the lower index (gpt_oss.rs:174-182, lfm2moe_q.rs:241-258), so the
kernel's exp must give the same f32 as the oracle's for every argument the
router can produce.  The kernel's exp is compiled here for the host from the
same header (g++, no GPU) and compared with the correctly rounded value the
oracle uses, (float)expl(x), over a strided sweep of every f32 in
[-104, 90] (the range where exp is neither 0 nor inf).  Setting
GB_EXP_SWEEP_STRIDE=1 sweeps every one of the 2,240,020,482 arguments.

Also here: the crafted near-tie cases, where two logits one unit in the last
place apart give the same probability and the lower index must win although
its logit is the smaller.
"""
import ctypes
import os
import subprocess

import numpy as np
import pytest

import oracle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "rs-gallium_b200", "csrc", "exp_f32.h")

HARNESS = r"""
#include "%s"
#include <math.h>
#include <stdint.h>
#include <string.h>
static float from_bits(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }
static uint32_t to_bits(float f) { uint32_t b; memcpy(&b, &f, 4); return b; }
extern "C" float kernel_exp(float x) { return gb::exp_f32(x); }
// Bit patterns a, a + stride, ... <= b (one sign): counts of arguments where
// the kernel's exp differs from (float)expl(x), and where glibc's expf does.
extern "C" void sweep(uint32_t a, uint32_t b, uint32_t stride, int64_t* out) {
  int64_t n = 0, bad = 0, glibc = 0;
  #pragma omp parallel for reduction(+:n, bad, glibc) schedule(static, 4096)
  for (int64_t u = a; u <= (int64_t)b; u += stride) {
    const float x = from_bits((uint32_t)u);
    const uint32_t want = to_bits((float)expl((long double)x));
    n++;
    bad += to_bits(gb::exp_f32(x)) != want;
    glibc += to_bits(expf(x)) != want;
  }
  out[0] = n; out[1] = bad; out[2] = glibc;
}
"""


@pytest.fixture(scope="module")
def harness(tmp_path_factory):
    d = tmp_path_factory.mktemp("exp")
    src = d / "exp_harness.cpp"
    src.write_text(HARNESS % HEADER)
    so = d / "libexp_harness.so"
    subprocess.run(["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-fopenmp",
                    "-ffp-contract=off", "-march=x86-64-v3", str(src), "-o", str(so)],
                   check=True)
    lib = ctypes.CDLL(str(so))
    lib.kernel_exp.restype = ctypes.c_float
    lib.kernel_exp.argtypes = [ctypes.c_float]
    lib.sweep.restype = None
    lib.sweep.argtypes = [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                          ctypes.POINTER(ctypes.c_int64)]
    return lib


def _bits(v: float) -> int:
    return int(np.array([v], np.float32).view(np.uint32)[0])


def test_kernel_exp_is_the_oracles_exp_on_a_sweep(harness):
    stride = int(os.environ.get("GB_EXP_SWEEP_STRIDE", "127"))
    out = (ctypes.c_int64 * 3)()
    total = bad = glibc = 0
    # negative arguments -0 .. -104, then +0 .. 90
    for a, b in ((0x80000000, _bits(-104.0)), (0, _bits(90.0))):
        harness.sweep(a, b, stride, out)
        total, bad, glibc = total + out[0], bad + out[1], glibc + out[2]
    assert total > 2_240_020_482 // stride - 4
    assert bad == 0, f"{bad} of {total} arguments differ from the correctly rounded exp"
    print(f"{total} arguments: kernel exp == oracle exp on all; glibc expf differs on {glibc}")


def test_kernel_exp_special_values(harness):
    f = harness.kernel_exp
    assert f(0.0) == 1.0 and f(-0.0) == 1.0
    assert f(89.5) == float("inf") and f(-104.5) == 0.0 and f(-1000.0) == 0.0
    assert np.isnan(f(float("nan")))
    assert f(float("inf")) == float("inf") and f(float("-inf")) == 0.0
    # the subnormal range rounds once, like the oracle
    for x in (-87.5, -95.0, -100.0, -103.9):
        assert _bits(f(x)) == _bits(oracle.exp_rn(x)), x
    for x in np.random.default_rng(3).uniform(-30, 30, 2000).astype(np.float32):
        assert _bits(f(float(x))) == _bits(oracle.exp_rn(float(x))), x


def near_tie_logits():
    """Logits of 8 experts where experts 2 and 5 hold adjacent f32 values,
    expert 5 the larger, with equal softmax probabilities: v - 3 and v' - 3
    round to the same f32 (ulp 2^-22 there against 2^-24 for v).  Expert 6 is
    clearly first, so top-2 picks between 2 and 5."""
    v = np.float32(0.75) + np.float32(2.0 ** -24)
    v2 = np.nextafter(v, np.float32(np.inf))
    lg = np.full(8, -4.0, np.float32)
    lg[6], lg[2], lg[5] = 3.0, v, v2
    return lg


def near_tie_division_logits():
    """Adjacent probabilities from distinct exps: a case where exp(l - max)
    differ in the last place but their quotients by the row sum are equal,
    found by search over adjacent logit pairs near the top of a small row."""
    rng = np.random.default_rng(11)
    for _ in range(20000):
        base = rng.uniform(-3.0, -1.5, 6).astype(np.float32)
        v = np.float32(rng.uniform(-1.0, 0.0))
        v2 = np.nextafter(v, np.float32(np.inf))
        lg = np.concatenate([[np.float32(1.5)], base, [v, v2]]).astype(np.float32)
        e = np.array([oracle.exp_rn(float(a - lg.max())) for a in lg], np.float32)
        if e[-2] == e[-1]:
            continue
        s = np.float32(0)
        for q in e:
            s = np.float32(s + q)
        if np.float32(e[-2] / s) == np.float32(e[-1] / s):
            return lg
    pytest.skip("no division near-tie found")


def test_oracle_near_tie_takes_the_lower_index():
    lg = near_tie_logits()
    assert lg[5] > lg[2]
    idx, w = oracle.route_softmax_topk(lg[None, :], 2)
    assert idx.tolist() == [[6, 2]]
    # ranking by logits would have chosen expert 5
    assert int(np.argsort(-lg, kind="stable")[1]) == 5


def test_oracle_division_near_tie_takes_the_lower_index():
    lg = near_tie_division_logits()
    E = lg.shape[0]
    idx, _ = oracle.route_softmax_topk(lg[None, :], 2)
    assert idx.tolist() == [[0, E - 2]]
    assert lg[E - 1] > lg[E - 2]
