"""The reference's grouped CPU forward, restated for timing on the host cores.

TEST INFRASTRUCTURE ONLY: bench.py times this as the CPU baseline and as the
reference arm (`--impl reference`); tests check it against the oracle.  The
product path never imports it.

It follows QMoEFFN::forward of crates/gallium-models/src/gpt_oss_q.rs:165-269
(and lfm2moe_q.rs:234-313 for LFM2.5), the reference's fastest CPU path:
  router logits (one matrix product, gpt_oss_q.rs:168), softmax or sigmoid
  top-k and the per-expert token lists (:169-192), then per active expert:
  dequantise its weights once (:203-209), gather its tokens, gate/up product
  with biases, the activation, down product with bias (:218-241), scale rows
  by their routing weights (:244-246), and add each token's rows (:252-266).
Active experts run in parallel on a pool of host threads, as
par_map_on_cpu spreads them over rayon's threads (device.rs:91-108); an
expert with more than CHUNK_ROWS tokens is split into several tasks so that
skewed routing still uses every core.  The matrix products run in OpenBLAS's
f32 GEMM through numpy (one BLAS thread per task), standing in for candle's
CPU matmul (the `gemm` crate, a blocked f32 GEMM of the same kind);
dequantisation, activation and top-k run in the oracle's C code.

gallium-core's generic MoEFFN (crates/gallium-core/src/ffn.rs:125-166: dense
gated experts, softmax top-k renormalised, an optional shared expert over
all tokens added after the routed sum) takes the same grouped form here.
The reference itself runs that block token by token (ffn.rs:139-157), so
this restatement times faster than the reference would: a conservative
baseline.
"""
from __future__ import annotations

import ctypes
import os
import threading
import time
from concurrent.futures import ThreadPoolExecutor

import numpy as np

from . import (OracleDense, OracleLfm2, OracleMoe, OrDesc, _p, lib, permute, route_sigmoid_topk,
               route_softmax_topk)

CHUNK_ROWS = 512


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


class CpuReference:
    """Runs the grouped CPU forward of one layer (GPT-OSS MXFP4 in the
    safetensors layout, LFM2.5 Q4_K, or the generic MoEFFN with dense
    experts) on `n_threads` host threads."""

    def __init__(self, layer, n_threads: int = 0):
        self.lfm2 = hasattr(layer, "sel_bias")
        self.dense = hasattr(layer, "shared_inter")
        self.orc = (OracleLfm2(layer) if self.lfm2 else
                    OracleDense(layer) if self.dense else OracleMoe(layer))
        self.layer = layer
        self.n_threads = n_threads if n_threads > 0 else host_threads()
        d = self.orc.desc
        self.H, self.I, self.E, self.k = d.hidden, d.inter, d.n_experts, d.top_k
        keep = self.orc._keep
        plain = self.lfm2 or self.dense  # no router or expert biases
        self.rw = np.ascontiguousarray(keep["router_w"] if plain else keep["rw"], np.float32)
        self.rb = None if plain else keep["rb"]
        self.gub = None if plain else keep.get("gub")
        self.dnb = None if plain else keep.get("db")
        self.Is = layer.shared_inter if self.dense else 0
        if self.Is:
            # the shared expert's activation: the experts' kind, its own width
            self.sh_desc = OrDesc.from_buffer_copy(d)
            self.sh_desc.inter = self.Is
        self.sel_bias = layer.sel_bias if self.lfm2 else None
        self._tls = threading.local()
        self._pool = ThreadPoolExecutor(self.n_threads)

    def close(self):
        self._pool.shutdown()

    # -- one task: rows [a, b) of expert e's grouped positions --------------------
    def _buffers(self):
        t = self._tls
        if not hasattr(t, "w"):
            H, I = self.H, self.I
            if self.lfm2:
                t.w = (np.empty((I, H), np.float32), np.empty((I, H), np.float32),
                       np.empty((H, I), np.float32))
            else:
                t.w = (np.empty((2 * I, H), np.float32), np.empty((H, I), np.float32))
        return t.w

    def _dequant(self, which, expert, out):
        if lib().or_dequant_expert_matrix(ctypes.byref(self.orc.desc), which, expert, _p(out), 1):
            raise RuntimeError(lib().or_last_error().decode())

    def _task(self, e, a, b, x, perm, wflat, y):
        H, I, k = self.H, self.I, self.k
        ent = perm[a:b]
        xe = x[ent // k]
        h = np.empty((xe.shape[0], I), np.float32)
        desc = ctypes.byref(self.orc.desc)
        if self.dense:
            kp = self.orc._keep
            g = xe @ kp["gate"][e].T
            u = xe @ kp["up"][e].T
            lib().or_act_rows(desc, _p(g), _p(u), g.shape[0], I, _p(h), 1)
            wd = kp["down"][e]
        elif self.lfm2:
            wg, wu, wd = self._buffers()
            self._dequant(0, e, wg)
            self._dequant(1, e, wu)
            self._dequant(2, e, wd)
            g = xe @ wg.T
            u = xe @ wu.T
            lib().or_act_rows(desc, _p(g), _p(u), g.shape[0], I, _p(h), 1)
        else:
            wgu, wd = self._buffers()
            self._dequant(0, e, wgu)
            self._dequant(2, e, wd)
            gu = xe @ wgu.T
            if self.gub is not None:
                gu += self.gub[e]
            base = gu.ctypes.data
            lib().or_act_rows(desc, base, base + 4, gu.shape[0], 2 * I, _p(h), 1)
        ye = h @ wd.T
        if self.dnb is not None:
            ye += self.dnb[e]
        ye *= wflat[ent][:, None]
        y[a:b] = ye

    def _shared_task(self, a, b, x, sh):
        kp = self.orc._keep
        g = x[a:b] @ kp["sh_gate"].T
        u = x[a:b] @ kp["sh_up"].T
        h = np.empty((b - a, self.Is), np.float32)
        lib().or_act_rows(ctypes.byref(self.sh_desc), _p(g), _p(u), b - a, self.Is, _p(h), 1)
        sh[a:b] = h @ kp["sh_down"].T

    def forward(self, x: np.ndarray, timings: dict | None = None) -> np.ndarray:
        """x [T, H] f32 -> out [T, H] f32.  `timings` (optional) receives the
        seconds spent in routing, experts and combine."""
        from threadpoolctl import threadpool_limits

        H, E, k = self.H, self.E, self.k
        x = np.ascontiguousarray(x, np.float32)
        T = x.shape[0]
        t0 = time.perf_counter()
        logits = x @ self.rw.T
        if self.rb is not None:
            logits += self.rb
        if self.lfm2:
            idx, w = route_sigmoid_topk(logits, self.sel_bias, k)
        else:
            idx, w = route_softmax_topk(logits, k)
        counts, offsets, perm, inv = permute(idx, E)
        t1 = time.perf_counter()
        y = np.empty((T * k, H), np.float32)  # rows in grouped order
        wflat = w.reshape(-1)
        tasks = []
        for e in np.nonzero(counts)[0]:
            a, b = int(offsets[e]), int(offsets[e + 1])
            for c in range(a, b, CHUNK_ROWS):
                tasks.append((int(e), c, min(b, c + CHUNK_ROWS)))
        sh = np.empty((T, H), np.float32) if self.Is else None
        with threadpool_limits(1, user_api="blas"):
            futs = [self._pool.submit(self._task, e, a, b, x, perm, wflat, y)
                    for e, a, b in tasks]
            if sh is not None:  # the shared expert over every token
                futs += [self._pool.submit(self._shared_task, c, min(T, c + CHUNK_ROWS), x, sh)
                         for c in range(0, T, CHUNK_ROWS)]
            for f in futs:
                f.result()
        t2 = time.perf_counter()
        # each token adds its k rows: in rank order for the safetensors layer
        # (gpt_oss.rs:223), in expert order for LFM2.5 (lfm2moe_q.rs:303-311)
        rows = inv.reshape(T, k)
        if self.lfm2:
            rows = np.take_along_axis(rows, np.argsort(idx, axis=1, kind="stable"), axis=1)
        out = y[rows[:, 0]].copy()
        for r in range(1, k):
            out += y[rows[:, r]]
        if sh is not None:  # after the routed sum (ffn.rs:160-163)
            out += sh
        t3 = time.perf_counter()
        if timings is not None:
            timings.update(route=t1 - t0, experts=t2 - t1, combine=t3 - t2,
                           active_experts=int((counts > 0).sum()), tasks=len(tasks))
        return out
