#!/usr/bin/env python
"""MoE-layer tokens/s on B200: GPT-OSS-120B-shaped MXFP4 MoE layer.

Workload (one step = one forward of the layer over one batch):
  hidden 2880, intermediate 2880, 128 experts, top-4, MXFP4 experts (E2M1
  codes uniform, E8M0 exponents uniform in [-8, -2]), bf16 router ~ N(0, 0.02)
  with zero bias, bf16 biases ~ N(0, 0.01), clamped SwiGLU (limit 7),
  x ~ N(0, 1) f32, seed 0 -- synthetic weights and inputs (no checkpoint).
  Headline batch: --tokens (default 8192) tokens per GPU; --sweep adds the
  other batch sizes of the workload as extra measurements.

The same line carries, under "configs", the workload's other layers:
  20b_balanced / 20b_skewed  the GPT-OSS-20B-shaped block (32 experts,
                             balanced router, or a Zipf(1.2) router bias) at
                             4096 tokens, one GPU only;
  lfm2_q4k                   the LFM2.5-shaped block (hidden 2048, 1792
                             intermediate, 32 experts, top-4, Q4_K experts,
                             sigmoid router) at 1, 16, 64 and 2048 tokens per GPU,
                             expert parallel over the N GPUs when N > 1;
  moeffn_dense               gallium-core's generic MoEFFN with dense bf16
                             experts (a Qwen3-MoE-like shape: hidden 2048,
                             128 experts, top-8, intermediate 768, SiLU) and a
                             512-wide shared expert, at 1, 64 and 2048 tokens
                             per GPU, expert parallel when N > 1;
  gptoss20b_decode           the GPT-OSS-20B-shaped decode stack around the
                             MoE block (24 layers, attention with sinks and a
                             128-token sliding window on even layers, vocab
                             201088): greedy decode of 256 tokens from random
                             128-token prompts at batch 1 and 32, tokens/s and
                             the MoE block's share of a step, one GPU only.
Each with its own roofline and a parity check against the oracle.

Arms:
  default            the CUDA path through the C ABI (gb_moe_forward on
                     device-resident inputs -> "value"; gb_moe_forward_host
                     with pinned host buffers, copies included -> "e2e").
  --impl reference   the reference's grouped CPU forward restated in
                     oracle/cpu_reference.py, on every host core, one whole
                     batch per step (all tokens routed, every active expert
                     run).

Parity: after timing, every rank checks its own forward against the oracle:
expert indices of every token bit for bit, and the output rows of a sample
(rows of the busiest expert plus random rows) within max-abs 2e-2 and
mean-rel 1e-3.  On one GPU the headline batch is also checked row by row
against the CPU baseline's own output of the same batch
("every_row_vs_cpu_forward").  The line's "parity" object has the worst
rank's figures; a failed check prints the line and exits with status 3.

--model lfm2 / dense measures the LFM2.5-shaped or the generic dense layer as
the headline instead.

Multi-GPU (python -m torch.distributed.run ... bench.py --gpus N): one process
per GPU, expert parallel: rank r holds experts [r*E/N, (r+1)*E/N) and its own
batch of --tokens tokens; inside the library the ranks exchange expert counts
by NCCL and move activation rows to the owning rank, and output rows back, by
NVLink peer stores.  Timing = max over ranks, value = all ranks' tokens / that
time (weak scaling).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "rs-gallium_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402

TOPK = 4
L2_BYTES = 126 * 1024 * 1024
MAX_ABS, MEAN_REL = 2e-2, 1e-3


class Model:
    """Shapes, loader and byte counts of one measured MoE layer."""

    def __init__(self, name, experts, skewed=False):
        self.name = name
        self.skewed = skewed
        self.k, self.Is = TOPK, 0
        if name == "gptoss":
            self.H, self.I, self.E = 2880, 2880, experts or 128
            self.metric = "MoE-layer tokens/s (GPT-OSS-120B shape, MXFP4)"
            size = "120b" if self.E == 128 else "20b" if self.E == 32 else f"E{self.E}"
            self.shape = (f"gpt-oss-{size}-shaped MoE layer, E={self.E}, H=I=2880, top-{TOPK}, "
                          f"MXFP4" + (", Zipf(1.2) router bias" if skewed else ""))
        elif name == "lfm2":
            self.H, self.I, self.E = 2048, 1792, experts or 32
            self.metric = "MoE-layer tokens/s (LFM2.5 shape, Q4_K)"
            self.shape = (f"lfm2.5-shaped MoE layer, E={self.E}, H=2048, I=1792, top-{TOPK}, "
                          f"Q4_K, sigmoid router")
        else:  # the generic MoEFFN with dense bf16 experts and a shared expert
            self.H, self.I, self.E, self.k, self.Is = 2048, 768, experts or 128, 8, 512
            self.metric = "MoE-layer tokens/s (generic MoEFFN, dense bf16 experts)"
            self.shape = (f"qwen3-moe-like generic MoEFFN layer, E={self.E}, H=2048, I=768, "
                          f"top-8, SiLU, dense bf16 experts, shared expert 512")

    def layer(self, seed):
        from gallium_b200 import synth
        if self.name == "gptoss":
            return synth.gptoss_layer(n_experts=self.E, seed=seed, skewed=self.skewed)
        if self.name == "lfm2":
            return synth.lfm2_layer(n_experts=self.E, seed=seed)
        return synth.dense_layer(n_experts=self.E, hidden=self.H, inter=self.I, top_k=self.k,
                                 shared_inter=self.Is, seed=seed)

    def load(self, layer, device, max_tokens, ep):
        from gallium_b200 import Lfm2QMoEFFN, MoEFFN, OssMoEFFN
        cls = {"gptoss": OssMoEFFN, "lfm2": Lfm2QMoEFFN, "dense": MoEFFN}[self.name]
        return cls.load(layer, device=device, max_tokens=max_tokens, ep=ep)

    def stage_weight_bytes(self):
        """(gate_up, down) bytes of one expert: codes + scales (+ bf16 biases)."""
        H, I = self.H, self.I
        if self.name == "gptoss":
            return (2 * I * H // 2 + 2 * I * H // 32 + 2 * I * 2, H * I // 2 + H * I // 32 + H * 2)
        if self.name == "lfm2":
            return (2 * I * H // 256 * 144, H * I // 256 * 144)
        return (2 * I * H * 2, H * I * 2)  # bf16

    def oracle(self, layer):
        import oracle
        return {"gptoss": oracle.OracleMoe, "lfm2": oracle.OracleLfm2,
                "dense": oracle.OracleDense}[self.name](layer)

    def route(self, layer, x):
        """Oracle routing of x: idx [T, k]."""
        import oracle
        if self.name == "gptoss":
            rw = (layer.router_w.astype(np.uint32) << 16).view(np.float32)
            rb = (layer.router_b.astype(np.uint32) << 16).view(np.float32)
            idx, _ = oracle.route_softmax_topk(oracle.router_logits(x, rw, rb), TOPK)
            return idx
        if self.name == "dense":
            rw = (layer.router_w.astype(np.uint32) << 16).view(np.float32)
            idx, _ = oracle.route_softmax_topk(oracle.router_logits(x, rw, None), self.k)
            return idx
        lg = oracle.router_logits(x, layer.router_w, None)
        idx, _ = oracle.route_sigmoid_topk(lg, layer.sel_bias, TOPK)
        return idx


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--model", choices=["gptoss", "lfm2", "dense"], default="gptoss")
    ap.add_argument("--experts", type=int, default=0, help="default 128 (gptoss) / 32 (lfm2)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--skewed", action="store_true", help="Zipf(1.2) router bias")
    ap.add_argument("--sweep", default="1,8,32,64,1024",
                    help="extra per-GPU batch sizes to measure ('' = none)")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the 20B-shaped and LFM2.5-shaped layers")
    ap.add_argument("--configs", default="all",
                    help="comma list of the extra layers to run (20b_balanced, 20b_skewed, "
                         "lfm2_q4k, moeffn_dense, gptoss20b_decode), or all")
    ap.add_argument("--decode-batches", default="1,32",
                    help="batches of the gptoss20b_decode config")
    ap.add_argument("--decode-steps", type=int, default=256,
                    help="greedy steps timed in the gptoss20b_decode config")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true")
    ap.add_argument("--parity-rows", type=int, default=64)
    ap.add_argument("--expert-path", default="auto",
                    choices=["auto", "cuda_cores", "tensor_cores", "tensor_cores_f16",
                             "fused_decode"],
                    help="force one expert kernel (gb_moe_set_expert_path)")
    ap.add_argument("--cpu-threads", type=int, default=0)
    return ap.parse_args()


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpu_id, f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def wait_first(self, timeout_s: float = 5.0):
        """Blocks until nvidia-smi printed its first sample (it takes a while
        to start, longer with one sampler per rank), at most timeout_s."""
        t0 = time.time()
        while self.proc is not None and not self.lines and time.time() - t0 < timeout_s:
            time.sleep(0.02)

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------

def dist_setup(args):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def allreduce(world, vals, op="max"):
    """Element-wise max or sum of a list of floats over the ranks."""
    if world == 1:
        return list(vals)
    import torch
    import torch.distributed as dist
    t = torch.tensor(list(vals), dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
    return [float(v) for v in t.cpu()]


def allmax(world, v: float) -> float:
    return allreduce(world, [v], "max")[0]


def new_ep(world, rank):
    """(rank, size, nccl_id) for a new expert-parallel handle, or None."""
    if world == 1:
        return None
    import torch.distributed as dist
    from gallium_b200 import nccl_unique_id
    obj = [nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    return (rank, world, obj[0])


def gpu_uuid(local: int) -> str:
    import torch
    try:
        u = str(torch.cuda.get_device_properties(local).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        return vis.split(",")[local] if vis else str(local)


def cpu_cores(requested: int) -> int:
    if requested > 0:
        return requested
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


# ---------------------------------------------------------------------------
# the reference arm: the reference's grouped CPU forward on the host cores
# ---------------------------------------------------------------------------

def cpu_reference_steps(layer, x, cores, warmup, steps):
    """Mean seconds per whole-batch forward of oracle/cpu_reference.py, and
    the last forward's output (every row of the batch)."""
    from oracle.cpu_reference import CpuReference
    ref = CpuReference(layer, n_threads=cores)
    try:
        times = []
        for i in range(warmup + steps):
            t0 = time.perf_counter()
            y = ref.forward(x)
            if i >= warmup:
                times.append(time.perf_counter() - t0)
    finally:
        ref.close()
    return statistics.mean(times), y


def rows_parity(got, want):
    """Every row of a forward against the CPU forward's rows, on the bar."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    finite = bool(np.all(np.isfinite(got)))
    err = np.abs(got - want)
    max_abs = float(err.max()) if finite else float("inf")
    mean_rel = float(err.sum() / max(np.abs(want).sum(), 1e-30)) if finite else float("inf")
    return {"rows": int(got.shape[0]), "max_abs": max_abs, "mean_rel": mean_rel,
            "pass": bool(max_abs <= MAX_ABS and mean_rel <= MEAN_REL)}


def run_reference(args, world, rank):
    if rank != 0:
        return
    from gallium_b200 import synth
    model = Model(args.model, args.experts, args.skewed)
    layer = model.layer(args.seed)
    T = args.tokens
    x = synth.tokens(T, model.H, seed=args.seed)
    cores = cpu_cores(args.cpu_threads)
    sec, _ = cpu_reference_steps(layer, x, cores, args.warmup, args.steps)
    value = T / sec
    sample = (f"full batch every step: all {T} tokens routed and every active expert run "
              f"(grouped forward of gpt_oss_q.rs / lfm2moe_q.rs, OpenBLAS f32 GEMMs)")
    line = {
        "impl": "reference", "metric": model.metric, "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * sec, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{model.shape}, T={T} tokens",
                   "tokens": T, "experts": model.E, "skewed": args.skewed},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# the CUDA arm
# ---------------------------------------------------------------------------

def stage_profile(moe, xd, out, T, flush, reps=3):
    """Median per-stage ms over `reps` forwards (CUDA events inside the library)."""
    import torch
    moe.set_profiling(True)
    acc = {}
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(reps):
        flush()
        moe.forward_raw(xd.data_ptr(), T, out.data_ptr(), stream)
        for k, v in moe.stage_times().items():
            acc.setdefault(k, []).append(v)
    moe.set_profiling(False)
    return {k: statistics.median(v) for k, v in acc.items()}


def measured_traffic(model, T, stage, n_gpus):
    """DRAM bytes per launch of `stage`'s GEMM from the committed ncu capture
    (profiles/roofline_traffic.json), or None when none matches."""
    path = os.path.join(ROOT, "profiles", "roofline_traffic.json")
    try:
        with open(path) as f:
            entries = json.load(f)["entries"]
    except (OSError, ValueError, KeyError):
        return None
    for e in entries:
        if (e["tokens"] == T and e["experts"] == model.E and e["stage"] == stage
                and e.get("n_gpus", 1) == n_gpus and e.get("model", "gptoss") == model.name
                and e.get("skewed", False) == model.skewed):
            return e["dram_read_bytes"] + e["dram_write_bytes"]
    return None


def roofline_for(model, stage_ms, T, n_touched, peaks, n_gpus=1):
    """Roofline of the dominant expert kernel (gate_up or down, or both when
    one launch runs them: the library then records an empty down stage)."""
    H, I, k = model.H, model.I, model.k
    rows = T * k
    gu_w, dn_w = model.stage_weight_bytes()
    stage_bytes = {
        "gate_up": n_touched * gu_w + rows * H * 4 + rows * I * 4,  # weights + gathered x + h
        "down": n_touched * dn_w + rows * I * 4 + rows * H * 4,
    }
    stage_flops = {"gate_up": 2 * rows * 2 * I * H, "down": 2 * rows * H * I}
    if model.Is:  # the shared expert runs in the gate_up stage's window
        stage_bytes["gate_up"] += 3 * model.Is * H * 2 + T * (2 * H + model.Is) * 4
        stage_flops["gate_up"] += 2 * T * 3 * H * model.Is
    stage_ms = dict(stage_ms)
    if stage_ms.get("down", 0.0) < 0.005:  # two adjacent events: no kernel between them
        stage_ms["gate_up+down"] = stage_ms["gate_up"]
        stage_bytes["gate_up+down"] = stage_bytes["gate_up"] + stage_bytes["down"]
        stage_flops["gate_up+down"] = stage_flops["gate_up"] + stage_flops["down"]
        stage_ms["gate_up"] = stage_ms["down"] = 0.0
    dom = max(stage_ms.keys() & stage_bytes.keys(), key=lambda s: stage_ms[s])
    t = stage_ms[dom] / 1e3
    traffic = measured_traffic(model, T, dom, n_gpus)
    if T <= 64:
        ach = stage_bytes[dom] / t / 1e9
        return {"kernel": dom, "bound": "hbm", "achieved": ach, "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": ach / peaks["hbm_gbs"],
                "peak_source": peaks["source"], "algorithmic_bytes": stage_bytes[dom],
                "launch_ms": stage_ms[dom], "traffic": traffic}
    ach = stage_flops[dom] / t / 1e12
    return {"kernel": dom, "bound": "tensor", "achieved": ach, "peak": peaks["bf16_tflops"],
            "unit": "TFLOP/s", "frac": ach / peaks["bf16_tflops"],
            "peak_source": peaks["source"], "algorithmic_flops": stage_flops[dom],
            "launch_ms": stage_ms[dom], "traffic": traffic}


class Arm:
    """One loaded layer on this rank's GPU, with device buffers for the largest
    batch it is timed at."""

    def __init__(self, model, layer, local, rank, world, max_T, seed, expert_path="auto"):
        import torch
        from gallium_b200 import synth
        self.model, self.layer, self.rank, self.world = model, layer, rank, world
        self.moe = model.load(layer, local, max_T, new_ep(world, rank))
        self.moe.set_expert_path(expert_path)
        self.x = synth.tokens(max_T, model.H, seed=seed + 1000 * rank)
        self.xd = torch.from_numpy(self.x).cuda()
        self.out = torch.empty_like(self.xd)
        self.stream = torch.cuda.current_stream()

    def fwd(self, T):
        self.moe.forward_raw(self.xd.data_ptr(), T, self.out.data_ptr(), self.stream.cuda_stream)

    def timed(self, n, T, fwd, flush):
        """Sum of n CUDA-event step times (ms), L2 flushed before each step."""
        import torch
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(n)]
        for s, e in ev:
            flush()
            s.record(self.stream)
            fwd(T)
            e.record(self.stream)
        torch.cuda.synchronize()
        return sum(s.elapsed_time(e) for s, e in ev)

    def touched(self, T):
        """Experts this rank's GPU runs for a batch of T tokens per rank:
        routed by any rank's tokens, among its own."""
        c = self.moe.route(self.xd[:T])["counts"].cpu().numpy().astype(np.int64)
        if self.world > 1:
            c = np.array(allreduce(self.world, c.tolist(), "sum"), np.int64)
            E = self.model.E
            lo, hi = self.rank * E // self.world, (self.rank + 1) * E // self.world
            mine = np.zeros(E, np.int64)
            mine[lo:hi] = c[lo:hi]
            return int((mine > 0).sum()), c
        return int((c > 0).sum()), c

    def measure(self, T, steps, warmup, flush, peaks):
        """Device-resident throughput, stages and roofline at T tokens per GPU."""
        for _ in range(warmup):
            self.fwd(T)
        n_touched, _ = self.touched(T)
        barrier(self.world)
        ms = allmax(self.world, self.timed(steps, T, self.fwd, flush)) / steps
        st = stage_profile(self.moe, self.xd, self.out, T, flush)
        return {"tokens": T, "value": self.world * T / (ms / 1e3), "ms_per_step": ms,
                "stages_ms": st,
                "roofline": roofline_for(self.model, st, T, n_touched, peaks, self.world)}

    def parity(self, T, n_rows, threads):
        """This rank's forward of T tokens against the oracle; the worst
        figures over the ranks.  Every rank takes the same collective steps."""
        import torch
        self.fwd(T)  # every rank: the expert-parallel forward is collective
        torch.cuda.synchronize()
        got_all = self.out[:T].cpu().numpy()
        self.last_out = got_all
        self.moe.device_status(self.stream.cuda_stream)
        idx_gpu = self.moe.route(self.xd[:T])["idx"].cpu().numpy()
        x = self.x[:T]
        idx_or = self.model.route(self.layer, x)
        mism = int((idx_gpu != idx_or).any(axis=1).sum())
        _, counts = self.touched(T)
        busiest = int(np.argmax(counts))
        rng = np.random.default_rng(1234 + self.rank)
        busy_rows = np.nonzero((idx_or == busiest).any(axis=1))[0][: max(1, n_rows // 4)]
        rand_rows = rng.choice(T, size=min(T, n_rows), replace=False)
        rows = np.unique(np.concatenate([busy_rows, rand_rows]))[:n_rows]
        want, _, _ = self.model.oracle(self.layer).forward(x[rows], n_threads=threads)
        got = got_all[rows].astype(np.float64)
        finite = bool(np.all(np.isfinite(got)))
        err = np.abs(got - want)
        max_abs = float(err.max()) if finite else float("inf")
        mean_rel = float(err.sum() / max(np.abs(want).sum(), 1e-30)) if finite else float("inf")
        mx = allreduce(self.world, [max_abs, mean_rel], "max")
        sm = allreduce(self.world, [mism, len(rows), T], "sum")
        ok = sm[0] == 0 and mx[0] <= MAX_ABS and mx[1] <= MEAN_REL
        return {"rows": int(sm[1]), "tokens_routed": int(sm[2]), "idx_bit_exact": sm[0] == 0,
                "idx_mismatched_tokens": int(sm[0]), "max_abs": mx[0], "mean_rel": mx[1],
                "busiest_expert": busiest, "bar": {"max_abs": MAX_ABS, "mean_rel": MEAN_REL},
                "pass": bool(ok)}

    def close(self):
        self.moe.close()


def run_config(model, seed, local, rank, world, tokens, args, flush, peaks, threads):
    """Throughput, roofline and parity of one of the workload's other layers."""
    layer = model.layer(seed)
    arm = Arm(model, layer, local, rank, world, max(tokens), seed)
    try:
        out = []
        for T in tokens:
            m = arm.measure(T, args.steps, args.warmup, flush, peaks)
            if not args.no_parity:
                m["parity"] = arm.parity(T, min(T, 32), threads)
            out.append(m)
        return {"workload": f"{model.shape}, tokens per GPU as listed", "results": out}
    finally:
        arm.close()


DEC_PROMPT, DEC_CONTEXT = 128, 4096


def run_decode_config(args, local, peaks, threads):
    """The GPT-OSS-20B-shaped decode stack (24 layers, 64 query / 8 KV heads
    of 64, sliding window 128 on even layers, vocab 201088, bf16 attention
    and LM head, the 32-expert MXFP4 MoE block in every layer): for each
    batch, a prompt of DEC_PROMPT random ids per sequence, then --decode-steps
    greedy steps timed on the device (each step one replayed CUDA graph).
    The MoE share comes from one profiled eager step.  Parity: the logits
    of a 4-token prompt against the oracle of the whole stack."""
    import torch
    from gallium_b200 import GptOssQ, synth

    batches = [int(b) for b in args.decode_batches.split(",") if b.strip()]
    steps = args.decode_steps
    w = synth.gptoss_decoder(n_layers=24, seed=args.seed, share_experts=True)
    Bmax = max(batches)
    out = {"workload": ("gpt-oss-20b-shaped decode stack: 24 layers, H=2880, 64/8 heads of 64, "
                        "sliding window 128 on even layers, vocab 201088, bf16 attention and LM "
                        "head, 32-expert MXFP4 MoE (top-4) per layer; KV cache context "
                        f"{DEC_CONTEXT}; prompt {DEC_PROMPT} random ids, {steps} greedy "
                        "steps timed"),
           "weights": "random; every layer's experts drawn from one seed (own device copy each)",
           "results": []}
    m = GptOssQ.load(w, device=local, max_batch=Bmax, max_tokens=DEC_PROMPT,
                     max_seq_len=DEC_CONTEXT)
    try:
        stream = torch.cuda.current_stream()
        H, L, V = w.hidden, w.n_layers, w.vocab
        # bf16 q/k/v rows [(nh + 2 nkv) hd][H] and o rows [H][nh hd]
        attn_bytes = L * 2 * H * ((w.n_heads + 2 * w.n_kv_heads) * w.head_dim +
                                  w.n_heads * w.head_dim)
        expert_bytes = w.layers[0].moe.base.expert_bytes + w.layers[0].moe.base.expert_bias_bytes
        for B in batches:
            rng = np.random.default_rng(args.seed + B)
            prompt = torch.from_numpy(rng.integers(0, V, (B, DEC_PROMPT)).astype(np.int32)).cuda()

            def prefill():
                m.reset()
                m.forward(prompt, 0, check_status=False)
                return m.last_next.clone()

            first = prefill()
            m.generate(first, DEC_PROMPT, 4)          # captures the step graph for B
            first = prefill()
            torch.cuda.synchronize()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            toks = m.generate(first, DEC_PROMPT, steps, check_status=False)
            e.record(stream)
            torch.cuda.synchronize()
            ms = s.elapsed_time(e)
            m._lib.gb_decoder_device_status(m._h, stream.cuda_stream)
            ms_step = ms / steps
            # MoE share: one profiled eager step after the same prefill
            first = prefill()
            m.set_profiling(True)
            m.generate(first, DEC_PROMPT, 2, check_status=False)
            st = m.stage_times()
            m.set_profiling(False)
            total = sum(st.values())
            # bytes one step must read: attention and LM-head weights, the
            # experts the step touches (expected for uniform routing), the KV
            # cache at the mean context of the timed steps
            ctx = DEC_PROMPT + steps / 2
            kv = B * w.n_kv_heads * w.head_dim * 4 * 2 * (
                (L // 2) * ctx + (L - L // 2) * min(ctx, w.sliding_window))
            E, k = 32, 4
            touched = E * (1 - (1 - k / E) ** B)
            bytes_step = attn_bytes + V * H * 2 + L * touched * expert_bytes + kv
            achieved = bytes_step / (ms_step / 1e3) / 1e9
            peak = peaks["hbm_gbs"]
            out["results"].append({
                "batch": B, "value": B * steps / (ms / 1e3), "unit": "tokens/s",
                "ms_per_step": ms_step,
                "stage_ms_eager_step": st,
                "moe_share": st["moe"] / total if total > 0 else None,
                "roofline": {"kernel": "whole decode step", "bound": "hbm",
                             "achieved": achieved, "peak": peak, "unit": "GB/s",
                             "frac": achieved / peak, "peak_source": peaks["source"],
                             "algorithmic_bytes": int(bytes_step),
                             "experts_touched_per_layer": touched, "traffic": None},
                "tokens_sample": toks[:4, :min(B, 4)].cpu().numpy().tolist(),
            })
        if not args.no_parity:
            out["parity"] = decode_parity(w, m, threads)
    finally:
        m.close()
    return out


def decode_parity(w, m, threads):
    """Logits of a 4-token prompt (batch 1) against the oracle of the whole
    stack, and the greedy token."""
    import torch
    from oracle import decoder_oracle as dor

    toks = np.random.default_rng(77).integers(0, w.vocab, (1, 4)).astype(np.int32)
    m.reset()
    got = m.forward(torch.from_numpy(toks).cuda(), 0).cpu().numpy()
    orc = dor.OracleDecoder(w, max_seq_len=8)
    want = orc.forward(toks, 0)
    err = np.abs(got.astype(np.float64) - want)
    max_abs, mean_rel = float(err.max()), float(err.sum() / np.abs(want).sum())
    g, o = int(dor.greedy(got)[0]), int(dor.greedy(want)[0])
    gap = abs(float(want[0, g]) - float(want[0, o]))
    ok = max_abs <= MAX_ABS and mean_rel <= MEAN_REL and (g == o or gap < 5e-3)
    return {"prompt_tokens": 4, "max_abs": max_abs, "mean_rel": mean_rel,
            "greedy_equal": g == o, "bar": {"max_abs": MAX_ABS, "mean_rel": MEAN_REL},
            "pass": bool(ok)}


def run_ours(args, world, rank, local):
    import torch
    from gallium_b200._lib import check, load_library

    lib = load_library()
    peaks = load_peaks()
    cores = cpu_cores(args.cpu_threads)
    threads = max(1, cores // world)
    model = Model(args.model, args.experts, args.skewed)
    H = model.H
    T = args.tokens
    sweep = [int(s) for s in args.sweep.split(",") if s.strip()] if args.sweep else []
    layer = model.layer(args.seed)
    arm = Arm(model, layer, local, rank, world, max([T] + sweep), args.seed, args.expert_path)
    flush_buf = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device="cuda")

    def flush():
        flush_buf.zero_()

    for _ in range(args.warmup):
        arm.fwd(T)
    torch.cuda.synchronize()
    n_touched, _ = arm.touched(T)

    # ---- timed region: exactly K steps --------------------------------------
    clocks = ClockSampler(gpu_uuid(local))
    clocks.start()
    clocks.wait_first()
    launches0 = arm.moe.info()["kernel_launches"]
    barrier(world)
    torch.cuda.synchronize()
    total_ms = arm.timed(args.steps, T, arm.fwd, flush)
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop()
    launches = arm.moe.info()["kernel_launches"] - launches0
    total_ms = allmax(world, total_ms)
    ms_per_step = total_ms / args.steps
    value = world * T / (ms_per_step / 1e3)

    # ---- e2e through the public host-buffer entry point ----------------------
    xh = torch.from_numpy(arm.x[:T]).pin_memory()
    oh = torch.empty_like(xh).pin_memory()

    def fwd_host(Tn):
        check(lib.gb_moe_forward_host(arm.moe.handle, xh.data_ptr(), Tn, oh.data_ptr(),
                                      arm.stream.cuda_stream))

    fwd_host(T)
    barrier(world)
    e2e_ms = allmax(world, arm.timed(args.steps, T, fwd_host, flush)) / args.steps
    e2e = {"value": world * T / (e2e_ms / 1e3), "unit": "tokens/s",
           "h2d_bytes_per_step": T * H * 4, "d2h_bytes_per_step": T * H * 4,
           "ms_per_step": e2e_ms}

    # ---- roofline of the dominant kernel ------------------------------------
    stages = stage_profile(arm.moe, arm.xd, arm.out, T, flush)
    roof = roofline_for(model, stages, T, n_touched, peaks, world)

    # ---- other batch sizes of the workload -----------------------------------
    sweep_out = [arm.measure(Ts, args.steps, 2, flush, peaks) for Ts in sweep]

    # ---- parity against the oracle (every rank, outside the timed region) ----
    parity = None if args.no_parity else arm.parity(T, args.parity_rows, threads)
    got_rows = getattr(arm, "last_out", None)
    arm.close()

    # ---- the workload's other layers ----------------------------------------
    configs = {}
    want = set(args.configs.split(",")) if args.configs != "all" else None

    def on(name):
        return want is None or name in want

    if not args.no_configs and args.model == "gptoss":
        if world == 1:
            for name, sk in (("20b_balanced", False), ("20b_skewed", True)):
                if on(name):
                    configs[name] = run_config(Model("gptoss", 32, sk), args.seed, local, rank,
                                               world, [4096], args, flush, peaks, threads)
        if on("lfm2_q4k"):
            configs["lfm2_q4k"] = run_config(Model("lfm2", 32), args.seed, local, rank, world,
                                             [1, 16, 64, 2048], args, flush, peaks, threads)
        if on("moeffn_dense"):
            configs["moeffn_dense"] = run_config(Model("dense", 128), args.seed, local, rank,
                                                 world, [1, 64, 2048], args, flush, peaks,
                                                 threads)
        if world == 1 and on("gptoss20b_decode"):
            configs["gptoss20b_decode"] = run_decode_config(args, local, peaks, threads)

    # ---- CPU baseline (rank 0, one GPU only) ---------------------------------
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sec, y_cpu = cpu_reference_steps(layer, arm.x[:T], cores, 1, 2)
        cpu = {"value": T / sec, "unit": "tokens/s", "cores": cores, "kind": "port",
               "sample": (f"full batch: all {T} tokens routed and every active expert run "
                          f"(oracle/cpu_reference.py), mean of 2 forwards after 1 warm-up")}
        # the CPU forward's output covers the whole batch: check every row of
        # the GPU forward against it, beside the oracle's sampled rows
        if parity is not None and got_rows is not None:
            parity["every_row_vs_cpu_forward"] = rows_parity(got_rows, y_cpu)
            parity["pass"] = bool(parity["pass"] and parity["every_row_vs_cpu_forward"]["pass"])

    all_parity = ([parity] + [r.get("parity") for c in configs.values() for r in c["results"]] +
                  [c.get("parity") for c in configs.values()])
    ok = all(p is None or p["pass"] for p in all_parity)
    if rank == 0:
        line = {
            "metric": model.metric, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded weights and inputs of the workload's shapes)",
            "config": {"workload": f"{model.shape}, T={T} tokens per GPU",
                       "tokens_per_gpu": T, "experts": model.E, "skewed": args.skewed,
                       "parallelism": (f"ep{world} (expert parallel, {model.E // world} experts "
                                       f"per GPU, NCCL dispatch/combine)") if world > 1 else "single GPU",
                       "l2": "flushed (256 MiB write) before every timed step",
                       "experts_touched": n_touched},
            "e2e": e2e,
            "roofline": roof,
            "stages_ms": stages,
            "cpu_baseline": cpu,
            "clocks": clk,
            "gpu_launches": int(launches),
            "parity": parity,
            "sweep": sweep_out,
            "configs": configs,
        }
        print(json.dumps(line), flush=True)
    return ok


def main():
    args = parse_args()
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        world = int(os.environ.get("WORLD_SIZE", "1"))
        run_reference(args, world, rank)
        return
    world, rank, local = dist_setup(args)
    ok = True
    try:
        ok = run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    if not ok:
        print("parity check against the oracle failed", file=sys.stderr)
        sys.exit(3)


if __name__ == "__main__":
    main()
