#!/usr/bin/env python
"""MoE-layer tokens/s on B200: GPT-OSS-120B-shaped MXFP4 MoE layer.

Workload (one step = one forward of the layer over one batch):
  hidden 2880, intermediate 2880, 128 experts, top-4, MXFP4 experts (E2M1
  codes uniform, E8M0 exponents uniform in [-8, -2]), bf16 router ~ N(0, 0.02)
  with zero bias, bf16 biases ~ N(0, 0.01), clamped SwiGLU (limit 7),
  x ~ N(0, 1) f32, seed 0 -- synthetic weights and inputs (no checkpoint).
  Headline batch: --tokens (default 8192) tokens per GPU; --sweep adds the
  other batch sizes of the workload (1, 32, 1024) as extra measurements.

Arms:
  default            the CUDA path through the C ABI (gb_moe_forward on
                     device-resident inputs -> "value"; gb_moe_forward_host
                     with pinned host buffers, copies included -> "e2e").
  --impl reference   the reference's CPU algorithm (the oracle restatement in
                     oracle/, built from the reference's Rust sources' logic)
                     on the host cores, one bounded sample per step.

--model lfm2 measures the LFM2.5-shaped layer instead (hidden 2048,
intermediate 1792, 32 experts, top-4, Q4_K experts, sigmoid router with a
selection bias, SiLU; d = 2^-11, dmin = 7.5 d).  The default is GPT-OSS.

Multi-GPU (python -m torch.distributed.run ... bench.py --gpus N): one process
per GPU, expert parallel: rank r holds experts [r*E/N, (r+1)*E/N) and its own
batch of --tokens tokens; routed rows go to the owning rank and back by NCCL
inside the library.  Timing = max over ranks, value = all ranks' tokens / that
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


class Model:
    """Shapes, loader and byte counts of one measured MoE layer."""

    def __init__(self, name, experts):
        self.name = name
        if name == "gptoss":
            self.H, self.I, self.E = 2880, 2880, experts or 128
            self.metric = "MoE-layer tokens/s (GPT-OSS-120B shape, MXFP4)"
            self.shape = f"gpt-oss-120b-shaped MoE layer, E={self.E}, H=I=2880, top-{TOPK}, MXFP4"
        else:
            self.H, self.I, self.E = 2048, 1792, experts or 32
            self.metric = "MoE-layer tokens/s (LFM2.5 shape, Q4_K)"
            self.shape = (f"lfm2.5-shaped MoE layer, E={self.E}, H=2048, I=1792, top-{TOPK}, "
                          f"Q4_K, sigmoid router")

    def layer(self, args):
        from gallium_b200 import synth
        if self.name == "gptoss":
            return synth.gptoss_layer(n_experts=self.E, seed=args.seed, skewed=args.skewed)
        return synth.lfm2_layer(n_experts=self.E, seed=args.seed)

    def load(self, layer, device, max_tokens, ep):
        from gallium_b200 import Lfm2QMoEFFN, OssMoEFFN
        cls = OssMoEFFN if self.name == "gptoss" else Lfm2QMoEFFN
        return cls.load(layer, device=device, max_tokens=max_tokens, ep=ep)

    def stage_weight_bytes(self):
        """(gate_up, down) bytes of one expert: codes + scales (+ bf16 biases)."""
        H, I = self.H, self.I
        if self.name == "gptoss":
            return (2 * I * H // 2 + 2 * I * H // 32 + 2 * I * 2, H * I // 2 + H * I // 32 + H * 2)
        return (2 * I * H // 256 * 144, H * I // 256 * 144)

    def route(self, layer, x):
        """Oracle routing of x: (idx [T, k], oracle object for the experts)."""
        import oracle
        if self.name == "gptoss":
            rw = (layer.router_w.astype(np.uint32) << 16).view(np.float32)
            rb = (layer.router_b.astype(np.uint32) << 16).view(np.float32)
            idx, _ = oracle.route_softmax_topk(oracle.router_logits(x, rw, rb), TOPK)
            return idx, oracle.OracleMoe(layer)
        lg = oracle.router_logits(x, layer.router_w, None)
        idx, _ = oracle.route_sigmoid_topk(lg, layer.sel_bias, TOPK)
        return idx, oracle.OracleLfm2(layer)


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--model", choices=["gptoss", "lfm2"], default="gptoss")
    ap.add_argument("--experts", type=int, default=0, help="default 128 (gptoss) / 32 (lfm2)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--skewed", action="store_true", help="Zipf(1.2) router bias")
    ap.add_argument("--sweep", default="1,32,1024",
                    help="extra per-GPU batch sizes to measure ('' = none)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--expert-path", default="auto",
                    choices=["auto", "cuda_cores", "tensor_cores", "tensor_cores_f16"],
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


def allmax(world, v: float) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gpu_uuid(local: int) -> str:
    import torch
    try:
        u = str(torch.cuda.get_device_properties(local).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        return vis.split(",")[local] if vis else str(local)


# ---------------------------------------------------------------------------
# CPU baseline (the oracle restatement of the reference's CPU path)
# ---------------------------------------------------------------------------

def cpu_cores(requested: int) -> int:
    if requested > 0:
        return requested
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_sample(model, layer, x, counts, cores):
    """Time the reference's per-expert work (dequantise once, f32 GEMMs, the
    activation; gpt_oss_q.rs:194-246, lfm2moe_q.rs:279-296) for a bounded set
    of experts with their real token counts, plus the routing of a bounded
    token sample, and scale both to the whole batch.  Returns (tokens/s,
    description)."""
    T = x.shape[0]
    tr = min(T, 256)
    t0 = time.perf_counter()
    _, om = model.route(layer, x[:tr])
    t_route = time.perf_counter() - t0
    active = [e for e in range(len(counts)) if counts[e] > 0]
    m = min(len(active), max(1, cores))
    sample = np.array(active[:m], np.int32)
    ntok = np.array([counts[e] for e in sample], np.int32)
    t0 = time.perf_counter()
    om.expert_sample(x[: int(ntok.max())], sample, ntok, n_threads=cores)
    t_exp = time.perf_counter() - t0
    est = t_exp * len(active) / m + t_route * T / tr
    desc = (f"{m} of {len(active)} active experts with their routed token counts "
            f"({int(ntok.sum())} token-expert rows) + routing of {tr} of {T} tokens, "
            f"scaled to the batch; {t_exp + t_route:.1f} s of CPU work")
    return T / est, desc


# ---------------------------------------------------------------------------
# arms
# ---------------------------------------------------------------------------

def run_reference(args, world, rank):
    if rank != 0:
        return
    from gallium_b200 import synth
    model = Model(args.model, args.experts)
    layer = model.layer(args)
    T = args.tokens
    x = synth.tokens(T, model.H, seed=args.seed)
    cores = cpu_cores(args.cpu_threads)
    idx, _ = model.route(layer, x)
    counts = np.bincount(idx.ravel(), minlength=model.E)
    vals, desc = [], ""
    for i in range(args.warmup + args.steps):
        v, desc = cpu_sample(model, layer, x, counts, cores)
        if i >= args.warmup:
            vals.append(v)
    value = statistics.mean(vals)
    line = {
        "impl": "reference", "metric": model.metric, "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * T / value, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{model.shape}, T={T} tokens",
                   "tokens": T, "experts": model.E, "skewed": args.skewed},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": desc},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


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


def measured_traffic(T, E, stage, n_gpus):
    """DRAM bytes per launch of `stage`'s GEMM from the committed ncu capture
    (profiles/roofline_traffic.json), or None when none matches."""
    path = os.path.join(ROOT, "profiles", "roofline_traffic.json")
    try:
        with open(path) as f:
            entries = json.load(f)["entries"]
    except (OSError, ValueError, KeyError):
        return None
    for e in entries:
        if (e["tokens"] == T and e["experts"] == E and e["stage"] == stage
                and e.get("n_gpus", 1) == n_gpus):
            return e["dram_read_bytes"] + e["dram_write_bytes"]
    return None


def roofline_for(model, stage_ms, T, n_touched, peaks, n_gpus=1):
    """Roofline of the dominant expert kernel (gate_up or down, or both when
    one launch runs them: the library then records an empty down stage)."""
    H, I, E, k = model.H, model.I, model.E, TOPK
    rows = T * k
    gu_w, dn_w = model.stage_weight_bytes()
    stage_bytes = {
        "gate_up": n_touched * gu_w + rows * H * 4 + rows * I * 4,  # weights + gathered x + h
        "down": n_touched * dn_w + rows * I * 4 + rows * H * 4,
    }
    stage_flops = {"gate_up": 2 * rows * 2 * I * H, "down": 2 * rows * H * I}
    stage_ms = dict(stage_ms)
    if stage_ms.get("down", 0.0) < 0.005:  # two adjacent events: no kernel between them
        stage_ms["gate_up+down"] = stage_ms["gate_up"]
        stage_bytes["gate_up+down"] = stage_bytes["gate_up"] + stage_bytes["down"]
        stage_flops["gate_up+down"] = stage_flops["gate_up"] + stage_flops["down"]
        stage_ms["gate_up"] = stage_ms["down"] = 0.0
    dom = max(stage_ms.keys() & stage_bytes.keys(), key=lambda s: stage_ms[s])
    t = stage_ms[dom] / 1e3
    traffic = measured_traffic(T, E, dom, n_gpus) if model.name == "gptoss" else None
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


def run_ours(args, world, rank, local):
    import torch
    from gallium_b200 import nccl_unique_id, synth
    from gallium_b200._lib import check, load_library

    lib = load_library()
    peaks = load_peaks()
    model = Model(args.model, args.experts)
    H = model.H
    T = args.tokens
    sweep = [int(s) for s in args.sweep.split(",") if s.strip()] if args.sweep else []
    layer = model.layer(args)
    ep = None
    if world > 1:
        import torch.distributed as dist
        obj = [nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        ep = (rank, world, obj[0])
    moe = model.load(layer, local, max([T] + sweep), ep)
    moe.set_expert_path(args.expert_path)
    # buffers hold the largest batch of the run (T and every sweep size)
    x = synth.tokens(max([T] + sweep), H, seed=args.seed + 1000 * rank)
    xd = torch.from_numpy(x).cuda()
    out = torch.empty_like(xd)
    x = x[:T]
    flush_buf = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device="cuda")

    def flush():
        flush_buf.zero_()

    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream

    def timed(n, Tn, fwd):
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(n)]
        for s, e in ev:
            flush()
            s.record(stream)
            fwd(Tn)
            e.record(stream)
        torch.cuda.synchronize()
        return sum(s.elapsed_time(e) for s, e in ev)

    fwd_dev = lambda Tn: moe.forward_raw(xd.data_ptr(), Tn, out.data_ptr(), sp)
    for _ in range(args.warmup):
        fwd_dev(T)
    torch.cuda.synchronize()
    counts = moe.route(xd[:T])["counts"].cpu().numpy()
    n_touched = int((counts > 0).sum())
    if world > 1:
        # experts this rank's GPU runs: touched by any rank's tokens, among its own
        import torch.distributed as dist
        ct = torch.from_numpy(counts.astype(np.int64)).cuda()
        dist.all_reduce(ct)
        lo, hi = rank * model.E // world, (rank + 1) * model.E // world
        n_touched = int((ct[lo:hi] > 0).sum())

    # ---- timed region: exactly K steps --------------------------------------
    clocks = ClockSampler(gpu_uuid(local))
    clocks.start()
    clocks.wait_first()
    launches0 = moe.info()["kernel_launches"]
    barrier(world)
    torch.cuda.synchronize()
    total_ms = timed(args.steps, T, fwd_dev)
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop()
    launches = moe.info()["kernel_launches"] - launches0
    total_ms = allmax(world, total_ms)
    ms_per_step = total_ms / args.steps
    value = world * T / (ms_per_step / 1e3)

    # ---- e2e through the public host-buffer entry point ----------------------
    xh = torch.from_numpy(x).pin_memory()
    oh = torch.empty_like(xh).pin_memory()

    def fwd_host(Tn):
        check(lib.gb_moe_forward_host(moe.handle, xh.data_ptr(), Tn, oh.data_ptr(), sp))

    fwd_host(T)
    barrier(world)
    e2e_ms = allmax(world, timed(args.steps, T, fwd_host)) / args.steps
    e2e = {"value": world * T / (e2e_ms / 1e3), "unit": "tokens/s",
           "h2d_bytes_per_step": T * H * 4, "d2h_bytes_per_step": T * H * 4,
           "ms_per_step": e2e_ms}

    # ---- roofline of the dominant kernel ------------------------------------
    stages = stage_profile(moe, xd, out, T, flush)
    roof = roofline_for(model, stages, T, n_touched, peaks, world)

    # ---- other batch sizes of the workload -----------------------------------
    sweep_out = []
    for Ts in sweep:
        for _ in range(2):
            fwd_dev(Ts)
        c = moe.route(xd[:Ts])["counts"].cpu().numpy()
        if world > 1:
            import torch.distributed as dist
            ct = torch.from_numpy(c.astype(np.int64)).cuda()
            dist.all_reduce(ct)
            lo, hi = rank * model.E // world, (rank + 1) * model.E // world
            c = np.zeros(model.E, np.int64)
            c[lo:hi] = ct[lo:hi].cpu().numpy()
        barrier(world)
        ms = allmax(world, timed(args.steps, Ts, fwd_dev)) / args.steps
        st = stage_profile(moe, xd, out, Ts, flush)
        sweep_out.append({"tokens": Ts, "value": world * Ts / (ms / 1e3), "ms_per_step": ms,
                          "stages_ms": st,
                          "roofline": roofline_for(model, st, Ts, int((c > 0).sum()), peaks,
                                                   world)})

    # ---- CPU baseline (rank 0, one GPU only) ---------------------------------
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cores = cpu_cores(args.cpu_threads)
        v, desc = cpu_sample(model, layer, x, counts, cores)
        cpu = {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": desc}

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
            "sweep": sweep_out,
        }
        print(json.dumps(line), flush=True)
    moe.close()


def main():
    args = parse_args()
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        world = int(os.environ.get("WORLD_SIZE", "1"))
        run_reference(args, world, rank)
        return
    world, rank, local = dist_setup(args)
    try:
        run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
