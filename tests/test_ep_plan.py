"""Expert-parallel data movement, on CPU ranks (gloo, world sizes 2 and 4).

Each rank routes its own tokens, sends every routed row to the rank that owns
the expert, the owner groups what it received by local expert (expert
ascending, then source rank, then the source's order), runs the experts, and
returns each output row to the slot it came from; the source then combines in
rank order.  This is the plan rs-gallium_b200/csrc/ep.cu executes with NCCL.
Here the exchanges are gloo collectives and the experts are the oracle's, so
the result must equal the single-process oracle bit for bit.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from gallium_b200 import synth

E, H, I, K = 8, 64, 64, 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def ep_forward_emulated(om, layer, x, rank, world):
    """One rank's part of the expert-parallel forward, exchanges via gloo."""
    e_per = E // world
    rw = synth.bf16_bits_to_f32(layer.router_w)
    rb = synth.bf16_bits_to_f32(layer.router_b)
    idx, w = oracle.route_softmax_topk(oracle.router_logits(x, rw, rb), K)
    counts, offsets, perm, inv = oracle.permute(idx, E)
    send_x = x[perm // K]  # grouped (expert-ascending, hence destination-ordered) rows

    # 1. counts: everyone learns everyone's per-expert counts
    all_counts = [torch.zeros(E, dtype=torch.int32) for _ in range(world)]
    dist.all_gather(all_counts, torch.from_numpy(counts))
    all_counts = [c.numpy() for c in all_counts]
    # 2-3. rows: the range of each destination, gathered everywhere (small test)
    chunks = [None] * world
    dist.all_gather_object(chunks, [send_x[offsets[d * e_per]:offsets[(d + 1) * e_per]]
                                    for d in range(world)])
    recv = [chunks[s][rank] for s in range(world)]  # source-major, expert-ascending inside
    # 4. group received rows by local expert, then source
    out_recv = [np.zeros_like(r) for r in recv]
    for le in range(e_per):
        g = rank * e_per + le
        rows, where = [], []
        for s in range(world):
            c = all_counts[s]
            start = sum(c[rank * e_per:g])  # rows of earlier local experts from source s
            n = c[g]
            rows.append(recv[s][start:start + n])
            where += [(s, start + i) for i in range(n)]
        grouped = np.concatenate(rows) if rows else np.zeros((0, H), np.float32)
        if grouped.shape[0]:
            # 5. experts; outputs go back to their received slots
            y = om.expert_ffn(g, grouped)
            for (s, j), yy in zip(where, y):
                out_recv[s][j] = yy
    # 6. return rows to their sources
    back = [None] * world
    dist.all_gather_object(back, out_recv)
    y_back = np.concatenate([back[d][rank] for d in range(world)])  # this rank's grouped order
    # 7. combine in rank order (gpt_oss.rs:223)
    out = np.zeros_like(x)
    for t in range(x.shape[0]):
        acc = np.zeros(H, np.float32)
        for r in range(K):
            acc = acc + (y_back[inv[t * K + r]] * w[t, r]).astype(np.float32)
        out[t] = acc
    return out


def _worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        layer = synth.gptoss_layer(n_experts=E, hidden=H, inter=I, top_k=K, seed=3)
        om = oracle.OracleMoe(layer)
        x = synth.tokens(7 + 3 * rank, H, seed=40 + rank)  # ragged: ranks hold different T
        got = ep_forward_emulated(om, layer, x, rank, world)
        want, _, _ = om.forward(x)
        results[rank] = bool(np.array_equal(got, want))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_expert_parallel_plan_reproduces_one_device_bit_for_bit(world):
    with mp.get_context("spawn").Manager() as mgr:
        results = mgr.dict()
        mp.spawn(_worker, args=(world, _free_port(), results), nprocs=world, join=True)
        assert dict(results) == {r: True for r in range(world)}
