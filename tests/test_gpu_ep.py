"""Expert parallelism on real GPUs (needs at least 2): every rank routes its
own tokens, experts are sharded E/N per GPU, rows move by NCCL.  Each rank's
output is checked against the single-process oracle on the same tokens, and
the ranks hold different token counts so one runs the decode kernels and the
other the tensor-core path."""
import os
import socket

import numpy as np
import pytest
import torch

import oracle
from gallium_b200 import OssMoEFFN, nccl_unique_id, synth

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs"),
]

MAX_ABS, MEAN_REL = 2e-2, 1e-3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, tokens, results):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        torch.cuda.set_device(rank)
        obj = [nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        layer = synth.gptoss_layer(n_experts=32, seed=0)
        T = tokens[rank]
        x = synth.tokens(T, 2880, seed=700 + rank)
        with OssMoEFFN.load(layer, device=rank, max_tokens=max(tokens),
                            ep=(rank, world, obj[0])) as moe:
            out = []
            for _ in range(2):  # twice: buffers reused, results identical
                out.append(moe.forward(torch.from_numpy(x).cuda()).cpu().numpy())
            info = moe.info()
        want, _, _ = oracle.OracleMoe(layer).forward(x)
        err = np.abs(out[0].astype(np.float64) - want)
        results[rank] = {
            "max_abs": float(err.max()),
            "mean_rel": float(err.sum() / np.abs(want).sum()),
            "repeat_equal": bool(np.array_equal(out[0], out[1])),
            "experts": (info["local_expert_begin"], info["local_expert_end"]),
        }
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_expert_parallel_forward_matches_oracle():
    import torch.multiprocessing as mp

    world = 2
    tokens = [37, 96]
    with mp.get_context("spawn").Manager() as mgr:
        results = mgr.dict()
        mp.spawn(_worker, args=(world, _free_port(), tokens, results), nprocs=world, join=True)
        res = dict(results)
    assert set(res) == {0, 1}
    assert res[0]["experts"] == (0, 16) and res[1]["experts"] == (16, 32)
    for r, v in res.items():
        assert v["repeat_equal"], r
        assert v["max_abs"] <= MAX_ABS and v["mean_rel"] <= MEAN_REL, (r, v)
