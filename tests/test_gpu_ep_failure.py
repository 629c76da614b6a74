"""A rank that leaves between forwards: the survivor gets an error, not a hang.

Two ranks on two GPUs run one expert-parallel forward together; then rank 1
leaves (its process exits, with nothing of its own in flight).  Rank 0's next
forward must end within the handle's short wait limit with GB_ERR_TIMEOUT or
GB_ERR_NCCL (its count exchange finds no peer, and the communicator is
aborted), and every forward after that must be refused with GB_ERR_NCCL
instead of touching the departed rank's memory.  This mirrors the reference's
failure contract: an error is returned rather than a silent fallback or a
hang (crates/gallium-core/src/device.rs:22-41).

The ranks run with NVLS off (no multicast objects) and NCCL's GPU peer-memory
transport off (NCCL moves the count exchange through host shared memory), so
nothing is written into the departed process's GPU memory; the library's own
peer stores happen only after a count exchange has succeeded.
"""
import os
import socket
import time

import numpy as np
import pytest
import torch

from gallium_b200 import GalliumError, OssMoEFFN, _lib, nccl_unique_id, synth

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs"),
]

TIMEOUT_MS = 2000


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    import datetime

    import torch.distributed as dist

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["NCCL_P2P_DISABLE"] = "1"
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    torch.cuda.set_device(rank)
    obj = [nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    layer = synth.gptoss_layer(n_experts=8, hidden=256, inter=256, seed=9)
    x = torch.from_numpy(synth.tokens(16, 256, seed=rank)).cuda()
    moe = OssMoEFFN.load(layer, device=rank, max_tokens=16, ep=(rank, world, obj[0], TIMEOUT_MS))
    first = moe.forward(x).cpu().numpy()
    torch.cuda.synchronize()
    dist.barrier()  # both forwards are complete: nothing of either rank in flight
    if rank == 1:
        results[1] = {"first_finite": bool(np.isfinite(first).all())}
        os._exit(0)  # leaves without a goodbye
    time.sleep(1.0)
    t0 = time.time()
    try:
        moe.forward(x)
        second = ("ok", None)
    except GalliumError as e:
        second = ("error", e.status)
    elapsed = time.time() - t0
    try:
        moe.forward(x)
        third = ("ok", None)
    except GalliumError as e:
        third = ("error", e.status)
    moe.close()
    results[0] = {"first_finite": bool(np.isfinite(first).all()), "second": second,
                  "elapsed": elapsed, "third": third}


def test_survivor_gets_an_error_when_a_rank_leaves():
    import torch.multiprocessing as mp

    with mp.get_context("spawn").Manager() as mgr:
        results = mgr.dict()
        ctx = mp.spawn(_worker, args=(2, _free_port(), results), nprocs=2, join=False)
        deadline = time.time() + 180
        while not ctx.join(timeout=5):
            if time.time() > deadline:
                for p in ctx.processes:
                    p.kill()
                pytest.fail("the surviving rank did not return within 180 s")
        res = dict(results)
    assert res[1]["first_finite"] and res[0]["first_finite"]
    kind, status = res[0]["second"]
    assert kind == "error" and status in (_lib.GB_ERR_TIMEOUT, _lib.GB_ERR_NCCL), res[0]
    # within the wait limit plus the communicator's abort and the stream drain
    assert res[0]["elapsed"] < TIMEOUT_MS / 1000 * 3 + 10, res[0]
    assert res[0]["third"] == ("error", _lib.GB_ERR_NCCL), res[0]
