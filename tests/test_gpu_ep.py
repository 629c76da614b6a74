"""Expert parallelism on real GPUs (needs at least 2; the 4-rank cases need 4):
every rank routes its own tokens, experts are sharded E/N per GPU, rows move
by NCCL.  Each rank's output is checked against the single-process oracle on
the same tokens, and the ranks hold different token counts, so some run the
decode-sized kernels and others the tensor-core path, and one rank may send
rows it receives none back for.  Cases: the 20B-shaped block (32 experts), a
128-expert layer (the 120B layer's routing and exchange shape at a smaller
hidden size, so the oracle stays fast), the LFM2.5 Q4_K block, and a generic
MoEFFN layer with dense experts and a shared expert (one rank with no tokens
at all in the 4-rank case)."""
import os
import socket

import numpy as np
import pytest
import torch

import oracle
from gallium_b200 import Lfm2QMoEFFN, MoEFFN, OssMoEFFN, nccl_unique_id, synth

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs"),
]

MAX_ABS, MEAN_REL = 2e-2, 1e-3

# name -> (layer factory, block class, oracle class, experts, hidden,
#          tokens per rank with 2 / 4 ranks)
CASES = {
    "gptoss-e32": (lambda: synth.gptoss_layer(n_experts=32, seed=0), OssMoEFFN,
                   oracle.OracleMoe, 32, 2880, ([37, 96], [37, 96, 5, 130])),
    "gptoss-e128": (lambda: synth.gptoss_layer(n_experts=128, hidden=512, inter=512, seed=4),
                    OssMoEFFN, oracle.OracleMoe, 128, 512, ([300, 64], [100, 37, 256, 3])),
    "lfm2-q4k": (lambda: synth.lfm2_layer(n_experts=32, seed=5), Lfm2QMoEFFN,
                 oracle.OracleLfm2, 32, 2048, ([5, 200], [64, 1, 300, 17])),
    "dense-shared": (lambda: synth.dense_layer(n_experts=32, hidden=512, inter=256, top_k=4,
                                               shared_inter=128, seed=6),
                     MoEFFN, oracle.OracleDense, 32, 512, ([9, 150], [150, 9, 0, 33])),
}


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, case, results):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        torch.cuda.set_device(rank)
        make, cls, orc, _, H, tokens = CASES[case]
        tokens = tokens[0] if world == 2 else tokens[1]
        obj = [nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        layer = make()
        T = tokens[rank]
        x = synth.tokens(T, H, seed=700 + rank)
        with cls.load(layer, device=rank, max_tokens=max(tokens), ep=(rank, world, obj[0])) as moe:
            out = []
            for _ in range(2):  # twice: buffers reused, results identical
                out.append(moe.forward(torch.from_numpy(x).cuda()).cpu().numpy())
            idx_gpu = moe.route(torch.from_numpy(x).cuda())["idx"].cpu().numpy()
            info = moe.info()
        want, idx, _ = orc(layer).forward(x, n_threads=2)
        err = np.abs(out[0].astype(np.float64) - want)
        results[rank] = {
            "max_abs": float(err.max()) if err.size else 0.0,
            "mean_rel": float(err.sum() / max(np.abs(want).sum(), 1e-30)),
            "repeat_equal": bool(np.array_equal(out[0], out[1])),
            "idx_equal": bool(np.array_equal(idx_gpu, idx)),
            "experts": (info["local_expert_begin"], info["local_expert_end"]),
        }
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("case", list(CASES))
def test_expert_parallel_forward_matches_oracle(case, world):
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    E = CASES[case][3]
    with mp.get_context("spawn").Manager() as mgr:
        results = mgr.dict()
        mp.spawn(_worker, args=(world, _free_port(), case, results), nprocs=world, join=True)
        res = dict(results)
    assert set(res) == set(range(world))
    per = E // world
    for r, v in res.items():
        assert v["experts"] == (r * per, (r + 1) * per), (r, v)
        assert v["idx_equal"], r
        assert v["repeat_equal"], r
        assert v["max_abs"] <= MAX_ABS and v["mean_rel"] <= MEAN_REL, (r, v)
