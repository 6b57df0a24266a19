"""Two GPUs, one sample: the branch split (conditional NFE on rank 0, exact 1-token NFE
on rank 1, velocities exchanged over NCCL) against the one-GPU sampler on the same
noise.  Runs as two spawned processes, one per GPU, with NVLS off; skipped on a box
with fewer than two GPUs."""
import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, q):
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2",
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    from __graft_entry__ import load_package
    load_package()
    import torch.distributed as dist
    from vdit import distributed as vd
    from tests.test_gpu_forward import build
    try:
        vd.init_from_env("nccl", timeout_s=60)
        _, _, runner, vox, ctx, xt = build(256, 128, 3, 1, 2000, 8, 1024, 61)
        dev = torch.device("cuda", rank)
        vox_d, ctx_d = torch.from_numpy(vox).to(dev), ctx.to(dev, torch.bfloat16)
        out = runner.sample_branch_split(vox_d, ctx_d, noise=xt.to(dev))
        torch.cuda.synchronize(dev)
        if rank == 0:
            ref = runner.sample_with_context(vox_d, ctx_d, noise=xt.to(dev), cuda_graph=False)
            d = (out - ref).float()
            q.put(("ok", float(d.norm() / ref.float().norm()), bool(torch.equal(out, ref))))
        else:
            q.put(("rank1", float(out.float().norm()), False))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:                     # reported to the test, never a hang
        q.put(("error", repr(exc), False))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_branch_split_two_gpus_matches_one_gpu():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=600) for _ in range(2)]
    for p in ps:
        p.join(timeout=120)
    tags = {r[0]: r for r in res}
    assert "error" not in tags, tags.get("error")
    _, rel, same = tags["ok"]
    assert rel < 1e-5, rel                       # the same kernels on the same inputs
