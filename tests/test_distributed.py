"""World-size-2 gloo tests of the multi-GPU host logic on CPU: sample sharding,
the variable-length latent gather, and a rank that dies mid-run being seen by
the survivor as a collective error within the process-group timeout."""
import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup(rank, world, port):
    sys.path.insert(0, str(ROOT))
    from __graft_entry__ import load_package
    load_package()
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from vdit import distributed as vd
    return vd


def _gather_worker(rank, world, port, q):
    vd = _setup(rank, world, port)
    r, w, _ = vd.init_from_env("gloo", timeout_s=30)
    mine = vd.shard_samples(5, r, w)
    lat = [torch.full((10 + 7 * i, 16), float(i)) for i in mine]
    while len(lat) < 3:                          # uneven shards are padded with empty tensors
        lat.append(torch.zeros(0, 16))
    got = vd.gather_latents(lat, r, w)
    if r == 0:
        q.put([(t.shape[0], float(t.mean()) if t.numel() else None) for t in got])
    import torch.distributed as dist
    dist.destroy_process_group()


def test_gather_latents_variable_sizes():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_gather_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = q.get(timeout=120)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    # rank 0 owns samples 0,2,4; rank 1 owns 1,3 (+ one empty pad)
    assert res == [(10, 0.0), (24, 2.0), (38, 4.0), (17, 1.0), (31, 3.0), (0, None)]


def _dying_worker(rank, world, port, q):
    vd = _setup(rank, world, port)
    r, w, _ = vd.init_from_env("gloo", timeout_s=5)
    import torch.distributed as dist
    if r == 1:
        os._exit(3)                              # a rank that leaves between steps
    try:
        vd.gather_latents([torch.zeros(4, 16)], r, w)
        q.put("no error")
    except Exception as exc:                     # the survivor sees an error, not a hang
        q.put(type(exc).__name__)


def test_dead_rank_surfaces_as_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    msg = q.get(timeout=120)
    for p in ps:
        p.join(timeout=60)
    assert msg != "no error"


def test_shard_samples_cover_all():
    sys.path.insert(0, str(ROOT))
    from vdit import distributed as vd
    for world in (1, 2, 4, 8):
        owned = sorted(i for r in range(world) for i in vd.shard_samples(16, r, world))
        assert owned == list(range(16))


def _fake_nfe(calls):
    def nfe(x, t, uncond):
        calls.append((t, uncond))
        return torch.sin(x * (1.0 + t)) + (0.25 * x if uncond else 0.0)
    return nfe


def _fake_cfg(x, v, vn, g, dt):
    vv = v if vn is None else v + g * (v - vn)
    x.sub_(dt * vv)


TL, GUIDED, G = [1.0, 0.9, 0.75, 0.5, 0.0], [True, True, True, False], 3.0


def _branch_worker(rank, world, port, q):
    vd = _setup(rank, world, port)
    r, w, _ = vd.init_from_env("gloo", timeout_s=30)
    calls = []
    x = torch.linspace(-1, 1, 64).view(4, 16).clone()
    vd.branch_split_steps(x, TL, GUIDED, G, _fake_nfe(calls), _fake_cfg)
    q.put((r, x.tolist(), calls))
    import torch.distributed as dist
    dist.destroy_process_group()


def test_branch_split_matches_one_process():
    """Two gloo ranks run the split loop with a stand-in NFE: rank 0 only the conditional
    branch, rank 1 only the unconditional one (guided steps), and both end with the x of
    the one-process loop, bit for bit."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_branch_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict((r, (x, calls)) for r, x, calls in (q.get(timeout=120), q.get(timeout=120)))
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    x = torch.linspace(-1, 1, 64).view(4, 16).clone()
    nfe = _fake_nfe([])
    for i, gd in enumerate(GUIDED):
        v = nfe(x, TL[i], False)
        _fake_cfg(x, v, nfe(x, TL[i], True) if gd else None, G, TL[i] - TL[i + 1])
    assert torch.equal(torch.tensor(res[0][0]), x) and torch.equal(torch.tensor(res[1][0]), x)
    assert res[0][1] == [(1.0, False), (0.9, False), (0.75, False), (0.5, False)]
    assert res[1][1] == [(1.0, True), (0.9, True), (0.75, True)]
