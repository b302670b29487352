"""Head-sharded RCSA over NCCL on two B200s: the gathered output of
``HeadShardedRCSA`` (each rank its half of the heads, then the all-gather)
against the single-GPU ``RCSAPlan`` on the same inputs.  Selection and
codes are per (batch, head), so each rank's selection equals its slice of
the single-GPU one exactly; the attention may be planned into other work
splits at fewer heads per launch (fp32 partial merges in another order), so
the outputs agree within the attention bar.  Skips with fewer than two GPUs."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(heads=4, nq=2, nh=6, block=880, seed=5):
    g = torch.Generator().manual_seed(seed)
    scale = 0.5 + 1.5 * torch.rand(1, heads, 1, 1, generator=g)
    q = (torch.randn(1, heads, nq * block, 128, generator=g) * scale).bfloat16()
    k = (torch.randn(1, heads, (nq + nh) * block, 128, generator=g) * scale).bfloat16()
    v = (torch.randn(1, heads, (nq + nh) * block, 128, generator=g) * scale).bfloat16()
    return q, k, v


def _worker(rank, world, port, out_dir):
    from datetime import timedelta

    from cast_b200 import distributed as cd

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    try:
        q, k, v = _inputs()
        layer = cd.HeadShardedRCSA(1, q.shape[1], q.shape[2], k.shape[2], 128, block_size=880, budget=3,
                                   policy="auto", device=dev, gather="nccl")
        out = layer(*(layer.local_heads(t).to(dev) for t in (q, k, v)))
        torch.cuda.synchronize()
        torch.save(layer.plan.indices.cpu(), os.path.join(out_dir, f"sel{rank}.pt"))
        if rank == 0:
            torch.save(out.cpu(), os.path.join(out_dir, "gathered.pt"))
    finally:
        dist.destroy_process_group()


def test_head_sharded_equals_single_gpu(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from cast_b200 import rcsa

    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    q, k, v = _inputs()
    plan = rcsa.RCSAPlan(1, q.shape[1], q.shape[2], k.shape[2], 128, block_size=880, budget=3,
                         policy="auto", device=torch.device("cuda", 0))
    single = plan(q.cuda(), k.cuda(), v.cuda()).cpu()
    gathered = torch.load(os.path.join(tmp_path, "gathered.pt"))
    assert gathered.shape == single.shape
    half = q.shape[1] // world
    for r in range(world):
        sel = torch.load(os.path.join(tmp_path, f"sel{r}.pt"))
        assert torch.equal(sel, plan.indices.cpu()[:, r * half:(r + 1) * half])
    # Both outputs are bf16 roundings of fp32 results that differ only in the
    # order of the partial merges (the fp32 rounding of sums over a row's
    # keys): each is within half a bf16 unit in the last place (of the row's
    # largest output) of its fp32 value, and the fp32 values differ by
    # rounding noise, so the two agree to two such units.
    g, s = gathered.float(), single.float()
    d = (g - s).abs()
    row_max = torch.maximum(g.abs(), s.abs()).amax(dim=-1, keepdim=True).clamp_min(2.0 ** -126)
    ulp = torch.exp2(torch.floor(torch.log2(row_max)) - 7)
    assert bool((d <= 2 * ulp).all()), float((d / ulp).max())
    assert float(d.mean()) < 2e-3


def _peer_worker(rank, world, port, out_dir, mode="peer"):
    from datetime import timedelta

    from cast_b200 import _lib
    from cast_b200 import distributed as cd

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    layer = None
    try:
        q, k, v = _inputs()
        kw = dict(block_size=880, budget=3, policy="auto", device=dev)
        ref_layer = cd.HeadShardedRCSA(1, q.shape[1], q.shape[2], k.shape[2], 128, gather="nccl", **kw)
        ql, kl, vl = (ref_layer.local_heads(t).to(dev) for t in (q, k, v))
        ref = ref_layer(ql, kl, vl).clone()
        layer = cd.HeadShardedRCSA(1, q.shape[1], q.shape[2], k.shape[2], 128, gather=mode, **kw)
        outs = [layer(ql, kl, vl).clone() for _ in range(3)]  # both buffers, then the first again
        torch.cuda.synchronize()
        _lib.check_device(torch.cuda.current_stream(dev).cuda_stream, "peer gather")
        for o in outs:
            assert torch.equal(o, ref)
        # a CUDA graph of the call replays with the device call counter
        par = layer.peer.calls_made & 1
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
            layer.plan.select(ql, kl)
            if mode == "fused":
                layer.plan.attend(ql, kl, vl, out=layer.peer.slot(par), peers=layer.peer.peers(par))
            else:
                layer.plan.attend(ql, kl, vl, out=layer.peer.slot(par))
                layer.peer.send(par) if mode == "ce" else layer.peer.push(par)
            layer.peer.wait()
        layer.peer.gathered[par].zero_()
        dist.barrier()
        for _ in range(2):
            g.replay()
        torch.cuda.synchronize()
        _lib.check_device(torch.cuda.current_stream(dev).cuda_stream, "peer gather graph")
        assert torch.equal(layer.peer.heads(par), ref)
        del g
        if rank == 0:
            torch.save(ref.cpu(), os.path.join(out_dir, "peer_ref.pt"))
    finally:
        if layer is not None:
            layer.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["peer", "fused", "ce"])
def test_peer_gather_equals_nccl_gather(tmp_path, mode):
    """The head outputs written into the peers' gathered buffers over NVLink
    (plain peer stores into IPC buffers: a streaming launch after the
    attention, or the attention's own epilogue) give the NCCL all-gather's
    result bit for bit, on three calls in a row (both buffers) and on
    CUDA-graph replays."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    mp.start_processes(_peer_worker, args=(world, _free_port(), str(tmp_path), mode), nprocs=world,
                       join=True, start_method="spawn")
    assert os.path.exists(os.path.join(tmp_path, "peer_ref.pt"))


def _missing_rank_worker(rank, world, port, out_dir):
    from datetime import timedelta

    from cast_b200 import _lib
    from cast_b200 import distributed as cd

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    pg = None
    try:
        pg = cd.PeerGather(1, 2, 880, 128, device=dev)
        stream = torch.cuda.current_stream(dev).cuda_stream
        if rank == 0:  # waits for a flag rank 1 never raises
            pg.wait()
            try:
                _lib.check_device(stream, "peer wait")
                status = "no error"
            except _lib.CastError as exc:
                status = str(exc.status)
            with open(os.path.join(out_dir, "status.txt"), "w") as fh:
                fh.write(status)
        torch.cuda.synchronize(dev)
    finally:
        if pg is not None:
            pg.close()
        dist.destroy_process_group()


def test_peer_wait_reports_a_missing_rank(tmp_path):
    """A rank that makes no call: the other rank's bounded wait for its flag
    gives up after a second and reports CAST_ERR_DEVICE_TIMEOUT; no hang, no
    fault, and both ranks leave through the collective close."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    mp.start_processes(_missing_rank_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    with open(os.path.join(tmp_path, "status.txt")) as fh:
        assert fh.read() == "6"  # CAST_ERR_DEVICE_TIMEOUT
