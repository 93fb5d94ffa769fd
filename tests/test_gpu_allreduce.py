"""Peer-memory all-reduce (gdn_allreduce, tp.PeerAllReduce) on 2 GPUs (4 when four are visible),
one process each.

Every rank can regenerate every rank's seeded input, so each checks its result bit for bit against
the fp32 sum in rank order rounded once to bf16: over sizes that change from call to call (the
double-buffered slots alternate), inside a CUDA graph replayed with fresh inputs, and against
NCCL's sum within its bf16 roundings (one per reduction step, bounded by the inputs' magnitudes).  A second instance with a short spin limit checks the failure
path: only rank 0 calls, its wait runs out, it reports error 3 and leaves its tensor untouched (a
later call returns without waiting), and the other rank stays in a host barrier (its buffer
mapped, no kernel in flight) until rank 0 is done.  Skipped when fewer than two GPUs are visible.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

SIZES = [8, 5120, 16 * 5120, 40 * 5120 + 8, 64 * 5120, 4096]
MAX = 64 * 5120


def inp(rank, case, n):
    g = torch.Generator(device="cpu").manual_seed(1000 * case + rank)
    return (torch.randn(n, generator=g) * 4).to(torch.bfloat16)


def expect(world, case, n):
    acc = torch.zeros(n, dtype=torch.float32)
    for r in range(world):
        acc += inp(r, case, n).float()
    return acc.to(torch.bfloat16)


def _rank(rank, world, port, q):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from conftest import pkg
    os.environ["LOCAL_RANK"] = str(rank)
    tp = pkg("tp")
    tp.init_tp(rank, world, "nccl", str(port), timeout_s=60)
    import torch.distributed as dist
    dev = torch.device("cuda", rank)
    out = {}
    try:
        ar = tp.PeerAllReduce(MAX, dev)
        # eager, sizes changing between calls
        ok = True
        for case, n in enumerate(SIZES * 2):
            y = inp(rank, case, n).to(dev)
            ar(y)
            ok &= torch.equal(y.cpu(), expect(world, case, n))
        torch.cuda.synchronize()
        out["eager"] = ok
        # NCCL agrees within one bf16 rounding
        n = 16 * 5120
        y = inp(rank, 99, n).to(dev)
        z = y.clone()
        ar(y)
        dist.all_reduce(z)
        mag = sum(inp(r, 99, n).float().abs() for r in range(world)).to(dev)
        out["nccl_close"] = bool(((y.float() - z.float()).abs() <= world * 2 ** -8 * mag + 1e-3).all())
        # CUDA graph: three captured calls of different sizes, replayed with fresh inputs
        bufs = [torch.zeros(n, dtype=torch.bfloat16, device=dev) for n in (5120, 64 * 5120, 8 * 5120)]
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(graph, stream=s):
                for b in bufs:
                    ar(b)
        torch.cuda.current_stream().wait_stream(s)
        ok = True
        for rep in range(4):
            for i, b in enumerate(bufs):
                b.copy_(inp(rank, 200 + 10 * rep + i, b.numel()))
            graph.replay()
            torch.cuda.synchronize()
            for i, b in enumerate(bufs):
                ok &= torch.equal(b.cpu(), expect(world, 200 + 10 * rep + i, b.numel()))
        out["graph"] = ok
        del graph
        out["err"] = int(ar.err.item())
        # a tensor larger than the slot is not taken
        out["applies_big"] = ar.applies(torch.zeros(MAX + 8, dtype=torch.bfloat16, device=dev))
        ar.close()
        # failure path: rank 0 alone calls; its bounded wait runs out
        ar2 = tp.PeerAllReduce(5120, dev, spin_limit=20000)
        if rank == 0:
            y = inp(0, 7, 5120).to(dev)
            ar2(y)
            torch.cuda.synchronize()
            out["timeout_err"] = int(ar2.err.item())
            out["timeout_untouched"] = torch.equal(y.cpu(), inp(0, 7, 5120))
            ar2(y)                           # out of step now: returns without waiting again
            torch.cuda.synchronize()
            out["timeout_untouched"] &= torch.equal(y.cpu(), inp(0, 7, 5120)) and int(ar2.err.item()) == 3
        dist.barrier()                       # rank 1 waits here while rank 0's kernel runs
        ar2.close()
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_peer_allreduce_multi_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 4 if torch.cuda.device_count() >= 4 else 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0] * world, codes
    res = dict(q.get(timeout=5) for _ in range(world))
    for r in range(world):
        assert res[r]["eager"] and res[r]["graph"] and res[r]["nccl_close"], res[r]
        assert res[r]["err"] == 0 and not res[r]["applies_big"], res[r]
    assert res[0]["timeout_err"] == 3 and res[0]["timeout_untouched"], res[0]
