"""The row-parallel projection fused with its sum over ranks (gdn_linear_allreduce,
tp.PeerLinearAllReduce) on 2 GPUs (4 when four are visible), one process each.

Each rank's product is rounded to bf16 as the unfused GEMM output would be, and the ranks'
partials are summed in rank order in fp32 and rounded once.  gdn_linear with the same split count
computes exactly that per-rank partial, so every rank checks its result BIT FOR BIT against
bf16(sum over r of fp32(gdn_linear(x_r, W_r)))
(the partials gathered with NCCL), and that all ranks hold identical results.  Shapes change from
call to call (the per-segment epochs and the double-buffered slots must stay in step; outputs
narrower than the buffers; 1-128 tokens), the calls are also captured in a CUDA graph and replayed
with fresh inputs, and the result is compared with F.linear + NCCL all-reduce within bf16
tolerance.  The push / pull split (gdn_linear_push, or a cuBLAS product pushed by gdn_push_partial,
then gdn_pull_add_rmsnorm summing the ranks, adding the residual and normalizing) must equal the all-reduce output added to the residual in bf16
and ops.rmsnorm BIT FOR BIT, eagerly, mixed with full fused calls, and captured in a graph; so must
the all-reduce fused into the residual add + RMSNorm (gdn_allreduce_add_rmsnorm) against
PeerAllReduce, the add and ops.rmsnorm, for 1-128 rows, eagerly and in a graph.  A second
instance with a short spin limit checks the failure path: only rank 0 calls, its waits run out (in
the fused call, and in the pull after a push), it reports error 3 and leaves y / x / out unwritten,
while the other ranks wait in a host barrier (buffers mapped, no kernel in flight).  Skipped when fewer than two GPUs are visible.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

HIDDEN = 5120
MAX_ROWS = 128
# (tokens, output features, local k): decode shapes of TP 2-8 and odd ones
CASES = [(32, 5120, 3072), (32, 5120, 8704), (7, 1040, 1000), (128, 5120, 768), (16, 5120, 2176), (1, 8, 64),
         (64, 2056, 4352)]


def inp(rank, case, n, n_out, k):
    g = torch.Generator(device="cpu").manual_seed(1000 * case + rank)
    x = torch.randn(n, k, generator=g).to(torch.bfloat16)
    w = (torch.randn(n_out, k, generator=g) / k ** 0.5).to(torch.bfloat16)
    return x, w


def _rank(rank, world, port, q):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from conftest import pkg
    os.environ["LOCAL_RANK"] = str(rank)
    tp = pkg("tp")
    ops = pkg("ops")
    tp.init_tp(rank, world, "nccl", str(port), timeout_s=60)
    import torch.distributed as dist
    dev = torch.device("cuda", rank)
    out = {}

    def expected(x, w, waits=True):
        # the split count of the launch: the fused call (which waits for the other ranks) keeps all
        # its clusters resident; the push (no wait) plans as a one-rank projection
        S = ops.linear_plan(x.shape[0], w.shape[0], x.shape[1], world=world if waits else 1)["splits"]
        part = ops.linear(x, w, splits=S)             # this rank's bf16 partial, same split count
        parts = [torch.empty_like(part) for _ in range(world)]
        dist.all_gather(parts, part)
        acc = torch.zeros(part.shape, dtype=torch.float32, device=dev)
        for p in parts:
            acc += p.float()
        return acc.to(torch.bfloat16)

    def same_on_all(y):
        ys = [torch.empty_like(y) for _ in range(world)]
        dist.all_gather(ys, y)
        return all(torch.equal(ys[0], t) for t in ys)

    try:
        fl = tp.PeerLinearAllReduce(MAX_ROWS, HIDDEN, dev)
        ok, same, close = True, True, True
        for rep in range(2):
            for case, (n, n_out, k) in enumerate(CASES):
                x, w = (t.to(dev) for t in inp(rank, 10 * rep + case, n, n_out, k))
                assert fl.applies(x, w)
                y = fl(x, w)
                ok &= torch.equal(y, expected(x, w))
                same &= same_on_all(y)
                if case == 0:
                    z = torch.nn.functional.linear(x, w)
                    dist.all_reduce(z)
                    mag = (x.float().abs() @ w.float().abs().t())
                    mag_all = mag.clone()
                    dist.all_reduce(mag_all)
                    close &= bool(((y.float() - z.float()).abs() <= 2 ** -6 * mag_all + 1e-2).all())
        torch.cuda.synchronize()
        out["eager"], out["same"], out["nccl_close"] = ok, same, close
        # CUDA graph: three fused projections captured, replayed with fresh inputs
        shapes = [CASES[0], CASES[3], CASES[1]]
        xs = [torch.zeros(n, k, dtype=torch.bfloat16, device=dev) for n, _, k in shapes]
        ws = [torch.zeros(n_out, k, dtype=torch.bfloat16, device=dev) for _, n_out, k in shapes]
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(graph, stream=s):
                ys = [fl(x, w) for x, w in zip(xs, ws)]
        torch.cuda.current_stream().wait_stream(s)
        ok = True
        for rep in range(3):
            for i, (n, n_out, k) in enumerate(shapes):
                x, w = inp(rank, 500 + 10 * rep + i, n, n_out, k)
                xs[i].copy_(x)
                ws[i].copy_(w)
            graph.replay()
            torch.cuda.synchronize()
            for i in range(len(shapes)):
                ok &= torch.equal(ys[i], expected(xs[i], ws[i]))
        out["graph"] = ok
        del graph
        # push / pull split: the projection sends its partial, the residual add + RMSNorm sums the
        # ranks (bit for bit: all-reduce output, x + h in bf16, then ops.rmsnorm)
        nw = (torch.randn(HIDDEN, generator=torch.Generator().manual_seed(3)) * 0.1).to(torch.bfloat16).to(dev)
        ok = True
        for rep in range(2):
            for case, (n, n_out, k) in enumerate([CASES[0], CASES[4], CASES[1], CASES[3]]):
                x, w = (t.to(dev) for t in inp(rank, 300 + 10 * rep + case, n, n_out, k))
                res = (torch.randn(n, HIDDEN, generator=torch.Generator().manual_seed(77 + case)) * 2).to(
                    torch.bfloat16).to(dev)
                ref_x = res + expected(x, w, waits=False)
                ref_out = ops.rmsnorm(ref_x, nw, 1e-6)
                fl.push(x, w)
                got = fl.pull_add_rmsnorm(res, nw, 1e-6)
                ok &= torch.equal(res, ref_x) and torch.equal(got, ref_out)
                if case == 1:                # a full fused call between push/pull pairs
                    ok &= torch.equal(fl(x, w), expected(x, w))
                # the push of a product computed elsewhere (cuBLAS): the sum of the ranks' cuBLAS partials
                part = torch.nn.functional.linear(x, w)
                parts = [torch.empty_like(part) for _ in range(world)]
                dist.all_gather(parts, part)
                acc = torch.zeros(part.shape, dtype=torch.float32, device=dev)
                for pp in parts:
                    acc += pp.float()
                res2 = (torch.randn(n, HIDDEN, generator=torch.Generator().manual_seed(91 + case)) * 2).to(
                    torch.bfloat16).to(dev)
                ref2_x = res2 + acc.to(torch.bfloat16)
                fl.push_partial(part)
                got2 = fl.pull_add_rmsnorm(res2, nw, 1e-6)
                ok &= torch.equal(res2, ref2_x) and torch.equal(got2, ops.rmsnorm(ref2_x, nw, 1e-6))
        out["push_pull"] = bool(ok)
        # push / pull captured in a graph (two pairs), replayed with fresh inputs
        pshapes = [CASES[0], CASES[1]]
        pxs = [torch.zeros(n, k, dtype=torch.bfloat16, device=dev) for n, _, k in pshapes]
        pws = [torch.zeros(n_out, k, dtype=torch.bfloat16, device=dev) for _, n_out, k in pshapes]
        pres = torch.zeros(32, HIDDEN, dtype=torch.bfloat16, device=dev)
        s.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(graph, stream=s):
                fl.push(pxs[0], pws[0])
                pout1 = fl.pull_add_rmsnorm(pres, nw, 1e-6)
                fl.push(pxs[1], pws[1])
                pout2 = fl.pull_add_rmsnorm(pres, nw, 1e-6)
        torch.cuda.current_stream().wait_stream(s)
        ok = True
        for rep in range(3):
            for i, (n, n_out, k) in enumerate(pshapes):
                x, w = inp(rank, 700 + 10 * rep + i, n, n_out, k)
                pxs[i].copy_(x)
                pws[i].copy_(w)
            r0 = (torch.randn(32, HIDDEN, generator=torch.Generator().manual_seed(800 + rep))).to(torch.bfloat16)
            pres.copy_(r0)
            graph.replay()
            torch.cuda.synchronize()
            x1 = r0.to(dev) + expected(pxs[0], pws[0], waits=False)
            x2 = x1 + expected(pxs[1], pws[1], waits=False)
            o2 = ops.rmsnorm(x2, nw, 1e-6)
            ok &= torch.equal(pres, x2) and torch.equal(pout2, o2) and torch.equal(pout1, ops.rmsnorm(x1, nw, 1e-6))
        out["push_pull_graph"] = bool(ok)
        del graph
        # the all-reduce fused into the residual add + RMSNorm (gdn_allreduce_add_rmsnorm): bit for
        # bit PeerAllReduce -> x + h -> ops.rmsnorm, eagerly and in a graph, rows changing per call
        arn = tp.PeerAllReduceAddNorm(MAX_ROWS, HIDDEN, dev)
        par = tp.PeerAllReduce(MAX_ROWS * HIDDEN, dev)
        ok = True
        for case, rows in enumerate([32, 1, 128, 17, 32]):
            g0 = torch.Generator().manual_seed(40 + case)
            h = (torch.randn(world, rows, HIDDEN, generator=g0) * 3).to(torch.bfloat16)[rank].to(dev)
            res0 = (torch.randn(rows, HIDDEN, generator=g0) * 2).to(torch.bfloat16).to(dev)
            hs = h.clone()
            par(hs)
            ref_x = res0 + hs
            res = res0.clone()
            got = arn(res, h, nw, 1e-6)
            ok &= torch.equal(res, ref_x) and torch.equal(got, ops.rmsnorm(ref_x, nw, 1e-6))
        hb = torch.zeros(32, HIDDEN, dtype=torch.bfloat16, device=dev)
        rb = torch.zeros(32, HIDDEN, dtype=torch.bfloat16, device=dev)
        s.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(graph, stream=s):
                go1 = arn(rb, hb, nw, 1e-6)
                go2 = arn(rb, hb, nw, 1e-6)
        torch.cuda.current_stream().wait_stream(s)
        for rep in range(3):
            g0 = torch.Generator().manual_seed(60 + rep)
            h = (torch.randn(world, 32, HIDDEN, generator=g0) * 3).to(torch.bfloat16)[rank].to(dev)
            r0 = (torch.randn(32, HIDDEN, generator=g0) * 2).to(torch.bfloat16).to(dev)
            hb.copy_(h)
            rb.copy_(r0)
            graph.replay()
            torch.cuda.synchronize()
            hs = h.clone()
            par(hs)
            x1 = r0 + hs
            x2 = x1 + hs
            ok &= torch.equal(rb, x2) and torch.equal(go1, ops.rmsnorm(x1, nw, 1e-6)) and torch.equal(
                go2, ops.rmsnorm(x2, nw, 1e-6))
        out["arnorm"] = bool(ok)
        del graph
        arn.close()
        par.close()
        out["err"] = int(fl.err.item())
        out["applies_big"] = fl.applies(torch.zeros(MAX_ROWS + 1, 64, dtype=torch.bfloat16, device=dev),
                                        torch.zeros(64, 64, dtype=torch.bfloat16, device=dev))
        fl.close()
        # failure path: rank 0 alone calls; its bounded waits run out
        fl2 = tp.PeerLinearAllReduce(16, 1024, dev, spin_limit=20000)
        arn2 = tp.PeerAllReduceAddNorm(16, 1024, dev, spin_limit=20000)
        if rank == 0:
            x, w = (t.to(dev) for t in inp(0, 7, 16, 1024, 512))
            y = fl2(x, w)
            torch.cuda.synchronize()
            out["timeout_err"] = int(fl2.err.item())
            fl2.err.zero_()
            res = torch.ones(16, 1024, dtype=torch.bfloat16, device=dev)
            fl2.push(x, w)
            o = fl2.pull_add_rmsnorm(res, torch.ones(1024, dtype=torch.bfloat16, device=dev), 1e-6)
            torch.cuda.synchronize()
            out["pull_timeout"] = int(fl2.err.item()) == 3 and bool((res == 1).all())
            o = arn2(res, torch.ones(16, 1024, dtype=torch.bfloat16, device=dev),
                     torch.ones(1024, dtype=torch.bfloat16, device=dev), 1e-6)
            torch.cuda.synchronize()
            out["arnorm_timeout"] = int(arn2.err.item()) == 3 and bool((res == 1).all())
        dist.barrier()                       # the other ranks wait here while rank 0's kernel runs
        fl2.close()
        arn2.close()
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_fused_linear_allreduce_multi_gpu():
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
        assert res[r]["eager"] and res[r]["same"] and res[r]["graph"] and res[r]["nccl_close"], res[r]
        assert res[r]["push_pull"] and res[r]["push_pull_graph"] and res[r]["arnorm"], res[r]
        assert res[r]["err"] == 0 and not res[r]["applies_big"], res[r]
    assert res[0]["timeout_err"] == 3 and res[0]["pull_timeout"] and res[0]["arnorm_timeout"], res[0]
