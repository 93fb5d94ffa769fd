"""Tensor-parallel engine on 2 GPUs (NCCL) against the single-GPU engine, same weights.

Two spawned ranks shard a small seeded Qwen3.5 (2 GDN k heads / 4 v heads, 4 attention q heads
over 1 KV head, so TP 2 also exercises the KV-head replication) with tp.shard_model, run
TPEngine over two prompts and four teacher-forced decode steps, eagerly (rank 0 writes the logits
of every step) and with CUDA-graph decode (the NCCL all-reduces captured in the graphs; its tokens
must equal the eager argmax bit for bit), for each way of summing the row-parallel projections:
cuBLAS + all-reduce fused into the add/norm (default), cuBLAS + peer all-reduce + add/norm and cuBLAS
+ push + pull/add/norm (both bit-identical logits), and the tcgen05 projection pushing its tiles
(gdn_linear_push).  The parent runs CBEngine on one GPU with the same model
and feed and compares the logits: the all-reduce changes the summation order, so the check is
bf16 tolerance (2e-2 relative to the logit scale), not bits.
Skipped when fewer than two GPUs are visible.
"""
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from conftest import pkg

pytestmark = pytest.mark.gpu

TEXT = dict(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=4, num_attention_heads=4,
            num_key_value_heads=1, head_dim=64, linear_num_key_heads=2, linear_num_value_heads=4,
            linear_key_head_dim=128, linear_value_head_dim=128, linear_conv_kernel_dim=4,
            layer_types=["linear_attention", "linear_attention", "linear_attention", "full_attention"],
            max_position_embeddings=512, rms_norm_eps=1e-6, attention_bias=False, hidden_act="silu")
VISION = dict(depth=1, hidden_size=32, num_heads=2, intermediate_size=64, out_hidden_size=256)


def build_model(device):
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5Config
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5ForConditionalGeneration
    torch.manual_seed(7)
    model = Qwen3_5ForConditionalGeneration(Qwen3_5Config(text_config=TEXT, vision_config=VISION))
    with torch.no_grad():
        for name, p in model.named_parameters():
            if p.dim() == 2 and "visual" not in name:
                p.mul_(4.0)
    return model.to(torch.bfloat16).to(device).eval()


def feed():
    """Two prompts and four teacher-forced decode tokens per slot (fixed, not argmax)."""
    g = torch.Generator(device="cpu").manual_seed(3)
    ids = [torch.randint(0, TEXT["vocab_size"], (1, L), generator=g) for L in (37, 70)]
    toks = [torch.randint(0, TEXT["vocab_size"], (2,), generator=g).tolist() for _ in range(4)]
    return ids, toks


def run(engine_cls, model, device, graph, **kw):
    """Eager: the logits of the prefill and of each decode step (hooked).  Graph: the tokens each
    graph-replayed decode step returns."""
    ids, toks = feed()
    logits = []
    h = None
    if not graph:                            # (a hook cannot copy to the host inside a graph capture)
        h = model.lm_head.register_forward_hook(lambda m, i, o: logits.append(o.detach().float().cpu().numpy()))
    eng = engine_cls(model, 2, 128, device, graph_decode=graph, **kw)
    eng.prefill_batch([0, 1], ids)
    outs = [eng.decode_step([0, 1], t) for t in toks]
    if h is not None:
        h.remove()
    if hasattr(eng, "close"):
        eng.check_errors()
        eng.close()
    else:
        eng._graphs.clear()
        eng._graph_out.clear()
    return outs if graph else logits


def _rank(rank, world, port, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["LOCAL_RANK"] = str(rank)
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from conftest import pkg as _pkg
    tp = _pkg("tp")
    tp.init_tp(rank, world, "nccl", str(port), timeout_s=60)
    try:
        dev = torch.device("cuda", rank)
        model = build_model(dev)
        tp.shard_model(model, rank, world)
        logits = run(tp.TPEngine, model, dev, False, tp=world)
        graph_toks = run(tp.TPEngine, model, dev, True, tp=world)
        # graph replay (all-reduces inside the graph) == eager, bit for bit on this rank
        eager_toks = [lg.argmax(-1).tolist() for lg in logits[1:]]
        assert graph_toks == eager_toks, (graph_toks, eager_toks)
        # the other decode sums: cuBLAS + peer all-reduce + add/norm, and the tcgen05 projection pushing
        # its tiles (gdn_linear_push) before the pull + add + norm
        other = {}
        for mode in ("peer", "push", "fused"):
            lg = run(tp.TPEngine, model, dev, False, tp=world, decode_sum=mode)
            gt = run(tp.TPEngine, model, dev, True, tp=world, decode_sum=mode)
            assert gt == [x.argmax(-1).tolist() for x in lg[1:]], mode
            other[mode] = lg
        flogits = other["fused"]
        # arnorm (default), push and peer sum the same cuBLAS partials in the same rank order: the same
        # logits bit for bit
        for mode in ("peer", "push"):
            for a, b in zip(logits, other[mode]):
                assert np.array_equal(a, b), mode
        # the LM head split by vocabulary (cross-rank packed argmax, captured in the graphs): the same
        # tokens wherever the eager logits' top two are not a near-tie
        vmodel = build_model(dev)
        tp.shard_model(vmodel, rank, world, vocab_parallel=True)
        vtoks = run(tp.TPEngine, vmodel, dev, True, tp=world)
        for lg, vt in zip(logits[1:], vtoks):
            top2 = np.sort(lg, axis=-1)[:, -2:]
            for row, tok in enumerate(vt):
                if top2[row, 1] - top2[row, 0] > 2e-2 * max(1.0, abs(top2[row, 1])):
                    assert tok == int(lg[row].argmax()), (row, tok, int(lg[row].argmax()))
        if rank == 0:
            np.savez(out_path, *logits)
            np.savez(out_path + ".fused.npz", *flogits)
    finally:
        import torch.distributed as dist
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_tp2_engine_matches_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    with tempfile.TemporaryDirectory() as d:
        out_path = os.path.join(d, "tp2.npz")
        ctx = mp.get_context("spawn")
        port = _free_port()
        procs = [ctx.Process(target=_rank, args=(r, 2, port, out_path)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=300)
        codes = [p.exitcode for p in procs]
        for p in procs:
            if p.is_alive():
                p.kill()
        assert codes == [0, 0], codes
        tp_logits = [v for _, v in sorted(np.load(out_path).items(), key=lambda kv: int(kv[0].split("_")[1]))]
        fused_logits = [v for _, v in sorted(np.load(out_path + ".fused.npz").items(),
                                             key=lambda kv: int(kv[0].split("_")[1]))]
    eng = pkg("engine")
    ref = run(eng.CBEngine, build_model(torch.device("cuda", 0)), torch.device("cuda", 0), False)
    assert len(ref) == len(tp_logits) == len(fused_logits) == 5
    for step, (a, f, b) in enumerate(zip(tp_logits, fused_logits, ref)):
        err = float(np.abs(a - b).max())
        assert err <= 2e-2 * float(np.abs(b).max()) + 2e-2, (step, err)
        ferr = float(np.abs(f - b).max())
        assert ferr <= 2e-2 * float(np.abs(b).max()) + 2e-2, (step, ferr)
