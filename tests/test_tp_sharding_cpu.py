"""CPU (gloo, world size 2 and 4) tests of the tensor-parallel sharding.

Every rank builds the same tiny fp32 Qwen3.5, shards it with ``tp.shard_model`` and checks that
each sharded projection is exactly the matching slice of the full one, and that the row-parallel
projections followed by the all-reduce of ``AllReduceLinear`` equal the full projection
(src/cb_tp.py:25-106).  World size 4 exercises KV-head replication (1 KV head over 4 ranks).
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _tiny_fp32():
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5Config
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5ForConditionalGeneration
    tc = dict(vocab_size=64, hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
              num_key_value_heads=1, head_dim=16, linear_num_key_heads=4, linear_num_value_heads=8,
              linear_key_head_dim=16, linear_value_head_dim=16, linear_conv_kernel_dim=4,
              layer_types=["linear_attention", "full_attention"], max_position_embeddings=128, rms_norm_eps=1e-6,
              attention_bias=False, hidden_act="silu")
    torch.manual_seed(0)
    cfg = Qwen3_5Config(text_config=tc, vision_config=dict(depth=1, hidden_size=32, num_heads=2,
                                                          intermediate_size=64, out_hidden_size=64))
    return Qwen3_5ForConditionalGeneration(cfg).float().eval()


def _worker(rank, world, port, q):
    import importlib
    import sys
    sys.path.insert(0, ROOT)
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        tp = importlib.import_module("910b_e2e_accleration_by_codex_b200.tp")
        full = _tiny_fp32()
        shard = tp.shard_model(_tiny_fp32(), rank, world)
        torch.manual_seed(1)
        x = torch.randn(3, 5, 64)
        lf, ls = full.model.language_model.layers, shard.model.language_model.layers
        with torch.no_grad():
            # GDN layer 0
            gf, gs = lf[0].linear_attn, ls[0].linear_attn
            kh_l, vh_l = 4 // world, 8 // world
            idx = torch.cat([torch.arange(rank * kh_l * 16, (rank + 1) * kh_l * 16),
                             64 + torch.arange(rank * kh_l * 16, (rank + 1) * kh_l * 16),
                             128 + torch.arange(rank * vh_l * 16, (rank + 1) * vh_l * 16)])
            # (GEMMs of different widths may sum in different orders: compare to fp32 rounding)
            assert torch.allclose(gs.in_proj_qkv(x), gf.in_proj_qkv(x)[..., idx], atol=1e-6)
            assert torch.equal(gs.conv1d.weight, gf.conv1d.weight[idx])
            vr = slice(rank * vh_l * 16, (rank + 1) * vh_l * 16)
            assert torch.allclose(gs.in_proj_z(x), gf.in_proj_z(x)[..., vr], atol=1e-6)
            hr = slice(rank * vh_l, (rank + 1) * vh_l)
            assert torch.allclose(gs.in_proj_a(x), gf.in_proj_a(x)[..., hr], atol=1e-6)
            assert torch.equal(gs.A_log, gf.A_log[hr]) and torch.equal(gs.dt_bias, gf.dt_bias[hr])
            core = torch.randn(3, 5, 128)
            assert torch.allclose(gs.out_proj(core[..., vr]), gf.out_proj(core), atol=1e-5)
            assert gs.num_v_heads == vh_l and gs.conv_dim == 2 * kh_l * 16 + vh_l * 16
            # attention layer 1: q heads split, the single KV head replicated on every rank
            af, as_ = lf[1].self_attn, ls[1].self_attn
            nh_l = 4 // world
            qf = af.q_proj(x).view(3, 5, 4, 32)
            assert torch.allclose(as_.q_proj(x).view(3, 5, nh_l, 32), qf[:, :, rank * nh_l:(rank + 1) * nh_l],
                                  atol=1e-6)
            assert torch.allclose(as_.k_proj(x), af.k_proj(x), atol=1e-6)
            assert torch.allclose(as_.v_proj(x), af.v_proj(x), atol=1e-6)
            o = torch.randn(3, 5, 64)
            os_ = o.view(3, 5, 4, 16)[:, :, rank * nh_l:(rank + 1) * nh_l].reshape(3, 5, -1)
            assert torch.allclose(as_.o_proj(os_), af.o_proj(o), atol=1e-5)
            # MLP with its all-reduce equals the full MLP
            assert torch.allclose(ls[0].mlp(x), lf[0].mlp(x), atol=1e-5)
            # vocabulary-parallel head: this rank's rows, and the cross-rank greedy pick equals the
            # full argmax, ties included (the lowest id wins, as torch.argmax)
            vp = tp.shard_model(_tiny_fp32(), rank, world, vocab_parallel=True)
            V = 64 // world
            h = torch.randn(7, 64)
            assert torch.allclose(vp.lm_head(h), full.lm_head(h)[:, rank * V:(rank + 1) * V], atol=1e-6)
            assert torch.equal(vp.lm_head.greedy(h), full.lm_head(h).argmax(-1))
            w = full.lm_head.weight.detach().clone()
            w[5] = w[60]                                     # ids 5 and 60 tie on every row
            vp.lm_head.lin.weight.data.copy_(w[rank * V:(rank + 1) * V])
            full.lm_head.weight.data.copy_(w)
            h2 = torch.randn(6, 64)
            h2[:3] = w[60] * 50                              # rows where the tied pair leads
            assert torch.equal(vp.lm_head.greedy(h2), full.lm_head(h2).argmax(-1))
            assert vp.lm_head.greedy(h2)[:3].tolist() == [5, 5, 5]
            vp.lm_head.lin.weight.data.copy_(torch.abs(w[rank * V:(rank + 1) * V]))
            full.lm_head.weight.data.copy_(torch.abs(w))
            neg = -torch.abs(torch.randn(4, 64))             # all logits negative: the order still holds
            assert (full.lm_head(neg) < 0).all()
            assert torch.equal(vp.lm_head.greedy(neg), full.lm_head(neg).argmax(-1))
        q.put((rank, "ok"))
    except Exception as e:  # report to the parent instead of hanging it
        import traceback
        q.put((rank, traceback.format_exc()[-800:]))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_shard_model_matches_full_model(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert all(v == "ok" for v in res.values()), res


def test_head_split_rules():
    import importlib
    tp = importlib.import_module("910b_e2e_accleration_by_codex_b200.tp")
    # Qwen3.5-27B-like: 24 q heads, 4 kv heads
    assert tp.attention_head_split(24, 4, 2, 1) == (12, 12, 2, 2)
    assert tp.attention_head_split(24, 4, 4, 3) == (18, 6, 3, 1)
    for r in range(8):  # tp=8 replicates each kv head on 2 ranks; a rank's 3 q heads read it
        q0, nq, kv, nkv = tp.attention_head_split(24, 4, 8, r)
        assert nq == 3 and nkv == 1 and kv == r // 2 and q0 // 6 == kv
    with pytest.raises(ValueError):
        tp.attention_head_split(24, 4, 5, 0)
