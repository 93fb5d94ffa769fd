"""Head-sharded tensor parallelism for the hybrid Qwen3.5 model (one process per GPU, NCCL).

Mirrors the reference's src/cb_tp.py:
  * ``AllReduceLinear`` (src/cb_tp.py:25-35): row-parallel projection followed by a sum over
    ranks; the engine's attention ``o_proj``, GDN ``out_proj`` and MLP ``down_proj`` become this.
  * ``shard_model`` (src/cb_tp.py:47-106): per rank, a contiguous block of attention q heads, GDN
    k heads (with their q/k conv channels) and v heads (with their v conv channels, a/b/A_log/
    dt_bias rows, z rows and out_proj columns), and a block of MLP columns.
  * ``TPEngine`` (src/cb_tp.py:117-285): the engine on sharded weights.
One difference: the reference requires the KV-head count to divide the TP degree
(src/cb_tp.py:54), so 4 KV heads cannot run at TP=8.  Here, when tp > kv heads (tp a multiple of
them), each KV head is replicated on tp / kvh consecutive ranks, and each rank keeps the q heads
that read it, so attention is still exact.
"""
from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist
import torch.nn as nn

from .engine import CBEngine


class AllReduceLinear(nn.Module):
    """Row-parallel linear: local partial product, then the sum over ranks (identical on all)."""

    def __init__(self, lin):
        super().__init__()
        self.lin = lin

    def forward(self, x):
        y = self.lin(x)
        dist.all_reduce(y)
        return y


def _set_weight(lin, w):
    lin.weight = nn.Parameter(w.contiguous(), requires_grad=False)
    lin.out_features, lin.in_features = w.shape[0], w.shape[1]


def _rows(start, count, device):
    return torch.arange(start, start + count, device=device)


def attention_head_split(nh, kvh, tp, rank):
    """(first q head, q heads per rank, first kv head, kv heads per rank) of ``rank``.

    kvh % tp == 0: kv heads split like q heads.  tp % kvh == 0: kv head rank // (tp // kvh) is
    replicated on tp // kvh ranks; the rank's q heads all read it (q head j reads kv head
    j // (nh // kvh), as HF's repeat_kv arranges them)."""
    if nh % tp != 0:
        raise ValueError(f"{nh} attention heads do not split over tp={tp}")
    nh_l = nh // tp
    if kvh % tp == 0:
        kvh_l = kvh // tp
        return rank * nh_l, nh_l, rank * kvh_l, kvh_l
    if tp % kvh != 0:
        raise ValueError(f"{kvh} kv heads neither divide nor are divided by tp={tp}")
    rep = tp // kvh
    kv = rank // rep
    q0 = rank * nh_l
    if (q0 // (nh // kvh)) != kv or ((q0 + nh_l - 1) // (nh // kvh)) != kv:
        raise ValueError("q heads of a rank would read two kv heads")
    return q0, nh_l, kv, 1


def shard_model(model, rank, tp):
    """In-place sharding of a freshly loaded Qwen3_5ForConditionalGeneration (src/cb_tp.py:47-106)."""
    cfg = model.config.text_config
    assert tp > 0 and rank < tp
    assert not getattr(cfg, "attention_bias", False), "attention_bias not supported in TP"
    hd = cfg.head_dim
    nh, kvh = cfg.num_attention_heads, cfg.num_key_value_heads
    lm = model.model.language_model
    H = cfg.hidden_size
    q0, nh_l, kv0, kvh_l = attention_head_split(nh, kvh, tp, rank)
    for i, layer in enumerate(lm.layers):
        if cfg.layer_types[i] == "full_attention":
            at = layer.self_attn
            # q_proj: per head [q(hd), gate(hd)] interleaved; a contiguous block of heads
            _set_weight(at.q_proj, at.q_proj.weight.view(nh, 2 * hd, H)[q0:q0 + nh_l].reshape(-1, H))
            _set_weight(at.k_proj, at.k_proj.weight[kv0 * hd:(kv0 + kvh_l) * hd])
            _set_weight(at.v_proj, at.v_proj.weight[kv0 * hd:(kv0 + kvh_l) * hd])
            _set_weight(at.o_proj, at.o_proj.weight.view(H, nh, hd)[:, q0:q0 + nh_l].reshape(H, -1))
            at.o_proj = AllReduceLinear(at.o_proj)
            at.num_key_value_groups = nh_l // kvh_l
        else:
            gd = layer.linear_attn
            kh, vh = gd.num_k_heads, gd.num_v_heads
            dk, dv = gd.head_k_dim, gd.head_v_dim
            if kh % tp or vh % tp:
                raise ValueError(f"GDN heads ({kh} k, {vh} v) do not split over tp={tp}")
            kh_l, vh_l = kh // tp, vh // tp
            key_dim = gd.key_dim
            # in_proj_qkv rows: [q (kh*dk) | k (kh*dk) | v (vh*dv)]; the same head blocks in each part
            dev = gd.in_proj_qkv.weight.device
            idx = torch.cat([_rows(rank * kh_l * dk, kh_l * dk, dev), _rows(key_dim + rank * kh_l * dk, kh_l * dk, dev),
                             _rows(2 * key_dim + rank * vh_l * dv, vh_l * dv, dev)])
            _set_weight(gd.in_proj_qkv, gd.in_proj_qkv.weight.index_select(0, idx))
            gd.conv1d.weight = nn.Parameter(gd.conv1d.weight.index_select(0, idx).contiguous(), requires_grad=False)
            if gd.conv1d.bias is not None:
                gd.conv1d.bias = nn.Parameter(gd.conv1d.bias.index_select(0, idx).contiguous(), requires_grad=False)
            gd.conv1d.out_channels = gd.conv1d.in_channels = idx.numel()
            gd.conv1d.groups = idx.numel()
            vrows = _rows(rank * vh_l * dv, vh_l * dv, dev)
            _set_weight(gd.in_proj_z, gd.in_proj_z.weight.index_select(0, vrows))
            hrows = _rows(rank * vh_l, vh_l, dev)
            _set_weight(gd.in_proj_b, gd.in_proj_b.weight.index_select(0, hrows))
            _set_weight(gd.in_proj_a, gd.in_proj_a.weight.index_select(0, hrows))
            gd.A_log = nn.Parameter(gd.A_log.data[hrows].contiguous(), requires_grad=False)
            gd.dt_bias = nn.Parameter(gd.dt_bias.data[hrows].contiguous(), requires_grad=False)
            _set_weight(gd.out_proj, gd.out_proj.weight[:, rank * vh_l * dv:(rank + 1) * vh_l * dv])
            gd.out_proj = AllReduceLinear(gd.out_proj)
            gd.num_k_heads, gd.num_v_heads = kh_l, vh_l
            gd.key_dim, gd.value_dim = kh_l * dk, vh_l * dv
            gd.conv_dim = 2 * gd.key_dim + gd.value_dim
        mlp = layer.mlp
        inter = mlp.gate_proj.weight.shape[0]
        if inter % tp:
            raise ValueError(f"MLP width {inter} does not split over tp={tp}")
        r0, r1 = rank * (inter // tp), (rank + 1) * (inter // tp)
        _set_weight(mlp.gate_proj, mlp.gate_proj.weight[r0:r1])
        _set_weight(mlp.up_proj, mlp.up_proj.weight[r0:r1])
        _set_weight(mlp.down_proj, mlp.down_proj.weight[:, r0:r1])
        mlp.down_proj = AllReduceLinear(mlp.down_proj)
    return model


def init_tp(rank, world, backend="nccl", master_port="29561", timeout_s=120):
    """Process group for one rank per GPU (src/cb_tp.py:109-114); a finite timeout makes a rank
    that never arrives end the others' next collective with an error instead of a hang."""
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", master_port)
    kw = {}
    if backend == "nccl":
        local = int(os.environ.get("LOCAL_RANK", rank))
        torch.cuda.set_device(local)
        kw["device_id"] = torch.device("cuda", local)
    dist.init_process_group(backend, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s),
                            **kw)


class TPEngine(CBEngine):
    """CBEngine on sharded weights (src/cb_tp.py:117-285).  Decode graphs capture the NCCL
    all-reduces of AllReduceLinear; every rank captures the same sequence of graphs."""

    def __init__(self, model, n_slots, t_max, device, tp, graph_decode=False):
        super().__init__(model, n_slots, t_max, device, graph_decode=graph_decode, tp=tp)
