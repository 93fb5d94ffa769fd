"""Head-sharded tensor parallelism for the hybrid Qwen3.5 model (one process per GPU, NCCL).

Mirrors the reference's src/cb_tp.py:
  * ``AllReduceLinear`` (src/cb_tp.py:25-35): row-parallel projection followed by a sum over
    ranks; the engine's attention ``o_proj``, GDN ``out_proj`` and MLP ``down_proj`` become this.
  * ``shard_model`` (src/cb_tp.py:47-106): per rank, a contiguous block of attention q heads, GDN
    k heads (with their q/k conv channels) and v heads (with their v conv channels, a/b/A_log/
    dt_bias rows, z rows and out_proj columns), and a block of MLP columns.
  * ``TPEngine`` (src/cb_tp.py:117-285): the engine on sharded weights.
  * ``PeerAllReduce``: the sum over ranks for decode-sized outputs by this library's own kernel over
    IPC-mapped peer buffers (gdn_allreduce); NCCL keeps the larger (prefill) ones.
One difference: the reference requires the KV-head count to divide the TP degree
(src/cb_tp.py:54), so 4 KV heads cannot run at TP=8.  Here, when tp > kv heads (tp a multiple of
them), each KV head is replicated on tp / kvh consecutive ranks, and each rank keeps the q heads
that read it, so attention is still exact.
"""
from __future__ import annotations

import ctypes as C
import datetime
import os

import torch
import torch.distributed as dist
import torch.nn as nn

from . import _lib
from .engine import CBEngine


class PeerAllReduce:
    """In-place sum over the ranks of the process group (one process per GPU, one node) by
    gdn_allreduce over IPC-mapped peer buffers, for bf16 outputs of up to ``max_elems`` elements.
    Collective: every rank constructs it, calls it on tensors of the same sizes in the same order
    (CUDA-graph capture included) and closes it.  Each rank's result is the fp32 sum in rank order
    rounded once to bf16, identical on all ranks.  If a rank does not arrive within ``spin_limit``
    polls the others set ``err`` to 3 and leave their tensor as it was; the instance is then out of
    step and must be closed."""

    def __init__(self, max_elems, device, spin_limit=0):
        lib = _lib.load()
        self.lib = lib
        self.rank, self.world = dist.get_rank(), dist.get_world_size()
        self.max_elems = int(max_elems)
        self.spin_limit = int(spin_limit)
        nbytes = lib.gdn_ar_buffer_bytes(self.world, self.max_elems, _lib.GDN_BF16)
        if nbytes == 0:
            raise RuntimeError(f"PeerAllReduce: world {self.world} not supported (1..8 ranks)")
        own = C.c_void_p()
        _lib.check(lib.gdn_ar_alloc(nbytes, C.byref(own)), "gdn_ar_alloc")
        handle = C.create_string_buffer(_lib.GDN_IPC_HANDLE_BYTES)
        _lib.check(lib.gdn_ar_ipc_handle(own, handle), "gdn_ar_ipc_handle")
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.raw)
        ptrs = []
        for r, hb in enumerate(handles):
            if r == self.rank:
                ptrs.append(own.value)
                continue
            peer = C.c_void_p()
            _lib.check(lib.gdn_ar_ipc_open(C.create_string_buffer(hb, _lib.GDN_IPC_HANDLE_BYTES), C.byref(peer)),
                       "gdn_ar_ipc_open")
            ptrs.append(peer.value)
        self._own, self._ptrs = own.value, ptrs
        self._table = (C.c_void_p * self.world)(*ptrs)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        self.closed = False

    def applies(self, y):
        """Whether ``y`` goes through this kernel (the same answer on every rank for the same shape)."""
        return (not self.closed and y.dtype == torch.bfloat16 and y.numel() <= self.max_elems
                and y.numel() % 8 == 0)

    def __call__(self, y):
        """Sum ``y`` over the ranks in place; returns ``y``."""
        if not y.is_contiguous() or y.data_ptr() % 16:
            z = y.contiguous().clone()
            self(z)
            y.copy_(z)
            return y
        _lib.check(self.lib.gdn_allreduce(y.data_ptr(), y.data_ptr(), y.numel(), _lib.GDN_BF16, self.rank,
                                          self.world, self._table, self.max_elems, self.spin_limit,
                                          self.err.data_ptr(), torch.cuda.current_stream().cuda_stream),
                   "gdn_allreduce")
        return y

    def close(self):
        """Collective: after every rank's last call, unmap the peers' buffers and free this one."""
        if self.closed:
            return
        self.closed = True
        torch.cuda.synchronize()
        dist.barrier()
        for r, ptr in enumerate(self._ptrs):
            if r != self.rank:
                _lib.check(self.lib.gdn_ar_ipc_close(ptr), "gdn_ar_ipc_close")
        dist.barrier()  # no rank writes into this buffer any more
        _lib.check(self.lib.gdn_ar_free(self._own), "gdn_ar_free")


_PEER_AR = None


def enable_peer_allreduce(max_elems, device, spin_limit=0):
    """Collective: route AllReduceLinear's sums of up to ``max_elems`` bf16 elements through a
    PeerAllReduce (returned); larger ones stay on NCCL."""
    global _PEER_AR
    disable_peer_allreduce()
    _PEER_AR = PeerAllReduce(max_elems, device, spin_limit)
    return _PEER_AR


def disable_peer_allreduce():
    """Collective: close the PeerAllReduce in use, if any."""
    global _PEER_AR
    if _PEER_AR is not None:
        _PEER_AR.close()
        _PEER_AR = None


class AllReduceLinear(nn.Module):
    """Row-parallel linear: local partial product, then the sum over ranks (identical on all):
    the peer-memory kernel for decode-sized outputs when enabled, NCCL otherwise."""

    def __init__(self, lin):
        super().__init__()
        self.lin = lin

    def forward(self, x):
        y = self.lin(x)
        ar = _PEER_AR
        if ar is not None and ar.applies(y):
            ar(y)
        else:
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
    """CBEngine on sharded weights (src/cb_tp.py:117-285).  With ``peer_allreduce`` (default) the
    decode steps' row-parallel sums ([slots, hidden] bf16) go through PeerAllReduce and prefill's
    larger ones through NCCL; decode graphs capture whichever runs, and every rank captures the same
    sequence of graphs.  ``close()`` (collective) releases the graphs and the peer buffers."""

    def __init__(self, model, n_slots, t_max, device, tp, graph_decode=False, peer_allreduce=True):
        self.peer_ar = None
        if peer_allreduce and tp > 1:
            hidden = model.config.text_config.hidden_size
            self.peer_ar = enable_peer_allreduce(n_slots * hidden, device)
        super().__init__(model, n_slots, t_max, device, graph_decode=graph_decode, tp=tp)

    def check_errors(self):
        """Raise if a peer all-reduce timed out (a rank did not arrive)."""
        if self.peer_ar is not None and int(self.peer_ar.err.item()) != 0:
            raise RuntimeError(f"peer all-reduce error {int(self.peer_ar.err.item())} (a rank did not arrive)")

    def close(self):
        """Collective: release the decode graphs and the peer all-reduce buffers."""
        self._graphs.clear()
        self._graph_out.clear()
        if self.peer_ar is not None:
            torch.cuda.synchronize()
            if _PEER_AR is self.peer_ar:
                disable_peer_allreduce()
            else:
                self.peer_ar.close()
            self.peer_ar = None
