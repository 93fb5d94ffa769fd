"""Head-sharded tensor parallelism for the hybrid Qwen3.5 model (one process per GPU, NCCL).

Mirrors the reference's src/cb_tp.py:
  * ``AllReduceLinear`` (src/cb_tp.py:25-35): row-parallel projection followed by a sum over
    ranks; the engine's attention ``o_proj``, GDN ``out_proj`` and MLP ``down_proj`` become this.
  * ``shard_model`` (src/cb_tp.py:47-106): per rank, a contiguous block of attention q heads, GDN
    k heads (with their q/k conv channels) and v heads (with their v conv channels, a/b/A_log/
    dt_bias rows, z rows and out_proj columns), and a block of MLP columns, applied from one
    table of (weight, axis, index) cuts; optionally the LM head split by vocabulary.
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

from . import _lib, ops
from .engine import CBEngine


class _PeerBuffers:
    """One device buffer per rank (gdn_ar_alloc, zero-filled) whose CUDA IPC handle every other rank
    opens, so each rank holds plain pointers to all buffers of the node.  Collective: every rank
    constructs it and closes it."""

    def __init__(self, nbytes, device, what):
        lib = _lib.load()
        self.lib = lib
        self.rank, self.world = dist.get_rank(), dist.get_world_size()
        if nbytes == 0:
            raise RuntimeError(f"{what}: world {self.world} or the sizes are not supported")
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


class PeerAllReduce(_PeerBuffers):
    """In-place sum over the ranks of the process group (one process per GPU, one node) by
    gdn_allreduce over IPC-mapped peer buffers, for bf16 outputs of up to ``max_elems`` elements.
    Collective: every rank constructs it, calls it on tensors of the same sizes in the same order
    (CUDA-graph capture included) and closes it.  Each rank's result is the fp32 sum in rank order
    rounded once to bf16, identical on all ranks.  If a rank does not arrive within ``spin_limit``
    polls the others set ``err`` to 3 and leave their tensor as it was; the instance is then out of
    step and must be closed."""

    def __init__(self, max_elems, device, spin_limit=0):
        self.max_elems = int(max_elems)
        self.spin_limit = int(spin_limit)
        nbytes = _lib.load().gdn_ar_buffer_bytes(dist.get_world_size(), self.max_elems, _lib.GDN_BF16)
        super().__init__(nbytes, device, "PeerAllReduce")

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


class PeerAllReduceAddNorm(_PeerBuffers):
    """The all-reduce of a row-parallel projection fused into its consumer
    (gdn_allreduce_add_rmsnorm): ``self(x, h, weight, eps)`` sums this rank's partial ``h``
    [rows, dim] over the ranks, adds it to the residual ``x`` in place and returns RMSNorm(x), one
    kernel with one NVLink round trip per token row; bit for bit PeerAllReduce, then x + h, then
    ops.rmsnorm.  Collective like PeerAllReduce (same calls, same shapes on every rank; a rank that
    does not arrive makes the others set ``err`` to 3)."""

    def __init__(self, max_rows, dim, device, spin_limit=0):
        self.max_rows, self.dim = int(max_rows), int(dim)
        self.spin_limit = int(spin_limit)
        nbytes = _lib.load().gdn_ar_norm_buffer_bytes(dist.get_world_size(), self.max_rows, self.dim, _lib.GDN_BF16)
        super().__init__(nbytes, device, "PeerAllReduceAddNorm")

    def applies(self, h):
        return (not self.closed and h.dtype == torch.bfloat16 and h.shape[-1] == self.dim
                and h.numel() // self.dim <= self.max_rows)

    def __call__(self, x, h, weight, eps, out=None):
        dim = self.dim
        x2, h2 = x.view(-1, dim), h.reshape(-1, dim)
        if h2.stride(-1) != 1 or h2.stride(0) % 8 or h2.data_ptr() % 16:
            h2 = h2.contiguous()
        w = weight.to(x.dtype).contiguous()
        y = torch.empty(x2.shape, dtype=x.dtype, device=x.device) if out is None else out.view(-1, dim)
        _lib.check(self.lib.gdn_allreduce_add_rmsnorm(x2.data_ptr(), x2.stride(0), h2.data_ptr(), h2.stride(0),
                                                      w.data_ptr(), y.data_ptr(), y.stride(0), x2.shape[0], dim,
                                                      float(eps), self.rank, self.world, self._table, self.max_rows,
                                                      self.spin_limit, self.err.data_ptr(), _lib.GDN_BF16,
                                                      torch.cuda.current_stream().cuda_stream),
                   "gdn_allreduce_add_rmsnorm")
        return y.view(x.shape)


class PeerLinearAllReduce(_PeerBuffers):
    """A row-parallel projection and its sum over the ranks in one kernel (gdn_linear_allreduce):
    ``self(x, weight)`` = sum over ranks of x_r weight_r^T, for up to ``max_rows`` tokens and
    ``max_out`` output features (bf16).  Each rank's product is rounded to bf16, as the unfused
    GEMM output, and the ranks' partials are summed in rank order in fp32 and rounded once, so all
    ranks get identical results.  Collective like PeerAllReduce (same calls, same shapes, same
    order on every rank; a rank that does not arrive makes the others set ``err`` to 3)."""

    def __init__(self, max_rows, max_out, device, spin_limit=0):
        self.max_rows, self.max_out = int(max_rows), int(max_out)
        self.spin_limit = int(spin_limit)
        nbytes = _lib.load().gdn_linear_ar_buffer_bytes(dist.get_world_size(), self.max_rows, self.max_out,
                                                        _lib.GDN_BF16)
        super().__init__(nbytes, device, "PeerLinearAllReduce")
        self.route_linear = True   # AllReduceLinear.forward may run gdn_linear_allreduce through it

    def applies(self, x, weight):
        """Whether this projection goes through the fused kernel (depends only on shapes and dtypes,
        so every rank answers alike)."""
        k = x.shape[-1]
        return (not self.closed and x.is_cuda and x.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16
                and x.numel() // max(k, 1) <= self.max_rows and weight.shape[0] <= self.max_out
                and weight.shape[0] % 8 == 0 and k % 8 == 0 and weight.shape[1] == k)

    def __call__(self, x, weight, splits=0):
        x2, w = ops._linear_operands(x, weight)
        n, n_out, k = x2.shape[0], w.shape[0], x2.shape[1]
        y = torch.empty(n, n_out, dtype=x.dtype, device=x.device)
        _lib.check(self.lib.gdn_linear_allreduce(x2.data_ptr(), x2.stride(0), w.data_ptr(), w.stride(0), y.data_ptr(),
                                                 n_out, n, n_out, k, int(splits), self.rank, self.world, self._table,
                                                 self.max_rows, self.max_out, self.spin_limit, self.err.data_ptr(),
                                                 _lib.GDN_BF16, torch.cuda.current_stream().cuda_stream),
                   "gdn_linear_allreduce")
        return y.view(*x.shape[:-1], n_out)

    def push(self, x, weight, splits=0):
        """First half of ``self(x, weight)``: this rank's bf16 partial and its flags go to every rank
        (gdn_linear_push).  Must be followed by ``pull_add_rmsnorm`` of the same shape."""
        x2, w = ops._linear_operands(x, weight)
        n, n_out, k = x2.shape[0], w.shape[0], x2.shape[1]
        _lib.check(self.lib.gdn_linear_push(x2.data_ptr(), x2.stride(0), w.data_ptr(), w.stride(0), n, n_out, k,
                                            int(splits), self.rank, self.world, self._table, self.max_rows,
                                            self.max_out, self.err.data_ptr(), _lib.GDN_BF16,
                                            torch.cuda.current_stream().cuda_stream), "gdn_linear_push")

    def push_partial(self, y):
        """First half for a product computed elsewhere: this rank's partial y [rows, n_out] bf16 goes to
        every rank (gdn_push_partial).  Must be followed by ``pull_add_rmsnorm`` of the same shape."""
        y2 = y.reshape(-1, y.shape[-1])
        if y2.stride(-1) != 1 or y2.stride(0) % 8 or y2.data_ptr() % 16:
            y2 = y2.contiguous()
        _lib.check(self.lib.gdn_push_partial(y2.data_ptr(), y2.stride(0), y2.shape[0], y2.shape[1], self.rank,
                                             self.world, self._table, self.max_rows, self.max_out, _lib.GDN_BF16,
                                             torch.cuda.current_stream().cuda_stream), "gdn_push_partial")

    def pull_add_rmsnorm(self, x, weight, eps, out=None):
        """Second half: h = the sum over ranks of the pushed partials; x <- bf16(x + h) IN PLACE;
        returns rmsnorm(x) (gdn_pull_add_rmsnorm).  x: [rows, dim] contiguous bf16, dim = the pushed
        n_out."""
        dim = x.shape[-1]
        x2 = x.view(-1, dim)
        w = weight.to(x.dtype).contiguous()
        y = torch.empty(x2.shape, dtype=x.dtype, device=x.device) if out is None else out.view(-1, dim)
        _lib.check(self.lib.gdn_pull_add_rmsnorm(x2.data_ptr(), x2.stride(0), w.data_ptr(), y.data_ptr(), y.stride(0),
                                                 x2.shape[0], dim, float(eps), self.rank, self.world, self._table,
                                                 self.max_rows, self.max_out, self.spin_limit, self.err.data_ptr(),
                                                 _lib.GDN_BF16, torch.cuda.current_stream().cuda_stream),
                   "gdn_pull_add_rmsnorm")
        return y.view(x.shape)


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


_PEER_LINEAR = None


def enable_peer_linear(max_rows, max_out, device, spin_limit=0):
    """Collective: run AllReduceLinear's projections of up to ``max_rows`` tokens and ``max_out``
    outputs as one fused kernel (PeerLinearAllReduce, returned)."""
    global _PEER_LINEAR
    disable_peer_linear()
    _PEER_LINEAR = PeerLinearAllReduce(max_rows, max_out, device, spin_limit)
    return _PEER_LINEAR


def disable_peer_linear():
    """Collective: close the PeerLinearAllReduce in use, if any."""
    global _PEER_LINEAR
    if _PEER_LINEAR is not None:
        _PEER_LINEAR.close()
        _PEER_LINEAR = None


class AllReduceLinear(nn.Module):
    """A row-parallel projection: this rank holds a block of the input columns, so its product is
    a partial sum; the full output is the sum of the partials over all ranks (the same on every
    rank afterwards).  Decode-sized inputs go through the fused projection + peer sum kernel when
    one is enabled (else the peer-memory all-reduce after a cuBLAS GEMM, when enabled), everything
    else through F.linear + NCCL (src/cb_tp.py:25-35 is the reference's version)."""

    def __init__(self, lin):
        super().__init__()
        self.lin = lin

    def forward(self, x):
        fused = _PEER_LINEAR
        if fused is not None and fused.route_linear and self.lin.bias is None and fused.applies(x, self.lin.weight):
            return fused(x, self.lin.weight)
        return self.reduce(self.lin(x))

    @staticmethod
    def reduce(partial):
        """Sum this rank's partial over the ranks in place (peer-memory kernel when one is enabled
        and the size fits, else NCCL); returns it."""
        reducer = _PEER_AR
        if reducer is None or not reducer.applies(partial):
            dist.all_reduce(partial)
        else:
            reducer(partial)
        return partial


class VocabParallelHead(nn.Module):
    """The LM head split by vocabulary: this rank keeps rows [v0, v0 + V/tp) of the full weight
    and returns their logits.  ``greedy`` gives the full-vocabulary argmax with one all-reduce of
    8 bytes per row: each rank packs (its best logit, its best global id) into an int64 whose
    signed order is (logit ascending, id descending), and the MAX over ranks is the winner, the
    lowest id among equal logits, as torch.argmax over the full row picks.  Not in the reference
    (its TP engine keeps the whole head on every rank, src/cb_tp.py:117-285)."""

    def __init__(self, lin, v0):
        super().__init__()
        self.lin = lin
        self.v0 = int(v0)

    def forward(self, x):
        return self.lin(x)

    def greedy(self, x):
        logits = self.lin(x).float()
        best, arg = logits.max(dim=-1)
        bits = best.contiguous().view(torch.int32).to(torch.int64)
        # IEEE order as a signed integer: negative floats have their magnitude bits flipped
        key = torch.where(bits < 0, bits ^ 0x7FFFFFFF, bits)
        gid = arg.to(torch.int64) + self.v0
        packed = (key << 32) | (0xFFFFFFFF - gid)
        dist.all_reduce(packed, op=dist.ReduceOp.MAX)
        return 0xFFFFFFFF - (packed & 0xFFFFFFFF)


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


def _span(first, count, width, base=0):
    """Indices of ``count`` consecutive blocks of ``width`` starting at block ``first``."""
    return torch.arange(base + first * width, base + (first + count) * width)


class ShardPlan:
    """Which output rows / input columns of each weight one rank keeps, as index tensors.

    The layouts are fixed by the checkpoint: q_proj holds, per attention head, its query rows
    followed by its gate rows; in_proj_qkv and the GDN conv hold the channels [q | k | v] with q
    and k by k-head and v by v-head; in_proj_z and out_proj hold v-head blocks of dv; in_proj_a /
    in_proj_b / A_log / dt_bias one entry per v-head; the MLP one entry per hidden unit.  A rank
    takes one contiguous block of heads (or units) of each kind."""

    def __init__(self, cfg, rank, tp):
        hd = cfg.head_dim
        nh, kvh = cfg.num_attention_heads, cfg.num_key_value_heads
        self.q0, self.nq, self.kv0, self.nkv = attention_head_split(nh, kvh, tp, rank)
        kh, vh = cfg.linear_num_key_heads, cfg.linear_num_value_heads
        dk, dv = cfg.linear_key_head_dim, cfg.linear_value_head_dim
        if kh % tp or vh % tp:
            raise ValueError(f"GDN heads ({kh} k, {vh} v) do not split over tp={tp}")
        self.nkh, self.nvh = kh // tp, vh // tp
        ffn = cfg.intermediate_size
        if ffn % tp:
            raise ValueError(f"MLP width {ffn} does not split over tp={tp}")
        k_first, v_first = rank * self.nkh, rank * self.nvh
        self.index = {
            "attn_qg": _span(self.q0, self.nq, 2 * hd),
            "attn_kv": _span(self.kv0, self.nkv, hd),
            "attn_o": _span(self.q0, self.nq, hd),
            "gdn_qkv": torch.cat([_span(k_first, self.nkh, dk), _span(k_first, self.nkh, dk, kh * dk),
                                  _span(v_first, self.nvh, dv, 2 * kh * dk)]),
            "gdn_v": _span(v_first, self.nvh, dv),
            "gdn_heads": _span(v_first, self.nvh, 1),
            "ffn": _span(rank, 1, ffn // tp),
        }


# (layer type or "*", path inside the decoder layer, axis kept, plan index, row-parallel).  Axis 0
# keeps output rows (the module's input stays whole); axis 1 keeps input columns, which makes the
# product a partial sum that AllReduceLinear completes.
_CUTS = (
    ("full_attention", "self_attn.q_proj", 0, "attn_qg", False),
    ("full_attention", "self_attn.k_proj", 0, "attn_kv", False),
    ("full_attention", "self_attn.v_proj", 0, "attn_kv", False),
    ("full_attention", "self_attn.o_proj", 1, "attn_o", True),
    ("linear_attention", "linear_attn.in_proj_qkv", 0, "gdn_qkv", False),
    ("linear_attention", "linear_attn.conv1d", 0, "gdn_qkv", False),
    ("linear_attention", "linear_attn.in_proj_z", 0, "gdn_v", False),
    ("linear_attention", "linear_attn.in_proj_b", 0, "gdn_heads", False),
    ("linear_attention", "linear_attn.in_proj_a", 0, "gdn_heads", False),
    ("linear_attention", "linear_attn.A_log", 0, "gdn_heads", False),
    ("linear_attention", "linear_attn.dt_bias", 0, "gdn_heads", False),
    ("linear_attention", "linear_attn.out_proj", 1, "gdn_v", True),
    ("*", "mlp.gate_proj", 0, "ffn", False),
    ("*", "mlp.up_proj", 0, "ffn", False),
    ("*", "mlp.down_proj", 1, "ffn", True),
)


def _keep(t, axis, idx):
    return nn.Parameter(t.detach().index_select(axis, idx.to(t.device)).contiguous(), requires_grad=False)


def _cut(layer, path, axis, idx, row_parallel):
    parent_path, _, name = path.rpartition(".")
    parent = layer.get_submodule(parent_path)
    obj = getattr(parent, name)
    if isinstance(obj, nn.Parameter):            # a per-head vector
        setattr(parent, name, _keep(obj, axis, idx))
        return
    obj.weight = _keep(obj.weight, axis, idx)
    if obj.bias is not None and axis == 0:       # a row-parallel bias would be summed tp times
        obj.bias = _keep(obj.bias, 0, idx)
    elif obj.bias is not None:
        raise ValueError(f"{path}: a bias on a row-parallel projection is not supported")
    n = idx.numel()
    if isinstance(obj, nn.Linear):
        if axis == 0:
            obj.out_features = n
        else:
            obj.in_features = n
    elif isinstance(obj, nn.Conv1d):             # depthwise: channels and groups follow the rows
        obj.in_channels = obj.out_channels = obj.groups = n
    if row_parallel:
        setattr(parent, name, AllReduceLinear(obj))


def shard_model(model, rank, tp, vocab_parallel=False):
    """Shard a freshly built Qwen3_5ForConditionalGeneration in place for ``rank`` of ``tp`` (the
    layout of src/cb_tp.py:47-106, with KV heads replicated when tp > kv heads).  With
    ``vocab_parallel`` the LM head keeps V / tp rows per rank (VocabParallelHead)."""
    cfg = model.config.text_config
    if not 0 <= rank < tp:
        raise ValueError(f"rank {rank} outside tp={tp}")
    if getattr(cfg, "attention_bias", False):
        raise ValueError("attention_bias is not supported under TP")
    plan = ShardPlan(cfg, rank, tp)
    lm = model.model.language_model
    for kind, layer in zip(cfg.layer_types, lm.layers):
        for want, path, axis, key, row_parallel in _CUTS:
            if want in ("*", kind):
                _cut(layer, path, axis, plan.index[key], row_parallel)
        if kind == "full_attention":
            layer.self_attn.num_key_value_groups = plan.nq // plan.nkv
        else:
            gd = layer.linear_attn
            gd.num_k_heads, gd.num_v_heads = plan.nkh, plan.nvh
            gd.key_dim, gd.value_dim = plan.nkh * gd.head_k_dim, plan.nvh * gd.head_v_dim
            gd.conv_dim = 2 * gd.key_dim + gd.value_dim
    if vocab_parallel and tp > 1:
        V = model.lm_head.weight.shape[0]
        if V % tp:
            raise ValueError(f"vocabulary {V} does not split over tp={tp}")
        rows = _span(rank, 1, V // tp)
        head = model.lm_head
        head.weight = _keep(head.weight, 0, rows)
        head.out_features = V // tp
        model.lm_head = VocabParallelHead(head, rank * (V // tp))
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
    """CBEngine on sharded weights (src/cb_tp.py:117-285).  ``decode_sum`` picks how a decode step's
    row-parallel projections (o_proj, out_proj, down_proj) are summed over the ranks:
      * "arnorm" (default): cuBLAS GEMM, then one kernel per token row that sums the partials over
        the ranks, adds the residual and applies the next RMSNorm (gdn_allreduce_add_rmsnorm);
      * "push": cuBLAS GEMM, its partial pushed to every rank (gdn_push_partial), and the
        following residual add + RMSNorm summing the ranks (gdn_pull_add_rmsnorm);
      * "fused": the same with the projection itself on this library's tensor cores sending its
        tiles as they finish (gdn_linear_push);
      * "peer": cuBLAS GEMM, peer-memory all-reduce (gdn_allreduce), gdn_add_rmsnorm;
      * "nccl": F.linear + NCCL all-reduce (the reference's AllReduceLinear).
    Prefill's larger sums go through F.linear + NCCL.  Decode graphs capture whichever runs, and
    every rank captures the same sequence of graphs.  ``close()`` (collective) releases the graphs
    and the peer buffers.  (``peer_allreduce=False`` / ``fused_linear=True`` are the older switches
    for "nccl" / "fused".)"""

    def __init__(self, model, n_slots, t_max, device, tp, graph_decode=False, decode_sum="arnorm",
                 peer_allreduce=None, fused_linear=None):
        if fused_linear:
            decode_sum = "fused"
        elif peer_allreduce is False:
            decode_sum = "nccl"
        if decode_sum not in ("arnorm", "push", "fused", "peer", "nccl"):
            raise ValueError(f"decode_sum {decode_sum!r}")
        self.decode_sum = decode_sum
        self.peer_ar = self.peer_linear = self.peer_norm = None
        if tp > 1:
            hidden = model.config.text_config.hidden_size
            if decode_sum != "nccl":
                self.peer_ar = enable_peer_allreduce(n_slots * hidden, device)
            if decode_sum == "arnorm":
                self.peer_norm = PeerAllReduceAddNorm(n_slots, hidden, device)
            if decode_sum in ("push", "fused"):
                self.peer_linear = enable_peer_linear(n_slots, hidden, device)
                # outside the decode step's projection + norm pairs, AllReduceLinear runs the fused
                # projection + sum only in "fused" mode
                self.peer_linear.route_linear = decode_sum == "fused"
        super().__init__(model, n_slots, t_max, device, graph_decode=graph_decode, tp=tp)

    def check_errors(self):
        """Raise if a kernel of the engine reported an error or a peer exchange timed out (a rank
        did not arrive)."""
        super().check_errors()
        for what, inst in (("peer all-reduce", self.peer_ar), ("fused projection + all-reduce", self.peer_linear),
                           ("all-reduce + add + RMSNorm", self.peer_norm)):
            if inst is not None and int(inst.err.item()) != 0:
                raise RuntimeError(f"{what} error {int(inst.err.item())} (a rank did not arrive)")

    def close(self):
        """Collective: release the decode graphs and the peer buffers."""
        self._graphs.clear()
        self._graph_out.clear()
        if self.peer_norm is not None:
            self.peer_norm.close()
            self.peer_norm = None
        if self.peer_linear is not None:
            torch.cuda.synchronize()
            if _PEER_LINEAR is self.peer_linear:
                disable_peer_linear()
            else:
                self.peer_linear.close()
            self.peer_linear = None
        if self.peer_ar is not None:
            torch.cuda.synchronize()
            if _PEER_AR is self.peer_ar:
                disable_peer_allreduce()
            else:
                self.peer_ar.close()
            self.peer_ar = None
