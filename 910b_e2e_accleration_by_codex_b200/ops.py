"""Torch-facing GDN operators backed by the CUDA library (C ABI in include/gdn_b200.h).

Two groups of functions:

* Drop-ins with the reference's signatures, for installation on HF modules by
  ``patch.patch_model`` exactly where the reference installs its own:
    - ``chunk_gated_delta_rule``      (src/gdn_chunk_fast2.py:11-12, transformers :234-244)
    - ``recurrent_gated_delta_rule``  (src/recurrent_single_step.py:8-9, transformers :314-316)
    - ``causal_conv1d_update``        (transformers :210-216)
    - ``elem_conv_update``            (src/cb_engine.py:43)
    - ``gated_rmsnorm`` / ``rmsnorm_gated_forward`` (transformers :181, src/cb_engine.py:65)
  They allocate their outputs like the reference functions do.
* Slot-indexed operators used by the engine (``engine.CBEngine``): state pools are read
  and written in place through a slot index inside the kernels, and nothing is
  allocated, so the calls can be captured in CUDA graphs.

Every call runs on ``torch.cuda.current_stream()``.  Failures raise RuntimeError with
the library's message.  There is no CPU path: CPU tensors raise.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib
from ._lib import GDN_BF16, GDN_CONV_ELEM, GDN_CONV_HF, GDN_F32

_DT = {torch.bfloat16: GDN_BF16, torch.float32: GDN_F32}


def _dtype_code(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError(f"GDN kernels take bfloat16 or float32 activations, got {t.dtype}") from None


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("GDN operators run on CUDA tensors only (no CPU fallback)")


def _p(t):
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _rows(t: torch.Tensor, d: int) -> torch.Tensor:
    """View as [..., d] with unit stride in the last dim and heads packed (stride d)."""
    if t.stride(-1) != 1 or (t.dim() >= 2 and t.shape[-2] > 1 and t.stride(-2) != d):
        t = t.contiguous()
    return t


def _i32(t):
    if t is None:
        return None
    if t.dtype != torch.int32 or not t.is_contiguous():
        t = t.to(torch.int32).contiguous()
    return t


# ============================================================================ a4: gated RMSNorm
def gated_rmsnorm(x: torch.Tensor, gate: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """Qwen3_5RMSNormGated.forward (transformers modeling_qwen3_5.py:181-191):
    y = weight * rnd(x * rsqrt(mean(x^2) + eps)) * silu(gate), in x's dtype."""
    _need_cuda(x, gate, weight)
    dim = x.shape[-1]
    x2 = x.reshape(-1, dim)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    g2 = gate.to(x.dtype).reshape(-1, dim)
    if g2.stride(-1) != 1:
        g2 = g2.contiguous()
    w = weight.to(x.dtype).contiguous()
    y = torch.empty_like(x2) if out is None else out.view(-1, dim)
    lib = _lib.load()
    _lib.check(lib.gdn_gated_rmsnorm(_p(x2), x2.stride(0), _p(g2), g2.stride(0), _p(w), _p(y), y.stride(0),
                                     x2.shape[0], dim, float(eps), _dtype_code(x), _stream()),
               "gdn_gated_rmsnorm")
    return y.view(x.shape)


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6, out: torch.Tensor | None = None) -> torch.Tensor:
    """Qwen3_5RMSNorm.forward (transformers modeling_qwen3_5.py): x * rsqrt(mean(x^2) + eps) * (1 + weight)
    in fp32, rounded once to x's dtype -- the layer norm the reference replaces with npu_rms_norm
    (src/cb_engine.py:62-63)."""
    _need_cuda(x, weight)
    dim = x.shape[-1]
    x2 = x.reshape(-1, dim)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    w = weight.to(x.dtype).contiguous()
    y = torch.empty(x2.shape, dtype=x.dtype, device=x.device) if out is None else out.view(-1, dim)
    lib = _lib.load()
    _lib.check(lib.gdn_rmsnorm(_p(x2), x2.stride(0), _p(w), _p(y), y.stride(0), x2.shape[0], dim, float(eps),
                               _dtype_code(x), _stream()), "gdn_rmsnorm")
    return y.view(x.shape)


def attn_decode_workspace(n, Hq, hd, max_len, device):
    """Workspace for ``attn_decode`` (split partials; no zero-fill needed)."""
    nb = int(_lib.load().gdn_attn_decode_workspace_size(n, Hq, hd, max_len))
    return torch.empty(max(nb, 16), dtype=torch.uint8, device=device)


def attn_decode_prep(y, q_norm_w, k_norm_w, eps, cos, sin, Hq, kvh, hd):
    """The attention decode preamble (gdn_attn_decode_prep): from the fused q|gate, k, v projection
    y [n, >= 2 Hq hd + 2 kvh hd] returns (q, k, v, gate) = (rotary(q_norm(q)), rotary(k_norm(k)), v,
    gate) as contiguous [n, heads, hd] tensors, bit for bit HF's q_norm / k_norm and
    apply_rotary_pos_emb (cos / sin [n, ..., rd]) in bf16 (src/cb_engine.py:295-316)."""
    _need_cuda(y, q_norm_w, k_norm_w, cos, sin)
    n = y.shape[0]
    y2 = y.reshape(n, -1)
    if y2.stride(-1) != 1 or y2.stride(0) % 8 or y2.data_ptr() % 16:
        y2 = y2.contiguous()
    rd = cos.shape[-1]
    c2, s2 = cos.reshape(n, rd).contiguous(), sin.reshape(n, rd).contiguous()
    q = torch.empty(n, Hq, hd, dtype=y.dtype, device=y.device)
    g = torch.empty(n, Hq, hd, dtype=y.dtype, device=y.device)
    k = torch.empty(n, kvh, hd, dtype=y.dtype, device=y.device)
    v = torch.empty(n, kvh, hd, dtype=y.dtype, device=y.device)
    _lib.check(_lib.load().gdn_attn_decode_prep(_p(y2), y2.stride(0), _p(q_norm_w.contiguous()),
                                                _p(k_norm_w.contiguous()), float(eps), _p(c2), _p(s2), c2.stride(0),
                                                int(rd), _p(q), _p(k), _p(v), _p(g), n, Hq, kvh, hd, _dtype_code(y),
                                                _stream()), "gdn_attn_decode_prep")
    return q, k, v, g


def attn_decode(q, k_new, v_new, kv_k, kv_v, slot_idx, pos, max_len, scale, gate=None, out=None, workspace=None,
                err=None):
    """Slot-indexed attention decode over the KV pool (CBEngine._attn, src/cb_engine.py:295-316): writes
    k_new/v_new [n, kvh, hd] at pos[n] of kv_k/kv_v[slot_idx] ([n_slots, kvh, T, hd]) and returns
    softmax(scale q k^T) v over positions 0..pos for q [n, Hq, hd] (kv-major head groups), times
    sigmoid(gate) [n, Hq, hd] when given, in bf16."""
    _need_cuda(q, k_new, v_new, kv_k, kv_v, slot_idx, pos)
    n, Hq, hd = q.shape[0], q.shape[-2], q.shape[-1]
    kvh, T = kv_k.shape[1], kv_k.shape[2]
    q = q.reshape(n, Hq, hd).contiguous()
    k_new = k_new.reshape(n, kvh, hd).contiguous()
    v_new = v_new.reshape(n, kvh, hd).contiguous()
    g = None if gate is None else gate.reshape(n, Hq, hd).contiguous()
    ws = attn_decode_workspace(n, Hq, hd, max_len, q.device) if workspace is None else workspace
    o = torch.empty(n, Hq, hd, dtype=q.dtype, device=q.device) if out is None else out
    lib = _lib.load()
    _lib.check(lib.gdn_attn_decode(_p(q), _p(k_new), _p(v_new), _p(kv_k), _p(kv_v), kv_k.shape[0], T,
                                   _p(_i32(slot_idx)), _p(_i32(pos)), int(max_len), _p(g), float(scale), _p(o), n,
                                   Hq, kvh, hd, _p(ws), ws.numel(), _dtype_code(q), _p(err), _stream()),
               "gdn_attn_decode")
    return o


def rmsnorm_forward(self, x):
    """Bound in place of Qwen3_5RMSNorm.forward, where the reference binds npu_rms_norm
    (src/cb_engine.py:62-63, 70-71)."""
    return rmsnorm(x, self.weight, self.eps)


def rmsnorm_gated_forward(self, hidden_states, gate=None):
    """Bound in place of Qwen3_5RMSNormGated.forward (src/cb_engine.py:65-67, 72-73)."""
    return gated_rmsnorm(hidden_states, gate, self.weight, self.variance_epsilon)


# ============================================================================ a3: decode conv
def _conv_update(x, state, weight, bias, mode, slot_idx=None, out=None, err=None):
    _need_cuda(x, state, weight, bias)
    if x.dim() == 2:
        x = x.unsqueeze(-1)
    B, Cc, T = x.shape
    K = state.shape[-1]
    if weight.dim() == 3:
        weight = weight.squeeze(1)
    if weight.shape != (Cc, K):
        raise ValueError(f"conv weight {tuple(weight.shape)} != ({Cc}, {K})")
    wd = weight.dtype
    if x.dtype != wd:
        x = x.to(wd)
    # the kernel updates a contiguous [slots, C, K] pool in place; other layouts (HF's cache may
    # hold a strided view) go through a contiguous copy that is written back
    st = state if (state.dtype == wd and state.is_contiguous()) else state.to(wd).contiguous()
    w = weight.contiguous()
    b = None if bias is None else bias.to(wd).contiguous()
    y = torch.empty(B, Cc, T, dtype=wd, device=x.device) if out is None else out
    n_slots = st.shape[0]
    lib = _lib.load()
    _lib.check(lib.gdn_conv_update(_p(x), x.stride(0), x.stride(1), x.stride(2), _p(st), _p(_i32(slot_idx)),
                                   n_slots, _p(w), _p(b), _p(y), y.stride(0), y.stride(1), y.stride(2), B, Cc, T,
                                   K, 1, mode, _dtype_code(w), _p(err), _stream()), "gdn_conv_update")
    if st is not state:
        state.copy_(st)
    return y


def causal_conv1d_update(hidden_states, conv_state, weight, bias=None, activation=None):
    """torch_causal_conv1d_update (transformers modeling_qwen3_5.py:210-226): conv_state [B,C,K]
    updated in place; returns silu(conv) [B,C,T] in hidden_states' dtype (the HF fallback applies
    silu whatever `activation` says)."""
    y = _conv_update(hidden_states, conv_state, weight, bias, GDN_CONV_HF)
    return y.to(hidden_states.dtype)


def elem_conv_update(x, state, weight, bias):
    """elem_conv_update (src/cb_engine.py:43-51): x [n,C,1], state [n,C,K] updated in place;
    products and sum rounded in the weight dtype as the reference's mul + sum does."""
    y = _conv_update(x, state, weight, bias, GDN_CONV_ELEM)
    return y.to(x.dtype)


# ============================================================================ a2: recurrence
def recurrent_gated_delta_rule(query, key, value, g, beta, initial_state, output_final_state,
                               use_qk_l2norm_in_kernel=False):
    """recurrent_single_step / torch_recurrent_gated_delta_rule (src/recurrent_single_step.py:8-32,
    transformers modeling_qwen3_5.py:314-353).  query/key [B,T,Hq,dk] (Hq divides Hv; HF passes
    them repeated to Hv heads), value [B,T,Hv,dv], g/beta [B,T,Hv].  Returns (out [B,T,Hv,dv] in
    query's dtype, new fp32 state [B,Hv,dk,dv] or None)."""
    _need_cuda(query, key, value, g, beta, initial_state)
    dt = query.dtype
    B, T, Hq, dk = query.shape
    Hv, dv = value.shape[2], value.shape[3]
    q = _rows(query, dk)
    k = _rows(key.to(dt), dk)
    v = _rows(value.to(dt), dv)
    gg = g.to(torch.float32).contiguous()
    bb = beta.to(torch.float32).contiguous()
    init = None if initial_state is None else initial_state.to(torch.float32).contiguous()
    final = torch.empty(B, Hv, dk, dv, dtype=torch.float32, device=query.device) if output_final_state else None
    out = torch.empty(B, T, Hv, dv, dtype=dt, device=query.device)
    lib = _lib.load()
    _lib.check(lib.gdn_recurrent(_p(q), q.stride(0), q.stride(1), _p(k), k.stride(0), k.stride(1), _p(v),
                                 v.stride(0), v.stride(1), _p(gg), _p(bb), T * Hv, Hv, _p(init), None,
                                 _p(final), None, B, _p(out), T * Hv * dv, Hv * dv, B, T, Hq, Hv, dk, dv,
                                 int(bool(use_qk_l2norm_in_kernel)), _dtype_code(q), None, _stream()),
               "gdn_recurrent")
    return out, final


def recurrent_step_slots(q, k, v, g, beta, state_pool, slot_idx, use_qk_l2norm=True, out=None, err=None):
    """One decode token per sequence with the state gathered from and scattered back to
    ``state_pool[slot_idx]`` inside the kernel (replaces src/cb_engine.py:344-347).
    q,k [n,Hk,dk], v [n,Hv,dv], g/beta [n,Hv] fp32, state_pool [S,Hv,dk,dv] fp32."""
    _need_cuda(q, k, v, g, beta, state_pool, slot_idx)
    n, Hk, dk = q.shape
    Hv, dv = v.shape[1], v.shape[2]
    q, k, v = _rows(q, dk), _rows(k, dk), _rows(v, dv)
    g = g.to(torch.float32)
    beta = beta.to(torch.float32)
    if g.stride(-1) != 1 or beta.stride(-1) != 1 or g.stride(0) != beta.stride(0):
        g, beta = g.contiguous(), beta.contiguous()
    o = torch.empty(n, Hv, dv, dtype=q.dtype, device=q.device) if out is None else out
    si = _i32(slot_idx)
    lib = _lib.load()
    _lib.check(lib.gdn_recurrent(_p(q), q.stride(0), 0, _p(k), k.stride(0), 0, _p(v), v.stride(0), 0, _p(g),
                                 _p(beta), g.stride(0), 0, _p(state_pool), _p(si), _p(state_pool), _p(si),
                                 state_pool.shape[0], _p(o), o.stride(0), 0, n, 1, Hk, Hv, dk, dv,
                                 int(bool(use_qk_l2norm)), _dtype_code(q), _p(err), _stream()),
               "gdn_recurrent")
    return o


# ============================================================================ a1: chunk prefill
def chunk_gated_delta_rule(query, key, value, g, beta, chunk_size=64, initial_state=None,
                           output_final_state=False, use_qk_l2norm_in_kernel=False):
    """fast_chunk_gated_delta_rule_v2 (src/gdn_chunk_fast2.py:11-62) / torch_chunk_gated_delta_rule
    (transformers modeling_qwen3_5.py:234-311).  [B,L,H,D] inputs of equal length L; returns
    (out [B,L,Hv,dv] in query's dtype, final fp32 state [B,Hv,dk,dv] or None).  The kernels use
    64-token chunks whatever ``chunk_size`` says (the chunked form is exact algebra; chunk size
    only changes fp32 rounding)."""
    _need_cuda(query, key, value, g, beta, initial_state)
    if chunk_size <= 0:
        raise ValueError(f"chunk_size must be positive, got {chunk_size}")
    dt = query.dtype
    B, L, Hq, dk = query.shape
    Hv, dv = value.shape[2], value.shape[3]
    out = torch.empty(B, L, Hv, dv, dtype=dt, device=query.device)
    final = torch.empty(B, Hv, dk, dv, dtype=torch.float32, device=query.device) if output_final_state else None
    init = None if initial_state is None else initial_state.to(torch.float32).contiguous()
    if B == 0 or L == 0:
        if final is not None:
            final.copy_(init if init is not None else torch.zeros_like(final))
        return out, final
    q = query.contiguous()
    k = key.to(dt).contiguous()
    v = value.to(dt).contiguous()
    gg = g.to(torch.float32).contiguous()
    bb = beta.to(torch.float32).contiguous()
    cu = torch.arange(0, B + 1, dtype=torch.int32, device=query.device) * L
    lib = _lib.load()
    _lib.check(lib.gdn_chunk_prefill(_p(q), Hq * dk, _p(k), Hq * dk, _p(v), Hv * dv, _p(gg), _p(bb), Hv, _p(cu),
                                     B, B * L, _p(init), None, None, _p(final), None, B, _p(out), Hv * dv, Hq,
                                     Hv, dk, dv, int(bool(use_qk_l2norm_in_kernel)), _dtype_code(q), None,
                                     _stream()), "gdn_chunk_prefill")
    return out, final


def chunk_prefill_varlen(q, k, v, g, beta, cu_seqlens, state_pool=None, slot_idx=None, use_initial=None,
                         use_qk_l2norm=True, out=None, err=None):
    """Packed varlen chunk prefill.  q,k [T,Hk,dk], v [T,Hv,dv] (token strides may be wider than
    the head block, e.g. column slices of the conv output), g/beta [T,Hv] fp32, cu_seqlens
    int32 [B+1] (device).  Sequence b starts from state_pool[slot_idx[b]] where use_initial[b]
    (else zeros) and its final state is written to state_pool[slot_idx[b]]."""
    _need_cuda(q, k, v, g, beta, cu_seqlens, state_pool)
    T, Hk, dk = q.shape
    Hv, dv = v.shape[1], v.shape[2]
    for t, d in ((q, dk), (k, dk), (v, dv)):
        if t.stride(-1) != 1 or t.stride(-2) != d:
            raise ValueError("q/k/v must have packed heads and unit stride in the last dim")
    g = g.to(torch.float32)
    beta = beta.to(torch.float32)
    if g.stride(-1) != 1 or beta.stride(-1) != 1 or g.stride(0) != beta.stride(0):
        g, beta = g.contiguous(), beta.contiguous()
    o = torch.empty(T, Hv, dv, dtype=q.dtype, device=q.device) if out is None else out
    B = cu_seqlens.numel() - 1
    si = _i32(slot_idx)
    ui = _i32(use_initial)
    # no use_initial: every sequence starts from zeros (the C ABI reads the pool only when given it)
    init_pool = None if use_initial is None else state_pool
    lib = _lib.load()
    _lib.check(lib.gdn_chunk_prefill(_p(q), q.stride(0), _p(k), k.stride(0), _p(v), v.stride(0), _p(g), _p(beta),
                                     g.stride(0), _p(_i32(cu_seqlens)), B, T, _p(init_pool), _p(si), _p(ui),
                                     _p(state_pool), _p(si), 0 if state_pool is None else state_pool.shape[0],
                                     _p(o), o.stride(0), Hk, Hv, dk, dv, int(bool(use_qk_l2norm)),
                                     _dtype_code(q), _p(err), _stream()), "gdn_chunk_prefill")
    return o


def chunk_prefill_varlen_gates(q, k, v, a, b, A_log, dt_bias, cu_seqlens, state_pool=None, slot_idx=None,
                               use_initial=None, use_qk_l2norm=True, out=None, err=None):
    """``chunk_prefill_varlen`` with the prefill's gate lines (src/cb_tp.py:170-171, transformers
    :491-493) done inside the kernel: a, b are the in_proj_a / in_proj_b outputs [T,Hv] in the
    activations' dtype, A_log / dt_bias [Hv]; beta = sigmoid(b) in that dtype and
    g = -exp(A_log) * softplus(float(a) + dt_bias) in fp32, bit-identical to those torch lines."""
    _need_cuda(q, k, v, a, b, A_log, dt_bias, cu_seqlens, state_pool)
    T, Hk, dk = q.shape
    Hv, dv = v.shape[1], v.shape[2]
    for t, d in ((q, dk), (k, dk), (v, dv)):
        if t.stride(-1) != 1 or t.stride(-2) != d:
            raise ValueError("q/k/v must have packed heads and unit stride in the last dim")
    if a.shape != (T, Hv) or b.shape != (T, Hv):
        raise ValueError(f"a/b must be [T, Hv] = [{T}, {Hv}], got {tuple(a.shape)} / {tuple(b.shape)}")
    a = a.to(q.dtype)
    b = b.to(q.dtype)
    if a.stride(-1) != 1 or b.stride(-1) != 1 or a.stride(0) != b.stride(0):
        a, b = a.contiguous(), b.contiguous()
    A_log = A_log.to(torch.float32).contiguous()
    dt_bias = dt_bias.to(torch.float32).contiguous()
    o = torch.empty(T, Hv, dv, dtype=q.dtype, device=q.device) if out is None else out
    B = cu_seqlens.numel() - 1
    si = _i32(slot_idx)
    ui = _i32(use_initial)
    init_pool = None if use_initial is None else state_pool
    lib = _lib.load()
    _lib.check(lib.gdn_chunk_prefill_gates(_p(q), q.stride(0), _p(k), k.stride(0), _p(v), v.stride(0), _p(a), _p(b),
                                           a.stride(0), _p(A_log), _p(dt_bias), _p(_i32(cu_seqlens)), B, T,
                                           _p(init_pool), _p(si), _p(ui), _p(state_pool), _p(si),
                                           0 if state_pool is None else state_pool.shape[0], _p(o), o.stride(0),
                                           Hk, Hv, dk, dv, int(bool(use_qk_l2norm)), _dtype_code(q), _p(err),
                                           _stream()), "gdn_chunk_prefill_gates")
    return o


# ============================================================================ prefill conv
def prefill_conv_varlen(x, cu_seqlens, weight, bias=None, conv_pool=None, slot_idx=None, use_initial=None,
                        out=None, err=None):
    """Varlen causal conv1d + silu over packed tokens x [T,C] (transformers :463-474,
    src/cb_tp.py:158-164 and :236-244); conv state carried from / written to conv_pool[slot_idx]."""
    _need_cuda(x, cu_seqlens, weight, bias, conv_pool)
    T, Cc = x.shape
    if x.stride(1) != 1:
        x = x.contiguous()
    if weight.dim() == 3:
        weight = weight.squeeze(1)
    K = weight.shape[-1]
    w = weight.to(x.dtype).contiguous()
    b = None if bias is None else bias.to(x.dtype).contiguous()
    y = torch.empty_like(x) if out is None else out
    B = cu_seqlens.numel() - 1
    lib = _lib.load()
    _lib.check(lib.gdn_prefill_conv(_p(x), x.stride(0), _p(y), y.stride(0), _p(_i32(cu_seqlens)), B, _p(conv_pool),
                                    _p(_i32(slot_idx)), _p(_i32(use_initial)),
                                    0 if conv_pool is None else conv_pool.shape[0], _p(w), _p(b), Cc, K, 1,
                                    _dtype_code(x), _p(err), _stream()), "gdn_prefill_conv")
    return y


# ============================================================================ fused decode layer
def decode_layer_workspace_bytes(n, Hk, Hv, dk, dv, dtype) -> int:
    """Bytes of device workspace ``decode_layer`` needs: for d = 128 the prepared q/k/v rows and gates
    passed from its prep kernel to its state kernel; for d = 64 one uint32 ticket counter per slot
    entry and k-head."""
    return int(_lib.load().gdn_decode_layer_workspace_size(n, Hk, Hv, dk, dv, _DT[dtype]))


def decode_layer_workspace(n, Hk, Hv, dk, dv, dtype, device):
    """Device workspace for ``decode_layer``, zero-filled: the d = 64 form's ticket counters must
    start at zero and every call leaves them at zero; the d = 128 form overwrites its rows on every
    call.  One workspace serves any number of calls on one stream."""
    return torch.zeros(decode_layer_workspace_bytes(n, Hk, Hv, dk, dv, dtype), dtype=torch.uint8, device=device)


def decode_layer(mixed_qkv, z, a, b, A_log, dt_bias, conv_w, conv_b, conv_pool, rec_pool, slot_idx, norm_w,
                 eps, Hk, Hv, dk, dv, conv_mode=GDN_CONV_ELEM, workspace=None, out=None, err=None):
    """The operator part of CBEngine._gdn (src/cb_engine.py:318-352) for n slots: conv update
    (conv_pool[slot_idx] in place) -> gates -> l2norm -> recurrence (rec_pool[slot_idx] in place)
    -> gated RMSNorm, as a prep kernel plus a persistent state kernel (d = 128) or one kernel
    (d = 64).  ``workspace`` (see decode_layer_workspace) must be zero-filled before its first use.
    mixed_qkv [n,C], z [n,Hv,dv] (or [n,Hv*dv]), a/b [n,Hv], A_log/dt_bias [Hv] fp32.  Each of
    mixed_qkv, z, a, b may be a row-strided view, e.g. column slices of one fused projection output
    (gdn_decode_layer_rows).  Returns out [n,Hv,dv]."""
    _need_cuda(mixed_qkv, z, a, b, A_log, dt_bias, conv_w, conv_pool, rec_pool, slot_idx, norm_w)
    n, Cc = mixed_qkv.shape[0], mixed_qkv.shape[-1]
    mixed = mixed_qkv.reshape(n, Cc)
    if mixed.stride(1) != 1:
        mixed = mixed.contiguous()

    def rows(t, width):
        """A [n, width] view of t with unit inner stride, or a contiguous copy."""
        v = t.reshape(n, width) if t.is_contiguous() else (t if t.dim() == 2 else None)
        if v is None or v.stride(1) != 1:
            v = t.contiguous().reshape(n, width)
        return v

    z2, a2, b2 = rows(z, Hv * dv), rows(a, Hv), rows(b, Hv)
    esz = z2.element_size()
    if z2.data_ptr() % 16 or (z2.stride(0) * esz) % 16:  # the state kernel bulk-copies [dv] rows of z
        z2 = z2.contiguous()
        if z2.data_ptr() % 16:
            z2 = z2.clone()
    K = conv_pool.shape[-1]
    if workspace is None:
        workspace = decode_layer_workspace(n, Hk, Hv, dk, dv, mixed.dtype, mixed.device)
    o = torch.empty(n, Hv, dv, dtype=mixed.dtype, device=mixed.device) if out is None else out
    w = conv_w.squeeze(1) if conv_w.dim() == 3 else conv_w
    lib = _lib.load()
    _lib.check(lib.gdn_decode_layer_rows(_p(mixed), mixed.stride(0), _p(z2), z2.stride(0), _p(a2), a2.stride(0),
                                         _p(b2), b2.stride(0), _p(A_log), _p(dt_bias), _p(w), _p(conv_b),
                                         _p(conv_pool), _p(rec_pool), _p(_i32(slot_idx)), rec_pool.shape[0],
                                         _p(norm_w), float(eps), _p(o), n, Hk, Hv, dk, dv, K, conv_mode,
                                         _p(workspace), workspace.numel(), _dtype_code(mixed), _p(err), _stream()),
               "gdn_decode_layer_rows")
    return o


def l2_scale(dk: int) -> float:
    """The q scale the reference applies after l2norm (1/sqrt(dk))."""
    return 1.0 / math.sqrt(dk)


# ============================================================================ f1: decode projections
def _linear_operands(x, weight):
    _need_cuda(x, weight)
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise TypeError("linear: bf16 x and weight")
    k = x.shape[-1]
    x2 = x.reshape(-1, k)
    if x2.stride(-1) != 1 or x2.stride(0) % 8 or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    w = weight if weight.stride(-1) == 1 and weight.stride(0) % 8 == 0 and weight.data_ptr() % 16 == 0 \
        else weight.contiguous()
    return x2, w


def linear(x: torch.Tensor, weight: torch.Tensor, out: torch.Tensor | None = None, splits: int = 0,
           err: torch.Tensor | None = None) -> torch.Tensor:
    """F.linear(x, weight) for a bias-free projection of a decode step (src/cb_engine.py:295-355) on
    the tensor cores (gdn_linear): x [..., k] bf16 with at most 256 rows, weight [n_out, k] bf16;
    fp32 accumulation, one bf16 rounding, deterministic.  ``splits`` forces the K split (0: the
    library picks)."""
    x2, w = _linear_operands(x, weight)
    n, n_out, k = x2.shape[0], w.shape[0], x2.shape[1]
    y = torch.empty(n, n_out, dtype=x.dtype, device=x.device) if out is None else out.view(-1, n_out)
    lib = _lib.load()
    _lib.check(lib.gdn_linear(_p(x2), x2.stride(0), _p(w), w.stride(0), _p(y), y.stride(0), n, n_out, k, int(splits),
                              GDN_BF16, _p(err), _stream()), "gdn_linear")
    return y.view(*x.shape[:-1], n_out)


def linear_plan(n, n_out, k, splits=0, world=1):
    """The launch gdn_linear (world 1) / gdn_linear_allreduce (world > 1) makes for this shape:
    dict(splits, stages, smem, tiles, kblocks)."""
    out = (ctypes.c_int32 * 5)()
    _lib.check(_lib.load().gdn_linear_plan(n, n_out, k, splits, world, out), "gdn_linear_plan")
    return dict(zip(("splits", "stages", "smem", "tiles", "kblocks"), list(out)))


def add_rmsnorm(x: torch.Tensor, h: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """The residual add and the next layer norm of a decode step in one kernel (gdn_add_rmsnorm):
    x <- bf16(x + h) IN PLACE, returns rmsnorm(x) = bf16(x * rsqrt(mean(x^2) + eps) * (1 + weight)),
    bit for bit ``x = x + h; ops.rmsnorm(x, weight, eps)`` (src/cb_engine.py:295-355)."""
    _need_cuda(x, h, weight)
    dim = x.shape[-1]
    x2, h2 = x.view(-1, dim), h.reshape(-1, dim)
    if h2.stride(-1) != 1 or h2.stride(0) % 8 or h2.data_ptr() % 16:
        h2 = h2.contiguous()
    w = weight.to(x.dtype).contiguous()
    y = torch.empty(x2.shape, dtype=x.dtype, device=x.device) if out is None else out.view(-1, dim)
    _lib.check(_lib.load().gdn_add_rmsnorm(_p(x2), x2.stride(0), _p(h2), h2.stride(0), _p(w), _p(y), y.stride(0),
                                           x2.shape[0], dim, float(eps), _dtype_code(x), _stream()),
               "gdn_add_rmsnorm")
    return y.view(x.shape)


def silu_mul(y: torch.Tensor, inter: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """act_fn(gate) * up of Qwen3_5MLP on the fused gate|up projection y [..., 2*inter] (gdn_silu_mul):
    bf16(bf16(silu(y[..., :inter])) * y[..., inter:2*inter]), bit for bit the two bf16 torch ops."""
    _need_cuda(y)
    y2 = y.reshape(-1, y.shape[-1])
    if y2.stride(-1) != 1 or y2.stride(0) % 8 or y2.data_ptr() % 16:
        y2 = y2.contiguous()
    o = torch.empty(y2.shape[0], inter, dtype=y.dtype, device=y.device) if out is None else out.view(-1, inter)
    _lib.check(_lib.load().gdn_silu_mul(_p(y2), y2.stride(0), int(inter), _p(o), o.stride(0), y2.shape[0],
                                        _dtype_code(y), _stream()), "gdn_silu_mul")
    return o.view(*y.shape[:-1], inter)

