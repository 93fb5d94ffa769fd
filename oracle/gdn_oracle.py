"""CPU oracle for the GatedDeltaNet (GDN) hot path.  TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the reference's torch implementation of the
four GDN operators and the decode/prefill glue around them.  It exists so the
CUDA kernels can be checked on the same seeded inputs; nothing on the product
path may import it (the product fails loudly when its CUDA library is absent).
Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of ``bench.py``
use it.

Parity of this restatement is pinned against golden vectors produced by the
reference itself (``tests/golden/make_golden.py`` imports the reference's
``src/`` and HF transformers' Qwen3.5 module and records inputs and outputs).

Reference citations (paths inside the reference project; ``TF`` is
transformers ``models/qwen3_5/modeling_qwen3_5.py``, 5.5.x):
  * l2norm                  src/gdn_chunk_fast.py:17-18, TF:228-231
  * _small_unit_lower_inv   src/gdn_chunk_fast.py:21-30
  * _unit_lower_inv         src/gdn_chunk_fast.py:33-62
  * chunk rule (v2)         src/gdn_chunk_fast2.py:11-62
  * recurrent single step   src/recurrent_single_step.py:8-32, TF:314-353
  * elem conv update        src/cb_engine.py:43-51, TF:210-226
  * gated RMSNorm           TF:181-191
  * decode gates            src/cb_engine.py:337-342, TF:491-496
  * prefill causal conv     TF:463-474, src/cb_tp.py:158-164, :236-244, :260

Numbers are carried as float32 arrays.  Where the reference computes in
bfloat16 (``dt="bf16"``) every torch op's rounding is emulated with
``bf16()`` (round-to-nearest-even onto the bf16 grid), op by op in the same
order as the reference.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


# --------------------------------------------------------------------------- dtypes
def bf16(x):
    """Round float32 values to the nearest bfloat16 (ties to even); returns float32."""
    x = np.ascontiguousarray(x, dtype=F32)
    u = x.view(np.uint32)
    # finite values and infinities cannot carry past bit 31; NaNs are restored below
    r = ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)).view(F32)
    nan = np.isnan(x)
    return np.where(nan, F32(np.nan), r) if nan.any() else r


def rnd(x, dt):
    """Round to the arithmetic type ``dt`` ("bf16" or "f32")."""
    return bf16(x) if dt == "bf16" else np.asarray(x, dtype=F32)


def bf16_bits(x):
    """float32 array -> uint16 bf16 bit patterns (rounded)."""
    return (bf16(x).view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(u):
    """uint16 bf16 bit patterns -> float32 array (exact)."""
    return (np.asarray(u, dtype=np.uint16).astype(np.uint32) << 16).view(F32)


def silu(x):
    x = np.asarray(x, dtype=F32)
    return (x / (F32(1) + np.exp(-x))).astype(F32)


def sigmoid(x):
    x = np.asarray(x, dtype=F32)
    return (F32(1) / (F32(1) + np.exp(-x))).astype(F32)


def softplus(x):
    """torch.nn.functional.softplus (beta=1, threshold=20)."""
    x = np.asarray(x, dtype=F32)
    return np.where(x > 20, x, np.log1p(np.exp(np.minimum(x, 20)))).astype(F32)


# --------------------------------------------------------------------------- l2norm
def l2norm(x, dt="f32", eps=1e-6):
    """x * rsqrt(sum(x*x, -1) + eps) in the input dtype (src/gdn_chunk_fast.py:17-18)."""
    x = np.asarray(x, dtype=F32)
    sq = rnd(x * x, dt)
    s = rnd(sq.sum(-1, keepdims=True, dtype=F32), dt)
    s = rnd(s + F32(eps), dt)
    inv = rnd(F32(1) / np.sqrt(s), dt)
    return rnd(x * inv, dt)


# --------------------------------------------------------------------------- triangular inverse
def small_unit_lower_inv(X):
    """(I - X)^-1 for small strictly-lower X by the row recurrence
    R_i = X_i + sum_{m<i} X_im R_m  (src/gdn_chunk_fast.py:21-30)."""
    n = X.shape[-1]
    R = X.astype(F32).copy()
    for i in range(1, n):
        row = R[..., i, :i].copy()
        sub = R[..., :i, :i].copy()
        R[..., i, :i] = row + (row[..., :, None] * sub).sum(-2, dtype=F32)
    return (R + np.eye(n, dtype=F32)).astype(F32)


def unit_lower_inv(X, base=16):
    """Blocked (I - X)^-1: diagonal base x base blocks by the row recurrence, then
    pairwise merges T21 = B @ X21 @ A (src/gdn_chunk_fast.py:33-62)."""
    n = X.shape[-1]
    nb = n // base
    if nb == 1:
        return small_unit_lower_inv(X)
    diag = np.stack([X[..., i * base:(i + 1) * base, i * base:(i + 1) * base] for i in range(nb)],
                    axis=-3)
    Td = small_unit_lower_inv(diag)
    blocks = [Td[..., i, :, :] for i in range(nb)]

    def merge(lo, hi):
        if hi - lo == 1:
            return blocks[lo]
        mid = (lo + hi) // 2
        A = merge(lo, mid)
        B = merge(mid, hi)
        X21 = X[..., mid * base:hi * base, lo * base:mid * base]
        T21 = np.matmul(np.matmul(B, X21), A)
        top = np.concatenate([A, np.zeros(A.shape[:-1] + (B.shape[-1],), F32)], axis=-1)
        bot = np.concatenate([T21, B], axis=-1)
        return np.concatenate([top, bot], axis=-2).astype(F32)

    return merge(0, nb)


# --------------------------------------------------------------------------- chunk rule
def chunk_gated_delta_rule(query, key, value, g, beta, chunk_size=64, initial_state=None,
                           output_final_state=False, use_qk_l2norm_in_kernel=False, dt="f32"):
    """Chunked gated delta rule, v2 formulation (src/gdn_chunk_fast2.py:11-62).

    query/key [B,L,H,dk], value [B,L,H,dv], g/beta [B,L,H] (float32 arrays holding values
    of dtype ``dt``; g is float32 in the reference).  Returns (out [B,L,H,dv] rounded to
    ``dt``, final state [B,H,dk,dv] float32 or None).

    L = 0 is defined as the zero-chunk limit (no output rows, final state = initial state or zeros);
    the reference raises there (torch.stack of an empty chunk list, src/gdn_chunk_fast2.py:60), and
    the library's packed prefill follows this definition for empty sequences."""
    q, k = np.asarray(query, F32), np.asarray(key, F32)
    if use_qk_l2norm_in_kernel:
        q = l2norm(q, dt)
        k = l2norm(k, dt)
    q, k, v, bt, gg = [np.ascontiguousarray(np.swapaxes(np.asarray(x, F32), 1, 2))
                       for x in (q, k, value, beta, g)]
    B, H, L, dk = k.shape
    dv = v.shape[-1]
    C = chunk_size
    pad = (C - L % C) % C
    q, k, v = [np.pad(x, ((0, 0), (0, 0), (0, pad), (0, 0))) for x in (q, k, v)]
    bt, gg = [np.pad(x, ((0, 0), (0, 0), (0, pad))) for x in (bt, gg)]
    Lp = L + pad
    q = (q * F32(1.0 / dk ** 0.5)).astype(F32)
    v_beta = v * bt[..., None]
    k_beta = k * bt[..., None]
    n = Lp // C
    q, k, v, k_beta, v_beta = [x.reshape(B, H, n, C, x.shape[-1]) for x in (q, k, v, k_beta, v_beta)]
    gc = np.cumsum(gg.reshape(B, H, n, C).astype(np.float64), axis=-1).astype(F32)
    diff = np.tril(gc[..., :, None] - gc[..., None, :])
    decay = np.tril(np.exp(diff)).astype(F32)
    kt = np.swapaxes(k, -1, -2)
    X = -(np.matmul(k_beta, kt) * decay)
    X = np.tril(X, -1).astype(F32)
    T = unit_lower_inv(X)
    V = np.matmul(T, v_beta)
    Kc = np.matmul(T, k_beta * np.exp(gc)[..., None])
    QK = np.tril(np.matmul(q, kt) * decay).astype(F32)
    Qg = q * np.exp(gc)[..., None]
    glast = gc[..., -1]
    Gl = np.exp(glast)
    Kd = np.swapaxes(k * np.exp(glast[..., None] - gc)[..., None], -1, -2)
    S = (np.zeros((B, H, dk, dv), F32) if initial_state is None
         else np.asarray(initial_state, F32).copy())
    outs = []
    for i in range(n):
        vn = V[:, :, i] - np.matmul(Kc[:, :, i], S)
        outs.append(np.matmul(Qg[:, :, i], S) + np.matmul(QK[:, :, i], vn))
        S = (S * Gl[:, :, i, None, None] + np.matmul(Kd[:, :, i], vn)).astype(F32)
    core = (np.stack(outs, axis=2).reshape(B, H, Lp, dv)[:, :, :L] if outs
            else np.zeros((B, H, 0, dv), F32))
    out = rnd(np.swapaxes(core, 1, 2), dt)
    return out, (S if output_final_state else None)


# --------------------------------------------------------------------------- recurrence
def recurrent_gated_delta_rule(query, key, value, g, beta, initial_state, output_final_state,
                               use_qk_l2norm_in_kernel=False, dt="f32"):
    """Token-by-token gated delta rule (src/recurrent_single_step.py:8-32 for T=1 and its
    T>1 fallback TF:314-353).  Shapes as chunk_gated_delta_rule."""
    q, k = np.asarray(query, F32), np.asarray(key, F32)
    if use_qk_l2norm_in_kernel:
        q = l2norm(q, dt)
        k = l2norm(k, dt)
    q, k, v, bt, gg = [np.swapaxes(np.asarray(x, F32), 1, 2) for x in (q, k, value, beta, g)]
    B, H, L, dk = k.shape
    dv = v.shape[-1]
    q = (q * F32(1.0 / dk ** 0.5)).astype(F32)
    S = (np.zeros((B, H, dk, dv), F32) if initial_state is None
         else np.asarray(initial_state, F32).copy())
    out = np.zeros((B, H, L, dv), F32)
    for t in range(L):
        S = (S * np.exp(gg[:, :, t])[..., None, None]).astype(F32)
        mem = (S * k[:, :, t, :, None]).sum(-2, dtype=F32)
        delta = (v[:, :, t] - mem) * bt[:, :, t, None]
        S = (S + k[:, :, t, :, None] * delta[:, :, None, :]).astype(F32)
        out[:, :, t] = (S * q[:, :, t, :, None]).sum(-2, dtype=F32)
    return rnd(np.swapaxes(out, 1, 2), dt), (S if output_final_state else None)


# --------------------------------------------------------------------------- conv
def conv_update_elem(x, state, weight, bias=None, dt="bf16"):
    """Decode causal depthwise conv as mul + sum (src/cb_engine.py:43-51).
    x [n,C,1], state [n,C,K] updated IN PLACE, weight [C,K], bias [C] or None."""
    hs = np.concatenate([state, x], axis=-1).astype(F32)
    state[...] = hs[:, :, -state.shape[-1]:]
    win = hs[:, :, -weight.shape[-1]:]
    out = rnd(rnd(win * weight, dt).sum(-1, keepdims=True, dtype=F32), dt)
    if bias is not None:
        out = rnd(out + np.asarray(bias, F32).reshape(1, -1, 1), dt)
    return rnd(silu(out), dt)


def conv_update(x, state, weight, bias=None, dt="bf16"):
    """HF torch_causal_conv1d_update (TF:210-226) with silu: one rounding of the
    fp32-accumulated conv (plus bias) per output.  x [n,C,T], state [n,C,K] updated in place."""
    n, C, T = x.shape
    K = state.shape[-1]
    Kw = weight.shape[-1]
    hs = np.concatenate([state, x], axis=-1).astype(F32)
    state[...] = hs[:, :, -K:]
    out = np.zeros((n, C, T), F32)
    base = hs.shape[-1] - T
    for t in range(T):
        win = hs[:, :, base + t - Kw + 1:base + t + 1]
        acc = (win * weight).sum(-1, dtype=F32)
        if bias is not None:
            acc = acc + np.asarray(bias, F32)
        out[:, :, t] = acc
    return rnd(silu(rnd(out, dt)), dt)


def prefill_conv(x, cu_seqlens, weight, bias=None, init_state=None, dt="bf16"):
    """Varlen causal depthwise conv1d + silu over packed tokens, with the decode conv state
    of each sequence (last K inputs, left zero-padded) (TF:463-474, src/cb_tp.py:158-164,
    :236-244, :260).  x [T,C]; init_state [B,C,K] or None (zeros).
    Returns (y [T,C], new_state [B,C,K])."""
    x = np.asarray(x, F32)
    T, C = x.shape
    K = weight.shape[-1]
    B = len(cu_seqlens) - 1
    y = np.zeros_like(x)
    st = np.zeros((B, C, K), F32)
    for b in range(B):
        s, e = int(cu_seqlens[b]), int(cu_seqlens[b + 1])
        prev = np.zeros((C, K), F32) if init_state is None else np.asarray(init_state[b], F32)
        full = np.concatenate([prev, x[s:e].T], axis=-1)
        L = e - s
        for t in range(L):
            acc = (full[:, t + 1:t + 1 + K] * weight).sum(-1, dtype=F32)
            if bias is not None:
                acc = acc + np.asarray(bias, F32)
            y[s + t] = rnd(silu(rnd(acc, dt)), dt)
        st[b] = full[:, -K:]
    return y, st


# --------------------------------------------------------------------------- norm / gates
def gated_rmsnorm(x, gate, weight, eps=1e-6, dt="bf16"):
    """Qwen3_5RMSNormGated.forward (TF:181-191): w * rnd(x*rsqrt(mean x^2+eps)) * silu(z)."""
    h = np.asarray(x, F32)
    var = (h * h).mean(-1, keepdims=True, dtype=F32)
    h = (h * (F32(1) / np.sqrt(var + F32(eps)))).astype(F32)
    h = rnd(np.asarray(weight, F32) * rnd(h, dt), dt)
    h = h * silu(np.asarray(gate, F32))
    return rnd(h, dt)


def decode_gates(a, b, A_log, dt_bias, dt="bf16"):
    """beta = sigmoid(b) (in b's dtype); g = -exp(A_log) * softplus(a + dt_bias) in fp32
    (src/cb_engine.py:337-338, TF:491-493)."""
    beta = rnd(sigmoid(b), dt)
    g = (-np.exp(np.asarray(A_log, F32)) * softplus(np.asarray(a, F32) + np.asarray(dt_bias, F32)))
    return beta, g.astype(F32)


# --------------------------------------------------------------------------- slot-indexed wrappers
def repeat_heads(x, r):
    """repeat_interleave(r, dim=2) on [..., T, H, D] (src/cb_engine.py:339-342)."""
    return np.repeat(x, r, axis=-2) if r > 1 else x


def decode_step_slots(q, k, v, g, beta, rec_pool, slot_idx, use_qk_l2norm=True, dt="bf16"):
    """One decode token for slots ``slot_idx``: gathers rec_pool[slot_idx], runs the single
    step, scatters the new state back (src/cb_engine.py:344-347).  q,k [n,Hk,dk] (un-repeated),
    v [n,Hv,dv], g/beta [n,Hv].  rec_pool updated IN PLACE.  Returns o [n,Hv,dv]."""
    Hk, Hv = q.shape[1], v.shape[1]
    r = Hv // Hk
    qq = repeat_heads(q, r)[:, None]
    kk = repeat_heads(k, r)[:, None]
    init = rec_pool[np.asarray(slot_idx)]
    o, S = recurrent_gated_delta_rule(qq, kk, v[:, None], g[:, None], beta[:, None], init, True,
                                      use_qk_l2norm, dt)
    rec_pool[np.asarray(slot_idx)] = S
    return o[:, 0]


def prefill_varlen(q, k, v, g, beta, cu_seqlens, state_pool=None, slot_idx=None, use_initial=None,
                   use_qk_l2norm=True, dt="bf16", chunk_size=64):
    """Packed varlen chunk prefill: each sequence b runs the chunk rule from zeros (or from
    state_pool[slot_idx[b]] when use_initial[b]) and its final state is written to
    state_pool[slot_idx[b]] (src/cb_tp.py:176-180, :256-261).  q,k [T,Hk,dk], v [T,Hv,dv],
    g/beta [T,Hv].  Returns (o [T,Hv,dv], list of final states)."""
    Hk, Hv = q.shape[1], v.shape[1]
    r = Hv // Hk
    outs, finals = [], []
    for b in range(len(cu_seqlens) - 1):
        s, e = int(cu_seqlens[b]), int(cu_seqlens[b + 1])
        init = None
        if use_initial is not None and use_initial[b]:
            init = state_pool[slot_idx[b]][None]
        o, S = chunk_gated_delta_rule(repeat_heads(q[s:e], r)[None], repeat_heads(k[s:e], r)[None],
                                      v[s:e][None], g[s:e][None], beta[s:e][None], chunk_size, init,
                                      True, use_qk_l2norm, dt)
        outs.append(o[0])
        finals.append(S[0])
        if state_pool is not None and slot_idx is not None:
            state_pool[slot_idx[b]] = S[0]
    return np.concatenate(outs, axis=0), finals
