"""CPU restatement of the reference's GDN path in torch ops, for the timed CPU baselines.

Test infrastructure, like gdn_oracle.py (the numpy oracle this module is checked against in
tests/test_oracle_golden.py): it restates the same algorithms with torch tensor ops so that, like
the reference's own code, it runs multi-threaded on the host cores.  bench.py's CPU legs
(``cpu_baseline`` and ``--impl reference``) time it; nothing in the product imports it.

  * chunk_gated_delta_rule  -- fast_chunk_gated_delta_rule_v2 (src/gdn_chunk_fast2.py:11-62),
                               l2norm and blocked inverse of src/gdn_chunk_fast.py:17-62
  * recurrent_step          -- recurrent_single_step (src/recurrent_single_step.py:14-32)
  * elem_conv_update        -- src/cb_engine.py:43-51
  * gated_rmsnorm           -- Qwen3_5RMSNormGated.forward (transformers Qwen3.5, TF:181-191)
  * decode_layer            -- the operator part of CBEngine._gdn (src/cb_engine.py:318-352)
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def l2norm(x, eps=1e-6):
    """x * rsqrt(sum(x*x) + eps) in x's dtype (src/gdn_chunk_fast.py:17-18)."""
    return x * torch.rsqrt((x * x).sum(dim=-1, keepdim=True) + eps)


def _small_inv(X):
    """(I - X)^-1 for a strictly lower block by the row recurrence (src/gdn_chunk_fast.py:21-30)."""
    n = X.shape[-1]
    R = X.clone()
    for i in range(1, n):
        row = R[..., i, :i].clone()
        sub = R[..., :i, :i].clone()
        R[..., i, :i] = row + (row.unsqueeze(-1) * sub).sum(-2)
    return R + torch.eye(n, dtype=X.dtype)


def _unit_lower_inv(X, base=16):
    """Blocked (I - X)^-1: 16 x 16 diagonal blocks, then merges T21 = B X21 A
    (src/gdn_chunk_fast.py:33-62)."""
    n = X.shape[-1]
    nb = n // base
    diag = torch.stack([X[..., i * base:(i + 1) * base, i * base:(i + 1) * base] for i in range(nb)], dim=-3)
    Td = _small_inv(diag)
    blocks = [Td[..., i, :, :] for i in range(nb)]

    def merge(lo, hi):
        if hi - lo == 1:
            return blocks[lo]
        mid = (lo + hi) // 2
        A = merge(lo, mid)
        B = merge(mid, hi)
        T21 = B @ X[..., mid * base:hi * base, lo * base:mid * base] @ A
        top = torch.cat([A, torch.zeros(A.shape[:-1] + (B.shape[-1],), dtype=A.dtype)], dim=-1)
        return torch.cat([top, torch.cat([T21, B], dim=-1)], dim=-2)

    return merge(0, nb)


def chunk_gated_delta_rule(q, k, v, g, beta, chunk_size=64, initial_state=None, output_final_state=True,
                           use_qk_l2norm_in_kernel=True):
    """v2 chunk rule (src/gdn_chunk_fast2.py:11-62); q, k, v [B, L, H, D] (k repeated to H heads),
    g, beta [B, L, H].  Returns (out [B, L, H, dv] in q's dtype, final state fp32 or None)."""
    dt = q.dtype
    if use_qk_l2norm_in_kernel:
        q, k = l2norm(q), l2norm(k)
    q, k, v, beta, g = [x.transpose(1, 2).contiguous().float() for x in (q, k, v, beta, g)]
    B, H, L, dk = k.shape
    dv = v.shape[-1]
    C = chunk_size
    pad = (C - L % C) % C
    q, k, v = [F.pad(x, (0, 0, 0, pad)) for x in (q, k, v)]
    beta, g = [F.pad(x, (0, pad)) for x in (beta, g)]
    n = (L + pad) // C
    q = q * dk ** -0.5
    v_beta, k_beta = v * beta[..., None], k * beta[..., None]
    q, k, v_beta, k_beta = [x.reshape(B, H, n, C, x.shape[-1]) for x in (q, k, v_beta, k_beta)]
    gc = g.reshape(B, H, n, C).cumsum(-1)
    decay = (gc[..., :, None] - gc[..., None, :]).tril().exp().tril()
    kt = k.transpose(-1, -2)
    X = (-(k_beta @ kt) * decay).tril(-1)
    T = _unit_lower_inv(X)
    V = T @ v_beta
    Kc = T @ (k_beta * gc.exp()[..., None])
    QK = ((q @ kt) * decay).tril()
    Qg = q * gc.exp()[..., None]
    glast = gc[..., -1]
    Kd = (k * (glast[..., None] - gc).exp()[..., None]).transpose(-1, -2)
    S = torch.zeros(B, H, dk, dv) if initial_state is None else initial_state.float().clone()
    outs = []
    for i in range(n):
        vn = V[:, :, i] - Kc[:, :, i] @ S
        outs.append(Qg[:, :, i] @ S + QK[:, :, i] @ vn)
        S = S * glast[:, :, i, None, None].exp() + Kd[:, :, i] @ vn
    o = torch.stack(outs, dim=2).reshape(B, H, n * C, dv)[:, :, :L]
    return o.transpose(1, 2).to(dt), (S if output_final_state else None)


def recurrent_step(q, k, v, g, beta, S):
    """One token (src/recurrent_single_step.py:14-32): q, k [n, H, dk] (l2-normalised, repeated),
    v [n, H, dv], g, beta [n, H], S [n, H, dk, dv] fp32 (new state returned).  Returns (o, S)."""
    dt = q.dtype
    q, k, v, g, beta = q.float() * q.shape[-1] ** -0.5, k.float(), v.float(), g.float(), beta.float()
    S = S * g.exp()[..., None, None]
    mem = (S * k[..., None]).sum(-2)
    delta = (v - mem) * beta[..., None]
    S = S + k[..., None] * delta[..., None, :]
    o = (S * q[..., None]).sum(-2)
    return o.to(dt), S


def elem_conv_update(x, state, weight, bias=None):
    """src/cb_engine.py:43-51: x [n, C], state [n, C, K] (updated in place); silu(conv) in x's dtype."""
    hs = torch.cat([state, x[..., None]], dim=-1)
    state.copy_(hs[..., -state.shape[-1]:])
    out = (hs[..., -weight.shape[-1]:] * weight).sum(-1)
    if bias is not None:
        out = out + bias
    return F.silu(out)


def gated_rmsnorm(x, z, w, eps=1e-6):
    """Qwen3_5RMSNormGated.forward (TF:181-191)."""
    dt = x.dtype
    h = x.float()
    h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps)
    h = w * h.to(dt)
    return (h * F.silu(z.float())).to(dt)


def decode_layer(mixed, z, a, b, A_log, dt_bias, conv_w, conv_pool, rec_pool, slot, norm_w, Hk, Hv, d):
    """The operator part of CBEngine._gdn (src/cb_engine.py:318-352) for n slots, with the
    reference's index_select / index_copy_ around the plug-ins; pools updated in place."""
    n = mixed.shape[0]
    st = conv_pool.index_select(0, slot)
    y = elem_conv_update(mixed, st, conv_w)
    conv_pool.index_copy_(0, slot, st)
    q = l2norm(y[:, :Hk * d].reshape(n, Hk, d)).repeat_interleave(Hv // Hk, dim=1)
    k = l2norm(y[:, Hk * d:2 * Hk * d].reshape(n, Hk, d)).repeat_interleave(Hv // Hk, dim=1)
    v = y[:, 2 * Hk * d:].reshape(n, Hv, d)
    beta = b.sigmoid()
    g = -A_log.float().exp() * F.softplus(a.float() + dt_bias)
    o, S = recurrent_step(q, k, v, g, beta, rec_pool.index_select(0, slot))
    rec_pool.index_copy_(0, slot, S)
    return gated_rmsnorm(o, z, norm_w)
