"""Slot-based continuous-batching engine for the hybrid Qwen3.5 model on B200.

Same public interface as the reference's ``CBEngine`` (src/cb_engine.py:80-355):
``CBEngine(model, n_slots, t_max, device, graph_decode=False, tp=1)`` with ``prefill(slot, ids)``,
``prefill_batch(slots, id_list)``, ``decode_step(slots, tokens)`` and ``free(slot)``, plus the
``prefill_chunk(slot, ids, start, last)`` of the reference's ``TPEngine`` (src/cb_tp.py:195-271).

What changes on B200:
  * GDN layers call the slot-indexed CUDA kernels: prefill writes the final recurrent state and
    the conv window straight into the slot's pool rows (no cache copy, src/cb_engine.py:198-205);
    decode runs one fused kernel pair per layer that gathers and scatters the state in-kernel.
  * ``prefill_batch`` packs prompts back to back (``cu_seqlens``) instead of left padding them
    (src/cb_engine.py:210-242).
  * Decode always covers all N slots, as the reference does (src/cb_engine.py:245-252), but an
    inactive slot's GDN update goes to a scratch pool row (index N) through the slot index, so
    slots that are idle or in the middle of a chunked prefill are left exactly as they were; the
    reference needs ``hold`` save/restore for that (src/cb_tp.py:273-285).
  * Decode steps are captured in CUDA graphs, one per attention-length bucket, from one shared
    memory pool (src/cb_engine.py:123-187).
Attention, MLP, norms, embeddings and the LM head are HF's own modules, as in the reference.
"""
from __future__ import annotations

import os

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops

# Decode conv rounding: False = HF torch_causal_conv1d_update (one rounding of the fp32 sum);
# True = the reference's elem_conv_update (products and sum rounded in bf16).  Set by the caller
# exactly like the reference's cb_engine.ELEM_CONV (src/cb_engine.py:25).
ELEM_CONV = False

# One captured decode graph per attention-length bucket of this many tokens (src/cb_engine.py:28).
GRAPH_BUCKET = int(os.environ.get("CB_GRAPH_BUCKET", "512"))


def fuse_linears(mods):
    """One weight matrix for bias-free linears that read the same input: their weights stacked by rows
    (padded with zero rows to a multiple of 8, so every slice of the product starts 16-byte aligned),
    and each module's weight becomes a view into it, so no second copy stays in memory.  Returns
    (W, the row count of each module)."""
    ws = [m.weight.detach() for m in mods]
    rows = sum(w.shape[0] for w in ws)
    pad = (-rows) % 8
    parts = ws + ([ws[0].new_zeros(pad, ws[0].shape[1])] if pad else [])
    W = torch.cat(parts, 0)
    off = 0
    for m, w in zip(mods, ws):
        m.weight = nn.Parameter(W[off:off + w.shape[0]], requires_grad=False)
        off += w.shape[0]
    return W, [w.shape[0] for w in ws]


def _check_slots(what, slots):
    """Each slot at most once per call: two prompts (or two decode entries) on one slot would write
    its pool rows from two sequences at once.  Slot indices outside the pools are left to the
    kernels, which flag them on the device (error 1) and touch no pool row."""
    if len(set(int(s) for s in slots)) != len(slots):
        raise ValueError(f"{what}: a slot appears more than once in {list(slots)}")


class CBEngine:
    def __init__(self, model, n_slots, t_max, device, graph_decode=False, tp=1):
        from transformers.models.qwen3_5 import modeling_qwen3_5 as M
        self.M = M
        self.model = model
        self.lm = model.model.language_model
        cfg = model.config.text_config
        self.cfg = cfg
        self.dev = torch.device(device)
        if self.dev.type != "cuda":
            raise RuntimeError("the B200 engine runs on CUDA devices only")
        self.N = n_slots
        self.T = t_max
        self.tp = tp
        self.K = cfg.linear_conv_kernel_dim
        self.lens = [0] * n_slots
        bf = torch.bfloat16
        self.kv_k, self.kv_v, self.conv, self.rec, self.gdn = {}, {}, {}, {}, {}
        ws_bytes = 0
        for i, t in enumerate(cfg.layer_types):
            layer = self.lm.layers[i]
            if t == "full_attention":
                at = layer.self_attn
                kvh = at.k_proj.weight.shape[0] // at.head_dim
                # row N is a scratch row: never read as a real slot
                self.kv_k[i] = torch.zeros(n_slots + 1, kvh, t_max, at.head_dim, dtype=bf, device=self.dev)
                self.kv_v[i] = torch.zeros(n_slots + 1, kvh, t_max, at.head_dim, dtype=bf, device=self.dev)
            else:
                gd = layer.linear_attn
                Hk, Hv, dk, dv = gd.num_k_heads, gd.num_v_heads, gd.head_k_dim, gd.head_v_dim
                self.conv[i] = torch.zeros(n_slots + 1, gd.conv_dim, self.K, dtype=bf, device=self.dev)
                self.rec[i] = torch.zeros(n_slots + 1, Hv, dk, dv, dtype=torch.float32, device=self.dev)
                self.gdn[i] = dict(
                    Hk=Hk, Hv=Hv, dk=dk, dv=dv,
                    A_log=gd.A_log.detach().float().contiguous(),
                    dt_bias=gd.dt_bias.detach().float().contiguous(),
                    conv_w=gd.conv1d.weight.detach().squeeze(1).contiguous(),
                    conv_b=None if gd.conv1d.bias is None else gd.conv1d.bias.detach().contiguous(),
                    norm_w=gd.norm.weight.detach().to(bf).contiguous(),
                    eps=float(getattr(gd.norm, "variance_epsilon", getattr(gd.norm, "eps", 1e-6))))
                ws_bytes = max(ws_bytes, ops.decode_layer_workspace_bytes(n_slots, Hk, Hv, dk, dv, bf))
        self._ws = torch.zeros(max(ws_bytes, 256), dtype=torch.uint8, device=self.dev)  # decode tickets
        # Decode runs one GEMM per group of projections that read the same input (the reference runs
        # each projection separately): attention q/k/v, the GDN in_proj_qkv/z/b/a, the MLP gate/up.
        # With 16-64 tokens a step these GEMMs are launch- and latency-bound, so fewer and wider ones
        # save time at every TP degree.  The modules keep working (their weights are views).
        self._fused = {}
        for i, t in enumerate(cfg.layer_types):
            layer = self.lm.layers[i]
            if t == "full_attention":
                at = layer.self_attn
                W, sizes = fuse_linears([at.q_proj, at.k_proj, at.v_proj])
            else:
                gd = layer.linear_attn
                W, sizes = fuse_linears([gd.in_proj_qkv, gd.in_proj_z, gd.in_proj_b, gd.in_proj_a])
            mlp = layer.mlp
            Wm, msz = fuse_linears([mlp.gate_proj, mlp.up_proj])
            self._fused[i] = dict(W=W, sizes=sizes, Wm=Wm, inter=msz[0])
        hq_max = max([self.lm.layers[i].self_attn.q_proj.weight.shape[0] // (2 * self.lm.layers[i].self_attn.head_dim)
                      for i, t in enumerate(cfg.layer_types) if t == "full_attention"] or [1])
        hd_max = max([self.lm.layers[i].self_attn.head_dim
                      for i, t in enumerate(cfg.layer_types) if t == "full_attention"] or [8])
        self._attn_ws = ops.attn_decode_workspace(n_slots, hq_max, hd_max, t_max, self.dev)
        self._tok = torch.zeros(n_slots, dtype=torch.long, device=self.dev)
        self._pos = torch.zeros(n_slots, dtype=torch.long, device=self.dev)
        self._slot = torch.arange(n_slots, dtype=torch.int32, device=self.dev)
        # Device error flag shared by every kernel call of the engine (0 = fine, 1 = a slot index
        # outside the pools, 2 = a bounded wait inside a kernel ran out, 3 = a peer exchange timed out).  It is read back with the
        # tokens each step already copies to the host, so checking it costs no extra sync.
        self._err = torch.zeros(1, dtype=torch.int32, device=self.dev)
        # a tensor-parallel engine's peer exchanges report into the same flag (3 = a rank did not
        # arrive in time), bound before any graph captures their calls
        for inst in (getattr(self, "peer_ar", None), getattr(self, "peer_linear", None),
                     getattr(self, "peer_norm", None)):
            if inst is not None:
                inst.err = self._err
        self.graph_decode = graph_decode
        if not hasattr(self, "peer_linear"):
            self.peer_linear = None       # TPEngine sets its tensor-parallel exchanges before this runs
            self.peer_norm = None
            self.decode_sum = None
        self._graphs, self._graph_out = {}, {}
        if graph_decode:
            self._capture_graphs()

    # ------------------------------------------------------------------ graph decode
    def _buckets(self):
        b = list(range(GRAPH_BUCKET, self.T + 1, GRAPH_BUCKET))
        if not b or b[-1] < self.T:
            b.append(self.T)
        return b

    def _bucket(self, L):
        for b in self._buckets():
            if b >= L:
                return b
        raise ValueError(f"decode length {L} > T {self.T}")

    def _capture_graphs(self):
        """One CUDA graph per attention-length bucket, all from one memory pool; must run before
        any prefill (state written by warm-up and capture is zeroed afterwards)."""
        pool = torch.cuda.graph_pool_handle()
        with torch.inference_mode():
            self._core(self._buckets()[0])               # eager warm-up outside capture
            torch.cuda.synchronize(self.dev)
            for b in self._buckets():
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, pool=pool):
                    out = self._core(b)
                self._graphs[b], self._graph_out[b] = g, out
            torch.cuda.synchronize(self.dev)
            self._reset_state()

    def _reset_state(self):
        for d in (self.kv_k, self.kv_v, self.conv, self.rec):
            for t in d.values():
                t.zero_()
        self._err.zero_()
        self.lens = [0] * self.N

    # ------------------------------------------------------------------ decode
    def _attn(self, at, i, h, cos, sin, pos32, Lmax):
        """Decode attention (src/cb_engine.py:295-316): projections, q/k norms and rotary as the
        reference; the K/V row write, the attention over positions 0..pos of each slot and the
        sigmoid output gate in one library call (gdn_attn_decode) instead of index_copy_ + masked
        SDPA over the Lmax bucket + gate."""
        n = h.shape[0]
        hd = at.head_dim
        kvh = self.kv_k[i].shape[1]
        f = self._fused[i]
        nq, nk, _ = f["sizes"]
        y = F.linear(h, f["W"])                       # [q | k | v] of one GEMM
        rd = cos.shape[-1]
        if (hd % 8 == 0 and hd <= 256 and rd % 16 == 0 and 16 <= rd <= hd and at.q_norm.eps == at.k_norm.eps
                and y.dtype == torch.bfloat16):
            # q/k norms, rotary and the layout attn_decode takes, in one kernel (bit for bit the ops below)
            q, k, v, gate = ops.attn_decode_prep(y.view(n, -1), at.q_norm.weight, at.k_norm.weight, at.q_norm.eps,
                                                 cos, sin, nq // (2 * hd), kvh, hd)
            o = ops.attn_decode(q, k, v, self.kv_k[i], self.kv_v[i], self._slot, pos32, Lmax, at.scaling, gate=gate,
                                workspace=self._attn_ws, err=self._err)
            return o.reshape(n, 1, -1), at.o_proj
        qg = y[..., :nq].view(n, 1, -1, hd * 2)
        q, gate = torch.chunk(qg, 2, dim=-1)
        q = at.q_norm(q).transpose(1, 2)
        k = at.k_norm(y[..., nq:nq + nk].view(n, 1, kvh, hd)).transpose(1, 2)
        v = y[..., nq + nk:nq + 2 * nk].view(n, 1, kvh, hd).transpose(1, 2)
        q, k = self.M.apply_rotary_pos_emb(q, k, cos, sin)
        o = ops.attn_decode(q[:, :, 0], k[:, :, 0], v[:, :, 0], self.kv_k[i], self.kv_v[i], self._slot, pos32, Lmax,
                            at.scaling, gate=gate, workspace=self._attn_ws, err=self._err)
        return o.reshape(n, 1, -1), at.o_proj

    def _gdn(self, gd, i, h):
        n = h.shape[0]
        p = self.gdn[i]
        f = self._fused[i]
        C, Z, Bn, An = f["sizes"]
        y = F.linear(h.reshape(n, -1), f["W"])       # [qkv | z | b | a] of one GEMM; row-strided slices
        mixed, z = y[:, :C], y[:, C:C + Z]
        b, a = y[:, C + Z:C + Z + Bn], y[:, C + Z + Bn:C + Z + Bn + An]
        core = ops.decode_layer(mixed, z, a, b, p["A_log"], p["dt_bias"], p["conv_w"], p["conv_b"], self.conv[i],
                                self.rec[i], self._slot, p["norm_w"], p["eps"], p["Hk"], p["Hv"], p["dk"], p["dv"],
                                ops.GDN_CONV_ELEM if ELEM_CONV else ops.GDN_CONV_HF, workspace=self._ws,
                                err=self._err)
        return core.reshape(n, 1, -1), gd.out_proj

    def _mlp_act(self, i, mlp, h):
        """The MLP up to its down projection, act(gate(h)) * up(h), with gate and up from one GEMM."""
        f = self._fused[i]
        I = f["inter"]
        y = F.linear(h, f["Wm"])
        if type(mlp.act_fn).__name__ in ("SiLU", "SiLUActivation"):   # both are F.silu
            return ops.silu_mul(y, I)         # one kernel for silu then product (bit for bit the same)
        return mlp.act_fn(y[..., :I]) * y[..., I:2 * I]

    def _proj_add_norm(self, proj, a, x, norm):
        """A layer's output projection, the residual add and the next RMSNorm of the decode step:
        x <- x + proj(a) in place; returns norm(x).  With a tensor-parallel exchange (``peer_linear``,
        set by TPEngine) the sum over ranks runs inside the add + norm kernel
        (gdn_allreduce_add_rmsnorm), or the projection pushes this rank's partial to every rank
        (gdn_linear_push, or a cuBLAS GEMM and gdn_push_partial) and one kernel sums the ranks'
        partials, adds and normalizes (gdn_pull_add_rmsnorm);
        otherwise the projection's own forward (cuBLAS, plus the all-reduce of AllReduceLinear under
        TP) is followed by gdn_add_rmsnorm.  Both equal the reference's ``x = x + proj(a)`` and the
        norm module of the next step (src/cb_engine.py:295-355)."""
        lin = getattr(proj, "lin", None)
        arn = self.peer_norm
        if arn is not None and lin is not None and lin.bias is None:
            h = F.linear(a, lin.weight)                   # this rank's partial (cuBLAS)
            if arn.applies(h):
                return arn(x, h, norm.weight, norm.eps)   # sum over ranks + add + norm, one kernel
            return ops.add_rmsnorm(x, proj.reduce(h), norm.weight, norm.eps)
        ex = self.peer_linear
        if ex is not None and lin is not None and lin.bias is None and ex.applies(a, lin.weight):
            if self.decode_sum == "fused":
                ex.push(a, lin.weight)                   # tcgen05 projection sending its tiles
            else:
                ex.push_partial(F.linear(a, lin.weight))  # cuBLAS projection, then the push
            return ex.pull_add_rmsnorm(x, norm.weight, norm.eps)
        return ops.add_rmsnorm(x, proj(a), norm.weight, norm.eps)

    def _core(self, Lmax):
        """One decode step for all N slots from the static buffers (capturable)."""
        N, pos = self.N, self._pos
        pos32 = pos.to(torch.int32)
        x = self.lm.embed_tokens(self._tok[:, None])
        pos3 = pos.view(1, N, 1).expand(3, N, 1)
        cos, sin = self.lm.rotary_emb(x, pos3)
        layers = self.lm.layers
        h = layers[0].input_layernorm(x)
        for i, layer in enumerate(layers):
            if self.cfg.layer_types[i] == "full_attention":
                a, proj = self._attn(layer.self_attn, i, h, cos, sin, pos32, Lmax)
            else:
                a, proj = self._gdn(layer.linear_attn, i, h)
            h = self._proj_add_norm(proj, a, x, layer.post_attention_layernorm)
            nxt = layers[i + 1].input_layernorm if i + 1 < len(layers) else self.lm.norm
            h = self._proj_add_norm(layer.mlp.down_proj, self._mlp_act(i, layer.mlp, h), x, nxt)
        # next tokens and, as the last entry, the error flag after this step's kernels
        return torch.cat([self._greedy(h[:, 0]), self._err.to(torch.long)])

    def _greedy(self, h):
        """Greedy next token per row of the final hidden states (a vocabulary-parallel head
        provides its own cross-rank argmax)."""
        head = self.model.lm_head
        pick = getattr(head, "greedy", None)
        return pick(h) if pick is not None else head(h).argmax(-1)

    _ERRORS = {1: "a slot index outside the state pools", 2: "a bounded wait inside a kernel ran out",
               3: "a peer rank did not arrive in time (tensor-parallel exchange)"}

    def _raise_on(self, code, what):
        if code:
            self._err.zero_()
            raise RuntimeError(f"{what}: device error {code} ({self._ERRORS.get(code, 'unknown')})")

    def check_errors(self):
        """Raise RuntimeError if a kernel of this engine reported an error since the last check."""
        self._raise_on(int(self._err.item()), "CBEngine")

    @torch.inference_mode()
    def decode_step(self, slots, tokens, hold=()):
        """One token for each slot in ``slots``; returns the next token per slot.  All N slots are
        computed (dense, as the reference); slots not in ``slots`` write their GDN update to the
        scratch row, so their conv/recurrent state is untouched (``hold`` is accepted for
        interface parity with TPEngine.decode_step and needs no save/restore)."""
        _check_slots("decode_step", slots)
        if len(tokens) != len(slots):
            raise ValueError(f"decode_step: {len(tokens)} tokens for {len(slots)} slots")
        N = self.N
        tok_full = [0] * N
        slot_map = [N] * N
        for s, t in zip(slots, tokens):
            tok_full[s] = int(t)
            slot_map[s] = s
        L = max(self.lens[s] for s in slots) + 1 if slots else 1
        if L > self.T:
            raise ValueError(f"decode length {L} > T {self.T}")
        self._pos.copy_(torch.tensor(self.lens, dtype=torch.long))
        self._tok.copy_(torch.tensor(tok_full, dtype=torch.long))
        self._slot.copy_(torch.tensor(slot_map, dtype=torch.int32))
        if self.graph_decode:
            b = self._bucket(L)
            self._graphs[b].replay()
            nxt = self._graph_out[b].tolist()
        else:
            nxt = self._core(L).tolist()
        self._raise_on(nxt[N], "decode_step")
        for s in slots:
            self.lens[s] += 1
        return [nxt[s] for s in slots]

    # ------------------------------------------------------------------ prefill
    def _attn_prefill(self, at, i, h, cos, sin, slots, starts, cu):
        T = h.shape[1]
        hd = at.head_dim
        kvh = self.kv_k[i].shape[1]
        qg = at.q_proj(h).view(1, T, -1, hd * 2)
        q, gate = torch.chunk(qg, 2, dim=-1)
        gate = gate.reshape(1, T, -1)
        q = at.q_norm(q).transpose(1, 2)
        k = at.k_norm(at.k_proj(h).view(1, T, kvh, hd)).transpose(1, 2)
        v = at.v_proj(h).view(1, T, kvh, hd).transpose(1, 2)
        q, k = self.M.apply_rotary_pos_emb(q, k, cos, sin)
        g = q.shape[1] // kvh
        o = torch.empty_like(q)
        for b, slot in enumerate(slots):
            s, e, st = cu[b], cu[b + 1], starts[b]
            L = e - s
            self.kv_k[i][slot, :, st:st + L] = k[0, :, s:e]
            self.kv_v[i][slot, :, st:st + L] = v[0, :, s:e]
            kr = self.kv_k[i][slot:slot + 1, :, :st + L].repeat_interleave(g, dim=1)
            vr = self.kv_v[i][slot:slot + 1, :, :st + L].repeat_interleave(g, dim=1)
            if st == 0:
                o[:, :, s:e] = F.scaled_dot_product_attention(q[:, :, s:e], kr, vr, is_causal=True, scale=at.scaling)
            else:
                qpos = torch.arange(st, st + L, device=self.dev)
                kpos = torch.arange(st + L, device=self.dev)
                causal = (kpos[None, :] <= qpos[:, None])[None, None]
                o[:, :, s:e] = F.scaled_dot_product_attention(q[:, :, s:e], kr, vr, attn_mask=causal,
                                                              scale=at.scaling)
        o = o.transpose(1, 2).reshape(1, T, -1) * torch.sigmoid(gate)
        return at.o_proj(o)

    def _gdn_prefill(self, gd, i, h, cu_d, slot_t, use_init):
        T = h.shape[1]
        p = self.gdn[i]
        Hk, Hv, dk, dv = p["Hk"], p["Hv"], p["dk"], p["dv"]
        mixed = gd.in_proj_qkv(h)[0]
        z = gd.in_proj_z(h)[0].reshape(T, Hv, dv)
        b = gd.in_proj_b(h)[0]
        a = gd.in_proj_a(h)[0]
        y = ops.prefill_conv_varlen(mixed, cu_d, p["conv_w"], p["conv_b"], self.conv[i], slot_t, use_init,
                                    err=self._err)
        q = y[:, :Hk * dk].view(T, Hk, dk)
        k = y[:, Hk * dk:2 * Hk * dk].view(T, Hk, dk)
        v = y[:, 2 * Hk * dk:].view(T, Hv, dv)
        # beta = sigmoid(b) and g = -exp(A_log) softplus(a + dt_bias) are formed inside the kernel
        core = ops.chunk_prefill_varlen_gates(q, k, v, a, b, p["A_log"], p["dt_bias"], cu_d, self.rec[i], slot_t,
                                              use_init, True, err=self._err)
        core = ops.gated_rmsnorm(core, z, p["norm_w"], p["eps"])
        return gd.out_proj(core.reshape(1, T, -1))

    @torch.inference_mode()
    def prefill_batch(self, slots, id_list, starts=None):
        """Prefill several prompts in one packed forward (no padding).  ``starts`` (optional)
        continues sequences whose first ``starts[b]`` tokens are already in their slot (chunked
        prefill).  Returns the greedy next token per prompt."""
        _check_slots("prefill_batch", slots)
        B = len(slots)
        starts = [0] * B if starts is None else [int(s) for s in starts]
        ids = [x.reshape(-1).to(self.dev) for x in id_list]
        lens = [int(x.numel()) for x in ids]
        for st, L in zip(starts, lens):
            if st + L >= self.T:
                raise ValueError(f"prompt {st + L} >= T {self.T}")
        cu = [0]
        for L in lens:
            cu.append(cu[-1] + L)
        cu_d = torch.tensor(cu, dtype=torch.int32, device=self.dev)
        slot_t = torch.tensor(slots, dtype=torch.int32, device=self.dev)
        use_init = torch.tensor([1 if st > 0 else 0 for st in starts], dtype=torch.int32, device=self.dev)
        pos = torch.cat([torch.arange(st, st + L, device=self.dev) for st, L in zip(starts, lens)])
        x = self.lm.embed_tokens(torch.cat(ids)[None])
        T = x.shape[1]
        cos, sin = self.lm.rotary_emb(x, pos.view(1, 1, T).expand(3, 1, T))
        for i, layer in enumerate(self.lm.layers):
            h = layer.input_layernorm(x)
            if self.cfg.layer_types[i] == "full_attention":
                h = self._attn_prefill(layer.self_attn, i, h, cos, sin, slots, starts, cu)
            else:
                h = self._gdn_prefill(layer.linear_attn, i, h, cu_d, slot_t, use_init)
            x = x + h
            x = x + layer.mlp(layer.post_attention_layernorm(x))
        last = torch.tensor([c - 1 for c in cu[1:]], dtype=torch.long, device=self.dev)
        xl = self.lm.norm(x[0, last])
        res = torch.cat([self._greedy(xl), self._err.to(torch.long)]).tolist()
        self._raise_on(res[-1], "prefill_batch")
        firsts = res[:-1]
        for slot, st, L in zip(slots, starts, lens):
            self.lens[slot] = st + L
        return firsts

    def prefill(self, slot, ids):
        """ids: [1, L] (or [L]). Returns the first generated token (greedy)."""
        return self.prefill_batch([slot], [ids])[0]

    def prefill_chunk(self, slot, ids, start, last):
        """Prefill tokens [start, start + C) of one prompt into ``slot``; earlier chunks must already
        be in the slot.  Returns the first generated token when ``last``, else None
        (src/cb_tp.py:195-271)."""
        first = self.prefill_batch([slot], [ids], starts=[start])[0]
        return first if last else None

    def free(self, slot):
        self.lens[slot] = 0
