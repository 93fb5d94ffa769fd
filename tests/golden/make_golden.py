"""Generate golden input/output vectors for the GDN hot path from the REFERENCE itself.

Run once on a machine that has the reference sources and HF transformers (Qwen3.5):

    python tests/golden/make_golden.py --reference-src <reference>/src

It imports the reference's own modules (``gdn_chunk_fast``, ``gdn_chunk_fast2``,
``recurrent_single_step``, ``cb_engine.elem_conv_update``) and HF's
``modeling_qwen3_5`` functions, runs them on seeded inputs on the CPU and writes
``tests/golden/*.npz``.  The reference imports ``torch_npu``; an empty stand-in
module is registered after transformers is imported so the pure-torch functions
load on a machine without Ascend hardware.  bf16 tensors are stored as uint16 bit
patterns (key suffix ``__bf16``).

The files are the pins for ``oracle/gdn_oracle.py`` (CPU tests) and for the CUDA
kernels (GPU tests); they are committed so that the GPU box, which has no copy of
the reference, can use them.
"""
import argparse
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def load_reference(src):
    import transformers.utils.import_utils as iu
    iu.is_torch_npu_available = lambda *a, **k: False
    from transformers.models.qwen3_5 import modeling_qwen3_5 as M  # noqa: F401  (import first)
    sys.modules.setdefault("torch_npu", types.ModuleType("torch_npu"))
    sys.path.insert(0, src)
    import gdn_chunk_fast
    import gdn_chunk_fast2
    import recurrent_single_step
    import cb_engine
    return dict(M=M, v1=gdn_chunk_fast.fast_chunk_gated_delta_rule,
                v2=gdn_chunk_fast2.fast_chunk_gated_delta_rule_v2,
                rec1=recurrent_single_step.recurrent_single_step,
                elem=cb_engine.elem_conv_update)


def pack(d):
    """torch tensors -> numpy; bf16 -> uint16 bits under key '<name>__bf16'."""
    out = {}
    for k, v in d.items():
        if isinstance(v, torch.Tensor):
            v = v.detach().cpu().contiguous()
            if v.dtype == torch.bfloat16:
                out[k + "__bf16"] = v.view(torch.int16).numpy().view(np.uint16)
            else:
                out[k] = v.numpy()
        else:
            out[k] = np.asarray(v)
    return out


def save(name, d):
    path = os.path.join(HERE, name)
    np.savez_compressed(path, **pack(d))
    print(f"wrote {path} ({os.path.getsize(path) / 1024:.0f} KiB)")


def gdn_inputs(gen, L, Hk, Hv, dk, dv, dtype):
    """Config-0 distributions: q,k ~ N(0,1) L2-normalised per head; v ~ N(0,1);
    beta = sigmoid(N(0,1)); g = -U(0.01, 1.0)."""
    q = torch.randn(1, L, Hk, dk, generator=gen)
    k = torch.randn(1, L, Hk, dk, generator=gen)
    q = q / q.norm(dim=-1, keepdim=True)
    k = k / k.norm(dim=-1, keepdim=True)
    v = torch.randn(1, L, Hv, dv, generator=gen)
    beta = torch.sigmoid(torch.randn(1, L, Hv, generator=gen))
    g = -(0.01 + 0.99 * torch.rand(1, L, Hv, generator=gen))
    return q.to(dtype), k.to(dtype), v.to(dtype), g.float(), beta.to(dtype)


def rep(x, r):
    return x.repeat_interleave(r, dim=2) if r > 1 else x


def make_chunk(ref, name, lens, Hk, Hv, d, dtype, init_std, seed):
    """Chunk prefill through the reference v2 (src/gdn_chunk_fast2.py:11-62), one sequence per call
    as TPEngine.prefill does.  v1, HF's chunk fallback and HF's token-by-token recurrence are run on
    the same inputs; their max-abs distance to v2 is recorded (the outputs are not stored).
    Initial states are drawn on the bf16 grid so they can be stored as bf16 bits exactly."""
    gen = torch.Generator().manual_seed(seed)
    M = ref["M"]
    r = Hv // Hk
    rec = {"lens": np.asarray(lens, np.int32), "Hk": Hk, "Hv": Hv, "d": d}
    for b, L in enumerate(lens):
        q, k, v, g, beta = gdn_inputs(gen, L, Hk, Hv, d, d, dtype)
        init = None
        if init_std > 0:
            init = (torch.randn(1, Hv, d, d, generator=gen) * init_std).to(torch.bfloat16)
            rec[f"init{b}"] = init[0]
            init = init.float()
        args = (rep(q, r), rep(k, r), v, g, beta)
        kw = dict(initial_state=init, output_final_state=True, use_qk_l2norm_in_kernel=True)
        o2, s2 = ref["v2"](*args, **kw)
        for tag, fn in (("v1", ref["v1"]), ("hfchunk", M.torch_chunk_gated_delta_rule),
                        ("hfrec", M.torch_recurrent_gated_delta_rule)):
            o, s = fn(*args, **kw)
            rec[f"maxdiff_out_{tag}_{b}"] = (o.float() - o2.float()).abs().max().item()
            rec[f"maxdiff_state_{tag}_{b}"] = (s - s2).abs().max().item()
        rec.update({f"q{b}": q[0], f"k{b}": k[0], f"v{b}": v[0], f"g{b}": g[0], f"beta{b}": beta[0],
                    f"out{b}": o2[0], f"state{b}": s2[0]})
    save(name, rec)


def make_recurrent(ref, seed):
    """Decode step through recurrent_single_step on a slot-indexed pool (src/cb_engine.py:344-347)
    plus a T=3 call (the reference falls back to HF's token loop, TF:314-353).  Pool and initial
    states are drawn on the bf16 grid and stored as bf16 bits; new states are stored in fp32."""
    gen = torch.Generator().manual_seed(seed)
    n, S, Hk, Hv, d = 3, 5, 1, 3, 128
    r = Hv // Hk
    q, k, v, g, beta = gdn_inputs(gen, n, Hk, Hv, d, d, torch.bfloat16)
    # decode tensors are [n, 1, H, D]: token axis 1
    q, k, v = q[0][:, None], k[0][:, None], v[0][:, None]
    g, beta = g[0][:, None], beta[0][:, None]
    pool = (torch.randn(S, Hv, d, d, generator=gen) * 0.3).to(torch.bfloat16)
    slot_idx = torch.randperm(S, generator=gen)[:n].to(torch.int32)
    init = pool[slot_idx.long()].float()
    o, s_new = ref["rec1"](rep(q, r), rep(k, r), v, g, beta, init.clone(), True, True)
    q3, k3, v3, g3, b3 = gdn_inputs(gen, 3, Hk, Hv, d, d, torch.bfloat16)
    init3 = (torch.randn(1, Hv, d, d, generator=gen) * 0.3).to(torch.bfloat16)
    o3, s3 = ref["rec1"](rep(q3, r), rep(k3, r), v3, g3, b3, init3.float(), True, True)
    save("recurrent_bf16.npz", dict(q=q[:, 0], k=k[:, 0], v=v[:, 0], g=g[:, 0], beta=beta[:, 0],
                                    pool=pool, slot_idx=slot_idx, out=o[:, 0], new_state=s_new,
                                    q3=q3[0], k3=k3[0], v3=v3[0], g3=g3[0], beta3=b3[0],
                                    init3=init3[0], out3=o3[0], state3=s3[0]))


def make_conv(ref, seed):
    """Decode conv-state update: reference elem_conv_update (src/cb_engine.py:43-51) and HF
    torch_causal_conv1d_update (TF:210-226), 3 consecutive steps; plus a T=2 HF call."""
    gen = torch.Generator().manual_seed(seed)
    M = ref["M"]
    n, C, K = 4, 384, 4
    w = (torch.rand(C, K, generator=gen) - 0.5).to(torch.bfloat16)
    b = (torch.randn(C, generator=gen) * 0.1).to(torch.bfloat16)
    s0 = torch.randn(n, C, K, generator=gen).to(torch.bfloat16)
    xs = torch.randn(3, n, C, 1, generator=gen).to(torch.bfloat16)
    se, sh = s0.clone(), s0.clone()
    ye, yh, st_e, st_h = [], [], [], []
    for t in range(3):
        ye.append(ref["elem"](xs[t].clone(), se, w, b))
        yh.append(M.torch_causal_conv1d_update(xs[t].clone(), sh, w, b, "silu"))
        st_e.append(se.clone())
        st_h.append(sh.clone())
    x2 = torch.randn(n, C, 2, generator=gen).to(torch.bfloat16)
    s2 = s0.clone()
    y2 = M.torch_causal_conv1d_update(x2, s2, w, None, "silu")
    save("conv_bf16.npz", dict(w=w, b=b, s0=s0, xs=xs, y_elem=torch.stack(ye), y_hf=torch.stack(yh),
                               st_elem=torch.stack(st_e), st_hf=torch.stack(st_h), x2=x2, y2=y2,
                               s2_after=s2))


def make_prefill_conv(ref, seed):
    """Prefill causal conv as HF's GatedDeltaNet forward runs it (nn.Conv1d with padding K-1, then
    silu over the first L outputs; conv state = last K inputs, left zero-padded) (TF:463-474), and the
    continuation form of TPEngine.prefill_chunk (src/cb_tp.py:236-244, :260)."""
    gen = torch.Generator().manual_seed(seed)
    C, K = 256, 4
    conv = torch.nn.Conv1d(C, C, K, groups=C, padding=K - 1, bias=False)
    with torch.no_grad():
        conv.weight.copy_((torch.rand(C, 1, K, generator=gen) - 0.5))
    conv = conv.to(torch.bfloat16)
    lens = [1, 3, 4, 37, 70]
    ys, sts, xs = [], [], []
    for L in lens:
        x = torch.randn(1, C, L, generator=gen).to(torch.bfloat16)
        with torch.no_grad():
            y = torch.nn.functional.silu(conv(x)[:, :, :L])
        st = torch.nn.functional.pad(x, (K - L, 0))
        xs.append(x[0].T)
        ys.append(y[0].T)
        sts.append(st[0])
    # continuation: previous K inputs from a slot, then C new tokens (src/cb_tp.py:236-244)
    prev = torch.randn(1, C, K, generator=gen).to(torch.bfloat16)
    xc = torch.randn(1, C, 9, generator=gen).to(torch.bfloat16)
    full = torch.cat([prev, xc], dim=-1)
    with torch.no_grad():
        yc = torch.nn.functional.silu(torch.nn.functional.conv1d(full[:, :, 1:], conv.weight, None,
                                                                 groups=C))
    save("prefill_conv_bf16.npz", dict(w=conv.weight[:, 0], lens=np.asarray(lens, np.int32),
                                       x=torch.cat(xs), y=torch.cat(ys), st=torch.stack(sts),
                                       prev=prev[0], xc=xc[0].T, yc=yc[0].T, stc=full[0, :, -K:]))


def make_norm(ref, seed):
    """Qwen3_5RMSNormGated (TF:175-191) in bf16, decode and prefill row counts."""
    gen = torch.Generator().manual_seed(seed)
    M = ref["M"]
    rows, dv = 96, 128
    mod = M.Qwen3_5RMSNormGated(dv, eps=1e-6)
    with torch.no_grad():
        mod.weight.copy_(1.0 + 0.1 * torch.randn(dv, generator=gen))
    mod = mod.to(torch.bfloat16)
    x = (torch.randn(rows, dv, generator=gen) * 0.5).to(torch.bfloat16)
    z = torch.randn(rows, dv, generator=gen).to(torch.bfloat16)
    with torch.no_grad():
        y = mod(x, z)
    mod32 = M.Qwen3_5RMSNormGated(dv, eps=1e-6)
    with torch.no_grad():
        mod32.weight.copy_(mod.weight.float())
        y32 = mod32(x.float(), z.float())
    save("norm_bf16.npz", dict(w=mod.weight, x=x, z=z, y=y, y32=y32))


def make_gates(ref, seed):
    """beta = sigmoid(b), g = -exp(A_log) * softplus(a + dt_bias) with bf16 parameters, as the HF
    module holds them after .to(bfloat16) (src/cb_engine.py:337-338)."""
    gen = torch.Generator().manual_seed(seed)
    n, Hv = 16, 48
    a = (torch.randn(n, Hv, generator=gen) * 2).to(torch.bfloat16)
    b = (torch.randn(n, Hv, generator=gen) * 2).to(torch.bfloat16)
    A_log = torch.log(torch.empty(Hv).uniform_(0, 16, generator=gen)).to(torch.bfloat16)
    dt_bias = (torch.rand(Hv, generator=gen) * 2 - 1).to(torch.bfloat16)
    beta = b.sigmoid()
    g = -A_log.float().exp() * torch.nn.functional.softplus(a.float() + dt_bias)
    save("gates_bf16.npz", dict(a=a, b=b, A_log=A_log, dt_bias=dt_bias, beta=beta, g=g))


ENGINE_TEXT_CONFIG = dict(
    vocab_size=256, hidden_size=128, intermediate_size=256, num_hidden_layers=4, num_attention_heads=2,
    num_key_value_heads=1, head_dim=64, linear_num_key_heads=1, linear_num_value_heads=2,
    linear_key_head_dim=128, linear_value_head_dim=128, linear_conv_kernel_dim=4,
    layer_types=["linear_attention", "linear_attention", "linear_attention", "full_attention"],
    max_position_embeddings=512, rms_norm_eps=1e-6, attention_bias=False, hidden_act="silu")
ENGINE_VISION_CONFIG = dict(depth=1, hidden_size=32, num_heads=2, intermediate_size=64, out_hidden_size=128)


def tiny_model(seed=0):
    """A tiny random Qwen3.5 (3 GDN : 1 attention, GDN heads of 128) in bf16; weights from HF's
    own init under `seed` with the gate projections scaled up so logits are not near-ties."""
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5Config
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5ForConditionalGeneration
    torch.manual_seed(seed)
    cfg = Qwen3_5Config(text_config=ENGINE_TEXT_CONFIG, vision_config=ENGINE_VISION_CONFIG)
    model = Qwen3_5ForConditionalGeneration(cfg)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if p.dim() == 2 and "visual" not in name:
                p.mul_(4.0)
    return model.to(torch.bfloat16).eval()


def make_engine(ref, seed):
    """Reference CBEngine (src/cb_engine.py:80-355) on a tiny model, on the CPU, with the
    reference's GDN plug-ins (v2 chunk prefill, recurrent_single_step) and HF's gated norm: two
    prompts prefilled into slots 1 and 0, then 5 dense decode steps with both slots active.
    Stores the weights, the tokens, the logits of every step and the GDN slot states."""
    import cb_engine
    M = ref["M"]
    model = tiny_model(seed)
    for m in model.modules():
        if isinstance(m, M.Qwen3_5GatedDeltaNet):
            m.recurrent_gated_delta_rule = ref["rec1"]
            m.chunk_gated_delta_rule = ref["v2"]
    cb_engine.ELEM_CONV = False
    logits = []
    hook = model.lm_head.register_forward_hook(lambda mod, inp, out: logits.append(out.detach().float().clone()))
    eng = cb_engine.CBEngine(model, n_slots=2, t_max=128, device="cpu")
    gen = torch.Generator().manual_seed(seed + 1)
    ids_a = torch.randint(0, 256, (1, 37), generator=gen)
    ids_b = torch.randint(0, 256, (1, 23), generator=gen)
    first_a = eng.prefill(1, ids_a)
    first_b = eng.prefill(0, ids_b)
    pre_logits = [logits[0][0, -1], logits[1][0, -1]]
    gdn_layers = sorted(eng.rec)
    rec_pre = torch.stack([eng.rec[i][:2].clone() for i in gdn_layers])
    conv_pre = torch.stack([eng.conv[i][:2].clone() for i in gdn_layers])
    logits.clear()
    toks = [[first_b, first_a]]
    for _ in range(5):
        toks.append(eng.decode_step([0, 1], toks[-1]))
    hook.remove()
    dec_logits = torch.stack([lg for lg in logits])            # [5, 2, vocab]
    rec_post = torch.stack([eng.rec[i][:2].clone() for i in gdn_layers])
    conv_post = torch.stack([eng.conv[i][:2].clone() for i in gdn_layers])
    sd = {f"w::{k}": v for k, v in model.state_dict().items()}
    save("engine_tiny.npz", dict(ids_a=ids_a[0], ids_b=ids_b[0], tokens=torch.tensor(toks),
                                 pre_logits=torch.stack(pre_logits), dec_logits=dec_logits, rec_pre=rec_pre,
                                 conv_pre=conv_pre, rec_post=rec_post, conv_post=conv_post,
                                 gdn_layers=torch.tensor(gdn_layers), **sd))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", required=True, help="the reference project's src/ directory")
    ap.add_argument("--only", default=None, help="generate one fixture family (e.g. engine)")
    a = ap.parse_args()
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    ref = load_reference(a.reference_src)
    if a.only == "engine":
        make_engine(ref, 8)
        return
    with torch.inference_mode():
        # config 0: fp32, B=2 ragged (256, 190), 4 q/k heads x 64, 8 v heads x 64, zero initial state
        make_chunk(ref, "chunk_c0_f32.npz", [256, 190], 4, 8, 64, torch.float32, 0.0, 0)
        # config 0 shapes with a non-zero initial state N(0, 0.02)
        make_chunk(ref, "chunk_c0init_f32.npz", [100], 4, 8, 64, torch.float32, 0.02, 1)
        # bf16, d=128, ragged edge lengths around the chunk size, GQA ratio 3
        make_chunk(ref, "chunk_bf16.npz", [1, 65, 200], 1, 3, 128, torch.bfloat16, 0.02, 2)
        make_recurrent(ref, 3)
        make_conv(ref, 4)
        make_prefill_conv(ref, 5)
        make_norm(ref, 6)
        make_gates(ref, 7)
        make_engine(ref, 8)


if __name__ == "__main__":
    main()
