#!/usr/bin/env python
"""Benchmark of the GDN hot path on B200.

Headline: one GDN chunk-prefill layer over 16 packed ragged sequences
(lengths U[200,1200], seeded), 16 q/k heads x 128, 48 v heads x 128, chunk 64, bf16 q/k/v,
beta/g on the bf16 grid, fp32 recurrent state N(0, 0.02) read from and written back to a
slot pool.  One step = one call of the slot-indexed chunk-prefill entry point over the whole
batch.  ``value`` = tokens/s with inputs resident in HBM; ``e2e`` = the same through the
public API with the step's inputs copied from pinned host memory and its output copied back,
inside the timed region.

Also reported (``decode``): one 16-slot decode step over 48 GDN layers
(fused conv + gates + recurrence + gated RMSNorm per layer, slot-indexed pools), replayed from a
CUDA graph, in microseconds per step with its HBM roofline.

``--impl reference`` times the reference's own torch prefill (fast_chunk_gated_delta_rule_v2, installed
into oracle/_ref by oracle/install_ref.py; its torch restatement when that is absent) on this host's
cores over a bounded sample of the same workload.

Multi-GPU (torchrun, one rank per GPU): every rank runs its own replica of the same seeded workload
(weak scaling, no collective on the data path); value = all ranks' tokens / max rank time.

Also reported (``model``, BASELINE configs 3/4; ``--no-model`` skips it): the ~27B hybrid (64 layers,
3 GDN : 1 attention, hidden 5120) with random bf16 weights run through the slot engine, serving the
synthetic multi-turn request workload (prompts U[300,700], 1-6 turns of 512 greedy tokens, later
turns append U[50,300] tokens) with continuous batching; ``--requests`` sets the request count (one
per slot by default; the configs name 128 and 512).  With N ranks the model is head-sharded over all
of them (TP = N, the LM head split by vocabulary) with min(64, 16 N) slots (64 at N = 8), and a
``tp_parity`` gate (peer all-reduce bit-exactness, a 4-layer TP model against the single-GPU engine)
runs first.
"""
from __future__ import annotations

import argparse
import importlib
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
PKG = "910b_e2e_accleration_by_codex_b200"
METRIC = "GDN chunk-prefill tokens/s & 16-slot decode-step µs; % of roofline"

HK, HV, D, CHUNK = 16, 48, 128, 64
N_SEQ, LMIN, LMAX = 16, 200, 1200
# algorithmic FLOPs per (value head, 64-token chunk), dense chunk form, d=128:
# 2C^2d*5 (KK^T, QK^T, T.Vb, T.Kb, QK.vn) + 2Cd^2*3 (W.S, Qg.S, Kd^T.vn) + 2C^3/3 (inverse)
FLOP_PER_HEAD_CHUNK = 2 * CHUNK * CHUNK * D * 5 + 2 * CHUNK * D * D * 3 + 2 * CHUNK ** 3 / 3
# decode config 2
DEC_LAYERS, DEC_SLOTS, CONV_K = 48, 16, 4
CONV_DIM = 2 * HK * D + HV * D
# model configs 3/4: ~27B hybrid (48 GDN layers of config-1 shape + 16 GQA attention layers)
MODEL_TEXT_CONFIG = dict(
    vocab_size=248320, hidden_size=5120, intermediate_size=17408, num_hidden_layers=64,
    num_attention_heads=24, num_key_value_heads=4, head_dim=256, linear_num_key_heads=HK,
    linear_num_value_heads=HV, linear_key_head_dim=D, linear_value_head_dim=D, linear_conv_kernel_dim=CONV_K,
    layer_types=["linear_attention", "linear_attention", "linear_attention", "full_attention"] * 16,
    max_position_embeddings=8192, rms_norm_eps=1e-6, attention_bias=False, hidden_act="silu")
MODEL_VISION_CONFIG = dict(depth=1, hidden_size=32, num_heads=2, intermediate_size=64, out_hidden_size=5120)
MODEL_PLEN = (300, 700)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-decode", action="store_true", help="skip the config-2 decode measurement")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end leg")
    ap.add_argument("--decode-layers", type=int, default=DEC_LAYERS,
                    help="GDN layers in the decode leg's step (48 in config 2; fewer for short profiler captures)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="target CPU-baseline sample time")
    ap.add_argument("--f1", action="store_true",
                    help="also time the decode projections of the model leg's shapes: gdn_linear against cuBLAS "
                         "(one GPU), and the row-parallel projection + sum over ranks fused (gdn_linear_allreduce, "
                         "gdn_linear_push + gdn_pull_add_rmsnorm) against cuBLAS + peer all-reduce / NCCL (N > 1)")
    ap.add_argument("--no-model", action="store_true",
                    help="skip the config 3/4 model leg (the ~27B hybrid with random weights through the engine, "
                         "tensor-parallel over all ranks when launched with more than one)")
    ap.add_argument("--requests", type=int, default=0,
                    help="requests of the model leg (0: one per slot; configs 3/4 name 128 / 512)")
    ap.add_argument("--model-turns", type=int, default=6, help="most turns per request of the model leg")
    ap.add_argument("--model-profile", action="store_true", default=True,
                    help="after the model leg, profile graph-replayed decode steps (torch.profiler, device time "
                         "per kernel) and report a per-category breakdown (default on)")
    ap.add_argument("--no-model-profile", dest="model_profile", action="store_false",
                    help="skip the decode breakdown of the model leg")
    ap.add_argument("--model-gen", type=int, default=512, help="greedy tokens per turn of the model leg")
    ap.add_argument("--model-allreduce", choices=["arnorm", "push", "fused", "peer", "nccl"], default="arnorm",
                    help="TP decode sums (TPEngine decode_sum): cuBLAS + one kernel summing the ranks inside the "
                         "residual add / RMSNorm (gdn_allreduce_add_rmsnorm); cuBLAS + push of the partial + "
                         "add / RMSNorm summing the ranks (gdn_push_partial + gdn_pull_add_rmsnorm); the same with "
                         "the tcgen05 projection pushing its tiles (gdn_linear_push); cuBLAS + peer-memory "
                         "all-reduce; or cuBLAS + NCCL")
    return ap.parse_args()


# ----------------------------------------------------------------------------- workload
def make_prefill_workload(seed: int):
    """Config-1 inputs on the host (CPU tensors)."""
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(LMIN, LMAX + 1, (N_SEQ,), generator=g).tolist()
    T = sum(lens)
    q = torch.randn(T, HK, D, generator=g)
    k = torch.randn(T, HK, D, generator=g)
    q = (q / q.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    k = (k / k.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    v = torch.randn(T, HV, D, generator=g).to(torch.bfloat16)
    beta = torch.sigmoid(torch.randn(T, HV, generator=g)).to(torch.bfloat16).float()
    gg = (-(0.01 + 0.99 * torch.rand(T, HV, generator=g))).to(torch.bfloat16).float()
    init = torch.randn(N_SEQ, HV, D, D, generator=g) * 0.02
    cu = torch.tensor([0] + np.cumsum(lens).tolist(), dtype=torch.int32)
    return dict(lens=lens, T=T, q=q, k=k, v=v, g=gg, beta=beta, init=init, cu=cu)


def workload_config(w):
    """The config block both arms print for the config-1 workload."""
    return {"workload": "config1: GDN chunk prefill, 16 packed ragged seqs U[200,1200], Hk=16 Hv=48 dk=dv=128, "
                        "chunk 64, bf16 q/k/v, fp32 state N(0,0.02) from a slot pool",
            "total_tokens_per_gpu": w["T"]}


def prefill_flops(lens):
    chunks = sum(math.ceil(L / CHUNK) for L in lens)
    return chunks * HV * FLOP_PER_HEAD_CHUNK, chunks


def prefill_bytes(w):
    """Algorithmic HBM bytes per launch: q,k (un-repeated), v, beta, g in; o out; state r+w."""
    T = w["T"]
    per_tok = (2 * HK * D + HV * D) * 2 + 2 * HV * 4 + HV * D * 2
    return T * per_tok + 2 * N_SEQ * HV * D * D * 4


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampled every 100 ms while the benchmark runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(gpu_index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n_, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(n_)
        if not sm:
            return None
        busy = [s for s in sm if s > 0.5 * max(sm)] or sm
        return {"sm_mhz": statistics.median(busy), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------- distributed
def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        if args.impl == "ours":
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local))
        else:
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def allreduce_max(x: float, world: int) -> float:
    if world <= 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def allreduce_min(x: float, world: int) -> float:
    if world <= 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return float(t.item())


def allreduce_sum(x: float, world: int) -> float:
    if world <= 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# ----------------------------------------------------------------------------- CPU legs
def cpu_kind():
    """'reference' when the reference's own modules are installed in oracle/_ref (oracle/install_ref.py),
    else 'port' (the torch restatement oracle/gdn_torch_cpu.py, pinned to the same golden vectors)."""
    from oracle import ref_cpu
    return "reference" if ref_cpu.available() else "port"


def cpu_prefill_sample(w, seconds: float):
    """The reference's prefill path on the host cores: its own fast_chunk_gated_delta_rule_v2
    (src/gdn_chunk_fast2.py:11-62, from oracle/_ref) -- or, without it, the torch restatement -- in
    the reference's dtypes, one sequence per call as TPEngine.prefill does, over the workload's
    sequences in order (repeated passes) until ~`seconds` elapse."""
    from oracle import gdn_torch_cpu as TC
    from oracle import ref_cpu
    if ref_cpu.available():
        def rule(q, k, v, g, b, init):
            return ref_cpu.chunk_prefill(q, k, v, g, b, init)
        what = "the reference's own fast_chunk_gated_delta_rule_v2 (src/gdn_chunk_fast2.py)"
    else:
        def rule(q, k, v, g, b, init):
            return TC.chunk_gated_delta_rule(q, k, v, g, b, 64, init, True, True)
        what = "the torch restatement of src/gdn_chunk_fast2.py"
    r = HV // HK
    nseq = len(w["lens"])
    toks, used, el = 0, 0, 0.0
    t0 = time.perf_counter()
    with torch.inference_mode():
        while used == 0 or el < seconds:
            b = used % nseq
            L = int(w["lens"][b])
            s, e = int(w["cu"][b]), int(w["cu"][b + 1])
            q = w["q"][s:e].repeat_interleave(r, dim=1)[None]
            k = w["k"][s:e].repeat_interleave(r, dim=1)[None]
            rule(q, k, w["v"][s:e][None], w["g"][s:e][None], w["beta"][s:e].to(torch.bfloat16)[None],
                 w["init"][b][None])
            toks += L
            used += 1
            el = time.perf_counter() - t0
    return toks / el, (f"{used} sequence calls ({used / nseq:.1f} passes over the {nseq} sequences, {toks} tokens), "
                       f"one call per sequence of {what}"), el


def cpu_decode_sample(seconds: float):
    """The reference's decode layer on the host cores: CBEngine._gdn's operators (src/cb_engine.py:
    318-352: elem conv update, split, gates, l2norm, recurrent_single_step, gated RMSNorm) for 16
    slots -- the reference's own functions from oracle/_ref, or without them the torch restatement
    (with index_select / index_copy_ on the pools) -- repeated over fresh layers until ~`seconds`
    elapse; returns µs per 48-layer step."""
    from oracle import gdn_torch_cpu as TC
    from oracle import ref_cpu
    own = ref_cpu.available()
    g = torch.Generator(device="cpu").manual_seed(1234)
    n, bf = DEC_SLOTS, torch.bfloat16
    layers, el = 0, 0.0
    t0 = time.perf_counter()
    with torch.inference_mode():
        while True:
            mixed = torch.randn(n, CONV_DIM, generator=g).to(bf)
            z = torch.randn(n, HV, D, generator=g).to(bf)
            a, b = torch.randn(n, HV, generator=g).to(bf), torch.randn(n, HV, generator=g).to(bf)
            A_log = torch.log(torch.empty(HV).uniform_(1, 16, generator=g))
            dt_bias = torch.rand(HV, generator=g) * 2 - 1
            conv_w = (torch.rand(CONV_DIM, CONV_K, generator=g) - 0.5).to(bf)
            conv_pool = torch.randn(n, CONV_DIM, CONV_K, generator=g).to(bf)
            rec_pool = torch.randn(n, HV, D, D, generator=g) * 0.02
            norm_w = (1 + 0.1 * torch.randn(D, generator=g)).to(bf)
            slot = torch.randperm(n, generator=g)
            t_l = time.perf_counter()
            if own:
                ref_cpu.decode_layer(mixed, z, a, b, A_log, dt_bias, conv_w, conv_pool, rec_pool, norm_w, HK, HV, D)
            else:
                TC.decode_layer(mixed, z, a, b, A_log, dt_bias, conv_w, conv_pool, rec_pool, slot, norm_w, HK, HV,
                                D)
            el += time.perf_counter() - t_l
            layers += 1
            if time.perf_counter() - t0 >= seconds:
                break
    what = ("the reference's own elem_conv_update / recurrent_single_step with HF's gated norm" if own
            else "the torch restatement")
    return el / layers * DEC_LAYERS * 1e6, (f"{layers} layers of 16 slots of {what} (src/cb_engine.py:318-352), "
                                            f"timed per layer, x {DEC_LAYERS}")


def cpu_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def run_reference(args, world, rank):
    """--impl reference: the reference's own torch prefill (from oracle/_ref; the restatement when it is
    absent) on the host cores, every thread it can use."""
    if rank != 0:
        return
    w = make_prefill_workload(args.seed)
    torch.set_num_threads(cpu_cores())
    for _ in range(max(0, min(args.warmup, 1))):
        cpu_prefill_sample(w, 0.0)
    vals, samples, secs = [], None, 0.0
    per_step = max(2.0, min(20.0, 120.0 / max(1, args.steps)))
    for _ in range(args.steps):
        v, samples, el = cpu_prefill_sample(w, per_step)
        vals.append(v)
        secs += el
    value = statistics.median(vals)
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 * w["T"] / value, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "impl": "reference",
            "config": dict(workload_config(w), parallelism="cpu"),
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cpu_cores(), "kind": cpu_kind(),
                             "sample": samples},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- GPU legs
def time_events(fn, steps, stream):
    """Run fn() `steps` times on `stream`; returns per-step CUDA-event durations in ms."""
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for a, b in evs:
        a.record(stream)
        fn()
        b.record(stream)
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in evs]


def load_traffic():
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


def measured_peaks():
    """(HBM GB/s, bf16 TFLOP/s burst, source) from MEASURED_PEAKS.json, else the pool's fallback."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
        return peaks.get("hbm_gbs", 6650.0), peaks.get("bf16_tflops", 1590.0), "of measured"
    except (OSError, ValueError):
        return 6650.0, 1590.0, "of fallback"


def run_ours(args, world, rank, local):
    ops = importlib.import_module(f"{PKG}.ops")
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except (OSError, ValueError):
        pass
    hbm_peak = peaks.get("hbm_gbs", 6650.0)
    tc_peak = peaks.get("bf16_tflops", 1590.0)
    peak_src = "of measured" if peaks else "of fallback"
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream()
    w = make_prefill_workload(args.seed)          # every replica runs the same seeded workload
    T = w["T"]
    # ---- device-resident inputs
    q, k, v = w["q"].to(dev), w["k"].to(dev), w["v"].to(dev)
    g, beta = w["g"].to(dev), w["beta"].to(dev)
    cu = w["cu"].to(dev)
    pool = w["init"].to(dev).contiguous()
    slot = torch.arange(N_SEQ, dtype=torch.int32, device=dev)
    use_init = torch.ones(N_SEQ, dtype=torch.int32, device=dev)
    out = torch.empty(T, HV, D, dtype=torch.bfloat16, device=dev)

    def step():
        ops.chunk_prefill_varlen(q, k, v, g, beta, cu, pool, slot, use_init, True, out=out)

    clocks = ClockSampler(local)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    durs = time_events(step, args.steps, stream)
    barrier(world)
    torch.cuda.synchronize()
    ms = sum(durs) / len(durs)
    ms_max = allreduce_max(ms, world)
    tot_tokens = allreduce_sum(float(T), world)
    value = tot_tokens / (ms_max / 1e3)

    # ---- e2e through the public API with pinned host buffers
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(ops, w, q, k, v, g, beta, cu, pool, slot, use_init, out, args, world, stream, tot_tokens)

    # ---- decode (config 2): 48 layers x 16 slots, CUDA-graph replay
    decode = None
    if not args.no_decode:
        decode = run_decode(ops, dev, args, world, hbm_peak, peak_src)
    clk = clocks.stop()

    flops, chunks = prefill_flops(w["lens"])
    achieved_tflops = flops / (ms / 1e3) / 1e12
    traffic = load_traffic().get("gdn_chunk_prefill")
    algo_bytes = prefill_bytes(w)
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded; config-1 distributions; no dataset or weights needed)",
        "config": dict(workload_config(w), chunks_per_head=chunks,
                       l2=f"inputs larger than L2 ({algo_bytes / 1e6:.0f} MB touched per step > 126 MB)",
                       parallelism=f"replicas x{world}" if world > 1 else "single GPU"),
        "roofline": {"bound": "tensor", "achieved": achieved_tflops, "peak": tc_peak, "unit": "TFLOP/s",
                     "frac": achieved_tflops / tc_peak, "peak_source": peak_src + " (bf16 burst)",
                     "traffic": traffic, "algorithmic_flops_per_launch": flops,
                     "algorithmic_bytes_per_launch": algo_bytes,
                     "hbm_frac": algo_bytes / (ms / 1e3) / 1e9 / hbm_peak},
        "e2e": e2e,
        "gpu_launches": args.steps * (2 if e2e is not None else 1),
        "clocks": clk,
    }
    if decode is not None:
        line["decode"] = decode
        line["gpu_launches"] += decode["gpu_launches"]
    if args.f1:
        line["f1"] = run_f1(world, rank)
    if not args.no_model:
        try:
            line["model"] = run_model(args, world, rank, local)
        except Exception as e:  # the headline stands on its own; report why the model leg is missing
            line["model"] = {"error": f"{type(e).__name__}: {e}"[:300]}
    if rank == 0 and world == 1 and not args.no_cpu:
        torch.set_num_threads(cpu_cores())
        v_cpu, sample, el = cpu_prefill_sample(w, args.cpu_seconds)
        line["cpu_baseline"] = {"value": v_cpu, "unit": "tokens/s", "cores": cpu_cores(), "kind": cpu_kind(),
                                "sample": sample + f", {el:.1f} s"}
        if decode is not None:
            us_cpu, dsample = cpu_decode_sample(max(2.0, args.cpu_seconds / 3))
            line["decode"]["cpu_baseline"] = {"us_per_step": us_cpu, "cores": cpu_cores(), "kind": cpu_kind(),
                                              "sample": dsample}
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_f1(world, rank, iters=64):
    """Decode projections of the model leg (``model_slots(world)`` tokens, hidden 5,120) timed on the
    device: CUDA graphs of ``iters`` calls, weights rotated through more than L2, max over ranks.
    One GPU: gdn_linear vs cuBLAS for the TP-1 shapes, against the HBM roofline (weight bytes).
    N > 1: per row-parallel shape (out_proj / o_proj k = 6,144 / N, down_proj k = 17,408 / N) the
    fused projection + sum (gdn_linear_allreduce), its push / pull split with the residual add +
    RMSNorm, and cuBLAS + peer all-reduce (+ gdn_add_rmsnorm) / cuBLAS + NCCL; the roofline target of a
    fused call is the slower of its weight bytes over the HBM peak and the bytes it sends over NVLink
    ((N - 1) x tokens x 5,120 x 2) over 770 GB/s per direction."""
    ops = importlib.import_module(f"{PKG}.ops")
    dev = torch.device("cuda", torch.cuda.current_device())
    n = model_slots(world)
    H = MODEL_TEXT_CONFIG["hidden_size"]
    hbm = measured_peaks()[0]
    out = {"tokens": n, "timing": "CUDA graph of %d calls, device time per call, max over ranks" % iters,
           "hbm_peak_gbs": hbm, "nvlink_gbs": 770.0, "shapes": []}

    def gtime(fn):
        fn()
        torch.cuda.synchronize()
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        g = torch.cuda.CUDAGraph()
        st = torch.cuda.Stream()
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            with torch.cuda.graph(g, stream=st):
                for _ in range(iters):
                    fn()
        torch.cuda.current_stream().wait_stream(st)
        best = 1e30
        for _ in range(3):
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            g.replay()
            e1.record()
            torch.cuda.synchronize()
            best = min(best, allreduce_max(e0.elapsed_time(e1) * 1e3 / iters, world))
        del g
        return best

    def rotating(n_out, k):
        copies = max(2, int(3e8 // (n_out * k * 2)) + 1)
        Ws = [torch.randn(n_out, k, device=dev, dtype=torch.bfloat16) * 0.02 for _ in range(copies)]
        it = iter(range(1 << 30))
        return Ws, (lambda: Ws[next(it) % copies])

    if world == 1:
        shapes = [("o_proj / out_proj", H, 6144), ("down_proj", H, 17408), ("gate|up", 2 * 17408, H),
                  ("GDN in_proj qkv|z|b|a", 16488, H), ("attention q|gate|k|v", 14336, H)]
        for name, n_out, k in shapes:
            Ws, nxt = rotating(n_out, k)
            x = torch.randn(n, k, device=dev, dtype=torch.bfloat16)
            y = torch.empty(n, n_out, device=dev, dtype=torch.bfloat16)
            t_cub = gtime(lambda: torch.matmul(x, nxt().t(), out=y))
            t_gdn = gtime(lambda: ops.linear(x, nxt(), out=y))
            wb = n_out * k * 2
            plan = ops.linear_plan(n, n_out, k)
            out["shapes"].append({"name": name, "n_out": n_out, "k": k, "weight_bytes": wb, "splits": plan["splits"],
                                  "gdn_linear_us": t_gdn, "cublas_us": t_cub,
                                  "gdn_linear_hbm_frac": wb / (t_gdn * 1e-6) / 1e9 / hbm,
                                  "cublas_hbm_frac": wb / (t_cub * 1e-6) / 1e9 / hbm})
            del Ws
        return out
    tp_mod = importlib.import_module(f"{PKG}.tp")
    import torch.distributed as dist
    fl = tp_mod.PeerLinearAllReduce(n, H, dev)
    ar = tp_mod.PeerAllReduce(n * H, dev)
    arn = tp_mod.PeerAllReduceAddNorm(n, H, dev)
    nw = torch.ones(H, device=dev, dtype=torch.bfloat16)
    try:
        for name, k in (("o_proj / out_proj", 6144 // world), ("down_proj", 17408 // world)):
            Ws, nxt = rotating(H, k)
            x = torch.randn(n, k, device=dev, dtype=torch.bfloat16)
            y = torch.empty(n, H, device=dev, dtype=torch.bfloat16)
            res = torch.zeros(n, H, device=dev, dtype=torch.bfloat16)
            nrm = torch.empty(n, H, device=dev, dtype=torch.bfloat16)

            def cub_ar_norm():
                torch.matmul(x, nxt().t(), out=y)
                ar(y)
                ops.add_rmsnorm(res, y, nw, 1e-6, out=nrm)

            def push_pull():
                fl.push(x, nxt())
                fl.pull_add_rmsnorm(res, nw, 1e-6, out=nrm)

            def cub_arnorm():
                torch.matmul(x, nxt().t(), out=y)
                arn(res, y, nw, 1e-6, out=nrm)

            def cub_push_pull():
                torch.matmul(x, nxt().t(), out=y)
                fl.push_partial(y)
                fl.pull_add_rmsnorm(res, nw, 1e-6, out=nrm)

            t = {"cublas": gtime(lambda: torch.matmul(x, nxt().t(), out=y)),
                 "cublas_peer_allreduce": gtime(lambda: (torch.matmul(x, nxt().t(), out=y), ar(y))),
                 "cublas_nccl": gtime(lambda: (torch.matmul(x, nxt().t(), out=y), dist.all_reduce(y))),
                 "fused_gdn_linear_allreduce": gtime(lambda: fl(x, nxt())),
                 "cublas_peer_allreduce_add_rmsnorm": gtime(cub_ar_norm),
                 "push_pull_add_rmsnorm": gtime(push_pull),
                 "cublas_push_pull_add_rmsnorm": gtime(cub_push_pull),
                 "cublas_allreduce_add_rmsnorm": gtime(cub_arnorm)}
            wb = H * k * 2
            link = (world - 1) * n * H * 2
            target = max(wb / (hbm * 1e9), link / 770e9) * 1e6
            out["shapes"].append({"name": name, "n_out": H, "k": k, "weight_bytes_per_rank": wb,
                                  "nvlink_bytes_out_per_rank": link, "roofline_target_us": target,
                                  "splits_fused": ops.linear_plan(n, H, k, world=world)["splits"],
                                  "splits_push": ops.linear_plan(n, H, k)["splits"],
                                  "us": t, "fused_frac_of_roofline": target / t["fused_gdn_linear_allreduce"]})
            del Ws
    finally:
        fl.close()
        ar.close()
        arn.close()
    return out


def model_slots(world):
    """Slot count of the model leg: 16 on one GPU; with TP over N ranks min(64, 16 N), 64 at N = 8."""
    return 16 if world <= 1 else min(64, 16 * world)


def build_model(text_cfg, dev, seed):
    """Random-init bf16 Qwen3.5 (identical on every rank for the same seed)."""
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5Config
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5ForConditionalGeneration
    torch.manual_seed(seed)
    cfg = Qwen3_5Config(text_config=text_cfg, vision_config=MODEL_VISION_CONFIG)
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with torch.device(dev):
            model = Qwen3_5ForConditionalGeneration(cfg)
    finally:
        torch.set_default_dtype(prev)
    return model.to(torch.bfloat16).eval()


def model_decode_bytes(model, eng):
    """(fixed bytes, bytes per context token) one decode step of ``eng`` moves on this rank: every
    local weight of the decoder layers, the final norm and the (local) LM head, and every slot's GDN
    recurrent state (read + write) and conv state; plus, per slot and attention layer, the KV rows
    0..ctx that the step reads."""
    lm = model.model.language_model
    w = sum(p.numel() * p.element_size() for n, p in lm.named_parameters() if "embed_tokens" not in n)
    w += sum(p.numel() * p.element_size() for p in model.lm_head.parameters())
    st = sum(t[:eng.N].numel() * t.element_size() * 2 for t in eng.rec.values())
    st += sum(t[:eng.N].numel() * t.element_size() * 2 for t in eng.conv.values())
    kv = sum(t.shape[1] * t.shape[3] * 2 * t.element_size() for t in eng.kv_k.values())
    return w + st, kv


def model_prefill_flops(model, tokens, seqs):
    """Approximate prefill FLOPs on this rank: 2 x (local matmul weights) per token, the GDN chunk
    algebra (per 64-token chunk and local value head) and causal attention (QK^T and PV over the
    causal half, per local head)."""
    lm = model.model.language_model
    cfg = model.config.text_config
    mat = sum(p.numel() for n, p in lm.named_parameters() if p.dim() == 2 and "embed_tokens" not in n)
    f = 2.0 * mat * tokens + 2.0 * sum(p.numel() for p in model.lm_head.parameters()) * len(seqs)
    for layer, kind in zip(lm.layers, cfg.layer_types):
        if kind == "full_attention":
            at = layer.self_attn
            nh = at.q_proj.weight.shape[0] // (2 * at.head_dim)
            f += sum(2.0 * L * L * at.head_dim * nh for L in seqs)
        else:
            hv = layer.linear_attn.num_v_heads
            f += sum(math.ceil(L / CHUNK) for L in seqs) * hv * FLOP_PER_HEAD_CHUNK
    return f


def tp_parity(world, rank, local):
    """Correctness gate of the tensor-parallel path, run before the timed model leg on N > 1 ranks.

    (1) The peer-memory all-reduce on the decode size [slots, hidden] bf16: bit-identical to the fp32
        sum of all ranks' inputs in rank order rounded once to bf16, and within NCCL's own bf16
        roundings (world - 1 along its ring) of NCCL's all-reduce.
    (3) f1, the o_proj-shaped projection fused with its sum (gdn_linear_allreduce): bit-identical to
        the rank-order sum of each rank's gdn_linear partial with the same split count, and within
        bf16 tolerance of the rank-order sum of cuBLAS partials; (4) the sum fused into the residual
        add + RMSNorm (gdn_allreduce_add_rmsnorm): bit-identical to the peer all-reduce, the add and
        gdn_rmsnorm.
    (2) A 4-layer model with the config-3 shapes (3 GDN : 1 attention, 24 q / 4 KV heads, so TP 8
        replicates KV heads; the LM head split by vocabulary): the TP engine over all ranks against
        the single-GPU engine on rank 0 with the same weights and feed (three prompts, then two
        teacher-forced decode steps): the logits of the prefill and of each decode step, gathered from
        the ranks' vocabulary slices, and the GDN slot states gathered from the ranks' head shards,
        within the engine test's bf16 tolerance (2e-2 + 2e-2 max|ref|)."""
    import torch.distributed as dist
    eng_mod = importlib.import_module(f"{PKG}.engine")
    tp_mod = importlib.import_module(f"{PKG}.tp")
    dev = torch.device("cuda", local)
    res = {}
    # ---- (1) peer all-reduce
    slots = model_slots(world)
    H = MODEL_TEXT_CONFIG["hidden_size"]
    xs = [torch.randn(slots, H, generator=torch.Generator().manual_seed(900 + r)).to(torch.bfloat16)
          for r in range(world)]
    ref = torch.zeros(slots, H)
    for x in xs:
        ref += x.float()
    ref = ref.to(torch.bfloat16).to(dev)
    ar = tp_mod.PeerAllReduce(slots * H, dev)
    y = xs[rank].to(dev).clone()
    ar(y)
    z = xs[rank].to(dev).clone()
    dist.all_reduce(z)
    torch.cuda.synchronize()
    ar_err = int(ar.err.item())
    ar.close()
    bit = bool(torch.equal(y, ref)) and ar_err == 0
    # NCCL rounds its partial sums to bf16 along its ring (world - 1 roundings): compare within that
    # many bf16 steps of the inputs' magnitude sum
    mag = torch.zeros(slots, H)
    for x in xs:
        mag += x.float().abs()
    dz = (z.float() - ref.float()).abs()
    nccl_ok = bool((dz <= world * 2.0 ** -8 * mag.to(dev)).all())
    res["allreduce"] = {"shape": [slots, H], "bitexact_vs_fp32_rank_order": bit, "err_flag": ar_err,
                        "nccl_within_bf16_roundings": nccl_ok, "max_abs_vs_nccl": float(dz.max().item())}
    # ---- (3) f1: the row-parallel projection fused with the sum (o_proj shape) and (4) the sum fused
    # into the residual add + RMSNorm
    ops = importlib.import_module(f"{PKG}.ops")
    k = 6144 // world
    gx = torch.Generator().manual_seed(950 + rank)
    xf = torch.randn(slots, k, generator=gx).to(torch.bfloat16).to(dev)
    wf = (torch.randn(H, k, generator=gx) / k ** 0.5).to(torch.bfloat16).to(dev)
    fl = tp_mod.PeerLinearAllReduce(slots, H, dev)
    yf = fl(xf, wf)
    S = ops.linear_plan(slots, H, k, world=world)["splits"]

    def rank_sum(part):
        parts = [torch.empty_like(part) for _ in range(world)]
        dist.all_gather(parts, part)
        acc = torch.zeros(part.shape, dtype=torch.float32, device=dev)
        for p_ in parts:
            acc += p_.float()
        return acc.to(torch.bfloat16)

    exp_f = rank_sum(ops.linear(xf, wf, splits=S))
    cub = rank_sum(torch.nn.functional.linear(xf, wf))
    mag = rank_sum((xf.float().abs() @ wf.float().abs().t()).to(torch.bfloat16)).float()
    torch.cuda.synchronize()
    f_err = int(fl.err.item())
    fl.close()
    f_bit = bool(torch.equal(yf, exp_f)) and f_err == 0
    f_close = bool(((yf.float() - cub.float()).abs() <= 2 ** -6 * mag + 1e-2).all())
    res["fused_linear_allreduce"] = {"shape": [slots, H, k], "splits": S, "err_flag": f_err,
                                     "bitexact_vs_rank_sum_of_gdn_linear": f_bit,
                                     "within_bf16_of_cublas_rank_sum": f_close}
    arn = tp_mod.PeerAllReduceAddNorm(slots, H, dev)
    par = tp_mod.PeerAllReduce(slots * H, dev)
    gh = torch.Generator().manual_seed(960)
    hs_all = (torch.randn(world, slots, H, generator=gh) * 3).to(torch.bfloat16)
    res0 = (torch.randn(slots, H, generator=gh) * 2).to(torch.bfloat16).to(dev)
    nw = (torch.randn(H, generator=gh) * 0.1).to(torch.bfloat16).to(dev)
    h = hs_all[rank].to(dev)
    hsum = h.clone()
    par(hsum)
    ref_x = res0 + hsum
    ref_o = ops.rmsnorm(ref_x, nw, 1e-6)
    xres = res0.clone()
    out_o = arn(xres, h, nw, 1e-6)
    torch.cuda.synchronize()
    a_err = int(arn.err.item())
    arn.close()
    par.close()
    a_bit = bool(torch.equal(xres, ref_x)) and bool(torch.equal(out_o, ref_o)) and a_err == 0
    res["allreduce_add_rmsnorm"] = {"shape": [slots, H], "err_flag": a_err,
                                    "bitexact_vs_allreduce_add_rmsnorm": a_bit}
    bit = bit and f_bit and f_close and a_bit
    # ---- (2) 4-layer model
    cfg = dict(MODEL_TEXT_CONFIG, num_hidden_layers=4,
               layer_types=["linear_attention", "linear_attention", "linear_attention", "full_attention"])
    g = torch.Generator().manual_seed(77)
    prompts = [torch.randint(0, cfg["vocab_size"], (1, L), generator=g) for L in (157, 64, 301)]
    feed = [torch.randint(0, cfg["vocab_size"], (3,), generator=g).tolist() for _ in range(2)]

    def run(eng, head):
        logits = []
        hk = head.register_forward_hook(lambda m, i, o: logits.append(o.detach().float()))
        eng.prefill_batch([0, 1, 2], prompts)
        for t in feed:
            eng.decode_step([0, 1, 2], t)
        hk.remove()
        return logits, [eng.rec[i][:3].clone() for i in sorted(eng.rec)]

    ref_logits = ref_states = None
    if rank == 0:
        full = build_model(cfg, dev, seed=4242)
        e1 = eng_mod.CBEngine(full, 3, 512, dev, graph_decode=False)
        ref_logits, ref_states = run(e1, full.lm_head)
        del e1, full
        torch.cuda.empty_cache()
    model = build_model(cfg, dev, seed=4242)
    tp_mod.shard_model(model, rank, world, vocab_parallel=True)
    eng = tp_mod.TPEngine(model, 3, 512, dev, world, graph_decode=False)
    logits, states = run(eng, model.lm_head.lin)            # this rank's vocabulary slice
    eng.check_errors()
    eng.close()
    full_logits, full_states = [], []
    for lg in logits:
        parts = [torch.empty_like(lg) for _ in range(world)]
        dist.all_gather(parts, lg.contiguous())
        full_logits.append(torch.cat(parts, dim=-1))
    for st in states:
        parts = [torch.empty_like(st) for _ in range(world)]
        dist.all_gather(parts, st.contiguous())
        full_states.append(torch.cat(parts, dim=1))          # value heads in rank order
    ok = bit
    if rank == 0:
        le = [float((a - b).abs().max().item()) for a, b in zip(full_logits, ref_logits)]
        lt = [2e-2 + 2e-2 * float(b.abs().max().item()) for b in ref_logits]
        se = max(float((a - b).abs().max().item()) for a, b in zip(full_states, ref_states))
        st_tol = 2e-2 + 2e-2 * max(float(b.abs().max().item()) for b in ref_states)
        ok = ok and len(le) == 3 and all(e <= t for e, t in zip(le, lt)) and se <= st_tol
        res["model"] = {"layers": 4, "hidden": cfg["hidden_size"], "vocab_parallel_head": True,
                        "prefill_logits_err": le[0], "decode_logits_err": le[1:], "logits_tol": lt,
                        "gdn_state_err": se, "gdn_state_tol": st_tol}
    flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=dev)
    dist.broadcast(flag, 0)
    res["ok"] = bool(flag.item())
    del model, eng
    torch.cuda.empty_cache()
    return res


def decode_breakdown(eng, slots, steps=8, ctx=500):
    """Device time per kernel category of graph-replayed decode steps (torch.profiler's CUPTI kernel
    records; no replay, so it is safe on every rank of a TP run).  Every slot holds a ``ctx``-token
    prompt; returns per-step milliseconds and kernel counts by category and the top kernels."""
    from torch.profiler import ProfilerActivity, profile
    V = MODEL_TEXT_CONFIG["vocab_size"]
    g = torch.Generator().manual_seed(7)
    all_slots = list(range(slots))
    toks = eng.prefill_batch(all_slots, [torch.randint(0, V, (1, ctx), generator=g) for _ in all_slots])
    for _ in range(3):
        toks = eng.decode_step(all_slots, toks)
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(steps):
            toks = eng.decode_step(all_slots, toks)
        torch.cuda.synchronize()
    for s_ in all_slots:
        eng.free(s_)
    cats = [("gdn decode layer (decode_prep + decode_state)", ("decode_prep_kernel", "decode_state_kernel")),
            ("attention decode (attn_decode + combine)", ("attn_decode_kernel", "attn_combine_kernel")),
            ("peer all-reduce (gdn_allreduce)", ("allreduce_bf16_kernel",)),
            ("tcgen05 projection (gdn_linear / gdn_linear_push)", ("linear_kernel",)),
            ("residual add + RMSNorm (gdn_add_rmsnorm / gdn_pull_add_rmsnorm)", ("add_rmsnorm_kernel",)),
            ("NCCL", ("nccl",)),
            ("layer RMSNorm (gdn_rmsnorm)", ("rmsnorm_kernel",)),
            ("GEMM (cuBLAS)", ("gemm", "nvjet", "xmma", "cublas", "cutlass", "gemv", "splitkreduce")),
            ("elementwise / copy / reduce (torch)", ("elementwise", "vectorized", "reduce", "copy", "cat", "index",
                                                     "fill", "softmax", "arange", "where", "unrolled"))]
    by = {name: [0.0, 0] for name, _ in cats}
    by["other"] = [0.0, 0]
    rows = []
    for e in prof.key_averages():
        t = float(getattr(e, "device_time_total", 0.0) or 0.0)
        if t <= 0 or e.count == 0:
            continue
        key = e.key
        low = key.lower()
        cat = next((name for name, pats in cats if any(p_ in low for p_ in pats)), "other")
        by[cat][0] += t
        by[cat][1] += e.count
        rows.append((t, e.count, key))
    rows.sort(reverse=True)
    total = sum(v[0] for v in by.values())
    return {"steps_profiled": steps, "context_tokens": ctx, "slots": slots,
            "device_ms_per_step": total / 1e3 / steps,
            "by_category_ms_per_step": {k: round(v[0] / 1e3 / steps, 4) for k, v in by.items() if v[1]},
            "kernels_per_step": {k: v[1] / steps for k, v in by.items() if v[1]},
            "top_kernels": [{"name": k[:90], "ms_per_step": round(t / 1e3 / steps, 4), "calls_per_step": c / steps}
                            for t, c, k in rows[:12]],
            "how": "torch.profiler CUDA kernel records of graph-replayed decode steps, device time summed per name"}


def run_model(args, world, rank, local):
    """Model leg (configs 3/4): the random-init ~27B hybrid through the slot engine, serving the
    synthetic multi-turn request workload with continuous batching (serve.run_requests)."""
    eng_mod = importlib.import_module(f"{PKG}.engine")
    tp_mod = importlib.import_module(f"{PKG}.tp")
    serve = importlib.import_module(f"{PKG}.serve")
    dev = torch.device("cuda", local)
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except (OSError, ValueError):
        pass
    hbm_peak = peaks.get("hbm_gbs", 6650.0)
    tc_peak = peaks.get("bf16_tflops_sustained", 1400.0)
    peak_src = "of measured" if peaks else "of fallback"
    parity = tp_parity(world, rank, local) if world > 1 else None
    t_build = time.time()
    model = build_model(MODEL_TEXT_CONFIG, dev, seed=1234)   # identical full model on every rank
    params = sum(p.numel() for n, p in model.named_parameters() if "visual" not in n)
    if world > 1:
        tp_mod.shard_model(model, rank, world, vocab_parallel=True)
    # as the reference's runs do before building the engine (src/cb_run.py:158): the layer RMSNorms
    # and the GDN plug-in points of the HF modules go to this library's kernels
    importlib.import_module(f"{PKG}.patch").patch_model(model, fast_gdn=True, gdn_v2=True)
    torch.cuda.empty_cache()
    slots = model_slots(world)
    n_req = args.requests if args.requests > 0 else slots
    reqs = serve.synthetic_requests(n_req, MODEL_TEXT_CONFIG["vocab_size"], seed=4321, max_turns=args.model_turns)
    bucket = eng_mod.GRAPH_BUCKET
    t_max = -(-(serve.max_context(reqs, args.model_gen) + 1) // bucket) * bucket
    eng = (tp_mod.TPEngine(model, slots, t_max, dev, world, graph_decode=True, decode_sum=args.model_allreduce)
           if world > 1
           else eng_mod.CBEngine(model, slots, t_max, dev, graph_decode=True))
    build_s = time.time() - t_build
    # warm-up: single-turn requests of the same prompt lengths through the same loop (GEMM shapes,
    # cuBLAS heuristics, kernel loading), a few tokens each
    warm = serve.synthetic_requests(slots, MODEL_TEXT_CONFIG["vocab_size"], seed=99, max_turns=1)
    serve.run_requests(eng, warm, gen_tokens=8)
    torch.cuda.synchronize()
    barrier(world)
    fixed_b, ctx_b = model_decode_bytes(model, eng)
    acc = {"dec_bytes": 0.0, "pre_flops": 0.0}

    def on_step(kind, dt, info):
        if kind == "decode":
            acc["dec_bytes"] += fixed_b + ctx_b * sum(c + 1 for c in info["ctx"])
        else:
            acc["pre_flops"] += model_prefill_flops(model, info["tokens"], info["seqs"])

    st = serve.run_requests(eng, reqs, gen_tokens=args.model_gen, on_step=on_step)
    torch.cuda.synchronize()
    barrier(world)
    breakdown = decode_breakdown(eng, slots) if args.model_profile else None
    eng.check_errors()
    if world > 1:
        eng.close()                              # graphs and peer buffers go before the process group
    else:
        eng._graphs.clear()
        eng._graph_out.clear()
    mk = allreduce_max(st["makespan_s"], world)
    dec_s = allreduce_max(st["decode_s"], world)
    pre_s = allreduce_max(st["prefill_s"], world)
    dec_gbs = acc["dec_bytes"] / st["decode_s"] / 1e9 if st["decode_s"] > 0 else 0.0
    pre_tf = acc["pre_flops"] / st["prefill_s"] / 1e12 if st["prefill_s"] > 0 else 0.0
    dec_gbs = allreduce_min(dec_gbs, world)
    pre_tf = allreduce_min(pre_tf, world)
    del eng, model
    torch.cuda.empty_cache()
    out = {"config": "config 3" if world <= 1 else f"config 4 (TP {world})",
           "params": params, "layers": MODEL_TEXT_CONFIG["num_hidden_layers"], "tp": world, "slots": slots,
           "requests": n_req, "requests_in_config": 128 if world <= 1 else 512,
           "workload": (f"synthetic multi-turn: prompts U[{MODEL_PLEN[0]},{MODEL_PLEN[1]}] random ids, 1-"
                        f"{args.model_turns} turns, {args.model_gen} greedy tokens per turn, later turns append "
                        "U[50,300] ids and re-prefill the whole conversation; FIFO continuous batching "
                        "(src/cb_run.py:254-378 scheduling)"),
           "turns": st["turns"], "t_max": t_max, "makespan_s": mk,
           "tokens_per_s": (st["prefill_tokens"] + st["decode_tokens"]) / mk,
           "prefill_tokens": st["prefill_tokens"], "prefill_calls": st["prefill_calls"], "prefill_s": pre_s,
           "prefill_tokens_per_s": st["prefill_tokens"] / pre_s,
           "decode_steps": st["decode_steps"], "decode_tokens": st["decode_tokens"], "decode_s": dec_s,
           "decode_ms_per_step": 1e3 * dec_s / max(1, st["decode_steps"]),
           "decode_tokens_per_s": st["decode_tokens"] / dec_s,
           "roofline": {"decode": {"bound": "hbm", "achieved": dec_gbs, "peak": hbm_peak, "unit": "GB/s",
                                   "frac": dec_gbs / hbm_peak, "peak_source": peak_src,
                                   "bytes": "per rank per step: local weights + LM head, KV rows read, "
                                            "GDN/conv state read + write; slowest rank"},
                        "prefill": {"bound": "tensor", "achieved": pre_tf, "peak": tc_peak, "unit": "TFLOP/s",
                                    "frac": pre_tf / tc_peak, "peak_source": peak_src + " (bf16 sustained)",
                                    "flops": "per rank, approximate: 2 x matmul weights x tokens + GDN chunk "
                                             "algebra + causal attention; slowest rank"}},
           "timing": "wall clock per engine call (each ends with its host read of the tokens), max over ranks",
           "graph": True, "weights": "random-init bf16",
           "allreduce": ("none" if world <= 1 else {
               "arnorm": "cuBLAS + gdn_allreduce_add_rmsnorm (peer memory) for decode, NCCL for prefill",
               "push": "cuBLAS + gdn_push_partial + gdn_pull_add_rmsnorm (peer memory) for decode, NCCL for prefill",
               "fused": "gdn_linear_push + gdn_pull_add_rmsnorm (peer memory) for decode, NCCL for prefill",
               "peer": "cuBLAS + gdn_allreduce (peer memory) for decode, NCCL for prefill",
               "nccl": "NCCL"}[args.model_allreduce]),
           "lm_head": "vocabulary-parallel" if world > 1 else "full", "build_s": build_s}
    if parity is not None:
        out["tp_parity"] = parity
    if breakdown is not None:
        out["decode_breakdown"] = breakdown
    return out


def run_e2e(ops, w, q, k, v, g, beta, cu, pool, slot, use_init, out, args, world, stream, tot_tokens):
    """Same step through the public API with the step's inputs in pinned host memory: every step
    copies its q, k, v, g, beta host -> device and its output device -> host inside the timed
    region.  As a serving loop would, consecutive steps overlap: device inputs and outputs are
    double-buffered, uploads, kernels and downloads run on their own streams, and step i's upload
    waits only for the kernel of step i - 2 that read the same buffers."""
    T = w["T"]
    hq, hk, hv = w["q"].pin_memory(), w["k"].pin_memory(), w["v"].pin_memory()
    hg, hb = w["g"].pin_memory(), w["beta"].pin_memory()
    hout = [torch.empty(T, HV, D, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv, hg, hb))
    d2h = hout[0].numel() * hout[0].element_size()
    sets = [(q, k, v, g, beta, out),
            tuple(torch.empty_like(t) for t in (q, k, v, g, beta, out))]
    s_in, s_cmp, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_cmp = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def steps(n):
        for i in range(n):
            bi = i & 1
            dq, dk, dv, dg, db, do = sets[bi]
            with torch.cuda.stream(s_in):
                s_in.wait_event(ev_cmp[bi])          # the kernel that last read this input set is done
                dq.copy_(hq, non_blocking=True)
                dk.copy_(hk, non_blocking=True)
                dv.copy_(hv, non_blocking=True)
                dg.copy_(hg, non_blocking=True)
                db.copy_(hb, non_blocking=True)
                ev_in[bi].record(s_in)
            with torch.cuda.stream(s_cmp):
                s_cmp.wait_event(ev_in[bi])
                s_cmp.wait_event(ev_out[bi])         # the download that last read this output is done
                ops.chunk_prefill_varlen(dq, dk, dv, dg, db, cu, pool, slot, use_init, True, out=do)
                ev_cmp[bi].record(s_cmp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_cmp[bi])
                hout[bi].copy_(do, non_blocking=True)
                ev_out[bi].record(s_out)

    steps(max(2, min(args.warmup, 3)))
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for st in (s_in, s_cmp, s_out):
        st.wait_event(e0)
    steps(args.steps)
    for st in (s_in, s_cmp, s_out):
        stream.wait_stream(st)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = allreduce_max(e0.elapsed_time(e1) / args.steps, world)
    e2e_value = tot_tokens / (e2e_ms / 1e3)
    return {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "overlap": "double-buffered device inputs/outputs; upload, kernel and download streams"}


def run_decode(ops, dev, args, world, hbm_peak, peak_src):
    g = torch.Generator(device="cpu").manual_seed(1234)
    n, L = DEC_SLOTS, args.decode_layers
    bf = torch.bfloat16
    layers = []
    for _ in range(L):
        layers.append(dict(
            conv_w=(torch.rand(CONV_DIM, CONV_K, generator=g) - 0.5).to(bf).to(dev),
            A_log=torch.log(torch.empty(HV).uniform_(1, 16, generator=g)).to(dev),
            dt_bias=(torch.rand(HV, generator=g) * 2 - 1).to(dev),
            norm_w=(1 + 0.1 * torch.randn(D, generator=g)).to(bf).to(dev),
            conv_pool=torch.randn(n, CONV_DIM, CONV_K, generator=g).to(bf).to(dev),
            rec_pool=(torch.randn(n, HV, D, D, generator=g) * 0.02).to(dev),
            mixed=torch.randn(n, CONV_DIM, generator=g).to(bf).to(dev),
            z=torch.randn(n, HV, D, generator=g).to(bf).to(dev),
            a=torch.randn(n, HV, generator=g).to(bf).to(dev),
            b=torch.randn(n, HV, generator=g).to(bf).to(dev),
            out=torch.empty(n, HV, D, dtype=bf, device=dev)))
    slot = torch.randperm(n, generator=g).to(torch.int32).to(dev)
    ws = ops.decode_layer_workspace(n, HK, HV, D, D, bf, dev)

    def step():
        for Ly in layers:
            ops.decode_layer(Ly["mixed"], Ly["z"], Ly["a"], Ly["b"], Ly["A_log"], Ly["dt_bias"], Ly["conv_w"], None,
                             Ly["conv_pool"], Ly["rec_pool"], slot, Ly["norm_w"], 1e-6, HK, HV, D, D,
                             workspace=ws, out=Ly["out"])

    step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream()
    cap.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(cap):
        with torch.cuda.graph(graph, stream=cap):
            step()
    torch.cuda.current_stream().wait_stream(cap)
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    barrier(world)
    durs = time_events(graph.replay, args.steps, torch.cuda.current_stream())
    barrier(world)
    us = 1000.0 * sum(durs) / len(durs)
    us_max = 1000.0 * allreduce_max(us / 1000.0, world)
    state_bytes = 2 * L * n * HV * D * D * 4
    conv_bytes = 2 * L * n * CONV_DIM * CONV_K * 2
    io_bytes = L * (n * CONV_DIM * 2 + 2 * n * HV * D * 2 + 2 * n * HV * 2 + CONV_DIM * CONV_K * 2)
    total = state_bytes + conv_bytes + io_bytes
    achieved = total / (us * 1e-6) / 1e9
    del graph
    return {"us_per_step": us_max, "layers": L, "slots": n, "graph": True,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                         "frac": achieved / hbm_peak, "peak_source": peak_src,
                         "algorithmic_bytes_per_step": total,
                         "traffic": (load_traffic().get("gdn_decode_layer", 0.0) * L) or None},
            "gpu_launches": args.steps * L * 2}


def main():
    args = parse()
    if args.warmup < 3:
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    world, rank, local = dist_setup(args)
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
