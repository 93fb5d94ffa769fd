"""GPU parity of the CUDA kernels against the reference's golden vectors and the CPU oracle.

Tolerances (stated per the task's contract):
  * fp32 path: max |a-b| <= 1e-4 * max|ref|                      ("<= 1e-4 relative")
  * bf16 activations with fp32 state: outputs and final states within 2e-2 max-abs
    (outputs additionally allowed one bf16 rounding step, 2^-7 relative, where |ref| > 1)
  * slot gather/scatter and state placement: bit-exact (untouched slots are compared
    bit for bit, poisoned with NaN where useful); conv states are pure data movement and
    are compared bit for bit.
"""
import numpy as np
import pytest
import torch

from conftest import load_golden, pkg
from oracle import gdn_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.fail("no CUDA device")
    return pkg("ops")


def T(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(DEV).to(dtype)


def N(t):
    return t.detach().float().cpu().numpy()


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.abs(a - b).max() / max(np.abs(b).max(), 1e-30)


def bf16_ok(a, b, atol=2e-2):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return bool(np.all(np.abs(a - b) <= atol + np.abs(b) * 2.0 ** -7))


# ----------------------------------------------------------------------------- a4 gated RMSNorm
def test_gated_rmsnorm_golden(ops):
    d = load_golden("norm_bf16.npz")
    y = ops.gated_rmsnorm(T(d["x"], torch.bfloat16), T(d["z"], torch.bfloat16), T(d["w"], torch.bfloat16))
    y = N(y)
    assert bf16_ok(y, d["y"], atol=0)
    assert (y != d["y"]).sum() <= y.size // 100
    y32 = N(ops.gated_rmsnorm(T(d["x"]), T(d["z"]), T(d["w"])))
    assert rel(y32, d["y32"]) < 1e-5


def test_gated_rmsnorm_strided_rows(ops):
    g = torch.Generator(device="cpu").manual_seed(1)
    x = torch.randn(37, 3, 256, generator=g).to(DEV, torch.bfloat16)[:, 1]      # row stride 768
    z = torch.randn(37, 256, generator=g).to(DEV, torch.bfloat16)
    w = (1 + 0.1 * torch.randn(256, generator=g)).to(DEV, torch.bfloat16)
    y = N(ops.gated_rmsnorm(x, z, w))
    ref = O.gated_rmsnorm(N(x), N(z), N(w), 1e-6, "bf16")
    assert bf16_ok(y, ref, atol=0)


# ----------------------------------------------------------------------------- a3 decode conv
def test_conv_update_golden_both_modes(ops):
    d = load_golden("conv_bf16.npz")
    bf = torch.bfloat16
    w, b = T(d["w"], bf), T(d["b"], bf)
    se, sh = T(d["s0"], bf), T(d["s0"], bf)
    for t in range(3):
        ye = ops.elem_conv_update(T(d["xs"][t], bf), se, w, b)
        yh = ops.causal_conv1d_update(T(d["xs"][t], bf), sh, w, b, "silu")
        assert np.array_equal(N(se), d["st_elem"][t]) and np.array_equal(N(sh), d["st_hf"][t])
        assert bf16_ok(N(ye), d["y_elem"][t], atol=0)
        assert bf16_ok(N(yh), d["y_hf"][t], atol=0)
    s2 = T(d["s0"], bf)
    y2 = ops.causal_conv1d_update(T(d["x2"], bf), s2, w, None, "silu")
    assert np.array_equal(N(s2), d["s2_after"])
    assert bf16_ok(N(y2), d["y2"], atol=0)


def test_conv_update_slot_indexed_leaves_other_slots_bitwise(ops):
    g = torch.Generator(device="cpu").manual_seed(2)
    S, n, C, K = 9, 5, 640, 4
    pool = torch.randn(S, C, K, generator=g).to(torch.bfloat16)
    pool[[0, 8]] = float("nan")                       # poison two slots nobody uses
    slot = torch.tensor([3, 1, 7, 4, 6], dtype=torch.int32)
    x = torch.randn(n, C, generator=g).to(torch.bfloat16)
    w = (torch.rand(C, K, generator=g) - 0.5).to(torch.bfloat16)
    pool_d = pool.to(DEV)
    y = ops._conv_update(x.to(DEV), pool_d, w.to(DEV), None, ops.GDN_CONV_ELEM, slot_idx=slot.to(DEV))
    ref_pool = pool.float().numpy().copy()
    st = ref_pool[slot.numpy()]
    yr = O.conv_update_elem(x.float().numpy()[:, :, None], st, w.float().numpy(), None, "bf16")
    ref_pool[slot.numpy()] = st
    got = N(pool_d)
    assert np.array_equal(got[slot.numpy()], ref_pool[slot.numpy()])
    untouched = [0, 2, 5, 8]
    assert np.array_equal(pool[untouched].view(torch.int16).numpy(),
                          pool_d[untouched].cpu().view(torch.int16).numpy())
    assert bf16_ok(N(y)[:, :, 0], yr[:, :, 0], atol=0)


def test_prefill_conv_golden(ops):
    d = load_golden("prefill_conv_bf16.npz")
    bf = torch.bfloat16
    lens = d["lens"]
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device=DEV)
    C, K = d["w"].shape
    pool = torch.full((len(lens) + 2, C, K), float("nan"), dtype=bf, device=DEV)
    slot = torch.arange(len(lens), dtype=torch.int32, device=DEV) + 1
    y = ops.prefill_conv_varlen(T(d["x"], bf), cu, T(d["w"], bf), None, pool, slot, None)
    assert bf16_ok(N(y), d["y"], atol=0)
    assert np.array_equal(N(pool[1:1 + len(lens)]), d["st"])
    assert torch.isnan(pool[0]).all() and torch.isnan(pool[-1]).all()
    # continuation from a slot's previous inputs (TPEngine.prefill_chunk form)
    pool2 = T(d["prev"][None], bf).contiguous()
    yc = ops.prefill_conv_varlen(T(d["xc"], bf), torch.tensor([0, d["xc"].shape[0]], dtype=torch.int32,
                                 device=DEV), T(d["w"], bf), None, pool2, None,
                                 torch.ones(1, dtype=torch.int32, device=DEV))
    assert bf16_ok(N(yc), d["yc"], atol=0)
    assert np.array_equal(N(pool2[0]), d["stc"])


# ----------------------------------------------------------------------------- a2 recurrence
def test_recurrent_slot_step_golden(ops):
    d = load_golden("recurrent_bf16.npz")
    bf = torch.bfloat16
    pool = T(d["pool"])
    before = pool.clone()
    o = ops.recurrent_step_slots(T(d["q"], bf), T(d["k"], bf), T(d["v"], bf), T(d["g"]), T(d["beta"], bf).float(),
                                 pool, T(d["slot_idx"]).to(torch.int32))
    si = d["slot_idx"].astype(np.int64)
    assert bf16_ok(N(o), d["out"], atol=1e-2)
    assert np.abs(N(pool)[si] - d["new_state"]).max() < 1e-5
    untouched = np.setdiff1d(np.arange(pool.shape[0]), si)
    assert torch.equal(pool[untouched], before[untouched])


def test_recurrent_multi_token_golden(ops):
    d = load_golden("recurrent_bf16.npz")
    bf = torch.bfloat16
    r = d["v3"].shape[1] // d["q3"].shape[1]
    q = T(O.repeat_heads(d["q3"], r)[None], bf)
    k = T(O.repeat_heads(d["k3"], r)[None], bf)
    o, s = ops.recurrent_gated_delta_rule(q, k, T(d["v3"][None], bf), T(d["g3"][None]),
                                          T(d["beta3"][None], bf), T(d["init3"][None]), True, True)
    assert bf16_ok(N(o)[0], d["out3"], atol=1e-2)
    assert np.abs(N(s)[0] - d["state3"]).max() < 1e-5
    # un-repeated q/k with the in-kernel head map gives the same result
    o2, s2 = ops.recurrent_gated_delta_rule(T(d["q3"][None], bf), T(d["k3"][None], bf), T(d["v3"][None], bf),
                                            T(d["g3"][None]), T(d["beta3"][None], bf), T(d["init3"][None]), True,
                                            True)
    assert torch.equal(o, o2) and torch.equal(s, s2)


def test_recurrent_known_answers(ops):
    """g = 0, beta = 0 leaves the state bit-unchanged; k = 0 is a pure decay."""
    g = torch.Generator(device="cpu").manual_seed(3)
    n, Hk, Hv, d = 4, 2, 6, 128
    pool = (torch.randn(6, Hv, d, d, generator=g) * 0.3).to(DEV)
    slot = torch.tensor([5, 0, 2, 3], dtype=torch.int32, device=DEV)
    q = torch.randn(n, Hk, d, generator=g).to(DEV, torch.bfloat16)
    k = torch.randn(n, Hk, d, generator=g).to(DEV, torch.bfloat16)
    v = torch.randn(n, Hv, d, generator=g).to(DEV, torch.bfloat16)
    zero = torch.zeros(n, Hv, device=DEV)
    before = pool.clone()
    ops.recurrent_step_slots(q, k, v, zero, zero, pool, slot)
    assert torch.equal(pool, before)
    gdec = -torch.rand(n, Hv, generator=g).to(DEV)
    ops.recurrent_step_slots(q, torch.zeros_like(k), v, gdec, torch.rand(n, Hv, device=DEV), pool, slot,
                             use_qk_l2norm=False)
    expect = before[slot.long()] * torch.exp(gdec)[:, :, None, None]
    assert torch.allclose(pool[slot.long()], expect, rtol=1e-6, atol=0)


def test_recurrent_fp32_matches_oracle(ops):
    rng = np.random.default_rng(4)
    B, Tn, Hk, Hv, d = 2, 5, 4, 8, 64
    q = rng.standard_normal((B, Tn, Hk, d)).astype(np.float32)
    k = rng.standard_normal((B, Tn, Hk, d)).astype(np.float32)
    v = rng.standard_normal((B, Tn, Hv, d)).astype(np.float32)
    gg = -rng.uniform(0.01, 1.0, (B, Tn, Hv)).astype(np.float32)
    bb = (1 / (1 + np.exp(-rng.standard_normal((B, Tn, Hv))))).astype(np.float32)
    init = (rng.standard_normal((B, Hv, d, d)) * 0.1).astype(np.float32)
    o, s = ops.recurrent_gated_delta_rule(T(q), T(k), T(v), T(gg), T(bb), T(init), True, True)
    ro, rs = O.recurrent_gated_delta_rule(O.repeat_heads(q, 2), O.repeat_heads(k, 2), v, gg, bb, init, True, True,
                                          "f32")
    assert rel(N(o), ro) < 1e-4 and rel(N(s), rs) < 1e-4


def test_recurrent_bad_slot_sets_error_flag(ops):
    n, Hk, Hv, d = 2, 1, 3, 128
    pool = torch.zeros(2, Hv, d, d, device=DEV)
    slot = torch.tensor([1, 7], dtype=torch.int32, device=DEV)      # 7 is out of range
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    x = torch.randn(n, Hk, d, device=DEV).to(torch.bfloat16)
    ops.recurrent_step_slots(x, x, torch.randn(n, Hv, d, device=DEV).to(torch.bfloat16),
                             torch.zeros(n, Hv, device=DEV), torch.ones(n, Hv, device=DEV), pool, slot, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 1
    assert torch.isfinite(pool).all()


# ----------------------------------------------------------------------------- a1 chunk prefill
@pytest.mark.parametrize("name", ["chunk_c0_f32.npz", "chunk_c0init_f32.npz"])
def test_chunk_fp32_golden(ops, name):
    d = load_golden(name)
    r = int(d["Hv"]) // int(d["Hk"])
    for b, L in enumerate(d["lens"]):
        init = T(d[f"init{b}"][None]) if f"init{b}" in d else None
        q = T(O.repeat_heads(d[f"q{b}"], r)[None])
        k = T(O.repeat_heads(d[f"k{b}"], r)[None])
        o, s = ops.chunk_gated_delta_rule(q, k, T(d[f"v{b}"][None]), T(d[f"g{b}"][None]), T(d[f"beta{b}"][None]),
                                          64, init, True, True)
        assert rel(N(o)[0], d[f"out{b}"]) < 1e-4
        assert rel(N(s)[0], d[f"state{b}"]) < 1e-4


def test_chunk_fp32_varlen_packed_config0(ops):
    """Config 0 as one packed varlen call (B=2, 256 + 190 tokens, un-repeated q/k heads), slot-indexed
    final states; equals the per-sequence reference outputs and states."""
    d = load_golden("chunk_c0_f32.npz")
    lens = d["lens"]
    q = T(np.concatenate([d["q0"], d["q1"]]))
    k = T(np.concatenate([d["k0"], d["k1"]]))
    v = T(np.concatenate([d["v0"], d["v1"]]))
    g = T(np.concatenate([d["g0"], d["g1"]]))
    be = T(np.concatenate([d["beta0"], d["beta1"]]))
    cu = torch.tensor([0, lens[0], lens[0] + lens[1]], dtype=torch.int32, device=DEV)
    pool = torch.full((4, 8, 64, 64), float("nan"), device=DEV)
    slot = torch.tensor([2, 0], dtype=torch.int32, device=DEV)
    o = ops.chunk_prefill_varlen(q, k, v, g, be, cu, pool, slot, None, True)
    o = N(o)
    assert rel(o[:lens[0]], d["out0"]) < 1e-4 and rel(o[lens[0]:], d["out1"]) < 1e-4
    assert rel(N(pool[2]), d["state0"]) < 1e-4 and rel(N(pool[0]), d["state1"]) < 1e-4
    assert torch.isnan(pool[1]).all() and torch.isnan(pool[3]).all()


def test_chunk_bf16_golden(ops):
    d = load_golden("chunk_bf16.npz")
    bf = torch.bfloat16
    r = int(d["Hv"]) // int(d["Hk"])
    for b, L in enumerate(d["lens"]):
        o, s = ops.chunk_gated_delta_rule(T(O.repeat_heads(d[f"q{b}"], r)[None], bf),
                                          T(O.repeat_heads(d[f"k{b}"], r)[None], bf), T(d[f"v{b}"][None], bf),
                                          T(d[f"g{b}"][None]), T(d[f"beta{b}"][None], bf), 64,
                                          T(d[f"init{b}"][None]), True, True)
        assert bf16_ok(N(o)[0], d[f"out{b}"]), f"seq {b} (L={L})"
        assert np.abs(N(s)[0] - d[f"state{b}"]).max() < 2e-2


def test_chunk_split_equals_unsplit(ops):
    """Prefill in two pieces (state carried through the slot, use_initial) == one piece
    (src/cb_tp.py:195-271 contract)."""
    rng = np.random.default_rng(5)
    L, a, Hk, Hv, dd = 300, 137, 2, 6, 128
    q = rng.standard_normal((L, Hk, dd)).astype(np.float32)
    k = rng.standard_normal((L, Hk, dd)).astype(np.float32)
    v = rng.standard_normal((L, Hv, dd)).astype(np.float32)
    g = -rng.uniform(0.01, 1, (L, Hv)).astype(np.float32)
    be = rng.uniform(0, 1, (L, Hv)).astype(np.float32)
    bf = torch.bfloat16
    qd, kd, vd = T(q, bf), T(k, bf), T(v, bf)
    gd, bd = T(g), T(be)
    pool = torch.zeros(2, Hv, dd, dd, device=DEV)
    one = torch.tensor([0, L], dtype=torch.int32, device=DEV)
    o_full = ops.chunk_prefill_varlen(qd, kd, vd, gd, bd, one, pool, torch.tensor([0], dtype=torch.int32, device=DEV))
    s1 = torch.tensor([1], dtype=torch.int32, device=DEV)
    o_a = ops.chunk_prefill_varlen(qd[:a], kd[:a], vd[:a], gd[:a], bd[:a], torch.tensor([0, a], dtype=torch.int32,
                                   device=DEV), pool, s1, None)
    o_b = ops.chunk_prefill_varlen(qd[a:], kd[a:], vd[a:], gd[a:], bd[a:], torch.tensor([0, L - a], dtype=torch.int32,
                                   device=DEV), pool, s1, torch.ones(1, dtype=torch.int32, device=DEV))
    assert (torch.cat([o_a, o_b]).float() - o_full.float()).abs().max().item() < 2e-2
    assert (pool[0] - pool[1]).abs().max().item() < 2e-2


def test_chunk_matches_token_recurrence_bf16(ops):
    """The chunked kernel and the token-by-token kernel agree (config-0 check at d=128, bf16)."""
    rng = np.random.default_rng(6)
    L, Hk, Hv, dd = 200, 1, 3, 128
    bf = torch.bfloat16
    q = T(rng.standard_normal((1, L, Hk, dd)), bf)
    k = T(rng.standard_normal((1, L, Hk, dd)), bf)
    v = T(rng.standard_normal((1, L, Hv, dd)), bf)
    g = T(-rng.uniform(0.01, 1, (1, L, Hv)))
    be = T(rng.uniform(0, 1, (1, L, Hv)))
    oc, sc = ops.chunk_gated_delta_rule(q, k, v, g, be, 64, None, True, True)
    orr, sr = ops.recurrent_gated_delta_rule(q, k, v, g, be, None, True, True)
    assert (oc.float() - orr.float()).abs().max().item() < 2e-2
    assert (sc - sr).abs().max().item() < 2e-2


@pytest.mark.parametrize("dd,dt", [(128, torch.bfloat16), (64, torch.float32)])
def test_chunk_prefill_gates_matches_torch_gate_lines(ops, dd, dt):
    """Gates formed in-kernel (chunk_prefill_varlen_gates) == the reference's torch gate lines
    (src/cb_tp.py:170-171) fed to chunk_prefill_varlen: identical g and beta give identical results
    (checked at the contract tolerance: bf16 2e-2 max-abs, fp32 1e-4 relative), slot placement bit for
    bit; and the bf16 path against the oracle.  a includes values past softplus's threshold of 20."""
    import torch.nn.functional as F
    rng = np.random.default_rng(21)
    lens, Hk, Hv = [70, 300, 1], 2, 6
    Tt = sum(lens)
    cu_h = np.array([0, lens[0], lens[0] + lens[1], Tt], np.int32)
    q = rng.standard_normal((Tt, Hk, dd)).astype(np.float32)
    k = rng.standard_normal((Tt, Hk, dd)).astype(np.float32)
    v = rng.standard_normal((Tt, Hv, dd)).astype(np.float32)
    a = (3 * rng.standard_normal((Tt, Hv))).astype(np.float32)
    a[::17, 1] = 25.0
    b = (2 * rng.standard_normal((Tt, Hv))).astype(np.float32)
    if dt == torch.bfloat16:
        q, k, v, a, b = (O.bf16(x) for x in (q, k, v, a, b))
    A_log = O.bf16(np.log(rng.uniform(1, 16, Hv)))
    dt_bias = O.bf16(rng.uniform(-1, 1, Hv))
    pool0 = (0.02 * rng.standard_normal((5, Hv, dd, dd))).astype(np.float32)
    slot_h = np.array([2, 0, 3], np.int32)
    use_h = np.array([1, 0, 1], np.int32)
    qd, kd, vd, ad, bd = T(q, dt), T(k, dt), T(v, dt), T(a, dt), T(b, dt)
    Ad, dbd = T(A_log), T(dt_bias)
    cu = torch.tensor(cu_h, device=DEV)
    slot = torch.tensor(slot_h, device=DEV)
    use = torch.tensor(use_h, device=DEV)
    beta_t = bd.sigmoid().float()
    g_t = -Ad.exp() * F.softplus(ad.float() + dbd)
    pool_ref, pool_raw = T(pool0), T(pool0)
    pool_raw[1] = float("nan")
    pool_raw[4] = float("nan")
    o_ref = ops.chunk_prefill_varlen(qd, kd, vd, g_t, beta_t, cu, pool_ref, slot, use, True)
    o_raw = ops.chunk_prefill_varlen_gates(qd, kd, vd, ad, bd, Ad, dbd, cu, pool_raw, slot, use, True)
    torch.cuda.synchronize()
    assert torch.isnan(pool_raw[1]).all() and torch.isnan(pool_raw[4]).all()
    sl = slot.long()
    if dt == torch.bfloat16:
        assert (o_raw.float() - o_ref.float()).abs().max().item() <= 2e-2
        assert (pool_raw[sl] - pool_ref[sl]).abs().max().item() <= 2e-2
        b_o, g_o = O.decode_gates(a, b, A_log, dt_bias, "bf16")
        ref_pool = pool0.copy()
        ro, _ = O.prefill_varlen(q, k, v, g_o, b_o, cu_h, ref_pool, slot_h, use_h, True, "bf16")
        assert bf16_ok(N(o_raw), ro)
        assert np.abs(N(pool_raw)[slot_h] - ref_pool[slot_h]).max() < 2e-2
    else:
        assert rel(N(o_raw), N(o_ref)) <= 1e-4
        assert rel(N(pool_raw[sl]), N(pool_ref[sl])) <= 1e-4


@pytest.mark.parametrize("dd,dt", [(128, torch.bfloat16), (64, torch.float32)])
def test_chunk_prefill_empty_and_ragged_sequences(ops, dd, dt):
    """Packed prefill with empty sequences between ragged ones (1, 64, 65, 127 tokens): outputs and
    states match the oracle; an empty sequence's final state is its initial state (bit for bit) or
    zeros; unused pool rows stay untouched.  A call whose sequences are all empty writes only states."""
    rng = np.random.default_rng(22)
    lens, Hk, Hv = [0, 65, 0, 1, 64, 127, 0], 1, 3
    Tt = sum(lens)
    cu_h = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    bfl = dt == torch.bfloat16
    cast = O.bf16 if bfl else (lambda x: x.astype(np.float32))
    q = cast(rng.standard_normal((Tt, Hk, dd)))
    k = cast(rng.standard_normal((Tt, Hk, dd)))
    v = cast(rng.standard_normal((Tt, Hv, dd)))
    g = -rng.uniform(0.01, 1, (Tt, Hv)).astype(np.float32)
    be = cast(rng.uniform(0, 1, (Tt, Hv)))
    pool0 = (0.02 * rng.standard_normal((9, Hv, dd, dd))).astype(np.float32)
    pool0[[0, 8]] = np.nan                                 # rows nobody uses
    slot_h = np.arange(1, 8, dtype=np.int32)
    use_h = np.array([1, 0, 0, 1, 0, 1, 0], np.int32)      # sequence 0 empty from a state, 2 and 6 from zeros
    pool = T(pool0)
    o = ops.chunk_prefill_varlen(T(q, dt), T(k, dt), T(v, dt), T(g), T(be), torch.tensor(cu_h, device=DEV), pool,
                                 torch.tensor(slot_h, device=DEV), torch.tensor(use_h, device=DEV), True)
    ref_pool = pool0.copy()
    ro, _ = O.prefill_varlen(q, k, v, g, be, cu_h, ref_pool, slot_h, use_h, True, "bf16" if bfl else "f32")
    got = N(pool)
    assert o.shape == (Tt, Hv, dd)
    if bfl:
        assert bf16_ok(N(o), ro)
        assert np.abs(got[slot_h] - ref_pool[slot_h]).max() < 2e-2
    else:
        assert rel(N(o), ro) < 1e-4
        assert rel(got[slot_h], ref_pool[slot_h]) < 1e-4
    assert np.array_equal(got[1], pool0[1])                # empty, initial state kept bit for bit
    assert not got[3].any() and not got[7].any()           # empty, from zeros
    assert np.isnan(got[0]).all() and np.isnan(got[8]).all()
    # every sequence empty: no tokens, only states
    pool2 = T(pool0)
    e = torch.empty(0, Hk, dd, dtype=dt, device=DEV)
    ev = torch.empty(0, Hv, dd, dtype=dt, device=DEV)
    eg = torch.empty(0, Hv, device=DEV)
    o2 = ops.chunk_prefill_varlen(e, e, ev, eg, eg, torch.zeros(4, dtype=torch.int32, device=DEV), pool2,
                                  torch.tensor([1, 2, 3], dtype=torch.int32, device=DEV),
                                  torch.tensor([1, 0, 1], dtype=torch.int32, device=DEV), True)
    got2 = N(pool2)
    assert o2.shape == (0, Hv, dd)
    assert np.array_equal(got2[1], pool0[1]) and np.array_equal(got2[3], pool0[3]) and not got2[2].any()
    assert np.array_equal(got2[4:8], pool0[4:8])


def test_prefill_conv_empty_sequences(ops):
    """Varlen prefill conv with empty sequences: an empty sequence keeps its carried conv state (or
    gets zeros without one), bit for bit; the others match the oracle."""
    rng = np.random.default_rng(23)
    bf = torch.bfloat16
    lens, C, K = [0, 3, 0, 5, 1], 256, 4
    Tt = sum(lens)
    cu_h = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    x = O.bf16(rng.standard_normal((Tt, C)))
    w = O.bf16(rng.uniform(-0.5, 0.5, (C, K)))
    pool0 = O.bf16(rng.standard_normal((len(lens) + 1, C, K)))
    slot_h = np.array([5, 1, 2, 3, 4], np.int32)
    use_h = np.array([1, 1, 0, 0, 1], np.int32)
    pool = T(pool0, bf)
    y = ops.prefill_conv_varlen(T(x, bf), torch.tensor(cu_h, device=DEV), T(w, bf), None, pool,
                                torch.tensor(slot_h, device=DEV), torch.tensor(use_h, device=DEV))
    init = np.where(use_h[:, None, None] != 0, pool0[slot_h], 0).astype(np.float32)
    yr, st = O.prefill_conv(x, cu_h, w, None, init, "bf16")
    assert bf16_ok(N(y), yr, atol=0)
    got = N(pool)
    assert np.array_equal(got[slot_h], st)
    assert np.array_equal(got[5], pool0[5]) and not got[2].any()
    assert np.array_equal(got[0], pool0[0])


# ----------------------------------------------------------------------------- fused decode layer
def test_rmsnorm_matches_hf_module(ops):
    """ops.rmsnorm == Qwen3_5RMSNorm.forward (fp32 statistics, x * r * (1 + w), one rounding) within one
    bf16 step (the row reduction order differs from torch's); fp32 rows within 1e-5 relative."""
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5RMSNorm
    torch.manual_seed(3)
    for dim, rows, dt in ((5120, 16, torch.bfloat16), (256, 384, torch.bfloat16), (1000, 7, torch.bfloat16),
                          (5120, 3, torch.float32), (8192, 2, torch.bfloat16)):
        m = Qwen3_5RMSNorm(dim, eps=1e-6).to(DEV)
        with torch.no_grad():
            m.weight.normal_(0, 0.2)
        m = m.to(dt)
        x = (torch.randn(rows, dim, device=DEV) * 3).to(dt)
        ref = m(x).float()
        got = ops.rmsnorm(x, m.weight, m.eps).float()
        tol = ref.abs() * (2.0 ** -7 if dt == torch.bfloat16 else 1e-5) + 1e-6
        assert ((got - ref).abs() <= tol).all(), (dim, rows, dt)
    # a strided view (q_norm on the chunked q projection): rows of hd inside rows of 2 hd
    qg = torch.randn(4, 1, 6, 512, device=DEV).to(torch.bfloat16)
    q, _ = torch.chunk(qg, 2, dim=-1)
    m = Qwen3_5RMSNorm(256, eps=1e-6).to(DEV).to(torch.bfloat16)
    assert ((ops.rmsnorm(q, m.weight, m.eps).float() - m(q).float()).abs()
            <= m(q).float().abs() * 2.0 ** -7 + 1e-6).all()


def test_attn_decode_matches_sdpa(ops):
    """gdn_attn_decode == the reference's decode attention (src/cb_engine.py:295-316): the new K/V rows
    land bit-exactly at (slot, pos) and nowhere else, and the output equals softmax(scale q k^T) v over
    positions 0..pos (fp32) rounded to bf16 times rnd(sigmoid(gate)), within bf16 rounding.  Positions at
    the 128-position split boundaries and 0 included; a bad slot sets the error flag."""
    torch.manual_seed(11)
    bf = torch.bfloat16
    n, S_, kvh, g, hd, T = 6, 9, 2, 6, 256, 600
    Hq = kvh * g
    kv_k = torch.randn(S_, kvh, T, hd, device=DEV).to(bf)
    kv_v = torch.randn(S_, kvh, T, hd, device=DEV).to(bf)
    k0, v0 = kv_k.clone(), kv_v.clone()
    slot = torch.tensor([3, 0, 8, 5, 1, 6], dtype=torch.int32, device=DEV)
    pos = torch.tensor([0, 127, 128, 255, 431, 599], dtype=torch.int32, device=DEV)
    q = torch.randn(n, Hq, hd, device=DEV).to(bf)
    kn = torch.randn(n, kvh, hd, device=DEV).to(bf)
    vn = torch.randn(n, kvh, hd, device=DEV).to(bf)
    gate = torch.randn(n, Hq, hd, device=DEV).to(bf)
    scale = hd ** -0.5
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = ops.attn_decode(q, kn, vn, kv_k, kv_v, slot, pos, T, scale, gate=gate, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    for b in range(n):
        s, p_ = int(slot[b]), int(pos[b])
        k0[s, :, p_] = kn[b]
        v0[s, :, p_] = vn[b]
    assert torch.equal(kv_k, k0) and torch.equal(kv_v, v0)
    for b in range(n):
        s, p_ = int(slot[b]), int(pos[b])
        for h in range(Hq):
            j = h // g
            sc = (q[b, h].float() @ k0[s, j, :p_ + 1].float().T) * scale
            o = (torch.softmax(sc, -1) @ v0[s, j, :p_ + 1].float()).to(bf).float()
            ref = (o * torch.sigmoid(gate[b, h].float()).to(bf).float()).to(bf).float()
            got = out[b, h].float()
            assert ((got - ref).abs() <= ref.abs() * 2 ** -6 + 2e-3).all(), (b, h, (got - ref).abs().max())
    bad = torch.tensor([2, 9, 0, 1, 4, 7], dtype=torch.int32, device=DEV)  # 9 is out of range
    ops.attn_decode(q, kn, vn, kv_k, kv_v, bad, pos, T, scale, gate=gate, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 1


def _decode_layer_case(ops, n, S, Hk, Hv, slot, steps, seed=7, conv_b=False, dd=128, K=4, hf=False):
    rng = np.random.default_rng(seed)
    Cc = 2 * Hk * dd + Hv * dd
    bf = torch.bfloat16
    r16 = lambda a: O.bf16(np.asarray(a, np.float32))
    A_log = np.log(rng.uniform(1, 16, Hv)).astype(np.float32)
    dt_bias = rng.uniform(-1, 1, Hv).astype(np.float32)
    conv_w = r16(rng.uniform(-0.5, 0.5, (Cc, K)))
    bias = r16(rng.uniform(-0.5, 0.5, Cc)) if conv_b else None
    conv_pool = r16(rng.standard_normal((S, Cc, K)))
    rec_pool = (rng.standard_normal((S, Hv, dd, dd)) * 0.1).astype(np.float32)
    norm_w = r16(1 + 0.1 * rng.standard_normal(dd))
    cp, rp = conv_pool.copy(), rec_pool.copy()
    conv_d, rec_d = T(conv_pool, bf), T(rec_pool)
    ws = ops.decode_layer_workspace(n, Hk, Hv, dd, dd, bf, DEV)
    slot_d = torch.tensor(slot, device=DEV)
    for _ in range(steps):
        mixed = r16(rng.standard_normal((n, Cc)))
        z = r16(rng.standard_normal((n, Hv, dd)))
        a = r16(rng.standard_normal((n, Hv)))
        b = r16(rng.standard_normal((n, Hv)))
        # oracle: elem conv -> split -> gates -> recurrence -> gated norm
        st = cp[slot]
        conv = O.conv_update if hf else O.conv_update_elem
        y = conv(mixed[:, :, None], st, conv_w, bias, "bf16")[:, :, 0]
        cp[slot] = st
        qo, ko, vo = y[:, :Hk * dd].reshape(n, Hk, dd), y[:, Hk * dd:2 * Hk * dd].reshape(n, Hk, dd), \
            y[:, 2 * Hk * dd:].reshape(n, Hv, dd)
        beta, g = O.decode_gates(a, b, A_log, dt_bias, "bf16")
        core = O.decode_step_slots(qo, ko, vo, g, beta, rp, slot, True, "bf16")
        ref = O.gated_rmsnorm(core, z, norm_w, 1e-6, "bf16")
        out = ops.decode_layer(T(mixed, bf), T(z, bf), T(a, bf), T(b, bf), T(A_log), T(dt_bias), T(conv_w, bf),
                               None if bias is None else T(bias, bf), conv_d, rec_d, slot_d, T(norm_w, bf), 1e-6,
                               Hk, Hv, dd, dd, conv_mode=ops.GDN_CONV_HF if hf else ops.GDN_CONV_ELEM,
                               workspace=ws)
        assert np.array_equal(N(conv_d), cp)
        assert bf16_ok(N(out), ref)
        assert np.abs(N(rec_d)[slot] - rp[slot]).max() < 1e-4
    untouched = np.setdiff1d(np.arange(S), slot)
    assert np.array_equal(N(rec_d)[untouched], rec_pool[untouched])
    assert np.array_equal(N(conv_d)[untouched], conv_pool[untouched])


def test_decode_layer_matches_oracle_composition(ops):
    _decode_layer_case(ops, 5, 8, 2, 6, np.array([6, 1, 3, 0, 4], np.int32), steps=1)


def test_decode_layer_hf_conv_mode_with_bias(ops):
    """HF conv rounding (one rounding of the fp32-accumulated conv plus bias) through the decode layer."""
    _decode_layer_case(ops, 4, 9, 2, 6, np.array([8, 2, 5, 0], np.int32), steps=2, seed=17, conv_b=True, hf=True)


def test_decode_layer_conv_width_3(ops):
    """Conv kernel width 3 (the window update for K != 4)."""
    _decode_layer_case(ops, 3, 5, 1, 3, np.array([4, 0, 2], np.int32), steps=2, seed=19, K=3)


def test_decode_layer_many_items_per_cta_two_steps(ops):
    # 32 x 16 = 512 (slot, head) items: every CTA of the persistent kernel runs several of them,
    # so each shared-memory stage is reused; two steps check the state and windows carry over
    rng = np.random.default_rng(3)
    slot = rng.permutation(40)[:32].astype(np.int32)
    _decode_layer_case(ops, 32, 40, 4, 16, slot, steps=2, seed=11, conv_b=True)


def test_decode_layer_large_batch(ops):
    # 32 x 48 = 1536 (slot, head) items: 10-11 per persistent CTA, so every stage of the state ring
    # is reused three times
    rng = np.random.default_rng(9)
    slot = rng.permutation(40)[:32].astype(np.int32)
    _decode_layer_case(ops, 32, 40, 16, 48, slot, steps=1, seed=13)


def test_decode_layer_bad_slot_sets_error_flag(ops):
    n, S, Hk, Hv, dd, K = 3, 4, 1, 2, 128, 4
    Cc = 2 * Hk * dd + Hv * dd
    bf = torch.bfloat16
    g = torch.Generator(device="cpu").manual_seed(0)
    rnd = lambda *sh: torch.randn(*sh, generator=g).to(DEV)
    conv_pool, rec_pool = rnd(S, Cc, K).to(bf), rnd(S, Hv, dd, dd) * 0.1
    conv0, rec0 = conv_pool.clone(), rec_pool.clone()
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    slot = torch.tensor([2, 7, 0], dtype=torch.int32, device=DEV)      # 7 is out of range
    ops.decode_layer(rnd(n, Cc).to(bf), rnd(n, Hv, dd).to(bf), rnd(n, Hv).to(bf), rnd(n, Hv).to(bf),
                     torch.zeros(Hv, device=DEV), torch.zeros(Hv, device=DEV), rnd(Cc, K).to(bf), None,
                     conv_pool, rec_pool, slot, torch.ones(dd, device=DEV).to(bf), 1e-6, Hk, Hv, dd, dd, err=err)
    torch.cuda.synchronize()
    assert err.item() == 1
    for s_ in (1, 3):   # rows no valid entry points at stay bit-identical
        assert torch.equal(conv_pool[s_], conv0[s_]) and torch.equal(rec_pool[s_], rec0[s_])
    assert not torch.equal(rec_pool[2], rec0[2]) and not torch.equal(rec_pool[0], rec0[0])


# ----------------------------------------------------------------------------- full config-1 size
def _config1(seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    lens = torch.randint(200, 1201, (16,), generator=g).tolist()
    Tt = sum(lens)
    q = torch.randn(Tt, 16, 128, generator=g)
    k = torch.randn(Tt, 16, 128, generator=g)
    q = (q / q.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    k = (k / k.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    v = torch.randn(Tt, 48, 128, generator=g).to(torch.bfloat16)
    beta = torch.sigmoid(torch.randn(Tt, 48, generator=g)).to(torch.bfloat16).float()
    gg = (-(0.01 + 0.99 * torch.rand(Tt, 48, generator=g))).to(torch.bfloat16).float()
    init = torch.randn(16, 48, 128, 128, generator=g) * 0.02
    cu = torch.tensor([0] + np.cumsum(lens).tolist(), dtype=torch.int32)
    return lens, q, k, v, gg, beta, init, cu


def test_chunk_tc_full_config1_vs_oracle_and_fp32_path(ops):
    """Config 1 at full size through the tensor-core kernel (bf16), checked (a) against the fp32
    CUDA-core kernel on every token and head, and (b) against the CPU oracle on two sequences."""
    lens, q, k, v, gg, beta, init, cu = _config1()
    dq, dk_, dv_ = q.to(DEV), k.to(DEV), v.to(DEV)
    dg, db, dcu = gg.to(DEV), beta.to(DEV), cu.to(DEV)
    slot = torch.arange(16, dtype=torch.int32, device=DEV).flip(0).contiguous()
    use = torch.ones(16, dtype=torch.int32, device=DEV)
    pool_tc = init.to(DEV)[slot.long()].contiguous()          # slot s holds sequence 15-s's state
    o_tc = ops.chunk_prefill_varlen(dq, dk_, dv_, dg, db, dcu, pool_tc, slot, use, True)
    pool_32 = init.to(DEV)[slot.long()].contiguous()
    o_32 = ops.chunk_prefill_varlen(dq.float(), dk_.float(), dv_.float(), dg, db, dcu, pool_32, slot, use, True)
    torch.cuda.synchronize()
    assert (o_tc.float() - o_32).abs().max().item() < 2e-2
    assert (pool_tc - pool_32).abs().max().item() < 2e-2
    for b in (0, 7):
        s, e = int(cu[b]), int(cu[b + 1])
        ro, rs = O.chunk_gated_delta_rule(O.repeat_heads(q[s:e].float().numpy(), 3)[None],
                                          O.repeat_heads(k[s:e].float().numpy(), 3)[None],
                                          v[s:e].float().numpy()[None], gg[s:e].numpy()[None],
                                          beta[s:e].numpy()[None], 64, init[b].numpy()[None], True, True, "bf16")
        assert bf16_ok(N(o_tc[s:e]), ro[0])
        assert np.abs(N(pool_tc[15 - b]) - rs[0]).max() < 2e-2


@pytest.mark.parametrize("d,Hk,Hv", [(128, 4, 12), (64, 2, 8)])
def test_decode_layer_row_strided_inputs_bit_exact(ops, d, Hk, Hv):
    """mixed_qkv, z, b and a as column slices of one fused projection output [n, C + Hv d + 2 Hv]
    (gdn_decode_layer_rows, what the engine's fused decode GEMM produces) give exactly what the same
    values as separate contiguous tensors give, outputs and both pools."""
    g = torch.Generator().manual_seed(11)
    n, S, K = 5, 9, 4
    C = 2 * Hk * d + Hv * d
    tot = C + Hv * d + 2 * Hv
    tot += (-tot) % 8
    bf = torch.bfloat16
    y = torch.randn(n, tot, generator=g).to(bf).to(DEV)
    mixed, z = y[:, :C], y[:, C:C + Hv * d]
    b, a = y[:, C + Hv * d:C + Hv * d + Hv], y[:, C + Hv * d + Hv:C + Hv * d + 2 * Hv]
    A_log = torch.log(torch.empty(Hv).uniform_(1, 16, generator=g)).to(DEV)
    dt_bias = (torch.rand(Hv, generator=g) * 2 - 1).to(DEV)
    cw = (torch.rand(C, K, generator=g) - 0.5).to(bf).to(DEV)
    nw = (1 + 0.1 * torch.randn(d, generator=g)).to(bf).to(DEV)
    cpool = torch.randn(S, C, K, generator=g).to(bf).to(DEV)
    rpool = (torch.randn(S, Hv, d, d, generator=g) * 0.05).to(DEV)
    slot = torch.randperm(S, generator=g)[:n].to(torch.int32).to(DEV)
    outs = []
    for strided in (True, False):
        cp, rp = cpool.clone(), rpool.clone()
        args = (mixed, z, a, b) if strided else tuple(t.contiguous() for t in (mixed, z, a, b))
        if strided:
            assert not args[1].is_contiguous() and not args[2].is_contiguous()
        o = ops.decode_layer(*args, A_log, dt_bias, cw, None, cp, rp, slot, nw, 1e-6, Hk, Hv, d, d,
                             ops.GDN_CONV_HF)
        torch.cuda.synchronize()
        outs.append((o, cp, rp))
    for x, y_ in zip(outs[0], outs[1]):
        assert torch.equal(x, y_)
