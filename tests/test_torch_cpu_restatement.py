"""Pin the torch CPU restatement (oracle/gdn_torch_cpu.py) that bench.py's CPU legs time.

It restates the reference's path with torch ops in the reference's dtypes (so it runs on the
host cores the way the reference's own torch code does); these tests hold it to the same golden
vectors as the numpy oracle, with the same tolerances (bf16: within 2e-2 max-abs plus one bf16
rounding step; states: 2e-2 max-abs; conv and slot states bit-exact).
"""
import numpy as np
import torch

from conftest import load_golden
from oracle import gdn_oracle as O
from oracle import gdn_torch_cpu as TC

bf = torch.bfloat16


def T(a, dt=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dt)


def bf16_close(a, b, atol=2e-2):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return bool(np.all(np.abs(a - b) <= atol + np.abs(b) * 2.0 ** -7))


def test_chunk_bf16_matches_golden():
    d = load_golden("chunk_bf16.npz")
    r = int(d["Hv"]) // int(d["Hk"])
    for b in range(len(d["lens"])):
        q = T(O.repeat_heads(d[f"q{b}"], r), bf)[None]
        k = T(O.repeat_heads(d[f"k{b}"], r), bf)[None]
        o, s = TC.chunk_gated_delta_rule(q, k, T(d[f"v{b}"], bf)[None], T(d[f"g{b}"])[None],
                                         T(d[f"beta{b}"], bf)[None], 64, T(d[f"init{b}"])[None], True, True)
        assert bf16_close(o[0].float().numpy(), d[f"out{b}"])
        assert np.abs(s[0].numpy() - d[f"state{b}"]).max() < 2e-2


def test_chunk_fp32_matches_golden():
    d = load_golden("chunk_c0init_f32.npz")
    r = int(d["Hv"]) // int(d["Hk"])
    for b in range(len(d["lens"])):
        q, k = T(O.repeat_heads(d[f"q{b}"], r))[None], T(O.repeat_heads(d[f"k{b}"], r))[None]
        o, s = TC.chunk_gated_delta_rule(q, k, T(d[f"v{b}"])[None], T(d[f"g{b}"])[None], T(d[f"beta{b}"])[None],
                                         64, T(d[f"init{b}"])[None], True, True)
        scale = np.abs(d[f"out{b}"]).max()
        assert np.abs(o[0].numpy() - d[f"out{b}"]).max() < 1e-4 * scale
        assert np.abs(s[0].numpy() - d[f"state{b}"]).max() < 1e-4 * np.abs(d[f"state{b}"]).max()


def test_recurrent_step_matches_golden():
    d = load_golden("recurrent_bf16.npz")
    r = d["v"].shape[1] // d["q"].shape[1]
    q = TC.l2norm(T(d["q"], bf)).repeat_interleave(r, dim=1)
    k = TC.l2norm(T(d["k"], bf)).repeat_interleave(r, dim=1)
    S0 = T(d["pool"])[torch.from_numpy(d["slot_idx"].astype(np.int64))]
    o, S = TC.recurrent_step(q, k, T(d["v"], bf), T(d["g"]), T(d["beta"], bf), S0)
    assert bf16_close(o.float().numpy(), d["out"], atol=1e-2)
    assert np.abs(S.numpy() - d["new_state"]).max() < 1e-5


def test_elem_conv_and_norm_match_golden():
    d = load_golden("conv_bf16.npz")
    st = T(d["s0"], bf)
    for t in range(3):
        y = TC.elem_conv_update(T(d["xs"][t][..., 0], bf), st, T(d["w"], bf), T(d["b"], bf))
        assert np.array_equal(st.float().numpy(), d["st_elem"][t])
        assert np.abs(y.float().numpy() - d["y_elem"][t][..., 0]).max() <= 2 ** -6
    n = load_golden("norm_bf16.npz")
    y = TC.gated_rmsnorm(T(n["x"], bf), T(n["z"], bf), T(n["w"], bf))
    assert bf16_close(y.float().numpy(), n["y"], atol=0)


def test_decode_layer_matches_numpy_oracle():
    rng = np.random.default_rng(5)
    n, S, Hk, Hv, d, K = 3, 5, 1, 3, 128, 4
    C = 2 * Hk * d + Hv * d
    r16 = lambda a: O.bf16(np.asarray(a, np.float32))
    mixed, z = r16(rng.standard_normal((n, C))), r16(rng.standard_normal((n, Hv, d)))
    a, b = r16(rng.standard_normal((n, Hv))), r16(rng.standard_normal((n, Hv)))
    A_log = np.log(rng.uniform(1, 16, Hv)).astype(np.float32)
    dt_bias = rng.uniform(-1, 1, Hv).astype(np.float32)
    conv_w, norm_w = r16(rng.uniform(-0.5, 0.5, (C, K))), r16(1 + 0.1 * rng.standard_normal(d))
    conv_pool = r16(rng.standard_normal((S, C, K)))
    rec_pool = (rng.standard_normal((S, Hv, d, d)) * 0.05).astype(np.float32)
    slot = np.array([4, 0, 2], np.int32)
    # numpy oracle composition
    cp, rp = conv_pool.copy(), rec_pool.copy()
    st = cp[slot]
    y = O.conv_update_elem(mixed[:, :, None], st, conv_w, None, "bf16")[:, :, 0]
    cp[slot] = st
    beta, g = O.decode_gates(a, b, A_log, dt_bias, "bf16")
    core = O.decode_step_slots(y[:, :Hk * d].reshape(n, Hk, d), y[:, Hk * d:2 * Hk * d].reshape(n, Hk, d),
                               y[:, 2 * Hk * d:].reshape(n, Hv, d), g, beta, rp, slot, True, "bf16")
    ref = O.gated_rmsnorm(core, z, norm_w, 1e-6, "bf16")
    # torch restatement
    cpt, rpt = T(conv_pool, bf), T(rec_pool)
    out = TC.decode_layer(T(mixed, bf), T(z, bf), T(a, bf), T(b, bf), T(A_log), T(dt_bias), T(conv_w, bf), cpt, rpt,
                          torch.from_numpy(slot.astype(np.int64)), T(norm_w, bf), Hk, Hv, d)
    assert np.array_equal(cpt.float().numpy(), cp)
    assert np.abs(rpt.numpy() - rp).max() < 1e-4
    assert bf16_close(out.float().numpy(), ref)


def test_installed_reference_reproduces_golden():
    """When oracle/_ref holds the reference's own modules (oracle/install_ref.py), the baseline that
    bench.py times is the code that wrote the golden vectors: it must reproduce them bit for bit."""
    import pytest
    from oracle import ref_cpu
    if not ref_cpu.available():
        pytest.skip("the reference is not installed in oracle/_ref")
    d = load_golden("chunk_bf16.npz")
    r = int(d["Hv"]) // int(d["Hk"])
    for b in range(len(d["lens"])):
        q = T(O.repeat_heads(d[f"q{b}"], r), bf)[None]
        k = T(O.repeat_heads(d[f"k{b}"], r), bf)[None]
        o, s = ref_cpu.chunk_prefill(q, k, T(d[f"v{b}"], bf)[None], T(d[f"g{b}"])[None], T(d[f"beta{b}"], bf)[None],
                                     T(d[f"init{b}"])[None])
        assert np.array_equal(o[0].float().numpy(), d[f"out{b}"])
        assert np.array_equal(s[0].numpy(), d[f"state{b}"])
