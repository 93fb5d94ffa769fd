"""Pin the CPU oracle (oracle/gdn_oracle.py) against golden vectors produced by the reference.

The fixtures come from tests/golden/make_golden.py, which runs the reference's own torch
functions.  Tolerances: fp32 paths <= 1e-4 relative (to the max magnitude); bf16 paths
compare bf16-rounded outputs to within 2e-2 max-abs (state) or one bf16 rounding step.
"""
import numpy as np
import pytest

from conftest import load_golden
from oracle import gdn_oracle as O


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.abs(a - b).max() / max(np.abs(b).max(), 1e-30)


def bf16_close(a, b, atol=2e-2):
    """|a-b| <= atol + one bf16 ulp of |b| (2^-7 relative)."""
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return bool(np.all(np.abs(a - b) <= atol + np.abs(b) * 2.0 ** -7))


@pytest.mark.parametrize("name", ["chunk_c0_f32.npz", "chunk_c0init_f32.npz"])
def test_chunk_fp32_matches_reference_v2(name):
    d = load_golden(name)
    r = int(d["Hv"]) // int(d["Hk"])
    for b, L in enumerate(d["lens"]):
        q, k = O.repeat_heads(d[f"q{b}"], r)[None], O.repeat_heads(d[f"k{b}"], r)[None]
        init = d[f"init{b}"][None] if f"init{b}" in d else None
        o, s = O.chunk_gated_delta_rule(q, k, d[f"v{b}"][None], d[f"g{b}"][None], d[f"beta{b}"][None],
                                        64, init, True, True, "f32")
        assert rel(o[0], d[f"out{b}"]) < 1e-4
        assert rel(s[0], d[f"state{b}"]) < 1e-4
        # the reference's own variants agree with v2 (recorded by the generator)
        for tag in ("v1", "hfchunk", "hfrec"):
            assert d[f"maxdiff_out_{tag}_{b}"] < 1e-4 * np.abs(d[f"out{b}"]).max()


def test_chunk_fp32_equals_token_recurrence():
    """Config 0: chunked output and final state == the token-by-token recurrence."""
    d = load_golden("chunk_c0_f32.npz")
    r = int(d["Hv"]) // int(d["Hk"])
    for b in range(len(d["lens"])):
        args = (O.repeat_heads(d[f"q{b}"], r)[None], O.repeat_heads(d[f"k{b}"], r)[None],
                d[f"v{b}"][None], d[f"g{b}"][None], d[f"beta{b}"][None])
        oc, sc = O.chunk_gated_delta_rule(*args, 64, None, True, True, "f32")
        orr, sr = O.recurrent_gated_delta_rule(*args, None, True, True, "f32")
        assert rel(oc, orr) < 1e-4 and rel(sc, sr) < 1e-4


def test_chunk_bf16_matches_reference_v2():
    d = load_golden("chunk_bf16.npz")
    r = int(d["Hv"]) // int(d["Hk"])
    for b, L in enumerate(d["lens"]):
        q, k = O.repeat_heads(d[f"q{b}"], r)[None], O.repeat_heads(d[f"k{b}"], r)[None]
        o, s = O.chunk_gated_delta_rule(q, k, d[f"v{b}"][None], d[f"g{b}"][None], d[f"beta{b}"][None],
                                        64, d[f"init{b}"][None], True, True, "bf16")
        assert bf16_close(o[0], d[f"out{b}"])
        assert np.abs(s[0] - d[f"state{b}"]).max() < 2e-2


def test_recurrent_bf16_matches_reference():
    d = load_golden("recurrent_bf16.npz")
    pool = d["pool"].copy()
    o = O.decode_step_slots(d["q"], d["k"], d["v"], d["g"], d["beta"], pool, d["slot_idx"], True, "bf16")
    assert bf16_close(o, d["out"], atol=1e-2)
    assert np.abs(pool[d["slot_idx"]] - d["new_state"]).max() < 1e-5
    untouched = np.setdiff1d(np.arange(pool.shape[0]), d["slot_idx"])
    assert np.array_equal(pool[untouched], d["pool"][untouched])
    r = d["v3"].shape[1] // d["q3"].shape[1]
    o3, s3 = O.recurrent_gated_delta_rule(O.repeat_heads(d["q3"], r)[None], O.repeat_heads(d["k3"], r)[None],
                                          d["v3"][None], d["g3"][None], d["beta3"][None], d["init3"][None],
                                          True, True, "bf16")
    assert bf16_close(o3[0], d["out3"], atol=1e-2)
    assert np.abs(s3[0] - d["state3"]).max() < 1e-5


def test_conv_update_matches_reference():
    d = load_golden("conv_bf16.npz")
    se, sh = d["s0"].copy(), d["s0"].copy()
    for t in range(3):
        ye = O.conv_update_elem(d["xs"][t], se, d["w"], d["b"], "bf16")
        yh = O.conv_update(d["xs"][t], sh, d["w"], d["b"], "bf16")
        # state is pure data movement: bit-exact
        assert np.array_equal(se, d["st_elem"][t]) and np.array_equal(sh, d["st_hf"][t])
        assert bf16_close(ye, d["y_elem"][t], atol=0) or np.abs(ye - d["y_elem"][t]).max() <= 2 ** -6
        assert bf16_close(yh, d["y_hf"][t], atol=1e-2)
    s2 = d["s0"].copy()
    y2 = O.conv_update(d["x2"], s2, d["w"], None, "bf16")
    assert np.array_equal(s2, d["s2_after"])
    assert bf16_close(y2, d["y2"], atol=1e-2)


def test_prefill_conv_matches_reference():
    d = load_golden("prefill_conv_bf16.npz")
    lens = d["lens"]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    y, st = O.prefill_conv(d["x"], cu, d["w"], None, None, "bf16")
    assert bf16_close(y, d["y"], atol=1e-2)
    assert np.array_equal(st, d["st"])
    yc, stc = O.prefill_conv(d["xc"], np.array([0, d["xc"].shape[0]], np.int32), d["w"], None,
                             d["prev"][None], "bf16")
    assert bf16_close(yc, d["yc"], atol=1e-2)
    assert np.array_equal(stc[0], d["stc"])


def test_gated_norm_matches_reference():
    d = load_golden("norm_bf16.npz")
    y = O.gated_rmsnorm(d["x"], d["z"], d["w"], 1e-6, "bf16")
    assert bf16_close(y, d["y"], atol=0)
    n_diff = int((y != d["y"]).sum())
    assert n_diff <= y.size // 100          # bit-equal except rare 1-ulp ties
    y32 = O.gated_rmsnorm(d["x"], d["z"], d["w"], 1e-6, "f32")
    assert rel(y32, d["y32"]) < 1e-5


def test_gates_match_reference():
    d = load_golden("gates_bf16.npz")
    beta, g = O.decode_gates(d["a"], d["b"], d["A_log"], d["dt_bias"], "bf16")
    assert np.array_equal(beta, d["beta"])
    assert rel(g, d["g"]) < 1e-6


def test_unit_lower_inv_is_inverse():
    rng = np.random.default_rng(0)
    X = np.tril(rng.standard_normal((3, 64, 64)).astype(np.float32) * 0.1, -1)
    T = O.unit_lower_inv(X)
    eye = np.eye(64, dtype=np.float32)
    assert np.abs(np.matmul(eye - X, T) - eye).max() < 1e-5


def test_bf16_rounding_known_values():
    x = np.array([1.0, 1.00390625, 1.005859375, -3.0e-3, 65504.0], np.float32)
    u = O.bf16_bits(x)
    assert u[0] == 0x3F80 and u[1] == 0x3F80          # 1 + 2^-8 is a tie -> even (1.0)
    assert u[2] == 0x3F81                              # above the tie -> rounds up
    assert np.array_equal(O.from_bf16_bits(u), O.bf16(x))


def test_empty_sequences_are_the_zero_chunk_limit():
    """Packed prefill with empty sequences (the library's definition; the reference's chunk function
    raises on L = 0): no output rows, final state = initial state or zeros, and the other sequences
    unchanged by the empty ones around them; the prefill conv keeps the carried window or zeros."""
    rng = np.random.default_rng(31)
    Hk, Hv, d = 1, 2, 64
    lens_a, lens_b = [0, 70, 0, 5, 0], [70, 5]
    Tt = sum(lens_a)
    q = rng.standard_normal((Tt, Hk, d)).astype(np.float32)
    k = rng.standard_normal((Tt, Hk, d)).astype(np.float32)
    v = rng.standard_normal((Tt, Hv, d)).astype(np.float32)
    g = -rng.uniform(0.01, 1, (Tt, Hv)).astype(np.float32)
    be = rng.uniform(0, 1, (Tt, Hv)).astype(np.float32)
    pool0 = (0.1 * rng.standard_normal((6, Hv, d, d))).astype(np.float32)
    cu_a = np.concatenate([[0], np.cumsum(lens_a)]).astype(np.int32)
    cu_b = np.concatenate([[0], np.cumsum(lens_b)]).astype(np.int32)
    pa, pb = pool0.copy(), pool0.copy()
    oa, _ = O.prefill_varlen(q, k, v, g, be, cu_a, pa, np.array([1, 2, 3, 4, 5]), np.array([1, 1, 0, 1, 0]), True, "f32")
    ob, _ = O.prefill_varlen(q, k, v, g, be, cu_b, pb, np.array([2, 4]), np.array([1, 1]), True, "f32")
    assert oa.shape == (Tt, Hv, d) and np.array_equal(oa, ob)
    assert np.array_equal(pa[2], pb[2]) and np.array_equal(pa[4], pb[4])
    assert np.array_equal(pa[1], pool0[1])           # empty, from its initial state
    assert not pa[3].any() and not pa[5].any()       # empty, from zeros
    # conv: an empty sequence keeps its window (carried) or gets zeros
    C, K = 8, 4
    x = rng.standard_normal((Tt, C)).astype(np.float32)
    w = rng.uniform(-0.5, 0.5, (C, K)).astype(np.float32)
    init = rng.standard_normal((len(lens_a), C, K)).astype(np.float32)
    y, st = O.prefill_conv(x, cu_a, w, None, init, "f32")
    assert np.array_equal(st[0], init[0]) and np.array_equal(st[2], init[2])
    y0, st0 = O.prefill_conv(x, cu_a, w, None, None, "f32")
    assert not st0[0].any() and not st0[4].any()

