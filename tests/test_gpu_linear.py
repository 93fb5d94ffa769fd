"""Decode projections on the tensor cores (gdn_linear) against an fp64 torch reference.

gdn_linear computes y = x W^T with bf16 operands, fp32 accumulation (the K range of each 128-feature
tile split over the CTAs of a cluster, summed through distributed shared memory in split order) and
one rounding to bf16.  Against the exact (fp64)
product of the same bf16 inputs, every element must be within half a bf16 step of the reference
(the rounding, 2^-8 |ref|) plus twice the fp32 accumulation error bound, k * 2^-23 * sum |x_i w_i|.
Shapes cover 1-256 tokens (the N dimension is rounded up to 16, rows past n are zero-filled by
TMA), output widths that are and are not multiples of the 128-feature tile, K tails that are not
multiples of the 64-wide stage, every split count 1-8, row-strided views of x, W and y, the model's
decode shapes, and repeated calls (bit-identical).
"""
import pytest
import torch

from conftest import pkg

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _ref_check(y, x, w):
    xf, wf = x.double(), w.double()
    ref = xf @ wf.t()
    mag = xf.abs() @ wf.abs().t()
    k = x.shape[-1]
    tol = ref.abs() * 2.0 ** -8 + mag * (k * 2.0 ** -23) + 1e-30
    err = (y.double() - ref).abs()
    bad = err > tol
    assert not bad.any(), f"{int(bad.sum())} elements off; worst {float((err - tol).max()):.3e} (k={k})"


def _inputs(n, n_out, k, seed, scale=1.0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = (torch.randn(n, k, generator=g) * scale).to(torch.bfloat16).to(DEV)
    w = (torch.randn(n_out, k, generator=g) / k ** 0.5).to(torch.bfloat16).to(DEV)
    return x, w


@pytest.mark.parametrize("n", [1, 5, 16, 17, 32, 64, 100, 128, 129, 200, 256])
@pytest.mark.parametrize("n_out,k", [(8, 8), (136, 72), (2064, 768), (5120, 2176)])
def test_linear_matches_fp32_reference(n, n_out, k):
    ops = pkg("ops")
    x, w = _inputs(n, n_out, k, seed=n * 7 + k)
    y = ops.linear(x, w)
    torch.cuda.synchronize()
    _ref_check(y, x, w)


@pytest.mark.parametrize("splits", [1, 2, 3, 4, 5, 6, 7, 8])
def test_linear_every_split_count(splits):
    ops = pkg("ops")
    x, w = _inputs(32, 1040, 1000, seed=splits)
    y = ops.linear(x, w, splits=splits)
    torch.cuda.synchronize()
    _ref_check(y, x, w)


@pytest.mark.parametrize("n,n_out,k", [
    (16, 5120, 6144),        # out_proj / o_proj, TP 1
    (16, 5120, 17408),       # down_proj, TP 1
    (16, 34816, 5120),       # gate | up, TP 1
    (16, 16488, 5120),       # GDN qkv | z | b | a, TP 1 (padded to a multiple of 8)
    (128, 5120, 2176),       # down_proj, TP 8
    (128, 2064, 5120),       # GDN fused input projection, TP 8
])
def test_linear_model_shapes(n, n_out, k):
    ops = pkg("ops")
    x, w = _inputs(n, n_out, k, seed=n_out + k, scale=3.0)
    y = ops.linear(x, w)
    torch.cuda.synchronize()
    _ref_check(y, x, w)


def test_linear_strided_views_and_determinism():
    ops = pkg("ops")
    g = torch.Generator(device="cpu").manual_seed(5)
    xb = torch.randn(24, 1104, generator=g).to(torch.bfloat16).to(DEV)
    wb = (torch.randn(600, 1104, generator=g) / 30).to(torch.bfloat16).to(DEV)
    x, w = xb[:, 16:1040], wb[40:560, 16:1040]           # row strides 1104, offsets 32 bytes
    yb = torch.full((24, 800), 7.0, dtype=torch.bfloat16, device=DEV)
    y = yb[:, 120:640]                                   # row stride 800
    ops.linear(x, w, out=y)
    y2 = ops.linear(x.contiguous(), w.contiguous())
    torch.cuda.synchronize()
    _ref_check(y, x, w)
    assert torch.equal(y, y2)                            # strides do not change the result
    assert (yb[:, :120] == 7).all() and (yb[:, 640:] == 7).all()   # nothing written outside y
    for _ in range(3):
        assert torch.equal(ops.linear(x, w), y2)


def test_linear_large_output_many_waves():
    """An LM-head-like width (1,940 tiles: several waves of CTAs)."""
    ops = pkg("ops")
    x, w = _inputs(16, 248320, 512, seed=11)
    y = ops.linear(x, w)
    torch.cuda.synchronize()
    _ref_check(y, x, w)


def test_linear_rejects_bad_arguments():
    ops = pkg("ops")
    L = pkg("_lib")
    lib = L.load()
    x, w = _inputs(8, 64, 64, seed=1)
    y = torch.empty(8, 64, dtype=torch.bfloat16, device=DEV)
    s = torch.cuda.current_stream().cuda_stream
    cases = [
        (x.data_ptr(), 64, w.data_ptr(), 64, y.data_ptr(), 64, 0, 64, 64, 0),      # no tokens
        (x.data_ptr(), 64, w.data_ptr(), 64, y.data_ptr(), 64, 257, 64, 64, 0),    # > 256 tokens
        (x.data_ptr(), 64, w.data_ptr(), 64, y.data_ptr(), 64, 8, 60, 64, 0),      # n_out not a multiple of 8
        (x.data_ptr(), 64, w.data_ptr(), 64, y.data_ptr(), 64, 8, 64, 60, 0),      # k not a multiple of 8
        (x.data_ptr() + 2, 64, w.data_ptr(), 64, y.data_ptr(), 64, 8, 64, 64, 0),  # misaligned x
        (x.data_ptr(), 60, w.data_ptr(), 64, y.data_ptr(), 64, 8, 64, 56, 0),      # stride not a multiple of 8
        (x.data_ptr(), 64, w.data_ptr(), 64, y.data_ptr(), 64, 8, 64, 64, 9),      # splits > 8
    ]
    for c in cases:
        assert lib.gdn_linear(*c, L.GDN_BF16, None, s) != 0
        assert lib.gdn_last_error()
    assert lib.gdn_linear(x.data_ptr(), 64, w.data_ptr(), 64, y.data_ptr(), 64, 8, 64, 64, 0, L.GDN_F32, None, s) != 0
    with pytest.raises(RuntimeError):
        ops.linear(x.cpu(), w.cpu())
