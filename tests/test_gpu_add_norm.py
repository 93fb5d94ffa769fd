"""Residual add fused with the next layer norm (gdn_add_rmsnorm, ops.add_rmsnorm).

The decode step's ``x = x + h`` followed by Qwen3_5RMSNorm runs as one kernel that keeps the
element-to-thread map, summation order and arithmetic of the plain RMSNorm kernel, so it must equal
``x + h`` (torch, bf16) then ops.rmsnorm BIT FOR BIT, for the model width (5,120), the widths of the
small test models, the widest row the kernel takes (8,192) and 1-128 rows, with the residual x
updated in place and row-strided inputs and outputs.
"""
import pytest
import torch

from conftest import pkg

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.mark.parametrize("rows,dim", [(1, 5120), (16, 5120), (128, 5120), (7, 256), (3, 8192), (32, 2048), (5, 8)])
def test_add_rmsnorm_bit_exact(rows, dim):
    ops = pkg("ops")
    g = torch.Generator(device="cpu").manual_seed(rows * 31 + dim)
    x = (torch.randn(rows, 1, dim, generator=g) * 3).to(torch.bfloat16).to(DEV)
    h = (torch.randn(rows, 1, dim, generator=g) * 5).to(torch.bfloat16).to(DEV)
    w = (torch.randn(dim, generator=g) * 0.1).to(torch.bfloat16).to(DEV)
    ref_x = x + h
    ref = ops.rmsnorm(ref_x, w, 1e-6)
    out = ops.add_rmsnorm(x, h, w, 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(x, ref_x)          # the residual stream, updated in place
    assert torch.equal(out, ref)


def test_add_rmsnorm_strided_rows():
    ops = pkg("ops")
    g = torch.Generator(device="cpu").manual_seed(9)
    xb = torch.randn(6, 5200, generator=g).to(torch.bfloat16).to(DEV)
    hb = torch.randn(6, 5200, generator=g).to(torch.bfloat16).to(DEV)
    w = (torch.randn(5120, generator=g) * 0.1).to(torch.bfloat16).to(DEV)
    x, h = xb[:, 40:5160], hb[:, 80:5200]
    ref_x = x + h
    ref = ops.rmsnorm(ref_x.contiguous(), w, 1e-6)
    outb = torch.zeros(6, 5248, dtype=torch.bfloat16, device=DEV)
    L = pkg("_lib")
    L.check(L.load().gdn_add_rmsnorm(x.data_ptr(), 5200, h.data_ptr(), 5200, w.data_ptr(), outb[:, 64:].data_ptr(),
                                     5248, 6, 5120, 1e-6, L.GDN_BF16, torch.cuda.current_stream().cuda_stream),
            "gdn_add_rmsnorm")
    torch.cuda.synchronize()
    assert torch.equal(x, ref_x) and torch.equal(outb[:, 64:5184], ref)
    assert (outb[:, :64] == 0).all() and (outb[:, 5184:] == 0).all()
