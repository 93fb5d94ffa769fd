"""Residual add fused with the next layer norm (gdn_add_rmsnorm, ops.add_rmsnorm), and the MLP
activation silu(gate) * up in one kernel (gdn_silu_mul).

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


@pytest.mark.parametrize("rows,inter", [(16, 17408), (128, 2176), (1, 8), (33, 4352)])
def test_silu_mul_bit_exact(rows, inter):
    ops = pkg("ops")
    g = torch.Generator(device="cpu").manual_seed(rows + inter)
    y = (torch.randn(rows, 1, 2 * inter + 8, generator=g) * 4).to(torch.bfloat16).to(DEV)   # padded fused rows
    ref = torch.nn.functional.silu(y[..., :inter]) * y[..., inter:2 * inter]
    got = ops.silu_mul(y, inter)
    torch.cuda.synchronize()
    assert torch.equal(got, ref)


@pytest.mark.parametrize("n,Hq,kvh,hd,rd", [(16, 24, 4, 256, 64), (32, 12, 2, 256, 64), (128, 3, 1, 256, 64),
                                           (5, 4, 1, 64, 16), (7, 2, 2, 128, 128)])
def test_attn_decode_prep_bit_exact(n, Hq, kvh, hd, rd):
    """q/k RMSNorm + partial rotary + the attn_decode layout in one kernel, against the torch
    sequence of CBEngine._attn (the patched Qwen3_5RMSNorm and HF's apply_rotary_pos_emb)."""
    from transformers.models.qwen3_5 import modeling_qwen3_5 as M
    ops = pkg("ops")
    g = torch.Generator(device="cpu").manual_seed(n * 7 + Hq + hd)
    nq, nk = 2 * Hq * hd, kvh * hd
    y = (torch.randn(n, 1, nq + 2 * nk + 8, generator=g) * 2).to(torch.bfloat16).to(DEV)   # padded fused rows
    qw = (torch.randn(hd, generator=g) * 0.2).to(torch.bfloat16).to(DEV)
    kw = (torch.randn(hd, generator=g) * 0.2).to(torch.bfloat16).to(DEV)
    ang = torch.rand(n, 1, rd, generator=g) * 6.3
    cos, sin = ang.cos().to(torch.bfloat16).to(DEV), ang.sin().to(torch.bfloat16).to(DEV)
    qg = y[..., :nq].view(n, 1, -1, hd * 2)
    q, gate = torch.chunk(qg, 2, dim=-1)
    q = ops.rmsnorm(q, qw, 1e-6).transpose(1, 2)
    k = ops.rmsnorm(y[..., nq:nq + nk].view(n, 1, kvh, hd), kw, 1e-6).transpose(1, 2)
    v = y[..., nq + nk:nq + 2 * nk].view(n, 1, kvh, hd).transpose(1, 2)
    q, k = M.apply_rotary_pos_emb(q, k, cos, sin)
    gq, gk, gv, gg = ops.attn_decode_prep(y.view(n, -1), qw, kw, 1e-6, cos, sin, Hq, kvh, hd)
    torch.cuda.synchronize()
    assert torch.equal(gq, q[:, :, 0]) and torch.equal(gk, k[:, :, 0])
    assert torch.equal(gv, v[:, :, 0]) and torch.equal(gg, gate.reshape(n, Hq, hd))
