"""Long-sequence parity of the tensor-core chunk prefill (chunk_tc_kernel).

The tensor-core kernel keeps the state in fp32 but feeds bf16 copies of it (and of vn) to the
tensor cores every chunk, so rounding could in principle build up over many chunks.  These tests
run single sequences of 4,096, 8,192 and 16,384 tokens (64, 128 and 256 chunks; the reference's
TP runs use t_max up to 16,384) with config-1 heads (16 q/k heads, 48 v heads, d = 128) and an
N(0, 0.02) initial state, under two gate distributions: config 1's g = -U(0.01, 1) per token, and a
weak decay g = -U(0.001, 0.02) under which the state remembers ~100 tokens and carries the
rounding of every chunk further.  Each run is checked

  * against the fp32 CUDA-core kernel on every token and head, and
  * against the CPU oracle (the reference's algorithm with its bf16 roundings) on two heads,

within the bf16 tolerance of the other GPU tests (2e-2 max-abs on outputs plus one bf16 rounding
step where |ref| > 1; 2e-2 max-abs on final states).  The errors reached are printed (``-s``).
"""
import numpy as np
import pytest
import torch

from conftest import pkg
from oracle import gdn_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda"
HK, HV, D = 16, 48, 128


def _inputs(L, weak, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(L, HK, D, generator=g)
    k = torch.randn(L, HK, D, generator=g)
    q = (q / q.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    k = (k / k.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    v = torch.randn(L, HV, D, generator=g).to(torch.bfloat16)
    beta = torch.sigmoid(torch.randn(L, HV, generator=g)).to(torch.bfloat16).float()
    lo, hi = (0.001, 0.02) if weak else (0.01, 1.0)
    gg = (-(lo + (hi - lo) * torch.rand(L, HV, generator=g))).to(torch.bfloat16).float()
    init = torch.randn(1, HV, D, D, generator=g) * 0.02
    return q, k, v, gg, beta, init


def _excess(a, b):
    """How far |a - b| goes past the bf16 output tolerance (<= 0 means within it)."""
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float((np.abs(a - b) - (2e-2 + np.abs(b) * 2.0 ** -7)).max())


@pytest.mark.parametrize("weak", [False, True], ids=["config1-gates", "weak-decay"])
@pytest.mark.parametrize("L", [4096, 8192, 16384])
def test_chunk_tc_long_sequence(L, weak):
    if not torch.cuda.is_available():
        pytest.fail("no CUDA device")
    ops = pkg("ops")
    q, k, v, gg, beta, init = _inputs(L, weak, seed=L + weak)
    dq, dk, dv = q.to(DEV), k.to(DEV), v.to(DEV)
    dg, db = gg.to(DEV), beta.to(DEV)
    cu = torch.tensor([0, L], dtype=torch.int32, device=DEV)
    slot = torch.zeros(1, dtype=torch.int32, device=DEV)
    use = torch.ones(1, dtype=torch.int32, device=DEV)
    pool_tc = init.to(DEV).contiguous()
    o_tc = ops.chunk_prefill_varlen(dq, dk, dv, dg, db, cu, pool_tc, slot, use, True)
    pool_32 = init.to(DEV).contiguous()
    o_32 = ops.chunk_prefill_varlen(dq.float(), dk.float(), dv.float(), dg, db, cu, pool_32, slot, use, True)
    torch.cuda.synchronize()
    e_o32 = (o_tc.float() - o_32).abs().max().item()
    e_s32 = (pool_tc - pool_32).abs().max().item()
    x_o32 = _excess(o_tc.float().cpu().numpy(), o_32.cpu().numpy())
    # the oracle on the first and the last value head (k-heads 0 and 15)
    e_or, e_sr, x_or = 0.0, 0.0, -1.0
    for h in (0, HV - 1):
        hk = h // (HV // HK)
        ro, rs = O.chunk_gated_delta_rule(q[:, hk:hk + 1].float().numpy()[None], k[:, hk:hk + 1].float().numpy()[None],
                                          v[:, h:h + 1].float().numpy()[None], gg[:, h:h + 1].numpy()[None],
                                          beta[:, h:h + 1].numpy()[None], 64, init[:, h:h + 1].numpy(), True, True,
                                          "bf16")
        got = o_tc[:, h].float().cpu().numpy()
        e_or = max(e_or, float(np.abs(got - ro[0, :, 0]).max()))
        x_or = max(x_or, _excess(got, ro[0, :, 0]))
        e_sr = max(e_sr, float(np.abs(pool_tc[0, h].cpu().numpy() - rs[0, 0]).max()))
    print(f"\nchunk_tc L={L} {'weak-decay' if weak else 'config1-gates'}: |o|max {o_32.abs().max().item():.3f} "
          f"|S|max {pool_32.abs().max().item():.3f}; vs fp32 kernel: out {e_o32:.2e} state {e_s32:.2e}; "
          f"vs oracle (2 heads): out {e_or:.2e} state {e_sr:.2e}")
    assert x_o32 <= 0 and e_s32 < 2e-2, (e_o32, e_s32)
    assert x_or <= 0 and e_sr < 2e-2, (e_or, e_sr)
