"""The fused decode layer for callers that cannot allocate device memory.

gdn_decode_layer_noalloc is for hosts that never let this library call cudaMalloc: a serving
runtime that owns the whole device-memory budget and hands over only the tensors to work on, or
a decode loop that cannot afford cudaMalloc's implicit synchronisation.  It takes its workspace
from a fixed array inside the library instead of from the caller.  This test calls it through
the C ABI and checks it against gdn_decode_layer (the entry point that takes a caller-owned
workspace) on two consecutive decode steps, with the same tolerances as the other GPU tests
(2e-2 max-abs on outputs and states, bit-exact conv-state placement).  The file is named so
that pytest collects it last.
"""
import ctypes

import pytest
import torch

from conftest import pkg

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _inputs(seed, n=16, S=20, Hk=16, Hv=48, d=128, K=4):
    g = torch.Generator(device="cpu").manual_seed(seed)
    C = 2 * Hk * d + Hv * d
    bf = torch.bfloat16
    return dict(
        mixed=torch.randn(n, C, generator=g).to(bf).to(DEV),
        z=torch.randn(n, Hv, d, generator=g).to(bf).to(DEV),
        a=torch.randn(n, Hv, generator=g).to(bf).to(DEV),
        b=torch.randn(n, Hv, generator=g).to(bf).to(DEV),
        A_log=torch.log(torch.empty(Hv).uniform_(1, 16, generator=g)).to(DEV),
        dt_bias=(torch.rand(Hv, generator=g) * 2 - 1).to(DEV),
        conv_w=(torch.rand(C, K, generator=g) - 0.5).to(bf).to(DEV),
        norm_w=(1 + 0.1 * torch.randn(d, generator=g)).to(bf).to(DEV),
        conv_pool=torch.randn(S, C, K, generator=g).to(bf).to(DEV),
        rec_pool=(torch.randn(S, Hv, d, d, generator=g) * 0.05).to(DEV),
        slot=torch.randperm(S, generator=g)[:n].to(torch.int32).to(DEV),
        dims=(n, Hk, Hv, d, K),
    )


def _call(lib, x, conv_pool, rec_pool, out, workspace):
    n, Hk, Hv, d, K = x["dims"]
    stream = torch.cuda.current_stream().cuda_stream
    args = [x["mixed"].data_ptr(), x["mixed"].stride(0), x["z"].data_ptr(), x["a"].data_ptr(), x["b"].data_ptr(),
            x["A_log"].data_ptr(), x["dt_bias"].data_ptr(), x["conv_w"].data_ptr(), None, conv_pool.data_ptr(),
            rec_pool.data_ptr(), x["slot"].data_ptr(), conv_pool.shape[0], x["norm_w"].data_ptr(), 1e-6,
            out.data_ptr(), n, Hk, Hv, d, d, K, 1]
    if workspace is None:
        return lib.gdn_decode_layer_noalloc(*args, 1, None, stream)
    return lib.gdn_decode_layer(*args, workspace.data_ptr(), workspace.numel(), 1, None, stream)


def test_noalloc_decode_matches_workspace_entry_point_two_steps():
    if not torch.cuda.is_available():
        pytest.fail("no CUDA device")
    L = pkg("_lib")
    lib = L.load()
    x = _inputs(0)
    n, Hk, Hv, d, K = x["dims"]
    need = lib.gdn_decode_layer_workspace_size(n, Hk, Hv, d, d, 1)
    assert need <= lib.gdn_decode_layer_noalloc_max_bytes()
    ws = torch.zeros(need, dtype=torch.uint8, device=DEV)   # the workspace starts zero-filled
    conv_a, rec_a = x["conv_pool"].clone(), x["rec_pool"].clone()
    conv_b, rec_b = x["conv_pool"].clone(), x["rec_pool"].clone()
    out_a = torch.empty(n, Hv, d, dtype=torch.bfloat16, device=DEV)
    out_b = torch.empty_like(out_a)
    for step in range(2):                  # two calls in a row: the state carries over
        x["mixed"] = torch.randn(n, x["mixed"].shape[1], device=DEV).to(torch.bfloat16)
        L.check(_call(lib, x, conv_a, rec_a, out_a, ws), "gdn_decode_layer")
        L.check(_call(lib, x, conv_b, rec_b, out_b, None), "gdn_decode_layer_noalloc")
        torch.cuda.synchronize()
        assert (out_a.float() - out_b.float()).abs().max().item() <= 2e-2, step
        assert (rec_a - rec_b).abs().max().item() <= 2e-2, step
        assert torch.equal(conv_a, conv_b), step
        assert torch.isfinite(out_b.float()).all()


def test_noalloc_rejects_requests_beyond_its_array():
    L = pkg("_lib")
    lib = L.load()
    cap = lib.gdn_decode_layer_noalloc_max_bytes()
    n = 1
    while lib.gdn_decode_layer_workspace_size(n, 16, 48, 128, 128, 1) <= cap:
        n *= 2                         # a slot count whose workspace does not fit
    rc = lib.gdn_decode_layer_noalloc(*([None, 0] + [None] * 10 + [1, None, 1e-6, None]),
                                      n, 16, 48, 128, 128, 4, 1, 1, None, None)
    assert rc == 5 and b"scratch" in lib.gdn_last_error()
