"""The fused decode layer for callers that cannot allocate device memory.

gdn_decode_layer_noalloc is for hosts that never let this library call cudaMalloc: a serving
runtime that owns the whole device-memory budget and hands over only the tensors to work on, or
a decode loop that cannot afford cudaMalloc's implicit synchronisation.  It takes its workspace
from a fixed array inside the library instead of from the caller.  These tests call it through
the C ABI and check it against gdn_decode_layer (the entry point that takes a caller-owned,
zero-filled workspace): both launch the same kernels on the same inputs, so outputs, recurrent
states and conv states must agree bit for bit, call after call.  The d = 64 path keeps ticket
counters in the library's array that must be back at zero after every call; running it several
times in a row, and after and before d = 128 calls (which use the other part of the array), shows
that they are.  The file is named so that pytest collects it last.
"""
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


class _Pair:
    """One decode layer run twice per step: with a caller workspace (a) and without one (b)."""

    def __init__(self, lib, seed, **shape):
        self.lib = lib
        self.x = _inputs(seed, **shape)
        n, Hk, Hv, d, _ = self.x["dims"]
        need = lib.gdn_decode_layer_workspace_size(n, Hk, Hv, d, d, 1)
        cap = (lib.gdn_decode_layer_noalloc_max_bytes() if d == 128
               else lib.gdn_decode_layer_noalloc_max_ticket_bytes())
        assert need <= cap
        self.ws = torch.zeros(need, dtype=torch.uint8, device=DEV)  # the workspace starts zero-filled
        self.conv = [self.x["conv_pool"].clone(), self.x["conv_pool"].clone()]
        self.rec = [self.x["rec_pool"].clone(), self.x["rec_pool"].clone()]
        self.out = [torch.empty(n, Hv, d, dtype=torch.bfloat16, device=DEV) for _ in range(2)]

    def step(self, L, what):
        x = self.x
        x["mixed"] = torch.randn(x["mixed"].shape, device=DEV).to(torch.bfloat16)
        L.check(_call(self.lib, x, self.conv[0], self.rec[0], self.out[0], self.ws), "gdn_decode_layer")
        L.check(_call(self.lib, x, self.conv[1], self.rec[1], self.out[1], None), "gdn_decode_layer_noalloc")
        torch.cuda.synchronize()
        assert torch.equal(self.out[0], self.out[1]), what
        assert torch.equal(self.rec[0], self.rec[1]), what
        assert torch.equal(self.conv[0], self.conv[1]), what
        assert torch.isfinite(self.out[1].float()).all(), what
        assert not torch.equal(self.rec[1], self.x["rec_pool"]), what   # the layer did update the states


def test_noalloc_decode_matches_workspace_entry_point_two_steps():
    L = pkg("_lib")
    lib = L.load()
    pair = _Pair(lib, 0)
    for step in range(2):                  # two calls in a row: the state carries over
        pair.step(L, f"d=128 step {step}")


def test_noalloc_decode_d64_tickets_return_to_zero():
    """Four d = 64 calls in a row: each must start from zeroed ticket counters in the shared array."""
    L = pkg("_lib")
    lib = L.load()
    pair = _Pair(lib, 1, n=6, S=9, Hk=4, Hv=12, d=64)
    for step in range(4):
        pair.step(L, f"d=64 step {step}")


def test_noalloc_decode_d128_and_d64_calls_interleaved():
    """d = 128 calls write their prepared rows into one part of the array and must leave the d = 64
    ticket counters (the other part) at zero: 128, 64, 128, 64."""
    L = pkg("_lib")
    lib = L.load()
    wide = _Pair(lib, 2, n=16, S=20)
    narrow = _Pair(lib, 3, n=5, S=7, Hk=2, Hv=8, d=64)
    for step in range(2):
        wide.step(L, f"interleaved d=128 step {step}")
        narrow.step(L, f"interleaved d=64 step {step}")


def test_noalloc_rejects_requests_beyond_its_array():
    L = pkg("_lib")
    lib = L.load()
    for d, cap in ((128, lib.gdn_decode_layer_noalloc_max_bytes()),
                   (64, lib.gdn_decode_layer_noalloc_max_ticket_bytes())):
        n = 1
        while lib.gdn_decode_layer_workspace_size(n, 16, 48, d, d, 1) <= cap:
            n *= 2                         # a slot count whose workspace does not fit
        rc = lib.gdn_decode_layer_noalloc(*([None, 0] + [None] * 10 + [1, None, 1e-6, None]),
                                          n, 16, 48, d, d, 4, 1, 1, None, None)
        assert rc == 5 and b"scratch" in lib.gdn_last_error(), d
