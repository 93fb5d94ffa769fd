"""The C-ABI library loads without a GPU and exports exactly what include/gdn_b200.h declares.

No compute is launched here: the only calls made are ones the library rejects during argument
validation, before any CUDA API call.
"""
import ctypes
import os
import re

import pytest

from conftest import ROOT, pkg

HEADER = os.path.join(ROOT, "include", "gdn_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    out = {}
    for m in re.finditer(r"(?:^|\n)\s*(?:GDN_API\s+)?(?:const\s+)?(\w+\s*\*?)\s+(gdn_\w+)\s*\(([^)]*)\)\s*;", src):
        params = [p.strip() for p in m.group(3).split(",") if p.strip() and p.strip() != "void"]
        out[m.group(2)] = len(params)
    return out


@pytest.fixture(scope="module")
def lib():
    L = pkg("_lib")
    if not os.path.exists(L.LIB_PATH):
        pytest.fail("libgdn_b200.so is not built (run __graft_entry__.build())")
    return L.load()


def test_header_parses():
    fns = declared_functions()
    assert "gdn_chunk_prefill" in fns and "gdn_decode_layer" in fns and len(fns) >= 9


def test_every_declared_symbol_is_exported_and_bound(lib):
    L = pkg("_lib")
    for name, nparams in declared_functions().items():
        assert hasattr(lib, name), f"{name} not exported"
        assert name in L.SIGNATURES, f"{name} has no ctypes signature"
        assert len(L.SIGNATURES[name][1]) == nparams, f"{name}: {nparams} params in header"


def test_no_undeclared_exports(lib):
    # every bound signature corresponds to a header declaration
    L = pkg("_lib")
    assert set(L.SIGNATURES) == set(declared_functions())


def test_validation_errors_without_gpu(lib):
    L = pkg("_lib")
    assert lib.gdn_version() >= 100
    rc = lib.gdn_gated_rmsnorm(None, 0, None, 0, None, None, 0, -1, 128, 1e-6, 1, None)
    assert rc == 1 and b"rows" in lib.gdn_last_error()
    rc = lib.gdn_chunk_prefill(None, 0, None, 0, None, 0, None, None, 0, None, 1, 10, None, None, None, None,
                               None, 0, None, 0, 16, 48, 128, 128, 1, 1, None, None)
    assert rc == 1 and b"null" in lib.gdn_last_error()
    rc = lib.gdn_chunk_prefill_gates(None, 0, None, 0, None, 0, None, None, 0, None, None, None, 1, 10, None, None,
                                     None, None, None, 0, None, 0, 16, 48, 128, 128, 1, 1, None, None)
    assert rc == 1 and b"gdn_chunk_prefill_gates: null" in lib.gdn_last_error()
    rc = lib.gdn_recurrent(*([None, 0, 0] * 3), None, None, 0, 0, None, None, None, None, 0, None, 0, 0,
                           1, 1, 16, 40, 128, 128, 1, 1, None, None)
    assert rc == 2 and b"multiple" in lib.gdn_last_error()
    with pytest.raises(RuntimeError, match="status 2"):
        L.check(2, "probe")
    # dk = 128: prepared q/k/v rows [n, C] bf16 + gates [n, Hv, 4] f32; dk = 64: a ticket per (slot, k-head)
    assert lib.gdn_decode_layer_workspace_size(16, 16, 48, 128, 128, 1) == 16 * 10240 * 2 + 16 * 48 * 16
    assert lib.gdn_decode_layer_workspace_size(16, 4, 8, 64, 64, 1) >= 16 * 4 * 4
    # the d = 128 decode layer bulk-copies rows of z: a z that is not 16-byte aligned is refused before
    # any CUDA call (the other pointers are never dereferenced on this path)
    ok, odd = 4096, 4096 + 2
    rc = lib.gdn_decode_layer(ok, 10240, odd, ok, ok, ok, ok, ok, None, ok, ok, ok, 4, ok, 1e-6, ok, 2, 16, 48,
                              128, 128, 4, L.GDN_CONV_ELEM, ok, 1 << 30, L.GDN_BF16, None, None)
    assert rc == 1 and b"aligned" in lib.gdn_last_error()
    # layer RMSNorm, attention decode and peer all-reduce: argument checks before any CUDA call
    assert lib.gdn_rmsnorm(ok, 8192, ok, ok, 8192, 4, 9000, 1e-6, L.GDN_BF16, None) == 2
    assert b"8192" in lib.gdn_last_error()
    assert lib.gdn_rmsnorm(ok, 64, ok, ok, 64, 0, 64, 1e-6, L.GDN_BF16, None) == 0        # no rows: no-op
    assert lib.gdn_attn_decode_workspace_size(16, 24, 256, 1024) == 16 * 24 * 8 * 258 * 4
    rc = lib.gdn_attn_decode(ok, ok, ok, ok, ok, 17, 1024, ok, ok, 1024, None, 0.0625, ok, 16, 24, 5, 256, ok,
                             1 << 30, L.GDN_BF16, None, None)                          # 24 q heads over 5 kv heads
    assert rc == 2 and b"Hq" in lib.gdn_last_error()
    rc = lib.gdn_attn_decode(ok, ok, ok, ok, ok, 17, 1024, ok, ok, 1024, None, 0.0625, ok, 16, 24, 4, 256, ok,
                             64, L.GDN_BF16, None, None)
    assert rc == 5 and b"workspace" in lib.gdn_last_error()
    assert lib.gdn_ar_buffer_bytes(9, 1024, L.GDN_BF16) == 0                           # world 1..8
    assert lib.gdn_ar_buffer_bytes(2, 1024, L.GDN_BF16) == 16384 + 2 * 2 * 2048
    table = (ctypes.c_void_p * 2)(ok, ok)
    rc = lib.gdn_allreduce(ok, ok, 2048, L.GDN_BF16, 0, 2, table, 1024, 0, None, None)  # n > slot
    assert rc == 1 and b"slot" in lib.gdn_last_error()
    rc = lib.gdn_allreduce(ok, ok, 16, L.GDN_BF16, 2, 2, table, 1024, 0, None, None)    # rank >= world
    assert rc == 1 and b"rank" in lib.gdn_last_error()


def test_decode_projection_and_glue_validation_without_gpu(lib):
    """The f1 projections, the peer exchanges around them and the decode-step glue reject bad
    arguments before any CUDA call (pointers here are never dereferenced)."""
    L = pkg("_lib")
    ok, odd = 4096, 4096 + 2
    BF, F32 = L.GDN_BF16, L.GDN_F32
    table = (ctypes.c_void_p * 2)(ok, ok)

    def rejects(rc, code, text):
        assert rc == code, (rc, lib.gdn_last_error())
        assert text in lib.gdn_last_error(), lib.gdn_last_error()

    # gdn_linear: tokens 1..256, n_out and k multiples of 8, 16-byte alignment, strides, split count
    rejects(lib.gdn_linear(ok, 64, ok, 64, ok, 64, 0, 64, 64, 0, BF, None, None), 1, b"tokens")
    rejects(lib.gdn_linear(ok, 64, ok, 64, ok, 64, 257, 64, 64, 0, BF, None, None), 1, b"tokens")
    rejects(lib.gdn_linear(ok, 64, ok, 64, ok, 64, 8, 60, 64, 0, BF, None, None), 1, b"n_out")
    rejects(lib.gdn_linear(ok, 64, ok, 64, ok, 64, 8, 64, 60, 0, BF, None, None), 1, b"k =")
    rejects(lib.gdn_linear(odd, 64, ok, 64, ok, 64, 8, 64, 64, 0, BF, None, None), 1, b"aligned")
    rejects(lib.gdn_linear(ok, 60, ok, 64, ok, 64, 8, 64, 56, 0, BF, None, None), 1, b"strides")
    rejects(lib.gdn_linear(ok, 64, ok, 64, ok, 64, 8, 64, 64, 9, BF, None, None), 1, b"splits")
    rejects(lib.gdn_linear(ok, 64, ok, 64, ok, 64, 8, 64, 64, 0, F32, None, None), 3, b"bf16")
    plan = (ctypes.c_int32 * 5)()
    rejects(lib.gdn_linear_plan(0, 64, 64, 0, 1, plan), 1, b"gdn_linear_plan")
    # exchange buffers: world 1..8, rows 1..256, widths multiples of 8
    assert lib.gdn_linear_ar_buffer_bytes(9, 16, 5120, BF) == 0
    assert lib.gdn_linear_ar_buffer_bytes(2, 0, 5120, BF) == 0
    assert lib.gdn_linear_ar_buffer_bytes(2, 16, 5124, BF) == 0
    assert lib.gdn_linear_ar_buffer_bytes(2, 16, 5120, BF) > 2 * 2 * 16 * 5120 * 2
    assert lib.gdn_ar_norm_buffer_bytes(9, 16, 5120, BF) == 0
    assert lib.gdn_ar_norm_buffer_bytes(2, 300, 5120, BF) == 0
    assert lib.gdn_ar_norm_buffer_bytes(2, 16, 5120, BF) > 2 * 2 * 16 * 5120 * 2
    # fused projection + sum, and its push / pull halves
    rejects(lib.gdn_linear_allreduce(ok, 64, ok, 64, ok, 64, 8, 64, 64, 0, 2, 2, table, 16, 64, 0, None, BF, None),
            1, b"rank")
    rejects(lib.gdn_linear_allreduce(ok, 64, ok, 64, ok, 64, 32, 64, 64, 0, 0, 2, table, 16, 64, 0, None, BF, None),
            1, b"buffer rows")
    rejects(lib.gdn_linear_allreduce(ok, 64, ok, 64, ok, 64, 8, 128, 64, 0, 0, 2, table, 16, 64, 0, None, BF, None),
            1, b"does not fit")
    rejects(lib.gdn_linear_allreduce(ok, 64, ok, 64, ok, 64, 8, 64, 64, 0, 0, 2, None, 16, 64, 0, None, BF, None),
            1, b"buffer table")
    rejects(lib.gdn_linear_push(ok, 64, ok, 64, 8, 64, 64, 0, 0, 1, table, 16, 64, None, BF, None), 1, b"world")
    rejects(lib.gdn_push_partial(ok, 64, 8, 64, 0, 1, table, 16, 64, BF, None), 1, b"world")
    rejects(lib.gdn_push_partial(ok, 64, 32, 64, 0, 2, table, 16, 64, BF, None), 1, b"does not fit")
    rejects(lib.gdn_pull_add_rmsnorm(ok, 64, ok, ok, 64, 4, 7, 1e-6, 0, 2, table, 16, 64, 0, None, BF, None), 1,
            b"dim")
    rejects(lib.gdn_pull_add_rmsnorm(ok, 64, ok, ok, 64, 4, 64, 1e-6, 0, 1, table, 16, 64, 0, None, BF, None), 1,
            b"world")
    rejects(lib.gdn_allreduce_add_rmsnorm(ok, 64, ok, 64, ok, ok, 64, 4, 64, 1e-6, 0, 1, table, 16, 0, None, BF,
                                          None), 1, b"world")
    rejects(lib.gdn_allreduce_add_rmsnorm(ok, 64, ok, 64, ok, ok, 64, 32, 64, 1e-6, 0, 2, table, 16, 0, None, BF,
                                          None), 1, b"rows")
    # decode-step glue
    rejects(lib.gdn_add_rmsnorm(ok, 64, ok, 64, ok, ok, 64, 4, 7, 1e-6, BF, None), 1, b"dim")
    rejects(lib.gdn_add_rmsnorm(ok, 64, odd, 64, ok, ok, 64, 4, 64, 1e-6, BF, None), 1, b"h rows")
    rejects(lib.gdn_add_rmsnorm(ok, 64, ok, 64, ok, ok, 64, 4, 64, 1e-6, F32, None), 3, b"bf16")
    rejects(lib.gdn_silu_mul(ok, 128, 7, ok, 64, 4, BF, None), 1, b"inter")
    rejects(lib.gdn_silu_mul(ok, 100, 64, ok, 64, 4, BF, None), 1, b"aligned")
    rejects(lib.gdn_silu_mul(ok, 128, 64, ok, 64, 4, F32, None), 3, b"bf16")
    assert lib.gdn_silu_mul(ok, 128, 64, ok, 64, 0, BF, None) == 0                      # no rows: no-op
    rejects(lib.gdn_attn_decode_prep(ok, 16384, ok, ok, 1e-6, ok, ok, 64, 64, ok, ok, ok, ok, 4, 24, 4, 300, BF,
                                     None), 1, b"hd")
    rejects(lib.gdn_attn_decode_prep(ok, 16384, ok, ok, 1e-6, ok, ok, 64, 24, ok, ok, ok, ok, 4, 24, 4, 256, BF,
                                     None), 1, b"rd")
    rejects(lib.gdn_attn_decode_prep(ok, 100, ok, ok, 1e-6, ok, ok, 64, 64, ok, ok, ok, ok, 4, 24, 4, 256, BF,
                                     None), 1, b"strides")
    rejects(lib.gdn_attn_decode_prep(ok, 16384, ok, ok, 1e-6, ok, ok, 64, 64, ok, ok, ok, ok, 4, 24, 4, 256, F32,
                                     None), 3, b"bf16")


def test_ops_refuse_cpu_tensors():
    import torch
    ops = pkg("ops")
    x = torch.zeros(4, 128, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.gated_rmsnorm(x, x, torch.ones(128, dtype=torch.bfloat16))
    q = torch.zeros(4, 1, 128, dtype=torch.bfloat16)
    ab = torch.zeros(4, 3, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.chunk_prefill_varlen_gates(q, q, torch.zeros(4, 3, 128, dtype=torch.bfloat16), ab, ab, torch.zeros(3),
                                       torch.zeros(3), torch.tensor([0, 4], dtype=torch.int32))


def test_header_compiles_as_c_and_links(tmp_path):
    """A C caller (no Python, no torch) includes include/gdn_b200.h, links libgdn_b200.so and gets the
    library's status codes and messages: the boundary is a plain C ABI.  Only argument validation runs
    (no CUDA call), so no GPU is needed."""
    import shutil
    import subprocess
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not available")
    L = pkg("_lib")
    if not os.path.exists(L.LIB_PATH):
        pytest.fail("libgdn_b200.so is not built (run __graft_entry__.build())")
    src = tmp_path / "caller.c"
    src.write_text(r'''
#include <stdio.h>
#include <string.h>
#include "gdn_b200.h"
int main(void) {
  if (gdn_version() < 100) return 1;
  /* one sequence of 10 tokens with every tensor pointer missing: rejected before any CUDA call */
  int rc = gdn_chunk_prefill(NULL, 0, NULL, 0, NULL, 0, NULL, NULL, 0, NULL, 1, 10, NULL, NULL, NULL, NULL,
                             NULL, 0, NULL, 0, 16, 48, 128, 128, 1, GDN_BF16, NULL, NULL);
  if (rc != GDN_ERR_ARG || strstr(gdn_last_error(), "null") == NULL) return 2;
  /* a head ratio the library does not build (40 value heads over 16 key heads); cu_seqlens is a device
     pointer the host never dereferences, so any non-null value reaches the shape check */
  const int32_t* cu = (const int32_t*)(uintptr_t)4096;
  rc = gdn_chunk_prefill_gates(NULL, 0, NULL, 0, NULL, 0, NULL, NULL, 0, NULL, NULL, cu, 1, 0, NULL, NULL, NULL,
                               NULL, NULL, 0, NULL, 0, 16, 40, 128, 128, 1, GDN_BF16, NULL, NULL);
  if (rc != GDN_ERR_SHAPE || strstr(gdn_last_error(), "multiple") == NULL) return 3;
  printf("ok %d\n", gdn_version());
  return 0;
}
''')
    exe = tmp_path / "caller"
    libdir = os.path.dirname(L.LIB_PATH)
    r = subprocess.run([gcc, "-std=c99", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), str(src), "-o",
                        str(exe), "-L", libdir, "-lgdn_b200", f"-Wl,-rpath,{libdir}"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.startswith("ok"), (r.returncode, r.stdout, r.stderr)
