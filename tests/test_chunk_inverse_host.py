"""The tensor-core chunk kernel's 64 x 64 triangular inverse, built for the host and run on the CPU.

tri_inverse64 (csrc/chunk_tc.cu) forms T = (I - X)^-1 of a chunk's strictly lower X (the WY/UT
inverse of src/gdn_chunk_fast.py:21-62) with 256 threads: diagonal 16 x 16 blocks on two warps, then
two merge levels whose products skip the zero steps of the triangular factors warp by warp.  Its thread
and index arithmetic is checked here without a GPU: the function is cut out of the kernel source,
compiled by g++ with stand-ins for shared-memory loads and the named barriers
(tests/host_inverse_harness.cpp), run as 256 host threads, and compared with numpy's solve of I - X
in float64 on chunks shaped like the kernel's inputs (unit keys, sigmoid betas, cumulative decays;
correlated keys; weak decay; padded rows).
"""
import os
import re
import shutil
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "910b_e2e_accleration_by_codex_b200", "csrc", "chunk_tc.cu")
HARNESS = os.path.join(ROOT, "tests", "host_inverse_harness.cpp")


@pytest.fixture(scope="module")
def host_inverse(tmp_path_factory):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not found")
    d = tmp_path_factory.mktemp("inv")
    src = open(SRC).read()
    m = re.search(r"^__device__ __forceinline__ void tri_inverse64\(.*?^\}\n", src, re.S | re.M)
    assert m, "tri_inverse64 not found in chunk_tc.cu"
    inc = d / "tri_inverse64.inc"
    inc.write_text(m.group(0))
    exe = d / "host_inverse"
    r = subprocess.run([gxx, "-O2", "-std=c++20", "-pthread", f'-DINV_INC="{inc}"', HARNESS, "-o", str(exe)],
                       capture_output=True, text=True)
    if r.returncode != 0 and "barrier" in r.stderr and "No such file" in r.stderr:
        pytest.skip("this g++ has no <barrier>")
    assert r.returncode == 0, r.stderr

    def run(X):
        xin, tout = d / "x.bin", d / "t.bin"
        np.ascontiguousarray(X, np.float32).tofile(xin)
        rr = subprocess.run([str(exe), str(xin), str(tout)], capture_output=True, text=True, timeout=60)
        assert rr.returncode == 0, rr.stderr
        return np.fromfile(tout, np.float32).reshape(64, 64)
    return run


def chunk_x(rng, correlated=False, weak=False, live=64):
    """X = -(beta k k^T * e^(g_i - g_j)) strictly lower, as the kernel's P1 epilogue forms it."""
    k = rng.standard_normal((64, 128))
    if correlated:
        k = rng.standard_normal(128)[None, :] + 0.15 * k
    k /= np.linalg.norm(k, axis=1, keepdims=True)
    beta = 1 / (1 + np.exp(-rng.standard_normal(64)))
    g = np.cumsum(-(rng.uniform(0.001, 0.02, 64) if weak else rng.uniform(0.01, 1.0, 64)))
    beta[live:] = 0.0  # rows past the sequence end
    k[live:] = 0.0
    X = -(beta[:, None] * (k @ k.T) * np.exp(g[:, None] - g[None, :]))
    return np.tril(X, -1).astype(np.float32)


@pytest.mark.parametrize("case", ["random", "correlated", "weak", "correlated-weak", "padded", "zero"])
def test_host_inverse_matches_solve(host_inverse, case):
    rng = np.random.default_rng({"random": 1, "correlated": 2, "weak": 3, "correlated-weak": 4, "padded": 5,
                                 "zero": 6}[case])
    for _ in range(3):
        if case == "zero":
            X = np.zeros((64, 64), np.float32)
        else:
            X = chunk_x(rng, correlated="correlated" in case, weak="weak" in case,
                        live=int(rng.integers(1, 64)) if case == "padded" else 64)
        T = host_inverse(X)
        ref = np.linalg.solve(np.eye(64) - X.astype(np.float64), np.eye(64))
        assert np.array_equal(np.triu(T, 1), np.zeros((64, 64), np.float32)), "nonzero above the diagonal"
        assert np.array_equal(np.diag(T), np.ones(64, np.float32)), "diagonal not exactly 1"
        err = np.abs(T - ref).max() / max(1.0, np.abs(ref).max())
        assert err < 2e-6, (case, err)
