"""The allocation-free GEMV entry point (spkv2_cuda_gemv_noalloc).

Callers inside a CUDA stream capture, latency-bound loops and fixed-memory
deployments cannot allocate device memory while they run, so this entry
point keeps its split-K scratch in a static device array instead.  The test
calls it through the C-ABI with device buffers prepared up front and checks
two consecutive calls against the Gemm node run by the regular runtime path
(spkv2_run), with the fp32 tolerance of the other GPU tests.  It lives in a
file of its own, collected last, and needs nothing from the tests before it.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import compile_pair, seeded_input

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-3, 1e-4


def _fn():
    from spinnv2_b200.runtime import load_library

    fn = load_library().spkv2_cuda_gemv_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 3 + [ctypes.c_float, ctypes.c_void_p]
    return fn


def test_gemv_noalloc_matches_gemm_node_on_two_calls(gpu):
    import torch

    from spinnv2_b200.runtime import Runtime
    from spinnv2_b200.spk import read_spk

    M, K, N = 4, 2048, 1000
    spk = compile_pair("gemm_2048_1000", M, targets=("cuda_b200",))["cuda_b200"]
    pkg = read_spk(spk)
    gemm = pkg.nodes[0]
    w = torch.from_numpy(np.array(pkg.weight(gemm.inputs[1]))).cuda()
    b = torch.from_numpy(np.array(pkg.weight(gemm.inputs[2]))).cuda()
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    inputs = [seeded_input((M, K), seed=s) for s in (3, 4)]
    a_dev = [torch.from_numpy(x).cuda() for x in inputs]
    torch.cuda.synchronize()
    fn = _fn()
    with Runtime(spk, device=0) as rt:
        for x, a in zip(inputs, a_dev):
            expected = rt.run(x)[0]
            rc = fn(a.data_ptr(), w.data_ptr(), b.data_ptr(), y.data_ptr(), M, K, N, 1.0, None)
            assert rc == 0
            torch.cuda.synchronize()
            np.testing.assert_allclose(y.cpu().numpy(), expected, atol=ATOL, rtol=RTOL)


def test_gemv_noalloc_shrinks_split_to_fit_its_scratch(gpu):
    """M = 8, K = 2048, N = 4000: the default split of K into 16 parts would
    need 16 * 8 * 4000 partial sums, over the 262144-float scratch, so the
    entry point drops to 8 parts (8 * 8 * 4000 = 256000 fit).  Two calls in a
    row against A @ B + bias computed in float64 by numpy."""
    import torch

    M, K, N = 8, 2048, 4000
    rng = np.random.default_rng(21)
    w = (rng.standard_normal((K, N), dtype=np.float32) * np.float32(np.sqrt(2.0 / K))).astype(np.float32)
    b = (rng.standard_normal(N, dtype=np.float32) * np.float32(0.01)).astype(np.float32)
    w_d, b_d = torch.from_numpy(w).cuda(), torch.from_numpy(b).cuda()
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    fn = _fn()
    for seed in (5, 6):
        x = seeded_input((M, K), seed=seed)
        a = torch.from_numpy(x).cuda()
        torch.cuda.synchronize()
        assert fn(a.data_ptr(), w_d.data_ptr(), b_d.data_ptr(), y.data_ptr(), M, K, N, 1.0, None) == 0
        torch.cuda.synchronize()
        expected = (x.astype(np.float64) @ w.astype(np.float64) + b).astype(np.float32)
        np.testing.assert_allclose(y.cpu().numpy(), expected, atol=ATOL, rtol=RTOL)


def test_gemv_noalloc_rejects_sizes_beyond_its_scratch(gpu):
    import torch

    fn = _fn()
    a = torch.zeros((9, 128), dtype=torch.float32, device="cuda")
    w = torch.zeros((128, 64), dtype=torch.float32, device="cuda")
    y = torch.zeros((9, 64), dtype=torch.float32, device="cuda")
    assert fn(a.data_ptr(), w.data_ptr(), None, y.data_ptr(), 9, 128, 64, 1.0, None) == -14  # M > 8
    big_n = 262144 // 8 + 1
    w2 = torch.zeros((128, big_n), dtype=torch.float32, device="cuda")
    y2 = torch.zeros((8, big_n), dtype=torch.float32, device="cuda")
    assert fn(a.data_ptr(), w2.data_ptr(), None, y2.data_ptr(), 8, 128, big_n, 1.0, None) == -14
