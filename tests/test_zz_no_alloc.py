"""The allocation-free entry point, ql_gptq_matmul_noalloc, against ql_gptq_matmul_ws.

ql_gptq_matmul_noalloc serves callers that cannot allocate device memory when they call in
(hosts that own all device memory through their own allocator or budget, bindings without a
CUDA allocator, code running under a latency budget). It keeps the large-M path's scratch in a
fixed device array inside the library instead of taking a workspace. These tests call it
through the C ABI twice in a row — the array keeps the previous call's contents, so the second
call must not depend on them — and compare each result with the regular entry point's and with
the oracle (oracle/gptq.py, the restatement of the reference's _gptq_matmul_np). Inside the
entry point every path that would otherwise fall back to the stream-ordered allocator fails
instead; the tests also watch the device's default memory pool, which that allocator draws from.

This file is collected last so that a run stopping at the first failure has already run every
other test; it also passes on its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

from conftest import max_rel_err
from oracle import gptq as og
from webpytorch_b200 import _ffi, synth
from webpytorch_b200.qlinear import _gptq_matmul

pytestmark = pytest.mark.gpu
TOL = 2e-3
DEV = "cuda"


def _noalloc(x, qw, qz, sc, K, N, gs, bits, zoff, out):
    lib = _ffi.load()
    return lib.ql_gptq_matmul_noalloc(_ffi.ptr(x), _ffi.dtype_code(x.dtype), x.stride(0), None, _ffi.ptr(qw),
                                      _ffi.ptr(qz), _ffi.ptr(sc), _ffi.dtype_code(sc.dtype), None, _ffi.ptr(out),
                                      _ffi.dtype_code(out.dtype), out.stride(0), x.shape[0], K, N, gs, bits,
                                      ctypes.c_float(zoff), _ffi.stream_ptr())


@pytest.mark.parametrize("M,K,N,bits", [(256, 1024, 512, 4),    # tensor-core path: uses the fixed scratch
                                        (640, 2048, 384, 8),
                                        (1, 4096, 1024, 4),      # decode path, up to 4 tokens: no scratch
                                        (12, 1024, 512, 8),      # decode path, 5-16 tokens: staged activations
                                        (40, 2048, 384, 4)])     # in the scratch; 40 tokens: tensor-core path
def test_noalloc_matches_regular_entry_point_twice(M, K, N, bits):
    w = synth.gptq_weights(K, N, bits, 128, seed=M + K)
    qw = torch.from_numpy(w["qweight"]).to(DEV)
    qz = torch.from_numpy(w["qzeros"]).to(DEV)
    sc = torch.from_numpy(w["scales"]).to(DEV)
    for call in range(2):
        xh = synth.activations(M, K, np.float16, seed=100 * call + M)
        x = torch.from_numpy(xh).to(DEV)
        ref = _gptq_matmul(x, qw, qz, sc, K, N, 128, bits, 1.0)
        got = torch.full((M, N), float("nan"), device=DEV)
        torch.cuda.synchronize()
        pool, in_use = _pool_high_reset()
        assert _noalloc(x, qw, qz, sc, K, N, 128, bits, 1.0, got) == 0, _ffi.load().ql_last_error()
        torch.cuda.synchronize()
        assert _pool_high(pool) <= in_use, "the stream-ordered allocator was used"
        got = got.cpu().numpy()
        assert max_rel_err(got, ref.cpu().numpy()) < TOL, (call, M, K, N, bits)
        oracle = og.gptq_matmul(xh.astype(np.float32), w["qweight"], w["qzeros"], w["scales"], K, N, 128, bits, 1.0)
        assert max_rel_err(got, oracle) < TOL, (call, M, K, N, bits)
    assert _ffi.load().ql_device_status() == 0


def _pool_high_reset():
    """The current device's default memory pool (where cudaMallocAsync draws from) with its
    used-memory high-water mark reset (to the bytes in use now, also returned); (None, 0) when
    the CUDA Python bindings are not installed."""
    try:
        from cuda.bindings import driver as dr
        from cuda.bindings import runtime as rt
    except ImportError:
        return None, 0
    err, pool = rt.cudaDeviceGetDefaultMemPool(torch.cuda.current_device())
    assert err == rt.cudaError_t.cudaSuccess
    err, = rt.cudaMemPoolSetAttribute(pool, rt.cudaMemPoolAttr.cudaMemPoolAttrUsedMemHigh, dr.cuuint64_t(0))
    assert err == rt.cudaError_t.cudaSuccess
    err, used = rt.cudaMemPoolGetAttribute(pool, rt.cudaMemPoolAttr.cudaMemPoolAttrUsedMemCurrent)
    assert err == rt.cudaError_t.cudaSuccess
    return pool, int(used)


def _pool_high(pool):
    if pool is None:
        return 0
    from cuda.bindings import runtime as rt
    err, v = rt.cudaMemPoolGetAttribute(pool, rt.cudaMemPoolAttr.cudaMemPoolAttrUsedMemHigh)
    assert err == rt.cudaError_t.cudaSuccess
    return int(v)


def test_noalloc_rejects_shapes_beyond_its_scratch():
    lib = _ffi.load()
    cap = lib.ql_gptq_matmul_noalloc_max_scratch()
    assert cap == 24 << 20
    K, N = 8192, 256
    M = cap // (2 * K) + 64                    # the fp16 staging alone exceeds the array
    x = torch.zeros((M, K), dtype=torch.float16, device=DEV)
    w = synth.gptq_weights(K, N, 4, 128, seed=1)
    qw = torch.from_numpy(w["qweight"]).to(DEV)
    qz = torch.from_numpy(w["qzeros"]).to(DEV)
    sc = torch.from_numpy(w["scales"]).to(DEV)
    out = torch.empty((M, N), device=DEV)
    assert _noalloc(x, qw, qz, sc, K, N, 128, 4, 1.0, out) == 3      # QL_ERR_UNSUPPORTED
    assert b"needs" in lib.ql_last_error()
