"""The allocation-free SSM scan entry point (hdc_ssm_scan_fwd_noalloc).

It exists for callers that cannot allocate device memory themselves (a host that only
passes the tensors it owns across a foreign-function boundary, or code that must not
call cudaMalloc at that point); its chunk statistics live in a fixed device array that
the library reserves at load time.  The GPU test checks it against the regular entry
points (hdc_ssm_chunk_stats + hdc_ssm_scan_out with a caller workspace) on two calls in
a row, so the shared array's leftover contents from the first call cannot leak into the
second, and against the CPU oracle's restatement of the reference's three SSM kernels
(oracle.ssm_chunk_fwd, hdcmamba/model.py:175-233).  This file is collected last on purpose."""
import ctypes

import pytest
import torch

import oracle as O
from hdcmamba_b200 import _lib, ops

BF16_TOL = 2e-2


def _noalloc(projs, A_log, ds, C, y):
    B, L, _ = projs.shape
    _lib.call("hdc_ssm_scan_fwd_noalloc", _lib.HDC_BF16 if projs.dtype == torch.bfloat16 else _lib.HDC_F32,
              ctypes.c_void_p(projs.data_ptr()), projs.stride(0), projs.stride(1),
              ctypes.c_void_p(A_log.data_ptr()), ctypes.c_void_p(y.data_ptr()), y.stride(0), y.stride(1),
              B, L, ds, C, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return y


def _inputs(seed, B, L, ds, extra, dtype, dev):
    g = torch.Generator().manual_seed(seed)
    projs = torch.randn(B, L, 3 * ds + extra, generator=g)
    projs[..., :ds] = projs[..., :ds] * 2 - 3
    return projs.to(dtype).to(dev)


def test_noalloc_rejects_oversized_requests_before_touching_the_gpu():
    lib = _lib.load()
    cap = lib.hdc_ssm_noalloc_capacity()
    assert cap == 1 << 20
    # B * (L / C) * 2 * ds = 1 * 8192 * 2 * 128 > capacity: rejected by the host-side check
    rc = lib.hdc_ssm_scan_fwd_noalloc(_lib.HDC_BF16, ctypes.c_void_p(16), 0, 384, ctypes.c_void_p(16),
                                      ctypes.c_void_p(16), 0, 128, 1, 8192 * 64, 128, 64, None)
    assert rc == -5
    assert b"capacity" in lib.hdc_error_string()


@pytest.mark.gpu
def test_noalloc_matches_regular_entry_points_on_two_calls():
    dev = "cuda"
    A_log = torch.log(torch.linspace(0.99, 0.9999, 64)).bfloat16().to(dev)
    cases = [(2, 2048, 64, 256, 40, 11), (1, 4096, 64, 64, 0, 12)]
    for B, L, ds, C, extra, seed in cases:  # two calls in a row with different shapes / data
        projs = _inputs(seed, B, L, ds, extra, torch.bfloat16, dev)
        ref = ops.ssm_scan(projs, A_log, ds, C)
        y = torch.full((B, L, ds), float("nan"), device=dev, dtype=torch.bfloat16)
        _noalloc(projs, A_log, ds, C, y)
        torch.cuda.synchronize()
        err = float((y.float() - ref.float()).abs().max() / ref.float().abs().max())
        assert err < BF16_TOL, err
        assert torch.equal(y, ref)  # same kernels, same statistics: bit-identical
        oracle = O.ssm_chunk_fwd(projs.cpu(), A_log.cpu(), ds, C)
        err_o = float((y.float().cpu() - oracle).abs().max() / oracle.abs().max())
        assert err_o < BF16_TOL, err_o
