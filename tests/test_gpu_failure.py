"""Failure detection without a GPU fault: a bounded device wait that runs out.

Every spin in the library's kernels (peer flags, mbarriers) gives up after a time limit,
records an error code in the device error word (hdc_device_error) and returns, so a peer
that never arrives cannot hang the GPU.  The GPU test waits, with a 50 ms limit, on a flag
in local device memory that nothing raises, and checks that the kernel returns, the code
is reported once, and the context keeps working afterwards.  Nothing traps and no peer or
multicast memory is involved."""
import ctypes
import time

import pytest
import torch

from hdcmamba_b200 import _lib, ops


def _wait_for(flags, mask, gen, timeout_ns):
    return _lib.load().hdc_peer_wait_for(ctypes.c_void_p(flags.data_ptr()), mask, ctypes.c_void_p(gen.data_ptr()),
                                         timeout_ns, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def test_wait_limit_is_checked_before_any_launch():
    lib = _lib.load()
    fake = ctypes.c_void_p(16)
    for bad in (0, 2_000_000_001):
        assert lib.hdc_peer_wait_for(fake, 1, fake, bad, None) == -2
        assert b"timeout" in lib.hdc_error_string()
    assert lib.hdc_peer_wait_for(None, 1, fake, 1000, None) == -4


@pytest.mark.gpu
def test_flag_wait_times_out_and_reports_without_hanging():
    lib = _lib.load()
    torch.cuda.synchronize()
    assert lib.hdc_device_error(1) == 0
    flags = torch.zeros(32, dtype=torch.int32, device="cuda")   # nobody ever raises these
    gen = torch.ones(1, dtype=torch.int32, device="cuda")       # the generation waited for
    t0 = time.monotonic()
    assert _wait_for(flags, 0b101, gen, 50_000_000) == 0       # 50 ms per flag
    torch.cuda.synchronize()
    waited = time.monotonic() - t0
    assert 0.04 < waited < 1.5, waited                           # returned after its own limit, not 2 s
    assert lib.hdc_device_error(1) == 41                         # the flag-wait code
    assert lib.hdc_device_error(0) == 0                          # reset by the read above

    # a flag that has been raised (generation reached, wrap-safe >=) passes at once
    flags[0] = 1
    flags[2] = 7
    t0 = time.monotonic()
    assert _wait_for(flags, 0b101, gen, 50_000_000) == 0
    torch.cuda.synchronize()
    assert time.monotonic() - t0 < 0.04
    assert lib.hdc_device_error(1) == 0

    # the context is still usable: a library kernel and a torch op after the timeout
    x = torch.randn(64, 768, device="cuda").bfloat16()
    y = ops.row_layernorm(x)
    ref = torch.nn.functional.layer_norm(x.float(), (768,))
    torch.cuda.synchronize()
    assert float((y.float() - ref).abs().max()) < 5e-2
    assert lib.hdc_device_error(1) == 0
