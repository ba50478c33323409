"""hdc_peer_put on one GPU: the "peers" are local device buffers, so the test needs no
second GPU and no IPC mapping.  Each target's copy is split over several CTAs; the CTA that
finishes a target's last slice raises the target's flag, and the per-target slice counters
come back to zero for the next call."""
import ctypes

import pytest
import torch

from hdcmamba_b200 import _lib

pytestmark = pytest.mark.gpu


def _vp(t):
    return ctypes.c_void_p(t.data_ptr())


@pytest.mark.parametrize("nbytes", [4608, 196_608 + 256, 1 << 20])
def test_put_to_local_targets_raises_flags_after_the_data(nbytes):
    dev = torch.device("cuda", 0)
    world, flag_off = 4, 16 << 20
    boxes = [torch.zeros((16 << 20) + 256, dtype=torch.uint8, device=dev) for _ in range(world)]
    bases = torch.tensor([b.data_ptr() for b in boxes], dtype=torch.int64, device=dev)
    counters = torch.zeros(world, dtype=torch.int32, device=dev)
    gen = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    g = torch.Generator(device=dev).manual_seed(0)
    for step in (1, 2):  # the second call reuses the counters
        src = torch.randint(0, 256, (nbytes,), dtype=torch.uint8, device=dev, generator=g)
        gen.fill_(step)
        mask = 0b1011  # targets 0, 1 and 3
        _lib.call("hdc_peer_put", _vp(src), nbytes, _vp(bases), 64, flag_off, mask, world, _vp(gen), _vp(counters),
                  stream)
        torch.cuda.synchronize()
        for t in range(world):
            flag = int(boxes[t][flag_off:flag_off + 4].view(torch.int32)[0])
            if (mask >> t) & 1:
                assert flag == step
                assert torch.equal(boxes[t][64:64 + nbytes], src)
            else:
                assert flag == 0
        assert int(counters.abs().sum()) == 0
    assert _lib.load().hdc_device_error(1) == 0
