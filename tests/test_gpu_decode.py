"""Recurrent decode (hdcmamba_b200.decode): a prompt of whole chunks prefilled, then tokens
decoded one by one, must give the logits of one prefill over the whole sequence at those
positions (same chunk alignment: the full length is a whole number of chunks too), across
a chunk boundary."""
import pytest
import torch

from hdcmamba_b200 import _lib
from hdcmamba_b200.decode import decode_step, prefill
from hdcmamba_b200.lm import HdcMambaLM, reinit_

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel(a, b):
    a, b = a.detach().float(), b.detach().float()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-6))


def _lm(dtype, chunk, use_model, d_model=256, heads=4):
    torch.manual_seed(5)
    lm = reinit_(HdcMambaLM(512, d_model, 2, 64, heads, chunk_size=chunk, use_model=use_model)).eval()
    return lm.to(DEV).to(dtype)


@pytest.mark.parametrize("dtype,chunk,use_model,L0,T,tol", [
    (torch.bfloat16, 64, False, 192, 128, 2e-2),
    (torch.float32, 64, False, 128, 128, 2e-3),
    (torch.bfloat16, 256, True, 256, 256, 2e-2),
])
def test_decode_matches_prefill(dtype, chunk, use_model, L0, T, tol):
    lm = _lm(dtype, chunk, use_model, d_model=256 if not use_model else 128, heads=4 if not use_model else 2)
    g = torch.Generator().manual_seed(9)
    ids = torch.randint(0, 512, (2, L0 + T), generator=g).to(DEV)
    with torch.no_grad():
        full = lm(ids)
    logits0, st = prefill(lm, ids[:, :L0])
    assert rel(logits0, full[:, :L0]) < 1e-6 if dtype == torch.float32 else rel(logits0, full[:, :L0]) < 1e-2
    worst = 0.0
    for t in range(T):
        lt = decode_step(lm, st, ids[:, L0 + t])
        worst = max(worst, rel(lt, full[:, L0 + t]))
    torch.cuda.synchronize()
    assert _lib.load().hdc_device_error(1) == 0
    assert st.pos == (L0 + T) % chunk
    assert worst < tol, worst


def test_decode_prompt_with_padding():
    """A prompt that is not a whole number of chunks is left-padded (as the Block does);
    decoding continues after it and stays finite and deterministic."""
    lm = _lm(torch.bfloat16, 64, False)
    ids = torch.randint(0, 512, (1, 100), generator=torch.Generator().manual_seed(2)).to(DEV)
    logits0, st = prefill(lm, ids)
    with torch.no_grad():
        ref = lm(ids)
    assert rel(logits0, ref) < 1e-2
    assert st.pos == 0
    outs = [decode_step(lm, st, ids[:, -1]) for _ in range(5)]
    assert all(torch.isfinite(o.float()).all() for o in outs)


def test_graphed_decode_equals_eager():
    """decode_step replayed as one CUDA graph (position on the device) gives the eager
    step's logits exactly, token after token across a chunk boundary."""
    from hdcmamba_b200.decode import GraphedDecode
    lm = _lm(torch.bfloat16, 64, False)
    g = torch.Generator().manual_seed(4)
    ids = torch.randint(0, 512, (3, 128 + 80), generator=g).to(DEV)
    _, st_e = prefill(lm, ids[:, :128])
    _, st_g = prefill(lm, ids[:, :128])
    gd = GraphedDecode(lm, st_g, ids[:, 128])
    for t in range(80):
        a = decode_step(lm, st_e, ids[:, 128 + t])
        b = gd(ids[:, 128 + t])
        assert torch.equal(a, b), t
    assert st_e.pos == st_g.pos == 80 % 64
