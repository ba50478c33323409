"""Device-side tracing (hdcmamba_b200.trace): stamps of a captured Block forward are in
stream order and attribute every op of the layer."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_trace_block_forward_ops_and_order():
    from hdcmamba_b200 import HdcMamba9v3Block
    from hdcmamba_b200.trace import trace
    torch.manual_seed(0)
    dev = torch.device("cuda", 0)
    blk = HdcMamba9v3Block(d_model=256, d_state=64, num_heads=4, chunk_size=256).eval().to(dev).bfloat16()
    x = torch.randn(1, 1024, 256, device=dev).bfloat16()

    def fwd():
        with torch.no_grad():
            return blk(x)[0]
    ref = fwd()
    torch.cuda.synchronize()
    r = trace(fwd, dev, replays=3)
    for name in ("ln_conv", "linear", "slot_scan_gate", "row_layernorm", "addmm"):
        assert name in r["ops"], (name, sorted(r["ops"]))
        assert r["ops"][name]["us"] > 0
    assert r["total_us"] >= sum(v["us"] * v["per_replay"] for k, v in r["ops"].items()
                                if k in ("ln_conv", "linear", "slot_scan_gate", "row_layernorm", "addmm"))
    # the traced functions are restored and the forward is unchanged
    assert torch.equal(fwd(), ref)
