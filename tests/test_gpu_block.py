"""GPU parity of the drop-in Block / Model / LM against the reference golden vectors
and the CPU oracle.  Tolerance: bf16 activations <= 2e-2 max-abs relative to the
fp32 reference scale."""
import pytest
import torch

import golden
import oracle as O
from hdcmamba_b200 import FusedNormConv1dFunction, HdcMamba9v3Block, HdcMamba9v3Model, _lib
from hdcmamba_b200.lm import CONFIGS, HdcMambaLM, build_lm, reinit_, synthetic_ids

pytestmark = pytest.mark.gpu
DEV = "cuda"
BF16_TOL = 2e-2


def rel(a, b):
    a, b = a.detach().float().cpu(), b.detach().float().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-6))


def _block_from(sd, B, L, ds, dm, H, C, semantics):
    blk = HdcMamba9v3Block(d_model=dm, d_state=ds, num_heads=H, chunk_size=C, semantics=semantics)
    blk.load_state_dict(sd)
    return blk.to(DEV).eval()


@pytest.mark.parametrize("tag", ["d64c64", "d64hd32c128pad"])
def test_block_shipped_fp32_matches_reference(tag):
    g = golden.load("block")
    B, L, ds, dm, H, C = [int(v) for v in g[f"{tag}_meta"]]
    sd = golden.state_dict(g, f"{tag}_")
    blk = _block_from(sd, B, L, ds, dm, H, C, "shipped")
    with torch.no_grad():
        y, aux = blk(g[f"{tag}_x"].to(DEV))
    assert aux is None
    assert rel(y, g[f"{tag}_y"]) < 5e-3
    assert rel(y, O.block_forward(sd, g[f"{tag}_x"], ds, H, C, mode="shipped")) < 5e-3


def test_block_fixed_fp32_matches_fixed_launch_reference_c256():
    g = golden.load("fixed_c256")
    B, L, ds, dm, H, C = [int(v) for v in g["meta"]]
    sd = golden.state_dict(g, "")
    blk = _block_from(sd, B, L, ds, dm, H, C, "fixed")
    with torch.no_grad():
        y, _ = blk(g["x"].to(DEV))
    assert rel(y, g["y"]) < 5e-3


@pytest.mark.parametrize("B,L,dm,H,ds,C", [(2, 1024, 256, 4, 64, 256), (1, 700, 256, 8, 64, 64),
                                           (2, 512, 384, 6, 128, 128)])
def test_block_fixed_bf16_vs_oracle(B, L, dm, H, ds, C):
    torch.manual_seed(5)
    blk = HdcMamba9v3Block(d_model=dm, d_state=ds, num_heads=H, chunk_size=C).eval()
    sd = {k: v.clone() for k, v in blk.state_dict().items()}
    blk = blk.to(DEV).bfloat16()
    x = torch.randn(B, L, dm).bfloat16()
    with torch.no_grad():
        y, _ = blk(x.to(DEV))
    torch.cuda.synchronize()
    assert _lib.load().hdc_device_error(1) == 0
    ref = O.block_forward({k: v.bfloat16() for k, v in sd.items()}, x, ds, H, C, mode="fixed")
    ref32 = O.block_forward({k: v.float() for k, v in sd.items()}, x.float(), ds, H, C, mode="fixed")
    assert rel(y, ref) < BF16_TOL
    assert rel(y, ref32) < BF16_TOL


def test_c1_lm_fp32_matches_reference_logits():
    """BASELINE config 1 through the CUDA path (shipped semantics, fp32) against the
    reference's own logits (TRITON_INTERPRET=1 golden rows)."""
    g = golden.load("c1_lm")
    cfg = CONFIGS["c1"]
    lm = build_lm("c1", semantics="shipped").to(DEV)
    ids = g["ids"]
    with torch.no_grad():
        logits = lm(ids.to(DEV)).cpu()
    rows = g["rows"].long()
    assert rel(logits[0, rows], g["logits_rows"]) < 5e-3
    sd = {k: v.float() for k, v in build_lm("c1").state_dict().items()}
    ref = O.lm_forward(sd, ids, cfg.n_layers, cfg.d_state, cfg.num_heads, cfg.chunk_size, mode="shipped")
    assert rel(logits, ref) < 5e-3


def test_small_c5_shape_lm_bf16_vs_oracle():
    """Config-5 layer shapes (d768, H12, ds64, C256) at 2 layers and L=2048."""
    torch.manual_seed(0)
    lm = reinit_(HdcMambaLM(50304, 768, 2, 64, 12, use_model=True)).eval()
    sd = {k: v.clone() for k, v in lm.state_dict().items()}
    lm = lm.to(DEV).bfloat16()
    ids = synthetic_ids("c5", seq_len=2048)
    with torch.no_grad():
        h = lm.hidden(ids.to(DEV)).cpu()
    sdb = {k: v.bfloat16() for k, v in sd.items()}
    emb = sdb["embedding.weight"][ids]
    ref = O.model_forward({k[len("backbone."):]: v for k, v in sdb.items() if k.startswith("backbone.")}, emb, 2, 64,
                          12, 256, mode="fixed")
    assert rel(h, ref) < BF16_TOL


def test_model_chunk_256_default_and_padding():
    torch.manual_seed(1)
    m = HdcMamba9v3Model(d_model=128, n_layers=2, d_state=64, num_slots=8, num_heads=2).eval()
    sd = {k: v.clone() for k, v in m.state_dict().items()}
    m = m.to(DEV)
    x = torch.randn(2, 300, 128)  # padded on the left to 512
    with torch.no_grad():
        y = m(x.to(DEV))
    ref = O.model_forward(sd, x, 2, 64, 2, 256, mode="fixed")
    assert y.shape == (2, 300, 128)
    assert rel(y, ref) < 5e-3


def test_train_mode_gradients_match_reference_behaviour():
    """Q8: the reference's kernels write outside autograd, so only out_proj.weight
    (and the residual path to x) receive gradients."""
    torch.manual_seed(2)
    blk = HdcMamba9v3Block(d_model=64, d_state=64, num_heads=2, chunk_size=64).to(DEV).train()
    x = torch.randn(1, 128, 64, device=DEV, requires_grad=True)
    y, _ = blk(x)
    y.sum().backward()
    grads = {n: p.grad for n, p in blk.named_parameters()}
    assert grads["out_proj.weight"] is not None
    assert all(g is None for n, g in grads.items() if n != "out_proj.weight")
    assert x.grad is not None


def test_fused_norm_conv_function_backward():
    torch.manual_seed(3)
    B, L, D = 2, 50, 64
    x = torch.randn(B, L, D, device=DEV, requires_grad=True)
    nw = (1 + 0.1 * torch.randn(D, device=DEV)).requires_grad_()
    nb = (0.1 * torch.randn(D, device=DEV)).requires_grad_()
    cw = (0.3 * torch.randn(D, 4, device=DEV)).requires_grad_()
    cb = (0.1 * torch.randn(D, device=DEV)).requires_grad_()
    out = FusedNormConv1dFunction.apply(x, nw, nb, cw, cb, 1e-5)
    go = torch.randn_like(out)
    out.backward(go)
    xs = x.detach().clone().requires_grad_()
    ps = [t.detach().clone().requires_grad_() for t in (nw, nb, cw, cb)]
    n = torch.nn.functional.layer_norm(xs, (D,), ps[0], ps[1], 1e-5)
    npad = torch.cat([ps[1].expand(B, 3, D), n], 1)
    ref = sum(npad[:, k:k + L] * ps[2][:, k] for k in range(4)) + ps[3]
    ref.backward(go)
    for a, b in zip([x, nw, nb, cw, cb], [xs, *ps]):
        torch.testing.assert_close(a.grad, b.grad, rtol=1e-4, atol=1e-4)


def test_repeated_forward_has_no_device_timeouts():
    """Many back-to-back bf16 forwards (the bench's pattern): every bounded device wait
    must complete, and repeated calls must agree exactly."""
    torch.manual_seed(4)
    blk = HdcMamba9v3Block(d_model=768, d_state=64, num_heads=12, chunk_size=256).to(DEV).bfloat16().eval()
    x = torch.randn(1, 8192, 768, device=DEV).bfloat16()
    with torch.no_grad():
        y0, _ = blk(x)
        for _ in range(20):
            y, _ = blk(x)
    torch.cuda.synchronize()
    assert _lib.load().hdc_device_error(1) == 0
    assert torch.equal(y, y0)


def test_graphed_forward_matches_eager():
    """GraphedForward (CUDA-graph capture of the LM forward) equals the eager forward,
    including after the static input changes."""
    from hdcmamba_b200.graph import GraphedForward
    torch.manual_seed(6)
    lm = reinit_(HdcMambaLM(1000, 256, 2, 64, 4, use_model=True)).eval().to(DEV).bfloat16()
    ids = torch.randint(0, 1000, (2, 1024), device=DEV)
    g = GraphedForward(lm, ids)
    assert g.launches_per_replay > 0
    with torch.no_grad():
        eager = lm(ids)
    assert torch.equal(g.replay(), eager)
    ids2 = torch.randint(0, 1000, (2, 1024)).pin_memory()
    out = g(ids2).clone()
    with torch.no_grad():
        eager2 = lm(ids2.to(DEV))
    torch.cuda.synchronize()
    assert torch.equal(out, eager2)
    assert _lib.load().hdc_device_error(1) == 0
