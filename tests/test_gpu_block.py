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


@pytest.mark.parametrize("dtype,B,L,D", [(torch.float32, 2, 50, 64), (torch.bfloat16, 2, 300, 768),
                                         (torch.float32, 1, 37, 2048), (torch.bfloat16, 3, 129, 96)])
def test_fused_norm_conv_function_backward(dtype, B, L, D):
    """FusedNormConv1dFunction.backward (hdc_ln_conv_bwd) against the oracle restatement of
    the reference's backward on the forward's bf16 statistics; dx also against autograd.
    (Rows of a multiple of 16 bytes: the shared-memory-staged kernel.)"""
    import oracle as O
    from hdcmamba_b200 import ops
    g = torch.Generator().manual_seed(3 + D)
    x = torch.randn(B, L, D, generator=g).to(dtype).to(DEV).requires_grad_()
    nw = (1 + 0.1 * torch.randn(D, generator=g)).to(dtype).to(DEV).requires_grad_()
    nb = (0.1 * torch.randn(D, generator=g)).to(dtype).to(DEV).requires_grad_()
    cw = (0.3 * torch.randn(D, 4, generator=g)).to(dtype).to(DEV).requires_grad_()
    cb = (0.1 * torch.randn(D, generator=g)).to(dtype).to(DEV).requires_grad_()
    go = torch.randn(B, L, D, generator=g).to(dtype).to(DEV)
    out = FusedNormConv1dFunction.apply(x, nw, nb, cw, cb, 1e-5)
    out.backward(go)
    torch.cuda.synchronize()
    assert _lib.load().hdc_device_error(1) == 0
    _, mean, rstd = ops.ln_conv(x.detach(), nw.detach(), nb.detach(), cw.detach(), cb.detach(), 1e-5, stats=True)
    ref = O.ln_conv_bwd(go.cpu(), x.detach().cpu(), mean.cpu(), rstd.cpu(), nw.detach().cpu(), cw.detach().cpu())
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    for got, r, name in zip([x.grad, nw.grad, nb.grad, cw.grad, cb.grad], ref, ["dx", "dnw", "dnb", "dcw", "dcb"]):
        assert got.dtype == dtype and got.shape == r.shape, name
        assert rel(got, r) < tol, (name, rel(got, r))
    # dx is the LayerNorm backward proper (on bf16-rounded statistics)
    xs = x.detach().float().requires_grad_()
    y = torch.nn.functional.layer_norm(xs, (D,), nw.detach().float(), None, 1e-5)
    dn = sum(torch.cat([go.float(), go.new_zeros(B, 3, D).float()], 1)[:, 3 - k:3 - k + L] * cw.detach().float()[:, k]
             for k in range(4))
    y.backward(dn)
    assert rel(x.grad, xs.grad) < 2e-2


def test_ln_conv_bwd_direct_load_path():
    """bf16 rows that are not a multiple of 16 bytes (D = 100) take the direct-load backward
    kernel (the forward needs D % 8 == 0, so the statistics come from the oracle)."""
    import oracle as O
    from hdcmamba_b200 import ops
    g = torch.Generator().manual_seed(17)
    B, L, D = 2, 45, 100
    x = torch.randn(B, L, D, generator=g).bfloat16()
    nw, nb = (1 + 0.1 * torch.randn(D, generator=g)).bfloat16(), (0.1 * torch.randn(D, generator=g)).bfloat16()
    cw, cb = (0.3 * torch.randn(D, 4, generator=g)).bfloat16(), torch.zeros(D).bfloat16()
    go = torch.randn(B, L, D, generator=g).bfloat16()
    _, mean, rstd = O.ln_conv_fwd(x, nw, nb, cw, cb, 1e-5)
    got = ops.ln_conv_bwd(go.to(DEV), x.to(DEV), mean.to(DEV), rstd.to(DEV), nw.to(DEV), cw.to(DEV))
    ref = O.ln_conv_bwd(go, x, mean, rstd, nw, cw)
    for a, r in zip(got, ref):
        assert rel(a, r) < 2e-2, rel(a, r)


@pytest.mark.parametrize("tag", ["f32", "bf16"])
def test_ln_conv_bwd_reference_golden(tag):
    """hdc_ln_conv_bwd on the inputs and bf16 statistics recorded from the reference's own
    backward (interpreter; its bf16 stores truncate, the GPU rounds to nearest)."""
    from hdcmamba_b200 import ops
    import golden
    gd = golden.load("lnconv_bwd")
    d = {k: gd[f"{tag}_{k}"].to(DEV) for k in ("go", "x", "mean", "rstd", "nw", "cw")}
    out = ops.ln_conv_bwd(d["go"], d["x"], d["mean"], d["rstd"], d["nw"], d["cw"])
    for got, key in zip(out, ["dx", "dnw", "dnb", "dcw", "dcb"]):
        r = gd[f"{tag}_{key}"]
        assert rel(got, r) < (1e-4 if tag == "f32" else 2e-2), (key, rel(got, r))


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
