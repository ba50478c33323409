"""Pin the CPU oracle (oracle/restate.py) against golden vectors produced by the
unmodified reference under TRITON_INTERPRET=1 (tests/golden/make_golden.py).

The interpreter converts fp32 -> bf16 inside kernels by truncation, so the pins
run the oracle with ``kernel_rounding("rtz")``; with that, every bf16 store
matches except where an fp32 sum lands on the other side of a bf16 boundary
because of summation order (a fraction of a percent of elements, one ulp)."""
import functools

import pytest
import torch

import golden
import oracle as O


def rtz(fn):
    @functools.wraps(fn)
    def wrapped(*a, **k):
        with O.kernel_rounding("rtz"):
            return fn(*a, **k)
    return wrapped


def ulp_flip_fraction(a, b):
    return float((a.float() != b.float()).float().mean())


def relmax(a, b):
    a, b = a.float(), b.float()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-6))


@pytest.mark.parametrize("tag", ["f32", "bf16"])
@rtz
def test_lnconv_matches_reference(tag):
    g = golden.load("lnconv")
    out, mean, rstd = O.ln_conv_fwd(g[f"{tag}_x"], g[f"{tag}_nw"], g[f"{tag}_nb"], g[f"{tag}_cw"],
                                    g[f"{tag}_cb"], 1e-5)
    ref = g[f"{tag}_out"]
    assert out.dtype == ref.dtype
    if tag == "f32":
        torch.testing.assert_close(out, ref, rtol=1e-5, atol=1e-5)
    else:
        assert relmax(out, ref) < 1e-2
        assert ulp_flip_fraction(out, ref) < 0.01
    assert ulp_flip_fraction(mean, g[f"{tag}_mean"]) < 0.02
    assert ulp_flip_fraction(rstd, g[f"{tag}_rstd"]) < 0.02
    torch.testing.assert_close(mean.float(), g[f"{tag}_mean"].float(), rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(rstd.float(), g[f"{tag}_rstd"].float(), rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("tag", ["f32", "bf16"])
@rtz
def test_lnconv_bwd_matches_reference(tag):
    """The restated backward against the reference's own FusedNormConv1dFunction.backward
    (model.py:148-166) run under the interpreter, on the forward's bf16 mean / rstd."""
    g = golden.load("lnconv_bwd")
    dx, dnw, dnb, dcw, dcb = O.ln_conv_bwd(g[f"{tag}_go"], g[f"{tag}_x"], g[f"{tag}_mean"], g[f"{tag}_rstd"],
                                           g[f"{tag}_nw"], g[f"{tag}_cw"])
    for got, key in ((dx, "dx"), (dnw, "dnw"), (dnb, "dnb"), (dcw, "dcw"), (dcb, "dcb")):
        ref = g[f"{tag}_{key}"]
        assert got.dtype == ref.dtype and got.shape == ref.shape, key
        # the reference sums rows per 16-row program and across programs with fp32 atomics
        assert relmax(got, ref) < (1e-5 if tag == "f32" else 1e-2), (key, relmax(got, ref))


def test_lnconv_bwd_quirks_are_material():
    """The reference's conv-weight / norm-bias gradients leave out the norm bias and the
    three zero rows before the sequence: they differ from autograd of the forward."""
    g = golden.load("lnconv_bwd")
    x, nw, nb, cw, cb, go = (g[f"f32_{k}"].clone().requires_grad_(True) for k in ("x", "nw", "nb", "cw", "cb", "go"))
    B, L, D = x.shape
    n = torch.nn.functional.layer_norm(x, (D,), nw, nb, 1e-5)
    npad = torch.cat([nb.expand(B, 3, D), n], 1)
    y = sum(npad[:, k:k + L] * cw[:, k] for k in range(4)) + cb
    y.backward(go)
    assert relmax(g["f32_dcw"], cw.grad) > 1e-2  # nb missing from xhat * nw
    assert relmax(g["f32_dnb"], nb.grad) > 1e-3   # padded rows missing
    torch.testing.assert_close(g["f32_dcb"], cb.grad, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("tag", ["f32c64", "f32c32", "bf16c64"])
@rtz
def test_ssm_matches_reference(tag):
    g = golden.load("ssm")
    B, L, ds, C = [int(v) for v in g[f"{tag}_meta"]]
    y = O.ssm_chunk_fwd(g[f"{tag}_projs"], g[f"{tag}_A_log"], ds, C)
    ref = g[f"{tag}_y"].float()
    # every value is a bf16 store; fp32 rounding-order noise may flip one bf16 ulp
    assert relmax(y, ref) < 1e-2, relmax(y, ref)
    assert ulp_flip_fraction(y, ref) < 0.01


@pytest.mark.parametrize("tag", ["f32hd64", "f32hd32c128"])
@rtz
def test_slot_matches_reference(tag):
    g = golden.load("slot")
    B, L, ds, dm, H, C = [int(v) for v in g[f"{tag}_meta"]]
    projs = g[f"{tag}_projs"]
    y = O.slot_fwd(projs, g[f"{tag}_gamma"], dm, H, C, 3 * ds, block_c=128)
    ref = g[f"{tag}_y"]
    tol = 1e-5 if projs.dtype == torch.float32 else 1e-2
    assert relmax(y, ref) < tol, relmax(y, ref)
    if projs.dtype == torch.bfloat16:
        assert ulp_flip_fraction(y, ref) < 0.02


def test_slot_feature_padding_quirk_is_material():
    """Q9: with head_dim 32 the reference pads q/k features with ones; dropping
    that padding must change the answer (so the fixture really pins it)."""
    g = golden.load("slot")
    B, L, ds, dm, H, C = [int(v) for v in g["f32hd32c128_meta"]]
    projs = g["f32hd32c128_projs"]
    hd = dm // H
    # restate without padding: treat head_dim 32 as a full 64-wide block by zero-extending v
    # and using phi features only (no ones) -- emulate by moving the data into a hd=64 layout
    # whose extra lanes hold raw -inf (phi(-inf) = 0).
    q = projs[..., :dm].reshape(B, L, H, hd)
    k = projs[..., dm:2 * dm].reshape(B, L, H, hd)
    v = projs[..., 2 * dm:3 * dm].reshape(B, L, H, hd)
    pad = torch.full((B, L, H, 64 - hd), float("-inf"))
    q2 = torch.cat([q, pad], -1).reshape(B, L, H * 64)
    k2 = torch.cat([k, pad], -1).reshape(B, L, H * 64)
    v2 = torch.cat([v, torch.zeros(B, L, H, 64 - hd)], -1).reshape(B, L, H * 64)
    p2 = torch.cat([q2, k2, v2, torch.zeros(B, L, H * 64)], -1)
    y2 = O.slot_fwd(p2, g["f32hd32c128_gamma"], 64 * H, H, C, 0, block_c=128)[..., :hd]
    assert relmax(y2, g["f32hd32c128_y"]) > 0.05


@pytest.mark.parametrize("tag", ["c64b1", "c128b2", "hd32c64b1"])
@rtz
def test_gate_matches_reference_shipped_launch(tag):
    g = golden.load("gate")
    B, L, ds, dm, H, C = [int(v) for v in g[f"{tag}_meta"]]
    comb = O.gnorm_gate_cat(g[f"{tag}_yslot"], g[f"{tag}_yssm"], g[f"{tag}_projs"], g[f"{tag}_gw"],
                            g[f"{tag}_gb"], ds, H, C, mode="shipped")
    ref = g[f"{tag}_comb"]
    assert relmax(comb, ref) < 1e-2
    assert ulp_flip_fraction(comb, ref) < 0.01
    fixed = O.gnorm_gate_cat(g[f"{tag}_yslot"], g[f"{tag}_yssm"], g[f"{tag}_projs"], g[f"{tag}_gw"],
                             g[f"{tag}_gb"], ds, H, C, mode="fixed")
    assert relmax(fixed, ref) > 0.05, "shipped strides must differ from the fixed ones here"


@pytest.mark.parametrize("tag", ["d64c64", "d64hd32c128pad"])
@rtz
def test_block_matches_reference(tag):
    g = golden.load("block")
    B, L, ds, dm, H, C = [int(v) for v in g[f"{tag}_meta"]]
    sd = golden.state_dict(g, f"{tag}_")
    y = O.block_forward(sd, g[f"{tag}_x"], ds, H, C, mode="shipped")
    ref = g[f"{tag}_y"]
    assert y.shape == ref.shape
    assert relmax(y, ref) < 5e-3, relmax(y, ref)


@rtz
def test_fixed_mode_matches_fixed_launch_reference_c256():
    g = golden.load("fixed_c256")
    B, L, ds, dm, H, C = [int(v) for v in g["meta"]]
    sd = golden.state_dict(g, "")
    y = O.block_forward(sd, g["x"], ds, H, C, mode="fixed")
    assert relmax(y, g["y"]) < 5e-3, relmax(y, g["y"])


def test_per_step_decay_generalisation_reduces_to_reference():
    """slot_scan_decay_fwd with a constant decay equals slot_fwd (the reference path)."""
    torch.manual_seed(0)
    B, L, H, hd, C = 2, 128, 2, 64, 64
    q, k, v = (0.5 * torch.randn(B, L, H, hd) for _ in range(3))
    gamma = torch.tensor([0.93, 0.97])
    y1, _ = O.slot_scan_decay_fwd(q, k, v, torch.log(gamma).expand(B, L, H).contiguous(), C)
    projs = torch.cat([q.reshape(B, L, -1), k.reshape(B, L, -1), v.reshape(B, L, -1),
                       torch.zeros(B, L, H * hd)], -1)
    y2 = O.slot_fwd(projs, gamma, H * hd, H, C, 0, block_c=128)             # [B*H, N, C, hd]
    y2 = y2.reshape(B, H, L, hd).permute(0, 2, 1, 3)
    assert relmax(y1, y2) < 1e-4
