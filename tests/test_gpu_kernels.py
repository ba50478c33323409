"""GPU parity of each kernel against the CPU oracle and the reference golden vectors.

Tolerances: bf16 activations <= 2e-2 max-abs relative
to the reference output scale; fp32 state <= 1e-3.  fp32 activations are held to
tighter bounds where the reference has no bf16 rounding point in between."""
import pytest
import torch

import golden
import oracle as O
from hdcmamba_b200 import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"
BF16_TOL = 2e-2
STATE_TOL = 1e-3


def rel(a, b):
    a, b = a.detach().float().cpu(), b.detach().float().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-6))


def gen(seed):
    return torch.Generator().manual_seed(seed)


# ------------------------------------------------------------------ LN + conv
@pytest.mark.parametrize("tag", ["f32", "bf16"])
def test_lnconv_golden(tag):
    g = golden.load("lnconv")
    x = g[f"{tag}_x"]
    out, mean, rstd = ops.ln_conv(x.to(DEV), g[f"{tag}_nw"].to(DEV), g[f"{tag}_nb"].to(DEV), g[f"{tag}_cw"].to(DEV),
                                  g[f"{tag}_cb"].to(DEV), 1e-5, stats=True)
    ref_o, ref_m, ref_r = O.ln_conv_fwd(x, g[f"{tag}_nw"], g[f"{tag}_nb"], g[f"{tag}_cw"], g[f"{tag}_cb"], 1e-5)
    if tag == "f32":
        torch.testing.assert_close(out.cpu(), ref_o, rtol=1e-5, atol=1e-5)
        assert rel(out, g["f32_out"]) < 1e-5
    else:
        assert rel(out, ref_o) < 1e-2 and rel(out, g["bf16_out"]) < BF16_TOL
        assert float((out.cpu().float() != ref_o.float()).float().mean()) < 0.01
    assert rel(mean, ref_m) < 1e-2 and rel(rstd, ref_r) < 1e-2


@pytest.mark.parametrize("B,L,D,act", [(2, 1000, 2048, "none"), (1, 777, 768, "silu"), (3, 64, 1024, "none"),
                                       (2, 300, 256, "silu"), (1, 40, 96, "none"), (1, 129, 4096, "none")])
def test_lnconv_shapes_bf16(B, L, D, act):
    x = torch.randn(B, L, D, generator=gen(1)).bfloat16()
    nw = (1 + 0.1 * torch.randn(D, generator=gen(2))).bfloat16()
    nb = (0.1 * torch.randn(D, generator=gen(3))).bfloat16()
    cw = (0.2 * torch.randn(D, 4, generator=gen(4))).bfloat16()
    cb = (0.1 * torch.randn(D, generator=gen(5))).bfloat16()
    out = ops.ln_conv(x.to(DEV), nw.to(DEV), nb.to(DEV), cw.to(DEV), cb.to(DEV), 1e-5, act=act)
    ref, _, _ = O.ln_conv_fwd(x, nw, nb, cw, cb, 1e-5, act=act)
    assert rel(out, ref) < 1e-2
    assert float((out.cpu().float() != ref.float()).float().mean()) < 0.01


def test_lnconv_halo_equals_unsplit():
    """A segment with the 3 preceding rows as halo equals the same rows of the full run."""
    B, L, D = 2, 512, 768
    x = torch.randn(B, L, D, generator=gen(6)).bfloat16().to(DEV)
    p = [t.to(DEV) for t in (torch.ones(D).bfloat16(), torch.zeros(D).bfloat16(),
                             (0.3 * torch.randn(D, 4, generator=gen(7))).bfloat16(), torch.zeros(D).bfloat16())]
    full = ops.ln_conv(x, *p, 1e-5)
    seg = ops.ln_conv(x[:, 200:].contiguous(), *p, 1e-5, halo=x[:, 197:200].contiguous())
    assert torch.equal(seg, full[:, 200:])


# ------------------------------------------------------------------ SSM
@pytest.mark.parametrize("tag", ["f32c64", "f32c32", "bf16c64"])
def test_ssm_golden(tag):
    g = golden.load("ssm")
    B, L, ds, C = [int(v) for v in g[f"{tag}_meta"]]
    projs, A_log = g[f"{tag}_projs"], g[f"{tag}_A_log"]
    y = ops.ssm_scan(projs.to(DEV), A_log.to(DEV), ds, C)
    ref = O.ssm_chunk_fwd(projs, A_log, ds, C)
    assert rel(y, ref) < 1e-2
    assert float((y.cpu().float() != ref).float().mean()) < 0.02
    assert rel(y, g[f"{tag}_y"]) < BF16_TOL


# C = 16, 32, 64, 128, 256: the 16-step kernels (1 to 16 segments per chunk); C = 8 and 512:
# the general kernels
@pytest.mark.parametrize("B,L,ds,C", [(2, 1024, 64, 256), (1, 2048, 128, 256), (3, 512, 64, 64), (1, 384, 16, 128),
                                      (2, 320, 32, 32), (1, 256, 16, 16), (2, 96, 16, 8), (1, 1024, 32, 512)])
def test_ssm_bf16_vs_oracle(B, L, ds, C):
    P = 3 * ds + 40
    projs = torch.randn(B, L, P, generator=gen(8))
    projs[..., :ds] = projs[..., :ds] * 2 - 3
    projs = projs.bfloat16()
    A_log = torch.log(torch.linspace(0.99, 0.9999, ds)).bfloat16()
    y = ops.ssm_scan(projs.to(DEV), A_log.to(DEV), ds, C)
    ref = O.ssm_chunk_fwd(projs, A_log, ds, C)
    assert rel(y, ref) < 1e-2


def test_ssm_segment_split_is_exact():
    """Sequence-parallel form: statistics of all chunks, outputs of a later segment."""
    B, L, ds, C = 2, 2048, 64, 256
    projs = torch.randn(B, L, 3 * ds, generator=gen(9))
    projs[..., :ds] = projs[..., :ds] * 2 - 3
    projs = projs.bfloat16().to(DEV)
    A_log = torch.log(torch.linspace(0.99, 0.9999, ds)).to(DEV)
    full = ops.ssm_scan(projs, A_log, ds, C)
    stats = torch.cat([ops.ssm_chunk_stats(projs[:, :1024], A_log, ds, C),
                       ops.ssm_chunk_stats(projs[:, 1024:], A_log, ds, C)], 1)
    second = ops.ssm_scan_out(projs[:, 1024:], A_log, stats, 4, ds, C)
    assert torch.equal(second, full[:, 1024:])


# ------------------------------------------------------------------ slot
@pytest.mark.parametrize("tag", ["f32hd64", "f32hd32c128"])
def test_slot_golden_fp32(tag):
    g = golden.load("slot")
    B, L, ds, dm, H, C = [int(v) for v in g[f"{tag}_meta"]]
    projs = g[f"{tag}_projs"].to(DEV)
    hd = dm // H
    so = 3 * ds
    y = torch.empty(B * H, L // C, C, hd, device=DEV)
    ops.slot_scan(projs[..., so:so + dm], projs[..., so + dm:so + 2 * dm], projs[..., so + 2 * dm:so + 3 * dm], H, C,
                  gamma=g[f"{tag}_gamma"].to(DEV), y=y, y_strides=(H * L * hd, L * hd, hd))
    assert rel(y, g[f"{tag}_y"]) < 1e-4


def _slot_inputs(B, L, H, hd, seed, dtype=torch.bfloat16):
    q, k, v = (0.5 * torch.randn(B, L, H * hd, generator=gen(seed + i)) for i in range(3))
    return [t.to(dtype) for t in (q, k, v)]


@pytest.mark.parametrize("B,L,H,hd,C", [(1, 512, 2, 64, 64), (2, 512, 3, 64, 128), (1, 1024, 2, 64, 256),
                                        (1, 256, 2, 32, 64), (1, 256, 1, 128, 128), (2, 256, 2, 48, 64)])
def test_slot_bf16_vs_oracle(B, L, H, hd, C):
    q, k, v = _slot_inputs(B, L, H, hd, 10)
    gamma = torch.tensor([0.95, 0.9, 0.99][:H]).bfloat16()
    y = ops.slot_scan(q.to(DEV), k.to(DEV), v.to(DEV), H, C, gamma=gamma.to(DEV))
    projs = torch.cat([q, k, v, torch.zeros_like(q)], -1)
    ref = O.slot_fwd(projs, gamma, H * hd, H, C, 0, block_c=C)          # [B*H, N, C, hd]
    ref = ref.reshape(B, H, L, hd).permute(0, 2, 1, 3).reshape(B, L, H, hd)
    assert rel(y, ref) < BF16_TOL, rel(y, ref)


@pytest.mark.parametrize("C", [64, 256])
def test_slot_per_step_decay_and_state(C):
    B, L, H, hd = 2, 1024, 2, 64
    q, k, v = _slot_inputs(B, L, H, hd, 20)
    log_a = torch.log(torch.sigmoid(torch.randn(B, L, H, generator=gen(23)) + 3.0))
    y, R = ops.slot_scan(q.to(DEV), k.to(DEV), v.to(DEV), H, C, log_a=log_a.to(DEV), return_state=True)
    yr, Rr = O.slot_scan_decay_fwd(q.reshape(B, L, H, hd), k.reshape(B, L, H, hd), v.reshape(B, L, H, hd), log_a, C)
    assert rel(y, yr) < BF16_TOL
    assert rel(R, Rr) < STATE_TOL, rel(R, Rr)


def test_slot_state_chaining():
    """Two halves chained through state_in / state_out equal one pass (fp32 state)."""
    B, L, H, hd, C = 1, 1024, 2, 64, 128
    q, k, v = (t.to(DEV) for t in _slot_inputs(B, L, H, hd, 30))
    gamma = torch.tensor([0.97, 0.93]).bfloat16().to(DEV)
    y, R = ops.slot_scan(q, k, v, H, C, gamma=gamma, return_state=True)
    h = L // 2
    y1, R1 = ops.slot_scan(q[:, :h], k[:, :h], v[:, :h], H, C, gamma=gamma, return_state=True)
    y2, R2 = ops.slot_scan(q[:, h:], k[:, h:], v[:, h:], H, C, gamma=gamma, state_in=R1, return_state=True)
    # the tcgen05 path splits each run into its own segment plan, so halves agree
    # with the full run to fp32 rounding (before the bf16 output rounding)
    assert rel(y1, y[:, :h]) < 1e-2
    assert rel(y2, y[:, h:]) < 1e-2
    assert rel(R2, R) < 1e-4


# ------------------------------------------------------------------ gate / LN
@pytest.mark.parametrize("tag", ["c64b1", "c128b2", "hd32c64b1"])
def test_gate_shipped_golden(tag):
    g = golden.load("gate")
    B, L, ds, dm, H, C = [int(v) for v in g[f"{tag}_meta"]]
    hd, N, P = dm // H, L // C, 3 * ds + 4 * dm
    projs = g[f"{tag}_projs"].to(DEV)
    ys, yssm = g[f"{tag}_yslot"].to(DEV), g[f"{tag}_yssm"].to(DEV)
    out = torch.empty(B, L, ds + dm, device=DEV)
    ops.gate_cat(ys, (N * C * hd, C * hd, hd), 128, yssm, (B * L, ds), projs[..., 3 * ds + 3 * dm:], (B * L, 4 * dm),
                 g[f"{tag}_gw"].to(DEV), g[f"{tag}_gb"].to(DEV), out, (L * (ds + dm), ds + dm), B, L, H, hd, ds)
    ref = O.gnorm_gate_cat(g[f"{tag}_yslot"], g[f"{tag}_yssm"], g[f"{tag}_projs"], g[f"{tag}_gw"], g[f"{tag}_gb"],
                           ds, H, C, mode="shipped")
    assert rel(out, ref) < 1e-2
    assert float((out.cpu() != ref).float().mean()) < 0.01
    assert rel(out, g[f"{tag}_comb"]) < BF16_TOL


@pytest.mark.parametrize("rows,width,dtype", [(1000, 832, torch.bfloat16), (77, 320, torch.float32),
                                              (4096, 1152, torch.bfloat16), (300, 100, torch.bfloat16),
                                              (33, 2048, torch.bfloat16)])
def test_row_layernorm(rows, width, dtype):
    """Vectorized path (bf16, width % 8 == 0, <= 2048) and the scalar one (the others)."""
    x = (3 * torch.randn(rows, width, generator=gen(40)) + 1).to(dtype)
    y = ops.row_layernorm(x.to(DEV))
    ref = torch.nn.functional.layer_norm(x.float(), (width,)).to(dtype)
    assert rel(y, ref) < (1e-2 if dtype == torch.bfloat16 else 1e-5)
    xi = x.to(DEV)
    ops.row_layernorm(xi, out=xi)  # in place, as the Block runs it
    assert torch.equal(xi, y)


@pytest.mark.parametrize("rows,width,dtype", [(1000, 768, torch.bfloat16), (77, 320, torch.float32),
                                              (300, 100, torch.bfloat16), (64, 2048, torch.bfloat16)])
def test_layer_norm_affine_matches_nn_layernorm(rows, width, dtype):
    """The final norms (HdcMamba9v3Model.norm_final, the LM wrapper's norm) against
    nn.LayerNorm on the same device, dtype and parameters."""
    x = (3 * torch.randn(rows, width, generator=gen(41)) + 1).to(dtype).to(DEV)
    ln = torch.nn.LayerNorm(width).to(DEV).to(dtype)
    with torch.no_grad():
        ln.weight.copy_(1 + 0.1 * torch.randn(width, generator=gen(42)))
        ln.bias.copy_(0.1 * torch.randn(width, generator=gen(43)))
        ref = ln(x)
    y = ops.layer_norm(x, ln.weight, ln.bias, ln.eps)
    assert rel(y, ref) < (1e-2 if dtype == torch.bfloat16 else 1e-5)
