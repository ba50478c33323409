"""Parity at BASELINE.json's own configurations, full size, against the CPU oracle.

The oracle (oracle/restate.py) restates the reference forward (hdcmamba/model.py:22-404)
with every bf16 rounding point and is pinned to vectors recorded from the reference
itself (tests/test_oracle_golden.py).  Here it runs at the configurations' stated sizes:

* config 2: LN + causal conv1d at [8, 8192, 2048] bf16 (and with the fused SiLU);
* config 3: the per-step-decay slot scan at [4, 32768, 16, 64], chunk 64: every output and
  the final fp32 state of every (batch, head);
* config 4: the first two full-width layers (d1024, H16, ds128, chunk 256) of the seeded
  24-layer model at B8 x L4096;
* config 5: all 12 layers of the seeded d768 model at B1 x L32768, layer by layer (the
  oracle gets the GPU's input of each layer), and the logits of 512 positions.

Tolerances: bf16 activations <= 2e-2 max-abs relative to the
reference output scale; fp32 state <= 1e-3."""
import os

import pytest
import torch

import oracle as O
from hdcmamba_b200 import _lib, ops
from hdcmamba_b200.lm import build_lm, synthetic_ids

pytestmark = pytest.mark.gpu
DEV = "cuda"
BF16_TOL = 2e-2
STATE_TOL = 1e-3


def rel(a, b):
    a, b = a.detach().float().cpu(), b.detach().float().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-6))


def no_device_error():
    torch.cuda.synchronize()
    return _lib.load().hdc_device_error(1) == 0


@pytest.fixture(autouse=True)
def _threads():
    n = torch.get_num_threads()
    torch.set_num_threads(max(n, min(32, os.cpu_count() or 1)))
    yield
    torch.set_num_threads(n)


def test_config2_ln_conv_full_shape():
    """x bf16 [8, 8192, 2048] ~ N(0,1); conv weights N(0, 0.02), conv bias 0, LN gamma 1,
    beta 0, eps 1e-5."""
    B, L, D = 8, 8192, 2048
    g = torch.Generator().manual_seed(0)
    x = torch.randn(B, L, D, generator=g).bfloat16()
    cw = (0.02 * torch.randn(D, 4, generator=g)).bfloat16()
    nw, nb, cb = torch.ones(D).bfloat16(), torch.zeros(D).bfloat16(), torch.zeros(D).bfloat16()
    args = [t.to(DEV) for t in (nw, nb, cw, cb)]
    xd = x.to(DEV)
    out, mean, rstd = ops.ln_conv(xd, *args, 1e-5, stats=True)
    out_silu = ops.ln_conv(xd, *args, 1e-5, act="silu")
    assert no_device_error()
    ref, ref_m, ref_r = O.ln_conv_fwd(x, nw, nb, cw, cb, 1e-5)
    assert rel(out, ref) < 1e-2, rel(out, ref)
    assert float((out.cpu().float() != ref.float()).float().mean()) < 0.01  # ties / reassociation only
    assert rel(mean, ref_m) < 1e-2 and rel(rstd, ref_r) < 1e-2
    del ref
    ref_s, _, _ = O.ln_conv_fwd(x, nw, nb, cw, cb, 1e-5, act="silu")
    assert rel(out_silu, ref_s) < 1e-2, rel(out_silu, ref_s)


def test_config3_slot_scan_full_size_outputs_and_final_state():
    """q, k, v bf16 [4, 32768, 16, 64] ~ N(0,1), per-step decay a = sigmoid(N(0,1)) fp32,
    chunk 64, zero initial state: all outputs and the final state."""
    B, L, H, hd, C = 4, 32768, 16, 64, 64
    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn(B, L, H * hd, generator=g).bfloat16() for _ in range(3))
    log_a = torch.nn.functional.logsigmoid(torch.randn(B, L, H, generator=g))
    y, R = ops.slot_scan(q.to(DEV), k.to(DEV), v.to(DEV), H, C, log_a=log_a.to(DEV), return_state=True, path="tc")
    assert no_device_error()
    yr, Rr = O.slot_scan_decay_fwd(q.reshape(B, L, H, hd), k.reshape(B, L, H, hd), v.reshape(B, L, H, hd), log_a, C)
    assert rel(y, yr) < BF16_TOL, rel(y, yr)
    assert rel(R, Rr) < STATE_TOL, rel(R, Rr)
    # per (batch, head) as well: no sequence's state hides behind a larger one's scale
    Rg, Rrc = R.float().cpu().reshape(B * H, -1), Rr.float().reshape(B * H, -1)
    per = ((Rg - Rrc).abs().amax(1) / Rrc.abs().amax(1)).max()
    assert float(per) < STATE_TOL, float(per)


def _delta_rel(out, inp, ref):
    """Relative error of a residual layer's update (output - input), scaled by the
    reference update: the residual input itself cannot hide an error."""
    inp = inp.detach().float().cpu()
    return rel(out.float().cpu() - inp, ref.float() - inp)


def test_config4_first_two_layers_full_width():
    """Config 4's seeded model (24 x d1024, H16, ds128, chunk 256, vocab 50304): its first
    two layers on the embedded synthetic ids, B8 x L4096, against the oracle chained through
    the same two layers."""
    lm = build_lm("c4").bfloat16()
    sd = lm.state_dict()
    ids = synthetic_ids("c4")
    emb = lm.embedding.to(DEV)
    l0, l1 = lm.backbone.layers[0].to(DEV), lm.backbone.layers[1].to(DEV)
    with torch.no_grad():
        h0 = emb(ids.to(DEV))
        h1, _ = l0(h0)
        h2, _ = l1(h1)
    assert no_device_error()
    h0c = h0.cpu()
    o1 = O.block_forward(O.restate._sub(sd, "backbone.layers.0."), h0c, 128, 16, 256)
    assert rel(h1, o1) < BF16_TOL, rel(h1, o1)
    assert _delta_rel(h1, h0c, o1) < BF16_TOL, _delta_rel(h1, h0c, o1)
    o2 = O.block_forward(O.restate._sub(sd, "backbone.layers.1."), o1, 128, 16, 256)
    assert rel(h2, o2) < BF16_TOL, rel(h2, o2)


def test_config5_all_layers_full_length():
    """Config 5's seeded model (12 x d768, H12, ds64, chunk 256, vocab 50304) at B1 x L32768:
    every layer against the oracle fed that layer's GPU input, then the final norms and tied
    head at 512 positions of the full forward's logits."""
    lm = build_lm("c5").bfloat16()
    sd = lm.state_dict()
    ids = synthetic_ids("c5")
    lmd = lm.to(DEV)
    hs = []
    with torch.no_grad():
        h = lmd.embedding(ids.to(DEV))
        hs.append(h.cpu())
        for blk in lmd.backbone.layers:
            h, _ = blk(h)
            hs.append(h.cpu())
        logits = lmd(ids.to(DEV))
    rows = torch.cat([torch.arange(0, 256), torch.arange(32768 - 256, 32768)])
    got_rows = logits[0, rows.to(DEV)].cpu()
    del logits
    assert no_device_error()
    errs = []
    for i in range(12):
        o = O.block_forward(O.restate._sub(sd, f"backbone.layers.{i}."), hs[i], 64, 12, 256)
        errs.append((rel(hs[i + 1], o), _delta_rel(hs[i + 1], hs[i], o)))
    assert max(e for pair in errs for e in pair) < BF16_TOL, errs
    hl = hs[12][:, rows]
    hl = torch.nn.functional.layer_norm(hl.float(), (768,), sd["backbone.norm_final.weight"].float(),
                                        sd["backbone.norm_final.bias"].float()).bfloat16()
    hl = torch.nn.functional.layer_norm(hl.float(), (768,), sd["norm.weight"].float(),
                                        sd["norm.bias"].float()).bfloat16()
    ref_rows = (hl.float() @ sd["embedding.weight"].float().t()).bfloat16()[0]
    assert rel(got_rows, ref_rows) < BF16_TOL, rel(got_rows, ref_rows)


def test_config4_batch_shards_equal_the_whole_batch():
    """Batch sharding (config 4 on N GPUs): rank r runs samples [r*B/N, (r+1)*B/N) through the
    whole model with no collective.  Each shard's forward (here: the first two layers of the
    seeded config-4 model, two samples per shard as on 4 GPUs) equals the corresponding rows
    of the whole batch's forward within the bf16 tolerance (the slot kernels' segment plan
    and the GEMM tiling depend on the batch size, so the bits may differ)."""
    lm = build_lm("c4").bfloat16()
    ids = synthetic_ids("c4").to(DEV)
    emb = lm.embedding.to(DEV)
    layers = [lm.backbone.layers[i].to(DEV) for i in range(2)]

    def fwd(x):
        h = emb(x)
        for blk in layers:
            h, _ = blk(h)
        return h

    with torch.no_grad():
        whole = fwd(ids)
        for r in range(4):
            part = fwd(ids[2 * r:2 * r + 2].contiguous())
            assert rel(part, whole[2 * r:2 * r + 2]) < 1e-2, (r, rel(part, whole[2 * r:2 * r + 2]))
    assert no_device_error()
