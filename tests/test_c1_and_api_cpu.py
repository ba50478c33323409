"""CPU tests: seeded C1 weights, oracle vs the reference's C1 logits, the drop-in
module contract, and the C ABI library's exports (no GPU compute here)."""
import ctypes
import os
import re

import pytest
import torch

import golden
import oracle as O
from hdcmamba_b200 import HdcMamba9v3Block, HdcMamba9v3Model, _lib
from hdcmamba_b200.lm import CONFIGS, build_lm, synthetic_ids

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_c1_seeded_weights_match_reference_construction():
    g = golden.load("c1_lm")
    sd = build_lm("c1").state_dict()
    keys = sorted(k[3:] for k in g if k.startswith("ck."))
    assert sorted(sd.keys()) == keys
    for k in keys:
        v = sd[k].double()
        got = torch.tensor([float(v.sum()), float(v.abs().sum()), float(v.reshape(-1)[0]), float(v.reshape(-1)[-1])],
                           dtype=torch.float64)
        torch.testing.assert_close(got, g["ck." + k].double(), rtol=1e-9, atol=1e-9)


def test_c1_ids_are_the_fixture_ids():
    g = golden.load("c1_lm")
    assert torch.equal(synthetic_ids("c1"), g["ids"])


@pytest.mark.slow
def test_c1_oracle_logits_match_reference():
    """Config 1 end to end: oracle (shipped semantics, interpreter rounding) vs the
    reference run under TRITON_INTERPRET=1."""
    g = golden.load("c1_lm")
    cfg = CONFIGS["c1"]
    sd = {k: v.float() for k, v in build_lm("c1").state_dict().items()}
    with O.kernel_rounding("rtz"):
        logits = O.lm_forward(sd, g["ids"], cfg.n_layers, cfg.d_state, cfg.num_heads, cfg.chunk_size,
                              mode="shipped")
    ref = g["logits_rows"]
    got = logits[0, g["rows"].long()]
    rel = float((got - ref).abs().max() / ref.abs().max())
    assert rel < 2e-3, rel
    s = torch.tensor([float(logits.double().sum()), float(logits.double().abs().sum())], dtype=torch.float64)
    assert abs(float(s[1] - g["logits_sum"][1])) / float(g["logits_sum"][1]) < 1e-3


def test_block_state_dict_contract():
    """Parameter names and shapes equal the reference's (hdcmamba/model.py:306-327)."""
    g = golden.load("block")
    ref = golden.state_dict(g, "d64hd32c128pad_")
    blk = HdcMamba9v3Block(d_model=64, d_state=64, num_heads=2, chunk_size=128)
    sd = blk.state_dict()
    assert sorted(sd) == sorted(ref)
    for k in sd:
        assert tuple(sd[k].shape) == tuple(ref[k].shape), k
    blk.load_state_dict({k: v.clone() for k, v in ref.items()})


def test_seeded_block_init_matches_reference_seed():
    """Same torch seed, same weights as the reference Block construction (fixture seed 22)."""
    g = golden.load("block")
    ref = golden.state_dict(g, "d64hd32c128pad_")
    torch.manual_seed(22)
    blk = HdcMamba9v3Block(d_model=64, d_state=64, num_heads=2, chunk_size=128)
    for k, v in blk.state_dict().items():
        torch.testing.assert_close(v.float(), ref[k].float(), rtol=0, atol=0)


def test_cpu_inputs_raise_no_fallback():
    blk = HdcMamba9v3Block(d_model=64, d_state=64, num_heads=2, chunk_size=64).eval()
    with pytest.raises(RuntimeError, match="CUDA"):
        blk(torch.randn(1, 64, 64))
    m = HdcMamba9v3Model(d_model=64, n_layers=1, d_state=64, num_slots=4, num_heads=2)
    with pytest.raises(RuntimeError, match="CUDA"):
        m(torch.randn(1, 256, 64))


def test_shipped_semantics_guard():
    with pytest.raises(ValueError):
        HdcMamba9v3Block(d_model=64, semantics="bogus")


def _header_symbols():
    txt = open(os.path.join(ROOT, "include", "hdcmamba_b200.h")).read()
    return sorted(set(re.findall(r"\b(hdc_[a-z0-9_]+)\s*\(", txt)))


def test_library_exports_every_header_symbol():
    lib = _lib.load()
    syms = _header_symbols()
    assert syms, "no declarations found"
    for s in syms:
        assert hasattr(lib, s), f"{s} declared in include/hdcmamba_b200.h but not exported"
    assert set(syms) <= set(_lib.SIGNATURES), set(syms) - set(_lib.SIGNATURES)
    assert lib.hdc_version() >= 100
    assert lib.hdc_built_arch() == 100


def test_library_rejects_bad_arguments_without_a_gpu():
    """Argument checks run before any CUDA call, so they work on a CPU-only host."""
    lib = _lib.load()
    rc = lib.hdc_ln_conv_fwd(7, None, None, None, None, None, None, None, None, None, 1, 1, 8, 1e-5, 0, None)
    assert rc == -1
    rc = lib.hdc_ln_conv_fwd(1, ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16),
                             ctypes.c_void_p(16), None, ctypes.c_void_p(32), None, None, 1, 4, 12, 1e-5, 0, None)
    assert rc == -2 and b"multiple of 8" in lib.hdc_error_string()
    rc = lib.hdc_ssm_chunk_stats(1, ctypes.c_void_p(16), 1, 1, ctypes.c_void_p(16), ctypes.c_void_p(16), 1, 100, 48, 64,
                                 None)
    assert rc == -2
    assert lib.hdc_slot_workspace_bytes(1, 256, 2, 64, 64) > 0
    # the one-call SSM scan checks its arguments the same way
    rc = lib.hdc_ssm_scan_fwd(7, ctypes.c_void_p(16), 1, 1, ctypes.c_void_p(16), ctypes.c_void_p(16),
                              ctypes.c_void_p(32), 1, 1, 1, 256, 64, 64, None)
    assert rc == -1
    rc = lib.hdc_ssm_scan_fwd(1, ctypes.c_void_p(16), 1, 1, ctypes.c_void_p(16), ctypes.c_void_p(16),
                              ctypes.c_void_p(32), 1, 1, 1, 100, 48, 64, None)
    assert rc == -2


@pytest.mark.parametrize("D", [768, 2048])
def test_lnconv_bwd_plan_stays_within_one_wave(D):
    """The backward's segment plan (visible through its workspace size: one fp32 [7, D]
    partial per CTA) never launches more CTAs than one wave holds on the 148-SM part the
    library assumes without a GPU; rounding the segments per batch row up had given B = 8,
    D = 2048 152 CTAs, whose last 4 ran as a second wave."""
    lib = _lib.load()
    per_sm = max(1, min(4, 512 // ((D // 4 + 31) // 32 * 32)))
    for B in (1, 3, 8, 16, 37, 148, 200):
        for L in (64, 1000, 8192):
            ctas = lib.hdc_ln_conv_bwd_workspace_bytes(B, L, D) // (7 * D * 4)
            assert ctas >= B
            assert ctas <= max(B, 148 * per_sm), (B, L, ctas)
