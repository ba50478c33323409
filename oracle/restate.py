"""PyTorch-CPU restatement of the HdcMamba-9v3 layer forward (parity oracle).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU legs of bench.py.  The product path never calls into this file.

Every function follows one reference kernel or host routine of
``hdcmamba/model.py`` (N01N9/hdcmamba) and cites the lines it restates.  All
arithmetic is fp32; values are rounded to bf16 exactly where the reference
rounds them (``.to(tl.bfloat16)`` stores, bf16 buffers, ``.to(x.dtype)`` casts).

Behaviours of the shipped reference that are reproduced on purpose:

* Q1/Q2/Q3 -- the gate/concat launch (model.py:375-380) passes literal strides
  ``stride_ssm_b=B*L``, ``stride_gate_b=B*L``, ``stride_gate_l=4*dm`` and the
  kernel maps token l to slot row ``(l//128, l%128)`` (model.py:288).
  ``mode="shipped"`` reproduces these; ``mode="fixed"`` uses the true strides.
* Q4 -- ``_slot_all_fused`` only covers ``slot_block_c`` rows of a chunk
  (model.py:17, 245).  Shipped uses 128; fixed uses ``max(128, pow2(C))``.
* Q5 -- the carried-in slot state is weighted by gamma**i, the chunk update by
  gamma**C (model.py:267, 272).
* Q6 -- bf16 rounding of y_ssm, chunk states, summed log-decay, the prefix
  states, ``combined`` and gamma (model.py:196-198, 209, 233, 293, 335).
* Q9 -- for head_dim < BLOCK_SIZE_D (= max(64, pow2(head_dim))) the masked
  feature lanes of q and k load 0 and become phi(0) = exp(0) = 1, so the
  slot kernel works on features padded with ones (v is padded with zeros)
  (model.py:245-262).
* Q10 -- in the GroupNorm of the gate kernel the padded lanes carry
  ``-mean`` into the variance sum (model.py:290), so for head_dim below the
  block width the variance is ``var + (BLOCK - hd) * mean**2 / hd``.
"""
from __future__ import annotations

import contextlib
import math
from typing import Dict, Optional

import torch
import torch.nn.functional as F

__all__ = [
    "kernel_rounding", "bf16r", "kbf16", "next_pow2", "feature_block", "ln_conv_fwd", "ln_conv_bwd",
    "ssm_chunk_fwd",
    "ssm_chunk_states", "ssm_prefix", "slot_fwd", "gnorm_gate_cat",
    "combined_layer_norm", "block_forward", "model_forward", "lm_forward",
    "slot_scan_decay_fwd",
]


_KERNEL_ROUNDING = ["rne"]


@contextlib.contextmanager
def kernel_rounding(mode: str):
    """Select how fp32 -> bf16 conversions *inside the reference kernels* round.

    "rne" (default) is what the compiled Triton kernels do on a GPU
    (``cvt.rn.bf16.f32``).  "rtz" reproduces the Triton CPU interpreter, whose
    ``cast_impl`` converts fp32 -> bf16 by dropping the low 16 bits; it is used
    only to pin this restatement against golden vectors recorded under
    TRITON_INTERPRET=1.  Casts done by torch ops (Linear, layer_norm,
    ``.to(x.dtype)``) always round to nearest even."""
    if mode not in ("rne", "rtz"):
        raise ValueError(mode)
    old = _KERNEL_ROUNDING[0]
    _KERNEL_ROUNDING[0] = mode
    try:
        yield
    finally:
        _KERNEL_ROUNDING[0] = old


def bf16r(t: torch.Tensor) -> torch.Tensor:
    """Round an fp32 tensor to bf16 (nearest even, as torch does) and widen it back."""
    return t.to(torch.bfloat16).to(torch.float32)


def kbf16(t: torch.Tensor) -> torch.Tensor:
    """A bf16 store/cast inside a reference kernel (``.to(tl.bfloat16)``), widened back."""
    if _KERNEL_ROUNDING[0] == "rtz":
        t = t.float().contiguous()
        return (t.view(torch.int32) & -65536).view(torch.float32)
    return bf16r(t.float())


def next_pow2(n: int) -> int:
    """``triton.next_power_of_2``."""
    return 1 if n <= 1 else 1 << (n - 1).bit_length()


def feature_block(head_dim: int) -> int:
    """Width of the reference's per-head feature tile: ``max(64, pow2(hd))`` (model.py:17)."""
    return max(64, next_pow2(head_dim))


def _round_to(t: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """A kernel-side cast to ``dtype`` (bf16 or fp32), kept in fp32."""
    return kbf16(t) if dtype == torch.bfloat16 else t


def _kstore(t: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """A kernel store of fp32 values into a ``dtype`` buffer."""
    return _round_to(t, dtype).to(dtype)


# ---------------------------------------------------------------------------
# LayerNorm + causal depthwise conv1d (width 4)        model.py:22-72, 126-146
# ---------------------------------------------------------------------------
def ln_conv_fwd(x, norm_w, norm_b, conv_w, conv_b, eps: float, act: str = "none",
                halo: Optional[torch.Tensor] = None):
    """Restates ``_fused_norm_conv_fwd_kernel`` (model.py:22-72).

    ``out[t] = sum_k cw[:,k] * n[t-3+k] + cb`` with ``n = LN(x)``; rows before
    the sequence start are x = 0, whose LayerNorm is exactly ``norm_b``
    (model.py:47-57).  ``halo`` (an extension used by the sequence-parallel
    path) supplies the three real rows that precede the segment instead.
    ``act="silu"`` (an extension for the fused-activation variant) applies
    SiLU in fp32 before the store.  Returns (out in x.dtype, mean bf16, rstd bf16).
    """
    dtype = x.dtype
    B, L, D = x.shape
    nw = norm_w.to(dtype).float()
    nb = norm_b.to(dtype).float()
    cw = conv_w.reshape(D, 4).to(dtype).float()
    cb = conv_b.to(dtype).float()
    xf = x.float()
    mean = xf.sum(-1) / D
    xc = xf - mean[..., None]
    var = (xc * xc).sum(-1) / D
    rstd = torch.rsqrt(var + eps)
    n = (xc * rstd[..., None]) * nw + nb
    if halo is None:
        pre = nb.expand(B, 3, D)
    else:
        hf = halo.float()
        hm = hf.sum(-1) / D
        hc = hf - hm[..., None]
        hv = (hc * hc).sum(-1) / D
        pre = (hc * torch.rsqrt(hv + eps)[..., None]) * nw + nb
    npad = torch.cat([pre, n], dim=1)
    out = npad[:, 0:L] * cw[:, 0] + npad[:, 1:L + 1] * cw[:, 1] + npad[:, 2:L + 2] * cw[:, 2] \
        + npad[:, 3:L + 3] * cw[:, 3] + cb
    if act == "silu":
        out = out * torch.sigmoid(out)
    elif act != "none":
        raise ValueError(f"unknown activation {act!r}")
    return _kstore(out, dtype), _kstore(mean, torch.bfloat16), _kstore(rstd, torch.bfloat16)


def ln_conv_bwd(grad_out, x, mean, rstd, norm_w, conv_w):
    """Restates ``_fused_norm_conv_bwd_kernel`` (model.py:74-124) and its launch in
    ``FusedNormConv1dFunction.backward`` (model.py:148-166), reference quirks included:

    * ``dn[t] = sum_k go[t+3-k] cw[:,k]`` with go = 0 beyond the sequence end;
    * dx is the LayerNorm backward with the forward's bf16-stored mean / rstd
      (``mean.float()``, ``rstd.float()``, model.py:159);
    * ``d_cw[:,k] = sum_t go[t] * xhat[t-3+k] * nw`` -- the normalised input *without* the
      norm bias, and nothing from the three zero rows before the sequence (t-3+k < 0),
      although the forward uses LayerNorm(0) = norm_b there (model.py:112-121);
    * ``d_nb = sum_t dn[t]`` over real rows only; ``d_cb = sum_t go[t]``.

    Returns (dx in x.dtype, dnorm_w, dnorm_b, dconv_w [D, 4], dconv_b), the parameter
    gradients accumulated in fp32 and cast to x.dtype (model.py:166)."""
    dtype = x.dtype
    B, L, D = x.shape
    go = grad_out.float()
    xf = x.float()
    m = mean.float()[..., None]
    r = rstd.float()[..., None]
    nw = norm_w.float()
    cw = conv_w.reshape(D, 4).float()
    gp = torch.cat([go, go.new_zeros(B, 3, D)], 1)
    dn = gp[:, 0:L] * cw[:, 3] + gp[:, 1:L + 1] * cw[:, 2] + gp[:, 2:L + 2] * cw[:, 1] + gp[:, 3:L + 3] * cw[:, 0]
    xhat = (xf - m) * r
    dxhat = dn * nw
    dx = r * (dxhat - dxhat.sum(-1, keepdim=True) / D - xhat * ((dxhat * xhat).sum(-1, keepdim=True) / D))
    xw = xhat * nw
    dcw = torch.stack([(go[:, 3:] * xw[:, :L - 3]).sum((0, 1)), (go[:, 2:] * xw[:, :L - 2]).sum((0, 1)),
                       (go[:, 1:] * xw[:, :L - 1]).sum((0, 1)), (go * xw).sum((0, 1))], -1)
    return (_kstore(dx, dtype), (dn * xhat).sum((0, 1)).to(dtype), dn.sum((0, 1)).to(dtype), dcw.to(dtype),
            go.sum((0, 1)).to(dtype))


# ---------------------------------------------------------------------------
# Diagonal SSM chunked scan                                   model.py:175-233
# ---------------------------------------------------------------------------
def _ssm_terms(projs, A_log, ds):
    p = projs.float()
    dt, xv, bv = p[..., :ds], p[..., ds:2 * ds], p[..., 2 * ds:3 * ds]
    A = -torch.exp(A_log.float())
    dts = torch.where(dt > 20.0, dt, torch.log(1.0 + torch.exp(dt)))     # model.py:192
    ld = dts * A                                                            # model.py:193
    u = dts * bv * xv                                                       # model.py:195
    return ld, u


def ssm_chunk_states(projs, A_log, ds: int, C: int):
    """Intra-chunk pass of ``_ssm_intra_v2`` (model.py:175-198).

    Returns (y_intra [B,N,C,ds] bf16-rounded, cum_log [B,N,C,ds] fp32 inclusive,
    last_state [B,N,ds] bf16-rounded, chunk_decay [B,N,ds] bf16-rounded)."""
    B, L, _ = projs.shape
    N = L // C
    ld, u = _ssm_terms(projs, A_log, ds)
    ld = ld.reshape(B, N, C, ds)
    u = u.reshape(B, N, C, ds)
    acc = torch.zeros(B, N, ds)
    sld = torch.zeros(B, N, ds)
    y = torch.empty(B, N, C, ds)
    cum = torch.empty(B, N, C, ds)
    for c in range(C):
        sld = sld + ld[:, :, c]
        acc = acc * torch.exp(ld[:, :, c]) + u[:, :, c]
        y[:, :, c] = kbf16(acc)
        cum[:, :, c] = sld
    return y, cum, kbf16(acc), kbf16(sld)


def ssm_prefix(last_state, chunk_decay):
    """``_ssm_scan_v2`` (model.py:200-212): exclusive fp32 prefix, stored bf16."""
    B, N, ds = last_state.shape
    state = torch.zeros(B, ds)
    G = torch.empty(B, N, ds)
    for n in range(N):
        G[:, n] = kbf16(state)
        state = state * torch.exp(chunk_decay[:, n]) + last_state[:, n]
    return G, state


def ssm_chunk_fwd(projs, A_log, ds: int, C: int):
    """The three SSM kernels end to end (model.py:175-233, launched 345-363).

    Returns y_ssm [B, L, ds] as fp32 holding bf16-representable values."""
    B, L, _ = projs.shape
    y, cum, last, cdec = ssm_chunk_states(projs, A_log, ds, C)
    G, _ = ssm_prefix(last, cdec)
    out = kbf16(y + G[:, :, None] * torch.exp(cum))                        # model.py:230-233
    return out.reshape(B, L, ds)


# ---------------------------------------------------------------------------
# Slot memory: chunked decayed linear attention            model.py:235-272
# ---------------------------------------------------------------------------
def _phi(t):
    return torch.where(t > 0, t + 1.0, torch.exp(t))                        # model.py:261-262


def _slot_core(q_raw, k_raw, v, C, rows, dtype, decays, R0=None):
    """Shared loop of ``_slot_all_fused`` over all chunks of one sequence set.

    q_raw, k_raw, v: [G, N, rows, hd] fp32 (G = independent (b,h) sequences).
    decays(n) -> (decay_matrix [G,rows,rows], q_decay [G,rows], k_decay [G,rows],
    gamma_C [G]) for chunk n.  Features are padded to the reference block width
    (Q9).  Returns (y [G,N,rows,hd] fp32 pre-output-rounding, R [G,bd,bd])."""
    G, N, _, hd = q_raw.shape
    bd = feature_block(hd)
    q = _round_to(_phi(q_raw), dtype)
    k = _round_to(_phi(k_raw), dtype)
    vv = _round_to(v, dtype)
    if bd > hd:
        ones = torch.ones(G, N, rows, bd - hd)
        q = torch.cat([q, ones], -1)
        k = torch.cat([k, ones], -1)
        vv = torch.cat([vv, torch.zeros(G, N, rows, bd - hd)], -1)
    running = torch.zeros(G, bd, bd) if R0 is None else R0.clone().float()
    ys = torch.empty(G, N, rows, hd)
    causal = torch.tril(torch.ones(rows, rows, dtype=torch.bool))
    for n in range(N):
        dmat, qdec, kdec, gC = decays(n)
        qn, kn, vn = q[:, n], k[:, n], vv[:, n]
        scores = qn @ kn.transpose(1, 2)
        scores = _round_to(torch.where(causal, scores * dmat, torch.zeros(())), dtype)
        y_intra = scores @ vn
        y_inter = _round_to(qn * qdec[..., None], dtype) @ _round_to(running, dtype)
        ys[:, n] = (y_intra + y_inter)[..., :hd]
        kd = _round_to(kn * kdec[..., None], dtype)
        running = running * gC[:, None, None] + kd.transpose(1, 2) @ vn
    return ys, running


def slot_fwd(projs, gamma, d_model: int, num_heads: int, C: int, proj_offset: int,
             block_c: int = 128, R0=None, return_state: bool = False):
    """``_slot_all_fused`` as launched at model.py:365-371.

    gamma: [H] per-head decay (the reference casts gamma_buf to x.dtype,
    model.py:335 -- pass it already cast).  Returns y_slot [B*H, N, C, hd] in
    projs.dtype; rows a launch never writes (Q4: block_c < C) are NaN."""
    dtype = projs.dtype
    B, L, _ = projs.shape
    H, hd = num_heads, d_model // num_heads
    N = L // C
    rows = min(C, block_c)
    p = projs.float()

    def take(off):
        t = p[..., off:off + d_model].reshape(B, N, C, H, hd)[:, :, :rows]
        return t.permute(0, 3, 1, 2, 4).reshape(B * H, N, rows, hd)

    q_raw, k_raw, v = take(proj_offset), take(proj_offset + d_model), take(proj_offset + 2 * d_model)
    lg = torch.log(gamma.to(dtype).float()).repeat(B)                      # [B*H], model.py:248
    i = torch.arange(rows, dtype=torch.float32)
    diff = i[:, None] - i[None, :]
    dmat = torch.exp(diff[None] * lg[:, None, None])                        # model.py:251
    qdec = torch.exp(i[None] * lg[:, None])                                 # model.py:267
    kdec = torch.exp((C - 1 - i)[None] * lg[:, None])                       # model.py:249
    gC = torch.exp(C * lg)                                                  # model.py:248
    ys, R = _slot_core(q_raw, k_raw, v, C, rows, dtype, lambda n: (dmat, qdec, kdec, gC), R0)
    out = torch.full((B * H, N, C, hd), float("nan"))
    out[:, :, :rows] = _round_to(ys, dtype)
    out = out.to(dtype)
    return (out, R) if return_state else out


def slot_scan_decay_fwd(q, k, v, log_a, C: int, R0=None):
    """Per-step-decay generalisation of ``_slot_all_fused`` (benchmark config 3).

    q, k, v: [B, L, H, hd] raw (phi applied here); log_a: [B, L, H] fp32 log of
    the per-step decay a_t.  gamma**(i-j), gamma**i, gamma**(C-1-j), gamma**C of
    model.py:248-272 become exp(c_i - c_j), exp(c_i), exp(c_{C-1} - c_j) and
    exp(c_{C-1} + log a_{c0}) with c_i = sum_{t=1..i} log a_{c0+t} (fp32,
    sequential), which is the Q5 convention; constant a reduces to the
    reference.  Returns (y [B,L,H,hd] in q.dtype, R_final [B,H,bd,bd] fp32)."""
    dtype = q.dtype
    B, L, H, hd = q.shape
    N = L // C

    def arr(t):
        return t.float().reshape(B, N, C, H, hd).permute(0, 3, 1, 2, 4).reshape(B * H, N, C, hd)

    la = log_a.float().reshape(B, N, C, H).permute(0, 3, 1, 2).reshape(B * H, N, C)
    cum = torch.zeros(B * H, N, C)
    run = torch.zeros(B * H, N)
    for t in range(1, C):
        run = run + la[:, :, t]
        cum[:, :, t] = run

    def decays(n):
        c = cum[:, n]
        dmat = torch.exp(c[:, :, None] - c[:, None, :])
        return dmat, torch.exp(c), torch.exp(c[:, -1:] - c), torch.exp(c[:, -1] + la[:, n, 0])

    ys, R = _slot_core(arr(q), arr(k), arr(v), C, C, dtype, decays, R0)
    y = _round_to(ys, dtype).reshape(B, H, N, C, hd).permute(0, 2, 3, 1, 4).reshape(B, L, H, hd)
    return y.to(dtype), R.reshape(B, H, R.shape[-2], R.shape[-1])


# ---------------------------------------------------------------------------
# GroupNorm + sigmoid gate + concat                          model.py:274-295
# ---------------------------------------------------------------------------
def gnorm_gate_cat(y_slot, y_ssm, projs, gn_w, gn_b, d_state: int, num_heads: int,
                   C: int, mode: str = "fixed", slot_rows: int = 128):
    """``_fused_gnorm_gate_cat_kernel`` with the launch of model.py:375-380.

    y_slot: [B*H, N, C, hd]; y_ssm: [B, L, ds]; projs: [B, L, P].  In
    ``shipped`` mode the literal launch strides are reproduced (Q1, Q2) together
    with the kernel's 128-row slot map (Q3); ``fixed`` uses true strides.
    Returns combined [B, L, ds+dm] in projs.dtype (values bf16-rounded)."""
    dtype = projs.dtype
    B, L, P = projs.shape
    H = num_heads
    ds = d_state
    dm = (P - 3 * ds) // 4
    hd = dm // H
    N = L // C
    bd = feature_block(hd)
    ys_flat = y_slot.float().reshape(-1)
    yssm_flat = y_ssm.float().reshape(-1)
    pj_flat = projs.float().reshape(-1)
    b = torch.arange(B)[:, None, None, None]
    l = torch.arange(L)[None, :, None, None]
    h = torch.arange(H)[None, None, :, None]
    d = torch.arange(hd)[None, None, None, :]
    gate_off = 3 * ds + 3 * dm
    if mode == "shipped":
        slot_addr = (b * H + h) * (N * C * hd) + (l // slot_rows) * (C * hd) + (l % slot_rows) * hd + d
        gate_addr = gate_off + b * (B * L) + l * (4 * dm) + h * hd + d
        ssm_addr = torch.arange(B)[:, None, None] * (B * L) + torch.arange(L)[None, :, None] * ds \
            + torch.arange(ds)[None, None, :]
    elif mode == "fixed":
        slot_addr = (b * H + h) * (N * C * hd) + l * hd + d
        gate_addr = gate_off + b * (L * P) + l * P + h * hd + d
        ssm_addr = torch.arange(B)[:, None, None] * (L * ds) + torch.arange(L)[None, :, None] * ds \
            + torch.arange(ds)[None, None, :]
    else:
        raise ValueError(mode)
    yv = ys_flat[slot_addr]                                                 # [B, L, H, hd]
    mean = yv.sum(-1, keepdim=True) / hd
    yc = yv - mean
    var = ((yc * yc).sum(-1, keepdim=True) + (bd - hd) * mean * mean) / hd   # Q10
    w = gn_w.float().reshape(H, hd)
    bb = gn_b.float().reshape(H, hd)
    ygn = (yc / torch.sqrt(var + 1e-5)) * w + bb                            # model.py:291
    g = pj_flat[gate_addr]
    out = kbf16(ygn * (1.0 / (1.0 + torch.exp(-g))))                        # model.py:292-293
    comb = torch.empty(B, L, ds + dm)
    comb[..., ds:] = out.reshape(B, L, dm)
    comb[..., :ds] = yssm_flat[ssm_addr]                                     # model.py:294-295
    return comb.to(dtype)


def combined_layer_norm(combined):
    """``F.layer_norm(combined.float(), (ds+dm,)).to(x.dtype)`` (model.py:382)."""
    return F.layer_norm(combined.float(), (combined.shape[-1],)).to(combined.dtype)


# ---------------------------------------------------------------------------
# Block / model / LM                                        model.py:300-404
# ---------------------------------------------------------------------------
def _linear(x, w, b=None):
    """``nn.Linear`` in x.dtype: fp32 accumulate, one rounding to x.dtype."""
    y = x.float() @ w.float().t()
    if b is not None:
        y = y + b.float()
    return y.to(x.dtype)


def block_forward(sd: Dict[str, torch.Tensor], x, d_state: int, num_heads: int, chunk_size: int,
                  mode: str = "fixed", eps: float = 1e-5):
    """``HdcMamba9v3Block.forward`` in eval mode (model.py:386-394 and 331-384).

    sd: the block's state_dict (names as in model.py:306-327).  Returns y."""
    dtype = x.dtype
    B, L_in, dm = x.shape
    C, H, ds = chunk_size, num_heads, d_state
    pad = (C - L_in % C) % C
    if pad:
        x = F.pad(x, (0, 0, pad, 0))                                        # model.py:389
    B, L, _ = x.shape
    x_conv, _, _ = ln_conv_fwd(x, sd["norm.weight"], sd["norm.bias"], sd["conv1d.weight"],
                               sd["conv1d.bias"], eps)                       # model.py:338
    projs = _linear(x_conv, sd["in_proj.weight"].to(dtype), sd["in_proj.bias"].to(dtype))
    y_ssm = ssm_chunk_fwd(projs, sd["A_log"].to(dtype), ds, C).to(dtype)
    block_c = 128 if mode == "shipped" else max(128, next_pow2(C))
    gamma = sd["gamma_buf"].to(dtype)                                       # model.py:335
    y_slot = slot_fwd(projs, gamma, dm, H, C, 3 * ds, block_c=block_c)
    comb = gnorm_gate_cat(y_slot, y_ssm, projs, sd["group_norm.weight"].to(dtype),
                          sd["group_norm.bias"].to(dtype), ds, H, C, mode=mode)
    comb = combined_layer_norm(comb)
    res = _linear(comb, sd["out_proj.weight"].to(dtype))
    return (x + res)[:, pad:, :]                                            # model.py:394


def _sub(sd, prefix):
    return {k[len(prefix):]: v for k, v in sd.items() if k.startswith(prefix)}


def model_forward(sd, x, n_layers: int, d_state: int, num_heads: int, chunk_size: int = 256,
                  mode: str = "fixed"):
    """``HdcMamba9v3Model.forward`` (model.py:396-404; chunk 256 at model.py:399)."""
    for i in range(n_layers):
        x = block_forward(_sub(sd, f"layers.{i}."), x, d_state, num_heads, chunk_size, mode)
    return F.layer_norm(x.float(), (x.shape[-1],), sd["norm_final.weight"].float(),
                        sd["norm_final.bias"].float()).to(x.dtype)


def lm_forward(sd, ids, n_layers: int, d_state: int, num_heads: int, chunk_size: int,
               mode: str = "fixed", dtype=torch.float32, use_model_norm: bool = False):
    """LM wrapper of train.py:116-137: embedding -> blocks -> LayerNorm -> tied head.

    With ``use_model_norm`` the backbone is ``HdcMamba9v3Model`` (its own
    norm_final, keys ``backbone.*``); otherwise a plain list of blocks
    (keys ``layers.*``), which allows chunk sizes other than 256."""
    emb = sd["embedding.weight"].to(dtype)
    h = emb[ids]
    if use_model_norm:
        h = model_forward(_sub(sd, "backbone."), h, n_layers, d_state, num_heads, chunk_size, mode)
    else:
        for i in range(n_layers):
            h = block_forward(_sub(sd, f"layers.{i}."), h, d_state, num_heads, chunk_size, mode)
    h = F.layer_norm(h.float(), (h.shape[-1],), sd["norm.weight"].float(), sd["norm.bias"].float()).to(dtype)
    return _linear(h, emb)
