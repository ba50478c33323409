"""Tensor-level wrappers over the C ABI (include/hdcmamba_b200.h).

Each op validates device / dtype / layout, allocates its outputs through the torch
caching allocator on the current stream, and launches through ``_lib.call``.
Only CUDA tensors are accepted: there is no CPU path.
"""
import ctypes

import torch

from . import _lib

_DT = {torch.float32: _lib.HDC_F32, torch.bfloat16: _lib.HDC_BF16}


def _code(t):
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError(f"hdcmamba_b200: unsupported dtype {t.dtype} (float32 or bfloat16)") from None


def _cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("hdcmamba_b200 kernels run on CUDA tensors only (got a CPU tensor)")


def _stream(t):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _same_dtype(ref, *ts):
    for t in ts:
        if t is not None and t.dtype != ref.dtype:
            raise TypeError(f"hdcmamba_b200: dtype mismatch ({t.dtype} vs {ref.dtype})")


# ------------------------------------------------------------------ LN + conv
def ln_conv(x, norm_w, norm_b, conv_w, conv_b, eps=1e-5, act="none", halo=None, stats=False, halo_flag=None):
    """LayerNorm + causal depthwise conv1d (width 4), optional SiLU.

    Replaces ``_fused_norm_conv_fwd_kernel`` (hdcmamba/model.py:22-72).
    x: [B, L, D]; conv_w: [D, 4] or [D, 1, 4]; halo: optional [B, 3, D].
    halo_flag: optional (flag address, generation address) of device uint32s: the CTAs that
    read the halo wait until the flag reaches the generation (a halo stored by another GPU).
    Returns out (and bf16 mean, rstd [B, L] if ``stats``)."""
    _cuda(x, norm_w, norm_b, conv_w, conv_b, halo)
    B, L, D = x.shape
    x = x.contiguous()
    nw, nb = norm_w.to(x.dtype).contiguous(), norm_b.to(x.dtype).contiguous()
    cw = conv_w.reshape(D, 4).to(x.dtype).contiguous()
    cb = conv_b.to(x.dtype).contiguous()
    if halo is not None:
        halo = halo.to(x.dtype).contiguous()
        if tuple(halo.shape) != (B, 3, D):
            raise ValueError(f"halo must be [B, 3, D], got {tuple(halo.shape)}")
    out = torch.empty_like(x)
    mean = rstd = None
    if stats:
        mean = torch.empty(B, L, device=x.device, dtype=torch.bfloat16)
        rstd = torch.empty(B, L, device=x.device, dtype=torch.bfloat16)
    a = {"none": _lib.HDC_ACT_NONE, "silu": _lib.HDC_ACT_SILU}[act]
    if halo_flag is not None:
        if halo is None:
            raise ValueError("halo_flag needs a halo")
        _lib.call("hdc_ln_conv_fwd_halo_flag", _code(x), _p(x), _p(nw), _p(nb), _p(cw), _p(cb), _p(halo), _p(out),
                  _p(mean), _p(rstd), B, L, D, float(eps), a, ctypes.c_void_p(halo_flag[0]),
                  ctypes.c_void_p(halo_flag[1]), _stream(x))
    else:
        _lib.call("hdc_ln_conv_fwd", _code(x), _p(x), _p(nw), _p(nb), _p(cw), _p(cb), _p(halo), _p(out),
                  _p(mean), _p(rstd), B, L, D, float(eps), a, _stream(x))
    return (out, mean, rstd) if stats else out


# ------------------------------------------------------------------ SSM scan
def ln_conv_bwd(grad_out, x, mean, rstd, norm_w, conv_w):
    """Backward of ``ln_conv`` (act="none"): the reference's FusedNormConv1dFunction.backward
    (hdcmamba/model.py:74-124, 148-166), its formulas included.  ``mean`` / ``rstd`` are the
    forward's bf16 statistics.  Returns (dx, d_norm_w, d_norm_b, d_conv_w [D, 4], d_conv_b)
    in x.dtype."""
    _cuda(grad_out, x, mean, rstd, norm_w, conv_w)
    B, L, D = x.shape
    grad_out = grad_out.contiguous()
    x = x.contiguous()
    _same_dtype(x, grad_out)
    nw = norm_w.to(x.dtype).contiguous()
    cw = conv_w.reshape(D, 4).to(x.dtype).contiguous()
    mean = mean.to(torch.bfloat16).contiguous()
    rstd = rstd.to(torch.bfloat16).contiguous()
    dx = torch.empty_like(x)
    dnw = torch.empty(D, device=x.device, dtype=x.dtype)
    dnb = torch.empty_like(dnw)
    dcw = torch.empty(D, 4, device=x.device, dtype=x.dtype)
    dcb = torch.empty_like(dnw)
    ws = torch.empty(max(int(_lib.load().hdc_ln_conv_bwd_workspace_bytes(B, L, D)), 16), device=x.device,
                     dtype=torch.uint8)
    _lib.call("hdc_ln_conv_bwd", _code(x), _p(grad_out), _p(x), _p(mean), _p(rstd), _p(nw), _p(cw), _p(dx), _p(dnw),
              _p(dnb), _p(dcw), _p(dcb), _p(ws), ws.numel(), B, L, D, _stream(x))
    return dx, dnw, dnb, dcw, dcb


def _row_view(t, what):
    """(batch stride, row stride) of a [B, L, cols] view whose last dim is unit-stride."""
    if t.dim() != 3 or t.stride(2) != 1:
        raise ValueError(f"{what} must be a [B, L, cols] view with unit column stride")
    return t.stride(0), t.stride(1)


def ssm_chunk_stats(projs, A_log, d_state, chunk, out=None):
    """Per-chunk statistics [B, N, 2*ds] fp32 (last state, summed log decay), bf16-rounded.

    Replaces the last_state / chunk_decay outputs of ``_ssm_intra_v2`` (hdcmamba/model.py:175-198).
    ``out``: optional contiguous fp32 [B, N, 2*ds] tensor to write into."""
    _cuda(projs, A_log, out)
    B, L, P = projs.shape
    if P < 3 * d_state or L % chunk != 0:
        raise ValueError(f"projs [B, L, {P}] needs >= 3*d_state columns and L % chunk == 0")
    sb, st = _row_view(projs, "projs")
    a = A_log.to(projs.dtype).contiguous()
    shape = (B, L // chunk, 2 * d_state)
    if out is not None and (tuple(out.shape) != shape or out.dtype != torch.float32 or not out.is_contiguous()):
        raise ValueError(f"out must be a contiguous fp32 {list(shape)} tensor")
    stats = out if out is not None else torch.empty(shape, device=projs.device, dtype=torch.float32)
    _lib.call("hdc_ssm_chunk_stats", _code(projs), _p(projs), sb, st, _p(a), _p(stats), B, L, d_state, chunk,
              _stream(projs))
    return stats


def ssm_scan_out(projs, A_log, stats, n_prev, d_state, chunk, out=None):
    """Outputs of the chunked scan given chunk statistics of [0, n_prev + N) chunks.

    Replaces ``_ssm_scan_v2`` + ``_ssm_inter_v2`` (hdcmamba/model.py:200-233).
    ``out``: optional [B, L, >=ds] view (unit column stride) to write into."""
    _cuda(projs, A_log, stats, out)
    B, L, P = projs.shape
    if P < 3 * d_state or L % chunk != 0:
        raise ValueError(f"projs [B, L, {P}] needs >= 3*d_state columns and L % chunk == 0")
    sb, st = _row_view(projs, "projs")
    a = A_log.to(projs.dtype).contiguous()
    if out is None:
        out = torch.empty(B, L, d_state, device=projs.device, dtype=projs.dtype)
    _same_dtype(projs, out)
    osb, ost = _row_view(out, "out")
    stats = stats.contiguous()
    if stats.dtype != torch.float32 or stats.shape[0] != B or stats.shape[1] != n_prev + L // chunk:
        raise ValueError("stats must be fp32 [B, n_prev + L/chunk, 2*d_state]")
    _lib.call("hdc_ssm_scan_out", _code(projs), _p(projs), sb, st, _p(a), _p(stats), stats.stride(0), n_prev,
              _p(out), osb, ost, B, L, d_state, chunk, _stream(projs))
    return out


def ssm_scan_out_blocked(projs, A_log, stats, stats_sb, block_chunks, block_stride, n_prev, d_state, chunk,
                         out=None, wait=None):
    """ssm_scan_out reading the statistics of chunks [0, n_prev + N) in place from a
    rank-major gathered buffer: ``stats`` is a 1-D fp32 tensor whose element 0 is chunk 0
    of block 0; chunk m of batch b is at (m // block_chunks) * block_stride + b * stats_sb
    + (m % block_chunks) * 2 * ds (hdc_ssm_scan_out_blocked).  ``wait``: optional
    (flags address, mask, generation address): the kernel waits for the flags before it
    reads statistics stored by other GPUs."""
    _cuda(projs, A_log, stats, out)
    B, L, P = projs.shape
    if P < 3 * d_state or L % chunk != 0:
        raise ValueError(f"projs [B, L, {P}] needs >= 3*d_state columns and L % chunk == 0")
    if stats.dtype != torch.float32 or stats.dim() != 1 or stats.stride(0) != 1:
        raise ValueError("stats must be a 1-D contiguous fp32 tensor")
    m_end = n_prev + L // chunk
    last_blk = (m_end - 1) // block_chunks
    rows_in_last = m_end - last_blk * block_chunks
    need = last_blk * block_stride + (B - 1) * stats_sb + rows_in_last * 2 * d_state
    if need > stats.numel():
        raise ValueError(f"stats holds {stats.numel()} floats, the layout reads up to {need}")
    sb, st = _row_view(projs, "projs")
    a = A_log.to(projs.dtype).contiguous()
    if out is None:
        out = torch.empty(B, L, d_state, device=projs.device, dtype=projs.dtype)
    _same_dtype(projs, out)
    osb, ost = _row_view(out, "out")
    wf, wm, wg = wait if wait is not None else (0, 0, 0)
    _lib.call("hdc_ssm_scan_out_blocked", _code(projs), _p(projs), sb, st, _p(a), _p(stats), stats_sb, block_chunks,
              block_stride, n_prev, _p(out), osb, ost, B, L, d_state, chunk, ctypes.c_void_p(wf), wm,
              ctypes.c_void_p(wg), _stream(projs))
    return out


def ssm_scan(projs, A_log, d_state, chunk, out=None):
    """The whole diagonal-SSM chunked scan (hdcmamba/model.py:175-233, launched 345-363):
    ``hdc_ssm_scan_fwd``, statistics then outputs, enqueued back to back.
    ``out``: optional [B, L, >=ds] view (unit column stride) to write into."""
    _cuda(projs, A_log, out)
    B, L, P = projs.shape
    if P < 3 * d_state or L % chunk != 0:
        raise ValueError(f"projs [B, L, {P}] needs >= 3*d_state columns and L % chunk == 0")
    sb, st = _row_view(projs, "projs")
    a = A_log.to(projs.dtype).contiguous()
    if out is None:
        out = torch.empty(B, L, d_state, device=projs.device, dtype=projs.dtype)
    _same_dtype(projs, out)
    osb, ost = _row_view(out, "out")
    stats = torch.empty(B, L // chunk, 2 * d_state, device=projs.device, dtype=torch.float32)
    _lib.call("hdc_ssm_scan_fwd", _code(projs), _p(projs), sb, st, _p(a), _p(stats), _p(out), osb, ost, B, L,
              d_state, chunk, _stream(projs))
    return out


# ------------------------------------------------------------------ slot scan
def slot_workspace_bytes(B, L, H, hd, chunk):
    return int(_lib.load().hdc_slot_workspace_bytes(B, L, H, hd, chunk))


def feature_block(hd):
    b = 1
    while b < hd:
        b <<= 1
    return max(64, b)


_SLOT_PATHS = {"auto": 0, "simt": 1, "tc": 2}


def slot_scan(q, k, v, num_heads, chunk, gamma=None, log_a=None, rows=None, y=None, y_strides=None,
              state_in=None, return_state=False, path="auto", path_used=None):
    """Slot memory scan (replaces ``_slot_all_fused``, hdcmamba/model.py:236-272).

    q, k, v: [B, L, H*hd] views sharing strides (unit last-dim stride), raw
    (before phi).  gamma: [H] (in the activation dtype) or log_a: fp32 [B, L, H].
    y: optional output tensor with element strides ``y_strides = (sb, sh, st)``
    (element (b, t, h, d) at b*sb + h*sh + t*st + d); default [B, L, H, hd].
    path: "auto", "simt" (CUDA-core kernel) or "tc" (tcgen05 required, error otherwise);
    ``path_used`` (a list) receives "tc" or "simt".
    Returns y (and the fp32 final state [B, H, bd, bd] if ``return_state``)."""
    _cuda(q, k, v, gamma, log_a, y, state_in)
    if path not in _SLOT_PATHS:
        raise ValueError(f"path must be one of {sorted(_SLOT_PATHS)}")
    _same_dtype(q, k, v)
    B, L, W = q.shape
    H = num_heads
    hd = W // H
    if W != H * hd or k.shape != q.shape or v.shape != q.shape:
        raise ValueError("q, k, v must be [B, L, H*hd] with equal shapes")
    if q.stride() != k.stride() or q.stride() != v.stride() or q.stride(2) != 1:
        raise ValueError("q, k, v must share strides with unit last-dim stride")
    if (gamma is None) == (log_a is None):
        raise ValueError("give exactly one of gamma (constant decay) or log_a (per-step decay)")
    if gamma is not None:
        gamma = gamma.to(q.dtype).contiguous()
    if log_a is not None:
        log_a = log_a.float().contiguous()
        if tuple(log_a.shape) != (B, L, H):
            raise ValueError("log_a must be [B, L, H]")
    rows = chunk if rows is None else rows
    if y is None:
        y = torch.empty(B, L, H, hd, device=q.device, dtype=q.dtype)
        y_strides = (L * H * hd, hd, H * hd)
    elif y_strides is None:
        raise ValueError("y_strides is required with y")
    _same_dtype(q, y)
    bd = feature_block(hd)
    state_out = torch.empty(B, H, bd, bd, device=q.device, dtype=torch.float32) if return_state else None
    if state_in is not None:
        state_in = state_in.float().contiguous()
    nbytes = slot_workspace_bytes(B, L, H, hd, chunk)
    ws = torch.empty(max(nbytes, 16), device=q.device, dtype=torch.uint8)
    used = ctypes.c_int(-1)
    _lib.call("hdc_slot_scan_fwd_path", _code(q), _p(q), _p(k), _p(v), q.stride(0), q.stride(1), _p(gamma),
              _p(log_a), _p(y), y_strides[0], y_strides[1], y_strides[2], _p(state_in), _p(state_out), _p(ws),
              ws.numel(), B, L, H, hd, chunk, rows, _SLOT_PATHS[path], ctypes.byref(used), _stream(q))
    if path_used is not None:
        path_used.append("tc" if used.value == 1 else "simt")
    return (y, state_out) if return_state else y


def slot_gate_supported(q, num_heads, chunk):
    """True when hdc_slot_gate_fwd (tcgen05, fused gate epilogue) accepts these inputs."""
    B, L, W = q.shape
    hd = W // num_heads
    return (q.dtype == torch.bfloat16 and hd <= 64 and hd % 8 == 0 and W >= 64 and chunk in (64, 128, 256)
            and L % chunk == 0 and q.stride(2) == 1 and q.stride(1) % 8 == 0 and q.data_ptr() % 16 == 0)


def slot_scan_gate(q, k, v, num_heads, chunk, gate, gn_w, gn_b, out, out_strides, gamma=None, log_a=None,
                   state_in=None, return_state=False):
    """Slot scan with GroupNorm(head) * sigmoid(gate) fused into its epilogue
    (replaces ``_slot_all_fused`` plus the slot half of ``_fused_gnorm_gate_cat_kernel``,
    hdcmamba/model.py:236-293).  gate: [B, L, H*hd] view (unit last stride); out:
    tensor with element strides ``out_strides = (sb, sh, st)``."""
    _cuda(q, k, v, gamma, log_a, gate, gn_w, gn_b, out, state_in)
    _same_dtype(q, k, v, gate, out)
    B, L, W = q.shape
    H = num_heads
    hd = W // H
    if q.stride() != k.stride() or q.stride() != v.stride() or gate.stride(2) != 1:
        raise ValueError("q, k, v must share strides; gate needs a unit last stride")
    if (gamma is None) == (log_a is None):
        raise ValueError("give exactly one of gamma or log_a")
    if gamma is not None:
        gamma = gamma.to(q.dtype).contiguous()
    if log_a is not None:
        log_a = log_a.float().contiguous()
    gw = gn_w.to(q.dtype).contiguous()
    gb = gn_b.to(q.dtype).contiguous()
    bd = feature_block(hd)
    state_out = torch.empty(B, H, bd, bd, device=q.device, dtype=torch.float32) if return_state else None
    if state_in is not None:
        state_in = state_in.float().contiguous()
    ws = torch.empty(max(slot_workspace_bytes(B, L, H, hd, chunk), 16), device=q.device, dtype=torch.uint8)
    _lib.call("hdc_slot_gate_fwd", _code(q), _p(q), _p(k), _p(v), q.stride(0), q.stride(1), _p(gamma), _p(log_a),
              _p(gate), gate.stride(0), gate.stride(1), _p(gw), _p(gb), _p(out), out_strides[0], out_strides[1],
              out_strides[2], _p(state_in), _p(state_out), _p(ws), ws.numel(), B, L, H, hd, chunk, _stream(q))
    return (out, state_out) if return_state else out


def slot_workspace(B, L, num_heads, head_dim, chunk, device):
    """A device workspace for one slot call of this shape (uint8)."""
    return torch.empty(max(slot_workspace_bytes(B, L, num_heads, head_dim, chunk), 16), device=device,
                       dtype=torch.uint8)


def _f32_out(t, shape, what):
    if t is not None and (tuple(t.shape) != tuple(shape) or t.dtype != torch.float32 or not t.is_contiguous()):
        raise ValueError(f"{what} must be a contiguous fp32 {list(shape)} tensor")


def slot_state(k, v, num_heads, chunk, gamma=None, log_a=None, state_out=None, decay_out=None, workspace=None):
    """State after the whole sequence from a zero start, fp32 [B, H, 64, 64], and the
    product of all chunk decays [B, H] (for sequence-parallel carries).  ``workspace``
    (from ``slot_workspace``) keeps the segment states for ``slot_scan_gate_carry``."""
    _cuda(k, v, gamma, log_a, state_out, decay_out, workspace)
    _same_dtype(k, v)
    B, L, W = k.shape
    H = num_heads
    hd = W // H
    if k.stride() != v.stride() or k.stride(2) != 1:
        raise ValueError("k, v must share strides with unit last-dim stride")
    if gamma is not None:
        gamma = gamma.to(k.dtype).contiguous()
    if log_a is not None:
        log_a = log_a.float().contiguous()
    _f32_out(state_out, (B, H, 64, 64), "state_out")
    _f32_out(decay_out, (B, H), "decay_out")
    state = state_out if state_out is not None else torch.empty(B, H, 64, 64, device=k.device, dtype=torch.float32)
    decay = decay_out if decay_out is not None else torch.empty(B, H, device=k.device, dtype=torch.float32)
    ws = workspace if workspace is not None else slot_workspace(B, L, H, hd, chunk, k.device)
    _lib.call("hdc_slot_state_fwd", _code(k), _p(k), _p(v), k.stride(0), k.stride(1), _p(gamma), _p(log_a),
              _p(state), _p(decay), _p(ws), ws.numel(), B, L, H, hd, chunk, _stream(k))
    return state, decay


def slot_scan_gate_carry(q, k, v, num_heads, chunk, gate, gn_w, gn_b, out, out_strides, prev_state, prev_decay,
                         prev_stride, n_prev, workspace, gamma=None, log_a=None, wait=None):
    """``slot_scan_gate`` for one rank's part of the sequence (hdc_slot_gate_carry_fwd):
    the entering state folds the n_prev earlier parts, part s with its fp32 state at
    prev_state[s*prev_stride:] ([B, H, 64, 64]) and decay at prev_decay[s*prev_stride:]
    ([B, H]); ``workspace`` is the one ``slot_state`` filled for the same k, v.  ``wait``:
    optional (flags address, mask, generation address): the kernel waits for the flags
    before it reads earlier parts stored by other GPUs."""
    _cuda(q, k, v, gamma, log_a, gate, gn_w, gn_b, out, prev_state, prev_decay, workspace)
    _same_dtype(q, k, v, gate, out)
    B, L, W = q.shape
    H = num_heads
    hd = W // H
    if q.stride() != k.stride() or q.stride() != v.stride() or gate.stride(2) != 1:
        raise ValueError("q, k, v must share strides; gate needs a unit last stride")
    if (gamma is None) == (log_a is None):
        raise ValueError("give exactly one of gamma or log_a")
    if n_prev > 0:
        if prev_state.data_ptr() % 16 != 0 or prev_stride % 4 != 0:
            raise ValueError("prev_state must be 16-byte aligned and prev_stride a multiple of 4")
        for t, per in ((prev_state, B * H * 4096), (prev_decay, B * H)):
            if t.dtype != torch.float32 or t.dim() != 1 or t.stride(0) != 1:
                raise ValueError("prev_state / prev_decay must be 1-D contiguous fp32 tensors")
            if (n_prev - 1) * prev_stride + per > t.numel():
                raise ValueError("prev_state / prev_decay too short for n_prev parts")
    if gamma is not None:
        gamma = gamma.to(q.dtype).contiguous()
    if log_a is not None:
        log_a = log_a.float().contiguous()
    gw = gn_w.to(q.dtype).contiguous()
    gb = gn_b.to(q.dtype).contiguous()
    _lib.call("hdc_slot_gate_carry_fwd", _code(q), _p(q), _p(k), _p(v), q.stride(0), q.stride(1), _p(gamma),
              _p(log_a), _p(gate), gate.stride(0), gate.stride(1), _p(gw), _p(gb), _p(out), out_strides[0],
              out_strides[1], out_strides[2], _p(prev_state if n_prev else None), _p(prev_decay if n_prev else None),
              prev_stride, n_prev, None, _p(workspace), workspace.numel(), B, L, H, hd, chunk,
              ctypes.c_void_p(wait[0] if wait else 0), wait[1] if wait else 0, ctypes.c_void_p(wait[2] if wait else 0),
              _stream(q))
    return out


# ------------------------------------------------------------------ gate / concat / LN
def gate_cat(y_slot, slot_strides, slot_rows, y_ssm, ssm_strides, gate, gate_strides, gn_w, gn_b, out,
             out_strides, B, L, H, hd, ds):
    """GroupNorm(head) * sigmoid(gate), concatenated after y_ssm (replaces
    ``_fused_gnorm_gate_cat_kernel``, hdcmamba/model.py:274-295).  Strides are in
    elements and follow the reference launch (hdcmamba/model.py:377); the
    pointers are the base addresses of the given tensors (views allowed)."""
    _cuda(y_slot, y_ssm, gate, gn_w, gn_b, out)
    _same_dtype(out, y_slot, y_ssm, gate)
    gw = gn_w.to(out.dtype).contiguous()
    gb = gn_b.to(out.dtype).contiguous()
    _lib.call("hdc_gate_cat_fwd", _code(out), _p(y_slot), slot_strides[0], slot_strides[1], slot_strides[2],
              slot_rows, _p(y_ssm), ssm_strides[0], ssm_strides[1], _p(gate), gate_strides[0], gate_strides[1],
              _p(gw), _p(gb), _p(out), out_strides[0], out_strides[1], B, L, H, hd, ds, _stream(out))
    return out


def row_layernorm(x, eps=1e-5, out=None):
    """LayerNorm over the last dim without affine, fp32 statistics, result in x.dtype
    (replaces ``F.layer_norm(combined.float(), (ds+dm,)).to(x.dtype)``, hdcmamba/model.py:382)."""
    _cuda(x, out)
    if not x.is_contiguous():
        raise ValueError("row_layernorm needs a contiguous input")
    if out is None:
        out = torch.empty_like(x)
    width = x.shape[-1]
    _lib.call("hdc_row_layernorm", _code(x), _p(x), _p(out), x.numel() // width, width, float(eps), _stream(x))
    return out


def layer_norm(x, weight, bias, eps=1e-5, out=None):
    """nn.LayerNorm over the last dim with its elementwise affine: fp32 statistics and
    affine, result in x.dtype (hdc_row_layernorm_affine; replaces the final norms,
    hdcmamba/model.py:400, 404 and train.py:121, 135)."""
    _cuda(x, weight, bias, out)
    if not x.is_contiguous():
        raise ValueError("layer_norm needs a contiguous input")
    if out is None:
        out = torch.empty_like(x)
    width = x.shape[-1]
    w, b = weight.to(x.dtype).contiguous(), bias.to(x.dtype).contiguous()
    _lib.call("hdc_row_layernorm_affine", _code(x), _p(x), _p(w), _p(b), _p(out), x.numel() // width, width,
              float(eps), _stream(x))
    return out


# ------------------------------------------------------------------ single-token decode
def ln_conv_step(x, norm_w, norm_b, conv_w, conv_b, window, eps=1e-5, out=None):
    """LN + conv of one new row per sequence, x [B, D]; ``window`` fp32 [B, 3, D] (the
    normalised rows t-3..t-1) is shifted in place (hdc_ln_conv_step)."""
    _cuda(x, norm_w, norm_b, conv_w, conv_b, window, out)
    B, D = x.shape
    x = x.contiguous()
    if window.dtype != torch.float32 or tuple(window.shape) != (B, 3, D) or not window.is_contiguous():
        raise ValueError(f"window must be a contiguous fp32 [{B}, 3, {D}] tensor")
    dt = x.dtype
    out = torch.empty_like(x) if out is None else out
    _lib.call("hdc_ln_conv_step", _code(x), _p(x), _p(norm_w.to(dt).contiguous()), _p(norm_b.to(dt).contiguous()),
              _p(conv_w.reshape(D, 4).to(dt).contiguous()), _p(conv_b.to(dt).contiguous()), _p(window), _p(out), B, D,
              float(eps), _stream(x))
    return out


def ssm_step(projs, A_log, h, cum, G, d_state, pos, chunk, out):
    """One diagonal-SSM step for rows projs [B, P]; h / cum / G fp32 [B, ds] updated in
    place; ``pos`` a device int32 tensor holding the row index within the chunk (the chunk
    is folded into G at row chunk-1); writes out [B, >=ds] (unit column stride)."""
    _cuda(projs, A_log, h, cum, G, out, pos)
    B = projs.shape[0]
    if projs.stride(1) != 1 or out.stride(1) != 1:
        raise ValueError("projs / out need a unit column stride")
    a = A_log.to(projs.dtype).contiguous()
    _lib.call("hdc_ssm_step", _code(projs), _p(projs), projs.stride(0), _p(a), _p(h), _p(cum), _p(G), _p(out),
              out.stride(0), B, d_state, _p(pos), chunk, _stream(projs))
    return out


def ssm_carry(stats, dtype):
    """Carry G [B, ds] fp32 after the chunks of ``stats`` [B, N, 2ds] (hdc_ssm_carry_fwd);
    ``dtype`` is the activation dtype (selects the exp of that prefill path)."""
    _cuda(stats)
    B, N, two_ds = stats.shape
    G = torch.empty(B, two_ds // 2, device=stats.device, dtype=torch.float32)
    code = 1 if dtype == torch.bfloat16 else 0
    _lib.call("hdc_ssm_carry_fwd", code, _p(stats.contiguous()), B, N, two_ds // 2, _p(G), _stream(stats))
    return G


def slot_step(q, k, v, gate, num_heads, gamma, gn_w, gn_b, R, U, k_cache, v_cache, out, pos):
    """The next row (index in the device int32 ``pos``) of the current chunk of the slot
    scan with GroupNorm(head) * sigmoid(gate) (hdc_slot_step).  q / k / v / gate: [B, H*hd] views sharing one batch stride; R / U fp32
    [B, H, 64, 64]; k_cache / v_cache [B, H, C, 64]; out [B, H*hd] view (unit column stride)."""
    _cuda(q, k, v, gate, gamma, gn_w, gn_b, R, U, k_cache, v_cache, out, pos)
    B, W = q.shape
    H = num_heads
    hd = W // H
    C = k_cache.shape[2]
    if not (q.stride() == k.stride() == v.stride() == gate.stride()) or q.stride(1) != 1 or out.stride(1) != 1:
        raise ValueError("q / k / v / gate must share strides with unit column stride")
    dt = q.dtype
    _lib.call("hdc_slot_step", _code(q), _p(q), _p(k), _p(v), _p(gate), q.stride(0), _p(gamma.to(dt).contiguous()),
              _p(gn_w.to(dt).contiguous()), _p(gn_b.to(dt).contiguous()), _p(R), _p(U), _p(k_cache), _p(v_cache),
              _p(out), out.stride(0), B, H, hd, C, _p(pos), _stream(q))
    return out

