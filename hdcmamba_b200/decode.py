"""Recurrent single-token decode for HdcMamba LMs (no counterpart in the reference, whose
generation re-runs the whole prefix for every new token, train.py:140-151).

``prefill(lm, ids)`` runs the prompt through the same kernels as the Block's forward
(fixed semantics) and keeps each layer's state at the end of the prompt; ``decode_step``
then adds one token per sequence in O(layer) work, with no re-run of the prefix:

* LN + conv: the three previous normalised rows;
* SSM: the chunk-local state, its summed log decay and the carry of the earlier chunks;
* slot memory: the state at the chunk start, the update of the chunk so far and the
  chunk's phi(k) / v rows.

The Block left-pads every sequence to a whole number of chunks (hdcmamba/model.py:386-394),
so a prompt always ends on a chunk boundary and decoding starts a fresh chunk.  Token i of
a chunk then gets row i of the chunked computation, with the prefill's rounding points:
decoding the tokens of chunk n one by one reproduces a prefill that ends with chunk n
(``tests/test_gpu_decode.py``).
"""
from dataclasses import dataclass, field
from typing import List

import torch
import torch.nn.functional as F

from . import ops


@dataclass
class LayerState:
    window: torch.Tensor    # fp32 [B, 3, dm]: normalised rows t-3..t-1
    ssm_h: torch.Tensor     # fp32 [B, ds]
    ssm_cum: torch.Tensor   # fp32 [B, ds]
    ssm_G: torch.Tensor     # fp32 [B, ds]
    R: torch.Tensor         # fp32 [B, H, 64, 64]: slot state at the chunk start
    U: torch.Tensor         # fp32 [B, H, 64, 64]: update of the chunk so far
    k_cache: torch.Tensor   # [B, H, C, 64]
    v_cache: torch.Tensor   # [B, H, C, 64]


@dataclass
class DecodeState:
    layers: List[LayerState] = field(default_factory=list)
    pos_dev: torch.Tensor = None   # device int32 [1]: index of the next token within its chunk
    chunk: int = 0

    @property
    def pos(self):
        return int(self.pos_dev.item())


def _blocks(lm):
    return list(lm.backbone.layers) if lm.use_model else list(lm.layers)


def _check(blk):
    if blk.semantics != "fixed":
        raise ValueError("decode needs semantics='fixed'")
    if blk.head_dim > 64:
        raise ValueError("decode supports head_dim <= 64")


def _window(xp, blk):
    """Normalised last three rows of the (padded) layer input, fp32 [B, 3, dm]."""
    x3 = xp[:, -3:, :].float()
    m = x3.mean(-1, keepdim=True)
    rs = torch.rsqrt(((x3 - m) ** 2).mean(-1, keepdim=True) + blk.norm.eps)
    nw = blk.norm.weight.to(xp.dtype).float()
    nb = blk.norm.bias.to(xp.dtype).float()
    return ((x3 * rs - m * rs) * nw + nb).contiguous()


def _prefill_block(blk, x):
    """HdcMamba9v3Block.forward (fixed semantics) that also returns the layer's state."""
    _check(blk)
    B, L_in, dm = x.shape
    C, H, hd, ds = blk.chunk_size, blk.num_heads, blk.head_dim, blk.d_state
    pad = (C - L_in % C) % C
    xp = F.pad(x, (0, 0, pad, 0)).contiguous() if pad else x.contiguous()
    L = xp.shape[1]
    x_conv = ops.ln_conv(xp, blk.norm.weight, blk.norm.bias, blk.conv1d.weight.squeeze(1), blk.conv1d.bias,
                         blk.norm.eps)
    projs = F.linear(x_conv, blk.in_proj.weight, blk.in_proj.bias)
    so = 3 * ds
    q, k, v = projs[..., so:so + dm], projs[..., so + dm:so + 2 * dm], projs[..., so + 2 * dm:so + 3 * dm]
    gate = projs[..., so + 3 * dm:]
    gamma = blk.gamma_buf.to(x.dtype)
    combined = torch.empty(B, L, ds + dm, device=x.device, dtype=x.dtype)
    stats = ops.ssm_chunk_stats(projs, blk.A_log, ds, C)
    ops.ssm_scan_out(projs, blk.A_log, stats, 0, ds, C, out=combined[..., :ds])
    if ops.slot_gate_supported(q, H, C):
        _, R = ops.slot_scan_gate(q, k, v, H, C, gate, blk.group_norm.weight, blk.group_norm.bias,
                                  combined[..., ds:], (L * (ds + dm), hd, ds + dm), gamma=gamma, return_state=True)
    else:
        N = L // C
        y_slot = torch.empty(B * H, N, C, hd, device=x.device, dtype=x.dtype)
        _, R = ops.slot_scan(q, k, v, H, C, gamma=gamma, y=y_slot, y_strides=(H * L * hd, L * hd, hd),
                             return_state=True)
        P = projs.shape[-1]
        ops.gate_cat(y_slot, (L * hd, C * hd, hd), C, combined, (L * (ds + dm), ds + dm), gate, (L * P, P),
                     blk.group_norm.weight, blk.group_norm.bias, combined, (L * (ds + dm), ds + dm), B, L, H, hd, ds)
    combined = ops.row_layernorm(combined, 1e-5, out=combined)
    y = torch.addmm(xp.reshape(-1, dm), combined.reshape(-1, ds + dm), blk.out_proj.weight.t()).reshape(B, L, dm)
    dev = x.device
    st = LayerState(
        window=_window(xp, blk),
        ssm_h=torch.zeros(B, ds, device=dev), ssm_cum=torch.zeros(B, ds, device=dev),
        ssm_G=ops.ssm_carry(stats, x.dtype),
        R=R.reshape(B, H, 64, 64).float().contiguous(), U=torch.zeros(B, H, 64, 64, device=dev),
        k_cache=torch.zeros(B, H, C, 64, device=dev, dtype=x.dtype),
        v_cache=torch.zeros(B, H, C, 64, device=dev, dtype=x.dtype))
    return y[:, pad:], st


def _step_block(blk, st, x, pos_dev):
    """One token per sequence through the Block: x [B, dm] -> [B, dm]."""
    B, dm = x.shape
    C, H, ds = blk.chunk_size, blk.num_heads, blk.d_state
    xc = ops.ln_conv_step(x, blk.norm.weight, blk.norm.bias, blk.conv1d.weight.squeeze(1), blk.conv1d.bias,
                          st.window, blk.norm.eps)
    projs = F.linear(xc, blk.in_proj.weight, blk.in_proj.bias)
    so = 3 * ds
    comb = torch.empty(B, ds + dm, device=x.device, dtype=x.dtype)
    ops.ssm_step(projs, blk.A_log, st.ssm_h, st.ssm_cum, st.ssm_G, ds, pos_dev, C, comb[:, :ds])
    ops.slot_step(projs[:, so:so + dm], projs[:, so + dm:so + 2 * dm], projs[:, so + 2 * dm:so + 3 * dm],
                  projs[:, so + 3 * dm:], H, blk.gamma_buf, blk.group_norm.weight, blk.group_norm.bias,
                  st.R, st.U, st.k_cache, st.v_cache, comb[:, ds:], pos_dev)
    comb = ops.row_layernorm(comb, 1e-5, out=comb)
    return torch.addmm(x, comb, blk.out_proj.weight.t())


@torch.no_grad()
def prefill(lm, ids):
    """Logits of the prompt ids [B, L] (as ``lm(ids)``) and the decode state after it."""
    h = lm.embedding(ids)
    state = DecodeState(pos_dev=torch.zeros(1, dtype=torch.int32, device=ids.device),
                        chunk=_blocks(lm)[0].chunk_size)
    for blk in _blocks(lm):
        h, st = _prefill_block(blk, h)
        state.layers.append(st)
    if lm.use_model:
        h = lm.backbone.norm_final(h)
    return F.linear(lm.norm(h), lm.embedding.weight), state


@torch.no_grad()
def decode_step(lm, state, ids):
    """Logits [B, vocab] of one new token per sequence (ids [B]); advances ``state``."""
    h = lm.embedding(ids)
    for blk, st in zip(_blocks(lm), state.layers):
        h = _step_block(blk, st, h, state.pos_dev)
    state.pos_dev.add_(1).remainder_(state.chunk)  # on the device: the step replays as a CUDA graph
    if lm.use_model:
        h = lm.backbone.norm_final(h)
    return F.linear(lm.norm(h), lm.embedding.weight)


class GraphedDecode:
    """``decode_step`` captured once as a CUDA graph for a fixed batch: ``__call__(ids)``
    copies ids [B] into the static input, replays, and returns the static logits.  The
    state tensors are updated in place by the replay."""

    def __init__(self, lm, state, example_ids, warmup=2):
        self.lm, self.state = lm, state
        self.static_ids = example_ids.clone()
        side = torch.cuda.Stream(device=example_ids.device)
        side.wait_stream(torch.cuda.current_stream(example_ids.device))
        saved = _snapshot(state)
        with torch.cuda.stream(side):
            for _ in range(warmup):
                decode_step(lm, state, self.static_ids)
        torch.cuda.current_stream(example_ids.device).wait_stream(side)
        _restore(state, saved)  # the warm-up steps must not advance the sequence
        self.graph = torch.cuda.CUDAGraph()
        _restore_after = _snapshot(state)
        with torch.cuda.graph(self.graph):
            self.static_out = decode_step(lm, state, self.static_ids)
        _restore(state, _restore_after)  # capturing does not run the kernels, but keep it exact

    def __call__(self, ids):
        self.static_ids.copy_(ids, non_blocking=True)
        self.graph.replay()
        return self.static_out


def _snapshot(state):
    return [t.clone() for st in state.layers for t in vars(st).values()] + [state.pos_dev.clone()]


def _restore(state, saved):
    it = iter(saved)
    for st in state.layers:
        for t in vars(st).values():
            t.copy_(next(it))
    state.pos_dev.copy_(next(it))

