"""Drop-in module API of ``hdcmamba/model.py`` (N01N9/hdcmamba) on B200 kernels.

``HdcMamba9v3Block``, ``HdcMamba9v3Model``, ``FusedNormConv1dFunction`` and
``fused_norm_conv1d_trainable`` keep the reference's names, constructor
arguments, parameter names / shapes / init (hdcmamba/model.py:300-329) and
``forward`` contracts, so reference state_dicts load unchanged.  The layer's
hot path runs through libhdcmamba_b200.so (hdcmamba_b200/ops.py); the dense
projections stay on cuBLAS through torch.  There is no CPU path: CPU inputs
raise.

Semantics switch (constructor keyword ``semantics``, default ``"fixed"``):
  * ``"shipped"`` reproduces the reference launch exactly, including its stride
    quirks in the gate/concat launch (hdcmamba/model.py:377) and its 128-row
    slot map (hdcmamba/model.py:288).  Those index other samples and rows, so it
    is only accepted for chunk_size <= 128 and shapes whose addresses stay in
    bounds.
  * ``"fixed"`` uses the true strides and a full-chunk slot tile.  It is the
    semantics of batch sharding, sequence parallelism and chunk 256.
"""
import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.utils.checkpoint import checkpoint

from . import ops

__all__ = ["HdcMamba9v3Block", "HdcMamba9v3Model", "FusedNormConv1dFunction", "fused_norm_conv1d_trainable"]


_SIDE_STREAMS = {}


def _side_stream(device):
    """A second stream per device for work that overlaps the slot scan (the SSM scan)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    st = _SIDE_STREAMS.get(idx)
    if st is None:
        st = _SIDE_STREAMS[idx] = torch.cuda.Stream(device=idx)
    return st


_EXCHANGE_STREAMS = {}


def _exchange_stream(device):
    """A third stream per device for sequence-parallel puts that no local kernel waits for."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    st = _EXCHANGE_STREAMS.get(idx)
    if st is None:
        st = _EXCHANGE_STREAMS[idx] = torch.cuda.Stream(device=idx)
    return st


def _require_cuda(x):
    if not x.is_cuda:
        raise RuntimeError("hdcmamba_b200 runs on CUDA devices only; move the module and input to a B200")


class FusedNormConv1dFunction(torch.autograd.Function):
    """LayerNorm + causal depthwise conv1d (hdcmamba/model.py:126-166).

    forward(x, norm_weight, norm_bias, conv_weight[D,4], conv_bias, eps) -> out.
    backward runs ``hdc_ln_conv_bwd``: the reference's backward formulas
    (model.py:74-124), which leave the norm bias and the rows before the sequence out
    of the conv-weight and norm-bias gradients."""

    @staticmethod
    def forward(ctx, x, norm_weight, norm_bias, conv_weight, conv_bias, eps):
        _require_cuda(x)
        out, mean, rstd = ops.ln_conv(x, norm_weight, norm_bias, conv_weight, conv_bias, eps, stats=True)
        ctx.save_for_backward(x, norm_weight, conv_weight, mean, rstd)
        ctx.eps = eps
        return out

    @staticmethod
    def backward(ctx, grad_out):
        x, nw, cw, mean, rstd = ctx.saved_tensors
        dx, dnw, dnb, dcw, dcb = ops.ln_conv_bwd(grad_out, x, mean, rstd, nw, cw)
        return dx, dnw.to(nw.dtype), dnb.to(nw.dtype), dcw.reshape(cw.shape).to(cw.dtype), dcb.to(nw.dtype), None


def final_layer_norm(norm, x):
    """``norm(x)`` for an ``nn.LayerNorm`` over the last dim: through
    hdc_row_layernorm_affine when no autograd graph is needed, else the module itself
    (gradients for its weight and bias)."""
    if torch.is_grad_enabled() and (x.requires_grad or norm.weight.requires_grad):
        return norm(x)
    _require_cuda(x)
    return ops.layer_norm(x.contiguous(), norm.weight, norm.bias, norm.eps)


def fused_norm_conv1d_trainable(x, norm_layer, conv_layer):
    """hdcmamba/model.py:168-172."""
    return FusedNormConv1dFunction.apply(
        x, norm_layer.weight.to(x.dtype), norm_layer.bias.to(x.dtype),
        conv_layer.weight.squeeze(1).to(x.dtype), conv_layer.bias.to(x.dtype), norm_layer.eps,
    )


class HdcMamba9v3Block(nn.Module):
    """hdcmamba/model.py:300-394 on B200 kernels."""

    def __init__(self, d_model=512, d_state=64, num_heads=8, chunk_size=256, semantics="fixed"):
        super().__init__()
        if semantics not in ("fixed", "shipped"):
            raise ValueError("semantics must be 'fixed' or 'shipped'")
        if d_model % num_heads != 0:
            raise ValueError("d_model must be a multiple of num_heads")
        self.d_model, self.d_state, self.num_heads, self.chunk_size = d_model, d_state, num_heads, chunk_size
        self.head_dim = d_model // num_heads
        self.semantics = semantics

        # Parameter construction and init in the reference's order (hdcmamba/model.py:306-327),
        # so that the same torch seed yields the same weights.
        self.norm = nn.LayerNorm(d_model)
        self.conv1d = nn.Conv1d(d_model, d_model, kernel_size=4, groups=d_model, padding=3, bias=True)
        with torch.no_grad():
            nn.init.normal_(self.conv1d.weight, std=0.02)
            self.conv1d.weight[:, 0, -1] += 1.0
            self.conv1d.bias.fill_(0.0)
        self.in_proj = nn.Linear(d_model, d_state * 3 + d_model * 4, bias=True)
        with torch.no_grad():
            dt = torch.rand(d_state) * (0.1 - 0.001) + 0.001
            self.in_proj.bias[:d_state] = torch.log(torch.exp(dt) - 1.0)
            qkv0, qkv1 = d_state * 3, d_state * 3 + d_model * 3
            nn.init.xavier_uniform_(self.in_proj.weight[qkv0:qkv1])
            self.in_proj.bias[qkv1:].fill_(1.0)
        self.A_log = nn.Parameter(torch.log(torch.linspace(0.99, 0.9999, d_state)))
        self.decay_log = nn.Parameter(torch.log(torch.ones(num_heads) * 0.05))
        self.out_proj = nn.Linear(d_state + d_model, d_model, bias=False)
        self.group_norm = nn.GroupNorm(num_heads, d_model)
        self.register_buffer("gamma_buf", torch.exp(-F.softplus(self.decay_log)))

    # -- the layer body ---------------------------------------------------------------
    def _mix(self, x):
        """Everything between the input and out_proj: returns LayerNorm(combined) [B, L, ds+dm]."""
        B, L, _ = x.shape
        C, H, hd, ds, dm = self.chunk_size, self.num_heads, self.head_dim, self.d_state, self.d_model
        N = L // C
        x_conv = fused_norm_conv1d_trainable(x, self.norm, self.conv1d)
        projs = self.in_proj(x_conv)
        gamma = self.gamma_buf.to(x.dtype)
        so = 3 * ds
        q, k, v = projs[..., so:so + dm], projs[..., so + dm:so + 2 * dm], projs[..., so + 2 * dm:so + 3 * dm]
        combined = torch.empty(B, L, ds + dm, device=x.device, dtype=x.dtype)
        P = projs.shape[-1]
        if self.semantics == "fixed" and ops.slot_gate_supported(q, H, C):
            # SSM written into combined[..., :ds] on a side stream, concurrently with the slot
            # scan (GroupNorm * sigmoid(gate) fused into its epilogue) into combined[..., ds:];
            # the slot kernels are enqueued first, so their CTAs take the SMs first and the
            # SSM's fill the SMs they leave
            cur = torch.cuda.current_stream(x.device)
            side = _side_stream(x.device)
            side.wait_stream(cur)
            ops.slot_scan_gate(q, k, v, H, C, projs[..., so + 3 * dm:], self.group_norm.weight,
                               self.group_norm.bias, combined[..., ds:], (L * (ds + dm), hd, ds + dm), gamma=gamma)
            with torch.cuda.stream(side):
                ops.ssm_scan(projs, self.A_log, ds, C, out=combined[..., :ds])
            cur.wait_stream(side)
        elif self.semantics == "fixed":
            y_ssm = ops.ssm_scan(projs, self.A_log, ds, C, out=combined[..., :ds])
            y_slot = torch.empty(B * H, N, C, hd, device=x.device, dtype=x.dtype)
            ops.slot_scan(q, k, v, H, C, gamma=gamma, y=y_slot, y_strides=(H * L * hd, L * hd, hd))
            ops.gate_cat(y_slot, (L * hd, C * hd, hd), C, combined, (L * (ds + dm), ds + dm),
                         projs[..., so + 3 * dm:], (L * P, P), self.group_norm.weight, self.group_norm.bias,
                         combined, (L * (ds + dm), ds + dm), B, L, H, hd, ds)
        else:
            self._check_shipped(B, L, P)
            y_ssm = ops.ssm_scan(projs, self.A_log, ds, C)
            y_slot = torch.empty(B * H, N, C, hd, device=x.device, dtype=x.dtype)
            ops.slot_scan(q, k, v, H, C, gamma=gamma, rows=min(C, 128), y=y_slot,
                          y_strides=(H * L * hd, L * hd, hd))
            # the reference's literal launch arguments (hdcmamba/model.py:377)
            ops.gate_cat(y_slot, (N * C * hd, C * hd, hd), 128, y_ssm, (B * L, ds),
                         projs[..., so + 3 * dm:], (B * L, dm * 4), self.group_norm.weight,
                         self.group_norm.bias, combined, (L * (ds + dm), ds + dm), B, L, H, hd, ds)
        return ops.row_layernorm(combined, 1e-5, out=combined)

    def _check_shipped(self, B, L, P):
        C, H, hd, ds, dm = self.chunk_size, self.num_heads, self.head_dim, self.d_state, self.d_model
        if C > 128:
            raise ValueError("semantics='shipped' reads past y_slot for chunk_size > 128 "
                             "(hdcmamba/model.py:288); use semantics='fixed'")
        last_gate = 3 * ds + 3 * dm + (B - 1) * B * L + (L - 1) * 4 * dm + dm
        last_ssm = (B - 1) * B * L + (L - 1) * ds + ds
        last_slot = (B * H - 1) * L * hd + ((L - 1) // 128) * C * hd + 127 * hd + hd
        if last_gate > B * L * P or last_ssm > B * L * ds or last_slot > B * H * L * hd:
            raise ValueError("semantics='shipped' would read out of bounds at this batch/length; "
                             "use semantics='fixed'")

    def _inner_forward(self, x):
        """hdcmamba/model.py:331-384."""
        return self.out_proj(self._mix(x))

    def forward(self, x):
        """hdcmamba/model.py:386-394: left-pad to a chunk multiple, residual, strip the pad."""
        _require_cuda(x)
        B, L_in, _ = x.shape
        pad = (self.chunk_size - (L_in % self.chunk_size)) % self.chunk_size
        if pad > 0:
            x = F.pad(x, (0, 0, pad, 0))
        x = x.contiguous()
        if self.training:
            with torch.no_grad():
                self.gamma_buf.copy_(torch.exp(-F.softplus(self.decay_log)))
            res = checkpoint(self._inner_forward, x, use_reentrant=False)
            y = x + res
        elif torch.is_grad_enabled() and (x.requires_grad or self.out_proj.weight.requires_grad):
            y = x + self._inner_forward(x)
        else:
            # inference: residual add fused into the out_proj GEMM (beta = 1)
            comb = self._mix(x)
            y = torch.addmm(x.reshape(-1, self.d_model), comb.reshape(-1, comb.shape[-1]),
                            self.out_proj.weight.t()).reshape(x.shape)
        return y[:, pad:, :], None

    def _forward_inplace(self, x):
        """``forward(x)[0]`` for an internal activation that nothing else reads (a layer input
        inside HdcMamba9v3Model / the LM wrapper): in inference the layer's update is added to
        x in place, inside the out_proj GEMM (beta = 1, output = x), which skips the copy of
        x into a new output tensor that the out-of-place addmm makes first.  Falls back to
        ``forward`` when autograd needs the graph or x is padded / not contiguous."""
        if (self.training or (torch.is_grad_enabled() and (x.requires_grad or self.out_proj.weight.requires_grad))
                or x.shape[1] % self.chunk_size != 0 or not x.is_contiguous()):
            return self.forward(x)[0]
        _require_cuda(x)
        comb = self._mix(x)
        x2 = x.view(-1, self.d_model)
        torch.addmm(x2, comb.reshape(-1, comb.shape[-1]), self.out_proj.weight.t(), out=x2)
        return x


class HdcMamba9v3Model(nn.Module):
    """hdcmamba/model.py:396-404 (chunk size 256 as in the reference; num_slots unused there too)."""

    def __init__(self, d_model, n_layers, d_state, num_slots, num_heads=8, semantics="fixed"):
        super().__init__()
        self.layers = nn.ModuleList([HdcMamba9v3Block(d_model=d_model, d_state=d_state, num_heads=num_heads,
                                                      chunk_size=256, semantics=semantics)
                                     for _ in range(n_layers)])
        self.norm_final = nn.LayerNorm(d_model)

    def forward(self, x):
        return self._forward(x)

    def _forward(self, x, owns_input=False):
        """The layers after the first (and the first too when ``owns_input``: x is an
        internal activation of the caller) update the residual stream in place."""
        for i, layer in enumerate(self.layers):
            x = layer._forward_inplace(x) if (i > 0 or owns_input) else layer(x)[0]
        return final_layer_norm(self.norm_final, x)
