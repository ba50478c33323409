"""Sequence parallelism for long prefill: one process per GPU.

Rank r of W holds the contiguous positions [r*L/W, (r+1)*L/W) of every sequence, so each
rank runs the whole layer on its own segment.  The layer has two cross-segment
dependencies, and each is exchanged once per layer with ``all_gather`` (NCCL over NVLink):

1. Halo.  The causal conv of LN+conv reads the three rows before the segment, i.e. the
   last three input rows of rank r-1 (rank 0 sees the reference's zero rows).
2. Carries, gathered in one call of one flat fp32 buffer that the kernels write directly:
   * SSM: every chunk's statistics (bf16-rounded last state and summed log decay).  Each
     rank then folds the same chunks in the same order as one GPU would, so its SSM prefix
     is bit-identical to the single-GPU one (``hdc_ssm_scan_out_blocked`` reads them in
     place from the gathered rank-major buffer).
   * Slot memory: each rank's local state (fp32 64x64 per head, from a zero start) and the
     product of its chunk decays.  Rank r folds those of ranks < r into its entering
     state, R_in(r) = D_{r-1} R_in(r-1) + A_{r-1}; this is the associativity of the
     per-chunk recurrence R <- gamma^C R + U (hdcmamba/model.py:272).  The fold runs inside
     the output kernel (``hdc_slot_gate_carry_fwd``), which also reuses the segment states
     that ``hdc_slot_state_fwd`` left in the workspace.

Two transports move the halo and the carries:

* ``"nccl"``: two ``all_gather`` calls per layer (every rank receives every rank's data).
* ``"p2p"``: each rank stores straight into the mailboxes of the ranks that need its data
  (carries to every higher rank, the halo to rank r+1) over NVLink, through CUDA-IPC-mapped
  buffers (``hdcmamba_b200.peer``), and raises a generation flag there; a rank waits
  (bounded) only for the flags of its senders.  The mailbox regions have the rank-major
  layout of the all-gather output, so the kernels read them the same way.

The kernels are those of the single-GPU Block (fixed semantics).  Only batch-independent
work crosses ranks, so batch sharding (config 4) needs no collective at all and uses the
plain module on each rank.
"""
import torch
import torch.distributed as dist
import torch.nn.functional as F

from . import ops


class CudaKernels:
    """The per-rank layer kernels (libhdcmamba_b200), looked up in ``ops`` at call time."""

    def __getattr__(self, name):
        return getattr(ops, name)


def _all_gather(t, group):
    """[W, *t.shape] stack of every rank's t (flat buffers, as every backend accepts)."""
    world = dist.get_world_size(group)
    flat = t.contiguous().reshape(-1)
    out = torch.empty(world * flat.numel(), device=t.device, dtype=t.dtype)
    dist.all_gather_into_tensor(out, flat, group=group)
    return out.reshape((world,) + tuple(t.shape))


class _Mailboxes:
    """Byte offsets of the per-layer regions in a rank's peer mailbox."""

    def __init__(self, n_layers, world, n_pad, halo_bytes):
        self.n_pad, self.world = n_pad, world
        self.carry_layer = world * n_pad * 4
        self.halo_bytes = (halo_bytes + 15) // 16 * 16
        self.halo0 = n_layers * self.carry_layer
        self.cflag0 = self.halo0 + n_layers * self.halo_bytes
        self.hflag0 = self.cflag0 + (n_layers * world * 4 + 15) // 16 * 16
        self.bar = self.hflag0 + (n_layers * 4 + 15) // 16 * 16
        self.total = self.bar + (world * 4 + 15) // 16 * 16

    def carries(self, layer, rank=0):
        return layer * self.carry_layer + rank * self.n_pad * 4

    def halo(self, layer):
        return self.halo0 + layer * self.halo_bytes

    def carry_flags(self, layer, rank=0):
        return self.cflag0 + (layer * self.world + rank) * 4

    def halo_flag(self, layer):
        return self.hflag0 + layer * 4


class SequenceParallel:
    """Runs HdcMamba blocks / LMs on this rank's segment of the sequence."""

    def __init__(self, group=None, kernels=None, transport="nccl", check_errors=False, ssm_placement="side"):
        """``check_errors``: after every forward, synchronise and raise HdcError if a bounded
        device wait (p2p halo / carry flags, the end-of-forward flag barrier, the kernels'
        mbarrier waits) gave up.  Off by default because it synchronises the stream (and
        cannot run inside CUDA-graph capture); ``check()`` does the same on demand.
        ``ssm_placement``: "side" runs the SSM kernels on a second stream next to the slot
        kernels, "main" after them on the current stream (see ``_pair``)."""
        if transport not in ("nccl", "p2p"):
            raise ValueError(f"transport {transport!r}: 'nccl' or 'p2p'")
        if ssm_placement not in ("side", "main"):
            raise ValueError(f"ssm_placement {ssm_placement!r}: 'side' or 'main'")
        self.ssm_placement = ssm_placement
        self.check_errors = check_errors
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.k = kernels if kernels is not None else CudaKernels()
        self.transport = transport
        self._mb = None       # PeerMailbox (p2p)
        self._lay = None      # _Mailboxes
        self._mb_key = None

    @staticmethod
    def _carry_len(B, N, ds, H):
        return (B * N * 2 * ds + B * H * 4096 + B * H + 3) // 4 * 4

    def _mailbox(self, n_layers, B, Ls, dm, ds, H, C, device):
        """The p2p mailbox for this shape (collective on first use and on a shape change)."""
        key = (n_layers, B, Ls, dm, ds, H, C)
        if self._mb_key != key:
            from .peer import PeerMailbox
            if self._mb is not None:
                self._mb.close()
            self._lay = _Mailboxes(n_layers, self.world, self._carry_len(B, Ls // C, ds, H), B * 3 * dm * 2)
            self._mb = PeerMailbox(self._lay.total, group=self.group, device=device)
            self._mb_key = key
        return self._mb, self._lay

    def check(self):
        """Synchronise this rank's device and raise HdcError if a bounded device wait timed
        out since the last check (the error word is cleared).  A timed-out p2p wait means
        the halo or carries of a peer never arrived, so the forward's output is invalid."""
        if not isinstance(self.k, CudaKernels):
            return
        from . import _lib
        torch.cuda.synchronize()
        code = _lib.load().hdc_device_error(1)
        if code != 0:
            raise _lib.HdcError(f"rank {self.rank}: a bounded device wait timed out (code {code}); "
                                "the sequence-parallel forward's output is invalid")

    def close(self):
        """Release the p2p mailbox (collective)."""
        if self._mb is not None:
            self._mb.close()
            self._mb = None
            self._mb_key = None

    def _final_norm(self, norm, h):
        """A final nn.LayerNorm: the affine row kernel for CUDA kernels, the module otherwise."""
        if h.is_cuda and isinstance(self.k, CudaKernels):
            from .model import final_layer_norm
            return final_layer_norm(norm, h)
        return norm(h)

    def _side(self, h):
        """The side stream for the SSM kernels (CUDA kernels only; None for CPU stand-ins)."""
        if not h.is_cuda or not isinstance(self.k, CudaKernels):
            return None
        from .model import _side_stream
        return _side_stream(h.device)

    def _begin(self, n_layers, h, blk):
        if self.transport == "p2p":
            B, Ls, dm = h.shape
            mb, _ = self._mailbox(n_layers, B, Ls, dm, blk.d_state, blk.num_heads, blk.chunk_size, h.device)
            mb.next_generation()

    def _end(self):
        if self.transport == "p2p":
            self._mb.barrier(self._lay.bar)

    def _finish(self):
        if self.check_errors:
            self.check()

    def _pair(self, side, cur, slot_fn, ssm_fn):
        """Run a slot kernel and the SSM kernel that does not depend on it.  "side": the SSM
        on the side stream, enqueued after the slot kernel so that the slot kernel's CTAs take
        their SMs first and the SSM fills the SMs they leave; "main": one after the other on
        the current stream.  Both are complete when this returns (in stream order)."""
        if side is None or self.ssm_placement == "main":
            slot_fn()
            ssm_fn()
            return
        side.wait_stream(cur)  # the SSM depends only on what precedes the slot kernel
        slot_fn()
        with torch.cuda.stream(side):
            ssm_fn()
        cur.wait_stream(side)

    def block(self, blk, h, layer=0, inplace=False):
        """One HdcMamba9v3Block on the local segment h [B, Ls, dm] (Ls a multiple of the
        chunk size; fixed semantics).  Returns the block output for the segment."""
        if blk.semantics != "fixed":
            raise ValueError("sequence parallelism needs semantics='fixed'")
        K = self.k
        B, Ls, dm = h.shape
        C, H, hd, ds = blk.chunk_size, blk.num_heads, blk.head_dim, blk.d_state
        if Ls % C != 0:
            raise ValueError(f"segment length {Ls} is not a multiple of the chunk size {C}")
        N = Ls // C
        h = h.contiguous()
        p2p = self.transport == "p2p"
        if p2p:
            if self._mb is None:
                raise RuntimeError("the p2p transport runs whole models: use SequenceParallel.model / .lm")
            mb, lay = self._mb, self._lay
        # (1) halo: the last three input rows of rank r-1
        side = self._side(h)
        halo_on_side = False
        if p2p:
            if self.rank < self.world - 1:
                last3 = h[:, -3:, :]
                if not last3.is_contiguous() or last3.data_ptr() % 16 or (last3.numel() * 2) % 16:
                    last3 = last3.contiguous()
                if side is not None:  # off this rank's critical path: its LN + conv does not wait for it
                    halo_on_side = True
                    side.wait_stream(torch.cuda.current_stream(h.device))
                    with torch.cuda.stream(side):
                        mb.put(last3, lay.halo(layer), lay.halo_flag(layer), [self.rank + 1], lane=1)
                    last3.record_stream(side)
                else:
                    mb.put(last3, lay.halo(layer), lay.halo_flag(layer), [self.rank + 1])
            halo = halo_flag = None
            if self.rank > 0:  # the LN+conv CTAs that read the halo wait for its flag themselves
                halo = mb.view(lay.halo(layer), (B, 3, dm), h.dtype)
                halo_flag = mb.flag_address(lay.halo_flag(layer))
        else:
            last3 = _all_gather(h[:, -3:, :], self.group)
            halo = last3[self.rank - 1] if self.rank > 0 else None
            halo_flag = None
        lnargs = (h, blk.norm.weight, blk.norm.bias, blk.conv1d.weight.squeeze(1), blk.conv1d.bias, blk.norm.eps)
        if halo_flag is not None:
            x_conv = K.ln_conv(*lnargs, halo=halo, halo_flag=halo_flag)
        else:
            x_conv = K.ln_conv(*lnargs, halo=halo)
        projs = F.linear(x_conv, blk.in_proj.weight, blk.in_proj.bias)
        so = 3 * ds
        q, k, v = projs[..., so:so + dm], projs[..., so + dm:so + 2 * dm], projs[..., so + 2 * dm:so + 3 * dm]
        gate = projs[..., so + 3 * dm:]
        gamma = blk.gamma_buf.to(h.dtype)
        # (2) carries, written by the kernels straight into one flat fp32 buffer per rank:
        #     [SSM chunk statistics B*N*2ds | slot state B*H*4096 | slot decay B*H | pad]
        n_st, n_sl, n_dc = B * N * 2 * ds, B * H * 4096, B * H
        n = self._carry_len(B, N, ds, H)
        if p2p:  # this rank's slot of the layer's carry region
            flat = mb.view(lay.carries(layer, self.rank), (n,), torch.float32)
        else:
            flat = torch.empty(n, device=h.device, dtype=torch.float32)
        ws = K.slot_workspace(B, Ls, H, hd, C, h.device)

        def ssm_stats():
            K.ssm_chunk_stats(projs, blk.A_log, ds, C, out=flat[:n_st].view(B, N, 2 * ds))

        def slot_state():
            K.slot_state(k, v, H, C, gamma=gamma, state_out=flat[n_st:n_st + n_sl].view(B, H, 64, 64),
                         decay_out=flat[n_st + n_sl:n_st + n_sl + n_dc].view(B, H), workspace=ws)
        cur = torch.cuda.current_stream(h.device) if side is not None else None
        self._pair(side, cur, slot_state, ssm_stats)  # the carries are complete after this
        exch = None
        if p2p:  # to every higher rank; from every lower rank
            if side is not None and self.rank + 1 < self.world:
                # no local kernel reads the peers' copies: the put runs on its own stream, off
                # this rank's critical path (joined at the end of the layer)
                from .model import _exchange_stream
                exch = _exchange_stream(h.device)
                exch.wait_stream(cur)
                with torch.cuda.stream(exch):
                    mb.put(flat, lay.carries(layer, self.rank), lay.carry_flags(layer, self.rank),
                           range(self.rank + 1, self.world), lane=2)
            else:
                mb.put(flat, lay.carries(layer, self.rank), lay.carry_flags(layer, self.rank),
                       range(self.rank + 1, self.world))
            # the consumers wait for the flags of every lower rank themselves (the SSM output
            # kernel after staging its inputs, the slot output kernel after its first chunk's P)
            fa, ga = mb.flag_address(lay.carry_flags(layer))
            wait = (fa, (1 << self.rank) - 1, ga) if self.rank > 0 else None
            g = mb.view(lay.carries(layer), (self.world * n,), torch.float32)  # [W * n], rank-major
        else:
            wait = None
            g = _all_gather(flat, self.group).reshape(-1)                     # [W * n], rank-major
        combined = torch.empty(B, Ls, ds + dm, device=h.device, dtype=h.dtype)
        # SSM: exclusive prefix over the chunks of ranks < r, then this rank's, in place (on
        # the side stream, next to the slot output kernel)
        wk = {"wait": wait} if wait is not None else {}

        def ssm_out():
            K.ssm_scan_out_blocked(projs, blk.A_log, g, N * 2 * ds, N, n, self.rank * N, ds, C,
                                   out=combined[..., :ds], **wk)

        def slot_out():  # fold the states of ranks < r in rank order, then the local segments
            K.slot_scan_gate_carry(q, k, v, H, C, gate, blk.group_norm.weight, blk.group_norm.bias,
                                   combined[..., ds:], (Ls * (ds + dm), hd, ds + dm), g[n_st:], g[n_st + n_sl:], n,
                                   self.rank, ws, gamma=gamma, **wk)
        self._pair(side, cur, slot_out, ssm_out)
        if halo_on_side:
            cur.wait_stream(side)  # the halo put joins the layer (already joined by a side pair)
        combined = K.row_layernorm(combined, 1e-5, out=combined)
        if inplace and h.is_cuda:
            # h is an internal activation: the update is added in place inside the GEMM (no
            # copy of h into a new output); the halo put that read h has joined above
            h2 = h.view(-1, dm)
            torch.addmm(h2, combined.reshape(-1, ds + dm), blk.out_proj.weight.t(), out=h2)
            out = h
        else:
            out = torch.addmm(h.reshape(-1, dm), combined.reshape(-1, ds + dm),
                              blk.out_proj.weight.t()).reshape(B, Ls, dm)
        if exch is not None:
            cur.wait_stream(exch)  # the carry put joins the layer
        return out

    def model(self, model, h):
        """HdcMamba9v3Model.forward on the local segment (hdcmamba/model.py:402-404)."""
        self._begin(len(model.layers), h, model.layers[0])
        for i, blk in enumerate(model.layers):
            h = self.block(blk, h, layer=i, inplace=i > 0)
        self._end()
        out = self._final_norm(model.norm_final, h)
        self._finish()
        return out

    def lm(self, lm, ids_local):
        """HdcMambaLM.forward (embedding -> backbone -> LayerNorm -> tied head) on the local
        segment of token ids [B, Ls]; returns the segment's logits [B, Ls, vocab]."""
        with torch.no_grad():
            h = lm.embedding(ids_local)  # a fresh activation: every layer updates it in place
            layers = list(lm.backbone.layers) if lm.use_model else list(lm.layers)
            self._begin(len(layers), h, layers[0])
            for i, blk in enumerate(layers):
                h = self.block(blk, h, layer=i, inplace=True)
            self._end()
            if lm.use_model:
                h = self._final_norm(lm.backbone.norm_final, h)
            self._finish()
            return F.linear(self._final_norm(lm.norm, h), lm.embedding.weight)
