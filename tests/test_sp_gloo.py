"""Sequence-parallel host logic on CPU: world-size-2 gloo ranks run SequenceParallel with
oracle-backed kernels (the halo exchange, the SSM prefix with n_prev, the fold of the slot
states) and the gathered result must equal the single-process oracle forward of the
whole sequence."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

import oracle as O

D_MODEL, D_STATE, HEADS, CHUNK, L, B = 64, 32, 1, 64, 512, 2


class OracleKernels:
    """CPU stand-ins with the hdcmamba_b200.ops signatures used by SequenceParallel."""

    @staticmethod
    def ln_conv(x, nw, nb, cw, cb, eps, halo=None):
        return O.ln_conv_fwd(x, nw, nb, cw, cb, eps, halo=halo)[0]

    @staticmethod
    def ssm_chunk_stats(projs, A_log, ds, C, out=None):
        _, _, last, cdec = O.ssm_chunk_states(projs, A_log.to(projs.dtype), ds, C)
        st = torch.cat([last, cdec], -1)
        if out is None:
            return st
        out.copy_(st)
        return out

    @staticmethod
    def ssm_scan_out_blocked(projs, A_log, stats, stats_sb, block_chunks, block_stride, n_prev, ds, C, out):
        """Reads chunk m of batch b at (m // block_chunks) * block_stride + b * stats_sb +
        (m % block_chunks) * 2ds, as hdc_ssm_scan_out_blocked does."""
        Bb, Ls, _ = projs.shape
        m_end = n_prev + Ls // C
        rows = []
        for b in range(Bb):
            per_b = []
            for m in range(m_end):
                blk, i = divmod(m, block_chunks)
                o = blk * block_stride + b * stats_sb + i * 2 * ds
                per_b.append(stats[o:o + 2 * ds])
            rows.append(torch.stack(per_b))
        stats_all = torch.stack(rows)
        y_intra, cum, _, _ = O.ssm_chunk_states(projs, A_log.to(projs.dtype), ds, C)
        G_all, _ = O.ssm_prefix(stats_all[..., :ds], stats_all[..., ds:])
        G = G_all[:, n_prev:]
        y = O.kbf16(y_intra + G[:, :, None] * torch.exp(cum)).reshape(Bb, Ls, ds)
        out.copy_(y.to(out.dtype))
        return out

    @staticmethod
    def _projs(q, k, v, gate, ds):
        Bb, Ls, _ = q.shape
        return torch.cat([torch.zeros(Bb, Ls, 3 * ds, dtype=q.dtype), q, k, v, gate], -1)

    @staticmethod
    def slot_workspace(B, L, H, hd, C, device):
        return None

    @staticmethod
    def slot_state(k, v, H, C, gamma, state_out, decay_out, workspace):
        Bb, Ls, dm = k.shape
        pj = torch.cat([k, k, v, torch.zeros_like(v)], -1)
        _, R = O.slot_fwd(pj, gamma, dm, H, C, 0, block_c=max(128, C), return_state=True)
        lg = torch.log(gamma.float())
        decay = torch.exp(C * lg).repeat(Bb).reshape(Bb, H) ** (Ls // C)
        state_out.copy_(R.reshape(Bb, H, 64, 64))
        decay_out.copy_(decay)
        return state_out, decay_out

    @staticmethod
    def slot_scan_gate_carry(q, k, v, H, C, gate, gn_w, gn_b, out, strides, prev_state, prev_decay, prev_stride,
                             n_prev, workspace, gamma):
        """Folds part s (state at prev_state[s*prev_stride:], decay at prev_decay[s*prev_stride:])
        into the entering state in order, as hdc_slot_gate_carry_fwd does."""
        Bb, Ls, dm = q.shape
        R_in = torch.zeros(Bb, H, 64, 64)
        for s in range(n_prev):
            o = s * prev_stride
            R_in = (prev_decay[o:o + Bb * H].view(Bb, H)[..., None, None] * R_in
                    + prev_state[o:o + Bb * H * 4096].view(Bb, H, 64, 64))
        pj = OracleKernels._projs(q, k, v, gate, D_STATE)
        y = O.slot_fwd(pj, gamma, dm, H, C, 3 * D_STATE, block_c=max(128, C), R0=R_in.reshape(Bb * H, 64, 64))
        comb = O.gnorm_gate_cat(y, torch.zeros(Bb, Ls, D_STATE, dtype=q.dtype), pj, gn_w, gn_b, D_STATE, H, C,
                                mode="fixed")
        out.copy_(comb[..., D_STATE:])
        return out

    @staticmethod
    def row_layernorm(x, eps, out):
        out.copy_(F.layer_norm(x.float(), (x.shape[-1],), eps=eps).to(x.dtype))
        return out


def _block_and_input():
    from hdcmamba_b200 import HdcMamba9v3Block
    torch.manual_seed(3)
    blk = HdcMamba9v3Block(d_model=D_MODEL, d_state=D_STATE, num_heads=HEADS, chunk_size=CHUNK).eval()
    x = torch.randn(B, L, D_MODEL)
    return blk, x


def _worker(rank, world, port, q):
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from hdcmamba_b200.sp import SequenceParallel
        blk, x = _block_and_input()
        Ls = L // world
        sp = SequenceParallel(kernels=OracleKernels())
        with torch.no_grad():
            y = sp.block(blk, x[:, rank * Ls:(rank + 1) * Ls])
            y = sp.block(blk, y)  # two layers: the second halo comes from the first layer's output
        out = [torch.empty_like(y) for _ in range(world)]
        dist.all_gather(out, y.contiguous())
        if rank == 0:
            q.put(torch.cat(out, 1))
    except Exception as e:  # report instead of leaving the test waiting
        q.put(RuntimeError(f"rank {rank}: {type(e).__name__}: {e}"))
        raise
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_sequence_parallel_matches_single_process(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    y_sp = q.get(timeout=300)
    if isinstance(y_sp, Exception):
        for p in procs:
            p.join(timeout=30)
        raise y_sp
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    blk, x = _block_and_input()
    sd = {k: v.clone() for k, v in blk.state_dict().items()}
    with torch.no_grad():
        ref = O.block_forward(sd, O.block_forward(sd, x, D_STATE, HEADS, CHUNK, mode="fixed"), D_STATE, HEADS,
                              CHUNK, mode="fixed")
    err = float((y_sp - ref).abs().max() / ref.abs().max())
    assert err < 5e-3, err
