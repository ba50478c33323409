"""Sequence parallelism on real GPUs (NCCL): the segments' outputs, gathered, equal the
single-GPU forward of the whole sequence.  Needs at least two visible GPUs."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
BF16_TOL = 2e-2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _model():
    from hdcmamba_b200.lm import HdcMambaLM, reinit_
    torch.manual_seed(0)
    return reinit_(HdcMambaLM(4096, 256, 2, 64, 4, use_model=True)).eval()


def _worker(rank, world, port, q, transport="nccl"):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        from hdcmamba_b200 import _lib
        from hdcmamba_b200.sp import SequenceParallel
        lm = _model().to(dev).bfloat16()
        L = 4096
        ids = torch.randint(0, 4096, (1, L), generator=torch.Generator().manual_seed(1)).to(dev)
        Ls = L // world
        sp = SequenceParallel(transport=transport, check_errors=True)  # raises on a timed-out wait
        logits = sp.lm(lm, ids[:, rank * Ls:(rank + 1) * Ls].contiguous())
        logits = sp.lm(lm, ids[:, rank * Ls:(rank + 1) * Ls].contiguous())  # a second generation
        out = torch.empty((world,) + tuple(logits.shape), device=dev, dtype=logits.dtype)
        dist.all_gather_into_tensor(out.reshape(-1), logits.contiguous().reshape(-1))
        torch.cuda.synchronize()
        # every rank reports its device error word: in p2p mode the higher ranks run the waits
        q.put(("dev", rank, _lib.load().hdc_device_error(1)))
        if rank == 0:
            with torch.no_grad():
                ref = lm(ids)
            got = out.permute(1, 0, 2, 3).reshape(1, L, -1)
            err = float((got.float() - ref.float()).abs().max() / ref.float().abs().max())
            q.put(("err", err))
        dist.barrier()
        sp.close()
    except Exception as e:
        q.put(RuntimeError(f"rank {rank}: {type(e).__name__}: {e}"))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("transport", ["nccl", "p2p"])
def test_sequence_parallel_two_gpus_matches_one_gpu(transport):
    """Both transports: NCCL all-gathers, and peer stores into IPC-mapped mailboxes with
    generation flags (two forwards, so the second generation is exercised too)."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, transport)) for r in range(world)]
    for p in procs:
        p.start()
    msgs = []
    for _ in range(world + 1):
        m = q.get(timeout=600)
        if isinstance(m, Exception):
            raise m
        msgs.append(m)
    for p in procs:
        p.join(timeout=120)
    dev = {m[1]: m[2] for m in msgs if m[0] == "dev"}
    assert dev == {r: 0 for r in range(world)}, dev
    err = [m[1] for m in msgs if m[0] == "err"][0]
    assert err < BF16_TOL, err
    assert all(p.exitcode == 0 for p in procs)


# ------------------------------------------------------------------ one GPU, ranks emulated
def _rel(a, b):
    a, b = a.detach().float().cpu(), b.detach().float().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-6))


@pytest.mark.parametrize("W,B,N,ds,C", [(4, 1, 8, 64, 256), (3, 2, 4, 32, 128)])
def test_ssm_scan_out_blocked_equals_contiguous_stats(W, B, N, ds, C):
    """hdc_ssm_scan_out_blocked over a rank-major buffer of per-part statistics gives the
    same bits as hdc_ssm_scan_out over the contiguous statistics of the whole sequence."""
    from hdcmamba_b200 import _lib, ops
    L = W * N * C
    g = torch.Generator().manual_seed(7 + W)
    projs = (0.7 * torch.randn(B, L, 3 * ds + 64, generator=g)).bfloat16().cuda()
    A_log = (0.3 * torch.randn(ds, generator=g)).cuda()
    y_ref = ops.ssm_scan(projs, A_log, ds, C)
    n = B * N * 2 * ds + 12  # a padded per-rank row, as the sequence-parallel buffer has
    gathered = torch.full((W * n,), float("nan"), device="cuda")
    Ls = N * C
    for r in range(W):
        ops.ssm_chunk_stats(projs[:, r * Ls:(r + 1) * Ls], A_log, ds, C,
                            out=gathered[r * n:r * n + B * N * 2 * ds].view(B, N, 2 * ds))
    for r in range(W):
        y = ops.ssm_scan_out_blocked(projs[:, r * Ls:(r + 1) * Ls], A_log, gathered, N * 2 * ds, N, n, r * N, ds, C)
        assert torch.equal(y, y_ref[:, r * Ls:(r + 1) * Ls]), r
    torch.cuda.synchronize()
    assert _lib.load().hdc_device_error(1) == 0


@pytest.mark.parametrize("W,B,L,H,C", [(4, 1, 4096, 4, 256), (2, 2, 1024, 4, 64), (3, 1, 3 * 512, 2, 128)])
def test_slot_gate_carry_matches_whole_sequence(W, B, L, H, C):
    """Per-part hdc_slot_state_fwd into a rank-major buffer, then hdc_slot_gate_carry_fwd
    for each part, equals hdc_slot_gate_fwd over the whole sequence."""
    from hdcmamba_b200 import _lib, ops
    dm, ds = 64 * H, 64
    hd = dm // H
    g = torch.Generator().manual_seed(90 + W)
    projs = (0.6 * torch.randn(B, L, 4 * dm, generator=g)).bfloat16().cuda()
    q, k, v, gate = (projs[..., i * dm:(i + 1) * dm] for i in range(4))
    gamma = torch.exp(-torch.nn.functional.softplus(torch.randn(H, generator=g) - 3.0)).bfloat16().cuda()
    gw = (1 + 0.2 * torch.randn(dm, generator=g)).bfloat16().cuda()
    gb = (0.2 * torch.randn(dm, generator=g)).bfloat16().cuda()
    strides = lambda Lx: (Lx * dm, hd, dm)  # noqa: E731
    ref = torch.empty(B, L, dm, device="cuda", dtype=torch.bfloat16)
    ops.slot_scan_gate(q, k, v, H, C, gate, gw, gb, ref, strides(L), gamma=gamma)
    Ls = L // W
    n_sl, n_dc = B * H * 4096, B * H
    n = (n_sl + n_dc + 4 + 3) // 4 * 4  # parts 16-byte aligned, as the entry point requires
    gathered = torch.full((W * n,), float("nan"), device="cuda")
    wss = []
    for r in range(W):
        sl = slice(r * Ls, (r + 1) * Ls)
        ws = ops.slot_workspace(B, Ls, H, hd, C, "cuda")
        ops.slot_state(k[:, sl], v[:, sl], H, C, gamma=gamma, state_out=gathered[r * n:r * n + n_sl].view(B, H, 64, 64),
                       decay_out=gathered[r * n + n_sl:r * n + n_sl + n_dc].view(B, H), workspace=ws)
        wss.append(ws)
    out = torch.empty(B, L, dm, device="cuda", dtype=torch.bfloat16)
    for r in range(W):
        sl = slice(r * Ls, (r + 1) * Ls)
        # out[:, sl] is a view into the whole [B, L, dm] output: batch stride L*dm
        ops.slot_scan_gate_carry(q[:, sl], k[:, sl], v[:, sl], H, C, gate[:, sl], gw, gb, out[:, sl], strides(L),
                                 gathered, gathered[n_sl:], n, r, wss[r], gamma=gamma)
    torch.cuda.synchronize()
    assert _lib.load().hdc_device_error(1) == 0
    assert _rel(out, ref) < BF16_TOL, _rel(out, ref)
