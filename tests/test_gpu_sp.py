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


def _worker(rank, world, port, q):
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
        sp = SequenceParallel()
        logits = sp.lm(lm, ids[:, rank * Ls:(rank + 1) * Ls].contiguous())
        out = torch.empty((world,) + tuple(logits.shape), device=dev, dtype=logits.dtype)
        dist.all_gather_into_tensor(out.reshape(-1), logits.contiguous().reshape(-1))
        torch.cuda.synchronize()
        if rank == 0:
            with torch.no_grad():
                ref = lm(ids)
            got = out.permute(1, 0, 2, 3).reshape(1, L, -1)
            err = float((got.float() - ref.float()).abs().max() / ref.float().abs().max())
            q.put((err, _lib.load().hdc_device_error(1)))
        dist.barrier()
    except Exception as e:
        q.put(RuntimeError(f"rank {rank}: {type(e).__name__}: {e}"))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sequence_parallel_two_gpus_matches_one_gpu():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = q.get(timeout=600)
    for p in procs:
        p.join(timeout=120)
    if isinstance(res, Exception):
        raise res
    err, dev_err = res
    assert dev_err == 0
    assert err < BF16_TOL, err
    assert all(p.exitcode == 0 for p in procs)
