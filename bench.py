"""Benchmark: HdcMamba-9v3 bf16 prefill tokens/s at L=32768.

Workload (config 5): 12 x HdcMamba9v3Block (d_model 768, 12 heads, d_state 64,
chunk 256) inside HdcMamba9v3Model, token embedding and tied lm_head over
vocab 50304; seeded synthetic weights (seed 0, N(0, 0.02)); B=1 x L=32768
uniform token ids; every step computes the logits of all 32768 positions.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One JSON line on rank 0.  ``value`` is device-timed throughput with the ids
already resident; ``e2e`` runs the same forward through the public module
call with the ids copied from pinned host memory and the last position's
logits copied back each step.  ``roofline`` covers the dominant custom kernel
(the slot-memory scan), timed with CUDA events on its launch stream during
the timed steps.  ``cpu_baseline`` times the CPU oracle port on the host cores
on a bounded sample (rank 0, N=1 only).  ``--impl reference`` times the CPU
port of the reference forward (the reference itself is Python + Triton with
no CPU path but the Triton interpreter) on the same config.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

MEASURED_PEAKS = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK_HBM_GBS = 6650.0
METRIC = "prefill tokens/sec at L=32768"
# DRAM bytes (read + write) of one config-5 slot op (pass A + pass B) from an ncu --set full
# capture of `bench.py --workload c5slot`
SLOT_TRAFFIC_BYTES = 97.19e6 + 3.49e6 + 205.99e6 + 28.82e6


def peaks():
    try:
        with open(MEASURED_PEAKS) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region."""
    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.proc = None
        self.lines = []
        self.marks = []
        try:
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            self.gid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
        except Exception:
            self.gid = None

    def start(self, ready_timeout=5.0):
        """Start sampling every 50 ms and wait (bounded) for the first sample, so that a
        short timed region that follows is covered."""
        cmd = ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms", "50"]
        if self.gid:
            cmd += ["-i", self.gid]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
            return
        t_end = time.monotonic() + ready_timeout
        while not self.lines and time.monotonic() < t_end:
            time.sleep(0.01)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.monotonic(), line.strip()))

    def mark(self):
        """Host time of a timed-region boundary (taken after a device synchronize)."""
        self.marks.append(time.monotonic())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.t.join(timeout=2)
        window = "timed region"
        lines = [ln for t, ln in self.lines if len(self.marks) >= 2 and self.marks[0] <= t <= self.marks[1] + 0.06]
        if not lines:  # timed region shorter than the sampling period: warm-up and timed steps
            window = "warm-up + timed steps (timed region shorter than the 50 ms sampling period)"
            lines = [ln for t, ln in self.lines if not self.marks or t <= self.marks[-1] + 0.06]
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[0]))
                mx.append(float(f[1]))
            except ValueError:
                continue
            for n, v in zip(names, f[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm), "window": window}


def _time_cuda(fn, iters, warmup=3):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def kernel_c2(dev, iters, hbm):
    """LayerNorm + causal conv1d (width 4) + SiLU, x bf16 [8, 8192, 2048]
    (268 MB in, 268 MB out: larger than L2, so no flush is needed)."""
    from hdcmamba_b200 import ops
    B, L, D = 8, 8192, 2048
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(B, L, D, device=dev, generator=g).bfloat16()
    cw = (0.02 * torch.randn(D, 4, device=dev, generator=g)).bfloat16()
    nw, nb, cb = (torch.ones(D, device=dev).bfloat16(), torch.zeros(D, device=dev).bfloat16(),
                  torch.zeros(D, device=dev).bfloat16())
    ms = _time_cuda(lambda: ops.ln_conv(x, nw, nb, cw, cb, 1e-5, act="silu"), iters)
    nbytes = 2 * B * L * D * 2
    return {"workload": "c2: ln_conv+silu bf16 [8,8192,2048]", "ms_per_launch": ms,
            "algorithmic_bytes": nbytes, "achieved_gbs": nbytes / ms / 1e6, "frac": nbytes / ms / 1e6 / hbm}


def kernel_c2bwd(dev, iters, hbm):
    """Backward of config 2's LN + conv (the reference's FusedNormConv1dFunction.backward
    formulas, hdc_ln_conv_bwd): grad_out and x read, dx written, bf16 [8, 8192, 2048]."""
    from hdcmamba_b200 import ops
    B, L, D = 8, 8192, 2048
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(B, L, D, device=dev, generator=g).bfloat16()
    go = torch.randn(B, L, D, device=dev, generator=g).bfloat16()
    cw = (0.02 * torch.randn(D, 4, device=dev, generator=g)).bfloat16()
    nw, nb, cb = (torch.ones(D, device=dev).bfloat16(), torch.zeros(D, device=dev).bfloat16(),
                  torch.zeros(D, device=dev).bfloat16())
    _, mean, rstd = ops.ln_conv(x, nw, nb, cw, cb, 1e-5, stats=True)
    ms = _time_cuda(lambda: ops.ln_conv_bwd(go, x, mean, rstd, nw, cw), iters)
    nbytes = 3 * B * L * D * 2
    return {"workload": "c2bwd: ln_conv backward bf16 [8,8192,2048]", "ms_per_launch": ms,
            "algorithmic_bytes": nbytes, "achieved_gbs": nbytes / ms / 1e6, "frac": nbytes / ms / 1e6 / hbm}


def decode_c5(dev, batch, steps=64):
    """Recurrent decode of the config-5 model (hdcmamba_b200.decode): a 256-token prompt,
    then ``steps`` single-token steps per sequence replayed as one CUDA graph; tokens/s =
    batch / step time."""
    from hdcmamba_b200.decode import GraphedDecode, prefill
    from hdcmamba_b200.lm import CONFIGS, build_lm
    cfg = CONFIGS["c5"]
    lm = build_lm(cfg).to(dev).bfloat16()
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, cfg.vocab, (batch, 256 + steps + 3), generator=g).to(dev)
    _, st = prefill(lm, ids[:, :256])
    gd = GraphedDecode(lm, st, ids[:, 256])
    for t in range(3):
        gd(ids[:, 256 + t])
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for t in range(steps):
        gd(ids[:, 259 + t])
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    del gd, st, lm
    return {"workload": f"decode c5 (12x d768, 256-token prompt), batch {batch}", "ms_per_step": ms,
            "tokens_per_s": batch / (ms * 1e-3)}


def layer_c5(dev, hbm, seq_len=32768, iters=10):
    """Per-op device time of one config-5 layer (B1, d768, H12, ds64, C256) at ``seq_len``:
    each op replayed as a CUDA graph between CUDA events, after a read-only pass over 512 MB
    that leaves L2 clean; ``floor_us`` is the same measurement of an empty op (graph launch
    and event overhead, included in every figure)."""
    import statistics as st_
    import torch.nn.functional as F
    from hdcmamba_b200 import ops
    from hdcmamba_b200.lm import CONFIGS, build_lm
    cfg = CONFIGS["c5"]
    torch.manual_seed(0)
    blk = build_lm(cfg).backbone.layers[0].to(dev).bfloat16()
    flush = torch.ones(256 << 20, dtype=torch.float16, device=dev)
    sink = torch.empty((), dtype=torch.float16, device=dev)

    def timed(fn):
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            fn()
        torch.cuda.current_stream(dev).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        ev = []
        for _ in range(iters + 1):
            torch.amax(flush, dim=0, out=sink)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            g.replay()
            b.record()
            ev.append((a, b))
        torch.cuda.synchronize()
        return round(st_.mean(a.elapsed_time(b) for a, b in ev[1:]) * 1000, 1)

    B, L, dm, ds, H, C = 1, seq_len, cfg.d_model, cfg.d_state, cfg.num_heads, cfg.chunk_size
    hd = dm // H
    h = torch.randn(B, L, dm, device=dev).bfloat16()
    res = {"workload": f"c5 layer ops, B1 L{L} d{dm}", "unit": "us per op (includes floor_us)"}
    with torch.no_grad():
        lnargs = (blk.norm.weight, blk.norm.bias, blk.conv1d.weight.squeeze(1), blk.conv1d.bias, 1e-5)
        xc = ops.ln_conv(h, *lnargs)
        projs = F.linear(xc, blk.in_proj.weight, blk.in_proj.bias)
        so = 3 * ds
        q, k, v = projs[..., so:so + dm], projs[..., so + dm:so + 2 * dm], projs[..., so + 2 * dm:so + 3 * dm]
        gate = projs[..., so + 3 * dm:]
        gamma = blk.gamma_buf.to(h.dtype)
        stats = ops.ssm_chunk_stats(projs, blk.A_log, ds, C)
        comb = torch.empty(B, L, ds + dm, device=dev, dtype=h.dtype)
        res["floor_us"] = timed(lambda: sink.add_(0))
        res["ln_conv"] = timed(lambda: ops.ln_conv(h, *lnargs))
        res["in_proj"] = timed(lambda: F.linear(xc, blk.in_proj.weight, blk.in_proj.bias))
        res["ssm_chunk_stats"] = timed(lambda: ops.ssm_chunk_stats(projs, blk.A_log, ds, C))
        res["ssm_scan_out"] = timed(lambda: ops.ssm_scan_out(projs, blk.A_log, stats, 0, ds, C, out=comb[..., :ds]))
        res["slot_scan_gate"] = timed(lambda: ops.slot_scan_gate(q, k, v, H, C, gate, blk.group_norm.weight,
                                                                 blk.group_norm.bias, comb[..., ds:],
                                                                 (L * (ds + dm), hd, ds + dm), gamma=gamma))
        res["row_layernorm"] = timed(lambda: ops.row_layernorm(comb, 1e-5, out=comb))
        res["out_proj"] = timed(lambda: torch.addmm(h.reshape(-1, dm), comb.reshape(-1, ds + dm),
                                                    blk.out_proj.weight.t()))
    del flush
    return res


def kernel_c3(dev, iters, hbm):
    """slot scan with per-step decay, q/k/v bf16 [4, 32768, 16, 64],
    a = sigmoid(N(0,1)) fp32, chunk 64, zero initial state, final state returned."""
    from hdcmamba_b200 import ops
    B, L, H, hd, C = 4, 32768, 16, 64, 64
    g = torch.Generator(device=dev).manual_seed(0)
    q, k, v = (torch.randn(B, L, H * hd, device=dev, generator=g).bfloat16() for _ in range(3))
    log_a = torch.nn.functional.logsigmoid(torch.randn(B, L, H, device=dev, generator=g))
    y = torch.empty(B, L, H, hd, device=dev, dtype=torch.bfloat16)
    ms = _time_cuda(lambda: ops.slot_scan(q, k, v, H, C, log_a=log_a, y=y, y_strides=(L * H * hd, hd, H * hd),
                                          return_state=True), iters)
    nbytes = 4 * B * L * H * hd * 2 + B * L * H * 4 + B * H * 64 * 64 * 4
    flops = B * L * H * (4 * C * hd + 4 * hd * hd)
    return {"workload": "c3: slot scan per-step decay bf16 [4,32768,16,64] C64", "ms_per_launch": ms,
            "algorithmic_bytes": nbytes, "achieved_gbs": nbytes / ms / 1e6, "frac": nbytes / ms / 1e6 / hbm,
            "algorithmic_flop": flops, "achieved_tflops": flops / ms / 1e9}


def kernel_c5slot(dev, iters, hbm):
    """One layer's slot scan with the fused GroupNorm * sigmoid(gate) epilogue at config-5
    shapes (projs [1, 32768, 3264] bf16, d_model 768, 12 heads, chunk 256)."""
    from hdcmamba_b200 import ops
    B, L, ds, dm, H, C = 1, 32768, 64, 768, 12, 256
    hd, P = dm // H, 3 * ds + 4 * dm
    g = torch.Generator(device=dev).manual_seed(0)
    projs = torch.randn(B, L, P, device=dev, generator=g).bfloat16()
    gamma = torch.full((H,), 0.952, device=dev).bfloat16()
    gw, gb = torch.ones(dm, device=dev).bfloat16(), torch.zeros(dm, device=dev).bfloat16()
    comb = torch.empty(B, L, ds + dm, device=dev, dtype=torch.bfloat16)
    so = 3 * ds
    q, k, v, gt = (projs[..., so + i * dm:so + (i + 1) * dm] for i in range(4))
    ms = _time_cuda(lambda: ops.slot_scan_gate(q, k, v, H, C, gt, gw, gb, comb[..., ds:],
                                               (L * (ds + dm), hd, ds + dm), gamma=gamma), iters)
    nbytes = 5 * B * L * dm * 2
    return {"workload": "c5slot: slot scan + GN*sigmoid(gate) bf16, L32768 d768 H12 C256", "ms_per_launch": ms,
            "algorithmic_bytes": nbytes, "achieved_gbs": nbytes / ms / 1e6, "frac": nbytes / ms / 1e6 / hbm}


class _AttnBlock(torch.nn.Module):
    """Decoder block of the comparison Transformer in the reference benchmark harness
    (benchmark.py:52-85): pre-LN causal self-attention through
    F.scaled_dot_product_attention (flash / cuDNN backends), then a pre-LN 4x GELU MLP."""

    def __init__(self, d, heads):
        super().__init__()
        nn = torch.nn
        self.heads = heads
        self.ln1, self.ln2 = nn.LayerNorm(d), nn.LayerNorm(d)
        self.qkv, self.proj = nn.Linear(d, 3 * d), nn.Linear(d, d)
        self.mlp = nn.Sequential(nn.Linear(d, 4 * d), nn.GELU(), nn.Linear(4 * d, d))

    def forward(self, x):
        B, L, d = x.shape
        q, k, v = self.qkv(self.ln1(x)).view(B, L, 3, self.heads, d // self.heads).permute(2, 0, 3, 1, 4)
        a = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True)
        x = x + self.proj(a.transpose(1, 2).reshape(B, L, d))
        return x + self.mlp(self.ln2(x))


class _AttnModel(torch.nn.Module):
    def __init__(self, d=512, heads=8, layers=6):
        super().__init__()
        self.blocks = torch.nn.ModuleList([_AttnBlock(d, heads) for _ in range(layers)])
        self.ln = torch.nn.LayerNorm(d)

    def forward(self, x):
        for b in self.blocks:
            x = b(x)
        return self.ln(x)


def harness(dev, runs=20, warmup=5):
    """The reference's benchmark harness (benchmark.py:215-362), B200 edition: forward
    throughput of HdcMamba9v3Model (6 x d768, d_state 128, 12 heads, the harness's shapes)
    against a 6 x d512, 8-head Transformer on torch's scaled_dot_product_attention, bf16,
    inputs x ~ N(0,1) of the models' widths.  Shapes (B, L) follow the harness: 4x1024, 4x4096,
    the "8K" row (HdcMamba 2x4096 as the harness builds it, benchmark.py:330; Transformer
    2x8192), 1x16384, 1x32768.  Each model is timed eagerly (CUDA events around ``runs``
    forwards after ``warmup``); the HdcMamba model also as one CUDA-graph replay per forward."""
    from hdcmamba_b200 import HdcMamba9v3Model
    from hdcmamba_b200.graph import GraphedForward
    torch.manual_seed(0)
    hdc = HdcMamba9v3Model(d_model=768, n_layers=6, d_state=128, num_slots=32, num_heads=12).to(dev).bfloat16().eval()
    tf = _AttnModel().to(dev).bfloat16().eval()
    rows = [("1K", (4, 1024), (4, 1024)), ("4K", (4, 4096), (4, 4096)), ("8K", (2, 4096), (2, 8192)),
            ("16K", (1, 16384), (1, 16384)), ("32K", (1, 32768), (1, 32768))]

    def timed(fn):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(runs):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / runs

    out = []
    with torch.no_grad():
        for label, (hb, hl), (tb, tlen) in rows:
            g = torch.Generator(device=dev).manual_seed(1)
            xh = torch.randn(hb, hl, 768, device=dev, generator=g).bfloat16()
            xt = torch.randn(tb, tlen, 512, device=dev, generator=g).bfloat16()
            ms_h = timed(lambda: hdc(xh))
            gf = GraphedForward(hdc, xh)
            ms_hg = timed(gf.replay)
            del gf
            ms_t = timed(lambda: tf(xt))
            r = {"row": label, "hdcmamba": {"B": hb, "L": hl, "ms": ms_h, "tok_s": hb * hl / ms_h * 1e3,
                                             "ms_graph": ms_hg, "tok_s_graph": hb * hl / ms_hg * 1e3},
                 "transformer_sdpa": {"B": tb, "L": tlen, "ms": ms_t, "tok_s": tb * tlen / ms_t * 1e3}}
            r["speedup_tok_s"] = r["hdcmamba"]["tok_s"] / r["transformer_sdpa"]["tok_s"]
            out.append(r)
            del xh, xt
            torch.cuda.empty_cache()
    return {"workload": "harness: HdcMamba9v3Model 6x d768 ds128 H12 vs Transformer 6x d512 H8 (SDPA), "
                        "forward, bf16, x ~ N(0,1)", "reference_claim": "3.37x tokens/s at L=32768 (README.md:12)",
            "rows": out}


def cpu_oracle_tokens_per_s(cfg, tokens, repeats=2):
    """CPU oracle port (oracle/restate.py, fp32 math with the bf16 rounding points) on
    the first ``tokens`` ids, all layers and the full vocab head."""
    import oracle as O
    from hdcmamba_b200.lm import build_lm, synthetic_ids
    torch.set_num_threads(os.cpu_count() or 1)
    sd = {k: v.bfloat16() for k, v in build_lm(cfg).state_dict().items()}
    ids = synthetic_ids(cfg, seq_len=tokens)
    times = []
    for _ in range(repeats):
        t = time.perf_counter()
        with torch.no_grad():
            O.lm_forward(sd, ids, cfg.n_layers, cfg.d_state, cfg.num_heads, cfg.chunk_size, mode="fixed",
                         dtype=torch.bfloat16, use_model_norm=cfg.use_model)
        times.append(time.perf_counter() - t)
    return tokens / min(times), torch.get_num_threads()


def run_reference(args, cfg, rank):
    if rank != 0:
        return
    tokens = args.ref_tokens
    import oracle as O
    from hdcmamba_b200.lm import build_lm, synthetic_ids
    torch.set_num_threads(os.cpu_count() or 1)
    sd = {k: v.bfloat16() for k, v in build_lm(cfg).state_dict().items()}
    ids = synthetic_ids(cfg, seq_len=tokens)

    def step():
        with torch.no_grad():
            O.lm_forward(sd, ids, cfg.n_layers, cfg.d_state, cfg.num_heads, cfg.chunk_size, mode="fixed",
                         dtype=torch.bfloat16, use_model_norm=cfg.use_model)

    for _ in range(args.warmup):
        step()
    t = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t) / args.steps
    v = tokens / dt
    sample = f"first {tokens} of {cfg.seq_len} tokens per step, all {cfg.n_layers} layers + vocab-{cfg.vocab} head"
    print(json.dumps({
        "metric": METRIC if cfg.seq_len == 32768 else f"prefill tokens/sec at L={cfg.seq_len}",
        "value": v, "unit": "tokens/s", "impl": "reference", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"{cfg.name}: {cfg.n_layers}x d{cfg.d_model} H{cfg.num_heads} ds{cfg.d_state} "
                               f"C{cfg.chunk_size}, vocab {cfg.vocab}, B{cfg.batch} L{cfg.seq_len}",
                   "global_batch": cfg.batch, "seq_len": cfg.seq_len, "parallelism": "cpu"},
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
                         "sample": sample},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "CPU port of the reference forward (oracle/restate.py); the reference has no CPU path "
                "besides the Triton interpreter",
    }), flush=True)


def run_timeline(args, cfg, world, rank, local):
    """Per-op device timeline of the LM forward (hdcmamba_b200.trace), CUDA-graph replay.
    One GPU: the config's model at L = 4096 (a sequence-parallel rank's length at 8 GPUs)
    and at the config's length; under torchrun: the sequence-parallel forward, one line
    per rank (rank 0 prints them all)."""
    import dataclasses
    from hdcmamba_b200.lm import build_lm, synthetic_ids
    from hdcmamba_b200.trace import trace
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    lm = build_lm(cfg).to(dev).bfloat16()
    if world == 1:
        for L in (4096, cfg.seq_len):
            ids = synthetic_ids(dataclasses.replace(cfg, seq_len=L)).to(dev)

            def fwd():
                with torch.no_grad():
                    return lm(ids)
            for _ in range(args.warmup):
                fwd()
            torch.cuda.synchronize()
            r = trace(fwd, dev, replays=args.steps)
            print(json.dumps({"workload": f"timeline {cfg.name} B{cfg.batch} L{L}, 1 GPU", "rank": 0, **r}), flush=True)
        return
    import torch.distributed as dist
    from datetime import timedelta
    from hdcmamba_b200.sp import SequenceParallel
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    sp = SequenceParallel(transport=args.sp_transport, ssm_placement=args.sp_ssm)
    Ls = cfg.seq_len // world
    ids = synthetic_ids(cfg)[:, rank * Ls:(rank + 1) * Ls].contiguous().to(dev)

    def fwd():
        return sp.lm(lm, ids)
    for _ in range(args.warmup):
        fwd()
    torch.cuda.synchronize()
    dist.barrier()
    r = trace(fwd, dev, replays=args.steps, before_replay=dist.barrier)
    r = {"workload": f"timeline {cfg.name} B{cfg.batch} L{cfg.seq_len}, sp{world} ({args.sp_transport})",
         "rank": rank, **r}
    rows = [None] * world
    dist.all_gather_object(rows, r)
    if rank == 0:
        for row in rows:
            print(json.dumps(row), flush=True)
    sp.close()
    torch.cuda.synchronize()
    dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c5")
    ap.add_argument("--sp-transport", default="p2p", choices=["p2p", "nccl"],
                    help="sequence parallelism: peer stores into IPC-mapped mailboxes, or NCCL all-gathers")
    ap.add_argument("--sp-ssm", default="side", choices=["side", "main"],
                    help="sequence parallelism: the SSM kernels on a second stream next to the slot kernels, "
                         "or after them on the main stream")
    ap.add_argument("--parallel", default="auto", choices=["auto", "sp", "batch"],
                    help="N > 1: batch = split the global batch over the ranks (no collective, config 4); "
                         "sp = split the sequence (config 5); auto = batch when the batch divides evenly")
    ap.add_argument("--ref-tokens", type=int, default=4096)
    ap.add_argument("--cpu-tokens", type=int, default=4096)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-kernels", action="store_true", help="skip the config-2/3 kernel lines")
    ap.add_argument("--eager", action="store_true", help="launch eagerly instead of replaying a CUDA graph")
    ap.add_argument("--workload", default=None,
                    choices=["c2", "c2bwd", "c3", "c5slot", "c5layer", "harness", "timeline"],
                    help="time one kernel workload alone (for profiling) and print its line; timeline: "
                         "per-op device times of the forward (hdcmamba_b200.trace), also under torchrun")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    from hdcmamba_b200.lm import CONFIGS
    cfg = CONFIGS[args.config]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        return run_reference(args, cfg, rank)
    if args.workload == "timeline":
        return run_timeline(args, cfg, world, rank, local)
    if args.workload:
        torch.cuda.set_device(local)
        dev = torch.device("cuda", local)
        if args.workload == "harness":
            print(json.dumps(harness(dev)), flush=True)
            return
        if args.workload == "c5layer":
            for L in (4096, 32768):  # a sequence-parallel rank's length at 8 GPUs, and one GPU's
                print(json.dumps(layer_c5(dev, peaks()[0], seq_len=L, iters=args.steps)), flush=True)
            return
        fn = {"c2": kernel_c2, "c2bwd": kernel_c2bwd, "c3": kernel_c3, "c5slot": kernel_c5slot}[args.workload]
        print(json.dumps(fn(dev, args.steps, peaks()[0])), flush=True)
        return

    import torch.distributed as dist
    from datetime import timedelta
    from hdcmamba_b200 import _lib, ops
    from hdcmamba_b200.lm import build_lm, synthetic_ids

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    lm = build_lm(cfg).to(dev).bfloat16()
    mode = "single"
    if world > 1:
        mode = args.parallel
        if mode == "auto":
            mode = "batch" if cfg.batch % world == 0 else "sp"
        if mode == "batch" and cfg.batch % world != 0:
            raise SystemExit(f"batch {cfg.batch} does not split over {world} ranks")
    if mode == "batch":
        # batch sharding: rank r runs samples [r*B/W, (r+1)*B/W) through the whole model, no
        # collective in the forward
        Bs = cfg.batch // world
        ids_host = synthetic_ids(cfg)[rank * Bs:(rank + 1) * Bs].contiguous().pin_memory()

        def forward(x):
            with torch.no_grad():
                return lm(x)
    elif mode == "sp":
        # sequence parallel: rank r runs positions [r*L/W, (r+1)*L/W) of the same sequence
        from hdcmamba_b200.sp import SequenceParallel
        if cfg.seq_len % (world * cfg.chunk_size) != 0:
            raise SystemExit(f"L={cfg.seq_len} does not split into {world} chunk-aligned segments")
        sp = SequenceParallel(transport=args.sp_transport, ssm_placement=args.sp_ssm)
        Ls = cfg.seq_len // world
        ids_host = synthetic_ids(cfg)[:, rank * Ls:(rank + 1) * Ls].contiguous().pin_memory()

        def forward(x):
            return sp.lm(lm, x)
    else:
        ids_host = synthetic_ids(cfg).pin_memory()

        def forward(x):
            with torch.no_grad():
                return lm(x)
    ids = ids_host.to(dev)
    tokens_per_rank = ids.numel()

    graphed = None
    if args.eager:
        def step():
            return forward(ids)

        def step_host():
            return forward(ids_host.to(dev, non_blocking=True))
    else:
        from hdcmamba_b200.graph import GraphedForward
        graphed = GraphedForward(forward, ids)
        ids = graphed.static_in

        def step():
            return graphed.replay()

        def step_host():
            return graphed(ids_host)  # pinned host -> static input (H2D), then replay

    # the slot op (roofline kernel) of one layer: its arguments are captured from an eager
    # forward; sequence parallel runs slot_state + slot_scan_gate_carry for one layer's op
    slot_names = ("slot_scan", "slot_scan_gate", "slot_state", "slot_scan_gate_carry")
    originals = {name: getattr(ops, name) for name in slot_names}
    slot_calls = []

    def grab(fn, name):
        def wrapper(*a, **k):
            slot_calls.append((fn, a, k))
            return fn(*a, **k)
        return wrapper

    sampler = ClockSampler(dev)
    sampler.start()  # samples the warm-up too, for timed regions shorter than its period
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler.mark()
    n0 = _lib.launch_count()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    sampler.mark()
    launches = _lib.launch_count() - n0
    if not args.eager:
        launches = graphed.launches_per_replay * args.steps  # replays issue the captured launches
    clocks = sampler.stop()
    if world > 1:
        dist.barrier()
    ms = t0.elapsed_time(t1) / args.steps
    # per-launch time of the slot op: one layer's slot calls (arguments captured from an
    # eager forward) replayed as a CUDA graph between CUDA events on the replay stream, each
    # replay preceded by a 512 MB write that evicts L2
    for name in slot_names:
        setattr(ops, name, grab(originals[name], name))
    with torch.no_grad():
        forward(ids)
    for name in slot_names:
        setattr(ops, name, originals[name])
    per_layer = 2 if mode == "sp" else 1
    layer_calls = slot_calls[:per_layer]
    slot_per_step = len(slot_calls) / per_layer

    def slot_layer():
        for fn, a, k in layer_calls:
            fn(*a, **k)

    slot_graph = torch.cuda.CUDAGraph()
    with torch.no_grad(), torch.cuda.graph(slot_graph):
        slot_layer()
    flush = torch.empty(512 << 20, dtype=torch.uint8, device=dev)
    durations = []
    for it in range(11):
        flush.zero_()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        slot_graph.replay()
        s1.record()
        durations.append((s0, s1))
    torch.cuda.synchronize()
    slot_ms = statistics.mean(s0.elapsed_time(s1) for s0, s1 in durations[1:])
    del flush, slot_calls, layer_calls, slot_graph

    # end to end through the public call: pinned host ids -> device, logits[:, -1] -> host
    out_host = torch.empty(ids_host.shape[0], cfg.vocab, dtype=torch.bfloat16).pin_memory()
    logits = step_host()  # one untimed step through the host path (every rank: same replay count)
    out_host.copy_(logits[:, -1], non_blocking=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()  # the ranks start the timed region together, as for the device-timed value
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        logits = step_host()
        out_host.copy_(logits[:, -1], non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps

    stats = torch.tensor([ms, e2e_ms, slot_ms], device=dev)
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    ms, e2e_ms, slot_ms = [float(v) for v in stats.tolist()]

    if rank == 0:
        hbm, src = peaks()
        # q, k, v and gate read, the gated slot half of `combined` written (bf16)
        slot_bytes = 5 * tokens_per_rank * cfg.d_model * 2
        achieved = slot_bytes / (slot_ms * 1e-3) / 1e9
        line = {
            "metric": METRIC if cfg.seq_len == 32768 else f"prefill tokens/sec at L={cfg.seq_len}",
            "value": world * tokens_per_rank / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded random weights N(0,0.02), uniform token ids)",
            "config": {"workload": f"{cfg.name}: {cfg.n_layers}x d{cfg.d_model} H{cfg.num_heads} ds{cfg.d_state} "
                                   f"C{cfg.chunk_size}, vocab {cfg.vocab}, B{cfg.batch} L{cfg.seq_len}, full logits",
                       "global_batch": cfg.batch, "seq_len": cfg.seq_len,
                       "parallelism": {"single": "single",
                                       "sp": f"sp{world} (sequence-parallel segments, "
                                             + ("peer-store carries and halos over NVLink)" if args.sp_transport == "p2p"
                                                else "NCCL all-gather carries and halos)"),
                                       "batch": f"dp{world} (batch-sharded, no collective)"}[mode],
                       "launch": "eager" if args.eager else "cuda_graph",
                       "l2": "working set > L2 (projs 214 MB/layer, weights 153 MB): no explicit flush"},
            "roofline": {"kernel": ("slot_state + slot_scan_gate_carry (slot_tc_state_pipe + slot_fold + slot_tc_pipe)"
                                    if mode == "sp" else "slot_scan_gate (slot_tc_state_pipe + slot_tc_pipe)"), "bound": "hbm", "achieved": achieved, "peak": hbm,
                         "unit": "GB/s", "frac": achieved / hbm, "peak_source": src,
                         "traffic": SLOT_TRAFFIC_BYTES * tokens_per_rank / (cfg.batch * cfg.seq_len),
                         "traffic_source": "ncu capture of the 1-GPU op" + (
                             ", scaled by this rank's share of the tokens" if world > 1 else ""),
                         "timing": "CUDA events around a CUDA-graph replay of one layer's slot calls, "
                                   "L2 flushed before each, mean of 10",
                         "algorithmic_bytes_per_launch": slot_bytes,
                         "ms_per_launch": slot_ms, "launches_per_step": slot_per_step},
            "e2e": {"value": world * tokens_per_rank / (e2e_ms * 1e-3), "unit": "tokens/s",
                    "h2d_bytes_per_step": world * ids_host.numel() * ids_host.element_size(),
                    "d2h_bytes_per_step": world * out_host.numel() * out_host.element_size(),
                    "result": "ids copied host->device from pinned memory each step; the full logits "
                              "[B, L, vocab] are computed and stay on the device, and the last position's "
                              "logits [B, vocab] are copied device->host each step"},
            "gpu_launches": launches,
            "clocks": clocks,
        }
        if world == 1 and not args.no_kernels:
            line["kernels"] = [kernel_c2(dev, 20, hbm), kernel_c2bwd(dev, 10, hbm), kernel_c3(dev, 10, hbm),
                               kernel_c5slot(dev, 10, hbm)]
        if world == 1 and not args.no_kernels:
            line["decode"] = [decode_c5(dev, 1), decode_c5(dev, 64)]
        if world == 1 and not args.no_cpu_baseline:
            v, cores = cpu_oracle_tokens_per_s(cfg, args.cpu_tokens)
            line["cpu_baseline"] = {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port",
                                    "sample": f"first {args.cpu_tokens} of {cfg.seq_len} tokens, all layers + head"}
        print(json.dumps(line), flush=True)
    if world > 1:
        del graphed  # a graph holding NCCL calls must go before the process group
        if mode == "sp":
            sp.close()
        torch.cuda.synchronize()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
