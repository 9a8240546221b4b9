"""Benchmark: W8 decode tokens/s of the 8B-shaped decoder.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (one GPU): the 8B-shaped Qwen3-style W8 decoder (36 layers, hidden
4096, 32 q / 8 kv heads, head_dim 128, SwiGLU 12288, vocab 151936, int8
per-channel weights, synthetic seeded values), a 2048-token random prompt fed
through the decoder, then greedy decode steps.  A "step" is one decode step
at batch 1 (the headline `value`); the same is measured at batch 64.

N > 1 (torchrun, one process per GPU): the same 8B model sharded tensor-
parallel over the N GPUs (heads, intermediate and vocab split; NCCL all-
reduce after o_proj and down_proj over NVLink); value = tokens/s of the
batch-1 sequence (and of batch 64), max-over-ranks time ("scaling": "strong").

`--impl reference`: the reference path's CPU restatement (oracle/, the
reference's Rust/XLA stack cannot run here) timed on all host cores, rank 0.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CONFIG4 = dict(layers=36, hidden=4096, q_heads=32, kv_heads=8, head_dim=128, intermediate=12288,
               vocab=151936, rms_eps=1e-6, rope_theta=1e6)
CONFIG5 = dict(layers=64, hidden=5120, q_heads=64, kv_heads=8, head_dim=128, intermediate=25600,
               vocab=151936, rms_eps=1e-6, rope_theta=1e6)
PROMPT = 2048
PROMPT5, BATCH5 = 4096, 32
METRIC = "W8 decode tokens/sec"
UNIT = "tokens/s"


def step_bytes(cfg, batch, ctx):
    """Algorithmic HBM bytes of one decode step: every weight byte once, the
    visible KV cache once, plus the per-token activations (negligible)."""
    H, D, I, V = cfg["hidden"], cfg["head_dim"], cfg["intermediate"], cfg["vocab"]
    hq, hkv = cfg["q_heads"], cfg["kv_heads"]
    per_layer = (hq + 2 * hkv) * D * H + H * hq * D + 2 * I * H + H * I
    weights = cfg["layers"] * per_layer + V * H
    kv = cfg["layers"] * batch * (ctx + 1) * hkv * D * 2 * 2
    return weights, kv


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during timing."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.idx = device_index
        self.rows = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except FileNotFoundError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm = [float(r[1]) for r in self.rows if len(r) >= 9 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) >= 9 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows if len(r) >= 9
                          for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(sm)}


def launches_per_step(cfg, tp=1):
    """Our kernels in one batch-1 decode step: embedding, per layer qkv (norm
    fused), attention, o_proj, gate/up (norm fused), down, and the LM head with
    the norm and the greedy argmax fused.  Tensor parallel adds per layer the
    two peer all-reduce kernels (fused with the residual add) and, after the
    head, the argmax candidate and merge kernels (the head's own argmax is
    not fused then); NCCL's all-gather of the candidates is not ours."""
    if tp == 1:
        return 1 + cfg["layers"] * 5 + 1
    return 1 + cfg["layers"] * 7 + 1 + 2


def measured_peaks():
    try:
        with open(ROOT / "MEASURED_PEAKS.json") as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ------------------------------------------------------------------ CPU legs

def cpu_decode_sample(threads_note=True):
    """Time the CPU oracle on a bounded sample of the config-4 decoder.

    Sample: the decoder with 2 of the 36 layers (full 151936-token tied head),
    4 decode steps after 4 prompt tokens; the per-layer time is
    (step - head) / 2 and a full token costs 36 layers + head.
    """
    import numpy as np
    import oracle
    cfg = dict(CONFIG4, layers=2)
    dec = oracle.Decoder(**cfg, max_batch=1, max_context=32)
    dec.init_synthetic(0)
    tok = np.array([1], np.int32)
    for _ in range(4):
        _, tok = dec.step(tok)
    t0 = time.perf_counter()
    n = 3
    for _ in range(n):
        _, tok = dec.step(tok)
    t_step = (time.perf_counter() - t0) / n
    emb_w = dec.parameter("embed_tokens.weight").reshape(CONFIG4["vocab"], CONFIG4["hidden"])
    emb_s = dec.parameter("embed_tokens.scale").reshape(CONFIG4["vocab"], 1)
    x = np.ones((1, CONFIG4["hidden"]), np.float32)
    t0 = time.perf_counter()
    oracle.w8_linear(x, emb_w, emb_s, CONFIG4["hidden"], mode=2)
    t_head = time.perf_counter() - t0
    dec.close()
    t_layer = max(t_step - t_head, 1e-9) / 2
    t_token = CONFIG4["layers"] * t_layer + t_head
    return {"value": 1.0 / t_token, "unit": UNIT, "cores": oracle.num_threads(), "kind": "port",
            "sample": f"oracle C restatement, 2 of 36 layers + full head, {n} timed decode steps "
                      f"(step {t_step:.3f}s, head {t_head:.3f}s), extrapolated to 36 layers"}


def cpu_prefill_sample():
    """Time the CPU oracle's full-sequence causal forward on a bounded sample
    of the config-4 prefill: 1 of the 36 layers over a 64-token prompt plus
    the tied head on the last row, extrapolated to 36 layers (the linears,
    nearly all of the work, scale with the prompt length)."""
    import numpy as np
    import oracle
    cfg = dict(CONFIG4, layers=1)
    dec = oracle.Decoder(**cfg, max_batch=1, max_context=80)
    dec.init_synthetic(0)
    n = 64
    prompt = np.arange(1, n + 1, dtype=np.int32)
    t0 = time.perf_counter()
    dec.forward(prompt)
    t_fwd = time.perf_counter() - t0
    emb_w = dec.parameter("embed_tokens.weight").reshape(CONFIG4["vocab"], CONFIG4["hidden"])
    emb_s = dec.parameter("embed_tokens.scale").reshape(CONFIG4["vocab"], 1)
    x = np.ones((1, CONFIG4["hidden"]), np.float32)
    t0 = time.perf_counter()
    oracle.w8_linear(x, emb_w, emb_s, CONFIG4["hidden"], mode=2)
    t_head = time.perf_counter() - t0
    dec.close()
    t_layer = max(t_fwd - t_head, 1e-9)
    t_prompt = CONFIG4["layers"] * t_layer + t_head
    return {"value": n / t_prompt, "unit": "tokens/s", "cores": oracle.num_threads(),
            "kind": "port",
            "sample": f"oracle C restatement, full-sequence causal forward, 1 of 36 layers over "
                      f"a {n}-token prompt ({t_fwd:.2f}s incl. head {t_head:.2f}s), "
                      f"extrapolated to 36 layers"}


# --------------------------------------------------------------- our path

def run_ours(args, rank, world, local_rank):
    import numpy as np
    import torch
    from rxla_b200 import _lib
    from rxla_b200.decoder import Comm, Decoder

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    stream = torch.cuda.current_stream()
    sptr = ctypes.c_void_p(stream.cuda_stream)
    lib = _lib.load()
    cfg = dict(CONFIG4)
    max_ctx = PROMPT + args.warmup + args.steps + 32
    b64 = 1 if args.no_batch64 else 64
    # N > 1: one 8B model sharded tensor-parallel over the N GPUs (NCCL over
    # NVLink), the same synthetic model at every N
    comm = None
    if world > 1:
        def share(data):
            obj = [data]
            torch.distributed.broadcast_object_list(obj, src=0)
            return obj[0]
        comm = Comm(rank, world, local_rank, share)
    dec = Decoder(**cfg, embedding_dtype="u8", max_batch=b64, max_context=max_ctx,
                  device=local_rank, comm=comm.handle if comm else None, tp_rank=rank,
                  tp_size=world)
    dec.init_synthetic(1234)

    tin = ctypes.c_void_p(dec.tokens_in_ptr)
    tout = ctypes.c_void_p(dec.tokens_out_ptr)

    def prompt_fill(batch):
        dec.reset(sptr)
        prompt = torch.randint(0, cfg["vocab"], (PROMPT, batch), dtype=torch.int32, device=dev,
                               generator=torch.Generator(device=dev).manual_seed(1))
        for t in range(PROMPT):
            _lib.call("rxla_b200_decoder_step", dec.handle, ctypes.c_void_p(prompt[t].data_ptr()),
                      batch, tout, None, sptr)
        torch.cuda.synchronize()

    def greedy(batch, n):
        for _ in range(n):
            _lib.call("rxla_b200_decoder_step", dec.handle, tout, batch, tout, None, sptr)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    def timed(batch, n):
        greedy(batch, args.warmup)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        greedy(batch, n)
        e1.record(stream)
        barrier()
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    sampler = ClockSampler(local_rank)
    # ---- batch 1 (headline)
    prompt_fill(1)
    sampler.start()
    ms1 = timed(1, args.steps)
    ctx_b1 = PROMPT + args.warmup + args.steps // 2
    # ---- end to end through the host-buffer C ABI: H2D tokens, D2H next tokens
    host_tok = np.zeros(1, np.int32)
    dec.step_host(host_tok)
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        host_tok = dec.step_host(host_tok)
    e2e_s = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([e2e_s], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_s = float(t.item())
    # ---- batch 64: every sequence at the 2048-token context (pages sized and
    # set by rxla_b200_decoder_set_context_lengths; the step's work does not
    # depend on the cached values)
    res64 = None
    if b64 == 64:
        dec.reset(sptr)
        dec.set_context_lengths([PROMPT] * 64, sptr)
        n64 = max(8, min(args.steps, 64))
        ms64 = timed(64, n64)
        w, kv = step_bytes(cfg, 64, PROMPT + args.warmup + n64 // 2)
        res64 = {"value": 64 * n64 / (ms64 / 1e3), "ms_per_step": ms64 / n64, "steps": n64,
                 "step_gbs": (w + kv) / (ms64 / n64 * 1e-3) / 1e9}
    clocks = sampler.stop()

    # ---- roofline of the dominant kernel: the W8 linear, all launches of one
    # batch-1 step (qkv, o, gate/up, down per layer + tied head) replayed in a graph
    roof = gemv_roofline(dec, cfg, dev, stream, lib, world)
    status = lib.rxla_b200_device_status(local_rank)
    dec.close()  # releases the captured graphs (they hold NCCL calls) before the comm
    res5 = None if args.no_config5 else run_config5(args, rank, world, local_rank, comm, barrier)
    if comm:
        comm.close()

    weights, kv1 = step_bytes(cfg, 1, ctx_b1)
    tok_s = args.steps / (ms1 / 1e3)  # one sequence, decoded by all N GPUs together
    out = {
        "metric": METRIC, "value": tok_s, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms1 / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "u8 weights, bf16 activations, fp32 accumulate",
        "data": "synthetic (seeded random W8 weights, random 2048-token prompt)",
        "config": {"workload": "config4: 8B-shaped W8 decoder, batch 1 decode after a 2048-token prompt",
                   "model": "qwen3-style-8B-shape", "layers": 36, "hidden": 4096, "vocab": 151936,
                   "global_batch": 1, "seq_len": PROMPT,
                   "parallelism": (f"tp{world} (" + ("NCCL" if os.environ.get("RXLA_B200_P2P") == "0"
                                                      else "one-shot NVLink peer")
                                   + " all-reduce after o_proj and down_proj)") if world > 1 else "single GPU",
                   "l2": "inputs > L2 (7.6 GB of weights per step)"},
        "step_gbs": (weights + kv1) / (ms1 / args.steps * 1e-3) / 1e9,
        "step_frac_of_hbm": (weights + kv1) / (ms1 / args.steps * 1e-3) / 1e9 / (world * measured_peaks()[0]),
        "batch64": res64,
        "config5": res5,
        "e2e": {"value": args.steps / e2e_s, "unit": UNIT, "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": 4},
        "roofline": roof,
        "clocks": clocks,
        "gpu_launches": args.steps * launches_per_step(cfg, world),
        "device_status": status,
    }
    return out


def run_config5(args, rank, world, local_rank, comm, barrier):
    """Config 5: the 32B-shaped W8 decoder, tensor-parallel over the N GPUs
    (N = 1 for the single-GPU reference point), batch 32 at a 4096-token
    context.  The K/V pages are sized for the context and the lengths set
    through rxla_b200_decoder_set_context_lengths instead of decoding 4096
    prompt steps (the step's work and bytes do not depend on the cached
    values); then timed greedy decode steps, max over ranks."""
    import torch
    from rxla_b200 import _lib
    from rxla_b200.decoder import Decoder
    stream = torch.cuda.current_stream()
    sptr = ctypes.c_void_p(stream.cuda_stream)
    n = max(8, min(args.steps, 32))
    dec = Decoder(**CONFIG5, embedding_dtype="u8", max_batch=BATCH5,
                  max_context=PROMPT5 + args.warmup + n + 16, device=local_rank,
                  comm=comm.handle if comm else None, tp_rank=rank, tp_size=world)
    dec.init_synthetic(4321)
    dec.set_context_lengths([PROMPT5] * BATCH5, sptr)
    tout = ctypes.c_void_p(dec.tokens_out_ptr)
    for _ in range(args.warmup):
        _lib.call("rxla_b200_decoder_step", dec.handle, tout, BATCH5, tout, None, sptr)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(n):
        _lib.call("rxla_b200_decoder_step", dec.handle, tout, BATCH5, tout, None, sptr)
    e1.record(stream)
    barrier()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device=torch.device("cuda", local_rank))
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    status = _lib.load().rxla_b200_device_status(local_rank)
    dec.close()
    w, kv = step_bytes(CONFIG5, BATCH5, PROMPT5 + args.warmup + n // 2)
    sec = ms / n / 1e3
    return {"workload": "config5: 32B-shaped W8 decoder, batch 32 decode at a 4096-token context",
            "value": BATCH5 / sec, "unit": UNIT, "ms_per_step": ms / n, "steps": n, "tp": world,
            "parallelism": f"tp{world}" if world > 1 else "single GPU",
            "step_gbs_per_gpu": (w + kv) / world / sec / 1e9,
            "frac_of_hbm": (w + kv) / world / sec / 1e9 / measured_peaks()[0],
            "kv_cache": "pages sized for the context, lengths set directly (zero-filled values)",
            "device_status": status}


def gemv_roofline(dec, cfg, dev, stream, lib, tp=1):
    """Time every W8 linear of one batch-1 step of this rank's shard, replayed as
    one CUDA graph.

    Algorithmic bytes per launch = N·K weights + 4·N scales + 2·K (x) + output;
    achieved = Σ bytes / Σ time of the launches (bytes-weighted mean)."""
    import torch
    H, D = cfg["hidden"], cfg["head_dim"]
    I, V, hq = cfg["intermediate"] // tp, cfg["vocab"] // tp, cfg["q_heads"] // tp
    qkv_rows = (hq + 2 * cfg["kv_heads"] // tp) * D
    x = torch.zeros(1, max(H, I, hq * D), dtype=torch.bfloat16, device=dev)
    ybf = torch.empty(1, max(qkv_rows, I), dtype=torch.bfloat16, device=dev)
    yf = torch.zeros(1, max(H, V), dtype=torch.float32, device=dev)
    s = ctypes.c_void_p(stream.cuda_stream)
    launches = []
    for l in range(cfg["layers"]):
        p = f"layers.{l}."
        launches.append((p + "self_attn.qkv", qkv_rows, H, ybf, 1, 0))
        launches.append((p + "self_attn.o_proj", H, hq * D, yf, 0, 1))
        launches.append((p + "mlp.gate_up", I, H, ybf, 1, 2))
        launches.append((p + "mlp.down_proj", H, I, yf, 0, 1))
    launches.append(("embed_tokens", V, H, yf, 0, 0))
    total_bytes = 0
    calls = []
    rank = int(os.environ.get("RANK", "0"))
    for name, n, k, y, ybf16, epi in launches:
        w, _, _ = dec.parameter(name + ".weight")
        sc, _, _ = dec.parameter(name + ".scale")
        if name == "embed_tokens":  # the rank's vocab slice of the tied head
            w, sc = w + rank * V * k, sc + rank * V * 4
        rows = 2 * n if epi == 2 else n
        total_bytes += rows * k + 4 * rows + 2 * k + (2 if ybf16 else 4) * n * (2 if epi == 1 else 1)
        calls.append((x.data_ptr(), w, sc, k, n, k, y.data_ptr(), 1 if ybf16 else 0, epi))

    def run():
        for xp, w, sc, g, n, k, yp, ybf16, epi in calls:
            st = lib.rxla_b200_w8a16_linear(xp, 1, w, sc, g, 1, n, k, yp, ybf16, epi,
                                            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
            assert st == 0
    run()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        run()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    reps = 10
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    sec = e0.elapsed_time(e1) / 1e3 / reps
    peak, kind = measured_peaks()
    achieved = total_bytes / sec / 1e9
    # DRAM bytes per launch: the algorithmic bytes scaled by the LM-head ncu
    # capture's measured ratio (dram read + write 626.74 MB / algorithmic
    # 623.25 MB, profiles/w8_gemv_lm_head_config4.md)
    traffic = total_bytes / len(calls) * (626.74 / 623.25)
    return {"bound": "hbm", "kernel": "w8_skinny_kernel (all W8 linears of one batch-1 step)",
            "achieved": achieved, "peak": peak, "peak_kind": kind, "unit": "GB/s",
            "frac": achieved / peak, "traffic": traffic,
            "traffic_note": "per launch, scaled from the LM-head ncu capture",
            "launches": len(calls), "avg_launch_us": sec / len(calls) * 1e6,
            "bytes_per_step": total_bytes}


def prefill_flops(cfg, tokens):
    """Algorithmic FLOPs of a prompt through the decoder: 2 per weight per row
    for every layer's linears, the causal attention (q·k and p·v, 4·Hq·D per
    key, row t seeing t + 1 keys), and the head for the last row only."""
    h, d, hq, hkv, i = cfg["hidden"], cfg["head_dim"], cfg["q_heads"], cfg["kv_heads"], cfg["intermediate"]
    per_layer = h * (hq + 2 * hkv) * d + hq * d * h + 2 * i * h + i * h
    lin = 2.0 * per_layer * cfg["layers"] * tokens
    att = 4.0 * hq * d * tokens * (tokens + 1) / 2 * cfg["layers"]
    return lin + att + 2.0 * cfg["vocab"] * h


def run_prefill(args):
    """Config 4 prefill: a PROMPT-token prompt of one sequence through
    rxla_b200_decoder_prefill (chunks of rows on the tcgen05 GEMM, causal
    paged attention), from position 0 each step.  Tensor-bound: the roofline
    is the measured bf16 GEMM peak.  Prints one JSON line."""
    import numpy as np
    import torch
    from rxla_b200.decoder import Decoder
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    dec = Decoder(**CONFIG4, embedding_dtype="u8", max_batch=1, max_context=PROMPT + 16)
    dec.init_synthetic(1)
    stream = torch.cuda.current_stream()
    s = ctypes.c_void_p(stream.cuda_stream)
    prompt = torch.from_numpy(np.random.default_rng(5).integers(0, CONFIG4["vocab"], PROMPT)
                              .astype(np.int32)).to(dev)
    host_prompt = prompt.cpu().pin_memory()
    for _ in range(args.warmup):
        dec.reset(s)
        dec.prefill(0, prompt, stream=s)
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    sampler = ClockSampler(0)
    sampler.start()
    t0 = time.perf_counter()
    ev[0].record(stream)
    for _ in range(args.steps):
        dec.reset(s)
        dec.prefill(0, prompt, stream=s)
    ev[1].record(stream)
    torch.cuda.synchronize()
    wall = (time.perf_counter() - t0) / args.steps
    ms = ev[0].elapsed_time(ev[1]) / args.steps
    # end to end: the prompt from pinned host memory, the token back to the host
    t0 = time.perf_counter()
    for _ in range(args.steps):
        dec.reset(s)
        prompt.copy_(host_prompt, non_blocking=True)
        tok = dec.prefill(0, prompt, stream=s)
        tok.cpu()
    e2e_s = (time.perf_counter() - t0) / args.steps
    clocks = sampler.stop()
    flops = prefill_flops(CONFIG4, PROMPT)
    try:
        with open(ROOT / "MEASURED_PEAKS.json") as f:
            peak, how = float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        peak, how = 1590.0, "fallback"
    achieved = flops / (ms * 1e-3) / 1e12
    line = {"metric": "W8 prefill tokens/sec", "value": PROMPT / (ms * 1e-3), "unit": "tokens/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "wall_ms_per_step": wall * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u8 weights, bf16 operands, f32 accumulate",
            "data": "synthetic",
            "config": {"workload": f"config4: 8B-shaped W8 decoder, {PROMPT}-token prompt, "
                                   "one sequence, prefill from position 0",
                       "l2": "weights 6.95 GB per pass, larger than L2"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak,
                         "unit": "TFLOP/s", "frac": achieved / peak, "peak_source": how,
                         "flops_per_step": flops, "traffic": None},
            "e2e": {"value": PROMPT / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": PROMPT * 4,
                    "d2h_bytes_per_step": 4},
            "clocks": clocks}
    dec.close()
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_prefill_sample()
    print(json.dumps(line), flush=True)


def profile_case(what: str):
    """Small, self-contained cases for ncu captures (no JSON line).

    gemv:      one W8 linear, N=32768 K=4096 M=1 (134 MB of weights > L2), 3 launches
    head:      the tied LM head of config 4, N=151936 K=4096 M=1 (622 MB), 3 launches
    gemm:      config-2 tensor-bound row, M=2048 N=4096 K=4096 on the tcgen05 GEMM, 3 launches
    step:      the config-4 decoder after a 256-token prompt, 2 decode steps inside
               the NVTX range "profile"
    step64:    config 4 at batch 64 (2048 context), 1 step inside "profile"
    step5:     config 5 (32B shape) at batch 32 (4096 context), 1 step inside "profile"
    gemmdec:   a 2-layer config-4-shaped decoder at batch 64, 1 step (the decode-batch
               GEMM launches: qkv, o, gate/up, down per layer, then the head)
    prefill:   a 2-layer config-4-shaped decoder, one 2048-token prompt (two
               1024-row chunks) after one warm-up prompt
    attention: config-3 paged decode attention (batch 64, 32 q / 8 kv heads, d 128,
               ctx ~U[512, 8192]), 3 launches
    """
    import numpy as np
    import torch
    from rxla_b200 import _lib, nn
    dev = torch.device("cuda:0")
    if what in ("head", "gemm"):
        m, n, k = (1, 151936, 4096) if what == "head" else (2048, 4096, 4096)
        w = torch.randint(0, 256, (n, k), dtype=torch.uint8, device=dev)
        sc = torch.rand(n, 1, device=dev) * 1e-2
        x = torch.randn(m, k, device=dev).bfloat16()
        y = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
        for _ in range(3):
            nn.quantized_linear(x, w, sc, k, out=y)
    elif what == "gemv":
        n, k = 32768, 4096
        w = torch.randint(0, 256, (n, k), dtype=torch.uint8, device=dev)
        sc = torch.rand(n, 1, device=dev) * 1e-2
        x = torch.randn(1, k, device=dev).bfloat16()
        y = torch.empty(1, n, dtype=torch.bfloat16, device=dev)
        for _ in range(3):
            nn.quantized_linear(x, w, sc, k, out=y)
    elif what == "step":
        from rxla_b200.decoder import Decoder
        dec = Decoder(**CONFIG4, embedding_dtype="u8", max_batch=1, max_context=320)
        dec.init_synthetic(1)
        s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        tout = ctypes.c_void_p(dec.tokens_out_ptr)
        for _ in range(256):
            _lib.call("rxla_b200_decoder_step", dec.handle, tout, 1, tout, None, s)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("profile")
        for _ in range(2):
            _lib.call("rxla_b200_decoder_step", dec.handle, tout, 1, tout, None, s)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        dec.close()
    elif what == "gemmdec":
        # the decode-batch GEMMs of a 2-layer config-4-shaped decoder at batch 64
        # (2048 context): 1 step, kernels launched directly (RXLA_B200_NO_GRAPH=1)
        from rxla_b200.decoder import Decoder
        cfg = dict(CONFIG4, layers=2)
        dec = Decoder(**cfg, embedding_dtype="u8", max_batch=64, max_context=PROMPT + 16)
        dec.init_synthetic(1)
        s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        dec.set_context_lengths([PROMPT] * 64, s)
        tout = ctypes.c_void_p(dec.tokens_out_ptr)
        _lib.call("rxla_b200_decoder_step", dec.handle, tout, 64, tout, None, s)
        torch.cuda.synchronize()
        dec.close()
    elif what == "prefill":
        from rxla_b200.decoder import Decoder
        cfg = dict(CONFIG4, layers=2)
        dec = Decoder(**cfg, embedding_dtype="u8", max_batch=1, max_context=PROMPT + 16)
        dec.init_synthetic(1)
        s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        prompt = torch.randint(0, cfg["vocab"], (PROMPT,), dtype=torch.int32, device=dev)
        for _ in range(2):
            dec.reset(s)
            dec.prefill(0, prompt, stream=s)
        torch.cuda.synchronize()
        dec.close()
    elif what in ("step64", "step5"):
        # batch 64 of config 4 at a 2048 context / batch 32 of config 5 at 4096:
        # 2 warm-up steps, then 1 step inside the NVTX range "profile"
        from rxla_b200.decoder import Decoder
        cfg, batch, ctx = (CONFIG4, 64, PROMPT) if what == "step64" else (CONFIG5, BATCH5, PROMPT5)
        dec = Decoder(**cfg, embedding_dtype="u8", max_batch=batch, max_context=ctx + 16)
        dec.init_synthetic(1)
        s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        dec.set_context_lengths([ctx] * batch, s)
        tout = ctypes.c_void_p(dec.tokens_out_ptr)
        for _ in range(2):
            _lib.call("rxla_b200_decoder_step", dec.handle, tout, batch, tout, None, s)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("profile")
        _lib.call("rxla_b200_decoder_step", dec.handle, tout, batch, tout, None, s)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        dec.close()
    elif what == "attention":
        batch, hq, hkv, d, max_ctx = 64, 32, 8, 128, 8192
        cache = nn.PagedKvCache(batch=batch, kv_heads=hkv, head_dim=d, max_context=max_ctx)
        cache.k.normal_()
        cache.v.normal_()
        g = torch.Generator(device=dev).manual_seed(3)
        cache.ctx_lens = torch.randint(512, 8192, (batch,), dtype=torch.int32, device=dev,
                                       generator=g)
        qkv = torch.randn(batch, (hq + 2 * hkv) * d, device=dev).bfloat16()
        ws = torch.zeros(nn.paged_decode_workspace_size(batch, hq, hkv, d, max_ctx),
                         dtype=torch.uint8, device=dev)
        inv = torch.from_numpy(nn.rope_inv_freq(1e6, d)).to(dev)
        for _ in range(3):
            nn.paged_decode_attention(qkv[:, :hq * d], qkv[:, hq * d:(hq + hkv) * d],
                                      qkv[:, (hq + hkv) * d:], cache, q_heads=hq, inv_freq=inv,
                                      rotary_dim=d, workspace=ws)
    torch.cuda.synchronize()
    print("profile case done:", what)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-batch64", action="store_true")
    ap.add_argument("--no-config5", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--prefill", action="store_true",
                    help="measure the config-4 prompt prefill instead of decode (one JSON line)")
    ap.add_argument("--profile", choices=["gemv", "head", "gemm", "gemmdec", "step", "step64", "step5", "prefill", "attention"], default=None,
                    help="run a small case for an ncu capture instead of the benchmark")
    args = ap.parse_args()
    if args.profile:
        profile_case(args.profile)
        return
    args.warmup = max(args.warmup, 3)
    if args.prefill:
        run_prefill(args)
        return

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return
        steps = []
        res = None
        for _ in range(max(1, min(args.steps, 2))):
            res = cpu_decode_sample()
            steps.append(res["value"])
        value = statistics.median(steps)
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                "impl": "reference", "scaling": "weak", "vs_baseline": None,
                "dtype": "u8 weights, f32 activations (CPU restatement)",
                "data": "synthetic", "config": {"workload": "config4: 8B-shaped W8 decoder, batch 1 decode"},
                "cpu_baseline": {**res, "value": value},
                "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    if world > 1:
        import torch
        import datetime
        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local_rank))
    out = run_ours(args, rank, world, local_rank)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_decode_sample()
    if world > 1:
        import torch
        torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
