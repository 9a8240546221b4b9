"""Benchmark: W8 decode tokens/s of the 8B-shaped decoder.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (one GPU): the 8B-shaped Qwen3-style W8 decoder (36 layers, hidden
4096, 32 q / 8 kv heads, head_dim 128, SwiGLU 12288, vocab 151936, int8
per-channel weights, synthetic seeded values), a 2048-token random prompt run
through the prefill, then greedy decode steps.  A "step" is one decode step at
batch 1 (the headline `value`); the same is measured at batch 64, and config
5 (the 32B shape, batch 32 at a 4096-token context).

Before any timing, every rank checks tensor-parallel parity: a small W8
decoder with 8 kv heads (so TP-8 divides it) runs 16 prompt and 32 greedy
decode steps at TP-N against the CPU oracle holding the same full model; the
line's `parity` key carries the logits errors and the token comparison, and
the run exits non-zero when it fails.

At N = 1 the line also carries the kernel-level BASELINE configs, each timed
with CUDA events on inputs larger than L2: config 2 (the W8A16 linear sweep,
24 (N, K, M) points), config 3 (paged GQA decode attention, batch 64) and the
config-4 prefill of the 2048-token prompt.

N > 1 (torchrun, one process per GPU): the same 8B model sharded tensor-
parallel over the N GPUs (heads, intermediate and vocab split; the
row-parallel partial sums all-reduced over NVLink peer memory after o_proj
and down_proj); value = tokens/s of the batch-1 sequence, max-over-ranks time
("scaling": "strong").

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
# tensor-parallel parity model: 8 kv heads (TP-8 divides heads, intermediate
# and vocab); weights and prompt seeds whose 33 oracle tokens all beat their
# runner-up by at least the 2e-2 logits tolerance (chosen by running the oracle)
PARITY_CFG = dict(layers=2, hidden=1024, q_heads=16, kv_heads=8, head_dim=64, intermediate=2048,
                  vocab=8192, rms_eps=1e-6, rope_theta=1e6)
PARITY_SEED, PARITY_PROMPT_SEED, PARITY_PROMPT, PARITY_STEPS = 6, 106, 16, 32
PARITY_MAX_ABS, PARITY_MEAN_ABS, PARITY_FLOOR_MARGIN = 2e-2, 2e-3, 1.25


def step_bytes(cfg, batch, ctx):
    """Algorithmic HBM bytes of one decode step: every weight byte once, the
    visible KV cache once, plus the per-token activations (negligible)."""
    H, D, I, V = cfg["hidden"], cfg["head_dim"], cfg["intermediate"], cfg["vocab"]
    hq, hkv = cfg["q_heads"], cfg["kv_heads"]
    per_layer = (hq + 2 * hkv) * D * H + H * hq * D + 2 * I * H + H * I
    weights = cfg["layers"] * per_layer + V * H
    kv = cfg["layers"] * batch * (ctx + 1) * hkv * D * 2 * 2
    return weights, kv


def workload_config(world):
    """The `config` of the JSON line: the same dict for both arms."""
    return {"workload": "config4: 8B-shaped W8 decoder, batch 1 decode after a 2048-token prompt",
            "model": "qwen3-style-8B-shape", "layers": 36, "hidden": 4096, "vocab": 151936,
            "global_batch": 1, "seq_len": PROMPT,
            "parallelism": f"tp{world} (one-shot NVLink peer all-reduce after o_proj and down_proj)"
                           if world > 1 else "single GPU",
            "l2": "inputs > L2 (7.6 GB of weights per step)"}


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


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
    """(HBM GB/s, bf16 TF/s burst, bf16 TF/s sustained, source)."""
    try:
        with open(ROOT / "MEASURED_PEAKS.json") as f:
            p = json.load(f)
        return (float(p["hbm_gbs"]), float(p["bf16_tflops"]),
                float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), "measured")
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


# ------------------------------------------------------------------ CPU legs

def cpu_decode_sample():
    """Time the CPU oracle on a bounded sample of the config-4 decode step.

    Sample: the decoder with 2 of the 36 layers and the full 151936-token
    tied head, sequence context set to the GPU arm's 2048 tokens, 3 timed
    decode steps; per layer (step - head) / 2, a token = 36 layers + head.
    All host cores (OpenMP threads set explicitly, whatever OMP_NUM_THREADS
    the launcher exported)."""
    import numpy as np
    import oracle
    cores = host_cores()
    oracle.set_num_threads(cores)
    cfg = dict(CONFIG4, layers=2)
    dec = oracle.Decoder(**cfg, max_batch=1, max_context=PROMPT + 16)
    dec.init_synthetic(0)
    dec.set_context(0, PROMPT)
    tok = np.array([1], np.int32)
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
            "sample": f"oracle C restatement on {oracle.num_threads()} host threads: 2 of 36 "
                      f"layers + the full tied head at a {PROMPT}-token context, {n} timed "
                      f"decode steps (step {t_step:.3f}s, head {t_head:.3f}s), extrapolated "
                      f"linearly to 36 layers"}


def cpu_prefill_sample():
    """Time the CPU oracle's full-sequence causal forward on a bounded sample
    of the config-4 prefill: 1 of the 36 layers over a 64-token prompt plus
    the tied head on the last row, extrapolated to 36 layers (the linears,
    nearly all of the work, scale with the prompt length)."""
    import numpy as np
    import oracle
    oracle.set_num_threads(host_cores())
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


# --------------------------------------------------------------- parity

def tp_parity(rank, world, local_rank, comm):
    """Tensor-parallel parity at this N against the CPU oracle (every rank).

    PARITY_CFG's W8 decoder (tied W8 head, per-channel scales) is built by the
    oracle from PARITY_SEED on every rank (deterministic, so every rank holds
    the same full model) and sliced to this rank's shard with
    shard_parameter.  16 prompt tokens and 32 greedy decode steps, teacher
    forced; each rank compares its vocab slice of the logits, the slices'
    errors are combined over the ranks (max, and the sum for the mean), and
    the greedy tokens (the cross-rank argmax) are compared with the oracle's.
    Pattern of the reference's stateful decode test
    (crates/rxla-core/tests/masked_decode.rs:54-142)."""
    import numpy as np
    import torch
    import oracle
    from rxla_b200 import _lib
    from rxla_b200.decoder import Decoder, shard_parameter
    cfg = PARITY_CFG
    oracle.set_num_threads(max(1, host_cores() // world))
    ref = oracle.Decoder(**cfg, embedding_bf16=False, group_size=0, max_batch=1, max_context=64)
    ref.init_synthetic(PARITY_SEED)
    # the same oracle with fp32 running sums in its linears: the accumulation
    # noise floor every fp32-accumulating implementation (XLA's CPU dot too)
    # sits at against the f64 oracle
    f32 = oracle.Decoder(**cfg, embedding_bf16=False, group_size=0, max_batch=1, max_context=64,
                         linear_mode=4)
    f32.init_synthetic(PARITY_SEED)
    gpu = Decoder(**cfg, embedding_dtype="u8", max_batch=1, max_context=64, device=local_rank,
                  comm=comm.handle if comm else None, tp_rank=rank, tp_size=world)
    H, D, I, V = cfg["hidden"], cfg["head_dim"], cfg["intermediate"], cfg["vocab"]
    rows = {"q_proj": cfg["q_heads"] * D, "k_proj": cfg["kv_heads"] * D,
            "v_proj": cfg["kv_heads"] * D, "o_proj": H, "gate_proj": I, "up_proj": I,
            "down_proj": H}
    names = ["embed_tokens.weight", "embed_tokens.scale", "norm.weight"]
    for l in range(cfg["layers"]):
        p = f"layers.{l}."
        names += [p + "input_layernorm.weight", p + "post_attention_layernorm.weight",
                  p + "self_attn.q_norm.weight", p + "self_attn.k_norm.weight"]
        names += [f"{p}self_attn.{pr}.{k}" for pr in ("q_proj", "k_proj", "v_proj", "o_proj")
                  for k in ("weight", "scale")]
        names += [f"{p}mlp.{pr}.{k}" for pr in ("gate_proj", "up_proj", "down_proj")
                  for k in ("weight", "scale")]
    kw = dict(q_heads=cfg["q_heads"], kv_heads=cfg["kv_heads"], head_dim=D, intermediate=I,
              hidden=H, vocab=V)
    for n in names:
        a = np.array(ref.parameter(n))
        for pr, r in rows.items():
            if f".{pr}." in n:
                a = a.reshape(r, -1)
        gpu.set_parameter(n, shard_parameter(n, a, rank, world, **kw))
    vl = V // world
    dev = torch.device("cuda", local_rank)
    lg = torch.empty(1, vl, dtype=torch.float32, device=dev)
    tin = torch.empty(1, dtype=torch.int32, device=dev)
    tout = torch.empty(1, dtype=torch.int32, device=dev)
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    prompt = oracle.randint(PARITY_PROMPT, PARITY_PROMPT_SEED, 0, V)
    errs_max, errs_sum, tok_ref, tok_gpu, gaps, fl_max, fl_mean = [], [], [], [], [], [], []
    cur = prompt[:1].copy()
    for t in range(PARITY_PROMPT + PARITY_STEPS):
        l_ref, n_ref = ref.step(cur)
        l_f32, _ = f32.step(cur)
        tin.copy_(torch.from_numpy(cur))
        _lib.call("rxla_b200_decoder_step", gpu.handle, ctypes.c_void_p(tin.data_ptr()), 1,
                  ctypes.c_void_p(tout.data_ptr()), ctypes.c_void_p(lg.data_ptr()), s)
        torch.cuda.synchronize()
        if t + 1 >= PARITY_PROMPT:  # last prompt row + the decode steps
            d = np.abs(lg.cpu().numpy()[0] - l_ref[0, rank * vl:(rank + 1) * vl])
            errs_max.append(float(d.max()))
            errs_sum.append(float(d.sum()))
            df = np.abs(l_f32[0] - l_ref[0])
            fl_max.append(float(df.max()))
            fl_mean.append(float(df.mean()))
            top2 = np.sort(l_ref[0])[-2:]
            gaps.append(float(top2[1] - top2[0]))
            tok_ref.append(int(n_ref[0]))
            tok_gpu.append(int(tout.cpu().item()))
            cur = n_ref.astype(np.int32)
        else:
            cur = prompt[t + 1:t + 2].copy()
    status = _lib.load().rxla_b200_device_status(0)
    gpu.close()
    ref.close()
    f32.close()
    mx, sm = max(errs_max), sum(errs_sum)
    floor_max, floor_mean = max(fl_max), float(np.mean(fl_mean))
    bar_max = max(PARITY_MAX_ABS, PARITY_FLOOR_MARGIN * floor_max)
    bar_mean = max(PARITY_MEAN_ABS, PARITY_FLOOR_MARGIN * floor_mean)
    if world > 1:
        t = torch.tensor([mx, sm, float(status != 0), float(tok_gpu != tok_ref)], device=dev,
                         dtype=torch.float64)
        u = t.clone()
        torch.distributed.all_reduce(t[:1], op=torch.distributed.ReduceOp.MAX)
        torch.distributed.all_reduce(u[1:], op=torch.distributed.ReduceOp.SUM)
        mx, sm = float(t[0]), float(u[1])
        bad_status, bad_tokens = float(u[2]) > 0, float(u[3]) > 0
    else:
        bad_status, bad_tokens = status != 0, tok_gpu != tok_ref
    mean = sm / (len(errs_sum) * V)
    ok = (mx <= bar_max and mean <= bar_mean and not bad_tokens and not bad_status
          and min(gaps) >= PARITY_MAX_ABS)
    return {"model": "2 layers, hidden 1024, 16 q / 8 kv heads, head_dim 64, intermediate 2048, "
                     "vocab 8192, W8 tied head", "tp": world,
            "window": f"last of {PARITY_PROMPT} prompt steps + {PARITY_STEPS} greedy steps",
            "max_abs": mx, "mean_abs": mean, "tokens_equal": not bad_tokens,
            "oracle_min_top2_gap": min(gaps), "device_status_ok": not bad_status,
            "north_star_bar": {"max_abs": PARITY_MAX_ABS, "mean_abs": PARITY_MEAN_ABS},
            "fp32_sum_floor": {"max_abs": floor_max, "mean_abs": floor_mean,
                               "what": "the oracle with fp32 instead of f64 running sums in its "
                                       "linears, against the f64 oracle"},
            "applied_bar": {"max_abs": bar_max, "mean_abs": bar_mean,
                            "rule": f"max(north star, {PARITY_FLOOR_MARGIN} x floor)"},
            "ok": bool(ok)}


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
    # N > 1: one 8B model sharded tensor-parallel over the N GPUs, the same
    # synthetic model at every N
    comm = None
    if world > 1:
        def share(data):
            obj = [data]
            torch.distributed.broadcast_object_list(obj, src=0)
            return obj[0]
        comm = Comm(rank, world, local_rank, share)
    # the 8B decoder first: the first decoder on a comm reserves the peer
    # all-reduce buffers, sized for its own batch x hidden (the parity model's
    # and config 5's all-reduces fit in them)
    dec = Decoder(**cfg, embedding_dtype="u8", max_batch=b64, max_context=max_ctx,
                  device=local_rank, comm=comm.handle if comm else None, tp_rank=rank,
                  tp_size=world)
    dec.init_synthetic(1234)
    parity = tp_parity(rank, world, local_rank, comm)
    tout = ctypes.c_void_p(dec.tokens_out_ptr)
    prompt = torch.randint(0, cfg["vocab"], (PROMPT,), dtype=torch.int32, device=dev,
                           generator=torch.Generator(device=dev).manual_seed(1))

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if world > 1:
            t = torch.tensor([v], device=dev, dtype=torch.float64)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            v = float(t.item())
        return v

    # ---- config-4 prefill of the 2048-token prompt (also fills the context
    # the decode steps run at)
    prefill = run_prefill_timed(args, dec, prompt, dev, stream, world) if world == 1 else None
    dec.reset(sptr)
    dec.prefill(0, prompt, stream=sptr)
    barrier()

    def greedy(batch, n):
        for _ in range(n):
            _lib.call("rxla_b200_decoder_step", dec.handle, tout, batch, tout, None, sptr)

    def timed(batch, n):
        greedy(batch, args.warmup)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        greedy(batch, n)
        e1.record(stream)
        barrier()
        return max_over_ranks(e0.elapsed_time(e1))

    sampler = ClockSampler(local_rank)
    # ---- batch 1 (headline)
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
    e2e_s = max_over_ranks(time.perf_counter() - t0)
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
                 "step_gbs": (w + kv) / (ms64 / n64 * 1e-3) / 1e9,
                 "step_frac_of_hbm": (w + kv) / world / (ms64 / n64 * 1e-3) / 1e9 / measured_peaks()[0]}
    clocks = sampler.stop()

    # ---- roofline of the dominant kernel: the W8 linears of one batch-1 step
    # of this rank's shard, the step's own instances, replayed in a graph
    roof = gemv_roofline(dec, cfg, dev, stream, lib, world, rank)
    status = lib.rxla_b200_device_status(0)
    dec.close()  # releases the captured graphs (they hold NCCL calls) before the comm
    res5 = None if args.no_config5 else run_config5(args, rank, world, local_rank, comm, barrier)
    kernels = None
    if world == 1 and not args.no_kernels:
        kernels = {"config2_linear_sweep": config2_sweep(dev),
                   "config3_attention": config3_attention(dev),
                   "gated_delta": gated_delta_bench(dev),
                   "qwen3_5_08b": qwen3_5_bench(dev)}
    if comm:
        comm.close()

    weights, kv1 = step_bytes(cfg, 1, ctx_b1)
    tok_s = args.steps / (ms1 / 1e3)  # one sequence, decoded by all N GPUs together
    out = {
        "metric": METRIC, "value": tok_s, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms1 / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "u8 weights, bf16 activations, fp32 accumulate",
        "data": "synthetic (seeded random W8 weights, random 2048-token prompt)",
        "config": workload_config(world),
        "step_gbs": (weights + kv1) / (ms1 / args.steps * 1e-3) / 1e9,
        "step_frac_of_hbm": (weights + kv1) / (ms1 / args.steps * 1e-3) / 1e9 / (world * measured_peaks()[0]),
        "parity": parity,
        "batch64": res64,
        "config5": res5,
        "prefill": prefill,
        "kernels": kernels,
        "e2e": {"value": args.steps / e2e_s, "unit": UNIT, "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": 4},
        "roofline": roof,
        "clocks": clocks,
        "gpu_launches": args.steps * launches_per_step(cfg, world),
        "device_status": status,
    }
    return out


def run_prefill_timed(args, dec, prompt, dev, stream, world):
    """Config-4 prefill of the PROMPT-token prompt through
    rxla_b200_decoder_prefill (chunks of rows on the tcgen05 GEMM, causal
    paged attention), from position 0 each time.  Tensor-bound: the roofline
    is the measured bf16 GEMM peak."""
    import torch
    s = ctypes.c_void_p(stream.cuda_stream)
    reps = 3
    for _ in range(2):
        dec.reset(s)
        dec.prefill(0, prompt, stream=s)
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    ev[0].record(stream)
    for _ in range(reps):
        dec.reset(s)
        dec.prefill(0, prompt, stream=s)
    ev[1].record(stream)
    torch.cuda.synchronize()
    ms = ev[0].elapsed_time(ev[1]) / reps
    # end to end: the prompt from pinned host memory, the token back to the host
    host_prompt = prompt.cpu().pin_memory()
    t0 = time.perf_counter()
    for _ in range(reps):
        dec.reset(s)
        prompt.copy_(host_prompt, non_blocking=True)
        tok = dec.prefill(0, prompt, stream=s)
        tok.cpu()
    e2e_s = (time.perf_counter() - t0) / reps
    flops = prefill_flops(CONFIG4, PROMPT)
    _, peak, peak_sus, how = measured_peaks()
    achieved = flops / (ms * 1e-3) / 1e12
    return {"workload": f"config4: {PROMPT}-token prompt, one sequence, prefill from position 0",
            "value": PROMPT / (ms * 1e-3), "unit": "tokens/s", "ms_per_prefill": ms, "reps": reps,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "peak_source": f"{how} (burst)",
                         "frac_of_sustained": achieved / peak_sus, "flops_per_prefill": flops},
            "e2e": {"value": PROMPT / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": PROMPT * 4,
                    "d2h_bytes_per_step": 4}}


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
    status = _lib.load().rxla_b200_device_status(0)
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


def gemv_roofline(dec, cfg, dev, stream, lib, tp=1, rank=0):
    """Time the W8 linears of one batch-1 decode step of this rank's shard as
    the step runs them, replayed as one CUDA graph: qkv and gate/up with the
    input RMSNorm fused (real norm weights, the evolving f32 residual h),
    o_proj and down_proj adding into h (tp 1) or storing f32 partials (tp > 1),
    the tied head with its norm fused (f32 logits; the step's head also picks
    the greedy token in its epilogue).

    Algorithmic bytes per launch = N·K weights + 4·N scales + x (2·K bf16 or
    4·K f32 for the norm's h) + the output; achieved = Σ bytes / Σ time."""
    import torch
    from rxla_b200 import _lib
    H, D = cfg["hidden"], cfg["head_dim"]
    I, V, hq = cfg["intermediate"] // tp, cfg["vocab"] // tp, cfg["q_heads"] // tp
    qkv_rows = (hq + 2 * cfg["kv_heads"] // tp) * D
    g = torch.Generator(device=dev).manual_seed(5)
    h = torch.randn(1, H, device=dev, generator=g)
    att = torch.randn(1, hq * D, device=dev, generator=g).bfloat16()
    act = torch.randn(1, I, device=dev, generator=g).bfloat16()
    qkv = torch.empty(1, qkv_rows, dtype=torch.bfloat16, device=dev)
    part = torch.zeros(1, H, dtype=torch.float32, device=dev)
    logits = torch.empty(1, V, dtype=torch.float32, device=dev)
    eps = ctypes.c_float(cfg["rms_eps"])
    calls, total_bytes = [], 0
    for l in range(cfg["layers"]):
        p = f"layers.{l}."
        ln1, _, _ = dec.parameter(p + "input_layernorm.weight")
        ln2, _, _ = dec.parameter(p + "post_attention_layernorm.weight")
        wqkv, _, _ = dec.parameter(p + "self_attn.qkv.weight")
        sqkv, _, _ = dec.parameter(p + "self_attn.qkv.scale")
        wo, _, _ = dec.parameter(p + "self_attn.o_proj.weight")
        so, _, _ = dec.parameter(p + "self_attn.o_proj.scale")
        wgu, _, _ = dec.parameter(p + "mlp.gate_up.weight")
        sgu, _, _ = dec.parameter(p + "mlp.gate_up.scale")
        wd, _, _ = dec.parameter(p + "mlp.down_proj.weight")
        sd, _, _ = dec.parameter(p + "mlp.down_proj.scale")
        res_ptr, res_epi = (h.data_ptr(), _lib.EPI_RESIDUAL_ADD) if tp == 1 else \
            (part.data_ptr(), _lib.EPI_STORE)
        calls.append(("norm", h.data_ptr(), ln1, wqkv, sqkv, H, qkv_rows, H, qkv.data_ptr(),
                      _lib.BF16, _lib.EPI_STORE))
        total_bytes += qkv_rows * H + 4 * qkv_rows + 4 * H + 2 * qkv_rows
        calls.append(("lin", att.data_ptr(), 0, wo, so, hq * D, H, hq * D, res_ptr, _lib.F32,
                      res_epi))
        total_bytes += H * hq * D + 4 * H + 2 * hq * D + (8 if tp == 1 else 4) * H
        calls.append(("norm", h.data_ptr(), ln2, wgu, sgu, H, I, H, act.data_ptr(), _lib.BF16,
                      _lib.EPI_SWIGLU))
        total_bytes += 2 * I * H + 8 * I + 4 * H + 2 * I
        calls.append(("lin", act.data_ptr(), 0, wd, sd, I, H, I, res_ptr, _lib.F32, res_epi))
        total_bytes += H * I + 4 * H + 2 * I + (8 if tp == 1 else 4) * H
    fn, _, _ = dec.parameter("norm.weight")
    we, _, _ = dec.parameter("embed_tokens.weight")
    se, _, _ = dec.parameter("embed_tokens.scale")
    calls.append(("norm", h.data_ptr(), fn, we + rank * V * H, se + rank * V * 4, H, V, H,
                  logits.data_ptr(), _lib.F32, _lib.EPI_STORE))
    total_bytes += V * H + 4 * V + 4 * H + 4 * V

    def run():
        s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        for kind, x, nw, w, sc, group, n, k, y, ydt, epi in calls:
            if kind == "norm":
                st = lib.rxla_b200_w8a16_norm_linear(x, nw, eps, w, sc, group, 1, n, k, y, ydt,
                                                     epi, s)
            else:
                st = lib.rxla_b200_w8a16_linear(x, _lib.BF16, w, sc, group, 1, n, k, y, ydt, epi, s)
            assert st == 0, _lib.load().rxla_b200_last_error_message()
    run()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        run()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    reps = 10
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    sec = e0.elapsed_time(e1) / 1e3 / reps
    peak, _, _, kind = measured_peaks()
    achieved = total_bytes / sec / 1e9
    del graph
    return {"bound": "hbm", "kernel": "w8_skinny_kernel (the W8 linears of one batch-1 step: "
                                      "fused-norm qkv / gate-up+SwiGLU / head, residual o / down)",
            "achieved": achieved, "peak": peak, "peak_kind": kind, "unit": "GB/s",
            "frac": achieved / peak, "traffic": total_bytes / len(calls) * TRAFFIC_RATIO,
            "traffic_note": TRAFFIC_NOTE, "launches": len(calls),
            "avg_launch_us": sec / len(calls) * 1e6, "bytes_per_step": total_bytes,
            "timing": "CUDA events around 10 replays of one graph of the step's linears"}


# DRAM bytes (read + write) per algorithmic byte of the W8 linears of a decode
# step, from the ncu capture without cache flushing summarised in
# profiles/w8_linear_dram_config4_b1.md (2-layer config-4-width decoder, the
# second of two steps: 946.5 MB over 1010.1 MB of algorithmic bytes; each
# kernel's count includes the next kernel's weights it pulls into L2)
TRAFFIC_RATIO = 946.5 / 1010.1
TRAFFIC_NOTE = ("per launch: algorithmic bytes x the measured DRAM / algorithmic ratio of the "
                "step's W8 linears (ncu, caches not flushed)")


def prefill_flops(cfg, tokens):
    """Algorithmic FLOPs of a prompt through the decoder: 2 per weight per row
    for every layer's linears, the causal attention (q·k and p·v, 4·Hq·D per
    key, row t seeing t + 1 keys), and the head for the last row only."""
    h, d, hq, hkv, i = cfg["hidden"], cfg["head_dim"], cfg["q_heads"], cfg["kv_heads"], cfg["intermediate"]
    per_layer = h * (hq + 2 * hkv) * d + hq * d * h + 2 * i * h + i * h
    lin = 2.0 * per_layer * cfg["layers"] * tokens
    att = 4.0 * hq * d * tokens * (tokens + 1) / 2 * cfg["layers"]
    return lin + att + 2.0 * cfg["vocab"] * h


def config2_sweep(dev):
    """BASELINE config 2 through rxla_b200_w8a16_linear_ws (the linear with a
    split-K workspace sized by rxla_b200_w8a16_linear_workspace_size; no
    workspace for the shapes that do not split): x bf16 N(0,1) [M,K], int8
    weights U{-127..127} stored +128 [N,K], f32 per-row scales U[1e-3,1e-2],
    bf16 out.  Each (N,K) cycles through enough weight copies to exceed 2x L2
    (126 MB) between launches; 3 warm-up launches, then 20 timed with CUDA
    events.  Algorithmic bytes N·K + 4·N + 2·M·K + 2·M·N, FLOPs 2·M·N·K;
    frac = max(t_mem, t_flop) at the measured peaks / measured time."""
    import torch
    hbm, tf, _, how = measured_peaks()
    g = torch.Generator(device=dev).manual_seed(2)
    points = []
    for n, k in ((4096, 4096), (12288, 4096), (4096, 12288), (6144, 4096)):
        copies = max(2, -(-2 * 126 * 2**20 // (n * k)))
        ws = [torch.randint(1, 256, (n, k), dtype=torch.uint8, device=dev, generator=g)
              for _ in range(copies)]
        sc = torch.rand(n, 1, device=dev, generator=g) * 9e-3 + 1e-3
        for m in (1, 8, 32, 128, 512, 2048):
            x = torch.randn(m, k, device=dev, generator=g).bfloat16()
            y = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
            s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
            from rxla_b200 import _lib, nn
            lib = _lib.load()
            wsb = nn.linear_workspace_size(m, n, k, k)
            wsp = torch.zeros(max(wsb, 16), dtype=torch.uint8, device=dev)

            def launch(i):
                st = lib.rxla_b200_w8a16_linear_ws(x.data_ptr(), _lib.BF16, ws[i % copies].data_ptr(),
                                                   sc.data_ptr(), k, m, n, k, y.data_ptr(), _lib.BF16,
                                                   _lib.EPI_STORE, wsp.data_ptr(), wsb, s)
                assert st == 0, _lib.load().rxla_b200_last_error_message()
            for i in range(3):
                launch(i)
            reps = 20
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for i in range(reps):
                launch(i)
            e1.record()
            torch.cuda.synchronize()
            sec = e0.elapsed_time(e1) / 1e3 / reps
            byt = n * k + 4 * n + 2 * m * k + 2 * m * n
            fl = 2.0 * m * n * k
            t_mem, t_flop = byt / (hbm * 1e9), fl / (tf * 1e12)
            points.append({"m": m, "n": n, "k": k, "workspace_bytes": wsb,
                           "us": sec * 1e6, "gbs": byt / sec / 1e9,
                           "tflops": fl / sec / 1e12,
                           "bound": "hbm" if t_mem >= t_flop else "tensor",
                           "frac": max(t_mem, t_flop) / sec})
            del x, y, wsp
        del ws
        torch.cuda.empty_cache()
    return {"points": points, "peaks": {"hbm_gbs": hbm, "bf16_tflops": tf, "source": how},
            "l2": "weight copies cycled, > 2x L2 between launches of one shape"}


def config3_attention(dev):
    """BASELINE config 3 through rxla_b200_paged_decode_attention: batch 64,
    32 q / 8 kv heads, head_dim 128, page 16, contexts U[512, 8192) (seeded),
    K/V/Q N(0,1) bf16, RoPE theta 1e6 on the new token, which is appended
    before attending.  Bytes = Σ_b (L_b + 1)·Hkv·D·2·2 (K and V) + q / out +
    the new K/V rows + the page table; ~1.1 GB per call, larger than L2."""
    import numpy as np
    import torch
    from rxla_b200 import nn
    batch, hq, hkv, d, max_ctx = 64, 32, 8, 128, 8192
    hbm, _, _, how = measured_peaks()
    g = torch.Generator(device=dev).manual_seed(3)
    cache = nn.PagedKvCache(batch=batch, kv_heads=hkv, head_dim=d, max_context=max_ctx + 16)
    cache.k.normal_(generator=g)
    cache.v.normal_(generator=g)
    lens = torch.randint(512, 8192, (batch,), dtype=torch.int32, device=dev, generator=g)
    cache.ctx_lens.copy_(lens)
    qkv = torch.randn(batch, (hq + 2 * hkv) * d, device=dev, generator=g).bfloat16()
    ws = torch.zeros(nn.paged_decode_workspace_size(batch, hq, hkv, d, cache.max_context),
                     dtype=torch.uint8, device=dev)
    inv = torch.from_numpy(nn.rope_inv_freq(1e6, d)).to(dev)

    def launch():
        nn.paged_decode_attention(qkv[:, :hq * d], qkv[:, hq * d:(hq + hkv) * d],
                                  qkv[:, (hq + hkv) * d:], cache, q_heads=hq, inv_freq=inv,
                                  rotary_dim=d, workspace=ws)
    for _ in range(3):
        launch()
    torch.cuda.synchronize()
    reps = 10
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        launch()
    e1.record()
    torch.cuda.synchronize()
    sec = e0.elapsed_time(e1) / 1e3 / reps
    L = lens.cpu().numpy().astype(np.int64)
    byt = int(((L + 1) * hkv * d * 2 * 2).sum() + 2 * batch * hq * d * 2 + batch * hkv * d * 2 * 2
              + cache.page_table.numel() * 4)
    return {"workload": "config3: batch 64, 32 q / 8 kv heads, head_dim 128, ctx U[512,8192)",
            "us": sec * 1e6, "bytes_per_call": byt, "gbs": byt / sec / 1e9, "bound": "hbm",
            "frac": byt / sec / 1e9 / hbm, "peak_gbs": hbm, "peak_source": how}


def gated_delta_bench(dev):
    """Qwen3.5-0.8B linear-attention mixer widths (16 heads of 128, conv 4)
    through rxla_b200_gated_delta (crates/rxla-models/src/qwen3_5/layers.rs:114-268).

    decode_b64: 64 sequences, one token each, continuing their states.  HBM
      bound: algorithmic bytes = the recurrent state read and written
      (64·16·128·128·4·2 = 134 MB) + the projections in, the conv history
      read and written, the bf16 output; two state sets are cycled (268 MB,
      > 2x L2) between timed calls.
    prefill_2048: one sequence, a 2048-token prompt from a zero state: the
      recurrence is sequential in the tokens (latency bound), reported as
      tokens/s and µs per token.
    layer_decode_b64: the whole mixer at batch 64 (fused W8 in-projection,
      the three kernels, W8 out_proj added into the residual)."""
    import torch
    from rxla_b200.gated_delta import (GatedDeltaAttention, GatedDeltaState, gated_delta,
                                       workspace_size)
    hbm, _, _, how = measured_peaks()
    H, D, K = 16, 128, 4
    W = H * D
    g = torch.Generator(device=dev).manual_seed(11)
    conv_w = torch.randn(3 * W, K, device=dev, generator=g) * 0.5
    a_log = torch.rand(H, device=dev, generator=g) * 2.7
    dt_bias = torch.randn(H, device=dev, generator=g) * 0.5
    norm_w = 1 + 0.1 * torch.randn(D, device=dev, generator=g)

    def timed(fn, reps):
        for i in range(3):
            fn(i)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(reps):
            fn(i)
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / 1e3 / reps

    out = {"workload": "Qwen3.5-0.8B linear-attention widths: 16 heads x 128, conv 4, hidden 1024"}
    # decode, batch 64
    B = 64
    proj = torch.randn(B, 4 * W + 2 * H, device=dev, generator=g).bfloat16()
    states = []
    for _ in range(2):
        st = GatedDeltaState(B, H, D, K, device=dev)
        st.state.normal_(generator=g).mul_(0.05)
        st.started = True
        states.append(st)
    y = torch.empty(B, W, dtype=torch.bfloat16, device=dev)
    ws = torch.empty(workspace_size(B, 1, H, D), dtype=torch.uint8, device=dev)

    def dec(i):
        gated_delta(proj[:, :3 * W], proj[:, 3 * W:4 * W], proj[:, 4 * W:4 * W + H],
                    proj[:, 4 * W + H:], conv_w, a_log, dt_bias, norm_w, state=states[i % 2],
                    out=y, workspace=ws)
    sec = timed(dec, 20)
    byt = B * H * D * D * 4 * 2 + B * (4 * W + 2 * H) * 2 + B * (K - 1) * 3 * W * 2 * 2 + B * W * 2
    out["decode_b64"] = {"us": sec * 1e6, "bytes_per_call": byt, "gbs": byt / sec / 1e9,
                         "bound": "hbm", "frac": byt / sec / 1e9 / hbm, "peak_gbs": hbm,
                         "peak_source": how, "launches_per_call": 3,
                         "l2": "two state sets cycled (268 MB > 2x L2)"}
    # prefill of one 2048-token sequence
    T = 2048
    proj = torch.randn(T, 4 * W + 2 * H, device=dev, generator=g).bfloat16()
    st = GatedDeltaState(1, H, D, K, device=dev)
    y = torch.empty(T, W, dtype=torch.bfloat16, device=dev)
    ws = torch.empty(workspace_size(1, T, H, D), dtype=torch.uint8, device=dev)

    def pre(i):
        st.started = False
        gated_delta(proj[:, :3 * W], proj[:, 3 * W:4 * W], proj[:, 4 * W:4 * W + H],
                    proj[:, 4 * W + H:], conv_w, a_log, dt_bias, norm_w, state=st, out=y,
                    workspace=ws)
    sec = timed(pre, 5)
    out["prefill_2048"] = {"us": sec * 1e6, "tokens_per_s": T / sec, "us_per_token": sec * 1e6 / T,
                           "bound": "latency (sequential recurrence over the tokens)"}
    # the whole mixer at batch 64 (W8 projections included)
    hidden, G = 1024, 128
    params = {}
    for name, (n, k) in {"in_proj_qkv": (3 * W, hidden), "in_proj_z": (W, hidden),
                         "in_proj_b": (H, hidden), "in_proj_a": (H, hidden),
                         "out_proj": (hidden, W)}.items():
        params[f"{name}.weight"] = torch.randint(1, 256, (n, k), dtype=torch.uint8, device=dev,
                                                 generator=g)
        params[f"{name}.scale"] = torch.rand(n, k // G, device=dev, generator=g) * 1e-3
    params.update({"conv1d.weight": conv_w.reshape(3 * W, 1, K), "A_log": a_log,
                   "dt_bias": dt_bias, "norm.weight": norm_w})
    layer = GatedDeltaAttention(params, hidden_size=hidden, linear_heads=H, linear_head_dim=D,
                                conv_kernel=K, quant_group_size=G)
    x = torch.randn(B, 1, hidden, device=dev, generator=g)
    res = torch.zeros(B, 1, hidden, device=dev)
    lst = [layer.new_state(B) for _ in range(2)]
    sec = timed(lambda i: layer.apply(x, lst[i % 2], residual=res), 20)
    wbytes = sum(params[f"{n}.weight"].numel() + params[f"{n}.scale"].numel() * 4
                 for n in GatedDeltaAttention.NAMES)
    lbyt = wbytes + byt
    out["layer_decode_b64"] = {"us": sec * 1e6, "bytes_per_call": lbyt, "gbs": lbyt / sec / 1e9,
                               "frac": lbyt / sec / 1e9 / hbm, "launches_per_call": 5}
    return out


def qwen3_5_bench(dev, steps: int = 32):
    """The Qwen3.5-0.8B-shaped hybrid model (crates/rxla-models/src/qwen3_5/
    mod.rs:57-85: 24 layers, every 4th full attention with 8 q / 2 kv heads of
    256 and rotary 64, the rest gated-delta with 16 heads of 128, hidden 1024,
    intermediate 3584, vocab 248320, W8 with 128-wide groups) with random
    weights through Qwen3_5Model: a 64-token prompt, then batch-1 decode steps
    each replayed as one CUDA graph; and a 16-token prompt from a fresh state
    as one graph (the sequence-16 forward the reference publishes).  Bytes per
    decode step: every W8 weight and scale once (the tied head included), the
    gated-delta states read and written, the KV rows of the full-attention
    layers."""
    import torch
    from rxla_b200.qwen3_5 import Qwen3_5Model
    hbm, _, _, how = measured_peaks()
    types = ["full" if (i + 1) % 4 == 0 else "linear" for i in range(24)]
    cfg = dict(vocabulary=248320, hidden_size=1024, intermediate_size=3584, layer_types=types,
               attention_heads=8, key_value_heads=2, head_dim=256, linear_heads=16,
               linear_head_dim=128, conv_kernel=4, rope_theta=1e7, rotary_dim=64, epsilon=1e-6,
               quant_group_size=128)
    g = torch.Generator(device=dev).manual_seed(21)
    H, I, G, V = 1024, 3584, 128, 248320
    params = {}

    def w8(name, n, k):
        params[name + ".weight"] = torch.randint(1, 256, (n, k), dtype=torch.uint8, device=dev,
                                                 generator=g)
        params[name + ".scale"] = torch.rand(n, k // G, device=dev, generator=g) * 2e-4

    def vec(name, n, scale=0.1):
        params[name] = torch.randn(n, device=dev, generator=g) * scale
    w8("embed_tokens", V, H)
    for i, kind in enumerate(types):
        pre = f"layers.{i}."
        vec(pre + "input_layernorm.weight", H)
        vec(pre + "post_attention_layernorm.weight", H)
        if kind == "linear":
            W = 16 * 128
            w8(pre + "linear_attn.in_proj_qkv", 3 * W, H)
            w8(pre + "linear_attn.in_proj_z", W, H)
            w8(pre + "linear_attn.in_proj_b", 16, H)
            w8(pre + "linear_attn.in_proj_a", 16, H)
            w8(pre + "linear_attn.out_proj", H, W)
            params[pre + "linear_attn.conv1d.weight"] = torch.randn(3 * W, 1, 4, device=dev,
                                                                    generator=g) * 0.5
            params[pre + "linear_attn.A_log"] = torch.rand(16, device=dev, generator=g) * 2.7
            vec(pre + "linear_attn.dt_bias", 16, 0.5)
            params[pre + "linear_attn.norm.weight"] = torch.ones(128, device=dev)
        else:
            w8(pre + "self_attn.q_proj", 2 * 8 * 256, H)
            w8(pre + "self_attn.k_proj", 2 * 256, H)
            w8(pre + "self_attn.v_proj", 2 * 256, H)
            w8(pre + "self_attn.o_proj", H, 8 * 256)
            vec(pre + "self_attn.q_norm.weight", 256)
            vec(pre + "self_attn.k_norm.weight", 256)
        w8(pre + "mlp.gate_proj", I, H)
        w8(pre + "mlp.up_proj", I, H)
        w8(pre + "mlp.down_proj", H, I)
    vec("norm.weight", H)
    wbytes = sum(t.numel() for n, t in params.items()
                 if n.endswith(".weight") and t.dtype == torch.uint8) + \
        sum(t.numel() * 4 for n, t in params.items() if n.endswith(".scale"))
    prompt = 64
    model = Qwen3_5Model(params, **cfg, batch=1, max_context=prompt + 3 + steps + 16)
    model.forward(torch.randint(0, V, (1, prompt), dtype=torch.int32, device=dev, generator=g))
    ids = torch.zeros(1, 1, dtype=torch.int32, device=dev)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):  # warm-up steps (also the state the graph starts from)
            model.forward(ids)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        model.forward(ids)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    sec = e0.elapsed_time(e1) / 1e3 / steps
    del graph
    # a 16-token prompt from a fresh state, one graph: the context lengths are
    # zeroed inside it and every gated-delta call starts from zero state
    p16 = torch.randint(0, V, (1, 16), dtype=torch.int32, device=dev, generator=g)
    caches = [m.cache for m in model.mixers if hasattr(m, "cache")]

    def fresh():
        for st in model.states:
            if st is not None:
                st.started = False
    fresh()
    with torch.cuda.stream(side):
        for c in caches:
            c.ctx_lens.zero_()
        model.forward(p16)
    torch.cuda.current_stream().wait_stream(side)
    fresh()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for c in caches:
            c.ctx_lens.zero_()
        model.forward(p16)
    torch.cuda.synchronize()
    reps = 10
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    sec16 = e0.elapsed_time(e1) / 1e3 / reps
    del graph
    ctx = prompt + 3 + steps // 2
    byt = wbytes + 18 * 16 * 128 * 128 * 4 * 2 + 6 * 2 * 256 * 2 * 2 * ctx
    return {"workload": "Qwen3.5-0.8B-shaped hybrid model (18 gated-delta + 6 full-attention "
                        "layers, vocab 248320), batch-1 decode after a 64-token prompt",
            "tokens_per_s": 1.0 / sec, "ms_per_step": sec * 1e3, "steps": steps,
            "bytes_per_step": byt, "gbs": byt / sec / 1e9, "frac": byt / sec / 1e9 / hbm,
            "peak_source": how, "timing": "CUDA events around graph replays of the whole step",
            "prompt16": {"ms": sec16 * 1e3, "tokens_per_s": 16 / sec16,
                         "what": "16-token prompt from a fresh state, one graph"},
            "l2": "0.8 GB of weights per step > L2"}


def profile_case(what: str):
    """Small, self-contained cases for ncu captures (no JSON line).

    gemv:      one W8 linear, N=32768 K=4096 M=1 (134 MB of weights > L2), 3 launches
    head:      the tied LM head of config 4, N=151936 K=4096 M=1 (622 MB), 3 launches
    gemm:      config-2 tensor-bound row, M=2048 N=4096 K=4096 on the tcgen05 GEMM, 3 launches
    step:      the config-4 decoder after a 256-token prompt, 2 decode steps inside
               the NVTX range "profile"
    step2l:    a 2-layer config-4-shaped decoder at batch 1, 256-token context, 2 steps
               inside "profile"
    step64:    config 4 at batch 64 (2048 context), 1 step inside "profile"
    step5:     config 5 (32B shape) at batch 32 (4096 context), 1 step inside "profile"
    gemmdec:   a 2-layer config-4-shaped decoder at batch 64, 1 step (the decode-batch
               GEMM launches: qkv, o, gate/up, down per layer, then the head)
    prefill:   a 2-layer config-4-shaped decoder, one 2048-token prompt (two
               1024-row chunks) after one warm-up prompt
    attention: config-3 paged decode attention (batch 64, 32 q / 8 kv heads, d 128,
               ctx ~U[512, 8192]), 3 launches
    attention1: the batch-1 decode attention of config 4 at a 2048-token context, 3 launches
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
    elif what == "step2l":
        # a 2-layer config-4-shaped decoder at batch 1 (256-token context),
        # 2 decode steps inside the NVTX range "profile" (~1 GB on the device)
        from rxla_b200.decoder import Decoder
        dec = Decoder(**dict(CONFIG4, layers=2), embedding_dtype="u8", max_batch=1, max_context=320)
        dec.init_synthetic(1)
        s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        dec.set_context_lengths([256], s)
        tout = ctypes.c_void_p(dec.tokens_out_ptr)
        for _ in range(3):
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
    elif what == "attention1":
        # the batch-1 decode attention of config 4 at a 2048-token context, 3 launches
        hq, hkv, d = 32, 8, 128
        cache = nn.PagedKvCache(batch=1, kv_heads=hkv, head_dim=d, max_context=PROMPT + 16)
        cache.k.normal_()
        cache.v.normal_()
        cache.ctx_lens.fill_(PROMPT)
        qkv = torch.randn(1, (hq + 2 * hkv) * d, device=dev).bfloat16()
        inv = torch.from_numpy(nn.rope_inv_freq(1e6, d)).to(dev)
        for _ in range(3):
            nn.paged_decode_attention(qkv[:, :hq * d], qkv[:, hq * d:(hq + hkv) * d],
                                      qkv[:, (hq + hkv) * d:], cache, q_heads=hq, inv_freq=inv,
                                      rotary_dim=d)
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
    elif what in ("gdn_decode", "gdn_prefill"):
        # the gated-delta mixer at the Qwen3.5-0.8B widths: 64 sequences x 1
        # token (state 134 MB > L2) or one 2048-token prompt; 3 calls
        from rxla_b200.gated_delta import GatedDeltaState, gated_delta
        H, D, K = 16, 128, 4
        W = H * D
        B, T = (64, 1) if what == "gdn_decode" else (1, 2048)
        proj = torch.randn(B * T, 4 * W + 2 * H, device=dev).bfloat16()
        st = GatedDeltaState(B, H, D, K, device=dev)
        st.state.normal_().mul_(0.05)
        args = (proj[:, :3 * W], proj[:, 3 * W:4 * W], proj[:, 4 * W:4 * W + H],
                proj[:, 4 * W + H:], torch.randn(3 * W, K, device=dev) * 0.5,
                torch.rand(H, device=dev) * 2.7, torch.randn(H, device=dev) * 0.5,
                torch.ones(D, device=dev))
        for _ in range(3):
            st.started = what == "gdn_decode"
            gated_delta(*args, state=st)
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
    ap.add_argument("--no-kernels", action="store_true",
                    help="skip the config-2 sweep, config-3 attention and gated-delta keys (N = 1)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile", choices=["gemv", "head", "gemm", "gemmdec", "step", "step2l", "step64",
                                          "step5", "prefill", "attention", "attention1", "gdn_decode",
                                          "gdn_prefill"], default=None,
                    help="run a small case for an ncu capture instead of the benchmark")
    args = ap.parse_args()
    if args.profile:
        profile_case(args.profile)
        return
    args.warmup = max(args.warmup, 3)

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
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                "impl": "reference", "scaling": "strong", "vs_baseline": None,
                "dtype": "u8 weights, f32 activations (CPU restatement)",
                "data": "synthetic (seeded random W8 weights, 2048-token context)",
                "config": workload_config(world),
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
    if not out["parity"]["ok"]:
        sys.stderr.write(f"tensor-parallel parity failed: {json.dumps(out['parity'])}\n")
        sys.exit(1)


if __name__ == "__main__":
    main()
