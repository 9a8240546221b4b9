"""Tensor-parallel decoding on two GPUs against the single-process oracle,
and the one-shot peer all-reduce against the rank-order sum.

Two ranks (one process per GPU) run the tiny W8 decoder at tp_size 2 over an
NCCL communicator: each holds its heads, its intermediate slice and its vocab
slice of the tied head, with the parameters sliced from the oracle's full
model by ``shard_parameter``.  Each rank's logits slice and the greedy tokens
(argmax over both slices) are compared with the oracle's full model.
Skipped with fewer than two GPUs.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

TINY = dict(layers=2, hidden=512, q_heads=8, kv_heads=2, head_dim=64, intermediate=1536,
            vocab=4096)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, batch, q):
    import ctypes
    import torch.distributed as dist

    import oracle
    from rxla_b200 import _lib
    from rxla_b200.decoder import Comm, Decoder, shard_parameter
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world)

        def share(data):
            obj = [data]
            dist.broadcast_object_list(obj, src=0)
            return obj[0]

        comm = Comm(rank, world, rank, share)
        ref = oracle.Decoder(**TINY, embedding_bf16=False, group_size=0, max_batch=batch,
                             max_context=64)
        ref.init_synthetic(9)
        gpu = Decoder(**TINY, embedding_dtype="u8", max_batch=batch, max_context=64, device=rank,
                      comm=comm.handle, tp_rank=rank, tp_size=world)
        H, D, I = TINY["hidden"], TINY["head_dim"], TINY["intermediate"]
        rows = {"q_proj": TINY["q_heads"] * D, "k_proj": TINY["kv_heads"] * D,
                "v_proj": TINY["kv_heads"] * D, "o_proj": H, "gate_proj": I, "up_proj": I,
                "down_proj": H}
        names = ["embed_tokens.weight", "embed_tokens.scale", "norm.weight"]
        for i in range(TINY["layers"]):
            p = f"layers.{i}."
            names += [p + "input_layernorm.weight", p + "post_attention_layernorm.weight",
                      p + "self_attn.q_norm.weight", p + "self_attn.k_norm.weight"]
            names += [f"{p}self_attn.{pr}.{k}" for pr in ("q_proj", "k_proj", "v_proj", "o_proj")
                      for k in ("weight", "scale")]
            names += [f"{p}mlp.{pr}.{k}" for pr in ("gate_proj", "up_proj", "down_proj")
                      for k in ("weight", "scale")]
        kw = dict(q_heads=TINY["q_heads"], kv_heads=TINY["kv_heads"], head_dim=D, intermediate=I,
                  hidden=H, vocab=TINY["vocab"])
        for n in names:
            a = np.array(ref.parameter(n))
            for pr, r in rows.items():
                if f".{pr}." in n:
                    a = a.reshape(r, -1)
            gpu.set_parameter(n, shard_parameter(n, a, rank, world, **kw))

        V, vl = TINY["vocab"], TINY["vocab"] // world
        prompt = oracle.randint(batch * 12, 21, 0, V).reshape(batch, 12)
        lg = torch.empty(batch, vl, dtype=torch.float32, device="cuda")
        tok_in = torch.empty(batch, dtype=torch.int32, device="cuda")
        tok_out = torch.empty(batch, dtype=torch.int32, device="cuda")
        s = torch.cuda.current_stream().cuda_stream
        cur = prompt[:, 0].copy()
        emax, flips, gaps, steps = 0.0, 0, [], 8
        for t in range(prompt.shape[1] + steps):
            l_ref, n_ref = ref.step(cur)
            tok_in.copy_(torch.from_numpy(cur))
            _lib.call("rxla_b200_decoder_step", gpu.handle, ctypes.c_void_p(tok_in.data_ptr()),
                      batch, ctypes.c_void_p(tok_out.data_ptr()), ctypes.c_void_p(lg.data_ptr()),
                      ctypes.c_void_p(s))
            torch.cuda.synchronize()
            err = float(np.abs(lg.cpu().numpy() - l_ref[:, rank * vl:(rank + 1) * vl]).max())
            emax = max(emax, err)
            if t + 1 >= prompt.shape[1]:
                got = tok_out.cpu().numpy()
                top2 = np.sort(l_ref, axis=1)[:, -2:]
                for b in range(batch):
                    if got[b] != n_ref[b]:
                        flips += 1
                        gaps.append(float(top2[b, 1] - top2[b, 0]))
                cur = n_ref
            else:
                cur = prompt[:, t + 1].copy()
        gpu.close()  # releases the captured graphs (they hold NCCL calls) before the comm
        comm.close()
        ref.close()
        dist.destroy_process_group()
        q.put((rank, emax, flips, gaps, None))
    except Exception as e:
        q.put((rank, None, None, None, repr(e)))


@pytest.mark.parametrize("batch", [2, 12])
def test_tp2_decoder_matches_oracle(batch):
    if torch.cuda.device_count() < 2:
        pytest.skip("tensor-parallel test needs two GPUs")
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, batch, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, emax, flips, gaps, err in results:
        assert err is None, f"rank {rank}: {err}"
        print(f"rank {rank}: logits max-abs {emax:.4g}, greedy flips {flips} (oracle gaps {gaps})")
        assert emax <= 2e-2
        assert all(g <= 2 * emax for g in gaps), "a greedy flip away from a near-tie"


def _p2p_main(rank, world, port, q):
    import ctypes
    import torch.distributed as dist

    from rxla_b200 import _lib
    from rxla_b200.decoder import Comm
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world)

        def share(data):
            obj = [data]
            dist.broadcast_object_list(obj, src=0)
            return obj[0]

        comm = Comm(rank, world, rank, share)
        cap = 64 * 4096
        _lib.call("rxla_b200_comm_p2p_enable", comm.handle, cap)
        s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        worst = 0.0
        # counts: one row, a ragged (non-float4) count, several CTAs, the capacity
        for it, count in enumerate([4096, 5, 2048 * 3 + 4, cap, 4096, 1]):
            for residual in (False, True):
                parts = [np.random.default_rng(100 * it + r).standard_normal(count).astype(np.float32)
                         for r in range(world)]
                total = parts[0].copy()
                for r in range(1, world):
                    total = total + parts[r]  # rank order, f32
                h0 = np.random.default_rng(7 + it).standard_normal(count).astype(np.float32)
                part = torch.from_numpy(parts[rank]).cuda()
                h = torch.from_numpy(h0).cuda()
                _lib.call("rxla_b200_p2p_allreduce_f32", comm.handle,
                          ctypes.c_void_p(part.data_ptr()),
                          ctypes.c_void_p(h.data_ptr()) if residual else None, count, s)
                torch.cuda.synchronize()
                if residual:  # h += bf16(sum), round to nearest even
                    want = h0 + torch.from_numpy(total).bfloat16().float().numpy()
                    got = h.cpu().numpy()
                else:
                    want, got = total, part.cpu().numpy()
                worst = max(worst, float(np.abs(got - want).max()))
        status = _lib.load().rxla_b200_device_status(1)
        comm.close()
        dist.destroy_process_group()
        q.put((rank, worst, status, None))
    except Exception as e:
        q.put((rank, None, None, repr(e)))


def test_p2p_allreduce_matches_rank_order_sum():
    """One-shot NVLink all-reduce (IPC-mapped peer buffers, bounded flag
    waits): store mode equals the f32 rank-order sum bit for bit; residual
    mode adds its bf16 rounding to the residual; several calls in a row
    exercise the alternating slots and the per-CTA epochs."""
    if torch.cuda.device_count() < 2:
        pytest.skip("peer all-reduce test needs two GPUs")
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_p2p_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, worst, status, err in results:
        assert err is None, f"rank {rank}: {err}"
        assert status == 0, f"rank {rank}: device status {status}"
        assert worst == 0.0, f"rank {rank}: max deviation {worst}"


def _rank_prefill_main(rank, world, port, path, q):
    import ctypes
    import torch.distributed as dist

    import oracle
    from rxla_b200 import _lib
    from rxla_b200.decoder import Comm, Decoder
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world)

        def share(data):
            obj = [data]
            dist.broadcast_object_list(obj, src=0)
            return obj[0]

        comm = Comm(rank, world, rank, share)
        ref = oracle.Decoder(**TINY, embedding_bf16=False, group_size=0, max_batch=1,
                             max_context=64)
        ref.init_synthetic(9)
        gpu = Decoder(**TINY, embedding_dtype="u8", max_batch=1, max_context=64, device=rank,
                      comm=comm.handle, tp_rank=rank, tp_size=world)
        loaded, skipped = gpu.load_safetensors(path)
        V, vl = TINY["vocab"], TINY["vocab"] // world
        prompt = oracle.randint(40, 31, 0, V)
        lg = torch.empty(vl, dtype=torch.float32, device="cuda")
        tok = gpu.prefill(0, prompt, logits_ptr=ctypes.c_void_p(lg.data_ptr()))
        torch.cuda.synchronize()
        for t in prompt:
            l_ref, n_ref = ref.step(np.array([t], np.int32))
        errs = [float(np.abs(lg.cpu().numpy() - l_ref[0, rank * vl:(rank + 1) * vl]).max())]
        top2 = np.sort(l_ref[0])[-2:]
        flip_ok = int(tok.item()) == int(n_ref[0]) or top2[1] - top2[0] <= 2 * max(errs)
        # decode from the prefilled cache (teacher forcing)
        lgb = torch.empty(1, vl, dtype=torch.float32, device="cuda")
        tin = torch.empty(1, dtype=torch.int32, device="cuda")
        tout = torch.empty(1, dtype=torch.int32, device="cuda")
        s = torch.cuda.current_stream().cuda_stream
        cur = n_ref.astype(np.int32)
        for _ in range(6):
            l_ref, n_ref = ref.step(cur)
            tin.copy_(torch.from_numpy(cur))
            _lib.call("rxla_b200_decoder_step", gpu.handle, ctypes.c_void_p(tin.data_ptr()), 1,
                      ctypes.c_void_p(tout.data_ptr()), ctypes.c_void_p(lgb.data_ptr()),
                      ctypes.c_void_p(s))
            torch.cuda.synchronize()
            errs.append(float(np.abs(lgb.cpu().numpy() - l_ref[:, rank * vl:(rank + 1) * vl]).max()))
            cur = n_ref.astype(np.int32)
        gpu.close()
        comm.close()
        ref.close()
        dist.destroy_process_group()
        q.put((rank, (loaded, skipped), errs, flip_ok, None))
    except Exception as e:
        q.put((rank, None, None, None, repr(e)))


def test_tp2_checkpoint_load_and_prefill(tmp_path):
    """Two ranks load their slices of one full W8 checkpoint
    (rxla_b200_decoder_load_safetensors), prefill a 40-token prompt (the
    row-parallel partial sums all-reduced over NCCL) and decode from the
    prefilled cache; each rank's logits slice against the oracle."""
    if torch.cuda.device_count() < 2:
        pytest.skip("tensor-parallel test needs two GPUs")
    import oracle
    from rxla_b200.checkpoint import save_file
    ref = oracle.Decoder(**TINY, embedding_bf16=False, group_size=0, max_batch=1, max_context=64)
    ref.init_synthetic(9)
    H, D, I = TINY["hidden"], TINY["head_dim"], TINY["intermediate"]
    rows = {"q_proj": TINY["q_heads"] * D, "k_proj": TINY["kv_heads"] * D,
            "v_proj": TINY["kv_heads"] * D, "o_proj": H, "gate_proj": I, "up_proj": I,
            "down_proj": H, "embed_tokens": TINY["vocab"]}
    names = ["embed_tokens.weight", "embed_tokens.scale", "norm.weight"]
    for i in range(TINY["layers"]):
        p = f"layers.{i}."
        names += [p + "input_layernorm.weight", p + "post_attention_layernorm.weight",
                  p + "self_attn.q_norm.weight", p + "self_attn.k_norm.weight"]
        names += [f"{p}self_attn.{pr}.{k}" for pr in ("q_proj", "k_proj", "v_proj", "o_proj")
                  for k in ("weight", "scale")]
        names += [f"{p}mlp.{pr}.{k}" for pr in ("gate_proj", "up_proj", "down_proj")
                  for k in ("weight", "scale")]
    tensors = {}
    for n in names:
        a = np.array(ref.parameter(n))
        for pr, r in rows.items():
            if n.startswith(pr) or f".{pr}." in n:
                a = a.reshape(r, -1)
        tensors["model.language_model." + n] = a
    ref.close()
    path = str(tmp_path / "tp.safetensors")
    save_file(path, tensors, metadata={"format": "rxla-qwen3.5-w8-v1"})
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_prefill_main, args=(r, world, port, path, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, counts, errs, flip_ok, err in results:
        assert err is None, f"rank {rank}: {err}"
        print(f"rank {rank}: loaded/skipped {counts}, logits max-abs per step {errs}")
        assert counts == (len(names), 0)
        assert max(errs) <= 2e-2
        assert flip_ok


def _spawn(target, world, *args):
    """Run `target(rank, world, port, *args, q)` in `world` spawned processes
    (NVLS off, as every multi-rank failure test here runs) and collect one
    result per rank."""
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    old = os.environ.get("NCCL_NVLS_ENABLE")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        procs = [ctx.Process(target=target, args=(r, world, port, *args, q)) for r in range(world)]
        for p in procs:
            p.start()
        results = [q.get(timeout=300) for _ in range(world)]
        for p in procs:
            p.join(timeout=60)
    finally:
        if old is None:
            del os.environ["NCCL_NVLS_ENABLE"]
        else:
            os.environ["NCCL_NVLS_ENABLE"] = old
    return sorted(results, key=lambda r: r[0])


def _comm_for(rank, world, port):
    import torch.distributed as dist
    from rxla_b200.decoder import Comm
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)

    def share(data):
        obj = [data]
        dist.broadcast_object_list(obj, src=0)
        return obj[0]

    return Comm(rank, world, rank, share)


def _p2p_setup_fail_main(rank, world, port, q):
    import ctypes
    import torch.distributed as dist
    from rxla_b200 import _lib
    try:
        comm = _comm_for(rank, world, port)
        lib = _lib.load()
        # rank 1 asks for a buffer no GPU holds (its cudaMalloc fails); rank 0
        # for an ordinary one.  Both must come back with an error, having run
        # the same collectives, and neither may keep the buffers.
        first = lib.rxla_b200_comm_p2p_enable(comm.handle, (1 << 36) if rank == 1 else 4096)
        msg = lib.rxla_b200_last_error_message().decode()
        # the communicator still works: an NCCL all-reduce, then a successful
        # enable and one peer all-reduce on every rank
        t = torch.full((16,), float(rank + 1), device="cuda")
        _lib.call("rxla_b200_allreduce", comm.handle, ctypes.c_void_p(t.data_ptr()), 16, _lib.F32,
                  ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        nccl_ok = bool((t == float(sum(range(1, world + 1)))).all())
        second = lib.rxla_b200_comm_p2p_enable(comm.handle, 4096)
        part = torch.full((4096,), float(rank + 1), device="cuda")
        _lib.call("rxla_b200_p2p_allreduce_f32", comm.handle, ctypes.c_void_p(part.data_ptr()),
                  None, 4096, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        p2p_ok = bool((part == float(sum(range(1, world + 1)))).all())
        status = lib.rxla_b200_device_status(1)
        comm.close()
        dist.destroy_process_group()
        q.put((rank, first, msg, nccl_ok, second, p2p_ok, status, None))
    except Exception as e:
        q.put((rank, None, None, None, None, None, None, repr(e)))


def test_p2p_enable_when_one_rank_fails():
    """rxla_b200_comm_p2p_enable when one rank's own set-up fails: every rank
    still runs the same collectives (handle all-gather, agreement), so none is
    left waiting; every rank reports an error and keeps no peer buffers, and
    the communicator stays usable (NCCL all-reduce, a later enable and a peer
    all-reduce succeed)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from rxla_b200 import _lib
    for rank, first, msg, nccl_ok, second, p2p_ok, status, err in _spawn(_p2p_setup_fail_main, 2):
        assert err is None, f"rank {rank}: {err}"
        print(f"rank {rank}: first enable {first} ({msg})")
        assert first != _lib.OK, f"rank {rank}: enable should fail when a peer failed"
        assert nccl_ok and second == _lib.OK and p2p_ok and status == 0, f"rank {rank}"


def _wait_timeout_main(rank, world, port, q):
    import ctypes
    import time as _time
    import torch.distributed as dist
    from rxla_b200 import _lib
    try:
        comm = _comm_for(rank, world, port)
        lib = _lib.load()
        _lib.call("rxla_b200_comm_p2p_enable", comm.handle, 4096)
        s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        part = torch.ones(4096, device="cuda")
        _lib.call("rxla_b200_p2p_allreduce_f32", comm.handle, ctypes.c_void_p(part.data_ptr()),
                  None, 4096, s)  # both ranks: an ordinary all-reduce first
        torch.cuda.synchronize()
        before = lib.rxla_b200_device_status(0)
        waited, status, answers = 0.0, 0, False
        if rank == 0:
            # rank 1 never joins this one: rank 0's flag waits must give up
            # after the 50 ms budget and the kernel return
            _lib.call("rxla_b200_set_wait_timeout", 50_000_000)
            t0 = _time.perf_counter()
            _lib.call("rxla_b200_p2p_allreduce_f32", comm.handle, ctypes.c_void_p(part.data_ptr()),
                      None, 4096, s)
            torch.cuda.synchronize()
            waited = _time.perf_counter() - t0
            status = lib.rxla_b200_device_status(1)  # read and clear
            x = torch.arange(1024, device="cuda", dtype=torch.float32)
            answers = float((x * 2).sum().item()) == float(1023 * 1024)  # the GPU still runs work
            _lib.call("rxla_b200_set_wait_timeout", 4_000_000_000)
        dist.barrier()  # rank 1 leaves its step only here, with nothing in flight
        comm.close()
        dist.destroy_process_group()
        q.put((rank, before, waited, status, answers, None))
    except Exception as e:
        q.put((rank, None, None, None, None, repr(e)))


def test_bounded_wait_runs_out_and_reports_deadline_exceeded():
    """The failure path of the bounded device waits, made on the host: rank 1
    skips a peer all-reduce that rank 0 enters.  With the wait budget set to
    50 ms (rxla_b200_set_wait_timeout), rank 0's kernel gives up, records
    RXLA_B200_DEADLINE_EXCEEDED in the device status word and returns; the
    GPU keeps running work and the communicator is torn down collectively."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from rxla_b200 import _lib
    res = _spawn(_wait_timeout_main, 2)
    for rank, before, waited, status, answers, err in res:
        assert err is None, f"rank {rank}: {err}"
        assert before == 0
    rank, before, waited, status, answers, err = res[0]
    print(f"rank 0: waited {waited * 1e3:.1f} ms, status {status}")
    assert status == _lib.DEADLINE_EXCEEDED
    assert 0.04 <= waited < 2.0
    assert answers
