"""Tensor-parallel host logic on CPU ranks (gloo, world size 2).

The decoder's tensor parallelism (Megatron split: q/k/v and gate/up by output
rows, o_proj / down_proj by input columns with an f32 all-reduce, the tied
head by vocab slice with a cross-rank argmax) is checked here without a GPU:

* the shard helper's slices reassemble every full parameter of the oracle's
  tiny decoder, and match the C++ shard sizes;
* row-parallel partial sums, all-reduced over gloo, equal the full product;
* the argmax merge rule (each rank's best (value, global index), then highest
  value / lowest index over ranks) equals a full argmax, ties included.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from rxla_b200.decoder import shard_parameter

TINY = dict(layers=2, hidden=512, q_heads=8, kv_heads=2, head_dim=64, intermediate=1536,
            vocab=4096)
SHARD_KW = dict(q_heads=8, kv_heads=2, head_dim=64, intermediate=1536, hidden=512, vocab=4096)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _full_params(group_size=0):
    ref = oracle.Decoder(**TINY, embedding_bf16=False, group_size=group_size, max_batch=1,
                         max_context=16)
    ref.init_synthetic(5)
    names = ["embed_tokens.weight", "embed_tokens.scale", "norm.weight"]
    for i in range(TINY["layers"]):
        p = f"layers.{i}."
        names += [p + "input_layernorm.weight", p + "post_attention_layernorm.weight",
                  p + "self_attn.q_norm.weight", p + "self_attn.k_norm.weight"]
        for proj in ("q_proj", "k_proj", "v_proj", "o_proj"):
            names += [f"{p}self_attn.{proj}.weight", f"{p}self_attn.{proj}.scale"]
        for proj in ("gate_proj", "up_proj", "down_proj"):
            names += [f"{p}mlp.{proj}.weight", f"{p}mlp.{proj}.scale"]
    out = {n: np.array(ref.parameter(n)) for n in names}
    ref.close()
    return out


def _reshape(name, a):
    """2-D views of the oracle's flat parameters: weights [rows, k], scales [rows, groups]."""
    H, D, I = TINY["hidden"], TINY["head_dim"], TINY["intermediate"]
    rows = {"q_proj": TINY["q_heads"] * D, "k_proj": TINY["kv_heads"] * D,
            "v_proj": TINY["kv_heads"] * D, "o_proj": H, "gate_proj": I, "up_proj": I,
            "down_proj": H}
    for proj, r in rows.items():
        if f".{proj}." in name:
            return a.reshape(r, -1)
    return a


@pytest.mark.parametrize("group", [0, 64])
def test_shards_reassemble_full_parameters(group):
    full = _full_params(group)
    tp = 2
    for name, a in full.items():
        a2 = _reshape(name, a)
        shards = [shard_parameter(name, a2, r, tp, **SHARD_KW) for r in range(tp)]
        if any(k in name for k in ("q_proj", "k_proj", "v_proj", "gate_proj", "up_proj")):
            np.testing.assert_array_equal(np.concatenate(shards, 0), a2)
            assert shards[0].shape[0] * tp == a2.shape[0]
        elif name.endswith(("o_proj.weight", "down_proj.weight")):
            np.testing.assert_array_equal(np.concatenate(shards, 1), a2)
        elif name.endswith(("o_proj.scale", "down_proj.scale")) and a2.shape[1] > 1:
            np.testing.assert_array_equal(np.concatenate(shards, 1), a2)
        else:  # replicated (norms, embeddings, per-channel row-parallel scales)
            for sh in shards:
                np.testing.assert_array_equal(sh, a2)


def _rank_main(rank, world, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        rng = np.random.default_rng(11)
        # row-parallel o_proj: x [B, Hq*D] (this rank's heads), W [H, Hq*D] (its columns)
        B, H, QD = 3, 512, 512
        x = rng.standard_normal((B, QD))
        W = rng.standard_normal((H, QD))
        full = x @ W.T
        Ws = shard_parameter("layers.0.self_attn.o_proj.weight", W, rank, world, **SHARD_KW)
        n = QD // world
        part = torch.from_numpy(x[:, rank * n:(rank + 1) * n] @ Ws.T)
        dist.all_reduce(part)
        err = float(np.abs(part.numpy() - full).max())
        # argmax over vocab slices, with planted cross-shard ties
        V = 4096
        logits = rng.standard_normal((4, V)).astype(np.float32)
        logits[0, 5] = logits[0, V // 2 + 7] = 9.0        # tie across ranks: lowest index wins
        logits[1, V // 2 + 1] = logits[1, V // 2 + 3] = 9.0  # tie inside rank 1
        logits[2, :] = -1.0                                # all equal
        vl = V // world
        sl = logits[:, rank * vl:(rank + 1) * vl]
        cv = sl.max(1)
        ci = sl.argmax(1) + rank * vl  # numpy argmax: first maximum, as the kernel's rule
        cand = torch.from_numpy(np.stack([cv, ci.astype(np.float32)], 1))
        gathered = [torch.zeros_like(cand) for _ in range(world)]
        dist.all_gather(gathered, cand)
        merged = []
        for b in range(4):
            best, idx = -np.inf, 2 ** 31 - 1
            for r in range(world):
                v, i = float(gathered[r][b, 0]), int(gathered[r][b, 1])
                if v > best or (v == best and i < idx):
                    best, idx = v, i
            merged.append(idx)
        ok_argmax = merged == logits.argmax(1).tolist()
        dist.destroy_process_group()
        q.put((rank, err, ok_argmax))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e), False))


def test_row_parallel_allreduce_and_argmax_merge_gloo():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, err, ok in results:
        assert not isinstance(err, str), err
        assert err < 1e-9, f"rank {rank}: row-parallel all-reduce error {err}"
        assert ok, f"rank {rank}: argmax merge differs from the full argmax"
