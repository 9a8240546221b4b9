"""Decoder runner: the W8 Qwen3-style decoder of librxla_b200 (rxla_b200_decoder_*).

Mirrors the reference's model surface for this path: parameters are named as
in the checkpoint (``layers.{i}.self_attn.q_proj.weight`` ...), a step is
``BoundModel::run`` (crates/rxla-nn/src/applied.rs:222-237) / ``Session::run``
(crates/rxla-core/src/state.rs:1200-1228) with the KV cache as session state
owned by the runner.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib

_NP = {_lib.F32: np.float32, _lib.BF16: np.uint16, _lib.U8: np.uint8, _lib.I32: np.int32}


class Decoder:
    def __init__(self, *, layers, hidden, q_heads, kv_heads, head_dim, intermediate, vocab,
                 rms_eps=1e-6, rope_theta=1e6, embedding_dtype="u8", group_size=0,
                 max_batch=1, max_context=4096, device=0, comm=None, tp_rank=0, tp_size=1):
        cfg = _lib.DecoderConfig()
        cfg.struct_size = ctypes.sizeof(_lib.DecoderConfig)
        cfg.layers, cfg.hidden, cfg.q_heads, cfg.kv_heads = layers, hidden, q_heads, kv_heads
        cfg.head_dim, cfg.intermediate, cfg.vocab = head_dim, intermediate, vocab
        cfg.rms_eps, cfg.rope_theta = rms_eps, rope_theta
        cfg.embedding_dtype = {"u8": _lib.U8, "bf16": _lib.BF16}[embedding_dtype]
        cfg.group_size = group_size
        cfg.max_batch, cfg.max_context = max_batch, max_context
        cfg.tp_rank, cfg.tp_size = tp_rank, tp_size
        self.cfg = cfg
        self.vocab = vocab
        self.max_batch = max_batch
        self._device = device
        h = ctypes.c_void_p()
        _lib.call("rxla_b200_decoder_create", ctypes.byref(cfg), device, comm, ctypes.byref(h))
        self._h = h
        tin, tout, lg = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
        _lib.call("rxla_b200_decoder_io", h, ctypes.byref(tin), ctypes.byref(tout), ctypes.byref(lg))
        self.tokens_in_ptr, self.tokens_out_ptr, self.logits_ptr = tin.value, tout.value, lg.value
        self._in_host = np.zeros(max_batch, np.int32)
        self._out_host = np.zeros(max_batch, np.int32)

    @property
    def handle(self):
        return self._h

    def close(self):
        if self._h:
            _lib.load().rxla_b200_decoder_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def parameter(self, name: str):
        """(device pointer, bytes, dtype code) of a named parameter of this shard."""
        ptr, n, dt = ctypes.c_void_p(), ctypes.c_int64(), ctypes.c_int32()
        _lib.call("rxla_b200_decoder_parameter", self._h, name.encode(), ctypes.byref(ptr),
                  ctypes.byref(n), ctypes.byref(dt))
        return ptr.value, n.value, dt.value

    def set_parameter(self, name: str, host: np.ndarray):
        host = np.ascontiguousarray(host)
        _lib.call("rxla_b200_decoder_set_parameter", self._h, name.encode(),
                  host.ctypes.data_as(ctypes.c_void_p), host.nbytes)

    def load(self, params: dict):
        for name, value in params.items():
            self.set_parameter(name, value)

    def kv_cache(self, layer: int):
        """(k_ptr, v_ptr, bytes) of one layer's paged bf16 cache."""
        k, v, n = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_int64()
        _lib.call("rxla_b200_decoder_kv_cache", self._h, layer, ctypes.byref(k), ctypes.byref(v),
                  ctypes.byref(n))
        return k.value, v.value, n.value

    def init_synthetic(self, seed: int):
        _lib.call("rxla_b200_decoder_init_synthetic", self._h, seed)

    def reset(self, stream=None):
        _lib.call("rxla_b200_decoder_reset", self._h, stream)

    def set_context_lengths(self, lens, stream=None):
        """Context length of sequences 0..len(lens)-1, after their K/V pages
        were written by another engine (rxla_b200_decoder_set_context_lengths)."""
        a = np.ascontiguousarray(np.asarray(lens, dtype=np.int32))
        _lib.call("rxla_b200_decoder_set_context_lengths", self._h,
                  a.ctypes.data_as(ctypes.c_void_p), len(a), stream)

    def step_device(self, batch: int, stream=None, logits_ptr=None):
        """One step on tokens already in the runner's device input buffer."""
        _lib.call("rxla_b200_decoder_step", self._h, self.tokens_in_ptr, batch,
                  self.tokens_out_ptr, logits_ptr, stream)

    def prefill(self, seq: int, tokens, stream=None, logits_ptr=None):
        """Run a prompt (device int32 tensor or any int sequence) through the
        layers for sequence ``seq`` (rxla_b200_decoder_prefill); returns the
        device int32 tensor [1] holding the greedy token after the prompt."""
        import torch
        dev = torch.device("cuda", self._device)
        t = torch.as_tensor(tokens, dtype=torch.int32).to(dev).contiguous()
        out = torch.empty(1, dtype=torch.int32, device=dev)
        _lib.call("rxla_b200_decoder_prefill", self._h, seq, t.data_ptr(), t.numel(),
                  out.data_ptr(), logits_ptr, stream)
        return out

    def load_safetensors(self, path, prefix: str = "model.language_model."):
        """Fill every parameter from a safetensors checkpoint
        (rxla_b200_decoder_load_safetensors); returns (loaded, skipped) tensor
        counts."""
        loaded, skipped = ctypes.c_int32(), ctypes.c_int32()
        _lib.call("rxla_b200_decoder_load_safetensors", self._h, str(path).encode(),
                  prefix.encode(), ctypes.byref(loaded), ctypes.byref(skipped))
        return loaded.value, skipped.value

    def step_host(self, tokens, stream=None) -> np.ndarray:
        """One step from host tokens to host next tokens (copies + sync inside)."""
        tokens = np.ascontiguousarray(tokens, np.int32)
        b = tokens.shape[0]
        _lib.call("rxla_b200_decoder_step_host", self._h, tokens.ctypes.data_as(ctypes.c_void_p),
                  b, self._out_host.ctypes.data_as(ctypes.c_void_p), stream)
        return self._out_host[:b].copy()


# ------------------------------------------------------------ tensor parallel

class Comm:
    """NCCL communicator of one tensor-parallel rank (rxla_b200_comm_*).

    Rank 0 creates the unique id; the 128 bytes reach the other ranks through
    any host channel — ``share`` is a callable that broadcasts them from rank 0
    (for example via ``torch.distributed.broadcast_object_list``), in the way
    rxla's KeyValueStore rendezvous moves its client id
    (crates/rxla-pjrt/src/distributed.rs:40-120)."""

    def __init__(self, rank: int, world: int, device: int, share):
        uid = (ctypes.c_uint8 * _lib.COMM_ID_BYTES)()
        if rank == 0:
            _lib.call("rxla_b200_comm_unique_id", uid)
        data = share(bytes(uid) if rank == 0 else None)
        uid = (ctypes.c_uint8 * _lib.COMM_ID_BYTES).from_buffer_copy(data)
        h = ctypes.c_void_p()
        _lib.call("rxla_b200_comm_init", uid, rank, world, device, ctypes.byref(h))
        self._h = h
        self.rank, self.world = rank, world

    @property
    def handle(self):
        return self._h

    def close(self):
        if self._h:
            _lib.load().rxla_b200_comm_destroy(self._h)
            self._h = None


def shard_parameter(name: str, full: np.ndarray, rank: int, tp: int, *, q_heads: int,
                    kv_heads: int, head_dim: int, intermediate: int, hidden: int,
                    vocab: int, group_size: int = 0) -> np.ndarray:
    """The slice of a full (tp = 1) parameter that rank `rank` of `tp` holds.

    Column-parallel (split output rows): q_proj / k_proj / v_proj by heads,
    gate_proj / up_proj by the intermediate slice.  Row-parallel (split input
    columns): o_proj / down_proj weights; their per-output-channel scales are
    whole, grouped scales are split with the columns.  Embeddings and norms
    are whole (the tied head reads its vocab slice of the whole embedding)."""
    if tp == 1:
        return full
    D = head_dim
    if name.endswith(("q_proj.weight", "q_proj.scale")):
        n = q_heads // tp * D
        return full[rank * n:(rank + 1) * n]
    if name.endswith(("k_proj.weight", "k_proj.scale", "v_proj.weight", "v_proj.scale")):
        n = kv_heads // tp * D
        return full[rank * n:(rank + 1) * n]
    if name.endswith(("gate_proj.weight", "gate_proj.scale", "up_proj.weight", "up_proj.scale")):
        n = intermediate // tp
        return full[rank * n:(rank + 1) * n]
    if name.endswith(("o_proj.weight", "down_proj.weight")):
        k_full = full.shape[1]
        n = k_full // tp
        return full[:, rank * n:(rank + 1) * n]
    if name.endswith(("o_proj.scale", "down_proj.scale")):
        if full.shape[1] == 1:  # per output channel: the same scale on every rank
            return full
        n = full.shape[1] // tp
        return full[:, rank * n:(rank + 1) * n]
    return full
