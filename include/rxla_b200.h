/*
 * rxla_b200.h — C ABI of the B200 (sm_100a) W8 decode hot path.
 *
 * This library replaces, for one path only, the device work that rxla hands
 * to XLA through PJRT: the int8-weight linear layers (QuantizedLinear) and the
 * grouped-query KV-cache attention of decoder-LLM decode.  Every entry point
 * is plain `extern "C"`: raw device pointers, sizes, a CUDA stream passed as
 * `void*`, and an `int32_t` status.  No C++ or torch types cross the ABI.
 *
 * Conventions
 *  - Ownership: the caller owns every tensor buffer (device pointers).  The
 *    library allocates only inside `*_create` objects (decoder runner, comm)
 *    and never on a launch path.
 *  - Streams: every launch is ordered on the given stream (NULL = legacy
 *    default stream).  Nothing synchronises implicitly.
 *  - Errors: 0 is success.  Failures return the negated absl/PJRT status class
 *    (the same classes rxla maps to `PjrtErrorCode`,
 *    crates/rxla-pjrt/src/runtime.rs:49-107).  A thread-local message is
 *    available from rxla_b200_last_error_message().  Nothing aborts or traps.
 *  - Threading: launches on distinct streams may come from distinct threads.
 *    A decoder or comm handle is used by one thread at a time.
 *  - Dtypes: bf16 tensors are raw IEEE bfloat16 (uint16_t storage).
 *
 * Reference interfaces replaced (paths inside the rxla project):
 *  - crates/rxla-nn/src/layers.rs:231-298   QuantizedLinear / apply_quantized_linear
 *  - crates/rxla-nn/src/layers.rs:784-793   Cx::quantized_linear(out, group)
 *  - crates/rxla-core/src/nn.rs:286-310     Tensor::linear (x · Wᵀ)
 *  - crates/rxla-core/src/attention.rs:83-252  grouped_query_attention / SDPA
 *  - crates/rxla-core/src/attention.rs:14-67   causal masks (decode form)
 *  - crates/rxla-core/src/kv_cache.rs:53-112   KvCache::update_at(_checked)
 *  - crates/rxla-core/src/rotary.rs:17-74      rotary_embedding(_angles), SplitHalf
 *  - crates/rxla-core/src/ops.rs:929-945       Tensor::rms_norm
 *  - crates/rxla-nn/src/applied.rs:222-237     BoundModel::run (decoder step)
 *  - crates/rxla-core/src/state.rs:1200-1228   Session::run (stateful step)
 *  - crates/rxla-pjrt/src/distributed.rs:40-120 distributed rendezvous (comm)
 */
#ifndef RXLA_B200_H_
#define RXLA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Every declaration below is an exported symbol of librxla_b200.so (the
 * library is built with hidden visibility for everything else). */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#define RXLA_B200_ABI_VERSION 1

/* Status codes: negated absl status classes, as PjrtErrorCode uses them
 * (crates/rxla-pjrt/src/runtime.rs:49-107). */
typedef enum rxla_b200_status {
  RXLA_B200_OK = 0,
  RXLA_B200_INVALID_ARGUMENT = -3,
  RXLA_B200_DEADLINE_EXCEEDED = -4, /* a bounded device wait ran out */
  RXLA_B200_NOT_FOUND = -5,
  RXLA_B200_RESOURCE_EXHAUSTED = -8,
  RXLA_B200_FAILED_PRECONDITION = -9,
  RXLA_B200_OUT_OF_RANGE = -11,
  RXLA_B200_UNIMPLEMENTED = -12,
  RXLA_B200_INTERNAL = -13,
  RXLA_B200_UNAVAILABLE = -14 /* CUDA / NCCL runtime failure */
} rxla_b200_status;

/* Element types used at the boundary (rxla DType subset). */
typedef enum rxla_b200_dtype {
  RXLA_B200_F32 = 0,
  RXLA_B200_BF16 = 1,
  RXLA_B200_U8 = 2,
  RXLA_B200_I32 = 3,
  RXLA_B200_F16 = 4
} rxla_b200_dtype;

/* Linear epilogues. */
typedef enum rxla_b200_epilogue {
  /* y[m,n] = out                                                         */
  RXLA_B200_EPI_STORE = 0,
  /* y[m,n] (f32, in place) += bf16(out): the residual add of a decoder block */
  RXLA_B200_EPI_RESIDUAL_ADD = 1,
  /* weight holds 2n rows [gate; up]; y[m,i] = silu(gate_i) * up_i, both
   * rounded to bf16 first (crates/rxla-models/src/qwen3_5/layers.rs:270-293) */
  RXLA_B200_EPI_SWIGLU = 2
} rxla_b200_epilogue;

/* KV update policy of the decode attention (crates/rxla-core/src/kv_cache.rs). */
typedef enum rxla_b200_kv_update {
  /* update_at: an out-of-range start is clamped to the last slot (:43-68) */
  RXLA_B200_KV_CLAMP = 0,
  /* update_at_checked: an out-of-range start leaves the cache unchanged and
   * reports accepted = 0 (:70-112) */
  RXLA_B200_KV_CHECKED = 1
} rxla_b200_kv_update;

/* ---------------------------------------------------------------- library */

int32_t rxla_b200_abi_version(void);
/* Thread-local message of the last failing call on this thread ("" if none). */
const char* rxla_b200_last_error_message(void);
/* Number of SMs and compute capability of `device`. */
int32_t rxla_b200_device_info(int32_t device, int32_t* sm_count, int32_t* cc_major,
                              int32_t* cc_minor);
/* Status word the kernels of the current device set when a bounded device-side
 * wait runs out (RXLA_B200_DEADLINE_EXCEEDED) — kernels return instead of
 * hanging.  0 when nothing went wrong; nonzero `reset` clears it. */
int32_t rxla_b200_device_status(int32_t reset);
/* Budget in nanoseconds of every bounded device-side wait in this library's
 * kernels on the current device (mbarrier rings, split-K hand-offs, the peer
 * all-reduce's flag waits); default 4 s, allowed range [1 ms, 60 s].  Kernels
 * that start after the call (graph replays included) use the new value.  A
 * wait that runs out records RXLA_B200_DEADLINE_EXCEEDED in the device status
 * word and its kernel returns early; the context stays usable.  Replaces no
 * reference interface (XLA's own kernels do not wait on peers). */
int32_t rxla_b200_set_wait_timeout(int64_t ns);
int32_t rxla_b200_get_wait_timeout(int64_t* ns);
/* Diagnostic of the bounded device-side waits: one thread waits, under the
 * current budget, either (kind 0) on a shared-memory mbarrier that nothing
 * arrives on — the wait of every TMA ring here, so it always runs out — or
 * (kind 1) for the u64 at `flag` (8-byte aligned; device, managed or pinned
 * host memory, else INVALID_ARGUMENT) to reach `target` —
 * the peer all-reduce's flag wait.  A wait that runs out records
 * RXLA_B200_DEADLINE_EXCEEDED in the device status word and the kernel
 * returns.  Asynchronous on `stream`.  Replaces no reference interface; it
 * lets a single GPU show the failure path of the waits. */
int32_t rxla_b200_bounded_wait_check(int32_t kind, const uint64_t* flag, uint64_t target,
                                     void* stream);

/* ------------------------------------------------------- W8A16 linear layer
 *
 * Replaces QuantizedLinear::apply (crates/rxla-nn/src/layers.rs:257-298) with
 * the layer compute dtype BF16 (crates/rxla-nn/src/lib.rs:487-500):
 *
 *   y = bf16(x) · ((weight - 128) ⊙ scale[n, k / group])ᵀ
 *
 * weight : u8 [n_rows, k] row-major, signed int8 stored as value + 128
 *          (benchmarks/quantize_qwen3_5_w8.py:33-44); n_rows = n, or 2n for
 *          RXLA_B200_EPI_SWIGLU.
 * scale  : f32 [n_rows, k / group_size]; group_size must divide k
 *          (layers.rs:266-275); group_size == k is per-output-channel.
 * x      : [m, k], RXLA_B200_BF16 or RXLA_B200_F32 (rounded to bf16 on load).
 * y      : [m, n].  The dot product is accumulated in fp32.
 *          EPI_STORE + BF16 y: stores bf16(dot), the reference's bf16 dot
 *          output (widen it to get the reference's F32 boundary value).
 *          EPI_STORE + F32 y: stores the fp32 dot unrounded (an F32-output
 *          dot, as the tied LM head of qwen3_5/mod.rs:157-173).
 *          EPI_RESIDUAL_ADD (F32 y): y += bf16(dot).
 *          EPI_SWIGLU: y = silu(bf16(gate)) * bf16(up), BF16 or F32 y.
 * m == 0 or n == 0 is a no-op.  Sizes are checked; a bad size returns
 * RXLA_B200_INVALID_ARGUMENT without launching anything.
 */
int32_t rxla_b200_w8a16_linear(const void* x, int32_t x_dtype, const uint8_t* weight,
                               const float* scale, int64_t group_size, int64_t m, int64_t n,
                               int64_t k, void* y, int32_t y_dtype, int32_t epilogue,
                               void* stream);

/* The same linear with a caller-owned workspace, which lets the tensor-core
 * GEMM (more than 8 tokens) split K across more CTAs than it has output
 * tiles — the depth the decoder's own GEMMs use.  Size it with
 * rxla_b200_w8a16_linear_workspace_size for the shape (0 bytes: no split
 * for this shape on this device; then workspace may be null).  The
 * workspace must be 16-byte aligned and zero-filled before its first use;
 * every call leaves its counters zero again.  Calls sharing one workspace
 * must be stream-ordered. */
int32_t rxla_b200_w8a16_linear_workspace_size(int64_t m, int64_t n, int64_t k, int64_t group_size,
                                              int32_t epilogue, size_t* bytes);
int32_t rxla_b200_w8a16_linear_ws(const void* x, int32_t x_dtype, const uint8_t* weight,
                                  const float* scale, int64_t group_size, int64_t m, int64_t n,
                                  int64_t k, void* y, int32_t y_dtype, int32_t epilogue,
                                  void* workspace, size_t workspace_bytes, void* stream);

/* The same linear with its input RMSNorm fused into the kernel's prologue, the
 * decoder block's `linear(rms_norm(h))` for decode shapes (each pass of up to
 * 8 tokens streams the weights once):
 *
 *   y = bf16(h * rsqrt(mean(h²) + eps) * norm_weight) · W_deqᵀ
 *
 * (crates/rxla-core/src/ops.rs:929-945, then the bf16 cast of the consuming
 * QuantizedLinear, crates/rxla-nn/src/layers.rs:289-297).  h f32 [m, k] (a
 * residual stream), norm_weight f32 [k]; weight / scale / y / epilogue as in
 * rxla_b200_w8a16_linear.  Needs k % 64 == 0, group_size == k or a multiple
 * of 64, 16-byte aligned h and weight; y must not overlap h. */
int32_t rxla_b200_w8a16_norm_linear(const float* h, const float* norm_weight, float eps,
                                    const uint8_t* weight, const float* scale,
                                    int64_t group_size, int64_t m, int64_t n, int64_t k, void* y,
                                    int32_t y_dtype, int32_t epilogue, void* stream);

/* Dense bf16-weight linear y = bf16(x) · wᵀ (the tied bf16 LM head of a
 * decoder whose embedding stays bf16; crates/rxla-core/src/nn.rs:286-310).
 * weight bf16 [n, k]; same x / y / epilogue rules as above (SWIGLU excluded). */
int32_t rxla_b200_bf16_linear(const void* x, int32_t x_dtype, const uint16_t* weight,
                              int64_t m, int64_t n, int64_t k, void* y, int32_t y_dtype,
                              int32_t epilogue, void* stream);

/* ----------------------------------------------- paged GQA decode attention
 *
 * One decode step for `batch` sequences: per-head RMSNorm of q and of the new
 * k (optional), RoPE (SplitHalf, crates/rxla-core/src/rotary.rs:29-74) at
 * position ctx_lens[b], append of the new k/v into the paged bf16 cache
 * (KvCache::update_at / update_at_checked semantics), then
 * softmax(q·Kᵀ·scale + causal mask)·V over the cache with consecutive query
 * heads sharing a kv head (crates/rxla-core/src/attention.rs:73-135).
 *
 * Cache layout: k_pages / v_pages bf16 [num_pages, kv_heads, page_size,
 * head_dim]; page_table int32 [batch, max_pages_per_seq] maps the p-th page of
 * sequence b; capacity of sequence b = pages_per_seq[b] * page_size (or
 * max_pages_per_seq * page_size when pages_per_seq is NULL).
 * head_dim 64, 128 or 256 (256: rotary_dim <= 128); 1 to 8 query heads per
 * kv head; rotary_dim a multiple of 32.
 */
typedef struct rxla_b200_paged_decode_args {
  uint32_t struct_size; /* sizeof(rxla_b200_paged_decode_args) */
  int32_t batch, q_heads, kv_heads, head_dim;
  /* new-token projections (bf16), row stride in elements; q [batch, q_heads*d],
   * k/v [batch, kv_heads*d] — a fused QKV output passes offsets into one row. */
  const uint16_t* q;
  const uint16_t* k_new;
  const uint16_t* v_new;
  int64_t q_row_stride, kv_row_stride;
  /* optional per-head RMSNorm weights [head_dim] (f32), NULL = no norm */
  const float* q_norm_weight;
  const float* k_norm_weight;
  float norm_eps;
  /* RoPE: inv_freq f32 [rotary_dim/2] (host-computed θ^(-2i/rotary_dim)),
   * NULL or rotary_dim == 0 = no rotation; rotation covers dims [0, rotary_dim) */
  const float* inv_freq;
  int32_t rotary_dim;
  float scale; /* 0 => 1/sqrt(head_dim) (attention.rs:190) */
  /* paged cache */
  uint16_t* k_pages;
  uint16_t* v_pages;
  int64_t num_pages;
  int32_t page_size; /* must be 16 */
  int32_t max_pages_per_seq;
  const int32_t* page_table;    /* [batch, max_pages_per_seq] */
  const int32_t* pages_per_seq; /* [batch] or NULL */
  const int32_t* ctx_lens;      /* [batch] tokens already cached = new position */
  int32_t kv_update;            /* rxla_b200_kv_update */
  int32_t advance_ctx;          /* nonzero: ctx_lens[b] += accepted (in place) */
  int32_t* accepted;            /* optional [batch] out: 1 written, 0 rejected */
  /* output [batch, q_heads*head_dim] bf16 */
  uint16_t* out;
  /* scratch for split-K partials; size from rxla_b200_paged_decode_workspace_size */
  void* workspace;
  size_t workspace_bytes;
  int32_t max_context; /* upper bound of ctx_lens[b]+1, sizes the split grid */
} rxla_b200_paged_decode_args;

/* Bytes of workspace the decode attention needs for this shape.  The first
 * 4*batch*kv_heads bytes are counters that must be zero before the first call
 * (cudaMemset once); every call leaves them zero again. */
int32_t rxla_b200_paged_decode_workspace_size(int32_t batch, int32_t q_heads,
                                              int32_t kv_heads, int32_t head_dim,
                                              int32_t max_context, size_t* bytes);

int32_t rxla_b200_paged_decode_attention(const rxla_b200_paged_decode_args* args,
                                         void* stream);

/* Paged decode attention that allocates nothing, for callers that may not
 * call cudaMalloc: code running inside another runtime's execute callback
 * (an XLA FFI custom call, a PJRT plugin, a serving engine's step), whose
 * runtime owns the device memory, and latency-critical decode loops, where an
 * allocation can synchronise the device.  No counterpart in the reference
 * (rxla's XLA path allocates through PJRT).
 *
 * Same arguments and results as rxla_b200_paged_decode_attention, except that
 * args->workspace / workspace_bytes are ignored: the split-K scratch is a
 * fixed array of RXLA_B200_NOALLOC_SCRATCH_BYTES compiled into the library
 * (held by every GPU that loads the library until the process exits).  A shape
 * whose rxla_b200_paged_decode_workspace_size exceeds it returns
 * RXLA_B200_OUT_OF_RANGE without launching.  The first call on a device looks
 * up the array's device address (make it before any stream capture); every
 * call clears the array's split counters on its stream, which must belong to
 * the current device (else RXLA_B200_INVALID_ARGUMENT).  All calls share the
 * one array, so calls that can run at the same time on the GPU race. */
#define RXLA_B200_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)
int32_t rxla_b200_paged_decode_attention_noalloc(const rxla_b200_paged_decode_args* args,
                                                 void* stream);

/* ------------------------------------------------------- small fused ops */

/* y[r, :] = bf16(x[r,:] * rsqrt(mean(x²) + eps) * w)  (ops.rs:929-945,
 * then the bf16 cast of the consuming linear).  x f32 [rows, width]. */
int32_t rxla_b200_rms_norm_bf16(const float* x, const float* weight, int64_t rows,
                                int64_t width, float eps, uint16_t* y, void* stream);

/* Greedy sampling: out[r] = first index of the maximum of logits[r, :]
 * (f32 [rows, vocab]), the ArgMax of crates/rxla-core/src/dtype_rules.rs:26. */
int32_t rxla_b200_argmax(const float* logits, int64_t rows, int64_t vocab, int32_t* out,
                         void* stream);

/* W8 token embedding (crates/rxla-models/src/qwen3_5/mod.rs:134-155):
 * out[r, :] = f32(weight[ids[r], :] - 128) · scale[ids[r], c / group_size]
 * for int32 ids [rows] (device), u8 weight [vocab, hidden], f32 scale
 * [vocab, hidden / group_size]; out f32 [rows, hidden].  An id outside
 * [0, vocab) gives a zero row. */
int32_t rxla_b200_w8_embedding(const int32_t* ids, int64_t rows, const uint8_t* weight,
                               const float* scale, int64_t vocab, int64_t hidden,
                               int64_t group_size, float* out, void* stream);

/* Output gate of Qwen3.5's full-attention layers
 * (crates/rxla-models/src/qwen3_5/layers.rs:50-55, 94-95):
 * y[r, c] = bf16(x[r, c] · sigmoid(gate[r, c])) for bf16 x (the attended
 * values) and gate (the gate half of q_proj), rows × width, each with its
 * own row stride in elements (a fused projection passes an offset into its
 * rows).  y may alias x. */
int32_t rxla_b200_sigmoid_gate(const uint16_t* x, int64_t x_row_stride, const uint16_t* gate,
                               int64_t gate_row_stride, int64_t rows, int64_t width, uint16_t* y,
                               int64_t y_row_stride, void* stream);

/* ------------------------------------------- gated-delta linear attention
 *
 * The mixer of Qwen3.5's linear-attention layers between its input
 * projections and its out_proj (gated_delta_attention,
 * crates/rxla-models/src/qwen3_5/layers.rs:114-268), for `tokens` new tokens
 * of each of `batch` sequences, continuing each sequence's state:
 *
 *   x    = silu(causal depthwise conv_K(mixed))        (layers.rs:131-145)
 *   q, k = l2_norm per head (x·rsqrt(Σx²+1e-6)); q ·= 1/sqrt(D)   (:103-160)
 *   beta = sigmoid(b);  g = exp(softplus(a + dt_bias) · -exp(A_log)) (:179-212)
 *   per token:  S = g·S;  S += k ⊗ beta·(v − Sᵀk);  o = Sᵀq          (:205-242)
 *   out  = bf16(o · rsqrt(mean(o²) + eps) · norm_weight · silu(z))   (:243-259)
 *
 * with H = heads, D = head_dim (key and value heads alike, D ∈ {32, 64,
 * 128}), W = H·D.  Inputs are the bf16 projections of the tokens, row r =
 * b·tokens + t: mixed [rows, 3W] (q | k | v channels), z [rows, W], b and a
 * [rows, H], each with its own row stride in elements (a fused projection
 * passes offsets into one row).  conv_weight f32 [3W, K] (the reference's
 * [3W, 1, K]), a_log / dt_bias f32 [H], norm_weight f32 [D].
 * State (in place): conv_state bf16 [batch, K-1, 3W], the last K-1 mixed rows
 * of each sequence, oldest first; state f32 [batch, H, D, D] with S[:, j]
 * (column j of the reference's [Dk, Dv] state) contiguous at [b, h, j, :].
 * has_state == 0 starts every sequence from zero state and zero history (the
 * reference's full-sequence forward); nonzero continues from the stored
 * state, so a prompt prefilled in one call or in several, then decoded one
 * token per call, gives the full forward's outputs.  Output out bf16
 * [rows, W] (the input of out_proj).  The workspace (256-byte aligned, size
 * from rxla_b200_gated_delta_workspace_size, no zero-fill needed) holds the
 * normalised q/k/v, the gates and o (single-token calls of at most 296
 * sequence × head pairs run as one kernel and leave it untouched).  Calls on
 * one state must be stream-ordered.
 */
typedef struct rxla_b200_gated_delta_args {
  uint32_t struct_size; /* sizeof(rxla_b200_gated_delta_args) */
  int32_t batch, tokens, heads, head_dim, conv_kernel;
  const uint16_t* mixed;
  const uint16_t* z;
  const uint16_t* beta_logits;
  const uint16_t* a;
  int64_t mixed_row_stride, z_row_stride, b_row_stride, a_row_stride;
  const float* conv_weight;
  const float* a_log;
  const float* dt_bias;
  const float* norm_weight;
  float eps;
  int32_t has_state;
  uint16_t* conv_state;
  float* state;
  uint16_t* out;
  void* workspace;
  size_t workspace_bytes;
} rxla_b200_gated_delta_args;

int32_t rxla_b200_gated_delta_workspace_size(int32_t batch, int32_t tokens, int32_t heads,
                                             int32_t head_dim, size_t* bytes);
int32_t rxla_b200_gated_delta(const rxla_b200_gated_delta_args* args, void* stream);

/* ---------------------------------------------------------- decoder runner
 *
 * A Qwen3-style W8 decoder (plain q_proj, per-head q_norm / k_norm, full
 * RoPE, SwiGLU MLP, tied LM head, greedy argmax) composed from the ops above
 * — the composition of crates/rxla-models/src/qwen3_5/{mod.rs,layers.rs}
 * restricted to full-attention layers.  It owns its weights and its paged KV
 * cache; one step is captured once into a CUDA graph and replayed.
 */
typedef struct rxla_b200_decoder_config {
  uint32_t struct_size; /* sizeof(rxla_b200_decoder_config) */
  int32_t layers, hidden, q_heads, kv_heads, head_dim, intermediate, vocab;
  float rms_eps, rope_theta;
  int32_t embedding_dtype; /* RXLA_B200_U8 (W8 tied head) or RXLA_B200_BF16 */
  int32_t group_size;      /* 0 = per-output-channel */
  int32_t max_batch, max_context;
  /* Tensor-parallel shard of this process (tp_size 1: the whole model).
   * Rank r holds q heads [r·Hq/tp, ...), kv heads [r·Hkv/tp, ...), the
   * matching q/k/v rows of the fused qkv, columns of o_proj, intermediate
   * slice [r·I/tp, ...) of gate/up rows and down_proj columns, and vocab
   * slice [r·V/tp, ...) of the tied head; embeddings and norms are whole.
   * o_proj / down_proj partial sums are all-reduced (f32) over `comm` before
   * the bf16 rounding and residual add; the greedy token is the argmax over
   * all ranks' slices (all-gathered candidates).  kv_heads, intermediate and
   * vocab must divide by tp_size. */
  int32_t tp_rank, tp_size;
} rxla_b200_decoder_config;

typedef struct rxla_b200_decoder rxla_b200_decoder;
typedef struct rxla_b200_comm rxla_b200_comm;

int32_t rxla_b200_decoder_create(const rxla_b200_decoder_config* config, int32_t device,
                                 rxla_b200_comm* comm, rxla_b200_decoder** out);
int32_t rxla_b200_decoder_destroy(rxla_b200_decoder* decoder);
/* Device pointer, byte size and dtype of a named parameter of this shard.
 * Names follow the checkpoint layout, e.g. "embed_tokens.weight",
 * "layers.3.self_attn.q_proj.weight", "layers.3.mlp.down_proj.scale",
 * "layers.3.input_layernorm.weight", "norm.weight". */
int32_t rxla_b200_decoder_parameter(rxla_b200_decoder* decoder, const char* name,
                                    void** device_ptr, int64_t* bytes, int32_t* dtype);
/* Copy `bytes` of host memory into the named parameter (sizes must match):
 * the loading path for checkpoint tensors. Synchronous. */
int32_t rxla_b200_decoder_set_parameter(rxla_b200_decoder* decoder, const char* name,
                                        const void* host, int64_t bytes);
/* Fill every parameter with seeded synthetic values on the device: W8 weights
 * N(0, 0.02) quantized per row (clip 4.5σ), norms 1 + N(0, 0.02), bf16
 * embedding N(0, 0.02). */
int32_t rxla_b200_decoder_init_synthetic(rxla_b200_decoder* decoder, uint64_t seed);
/* Drop all cached context of every sequence. */
int32_t rxla_b200_decoder_reset(rxla_b200_decoder* decoder, void* stream);
/* One decode step of `batch` sequences: tokens (device int32 [batch]) at the
 * next position of each sequence.  Writes the greedy next token (device
 * int32 [batch]) and, if logits is non-NULL, the f32 logits [batch, vocab/tp]
 * of this shard's vocab slice.  Stream-ordered; replays a captured CUDA graph.
 * With tp_size > 1 every rank calls this for the same step (collectives). */
int32_t rxla_b200_decoder_step(rxla_b200_decoder* decoder, const int32_t* tokens,
                               int32_t batch, int32_t* next_tokens, float* logits,
                               void* stream);
/* Prefill: run `count` prompt tokens (int32 [count] in device, managed or
 * pinned host memory; ordinary host memory is refused) of sequence `seq`
 * through every layer at positions ctx[seq] .. ctx[seq] + count - 1, append
 * their K/V to the sequence's pages and advance ctx[seq] by count.  The
 * linears run over a whole chunk of prompt rows (tcgen05 GEMM) and each row
 * attends causally over the cache up to its own position.  Writes the greedy
 * token after the prompt to next_tokens[seq] of rxla_b200_decoder_io (and to
 * next_token, device int32 [1], if non-NULL) and, if logits is non-NULL, the
 * last row's f32 logits [vocab/tp].  Replaces the full-sequence forward of
 * crates/rxla-models/src/qwen3_5/mod.rs:199-260 (qwen3_5() over a [1, T]
 * prompt with the causal mask of mod.rs:229) for the full-attention layers,
 * one sequence of the paged state at a time.  Synchronises `stream`
 * once to read the position; ctx[seq] + count must not exceed max_context.
 * With tp_size > 1 every rank calls this with the same arguments. */
int32_t rxla_b200_decoder_prefill(rxla_b200_decoder* decoder, int32_t seq, const int32_t* tokens,
                                  int32_t count, int32_t* next_token, float* logits,
                                  void* stream);
/* ---------------------------------------------------------------------------
 * Checkpoints: safetensors reader and the decoder's W8 checkpoint loader
 * (crates/rxla-safetensors/src/lib.rs).  Host code; no GPU needed for the
 * reader.
 * ------------------------------------------------------------------------- */
typedef struct rxla_b200_safetensors rxla_b200_safetensors;
/* Open and validate a .safetensors file (SafeTensors::new, lib.rs:147-177):
 * header of at most 100 MB, tensors tiling the payload exactly, byte ranges
 * matching shape × dtype size, payload length matching the file. */
int32_t rxla_b200_safetensors_open(const char* path, rxla_b200_safetensors** out);
int32_t rxla_b200_safetensors_close(rxla_b200_safetensors* reader);
int32_t rxla_b200_safetensors_count(const rxla_b200_safetensors* reader, int32_t* count);
/* Tensor `index` (header order): name (valid while open), dtype (RXLA_B200_*,
 * -1 for a type without a code here, e.g. F64), rank, shape [<= 8], bytes. */
int32_t rxla_b200_safetensors_info(const rxla_b200_safetensors* reader, int32_t index,
                                   const char** name, int32_t* dtype, int32_t* ndim,
                                   int64_t* shape, int64_t* bytes);
/* Index of a tensor by name (SafeTensors::info); RXLA_B200_NOT_FOUND if absent. */
int32_t rxla_b200_safetensors_find(const rxla_b200_safetensors* reader, const char* name,
                                   int32_t* index);
/* A "__metadata__" string (SafeTensors::metadata); RXLA_B200_NOT_FOUND if absent. */
int32_t rxla_b200_safetensors_metadata(const rxla_b200_safetensors* reader, const char* key,
                                       const char** value);
/* Exact payload bytes (read_u8 / read_f32 without conversion, lib.rs:299-386)
 * of the block [row0, row0 + rows) × [col0, col0 + cols) of the tensor seen
 * as a matrix (rank 0/1: one row; rank >= 2: first dimension × the rest).
 * dst_bytes must equal rows × cols × element size. */
int32_t rxla_b200_safetensors_read(const rxla_b200_safetensors* reader, int32_t index,
                                   int64_t row0, int64_t rows, int64_t col0, int64_t cols,
                                   void* dst, int64_t dst_bytes);
/* Load a checkpoint into the decoder's parameters: every tensor whose name
 * starts with `prefix` (e.g. "model.language_model." of the rxla-qwen3.5-w8-v1
 * format, benchmarks/quantize_qwen3_5_w8.py) is matched, prefix removed,
 * against rxla_b200_decoder_parameter names (q/k/v_proj and gate/up_proj
 * land in the fused matrices); U8 weights and F32 scales are uploaded as
 * stored (upload_u8, lib.rs:664-700).  With tp_size > 1 each rank takes its
 * slice of the full tensors.  Fails if a tensor's dtype or size does not
 * match, if metadata "group_size" differs from the decoder's, or if any
 * decoder parameter is left unfilled.  Synchronous. */
int32_t rxla_b200_decoder_load_safetensors(rxla_b200_decoder* decoder, const char* path,
                                           const char* prefix, int32_t* loaded,
                                           int32_t* skipped);
/* Host-buffer convenience for one step: copies tokens in and next tokens out
 * through pinned staging on `stream` and synchronises it. */
int32_t rxla_b200_decoder_step_host(rxla_b200_decoder* decoder, const int32_t* tokens_host,
                                    int32_t batch, int32_t* next_tokens_host, void* stream);
/* Device buffers the step reads and writes: tokens in (int32 [max_batch]),
 * next tokens out (int32 [max_batch]) and logits (f32 [max_batch, vocab/tp]).
 * Passing tokens_in / tokens_out to rxla_b200_decoder_step skips its copies. */
int32_t rxla_b200_decoder_io(rxla_b200_decoder* decoder, int32_t** tokens_in,
                             int32_t** tokens_out, float** logits);
/* The paged K/V cache of one layer (session state, like Session::state of
 * crates/rxla-core/src/state.rs): bf16 [max_batch * pages_per_seq, kv_heads,
 * 16, head_dim] each; sequence b owns pages [b * pages_per_seq, (b+1) * ...). */
int32_t rxla_b200_decoder_kv_cache(rxla_b200_decoder* decoder, int32_t layer, void** k_pages,
                                   void** v_pages, int64_t* bytes);
/* Current context length of each sequence (device int32 [max_batch]). */
int32_t rxla_b200_decoder_context_lengths(rxla_b200_decoder* decoder, const int32_t** lens);
/* Set the context length of sequences 0..count-1 (host int32, each below
 * max_context) after their K/V pages were written by another engine, e.g. a
 * prefill: the next step appends at that position.  Synchronises `stream`. */
int32_t rxla_b200_decoder_set_context_lengths(rxla_b200_decoder* decoder,
                                              const int32_t* lens_host, int32_t count,
                                              void* stream);

/* ---------------------------------------------------- tensor-parallel comm
 *
 * Replaces the PJRT distributed client + KV-store rendezvous
 * (crates/rxla-pjrt/src/distributed.rs:40-120): rank 0 creates an id, the
 * caller moves its bytes to every rank (any host store), every rank inits.
 */
#define RXLA_B200_COMM_ID_BYTES 128
int32_t rxla_b200_comm_unique_id(uint8_t id[RXLA_B200_COMM_ID_BYTES]);
int32_t rxla_b200_comm_init(const uint8_t id[RXLA_B200_COMM_ID_BYTES], int32_t rank,
                            int32_t world_size, int32_t device, rxla_b200_comm** out);
int32_t rxla_b200_comm_destroy(rxla_b200_comm* comm);
/* In-place bf16 or f32 sum all-reduce of `count` elements on `stream`. */
int32_t rxla_b200_allreduce(rxla_b200_comm* comm, void* buffer, int64_t count,
                            int32_t dtype, void* stream);
/* Collective: reserve IPC-shared peer buffers for one-shot all-reduces of up
 * to `max_count` f32 (handles exchanged through the comm itself).  The
 * decoder runner enables it for its row-parallel linears. */
int32_t rxla_b200_comm_p2p_enable(rxla_b200_comm* comm, int64_t max_count);
/* One-shot f32 sum all-reduce over NVLink peer memory: every rank pushes its
 * `partial` [count] into every rank's buffer, waits (bounded, ~4 s, then
 * RXLA_B200_DEADLINE_EXCEEDED in the device status word) for all pushes, and
 * sums in rank order, so every rank gets the same bits.  residual == NULL:
 * partial = sum; else residual += bf16(sum) (the row-parallel epilogue of
 * o_proj / down_proj, crates/rxla-nn/src/layers.rs:293-298 rounding). */
int32_t rxla_b200_p2p_allreduce_f32(rxla_b200_comm* comm, float* partial, float* residual,
                                    int64_t count, void* stream);

/* ------------------------------------------------- XLA custom-call adapters
 *
 * The linear and the decode attention as XLA GPU custom calls with XLA's
 * legacy untyped ABI, for registration through PJRT's GPU custom-call
 * extension with api_version 0:
 *   Plugin::register_gpu_custom_call(name, GpuCustomCallApi::Legacy,
 *       GpuCustomCallHandlers::execute_only(handler))
 * (crates/rxla-pjrt/src/runtime.rs:265-270, :395-436), `name` being the
 * function's own name.  XLA calls a handler with its stream, the device
 * pointers of the custom call's operands followed by its results, and the
 * call's backend_config bytes (`opaque`), which must be one of the config
 * structs below byte for byte (little-endian, this layout, version 1).
 * The *_status forms take XLA's status-returning signature (custom-call
 * api_version 2) and report a failure with XlaCustomCallStatusSetFailure,
 * resolved in the process at run time; the plain forms (api_version 1) have
 * no failure channel and only set the calling thread's error message.
 * Handlers allocate nothing: the attention uses the fixed scratch of
 * rxla_b200_paged_decode_attention_noalloc (same size limit; its first call
 * on a device should come before any stream capture).
 */
#define RXLA_B200_XLA_LINEAR_MAGIC 0x4E4C3852u    /* "R8LN" */
#define RXLA_B200_XLA_ATTENTION_MAGIC 0x54413852u /* "R8AT" */

/* backend_config of rxla_b200_xla_w8a16_linear(_status) — 64 bytes.
 * Operands: fused_norm == 0: x [m, k] (x_dtype), weight u8 [n_rows, k],
 *           scale f32 [n_rows, k / group_size];
 *           fused_norm != 0: h f32 [m, k], norm_weight f32 [k], weight, scale
 *           (rxla_b200_w8a16_norm_linear);
 *           then, for RXLA_B200_EPI_RESIDUAL_ADD only, the residual f32 [m, n].
 * Result:  y [m, n] (y_dtype).  With the residual epilogue y = residual +
 *          bf16(dot); y may alias the residual operand (it is copied first
 *          when it does not). */
typedef struct rxla_b200_xla_linear_config {
  uint32_t magic;   /* RXLA_B200_XLA_LINEAR_MAGIC */
  uint32_t version; /* 1 */
  int64_t m, n, k, group_size;
  int32_t x_dtype, y_dtype, epilogue, fused_norm;
  float eps; /* RMSNorm epsilon (fused_norm) */
  int32_t reserved;
} rxla_b200_xla_linear_config;

/* backend_config of rxla_b200_xla_paged_decode_attention(_status) — 64 bytes.
 * Operands: q bf16 [batch, q_heads*D], k_new / v_new bf16 [batch, kv_heads*D],
 *           (has_qk_norm) q_norm_weight f32 [D], k_norm_weight f32 [D],
 *           (rotary_dim > 0) inv_freq f32 [rotary_dim / 2],
 *           page_table i32 [batch, max_pages_per_seq], ctx_lens i32 [batch],
 *           k_pages, v_pages bf16 [num_pages, kv_heads, 16, D].
 * Results:  out bf16 [batch, q_heads*D], ctx_lens i32 [batch] (each advanced
 *           by the accepted token), k_pages, v_pages (the new row appended).
 *           The state results should alias their operands (donated buffers,
 *           KvCache semantics of crates/rxla-core/src/kv_cache.rs:53-112);
 *           when they do not, the operands are copied into them first. */
typedef struct rxla_b200_xla_attention_config {
  uint32_t magic;   /* RXLA_B200_XLA_ATTENTION_MAGIC */
  uint32_t version; /* 1 */
  int32_t batch, q_heads, kv_heads, head_dim;
  int32_t page_size; /* 16 */
  int32_t max_pages_per_seq;
  int64_t num_pages;
  int32_t max_context;
  int32_t has_qk_norm;
  int32_t rotary_dim; /* 0: no RoPE */
  int32_t kv_update;  /* rxla_b200_kv_update */
  float norm_eps;
  float scale; /* 0 => 1/sqrt(head_dim) */
} rxla_b200_xla_attention_config;

void rxla_b200_xla_w8a16_linear(void* stream, void** buffers, const char* opaque,
                                size_t opaque_len);
void rxla_b200_xla_w8a16_linear_status(void* stream, void** buffers, const char* opaque,
                                       size_t opaque_len, void* status);
void rxla_b200_xla_paged_decode_attention(void* stream, void** buffers, const char* opaque,
                                          size_t opaque_len);
void rxla_b200_xla_paged_decode_attention_status(void* stream, void** buffers,
                                                 const char* opaque, size_t opaque_len,
                                                 void* status);
/* Validate a backend_config for the named target before emitting it (the
 * lowering's compile-time check): RXLA_B200_OK, RXLA_B200_INVALID_ARGUMENT /
 * RXLA_B200_UNIMPLEMENTED for a bad blob, RXLA_B200_NOT_FOUND for an unknown
 * target.  No CUDA call. */
int32_t rxla_b200_xla_check_config(const char* target, const void* opaque, size_t opaque_len);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* RXLA_B200_H_ */
