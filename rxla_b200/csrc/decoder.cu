// decoder.cu — Qwen3-style W8 decoder runner (one decode step per call).
//
// Composition (crates/rxla-models/src/qwen3_5/mod.rs:199-273 and layers.rs,
// restricted to full-attention layers, with the Qwen3 differences: plain
// q_proj, per-head q_norm / k_norm, full RoPE, tied LM head):
//
//   h = embed(token)                                   (W8: (u8-128)*scale, or bf16)
//   per layer:
//     x  = bf16(rms_norm(h, input_layernorm))
//     qkv = W8(x, [q_proj; k_proj; v_proj])             (one fused GEMV)
//     a  = attention(q_norm/k_norm, RoPE, append, GQA)  (paged bf16 cache)
//     h += bf16(W8(a, o_proj))
//     x  = bf16(rms_norm(h, post_attention_layernorm))
//     g  = silu(bf16(W8(x, gate))) * bf16(W8(x, up))    (one fused GEMV)
//     h += bf16(W8(g, down_proj))
//   logits = bf16(rms_norm(h, norm)) · Eᵀ  (f32, unrounded), token = argmax
//
// The residual stream is f32; every linear computes in bf16 with fp32
// accumulation (the layer compute dtype BF16 of crates/rxla-nn/src/layers.rs:
// 289-297).  A step is 5 kernels per layer + 2 (W8 embedding), all launched with
// programmatic dependent launch and captured once per batch size into a CUDA
// graph; ctx_lens (the next position of each sequence) changes only in the
// last kernel of the step (the LM head's argmax epilogue), so the attention
// kernels may prefetch cache pages before griddepcontrol.wait.  The RMSNorms
// in front of qkv, gate/up and the head run in those GEMVs' prologues.
//
// Tensor parallelism (tp_size > 1): each rank holds its q/kv heads, its
// slices of gate/up rows and the matching columns of o_proj/down_proj; the
// row-parallel partial sums are all-reduced before the residual add.
#include <cmath>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "internal.cuh"

namespace rxla {

namespace dec {

__device__ __forceinline__ uint64_t mix64(uint64_t x) {
  uint64_t z = x + 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

// standard normal from a counter (Box-Muller on two 24-bit uniforms)
__device__ __forceinline__ float normal_at(uint64_t seed, uint64_t i) {
  const uint64_t r = mix64(seed ^ mix64(i));
  const float u1 = ((float)(r >> 40) + 1.0f) * (1.0f / 16777217.0f);
  const float u2 = (float)((r >> 16) & 0xffffff) * (1.0f / 16777216.0f);
  return sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}

// Synthetic W8 weights: N(0, 0.02) quantized symmetrically per row with the
// clip at 4.5σ (scale = 0.02·4.5/127): q = clamp(round(z·127/4.5)).
// Where the rows and columns of a rank's shard sit in the full (tp = 1)
// matrix: up to three row segments, then a column offset.  Synthetic weights
// are a function of the element's index in the full matrix, so every tensor-
// parallel degree holds slices of one and the same model.
struct Shard {
  int64_t k_full;                 // columns of the full matrix
  int64_t col_off;                // first full column of the shard
  int32_t nseg;
  int64_t seg_rows[3], seg_full_row[3];
};

__device__ __forceinline__ int64_t full_index(const Shard& sh, int64_t row, int64_t col) {
  int64_t r = row;
  for (int i = 0; i < sh.nseg; ++i) {
    if (r < sh.seg_rows[i]) return (sh.seg_full_row[i] + r) * sh.k_full + sh.col_off + col;
    r -= sh.seg_rows[i];
  }
  return 0;
}

__global__ void fill_w8_kernel(uint8_t* w, float* scale, int64_t rows, int64_t k, int64_t groups,
                               uint64_t seed, Shard sh) {
  const int64_t n = rows * k;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t g = (uint64_t)full_index(sh, i / k, i % k);
    float q = rintf(normal_at(seed, g) * (127.0f / 4.5f));
    q = fminf(127.0f, fmaxf(-127.0f, q));
    w[i] = (uint8_t)((int)q + 128);
    if (i < rows * groups) scale[i] = 0.02f * 4.5f / 127.0f;
  }
}

__global__ void fill_norm_kernel(float* w, int64_t n, uint64_t seed) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    w[i] = bf16_round(1.0f + 0.02f * normal_at(seed, (uint64_t)i));
}

__global__ void fill_bf16_kernel(__nv_bfloat16* w, int64_t n, uint64_t seed) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    w[i] = __float2bfloat16_rn(0.02f * normal_at(seed, (uint64_t)i));
}

// h[b, :] = embedding row of tokens[b] (token ids clamped into [0, vocab),
// as a gather clamps its indices).
__global__ void embed_kernel(const int32_t* __restrict__ tokens, const uint8_t* __restrict__ w8,
                             const float* __restrict__ scale, const __nv_bfloat16* __restrict__ wb,
                             int64_t vocab, int64_t hidden, int64_t groups, int64_t group,
                             float* __restrict__ h) {
  pdl_wait();
  pdl_launch_dependents();
  int64_t t = tokens[blockIdx.x];
  t = t < 0 ? 0 : (t >= vocab ? vocab - 1 : t);
  float* out = h + blockIdx.x * hidden;
  // 16 consecutive elements per thread, loaded before any is used (the row
  // is a single round trip for hidden <= 16 * blockDim)
  const bool vec = hidden % 16 == 0 && group % 16 == 0 &&
                   (reinterpret_cast<uintptr_t>(w8 ? (const void*)w8 : (const void*)wb) % 16) == 0;
  if (vec) {
    for (int64_t j0 = threadIdx.x * 16; j0 < hidden; j0 += blockDim.x * 16) {
      float v[16];
      if (w8) {
        const uint4 q = *reinterpret_cast<const uint4*>(w8 + t * hidden + j0);
        const float sc = scale[t * groups + j0 / group];
        const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int i = 0; i < 16; ++i)
          v[i] = (float)((int)((qw[i >> 2] >> (8 * (i & 3))) & 0xffu) - 128) * sc;
      } else {
        const uint4 a = *reinterpret_cast<const uint4*>(wb + t * hidden + j0);
        const uint4 b = *reinterpret_cast<const uint4*>(wb + t * hidden + j0 + 8);
        const uint32_t bw[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = (i & 1) ? bf16_hi(bw[i >> 1]) : bf16_lo(bw[i >> 1]);
      }
#pragma unroll
      for (int i = 0; i < 16; i += 4)
        *reinterpret_cast<float4*>(out + j0 + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    }
    return;
  }
  for (int64_t j = threadIdx.x; j < hidden; j += blockDim.x) {
    float v;
    if (w8) v = (float)((int)w8[t * hidden + j] - 128) * scale[t * groups + j / group];
    else v = __bfloat162float(wb[t * hidden + j]);
    out[j] = v;
  }
}

// h[b, :] += bf16(partial[b, :]) (tensor-parallel residual add after the
// all-reduce of the row-parallel partial sums).
__global__ void residual_add_kernel(const float* __restrict__ part, float* __restrict__ h,
                                    int64_t n) {
  pdl_wait();
  pdl_launch_dependents();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    h[i] = h[i] + bf16_round(part[i]);
}

// Rows of a prefill chunk: row t gets a copy of the sequence's page-table row
// and the position pos0 + t.
__global__ void prefill_rows_kernel(const int32_t* __restrict__ page_table, int32_t max_pages,
                                    int32_t seq, int32_t pos0, int32_t* __restrict__ pt_out,
                                    int32_t* __restrict__ ctx_out) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t t = blockIdx.x;
  for (int i = threadIdx.x; i < max_pages; i += blockDim.x)
    pt_out[t * max_pages + i] = page_table[(int64_t)seq * max_pages + i];
  if (threadIdx.x == 0) ctx_out[t] = pos0 + (int32_t)t;
}

__global__ void set_position_kernel(int32_t* __restrict__ ctx, int32_t seq, int32_t pos) {
  pdl_wait();
  pdl_launch_dependents();
  ctx[seq] = pos;
}

// Tensor-parallel greedy head: each rank's best logit of its vocab slice
// (value, global index), then the best over all ranks' candidates with the
// same tie rule as a full argmax (highest value, then lowest index).
struct Cand {
  float v;
  int32_t i;
};

__global__ void argmax_candidates_kernel(const float* __restrict__ logits, int64_t vocab_local,
                                         int32_t index_offset, Cand* __restrict__ cand) {
  pdl_wait();
  pdl_launch_dependents();
  const float* r = logits + blockIdx.x * vocab_local;
  float best = -INFINITY;
  int32_t idx = 0x7fffffff;
  for (int64_t c = threadIdx.x; c < vocab_local; c += blockDim.x) {
    const float v = r[c];
    if (v > best || (v == best && (int32_t)c < idx)) {
      best = v;
      idx = (int32_t)c;
    }
  }
  __shared__ float sb[32];
  __shared__ int32_t si[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int32_t oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ob > best || (ob == best && oi < idx)) {
      best = ob;
      idx = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    sb[threadIdx.x >> 5] = best;
    si[threadIdx.x >> 5] = idx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (sb[w] > best || (sb[w] == best && si[w] < idx)) {
        best = sb[w];
        idx = si[w];
      }
    cand[blockIdx.x].v = best;
    cand[blockIdx.x].i = idx == 0x7fffffff ? 0x7fffffff : idx + index_offset;
  }
}

__global__ void argmax_merge_kernel(const Cand* __restrict__ all, int32_t ranks, int32_t batch,
                                    int32_t* __restrict__ out, int32_t* __restrict__ advance) {
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  float best = -INFINITY;
  int32_t idx = 0x7fffffff;
  for (int r = 0; r < ranks; ++r) {
    const Cand c = all[(int64_t)r * batch + b];
    if (c.v > best || (c.v == best && c.i < idx)) {
      best = c.v;
      idx = c.i;
    }
  }
  out[b] = idx == 0x7fffffff ? 0 : idx;
  if (advance) advance[b] += 1;
}

struct Param {
  std::string name;
  void* ptr;
  int64_t bytes;
  int32_t dtype;
};

struct Layer {
  float* ln1;
  float* ln2;
  uint8_t* wqkv;
  float* sqkv;
  float* qn;
  float* kn;
  uint8_t* wo;
  float* so;
  uint8_t* wgu;
  float* sgu;
  uint8_t* wd;
  float* sd;
  uint16_t* kc;
  uint16_t* vc;
};

}  // namespace dec
}  // namespace rxla

struct rxla_b200_decoder {
  rxla_b200_decoder_config cfg;
  int device = 0;
  rxla_b200_comm* comm = nullptr;
  bool use_p2p = false;  // row-parallel all-reduces over the comm's peer buffers
  // batch <= 8: the all-reduce runs in the o_proj / down_proj GEMV epilogue
  // (RXLA_B200_TP_FUSED=0: a separate all-reduce kernel after each; TP-2
  // batch-1 decode 419.6 -> 435.9 tok/s fused)
  bool tp_fused = false;
  rxla::P2pView p2p{};
  // shard sizes
  int hq = 0, hkv = 0, inter = 0, vocab = 0, groups_h = 1, groups_i = 1, groups_o = 1;
  int64_t qkv_rows = 0;
  int group_h = 0, group_i = 0, group_o = 0;  // group sizes per input width
  uint8_t* arena = nullptr;
  size_t arena_bytes = 0;
  std::vector<rxla::dec::Param> params;
  std::vector<rxla::dec::Layer> layers;
  uint8_t* emb_w8 = nullptr;
  float* emb_scale = nullptr;
  uint16_t* emb_bf16 = nullptr;
  float* final_norm = nullptr;
  // cache
  int max_pages = 0;
  int32_t* page_table = nullptr;
  int32_t* ctx = nullptr;
  // activations
  float* h = nullptr;
  uint16_t* xn = nullptr;
  uint16_t* qkv = nullptr;
  uint16_t* att = nullptr;
  uint16_t* act = nullptr;
  float* part = nullptr;
  float* logits = nullptr;
  int32_t* tok_in = nullptr;
  int32_t* tok_out = nullptr;
  float* inv_freq = nullptr;
  void* ws = nullptr;
  size_t ws_bytes = 0;
  // tensor-parallel head: this rank's vocab slice and the argmax candidates
  int64_t vocab_local = 0;
  rxla::dec::Cand* cand = nullptr;      // [max_batch]
  rxla::dec::Cand* cand_all = nullptr;  // [tp][max_batch]
  // split-K workspace of the tcgen05 GEMM path (batch > 8)
  void* gws = nullptr;
  size_t gws_bytes = 0;
  // fused LM-head argmax: per-CTA partials and the arrival counter
  float* arg_val = nullptr;
  int32_t* arg_idx = nullptr;
  uint32_t* arg_count = nullptr;
  int32_t* host_pinned = nullptr;
  std::map<int, cudaGraphExec_t> graphs;
  // multi-token prefill: chunk buffers (rows = tokens of one prompt chunk),
  // allocated by the first rxla_b200_decoder_prefill
  int pf_chunk = 0;
  uint8_t* pf_mem = nullptr;
  float* pf_h = nullptr;
  uint16_t* pf_xn = nullptr;
  uint16_t* pf_qkv = nullptr;
  uint16_t* pf_att = nullptr;
  uint16_t* pf_act = nullptr;
  float* pf_part = nullptr;
  int32_t* pf_pt = nullptr;
  int32_t* pf_ctx = nullptr;
  void* pf_ws = nullptr;
  size_t pf_ws_bytes = 0;
  void* pf_gws = nullptr;
  size_t pf_gws_bytes = 0;
};

namespace rxla {
namespace dec {

// Batches above one skinny-GEMV pass run their linears on the tcgen05 GEMM.
constexpr int kSkinnyTokens = 8;

// Split-K depth of the decoder's GEMMs (w8_gemm_splits); the group size is
// the runner's for that input width.
static int gemm_splits(int64_t m, int64_t n, int64_t k, int64_t group, bool swiglu) {
  return w8_gemm_splits(m, n, k, group, swiglu);
}

static int32_t alloc_dev(void** p, size_t bytes) {
  cudaError_t e = cudaMalloc(p, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "decoder allocation");
  return RXLA_B200_OK;
}

// Row buffers of a batched pass through the layers: the decode step's
// (one row per sequence) or a prefill chunk's (one row per prompt token of a
// single sequence, each with its own copy of that sequence's page-table row
// and its own position).
struct Rows {
  int n;
  float* h;
  uint16_t* xn;
  uint16_t* qkv;
  uint16_t* att;
  uint16_t* act;
  float* part;
  void* gws;
  size_t gws_bytes;
  int32_t* page_table;
  int32_t* ctx;
  void* ws;
  size_t ws_bytes;
  bool prefill;
};

static Rows step_rows(rxla_b200_decoder* d, int batch) {
  return Rows{batch,     d->h,  d->xn,  d->qkv,      d->att, d->act,      d->part,
              d->gws,    d->gws_bytes,  d->page_table, d->ctx, d->ws, d->ws_bytes, false};
}

// Paged decode attention arguments of one layer of the runner.
static rxla_b200_paged_decode_args attention_args(const rxla_b200_decoder* d, const Layer& L,
                                                  int batch) {
  const auto& c = d->cfg;
  const int64_t D = c.head_dim;
  const int64_t qd = (int64_t)d->hq * D, kd = (int64_t)d->hkv * D;
  rxla_b200_paged_decode_args a{};
  a.struct_size = sizeof(a);
  a.batch = batch;
  a.q_heads = d->hq;
  a.kv_heads = d->hkv;
  a.head_dim = (int32_t)D;
  a.q = d->qkv;
  a.k_new = d->qkv + qd;
  a.v_new = d->qkv + qd + kd;
  a.q_row_stride = d->qkv_rows;
  a.kv_row_stride = d->qkv_rows;
  a.q_norm_weight = L.qn;
  a.k_norm_weight = L.kn;
  a.norm_eps = c.rms_eps;
  a.inv_freq = d->inv_freq;
  a.rotary_dim = (int32_t)D;
  a.scale = 0.0f;
  a.k_pages = L.kc;
  a.v_pages = L.vc;
  a.num_pages = (int64_t)c.max_batch * d->max_pages;
  a.page_size = 16;
  a.max_pages_per_seq = d->max_pages;
  a.page_table = d->page_table;
  a.pages_per_seq = nullptr;
  a.ctx_lens = d->ctx;
  a.kv_update = RXLA_B200_KV_CLAMP;
  a.advance_ctx = 0;
  a.accepted = nullptr;
  a.out = d->att;
  a.workspace = d->ws;
  a.workspace_bytes = d->ws_bytes;
  a.max_context = c.max_context;
  return a;
}

static rxla_b200_paged_decode_args attention_args(const rxla_b200_decoder* d, const Layer& L,
                                                  const Rows& r) {
  rxla_b200_paged_decode_args a = attention_args(d, L, r.n);
  const int64_t qd = (int64_t)d->hq * d->cfg.head_dim, kd = (int64_t)d->hkv * d->cfg.head_dim;
  a.q = r.qkv;
  a.k_new = r.qkv + qd;
  a.v_new = r.qkv + qd + kd;
  a.page_table = r.page_table;
  a.ctx_lens = r.ctx;
  a.out = r.att;
  a.workspace = r.ws;
  a.workspace_bytes = r.ws_bytes;
  return a;
}

// Tensor-parallel LM head: this rank's logits slice [batch, vocab_local] is in
// d->logits; pick its best per row, gather every rank's candidates, merge.
static int32_t tp_head_tail(rxla_b200_decoder* d, int batch, cudaStream_t s, int32_t* out,
                            int32_t* advance) {
  const int tp = d->cfg.tp_size;
  cudaError_t e = launch_pdl(argmax_candidates_kernel, dim3(batch), dim3(1024), 0, s,
                             (const float*)d->logits, d->vocab_local,
                             (int32_t)(d->cfg.tp_rank * d->vocab_local), d->cand);
  if (e != cudaSuccess) return cuda_fail(e, "argmax candidates launch");
  int32_t st = comm_allgather_bytes(d->comm, d->cand, d->cand_all, (int64_t)batch * sizeof(Cand), s);
  if (st) return st;
  e = launch_pdl(argmax_merge_kernel, dim3((batch + 127) / 128), dim3(128), 0, s,
                 (const Cand*)d->cand_all, (int32_t)tp, (int32_t)batch, out, advance);
  if (e != cudaSuccess) return cuda_fail(e, "argmax merge launch");
  return RXLA_B200_OK;
}

// h += bf16(part): the all-reduced row-parallel partial sums of o_proj / down.
static int32_t tp_residual(rxla_b200_decoder* d, int batch, cudaStream_t s, float* part,
                           float* h, bool p2p) {
  const int64_t H = d->cfg.hidden;
  // one-shot peer all-reduce fused with the residual add (its buffers hold
  // max_batch rows), else NCCL + a kernel
  if (p2p && d->use_p2p) return comm_p2p_allreduce(d->comm, part, h, batch * H, true, s);
  int32_t st = comm_allreduce_f32(d->comm, part, batch * H, s);
  if (st) return st;
  cudaError_t e = launch_pdl(residual_add_kernel, dim3(std::max(1, (int)((batch * H + 1023) / 1024))),
                             dim3(1024), 0, s, (const float*)part, h, (int64_t)batch * H);
  if (e != cudaSuccess) return cuda_fail(e, "residual add launch");
  return RXLA_B200_OK;
}

// The layers over a batch of rows: bf16 x from a separate RMSNorm kernel,
// the W8 linears (the tcgen05 GEMM with split-K over the rows' workspace;
// skinny passes for a prefill chunk of at most kSkinnyTokens rows), the same
// epilogues.  A prefill chunk's attention runs twice: an append-only pass
// writes every row's K/V to its slot, then the full pass lets row t attend
// over the sequence's cache up to its own slot (the causal mask of the
// prompt), re-writing identical K/V bytes.
static int32_t enqueue_rows_layers(rxla_b200_decoder* d, const Rows& r, cudaStream_t s) {
  const auto& c = d->cfg;
  const bool tp = c.tp_size > 1;
  const int64_t H = c.hidden, D = c.head_dim;
  const int64_t qd = (int64_t)d->hq * D;
  auto gemm = [&](const void* x, int64_t k, const uint8_t* w, const float* sc, int64_t group,
                  int64_t n, void* y, int32_t y_dtype, int32_t epi) {
    if (r.n <= kSkinnyTokens)
      return w8_linear(x, RXLA_B200_BF16, w, sc, group, r.n, n, k, y, y_dtype, epi, s, nullptr);
    GemmArgs g{};
    g.x = x;
    g.ldx = k;
    g.w = w;
    g.scale = sc;
    g.group = group;
    g.m = r.n;
    g.n = n;
    g.k = k;
    g.y = y;
    g.ldy = n;
    g.y_dtype = y_dtype;
    g.epilogue = epi;
    g.splits = gemm_splits(r.n, n, k, group, epi == RXLA_B200_EPI_SWIGLU);
    g.ws = r.gws;
    g.ws_bytes = r.gws_bytes;
    return w8_gemm(g, s);
  };
  for (int l = 0; l < c.layers; ++l) {
    const Layer& L = d->layers[l];
    int32_t st = rxla_b200_rms_norm_bf16(r.h, L.ln1, r.n, H, c.rms_eps, r.xn, s);
    if (!st) st = gemm(r.xn, H, L.wqkv, L.sqkv, d->group_h, d->qkv_rows, r.qkv, RXLA_B200_BF16,
                       RXLA_B200_EPI_STORE);
    if (st) return st;
    rxla_b200_paged_decode_args a = attention_args(d, L, r);
    if (r.prefill) {
      // positions were written before the layers; the causal pass reads the
      // pages only after the append pass has finished
      st = attn::launch(&a, s, true, nullptr, true);
      if (!st) st = attn::prefill_launch(&a, s);
    } else {
      st = attn::launch(&a, s, true);
    }
    // row-parallel linears: the full residual add, or (tensor parallel) an
    // unrounded partial that is all-reduced first
    if (!st) st = tp ? gemm(r.att, qd, L.wo, L.so, d->group_o, H, r.part, RXLA_B200_F32,
                            RXLA_B200_EPI_STORE)
                     : gemm(r.att, qd, L.wo, L.so, d->group_o, H, r.h, RXLA_B200_F32,
                            RXLA_B200_EPI_RESIDUAL_ADD);
    if (!st && tp) st = tp_residual(d, r.n, s, r.part, r.h, !r.prefill);
    if (!st) st = rxla_b200_rms_norm_bf16(r.h, L.ln2, r.n, H, c.rms_eps, r.xn, s);
    if (!st) st = gemm(r.xn, H, L.wgu, L.sgu, d->group_h, d->inter, r.act, RXLA_B200_BF16,
                       RXLA_B200_EPI_SWIGLU);
    if (!st) st = tp ? gemm(r.act, d->inter, L.wd, L.sd, d->group_i, H, r.part, RXLA_B200_F32,
                            RXLA_B200_EPI_STORE)
                     : gemm(r.act, d->inter, L.wd, L.sd, d->group_i, H, r.h, RXLA_B200_F32,
                            RXLA_B200_EPI_RESIDUAL_ADD);
    if (!st && tp) st = tp_residual(d, r.n, s, r.part, r.h, !r.prefill);
    if (st) return st;
  }
  return RXLA_B200_OK;
}

// Linears of a step with more tokens than one skinny pass: the layers over
// the step's rows; the LM head writes f32 logits and a per-row argmax kernel
// picks the token and advances the position.
static int32_t enqueue_gemm_layers(rxla_b200_decoder* d, int batch, cudaStream_t s) {
  const auto& c = d->cfg;
  const bool tp = c.tp_size > 1;
  const int64_t H = c.hidden;
  auto gemm = [&](const void* x, int64_t k, const uint8_t* w, const float* sc, int64_t group,
                  int64_t n, void* y, int32_t y_dtype, int32_t epi) {
    GemmArgs g{};
    g.x = x;
    g.ldx = k;
    g.w = w;
    g.scale = sc;
    g.group = group;
    g.m = batch;
    g.n = n;
    g.k = k;
    g.y = y;
    g.ldy = n;
    g.y_dtype = y_dtype;
    g.epilogue = epi;
    g.splits = gemm_splits(batch, n, k, group, epi == RXLA_B200_EPI_SWIGLU);
    g.ws = d->gws;
    g.ws_bytes = d->gws_bytes;
    return w8_gemm(g, s);
  };
  {
    int32_t st = enqueue_rows_layers(d, step_rows(d, batch), s);
    if (st) return st;
  }
  int32_t st = rxla_b200_rms_norm_bf16(d->h, d->final_norm, batch, H, c.rms_eps, d->xn, s);
  if (st) return st;
  // the head over this rank's vocab slice (all of it without tensor parallelism)
  const int64_t v0 = (int64_t)c.tp_rank * d->vocab_local;
  if (d->emb_w8) {
    st = gemm(d->xn, H, d->emb_w8 + v0 * H, d->emb_scale + v0 * d->groups_h, d->group_h,
              d->vocab_local, d->logits, RXLA_B200_F32, RXLA_B200_EPI_STORE);
  } else {
    st = rxla_b200_bf16_linear(d->xn, RXLA_B200_BF16, d->emb_bf16 + v0 * H, batch, d->vocab_local,
                               H, d->logits, RXLA_B200_F32, RXLA_B200_EPI_STORE, s);
  }
  if (st) return st;
  if (tp) return tp_head_tail(d, batch, s, d->tok_out, d->ctx);
  cudaError_t e = launch_pdl(argmax_kernel, dim3(batch), dim3(1024), 0, s, (const float*)d->logits,
                             (int64_t)d->vocab, d->tok_out, d->ctx);
  if (e != cudaSuccess) return cuda_fail(e, "argmax launch");
  return RXLA_B200_OK;
}

// One decode step for `batch` sequences, enqueued on `s` (graph-capturable).
static int32_t enqueue_step(rxla_b200_decoder* d, int batch, cudaStream_t s) {
  const auto& c = d->cfg;
  const int64_t H = c.hidden, D = c.head_dim;
  cudaError_t e = launch_pdl(embed_kernel, dim3(batch), dim3(256), 0, s, (const int32_t*)d->tok_in,
                             (const uint8_t*)d->emb_w8, (const float*)d->emb_scale,
                             (const __nv_bfloat16*)d->emb_bf16, (int64_t)c.vocab, H,
                             (int64_t)d->groups_h, (int64_t)d->group_h, d->h);
  if (e != cudaSuccess) return cuda_fail(e, "embed launch");
  const bool tp = c.tp_size > 1;
  if (batch > kSkinnyTokens && d->gws_bytes > 0 && d->group_h % 64 == 0 &&
      d->group_o % 64 == 0 && d->group_i % 64 == 0)
    return enqueue_gemm_layers(d, batch, s);
  const int64_t qd = (int64_t)d->hq * D;
  // each kernel pulls the start of the next weight matrix into L2 while it drains
  auto pf = [](const void* w, int64_t bytes, int32_t per_cta) {
    L2Prefetch f{};
    f.seg[0] = w;
    f.bytes[0] = bytes;
    f.nseg = 1;
    f.per_cta = per_cta;
    return f;
  };
  // bytes of the next kernel's weights each CTA pulls into L2 (measured on
  // the batch-1 step at 2048 context: 0 KB 2.49 ms, 96 KB 2.40, 192 KB 2.41,
  // 384 KB 2.50, 768 KB 2.61)
  constexpr int32_t kRingShare = 96 * 1024;
  for (int l = 0; l < c.layers; ++l) {
    const Layer& L = d->layers[l];
    const L2Prefetch to_o = pf(L.wo, H * qd, 256 * 1024);
    L2Prefetch to_gu = pf(L.wgu, d->inter * H, kRingShare);
    to_gu.seg[1] = L.wgu + d->inter * H;
    to_gu.bytes[1] = d->inter * H;
    to_gu.nseg = 2;
    const L2Prefetch to_down = pf(L.wd, H * d->inter, kRingShare);
    const L2Prefetch to_next =
        l + 1 < c.layers ? pf(d->layers[l + 1].wqkv, d->qkv_rows * H, kRingShare)
                         : (d->emb_w8 ? pf(d->emb_w8, d->vocab * H, kRingShare) : L2Prefetch{});
    // qkv = W8(bf16(rms_norm(h) * input_layernorm)), the norm fused in the prologue
    NormLinearArgs na{};
    na.h = d->h;
    na.norm_w = L.ln1;
    na.eps = c.rms_eps;
    na.w = L.wqkv;
    na.scale = L.sqkv;
    na.group = d->group_h;
    na.m = batch;
    na.n = d->qkv_rows;
    na.k = H;
    na.y = d->qkv;
    na.y_dtype = RXLA_B200_BF16;
    na.epilogue = RXLA_B200_EPI_STORE;
    na.next = to_o;
    int32_t st = w8_norm_linear(na, s);
    if (st) return st;
    rxla_b200_paged_decode_args a = attention_args(d, L, batch);
    st = attn::launch(&a, s, true, &to_o);
    if (st) return st;
    if (!tp) {
      st = w8_linear(d->att, RXLA_B200_BF16, L.wo, L.so, d->group_o, batch, H, qd, d->h,
                     RXLA_B200_F32, RXLA_B200_EPI_RESIDUAL_ADD, s, &to_gu);
      if (st) return st;
    } else if (d->tp_fused) {
      // o_proj partials all-reduced in the GEMV's epilogue, added to h
      st = w8_linear(d->att, RXLA_B200_BF16, L.wo, L.so, d->group_o, batch, H, qd, d->h,
                     RXLA_B200_F32, RXLA_B200_EPI_RESIDUAL_ADD, s, &to_gu, &d->p2p);
      if (st) return st;
    } else {
      st = rxla_b200_w8a16_linear(d->att, RXLA_B200_BF16, L.wo, L.so, d->group_o, batch, H, qd,
                                  d->part, RXLA_B200_F32, RXLA_B200_EPI_STORE, s);
      if (st) return st;
      st = tp_residual(d, batch, s, d->part, d->h, true);
      if (st) return st;
    }
    // act = silu(gate) * up of bf16(rms_norm(h) * post_attention_layernorm)
    na.norm_w = L.ln2;
    na.w = L.wgu;
    na.scale = L.sgu;
    na.n = d->inter;
    na.y = d->act;
    na.epilogue = RXLA_B200_EPI_SWIGLU;
    na.next = to_down;
    st = w8_norm_linear(na, s);
    if (st) return st;
    if (!tp) {
      st = w8_linear(d->act, RXLA_B200_BF16, L.wd, L.sd, d->group_i, batch, H, d->inter, d->h,
                     RXLA_B200_F32, RXLA_B200_EPI_RESIDUAL_ADD, s, &to_next);
      if (st) return st;
    } else if (d->tp_fused) {
      st = w8_linear(d->act, RXLA_B200_BF16, L.wd, L.sd, d->group_i, batch, H, d->inter, d->h,
                     RXLA_B200_F32, RXLA_B200_EPI_RESIDUAL_ADD, s, &to_next, &d->p2p);
      if (st) return st;
    } else {
      st = rxla_b200_w8a16_linear(d->act, RXLA_B200_BF16, L.wd, L.sd, d->group_i, batch, H,
                                  d->inter, d->part, RXLA_B200_F32, RXLA_B200_EPI_STORE, s);
      if (st) return st;
      st = tp_residual(d, batch, s, d->part, d->h, true);
      if (st) return st;
    }
  }
  if (tp) {
    // this rank's vocab slice of the tied head into d->logits, then the
    // cross-rank argmax
    const int64_t v0 = (int64_t)c.tp_rank * d->vocab_local;
    int32_t st;
    if (d->emb_w8) {
      NormLinearArgs na{};
      na.h = d->h;
      na.norm_w = d->final_norm;
      na.eps = c.rms_eps;
      na.w = d->emb_w8 + v0 * H;
      na.scale = d->emb_scale + v0 * d->groups_h;
      na.group = d->group_h;
      na.m = batch;
      na.n = d->vocab_local;
      na.k = H;
      na.y = d->logits;
      na.y_dtype = RXLA_B200_F32;
      na.epilogue = RXLA_B200_EPI_STORE;
      st = w8_norm_linear(na, s);
    } else {
      st = rxla_b200_rms_norm_bf16(d->h, d->final_norm, batch, H, c.rms_eps, d->xn, s);
      if (!st)
        st = rxla_b200_bf16_linear(d->xn, RXLA_B200_BF16, d->emb_bf16 + v0 * H, batch,
                                   d->vocab_local, H, d->logits, RXLA_B200_F32,
                                   RXLA_B200_EPI_STORE, s);
    }
    if (st) return st;
    return tp_head_tail(d, batch, s, d->tok_out, d->ctx);
  }
  if (d->emb_w8) {
    // tied W8 head: logits = bf16(rms_norm(h) * norm) · Eᵀ (f32), greedy token
    // and the position advance in the same kernel
    NormLinearArgs na{};
    na.h = d->h;
    na.norm_w = d->final_norm;
    na.eps = c.rms_eps;
    na.w = d->emb_w8;
    na.scale = d->emb_scale;
    na.group = d->group_h;
    na.m = batch;
    na.n = d->vocab;
    na.k = H;
    na.y = d->logits;
    na.y_dtype = RXLA_B200_F32;
    na.epilogue = kArgmaxEpilogue;
    na.arg_val = d->arg_val;
    na.arg_idx = d->arg_idx;
    na.arg_count = d->arg_count;
    na.arg_out = d->tok_out;
    na.arg_advance = d->ctx;
    if (c.layers > 0) {  // the next step starts with layer 0's qkv
      na.next.seg[0] = d->layers[0].wqkv;
      na.next.bytes[0] = d->qkv_rows * H;
      na.next.nseg = 1;
      na.next.per_cta = kRingShare;
    }
    return w8_norm_linear(na, s);
  }
  int32_t st = rxla_b200_rms_norm_bf16(d->h, d->final_norm, batch, H, c.rms_eps, d->xn, s);
  if (st) return st;
  st = rxla_b200_bf16_linear(d->xn, RXLA_B200_BF16, d->emb_bf16, batch, d->vocab, H, d->logits,
                             RXLA_B200_F32, RXLA_B200_EPI_STORE, s);
  if (st) return st;
  e = launch_pdl(argmax_kernel, dim3(batch), dim3(1024), 0, s, (const float*)d->logits,
                 (int64_t)d->vocab, d->tok_out, d->ctx);
  if (e != cudaSuccess) return cuda_fail(e, "argmax launch");
  return RXLA_B200_OK;
}

}  // namespace dec
}  // namespace rxla

using namespace rxla;

extern "C" int32_t rxla_b200_decoder_create(const rxla_b200_decoder_config* cfg, int32_t device,
                                            rxla_b200_comm* comm, rxla_b200_decoder** out) {
  RXLA_REQUIRE(cfg && out && cfg->struct_size >= sizeof(rxla_b200_decoder_config),
               "decoder_create: config struct missing or too small");
  const auto& c = *cfg;
  RXLA_REQUIRE(c.layers > 0 && c.hidden > 0 && c.q_heads > 0 && c.kv_heads > 0 &&
                   c.head_dim > 0 && c.intermediate > 0 && c.vocab > 0,
               "decoder_create: sizes must be positive");
  RXLA_REQUIRE(c.q_heads % c.kv_heads == 0, "decoder_create: q_heads % kv_heads != 0");
  RXLA_REQUIRE(c.rms_eps > 0.0f && std::isfinite(c.rms_eps), "decoder_create: bad rms_eps");
  RXLA_REQUIRE(c.rope_theta > 0.0f && std::isfinite(c.rope_theta), "decoder_create: bad rope_theta");
  RXLA_REQUIRE(c.embedding_dtype == RXLA_B200_U8 || c.embedding_dtype == RXLA_B200_BF16,
               "decoder_create: embedding_dtype must be U8 or BF16");
  RXLA_REQUIRE(c.max_batch > 0 && c.max_context > 0, "decoder_create: max_batch / max_context");
  const int tp = c.tp_size <= 0 ? 1 : c.tp_size;
  RXLA_REQUIRE(c.tp_rank >= 0 && c.tp_rank < tp, "decoder_create: tp_rank out of range");
  RXLA_REQUIRE(c.kv_heads % tp == 0 && c.intermediate % tp == 0,
               "decoder_create: kv_heads and intermediate must divide by tp_size");
  RXLA_REQUIRE(tp == 1 || comm, "decoder_create: tensor parallel needs a comm");
  RXLA_REQUIRE(c.vocab % tp == 0, "decoder_create: vocab must divide by tp_size (sharded head)");
  const int gsz = c.group_size;
  auto groups_for = [&](int64_t k) -> int64_t { return gsz > 0 ? k / gsz : 1; };
  RXLA_REQUIRE(gsz <= 0 || (c.hidden % gsz == 0 && (c.q_heads * c.head_dim / tp) % gsz == 0 &&
                            (c.intermediate / tp) % gsz == 0),
               "decoder_create: group_size must divide every input width");
  RXLA_REQUIRE(c.head_dim == 64 || c.head_dim == 128, "decoder: head_dim must be 64 or 128");
  RXLA_REQUIRE(c.hidden % 64 == 0 && (c.q_heads * c.head_dim / tp) % 64 == 0 &&
                   (c.intermediate / tp) % 64 == 0 && (gsz <= 0 || gsz % 64 == 0),
               "decoder_create: hidden, q_heads*head_dim, intermediate (and group_size) must be "
               "multiples of 64");
  RXLA_CUDA_CHECK(cudaSetDevice(device));

  auto* d = new rxla_b200_decoder();
  d->cfg = c;
  d->cfg.tp_size = tp;
  d->device = device;
  d->comm = comm;
  d->hq = c.q_heads / tp;
  d->hkv = c.kv_heads / tp;
  d->inter = c.intermediate / tp;
  d->vocab = c.vocab;
  d->vocab_local = c.vocab / tp;
  const int64_t H = c.hidden, D = c.head_dim, I = d->inter;
  d->qkv_rows = (int64_t)(d->hq + 2 * d->hkv) * D;
  d->groups_h = (int)groups_for(H);
  d->groups_o = (int)groups_for((int64_t)d->hq * D);
  d->groups_i = (int)groups_for(I);
  d->group_h = gsz > 0 ? gsz : (int)H;
  d->group_o = gsz > 0 ? gsz : (int)(d->hq * D);
  d->group_i = gsz > 0 ? gsz : (int)I;
  d->max_pages = (c.max_context + 15) / 16;

  // ---- parameter arena (256-byte aligned views)
  struct Spec {
    std::string name;
    int64_t bytes;
    int32_t dtype;
  };
  std::vector<Spec> specs;
  auto add = [&](const std::string& n, int64_t bytes, int32_t dt) { specs.push_back({n, bytes, dt}); };
  const bool w8emb = c.embedding_dtype == RXLA_B200_U8;
  if (w8emb) {
    add("embed_tokens.weight", (int64_t)c.vocab * H, RXLA_B200_U8);
    add("embed_tokens.scale", (int64_t)c.vocab * d->groups_h * 4, RXLA_B200_F32);
  } else {
    add("embed_tokens.weight", (int64_t)c.vocab * H * 2, RXLA_B200_BF16);
  }
  for (int l = 0; l < c.layers; ++l) {
    const std::string p = "layers." + std::to_string(l) + ".";
    add(p + "input_layernorm.weight", H * 4, RXLA_B200_F32);
    add(p + "self_attn.qkv.weight", d->qkv_rows * H, RXLA_B200_U8);
    add(p + "self_attn.qkv.scale", d->qkv_rows * d->groups_h * 4, RXLA_B200_F32);
    add(p + "self_attn.q_norm.weight", D * 4, RXLA_B200_F32);
    add(p + "self_attn.k_norm.weight", D * 4, RXLA_B200_F32);
    add(p + "self_attn.o_proj.weight", H * d->hq * D, RXLA_B200_U8);
    add(p + "self_attn.o_proj.scale", H * d->groups_o * 4, RXLA_B200_F32);
    add(p + "post_attention_layernorm.weight", H * 4, RXLA_B200_F32);
    add(p + "mlp.gate_up.weight", 2 * I * H, RXLA_B200_U8);
    add(p + "mlp.gate_up.scale", 2 * I * d->groups_h * 4, RXLA_B200_F32);
    add(p + "mlp.down_proj.weight", H * I, RXLA_B200_U8);
    add(p + "mlp.down_proj.scale", H * d->groups_i * 4, RXLA_B200_F32);
  }
  add("norm.weight", H * 4, RXLA_B200_F32);
  size_t total = 0;
  for (auto& sp : specs) total += (size_t)((sp.bytes + 255) / 256 * 256);
  int32_t st = dec::alloc_dev(reinterpret_cast<void**>(&d->arena), total);
  if (st) {
    delete d;
    return st;
  }
  d->arena_bytes = total;
  size_t off = 0;
  for (auto& sp : specs) {
    d->params.push_back({sp.name, d->arena + off, sp.bytes, sp.dtype});
    off += (size_t)((sp.bytes + 255) / 256 * 256);
  }
  auto find = [&](const std::string& n) -> void* {
    for (auto& p : d->params)
      if (p.name == n) return p.ptr;
    return nullptr;
  };
  if (w8emb) {
    d->emb_w8 = static_cast<uint8_t*>(find("embed_tokens.weight"));
    d->emb_scale = static_cast<float*>(find("embed_tokens.scale"));
  } else {
    d->emb_bf16 = static_cast<uint16_t*>(find("embed_tokens.weight"));
  }
  d->final_norm = static_cast<float*>(find("norm.weight"));
  // ---- KV cache (per layer), page table, activations
  const int64_t pages = (int64_t)c.max_batch * d->max_pages;
  const size_t cache_bytes = (size_t)pages * d->hkv * 16 * D * 2;
  d->layers.resize(c.layers);
  for (int l = 0; l < c.layers; ++l) {
    const std::string p = "layers." + std::to_string(l) + ".";
    dec::Layer& L = d->layers[l];
    L.ln1 = static_cast<float*>(find(p + "input_layernorm.weight"));
    L.ln2 = static_cast<float*>(find(p + "post_attention_layernorm.weight"));
    L.wqkv = static_cast<uint8_t*>(find(p + "self_attn.qkv.weight"));
    L.sqkv = static_cast<float*>(find(p + "self_attn.qkv.scale"));
    L.qn = static_cast<float*>(find(p + "self_attn.q_norm.weight"));
    L.kn = static_cast<float*>(find(p + "self_attn.k_norm.weight"));
    L.wo = static_cast<uint8_t*>(find(p + "self_attn.o_proj.weight"));
    L.so = static_cast<float*>(find(p + "self_attn.o_proj.scale"));
    L.wgu = static_cast<uint8_t*>(find(p + "mlp.gate_up.weight"));
    L.sgu = static_cast<float*>(find(p + "mlp.gate_up.scale"));
    L.wd = static_cast<uint8_t*>(find(p + "mlp.down_proj.weight"));
    L.sd = static_cast<float*>(find(p + "mlp.down_proj.scale"));
    st = dec::alloc_dev(reinterpret_cast<void**>(&L.kc), cache_bytes);
    if (!st) st = dec::alloc_dev(reinterpret_cast<void**>(&L.vc), cache_bytes);
    if (st) {
      rxla_b200_decoder_destroy(d);
      return st;
    }
  }
  const int64_t B = c.max_batch;
  size_t need_ws = 0;
  rxla_b200_paged_decode_workspace_size(c.max_batch, d->hq, d->hkv, (int32_t)D, c.max_context,
                                        &need_ws);
  d->ws_bytes = need_ws;
  if (B > dec::kSkinnyTokens) {
    size_t g = 0;
    const int64_t shapes[][4] = {{d->qkv_rows, H, 0, d->group_h},
                                 {H, (int64_t)d->hq * D, 0, d->group_o},
                                 {(int64_t)I, H, 1, d->group_h},
                                 {H, (int64_t)I, 0, d->group_i},
                                 {d->vocab_local, H, 0, d->group_h}};
    for (auto& sh : shapes)
      g = std::max(g, w8_gemm_workspace_bytes(B, sh[2] ? 2 * sh[0] : sh[0],
                                              dec::gemm_splits(B, sh[0], sh[1], sh[3], sh[2] != 0)));
    d->gws_bytes = g;
  }
  struct A {
    void** p;
    size_t bytes;
  } acts[] = {
      {(void**)&d->page_table, (size_t)B * d->max_pages * 4},
      {(void**)&d->ctx, (size_t)B * 4},
      {(void**)&d->h, (size_t)B * H * 4},
      {(void**)&d->xn, (size_t)B * H * 2},
      {(void**)&d->qkv, (size_t)B * d->qkv_rows * 2},
      {(void**)&d->att, (size_t)B * d->hq * D * 2},
      {(void**)&d->act, (size_t)B * I * 2},
      {(void**)&d->part, (size_t)B * H * 4},
      {(void**)&d->logits, (size_t)B * d->vocab_local * 4},
      {(void**)&d->cand, (size_t)B * sizeof(dec::Cand)},
      {(void**)&d->cand_all, (size_t)tp * B * sizeof(dec::Cand)},
      {(void**)&d->tok_in, (size_t)B * 4},
      {(void**)&d->tok_out, (size_t)B * 4},
      {(void**)&d->inv_freq, (size_t)D * 2},
      {&d->ws, need_ws},
      {&d->gws, d->gws_bytes},
      {(void**)&d->arg_val, (size_t)1024 * 8 * 4},
      {(void**)&d->arg_idx, (size_t)1024 * 8 * 4},
      {(void**)&d->arg_count, 256},
  };
  for (auto& a : acts) {
    st = dec::alloc_dev(a.p, std::max<size_t>(a.bytes, 256));
    if (st) {
      rxla_b200_decoder_destroy(d);
      return st;
    }
  }
  if (cudaMallocHost(reinterpret_cast<void**>(&d->host_pinned), (size_t)B * 8) != cudaSuccess) {
    rxla_b200_decoder_destroy(d);
    return fail(RXLA_B200_RESOURCE_EXHAUSTED, "decoder_create: pinned staging");
  }
  // page table: sequence b owns pages [b * max_pages, (b+1) * max_pages)
  std::vector<int32_t> pt((size_t)B * d->max_pages);
  for (size_t i = 0; i < pt.size(); ++i) pt[i] = (int32_t)i;
  // RoPE frequencies on the host in f32, as qwen3_5/mod.rs:213-222 computes them
  std::vector<float> inv((size_t)D / 2);
  for (int64_t i = 0; i < D / 2; ++i)
    inv[(size_t)i] = std::pow(c.rope_theta, (-2.0f * (float)i) / (float)D);
  if (cudaMemcpy(d->page_table, pt.data(), pt.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(d->inv_freq, inv.data(), inv.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemset(d->ctx, 0, (size_t)B * 4) != cudaSuccess ||
      cudaMemset(d->ws, 0, need_ws) != cudaSuccess ||
      // the split-K GEMMs' arrival counters sit at the head of gws and must
      // start at zero (every launch leaves them zero again)
      (d->gws && cudaMemset(d->gws, 0, std::max<size_t>(d->gws_bytes, 256)) != cudaSuccess) ||
      cudaMemset(d->arg_count, 0, 256) != cudaSuccess ||
      cudaMemset(d->arena, 0, d->arena_bytes) != cudaSuccess) {
    rxla_b200_decoder_destroy(d);
    return fail(RXLA_B200_UNAVAILABLE, "decoder_create: initial copies failed");
  }
  for (auto& L : d->layers) {
    cudaMemset(L.kc, 0, cache_bytes);
    cudaMemset(L.vc, 0, cache_bytes);
  }
  RXLA_CUDA_CHECK(cudaDeviceSynchronize());
  if (tp > 1) {
    // row-parallel all-reduces over NVLink peer memory (collective; every rank
    // ends up on the same path).  RXLA_B200_P2P=0 keeps NCCL.
    const char* pv = getenv("RXLA_B200_P2P");
    if (!(pv && pv[0] == '0') &&
        rxla_b200_comm_p2p_enable(comm, (int64_t)c.max_batch * H) != RXLA_B200_OK)
      cudaGetLastError();  // NCCL path
    // the peer buffers may have been enabled earlier, by a decoder with a
    // smaller batch or width: this decoder uses them only when its
    // all-reduces fit (the same answer on every rank, whose decoders and
    // comm capacity are the same)
    d->use_p2p = comm_p2p_capacity(comm) >= (int64_t)c.max_batch * H;
    const char* fv = getenv("RXLA_B200_TP_FUSED");
    d->tp_fused = d->use_p2p && comm_p2p_view(comm, &d->p2p) && !(fv && fv[0] == '0');
  }
  *out = d;
  return RXLA_B200_OK;
}

extern "C" int32_t rxla_b200_decoder_destroy(rxla_b200_decoder* d) {
  if (!d) return RXLA_B200_OK;
  cudaSetDevice(d->device);
  for (auto& g : d->graphs) cudaGraphExecDestroy(g.second);
  for (auto& L : d->layers) {
    cudaFree(L.kc);
    cudaFree(L.vc);
  }
  void* ptrs[] = {d->arena, d->page_table, d->ctx, d->h, d->xn, d->qkv, d->att, d->act,
                  d->part, d->logits, d->tok_in, d->tok_out, d->inv_freq, d->ws,
                  d->gws, d->arg_val, d->arg_idx, d->arg_count, d->cand, d->cand_all,
                  d->pf_mem};
  for (void* p : ptrs) cudaFree(p);
  if (d->host_pinned) cudaFreeHost(d->host_pinned);
  delete d;
  return RXLA_B200_OK;
}

extern "C" int32_t rxla_b200_decoder_parameter(rxla_b200_decoder* d, const char* name,
                                               void** ptr, int64_t* bytes, int32_t* dtype) {
  RXLA_REQUIRE(d && name && ptr, "decoder_parameter: null argument");
  const std::string n(name);
  const auto& c = d->cfg;
  const int64_t H = c.hidden, D = c.head_dim;
  // q_proj / k_proj / v_proj are row ranges of the fused qkv weight, gate/up of gate_up
  auto sub = [&](const std::string& fused, int64_t row0, int64_t rows, int64_t row_bytes) -> int32_t {
    for (auto& p : d->params)
      if (p.name == fused) {
        *ptr = static_cast<uint8_t*>(p.ptr) + row0 * row_bytes;
        if (bytes) *bytes = rows * row_bytes;
        if (dtype) *dtype = p.dtype;
        return RXLA_B200_OK;
      }
    return fail(RXLA_B200_NOT_FOUND, "decoder_parameter: no parameter " + n);
  };
  for (auto& p : d->params)
    if (p.name == n) {
      *ptr = p.ptr;
      if (bytes) *bytes = p.bytes;
      if (dtype) *dtype = p.dtype;
      return RXLA_B200_OK;
    }
  const auto dot = n.rfind('.');
  const auto proj = n.rfind('.', dot - 1);
  if (dot != std::string::npos && proj != std::string::npos) {
    const std::string prefix = n.substr(0, proj), which = n.substr(proj + 1, dot - proj - 1),
                      kind = n.substr(dot + 1);
    const bool is_w = kind == "weight", is_s = kind == "scale";
    if (is_w || is_s) {
      const int64_t rb_w = H, rb_s = (int64_t)d->groups_h * 4;
      const int64_t rb = is_w ? rb_w : rb_s;
      const int64_t qd = (int64_t)d->hq * D, kd = (int64_t)d->hkv * D;
      if (which == "q_proj") return sub(prefix + ".qkv." + kind, 0, qd, rb);
      if (which == "k_proj") return sub(prefix + ".qkv." + kind, qd, kd, rb);
      if (which == "v_proj") return sub(prefix + ".qkv." + kind, qd + kd, kd, rb);
      if (which == "gate_proj") return sub(prefix + ".gate_up." + kind, 0, d->inter, rb);
      if (which == "up_proj") return sub(prefix + ".gate_up." + kind, d->inter, d->inter, rb);
    }
  }
  return fail(RXLA_B200_NOT_FOUND, "decoder_parameter: no parameter " + n);
}

extern "C" int32_t rxla_b200_decoder_set_parameter(rxla_b200_decoder* d, const char* name,
                                                   const void* host, int64_t bytes) {
  RXLA_REQUIRE(d && name && host, "decoder_set_parameter: null argument");
  void* ptr = nullptr;
  int64_t have = 0;
  int32_t dt = 0;
  int32_t st = rxla_b200_decoder_parameter(d, name, &ptr, &have, &dt);
  if (st) return st;
  RXLA_REQUIRE(have == bytes, std::string("decoder_set_parameter: ") + name + " holds " +
                                  std::to_string(have) + " bytes, got " + std::to_string(bytes));
  RXLA_CUDA_CHECK(cudaSetDevice(d->device));
  RXLA_CUDA_CHECK(cudaMemcpy(ptr, host, (size_t)bytes, cudaMemcpyHostToDevice));
  return RXLA_B200_OK;
}

extern "C" int32_t rxla_b200_decoder_init_synthetic(rxla_b200_decoder* d, uint64_t seed) {
  RXLA_REQUIRE(d, "decoder_init_synthetic: null decoder");
  RXLA_CUDA_CHECK(cudaSetDevice(d->device));
  const int grid = sm_count(d->device) * 8;
  uint64_t idx = 0;
  for (size_t i = 0; i < d->params.size(); ++i, ++idx) {
    auto& p = d->params[i];
    const uint64_t s = seed * 1000003ull + idx;
    if (p.dtype == RXLA_B200_U8) {
      // the scale is the next parameter; rows = scale elements / groups
      auto& sc = d->params[i + 1];
      const int64_t k = (p.name.find("down_proj") != std::string::npos)
                            ? d->inter
                            : (p.name.find("o_proj") != std::string::npos ? (int64_t)d->hq * d->cfg.head_dim
                                                                           : d->cfg.hidden);
      const int64_t rows = p.bytes / k;
      const int64_t groups = sc.bytes / 4 / rows;
      // this rank's slice of the full matrix
      const int r = d->cfg.tp_rank, tp = d->cfg.tp_size;
      const int64_t H = d->cfg.hidden, D = d->cfg.head_dim;
      const int64_t hq = d->hq, hkv = d->hkv, I = d->inter;
      dec::Shard sh{};
      sh.k_full = k;
      sh.nseg = 1;
      sh.seg_rows[0] = rows;
      if (p.name.find("self_attn.qkv") != std::string::npos) {  // [q; k; v] of local heads
        sh.nseg = 3;
        sh.seg_rows[0] = hq * D;
        sh.seg_full_row[0] = r * hq * D;
        sh.seg_rows[1] = hkv * D;
        sh.seg_full_row[1] = tp * hq * D + r * hkv * D;
        sh.seg_rows[2] = hkv * D;
        sh.seg_full_row[2] = tp * (hq + hkv) * D + r * hkv * D;
      } else if (p.name.find("o_proj") != std::string::npos) {  // columns of local heads
        sh.k_full = tp * hq * D;
        sh.col_off = r * hq * D;
      } else if (p.name.find("gate_up") != std::string::npos) {  // [gate; up] of local slice
        sh.nseg = 2;
        sh.seg_rows[0] = I;
        sh.seg_full_row[0] = r * I;
        sh.seg_rows[1] = I;
        sh.seg_full_row[1] = tp * I + r * I;
      } else if (p.name.find("down_proj") != std::string::npos) {  // columns of local slice
        sh.k_full = tp * I;
        sh.col_off = r * I;
      }
      (void)H;
      dec::fill_w8_kernel<<<grid, 256>>>(static_cast<uint8_t*>(p.ptr), static_cast<float*>(sc.ptr),
                                         rows, k, groups, s, sh);
    } else if (p.dtype == RXLA_B200_BF16) {
      dec::fill_bf16_kernel<<<grid, 256>>>(static_cast<__nv_bfloat16*>(p.ptr), p.bytes / 2, s);
    } else if (p.name.find(".scale") == std::string::npos) {
      dec::fill_norm_kernel<<<grid, 256>>>(static_cast<float*>(p.ptr), p.bytes / 4, s);
    }
  }
  RXLA_CUDA_CHECK(cudaGetLastError());
  RXLA_CUDA_CHECK(cudaDeviceSynchronize());
  return RXLA_B200_OK;
}

extern "C" int32_t rxla_b200_decoder_reset(rxla_b200_decoder* d, void* stream) {
  RXLA_REQUIRE(d, "decoder_reset: null decoder");
  RXLA_CUDA_CHECK(cudaMemsetAsync(d->ctx, 0, (size_t)d->cfg.max_batch * 4,
                                  static_cast<cudaStream_t>(stream)));
  return RXLA_B200_OK;
}

extern "C" int32_t rxla_b200_decoder_kv_cache(rxla_b200_decoder* d, int32_t layer, void** k,
                                              void** v, int64_t* bytes) {
  RXLA_REQUIRE(d && layer >= 0 && layer < d->cfg.layers, "decoder_kv_cache: bad layer");
  if (k) *k = d->layers[layer].kc;
  if (v) *v = d->layers[layer].vc;
  if (bytes)
    *bytes = (int64_t)d->cfg.max_batch * d->max_pages * d->hkv * 16 * d->cfg.head_dim * 2;
  return RXLA_B200_OK;
}

extern "C" int32_t rxla_b200_decoder_context_lengths(rxla_b200_decoder* d, const int32_t** lens) {
  RXLA_REQUIRE(d && lens, "decoder_context_lengths: null argument");
  *lens = d->ctx;
  return RXLA_B200_OK;
}

extern "C" int32_t rxla_b200_decoder_set_context_lengths(rxla_b200_decoder* d,
                                                         const int32_t* lens_host, int32_t count,
                                                         void* stream) {
  RXLA_REQUIRE(d && lens_host, "decoder_set_context_lengths: null argument");
  RXLA_REQUIRE(count >= 0 && count <= d->cfg.max_batch,
               "decoder_set_context_lengths: count out of range");
  for (int32_t b = 0; b < count; ++b)
    RXLA_REQUIRE(lens_host[b] >= 0 && lens_host[b] < d->cfg.max_context,
                 "decoder_set_context_lengths: length must leave room for the next token");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  RXLA_CUDA_CHECK(cudaSetDevice(d->device));
  if (count == 0) return RXLA_B200_OK;
  // staged through the pinned buffer so the copy is stream-ordered
  RXLA_CUDA_CHECK(cudaStreamSynchronize(s));
  std::memcpy(d->host_pinned, lens_host, (size_t)count * 4);
  RXLA_CUDA_CHECK(cudaMemcpyAsync(d->ctx, d->host_pinned, (size_t)count * 4,
                                  cudaMemcpyHostToDevice, s));
  RXLA_CUDA_CHECK(cudaStreamSynchronize(s));
  return RXLA_B200_OK;
}

extern "C" int32_t rxla_b200_decoder_step(rxla_b200_decoder* d, const int32_t* tokens,
                                          int32_t batch, int32_t* next_tokens, float* logits,
                                          void* stream) {
  RXLA_REQUIRE(d && tokens && next_tokens, "decoder_step: null argument");
  RXLA_REQUIRE(batch > 0 && batch <= d->cfg.max_batch, "decoder_step: batch out of range");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  RXLA_CUDA_CHECK(cudaSetDevice(d->device));
  if (tokens != d->tok_in)
    RXLA_CUDA_CHECK(cudaMemcpyAsync(d->tok_in, tokens, (size_t)batch * 4,
                                    cudaMemcpyDeviceToDevice, s));
  // RXLA_B200_NO_GRAPH=1: launch the step's kernels directly on `stream`
  // (for profilers that attribute work per kernel launch)
  static const bool no_graph = [] {
    const char* v = getenv("RXLA_B200_NO_GRAPH");
    return v && v[0] == '1';
  }();
  if (no_graph) {
    int32_t st = dec::enqueue_step(d, batch, s);
    if (st) return st;
    if (next_tokens != d->tok_out)
      RXLA_CUDA_CHECK(cudaMemcpyAsync(next_tokens, d->tok_out, (size_t)batch * 4,
                                      cudaMemcpyDeviceToDevice, s));
    if (logits)
      RXLA_CUDA_CHECK(cudaMemcpyAsync(logits, d->logits, (size_t)batch * d->vocab_local * 4,
                                      cudaMemcpyDeviceToDevice, s));
    return RXLA_B200_OK;
  }
  auto it = d->graphs.find(batch);
  if (it == d->graphs.end()) {
    // first use of this batch size: one eager step (sets kernel attributes and
    // resolves driver entry points outside capture) would advance the state,
    // so capture directly on a private stream and launch the graph.
    cudaStream_t cs;
    RXLA_CUDA_CHECK(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking));
    cudaGraph_t graph = nullptr;
    cudaError_t e = cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal);
    int32_t st = e == cudaSuccess ? dec::enqueue_step(d, batch, cs) : cuda_fail(e, "begin capture");
    cudaError_t e2 = cudaStreamEndCapture(cs, &graph);
    cudaStreamDestroy(cs);
    if (st) {
      if (graph) cudaGraphDestroy(graph);
      return st;
    }
    if (e2 != cudaSuccess) return cuda_fail(e2, "end capture");
    cudaGraphExec_t exec = nullptr;
    e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) return cuda_fail(e, "graph instantiate");
    it = d->graphs.emplace(batch, exec).first;
  }
  RXLA_CUDA_CHECK(cudaGraphLaunch(it->second, s));
  if (next_tokens != d->tok_out)
    RXLA_CUDA_CHECK(cudaMemcpyAsync(next_tokens, d->tok_out, (size_t)batch * 4,
                                    cudaMemcpyDeviceToDevice, s));
  if (logits)
    RXLA_CUDA_CHECK(cudaMemcpyAsync(logits, d->logits, (size_t)batch * d->vocab_local * 4,
                                    cudaMemcpyDeviceToDevice, s));
  return RXLA_B200_OK;
}

namespace rxla {
namespace dec {

// Prefill chunk rows (RXLA_B200_PREFILL_CHUNK, default 2048, at most
// max_context): buffers for that many rows are allocated once.
static int32_t prefill_alloc(rxla_b200_decoder* d) {
  if (d->pf_mem) return RXLA_B200_OK;
  const auto& c = d->cfg;
  const char* v = getenv("RXLA_B200_PREFILL_CHUNK");
  int C = v ? atoi(v) : 2048;
  C = std::max(1, std::min(C, c.max_context));
  const int64_t H = c.hidden, D = c.head_dim, I = d->inter;
  // workspaces: the largest any chunk of 1..C rows plans
  size_t ws = 0, gws = 0;
  const int64_t shapes[][4] = {{d->qkv_rows, H, 0, d->group_h},
                               {H, (int64_t)d->hq * D, 0, d->group_o},
                               {I, H, 1, d->group_h},
                               {H, I, 0, d->group_i}};
  for (int n = 1; n <= C; ++n) {
    size_t w = 0;
    rxla_b200_paged_decode_workspace_size(n, d->hq, d->hkv, (int32_t)D, c.max_context, &w);
    ws = std::max(ws, w);
    if (n <= kSkinnyTokens) continue;
    for (auto& sh : shapes)
      gws = std::max(gws, w8_gemm_workspace_bytes(n, sh[2] ? 2 * sh[0] : sh[0],
                                                  gemm_splits(n, sh[0], sh[1], sh[3], sh[2] != 0)));
  }
  const size_t sizes[] = {(size_t)C * H * 4,           (size_t)C * H * 2,
                          (size_t)C * d->qkv_rows * 2, (size_t)C * d->hq * D * 2,
                          (size_t)C * I * 2,           (size_t)C * H * 4,
                          (size_t)C * d->max_pages * 4, (size_t)C * 4,
                          ws,                          gws};
  size_t off[10], total = 0;
  for (int i = 0; i < 10; ++i) {
    off[i] = total;
    total += (std::max<size_t>(sizes[i], 1) + 255) / 256 * 256;
  }
  int32_t st = alloc_dev(reinterpret_cast<void**>(&d->pf_mem), total);
  if (st) return st;
  RXLA_CUDA_CHECK(cudaMemset(d->pf_mem, 0, total));
  uint8_t* b = d->pf_mem;
  d->pf_h = reinterpret_cast<float*>(b + off[0]);
  d->pf_xn = reinterpret_cast<uint16_t*>(b + off[1]);
  d->pf_qkv = reinterpret_cast<uint16_t*>(b + off[2]);
  d->pf_att = reinterpret_cast<uint16_t*>(b + off[3]);
  d->pf_act = reinterpret_cast<uint16_t*>(b + off[4]);
  d->pf_part = reinterpret_cast<float*>(b + off[5]);
  d->pf_pt = reinterpret_cast<int32_t*>(b + off[6]);
  d->pf_ctx = reinterpret_cast<int32_t*>(b + off[7]);
  d->pf_ws = b + off[8];
  d->pf_ws_bytes = ws;
  d->pf_gws = gws ? b + off[9] : nullptr;
  d->pf_gws_bytes = gws;
  d->pf_chunk = C;
  return RXLA_B200_OK;
}

}  // namespace dec
}  // namespace rxla

extern "C" int32_t rxla_b200_decoder_prefill(rxla_b200_decoder* d, int32_t seq,
                                             const int32_t* tokens, int32_t count,
                                             int32_t* next_token, float* logits, void* stream) {
  RXLA_REQUIRE(d && tokens, "decoder_prefill: null argument");
  RXLA_REQUIRE(seq >= 0 && seq < d->cfg.max_batch, "decoder_prefill: sequence out of range");
  RXLA_REQUIRE(count > 0, "decoder_prefill: count must be positive");
  const auto& c = d->cfg;
  const int64_t H = c.hidden;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  RXLA_CUDA_CHECK(cudaSetDevice(d->device));
  {
    // the embedding kernel reads the prompt directly: ordinary (unregistered)
    // host memory would be an illegal address there, so refuse it here
    cudaPointerAttributes pa{};
    const cudaError_t e = cudaPointerGetAttributes(&pa, tokens);
    if (e != cudaSuccess) cudaGetLastError();
    RXLA_REQUIRE(e == cudaSuccess && pa.type != cudaMemoryTypeUnregistered,
                 "decoder_prefill: tokens must be device, managed or pinned host memory");
  }
  int32_t st = dec::prefill_alloc(d);
  if (st) return st;
  // the sequence's position: one synchronous read
  RXLA_CUDA_CHECK(cudaMemcpyAsync(d->host_pinned, d->ctx + seq, 4, cudaMemcpyDeviceToHost, s));
  RXLA_CUDA_CHECK(cudaStreamSynchronize(s));
  const int32_t pos0 = d->host_pinned[0];
  RXLA_REQUIRE(pos0 >= 0 && (int64_t)pos0 + count <= c.max_context,
               "decoder_prefill: the prompt does not fit the sequence's remaining context");
  int32_t n = 0;
  for (int32_t c0 = 0; c0 < count; c0 += n) {
    n = std::min(count - c0, d->pf_chunk);
    cudaError_t e = launch_pdl(dec::prefill_rows_kernel, dim3(n), dim3(128), 0, s,
                               (const int32_t*)d->page_table, (int32_t)d->max_pages, seq,
                               pos0 + c0, d->pf_pt, d->pf_ctx);
    if (e == cudaSuccess)
      e = launch_pdl(dec::embed_kernel, dim3(n), dim3(256), 0, s, tokens + c0,
                     (const uint8_t*)d->emb_w8, (const float*)d->emb_scale,
                     (const __nv_bfloat16*)d->emb_bf16, (int64_t)c.vocab, H,
                     (int64_t)d->groups_h, (int64_t)d->group_h, d->pf_h);
    if (e != cudaSuccess) return cuda_fail(e, "prefill rows launch");
    const dec::Rows r{n,         d->pf_h,         d->pf_xn, d->pf_qkv, d->pf_att,
                      d->pf_act, d->pf_part,      d->pf_gws, d->pf_gws_bytes, d->pf_pt,
                      d->pf_ctx, d->pf_ws,        d->pf_ws_bytes, true};
    st = dec::enqueue_rows_layers(d, r, s);
    if (st) return st;
  }
  // greedy head on the prompt's last row; the token goes to the sequence's
  // slot of the step output
  const float* hl = d->pf_h + (int64_t)(n - 1) * H;
  int32_t* out = d->tok_out + seq;
  const int64_t v0 = (int64_t)c.tp_rank * d->vocab_local;
  if (d->emb_w8) {
    NormLinearArgs na{};
    na.h = hl;
    na.norm_w = d->final_norm;
    na.eps = c.rms_eps;
    na.w = d->emb_w8 + v0 * H;
    na.scale = d->emb_scale + v0 * d->groups_h;
    na.group = d->group_h;
    na.m = 1;
    na.n = d->vocab_local;
    na.k = H;
    na.y = d->logits;
    na.y_dtype = RXLA_B200_F32;
    na.epilogue = c.tp_size > 1 ? RXLA_B200_EPI_STORE : kArgmaxEpilogue;
    na.arg_val = d->arg_val;
    na.arg_idx = d->arg_idx;
    na.arg_count = d->arg_count;
    na.arg_out = out;
    na.arg_advance = nullptr;
    st = w8_norm_linear(na, s);
  } else {
    st = rxla_b200_rms_norm_bf16(hl, d->final_norm, 1, H, c.rms_eps, d->xn, s);
    if (!st)
      st = rxla_b200_bf16_linear(d->xn, RXLA_B200_BF16, d->emb_bf16 + v0 * H, 1, d->vocab_local,
                                 H, d->logits, RXLA_B200_F32, RXLA_B200_EPI_STORE, s);
    if (!st && c.tp_size == 1) {
      cudaError_t e = launch_pdl(argmax_kernel, dim3(1), dim3(1024), 0, s,
                                 (const float*)d->logits, (int64_t)d->vocab, out, (int32_t*)nullptr);
      if (e != cudaSuccess) st = cuda_fail(e, "argmax launch");
    }
  }
  if (!st && c.tp_size > 1) st = dec::tp_head_tail(d, 1, s, out, nullptr);
  if (st) return st;
  cudaError_t e = launch_pdl(dec::set_position_kernel, dim3(1), dim3(1), 0, s, d->ctx, seq,
                             pos0 + count);
  if (e != cudaSuccess) return cuda_fail(e, "prefill position launch");
  if (next_token && next_token != out)
    RXLA_CUDA_CHECK(cudaMemcpyAsync(next_token, out, 4, cudaMemcpyDeviceToDevice, s));
  if (logits)
    RXLA_CUDA_CHECK(cudaMemcpyAsync(logits, d->logits, (size_t)d->vocab_local * 4,
                                    cudaMemcpyDeviceToDevice, s));
  return RXLA_B200_OK;
}

extern "C" int32_t rxla_b200_decoder_step_host(rxla_b200_decoder* d, const int32_t* tokens_host,
                                               int32_t batch, int32_t* next_tokens_host,
                                               void* stream) {
  RXLA_REQUIRE(d && tokens_host && next_tokens_host, "decoder_step_host: null argument");
  RXLA_REQUIRE(batch > 0 && batch <= d->cfg.max_batch, "decoder_step_host: batch out of range");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  std::memcpy(d->host_pinned, tokens_host, (size_t)batch * 4);
  RXLA_CUDA_CHECK(cudaMemcpyAsync(d->tok_in, d->host_pinned, (size_t)batch * 4,
                                  cudaMemcpyHostToDevice, s));
  int32_t st = rxla_b200_decoder_step(d, d->tok_in, batch, d->tok_out, nullptr, stream);
  if (st) return st;
  RXLA_CUDA_CHECK(cudaMemcpyAsync(d->host_pinned + d->cfg.max_batch, d->tok_out, (size_t)batch * 4,
                                  cudaMemcpyDeviceToHost, s));
  RXLA_CUDA_CHECK(cudaStreamSynchronize(s));
  std::memcpy(next_tokens_host, d->host_pinned + d->cfg.max_batch, (size_t)batch * 4);
  return RXLA_B200_OK;
}

// Device buffers of the step's inputs and outputs (write tokens_in directly to
// skip the copy in rxla_b200_decoder_step).
extern "C" int32_t rxla_b200_decoder_io(rxla_b200_decoder* d, int32_t** tokens_in,
                                        int32_t** tokens_out, float** logits) {
  RXLA_REQUIRE(d, "decoder_io: null decoder");
  if (tokens_in) *tokens_in = d->tok_in;
  if (tokens_out) *tokens_out = d->tok_out;
  if (logits) *logits = d->logits;
  return RXLA_B200_OK;
}
