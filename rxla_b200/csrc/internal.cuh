// internal.cuh — library-internal entry points shared by the decoder runner.
#pragma once

#include "common.cuh"

namespace rxla {

// W8 linear whose x is bf16(rms_norm(h) * norm_w) of the f32 residual h, the
// norm computed in each CTA's prologue; optionally with the greedy-argmax
// epilogue of the tied LM head (epilogue = kArgmaxEpilogue).
struct NormLinearArgs {
  const float* h;
  const float* norm_w;
  float eps;
  const uint8_t* w;
  const float* scale;
  int64_t group, m, n, k;
  void* y;  // y (STORE / SWIGLU) or logits (argmax; may be null)
  int32_t y_dtype, epilogue;
  // argmax scratch and results: per-CTA partials [>= grid][8], a counter that
  // is zero between launches, the chosen token per row, optional position += 1
  float* arg_val;
  int32_t* arg_idx;
  uint32_t* arg_count;
  int32_t* arg_out;
  int32_t* arg_advance;
  L2Prefetch next;  // what the following kernel reads first (nseg = 0: none)
};

constexpr int kArgmaxEpilogue = 16;

// W8A16 GEMM on tcgen05 tensor cores (tokens > 8): y = x · W_deqᵀ with the
// skinny kernel's epilogues.  x bf16 [m, ldx]; weight [n_rows, k] (n_rows =
// 2n for SwiGLU); split-K over `splits` CTAs per tile needs `ws`.
struct GemmArgs {
  const void* x;
  int64_t ldx;
  const uint8_t* w;
  const float* scale;
  int64_t group, m, n, k;
  void* y;
  int64_t ldy;
  int32_t y_dtype, epilogue;
  int32_t splits;
  void* ws;
  size_t ws_bytes;
};

int32_t w8_norm_linear(const NormLinearArgs& a, cudaStream_t stream);

// A comm's one-shot peer all-reduce buffers as a kernel sees them: every
// rank's buffer mapped here (two slots of [8][cap] f32 partials, then
// [8][max_ctas] u64 arrival flags) and this rank's per-CTA epoch counters.
constexpr int kP2pMaxRanks = 8;
struct P2pView {
  uint8_t* peer[kP2pMaxRanks];
  uint64_t* epoch;  // [max_ctas]
  int64_t cap;      // floats per (slot, rank)
  int32_t rank, world, max_ctas;
};
// false when the comm has no peer buffers
bool comm_p2p_view(const rxla_b200_comm* c, P2pView* out);

// rxla_b200_w8a16_linear with an L2 prefetch of the next kernel's first bytes.
// With `tp` (a row-parallel linear of a tensor-parallel decoder: epilogue
// RESIDUAL_ADD, f32 y = the residual, one pass of at most 8 tokens) the
// kernel's epilogue all-reduces the partial dot across the ranks through the
// peer buffers and adds bf16(Σ over ranks, in rank order) into y.
int32_t w8_linear(const void* x, int32_t x_dtype, const uint8_t* weight, const float* scale,
                  int64_t group_size, int64_t m, int64_t n, int64_t k, void* y, int32_t y_dtype,
                  int32_t epilogue, cudaStream_t stream, const L2Prefetch* next,
                  const P2pView* tp = nullptr, void* ws = nullptr, size_t ws_bytes = 0);
int32_t w8_gemm(const GemmArgs& a, cudaStream_t stream);
// split-K workspace: a fixed counter region (the same for every shape, so
// GEMMs sharing a workspace never overlap one another's counters), then the
// [splits][m][n_rows] f32 partials
constexpr size_t kGemmCounterBytes = 1u << 20;
size_t w8_gemm_workspace_bytes(int64_t m, int64_t n_rows, int splits);
// Decode batches (m <= kGemmDecMaxTokens) run the weights-on-M variant.
constexpr int64_t kGemmDecMaxTokens = 128;
int32_t w8_gemm_dec(const GemmArgs& a, cudaStream_t stream);
bool w8_gemm_dec_applies(int64_t m, int64_t k, int64_t group);
// CTAs per split of the GEMM w8_gemm runs for this shape (m tokens, n outputs)
int64_t w8_gemm_tiles(int64_t m, int64_t n, int64_t k, int64_t group, bool swiglu);
// split-K depth w8_gemm should be given for this shape (decoder workspace plan)
int w8_gemm_splits(int64_t m, int64_t n, int64_t k, int64_t group, bool swiglu);
int32_t comm_allreduce_f32(rxla_b200_comm* comm, float* buf, int64_t count, cudaStream_t s);
// every rank's `bytes` from `in`, concatenated in rank order into `out`
int32_t comm_allgather_bytes(rxla_b200_comm* comm, const void* in, void* out, int64_t bytes,
                             cudaStream_t s);
int32_t comm_world(const rxla_b200_comm* comm);
bool comm_has_p2p(const rxla_b200_comm* comm);
// f32 elements the comm's peer buffers hold per rank (0: not enabled)
int64_t comm_p2p_capacity(const rxla_b200_comm* comm);
// out = Σ partial over ranks (residual false) or out += bf16(Σ partial)
int32_t comm_p2p_allreduce(rxla_b200_comm* comm, const float* partial, float* out, int64_t count,
                           bool residual, cudaStream_t s);

namespace attn {
// append_only: write the new K/V rows and nothing else (no page loop, no
// output, no context advance)
int32_t launch(const rxla_b200_paged_decode_args* a, cudaStream_t s, bool ctx_stable,
               const L2Prefetch* next = nullptr, bool append_only = false);
// causal attention of a prompt chunk's rows after an append-only launch
int32_t prefill_launch(const rxla_b200_paged_decode_args* a, cudaStream_t s);
}

}  // namespace rxla
