/*
 * rxla_oracle.h — CPU restatement of rxla's W8 decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline / reference legs may load this library, and only
 * as the checker or the timed CPU baseline — never as a product path.
 *
 * Each function restates one reference function (file:line inside the rxla
 * project, which is Rust + XLA and cannot run in this image: no cargo, no
 * PJRT plugin).  Arithmetic is f64 unless a reference rounding point is
 * named; bf16 rounding is round-to-nearest-even, as XLA's convert does.
 *
 * Pinning: the reference has no golden files for this path; its known-answer
 * tests (F64 formulas over literal inputs) are restated as fixtures under
 * tests/golden/ and every function here is checked against them.
 */
#ifndef RXLA_ORACLE_H_
#define RXLA_ORACLE_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- numerics helpers */
float oracle_bf16_round(float x);      /* f32 -> nearest-even bf16 -> f32 */
uint16_t oracle_f32_to_bf16(float x);  /* f32 -> bf16 bits (RNE, NaN kept) */
float oracle_bf16_to_f32(uint16_t b);

/* ---- deterministic data (splitmix64, counter based; element i of stream
 * `seed` depends on (seed, i) only, so any slice is reproducible) */
uint64_t oracle_splitmix64(uint64_t x);
void oracle_fill_normal(float* out, int64_t n, uint64_t seed, float mean, float std);
void oracle_fill_uniform(float* out, int64_t n, uint64_t seed, float lo, float hi);
void oracle_fill_randint(int32_t* out, int64_t n, uint64_t seed, int32_t lo, int32_t hi);

/* ---- W8 storage (benchmarks/quantize_qwen3_5_w8.py:33-44):
 * scale = max|w| over the group, clamped to 1e-12, / 127; q = clamp(round_half_even(w/scale),
 * -127, 127) + 128 stored as u8. */
void oracle_quantize_w8(const float* w, int64_t n, int64_t k, int64_t group, uint8_t* q,
                        float* scale);

/* ---- QuantizedLinear (crates/rxla-nn/src/layers.rs:257-298)
 * mode 0: compute dtype F32: y = x · ((q-128)·s)ᵀ, f64 accumulate, f32 out.
 * mode 1: compute dtype BF16 (:289-297): x -> bf16, W_deq (f32) -> bf16, dot,
 *         output rounded to bf16 (the dot's dtype), widened to f32.
 * mode 2: the kernel's algebra without roundings of W: Σ_g s_g Σ bf16(x)·(q-128),
 *         f64 throughout, f32 out (used to bound the kernel's accumulation error).
 * mode 3: mode 2 with the output rounded to bf16.
 * mode 4: mode 1 with an fp32 running sum in index order (a second valid
 *         implementation of the reference's arithmetic: the noise floor).
 * mode 5: mode 4 without the output rounding (f32 out): bf16 operands, fp32
 *         sum — the precision of a bf16-activation tied head. */
void oracle_w8_linear(const float* x, int64_t m, int64_t k, const uint8_t* w,
                      const float* scale, int64_t n, int64_t group, int32_t mode, float* y);

/* Dense linear y = x·wᵀ with w f32 [n,k] (crates/rxla-core/src/nn.rs:286-310);
 * bf16 = 1 rounds x and the output to bf16 (w assumed bf16-representable). */
void oracle_linear(const float* x, int64_t m, int64_t k, const float* w, int64_t n,
                   int32_t bf16, float* y);

/* ---- RMSNorm (crates/rxla-core/src/ops.rs:929-945): x * rsqrt(mean(x²)+eps) * w,
 * in f32 operation order (square, mean, +eps, rsqrt, ·, ·). */
void oracle_rms_norm(const float* x, int64_t rows, int64_t width, const float* w, float eps,
                     float* y);

/* ---- RoPE.  Frequencies θ^(-2i/rot) in f32 (crates/rxla-models/src/qwen3_5/mod.rs:211-228),
 * angle = f32(pos) * freq in f32; SplitHalf rotation of dims [0,rot)
 * (crates/rxla-core/src/rotary.rs:29-74): (a·cos - b·sin, b·cos + a·sin). */
void oracle_rope_inv_freq(float theta, int32_t rotary_dim, float* inv_freq);
void oracle_rope_split_half(float* x, int64_t rows, int64_t width, int32_t rotary_dim,
                            const int32_t* positions /* [rows] */, const float* inv_freq);
/* Rotation with explicit cos/sin tables [rows, rot/2] (rotary.rs:29-74), layout
 * 0 = SplitHalf, 1 = Interleaved. */
void oracle_rope_cos_sin(const float* x, int64_t rows, int64_t width, const float* cos_t,
                         const float* sin_t, int32_t layout, float* y);

/* ---- Attention (crates/rxla-core/src/attention.rs:83-252, decomposition of
 * crates/rxla-ir/src/pliron/stablehlo/conversion.rs:400-500): per batch b, query head h
 * (kv head h / (Hq/Hkv)), softmax(q·kᵀ·scale + mask)·v in f64.
 * q [B,Hq,T,D], k [B,Hkv,S,D], v [B,Hkv,S,Dv]; mask additive, indexed
 * mask[((b*mask_b_stride) + h*mask_h_stride + t*S + s)] (strides may be 0 to broadcast),
 * NULL = no mask. */
void oracle_gqa_attention(const float* q, const float* k, const float* v, const float* mask,
                          int64_t mask_b_stride, int64_t mask_h_stride, int64_t B, int64_t hq,
                          int64_t hkv, int64_t T, int64_t S, int64_t D, int64_t Dv, float scale,
                          float* out);

/* Additive causal mask [Q,K] from I32 positions (attention.rs:14-32): 0 if kpos<=qpos
 * else -inf; signed comparison, no subtraction. */
void oracle_causal_mask(const int32_t* qpos, int64_t nq, const int32_t* kpos, int64_t nk,
                        float* mask);

/* ---- KvCache::update_at / update_at_checked (crates/rxla-core/src/kv_cache.rs:53-112)
 * on a dense cache of `rank` dims; starts are clamped (checked=0) or validated
 * (checked=1: invalid -> caches unchanged, returns 0).  Returns accepted (1/0). */
int32_t oracle_kv_update(float* k_cache, float* v_cache, const int64_t* cache_shape,
                         const float* k_upd, const float* v_upd, const int64_t* upd_shape,
                         int32_t rank, const int32_t* starts, int32_t checked);

/* ---- Paged decode attention: the contract of rxla_b200_paged_decode_attention
 * restated on the dense semantics above.  k/v pages bf16 [P, Hkv, 16, D];
 * writes the new (normed, rotated, bf16-rounded) k/v into the pages and the
 * attention output (bf16-rounded, as f32) into out [B, Hq*D].  accepted/ctx as in
 * the header.  f64 softmax. */
void oracle_paged_decode_attention(
    int32_t batch, int32_t hq, int32_t hkv, int32_t d, const float* q, const float* k_new,
    const float* v_new, int64_t q_row_stride, int64_t kv_row_stride, const float* q_norm_w,
    const float* k_norm_w, float eps, const float* inv_freq, int32_t rotary_dim, float scale,
    uint16_t* k_pages, uint16_t* v_pages, int32_t page_size, int32_t max_pages_per_seq,
    const int32_t* page_table, const int32_t* pages_per_seq, int32_t* ctx_lens,
    int32_t kv_update, int32_t advance_ctx, int32_t* accepted, float* out);

/* ---- Qwen3-style W8 decoder (composition of crates/rxla-models/src/qwen3_5/
 * {mod.rs:199-273, layers.rs:28-101,270-293} with Qwen3 differences: plain q_proj,
 * per-head q/k RMSNorm, full RoPE, tied head).  One decode step for a batch,
 * with a dense bf16 KV cache [layers][batch][Hkv][max_ctx][D]. */
typedef struct oracle_decoder_config {
  int32_t layers, hidden, q_heads, kv_heads, head_dim, intermediate, vocab;
  float rms_eps, rope_theta;
  int32_t embedding_bf16; /* 1: bf16 embedding + bf16 tied head; 0: W8 */
  int32_t group_size;     /* 0 = per channel */
  int32_t max_batch, max_context;
  /* QuantizedLinear arithmetic: 1 = the reference's (bf16(W_deq), output bf16),
   * 3 = exact q with the scale applied to the fp32 dot, output bf16,
   * 4 = the reference's with an fp32 running sum */
  int32_t linear_mode;
} oracle_decoder_config;

typedef struct oracle_decoder oracle_decoder;

oracle_decoder* oracle_decoder_create(const oracle_decoder_config* cfg);
void oracle_decoder_destroy(oracle_decoder* dec);
/* Named parameter storage (same names as the CUDA runner); returns byte size, or -1. */
int64_t oracle_decoder_parameter(oracle_decoder* dec, const char* name, void** ptr,
                                 int32_t* dtype);
/* Seeded synthetic weights: N(0, 0.02) quantized per channel (or bf16), norms 1+N(0,0.02)
 * rounded to bf16.  Each parameter uses stream seed + index of the parameter. */
void oracle_decoder_init_synthetic(oracle_decoder* dec, uint64_t seed);
void oracle_decoder_reset(oracle_decoder* dec);
/* One step: tokens [batch] -> logits [batch, vocab] (f32), next tokens [batch]. */
/* full-sequence forward of one prompt with the causal mask (state untouched) */
void oracle_decoder_forward(oracle_decoder* dec, const int32_t* tokens, int32_t T, float* logits,
                            int32_t* next_token);
void oracle_decoder_step(oracle_decoder* dec, const int32_t* tokens, int32_t batch,
                         float* logits, int32_t* next_tokens);
int32_t oracle_decoder_context(oracle_decoder* dec, int32_t b);
/* Dense bf16 cache of one layer: [max_batch][kv_heads][max_context][head_dim]. */
void oracle_decoder_kv(oracle_decoder* dec, int32_t layer, uint16_t** k, uint16_t** v);

/* Number of OpenMP threads the oracle uses (for the CPU baseline report). */
int32_t oracle_decoder_prefill(oracle_decoder* dec, int32_t seq, const int32_t* tokens, int32_t T,
                               float* logits, int32_t* next_token);
int32_t oracle_decoder_set_context(oracle_decoder* dec, int32_t seq, int32_t ctx);
void oracle_set_num_threads(int32_t n);
int32_t oracle_num_threads(void);

#ifdef __cplusplus
}
#endif

#endif
