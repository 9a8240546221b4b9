// gated_delta.cu — Qwen3.5 gated-delta linear attention (the "linear_attn"
// mixer of crates/rxla-models/src/qwen3_5/layers.rs:114-268), between its
// input projections and its out_proj.
//
// Single-token calls of at most kFusedMaxCtas (sequence, head) pairs run
// as one kernel, gdn_decode_fused_kernel (below); every other call as three
// kernels, stream-ordered (programmatic dependent launch):
//  1. gdn_prep_kernel — CTA = (channel block of D channels, 16 tokens,
//     sequence), thread = channel: the causal depthwise conv of the mixed
//     q/k/v projection over the last `conv_kernel` rows (rows before the
//     call come from the sequence's conv state; each input row is loaded once
//     per CTA and slid over the 16 tokens), SiLU, the L2 norm of every q and
//     k head (q then scaled by 1/sqrt(D)); one extra channel block computes
//     the gates beta = sigmoid(b) and exp(-exp(A_log) * softplus(a + dt_bias)).
//  2. gdn_recurrence_kernel — the delta rule over the call's tokens, in
//     order, with the state on chip.  Column j of a head's state S [Dk, Dv]
//     evolves on its own:  S[:,j] = g S[:,j] + k δ_j,
//     δ_j = beta (v_j − k·(g S[:,j])),  o_j = q·S[:,j].  Sixteen lanes hold
//     one column (eight for D = 32), a warp two columns, a CTA a block of
//     columns of one (sequence, head), so a 2048-token prompt of 16 heads
//     still spreads over ~1000 warps.  One pass over a lane's rows per token
//     updates S and forms both o_t = q_t·S_t and the next token's
//     k_{t+1}·S_t, so one shuffle reduction of two values per token is the
//     only cross-lane step on the recurrence's critical path.  Token rows of q, k,
//     v and the gates stream through a double-buffered shared-memory stage
//     (cp.async).  f32 throughout, as the reference's F32 graph.
//  3. gdn_gated_norm_kernel — CTA = token row, warp = head: RMSNorm of each
//     head's output over Dv, times norm.weight and silu(z), rounded to bf16
//     for out_proj; the last row of each sequence also writes the new conv
//     state.
//
// State layout (session state; the reference recomputes the whole sequence
// each call and keeps none): the recurrent state f32 [batch, heads, Dv, Dk],
// i.e. column j of S contiguous, and the conv state bf16
// [batch, conv_kernel - 1, 3·heads·D] holding the last conv_kernel - 1 mixed
// rows, oldest first.
#include "common.cuh"

namespace rxla {
namespace gdn {

constexpr int kMaxConvKernel = 8;
constexpr int kPrepTokens = 16;  // tokens per prep CTA
constexpr int kRecWarps = 4;     // warps per recurrence CTA
constexpr int kLongCall = 32;    // calls with more tokens per sequence use the prompt shape

__device__ __forceinline__ float sigmoid_f(float x) {
  // logistic with a nonpositive exponent argument (crates/rxla-core/src/ops.rs:332-337)
  const float e = __expf(-fabsf(x));
  const float r = __fdividef(1.0f, 1.0f + e);
  return x >= 0.0f ? r : e * r;
}

__device__ __forceinline__ float softplus_f(float x) {
  // max(x, 0) + log1p(exp(-|x|)), the stable form the reference emits
  // (crates/rxla-core/src/ops.rs:256-262)
  return fmaxf(x, 0.0f) + log1pf(__expf(-fabsf(x)));
}

__device__ __forceinline__ float ld_bf16(const uint16_t* p) {
  return __uint_as_float(((uint32_t)*p) << 16);
}

struct PrepArgs {
  const uint16_t* mixed;
  const uint16_t* b;
  const uint16_t* a;
  int64_t mixed_ld, b_ld, a_ld;
  const float* conv_w;  // [3W, K]
  const float* a_log;
  const float* dt_bias;
  const uint16_t* conv_state;  // [B, K-1, 3W] or null (zero history)
  uint16_t* conv_state_out;    // the same array: written here for calls of <= 16 tokens
  float* qkv;                  // [B*T, 3W]
  float2* gb;                  // [B*T, H]: (exp(decay), beta)
  int32_t T, H, K;
  float q_scale;
};

// Per-token sums of squares of a warp's 32 channels for TB tokens: a
// reduce-scatter butterfly (TB = 16: 16 shuffles instead of 16 × 5); lane l
// ends with the full sum of token `tok`; lanes with tok_owner true write it.
template <int TB>
__device__ __forceinline__ void token_sums(const float (&y)[TB], int lane, float& sum, int& tok,
                                           bool& tok_owner) {
  if constexpr (TB == 16) {
    float v[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = y[i] * y[i];
    tok = 0;
#pragma unroll
    for (int half = 8; half >= 1; half >>= 1) {
      const int off = 2 * half;  // lane distance 16, 8, 4, 2
      const bool up = (lane & off) != 0;
#pragma unroll
      for (int i = 0; i < half; ++i) {
        const float send = up ? v[i] : v[i + half];
        const float keep = up ? v[i + half] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
      }
      tok += up ? half : 0;
    }
    sum = v[0] + __shfl_xor_sync(0xffffffffu, v[0], 1);
    tok_owner = (lane & 1) == 0;
  } else {
    static_assert(TB == 1, "token blocks of 1 or 16");
    float ss = y[0] * y[0];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    sum = ss;
    tok = 0;
    tok_owner = lane == 0;
  }
}

// grid (3H + 1 channel blocks, ceil(T / TB), B); block D threads.  TB = 16
// tokens per CTA, or 1 for single-token (decode) calls, whose unrolled loops
// are then 16 times shorter.  KC = 4: the conv width as a constant (Qwen3.5's
// conv_kernel, weights read as one float4); KC = 0: the runtime width (<= 8).
template <int D, int TB, int KC>
__global__ void __launch_bounds__(D) gdn_prep_kernel(PrepArgs p) {
  constexpr int KM = KC > 0 ? KC : kMaxConvKernel;  // taps unrolled
  constexpr int WIN = TB + KM - 1;
  pdl_wait();
  pdl_launch_dependents();
  const int K = KC > 0 ? KC : p.K;
  const int u = blockIdx.x, t0 = blockIdx.y * TB, b = blockIdx.z;
  const int n = min(TB, p.T - t0);
  const int W = p.H * D, C3 = 3 * W;
  const int c = threadIdx.x;
  const int64_t row0 = (int64_t)b * p.T + t0;
  if (u == 3 * p.H) {
    // gates (layers.rs:179-197, :205-212): beta = sigmoid(b);
    // decay = softplus(a + dt_bias) * -exp(A_log), applied as exp(decay)
    for (int i = c; i < n * p.H; i += D) {
      const int tt = i / p.H, h = i % p.H;
      const int64_t row = row0 + tt;
      const float bl = ld_bf16(p.b + row * p.b_ld + h);
      const float al = ld_bf16(p.a + row * p.a_ld + h);
      const float decay = softplus_f(al + p.dt_bias[h]) * -__expf(p.a_log[h]);
      p.gb[row * p.H + h] = make_float2(__expf(decay), sigmoid_f(bl));
    }
    return;
  }
  const int gc = u * D + c;  // global channel
  // input rows t0 - (K-1) .. t0 + n - 1 of this channel (history from the
  // conv state), each loaded once
  float x[WIN];
  if (t0 >= K - 1) {  // every row inside this call: one strided walk
    const uint16_t* mp = p.mixed + (row0 - (K - 1)) * p.mixed_ld + gc;
#pragma unroll
    for (int w = 0; w < WIN; ++w) x[w] = w < n + K - 1 ? ld_bf16(mp + (int64_t)w * p.mixed_ld) : 0.0f;
  } else {
#pragma unroll
    for (int w = 0; w < WIN; ++w) {
      x[w] = 0.0f;
      const int tau = t0 - (K - 1) + w;
      if (w < n + K - 1) {
        if (tau >= 0)
          x[w] = ld_bf16(p.mixed + ((int64_t)b * p.T + tau) * p.mixed_ld + gc);
        else if (p.conv_state)
          x[w] = ld_bf16(p.conv_state + ((int64_t)b * (K - 1) + (K - 1 + tau)) * C3 + gc);
      }
    }
  }
  // A call of at most 16 tokens per sequence has one token block: this
  // thread is then the only reader of its channel's history in the call, and
  // it holds the channel's new history (inputs n .. n + K - 2) in registers,
  // so it writes it (longer calls: the last row's gdn_gated_norm_kernel CTA)
  if (gridDim.y == 1 && p.conv_state_out) {
    uint16_t* cs = p.conv_state_out + (int64_t)b * (K - 1) * C3 + gc;
#pragma unroll
    for (int w = 0; w < WIN; ++w)  // slot w - n holds x[w] (static register indices)
      if (w >= n && w < n + K - 1)
        cs[(int64_t)(w - n) * C3] = __bfloat16_as_ushort(__float2bfloat16_rn(x[w]));
  }
  float wk[KM];
  if constexpr (KC == 4) {
    const float4 w4 = *reinterpret_cast<const float4*>(p.conv_w + (int64_t)gc * 4);
    wk[0] = w4.x;
    wk[1] = w4.y;
    wk[2] = w4.z;
    wk[3] = w4.w;
  } else {
#pragma unroll
    for (int j = 0; j < KM; ++j) wk[j] = j < K ? p.conv_w[(int64_t)gc * K + j] : 0.0f;
  }
  // causal depthwise conv: out_t = Σ_j w[c, j] x[t - (K-1) + j] (padding
  // [[K-1, 0]], no kernel reversal), then SiLU (layers.rs:131-145)
  float y[TB];
#pragma unroll
  for (int tt = 0; tt < TB; ++tt) {
    y[tt] = 0.0f;
    if (tt < n) {  // n is uniform across the CTA
      float acc = 0.0f;
#pragma unroll
      for (int j = 0; j < KM; ++j)
        if (KC > 0 || j < K) acc = fmaf(wk[j], x[tt + j], acc);
      y[tt] = acc * sigmoid_f(acc);
    }
  }
  float* out = p.qkv + row0 * C3 + gc;
  if (u >= 2 * p.H) {  // v channels: conv + SiLU only
#pragma unroll
    for (int tt = 0; tt < TB; ++tt)
      if (tt < n) out[(int64_t)tt * C3] = y[tt];
    return;
  }
  // q / k heads: L2 norm over the head's D channels (l2_norm of
  // layers.rs:103-112: x * rsqrt(Σx² + 1e-6)); q also times the f32 constant
  // 1/sqrt(D) (layers.rs:146-152)
  __shared__ float red[TB][D / 32];
  const int lane = c & 31, warp = c >> 5;
  {
    float sum;
    int tok;
    bool owner;
    token_sums<TB>(y, lane, sum, tok, owner);
    if (owner) red[tok][warp] = sum;
  }
  __syncthreads();
  const float scale = u < p.H ? p.q_scale : 1.0f;
#pragma unroll
  for (int tt = 0; tt < TB; ++tt) {
    if (tt < n) {
      float ss = 0.0f;
#pragma unroll
      for (int w = 0; w < D / 32; ++w) ss += red[tt][w];
      float v = y[tt] * rsqrtf(ss + 1e-6f);
      if (u < p.H) v *= scale;
      out[(int64_t)tt * C3] = v;
    }
  }
}

struct RecArgs {
  const float* qkv;  // [B*T, 3W]
  const float2* gb;  // [B*T, H]
  float* state;      // [B, H, D(v), D(k)]
  int32_t has_state;
  float* o;  // [B*T, W]
  int32_t T, H;
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Shared-memory stage of CH tokens: q [CH][D], k [CH + 1][D] (the first row
// of the next chunk too: a token needs the next token's k), v [CH][CPB],
// gates [CH], o [CH][CPB].
template <int D, int CPB, int CH>
struct Stage {
  float q[CH][D];
  float k[CH + 1][D];
  float v[CH][CPB];
  float2 g[CH];
  float o[CH][CPB];
};

// Sum over the LPC lanes of a column (the low lane bits), two values at once.
template <int LPC>
__device__ __forceinline__ void reduce_col2(float& a, float& b) {
#pragma unroll
  for (int o = 1; o < LPC; o <<= 1) {
    const float ta = __shfl_xor_sync(0xffffffffu, a, o);
    const float tb = __shfl_xor_sync(0xffffffffu, b, o);
    a += ta;
    b += tb;
  }
}

// Thread layout of the recurrence for head_dim D: LPC lanes hold a column,
// R rows each, as float4 groups at rows 4·LPC·i + 4·part + e (conflict-free
// shared-memory reads, 16-byte state accesses); CH tokens per shared-memory
// stage; ACC independent partial sums per dot product.
//  - PROMPT (long calls): 8 lanes per column, 64-token stages, 4 partial sums
//    — fewer shuffle levels and fewer barriers on the sequential chain;
//  - DECODE (a few tokens per sequence, many sequences): 8 lanes per column
//    and 8-token stages — small CTAs (~20 KB of shared memory), many
//    resident, 64 bytes of state per thread in flight.
// (2048-token prompt, 16 heads of 128: 335 µs against 413 µs with 16 lanes
// and 16-token stages; batch-64 decode: 35 µs against 86 µs with the prompt
// shape.)
template <int D, bool PROMPT>
struct RecShape {
  static constexpr int LPC = 8;               // lanes per column
  static constexpr int CH = PROMPT ? 64 : 8;  // tokens per stage
  static constexpr int ACC = PROMPT ? 4 : 2;
  static constexpr int R = D / LPC;            // rows per lane
  static constexpr int NI = R / 4;             // float4 groups per lane
  static constexpr int CPW = 32 / LPC;         // columns per warp
  static constexpr int CPB = kRecWarps * CPW;  // columns per CTA
  static_assert(R % 4 == 0 && R % ACC == 0, "rows per lane: whole float4 groups and sums");
};

// grid (D / CPB column blocks, H, B); block kRecWarps warps.
template <int D, bool PROMPT>
__global__ void __launch_bounds__(kRecWarps * 32) gdn_recurrence_kernel(RecArgs p) {
  using Sh = RecShape<D, PROMPT>;
  constexpr int LPC = Sh::LPC, R = Sh::R, NI = Sh::NI, CPB = Sh::CPB, CH = Sh::CH;
  constexpr int ACC = Sh::ACC;
  constexpr int NT = kRecWarps * 32;
  using StageT = Stage<D, CPB, CH>;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  StageT* st = reinterpret_cast<StageT*>(smem_raw);
  const int cb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int W = p.H * D, C3 = 3 * W;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int part = lane & (LPC - 1);
  const int col_local = warp * Sh::CPW + lane / LPC;
  const int j = cb * CPB + col_local;
  float s[R];
  float* sp = p.state + (((int64_t)b * p.H + h) * D + j) * D;
  // The state is read before griddepcontrol.wait: its last writer is the
  // previous call's recurrence kernel, two or more grids back on the stream,
  // which has completed when this grid starts (every kernel of this library
  // triggers its dependents only after its own wait), so the load overlaps
  // the prep kernel that directly precedes this one.
  if (p.has_state) {
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      const float4 v = *reinterpret_cast<const float4*>(sp + 4 * LPC * i + 4 * part);
      s[4 * i] = v.x;
      s[4 * i + 1] = v.y;
      s[4 * i + 2] = v.z;
      s[4 * i + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int r = 0; r < R; ++r) s[r] = 0.0f;
  }
  pdl_wait();
  const int64_t row0 = (int64_t)b * p.T;
  const int nchunks = (p.T + CH - 1) / CH;
  auto load = [&](int c, int buf) {
    StageT& S = st[buf];
    const int t0 = c * CH;
    const int n = min(CH, p.T - t0);
    const int nk = min(CH + 1, p.T - t0);  // k rows: this chunk's and the next one's first
    for (int i = tid; i < n * (D / 4); i += NT) {
      const int tt = i / (D / 4), piece = i % (D / 4);
      cp_async16(&S.q[tt][piece * 4], p.qkv + (row0 + t0 + tt) * C3 + h * D + piece * 4);
    }
    for (int i = tid; i < nk * (D / 4); i += NT) {
      const int tt = i / (D / 4), piece = i % (D / 4);
      cp_async16(&S.k[tt][piece * 4], p.qkv + (row0 + t0 + tt) * C3 + W + h * D + piece * 4);
    }
    for (int i = tid; i < n * (CPB / 4); i += NT) {
      const int tt = i / (CPB / 4), piece = i % (CPB / 4);
      cp_async16(&S.v[tt][piece * 4],
                 p.qkv + (row0 + t0 + tt) * C3 + 2 * W + h * D + cb * CPB + piece * 4);
    }
    for (int tt = tid; tt < n; tt += NT) S.g[tt] = p.gb[(row0 + t0 + tt) * p.H + h];
    cp_async_commit();
  };
  auto ld_rows = [&](const float* src, float (&dst)[R]) {
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      const float4 v = *reinterpret_cast<const float4*>(src + 4 * LPC * i + 4 * part);
      dst[4 * i] = v.x;
      dst[4 * i + 1] = v.y;
      dst[4 * i + 2] = v.z;
      dst[4 * i + 3] = v.w;
    }
  };
  float a = 0.0f;  // k_t · S_{t-1}[:, j] of the token about to be processed
  // One token: S_t = g S + k_t δ (the reference's state.mul(decay) then
  // add(k ⊗ δ)), δ = beta (v - g (k_t·S)), o_t = q_t · S_t, and the next
  // token's k_{t+1} · S_t — one pass over the rows.  Row tt + 1 of the k
  // stage exists for every tt; after the sequence's last token it holds
  // stale values whose dot is never used.
  auto step = [&](StageT& S, int tt, const float (&kc)[R], float (&kn)[R]) {
    const float2 g = S.g[tt];
    const float vj = S.v[tt][col_local];
    float qv[R];
    ld_rows(&S.q[tt][0], qv);
    ld_rows(&S.k[tt + 1][0], kn);
    const float delta = (vj - g.x * a) * g.y;
    float oa[ACC], na[ACC];
#pragma unroll
    for (int u = 0; u < ACC; ++u) oa[u] = na[u] = 0.0f;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      s[r] = fmaf(kc[r], delta, s[r] * g.x);
      oa[r % ACC] = fmaf(s[r], qv[r], oa[r % ACC]);
      na[r % ACC] = fmaf(s[r], kn[r], na[r % ACC]);
    }
#pragma unroll
    for (int u = 1; u < ACC; ++u) {
      oa[0] += oa[u];
      na[0] += na[u];
    }
    float o = oa[0];
    a = na[0];
    reduce_col2<LPC>(o, a);
    if (part == 0) S.o[tt][col_local] = o;
  };
  float kA[R], kB[R];  // this token's k and the next one's, alternating
  load(0, 0);
  for (int c = 0; c < nchunks; ++c) {
    const int buf = c & 1;
    if (c + 1 < nchunks) {
      load(c + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    StageT& S = st[buf];
    const int t0 = c * CH;
    const int n = min(CH, p.T - t0);
    if (c == 0) {
      ld_rows(&S.k[0][0], kA);
      if (p.has_state) {
        float a0 = 0.f, a1 = 0.f;
#pragma unroll
        for (int r = 0; r < R; r += 2) {
          a0 = fmaf(s[r], kA[r], a0);
          a1 = fmaf(s[r + 1], kA[r + 1], a1);
        }
        a = a0 + a1;
        float unused = 0.0f;
        reduce_col2<LPC>(a, unused);
      }
    }
    // two tokens per iteration, so the k registers alternate without copies
    int tt = 0;
    for (; tt + 1 < n; tt += 2) {
      step(S, tt, kA, kB);
      step(S, tt + 1, kB, kA);
    }
    if (tt < n) {
      step(S, tt, kA, kB);
#pragma unroll
      for (int r = 0; r < R; ++r) kA[r] = kB[r];
    }
    __syncthreads();
    // the chunk's outputs, CPB contiguous floats per token
    for (int i = tid; i < n * (CPB / 4); i += NT) {
      const int tt = i / (CPB / 4), piece = i % (CPB / 4);
      *reinterpret_cast<float4*>(p.o + (row0 + t0 + tt) * W + h * D + cb * CPB + piece * 4) =
          *reinterpret_cast<const float4*>(&S.o[tt][piece * 4]);
    }
    // buffer reuse: the load of chunk c + 2 into this buffer is issued at
    // the top of the next iteration, after the __syncthreads above, when no
    // thread reads this chunk's q, k, v or gates any more; S.o is written
    // again only after that iteration's own __syncthreads, when every thread
    // has finished the stores here
  }
  pdl_launch_dependents();
#pragma unroll
  for (int i = 0; i < NI; ++i)
    *reinterpret_cast<float4*>(sp + 4 * LPC * i + 4 * part) =
        make_float4(s[4 * i], s[4 * i + 1], s[4 * i + 2], s[4 * i + 3]);
}

struct NormArgs {
  const float* o;  // [B*T, W]
  const uint16_t* z;
  int64_t z_ld;
  const float* norm_w;  // [D]
  float eps;
  uint16_t* out;  // [B*T, W] bf16
  // conv-state update (done by the last row of each sequence)
  const uint16_t* mixed;
  int64_t mixed_ld;
  uint16_t* conv_state;  // [B, K-1, 3W]
  int32_t has_state;
  int32_t T, H, K;
  int32_t vec;  // z rows and norm_w allow 8- / 16-byte loads (D = 128)
};

constexpr int kNormWarps = 16;

// grid B*T (one token row per CTA); warp = head.
template <int D>
__global__ void __launch_bounds__(kNormWarps * 32) gdn_gated_norm_kernel(NormArgs p) {
  constexpr int E = D / 32;  // consecutive elements per lane
  pdl_wait();
  pdl_launch_dependents();
  const int row = blockIdx.x;
  const int W = p.H * D;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // output norm (layers.rs:243-259): o * rsqrt(mean(o²) + eps) * w * silu(z)
  for (int h = warp; h < p.H; h += kNormWarps) {
    const int64_t base = (int64_t)row * W + h * D + lane * E;
    const uint16_t* zr = p.z + (int64_t)row * p.z_ld + h * D + lane * E;
    float v[E], z[E], w[E];
    if constexpr (E == 4) {
      const float4 o4 = *reinterpret_cast<const float4*>(p.o + base);
      v[0] = o4.x;
      v[1] = o4.y;
      v[2] = o4.z;
      v[3] = o4.w;
    } else {
#pragma unroll
      for (int e = 0; e < E; ++e) v[e] = p.o[base + e];
    }
    if (E == 4 && p.vec) {
      const uint2 z4 = *reinterpret_cast<const uint2*>(zr);
      z[0] = bf16_lo(z4.x);
      z[1] = bf16_hi(z4.x);
      z[2] = bf16_lo(z4.y);
      z[3] = bf16_hi(z4.y);
      const float4 w4 = *reinterpret_cast<const float4*>(p.norm_w + lane * E);
      w[0] = w4.x;
      w[1] = w4.y;
      w[2] = w4.z;
      w[3] = w4.w;
    } else {
#pragma unroll
      for (int e = 0; e < E; ++e) {
        z[e] = ld_bf16(zr + e);
        w[e] = p.norm_w[lane * E + e];
      }
    }
    float ss = 0.0f;
#pragma unroll
    for (int e = 0; e < E; ++e) ss = fmaf(v[e], v[e], ss);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float ns = rsqrtf(ss / (float)D + p.eps);
    float y[E];
#pragma unroll
    for (int e = 0; e < E; ++e) y[e] = ((v[e] * ns) * w[e]) * (z[e] * sigmoid_f(z[e]));
    if (E == 4 && p.vec) {
      *reinterpret_cast<uint2*>(p.out + base) = make_uint2(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]));
    } else {
#pragma unroll
      for (int e = 0; e < E; ++e) p.out[base + e] = __bfloat16_as_ushort(__float2bfloat16_rn(y[e]));
    }
  }
  // new conv state of sequence b: its last K-1 mixed rows (older rows from
  // the previous state when the call has fewer than K-1 tokens).  Each
  // channel belongs to one thread, which reads all of its new slots into
  // registers before writing any, so an in-place move never overwrites an
  // old slot it has still to read.
  const int t = row % p.T, b = row / p.T;
  if (t != p.T - 1 || p.K <= 1 || p.T <= kPrepTokens) return;  // short calls: the prep kernel
  const int C3 = 3 * W, hist = p.K - 1;
  uint16_t* cs = p.conv_state + (int64_t)b * hist * C3;
  for (int c = threadIdx.x; c < C3; c += blockDim.x) {
    uint16_t v[kMaxConvKernel - 1];
#pragma unroll
    for (int s = 0; s < kMaxConvKernel - 1; ++s) {
      v[s] = 0;
      if (s < hist) {
        const int tau = p.T - hist + s;  // call-relative position of slot s
        if (tau >= 0)
          v[s] = p.mixed[((int64_t)b * p.T + tau) * p.mixed_ld + c];
        else if (p.has_state)
          v[s] = cs[(int64_t)(hist + tau) * C3 + c];
      }
    }
#pragma unroll
    for (int s = 0; s < kMaxConvKernel - 1; ++s)
      if (s < hist) cs[(int64_t)s * C3 + c] = v[s];
  }
}

// ------------------------------------------------ single-token fused step
//
// Decode calls (one token per sequence) of few sequences: the three kernels
// above would each be a handful of CTAs whose launch and dependency latency
// is most of the call.  Here one CTA of 4·D threads is one (head, sequence)
// and does the whole step on chip: the conv of the head's 3·D channels with
// the conv-state shift (thread = channel), the gates (one extra thread), the
// q / k L2 norms, the delta rule over the head's state (four lanes per
// column, D / 4 rows each) and the gated RMSNorm.  Every sum is formed in the
// order the three kernels use, except the column dots, whose lane split
// differs (4 lanes of D / 4 rows against 8 of D / 8).
struct FusedArgs {
  PrepArgs prep;        // mixed / b / a, conv weights, gates, conv state
  float* state;         // [B, H, D(v), D(k)]
  int32_t has_state;
  const uint16_t* z;
  int64_t z_ld;
  const float* norm_w;  // [D]
  float eps;
  uint16_t* out;        // [B, W] bf16
};

constexpr int kFusedMaxCtas = 2 * 148;  // (sequence, head) pairs up to which T = 1 calls fuse

template <int D, int KC>
__global__ void __launch_bounds__(4 * D) gdn_decode_fused_kernel(FusedArgs f) {
  constexpr int KM = KC > 0 ? KC : kMaxConvKernel;
  constexpr int NW = D / 32;  // warps per q / k / v part
  constexpr int LPC = 4;      // lanes per state column
  constexpr int R = D / LPC;  // rows per lane
  constexpr int NI = R / 4;   // float4 groups per lane: rows 4·LPC·i + 4·pl + e
  constexpr int E = D / 32;   // output elements per lane of the norm warp
  const PrepArgs& p = f.prep;
  const int h = blockIdx.x, b = blockIdx.y;
  const int H = p.H, W = H * D, C3 = 3 * W;
  const int K = KC > 0 ? KC : p.K;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __shared__ __align__(16) float qs[D];
  __shared__ __align__(16) float ks[D];
  __shared__ float vs[D];
  __shared__ float os[D];
  __shared__ float red[2 * NW];
  __shared__ float2 gate;
  // The state's last writer may be the grid just before this one (two calls
  // in a row on one state), so it is read after the wait; its lines are
  // pulled into L2 now.
  float* sp = f.state + ((int64_t)b * H + h) * D * D;
  if (f.has_state)
    for (int i = tid; i < D * D / 32; i += 4 * D)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(sp + (int64_t)i * 32));
  const int part = tid / D, c = tid % D;  // parts 0, 1, 2: q, k, v channel c of head h
  const int gc = part * W + h * D + c;
  float wk[KM];
#pragma unroll
  for (int j = 0; j < KM; ++j) wk[j] = 0.0f;
  if (part < 3) {  // conv weights are constants: loaded before the wait
    if constexpr (KC == 4) {
      const float4 w4 = *reinterpret_cast<const float4*>(p.conv_w + (int64_t)gc * 4);
      wk[0] = w4.x;
      wk[1] = w4.y;
      wk[2] = w4.z;
      wk[3] = w4.w;
    } else {
#pragma unroll
      for (int j = 0; j < KM; ++j) wk[j] = j < K ? p.conv_w[(int64_t)gc * K + j] : 0.0f;
    }
  }
  pdl_wait();
  pdl_launch_dependents();
  float y = 0.0f;
  if (part < 3) {
    // window: history slots 0 .. K-2 (oldest first), then this token's row
    float x[KM];
#pragma unroll
    for (int w = 0; w < KM; ++w) {
      x[w] = 0.0f;
      if (w < K - 1) {
        if (p.conv_state) x[w] = ld_bf16(p.conv_state + ((int64_t)b * (K - 1) + w) * C3 + gc);
      } else if (w == K - 1) {
        x[w] = ld_bf16(p.mixed + (int64_t)b * p.mixed_ld + gc);
      }
    }
    if (p.conv_state_out) {  // slot s takes x[s + 1]; this thread alone owns the channel
      uint16_t* cs = p.conv_state_out + (int64_t)b * (K - 1) * C3 + gc;
#pragma unroll
      for (int w = 1; w < KM; ++w)
        if (w < K) cs[(int64_t)(w - 1) * C3] = __bfloat16_as_ushort(__float2bfloat16_rn(x[w]));
    }
    float acc = 0.0f;
#pragma unroll
    for (int j = 0; j < KM; ++j)
      if (KC > 0 || j < K) acc = fmaf(wk[j], x[j], acc);
    y = acc * sigmoid_f(acc);
  }
  if (part == 2) vs[c] = y;
  if (part < 2) {  // whole warps: the q and k sums of squares
    float ss = y * y;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[warp] = ss;
  }
  if (part == 3 && c == 0) {  // gates, as gdn_prep_kernel
    const float bl = ld_bf16(p.b + (int64_t)b * p.b_ld + h);
    const float al = ld_bf16(p.a + (int64_t)b * p.a_ld + h);
    const float decay = softplus_f(al + p.dt_bias[h]) * -__expf(p.a_log[h]);
    gate = make_float2(__expf(decay), sigmoid_f(bl));
  }
  __syncthreads();
  if (part < 2) {
    float tot = 0.0f;
#pragma unroll
    for (int w = 0; w < NW; ++w) tot += red[part * NW + w];
    const float v = y * rsqrtf(tot + 1e-6f);
    if (part == 0)
      qs[c] = v * p.q_scale;
    else
      ks[c] = v;
  }
  __syncthreads();
  // delta rule on column j of the head's state (gdn_recurrence_kernel's step
  // for one token): a = k·S, δ = beta (v_j - g a), S = g S + k δ, o_j = q·S
  const int j = warp * (32 / LPC) + lane / LPC, pl = lane & (LPC - 1);
  float* colp = sp + (int64_t)j * D + 4 * pl;
  float st[R];
  if (f.has_state) {
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      const float4 v = *reinterpret_cast<const float4*>(colp + 4 * LPC * i);
      st[4 * i] = v.x;
      st[4 * i + 1] = v.y;
      st[4 * i + 2] = v.z;
      st[4 * i + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int r = 0; r < R; ++r) st[r] = 0.0f;
  }
  const float2 g = gate;
  float a = 0.0f;
  if (f.has_state) {
    float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      const float4 k4 = *reinterpret_cast<const float4*>(&ks[4 * LPC * i + 4 * pl]);
      a0 = fmaf(st[4 * i], k4.x, a0);
      a1 = fmaf(st[4 * i + 1], k4.y, a1);
      a0 = fmaf(st[4 * i + 2], k4.z, a0);
      a1 = fmaf(st[4 * i + 3], k4.w, a1);
    }
    a = a0 + a1;
#pragma unroll
    for (int o = 1; o < LPC; o <<= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
  }
  const float delta = (vs[j] - g.x * a) * g.y;
  float o0 = 0.0f, o1 = 0.0f;
#pragma unroll
  for (int i = 0; i < NI; ++i) {
    const float4 k4 = *reinterpret_cast<const float4*>(&ks[4 * LPC * i + 4 * pl]);
    const float4 q4 = *reinterpret_cast<const float4*>(&qs[4 * LPC * i + 4 * pl]);
    st[4 * i] = fmaf(k4.x, delta, st[4 * i] * g.x);
    st[4 * i + 1] = fmaf(k4.y, delta, st[4 * i + 1] * g.x);
    st[4 * i + 2] = fmaf(k4.z, delta, st[4 * i + 2] * g.x);
    st[4 * i + 3] = fmaf(k4.w, delta, st[4 * i + 3] * g.x);
    o0 = fmaf(st[4 * i], q4.x, o0);
    o1 = fmaf(st[4 * i + 1], q4.y, o1);
    o0 = fmaf(st[4 * i + 2], q4.z, o0);
    o1 = fmaf(st[4 * i + 3], q4.w, o1);
    *reinterpret_cast<float4*>(colp + 4 * LPC * i) =
        make_float4(st[4 * i], st[4 * i + 1], st[4 * i + 2], st[4 * i + 3]);
  }
  float o = o0 + o1;
#pragma unroll
  for (int s = 1; s < LPC; s <<= 1) o += __shfl_xor_sync(0xffffffffu, o, s);
  if (pl == 0) os[j] = o;
  __syncthreads();
  if (warp == 0) {  // gated RMSNorm over the head, as gdn_gated_norm_kernel
    float v[E], ss = 0.0f;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      v[e] = os[lane * E + e];
      ss = fmaf(v[e], v[e], ss);
    }
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, s);
    const float ns = rsqrtf(ss / (float)D + f.eps);
    const uint16_t* zr = f.z + (int64_t)b * f.z_ld + h * D + lane * E;
    uint16_t* outp = f.out + (int64_t)b * W + h * D + lane * E;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float z = ld_bf16(zr + e);
      const float r = ((v[e] * ns) * f.norm_w[lane * E + e]) * (z * sigmoid_f(z));
      outp[e] = __bfloat16_as_ushort(__float2bfloat16_rn(r));
    }
  }
}

template <int D, bool PROMPT>
int32_t launch_recurrence(const RecArgs& ra, int B, cudaStream_t s) {
  using Sh = RecShape<D, PROMPT>;
  const size_t smem = 2 * sizeof(Stage<D, Sh::CPB, Sh::CH>);
  auto rec = gdn_recurrence_kernel<D, PROMPT>;
  RXLA_CUDA_CHECK(cudaFuncSetAttribute(rec, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  cudaError_t e = launch_pdl(rec, dim3(D / Sh::CPB, ra.H, B), dim3(kRecWarps * 32), smem, s, ra);
  if (e != cudaSuccess) return cuda_fail(e, "gated_delta recurrence launch");
  return RXLA_B200_OK;
}

template <int D>
int32_t launch_all(const PrepArgs& pa, const RecArgs& ra, const NormArgs& na, int B, int T,
                   cudaStream_t s) {
  const bool k4 = pa.K == 4 && reinterpret_cast<uintptr_t>(pa.conv_w) % 16 == 0;
  const dim3 g1(3 * pa.H + 1, 1, B), gt(3 * pa.H + 1, (T + kPrepTokens - 1) / kPrepTokens, B);
  cudaError_t e;
  if (T == 1 && (int64_t)B * pa.H <= kFusedMaxCtas) {
    FusedArgs f;
    f.prep = pa;
    f.state = ra.state;
    f.has_state = ra.has_state;
    f.z = na.z;
    f.z_ld = na.z_ld;
    f.norm_w = na.norm_w;
    f.eps = na.eps;
    f.out = na.out;
    const dim3 gf(pa.H, B);
    e = k4 ? launch_pdl(gdn_decode_fused_kernel<D, 4>, gf, dim3(4 * D), 0, s, f)
           : launch_pdl(gdn_decode_fused_kernel<D, 0>, gf, dim3(4 * D), 0, s, f);
    if (e != cudaSuccess) return cuda_fail(e, "gated_delta fused decode launch");
    return RXLA_B200_OK;
  }
  if (T == 1)
    e = k4 ? launch_pdl(gdn_prep_kernel<D, 1, 4>, g1, dim3(D), 0, s, pa)
           : launch_pdl(gdn_prep_kernel<D, 1, 0>, g1, dim3(D), 0, s, pa);
  else
    e = k4 ? launch_pdl(gdn_prep_kernel<D, kPrepTokens, 4>, gt, dim3(D), 0, s, pa)
           : launch_pdl(gdn_prep_kernel<D, kPrepTokens, 0>, gt, dim3(D), 0, s, pa);
  if (e != cudaSuccess) return cuda_fail(e, "gated_delta prep launch");
  const int32_t rc = T > kLongCall ? launch_recurrence<D, true>(ra, B, s)
                                   : launch_recurrence<D, false>(ra, B, s);
  if (rc != RXLA_B200_OK) return rc;
  e = launch_pdl(gdn_gated_norm_kernel<D>, dim3((unsigned)(B * T)), dim3(kNormWarps * 32), 0, s, na);
  if (e != cudaSuccess) return cuda_fail(e, "gated_delta norm launch");
  return RXLA_B200_OK;
}

size_t workspace_bytes(int64_t rows, int64_t H, int64_t D) {
  // qkv [rows, 3W] f32, gates [rows, H] float2, o [rows, W] f32; each region
  // 256-byte aligned
  auto al = [](size_t v) { return (v + 255) & ~(size_t)255; };
  const int64_t W = H * D;
  return al((size_t)rows * 3 * W * 4) + al((size_t)rows * H * 8) + al((size_t)rows * W * 4);
}

}  // namespace gdn
}  // namespace rxla

extern "C" int32_t rxla_b200_gated_delta_workspace_size(int32_t batch, int32_t tokens,
                                                        int32_t heads, int32_t head_dim,
                                                        size_t* bytes) {
  using namespace rxla;
  RXLA_REQUIRE(bytes, "gated_delta_workspace_size: null argument");
  RXLA_REQUIRE(batch >= 0 && tokens >= 0 && heads > 0 && head_dim > 0,
               "gated_delta_workspace_size: bad shape");
  *bytes = gdn::workspace_bytes((int64_t)batch * tokens, heads, head_dim);
  return RXLA_B200_OK;
}

extern "C" int32_t rxla_b200_gated_delta(const rxla_b200_gated_delta_args* a, void* stream) {
  using namespace rxla;
  RXLA_REQUIRE(a && a->struct_size == sizeof(rxla_b200_gated_delta_args),
               "gated_delta: args null or struct_size mismatch");
  const int64_t B = a->batch, T = a->tokens, H = a->heads, D = a->head_dim, K = a->conv_kernel;
  RXLA_REQUIRE(B >= 0 && T >= 0, "gated_delta: batch and tokens must be >= 0");
  RXLA_REQUIRE(D == 32 || D == 64 || D == 128, "gated_delta: head_dim must be 32, 64 or 128");
  RXLA_REQUIRE(H > 0 && H <= 4096, "gated_delta: heads must lie in [1, 4096]");
  RXLA_REQUIRE(K >= 1 && K <= gdn::kMaxConvKernel, "gated_delta: conv_kernel must lie in [1, 8]");
  RXLA_REQUIRE(a->eps > 0.0f && a->eps == a->eps && a->eps < INFINITY,
               "gated_delta: epsilon must be finite and positive");
  if (B == 0 || T == 0) return RXLA_B200_OK;
  RXLA_REQUIRE(B * T <= INT32_MAX && B <= 65535 && (T + gdn::kPrepTokens - 1) / gdn::kPrepTokens <= 65535,
               "gated_delta: batch or tokens too large");
  const int64_t W = H * D;
  RXLA_REQUIRE(a->mixed && a->z && a->beta_logits && a->a && a->conv_weight && a->a_log &&
                   a->dt_bias && a->norm_weight && a->state && a->out && a->workspace,
               "gated_delta: null pointer");
  RXLA_REQUIRE(K == 1 || a->conv_state, "gated_delta: conv_state is required for conv_kernel > 1");
  RXLA_REQUIRE(a->mixed_row_stride >= 3 * W && a->z_row_stride >= W &&
                   a->b_row_stride >= H && a->a_row_stride >= H,
               "gated_delta: a row stride is shorter than its row");
  RXLA_REQUIRE(reinterpret_cast<uintptr_t>(a->state) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(a->workspace) % 256 == 0,
               "gated_delta: state must be 16-byte and workspace 256-byte aligned");
  const size_t need = gdn::workspace_bytes(B * T, H, D);
  RXLA_REQUIRE(a->workspace_bytes >= need, "gated_delta: workspace too small (see workspace_size)");
  auto al = [](size_t v) { return (v + 255) & ~(size_t)255; };
  uint8_t* ws = static_cast<uint8_t*>(a->workspace);
  float* qkv = reinterpret_cast<float*>(ws);
  float2* gb = reinterpret_cast<float2*>(ws + al((size_t)B * T * 3 * W * 4));
  float* o = reinterpret_cast<float*>(ws + al((size_t)B * T * 3 * W * 4) + al((size_t)B * T * H * 8));

  gdn::PrepArgs pa;
  pa.mixed = a->mixed;
  pa.b = a->beta_logits;
  pa.a = a->a;
  pa.mixed_ld = a->mixed_row_stride;
  pa.b_ld = a->b_row_stride;
  pa.a_ld = a->a_row_stride;
  pa.conv_w = a->conv_weight;
  pa.a_log = a->a_log;
  pa.dt_bias = a->dt_bias;
  pa.conv_state = (a->has_state && K > 1) ? a->conv_state : nullptr;
  pa.conv_state_out = K > 1 ? a->conv_state : nullptr;
  pa.qkv = qkv;
  pa.gb = gb;
  pa.T = (int32_t)T;
  pa.H = (int32_t)H;
  pa.K = (int32_t)K;
  pa.q_scale = 1.0f / sqrtf((float)D);

  gdn::RecArgs ra;
  ra.qkv = qkv;
  ra.gb = gb;
  ra.state = a->state;
  ra.has_state = a->has_state;
  ra.o = o;
  ra.T = (int32_t)T;
  ra.H = (int32_t)H;

  gdn::NormArgs na;
  na.o = o;
  na.z = a->z;
  na.z_ld = a->z_row_stride;
  na.norm_w = a->norm_weight;
  na.eps = a->eps;
  na.out = a->out;
  na.mixed = a->mixed;
  na.mixed_ld = a->mixed_row_stride;
  na.conv_state = a->conv_state;
  na.has_state = a->has_state;
  na.T = (int32_t)T;
  na.H = (int32_t)H;
  na.K = (int32_t)K;
  na.vec = D == 128 && reinterpret_cast<uintptr_t>(a->z) % 8 == 0 && a->z_row_stride % 4 == 0 &&
           reinterpret_cast<uintptr_t>(a->norm_weight) % 16 == 0 &&
           reinterpret_cast<uintptr_t>(a->out) % 8 == 0;

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (D == 128) return gdn::launch_all<128>(pa, ra, na, (int)B, (int)T, s);
  if (D == 64) return gdn::launch_all<64>(pa, ra, na, (int)B, (int)T, s);
  return gdn::launch_all<32>(pa, ra, na, (int)B, (int)T, s);
}
