// w8_linear.cu — W8A16 linear for decode shapes (M <= 32 tokens per pass).
//
// Replaces QuantizedLinear::apply (crates/rxla-nn/src/layers.rs:257-298) with
// BF16 layer compute, at the reference's rounding points: every weight is
// dequantized in f32 (q = u8 - 128, exact; q·s rounded once to f32), rounded
// to bf16 (the cast of W_deq, :293-296), multiplied with bf16(x) exactly and
// accumulated in fp32; the dot is rounded to bf16.
//
// Design (HBM-bound: one byte of weight per multiply-add at M = 1):
//  * persistent grid, one CTA per SM; CTA c owns output rows
//    [c·R/G, (c+1)·R/G) — balanced to one row, so no SM streams more than
//    ceil(R/G) rows;
//  * a producer warp streams the CTA's rows through a ring of shared-memory
//    stages with the TMA bulk-copy engine (cp.async.bulk, L2 evict-first).  A
//    stage is 8 consecutive rows × KC columns: when KC == K it is ONE
//    contiguous copy of up to 48 KB, otherwise one copy per row.  The engine
//    costs ~70 cycles per request on an SM, so large copies are what let it
//    stream at HBM speed (512 B copies cap it near 2 TB/s);
//  * the ring is filled before griddepcontrol.wait — weights do not depend on
//    the previous kernel — so with PDL the CTA's first 100-200 KB of weights
//    are in flight while the previous kernel finishes; x (the previous
//    kernel's output) is then copied once into shared memory;
//  * 16 consumer warps split each stage into 64-column boxes of 16 rows and
//    feed mma.sync m16n8k16 (bf16 in, fp32 accumulate) with weight rows on
//    the M side and tokens on the N side, so there is no cross-lane reduction
//    over K.  Dequantization runs in registers: PRMT puts the byte b in a
//    denormal's mantissa (b·2^-133, exact), one FFMA with s·2^133 and -128·s
//    rounds (b - 128)·s once (the reference's f32 product), cvt.rn.bf16x2
//    rounds to bf16: 1.5 integer-pipe + 1 FMA-pipe instruction per weight.  For SwiGLU, rows 0-7 of the A tile are
//    gate rows and rows 8-15 the matching up rows.  The K columns are permuted
//    consistently for A and B: a lane reads 16 contiguous weight bytes and the
//    16 matching x values, which covers four k-steps;
//  * an epilogue warp sums the 16 warps' partial tiles in a fixed order
//    (deterministic), scales, rounds to bf16 and stores / adds to the f32
//    residual / gates with SiLU, double-buffered so the consumers never wait
//    for it.
#include <algorithm>

#include <cuda_fp16.h>

#include "internal.cuh"

namespace rxla {
namespace w8 {

constexpr int kConsumerWarps = 16;
constexpr int kProducerWarp = kConsumerWarps;
constexpr int kEpilogueWarp = kConsumerWarps + 1;
constexpr int kThreads = (kConsumerWarps + 2) * 32;
constexpr int kTileRows = 16;       // A rows per block (16 outputs, or 8 gate + 8 up)
constexpr int kMaxStages = 8;
constexpr int kMaxTokens = 8;       // tokens per pass (one n-tile)
constexpr int kRedFloats = kConsumerWarps * kTileRows * kMaxTokens;
constexpr int kHeader = 1024;       // barriers + norm partials
constexpr int kEarlyBytes = 64 * 1024;  // weights requested before griddepcontrol.wait

// Where x comes from.
enum XMode : int {
  kXBf16 = 0,  // bf16 [m, k]: bulk-copied into shared memory by the producer
  kXF32 = 1,   // f32 [m, k]: rounded to bf16 by the consumers (QuantizedLinear's cast)
  kXNorm = 2   // f32 residual h [m, k]: bf16(rms_norm(h) * norm_w), ops.rs:929-945
};

// Epilogue codes beyond the public ones (rxla_b200_epilogue).
constexpr int kEpiArgmax = 16;  // logits (f32, optional) + greedy token per row

struct Params {
  const uint8_t* w;
  const float* scale;
  const void* x;
  void* y;
  int32_t m, k;        // tokens in this pass (<= 8), reduction width
  int32_t n;           // output columns (pairs for SwiGLU)
  int32_t groups;      // k / group_size
  int32_t group_size;
  int64_t ldx, ldy;    // row strides of x and y in elements
  int32_t x_f32, y_f32, epilogue;
  // fused RMSNorm (kXNorm)
  const float* norm_w;
  float norm_eps;
  // fused greedy argmax (kEpiArgmax): per-CTA partials, arrival counter, result
  float* arg_val;       // [grid][8]
  int32_t* arg_idx;     // [grid][8]
  uint32_t* arg_count;  // one counter, zero between launches
  int32_t* arg_out;     // [m]
  int32_t* arg_advance; // optional [m], += 1 per row (decoder position)
  // shared-memory plan (set by the host)
  int32_t kc;           // K columns per stage (multiple of 64)
  int32_t k_chunks;     // ceil(k / kc)
  int32_t stages;       // ring depth
  int32_t x_pitch;      // bytes of one resident bf16 token row of x
  int32_t stage_bytes;  // 16 rows × kc
  L2Prefetch next;      // the following kernel's first bytes (last pass only)
  // row-parallel all-reduce in the epilogue (tp.world > 1, RESIDUAL_ADD into
  // the f32 residual y): partials to every rank's peer buffer, then the sum
  // over ranks in rank order once the same CTA of every rank has pushed
  P2pView tp;
};

struct Bars {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t x_issued;  // every consumer warp has issued its loads of x
  uint64_t grp[2];
  uint64_t ss_free;  // norm: every warp has read a round's sums
  uint64_t epi_full[2];
  uint64_t epi_free[2];
  float ss[kConsumerWarps][kMaxTokens];  // norm: per-warp sums of squares
};
static_assert(sizeof(Bars) <= kHeader, "header");

// Row constants of the exact dequantization below: sbig = s·2^133 and
// c = -128·s, both exact while s < 2^-5 (larger scales are pre-divided by a
// power of two and the product multiplied back: `post`).  Each constant is
// held twice, as the f32x2 operand of the packed FMA.
struct RowScale {
  uint64_t sbig, c, post;
};

__device__ __forceinline__ uint64_t dup_f32(float v) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %1};" : "=l"(r) : "f"(v));
  return r;
}

__device__ __forceinline__ RowScale row_scale(float s) {
  float post = 1.0f;
  if (!(fabsf(s) < 0.03125f) && s == s && fabsf(s) < INFINITY) {
    const int e = ((__float_as_int(s) >> 23) & 0xff) - 127;  // s in [2^e, 2^(e+1))
    const int k = e + 6;                                     // s·2^-k < 2^-5
    s = s * __int_as_float((127 - k) << 23);
    post = __int_as_float((127 + k) << 23);
  }
  RowScale r;
  r.c = dup_f32(-128.0f * s);
  r.sbig = dup_f32((s * 0x1p100f) * 0x1p33f);  // s·2^133 (exact: two power-of-two steps)
  r.post = dup_f32(post);
  return r;
}

__device__ __forceinline__ bool needs_post(const RowScale& r) {
  return r.post != 0x3f8000003f800000ull;  // post != 1
}

// Four u8 weights of one row (value b, q = b - 128) -> two bf16x2 registers of
// bf16(f32(q)·s), the reference's rounding: lo = (w0, w1), hi = (w2, w3).
// PRMT places b in the mantissa of a denormal (b·2^-133, exact); the packed
// fma(b·2^-133, s·2^133, -128·s) rounds (b - 128)·s once, as f32(q)·s does
// (denormal operands are kept: no .ftz).
template <bool POST>
__device__ __forceinline__ void deq4(uint32_t w, const RowScale& r, uint32_t& lo, uint32_t& hi) {
  uint64_t a01, a23, p01, p23;
  asm("mov.b64 %0, {%1, %2};" : "=l"(a01) : "r"(__byte_perm(w, 0u, 0x4044u)),
      "r"(__byte_perm(w, 0u, 0x4144u)));
  asm("mov.b64 %0, {%1, %2};" : "=l"(a23) : "r"(__byte_perm(w, 0u, 0x4244u)),
      "r"(__byte_perm(w, 0u, 0x4344u)));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(p01) : "l"(a01), "l"(r.sbig), "l"(r.c));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(p23) : "l"(a23), "l"(r.sbig), "l"(r.c));
  if (POST) {
    asm("mul.rn.f32x2 %0, %0, %1;" : "+l"(p01) : "l"(r.post));
    asm("mul.rn.f32x2 %0, %0, %1;" : "+l"(p23) : "l"(r.post));
  }
  float f0, f1, f2, f3;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(f0), "=f"(f1) : "l"(p01));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(f2), "=f"(f3) : "l"(p23));
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(lo) : "f"(f1), "f"(f0));
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(hi) : "f"(f3), "f"(f2));
}

// Bounded barrier among the 16 consumer warps (one arrival per warp).
__device__ __forceinline__ bool consumer_sync(uint64_t* bar, uint32_t parity) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
  return mbar_wait(bar, parity);
}

// One 64-column box of a 16-row tile: 16 B of rows g and g+8 per lane, the
// lane's 16 x values, four k-steps of m16n8k16.  Lanes whose token column is
// beyond the batch read a real token's x: those output columns are ignored.
template <bool POST>
__device__ __forceinline__ void box_mma(float (&acc)[4], const uint8_t* wg, int row8,
                                        const uint8_t* xcol, const RowScale& ra,
                                        const RowScale& rb) {
  const uint4 v0 = *reinterpret_cast<const uint4*>(xcol);
  const uint4 v1 = *reinterpret_cast<const uint4*>(xcol + 16);
  const uint32_t bx[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
  const uint4 lo = *reinterpret_cast<const uint4*>(wg);
  const uint4 hi = *reinterpret_cast<const uint4*>(wg + row8);
  const uint32_t wl[4] = {lo.x, lo.y, lo.z, lo.w};
  const uint32_t wh[4] = {hi.x, hi.y, hi.z, hi.w};
#pragma unroll
  for (int st = 0; st < 4; ++st) {
    uint32_t a[4];
    deq4<POST>(wl[st], ra, a[0], a[2]);  // row g: k-low pair, k-high pair
    deq4<POST>(wh[st], rb, a[1], a[3]);  // row g+8
    mma_bf16_16816(acc, a, bx[2 * st], bx[2 * st + 1]);
  }
}

// The same box with the lane's x fragments held in registers (loaded once per
// launch when the whole row is one stage: the x shared-memory loads per box
// were half of the loop's shared traffic).
template <bool POST>
__device__ __forceinline__ void box_mma_xr(float (&acc)[4], const uint8_t* wg, int row8,
                                           const uint32_t (&bx)[8], const RowScale& ra,
                                           const RowScale& rb) {
  const uint4 lo = *reinterpret_cast<const uint4*>(wg);
  const uint4 hi = *reinterpret_cast<const uint4*>(wg + row8);
  const uint32_t wl[4] = {lo.x, lo.y, lo.z, lo.w};
  const uint32_t wh[4] = {hi.x, hi.y, hi.z, hi.w};
#pragma unroll
  for (int st = 0; st < 4; ++st) {
    uint32_t a[4];
    deq4<POST>(wl[st], ra, a[0], a[2]);
    deq4<POST>(wh[st], rb, a[1], a[3]);
    mma_bf16_16816(acc, a, bx[2 * st], bx[2 * st + 1]);
  }
}

constexpr int kXRegBoxes = 4;  // x of up to 4 boxes per warp (k <= 4096) in registers

template <bool SWIGLU, bool GROUPED, int XMODE, bool XREG = false>
__global__ void __launch_bounds__(kThreads, 1) w8_skinny_kernel(const Params p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  Bars& bars = *reinterpret_cast<Bars*>(smem_raw);
  float* red = reinterpret_cast<float*>(smem_raw + kHeader);  // [2][warp][16 rows][8 tokens]
  uint8_t* xs = smem_raw + kHeader + 2 * kRedFloats * 4;       // bf16 [m][x_pitch]
  uint8_t* stages = xs + (size_t)p.m * p.x_pitch;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  constexpr int out_rows = SWIGLU ? kTileRows / 2 : kTileRows;

  // balanced contiguous share of output rows for this CTA
  const int64_t R = p.n;
  const int r_begin = (int)((R * blockIdx.x) / gridDim.x);
  const int r_end = (int)((R * (blockIdx.x + 1)) / gridDim.x);
  const int n_blocks = (r_end - r_begin + out_rows - 1) / out_rows;
  const int total = n_blocks * p.k_chunks;
  const int S = p.stages;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&bars.full[s], 1);
      mbar_init(&bars.empty[s], kConsumerWarps);
    }
    mbar_init(&bars.x_issued, kConsumerWarps);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars.grp[i], kConsumerWarps);
      if (i == 0) mbar_init(&bars.ss_free, kConsumerWarps);
      mbar_init(&bars.epi_full[i], kConsumerWarps);
      mbar_init(&bars.epi_free[i], 1);
    }
    fence_mbarrier_init();
  }
  __syncthreads();

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------ producer
    const uint64_t policy = l2_evict_first_policy();
    auto issue = [&](int it, int s) {
      const int blk = it / p.k_chunks, kc = it % p.k_chunks;
      const int r0 = r_begin + blk * out_rows;
      const int nr = min(out_rows, r_end - r0);
      const int col0 = kc * p.kc;
      const int cols = min(p.kc, p.k - col0);
      const uint32_t tx = (uint32_t)cols * (uint32_t)nr * (SWIGLU ? 2u : 1u);
      if (lane == 0) mbar_arrive_expect_tx(&bars.full[s], tx);
      __syncwarp();
      uint8_t* dst = stages + (size_t)s * p.stage_bytes;
      if (cols == p.k) {
        // whole rows: the block is one contiguous range (two for SwiGLU)
        if (lane == 0)
          bulk_g2s(dst, p.w + (int64_t)r0 * p.k, (uint32_t)(nr * p.k), &bars.full[s], policy);
        if (SWIGLU && lane == 1)
          bulk_g2s(dst + (kTileRows / 2) * p.kc, p.w + (int64_t)(p.n + r0) * p.k,
                   (uint32_t)(nr * p.k), &bars.full[s], policy);
      } else {
        const int i = SWIGLU ? (lane & 7) : lane;
        const bool up = SWIGLU && lane >= 8;
        if (lane < kTileRows && i < nr) {
          const int64_t row = up ? (int64_t)p.n + r0 + i : (int64_t)r0 + i;
          bulk_g2s(dst + (size_t)lane * p.kc, p.w + row * p.k + col0, (uint32_t)cols,
                   &bars.full[s], policy);
        }
      }
    };
    // Weights do not depend on the previous kernel: up to kEarlyBytes of them
    // are requested before griddepcontrol.wait, so the stream starts while
    // the previous kernel drains.  The rest of the ring waits until every
    // consumer warp has issued its loads of x (the previous kernel's output,
    // read after the wait): loads issued behind a full ring of this SM's
    // weight copies wait for those copies first (~190 KB at this SM's share
    // of HBM bandwidth is ~4 µs).
    const int pre = min(S, total);
    const int early = min(pre, max(1, kEarlyBytes / p.stage_bytes));
    for (int it = 0; it < early; ++it) issue(it, it);
    if (!mbar_wait(&bars.x_issued, 0)) return;
    for (int it = early; it < pre; ++it) issue(it, it);
    // bf16 x is copied by the consumers after griddepcontrol.wait: a bulk
    // copy issued here would queue behind the ring's weight copies in this
    // SM's TMA engine (down_proj's 48 row copies delayed x by ~1.7 µs)
    for (int it = pre; it < total; ++it) {
      const int s = it % S;
      if (!mbar_wait(&bars.empty[s], ((it / S) - 1) & 1)) return;
      issue(it, s);
    }
    // own loads are all issued: pull the next kernel's first bytes into L2
    if (lane == 0 && p.next.nseg > 0) l2_prefetch_share(p.next, blockIdx.x, gridDim.x);
    return;
  }

  const int g = lane >> 2;  // mma group id: A rows g, g+8; B column (token) g
  const int q = lane & 3;   // k-quad

  if (warp == kEpilogueWarp) {
    // ------------------------------------------------------------ epilogue
    pdl_wait();  // y (or the residual it adds into) may be used by the previous kernel
    pdl_launch_dependents();
    const bool argmax = p.epilogue == kEpiArgmax;
    // tensor parallelism: this CTA's call number on its flag slot, read after
    // the wait (the previous user of the slot, two row-parallel linears ago,
    // has completed), and the data slot it selects
    const bool tp = p.tp.world > 1;
    const uint64_t tp_e = tp ? p.tp.epoch[blockIdx.x] + 1 : 0;
    const int64_t tp_off = tp ? ((int64_t)(tp_e & 1) * kP2pMaxRanks + p.tp.rank) * p.tp.cap : 0;
    float best_v[kMaxTokens];
    int best_i[kMaxTokens];
#pragma unroll
    for (int t = 0; t < kMaxTokens; ++t) {
      best_v[t] = -INFINITY;
      best_i[t] = 0x7fffffff;
    }
    constexpr int kPerLane = (out_rows * kMaxTokens) / 32;
    for (int blk = 0; blk < n_blocks; ++blk) {
      const int b2 = blk & 1;
      const int r0 = r_begin + blk * out_rows;
      const int nr = min(out_rows, r_end - r0);
      // the residual this block adds into is read before its partials are
      // waited for, so the load overlaps the consumers' tiles
      float resid[kPerLane];
#pragma unroll
      for (int tt = 0; tt < kPerLane; ++tt) {
        const int idx = lane + 32 * tt;
        const int row = idx % out_rows, tok = idx / out_rows;
        resid[tt] = (!SWIGLU && !tp && p.epilogue == RXLA_B200_EPI_RESIDUAL_ADD && row < nr &&
                     tok < p.m)
                        ? static_cast<const float*>(p.y)[(int64_t)tok * p.ldy + r0 + row]
                        : 0.0f;
      }
      if (!mbar_wait(&bars.epi_full[b2], (blk >> 1) & 1)) return;
      const float* rb = red + b2 * kRedFloats;
#pragma unroll
      for (int tt = 0; tt < kPerLane; ++tt) {
        const int idx = lane + 32 * tt;
        const int row = idx % out_rows, tok = idx / out_rows;
        if (row >= nr || tok >= p.m) continue;
        float v = 0.0f, u = 0.0f;
#pragma unroll
        for (int w2 = 0; w2 < kConsumerWarps; ++w2) {
          v += rb[(w2 * kTileRows + row) * kMaxTokens + tok];
          if (SWIGLU) u += rb[(w2 * kTileRows + row + 8) * kMaxTokens + tok];
        }
        const int out_col = r0 + row;
        const int64_t o = (int64_t)tok * p.ldy + out_col;
        if (SWIGLU) {
          const float r = silu(bf16_round(v)) * bf16_round(u);
          if (p.y_f32) static_cast<float*>(p.y)[o] = r;
          else static_cast<__nv_bfloat16*>(p.y)[o] = __float2bfloat16_rn(r);
        } else if (argmax) {
          if (p.y) static_cast<float*>(p.y)[o] = v;
#pragma unroll
          for (int t = 0; t < kMaxTokens; ++t)
            if (t == tok && (v > best_v[t] || (v == best_v[t] && out_col < best_i[t]))) {
              best_v[t] = v;
              best_i[t] = out_col;
            }
        } else if (p.epilogue == RXLA_B200_EPI_RESIDUAL_ADD) {
          if (tp) {
            // this rank's partial of (token, column) into every rank's slot
            for (int q2 = 0; q2 < p.tp.world; ++q2)
              reinterpret_cast<float*>(p.tp.peer[q2])[tp_off + o] = v;
          } else {
            static_cast<float*>(p.y)[o] = resid[tt] + bf16_round(v);
          }
        } else if (p.y_f32) {
          static_cast<float*>(p.y)[o] = v;
        } else {
          static_cast<__nv_bfloat16*>(p.y)[o] = __float2bfloat16_rn(v);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars.epi_free[b2]);
    }
    if (tp) {
      // Every partial of this CTA's rows is in every rank's slot: publish the
      // call number in each rank's flag [rank][cta] (a system-scope fence
      // first, cumulative over the warp's stores), wait (bounded) until every
      // rank's flag [q][cta] here reached it, then sum the ranks' rows in rank
      // order 0..world-1 — the same bits on every rank — and add bf16(sum) to
      // the residual.  The same CTA index covers the same rows on every rank
      // (same grid, same row split).
      const size_t data_bytes = (size_t)2 * kP2pMaxRanks * p.tp.cap * 4;
      __syncwarp();
      if (lane == 0) {
        __threadfence_system();
        for (int q2 = 0; q2 < p.tp.world; ++q2)
          st_relaxed_sys(reinterpret_cast<uint64_t*>(p.tp.peer[q2] + data_bytes) +
                             (int64_t)p.tp.rank * p.tp.max_ctas + blockIdx.x,
                         tp_e);
      }
      bool arrived = true;
      if (lane < p.tp.world) {
        const uint64_t* flag = reinterpret_cast<const uint64_t*>(p.tp.peer[p.tp.rank] + data_bytes) +
                               (int64_t)lane * p.tp.max_ctas + blockIdx.x;
        if (ld_acquire_sys(flag) < tp_e) {
          const unsigned long long limit = wait_timeout_ns();
          const uint64_t t0 = globaltimer();
          while (ld_acquire_sys(flag) < tp_e) {
            if (globaltimer() - t0 > limit) {
              record_device_error(RXLA_B200_DEADLINE_EXCEEDED);
              arrived = false;
              break;
            }
          }
        }
      }
      if (!__all_sync(0xffffffffu, arrived)) return;
      const float* rows = reinterpret_cast<const float*>(p.tp.peer[p.tp.rank]) +
                          (int64_t)(tp_e & 1) * kP2pMaxRanks * p.tp.cap;
      const int nrow = r_end - r_begin;
      for (int idx = lane; idx < nrow * p.m; idx += 32) {
        const int64_t o = (int64_t)(idx / nrow) * p.ldy + r_begin + idx % nrow;
        float acc = __ldcv(rows + o);
        for (int q2 = 1; q2 < p.tp.world; ++q2) acc += __ldcv(rows + (int64_t)q2 * p.tp.cap + o);
        float* hh = static_cast<float*>(p.y) + o;
        *hh = *hh + bf16_round(acc);
      }
      if (lane == 0) p.tp.epoch[blockIdx.x] = tp_e;
    }
    if (argmax) {
      // per-CTA best of each row, then the last CTA to arrive picks the token
#pragma unroll
      for (int t = 0; t < kMaxTokens; ++t) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, best_v[t], o);
          const int oi = __shfl_xor_sync(0xffffffffu, best_i[t], o);
          if (ov > best_v[t] || (ov == best_v[t] && oi < best_i[t])) {
            best_v[t] = ov;
            best_i[t] = oi;
          }
        }
      }
      if (lane == 0) {
#pragma unroll
        for (int t = 0; t < kMaxTokens; ++t) {  // compile-time t: best_v / best_i stay in registers
          if (t < p.m) {
            p.arg_val[blockIdx.x * kMaxTokens + t] = best_v[t];
            p.arg_idx[blockIdx.x * kMaxTokens + t] = best_i[t];
          }
        }
        __threadfence();
      }
      uint32_t prev = 0;
      if (lane == 0) prev = atomicAdd(p.arg_count, 1u);
      prev = __shfl_sync(0xffffffffu, prev, 0);
      if (prev == gridDim.x - 1) {
        // the last CTA picks each row's token from all CTAs' partials: the
        // lanes scan CTAs in parallel, then (value desc, index asc) reduce
        __threadfence();
        for (int t = 0; t < p.m; ++t) {
          float bv = -INFINITY;
          int bi = 0x7fffffff;
          for (int c = lane; c < (int)gridDim.x; c += 32) {
            const float v = __ldcg(p.arg_val + c * kMaxTokens + t);
            const int i = __ldcg(p.arg_idx + c * kMaxTokens + t);
            if (v > bv || (v == bv && i < bi)) {
              bv = v;
              bi = i;
            }
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) {
              bv = ov;
              bi = oi;
            }
          }
          if (lane == 0) {
            p.arg_out[t] = bi == 0x7fffffff ? 0 : bi;
            if (p.arg_advance) p.arg_advance[t] += 1;
          }
        }
        if (lane == 0) *p.arg_count = 0u;
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int ctid = threadIdx.x;  // 0 .. 511
  // weight rows of this lane's A fragment in block blk: tile rows g and g + 8
  // (the first block's scales are constants: loaded before the wait below)
  auto block_rows = [&](int blk, bool& va, bool& vb, int& ra, int& rb) {
    const int r0 = r_begin + blk * out_rows;
    const int nr = min(out_rows, r_end - r0);
    if (SWIGLU) {
      va = vb = g < nr;
      ra = r0 + g;
      rb = p.n + r0 + g;
    } else {
      va = g < nr;
      vb = g + 8 < nr;
      ra = r0 + g;
      rb = r0 + g + 8;
    }
  };
  // per-channel scales are loaded one block ahead, so their latency hides
  // behind the current block's tiles
  float next_sa = 0.0f, next_sb = 0.0f;
  if (!GROUPED && n_blocks > 0) {
    bool va, vb;
    int ra, rb;
    block_rows(0, va, vb, ra, rb);
    next_sa = va ? __ldg(p.scale + ra) : 0.0f;
    next_sb = vb ? __ldg(p.scale + rb) : 0.0f;
  }

  if (XMODE == kXBf16) {
    pdl_wait();  // x is the previous kernel's output
    const int chunks = p.k / 8;  // 16-byte chunks of a token row (k % 64 == 0)
    for (int t = 0; t < p.m; ++t) {
      const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(p.x) +
                                                        (int64_t)t * p.ldx * 2);
      uint4* dst = reinterpret_cast<uint4*>(xs + t * p.x_pitch);
      for (int c = ctid; c < chunks; c += kConsumerWarps * 32) dst[c] = __ldcg(src + c);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&bars.x_issued);
    if (!consumer_sync(&bars.grp[1], 0)) return;
  } else {
    const float* xf = static_cast<const float*>(p.x);
    // This runs between the previous kernel and the first tile, so every
    // global load of a token is issued before any is used: one round trip per
    // two tokens (each consumer thread holds kXV float4 of a row; larger k
    // falls back to a strided loop).
    constexpr int kXV = 4;
    constexpr int kCT = kConsumerWarps * 32;
    const bool regs = p.k <= kXV * 4 * kCT;
    // the norm weights are constants: fetched before the wait, so their
    // latency overlaps the previous kernel's tail
    float4 nw[kXV];
#pragma unroll
    for (int i = 0; i < kXV; ++i) {
      const int c = (ctid + i * kCT) * 4;
      nw[i] = (XMODE == kXNorm && regs && c < p.k)
                  ? __ldg(reinterpret_cast<const float4*>(p.norm_w + c))
                  : make_float4(1.0f, 1.0f, 1.0f, 1.0f);
    }
    pdl_wait();  // x / h come from the previous kernel
    int round = 0;
    if (!regs) {  // strided loads below: let the ring fill right away
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars.x_issued);
    }
    for (int t0 = 0; t0 < p.m; t0 += 2, ++round) {
      const int nt = min(2, p.m - t0);
      float4 hv[2][kXV];
      float ss[2] = {0.0f, 0.0f};
      if (regs) {
#pragma unroll
        for (int u = 0; u < 2; ++u)
#pragma unroll
          for (int i = 0; i < kXV; ++i) {
            const int c = (ctid + i * kCT) * 4;
            hv[u][i] = (u < nt && c < p.k)
                           ? __ldg(reinterpret_cast<const float4*>(xf + (int64_t)(t0 + u) * p.ldx + c))
                           : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          }
        if (round == 0) {  // the first tokens' loads are in flight: the ring may fill up
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars.x_issued);
        }
#pragma unroll
        for (int u = 0; u < 2; ++u)
#pragma unroll
          for (int i = 0; i < kXV; ++i)
            ss[u] += hv[u][i].x * hv[u][i].x + hv[u][i].y * hv[u][i].y +
                     hv[u][i].z * hv[u][i].z + hv[u][i].w * hv[u][i].w;
      } else if (XMODE == kXNorm) {
        for (int u = 0; u < nt; ++u) {
          const float* row = xf + (int64_t)(t0 + u) * p.ldx;
          for (int c = ctid * 4; c < p.k; c += kCT * 4) {
            const float4 h = __ldg(reinterpret_cast<const float4*>(row + c));
            ss[u] += h.x * h.x + h.y * h.y + h.z * h.z + h.w * h.w;
          }
        }
      }
      float inv[2] = {1.0f, 1.0f};
      if (XMODE == kXNorm) {
        // sum of squares per token: threads, then warps, then the CTA
#pragma unroll
        for (int u = 0; u < 2; ++u) {
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) ss[u] += __shfl_xor_sync(0xffffffffu, ss[u], o);
        }
        if (lane == 0) {
          bars.ss[warp][0] = ss[0];
          bars.ss[warp][1] = ss[1];
        }
        if (!consumer_sync(&bars.grp[0], round & 1)) return;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          float tot = 0.0f;
          for (int w2 = 0; w2 < kConsumerWarps; ++w2) tot += bars.ss[w2][u];
          inv[u] = 1.0f / sqrtf(tot / (float)p.k + p.norm_eps);
        }
        // every warp has read the sums before the next round overwrites them
        if (t0 + 2 < p.m && !consumer_sync(&bars.ss_free, round & 1)) return;
      }
      // u is a compile-time index (a runtime one would move hv to local memory,
      // which misses the small L1 left beside a full shared-memory carve-out)
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (u >= nt) break;
        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(xs + (t0 + u) * p.x_pitch);
        if (regs) {
#pragma unroll
          for (int i = 0; i < kXV; ++i) {
            const int c = (ctid + i * kCT) * 4;
            if (c < p.k) {
              float4 h = hv[u][i];
              if (XMODE == kXNorm) {
                h.x = (h.x * inv[u]) * nw[i].x;
                h.y = (h.y * inv[u]) * nw[i].y;
                h.z = (h.z * inv[u]) * nw[i].z;
                h.w = (h.w * inv[u]) * nw[i].w;
              }
              uint2 pk;
              pk.x = pack_bf16x2(h.x, h.y);
              pk.y = pack_bf16x2(h.z, h.w);
              *reinterpret_cast<uint2*>(out + c) = pk;
            }
          }
        } else {
          const float* row = xf + (int64_t)(t0 + u) * p.ldx;
          for (int c = ctid * 4; c < p.k; c += kCT * 4) {
            float4 h = __ldg(reinterpret_cast<const float4*>(row + c));
            if (XMODE == kXNorm) {
              const float4 w = __ldg(reinterpret_cast<const float4*>(p.norm_w + c));
              h.x = (h.x * inv[u]) * w.x;
              h.y = (h.y * inv[u]) * w.y;
              h.z = (h.z * inv[u]) * w.z;
              h.w = (h.w * inv[u]) * w.w;
            }
            uint2 pk;
            pk.x = pack_bf16x2(h.x, h.y);
            pk.y = pack_bf16x2(h.z, h.w);
            *reinterpret_cast<uint2*>(out + c) = pk;
          }
        }
      }
    }
    if (!consumer_sync(&bars.grp[1], 0)) return;
  }
  const uint8_t* xrow = xs + (g % p.m) * p.x_pitch;
  // XREG (one stage holds whole rows, k <= 4096): this warp's boxes of the
  // row are column blocks warp + 16 i; their x fragments stay in registers
  uint32_t xr[XREG ? kXRegBoxes : 1][8];
  const int nbx = XREG ? p.k / (kConsumerWarps * 64) : 0;
  if (XREG) {
#pragma unroll
    for (int i = 0; i < (XREG ? kXRegBoxes : 1); ++i) {
      if (i < nbx) {
        const uint8_t* xc = xrow + ((warp + kConsumerWarps * i) * 64 + 16 * q) * 2;
        const uint4 v0 = *reinterpret_cast<const uint4*>(xc);
        const uint4 v1 = *reinterpret_cast<const uint4*>(xc + 16);
        xr[i][0] = v0.x; xr[i][1] = v0.y; xr[i][2] = v0.z; xr[i][3] = v0.w;
        xr[i][4] = v1.x; xr[i][5] = v1.y; xr[i][6] = v1.z; xr[i][7] = v1.w;
      }
    }
  }

  // ring position, advanced incrementally (no division in the loop)
  int s = 0;
  uint32_t ph = 0;
  // this lane's bytes in a stage: row g of the warp's first box; row g + 8 is
  // row8 further, and the warp's boxes are kConsumerWarps * 64 bytes apart
  const int lane_off = g * p.kc + warp * 64 + 16 * q;
  const int row8 = 8 * p.kc;
  constexpr int kBoxStep = kConsumerWarps * 64;
  for (int blk = 0; blk < n_blocks; ++blk) {
    bool va, vb;
    int ra, rb;
    block_rows(blk, va, vb, ra, rb);
    const float* sa = p.scale + (int64_t)ra * p.groups;
    const float* sb = p.scale + (int64_t)rb * p.groups;
    RowScale rsa = row_scale(0.0f), rsb = row_scale(0.0f);
    bool post = false;  // warp-uniform: some row's scale needs the power-of-two fixup
    if (!GROUPED) {
      rsa = row_scale(next_sa);
      rsb = row_scale(next_sb);
      post = __any_sync(0xffffffffu, needs_post(rsa) || needs_post(rsb));
      if (blk + 1 < n_blocks) {
        bool na, nb;
        int rna, rnb;
        block_rows(blk + 1, na, nb, rna, rnb);
        next_sa = na ? __ldg(p.scale + rna) : 0.0f;
        next_sb = nb ? __ldg(p.scale + rnb) : 0.0f;
      }
    }
    float acc0[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    float acc1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (XREG) {
      // one stage per block; boxes i and i + 1 go to the two accumulators,
      // as in the loop below (the same sums)
      if (!mbar_wait(&bars.full[s], ph)) return;
      const uint8_t* wg = stages + (size_t)s * p.stage_bytes + lane_off;
#pragma unroll
      for (int i = 0; i < (XREG ? kXRegBoxes : 1); i += 2) {
        if (i >= nbx) break;
        const bool two = i + 1 < nbx;
        if (post) {
          box_mma_xr<true>(acc0, wg + i * kBoxStep, row8, xr[i], rsa, rsb);
          if (two) box_mma_xr<true>(acc1, wg + (i + 1) * kBoxStep, row8, xr[i + 1], rsa, rsb);
        } else {
          box_mma_xr<false>(acc0, wg + i * kBoxStep, row8, xr[i], rsa, rsb);
          if (two) box_mma_xr<false>(acc1, wg + (i + 1) * kBoxStep, row8, xr[i + 1], rsa, rsb);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars.empty[s]);
      if (++s == S) {
        s = 0;
        ph ^= 1u;
      }
    }
    for (int kc = 0; kc < (XREG ? 0 : p.k_chunks); ++kc) {
      const int col0 = kc * p.kc;
      const int nbox = min(p.kc, p.k - col0) >> 6;
      if (!mbar_wait(&bars.full[s], ph)) return;
      const uint8_t* wg = stages + (size_t)s * p.stage_bytes + lane_off;
      const uint8_t* xc = xrow + (col0 + warp * 64 + 16 * q) * 2;
      int box = warp;
      // two independent boxes per iteration (separate accumulators)
      for (; box + kConsumerWarps < nbox;
           box += 2 * kConsumerWarps, wg += 2 * kBoxStep, xc += 4 * kBoxStep) {
        RowScale a0 = rsa, b0 = rsb, a1 = rsa, b1 = rsb;
        bool pst = post;
        if (GROUPED) {
          const int l0 = box * 64 + 16 * q, l1 = l0 + kBoxStep;
          const int g0 = (col0 + l0) / p.group_size, g1 = (col0 + l1) / p.group_size;
          a0 = row_scale(va ? __ldg(sa + g0) : 0.0f);
          b0 = row_scale(vb ? __ldg(sb + g0) : 0.0f);
          a1 = row_scale(va ? __ldg(sa + g1) : 0.0f);
          b1 = row_scale(vb ? __ldg(sb + g1) : 0.0f);
          pst = __any_sync(0xffffffffu, needs_post(a0) || needs_post(b0) ||
                                            needs_post(a1) || needs_post(b1));
        }
        if (pst) {
          box_mma<true>(acc0, wg, row8, xc, a0, b0);
          box_mma<true>(acc1, wg + kBoxStep, row8, xc + 2 * kBoxStep, a1, b1);
        } else {
          box_mma<false>(acc0, wg, row8, xc, a0, b0);
          box_mma<false>(acc1, wg + kBoxStep, row8, xc + 2 * kBoxStep, a1, b1);
        }
      }
      if (box < nbox) {
        RowScale a0 = rsa, b0 = rsb;
        bool pst = post;
        if (GROUPED) {
          const int g0 = (col0 + box * 64 + 16 * q) / p.group_size;
          a0 = row_scale(va ? __ldg(sa + g0) : 0.0f);
          b0 = row_scale(vb ? __ldg(sb + g0) : 0.0f);
          pst = __any_sync(0xffffffffu, needs_post(a0) || needs_post(b0));
        }
        if (pst) box_mma<true>(acc0, wg, row8, xc, a0, b0);
        else box_mma<false>(acc0, wg, row8, xc, a0, b0);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars.empty[s]);
      if (++s == S) {
        s = 0;
        ph ^= 1u;
      }
    }
    // hand the partial tile to the epilogue warp (double-buffered)
    const int b2 = blk & 1;
    if (blk >= 2 && !mbar_wait(&bars.epi_free[b2], ((blk >> 1) - 1) & 1)) return;
    float* mine = red + b2 * kRedFloats + warp * kTileRows * kMaxTokens;
    mine[g * kMaxTokens + 2 * q] = acc0[0] + acc1[0];
    mine[g * kMaxTokens + 2 * q + 1] = acc0[1] + acc1[1];
    mine[(g + 8) * kMaxTokens + 2 * q] = acc0[2] + acc1[2];
    mine[(g + 8) * kMaxTokens + 2 * q + 1] = acc0[3] + acc1[3];
    __syncwarp();
    if (lane == 0) mbar_arrive(&bars.epi_full[b2]);
  }
}

// ----------------------------------------------------------- generic path
// Any shape / alignment: one warp per (output, token), lane-strided K, the
// same factored-scale algebra and epilogues.  Used when the fast path's
// layout conditions do not hold.
__global__ void w8_generic_kernel(const Params p) {
  const int warp_global = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  const bool swiglu = p.epilogue == RXLA_B200_EPI_SWIGLU;
  pdl_wait();
  pdl_launch_dependents();
  const int64_t items = (int64_t)p.n * p.m;
  for (int64_t it = warp_global; it < items; it += nwarps) {
    const int col = (int)(it % p.n);
    const int tok = (int)(it / p.n);
    float res[2];
    for (int half = 0; half < (swiglu ? 2 : 1); ++half) {
      const int row = half ? p.n + col : col;
      const uint8_t* wr = p.w + (int64_t)row * p.k;
      float tot = 0.0f;
      for (int gi = 0; gi < p.groups; ++gi) {
        float part = 0.0f;
        const float sc = __ldg(p.scale + (int64_t)row * p.groups + gi);
        for (int c = gi * p.group_size + lane; c < (gi + 1) * p.group_size; c += 32) {
          float xv = p.x_f32 ? static_cast<const float*>(p.x)[(int64_t)tok * p.ldx + c]
                             : __bfloat162float(static_cast<const __nv_bfloat16*>(p.x)[(int64_t)tok * p.ldx + c]);
          xv = bf16_round(xv);
          part += xv * bf16_round(__fmul_rn((float)((int)wr[c] - 128), sc));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
        tot += part;
      }
      res[half] = tot;
    }
    if (lane == 0) {
      const int64_t o = (int64_t)tok * p.ldy + col;
      if (swiglu) {
        const float r = silu(bf16_round(res[0])) * bf16_round(res[1]);
        if (p.y_f32) static_cast<float*>(p.y)[o] = r;
        else static_cast<__nv_bfloat16*>(p.y)[o] = __float2bfloat16_rn(r);
      } else if (p.epilogue == RXLA_B200_EPI_RESIDUAL_ADD) {
        float* yy = static_cast<float*>(p.y);
        yy[o] = yy[o] + bf16_round(res[0]);
      } else if (p.y_f32) {
        static_cast<float*>(p.y)[o] = res[0];
      } else {
        static_cast<__nv_bfloat16*>(p.y)[o] = __float2bfloat16_rn(res[0]);
      }
    }
  }
}

// Shared-memory plan.  K is cut into k_chunks of kc columns so that one
// stage (16 rows × kc) stays within 64 KB (80 KB if that avoids a split);
// x (m tokens, bf16) is resident; the ring takes the rest, 2..8 stages.
static int32_t plan_skinny(Params& p, size_t& smem) {
  // largest stage and shared-memory budget of one CTA (bytes)
  constexpr size_t max_stage = 80 * 1024;
  constexpr size_t budget = 227 * 1024;
  int chunks = (int)(((int64_t)kTileRows * p.k + max_stage - 1) / max_stage);
  int kc = (int)((((int64_t)p.k + chunks - 1) / chunks + 63) / 64 * 64);
  p.kc = kc;
  p.k_chunks = (p.k + kc - 1) / kc;
  p.stage_bytes = kTileRows * kc;
  p.x_pitch = p.k * 2 + 16;
  const size_t fixed = kHeader + 2 * kRedFloats * 4 + (size_t)p.m * p.x_pitch;
  if (fixed + 2 * (size_t)p.stage_bytes > budget) return -1;
  p.stages = (int)std::min<size_t>(kMaxStages, (budget - fixed) / p.stage_bytes);
  smem = fixed + (size_t)p.stages * p.stage_bytes;
  return 0;
}

template <bool SWIGLU, bool GROUPED, int XMODE>
static cudaError_t launch_variant(const Params& p, int grid, size_t smem, cudaStream_t stream) {
  auto k = w8_skinny_kernel<SWIGLU, GROUPED, XMODE, false>;
  if (!GROUPED && p.k_chunks == 1 && p.k % (kConsumerWarps * 64) == 0 &&
      p.k <= kXRegBoxes * kConsumerWarps * 64)
    k = w8_skinny_kernel<SWIGLU, GROUPED, XMODE, !GROUPED>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(k, dim3(grid), dim3(kThreads), smem, stream, p);
}

template <bool SWIGLU, bool GROUPED>
static cudaError_t launch_x(const Params& p, int xmode, int grid, size_t smem, cudaStream_t s) {
  if (xmode == kXNorm) return launch_variant<SWIGLU, GROUPED, kXNorm>(p, grid, smem, s);
  if (xmode == kXF32) return launch_variant<SWIGLU, GROUPED, kXF32>(p, grid, smem, s);
  return launch_variant<SWIGLU, GROUPED, kXBf16>(p, grid, smem, s);
}

static cudaError_t launch_skinny(Params p, int xmode, int grid, cudaStream_t stream) {
  size_t smem = 0;
  if (plan_skinny(p, smem) != 0) return cudaErrorInvalidValue;
  const bool swiglu = p.epilogue == RXLA_B200_EPI_SWIGLU;
  const bool grouped = p.groups != 1;
  if (swiglu) {
    return grouped ? launch_x<true, true>(p, xmode, grid, smem, stream)
                   : launch_x<true, false>(p, xmode, grid, smem, stream);
  }
  return grouped ? launch_x<false, true>(p, xmode, grid, smem, stream)
                 : launch_x<false, false>(p, xmode, grid, smem, stream);
}

// Tokens per pass of the skinny kernel: up to 8, as long as the resident x
// still leaves room for a ring of at least two stages.
static int tokens_per_pass(Params p) {
  for (int m = kMaxTokens; m >= 1; --m) {
    p.m = m;
    size_t smem = 0;
    if (plan_skinny(p, smem) == 0) return m;
  }
  return 0;
}

static int grid_for(const Params& p) {
  int dev = 0;
  cudaGetDevice(&dev);
  const int rows_min = 4;  // avoid CTAs with almost no rows on tiny layers
  return (int)std::min<int64_t>(sm_count(dev), std::max<int64_t>(1, p.n / rows_min));
}

}  // namespace w8

// Fast-path eligibility and launch of one pass of at most `pass_m` tokens.
static int32_t w8_linear_pass(w8::Params p, bool fast, int xmode, cudaStream_t stream) {
  cudaError_t e;
  if (fast) {
    e = w8::launch_skinny(p, xmode, w8::grid_for(p), stream);
  } else {
    int dev = 0;
    cudaGetDevice(&dev);
    const int64_t warps = (int64_t)p.n * p.m;
    int blocks = (int)std::min<int64_t>((warps + 7) / 8, (int64_t)sm_count(dev) * 16);
    e = launch_pdl(w8::w8_generic_kernel, dim3(std::max(blocks, 1)), dim3(256), 0, stream, p);
  }
  if (e != cudaSuccess) return cuda_fail(e, "w8a16 linear launch");
  return RXLA_B200_OK;
}

int32_t w8_norm_linear(const NormLinearArgs& a, cudaStream_t stream) {
  RXLA_REQUIRE(a.k % 64 == 0 && (a.group == a.k || a.group % 64 == 0) &&
                   reinterpret_cast<uintptr_t>(a.w) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(a.h) % 16 == 0,
               "norm linear: shape is off the fused fast path");
  w8::Params p{};
  p.w = a.w;
  p.scale = a.scale;
  p.k = (int32_t)a.k;
  p.n = (int32_t)a.n;
  p.groups = (int32_t)(a.k / a.group);
  p.group_size = (int32_t)a.group;
  p.ldx = a.k;
  p.ldy = a.n;
  p.x_f32 = 1;
  p.y_f32 = a.y_dtype == RXLA_B200_F32;
  p.epilogue = a.epilogue;
  p.norm_w = a.norm_w;
  p.norm_eps = a.eps;
  p.arg_val = a.arg_val;
  p.arg_idx = a.arg_idx;
  p.arg_count = a.arg_count;
  const int per_pass = w8::tokens_per_pass(p);
  RXLA_REQUIRE(per_pass > 0, "norm linear: k too large for the resident x");
  const size_t ye = p.y_f32 ? 4 : 2;
  for (int64_t m0 = 0; m0 < a.m; m0 += per_pass) {
    p.m = (int32_t)std::min<int64_t>(per_pass, a.m - m0);
    p.x = a.h + m0 * a.k;
    p.y = a.y ? static_cast<uint8_t*>(a.y) + m0 * a.n * ye : nullptr;
    p.arg_out = a.arg_out ? a.arg_out + m0 : nullptr;
    p.arg_advance = a.arg_advance ? a.arg_advance + m0 : nullptr;
    p.next = m0 + per_pass >= a.m ? a.next : L2Prefetch{};
    cudaError_t e = w8::launch_skinny(p, w8::kXNorm, w8::grid_for(p), stream);
    if (e != cudaSuccess) return cuda_fail(e, "norm linear launch");
  }
  return RXLA_B200_OK;
}

static_assert(kArgmaxEpilogue == w8::kEpiArgmax, "argmax epilogue code");

}  // namespace rxla

namespace rxla {
int32_t w8_linear(const void* x, int32_t x_dtype, const uint8_t* weight, const float* scale,
                  int64_t group_size, int64_t m, int64_t n, int64_t k, void* y, int32_t y_dtype,
                  int32_t epilogue, cudaStream_t stream, const L2Prefetch* next,
                  const P2pView* tp, void* ws, size_t ws_bytes) {
  RXLA_REQUIRE(m >= 0 && n >= 0 && k > 0, "w8a16_linear: m, n must be >= 0 and k > 0");
  RXLA_REQUIRE(group_size > 0 && k % group_size == 0,
               "w8a16_linear: group_size must be positive and divide k (layers.rs:266-275)");
  RXLA_REQUIRE(x_dtype == RXLA_B200_BF16 || x_dtype == RXLA_B200_F32,
               "w8a16_linear: x must be BF16 or F32");
  RXLA_REQUIRE(y_dtype == RXLA_B200_BF16 || y_dtype == RXLA_B200_F32,
               "w8a16_linear: y must be BF16 or F32");
  RXLA_REQUIRE(epilogue >= RXLA_B200_EPI_STORE && epilogue <= RXLA_B200_EPI_SWIGLU,
               "w8a16_linear: unknown epilogue");
  RXLA_REQUIRE(epilogue != RXLA_B200_EPI_RESIDUAL_ADD || y_dtype == RXLA_B200_F32,
               "w8a16_linear: the residual epilogue adds into an F32 y");
  RXLA_REQUIRE(k <= INT32_MAX && n <= INT32_MAX && m <= INT32_MAX, "w8a16_linear: size too large");
  if (m == 0 || n == 0) return RXLA_B200_OK;
  RXLA_REQUIRE(x && weight && scale && y, "w8a16_linear: null pointer");
  w8::Params p{};
  p.w = weight;
  p.scale = scale;
  p.k = (int32_t)k;
  p.n = (int32_t)n;
  p.groups = (int32_t)(k / group_size);
  p.group_size = (int32_t)group_size;
  p.ldx = k;
  p.ldy = n;
  p.x_f32 = x_dtype == RXLA_B200_F32;
  p.y_f32 = y_dtype == RXLA_B200_F32;
  p.epilogue = epilogue;
  const size_t xe = p.x_f32 ? 4 : 2, ye = p.y_f32 ? 4 : 2;
  const bool aligned = (reinterpret_cast<uintptr_t>(weight) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(x) % 16 == 0);
  const int per_pass = w8::tokens_per_pass(p);
  const bool fast = aligned && (k % 64 == 0) && (p.groups == 1 || group_size % 64 == 0) &&
                    per_pass > 0;
  // more tokens than one skinny pass: the tcgen05 GEMM reads the weights once
  if (m > w8::kMaxTokens && x_dtype == RXLA_B200_BF16 && aligned && k % 64 == 0 &&
      group_size % 64 == 0) {
    GemmArgs g{};
    g.x = x;
    g.ldx = k;
    g.w = weight;
    g.scale = scale;
    g.group = group_size;
    g.m = m;
    g.n = n;
    g.k = k;
    g.y = y;
    g.ldy = n;
    g.y_dtype = y_dtype;
    g.epilogue = epilogue;
    g.splits = 1;
    if (ws) {
      // split-K over the caller's workspace, the depth the decoder's GEMMs use
      const bool swiglu = epilogue == RXLA_B200_EPI_SWIGLU;
      const int sp = w8_gemm_splits(m, n, k, group_size, swiglu);
      if (sp > 1) {
        RXLA_REQUIRE(reinterpret_cast<uintptr_t>(ws) % 16 == 0 &&
                         ws_bytes >= w8_gemm_workspace_bytes(m, swiglu ? 2 * n : n, sp),
                     "w8a16_linear: workspace smaller than rxla_b200_w8a16_linear_workspace_size "
                     "or not 16-byte aligned");
        g.splits = sp;
        g.ws = ws;
        g.ws_bytes = ws_bytes;
      }
    }
    return w8_gemm(g, stream);
  }
  const int xmode = p.x_f32 ? w8::kXF32 : w8::kXBf16;
  const int64_t step = fast ? per_pass : 32;
  if (tp && tp->world > 1) {
    // the row-parallel all-reduce runs in the epilogue of one fast pass; the
    // flags are per CTA of the grid, the same grid on every rank
    RXLA_REQUIRE(fast && m <= per_pass && epilogue == RXLA_B200_EPI_RESIDUAL_ADD &&
                     tp->world <= kP2pMaxRanks && tp->rank >= 0 && tp->rank < tp->world &&
                     m * n <= tp->cap && w8::grid_for(p) <= tp->max_ctas,
                 "w8a16_linear: the fused all-reduce needs one fast pass within the peer buffers");
    p.tp = *tp;
  }
  for (int64_t m0 = 0; m0 < m; m0 += step) {
    p.m = (int32_t)std::min<int64_t>(step, m - m0);
    p.x = static_cast<const uint8_t*>(x) + m0 * k * xe;
    p.y = static_cast<uint8_t*>(y) + m0 * n * ye;
    p.next = (next && m0 + step >= m) ? *next : L2Prefetch{};
    int32_t st = w8_linear_pass(p, fast, xmode, stream);
    if (st != RXLA_B200_OK) return st;
  }
  return RXLA_B200_OK;
}
}  // namespace rxla

extern "C" int32_t rxla_b200_w8a16_norm_linear(const float* h, const float* norm_weight,
                                               float eps, const uint8_t* weight,
                                               const float* scale, int64_t group_size, int64_t m,
                                               int64_t n, int64_t k, void* y, int32_t y_dtype,
                                               int32_t epilogue, void* stream) {
  using namespace rxla;
  RXLA_REQUIRE(m >= 0 && n >= 0 && k > 0 && k <= INT32_MAX && n <= INT32_MAX,
               "w8a16_norm_linear: m, n must be >= 0 and k > 0");
  RXLA_REQUIRE(eps > 0.0f && eps == eps && eps < INFINITY,
               "w8a16_norm_linear: epsilon must be finite and positive (ops.rs:930)");
  RXLA_REQUIRE(group_size > 0 && k % group_size == 0,
               "w8a16_norm_linear: group_size must be positive and divide k (layers.rs:266-275)");
  RXLA_REQUIRE(y_dtype == RXLA_B200_BF16 || y_dtype == RXLA_B200_F32,
               "w8a16_norm_linear: y must be BF16 or F32");
  RXLA_REQUIRE(epilogue >= RXLA_B200_EPI_STORE && epilogue <= RXLA_B200_EPI_SWIGLU,
               "w8a16_norm_linear: unknown epilogue");
  RXLA_REQUIRE(epilogue != RXLA_B200_EPI_RESIDUAL_ADD || y_dtype == RXLA_B200_F32,
               "w8a16_norm_linear: the residual epilogue adds into an F32 y");
  if (m == 0 || n == 0) return RXLA_B200_OK;
  RXLA_REQUIRE(h && norm_weight && weight && scale && y, "w8a16_norm_linear: null pointer");
  // every CTA reads all of h while the epilogue writes y: they must not overlap
  const uintptr_t h0 = reinterpret_cast<uintptr_t>(h), h1 = h0 + (uintptr_t)(m * k * 4);
  const uintptr_t y0 = reinterpret_cast<uintptr_t>(y);
  const uintptr_t y1 = y0 + (uintptr_t)(m * n * (y_dtype == RXLA_B200_F32 ? 4 : 2));
  RXLA_REQUIRE(y1 <= h0 || h1 <= y0, "w8a16_norm_linear: y must not overlap h");
  NormLinearArgs a{};
  a.h = h;
  a.norm_w = norm_weight;
  a.eps = eps;
  a.w = weight;
  a.scale = scale;
  a.group = group_size;
  a.m = m;
  a.n = n;
  a.k = k;
  a.y = y;
  a.y_dtype = y_dtype;
  a.epilogue = epilogue;
  return w8_norm_linear(a, static_cast<cudaStream_t>(stream));
}

extern "C" int32_t rxla_b200_w8a16_linear(const void* x, int32_t x_dtype, const uint8_t* weight,
                                          const float* scale, int64_t group_size, int64_t m,
                                          int64_t n, int64_t k, void* y, int32_t y_dtype,
                                          int32_t epilogue, void* stream) {
  return rxla::w8_linear(x, x_dtype, weight, scale, group_size, m, n, k, y, y_dtype, epilogue,
                         static_cast<cudaStream_t>(stream), nullptr);
}

extern "C" int32_t rxla_b200_w8a16_linear_workspace_size(int64_t m, int64_t n, int64_t k,
                                                         int64_t group_size, int32_t epilogue,
                                                         size_t* bytes) {
  using namespace rxla;
  RXLA_REQUIRE(bytes && m >= 0 && n >= 0 && k > 0 && group_size > 0 && k % group_size == 0,
               "w8a16_linear_workspace_size: bad arguments");
  RXLA_REQUIRE(epilogue >= RXLA_B200_EPI_STORE && epilogue <= RXLA_B200_EPI_SWIGLU,
               "w8a16_linear_workspace_size: unknown epilogue");
  *bytes = 0;
  // only the tcgen05 GEMM (more tokens than one skinny pass) splits K
  if (m <= w8::kMaxTokens || n == 0 || k % 64 != 0 || group_size % 64 != 0) return RXLA_B200_OK;
  const bool swiglu = epilogue == RXLA_B200_EPI_SWIGLU;
  const int sp = w8_gemm_splits(m, n, k, group_size, swiglu);
  *bytes = w8_gemm_workspace_bytes(m, swiglu ? 2 * n : n, sp);
  return RXLA_B200_OK;
}

extern "C" int32_t rxla_b200_w8a16_linear_ws(const void* x, int32_t x_dtype,
                                             const uint8_t* weight, const float* scale,
                                             int64_t group_size, int64_t m, int64_t n, int64_t k,
                                             void* y, int32_t y_dtype, int32_t epilogue,
                                             void* workspace, size_t workspace_bytes,
                                             void* stream) {
  RXLA_REQUIRE(workspace || workspace_bytes == 0, "w8a16_linear_ws: null workspace");
  return rxla::w8_linear(x, x_dtype, weight, scale, group_size, m, n, k, y, y_dtype, epilogue,
                         static_cast<cudaStream_t>(stream), nullptr, nullptr, workspace,
                         workspace_bytes);
}
