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
//    over K.  Dequantization runs in registers with packed f32x2 arithmetic:
//    PRMT makes 2^23 + b, add.f32x2 subtracts 2^23 + 128 (exact q),
//    mul.f32x2 applies the row's scale (the reference's f32 product) and
//    cvt.rn.bf16x2 rounds to bf16.  For SwiGLU, rows 0-7 of the A tile are
//    gate rows and rows 8-15 the matching up rows.  The K columns are permuted
//    consistently for A and B: a lane reads 16 contiguous weight bytes and the
//    16 matching x values, which covers four k-steps;
//  * an epilogue warp sums the 16 warps' partial tiles in a fixed order
//    (deterministic), scales, rounds to bf16 and stores / adds to the f32
//    residual / gates with SiLU, double-buffered so the consumers never wait
//    for it.
#include <algorithm>

#include <cuda_fp16.h>

#include "common.cuh"

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
constexpr int kHeader = 1024;       // barriers + per-token exponents

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
  // shared-memory plan (set by the host)
  int32_t kc;           // K columns per stage (multiple of 64)
  int32_t k_chunks;     // ceil(k / kc)
  int32_t stages;       // ring depth
  int32_t x_pitch;      // bytes of one resident token row of x
  int32_t stage_bytes;  // 16 rows × kc
};

struct Bars {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t x_full;
  uint64_t grp[2];
  uint64_t epi_full[2];
  uint64_t epi_free[2];
};
static_assert(sizeof(Bars) <= kHeader, "header");

__device__ __forceinline__ uint64_t f32x2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}

// Four u8 weights of one row (value b, q = b - 128) with the row's scale pair
// (s, s) -> two bf16x2 registers of bf16(f32(q)·s): lo = (w0, w1), hi = (w2, w3).
__device__ __forceinline__ void deq4(uint32_t w, uint64_t s2, uint32_t& lo, uint32_t& hi) {
  const uint64_t bias = 0xCB000080CB000080ull;  // (-(2^23 + 128), -(2^23 + 128))
  uint64_t a = f32x2(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u)),
                     __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7541u)));
  uint64_t c = f32x2(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7542u)),
                     __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7543u)));
  asm("add.rn.f32x2 %0, %0, %1;" : "+l"(a) : "l"(bias));
  asm("add.rn.f32x2 %0, %0, %1;" : "+l"(c) : "l"(bias));
  asm("mul.rn.f32x2 %0, %0, %1;" : "+l"(a) : "l"(s2));
  asm("mul.rn.f32x2 %0, %0, %1;" : "+l"(c) : "l"(s2));
  float a0, a1, c0, c1;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a0), "=f"(a1) : "l"(a));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(c0), "=f"(c1) : "l"(c));
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(lo) : "f"(a1), "f"(a0));
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(hi) : "f"(c1), "f"(c0));
}

// Bounded barrier among the 16 consumer warps (one arrival per warp).
__device__ __forceinline__ bool consumer_sync(uint64_t* bar, uint32_t parity) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
  return mbar_wait(bar, parity);
}

__global__ void __launch_bounds__(kThreads, 1) w8_skinny_kernel(const Params p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  Bars& bars = *reinterpret_cast<Bars*>(smem_raw);
  float* red = reinterpret_cast<float*>(smem_raw + kHeader);  // [2][warp][16 rows][8 tokens]
  uint8_t* xs = smem_raw + kHeader + 2 * kRedFloats * 4;
  uint8_t* stages = xs + (size_t)p.m * p.x_pitch;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const bool swiglu = p.epilogue == RXLA_B200_EPI_SWIGLU;
  const int xe = p.x_f32 ? 4 : 2;
  const int out_rows = swiglu ? kTileRows / 2 : kTileRows;

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
    mbar_init(&bars.x_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars.grp[i], kConsumerWarps);
      mbar_init(&bars.epi_full[i], kConsumerWarps);
      mbar_init(&bars.epi_free[i], 1);
    }
    fence_mbarrier_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------ producer
    const uint64_t policy = l2_evict_first_policy();
    auto issue = [&](int it, int s) {
      const int blk = it / p.k_chunks, kc = it % p.k_chunks;
      const int r0 = r_begin + blk * out_rows;
      const int nr = min(out_rows, r_end - r0);
      const int col0 = kc * p.kc;
      const int cols = min(p.kc, p.k - col0);
      const uint32_t tx = (uint32_t)cols * (uint32_t)nr * (swiglu ? 2u : 1u);
      if (lane == 0) mbar_arrive_expect_tx(&bars.full[s], tx);
      __syncwarp();
      uint8_t* dst = stages + (size_t)s * p.stage_bytes;
      if (cols == p.k) {
        // whole rows: the block is one contiguous range (two for SwiGLU)
        if (lane == 0)
          bulk_g2s(dst, p.w + (int64_t)r0 * p.k, (uint32_t)(nr * p.k), &bars.full[s], policy);
        if (swiglu && lane == 1)
          bulk_g2s(dst + (kTileRows / 2) * p.kc, p.w + (int64_t)(p.n + r0) * p.k,
                   (uint32_t)(nr * p.k), &bars.full[s], policy);
      } else {
        const int i = swiglu ? (lane & 7) : lane;
        const bool up = swiglu && lane >= 8;
        if (lane < kTileRows && i < nr) {
          const int64_t row = up ? (int64_t)p.n + r0 + i : (int64_t)r0 + i;
          bulk_g2s(dst + (size_t)lane * p.kc, p.w + row * p.k + col0, (uint32_t)cols,
                   &bars.full[s], policy);
        }
      }
    };
    // weights do not depend on the previous kernel: fill the ring first
    const int pre = min(S, total);
    for (int it = 0; it < pre; ++it) issue(it, it);
    pdl_wait();  // x is the previous kernel's output
    if (lane == 0) mbar_arrive_expect_tx(&bars.x_full, (uint32_t)(p.m * p.k * xe));
    __syncwarp();
    if (lane < p.m)
      bulk_g2s_nohint(xs + lane * p.x_pitch,
                      static_cast<const uint8_t*>(p.x) + (int64_t)lane * p.ldx * xe,
                      (uint32_t)(p.k * xe), &bars.x_full);
    for (int it = pre; it < total; ++it) {
      const int s = it % S;
      if (!mbar_wait(&bars.empty[s], ((it / S) - 1) & 1)) return;
      issue(it, s);
    }
    return;
  }

  const int g = lane >> 2;  // mma group id: A rows g, g+8; B column (token) g
  const int q = lane & 3;   // k-quad
  const bool per_channel = p.groups == 1;

  if (warp == kEpilogueWarp) {
    // ------------------------------------------------------------ epilogue
    pdl_wait();  // y (or the residual it adds into) may be used by the previous kernel
    for (int blk = 0; blk < n_blocks; ++blk) {
      const int b2 = blk & 1;
      if (!mbar_wait(&bars.epi_full[b2], (blk >> 1) & 1)) return;
      const int r0 = r_begin + blk * out_rows;
      const int nr = min(out_rows, r_end - r0);
      const float* rb = red + b2 * kRedFloats;
      for (int idx = lane; idx < out_rows * kMaxTokens; idx += 32) {
        const int row = idx % out_rows, tok = idx / out_rows;
        if (row >= nr || tok >= p.m) continue;
        float v = 0.0f, u = 0.0f;
#pragma unroll
        for (int w2 = 0; w2 < kConsumerWarps; ++w2) {
          v += rb[(w2 * kTileRows + row) * kMaxTokens + tok];
          if (swiglu) u += rb[(w2 * kTileRows + row + 8) * kMaxTokens + tok];
        }
        const int out_col = r0 + row;
        const int64_t o = (int64_t)tok * p.ldy + out_col;
        if (swiglu) {
          const float r = silu(bf16_round(v)) * bf16_round(u);
          if (p.y_f32) static_cast<float*>(p.y)[o] = r;
          else static_cast<__nv_bfloat16*>(p.y)[o] = __float2bfloat16_rn(r);
        } else if (p.epilogue == RXLA_B200_EPI_RESIDUAL_ADD) {
          float* yy = static_cast<float*>(p.y);
          yy[o] = yy[o] + bf16_round(v);
        } else if (p.y_f32) {
          static_cast<float*>(p.y)[o] = v;
        } else {
          static_cast<__nv_bfloat16*>(p.y)[o] = __float2bfloat16_rn(v);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars.epi_free[b2]);
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  if (!mbar_wait(&bars.x_full, 0)) return;
  const bool has_tok = g < p.m;
  const uint8_t* xrow = xs + g * p.x_pitch;

  int it = 0;
  for (int blk = 0; blk < n_blocks; ++blk) {
    const int r0 = r_begin + blk * out_rows;
    const int nr = min(out_rows, r_end - r0);
    // weight rows of this lane's A fragment: tile rows g and g + 8
    int ra, rb;
    bool va, vb;
    if (swiglu) {
      va = vb = g < nr;
      ra = r0 + g;
      rb = p.n + r0 + g;
    } else {
      va = g < nr;
      vb = g + 8 < nr;
      ra = r0 + g;
      rb = r0 + g + 8;
    }
    const float* sa = p.scale + (int64_t)ra * p.groups;
    const float* sb = p.scale + (int64_t)rb * p.groups;
    uint64_t s2a = 0, s2b = 0;
    if (per_channel) {
      const float x0 = va ? __ldg(sa) : 0.0f, x1 = vb ? __ldg(sb) : 0.0f;
      s2a = f32x2(x0, x0);
      s2b = f32x2(x1, x1);
    }
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int kc = 0; kc < p.k_chunks; ++kc, ++it) {
      const int s = it % S;
      const int col0 = kc * p.kc;
      const int nbox = min(p.kc, p.k - col0) >> 6;
      if (!mbar_wait(&bars.full[s], (it / S) & 1)) return;
      const uint8_t* stage = stages + (size_t)s * p.stage_bytes;
#pragma unroll 2
      for (int box = warp; box < nbox; box += kConsumerWarps) {
        const int lcol = box * 64 + 16 * q;  // stage-local column of this lane's 16 bytes
        const int gcol = col0 + lcol;        // global K column
        if (!per_channel) {
          const int grp = gcol / p.group_size;
          const float x0 = va ? __ldg(sa + grp) : 0.0f, x1 = vb ? __ldg(sb + grp) : 0.0f;
          s2a = f32x2(x0, x0);
          s2b = f32x2(x1, x1);
        }
        uint32_t bx[8];
        if (has_tok) {
          if (p.x_f32) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float4 v = *reinterpret_cast<const float4*>(xrow + (gcol + 4 * j) * 4);
              bx[2 * j] = pack_bf16x2(v.x, v.y);
              bx[2 * j + 1] = pack_bf16x2(v.z, v.w);
            }
          } else {
            const uint4 v0 = *reinterpret_cast<const uint4*>(xrow + gcol * 2);
            const uint4 v1 = *reinterpret_cast<const uint4*>(xrow + gcol * 2 + 16);
            bx[0] = v0.x; bx[1] = v0.y; bx[2] = v0.z; bx[3] = v0.w;
            bx[4] = v1.x; bx[5] = v1.y; bx[6] = v1.z; bx[7] = v1.w;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) bx[j] = 0u;
        }
        const uint4 lo = *reinterpret_cast<const uint4*>(stage + g * p.kc + lcol);
        const uint4 hi = *reinterpret_cast<const uint4*>(stage + (g + 8) * p.kc + lcol);
        const uint32_t wl[4] = {lo.x, lo.y, lo.z, lo.w};
        const uint32_t wh[4] = {hi.x, hi.y, hi.z, hi.w};
#pragma unroll
        for (int st = 0; st < 4; ++st) {
          uint32_t a[4];
          deq4(wl[st], s2a, a[0], a[2]);  // row g: k-low pair, k-high pair
          deq4(wh[st], s2b, a[1], a[3]);  // row g+8
          mma_bf16_16816(acc, a, bx[2 * st], bx[2 * st + 1]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars.empty[s]);
    }
    // hand the partial tile to the epilogue warp (double-buffered)
    const int b2 = blk & 1;
    if (blk >= 2 && !mbar_wait(&bars.epi_free[b2], ((blk >> 1) - 1) & 1)) return;
    float* mine = red + b2 * kRedFloats + warp * kTileRows * kMaxTokens;
    mine[g * kMaxTokens + 2 * q] = acc[0];
    mine[g * kMaxTokens + 2 * q + 1] = acc[1];
    mine[(g + 8) * kMaxTokens + 2 * q] = acc[2];
    mine[(g + 8) * kMaxTokens + 2 * q + 1] = acc[3];
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
  pdl_launch_dependents();
  pdl_wait();
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
// x (m tokens) is resident; the ring takes the rest, 2..8 stages.
static int32_t plan_skinny(Params& p, size_t& smem) {
  const int xe = p.x_f32 ? 4 : 2;
  int chunks = (int)(((int64_t)kTileRows * p.k + 80 * 1024 - 1) / (80 * 1024));
  if (chunks > 1) chunks = (int)(((int64_t)kTileRows * p.k + 64 * 1024 - 1) / (64 * 1024));
  int kc = (int)((((int64_t)p.k + chunks - 1) / chunks + 63) / 64 * 64);
  p.kc = kc;
  p.k_chunks = (p.k + kc - 1) / kc;
  p.stage_bytes = kTileRows * kc;
  p.x_pitch = p.k * xe + 16;
  const size_t fixed = kHeader + 2 * kRedFloats * 4 + (size_t)p.m * p.x_pitch;
  const size_t budget = 227 * 1024;
  if (fixed + 2 * (size_t)p.stage_bytes > budget) return -1;
  p.stages = (int)std::min<size_t>(kMaxStages, (budget - fixed) / p.stage_bytes);
  smem = fixed + (size_t)p.stages * p.stage_bytes;
  return 0;
}

static cudaError_t launch_skinny(Params p, int grid, cudaStream_t stream) {
  size_t smem = 0;
  if (plan_skinny(p, smem) != 0) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(w8_skinny_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(w8_skinny_kernel, dim3(grid), dim3(kThreads), smem, stream, p);
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

}  // namespace w8

// Fast-path eligibility and launch of one pass of at most `pass_m` tokens.
static int32_t w8_linear_pass(w8::Params p, bool fast, cudaStream_t stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  const int sms = sm_count(dev);
  cudaError_t e;
  if (fast) {
    const int rows_min = 4;  // avoid CTAs with almost no rows on tiny layers
    int grid = (int)std::min<int64_t>(sms, std::max<int64_t>(1, p.n / rows_min));
    e = w8::launch_skinny(p, grid, stream);
  } else {
    const int64_t warps = (int64_t)p.n * p.m;
    int blocks = (int)std::min<int64_t>((warps + 7) / 8, (int64_t)sms * 16);
    e = launch_pdl(w8::w8_generic_kernel, dim3(std::max(blocks, 1)), dim3(256), 0, stream, p);
  }
  if (e != cudaSuccess) return cuda_fail(e, "w8a16 linear launch");
  return RXLA_B200_OK;
}

}  // namespace rxla

extern "C" int32_t rxla_b200_w8a16_linear(const void* x, int32_t x_dtype, const uint8_t* weight,
                                          const float* scale, int64_t group_size, int64_t m,
                                          int64_t n, int64_t k, void* y, int32_t y_dtype,
                                          int32_t epilogue, void* stream) {
  using namespace rxla;
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
  const int64_t step = fast ? per_pass : 32;
  for (int64_t m0 = 0; m0 < m; m0 += step) {
    p.m = (int32_t)std::min<int64_t>(step, m - m0);
    p.x = static_cast<const uint8_t*>(x) + m0 * k * xe;
    p.y = static_cast<uint8_t*>(y) + m0 * n * ye;
    int32_t st = w8_linear_pass(p, fast, static_cast<cudaStream_t>(stream));
    if (st != RXLA_B200_OK) return st;
  }
  return RXLA_B200_OK;
}
