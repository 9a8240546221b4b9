// w8_gemm.cu — W8A16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM)
// for more than a handful of tokens: prefill, and decode at batch > 8.
//
// Reference semantics (crates/rxla-nn/src/layers.rs:257-298, bf16 compute):
// y[m, n] = bf16( Σ_k bf16(x[m, k]) · bf16(f32(q[n, k] - 128) · s[n, k / G]) ),
// fp32 accumulation; the same epilogues as the skinny kernel (bf16 / f32
// store, f32 residual add of the bf16 dot, SwiGLU of a fused [gate; up]).
//
// Tile: 128 tokens (MMA M) × 128 weight rows (MMA N), K staged 64 at a time.
//  * warp 0 (producer): TMA loads of the weight tile [128 × 64] u8 (two
//    64-row boxes; for SwiGLU the gate rows and the matching up rows), which
//    do not depend on the previous kernel; x tiles [128 × 64] bf16 use the
//    128-byte swizzle, the UMMA K-major SW128 layout;
//  * warp 2 (producer): the x tiles, in a ring of their own (they are L2
//    hits with long latency, so it runs deeper than the weight ring);
//  * warps 3-10 (dequant, then epilogue): two threads per weight row turn the
//    stage's u8 tile into bf16 with the reference's rounding (packed denormal
//    FMA, as in the skinny kernel), store it in the SW128 K-major layout the
//    MMA reads, fence the generic->async proxy and arrive;
//  * warp 1 (MMA): allocates 128 TMEM columns (fp32 accumulator 128 × 128),
//    one elected thread issues four tcgen05.mma (K = 16 each) per stage and
//    commits to the stage's "empty" barrier, finally to "acc_full";
//  * the epilogue warps read the accumulator with tcgen05.ld (warp w reads
//    TMEM lanes 32·(w % 4) …), apply the epilogue and store.
// Split-K (grid.z > 1, decoder shapes with few tiles): fp32 partials go to a
// workspace and the last CTA of a tile (arrival counter) sums them in split
// order and applies the epilogue.
#include <cudaTypedefs.h>

#include "internal.cuh"

namespace rxla {
namespace gemm {

using w8::deq4;
using w8::needs_post;
using w8::row_scale;
using w8::RowScale;

constexpr int kBM = 128, kBN = 256, kBK = 64;
constexpr int kHalfN = kBN / 2;         // rows per weight TMA box; SwiGLU outputs per tile
constexpr int kWStages = 4;             // u8 weight tiles (TMA), 16 KB each
constexpr int kXStages = 6;             // x tiles (TMA): deep, they are L2 hits with long latency
constexpr int kBStages = 2;             // dequantized bf16 weight tiles, 32 KB each
constexpr int kXTile = kBM * kBK * 2;   // 16 KB bf16, SW128
constexpr int kBTile = kBN * kBK * 2;   // 32 KB bf16, SW128
constexpr int kWTile = kBN * kBK;       // 16 KB u8
constexpr int kDeqWarps = 16;           // two threads per weight row
constexpr int kThreads = (3 + kDeqWarps) * 32;
constexpr int kTmemCols = kBN;          // fp32 accumulator 128 lanes × 256 columns
constexpr int kChunk = 16;              // accumulator columns per tcgen05.ld in the epilogue

struct Params {
  const float* scale;
  int32_t groups, group_size;
  int32_t m, n, k;            // tokens, output columns (SwiGLU: outputs), K
  int32_t n_rows;             // weight rows (2n for SwiGLU)
  void* y;
  int64_t ldy;
  int32_t y_f32, epilogue;    // RXLA_B200_EPI_*
  int32_t k_per_split;        // multiple of kBK
  float* ws;                  // [splits][m][n_rows] fp32 partials (splits > 1)
  uint32_t* counters;         // [tiles], zero between launches
};

struct Smem {
  uint64_t w_full[kWStages];   // u8 weight tile landed (TMA)
  uint64_t w_empty[kWStages];  // dequant warps are done with it
  uint64_t x_full[kXStages];   // x tile landed (TMA)
  uint64_t b_full[kBStages];   // bf16 weight tile written (dequant warps)
  // MMAs of k-block it are complete (one commit per k-block, slot it % kXStages):
  // frees x slot it % kXStages and bf16 slot it % kBStages
  uint64_t mma_done[kXStages];
  uint64_t acc_full;
  uint32_t tmem_base;
  uint32_t last;
};
static_assert(sizeof(Smem) <= 1024, "barrier block");
static_assert(kXStages >= kBStages, "one commit slot per x slot covers the bf16 ring");

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// UMMA shared-memory descriptor of a K-major SW128 tile whose rows are 128
// bytes and whose 8-row groups are 1024 bytes apart (start 1024-aligned).
__device__ __forceinline__ uint64_t sw128_desc(const void* tile) {
  const uint64_t addr = smem_u32(tile);
  uint64_t d = (addr >> 4) & 0x3FFFull;  // start address
  d |= 1ull << 16;                        // leading byte offset (unused for SW128 K-major)
  d |= (uint64_t)(1024 >> 4) << 32;       // stride byte offset: 8-row group pitch
  d |= 1ull << 46;                        // descriptor version (sm100)
  d |= 2ull << 61;                        // SWIZZLE_128B
  return d;
}

// Instruction descriptor: kind::f16, bf16 A and B (K-major), f32 accumulate,
// M = 128, N = 128.
constexpr uint32_t kIdesc = (1u << 4)             // D format f32
                            | (1u << 7)           // A bf16
                            | (1u << 10)          // B bf16
                            | ((kBN >> 3) << 17)  // N / 8
                            | ((kBM >> 4) << 24); // M / 16

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                         bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate ? 1 : 0)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t addr, float (&v)[kChunk]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(addr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Reference dequantization of 8 bytes (k order) into 4 bf16x2 words.
__device__ __forceinline__ void deq8(uint32_t w0, uint32_t w1, const RowScale& r, bool post,
                                     uint32_t (&o)[4]) {
  if (post) {
    deq4<true>(w0, r, o[0], o[1]);
    deq4<true>(w1, r, o[2], o[3]);
  } else {
    deq4<false>(w0, r, o[0], o[1]);
    deq4<false>(w1, r, o[2], o[3]);
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    w8_gemm_kernel(const __grid_constant__ CUtensorMap xmap,
                   const __grid_constant__ CUtensorMap wmap, const Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t* base = smem_raw + pad;
  Smem& sm = *reinterpret_cast<Smem*>(base);
  uint8_t* x_ring = base + 1024;                            // [kXStages][x tile]
  uint8_t* b_ring = x_ring + (size_t)kXStages * kXTile;     // [kBStages][bf16 tile]
  uint8_t* w_ring = b_ring + (size_t)kBStages * kBTile;     // [kWStages][u8 tile]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kBM;
  const int tile_n = blockIdx.y;
  const int split = blockIdx.z;
  const bool swiglu = p.epilogue == RXLA_B200_EPI_SWIGLU;
  // weight rows of this tile: [wr0, wr0 + 128) and [wr1, wr1 + 128); for
  // SwiGLU the gate rows of outputs out0 .. out0 + 127 and the matching up rows
  const int out0 = tile_n * (swiglu ? kHalfN : kBN);  // first output column
  const int wr0 = out0;
  const int wr1 = swiglu ? p.n + out0 : out0 + kHalfN;
  const int k_begin = split * p.k_per_split;
  const int k_end = min(p.k, k_begin + p.k_per_split);
  const int n_k = (k_end - k_begin) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kWStages; ++s) {
      mbar_init(&sm.w_full[s], 1);
      mbar_init(&sm.w_empty[s], kDeqWarps);
    }
    for (int s = 0; s < kXStages; ++s) {
      mbar_init(&sm.x_full[s], 1);
      mbar_init(&sm.mma_done[s], 1);
    }
    for (int s = 0; s < kBStages; ++s) mbar_init(&sm.b_full[s], kDeqWarps);
    mbar_init(&sm.acc_full, 1);
    fence_mbarrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&sm.tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0) {
    // ------------------------------------------------- weight producer (TMA)
    // weights do not depend on the previous kernel: no wait before streaming
    if (lane == 0) {
      for (int it = 0; it < n_k; ++it) {
        const int s = it % kWStages;
        if (it >= kWStages && !mbar_wait(&sm.w_empty[s], ((it / kWStages) - 1) & 1)) break;
        uint8_t* dst = w_ring + (size_t)s * kWTile;
        const int k0 = k_begin + it * kBK;
        mbar_arrive_expect_tx(&sm.w_full[s], (uint32_t)kWTile);
        tma_load_2d(dst, &wmap, k0, wr0, &sm.w_full[s]);
        tma_load_2d(dst + kHalfN * kBK, &wmap, k0, wr1, &sm.w_full[s]);
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------------ x producer (TMA)
    if (lane == 0) {
      pdl_wait();  // x (and the residual) come from the previous kernel
      for (int it = 0; it < n_k; ++it) {
        const int s = it % kXStages;
        // slot s was last read by the MMAs of k-block it - kXStages
        if (it >= kXStages && !mbar_wait(&sm.mma_done[s], ((it / kXStages) - 1) & 1)) break;
        mbar_arrive_expect_tx(&sm.x_full[s], (uint32_t)kXTile);
        tma_load_2d(x_ring + (size_t)s * kXTile, &xmap, k_begin + it * kBK, m0, &sm.x_full[s]);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      for (int it = 0; it < n_k; ++it) {
        const int xs = it % kXStages, bs = it % kBStages;
        if (!mbar_wait(&sm.x_full[xs], (it / kXStages) & 1) ||
            !mbar_wait(&sm.b_full[bs], (it / kBStages) & 1))
          break;
        tc_fence_after();
        const uint64_t ad = sw128_desc(x_ring + (size_t)xs * kXTile);
        const uint64_t bd = sw128_desc(b_ring + (size_t)bs * kBTile);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)  // +32 bytes per K = 16 step
          mma_bf16(tmem, ad + 2 * kk, bd + 2 * kk, it > 0 || kk > 0);
        mma_commit(&sm.mma_done[xs]);
      }
      mma_commit(&sm.acc_full);
    }
  } else {
    // ------------------------------------------- dequant, then epilogue
    // thread d (0 .. 511): weight row d / 2 of the tile, bytes 32·(d % 2) ..
    const int d = threadIdx.x - 96;
    const int t = d >> 1, half = d & 1;
    const int wrow = t < kHalfN ? wr0 + t : wr1 + (t - kHalfN);
    const bool wvalid =
        wrow < p.n_rows && (swiglu ? (t < kHalfN ? out0 + t : out0 + t - kHalfN) < p.n : true);
    const float* srow = p.scale + (int64_t)(wvalid ? wrow : 0) * p.groups;
    RowScale rs = row_scale(wvalid ? __ldg(srow + k_begin / p.group_size) : 0.0f);
    int cur_group = k_begin / p.group_size;
    for (int it = 0; it < n_k; ++it) {
      const int ws = it % kWStages, bs = it % kBStages;
      if (!mbar_wait(&sm.w_full[ws], (it / kWStages) & 1)) break;
      // bf16 slot bs was last read by the MMAs of k-block it - kBStages
      if (it >= kBStages) {
        const int j = it - kBStages;
        if (!mbar_wait(&sm.mma_done[j % kXStages], (j / kXStages) & 1)) break;
      }
      const int k0 = k_begin + it * kBK;
      if (p.groups > 1 && k0 / p.group_size != cur_group) {
        cur_group = k0 / p.group_size;
        rs = row_scale(wvalid ? __ldg(srow + cur_group) : 0.0f);
      }
      const bool post = __any_sync(0xffffffffu, needs_post(rs));
      const uint8_t* wsrc = w_ring + (size_t)ws * kWTile + t * kBK + 32 * half;
      uint8_t* bdst = b_ring + (size_t)bs * kBTile + (t >> 3) * 1024 + (t & 7) * 128;
      uint4 wv[2];
#pragma unroll
      for (int c = 0; c < 2; ++c) wv[c] = *reinterpret_cast<const uint4*>(wsrc + 16 * c);
#pragma unroll
      for (int c = 0; c < 2; ++c) {  // 16 bytes -> two 16-byte bf16 chunks
        uint32_t o0[4], o1[4];
        deq8(wv[c].x, wv[c].y, rs, post, o0);
        deq8(wv[c].z, wv[c].w, rs, post, o1);
        const int c0 = 4 * half + 2 * c, c1 = c0 + 1;
        *reinterpret_cast<uint4*>(bdst + ((c0 ^ (t & 7)) << 4)) = make_uint4(o0[0], o0[1], o0[2], o0[3]);
        *reinterpret_cast<uint4*>(bdst + ((c1 ^ (t & 7)) << 4)) = make_uint4(o1[0], o1[1], o1[2], o1[3]);
      }
      // the u8 slot is released only after its values are consumed, and the
      // proxy fence orders these generic-proxy accesses before the TMA's
      // (async-proxy) rewrite of the slot and the MMA's read of the tile
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&sm.w_empty[ws]);
        mbar_arrive(&sm.b_full[bs]);
      }
    }

    // epilogue: this warp reads TMEM lanes 32·(warp % 4) .. +31 = tokens; the
    // four warps of a lane quarter split the columns: set cs takes columns
    // [64·cs, 64·cs + 64) (SwiGLU: gate columns [32·cs, 32·cs + 32) and the
    // matching up columns 128 further)
    const int q = warp & 3;
    const int cs = (warp - 3) >> 2;
    const int tok = m0 + 32 * q + lane;
    const bool ok = mbar_wait(&sm.acc_full, 0);
    tc_fence_after();
    const int nsplit = gridDim.z;
    const uint32_t lane_addr = tmem + ((uint32_t)(32 * q) << 16);
    const int ncols = p.n_rows;  // workspace row width
    // workspace column of accumulator column j
    auto ws_col = [&](int j) {
      return swiglu ? (j < kHalfN ? out0 + j : p.n + out0 + j - kHalfN) : out0 + j;
    };
    // accumulator column j holds a real output column (split-K runs only for
    // n % 64 == 0, so 16-column chunks are whole)
    auto col_valid = [&](int j) { return (swiglu ? out0 + (j % kHalfN) : out0 + j) < p.n; };
    bool finish = true;
    if (nsplit > 1) {
      // partial -> workspace; the last CTA of the tile sums all splits in order
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        const int j0 = swiglu ? (c < 2 ? 32 * cs + 16 * c : kHalfN + 32 * cs + 16 * (c - 2))
                              : 64 * cs + 16 * c;
        float v[kChunk];
        tmem_ld16(lane_addr + j0, v);
        if (tok < p.m && col_valid(j0)) {
          float* dst = p.ws + ((int64_t)split * p.m + tok) * ncols + ws_col(j0);
#pragma unroll
          for (int i = 0; i < kChunk; i += 4)
            *reinterpret_cast<float4*>(dst + i) =
                ok ? make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      __threadfence();
      asm volatile("bar.sync 1, %0;" ::"r"(kDeqWarps * 32) : "memory");
      if (d == 0) {
        const uint32_t prev = atomicAdd(&p.counters[blockIdx.y * gridDim.x + blockIdx.x], 1u);
        sm.last = prev == (uint32_t)(nsplit - 1) ? 1u : 0u;
      }
      asm volatile("bar.sync 1, %0;" ::"r"(kDeqWarps * 32) : "memory");
      finish = false;  // the split partials are reduced below, not from TMEM
      if (sm.last != 0) {
        // the last CTA of the tile: all epilogue threads sum the splits of
        // 4 consecutive output columns of one token each, in split order, with
        // up to 4 splits' loads in flight, and apply the epilogue
        __threadfence();
        const int ntok = min(kBM, p.m - m0);
        const int nout = swiglu ? min(kHalfN, p.n - out0) : min(kBN, p.n - out0);
        const int nq = nout / 4;  // split-K runs only for n % 64 == 0
        const bool vec_y = (reinterpret_cast<uintptr_t>(p.y) & 15) == 0 && p.ldy % 4 == 0;
        for (int e = d; e < ntok * nq; e += kDeqWarps * 32) {
          const int tt = m0 + e / nq, c4 = (e % nq) * 4;
          float4 g = make_float4(0.f, 0.f, 0.f, 0.f), u = g;
          for (int sp0 = 0; sp0 < nsplit; sp0 += 4) {
            float4 gv[4], uv[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              if (sp0 + j < nsplit) {
                const float* row = p.ws + ((int64_t)(sp0 + j) * p.m + tt) * ncols;
                gv[j] = __ldcg(reinterpret_cast<const float4*>(row + out0 + c4));
                if (swiglu) uv[j] = __ldcg(reinterpret_cast<const float4*>(row + p.n + out0 + c4));
              }
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              if (sp0 + j < nsplit) {
                g.x += gv[j].x; g.y += gv[j].y; g.z += gv[j].z; g.w += gv[j].w;
                if (swiglu) { u.x += uv[j].x; u.y += uv[j].y; u.z += uv[j].z; u.w += uv[j].w; }
              }
            }
          }
          const float gg[4] = {g.x, g.y, g.z, g.w}, uu[4] = {u.x, u.y, u.z, u.w};
          const int64_t off = (int64_t)tt * p.ldy + out0 + c4;
          if (swiglu) {
            float r4[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) r4[i] = silu(bf16_round(gg[i])) * bf16_round(uu[i]);
            if (p.y_f32) {
#pragma unroll
              for (int i = 0; i < 4; ++i) static_cast<float*>(p.y)[off + i] = r4[i];
            } else {
#pragma unroll
              for (int i = 0; i < 4; ++i) static_cast<__nv_bfloat16*>(p.y)[off + i] = __float2bfloat16_rn(r4[i]);
            }
          } else if (p.epilogue == RXLA_B200_EPI_RESIDUAL_ADD) {
            float* yy = static_cast<float*>(p.y) + off;
            if (vec_y) {
              float4 h4 = *reinterpret_cast<float4*>(yy);
              h4.x += bf16_round(gg[0]); h4.y += bf16_round(gg[1]);
              h4.z += bf16_round(gg[2]); h4.w += bf16_round(gg[3]);
              *reinterpret_cast<float4*>(yy) = h4;
            } else {
#pragma unroll
              for (int i = 0; i < 4; ++i) yy[i] = yy[i] + bf16_round(gg[i]);
            }
          } else if (p.y_f32) {
#pragma unroll
            for (int i = 0; i < 4; ++i) static_cast<float*>(p.y)[off + i] = gg[i];
          } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) static_cast<__nv_bfloat16*>(p.y)[off + i] = __float2bfloat16_rn(gg[i]);
          }
        }
        if (d == 0) p.counters[blockIdx.y * gridDim.x + blockIdx.x] = 0u;
      }
    }
    // accumulator columns j0 .. j0 + 15 of this token (no split-K)
    auto chunk = [&](int j0, float (&v)[kChunk]) {
      tmem_ld16(lane_addr + j0, v);
      if (!ok)
#pragma unroll
        for (int i = 0; i < kChunk; ++i) v[i] = 0.0f;
    };
    if (finish) {
      if (swiglu) {
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          const int j0 = 32 * cs + 16 * c;  // gate columns; up columns j0 + 128
          float g[kChunk], u[kChunk];
          chunk(j0, g);
          chunk(kHalfN + j0, u);
          if (tok < p.m) {
            const int64_t o0 = (int64_t)tok * p.ldy + out0 + j0;
            __nv_bfloat16* yb = static_cast<__nv_bfloat16*>(p.y) + o0;
            if (!p.y_f32 && out0 + j0 + kChunk <= p.n &&
                (reinterpret_cast<uintptr_t>(yb) & 15) == 0) {
              // a whole chunk: two 16-byte stores instead of 16 scattered ones
              uint32_t pk[kChunk / 2];
#pragma unroll
              for (int i = 0; i < kChunk; i += 2)
                pk[i / 2] = pack_bf16x2(silu(bf16_round(g[i])) * bf16_round(u[i]),
                                        silu(bf16_round(g[i + 1])) * bf16_round(u[i + 1]));
              reinterpret_cast<uint4*>(yb)[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
              reinterpret_cast<uint4*>(yb)[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
            } else {
#pragma unroll
              for (int i = 0; i < kChunk; ++i) {
                if (out0 + j0 + i < p.n) {
                  const float r = silu(bf16_round(g[i])) * bf16_round(u[i]);
                  if (p.y_f32) static_cast<float*>(p.y)[o0 + i] = r;
                  else yb[i] = __float2bfloat16_rn(r);
                }
              }
            }
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          const int j0 = 64 * cs + 16 * c;
          float v[kChunk];
          chunk(j0, v);
          const int col = out0 + j0;
          if (tok >= p.m || col >= p.n) continue;
          const int nv = min(kChunk, p.n - col);
          const int64_t o = (int64_t)tok * p.ldy + col;
          if (p.epilogue == RXLA_B200_EPI_RESIDUAL_ADD) {
            float* yy = static_cast<float*>(p.y) + o;
            if (nv == kChunk && (reinterpret_cast<uintptr_t>(yy) & 15) == 0) {
              // all four 16-byte loads in flight, then the stores
              float4 r[kChunk / 4];
#pragma unroll
              for (int i = 0; i < kChunk / 4; ++i) r[i] = reinterpret_cast<const float4*>(yy)[i];
#pragma unroll
              for (int i = 0; i < kChunk / 4; ++i) {
                r[i].x += bf16_round(v[4 * i]);
                r[i].y += bf16_round(v[4 * i + 1]);
                r[i].z += bf16_round(v[4 * i + 2]);
                r[i].w += bf16_round(v[4 * i + 3]);
                reinterpret_cast<float4*>(yy)[i] = r[i];
              }
            } else {
#pragma unroll
              for (int i = 0; i < kChunk; ++i)
                if (i < nv) yy[i] = yy[i] + bf16_round(v[i]);
            }
          } else if (p.y_f32) {
            float* yy = static_cast<float*>(p.y) + o;
            if (nv == kChunk && (reinterpret_cast<uintptr_t>(yy) & 15) == 0) {
#pragma unroll
              for (int i = 0; i < kChunk / 4; ++i)
                reinterpret_cast<float4*>(yy)[i] =
                    make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
            } else {
#pragma unroll
              for (int i = 0; i < kChunk; ++i)
                if (i < nv) yy[i] = v[i];
            }
          } else {
            __nv_bfloat16* yy = static_cast<__nv_bfloat16*>(p.y) + o;
            if (nv == kChunk && (reinterpret_cast<uintptr_t>(yy) & 15) == 0) {
#pragma unroll
              for (int i = 0; i < kChunk; i += 8) {
                uint4 pk;
                pk.x = pack_bf16x2(v[i], v[i + 1]);
                pk.y = pack_bf16x2(v[i + 2], v[i + 3]);
                pk.z = pack_bf16x2(v[i + 4], v[i + 5]);
                pk.w = pack_bf16x2(v[i + 6], v[i + 7]);
                *reinterpret_cast<uint4*>(yy + i) = pk;
              }
            } else {
#pragma unroll
              for (int i = 0; i < kChunk; ++i)
                if (i < nv) yy[i] = __float2bfloat16_rn(v[i]);
            }
          }
        }
      }
    }
    tc_fence_before();
  }
  // dependents wait for this grid's completion before reading its output; the
  // trigger comes from the thread that waited for the previous grid
  if (threadIdx.x == 64) pdl_launch_dependents();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

}  // namespace gemm

// A split-K workspace is [kGemmCounterBytes of tile counters][partials].  The
// counter region has the same size for every shape: a decoder's GEMMs share
// one workspace, and a region sized by the current shape let a GEMM with few
// tiles write its partials over the counters of one with many tiles (which
// must stay zero between launches).
size_t w8_gemm_workspace_bytes(int64_t m, int64_t n_rows, int splits) {
  if (splits <= 1) return 0;
  return kGemmCounterBytes + (size_t)splits * m * n_rows * 4;
}

int32_t w8_gemm(const GemmArgs& a, cudaStream_t stream) {
  using namespace gemm;
  RXLA_REQUIRE(a.m > 0 && a.n > 0 && a.k > 0, "w8 gemm: empty shape");
  // decode batches: weights on the MMA's M side, dequantized into tensor memory
  if (w8_gemm_dec_applies(a.m, a.k, a.group)) return w8_gemm_dec(a, stream);
  RXLA_REQUIRE(a.k % kBK == 0, "w8 gemm: K must be a multiple of 64");
  RXLA_REQUIRE(a.group % kBK == 0 && a.k % a.group == 0, "w8 gemm: group must be a multiple of 64");
  RXLA_REQUIRE(reinterpret_cast<uintptr_t>(a.x) % 16 == 0 && reinterpret_cast<uintptr_t>(a.w) % 16 == 0,
               "w8 gemm: x and weight must be 16-byte aligned");
  RXLA_REQUIRE(a.m <= INT32_MAX && a.n <= INT32_MAX && a.k <= INT32_MAX, "w8 gemm: size too large");
  const bool swiglu = a.epilogue == RXLA_B200_EPI_SWIGLU;
  const int64_t n_rows = swiglu ? 2 * a.n : a.n;
  const int64_t tiles_m = (a.m + kBM - 1) / kBM;
  const int64_t tiles_n = swiglu ? (a.n + kHalfN - 1) / kHalfN : (a.n + kBN - 1) / kBN;
  RXLA_REQUIRE(tiles_m <= 65535 && tiles_n <= 65535, "w8 gemm: too many tiles");
  int splits = std::max(1, a.splits);
  const int64_t kb = a.k / kBK;
  splits = (int)std::min<int64_t>(splits, kb);
  const int64_t kb_per = (kb + splits - 1) / splits;
  splits = (int)((kb + kb_per - 1) / kb_per);
  if (a.n % 64 != 0) splits = 1;
  if (splits > 1) {
    RXLA_REQUIRE(a.ws && a.ws_bytes >= w8_gemm_workspace_bytes(a.m, n_rows, splits),
                 "w8 gemm: split-K workspace missing or too small");
  }
  auto fn = encode_fn();
  if (!fn) return fail(RXLA_B200_UNAVAILABLE, "cuTensorMapEncodeTiled is unavailable");
  CUtensorMap xmap, wmap;
  {
    const cuuint64_t dims[2] = {(cuuint64_t)a.k, (cuuint64_t)a.m};
    const cuuint64_t strides[1] = {(cuuint64_t)a.ldx * 2};
    const cuuint32_t box[2] = {kBK, kBM};
    const cuuint32_t estr[2] = {1, 1};
    RXLA_REQUIRE((a.ldx * 2) % 16 == 0, "w8 gemm: x row stride must be a multiple of 16 bytes");
    if (fn(&xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(a.x), dims, strides, box,
           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return fail(RXLA_B200_INVALID_ARGUMENT, "w8 gemm: x tensor map encoding failed");
  }
  {
    const cuuint64_t dims[2] = {(cuuint64_t)a.k, (cuuint64_t)n_rows};
    const cuuint64_t strides[1] = {(cuuint64_t)a.k};
    const cuuint32_t box[2] = {kBK, kHalfN};
    const cuuint32_t estr[2] = {1, 1};
    if (fn(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(a.w), dims, strides, box,
           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return fail(RXLA_B200_INVALID_ARGUMENT, "w8 gemm: weight tensor map encoding failed");
  }
  Params p{};
  p.scale = a.scale;
  p.groups = (int32_t)(a.k / a.group);
  p.group_size = (int32_t)a.group;
  p.m = (int32_t)a.m;
  p.n = (int32_t)a.n;
  p.k = (int32_t)a.k;
  p.n_rows = (int32_t)n_rows;
  p.y = a.y;
  p.ldy = a.ldy;
  p.y_f32 = a.y_dtype == RXLA_B200_F32;
  p.epilogue = a.epilogue;
  p.k_per_split = (int32_t)(kb_per * kBK);
  if (splits > 1) {
    RXLA_REQUIRE(tiles_m * tiles_n <= (int64_t)(kGemmCounterBytes / 4),
                 "w8 gemm: too many tiles for the split-K counters");
    p.counters = static_cast<uint32_t*>(a.ws);
    p.ws = reinterpret_cast<float*>(static_cast<uint8_t*>(a.ws) + kGemmCounterBytes);
  }
  const size_t smem = 1024 /*align*/ + 1024 /*barriers*/ + (size_t)kXStages * kXTile +
                      (size_t)kBStages * kBTile + (size_t)kWStages * kWTile;
  cudaError_t e = cudaFuncSetAttribute(w8_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e == cudaSuccess)
    e = launch_pdl(w8_gemm_kernel, dim3((unsigned)tiles_m, (unsigned)tiles_n, (unsigned)splits),
                   dim3(kThreads), smem, stream, xmap, wmap, p);
  if (e != cudaSuccess) return cuda_fail(e, "w8 gemm launch");
  return RXLA_B200_OK;
}

}  // namespace rxla
