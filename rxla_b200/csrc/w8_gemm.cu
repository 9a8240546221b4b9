// w8_gemm.cu — W8A16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM)
// for more than a handful of tokens: prefill, and decode at batch > 8.
//
// Reference semantics (crates/rxla-nn/src/layers.rs:257-298, bf16 compute):
// y[m, n] = bf16( Σ_k bf16(x[m, k]) · bf16(f32(q[n, k] - 128) · s[n, k / G]) ),
// fp32 accumulation; the same epilogues as the skinny kernel (bf16 / f32
// store, f32 residual add of the bf16 dot, SwiGLU of a fused [gate; up]).
//
// Tile: 128 tokens (MMA M) × 128 weight rows (MMA N), K staged 64 at a time.
//  * warp 0 (producer): TMA loads of the x tile [128 × 64] bf16 (128-byte
//    swizzle, the UMMA K-major SW128 layout) and the weight tile [128 × 64] u8
//    (two 64-row boxes; for SwiGLU the gate rows and the matching up rows);
//  * warps 2-5 (dequant, then epilogue): each thread turns one weight row of
//    the stage into bf16 with the reference's rounding (packed denormal FMA,
//    as in the skinny kernel) and stores it in the SW128 K-major layout the
//    MMA reads, fences the generic->async proxy and arrives;
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

constexpr int kBM = 128, kBN = 128, kBK = 64;
constexpr int kStages = 4;
constexpr int kXTile = kBM * kBK * 2;   // 16 KB bf16, SW128
constexpr int kBTile = kBN * kBK * 2;   // 16 KB bf16, SW128
constexpr int kWTile = kBN * kBK;       // 8 KB u8
constexpr int kStageBytes = kXTile + kBTile + kWTile;
constexpr int kThreads = 6 * 32;
constexpr int kTmemCols = 128;

struct Params {
  const float* scale;
  int32_t groups, group_size;
  int32_t m, n, k;            // tokens, output columns (SwiGLU: outputs), K
  int32_t n_rows;             // weight rows (2n for SwiGLU)
  void* y;
  int64_t ldy;
  int32_t y_f32, epilogue;    // RXLA_B200_EPI_*
  int32_t k_per_split;        // multiple of kBK
  float* ws;                  // [splits][m][n] fp32 partials (splits > 1)
  uint32_t* counters;         // [tiles], zero between launches
};

struct Smem {
  uint64_t full[kStages];
  uint64_t bready[kStages];
  uint64_t empty[kStages];
  uint64_t acc_full;
  uint32_t tmem_base;
  uint32_t last;
};

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

__device__ __forceinline__ void tmem_ld32(uint32_t addr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(addr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
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
  uint8_t* stages = base + 1024;  // stage s: x tile | bf16 weight tile | u8 weight tile

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kBM;
  const int tile_n = blockIdx.y;
  const int split = blockIdx.z;
  const bool swiglu = p.epilogue == RXLA_B200_EPI_SWIGLU;
  // weight rows of this tile: rows [wr0, wr0 + 64) and [wr1, wr1 + 64)
  const int out0 = tile_n * (swiglu ? kBN / 2 : kBN);  // first output column
  const int wr0 = out0;
  const int wr1 = swiglu ? p.n + out0 : out0 + 64;
  const int k_begin = split * p.k_per_split;
  const int k_end = min(p.k, k_begin + p.k_per_split);
  const int n_k = (k_end - k_begin) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.bready[s], 4);
      mbar_init(&sm.empty[s], 1);
    }
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
    // ---------------------------------------------------------------- TMA
    if (lane == 0) {
      pdl_wait();  // x (and the residual) come from the previous kernel
      for (int it = 0; it < n_k; ++it) {
        const int s = it % kStages;
        if (it >= kStages && !mbar_wait(&sm.empty[s], ((it / kStages) - 1) & 1)) break;
        uint8_t* st = stages + (size_t)s * kStageBytes;
        const int k0 = k_begin + it * kBK;
        mbar_arrive_expect_tx(&sm.full[s], (uint32_t)(kXTile + kWTile));
        tma_load_2d(st, &xmap, k0, m0, &sm.full[s]);
        tma_load_2d(st + kXTile + kBTile, &wmap, k0, wr0, &sm.full[s]);
        tma_load_2d(st + kXTile + kBTile + 64 * kBK, &wmap, k0, wr1, &sm.full[s]);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      for (int it = 0; it < n_k; ++it) {
        const int s = it % kStages;
        const uint32_t ph = (it / kStages) & 1;
        if (!mbar_wait(&sm.full[s], ph) || !mbar_wait(&sm.bready[s], ph)) break;
        tc_fence_after();
        uint8_t* st = stages + (size_t)s * kStageBytes;
        const uint64_t ad = sw128_desc(st), bd = sw128_desc(st + kXTile);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)  // +32 bytes per K = 16 step
          mma_bf16(tmem, ad + 2 * kk, bd + 2 * kk, it > 0 || kk > 0);
        mma_commit(&sm.empty[s]);
      }
      mma_commit(&sm.acc_full);
    }
  } else {
    // ------------------------------------------- dequant, then epilogue
    const int t = threadIdx.x - 64;  // 0 .. 127: weight row of the tile / token row
    const int wrow = t < 64 ? wr0 + t : wr1 + (t - 64);
    const bool wvalid = wrow < p.n_rows && (swiglu ? (t < 64 ? out0 + t : out0 + t - 64) < p.n : true);
    const float* srow = p.scale + (int64_t)(wvalid ? wrow : 0) * p.groups;
    RowScale rs = row_scale(wvalid ? __ldg(srow + k_begin / p.group_size) : 0.0f);
    int cur_group = k_begin / p.group_size;
    for (int it = 0; it < n_k; ++it) {
      const int s = it % kStages;
      if (!mbar_wait(&sm.full[s], (it / kStages) & 1)) break;
      const int k0 = k_begin + it * kBK;
      if (p.groups > 1 && k0 / p.group_size != cur_group) {
        cur_group = k0 / p.group_size;
        rs = row_scale(wvalid ? __ldg(srow + cur_group) : 0.0f);
      }
      const bool post = __any_sync(0xffffffffu, needs_post(rs));
      uint8_t* st = stages + (size_t)s * kStageBytes;
      const uint8_t* wsrc = st + kXTile + kBTile + t * kBK;
      uint8_t* bdst = st + kXTile + (t >> 3) * 1024 + (t & 7) * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) {  // 16 bytes -> two 16-byte bf16 chunks
        const uint4 w = *reinterpret_cast<const uint4*>(wsrc + 16 * c);
        uint32_t o0[4], o1[4];
        deq8(w.x, w.y, rs, post, o0);
        deq8(w.z, w.w, rs, post, o1);
        const int c0 = 2 * c, c1 = 2 * c + 1;
        *reinterpret_cast<uint4*>(bdst + ((c0 ^ (t & 7)) << 4)) = make_uint4(o0[0], o0[1], o0[2], o0[3]);
        *reinterpret_cast<uint4*>(bdst + ((c1 ^ (t & 7)) << 4)) = make_uint4(o1[0], o1[1], o1[2], o1[3]);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.bready[s]);
    }

    // epilogue: this warp reads TMEM lanes 32·(warp % 4) .. +31 = tokens, in
    // chunks of 32 accumulator columns (SwiGLU: a gate chunk and its up chunk)
    const int q = warp & 3;
    const int tok = m0 + 32 * q + lane;
    const bool ok = mbar_wait(&sm.acc_full, 0);
    tc_fence_after();
    const int nsplit = gridDim.z;
    const uint32_t lane_addr = tmem + ((uint32_t)(32 * q) << 16);
    const int ncols = p.n_rows;  // workspace row width
    // workspace column of accumulator column j
    auto ws_col = [&](int j) { return swiglu ? (j < 64 ? out0 + j : p.n + out0 + j - 64) : out0 + j; };
    // a 32-column chunk exists when its first output column does (split-K
    // runs only for n % 64 == 0, so chunks are whole)
    auto chunk_valid = [&](int c) { return (swiglu ? out0 + 32 * (c & 1) : out0 + 32 * c) < p.n; };
    bool finish = true;
    if (nsplit > 1) {
      // partial -> workspace; the last CTA of the tile sums all splits in order
#pragma unroll 1
      for (int c = 0; c < kBN / 32; ++c) {
        float v[32];
        tmem_ld32(lane_addr + 32 * c, v);
        if (tok < p.m && chunk_valid(c)) {
          float* dst = p.ws + ((int64_t)split * p.m + tok) * ncols + ws_col(32 * c);
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            *reinterpret_cast<float4*>(dst + i) =
                ok ? make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      __threadfence();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (t == 0) {
        const uint32_t prev = atomicAdd(&p.counters[blockIdx.y * gridDim.x + blockIdx.x], 1u);
        sm.last = prev == (uint32_t)(nsplit - 1) ? 1u : 0u;
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      finish = sm.last != 0;
      if (finish) __threadfence();
    }
    // accumulator chunk c (32 columns) of this token: from TMEM, or the sum of
    // all splits' partials in split order
    auto chunk = [&](int c, float (&v)[32]) {
      if (nsplit == 1) {
        tmem_ld32(lane_addr + 32 * c, v);
        if (!ok)
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = 0.0f;
        return;
      }
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = 0.0f;
      if (tok >= p.m || !chunk_valid(c)) return;
      for (int sp = 0; sp < nsplit; ++sp) {
        const float* src = p.ws + ((int64_t)sp * p.m + tok) * ncols + ws_col(32 * c);
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          const float4 x4 = __ldcg(reinterpret_cast<const float4*>(src + i));
          v[i] += x4.x;
          v[i + 1] += x4.y;
          v[i + 2] += x4.z;
          v[i + 3] += x4.w;
        }
      }
    };
    if (finish) {
      if (swiglu) {
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          float g[32], u[32];
          chunk(c, g);
          chunk(c + 2, u);
          const int j0 = out0 + 32 * c;
          if (tok < p.m) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              if (j0 + i < p.n) {
                const float r = silu(bf16_round(g[i])) * bf16_round(u[i]);
                const int64_t o = (int64_t)tok * p.ldy + j0 + i;
                if (p.y_f32) static_cast<float*>(p.y)[o] = r;
                else static_cast<__nv_bfloat16*>(p.y)[o] = __float2bfloat16_rn(r);
              }
            }
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < kBN / 32; ++c) {
          float v[32];
          chunk(c, v);
          const int j0 = out0 + 32 * c;
          if (tok >= p.m || j0 >= p.n) continue;
          const int nv = min(32, p.n - j0);
          const int64_t o = (int64_t)tok * p.ldy + j0;
          if (p.epilogue == RXLA_B200_EPI_RESIDUAL_ADD) {
            float* yy = static_cast<float*>(p.y) + o;
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (i < nv) yy[i] = yy[i] + bf16_round(v[i]);
          } else if (p.y_f32) {
            float* yy = static_cast<float*>(p.y) + o;
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (i < nv) yy[i] = v[i];
          } else {
            __nv_bfloat16* yy = static_cast<__nv_bfloat16*>(p.y) + o;
            if (nv == 32 && (reinterpret_cast<uintptr_t>(yy) & 15) == 0) {
#pragma unroll
              for (int i = 0; i < 32; i += 8) {
                uint4 pk;
                pk.x = pack_bf16x2(v[i], v[i + 1]);
                pk.y = pack_bf16x2(v[i + 2], v[i + 3]);
                pk.z = pack_bf16x2(v[i + 4], v[i + 5]);
                pk.w = pack_bf16x2(v[i + 6], v[i + 7]);
                *reinterpret_cast<uint4*>(yy + i) = pk;
              }
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (i < nv) yy[i] = __float2bfloat16_rn(v[i]);
            }
          }
        }
      }
      if (nsplit > 1 && t == 0) p.counters[blockIdx.y * gridDim.x + blockIdx.x] = 0u;
    }
    tc_fence_before();
  }
  // dependents wait for this grid's completion before reading its output
  if (threadIdx.x == 0) pdl_launch_dependents();
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

size_t w8_gemm_workspace_bytes(int64_t m, int64_t n_rows, int splits) {
  if (splits <= 1) return 0;
  const int64_t tiles = ((m + gemm::kBM - 1) / gemm::kBM) * ((n_rows + gemm::kBN - 1) / gemm::kBN);
  const size_t counters = ((size_t)tiles * 4 + 255) / 256 * 256;
  return counters + (size_t)splits * m * n_rows * 4;
}

int32_t w8_gemm(const GemmArgs& a, cudaStream_t stream) {
  using namespace gemm;
  RXLA_REQUIRE(a.m > 0 && a.n > 0 && a.k > 0, "w8 gemm: empty shape");
  RXLA_REQUIRE(a.k % kBK == 0, "w8 gemm: K must be a multiple of 64");
  RXLA_REQUIRE(a.group % kBK == 0 && a.k % a.group == 0, "w8 gemm: group must be a multiple of 64");
  RXLA_REQUIRE(reinterpret_cast<uintptr_t>(a.x) % 16 == 0 && reinterpret_cast<uintptr_t>(a.w) % 16 == 0,
               "w8 gemm: x and weight must be 16-byte aligned");
  RXLA_REQUIRE(a.m <= INT32_MAX && a.n <= INT32_MAX && a.k <= INT32_MAX, "w8 gemm: size too large");
  const bool swiglu = a.epilogue == RXLA_B200_EPI_SWIGLU;
  const int64_t n_rows = swiglu ? 2 * a.n : a.n;
  const int64_t tiles_m = (a.m + kBM - 1) / kBM;
  const int64_t tiles_n = swiglu ? (a.n + 63) / 64 : (a.n + kBN - 1) / kBN;
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
    const cuuint32_t box[2] = {kBK, 64};
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
    const int64_t tiles = tiles_m * tiles_n;
    const size_t counters = ((size_t)tiles * 4 + 255) / 256 * 256;
    p.counters = static_cast<uint32_t*>(a.ws);
    p.ws = reinterpret_cast<float*>(static_cast<uint8_t*>(a.ws) + counters);
  }
  const size_t smem = 1024 /*align*/ + 1024 /*barriers*/ + (size_t)kStages * kStageBytes;
  cudaError_t e = cudaFuncSetAttribute(w8_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e == cudaSuccess)
    e = launch_pdl(w8_gemm_kernel, dim3((unsigned)tiles_m, (unsigned)tiles_n, (unsigned)splits),
                   dim3(kThreads), smem, stream, xmap, wmap, p);
  if (e != cudaSuccess) return cuda_fail(e, "w8 gemm launch");
  return RXLA_B200_OK;
}

}  // namespace rxla
