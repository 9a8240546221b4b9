// w8_gemm_dec.cu — W8A16 GEMM for decode batches (9 .. 128 tokens) on the
// 5th-generation tensor cores with the weights on the MMA's M side, held in
// tensor memory.
//
// Same reference semantics as w8_gemm.cu (crates/rxla-nn/src/layers.rs:
// 257-298): y[m, n] = bf16(Σ_k bf16(x[m, k]) · bf16(f32(q[n, k] - 128) · s)),
// fp32 accumulation, the same epilogues and split-K reduction order.
//
// Why a second GEMM: with few tokens the work is a weight stream.  The
// prefill kernel puts 128 tokens on M and writes each dequantized weight
// tile to shared memory for the MMA to read back (8 bytes of shared-memory
// traffic per weight byte).  Here a CTA owns 128 weight rows (64 gate + 64
// up rows for SwiGLU) and all tokens (N = 32, 64 or 128, zero-filled by TMA):
//  * warp 0 streams u8 weight tiles [128 rows × 128 k] with TMA (128-byte
//    rows, 128-byte swizzle, so that one thread per row reads its 32-byte
//    slice without bank conflicts) through a deep ring — they do not depend
//    on the previous kernel and are requested before griddepcontrol.wait;
//  * warp 2 loads x tiles [N tokens × 128 k] bf16 (two 64-column halves in
//    the 128-byte-swizzled UMMA K-major layout) after griddepcontrol.wait;
//  * warps 3-18 dequantize: warp w owns TMEM lanes 32·(w % 4) (its 32 weight
//    rows) and k-slice (w - 3) / 4 (32 of the 128 columns = two MMAs' K);
//    each thread turns its row's 32 bytes into 16 bf16x2 words and writes
//    them to the A operand in tensor memory with tcgen05.st — no bf16 tile in
//    shared memory;
//  * warp 1 allocates all 512 TMEM columns (the fp32 accumulator [128 rows ×
//    N] at column 0, four 64-column A stages from column 128) and one thread
//    issues tcgen05.mma (A from TMEM, B = x from shared memory, M = 128,
//    N = tokens, K = 16) eight per k-block, committing each k-block to the
//    barrier that frees its x slot and A stage;
//  * the dequant warps then read the accumulator (thread = weight row, 32
//    lanes = 32 consecutive output columns, so every token's stores are
//    coalesced) and apply the epilogue; SwiGLU's up rows reach the gate rows'
//    threads through shared memory.  Split-K writes fp32 partials and the
//    tile's last CTA sums them in split order, as in w8_gemm.cu.
#include "internal.cuh"

namespace rxla {
namespace gemmdec {

using gemm::mma_commit;
using gemm::sw128_desc;
using gemm::tc_fence_after;
using gemm::tc_fence_before;
using gemm::tma_load_2d;
using w8::deq4;
using w8::needs_post;
using w8::row_scale;
using w8::RowScale;

constexpr int kRows = 128;             // weight rows per tile (MMA M)
constexpr int kHalf = kRows / 2;       // rows per weight TMA box; SwiGLU outputs per tile
constexpr int kBK = 128;               // k per stage
constexpr int kAColsPerStage = kBK / 2;
constexpr int kWTile = kRows * kBK;    // 16 KB

// Per token width: N = 32 runs two CTAs per SM (8 dequant warps, 256 TMEM
// columns and ~90 KB of rings each), so that one CTA's pipeline fill and
// epilogue overlap the other's weight stream; wider N keeps one CTA per SM
// with 16 dequant warps and deep rings (measured: batch 32 +9 %, batch 64
// -6 % with two CTAs).
template <int N>
struct Shape {
  static constexpr int kCtasPerSm = N <= 32 ? 2 : 1;
  static constexpr int kDeqWarps = N <= 32 ? 8 : 16;
  static constexpr int kThreads = (3 + kDeqWarps) * 32;
  // bf16 A stages in TMEM, 64 columns each, after the N accumulator columns:
  // as many as the allocation holds (dequant warps waited ~300 cycles per
  // k-block for a free stage with 2 / 4)
  static constexpr int kAStages = N <= 32 ? 3 : (N <= 64 ? 6 : 4);
  static constexpr int kTmemCols = N <= 32 ? 256 : 512;
  static constexpr int kACol = N;  // first TMEM column of the A stages
  // kXStages >= kAStages: a dequant warp waits on the commit barrier of the
  // x slot of k-block it - kAStages, which must not have moved two phases on
  static constexpr int kXStages = N <= 32 ? 3 : (N <= 64 ? 6 : 4);
  static constexpr int kWStages = N <= 32 ? 4 : (N <= 64 ? 6 : 5);  // u8 tiles, 16 KB each
  static_assert(kACol + kAStages * kBK / 2 <= kTmemCols, "A stages fit the TMEM allocation");
  static constexpr int kXHalf = N * 64 * 2;          // one 64-column half, bf16 SW128
  static constexpr int kXTile = 2 * kXHalf;
  // kind::f16, bf16 A and B (K-major), f32 accumulate, M = 128, N tokens
  static constexpr uint32_t kIdesc =
      (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(kRows >> 4) << 24);
};

struct Params {
  const float* scale;
  int32_t groups, group_size;
  int32_t m, n, k;      // tokens, output columns (SwiGLU: outputs), K
  int32_t n_rows;       // weight rows (2n for SwiGLU)
  void* y;
  int64_t ldy;
  int32_t y_f32, epilogue;
  int32_t k_per_split;  // multiple of kBK
  float* ws;            // [splits][m][n_rows] fp32 partials (splits > 1)
  uint32_t* counters;   // [tiles], zero between launches
};

template <int XS, int WS, int AS>
struct Smem {
  uint64_t w_full[WS];
  uint64_t w_empty[WS];
  uint64_t x_full[XS];
  uint64_t a_full[AS];
  uint64_t mma_done[XS];  // k-block it done: frees x slot it % XS and A stage it % kAStages
  uint64_t acc_full;
  uint32_t tmem_base;
  uint32_t last;
};

// tcgen05.mma with A in tensor memory, B from a shared-memory descriptor
template <uint32_t IDESC>
__device__ __forceinline__ void mma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc,
                                       bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(IDESC), "r"(accumulate ? 1 : 0)
      : "memory");
}

__device__ __forceinline__ void tmem_st8(uint32_t addr, const uint32_t (&v)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(addr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
      : "memory");
}

__device__ __forceinline__ void tmem_ld8(uint32_t addr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "r"(addr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// The tile's last split CTA: y[m0 + t, out0 + c] = epilogue(Σ_s partial_s)
// for its tt_n tokens and 4·nq columns, the sums in split order.  Thread d of
// `stride` takes EU float4 elements per round with SU splits of each (and the
// residual row) in flight, so a round costs one L2 round trip.
template <int EU, int SU, bool SWIGLU>
__device__ __forceinline__ void split_reduce(const Params& p, int d, int stride, int m0, int tt_n,
                                             int nq, int out0, bool vec_y, int nsplit) {
  const int total = tt_n * nq;
  const bool resid = !SWIGLU && p.epilogue == RXLA_B200_EPI_RESIDUAL_ADD;
  for (int e0 = d; e0 < total; e0 += EU * stride) {
    float4 g[EU], u[EU], hres[EU];
    int64_t off[EU], src[EU];
#pragma unroll
    for (int uu = 0; uu < EU; ++uu) {
      const int e = min(e0 + uu * stride, total - 1);
      const int tt = m0 + e / nq, c4 = (e % nq) * 4;
      off[uu] = (int64_t)tt * p.ldy + out0 + c4;
      src[uu] = (int64_t)tt * p.n_rows + out0 + c4;
      g[uu] = make_float4(0.f, 0.f, 0.f, 0.f);
      u[uu] = g[uu];
      if (resid && vec_y) hres[uu] = *reinterpret_cast<const float4*>(static_cast<float*>(p.y) + off[uu]);
    }
    for (int sp0 = 0; sp0 < nsplit; sp0 += SU) {
      float4 gv[EU][SU], uv[EU][SWIGLU ? SU : 1];
#pragma unroll
      for (int uu = 0; uu < EU; ++uu)
#pragma unroll
        for (int jj = 0; jj < SU; ++jj)
          if (sp0 + jj < nsplit) {
            const float* row = p.ws + (int64_t)(sp0 + jj) * p.m * p.n_rows + src[uu];
            gv[uu][jj] = __ldcg(reinterpret_cast<const float4*>(row));
            if (SWIGLU) uv[uu][jj] = __ldcg(reinterpret_cast<const float4*>(row + p.n));
          }
#pragma unroll
      for (int uu = 0; uu < EU; ++uu)
#pragma unroll
        for (int jj = 0; jj < SU; ++jj)
          if (sp0 + jj < nsplit) {
            g[uu].x += gv[uu][jj].x; g[uu].y += gv[uu][jj].y;
            g[uu].z += gv[uu][jj].z; g[uu].w += gv[uu][jj].w;
            if (SWIGLU) {
              u[uu].x += uv[uu][jj].x; u[uu].y += uv[uu][jj].y;
              u[uu].z += uv[uu][jj].z; u[uu].w += uv[uu][jj].w;
            }
          }
    }
#pragma unroll
    for (int uu = 0; uu < EU; ++uu) {
      if (e0 + uu * stride >= total) break;
      const float gg[4] = {g[uu].x, g[uu].y, g[uu].z, g[uu].w};
      if (SWIGLU) {
        const float ug[4] = {u[uu].x, u[uu].y, u[uu].z, u[uu].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float rr = silu(bf16_round(gg[i])) * bf16_round(ug[i]);
          if (p.y_f32) static_cast<float*>(p.y)[off[uu] + i] = rr;
          else static_cast<__nv_bfloat16*>(p.y)[off[uu] + i] = __float2bfloat16_rn(rr);
        }
      } else if (resid) {
        float* yy = static_cast<float*>(p.y) + off[uu];
        if (vec_y) {
          float4 h4 = hres[uu];
          h4.x += bf16_round(gg[0]); h4.y += bf16_round(gg[1]);
          h4.z += bf16_round(gg[2]); h4.w += bf16_round(gg[3]);
          *reinterpret_cast<float4*>(yy) = h4;
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i) yy[i] = yy[i] + bf16_round(gg[i]);
        }
      } else if (p.y_f32) {
#pragma unroll
        for (int i = 0; i < 4; ++i) static_cast<float*>(p.y)[off[uu] + i] = gg[i];
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) static_cast<__nv_bfloat16*>(p.y)[off[uu] + i] = __float2bfloat16_rn(gg[i]);
      }
    }
  }
}

template <int N>
__global__ void __launch_bounds__(Shape<N>::kThreads, Shape<N>::kCtasPerSm)
    w8_gemm_dec_kernel(const __grid_constant__ CUtensorMap xmap,
                       const __grid_constant__ CUtensorMap wmap, const Params p) {
  constexpr int XS = Shape<N>::kXStages;
  constexpr int kWStages = Shape<N>::kWStages;
  constexpr int kAStages = Shape<N>::kAStages;
  constexpr int kDeqWarps = Shape<N>::kDeqWarps;
  constexpr int kTmemCols = Shape<N>::kTmemCols;
  constexpr int kXTile = Shape<N>::kXTile;
  constexpr int kXHalf = Shape<N>::kXHalf;
  constexpr int kSlices = kDeqWarps / 4;  // warps per TMEM lane quarter
  constexpr int kSlice = N / kSlices;     // tokens per epilogue warp
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t* base = smem_raw + pad;
  Smem<XS, kWStages, kAStages>& sm = *reinterpret_cast<Smem<XS, kWStages, kAStages>*>(base);
  uint8_t* x_ring = base + 1024;                          // [XS][x tile]
  uint8_t* w_ring = x_ring + (size_t)XS * kXTile;         // [kWStages][u8 tile]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * N;
  const int tile_n = blockIdx.y;
  const int split = blockIdx.z;
  const bool swiglu = p.epilogue == RXLA_B200_EPI_SWIGLU;
  // weight rows of the tile: [wr0, wr0 + 64) and [wr1, wr1 + 64)
  const int out0 = tile_n * (swiglu ? kHalf : kRows);
  const int wr0 = out0;
  const int wr1 = swiglu ? p.n + out0 : out0 + kHalf;
  const int k_begin = split * p.k_per_split;
  const int k_end = min(p.k, k_begin + p.k_per_split);
  const int n_k = (k_end - k_begin) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kWStages; ++s) {
      mbar_init(&sm.w_full[s], 1);
      mbar_init(&sm.w_empty[s], kDeqWarps);
    }
    for (int s = 0; s < XS; ++s) {
      mbar_init(&sm.x_full[s], 1);
      mbar_init(&sm.mma_done[s], 1);
    }
    for (int s = 0; s < kAStages; ++s) mbar_init(&sm.a_full[s], kDeqWarps);
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
    if (lane == 0) {
      for (int it = 0; it < n_k; ++it) {
        const int s = it % kWStages;
        if (it >= kWStages && !mbar_wait(&sm.w_empty[s], ((it / kWStages) - 1) & 1)) break;
        uint8_t* dst = w_ring + (size_t)s * kWTile;
        const int k0 = k_begin + it * kBK;
        mbar_arrive_expect_tx(&sm.w_full[s], (uint32_t)kWTile);
        tma_load_2d(dst, &wmap, k0, wr0, &sm.w_full[s]);
        tma_load_2d(dst + kHalf * kBK, &wmap, k0, wr1, &sm.w_full[s]);
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------------ x producer (TMA)
    if (lane == 0) {
      pdl_wait();  // x (and the residual) come from the previous kernel
      for (int it = 0; it < n_k; ++it) {
        const int s = it % XS;
        if (it >= XS && !mbar_wait(&sm.mma_done[s], ((it / XS) - 1) & 1)) break;
        mbar_arrive_expect_tx(&sm.x_full[s], (uint32_t)kXTile);
        uint8_t* dst = x_ring + (size_t)s * kXTile;
        tma_load_2d(dst, &xmap, k_begin + it * kBK, m0, &sm.x_full[s]);
        tma_load_2d(dst + kXHalf, &xmap, k_begin + it * kBK + 64, m0, &sm.x_full[s]);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      for (int it = 0; it < n_k; ++it) {
        const int xs = it % XS, as = it % kAStages;
        if (!mbar_wait(&sm.x_full[xs], (it / XS) & 1) ||
            !mbar_wait(&sm.a_full[as], (it / kAStages) & 1))
          break;
        tc_fence_after();
        const uint64_t bd0 = sw128_desc(x_ring + (size_t)xs * kXTile);
        const uint64_t bd1 = sw128_desc(x_ring + (size_t)xs * kXTile + kXHalf);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)  // A: 8 TMEM columns per K = 16; B: +32 bytes
          mma_ts<Shape<N>::kIdesc>(tmem, tmem + Shape<N>::kACol + as * kAColsPerStage + 8 * kk,
                                   (kk < 4 ? bd0 : bd1) + 2 * (kk & 3), it > 0 || kk > 0);
        mma_commit(&sm.mma_done[xs]);
      }
      mma_commit(&sm.acc_full);
    }
  } else {
    // ------------------------------------------- dequant, then epilogue
    const int q = warp & 3;             // TMEM lane quarter: rows 32q .. 32q + 31
    const int j = (warp - 3) >> 2;      // k-slice (64 columns of a stage) / token slice
    const int r = 32 * q + lane;        // tile row
    const int wrow = r < kHalf ? wr0 + r : wr1 + (r - kHalf);
    const int ocol = swiglu ? out0 + (r % kHalf) : wr0 + r;  // output column of the row
    const bool wvalid = wrow < p.n_rows && ocol < p.n;
    const float* srow = p.scale + (int64_t)(wvalid ? wrow : 0) * p.groups;
    RowScale rs = row_scale(wvalid ? __ldg(srow + k_begin / p.group_size) : 0.0f);
    int cur_group = k_begin / p.group_size;
    const uint32_t lane_base = (uint32_t)(32 * q) << 16;
    // 16-byte unit c of row r sits at unit c ^ (r % 8) (128-byte TMA swizzle);
    // this thread's units are 4j .. 4j + 3, two per pass
    constexpr int kUnits = 8 / kSlices;
    bool ok = true;
    for (int it = 0; it < n_k; ++it) {
      const int ws = it % kWStages, as = it % kAStages;
      if (!mbar_wait(&sm.w_full[ws], (it / kWStages) & 1)) {
        ok = false;
        break;
      }
      // A stage `as` was last read by the MMAs of k-block it - kAStages
      if (it >= kAStages) {
        const int jb = it - kAStages;
        if (!mbar_wait(&sm.mma_done[jb % XS], (jb / XS) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      const int k0 = k_begin + it * kBK;
      if (p.groups > 1 && k0 / p.group_size != cur_group) {
        cur_group = k0 / p.group_size;
        rs = row_scale(wvalid ? __ldg(srow + cur_group) : 0.0f);
      }
      const bool post = __any_sync(0xffffffffu, needs_post(rs));
      const uint8_t* wt = w_ring + (size_t)ws * kWTile + 128 * r;
#pragma unroll
      for (int h = 0; h < kUnits / 2; ++h) {
      const int u0 = kUnits * j + 2 * h;
      const uint4 wv0 = *reinterpret_cast<const uint4*>(wt + 16 * (u0 ^ (r & 7)));
      const uint4 wv1 = *reinterpret_cast<const uint4*>(wt + 16 * ((u0 + 1) ^ (r & 7)));
      uint32_t o0[8], o1[8];
      if (post) {
        deq4<true>(wv0.x, rs, o0[0], o0[1]);
        deq4<true>(wv0.y, rs, o0[2], o0[3]);
        deq4<true>(wv0.z, rs, o0[4], o0[5]);
        deq4<true>(wv0.w, rs, o0[6], o0[7]);
        deq4<true>(wv1.x, rs, o1[0], o1[1]);
        deq4<true>(wv1.y, rs, o1[2], o1[3]);
        deq4<true>(wv1.z, rs, o1[4], o1[5]);
        deq4<true>(wv1.w, rs, o1[6], o1[7]);
      } else {
        deq4<false>(wv0.x, rs, o0[0], o0[1]);
        deq4<false>(wv0.y, rs, o0[2], o0[3]);
        deq4<false>(wv0.z, rs, o0[4], o0[5]);
        deq4<false>(wv0.w, rs, o0[6], o0[7]);
        deq4<false>(wv1.x, rs, o1[0], o1[1]);
        deq4<false>(wv1.y, rs, o1[2], o1[3]);
        deq4<false>(wv1.z, rs, o1[4], o1[5]);
        deq4<false>(wv1.w, rs, o1[6], o1[7]);
      }
      const uint32_t adst = tmem + lane_base + Shape<N>::kACol + as * kAColsPerStage + 8 * u0;
      tmem_st8(adst, o0);
      tmem_st8(adst + 8, o1);
      }
      // the u8 slot is released after its bytes are in registers (generic-proxy
      // reads ordered before the TMA's rewrite); the A stage after the
      // tensor-memory stores complete
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&sm.w_empty[ws]);
        mbar_arrive(&sm.a_full[as]);
      }
    }

    // epilogue: thread = tile row r, tokens [kSlice·j, kSlice·j + kSlice)
    ok = ok && mbar_wait(&sm.acc_full, 0);
    tc_fence_after();
    const int nsplit = gridDim.z;
    const int t0 = m0 + kSlice * j;
    float v[kSlice];
#pragma unroll
    for (int c = 0; c < kSlice; c += 8) {
      float t8[8];
      tmem_ld8(tmem + lane_base + (uint32_t)(kSlice * j + c), t8);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[c + i] = ok ? t8[i] : 0.0f;
    }
    const int ntok = min(kSlice, p.m - t0);  // may be <= 0
    if (nsplit > 1) {
      // partial -> workspace [split][m][n_rows]; the tile's last CTA sums the
      // splits in order and applies the epilogue
      if (wvalid)
        for (int i = 0; i < ntok; ++i) p.ws[((int64_t)split * p.m + t0 + i) * p.n_rows + wrow] = v[i];
      __threadfence();
      asm volatile("bar.sync 1, %0;" ::"r"(kDeqWarps * 32) : "memory");
      const int d = threadIdx.x - 96;
      if (d == 0) {
        const uint32_t prev = atomicAdd(&p.counters[blockIdx.y * gridDim.x + blockIdx.x], 1u);
        sm.last = prev == (uint32_t)(nsplit - 1) ? 1u : 0u;
      }
      asm volatile("bar.sync 1, %0;" ::"r"(kDeqWarps * 32) : "memory");
      if (sm.last != 0) {
        __threadfence();
        const int tt_n = min(N, p.m - m0);
        const int nout = swiglu ? min(kHalf, p.n - out0) : min(kRows, p.n - out0);
        const int nq = nout / 4;  // split-K runs only for n % 64 == 0
        const bool vec_y = (reinterpret_cast<uintptr_t>(p.y) & 15) == 0 && p.ldy % 4 == 0;
        if (swiglu)
          split_reduce<(N <= 32 ? 1 : 2), 2, true>(p, d, kDeqWarps * 32, m0, tt_n, nq, out0, vec_y, nsplit);
        else
          split_reduce<(N <= 32 ? 1 : 2), 4, false>(p, d, kDeqWarps * 32, m0, tt_n, nq, out0, vec_y, nsplit);
        if (d == 0) p.counters[blockIdx.y * gridDim.x + blockIdx.x] = 0u;
      }
    } else if (swiglu) {
      // up rows (lane quarters 2, 3) hand their values to the gate rows'
      // threads through shared memory (the weight ring is idle now)
      float* up = reinterpret_cast<float*>(w_ring);  // [64 rows][N]
      if (r >= kHalf)
#pragma unroll
        for (int i = 0; i < kSlice; ++i) up[(r - kHalf) * N + kSlice * j + i] = v[i];
      asm volatile("bar.sync 1, %0;" ::"r"(kDeqWarps * 32) : "memory");
      if (r < kHalf && wvalid) {
        for (int i = 0; i < ntok; ++i) {
          const float rr = silu(bf16_round(v[i])) * bf16_round(up[r * N + kSlice * j + i]);
          const int64_t o = (int64_t)(t0 + i) * p.ldy + ocol;
          if (p.y_f32) static_cast<float*>(p.y)[o] = rr;
          else static_cast<__nv_bfloat16*>(p.y)[o] = __float2bfloat16_rn(rr);
        }
      }
    } else if (wvalid) {
      for (int i = 0; i < ntok; ++i) {
        const int64_t o = (int64_t)(t0 + i) * p.ldy + ocol;
        if (p.epilogue == RXLA_B200_EPI_RESIDUAL_ADD) {
          float* yy = static_cast<float*>(p.y) + o;
          *yy = *yy + bf16_round(v[i]);
        } else if (p.y_f32) {
          static_cast<float*>(p.y)[o] = v[i];
        } else {
          static_cast<__nv_bfloat16*>(p.y)[o] = __float2bfloat16_rn(v[i]);
        }
      }
    }
    tc_fence_before();
  }
  // dependents wait for this grid's completion; the trigger comes from the
  // thread that waited for the previous grid
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

template <int N>
static cudaError_t launch(const CUtensorMap& xmap, const CUtensorMap& wmap, const Params& p,
                          dim3 grid, cudaStream_t stream) {
  constexpr int XS = Shape<N>::kXStages;
  constexpr int WS = Shape<N>::kWStages;
  const size_t smem = 1024 /*align*/ + 1024 /*barriers*/ + (size_t)XS * Shape<N>::kXTile +
                      (size_t)WS * kWTile;
  static_assert(sizeof(Smem<XS, WS, Shape<N>::kAStages>) <= 1024, "barrier block");
  static_assert(XS >= Shape<N>::kAStages, "one commit slot per x slot covers the A stages");
  static_assert((size_t)kHalf * N * 4 <= (size_t)WS * kWTile, "SwiGLU exchange fits the ring");
  auto kern = w8_gemm_dec_kernel<N>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(kern, grid, dim3(Shape<N>::kThreads), smem, stream, xmap, wmap, p);
}

}  // namespace gemmdec

bool w8_gemm_dec_applies(int64_t m, int64_t k, int64_t group) {
  return m <= kGemmDecMaxTokens && k % gemmdec::kBK == 0 &&
         group % gemmdec::kBK == 0;
}

int64_t w8_gemm_tiles(int64_t m, int64_t n, int64_t k, int64_t group, bool swiglu) {
  if (w8_gemm_dec_applies(m, k, group))
    return swiglu ? (n + gemmdec::kHalf - 1) / gemmdec::kHalf : (n + gemmdec::kRows - 1) / gemmdec::kRows;
  return ((m + gemm::kBM - 1) / gemm::kBM) *
         (swiglu ? (n + gemm::kHalfN - 1) / gemm::kHalfN : (n + gemm::kBN - 1) / gemm::kBN);
}

// Split-K depth (one CTA per SM): the depth that minimises the grid's
// critical path, counted in k-blocks (k per pipeline stage): waves ×
// (k-blocks per split + the split's partial tile write) + the tile's last CTA
// reading every split's partial; at least two k-blocks per split, at most 16
// splits.  ceil(SMs / tiles) — the earlier rule — put a few CTAs in a second,
// nearly empty wave (config 4 batch 64: 5.7k -> 6.4k tok/s with this rule on
// the prefill-shaped kernel).  RXLA_B200_SPLIT_POLICY=0 restores the old rule.
int w8_gemm_splits(int64_t m, int64_t n, int64_t k, int64_t group, bool swiglu) {
  if (n % 64 != 0) return 1;
  int dev = 0;
  cudaGetDevice(&dev);
  const bool dec = w8_gemm_dec_applies(m, k, group);
  const int ctas_per_sm = !dec ? 1 : (m <= 32 ? gemmdec::Shape<32>::kCtasPerSm : gemmdec::Shape<64>::kCtasPerSm);
  const int64_t sms = (int64_t)sm_count(dev) * ctas_per_sm;  // CTA slots of one wave
  const int64_t tiles = w8_gemm_tiles(m, n, k, group, swiglu);
  const int64_t kblock = dec ? gemmdec::kBK : gemm::kBK;
  const int64_t rows = dec ? gemmdec::kRows : gemm::kBN;  // weight rows per tile
  const int64_t kb = (k + kblock - 1) / kblock;
  const int64_t smax = std::max<int64_t>(1, std::min<int64_t>(16, kb / 2));
  // a split's partial tile (m × rows f32) in units of one k-block of weights
  const double pu = (double)std::min<int64_t>(m, 128) * rows * 4 / (double)(rows * kblock);
  int64_t best = 1;
  double best_cost = 1e300;
  for (int64_t sp = 1; sp <= smax; ++sp) {
    const double waves = (double)((tiles * sp + sms - 1) / sms);
    const double cost = waves * ((double)((kb + sp - 1) / sp) + (sp > 1 ? pu : 0.0)) +
                        (sp > 1 ? (double)sp * pu : 0.0);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = sp;
    }
  }
  return (int)best;
}

int32_t w8_gemm_dec(const GemmArgs& a, cudaStream_t stream) {
  using namespace gemmdec;
  RXLA_REQUIRE(a.m > 0 && a.m <= kGemmDecMaxTokens && a.n > 0 && a.k > 0,
               "w8 gemm (decode): 1..128 tokens");
  RXLA_REQUIRE(a.k % kBK == 0, "w8 gemm (decode): K must be a multiple of 128");
  RXLA_REQUIRE(a.group % kBK == 0 && a.k % a.group == 0,
               "w8 gemm (decode): group must be a multiple of 128");
  RXLA_REQUIRE(reinterpret_cast<uintptr_t>(a.x) % 16 == 0 && reinterpret_cast<uintptr_t>(a.w) % 16 == 0,
               "w8 gemm (decode): x and weight must be 16-byte aligned");
  RXLA_REQUIRE((a.ldx * 2) % 16 == 0, "w8 gemm (decode): x row stride must be a multiple of 16 bytes");
  const bool swiglu = a.epilogue == RXLA_B200_EPI_SWIGLU;
  const int64_t n_rows = swiglu ? 2 * a.n : a.n;
  const int N = a.m <= 32 ? 32 : (a.m <= 64 ? 64 : 128);
  const int64_t tiles_n = w8_gemm_tiles(a.m, a.n, a.k, a.group, swiglu);
  RXLA_REQUIRE(tiles_n <= 65535, "w8 gemm (decode): too many tiles");
  int splits = std::max(1, a.splits);
  const int64_t kb = a.k / kBK;
  splits = (int)std::min<int64_t>(splits, kb);
  const int64_t kb_per = (kb + splits - 1) / splits;
  splits = (int)((kb + kb_per - 1) / kb_per);
  if (a.n % 64 != 0) splits = 1;
  if (splits > 1)
    RXLA_REQUIRE(a.ws && a.ws_bytes >= w8_gemm_workspace_bytes(a.m, n_rows, splits),
                 "w8 gemm (decode): split-K workspace missing or too small");
  auto fn = gemm::encode_fn();
  if (!fn) return fail(RXLA_B200_UNAVAILABLE, "cuTensorMapEncodeTiled is unavailable");
  CUtensorMap xmap, wmap;
  {
    const cuuint64_t dims[2] = {(cuuint64_t)a.k, (cuuint64_t)a.m};
    const cuuint64_t strides[1] = {(cuuint64_t)a.ldx * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)N};
    const cuuint32_t estr[2] = {1, 1};
    if (fn(&xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(a.x), dims, strides, box,
           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return fail(RXLA_B200_INVALID_ARGUMENT, "w8 gemm (decode): x tensor map encoding failed");
  }
  {
    const cuuint64_t dims[2] = {(cuuint64_t)a.k, (cuuint64_t)n_rows};
    const cuuint64_t strides[1] = {(cuuint64_t)a.k};
    const cuuint32_t box[2] = {kBK, kHalf};
    const cuuint32_t estr[2] = {1, 1};
    if (fn(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(a.w), dims, strides, box,
           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return fail(RXLA_B200_INVALID_ARGUMENT, "w8 gemm (decode): weight tensor map encoding failed");
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
    RXLA_REQUIRE(tiles_n <= (int64_t)(kGemmCounterBytes / 4),
                 "w8 gemm (decode): too many tiles for the split-K counters");
    p.counters = static_cast<uint32_t*>(a.ws);
    p.ws = reinterpret_cast<float*>(static_cast<uint8_t*>(a.ws) + kGemmCounterBytes);
  }
  const dim3 grid(1, (unsigned)tiles_n, (unsigned)splits);
  cudaError_t e = N == 32 ? launch<32>(xmap, wmap, p, grid, stream)
                : N == 64 ? launch<64>(xmap, wmap, p, grid, stream)
                          : launch<128>(xmap, wmap, p, grid, stream);
  if (e != cudaSuccess) return cuda_fail(e, "w8 gemm (decode) launch");
  return RXLA_B200_OK;
}

}  // namespace rxla
