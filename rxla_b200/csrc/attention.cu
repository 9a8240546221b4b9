// attention.cu — paged GQA decode attention with fused q/k RMSNorm, RoPE and
// KV append (one decode token per sequence).
//
// Reference semantics (paths inside the rxla project):
//   grouped_query_attention / SDPA   crates/rxla-core/src/attention.rs:83-252
//     softmax(q·kᵀ·scale + mask)·v, scale 1/sqrt(D), consecutive query heads
//     share a kv head (:73-75); decode mask = key position <= query position
//   KvCache::update_at(_checked)     crates/rxla-core/src/kv_cache.rs:53-112
//     clamped start, or checked start that leaves the cache unchanged
//   rotary_embedding, SplitHalf      crates/rxla-core/src/rotary.rs:29-74
//   per-head q_norm / k_norm         crates/rxla-models/src/qwen3_5/layers.rs:51-74
//
// Cache: bf16 [num_pages, kv_heads, 16, D] for K and V; page_table maps the
// p-th page of a sequence.  The kernel stores the new k (normed, rotated,
// rounded to bf16) and v at slot ctx_len of each sequence.
//
// Design (HBM-bound: the whole visible cache is read once):
//  * CTA = (split of `pps` pages, kv head, sequence); four compute warps take
//    the split's pages round-robin while a producer warp streams them through
//    an 8-stage shared-memory ring with TMA tensor loads (one box is
//    [64 dims × 16 rows] with 128-byte swizzle).  Splits are sized so the
//    grid holds a few CTAs per SM at full context, with at most 32 splits;
//  * q is normalised and rotated lane-locally in the layout of the mma B
//    fragment (a RoPE pair (i, i + rot/2) lives in one lane), split into
//    bf16 hi + lo so q·k keeps fp32 accuracy against the bf16 cache;
//  * S^T = K·Q^T with tokens on the mma M side (16 per page) and the G query
//    heads of the kv head on the N side; online softmax per head column;
//    P^T (split into bf16 hi + lo, so the weights keep f32 accuracy) is moved
//    into the B-fragment layout with movmatrix.trans and O^T += V^T·P^T (V^T
//    from ldmatrix.trans of the swizzled tile);
//  * the CTA owning the new slot writes k/v to the cache and patches the row
//    into its loaded tile; every CTA fences and then triggers dependent
//    launches, so later kernels (including the next step's attention, whose
//    page prefetch runs before griddepcontrol.wait) see the appended rows;
//  * the four warps' softmax states merge in shared memory; splits write
//    (O, m, l) partials to the workspace and the last CTA of a (sequence,
//    kv head) (atomic counter) merges them with log-sum-exp weights and
//    resets the counter.  A single split writes the output directly.
#include <cudaTypedefs.h>

#include "common.cuh"

namespace rxla {
namespace attn {

constexpr int kPage = 16;

struct Params {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k_new;
  const __nv_bfloat16* v_new;
  int64_t q_stride, kv_stride;
  const float* q_norm_w;
  const float* k_norm_w;
  float eps;
  const float* inv_freq;
  int32_t rot;  // rotary dims (multiple of 32) or 0
  float scale;
  __nv_bfloat16* k_pages;
  __nv_bfloat16* v_pages;
  const int32_t* page_table;
  const int32_t* pages_per_seq;
  int32_t max_pages;
  int32_t* ctx_lens;
  int32_t kv_update, advance_ctx;
  int32_t* accepted;
  __nv_bfloat16* out;
  int32_t hq, hkv, group;  // group = hq / hkv <= 8
  int32_t pps;             // pages per split
  int32_t max_splits;
  float* ws_o;     // [batch][hkv][max_splits][group][D]
  float* ws_ml;    // [batch][hkv][max_splits][group][2]
  uint32_t* ws_counter;  // [batch * hkv] split arrivals, then [1] CTA exits
  int32_t batch;
  int32_t ctx_stable;    // ctx_lens is not written by the previous kernel: prefetch early
  int32_t stages;
  int32_t stage_bytes;  // K + V of one page of one kv head
  L2Prefetch next;      // the following kernel's first bytes
};

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ uint32_t movmatrix_t(uint32_t a) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}

// Byte offset of (row r, dim d) inside a [rows × D] bf16 region stored as
// D/64 swizzled 128-byte boxes of `rows` rows each (TMA SWIZZLE_128B).
__device__ __forceinline__ uint32_t swz(int r, int d, int rows) {
  const int j = d >> 6, c = (d & 63) >> 3;
  return (uint32_t)(j * rows * 128 + r * 128 + ((c ^ (r & 7)) << 4) + (d & 7) * 2);
}

// Grid-wide tail: the last CTA to finish publishes accepted / advanced
// context lengths (no CTA may still read ctx_lens by then) and resets the
// exit counter.
__device__ __forceinline__ void finish_cta(const Params& p) {
  if (!p.advance_ctx && !p.accepted) return;
  __threadfence();
  uint32_t* exits = p.ws_counter + (size_t)p.batch * p.hkv;
  const uint32_t prev = atomicAdd(exits, 1u);
  if (prev != gridDim.x * gridDim.y * gridDim.z - 1) return;
  __threadfence();
  for (int b = 0; b < p.batch; ++b) {
    const int pos = __ldcg(p.ctx_lens + b);
    const int cap = (p.pages_per_seq ? p.pages_per_seq[b] : p.max_pages) * kPage;
    const bool accept = cap > 0 && ((pos >= 0 && pos < cap) || p.kv_update == RXLA_B200_KV_CLAMP);
    if (p.accepted) p.accepted[b] = accept ? 1 : 0;
    if (p.advance_ctx) p.ctx_lens[b] = pos + (accept ? 1 : 0);
  }
  *exits = 0u;
}

// SplitHalf RoPE of q in the mma B-fragment layout: lane (g, q4) holds dims
// ks*16 + 2*q4 + {0,1,8,9} of k-step ks; dim d pairs with d + 16*HS.
template <int KS, int HS>
__device__ __forceinline__ void rope_q(float (&qv)[KS][4], const float2* cs, int q4) {
#pragma unroll
  for (int ks = 0; ks < HS; ++ks)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int d = ks * 16 + 2 * q4 + (i & 1) + (i >> 1) * 8;
      const float2 t = cs[d];
      const float x0 = qv[ks][i], x1 = qv[ks + HS][i];
      qv[ks][i] = x0 * t.x - x1 * t.y;
      qv[ks + HS][i] = x1 * t.x + x0 * t.y;
    }
}

// The new k / v row of one kv head (lane holds dims DL·lane ..): k RMSNorm
// over the head (kw null: none), SplitHalf RoPE from the position table cs
// (the partner of dim d < rot/2 is d + rot/2, held by lane + rot/(2·DL)),
// both rounded to bf16 — the values the cache stores.
template <int DL>
__device__ __forceinline__ void prep_new_kv(float (&kn)[DL], float (&vn)[DL], int lane,
                                            const float* kw, const float2* cs, int rot,
                                            float eps) {
  constexpr int D = DL * 32;
  if (kw) {
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < DL; ++i) ss += kn[i] * kn[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float rs = 1.0f / sqrtf(ss / (float)D + eps);
#pragma unroll
    for (int i = 0; i < DL; ++i) kn[i] = (kn[i] * rs) * kw[DL * lane + i];
  }
  if (rot > 0) {
    const int half = rot / 2, off = half / DL;
#pragma unroll
    for (int i = 0; i < DL; ++i) {
      const int d = DL * lane + i;
      const float up = __shfl_sync(0xffffffffu, kn[i], (lane + off) & 31);
      const float dn = __shfl_sync(0xffffffffu, kn[i], (lane - off) & 31);
      if (d < half) {
        const float2 t = cs[d];
        kn[i] = kn[i] * t.x - up * t.y;
      } else if (d < rot) {
        const float2 t = cs[d - half];
        kn[i] = kn[i] * t.x + dn * t.y;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < DL; ++i) {
    kn[i] = bf16_round(kn[i]);
    vn[i] = bf16_round(vn[i]);
  }
}

constexpr int kComputeWarps = 4;

// Thread-block cluster helpers: a full cluster barrier (release / acquire),
// this CTA's rank, and loads from another CTA's shared memory at the address
// `p` has in this CTA.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t dsmem_addr(const void* p, int rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(p)), "r"(rank));
  return a;
}
__device__ __forceinline__ float ld_dsmem_f32(const float* p, int rank) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(dsmem_addr(p, rank)) : "memory");
  return v;
}
__device__ __forceinline__ float4 ld_dsmem_f32x4(const float* p, int rank) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(dsmem_addr(p, rank))
               : "memory");
  return v;
}
// Ring depth and occupancy: small batches (few CTAs, latency-bound) use a
// deep ring; large batches fit three CTAs per SM with a shallower ring.  The
// page iterations of a split go round-robin to the compute warps, so a stage
// is always consumed by the same warp only if the depth is a multiple of the
// warp count — otherwise a warp could wait on a stage barrier two phases
// ahead, where the parity test aliases.
constexpr int kStagesSmall = 8, kStagesLarge = 4;
constexpr int kMergeBatch = 16;  // split partials in flight per thread in the final merge

template <int D, int kStagesV2, int kMinBlocks, int CW = kComputeWarps, bool CLUSTER = false>
__global__ void __launch_bounds__((CW + 1) * 32, kMinBlocks)
    paged_decode_kernel(const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap, const Params p) {
  static_assert(kStagesV2 % CW == 0, "ring depth must be a multiple of the warps");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  constexpr int DL = D / 32;     // dims per lane for the new k / v and the merges
  constexpr int KS = D / 16;     // k-steps of q·kᵀ
  constexpr int kTile = kPage * D * 2;            // one page of one kv head, bytes
  constexpr int kStage = 2 * kTile;               // K + V
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw);
  uint64_t* empty = full + kStagesV2;
  float* misc = reinterpret_cast<float*>(empty + kStagesV2);  // 8 floats: flags
  float2* cs = reinterpret_cast<float2*>(misc + 8);               // [64] cos, sin
  float* qw = reinterpret_cast<float*>(cs + 64);                  // [D] q norm weight
  float* kw = qw + D;                                             // [D] k norm weight
  // the swizzled ring must start on a 1024-byte boundary, after the above
  // (barriers, flags, tables: at most 2048 bytes up to D = 128, 3072 for 256)
  constexpr uint32_t kHdr = D > 128 ? 3072u : 2048u;
  const uint32_t base_u32 = smem_u32(smem_raw);
  uint8_t* ring = smem_raw + ((1024u - (base_u32 & 1023u)) & 1023u) + kHdr;
  // per-warp softmax states for the in-CTA merge: O [warp][8][D], m/l [warp][8][2]
  float* st_o = reinterpret_cast<float*>(ring + kStagesV2 * kStage);
  float* st_ml = st_o + CW * 8 * D;
  float* wts = st_ml + CW * 8 * 2;  // cross-split maxima [max_splits][8]
  float* wls = wts + p.max_splits * 8;           // cross-split sums [max_splits][8]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hkv = p.hkv, G = p.group;

  if (!p.ctx_stable) pdl_wait();
  const int pos = p.ctx_lens[b];
  const int cap = (p.pages_per_seq ? p.pages_per_seq[b] : p.max_pages) * kPage;
  const int n_keys = pos < 0 ? 0 : min(pos + 1, cap);
  const int n_pages = (n_keys + kPage - 1) / kPage;
  const int n_splits = max(1, (n_pages + p.pps - 1) / p.pps);
  const int pg0 = split * p.pps;
  const int pg1 = min(n_pages, pg0 + p.pps);
  const int n_it = max(0, pg1 - pg0);
  const bool in_range = pos >= 0 && pos < cap;
  const bool accept = cap > 0 && (in_range || p.kv_update == RXLA_B200_KV_CLAMP);
  const int slot = pos < 0 ? 0 : (pos >= cap ? cap - 1 : pos);
  const bool owner = accept && split == (slot / kPage) / p.pps;

  const int cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  const int ctas = gridDim.x * gridDim.y * gridDim.z;
  // nothing of this sequence in this split (exit = trigger); a cluster's CTAs
  // all stay for the cluster barriers, with no pages
  if (!CLUSTER && split >= n_splits) {
    if (threadIdx.x == 0) {
      if (p.next.nseg > 0) l2_prefetch_share(p.next, cta, ctas);
      finish_cta(p);
    }
    return;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStagesV2; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    fence_mbarrier_init();
  }
  __syncthreads();

  if (warp == CW) {
    // ------------------------------------------------------------ producer
    // Pages hold rows appended by earlier kernels only (the new row is patched
    // in from registers); with a stable ctx_lens they are fetched before
    // griddepcontrol.wait.
    if (lane == 0) {
      for (int it = 0; it < n_it; ++it) {
        const int s = it % kStagesV2;
        if (it >= kStagesV2 && !mbar_wait(&empty[s], ((it / kStagesV2) - 1) & 1)) break;
        const int page = p.page_table[(int64_t)b * p.max_pages + pg0 + it];
        const int row = (page * hkv + h) * kPage;
        mbar_arrive_expect_tx(&full[s], (uint32_t)kStage);
        uint8_t* kdst = ring + (size_t)s * kStage;
#pragma unroll
        for (int j = 0; j < D / 64; ++j) {
          tma_load_2d(kdst + j * kPage * 128, &kmap, 64 * j, row, &full[s]);
          tma_load_2d(kdst + kTile + j * kPage * 128, &vmap, 64 * j, row, &full[s]);
        }
      }
      // pages are all requested: pull the next kernel's first bytes into L2
      if (p.next.nseg > 0) l2_prefetch_share(p.next, cta, ctas);
    }
  } else {
    // ------------------------------------------------------- compute warps
    const int tid = threadIdx.x;  // 0 .. 127
    // Position tables (cos, sin of pos·inv_freq) and the norm weights go to
    // shared memory first; with a stable ctx_lens this overlaps the previous
    // kernel.  The angle is f32(pos) · inv_freq in f32, as the oracle forms it.
    if (p.rot > 0 && tid < p.rot / 2) {
      const float ang = (float)pos * p.inv_freq[tid];
      cs[tid] = make_float2(cosf(ang), sinf(ang));
    }
    for (int i = tid; i < D; i += CW * 32) {
      if (p.q_norm_w) qw[i] = p.q_norm_w[i];
      if (p.k_norm_w) kw[i] = p.k_norm_w[i];
    }
    if (p.ctx_stable) pdl_wait();  // q / k_new / v_new come from the previous kernel
    // dependents wait for this grid's completion before reading its output
    if (tid == 0) pdl_launch_dependents();
    const int g = lane >> 2, q4 = lane & 3;

    // raw q (lane (g, q4) holds head g, dims ks*16 + 2*q4 + {0,1,8,9}) and,
    // in the warp that meets the slot's page, the new k / v: all loads first
    float qv[KS][4];
    const bool qvalid = g < G;
    {
      const __nv_bfloat16* qr =
          p.q + (int64_t)b * p.q_stride + (int64_t)(h * G + (qvalid ? g : 0)) * D;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        const int d0 = ks * 16 + 2 * q4;
        const __nv_bfloat162 x0 = *reinterpret_cast<const __nv_bfloat162*>(qr + d0);
        const __nv_bfloat162 x1 = *reinterpret_cast<const __nv_bfloat162*>(qr + d0 + 8);
        qv[ks][0] = qvalid ? __low2float(x0) : 0.0f;
        qv[ks][1] = qvalid ? __high2float(x0) : 0.0f;
        qv[ks][2] = qvalid ? __low2float(x1) : 0.0f;
        qv[ks][3] = qvalid ? __high2float(x1) : 0.0f;
      }
    }
    const int slot_pg = slot / kPage;
    const bool appender = owner && warp == (slot_pg - pg0) % CW;
    float kn[DL], vn[DL];
    if (appender) {
      const __nv_bfloat16* kr = p.k_new + (int64_t)b * p.kv_stride + (int64_t)h * D;
      const __nv_bfloat16* vr = p.v_new + (int64_t)b * p.kv_stride + (int64_t)h * D;
#pragma unroll
      for (int i = 0; i < DL; ++i) {
        kn[i] = __bfloat162float(kr[DL * lane + i]);
        vn[i] = __bfloat162float(vr[DL * lane + i]);
      }
    }
    asm volatile("bar.sync 1, %0;" ::"r"(CW * 32) : "memory");  // tables ready

    if (appender) {
      // k: RMSNorm over the head, RoPE, bf16; appended at the slot and patched
      // into this warp's tile of the slot's page below
      prep_new_kv<DL>(kn, vn, lane, p.k_norm_w ? kw : nullptr, cs, p.rot, p.eps);
      const int page = p.page_table[(int64_t)b * p.max_pages + slot_pg];
      const int64_t base = (((int64_t)page * hkv + h) * kPage + slot % kPage) * D + DL * lane;
#pragma unroll
      for (int i = 0; i < DL; ++i) {
        p.k_pages[base + i] = __float2bfloat16_rn(kn[i]);
        p.v_pages[base + i] = __float2bfloat16_rn(vn[i]);
      }
    }

    // q of the G heads of this kv head in B-fragment layout, normed, rotated
    // and split into bf16 hi + lo
    uint32_t qhi[KS][2], qlo[KS][2];
    {
      if (p.q_norm_w) {
        float ss = 0.0f;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks)
#pragma unroll
          for (int i = 0; i < 4; ++i) ss += qv[ks][i] * qv[ks][i];
        ss += __shfl_xor_sync(0xffffffffu, ss, 1);
        ss += __shfl_xor_sync(0xffffffffu, ss, 2);
        const float rs = 1.0f / sqrtf(ss / (float)D + p.eps);
#pragma unroll
        for (int ks = 0; ks < KS; ++ks)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int d = ks * 16 + 2 * q4 + (i & 1) + (i >> 1) * 8;
            qv[ks][i] = (qv[ks][i] * rs) * qw[d];
          }
      }
      // a RoPE pair (d, d + rot/2) is rot/32 k-steps apart; the distance is a
      // template argument so qv stays in registers
      switch (p.rot / 32) {
        case 1: rope_q<KS, 1>(qv, cs, q4); break;
        case 2: rope_q<KS, 2>(qv, cs, q4); break;
        case 3: if constexpr (KS >= 6) rope_q<KS, 3>(qv, cs, q4); break;
        case 4: if constexpr (KS >= 8) rope_q<KS, 4>(qv, cs, q4); break;
        default: break;
      }
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        const float h0 = bf16_round(qv[ks][0]), h1 = bf16_round(qv[ks][1]);
        const float h2 = bf16_round(qv[ks][2]), h3 = bf16_round(qv[ks][3]);
        qhi[ks][0] = pack_bf16x2(h0, h1);
        qhi[ks][1] = pack_bf16x2(h2, h3);
        qlo[ks][0] = pack_bf16x2(qv[ks][0] - h0, qv[ks][1] - h1);
        qlo[ks][1] = pack_bf16x2(qv[ks][2] - h2, qv[ks][3] - h3);
      }
    }
    const float scale = p.scale;

    // running softmax state of head columns 2*q4, 2*q4+1 over this warp's pages
    float m_run[2] = {-INFINITY, -INFINITY};
    float l_part[2] = {0.0f, 0.0f};
    float o[D / 16][4];
#pragma unroll
    for (int mt = 0; mt < D / 16; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) o[mt][i] = 0.0f;

    const int mi = lane >> 3, rr = lane & 7;
    for (int it = warp; it < n_it; it += CW) {
      const int s = it % kStagesV2;
      if (!mbar_wait(&full[s], (it / kStagesV2) & 1)) break;
      const int pg = pg0 + it;
      uint8_t* kt = ring + (size_t)s * kStage;
      uint8_t* vt = kt + kTile;
      if (appender && pg == slot_pg) {
        // patch the appended row into the loaded tile
        const int r = slot % kPage;
#pragma unroll
        for (int i = 0; i < DL; i += 2) {
          const int d = DL * lane + i;
          *reinterpret_cast<uint32_t*>(kt + swz(r, d, kPage)) = pack_bf16x2(kn[i], kn[i + 1]);
          *reinterpret_cast<uint32_t*>(vt + swz(r, d, kPage)) = pack_bf16x2(vn[i], vn[i + 1]);
        }
        __syncwarp();
      }
      // ---- S^T (16 tokens x 8 head columns) = K · Q^T
      float sc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      const uint32_t kbase = smem_u32(kt);
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        // matrices: (tok 0-7, d 0-7), (tok 8-15, d 0-7), (tok 0-7, d 8-15), (tok 8-15, d 8-15)
        uint32_t a[4];
        ldsm_x4(a, kbase + swz(rr + ((mi & 1) << 3), ks * 16 + ((mi >> 1) << 3), kPage));
        mma_bf16_16816(sc, a, qhi[ks][0], qhi[ks][1]);
        mma_bf16_16816(sc, a, qlo[ks][0], qlo[ks][1]);
      }
      // sc[0], sc[1]: token g, heads 2q4, 2q4+1; sc[2], sc[3]: token g+8
      const int t0 = pg * kPage + g, t1 = t0 + 8;
      float alpha[2], pv0[2], pv1[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float s0 = t0 < n_keys ? sc[j] * scale : -INFINITY;
        const float s1 = t1 < n_keys ? sc[2 + j] * scale : -INFINITY;
        float mt = fmaxf(s0, s1);
        mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 4));
        mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 8));
        mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 16));
        const float mn = fmaxf(m_run[j], mt);
        if (mn == -INFINITY) {
          alpha[j] = 1.0f;
          pv0[j] = 0.0f;
          pv1[j] = 0.0f;
        } else {
          alpha[j] = expf(m_run[j] - mn);
          pv0[j] = expf(s0 - mn);
          pv1[j] = expf(s1 - mn);
        }
        m_run[j] = mn;
        l_part[j] = l_part[j] * alpha[j] + pv0[j] + pv1[j];
      }
#pragma unroll
      for (int mt = 0; mt < D / 16; ++mt) {
        o[mt][0] *= alpha[0];
        o[mt][1] *= alpha[1];
        o[mt][2] *= alpha[0];
        o[mt][3] *= alpha[1];
      }
      // P^T (tokens x heads) -> B fragments of O^T += V^T · P^T; P = hi + lo
      // in bf16 keeps the f32 softmax weights (the reference's F32 attention)
      const float h00 = bf16_round(pv0[0]), h01 = bf16_round(pv0[1]);
      const float h10 = bf16_round(pv1[0]), h11 = bf16_round(pv1[1]);
      const uint32_t b0 = movmatrix_t(pack_bf16x2(h00, h01));
      const uint32_t b1 = movmatrix_t(pack_bf16x2(h10, h11));
      const uint32_t c0 = movmatrix_t(pack_bf16x2(pv0[0] - h00, pv0[1] - h01));
      const uint32_t c1 = movmatrix_t(pack_bf16x2(pv1[0] - h10, pv1[1] - h11));
      const uint32_t vbase = smem_u32(vt);
#pragma unroll
      for (int mt = 0; mt < D / 16; ++mt) {
        // A = V^T (16 dims x 16 tokens): (d 0-7,t 0-7), (d 8-15,t 0-7), (d 0-7,t 8-15), (d 8-15,t 8-15)
        uint32_t a[4];
        ldsm_x4_t(a, vbase + swz(rr + ((mi >> 1) << 3), mt * 16 + ((mi & 1) << 3), kPage));
        mma_bf16_16816(o[mt], a, b0, b1);
        mma_bf16_16816(o[mt], a, c0, c1);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }

    // ---- this warp's state -> shared memory (head column j = 2*q4 + jj)
    {
      float* wo = st_o + (size_t)warp * 8 * D;
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        float l = l_part[jj];
        l += __shfl_xor_sync(0xffffffffu, l, 4);
        l += __shfl_xor_sync(0xffffffffu, l, 8);
        l += __shfl_xor_sync(0xffffffffu, l, 16);
        const int j = 2 * q4 + jj;
#pragma unroll
        for (int mt = 0; mt < D / 16; ++mt) {
          wo[j * D + mt * 16 + g] = o[mt][jj];
          wo[j * D + mt * 16 + g + 8] = o[mt][2 + jj];
        }
        if (g == 0) {
          st_ml[(warp * 8 + j) * 2] = m_run[jj];
          st_ml[(warp * 8 + j) * 2 + 1] = l;
        }
      }
    }
    asm volatile("bar.sync 1, %0;" ::"r"(CW * 32) : "memory");

    // ---- merge the 4 warps (in-CTA) -> this split's (O, m, l) per head;
    // a thread takes 4 consecutive dims of one head
    const int64_t seg = (((int64_t)b * hkv + h) * p.max_splits + split) * G;
    for (int e = tid; e < G * D / 4; e += CW * 32) {
      const int j = (4 * e) / D, d = (4 * e) % D;
      float m = -INFINITY;
#pragma unroll
      for (int w2 = 0; w2 < CW; ++w2) m = fmaxf(m, st_ml[(w2 * 8 + j) * 2]);
      float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      float l = 0.0f;
#pragma unroll
      for (int w2 = 0; w2 < CW; ++w2) {
        const float mw = st_ml[(w2 * 8 + j) * 2];
        const float wgt = mw == -INFINITY ? 0.0f : expf(mw - m);
        const float4 x = *reinterpret_cast<const float4*>(st_o + ((size_t)w2 * 8 + j) * D + d);
        acc.x += wgt * x.x;
        acc.y += wgt * x.y;
        acc.z += wgt * x.z;
        acc.w += wgt * x.w;
        l += wgt * st_ml[(w2 * 8 + j) * 2 + 1];
      }
      if (CLUSTER) {
        // this split's partial stays in shared memory for the cluster's
        // leader: O over warp slot 0 (only this thread reads these four
        // floats of every slot), (m, l) in the cross-split area
        *reinterpret_cast<float4*>(st_o + (size_t)j * D + d) = acc;
        if (d == 0) {
          wts[j * 2] = m;
          wts[j * 2 + 1] = l;
        }
      } else if (n_splits == 1) {
        const float inv = l > 0.0f ? 1.0f / l : 0.0f;
        uint2 pk;
        pk.x = pack_bf16x2(acc.x * inv, acc.y * inv);
        pk.y = pack_bf16x2(acc.z * inv, acc.w * inv);
        *reinterpret_cast<uint2*>(p.out + (int64_t)b * p.hq * D + (int64_t)(h * G + j) * D + d) = pk;
      } else {
        *reinterpret_cast<float4*>(p.ws_o + (seg + j) * D + d) = acc;
        if (d == 0) *reinterpret_cast<float2*>(p.ws_ml + (seg + j) * 2) = make_float2(m, l);
      }
    }
    if (!CLUSTER && n_splits > 1) {
      __threadfence();
      asm volatile("bar.sync 1, %0;" ::"r"(CW * 32) : "memory");
      if (tid == 0) {
        const uint32_t prev = atomicAdd(&p.ws_counter[b * hkv + h], 1u);
        misc[0] = prev == (uint32_t)(n_splits - 1) ? 1.0f : 0.0f;
      }
      asm volatile("bar.sync 1, %0;" ::"r"(CW * 32) : "memory");
      if (misc[0] != 0.0f) {
        // the last split of (b, h) merges all splits' partials: (m, l) of
        // every split in one round of loads, then up to 8 partial rows in flight
        __threadfence();
        const int64_t base = ((int64_t)b * hkv + h) * p.max_splits * G;
        for (int e = tid; e < n_splits * G; e += CW * 32) {
          const int sp = e / G, j = e % G;
          const float2 ml =
              __ldcg(reinterpret_cast<const float2*>(p.ws_ml + (base + (int64_t)sp * G + j) * 2));
          wts[sp * 8 + j] = ml.x;
          wls[sp * 8 + j] = ml.y;
        }
        asm volatile("bar.sync 1, %0;" ::"r"(CW * 32) : "memory");
        for (int e = tid; e < G * D / 4; e += CW * 32) {
          const int j = (4 * e) / D, d = (4 * e) % D;
          float m = -INFINITY;
          for (int sp = 0; sp < n_splits; ++sp) m = fmaxf(m, wts[sp * 8 + j]);
          float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          float l = 0.0f;
          for (int sp0 = 0; sp0 < n_splits; sp0 += kMergeBatch) {
            float4 x[kMergeBatch];
#pragma unroll
            for (int u = 0; u < kMergeBatch; ++u)
              if (sp0 + u < n_splits)
                x[u] = __ldcg(reinterpret_cast<const float4*>(
                    p.ws_o + (base + (int64_t)(sp0 + u) * G + j) * D + d));
#pragma unroll
            for (int u = 0; u < kMergeBatch; ++u) {
              if (sp0 + u < n_splits) {
                const float mw = wts[(sp0 + u) * 8 + j];
                const float wgt = mw == -INFINITY ? 0.0f : expf(mw - m);
                acc.x += wgt * x[u].x;
                acc.y += wgt * x[u].y;
                acc.z += wgt * x[u].z;
                acc.w += wgt * x[u].w;
                l += wgt * wls[(sp0 + u) * 8 + j];
              }
            }
          }
          const float inv = l > 0.0f ? 1.0f / l : 0.0f;
          uint2 pk;
          pk.x = pack_bf16x2(acc.x * inv, acc.y * inv);
          pk.y = pack_bf16x2(acc.z * inv, acc.w * inv);
          *reinterpret_cast<uint2*>(p.out + (int64_t)b * p.hq * D + (int64_t)(h * G + j) * D + d) =
              pk;
        }
        if (tid == 0) p.ws_counter[b * hkv + h] = 0u;
      }
    }
  }
  __syncthreads();
  if constexpr (CLUSTER) {
    // The cluster is the (sequence, kv head): CTA rank r holds split r.  Once
    // every CTA's partial is in its shared memory, rank 0 merges them through
    // distributed shared memory with log-sum-exp weights (splits in order)
    // and writes the output; the second barrier keeps every CTA's shared
    // memory alive until the leader has read it.  Every thread of every CTA
    // reaches both barriers (no early exit in this variant).
    cluster_sync();
    if (cluster_rank() == 0 && warp < CW) {
      const int tid = threadIdx.x;
      const int ns = min(n_splits, (int)gridDim.x);
      for (int e = tid; e < G * D / 4; e += CW * 32) {
        const int j = (4 * e) / D, d = (4 * e) % D;
        float mr[8], lr[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          mr[r] = -INFINITY;
          lr[r] = 0.0f;
          if (r < ns) {
            mr[r] = ld_dsmem_f32(wts + j * 2, r);
            lr[r] = ld_dsmem_f32(wts + j * 2 + 1, r);
          }
        }
        float m = -INFINITY;
#pragma unroll
        for (int r = 0; r < 8; ++r) m = fmaxf(m, mr[r]);
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        float l = 0.0f;
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          if (r < ns && mr[r] != -INFINITY) {
            const float wgt = expf(mr[r] - m);
            const float4 x = ld_dsmem_f32x4(st_o + (size_t)j * D + d, r);
            acc.x += wgt * x.x;
            acc.y += wgt * x.y;
            acc.z += wgt * x.z;
            acc.w += wgt * x.w;
            l += wgt * lr[r];
          }
        }
        const float inv = l > 0.0f ? 1.0f / l : 0.0f;
        uint2 pk;
        pk.x = pack_bf16x2(acc.x * inv, acc.y * inv);
        pk.y = pack_bf16x2(acc.z * inv, acc.w * inv);
        *reinterpret_cast<uint2*>(p.out + (int64_t)b * p.hq * D + (int64_t)(h * G + j) * D + d) = pk;
      }
    }
    cluster_sync();
  }
  if (threadIdx.x == 0) finish_cta(p);
}

// The new K/V rows of a batch without the attention (the decoder's prefill
// appends all rows of a prompt chunk before any row attends): block = row,
// warp = kv head; positions, slots, normalisation, rotation and rounding as
// paged_decode_kernel's append.
template <int D>
__global__ void __launch_bounds__(256) append_rows_kernel(const Params p) {
  constexpr int DL = D / 32;
  __shared__ float2 cs[64];
  __shared__ float kw[128];
  const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31;
  pdl_wait();  // k_new / v_new come from the previous kernel
  if (tid == 0) pdl_launch_dependents();
  const int pos = p.ctx_lens[b];
  const int cap = (p.pages_per_seq ? p.pages_per_seq[b] : p.max_pages) * kPage;
  const bool accept = cap > 0 && ((pos >= 0 && pos < cap) || p.kv_update == RXLA_B200_KV_CLAMP);
  const int slot = pos < 0 ? 0 : (pos >= cap ? cap - 1 : pos);
  if (p.rot > 0 && tid < p.rot / 2) {
    const float ang = (float)pos * p.inv_freq[tid];
    cs[tid] = make_float2(cosf(ang), sinf(ang));
  }
  if (p.k_norm_w && tid < D) kw[tid] = p.k_norm_w[tid];
  __syncthreads();
  if (!accept) return;
  for (int h = tid >> 5; h < p.hkv; h += blockDim.x >> 5) {
    const __nv_bfloat16* kr = p.k_new + (int64_t)b * p.kv_stride + (int64_t)h * D;
    const __nv_bfloat16* vr = p.v_new + (int64_t)b * p.kv_stride + (int64_t)h * D;
    float kn[DL], vn[DL];
#pragma unroll
    for (int i = 0; i < DL; ++i) {
      kn[i] = __bfloat162float(kr[DL * lane + i]);
      vn[i] = __bfloat162float(vr[DL * lane + i]);
    }
    prep_new_kv<DL>(kn, vn, lane, p.k_norm_w ? kw : nullptr, cs, p.rot, p.eps);
    const int page = p.page_table[(int64_t)b * p.max_pages + slot / kPage];
    const int64_t base = (((int64_t)page * p.hkv + h) * kPage + slot % kPage) * D + DL * lane;
#pragma unroll
    for (int i = 0; i < DL; ++i) {
      p.k_pages[base + i] = __float2bfloat16_rn(kn[i]);
      p.v_pages[base + i] = __float2bfloat16_rn(vn[i]);
    }
  }
}

// ------------------------------------------------ prefill (causal) attention
//
// The rows of a prompt chunk of one sequence after their K/V were appended
// (the append-only pass of paged_decode_kernel): row t holds the query at
// position pos[t] and attends over keys 0 .. pos[t] of the sequence's pages —
// the causal mask of the reference's full-sequence forward
// (crates/rxla-models/src/qwen3_5/mod.rs:229 with the SDPA of
// crates/rxla-core/src/attention.rs:83-252).  Same numerics as the decode
// kernel: q normed, rotated and split into bf16 hi + lo, the softmax weights
// split likewise, f32 accumulation.
//
// CTA = (block of kPfRows / G queries, kv head).  Its kPfRows (query, head)
// rows are the MMA M side — eight warps of 16 rows, row r is query r / G and
// head r % G — with q held as A fragments in registers.  The key pages
// 0 .. (the block's last position) stream through a ring (TMA, the decode
// kernel's [64 dims × 16 rows] swizzled boxes) that lane 0 of warp 0 keeps
// filled — no separate producer warp, so with 8 warps per CTA a thread may
// hold up to 255 registers — and every warp consumes every page, two per
// iteration: S = Q·Kᵀ (four 8-key n-blocks, K by ldmatrix), an online
// softmax per row, O += P·V with P taken from the S accumulators (the m16n8
// C fragment is the next MMA's A fragment) and V by ldmatrix.trans.  Pages
// above a warp's last position are skipped; the heaviest query blocks are
// scheduled first.
constexpr int kPfWarps = 8;
constexpr int kPfRows = kPfWarps * 16;
constexpr int kPfStages = 8;

struct PrefillParams {
  const __nv_bfloat16* q;
  int64_t q_stride;
  const float* q_norm_w;
  float eps;
  const float* inv_freq;
  int32_t rot;
  float scale;
  const int32_t* page_table;  // the sequence's pages
  const int32_t* pos;         // [n] position of each row (increasing)
  int32_t n, hq, hkv, group, bq;
  __nv_bfloat16* out;         // [n, hq, D]
};

// RoPE of one q row in the A-fragment layout at position pos: the angles are
// f32(pos) · inv_freq as paged_decode_kernel forms its table.
template <int KS, int HS>
__device__ __forceinline__ void rope_q_at(float (&qv)[KS][4], int pos, const float* inv_freq,
                                          int q4) {
#pragma unroll
  for (int ks = 0; ks < HS; ++ks)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int d = ks * 16 + 2 * q4 + (i & 1) + (i >> 1) * 8;
      const float ang = (float)pos * inv_freq[d];
      const float c = cosf(ang), sn = sinf(ang);
      const float x0 = qv[ks][i], x1 = qv[ks + HS][i];
      qv[ks][i] = x0 * c - x1 * sn;
      qv[ks + HS][i] = x1 * c + x0 * sn;
    }
}

template <int D>
__global__ void __launch_bounds__(kPfWarps * 32, 1)
    prefill_attention_kernel(const __grid_constant__ CUtensorMap kmap,
                             const __grid_constant__ CUtensorMap vmap, const PrefillParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  constexpr int KS = D / 16;
  constexpr int kTile = kPage * D * 2;
  constexpr int kStage = 2 * kTile;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw);
  uint64_t* empty = full + kPfStages;
  const uint32_t base_u32 = smem_u32(smem_raw);
  uint8_t* ring = smem_raw + ((1024u - (base_u32 & 1023u)) & 1023u) + 1024;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int blk = gridDim.x - 1 - blockIdx.x, h = blockIdx.y;
  const int G = p.group;
  const int t_begin = blk * p.bq;
  const int t_last = min(p.n, t_begin + p.bq) - 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPfStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kPfWarps);
    }
    fence_mbarrier_init();
  }
  __syncthreads();
  // the pages were written by the append pass, q by the qkv linear
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();
  const int n_keys = p.pos[t_last] + 1;
  const int n_pages = (n_keys + kPage - 1) / kPage;

  // page pg -> ring stage pg % kPfStages (K then V); issued by lane 0 of
  // warp 0: the first kPfStages pages now, page pg + kPfStages once every
  // warp has released page pg
  auto issue = [&](int pg) {
    const int s = pg % kPfStages;
    const int row = (p.page_table[pg] * p.hkv + h) * kPage;
    mbar_arrive_expect_tx(&full[s], (uint32_t)kStage);
    uint8_t* kdst = ring + (size_t)s * kStage;
#pragma unroll
    for (int j = 0; j < D / 64; ++j) {
      tma_load_2d(kdst + j * kPage * 128, &kmap, 64 * j, row, &full[s]);
      tma_load_2d(kdst + kTile + j * kPage * 128, &vmap, 64 * j, row, &full[s]);
    }
  };
  if (threadIdx.x == 0)
    for (int pg = 0; pg < min(n_pages, kPfStages); ++pg) issue(pg);
  bool ring_ok = true;  // lane 0 of warp 0: a refill wait has not timed out

  const int g = lane >> 2, q4 = lane & 3;
  // this thread's rows g and g + 8 of the warp: (query, head), position, q
  int pos_r[2];
  float qv[2][KS][4];
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int r = warp * 16 + g + 8 * rr;
    const int qi = r / G, j = r % G, t = t_begin + qi;
    const bool valid = qi < p.bq && t <= t_last;
    pos_r[rr] = valid ? p.pos[t] : -1;  // -1: every key masked, nothing stored
    const __nv_bfloat16* qr =
        p.q + (int64_t)(valid ? t : t_begin) * p.q_stride + (int64_t)(h * G + j) * D;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      const int d0 = ks * 16 + 2 * q4;
      const __nv_bfloat162 x0 = *reinterpret_cast<const __nv_bfloat162*>(qr + d0);
      const __nv_bfloat162 x1 = *reinterpret_cast<const __nv_bfloat162*>(qr + d0 + 8);
      qv[rr][ks][0] = __low2float(x0);
      qv[rr][ks][1] = __high2float(x0);
      qv[rr][ks][2] = __low2float(x1);
      qv[rr][ks][3] = __high2float(x1);
    }
    if (p.q_norm_w) {
      float ss = 0.0f;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks)
#pragma unroll
        for (int i = 0; i < 4; ++i) ss += qv[rr][ks][i] * qv[rr][ks][i];
      ss += __shfl_xor_sync(0xffffffffu, ss, 1);
      ss += __shfl_xor_sync(0xffffffffu, ss, 2);
      const float rs = 1.0f / sqrtf(ss / (float)D + p.eps);
#pragma unroll
      for (int ks = 0; ks < KS; ++ks)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int d = ks * 16 + 2 * q4 + (i & 1) + (i >> 1) * 8;
          qv[rr][ks][i] = (qv[rr][ks][i] * rs) * __ldg(p.q_norm_w + d);
        }
    }
    switch (p.rot / 32) {
      case 1: rope_q_at<KS, 1>(qv[rr], pos_r[rr], p.inv_freq, q4); break;
      case 2: rope_q_at<KS, 2>(qv[rr], pos_r[rr], p.inv_freq, q4); break;
      case 3: if constexpr (KS >= 6) rope_q_at<KS, 3>(qv[rr], pos_r[rr], p.inv_freq, q4); break;
      case 4: if constexpr (KS >= 8) rope_q_at<KS, 4>(qv[rr], pos_r[rr], p.inv_freq, q4); break;
      default: break;
    }
  }
  // A fragments: {row g dims 2q4..+1, row g+8 dims 2q4..+1, row g dims +8..9, row g+8 dims +8..9}
  uint32_t qhi[KS][4], qlo[KS][4];
#pragma unroll
  for (int ks = 0; ks < KS; ++ks)
#pragma unroll
    for (int rr = 0; rr < 2; ++rr)
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const float x0 = qv[rr][ks][2 * half], x1 = qv[rr][ks][2 * half + 1];
        const float h0 = bf16_round(x0), h1 = bf16_round(x1);
        qhi[ks][rr + 2 * half] = pack_bf16x2(h0, h1);
        qlo[ks][rr + 2 * half] = pack_bf16x2(x0 - h0, x1 - h1);
      }
  int wmax = max(pos_r[0], pos_r[1]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) wmax = max(wmax, __shfl_xor_sync(0xffffffffu, wmax, o));
  const float scale = p.scale;

  float m_run[2] = {-INFINITY, -INFINITY};
  float l_part[2] = {0.0f, 0.0f};
  float o[D / 8][4];
#pragma unroll
  for (int nd = 0; nd < D / 8; ++nd)
#pragma unroll
    for (int i = 0; i < 4; ++i) o[nd][i] = 0.0f;

  const int mi = lane >> 3, r8 = lane & 7;
  // two pages (32 keys) per iteration: twice the independent MMA chains in
  // S = Q·Kᵀ and one softmax rescale per 32 keys
  for (int it = 0; it < n_pages; it += 2) {
    if (threadIdx.x == 0 && it > 0 && ring_ok) {
      // refill the stages of the previous iteration's pages
      for (int pg = it - 2; pg < it; ++pg) {
        if (pg + kPfStages >= n_pages) break;
        if (!mbar_wait(&empty[pg % kPfStages], (pg / kPfStages) & 1)) {
          ring_ok = false;
          break;
        }
        issue(pg + kPfStages);
      }
    }
    __syncwarp();
    const int s0 = it % kPfStages, s1 = (it + 1) % kPfStages;
    const bool two = it + 1 < n_pages;
    if (!mbar_wait(&full[s0], (it / kPfStages) & 1)) break;
    if (two && !mbar_wait(&full[s1], ((it + 1) / kPfStages) & 1)) break;
    const int kb = it * kPage;
    if (kb <= wmax) {
      const uint32_t kbase[2] = {smem_u32(ring + (size_t)s0 * kStage),
                                 smem_u32(ring + (size_t)s1 * kStage)};
      // ---- S (16 rows × 32 keys) = Q · Kᵀ, hi and lo in separate chains
      float sc[4][4], sl[4][4];
#pragma unroll
      for (int nb = 0; nb < 4; ++nb)
#pragma unroll
        for (int i = 0; i < 4; ++i) sc[nb][i] = sl[nb][i] = 0.0f;
#pragma unroll
      for (int pg = 0; pg < 2; ++pg) {
        if (pg == 1 && !two) break;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
          // matrices: (keys 0-7, d 0-7), (keys 0-7, d 8-15), (keys 8-15, d 0-7), (keys 8-15, d 8-15)
          uint32_t b[4];
          ldsm_x4(b, kbase[pg] + swz(r8 + ((mi >> 1) << 3), ks * 16 + ((mi & 1) << 3), kPage));
          mma_bf16_16816(sc[2 * pg], qhi[ks], b[0], b[1]);
          mma_bf16_16816(sl[2 * pg], qlo[ks], b[0], b[1]);
          mma_bf16_16816(sc[2 * pg + 1], qhi[ks], b[2], b[3]);
          mma_bf16_16816(sl[2 * pg + 1], qlo[ks], b[2], b[3]);
        }
      }
      // sc[nb][2*rr + e]: row g + 8*rr, key kb + nb*8 + 2*q4 + e (keys of an
      // absent second page lie past every row's position)
      float pv[2][8], alpha[2];
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        float sv[8];
        float mt = -INFINITY;
#pragma unroll
        for (int nb = 0; nb < 4; ++nb)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int key = kb + nb * 8 + 2 * q4 + e;
            const float v = sc[nb][2 * rr + e] + sl[nb][2 * rr + e];
            sv[2 * nb + e] = key <= pos_r[rr] ? v * scale : -INFINITY;
            mt = fmaxf(mt, sv[2 * nb + e]);
          }
        mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
        mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
        const float mn = fmaxf(m_run[rr], mt);
        float sum = 0.0f;
        if (mn == -INFINITY) {
          alpha[rr] = 1.0f;
#pragma unroll
          for (int i = 0; i < 8; ++i) pv[rr][i] = 0.0f;
        } else {
          alpha[rr] = expf(m_run[rr] - mn);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            pv[rr][i] = expf(sv[i] - mn);
            sum += pv[rr][i];
          }
        }
        m_run[rr] = mn;
        l_part[rr] = l_part[rr] * alpha[rr] + sum;
      }
#pragma unroll
      for (int nd = 0; nd < D / 8; ++nd) {
        o[nd][0] *= alpha[0];
        o[nd][1] *= alpha[0];
        o[nd][2] *= alpha[1];
        o[nd][3] *= alpha[1];
      }
      // P as A fragments per page: {row g keys 2q4..+1, row g+8 keys 2q4..+1,
      // row g keys 8+2q4.., row g+8 keys 8+2q4..}, split into bf16 hi + lo
      uint32_t ph[2][4], pl[2][4];
#pragma unroll
      for (int pg = 0; pg < 2; ++pg)
#pragma unroll
        for (int nb = 0; nb < 2; ++nb)
#pragma unroll
          for (int rr = 0; rr < 2; ++rr) {
            const float x0 = pv[rr][4 * pg + 2 * nb], x1 = pv[rr][4 * pg + 2 * nb + 1];
            const float h0 = bf16_round(x0), h1 = bf16_round(x1);
            ph[pg][2 * nb + rr] = pack_bf16x2(h0, h1);
            pl[pg][2 * nb + rr] = pack_bf16x2(x0 - h0, x1 - h1);
          }
      // ---- O += P · V: V (keys × dims) by ldmatrix.trans
#pragma unroll
      for (int pg = 0; pg < 2; ++pg) {
        if (pg == 1 && !two) break;
        const uint32_t vbase = kbase[pg] + kTile;
#pragma unroll
        for (int n2 = 0; n2 < D / 16; ++n2) {
          // matrices: (keys 0-7, d 0-7), (keys 8-15, d 0-7), (keys 0-7, d 8-15), (keys 8-15, d 8-15)
          uint32_t b[4];
          ldsm_x4_t(b, vbase + swz(r8 + ((mi & 1) << 3), n2 * 16 + ((mi >> 1) << 3), kPage));
          mma_bf16_16816(o[2 * n2], ph[pg], b[0], b[1]);
          mma_bf16_16816(o[2 * n2], pl[pg], b[0], b[1]);
          mma_bf16_16816(o[2 * n2 + 1], ph[pg], b[2], b[3]);
          mma_bf16_16816(o[2 * n2 + 1], pl[pg], b[2], b[3]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(&empty[s0]);
      if (two) mbar_arrive(&empty[s1]);
    }
  }

  // ---- normalise and store: o[nd][2*rr + e] = O[row g + 8*rr][nd*8 + 2*q4 + e]
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    float l = l_part[rr];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    if (pos_r[rr] < 0) continue;
    const float inv = l > 0.0f ? 1.0f / l : 0.0f;
    const int r = warp * 16 + g + 8 * rr;
    const int t = t_begin + r / G, j = r % G;
    __nv_bfloat16* orow = p.out + (int64_t)t * p.hq * D + (int64_t)(h * G + j) * D + 2 * q4;
#pragma unroll
    for (int nd = 0; nd < D / 8; ++nd)
      *reinterpret_cast<uint32_t*>(orow + nd * 8) =
          pack_bf16x2(o[nd][2 * rr] * inv, o[nd][2 * rr + 1] * inv);
  }
}

// ---------------------------------------------------------- host helpers

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

static int32_t make_page_map(CUtensorMap* map, void* base, int64_t num_pages, int hkv, int d) {
  auto fn = encode_fn();
  if (!fn) return fail(RXLA_B200_UNAVAILABLE, "cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t dims[2] = {(cuuint64_t)d, (cuuint64_t)(num_pages * hkv * kPage)};
  const cuuint64_t strides[1] = {(cuuint64_t)d * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)kPage};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(RXLA_B200_INVALID_ARGUMENT, "page tensor map encoding failed");
  return RXLA_B200_OK;
}

// Pages per split: CTAs are (sequence, kv head, split): enough CTAs for ~4
// per SM over all (sequence, kv head) pairs, at least ceil(pages / 16) pages
// (at most 16 splits per sequence and head; batch 1 at 2048 context: 9.8 µs
// with 16, 11.2 with 32, 16.9 with 48 — the last CTA merges every split), at
// most 48 (longer splits cost a fuller last wave but fewer merges; batch 64
// at 2048 context: 111.4 µs with 32, 105.8 with 48, 109.7 with 64).
// Small grids — fewer than 16 sequences and at most 32 (sequence, kv head)
// pairs — run one thread-block cluster of kClusterSplits CTAs per pair, each
// with kClusterWarps compute warps, and merge the splits through distributed
// shared memory instead of a workspace round trip (head_dim up to 128: the
// cluster variant's 16-stage ring of 256-dim pages would not fit).
constexpr int kClusterSplits = 8, kClusterWarps = 8, kStagesCluster = 16;
static bool use_cluster(int batch, int kv_heads, int head_dim) {
  return head_dim <= 128 && batch < 16 && (int64_t)batch * kv_heads <= 32;
}

static int pages_per_split(int batch, int kv_heads, int max_pages, int head_dim) {
  if (use_cluster(batch, kv_heads, head_dim))
    return std::max(1, (max_pages + kClusterSplits - 1) / kClusterSplits);
  constexpr int64_t cap = 48;   // pages per split at most
  constexpr int64_t most = 16;  // splits per (sequence, kv head) at most
  const int64_t want = ((int64_t)batch * kv_heads * max_pages + 4 * 148 - 1) / (4 * 148);
  const int64_t depth = ((int64_t)max_pages + most - 1) / most;
  return (int)std::max<int64_t>(1, std::max(depth, std::min<int64_t>(cap, want)));
}

}  // namespace attn
}  // namespace rxla

extern "C" int32_t rxla_b200_paged_decode_workspace_size(int32_t batch, int32_t q_heads,
                                                         int32_t kv_heads, int32_t head_dim,
                                                         int32_t max_context, size_t* bytes) {
  using namespace rxla;
  RXLA_REQUIRE(bytes && batch >= 0 && kv_heads > 0 && q_heads > 0 && q_heads % kv_heads == 0 &&
                   head_dim > 0 && max_context >= 0,
               "paged_decode_workspace_size: bad arguments");
  const int max_pages = (max_context + attn::kPage - 1) / attn::kPage;
  const int pps = attn::pages_per_split(batch, kv_heads, max_pages, head_dim);
  const int64_t splits = attn::use_cluster(batch, kv_heads, head_dim)
                             ? attn::kClusterSplits
                             : std::max(1, (max_pages + pps - 1) / pps);
  const int64_t G = q_heads / kv_heads;
  const int64_t part = (int64_t)batch * kv_heads * splits * G;
  const int64_t counters = ((int64_t)batch * kv_heads + 1) * 4;
  *bytes = (size_t)((counters + 255) / 256 * 256 + part * head_dim * 4 + part * 2 * 4);
  return RXLA_B200_OK;
}

namespace rxla {
namespace attn {
// Validate, plan and launch.  `ctx_stable`: no kernel between the last write
// of ctx_lens and this one may still be running, so pages can be fetched
// before griddepcontrol.wait (the decoder runner advances ctx_lens only at
// the end of a step).  `append_only`: write the new K/V rows and nothing else
// (append_rows_kernel).
int32_t launch(const rxla_b200_paged_decode_args* a, cudaStream_t s_in, bool ctx_stable,
               const L2Prefetch* next, bool append_only) {
  RXLA_REQUIRE(a && a->struct_size >= sizeof(rxla_b200_paged_decode_args),
               "paged_decode: args struct missing or too small");
  const int D = a->head_dim;
  RXLA_REQUIRE(a->batch >= 0 && a->kv_heads > 0 && a->q_heads > 0 &&
                   a->q_heads % a->kv_heads == 0,
               "paged_decode: query heads must be a positive multiple of kv heads (attention.rs:99-112)");
  RXLA_REQUIRE(a->q_heads / a->kv_heads <= 8, "paged_decode: at most 8 query heads per kv head");
  RXLA_REQUIRE(a->kv_heads <= 65535 && a->batch <= 65535,
               "paged_decode: kv_heads and batch must be <= 65535 (grid dimensions)");
  RXLA_REQUIRE(D == 64 || D == 128 || (D == 256 && !append_only),
               "paged_decode: head_dim must be 64 or 128 (or 256 for the decode step)");
  RXLA_REQUIRE(D != 256 || a->inv_freq == nullptr || a->rotary_dim <= 128,
               "paged_decode: rotary_dim must be <= 128 at head_dim 256");
  RXLA_REQUIRE(a->page_size == attn::kPage, "paged_decode: page_size must be 16");
  RXLA_REQUIRE(a->rotary_dim == 0 || a->inv_freq == nullptr ||
                   (a->rotary_dim % 32 == 0 && a->rotary_dim <= D),
               "paged_decode: rotary_dim must be a multiple of 32 and <= head_dim");
  RXLA_REQUIRE(a->kv_update == RXLA_B200_KV_CLAMP || a->kv_update == RXLA_B200_KV_CHECKED,
               "paged_decode: unknown kv_update");
  RXLA_REQUIRE(a->max_pages_per_seq > 0 && a->num_pages > 0, "paged_decode: empty cache");
  RXLA_REQUIRE(a->scale == 0.0f || std::isfinite(a->scale), "paged_decode: scale must be finite (attention.rs:191)");
  RXLA_REQUIRE(a->max_context > 0 && a->max_context <= a->max_pages_per_seq * attn::kPage,
               "paged_decode: max_context must be in [1, max_pages_per_seq * 16]");
  RXLA_REQUIRE((reinterpret_cast<uintptr_t>(a->k_pages) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(a->v_pages) % 16 == 0),
               "paged_decode: cache pages must be 16-byte aligned");
  RXLA_REQUIRE(a->q_row_stride % 2 == 0 && a->kv_row_stride % 2 == 0 &&
                   (reinterpret_cast<uintptr_t>(a->q) % 4 == 0),
               "paged_decode: q / kv rows must be 4-byte aligned");
  RXLA_REQUIRE(reinterpret_cast<uintptr_t>(a->out) % 8 == 0,
               "paged_decode: out must be 8-byte aligned");
  if (a->batch == 0) return RXLA_B200_OK;
  RXLA_REQUIRE(a->q && a->k_new && a->v_new && a->k_pages && a->v_pages && a->page_table &&
                   a->ctx_lens && a->out,
               "paged_decode: null pointer");
  size_t need = 0;
  rxla_b200_paged_decode_workspace_size(a->batch, a->q_heads, a->kv_heads, D, a->max_context,
                                        &need);
  RXLA_REQUIRE(a->workspace && a->workspace_bytes >= need,
               "paged_decode: workspace missing or smaller than paged_decode_workspace_size");

  attn::Params p{};
  p.q = reinterpret_cast<const __nv_bfloat16*>(a->q);
  p.k_new = reinterpret_cast<const __nv_bfloat16*>(a->k_new);
  p.v_new = reinterpret_cast<const __nv_bfloat16*>(a->v_new);
  p.q_stride = a->q_row_stride;
  p.kv_stride = a->kv_row_stride;
  p.q_norm_w = a->q_norm_weight;
  p.k_norm_w = a->k_norm_weight;
  p.eps = a->norm_eps;
  p.inv_freq = a->inv_freq;
  p.rot = a->inv_freq ? a->rotary_dim : 0;
  p.scale = a->scale == 0.0f ? 1.0f / std::sqrt((float)D) : a->scale;
  p.k_pages = reinterpret_cast<__nv_bfloat16*>(a->k_pages);
  p.v_pages = reinterpret_cast<__nv_bfloat16*>(a->v_pages);
  p.page_table = a->page_table;
  p.pages_per_seq = a->pages_per_seq;
  p.max_pages = a->max_pages_per_seq;
  p.ctx_lens = const_cast<int32_t*>(a->ctx_lens);
  p.kv_update = a->kv_update;
  p.advance_ctx = a->advance_ctx;
  p.accepted = a->accepted;
  p.out = reinterpret_cast<__nv_bfloat16*>(a->out);
  p.hq = a->q_heads;
  p.hkv = a->kv_heads;
  p.group = a->q_heads / a->kv_heads;
  const int max_pages = (a->max_context + attn::kPage - 1) / attn::kPage;
  p.pps = attn::pages_per_split(a->batch, a->kv_heads, max_pages, D);
  // a cluster holds all kClusterSplits CTAs of a (sequence, kv head), some
  // possibly without pages
  const bool cluster = !append_only && attn::use_cluster(a->batch, a->kv_heads, D);
  p.max_splits = cluster ? attn::kClusterSplits : std::max(1, (max_pages + p.pps - 1) / p.pps);
  uint8_t* ws = static_cast<uint8_t*>(a->workspace);
  const size_t cnt_bytes = (((size_t)a->batch * a->kv_heads + 1) * 4 + 255) / 256 * 256;
  p.ws_counter = reinterpret_cast<uint32_t*>(ws);
  p.ws_o = reinterpret_cast<float*>(ws + cnt_bytes);
  const int64_t part = (int64_t)a->batch * a->kv_heads * p.max_splits * p.group;
  p.ws_ml = p.ws_o + part * D;
  p.stage_bytes = 2 * attn::kPage * D * 2;
  p.batch = a->batch;
  p.ctx_stable = ctx_stable ? 1 : 0;
  if (append_only) {
    const int warps = std::max(4, std::min(a->kv_heads, 8));
    cudaError_t e = D == 128 ? launch_pdl(attn::append_rows_kernel<128>, dim3(a->batch),
                                          dim3(warps * 32), 0, s_in, p)
                             : launch_pdl(attn::append_rows_kernel<64>, dim3(a->batch),
                                          dim3(warps * 32), 0, s_in, p);
    if (e != cudaSuccess) return cuda_fail(e, "kv append launch");
    return RXLA_B200_OK;
  }
  const bool large = a->batch >= 16;  // enough CTAs to fill the SMs several times
  p.stages = cluster ? attn::kStagesCluster : (large ? attn::kStagesLarge : attn::kStagesSmall);
  const int cw = cluster ? attn::kClusterWarps : attn::kComputeWarps;
  if (next) p.next = *next;

  CUtensorMap kmap, vmap;
  int32_t st = attn::make_page_map(&kmap, a->k_pages, a->num_pages, a->kv_heads, D);
  if (st != RXLA_B200_OK) return st;
  st = attn::make_page_map(&vmap, a->v_pages, a->num_pages, a->kv_heads, D);
  if (st != RXLA_B200_OK) return st;

  // 1024 bytes of alignment slack + the header region (kHdr in the kernel)
  const size_t smem = (D > 128 ? 4096 : 3072) + (size_t)p.stages * p.stage_bytes +
                      (size_t)cw * 8 * (D + 2) * 4 + (size_t)p.max_splits * 8 * 2 * 4;
  const dim3 grid(p.max_splits, a->kv_heads, a->batch);
  const dim3 block((cw + 1) * 32);
  cudaStream_t s = s_in;
  auto go = [&](auto kernel) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    return cluster ? launch_pdl_cluster(kernel, grid, block, smem, s, attn::kClusterSplits, kmap,
                                        vmap, p)
                   : launch_pdl(kernel, grid, block, smem, s, kmap, vmap, p);
  };
  using namespace attn;
  cudaError_t e;
  if (D == 256)  // one CTA per SM: ~170 KB of shared memory, ~200 registers a thread
    e = large ? go(paged_decode_kernel<256, kStagesLarge, 1>)
              : go(paged_decode_kernel<256, kStagesSmall, 1>);
  else if (D == 128)
    e = cluster ? go(paged_decode_kernel<128, kStagesCluster, 1, kClusterWarps, true>)
        : large ? go(paged_decode_kernel<128, kStagesLarge, 3>)
                : go(paged_decode_kernel<128, kStagesSmall, 1>);
  else
    e = cluster ? go(paged_decode_kernel<64, kStagesCluster, 1, kClusterWarps, true>)
        : large ? go(paged_decode_kernel<64, kStagesLarge, 3>)
                : go(paged_decode_kernel<64, kStagesSmall, 1>);
  if (e != cudaSuccess) return cuda_fail(e, "paged decode attention launch");
  return RXLA_B200_OK;
}

// Causal attention of a prompt chunk's rows (the decoder's prefill) after the
// append-only pass wrote their K/V: a->batch rows of one sequence, row t at
// position a->ctx_lens[t] (increasing), the sequence's pages in
// a->page_table's first row.  Output [rows, q_heads, D] bf16.
int32_t prefill_launch(const rxla_b200_paged_decode_args* a, cudaStream_t s) {
  RXLA_REQUIRE(a && a->struct_size >= sizeof(rxla_b200_paged_decode_args),
               "prefill_attention: args struct missing or too small");
  const int D = a->head_dim;
  RXLA_REQUIRE(a->batch >= 0 && a->kv_heads > 0 && a->q_heads > 0 &&
                   a->q_heads % a->kv_heads == 0 && a->q_heads / a->kv_heads <= 8,
               "prefill_attention: 1 to 8 query heads per kv head");
  RXLA_REQUIRE(D == 64 || D == 128, "prefill_attention: head_dim must be 64 or 128");
  RXLA_REQUIRE(a->page_size == attn::kPage && a->kv_heads <= 65535,
               "prefill_attention: page_size must be 16");
  RXLA_REQUIRE(a->rotary_dim == 0 || a->inv_freq == nullptr ||
                   (a->rotary_dim % 32 == 0 && a->rotary_dim <= D),
               "prefill_attention: rotary_dim must be a multiple of 32 and <= head_dim");
  RXLA_REQUIRE(a->scale == 0.0f || std::isfinite(a->scale), "prefill_attention: scale must be finite");
  RXLA_REQUIRE(a->q_row_stride % 2 == 0 && reinterpret_cast<uintptr_t>(a->q) % 4 == 0 &&
                   reinterpret_cast<uintptr_t>(a->out) % 4 == 0,
               "prefill_attention: q rows and out must be 4-byte aligned");
  if (a->batch == 0) return RXLA_B200_OK;
  RXLA_REQUIRE(a->q && a->k_pages && a->v_pages && a->page_table && a->ctx_lens && a->out,
               "prefill_attention: null pointer");
  attn::PrefillParams p{};
  p.q = reinterpret_cast<const __nv_bfloat16*>(a->q);
  p.q_stride = a->q_row_stride;
  p.q_norm_w = a->q_norm_weight;
  p.eps = a->norm_eps;
  p.inv_freq = a->inv_freq;
  p.rot = a->inv_freq ? a->rotary_dim : 0;
  p.scale = a->scale == 0.0f ? 1.0f / std::sqrt((float)D) : a->scale;
  p.page_table = a->page_table;
  p.pos = a->ctx_lens;
  p.n = a->batch;
  p.hq = a->q_heads;
  p.hkv = a->kv_heads;
  p.group = a->q_heads / a->kv_heads;
  p.bq = attn::kPfRows / p.group;
  p.out = reinterpret_cast<__nv_bfloat16*>(a->out);
  CUtensorMap kmap, vmap;
  int32_t st = attn::make_page_map(&kmap, a->k_pages, a->num_pages, a->kv_heads, D);
  if (st != RXLA_B200_OK) return st;
  st = attn::make_page_map(&vmap, a->v_pages, a->num_pages, a->kv_heads, D);
  if (st != RXLA_B200_OK) return st;
  const size_t smem = 2048 + (size_t)attn::kPfStages * 2 * attn::kPage * D * 2;
  const dim3 grid((unsigned)((p.n + p.bq - 1) / p.bq), (unsigned)a->kv_heads);
  const dim3 block(attn::kPfWarps * 32);
  auto go = [&](auto kernel) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e == cudaSuccess) e = launch_pdl(kernel, grid, block, smem, s, kmap, vmap, p);
    return e;
  };
  cudaError_t e = D == 128 ? go(attn::prefill_attention_kernel<128>)
                           : go(attn::prefill_attention_kernel<64>);
  if (e != cudaSuccess) return cuda_fail(e, "prefill attention launch");
  return RXLA_B200_OK;
}
}  // namespace attn
}  // namespace rxla

extern "C" int32_t rxla_b200_paged_decode_attention(const rxla_b200_paged_decode_args* args,
                                                    void* stream) {
  // a standalone call cannot know which kernel last wrote ctx_lens
  return rxla::attn::launch(args, static_cast<cudaStream_t>(stream), false);
}
