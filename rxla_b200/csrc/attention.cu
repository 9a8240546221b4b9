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
//  * CTA = (sequence, split of `pps` pages); warp h = kv head h, a producer
//    warp streams pages through a shared-memory ring with TMA tensor loads.
//    One box is [64 dims × kv_heads·16 rows] with 128-byte swizzle, so a page
//    of K for all kv heads is D/64 requests of up to 16 KB (the TMA engine is
//    request-rate bound below ~4 KB per request);
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
//  * splits write (O, m, l) partials to the workspace; the last CTA of a
//    sequence (atomic counter) merges them with log-sum-exp weights and
//    resets the counter.  A single split writes the output directly.
#include <cudaTypedefs.h>

#include "common.cuh"

namespace rxla {
namespace attn {

constexpr int kPage = 16;
constexpr int kMaxStages = 4;

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
  int32_t stage_bytes;  // K + V of one page, all kv heads
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
  if (prev != gridDim.x * gridDim.y - 1) return;
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

template <int D>
__global__ void __launch_bounds__(17 * 32, 1)
    paged_decode_kernel(const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap, const Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw);
  uint64_t* empty = full + kMaxStages;
  // the swizzled ring must start on a 1024-byte boundary
  const uint32_t base_u32 = smem_u32(smem_raw);
  uint8_t* ring = smem_raw + ((1024u - (base_u32 & 1023u)) & 1023u) + 1024;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.y, split = blockIdx.x;
  const int hkv = p.hkv, G = p.group;
  const int rows = hkv * kPage;  // rows of one page box (all kv heads)
  const int S = p.stages;

  if (!p.ctx_stable) pdl_wait();
  const int pos = p.ctx_lens[b];
  const int cap = (p.pages_per_seq ? p.pages_per_seq[b] : p.max_pages) * kPage;
  const int n_keys = pos < 0 ? 0 : min(pos + 1, cap);
  const int n_pages = (n_keys + kPage - 1) / kPage;
  const int n_splits = max(1, (n_pages + p.pps - 1) / p.pps);
  const int pg0 = split * p.pps;
  const int pg1 = min(n_pages, pg0 + p.pps);
  const bool in_range = pos >= 0 && pos < cap;
  const bool accept = cap > 0 && (in_range || p.kv_update == RXLA_B200_KV_CLAMP);
  const int slot = pos < 0 ? 0 : (pos >= cap ? cap - 1 : pos);
  const bool owner = accept && split == (slot / kPage) / p.pps;

  if (split >= n_splits) {  // nothing of this sequence in this split
    if (threadIdx.x == 0) finish_cta(p);
    pdl_launch_dependents();
    return;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], hkv);
    }
    fence_mbarrier_init();
  }
  __syncthreads();

  if (warp == hkv) {
    // ------------------------------------------------------------ producer
    // Pages hold rows appended by earlier kernels only (the new row is patched
    // in from registers); with a stable ctx_lens they are fetched before
    // griddepcontrol.wait.
    if (lane == 0) {
      const uint32_t bytes = (uint32_t)p.stage_bytes;
      for (int pg = pg0, it = 0; pg < pg1; ++pg, ++it) {
        const int s = it % S;
        if (it >= S && !mbar_wait(&empty[s], ((it / S) - 1) & 1)) break;
        const int page = p.page_table[(int64_t)b * p.max_pages + pg];
        const int row = page * rows;
        mbar_arrive_expect_tx(&full[s], bytes);
        uint8_t* kdst = ring + (size_t)s * p.stage_bytes;
        uint8_t* vdst = kdst + p.stage_bytes / 2;
#pragma unroll
        for (int j = 0; j < D / 64; ++j) {
          tma_load_2d(kdst + j * rows * 128, &kmap, 64 * j, row, &full[s]);
          tma_load_2d(vdst + j * rows * 128, &vmap, 64 * j, row, &full[s]);
        }
      }
    }
  } else {
    // -------------------------------------------------------- kv-head warps
    const int h = warp;
    if (p.ctx_stable) pdl_wait();  // q / k_new / v_new come from the previous kernel
    const int g = lane >> 2, q4 = lane & 3;

    // new k / v of this kv head: lane holds dims [DL*lane, DL*lane + DL)
    constexpr int DL = D / 32;
    float kn[DL], vn[DL];
    if (owner) {
      const __nv_bfloat16* kr = p.k_new + (int64_t)b * p.kv_stride + (int64_t)h * D;
      const __nv_bfloat16* vr = p.v_new + (int64_t)b * p.kv_stride + (int64_t)h * D;
      float ss = 0.0f;
#pragma unroll
      for (int i = 0; i < DL; ++i) {
        kn[i] = __bfloat162float(kr[DL * lane + i]);
        vn[i] = __bfloat162float(vr[DL * lane + i]);
        ss += kn[i] * kn[i];
      }
      if (p.k_norm_w) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float rs = 1.0f / sqrtf(ss / (float)D + p.eps);
#pragma unroll
        for (int i = 0; i < DL; ++i) kn[i] = (kn[i] * rs) * p.k_norm_w[DL * lane + i];
      }
      if (p.rot > 0) {
        // partner of dim d < rot/2 is d + rot/2, held by lane + rot/(2·DL)
        const int half = p.rot / 2, off = half / DL;
        const float fpos = (float)pos;
#pragma unroll
        for (int i = 0; i < DL; ++i) {
          const int d = DL * lane + i;
          const float up = __shfl_sync(0xffffffffu, kn[i], (lane + off) & 31);
          const float dn = __shfl_sync(0xffffffffu, kn[i], (lane - off) & 31);
          if (d < half) {
            const float ang = fpos * p.inv_freq[d];
            kn[i] = kn[i] * cosf(ang) - up * sinf(ang);
          } else if (d < p.rot) {
            const float ang = fpos * p.inv_freq[d - half];
            kn[i] = kn[i] * cosf(ang) + dn * sinf(ang);
          }
        }
      }
#pragma unroll
      for (int i = 0; i < DL; ++i) {
        kn[i] = bf16_round(kn[i]);
        vn[i] = bf16_round(vn[i]);
      }
      // append into the cache (global)
      const int page = p.page_table[(int64_t)b * p.max_pages + slot / kPage];
      const int64_t base = (((int64_t)page * hkv + h) * kPage + slot % kPage) * D + DL * lane;
#pragma unroll
      for (int i = 0; i < DL; ++i) {
        p.k_pages[base + i] = __float2bfloat16_rn(kn[i]);
        p.v_pages[base + i] = __float2bfloat16_rn(vn[i]);
      }
      __threadfence();
    }
    // every kv-head warp has appended: let dependent kernels launch
    asm volatile("bar.sync 1, %0;" ::"r"(hkv * 32) : "memory");
    if (warp == 0 && lane == 0) pdl_launch_dependents();

    // q of the G heads of this kv head, in B-fragment layout: lane (g, q4)
    // holds head g, dims ks*16 + 2*q4 + {0,1,8,9} for ks = 0..D/16-1.
    constexpr int KS = D / 16;
    uint32_t qhi[KS][2], qlo[KS][2];
    {
      float qv[KS][4];
      const bool valid = g < G;
      const __nv_bfloat16* qr =
          p.q + (int64_t)b * p.q_stride + (int64_t)(h * G + (valid ? g : 0)) * D;
      float ss = 0.0f;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        const int d0 = ks * 16 + 2 * q4;
        const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(qr + d0);
        const __nv_bfloat162 c = *reinterpret_cast<const __nv_bfloat162*>(qr + d0 + 8);
        qv[ks][0] = valid ? __low2float(a) : 0.0f;
        qv[ks][1] = valid ? __high2float(a) : 0.0f;
        qv[ks][2] = valid ? __low2float(c) : 0.0f;
        qv[ks][3] = valid ? __high2float(c) : 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) ss += qv[ks][i] * qv[ks][i];
      }
      if (p.q_norm_w) {
        ss += __shfl_xor_sync(0xffffffffu, ss, 1);
        ss += __shfl_xor_sync(0xffffffffu, ss, 2);
        const float rs = 1.0f / sqrtf(ss / (float)D + p.eps);
#pragma unroll
        for (int ks = 0; ks < KS; ++ks)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int d = ks * 16 + 2 * q4 + (i & 1) + (i >> 1) * 8;
            qv[ks][i] = (qv[ks][i] * rs) * p.q_norm_w[d];
          }
      }
      if (p.rot > 0) {
        const int hs = p.rot / 32;  // k-step distance of a RoPE pair
        const float fpos = (float)pos;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
          if (ks >= hs) continue;  // upper halves are rotated with their partner
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int d = ks * 16 + 2 * q4 + (i & 1) + (i >> 1) * 8;
            const float ang = fpos * p.inv_freq[d];
            const float c = cosf(ang), sn = sinf(ang);
            const float a = qv[ks][i], bb = qv[ks + hs][i];
            qv[ks][i] = a * c - bb * sn;
            qv[ks + hs][i] = bb * c + a * sn;
          }
        }
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

    // running softmax state of head columns 2*q4, 2*q4+1
    float m_run[2] = {-INFINITY, -INFINITY};
    float l_part[2] = {0.0f, 0.0f};
    float o[D / 16][4];
#pragma unroll
    for (int mt = 0; mt < D / 16; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) o[mt][i] = 0.0f;

    const int r0 = h * kPage;
    for (int pg = pg0, it = 0; pg < pg1; ++pg, ++it) {
      const int s = it % S;
      if (!mbar_wait(&full[s], (it / S) & 1)) break;
      uint8_t* kt = ring + (size_t)s * p.stage_bytes;
      uint8_t* vt = kt + p.stage_bytes / 2;
      if (owner && pg == slot / kPage) {
        // patch the appended row into the loaded tile
        const int r = r0 + slot % kPage;
#pragma unroll
        for (int i = 0; i < DL; i += 2) {
          const int d = DL * lane + i;
          *reinterpret_cast<uint32_t*>(kt + swz(r, d, rows)) = pack_bf16x2(kn[i], kn[i + 1]);
          *reinterpret_cast<uint32_t*>(vt + swz(r, d, rows)) = pack_bf16x2(vn[i], vn[i + 1]);
        }
        __syncwarp();
      }
      // ---- S^T (16 tokens x 8 head columns) = K · Q^T
      float sc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      const uint32_t kbase = smem_u32(kt);
      const int mi = lane >> 3, rr = lane & 7;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        // matrices: (tok 0-7, d 0-7), (tok 8-15, d 0-7), (tok 0-7, d 8-15), (tok 8-15, d 8-15)
        uint32_t a[4];
        ldsm_x4(a, kbase + swz(r0 + rr + ((mi & 1) << 3), ks * 16 + ((mi >> 1) << 3), rows));
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
        ldsm_x4_t(a, vbase + swz(r0 + rr + ((mi >> 1) << 3), mt * 16 + ((mi & 1) << 3), rows));
        mma_bf16_16816(o[mt], a, b0, b1);
        mma_bf16_16816(o[mt], a, c0, c1);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }

    // ---- finalize this split
    float l_tot[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float l = l_part[j];
      l += __shfl_xor_sync(0xffffffffu, l, 4);
      l += __shfl_xor_sync(0xffffffffu, l, 8);
      l += __shfl_xor_sync(0xffffffffu, l, 16);
      l_tot[j] = l;
    }
    const int hc0 = 2 * q4;  // head columns of this lane
    if (n_splits == 1) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        if (hc0 + j >= G) continue;
        const float inv = l_tot[j] > 0.0f ? 1.0f / l_tot[j] : 0.0f;
        __nv_bfloat16* orow = p.out + (int64_t)b * p.hq * D + (int64_t)(h * G + hc0 + j) * D;
#pragma unroll
        for (int mt = 0; mt < D / 16; ++mt) {
          orow[mt * 16 + g] = __float2bfloat16_rn(o[mt][j] * inv);
          orow[mt * 16 + g + 8] = __float2bfloat16_rn(o[mt][2 + j] * inv);
        }
      }
    } else {
      // partials of this split, then the last split of (b, h) merges them
      const int64_t seg = (((int64_t)b * hkv + h) * p.max_splits + split) * G;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        if (hc0 + j >= G) continue;
        float* po = p.ws_o + (seg + hc0 + j) * D;
#pragma unroll
        for (int mt = 0; mt < D / 16; ++mt) {
          po[mt * 16 + g] = o[mt][j];
          po[mt * 16 + g + 8] = o[mt][2 + j];
        }
        if (g == 0) {
          p.ws_ml[(seg + hc0 + j) * 2] = m_run[j];
          p.ws_ml[(seg + hc0 + j) * 2 + 1] = l_tot[j];
        }
      }
      __threadfence();
      __syncwarp();
      int last = 0;
      if (lane == 0) {
        const uint32_t prev = atomicAdd(&p.ws_counter[b * hkv + h], 1u);
        last = prev == (uint32_t)(n_splits - 1);
      }
      last = __shfl_sync(0xffffffffu, last, 0);
      if (last) {
        __threadfence();
        for (int j = 0; j < G; ++j) {
          const int64_t segj = ((int64_t)b * hkv + h) * p.max_splits * G + j;
          float mstar = -INFINITY;
          for (int sp = 0; sp < n_splits; ++sp)
            mstar = fmaxf(mstar, __ldcg(p.ws_ml + (segj + (int64_t)sp * G) * 2));
          float den = 0.0f;
          float acc[DL];
#pragma unroll
          for (int i = 0; i < DL; ++i) acc[i] = 0.0f;
          for (int sp = 0; sp < n_splits; ++sp) {
            const int64_t e = segj + (int64_t)sp * G;
            const float m = __ldcg(p.ws_ml + e * 2), l = __ldcg(p.ws_ml + e * 2 + 1);
            const float w = (m == -INFINITY) ? 0.0f : expf(m - mstar);
            den += w * l;
#pragma unroll
            for (int i = 0; i < DL; ++i) acc[i] += w * __ldcg(p.ws_o + e * D + lane + 32 * i);
          }
          const float inv = den > 0.0f ? 1.0f / den : 0.0f;
          __nv_bfloat16* orow = p.out + (int64_t)b * p.hq * D + (int64_t)(h * G + j) * D;
#pragma unroll
          for (int i = 0; i < DL; ++i) orow[lane + 32 * i] = __float2bfloat16_rn(acc[i] * inv);
        }
        if (lane == 0) p.ws_counter[b * hkv + h] = 0u;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) finish_cta(p);
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
  const cuuint32_t box[2] = {64, (cuuint32_t)(hkv * kPage)};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(RXLA_B200_INVALID_ARGUMENT, "page tensor map encoding failed");
  return RXLA_B200_OK;
}

// pages per split: enough CTAs for ~4 waves when sequences average half of
// max_context, at most 16 pages (256 tokens) per split for balance.
static int pages_per_split(int batch, int max_pages) {
  int64_t v = ((int64_t)batch * max_pages) / (8 * 148);
  return (int)std::max<int64_t>(1, std::min<int64_t>(16, v));
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
  const int pps = attn::pages_per_split(batch, max_pages);
  const int64_t splits = std::max(1, (max_pages + pps - 1) / pps);
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
// the end of a step).
int32_t launch(const rxla_b200_paged_decode_args* a, cudaStream_t s_in, bool ctx_stable) {
  RXLA_REQUIRE(a && a->struct_size >= sizeof(rxla_b200_paged_decode_args),
               "paged_decode: args struct missing or too small");
  const int D = a->head_dim;
  RXLA_REQUIRE(a->batch >= 0 && a->kv_heads > 0 && a->q_heads > 0 &&
                   a->q_heads % a->kv_heads == 0,
               "paged_decode: query heads must be a positive multiple of kv heads (attention.rs:99-112)");
  RXLA_REQUIRE(a->q_heads / a->kv_heads <= 8, "paged_decode: at most 8 query heads per kv head");
  RXLA_REQUIRE(a->kv_heads <= 16, "paged_decode: at most 16 kv heads per call (shard larger models)");
  RXLA_REQUIRE(D == 64 || D == 128, "paged_decode: head_dim must be 64 or 128");
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
  p.pps = attn::pages_per_split(a->batch, max_pages);
  p.max_splits = std::max(1, (max_pages + p.pps - 1) / p.pps);
  uint8_t* ws = static_cast<uint8_t*>(a->workspace);
  const size_t cnt_bytes = (((size_t)a->batch * a->kv_heads + 1) * 4 + 255) / 256 * 256;
  p.ws_counter = reinterpret_cast<uint32_t*>(ws);
  p.ws_o = reinterpret_cast<float*>(ws + cnt_bytes);
  const int64_t part = (int64_t)a->batch * a->kv_heads * p.max_splits * p.group;
  p.ws_ml = p.ws_o + part * D;
  p.stage_bytes = 2 * a->kv_heads * attn::kPage * D * 2;
  p.batch = a->batch;
  p.ctx_stable = ctx_stable ? 1 : 0;
  p.stages = (int)std::min<int64_t>(attn::kMaxStages, (200 * 1024) / p.stage_bytes);
  if (p.stages < 2) p.stages = 2;

  CUtensorMap kmap, vmap;
  int32_t st = attn::make_page_map(&kmap, a->k_pages, a->num_pages, a->kv_heads, D);
  if (st != RXLA_B200_OK) return st;
  st = attn::make_page_map(&vmap, a->v_pages, a->num_pages, a->kv_heads, D);
  if (st != RXLA_B200_OK) return st;

  const size_t smem = 2048 + (size_t)p.stages * p.stage_bytes;
  const dim3 grid(p.max_splits, a->batch);
  const dim3 block((a->kv_heads + 1) * 32);
  cudaStream_t s = s_in;
  cudaError_t e;
  if (D == 128) {
    e = cudaFuncSetAttribute(attn::paged_decode_kernel<128>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess)
      e = launch_pdl(attn::paged_decode_kernel<128>, grid, block, smem, s, kmap, vmap, p);
  } else {
    e = cudaFuncSetAttribute(attn::paged_decode_kernel<64>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess)
      e = launch_pdl(attn::paged_decode_kernel<64>, grid, block, smem, s, kmap, vmap, p);
  }
  if (e != cudaSuccess) return cuda_fail(e, "paged decode attention launch");
  return RXLA_B200_OK;
}
}  // namespace attn
}  // namespace rxla

extern "C" int32_t rxla_b200_paged_decode_attention(const rxla_b200_paged_decode_args* args,
                                                    void* stream) {
  // a standalone call cannot know which kernel last wrote ctx_lens
  return rxla::attn::launch(args, static_cast<cudaStream_t>(stream), false);
}
