// w8_chain.cu — several W8 linears of a decode step in one persistent launch.
//
// A decoder layer after attention is a chain of dependent W8 linears:
// o_proj (+ residual) → gate/up (RMSNorm, SwiGLU) → down_proj (+ residual) →
// the next layer's qkv (RMSNorm), or the tied LM head (RMSNorm, greedy argmax)
// after the last layer.  As separate kernels each one pays a launch, a ring
// ramp-up and a drain, with HBM idle in between.  Here one CTA per SM runs
// every phase of the chain with the skinny GEMV's warp roles (16 consumer
// warps on mma.sync, a TMA producer warp, an epilogue warp): the producer
// streams phase after phase through one shared-memory ring without waiting
// for any phase to finish, so the next phase's first weights are in shared
// memory when its input is ready; a phase's input readiness is a grid-wide
// arrival counter (each CTA adds one after its epilogue wrote its rows).
// Every wait is bounded (%globaltimer): an expired wait records
// DEADLINE_EXCEEDED in the device status word and the CTA returns.
//
// Numerics are the skinny kernel's (the reference's QuantizedLinear,
// crates/rxla-nn/src/layers.rs:257-298, and RMSNorm, crates/rxla-core/src/
// ops.rs:929-945): the same dequantization, products, per-warp fp32 sums,
// fixed-order cross-warp sum and epilogues.
#include "internal.cuh"

namespace rxla {
namespace chain {

using w8::box_mma;
using w8::kConsumerWarps;
using w8::kEpilogueWarp;
using w8::kProducerWarp;
using w8::kRedFloats;
using w8::kEpiArgmax;
using w8::kMaxTokens;
using w8::kTileRows;
using w8::needs_post;
using w8::row_scale;
using w8::RowScale;

constexpr int kStagesMax = 8;
constexpr int kHeaderBytes = 1024;

struct Bars {
  uint64_t full[kStagesMax];
  uint64_t empty[kStagesMax];
  uint64_t epi_full[2];
  uint64_t epi_free[2];
  uint64_t csync;           // the consumer warps
  int32_t flag;             // broadcast of a global wait's outcome
  float ss[16][2];  // per consumer warp (at most 16)
};
static_assert(sizeof(Bars) <= kHeaderBytes, "chain header");

__device__ __forceinline__ void red_release_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Wait until every CTA of the grid has finished a phase (bounded).
__device__ __forceinline__ bool wait_grid(const uint32_t* counter, uint32_t target) {
  if (ld_acquire(counter) >= target) return true;
  const uint64_t t0 = globaltimer();
  while (ld_acquire(counter) < target) {
    if (globaltimer() - t0 > kWaitTimeoutNs) {
      record_device_error(RXLA_B200_DEADLINE_EXCEEDED);
      return false;
    }
  }
  return true;
}

// Bounded barrier of the consumer warps on an mbarrier (phase toggles).
__device__ __forceinline__ bool csync(Bars& b, uint32_t& par) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&b.csync);
  const bool ok = mbar_wait(&b.csync, par);
  par ^= 1u;
  return ok;
}

__global__ void __launch_bounds__(w8::kThreads, 1)
    w8_chain_kernel(const __grid_constant__ ChainParams p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  Bars& bars = *reinterpret_cast<Bars*>(smem_raw);
  float* red = reinterpret_cast<float*>(smem_raw + kHeaderBytes);  // [2][warp][16 rows][8 tokens]
  uint8_t* xs = smem_raw + kHeaderBytes + 2 * kRedFloats * 4;       // bf16 [m][x_pitch]
  uint8_t* stages = xs + (size_t)p.m * p.x_pitch;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int S = p.stages;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&bars.full[s], 1);
      mbar_init(&bars.empty[s], kConsumerWarps);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars.epi_full[i], kConsumerWarps);
      mbar_init(&bars.epi_free[i], 1);
    }
    mbar_init(&bars.csync, kConsumerWarps);
    fence_mbarrier_init();
  }
  __syncthreads();

  // rows of phase ph owned by this CTA, in blocks of 16 (8 gate + 8 up for SwiGLU)
  auto rows_of = [&](const ChainPhase& ph, int& r_begin, int& r_end, int& n_blocks, int& out_rows) {
    const bool sw = ph.epilogue == RXLA_B200_EPI_SWIGLU;
    out_rows = sw ? kTileRows / 2 : kTileRows;
    r_begin = (int)(((int64_t)ph.n * blockIdx.x) / gridDim.x);
    r_end = (int)(((int64_t)ph.n * (blockIdx.x + 1)) / gridDim.x);
    n_blocks = (r_end - r_begin + out_rows - 1) / out_rows;
  };

  if (warp == kProducerWarp) {
    // -------------------------------------------------------------- producer
    // Weights only: never waits for a phase, only for ring slots.
    if (lane != 0) return;
    const uint64_t policy = l2_evict_first_policy();
    // L2 lookahead: the bytes of this CTA's stream up to l2_ahead past the
    // last stage requested are prefetched into L2, so HBM keeps streaming
    // while the ring is full at a phase boundary.  Packed phases only (a
    // CTA's share of a packed matrix is one contiguous range).
    int pf_pi = 0;
    int64_t pf_off = 0, pf_pos = 0, issued = 0;
    auto prefetch_upto = [&](int64_t target) {
      while (pf_pos < target && pf_pi < p.nphases) {
        const ChainPhase& q = p.ph[pf_pi];
        int rb, re, nb, orows;
        rows_of(q, rb, re, nb, orows);
        const int mult = q.epilogue == RXLA_B200_EPI_SWIGLU ? 2 : 1;
        const int64_t len = (int64_t)(re - rb) * mult * q.k;
        if (pf_off >= len) {
          ++pf_pi;
          pf_off = 0;
          continue;
        }
        const int64_t take = min((int64_t)32768, len - pf_off);
        if (q.packed)
          asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(
                           q.w + (int64_t)rb * mult * q.k + pf_off),
                       "r"((uint32_t)take)
                       : "memory");
        pf_off += take;
        pf_pos += take;
      }
    };
    int it = 0;
    for (int pi = 0; pi < p.nphases; ++pi) {
      const ChainPhase& ph = p.ph[pi];
      const bool sw = ph.epilogue == RXLA_B200_EPI_SWIGLU;
      int r_begin, r_end, n_blocks, out_rows;
      rows_of(ph, r_begin, r_end, n_blocks, out_rows);
      for (int blk = 0; blk < n_blocks; ++blk) {
        const int r0 = r_begin + blk * out_rows;
        const int nr = min(out_rows, r_end - r0);
        for (int kc = 0; kc < ph.k_chunks; ++kc, ++it) {
          const int s = it % S;
          if (it >= S && !mbar_wait(&bars.empty[s], ((it / S) - 1) & 1)) return;
          const int col0 = kc * p.kc;
          const uint32_t tx = (uint32_t)p.kc * (uint32_t)nr * (sw ? 2u : 1u);
          mbar_arrive_expect_tx(&bars.full[s], tx);
          issued += tx;
          if (p.l2_ahead > 0) prefetch_upto(issued + p.l2_ahead);
          uint8_t* dst = stages + (size_t)s * p.stage_bytes;
          if (ph.packed) {
            // stream order: the block's k-chunk is nr (gate) rows, then nr up rows
            const uint8_t* src = ph.w + ((int64_t)r0 * ph.k + (int64_t)kc * nr * p.kc) * (sw ? 2 : 1);
            if (sw && nr < out_rows) {
              bulk_g2s(dst, src, (uint32_t)(nr * p.kc), &bars.full[s], policy);
              bulk_g2s(dst + (size_t)(kTileRows / 2) * p.kc, src + (size_t)nr * p.kc,
                       (uint32_t)(nr * p.kc), &bars.full[s], policy);
            } else {
              bulk_g2s(dst, src, tx, &bars.full[s], policy);
            }
            continue;
          }
          if (ph.k == p.kc) {
            // whole rows: the block is one contiguous range (two for SwiGLU)
            bulk_g2s(dst, ph.w + (int64_t)r0 * ph.k, (uint32_t)(nr * ph.k), &bars.full[s], policy);
            if (sw)
              bulk_g2s(dst + (size_t)(kTileRows / 2) * p.kc, ph.w + (int64_t)(ph.n + r0) * ph.k,
                       (uint32_t)(nr * ph.k), &bars.full[s], policy);
            continue;
          }
          for (int i = 0; i < nr; ++i) {
            bulk_g2s(dst + (size_t)i * p.kc, ph.w + (int64_t)(r0 + i) * ph.k + col0, (uint32_t)p.kc,
                     &bars.full[s], policy);
            if (sw)
              bulk_g2s(dst + (size_t)(kTileRows / 2 + i) * p.kc,
                       ph.w + (int64_t)(ph.n + r0 + i) * ph.k + col0, (uint32_t)p.kc, &bars.full[s],
                       policy);
          }
        }
      }
    }
    return;
  }

  const int g = lane >> 2;  // mma group id: A rows g, g+8; B column (token) g
  const int q = lane & 3;

  if (warp == kEpilogueWarp) {
    // -------------------------------------------------------------- epilogue
    pdl_wait();  // the residual / outputs may be used by the previous kernel
    int gb = 0;  // blocks handed over so far (parity of the partial buffers)
    for (int pi = 0; pi < p.nphases; ++pi) {
      const ChainPhase& ph = p.ph[pi];
      const bool sw = ph.epilogue == RXLA_B200_EPI_SWIGLU;
      const bool argmax = ph.epilogue == kEpiArgmax;
      const bool resid = ph.epilogue == RXLA_B200_EPI_RESIDUAL_ADD;
      // an earlier phase of this chain may have written this phase's residual
      if (pi > 0) {
        int ok = 1;
        if (lane == 0) ok = wait_grid(p.bar + pi - 1, gridDim.x) ? 1 : 0;
        if (!__shfl_sync(0xffffffffu, ok, 0)) return;
      }
      int r_begin, r_end, n_blocks, out_rows;
      rows_of(ph, r_begin, r_end, n_blocks, out_rows);
      float best_v[kMaxTokens];
      int best_i[kMaxTokens];
#pragma unroll
      for (int t = 0; t < kMaxTokens; ++t) {
        best_v[t] = -INFINITY;
        best_i[t] = 0x7fffffff;
      }
      constexpr int kPerLane = (kTileRows * kMaxTokens) / 32;
      for (int blk = 0; blk < n_blocks; ++blk, ++gb) {
        const int b2 = gb & 1;
        const int r0 = r_begin + blk * out_rows;
        const int nr = min(out_rows, r_end - r0);
        float rv[kPerLane];
#pragma unroll
        for (int tt = 0; tt < kPerLane; ++tt) {
          const int idx = lane + 32 * tt;
          const int row = idx % out_rows, tok = idx / out_rows;
          rv[tt] = (resid && row < nr && tok < p.m && idx < out_rows * kMaxTokens)
                       ? __ldcg(static_cast<const float*>(ph.y) + (int64_t)tok * ph.n + r0 + row)
                       : 0.0f;
        }
        if (!mbar_wait(&bars.epi_full[b2], (gb >> 1) & 1)) return;
        const float* rb = red + b2 * kRedFloats;
#pragma unroll
        for (int tt = 0; tt < kPerLane; ++tt) {
          const int idx = lane + 32 * tt;
          const int row = idx % out_rows, tok = idx / out_rows;
          if (idx >= out_rows * kMaxTokens || row >= nr || tok >= p.m) continue;
          float v = 0.0f, u = 0.0f;
#pragma unroll
          for (int w2 = 0; w2 < kConsumerWarps; ++w2) {
            v += rb[(w2 * kTileRows + row) * kMaxTokens + tok];
            if (sw) u += rb[(w2 * kTileRows + row + 8) * kMaxTokens + tok];
          }
          const int out_col = r0 + row;
          const int64_t o = (int64_t)tok * ph.n + out_col;
          if (sw) {
            const float r = silu(bf16_round(v)) * bf16_round(u);
            if (ph.y_f32) static_cast<float*>(ph.y)[o] = r;
            else static_cast<__nv_bfloat16*>(ph.y)[o] = __float2bfloat16_rn(r);
          } else if (argmax) {
            if (ph.y) static_cast<float*>(ph.y)[o] = v;
#pragma unroll
            for (int t = 0; t < kMaxTokens; ++t)
              if (t == tok && (v > best_v[t] || (v == best_v[t] && out_col < best_i[t]))) {
                best_v[t] = v;
                best_i[t] = out_col;
              }
          } else if (resid) {
            static_cast<float*>(ph.y)[o] = rv[tt] + bf16_round(v);
          } else if (ph.y_f32) {
            static_cast<float*>(ph.y)[o] = v;
          } else {
            static_cast<__nv_bfloat16*>(ph.y)[o] = __float2bfloat16_rn(v);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars.epi_free[b2]);
      }
      if (argmax) {
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
          for (int t = 0; t < p.m; ++t) {
            ph.arg_val[blockIdx.x * kMaxTokens + t] = best_v[t];
            ph.arg_idx[blockIdx.x * kMaxTokens + t] = best_i[t];
          }
          __threadfence();
        }
        uint32_t prev = 0;
        if (lane == 0) prev = atomicAdd(ph.arg_count, 1u);
        prev = __shfl_sync(0xffffffffu, prev, 0);
        if (prev == gridDim.x - 1) {
          __threadfence();
          for (int t = 0; t < p.m; ++t) {
            float bv = -INFINITY;
            int bi = 0x7fffffff;
            for (int c = lane; c < (int)gridDim.x; c += 32) {
              const float v = __ldcg(ph.arg_val + c * kMaxTokens + t);
              const int i = __ldcg(ph.arg_idx + c * kMaxTokens + t);
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
              ph.arg_out[t] = bi == 0x7fffffff ? 0 : bi;
              if (ph.arg_advance) ph.arg_advance[t] += 1;
            }
          }
          if (lane == 0) *ph.arg_count = 0u;
        }
      }
      // this CTA's rows of the phase are written: count it in (the release
      // after the warp barrier is cumulative over every lane's stores)
      __syncwarp();
      if (lane == 0) red_release_add(p.bar + pi, 1u);
    }
    // dependents wait for this grid's completion; triggered only when this
    // CTA is done, so no dependent CTA takes an SM a chain CTA still needs
    if (lane == 0) pdl_launch_dependents();
    return;
  }

  // ---------------------------------------------------------------- consumers
  const int ctid = threadIdx.x;  // 0 .. 511
  constexpr int kCT = kConsumerWarps * 32;
  uint32_t cpar = 0;  // csync phase
  int s = 0;          // ring position
  uint32_t rph = 0;
  int gb = 0;
  const int lane_off = g * p.kc + warp * 64 + 16 * q;
  const int row8 = 8 * p.kc;
  constexpr int kBoxStep = kConsumerWarps * 64;
  constexpr int kXV = 4;  // float4 of the normalised row per thread (k <= 8192)
  for (int pi = 0; pi < p.nphases; ++pi) {
    const ChainPhase& ph = p.ph[pi];
    const bool sw = ph.epilogue == RXLA_B200_EPI_SWIGLU;
    int r_begin, r_end, n_blocks, out_rows;
    rows_of(ph, r_begin, r_end, n_blocks, out_rows);
    auto block_rows = [&](int blk, bool& va, bool& vb, int& ra, int& rb) {
      const int r0 = r_begin + blk * out_rows;
      const int nr = min(out_rows, r_end - r0);
      if (sw) {
        va = vb = g < nr;
        ra = r0 + g;
        rb = ph.n + r0 + g;
      } else {
        va = g < nr;
        vb = g + 8 < nr;
        ra = r0 + g;
        rb = r0 + g + 8;
      }
    };
    // ---- what does not depend on the previous phase is loaded before the
    // wait: the norm weights and the first block's row scales
    float4 nw[kXV];
    if (ph.x_norm && n_blocks > 0) {
#pragma unroll
      for (int i = 0; i < kXV; ++i) {
        const int c = (ctid + i * kCT) * 4;
        nw[i] = c < ph.k ? __ldg(reinterpret_cast<const float4*>(ph.norm_w + c))
                         : make_float4(1.f, 1.f, 1.f, 1.f);
      }
    }
    float next_sa = 0.0f, next_sb = 0.0f;
    if (n_blocks > 0) {
      bool va, vb;
      int ra, rb;
      block_rows(0, va, vb, ra, rb);
      next_sa = va ? __ldg(ph.scale + ra) : 0.0f;
      next_sb = vb ? __ldg(ph.scale + rb) : 0.0f;
    }
    // ---- wait for this phase's input
    if (pi == 0) {
      pdl_wait();  // x comes from the previous kernel
    } else {
      if (ctid == 0) bars.flag = wait_grid(p.bar + pi - 1, gridDim.x) ? 1 : 0;
      if (!csync(bars, cpar) || !bars.flag) return;
    }
    if (n_blocks == 0) continue;  // same for every consumer warp of the CTA
    // ---- x into shared memory: bf16 copy, or bf16(rms_norm(h) * norm_w)
    if (!ph.x_norm) {
      const int chunks = ph.k / 8;  // 16-byte chunks per token row
      for (int t = 0; t < p.m; ++t) {
        const uint4* src = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(ph.x) +
                                                          (int64_t)t * ph.k);
        uint4* dst = reinterpret_cast<uint4*>(xs + t * p.x_pitch);
        for (int c = ctid; c < chunks; c += kCT) dst[c] = __ldcg(src + c);
      }
    } else {
      const float* hf = static_cast<const float*>(ph.x);
      for (int t0 = 0; t0 < p.m; t0 += 2) {
        const int nt = min(2, p.m - t0);
        float4 hv[2][kXV];
        float ss[2] = {0.0f, 0.0f};
#pragma unroll
        for (int u = 0; u < 2; ++u)
#pragma unroll
          for (int i = 0; i < kXV; ++i) {
            const int c = (ctid + i * kCT) * 4;
            hv[u][i] = (u < nt && c < ph.k)
                           ? __ldcg(reinterpret_cast<const float4*>(hf + (int64_t)(t0 + u) * ph.k + c))
                           : make_float4(0.f, 0.f, 0.f, 0.f);
            ss[u] += hv[u][i].x * hv[u][i].x + hv[u][i].y * hv[u][i].y +
                     hv[u][i].z * hv[u][i].z + hv[u][i].w * hv[u][i].w;
          }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) ss[u] += __shfl_xor_sync(0xffffffffu, ss[u], o);
        }
        if (lane == 0) {
          bars.ss[warp][0] = ss[0];
          bars.ss[warp][1] = ss[1];
        }
        if (!csync(bars, cpar)) return;
        float inv[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          float tot = 0.0f;
          for (int w2 = 0; w2 < kConsumerWarps; ++w2) tot += bars.ss[w2][u];
          inv[u] = 1.0f / sqrtf(tot / (float)ph.k + ph.norm_eps);
        }
        // every warp has read the sums before the next round overwrites them
        if (!csync(bars, cpar)) return;
        for (int u = 0; u < nt; ++u) {
          __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(xs + (t0 + u) * p.x_pitch);
#pragma unroll
          for (int i = 0; i < kXV; ++i) {
            const int c = (ctid + i * kCT) * 4;
            if (c < ph.k) {
              float4 h = hv[u][i];
              h.x = (h.x * inv[u]) * nw[i].x;
              h.y = (h.y * inv[u]) * nw[i].y;
              h.z = (h.z * inv[u]) * nw[i].z;
              h.w = (h.w * inv[u]) * nw[i].w;
              uint2 pk;
              pk.x = pack_bf16x2(h.x, h.y);
              pk.y = pack_bf16x2(h.z, h.w);
              *reinterpret_cast<uint2*>(out + c) = pk;
            }
          }
        }
      }
    }
    if (!csync(bars, cpar)) return;  // x is resident
    const uint8_t* xrow = xs + (g % p.m) * p.x_pitch;
    // ---- this CTA's rows of the phase
    for (int blk = 0; blk < n_blocks; ++blk, ++gb) {
      const RowScale rsa = row_scale(next_sa), rsb = row_scale(next_sb);
      const bool post = __any_sync(0xffffffffu, needs_post(rsa) || needs_post(rsb));
      if (blk + 1 < n_blocks) {
        bool na, nb;
        int rna, rnb;
        block_rows(blk + 1, na, nb, rna, rnb);
        next_sa = na ? __ldg(ph.scale + rna) : 0.0f;
        next_sb = nb ? __ldg(ph.scale + rnb) : 0.0f;
      }
      float acc0[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      float acc1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      for (int kc = 0; kc < ph.k_chunks; ++kc) {
        const int col0 = kc * p.kc;
        const int nbox = p.kc >> 6;
        if (!mbar_wait(&bars.full[s], rph)) return;
        const uint8_t* wg = stages + (size_t)s * p.stage_bytes + lane_off;
        const uint8_t* xc = xrow + (col0 + warp * 64 + 16 * q) * 2;
        int box = warp;
        for (; box + kConsumerWarps < nbox;
             box += 2 * kConsumerWarps, wg += 2 * kBoxStep, xc += 4 * kBoxStep) {
          if (post) {
            box_mma<true>(acc0, wg, row8, xc, rsa, rsb);
            box_mma<true>(acc1, wg + kBoxStep, row8, xc + 2 * kBoxStep, rsa, rsb);
          } else {
            box_mma<false>(acc0, wg, row8, xc, rsa, rsb);
            box_mma<false>(acc1, wg + kBoxStep, row8, xc + 2 * kBoxStep, rsa, rsb);
          }
        }
        if (box < nbox) {
          if (post) box_mma<true>(acc0, wg, row8, xc, rsa, rsb);
          else box_mma<false>(acc0, wg, row8, xc, rsa, rsb);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars.empty[s]);
        if (++s == S) {
          s = 0;
          rph ^= 1u;
        }
      }
      // hand the partial tile to the epilogue warp (double-buffered)
      const int b2 = gb & 1;
      if (gb >= 2 && !mbar_wait(&bars.epi_free[b2], ((gb >> 1) - 1) & 1)) return;
      float* mine = red + b2 * kRedFloats + warp * kTileRows * kMaxTokens;
      mine[g * kMaxTokens + 2 * q] = acc0[0] + acc1[0];
      mine[g * kMaxTokens + 2 * q + 1] = acc0[1] + acc1[1];
      mine[(g + 8) * kMaxTokens + 2 * q] = acc0[2] + acc1[2];
      mine[(g + 8) * kMaxTokens + 2 * q + 1] = acc0[3] + acc1[3];
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars.epi_full[b2]);
    }
  }
}

// Stream-order packing: source row r (for SwiGLU, half = r >= n selects the
// up rows) of output row lr = r - half·n lies in the block starting at r0 of
// the CTA owning lr; column col in chunk j = col / kc.  Its byte goes to
//   r0·mult·k + j·nr·mult·kc + (half·nr + lr - r0)·kc + col % kc
// (mult = 2 for SwiGLU, nr = rows of that block), which tiles [0, rows·k).
__global__ void chain_pack_kernel(const uint8_t* __restrict__ w, uint8_t* __restrict__ out,
                                  int64_t n, int64_t k, int mult, int kc, int grid) {
  const int out_rows = mult == 2 ? kTileRows / 2 : kTileRows;
  const int64_t units = (int64_t)mult * n * (k / 16);
  for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < units;
       u += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = u / (k / 16);
    const int64_t col = (u % (k / 16)) * 16;
    const int half = r >= n ? 1 : 0;
    const int64_t lr = r - half * n;
    int64_t c = (lr * grid) / n;
    while (c + 1 < grid && (n * (c + 1)) / grid <= lr) ++c;
    while (c > 0 && (n * c) / grid > lr) --c;
    const int64_t rb = (n * c) / grid, re = (n * (c + 1)) / grid;
    const int64_t r0 = rb + ((lr - rb) / out_rows) * out_rows;
    const int64_t nr = min((int64_t)out_rows, re - r0);
    const int64_t j = col / kc;
    const int64_t dst = r0 * mult * k + j * nr * mult * kc + (half * nr + lr - r0) * kc + col % kc;
    *reinterpret_cast<uint4*>(out + dst) = *reinterpret_cast<const uint4*>(w + r * k + col);
  }
}

}  // namespace chain

int32_t w8_chain_pack(const uint8_t* w, uint8_t* packed, int64_t n, int64_t k, bool swiglu,
                      int kc, int grid, cudaStream_t stream) {
  RXLA_REQUIRE(w && packed && n > 0 && kc > 0 && kc % 64 == 0 && k % kc == 0 && grid > 0,
               "w8 chain pack: shape");
  RXLA_REQUIRE(reinterpret_cast<uintptr_t>(w) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(packed) % 16 == 0,
               "w8 chain pack: 16-byte aligned buffers");
  int dev = 0;
  cudaGetDevice(&dev);
  chain::chain_pack_kernel<<<sm_count(dev) * 4, 256, 0, stream>>>(w, packed, n, k, swiglu ? 2 : 1,
                                                                 kc, grid);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "w8 chain pack launch");
  return RXLA_B200_OK;
}

size_t w8_chain_smem(int m, int64_t max_k, int64_t kc, int* stages) {
  const size_t fixed = chain::kHeaderBytes + 2 * w8::kRedFloats * 4 +
                       (size_t)m * (size_t)(max_k * 2 + 16);
  const size_t stage = (size_t)w8::kTileRows * kc;
  const size_t budget = 227 * 1024;
  if (fixed + 2 * stage > budget) return 0;
  const int s = (int)std::min<size_t>(chain::kStagesMax, (budget - fixed) / stage);
  if (stages) *stages = s;
  return fixed + (size_t)s * stage;
}

int32_t w8_chain(ChainParams p, cudaStream_t stream) {
  RXLA_REQUIRE(p.nphases > 0 && p.nphases <= kChainMaxPhases, "w8 chain: 1..8 phases");
  RXLA_REQUIRE(p.m >= 1 && p.m <= kChainMaxTokens, "w8 chain: 1..4 tokens");
  RXLA_REQUIRE(p.kc > 0 && p.kc % 64 == 0 && p.bar, "w8 chain: stage width / counters");
  int64_t max_k = 0;
  for (int i = 0; i < p.nphases; ++i) {
    ChainPhase& ph = p.ph[i];
    RXLA_REQUIRE(ph.w && ph.scale && ph.x && ph.n > 0 && ph.k > 0, "w8 chain: incomplete phase");
    RXLA_REQUIRE(ph.k % p.kc == 0, "w8 chain: every K must be a multiple of the stage width");
    RXLA_REQUIRE(!ph.x_norm || ph.k <= 4 * 4 * w8::kConsumerWarps * 32,
                 "w8 chain: normed input wider than the register plan");
    RXLA_REQUIRE(ph.epilogue != w8::kEpiArgmax || (ph.arg_val && ph.arg_idx && ph.arg_count &&
                                                   ph.arg_out),
                 "w8 chain: argmax phase without its buffers");
    RXLA_REQUIRE(reinterpret_cast<uintptr_t>(ph.w) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(ph.x) % 16 == 0,
                 "w8 chain: weights and x must be 16-byte aligned");
    ph.k_chunks = ph.k / p.kc;
    max_k = std::max<int64_t>(max_k, ph.k);
  }
  int stages = 0;
  const size_t smem = w8_chain_smem(p.m, max_k, p.kc, &stages);
  RXLA_REQUIRE(smem > 0, "w8 chain: shared-memory plan does not fit");
  p.stages = stages;
  p.stage_bytes = w8::kTileRows * p.kc;
  p.x_pitch = (int32_t)(max_k * 2 + 16);
  int dev = 0;
  cudaGetDevice(&dev);
  // every CTA must be resident at once (grid-wide phase counters)
  const int grid = p.grid > 0 ? p.grid : sm_count(dev);
  RXLA_REQUIRE(grid <= sm_count(dev), "w8 chain: at most one CTA per SM");
  cudaError_t e = cudaFuncSetAttribute(chain::w8_chain_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e == cudaSuccess)
    e = launch_pdl(chain::w8_chain_kernel, dim3(grid), dim3(w8::kThreads), smem, stream, p);
  if (e != cudaSuccess) return cuda_fail(e, "w8 chain launch");
  return RXLA_B200_OK;
}

}  // namespace rxla
