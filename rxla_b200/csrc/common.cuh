// common.cuh — shared host/device helpers of librxla_b200 (sm_100a only).
//
// Device side: bf16 packing, mbarrier / bulk-copy (TMA engine) wrappers,
// programmatic dependent launch (PDL) controls, and bounded waits: every spin
// on an mbarrier gives up after kWaitTimeoutNs of %globaltimer time, records
// RXLA_B200_DEADLINE_EXCEEDED in the device status word and lets the kernel
// return, so a lost wake-up never hangs the GPU.
//
// Host side: thread-local error message, status helpers, PDL launch helper.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/rxla_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "librxla_b200 is built for sm_100a only"
#endif

namespace rxla {

// ------------------------------------------------------------------ host

void set_error(const std::string& msg);
int32_t fail(int32_t code, const std::string& msg);
int32_t cuda_fail(cudaError_t err, const char* what);
int sm_count(int device);

#define RXLA_CUDA_CHECK(expr)                                   \
  do {                                                          \
    cudaError_t _e = (expr);                                    \
    if (_e != cudaSuccess) return ::rxla::cuda_fail(_e, #expr); \
  } while (0)

#define RXLA_REQUIRE(cond, msg)                                                  \
  do {                                                                           \
    if (!(cond)) return ::rxla::fail(RXLA_B200_INVALID_ARGUMENT, std::string(msg)); \
  } while (0)

// Launch `kernel` with programmatic stream serialization, so its prologue
// (weight prefetch) overlaps the tail of the previous kernel on the stream.
template <typename Kernel, typename... Args>
cudaError_t launch_pdl(Kernel kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// The same launch with a thread-block cluster of `cluster_x` CTAs along x
// (gridDim.x a multiple of it).
template <typename Kernel, typename... Args>
cudaError_t launch_pdl_cluster(Kernel kernel, dim3 grid, dim3 block, size_t smem,
                               cudaStream_t stream, unsigned cluster_x, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster_x;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Device status word (per device): 0 = fine, else a negative rxla_b200_status.
int32_t read_device_status(bool reset);

// ------------------------------------------------------------------ device

// Default bounded-wait budget.  Kernels here last microseconds; a wait this
// long means a lost arrival, never a slow peer.  rxla_b200_set_wait_timeout
// changes it per device.
constexpr unsigned long long kWaitTimeoutNs = 4000000000ull;
constexpr int64_t kMinWaitTimeoutNs = 1000000;      // 1 ms
constexpr int64_t kMaxWaitTimeoutNs = 60000000000;  // 60 s

}  // namespace rxla

// Device status word of this library on each device (single translation unit).
__device__ int g_rxla_device_status = 0;
// Bounded-wait budget of every spin in this library's kernels on each device
// (ns of %globaltimer); set by rxla_b200_set_wait_timeout.
__device__ unsigned long long g_rxla_wait_timeout_ns = rxla::kWaitTimeoutNs;

namespace rxla {

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// The current wait budget (read only once a wait has spun for a while).
__device__ __forceinline__ unsigned long long wait_timeout_ns() {
  return *reinterpret_cast<volatile unsigned long long*>(&g_rxla_wait_timeout_ns);
}

__device__ __forceinline__ void record_device_error(int code) {
  atomicCAS(&g_rxla_device_status, 0, code);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete; false after the
// timeout (the status word is set).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer() - t0 > wait_timeout_ns()) {
      record_device_error(RXLA_B200_DEADLINE_EXCEEDED);
      return false;
    }
  }
}

// L2 policy for data read exactly once (streamed weights): evict first.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// 1-D bulk copy global -> shared on the TMA engine, completing on `bar`.
// dst, src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void bulk_g2s_nohint(void* dst, const void* src, uint32_t bytes,
                                                uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Bytes the NEXT kernel of a chain will read first (up to two contiguous
// segments, e.g. the gate and up halves of a fused weight).  A kernel that is
// done issuing its own loads pulls its share of them into L2, so the HBM
// stays busy while it drains and the next kernel's first tiles hit in L2.
struct L2Prefetch {
  const void* seg[2];
  int64_t bytes[2];
  int32_t nseg;
  int32_t per_cta;  // bytes per CTA over all segments
};

// CTA `cta` of `ctas` prefetches the start of its proportional share of each
// segment (the next kernel partitions its rows the same way).  One thread.
__device__ __forceinline__ void l2_prefetch_share(const L2Prefetch& pf, int cta, int ctas) {
  for (int i = 0; i < pf.nseg && i < 2; ++i) {
    const int64_t total = pf.bytes[i];
    if (!pf.seg[i] || total <= 0) continue;
    int64_t start = (total * cta) / ctas;
    int64_t end = (total * (cta + 1)) / ctas;
    end = min(end, start + (int64_t)(pf.per_cta / pf.nseg));
    start &= ~(int64_t)15;
    end &= ~(int64_t)15;
    const uint8_t* base = static_cast<const uint8_t*>(pf.seg[i]);
    for (int64_t off = start; off < end; off += 32768) {
      const uint32_t len = (uint32_t)min((int64_t)32768, end - off);
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(base + off), "r"(len)
                   : "memory");
    }
  }
}

// System-scope flag accesses of the peer all-reduces (flags live in
// IPC-mapped memory that other GPUs write over NVLink).
__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_relaxed_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Wait until *flag >= target; false after the timeout (the status word is set).
__device__ __forceinline__ bool flag_wait_geq(const uint64_t* flag, uint64_t target) {
  if (ld_acquire_sys(flag) >= target) return true;
  const uint64_t t0 = globaltimer();
  while (ld_acquire_sys(flag) < target) {
    if (globaltimer() - t0 > wait_timeout_ns()) {
      record_device_error(RXLA_B200_DEADLINE_EXCEEDED);
      return false;
    }
  }
  return true;
}

// Programmatic dependent launch: wait for the previous grid's results, and
// allow the next grid to start its prologue.  Every kernel of this library
// triggers its dependents only after its own griddepcontrol.wait, so when a
// grid starts, every grid before the one directly preceding it has completed:
// code before griddepcontrol.wait overlaps only that one grid, and may read
// anything the grids before it wrote.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// u8 byte i of w (value b, signed weight q = b - 128) -> exact float q.
// 0x4B0000bb is 2^23 + b; subtracting 2^23 + 128 leaves q exactly.
template <int I>
__device__ __forceinline__ float u8_to_q(uint32_t w) {
  return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u | I)) - 8388736.0f;
}

// Four u8 weights (one 32-bit word) -> two bf16x2 registers of exact q values:
// lo = (q0, q1), hi = (q2, q3).
__device__ __forceinline__ void u8x4_to_bf16x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  lo = pack_bf16x2(u8_to_q<0>(w), u8_to_q<1>(w));
  hi = pack_bf16x2(u8_to_q<2>(w), u8_to_q<3>(w));
}

// D += A(16x16 bf16, row) * B(16x8 bf16, col), fp32 accumulate.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4],
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float silu(float g) {
  // x * sigmoid(x) with a nonpositive exponent argument
  // (crates/rxla-core/src/ops.rs:336-341)
  float e = expf(-fabsf(g));
  float sig = g >= 0.0f ? 1.0f / (1.0f + e) : e / (1.0f + e);
  return g * sig;
}

}  // namespace rxla
