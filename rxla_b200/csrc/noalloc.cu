// noalloc.cu — paged decode attention for callers that cannot allocate.
//
// Some callers of this library may not call cudaMalloc at all:
//  * a handler running inside another runtime's execute callback (an XLA FFI
//    custom call, a PJRT plugin, a serving engine's step function), where that
//    runtime owns all device memory and a cudaMalloc behind its back can fail
//    or fragment its pool;
//  * latency-critical decode loops, where cudaMalloc / cudaFree can
//    synchronise the device and stall every other stream.
// Such a caller cannot provide the scratch buffer that
// rxla_b200_paged_decode_attention needs for its split-K partials. This entry
// point runs the same kernel with that scratch taken from a fixed array
// compiled into the library (kNoallocScratchBytes, held by every GPU that
// loads the library until the process exits).
//
// Set-up: the first call on each device looks up the array's device address
// with cudaGetSymbolAddress while that device is current (the array's name is
// only a host-side stand-in, not a device address), so make that first call
// before any stream capture.  Every call uses the same array: calls whose
// kernels can overlap on the GPU (different streams, no ordering) race on it.
// Each call clears the array's split counters on its stream before launching.
#include <mutex>

#include "internal.cuh"

namespace rxla {

namespace noalloc {

constexpr size_t kNoallocScratchBytes = RXLA_B200_NOALLOC_SCRATCH_BYTES;

static __device__ __align__(256) unsigned char g_scratch[kNoallocScratchBytes];

static std::mutex g_mu;
static void* g_ptr[64] = {};

// Device address of g_scratch on device `dev`, which must be current (looked
// up once per device).
static int32_t scratch_address(int dev, void** out) {
  if (dev < 0 || dev >= 64) return fail(RXLA_B200_OUT_OF_RANGE, "noalloc: device index >= 64");
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_ptr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "noalloc: cudaGetSymbolAddress(scratch)");
    g_ptr[dev] = p;
  }
  *out = g_ptr[dev];
  return RXLA_B200_OK;
}

}  // namespace noalloc
}  // namespace rxla

extern "C" int32_t rxla_b200_paged_decode_attention_noalloc(const rxla_b200_paged_decode_args* a,
                                                            void* stream) {
  using namespace rxla;
  RXLA_REQUIRE(a && a->struct_size >= sizeof(rxla_b200_paged_decode_args),
               "paged_decode_noalloc: args struct missing or too small");
  size_t need = 0;
  int32_t st = rxla_b200_paged_decode_workspace_size(a->batch, a->q_heads, a->kv_heads,
                                                     a->head_dim, a->max_context, &need);
  if (st != RXLA_B200_OK) return st;
  if (need > noalloc::kNoallocScratchBytes)
    return fail(RXLA_B200_OUT_OF_RANGE,
                "paged_decode_noalloc: this shape needs " + std::to_string(need) +
                    " bytes of scratch, more than the built-in " +
                    std::to_string(noalloc::kNoallocScratchBytes) +
                    "; use rxla_b200_paged_decode_attention with a caller workspace");
  if (a->batch == 0) return RXLA_B200_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // the array used is the current device's: a stream of another device would
  // clear that device's counters under a call it may have in flight
  int dev = 0, sdev = 0;
  RXLA_CUDA_CHECK(cudaGetDevice(&dev));
  sdev = dev;
  if (s) RXLA_CUDA_CHECK(cudaStreamGetDevice(s, &sdev));
  if (sdev != dev)
    return fail(RXLA_B200_INVALID_ARGUMENT,
                "paged_decode_noalloc: the stream belongs to device " + std::to_string(sdev) +
                    " but device " + std::to_string(dev) + " is current");
  void* scratch = nullptr;
  st = noalloc::scratch_address(dev, &scratch);
  if (st != RXLA_B200_OK) return st;
  // the split counters (the first bytes of the workspace) must start at zero
  const size_t counters = ((size_t)a->batch * a->kv_heads + 1) * 4;
  RXLA_CUDA_CHECK(cudaMemsetAsync(scratch, 0, counters, s));
  rxla_b200_paged_decode_args b = *a;
  b.workspace = scratch;
  b.workspace_bytes = noalloc::kNoallocScratchBytes;
  return attn::launch(&b, s, false);
}
