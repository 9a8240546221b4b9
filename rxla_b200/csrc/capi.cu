// capi.cu — library-level entry points: errors, device info, small fused ops.
#include <mutex>
#include <string>

#include "common.cuh"

namespace rxla {

static thread_local std::string t_last_error;

void set_error(const std::string& msg) { t_last_error = msg; }

int32_t fail(int32_t code, const std::string& msg) {
  t_last_error = msg;
  return code;
}

int32_t cuda_fail(cudaError_t err, const char* what) {
  t_last_error = std::string(what) + ": " + cudaGetErrorName(err) + " (" +
                 cudaGetErrorString(err) + ")";
  return err == cudaErrorMemoryAllocation ? RXLA_B200_RESOURCE_EXHAUSTED : RXLA_B200_UNAVAILABLE;
}

int sm_count(int device) {
  static int cache[64] = {};
  if (device < 0 || device >= 64) return 148;
  if (cache[device] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || v <= 0)
      v = 148;
    cache[device] = v;
  }
  return cache[device];
}

int32_t read_device_status(bool reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_rxla_device_status, sizeof(int)) != cudaSuccess)
    return RXLA_B200_UNAVAILABLE;
  if (reset && v != 0) {
    int z = 0;
    cudaMemcpyToSymbol(g_rxla_device_status, &z, sizeof(int));
  }
  return v;
}

// ------------------------------------------------------------ RMSNorm -> bf16
// One CTA per row: f32 sum of squares, then x * rsqrt(mean + eps) * w rounded
// to bf16 (crates/rxla-core/src/ops.rs:929-945 followed by the consuming
// linear's bf16 cast).
__global__ void rms_norm_bf16_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                     int64_t width, float eps, __nv_bfloat16* __restrict__ y) {
  pdl_wait();
  pdl_launch_dependents();
  const float* xr = x + blockIdx.x * width;
  __nv_bfloat16* yr = y + blockIdx.x * width;
  // rows of up to 8 float4 per thread are held in registers, all loads issued
  // before any is used (one round trip); wider or unaligned rows use a loop
  constexpr int kV = 8;
  const bool regs = width % 4 == 0 && width <= (int64_t)kV * 4 * blockDim.x &&
                    (reinterpret_cast<uintptr_t>(xr) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(w) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(yr) & 7) == 0;
  float4 v[kV];
  float ss = 0.0f;
  if (regs) {
#pragma unroll
    for (int i = 0; i < kV; ++i) {
      const int64_t c = ((int64_t)threadIdx.x + (int64_t)i * blockDim.x) * 4;
      v[i] = c < width ? *reinterpret_cast<const float4*>(xr + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int i = 0; i < kV; ++i) ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
  } else {
    for (int64_t c = threadIdx.x; c < width; c += blockDim.x) ss += xr[c] * xr[c];
  }
  __shared__ float red[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float mean = red[0] / (float)width;
  const float rs = 1.0f / sqrtf(mean + eps);
  if (regs) {
#pragma unroll
    for (int i = 0; i < kV; ++i) {
      const int64_t c = ((int64_t)threadIdx.x + (int64_t)i * blockDim.x) * 4;
      if (c < width) {
        const float4 ww = *reinterpret_cast<const float4*>(w + c);
        uint2 pk;
        pk.x = pack_bf16x2((v[i].x * rs) * ww.x, (v[i].y * rs) * ww.y);
        pk.y = pack_bf16x2((v[i].z * rs) * ww.z, (v[i].w * rs) * ww.w);
        *reinterpret_cast<uint2*>(yr + c) = pk;
      }
    }
  } else {
    for (int64_t c = threadIdx.x; c < width; c += blockDim.x)
      yr[c] = __float2bfloat16_rn((xr[c] * rs) * w[c]);
  }
}

// ------------------------------------------------------------------- argmax
// First index of the maximum (ties -> lowest index), one CTA per row.
// `advance` (optional): ctx_lens[row] += 1 once the row's token is chosen —
// the decoder runner's end-of-step position update.
__global__ void argmax_kernel(const float* __restrict__ logits, int64_t vocab,
                              int32_t* __restrict__ out, int32_t* __restrict__ advance) {
  pdl_wait();
  pdl_launch_dependents();
  const float* r = logits + blockIdx.x * vocab;
  float best = -INFINITY;
  int32_t idx = 0x7fffffff;
  auto take = [&](float v, int32_t c) {
    if (v > best || (v == best && c < idx)) {
      best = v;
      idx = c;
    }
  };
  if (vocab % 4 == 0 && (reinterpret_cast<uintptr_t>(r) & 15) == 0) {
    // float4 loads, four per thread in flight before they are compared
    const int64_t nq = vocab / 4;
    const float4* r4 = reinterpret_cast<const float4*>(r);
    int64_t q = threadIdx.x;
    for (; q + 3 * (int64_t)blockDim.x < nq; q += 4 * (int64_t)blockDim.x) {
      float4 v[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = r4[q + j * (int64_t)blockDim.x];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int32_t c = (int32_t)(4 * (q + j * (int64_t)blockDim.x));
        take(v[j].x, c);
        take(v[j].y, c + 1);
        take(v[j].z, c + 2);
        take(v[j].w, c + 3);
      }
    }
    for (; q < nq; q += blockDim.x) {
      const float4 v = r4[q];
      const int32_t c = (int32_t)(4 * q);
      take(v.x, c);
      take(v.y, c + 1);
      take(v.z, c + 2);
      take(v.w, c + 3);
    }
  } else {
    for (int64_t c = threadIdx.x; c < vocab; c += blockDim.x) take(r[c], (int32_t)c);
  }
  __shared__ float sb[32];
  __shared__ int32_t si[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ob = __shfl_xor_sync(0xffffffffu, best, o);
    int32_t oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ob > best || (ob == best && oi < idx)) {
      best = ob;
      idx = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    sb[threadIdx.x >> 5] = best;
    si[threadIdx.x >> 5] = idx;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int nw = blockDim.x >> 5;
    best = threadIdx.x < nw ? sb[threadIdx.x] : -INFINITY;
    idx = threadIdx.x < nw ? si[threadIdx.x] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float ob = __shfl_xor_sync(0xffffffffu, best, o);
      int32_t oi = __shfl_xor_sync(0xffffffffu, idx, o);
      if (ob > best || (ob == best && oi < idx)) {
        best = ob;
        idx = oi;
      }
    }
    if (threadIdx.x == 0) {
      out[blockIdx.x] = idx == 0x7fffffff ? 0 : idx;
      if (advance) advance[blockIdx.x] += 1;
    }
  }
}

// ------------------------------------------------------ sigmoid output gate
// y[r, c] = bf16(x[r, c] · sigmoid(gate[r, c])), the output gate of Qwen3.5's
// full-attention layers (crates/rxla-models/src/qwen3_5/layers.rs:50-55,
// 94-95): the gate half of q_proj, through the logistic, times the attended
// values, in f32, rounded once for o_proj's bf16 input.
__global__ void sigmoid_gate_kernel(const uint16_t* __restrict__ x, int64_t x_ld,
                                    const uint16_t* __restrict__ g, int64_t g_ld, int64_t width,
                                    uint16_t* __restrict__ y, int64_t y_ld) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t r = blockIdx.y;
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < width;
       c += (int64_t)gridDim.x * blockDim.x) {
    const float xv = __uint_as_float((uint32_t)x[r * x_ld + c] << 16);
    const float gv = __uint_as_float((uint32_t)g[r * g_ld + c] << 16);
    // logistic with a nonpositive exponent argument (crates/rxla-core/src/ops.rs:332-337)
    const float e = expf(-fabsf(gv));
    const float sig = gv >= 0.0f ? 1.0f / (1.0f + e) : e / (1.0f + e);
    y[r * y_ld + c] = __bfloat16_as_ushort(__float2bfloat16_rn(xv * sig));
  }
}

// ------------------------------------------------------------ W8 embedding
// out[r, c] = f32(weight[id_r, c] - 128) · scale[id_r, c / group]: the W8
// token embedding of qwen3_5/mod.rs:134-155 (take, cast, -128, × group
// scale), one CTA per row, ids outside [0, vocab) give zero rows.
__global__ void w8_embedding_kernel(const int32_t* __restrict__ ids, const uint8_t* __restrict__ w,
                                    const float* __restrict__ scale, int64_t vocab, int64_t hidden,
                                    int64_t group, float* __restrict__ out) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t r = blockIdx.x;
  const int32_t id = ids[r];
  const bool ok = id >= 0 && id < vocab;
  const int64_t groups = hidden / group;
  for (int64_t c = threadIdx.x; c < hidden; c += blockDim.x) {
    float v = 0.0f;
    if (ok) v = (float)((int32_t)w[(int64_t)id * hidden + c] - 128) * scale[(int64_t)id * groups + c / group];
    out[r * hidden + c] = v;
  }
}

}  // namespace rxla

extern "C" int32_t rxla_b200_abi_version(void) { return RXLA_B200_ABI_VERSION; }

extern "C" const char* rxla_b200_last_error_message(void) { return rxla::t_last_error.c_str(); }

extern "C" int32_t rxla_b200_device_info(int32_t device, int32_t* sm, int32_t* major,
                                         int32_t* minor) {
  cudaDeviceProp prop;
  RXLA_CUDA_CHECK(cudaGetDeviceProperties(&prop, device));
  if (sm) *sm = prop.multiProcessorCount;
  if (major) *major = prop.major;
  if (minor) *minor = prop.minor;
  return RXLA_B200_OK;
}

extern "C" int32_t rxla_b200_device_status(int32_t reset) {
  return rxla::read_device_status(reset != 0);
}

extern "C" int32_t rxla_b200_set_wait_timeout(int64_t ns) {
  using namespace rxla;
  RXLA_REQUIRE(ns >= kMinWaitTimeoutNs && ns <= kMaxWaitTimeoutNs,
               "set_wait_timeout: the budget must lie in [1 ms, 60 s]");
  const unsigned long long v = (unsigned long long)ns;
  RXLA_CUDA_CHECK(cudaMemcpyToSymbol(g_rxla_wait_timeout_ns, &v, sizeof(v)));
  return RXLA_B200_OK;
}

extern "C" int32_t rxla_b200_get_wait_timeout(int64_t* ns) {
  using namespace rxla;
  RXLA_REQUIRE(ns, "get_wait_timeout: null argument");
  unsigned long long v = 0;
  RXLA_CUDA_CHECK(cudaMemcpyFromSymbol(&v, g_rxla_wait_timeout_ns, sizeof(v)));
  *ns = (int64_t)v;
  return RXLA_B200_OK;
}

namespace rxla {
// One thread waits through the library's bounded-wait helpers: kind 0 on a
// fresh mbarrier that nothing arrives on, kind 1 for *flag >= target.
__global__ void bounded_wait_check_kernel(int kind, const uint64_t* flag, uint64_t target) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  if (kind == 0) {
    mbar_init(&bar, 1);
    fence_mbarrier_init();
    mbar_wait(&bar, 0);
  } else {
    flag_wait_geq(flag, target);
  }
}
}  // namespace rxla

extern "C" int32_t rxla_b200_bounded_wait_check(int32_t kind, const uint64_t* flag,
                                                uint64_t target, void* stream) {
  using namespace rxla;
  RXLA_REQUIRE(kind == 0 || kind == 1, "bounded_wait_check: kind must be 0 or 1");
  RXLA_REQUIRE(kind == 0 || (flag && (reinterpret_cast<uintptr_t>(flag) & 7) == 0),
               "bounded_wait_check: kind 1 needs an 8-byte aligned device flag");
  if (kind == 1) {
    // the kernel loads the flag: ordinary host memory would be an illegal
    // address there, so refuse it here
    cudaPointerAttributes pa{};
    const cudaError_t e = cudaPointerGetAttributes(&pa, flag);
    if (e != cudaSuccess) cudaGetLastError();
    RXLA_REQUIRE(e == cudaSuccess && pa.type != cudaMemoryTypeUnregistered,
                 "bounded_wait_check: the flag must be device, managed or pinned host memory");
  }
  bounded_wait_check_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(kind, flag, target);
  RXLA_CUDA_CHECK(cudaGetLastError());
  return RXLA_B200_OK;
}

extern "C" int32_t rxla_b200_rms_norm_bf16(const float* x, const float* weight, int64_t rows,
                                           int64_t width, float eps, uint16_t* y, void* stream) {
  using namespace rxla;
  RXLA_REQUIRE(rows >= 0 && width > 0, "rms_norm_bf16: rows >= 0 and width > 0");
  RXLA_REQUIRE(eps > 0.0f && eps == eps && eps < INFINITY,
               "rms_norm_bf16: epsilon must be finite and positive (ops.rs:930)");
  if (rows == 0) return RXLA_B200_OK;
  RXLA_REQUIRE(x && weight && y, "rms_norm_bf16: null pointer");
  cudaError_t e = launch_pdl(rms_norm_bf16_kernel, dim3((unsigned)rows), dim3(256), 0,
                             static_cast<cudaStream_t>(stream), x, weight, width, eps,
                             reinterpret_cast<__nv_bfloat16*>(y));
  if (e != cudaSuccess) return cuda_fail(e, "rms_norm_bf16 launch");
  return RXLA_B200_OK;
}

extern "C" int32_t rxla_b200_argmax(const float* logits, int64_t rows, int64_t vocab,
                                    int32_t* out, void* stream) {
  using namespace rxla;
  RXLA_REQUIRE(rows >= 0 && vocab > 0 && vocab <= INT32_MAX, "argmax: bad shape");
  if (rows == 0) return RXLA_B200_OK;
  RXLA_REQUIRE(logits && out, "argmax: null pointer");
  cudaError_t e = launch_pdl(argmax_kernel, dim3((unsigned)rows), dim3(1024), 0,
                             static_cast<cudaStream_t>(stream), logits, vocab, out,
                             (int32_t*)nullptr);
  if (e != cudaSuccess) return cuda_fail(e, "argmax launch");
  return RXLA_B200_OK;
}

extern "C" int32_t rxla_b200_sigmoid_gate(const uint16_t* x, int64_t x_row_stride,
                                          const uint16_t* gate, int64_t gate_row_stride,
                                          int64_t rows, int64_t width, uint16_t* y,
                                          int64_t y_row_stride, void* stream) {
  using namespace rxla;
  RXLA_REQUIRE(rows >= 0 && width >= 0 && rows <= 65535, "sigmoid_gate: bad shape");
  if (rows == 0 || width == 0) return RXLA_B200_OK;
  RXLA_REQUIRE(x && gate && y, "sigmoid_gate: null pointer");
  RXLA_REQUIRE(x_row_stride >= width && gate_row_stride >= width && y_row_stride >= width,
               "sigmoid_gate: a row stride is shorter than the row");
  const unsigned bx = (unsigned)std::min<int64_t>((width + 255) / 256, 64);
  cudaError_t e = launch_pdl(sigmoid_gate_kernel, dim3(bx, (unsigned)rows), dim3(256), 0,
                             static_cast<cudaStream_t>(stream), x, x_row_stride, gate,
                             gate_row_stride, width, y, y_row_stride);
  if (e != cudaSuccess) return cuda_fail(e, "sigmoid_gate launch");
  return RXLA_B200_OK;
}

extern "C" int32_t rxla_b200_w8_embedding(const int32_t* ids, int64_t rows, const uint8_t* weight,
                                          const float* scale, int64_t vocab, int64_t hidden,
                                          int64_t group_size, float* out, void* stream) {
  using namespace rxla;
  RXLA_REQUIRE(rows >= 0 && rows <= INT32_MAX && vocab > 0 && hidden > 0 && group_size > 0 &&
                   hidden % group_size == 0,
               "w8_embedding: bad shape (group_size must divide hidden)");
  if (rows == 0) return RXLA_B200_OK;
  RXLA_REQUIRE(ids && weight && scale && out, "w8_embedding: null pointer");
  cudaError_t e = launch_pdl(w8_embedding_kernel, dim3((unsigned)rows), dim3(256), 0,
                             static_cast<cudaStream_t>(stream), ids, weight, scale, vocab, hidden,
                             group_size, out);
  if (e != cudaSuccess) return cuda_fail(e, "w8_embedding launch");
  return RXLA_B200_OK;
}
