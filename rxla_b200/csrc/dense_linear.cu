// dense_linear.cu — bf16-weight linear y = bf16(x) · wᵀ (crates/rxla-core/src/nn.rs:286-310),
// used for the tied bf16 LM head of a decoder whose embedding table stays bf16.
// One warp per (output row, token): 16-byte weight loads, fp32 accumulate.
#include "common.cuh"

namespace rxla {

__global__ void bf16_linear_kernel(const void* __restrict__ x, int x_f32,
                                   const __nv_bfloat16* __restrict__ w, int m, int n, int k,
                                   void* __restrict__ y, int y_f32, int epilogue) {
  pdl_wait();
  pdl_launch_dependents();
  const int warp_global = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  const bool vec = (k % 8 == 0) && (reinterpret_cast<uintptr_t>(w) % 16 == 0);
  for (int64_t it = warp_global; it < (int64_t)n * m; it += nwarps) {
    const int row = (int)(it % n);
    const int tok = (int)(it / n);
    const __nv_bfloat16* wr = w + (int64_t)row * k;
    float acc = 0.0f;
    auto xval = [&](int c) -> float {
      float v = x_f32 ? static_cast<const float*>(x)[(int64_t)tok * k + c]
                      : __bfloat162float(static_cast<const __nv_bfloat16*>(x)[(int64_t)tok * k + c]);
      return bf16_round(v);
    };
    if (vec) {
      for (int c = lane * 8; c < k; c += 256) {
        uint4 wv = *reinterpret_cast<const uint4*>(wr + c);
        const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc += xval(c + 2 * j) * bf16_lo(ww[j]);
          acc += xval(c + 2 * j + 1) * bf16_hi(ww[j]);
        }
      }
    } else {
      for (int c = lane; c < k; c += 32) acc += xval(c) * __bfloat162float(wr[c]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) {
      const int64_t o = (int64_t)tok * n + row;
      if (epilogue == RXLA_B200_EPI_RESIDUAL_ADD) {
        float* yy = static_cast<float*>(y);
        yy[o] = yy[o] + bf16_round(acc);
      } else if (y_f32) {
        static_cast<float*>(y)[o] = acc;
      } else {
        static_cast<__nv_bfloat16*>(y)[o] = __float2bfloat16_rn(acc);
      }
    }
  }
}

}  // namespace rxla

extern "C" int32_t rxla_b200_bf16_linear(const void* x, int32_t x_dtype, const uint16_t* weight,
                                         int64_t m, int64_t n, int64_t k, void* y,
                                         int32_t y_dtype, int32_t epilogue, void* stream) {
  using namespace rxla;
  RXLA_REQUIRE(m >= 0 && n >= 0 && k > 0 && m <= INT32_MAX && n <= INT32_MAX && k <= INT32_MAX,
               "bf16_linear: bad shape");
  RXLA_REQUIRE(x_dtype == RXLA_B200_BF16 || x_dtype == RXLA_B200_F32, "bf16_linear: x dtype");
  RXLA_REQUIRE(y_dtype == RXLA_B200_BF16 || y_dtype == RXLA_B200_F32, "bf16_linear: y dtype");
  RXLA_REQUIRE(epilogue == RXLA_B200_EPI_STORE || epilogue == RXLA_B200_EPI_RESIDUAL_ADD,
               "bf16_linear: epilogue must be STORE or RESIDUAL_ADD");
  RXLA_REQUIRE(epilogue != RXLA_B200_EPI_RESIDUAL_ADD || y_dtype == RXLA_B200_F32,
               "bf16_linear: the residual epilogue adds into an F32 y");
  if (m == 0 || n == 0) return RXLA_B200_OK;
  RXLA_REQUIRE(x && weight && y, "bf16_linear: null pointer");
  int dev = 0;
  cudaGetDevice(&dev);
  const int64_t warps = n * m;
  int blocks = (int)std::min<int64_t>((warps + 7) / 8, (int64_t)sm_count(dev) * 16);
  cudaError_t e = launch_pdl(bf16_linear_kernel, dim3(blocks), dim3(256), 0,
                             static_cast<cudaStream_t>(stream), x, (int)(x_dtype == RXLA_B200_F32),
                             reinterpret_cast<const __nv_bfloat16*>(weight), (int)m, (int)n,
                             (int)k, y, (int)(y_dtype == RXLA_B200_F32), (int)epilogue);
  if (e != cudaSuccess) return cuda_fail(e, "bf16_linear launch");
  return RXLA_B200_OK;
}
