// librxla_b200.cu — single translation unit of the library (one device
// module, so the device status word and kernels share one symbol space).
#include <algorithm>

#include "capi.cu"
#include "w8_linear.cu"
#include "w8_gemm.cu"
#include "w8_gemm_dec.cu"
#include "dense_linear.cu"
#include "attention.cu"
#include "decoder.cu"
#include "loader.cu"
#include "comm.cu"
#include "noalloc.cu"
#include "xla_custom_call.cu"
#include "gated_delta.cu"
