// xla_custom_call.cu — the hot path as XLA GPU custom calls (legacy ABI).
//
// rxla registers GPU custom calls through PJRT's GPU custom-call extension,
// choosing XLA's legacy untyped ABI (GpuCustomCallApi::Legacy = 0) or the
// typed FFI (crates/rxla-pjrt/src/runtime.rs:265-270, registration :395-436).
// The legacy ABI needs no XLA header: XLA calls
//
//   void handler(cudaStream_t stream, void** buffers, const char* opaque,
//                size_t opaque_len[, XlaCustomCallStatus* status])
//
// with `buffers` = the device pointers of the operands followed by those of
// the results, and `opaque` = the stablehlo.custom_call's backend_config
// bytes.  Here the backend config is one of the fixed little-endian structs
// of include/rxla_b200.h (magic, version, shape), so the lowering writes it
// once and the handler decodes it with a size / magic / version check.
//
// Failures: the status-returning form reports through
// XlaCustomCallStatusSetFailure, looked up at run time in the process (XLA
// exports it; nothing here links against XLA); the original form has no
// failure channel in XLA and leaves the message in
// rxla_b200_last_error_message() of the executing thread.  Nothing aborts.
//
// Allocation: none.  The attention's split-K scratch is the library's fixed
// allocation-free array (rxla_b200_paged_decode_attention_noalloc): a handler
// running inside XLA's execute must not cudaMalloc behind the runtime that
// owns the device memory.
#include <dlfcn.h>

#include <cstddef>
#include <cstring>

#include "internal.cuh"

// The configs are a wire format (the lowering writes them byte for byte):
// pin their size and field offsets.
static_assert(sizeof(rxla_b200_xla_linear_config) == 64, "linear config layout");
static_assert(offsetof(rxla_b200_xla_linear_config, m) == 8, "linear config layout");
static_assert(offsetof(rxla_b200_xla_linear_config, x_dtype) == 40, "linear config layout");
static_assert(offsetof(rxla_b200_xla_linear_config, eps) == 56, "linear config layout");
static_assert(sizeof(rxla_b200_xla_attention_config) == 64, "attention config layout");
static_assert(offsetof(rxla_b200_xla_attention_config, num_pages) == 32, "attention config layout");
static_assert(offsetof(rxla_b200_xla_attention_config, max_context) == 40, "attention config layout");
static_assert(offsetof(rxla_b200_xla_attention_config, scale) == 60, "attention config layout");

namespace rxla {
namespace xla {

using StatusSetFailure = void (*)(void* status, const char* message, size_t message_len);

static StatusSetFailure status_set_failure() {
  static StatusSetFailure fn = [] {
    void* sym = dlsym(RTLD_DEFAULT, "XlaCustomCallStatusSetFailure");
    return reinterpret_cast<StatusSetFailure>(sym);
  }();
  return fn;
}

// Report a failing status to XLA (status form) — the message is also the
// thread's last error message.
static void report(int32_t st, void* status) {
  if (st == RXLA_B200_OK || !status) return;
  const char* msg = rxla_b200_last_error_message();
  if (StatusSetFailure fn = status_set_failure()) fn(status, msg, std::strlen(msg));
}

template <typename T>
static int32_t decode(const char* what, const void* opaque, size_t len, uint32_t magic, T* out) {
  if (!opaque || len != sizeof(T))
    return fail(RXLA_B200_INVALID_ARGUMENT,
                std::string(what) + ": backend_config is " + std::to_string(len) +
                    " bytes, expected " + std::to_string(sizeof(T)));
  std::memcpy(out, opaque, sizeof(T));
  if (out->magic != magic)
    return fail(RXLA_B200_INVALID_ARGUMENT, std::string(what) + ": backend_config magic mismatch");
  if (out->version != 1)
    return fail(RXLA_B200_UNIMPLEMENTED,
                std::string(what) + ": backend_config version " + std::to_string(out->version) +
                    " (this library reads version 1)");
  return RXLA_B200_OK;
}

static int32_t check_linear(const rxla_b200_xla_linear_config& c) {
  RXLA_REQUIRE(c.m >= 0 && c.n >= 0 && c.k > 0 && c.group_size > 0 && c.k % c.group_size == 0,
               "xla w8a16_linear: m, n >= 0, k > 0 and a group size dividing k");
  RXLA_REQUIRE(c.epilogue >= RXLA_B200_EPI_STORE && c.epilogue <= RXLA_B200_EPI_SWIGLU,
               "xla w8a16_linear: unknown epilogue");
  RXLA_REQUIRE(c.y_dtype == RXLA_B200_BF16 || c.y_dtype == RXLA_B200_F32,
               "xla w8a16_linear: y must be BF16 or F32");
  RXLA_REQUIRE(c.fused_norm ? (c.x_dtype == RXLA_B200_F32 && c.eps > 0.0f)
                            : (c.x_dtype == RXLA_B200_BF16 || c.x_dtype == RXLA_B200_F32),
               "xla w8a16_linear: x BF16 or F32 (fused norm: an F32 h and eps > 0)");
  RXLA_REQUIRE(c.epilogue != RXLA_B200_EPI_RESIDUAL_ADD || c.y_dtype == RXLA_B200_F32,
               "xla w8a16_linear: the residual epilogue adds into an F32 y");
  return RXLA_B200_OK;
}

static int32_t check_attention(const rxla_b200_xla_attention_config& c) {
  RXLA_REQUIRE(c.batch >= 0 && c.q_heads > 0 && c.kv_heads > 0 && c.q_heads % c.kv_heads == 0 &&
                   c.head_dim > 0 && c.page_size == 16 && c.max_pages_per_seq > 0 &&
                   c.num_pages > 0 && c.max_context > 0 &&
                   c.max_context <= c.max_pages_per_seq * c.page_size && c.rotary_dim >= 0 &&
                   c.rotary_dim <= c.head_dim,
               "xla paged_decode_attention: inconsistent shape in the backend config");
  RXLA_REQUIRE(c.kv_update == RXLA_B200_KV_CLAMP || c.kv_update == RXLA_B200_KV_CHECKED,
               "xla paged_decode_attention: unknown kv_update");
  return RXLA_B200_OK;
}

static int32_t copy_if_distinct(void* dst, const void* src, size_t bytes, cudaStream_t s) {
  if (dst == src || bytes == 0) return RXLA_B200_OK;
  RXLA_REQUIRE(dst && src, "xla custom call: null state buffer");
  RXLA_CUDA_CHECK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, s));
  return RXLA_B200_OK;
}

static int32_t linear(cudaStream_t s, void** b, const void* opaque, size_t len) {
  rxla_b200_xla_linear_config c;
  int32_t st = decode("xla w8a16_linear", opaque, len, RXLA_B200_XLA_LINEAR_MAGIC, &c);
  if (st) return st;
  st = check_linear(c);
  if (st) return st;
  RXLA_REQUIRE(b, "xla w8a16_linear: null buffer array");
  int i = 0;
  const void* x = b[i++];
  const float* norm_w = c.fused_norm ? static_cast<const float*>(b[i++]) : nullptr;
  const uint8_t* w = static_cast<const uint8_t*>(b[i++]);
  const float* sc = static_cast<const float*>(b[i++]);
  const bool residual = c.epilogue == RXLA_B200_EPI_RESIDUAL_ADD;
  const void* y_in = residual ? b[i++] : nullptr;
  void* y = b[i];
  if (residual) {
    // the residual stream is an operand; the result aliases it or gets a copy first
    st = copy_if_distinct(y, y_in, (size_t)(c.m * c.n * 4), s);
    if (st) return st;
  }
  if (c.fused_norm)
    return rxla_b200_w8a16_norm_linear(static_cast<const float*>(x), norm_w, c.eps, w, sc,
                                       c.group_size, c.m, c.n, c.k, y, c.y_dtype, c.epilogue, s);
  return rxla_b200_w8a16_linear(x, c.x_dtype, w, sc, c.group_size, c.m, c.n, c.k, y, c.y_dtype,
                                c.epilogue, s);
}

static int32_t attention(cudaStream_t s, void** b, const void* opaque, size_t len) {
  rxla_b200_xla_attention_config c;
  int32_t st = decode("xla paged_decode_attention", opaque, len, RXLA_B200_XLA_ATTENTION_MAGIC, &c);
  if (st) return st;
  st = check_attention(c);
  if (st) return st;
  RXLA_REQUIRE(b, "xla paged_decode_attention: null buffer array");
  int i = 0;
  rxla_b200_paged_decode_args a{};
  a.struct_size = sizeof(a);
  a.batch = c.batch;
  a.q_heads = c.q_heads;
  a.kv_heads = c.kv_heads;
  a.head_dim = c.head_dim;
  a.q = static_cast<const uint16_t*>(b[i++]);
  a.k_new = static_cast<const uint16_t*>(b[i++]);
  a.v_new = static_cast<const uint16_t*>(b[i++]);
  a.q_row_stride = (int64_t)c.q_heads * c.head_dim;
  a.kv_row_stride = (int64_t)c.kv_heads * c.head_dim;
  if (c.has_qk_norm) {
    a.q_norm_weight = static_cast<const float*>(b[i++]);
    a.k_norm_weight = static_cast<const float*>(b[i++]);
  }
  a.norm_eps = c.norm_eps;
  if (c.rotary_dim > 0) a.inv_freq = static_cast<const float*>(b[i++]);
  a.rotary_dim = c.rotary_dim;
  a.scale = c.scale;
  const int32_t* page_table = static_cast<const int32_t*>(b[i++]);
  const int32_t* ctx_in = static_cast<const int32_t*>(b[i++]);
  const void* k_in = b[i++];
  const void* v_in = b[i++];
  a.out = static_cast<uint16_t*>(b[i++]);
  int32_t* ctx_out = static_cast<int32_t*>(b[i++]);
  void* k_out = b[i++];
  void* v_out = b[i++];
  // the cache and the lengths are state: results alias the operands (donated
  // buffers) or receive a copy before the step updates them in place
  const size_t cache_bytes = (size_t)c.num_pages * c.kv_heads * c.page_size * c.head_dim * 2;
  st = copy_if_distinct(k_out, k_in, cache_bytes, s);
  if (!st) st = copy_if_distinct(v_out, v_in, cache_bytes, s);
  if (!st) st = copy_if_distinct(ctx_out, ctx_in, (size_t)c.batch * 4, s);
  if (st) return st;
  a.k_pages = static_cast<uint16_t*>(k_out);
  a.v_pages = static_cast<uint16_t*>(v_out);
  a.num_pages = c.num_pages;
  a.page_size = c.page_size;
  a.max_pages_per_seq = c.max_pages_per_seq;
  a.page_table = page_table;
  a.ctx_lens = ctx_out;
  a.kv_update = c.kv_update;
  a.advance_ctx = 1;
  a.max_context = c.max_context;
  return rxla_b200_paged_decode_attention_noalloc(&a, s);
}

}  // namespace xla
}  // namespace rxla

extern "C" int32_t rxla_b200_xla_check_config(const char* target, const void* opaque,
                                              size_t opaque_len) {
  using namespace rxla;
  RXLA_REQUIRE(target, "xla_check_config: null target name");
  const std::string t(target);
  if (t == "rxla_b200_xla_w8a16_linear" || t == "rxla_b200_xla_w8a16_linear_status") {
    rxla_b200_xla_linear_config c;
    int32_t st = xla::decode("xla w8a16_linear", opaque, opaque_len, RXLA_B200_XLA_LINEAR_MAGIC, &c);
    return st ? st : xla::check_linear(c);
  }
  if (t == "rxla_b200_xla_paged_decode_attention" ||
      t == "rxla_b200_xla_paged_decode_attention_status") {
    rxla_b200_xla_attention_config c;
    int32_t st = xla::decode("xla paged_decode_attention", opaque, opaque_len,
                             RXLA_B200_XLA_ATTENTION_MAGIC, &c);
    return st ? st : xla::check_attention(c);
  }
  return fail(RXLA_B200_NOT_FOUND, "xla_check_config: unknown custom-call target " + t);
}

extern "C" void rxla_b200_xla_w8a16_linear(void* stream, void** buffers, const char* opaque,
                                           size_t opaque_len) {
  rxla::xla::linear(static_cast<cudaStream_t>(stream), buffers, opaque, opaque_len);
}

extern "C" void rxla_b200_xla_w8a16_linear_status(void* stream, void** buffers, const char* opaque,
                                                  size_t opaque_len, void* status) {
  rxla::xla::report(
      rxla::xla::linear(static_cast<cudaStream_t>(stream), buffers, opaque, opaque_len), status);
}

extern "C" void rxla_b200_xla_paged_decode_attention(void* stream, void** buffers,
                                                     const char* opaque, size_t opaque_len) {
  rxla::xla::attention(static_cast<cudaStream_t>(stream), buffers, opaque, opaque_len);
}

extern "C" void rxla_b200_xla_paged_decode_attention_status(void* stream, void** buffers,
                                                            const char* opaque, size_t opaque_len,
                                                            void* status) {
  rxla::xla::report(
      rxla::xla::attention(static_cast<cudaStream_t>(stream), buffers, opaque, opaque_len),
      status);
}
