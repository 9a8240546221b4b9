// comm.cu — tensor-parallel communicator over NCCL (NVLink 5 / NVSwitch).
//
// Replaces rxla's PJRT distributed client + KV-store rendezvous
// (crates/rxla-pjrt/src/distributed.rs:40-120): rank 0 creates an id, the
// caller moves the bytes to the other ranks through any host store, every
// rank initialises.  NCCL is loaded with dlopen (libnccl.so.2 — the copy
// torch already loaded, when there is one), so the library has no link-time
// NCCL dependency.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <vector>

#include "internal.cuh"

namespace rxla {
namespace p2p {
constexpr int kMaxRanks = 8;
constexpr int kChunk = 2048;  // floats of the all-reduce per CTA
constexpr int kThreads = 256;
constexpr int kFusedCtas = 1024;  // flag slots for grids of one CTA per SM

// One rank's IPC-shared all-reduce buffer: two slots of [world][cap] f32
// partials (alternating per call, so a rank may start the next all-reduce
// while a slower peer still reads the last one), then [world][max_ctas]
// arrival flags (monotonic epochs).
struct Layout {
  int64_t cap = 0;  // floats per (slot, rank)
  int max_ctas = 0;
  size_t data_bytes() const { return (size_t)2 * kMaxRanks * cap * 4; }
  size_t bytes() const { return data_bytes() + (size_t)kMaxRanks * max_ctas * 8; }
};

struct Args {
  const float* partial;  // this rank's partial sums [count]
  float* out;            // sum (STORE) or the f32 residual (RESIDUAL_BF16)
  int64_t count, cap;
  int32_t rank, world, max_ctas, residual;
  uint8_t* peer[kMaxRanks];  // every rank's buffer, mapped here (own one included)
  uint64_t* epoch;           // [max_ctas] per-CTA call counter of this rank
};
}  // namespace p2p
}  // namespace rxla

struct rxla_b200_comm {
  ncclComm_t nccl = nullptr;
  int rank = 0, world = 1, device = 0;
  // one-shot peer all-reduce (rxla_b200_comm_p2p_enable)
  rxla::p2p::Layout p2p;
  uint8_t* p2p_local = nullptr;
  uint8_t* p2p_peer[rxla::p2p::kMaxRanks] = {};
  uint64_t* p2p_epoch = nullptr;
};

namespace rxla {
namespace comm {

struct Nccl {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  bool ok = false;
};

static Nccl& nccl() {
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    n.get_unique_id = reinterpret_cast<decltype(n.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    n.init_rank = reinterpret_cast<decltype(n.init_rank)>(dlsym(h, "ncclCommInitRank"));
    n.destroy = reinterpret_cast<decltype(n.destroy)>(dlsym(h, "ncclCommDestroy"));
    n.all_reduce = reinterpret_cast<decltype(n.all_reduce)>(dlsym(h, "ncclAllReduce"));
    n.all_gather = reinterpret_cast<decltype(n.all_gather)>(dlsym(h, "ncclAllGather"));
    n.error_string = reinterpret_cast<decltype(n.error_string)>(dlsym(h, "ncclGetErrorString"));
    n.ok = n.get_unique_id && n.init_rank && n.destroy && n.all_reduce && n.all_gather &&
           n.error_string;
  });
  return n;
}

static int32_t nccl_fail(ncclResult_t r, const char* what) {
  return fail(RXLA_B200_UNAVAILABLE,
              std::string(what) + ": " + (nccl().error_string ? nccl().error_string(r) : "nccl"));
}

}  // namespace comm

namespace p2p {

// CTA c owns floats [c·kChunk, (c+1)·kChunk): it pushes this rank's partial of
// that range into slot (e & 1), row `rank`, of every rank's buffer (NVLink
// stores), publishes epoch e in each rank's flag [rank][c], waits (bounded)
// until every rank's flag [q][c] reached e in its own buffer, then sums the
// rows in rank order 0..world-1 (the same order on every rank, so the result
// is bit-identical everywhere) and stores the sum, or adds bf16(sum) to the
// f32 residual (the row-parallel epilogue of o_proj / down_proj).
__global__ void __launch_bounds__(kThreads) allreduce_kernel(const Args a) {
  pdl_wait();  // the partials come from the previous kernel
  pdl_launch_dependents();
  const int c = blockIdx.x;
  const uint64_t e = a.epoch[c] + 1;
  const int slot = (int)(e & 1);
  const int64_t lo = (int64_t)c * kChunk;
  const int64_t n = min((int64_t)kChunk, a.count - lo);
  const size_t data_bytes = (size_t)2 * kMaxRanks * a.cap * 4;
  const bool vec = (a.count % 4) == 0;
  // push
  for (int q = 0; q < a.world; ++q) {
    float* dst = reinterpret_cast<float*>(a.peer[q]) + ((int64_t)slot * kMaxRanks + a.rank) * a.cap + lo;
    if (vec) {
      for (int64_t i = threadIdx.x * 4; i < n; i += kThreads * 4)
        *reinterpret_cast<float4*>(dst + i) = *reinterpret_cast<const float4*>(a.partial + lo + i);
    } else {
      for (int64_t i = threadIdx.x; i < n; i += kThreads) dst[i] = a.partial[lo + i];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();  // cumulative over the CTA's pushes (ordered by the barrier)
    for (int q = 0; q < a.world; ++q)
      st_relaxed_sys(reinterpret_cast<uint64_t*>(a.peer[q] + data_bytes) +
                         (int64_t)a.rank * a.max_ctas + c,
                     e);
  }
  // wait for every rank's push of this range
  __shared__ int ok;
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  if (threadIdx.x < a.world) {
    const uint64_t* flag = reinterpret_cast<const uint64_t*>(a.peer[a.rank] + data_bytes) +
                           (int64_t)threadIdx.x * a.max_ctas + c;
    if (!flag_wait_geq(flag, e)) ok = 0;
  }
  __syncthreads();
  if (!ok) return;
  const float* rows = reinterpret_cast<const float*>(a.peer[a.rank]) + (int64_t)slot * kMaxRanks * a.cap + lo;
  if (vec) {
    for (int64_t i = threadIdx.x * 4; i < n; i += kThreads * 4) {
      float4 acc = __ldcv(reinterpret_cast<const float4*>(rows + i));
      for (int q = 1; q < a.world; ++q) {
        const float4 v = __ldcv(reinterpret_cast<const float4*>(rows + (int64_t)q * a.cap + i));
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      float4* o = reinterpret_cast<float4*>(a.out + lo + i);
      if (a.residual) {
        float4 h = *o;
        h.x += bf16_round(acc.x);
        h.y += bf16_round(acc.y);
        h.z += bf16_round(acc.z);
        h.w += bf16_round(acc.w);
        *o = h;
      } else {
        *o = acc;
      }
    }
  } else {
    for (int64_t i = threadIdx.x; i < n; i += kThreads) {
      float acc = __ldcv(rows + i);
      for (int q = 1; q < a.world; ++q) acc += __ldcv(rows + (int64_t)q * a.cap + i);
      if (a.residual) a.out[lo + i] += bf16_round(acc);
      else a.out[lo + i] = acc;
    }
  }
  if (threadIdx.x == 0) a.epoch[c] = e;
}

}  // namespace p2p

// The peer all-reduce of the decoder's row-parallel linears: out = Σ partial
// (residual false) or out += bf16(Σ partial) (residual true).  Falls back to
// NCCL + a residual kernel when the comm has no peer buffers.
bool comm_has_p2p(const rxla_b200_comm* c) { return c && c->p2p_local != nullptr; }
int64_t comm_p2p_capacity(const rxla_b200_comm* c) { return comm_has_p2p(c) ? c->p2p.cap : 0; }

bool comm_p2p_view(const rxla_b200_comm* c, P2pView* out) {
  static_assert(kP2pMaxRanks == p2p::kMaxRanks, "peer buffer layout");
  if (!comm_has_p2p(c) || !out) return false;
  *out = P2pView{};
  for (int q = 0; q < c->world; ++q) out->peer[q] = c->p2p_peer[q];
  out->epoch = c->p2p_epoch;
  out->cap = c->p2p.cap;
  out->rank = c->rank;
  out->world = c->world;
  out->max_ctas = c->p2p.max_ctas;
  return true;
}

int32_t comm_p2p_allreduce(rxla_b200_comm* c, const float* partial, float* out, int64_t count,
                           bool residual, cudaStream_t s) {
  RXLA_REQUIRE(c && c->p2p_local, "p2p allreduce: not enabled on this comm");
  RXLA_REQUIRE(count >= 0 && count <= c->p2p.cap, "p2p allreduce: count above the reserved capacity");
  RXLA_REQUIRE(partial && out, "p2p allreduce: null buffer");
  if (count == 0) return RXLA_B200_OK;
  p2p::Args a{};
  a.partial = partial;
  a.out = out;
  a.count = count;
  a.cap = c->p2p.cap;
  a.rank = c->rank;
  a.world = c->world;
  a.max_ctas = c->p2p.max_ctas;
  a.residual = residual ? 1 : 0;
  for (int q = 0; q < c->world; ++q) a.peer[q] = c->p2p_peer[q];
  a.epoch = c->p2p_epoch;
  const int grid = (int)((count + p2p::kChunk - 1) / p2p::kChunk);
  cudaError_t e = launch_pdl(p2p::allreduce_kernel, dim3(grid), dim3(p2p::kThreads), 0, s, a);
  if (e != cudaSuccess) return cuda_fail(e, "p2p allreduce launch");
  return RXLA_B200_OK;
}

int32_t comm_allreduce_f32(rxla_b200_comm* c, float* buf, int64_t count, cudaStream_t s) {
  return rxla_b200_allreduce(c, buf, count, RXLA_B200_F32, s);
}

int32_t comm_allgather_bytes(rxla_b200_comm* c, const void* in, void* out, int64_t bytes,
                             cudaStream_t s) {
  RXLA_REQUIRE(c && c->nccl && in && out && bytes >= 0, "allgather: bad arguments");
  if (bytes == 0) return RXLA_B200_OK;
  ncclResult_t r = comm::nccl().all_gather(in, out, (size_t)bytes, ncclUint8, c->nccl, s);
  if (r != ncclSuccess) return comm::nccl_fail(r, "ncclAllGather");
  return RXLA_B200_OK;
}

int32_t comm_world(const rxla_b200_comm* c) { return c ? c->world : 1; }

}  // namespace rxla

using namespace rxla;

static_assert(sizeof(ncclUniqueId) <= RXLA_B200_COMM_ID_BYTES, "nccl id size");

extern "C" int32_t rxla_b200_comm_unique_id(uint8_t id[RXLA_B200_COMM_ID_BYTES]) {
  RXLA_REQUIRE(id, "comm_unique_id: null id");
  auto& n = comm::nccl();
  if (!n.ok) return fail(RXLA_B200_UNAVAILABLE, "comm_unique_id: libnccl.so.2 not loadable");
  ncclUniqueId uid;
  ncclResult_t r = n.get_unique_id(&uid);
  if (r != ncclSuccess) return comm::nccl_fail(r, "ncclGetUniqueId");
  std::memset(id, 0, RXLA_B200_COMM_ID_BYTES);
  std::memcpy(id, &uid, sizeof(uid));
  return RXLA_B200_OK;
}

extern "C" int32_t rxla_b200_comm_init(const uint8_t id[RXLA_B200_COMM_ID_BYTES], int32_t rank,
                                       int32_t world_size, int32_t device,
                                       rxla_b200_comm** out) {
  RXLA_REQUIRE(id && out && world_size > 0 && rank >= 0 && rank < world_size,
               "comm_init: bad arguments");
  auto& n = comm::nccl();
  if (!n.ok) return fail(RXLA_B200_UNAVAILABLE, "comm_init: libnccl.so.2 not loadable");
  RXLA_CUDA_CHECK(cudaSetDevice(device));
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  auto* c = new rxla_b200_comm();
  c->rank = rank;
  c->world = world_size;
  c->device = device;
  ncclResult_t r = n.init_rank(&c->nccl, world_size, uid, rank);
  if (r != ncclSuccess) {
    delete c;
    return comm::nccl_fail(r, "ncclCommInitRank");
  }
  *out = c;
  return RXLA_B200_OK;
}

namespace rxla {
namespace p2p {
// What each rank contributes to the set-up exchange: its buffer's IPC handle
// (zeroed when its own set-up failed) and whether that set-up succeeded.
struct Offer {
  cudaIpcMemHandle_t handle;
  int32_t ok;
  int32_t pad[3];
};
// Exchange area of the set-up collectives: [kMaxRanks] offers, then one int32
// for the agreement.  A file-scope array, so the exchange itself allocates
// nothing and cannot fail where a rank's own allocations did.
static __device__ __align__(16) unsigned char g_xfer[kMaxRanks * sizeof(Offer) + 16];
}  // namespace p2p
}  // namespace rxla

// Every rank runs the same two collectives in the same order whatever its own
// result (the all-gather of offers, then a min-agreement), so a rank whose
// cudaMalloc or cudaIpcGetMemHandle failed never leaves its peers waiting in a
// collective it skipped.  A rank opens its peers' handles only when every
// offer says ok; the agreement then tells every rank whether all openings
// succeeded, and every rank keeps the buffers or releases them together.
extern "C" int32_t rxla_b200_comm_p2p_enable(rxla_b200_comm* c, int64_t max_count) {
  RXLA_REQUIRE(c && c->nccl, "comm_p2p_enable: comm not initialised");
  RXLA_REQUIRE(max_count > 0, "comm_p2p_enable: max_count must be positive");
  RXLA_REQUIRE(c->world <= p2p::kMaxRanks, "comm_p2p_enable: at most 8 ranks");
  if (c->p2p_local) {
    RXLA_REQUIRE(max_count <= c->p2p.cap, "comm_p2p_enable: already enabled with a smaller capacity");
    return RXLA_B200_OK;
  }
  RXLA_CUDA_CHECK(cudaSetDevice(c->device));
  void* xfer_v = nullptr;
  RXLA_CUDA_CHECK(cudaGetSymbolAddress(&xfer_v, p2p::g_xfer));
  uint8_t* xfer = static_cast<uint8_t*>(xfer_v);
  p2p::Offer* offers = reinterpret_cast<p2p::Offer*>(xfer);
  int32_t* agree = reinterpret_cast<int32_t*>(xfer + p2p::kMaxRanks * sizeof(p2p::Offer));
  p2p::Layout L;
  L.cap = (max_count + 3) / 4 * 4;
  // flags for the all-reduce kernel's CTAs and for the row-parallel GEMV
  // epilogue's (one CTA per SM)
  L.max_ctas = std::max((int)((L.cap + p2p::kChunk - 1) / p2p::kChunk), p2p::kFusedCtas);
  uint8_t* local = nullptr;
  uint64_t* epoch = nullptr;
  // 1. this rank's own set-up (no collective yet)
  cudaError_t e = cudaMalloc(&local, L.bytes());
  if (e == cudaSuccess) e = cudaMemset(local, 0, L.bytes());
  if (e == cudaSuccess) e = cudaMalloc(&epoch, (size_t)L.max_ctas * 8);
  if (e == cudaSuccess) e = cudaMemset(epoch, 0, (size_t)L.max_ctas * 8);
  p2p::Offer mine{};
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&mine.handle, local);
  if (e != cudaSuccess) {
    cudaGetLastError();
    std::memset(&mine, 0, sizeof(mine));
  }
  mine.ok = e == cudaSuccess ? 1 : 0;
  cudaError_t local_err = e;
  // 2. all-gather of the offers: always called
  bool ok = cudaMemcpy(offers + c->rank, &mine, sizeof(mine), cudaMemcpyHostToDevice) == cudaSuccess;
  int32_t st = RXLA_B200_OK;
  ncclResult_t r = comm::nccl().all_gather(offers + c->rank, offers, sizeof(mine), ncclUint8,
                                           c->nccl, nullptr);
  if (r != ncclSuccess) st = comm::nccl_fail(r, "comm_p2p_enable: handle exchange");
  std::vector<p2p::Offer> all(c->world);
  ok = ok && !st && cudaDeviceSynchronize() == cudaSuccess &&
       cudaMemcpy(all.data(), offers, c->world * sizeof(mine), cudaMemcpyDeviceToHost) == cudaSuccess;
  for (int q = 0; q < c->world && ok; ++q) ok = all[q].ok == 1;
  // 3. open the peers' buffers only if every rank offered one
  uint8_t* peer[p2p::kMaxRanks] = {};
  for (int q = 0; q < c->world && ok; ++q) {
    if (q == c->rank) {
      peer[q] = local;
      continue;
    }
    void* ptr = nullptr;
    ok = cudaIpcOpenMemHandle(&ptr, all[q].handle, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
    peer[q] = static_cast<uint8_t*>(ptr);
  }
  if (!ok) cudaGetLastError();
  // 4. min-agreement over the ranks: always called
  const int32_t opened = ok ? 1 : 0;
  int32_t all_ok = 0;
  const bool sent = cudaMemcpy(agree, &opened, 4, cudaMemcpyHostToDevice) == cudaSuccess;
  r = comm::nccl().all_reduce(agree, agree, 1, ncclInt32, ncclMin, c->nccl, nullptr);
  if (r != ncclSuccess && !st) st = comm::nccl_fail(r, "comm_p2p_enable: agreement");
  if (!(sent && r == ncclSuccess && cudaDeviceSynchronize() == cudaSuccess &&
        cudaMemcpy(&all_ok, agree, 4, cudaMemcpyDeviceToHost) == cudaSuccess))
    all_ok = 0;
  if (!all_ok || st) {
    for (int q = 0; q < c->world; ++q)
      if (q != c->rank && peer[q]) cudaIpcCloseMemHandle(peer[q]);
    if (local) cudaFree(local);
    if (epoch) cudaFree(epoch);
    cudaGetLastError();
    if (st) return st;
    if (local_err != cudaSuccess) return cuda_fail(local_err, "comm_p2p_enable: local set-up");
    return fail(RXLA_B200_UNAVAILABLE,
                "comm_p2p_enable: a rank could not set up or map the peer buffers; no rank uses them");
  }
  c->p2p = L;
  c->p2p_local = local;
  c->p2p_epoch = epoch;
  for (int q = 0; q < c->world; ++q) c->p2p_peer[q] = peer[q];
  return RXLA_B200_OK;
}

extern "C" int32_t rxla_b200_p2p_allreduce_f32(rxla_b200_comm* c, float* partial, float* residual,
                                               int64_t count, void* stream) {
  return comm_p2p_allreduce(c, partial, residual ? residual : partial, count, residual != nullptr,
                            static_cast<cudaStream_t>(stream));
}

extern "C" int32_t rxla_b200_comm_destroy(rxla_b200_comm* c) {
  if (!c) return RXLA_B200_OK;
  if (c->p2p_local) {
    cudaSetDevice(c->device);
    cudaDeviceSynchronize();
    for (int q = 0; q < c->world; ++q)
      if (q != c->rank && c->p2p_peer[q]) cudaIpcCloseMemHandle(c->p2p_peer[q]);
    // every rank has unmapped the peers' buffers before any rank frees its own
    // (collective, like the rest of the comm's life cycle)
    if (c->nccl &&
        comm::nccl().all_reduce(c->p2p_epoch, c->p2p_epoch, 1, ncclUint64, ncclSum, c->nccl,
                                nullptr) == ncclSuccess)
      cudaDeviceSynchronize();
    cudaFree(c->p2p_local);
    cudaFree(c->p2p_epoch);
  }
  if (c->nccl) comm::nccl().destroy(c->nccl);
  delete c;
  return RXLA_B200_OK;
}

extern "C" int32_t rxla_b200_allreduce(rxla_b200_comm* c, void* buf, int64_t count, int32_t dtype,
                                       void* stream) {
  RXLA_REQUIRE(c && c->nccl, "allreduce: comm not initialised");
  RXLA_REQUIRE(count >= 0, "allreduce: negative count");
  RXLA_REQUIRE(dtype == RXLA_B200_F32 || dtype == RXLA_B200_BF16, "allreduce: dtype F32 or BF16");
  if (count == 0) return RXLA_B200_OK;
  RXLA_REQUIRE(buf, "allreduce: null buffer");
  ncclResult_t r = comm::nccl().all_reduce(buf, buf, (size_t)count,
                                           dtype == RXLA_B200_F32 ? ncclFloat32 : ncclBfloat16,
                                           ncclSum, c->nccl, static_cast<cudaStream_t>(stream));
  if (r != ncclSuccess) return comm::nccl_fail(r, "ncclAllReduce");
  return RXLA_B200_OK;
}
