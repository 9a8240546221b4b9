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

#include "internal.cuh"

struct rxla_b200_comm {
  ncclComm_t nccl = nullptr;
  int rank = 0, world = 1, device = 0;
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

extern "C" int32_t rxla_b200_comm_destroy(rxla_b200_comm* c) {
  if (!c) return RXLA_B200_OK;
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
