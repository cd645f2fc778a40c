// race_comm.cu -- the library's own multi-GPU hook: with an NCCL communicator
// set (race_set_comm), race_forward / race_backward run a sequence-sharded
// call themselves, the bucket-state exchange on the caller's stream between
// the split phases.  NCCL is opened at run time (dlopen of libnccl.so.2), so
// the library has no link-time dependency on it and single-GPU callers never
// load it.
#include <dlfcn.h>

#include <cstdio>
#include <cstring>
#include <mutex>

#include "race_b200.h"
#include "race_launch.h"

namespace race {
namespace comm {

// The few NCCL types and constants used here (NCCL's public API, nccl.h).
using ncclResult_t = int;
using ncclComm_t = void*;
struct ncclUniqueId {
  char internal[128];
};
constexpr int ncclSum = 0;
constexpr int ncclFloat32 = 7;

struct Api {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_count)(ncclComm_t, int*) = nullptr;
  ncclResult_t (*comm_user_rank)(ncclComm_t, int*) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, int, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, int, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  bool ok = false;
};

std::mutex g_mu;
Api g_api;
bool g_tried = false;
ncclComm_t g_comm = nullptr;
thread_local char g_err[256] = "";

const Api* api() {
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_tried) {
    g_tried = true;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (h == nullptr) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (h != nullptr) {
      Api a;
      a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
      a.comm_init_rank = reinterpret_cast<decltype(a.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
      a.comm_destroy = reinterpret_cast<decltype(a.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
      a.comm_count = reinterpret_cast<decltype(a.comm_count)>(dlsym(h, "ncclCommCount"));
      a.comm_user_rank = reinterpret_cast<decltype(a.comm_user_rank)>(dlsym(h, "ncclCommUserRank"));
      a.all_reduce = reinterpret_cast<decltype(a.all_reduce)>(dlsym(h, "ncclAllReduce"));
      a.all_gather = reinterpret_cast<decltype(a.all_gather)>(dlsym(h, "ncclAllGather"));
      a.error_string = reinterpret_cast<decltype(a.error_string)>(dlsym(h, "ncclGetErrorString"));
      a.ok = a.get_unique_id && a.comm_init_rank && a.comm_destroy && a.comm_count &&
             a.comm_user_rank && a.all_reduce && a.all_gather && a.error_string;
      g_api = a;
    }
  }
  return g_api.ok ? &g_api : nullptr;
}

int nccl_fail(const Api* a, ncclResult_t r, const char* what) {
  std::snprintf(g_err, sizeof(g_err), "%s: %s", what, a ? a->error_string(r) : "NCCL not found");
  return RACE_ERR_CUDA;
}

// offset[e] = sum of gathered[r][e] over ranks r in [r0, r1), in rank order
__global__ void k_sum_ranks(const float* __restrict__ gathered, int64_t count, int r0, int r1,
                            float* __restrict__ offset) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count;
       i += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int r = r0; r < r1; ++r) s += gathered[(size_t)r * count + i];
    offset[i] = s;
  }
}

}  // namespace comm
}  // namespace race

using namespace race::comm;

extern "C" {

const char* race_comm_error(void) { return g_err; }

int race_comm_unique_id(void* id) {
  if (id == nullptr) return RACE_ERR_INVALID;
  const Api* a = api();
  if (a == nullptr) return nccl_fail(a, 0, "dlopen libnccl.so.2");
  ncclUniqueId u;
  const ncclResult_t r = a->get_unique_id(&u);
  if (r != 0) return nccl_fail(a, r, "ncclGetUniqueId");
  std::memcpy(id, u.internal, sizeof(u.internal));
  return RACE_OK;
}

int race_comm_init(void** comm, int nranks, const void* id, int rank) {
  if (comm == nullptr || id == nullptr || nranks < 1 || rank < 0 || rank >= nranks)
    return RACE_ERR_INVALID;
  const Api* a = api();
  if (a == nullptr) return nccl_fail(a, 0, "dlopen libnccl.so.2");
  ncclUniqueId u;
  std::memcpy(u.internal, id, sizeof(u.internal));
  ncclComm_t c = nullptr;
  const ncclResult_t r = a->comm_init_rank(&c, nranks, u, rank);
  if (r != 0) return nccl_fail(a, r, "ncclCommInitRank");
  *comm = c;
  return RACE_OK;
}

int race_comm_destroy(void* comm) {
  if (comm == nullptr) return RACE_ERR_INVALID;
  const Api* a = api();
  if (a == nullptr) return nccl_fail(a, 0, "dlopen libnccl.so.2");
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_comm == comm) g_comm = nullptr;
  }
  const ncclResult_t r = a->comm_destroy(comm);
  return r == 0 ? RACE_OK : nccl_fail(a, r, "ncclCommDestroy");
}

int race_set_comm(void* comm) {
  if (comm != nullptr && api() == nullptr) return nccl_fail(nullptr, 0, "dlopen libnccl.so.2");
  std::lock_guard<std::mutex> lock(g_mu);
  g_comm = comm;
  return RACE_OK;
}

}  // extern "C"

namespace race {

// Rank and world size of the communicator set by race_set_comm (world 1 and
// rank 0 without one).
int comm_rank_size(void** comm, int* rank, int* world) {
  {
    std::lock_guard<std::mutex> lock(g_mu);
    *comm = g_comm;
  }
  *rank = 0;
  *world = 1;
  if (*comm == nullptr) return RACE_OK;
  const Api* a = api();
  ncclResult_t r = a->comm_count(*comm, world);
  if (r != 0) return nccl_fail(a, r, "ncclCommCount");
  r = a->comm_user_rank(*comm, rank);
  return r == 0 ? RACE_OK : nccl_fail(a, r, "ncclCommUserRank");
}

// Non-causal: sum of `count` floats over the ranks, in place.
int comm_all_reduce(void* comm, float* buf, size_t count, cudaStream_t stream) {
  const Api* a = api();
  const ncclResult_t r = a->all_reduce(buf, buf, count, ncclFloat32, ncclSum, comm, stream);
  return r == 0 ? RACE_OK : nccl_fail(a, r, "ncclAllReduce");
}

// Causal: offset = sum over ranks [r0, r1) of every rank's `total`
// (count floats), through an all-gather into `gathered` [world][count].
int comm_gather_sum(void* comm, const float* total, float* gathered, size_t count, int r0, int r1,
                    float* offset, cudaStream_t stream) {
  const Api* a = api();
  const ncclResult_t r = a->all_gather(total, gathered, count, ncclFloat32, comm, stream);
  if (r != 0) return nccl_fail(a, r, "ncclAllGather");
  const int blocks = (int)std::min<int64_t>(((int64_t)count + 255) / 256, 1024);
  k_sum_ranks<<<blocks, 256, 0, stream>>>(gathered, (int64_t)count, r0, r1, offset);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? RACE_OK : RACE_ERR_CUDA;
}

}  // namespace race
