// race_launch.h -- internal table of kernel instantiations (host side).
#pragma once
#include "race_kernels.cuh"

namespace race {

enum KernelId {
  K_NC_REDUCE = 0,
  K_NC_READOUT,
  K_NC_BWD_Q,
  K_NC_BWD_KV,
  K_NC_READOUT_SYNC,   // warp-level mma.sync generation (comparison)
  K_NC_REDUCE_SYNC,    // warp-level range totals (fallback of the tcgen05 reduce)
  K_NC_BWD_Q_SYNC,
  K_NC_BWD_KV_SYNC,
  K_C5_PROJ,           // causal: fp32 projections of q or k (pre-pass)
  K_C5_FWD,            // causal: chunkwise tcgen05 forward readout
  K_C5_BWD_Q,          // causal: chunkwise tcgen05 query backward
  K_C5_BWD_KV,         // causal: chunkwise tcgen05 key/value backward (reverse walk)
  K_COUNT
};

struct KernelInfo {
  const void* fn;   // __global__ symbol, launched with one `Params` argument
  int groups;       // token groups per CTA
  int smem_bytes;   // dynamic shared memory
  int threads;      // threads per CTA
  int persist;      // >0: persistent grid of persist CTAs per SM over (stream, range) items
  int tma;          // >0: the kernel takes a TmaMaps of its streamed inputs as a second argument
};

// Padded bucket counts the kernels are instantiated for.
constexpr int kSpadList[] = {8, 16, 20, 24, 32, 64};

inline int spad_for(int S) {
  for (int s : kSpadList)
    if (S <= s) return s;
  return -1;
}

// One table per (element type, head dim); K selects the non-causal tile
// kernels' compile-time hyperplane count (the causal kernels take it at run time).
bool kernels_f32_d32(int spad, int K, KernelId id, KernelInfo* info);
bool kernels_f32_d64(int spad, int K, KernelId id, KernelInfo* info);
bool kernels_bf16_d32(int spad, int K, KernelId id, KernelInfo* info);
bool kernels_bf16_d64(int spad, int K, KernelId id, KernelInfo* info);

// Bucket-probability export (race_probs.cu): forward writes [N][T][S] fp32
// probabilities of the tensor in prm.q; backward reads dprobs and writes
// prm.dq plus one temperature partial per block.
cudaError_t launch_probs(bool bwd, bool bf16, int D, const Params& prm, float* out_or_dp,
                         float* part, cudaStream_t s);
int64_t probs_blocks(int64_t T);

// race_comm.cu: the communicator set by race_set_comm (none: world 1, rank 0)
// and the two exchanges of a sequence-sharded call, on the caller's stream.
int comm_rank_size(void** comm, int* rank, int* world);
int comm_all_reduce(void* comm, float* buf, size_t count, cudaStream_t stream);
int comm_gather_sum(void* comm, const float* total, float* gathered, size_t count, int r0, int r1,
                    float* offset, cudaStream_t stream);

}  // namespace race
