/*
 * race_b200.h -- C ABI of the B200 (sm_100a) RACE attention library.
 *
 * RACE attention soft-hashes queries and keys onto L tables of K seeded random
 * hyperplanes (R = 2^K buckets per table, S = L*R buckets in all), aggregates
 * the values into per-bucket [V | 1] states and reads them back out per query.
 * Both the non-causal form and the causal per-bucket prefix-mean form are
 * provided, forward and backward (the backward recomputes the bucket
 * probabilities instead of storing them).
 *
 * Conventions
 *   - All pointers are device pointers unless stated otherwise.  Nothing in
 *     this library allocates device memory: the caller passes every buffer,
 *     sized by race_query().
 *   - Work is stream-ordered on the cudaStream_t the caller passes.  Entry
 *     points return a race_status_t; they never throw or abort.
 *   - Streams of the computation (one per ensemble m, batch b, head h) are
 *     numbered n = (m * B + b) * H + h.  q/k/v/out and every gradient are
 *     addressed through race_tensor_t strides, so [B,T,H,d] activations (the
 *     layout of a Linear output viewed per head) are consumed in place and the
 *     ensemble dimension may have stride 0 (an expanded view).
 *   - Planes are float32 [Mp][L*K][d] (Mp = 1 when shared by all ensembles,
 *     else M), i.e. the transpose of the reference's planes_T buffer.
 *   - `scale` is a device pointer to the float32 temperature divisor (the
 *     reference's exp(logit_temp).clamp(...) or sqrt(d)), so a learnable
 *     temperature never forces a host synchronisation.
 *
 * State buffers
 *   A "slot" is the [S][d] bucket sum B followed by the [S] bucket mass A,
 *   padded to a multiple of 4 floats (race_sizes_t.slot_floats).
 *   non-causal: state  = N slots (totals over this rank's tokens, then over
 *                all ranks after the caller's all-reduce);
 *               gstate = N slots of dE = sum_t pQ(t) dO(t).
 *   causal:     state  = N * num_chunks slots holding the EXCLUSIVE prefix at
 *                the start of every chunk (a range of whole 128-token tiles),
 *                then the fp32 projections of q and k onto the planes;
 *                gstate = N * num_chunks gradient slots (exclusive suffix
 *                sums), then per-token alpha and per-tile key masses.
 *
 * Single GPU: race_forward() then race_backward().  Sequence-sharded multi-GPU
 * (each rank holds a contiguous token range of every stream): the split entry
 * points below, with the caller's collective in between (see each comment).
 */
#ifndef RACE_B200_H
#define RACE_B200_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RACE_ABI_VERSION 3

typedef enum {
  RACE_OK = 0,
  RACE_ERR_INVALID = 1,      /* bad descriptor field or null pointer            */
  RACE_ERR_UNSUPPORTED = 2,  /* shape outside what the kernels are built for    */
  RACE_ERR_ALIGN = 3,        /* pointer or stride breaks the vector alignment   */
  RACE_ERR_WORKSPACE = 4,    /* workspace smaller than race_query() asked for   */
  RACE_ERR_CUDA = 5,         /* a CUDA launch failed (see race_last_cuda_error) */
  RACE_ERR_TOO_LARGE = 6,    /* shape needs more than the static scratch holds  */
  RACE_ERR_DEVICE = 7        /* a kernel gave up on a bounded device-side wait  */
} race_status_t;

/* race_desc_t.flags bits. */
#define RACE_FLAG_STRICT_TMA 1u   /* never fall back to the mma.sync kernels: a layout
                                     the copy engine cannot map (a broadcast batch or
                                     head axis) returns RACE_ERR_UNSUPPORTED instead */
#define RACE_FLAG_NORMALIZE_QK 2u /* hash L2-normalised q and k (q/|q|, k/|k|); the
                                     values and the output are unchanged.  Off by
                                     default: the reference never normalises on the
                                     RACE path, and tanh is not scale-invariant */

/* Bits of the device status word (race_device_status). */
#define RACE_DEV_TIMEOUT 1u  /* a bounded wait ran out; outputs of that call are partial */
#define RACE_DEV_STUCK 2u    /* after a timeout, copies or MMAs in flight did not drain */

typedef enum { RACE_F32 = 0, RACE_BF16 = 1 } race_dtype_t;

/* Causal normalisation.  BUCKET: every bucket's prefix mean is normalised by
 * its own mass, out(t) = sum_s pQ_s(t) B_s(t) / (A_s(t) + eps) (misc/race.py).
 * GLOBAL: one denominator per token summed over all buckets and tables,
 * out(t) = sum_s pQ_s(t) B_s(t) / max(sum_s pQ_s(t) A_s(t), eps), the chunked
 * ELSAA form (misc/race_kernel.py:9-124 + misc/elsaa_causal_complete.py:551-560;
 * eps is its clamp_min floor: 1e-6 for the Triton path, which sums over tables,
 * L * 1e-6 for the torch fallback, which averages num and den over tables).
 * GLOBAL is causal only. */
typedef enum { RACE_NORM_BUCKET = 0, RACE_NORM_GLOBAL = 1 } race_norm_t;

/* One activation tensor: element strides of the (m, b, h, t) axes; the head
 * dimension is contiguous. */
typedef struct {
  void* data;
  int64_t stride_m, stride_b, stride_h, stride_t;
} race_tensor_t;

typedef struct {
  int32_t dtype;          /* race_dtype_t of q, k, v, out and all gradients     */
  int32_t causal;         /* 0: non-causal (misc/vit.py), 1: prefix mean         */
  int32_t head_dim;       /* d: 32 or 64                                         */
  int32_t num_bits;       /* K hyperplanes per table (R = 2^K)                   */
  int32_t num_tables;     /* L tables; S = L * 2^K <= 64, L*K <= 16              */
  int32_t ensembles;      /* M                                                   */
  int32_t batch;          /* B                                                   */
  int32_t heads;          /* H                                                   */
  int64_t tokens;         /* T held by this rank                                 */
  int32_t chunk;          /* accepted and ignored (the causal kernels use
                             128-token tiles and choose the ranges)           */
  int32_t shared_planes;  /* 1: planes [1][L*K][d]; 0: planes [M][L*K][d]        */
  float eps;              /* added to the bucket mass (reference: 1e-6); GLOBAL:
                             the floor of the per-token denominator             */
  int32_t normalize;      /* race_norm_t (0 = BUCKET)                            */
  uint32_t flags;         /* RACE_FLAG_* bits (0 = default behaviour)            */
  int32_t wait_polls;     /* polls of each bounded device wait before a kernel
                             gives up (0 = the library default, 2^22).  A small
                             value exists to test the timeout path.             */
} race_desc_t;

typedef struct {
  size_t state_bytes;      /* forward -> backward saved state                   */
  size_t gstate_bytes;     /* backward_q -> backward_kv gradient state          */
  size_t workspace_bytes;  /* scratch, contents not preserved between calls     */
  size_t total_bytes;      /* one [N] slot array (causal rank totals/offsets)   */
  int32_t slot_floats;     /* floats per state slot                             */
  int32_t chunk;           /* causal tile length (128)                          */
  int64_t num_chunks;      /* causal chunks per stream                          */
} race_sizes_t;

const char* race_version(void);
const char* race_strerror(int status);
/* Text of the last CUDA error seen by this library on the calling thread. */
const char* race_last_cuda_error(void);

/* Comma-separated names of the kernels launched by the most recent
 * entry-point call in this process (e.g. "t5_reduce,sum_partials,t5_readout";
 * process-wide because frameworks often run the backward on a thread of
 * their own; with concurrent callers it is one of the latest calls).  A
 * launch that fell back from the tcgen05 + TMA kernels to the mma.sync ones is
 * listed with the reason, e.g. "tc_bwd_q(fallback: dout: broadcast axis)". */
const char* race_last_kernels(void);

/* Device status word.  Every tcgen05 kernel bounds its waits on the copy
 * engine and the tensor core; a wait that runs out ends the kernel early (its
 * outputs are then partial) and ORs RACE_DEV_* bits into a status word kept
 * in the last 64 bytes of the workspace the caller passed.  race_forward,
 * race_backward and race_forward_static clear the word when they start;
 * callers of the split phases clear it with race_status_clear at the start of
 * their step.  race_device_status copies the word (one uint32) to `status`
 * (device or pinned host memory) in stream order, without synchronising. */
int race_status_clear(void* workspace, size_t workspace_bytes, cudaStream_t stream);
int race_device_status(const void* workspace, size_t workspace_bytes, uint32_t* status,
                       cudaStream_t stream);

/* Validates the descriptor and reports the buffer sizes for it. */
int race_query(const race_desc_t* desc, race_sizes_t* sizes);

/* Full forward on one GPU.  Replaces the reference's BatchedACE.forward
 * (misc/vit.py:918-978 non-causal; misc/race.py:63-142 causal) and the
 * unbound host function race_fused_fwd (kernels/gpu/forward_kernel.cu:64-96).
 * Writes out and the saved state. */
int race_forward(const race_desc_t* desc, race_tensor_t q, race_tensor_t k,
                 race_tensor_t v, const float* planes, const float* scale,
                 race_tensor_t out, float* state, void* workspace,
                 size_t workspace_bytes, cudaStream_t stream);

/* Full backward on one GPU.  Replaces autograd through BatchedACE.forward and
 * the reference's race_bwd_kq_noscan / race_bwd_v_noscan
 * (kernels/gpu/backward_kernels.cu:145-255) and race_prefix_mean_flat_bw
 * (kernels/cpu/race_pref.cpp:104-220).  Writes dq, dk, dv and the gradient of
 * the temperature divisor into *dscale (device float). */
int race_backward(const race_desc_t* desc, race_tensor_t q, race_tensor_t k,
                  race_tensor_t v, const float* planes, const float* scale,
                  const float* state, race_tensor_t dout, race_tensor_t dq,
                  race_tensor_t dk, race_tensor_t dv, float* dscale,
                  float* gstate, void* workspace, size_t workspace_bytes,
                  cudaStream_t stream);

/* ---- split phases for sequence-sharded runs ------------------------------
 * forward:  race_forward_reduce -> [caller collective] -> race_forward_readout
 *   non-causal: state holds this rank's bucket sums; the caller all-reduces
 *               the whole state buffer (sum) before the readout.
 *   causal (per-bucket): forward_reduce also stores the key projections and
 *               forward_readout the query projections in the state (the
 *               backward reads them instead of q and k), so the readout
 *               writes to `state` as well; only the leading slots are
 *               exchanged between ranks.
 *   causal:     state holds rank-local chunk prefixes and `total` (N slots)
 *               the rank's totals; the caller gathers all ranks' totals, sums
 *               those of LOWER ranks into an offset (N slots) and calls
 *               race_add_offset(state, offset) before the readout.
 * backward: race_backward_q -> [caller collective] -> race_backward_kv
 *   non-causal: gstate holds this rank's dE; the caller all-reduces it.
 *   causal:     gstate holds rank-local chunk suffixes and `total` the rank's
 *               gradient totals; the caller sums those of HIGHER ranks into
 *               an offset and calls race_add_offset(gstate, offset).
 *   race_backward_q overwrites *dscale with the query-side part;
 *   race_backward_kv adds the key-side part.  Each rank's *dscale covers its
 *   own tokens (sum it across ranks like any parameter gradient). */
int race_forward_reduce(const race_desc_t* desc, race_tensor_t k,
                        race_tensor_t v, const float* planes,
                        const float* scale, float* state, float* total,
                        void* workspace, size_t workspace_bytes,
                        cudaStream_t stream);
int race_forward_readout(const race_desc_t* desc, race_tensor_t q,
                         race_tensor_t k, race_tensor_t v, const float* planes,
                         const float* scale, float* state,
                         race_tensor_t out, void* workspace,
                         size_t workspace_bytes, cudaStream_t stream);
int race_backward_q(const race_desc_t* desc, race_tensor_t q, race_tensor_t k,
                    race_tensor_t v, const float* planes, const float* scale,
                    const float* state, race_tensor_t dout, race_tensor_t dq,
                    float* dscale, float* gstate, float* total,
                    void* workspace, size_t workspace_bytes,
                    cudaStream_t stream);
int race_backward_kv(const race_desc_t* desc, race_tensor_t q,
                     race_tensor_t k, race_tensor_t v, const float* planes,
                     const float* scale, const float* state,
                     const float* gstate, race_tensor_t dout, race_tensor_t dk,
                     race_tensor_t dv, float* dscale, void* workspace,
                     size_t workspace_bytes, cudaStream_t stream);
/* The same calls with the global-normalisation denominator exposed
 * (desc->normalize == RACE_NORM_GLOBAL only; otherwise a non-NULL den / dden
 * is RACE_ERR_INVALID).  den: optional float32 [N][T] output, the unclamped
 * per-token denominator sum_s pQ_s(t) A_s(t) (the reference's den_sumL,
 * misc/elsaa_causal_complete.py:553-561, from which it derives d_token).
 * dden: optional float32 [N][T] incoming gradient of that den, added to the
 * gradient the output contributes.  Both follow the (m, b, h) stream order. */
int race_forward_ex(const race_desc_t* desc, race_tensor_t q, race_tensor_t k,
                    race_tensor_t v, const float* planes, const float* scale,
                    race_tensor_t out, float* den, float* state, void* workspace,
                    size_t workspace_bytes, cudaStream_t stream);
int race_forward_readout_ex(const race_desc_t* desc, race_tensor_t q,
                            race_tensor_t k, race_tensor_t v,
                            const float* planes, const float* scale,
                            float* state, race_tensor_t out, float* den,
                            void* workspace, size_t workspace_bytes,
                            cudaStream_t stream);
int race_backward_ex(const race_desc_t* desc, race_tensor_t q, race_tensor_t k,
                     race_tensor_t v, const float* planes, const float* scale,
                     const float* state, race_tensor_t dout, const float* dden,
                     race_tensor_t dq, race_tensor_t dk, race_tensor_t dv,
                     float* dscale, float* gstate, void* workspace,
                     size_t workspace_bytes, cudaStream_t stream);
int race_backward_q_ex(const race_desc_t* desc, race_tensor_t q, race_tensor_t k,
                       race_tensor_t v, const float* planes, const float* scale,
                       const float* state, race_tensor_t dout, const float* dden,
                       race_tensor_t dq, float* dscale, float* gstate, float* total,
                       void* workspace, size_t workspace_bytes,
                       cudaStream_t stream);

/* ---- multi-GPU hook -------------------------------------------------------
 * With a communicator set, race_forward / race_forward_ex and race_backward /
 * race_backward_ex run a sequence-sharded call: every rank passes its own
 * contiguous token range of every stream (ranks in token order) and the
 * library runs the exchange between the split phases on `stream` -- an NCCL
 * all-reduce of the bucket sums and of dE (non-causal), or an all-gather of
 * the range totals whose lower- (forward) or higher- (backward) rank sum is
 * added to the local prefixes (causal).  The temperature gradient stays
 * rank-local.  Replaces the reference's missing multi-GPU path (it runs one
 * sequence per GPU); NCCL is opened at run time (libnccl.so.2).  Set the
 * communicator before race_query: the workspace then includes the exchange
 * buffers.  The setting is process-wide; NULL returns to single-GPU calls. */
int race_comm_unique_id(void* id128);   /* NCCL unique id, 128 bytes, on one rank */
int race_comm_init(void** comm, int nranks, const void* id128, int rank);
int race_comm_destroy(void* comm);
int race_set_comm(void* comm);
const char* race_comm_error(void);      /* text of the last NCCL failure on this thread */

/* Causal only: adds offset (N slots) to every chunk slot of `slots`
 * (state or gstate).  Gradient slots also carry the per-chunk key mass,
 * which the offset does not touch. */
int race_add_offset(const race_desc_t* desc, float* slots, const float* offset,
                    int is_gradient, cudaStream_t stream);

/* Bucket probabilities of one tensor, for hybrid models that gate on them.
 * Replaces the torch sequence of race_bucket_probs_from_qk
 * (misc/arxiv_64K.py:1580-1642: x @ planes_T, tanh, / scale, @ protos_T,
 * softmax per table), which the reference runs for q and k separately.
 * x: [M, B, T, H, d] through its strides (desc->causal is ignored).
 * probs: float32 [N][T][S], N = M*B*H streams in (m, b, h) order and bucket
 * s = l*2^K + r with r in itertools.product([-1, 1]) order -- the
 * reference's [M, B, H, T, L, R] tensor. */
int race_probs(const race_desc_t* desc, race_tensor_t x, const float* planes,
               const float* scale, float* probs, cudaStream_t stream);
/* Workspace bytes race_probs_backward needs (temperature partial sums). */
size_t race_probs_workspace(const race_desc_t* desc);
/* Gradient of race_probs: dx from dprobs (float32 [N][T][S]); *dscale is
 * set (accumulate = 0) or incremented (accumulate = 1) by dL/dscale. */
int race_probs_backward(const race_desc_t* desc, race_tensor_t x, const float* planes,
                        const float* scale, const float* dprobs, race_tensor_t dx,
                        float* dscale, int accumulate, void* workspace,
                        size_t workspace_bytes, cudaStream_t stream);

/* Forward without any device allocation: for callers that cannot call
 * cudaMalloc or own a caching allocator -- e.g. code running inside another
 * runtime's memory pool, a plugin host that forbids allocation after start-up,
 * or an inference loop with a fixed memory budget.  No counterpart exists in
 * the reference.  The caller passes only inputs and `out`; the bucket state and
 * all scratch live in one library-owned static device array of
 * RACE_STATIC_SCRATCH_BYTES (8 MiB), which every GPU that loads the library
 * keeps until process exit.  Shapes whose state + scratch exceed it return
 * RACE_ERR_TOO_LARGE (see race_query: state_bytes + workspace_bytes).
 * The first call on a device looks up that array's device address (once per
 * device, on the current device), so make the first call before any stream
 * capture.  All calls share the array: two calls that overlap on the GPU
 * (different streams, or different host threads) race and corrupt each other;
 * serialize them.  Every value a call reads from the array is written earlier
 * in the same call; the only value cleared at the start of a call is the
 * device status word at the array's end (read it with race_device_status on
 * the array: pass workspace = NULL, workspace_bytes = 0).  No saved state is
 * returned, so there is no matching backward: use race_forward for training. */
#define RACE_STATIC_SCRATCH_BYTES (8u << 20)
int race_forward_static(const race_desc_t* desc, race_tensor_t q, race_tensor_t k,
                        race_tensor_t v, const float* planes, const float* scale,
                        race_tensor_t out, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* RACE_B200_H */
