// race_capi.cu -- the extern "C" boundary of librace_b200.so plus the small
// fixed-order reduction / scan kernels that sit between the streaming passes.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "race_b200.h"
#include "race_launch.h"

#define RACE_TRY(x)                  \
  do {                               \
    const int rc_ = (x);             \
    if (rc_ != RACE_OK) return rc_;  \
  } while (0)

namespace race {
namespace {

thread_local char g_cuda_err[256] = "";
// Names of the kernels the most recent entry-point call launched
// (race_last_kernels).  Process-wide, because frameworks often run the
// backward on a thread of their own; the log is built per call on the
// calling thread and published when the outermost entry point returns.
std::mutex g_log_mu;
char g_kernels_last[512] = "";
char g_kernels_copy[512] = "";
thread_local char g_kernels[512] = "";
thread_local int g_api_depth = 0;
thread_local bool g_bound_valid = false;   // bind_device already ran in this call
thread_local cudaStream_t g_bound_stream = nullptr;

// Clears the calling thread's log when the outermost entry point of a call
// starts and publishes it when that entry point returns.
struct ApiScope {
  ApiScope() {
    if (g_api_depth++ == 0) {
      g_kernels[0] = '\0';
      g_cuda_err[0] = '\0';
      g_bound_valid = false;
    }
  }
  ~ApiScope() {
    if (--g_api_depth == 0) {
      std::lock_guard<std::mutex> lock(g_log_mu);
      std::memcpy(g_kernels_last, g_kernels, sizeof(g_kernels));
    }
  }
};

void log_kernel(const char* name, const char* note = nullptr) {
  const size_t n = std::strlen(g_kernels);
  if (n + 2 >= sizeof(g_kernels)) return;
  if (note != nullptr)
    std::snprintf(g_kernels + n, sizeof(g_kernels) - n, "%s%s(%s)", n ? "," : "", name, note);
  else
    std::snprintf(g_kernels + n, sizeof(g_kernels) - n, "%s%s", n ? "," : "", name);
}

int cuda_fail(cudaError_t e) {
  std::snprintf(g_cuda_err, sizeof(g_cuda_err), "%s: %s", cudaGetErrorName(e),
                cudaGetErrorString(e));
  return RACE_ERR_CUDA;
}

// The caller's stream decides the device.  This library carries its own
// (static) CUDA runtime, whose per-thread current device is not the caller
// runtime's, and threads that only ever ran the caller's runtime (a
// framework's autograd worker, for one) may have no current driver context
// at all -- which the tensor-map encoder needs.  So every entry point makes
// the stream's device current (cudaSetDevice also binds its primary context).
int bind_device(cudaStream_t stream) {
  if (g_bound_valid && g_bound_stream == stream) return RACE_OK;
  int dev = -1;
  cudaError_t e = cudaStreamGetDevice(stream, &dev);
  if (e != cudaSuccess) return cuda_fail(e);
  e = cudaSetDevice(dev);
  if (e != cudaSuccess) return cuda_fail(e);
  g_bound_valid = true;
  g_bound_stream = stream;
  return RACE_OK;
}

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    return 148;
  return n;
}

// ------------------------------------------------------------ small kernels
}  // namespace

// out[n][e] = sum_p part[n][p][e] for e < SS, summed in a fixed order.
__global__ void __launch_bounds__(1024) k_sum_partials(const float* __restrict__ part, int P, int SS,
                                                       float* __restrict__ out) {
  __shared__ float red[32][33];
  const int e = blockIdx.x * 32 + threadIdx.x;
  const int n = blockIdx.y;
  float acc = 0.f;
  if (e < SS)
    for (int p = threadIdx.y; p < P; p += 32) acc += part[((size_t)n * P + p) * SS + e];
  red[threadIdx.y][threadIdx.x] = acc;
  __syncthreads();
  if (threadIdx.y == 0 && e < SS) {
    float t = 0.f;
    for (int i = 0; i < 32; ++i) t += red[i][threadIdx.x];
    out[(size_t)n * SS + e] = t;
  }
}

namespace {

// Exclusive scan over the chunk axis of slots[n][chunk][0..width):
// forward (prefix over earlier chunks) or reverse (suffix over later chunks).
// Optionally writes the per-stream totals to total[n][0..width).  One block
// per (32 columns, stream); warp w owns a contiguous segment of chunks.
// Running sums are kept in float64.
__global__ void __launch_bounds__(1024) k_chunk_scan(float* __restrict__ slots, int64_t NC, int SS,
                                                     int width, int reverse,
                                                     float* __restrict__ total) {
  __shared__ double seg_sum[32][33];
  const int col = blockIdx.x * 32 + threadIdx.x;
  const int n = blockIdx.y;
  const int w = threadIdx.y;
  const int64_t seg = (NC + 31) / 32;
  const int64_t c0 = min(NC, (int64_t)w * seg), c1 = min(NC, c0 + seg);
  float* base = slots + (size_t)n * NC * SS + col;
  const bool live = col < width;
  double s = 0.0;
  if (live)
    for (int64_t ch = c0; ch < c1; ++ch) s += (double)base[(size_t)ch * SS];
  seg_sum[w][threadIdx.x] = s;
  __syncthreads();
  if (w == 0) {
    double run = 0.0;
    if (!reverse) {
      for (int i = 0; i < 32; ++i) {
        const double x = seg_sum[i][threadIdx.x];
        seg_sum[i][threadIdx.x] = run;
        run += x;
      }
    } else {
      for (int i = 31; i >= 0; --i) {
        const double x = seg_sum[i][threadIdx.x];
        seg_sum[i][threadIdx.x] = run;
        run += x;
      }
    }
    if (total != nullptr && live) total[(size_t)n * SS + col] = (float)run;
  }
  __syncthreads();
  if (!live) return;
  double run = seg_sum[w][threadIdx.x];
  constexpr int kB = 8;
  if (!reverse) {
    for (int64_t ch = c0; ch < c1; ch += kB) {
      float x[kB];
#pragma unroll
      for (int i = 0; i < kB; ++i) x[i] = ch + i < c1 ? base[(size_t)(ch + i) * SS] : 0.f;
#pragma unroll
      for (int i = 0; i < kB; ++i)
        if (ch + i < c1) {
          base[(size_t)(ch + i) * SS] = (float)run;
          run += (double)x[i];
        }
    }
  } else {
    for (int64_t ch = c1 - 1; ch >= c0; ch -= kB) {
      float x[kB];
#pragma unroll
      for (int i = 0; i < kB; ++i) x[i] = ch - i >= c0 ? base[(size_t)(ch - i) * SS] : 0.f;
#pragma unroll
      for (int i = 0; i < kB; ++i)
        if (ch - i >= c0) {
          base[(size_t)(ch - i) * SS] = (float)run;
          run += (double)x[i];
        }
    }
  }
}

// L2 normalisation of the head-dim rows of one [M, B, T, H, D] tensor (the
// hashing input of normalize_qk): xn = x / max(|x|, 1e-12), the semantics of
// torch.nn.functional.normalize.  One warp per row, dst contiguous [N][T][D].
template <typename T>
__device__ __forceinline__ float to_f(T x) {
  if constexpr (sizeof(T) == 4) return x; else return __bfloat162float(x);
}
template <typename T>
__device__ __forceinline__ T from_f(float x) {
  if constexpr (sizeof(T) == 4) return x; else return __float2bfloat16_rn(x);
}
constexpr float kNormFloor = 1e-12f;

template <typename T>
__global__ void __launch_bounds__(256) k_l2norm_rows(const T* __restrict__ x, Layout l, int B,
                                                     int H, int64_t Tn, int D, int64_t rows,
                                                     T* __restrict__ dst) {
  const int lane = threadIdx.x & 31;
  for (int64_t r = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; r < rows;
       r += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int n = (int)(r / Tn);
    const int64_t t = r % Tn;
    const T* src = x + stream_offset(l, n, B, H) + t * l.st;
    float v[2], ss = 0.f;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int c = lane + 32 * i;
      v[i] = c < D ? to_f(src[c]) : 0.f;
      ss = fmaf(v[i], v[i], ss);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = 1.f / fmaxf(sqrtf(ss), kNormFloor);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int c = lane + 32 * i;
      if (c < D) dst[r * D + c] = from_f<T>(v[i] * inv);
    }
  }
}

// Backward of k_l2norm_rows in place: g holds dL/dxn on entry and dL/dx on
// exit, dx = (g - xn (xn . g)) / |x| (g / floor where |x| < floor).
template <typename T>
__global__ void __launch_bounds__(256) k_l2norm_rows_bwd(const T* __restrict__ x, Layout l,
                                                         T* __restrict__ g, Layout lg, int B,
                                                         int H, int64_t Tn, int D, int64_t rows) {
  const int lane = threadIdx.x & 31;
  for (int64_t r = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; r < rows;
       r += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int n = (int)(r / Tn);
    const int64_t t = r % Tn;
    const T* src = x + stream_offset(l, n, B, H) + t * l.st;
    T* gr = g + stream_offset(lg, n, B, H) + t * lg.st;
    float v[2], gv[2], ss = 0.f, xg = 0.f;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int c = lane + 32 * i;
      v[i] = c < D ? to_f(src[c]) : 0.f;
      gv[i] = c < D ? to_f(gr[c]) : 0.f;
      ss = fmaf(v[i], v[i], ss);
      xg = fmaf(v[i], gv[i], xg);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      ss += __shfl_xor_sync(0xffffffffu, ss, o);
      xg += __shfl_xor_sync(0xffffffffu, xg, o);
    }
    const float nrm = sqrtf(ss);
    const bool clamp = nrm < kNormFloor;
    const float inv = 1.f / (clamp ? kNormFloor : nrm);
    const float c2 = clamp ? 0.f : xg * inv * inv;   // (xn . g) / |x|
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int c = lane + 32 * i;
      if (c < D) gr[c] = from_f<T>((gv[i] - v[i] * c2) * inv);
    }
  }
}

// slots[n][chunk][e] += offset[n][e] for e < width.
__global__ void k_add_offset(float* __restrict__ slots, const float* __restrict__ offset,
                             int64_t NC, int SS, int width, int64_t total) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = i % width;
    const int64_t rest = i / width;        // n * NC + chunk
    const int64_t n = rest / NC;
    slots[rest * SS + e] += offset[n * SS + e];
  }
}

// *dscale (=|+=) -(sum of partials) / scale^2, summed in a fixed order.
__global__ void __launch_bounds__(1024) k_dscale_final(const float* __restrict__ part, int count,
                                                       const float* __restrict__ scale,
                                                       float* __restrict__ dscale, int accumulate) {
  __shared__ float red[32];
  float acc = 0.f;
  for (int i = threadIdx.x; i < count; i += blockDim.x) acc += part[i];
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += red[i];
    const float s = *scale;
    const float v = -t / (s * s);
    *dscale = accumulate ? *dscale + v : v;
  }
}

// ------------------------------------------------------------ host helpers
struct Plan {
  int N, S, LK, SS, width, spad, P, CL;
  bool c5;             // causal per-bucket mode on the chunkwise tcgen05 kernels
  int64_t NC;
  size_t proj_off;     // c5: floats of the state before the q / k projections
  size_t alpha_off;    // c5: floats of the gradient state before alpha [N][T][SA]
  size_t mass_off;     // c5: floats of the gradient state before the tile key masses
  int SA;              // c5: floats per token of alpha
  size_t state_floats, gstate_floats, part_floats, dscale_floats;
  size_t norm_bytes;   // normalize_qk: one normalised [N][T][D] copy (q, then k)
  void* comm;          // race_set_comm's communicator (nullptr: single GPU)
  int rank, world;
  size_t comm_floats;  // world > 1: gathered totals [world][N][SS], total, offset
};

bool tensor_ok(const race_tensor_t& t, int elem_bytes) {
  if (t.data == nullptr) return false;
  if (reinterpret_cast<uintptr_t>(t.data) % 16 != 0) return false;
  // rows are moved by 16-byte vector loads and bulk copies: every row must
  // start on a 16-byte boundary (strides in multiples of 16 bytes)
  const int64_t q = 16 / elem_bytes;
  return t.stride_m % q == 0 && t.stride_b % q == 0 && t.stride_h % q == 0 && t.stride_t % q == 0;
}

constexpr int PJW = 16;   // projection columns kept per token (L K <= 16)

int make_plan(const race_desc_t* d, Plan* p) {
  if (d == nullptr || p == nullptr) return RACE_ERR_INVALID;
  if (d->dtype != RACE_F32 && d->dtype != RACE_BF16) return RACE_ERR_INVALID;
  if (d->num_bits < 1 || d->num_tables < 1 || d->ensembles < 1 || d->batch < 1 || d->heads < 1 ||
      d->tokens < 0 || d->head_dim < 1 || d->chunk < 0 || !(d->eps >= 0.f) ||
      (d->normalize != RACE_NORM_BUCKET && d->normalize != RACE_NORM_GLOBAL))
    return RACE_ERR_INVALID;
  if (d->flags & ~(RACE_FLAG_STRICT_TMA | RACE_FLAG_NORMALIZE_QK)) return RACE_ERR_INVALID;
  // the global denominator exists only for the causal form (misc/race_kernel.py)
  if (d->normalize == RACE_NORM_GLOBAL && !d->causal) return RACE_ERR_UNSUPPORTED;
  if (d->head_dim != 32 && d->head_dim != 64) return RACE_ERR_UNSUPPORTED;
  if (d->num_bits > 5) return RACE_ERR_UNSUPPORTED;
  const int S = d->num_tables << d->num_bits;
  const int LK = d->num_tables * d->num_bits;
  if (S > 64 || LK > kLKMax) return RACE_ERR_UNSUPPORTED;
  // above 32 buckets only the tcgen05 non-causal kernels are built
  if (S > 32 && d->causal) return RACE_ERR_UNSUPPORTED;
  const int64_t N64 = (int64_t)d->ensembles * d->batch * d->heads;
  if (N64 > 65535) return RACE_ERR_UNSUPPORTED;   // streams map to gridDim.y
  p->N = (int)N64;
  p->c5 = false;
  p->proj_off = p->alpha_off = p->mass_off = 0;
  p->SA = 0;
  p->S = S;
  p->LK = LK;
  p->spad = spad_for(S);
  const int D = d->head_dim;
  p->width = S * D + S;
  p->SS = round_up(S * D + S, 4);
  const int sms = sm_count();
  const int64_t T = d->tokens;
  // contiguous token ranges, one CTA each, every range at least a few 32-token
  // tiles long.  Non-causal kernels hold 2 (query backward) or 3 CTAs per SM:
  // 6 ranges per SM fill both evenly.  The causal walks hold one CTA per SM.
  const int64_t target = (int64_t)sms * (d->causal ? 2 : 6);
  int64_t P = (target + p->N - 1) / p->N;
  const int64_t by_len = (T + 127) / 128;
  if (P > by_len) P = by_len;
  if (P < 1) P = 1;
  p->P = (int)P;
  p->dscale_floats = (size_t)p->N * p->P;
  {
    const int rc = comm_rank_size(&p->comm, &p->rank, &p->world);
    if (rc != RACE_OK) return rc;
    p->comm_floats = p->world > 1 ? (size_t)(p->world + 2) * p->N * p->SS : 0;
  }
  const size_t es = d->dtype == RACE_F32 ? 4 : 2;
  p->norm_bytes = (d->flags & RACE_FLAG_NORMALIZE_QK)
                      ? ((size_t)p->N * (size_t)T * D * es + 255) / 256 * 256 : 0;
  if (!d->causal) {
    p->CL = 0;
    p->NC = 0;
    p->state_floats = (size_t)p->N * p->SS;
    p->gstate_floats = (size_t)p->N * p->SS;
    p->part_floats = (size_t)p->N * p->P * p->SS;
  } else {
    // state: the exclusive prefix slot of every range, then the fp32
    // projections of q and k ([N][T][16] each); gstate: the exclusive suffix
    // slot of every range, then alpha [N][T][SA] and the float64 key mass at
    // every 128-token tile start [N][tiles][SP]
    p->c5 = true;
    p->CL = 128;
    p->NC = p->P;
    const size_t slots = (size_t)p->N * p->P;
    p->proj_off = (slots * p->SS + 63) / 64 * 64;
    p->state_floats = p->proj_off + 2 * (size_t)p->N * T * PJW;
    p->SA = round_up(S, 4);
    p->alpha_off = (slots * p->SS + 63) / 64 * 64;
    p->mass_off = (p->alpha_off + (size_t)p->N * T * p->SA + 63) / 64 * 64;
    p->gstate_floats = p->mass_off + 2 * (size_t)p->N * ((T + 127) / 128) * round_up(p->spad, 16) + 2;
    p->part_floats = 0;
  }
  return RACE_OK;
}

size_t ws_bytes(const Plan& p) {
  return 2 * p.norm_bytes +
         (p.comm_floats + p.part_floats + (p.dscale_floats + 3) / 4 * 4 + 64) * sizeof(float);
}

// The device status word: the last 64 bytes of the workspace the caller
// passed (ws_bytes() keeps 256 bytes of slack behind the partial slots, so the
// word never overlaps them whatever the shape).
unsigned* status_word(void* ws, size_t bytes) {
  const uintptr_t end = reinterpret_cast<uintptr_t>(ws) + bytes;
  return reinterpret_cast<unsigned*>((end - 64) & ~uintptr_t(15));
}

struct Call {
  bool strict = false;
  bool normalize_qk = false;
  char* norm_q = nullptr;   // normalised copies in the workspace (normalize_qk)
  char* norm_k = nullptr;
  float* comm_ws = nullptr;  // world > 1: gathered totals, total, offset
  Plan plan;
  Params prm;
  float* part = nullptr;
  float* dscale_part = nullptr;
};

void fill_layout(Layout& l, const race_tensor_t& t) {
  l.sm = t.stride_m;
  l.sb = t.stride_b;
  l.sh = t.stride_h;
  l.st = t.stride_t;
}

int prepare(const race_desc_t* d, const float* planes, const float* scale, void* ws,
            size_t ws_bytes_given, Call* c) {
  int rc = make_plan(d, &c->plan);
  if (rc != RACE_OK) return rc;
  if (planes == nullptr || scale == nullptr) return RACE_ERR_INVALID;
  if (reinterpret_cast<uintptr_t>(planes) % 16 != 0) return RACE_ERR_ALIGN;
  const size_t need = ws_bytes(c->plan);
  if (ws == nullptr || ws_bytes_given < need) return RACE_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(ws) % 16 != 0) return RACE_ERR_ALIGN;
  c->normalize_qk = (d->flags & RACE_FLAG_NORMALIZE_QK) != 0;
  c->norm_q = static_cast<char*>(ws);
  c->norm_k = c->norm_q + c->plan.norm_bytes;
  c->comm_ws = reinterpret_cast<float*>(c->norm_k + c->plan.norm_bytes);
  c->part = c->comm_ws + c->plan.comm_floats;
  c->dscale_part = c->part + c->plan.part_floats;
  Params& p = c->prm;
  std::memset(&p, 0, sizeof(p));
  p.N = c->plan.N;
  p.M = d->ensembles;
  p.B = d->batch;
  p.H = d->heads;
  p.T = d->tokens;
  p.K = d->num_bits;
  p.L = d->num_tables;
  p.R = 1 << d->num_bits;
  p.S = c->plan.S;
  p.LK = c->plan.LK;
  p.Mp = d->shared_planes ? 1 : d->ensembles;
  p.eps = d->eps;
  p.global_norm = d->normalize == RACE_NORM_GLOBAL ? 1 : 0;
  p.planes = planes;
  p.scale = scale;
  p.part = c->part;
  p.dscale_part = c->dscale_part;
  p.err = status_word(ws, ws_bytes_given);
  p.wait_polls = d->wait_polls > 0 ? d->wait_polls : (1 << 22);
  c->strict = (d->flags & RACE_FLAG_STRICT_TMA) != 0;
  p.P = c->plan.P;
  p.CL = c->plan.CL;
  p.NC = c->plan.NC;
  p.SS = c->plan.SS;
  return RACE_OK;
}

int check_tensor(const race_desc_t* d, const race_tensor_t& t) {
  if (t.data == nullptr) return RACE_ERR_INVALID;
  return tensor_ok(t, d->dtype == RACE_F32 ? 4 : 2) ? RACE_OK : RACE_ERR_ALIGN;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link)
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn() {
  static const EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<EncodeTiledFn>(nullptr);
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

// Maps a [M, B, T, H, D] tensor as 5-D (D, T, H, B, M) with boxes of 128 rows
// x min(row, 128 B) (128-byte swizzle when the box row is 128 B), matching
// t5::Box.  Returns false when the layout cannot be mapped (a broadcast batch
// or head axis); the caller then uses the mma.sync kernels.
bool encode_map(CUtensorMap* m, const void* base, const Layout& l, int dtype, const Params& p,
                int D, const char* name, char* why, size_t why_len) {
  const EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) {
    std::snprintf(why, why_len, "cuTensorMapEncodeTiled not found");
    return false;
  }
  const int64_t es = dtype == RACE_F32 ? 4 : 2;
  const int64_t ext[5] = {D, p.T, p.H, p.B, l.sm == 0 ? 1 : p.M};
  const int64_t str[4] = {l.st, l.sh, l.sb, l.sm};
  cuuint64_t dims[5], strides[4];
  for (int i = 0; i < 5; ++i) dims[i] = (cuuint64_t)ext[i];
  static const char* const axis[4] = {"token", "head", "batch", "ensemble"};
  for (int i = 0; i < 4; ++i) {
    if (str[i] == 0 && ext[i + 1] > 1) {
      std::snprintf(why, why_len, "%s: broadcast %s axis", name, axis[i]);
      return false;
    }
    strides[i] = str[i] == 0 ? 16 : (cuuint64_t)(str[i] * es);
    if (str[i] < 0) {
      std::snprintf(why, why_len, "%s: negative %s stride", name, axis[i]);
      return false;
    }
  }
  if (p.T >= (int64_t(1) << 31)) {
    std::snprintf(why, why_len, "%s: more than 2^31 tokens", name);
    return false;
  }
  const int ib = (int)(D * es < 128 ? D * es : 128);
  const cuuint32_t box[5] = {(cuuint32_t)(ib / es), 128, 1, 1, 1};
  const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  const CUresult r = fn(m, es == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                        5, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        ib == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    std::snprintf(why, why_len,
                  "%s: encode error %d (strides %llu %llu %llu %llu B, dims %llu %llu %llu %llu %llu)",
                  name, (int)r, (unsigned long long)strides[0], (unsigned long long)strides[1],
                  (unsigned long long)strides[2], (unsigned long long)strides[3],
                  (unsigned long long)dims[0], (unsigned long long)dims[1],
                  (unsigned long long)dims[2], (unsigned long long)dims[3],
                  (unsigned long long)dims[4]);
    return false;
  }
  return true;
}

// Maps a float32 [N][T][C] array (C * 4 bytes a multiple of 16) as 3-D
// (C, T, N) with boxes of 128 whole rows.
bool encode_map3(CUtensorMap* m, const float* base, int64_t N, int64_t T, int C, const char* name,
                 char* why, size_t why_len) {
  const EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) {
    std::snprintf(why, why_len, "cuTensorMapEncodeTiled not found");
    return false;
  }
  const cuuint64_t dims[3] = {(cuuint64_t)C, (cuuint64_t)T, (cuuint64_t)N};
  const cuuint64_t strides[2] = {(cuuint64_t)C * 4, (cuuint64_t)(T * C * 4)};
  const cuuint32_t box[3] = {(cuuint32_t)C, 128, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    std::snprintf(why, why_len, "%s: encode error %d ([%lld][%lld][%d] float32)", name, (int)r,
                  (long long)N, (long long)T, C);
    return false;
  }
  return true;
}

const char* kernel_name(KernelId id) {
  switch (id) {
    case K_NC_REDUCE: return "t5_reduce";
    case K_NC_READOUT: return "t5_readout";
    case K_NC_BWD_Q: return "t5_bwd_q";
    case K_NC_BWD_KV: return "t5_bwd_kv";
    case K_NC_READOUT_SYNC: return "tc_readout";
    case K_NC_REDUCE_SYNC: return "tc_reduce";
    case K_NC_BWD_Q_SYNC: return "tc_bwd_q";
    case K_NC_BWD_KV_SYNC: return "tc_bwd_kv";
    case K_C5_PROJ: return "c5_proj";
    case K_C5_FWD: return "c5_fwd";
    case K_C5_BWD_Q: return "c5_bwd_q";
    case K_C5_BWD_KV: return "c5_bwd_kv";
    default: return "?";
  }
}

int launch(const race_desc_t* d, const Call& c, KernelId id, cudaStream_t stream,
           const char* note = nullptr) {
  RACE_TRY(bind_device(stream));
  KernelInfo ki;
  const int K = d->num_bits, sp = c.plan.spad;
  bool ok;
  if (d->dtype == RACE_F32)
    ok = d->head_dim == 32 ? kernels_f32_d32(sp, K, id, &ki) : kernels_f32_d64(sp, K, id, &ki);
  else
    ok = d->head_dim == 32 ? kernels_bf16_d32(sp, K, id, &ki) : kernels_bf16_d64(sp, K, id, &ki);
  if (!ok) return RACE_ERR_UNSUPPORTED;
  dim3 grid(c.plan.P, c.plan.N, 1);
  if (ki.persist > 0) {
    const int64_t items = (int64_t)c.plan.P * c.plan.N;
    const int64_t ctas = (int64_t)sm_count() * ki.persist;
    grid = dim3((unsigned)(items < ctas ? items : ctas), 1, 1);
  }
  Params prm = c.prm;
  TmaMaps maps;
  std::memset(&maps, 0, sizeof(maps));
  if (ki.tma > 0) {
    bool ok_map = false;
    const int hd = d->head_dim;
    char why[200] = "";
    const size_t wl = sizeof(why);
    if (id == K_NC_READOUT)
      ok_map = encode_map(&maps.map[0], prm.q, prm.lq, d->dtype, prm, hd, "q", why, wl) &&
               encode_map(&maps.map[1], prm.out, prm.lo, d->dtype, prm, hd, "out", why, wl);
    else if (id == K_NC_BWD_Q)
      ok_map = encode_map(&maps.map[0], prm.q, prm.lq, d->dtype, prm, hd, "q", why, wl) &&
               encode_map(&maps.map[1], prm.dout, prm.ldo, d->dtype, prm, hd, "dout", why, wl) &&
               encode_map(&maps.map[2], prm.dq, prm.ldq, d->dtype, prm, hd, "dq", why, wl);
    else if (id == K_NC_BWD_KV)
      ok_map = encode_map(&maps.map[0], prm.k, prm.lk, d->dtype, prm, hd, "k", why, wl) &&
               encode_map(&maps.map[1], prm.v, prm.lv, d->dtype, prm, hd, "v", why, wl) &&
               encode_map(&maps.map[2], prm.dk, prm.ldk, d->dtype, prm, hd, "dk", why, wl) &&
               encode_map(&maps.map[3], prm.dv, prm.ldv, d->dtype, prm, hd, "dv", why, wl);
    else if (id == K_NC_REDUCE)
      ok_map = encode_map(&maps.map[0], prm.k, prm.lk, d->dtype, prm, hd, "k", why, wl) &&
               encode_map(&maps.map[1], prm.v, prm.lv, d->dtype, prm, hd, "v", why, wl);
    else if (id == K_C5_PROJ)
      ok_map = encode_map(&maps.map[0], prm.q, prm.lq, d->dtype, prm, hd, "x", why, wl) &&
               encode_map3(&maps.map[1], prm.projq, prm.N, prm.T, PJW, "proj", why, wl);
    else if (id == K_C5_BWD_Q)
      ok_map = encode_map3(&maps.map[0], prm.projq, prm.N, prm.T, PJW, "projq", why, wl) &&
               encode_map3(&maps.map[1], prm.projk, prm.N, prm.T, PJW, "projk", why, wl) &&
               encode_map(&maps.map[2], prm.v, prm.lv, d->dtype, prm, hd, "v", why, wl) &&
               encode_map(&maps.map[3], prm.dout, prm.ldo, d->dtype, prm, hd, "dout", why, wl) &&
               encode_map(&maps.map[4], prm.dq, prm.ldq, d->dtype, prm, hd, "dq", why, wl) &&
               encode_map3(&maps.map[5], prm.alpha, prm.N, prm.T, prm.SA, "alpha", why, wl);
    else if (id == K_C5_BWD_KV)
      ok_map = encode_map3(&maps.map[0], prm.projq, prm.N, prm.T, PJW, "projq", why, wl) &&
               encode_map3(&maps.map[1], prm.projk, prm.N, prm.T, PJW, "projk", why, wl) &&
               encode_map(&maps.map[2], prm.v, prm.lv, d->dtype, prm, hd, "v", why, wl) &&
               encode_map(&maps.map[3], prm.dout, prm.ldo, d->dtype, prm, hd, "dout", why, wl) &&
               encode_map(&maps.map[5], prm.dk, prm.ldk, d->dtype, prm, hd, "dk", why, wl) &&
               encode_map(&maps.map[6], prm.dv, prm.ldv, d->dtype, prm, hd, "dv", why, wl);
    else if (id == K_C5_FWD)
      ok_map = encode_map3(&maps.map[0], prm.projq, prm.N, prm.T, PJW, "projq", why, wl) &&
               encode_map3(&maps.map[1], prm.projk, prm.N, prm.T, PJW, "projk", why, wl) &&
               encode_map(&maps.map[2], prm.v, prm.lv, d->dtype, prm, hd, "v", why, wl) &&
               encode_map(&maps.map[3], prm.out, prm.lo, d->dtype, prm, hd, "out", why, wl);
    if (!ok_map) {   // layouts the copy engine cannot walk: warp-level kernels
      char note[220];
      std::snprintf(note, sizeof(note), "fallback: %s", why);
      if (c.strict || c.plan.S > 32 || id >= K_C5_PROJ) {
        log_kernel(kernel_name(id), note);
        std::snprintf(g_cuda_err, sizeof(g_cuda_err), "%s: %s", kernel_name(id), why);
        return RACE_ERR_UNSUPPORTED;
      }
      const KernelId alt = id == K_NC_READOUT  ? K_NC_READOUT_SYNC
                           : id == K_NC_BWD_KV ? K_NC_BWD_KV_SYNC
                           : id == K_NC_BWD_Q  ? K_NC_BWD_Q_SYNC
                                               : K_NC_REDUCE_SYNC;
      return launch(d, c, alt, stream, note);
    }
  }
  void* args[] = {&prm, &maps};
  if (ki.smem_bytes > 48 * 1024) {
    const cudaError_t ea =
        cudaFuncSetAttribute(ki.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, ki.smem_bytes);
    if (ea != cudaSuccess) return cuda_fail(ea);
  }
  const cudaError_t e = cudaLaunchKernel(ki.fn, grid, dim3(ki.threads), args, ki.smem_bytes, stream);
  if (e != cudaSuccess) return cuda_fail(e);
  log_kernel(kernel_name(id), note);
  return RACE_OK;
}

// causal pre-pass: fp32 projections of x (q or k) into proj [N][T][16]
int launch_proj(const race_desc_t* d, Call& c, const race_tensor_t& x, float* proj,
                cudaStream_t stream) {
  c.prm.q = x.data;
  fill_layout(c.prm.lq, x);
  c.prm.projq = proj;
  return launch(d, c, K_C5_PROJ, stream);
}

int post(cudaStream_t) {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? RACE_OK : cuda_fail(e);
}

int sum_partials(const Call& c, float* out, cudaStream_t stream) {
  RACE_TRY(bind_device(stream));
  log_kernel("sum_partials");
  dim3 grid((c.plan.SS + 31) / 32, c.plan.N), block(32, 32);
  k_sum_partials<<<grid, block, 0, stream>>>(c.part, c.plan.P, c.plan.SS, out);
  return post(stream);
}

int chunk_scan(const Call& c, float* slots, int reverse, float* total, cudaStream_t stream) {
  RACE_TRY(bind_device(stream));
  log_kernel("chunk_scan");
  dim3 grid((c.plan.width + 31) / 32, c.plan.N), block(32, 32);
  k_chunk_scan<<<grid, block, 0, stream>>>(slots, c.plan.NC, c.plan.SS, c.plan.width, reverse,
                                           total);
  return post(stream);
}

int dscale_final(const Call& c, int count, float* dscale, int accumulate, cudaStream_t stream) {
  RACE_TRY(bind_device(stream));
  log_kernel("dscale_final");
  k_dscale_final<<<1, 1024, 0, stream>>>(c.dscale_part, count, c.prm.scale, dscale, accumulate);
  return post(stream);
}

// c5: the projections behind the prefix slots of the state; alpha and the
// tile key masses behind the gradient slots
void c5_pointers(Call& c, const float* state, const float* gstate, int64_t T) {
  float* st = const_cast<float*>(state);
  c.prm.projq = st + c.plan.proj_off;
  c.prm.projk = c.prm.projq + (size_t)c.plan.N * T * PJW;
  float* gs = const_cast<float*>(gstate);
  c.prm.alpha = gs + c.plan.alpha_off;
  c.prm.range_mass = reinterpret_cast<double*>(gs + c.plan.mass_off);
  c.prm.SA = c.plan.SA;
}

int zero_fill(void* p, size_t bytes, cudaStream_t stream) {
  if (bytes == 0 || p == nullptr) return RACE_OK;
  RACE_TRY(bind_device(stream));
  const cudaError_t e = cudaMemsetAsync(p, 0, bytes, stream);
  return e == cudaSuccess ? RACE_OK : cuda_fail(e);
}

int launch_rows(int64_t rows) {
  const int64_t blocks = (rows + 7) / 8;   // 8 rows (warps) per 256-thread block
  return (int)std::min<int64_t>(blocks, (int64_t)sm_count() * 16);
}

// normalize_qk: replaces `t` by its row-normalised copy in `dst` (contiguous
// [M, B, T, H, D] order of the streams, i.e. [N][T][D]).
int normalize_into(const race_desc_t* d, const Call& c, race_tensor_t* t, char* dst,
                   cudaStream_t stream) {
  const int64_t T = d->tokens, D = d->head_dim;
  const int64_t rows = (int64_t)c.plan.N * T;
  if (rows == 0) return RACE_OK;
  RACE_TRY(bind_device(stream));
  Layout l;
  fill_layout(l, *t);
  if (d->dtype == RACE_F32)
    k_l2norm_rows<float><<<launch_rows(rows), 256, 0, stream>>>(
        static_cast<const float*>(t->data), l, d->batch, d->heads, T, (int)D, rows,
        reinterpret_cast<float*>(dst));
  else
    k_l2norm_rows<__nv_bfloat16><<<launch_rows(rows), 256, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(t->data), l, d->batch, d->heads, T, (int)D, rows,
        reinterpret_cast<__nv_bfloat16*>(dst));
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e);
  log_kernel("l2norm");
  t->data = dst;
  t->stride_t = D;
  t->stride_h = T * D;
  t->stride_b = (int64_t)d->heads * T * D;
  t->stride_m = (int64_t)d->batch * d->heads * T * D;
  return RACE_OK;
}

// normalize_qk backward: g (the gradient of the normalised copy, written by
// the kernels into the caller's dq / dk) becomes the gradient of x, in place.
int normalize_backward(const race_desc_t* d, const Call& c, const race_tensor_t& x,
                       const race_tensor_t& g, cudaStream_t stream) {
  const int64_t T = d->tokens;
  const int64_t rows = (int64_t)c.plan.N * T;
  if (rows == 0) return RACE_OK;
  RACE_TRY(bind_device(stream));
  Layout lx, lg;
  fill_layout(lx, x);
  fill_layout(lg, g);
  if (d->dtype == RACE_F32)
    k_l2norm_rows_bwd<float><<<launch_rows(rows), 256, 0, stream>>>(
        static_cast<const float*>(x.data), lx, static_cast<float*>(g.data), lg, d->batch,
        d->heads, T, d->head_dim, rows);
  else
    k_l2norm_rows_bwd<__nv_bfloat16><<<launch_rows(rows), 256, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(x.data), lx, static_cast<__nv_bfloat16*>(g.data), lg,
        d->batch, d->heads, T, d->head_dim, rows);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e);
  log_kernel("l2norm_bwd");
  return RACE_OK;
}


}  // namespace
}  // namespace race

using namespace race;

namespace {
// Parameters of the probability export: the plan's shape checks and a Params
// carrying x in the q slot and dx in the dq slot.
int probs_params(const race_desc_t* d, race_tensor_t x, const float* planes, const float* scale,
                 Plan* plan, Params* p) {
  const int rc = make_plan(d, plan);
  if (rc != RACE_OK) return rc;
  if (planes == nullptr || scale == nullptr) return RACE_ERR_INVALID;
  if (reinterpret_cast<uintptr_t>(planes) % 16 != 0) return RACE_ERR_ALIGN;
  const int rt = check_tensor(d, x);
  if (rt != RACE_OK) return rt;
  std::memset(p, 0, sizeof(*p));
  p->N = plan->N;
  p->M = d->ensembles;
  p->B = d->batch;
  p->H = d->heads;
  p->T = d->tokens;
  p->K = d->num_bits;
  p->L = d->num_tables;
  p->R = 1 << d->num_bits;
  p->S = plan->S;
  p->LK = plan->LK;
  p->Mp = d->shared_planes ? 1 : d->ensembles;
  p->planes = planes;
  p->scale = scale;
  fill_layout(p->lq, x);
  p->q = x.data;
  return RACE_OK;
}
}  // namespace

extern "C" {

int race_probs(const race_desc_t* desc, race_tensor_t x, const float* planes, const float* scale,
               float* probs, cudaStream_t stream) {
  ApiScope scope_;
  Plan plan;
  Params p;
  RACE_TRY(probs_params(desc, x, planes, scale, &plan, &p));
  if (probs == nullptr) return RACE_ERR_INVALID;
  if (desc->tokens == 0) return RACE_OK;
  RACE_TRY(bind_device(stream));
  const cudaError_t e =
      launch_probs(false, desc->dtype == RACE_BF16, desc->head_dim, p, probs, nullptr, stream);
  return e == cudaSuccess ? RACE_OK : cuda_fail(e);
}

size_t race_probs_workspace(const race_desc_t* desc) {
  Plan plan;
  if (make_plan(desc, &plan) != RACE_OK) return 0;
  return (size_t)plan.N * (size_t)probs_blocks(desc->tokens) * sizeof(float) + 16;
}

int race_probs_backward(const race_desc_t* desc, race_tensor_t x, const float* planes,
                        const float* scale, const float* dprobs, race_tensor_t dx, float* dscale,
                        int accumulate, void* workspace, size_t workspace_bytes,
                        cudaStream_t stream) {
  ApiScope scope_;
  Plan plan;
  Params p;
  RACE_TRY(probs_params(desc, x, planes, scale, &plan, &p));
  if (dprobs == nullptr || dscale == nullptr) return RACE_ERR_INVALID;
  RACE_TRY(check_tensor(desc, dx));
  if (workspace == nullptr || workspace_bytes < race_probs_workspace(desc))
    return RACE_ERR_WORKSPACE;
  if (desc->tokens == 0) {
    if (!accumulate) RACE_TRY(zero_fill(dscale, sizeof(float), stream));
    return RACE_OK;
  }
  fill_layout(p.ldq, dx);
  p.dq = dx.data;
  RACE_TRY(bind_device(stream));
  float* part = static_cast<float*>(workspace);
  cudaError_t e = launch_probs(true, desc->dtype == RACE_BF16, desc->head_dim, p,
                               const_cast<float*>(dprobs), part, stream);
  if (e != cudaSuccess) return cuda_fail(e);
  const int count = (int)((int64_t)plan.N * probs_blocks(desc->tokens));
  k_dscale_final<<<1, 1024, 0, stream>>>(part, count, scale, dscale, accumulate);
  e = cudaGetLastError();
  return e == cudaSuccess ? RACE_OK : cuda_fail(e);
}

}  // extern "C"

extern "C" {

const char* race_version(void) { return "race_b200 1.0 (sm_100a)"; }

const char* race_strerror(int status) {
  switch (status) {
    case RACE_OK: return "ok";
    case RACE_ERR_INVALID: return "invalid argument";
    case RACE_ERR_UNSUPPORTED: return "unsupported shape or layout (d in {32,64}, L*2^K <= 64, L*K <= 16, K <= 6; see race_last_cuda_error)";
    case RACE_ERR_ALIGN: return "pointer or stride not 16-byte aligned for vector access";
    case RACE_ERR_WORKSPACE: return "workspace missing or smaller than race_query() reported";
    case RACE_ERR_CUDA: return "CUDA error (see race_last_cuda_error)";
    case RACE_ERR_TOO_LARGE:
      return "state + scratch exceed RACE_STATIC_SCRATCH_BYTES (use race_forward with caller buffers)";
    case RACE_ERR_DEVICE: return "a kernel gave up on a bounded device-side wait (outputs partial)";
    default: return "unknown status";
  }
}

const char* race_last_cuda_error(void) { return g_cuda_err; }

const char* race_last_kernels(void) {
  std::lock_guard<std::mutex> lock(g_log_mu);
  std::memcpy(g_kernels_copy, g_kernels_last, sizeof(g_kernels_last));
  return g_kernels_copy;
}

int race_status_clear(void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  if (workspace == nullptr || workspace_bytes < 64) return RACE_ERR_WORKSPACE;
  return zero_fill(status_word(workspace, workspace_bytes), sizeof(unsigned), stream);
}

int race_query(const race_desc_t* desc, race_sizes_t* sizes) {
  ApiScope scope_;
  if (sizes == nullptr) return RACE_ERR_INVALID;
  Plan p;
  RACE_TRY(make_plan(desc, &p));
  sizes->state_bytes = p.state_floats * sizeof(float);
  sizes->gstate_bytes = p.gstate_floats * sizeof(float);
  sizes->workspace_bytes = ws_bytes(p);
  sizes->total_bytes = (size_t)p.N * p.SS * sizeof(float);
  sizes->slot_floats = p.SS;
  sizes->chunk = p.CL;
  sizes->num_chunks = p.NC;
  return RACE_OK;
}

int race_forward_reduce(const race_desc_t* desc, race_tensor_t k, race_tensor_t v,
                        const float* planes, const float* scale, float* state, float* total,
                        void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  ApiScope scope_;
  Call c;
  RACE_TRY(prepare(desc, planes, scale, workspace, workspace_bytes, &c));
  if (state == nullptr) return RACE_ERR_INVALID;
  if (desc->tokens == 0) {
    RACE_TRY(zero_fill(state, c.plan.state_floats * sizeof(float), stream));
    if (total) RACE_TRY(zero_fill(total, (size_t)c.plan.N * c.plan.SS * sizeof(float), stream));
    return RACE_OK;
  }
  RACE_TRY(check_tensor(desc, k));
  RACE_TRY(check_tensor(desc, v));
  if (c.normalize_qk) RACE_TRY(normalize_into(desc, c, &k, c.norm_k, stream));
  fill_layout(c.prm.lk, k);
  fill_layout(c.prm.lv, v);
  c.prm.k = k.data;
  c.prm.v = v.data;
  if (!desc->causal) {
    RACE_TRY(launch(desc, c, K_NC_REDUCE, stream));
    RACE_TRY(sum_partials(c, state, stream));
    if (total) {
      const cudaError_t e = cudaMemcpyAsync(total, state, (size_t)c.plan.N * c.plan.SS * 4,
                                            cudaMemcpyDeviceToDevice, stream);
      if (e != cudaSuccess) return cuda_fail(e);
    }
  } else {
    // the key projections (kept for the readout and the backward), the range
    // totals straight into the state slots, then the exclusive scan
    float* projk = state + c.plan.proj_off + (size_t)c.plan.N * desc->tokens * PJW;
    RACE_TRY(launch_proj(desc, c, k, projk, stream));
    c.prm.part = state;
    RACE_TRY(launch(desc, c, K_NC_REDUCE, stream));
    RACE_TRY(chunk_scan(c, state, 0, total, stream));
  }
  return RACE_OK;
}

int race_forward_readout_ex(const race_desc_t* desc, race_tensor_t q, race_tensor_t k,
                            race_tensor_t v, const float* planes, const float* scale,
                            float* state, race_tensor_t out, float* den, void* workspace,
                            size_t workspace_bytes, cudaStream_t stream) {
  ApiScope scope_;
  Call c;
  RACE_TRY(prepare(desc, planes, scale, workspace, workspace_bytes, &c));
  if (state == nullptr) return RACE_ERR_INVALID;
  if (den != nullptr && !c.prm.global_norm) return RACE_ERR_INVALID;
  c.prm.den_out = den;
  if (desc->tokens == 0) return RACE_OK;
  RACE_TRY(check_tensor(desc, q));
  RACE_TRY(check_tensor(desc, out));
  if (c.normalize_qk) RACE_TRY(normalize_into(desc, c, &q, c.norm_q, stream));
  fill_layout(c.prm.lq, q);
  fill_layout(c.prm.lo, out);
  c.prm.q = q.data;
  c.prm.out = out.data;
  c.prm.state = state;
  if (!desc->causal) {
    RACE_TRY(launch(desc, c, K_NC_READOUT, stream));
  } else {
    RACE_TRY(check_tensor(desc, k));
    RACE_TRY(check_tensor(desc, v));
    if (c.normalize_qk) RACE_TRY(normalize_into(desc, c, &k, c.norm_k, stream));
    fill_layout(c.prm.lk, k);
    fill_layout(c.prm.lv, v);
    c.prm.k = k.data;
    c.prm.v = v.data;
    float* projq = state + c.plan.proj_off;
    RACE_TRY(launch_proj(desc, c, q, projq, stream));
    c.prm.projq = projq;
    c.prm.projk = projq + (size_t)c.plan.N * desc->tokens * PJW;
    RACE_TRY(launch(desc, c, K_C5_FWD, stream));
  }
  return RACE_OK;
}

int race_forward_readout(const race_desc_t* desc, race_tensor_t q, race_tensor_t k, race_tensor_t v,
                         const float* planes, const float* scale, float* state,
                         race_tensor_t out, void* workspace, size_t workspace_bytes,
                         cudaStream_t stream) {
  ApiScope scope_;
  return race_forward_readout_ex(desc, q, k, v, planes, scale, state, out, nullptr, workspace,
                                 workspace_bytes, stream);
}

int race_forward_ex(const race_desc_t* desc, race_tensor_t q, race_tensor_t k, race_tensor_t v,
                    const float* planes, const float* scale, race_tensor_t out, float* den,
                    float* state, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  ApiScope scope_;
  RACE_TRY(race_status_clear(workspace, workspace_bytes, stream));
  Call c;
  RACE_TRY(prepare(desc, planes, scale, workspace, workspace_bytes, &c));
  const Plan& pl = c.plan;
  if (pl.world > 1 && desc->tokens > 0) {
    // sequence-sharded over the communicator's ranks (this rank holds a
    // contiguous token range): bucket sums all-reduced, or the causal range
    // prefixes offset by the totals of the lower ranks
    const size_t cnt = (size_t)pl.N * pl.SS;
    float* gathered = c.comm_ws;
    float* tot = gathered + (size_t)pl.world * cnt;
    float* off = tot + cnt;
    RACE_TRY(race_forward_reduce(desc, k, v, planes, scale, state, desc->causal ? tot : nullptr,
                                 workspace, workspace_bytes, stream));
    if (!desc->causal) {
      RACE_TRY(comm_all_reduce(pl.comm, state, cnt, stream));
    } else {
      RACE_TRY(comm_gather_sum(pl.comm, tot, gathered, cnt, 0, pl.rank, off, stream));
      if (pl.rank > 0) RACE_TRY(race_add_offset(desc, state, off, 0, stream));
    }
    return race_forward_readout_ex(desc, q, k, v, planes, scale, state, out, den, workspace,
                                   workspace_bytes, stream);
  }
  RACE_TRY(race_forward_reduce(desc, k, v, planes, scale, state, nullptr, workspace,
                               workspace_bytes, stream));
  return race_forward_readout_ex(desc, q, k, v, planes, scale, state, out, den, workspace,
                                 workspace_bytes, stream);
}

int race_forward(const race_desc_t* desc, race_tensor_t q, race_tensor_t k, race_tensor_t v,
                 const float* planes, const float* scale, race_tensor_t out, float* state,
                 void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  ApiScope scope_;
  return race_forward_ex(desc, q, k, v, planes, scale, out, nullptr, state, workspace,
                         workspace_bytes, stream);
}

int race_backward_q_ex(const race_desc_t* desc, race_tensor_t q, race_tensor_t k, race_tensor_t v,
                       const float* planes, const float* scale, const float* state,
                       race_tensor_t dout, const float* dden, race_tensor_t dq, float* dscale,
                       float* gstate, float* total, void* workspace, size_t workspace_bytes,
                       cudaStream_t stream) {
  ApiScope scope_;
  Call c;
  RACE_TRY(prepare(desc, planes, scale, workspace, workspace_bytes, &c));
  if (state == nullptr || gstate == nullptr || dscale == nullptr) return RACE_ERR_INVALID;
  if (dden != nullptr && !c.prm.global_norm) return RACE_ERR_INVALID;
  c.prm.dden_in = dden;
  if (desc->tokens == 0) {
    RACE_TRY(zero_fill(gstate, c.plan.gstate_floats * sizeof(float), stream));
    if (total) RACE_TRY(zero_fill(total, (size_t)c.plan.N * c.plan.SS * sizeof(float), stream));
    return zero_fill(dscale, sizeof(float), stream);
  }
  RACE_TRY(check_tensor(desc, q));
  RACE_TRY(check_tensor(desc, dout));
  RACE_TRY(check_tensor(desc, dq));
  const race_tensor_t q_in = q;
  // (the chunkwise causal kernels read the saved projections, not q or k)
  if (c.normalize_qk && !c.plan.c5) RACE_TRY(normalize_into(desc, c, &q, c.norm_q, stream));
  fill_layout(c.prm.lq, q);
  fill_layout(c.prm.ldo, dout);
  fill_layout(c.prm.ldq, dq);
  c.prm.q = q.data;
  c.prm.dout = dout.data;
  c.prm.dq = dq.data;
  c.prm.state = state;
  if (!desc->causal) {
    RACE_TRY(launch(desc, c, K_NC_BWD_Q, stream));
    RACE_TRY(sum_partials(c, gstate, stream));
    if (total) {
      const cudaError_t e = cudaMemcpyAsync(total, gstate, (size_t)c.plan.N * c.plan.SS * 4,
                                            cudaMemcpyDeviceToDevice, stream);
      if (e != cudaSuccess) return cuda_fail(e);
    }
    RACE_TRY(dscale_final(c, c.plan.N * c.plan.P, dscale, 0, stream));
  } else {
    RACE_TRY(check_tensor(desc, v));
    fill_layout(c.prm.lv, v);
    c.prm.v = v.data;
    c.prm.gstate_out = gstate;
    c5_pointers(c, state, gstate, desc->tokens);
    RACE_TRY(launch(desc, c, K_C5_BWD_Q, stream));
    RACE_TRY(chunk_scan(c, gstate, 1, total, stream));
    RACE_TRY(dscale_final(c, c.plan.N * c.plan.P, dscale, 0, stream));
  }
  if (c.normalize_qk) RACE_TRY(normalize_backward(desc, c, q_in, dq, stream));
  return RACE_OK;
}

int race_backward_q(const race_desc_t* desc, race_tensor_t q, race_tensor_t k, race_tensor_t v,
                    const float* planes, const float* scale, const float* state,
                    race_tensor_t dout, race_tensor_t dq, float* dscale, float* gstate,
                    float* total, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  ApiScope scope_;
  return race_backward_q_ex(desc, q, k, v, planes, scale, state, dout, nullptr, dq, dscale, gstate,
                            total, workspace, workspace_bytes, stream);
}

int race_backward_kv(const race_desc_t* desc, race_tensor_t q, race_tensor_t k, race_tensor_t v,
                     const float* planes, const float* scale, const float* state,
                     const float* gstate, race_tensor_t dout, race_tensor_t dk, race_tensor_t dv,
                     float* dscale, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  ApiScope scope_;
  Call c;
  RACE_TRY(prepare(desc, planes, scale, workspace, workspace_bytes, &c));
  if (state == nullptr || gstate == nullptr || dscale == nullptr) return RACE_ERR_INVALID;
  if (desc->tokens == 0) return RACE_OK;
  RACE_TRY(check_tensor(desc, k));
  RACE_TRY(check_tensor(desc, v));
  RACE_TRY(check_tensor(desc, dk));
  RACE_TRY(check_tensor(desc, dv));
  const race_tensor_t k_in = k;
  if (c.normalize_qk && !c.plan.c5) RACE_TRY(normalize_into(desc, c, &k, c.norm_k, stream));
  fill_layout(c.prm.lk, k);
  fill_layout(c.prm.lv, v);
  fill_layout(c.prm.ldk, dk);
  fill_layout(c.prm.ldv, dv);
  c.prm.k = k.data;
  c.prm.v = v.data;
  c.prm.dk = dk.data;
  c.prm.dv = dv.data;
  c.prm.state = state;
  c.prm.gstate_in = gstate;
  if (!desc->causal) {
    RACE_TRY(launch(desc, c, K_NC_BWD_KV, stream));
    RACE_TRY(dscale_final(c, c.plan.N * c.plan.P, dscale, 1, stream));
  } else {
    RACE_TRY(check_tensor(desc, dout));
    fill_layout(c.prm.ldo, dout);
    c.prm.dout = dout.data;
    c5_pointers(c, state, gstate, desc->tokens);
    RACE_TRY(launch(desc, c, K_C5_BWD_KV, stream));
    RACE_TRY(dscale_final(c, c.plan.N * c.plan.P, dscale, 1, stream));
  }
  if (c.normalize_qk) RACE_TRY(normalize_backward(desc, c, k_in, dk, stream));
  return RACE_OK;
}

int race_backward(const race_desc_t* desc, race_tensor_t q, race_tensor_t k, race_tensor_t v,
                  const float* planes, const float* scale, const float* state, race_tensor_t dout,
                  race_tensor_t dq, race_tensor_t dk, race_tensor_t dv, float* dscale,
                  float* gstate, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  ApiScope scope_;
  return race_backward_ex(desc, q, k, v, planes, scale, state, dout, nullptr, dq, dk, dv, dscale,
                          gstate, workspace, workspace_bytes, stream);
}

int race_backward_ex(const race_desc_t* desc, race_tensor_t q, race_tensor_t k, race_tensor_t v,
                     const float* planes, const float* scale, const float* state,
                     race_tensor_t dout, const float* dden, race_tensor_t dq, race_tensor_t dk,
                     race_tensor_t dv, float* dscale, float* gstate, void* workspace,
                     size_t workspace_bytes, cudaStream_t stream) {
  ApiScope scope_;
  RACE_TRY(race_status_clear(workspace, workspace_bytes, stream));
  Call c;
  RACE_TRY(prepare(desc, planes, scale, workspace, workspace_bytes, &c));
  const Plan& pl = c.plan;
  if (pl.world > 1 && desc->tokens > 0) {
    // dE all-reduced, or the causal gradient suffixes offset by the totals of
    // the higher ranks; *dscale covers this rank's tokens
    const size_t cnt = (size_t)pl.N * pl.SS;
    float* gathered = c.comm_ws;
    float* tot = gathered + (size_t)pl.world * cnt;
    float* off = tot + cnt;
    RACE_TRY(race_backward_q_ex(desc, q, k, v, planes, scale, state, dout, dden, dq, dscale, gstate,
                                desc->causal ? tot : nullptr, workspace, workspace_bytes, stream));
    if (!desc->causal) {
      RACE_TRY(comm_all_reduce(pl.comm, gstate, cnt, stream));
    } else {
      RACE_TRY(comm_gather_sum(pl.comm, tot, gathered, cnt, pl.rank + 1, pl.world, off, stream));
      if (pl.rank + 1 < pl.world) RACE_TRY(race_add_offset(desc, gstate, off, 1, stream));
    }
    return race_backward_kv(desc, q, k, v, planes, scale, state, gstate, dout, dk, dv, dscale,
                            workspace, workspace_bytes, stream);
  }
  RACE_TRY(race_backward_q_ex(desc, q, k, v, planes, scale, state, dout, dden, dq, dscale, gstate,
                              nullptr, workspace, workspace_bytes, stream));
  return race_backward_kv(desc, q, k, v, planes, scale, state, gstate, dout, dk, dv, dscale,
                          workspace, workspace_bytes, stream);
}

int race_add_offset(const race_desc_t* desc, float* slots, const float* offset, int is_gradient,
                    cudaStream_t stream) {
  ApiScope scope_;
  Plan p;
  RACE_TRY(make_plan(desc, &p));
  (void)is_gradient;  // both slot kinds carry [S][d] sums then [S] masses up front
  if (!desc->causal || slots == nullptr || offset == nullptr) return RACE_ERR_INVALID;
  const int64_t total = (int64_t)p.N * p.NC * p.width;
  if (total == 0) return RACE_OK;
  RACE_TRY(bind_device(stream));
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, 4096);
  k_add_offset<<<blocks, 256, 0, stream>>>(slots, offset, p.NC, p.SS, p.width, total);
  return post(stream);
}

}  // extern "C"

// ------------------------------------------------------------ allocation-free forward
// Library-owned scratch for race_forward_static: the bucket state followed by
// the workspace.  In host code `g_static_scratch` is only a symbol handle; its
// device address is fetched per device with cudaGetSymbolAddress.
namespace race {
namespace {
constexpr size_t kStaticFloats = RACE_STATIC_SCRATCH_BYTES / sizeof(float);
static __device__ __align__(256) float g_static_scratch[kStaticFloats];

constexpr int kMaxDevices = 64;
std::mutex g_static_mu;
float* g_static_ptr[kMaxDevices] = {};

int static_scratch(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e);
  if (dev < 0 || dev >= kMaxDevices) return RACE_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (g_static_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return cuda_fail(e);
    g_static_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_static_ptr[dev];
  return RACE_OK;
}
}  // namespace
}  // namespace race

extern "C" int race_forward_static(const race_desc_t* desc, race_tensor_t q, race_tensor_t k,
                                   race_tensor_t v, const float* planes, const float* scale,
                                   race_tensor_t out, cudaStream_t stream) {
  ApiScope scope_;
  race_sizes_t sz;
  RACE_TRY(race_query(desc, &sz));
  const size_t state_bytes = (sz.state_bytes + 255) / 256 * 256;
  if (state_bytes + sz.workspace_bytes > RACE_STATIC_SCRATCH_BYTES) return RACE_ERR_TOO_LARGE;
  RACE_TRY(bind_device(stream));   // the array's address is per device
  float* base = nullptr;
  RACE_TRY(static_scratch(&base));
  float* state = base;
  void* ws = reinterpret_cast<char*>(base) + state_bytes;
  return race_forward(desc, q, k, v, planes, scale, out, state, ws,
                      RACE_STATIC_SCRATCH_BYTES - state_bytes, stream);
}

extern "C" int race_device_status(const void* workspace, size_t workspace_bytes,
                                  uint32_t* status, cudaStream_t stream) {
  if (status == nullptr) return RACE_ERR_INVALID;
  RACE_TRY(bind_device(stream));
  if (workspace == nullptr) {   // the allocation-free forward's array
    float* base = nullptr;
    RACE_TRY(static_scratch(&base));
    workspace = base;
    workspace_bytes = RACE_STATIC_SCRATCH_BYTES;
  }
  if (workspace_bytes < 64) return RACE_ERR_WORKSPACE;
  const cudaError_t e =
      cudaMemcpyAsync(status, status_word(const_cast<void*>(workspace), workspace_bytes),
                      sizeof(uint32_t), cudaMemcpyDefault, stream);
  return e == cudaSuccess ? RACE_OK : cuda_fail(e);
}
