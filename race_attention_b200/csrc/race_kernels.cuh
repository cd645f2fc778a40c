// race_kernels.cuh -- shared definitions of the RACE attention kernels:
// launch parameters, row I/O helpers and small reductions.  The kernels
// themselves live in race_t5.cuh (non-causal, tcgen05 + TMA), race_mma.cuh
// (mma.sync generation: the fallback of the non-causal kernels for layouts the
// copy engine cannot map) and race_causal5.cuh (causal, tcgen05 + TMA);
// race_tiles.cuh has the shared-memory tile staging the mma.sync kernels use.
//
// Soft hash.  softmax over the 2^K corners of sum_k c_rk u_k factorises:
//   p_r = prod_k sigmoid(2 c_rk u_k),  u_k = tanh(x . P_k) / scale,
// which is the reference's tanh -> /scale -> @protos_T -> softmax
// (misc/vit.py:955-958) evaluated without the R-way exp/sum.  Both
// sigmoid(+2|u|) and sigmoid(-2|u|) are formed from one exp(-2|u|), so the
// small probabilities keep full relative precision.
//
// Reductions across CTAs write per-CTA partials that a separate kernel sums
// in a fixed order, so every result is bitwise reproducible run to run.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace race {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kLKMax = 16;     // L*K planes per stream supported

struct Layout {
  int64_t sm, sb, sh, st;
};

struct Params {
  int N, M, B, H;
  int64_t T;
  int K, L, R, S, LK;
  int Mp;
  float eps;
  const void* q;    Layout lq;
  const void* k;    Layout lk;
  const void* v;    Layout lv;
  const void* dout; Layout ldo;
  void* out;        Layout lo;
  void* dq;         Layout ldq;
  void* dk;         Layout ldk;
  void* dv;         Layout ldv;
  const float* planes;   // [Mp][LK][D]
  const float* scale;    // device scalar
  const float* state;    // saved slots
  const float* gstate_in;
  float* state_out;
  float* gstate_out;
  float* part;           // [N][P][SS] partial slots
  float* dscale_part;    // per-CTA partials
  float* alpha;          // causal [N][T][S]
  int P;                 // CTAs per stream (non-causal)
  int CL;                // causal chunk length
  int64_t NC;            // causal chunks per stream
  int SS;                // floats per slot
  unsigned* err;         // device status word (last 64 bytes of the workspace), 0 = ok
  int wait_polls;        // polls of each bounded wait in the kernels' main loops
  int global_norm;       // causal: 1 = one denominator per token summed over all buckets
  float* den_out;        // causal global: [N][T] denominators (optional)
  const float* dden_in;  // causal global: [N][T] incoming gradient of den (optional)
  float* projq;          // causal: fp32 projections of q onto the planes [N][T][16]
  float* projk;          // causal: fp32 projections of k [N][T][16]
  int SA;                // causal: floats per token of alpha ([N][T][SA], S rounded up to 4)
  double* range_mass;    // causal: key mass at the start of every tile [N][tiles][SP] (float64)
};

__host__ __device__ constexpr int round_up(int a, int b) { return (a + b - 1) / b * b; }

// TMA descriptors of a kernel's streamed inputs and outputs (encoded per call
// on the host; a __grid_constant__ kernel parameter).  Each maps a
// [M, B, T, H, D] tensor as 5-D (D, T, H, B, M) with 128-row boxes, or a
// [N][T][C] float32 array as 3-D (C, T, N); which map holds which tensor is
// fixed per kernel.
struct TmaMaps {
  CUtensorMap map[8];
};

// ---------------------------------------------------------------- row I/O
template <typename T, int C>
__device__ __forceinline__ void ld_row(const T* __restrict__ p, float (&x)[C]) {
  if constexpr (sizeof(T) == 4) {
    if constexpr (C == 4) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(p));
      x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
    } else {
      const float2 v = __ldg(reinterpret_cast<const float2*>(p));
      x[0] = v.x; x[1] = v.y;
    }
  } else {
    if constexpr (C == 4) {
      const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
      const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&u.x);
      const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&u.y);
      const float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
      x[0] = fa.x; x[1] = fa.y; x[2] = fb.x; x[3] = fb.y;
    } else {
      const unsigned u = __ldg(reinterpret_cast<const unsigned*>(p));
      const float2 fa = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u));
      x[0] = fa.x; x[1] = fa.y;
    }
  }
}

template <typename T, int C>
__device__ __forceinline__ void st_row(T* __restrict__ p, const float (&x)[C]) {
  if constexpr (sizeof(T) == 4) {
    if constexpr (C == 4) {
      *reinterpret_cast<float4*>(p) = make_float4(x[0], x[1], x[2], x[3]);
    } else {
      *reinterpret_cast<float2*>(p) = make_float2(x[0], x[1]);
    }
  } else {
    if constexpr (C == 4) {
      const __nv_bfloat162 a = __floats2bfloat162_rn(x[0], x[1]);
      const __nv_bfloat162 b = __floats2bfloat162_rn(x[2], x[3]);
      uint2 u;
      u.x = *reinterpret_cast<const unsigned*>(&a);
      u.y = *reinterpret_cast<const unsigned*>(&b);
      *reinterpret_cast<uint2*>(p) = u;
    } else {
      const __nv_bfloat162 a = __floats2bfloat162_rn(x[0], x[1]);
      *reinterpret_cast<__nv_bfloat162*>(p) = a;
    }
  }
}

template <int C>
__device__ __forceinline__ void ld_f(const float* p, float (&x)[C]) {
  if constexpr (C == 4) {
    const float4 v = *reinterpret_cast<const float4*>(p);
    x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
  } else {
    const float2 v = *reinterpret_cast<const float2*>(p);
    x[0] = v.x; x[1] = v.y;
  }
}

template <int C>
__device__ __forceinline__ void st_f(float* p, const float (&x)[C]) {
  if constexpr (C == 4) {
    *reinterpret_cast<float4*>(p) = make_float4(x[0], x[1], x[2], x[3]);
  } else {
    *reinterpret_cast<float2*>(p) = make_float2(x[0], x[1]);
  }
}

__device__ __forceinline__ int64_t stream_offset(const Layout& l, int n, int B, int H) {
  const int h = n % H;
  const int b = (n / H) % B;
  const int m = n / (H * B);
  return (int64_t)m * l.sm + (int64_t)b * l.sb + (int64_t)h * l.sh;
}

struct Shape {
  int K, L, R, S, LK;
  __device__ __forceinline__ explicit Shape(const Params& p)
      : K(p.K), L(p.L), R(p.R), S(p.S), LK(p.LK) {}
};

// Sums a per-lane value over the CTA in a fixed order; thread 0 gets the total.
__device__ __forceinline__ float cta_sum(float x, float* red32) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  const int w = threadIdx.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red32[w] = x;
  __syncthreads();
  float t = 0.f;
  if (threadIdx.x == 0)
    for (int i = 0; i < kWarps; ++i) t += red32[i];
  return t;
}

// Sums P partial slots per stream in a fixed order: out[n] = sum_p part[n][p].
__global__ void __launch_bounds__(1024) k_sum_partials(const float* __restrict__ part, int P, int SS,
                                                       float* __restrict__ out);

}  // namespace race
