// race_probs.cu -- soft-hash bucket probabilities as a product of their own,
// and their backward.
//
// The reference's hybrid models read RACE's bucket probabilities directly
// (race_bucket_probs_from_qk, misc/arxiv_64K.py:1580-1642: projection onto the
// planes, tanh, / scale, corner logits, softmax per table).  Here one thread
// owns one token: it projects its row onto the L*K planes (CUDA-core fp32
// FMAs, planes in shared memory), forms the L softmaxes over the 2^K corners
// as products of sigmoids (softmax over {+-1}^K . u factorises per plane) and
// writes the S = L*2^K probabilities of the token, [N][T][S] fp32, bucket
// s = l*R + r with r in itertools.product([-1, 1]) order.  The backward
// recomputes the probabilities and returns dx and the temperature's partial
// sums (fixed-order per block, summed by the C ABI's final kernel).
#include "race_kernels.cuh"
#include "race_launch.h"
#include "race_tiles.cuh"

namespace race {
namespace probs {

constexpr int NT = 128;     // threads (tokens) per block
constexpr int LKM = 16;     // L*K <= 16
constexpr int KM = 5;       // K <= 5

template <typename T, int D>
__device__ __forceinline__ void load_row(const T* p, float (&x)[D]) {
  if constexpr (sizeof(T) == 4) {
#pragma unroll
    for (int i = 0; i < D / 4; ++i) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(p) + i);
      x[4 * i] = v.x; x[4 * i + 1] = v.y; x[4 * i + 2] = v.z; x[4 * i + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(p) + i);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(h[j]);
        x[8 * i + 2 * j] = f.x;
        x[8 * i + 2 * j + 1] = f.y;
      }
    }
  }
}

// proj[j] = x . planes[j] for j < LK (planes [LK][D] in shared memory)
template <int D>
__device__ __forceinline__ void project(const float (&x)[D], const float* pl, int LK,
                                        float (&proj)[LKM]) {
#pragma unroll
  for (int j = 0; j < LKM; ++j) {
    float a = 0.f;
    if (j < LK) {
      const float4* p4 = reinterpret_cast<const float4*>(pl + j * D);
#pragma unroll
      for (int i = 0; i < D / 4; ++i) {
        const float4 w = p4[i];
        a = fmaf(x[4 * i], w.x, a);
        a = fmaf(x[4 * i + 1], w.y, a);
        a = fmaf(x[4 * i + 2], w.z, a);
        a = fmaf(x[4 * i + 3], w.w, a);
      }
    }
    proj[j] = a;
  }
}

// sigmoid(2u) and sigmoid(-2u) of u = tanh(proj) / scale, per plane
__device__ __forceinline__ void plane_sigmoids(float pr, float inv_scale, float& h, float& sp,
                                               float& sn) {
  h = tiles::tanh_exp(pr);
  const float u = h * inv_scale;
  const float ex = __expf(-2.f * fabsf(u));
  const float rc = __frcp_rn(1.f + ex);
  sp = u >= 0.f ? rc : ex * rc;
  sn = u >= 0.f ? ex * rc : rc;
}

template <typename T, int D>
__global__ void __launch_bounds__(NT) k_probs_fwd(const Params prm, float* __restrict__ out) {
  __shared__ __align__(16) float pl[LKM * D];
  const int n = blockIdx.y;
  const int m = prm.Mp == 1 ? 0 : n / (prm.B * prm.H);
  const float* src = prm.planes + (size_t)m * prm.LK * D;
  for (int i = threadIdx.x; i < prm.LK * D; i += NT) pl[i] = src[i];
  __syncthreads();
  const int64_t t = (int64_t)blockIdx.x * NT + threadIdx.x;
  if (t >= prm.T) return;
  const T* xb = static_cast<const T*>(prm.q) + stream_offset(prm.lq, n, prm.B, prm.H);
  float x[D];
  load_row<T, D>(xb + t * prm.lq.st, x);
  float proj[LKM];
  project<D>(x, pl, prm.LK, proj);
  const float inv_scale = 1.f / __ldg(prm.scale);
  const int K = prm.K, R = prm.R;
  float* o = out + ((size_t)n * prm.T + t) * prm.S;
  for (int l = 0; l < prm.L; ++l) {
    float sp[KM], sn[KM];
#pragma unroll
    for (int k = 0; k < KM; ++k) {
      float h;
      const float pr = k < K ? proj[l * K + k] : 0.f;
      plane_sigmoids(pr, inv_scale, h, sp[k], sn[k]);
    }
    for (int r = 0; r < R; ++r) {
      float v = 1.f;
#pragma unroll
      for (int k = 0; k < KM; ++k)
        if (k < K) v *= ((r >> (K - 1 - k)) & 1) ? sp[k] : sn[k];
      o[l * R + r] = v;
    }
  }
}

// dx = J^T dprobs; per-block partial of sum_j du_j h_j (the temperature's share)
template <typename T, int D>
__global__ void __launch_bounds__(NT) k_probs_bwd(const Params prm, const float* __restrict__ dp,
                                                  float* __restrict__ dscale_part) {
  __shared__ __align__(16) float pl[LKM * D];
  __shared__ float red[NT / 32];
  const int n = blockIdx.y;
  const int m = prm.Mp == 1 ? 0 : n / (prm.B * prm.H);
  const float* src = prm.planes + (size_t)m * prm.LK * D;
  for (int i = threadIdx.x; i < prm.LK * D; i += NT) pl[i] = src[i];
  __syncthreads();
  const int64_t t = (int64_t)blockIdx.x * NT + threadIdx.x;
  float ds = 0.f;
  if (t < prm.T) {
    const T* xb = static_cast<const T*>(prm.q) + stream_offset(prm.lq, n, prm.B, prm.H);
    T* dxb = static_cast<T*>(prm.dq) + stream_offset(prm.ldq, n, prm.B, prm.H);
    float x[D];
    load_row<T, D>(xb + t * prm.lq.st, x);
    float proj[LKM];
    project<D>(x, pl, prm.LK, proj);
    const float inv_scale = 1.f / __ldg(prm.scale);
    const int K = prm.K, R = prm.R;
    const float* g = dp + ((size_t)n * prm.T + t) * prm.S;
    float dj[LKM];
#pragma unroll
    for (int j = 0; j < LKM; ++j) dj[j] = 0.f;
    for (int l = 0; l < prm.L; ++l) {
      float sp[KM], sn[KM], h[KM];
#pragma unroll
      for (int k = 0; k < KM; ++k) {
        const float pr = k < K ? proj[l * K + k] : 0.f;
        plane_sigmoids(pr, inv_scale, h[k], sp[k], sn[k]);
      }
      // pbar = sum_r p_r g_r, then du_k = sum_r (+-1) p_r (g_r - pbar)
      float pbar = 0.f;
      for (int r = 0; r < R; ++r) {
        float v = 1.f;
#pragma unroll
        for (int k = 0; k < KM; ++k)
          if (k < K) v *= ((r >> (K - 1 - k)) & 1) ? sp[k] : sn[k];
        pbar = fmaf(v, g[l * R + r], pbar);
      }
      float du[KM];
#pragma unroll
      for (int k = 0; k < KM; ++k) du[k] = 0.f;
      for (int r = 0; r < R; ++r) {
        float v = 1.f;
#pragma unroll
        for (int k = 0; k < KM; ++k)
          if (k < K) v *= ((r >> (K - 1 - k)) & 1) ? sp[k] : sn[k];
        const float q = v * (g[l * R + r] - pbar);
#pragma unroll
        for (int k = 0; k < KM; ++k)
          if (k < K) du[k] += ((r >> (K - 1 - k)) & 1) ? q : -q;
      }
#pragma unroll
      for (int k = 0; k < KM; ++k) {
        if (k < K) {
          ds = fmaf(du[k], h[k], ds);
          const float dv = du[k] * inv_scale * (1.f - h[k] * h[k]);
#pragma unroll
          for (int j = 0; j < LKM; ++j)
            if (j == l * K + k) dj[j] = dv;
        }
      }
    }
    float dx[D];
#pragma unroll
    for (int d = 0; d < D; ++d) dx[d] = 0.f;
#pragma unroll
    for (int j = 0; j < LKM; ++j) {
      if (j < prm.LK) {
        const float4* p4 = reinterpret_cast<const float4*>(pl + j * D);
#pragma unroll
        for (int i = 0; i < D / 4; ++i) {
          const float4 w = p4[i];
          dx[4 * i] = fmaf(dj[j], w.x, dx[4 * i]);
          dx[4 * i + 1] = fmaf(dj[j], w.y, dx[4 * i + 1]);
          dx[4 * i + 2] = fmaf(dj[j], w.z, dx[4 * i + 2]);
          dx[4 * i + 3] = fmaf(dj[j], w.w, dx[4 * i + 3]);
        }
      }
    }
    T* o = dxb + t * prm.ldq.st;
    if constexpr (sizeof(T) == 4) {
#pragma unroll
      for (int i = 0; i < D / 4; ++i)
        reinterpret_cast<float4*>(o)[i] = make_float4(dx[4 * i], dx[4 * i + 1], dx[4 * i + 2], dx[4 * i + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < D / 2; ++i)
        reinterpret_cast<__nv_bfloat162*>(o)[i] = __floats2bfloat162_rn(dx[2 * i], dx[2 * i + 1]);
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) ds += __shfl_xor_sync(0xffffffffu, ds, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ds;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int i = 0; i < NT / 32; ++i) tot += red[i];
    dscale_part[(size_t)blockIdx.y * gridDim.x + blockIdx.x] = tot;
  }
}

template <typename T, int D>
cudaError_t launch_pair(bool bwd, const Params& prm, float* out_or_dp, float* part,
                        cudaStream_t s) {
  const dim3 grid((unsigned)((prm.T + NT - 1) / NT), (unsigned)prm.N);
  if (!bwd)
    k_probs_fwd<T, D><<<grid, NT, 0, s>>>(prm, out_or_dp);
  else
    k_probs_bwd<T, D><<<grid, NT, 0, s>>>(prm, out_or_dp, part);
  return cudaGetLastError();
}

}  // namespace probs

cudaError_t launch_probs(bool bwd, bool bf16, int D, const Params& prm, float* out_or_dp,
                         float* part, cudaStream_t s) {
  if (bf16)
    return D == 32 ? probs::launch_pair<__nv_bfloat16, 32>(bwd, prm, out_or_dp, part, s)
                   : probs::launch_pair<__nv_bfloat16, 64>(bwd, prm, out_or_dp, part, s);
  return D == 32 ? probs::launch_pair<float, 32>(bwd, prm, out_or_dp, part, s)
                 : probs::launch_pair<float, 64>(bwd, prm, out_or_dp, part, s);
}

int64_t probs_blocks(int64_t T) { return (T + probs::NT - 1) / probs::NT; }

}  // namespace race
