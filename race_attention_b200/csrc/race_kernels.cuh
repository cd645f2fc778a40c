// race_kernels.cuh -- sm_100a kernels of RACE attention (forward + backward).
//
// Work mapping ("column owners").  A token is handled by a GROUP of W = D/C
// consecutive lanes; lane c of the group owns head-dim columns [c*C, c*C+C).
// A group streams its tokens' rows straight from HBM with coalesced vector
// loads (a group reads one contiguous d-row per token) and keeps the [S][C]
// slice of every bucket state it needs in registers, so the bucket
// aggregation B += p v^T, the readout out = sum_s p_s E_s, dv = sum_s p_s dB_s
// and the causal recurrences need no cross-lane traffic at all.  Only the
// hyperplane projections (dot products over d) and dp_s = <row, state_s> need
// a reduction across the group: a transpose-reduce over W lanes that leaves
// lane c with the totals of a contiguous block of entries.
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
  unsigned* err;         // sticky device error word (workspace tail), 0 = ok
  double* tilemass;      // causal: key mass at every 32-token tile start [N][tiles][S8]
};

__host__ __device__ constexpr int round_up(int a, int b) { return (a + b - 1) / b * b; }

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

// ---------------------------------------------------------------- group reduce
// Sums v[0..NV) over the W lanes of a group (lane index c).  Afterwards lane c
// holds in v[0..NV/W) the totals of entries [c*NV/W, (c+1)*NV/W).  Each round
// halves the live entries: lanes with bit O set keep the upper half and send
// the lower half to their partner, which does the opposite.
template <int NV, int O>
struct TransposeReduce {
  static __device__ __forceinline__ void run(float* v, int c) {
    const bool upper = (c & O) != 0;
#pragma unroll
    for (int i = 0; i < NV / 2; ++i) {
      const float send = upper ? v[i] : v[i + NV / 2];
      const float keep = upper ? v[i + NV / 2] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, O);
    }
    TransposeReduce<NV / 2, O / 2>::run(v, c);
  }
};
template <int NV>
struct TransposeReduce<NV, 0> {
  static __device__ __forceinline__ void run(float*, int) {}
};

template <int NV, int W>
__device__ __forceinline__ void group_reduce(float (&v)[NV], int c) {
  static_assert(NV % W == 0, "NV must be a multiple of the group width");
  TransposeReduce<NV, W / 2>::run(v, c);
}

// ---------------------------------------------------------------- per-group scratch
template <int D, int C, int SPAD>
struct Geo {
  static constexpr int W = D / C;                       // lanes per token
  static constexpr int GPW = 32 / W;                    // groups per warp
  static constexpr int G = kThreads / W;                // groups per CTA
  static constexpr int NVH = round_up(kLKMax, W);       // padded plane count
  static constexpr int KH = NVH / W;                    // planes finalised per lane
  static constexpr int SPV = round_up(SPAD, W);         // padded bucket count
  static constexpr int KS = SPV / W;                    // buckets owned per lane
  // scratch floats per group: sigmoid(+), sigmoid(-), p, dp, w, dproj
  static constexpr int SP_OFF = 0;
  static constexpr int SM_OFF = NVH;
  static constexpr int P_OFF = 2 * NVH;
  static constexpr int DP_OFF = P_OFF + SPV;
  static constexpr int W_OFF = DP_OFF + SPV;
  static constexpr int DPROJ_OFF = W_OFF + SPV;
  static constexpr int SCR = round_up(DPROJ_OFF + NVH, 4);
  static_assert(W >= 1 && W <= 32 && (32 % W) == 0, "bad group width");
};

struct Shape {
  int K, L, R, S, LK;
  __device__ __forceinline__ explicit Shape(const Params& p)
      : K(p.K), L(p.L), R(p.R), S(p.S), LK(p.LK) {}
};

// Projects the row x (this lane's C columns) onto the stream's planes and
// turns the projections into bucket probabilities.  On return
//   scr[P_OFF + s] = p_s for every s (0 for padding and invalid tokens),
//   pmine[i]       = p_s for the buckets s = c*KS + i this lane owns,
//   h[i]           = tanh(x . P_j) for the planes j = c*KH + i it finalised.
template <int D, int C, int SPAD>
__device__ __forceinline__ void soft_hash(const float (&x)[C], const float* __restrict__ pl,
                                          const Shape& sh, float inv_scale, int c, float* scr,
                                          bool valid, float (&pmine)[Geo<D, C, SPAD>::KS],
                                          float (&h)[Geo<D, C, SPAD>::KH]) {
  using Gm = Geo<D, C, SPAD>;
  float v[Gm::NVH];
#pragma unroll
  for (int j = 0; j < Gm::NVH; ++j) {
    float acc = 0.f;
    if (j < kLKMax && j < sh.LK) {
      float w[C];
      ld_row<float, C>(pl + j * D + c * C, w);
#pragma unroll
      for (int i = 0; i < C; ++i) acc = fmaf(x[i], w[i], acc);
    }
    v[j] = acc;
  }
  group_reduce<Gm::NVH, Gm::W>(v, c);
#pragma unroll
  for (int i = 0; i < Gm::KH; ++i) {
    const int j = c * Gm::KH + i;
    const float hh = tanhf(v[i]);
    h[i] = hh;
    const float u = hh * inv_scale;
    const float e = __expf(-2.f * fabsf(u));
    const float r = __frcp_rn(1.f + e);
    const float big = r, small = e * r;  // sigmoid(2|u|), sigmoid(-2|u|)
    if (j < sh.LK) {
      scr[Gm::SP_OFF + j] = u >= 0.f ? big : small;
      scr[Gm::SM_OFF + j] = u >= 0.f ? small : big;
    }
  }
  __syncwarp();
#pragma unroll
  for (int i = 0; i < Gm::KS; ++i) {
    const int s = c * Gm::KS + i;
    float pr = 0.f;
    if (valid && s < sh.S) {
      const int l = s >> sh.K;
      const int r = s & (sh.R - 1);
      pr = 1.f;
      for (int kk = 0; kk < sh.K; ++kk) {
        const int j = l * sh.K + kk;
        pr *= ((r >> (sh.K - 1 - kk)) & 1) ? scr[Gm::SP_OFF + j] : scr[Gm::SM_OFF + j];
      }
    }
    pmine[i] = pr;
    scr[Gm::P_OFF + s] = pr;
  }
  __syncwarp();
}

// Backward of soft_hash.  Needs scr[P_OFF..] = p and scr[DP_OFF..] = dL/dp for
// every bucket.  Accumulates sum_j du_j h_j into ds (the caller scales it by
// -1/scale^2) and returns this lane's columns of dx = sum_j dproj_j P_j.
template <int D, int C, int SPAD>
__device__ __forceinline__ void soft_hash_backward(const float* __restrict__ pl, const Shape& sh,
                                                   float inv_scale, int c, float* scr, bool valid,
                                                   const float (&h)[Geo<D, C, SPAD>::KH],
                                                   float& ds, float (&dx)[C]) {
  using Gm = Geo<D, C, SPAD>;
#pragma unroll
  for (int i = 0; i < Gm::KH; ++i) {
    const int j = c * Gm::KH + i;
    float dproj = 0.f;
    if (valid && j < sh.LK) {
      const int l = j / sh.K;
      const int bit = sh.K - 1 - (j - l * sh.K);
      const float* pp = scr + Gm::P_OFF + l * sh.R;
      const float* dd = scr + Gm::DP_OFF + l * sh.R;
      float pbar = 0.f;
      for (int r = 0; r < sh.R; ++r) pbar = fmaf(pp[r], dd[r], pbar);
      float du = 0.f;
      for (int r = 0; r < sh.R; ++r) {
        const float g = pp[r] * (dd[r] - pbar);
        du += ((r >> bit) & 1) ? g : -g;
      }
      ds = fmaf(du, h[i], ds);
      dproj = du * inv_scale * (1.f - h[i] * h[i]);
    }
    scr[Gm::DPROJ_OFF + j] = dproj;
  }
  __syncwarp();
#pragma unroll
  for (int i = 0; i < C; ++i) dx[i] = 0.f;
  for (int j = 0; j < sh.LK; ++j) {
    const float g = scr[Gm::DPROJ_OFF + j];
    float w[C];
    ld_row<float, C>(pl + j * D + c * C, w);
#pragma unroll
    for (int i = 0; i < C; ++i) dx[i] = fmaf(g, w[i], dx[i]);
  }
  __syncwarp();
}

// Reads p (or any per-bucket vector) for all SPAD buckets from group scratch.
template <int SPAD>
__device__ __forceinline__ void ld_buckets(const float* src, float (&p)[SPAD]) {
#pragma unroll
  for (int s = 0; s < SPAD; s += 4) {
    const float4 t = *reinterpret_cast<const float4*>(src + s);
    p[s] = t.x; p[s + 1] = t.y; p[s + 2] = t.z; p[s + 3] = t.w;
  }
}

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

// Reduces acc[SPAD][C] of every group of the CTA into red[SPAD*D] (fixed
// order: groups of a warp by xor-shuffle, then warps one after another).
template <int D, int C, int SPAD>
__device__ __forceinline__ void cta_reduce_slots(float (&acc)[SPAD][C], float* red, int c) {
  using Gm = Geo<D, C, SPAD>;
#pragma unroll
  for (int o = Gm::W; o < 32; o <<= 1)
#pragma unroll
    for (int s = 0; s < SPAD; ++s)
#pragma unroll
      for (int i = 0; i < C; ++i) acc[s][i] += __shfl_xor_sync(0xffffffffu, acc[s][i], o);
  const int warp = threadIdx.x >> 5;
  const bool leader = (threadIdx.x & 31) < Gm::W;
  for (int w = 0; w < kWarps; ++w) {
    if (warp == w && leader) {
#pragma unroll
      for (int s = 0; s < SPAD; ++s) {
        float t[C];
        if (w == 0) {
#pragma unroll
          for (int i = 0; i < C; ++i) t[i] = acc[s][i];
        } else {
          ld_f<C>(red + s * D + c * C, t);
#pragma unroll
          for (int i = 0; i < C; ++i) t[i] += acc[s][i];
        }
        st_f<C>(red + s * D + c * C, t);
      }
    }
    __syncthreads();
  }
}

// Same for lane-owned bucket scalars a[KS] (bucket s = c*KS + i) into red[SPV].
template <int D, int C, int SPAD>
__device__ __forceinline__ void cta_reduce_mine(const float (&a)[Geo<D, C, SPAD>::KS], float* red,
                                                int c) {
  using Gm = Geo<D, C, SPAD>;
  float t[Gm::KS];
#pragma unroll
  for (int i = 0; i < Gm::KS; ++i) {
    t[i] = a[i];
#pragma unroll
    for (int o = Gm::W; o < 32; o <<= 1) t[i] += __shfl_xor_sync(0xffffffffu, t[i], o);
  }
  const int warp = threadIdx.x >> 5;
  const bool leader = (threadIdx.x & 31) < Gm::W;
  for (int w = 0; w < kWarps; ++w) {
    if (warp == w && leader) {
#pragma unroll
      for (int i = 0; i < Gm::KS; ++i) {
        const int s = c * Gm::KS + i;
        red[s] = (w == 0) ? t[i] : red[s] + t[i];
      }
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------- kernels
// Dynamic shared memory: per-group scratch, then a CTA reduction area.
template <int D, int C, int SPAD>
__host__ __device__ constexpr int smem_floats() {
  using Gm = Geo<D, C, SPAD>;
  return Gm::G * Gm::SCR + SPAD * D + Gm::SPV + 32 + SPAD * D;
}

#define RACE_KERNEL_PROLOGUE                                              \
  using Gm = Geo<D, C, SPAD>;                                            \
  extern __shared__ __align__(16) float smem[];                          \
  const int lane = threadIdx.x & 31;                                     \
  const int c = lane % Gm::W;                                            \
  const int g = threadIdx.x / Gm::W;                                     \
  float* scr = smem + g * Gm::SCR;                                       \
  float* red = smem + Gm::G * Gm::SCR;       /* SPAD*D + SPV floats */   \
  float* red32 = red + SPAD * D + Gm::SPV;   /* 32 floats */             \
  float* tab = red32 + 32;                   /* SPAD*D floats */         \
  const Shape sh(prm);                                                   \
  const float inv_scale = 1.f / __ldg(prm.scale);                        \
  (void)tab; (void)red32;

__device__ __forceinline__ void token_range(int64_t T, int P, int part, int64_t& t0, int64_t& t1) {
  t0 = (T * part) / P;
  t1 = (T * (part + 1)) / P;
}

// Sums P partial slots per stream in a fixed order: out[n] = sum_p part[n][p].
__global__ void __launch_bounds__(1024) k_sum_partials(const float* __restrict__ part, int P, int SS,
                                                       float* __restrict__ out);

// ---------------------------------------------------------------- causal
// Work unit = one chunk of CL consecutive tokens of one stream, walked in
// order by one group.  Units u = n * NC + chunk are spread over the grid.
struct Unit {
  int n;
  int64_t chunk, t0, t1;
  bool live;
};

__device__ __forceinline__ Unit unit_of(const Params& prm, int64_t u) {
  Unit r;
  const int64_t total = (int64_t)prm.N * prm.NC;
  r.live = u < total;
  const int64_t uu = r.live ? u : 0;
  r.n = (int)(uu / prm.NC);
  r.chunk = uu % prm.NC;
  r.t0 = r.chunk * prm.CL;
  r.t1 = min(prm.T, r.t0 + prm.CL);
  if (!r.live) r.t1 = r.t0;
  return r;
}

// CF1: chunk totals of p_K v^T and p_K, one slot per chunk.
template <typename T, int D, int C, int SPAD>
__global__ void __launch_bounds__(kThreads) k_c_totals(const Params prm) {
  RACE_KERNEL_PROLOGUE
  const int64_t u = (int64_t)blockIdx.x * Gm::G + g;
  const Unit U = unit_of(prm, u);
  const int m = prm.Mp == 1 ? 0 : U.n / (prm.B * prm.H);
  const float* pl = prm.planes + (size_t)m * prm.LK * D;
  const T* kb = static_cast<const T*>(prm.k) + stream_offset(prm.lk, U.n, prm.B, prm.H) + c * C;
  const T* vb = static_cast<const T*>(prm.v) + stream_offset(prm.lv, U.n, prm.B, prm.H) + c * C;
  float acc[SPAD][C];
#pragma unroll
  for (int s = 0; s < SPAD; ++s)
#pragma unroll
    for (int i = 0; i < C; ++i) acc[s][i] = 0.f;
  float amass[Gm::KS];
#pragma unroll
  for (int i = 0; i < Gm::KS; ++i) amass[i] = 0.f;
  float xk[C] = {}, xv[C] = {}, nk[C] = {}, nv[C] = {};
  if (U.t0 < U.t1) {
    ld_row<T, C>(kb + U.t0 * prm.lk.st, xk);
    ld_row<T, C>(vb + U.t0 * prm.lv.st, xv);
  }
  for (int i = 0; i < prm.CL; ++i) {
    const int64_t t = U.t0 + i;
    const bool valid = t < U.t1;
    if (t + 1 < U.t1) {
      ld_row<T, C>(kb + (t + 1) * prm.lk.st, nk);
      ld_row<T, C>(vb + (t + 1) * prm.lv.st, nv);
    }
    float pm[Gm::KS], hk[Gm::KH];
    soft_hash<D, C, SPAD>(xk, pl, sh, inv_scale, c, scr, valid, pm, hk);
#pragma unroll
    for (int j = 0; j < Gm::KS; ++j) amass[j] += pm[j];
    float p[SPAD];
    ld_buckets<SPAD>(scr + Gm::P_OFF, p);
#pragma unroll
    for (int s = 0; s < SPAD; ++s)
#pragma unroll
      for (int j = 0; j < C; ++j) acc[s][j] = fmaf(p[s], xv[j], acc[s][j]);
#pragma unroll
    for (int j = 0; j < C; ++j) { xk[j] = nk[j]; xv[j] = nv[j]; }
  }
  if (U.live) {
    float* dst = prm.state_out + (size_t)u * prm.SS;
#pragma unroll
    for (int s = 0; s < SPAD; ++s)
      if (s < sh.S) st_f<C>(dst + s * D + c * C, acc[s]);
#pragma unroll
    for (int j = 0; j < Gm::KS; ++j) {
      const int s = c * Gm::KS + j;
      if (s < sh.S) dst[sh.S * D + s] = amass[j];
    }
  }
}

// CF2: per-chunk recurrence from the chunk's exclusive prefix:
//   A += pK, B += pK v, out = sum_s pQ_s / (A_s + eps) * B_s.
// The bucket mass is carried in float64 (lane-owned buckets).
template <typename T, int D, int C, int SPAD>
__global__ void __launch_bounds__(kThreads) k_c_fwd(const Params prm) {
  RACE_KERNEL_PROLOGUE
  const int64_t u = (int64_t)blockIdx.x * Gm::G + g;
  const Unit U = unit_of(prm, u);
  const int m = prm.Mp == 1 ? 0 : U.n / (prm.B * prm.H);
  const float* pl = prm.planes + (size_t)m * prm.LK * D;
  const float* st = prm.state + (size_t)(U.live ? u : 0) * prm.SS;
  float Bs[SPAD][C];
#pragma unroll
  for (int s = 0; s < SPAD; ++s) {
    if (s < sh.S) ld_f<C>(st + s * D + c * C, Bs[s]);
    else
#pragma unroll
      for (int j = 0; j < C; ++j) Bs[s][j] = 0.f;
  }
  double Am[Gm::KS];
#pragma unroll
  for (int j = 0; j < Gm::KS; ++j) {
    const int s = c * Gm::KS + j;
    Am[j] = s < sh.S ? (double)st[sh.S * D + s] : 0.0;
  }
  const int64_t ob = stream_offset(prm.lo, U.n, prm.B, prm.H) + c * C;
  const T* qb = static_cast<const T*>(prm.q) + stream_offset(prm.lq, U.n, prm.B, prm.H) + c * C;
  const T* kb = static_cast<const T*>(prm.k) + stream_offset(prm.lk, U.n, prm.B, prm.H) + c * C;
  const T* vb = static_cast<const T*>(prm.v) + stream_offset(prm.lv, U.n, prm.B, prm.H) + c * C;
  T* outb = static_cast<T*>(prm.out) + ob;
  float xq[C] = {}, xk[C] = {}, xv[C] = {}, nq[C] = {}, nk[C] = {}, nv[C] = {};
  if (U.t0 < U.t1) {
    ld_row<T, C>(qb + U.t0 * prm.lq.st, xq);
    ld_row<T, C>(kb + U.t0 * prm.lk.st, xk);
    ld_row<T, C>(vb + U.t0 * prm.lv.st, xv);
  }
  for (int i = 0; i < prm.CL; ++i) {
    const int64_t t = U.t0 + i;
    const bool valid = t < U.t1;
    if (t + 1 < U.t1) {
      ld_row<T, C>(qb + (t + 1) * prm.lq.st, nq);
      ld_row<T, C>(kb + (t + 1) * prm.lk.st, nk);
      ld_row<T, C>(vb + (t + 1) * prm.lv.st, nv);
    }
    float pm[Gm::KS], hh[Gm::KH];
    soft_hash<D, C, SPAD>(xk, pl, sh, inv_scale, c, scr, valid, pm, hh);
    {
      float p[SPAD];
      ld_buckets<SPAD>(scr + Gm::P_OFF, p);
#pragma unroll
      for (int s = 0; s < SPAD; ++s)
#pragma unroll
        for (int j = 0; j < C; ++j) Bs[s][j] = fmaf(p[s], xv[j], Bs[s][j]);
    }
#pragma unroll
    for (int j = 0; j < Gm::KS; ++j) Am[j] += (double)pm[j];
    soft_hash<D, C, SPAD>(xq, pl, sh, inv_scale, c, scr, valid, pm, hh);
#pragma unroll
    for (int j = 0; j < Gm::KS; ++j)
      scr[Gm::DP_OFF + c * Gm::KS + j] = pm[j] / (float)(Am[j] + (double)prm.eps);
    __syncwarp();
    float w[SPAD];
    ld_buckets<SPAD>(scr + Gm::DP_OFF, w);
    float o[C];
#pragma unroll
    for (int j = 0; j < C; ++j) o[j] = 0.f;
#pragma unroll
    for (int s = 0; s < SPAD; ++s)
#pragma unroll
      for (int j = 0; j < C; ++j) o[j] = fmaf(w[s], Bs[s][j], o[j]);
    if (valid) st_row<T, C>(outb + t * prm.lo.st, o);
    __syncwarp();
#pragma unroll
    for (int j = 0; j < C; ++j) { xq[j] = nq[j]; xk[j] = nk[j]; xv[j] = nv[j]; }
  }
}

// CB1: forward walk of the chunk with the saved prefix.  Per token:
//   dpQ_s = <dO, B_s> / (A_s + eps)  -> dq (through the soft hash)
//   alpha_s = -W_s dpQ_s (stored per token), W_s = pQ_s / (A_s + eps)
// and the chunk's gradient totals sum_t W_s dO, sum_t alpha_s plus its key
// mass (float64) for the reverse walk of CB2.
template <typename T, int D, int C, int SPAD>
__global__ void __launch_bounds__(kThreads) k_c_bwd_q(const Params prm) {
  RACE_KERNEL_PROLOGUE
  const int64_t u = (int64_t)blockIdx.x * Gm::G + g;
  const Unit U = unit_of(prm, u);
  const int m = prm.Mp == 1 ? 0 : U.n / (prm.B * prm.H);
  const float* pl = prm.planes + (size_t)m * prm.LK * D;
  const float* st = prm.state + (size_t)(U.live ? u : 0) * prm.SS;
  float Bs[SPAD][C], GB[SPAD][C];
#pragma unroll
  for (int s = 0; s < SPAD; ++s) {
    if (s < sh.S) ld_f<C>(st + s * D + c * C, Bs[s]);
    else
#pragma unroll
      for (int j = 0; j < C; ++j) Bs[s][j] = 0.f;
#pragma unroll
    for (int j = 0; j < C; ++j) GB[s][j] = 0.f;
  }
  double A0[Gm::KS], Al[Gm::KS];
  float GA[Gm::KS];
#pragma unroll
  for (int j = 0; j < Gm::KS; ++j) {
    const int s = c * Gm::KS + j;
    A0[j] = s < sh.S ? (double)st[sh.S * D + s] : 0.0;
    Al[j] = 0.0;
    GA[j] = 0.f;
  }
  const T* qb = static_cast<const T*>(prm.q) + stream_offset(prm.lq, U.n, prm.B, prm.H) + c * C;
  const T* kb = static_cast<const T*>(prm.k) + stream_offset(prm.lk, U.n, prm.B, prm.H) + c * C;
  const T* vb = static_cast<const T*>(prm.v) + stream_offset(prm.lv, U.n, prm.B, prm.H) + c * C;
  const T* gb = static_cast<const T*>(prm.dout) + stream_offset(prm.ldo, U.n, prm.B, prm.H) + c * C;
  T* dqb = static_cast<T*>(prm.dq) + stream_offset(prm.ldq, U.n, prm.B, prm.H) + c * C;
  float* alpha = prm.alpha + (size_t)U.n * prm.T * sh.S;
  float ds = 0.f;
  float xq[C] = {}, xk[C] = {}, xv[C] = {}, xg[C] = {}, nq[C] = {}, nk[C] = {}, nv[C] = {}, ng[C] = {};
  if (U.t0 < U.t1) {
    ld_row<T, C>(qb + U.t0 * prm.lq.st, xq);
    ld_row<T, C>(kb + U.t0 * prm.lk.st, xk);
    ld_row<T, C>(vb + U.t0 * prm.lv.st, xv);
    ld_row<T, C>(gb + U.t0 * prm.ldo.st, xg);
  }
  for (int i = 0; i < prm.CL; ++i) {
    const int64_t t = U.t0 + i;
    const bool valid = t < U.t1;
    if (t + 1 < U.t1) {
      ld_row<T, C>(qb + (t + 1) * prm.lq.st, nq);
      ld_row<T, C>(kb + (t + 1) * prm.lk.st, nk);
      ld_row<T, C>(vb + (t + 1) * prm.lv.st, nv);
      ld_row<T, C>(gb + (t + 1) * prm.ldo.st, ng);
    }
    if (!valid) {
#pragma unroll
      for (int j = 0; j < C; ++j) xg[j] = 0.f;
    }
    float pm[Gm::KS], hh[Gm::KH];
    soft_hash<D, C, SPAD>(xk, pl, sh, inv_scale, c, scr, valid, pm, hh);
    {
      float p[SPAD];
      ld_buckets<SPAD>(scr + Gm::P_OFF, p);
#pragma unroll
      for (int s = 0; s < SPAD; ++s)
#pragma unroll
        for (int j = 0; j < C; ++j) Bs[s][j] = fmaf(p[s], xv[j], Bs[s][j]);
    }
#pragma unroll
    for (int j = 0; j < Gm::KS; ++j) Al[j] += (double)pm[j];
    // <dO, B_s> for every bucket
    float dpv[Gm::SPV];
#pragma unroll
    for (int s = 0; s < Gm::SPV; ++s) dpv[s] = 0.f;
#pragma unroll
    for (int s = 0; s < SPAD; ++s) {
      float d = 0.f;
#pragma unroll
      for (int j = 0; j < C; ++j) d = fmaf(xg[j], Bs[s][j], d);
      dpv[s] = d;
    }
    group_reduce<Gm::SPV, Gm::W>(dpv, c);
    soft_hash<D, C, SPAD>(xq, pl, sh, inv_scale, c, scr, valid, pm, hh);
    float* arow = alpha + (size_t)t * sh.S;
#pragma unroll
    for (int j = 0; j < Gm::KS; ++j) {
      const int s = c * Gm::KS + j;
      const float inv = (float)(1.0 / (A0[j] + Al[j] + (double)prm.eps));
      const float w = pm[j] * inv;
      const float dpq = dpv[j] * inv;
      const float al = -w * dpq;
      GA[j] += al;
      scr[Gm::DP_OFF + s] = dpq;
      scr[Gm::W_OFF + s] = w;
      if (valid && s < sh.S) arow[s] = al;
    }
    __syncwarp();
    {
      float w[SPAD];
      ld_buckets<SPAD>(scr + Gm::W_OFF, w);
#pragma unroll
      for (int s = 0; s < SPAD; ++s)
#pragma unroll
        for (int j = 0; j < C; ++j) GB[s][j] = fmaf(w[s], xg[j], GB[s][j]);
    }
    __syncwarp();
    float dx[C];
    soft_hash_backward<D, C, SPAD>(pl, sh, inv_scale, c, scr, valid, hh, ds, dx);
    if (valid) st_row<T, C>(dqb + t * prm.ldq.st, dx);
#pragma unroll
    for (int j = 0; j < C; ++j) { xq[j] = nq[j]; xk[j] = nk[j]; xv[j] = nv[j]; xg[j] = ng[j]; }
  }
  if (U.live) {
    float* dst = prm.gstate_out + (size_t)u * prm.SS;
#pragma unroll
    for (int s = 0; s < SPAD; ++s)
      if (s < sh.S) st_f<C>(dst + s * D + c * C, GB[s]);
    double* amass = reinterpret_cast<double*>(dst + sh.S * D + sh.S);
#pragma unroll
    for (int j = 0; j < Gm::KS; ++j) {
      const int s = c * Gm::KS + j;
      if (s < sh.S) {
        dst[sh.S * D + s] = GA[j];
        amass[s] = Al[j];
      }
    }
  }
  const float tot = cta_sum(ds, red32);
  if (threadIdx.x == 0) prm.dscale_part[blockIdx.x] = tot;
}

// CB2 is instantiated with the same column split as CB1 (C = 2) so both walks
// hash every key to bit-identical probabilities: the key mass A_s(t) is
// rebuilt here by subtracting them from CB1's chunk total, and for the first
// tokens of a sequence A_s(t) can be ~1e-5, where two differently rounded
// hashes would disagree by 1e-3 relative.
// CB2: reverse walk of the chunk from its exclusive gradient suffix:
//   beta_s += W_s dO, alpha_suf_s += alpha_s, dv = sum_s pK_s beta_s,
//   dpK_s = alpha_suf_s + <beta_s, v>  -> dk.
// The key mass A_s(t) is rebuilt backwards in float64 from the chunk's
// prefix plus its float64 chunk mass written by CB1.
template <typename T, int D, int C, int SPAD>
__global__ void __launch_bounds__(kThreads) k_c_bwd_kv(const Params prm) {
  RACE_KERNEL_PROLOGUE
  const int64_t u = (int64_t)blockIdx.x * Gm::G + g;
  const Unit U = unit_of(prm, u);
  const int m = prm.Mp == 1 ? 0 : U.n / (prm.B * prm.H);
  const float* pl = prm.planes + (size_t)m * prm.LK * D;
  const size_t uu = (size_t)(U.live ? u : 0);
  const float* st = prm.state + uu * prm.SS;
  const float* gsuf = prm.gstate_in + uu * prm.SS;
  const double* amass = reinterpret_cast<const double*>(gsuf + sh.S * D + sh.S);
  float beta[SPAD][C];
#pragma unroll
  for (int s = 0; s < SPAD; ++s) {
    if (s < sh.S) ld_f<C>(gsuf + s * D + c * C, beta[s]);
    else
#pragma unroll
      for (int j = 0; j < C; ++j) beta[s][j] = 0.f;
  }
  double A[Gm::KS];
  float asuf[Gm::KS];
#pragma unroll
  for (int j = 0; j < Gm::KS; ++j) {
    const int s = c * Gm::KS + j;
    A[j] = s < sh.S ? (double)st[sh.S * D + s] + amass[s] : 0.0;
    asuf[j] = s < sh.S ? gsuf[sh.S * D + s] : 0.f;
  }
  const T* qb = static_cast<const T*>(prm.q) + stream_offset(prm.lq, U.n, prm.B, prm.H) + c * C;
  const T* kb = static_cast<const T*>(prm.k) + stream_offset(prm.lk, U.n, prm.B, prm.H) + c * C;
  const T* vb = static_cast<const T*>(prm.v) + stream_offset(prm.lv, U.n, prm.B, prm.H) + c * C;
  const T* gb = static_cast<const T*>(prm.dout) + stream_offset(prm.ldo, U.n, prm.B, prm.H) + c * C;
  T* dkb = static_cast<T*>(prm.dk) + stream_offset(prm.ldk, U.n, prm.B, prm.H) + c * C;
  T* dvb = static_cast<T*>(prm.dv) + stream_offset(prm.ldv, U.n, prm.B, prm.H) + c * C;
  const float* alpha = prm.alpha + (size_t)U.n * prm.T * sh.S;
  float ds = 0.f;
  const int64_t last = U.t1 - 1;
  float xq[C] = {}, xk[C] = {}, xv[C] = {}, xg[C] = {}, nq[C] = {}, nk[C] = {}, nv[C] = {}, ng[C] = {};
  if (U.t0 < U.t1) {
    ld_row<T, C>(qb + last * prm.lq.st, xq);
    ld_row<T, C>(kb + last * prm.lk.st, xk);
    ld_row<T, C>(vb + last * prm.lv.st, xv);
    ld_row<T, C>(gb + last * prm.ldo.st, xg);
  }
  // iteration i handles token t1-1-i; tokens before t0 are invalid padding
  for (int i = 0; i < prm.CL; ++i) {
    const int64_t t = last - i;
    const bool valid = t >= U.t0;
    if (t - 1 >= U.t0) {
      ld_row<T, C>(qb + (t - 1) * prm.lq.st, nq);
      ld_row<T, C>(kb + (t - 1) * prm.lk.st, nk);
      ld_row<T, C>(vb + (t - 1) * prm.lv.st, nv);
      ld_row<T, C>(gb + (t - 1) * prm.ldo.st, ng);
    }
    if (!valid) {
#pragma unroll
      for (int j = 0; j < C; ++j) xg[j] = 0.f;
    }
    float pm[Gm::KS], hh[Gm::KH];
    soft_hash<D, C, SPAD>(xq, pl, sh, inv_scale, c, scr, valid, pm, hh);
    const float* arow = alpha + (size_t)(valid ? t : 0) * sh.S;
#pragma unroll
    for (int j = 0; j < Gm::KS; ++j) {
      const int s = c * Gm::KS + j;
      const float w = pm[j] * (float)(1.0 / (A[j] + (double)prm.eps));
      scr[Gm::DP_OFF + s] = w;
      if (valid && s < sh.S) asuf[j] += arow[s];
    }
    __syncwarp();
    {
      float w[SPAD];
      ld_buckets<SPAD>(scr + Gm::DP_OFF, w);
#pragma unroll
      for (int s = 0; s < SPAD; ++s)
#pragma unroll
        for (int j = 0; j < C; ++j) beta[s][j] = fmaf(w[s], xg[j], beta[s][j]);
    }
    __syncwarp();
    soft_hash<D, C, SPAD>(xk, pl, sh, inv_scale, c, scr, valid, pm, hh);
    float p[SPAD];
    ld_buckets<SPAD>(scr + Gm::P_OFF, p);
    float dvv[C];
#pragma unroll
    for (int j = 0; j < C; ++j) dvv[j] = 0.f;
    float dpv[Gm::SPV];
#pragma unroll
    for (int s = 0; s < Gm::SPV; ++s) dpv[s] = 0.f;
#pragma unroll
    for (int s = 0; s < SPAD; ++s) {
      float d = 0.f;
#pragma unroll
      for (int j = 0; j < C; ++j) {
        dvv[j] = fmaf(p[s], beta[s][j], dvv[j]);
        d = fmaf(xv[j], beta[s][j], d);
      }
      dpv[s] = d;
    }
    if (valid) st_row<T, C>(dvb + t * prm.ldv.st, dvv);
    group_reduce<Gm::SPV, Gm::W>(dpv, c);
#pragma unroll
    for (int j = 0; j < Gm::KS; ++j) {
      scr[Gm::DP_OFF + c * Gm::KS + j] = dpv[j] + asuf[j];
      A[j] -= (double)pm[j];
    }
    __syncwarp();
    float dx[C];
    soft_hash_backward<D, C, SPAD>(pl, sh, inv_scale, c, scr, valid, hh, ds, dx);
    if (valid) st_row<T, C>(dkb + t * prm.ldk.st, dx);
#pragma unroll
    for (int j = 0; j < C; ++j) { xq[j] = nq[j]; xk[j] = nk[j]; xv[j] = nv[j]; xg[j] = ng[j]; }
  }
  const float tot = cta_sum(ds, red32);
  if (threadIdx.x == 0) prm.dscale_part[blockIdx.x] = tot;
}

}  // namespace race
