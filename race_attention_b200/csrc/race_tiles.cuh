// race_tiles.cuh -- tiled non-causal RACE kernels for sm_100a.
//
// A CTA (256 threads, 8 warps) walks a contiguous range of 64-token tiles of
// one stream.  The q/k/v/dO rows of the next tile are brought into shared
// memory with cp.async while the current tile is computed (two stages), so
// HBM streaming overlaps the arithmetic.  Per tile the work is a short chain
// of shared-memory tile operations:
//
//   hash     thread (token, quarter of d): projections onto the L*K planes,
//            combined over the 4 quarter-threads by two xor-shuffles; each
//            quarter-thread then owns tables l = q, q+4, ... of its token and
//            forms tanh, the sigmoids and the 2^K corner probabilities.
//   agg      B[s][d] += sum_t P[t][s] Y[t][d]: a warp owns 8 (or 16) tokens of
//            the tile, a lane owns 2 columns of every bucket row (registers,
//            kept across tiles, reduced over warps in a fixed order at the end).
//   readout  O[t][d] = sum_k A^T[k][t] B[k][d]: 2 tokens x 8 columns a thread.
//   rowdot   DP[t][s] = sum_d X[t][d] TAB[s][d]: 2 tokens x S/4 buckets a
//            thread.
//   softmax backward per (token, table) in the hash layout, then the
//   back-projection dx = dproj . planes as a readout.
//
// Register tiles are shaped so each shared-memory wavefront feeds >= 5 warp
// FMAs (the SM issues 4 warp instructions per clock but serves one
// wavefront).  Row strides of D+4 floats keep the row-parallel accesses
// conflict-free.
#pragma once

#include "race_kernels.cuh"

namespace race {
namespace tiles {

constexpr int TT = 64;     // tokens per tile
constexpr int NT = 256;    // threads per CTA
constexpr int LKP = 16;    // plane rows (L*K <= 16)

template <int D, int SPAD, bool BF = false>
struct Lay {
  static constexpr int NSTAGE = BF ? 1 : 2;   // fp32 tile stages (bf16 stages raw rows)
  static constexpr int RS = D + 4;       // fp32 row stride of X / Y / PL / TAB
  // row stride of P / DP [t][s]; 16 makes the float4 reads of one table by a
  // quarter-warp (2 tokens x 4 tables) conflict-free; SPAD + 4 for wider rows
  // (at most 2-way conflicts) keeps two CTAs' shared memory within the SM
  static constexpr int PS = SPAD <= 16 ? 16 : SPAD + 4;
  static constexpr int TS = TT + 4;      // row stride of PT / DJT [k][t]
  static constexpr int SQ = SPAD / 4;    // buckets per rowdot thread
  static constexpr int XS = 0;                       // [NSTAGE][TT][RS]
  static constexpr int YS = XS + NSTAGE * TT * RS;   // [NSTAGE][TT][RS]
  static constexpr int PL = YS + NSTAGE * TT * RS;   // [LKP][RS]
  static constexpr int TAB = PL + LKP * RS;          // [SPAD][RS]
  static constexpr int H = TAB + SPAD * RS;          // [TT][LKP+1] tanh(proj)
  static constexpr int P = H + TT * (LKP + 1);       // [TT][PS]
  static constexpr int PT = P + TT * PS;             // [SPAD][TS]
  static constexpr int DP = PT + SPAD * TS;          // [TT][PS]
  static constexpr int DJT = DP + TT * PS;           // [LKP][TS]
  static constexpr int MISC = DJT + LKP * TS;        // 64 floats: dA[s], reductions
  static constexpr int RAW = MISC + 64;              // bf16 staging [2][2][TT][D] halves
  static constexpr int RAW_FLOATS = BF ? 2 * 2 * TT * D / 2 : 0;
  static constexpr int FLOATS = RAW + RAW_FLOATS;
  static constexpr int Dv = D;
  static constexpr int Sv = SPAD;
  static_assert(SPAD % 4 == 0, "SPAD must be a multiple of 4");
};

// ------------------------------------------------------------------ cp.async
__device__ __forceinline__ unsigned smem_u32(const void* p) {
  return static_cast<unsigned>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(dst)), "l"(src),
               "r"(valid ? 16 : 0));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// tanh(x) = sign(x) (1 - e) / (1 + e), e = exp(-2|x|) (the exponential
// identity of the hyperbolic tangent); absolute error ~1e-7, which is all the
// soft hash needs since it only uses tanh(x)/scale as a logit.
__device__ __forceinline__ float tanh_exp(float x) {
  const float e = __expf(-2.f * fabsf(x));
  const float t = (1.f - e) * __frcp_rn(1.f + e);
  return copysignf(t, x);
}

// Stage one tile (rows t0 .. t0+TT-1 of a stream) of an element type T into
// shared memory: fp32 rows go straight into the padded fp32 tile, bf16 rows
// into the unpadded raw buffer (converted later by convert_tile).  Rows past
// the range are zero-filled.
template <typename T, int D, int NTH = NT, int TTL = TT>
__device__ __forceinline__ void stage_tile(float* fdst, void* rawdst, const T* base, int64_t st,
                                           int64_t t0, int64_t t1) {
  constexpr int RS = D + 4;
  if constexpr (sizeof(T) == 4) {
    constexpr int CPR = D / 4;  // 16-byte chunks per row
    for (int i = threadIdx.x; i < TTL * CPR; i += NTH) {
      const int r = i / CPR, ch = i % CPR;
      const int64_t t = t0 + r;
      const bool ok = t < t1;
      const T* src = base + (ok ? t : t0) * st + ch * 4;
      cp_async16(fdst + r * RS + ch * 4, src, ok);
    }
  } else {
    constexpr int CPR = D / 8;
    __nv_bfloat16* raw = static_cast<__nv_bfloat16*>(rawdst);
    for (int i = threadIdx.x; i < TTL * CPR; i += NTH) {
      const int r = i / CPR, ch = i % CPR;
      const int64_t t = t0 + r;
      const bool ok = t < t1;
      const T* src = base + (ok ? t : t0) * st + ch * 8;
      cp_async16(raw + r * D + ch * 8, src, ok);
    }
  }
}

template <int D, int NTH = NT, int TTL = TT>
__device__ __forceinline__ void convert_tile(float* fdst, const void* rawsrc) {
  constexpr int RS = D + 4;
  const __nv_bfloat16* raw = static_cast<const __nv_bfloat16*>(rawsrc);
  for (int i = threadIdx.x; i < TTL * D / 8; i += NTH) {
    const int r = i / (D / 8), ch = i % (D / 8);
    const uint4 u = *reinterpret_cast<const uint4*>(raw + r * D + ch * 8);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
    float4 a, b;
    float2 f;
    f = __bfloat1622float2(h[0]); a.x = f.x; a.y = f.y;
    f = __bfloat1622float2(h[1]); a.z = f.x; a.w = f.y;
    f = __bfloat1622float2(h[2]); b.x = f.x; b.y = f.y;
    f = __bfloat1622float2(h[3]); b.z = f.x; b.w = f.y;
    *reinterpret_cast<float4*>(fdst + r * RS + ch * 8) = a;
    *reinterpret_cast<float4*>(fdst + r * RS + ch * 8 + 4) = b;
  }
}

// ------------------------------------------------------------------ hash
// Thread (token t = 8*warp + lane/4, quarter q = lane%4).  The quarter owns the
// 16-byte column chunks {2q, 2q+1, 2q+8, 2q+9} (D=64; {2q, 2q+1} for D=32),
// which keeps each quarter-warp's row reads on distinct banks.  For every
// table l the four quarters form partial dot products with its K planes and
// combine them with two xor-shuffles; quarter l%4 owns the table and turns the
// projections into tanh (kept in H[t][l*K+k]), the sigmoids and the 2^K corner
// probabilities (P[t][s] and PT[s][t]).  K is a compile-time constant, so the
// corner products and the per-table loops carry no guards.
template <class LY, int K>
__device__ __forceinline__ void hash_tile(const float* __restrict__ X, float* sm, const Shape& sh,
                                          float inv_scale, int64_t valid_rows) {
  constexpr int D = LY::Dv;
  constexpr int R = 1 << K;
  constexpr int NCH = D / 16;  // chunks per quarter
  const int lane = threadIdx.x & 31;
  const int t = (threadIdx.x >> 5) * 8 + (lane >> 2);
  const int q = lane & 3;
  float x[NCH][4];
  const float* xr = X + t * LY::RS;
#pragma unroll
  for (int i = 0; i < NCH; ++i) {
    const int ch = 2 * q + (i & 1) + 8 * (i >> 1);
    const float4 v = *reinterpret_cast<const float4*>(xr + ch * 4);
    x[i][0] = v.x; x[i][1] = v.y; x[i][2] = v.z; x[i][3] = v.w;
  }
  const float pv = t < valid_rows ? 1.f : 0.f;
  float* Hrow = sm + LY::H + t * (LKP + 1);
  float* Prow = sm + LY::P + t * LY::PS;
  float* PT = sm + LY::PT;
  const float* pl = sm + LY::PL;
  for (int l = 0; l < sh.L; ++l) {
    float acc[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const float* row = pl + (l * K + k) * LY::RS;
      float a = 0.f;
#pragma unroll
      for (int i = 0; i < NCH; ++i) {
        const int ch = 2 * q + (i & 1) + 8 * (i >> 1);
        const float4 w = *reinterpret_cast<const float4*>(row + ch * 4);
        a = fmaf(x[i][0], w.x, fmaf(x[i][1], w.y, fmaf(x[i][2], w.z, fmaf(x[i][3], w.w, a))));
      }
      a += __shfl_xor_sync(0xffffffffu, a, 1);
      a += __shfl_xor_sync(0xffffffffu, a, 2);
      acc[k] = a;
    }
    if ((l & 3) == q) {
      float sp[K], sn[K];   // sigmoid(+2u), sigmoid(-2u) per plane of the table
#pragma unroll
      for (int k = 0; k < K; ++k) {
        const float h = tanh_exp(acc[k]);
        Hrow[l * K + k] = h;
        const float u = h * inv_scale;
        const float e = __expf(-2.f * fabsf(u));
        const float r = __frcp_rn(1.f + e);
        sp[k] = u >= 0.f ? r : e * r;
        sn[k] = u >= 0.f ? e * r : r;
      }
#pragma unroll
      for (int r = 0; r < R; ++r) {
        float p = pv;
#pragma unroll
        for (int k = 0; k < K; ++k) p *= ((r >> (K - 1 - k)) & 1) ? sp[k] : sn[k];
        const int s = l * R + r;
        Prow[s] = p;
        PT[s * LY::TS + t] = p;
      }
    }
  }
}

// Softmax / corner / tanh backward in the hash layout: reads P, DP (+dA when
// HAS_DA), H; writes DJT[j][t] = dL/dproj_j and accumulates sum_j du_j h_j.
// The owner quarter of each table loads its R probabilities and gradients
// once, forms g_r = p_r (dp_r - sum p dp) and the K plane sums from them.
template <class LY, int K, bool HAS_DA>
__device__ __forceinline__ void hash_backward(float* sm, const Shape& sh, float inv_scale,
                                              const float* dA, float& ds) {
  constexpr int R = 1 << K;
  const int lane = threadIdx.x & 31;
  const int t = (threadIdx.x >> 5) * 8 + (lane >> 2);
  const int q = lane & 3;
  const float* Hrow = sm + LY::H + t * (LKP + 1);
  const float* Prow = sm + LY::P + t * LY::PS;
  const float* Drow = sm + LY::DP + t * LY::PS;
  float* DJT = sm + LY::DJT;
  for (int l = q; l < sh.L; l += 4) {
    const int s0 = l * R;
    float p[R], d[R];
    if constexpr (R >= 4) {
#pragma unroll
      for (int c = 0; c < R / 4; ++c) {
        const float4 pp = *reinterpret_cast<const float4*>(Prow + s0 + 4 * c);
        const float4 dd = *reinterpret_cast<const float4*>(Drow + s0 + 4 * c);
        p[4 * c] = pp.x; p[4 * c + 1] = pp.y; p[4 * c + 2] = pp.z; p[4 * c + 3] = pp.w;
        d[4 * c] = dd.x; d[4 * c + 1] = dd.y; d[4 * c + 2] = dd.z; d[4 * c + 3] = dd.w;
        if constexpr (HAS_DA) {
          const float4 aa = *reinterpret_cast<const float4*>(dA + s0 + 4 * c);
          d[4 * c] += aa.x; d[4 * c + 1] += aa.y; d[4 * c + 2] += aa.z; d[4 * c + 3] += aa.w;
        }
      }
    } else {
      const float2 pp = *reinterpret_cast<const float2*>(Prow + s0);
      const float2 dd = *reinterpret_cast<const float2*>(Drow + s0);
      p[0] = pp.x; p[1] = pp.y; d[0] = dd.x; d[1] = dd.y;
      if constexpr (HAS_DA) {
        const float2 aa = *reinterpret_cast<const float2*>(dA + s0);
        d[0] += aa.x; d[1] += aa.y;
      }
    }
    float pbar = 0.f;
#pragma unroll
    for (int r = 0; r < R; ++r) pbar = fmaf(p[r], d[r], pbar);
#pragma unroll
    for (int r = 0; r < R; ++r) p[r] *= d[r] - pbar;   // p now holds g_r
#pragma unroll
    for (int k = 0; k < K; ++k) {
      float du = 0.f;
#pragma unroll
      for (int r = 0; r < R; ++r) du += ((r >> (K - 1 - k)) & 1) ? p[r] : -p[r];
      const int j = l * K + k;
      const float h = Hrow[j];
      ds = fmaf(du, h, ds);
      DJT[j * LY::TS + t] = du * inv_scale * (1.f - h * h);
    }
  }
}

// O[t][d] = sum_k AT[k][t] B[k][d] for t in {8w+2g, 8w+2g+1} (w counted from
// warp0), d in {4c..4c+3, 32+4c..32+4c+3} (D=64) or {4c..4c+3} (D=32), with
// c = lane & 7, g = lane >> 3.
template <class LY>
__device__ __forceinline__ void readout(const float* __restrict__ AT, const float* __restrict__ B,
                                        int K, int warp0, float (&o)[2][8], int& t_out,
                                        int& c_out) {
  constexpr int D = LY::Dv;
  const int lane = threadIdx.x & 31;
  const int w = (threadIdx.x >> 5) - warp0;
  const int c = lane & 7, g = lane >> 3;
  const int t = w * 8 + 2 * g;
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) o[i][j] = 0.f;
  for (int k = 0; k < K; ++k) {
    const float2 a = *reinterpret_cast<const float2*>(AT + k * LY::TS + t);
    const float4 b0 = *reinterpret_cast<const float4*>(B + k * LY::RS + 4 * c);
    o[0][0] = fmaf(a.x, b0.x, o[0][0]); o[1][0] = fmaf(a.y, b0.x, o[1][0]);
    o[0][1] = fmaf(a.x, b0.y, o[0][1]); o[1][1] = fmaf(a.y, b0.y, o[1][1]);
    o[0][2] = fmaf(a.x, b0.z, o[0][2]); o[1][2] = fmaf(a.y, b0.z, o[1][2]);
    o[0][3] = fmaf(a.x, b0.w, o[0][3]); o[1][3] = fmaf(a.y, b0.w, o[1][3]);
    if constexpr (D == 64) {
      const float4 b1 = *reinterpret_cast<const float4*>(B + k * LY::RS + 32 + 4 * c);
      o[0][4] = fmaf(a.x, b1.x, o[0][4]); o[1][4] = fmaf(a.y, b1.x, o[1][4]);
      o[0][5] = fmaf(a.x, b1.y, o[0][5]); o[1][5] = fmaf(a.y, b1.y, o[1][5]);
      o[0][6] = fmaf(a.x, b1.z, o[0][6]); o[1][6] = fmaf(a.y, b1.z, o[1][6]);
      o[0][7] = fmaf(a.x, b1.w, o[0][7]); o[1][7] = fmaf(a.y, b1.w, o[1][7]);
    }
  }
  t_out = t;
  c_out = c;
}

// Writes a readout tile row pair to global memory (T = float or bf16).
template <typename T, int D>
__device__ __forceinline__ void store_readout(T* base, int64_t st, int64_t tile0, int64_t t1,
                                              int t, int c, const float (&o)[2][8]) {
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int64_t tok = tile0 + t + i;
    if (tok < t1) {
      T* row = base + tok * st;
      const float a[4] = {o[i][0], o[i][1], o[i][2], o[i][3]};
      st_row<T, 4>(row + 4 * c, a);
      if constexpr (D == 64) {
        const float b[4] = {o[i][4], o[i][5], o[i][6], o[i][7]};
        st_row<T, 4>(row + 32 + 4 * c, b);
      }
    }
  }
}

// DP[t][s] = sum_d X[t][d] TAB[s][d] for t in {16w + p, 16w + p + 8}, s = sq + 4j.
// Uses 4 warps (warp0 .. warp0+3), 16 tokens each.
template <class LY>
__device__ __forceinline__ void rowdot(const float* __restrict__ X, const float* __restrict__ TAB,
                                       float* __restrict__ DP, int warp0) {
  constexpr int D = LY::Dv;
  constexpr int SQ = LY::SQ;
  const int lane = threadIdx.x & 31;
  const int w = (threadIdx.x >> 5) - warp0;
  const int p = lane >> 2, sq = lane & 3;
  const int t = w * 16 + p;
  float acc[2][SQ];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < SQ; ++j) acc[i][j] = 0.f;
#pragma unroll 4
  for (int d = 0; d < D; d += 4) {
    const float4 x0 = *reinterpret_cast<const float4*>(X + t * LY::RS + d);
    const float4 x1 = *reinterpret_cast<const float4*>(X + (t + 8) * LY::RS + d);
#pragma unroll
    for (int j = 0; j < SQ; ++j) {
      const float4 e = *reinterpret_cast<const float4*>(TAB + (sq + 4 * j) * LY::RS + d);
      acc[0][j] = fmaf(x0.x, e.x, fmaf(x0.y, e.y, fmaf(x0.z, e.z, fmaf(x0.w, e.w, acc[0][j]))));
      acc[1][j] = fmaf(x1.x, e.x, fmaf(x1.y, e.y, fmaf(x1.z, e.z, fmaf(x1.w, e.w, acc[1][j]))));
    }
  }
#pragma unroll
  for (int j = 0; j < SQ; ++j) {
    DP[t * LY::PS + sq + 4 * j] = acc[0][j];
    DP[(t + 8) * LY::PS + sq + 4 * j] = acc[1][j];
  }
}

// Bucket aggregation over one tile: a warp takes a token range, a lane owns
// columns {2*lane, 2*lane+1} (D=64) / {lane} (D=32) of every bucket row.
template <class LY>
struct Agg {
  static constexpr int D = LY::Dv, SPAD = LY::Sv;
  static constexpr int CPL = D / 32;   // columns per lane
  float a[SPAD][CPL];
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int s = 0; s < SPAD; ++s)
#pragma unroll
      for (int c = 0; c < CPL; ++c) a[s][c] = 0.f;
  }
  __device__ __forceinline__ void add_tile(const float* __restrict__ P, const float* __restrict__ Y,
                                           int tb, int te) {
    const int lane = threadIdx.x & 31;
    for (int t = tb; t < te; ++t) {
      float y[CPL];
      if constexpr (CPL == 2) {
        const float2 v = *reinterpret_cast<const float2*>(Y + t * LY::RS + 2 * lane);
        y[0] = v.x; y[1] = v.y;
      } else {
        y[0] = Y[t * LY::RS + lane];
      }
#pragma unroll
      for (int s = 0; s < SPAD; s += 4) {
        const float4 p = *reinterpret_cast<const float4*>(P + t * LY::PS + s);
        const float pp[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int c = 0; c < CPL; ++c) a[s + i][c] = fmaf(pp[i], y[c], a[s + i][c]);
      }
    }
  }
  // Fixed-order reduction of the warps [warp0, warp0+nw) into red[SPAD][D].
  __device__ __forceinline__ void reduce(float* red, int warp0, int nw) {
    const int lane = threadIdx.x & 31;
    const int w = threadIdx.x >> 5;
    for (int k = 0; k < nw; ++k) {
      if (w == warp0 + k) {
#pragma unroll
        for (int s = 0; s < SPAD; ++s)
#pragma unroll
          for (int c = 0; c < CPL; ++c) {
            float* dst = red + s * D + CPL * lane + c;
            *dst = (k == 0) ? a[s][c] : *dst + a[s][c];
          }
      }
      __syncthreads();
    }
  }
};

// ------------------------------------------------------------------ common setup
template <class LY>
__device__ __forceinline__ void load_planes(float* sm, const Params& prm, int n) {
  constexpr int D = LY::Dv;
  const int m = prm.Mp == 1 ? 0 : n / (prm.B * prm.H);
  const float* pl = prm.planes + (size_t)m * prm.LK * D;
  for (int i = threadIdx.x; i < LKP * D; i += NT) {
    const int j = i / D, d = i % D;
    sm[LY::PL + j * LY::RS + d] = j < prm.LK ? pl[j * D + d] : 0.f;
  }
}

// TAB[s][d] = slot[s][d] / (mass[s] + eps), zero rows beyond S.
template <class LY>
__device__ __forceinline__ void load_table(float* sm, const float* slot, const float* mass, int S,
                                           float eps) {
  constexpr int D = LY::Dv, SPAD = LY::Sv;
  for (int i = threadIdx.x; i < SPAD * D; i += NT) {
    const int s = i / D, d = i % D;
    float v = 0.f;
    if (s < S) v = slot[s * D + d] / (mass[s] + eps);
    sm[LY::TAB + s * LY::RS + d] = v;
  }
}

struct TileRange {
  int64_t t0, t1;
  int ntiles;
};
template <int TTL = TT>
__device__ __forceinline__ TileRange tile_range(int64_t T, int P, int part) {
  const int64_t tiles = (T + TTL - 1) / TTL;
  const int64_t a = tiles * part / P, b = tiles * (part + 1) / P;
  TileRange r;
  r.t0 = a * TTL;
  r.t1 = min(T, b * TTL);
  r.ntiles = (int)(b - a);
  return r;
}

// Pipelined walk over the tiles: tile i+1 is staged while tile i is
// computed.  Usage:
//   TilePipe<T, LY, TWO> pipe{...};  pipe.start();
//   for (i < ntiles) { pipe.acquire(i, X, Y, tile0); ...compute...; __syncthreads(); }
//   pipe.finish();
template <typename T, class LY, bool TWO, int NTH = NT, int TTL = TT>
struct TilePipe {
  static constexpr int D = LY::Dv;
  static constexpr bool BF = sizeof(T) == 2;
  float* sm;
  const T* xb;
  int64_t xst;
  const T* yb;
  int64_t yst;
  TileRange tr;
  __device__ __forceinline__ float* fx(int st) const { return sm + LY::XS + (BF ? 0 : st * TTL * LY::RS); }
  __device__ __forceinline__ float* fy(int st) const { return sm + LY::YS + (BF ? 0 : st * TTL * LY::RS); }
  __device__ __forceinline__ void* rx(int st) const { return sm + LY::RAW + (st * 2 + 0) * (TTL * D / 2); }
  __device__ __forceinline__ void* ry(int st) const { return sm + LY::RAW + (st * 2 + 1) * (TTL * D / 2); }
  __device__ __forceinline__ void start() const {
    if (tr.ntiles <= 0) return;
    stage_tile<T, D, NTH, TTL>(fx(0), rx(0), xb, xst, tr.t0, tr.t1);
    if (TWO) stage_tile<T, D, NTH, TTL>(fy(0), ry(0), yb, yst, tr.t0, tr.t1);
    cp_commit();
  }
  __device__ __forceinline__ void acquire(int i, float*& X, float*& Y, int64_t& tile0) const {
    const int st = i & 1;
    tile0 = tr.t0 + (int64_t)i * TTL;
    if (i + 1 < tr.ntiles) {
      stage_tile<T, D, NTH, TTL>(fx(st ^ 1), rx(st ^ 1), xb, xst, tile0 + TTL, tr.t1);
      if (TWO) stage_tile<T, D, NTH, TTL>(fy(st ^ 1), ry(st ^ 1), yb, yst, tile0 + TTL, tr.t1);
    }
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    if constexpr (BF) {
      convert_tile<D, NTH, TTL>(fx(0), rx(st));
      if (TWO) convert_tile<D, NTH, TTL>(fy(0), ry(st));
      __syncthreads();
    }
    X = fx(st);
    Y = fy(st);
  }
  __device__ __forceinline__ void finish() const { cp_wait<0>(); }
};

#define RACE_TILE_PROLOGUE                                                        \
  using LY = Lay<D, SPAD, sizeof(T) == 2>;                                        \
  extern __shared__ __align__(16) float sm[];                                     \
  const Shape sh(prm);                                                            \
  const float inv_scale = 1.f / __ldg(prm.scale);                                 \
  const int n = blockIdx.y, part = blockIdx.x;                                    \
  const TileRange tr = tile_range(prm.T, prm.P, part);                            \
  load_planes<LY>(sm, prm, n);                                                    \
  for (int i = threadIdx.x; i < SPAD * LY::TS; i += NT) sm[LY::PT + i] = 0.f;     \
  for (int i = threadIdx.x; i < TT * LY::PS; i += NT) {                           \
    sm[LY::P + i] = 0.f;                                                          \
    sm[LY::DP + i] = 0.f;                                                         \
  }

// F1: per-CTA partial [V|1] bucket sums of the key side.
template <typename T, int D, int SPAD, int K>
__global__ void __launch_bounds__(NT, 2) k_tile_reduce(const Params prm) {
  RACE_TILE_PROLOGUE
  const T* kb = static_cast<const T*>(prm.k) + stream_offset(prm.lk, n, prm.B, prm.H);
  const T* vb = static_cast<const T*>(prm.v) + stream_offset(prm.lv, n, prm.B, prm.H);
  __syncthreads();
  Agg<LY> agg;
  agg.zero();
  float amass = 0.f;   // thread (s = tid/8, part = tid%8): bucket mass partial
  const int w = threadIdx.x >> 5;
  TilePipe<T, LY, true> pipe{sm, kb, prm.lk.st, vb, prm.lv.st, tr};
  pipe.start();
  for (int it = 0; it < tr.ntiles; ++it) {
    float *X, *Y;
    int64_t tile0;
    pipe.acquire(it, X, Y, tile0);
    hash_tile<LY, K>(X, sm, sh, inv_scale, tr.t1 - tile0);
    __syncthreads();
    agg.add_tile(sm + LY::P, Y, w * 8, w * 8 + 8);
    if (threadIdx.x < SPAD * 8) {
      const int s = threadIdx.x >> 3, pp = threadIdx.x & 7;
      const float* row = sm + LY::PT + s * LY::TS + pp * 8;
      const float4 a = *reinterpret_cast<const float4*>(row);
      const float4 b = *reinterpret_cast<const float4*>(row + 4);
      amass += ((a.x + a.y) + (a.z + a.w)) + ((b.x + b.y) + (b.z + b.w));
    }
    __syncthreads();
  }
  pipe.finish();
  amass += __shfl_xor_sync(0xffffffffu, amass, 1);
  amass += __shfl_xor_sync(0xffffffffu, amass, 2);
  amass += __shfl_xor_sync(0xffffffffu, amass, 4);
  float* red = sm + LY::XS;   // tiles are free now: [SPAD][D] + [SPAD]
  __syncthreads();
  agg.reduce(red, 0, 8);
  if (threadIdx.x < SPAD * 8 && (threadIdx.x & 7) == 0) red[SPAD * D + (threadIdx.x >> 3)] = amass;
  __syncthreads();
  float* dst = prm.part + ((size_t)n * prm.P + part) * prm.SS;
  for (int e = threadIdx.x; e < prm.S * D; e += NT) dst[e] = red[e];
  for (int s = threadIdx.x; s < prm.S; s += NT) dst[prm.S * D + s] = red[SPAD * D + s];
}

// F2: out = sum_s pQ_s E_s.
template <typename T, int D, int SPAD, int K>
__global__ void __launch_bounds__(NT, 2) k_tile_readout(const Params prm) {
  RACE_TILE_PROLOGUE
  const float* st = prm.state + (size_t)n * prm.SS;
  load_table<LY>(sm, st, st + prm.S * D, prm.S, prm.eps);
  const T* qb = static_cast<const T*>(prm.q) + stream_offset(prm.lq, n, prm.B, prm.H);
  T* ob = static_cast<T*>(prm.out) + stream_offset(prm.lo, n, prm.B, prm.H);
  __syncthreads();
  TilePipe<T, LY, false> pipe{sm, qb, prm.lq.st, qb, prm.lq.st, tr};
  pipe.start();
  for (int it = 0; it < tr.ntiles; ++it) {
    float *X, *Y;
    int64_t tile0;
    pipe.acquire(it, X, Y, tile0);
    hash_tile<LY, K>(X, sm, sh, inv_scale, tr.t1 - tile0);
    __syncthreads();
    float o[2][8];
    int t, c;
    readout<LY>(sm + LY::PT, sm + LY::TAB, sh.S, 0, o, t, c);
    store_readout<T, D>(ob, prm.lo.st, tile0, tr.t1, t, c, o);
    __syncthreads();
  }
  pipe.finish();
}

// B1: dq and the per-CTA partial dE = sum_t pQ dO^T (warps 4-7), dp = dO E^T
// (warps 0-3), then the hash backward and dq = dproj . planes.
template <typename T, int D, int SPAD, int K>
__global__ void __launch_bounds__(NT, 2) k_tile_bwd_q(const Params prm) {
  RACE_TILE_PROLOGUE
  const float* st = prm.state + (size_t)n * prm.SS;
  load_table<LY>(sm, st, st + prm.S * D, prm.S, prm.eps);
  const T* qb = static_cast<const T*>(prm.q) + stream_offset(prm.lq, n, prm.B, prm.H);
  const T* gb = static_cast<const T*>(prm.dout) + stream_offset(prm.ldo, n, prm.B, prm.H);
  T* dqb = static_cast<T*>(prm.dq) + stream_offset(prm.ldq, n, prm.B, prm.H);
  __syncthreads();
  Agg<LY> agg;
  agg.zero();
  float ds = 0.f;
  const int w = threadIdx.x >> 5;
  TilePipe<T, LY, true> pipe{sm, qb, prm.lq.st, gb, prm.ldo.st, tr};
  pipe.start();
  for (int it = 0; it < tr.ntiles; ++it) {
    float *X, *Y;
    int64_t tile0;
    pipe.acquire(it, X, Y, tile0);
    hash_tile<LY, K>(X, sm, sh, inv_scale, tr.t1 - tile0);
    __syncthreads();
    if (w < 4) rowdot<LY>(Y, sm + LY::TAB, sm + LY::DP, 0);
    else agg.add_tile(sm + LY::P, Y, (w - 4) * 16, (w - 4) * 16 + 16);
    __syncthreads();
    hash_backward<LY, K, false>(sm, sh, inv_scale, nullptr, ds);
    __syncthreads();
    float o[2][8];
    int t, c;
    readout<LY>(sm + LY::DJT, sm + LY::PL, sh.LK, 0, o, t, c);
    store_readout<T, D>(dqb, prm.ldq.st, tile0, tr.t1, t, c, o);
    __syncthreads();
  }
  pipe.finish();
  float* red = sm + LY::XS;
  __syncthreads();
  agg.reduce(red, 4, 4);
  float* dst = prm.part + ((size_t)n * prm.P + part) * prm.SS;
  for (int e = threadIdx.x; e < prm.S * D; e += NT) dst[e] = red[e];
  const float tot = cta_sum(ds, sm + LY::MISC);
  if (threadIdx.x == 0) prm.dscale_part[(size_t)n * prm.P + part] = tot;
}

// B2: dv = pK . dB (warps 4-7), dpK = v . dB^T + dA (warps 0-3), then dk.
template <typename T, int D, int SPAD, int K>
__global__ void __launch_bounds__(NT, 2) k_tile_bwd_kv(const Params prm) {
  RACE_TILE_PROLOGUE
  const float* st = prm.state + (size_t)n * prm.SS;
  const float* gs = prm.gstate_in + (size_t)n * prm.SS;
  // TAB = dB = dE / (A + eps); dA_s = -sum_d dB_sd E_sd
  load_table<LY>(sm, gs, st + prm.S * D, prm.S, prm.eps);
  float* dA = sm + LY::MISC;
  __syncthreads();
  {
    const int lane = threadIdx.x & 31;
    for (int s = threadIdx.x >> 5; s < SPAD; s += 8) {
      float a = 0.f;
      if (s < prm.S) {
        const float inv = 1.f / (st[prm.S * D + s] + prm.eps);
        for (int d = lane; d < D; d += 32)
          a = fmaf(sm[LY::TAB + s * LY::RS + d], st[s * D + d] * inv, a);
      }
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
      if (lane == 0) dA[s] = -a;
    }
  }
  const T* kb = static_cast<const T*>(prm.k) + stream_offset(prm.lk, n, prm.B, prm.H);
  const T* vb = static_cast<const T*>(prm.v) + stream_offset(prm.lv, n, prm.B, prm.H);
  T* dkb = static_cast<T*>(prm.dk) + stream_offset(prm.ldk, n, prm.B, prm.H);
  T* dvb = static_cast<T*>(prm.dv) + stream_offset(prm.ldv, n, prm.B, prm.H);
  __syncthreads();
  float ds = 0.f;
  const int w = threadIdx.x >> 5;
  TilePipe<T, LY, true> pipe{sm, kb, prm.lk.st, vb, prm.lv.st, tr};
  pipe.start();
  for (int it = 0; it < tr.ntiles; ++it) {
    float *X, *Y;
    int64_t tile0;
    pipe.acquire(it, X, Y, tile0);
    hash_tile<LY, K>(X, sm, sh, inv_scale, tr.t1 - tile0);
    __syncthreads();
    if (w < 4) {
      rowdot<LY>(Y, sm + LY::TAB, sm + LY::DP, 0);
    } else {
      // dv for the 64 tokens: 4 warps x 2 passes of 32 tokens
      for (int pass = 0; pass < 2; ++pass) {
        float o[2][8];
        int t, c;
        readout<LY>(sm + LY::PT + pass * 32, sm + LY::TAB, sh.S, 4, o, t, c);
        store_readout<T, D>(dvb, prm.ldv.st, tile0 + pass * 32, tr.t1, t, c, o);
      }
    }
    __syncthreads();
    hash_backward<LY, K, true>(sm, sh, inv_scale, dA, ds);
    __syncthreads();
    float o[2][8];
    int t, c;
    readout<LY>(sm + LY::DJT, sm + LY::PL, sh.LK, 0, o, t, c);
    store_readout<T, D>(dkb, prm.ldk.st, tile0, tr.t1, t, c, o);
    __syncthreads();
  }
  pipe.finish();
  const float tot = cta_sum(ds, sm + LY::MISC + 32);
  if (threadIdx.x == 0) prm.dscale_part[(size_t)n * prm.P + part] = tot;
}

}  // namespace tiles
}  // namespace race
