// race_causal_tc.cuh -- causal (per-bucket prefix mean) RACE kernels on the
// tensor cores.
//
// Every stream's tokens are split into P contiguous ranges, one CTA each
// (256 threads, 32-token tiles, rows staged by cp.async).  The range totals
// come from the non-causal reduce kernel; a float64 scan over ranges gives
// each CTA the exclusive prefix (B0 = sum pK v^T, A0 = sum pK) of its range.
// Within a tile of tokens t, tau (A(t) inclusive, W_s(t) = pQ_s(t)/(A_s(t)+eps)):
//
//   forward   out(t)   = W(t) . B0 + sum_{tau<=t} G(t,tau) v(tau),  G = W pK^T
//   backward  dpQ(t)   = invA(t) (dO(t) . B0 + sum_{tau<=t} M(t,tau) pK(tau)),
//             M = dO V^T;  alpha = -W dpQ (stored per token)
//   reverse   dpK(t)   = asuf(t) + v(t) . beta + sum_{tau>=t} M(tau,t) W(tau)
//             dv(t)    = pK(t) . beta + sum_{tau>=t} G(tau,t) dO(tau)
// with beta / asuf the suffix sums of W dO / alpha over later tokens
// (kernels/cpu/race_pref.cpp:104-220 restated with W folded in).  All the
// products are 3xTF32 warp MMAs (race_mma.cuh); the masks are applied when
// the 32 x 32 intra-tile matrices are written back to shared memory.  The
// key mass is carried in float64 and recorded per tile by the forward walk of
// the backward pass, so the reverse walk never rebuilds it by subtraction.
#pragma once

#include "race_mma.cuh"

namespace race {
namespace ctc {

using tc::NT;
using tc::NW;
using tc::TT;
using tiles::LKP;
using namespace tc;

template <int D, int SPAD, bool BF, int NIN>
struct CLay {
  static constexpr int NSTAGE = BF ? 1 : 2;
  static constexpr int S8 = round_up(SPAD, 8);
  static constexpr int SM16 = round_up(S8, 16);
  static constexpr int RS = D + 4;
  static constexpr int P2S = S8 <= 16 ? 20 : 36;   // float2 rows, = 4 (mod 16)
  static constexpr int PT2S = TT + 4;              // 36
  static constexpr int MS = TT + 4;                // 32 x 32 split matrices
  static constexpr int DJ2S = LKP + 4;
  static constexpr int PS = odd4(S8 + 4);
  static constexpr int JS = LKP + 4;
  static constexpr int B2S = D + 4;
  static constexpr int ACS = S8 + 1;               // fp32 [t][s] scratch rows
  static constexpr int IN = 0;                     // [NIN][NSTAGE][TT][RS]
  static constexpr int PLB = IN + NIN * NSTAGE * TT * RS;   // float2 [LKP][B2S]
  static constexpr int STB = PLB + 2 * LKP * B2S;  // float2 [S8][B2S] state table (split)
  static constexpr int STF = STB + 2 * S8 * B2S;   // fp32 [S8][D] state (master)
  static constexpr int H = STF + S8 * D;           // [TT][LKP+1] tanh (gradient side)
  static constexpr int P2 = H + TT * (LKP + 1) + ((TT * (LKP + 1)) & 1);  // float2 [TT][P2S] probs (gradient side)
  static constexpr int K2 = P2 + 2 * TT * P2S;     // float2 [TT][P2S] key probs
  static constexpr int KT2 = K2 + 2 * TT * P2S;    // float2 [SM16][PT2S] key probs^T
  static constexpr int W2 = KT2 + 2 * SM16 * PT2S; // float2 [TT][P2S] W
  static constexpr int WT2 = W2 + 2 * TT * P2S;    // float2 [SM16][PT2S] W^T
  static constexpr int MM2 = WT2 + 2 * SM16 * PT2S;  // float2 [TT][MS] masked 32x32
  static constexpr int Q2 = MM2 + 2 * TT * MS;     // float2 [TT][P2S] query probs (reverse walk)
  static constexpr int DJ2 = Q2 + 2 * TT * P2S;    // float2 [TT][DJ2S]
  static constexpr int ACUM = DJ2 + 2 * TT * DJ2S; // fp32 [TT][ACS] inclusive key mass
  static constexpr int AUX = ACUM + TT * ACS;      // fp32 [TT][ACS] (pQ / alpha suffix)
  static constexpr int DP = AUX + TT * ACS;        // fp32 [TT][PS]; PROJ aliases it
  static constexpr int PROJ = DP;
  static constexpr int A0 = DP + (PS > JS ? TT * PS : TT * JS) + 1;  // double [32]
  static constexpr int VEC = A0 + ((A0 & 1) ? 1 : 0) + 64;           // fp32 [32] per-bucket values
  static constexpr int MISC = VEC + 32;            // 32 floats
  static constexpr int RAW = round_up(MISC + 32, 4);
  static constexpr int RAW_FLOATS = BF ? NIN * 2 * TT * D / 2 : 0;
  static constexpr int FLOATS = RAW + RAW_FLOATS;
  static constexpr int A0D = A0 + ((A0 & 1) ? 1 : 0);  // double-aligned start
  static constexpr int Dv = D;
  static constexpr int Sv = SPAD;
  static_assert(S8 <= 32, "bucket count above 32");
  static_assert(PLB % 2 == 0 && STB % 2 == 0 && P2 % 2 == 0 && K2 % 2 == 0 && MM2 % 2 == 0 &&
                    Q2 % 2 == 0 && DJ2 % 2 == 0, "float2 alignment");
};

// ------------------------------------------------------------------ staging
// NIN input tensors, tiles walked forward or backward through the range.
template <typename T, class LY, int NIN, bool REV>
struct MultiPipe {
  static constexpr int D = LY::Dv;
  static constexpr bool BF = sizeof(T) == 2;
  float* sm;
  const T* base[4];
  int64_t st[4];
  tiles::TileRange tr;
  __device__ __forceinline__ float* buf(int w, int s) const {
    return sm + LY::IN + (w * LY::NSTAGE + (BF ? 0 : s)) * TT * LY::RS;
  }
  __device__ __forceinline__ void* raw(int w, int s) const {
    return sm + LY::RAW + (s * NIN + w) * (TT * D / 2);
  }
  __device__ __forceinline__ int64_t tile_start(int i) const {
    const int k = REV ? tr.ntiles - 1 - i : i;
    return tr.t0 + (int64_t)k * TT;
  }
  __device__ __forceinline__ void stage(int i, int s) const {
    const int64_t t0 = tile_start(i);
#pragma unroll
    for (int w = 0; w < NIN; ++w)
      tiles::stage_tile<T, D, NT, TT>(buf(w, s), raw(w, s), base[w], st[w], t0, tr.t1);
  }
  __device__ __forceinline__ void start() const {
    if (tr.ntiles <= 0) return;
    stage(0, 0);
    tiles::cp_commit();
  }
  // returns the tile's first token; buffers via in(w)
  __device__ __forceinline__ int64_t acquire(int i) const {
    const int s = i & 1;
    if (i + 1 < tr.ntiles) stage(i + 1, s ^ 1);
    tiles::cp_commit();
    tiles::cp_wait<1>();
    __syncthreads();
    if constexpr (BF) {
#pragma unroll
      for (int w = 0; w < NIN; ++w) tiles::convert_tile<D, NT, TT>(buf(w, 0), raw(w, s));
      __syncthreads();
    }
    return tile_start(i);
  }
  __device__ __forceinline__ const float* in(int w, int i) const { return buf(w, i & 1); }
  __device__ __forceinline__ void finish() const { tiles::cp_wait<0>(); }
};

// ------------------------------------------------------------------ per-tile pieces
// Corner probabilities of a projected tile: p[t][s] (split) into P2 (and its
// transpose into PT2 when given), tanh into Hrow when given.
template <class LY, int K>
__device__ __forceinline__ void probs_to(float* sm, const Shape& sh, float inv_scale,
                                         int64_t valid_rows, float2* P2, float2* PT2, float* Hm) {
  constexpr int R = 1 << K;
  const int t = threadIdx.x >> 3, e = threadIdx.x & 7;
  const float pv = t < valid_rows ? 1.f : 0.f;
  const float* proj = sm + LY::PROJ + t * LY::JS;
  for (int l = e; l < sh.L; l += 8) {
    float sp[K], sn[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const float h = tiles::tanh_exp(proj[l * K + k]);
      if (Hm) Hm[t * (LKP + 1) + l * K + k] = h;
      const float u = h * inv_scale;
      const float ex = __expf(-2.f * fabsf(u));
      const float r = __frcp_rn(1.f + ex);
      sp[k] = u >= 0.f ? r : ex * r;
      sn[k] = u >= 0.f ? ex * r : r;
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float p = pv;
#pragma unroll
      for (int k = 0; k < K; ++k) p *= ((r >> (K - 1 - k)) & 1) ? sp[k] : sn[k];
      const int s = l * R + r;
      const float2 p2 = split2(p);
      P2[t * LY::P2S + s] = p2;
      if (PT2) PT2[s * LY::PT2S + t] = p2;
    }
  }
}

// ACUM[t][s] = A0_s + sum_{tau<=t} pK_s(tau) and A0 += the tile's key mass
// (A0 in float64, the in-tile sum of <= 32 terms in float32).  Warp w scans
// buckets s = w, w+8, ... with lane = token.  Kp holds pK split [t][s].
template <class LY>
__device__ __forceinline__ void key_mass(float* sm, const float2* Kp, int S) {
  const int lane = threadIdx.x & 31;
  double* A0 = reinterpret_cast<double*>(sm + LY::A0D);
  for (int s = threadIdx.x >> 5; s < S; s += NW) {
    const float2 p = Kp[lane * LY::P2S + s];
    float v = p.x + p.y;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float u = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += u;
    }
    const double a0 = A0[s];
    sm[LY::ACUM + lane * LY::ACS + s] = (float)(a0 + (double)v);
    __syncwarp();
    if (lane == 31) A0[s] = a0 + (double)v;
  }
}

// In place: X[t][s] = base_s + sum_{tau >= t} X[tau][s] for s < S (lane = t),
// and base_s += sum over the tile.  Returns nothing; base lives in smem.
template <class LY>
__device__ __forceinline__ void suffix_scan(float* X, float* base, int S) {
  const int lane = threadIdx.x & 31;
  for (int s = threadIdx.x >> 5; s < S; s += NW) {
    float v = X[lane * LY::ACS + s];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float u = __shfl_down_sync(0xffffffffu, v, o);
      if (lane + o < 32) v += u;
    }
    const float b = base[s];
    X[lane * LY::ACS + s] = b + v;
    __syncwarp();
    if (lane == 0) base[s] = b + v;
  }
}

// sum over the tile's tokens of X[t][s], added into acc (thread s < S holds acc).
template <class LY>
__device__ __forceinline__ void column_sums(const float* X, float* out, int S) {
  const int lane = threadIdx.x & 31;
  for (int s = threadIdx.x >> 5; s < S; s += NW) {
    float v = X[lane * LY::ACS + s];
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) out[s] += v;
  }
}

// W of the tile (split, [t][s] into W2 and, when given, [s][t] into WT2) from
// the query probabilities PQ and the inclusive key mass ACUM.  Per-bucket
// normalisation: W_s(t) = pQ_s(t) / (A_s(t) + eps).  Global normalisation
// (misc/elsaa_causal_complete.py:551-560, misc/race_kernel.py:9-124): one
// denominator per token, den(t) = sum_s pQ_s(t) A_s(t), and
// W_s(t) = pQ_s(t) / max(den(t), eps).  Thread (t = tid / 8, e = tid % 8)
// handles buckets e, e + 8, ...; returns den(t) (0 in per-bucket mode).
template <class LY>
__device__ __forceinline__ float weights(float* sm, const Params& prm, int S, const float2* PQ,
                                         float2* W2, float2* WT2) {
  const int t = threadIdx.x >> 3, e = threadIdx.x & 7;
  const float* acum = sm + LY::ACUM + t * LY::ACS;
  float den = 0.f;
  if (prm.global_norm) {
    for (int s = e; s < S; s += 8) {
      const float2 p = PQ[t * LY::P2S + s];
      den = fmaf(p.x + p.y, acum[s], den);
    }
    den += __shfl_xor_sync(0xffffffffu, den, 1);
    den += __shfl_xor_sync(0xffffffffu, den, 2);
    den += __shfl_xor_sync(0xffffffffu, den, 4);
  }
  const float dd = fmaxf(den, prm.eps);
  for (int s = e; s < S; s += 8) {
    const float2 p = PQ[t * LY::P2S + s];
    const float w = prm.global_norm ? (p.x + p.y) / dd : (p.x + p.y) / (acum[s] + prm.eps);
    const float2 w2 = split2(w);
    W2[t * LY::P2S + s] = w2;
    if (WT2) WT2[s * LY::PT2S + t] = w2;
  }
  return den;
}

// 32 x 32 products C = A . B (M = N = 32) written back split, keeping
// (col <= row) for LOWER or (col >= row) for UPPER.  Warp w: C tile
// (rows 16(w&1), cols 8(w>>1)).
template <class LY, bool LOWER, int KSTEPS, class VA, class VB>
__device__ __forceinline__ void masked_32x32(float* sm, const VA& A, const VB& B) {
  const int w = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int m0 = 16 * (w & 1), n0 = 8 * (w >> 1);
  float c[1][4];
  zero(c);
  wgemm<1, KSTEPS>(c, A, m0, B, n0);
  float2* M2 = reinterpret_cast<float2*>(sm + LY::MM2);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int row = m0 + g + 8 * h;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int col = n0 + 2 * q + j;
      const bool keep = LOWER ? (col <= row) : (col >= row);
      M2[row * LY::MS + col] = split2(keep ? c[0][2 * h + j] : 0.f);
    }
  }
}

// Rebuilds the split state table STB from the fp32 master STF.
template <class LY>
__device__ __forceinline__ void refresh_state_table(float* sm) {
  constexpr int D = LY::Dv;
  float2* stb = reinterpret_cast<float2*>(sm + LY::STB);
  for (int i = threadIdx.x; i < LY::S8 * D; i += NT) {
    const int s = i / D, d = i % D;
    stb[s * LY::B2S + d] = split2(sm[LY::STF + i]);
  }
}

// STF[s][d] += sum_t A^T[s][t] Y[t][d] (A^T given split [SM16][PT2S]),
// for buckets s < S8; warp w owns (S8/16 rounded) x (D/8) tiles like AggTC.
template <class LY, bool EX = false>
__device__ __forceinline__ void state_add(float* sm, const float2* AT, const float* Y) {
  constexpr int D = LY::Dv;
  constexpr int NTILES = D / 8;
  constexpr int TILES = (LY::SM16 / 16) * NTILES;
  constexpr int PER = (TILES + NW - 1) / NW;
  const int first = (threadIdx.x >> 5) * PER;
  if (first >= TILES) return;
  const int m0 = 16 * (first / NTILES), n0 = 8 * (first % NTILES);
  float c[PER][4];
  zero(c);
  wgemm<PER, TT / 8>(c, ASplit<LY::PT2S>{AT}, m0, BView<LY::RS, 1, EX>{Y}, n0);
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
#pragma unroll
  for (int i = 0; i < PER; ++i)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int s = m0 + g + 8 * h;
      if (s < LY::S8) {
        float* p = sm + LY::STF + s * D + n0 + 8 * i + 2 * q;
        p[0] += c[i][2 * h];
        p[1] += c[i][2 * h + 1];
      }
    }
}

template <class LY>
__device__ __forceinline__ void load_state(float* sm, const float* slot, int S, bool with_mass) {
  constexpr int D = LY::Dv;
  for (int i = threadIdx.x; i < LY::S8 * D; i += NT) {
    const int s = i / D;
    sm[LY::STF + i] = s < S ? slot[i] : 0.f;
  }
  if (with_mass && threadIdx.x < 32) {
    double* A0 = reinterpret_cast<double*>(sm + LY::A0D);
    A0[threadIdx.x] = threadIdx.x < S ? (double)slot[S * D + threadIdx.x] : 0.0;
  }
}

template <class LY>
__device__ __forceinline__ void clear_all(float* sm) {
  // padding buckets / columns are read as zeros by the 8-wide k steps
  for (int i = threadIdx.x; i < LY::ACUM - LY::H; i += NT) sm[LY::H + i] = 0.f;
  for (int i = threadIdx.x; i < TT * LY::ACS; i += NT) sm[LY::AUX + i] = 0.f;
}

#define RACE_CTC_PROLOGUE(NIN)                                                    \
  using LY = CLay<D, SPAD, sizeof(T) == 2, NIN>;                                  \
  extern __shared__ __align__(16) float sm[];                                     \
  const Shape sh(prm);                                                            \
  const float inv_scale = 1.f / __ldg(prm.scale);                                 \
  const int n = blockIdx.y, part = blockIdx.x;                                    \
  const tiles::TileRange tr = tiles::tile_range<TT>(prm.T, prm.P, part);          \
  clear_all<LY>(sm);                                                              \
  tc::load_planes<LY>(sm, prm, n);

template <class T>
__device__ __forceinline__ const T* row0(const void* p, const Layout& l, const Params& prm, int n) {
  return static_cast<const T*>(p) + stream_offset(l, n, prm.B, prm.H);
}

// ------------------------------------------------------------------ forward
template <typename T, int D, int SPAD, int K>
__global__ void __launch_bounds__(NT, 1) k_ctc_fwd(const Params prm) {
  RACE_CTC_PROLOGUE(3)
  const size_t slot = (size_t)n * prm.P + part;
  load_state<LY>(sm, prm.state + slot * prm.SS, prm.S, true);
  T* ob = static_cast<T*>(prm.out) + stream_offset(prm.lo, n, prm.B, prm.H);
  MultiPipe<T, LY, 3, false> pipe{sm,
                                   {row0<T>(prm.q, prm.lq, prm, n), row0<T>(prm.k, prm.lk, prm, n),
                                    row0<T>(prm.v, prm.lv, prm, n), nullptr},
                                   {prm.lq.st, prm.lk.st, prm.lv.st, 0},
                                   tr};
  __syncthreads();
  refresh_state_table<LY>(sm);
  pipe.start();
  float2* K2 = reinterpret_cast<float2*>(sm + LY::K2);
  float2* KT2 = reinterpret_cast<float2*>(sm + LY::KT2);
  float2* W2 = reinterpret_cast<float2*>(sm + LY::W2);
  for (int it = 0; it < tr.ntiles; ++it) {
    const int64_t tile0 = pipe.acquire(it);
    const float* Q = pipe.in(0, it);
    const float* Kx = pipe.in(1, it);
    const float* V = pipe.in(2, it);
    const int64_t valid = tr.t1 - tile0;
    projections<LY, sizeof(T) == 2>(Kx, sm);
    __syncthreads();
    probs_to<LY, K>(sm, sh, inv_scale, valid, K2, KT2, nullptr);
    __syncthreads();
    key_mass<LY>(sm, K2, prm.S);
    projections<LY, sizeof(T) == 2>(Q, sm);
    __syncthreads();
    probs_to<LY, K>(sm, sh, inv_scale, valid, reinterpret_cast<float2*>(sm + LY::P2), nullptr,
                    nullptr);
    __syncthreads();
    {
      const float den =
          weights<LY>(sm, prm, sh.S, reinterpret_cast<const float2*>(sm + LY::P2), W2, nullptr);
      const int64_t tok = tile0 + (threadIdx.x >> 3);
      if (prm.den_out && (threadIdx.x & 7) == 0 && tok < tr.t1)
        prm.den_out[(size_t)n * prm.T + tok] = den;
    }
    __syncthreads();
    // G = W pK^T, lower-triangular
    masked_32x32<LY, true, LY::S8 / 8>(sm, ASplit<LY::P2S>{W2}, BSplit<1, LY::P2S>{K2});
    __syncthreads();
    {   // out = W . B0 + G . V
      const int w = threadIdx.x >> 5;
      const int m0 = 16 * (w & 1), n0 = (D / 4) * (w >> 1);
      float c[D / 32][4];
      zero(c);
      wgemm<D / 32, LY::S8 / 8>(c, ASplit<LY::P2S>{W2}, m0,
                                BSplit<LY::B2S, 1>{reinterpret_cast<const float2*>(sm + LY::STB)}, n0);
      wgemm<D / 32, TT / 8>(c, ASplit<LY::MS>{reinterpret_cast<const float2*>(sm + LY::MM2)}, m0,
                            BView<LY::RS, 1, sizeof(T) == 2>{V}, n0);
      store_c_global<T, D / 32>(c, ob, prm.lo.st, tile0, tr.t1, m0, n0);
    }
    __syncthreads();
    state_add<LY, sizeof(T) == 2>(sm, KT2, V);   // B0 += pK^T V
    __syncthreads();
    refresh_state_table<LY>(sm);
    __syncthreads();
  }
  pipe.finish();
}

// ------------------------------------------------------------------ backward, forward walk
// dq, alpha (per token, global scratch), per-tile key mass A0 (global
// scratch), and the range totals of W dO (gradient slot) and alpha.
template <typename T, int D, int SPAD, int K>
__global__ void __launch_bounds__(NT, 1) k_ctc_bwd_q(const Params prm) {
  RACE_CTC_PROLOGUE(4)
  const size_t slot = (size_t)n * prm.P + part;
  load_state<LY>(sm, prm.state + slot * prm.SS, prm.S, true);
  T* dqb = static_cast<T*>(prm.dq) + stream_offset(prm.ldq, n, prm.B, prm.H);
  MultiPipe<T, LY, 4, false> pipe{sm,
                                   {row0<T>(prm.q, prm.lq, prm, n), row0<T>(prm.k, prm.lk, prm, n),
                                    row0<T>(prm.v, prm.lv, prm, n),
                                    row0<T>(prm.dout, prm.ldo, prm, n)},
                                   {prm.lq.st, prm.lk.st, prm.lv.st, prm.ldo.st},
                                   tr};
  __syncthreads();
  refresh_state_table<LY>(sm);
  pipe.start();
  float2* K2 = reinterpret_cast<float2*>(sm + LY::K2);
  float2* KT2 = reinterpret_cast<float2*>(sm + LY::KT2);
  float2* W2 = reinterpret_cast<float2*>(sm + LY::W2);
  float2* WT2 = reinterpret_cast<float2*>(sm + LY::WT2);
  float* alpha = prm.alpha + (size_t)n * prm.T * prm.S;
  double* tileA = prm.tilemass;
  const int64_t ntile_stream = (prm.T + TT - 1) / TT;
  // range totals of W dO: per-warp C tiles kept across the walk
  constexpr int NTILES = D / 8;
  constexpr int TILES = (LY::SM16 / 16) * NTILES;
  constexpr int PER = (TILES + NW - 1) / NW;
  float gb[PER][4];
  zero(gb);
  const int gfirst = (threadIdx.x >> 5) * PER;
  const bool glive = gfirst < TILES;
  const int gm0 = 16 * (glive ? gfirst / NTILES : 0), gn0 = 8 * (glive ? gfirst % NTILES : 0);
  if (threadIdx.x < 32) sm[LY::VEC + threadIdx.x] = 0.f;   // range total of alpha_s
  float ds = 0.f;
  for (int it = 0; it < tr.ntiles; ++it) {
    const int64_t tile0 = pipe.acquire(it);
    const float* Q = pipe.in(0, it);
    const float* Kx = pipe.in(1, it);
    const float* V = pipe.in(2, it);
    const float* G = pipe.in(3, it);
    const int64_t valid = tr.t1 - tile0;
    // record A0 at the tile start for the reverse walk
    if (threadIdx.x < prm.S)
      tileA[((size_t)n * ntile_stream + tile0 / TT) * LY::S8 + threadIdx.x] =
          reinterpret_cast<const double*>(sm + LY::A0D)[threadIdx.x];
    projections<LY, sizeof(T) == 2>(Kx, sm);
    __syncthreads();
    probs_to<LY, K>(sm, sh, inv_scale, valid, K2, KT2, nullptr);
    __syncthreads();
    key_mass<LY>(sm, K2, prm.S);
    projections<LY, sizeof(T) == 2>(Q, sm);
    __syncthreads();
    probs_to<LY, K>(sm, sh, inv_scale, valid, reinterpret_cast<float2*>(sm + LY::P2), nullptr,
                    sm + LY::H);
    // M = dO V^T, lower-triangular (other warps' reads of PROJ are done: the
    // product only touches MM2)
    masked_32x32<LY, true, D / 8>(sm, AView<LY::RS, 1, sizeof(T) == 2>{G}, BView<1, LY::RS, sizeof(T) == 2>{V});
    __syncthreads();
    // W and its transpose; den(t) stays in this thread's register
    const float den =
        weights<LY>(sm, prm, sh.S, reinterpret_cast<const float2*>(sm + LY::P2), W2, WT2);
    {   // R = dO . B0^T + M . pK  -> DP (warp w: rows 16(w&1), bucket n-tile w>>1)
      const int w = threadIdx.x >> 5;
      const int nt = w >> 1;
      if (nt < LY::S8 / 8) {
        float c[1][4];
        zero(c);
        wgemm<1, D / 8>(c, AView<LY::RS, 1, sizeof(T) == 2>{G}, 16 * (w & 1),
                        BSplit<1, LY::B2S>{reinterpret_cast<const float2*>(sm + LY::STB)}, 8 * nt);
        wgemm<1, TT / 8>(c, ASplit<LY::MS>{reinterpret_cast<const float2*>(sm + LY::MM2)},
                         16 * (w & 1), BSplit<LY::P2S, 1>{K2}, 8 * nt);
        store_c_smem<1>(c, sm + LY::DP, LY::PS, 16 * (w & 1), 8 * nt);
      }
    }
    __syncthreads();
    if (prm.global_norm) {
      // out = num / dd, dd = max(den, eps), num = sum_s pQ_s B_s, den = sum_s pQ_s A_s:
      //   gden  = -(dO . out) / dd (0 where the clamp holds) + incoming d(den)
      //   dpQ_s = R_s / dd + A_s gden,  alpha_s = pQ_s gden  (d of A_s(t))
      // with dO . out = sum_s W_s R_s.
      const int t = threadIdx.x >> 3, e = threadIdx.x & 7;
      const int64_t tok = tile0 + t;
      const float2* P2 = reinterpret_cast<const float2*>(sm + LY::P2);
      float wr = 0.f;
      for (int s = e; s < sh.S; s += 8) {
        const float2 w = W2[t * LY::P2S + s];
        wr = fmaf(w.x + w.y, sm[LY::DP + t * LY::PS + s], wr);
      }
      wr += __shfl_xor_sync(0xffffffffu, wr, 1);
      wr += __shfl_xor_sync(0xffffffffu, wr, 2);
      wr += __shfl_xor_sync(0xffffffffu, wr, 4);
      const float dd = fmaxf(den, prm.eps);
      float gden = den >= prm.eps ? -wr / dd : 0.f;
      if (prm.dden_in && tok < tr.t1) gden += prm.dden_in[(size_t)n * prm.T + tok];
      for (int s = e; s < sh.S; s += 8) {
        const float dpq = sm[LY::DP + t * LY::PS + s] / dd + sm[LY::ACUM + t * LY::ACS + s] * gden;
        sm[LY::DP + t * LY::PS + s] = dpq;
        const float2 p = P2[t * LY::P2S + s];
        const float al = (p.x + p.y) * gden;
        sm[LY::AUX + t * LY::ACS + s] = al;
        if (tok < tr.t1) alpha[tok * prm.S + s] = al;
      }
    } else {   // dpQ = invA R, alpha = -W dpQ
      const int t = threadIdx.x >> 3, e = threadIdx.x & 7;
      const int64_t tok = tile0 + t;
      for (int s = e; s < sh.S; s += 8) {
        const float inv = 1.f / (sm[LY::ACUM + t * LY::ACS + s] + prm.eps);
        const float dpq = sm[LY::DP + t * LY::PS + s] * inv;
        sm[LY::DP + t * LY::PS + s] = dpq;
        const float2 w = W2[t * LY::P2S + s];
        const float al = -(w.x + w.y) * dpq;
        sm[LY::AUX + t * LY::ACS + s] = al;
        if (tok < tr.t1) alpha[tok * prm.S + s] = al;
      }
    }
    __syncthreads();
    column_sums<LY>(sm + LY::AUX, sm + LY::VEC, prm.S);   // range total of alpha
    hash_backward<LY, K, false>(sm, sh, inv_scale, nullptr, ds);
    if (glive)   // range total of W^T dO
      wgemm<PER, TT / 8>(gb, ASplit<LY::PT2S>{WT2}, gm0, BView<LY::RS, 1, sizeof(T) == 2>{G}, gn0);
    __syncthreads();
    {
      float c[D / 32][4];
      int m0, n0;
      readout_tc<LY, true>(sm, c, m0, n0);
      store_c_global<T, D / 32>(c, dqb, prm.ldq.st, tile0, tr.t1, m0, n0);
    }
    state_add<LY, sizeof(T) == 2>(sm, KT2, V);
    __syncthreads();
    refresh_state_table<LY>(sm);
    __syncthreads();
  }
  pipe.finish();
  // gradient slot: [S][D] sum W dO, then [S] sum alpha
  float* dst = prm.gstate_out + slot * prm.SS;
  if (glive) {
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2, q = lane & 3;
#pragma unroll
    for (int i = 0; i < PER; ++i)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int s = gm0 + g + 8 * h;
        if (s < prm.S) {
          dst[s * D + gn0 + 8 * i + 2 * q] = gb[i][2 * h];
          dst[s * D + gn0 + 8 * i + 2 * q + 1] = gb[i][2 * h + 1];
        }
      }
  }
  __syncthreads();
  if (threadIdx.x < prm.S) dst[prm.S * D + threadIdx.x] = sm[LY::VEC + threadIdx.x];
  const float tot = cta_sum_nw(ds, sm + LY::MISC);
  if (threadIdx.x == 0) prm.dscale_part[slot] = tot;
}

// ------------------------------------------------------------------ backward, reverse walk
template <typename T, int D, int SPAD, int K>
__global__ void __launch_bounds__(NT, 1) k_ctc_bwd_kv(const Params prm) {
  RACE_CTC_PROLOGUE(4)
  const size_t slot = (size_t)n * prm.P + part;
  // beta (exclusive suffix of W dO over later ranges) into the state table
  load_state<LY>(sm, prm.gstate_in + slot * prm.SS, prm.S, false);
  float* asuf = sm + LY::VEC;   // asuf_s at the end of the current tile
  if (threadIdx.x < 32)
    asuf[threadIdx.x] = threadIdx.x < prm.S ? prm.gstate_in[slot * prm.SS + prm.S * D + threadIdx.x] : 0.f;
  T* dkb = static_cast<T*>(prm.dk) + stream_offset(prm.ldk, n, prm.B, prm.H);
  T* dvb = static_cast<T*>(prm.dv) + stream_offset(prm.ldv, n, prm.B, prm.H);
  MultiPipe<T, LY, 4, true> pipe{sm,
                                  {row0<T>(prm.q, prm.lq, prm, n), row0<T>(prm.k, prm.lk, prm, n),
                                   row0<T>(prm.v, prm.lv, prm, n),
                                   row0<T>(prm.dout, prm.ldo, prm, n)},
                                  {prm.lq.st, prm.lk.st, prm.lv.st, prm.ldo.st},
                                  tr};
  __syncthreads();
  refresh_state_table<LY>(sm);
  pipe.start();
  float2* W2 = reinterpret_cast<float2*>(sm + LY::W2);
  float2* WT2 = reinterpret_cast<float2*>(sm + LY::WT2);
  float2* P2 = reinterpret_cast<float2*>(sm + LY::P2);   // key probabilities (gradient side)
  const float* alpha = prm.alpha + (size_t)n * prm.T * prm.S;
  const double* tileA = prm.tilemass;
  const int64_t ntile_stream = (prm.T + TT - 1) / TT;
  float ds = 0.f;
  for (int it = 0; it < tr.ntiles; ++it) {
    const int64_t tile0 = pipe.acquire(it);
    const float* Q = pipe.in(0, it);
    const float* Kx = pipe.in(1, it);
    const float* V = pipe.in(2, it);
    const float* G = pipe.in(3, it);
    const int64_t valid = tr.t1 - tile0;
    if (threadIdx.x < 32)
      reinterpret_cast<double*>(sm + LY::A0D)[threadIdx.x] =
          threadIdx.x < prm.S
              ? tileA[((size_t)n * ntile_stream + tile0 / TT) * LY::S8 + threadIdx.x]
              : 0.0;
    projections<LY, sizeof(T) == 2>(Kx, sm);
    __syncthreads();
    // key probabilities into P2 (gradient side) and K2 (for key_mass); tanh into H
    probs_to<LY, K>(sm, sh, inv_scale, valid, P2, nullptr, sm + LY::H);
    __syncthreads();
    key_mass<LY>(sm, P2, prm.S);
    projections<LY, sizeof(T) == 2>(Q, sm);
    __syncthreads();
    probs_to<LY, K>(sm, sh, inv_scale, valid, reinterpret_cast<float2*>(sm + LY::Q2), nullptr,
                    nullptr);
    __syncthreads();
    {   // W, W^T; asuf(t) = asuf_end + sum_{tau >= t in tile} alpha(tau) (AUX)
      weights<LY>(sm, prm, sh.S, reinterpret_cast<const float2*>(sm + LY::Q2), W2, WT2);
      // alpha of the tile (contiguous [t][s]) into AUX
      for (int i = threadIdx.x; i < TT * prm.S; i += NT) {
        const int t = i / prm.S, ss = i - t * prm.S;
        sm[LY::AUX + t * LY::ACS + ss] = tile0 + t < tr.t1 ? alpha[tile0 * prm.S + i] : 0.f;
      }
    }
    __syncthreads();
    suffix_scan<LY>(sm + LY::AUX, asuf, prm.S);   // asuf(t), and asuf -> the previous tile's end
    __syncthreads();
    // Mt(t, tau) = v_t . dO_tau, kept for tau >= t
    masked_32x32<LY, false, D / 8>(sm, AView<LY::RS, 1, sizeof(T) == 2>{V}, BView<1, LY::RS, sizeof(T) == 2>{G});
    __syncthreads();
    {   // dpK = asuf + V . beta^T + Mt . W  -> DP
      const int w = threadIdx.x >> 5;
      const int nt = w >> 1;
      if (nt < LY::S8 / 8) {
        float c[1][4];
        zero(c);
        wgemm<1, D / 8>(c, AView<LY::RS, 1, sizeof(T) == 2>{V}, 16 * (w & 1),
                        BSplit<1, LY::B2S>{reinterpret_cast<const float2*>(sm + LY::STB)}, 8 * nt);
        wgemm<1, TT / 8>(c, ASplit<LY::MS>{reinterpret_cast<const float2*>(sm + LY::MM2)},
                         16 * (w & 1), BSplit<LY::P2S, 1>{W2}, 8 * nt);
        const int lane = threadIdx.x & 31;
        const int g = lane >> 2, q = lane & 3;
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int t = 16 * (w & 1) + g + 8 * h, s = 8 * nt + 2 * q + j;
            sm[LY::DP + t * LY::PS + s] = c[0][2 * h + j] + sm[LY::AUX + t * LY::ACS + s];
          }
      }
    }
    __syncthreads();
    // Gt(t, tau) = pK_t . W_tau, kept for tau >= t (overwrites MM2)
    masked_32x32<LY, false, LY::S8 / 8>(sm, ASplit<LY::P2S>{P2}, BSplit<1, LY::P2S>{W2});
    hash_backward<LY, K, false>(sm, sh, inv_scale, nullptr, ds);
    __syncthreads();
    {   // dk
      float c[D / 32][4];
      int m0, n0;
      readout_tc<LY, true>(sm, c, m0, n0);
      store_c_global<T, D / 32>(c, dkb, prm.ldk.st, tile0, tr.t1, m0, n0);
    }
    {   // dv = pK . beta + Gt . dO
      const int w = threadIdx.x >> 5;
      const int m0 = 16 * (w & 1), n0 = (D / 4) * (w >> 1);
      float c[D / 32][4];
      zero(c);
      wgemm<D / 32, LY::S8 / 8>(c, ASplit<LY::P2S>{P2}, m0,
                                BSplit<LY::B2S, 1>{reinterpret_cast<const float2*>(sm + LY::STB)}, n0);
      wgemm<D / 32, TT / 8>(c, ASplit<LY::MS>{reinterpret_cast<const float2*>(sm + LY::MM2)}, m0,
                            BView<LY::RS, 1, sizeof(T) == 2>{G}, n0);
      store_c_global<T, D / 32>(c, dvb, prm.ldv.st, tile0, tr.t1, m0, n0);
    }
    __syncthreads();
    // carry the suffix states to the previous tile: beta += W^T dO, asuf = AUX[0]
    state_add<LY, sizeof(T) == 2>(sm, WT2, G);
    __syncthreads();
    refresh_state_table<LY>(sm);
    __syncthreads();
  }
  pipe.finish();
  const float tot = cta_sum_nw(ds, sm + LY::MISC);
  if (threadIdx.x == 0) prm.dscale_part[slot] = tot;
}

}  // namespace ctc
}  // namespace race
