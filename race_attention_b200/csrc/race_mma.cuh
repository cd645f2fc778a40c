// race_mma.cuh -- non-causal RACE kernels with tensor-core tile contractions.
//
// A CTA of 256 threads (8 warps; two CTAs per SM) walks a contiguous range of
// 32-token tiles of one stream; cp.async double-buffers the next tile's rows
// (race_tiles.cuh TilePipe).  Every dense contraction of a tile runs on the tensor cores as
// warp-level mma.sync.m16n8k8 TF32 products in "3xTF32" form: each fp32
// operand x is split into a TF32 high part and the TF32 truncation of x - hi,
// and lo*hi + hi*lo + hi*hi is accumulated in fp32 (relative error ~2^-19 per
// product, so the float32 parity bar holds; bf16 inputs have lo = 0 exactly).
// Measured on this B200, mma.sync TF32 runs at ~277 TFLOP/s against
// ~70 TFLOP/s for FP32 FMA.
//
// Contractions per 32-token tile (S8 = S rounded up to 8):
//   projection  PROJ[64][16]  = X[64][d]   . PL^T          (K = d)
//   readout     O[64][d]      = P[64][S8]  . TAB[S8][d]    (out = pQ E, dv = pK dB)
//   rowdot      DP[64][S8]    = Y[64][d]   . TAB^T         (dp = dO E^T, v dB^T)
//   backproj    DX[64][d]     = DJ[64][16] . PL            (dq, dk)
//   aggregate   ACC[S8][d]   += P^T[S8][64] . Y[64][d]     (bucket sums, dE)
// The planes and the per-stream table (E or dB) are constant over the CTA's
// tiles, so they are split into {hi, lo} TF32 pairs once and stored as
// float2 rows of stride d+4 pairs: that one layout serves the B fragment
// reads of both the table and its transpose without bank conflicts.  The
// probabilities (P, PT) and the projection gradients (DJ) are written
// pre-split by the CUDA-core stages that produce them; only the staged input
// rows (X, Y) are split as their fragments are read.
// The soft hash's nonlinear part (tanh, sigmoids, corner products) and its
// backward run per (token, table) on CUDA cores.
#pragma once

#include "race_tiles.cuh"

namespace race {
namespace tc {

using tiles::LKP;
constexpr int TT = 32;   // tokens per tile
constexpr int NT = 256;  // threads per CTA (two CTAs share an SM)
constexpr int NW = NT / 32;

__host__ __device__ constexpr int odd4(int n) { return ((n / 4) % 2 == 1) ? n : n + 4; }

// Kernel kinds and the shared-memory buffers each one touches.
enum Kind { kReduce = 0, kReadout = 1, kBwdQ = 2, kBwdKV = 3 };

template <int D, int SPAD, bool BF = false, int KIND = kBwdQ>
struct Lay {
  static constexpr bool kTwo = KIND != kReadout;        // X and Y staged
  static constexpr bool kP = KIND != kReduce;           // P2  (readout / hash backward)
  static constexpr bool kPT = KIND == kReduce || KIND == kBwdQ;   // PT2 (aggregation)
  static constexpr bool kTab = KIND != kReduce;         // E / dB table
  static constexpr bool kBwd = KIND >= kBwdQ;           // H, DJ2
  static constexpr int NSTAGE = BF ? 1 : 2;
  static constexpr int S8 = round_up(SPAD, 8);          // bucket extent as a k / n dim
  static constexpr int SM16 = round_up(S8, 16);         // bucket extent as an m dim
  static constexpr int RS = D + 4;                      // X / Y rows     (A: t x d)
  // float2 {hi, lo} arrays; row strides = 4 (mod 16) pairs keep the 64-bit
  // fragment reads of a half-warp on distinct banks
  static constexpr int P2S = S8 <= 16 ? 20 : 36;        // P2 rows        (A: t x s)
  static constexpr int PT2S = TT + 4;                   // PT2 rows       (A: s x t)
  static constexpr int DJ2S = LKP + 4;                  // DJ2 rows       (A: t x j)
  static constexpr int PS = odd4(S8 + 4);               // DP rows (fp32)
  static constexpr int JS = LKP + 4;                    // PROJ rows (fp32)
  static constexpr int B2S = D + 4;                     // split table / plane rows (float2)
  static constexpr int XS = 0;
  static constexpr int YS = XS + NSTAGE * TT * RS;
  static constexpr int PLB = YS + (kTwo ? NSTAGE * TT * RS : 0);   // float2 [LKP][B2S]
  static constexpr int TABB = PLB + 2 * LKP * B2S;      // float2 [S8][B2S]
  static constexpr int H = TABB + (kTab ? 2 * S8 * B2S : 0);        // [TT][LKP+1]
  static constexpr int HN = kBwd ? TT * (LKP + 1) + ((TT * (LKP + 1)) & 1) : 0;
  static constexpr int P2 = H + HN;                     // float2 [TT][P2S]
  static constexpr int PT2 = P2 + (kP ? 2 * TT * P2S : 0);          // float2 [SM16][PT2S]
  static constexpr int DJ2 = PT2 + (kPT ? 2 * SM16 * PT2S : 0);     // float2 [TT][DJ2S]
  static constexpr int DP = DJ2 + (kBwd ? 2 * TT * DJ2S : 0);       // [TT][PS]; PROJ aliases it
  static constexpr int PROJ = DP;                       // [TT][JS]
  static constexpr int MISC = DP + (kBwd && PS > JS ? TT * PS : TT * JS);  // 64 floats
  static constexpr int RAW = MISC + 64;
  // TilePipe addresses raw bf16 rows as [stage][X, Y]: keep both slots
  static constexpr int RAW_FLOATS = BF ? 2 * 2 * TT * D / 2 : 0;
  static constexpr int FLOATS = RAW + RAW_FLOATS;
  static constexpr int Dv = D;
  static constexpr int Sv = SPAD;
  static_assert(S8 <= 32, "bucket count above 32");
  static_assert(RAW % 4 == 0 && YS % 4 == 0, "alignment");
  static_assert(PLB % 2 == 0 && TABB % 2 == 0 && P2 % 2 == 0 && PT2 % 2 == 0 && DJ2 % 2 == 0,
                "float2 alignment");
};

// ------------------------------------------------------------------ MMA
// x = hi + lo with hi = x truncated to TF32 (19 high bits, exact) and lo the
// TF32 truncation of the exact remainder x - hi: |x - hi - lo| < 2^-20 |x|.
// With the lo*lo product dropped, each 3xTF32 product is within ~2^-19 of
// the fp32 one.  Three integer/float ops instead of two conversions.
__device__ __forceinline__ void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
  hi = __float_as_uint(x) & 0xffffe000u;
  lo = __float_as_uint(x - __uint_as_float(hi)) & 0xffffe000u;
}

__device__ __forceinline__ void mma_tf32(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// A operand: fp32 matrix in shared memory, element (r, c) at p[r*RS + c*CS].
// EXACT: every value is a bf16 widened to fp32 (exact in TF32, lo = 0).
template <int RS, int CS, bool EXACT = false>
struct AView {
  const float* p;
  static constexpr bool kExact = EXACT;
};
// A operand from a pre-split float2 {hi, lo} matrix, (r, c) at p2[r*RS + c].
template <int RS>
struct ASplit {
  const float2* p2;
  static constexpr bool kExact = false;
};
// B operand from an fp32 matrix (split on the fly), (k, n) at p[k*KS + n*NS].
template <int KS, int NS, bool EXACT = false>
struct BView {
  const float* p;
  static constexpr bool kExact = EXACT;
};
// B operand from a pre-split float2 {hi, lo} matrix, (k, n) at p2[k*KS + n*NS].
template <int KS, int NS>
struct BSplit {
  const float2* p2;
  static constexpr bool kExact = false;
};

template <int RS, int CS, bool EX>
__device__ __forceinline__ void load_a(const AView<RS, CS, EX>& A, int m0, int k0, uint32_t (&ah)[4],
                                       uint32_t (&al)[4]) {
  const int lane = threadIdx.x & 31;
  const float* b = A.p + (m0 + (lane >> 2)) * RS + (k0 + (lane & 3)) * CS;
  if constexpr (EX) {
    ah[0] = __float_as_uint(b[0]);
    ah[1] = __float_as_uint(b[8 * RS]);
    ah[2] = __float_as_uint(b[4 * CS]);
    ah[3] = __float_as_uint(b[8 * RS + 4 * CS]);
  } else {
    split_tf32(b[0], ah[0], al[0]);
    split_tf32(b[8 * RS], ah[1], al[1]);
    split_tf32(b[4 * CS], ah[2], al[2]);
    split_tf32(b[8 * RS + 4 * CS], ah[3], al[3]);
  }
}

template <int RS>
__device__ __forceinline__ void load_a(const ASplit<RS>& A, int m0, int k0, uint32_t (&ah)[4],
                                       uint32_t (&al)[4]) {
  const int lane = threadIdx.x & 31;
  const float2* b = A.p2 + (m0 + (lane >> 2)) * RS + k0 + (lane & 3);
  const float2 x0 = b[0], x1 = b[8 * RS], x2 = b[4], x3 = b[8 * RS + 4];
  ah[0] = __float_as_uint(x0.x); al[0] = __float_as_uint(x0.y);
  ah[1] = __float_as_uint(x1.x); al[1] = __float_as_uint(x1.y);
  ah[2] = __float_as_uint(x2.x); al[2] = __float_as_uint(x2.y);
  ah[3] = __float_as_uint(x3.x); al[3] = __float_as_uint(x3.y);
}

__device__ __forceinline__ float2 split2(float x) {
  uint32_t h, l;
  split_tf32(x, h, l);
  return make_float2(__uint_as_float(h), __uint_as_float(l));
}

template <int KS, int NS, bool EX>
__device__ __forceinline__ void load_b(const BView<KS, NS, EX>& B, int k0, int n, uint32_t& h0,
                                       uint32_t& l0, uint32_t& h1, uint32_t& l1) {
  const int lane = threadIdx.x & 31;
  const float* b = B.p + (k0 + (lane & 3)) * KS + (n + (lane >> 2)) * NS;
  if constexpr (EX) {
    h0 = __float_as_uint(b[0]);
    h1 = __float_as_uint(b[4 * KS]);
  } else {
    split_tf32(b[0], h0, l0);
    split_tf32(b[4 * KS], h1, l1);
  }
}

template <int KS, int NS>
__device__ __forceinline__ void load_b(const BSplit<KS, NS>& B, int k0, int n, uint32_t& h0,
                                       uint32_t& l0, uint32_t& h1, uint32_t& l1) {
  const int lane = threadIdx.x & 31;
  const float2* b = B.p2 + (k0 + (lane & 3)) * KS + (n + (lane >> 2)) * NS;
  const float2 x0 = b[0], x1 = b[4 * KS];
  h0 = __float_as_uint(x0.x); l0 = __float_as_uint(x0.y);
  h1 = __float_as_uint(x1.x); l1 = __float_as_uint(x1.y);
}

// C[i] (16 x 8, i < ntl) += A[m0.., 0..8*KSTEPS) . B[0..8*KSTEPS, n0 + 8i ..].
// Fragments (lane = 4g + q): A (g,q) (g+8,q) (g,q+4) (g+8,q+4); B (k=q,n=g)
// (k=q+4,n=g); C (g,2q) (g,2q+1) (g+8,2q) (g+8,2q+1).
template <int NTL, int KSTEPS, class VA, class VB>
__device__ __forceinline__ void wgemm(float (&c)[NTL][4], const VA& A, int m0, const VB& B, int n0,
                                      int ntl = NTL) {
#pragma unroll
  for (int ks = 0; ks < KSTEPS; ++ks) {
    uint32_t ah[4], al[4];
    load_a(A, m0, ks * 8, ah, al);
#pragma unroll
    for (int i = 0; i < NTL; ++i) {
      if (i < ntl) {
        uint32_t h0, l0, h1, l1;
        load_b(B, ks * 8, n0 + 8 * i, h0, l0, h1, l1);
        if constexpr (!VA::kExact) mma_tf32(c[i], al, h0, h1);
        if constexpr (!VB::kExact) mma_tf32(c[i], ah, l0, l1);
        mma_tf32(c[i], ah, h0, h1);
      }
    }
  }
}

template <int NTL>
__device__ __forceinline__ void zero(float (&c)[NTL][4]) {
#pragma unroll
  for (int i = 0; i < NTL; ++i) c[i][0] = c[i][1] = c[i][2] = c[i][3] = 0.f;
}

template <int NTL>
__device__ __forceinline__ void store_c_smem(const float (&c)[NTL][4], float* dst, int ld, int m0,
                                             int n0, int ntl = NTL) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
#pragma unroll
  for (int i = 0; i < NTL; ++i) {
    if (i < ntl) {
      float* r0 = dst + (m0 + g) * ld + n0 + 8 * i + 2 * q;
      float* r1 = r0 + 8 * ld;
      r0[0] = c[i][0]; r0[1] = c[i][1];
      r1[0] = c[i][2]; r1[1] = c[i][3];
    }
  }
}

template <typename T, int NTL>
__device__ __forceinline__ void store_c_global(const float (&c)[NTL][4], T* base, int64_t st,
                                               int64_t tile0, int64_t t1, int m0, int n0) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int64_t tok = tile0 + m0 + g + 8 * h;
    if (tok < t1) {
      T* row = base + tok * st + n0 + 2 * q;
#pragma unroll
      for (int i = 0; i < NTL; ++i) {
        if constexpr (sizeof(T) == 4) {
          *reinterpret_cast<float2*>(row + 8 * i) = make_float2(c[i][2 * h], c[i][2 * h + 1]);
        } else {
          *reinterpret_cast<__nv_bfloat162*>(row + 8 * i) =
              __floats2bfloat162_rn(c[i][2 * h], c[i][2 * h + 1]);
        }
      }
    }
  }
}

// ------------------------------------------------------------------ tile ops
// PROJ = X . PL^T: warps 0..3 compute token rows 16(w&1).. and planes 8(w>>1)..
template <class LY, bool EX = false>
__device__ __forceinline__ void projections(const float* X, float* sm) {
  constexpr int D = LY::Dv;
  const int w = threadIdx.x >> 5;
  if (w < 4) {
    float c[1][4];
    zero(c);
    const float2* plb = reinterpret_cast<const float2*>(sm + LY::PLB);
    wgemm<1, D / 8>(c, AView<LY::RS, 1, EX>{X}, 16 * (w & 1), BSplit<1, LY::B2S>{plb}, 8 * (w >> 1));
    store_c_smem<1>(c, sm + LY::PROJ, LY::JS, 16 * (w & 1), 8 * (w >> 1));
  }
}

// Thread (token t = tid / 8, slot e = tid % 8) owns tables l = e, e+8:
// tanh of the projections (kept in H), sigmoids and corner probabilities.
template <class LY, int K>
__device__ __forceinline__ void probabilities(float* sm, const Shape& sh, float inv_scale,
                                              int64_t valid_rows) {
  constexpr int R = 1 << K;
  const int t = threadIdx.x >> 3, e = threadIdx.x & 7;
  const float pv = t < valid_rows ? 1.f : 0.f;
  const float* proj = sm + LY::PROJ + t * LY::JS;
  float* Hrow = sm + LY::H + t * (LKP + 1);
  float2* Prow = reinterpret_cast<float2*>(sm + LY::P2) + t * LY::P2S;
  float2* PT = reinterpret_cast<float2*>(sm + LY::PT2);
  for (int l = e; l < sh.L; l += 8) {
    float sp[K], sn[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const float h = tiles::tanh_exp(proj[l * K + k]);
      if constexpr (LY::kBwd) Hrow[l * K + k] = h;
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
      if constexpr (LY::kP) Prow[s] = p2;
      if constexpr (LY::kPT) PT[s * LY::PT2S + t] = p2;
    }
  }
}

// Hash backward per (token, table): DJ[t][j] = dL/dproj_j, ds += sum du h.
template <class LY, int K, bool HAS_DA>
__device__ __forceinline__ void hash_backward(float* sm, const Shape& sh, float inv_scale,
                                              const float* dA, float& ds) {
  constexpr int R = 1 << K;
  const int t = threadIdx.x >> 3, e = threadIdx.x & 7;
  const float* Hrow = sm + LY::H + t * (LKP + 1);
  const float2* Prow = reinterpret_cast<const float2*>(sm + LY::P2) + t * LY::P2S;
  const float* Drow = sm + LY::DP + t * LY::PS;
  float2* DJrow = reinterpret_cast<float2*>(sm + LY::DJ2) + t * LY::DJ2S;
  for (int l = e; l < sh.L; l += 8) {
    const int s0 = l * R;
    float p[R], d[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float2 pp = Prow[s0 + r];
      p[r] = pp.x + pp.y;
      d[r] = Drow[s0 + r];
      if constexpr (HAS_DA) d[r] += dA[s0 + r];
    }
    float pbar = 0.f;
#pragma unroll
    for (int r = 0; r < R; ++r) pbar = fmaf(p[r], d[r], pbar);
#pragma unroll
    for (int r = 0; r < R; ++r) p[r] *= d[r] - pbar;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      float du = 0.f;
#pragma unroll
      for (int r = 0; r < R; ++r) du += ((r >> (K - 1 - k)) & 1) ? p[r] : -p[r];
      const int j = l * K + k;
      const float h = Hrow[j];
      ds = fmaf(du, h, ds);
      DJrow[j] = split2(du * inv_scale * (1.f - h * h));
    }
  }
}

// O[32][d] = P . TAB (buckets) or DJ . PL (planes): warp w -> token rows
// 16(w&1).., columns (D/4)(w>>1) .. +D/4.
template <class LY, bool PLANES>
__device__ __forceinline__ void readout_tc(const float* sm, float (&c)[LY::Dv / 32][4], int& m0,
                                           int& n0) {
  constexpr int D = LY::Dv;
  constexpr int NTL = D / 32;
  const int w = threadIdx.x >> 5;
  m0 = 16 * (w & 1);
  n0 = (D / 4) * (w >> 1);
  zero(c);
  if constexpr (PLANES) {
    const float2* b = reinterpret_cast<const float2*>(sm + LY::PLB);
    const float2* a = reinterpret_cast<const float2*>(sm + LY::DJ2);
    wgemm<NTL, LKP / 8>(c, ASplit<LY::DJ2S>{a}, m0, BSplit<LY::B2S, 1>{b}, n0);
  } else {
    const float2* b = reinterpret_cast<const float2*>(sm + LY::TABB);
    const float2* a = reinterpret_cast<const float2*>(sm + LY::P2);
    wgemm<NTL, LY::S8 / 8>(c, ASplit<LY::P2S>{a}, m0, BSplit<LY::B2S, 1>{b}, n0);
  }
}

// DP[32][S8] = Y . TAB^T: warp w -> rows 16(w&1), bucket n-tile w>>1.
template <class LY, bool EX = false>
__device__ __forceinline__ void rowdot_tc(const float* Y, float* sm) {
  constexpr int D = LY::Dv;
  const int w = threadIdx.x >> 5;
  const int nt = w >> 1;
  if (nt < LY::S8 / 8) {
    float c[1][4];
    zero(c);
    const float2* b = reinterpret_cast<const float2*>(sm + LY::TABB);
    wgemm<1, D / 8>(c, AView<LY::RS, 1, EX>{Y}, 16 * (w & 1), BSplit<1, LY::B2S>{b}, 8 * nt);
    store_c_smem<1>(c, sm + LY::DP, LY::PS, 16 * (w & 1), 8 * nt);
  }
}

// ACC[SM16][d] += PT . Y: warp w owns PER consecutive C tiles (same bucket
// row block) of the (SM16/16) x (d/8) grid for the whole kernel, so no
// cross-warp reduction is needed.
template <class LY>
struct AggTC {
  static constexpr int D = LY::Dv;
  static constexpr int NTILES = D / 8;
  static constexpr int TILES = (LY::SM16 / 16) * NTILES;   // <= 16
  static constexpr int PER = (TILES + NW - 1) / NW;
  float c[PER][4];
  int m0, n0;
  bool live;
  __device__ __forceinline__ void init() {
    zero(c);
    const int first = (threadIdx.x >> 5) * PER;
    live = first < TILES;
    m0 = 16 * (first / NTILES);
    n0 = 8 * (first % NTILES);
  }
  template <bool EX = false>
  __device__ __forceinline__ void add_tile(const float* sm, const float* Y) {
    if (live)
      wgemm<PER, TT / 8>(c, ASplit<LY::PT2S>{reinterpret_cast<const float2*>(sm + LY::PT2)}, m0,
                         BView<LY::RS, 1, EX>{Y}, n0);
  }
  __device__ __forceinline__ void write(float* dst, int S) const {
    if (!live) return;
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2, q = lane & 3;
#pragma unroll
    for (int i = 0; i < PER; ++i)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int s = m0 + g + 8 * h;
        if (s < S) {
          dst[s * D + n0 + 8 * i + 2 * q] = c[i][2 * h];
          dst[s * D + n0 + 8 * i + 2 * q + 1] = c[i][2 * h + 1];
        }
      }
  }
};

// ------------------------------------------------------------------ setup
template <class LY>
__device__ __forceinline__ void load_planes(float* sm, const Params& prm, int n) {
  constexpr int D = LY::Dv;
  const int m = prm.Mp == 1 ? 0 : n / (prm.B * prm.H);
  const float* pl = prm.planes + (size_t)m * prm.LK * D;
  float2* plb = reinterpret_cast<float2*>(sm + LY::PLB);
  for (int i = threadIdx.x; i < LKP * D; i += NT) {
    const int j = i / D, d = i % D;
    uint32_t h, l;
    split_tf32(j < prm.LK ? pl[j * D + d] : 0.f, h, l);
    plb[j * LY::B2S + d] = make_float2(__uint_as_float(h), __uint_as_float(l));
  }
}

// TAB[s][d] = slot[s][d] / (mass[s] + eps) (zero for s >= S), pre-split.
template <class LY>
__device__ __forceinline__ void load_table(float* sm, const float* slot, const float* mass, int S,
                                           float eps) {
  constexpr int D = LY::Dv;
  float2* tb = reinterpret_cast<float2*>(sm + LY::TABB);
  for (int i = threadIdx.x; i < LY::S8 * D; i += NT) {
    const int s = i / D, d = i % D;
    uint32_t h, l;
    split_tf32(s < S ? slot[s * D + d] / (mass[s] + eps) : 0.f, h, l);
    tb[s * LY::B2S + d] = make_float2(__uint_as_float(h), __uint_as_float(l));
  }
}

template <class LY>
__device__ __forceinline__ void clear_buckets(float* sm) {
  // bucket padding (s >= S) of P2 / PT2 and DJ2 columns >= L*K are read as
  // zeros by the 8-wide k steps; DP padding is never read
  if constexpr (LY::kPT)
    for (int i = threadIdx.x; i < 2 * LY::SM16 * LY::PT2S; i += NT) sm[LY::PT2 + i] = 0.f;
  if constexpr (LY::kP)
    for (int i = threadIdx.x; i < 2 * TT * LY::P2S; i += NT) sm[LY::P2 + i] = 0.f;
  if constexpr (LY::kBwd) {
    for (int i = threadIdx.x; i < 2 * TT * LY::DJ2S; i += NT) sm[LY::DJ2 + i] = 0.f;
    for (int i = threadIdx.x; i < TT * LY::PS; i += NT) sm[LY::DP + i] = 0.f;
  }
}

__device__ __forceinline__ float cta_sum_nw(float x, float* red) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = x;
  __syncthreads();
  float t = 0.f;
  if (threadIdx.x == 0)
    for (int i = 0; i < NW; ++i) t += red[i];
  return t;
}

#define RACE_TC_PROLOGUE(KIND)                                                    \
  using LY = Lay<D, SPAD, sizeof(T) == 2, KIND>;                                  \
  extern __shared__ __align__(16) float sm[];                                     \
  const Shape sh(prm);                                                            \
  const float inv_scale = 1.f / __ldg(prm.scale);                                 \
  const int n = blockIdx.y, part = blockIdx.x;                                    \
  const tiles::TileRange tr = tiles::tile_range<TT>(prm.T, prm.P, part);              \
  load_planes<LY>(sm, prm, n);                                                    \
  clear_buckets<LY>(sm);

#define RACE_TC_LOOP(TWO, XB, XST, YB, YST)                                       \
  tiles::TilePipe<T, LY, TWO, NT, TT> pipe{sm, XB, XST, YB, YST, tr};                 \
  pipe.start();                                                                   \
  for (int it = 0; it < tr.ntiles; ++it) {                                        \
    float *X, *Y;                                                                 \
    int64_t tile0;                                                                \
    pipe.acquire(it, X, Y, tile0);

#define RACE_TC_LOOP_END                                                          \
    __syncthreads();                                                              \
  }                                                                               \
  pipe.finish();

// F1: per-CTA partial [V|1] bucket sums of the key side.
template <typename T, int D, int SPAD, int K>
__global__ void __launch_bounds__(NT, 3) k_tc_reduce(const Params prm) {
  RACE_TC_PROLOGUE(kReduce)
  const T* kb = static_cast<const T*>(prm.k) + stream_offset(prm.lk, n, prm.B, prm.H);
  const T* vb = static_cast<const T*>(prm.v) + stream_offset(prm.lv, n, prm.B, prm.H);
  __syncthreads();
  AggTC<LY> agg;
  agg.init();
  float amass = 0.f;   // thread (s = tid/4, quarter pp = tid%4) of the first SPAD*4
  RACE_TC_LOOP(true, kb, prm.lk.st, vb, prm.lv.st)
    projections<LY, sizeof(T) == 2>(X, sm);
    __syncthreads();
    probabilities<LY, K>(sm, sh, inv_scale, tr.t1 - tile0);
    __syncthreads();
    agg.template add_tile<sizeof(T) == 2>(sm, Y);
    if (threadIdx.x < SPAD * 4) {
      const int s = threadIdx.x >> 2, pp = threadIdx.x & 3;
      const float2* row = reinterpret_cast<const float2*>(sm + LY::PT2) + s * LY::PT2S + pp * 8;
      float a = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) a += row[i].x + row[i].y;
      amass += a;
    }
  RACE_TC_LOOP_END
  amass += __shfl_xor_sync(0xffffffffu, amass, 1);
  amass += __shfl_xor_sync(0xffffffffu, amass, 2);
  float* dst = prm.part + ((size_t)n * prm.P + part) * prm.SS;
  agg.write(dst, prm.S);
  if (threadIdx.x < SPAD * 4 && (threadIdx.x & 3) == 0 && (threadIdx.x >> 2) < prm.S)
    dst[prm.S * D + (threadIdx.x >> 2)] = amass;
}

// F2: out = sum_s pQ_s E_s.
template <typename T, int D, int SPAD, int K>
__global__ void __launch_bounds__(NT, 3) k_tc_readout(const Params prm) {
  RACE_TC_PROLOGUE(kReadout)
  const float* st = prm.state + (size_t)n * prm.SS;
  load_table<LY>(sm, st, st + prm.S * D, prm.S, prm.eps);
  const T* qb = static_cast<const T*>(prm.q) + stream_offset(prm.lq, n, prm.B, prm.H);
  T* ob = static_cast<T*>(prm.out) + stream_offset(prm.lo, n, prm.B, prm.H);
  __syncthreads();
  RACE_TC_LOOP(false, qb, prm.lq.st, qb, prm.lq.st)
    (void)Y;
    projections<LY, sizeof(T) == 2>(X, sm);
    __syncthreads();
    probabilities<LY, K>(sm, sh, inv_scale, tr.t1 - tile0);
    __syncthreads();
    float c[D / 32][4];
    int m0, n0;
    readout_tc<LY, false>(sm, c, m0, n0);
    store_c_global<T, D / 32>(c, ob, prm.lo.st, tile0, tr.t1, m0, n0);
  RACE_TC_LOOP_END
}

// B1: dq, the per-CTA partial dE = sum_t pQ dO^T and the q-side dscale.
template <typename T, int D, int SPAD, int K>
__global__ void __launch_bounds__(NT, 2) k_tc_bwd_q(const Params prm) {
  RACE_TC_PROLOGUE(kBwdQ)
  const float* st = prm.state + (size_t)n * prm.SS;
  load_table<LY>(sm, st, st + prm.S * D, prm.S, prm.eps);
  const T* qb = static_cast<const T*>(prm.q) + stream_offset(prm.lq, n, prm.B, prm.H);
  const T* gb = static_cast<const T*>(prm.dout) + stream_offset(prm.ldo, n, prm.B, prm.H);
  T* dqb = static_cast<T*>(prm.dq) + stream_offset(prm.ldq, n, prm.B, prm.H);
  __syncthreads();
  AggTC<LY> agg;
  agg.init();
  float ds = 0.f;
  RACE_TC_LOOP(true, qb, prm.lq.st, gb, prm.ldo.st)
    projections<LY, sizeof(T) == 2>(X, sm);
    __syncthreads();
    probabilities<LY, K>(sm, sh, inv_scale, tr.t1 - tile0);
    __syncthreads();
    agg.template add_tile<sizeof(T) == 2>(sm, Y);
    rowdot_tc<LY, sizeof(T) == 2>(Y, sm);
    __syncthreads();
    hash_backward<LY, K, false>(sm, sh, inv_scale, nullptr, ds);
    __syncthreads();
    float c[D / 32][4];
    int m0, n0;
    readout_tc<LY, true>(sm, c, m0, n0);
    store_c_global<T, D / 32>(c, dqb, prm.ldq.st, tile0, tr.t1, m0, n0);
  RACE_TC_LOOP_END
  float* dst = prm.part + ((size_t)n * prm.P + part) * prm.SS;
  agg.write(dst, prm.S);
  const float tot = cta_sum_nw(ds, sm + LY::MISC);
  if (threadIdx.x == 0) prm.dscale_part[(size_t)n * prm.P + part] = tot;
}

// B2: dv = pK . dB, dpK = v . dB^T + dA, then dk; the k-side dscale.
template <typename T, int D, int SPAD, int K>
__global__ void __launch_bounds__(NT, 3) k_tc_bwd_kv(const Params prm) {
  RACE_TC_PROLOGUE(kBwdKV)
  const float* st = prm.state + (size_t)n * prm.SS;
  const float* gs = prm.gstate_in + (size_t)n * prm.SS;
  load_table<LY>(sm, gs, st + prm.S * D, prm.S, prm.eps);   // dB = dE / (A + eps)
  float* dA = sm + LY::MISC;   // dA_s = -sum_d dE_sd B_sd / (A_s + eps)^2
  {
    const int lane = threadIdx.x & 31;
    for (int s = threadIdx.x >> 5; s < LY::S8; s += NW) {
      float a = 0.f;
      if (s < prm.S) {
        const float inv = 1.f / (st[prm.S * D + s] + prm.eps);
        for (int d = lane; d < D; d += 32) a = fmaf(gs[s * D + d], st[s * D + d], a);
        a *= inv * inv;
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
  RACE_TC_LOOP(true, kb, prm.lk.st, vb, prm.lv.st)
    projections<LY, sizeof(T) == 2>(X, sm);
    __syncthreads();
    probabilities<LY, K>(sm, sh, inv_scale, tr.t1 - tile0);
    __syncthreads();
    {
      float c[D / 32][4];
      int m0, n0;
      readout_tc<LY, false>(sm, c, m0, n0);
      store_c_global<T, D / 32>(c, dvb, prm.ldv.st, tile0, tr.t1, m0, n0);
    }
    rowdot_tc<LY, sizeof(T) == 2>(Y, sm);
    __syncthreads();
    hash_backward<LY, K, true>(sm, sh, inv_scale, dA, ds);
    __syncthreads();
    float c[D / 32][4];
    int m0, n0;
    readout_tc<LY, true>(sm, c, m0, n0);
    store_c_global<T, D / 32>(c, dkb, prm.ldk.st, tile0, tr.t1, m0, n0);
  RACE_TC_LOOP_END
  const float tot = cta_sum_nw(ds, sm + LY::MISC + 32);
  if (threadIdx.x == 0) prm.dscale_part[(size_t)n * prm.P + part] = tot;
}

}  // namespace tc
}  // namespace race
