// race_causal5.cuh -- causal (per-bucket prefix mean) RACE attention on the
// 5th-generation tensor cores, chunkwise.
//
// Per stream n, with W_s(t) = pQ_s(t) / (A_s(t) + eps), A_s(t) = sum_{tau<=t}
// pK_s(tau) and B_s(t) = sum_{tau<=t} pK_s(tau) v(tau) (misc/race.py:108-138),
//
//   out(t) = sum_s W_s(t) B_s(t).
//
// The token axis of a stream is cut into P contiguous ranges of whole
// 128-token tiles; the exclusive prefix (B0, A0) of every range comes from the
// range totals (the non-causal tcgen05 reduce) and a float64 scan over ranges.
// A persistent CTA walks its range tile by tile and, inside a tile,
//
//   out = W . B0^T + mask(W . pK^T) . V         (mask: tau <= t)
//
// with B0 the prefix at the tile start: the 128 x 128 intra-tile matrix
// G = W pK^T, masked and split into bf16 parts (in place in tensor memory,
// or in shared memory for the query backward), is the A operand of the
// second product.  The state B0 is carried from tile to tile
// by the tensor core (B0 += V^T pK accumulates in tensor memory over the
// range); A(t) is a warp scan of pK over the tile's tokens.
//
// The soft hash reads fp32 projections x . P^T of q and k computed once by a
// pre-pass (k_c5_proj) and kept in the forward's saved state, so the backward
// passes never read q or k again (16 floats per token instead of D).
//
// Precision: split bf16 as in race_t5.cuh -- W, pK, V, B0 and the masked G in
// two parts (hi + lo, 16 significant bits), every product accumulated in fp32
// (hi.hi + hi.lo + lo.hi).
#pragma once

#include "race_t5.cuh"

namespace race {
namespace c5 {

using namespace t5;

// ------------------------------------------------------------------ TMA, 3-D
// [N][T][C] float32 arrays (projections, alpha) are mapped as (C, T, N) with
// 128-row boxes of whole rows (C * 4 bytes, a multiple of 16, no swizzle).
__device__ __forceinline__ void tma_load3(void* dst, const CUtensorMap* map, int c0, int c1, int c2,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, "
      "{%2, %3, %4}], [%5];" ::"r"(saddr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(saddr(bar))
      : "memory");
}
__device__ __forceinline__ void tma_store3(const CUtensorMap* map, const void* src, int c0, int c1,
                                           int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(saddr(src)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// 5-D tile of one [M, B, T, H, D] tensor onto `bar` (the caller arms it).
template <typename T, int D>
__device__ __forceinline__ void tma_rows5(const CUtensorMap* map, void* dst, const Layout& lay,
                                          const Params& prm, int n, int64_t t0, uint64_t* bar) {
  using BX = Box<T, D>;
  const int h = n % prm.H, b = (n / prm.H) % prm.B, m = n / (prm.H * prm.B);
#pragma unroll
  for (int x = 0; x < BX::NB; ++x)
    tma_load5(static_cast<char*>(dst) + x * TT * BX::IB, map, x * BX::IB / (int)sizeof(T), (int)t0,
              h, b, lay.sm == 0 ? 0 : m, bar);
}

// instruction descriptor, M = 128, A K-major, B MN-major
template <int N>
__host__ __device__ constexpr uint32_t idesc_bmn() {
  static_assert(N % 16 == 0 && N >= 16 && N <= 256, "M = 128 needs N % 16 == 0, N <= 256");
  return (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(128 >> 4) << 24);
}

// Inclusive scan over the 32 tokens of a warp (lane = token); returns the
// warp total in `tot`.
__device__ __forceinline__ float warp_scan(float x, float& tot) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  tot = __shfl_sync(0xffffffffu, x, 31);
  return x;
}

// Writes the 8 bf16 values of one 16-byte chunk (columns 8 c8 .. of row r) of
// an operand with C columns.
template <int C>
__device__ __forceinline__ void put_chunk(bf16* op, int r, int c8, const uint4& u) {
  reinterpret_cast<uint4*>(op)[chunk<C>(r, c8)] = u;
}

// hi / lo parts of 8 floats as two 16-byte chunks
__device__ __forceinline__ void split8(const float* v, uint4& hi, uint4& lo) {
  split2(v[0], v[1], hi.x, lo.x);
  split2(v[2], v[3], hi.y, lo.y);
  split2(v[4], v[5], hi.z, lo.z);
  split2(v[6], v[7], hi.w, lo.w);
}

// the 8 floats as one 16-byte chunk of bf16 (single-part operands)
__device__ __forceinline__ void cvt8(const float* v, uint4& hi) {
  uint32_t* h = &hi.x;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const __nv_bfloat162 b = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
    h[j] = *reinterpret_cast<const uint32_t*>(&b);
  }
}

// Writes 8 values as the hi chunk c8 (and, with two parts, the lo chunk
// c8 + LOFF) of row r of an operand with C columns.
template <int C, int LOFF, bool ONE>
__device__ __forceinline__ void put_parts8(bf16* op, int r, int c8, const float* v) {
  uint4 hi, lo;
  if constexpr (ONE) {
    cvt8(v, hi);
  } else {
    split8(v, hi, lo);
    put_chunk<C>(op, r, c8 + LOFF, lo);
  }
  put_chunk<C>(op, r, c8, hi);
}

// ------------------------------------------------------------------ projections
// proj[n][t][j] = x[n][t] . planes[m][j] (j < L K; columns up to 16 are zero)
// for one of q or k: the soft hash of every causal kernel reads these, so q and
// k are read once.  128-token tiles land by TMA, are split into three bf16
// parts (24 significant bits: fp32 accuracy, which the temperature gradient's
// cancelling sum needs) and multiplied on the tensor core by the planes' three
// parts (all nine cross products, N = 3 x 16); the fp32 rows leave by a TMA
// store.  Persistent, two CTAs of 256 threads per SM (two per token), the
// next tile loading while this one is converted.
template <int D>
struct ProjLay {
  static constexpr int NTH = 2;                            // threads per token (half a row each)
  static constexpr int NFULL = 2;
  static constexpr int XS = 0;                             // [2] slots: landed, then 3 parts
  static constexpr int PS = XS + 2 * Slot<D, 3>::FLOATS;   // bf16 [3 PJ x D] planes (hi; mid; lo)
  static constexpr int STG = PS + 3 * PJ * D / 2;          // fp32 [TT][PJ] staging of the store
  static constexpr int BAR = STG + TT * PJ;
  static constexpr int FLOATS = BAR + 16 + 256;
  static constexpr int TCOLS = 64;                         // three PJ-column blocks
  static_assert(FLOATS * 4 <= 113 * 1024, "two CTAs per SM");
};

// maps: 0 x (5-D), 1 proj ([N][T][16] float32)
template <typename T, int D>
__global__ void __launch_bounds__(TT * ProjLay<D>::NTH, 2)
    k_c5_proj(const Params prm, const __grid_constant__ TmaMaps maps) {
  using LY = ProjLay<D>;
  constexpr int NTH = LY::NTH, W = D / NTH, PW = PJ / NTH;
  constexpr bool F32 = sizeof(T) == 4;
  T5_PROLOGUE
  (void)cur_n;
  (void)L;
  (void)inv_scale;
  bf16* ps = reinterpret_cast<bf16*>(sm + LY::PS);
  float* stg = sm + LY::STG;
  for (int w = blockIdx.x; w < items && !failed; w += gridDim.x) {
    const Item it = item_of(prm, w);
    if (it.ntiles <= 0) continue;
    const int n = it.n;
    const int m = prm.Mp == 1 ? 0 : n / (prm.B * prm.H);
    __syncthreads();
    if (m != cur_m) {
      const float* pl = prm.planes + (size_t)m * prm.LK * D;
      put_stack<PJ, D, 3, TT * NTH>(ps, [&](int j, int d) { return j < prm.LK ? pl[j * D + d] : 0.f; });
      cur_m = m;
    }
    auto load = [&](int j) {
      if (failed) return;
      const int f = j & 1;
      inflight |= 1u << f;
      if (tid == 0) {
        fence_async_smem();
        bar_expect_tx(full + f, (uint32_t)Box<T, D>::BYTES);
        tma_rows5<T, D>(&maps.map[0], sm + LY::XS + f * Slot<D, 3>::FLOATS, prm.lq, prm, n,
                        it.t0 + (int64_t)j * TT, full + f);
      }
    };
    load(0);
    for (int i = 0; i < it.ntiles; ++i) {
      const int64_t tile0 = it.t0 + (int64_t)i * TT;
      const int f = i & 1;
      float* X = sm + LY::XS + f * Slot<D, 3>::FLOATS;
      if (i + 1 < it.ntiles) load(i + 1);
      T5_WAIT(full + f, (phF >> f) & 1);
      if (!failed) {
        phF ^= 1u << f;
        inflight &= ~(1u << f);
      }
      {
        float x[W];
        read_cols<T, D, W>(X, row, sub * W, x);
        __syncthreads();
        put_cols<D, W, F32 ? 3 : 1>(Slot<D, 3>::part(X, 0), Slot<D, 3>::part(X, 1),
                                    Slot<D, 3>::part(X, 2), row, sub * W, x);
      }
      fence_async_smem();
      fence_before();
      __syncthreads();
      if (tid == 0 && !failed) {
        fence_after();
        bulk_wait_read();   // the previous tile's store has left the staging rows
        gemm_parts<PJ, 3, D / 16, D, D>(tbase, Slot<D, 3>::part(X, 0), Slot<D, 3>::part(X, 1),
                                        Slot<D, 3>::part(X, 2), F32 ? 3 : 1, ps, false);
        { commit(barA); ++issA; }
      }
      T5_WAIT(barA, phA);
      phA ^= 1;
      fence_after();
      {
        float pr[PW];
        tld_sum<PW, 3>(tlane + sub * PW, PJ, pr);
        float4* dst = reinterpret_cast<float4*>(stg + row * PJ + sub * PW);
#pragma unroll
        for (int q4 = 0; q4 < PW / 4; ++q4)
          dst[q4] = make_float4(pr[4 * q4], pr[4 * q4 + 1], pr[4 * q4 + 2], pr[4 * q4 + 3]);
      }
      fence_async_smem();
      fence_before();
      __syncthreads();
      if (tid == 0 && !failed) {
        tma_store3(&maps.map[1], stg, 0, (int)tile0, n);
        bulk_commit();
      }
      if (T5_VOTE()) break;
    }
  }
  T5_EPILOGUE
}

// Sum of one value over the NTH threads (row, sub) of each token, in a fixed
// order, through shared memory (the threads of a token sit in different warps).
template <int NTH>
__device__ __forceinline__ float token_sum(float x, float* xs, int row, int sub) {
  xs[sub * TT + row] = x;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int k = 0; k < NTH; ++k) t += xs[k * TT + row];
  return t;
}

// ------------------------------------------------------------------ F2 forward
// Per tile of a range, with the prefix B0, A0 at the tile start: the hash from
// the projections, A by a warp scan, W, then on the tensor core G = W pK^T,
// out = W B0^T + mask(G) V and the state B0 += V^T pK.  The masked intra-tile
// matrix is kept in tensor memory:
// the G accumulator's 128 columns are read by the threads, masked, split into
// bf16 hi / lo and written back in place (packed, 64 columns each) as the A
// operand of mask(G) . V, so the shared memory holds only one set of input
// slots and the operands (about 110 KB) and two CTAs of 256 threads share an
// SM: one CTA's thread phases run while the other's MMAs and loads are in
// flight.  The out tile leaves through the consumed v slot.
template <int D, int SPAD>
struct FwdLay {
  static constexpr int NTH = 2;
  static constexpr int SP = (SPAD + 15) / 16 * 16;
  static constexpr int NFULL = 2;                       // 0: projections, 1: v
  static constexpr int VX = 0;                          // v (landed, hi | lo), then out staging
  static constexpr int PJX = VX + Slot<D>::FLOATS;      // projQ [TT][16] then projK [TT][16]
  static constexpr int PK = PJX + 2 * TT * PJ;          // bf16 [TT x 2SP] pK (hi | lo)
  static constexpr int WH = PK + TT * SP;               // bf16 [TT x 2SP] W (hi | hi)
  static constexpr int WL = WH + TT * SP;               // bf16 [TT x SP] W lo
  static constexpr int B0 = WL + TT * SP / 2;           // bf16 [D x 2SP] B0^T (hi | lo)
  static constexpr int B0F = B0 + D * SP;               // fp32 [SP][D]
  static constexpr int A0 = B0F + SP * D;               // double [SP]
  static constexpr int SCAN = A0 + 2 * SP;              // [SP][4]
  static constexpr int DENX = SCAN + 4 * SP;            // [NTH][TT]
  static constexpr int BAR = DENX + NTH * TT;
  static constexpr int FLOATS = BAR + 16 + 256;
  static constexpr int TCOLS = 256;
  // G [0, 128) (then mask(G) hi [0, 64), lo [64, 128) as packed bf16), OUT, ST (M = 64)
  static constexpr int C_G = 0, C_OUT = 128, C_ST = 128 + D;
  static_assert(C_ST + 2 * SP <= TCOLS, "tensor-memory columns");
  static_assert(FLOATS * 4 <= 113 * 1024, "two CTAs per SM");
};

__device__ __forceinline__ void mma_ta(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t id,
                                       bool acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(b), "r"(id), "r"((uint32_t)acc));
}
// 8 consecutive 32-bit columns of this thread's lane
__device__ __forceinline__ void tst8(uint32_t taddr, const uint32_t (&v)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
      : "memory");
}
__device__ __forceinline__ void tst_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

template <typename T, int D, int SPAD, int K>
__global__ void __launch_bounds__(TT * FwdLay<D, SPAD>::NTH, 2)
    k_c5_fwd(const Params prm, const __grid_constant__ TmaMaps maps) {
  using LY = FwdLay<D, SPAD>;
  constexpr int SP = LY::SP, NTH = LY::NTH, W = D / NTH;
  using G = Groups<K>;
  constexpr int NG = SP / G::GB;
  constexpr int MYG = (NG + NTH - 1) / NTH;
  constexpr int GC = TT / NTH;                         // G columns per thread
  // bf16 inputs: W, pK, B0 and the masked G as one bf16 part each (the
  // path's bf16 tolerance), fp32: two (hi + lo)
  constexpr bool ONE = sizeof(T) == 2;
  constexpr int KP = ONE ? SP : 2 * SP;                // K extent of the W / pK / B0 products
  constexpr bool DIRECT = ONE && D == 64;              // the landed v tile is the MMA operand
  T5_PROLOGUE
  (void)cur_m;
  (void)cur_n;
  bf16* pk = reinterpret_cast<bf16*>(sm + LY::PK);
  bf16* wh = reinterpret_cast<bf16*>(sm + LY::WH);
  bf16* wl = reinterpret_cast<bf16*>(sm + LY::WL);
  bf16* b0 = reinterpret_cast<bf16*>(sm + LY::B0);
  float* b0f = sm + LY::B0F;
  double* a0 = reinterpret_cast<double*>(sm + LY::A0);
  float* scan = sm + LY::SCAN;
  const int lane = tid & 31, quad = warp & 3;
  for (int w = blockIdx.x; w < items && !failed; w += gridDim.x) {
    const Item it = item_of(prm, w);
    if (it.ntiles <= 0) continue;
    const int n = it.n;
    __syncthreads();
    {
      const float* st = prm.state + ((size_t)n * prm.P + it.part) * prm.SS;
      for (int e = tid; e < SP * D; e += TT * NTH) b0f[e] = e / D < prm.S ? st[e] : 0.f;
      for (int s = tid; s < SP; s += TT * NTH) a0[s] = s < prm.S ? (double)st[prm.S * D + s] : 0.0;
    }
    __syncthreads();
    if (tid < D) {
      for (int s8 = 0; s8 < SP / 8; ++s8) {
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = b0f[(s8 * 8 + e) * D + tid];
        put_parts8<2 * SP, SP / 8, ONE>(b0, tid, s8, v);
      }
    }
    auto load_p = [&](int j) {
      if (failed) return;
      inflight |= 1u;
      if (tid == 0) {
        const int64_t t0 = it.t0 + (int64_t)j * TT;
        float* pj = sm + LY::PJX;
        fence_async_smem();
        bar_expect_tx(full, (uint32_t)(2 * TT * PJ * 4));
        tma_load3(pj, &maps.map[0], 0, (int)t0, n, full);
        tma_load3(pj + TT * PJ, &maps.map[1], 0, (int)t0, n, full);
      }
    };
    auto load_v = [&](int j) {   // thread 0 only after the out store has read the slot
      if (failed) return;
      inflight |= 2u;
      if (tid == 0) {
        bulk_wait_read();
        fence_async_smem();
        bar_expect_tx(full + 1, (uint32_t)Box<T, D>::BYTES);
        tma_rows5<T, D>(&maps.map[2], sm + LY::VX, prm.lv, prm, n, it.t0 + (int64_t)j * TT,
                        full + 1);
      }
    };
    load_p(0);
    load_v(0);
    for (int i = 0; i < it.ntiles; ++i) {
      const int64_t tile0 = it.t0 + (int64_t)i * TT;
      float* VXt = sm + LY::VX;
      const float* pj = sm + LY::PJX;
      T5_WAIT(full, phF & 1);
      if (!failed) {
        phF ^= 1u;
        inflight &= ~1u;
      }
      T5_WAIT(full + 1, (phF >> 1) & 1);
      if (!failed) {
        phF ^= 2u;
        inflight &= ~2u;
      }
      const bool valid = tile0 + row < it.t1;
      {
        float y[W];
        if constexpr (!DIRECT) read_cols<T, D, W>(VXt, row, sub * W, y);
        float pq[MYG][G::GB], pkv[MYG][G::GB];
#pragma unroll
        for (int a = 0; a < MYG; ++a) {
          const int gi = sub + a * NTH;
          if (gi < NG) {
            float pj_[G::GK], h[G::GK];
            const bool has = gi * G::GK < PJ;
#pragma unroll
            for (int k = 0; k < G::GK; ++k) pj_[k] = has ? pj[row * PJ + gi * G::GK + k] : 0.f;
            group_probs<K>(pj_, gi * G::GT, has ? L : 0, inv_scale, pq[a], h);
#pragma unroll
            for (int k = 0; k < G::GK; ++k)
              pj_[k] = has ? pj[TT * PJ + row * PJ + gi * G::GK + k] : 0.f;
            group_probs<K>(pj_, gi * G::GT, has ? L : 0, inv_scale, pkv[a], h);
            if (!valid) {
#pragma unroll
              for (int b = 0; b < G::GB; ++b) pq[a][b] = pkv[a][b] = 0.f;
            }
          }
        }
        __syncthreads();   // v and the projections read
        if (i + 1 < it.ntiles) load_p(i + 1);
        if constexpr (!DIRECT)
          put_cols<D, W, sizeof(T) == 4 ? 2 : 1>(Slot<D>::part(VXt, 0), Slot<D>::part(VXt, 1),
                                                 nullptr, row, sub * W, y);
        float incl[MYG][G::GB];
#pragma unroll
        for (int a = 0; a < MYG; ++a) {
          const int gi = sub + a * NTH;
          if (gi < NG) {
#pragma unroll
            for (int b = 0; b < G::GB; ++b) {
              float tot;
              incl[a][b] = warp_scan(pkv[a][b], tot);
              if (lane == 31) scan[(gi * G::GB + b) * 4 + quad] = tot;
            }
          }
        }
        __syncthreads();
        float av[MYG][G::GB], dpart = 0.f;
#pragma unroll
        for (int a = 0; a < MYG; ++a) {
          const int gi = sub + a * NTH;
          if (gi < NG) {
#pragma unroll
            for (int b = 0; b < G::GB; ++b) {
              const int s = gi * G::GB + b;
              float before = 0.f;
              for (int q2 = 0; q2 < quad; ++q2) before += scan[s * 4 + q2];
              av[a][b] = (float)(a0[s] + (double)(before + incl[a][b]));
              dpart = fmaf(pq[a][b], av[a][b], dpart);
            }
          }
        }
        float rden = 0.f;
        if (prm.global_norm) {
          const float den = token_sum<NTH>(dpart, sm + LY::DENX, row, sub);
          rden = 1.f / fmaxf(den, prm.eps);
          if (prm.den_out != nullptr && sub == 0 && valid) prm.den_out[(size_t)n * prm.T + tile0 + row] = den;
        }
#pragma unroll
        for (int a = 0; a < MYG; ++a) {
          const int gi = sub + a * NTH;
          if (gi < NG) {
            float wv[G::GB];
#pragma unroll
            for (int b = 0; b < G::GB; ++b)
              wv[b] = prm.global_norm ? pq[a][b] * rden : __fdividef(pq[a][b], av[a][b] + prm.eps);
#pragma unroll
            for (int c8 = 0; c8 < G::GB / 8; ++c8) {
              const int c = gi * G::GB / 8 + c8;
              put_parts8<2 * SP, SP / 8, ONE>(pk, row, c, pkv[a] + 8 * c8);
              if constexpr (ONE) {
                uint4 hi;
                cvt8(wv + 8 * c8, hi);
                put_chunk<2 * SP>(wh, row, c, hi);
              } else {
                uint4 hi, lo;
                split8(wv + 8 * c8, hi, lo);
                put_chunk<2 * SP>(wh, row, c, hi);
                put_chunk<2 * SP>(wh, row, SP / 8 + c, hi);
                put_chunk<SP>(wl, row, c, lo);
              }
            }
          }
        }
      }
      fence_async_smem();
      fence_before();
      __syncthreads();
      if (tid == 0 && !failed) {
        fence_after();
#pragma unroll
        for (int ks = 0; ks < KP / 16; ++ks)
          mma(tbase + LY::C_G, desc<2 * SP>(wh, ks), desc<2 * SP>(pk, ks), idesc<TT>(), ks > 0);
        if constexpr (!ONE) {
#pragma unroll
          for (int ks = 0; ks < SP / 16; ++ks)
            mma(tbase + LY::C_G, desc<SP>(wl, ks), desc<2 * SP>(pk, ks), idesc<TT>(), true);
        }
#pragma unroll
        for (int ks = 0; ks < KP / 16; ++ks)
          mma(tbase + LY::C_OUT, desc<2 * SP>(wh, ks), desc<2 * SP>(b0, ks), idesc<D>(), ks > 0);
        if constexpr (!ONE) {
#pragma unroll
          for (int ks = 0; ks < SP / 16; ++ks)
            mma(tbase + LY::C_OUT, desc<SP>(wl, ks), desc<2 * SP>(b0, ks), idesc<D>(), true);
        }
        { commit(barA); ++issA; }
      }
      if (sub == 0 && tid < SP) {
        float tot = 0.f;
        for (int q2 = 0; q2 < 4; ++q2) tot += scan[tid * 4 + q2];
        a0[tid] += (double)tot;
      }
      T5_WAIT(barA, phA);
      phA ^= 1;
      fence_after();
      {
        {
          // masked G row (columns [GC sub, GC sub + GC)) as packed bf16 parts
          // over the thread's own columns -- hi in the first half, lo (fp32
          // inputs) in the second -- so no other thread's reads are in the way
          uint32_t hw[GC / 2], lw[GC / 2];
#pragma unroll
          for (int c0 = 0; c0 < GC; c0 += 16) {
            float g[16];
            tld16(tlane + LY::C_G + GC * sub + c0, g);
            tld_wait();
#pragma unroll
            for (int e = 0; e < 16; e += 2) {
              const float x0 = GC * sub + c0 + e > row ? 0.f : g[e];
              const float x1 = GC * sub + c0 + e + 1 > row ? 0.f : g[e + 1];
              if constexpr (ONE) {
                const __nv_bfloat162 h2 = __floats2bfloat162_rn(x0, x1);
                hw[(c0 + e) / 2] = *reinterpret_cast<const uint32_t*>(&h2);
              } else {
                split2(x0, x1, hw[(c0 + e) / 2], lw[(c0 + e) / 2]);
              }
            }
          }
#pragma unroll
          for (int c = 0; c < GC / 2; c += 8) {
            uint32_t h8[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) h8[e] = hw[c + e];
            tst8(tlane + LY::C_G + GC * sub + c, h8);
            if constexpr (!ONE) {
#pragma unroll
              for (int e = 0; e < 8; ++e) h8[e] = lw[c + e];
              tst8(tlane + LY::C_G + GC * sub + GC / 2 + c, h8);
            }
          }
          tst_wait();
        }
      }
      fence_before();
      __syncthreads();
      if (tid == 0 && !failed) {
        fence_after();
        const bf16* vp[2] = {Slot<D>::part(VXt, 0), Slot<D>::part(VXt, 1)};
        // part a of the masked G for tokens [GC j, GC j + GC): columns GC j + a GC / 2 + ...
#pragma unroll
        for (int a2 = 0; a2 < (ONE ? 1 : 2); ++a2)
#pragma unroll
          for (int b2 = 0; b2 < (ONE ? 1 : 2); ++b2) {
            if (a2 + b2 == 2) continue;
#pragma unroll
            for (int ks = 0; ks < TT / 16; ++ks)
              mma_ta(tbase + LY::C_OUT,
                     tbase + LY::C_G + GC * (16 * ks / GC) + a2 * (GC / 2) + (16 * ks % GC) / 2,
                     desc_a_mn<D, DIRECT>(vp[b2], ks), idesc_bmn<D>(), true);
          }
#pragma unroll
        for (int a = 0; a < (sizeof(T) == 4 ? 2 : 1); ++a)
#pragma unroll
          for (int ks = 0; ks < TT / 16; ++ks)
            mma(tbase + LY::C_ST, desc_a_mn<D, DIRECT>(vp[a], ks), desc_mn<2 * SP>(pk, ks),
                idesc64_mn<KP>(), i > 0 || a > 0 || ks > 0);
        { commit(barB); ++issB; }
      }
      T5_WAIT(barB, phB);
      phB ^= 1;
      fence_after();
      {
        float o[W];
        tld_sum<W, 1>(tlane + LY::C_OUT + sub * W, 0, o);
        put_tile_cols<T, D, W>(sm + LY::VX, row, sub * W, o);   // v consumed: out staging
      }
      // B0 of the next tile (M = 64 lanes: row d = 16 q + l); the NTH warps of
      // a lane quarter take every NTH-th 8-bucket chunk
      if (i + 1 < it.ntiles) {
        const int d = 16 * quad + lane;
        for (int s8 = sub; s8 < SP / 8; s8 += NTH) {
          float lo8[8] = {}, v[8];
          tld8(tlane + LY::C_ST + 8 * s8, v);
          if constexpr (!ONE) tld8(tlane + LY::C_ST + SP + 8 * s8, lo8);
          tld_wait();
          if (lane < 16 && d < D) {
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] += b0f[(s8 * 8 + e) * D + d] + lo8[e];
            put_parts8<2 * SP, SP / 8, ONE>(b0, d, s8, v);
          }
        }
      }
      fence_async_smem();
      fence_before();
      __syncthreads();
      if (tid == 0 && !failed) {
        tma_store_tile<T, D>(&maps.map[3], sm + LY::VX, prm.lo, prm, n, tile0);
        bulk_commit();
      }
      if (i + 1 < it.ntiles) load_v(i + 1);
      if (T5_VOTE()) break;
    }
  }
  T5_EPILOGUE
}

// ------------------------------------------------------------------ B1 query backward
// Per tile (prefix B0, A0 at the tile start as in the forward):
//   R = dO . B0^T + mask(dO . V^T) . pK       R_s(t) = dO(t) . B_s(t)
//   dpQ_s = R_s / (A_s + eps),  alpha_s = -W_s dpQ_s,  dq = dproj(pQ, dpQ) . P
// (misc/race.py:108-138 differentiated; kernels/cpu/race_pref.cpp:104-181 with
// W folded in).  Per range: sum_t W_s(t) dO(t) and sum_t alpha_s(t) into the
// range's gradient slot (the reverse scan over ranges makes them suffixes);
// alpha per token and the key mass at every tile start for the key backward.
template <int D, int SPAD>
struct BwdQLayC {
  static constexpr int NTH = 4;
  static constexpr int SP = (SPAD + 15) / 16 * 16;
  static constexpr int NFULL = 1;                       // one set of input slots
  static constexpr int VX = 0;                          // v (landed, then hi | lo)
  static constexpr int GX = VX + Slot<D>::FLOATS;       // dO (landed, then hi | lo)
  static constexpr int PJX = GX + Slot<D>::FLOATS;      // projQ [TT][16] then projK [TT][16]
  static constexpr int MM = PJX + 2 * TT * PJ;          // alpha [TT][SA] and dq staging
  static constexpr int STG_DQ = MM + TT * SP;           // dq staging (1 KB aligned)
  static constexpr int PK = MM + TT * TT;               // bf16 [TT x 2SP] pK (hi | lo)
  static constexpr int WP = PK + TT * SP;               // bf16 [TT x 2SP] W (hi | lo)
  static constexpr int B0S = WP + TT * SP;              // bf16 [2SP x D] B0 (hi rows; lo rows)
  static constexpr int DJ = B0S + SP * D;               // bf16 [TT x PJ] dproj hi, then lo
  static constexpr int PT = DJ + TT * PJ;               // bf16 [2D x PJ] planes^T (hi; lo)
  static constexpr int B0F = PT + D * PJ;               // fp32 [SP][D] prefix at the range start
  static constexpr int A0 = B0F + SP * D;               // double [SP]
  static constexpr int SCAN = A0 + 2 * SP;              // [SP][4]
  static constexpr int DENX = SCAN + 4 * SP;            // [NTH][TT] global mode: row-sum parts
  static constexpr int RED = DENX + NTH * TT;           // [16]
  static constexpr int BAR = RED + 16;
  static constexpr int FLOATS = BAR + 16 + 256;
  static constexpr int TCOLS = 512;
  // M [0, 128), R [128, 128 + 2SP), DQ [192, 192 + 2D), ST / WD (M = 64) 2SP each
  static constexpr int C_M = 0, C_R = 128, C_DQ = 192, C_ST = 192 + 2 * D, C_WD = C_ST + 64;
  static_assert(C_R + 2 * SP <= C_DQ && C_WD + 2 * SP <= TCOLS, "tensor-memory columns");
  static_assert(STG_DQ + TT * D <= PK, "staging inside the masked-matrix area");
  static_assert(MM % 256 == 0 && STG_DQ % 256 == 0, "1 KB aligned TMA boxes");
  static_assert(FLOATS * 4 <= 227 * 1024, "shared memory");
};

// maps: 0 projQ, 1 projK, 2 v, 3 dO, 4 dq, 5 alpha ([N][T][SA] float32)
template <typename T, int D, int SPAD, int K>
__global__ void __launch_bounds__(TT * BwdQLayC<D, SPAD>::NTH, 1)
    k_c5_bwd_q(const Params prm, const __grid_constant__ TmaMaps maps) {
  using LY = BwdQLayC<D, SPAD>;
  constexpr int SP = LY::SP, NTH = LY::NTH, NTHR = TT * NTH, W = D / NTH;
  using G = Groups<K>;
  constexpr int NG = SP / G::GB;
  constexpr int MYG = (NG + NTH - 1) / NTH;
  constexpr int GC = TT / NTH;
  constexpr bool F32 = sizeof(T) == 4;
  // bf16 inputs: pK, W, B0, the masked M and dproj as one bf16 part each
  // (the path's bf16 tolerance); fp32: two
  constexpr bool ONE = !F32;
  constexpr int KP = ONE ? SP : 2 * SP;                // N extent of the bucket products
  constexpr bool DIRECT = ONE && D == 64;              // landed v / dO tiles are MMA operands
  T5_PROLOGUE
  (void)cur_n;
  bf16* pk = reinterpret_cast<bf16*>(sm + LY::PK);
  bf16* wp = reinterpret_cast<bf16*>(sm + LY::WP);
  bf16* b0s = reinterpret_cast<bf16*>(sm + LY::B0S);
  bf16* dj = reinterpret_cast<bf16*>(sm + LY::DJ);
  bf16* pt = reinterpret_cast<bf16*>(sm + LY::PT);
  float* b0f = sm + LY::B0F;
  double* a0 = reinterpret_cast<double*>(sm + LY::A0);
  float* scan = sm + LY::SCAN;
  const int lane = tid & 31, quad = warp & 3;
  const int64_t tiles_n = (prm.T + TT - 1) / TT;
  // planes of DJ not covered by any bucket group stay zero
  for (int i = tid; i < TT * PJ; i += NTHR) reinterpret_cast<float*>(dj)[i] = 0.f;
  for (int w = blockIdx.x; w < items && !failed; w += gridDim.x) {
    const Item it = item_of(prm, w);
    const int n = it.n;
    float* slot = prm.gstate_out + ((size_t)n * prm.P + it.part) * prm.SS;
    float ds = 0.f;
    float asum[MYG][G::GB];
#pragma unroll
    for (int a = 0; a < MYG; ++a)
#pragma unroll
      for (int b = 0; b < G::GB; ++b) asum[a][b] = 0.f;
    if (it.ntiles > 0) {
      const int m = prm.Mp == 1 ? 0 : n / (prm.B * prm.H);
      __syncthreads();
      if (m != cur_m) {
        const float* pl = prm.planes + (size_t)m * prm.LK * D;
        put_stack<D, PJ, 2, NTHR>(pt, [&](int d, int j) { return j < prm.LK ? pl[j * D + d] : 0.f; });
        cur_m = m;
      }
      const float* st = prm.state + ((size_t)n * prm.P + it.part) * prm.SS;
      for (int e = tid; e < SP * D; e += NTHR) b0f[e] = e / D < prm.S ? st[e] : 0.f;
      for (int s2 = tid; s2 < SP; s2 += NTHR) a0[s2] = s2 < prm.S ? (double)st[prm.S * D + s2] : 0.0;
      __syncthreads();
      // B0 operand of the first tile: rows s (hi), SP + s (lo), columns d
      for (int e = tid; e < SP * D; e += NTHR) {
        const int s2 = e / D, d = e % D;
        const float x = b0f[e];
        const bf16 h = __float2bfloat16_rn(x);
        b0s[elem<D>(s2, d)] = h;
        if constexpr (!ONE) b0s[elem<D>(SP + s2, d)] = __float2bfloat16_rn(x - __bfloat162float(h));
      }
      auto load = [&](int j) {
        if (failed) return;
        inflight |= 1u;
        if (tid == 0) {
          const int64_t t0 = it.t0 + (int64_t)j * TT;
          float* pj = sm + LY::PJX;
          fence_async_smem();
          bar_expect_tx(full, (uint32_t)(2 * Box<T, D>::BYTES + 2 * TT * PJ * 4));
          tma_load3(pj, &maps.map[0], 0, (int)t0, n, full);
          tma_load3(pj + TT * PJ, &maps.map[1], 0, (int)t0, n, full);
          tma_rows5<T, D>(&maps.map[2], sm + LY::VX, prm.lv, prm, n, t0, full);
          tma_rows5<T, D>(&maps.map[3], sm + LY::GX, prm.ldo, prm, n, t0, full);
        }
      };
      load(0);
      for (int i = 0; i < it.ntiles; ++i) {
        const int64_t tile0 = it.t0 + (int64_t)i * TT;
        float* VXt = sm + LY::VX;
        float* GXt = sm + LY::GX;
        const float* pj = sm + LY::PJX;
        T5_WAIT(full, phF & 1);
        if (!failed) {
          phF ^= 1u;
          inflight &= ~1u;
        }
        const bool valid = tile0 + row < it.t1;
        float pq[MYG][G::GB], hq[MYG][G::GK], am[MYG][G::GB], wv[MYG][G::GB];
        float den = 0.f, rden = 0.f;   // global mode
        {
          float y[W], g[W];
          if constexpr (!DIRECT) {
            read_cols<T, D, W>(VXt, row, sub * W, y);
            read_cols<T, D, W>(GXt, row, sub * W, g);
          }
          float pkv[MYG][G::GB];
#pragma unroll
          for (int a = 0; a < MYG; ++a) {
            const int gi = sub + a * NTH;
            if (gi < NG) {
              float pj_[G::GK], h[G::GK];
              const bool has = gi * G::GK < PJ;
#pragma unroll
              for (int k = 0; k < G::GK; ++k) pj_[k] = has ? pj[row * PJ + gi * G::GK + k] : 0.f;
              group_probs<K>(pj_, gi * G::GT, has ? L : 0, inv_scale, pq[a], hq[a]);
#pragma unroll
              for (int k = 0; k < G::GK; ++k)
                pj_[k] = has ? pj[TT * PJ + row * PJ + gi * G::GK + k] : 0.f;
              group_probs<K>(pj_, gi * G::GT, has ? L : 0, inv_scale, pkv[a], h);
              if (!valid) {
#pragma unroll
                for (int b = 0; b < G::GB; ++b) pq[a][b] = pkv[a][b] = 0.f;
              }
            }
          }
          __syncthreads();   // raw tiles read; scan scratch free
          if constexpr (!DIRECT) {
            put_cols<D, W, F32 ? 2 : 1>(Slot<D>::part(VXt, 0), Slot<D>::part(VXt, 1), nullptr, row,
                                        sub * W, y);
            put_cols<D, W, F32 ? 2 : 1>(Slot<D>::part(GXt, 0), Slot<D>::part(GXt, 1), nullptr, row,
                                        sub * W, g);
          }
          float incl[MYG][G::GB];
#pragma unroll
          for (int a = 0; a < MYG; ++a) {
            const int gi = sub + a * NTH;
            if (gi < NG) {
#pragma unroll
              for (int b = 0; b < G::GB; ++b) {
                float tot;
                incl[a][b] = warp_scan(pkv[a][b], tot);
                if (lane == 31) scan[(gi * G::GB + b) * 4 + quad] = tot;
              }
            }
          }
          __syncthreads();
          float dpart = 0.f;
#pragma unroll
          for (int a = 0; a < MYG; ++a) {
            const int gi = sub + a * NTH;
            if (gi < NG) {
#pragma unroll
              for (int b = 0; b < G::GB; ++b) {
                const int s2 = gi * G::GB + b;
                float before = 0.f;
                for (int q2 = 0; q2 < quad; ++q2) before += scan[s2 * 4 + q2];
                am[a][b] = (float)(a0[s2] + (double)(before + incl[a][b]));
                dpart = fmaf(pq[a][b], am[a][b], dpart);
              }
            }
          }
          if (prm.global_norm) {
            den = token_sum<NTH>(dpart, sm + LY::DENX, row, sub);
            rden = 1.f / fmaxf(den, prm.eps);
          }
#pragma unroll
          for (int a = 0; a < MYG; ++a) {
            const int gi = sub + a * NTH;
            if (gi < NG) {
              // per-bucket mode keeps 1 / (A + eps) in am, global mode keeps A
#pragma unroll
              for (int b = 0; b < G::GB; ++b) {
                if (!prm.global_norm) am[a][b] = __fdividef(1.f, am[a][b] + prm.eps);
                wv[a][b] = pq[a][b] * (prm.global_norm ? rden : am[a][b]);
              }
#pragma unroll
              for (int c8 = 0; c8 < G::GB / 8; ++c8) {
                const int c = gi * G::GB / 8 + c8;
                put_parts8<2 * SP, SP / 8, ONE>(pk, row, c, pkv[a] + 8 * c8);
                put_parts8<2 * SP, SP / 8, ONE>(wp, row, c, wv[a] + 8 * c8);
              }
            }
          }
        }
        // the key mass at this tile's start, for the key-side walk
        if (sub == 0 && tid < SP)
          prm.range_mass[((size_t)n * tiles_n + tile0 / TT) * SP + tid] = a0[tid];
        fence_async_smem();
        fence_before();
        __syncthreads();
        if (tid == 0 && !failed) {
          fence_after();
          bulk_wait_read();   // the previous tile's alpha / dq staging sits in MM
          const bf16* vp[2] = {Slot<D>::part(VXt, 0), Slot<D>::part(VXt, 1)};
          const bf16* gp[2] = {Slot<D>::part(GXt, 0), Slot<D>::part(GXt, 1)};
          // M = dO . V^T  (hi.hi, hi.lo, lo.hi)
#pragma unroll
          for (int a = 0; a < 2; ++a)
#pragma unroll
            for (int b = 0; b < 2; ++b) {
              if (a + b == 2 || (!F32 && a + b > 0)) continue;
#pragma unroll
              for (int ks = 0; ks < D / 16; ++ks)
                mma(tbase + LY::C_M, desc_a_k<D, DIRECT>(gp[a], ks), desc_a_k<D, DIRECT>(vp[b], ks),
                    idesc<TT>(), a + b > 0 || ks > 0);
            }
          // R = dO . B0^T (B0 hi and lo stacked along N)
#pragma unroll
          for (int a = 0; a < (F32 ? 2 : 1); ++a)
#pragma unroll
            for (int ks = 0; ks < D / 16; ++ks)
              mma(tbase + LY::C_R, desc_a_k<D, DIRECT>(gp[a], ks), desc<D>(b0s, ks), idesc<KP>(),
                  a > 0 || ks > 0);
          // ST[d][s] += v^T pK (the next tiles' B0);  WD[d][s] += dO^T W (range total)
#pragma unroll
          for (int a = 0; a < (F32 ? 2 : 1); ++a)
#pragma unroll
            for (int ks = 0; ks < TT / 16; ++ks) {
              mma(tbase + LY::C_ST, desc_a_mn<D, DIRECT>(vp[a], ks), desc_mn<2 * SP>(pk, ks),
                  idesc64_mn<KP>(), i > 0 || a > 0 || ks > 0);
              mma(tbase + LY::C_WD, desc_a_mn<D, DIRECT>(gp[a], ks), desc_mn<2 * SP>(wp, ks),
                  idesc64_mn<KP>(), i > 0 || a > 0 || ks > 0);
            }
          { commit(barA); ++issA; }
        }
        if (sub == 0 && tid < SP) {
          float tot = 0.f;
          for (int q2 = 0; q2 < 4; ++q2) tot += scan[tid * 4 + q2];
          a0[tid] += (double)tot;
        }
        T5_WAIT(barA, phA);
        phA ^= 1;
        // every MMA that reads the input slots has completed: next tile's loads
        if (i + 1 < it.ntiles) load(i + 1);
        fence_after();
        {
          // masked M row (columns [GC sub, GC sub + GC)) as packed bf16 parts
          // over the thread's own tensor-memory columns -- hi in the first
          // half, lo (fp32 inputs) in the second: the A operand of R += mask(M) pK
          uint32_t hw[GC / 2], lw[GC / 2];
#pragma unroll
          for (int c0 = 0; c0 < GC; c0 += 16) {
            float g[16];
            tld16(tlane + LY::C_M + GC * sub + c0, g);
            tld_wait();
#pragma unroll
            for (int e = 0; e < 16; e += 2) {
              const float x0 = GC * sub + c0 + e > row ? 0.f : g[e];
              const float x1 = GC * sub + c0 + e + 1 > row ? 0.f : g[e + 1];
              if constexpr (ONE) {
                const __nv_bfloat162 h2 = __floats2bfloat162_rn(x0, x1);
                hw[(c0 + e) / 2] = *reinterpret_cast<const uint32_t*>(&h2);
              } else {
                split2(x0, x1, hw[(c0 + e) / 2], lw[(c0 + e) / 2]);
              }
            }
          }
#pragma unroll
          for (int c = 0; c < GC / 2; c += 8) {
            uint32_t h8[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) h8[e] = hw[c + e];
            tst8(tlane + LY::C_M + GC * sub + c, h8);
            if constexpr (!ONE) {
#pragma unroll
              for (int e = 0; e < 8; ++e) h8[e] = lw[c + e];
              tst8(tlane + LY::C_M + GC * sub + GC / 2 + c, h8);
            }
          }
          tst_wait();
        }
        fence_before();
        __syncthreads();
        if (tid == 0 && !failed) {
          fence_after();
          // R += mask(M) . pK  (both parts of M, both parts of pK along N)
#pragma unroll
          for (int a = 0; a < (ONE ? 1 : 2); ++a)
#pragma unroll
            for (int ks = 0; ks < TT / 16; ++ks)
              mma_ta(tbase + LY::C_R,
                     tbase + LY::C_M + GC * (16 * ks / GC) + a * (GC / 2) + (16 * ks % GC) / 2,
                     desc_mn<2 * SP>(pk, ks), idesc_bmn<KP>(), true);
          { commit(barB); ++issB; }
        }
        T5_WAIT(barB, phB);
        phB ^= 1;
        fence_after();
        float* stg_a = sm + LY::MM;   // alpha staging [TT][SA] (the masked matrix is consumed)
        // R_s(t) = dO(t) . B_s(t); global mode: dO . out = sum_s W_s R_s over the token
        float rr[MYG][G::GB], wr = 0.f;
#pragma unroll
        for (int a = 0; a < MYG; ++a) {
          const int gi = sub + a * NTH;
          if (gi < NG) {
            tld_sum<G::GB, ONE ? 1 : 2>(tlane + LY::C_R + gi * G::GB, SP, rr[a]);
#pragma unroll
            for (int b = 0; b < G::GB; ++b) wr = fmaf(wv[a][b], rr[a][b], wr);
          }
        }
        // global mode (out = num / max(den, eps), den = sum_s pQ_s A_s):
        //   gden = -(dO . out) / max(den, eps) (0 where the clamp holds) + d(den) given,
        //   dpQ_s = R_s / max(den, eps) + A_s gden,  alpha_s = pQ_s gden
        float gden = 0.f;
        if (prm.global_norm) {
          const float dotw = token_sum<NTH>(wr, sm + LY::DENX, row, sub);
          gden = den >= prm.eps ? -dotw * rden : 0.f;
          if (prm.dden_in != nullptr && valid) gden += prm.dden_in[(size_t)n * prm.T + tile0 + row];
        }
#pragma unroll
        for (int a = 0; a < MYG; ++a) {
          const int gi = sub + a * NTH;
          if (gi < NG) {
            float dpq[G::GB], dj_[G::GK], al[G::GB];
#pragma unroll
            for (int b = 0; b < G::GB; ++b) {
              if (prm.global_norm) {
                dpq[b] = valid ? rr[a][b] * rden + am[a][b] * gden : 0.f;
                al[b] = valid ? pq[a][b] * gden : 0.f;
              } else {
                dpq[b] = valid ? rr[a][b] * am[a][b] : 0.f;
                al[b] = -wv[a][b] * dpq[b];
              }
              asum[a][b] += al[b];
            }
            float dsl = 0.f;
            group_probs_bwd<K>(pq[a], dpq, hq[a], inv_scale, dj_, dsl);
            if (valid) ds += dsl;
#pragma unroll
            for (int b = 0; b < G::GB; ++b) {
              const int s2 = gi * G::GB + b;
              if (s2 < prm.SA) stg_a[row * prm.SA + s2] = s2 < prm.S ? al[b] : 0.f;
            }
            if (gi * G::GK < PJ) {
#pragma unroll
              for (int j = 0; j < G::GK; ++j) {
                const int jj = gi * G::GK + j;
                if (jj < PJ) {
                  const bf16 hb = __float2bfloat16_rn(valid ? dj_[j] : 0.f);
                  dj[elem<PJ>(row, jj)] = hb;
                  if constexpr (!ONE)
                    dj[TT * PJ + elem<PJ>(row, jj)] =
                        __float2bfloat16_rn((valid ? dj_[j] : 0.f) - __bfloat162float(hb));
                }
              }
            }
          }
        }
        fence_async_smem();
        fence_before();
        __syncthreads();
        if (tid == 0 && !failed) {
          fence_after();
          gemm_parts<D, 2, PJ / 16, PJ, PJ>(tbase + LY::C_DQ, dj, dj + TT * PJ, nullptr,
                                            ONE ? 1 : 2, pt, false);
          { commit(barA); ++issA; }
          tma_store3(&maps.map[5], stg_a, 0, (int)tile0, n);
          bulk_commit();
        }
        T5_WAIT(barA, phA);
        phA ^= 1;
        fence_after();
        {
          float o[W];
          tld_sum<W>(tlane + LY::C_DQ + sub * W, D, o);
          put_tile_cols<T, D, W>(sm + LY::STG_DQ, row, sub * W, o);
        }
        // B0 of the next tile: range prefix + the state so far (M = 64 lanes)
        if (i + 1 < it.ntiles) {   // the NTH warps of a lane quarter take every NTH-th chunk
          const int d = 16 * quad + lane;
          for (int s8 = sub; s8 < SP / 8; s8 += NTH) {
            float lo8[8] = {}, v[8];
            tld8(tlane + LY::C_ST + 8 * s8, v);
            if constexpr (!ONE) tld8(tlane + LY::C_ST + SP + 8 * s8, lo8);
            tld_wait();
            if (lane < 16 && d < D) {
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const int s2 = 8 * s8 + e;
                const float x = b0f[s2 * D + d] + v[e] + lo8[e];
                const bf16 h = __float2bfloat16_rn(x);
                b0s[elem<D>(s2, d)] = h;
                if constexpr (!ONE) b0s[elem<D>(SP + s2, d)] = __float2bfloat16_rn(x - __bfloat162float(h));
              }
            }
          }
        }
        fence_async_smem();
        fence_before();
        __syncthreads();
        if (tid == 0 && !failed) {
          tma_store_tile<T, D>(&maps.map[4], sm + LY::STG_DQ, prm.ldq, prm, n, tile0);
          bulk_commit();
        }
        if (T5_VOTE()) break;
      }
      if (failed) break;
      // range totals: sum_t W dO (M = 64 lanes) and sum_t alpha
      fence_after();
      if (sub == 0) {
        const int d = 16 * quad + lane;
#pragma unroll
        for (int c = 0; c < SP; c += 8) {
          float e0[8], e1[8] = {};
          tld8(tlane + LY::C_WD + c, e0);
          if constexpr (!ONE) tld8(tlane + LY::C_WD + SP + c, e1);
          tld_wait();
          if (lane < 16 && d < D) {
#pragma unroll
            for (int x = 0; x < 8; ++x)
              if (c + x < prm.S) slot[(c + x) * D + d] = e0[x] + e1[x];
          }
        }
      }
      fence_before();
      if (tid == 0) bulk_wait_read();
      __syncthreads();
      float* ms = sm + LY::MM;   // [TT][SP] per-thread alpha sums
#pragma unroll
      for (int a = 0; a < MYG; ++a)
        if (sub + a * NTH < NG)
#pragma unroll
          for (int b = 0; b < G::GB; ++b) ms[row * SP + (sub + a * NTH) * G::GB + b] = asum[a][b];
      __syncthreads();
      if (tid < prm.S) {
        float tot = 0.f;
        for (int r2 = 0; r2 < TT; ++r2) tot += ms[r2 * SP + tid];
        slot[prm.S * D + tid] = tot;
      }
    } else {
      for (int e2 = tid; e2 < prm.S * D + prm.S; e2 += NTHR) slot[e2] = 0.f;
    }
    float x = ds;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    __syncthreads();
    if ((tid & 31) == 0) sm[LY::RED + warp] = x;
    __syncthreads();
    if (tid == 0) {
      float tot = 0.f;
      for (int i = 0; i < NTHR / 32; ++i) tot += sm[LY::RED + i];
      prm.dscale_part[(size_t)n * prm.P + it.part] = tot;
    }
  }
  T5_EPILOGUE
}


// ------------------------------------------------------------------ B2 key/value backward
// Walks each range from its last tile to its first with the exclusive suffix
// (BS = sum_{later t} W_s(t) dO(t), AS = sum_{later t} alpha_s(t)) of the
// range's end.  Per tile, with asuf(tau) = AS + the in-tile suffix of alpha:
//   dpK(tau) = asuf(tau) + v . BS^T + mask'(V . dO^T) . W
//   dv(tau)  = pK . BS + mask'(pK . W^T) . dO          (mask': t >= tau)
//   dk       = dproj(pK, dpK) . P
// (kernels/cpu/race_pref.cpp:183-220 with W folded in).  The key mass at the
// tile start comes from the query walk's records.
template <int D, int SPAD>
struct BwdKVLayC {
  static constexpr int NTH = 4;
  static constexpr int SP = (SPAD + 15) / 16 * 16;
  static constexpr int NFULL = 2;                       // 0: v + projections, 1: dO
  static constexpr int VX = 0;
  static constexpr int GX = VX + Slot<D>::FLOATS;
  static constexpr int PJX = GX + Slot<D>::FLOATS;      // projQ [TT][16] then projK [TT][16]
  static constexpr int MM = PJX + 2 * TT * PJ;          // dv and dk staging (fp32 [TT x D] each)
  static constexpr int PK = MM + TT * TT;               // bf16 [TT x 2SP] pK (hi | lo)
  static constexpr int WH = PK + TT * SP;               // bf16 [TT x 2SP] W (hi | hi)
  static constexpr int WL = WH + TT * SP;               // bf16 [TT x SP] W lo
  static constexpr int BSS = WL + TT * SP / 2;          // bf16 [2SP x D] BS (hi rows; lo rows)
  static constexpr int DJ = BSS + SP * D;               // bf16 [TT x PJ] hi, then lo
  static constexpr int PT = DJ + TT * PJ;               // bf16 [2D x PJ] planes^T (hi; lo)
  static constexpr int BSF = PT + D * PJ;               // fp32 [SP][D] suffix at the range end
  static constexpr int AS = BSF + SP * D;               // double [SP] alpha suffix, running
  static constexpr int A0T = AS + 2 * SP;               // double [SP] key mass at the tile start
  static constexpr int SCAN = A0T + 2 * SP;             // [SP][4] per-warp key-mass totals
  static constexpr int SCAN2 = SCAN + 4 * SP;           // [SP][4] per-warp alpha totals
  // [NTH][TT] global mode: den parts, in the projection slot (read before the
  // scan barrier, reloaded after the first MMA batch)
  static constexpr int DENX = PJX;
  static constexpr int RED = SCAN2 + 4 * SP;
  static constexpr int BAR = RED + 16;
  static constexpr int FLOATS = BAR + 16 + 256;
  static constexpr int TCOLS = 512;
  // MT / DK [0, 128), GT [128, 256), VB [256, 256 + 2SP), DV [C_DV, C_DV + D), BS (M = 64) 2SP
  static constexpr int C_MT = 0, C_DK = 0, C_GT = 128, C_VB = 256, C_DV = 256 + 2 * SP,
                       C_BS = C_DV + D;
  static_assert(C_BS + 2 * SP <= TCOLS, "tensor-memory columns");
  static_assert(2 * TT * D <= TT * TT, "dv and dk staging inside the masked-matrix area");
  static_assert(MM % 256 == 0, "1 KB aligned TMA boxes");
  static_assert(FLOATS * 4 <= 227 * 1024, "shared memory");
};

// maps: 0 projQ, 1 projK, 2 v, 3 dO, 5 dk, 6 dv; alpha is read directly
template <typename T, int D, int SPAD, int K>
__global__ void __launch_bounds__(TT * BwdKVLayC<D, SPAD>::NTH, 1)
    k_c5_bwd_kv(const Params prm, const __grid_constant__ TmaMaps maps) {
  using LY = BwdKVLayC<D, SPAD>;
  constexpr int SP = LY::SP, NTH = LY::NTH, NTHR = TT * NTH, W = D / NTH;
  using G = Groups<K>;
  constexpr int NG = SP / G::GB;
  constexpr int MYG = (NG + NTH - 1) / NTH;
  constexpr int GC = TT / NTH;
  constexpr bool F32 = sizeof(T) == 4;
  // bf16 inputs: pK, W, BS, the masked MT / GT and dproj as one bf16 part
  // each (the path's bf16 tolerance); fp32: two
  constexpr bool ONE = !F32;
  constexpr int KP = ONE ? SP : 2 * SP;                // K / N extent of the bucket products
  constexpr bool DIRECT = ONE && D == 64;              // landed v / dO tiles are MMA operands
  T5_PROLOGUE
  (void)cur_n;
  bf16* pk = reinterpret_cast<bf16*>(sm + LY::PK);
  bf16* wh = reinterpret_cast<bf16*>(sm + LY::WH);
  bf16* wl = reinterpret_cast<bf16*>(sm + LY::WL);
  bf16* bss = reinterpret_cast<bf16*>(sm + LY::BSS);
  bf16* dj = reinterpret_cast<bf16*>(sm + LY::DJ);
  bf16* pt = reinterpret_cast<bf16*>(sm + LY::PT);
  float* bsf = sm + LY::BSF;
  double* as = reinterpret_cast<double*>(sm + LY::AS);
  double* a0t = reinterpret_cast<double*>(sm + LY::A0T);
  float* scan = sm + LY::SCAN;
  float* scan2 = sm + LY::SCAN2;
  const int lane = tid & 31, quad = warp & 3;
  const int64_t tiles_n = (prm.T + TT - 1) / TT;
  for (int i = tid; i < TT * PJ; i += NTHR) reinterpret_cast<float*>(dj)[i] = 0.f;

  // BS operand from BS values x(s, d): rows s (hi) and SP + s (lo), column d
  // (K-major B of v . BS^T, MN-major B of pK . BS)
  auto put_bs = [&](int s2, int d, float x) {
    const bf16 h = __float2bfloat16_rn(x);
    bss[elem<D>(s2, d)] = h;
    if constexpr (!ONE) bss[elem<D>(SP + s2, d)] = __float2bfloat16_rn(x - __bfloat162float(h));
  };

  for (int w = blockIdx.x; w < items && !failed; w += gridDim.x) {
    const Item it = item_of(prm, w);
    const int n = it.n;
    float ds = 0.f;
    if (it.ntiles > 0) {
      const int m = prm.Mp == 1 ? 0 : n / (prm.B * prm.H);
      __syncthreads();
      if (m != cur_m) {
        const float* pl = prm.planes + (size_t)m * prm.LK * D;
        put_stack<D, PJ, 2, NTHR>(pt, [&](int d, int j) { return j < prm.LK ? pl[j * D + d] : 0.f; });
        cur_m = m;
      }
      const float* gs = prm.gstate_in + ((size_t)n * prm.P + it.part) * prm.SS;
      for (int e = tid; e < SP * D; e += NTHR) bsf[e] = e / D < prm.S ? gs[e] : 0.f;
      for (int s2 = tid; s2 < SP; s2 += NTHR) as[s2] = s2 < prm.S ? (double)gs[prm.S * D + s2] : 0.0;
      __syncthreads();
      for (int e = tid; e < SP * D; e += NTHR) put_bs(e / D, e % D, bsf[e]);
      auto tile_t0 = [&](int j) { return it.t0 + (int64_t)(it.ntiles - 1 - j) * TT; };
      auto load_v = [&](int j) {   // v and the projections of walk step j
        if (failed) return;
        inflight |= 1u;
        if (tid == 0) {
          const int64_t t0 = tile_t0(j);
          float* pj = sm + LY::PJX;
          fence_async_smem();
          bar_expect_tx(full, (uint32_t)(Box<T, D>::BYTES + 2 * TT * PJ * 4));
          tma_load3(pj, &maps.map[0], 0, (int)t0, n, full);
          tma_load3(pj + TT * PJ, &maps.map[1], 0, (int)t0, n, full);
          tma_rows5<T, D>(&maps.map[2], sm + LY::VX, prm.lv, prm, n, t0, full);
        }
      };
      auto load_do = [&](int j) {
        if (failed) return;
        inflight |= 2u;
        if (tid == 0) {
          fence_async_smem();
          bar_expect_tx(full + 1, (uint32_t)Box<T, D>::BYTES);
          tma_rows5<T, D>(&maps.map[3], sm + LY::GX, prm.ldo, prm, n, tile_t0(j), full + 1);
        }
      };
      load_v(0);
      load_do(0);
      for (int i = 0; i < it.ntiles; ++i) {
        const int64_t tile0 = tile_t0(i);
        float* VXt = sm + LY::VX;
        float* GXt = sm + LY::GX;
        const float* pj = sm + LY::PJX;
        if (tid < SP) a0t[tid] = prm.range_mass[((size_t)n * tiles_n + tile0 / TT) * SP + tid];
        // the tile's alpha rows from global memory, issued before the waits so
        // their latency overlaps the copies in flight
        float alr[MYG][G::GB];
        {
          const int64_t ta = tile0 + row;
          const bool va = ta < it.t1;
          const float* arow = prm.alpha + ((size_t)n * prm.T + (va ? ta : 0)) * prm.SA;
#pragma unroll
          for (int a = 0; a < MYG; ++a) {
            const int gi = sub + a * NTH;
#pragma unroll
            for (int b = 0; b < G::GB; ++b) {
              const int s2 = gi * G::GB + b;
              alr[a][b] = (gi < NG && va && s2 < prm.S) ? __ldg(arow + s2) : 0.f;
            }
          }
        }
        T5_WAIT(full, phF & 1);
        if (!failed) {
          phF ^= 1u;
          inflight &= ~1u;
        }
        T5_WAIT(full + 1, (phF >> 1) & 1);
        if (!failed) {
          phF ^= 2u;
          inflight &= ~2u;
        }
        const int64_t t = tile0 + row;
        const bool valid = t < it.t1;
        float pkv[MYG][G::GB], hk[MYG][G::GK], asf[MYG][G::GB], wv[MYG][G::GB];
        {
          float y[W], g[W];
          if constexpr (!DIRECT) {
            read_cols<T, D, W>(VXt, row, sub * W, y);
            read_cols<T, D, W>(GXt, row, sub * W, g);
          }
          float pq[MYG][G::GB], al[MYG][G::GB];
#pragma unroll
          for (int a = 0; a < MYG; ++a) {
            const int gi = sub + a * NTH;
            if (gi < NG) {
              float pj_[G::GK], h[G::GK];
              const bool has = gi * G::GK < PJ;
#pragma unroll
              for (int k = 0; k < G::GK; ++k) pj_[k] = has ? pj[row * PJ + gi * G::GK + k] : 0.f;
              group_probs<K>(pj_, gi * G::GT, has ? L : 0, inv_scale, pq[a], h);
#pragma unroll
              for (int k = 0; k < G::GK; ++k)
                pj_[k] = has ? pj[TT * PJ + row * PJ + gi * G::GK + k] : 0.f;
              group_probs<K>(pj_, gi * G::GT, has ? L : 0, inv_scale, pkv[a], hk[a]);
#pragma unroll
              for (int b = 0; b < G::GB; ++b) al[a][b] = alr[a][b];
              if (!valid) {
#pragma unroll
                for (int b = 0; b < G::GB; ++b) pq[a][b] = pkv[a][b] = 0.f;
              }
            }
          }
          __syncthreads();   // raw tiles read, the tile's key mass loaded, scratch free
          if constexpr (!DIRECT) {
            put_cols<D, W, F32 ? 2 : 1>(Slot<D>::part(VXt, 0), Slot<D>::part(VXt, 1), nullptr, row,
                                        sub * W, y);
            put_cols<D, W, F32 ? 2 : 1>(Slot<D>::part(GXt, 0), Slot<D>::part(GXt, 1), nullptr, row,
                                        sub * W, g);
          }
          float incl[MYG][G::GB], rincl[MYG][G::GB];
#pragma unroll
          for (int a = 0; a < MYG; ++a) {
            const int gi = sub + a * NTH;
            if (gi < NG) {
#pragma unroll
              for (int b = 0; b < G::GB; ++b) {
                float tot;
                incl[a][b] = warp_scan(pkv[a][b], tot);
                if (lane == 31) scan[(gi * G::GB + b) * 4 + quad] = tot;
                // suffix of alpha over the warp's tokens
                float x = al[a][b];
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                  const float yv = __shfl_down_sync(0xffffffffu, x, o);
                  if (lane + o < 32) x += yv;
                }
                rincl[a][b] = x;
                const float rt = __shfl_sync(0xffffffffu, x, 0);
                if (lane == 0) scan2[(gi * G::GB + b) * 4 + quad] = rt;
              }
            }
          }
          __syncthreads();
          float am[MYG][G::GB], dpart = 0.f;
#pragma unroll
          for (int a = 0; a < MYG; ++a) {
            const int gi = sub + a * NTH;
            if (gi < NG) {
#pragma unroll
              for (int b = 0; b < G::GB; ++b) {
                const int s2 = gi * G::GB + b;
                float before = 0.f, after = 0.f;
                for (int q2 = 0; q2 < quad; ++q2) before += scan[s2 * 4 + q2];
                for (int q2 = quad + 1; q2 < 4; ++q2) after += scan2[s2 * 4 + q2];
                am[a][b] = (float)(a0t[s2] + (double)(before + incl[a][b]));
                dpart = fmaf(pq[a][b], am[a][b], dpart);
                asf[a][b] = (float)(as[s2] + (double)(after + rincl[a][b]));
              }
            }
          }
          float rden = 0.f;   // global mode: W_s = pQ_s / max(den, eps)
          if (prm.global_norm)
            rden = 1.f / fmaxf(token_sum<NTH>(dpart, sm + LY::DENX, row, sub), prm.eps);
#pragma unroll
          for (int a = 0; a < MYG; ++a) {
            const int gi = sub + a * NTH;
            if (gi < NG) {
#pragma unroll
              for (int b = 0; b < G::GB; ++b)
                wv[a][b] = prm.global_norm ? pq[a][b] * rden : __fdividef(pq[a][b], am[a][b] + prm.eps);
#pragma unroll
              for (int c8 = 0; c8 < G::GB / 8; ++c8) {
                const int c = gi * G::GB / 8 + c8;
                put_parts8<2 * SP, SP / 8, ONE>(pk, row, c, pkv[a] + 8 * c8);
                if constexpr (ONE) {
                  uint4 hi;
                  cvt8(wv[a] + 8 * c8, hi);
                  put_chunk<2 * SP>(wh, row, c, hi);
                } else {
                  uint4 hi, lo;
                  split8(wv[a] + 8 * c8, hi, lo);
                  put_chunk<2 * SP>(wh, row, c, hi);
                  put_chunk<2 * SP>(wh, row, SP / 8 + c, hi);
                  put_chunk<SP>(wl, row, c, lo);
                }
              }
            }
          }
        }
        fence_async_smem();
        fence_before();
        __syncthreads();
        if (tid == 0 && !failed) {
          fence_after();
          bulk_wait_read();   // the previous tile's dv / dk staging sits in MM
          const bf16* vp[2] = {Slot<D>::part(VXt, 0), Slot<D>::part(VXt, 1)};
          const bf16* gp[2] = {Slot<D>::part(GXt, 0), Slot<D>::part(GXt, 1)};
          // MT[tau][t] = v(tau) . dO(t)
#pragma unroll
          for (int a = 0; a < 2; ++a)
#pragma unroll
            for (int b = 0; b < 2; ++b) {
              if (a + b == 2 || (!F32 && a + b > 0)) continue;
#pragma unroll
              for (int ks = 0; ks < D / 16; ++ks)
                mma(tbase + LY::C_MT, desc_a_k<D, DIRECT>(vp[a], ks), desc_a_k<D, DIRECT>(gp[b], ks),
                    idesc<TT>(), a + b > 0 || ks > 0);
            }
          // GT[tau][t] = pK(tau) . W(t)
#pragma unroll
          for (int ks = 0; ks < KP / 16; ++ks)
            mma(tbase + LY::C_GT, desc<2 * SP>(pk, ks), desc<2 * SP>(wh, ks), idesc<TT>(), ks > 0);
          if constexpr (!ONE) {
#pragma unroll
            for (int ks = 0; ks < SP / 16; ++ks)
              mma(tbase + LY::C_GT, desc<2 * SP>(pk, ks), desc<SP>(wl, ks), idesc<TT>(), true);
          }
          // VB = v . BS^T (BS hi and lo along N)
#pragma unroll
          for (int a = 0; a < (F32 ? 2 : 1); ++a)
#pragma unroll
            for (int ks = 0; ks < D / 16; ++ks)
              mma(tbase + LY::C_VB, desc_a_k<D, DIRECT>(vp[a], ks), desc<D>(bss, ks), idesc<KP>(),
                  a > 0 || ks > 0);
          // DV = pK . BS (hi.hi, lo.hi, hi.lo; BS rows read MN-major)
#pragma unroll
          for (int ks = 0; ks < SP / 16; ++ks) {
            mma(tbase + LY::C_DV, desc<2 * SP>(pk, ks), desc_mn<D>(bss, ks), idesc_bmn<D>(), ks > 0);
            if constexpr (!ONE) {
              mma(tbase + LY::C_DV, desc<2 * SP>(pk, SP / 16 + ks), desc_mn<D>(bss, ks),
                  idesc_bmn<D>(), true);
              mma(tbase + LY::C_DV, desc<2 * SP>(pk, ks), desc_mn<D>(bss, SP / 16 + ks),
                  idesc_bmn<D>(), true);
            }
          }
          // BS[d][s] += dO^T W over the range (block 0: W hi, block 1: W lo)
#pragma unroll
          for (int a = 0; a < (F32 ? 2 : 1); ++a)
#pragma unroll
            for (int ks = 0; ks < TT / 16; ++ks) {
              mma(tbase + LY::C_BS, desc_a_mn<D, DIRECT>(gp[a], ks), desc_mn<2 * SP>(wh, ks),
                  idesc64_mn<SP>(), i > 0 || a > 0 || ks > 0);
              if (!ONE && a == 0)
                mma(tbase + LY::C_BS + SP, desc_mn<D>(gp[a], ks), desc_mn<SP>(wl, ks),
                    idesc64_mn<SP>(), i > 0 || ks > 0);
            }
          { commit(barA); ++issA; }
        }
        // the tile's alpha moves the suffix on (every thread has read `as`)
        if (sub == 0 && tid < SP) {
          float tot = 0.f;
          for (int q2 = 0; q2 < 4; ++q2) tot += scan2[tid * 4 + q2];
          as[tid] += (double)tot;
        }
        T5_WAIT(barA, phA);
        phA ^= 1;
        // v and the projections are consumed: the next walk step's
        if (i + 1 < it.ntiles) load_v(i + 1);
        fence_after();
        {
          // masked MT and GT rows (t >= tau kept) as packed bf16 parts over the
          // thread's own columns -- hi in the first half, lo (fp32 inputs) in
          // the second -- so no other thread's reads are in the way
          uint32_t mh[GC / 2], ml[GC / 2], gh[GC / 2], gl[GC / 2];
#pragma unroll
          for (int c0 = 0; c0 < GC; c0 += 16) {
            float g[16], h[16];
            tld16(tlane + LY::C_MT + GC * sub + c0, g);
            tld16(tlane + LY::C_GT + GC * sub + c0, h);
            tld_wait();
#pragma unroll
            for (int e = 0; e < 16; e += 2) {
              const bool k0 = GC * sub + c0 + e >= row, k1 = GC * sub + c0 + e + 1 >= row;
              const float m0 = k0 ? g[e] : 0.f, m1 = k1 ? g[e + 1] : 0.f;
              const float g0 = k0 ? h[e] : 0.f, g1 = k1 ? h[e + 1] : 0.f;
              if constexpr (ONE) {
                __nv_bfloat162 x = __floats2bfloat162_rn(m0, m1);
                mh[(c0 + e) / 2] = *reinterpret_cast<const uint32_t*>(&x);
                x = __floats2bfloat162_rn(g0, g1);
                gh[(c0 + e) / 2] = *reinterpret_cast<const uint32_t*>(&x);
              } else {
                split2(m0, m1, mh[(c0 + e) / 2], ml[(c0 + e) / 2]);
                split2(g0, g1, gh[(c0 + e) / 2], gl[(c0 + e) / 2]);
              }
            }
          }
#pragma unroll
          for (int c = 0; c < GC / 2; c += 8) {
            uint32_t x8[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) x8[e] = mh[c + e];
            tst8(tlane + LY::C_MT + GC * sub + c, x8);
#pragma unroll
            for (int e = 0; e < 8; ++e) x8[e] = gh[c + e];
            tst8(tlane + LY::C_GT + GC * sub + c, x8);
            if constexpr (!ONE) {
#pragma unroll
              for (int e = 0; e < 8; ++e) x8[e] = ml[c + e];
              tst8(tlane + LY::C_MT + GC * sub + GC / 2 + c, x8);
#pragma unroll
              for (int e = 0; e < 8; ++e) x8[e] = gl[c + e];
              tst8(tlane + LY::C_GT + GC * sub + GC / 2 + c, x8);
            }
          }
          tst_wait();
        }
        fence_before();
        __syncthreads();
        if (tid == 0 && !failed) {
          fence_after();
          const bf16* gp[2] = {Slot<D>::part(GXt, 0), Slot<D>::part(GXt, 1)};
          // VB += mask'(MT) . W  (block 0: W hi, block 1: W lo; lo.lo dropped)
#pragma unroll
          // part a of the masked MT / GT for tokens [GC j, GC j + GC): columns GC j + a GC / 2 + ...
#pragma unroll
          for (int a2 = 0; a2 < (ONE ? 1 : 2); ++a2)
#pragma unroll
            for (int ks = 0; ks < TT / 16; ++ks) {
              const uint32_t col = GC * (16 * ks / GC) + a2 * (GC / 2) + (16 * ks % GC) / 2;
              // VB += mask'(MT) . W  (block 0: W hi, block 1: W lo; lo.lo dropped)
              mma_ta(tbase + LY::C_VB, tbase + LY::C_MT + col, desc_mn<2 * SP>(wh, ks),
                     idesc_bmn<SP>(), true);
              if (!ONE && a2 == 0)
                mma_ta(tbase + LY::C_VB + SP, tbase + LY::C_MT + col, desc_mn<SP>(wl, ks),
                       idesc_bmn<SP>(), true);
              // DV += mask'(GT) . dO  (lo.lo dropped)
#pragma unroll
              for (int b2 = 0; b2 < (ONE ? 1 : 2); ++b2)
                if (a2 + b2 < 2)
                  mma_ta(tbase + LY::C_DV, tbase + LY::C_GT + col, desc_a_mn<D, DIRECT>(gp[b2], ks),
                         idesc_bmn<D>(), true);
            }
          { commit(barB); ++issB; }
        }
        T5_WAIT(barB, phB);
        phB ^= 1;
        // dO is consumed: the next walk step's
        if (i + 1 < it.ntiles) load_do(i + 1);
        fence_after();
        // dpK and the hash backward of the keys
#pragma unroll 1
        for (int a = 0; a < MYG; ++a) {
          const int gi = sub + a * NTH;
          if (gi < NG) {
            float vb[G::GB], dpk[G::GB], dj_[G::GK];
            tld_sum<G::GB, ONE ? 1 : 2>(tlane + LY::C_VB + gi * G::GB, SP, vb);
#pragma unroll
            for (int b = 0; b < G::GB; ++b) dpk[b] = valid ? asf[a][b] + vb[b] : 0.f;
            float dsl = 0.f;
            group_probs_bwd<K>(pkv[a], dpk, hk[a], inv_scale, dj_, dsl);
            if (valid) ds += dsl;
            if (gi * G::GK < PJ) {
#pragma unroll
              for (int j = 0; j < G::GK; ++j) {
                const int jj = gi * G::GK + j;
                if (jj < PJ) {
                  const float x = valid ? dj_[j] : 0.f;
                  const bf16 hb = __float2bfloat16_rn(x);
                  dj[elem<PJ>(row, jj)] = hb;
                  if constexpr (!ONE)
                    dj[TT * PJ + elem<PJ>(row, jj)] = __float2bfloat16_rn(x - __bfloat162float(hb));
                }
              }
            }
          }
        }
        fence_async_smem();
        fence_before();
        __syncthreads();
        if (tid == 0 && !failed) {
          fence_after();
          // DK = dproj . P (into the consumed MT columns)
          gemm_parts<D, 2, PJ / 16, PJ, PJ>(tbase + LY::C_DK, dj, dj + TT * PJ, nullptr,
                                            ONE ? 1 : 2, pt, false);
          { commit(barA); ++issA; }
        }
        T5_WAIT(barA, phA);
        phA ^= 1;
        fence_after();
        {
          float o[W];
          tld_sum<W, 1>(tlane + LY::C_DV + sub * W, 0, o);
          put_tile_cols<T, D, W>(sm + LY::MM, row, sub * W, o);
          tld_sum<W>(tlane + LY::C_DK + sub * W, D, o);
          put_tile_cols<T, D, W>(sm + LY::MM + TT * D, row, sub * W, o);
        }
        // BS operands of the next (earlier) tile: range-end suffix + the
        // tiles walked so far (M = 64 lanes: row d = 16 q + l)
        if (i + 1 < it.ntiles) {   // the NTH warps of a lane quarter take every NTH-th chunk
          const int d = 16 * quad + lane;
          for (int s8 = sub; s8 < SP / 8; s8 += NTH) {
            float lo8[8] = {}, v[8];
            tld8(tlane + LY::C_BS + 8 * s8, v);
            if constexpr (!ONE) tld8(tlane + LY::C_BS + SP + 8 * s8, lo8);
            tld_wait();
            if (lane < 16 && d < D) {
#pragma unroll
              for (int e = 0; e < 8; ++e)
                put_bs(8 * s8 + e, d, bsf[(8 * s8 + e) * D + d] + v[e] + lo8[e]);
            }
          }
        }
        fence_async_smem();
        fence_before();
        __syncthreads();
        if (tid == 0 && !failed) {
          tma_store_tile<T, D>(&maps.map[6], sm + LY::MM, prm.ldv, prm, n, tile0);
          tma_store_tile<T, D>(&maps.map[5], sm + LY::MM + TT * D, prm.ldk, prm, n, tile0);
          bulk_commit();
        }
        if (T5_VOTE()) break;
      }
    }
    float x = ds;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    __syncthreads();
    if ((tid & 31) == 0) sm[LY::RED + warp] = x;
    __syncthreads();
    if (tid == 0) {
      float tot = 0.f;
      for (int i = 0; i < NTHR / 32; ++i) tot += sm[LY::RED + i];
      prm.dscale_part[(size_t)n * prm.P + it.part] = tot;
    }
  }
  T5_EPILOGUE
}

#undef T5_WAIT
#undef T5_VOTE
#undef T5_PROLOGUE
#undef T5_EPILOGUE
#undef T5_STAGE_DRAIN

}  // namespace c5
}  // namespace race
