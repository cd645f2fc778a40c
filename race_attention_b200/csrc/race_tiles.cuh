// race_tiles.cuh -- staging of token tiles into shared memory.
//
// A CTA walks a contiguous range of tiles of one stream.  The q/k/v/dO rows of
// the next tile are brought into padded shared-memory rows with cp.async
// while the current tile is computed (two stages; bf16 rows are staged raw
// and widened to fp32 once per tile), so HBM streaming overlaps the
// arithmetic.  Rows past the range are zero-filled.
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

// Hardware approximate reciprocal (one MUFU op, relative error ~2^-23);
// the hash only takes it of 1 + e with e in [0, 1].
__device__ __forceinline__ float rcp_approx(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// tanh(x) = sign(x) (1 - e) / (1 + e), e = exp(-2|x|) (the exponential
// identity of the hyperbolic tangent); absolute error ~1e-7, which is all the
// soft hash needs since it only uses tanh(x)/scale as a logit.
__device__ __forceinline__ float tanh_exp(float x) {
  const float e = __expf(-2.f * fabsf(x));
  const float t = (1.f - e) * rcp_approx(1.f + e);
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

}  // namespace tiles
}  // namespace race
