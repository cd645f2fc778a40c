// race_t5.cuh -- non-causal readout and key/value backward on the 5th-generation
// tensor cores (tcgen05 + tensor memory).
//
// NTH threads per token: a CTA of 128 NTH threads walks 128-token tiles; every
// token-major product (projections x.P^T, readout pQ.E, key-side dpK = v.dB^T,
// dv = pK.dB, dk = dproj.P) is an M = 128 tcgen05.mma chain issued by one
// thread, both operands in shared memory, fp32 accumulators in tensor memory.
// Row t of an accumulator is TMEM lane t, so after a tcgen05.ld the threads
// of token t hold its row and the hash arithmetic (tanh, corner
// probabilities and their backward) runs in registers: thread (t, sub) owns
// columns [sub W, sub W + W) of every row-wise pass (W = D / NTH) and every
// NTH-th group of buckets of the hash.
//
// Precision: split bf16.  Every fp32 operand x is held as two bf16 parts,
// hi = bf16(x) and lo = bf16(x - hi) (16 significant bits; the remainder is
// below 2^-17 |x|), and each product is hi.hi + lo.hi + hi.lo + lo.lo with
// fp32 accumulation: relative error ~1e-6, inside the path's 1e-4.  The
// key-side dpK = v . dB^T uses three parts (hi, mid, lo: 24 bits) on both
// sides, because it cancels against dA where a bucket holds few tokens.  bf16
// inputs are exact in hi, so their other parts are skipped.  (kind::f16 is chosen over
// kind::tf32 because one M = 128 instruction costs ~100 cycles for K = 16 bf16
// against 150-300 for K = 8 tf32, largely independent of N; the B operands'
// hi and lo parts are therefore stacked along N so each A tile streams once
// per K step.)
//
// Operand layout (K-major, no swizzle): element (r, c) of an operand with C
// columns is bf16 number (r/8)*8C + (c/8)*64 + (r%8)*8 + c%8 -- 8-row x 16-byte
// core matrices; descriptor leading offset 128 B (next 8 columns), stride
// offset 16C B (next 8 rows); a K = 16 step advances the start by 256 B.
// fp32 tiles land by TMA (box layout, see Box below) and are converted in
// place to their bf16 parts.
#pragma once

#include <cuda_bf16.h>

#include "race_kernels.cuh"
#include "race_tiles.cuh"

namespace race {
namespace t5 {

using bf16 = __nv_bfloat16;

constexpr int TT = 128;   // tokens per tile = MMA M = TMEM lanes
constexpr int PJ = 16;    // projection columns (L*K <= 16)
constexpr int kWaitPolls = 1 << 22;   // polls of the drain waits after a timeout
constexpr unsigned kErrTimeout = 1u;  // status bit: a main-loop wait ran out (RACE_DEV_TIMEOUT)
constexpr unsigned kErrStuck = 2u;    // status bit: in-flight work did not drain (RACE_DEV_STUCK)

__device__ __forceinline__ uint32_t saddr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte chunk (r, c8) -- columns 8 c8 .. 8 c8 + 7 of row r -- of an operand with C columns
template <int C>
__device__ __forceinline__ int chunk(int r, int c8) {
  return (r >> 3) * C + c8 * 8 + (r & 7);
}
// bf16 index of element (r, c)
template <int C>
__device__ __forceinline__ int elem(int r, int c) {
  return (r >> 3) * (8 * C) + (c >> 3) * 64 + (r & 7) * 8 + (c & 7);
}

// shared-memory matrix descriptor of K step ks (16 columns) of an operand with C columns
template <int C>
__device__ __forceinline__ uint64_t desc(const void* base, int ks) {
  const uint32_t a = saddr(base) + ks * 256;
  uint64_t d = (uint64_t)((a >> 4) & 0x3fff);
  d |= (uint64_t)(128 >> 4) << 16;                   // leading byte offset: next 8 columns
  d |= (uint64_t)(((16 * C) >> 4) & 0x3fff) << 32;   // stride byte offset: next 8 rows
  d |= (uint64_t)1 << 46;                            // descriptor version (sm_100)
  return d;
}

// instruction descriptor: kind::f16 with bf16 A and B, fp32 accumulate, K-major, M = 128
template <int N>
__host__ __device__ constexpr uint32_t idesc() {
  static_assert(N % 16 == 0 && N >= 16 && N <= 256, "M = 128 needs N % 16 == 0, N <= 256");
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ void mma(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t id,
                                    bool acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(id), "r"((uint32_t)acc));
}

// Contractions over the tokens of a tile read the token-major operands
// directly as MN-major operands (rows of the result along the columns C of
// the operand, K along its tokens): 8-column blocks 128 B apart (stride byte
// offset), 8-token blocks 16C B apart (leading byte offset); a K = 16 step
// advances the start by 32C B.
template <int C>
__device__ __forceinline__ uint64_t desc_mn(const void* base, int ks) {
  const uint32_t a = saddr(base) + ks * 32 * C;
  uint64_t d = (uint64_t)((a >> 4) & 0x3fff);
  d |= (uint64_t)(((16 * C) >> 4) & 0x3fff) << 16;   // leading byte offset: next 8 tokens
  d |= (uint64_t)(128 >> 4) << 32;                   // stride byte offset: next 8 columns
  d |= (uint64_t)1 << 46;
  return d;
}
// instruction descriptor, M = 64, both operands MN-major (accumulator row m
// in TMEM lane 32 (m/16) + m%16)
template <int N>
__host__ __device__ constexpr uint32_t idesc64_mn() {
  static_assert(N % 8 == 0 && N >= 8 && N <= 256, "M = 64 needs N % 8 == 0, N <= 256");
  return (1u << 4) | (1u << 7) | (1u << 10) | (1u << 15) | (1u << 16) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(64 >> 4) << 24);
}

// Landed bf16 tiles used in place (D = 64: one 128-byte row per token, the
// copy engine's 128-byte swizzle, 1 KB aligned slots).  K-major: the row is
// the K axis and fits one swizzle atom, 8-row groups 1024 B apart (stride
// byte offset), a K = 16 step moves the start 32 B inside the atom.
__device__ __forceinline__ uint64_t desc_sw128(const void* base, int ks) {
  const uint32_t a = saddr(base) + ks * 32;
  uint64_t d = (uint64_t)((a >> 4) & 0x3fff);
  d |= (uint64_t)1 << 16;                  // leading byte offset (unused inside one atom)
  d |= (uint64_t)(1024 >> 4) << 32;        // stride byte offset: next 8 rows
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;                  // 128-byte swizzle
  return d;
}
// MN-major: the row holds the 64 MN elements (one atom), K runs over the
// tokens; 8-token groups 1024 B apart (stride byte offset), a K = 16 step is
// 16 rows = 2048 B.
__device__ __forceinline__ uint64_t desc_sw128_mn(const void* base, int ks) {
  const uint32_t a = saddr(base) + ks * 2048;
  uint64_t d = (uint64_t)((a >> 4) & 0x3fff);
  d |= (uint64_t)1 << 16;                  // leading byte offset (one atom along MN)
  d |= (uint64_t)(1024 >> 4) << 32;        // stride byte offset: next 8 tokens
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}
// K-major operand with C columns: a converted part, or (SW) the landed tile
template <int C, bool SW>
__device__ __forceinline__ uint64_t desc_a_k(const void* base, int ks) {
  if constexpr (SW) {
    return desc_sw128(base, ks);
  } else {
    return desc<C>(base, ks);
  }
}
// MN-major operand over a tile's tokens: a converted part, or (SW) the landed tile
template <int C, bool SW>
__device__ __forceinline__ uint64_t desc_a_mn(const void* base, int ks) {
  if constexpr (SW) {
    return desc_sw128_mn(base, ks);
  } else {
    return desc_mn<C>(base, ks);
  }
}

// Split product D = A . B^T with K = 16 KS.  A is given as NA bf16 parts
// (a[0] + a[1] + ..., the later ones nullptr-free), B as BP parts stacked
// along its rows ([B0; B1; ...], BP*N rows).  Column block j of D receives
// sum_i A_i . B_j^T -- every part product, since an instruction costs the
// same at N and BP*N.  The caller adds the BP column blocks.
// SW: A is one landed bf16 tile read in place (desc_sw128).
template <int N, int BP, int KS, int CA, int CB, bool SW = false>
__device__ __forceinline__ void gemm_parts(uint32_t d, const bf16* a0, const bf16* a1,
                                           const bf16* a2, int na, const bf16* b, bool acc) {
  if constexpr (SW) {
#pragma unroll
    for (int ks = 0; ks < KS; ++ks)
      mma(d, desc_sw128(a0, ks), desc<CB>(b, ks), idesc<BP * N>(), acc || ks > 0);
  } else {
    const bf16* a[3] = {a0, a1, a2};
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      if (i < na) {
#pragma unroll
        for (int ks = 0; ks < KS; ++ks)
          mma(d, desc<CA>(a[i], ks), desc<CB>(b, ks), idesc<BP * N>(), acc || i > 0 || ks > 0);
      }
    }
  }
}

__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   saddr(bar))
               : "memory");
}
__device__ __forceinline__ void fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// makes generic-proxy shared-memory writes (st.shared, cp.async) visible to the tensor core
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void bar_init(uint64_t* bar) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(saddr(bar)));
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
// Waits for phase `parity` of the barrier with a bounded number of polls.
// With an abort word: gives up early once another thread has set it, and
// sets it when its own polls run out.
__device__ __forceinline__ bool bar_try(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(saddr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Non-blocking probe of the same phase (try_wait may suspend the thread for a
// hardware-defined interval; this never does).
__device__ __forceinline__ bool bar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(saddr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool bar_wait(uint64_t* bar, uint32_t parity) {
  for (int i = 0; i < kWaitPolls; ++i)
    if (bar_try(bar, parity)) return true;
  return false;
}
__device__ __forceinline__ bool bar_wait(uint64_t* bar, uint32_t parity, volatile uint32_t* abort,
                                         int polls) {
  if (polls < 64) {   // a short bound (the timeout test) counts non-blocking probes
    for (int i = 0; i < polls; ++i)
      if (bar_test(bar, parity)) return true;
    *abort = 1;
    return false;
  }
  for (int i = 0; i < polls; ++i) {
    if (bar_try(bar, parity)) return true;
    if ((i & 63) == 63 && *abort != 0) return false;
  }
  *abort = 1;
  return false;
}

// 16 consecutive fp32 columns of this thread's TMEM lane
__device__ __forceinline__ void tld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tld8(uint32_t taddr, float* v) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tld4(uint32_t taddr, float* v) {
  uint32_t r[4];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tld1(uint32_t taddr, float& v) {
  uint32_t r;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr));
  v = __uint_as_float(r);
}
__device__ __forceinline__ void tld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// C columns (C % 8 == 0) of this lane as the sum of BP column blocks
// [taddr + j off, taddr + j off + C)
template <int C, int BP = 2>
__device__ __forceinline__ void tld_sum(uint32_t taddr, int off, float* out) {
  float v[BP][C];
#pragma unroll
  for (int j = 0; j < BP; ++j)
#pragma unroll
    for (int c = 0; c < C; c += 8) tld8(taddr + j * off + c, &v[j][c]);
  tld_wait();
#pragma unroll
  for (int c = 0; c < C; ++c) {
    float x = v[0][c];
#pragma unroll
    for (int j = 1; j < BP; ++j) x += v[j][c];
    out[c] = x;
  }
}

// The GK projection columns [c0, c0 + GK) of this lane, summed over NB
// column blocks PJ apart (c0 may vary at run time; warp-uniform).
template <int GK, int NB>
__device__ __forceinline__ void tld_group(uint32_t taddr, int c0, float (&out)[GK]) {
  float v[NB][GK];
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    if constexpr (GK % 4 == 0) {   // c0 is then a multiple of 4: x4 loads
#pragma unroll
      for (int k = 0; k < GK; k += 4) tld4(taddr + b * PJ + c0 + k, &v[b][k]);
    } else {
#pragma unroll
      for (int k = 0; k < GK; ++k) tld1(taddr + b * PJ + c0 + k, v[b][k]);
    }
  }
  tld_wait();
#pragma unroll
  for (int k = 0; k < GK; ++k) {
    float x = v[0][k];
#pragma unroll
    for (int b = 1; b < NB; ++b) x += v[b][k];
    out[k] = x;
  }
}

// Conversion barrier.  At D = 64 the in-place conversion of a landed tile
// (box layout -> K-major bf16 parts) moves data only within 8-row groups, so
// only the NTH warps that hold rows [32 q, 32 q + 32) (warps q, q + 4, ...)
// must have read before any of them writes: a named barrier per row quarter
// (ids 1..4) instead of the CTA-wide one.  Other widths cross row groups.
template <int D, int NTH>
__device__ __forceinline__ void convert_sync(int warp) {
  if constexpr (D == 64) {
    asm volatile("bar.sync %0, %1;" ::"r"(1 + (warp & 3)), "n"(32 * NTH) : "memory");
  } else {
    __syncthreads();
  }
}

template <int COLS>
__device__ __forceinline__ void tmem_alloc(uint32_t* slot) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   saddr(slot)),
               "n"(COLS));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
template <int COLS>
__device__ __forceinline__ void tmem_free(uint32_t base) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "n"(COLS));
}

// hi / lo bf16 parts of two floats, packed (the residual with one packed
// fp32x2 fused multiply-add)
__device__ __forceinline__ void split2(float a, float b, uint32_t& hi, uint32_t& lo) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  const float2 r = __ffma2_rn(__bfloat1622float2(h), make_float2(-1.f, -1.f), make_float2(a, b));
  const __nv_bfloat162 l = __float22bfloat162_rn(r);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}

// hi / mid / lo bf16 parts of two floats (24 significant bits), packed
__device__ __forceinline__ void split3(float a, float b, uint32_t& hi, uint32_t& mid, uint32_t& lo) {
  const float2 m1 = make_float2(-1.f, -1.f);
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  const float2 r1 = __ffma2_rn(__bfloat1622float2(h), m1, make_float2(a, b));
  const __nv_bfloat162 m = __float22bfloat162_rn(r1);
  const float2 r2 = __ffma2_rn(__bfloat1622float2(m), m1, r1);
  const __nv_bfloat162 l = __float22bfloat162_rn(r2);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  mid = *reinterpret_cast<const uint32_t*>(&m);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}

// Tiles arrive by TMA: the host maps each streamed input as a 5-D tensor
// (D, T, H, B, M) and a tile is NB boxes of 128 rows x IB bytes (IB = 128 with
// the 128-byte swizzle -- 16-byte chunk c of row r stored at chunk c ^ (r % 8)
// -- or the whole row when it is shorter).  Rows past the tensor's end are
// zero-filled by the copy engine; rows past a range's end are read but never
// written back or counted.
template <typename T, int D>
struct Box {
  static constexpr int RB = D * (int)sizeof(T);      // bytes per row
  static constexpr int IB = RB < 128 ? RB : 128;     // bytes per box row
  static constexpr bool SWZ = IB == 128;
  static constexpr int NB = RB / IB;                 // boxes per tile
  static constexpr int BYTES = TT * RB;              // bytes per tile
};

__device__ __forceinline__ void bar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void tma_load5(void* dst, const CUtensorMap* map, int c0, int c1, int c2,
                                          int c3, int c4, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, "
      "{%2, %3, %4, %5, %6}], [%7];" ::"r"(saddr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4),
      "r"(saddr(bar))
      : "memory");
}

// One thread: loads tile rows [t0, t0 + TT) of stream n of NTS mapped tensors
// into their slots and arms `bar` with the byte count.
// A tensor whose ensemble axis has stride 0 is mapped with one ensemble.
template <typename T, int D, int NTS>
__device__ __forceinline__ void tma_tile(const TmaMaps& maps, float* const (&dst)[NTS],
                                         const Layout* const (&lay)[NTS], const Params& prm,
                                         int n, int64_t t0, uint64_t* bar) {
  using BX = Box<T, D>;
  const int h = n % prm.H, b = (n / prm.H) % prm.B, m = n / (prm.H * prm.B);
  fence_async_smem();
  bar_expect_tx(bar, (uint32_t)(BX::BYTES * NTS));
#pragma unroll
  for (int k = 0; k < NTS; ++k)
#pragma unroll
    for (int x = 0; x < BX::NB; ++x)
      tma_load5(reinterpret_cast<char*>(dst[k]) + x * TT * BX::IB, &maps.map[k],
                x * BX::IB / (int)sizeof(T), (int)t0, h, b, lay[k]->sm == 0 ? 0 : m, bar);
}

// Columns [c0, c0 + W) (c0, W multiples of 16 bytes) of row r of a landed
// tile, as fp32.
template <typename T, int D, int W>
__device__ __forceinline__ void read_cols(const void* tile, int r, int c0, float* x) {
  using BX = Box<T, D>;
  constexpr int EPC = 16 / (int)sizeof(T);
  const char* base = static_cast<const char*>(tile);
#pragma unroll
  for (int i = 0; i < W / EPC; ++i) {
    const int gc = c0 / EPC + i;                       // 16-byte chunk of the row
    const int bx = gc / (BX::IB / 16), c = gc % (BX::IB / 16);
    const int pc = BX::SWZ ? (c ^ (r & 7)) : c;
    const uint4 u =
        *reinterpret_cast<const uint4*>(base + bx * TT * BX::IB + r * BX::IB + pc * 16);
    if constexpr (sizeof(T) == 4) {
      x[4 * i] = __uint_as_float(u.x);
      x[4 * i + 1] = __uint_as_float(u.y);
      x[4 * i + 2] = __uint_as_float(u.z);
      x[4 * i + 3] = __uint_as_float(u.w);
    } else {
      const __nv_bfloat162* hb = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(hb[j]);
        x[8 * i + 2 * j] = f.x;
        x[8 * i + 2 * j + 1] = f.y;
      }
    }
  }
}

// Writes columns [c0, c0 + W) of row r into a tile in the box layout (the
// inverse of read_cols), for a TMA store.
template <typename T, int D, int W>
__device__ __forceinline__ void put_tile_cols(void* tile, int r, int c0, const float* v) {
  using BX = Box<T, D>;
  constexpr int EPC = 16 / (int)sizeof(T);
  char* base = static_cast<char*>(tile);
#pragma unroll
  for (int i = 0; i < W / EPC; ++i) {
    const int gc = c0 / EPC + i;
    const int bx = gc / (BX::IB / 16), c = gc % (BX::IB / 16);
    const int pc = BX::SWZ ? (c ^ (r & 7)) : c;
    uint4 u;
    if constexpr (sizeof(T) == 4) {
      u = make_uint4(__float_as_uint(v[4 * i]), __float_as_uint(v[4 * i + 1]),
                     __float_as_uint(v[4 * i + 2]), __float_as_uint(v[4 * i + 3]));
    } else {
      uint32_t* up = &u.x;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const __nv_bfloat162 b2 = __floats2bfloat162_rn(v[8 * i + 2 * j], v[8 * i + 2 * j + 1]);
        up[j] = *reinterpret_cast<const uint32_t*>(&b2);
      }
    }
    *reinterpret_cast<uint4*>(base + bx * TT * BX::IB + r * BX::IB + pc * 16) = u;
  }
}

__device__ __forceinline__ void tma_store5(const CUtensorMap* map, const void* src, int c0, int c1,
                                           int c2, int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4, %5, %6}], "
      "[%1];" ::"l"(reinterpret_cast<uint64_t>(map)),
      "r"(saddr(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// the shared-memory sources of this thread's bulk stores may be reused
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// this thread's bulk stores are complete
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// One thread: stores a staged tile (box layout) to rows [t0, t0 + TT) of
// stream n of a mapped output.  Ranges are whole tiles, so only the tensor's
// last tile is ragged, and the copy engine clips rows past its end.
template <typename T, int D>
__device__ __forceinline__ void tma_store_tile(const CUtensorMap* map, const void* tile,
                                               const Layout& lay, const Params& prm, int n,
                                               int64_t t0) {
  using BX = Box<T, D>;
  const int h = n % prm.H, b = (n / prm.H) % prm.B, m = n / (prm.H * prm.B);
#pragma unroll
  for (int x = 0; x < BX::NB; ++x)
    tma_store5(map, static_cast<const char*>(tile) + x * TT * BX::IB, x * BX::IB / (int)sizeof(T),
               (int)t0, h, b, lay.sm == 0 ? 0 : m);
}

// Writes W values (columns [c0, c0 + W), W and c0 multiples of 8) of row r
// as NP bf16 parts into operands p0 (, p1, p2) with C columns (NP = 1: the
// values are exact in bf16).
template <int C, int W, int NP>
__device__ __forceinline__ void put_cols(bf16* p0, bf16* p1, bf16* p2, int r, int c0,
                                         const float* v) {
#pragma unroll
  for (int i = 0; i < W / 8; ++i) {
    const int q = chunk<C>(r, c0 / 8 + i);
    uint4 h, m, l;
    uint32_t* hp = &h.x;
    uint32_t* mp = &m.x;
    uint32_t* lp = &l.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float a = v[8 * i + 2 * j], b = v[8 * i + 2 * j + 1];
      if constexpr (NP == 1) {
        const __nv_bfloat162 x = __floats2bfloat162_rn(a, b);
        hp[j] = *reinterpret_cast<const uint32_t*>(&x);
      } else if constexpr (NP == 2) {
        split2(a, b, hp[j], mp[j]);
      } else {
        split3(a, b, hp[j], mp[j], lp[j]);
      }
    }
    reinterpret_cast<uint4*>(p0)[q] = h;
    if constexpr (NP >= 2) reinterpret_cast<uint4*>(p1)[q] = m;
    if constexpr (NP >= 3) reinterpret_cast<uint4*>(p2)[q] = l;
  }
}

// Fills a stacked constant operand [part 0; part 1; ...] of BP*R rows and C
// columns with the BP bf16 parts of f(r, c).
template <int R, int C, int BP, int NTHR, class F>
__device__ __forceinline__ void put_stack(bf16* base, F f) {
  for (int i = threadIdx.x; i < R * C; i += NTHR) {
    const int r = i / C, c = i % C;
    float x = f(r, c);
#pragma unroll
    for (int b = 0; b < BP; ++b) {
      const bf16 h = __float2bfloat16_rn(x);
      base[elem<C>(b * R + r, c)] = h;
      x -= __bfloat162float(h);
    }
  }
}

// Bucket groups of the hash: GB = max(8, R) buckets (GT = GB / R tables, GK =
// GT K planes) -- whole 16-byte chunks of a probability row and whole tables.
template <int K>
struct Groups {
  static constexpr int R = 1 << K;
  static constexpr int GB = R > 8 ? R : 8;
  static constexpr int GT = GB / R;
  static constexpr int GK = GT * K;
};

// Corner probabilities of tables l0 .. l0 + GT - 1 of one token (tables >= L
// give 0); h = tanh of their projections, kept for the backward.
template <int K>
__device__ __forceinline__ void group_probs(const float* proj, int l0, int L, float inv_scale,
                                            float (&p)[Groups<K>::GB], float (&h)[Groups<K>::GK]) {
  constexpr int R = 1 << K, GT = Groups<K>::GT;
#pragma unroll
  for (int u = 0; u < GT; ++u) {
    const bool live = l0 + u < L;
    float sp[K], sn[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const float hh = live ? tiles::tanh_exp(proj[u * K + k]) : 0.f;
      h[u * K + k] = hh;
      const float uu = hh * inv_scale;
      const float ex = __expf(-2.f * fabsf(uu));
      const float rc = tiles::rcp_approx(1.f + ex);
      sp[k] = uu >= 0.f ? rc : ex * rc;
      sn[k] = uu >= 0.f ? ex * rc : rc;
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float v = live ? 1.f : 0.f;
#pragma unroll
      for (int k = 0; k < K; ++k) v *= ((r >> (K - 1 - k)) & 1) ? sp[k] : sn[k];
      p[u * R + r] = v;
    }
  }
}

// Backward of group_probs: g = dL/dp of the group's buckets -> dj = dL/dproj
// of its planes; ds += sum du h.
template <int K>
__device__ __forceinline__ void group_probs_bwd(const float (&p)[Groups<K>::GB],
                                                const float (&g)[Groups<K>::GB],
                                                const float (&h)[Groups<K>::GK], float inv_scale,
                                                float (&dj)[Groups<K>::GK], float& ds) {
  constexpr int R = 1 << K, GT = Groups<K>::GT;
#pragma unroll
  for (int u = 0; u < GT; ++u) {
    float pbar = 0.f;
#pragma unroll
    for (int r = 0; r < R; ++r) pbar = fmaf(p[u * R + r], g[u * R + r], pbar);
    float q[R];
#pragma unroll
    for (int r = 0; r < R; ++r) q[r] = p[u * R + r] * (g[u * R + r] - pbar);
#pragma unroll
    for (int k = 0; k < K; ++k) {
      float du = 0.f;
#pragma unroll
      for (int r = 0; r < R; ++r) du += ((r >> (K - 1 - k)) & 1) ? q[r] : -q[r];
      const float hh = h[u * K + k];
      ds = fmaf(du, hh, ds);
      dj[u * K + k] = du * inv_scale * (1.f - hh * hh);
    }
  }
}

template <typename T, int W>
__device__ __forceinline__ void store_cols(T* dst, const float* v) {
  if constexpr (sizeof(T) == 4) {
    float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
    for (int i = 0; i < W / 4; ++i)
      d4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  } else {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int i = 0; i < W / 8; ++i) {
      uint4 u;
      __nv_bfloat162 b;
      b = __floats2bfloat162_rn(v[8 * i + 0], v[8 * i + 1]); u.x = *reinterpret_cast<uint32_t*>(&b);
      b = __floats2bfloat162_rn(v[8 * i + 2], v[8 * i + 3]); u.y = *reinterpret_cast<uint32_t*>(&b);
      b = __floats2bfloat162_rn(v[8 * i + 4], v[8 * i + 5]); u.z = *reinterpret_cast<uint32_t*>(&b);
      b = __floats2bfloat162_rn(v[8 * i + 6], v[8 * i + 7]); u.w = *reinterpret_cast<uint32_t*>(&b);
      d4[i] = u;
    }
  }
}

// Work items are (stream n, range part) pairs; a persistent CTA takes items
// blockIdx.x, blockIdx.x + gridDim.x, ...
struct Item {
  int n, part;
  int64_t t0, t1;
  int ntiles;
};
__device__ __forceinline__ Item item_of(const Params& prm, int w) {
  Item it;
  it.n = w / prm.P;
  it.part = w % prm.P;
  const tiles::TileRange tr = tiles::tile_range<TT>(prm.T, prm.P, it.part);
  it.t0 = tr.t0;
  it.t1 = tr.t1;
  it.ntiles = tr.ntiles;
  return it;
}

// A tile slot first holds the landed tile (TMA boxes, input type), then --
// converted in place -- NP bf16 operand parts (hi, lo or hi, mid, lo) of TT x D
// each.  Slots are 1 KB aligned (the 128-byte swizzle works in 1 KB atoms).
template <int D, int NP = 2>
struct Slot {
  static constexpr int FLOATS = (TT * D * (NP < 2 ? 2 : NP) / 2 + 255) / 256 * 256;
  __device__ static bf16* part(float* s, int i) { return reinterpret_cast<bf16*>(s) + i * TT * D; }
};

// ------------------------------------------------------------------ layouts (in floats)
template <int D, int SPAD>
struct ReadoutLay {
  static constexpr int NTH = 2;          // threads per token
  static constexpr int SP = (SPAD + 15) / 16 * 16;   // bucket columns (MMA K)
  static constexpr int QX = 0;                        // [2] slots
  static constexpr int PQ = QX + 2 * Slot<D>::FLOATS; // bf16 [TT x SP] hi, then lo
  static constexpr int PS = PQ + TT * SP;             // bf16 [2*PJ x D] planes [hi; lo]
  static constexpr int ET = PS + PJ * D;              // bf16 [2*D x SP] E^T [hi; lo]
  static constexpr int NFULL = 2;                      // tile-landed barriers
  static constexpr int BAR = ET + D * SP;             // mbarriers + TMEM base slot
  static constexpr int FLOATS = BAR + 16 + 256;       // + slack for 1 KB alignment
  static constexpr int TCOLS = 256;                   // PROJ [0, 32), OUT [128, 128 + 2D)
  static constexpr int C_PROJ = 0, C_OUT = 128;
};

// Up to 32 buckets: two k and two v slots (tile i+1 loads as tile i starts);
// above 32 (LATE) one of each, reloaded once dk, dv of tile i-1 have left
// through them.
template <int D, int SPAD>
struct BwdKVLay {
  static constexpr int NTH = 4;           // threads per token
  static constexpr int SP = (SPAD + 15) / 16 * 16;    // bucket columns (MMA K and N)
  static constexpr bool LATE = SP > 32;
  static constexpr int NS = LATE ? 1 : 2;              // k and v slots
  static constexpr int KX = 0;                         // [NS] k slots (landed, then hi | mid)
  static constexpr int VX = KX + NS * Slot<D>::FLOATS; // [NS] v slots (landed, then hi | mid)
  static constexpr int KL = VX + NS * Slot<D>::FLOATS; // bf16 [TT x D] third part of k
  static constexpr int VL = KL + TT * D / 2;           // bf16 [TT x D] third part of v
  static constexpr int PK = VL + TT * D / 2;           // bf16 [TT x SP] hi, then lo
  static constexpr int DJ = PK + TT * SP;              // bf16 [TT x PJ] hi, then lo
  static constexpr int PS = DJ + TT * PJ;              // bf16 [3*PJ x D] planes [hi; mid; lo]
  static constexpr int PT = PS + 3 * PJ * D / 2;       // bf16 [2*D x PJ] planes^T [hi; lo]
  static constexpr int DB = PT + D * PJ;               // bf16 [3*SP x D] dB [hi; mid; lo]
  static constexpr int DBT = DB + 3 * SP * D / 2;      // bf16 [2*D x SP] dB^T [hi; lo]
  static constexpr int DA = DBT + D * SP;              // [SP] dA
  static constexpr int RED = DA + SP;                  // [16] reductions
  static constexpr int NFULL = NS;                      // tile-landed barriers
  static constexpr int BAR = RED + 16;                 // mbarriers + TMEM base slot
  static constexpr int FLOATS = BAR + 16 + 256;        // + slack for 1 KB alignment
  // PROJ [0, 48), DPK [64, 64 + 3SP), DV [C_DV, C_DV + 2D), DK [C_DK, C_DK + 2D)
  static constexpr int TCOLS = 512;
  static constexpr int C_PROJ = 0, C_DPK = 64, C_DV = LATE ? 256 : 160, C_DK = LATE ? 384 : 288;
  static_assert(C_DPK + 3 * SP <= C_DV && C_DV + 2 * D <= C_DK && C_DK + 2 * D <= TCOLS,
                "tensor-memory columns");
  static_assert(FLOATS * 4 <= 227 * 1024, "shared memory");
};

// A wait that times out sets the CTA's abort word (so the other threads'
// waits return at once) and the thread's `failed`; side effects (stores,
// MMA and copy issue) are skipped from then on, and every tile ends with one
// CTA-wide vote so all threads leave the loops together.  The kernel then
// waits for its own copies in flight and frees its tensor memory.
#define T5_WAIT(bar_, ph_)                                       \
  do {                                                           \
    if (!bar_wait(bar_, ph_, abort_flag, prm.wait_polls)) failed = true; \
  } while (0)
#define T5_VOTE()                                                \
  (__syncthreads_or(failed) ? (failed = true) : false)

#define T5_PROLOGUE                                                          \
  extern __shared__ __align__(1024) float sm_raw[];                          \
  float* sm = sm_raw + ((1024 - (saddr(sm_raw) & 1023)) & 1023) / 4;         \
  uint64_t* barA = reinterpret_cast<uint64_t*>(sm + LY::BAR);                \
  uint64_t* barB = barA + 1;                                                 \
  uint64_t* full = barA + 2; /* [LY::NFULL]: the tile of a slot landed */   \
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + LY::BAR + 2 * (2 + LY::NFULL)); \
  volatile uint32_t* abort_flag = tslot + 1;                                 \
  const int tid = threadIdx.x, warp = tid >> 5;                              \
  const int row = tid & (TT - 1), sub = tid / TT;                            \
  const float inv_scale = 1.f / __ldg(prm.scale);                            \
  const int L = prm.L;                                                       \
  const int items = prm.N * prm.P;                                           \
  if ((int)blockIdx.x >= items) return;                                      \
  if (tid == 0) {                                                            \
    *abort_flag = 0;                                                         \
    bar_init(barA);                                                          \
    bar_init(barB);                                                          \
    for (int f_ = 0; f_ < LY::NFULL; ++f_) bar_init(full + f_);              \
  }                                                                          \
  if (warp == 0) tmem_alloc<LY::TCOLS>(tslot);                               \
  fence_before();                                                            \
  __syncthreads();                                                           \
  fence_after();                                                             \
  const uint32_t tbase = *tslot;                                             \
  const uint32_t tlane = tbase + ((uint32_t)((warp & 3) * 32) << 16);        \
  uint32_t phA = 0, phB = 0, phF = 0; /* phF bit s: parity of full[s] */   \
  uint32_t inflight = 0;              /* bit s: a tile of slot s in flight */\
  uint32_t issA = 0, issB = 0;        /* thread 0: MMA commits issued     */\
  bool failed = false;                                                       \
  int cur_n = -1, cur_m = -1;

// Before staging into a slot that a bulk store issued by thread 0 may still
// be reading: thread 0 waits for its stores' reads, then the CTA.
#define T5_STAGE_DRAIN()                 \
  do {                                  \
    if (tid == 0) bulk_wait_read();     \
    __syncthreads();                    \
  } while (0)

// On the way out every thread waits (full poll count) for the tiles it saw
// issued into its slots, thread 0 for its bulk stores and for the last MMA
// commit of each barrier (MMAs complete in issue order, and at most one
// commit per barrier is ever outstanding), so no copy or MMA still targets
// this CTA's shared or tensor memory when it is freed.
#define T5_EPILOGUE                                                          \
  {                                                                          \
    bool drained_ = true;                                                    \
    if (tid == 0) {                                                          \
      bulk_wait_all();                                                       \
      if (issA > 0 && !bar_wait(barA, (issA - 1) & 1)) drained_ = false;     \
      if (issB > 0 && !bar_wait(barB, (issB - 1) & 1)) drained_ = false;     \
    }                                                                        \
    for (int s_ = 0; s_ < LY::NFULL; ++s_)                                   \
      if ((inflight >> s_) & 1)                                              \
        if (!bar_wait(full + s_, (phF >> s_) & 1)) drained_ = false;         \
    if (!drained_) atomicOr(prm.err, kErrStuck);                             \
  }                                                                          \
  if (tid == 0 && *abort_flag != 0) atomicOr(prm.err, kErrTimeout);          \
  fence_before();                                                            \
  __syncthreads();                                                           \
  fence_after();                                                             \
  if (warp == 0) tmem_free<LY::TCOLS>(tbase);

// ------------------------------------------------------------------ F2 readout
// out[t] = sum_s pQ[t][s] E[s]  with E = B / (A + eps) of the stream's state.
template <typename T, int D, int SPAD, int K>
__global__ void __launch_bounds__(TT * ReadoutLay<D, SPAD>::NTH, 2) k_t5_readout(const Params prm, const __grid_constant__ TmaMaps maps) {
  using LY = ReadoutLay<D, SPAD>;
  constexpr int SP = LY::SP, NTH = LY::NTH, NTHR = TT * NTH, W = D / NTH;
  using G = Groups<K>;
  constexpr bool F32 = sizeof(T) == 4;
  constexpr bool DIRECT = !F32 && D == 64;   // bf16 tiles are MMA operands as they land
  // bf16 inputs: the per-token operands (pQ / pK, dproj) and the readout's
  // tables as one bf16 part -- the path's bf16 tolerance; the tables whose
  // products cancel (E against its bucket average in dpQ, dB against dA in
  // dpK, the key state against its mass, the backward projections) keep
  // their three parts; fp32: 2 or 3 parts throughout
  constexpr int B2 = F32 ? 2 : 1;
  T5_PROLOGUE
  bf16* pq = reinterpret_cast<bf16*>(sm + LY::PQ);
  bf16* ps = reinterpret_cast<bf16*>(sm + LY::PS);
  bf16* et = reinterpret_cast<bf16*>(sm + LY::ET);
  for (int w = blockIdx.x; w < items && !failed; w += gridDim.x) {
    const Item it = item_of(prm, w);
    if (it.ntiles <= 0) continue;
    const int n = it.n;
    const int m = prm.Mp == 1 ? 0 : n / (prm.B * prm.H);
    __syncthreads();   // the previous item's MMAs are complete; tables may change
    if (m != cur_m) {
      const float* pl = prm.planes + (size_t)m * prm.LK * D;
      put_stack<PJ, D, B2, NTHR>(ps, [&](int j, int d) { return j < prm.LK ? pl[j * D + d] : 0.f; });
      cur_m = m;
    }
    if (n != cur_n) {
      const float* st = prm.state + (size_t)n * prm.SS;
      const float* mass = st + prm.S * D;
      put_stack<D, SP, B2, NTHR>(et, [&](int d, int s) {
        return s < prm.S ? st[s * D + d] / (mass[s] + prm.eps) : 0.f;
      });
      cur_n = n;
    }
    // Pipeline per tile i: load(i+1) | convert(i) -> MMA proj(i) -> store(i-1)
    // through slot i (its parts are consumed) -> probabilities(i) -> MMA out(i)
    auto store_prev = [&](int64_t tprev, float* stage_slot) {
      T5_WAIT(barB, phB);
      phB ^= 1;
      fence_after();
      float o[W];
      tld_sum<W, B2>(tlane + LY::C_OUT + sub * W, D, o);
      put_tile_cols<T, D, W>(stage_slot, row, sub * W, o);
      fence_async_smem();
      fence_before();
      __syncthreads();
      if (tid == 0 && !failed) {
        tma_store_tile<T, D>(&maps.map[1], stage_slot, prm.lo, prm, n, tprev);
        bulk_commit();
      }
    };
    auto load = [&](int j) {
      if (failed) return;
      inflight |= 1u << (j & 1);
      if (tid == 0) {
        bulk_wait_read();   // a store may still be reading this slot
        float* const dst[1] = {sm + LY::QX + (j & 1) * Slot<D>::FLOATS};
        const Layout* const lay[1] = {&prm.lq};
        tma_tile<T, D, 1>(maps, dst, lay, prm, n, it.t0 + (int64_t)j * TT, full + (j & 1));
      }
    };
    load(0);
    for (int i = 0; i < it.ntiles; ++i) {
      const int64_t tile0 = it.t0 + (int64_t)i * TT;
      float* X = sm + LY::QX + (i & 1) * Slot<D>::FLOATS;
      if (i + 1 < it.ntiles) load(i + 1);
      T5_WAIT(full + (i & 1), (phF >> (i & 1)) & 1);
      if (!failed) {
        phF ^= 1u << (i & 1);
        inflight &= ~(1u << (i & 1));
      }
      if constexpr (!DIRECT) {   // bf16 at D = 64: the landed tiles are the operands
        float x[W];
        read_cols<T, D, W>(X, row, sub * W, x);
        convert_sync<D, NTH>(warp);
        put_cols<D, W, F32 ? 2 : 1>(Slot<D>::part(X, 0), Slot<D>::part(X, 1), nullptr, row,
                                    sub * W, x);
      }
      fence_async_smem();
      fence_before();
      if constexpr (!DIRECT) __syncthreads();   // bf16 in place: nothing was converted
      if (tid == 0 && !failed) {
        fence_after();
        gemm_parts<PJ, B2, D / 16, D, D, DIRECT>(tbase + LY::C_PROJ, Slot<D>::part(X, 0),
                                        Slot<D>::part(X, 1), nullptr, F32 ? 2 : 1, ps, false);
        { commit(barA); ++issA; }
      }
      T5_WAIT(barA, phA);   // also covers the previous tile's output MMAs
      phA ^= 1;
      if (i > 0) store_prev(tile0 - TT, X);
      fence_after();
      {
        // two threads per token take two groups each: unrolled (constant offsets)
        float proj[PJ];
        tld_sum<PJ, B2>(tlane + LY::C_PROJ, PJ, proj);
#pragma unroll
        for (int gi = 0; gi < SP / G::GB; ++gi) {
          if (gi % NTH == sub) {
            float p[G::GB], h[G::GK];
            const bool has = gi * G::GK < PJ;
            group_probs<K>(has ? proj + gi * G::GK : proj, gi * G::GT, has ? L : 0, inv_scale, p,
                           h);
            put_cols<SP, G::GB, B2>(pq, pq + TT * SP, nullptr, row, gi * G::GB, p);
          }
        }
      }
      fence_async_smem();
      fence_before();
      if (__syncthreads_or(failed)) failed = true;   // the tile's vote
      if (tid == 0 && !failed) {
        fence_after();
        gemm_parts<D, B2, SP / 16, SP, SP>(tbase + LY::C_OUT, pq, pq + TT * SP, nullptr, B2, et,
                                          false);
        { commit(barB); ++issB; }
      }
      if (failed) break;
    }
    // the last tile leaves through its own slot, which the store of the
    // tile before may still be reading
    T5_STAGE_DRAIN();
    if (!failed)
      store_prev(it.t0 + (int64_t)(it.ntiles - 1) * TT,
                 sm + LY::QX + ((it.ntiles - 1) & 1) * Slot<D>::FLOATS);
    T5_VOTE();
  }
  T5_EPILOGUE
}

// ------------------------------------------------------------------ F1 reduce
template <int D, int SPAD>
struct ReduceLay {
  static constexpr int NTH = 2;           // threads per token (two CTAs per SM)
  static constexpr int SP = (SPAD + 15) / 16 * 16;     // bucket columns
  static constexpr int NFULL = 2;                       // k slot 0, v slot 1
  static constexpr int KX = 0;                          // k slot (landed, then 2 parts)
  static constexpr int VX = KX + Slot<D>::FLOATS;       // v slot (landed, then hi | mid)
  static constexpr int VL = VX + Slot<D>::FLOATS;       // third part of v: [TT x D]
  static constexpr int PK3 = VL + TT * D / 2;           // pK parts: [TT x 3 SP] = [hi | mid | lo]
  static constexpr int PS = PK3 + 3 * TT * SP / 2;      // bf16 [2*PJ x D] planes [hi; lo]
  static constexpr int BAR = PS + PJ * D;
  static constexpr int FLOATS = BAR + 16 + 256;
  // PROJ [0, 32), STATE [C_ST, C_ST + 3 SP) (M = 64)
  static constexpr int TCOLS = 256;
  static constexpr int C_PROJ = 0, C_ST = SP > 32 ? 64 : 128;
  static_assert(3 * TT * SP / 2 >= TT * SP, "pK area doubles as the mass scratch");
  static_assert(C_ST + 3 * SP <= TCOLS, "tensor-memory columns");
  static_assert(FLOATS * 4 <= 227 * 1024, "shared memory");
};

// Per range: B[s][d] = sum_t pK[t][s] v[t][d] and A[s] = sum_t pK[t][s] into
// the range's partial slot ([S][D] then [S]).  The tensor core accumulates
// v^T . pK over every tile of the range in tensor memory (M = 64 rows of d,
// both operands read MN-major from the token-major parts) with three bf16
// parts on both sides (24 significant bits: a bucket that holds one token
// must reproduce that token's v to fp32 accuracy, or the backward's
// v . dB - dB . E loses it); the bucket mass is summed by the threads that
// own each bucket group.
template <typename T, int D, int SPAD, int K>
__global__ void __launch_bounds__(TT * ReduceLay<D, SPAD>::NTH, 2)
    k_t5_reduce(const Params prm, const __grid_constant__ TmaMaps maps) {
  using LY = ReduceLay<D, SPAD>;
  constexpr int SP = LY::SP, NTH = LY::NTH, NTHR = TT * NTH, W = D / NTH;
  using G = Groups<K>;
  constexpr int NG = SP / G::GB;                       // bucket groups
  constexpr int MYG = (NG + NTH - 1) / NTH;            // groups per thread (at most)
  constexpr bool F32 = sizeof(T) == 4;
  constexpr bool DIRECT = !F32 && D == 64;   // bf16 tiles are MMA operands as they land
  // bf16 inputs: the per-token operands (pQ / pK, dproj) and the readout's
  // tables as one bf16 part -- the path's bf16 tolerance; the tables whose
  // products cancel (E against its bucket average in dpQ, dB against dA in
  // dpK, the key state against its mass, the backward projections) keep
  // their three parts; fp32: 2 or 3 parts throughout
  constexpr int B2 = F32 ? 2 : 1;
  T5_PROLOGUE
  (void)cur_n;
  bf16* pk3 = reinterpret_cast<bf16*>(sm + LY::PK3);
  bf16* ps = reinterpret_cast<bf16*>(sm + LY::PS);
  for (int w = blockIdx.x; w < items && !failed; w += gridDim.x) {
    const Item it = item_of(prm, w);
    const int n = it.n;
    float* dst = prm.part + ((size_t)n * prm.P + it.part) * prm.SS;
    const int m = prm.Mp == 1 ? 0 : n / (prm.B * prm.H);
    __syncthreads();
    if (m != cur_m) {
      const float* pl = prm.planes + (size_t)m * prm.LK * D;
      put_stack<PJ, D, B2, NTHR>(ps, [&](int j, int d) { return j < prm.LK ? pl[j * D + d] : 0.f; });
      cur_m = m;
    }
    float mass[MYG][G::GB];
#pragma unroll
    for (int a = 0; a < MYG; ++a)
#pragma unroll
      for (int b = 0; b < G::GB; ++b) mass[a][b] = 0.f;
    // One slot each for k and v (two CTAs per SM hide each other's load
    // latency), landing on separate barriers: the k slot is free once the
    // projection MMAs of the previous tile are done, the v slot (whose parts
    // the state MMAs read in place) once the state MMAs are.
    auto load_one = [&](int j, int which) {   // which 0: k, 1: v
      if (failed) return;
      const int f = which;
      inflight |= 1u << f;
      if (tid == 0) {
        using BX = Box<T, D>;
        const int h = n % prm.H, b = (n / prm.H) % prm.B, mm = n / (prm.H * prm.B);
        const Layout& lay = which ? prm.lv : prm.lk;
        char* dst = reinterpret_cast<char*>(sm + (which ? LY::VX : LY::KX));
        fence_async_smem();
        bar_expect_tx(full + f, (uint32_t)BX::BYTES);
#pragma unroll
        for (int x = 0; x < BX::NB; ++x)
          tma_load5(dst + x * TT * BX::IB, &maps.map[which], x * BX::IB / (int)sizeof(T),
                    (int)(it.t0 + (int64_t)j * TT), h, b, lay.sm == 0 ? 0 : mm, full + f);
      }
    };
    auto landed = [&](int f) {
      T5_WAIT(full + f, (phF >> f) & 1);
      if (!failed) {
        phF ^= 1u << f;
        inflight &= ~(1u << f);
      }
    };
    // Per tile i: k parts -> MMA proj(i) -> load k(i+1) -> probabilities ->
    // pK parts -> v parts (in place) -> MMA state(i) -> [thread 0: state(i)
    // done] load v(i+1).  v(i+1) lands while tile i+1's projections and
    // probabilities are formed; only thread 0 waits for the state MMAs.
    if (it.ntiles > 0) {
      load_one(0, 0);
      load_one(0, 1);
    }
    for (int i = 0; i < it.ntiles; ++i) {
      const int64_t tile0 = it.t0 + (int64_t)i * TT;
      float* KXt = sm + LY::KX;
      float* VXt = sm + LY::VX;
      bf16* vl = reinterpret_cast<bf16*>(sm + LY::VL);
      landed(0);
      const bool valid = tile0 + row < it.t1;
      if constexpr (!DIRECT) {   // bf16 at D = 64: the landed tiles are the operands
        float x[W];
        read_cols<T, D, W>(KXt, row, sub * W, x);
        convert_sync<D, NTH>(warp);
        put_cols<D, W, F32 ? 2 : 1>(Slot<D>::part(KXt, 0), Slot<D>::part(KXt, 1), nullptr, row,
                                    sub * W, x);
      }
      fence_async_smem();
      fence_before();
      if constexpr (!DIRECT) __syncthreads();   // bf16 in place: nothing was converted
      if (tid == 0 && !failed) {
        fence_after();
        gemm_parts<PJ, B2, D / 16, D, D, DIRECT>(tbase + LY::C_PROJ, Slot<D>::part(KXt, 0),
                                        Slot<D>::part(KXt, 1), nullptr, F32 ? 2 : 1, ps, false);
        { commit(barA); ++issA; }
      }
      T5_WAIT(barA, phA);
      phA ^= 1;
      if (i + 1 < it.ntiles) load_one(i + 1, 0);
      fence_after();
      {
#pragma unroll
        for (int a = 0; a < MYG; ++a) {
          const int gi = sub + a * NTH;
          if (gi < NG) {
            float pj[G::GK], p[G::GB], h[G::GK];
            const bool has = gi * G::GK < PJ;
            tld_group<G::GK, B2>(tlane + LY::C_PROJ, has ? gi * G::GK : 0, pj);
            group_probs<K>(pj, gi * G::GT, has ? L : 0, inv_scale, p, h);
#pragma unroll
            for (int b = 0; b < G::GB; ++b) {
              if (!valid) p[b] = 0.f;
              mass[a][b] += p[b];
            }
            // one row of [hi | mid | lo] bucket blocks
#pragma unroll
            for (int c8 = 0; c8 < G::GB / 8; ++c8) {
              uint4 h, mq, l;
              split3(p[8 * c8 + 0], p[8 * c8 + 1], h.x, mq.x, l.x);
              split3(p[8 * c8 + 2], p[8 * c8 + 3], h.y, mq.y, l.y);
              split3(p[8 * c8 + 4], p[8 * c8 + 5], h.z, mq.z, l.z);
              split3(p[8 * c8 + 6], p[8 * c8 + 7], h.w, mq.w, l.w);
              uint4* q4 = reinterpret_cast<uint4*>(pk3);
              const int c0 = gi * G::GB / 8 + c8;
              q4[chunk<3 * SP>(row, c0)] = h;
              q4[chunk<3 * SP>(row, SP / 8 + c0)] = mq;
              q4[chunk<3 * SP>(row, 2 * SP / 8 + c0)] = l;
            }
          }
        }
      }
      landed(1);
      if constexpr (!DIRECT) {
        float y[W];
        read_cols<T, D, W>(VXt, row, sub * W, y);
        if (!valid) {   // v rows past the range are zero
#pragma unroll
          for (int c = 0; c < W; ++c) y[c] = 0.f;
        }
        convert_sync<D, NTH>(warp);
        put_cols<D, W, F32 ? 3 : 1>(Slot<D>::part(VXt, 0), Slot<D>::part(VXt, 1), vl, row,
                                    sub * W, y);
      }
      fence_async_smem();
      fence_before();
      __syncthreads();
      if (tid == 0 && !failed) {
        fence_after();
        // state^T[d][s-block j] += sum_a v_a^T . pK_j  (v_a, pK MN-major over the tile's tokens)
        const bf16* va[3] = {Slot<D>::part(VXt, 0), Slot<D>::part(VXt, 1), vl};
#pragma unroll
        for (int a = 0; a < (F32 ? 3 : 1); ++a)   // bf16 v is exact in its first part
#pragma unroll
          for (int ks = 0; ks < TT / 16; ++ks)
            mma(tbase + LY::C_ST, desc_a_mn<D, DIRECT>(va[a], ks), desc_mn<3 * SP>(pk3, ks),
                idesc64_mn<3 * SP>(), i > 0 || a > 0 || ks > 0);
        { commit(barB); ++issB; }
      }
      if (i + 1 < it.ntiles) {   // the state MMAs read the v slot in place
        if (tid == 0) T5_WAIT(barB, phB);   // the other threads move on to tile i + 1
        phB ^= 1;
        load_one(i + 1, 1);
      }
      if (T5_VOTE()) break;
    }
    if (failed) break;
    if (it.ntiles > 0) {
      T5_WAIT(barB, phB);
      phB ^= 1;
      if (T5_VOTE()) break;
      fence_after();
      // state: lane 32 q + l (l < 16) of warps 0..3 holds row d = 16 q + l;
      // eight bucket columns of the three part blocks at a time
      if (sub == 0) {
        const int l = tid & 31, d = 16 * (warp & 3) + l;
#pragma unroll
        for (int c = 0; c < SP; c += 8) {
          float st[3][8] = {};
#pragma unroll
          for (int j = 0; j < 3; ++j) tld8(tlane + LY::C_ST + j * SP + c, st[j]);
          tld_wait();
          if (l < 16 && d < D) {
#pragma unroll
            for (int e = 0; e < 8; ++e)
              if (c + e < prm.S) dst[(c + e) * D + d] = st[0][e] + st[1][e] + st[2][e];
          }
        }
      }
      fence_before();
      // bucket mass: per-thread sums -> scratch (pK area is free) -> fixed-order sum
      float* ms = sm + LY::PK3;
#pragma unroll
      for (int a = 0; a < MYG; ++a)
        if (sub + a * NTH < NG)
#pragma unroll
          for (int b = 0; b < G::GB; ++b) ms[row * SP + (sub + a * NTH) * G::GB + b] = mass[a][b];
      __syncthreads();
      if (tid < prm.S) {
        float tot = 0.f;
        for (int r = 0; r < TT; ++r) tot += ms[r * SP + tid];
        dst[prm.S * D + tid] = tot;
      }
    } else {
      for (int e = tid; e < prm.S * D + prm.S; e += NTHR) dst[e] = 0.f;
    }
  }
  T5_EPILOGUE
}

// ------------------------------------------------------------------ B1 query backward
// Up to 32 buckets: two q slots and three dO slots, and tile i+1 is loaded as
// tile i starts.  Above 32 buckets (LATE) the larger pQ / E operands leave
// room for one q slot and two dO slots: tile i+1 is then loaded once tile i's
// projections are done and dq of tile i-1 has left through the q slot.
template <int D, int SPAD>
struct BwdQLay {
  static constexpr int NTH = 4;           // threads per token
  static constexpr int SP = (SPAD + 15) / 16 * 16;     // bucket columns
  static constexpr bool LATE = SP > 32;
  static constexpr int NQ = LATE ? 1 : 2;               // q slots
  static constexpr int NFULL = LATE ? 2 : 3;            // dO slots in rotation (one barrier each)
  static constexpr int QX = 0;                          // [NQ] q slots (landed, then hi | mid)
  static constexpr int GX = QX + NQ * Slot<D>::FLOATS;  // [NFULL] dO slots (landed, then hi | lo)
  static constexpr int QL = GX + NFULL * Slot<D>::FLOATS;   // bf16 [TT x D] third part of q
  static constexpr int PQ = QL + TT * D / 2;            // pQ parts [TT x 2 SP] = [hi | lo]
  static constexpr int DJ = PQ + TT * SP;               // bf16 [TT x PJ] hi, then lo
  static constexpr int PS = DJ + TT * PJ;               // bf16 [3*PJ x D] planes [hi; mid; lo]
  static constexpr int PT = PS + 3 * PJ * D / 2;        // bf16 [2*D x PJ] planes^T [hi; lo]
  static constexpr int ET = PT + D * PJ;                // bf16 [3*SP x D] E [hi; mid; lo]
  static constexpr int RED = ET + 3 * SP * D / 2;       // [16] reductions
  static constexpr int BAR = RED + 16;
  static constexpr int FLOATS = BAR + 16 + 256;
  // PROJ [0, 48), DPQ [64, 64 + 3SP), DQ [C_DQ, C_DQ + 2D), DE [384, 384 + 2SP) (M = 64)
  static constexpr int TCOLS = 512;
  static constexpr int C_PROJ = 0, C_DPQ = 64, C_DQ = LATE ? 256 : 160, C_DE = 384;
  static_assert(C_DPQ + 3 * SP <= C_DQ && C_DQ + 2 * D <= C_DE && C_DE + 2 * SP <= TCOLS,
                "tensor-memory columns");
  static_assert(FLOATS * 4 <= 227 * 1024, "shared memory");
};

// dq = dproj(pQ, dO . E^T) . P per token; per range the partial dE[s][d] =
// sum_t pQ[t][s] dO[t][d] (accumulated over the range's tiles in tensor memory,
// M = 64 rows of d, dO and pQ read MN-major) and the q-side dscale.
template <typename T, int D, int SPAD, int K>
__global__ void __launch_bounds__(TT * BwdQLay<D, SPAD>::NTH, 1)
    k_t5_bwd_q(const Params prm, const __grid_constant__ TmaMaps maps) {
  using LY = BwdQLay<D, SPAD>;
  constexpr int SP = LY::SP, NTH = LY::NTH, NTHR = TT * NTH, W = D / NTH;
  using G = Groups<K>;
  constexpr bool F32 = sizeof(T) == 4;
  constexpr bool DIRECT = !F32 && D == 64;   // bf16 tiles are MMA operands as they land
  // bf16 inputs: the per-token operands (pQ / pK, dproj) and the readout's
  // tables as one bf16 part -- the path's bf16 tolerance; the tables whose
  // products cancel (E against its bucket average in dpQ, dB against dA in
  // dpK, the key state against its mass, the backward projections) keep
  // their three parts; fp32: 2 or 3 parts throughout
  constexpr int B2 = F32 ? 2 : 1;
  T5_PROLOGUE
  bf16* pq = reinterpret_cast<bf16*>(sm + LY::PQ);
  bf16* dj = reinterpret_cast<bf16*>(sm + LY::DJ);
  bf16* ps = reinterpret_cast<bf16*>(sm + LY::PS);
  bf16* pt = reinterpret_cast<bf16*>(sm + LY::PT);
  bf16* et = reinterpret_cast<bf16*>(sm + LY::ET);
  // planes of DJ not covered by any bucket group stay zero
  for (int i = tid; i < TT * PJ; i += NTHR) reinterpret_cast<float*>(dj)[i] = 0.f;
  for (int w = blockIdx.x; w < items && !failed; w += gridDim.x) {
    const Item it = item_of(prm, w);
    const int n = it.n;
    float* dst = prm.part + ((size_t)n * prm.P + it.part) * prm.SS;
    float ds = 0.f;
    if (it.ntiles > 0) {
      const int m = prm.Mp == 1 ? 0 : n / (prm.B * prm.H);
      __syncthreads();
      if (m != cur_m) {
        const float* pl = prm.planes + (size_t)m * prm.LK * D;
        put_stack<PJ, D, 3, NTHR>(ps, [&](int j, int d) { return j < prm.LK ? pl[j * D + d] : 0.f; });
        put_stack<D, PJ, B2, NTHR>(pt, [&](int d, int j) { return j < prm.LK ? pl[j * D + d] : 0.f; });
        cur_m = m;
      }
      if (n != cur_n) {
        const float* st = prm.state + (size_t)n * prm.SS;
        const float* mass = st + prm.S * D;
        // E in three parts: dpQ cancels against its bucket average where a
        // bucket's means are nearly equal
        put_stack<SP, D, 3, NTHR>(et, [&](int sidx, int d) {
          return sidx < prm.S ? st[sidx * D + d] / (mass[sidx] + prm.eps) : 0.f;
        });
        cur_n = n;
      }
      __syncthreads();
      // dq of tile i-1 leaves through a consumed dO slot (or, LATE, the q slot)
      auto store_prev = [&](int64_t tprev, float* stage_slot) {
        T5_WAIT(barB, phB);
        phB ^= 1;
        fence_after();
        float o[W];
        tld_sum<W, B2>(tlane + LY::C_DQ + sub * W, D, o);
        put_tile_cols<T, D, W>(stage_slot, row, sub * W, o);
        fence_async_smem();
        fence_before();
        __syncthreads();
        if (tid == 0 && !failed) {
          tma_store_tile<T, D>(&maps.map[2], stage_slot, prm.ldq, prm, n, tprev);
          bulk_commit();
        }
      };
      auto load = [&](int j) {
        if (failed) return;
        inflight |= 1u << (j % LY::NFULL);
        if (tid == 0) {
          bulk_wait_read();   // a store may still be reading the q slot
          float* const dsts[2] = {sm + LY::QX + (j % LY::NQ) * Slot<D>::FLOATS,
                                  sm + LY::GX + (j % LY::NFULL) * Slot<D>::FLOATS};
          const Layout* const lay[2] = {&prm.lq, &prm.ldo};
          tma_tile<T, D, 2>(maps, dsts, lay, prm, n, it.t0 + (int64_t)j * TT, full + (j % LY::NFULL));
        }
      };
      // Per tile i: q, dO parts -> MMA proj, dpQ (i) || store dq(i-1) -> hash
      // backward(i) -> MMA dE += dO^T pQ, dq (i) || next tile
      load(0);
      for (int i = 0; i < it.ntiles; ++i) {
        const int64_t tile0 = it.t0 + (int64_t)i * TT;
        float* QXt = sm + LY::QX + (i % LY::NQ) * Slot<D>::FLOATS;
        float* GXt = sm + LY::GX + (i % LY::NFULL) * Slot<D>::FLOATS;
        const int fb = i % LY::NFULL;
        bf16* ql = reinterpret_cast<bf16*>(sm + LY::QL);
        if (!LY::LATE && i + 1 < it.ntiles) load(i + 1);
        T5_WAIT(full + fb, (phF >> fb) & 1);
        if (!failed) {
          phF ^= 1u << fb;
          inflight &= ~(1u << fb);
        }
        const bool valid = tile0 + row < it.t1;
        if constexpr (!DIRECT) {   // bf16 at D = 64: the landed tiles are the operands
          float x[W], y[W];
          read_cols<T, D, W>(QXt, row, sub * W, x);
          read_cols<T, D, W>(GXt, row, sub * W, y);
          if (!valid) {   // rows past the range add nothing to dE
#pragma unroll
            for (int c = 0; c < W; ++c) y[c] = 0.f;
          }
          convert_sync<D, NTH>(warp);
          // hi | mid in place, the third part beside (read only by this tile's
          // projection MMAs, which finish before the next conversion)
          put_cols<D, W, F32 ? 3 : 1>(Slot<D>::part(QXt, 0), Slot<D>::part(QXt, 1), ql, row,
                                      sub * W, x);
          put_cols<D, W, F32 ? 2 : 1>(Slot<D>::part(GXt, 0), Slot<D>::part(GXt, 1), nullptr, row,
                                      sub * W, y);
        }
        fence_async_smem();
        fence_before();
        if constexpr (!DIRECT) __syncthreads();   // bf16 in place: nothing was converted
        if (tid == 0 && !failed) {
          fence_after();
          // projections in three parts on both sides: they feed the
          // temperature gradient, a sum with heavy cancellation
          gemm_parts<PJ, 3, D / 16, D, D, DIRECT>(tbase + LY::C_PROJ, Slot<D>::part(QXt, 0),
                                          Slot<D>::part(QXt, 1), ql, F32 ? 3 : 1, ps, false);
          gemm_parts<SP, 3, D / 16, D, D, DIRECT>(tbase + LY::C_DPQ, Slot<D>::part(GXt, 0),
                                          Slot<D>::part(GXt, 1), nullptr, F32 ? 2 : 1, et, false);
          { commit(barA); ++issA; }
        }
        // Up to 32 buckets dq of tile i-1 leaves through dO slot i-1 (free
        // once its dE MMAs are done; the next load into it waits for the
        // store's reads) while the tensor core forms tile i's projections;
        // LATE through the q slot once those are done.
        if (!LY::LATE && i > 0)
          store_prev(tile0 - TT, sm + LY::GX + ((i + LY::NFULL - 1) % LY::NFULL) * Slot<D>::FLOATS);
        T5_WAIT(barA, phA);   // also covers the previous tile's dE / dq MMAs
        phA ^= 1;
        if (LY::LATE && i > 0) store_prev(tile0 - TT, QXt);
        // LATE: the q slot is free (projections done, dq(i-1) read by its
        // store) and so is dO slot i+1 (dE(i-1) done)
        if (LY::LATE && i + 1 < it.ntiles) load(i + 1);
        fence_after();
        {

          // one copy of the group code: groups gi = sub, sub + NTH, ... (warp-uniform)
#pragma unroll 1
          for (int gi = sub; gi < SP / G::GB; gi += NTH) {
            {
              float pj[G::GK], p[G::GB], h[G::GK], g[G::GB], dj_[G::GK];
              const bool has = gi * G::GK < PJ;
              tld_group<G::GK, 3>(tlane + LY::C_PROJ, has ? gi * G::GK : 0, pj);
              group_probs<K>(pj, gi * G::GT, has ? L : 0, inv_scale, p, h);
              tld_sum<G::GB, 3>(tlane + LY::C_DPQ + gi * G::GB, SP, g);
              float dsl = 0.f;
              group_probs_bwd<K>(p, g, h, inv_scale, dj_, dsl);
              if (valid) ds += dsl;
              if (!valid) {
#pragma unroll
                for (int b = 0; b < G::GB; ++b) p[b] = 0.f;
              }
              // one row of [hi | lo] bucket blocks
#pragma unroll
              for (int c8 = 0; c8 < G::GB / 8; ++c8) {
                if constexpr (!F32) {
                  put_cols<2 * SP, 8, 1>(pq, nullptr, nullptr, row, gi * G::GB + 8 * c8, p + 8 * c8);
                  continue;
                }
                uint4 hq, lq;
                split2(p[8 * c8 + 0], p[8 * c8 + 1], hq.x, lq.x);
                split2(p[8 * c8 + 2], p[8 * c8 + 3], hq.y, lq.y);
                split2(p[8 * c8 + 4], p[8 * c8 + 5], hq.z, lq.z);
                split2(p[8 * c8 + 6], p[8 * c8 + 7], hq.w, lq.w);
                uint4* q4 = reinterpret_cast<uint4*>(pq);
                const int c0 = gi * G::GB / 8 + c8;
                q4[chunk<2 * SP>(row, c0)] = hq;
                q4[chunk<2 * SP>(row, SP / 8 + c0)] = lq;
              }
              if (has) {
#pragma unroll
                for (int j = 0; j < G::GK; ++j) {
                  const int jj = gi * G::GK + j;
                  if (jj < PJ) {
                    const bf16 hb = __float2bfloat16_rn(dj_[j]);
                    dj[elem<PJ>(row, jj)] = hb;
                    if constexpr (F32)
                      dj[TT * PJ + elem<PJ>(row, jj)] = __float2bfloat16_rn(dj_[j] - __bfloat162float(hb));
                  }
                }
              }
            }
          }
        }
        fence_async_smem();
        fence_before();
        if (__syncthreads_or(failed)) failed = true;   // the tile's vote
        if (tid == 0 && !failed) {
          fence_after();
          // dE^T[d][s-block j] += sum_a dO_a^T . pQ_j (MN-major over the tile's tokens)
#pragma unroll
          for (int a = 0; a < (F32 ? 2 : 1); ++a)
#pragma unroll
            for (int ks = 0; ks < TT / 16; ++ks)
              mma(tbase + LY::C_DE, desc_a_mn<D, DIRECT>(Slot<D>::part(GXt, a), ks), desc_mn<2 * SP>(pq, ks),
                  idesc64_mn<B2 * SP>(), i > 0 || a > 0 || ks > 0);
          gemm_parts<D, B2, PJ / 16, PJ, PJ>(tbase + LY::C_DQ, dj, dj + TT * PJ, nullptr, B2, pt,
                                            false);
          { commit(barB); ++issB; }
        }
        if (failed) break;
      }
      T5_STAGE_DRAIN();   // LATE: the store of the tile before may still read the q slot
      if (!failed)
        store_prev(it.t0 + (int64_t)(it.ntiles - 1) * TT,
                   sm + LY::QX + ((it.ntiles - 1) % LY::NQ) * Slot<D>::FLOATS);
      if (T5_VOTE()) break;
      fence_after();
      // dE: lane 32 q + l (l < 16) of warps 0..3 holds row d = 16 q + l;
      // eight bucket columns of both part blocks at a time
      if (sub == 0) {
        const int l = tid & 31, d = 16 * (warp & 3) + l;
#pragma unroll
        for (int c = 0; c < SP; c += 8) {
          float e[2][8] = {};
          tld8(tlane + LY::C_DE + c, e[0]);
          if constexpr (F32) tld8(tlane + LY::C_DE + SP + c, e[1]);
          tld_wait();
          if (l < 16 && d < D) {
#pragma unroll
            for (int x = 0; x < 8; ++x)
              if (c + x < prm.S) dst[(c + x) * D + d] = e[0][x] + e[1][x];
          }
        }
      }
      fence_before();
      for (int e2 = tid; e2 < prm.S; e2 += NTHR) dst[prm.S * D + e2] = 0.f;
    } else {
      for (int e2 = tid; e2 < prm.S * D + prm.S; e2 += NTHR) dst[e2] = 0.f;
    }
    // per-item dscale partial (zero for an empty range), fixed-order CTA sum
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
// dv = pK . dB,  dpK = v . dB^T + dA,  dk = dproj(pK, dpK) . P;  the k-side dscale.
template <typename T, int D, int SPAD, int K>
__global__ void __launch_bounds__(TT * BwdKVLay<D, SPAD>::NTH, 1) k_t5_bwd_kv(const Params prm, const __grid_constant__ TmaMaps maps) {
  using LY = BwdKVLay<D, SPAD>;
  constexpr int SP = LY::SP, NTH = LY::NTH, NTHR = TT * NTH, W = D / NTH;
  using G = Groups<K>;
  constexpr bool F32 = sizeof(T) == 4;
  constexpr bool DIRECT = !F32 && D == 64;   // bf16 tiles are MMA operands as they land
  // bf16 inputs: the per-token operands (pQ / pK, dproj) and the readout's
  // tables as one bf16 part -- the path's bf16 tolerance; the tables whose
  // products cancel (E against its bucket average in dpQ, dB against dA in
  // dpK, the key state against its mass, the backward projections) keep
  // their three parts; fp32: 2 or 3 parts throughout
  constexpr int B2 = F32 ? 2 : 1;
  T5_PROLOGUE
  bf16* pk = reinterpret_cast<bf16*>(sm + LY::PK);
  bf16* dj = reinterpret_cast<bf16*>(sm + LY::DJ);
  bf16* ps = reinterpret_cast<bf16*>(sm + LY::PS);
  bf16* pt = reinterpret_cast<bf16*>(sm + LY::PT);
  bf16* db = reinterpret_cast<bf16*>(sm + LY::DB);
  bf16* dbt = reinterpret_cast<bf16*>(sm + LY::DBT);
  float* dA = sm + LY::DA;
  // planes of DJ not covered by any bucket group stay zero
  for (int i = tid; i < TT * PJ; i += NTHR) reinterpret_cast<float*>(dj)[i] = 0.f;
  for (int w = blockIdx.x; w < items && !failed; w += gridDim.x) {
    const Item it = item_of(prm, w);
    const int n = it.n;
    float ds = 0.f;
    if (it.ntiles > 0) {
      const int m = prm.Mp == 1 ? 0 : n / (prm.B * prm.H);
      __syncthreads();
      if (m != cur_m) {
        const float* pl = prm.planes + (size_t)m * prm.LK * D;
        put_stack<PJ, D, 3, NTHR>(ps, [&](int j, int d) { return j < prm.LK ? pl[j * D + d] : 0.f; });
        put_stack<D, PJ, B2, NTHR>(pt, [&](int d, int j) { return j < prm.LK ? pl[j * D + d] : 0.f; });
        cur_m = m;
      }
      if (n != cur_n) {
        const float* st = prm.state + (size_t)n * prm.SS;
        const float* gs = prm.gstate_in + (size_t)n * prm.SS;
        const float* mass = st + prm.S * D;
        // dB = dE / (A + eps);  dA_s = -sum_d dE_sd B_sd / (A_s + eps)^2
        put_stack<SP, D, 3, NTHR>(db, [&](int s, int d) {
          return s < prm.S ? gs[s * D + d] / (mass[s] + prm.eps) : 0.f;
        });
        put_stack<D, SP, B2, NTHR>(dbt, [&](int d, int s) {
          return s < prm.S ? gs[s * D + d] / (mass[s] + prm.eps) : 0.f;
        });
        if (tid < SP) {
          float a = 0.f;
          if (tid < prm.S) {
            const float inv = 1.f / (mass[tid] + prm.eps);
            for (int d = 0; d < D; ++d) a = fmaf(gs[tid * D + d], st[tid * D + d], a);
            a = -a * inv * inv;
          }
          dA[tid] = a;
        }
        cur_n = n;
      }
      __syncthreads();
      // Pipeline per tile i: load(i+1) | convert(i) -> MMA proj, dpK (i) ||
      // store(i-1) -> hash backward(i) -> MMA dv, dk (i) || next tile ...
      // dv, dk of tile i-1 leave through k, v slots i (their parts are consumed)
      auto store_prev = [&](int64_t tprev, float* stage_k, float* stage_v) {
        T5_WAIT(barB, phB);
        phB ^= 1;
        fence_after();
        {
          float o[W];
          tld_sum<W, B2>(tlane + LY::C_DV + sub * W, D, o);
          put_tile_cols<T, D, W>(stage_k, row, sub * W, o);
          tld_sum<W, B2>(tlane + LY::C_DK + sub * W, D, o);
          put_tile_cols<T, D, W>(stage_v, row, sub * W, o);
        }
        fence_async_smem();
        fence_before();
        __syncthreads();
        if (tid == 0 && !failed) {
          tma_store_tile<T, D>(&maps.map[3], stage_k, prm.ldv, prm, n, tprev);
          tma_store_tile<T, D>(&maps.map[2], stage_v, prm.ldk, prm, n, tprev);
          bulk_commit();
        }
      };
      auto load = [&](int j) {
        if (failed) return;
        inflight |= 1u << (j % LY::NS);
        if (tid == 0) {
          bulk_wait_read();   // stores may still be reading these slots
          float* const dst[2] = {sm + LY::KX + (j % LY::NS) * Slot<D>::FLOATS,
                                 sm + LY::VX + (j % LY::NS) * Slot<D>::FLOATS};
          const Layout* const lay[2] = {&prm.lk, &prm.lv};
          tma_tile<T, D, 2>(maps, dst, lay, prm, n, it.t0 + (int64_t)j * TT, full + (j % LY::NS));
        }
      };
      load(0);
      for (int i = 0; i < it.ntiles; ++i) {
        const int64_t tile0 = it.t0 + (int64_t)i * TT;
        float* KXt = sm + LY::KX + (i % LY::NS) * Slot<D>::FLOATS;
        float* VXt = sm + LY::VX + (i % LY::NS) * Slot<D>::FLOATS;
        const int fb = i % LY::NS;
        bf16* kl = reinterpret_cast<bf16*>(sm + LY::KL);
        bf16* vl = reinterpret_cast<bf16*>(sm + LY::VL);
        if (!LY::LATE && i + 1 < it.ntiles) load(i + 1);
        T5_WAIT(full + fb, (phF >> fb) & 1);
        if (!failed) {
          phF ^= 1u << fb;
          inflight &= ~(1u << fb);
        }
        if constexpr (!DIRECT) {   // bf16 at D = 64: the landed tiles are the operands
          float x[W], y[W];
          read_cols<T, D, W>(KXt, row, sub * W, x);
          read_cols<T, D, W>(VXt, row, sub * W, y);
          convert_sync<D, NTH>(warp);
          // hi | mid in place, the third part beside (read only by this tile's
          // projection / dpK MMAs, which finish before the next conversion)
          put_cols<D, W, F32 ? 3 : 1>(Slot<D>::part(KXt, 0), Slot<D>::part(KXt, 1), kl, row,
                                      sub * W, x);
          put_cols<D, W, F32 ? 3 : 1>(Slot<D>::part(VXt, 0), Slot<D>::part(VXt, 1), vl, row,
                                      sub * W, y);
        }
        fence_async_smem();
        fence_before();
        if constexpr (!DIRECT) __syncthreads();   // bf16 in place: nothing was converted
        // projections and dpK = v . dB^T
        if (tid == 0 && !failed) {
          fence_after();
          // three parts on both sides: the projections feed the temperature
          // gradient (a sum with heavy cancellation), and where v matches a
          // bucket's mean (tiny buckets) v . dB and dA cancel to far below |v| |dB|
          gemm_parts<PJ, 3, D / 16, D, D, DIRECT>(tbase + LY::C_PROJ, Slot<D>::part(KXt, 0),
                                          Slot<D>::part(KXt, 1), kl, F32 ? 3 : 1, ps, false);
          gemm_parts<SP, 3, D / 16, D, D, DIRECT>(tbase + LY::C_DPK, Slot<D>::part(VXt, 0),
                                          Slot<D>::part(VXt, 1), vl, F32 ? 3 : 1, db, false);
          { commit(barA); ++issA; }
        }
        T5_WAIT(barA, phA);   // also covers the previous tile's dv / dk MMAs
        phA ^= 1;
        if (i > 0) store_prev(tile0 - TT, KXt, VXt);
        // LATE: the single k / v slots are free once dv, dk of tile i-1 have been read out of them
        if (LY::LATE && i + 1 < it.ntiles) load(i + 1);
        fence_after();
        {

          const bool valid = tile0 + row < it.t1;
          // one copy of the group code: groups gi = sub, sub + NTH, ... (warp-uniform)
#pragma unroll 1
          for (int gi = sub; gi < SP / G::GB; gi += NTH) {
            {
              float pj[G::GK], p[G::GB], h[G::GK], g[G::GB], dj_[G::GK];
              const bool has = gi * G::GK < PJ;
              tld_group<G::GK, 3>(tlane + LY::C_PROJ, has ? gi * G::GK : 0, pj);
              group_probs<K>(pj, gi * G::GT, has ? L : 0, inv_scale, p, h);
              tld_sum<G::GB, 3>(tlane + LY::C_DPK + gi * G::GB, SP, g);
#pragma unroll
              for (int b = 0; b < G::GB; ++b) g[b] += dA[gi * G::GB + b];
              float dsl = 0.f;
              group_probs_bwd<K>(p, g, h, inv_scale, dj_, dsl);
              if (valid) ds += dsl;
              put_cols<SP, G::GB, B2>(pk, pk + TT * SP, nullptr, row, gi * G::GB, p);
              if (has) {
#pragma unroll
                for (int j = 0; j < G::GK; ++j) {
                  const int jj = gi * G::GK + j;
                  if (jj < PJ) {
                    const bf16 hb = __float2bfloat16_rn(dj_[j]);
                    dj[elem<PJ>(row, jj)] = hb;
                    if constexpr (F32)
                      dj[TT * PJ + elem<PJ>(row, jj)] = __float2bfloat16_rn(dj_[j] - __bfloat162float(hb));
                  }
                }
              }
            }
          }
        }
        fence_async_smem();
        fence_before();
        if (__syncthreads_or(failed)) failed = true;   // the tile's vote
        if (tid == 0 && !failed) {
          fence_after();
          gemm_parts<D, B2, SP / 16, SP, SP>(tbase + LY::C_DV, pk, pk + TT * SP, nullptr, B2, dbt,
                                            false);
          gemm_parts<D, B2, PJ / 16, PJ, PJ>(tbase + LY::C_DK, dj, dj + TT * PJ, nullptr, B2, pt,
                                            false);
          { commit(barB); ++issB; }
        }
        if (failed) break;
      }
      T5_STAGE_DRAIN();   // the stores of the tile before may still read these slots
      if (!failed) {
        const int lt = (it.ntiles - 1) % LY::NS;
        store_prev(it.t0 + (int64_t)(it.ntiles - 1) * TT, sm + LY::KX + lt * Slot<D>::FLOATS,
                   sm + LY::VX + lt * Slot<D>::FLOATS);
      }
      T5_VOTE();
    }
    // per-item dscale partial (zero for an empty range), fixed-order CTA sum
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

// T5_WAIT, T5_VOTE, T5_PROLOGUE and T5_EPILOGUE stay defined for the causal
// kernels of race_causal5.cuh, which undefines them.

}  // namespace t5
}  // namespace race
