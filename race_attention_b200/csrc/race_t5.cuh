// race_t5.cuh -- non-causal readout and key/value backward on the 5th-generation
// tensor cores (tcgen05 + tensor memory).
//
// One thread per token: a CTA of 128 threads walks 128-token tiles; every
// token-major product (projections x.P^T, readout pQ.E, key-side dpK = v.dB^T,
// dv = pK.dB, dk = dproj.P) is an M = 128 tcgen05.mma chain issued by one
// thread, both operands in shared memory, fp32 accumulators in tensor memory.
// Row t of an accumulator is TMEM lane t, so after a tcgen05.ld every thread
// holds its own token's row and the hash arithmetic (tanh, corner
// probabilities and their backward) runs in registers.
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
// fp32 tiles are staged by cp.async in the same arrangement of 16-byte chunks
// (chunk i of a tile at byte 16 i), then converted in place to hi | lo.
#pragma once

#include <cuda_bf16.h>

#include "race_kernels.cuh"
#include "race_tiles.cuh"

namespace race {
namespace t5 {

using bf16 = __nv_bfloat16;

constexpr int TT = 128;   // tokens per tile = MMA M = TMEM lanes
constexpr int NT = 128;   // threads per CTA, one per token
constexpr int PJ = 16;    // projection columns (L*K <= 16)
constexpr int kWaitPolls = 1 << 22;   // bounded mbarrier polls before giving up
constexpr unsigned kErrTimeout = 1u;  // device error bit: an MMA wait timed out

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

// Split product D = A . B^T with K = 16 KS.  A is given as NA bf16 parts
// (a[0] + a[1] + ..., the later ones nullptr-free), B as BP parts stacked
// along its rows ([B0; B1; ...], BP*N rows).  Column block j of D receives
// sum_i A_i . B_j^T -- every part product, since an instruction costs the
// same at N and BP*N.  The caller adds the BP column blocks.
template <int N, int BP, int KS, int CA, int CB>
__device__ __forceinline__ void gemm_parts(uint32_t d, const bf16* a0, const bf16* a1,
                                           const bf16* a2, int na, const bf16* b, bool acc) {
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
__device__ __forceinline__ bool bar_wait(uint64_t* bar, uint32_t parity) {
  for (int i = 0; i < kWaitPolls; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(saddr(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
  }
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
__device__ __forceinline__ void tld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// C columns of this lane as the sum of BP column blocks [c0 + j off, c0 + j off + C)
template <int C, int BP = 2>
__device__ __forceinline__ void tld_sum(uint32_t taddr, int off, float* out) {
#pragma unroll
  for (int c = 0; c < C; c += 16) {
    float a[16], b[16];
    tld16(taddr + c, a);
    tld16(taddr + off + c, b);
    float e[16];
    if constexpr (BP == 3) tld16(taddr + 2 * off + c, e);
    tld_wait();
#pragma unroll
    for (int i = 0; i < 16 && c + i < C; ++i) {
      out[c + i] = a[i] + b[i];
      if constexpr (BP == 3) out[c + i] += e[i];
    }
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

// hi / lo bf16 parts of two floats, packed
__device__ __forceinline__ void split2(float a, float b, uint32_t& hi, uint32_t& lo) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  const float2 hf = __bfloat1622float2(h);
  const __nv_bfloat162 l = __floats2bfloat162_rn(a - hf.x, b - hf.y);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}

// hi / mid / lo bf16 parts of two floats (24 significant bits), packed
__device__ __forceinline__ void split3(float a, float b, uint32_t& hi, uint32_t& mid, uint32_t& lo) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  const float2 hf = __bfloat1622float2(h);
  const float ra = a - hf.x, rb = b - hf.y;
  const __nv_bfloat162 m = __floats2bfloat162_rn(ra, rb);
  const float2 mf = __bfloat1622float2(m);
  const __nv_bfloat162 l = __floats2bfloat162_rn(ra - mf.x, rb - mf.y);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  mid = *reinterpret_cast<const uint32_t*>(&m);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}

// Stages tile rows [t0, t0 + TT) of a [T][D] stream of element type T (row
// stride st) as 16-byte chunks, chunk i of the tile at dst + 16 i -- the
// K-major chunk order (fp32 rows: 4 columns per chunk, bf16: 8).  Rows >= t1
// are zero-filled.
template <typename T, int D>
__device__ __forceinline__ void stage(void* dst, const T* base, int64_t st, int64_t t0, int64_t t1) {
  constexpr int EPC = 16 / (int)sizeof(T);   // elements per chunk
  constexpr int CPR = D / EPC;               // chunks per row
  char* d = static_cast<char*>(dst);
#pragma unroll 4
  for (int i = threadIdx.x; i < TT * CPR; i += NT) {
    const int g = i / (8 * CPR), j = i % (8 * CPR);
    const int c = j >> 3, r = g * 8 + (j & 7);
    const int64_t t = t0 + r;
    const bool ok = t < t1;
    tiles::cp_async16(d + 16 * i, base + (ok ? t : t0) * st + EPC * c, ok);
  }
}

// Reads this thread's row of a staged fp32 tile (4 columns per chunk).
template <int D>
__device__ __forceinline__ void read_row_f32(const void* tile, float (&x)[D]) {
  const float4* t4 = static_cast<const float4*>(tile);
  const int r = threadIdx.x;
#pragma unroll
  for (int c4 = 0; c4 < D / 4; ++c4) {
    const float4 v = t4[(r >> 3) * (D / 4) * 8 + c4 * 8 + (r & 7)];
    x[4 * c4] = v.x;
    x[4 * c4 + 1] = v.y;
    x[4 * c4 + 2] = v.z;
    x[4 * c4 + 3] = v.w;
  }
}

// Writes a register row (C values) of this thread's token as bf16 hi and lo
// operands (C columns each).
template <int C>
__device__ __forceinline__ void put_row(bf16* hi, bf16* lo, const float* v) {
  uint4* h4 = reinterpret_cast<uint4*>(hi);
  uint4* l4 = reinterpret_cast<uint4*>(lo);
  const int r = threadIdx.x;
#pragma unroll
  for (int c8 = 0; c8 < C / 8; ++c8) {
    uint4 h, l;
    split2(v[8 * c8 + 0], v[8 * c8 + 1], h.x, l.x);
    split2(v[8 * c8 + 2], v[8 * c8 + 3], h.y, l.y);
    split2(v[8 * c8 + 4], v[8 * c8 + 5], h.z, l.z);
    split2(v[8 * c8 + 6], v[8 * c8 + 7], h.w, l.w);
    h4[chunk<C>(r, c8)] = h;
    l4[chunk<C>(r, c8)] = l;
  }
}

// Writes a register row as three bf16 parts (hi, mid, lo operands).
template <int C>
__device__ __forceinline__ void put_row3(bf16* hi, bf16* mid, bf16* lo, const float* v) {
  uint4* h4 = reinterpret_cast<uint4*>(hi);
  uint4* m4 = reinterpret_cast<uint4*>(mid);
  uint4* l4 = reinterpret_cast<uint4*>(lo);
  const int r = threadIdx.x;
#pragma unroll
  for (int c8 = 0; c8 < C / 8; ++c8) {
    uint4 h, m, l;
    split3(v[8 * c8 + 0], v[8 * c8 + 1], h.x, m.x, l.x);
    split3(v[8 * c8 + 2], v[8 * c8 + 3], h.y, m.y, l.y);
    split3(v[8 * c8 + 4], v[8 * c8 + 5], h.z, m.z, l.z);
    split3(v[8 * c8 + 6], v[8 * c8 + 7], h.w, m.w, l.w);
    h4[chunk<C>(r, c8)] = h;
    m4[chunk<C>(r, c8)] = m;
    l4[chunk<C>(r, c8)] = l;
  }
}

// Fills a stacked constant operand [part 0; part 1; ...] of BP*R rows and C
// columns with the BP bf16 parts of f(r, c).
template <int R, int C, int BP = 2, class F>
__device__ __forceinline__ void put_stack(bf16* base, F f) {
  for (int i = threadIdx.x; i < R * C; i += NT) {
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

// Corner probabilities of one token from its projections (registers).
// p[s] for s = l*R + r, tables l < L; h[j] = tanh(proj_j) kept for the backward.
template <int K, int SP>
__device__ __forceinline__ void token_probs(const float (&proj)[PJ], int L, float inv_scale,
                                            float (&p)[SP], float (&h)[PJ]) {
  constexpr int R = 1 << K;
  constexpr int LMAX = (SP / R < PJ / K) ? SP / R : PJ / K;
#pragma unroll
  for (int s = 0; s < SP; ++s) p[s] = 0.f;
#pragma unroll
  for (int j = 0; j < PJ; ++j) h[j] = 0.f;
#pragma unroll
  for (int l = 0; l < LMAX; ++l) {
    if (l < L) {
      float sp[K], sn[K];
#pragma unroll
      for (int k = 0; k < K; ++k) {
        const float hh = tiles::tanh_exp(proj[l * K + k]);
        h[l * K + k] = hh;
        const float u = hh * inv_scale;
        const float ex = __expf(-2.f * fabsf(u));
        const float rc = __frcp_rn(1.f + ex);
        sp[k] = u >= 0.f ? rc : ex * rc;
        sn[k] = u >= 0.f ? ex * rc : rc;
      }
#pragma unroll
      for (int r = 0; r < R; ++r) {
        float v = 1.f;
#pragma unroll
        for (int k = 0; k < K; ++k) v *= ((r >> (K - 1 - k)) & 1) ? sp[k] : sn[k];
        p[l * R + r] = v;
      }
    }
  }
}

// Backward of the corner probabilities of one token: given g[s] = dL/dp_s,
// dj[j] = dL/dproj_j; ds += sum_j du_j h_j (the temperature's share).
template <int K, int SP>
__device__ __forceinline__ void token_probs_bwd(const float (&p)[SP], const float (&g)[SP],
                                                const float (&h)[PJ], int L, float inv_scale,
                                                float (&dj)[PJ], float& ds) {
  constexpr int R = 1 << K;
  constexpr int LMAX = (SP / R < PJ / K) ? SP / R : PJ / K;
#pragma unroll
  for (int j = 0; j < PJ; ++j) dj[j] = 0.f;
#pragma unroll
  for (int l = 0; l < LMAX; ++l) {
    if (l < L) {
      float pbar = 0.f;
#pragma unroll
      for (int r = 0; r < R; ++r) pbar = fmaf(p[l * R + r], g[l * R + r], pbar);
      float q[R];
#pragma unroll
      for (int r = 0; r < R; ++r) q[r] = p[l * R + r] * (g[l * R + r] - pbar);
#pragma unroll
      for (int k = 0; k < K; ++k) {
        float du = 0.f;
#pragma unroll
        for (int r = 0; r < R; ++r) du += ((r >> (K - 1 - k)) & 1) ? q[r] : -q[r];
        const float hh = h[l * K + k];
        ds = fmaf(du, hh, ds);
        dj[l * K + k] = du * inv_scale * (1.f - hh * hh);
      }
    }
  }
}

template <typename T, int D>
__device__ __forceinline__ void store_row(T* dst, const float* v) {
  if constexpr (sizeof(T) == 4) {
    float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
    for (int i = 0; i < D / 4; ++i)
      d4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  } else {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
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

// A tile slot holds TT x D fp32 as staged (4 B / element), converted in
// place to NP bf16 parts (hi, lo or hi, mid, lo) of TT x D each; bf16 inputs
// are staged straight into part 0.
template <int D, int NP = 2>
struct Slot {
  static constexpr int FLOATS = TT * D * NP / 2;
  __device__ static bf16* part(float* s, int i) { return reinterpret_cast<bf16*>(s) + i * TT * D; }
};

// ------------------------------------------------------------------ layouts (in floats)
template <int D, int SPAD>
struct ReadoutLay {
  static constexpr int SP = (SPAD + 15) / 16 * 16;   // bucket columns (MMA K)
  static constexpr int QX = 0;                        // [2] slots
  static constexpr int PQ = QX + 2 * Slot<D>::FLOATS; // bf16 [TT x SP] hi, then lo
  static constexpr int PS = PQ + TT * SP;             // bf16 [2*PJ x D] planes [hi; lo]
  static constexpr int ET = PS + PJ * D;              // bf16 [2*D x SP] E^T [hi; lo]
  static constexpr int BAR = ET + D * SP;             // mbarrier (8 B) + TMEM base slot
  static constexpr int FLOATS = BAR + 8;
  static constexpr int TCOLS = 256;                   // PROJ [0, 32), OUT [128, 128 + 2D)
  static constexpr int C_PROJ = 0, C_OUT = 128;
};

template <int D, int SPAD>
struct BwdKVLay {
  static constexpr int SP = (SPAD + 15) / 16 * 16;    // bucket columns (MMA K and N)
  static constexpr int KX = 0;                         // [2] slots
  static constexpr int VX = KX + 2 * Slot<D>::FLOATS;  // [2] slots of three parts
  static constexpr int PK = VX + 2 * Slot<D, 3>::FLOATS;  // bf16 [TT x SP] hi, then lo
  static constexpr int DJ = PK + TT * SP;              // bf16 [TT x PJ] hi, then lo
  static constexpr int PS = DJ + TT * PJ;              // bf16 [2*PJ x D] planes [hi; lo]
  static constexpr int PT = PS + PJ * D;               // bf16 [2*D x PJ] planes^T [hi; lo]
  static constexpr int DB = PT + D * PJ;               // bf16 [3*SP x D] dB [hi; mid; lo]
  static constexpr int DBT = DB + 3 * SP * D / 2;      // bf16 [2*D x SP] dB^T [hi; lo]
  static constexpr int DA = DBT + D * SP;              // [32] dA
  static constexpr int RED = DA + 32;                  // [8] reductions
  static constexpr int BAR = RED + 8;
  static constexpr int FLOATS = BAR + 8;
  static constexpr int TCOLS = 512;   // PROJ [0,32), DPK [32, 32+3SP), DV [128, 128+2D), DK [256, 256+2D)
  static constexpr int C_PROJ = 0, C_DPK = 32, C_DV = 128, C_DK = 256;
};

// After a timed-out wait every thread of the CTA leaves its loops; the kernel
// then waits for its own copies and frees its tensor memory.
#define T5_CHECK(ok_expr)                                        \
  do {                                                           \
    const bool ok_ = (ok_expr);                                  \
    if (__syncthreads_or(!ok_)) {                                \
      if (threadIdx.x == 0) atomicOr(prm.err, kErrTimeout);      \
      failed = true;                                             \
    }                                                            \
  } while (0)

// Converts this thread's rows of staged fp32 slots in place to hi | lo (all
// threads read before any writes).
template <int D>
__device__ __forceinline__ void convert_one(float* slot) {
  float x[D];
  read_row_f32<D>(slot, x);
  __syncthreads();
  put_row<D>(Slot<D>::part(slot, 0), Slot<D>::part(slot, 1), x);
}
// a -> hi, lo;  b -> hi, mid, lo
template <int D>
__device__ __forceinline__ void convert_two(float* a, float* b) {
  float x[D], y[D];
  read_row_f32<D>(a, x);
  read_row_f32<D>(b, y);
  __syncthreads();
  put_row<D>(Slot<D>::part(a, 0), Slot<D>::part(a, 1), x);
  put_row3<D>(Slot<D, 3>::part(b, 0), Slot<D, 3>::part(b, 1), Slot<D, 3>::part(b, 2), y);
}

// ------------------------------------------------------------------ F2 readout
// out[t] = sum_s pQ[t][s] E[s]  with E = B / (A + eps) of the stream's state.
template <typename T, int D, int SPAD, int K>
__global__ void __launch_bounds__(NT, 1) k_t5_readout(const Params prm) {
  using LY = ReadoutLay<D, SPAD>;
  constexpr int SP = LY::SP;
  constexpr bool F32 = sizeof(T) == 4;
  extern __shared__ __align__(128) float sm[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + LY::BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + LY::BAR + 2);
  bf16* pq = reinterpret_cast<bf16*>(sm + LY::PQ);
  bf16* ps = reinterpret_cast<bf16*>(sm + LY::PS);
  bf16* et = reinterpret_cast<bf16*>(sm + LY::ET);
  const int tid = threadIdx.x, warp = tid >> 5;
  const float inv_scale = 1.f / __ldg(prm.scale);
  const int L = prm.L;
  const int items = prm.N * prm.P;
  if ((int)blockIdx.x >= items) return;
  if (tid == 0) bar_init(bar);
  if (warp == 0) tmem_alloc<LY::TCOLS>(tslot);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tbase = *tslot;
  const uint32_t tlane = tbase + ((uint32_t)(warp * 32) << 16);
  uint32_t phase = 0;
  bool failed = false;
  int cur_n = -1, cur_m = -1;
  for (int w = blockIdx.x; w < items && !failed; w += gridDim.x) {
    const Item it = item_of(prm, w);
    if (it.ntiles <= 0) continue;
    const int n = it.n;
    const int m = prm.Mp == 1 ? 0 : n / (prm.B * prm.H);
    __syncthreads();   // the previous item's MMAs are complete; tables may change
    if (m != cur_m) {
      const float* pl = prm.planes + (size_t)m * prm.LK * D;
      put_stack<PJ, D>(ps, [&](int j, int d) { return j < prm.LK ? pl[j * D + d] : 0.f; });
      cur_m = m;
    }
    if (n != cur_n) {
      const float* st = prm.state + (size_t)n * prm.SS;
      const float* mass = st + prm.S * D;
      put_stack<D, SP>(et, [&](int d, int s) {
        return s < prm.S ? st[s * D + d] / (mass[s] + prm.eps) : 0.f;
      });
      cur_n = n;
    }
    const T* qb = static_cast<const T*>(prm.q) + stream_offset(prm.lq, n, prm.B, prm.H);
    T* ob = static_cast<T*>(prm.out) + stream_offset(prm.lo, n, prm.B, prm.H);
    stage<T, D>(sm + LY::QX, qb, prm.lq.st, it.t0, it.t1);
    tiles::cp_commit();
    for (int i = 0; i < it.ntiles; ++i) {
      const int64_t tile0 = it.t0 + (int64_t)i * TT;
      float* X = sm + LY::QX + (i & 1) * Slot<D>::FLOATS;
      if (i + 1 < it.ntiles)
        stage<T, D>(sm + LY::QX + ((i + 1) & 1) * Slot<D>::FLOATS, qb, prm.lq.st, tile0 + TT,
                    it.t1);
      tiles::cp_commit();
      tiles::cp_wait<1>();
      if constexpr (F32) {
        __syncthreads();
        convert_one<D>(X);
      }
      fence_async_smem();
      __syncthreads();
      if (tid == 0) {
        fence_after();
        gemm_parts<PJ, 2, D / 16, D, D>(tbase + LY::C_PROJ, Slot<D>::part(X, 0),
                                        Slot<D>::part(X, 1), nullptr, F32 ? 2 : 1, ps, false);
        commit(bar);
      }
      T5_CHECK(bar_wait(bar, phase));
      phase ^= 1;
      if (failed) break;
      fence_after();
      {
        float proj[PJ], h[PJ], p[SP];
        tld_sum<PJ>(tlane + LY::C_PROJ, PJ, proj);
        token_probs<K, SP>(proj, L, inv_scale, p, h);
        put_row<SP>(pq, pq + TT * SP, p);
      }
      fence_async_smem();
      fence_before();
      __syncthreads();
      if (tid == 0) {
        fence_after();
        gemm_parts<D, 2, SP / 16, SP, SP>(tbase + LY::C_OUT, pq, pq + TT * SP, nullptr, 2, et,
                                          false);
        commit(bar);
      }
      T5_CHECK(bar_wait(bar, phase));
      phase ^= 1;
      if (failed) break;
      fence_after();
      {
        float o[D];
        tld_sum<D>(tlane + LY::C_OUT, D, o);
        const int64_t t = tile0 + tid;
        if (t < it.t1) store_row<T, D>(ob + t * prm.lo.st, o);
      }
      fence_before();
    }
    tiles::cp_wait<0>();
  }
  tiles::cp_wait<0>();
  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 0) tmem_free<LY::TCOLS>(tbase);
}

// ------------------------------------------------------------------ B2 key/value backward
// dv = pK . dB,  dpK = v . dB^T + dA,  dk = dproj(pK, dpK) . P;  the k-side dscale.
template <typename T, int D, int SPAD, int K>
__global__ void __launch_bounds__(NT, 1) k_t5_bwd_kv(const Params prm) {
  using LY = BwdKVLay<D, SPAD>;
  constexpr int SP = LY::SP;
  constexpr bool F32 = sizeof(T) == 4;
  extern __shared__ __align__(128) float sm[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + LY::BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + LY::BAR + 2);
  bf16* pk = reinterpret_cast<bf16*>(sm + LY::PK);
  bf16* dj = reinterpret_cast<bf16*>(sm + LY::DJ);
  bf16* ps = reinterpret_cast<bf16*>(sm + LY::PS);
  bf16* pt = reinterpret_cast<bf16*>(sm + LY::PT);
  bf16* db = reinterpret_cast<bf16*>(sm + LY::DB);
  bf16* dbt = reinterpret_cast<bf16*>(sm + LY::DBT);
  const int tid = threadIdx.x, warp = tid >> 5;
  const float inv_scale = 1.f / __ldg(prm.scale);
  const int L = prm.L;
  const int items = prm.N * prm.P;
  if ((int)blockIdx.x >= items) return;
  if (tid == 0) bar_init(bar);
  if (warp == 0) tmem_alloc<LY::TCOLS>(tslot);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tbase = *tslot;
  const uint32_t tlane = tbase + ((uint32_t)(warp * 32) << 16);
  uint32_t phase = 0;
  bool failed = false;
  int cur_n = -1, cur_m = -1;
  float* dA = sm + LY::DA;
  for (int w = blockIdx.x; w < items && !failed; w += gridDim.x) {
    const Item it = item_of(prm, w);
    const int n = it.n;
    float ds = 0.f;
    if (it.ntiles > 0) {
      const int m = prm.Mp == 1 ? 0 : n / (prm.B * prm.H);
      __syncthreads();
      if (m != cur_m) {
        const float* pl = prm.planes + (size_t)m * prm.LK * D;
        put_stack<PJ, D>(ps, [&](int j, int d) { return j < prm.LK ? pl[j * D + d] : 0.f; });
        put_stack<D, PJ>(pt, [&](int d, int j) { return j < prm.LK ? pl[j * D + d] : 0.f; });
        cur_m = m;
      }
      if (n != cur_n) {
        const float* st = prm.state + (size_t)n * prm.SS;
        const float* gs = prm.gstate_in + (size_t)n * prm.SS;
        const float* mass = st + prm.S * D;
        // dB = dE / (A + eps);  dA_s = -sum_d dE_sd B_sd / (A_s + eps)^2
        put_stack<SP, D, 3>(db, [&](int s, int d) {
          return s < prm.S ? gs[s * D + d] / (mass[s] + prm.eps) : 0.f;
        });
        put_stack<D, SP>(dbt, [&](int d, int s) {
          return s < prm.S ? gs[s * D + d] / (mass[s] + prm.eps) : 0.f;
        });
        if (tid < 32) {
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
      float dAr[SP];
#pragma unroll
      for (int s = 0; s < SP; ++s) dAr[s] = s < 32 ? dA[s] : 0.f;
      const T* kb = static_cast<const T*>(prm.k) + stream_offset(prm.lk, n, prm.B, prm.H);
      const T* vb = static_cast<const T*>(prm.v) + stream_offset(prm.lv, n, prm.B, prm.H);
      T* dkb = static_cast<T*>(prm.dk) + stream_offset(prm.ldk, n, prm.B, prm.H);
      T* dvb = static_cast<T*>(prm.dv) + stream_offset(prm.ldv, n, prm.B, prm.H);
      stage<T, D>(sm + LY::KX, kb, prm.lk.st, it.t0, it.t1);
      stage<T, D>(sm + LY::VX, vb, prm.lv.st, it.t0, it.t1);
      tiles::cp_commit();
      for (int i = 0; i < it.ntiles; ++i) {
        const int64_t tile0 = it.t0 + (int64_t)i * TT;
        float* KXt = sm + LY::KX + (i & 1) * Slot<D>::FLOATS;
        float* VXt = sm + LY::VX + (i & 1) * Slot<D, 3>::FLOATS;
        if (i + 1 < it.ntiles) {
          stage<T, D>(sm + LY::KX + ((i + 1) & 1) * Slot<D>::FLOATS, kb, prm.lk.st, tile0 + TT,
                      it.t1);
          stage<T, D>(sm + LY::VX + ((i + 1) & 1) * Slot<D, 3>::FLOATS, vb, prm.lv.st, tile0 + TT,
                      it.t1);
        }
        tiles::cp_commit();
        tiles::cp_wait<1>();
        if constexpr (F32) {
          __syncthreads();
          convert_two<D>(KXt, VXt);
        }
        fence_async_smem();
        __syncthreads();
        // projections and dpK = v . dB^T
        if (tid == 0) {
          fence_after();
          gemm_parts<PJ, 2, D / 16, D, D>(tbase + LY::C_PROJ, Slot<D>::part(KXt, 0),
                                          Slot<D>::part(KXt, 1), nullptr, F32 ? 2 : 1, ps, false);
          // dpK carries three parts on both sides: where v matches a bucket's
          // mean (tiny buckets), v . dB and dA cancel to far below |v| |dB|
          gemm_parts<SP, 3, D / 16, D, D>(tbase + LY::C_DPK, Slot<D, 3>::part(VXt, 0),
                                          Slot<D, 3>::part(VXt, 1), Slot<D, 3>::part(VXt, 2),
                                          F32 ? 3 : 1, db, false);
          commit(bar);
        }
        T5_CHECK(bar_wait(bar, phase));
        phase ^= 1;
        if (failed) break;
        fence_after();
        {
          float proj[PJ], h[PJ], p[SP], g[SP], dj_[PJ];
          tld_sum<PJ>(tlane + LY::C_PROJ, PJ, proj);
          tld_sum<SP, 3>(tlane + LY::C_DPK, SP, g);
#pragma unroll
          for (int s = 0; s < SP; ++s) g[s] += dAr[s];
          token_probs<K, SP>(proj, L, inv_scale, p, h);
          float dsl = 0.f;
          token_probs_bwd<K, SP>(p, g, h, L, inv_scale, dj_, dsl);
          if (tile0 + tid < it.t1) ds += dsl;
          put_row<SP>(pk, pk + TT * SP, p);
          put_row<PJ>(dj, dj + TT * PJ, dj_);
        }
        fence_async_smem();
        fence_before();
        __syncthreads();
        if (tid == 0) {
          fence_after();
          gemm_parts<D, 2, SP / 16, SP, SP>(tbase + LY::C_DV, pk, pk + TT * SP, nullptr, 2, dbt,
                                            false);
          gemm_parts<D, 2, PJ / 16, PJ, PJ>(tbase + LY::C_DK, dj, dj + TT * PJ, nullptr, 2, pt,
                                            false);
          commit(bar);
        }
        T5_CHECK(bar_wait(bar, phase));
        phase ^= 1;
        if (failed) break;
        fence_after();
        {
          const int64_t t = tile0 + tid;
          float o[D];
          tld_sum<D>(tlane + LY::C_DV, D, o);
          if (t < it.t1) store_row<T, D>(dvb + t * prm.ldv.st, o);
          tld_sum<D>(tlane + LY::C_DK, D, o);
          if (t < it.t1) store_row<T, D>(dkb + t * prm.ldk.st, o);
        }
        fence_before();
      }
      tiles::cp_wait<0>();
    }
    // per-item dscale partial (zero for an empty range), fixed-order CTA sum
    float x = ds;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    __syncthreads();
    if ((tid & 31) == 0) sm[LY::RED + warp] = x;
    __syncthreads();
    if (tid == 0)
      prm.dscale_part[(size_t)n * prm.P + it.part] =
          (sm[LY::RED] + sm[LY::RED + 1]) + (sm[LY::RED + 2] + sm[LY::RED + 3]);
  }
  tiles::cp_wait<0>();
  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 0) tmem_free<LY::TCOLS>(tbase);
}

#undef T5_CHECK

}  // namespace t5
}  // namespace race
