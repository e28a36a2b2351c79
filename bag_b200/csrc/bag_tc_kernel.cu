// 3xTF32 tcgen05 leaf kernel of the BAG FP32 matmul (sm_100a), the
// error-compensated tensor-core variant.
//
// Every leaf product is computed as A_hi*B_hi + A_hi*B_lo + A_lo*B_hi where
// x_hi = rn_tf32(x) and x_lo = rn_tf32(x - x_hi) split each transformed
// operand element (the lo*lo term, below 2^-22 relative, is dropped).  The
// tensor core accumulates only 256-long K chunks; each finished chunk is added
// into an FP32 running sum with round-to-nearest on the CUDA cores, which keeps
// the error below an FP32 FFMA dot product's (a whole-K tensor-core accumulation
// grows with K instead).
//
// One CTA (288 threads) computes a 128 x 128 output tile of one product:
//  * warps 5-8 (producers) load every signed operand term two k-blocks ahead
//    (A: one row of 8 per thread, coalesced along m; B: 128-bit loads along
//    k), sum the terms in the reference's order (x + delta*y, bag.cuh:69-73),
//    split hi/lo and store the four 128 x 8 operand tiles of a k-block into a
//    6-stage shared-memory ring in the tensor core's canonical K-major
//    no-swizzle layout, then arrive on "full".  (TF32 operands are staged
//    K-major: an M-major no-swizzle A operand produced no output on B200.)
//  * warp 4 allocates 384 TMEM columns (two chunk accumulators and the running
//    sum) and one elected thread issues the three tcgen05.mma.kind::tf32 per
//    k-block into the current chunk buffer, committing "empty" (stage free)
//    and, at the end of a chunk, "chunk_full";
//  * warps 0-3 (one per TMEM lane quadrant, thread = output row) fold each
//    finished chunk into the running sum (tcgen05.ld/st), release the chunk
//    buffer, and finally add coef*sum into every target C block (red.global).
//
// All waits are bounded (kWaitLimitNs of wall time, then this file's device
// error word is set); on any timeout every role skips the rest of its work and meets the
// others at the final barrier, after the MMA thread has waited (bounded) for its
// outstanding MMAs, so TMEM is always freed.
#include <cuda_runtime.h>

#include <cstdint>

#include "bag_kernels.h"

namespace bag_b200 {

// This file's device error word (read by read_and_clear_tc_device_error).
__device__ unsigned int g_tc_device_error = 0;

namespace {

constexpr int kBM = 128, kBN = 128, kBK = 8, kStages = 6;
#ifndef BAG_TC_CHUNK_BLOCKS
#define BAG_TC_CHUNK_BLOCKS 4
#endif
// k-blocks per tensor-core accumulation chunk (K = 8 * kChunkBlocks).  The
// tensor core accumulates with round-toward-zero, so its error grows linearly
// with the chunk length; chunks are kept short and summed in FP32 with
// round-to-nearest (Ootomo & Yokota 2022, sec. 4).
constexpr int kChunkBlocks = BAG_TC_CHUNK_BLOCKS;
constexpr int kEpiThreads = 128, kProdThreads = 128;
constexpr int kThreads = kEpiThreads + 32 + kProdThreads;   // 288
constexpr int kMmaWarp = 4;
constexpr unsigned kTmemCols = 512;   // power of two >= 3 x 128 columns
constexpr unsigned kSuspendNs = 1000000;
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

// Instruction descriptor: F32 accumulate, TF32 A and B, both K-major,
// N = 128, M = 128 (bits: c_format[4,6)=1, a_format[7,10)=2, b_format[10,13)=2,
// a_major[15]=b_major[16]=0, n_dim[17,23)=N/8, m_dim[24,29)=M/16).
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) |
                            (uint32_t(kBN >> 3) << 17) | (uint32_t(kBM >> 4) << 24);

struct TcSmem {
  // Per stage: four 128 x 8 TF32 tiles of 4 KB each, K-major without swizzle:
  // core matrices of 8 rows x 4 k (16 B rows), element (r, k) of a tile at byte
  // (r/8)*256 + (k/4)*128 + (r%8)*16 + (k%4)*4 (r = m for A, n for B).
  float a_hi[kStages][kBM * kBK];
  float a_lo[kStages][kBM * kBK];
  float b_hi[kStages][kBN * kBK];
  float b_lo[kStages][kBN * kBK];
  unsigned long long full[kStages];
  unsigned long long empty[kStages];
  unsigned long long chunk_full[2];
  unsigned long long chunk_empty[2];
  unsigned long long mma_done;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(unsigned long long* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(unsigned long long* bar) {
  unsigned long long state;
  asm volatile("mbarrier.arrive.shared::cta.b64 %0, [%1];"
               : "=l"(state)
               : "r"(smem_u32(bar))
               : "memory");
  (void)state;
}

__device__ __forceinline__ bool mbar_try_wait(unsigned long long* bar, unsigned parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendNs)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait; on timeout sets the error word and the CTA's abort flag.
__device__ __forceinline__ bool mbar_wait(TcSmem& sm, unsigned long long* bar, unsigned parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long start = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_ns() - start > kWaitLimitNs || *(volatile int*)&sm.abort) {
      atomicOr(&g_tc_device_error, 1u);
      *(volatile int*)&sm.abort = 1;
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor, no swizzle: start, leading and stride byte
// offsets in 16-byte units, version 1 (bit 46).
__device__ __forceinline__ uint64_t smem_desc(const void* p, uint32_t lbo, uint32_t sbo) {
  const uint32_t addr = smem_u32(p);
  return uint64_t((addr >> 4) & 0x3FFF) | (uint64_t((lbo >> 4) & 0x3FFF) << 16) |
         (uint64_t((sbo >> 4) & 0x3FFF) << 32) | (uint64_t(1) << 46);
}

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         bool accumulate) {
  const uint32_t acc = accumulate ? 1u : 0u;
  const uint32_t zero = 0u;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}"
      :
      : "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(kIdesc), "r"(acc), "r"(zero)
      : "memory");
}

__device__ __forceinline__ void mma_commit(unsigned long long* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

__device__ __forceinline__ float tf32_rn(float x) {
  uint32_t u;
  asm("cvt.rn.tf32.f32 %0, %1;" : "=r"(u) : "f"(x));
  return __uint_as_float(u);
}

__device__ __forceinline__ float4 split_hi(float4 v) {
  return make_float4(tf32_rn(v.x), tf32_rn(v.y), tf32_rn(v.z), tf32_rn(v.w));
}
__device__ __forceinline__ float4 split_lo(float4 v, float4 hi) {
  return make_float4(tf32_rn(v.x - hi.x), tf32_rn(v.y - hi.y), tf32_rn(v.z - hi.z),
                     tf32_rn(v.w - hi.w));
}

__device__ __forceinline__ const Prod& find_prod(const LeafPlan& plan, int item) {
  int pid = 0;
  while (pid + 1 < plan.nprod && plan.prod[pid + 1].tile_begin <= item) ++pid;
  return plan.prod[pid];
}

__device__ __forceinline__ float4 ldg4(const float* p) {
  return __ldg(reinterpret_cast<const float4*>(p));
}

__device__ __forceinline__ float4 add_signed(float4 acc, float4 v, float coef) {
  return make_float4(fmaf(coef, v.x, acc.x), fmaf(coef, v.y, acc.y), fmaf(coef, v.z, acc.z),
                     fmaf(coef, v.w, acc.w));
}

__device__ __forceinline__ float4 signed_first(float4 v, float coef) {
  return coef < 0.f ? make_float4(-v.x, -v.y, -v.z, -v.w) : v;
}

// Producer thread p (0..127) stages, per k-block, row p of the A tile (its 8
// k values as two 4-vectors, q = k/4; scalar loads, coalesced along m across
// the warp) and the B vectors (k-chunk kc of column n) for
// n = (idx/16)*8 + idx%8, kc = (idx/8)%2 with idx = p and p+128.  Every 16-byte
// shared store of a quarter warp covers 128 contiguous bytes (no conflicts).
template <int NL, int NR>
__device__ __forceinline__ void produce(const LeafPlan& plan, const Prod& P, int m0, int n0,
                                        long long batch, TcSmem& sm, int p, int kblocks) {
  int bn[2], bkc[2];
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int idx = p + 128 * q;
    bn[q] = (idx / 16) * 8 + idx % 8;
    bkc[q] = (idx / 8) % 2;
  }
  const long long lda = plan.terms[P.l0].ld, ldb = plan.terms[P.r0].ld;
  const float* ba[NL];
  float ca[NL];
#pragma unroll
  for (int t = 0; t < NL; ++t) {
    const Term& T = plan.terms[P.l0 + t];
    ba[t] = T.p + batch * T.bstride;
    ca[t] = T.coef;
  }
  const float* bb[NR];
  float cb[NR];
#pragma unroll
  for (int t = 0; t < NR; ++t) {
    const Term& T = plan.terms[P.r0 + t];
    bb[t] = T.p + batch * T.bstride;
    cb[t] = T.coef;
  }
  // Clamped addresses: rows >= m and columns >= n are loaded but never stored.
  long long oa = min(m0 + p, P.m - 1), ob[2];
#pragma unroll
  for (int q = 0; q < 2; ++q) ob[q] = 4 * bkc[q] + (long long)min(n0 + bn[q], P.n - 1) * ldb;
  const int kfull = P.k / kBK;
  const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);

  float4 la[2][NL][2], lb[2][NR][2];
  auto load = [&](float4 (&xa)[NL][2], float4 (&xb)[NR][2], int kb) {
    const bool full_tile = kb < kfull;
    const int k0 = kb * kBK;
#pragma unroll
    for (int t = 0; t < NL; ++t) {
      const float* col = ba[t] + oa;
      float e[kBK];
#pragma unroll
      for (int j = 0; j < kBK; ++j)
        e[j] = (full_tile || k0 + j < P.k) ? __ldg(col + (long long)j * lda) : 0.f;
      xa[t][0] = make_float4(e[0], e[1], e[2], e[3]);
      xa[t][1] = make_float4(e[4], e[5], e[6], e[7]);
    }
    oa += kBK * lda;
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const bool bv = full_tile || k0 + 4 * bkc[q] < P.k;
#pragma unroll
      for (int t = 0; t < NR; ++t) xb[t][q] = bv ? ldg4(bb[t] + ob[q]) : z;
      ob[q] += kBK;
    }
  };
  auto store = [&](const float4 (&xa)[NL][2], const float4 (&xb)[NR][2], int s) {
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      float4 v = signed_first(xa[0][q], ca[0]);
#pragma unroll
      for (int t = 1; t < NL; ++t) v = add_signed(v, xa[t][q], ca[t]);
      const float4 hi = split_hi(v);
      const int off = (p / 8) * 64 + q * 32 + (p % 8) * 4;   // floats
      *reinterpret_cast<float4*>(&sm.a_hi[s][off]) = hi;
      *reinterpret_cast<float4*>(&sm.a_lo[s][off]) = split_lo(v, hi);
    }
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      float4 v = signed_first(xb[0][q], cb[0]);
#pragma unroll
      for (int t = 1; t < NR; ++t) v = add_signed(v, xb[t][q], cb[t]);
      const float4 hi = split_hi(v);
      const int off = (bn[q] / 8) * 64 + bkc[q] * 32 + (bn[q] % 8) * 4;   // floats
      *reinterpret_cast<float4*>(&sm.b_hi[s][off]) = hi;
      *reinterpret_cast<float4*>(&sm.b_lo[s][off]) = split_lo(v, hi);
    }
  };
  auto publish = [&](const float4 (&xa)[NL][2], const float4 (&xb)[NR][2], int kb) {
    const int s = kb % kStages;
    if (kb >= kStages && !mbar_wait(sm, &sm.empty[s], ((kb / kStages) - 1) & 1)) return false;
    store(xa, xb, s);
    // The tensor core reads these tiles through the async proxy.
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_arrive(&sm.full[s]);
    return true;
  };
  if (kblocks > 0) load(la[0], lb[0], 0);
  if (kblocks > 1) load(la[1], lb[1], 1);
  for (int kb = 0; kb < kblocks; kb += 2) {
    if (!publish(la[0], lb[0], kb)) return;
    if (kb + 2 < kblocks) load(la[0], lb[0], kb + 2);
    if (kb + 1 < kblocks) {
      if (!publish(la[1], lb[1], kb + 1)) return;
      if (kb + 3 < kblocks) load(la[1], lb[1], kb + 3);
    }
  }
}

// Single elected thread of the MMA warp.
__device__ __forceinline__ void issue_mmas(TcSmem& sm, uint32_t tmem, int kblocks) {
  int issued = 0;
  for (int kb = 0; kb < kblocks; ++kb) {
    const int chunk = kb / kChunkBlocks, in_chunk = kb % kChunkBlocks;
    const int buf = chunk & 1;
    if (in_chunk == 0 && chunk >= 2 && !mbar_wait(sm, &sm.chunk_empty[buf], ((chunk >> 1) - 1) & 1))
      break;
    const int s = kb % kStages;
    if (!mbar_wait(sm, &sm.full[s], (kb / kStages) & 1)) break;
    tc_fence_after();
    const uint32_t d = tmem + uint32_t(buf * kBN);
    // A and B: 8-row groups 256 B apart (SBO), the two K halves 128 B apart (LBO).
    const uint64_t ahi = smem_desc(sm.a_hi[s], 128, 256);
    const uint64_t alo = smem_desc(sm.a_lo[s], 128, 256);
    const uint64_t bhi = smem_desc(sm.b_hi[s], 128, 256);
    const uint64_t blo = smem_desc(sm.b_lo[s], 128, 256);
    mma_tf32(d, ahi, bhi, in_chunk > 0);
    mma_tf32(d, ahi, blo, true);
    mma_tf32(d, alo, bhi, true);
    mma_commit(&sm.empty[s]);
    ++issued;
    if (in_chunk == kChunkBlocks - 1 || kb == kblocks - 1) mma_commit(&sm.chunk_full[buf]);
  }
  // Drain: all issued MMAs must finish before TMEM is released.
  mma_commit(&sm.mma_done);
  mbar_wait(sm, &sm.mma_done, 0);
  (void)issued;
}

// Epilogue warps 0-3: thread = TMEM lane = output row of the tile.
__device__ __forceinline__ bool fold_chunks(TcSmem& sm, uint32_t tmem, int kblocks) {
  const int warp = threadIdx.x >> 5;
  const uint32_t lane_base = uint32_t(warp * 32) << 16;
  const uint32_t total = tmem + lane_base + uint32_t(2 * kBN);
  const int chunks = (kblocks + kChunkBlocks - 1) / kChunkBlocks;
  for (int c = 0; c < chunks; ++c) {
    const int buf = c & 1;
    // Warp-uniform outcome: the tcgen05.ld/st below are warp-collective.
    const bool ok = mbar_wait(sm, &sm.chunk_full[buf], (c >> 1) & 1);
    if (!__all_sync(0xffffffffu, ok)) return false;
    tc_fence_after();
    const uint32_t chunk = tmem + lane_base + uint32_t(buf * kBN);
#pragma unroll 1
    for (int piece = 0; piece < kBN / 32; ++piece) {
      float v[32];
      tmem_ld32(chunk + piece * 32, v);
      if (c > 0) {
        float t[32];
        tmem_ld32(total + piece * 32, t);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __fadd_rn(t[i], v[i]);
      } else {
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      }
      tmem_st32(total + piece * 32, v);
    }
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    tc_fence_before();
    mbar_arrive(&sm.chunk_empty[buf]);
  }
  return true;
}

__device__ __forceinline__ void store_outputs(const LeafPlan& plan, const Prod& P, int m0, int n0,
                                              long long batch, uint32_t tmem) {
  const int warp = threadIdx.x >> 5;
  const int row = warp * 32 + (threadIdx.x & 31);
  const uint32_t total = tmem + (uint32_t(warp * 32) << 16) + uint32_t(2 * kBN);
  const int r = m0 + row;
#pragma unroll 1
  for (int piece = 0; piece < kBN / 32; ++piece) {
    float v[32];
    tmem_ld32(total + piece * 32, v);
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
    if (r >= P.m) continue;
    for (int o = 0; o < P.no; ++o) {
      const Term& T = plan.terms[P.o0 + o];
      float* base = const_cast<float*>(T.p) + batch * T.bstride + r;
      const float coef = T.coef;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int col = n0 + piece * 32 + i;
        if (col >= P.n) break;
        float* q = base + (long long)col * T.ld;
        if (T.mode == kOutAtomic) atomicAdd(q, coef * v[i]);
        else if (T.mode == kOutAdd) *q += coef * v[i];
        else *q = coef * v[i];
      }
    }
  }
}

}  // namespace

__global__ void __launch_bounds__(kThreads, 1) leaf_tc_kernel(const __grid_constant__ LeafPlan plan) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  TcSmem& sm = *reinterpret_cast<TcSmem*>(smem_raw);
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], kProdThreads);
      mbar_init(&sm.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.chunk_full[b], 1);
      mbar_init(&sm.chunk_empty[b], kEpiThreads);
    }
    mbar_init(&sm.mma_done, 1);
    sm.abort = 0;
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&sm.tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  const Prod& P = find_prod(plan, blockIdx.x);
  const int local = blockIdx.x - P.tile_begin;
  constexpr int GROUP_M = 8;
  const int in_group = GROUP_M * P.tiles_n;
  const int first_m = (local / in_group) * GROUP_M;
  const int gsize = min(P.tiles_m - first_m, GROUP_M);
  const int m0 = (first_m + (local % in_group) % gsize) * kBM;
  const int n0 = ((local % in_group) / gsize) * kBN;
  const long long batch = blockIdx.y;
  const int kblocks = (P.k + kBK - 1) / kBK;

  if (warp > kMmaWarp) {
    const int p = threadIdx.x - (kEpiThreads + 32);
    switch (P.sig) {
      case kSig11: produce<1, 1>(plan, P, m0, n0, batch, sm, p, kblocks); break;
      case kSig12: produce<1, 2>(plan, P, m0, n0, batch, sm, p, kblocks); break;
      case kSig21: produce<2, 1>(plan, P, m0, n0, batch, sm, p, kblocks); break;
      case kSig22: produce<2, 2>(plan, P, m0, n0, batch, sm, p, kblocks); break;
      case kSig33: produce<3, 3>(plan, P, m0, n0, batch, sm, p, kblocks); break;
      case kSig41: produce<4, 1>(plan, P, m0, n0, batch, sm, p, kblocks); break;
      case kSig14: produce<1, 4>(plan, P, m0, n0, batch, sm, p, kblocks); break;
      default:
        atomicOr(&g_tc_device_error, 2u);
        *(volatile int*)&sm.abort = 1;
        break;
    }
  } else if (warp == kMmaWarp) {
    if (P.sig != kSigGeneric && (threadIdx.x & 31) == 0) issue_mmas(sm, tmem, kblocks);
    __syncwarp();
  } else {
    bool ok = P.sig != kSigGeneric;
    if (ok && kblocks > 0) ok = fold_chunks(sm, tmem, kblocks);
    if (ok) {
      if (kblocks == 0) {   // empty reduction: the sum is zero
        float zero[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) zero[i] = 0.f;
        const uint32_t total = tmem + (uint32_t(warp * 32) << 16) + uint32_t(2 * kBN);
        for (int piece = 0; piece < kBN / 32; ++piece) tmem_st32(total + piece * 32, zero);
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      }
      if (!*(volatile int*)&sm.abort) store_outputs(plan, P, m0, n0, batch, tmem);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

TileShape tc_tile_shape() { return {kBM, kBN}; }

cudaError_t read_and_clear_tc_device_error(unsigned* value) {
  cudaError_t e = cudaMemcpyFromSymbol(value, g_tc_device_error, sizeof(unsigned));
  if (e != cudaSuccess) return e;
  const unsigned zero = 0;
  return cudaMemcpyToSymbol(g_tc_device_error, &zero, sizeof(unsigned));
}

// Dynamic shared memory per CTA: the ring, padded past half of the SM's 228 KB
// so that only one CTA (and one 512-column TMEM allocation) fits per SM.
constexpr int kTcSmemBytes = sizeof(TcSmem) > 120 * 1024 ? int(sizeof(TcSmem)) : 120 * 1024;

cudaError_t launch_leaf_tc(const LeafPlan& plan, int batch, cudaStream_t stream) {
  if (plan.nprod == 0 || plan.ntiles == 0 || batch == 0) return cudaSuccess;
  // The attribute is per device: set it before every launch (cheap).
  cudaError_t e = cudaFuncSetAttribute(leaf_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kTcSmemBytes);
  if (e != cudaSuccess) return e;
  leaf_tc_kernel<<<dim3(plan.ntiles, batch), kThreads, kTcSmemBytes, stream>>>(plan);
  return cudaGetLastError();
}

}  // namespace bag_b200
