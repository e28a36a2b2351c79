// 3xTF32 tcgen05 leaf kernel of the BAG FP32 matmul (sm_100a), the
// error-compensated tensor-core variant.
//
// Every leaf product is computed as A_hi*B_hi + A_hi*B_lo + A_lo*B_hi where
// x_hi = rn_tf32(x) and x_lo = rn_tf32(x - x_hi) split each transformed
// operand element (the lo*lo term, below 2^-22 relative, is dropped).  The
// tensor core accumulates with round-toward-zero, so it only sums 32-long K
// chunks; each finished chunk is added into an FP32 running sum with
// round-to-nearest on the CUDA cores (Ootomo & Yokota 2022, "Recovering single
// precision accuracy from Tensor Cores while surpassing the FP32 theoretical
// peak performance", sec. 4).  Measured error: 0.3-0.6x an FP32 FFMA dot
// product's for K >= 1024.
//
// One CTA (576 threads, 227 KB shared memory, 1 per SM) computes a 128 x 128
// output tile of one product; the K loop runs in stages of 32 k (products of
// up to five operand terms) or 16 k (more terms: their raw stages are larger):
//  * warp 8, lane 0 (producer): TMA-loads the raw FP32 tile of every signed
//    operand term of the stage (A term: boxes of 128 m x 16 k, M-contiguous;
//    B term: boxes of 16 k x 128 n with 64-byte swizzle) into a ring of raw
//    stages whose depth is sized per product.  Tensor maps come from the host:
//    one per source matrix (A, B) addressed by block coordinates, one per
//    workspace block.  Warp 8 also owns TMEM.
//  * warps 0-3 (A side; thread = tile row = TMEM lane): sum the A terms in the
//    reference's order (x + delta*y, bag.cuh:69-73), zero the K tail, split
//    hi/lo and store them into a TMEM A slot (tcgen05.st).
//  * warps 4-7 (B side; thread = tile column): sum, split and store the B terms
//    as K-major no-swizzle hi/lo tiles in a shared-memory ring.
//  * warp 9, lane 0: per K-step of 8 issues three tcgen05.mma.kind::tf32 with A
//    from TMEM and B from shared memory into the chunk's TMEM accumulator;
//    commits free the A slot, the B stage and, at the end of a 32-k chunk,
//    publish the chunk.
//  * warps 10-17 (fold; two per TMEM lane quadrant, 64 columns each): add each
//    finished chunk into 64 running sums held in registers, then add coef*sum
//    into every target C block (red.global, coalesced along the column).
// TMEM columns: [0, 256) two chunk accumulators, [256, 512) the A slots
// (four of 32 k or eight of 16 k, hi then lo).
//
// All waits are bounded (kWaitLimitNs of wall time, then this file's device
// error word is set and the CTA's abort flag raised); on a timeout every role
// skips the rest of its work and meets the others at the final barrier, after
// the producer has waited (bounded) for its copies in flight and the MMA thread
// for its MMAs, so TMEM is always freed and no copy outlives the CTA.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <cstring>
#include <vector>

#include "bag_kernels.h"

namespace bag_b200 {

// This file's device error word (read by read_and_clear_tc_device_error).
__device__ unsigned int g_tc_device_error = 0;

namespace {

constexpr int kBM = 128, kBN = 128;
// k per pipeline stage: 32 (four MMA K-steps of 8) for products with at most
// four operand terms, 16 otherwise (their raw stages are larger).
constexpr int kChunkK = 32;        // k per tensor-core accumulation chunk
constexpr int kMaxRaw = 12;        // raw operand stages, upper bound
constexpr int kTmaWarp = 8, kMmaWarp = 9, kFoldWarp0 = 10, kFoldWarps = 8;
constexpr int kThreads = (kFoldWarp0 + kFoldWarps) * 32;   // 576
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColA = 256, kColsA = 256;   // chunk accumulators in [0, 256)
constexpr int kBRegion = 65536;    // shared-memory ring of B hi/lo stages
constexpr int kBoxBytes = 128 * 16 * 4;   // one TMA box: 128 m x 16 k or 16 k x 128 n
constexpr int kSmemBytes = 232448;        // 227 KB, the sm_100 per-CTA maximum
constexpr unsigned kSuspendNs = 1000000;
constexpr unsigned long long kWaitLimitNs = 2000000000ull;
constexpr int kMaxMaps = 64;

// Instruction descriptor: F32 accumulate, TF32 A and B, both K-major,
// N = 128, M = 128 (bits: c_format[4,6)=1, a_format[7,10)=2, b_format[10,13)=2,
// a_major[15]=b_major[16]=0, n_dim[17,23)=N/8, m_dim[24,29)=M/16).
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) |
                            (uint32_t(kBN >> 3) << 17) | (uint32_t(kBM >> 4) << 24);

struct TcShared {
  // B stage s (KS k) at b_region + s*KS*1024: KS/8 hi tiles then KS/8 lo
  // tiles of 4 KB, one per MMA K-step, K-major without swizzle: core matrices
  // of 8 rows x 4 k (16-byte rows), element (n, k) at byte
  // (n/8)*256 + (k/4)*128 + (n%8)*16 + (k%4)*4 of its tile.
  unsigned char b_region[kBRegion];
  unsigned long long raw_full[kMaxRaw], raw_empty[kMaxRaw];
  unsigned long long a_full[8], a_empty[8];
  unsigned long long b_full[4], b_empty[4];
  unsigned long long chunk_full[2], chunk_empty[2];
  unsigned long long mma_done;
  uint32_t tmem_base;
  int abort;
};
constexpr int kRawOffset = (int(sizeof(TcShared)) + 1023) / 1024 * 1024;
constexpr int kRawBytes = kSmemBytes - kRawOffset;
// Two raw stages of the largest product: 4 terms x 32 k, or 8 terms x 16 k.
static_assert(kRawBytes >= 2 * 2 * kMaxOperandTerms * 16 * kBM * 4, "raw ring too small");

// Kernel-parameter tensor maps: operand term i of the plan is read through
// map[op_map[i] & 0xffff] at block origin (op_x[i], op_y[i]); bit 16 of
// op_map marks an operand shared by every batch entry (batch coordinate 0).
struct alignas(64) TcMaps {
  CUtensorMap map[kMaxMaps];
  int op_map[kMaxTerms];
  int op_x[kMaxTerms];
  int op_y[kMaxTerms];
};
static_assert(sizeof(LeafPlan) + sizeof(TcMaps) + 64 <= 32764, "kernel parameters too large");

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(unsigned long long* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(unsigned long long* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(unsigned long long* bar, int bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
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

// Bounded wait; on timeout (or when another role gave up) sets the error word
// and the CTA's abort flag and returns false.
__device__ __forceinline__ bool mbar_wait(TcShared& sm, unsigned long long* bar, unsigned parity) {
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

// Bounded wait that ignores the abort flag: for copies and MMAs already in
// flight, which must land before the CTA exits.
__device__ __forceinline__ void mbar_drain(unsigned long long* bar, unsigned parity) {
  if (mbar_try_wait(bar, parity)) return;
  const unsigned long long start = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_ns() - start > kWaitLimitNs) {
      atomicOr(&g_tc_device_error, 1u);
      return;
    }
  }
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z,
                                            unsigned long long* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// Shared-memory matrix descriptor, no swizzle: start, leading and stride byte
// offsets in 16-byte units, version 1 (bit 46).
__device__ __forceinline__ uint64_t smem_desc(const void* p, uint32_t lbo, uint32_t sbo) {
  const uint32_t addr = smem_u32(p);
  return uint64_t((addr >> 4) & 0x3FFF) | (uint64_t((lbo >> 4) & 0x3FFF) << 16) |
         (uint64_t((sbo >> 4) & 0x3FFF) << 32) | (uint64_t(1) << 46);
}

// D[tmem] (+)= A[tmem] * B[smem]^T, one K-step of 8.
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                       bool accumulate) {
  const uint32_t acc = accumulate ? 1u : 0u;
  const uint32_t zero = 0u;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}"
      :
      : "r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(kIdesc), "r"(acc), "r"(zero)
      : "memory");
}

__device__ __forceinline__ void mma_commit(unsigned long long* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
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

__device__ __forceinline__ float4 add_signed(float4 acc, float4 v, float coef) {
  return make_float4(fmaf(coef, v.x, acc.x), fmaf(coef, v.y, acc.y), fmaf(coef, v.z, acc.z),
                     fmaf(coef, v.w, acc.w));
}

__device__ __forceinline__ float4 signed_first(float4 v, float coef) {
  return coef < 0.f ? make_float4(-v.x, -v.y, -v.z, -v.w) : v;
}

// Position in a ring of n stages: slot index and the parity of its current use.
struct Ring {
  int idx = 0;
  unsigned phase = 0;
  __device__ __forceinline__ void next(int n) {
    if (++idx == n) {
      idx = 0;
      phase ^= 1u;
    }
  }
};

__device__ __forceinline__ const Prod& find_prod(const LeafPlan& plan, int item) {
  int pid = 0;
  while (pid + 1 < plan.nprod && plan.prod[pid + 1].tile_begin <= item) ++pid;
  return plan.prod[pid];
}

// ---- producer (warp 8, lane 0) --------------------------------------------
// Stage s of `ks` k: per left term ks/16 boxes {128 m, 16 k}, per right term
// ks/16 boxes {16 k, 128 n}, each term's boxes contiguous in the slot.
__device__ void run_producer(TcShared& sm, unsigned char* raw, const TcMaps& maps, const Prod& P,
                             int m0, int n0, int batch, int nraw, int slot_bytes, int stages,
                             int ks) {
  const int boxes = ks / 16, term_bytes = boxes * kBoxBytes;
  int issued = 0;
  Ring r;
  for (int s = 0; s < stages; ++s, r.next(nraw)) {
    const int slot = r.idx;
    if (s >= nraw && !mbar_wait(sm, &sm.raw_empty[slot], r.phase ^ 1u)) break;
    unsigned char* dst = raw + slot * slot_bytes;
    mbar_expect_tx(&sm.raw_full[slot], slot_bytes);
    const int k0 = s * ks;
    for (int t = 0; t < P.nl; ++t) {
      const int ti = P.l0 + t, id = maps.op_map[ti], z = (id >> 16) ? 0 : batch;
      for (int b = 0; b < boxes; ++b)
        tma_load_3d(dst + t * term_bytes + b * kBoxBytes, &maps.map[id & 0xffff],
                    maps.op_x[ti] + m0, maps.op_y[ti] + k0 + 16 * b, z, &sm.raw_full[slot]);
    }
    for (int t = 0; t < P.nr; ++t) {
      const int ti = P.r0 + t, id = maps.op_map[ti], z = (id >> 16) ? 0 : batch;
      for (int b = 0; b < boxes; ++b)
        tma_load_3d(dst + (P.nl + t) * term_bytes + b * kBoxBytes, &maps.map[id & 0xffff],
                    maps.op_x[ti] + k0 + 16 * b, maps.op_y[ti] + n0, z, &sm.raw_full[slot]);
    }
    ++issued;
  }
  // No copy may outlive the CTA: wait for the latest phase of every slot that
  // still has one in flight (the earlier phases of a slot completed before the
  // consumers released it).
  for (int s = max(0, issued - nraw); s < issued; ++s) mbar_drain(&sm.raw_full[s % nraw], (s / nraw) & 1);
}

// ---- MMA issuer (warp 9, lane 0) ------------------------------------------
template <int KS>
__device__ void run_mma(TcShared& sm, uint32_t tmem, int stages) {
  constexpr int kSteps = KS / 8, kNA = kColsA / (2 * KS), kNB = kBRegion / (KS * 1024);
  constexpr int kCS = kChunkK / KS;   // stages per accumulation chunk
  Ring ra, rb;
  for (int s = 0; s < stages; ++s, ra.next(kNA), rb.next(kNB)) {
    const int c = s / kCS, buf = c & 1;
    const bool first = s % kCS == 0;
    if (first && c >= 2 && !mbar_wait(sm, &sm.chunk_empty[buf], ((c >> 1) - 1) & 1)) break;
    if (!mbar_wait(sm, &sm.a_full[ra.idx], ra.phase)) break;
    if (!mbar_wait(sm, &sm.b_full[rb.idx], rb.phase)) break;
    tc_fence_after();
    const uint32_t d = tmem + uint32_t(buf * kBN);
    const unsigned char* bst = sm.b_region + rb.idx * KS * 1024;
#pragma unroll
    for (int j = 0; j < kSteps; ++j) {
      const uint32_t a_hi = tmem + kColA + uint32_t(ra.idx * 2 * KS + j * 8);
      const uint32_t a_lo = a_hi + KS;
      // B tiles: 8-row groups 256 B apart (SBO), the two K halves 128 B apart (LBO).
      const uint64_t b_hi = smem_desc(bst + j * 4096, 128, 256);
      const uint64_t b_lo = smem_desc(bst + (kSteps + j) * 4096, 128, 256);
      mma_ts(d, a_hi, b_hi, !(first && j == 0));
      mma_ts(d, a_hi, b_lo, true);
      mma_ts(d, a_lo, b_hi, true);
    }
    mma_commit(&sm.a_empty[ra.idx]);
    mma_commit(&sm.b_empty[rb.idx]);
    if (s % kCS == kCS - 1 || s == stages - 1) mma_commit(&sm.chunk_full[buf]);
  }
  // All issued MMAs must finish before TMEM is released.
  mma_commit(&sm.mma_done);
  mbar_drain(&sm.mma_done, 0);
}

// ---- B side (warps 4-7; thread = tile column n) -----------------------------
template <int KS>
__device__ void run_b_side(TcShared& sm, const unsigned char* raw, const LeafPlan& plan,
                           const Prod& P, int nraw, int slot_bytes, int stages) {
  constexpr int kQ = KS / 4, kSteps = KS / 8, kNB = kBRegion / (KS * 1024);
  constexpr int kTermBytes = KS / 16 * kBoxBytes;
  const int lane = threadIdx.x & 31;
  const int n = threadIdx.x - 128;
  float coef[kMaxOperandTerms];
#pragma unroll
  for (int t = 0; t < kMaxOperandTerms; ++t) coef[t] = t < P.nr ? plan.terms[P.r0 + t].coef : 0.f;
  // Raw B box: row n of 64 bytes, 16-byte chunk j at chunk j ^ ((n >> 1) & 3).
  int chunk_off[kQ];
#pragma unroll
  for (int q = 0; q < kQ; ++q)
    chunk_off[q] = (q / 4) * kBoxBytes + n * 64 + (((q % 4) ^ ((n >> 1) & 3)) * 16);
  const int tile_off = (n / 8) * 256 + (n % 8) * 16;   // bytes, within a 4 KB hi/lo tile
  Ring r, rb;
  for (int s = 0; s < stages; ++s, r.next(nraw), rb.next(kNB)) {
    bool w = mbar_wait(sm, &sm.raw_full[r.idx], r.phase);
    if (w && s >= kNB) w = mbar_wait(sm, &sm.b_empty[rb.idx], rb.phase ^ 1u);
    if (!__all_sync(0xffffffffu, w)) return;
    const unsigned char* src = raw + r.idx * slot_bytes + P.nl * kTermBytes;
    float4 v[kQ];
#pragma unroll
    for (int q = 0; q < kQ; ++q)
      v[q] = signed_first(*reinterpret_cast<const float4*>(src + chunk_off[q]), coef[0]);
#pragma unroll
    for (int t = 1; t < kMaxOperandTerms; ++t) {
      if (t >= P.nr) break;
#pragma unroll
      for (int q = 0; q < kQ; ++q)
        v[q] = add_signed(v[q], *reinterpret_cast<const float4*>(src + t * kTermBytes + chunk_off[q]),
                          coef[t]);
    }
    const int k0 = s * KS;
    if (k0 + KS > P.k) {   // K tail: the box reaches past the block
#pragma unroll
      for (int q = 0; q < kQ; ++q) {
        if (k0 + 4 * q + 0 >= P.k) v[q].x = 0.f;
        if (k0 + 4 * q + 1 >= P.k) v[q].y = 0.f;
        if (k0 + 4 * q + 2 >= P.k) v[q].z = 0.f;
        if (k0 + 4 * q + 3 >= P.k) v[q].w = 0.f;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.raw_empty[r.idx]);
    unsigned char* bst = sm.b_region + rb.idx * KS * 1024;
#pragma unroll
    for (int q = 0; q < kQ; ++q) {
      const float4 hi = split_hi(v[q]);
      const int off = (q / 2) * 4096 + tile_off + (q % 2) * 128;
      *reinterpret_cast<float4*>(bst + off) = hi;
      *reinterpret_cast<float4*>(bst + kSteps * 4096 + off) = split_lo(v[q], hi);
    }
    // The tensor core reads these tiles through the async proxy.
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.b_full[rb.idx]);
  }
}

// ---- fold warps (10-17): quadrant q = warp % 4, columns [col0, col0 + 64) ----
// Adds accumulation chunk c into this thread's running sums (registers).
__device__ bool fold_chunk(TcShared& sm, uint32_t tmem, uint32_t lane_base, int col0, int c,
                           float (&total)[64]) {
  const int buf = c & 1;
  const bool w = mbar_wait(sm, &sm.chunk_full[buf], (c >> 1) & 1);
  if (!__all_sync(0xffffffffu, w)) return false;   // tcgen05.ld below is warp-collective
  tc_fence_after();
  const uint32_t chunk = tmem + lane_base + uint32_t(buf * kBN + col0);
#pragma unroll
  for (int piece = 0; piece < 4; ++piece) {
    float v[16];
    tmem_ld16(chunk + 16 * piece, v);
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) total[16 * piece + i] = __fadd_rn(total[16 * piece + i], v[i]);
  }
  tc_fence_before();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&sm.chunk_empty[buf]);
  return true;
}

__device__ void store_outputs(const LeafPlan& plan, const Prod& P, int m0, int n0, long long batch,
                              int row, int col0, const float (&total)[64]) {
  const int r = m0 + row;
  if (r >= P.m) return;
  for (int o = 0; o < P.no; ++o) {
    const Term& T = plan.terms[P.o0 + o];
    float* base = const_cast<float*>(T.p) + batch * T.bstride + r;
    const float coef = T.coef;
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      const int col = n0 + col0 + i;
      if (col >= P.n) break;
      float* q = base + (long long)col * T.ld;
      if (T.mode == kOutAtomic) atomicAdd(q, coef * total[i]);
      else if (T.mode == kOutAdd) *q += coef * total[i];
      else *q = coef * total[i];
    }
  }
}

// ---- A side (warps 0-3; thread = tile row = TMEM lane) ----------------------
template <int KS>
__device__ void run_a_side(TcShared& sm, const unsigned char* raw, const LeafPlan& plan,
                           const Prod& P, uint32_t tmem, int nraw, int slot_bytes, int stages) {
  constexpr int kNA = kColsA / (2 * KS);
  constexpr int kTermFloats = KS / 16 * kBoxBytes / 4;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = threadIdx.x;
  const uint32_t lane_base = uint32_t(warp * 32) << 16;
  float coef[kMaxOperandTerms];
#pragma unroll
  for (int t = 0; t < kMaxOperandTerms; ++t) coef[t] = t < P.nl ? plan.terms[P.l0 + t].coef : 0.f;
  Ring r, ra;
  for (int s = 0; s < stages; ++s, r.next(nraw), ra.next(kNA)) {
    bool w = mbar_wait(sm, &sm.raw_full[r.idx], r.phase);
    if (w && s >= kNA) w = mbar_wait(sm, &sm.a_empty[ra.idx], ra.phase ^ 1u);
    if (!__all_sync(0xffffffffu, w)) return;   // tcgen05.st below is warp-collective
    // Raw A term: KS k-rows of 128 m (512 B each); a warp reads 128 contiguous bytes.
    const float* src = reinterpret_cast<const float*>(raw + r.idx * slot_bytes) + row;
    float v[KS];
#pragma unroll
    for (int k = 0; k < KS; ++k) {
      const float x = src[k * kBM];
      v[k] = coef[0] < 0.f ? -x : x;
    }
#pragma unroll
    for (int t = 1; t < kMaxOperandTerms; ++t) {
      if (t >= P.nl) break;
#pragma unroll
      for (int k = 0; k < KS; ++k) v[k] = fmaf(coef[t], src[t * kTermFloats + k * kBM], v[k]);
    }
    const int k0 = s * KS;
    if (k0 + KS > P.k) {   // K tail: the box reaches past the block
#pragma unroll
      for (int k = 0; k < KS; ++k)
        if (k0 + k >= P.k) v[k] = 0.f;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.raw_empty[r.idx]);
    const uint32_t a_col = tmem + lane_base + kColA + uint32_t(ra.idx * 2 * KS);
#pragma unroll
    for (int h = 0; h < KS / 16; ++h) {
      uint32_t hi[16], lo[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const float x = v[16 * h + k];
        const float hv = tf32_rn(x);
        hi[k] = __float_as_uint(hv);
        lo[k] = __float_as_uint(tf32_rn(x - hv));
      }
      tmem_st16(a_col + 16 * h, hi);
      tmem_st16(a_col + KS + 16 * h, lo);
    }
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.a_full[ra.idx]);
  }
}

__device__ void run_fold(TcShared& sm, const LeafPlan& plan, const Prod& P, int m0, int n0,
                         long long batch, uint32_t tmem) {
  const int warp = threadIdx.x >> 5;
  const int q = warp % 4, col0 = ((warp - kFoldWarp0) / 4) * 64;
  const uint32_t lane_base = uint32_t(q * 32) << 16;
  const int chunks = (P.k + kChunkK - 1) / kChunkK;
  float total[64];
#pragma unroll
  for (int i = 0; i < 64; ++i) total[i] = 0.f;
  for (int c = 0; c < chunks; ++c)
    if (!fold_chunk(sm, tmem, lane_base, col0, c, total)) return;
  if (*(volatile int*)&sm.abort) return;
  store_outputs(plan, P, m0, n0, batch, q * 32 + (threadIdx.x & 31), col0, total);
}

}  // namespace

// 18 warps put 5 on one SM sub-partition (16K registers): at most 96 per
// thread.  The fold warps hold 64 running sums each.
__global__ void __maxnreg__(96)
    leaf_tc_kernel(const __grid_constant__ LeafPlan plan, const __grid_constant__ TcMaps maps) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  TcShared& sm = *reinterpret_cast<TcShared*>(smem_raw);
  unsigned char* raw = smem_raw + kRawOffset;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const Prod& P = find_prod(plan, blockIdx.x);
  const int local = blockIdx.x - P.tile_begin;
  constexpr int GROUP_M = 8;
  const int in_group = GROUP_M * P.tiles_n;
  const int first_m = (local / in_group) * GROUP_M;
  const int gsize = min(P.tiles_m - first_m, GROUP_M);
  const int m0 = (first_m + (local % in_group) % gsize) * kBM;
  const int n0 = ((local % in_group) / gsize) * kBN;
  const int batch = blockIdx.y;
  const bool valid = P.nl >= 1 && P.nl <= kMaxOperandTerms && P.nr >= 1 && P.nr <= kMaxOperandTerms;
  const int terms = valid ? P.nl + P.nr : 1;
  const int ks = 2 * terms * 32 * kBM * 4 <= kRawBytes ? 32 : 16;   // up to five terms
  const int slot_bytes = terms * ks * kBM * 4;
  const int nraw = min(kMaxRaw, kRawBytes / slot_bytes);
  const int stages = (P.k + ks - 1) / ks;

  if (threadIdx.x == 0) {
    for (int i = 0; i < nraw; ++i) {
      mbar_init(&sm.raw_full[i], 1);
      mbar_init(&sm.raw_empty[i], 8);   // the 8 transform warps
    }
    for (int i = 0; i < 8; ++i) {
      mbar_init(&sm.a_full[i], 4);
      mbar_init(&sm.a_empty[i], 1);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&sm.b_full[i], 4);
      mbar_init(&sm.b_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.chunk_full[i], 1);
      mbar_init(&sm.chunk_empty[i], kFoldWarps);
    }
    mbar_init(&sm.mma_done, 1);
    sm.abort = 0;
    // Make the initialised barriers visible to the async proxy (TMA, tcgen05).
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kTmaWarp) {
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

  if (!valid) {
    if (threadIdx.x == 0) atomicOr(&g_tc_device_error, 2u);
  } else if (warp == kTmaWarp) {
    if (lane == 0) run_producer(sm, raw, maps, P, m0, n0, batch, nraw, slot_bytes, stages, ks);
    __syncwarp();
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      if (ks == 32) run_mma<32>(sm, tmem, stages);
      else run_mma<16>(sm, tmem, stages);
    }
    __syncwarp();
  } else if (warp >= kFoldWarp0) {
    run_fold(sm, plan, P, m0, n0, batch, tmem);
  } else if (warp >= 4) {
    if (ks == 32) run_b_side<32>(sm, raw, plan, P, nraw, slot_bytes, stages);
    else run_b_side<16>(sm, raw, plan, P, nraw, slot_bytes, stages);
  } else {
    if (ks == 32) run_a_side<32>(sm, raw, plan, P, tmem, nraw, slot_bytes, stages);
    else run_a_side<16>(sm, raw, plan, P, tmem, nraw, slot_bytes, stages);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kTmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

namespace {

using EncodeTiled = PFN_cuTensorMapEncodeTiled_v12000;

EncodeTiled encode_fn() {
  static const EncodeTiled fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return EncodeTiled(nullptr);
    return reinterpret_cast<EncodeTiled>(p);
  }();
  return fn;
}

struct MapKey {
  const float* base;
  long long ld, bstride, rows, cols, nb;
  bool left;
  bool operator==(const MapKey& o) const {
    return base == o.base && ld == o.ld && bstride == o.bstride && rows == o.rows &&
           cols == o.cols && nb == o.nb && left == o.left;
  }
};

// Tensor maps of one launch.  Left operands use box {128 m, 16 k} without
// swizzle, right operands box {16 k, 128 n} with 64-byte swizzle.
class MapTable {
 public:
  explicit MapTable(TcMaps& out) : out_(out) {}
  void reset() {
    keys_.clear();
    std::memset(&out_, 0, sizeof(out_));
  }
  // Map id for `key`, encoding a new map when needed; -1 when the table is
  // full, -2 when the driver rejects the map.
  int get(const MapKey& key) {
    for (size_t i = 0; i < keys_.size(); ++i)
      if (keys_[i] == key) return int(i);
    if (keys_.size() >= size_t(kMaxMaps)) return -1;
    const EncodeTiled enc = encode_fn();
    if (!enc) return -2;
    const cuuint64_t dims[3] = {cuuint64_t(key.rows), cuuint64_t(key.cols), cuuint64_t(key.nb)};
    const long long bs = key.bstride ? key.bstride : key.ld * key.cols;
    const cuuint64_t strides[2] = {cuuint64_t(key.ld) * 4, cuuint64_t(bs) * 4};
    const cuuint32_t box[3] = {key.left ? 128u : 16u, key.left ? 16u : 128u, 1u};
    const cuuint32_t estr[3] = {1, 1, 1};
    CUtensorMap& m = out_.map[keys_.size()];
    const CUresult r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(key.base),
                           dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           key.left ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_64B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return -2;
    keys_.push_back(key);
    return int(keys_.size()) - 1;
  }

 private:
  TcMaps& out_;
  std::vector<MapKey> keys_;
};

// Map and origin of operand term `t` (extent rows x cols): the containing
// source matrix when there is one, else a map of the block itself (whose
// zero fill then also covers the tile's overhang).
int assign_operand(MapTable& maps, TcMaps& out, int ti, const Term& t, long long rows,
                   long long cols, bool left, const TcSource* src, int nsrc, int batch) {
  const long long nb = t.bstride ? batch : 1;
  for (int i = 0; i < nsrc; ++i) {
    const TcSource& S = src[i];
    if (S.ld != t.ld || S.bstride != t.bstride || t.p < S.base) continue;
    const long long off = t.p - S.base;
    const long long x = off % S.ld, y = off / S.ld;
    if (x + rows > S.rows || y + cols > S.cols) continue;
    const int id = maps.get({S.base, S.ld, S.bstride, S.rows, S.cols, nb, left});
    if (id < 0) return id;
    out.op_map[ti] = id | (t.bstride ? 0 : 0x10000);
    out.op_x[ti] = int(x);
    out.op_y[ti] = int(y);
    return id;
  }
  const int id = maps.get({t.p, t.ld, t.bstride, rows, cols, nb, left});
  if (id < 0) return id;
  out.op_map[ti] = id | (t.bstride ? 0 : 0x10000);
  out.op_x[ti] = 0;
  out.op_y[ti] = 0;
  return id;
}

cudaError_t launch_subplan(const LeafPlan& full, int p0, int p1, const TcMaps& maps, int batch,
                           cudaStream_t stream) {
  if (p1 <= p0) return cudaSuccess;
  LeafPlan sub;
  sub.nprod = p1 - p0;
  const int base = full.prod[p0].tile_begin;
  const int end = p1 < full.nprod ? full.prod[p1].tile_begin : full.ntiles;
  sub.ntiles = end - base;
  for (int i = p0; i < p1; ++i) {
    sub.prod[i - p0] = full.prod[i];
    sub.prod[i - p0].tile_begin -= base;
  }
  std::memcpy(sub.terms, full.terms, sizeof(full.terms));
  if (sub.ntiles <= 0) return cudaSuccess;
  leaf_tc_kernel<<<dim3(sub.ntiles, batch), kThreads, kSmemBytes, stream>>>(sub, maps);
  return cudaGetLastError();
}

}  // namespace

TileShape tc_tile_shape() { return {kBM, kBN}; }

bool tc_supported(int nl, int nr) {
  return nl >= 1 && nl <= kMaxOperandTerms && nr >= 1 && nr <= kMaxOperandTerms &&
         encode_fn() != nullptr;
}

cudaError_t launch_leaf_tc(const LeafPlan& plan, const TcSource* sources, int nsources, int batch,
                           cudaStream_t stream) {
  if (plan.nprod == 0 || plan.ntiles == 0 || batch == 0) return cudaSuccess;
  // The attribute is per device: set it before every launch (cheap).
  cudaError_t e = cudaFuncSetAttribute(leaf_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kSmemBytes);
  if (e != cudaSuccess) return e;
  // Products are launched in runs whose tensor maps fit the parameter block.
  static thread_local TcMaps maps;
  MapTable table(maps);
  table.reset();
  int run_begin = 0;
  for (int p = 0; p < plan.nprod; ++p) {
    const Prod& P = plan.prod[p];
    for (int attempt = 0; attempt < 2; ++attempt) {
      bool ok = true;
      for (int t = 0; t < P.nl && ok; ++t) {
        const int id = assign_operand(table, maps, P.l0 + t, plan.terms[P.l0 + t], P.m, P.k, true,
                                      sources, nsources, batch);
        if (id == -2) return cudaErrorInvalidValue;
        ok = id >= 0;
      }
      for (int t = 0; t < P.nr && ok; ++t) {
        const int id = assign_operand(table, maps, P.r0 + t, plan.terms[P.r0 + t], P.k, P.n, false,
                                      sources, nsources, batch);
        if (id == -2) return cudaErrorInvalidValue;
        ok = id >= 0;
      }
      if (ok) break;
      if (attempt == 1 || p == run_begin) return cudaErrorInvalidValue;   // one product > kMaxMaps
      // Table full: launch the run so far and start a new one with this product.
      e = launch_subplan(plan, run_begin, p, maps, batch, stream);
      if (e != cudaSuccess) return e;
      run_begin = p;
      table.reset();
    }
  }
  return launch_subplan(plan, run_begin, plan.nprod, maps, batch, stream);
}

cudaError_t read_and_clear_tc_device_error(unsigned* value) {
  cudaError_t e = cudaMemcpyFromSymbol(value, g_tc_device_error, sizeof(unsigned));
  if (e != cudaSuccess) return e;
  const unsigned zero = 0;
  return cudaMemcpyToSymbol(g_tc_device_error, &zero, sizeof(unsigned));
}

}  // namespace bag_b200
