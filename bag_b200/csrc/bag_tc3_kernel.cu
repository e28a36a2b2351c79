// Prepared-operand 3xTF32 path of the BAG FP32 matmul (sm_100a).
//
// prep_tree_kernel: one HBM-speed pass writes every distinct leaf operand of
//   the plan -- a signed sum of mids, each mid a signed sum of source blocks,
//   both in the reference's evaluation order (x + delta*y, bag.cuh:69-73;
//   prepare_child, bag.cuh:124-135) -- as TF32 hi = rn_tf32(x) and
//   lo = rn_tf32(x - hi) rows of a workspace region, k contiguous (left
//   operands are transposed on the way through shared memory) and
//   zero-padded to the region's row length; all operands of a tree group are
//   written together, each source block read once per tile.
//
// leaf_prep_kernel<BN>: persistent (one CTA per SM); each CTA computes 128 x BN
//   output tiles of the leaf products in turn, straight from the region:
//  * warp 0, lane 0: per 32-k stage four TMA loads (A hi, A lo: 128 rows x
//    32 k; B hi, B lo: BN rows x 32 k; 128-byte swizzle, K-major) into a ring
//    of stages; warp 0 also owns TMEM.
//  * warp 1, lane 0: per stage four K-steps of three tcgen05.mma.kind::tf32
//    (A_hi*B_hi + A_hi*B_lo + A_lo*B_hi, both operands by shared-memory
//    descriptor) into one TMEM chunk accumulator -- kChunkStages stages form
//    one accumulation chunk, since the tensor core accumulates with
//    round-toward-zero (Ootomo & Yokota 2022, sec. 4) -- then commits the
//    stage free and, at a chunk's end, the chunk done.
//  * warps 2.. (fold; BN/64 per TMEM lane quadrant, 64 columns each): add each
//    finished chunk into 64 FP32 running sums in registers (round-to-nearest),
//    then add coef*sum into every target C block (red.global, coalesced along
//    the column).
// TMEM: 512 / BN chunk accumulators of BN columns.
//
// All mbarrier waits are bounded (kWaitLimitNs of wall time; then this file's
// device error word is set and the CTA's abort flag raised); every role then
// skips the rest of its work, the producer drains its copies in flight and
// the MMA thread its MMAs (bounded) before TMEM is freed.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <utility>
#include <cstdint>
#include <cstring>

#include "bag_kernels.h"

namespace bag_b200 {

// This file's device error word (read by read_and_clear_tc3_device_error).
__device__ unsigned int g_tc3_device_error = 0;

namespace {

constexpr int kStageK = 32;
// Stages accumulated in TMEM per chunk before the fold warps add the chunk
// into their FP32 running sums: 2 x 32 k = 64 k.  Longer chunks mean fewer
// TMEM reads, adds and hand-offs per product (the fold is energy the
// power-capped leaf launch pays for), but the tensor core's round-toward-zero
// accumulation runs over the whole chunk, and its bias does not cancel on
// same-signed data.  Measured on B200 (interleaved runs, one box each): cfg3
// 32 -> 64 k +3.5%, rel-F 1.76e-6 -> 1.66e-6; 64 -> 128 k another +2.6%, but
// cfg5 (U[0,1), 1024-long leaves) then reached 1.12e-6 against its bound of
// 1.25 x 6.76e-7, so 64 k it is.
constexpr int kChunkStages = 2;
constexpr unsigned kSuspendNs = 1000000;
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

template <int BN>
struct Cfg {
  static constexpr int kStages = BN == 128 ? 3 : 2;
  static constexpr int kABytes = 128 * kStageK * 4;   // one 128-row plane tile (16 KB)
  static constexpr int kBBytes = BN * kStageK * 4;
  static constexpr int kStageBytes = 2 * kABytes + 2 * kBBytes;
  static constexpr int kChunkBufs = 512 / BN;
  static constexpr int kFoldWarps = 4 * (BN / 64);
  static constexpr int kThreads = (2 + kFoldWarps) * 32;
  static constexpr int kBarOffset = kStages * kStageBytes;
  static constexpr int kSmemBytes = kBarOffset + 1024;
  // Instruction descriptor: F32 accumulate, TF32 A and B, both K-major,
  // N = BN, M = 128 (c_format[4,6)=1, a_format[7,10)=2, b_format[10,13)=2,
  // n_dim[17,23)=N/8, m_dim[24,29)=M/16).
  static constexpr uint32_t kIdesc =
      (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(BN >> 3) << 17) | (uint32_t(128 >> 4) << 24);
};

struct alignas(64) PrepMaps {
  CUtensorMap a;   // box 32 k x 128 rows
  CUtensorMap b;   // box 32 k x BN rows
};

struct Bars {
  unsigned long long full[4], empty[4];
  unsigned long long chunk_full[4], chunk_empty[4];
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
__device__ __forceinline__ bool mbar_wait(int& abort, unsigned long long* bar, unsigned parity,
                                          unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long start = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_ns() - start > limit_ns || *(volatile int*)&abort) {
      atomicOr(&g_tc3_device_error, 1u);
      *(volatile int*)&abort = 1;
      return false;
    }
  }
  return true;
}

// Bounded wait that ignores the abort flag (copies and MMAs already in flight).
__device__ __forceinline__ void mbar_drain(unsigned long long* bar, unsigned parity) {
  if (mbar_try_wait(bar, parity)) return;
  const unsigned long long start = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_ns() - start > kWaitLimitNs) {
      atomicOr(&g_tc3_device_error, 1u);
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

// Tile load for a CTA pair: the copy lands in this CTA's shared memory and
// completes on the mbarrier at `bar`, a shared::cluster address in either CTA
// of the pair (.cta_group::2): a plain load into this CTA's own tile.  The
// prepared operands are re-read by every tile that shares their block, so the
// load asks L2 to keep them (evict_last); the product buffers the epilogue
// writes are streamed (st.global.cs).  Measured on the cfg3 leaf launch: DRAM
// reads 71.1 -> 68.5 GB.
__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* map, int x, int y,
                                                 int z, uint32_t bar) {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(policy));
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar), "l"(policy)
      : "memory");
}

// K-major, 128-byte-swizzled operand tile (rows of 32 k = 128 B, 8-row atoms of
// 1024 B): start address in 16-byte units, LBO 16 B (unused for this layout),
// SBO 1024 B, version 1 (bit 46), layout SWIZZLE_128B (2 at bits 61-63).  A
// K-step of 8 TF32 advances the start address by 32 B inside the swizzle row.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
  return uint64_t((addr >> 4) & 0x3FFF) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
         (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

template <int BN>
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       bool accumulate) {
  const uint32_t acc = accumulate ? 1u : 0u;
  const uint32_t zero = 0u;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}"
      :
      : "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(Cfg<BN>::kIdesc), "r"(acc), "r"(zero)
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

__device__ __forceinline__ float tf32_rn(float x) {
  uint32_t u;
  asm("cvt.rn.tf32.f32 %0, %1;" : "=r"(u) : "f"(x));
  return __uint_as_float(u);
}

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

}  // namespace

// ---- prepare pass (tree groups) ---------------------------------------------
__device__ __forceinline__ float4 load4(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}

__device__ __forceinline__ float4 hi4(float4 v) {
  return make_float4(tf32_rn(v.x), tf32_rn(v.y), tf32_rn(v.z), tf32_rn(v.w));
}
__device__ __forceinline__ float4 lo4(float4 v, float4 h) {
  return make_float4(tf32_rn(v.x - h.x), tf32_rn(v.y - h.y), tf32_rn(v.z - h.z),
                     tf32_rn(v.w - h.w));
}

// Signed sum in FP32: the first term with its sign (exact), then fmaf with
// +-1 per further term -- the rounding of the materialisation pass and of the
// fused prologue.
__device__ __forceinline__ float4 signed_add(float4 acc, float4 v, int code, bool first) {
  const float c = code > 0 ? 1.f : -1.f;
  if (first) return make_float4(c * v.x, c * v.y, c * v.z, c * v.w);
  return make_float4(fmaf(c, v.x, acc.x), fmaf(c, v.y, acc.y), fmaf(c, v.z, acc.z),
                     fmaf(c, v.w, acc.w));
}

// One CTA (256 threads) writes a 16-row x 64-k tile of every operand of a
// tree group.  Thread t owns row t / 16 of the tile and its k values
// 4 (t % 16) .. +3, so a warp's store covers 2 rows x 256 contiguous bytes of
// a plane.  Every input's tile is staged in shared memory in that same
// [row][k] layout (pitch 68 floats: 16-byte aligned rows, and a warp's
// 16-byte reads of 2 rows x 256 bytes take the minimum four wavefronts), so
// the thread reads each input as one float4.  A right operand (k contiguous
// in its source) is loaded in that layout; a left operand (rows contiguous)
// is loaded as 4 rows x 1 k per thread (a warp reads 8 columns x 64 bytes)
// and transposed on its way into shared memory.  Then, segment by segment,
// the thread evaluates the segment's mids from the inputs (the mids stay in
// the thread's registers, picked by the plan's codes with selects), each
// output from the mids, splits it into TF32 hi/lo and stores both.  Inputs
// past the block (rows or k) read as zero, so the region's padding past an
// operand's k extent is written as zero.
//
// The tile shape is the measured one: on B200, stores of 98 planes in this
// pattern ran at 6.89 TB/s against 5.47 for 32 x 32 tiles (a warp writing
// 4 rows x 128 bytes), and 16-row column segments of a column-major source
// read at 6.09 TB/s against 5.12 for 32-row ones.
//
// kIn bounds the inputs of every group of the launch: 16 at depth 2, 4 at
// depth 1.  Inputs are loaded eight at a time (eight 16-byte loads in flight
// per thread), three CTAs per SM at depth 2 (70 KB of staging each) and five
// at depth 1.
constexpr int kTreeRows = kPrepTreeRows;   // 16
constexpr int kTreeK = kPrepTreeK;         // 64
constexpr int kTreePitch = kTreeK + 4;
constexpr int kTreeThreads = 256;
constexpr int kTreeSmallIn = 4;
constexpr int kTreeLoadBatch = 8;
thread_local int g_last_tree_table = -1;   // host side: the last launch's basis pair (0 = none)
static_assert(kTreeRows * kTreeK == 4 * kTreeThreads, "one float4 per thread per input");

template <int kIn>
constexpr int tree_smem_bytes() { return kIn * kTreeRows * kTreePitch * 4; }

__device__ __forceinline__ float4 pick_mid(const float4 (&md)[kTreeMid], int i) {
  float4 r = md[0];
#pragma unroll
  for (int j = 1; j < kTreeMid; ++j)
    if (i == j) r = md[j];
  return r;
}

// The operand expressions of a tree group are one basis's inner transform,
// the same in every segment: 7 operands, each a signed sum of up to 4 of the
// segment's 4 mids (1-based, sign = subtract, 0 = end), in evaluation order;
// left operands (transposed groups) and right ones have their own table.  A
// launch with groups that hold one basis's pair of tables runs a kernel with
// the pair compiled in (kP = 1 Minimal, 2 Full, 3 Classic, 4 Winograd): in
// those groups (TreeGroup::table, set by the host after comparing every
// segment with its side's table) the mids stay in registers with fixed
// indices and an operand costs its arithmetic alone; other groups of the
// launch (peeled strips of ragged shapes) read their terms from the plan.
struct TreeExprTable {
  signed char e[7][4];
};
constexpr TreeExprTable kTreeExprTables[kTreeExprCount] = {
    {{{1, 2, 0, 0}, {2, -3, 0, 0}, {1, -3, 2, 0}, {4, 0, 0, 0}, {1, 0, 0, 0}, {1, -3, 2, -4},
      {3, 0, 0, 0}}},                                                    // Minimal, left
    {{{1, 2, 0, 0}, {2, -3, 0, 0}, {1, -3, 2, 0}, {4, 0, 0, 0}, {3, 0, 0, 0}, {1, 0, 0, 0},
      {1, -3, 2, -4}}},                                                  // Minimal, right
    {{{1, 0, 0, 0}, {2, 0, 0, 0}, {3, 0, 0, 0}, {4, 0, 0, 0}, {3, -2, 0, 0}, {3, -4, 0, 0},
      {1, -3, 0, 0}}},                                                   // Full, left
    {{{1, 0, 0, 0}, {2, 0, 0, 0}, {3, 0, 0, 0}, {4, 0, 0, 0}, {1, -3, 0, 0}, {3, -2, 0, 0},
      {3, -4, 0, 0}}},                                                   // Full, right
    {{{1, 2, 0, 0}, {3, 4, 0, 0}, {1, -3, 0, 0}, {4, -2, 0, 0}, {3, 0, 0, 0}, {2, 0, 0, 0},
      {3, 2, 0, 0}}},                                                    // Classic, left
    {{{1, 0, 0, 0}, {2, 0, 0, 0}, {1, 3, 0, 0}, {4, 2, 0, 0}, {3, -2, 0, 0}, {4, -1, 0, 0},
      {1, 2, 0, 0}}},                                                    // Classic, right
    {{{1, 0, 0, 0}, {2, 0, 0, 0}, {2, -3, -4, 1}, {4, 0, 0, 0}, {3, 4, 0, 0}, {3, 4, -1, 0},
      {1, -3, 0, 0}}},                                                   // Winograd, left
    {{{1, 0, 0, 0}, {2, 0, 0, 0}, {3, 0, 0, 0}, {3, -4, 1, -2}, {4, -1, 0, 0}, {3, -4, 1, 0},
      {3, -4, 0, 0}}},                                                   // Winograd, right
};

template <int kX, int O, int Q>
__device__ __forceinline__ float4 table_term(const float4 (&md)[kTreeMid], float4 x) {
  constexpr int code = kTreeExprTables[kX - 1].e[O][Q];
  if constexpr (code == 0) {
    return x;
  } else {
    constexpr int idx = (code > 0 ? code : -code) - 1;
    static_assert(idx < kTreeMid, "table names a mid past the segment's four");
    return signed_add(x, md[idx], code, Q == 0);
  }
}

// Operand O of the table: its terms in order (the rounding of signed_add).
template <int kX, int O>
__device__ __forceinline__ float4 table_operand(const float4 (&md)[kTreeMid]) {
  float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
  x = table_term<kX, O, 0>(md, x);
  x = table_term<kX, O, 1>(md, x);
  x = table_term<kX, O, 2>(md, x);
  return table_term<kX, O, 3>(md, x);
}

__device__ __forceinline__ void store_hi_lo(float* dst, long long plane, float4 x) {
  const float4 h = hi4(x);
  *reinterpret_cast<float4*>(dst) = h;
  *reinterpret_cast<float4*>(dst + plane) = lo4(x, h);
}

template <int kX, int... O>
__device__ __forceinline__ void table_operands(const float4 (&md)[kTreeMid], const TreeSeg& S,
                                               float* base, long long ld, long long plane,
                                               std::integer_sequence<int, O...>) {
  (store_hi_lo(base + (long long)S.out_hi[O] * ld, plane, table_operand<kX, O>(md)), ...);
}

// The operands of one tile from its staged inputs ([input][row][k], pitch
// kTreePitch): per segment, the mids in registers, then each operand split
// into TF32 hi/lo and stored (rows past the group's are skipped).
template <int kP>
__device__ __forceinline__ void tree_operands(const PrepTreePlan& plan, const TreeGroup& G,
                                              const float* staged, int r0, int k0,
                                              long long batch, int t) {
  const int row = t / (kTreeK / 4), kc = 4 * (t % (kTreeK / 4));
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  const int r = r0 + row;
  if (r >= G.rows) return;
  auto input = [&](int u) {
    return *reinterpret_cast<const float4*>(staged + (u * kTreeRows + row) * kTreePitch + kc);
  };
  float* region = plan.region + batch * plan.region_bstride;
  const long long ld = plan.row_len;
  for (int sg = 0; sg < G.nseg; ++sg) {
    const TreeSeg& S = G.seg[sg];
    float4 md[kTreeMid];
#pragma unroll
    for (int i = 0; i < kTreeMid; ++i) {
      md[i] = zero;
      if (i < S.nmid) {
#pragma unroll
        for (int q = 0; q < kMaxOperandTerms; ++q) {
          const int code = S.mid[i][q];
          if (code == 0) break;
          md[i] = signed_add(md[i], input((code > 0 ? code : -code) - 1), code, q == 0);
        }
      }
    }
    bool tabled = false;
    if constexpr (kP > 0) {
      if (G.table) {
        float* base = region + (long long)r * ld + k0 + kc;
        const long long plane = (long long)G.rows * ld;
        if (G.transpose)
          table_operands<2 * kP - 1>(md, S, base, ld, plane, std::make_integer_sequence<int, 7>{});
        else
          table_operands<2 * kP>(md, S, base, ld, plane, std::make_integer_sequence<int, 7>{});
        tabled = true;
      }
    }
    if (!tabled) {
      for (int o = 0; o < S.nout; ++o) {
        float4 x = zero;
#pragma unroll
        for (int q = 0; q < kMaxOperandTerms; ++q) {
          const int code = S.expr[o][q];
          if (code == 0) break;
          x = signed_add(x, pick_mid(md, (code > 0 ? code : -code) - 1), code, q == 0);
        }
        store_hi_lo(region + (long long)(S.out_hi[o] + r) * ld + k0 + kc, (long long)G.rows * ld,
                    x);
      }
    }
  }
}

template <int kIn, int kP>
__global__ void __launch_bounds__(kTreeThreads, kIn <= kTreeSmallIn ? 5 : 3)
    prep_tree_kernel(const __grid_constant__ PrepTreePlan plan) {
  extern __shared__ __align__(16) float staged[];     // [input][row][k], pitch kTreePitch
  const long long item = blockIdx.x;
  int gi = 0;
  while (gi + 1 < plan.ngroups && plan.group[gi + 1].tile_begin <= item) ++gi;
  const TreeGroup& G = plan.group[gi];
  const long long local = item - G.tile_begin;
  const int ktiles = plan.row_len / kTreeK;
  const int r0 = int(local / ktiles) * kTreeRows, k0 = int(local % ktiles) * kTreeK;
  const long long batch = blockIdx.y;
  const int t = threadIdx.x;
  const int row = t / (kTreeK / 4), kc = 4 * (t % (kTreeK / 4));
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  constexpr int kBatch = kIn < kTreeLoadBatch ? kIn : kTreeLoadBatch;

#pragma unroll
  for (int u0 = 0; u0 < kIn; u0 += kBatch) {
    if (u0 >= G.nin) break;
    float4 v[kBatch];
    if (G.transpose) {
      // Left operand: element (r, k) at p + r + k * ld; rows 4 (t % 4) .. +3
      // of k column t / 4 of the tile.
      const int rr = 4 * (t % (kTreeRows / 4)), kk = t / (kTreeRows / 4);
      const int r = r0 + rr, k = k0 + kk;
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        const int u = u0 + j;
        v[j] = zero;
        if (u < G.nin && k < G.cols) {
          const Term& T = G.in[u];
          const float* p = T.p + batch * T.bstride + r + (long long)k * T.ld;
          if (r + 3 < G.rows) {
            v[j] = load4(p);
          } else {
            if (r + 0 < G.rows) v[j].x = p[0];
            if (r + 1 < G.rows) v[j].y = p[1];
            if (r + 2 < G.rows) v[j].z = p[2];
          }
        }
      }
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        if (u0 + j < G.nin) {
          float* s = staged + ((u0 + j) * kTreeRows + rr) * kTreePitch + kk;
          s[0] = v[j].x;
          s[kTreePitch] = v[j].y;
          s[2 * kTreePitch] = v[j].z;
          s[3 * kTreePitch] = v[j].w;
        }
      }
    } else {
      // Right operand: element (k, r) at p + k + r * ld; k values kc .. +3 of
      // row `row` of the tile, the layout the thread computes in.
      const int r = r0 + row, k = k0 + kc;
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        const int u = u0 + j;
        v[j] = zero;
        if (u < G.nin && r < G.rows) {
          const Term& T = G.in[u];
          const float* p = T.p + batch * T.bstride + k + (long long)r * T.ld;
          if (k + 3 < G.cols) {
            v[j] = load4(p);
          } else {
            if (k + 0 < G.cols) v[j].x = p[0];
            if (k + 1 < G.cols) v[j].y = p[1];
            if (k + 2 < G.cols) v[j].z = p[2];
          }
        }
      }
#pragma unroll
      for (int j = 0; j < kBatch; ++j)
        if (u0 + j < G.nin)
          *reinterpret_cast<float4*>(staged + ((u0 + j) * kTreeRows + row) * kTreePitch + kc) =
              v[j];
    }
  }
  __syncthreads();
  tree_operands<kP>(plan, G, staged, r0, k0, batch, t);
}

// ---- leaf products on prepared operands -------------------------------------
// Persistent: CTA b processes work items b, b + gridDim.x, ... (item = batch *
// ntiles + tile); the stage and chunk rings run on across items, so the fold
// warps' epilogue of one tile overlaps the next tile's loads and MMAs.
struct TileCoord {
  const PrepProd* P;
  int m0, n0, batch, stages;
};

template <int BN>
__device__ __forceinline__ TileCoord tile_of(const PrepLeafPlan& plan, int item) {
  const int batch = item / plan.ntiles, t = item - batch * plan.ntiles;
  int pid = 0;
  while (pid + 1 < plan.nprod && plan.prod[pid + 1].tile_begin <= t) ++pid;
  const PrepProd& P = plan.prod[pid];
  const int local = t - P.tile_begin;
  constexpr int GROUP_M = 8;
  const int in_group = GROUP_M * P.tiles_n;
  const int first_m = (local / in_group) * GROUP_M;
  const int gsize = min(P.tiles_m - first_m, GROUP_M);
  TileCoord c;
  c.P = &P;
  c.m0 = (first_m + (local % in_group) % gsize) * 128;
  c.n0 = ((local % in_group) / gsize) * BN;
  c.batch = batch;
  c.stages = (P.k + kStageK - 1) / kStageK;
  return c;
}

template <int BN>
__global__ void __launch_bounds__(Cfg<BN>::kThreads, 1)
    leaf_prep_kernel(const __grid_constant__ PrepLeafPlan plan, const __grid_constant__ PrepMaps maps,
                     int items) {
  using C = Cfg<BN>;
  extern __shared__ __align__(1024) unsigned char smem[];
  Bars& sb = *reinterpret_cast<Bars*>(smem + C::kBarOffset);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::kStages; ++i) {
      mbar_init(&sb.full[i], 1);
      mbar_init(&sb.empty[i], 1);
    }
    for (int i = 0; i < C::kChunkBufs; ++i) {
      mbar_init(&sb.chunk_full[i], 1);
      mbar_init(&sb.chunk_empty[i], C::kFoldWarps);
    }
    mbar_init(&sb.mma_done, 1);
    sb.abort = 0;
    // Make the initialised barriers visible to the async proxy (TMA, tcgen05).
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(
                     smem_u32(&sb.tmem_base))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sb.tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      long long issued = 0;
      Ring r;
      bool ok = true;
      for (int item = blockIdx.x; item < items && ok; item += gridDim.x) {
        const TileCoord tc = tile_of<BN>(plan, item);
        for (int s = 0; s < tc.stages; ++s, r.next(C::kStages)) {
          if (issued >= C::kStages && !mbar_wait(sb.abort, &sb.empty[r.idx], r.phase ^ 1u)) {
            ok = false;
            break;
          }
          unsigned char* st = smem + r.idx * C::kStageBytes;
          mbar_expect_tx(&sb.full[r.idx], C::kStageBytes);
          const int k0 = s * kStageK;
          const PrepProd& P = *tc.P;
          tma_load_3d(st, &maps.a, k0, P.a_hi + tc.m0, tc.batch, &sb.full[r.idx]);
          tma_load_3d(st + C::kABytes, &maps.a, k0, P.a_lo + tc.m0, tc.batch, &sb.full[r.idx]);
          tma_load_3d(st + 2 * C::kABytes, &maps.b, k0, P.b_hi + tc.n0, tc.batch, &sb.full[r.idx]);
          tma_load_3d(st + 2 * C::kABytes + C::kBBytes, &maps.b, k0, P.b_lo + tc.n0, tc.batch,
                      &sb.full[r.idx]);
          ++issued;
        }
      }
      // No copy may outlive the CTA: wait for the latest phase of every stage
      // slot that may still be loading.
      for (long long s = issued > C::kStages ? issued - C::kStages : 0; s < issued; ++s)
        mbar_drain(&sb.full[s % C::kStages], unsigned((s / C::kStages) & 1));
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      Ring r, rc;
      long long chunks = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < items && ok; item += gridDim.x) {
        const TileCoord tc = tile_of<BN>(plan, item);
        for (int s = 0; s < tc.stages; ++s, r.next(C::kStages)) {
          const bool first = s % kChunkStages == 0;
          const bool last = s % kChunkStages == kChunkStages - 1 || s == tc.stages - 1;
          if (first && chunks >= C::kChunkBufs &&
              !mbar_wait(sb.abort, &sb.chunk_empty[rc.idx], rc.phase ^ 1u)) {
            ok = false;
            break;
          }
          if (!mbar_wait(sb.abort, &sb.full[r.idx], r.phase)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = smem_u32(smem + r.idx * C::kStageBytes);
          const uint32_t d = tmem + uint32_t(rc.idx * BN);
#pragma unroll
          for (int j = 0; j < kStageK / 8; ++j) {
            const uint64_t a_hi = sw128_desc(st + 32 * j);
            const uint64_t a_lo = sw128_desc(st + C::kABytes + 32 * j);
            const uint64_t b_hi = sw128_desc(st + 2 * C::kABytes + 32 * j);
            const uint64_t b_lo = sw128_desc(st + 2 * C::kABytes + C::kBBytes + 32 * j);
            mma_ss<BN>(d, a_hi, b_hi, j > 0 || !first);
            mma_ss<BN>(d, a_hi, b_lo, true);
            mma_ss<BN>(d, a_lo, b_hi, true);
          }
          mma_commit(&sb.empty[r.idx]);
          if (last) {
            mma_commit(&sb.chunk_full[rc.idx]);
            ++chunks;
            rc.next(C::kChunkBufs);
          }
        }
      }
      // All issued MMAs must finish before TMEM is released.
      mma_commit(&sb.mma_done);
      mbar_drain(&sb.mma_done, 0);
    }
    __syncwarp();
  } else {
    // Fold warp: TMEM lane quadrant q = warp % 4, columns [col0, col0 + 64).
    const int q = warp % 4, col0 = ((warp - 2) / 4) * 64;
    const uint32_t lane_base = uint32_t(q * 32) << 16;
    Ring rc;
    bool ok = true;
    for (int item = blockIdx.x; item < items && ok; item += gridDim.x) {
      const TileCoord tc = tile_of<BN>(plan, item);
      float total[64];
#pragma unroll
      for (int i = 0; i < 64; ++i) total[i] = 0.f;
      const int nchunks = (tc.stages + kChunkStages - 1) / kChunkStages;
      for (int c = 0; c < nchunks; ++c, rc.next(C::kChunkBufs)) {
        const bool w = mbar_wait(sb.abort, &sb.chunk_full[rc.idx], rc.phase);
        if (!__all_sync(0xffffffffu, w)) {   // tcgen05.ld below is warp-collective
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t chunk = tmem + lane_base + uint32_t(rc.idx * BN + col0);
#pragma unroll
        for (int piece = 0; piece < 4; ++piece) {
          float v[16];
          tmem_ld16(chunk + 16 * piece, v);
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
          for (int i = 0; i < 16; ++i)
            total[16 * piece + i] = __fadd_rn(total[16 * piece + i], v[i]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sb.chunk_empty[rc.idx]);
      }
      if (!ok || *(volatile int*)&sb.abort) break;
      const PrepProd& P = *tc.P;
      const int r = tc.m0 + q * 32 + lane;
      if (r < P.m) {
        for (int o = 0; o < P.no; ++o) {
          const Term& T = plan.outs[P.o0 + o];
          float* base = const_cast<float*>(T.p) + (long long)tc.batch * T.bstride + r;
          const float coef = T.coef;
#pragma unroll
          for (int i = 0; i < 64; ++i) {
            const int col = tc.n0 + col0 + i;
            if (col >= P.n) break;
            float* dst = base + (long long)col * T.ld;
            if (T.mode == kOutAtomic) atomicAdd(dst, coef * total[i]);
            else if (T.mode == kOutAdd) *dst += coef * total[i];
            else __stcs(dst, coef * total[i]);   // streamed: keep L2 for the operands
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
  }
}

// ---- leaf products on prepared operands, CTA pairs ---------------------------
// A cluster of two CTAs (one per SM) computes 256 x 256 output tiles with
// tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 8, issued by the even CTA):
// CTA r of the pair stages rows [128r, 128r + 128) of both the A and the B
// tile, and its TMEM receives output rows [128r, 128r + 128) x 256 columns.
// Per SM that is the single-CTA kernel's 128 x 256 tile at two thirds of its
// operand bytes (each CTA loads half of B) and the same MMA instruction size.
//  * warp 0, lane 0 (each CTA): per stage TMA loads (.cta_group::2) of its A
//    hi/lo and B hi/lo rows into its own stage ring; both CTAs' copies
//    complete on the even CTA's full barrier, whose expected byte count the
//    even CTA sets for both.  Warp 0 also allocates the pair's TMEM.
//  * warp 1, lane 0 of the even CTA: the MMA thread: it waits for the full
//    barrier, issues the stage's twelve MMAs into one of two 256-column TMEM
//    chunk accumulators (kChunkStages 32-k stages form one accumulation chunk),
//    then commits to the stage's empty barrier, and at a chunk's end to the
//    chunk's full barrier, in both CTAs.
//  * warps 2-17 (fold): TMEM lane quadrant warp % 4, 64 columns each; add
//    each finished chunk into 64 FP32 running sums (round-to-nearest),
//    release it to the even CTA's chunk_empty barrier, and per tile add
//    coef * sum into every target C block (red.global, coalesced along the
//    column).
namespace pairk {
constexpr int kStages = 3;
constexpr int kABytes = 128 * kStageK * 4;                 // 16 KB: 128 rows x 32 k
constexpr int kBBytes = 128 * kStageK * 4;                 // 16 KB: 128 rows x 32 k
constexpr int kStageBytes = 2 * kABytes + 2 * kBBytes;     // 64 KB
constexpr int kChunks = 2;
constexpr int kChunkCols = 256;
constexpr int kFoldWarps = 16;
constexpr int kThreads = (2 + kFoldWarps) * 32;            // 576
constexpr int kBarOffset = kStages * kStageBytes;
constexpr int kSmemBytes = kBarOffset + 1024;
constexpr int kTileM = 256, kTileN = 256;
// F32 accumulate, TF32 A and B, both K-major, N = 256, M = 256.
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(kTileN >> 3) << 17) |
                            (uint32_t(kTileM >> 4) << 24);
}  // namespace pairk

struct PairBars {
  // full: the even CTA's counts both CTAs' copies of the stage.
  unsigned long long full[pairk::kStages], empty[pairk::kStages];
  unsigned long long chunk_full[pairk::kChunks], chunk_empty[pairk::kChunks];
  unsigned long long mma_done;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_count_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// Shared::cluster address of the same shared-memory object in CTA `rank`.
__device__ __forceinline__ uint32_t peer_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
// Arrive on an mbarrier of either CTA of the cluster (default semantics:
// release at CTA scope; a cluster-scope release costs ~0.5 us per arrive).
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Completion of this thread's earlier cta_group::2 MMAs, signalled on the
// mbarrier at a shared::cluster address (either CTA of the pair).
__device__ __forceinline__ void mma_commit_pair(uint32_t cluster_addr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   cluster_addr)
               : "memory");
}
__device__ __forceinline__ void mma_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         bool accumulate) {
  const uint32_t acc = accumulate ? 1u : 0u;
  const uint32_t zero = 0u;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;"
      "\n\t}"
      :
      : "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(pairk::kIdesc), "r"(acc), "r"(zero)
      : "memory");
}

// Work item (pair tile) -> product and coordinates; same grouped order as the
// single-CTA kernel, over 256 x 256 tiles.
__device__ __forceinline__ TileCoord pair_tile_of(const PrepLeafPlan& plan, int item) {
  const int batch = item / plan.ntiles, t = item - batch * plan.ntiles;
  int pid = 0;
  while (pid + 1 < plan.nprod && plan.prod[pid + 1].tile_begin <= t) ++pid;
  const PrepProd& P = plan.prod[pid];
  const int local = t - P.tile_begin;
  constexpr int GROUP_M = 8;
  const int in_group = GROUP_M * P.tiles_n;
  const int first_m = (local / in_group) * GROUP_M;
  const int gsize = min(P.tiles_m - first_m, GROUP_M);
  TileCoord c;
  c.P = &P;
  c.m0 = (first_m + (local % in_group) % gsize) * pairk::kTileM;
  c.n0 = ((local % in_group) / gsize) * pairk::kTileN;
  c.batch = batch;
  c.stages = (P.k + kStageK - 1) / kStageK;
  return c;
}

__global__ void __launch_bounds__(pairk::kThreads, 1)
    leaf_pair_kernel(const __grid_constant__ PrepLeafPlan plan,
                     const __grid_constant__ PrepMaps maps, int items) {
  using namespace pairk;
  extern __shared__ __align__(1024) unsigned char smem[];
  PairBars& sb = *reinterpret_cast<PairBars*>(smem + kBarOffset);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cid = int(cluster_id_x()), ncl = int(cluster_count_x());
  const int nparts = cid < items ? (items - 1 - cid) / ncl + 1 : 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&sb.full[i], 1);
      mbar_init(&sb.empty[i], 1);
    }
    for (int i = 0; i < kChunks; ++i) {
      mbar_init(&sb.chunk_full[i], 1);
      mbar_init(&sb.chunk_empty[i], 2 * kFoldWarps);   // fold warps of both CTAs
    }
    mbar_init(&sb.mma_done, 1);
    sb.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(
                     smem_u32(&sb.tmem_base))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();   // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem = sb.tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      long long issued = 0;
      Ring r;
      bool ok = true;
      for (int p = 0; p < nparts && ok; ++p) {
        const TileCoord tc = pair_tile_of(plan, cid + p * ncl);
        const PrepProd& P = *tc.P;
        const int arow = tc.m0 + 128 * int(rank), brow = tc.n0 + 128 * int(rank);
        for (int s = 0; s < tc.stages; ++s, r.next(kStages)) {
          if (issued >= kStages && !mbar_wait(sb.abort, &sb.empty[r.idx], r.phase ^ 1u)) {
            ok = false;
            break;
          }
          unsigned char* st = smem + r.idx * kStageBytes;
          if (leader) mbar_expect_tx(&sb.full[r.idx], 2 * kStageBytes);
          const uint32_t bar = peer_addr(&sb.full[r.idx], 0);
          const int k0 = s * kStageK;
          tma_load_3d_pair(st, &maps.a, k0, P.a_hi + arow, tc.batch, bar);
          tma_load_3d_pair(st + kABytes, &maps.a, k0, P.a_lo + arow, tc.batch, bar);
          tma_load_3d_pair(st + 2 * kABytes, &maps.b, k0, P.b_hi + brow, tc.batch, bar);
          tma_load_3d_pair(st + 2 * kABytes + kBBytes, &maps.b, k0, P.b_lo + brow, tc.batch, bar);
          ++issued;
        }
      }
      // No copy may outlive the CTA.  The even CTA waits for the latest phase
      // of every full barrier that may still be loading (they count both
      // CTAs' copies); the odd CTA, whose copies complete on the even CTA's
      // barriers, for the empty phase that follows each of its last stages
      // (the MMA consumed it, so its copies had landed) -- bounded, and on
      // the abort path long after any copy could still be in flight.
      for (long long s = issued > kStages ? issued - kStages : 0; s < issued; ++s) {
        const unsigned ph = unsigned((s / kStages) & 1);
        mbar_drain(leader ? &sb.full[s % kStages] : &sb.empty[s % kStages], ph);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      Ring r, rc;
      long long chunks = 0;
      bool ok = true;
      for (int p = 0; p < nparts && ok; ++p) {
        const TileCoord tc = pair_tile_of(plan, cid + p * ncl);
        for (int s = 0; s < tc.stages; ++s, r.next(kStages)) {
          const bool first = s % kChunkStages == 0;
          const bool last = s % kChunkStages == kChunkStages - 1 || s == tc.stages - 1;
          if (first && chunks >= kChunks &&
              !mbar_wait(sb.abort, &sb.chunk_empty[rc.idx], rc.phase ^ 1u)) {
            ok = false;
            break;
          }
          if (!mbar_wait(sb.abort, &sb.full[r.idx], r.phase)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = smem_u32(smem + r.idx * kStageBytes);
          const uint32_t d = tmem + uint32_t(rc.idx * kChunkCols);
#pragma unroll
          for (int j = 0; j < kStageK / 8; ++j) {
            const uint64_t a_hi = sw128_desc(st + 32 * j);
            const uint64_t a_lo = sw128_desc(st + kABytes + 32 * j);
            const uint64_t b_hi = sw128_desc(st + 2 * kABytes + 32 * j);
            const uint64_t b_lo = sw128_desc(st + 2 * kABytes + kBBytes + 32 * j);
            mma_pair(d, a_hi, b_hi, j > 0 || !first);
            mma_pair(d, a_hi, b_lo, true);
            mma_pair(d, a_lo, b_hi, true);
          }
          mma_commit_pair(peer_addr(&sb.empty[r.idx], 0));
          mma_commit_pair(peer_addr(&sb.empty[r.idx], 1));
          if (last) {
            mma_commit_pair(peer_addr(&sb.chunk_full[rc.idx], 0));
            mma_commit_pair(peer_addr(&sb.chunk_full[rc.idx], 1));
            ++chunks;
            rc.next(kChunks);
          }
        }
      }
      // All issued MMAs (which write both CTAs' TMEM and read both CTAs'
      // shared memory) must finish before either CTA frees TMEM or exits.
      mma_commit_pair(peer_addr(&sb.mma_done, 0));
      mma_commit_pair(peer_addr(&sb.mma_done, 1));
    }
    __syncwarp();
  } else {
    // Fold warp: TMEM lane quadrant q = warp % 4, columns [col0, col0 + 64).
    const int q = warp % 4, col0 = ((warp - 2) / 4) * 64;
    const uint32_t lane_base = uint32_t(q * 32) << 16;
    const uint32_t empty0 = peer_addr(&sb.chunk_empty[0], 0);
    const uint32_t stride = uint32_t(sizeof(unsigned long long));
    Ring rc;
    bool ok = true;
    for (int p = 0; p < nparts && ok; ++p) {
      const TileCoord tc = pair_tile_of(plan, cid + p * ncl);
      float total[64];
#pragma unroll
      for (int i = 0; i < 64; ++i) total[i] = 0.f;
      const int nchunks = (tc.stages + kChunkStages - 1) / kChunkStages;
      for (int c = 0; c < nchunks; ++c, rc.next(kChunks)) {
        const bool w = mbar_wait(sb.abort, &sb.chunk_full[rc.idx], rc.phase);
        if (!__all_sync(0xffffffffu, w)) {   // tcgen05.ld below is warp-collective
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t chunk = tmem + lane_base + uint32_t(rc.idx * kChunkCols + col0);
#pragma unroll
        for (int piece = 0; piece < 4; ++piece) {
          float v[16];
          tmem_ld16(chunk + 16 * piece, v);
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
          for (int i = 0; i < 16; ++i)
            total[16 * piece + i] = __fadd_rn(total[16 * piece + i], v[i]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(empty0 + uint32_t(rc.idx) * stride);
      }
      if (!ok || *(volatile int*)&sb.abort) break;
      const PrepProd& P = *tc.P;
      const int r = tc.m0 + 128 * int(rank) + q * 32 + lane;
      if (r < P.m) {
        for (int o = 0; o < P.no; ++o) {
          const Term& T = plan.outs[P.o0 + o];
          float* base = const_cast<float*>(T.p) + (long long)tc.batch * T.bstride + r;
          const float coef = T.coef;
#pragma unroll
          for (int i = 0; i < 64; ++i) {
            const int col = tc.n0 + col0 + i;
            if (col >= P.n) break;
            float* dst = base + (long long)col * T.ld;
            if (T.mode == kOutAtomic) atomicAdd(dst, coef * total[i]);
            else if (T.mode == kOutAdd) *dst += coef * total[i];
            else __stcs(dst, coef * total[i]);   // streamed: keep L2 for the operands
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    // The even CTA's MMAs write this CTA's TMEM and read its shared memory.
    if (lane == 0) mbar_drain(&sb.mma_done, 0);
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
  }
  // Neither CTA leaves while the other may still arrive on its barriers.
  cluster_sync_all();
}

// ---- deferred inverse transform ---------------------------------------------
// A CTA (16 warps) takes a slice of kPer x 256 rows of one column of the
// common m x n extent: 256 rows per warp of each target, so with few targets
// (4 at depth 1) the slice grows to 1024 rows and every warp still works.
// Threads 0 .. nin-1 each bring that slice of one product buffer (and, when
// accumulating, of one target) into shared memory with one bulk copy
// (cp.async.bulk, completing on the CTA's mbarrier; a slice is contiguous in
// the column-major blocks and a multiple of 16 bytes), so staging costs a
// handful of instructions per CTA.  Then warp w adds target w / W's products
// in plan order over its 256 rows (lane l: rows 4l .. 4l+3 and 128+4l ..
// 128+4l+3, so each float4 access of a warp covers 512 contiguous bytes) and
// writes them once.  The wait is bounded like every wait here.
constexpr int kDecodeWarpRows = 256;
constexpr int kDecodeMaxSmem = 96 * 1024;

__device__ __forceinline__ void bulk_load(void* dst, const void* src, int bytes,
                                          unsigned long long* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Three CTAs per SM (65 KB of staging each at cfg3 with beta 1): at most 40
// registers a thread; with 48 only two fit, and the cfg3 pass took 1.5x.
// kPer warps per target (a power of two); the slice is kPer x 256 rows.
template <int kPer>
__global__ void __launch_bounds__(kMaxDecodeTargets * 32, 3) decode_kernel(
    const __grid_constant__ DecodePlan plan) {
  extern __shared__ __align__(128) float slice[];   // [np + nt][span]
  __shared__ unsigned long long bar;
  __shared__ int abort;
  constexpr int span = kPer * kDecodeWarpRows, per_target = kPer;
  const int slices = (plan.m + span - 1) / span;
  const int col = int(blockIdx.x / slices), r0 = int(blockIdx.x % slices) * span;
  const long long batch = blockIdx.y;
  const int nin = plan.np + (plan.accumulate ? plan.nt : 0);
  const int rows = min(span, plan.m - r0);   // a multiple of 4 (m % 4 == 0)
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_expect_tx(&bar, nin * rows * 4);
  if (threadIdx.x < nin) {
    const int j = threadIdx.x;
    const Term& T = j < plan.np ? plan.in[j] : plan.out[j - plan.np];
    bulk_load(slice + j * span, T.p + batch * T.bstride + (long long)col * T.ld + r0, rows * 4,
              &bar);
  }
  if (!mbar_wait(abort, &bar, 0)) {
    if (threadIdx.x < nin) mbar_drain(&bar, 0);   // no copy outlives the CTA
    return;
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int t = warp / per_target, sub = (warp % per_target) * kDecodeWarpRows;
  if (t >= plan.nt || sub >= rows) return;
  constexpr int kHalf = kDecodeWarpRows / 2;
  float acc[8];   // rows sub + lane*4 + i (i < 4) and sub + kHalf + lane*4 + (i - 4)
  const float* own = slice + (plan.np + t) * span + sub + lane * 4;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    acc[i] = plan.accumulate ? own[i] : 0.f;
    acc[4 + i] = plan.accumulate ? own[kHalf + i] : 0.f;
  }
  for (int e = 0; e < plan.count[t]; ++e) {
    const int code = plan.list[t][e];
    const float* v = slice + ((code > 0 ? code : -code) - 1) * span + sub + lane * 4;
    const float4 v0 = *reinterpret_cast<const float4*>(v);
    const float4 v1 = *reinterpret_cast<const float4*>(v + kHalf);
    const float s = code > 0 ? 1.f : -1.f;
    acc[0] = fmaf(s, v0.x, acc[0]); acc[1] = fmaf(s, v0.y, acc[1]);
    acc[2] = fmaf(s, v0.z, acc[2]); acc[3] = fmaf(s, v0.w, acc[3]);
    acc[4] = fmaf(s, v1.x, acc[4]); acc[5] = fmaf(s, v1.y, acc[5]);
    acc[6] = fmaf(s, v1.z, acc[6]); acc[7] = fmaf(s, v1.w, acc[7]);
  }
  const Term& T = plan.out[t];
  float* column = const_cast<float*>(T.p) + batch * T.bstride + (long long)col * T.ld + r0 + sub;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = h * kHalf + lane * 4;
    if (sub + r < rows)
      *reinterpret_cast<float4*>(column + r) =
          make_float4(acc[4 * h], acc[4 * h + 1], acc[4 * h + 2], acc[4 * h + 3]);
  }
}

// Self-test of the bounded wait the leaf kernels use: thread 0 waits on an
// mbarrier that nothing arrives on, with a short limit; the wait must give
// up, set this file's device error word and the CTA's abort flag, and the
// kernel must return (the context stays usable).  *gave_up = 1 when it did.
__global__ void wait_selftest_kernel(unsigned long long limit_ns, int* gave_up) {
  __shared__ unsigned long long bar;
  __shared__ int abort;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x == 0) *gave_up = mbar_wait(abort, &bar, 0, limit_ns) ? 0 : 1;
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

// 3-D map {row_len k, rows, batch} over the prepared region, box 32 k x box_rows.
bool encode_region(CUtensorMap* m, const float* region, long long row_len, long long rows,
                   long long bstride, int batch, int box_rows) {
  const EncodeTiled enc = encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[3] = {cuuint64_t(row_len), cuuint64_t(rows), cuuint64_t(batch)};
  const long long bs = batch > 1 ? bstride : row_len * rows;
  const cuuint64_t strides[2] = {cuuint64_t(row_len) * 4, cuuint64_t(bs) * 4};
  const cuuint32_t box[3] = {cuuint32_t(kStageK), cuuint32_t(box_rows), 1u};
  const cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(region), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN>
cudaError_t launch_bn(const PrepLeafPlan& plan, const PrepMaps& maps, int batch,
                      cudaStream_t stream) {
  cudaError_t e = cudaFuncSetAttribute(leaf_prep_kernel<BN>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       Cfg<BN>::kSmemBytes);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 0;
  e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  const long long items = (long long)plan.ntiles * batch;
  if (items > INT32_MAX) return cudaErrorInvalidValue;
  const int grid = int(items < sms ? items : sms);   // one resident CTA per SM
  leaf_prep_kernel<BN><<<grid, Cfg<BN>::kThreads, Cfg<BN>::kSmemBytes, stream>>>(plan, maps,
                                                                                 int(items));
  return cudaGetLastError();
}

// Clusters of two leaf_pair_kernel CTAs that fit on the device at once (0 if
// none do); cached per device (value + 1; 0 = not yet known), safe to query
// from several host threads.
int pair_clusters() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  const int known = cache[dev].load(std::memory_order_acquire);
  if (known > 0) return known - 1;
  int n = 0;
  if (cudaFuncSetAttribute(leaf_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           pairk::kSmemBytes) == cudaSuccess) {
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2, 1, 1);
    cfg.blockDim = dim3(pairk::kThreads, 1, 1);
    cfg.dynamicSmemBytes = pairk::kSmemBytes;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, leaf_pair_kernel, &cfg) != cudaSuccess) n = 0;
  }
  cudaGetLastError();   // a refused query leaves no sticky error behind
  cache[dev].store(n + 1, std::memory_order_release);
  return n;
}

cudaError_t launch_pair(const PrepLeafPlan& plan, const PrepMaps& maps, int batch,
                        cudaStream_t stream) {
  const int clusters = pair_clusters();
  if (clusters < 1) return cudaErrorNotSupported;
  const long long items = (long long)plan.ntiles * batch;
  if (items > INT32_MAX) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(unsigned(2 * (items < clusters ? items : clusters)), 1, 1);
  cfg.blockDim = dim3(pairk::kThreads, 1, 1);
  cfg.dynamicSmemBytes = pairk::kSmemBytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, leaf_pair_kernel, plan, maps, int(items));
}

}  // namespace

bool prep_supported() { return encode_fn() != nullptr; }

bool prep_pair_supported() { return prep_supported() && pair_clusters() > 0; }

int prep_row_align() { return 64; }   // a multiple of the 32-k stage and the 64-k prepare tile

template <int kIn, int kP>
cudaError_t launch_prep_tree_kp(const PrepTreePlan& plan, int batch, cudaStream_t stream) {
  constexpr int smem = tree_smem_bytes<kIn>();
  cudaError_t e = cudaFuncSetAttribute(prep_tree_kernel<kIn, kP>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  prep_tree_kernel<kIn, kP>
      <<<dim3(unsigned(plan.ntiles), batch), kTreeThreads, smem, stream>>>(plan);
  return cudaGetLastError();
}

template <int kIn, int... P>
cudaError_t launch_prep_tree_in(const PrepTreePlan& plan, int kp, int batch, cudaStream_t stream,
                                std::integer_sequence<int, P...>) {
  cudaError_t e = cudaErrorInvalidValue;
  ((kp == P ? (e = launch_prep_tree_kp<kIn, P>(plan, batch, stream), true) : false) || ...);
  return e;
}

// Whether every segment of group G holds basis p's table for G's side (left
// operands the first table of the pair, right ones the second).
bool group_holds_pair(const TreeGroup& G, int p) {
  const TreeExprTable& T = kTreeExprTables[G.transpose ? 2 * p - 2 : 2 * p - 1];
  bool all = G.nseg > 0;
  for (int sg = 0; sg < G.nseg && all; ++sg) {
    const TreeSeg& S = G.seg[sg];
    all = S.nout == 7 && S.nmid >= 0 && S.nmid <= kTreeMid;
    for (int o = 0; o < 7 && all; ++o)
      for (int q = 0; q < kMaxOperandTerms && all; ++q) {
        const int want = q < 4 ? T.e[o][q] : 0;
        const int code = S.expr[o][q];
        all = code == want && (code == 0 || std::abs(code) <= S.nmid);
        if (code == 0) break;
      }
  }
  return all;
}

// The basis whose tables the launch's groups hold (1..4; the first that any
// group holds), with TreeGroup::table set on those groups; 0 when none does.
int mark_tree_tables(PrepTreePlan& plan) {
  for (int p = 1; 2 * p <= kTreeExprCount; ++p) {
    int held = 0;
    for (int g = 0; g < plan.ngroups; ++g) {
      plan.group[g].table = group_holds_pair(plan.group[g], p) ? 1 : 0;
      held += plan.group[g].table;
    }
    if (held) return p;
  }
  return 0;
}

cudaError_t launch_prep_tree(PrepTreePlan& plan, int batch, cudaStream_t stream) {
  if (plan.ngroups == 0 || plan.ntiles == 0 || batch == 0) return cudaSuccess;
  int nin = 0;
  for (int g = 0; g < plan.ngroups; ++g) {
    if (plan.group[g].nin < 0 || plan.group[g].nin > kTreeIn) return cudaErrorInvalidValue;
    nin = std::max(nin, plan.group[g].nin);
  }
  const int kp = mark_tree_tables(plan);
  g_last_tree_table = kp;
  constexpr auto pairs = std::make_integer_sequence<int, kTreeExprCount / 2 + 1>{};
  return nin <= kTreeSmallIn ? launch_prep_tree_in<kTreeSmallIn>(plan, kp, batch, stream, pairs)
                             : launch_prep_tree_in<kTreeIn>(plan, kp, batch, stream, pairs);
}

int last_tree_expr_table() { return g_last_tree_table; }

cudaError_t launch_leaf_prep(const PrepLeafPlan& plan, int kind, const float* region,
                             long long row_len, long long rows, long long region_bstride,
                             int batch, cudaStream_t stream) {
  if (plan.nprod == 0 || plan.ntiles == 0 || batch == 0) return cudaSuccess;
  if (kind != kPrepLeafSingle && kind != kPrepLeafPair) return cudaErrorInvalidValue;
  const int b_rows = kind == kPrepLeafPair ? 128 : 256;
  PrepMaps maps;
  std::memset(&maps, 0, sizeof(maps));
  if (!encode_region(&maps.a, region, row_len, rows, region_bstride, batch, 128) ||
      !encode_region(&maps.b, region, row_len, rows, region_bstride, batch, b_rows))
    return cudaErrorInvalidValue;
  return kind == kPrepLeafPair ? launch_pair(plan, maps, batch, stream)
                               : launch_bn<256>(plan, maps, batch, stream);
}

cudaError_t launch_decode(const DecodePlan& plan, int batch, cudaStream_t stream) {
  if (plan.np == 0 || plan.nt == 0 || plan.m == 0 || plan.n == 0 || batch == 0)
    return cudaSuccess;
  if (plan.m % 4) return cudaErrorInvalidValue;   // bulk copies move 16-byte multiples
  if (plan.nt > kMaxDecodeTargets || plan.np > kMaxDecodeProducts) return cudaErrorInvalidValue;
  const int nin = plan.np + (plan.accumulate ? plan.nt : 0);
  // Warps per target: a power of two keeping all 16 warps busy, a slice no
  // longer than the blocks need, and its staging within the shared-memory
  // budget.
  int per_target = 1;
  while (2 * per_target * plan.nt <= kMaxDecodeTargets) per_target *= 2;
  while (per_target > 1 && ((per_target / 2) * kDecodeWarpRows >= plan.m ||
                            size_t(nin) * per_target * kDecodeWarpRows * 4 > kDecodeMaxSmem))
    per_target /= 2;
  const int span = per_target * kDecodeWarpRows;
  const long long slices = (plan.m + span - 1) / span;
  const long long blocks = slices * plan.n;
  if (blocks > INT32_MAX) return cudaErrorInvalidValue;
  const size_t smem = size_t(nin) * span * sizeof(float);
  auto go = [&](auto kernel) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         int(smem));
    if (e != cudaSuccess) return e;
    kernel<<<dim3(unsigned(blocks), unsigned(batch)), kMaxDecodeTargets * 32, smem, stream>>>(plan);
    return cudaGetLastError();
  };
  switch (per_target) {
    case 1: return go(decode_kernel<1>);
    case 2: return go(decode_kernel<2>);
    case 4: return go(decode_kernel<4>);
    case 8: return go(decode_kernel<8>);
    default: return go(decode_kernel<16>);
  }
}

cudaError_t run_wait_selftest(unsigned long long limit_ns, int* gave_up_device,
                              cudaStream_t stream) {
  wait_selftest_kernel<<<1, 32, 0, stream>>>(limit_ns, gave_up_device);
  return cudaGetLastError();
}

cudaError_t read_and_clear_tc3_device_error(unsigned* value) {
  cudaError_t e = cudaMemcpyFromSymbol(value, g_tc3_device_error, sizeof(unsigned));
  if (e != cudaSuccess) return e;
  const unsigned zero = 0;
  return cudaMemcpyToSymbol(g_tc3_device_error, &zero, sizeof(unsigned));
}

TileShape prep_tile_shape(int kind) {
  return kind == kPrepLeafPair ? TileShape{pairk::kTileM, pairk::kTileN} : TileShape{128, 256};
}

}  // namespace bag_b200
