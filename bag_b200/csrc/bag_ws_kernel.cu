// Warp-specialised leaf kernel of the BAG FP32 matmul (sm_100a).
//
// One launch runs every leaf product of a plan whose operands are 16-byte
// aligned (the fast signatures of bag_plan.h).  Each CTA of 384 threads owns a
// 128 x 128 output tile of one product:
//
//  * 4 producer warps copy the raw k-tiles of every signed operand term
//    several tiles ahead into a shared-memory ring with 16-byte cp.async (each
//    thread its own chunks, so no barrier between producers; the prefetch
//    distance is the ring depth, 5-7 tiles, not registers), then sum the
//    terms in the reference's order (x + delta*y, bag.cuh:69-73), and store
//    the transformed A tile (k-major)
//    and B tile (in its natural K-contiguous layout, 16-byte chunks
//    XOR-swizzled so both the stores and the consumers' column reads hit 32
//    distinct banks) into a 4-stage shared-memory ring, then arrive on the
//    stage's "full" mbarrier;
//  * 8 consumer warps wait on "full", run the register-blocked outer product
//    (8 x 8 outputs per thread) with Blackwell's paired FMA __ffma2_rn (two
//    IEEE round-to-nearest fmaf per instruction, so every output stays one
//    sequential fmaf chain over k), arrive on the stage's "empty" mbarrier,
//    and finally add coef*M into every target C block (128-bit red.global).
//
// Every mbarrier wait polls try_wait (which waits in hardware for a short
// system-defined time per call) and is bounded: after kWaitLimitNs of wall time the thread sets
// g_device_error and leaves its loop, so a logic error cannot hang the GPU;
// a producer that gives up first waits for its own copies in flight.
#include <cuda_runtime.h>

#include <cstdint>

#include "bag_kernels.h"

namespace bag_b200 {

__device__ unsigned int g_device_error = 0;

namespace {

constexpr int kBM = 128, kBN = 128, kBK = 8, kStages = 4;
constexpr int kConsumers = 256, kProducers = 128, kThreads = kConsumers + kProducers;
// Raw operand ring of the producers (dynamic shared memory): per tile and
// producer thread 2 float4 chunks per operand term.
constexpr int kRawBytes = 144 * 1024;
constexpr unsigned long long kWaitLimitNs = 2000000000ull; // give up after 2 s

struct WsSmem {
  float a[kStages][kBK][kBM];   // A tile, k-major: a[s][k][m]
  float b[kStages][kBN][kBK];   // B tile, n-major: b[s][n][chunk' * 4 + e], chunk' swizzled
  unsigned long long full[kStages];
  unsigned long long empty[kStages];
};

constexpr int kWsSmemBytes = (int(sizeof(WsSmem)) + 127) / 128 * 128;
constexpr int kWsDynBytes = kWsSmemBytes + kRawBytes;
static_assert(kWsDynBytes <= 227 * 1024, "shared memory per CTA");

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

// One try_wait with the hardware's own (short) time limit.  A suspend-time
// hint here compiled to sleeps whose wake-up came well after the stage was
// ready: measured on B200, 3.4 sleeps per warp per k-tile and the FMA pipe
// idle a third of the time.
__device__ __forceinline__ bool mbar_try_wait(unsigned long long* bar, unsigned parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait for the phase of parity `parity`: gives up (error word set,
// false) when the phase has not completed after kWaitLimitNs of wall time.
__device__ __forceinline__ bool mbar_wait(unsigned long long* bar, unsigned parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long start = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_ns() - start > kWaitLimitNs) {
      atomicOr(&g_device_error, 1u);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ const Prod& find_prod(const LeafPlan& plan, int item) {
  int pid = 0;
  while (pid + 1 < plan.nprod && plan.prod[pid + 1].tile_begin <= item) ++pid;
  return plan.prod[pid];
}

__device__ __forceinline__ float4 add_signed(float4 acc, float4 v, float coef) {
  return make_float4(fmaf(coef, v.x, acc.x), fmaf(coef, v.y, acc.y), fmaf(coef, v.z, acc.z),
                     fmaf(coef, v.w, acc.w));
}

__device__ __forceinline__ float4 signed_first(float4 v, float coef) {
  return coef < 0.f ? make_float4(-v.x, -v.y, -v.z, -v.w) : v;
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Raw ring geometry for a signature: slots of 2 (NL + NR) float4 per
// producer thread; the prefetch distance is one less than the slot count.
template <int NL, int NR>
struct RawRing {
  static constexpr int kChunks = 2 * (NL + NR);
  static constexpr int kSlotBytes = kChunks * kProducers * 16;
  static constexpr int kSlots = (kRawBytes / kSlotBytes) < 8 ? (kRawBytes / kSlotBytes) : 8;
  static constexpr int kAhead = kSlots - 1;
  static_assert(kSlots >= 3, "raw ring too shallow");
};

// Producer: 128 threads.  Thread p copies A chunks (rows a_m..a_m+3 of
// columns a_k and a_k+4) and B chunks (k-chunk b_kc of columns b_n and
// b_n+64) of every term into its own slots of the raw ring, kAhead tiles
// ahead, and later sums them into the stage ring.
template <int NL, int NR>
__device__ __forceinline__ void produce(const LeafPlan& plan, const Prod& P, int m0, int n0,
                                        long long batch, WsSmem& sm, float4* raw, int p,
                                        int ktiles) {
  using R = RawRing<NL, NR>;
  const int a_m = (p % 32) * 4, a_k = p / 32;
  const int b_n = p / 2, b_kc = p % 2;
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
  const long long oa = min(m0 + a_m, P.m - 4) + (long long)a_k * lda;
  const long long ob0 = b_kc * 4 + (long long)min(n0 + b_n, P.n - 1) * ldb;
  const long long ob1 = b_kc * 4 + (long long)min(n0 + b_n + 64, P.n - 1) * ldb;

  // Copy tile kt's chunks of this thread into slot kt % kSlots; chunks past k
  // are zero-filled (k % 4 == 0 here), their source clamped to the tile start.
  auto issue = [&](int kt) {
    float4* slot = raw + (kt % R::kSlots) * R::kChunks * kProducers + p;
    const int k0 = kt * kBK;
    const bool a0 = k0 + a_k < P.k, a1 = k0 + a_k + 4 < P.k, bk = k0 + b_kc * 4 < P.k;
    const long long oak0 = a0 ? oa + (long long)k0 * lda : oa;
    const long long oak1 = a1 ? oa + (long long)(k0 + 4) * lda : oa;
    const long long ok0 = bk ? ob0 + k0 : ob0, ok1 = bk ? ob1 + k0 : ob1;
#pragma unroll
    for (int t = 0; t < NL; ++t) {
      cp_async16(slot + (2 * t) * kProducers, ba[t] + oak0, a0 ? 16 : 0);
      cp_async16(slot + (2 * t + 1) * kProducers, ba[t] + oak1, a1 ? 16 : 0);
    }
#pragma unroll
    for (int t = 0; t < NR; ++t) {
      cp_async16(slot + (2 * (NL + t)) * kProducers, bb[t] + ok0, bk ? 16 : 0);
      cp_async16(slot + (2 * (NL + t) + 1) * kProducers, bb[t] + ok1, bk ? 16 : 0);
    }
  };
  // Sum slot kt's terms and store the transformed tiles into stage s.
  auto store = [&](int kt, int s) {
    const float4* slot = raw + (kt % R::kSlots) * R::kChunks * kProducers + p;
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      float4 v = signed_first(slot[q * kProducers], ca[0]);
#pragma unroll
      for (int t = 1; t < NL; ++t) v = add_signed(v, slot[(2 * t + q) * kProducers], ca[t]);
      *reinterpret_cast<float4*>(&sm.a[s][a_k + 4 * q][a_m]) = v;
    }
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      float4 v = signed_first(slot[(2 * NL + q) * kProducers], cb[0]);
#pragma unroll
      for (int t = 1; t < NR; ++t) v = add_signed(v, slot[(2 * (NL + t) + q) * kProducers], cb[t]);
      const int n = b_n + 64 * q;
      *reinterpret_cast<float4*>(&sm.b[s][n][(b_kc ^ ((n >> 2) & 1)) * 4]) = v;
    }
  };

  // Every iteration commits one group (empty past the last tile), so
  // wait_group kAhead always means "tile kt has landed".
#pragma unroll
  for (int d = 0; d < R::kAhead; ++d) {
    if (d < ktiles) issue(d);
    cp_async_commit();
  }
  for (int kt = 0; kt < ktiles; ++kt) {
    // Slot (kt + kAhead) % kSlots held tile kt - 1, already summed.
    if (kt + R::kAhead < ktiles) issue(kt + R::kAhead);
    cp_async_commit();
    cp_async_wait<R::kAhead>();
    const int s = kt % kStages;
    if (kt >= kStages && !mbar_wait(&sm.empty[s], ((kt / kStages) - 1) & 1)) {
      cp_async_wait<0>();   // no copy outlives the CTA
      return;
    }
    store(kt, s);
    mbar_arrive(&sm.full[s]);
  }
  cp_async_wait<0>();
}

// Consumer: 256 threads in 8 warps (4 along M x 2 along N).  Thread rows are
// wm + lane_m*4 + {0..3, 16..19}; columns wn + lane_n + 8c, c = 0..7.  The
// fragment loads are software-pipelined: while the FFMA2s of step k run, the
// A fragment of step k+1 (and, at the end of a 4-k group, the B fragments of
// the next group; at the end of a stage, the first fragments of the next
// stage) are already in flight, so a warp never starts a step waiting on
// shared memory -- the eight consumer warps leave each stage barrier
// together, and without this their load stalls coincide.  Every output is
// still one sequential fmaf chain over k.
__device__ __forceinline__ void load_b(const WsSmem& sm, int s, int kq, int col, int swz,
                                       float4 (&b)[8]) {
#pragma unroll
  for (int c = 0; c < 8; ++c)
    b[c] = *reinterpret_cast<const float4*>(&sm.b[s][col + 8 * c][(kq ^ swz) * 4]);
}

__device__ __forceinline__ void load_a(const WsSmem& sm, int s, int k, int am, float4& a0,
                                       float4& a1) {
  a0 = *reinterpret_cast<const float4*>(&sm.a[s][k][am]);
  a1 = *reinterpret_cast<const float4*>(&sm.a[s][k][am + 16]);
}

template <int KK>
__device__ __forceinline__ void ffma_step(const float4 (&b)[8], float4 a0, float4 a1,
                                          float2 (&acc)[4][8]) {
  const float2 ap[4] = {make_float2(a0.x, a0.y), make_float2(a0.z, a0.w),
                        make_float2(a1.x, a1.y), make_float2(a1.z, a1.w)};
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const float bv = KK == 0 ? b[c].x : KK == 1 ? b[c].y : KK == 2 ? b[c].z : b[c].w;
    const float2 b2 = make_float2(bv, bv);
#pragma unroll
    for (int ip = 0; ip < 4; ++ip) acc[ip][c] = __ffma2_rn(ap[ip], b2, acc[ip][c]);
  }
}

__device__ __forceinline__ bool consume(WsSmem& sm, int ctid, int ktiles, float2 (&acc)[4][8]) {
  static_assert(kBK == 8, "two 4-k groups per stage");
  const int warp = ctid >> 5, lane = ctid & 31;
  const int lane_m = lane >> 3, lane_n = lane & 7;
  const int wm = (warp & 3) * 32, wn = (warp >> 2) * 64;
  const int am = wm + lane_m * 4, col = wn + lane_n;
  const int swz = (lane_n >> 2) & 1;   // bit 2 of every column this thread reads
  if (ktiles <= 0) return true;
  float4 b0[8], b1[8];   // the current and the next 4-k group's B fragments
  float4 a0, a1, n0, n1;
  if (!mbar_wait(&sm.full[0], 0)) return false;
  load_b(sm, 0, 0, col, swz, b0);
  load_a(sm, 0, 0, am, a0, a1);
  for (int kt = 0; kt < ktiles; ++kt) {
    const int s = kt % kStages;
    // Group 0 (k 0..3) on b0; its last step also fetches group 1's B.
    load_a(sm, s, 1, am, n0, n1);
    ffma_step<0>(b0, a0, a1, acc);
    load_a(sm, s, 2, am, a0, a1);
    ffma_step<1>(b0, n0, n1, acc);
    load_a(sm, s, 3, am, n0, n1);
    ffma_step<2>(b0, a0, a1, acc);
    load_b(sm, s, 1, col, swz, b1);
    load_a(sm, s, 4, am, a0, a1);
    ffma_step<3>(b0, n0, n1, acc);
    // Group 1 (k 4..7) on b1; its last step fetches the next stage's first
    // fragments once that stage has landed.
    load_a(sm, s, 5, am, n0, n1);
    ffma_step<0>(b1, a0, a1, acc);
    load_a(sm, s, 6, am, a0, a1);
    ffma_step<1>(b1, n0, n1, acc);
    load_a(sm, s, 7, am, n0, n1);
    ffma_step<2>(b1, a0, a1, acc);
    if (kt + 1 < ktiles) {
      const int s1 = (kt + 1) % kStages;
      if (!mbar_wait(&sm.full[s1], ((kt + 1) / kStages) & 1)) return false;
      load_b(sm, s1, 0, col, swz, b0);
      load_a(sm, s1, 0, am, a0, a1);
    }
    ffma_step<3>(b1, n0, n1, acc);
    mbar_arrive(&sm.empty[s]);
  }
  return true;
}

__device__ __forceinline__ void store_outputs(const LeafPlan& plan, const Prod& P, int m0, int n0,
                                              long long batch, int ctid,
                                              const float2 (&acc)[4][8]) {
  const int warp = ctid >> 5, lane = ctid & 31;
  const int lane_m = lane >> 3, lane_n = lane & 7;
  const int wm = (warp & 3) * 32, wn = (warp >> 2) * 64;
  for (int o = 0; o < P.no; ++o) {
    const Term& T = plan.terms[P.o0 + o];
    float* base = const_cast<float*>(T.p) + batch * T.bstride;
    const float coef = T.coef;
    const int mode = T.mode;
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      const int r = m0 + wm + lane_m * 4 + 16 * g;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const int col = n0 + wn + lane_n + 8 * c;
        if (col >= P.n || r >= P.m) continue;
        float* q = base + r + (long long)col * T.ld;
        const float v[4] = {coef * acc[2 * g][c].x, coef * acc[2 * g][c].y,
                            coef * acc[2 * g + 1][c].x, coef * acc[2 * g + 1][c].y};
        if (r + 3 < P.m) {
          float4* q4 = reinterpret_cast<float4*>(q);
          if (mode == kOutAtomic) {
            atomicAdd(q4, make_float4(v[0], v[1], v[2], v[3]));
          } else if (mode == kOutAdd) {
            const float4 old = *q4;
            *q4 = make_float4(old.x + v[0], old.y + v[1], old.z + v[2], old.w + v[3]);
          } else {
            *q4 = make_float4(v[0], v[1], v[2], v[3]);
          }
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            if (r + e >= P.m) break;
            if (mode == kOutAtomic) atomicAdd(q + e, v[e]);
            else if (mode == kOutAdd) q[e] += v[e];
            else q[e] = v[e];
          }
        }
      }
    }
  }
}

}  // namespace

__global__ void __launch_bounds__(kThreads, 1) leaf_ws_kernel(const __grid_constant__ LeafPlan plan) {
  // Dynamic shared memory: the stage ring and barriers, then the producers'
  // raw ring (kRawBytes).
  extern __shared__ __align__(16) unsigned char dyn[];
  WsSmem& sm = *reinterpret_cast<WsSmem*>(dyn);
  float4* raw = reinterpret_cast<float4*>(dyn + kWsSmemBytes);
  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], kProducers);
      mbar_init(&sm.empty[s], kConsumers);
    }
  }
  __syncthreads();
  const Prod& P = find_prod(plan, blockIdx.x);
  const int local = blockIdx.x - P.tile_begin;
  constexpr int GROUP_M = 8;   // CTAs resident together share operand panels in L2
  const int in_group = GROUP_M * P.tiles_n;
  const int first_m = (local / in_group) * GROUP_M;
  const int gsize = min(P.tiles_m - first_m, GROUP_M);
  const int m0 = (first_m + (local % in_group) % gsize) * kBM;
  const int n0 = ((local % in_group) / gsize) * kBN;
  const long long batch = blockIdx.y;
  const int ktiles = (P.k + kBK - 1) / kBK;

  if (threadIdx.x >= kConsumers) {
    const int p = threadIdx.x - kConsumers;
    switch (P.sig) {
      case kSig11: produce<1, 1>(plan, P, m0, n0, batch, sm, raw, p, ktiles); break;
      case kSig12: produce<1, 2>(plan, P, m0, n0, batch, sm, raw, p, ktiles); break;
      case kSig21: produce<2, 1>(plan, P, m0, n0, batch, sm, raw, p, ktiles); break;
      case kSig22: produce<2, 2>(plan, P, m0, n0, batch, sm, raw, p, ktiles); break;
      case kSig33: produce<3, 3>(plan, P, m0, n0, batch, sm, raw, p, ktiles); break;
      case kSig41: produce<4, 1>(plan, P, m0, n0, batch, sm, raw, p, ktiles); break;
      case kSig14: produce<1, 4>(plan, P, m0, n0, batch, sm, raw, p, ktiles); break;
      default: atomicOr(&g_device_error, 2u); break;   // the host never sends these here
    }
    return;
  }
  float2 acc[4][8];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[i][c] = make_float2(0.f, 0.f);
  if (P.sig == kSigGeneric) return;
  if (!consume(sm, threadIdx.x, ktiles, acc)) return;
  store_outputs(plan, P, m0, n0, batch, threadIdx.x, acc);
}

TileShape ws_tile_shape() { return {kBM, kBN}; }

cudaError_t launch_leaf_ws(const LeafPlan& plan, int batch, cudaStream_t stream) {
  if (plan.nprod == 0 || plan.ntiles == 0 || batch == 0) return cudaSuccess;
  const cudaError_t e =
      cudaFuncSetAttribute(leaf_ws_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kWsDynBytes);
  if (e != cudaSuccess) return e;
  leaf_ws_kernel<<<dim3(plan.ntiles, batch), kThreads, kWsDynBytes, stream>>>(plan);
  return cudaGetLastError();
}

cudaError_t read_and_clear_device_error(unsigned* value) {
  cudaError_t e = cudaMemcpyFromSymbol(value, g_device_error, sizeof(unsigned));
  if (e != cudaSuccess) return e;
  const unsigned zero = 0;
  return cudaMemcpyToSymbol(g_device_error, &zero, sizeof(unsigned));
}

}  // namespace bag_b200
