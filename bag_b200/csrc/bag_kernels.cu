// sm_100a kernels of the BAG FP32 matmul.
//
// leaf_gemm_kernel: one launch runs every leaf product of a plan.  Each CTA
//   owns a BM x BN output tile of one product.  Its prologue loads 128-bit
//   column-major vectors of every signed operand term into registers one
//   k-tile ahead, sums them in FP32 in the reference's evaluation order
//   (x+delta*y, bag.cuh:69-73 / simt.cuh:14-33) just before staging the
//   transformed tile into double-buffered shared memory; the main loop is a
//   register-blocked FFMA outer product (TM x TN per thread) in which every
//   output is a sequential fmaf chain over k; the epilogue adds coef*M into
//   each C block the inverse transform sends the product to (bag.py:530-533
//   direct decode), with 128-bit red.global adds when products share outputs.
//
//   The common term counts per operand (1..4) have compile-time main loops
//   with no bounds checks: M/N addresses of edge tiles are clamped (those rows
//   and columns are never stored) and only a partial last k-tile is masked.
//   Anything else -- misaligned operands, ragged extents, other term counts --
//   runs the generic loop with runtime term counts and element masks.
//
// materialize_kernel: elementwise signed sums of up to four blocks into the
//   workspace, for operands the reference rounds before recursing.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>

#include "bag_kernels.h"

namespace bag_b200 {
namespace {

template <int BM_, int BN_, int BK_, int TM_, int TN_, int MINB_, bool DB_, bool F2_>
struct Cfg {
  static constexpr int BM = BM_, BN = BN_, BK = BK_, TM = TM_, TN = TN_, MINB = MINB_;
  static constexpr bool DB = DB_;                  // double-buffered register fragments
  static constexpr bool F2 = F2_;                  // paired FMA (__ffma2_rn) outer product
  static constexpr int NT = (BM / TM) * (BN / TN); // threads
  static constexpr int WM = 4 * TM;                // warp tile: 4 x 8 lanes of TM x TN
  static constexpr int WN = 8 * TN;
  static constexpr int WARPS_M = BM / WM;
  static constexpr int A_VECS = BM * BK / 4 / NT;  // float4 per thread per term
  static constexpr int B_VECS = BN * BK / 4 / NT;
  static constexpr int SWZ = 128 / BK;             // XOR key step per 4-row group of B
  static_assert((BM / WM) * (BN / WN) * 32 == NT, "warp layout");
  static_assert(TM % 4 == 0 && TN % 4 == 0, "fragments are float4 groups");
  static_assert(A_VECS >= 1 && A_VECS * NT * 4 == BM * BK, "A load split");
  static_assert(B_VECS >= 1 && B_VECS * NT * 4 == BN * BK, "B load split");
  static_assert(NT % (BM / 4) == 0 && NT % (BK / 4) == 0, "vector rows repeat across q");
  static_assert(BK % 4 == 0 && BK <= 32, "k tiling");
};

template <class C>
struct Smem {
  float a[2][C::BK][C::BM];
  float b[2][C::BK][C::BN];
};

struct Ctx {
  int m0, n0;
  long long batch;
  int tid, lane_m, lane_n, wm, wn;
};

__device__ __forceinline__ const Prod& find_product(const LeafPlan& plan, int item) {
  int pid = 0;
  while (pid + 1 < plan.nprod && plan.prod[pid + 1].tile_begin <= item) ++pid;
  return plan.prod[pid];
}

__device__ __forceinline__ float4 ldg4(const float* p) {
  return __ldg(reinterpret_cast<const float4*>(p));
}

// acc (+)= coef * v, rounded once per element: coef is +-1, so the product is
// exact and fmaf gives RN(acc +- v), the reference's x + delta*y.
__device__ __forceinline__ float4 accumulate(float4 acc, float4 v, float coef, bool first) {
  if (first) return make_float4(coef * v.x, coef * v.y, coef * v.z, coef * v.w);
  return make_float4(fmaf(coef, v.x, acc.x), fmaf(coef, v.y, acc.y), fmaf(coef, v.z, acc.z),
                     fmaf(coef, v.w, acc.w));
}

// Load four consecutive rows (r..r+3) of column c, zero outside [0,rows)x[0,cols).
template <bool VEC>
__device__ __forceinline__ float4 load4_masked(const float* __restrict__ p, int ld, int r, int c,
                                               int rows, int cols) {
  float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
  if (c >= cols) return v;
  const float* q = p + r + (long long)c * ld;
  if (VEC && r + 3 < rows) {
    v = ldg4(q);
  } else {
    if (r + 0 < rows) v.x = __ldg(q + 0);
    if (r + 1 < rows) v.y = __ldg(q + 1);
    if (r + 2 < rows) v.z = __ldg(q + 2);
    if (r + 3 < rows) v.w = __ldg(q + 3);
  }
  return v;
}

template <class C>
__device__ __forceinline__ void store_a(Smem<C>& sm, int s, int r, int c, float4 v) {
  *reinterpret_cast<float4*>(&sm.a[s][c][r]) = v;
}

// The K-contiguous B vector is transposed into four rows; XOR-swizzling the
// column by the 4-row group keeps one warp's stores on 32 distinct banks and
// leaves every 4-column group contiguous for the float4 fragment reads.
template <class C>
__device__ __forceinline__ void store_b(Smem<C>& sm, int s, int k, int c, float4 v) {
  const int col = c ^ ((k >> 2) * C::SWZ);
  sm.b[s][k + 0][col] = v.x;
  sm.b[s][k + 1][col] = v.y;
  sm.b[s][k + 2][col] = v.z;
  sm.b[s][k + 3][col] = v.w;
}

template <class C>
__device__ __forceinline__ void load_fragments(const Smem<C>& sm, int s, int kk, const Ctx& x,
                                               float (&a)[C::TM], float (&b)[C::TN]) {
#pragma unroll
  for (int i = 0; i < C::TM / 4; ++i)
    *reinterpret_cast<float4*>(&a[4 * i]) =
        *reinterpret_cast<const float4*>(&sm.a[s][kk][x.wm + x.lane_m * 4 + i * 16]);
  const int key = (kk >> 2) * C::SWZ;
#pragma unroll
  for (int j = 0; j < C::TN / 4; ++j)
    *reinterpret_cast<float4*>(&b[4 * j]) = *reinterpret_cast<const float4*>(
        &sm.b[s][kk][(x.wn + x.lane_n * 4 + j * 32) ^ key]);
}

// Accumulators are packed in pairs of consecutive rows: acc[i/2][j] holds
// outputs (i, j) and (i+1, j) for even i.
template <class C>
using Acc = float2[C::TM / 2][C::TN];

// BK k-steps of the register-blocked outer product on stage s, with the
// fragments of step kk+1 read from shared memory while step kk's FMAs issue.
// Blackwell's paired FMA (__ffma2_rn: two IEEE round-to-nearest fmaf per
// instruction) halves the issue slots of the outer product, so the FP32 pipe
// rather than instruction issue bounds the loop; every output is still one
// sequential fmaf chain over k.
template <class C>
__device__ __forceinline__ void compute_tile(const Smem<C>& sm, int s, const Ctx& x,
                                             Acc<C>& acc) {
  constexpr int NB = C::DB ? 2 : 1;
  float a[NB][C::TM], b[NB][C::TN];
  if (C::DB) load_fragments<C>(sm, s, 0, x, a[0], b[0]);
#pragma unroll
  for (int kk = 0; kk < C::BK; ++kk) {
    if (!C::DB) load_fragments<C>(sm, s, kk, x, a[0], b[0]);
    else if (kk + 1 < C::BK)
      load_fragments<C>(sm, s, kk + 1, x, a[(kk + 1) % NB], b[(kk + 1) % NB]);
    const float* ak = a[kk % NB];
    const float* bk = b[kk % NB];
#pragma unroll
    for (int j = 0; j < C::TN; ++j) {
      if constexpr (C::F2) {
        const float2 bj = make_float2(bk[j], bk[j]);
#pragma unroll
        for (int i = 0; i < C::TM / 2; ++i)
          acc[i][j] = __ffma2_rn(make_float2(ak[2 * i], ak[2 * i + 1]), bj, acc[i][j]);
      } else {
#pragma unroll
        for (int i = 0; i < C::TM / 2; ++i) {
          acc[i][j].x = fmaf(ak[2 * i], bk[j], acc[i][j].x);
          acc[i][j].y = fmaf(ak[2 * i + 1], bk[j], acc[i][j].y);
        }
      }
    }
  }
}

template <class C>
__device__ __forceinline__ float acc_at(const Acc<C>& acc, int i, int j) {
  return (i & 1) ? acc[i >> 1][j].y : acc[i >> 1][j].x;
}

// ---------------------------------------------------------------------------
// Fast path: NL left and NR right terms known at compile time, every operand
// 16-byte aligned with ld % 4 == 0, m % 4 == 0 and k % 4 == 0.
// ---------------------------------------------------------------------------
template <class C, int NL, int NR>
__device__ __forceinline__ void tile_fast(const LeafPlan& plan, const Prod& P, const Ctx& x,
                                          Smem<C>& sm, Acc<C>& acc) {
  constexpr int AQ = C::NT / (C::BM / 4);   // A columns between a thread's vectors
  constexpr int BQ = C::NT / (C::BK / 4);   // B columns between a thread's vectors
  const int a_r = (x.tid % (C::BM / 4)) * 4;
  const int a_c = x.tid / (C::BM / 4);
  const int b_k = (x.tid % (C::BK / 4)) * 4;
  const int b_c = x.tid / (C::BK / 4);

  // Every term of an operand shares one leading dimension (the host routes
  // plans where they differ to the generic loop), so one per-thread offset
  // serves all terms; the term bases are warp-uniform.
  const long long lda = plan.terms[P.l0].ld;
  const long long ldb = plan.terms[P.r0].ld;
  const float* ba[NL];
  float ca[NL];
#pragma unroll
  for (int t = 0; t < NL; ++t) {
    const Term& T = plan.terms[P.l0 + t];
    ba[t] = T.p + x.batch * T.bstride;
    ca[t] = T.coef;
  }
  const float* bb[NR];
  float cb[NR];
#pragma unroll
  for (int t = 0; t < NR; ++t) {
    const Term& T = plan.terms[P.r0 + t];
    bb[t] = T.p + x.batch * T.bstride;
    cb[t] = T.coef;
  }
  // Clamped: rows >= m and columns >= n are loaded but never stored.
  long long oa = min(x.m0 + a_r, P.m - 4) + (long long)a_c * lda;
  long long ob[C::B_VECS];
#pragma unroll
  for (int q = 0; q < C::B_VECS; ++q)
    ob[q] = b_k + (long long)min(x.n0 + b_c + q * BQ, P.n - 1) * ldb;

  float4 la[NL][C::A_VECS], lb[NR][C::B_VECS];
  auto load_full = [&]() {
#pragma unroll
    for (int t = 0; t < NL; ++t)
#pragma unroll
      for (int q = 0; q < C::A_VECS; ++q) la[t][q] = ldg4(ba[t] + oa + q * AQ * lda);
#pragma unroll
    for (int t = 0; t < NR; ++t)
#pragma unroll
      for (int q = 0; q < C::B_VECS; ++q) lb[t][q] = ldg4(bb[t] + ob[q]);
    oa += C::BK * lda;
#pragma unroll
    for (int q = 0; q < C::B_VECS; ++q) ob[q] += C::BK;
  };
  auto load_tail = [&](int k0) {   // last, partial k-tile: zero beyond k
#pragma unroll
    for (int t = 0; t < NL; ++t)
#pragma unroll
      for (int q = 0; q < C::A_VECS; ++q)
        la[t][q] = (k0 + a_c + q * AQ < P.k) ? ldg4(ba[t] + oa + q * AQ * lda)
                                             : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int t = 0; t < NR; ++t)
#pragma unroll
      for (int q = 0; q < C::B_VECS; ++q)
        lb[t][q] = (k0 + b_k < P.k) ? ldg4(bb[t] + ob[q]) : make_float4(0.f, 0.f, 0.f, 0.f);
  };
  auto store = [&](int s) {
#pragma unroll
    for (int q = 0; q < C::A_VECS; ++q) {
      float4 v = la[0][q];
      if (ca[0] < 0.f) v = make_float4(-v.x, -v.y, -v.z, -v.w);
#pragma unroll
      for (int t = 1; t < NL; ++t) v = accumulate(v, la[t][q], ca[t], false);
      store_a<C>(sm, s, a_r, a_c + q * AQ, v);
    }
#pragma unroll
    for (int q = 0; q < C::B_VECS; ++q) {
      float4 v = lb[0][q];
      if (cb[0] < 0.f) v = make_float4(-v.x, -v.y, -v.z, -v.w);
#pragma unroll
      for (int t = 1; t < NR; ++t) v = accumulate(v, lb[t][q], cb[t], false);
      store_b<C>(sm, s, b_k, b_c + q * BQ, v);
    }
  };

  const int kfull = P.k / C::BK;
  const int ktiles = (P.k + C::BK - 1) / C::BK;
  if (ktiles == 0) return;
  if (kfull > 0) load_full();
  else load_tail(0);
  store(0);
  __syncthreads();
  for (int kt = 0; kt < ktiles; ++kt) {
    const int s = kt & 1;
    if (kt + 1 < ktiles) {
      if (kt + 1 < kfull) load_full();
      else load_tail((kt + 1) * C::BK);
    }
    compute_tile<C>(sm, s, x, acc);
    if (kt + 1 < ktiles) store(s ^ 1);
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Generic path: runtime term counts, masked element loads.
// ---------------------------------------------------------------------------
template <class C, bool VEC>
__device__ __forceinline__ void tile_generic(const LeafPlan& plan, const Prod& P, const Ctx& x,
                                             Smem<C>& sm, Acc<C>& acc) {
  int a_r[C::A_VECS], a_c[C::A_VECS], b_k[C::B_VECS], b_c[C::B_VECS];
#pragma unroll
  for (int q = 0; q < C::A_VECS; ++q) {
    const int idx = x.tid + q * C::NT;
    a_r[q] = (idx % (C::BM / 4)) * 4;
    a_c[q] = idx / (C::BM / 4);
  }
#pragma unroll
  for (int q = 0; q < C::B_VECS; ++q) {
    const int idx = x.tid + q * C::NT;
    b_k[q] = (idx % (C::BK / 4)) * 4;
    b_c[q] = idx / (C::BK / 4);
  }
  float4 ra[C::A_VECS], rb[C::B_VECS];
  auto load_tile = [&](int k0) {
    for (int t = 0; t < P.nl; ++t) {
      const Term& T = plan.terms[P.l0 + t];
      const float* base = T.p + x.batch * T.bstride;
#pragma unroll
      for (int q = 0; q < C::A_VECS; ++q)
        ra[q] = accumulate(ra[q],
                           load4_masked<VEC>(base, T.ld, x.m0 + a_r[q], k0 + a_c[q], P.m, P.k),
                           T.coef, t == 0);
    }
    for (int t = 0; t < P.nr; ++t) {
      const Term& T = plan.terms[P.r0 + t];
      const float* base = T.p + x.batch * T.bstride;
#pragma unroll
      for (int q = 0; q < C::B_VECS; ++q)
        rb[q] = accumulate(rb[q],
                           load4_masked<VEC>(base, T.ld, k0 + b_k[q], x.n0 + b_c[q], P.k, P.n),
                           T.coef, t == 0);
    }
  };
  auto store = [&](int s) {
#pragma unroll
    for (int q = 0; q < C::A_VECS; ++q) store_a<C>(sm, s, a_r[q], a_c[q], ra[q]);
#pragma unroll
    for (int q = 0; q < C::B_VECS; ++q) store_b<C>(sm, s, b_k[q], b_c[q], rb[q]);
  };
  const int ktiles = (P.k + C::BK - 1) / C::BK;
  if (ktiles == 0) return;
  load_tile(0);
  store(0);
  __syncthreads();
  for (int kt = 0; kt < ktiles; ++kt) {
    const int s = kt & 1;
    if (kt + 1 < ktiles) load_tile((kt + 1) * C::BK);
    compute_tile<C>(sm, s, x, acc);
    if (kt + 1 < ktiles) store(s ^ 1);
    __syncthreads();
  }
}

// Inverse transform: signed updates of every target block of the product.
template <class C, bool VEC>
__device__ __forceinline__ void epilogue(const LeafPlan& plan, const Prod& P, const Ctx& x,
                                         const Acc<C>& acc) {
  for (int o = 0; o < P.no; ++o) {
    const Term& T = plan.terms[P.o0 + o];
    float* base = const_cast<float*>(T.p) + x.batch * T.bstride;
    const float coef = T.coef;
    const int mode = T.mode;
#pragma unroll
    for (int i = 0; i < C::TM / 4; ++i) {
      const int r = x.m0 + x.wm + x.lane_m * 4 + i * 16;
#pragma unroll
      for (int j = 0; j < C::TN; ++j) {
        const int c = x.n0 + x.wn + x.lane_n * 4 + (j / 4) * 32 + (j % 4);
        if (c >= P.n || r >= P.m) continue;
        float* q = base + r + (long long)c * T.ld;
        const float v0 = coef * acc_at<C>(acc, 4 * i + 0, j);
        const float v1 = coef * acc_at<C>(acc, 4 * i + 1, j);
        const float v2 = coef * acc_at<C>(acc, 4 * i + 2, j);
        const float v3 = coef * acc_at<C>(acc, 4 * i + 3, j);
        if (VEC && r + 3 < P.m) {
          float4* q4 = reinterpret_cast<float4*>(q);
          if (mode == kOutAtomic) {
            atomicAdd(q4, make_float4(v0, v1, v2, v3));
          } else if (mode == kOutAdd) {
            float4 old = *q4;
            *q4 = make_float4(old.x + v0, old.y + v1, old.z + v2, old.w + v3);
          } else {
            *q4 = make_float4(v0, v1, v2, v3);
          }
        } else {
          const float vals[4] = {v0, v1, v2, v3};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            if (r + e >= P.m) break;
            if (mode == kOutAtomic) atomicAdd(q + e, vals[e]);
            else if (mode == kOutAdd) q[e] += vals[e];
            else q[e] = vals[e];
          }
        }
      }
    }
  }
}

}  // namespace

template <class C, bool VEC>
__global__ void __launch_bounds__(C::NT, C::MINB)
    leaf_gemm_kernel(const __grid_constant__ LeafPlan plan) {
  __shared__ __align__(16) Smem<C> sm;
  const Prod& P = find_product(plan, blockIdx.x);
  const int local = blockIdx.x - P.tile_begin;
  // Group tiles along M so CTAs resident together share operand panels in L2.
  constexpr int GROUP_M = 8;
  const int in_group = GROUP_M * P.tiles_n;
  const int group = local / in_group;
  const int first_m = group * GROUP_M;
  const int gsize = min(P.tiles_m - first_m, GROUP_M);
  Ctx x;
  x.m0 = (first_m + (local % in_group) % gsize) * C::BM;
  x.n0 = ((local % in_group) / gsize) * C::BN;
  x.batch = blockIdx.y;
  x.tid = threadIdx.x;
  const int lane = x.tid & 31, warp = x.tid >> 5;
  x.lane_m = lane >> 3;
  x.lane_n = lane & 7;
  x.wm = (warp % C::WARPS_M) * C::WM;
  x.wn = (warp / C::WARPS_M) * C::WN;

  Acc<C> acc;
#pragma unroll
  for (int i = 0; i < C::TM / 2; ++i)
#pragma unroll
    for (int j = 0; j < C::TN; ++j) acc[i][j] = make_float2(0.f, 0.f);

  if constexpr (VEC) {
    switch (P.sig) {
      case kSig11: tile_fast<C, 1, 1>(plan, P, x, sm, acc); break;
      case kSig12: tile_fast<C, 1, 2>(plan, P, x, sm, acc); break;
      case kSig21: tile_fast<C, 2, 1>(plan, P, x, sm, acc); break;
      case kSig22: tile_fast<C, 2, 2>(plan, P, x, sm, acc); break;
      case kSig33: tile_fast<C, 3, 3>(plan, P, x, sm, acc); break;
      case kSig41: tile_fast<C, 4, 1>(plan, P, x, sm, acc); break;
      case kSig14: tile_fast<C, 1, 4>(plan, P, x, sm, acc); break;
      default: tile_generic<C, true>(plan, P, x, sm, acc); break;
    }
  } else {
    tile_generic<C, false>(plan, P, x, sm, acc);
  }
  epilogue<C, VEC>(plan, P, x, acc);
}

__global__ void __launch_bounds__(256) materialize_kernel(const __grid_constant__ MatPlan plan) {
  const long long total = plan.chunk_begin[plan.njobs];
  const long long batch = blockIdx.y;
  for (long long q = (long long)blockIdx.x * blockDim.x + threadIdx.x; q < total;
       q += (long long)gridDim.x * blockDim.x) {
    int j = 0;
    while (j + 1 < plan.njobs && plan.chunk_begin[j + 1] <= q) ++j;
    const MatJob& J = plan.job[j];
    const long long local = q - plan.chunk_begin[j];
    const int rows4 = (J.rows + 3) / 4;
    // 32-bit division where the job's chunk index fits (a 64-bit divide per
    // float4 made this pass instruction-bound).
    int c, r;
    if (local <= 0x7fffffffLL) {
      const unsigned l32 = (unsigned)local, d = (unsigned)rows4;
      c = (int)(l32 / d);
      r = (int)(l32 - (unsigned)c * d) * 4;
    } else {
      c = (int)(local / rows4);
      r = (int)(local % rows4) * 4;
    }
    float4 in[kMaxJobInputs];
#pragma unroll
    for (int t = 0; t < kMaxJobInputs; ++t) in[t] = make_float4(0.f, 0.f, 0.f, 0.f);
    bool vec = r + 3 < J.rows;
#pragma unroll
    for (int t = 0; t < kMaxJobInputs; ++t) {
      if (t < J.nin) {
        const float* p = J.in[t].p + batch * J.in[t].bstride + r + (long long)c * J.in[t].ld;
        vec = vec && ((reinterpret_cast<uintptr_t>(p) & 15) == 0);
      }
    }
#pragma unroll
    for (int t = 0; t < kMaxJobInputs; ++t) {
      if (t < J.nin) {
        const float* p = J.in[t].p + batch * J.in[t].bstride + r + (long long)c * J.in[t].ld;
        if (vec) {
          in[t] = ldg4(p);
        } else {
          if (r + 0 < J.rows) in[t].x = p[0];
          if (r + 1 < J.rows) in[t].y = p[1];
          if (r + 2 < J.rows) in[t].z = p[2];
          if (r + 3 < J.rows) in[t].w = p[3];
        }
      }
    }
#pragma unroll
    for (int o = 0; o < kMaxJobOutputs; ++o) {
      if (o < J.nout) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int t = 0; t < kMaxJobInputs; ++t) {
          const int code = J.expr[o][t];
          if (code == 0) break;
          const int src = (code > 0 ? code : -code) - 1;
          // Select without indexing the register array by a runtime value.
          float4 v = in[0];
#pragma unroll
          for (int u = 1; u < kMaxJobInputs; ++u)
            if (src == u) v = in[u];
          acc = accumulate(acc, v, code > 0 ? 1.f : -1.f, t == 0);
        }
        float* p = const_cast<float*>(J.out[o].p) + batch * J.out[o].bstride + r +
                   (long long)c * J.out[o].ld;
        if (vec && (reinterpret_cast<uintptr_t>(p) & 15) == 0) {
          *reinterpret_cast<float4*>(p) = acc;
        } else {
          if (r + 0 < J.rows) p[0] = acc.x;
          if (r + 1 < J.rows) p[1] = acc.y;
          if (r + 2 < J.rows) p[2] = acc.z;
          if (r + 3 < J.rows) p[3] = acc.w;
        }
      }
    }
  }
}

// FP32 FFMA throughput probe: register-only independent fmaf chains, the FP32
// analogue of a STREAM copy for the roofline denominator.  Each thread runs
// kProbeChains chains of `iters` dependent fmaf; the sum is stored so nothing
// is dead code.
constexpr int kProbeChains = 16;

__global__ void __launch_bounds__(256) ffma_probe_kernel(float* sink, int iters, float a, float b) {
  float x[kProbeChains];
#pragma unroll
  for (int c = 0; c < kProbeChains; ++c) x[c] = threadIdx.x * 1e-7f + c * 1e-3f;
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int c = 0; c < kProbeChains; ++c) x[c] = fmaf(x[c], a, b);
  }
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < kProbeChains; ++c) s += x[c];
  sink[blockIdx.x * blockDim.x + threadIdx.x] = s;
}

// ---------------------------------------------------------------------------
// Launchers.
// ---------------------------------------------------------------------------

namespace {

// Measured on B200 (cfg3, 16384^3 depth 2): Tall with scalar FFMA is fastest
// for the register-staged loop; the paired-FMA variants are kept for tuning.
using CfgLarge = Cfg<128, 128, 8, 8, 8, 2, true, false>;    // 256 threads, 2 CTAs per SM
using CfgWide = Cfg<128, 256, 8, 8, 16, 1, true, false>;    // 256 threads, 1 CTA per SM
using CfgSmall = Cfg<64, 64, 8, 8, 8, 4, true, false>;      // 64 threads
using CfgTall = Cfg<256, 128, 8, 16, 8, 1, true, false>;    // 256 threads, 1 CTA per SM
using CfgLarge1 = Cfg<128, 128, 8, 8, 8, 1, true, true>;    // 256 threads, 1 CTA/SM, FFMA2
using CfgHalf = Cfg<128, 64, 8, 8, 8, 2, true, true>;       // 128 threads, 2 CTAs/SM, FFMA2
using CfgTallS = Cfg<256, 128, 8, 16, 8, 1, false, true>;   // Tall, single-buffered, FFMA2
// Tiny problems (cfg1: 7 leaves of 256^3 make 28 tiles of 128 x 128, 112 of
// 64 x 64): 448 CTAs of two warps spread over every SM; each output is still
// one sequential fmaf chain, so the results do not depend on the tile.  16-k
// steps: measured on cfg1 the leaf phase takes 29.5 us with 8-k steps, 25.5
// with 16, 32.3 with 32.
using CfgMicro = Cfg<32, 32, 16, 4, 4, 8, true, false>;     // 64 threads

template <class C>
cudaError_t launch_cfg(const LeafPlan& plan, bool vec, int batch, cudaStream_t stream) {
  const dim3 grid(plan.ntiles, batch);
  if (vec) leaf_gemm_kernel<C, true><<<grid, C::NT, 0, stream>>>(plan);
  else leaf_gemm_kernel<C, false><<<grid, C::NT, 0, stream>>>(plan);
  return cudaGetLastError();
}

}  // namespace

TileShape leaf_tile_shape(int config) {
  switch (config) {
    case kTileSmall: return {CfgSmall::BM, CfgSmall::BN};
    case kTileWide: return {CfgWide::BM, CfgWide::BN};
    case kTileTall: return {CfgTall::BM, CfgTall::BN};
    case kTileLarge1: return {CfgLarge1::BM, CfgLarge1::BN};
    case kTileHalf: return {CfgHalf::BM, CfgHalf::BN};
    case kTileTallS: return {CfgTallS::BM, CfgTallS::BN};
    case kTileMicro: return {CfgMicro::BM, CfgMicro::BN};
    case kTileWS: return ws_tile_shape();
    default: return {CfgLarge::BM, CfgLarge::BN};
  }
}

cudaError_t launch_leaf(const LeafPlan& plan, int config, bool vec, int batch, cudaStream_t stream) {
  if (plan.nprod == 0 || plan.ntiles == 0 || batch == 0) return cudaSuccess;
  switch (config) {
    case kTileSmall: return launch_cfg<CfgSmall>(plan, vec, batch, stream);
    case kTileWide: return launch_cfg<CfgWide>(plan, vec, batch, stream);
    case kTileTall: return launch_cfg<CfgTall>(plan, vec, batch, stream);
    case kTileLarge1: return launch_cfg<CfgLarge1>(plan, vec, batch, stream);
    case kTileHalf: return launch_cfg<CfgHalf>(plan, vec, batch, stream);
    case kTileTallS: return launch_cfg<CfgTallS>(plan, vec, batch, stream);
    case kTileMicro: return launch_cfg<CfgMicro>(plan, vec, batch, stream);
    case kTileWS: return launch_leaf_ws(plan, batch, stream);
    default: return launch_cfg<CfgLarge>(plan, vec, batch, stream);
  }
}

cudaError_t launch_materialize(const MatPlan& plan, int batch, cudaStream_t stream, int sm_count) {
  if (plan.njobs == 0 || batch == 0) return cudaSuccess;
  const long long chunks = plan.chunk_begin[plan.njobs];
  if (chunks == 0) return cudaSuccess;
  long long blocks = (chunks + 255) / 256;
  const long long cap = (long long)sm_count * 8;
  if (blocks > cap) blocks = cap;
  materialize_kernel<<<dim3((unsigned)blocks, batch), 256, 0, stream>>>(plan);
  return cudaGetLastError();
}

cudaError_t launch_ffma_probe(float* sink, int blocks, int iters, cudaStream_t stream,
                              double* flops) {
  ffma_probe_kernel<<<blocks, 256, 0, stream>>>(sink, iters, 0.999999f, 1e-6f);
  *flops = 2.0 * kProbeChains * double(iters) * blocks * 256;
  return cudaGetLastError();
}

}  // namespace bag_b200
