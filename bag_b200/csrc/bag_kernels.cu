// sm_100a kernels of the BAG FP32 matmul.
//
// leaf_gemm_kernel: one launch runs every leaf product of a plan.  Each CTA
//   owns a BM x BN output tile of one product.  Its prologue loads 128-bit
//   column-major vectors of every signed operand term, sums them in FP32 in
//   the reference's evaluation order (x+delta*y, bag.cuh:69-73 /
//   simt.cuh:14-33) and stages the transformed tile into double-buffered
//   shared memory; the main loop is a register-blocked FFMA outer product
//   (TM x TN per thread) with every output a sequential fmaf chain over k;
//   the epilogue adds coef*M into each C block the inverse transform sends the
//   product to (bag.py:530-533 direct decode), with 128-bit red.global adds
//   when products share outputs.
//
// materialize_kernel: elementwise signed sums of up to four blocks into the
//   workspace, for operands the reference rounds before recursing.
#include <cuda_runtime.h>

#include <cstdio>

#include "bag_kernels.h"

namespace bag_b200 {
namespace {

__device__ __forceinline__ const Prod& find_product(const LeafPlan& plan, int item) {
  int pid = 0;
  while (pid + 1 < plan.nprod && plan.prod[pid + 1].tile_begin <= item) ++pid;
  return plan.prod[pid];
}

// Load four consecutive rows (r..r+3) of column c, zero outside [0,rows)x[0,cols).
template <bool VEC>
__device__ __forceinline__ float4 load4(const float* __restrict__ p, int ld, int r, int c, int rows,
                                        int cols) {
  float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
  if (c >= cols) return v;
  const float* q = p + r + (long long)c * ld;
  if (VEC && r + 3 < rows) {
    v = __ldg(reinterpret_cast<const float4*>(q));
  } else {
    if (r + 0 < rows) v.x = __ldg(q + 0);
    if (r + 1 < rows) v.y = __ldg(q + 1);
    if (r + 2 < rows) v.z = __ldg(q + 2);
    if (r + 3 < rows) v.w = __ldg(q + 3);
  }
  return v;
}

// acc (+)= coef * v, rounded once per element: coef is +-1, so the product is
// exact and fmaf gives RN(acc +- v), the reference's x + delta*y.
__device__ __forceinline__ float4 accumulate(float4 acc, float4 v, float coef, bool first) {
  if (first) return make_float4(coef * v.x, coef * v.y, coef * v.z, coef * v.w);
  return make_float4(fmaf(coef, v.x, acc.x), fmaf(coef, v.y, acc.y), fmaf(coef, v.z, acc.z),
                     fmaf(coef, v.w, acc.w));
}

}  // namespace

template <int BM, int BN, int BK, int TM, int TN, int MINB, bool VEC>
__global__ void __launch_bounds__((BM / TM) * (BN / TN), MINB)
    leaf_gemm_kernel(const __grid_constant__ LeafPlan plan) {
  constexpr int NT = (BM / TM) * (BN / TN);
  constexpr int WM = 4 * TM;   // warp tile: 4 x 8 lanes, TM x TN each
  constexpr int WN = 8 * TN;
  constexpr int WARPS_M = BM / WM;
  static_assert((BM / WM) * (BN / WN) * 32 == NT, "warp layout");
  static_assert(TM % 4 == 0 && TN % 4 == 0, "fragments are float4 groups");
  constexpr int A_VECS = BM * BK / 4 / NT;   // float4 per thread per term
  constexpr int B_VECS = BN * BK / 4 / NT;
  static_assert(A_VECS * NT * 4 == BM * BK && B_VECS * NT * 4 == BN * BK, "load split");
  static_assert(BK % 4 == 0 && BK <= 32, "B swizzle assumes BK/4 <= 8");
  constexpr int SWZ = 128 / BK;   // XOR key step per 4-row group of the B tile

  __shared__ __align__(16) float As[2][BK][BM];
  __shared__ __align__(16) float Bs[2][BK][BN];

  const Prod& P = find_product(plan, blockIdx.x);
  const int local = blockIdx.x - P.tile_begin;
  // Group tiles along M so CTAs resident together share operand panels in L2.
  constexpr int GROUP_M = 8;
  const int in_group = GROUP_M * P.tiles_n;
  const int group = local / in_group;
  const int first_m = group * GROUP_M;
  const int gsize = min(P.tiles_m - first_m, GROUP_M);
  const int tile_m = first_m + (local % in_group) % gsize;
  const int tile_n = (local % in_group) / gsize;
  const int m0 = tile_m * BM, n0 = tile_n * BN;
  const long long batch = blockIdx.y;

  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int lane_m = lane >> 3, lane_n = lane & 7;
  const int wm = (warp % WARPS_M) * WM, wn = (warp / WARPS_M) * WN;

  int a_r[A_VECS], a_c[A_VECS], b_k[B_VECS], b_c[B_VECS];
#pragma unroll
  for (int q = 0; q < A_VECS; ++q) {
    const int idx = tid + q * NT;
    a_r[q] = (idx % (BM / 4)) * 4;
    a_c[q] = idx / (BM / 4);
  }
#pragma unroll
  for (int q = 0; q < B_VECS; ++q) {
    const int idx = tid + q * NT;
    b_k[q] = (idx % (BK / 4)) * 4;
    b_c[q] = idx / (BK / 4);
  }

  float4 ra[A_VECS], rb[B_VECS];
  auto load_tile = [&](int k0) {
#pragma unroll
    for (int t = 0; t < kMaxOperandTerms; ++t) {
      if (t < P.nl) {
        const Term& T = plan.terms[P.l0 + t];
        const float* base = T.p + batch * T.bstride;
#pragma unroll
        for (int q = 0; q < A_VECS; ++q)
          ra[q] = accumulate(ra[q], load4<VEC>(base, T.ld, m0 + a_r[q], k0 + a_c[q], P.m, P.k),
                             T.coef, t == 0);
      }
    }
#pragma unroll
    for (int t = 0; t < kMaxOperandTerms; ++t) {
      if (t < P.nr) {
        const Term& T = plan.terms[P.r0 + t];
        const float* base = T.p + batch * T.bstride;
#pragma unroll
        for (int q = 0; q < B_VECS; ++q)
          rb[q] = accumulate(rb[q], load4<VEC>(base, T.ld, k0 + b_k[q], n0 + b_c[q], P.k, P.n),
                             T.coef, t == 0);
      }
    }
  };
  auto store_tile = [&](int s) {
#pragma unroll
    for (int q = 0; q < A_VECS; ++q) *reinterpret_cast<float4*>(&As[s][a_c[q]][a_r[q]]) = ra[q];
#pragma unroll
    for (int q = 0; q < B_VECS; ++q) {
      // The K-contiguous B vector is transposed into four rows; XOR-swizzling
      // the column by the 4-row group keeps one warp's stores on 32 banks.
      const int col = b_c[q] ^ ((b_k[q] >> 2) * SWZ);
      Bs[s][b_k[q] + 0][col] = rb[q].x;
      Bs[s][b_k[q] + 1][col] = rb[q].y;
      Bs[s][b_k[q] + 2][col] = rb[q].z;
      Bs[s][b_k[q] + 3][col] = rb[q].w;
    }
  };

  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;

  const int ktiles = (P.k + BK - 1) / BK;
  if (ktiles > 0) {
    load_tile(0);
    store_tile(0);
    __syncthreads();
  }
  for (int kt = 0; kt < ktiles; ++kt) {
    const int s = kt & 1;
    if (kt + 1 < ktiles) load_tile((kt + 1) * BK);
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[TM], b[TN];
#pragma unroll
      for (int i = 0; i < TM / 4; ++i)
        *reinterpret_cast<float4*>(&a[4 * i]) =
            *reinterpret_cast<const float4*>(&As[s][kk][wm + lane_m * 4 + i * 16]);
#pragma unroll
      for (int j = 0; j < TN / 4; ++j)
        *reinterpret_cast<float4*>(&b[4 * j]) = *reinterpret_cast<const float4*>(
            &Bs[s][kk][(wn + lane_n * 4 + j * 32) ^ ((kk >> 2) * SWZ)]);
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    if (kt + 1 < ktiles) store_tile(s ^ 1);
    __syncthreads();
  }

  // Epilogue: inverse transform as signed updates of every target block.
  for (int o = 0; o < P.no; ++o) {
    const Term& T = plan.terms[P.o0 + o];
    float* base = const_cast<float*>(T.p) + batch * T.bstride;
    const float coef = T.coef;
    const int mode = T.mode;
#pragma unroll
    for (int i = 0; i < TM / 4; ++i) {
      const int r = m0 + wm + lane_m * 4 + i * 16;
#pragma unroll
      for (int j = 0; j < TN; ++j) {
        const int c = n0 + wn + lane_n * 4 + (j / 4) * 32 + (j % 4);
        if (c >= P.n || r >= P.m) continue;
        float* q = base + r + (long long)c * T.ld;
        const float v0 = coef * acc[4 * i + 0][j], v1 = coef * acc[4 * i + 1][j];
        const float v2 = coef * acc[4 * i + 2][j], v3 = coef * acc[4 * i + 3][j];
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
    const int c = (int)(local / rows4);
    const int r = (int)(local % rows4) * 4;
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
          in[t] = __ldg(reinterpret_cast<const float4*>(p));
        } else {
          in[t] = make_float4(0.f, 0.f, 0.f, 0.f);
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
// kChains chains of `iters` dependent fmaf; the sum is stored so nothing is
// dead code.
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

cudaError_t launch_ffma_probe(float* sink, int blocks, int iters, cudaStream_t stream,
                              double* flops) {
  ffma_probe_kernel<<<blocks, 256, 0, stream>>>(sink, iters, 0.999999f, 1e-6f);
  *flops = 2.0 * kProbeChains * double(iters) * blocks * 256;
  return cudaGetLastError();
}

namespace {

template <int BM, int BN, int BK, int TM, int TN, int MINB, bool VEC>
cudaError_t launch_leaf_cfg(const LeafPlan& plan, int batch, cudaStream_t stream) {
  constexpr int NT = (BM / TM) * (BN / TN);
  auto kernel = leaf_gemm_kernel<BM, BN, BK, TM, TN, MINB, VEC>;
  kernel<<<dim3(plan.ntiles, batch), NT, 0, stream>>>(plan);
  return cudaGetLastError();
}

}  // namespace

TileShape leaf_tile_shape(int config) {
  switch (config) {
    case kTileSmall: return {64, 64};
    default: return {128, 128};
  }
}

cudaError_t launch_leaf(const LeafPlan& plan, int config, bool vec, int batch, cudaStream_t stream) {
  if (plan.nprod == 0 || plan.ntiles == 0 || batch == 0) return cudaSuccess;
  switch (config) {
    case kTileSmall:
      return vec ? launch_leaf_cfg<64, 64, 8, 8, 8, 4, true>(plan, batch, stream)
                 : launch_leaf_cfg<64, 64, 8, 8, 8, 4, false>(plan, batch, stream);
    default:
      return vec ? launch_leaf_cfg<128, 128, 8, 8, 8, 2, true>(plan, batch, stream)
                 : launch_leaf_cfg<128, 128, 8, 8, 8, 2, false>(plan, batch, stream);
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

}  // namespace bag_b200
