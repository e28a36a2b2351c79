// Drop-in replacement for the reference's include/bag/cuda/strassen.cuh
// (liuyao0322/bag): the same namespace, types and function signatures, so code
// written against bag::cuda compiles unchanged, with every call forwarded to
// the B200 kernels of libbag_b200.so through the C ABI (include/bag_capi.h).
//
// Backend: all 42 names of the reference (strassen.cuh:11-55) are kept and all
// run this library's single kernel family; valid_shape keeps each backend's
// tile constraint (strassen.cuh:57-66) and the atomic-only backends keep their
// errors (strassen.cuh:72-88).  Schedule: every schedule is one grouped launch
// on the caller stream (the worker streams of Workspace stay available to
// callers that use them directly).
#pragma once

#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

#include "../../bag_capi.h"

// Pointers of two products sharing coefficients (legacy/base_components.cuh:10-23).
struct PrimBatchedPairArgs {
  const float* X0;
  const float* Y0;
  const float* V0;
  const float* W0;
  float* D0;
  float* E0;
  const float* X1;
  const float* Y1;
  const float* V1;
  const float* W1;
  float* D1;
  float* E1;
};

namespace strassen_cuda {

enum class Backend {
  Legacy, Large, Medium, Huge, Sync64, Pipe64, Pipe64K16, Pipe64R4, Pipe64x32, Pipe128x64,
  Pipe128, Swizzle64, Swizzle64x32, Swizzle32x64, Coalesced64, SwizzleCoalesced64, BalancedK8R8,
  BalancedK16R8, BalancedK8R4, BalancedK32R4, Exact64, ExactSwizzle64, Deferred64,
  DeferredSwizzle64, Sliced1, Sliced2, Sliced4, Striped1, Striped2, Striped4, CgExact64,
  CgDeferred64, ReadonlyDeferred64, StripedTile64, StripedTile128x64, StripedTile64x128,
  RegisterStage4, ColumnTile8, RegisterStage8, ColumnK8, ColumnImmediate, ColumnMin5
};

struct NamedBackend {
  const char* name;
  Backend backend;
  bool normal;          // accepts non-atomic ("normal") schedules
  bool paired = false;  // accepts the paired / batched schedules
};

// Command-line names of the backends, in enum order.
inline const NamedBackend backends[] = {
    {"legacy", Backend::Legacy, false}, {"large", Backend::Large, true},
    {"medium", Backend::Medium, false}, {"huge", Backend::Huge, false, true},
    {"sync64_k8_r8", Backend::Sync64, true}, {"pipe64_k8_r8", Backend::Pipe64, true},
    {"pipe64_k16_r8", Backend::Pipe64K16, true}, {"pipe64_k16_r4", Backend::Pipe64R4, true},
    {"pipe64x32_k16_r4", Backend::Pipe64x32, true, true},
    {"pipe128x64_k16_r8x4", Backend::Pipe128x64, true}, {"pipe128_k16_r8", Backend::Pipe128, true},
    {"swizzle64_k16_r4", Backend::Swizzle64, true},
    {"swizzle64x32_k16_r4", Backend::Swizzle64x32, true},
    {"swizzle32x64_k16_r4", Backend::Swizzle32x64, true},
    {"coalesced64_k16_r4", Backend::Coalesced64, true},
    {"swizzle_coalesced64_k16_r4", Backend::SwizzleCoalesced64, true},
    {"swizzle64_k8_r8x4", Backend::BalancedK8R8, true},
    {"swizzle64_k16_r8x4", Backend::BalancedK16R8, true},
    {"swizzle_coalesced64_k8_r4", Backend::BalancedK8R4, true},
    {"swizzle_coalesced64_k32_r4", Backend::BalancedK32R4, true},
    {"exact_coalesced64_k16_r4", Backend::Exact64, true},
    {"exact_swizzle_coalesced64_k16_r4", Backend::ExactSwizzle64, true},
    {"deferred_exact_coalesced64_k16_r4", Backend::Deferred64, true},
    {"deferred_exact_swizzle_coalesced64_k16_r4", Backend::DeferredSwizzle64, true, true},
    {"sliced1_64x32_k8_r8x4", Backend::Sliced1, true},
    {"sliced2_64x32_k8_r8x4", Backend::Sliced2, true},
    {"sliced4_64x32_k8_r8x4", Backend::Sliced4, true},
    {"striped_sliced1_64x32_k8_r8x4", Backend::Striped1, true},
    {"striped_sliced2_64x32_k8_r8x4", Backend::Striped2, true},
    {"striped_sliced4_64x32_k8_r8x4", Backend::Striped4, true},
    {"cg_exact_swizzle_coalesced64_k16_r4", Backend::CgExact64, true},
    {"cg_deferred_exact_swizzle_coalesced64_k16_r4", Backend::CgDeferred64, true},
    {"ldg_deferred_exact_swizzle_coalesced64_k16_r4", Backend::ReadonlyDeferred64, true},
    {"striped_tile64_k16_r8x4", Backend::StripedTile64, true},
    {"striped_tile128x64_k16_r8x4", Backend::StripedTile128x64, true},
    {"striped_tile64x128_k16_r8x4", Backend::StripedTile64x128, true},
    {"register_stage64_k16_r4x4", Backend::RegisterStage4, true},
    {"column_tile64_k16_r4x8", Backend::ColumnTile8, true, true},
    {"register_stage64_k16_r4x8", Backend::RegisterStage8, true},
    {"column_tile64_k8_r4x8", Backend::ColumnK8, true},
    {"column_immediate64_k16_r4x8", Backend::ColumnImmediate, true},
    {"column_min5_64_k16_r4x8", Backend::ColumnMin5, true}};

namespace detail {
inline void check(bag_status status) {
  if (status != BAG_OK) throw std::runtime_error(bag_last_error());
}
inline bag_stream_t stream(cudaStream_t s) { return reinterpret_cast<bag_stream_t>(s); }
}  // namespace detail

inline void checked(cudaError_t status) {
  if (status != cudaSuccess) throw std::runtime_error(cudaGetErrorString(status));
}

inline bool valid_shape(Backend backend, int s) {
  int valid = 0;
  detail::check(bag_valid_shape(static_cast<int>(backend), s, &valid));
  return valid != 0;
}

// d (+)= GD*(x + D*y)(v + E*w), e (+)= GE*(...); square s x s blocks with a
// common leading dimension ld, column-major.
template <int D, int E, int GD, int GE, bool Atomic>
void primitive(Backend backend, const float* x, const float* y, const float* v, const float* w,
               float* d, float* e, int s, int ld, cudaStream_t stream) {
  static_assert(D >= -1 && D <= 1 && E >= -1 && E <= 1, "operand coefficients are -1, 0 or 1");
  static_assert(GD >= -2 && GD <= 2 && GE >= -2 && GE <= 2, "output codes are -2..2");
  if (!Atomic && backend == Backend::Legacy)
    throw std::runtime_error("legacy backend requires atomic updates");
  if (!Atomic && backend == Backend::Medium)
    throw std::runtime_error("medium backend requires atomic updates");
  if (!Atomic && backend == Backend::Huge)
    throw std::runtime_error("huge backend requires atomic updates");
  detail::check(bag_primitive(D, E, GD, GE, Atomic ? 1 : 0, x, y, v, w, d, e, s, s, s, ld, ld, ld,
                              ld, ld, ld, detail::stream(stream)));
}

struct Operand {
  const float *x, *y, *v, *w;
  float *d, *e;
};

// Operands of classic Strassen-1969 product i (quadrant offsets of a
// column-major n x n matrix: +s is X21, +col is X12, +diag is X22).
inline Operand operands(int i, const float* a, const float* b, float* c, int n) {
  const int s = n / 2;
  const size_t col = size_t(s) * n, diag = col + s;
  switch (i) {
    case 0: return {a + s, a + diag, b, b, c + s, c + diag};
    case 1: return {a, a + col, b + diag, b + diag, c + col, c};
    case 2: return {a + s, a, b, b + col, c + diag, c + diag};
    case 3: return {a + col, a + diag, b + s, b + diag, c, c};
    case 4: return {a, a, b + col, b + diag, c + col, c + diag};
    case 5: return {a + diag, a + diag, b + s, b, c, c + s};
    default: return {a, a + diag, b, b + diag, c, c + diag};
  }
}

template <bool Atomic>
void product(int i, Backend backend, const float* a, const float* b, float* c, int n,
             cudaStream_t stream) {
  const Operand p = operands(i, a, b, c, n);
  const int s = n / 2;
  switch (i) {
    case 0:
    case 1: primitive<1, 0, 1, -1, Atomic>(backend, p.x, p.y, p.v, p.w, p.d, p.e, s, n, stream); break;
    case 2: primitive<-1, 1, 0, 1, Atomic>(backend, p.x, p.y, p.v, p.w, p.d, p.e, s, n, stream); break;
    case 3: primitive<-1, 1, 1, 0, Atomic>(backend, p.x, p.y, p.v, p.w, p.d, p.e, s, n, stream); break;
    case 4:
    case 5: primitive<0, -1, 1, 1, Atomic>(backend, p.x, p.y, p.v, p.w, p.d, p.e, s, n, stream); break;
    default: primitive<1, 1, 1, 1, Atomic>(backend, p.x, p.y, p.v, p.w, p.d, p.e, s, n, stream); break;
  }
}

// Worker streams and events, as the reference's Workspace provides them.
struct Workspace {
  cudaStream_t streams[7];
  cudaEvent_t start, stage, done[7];
  Workspace() {
    checked(cudaEventCreateWithFlags(&start, cudaEventDisableTiming));
    checked(cudaEventCreateWithFlags(&stage, cudaEventDisableTiming));
    for (int i = 0; i < 7; ++i) {
      checked(cudaStreamCreateWithFlags(&streams[i], cudaStreamNonBlocking));
      checked(cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming));
    }
  }
  ~Workspace() {
    for (int i = 0; i < 7; ++i) {
      cudaStreamDestroy(streams[i]);
      cudaEventDestroy(done[i]);
    }
    cudaEventDestroy(start);
    cudaEventDestroy(stage);
  }
  Workspace(const Workspace&) = delete;
  Workspace& operator=(const Workspace&) = delete;
};

enum class Schedule {
  SerialAtomic, SerialNormal, SevenAtomic, DependencyNormal, PairedAtomic, PairedNormal,
  FourBatchedAtomic
};

// Two products with shared coefficients in one launch.
template <int D, int E, int GD, int GE, bool Atomic>
void pair(Backend backend, Operand a, Operand b, int s, int ld, cudaStream_t stream) {
  if (backend != Backend::Huge && backend != Backend::Pipe64x32 &&
      backend != Backend::ColumnTile8 && backend != Backend::DeferredSwizzle64)
    throw std::runtime_error("backend has no paired implementation");
  if (!Atomic && backend == Backend::Huge)
    throw std::runtime_error("huge pairs require atomic updates");
  const float* ops[8] = {a.x, a.y, a.v, a.w, b.x, b.y, b.v, b.w};
  float* outs[4] = {a.d, a.e, b.d, b.e};
  detail::check(bag_primitive_pair(D, E, GD, GE, Atomic ? 1 : 0, ops, outs, s, ld,
                                   detail::stream(stream)));
}

template <bool Atomic>
void paired_level(Backend backend, const float* a, const float* b, float* c, int n,
                  cudaStream_t stream) {
  const int s = n / 2;
  pair<1, 0, 1, -1, Atomic>(backend, operands(0, a, b, c, n), operands(1, a, b, c, n), s, n, stream);
  Operand p2 = operands(2, a, b, c, n);
  p2.d = p2.e;   // M3's single output moves to D to share M4's coefficients
  pair<-1, 1, 1, 0, Atomic>(backend, p2, operands(3, a, b, c, n), s, n, stream);
  pair<0, -1, 1, 1, Atomic>(backend, operands(4, a, b, c, n), operands(5, a, b, c, n), s, n, stream);
  product<Atomic>(6, backend, a, b, c, n, stream);
}

inline void batched_variant(int variant, Backend backend, const float* a, const float* b, float* c,
                            int n, cudaStream_t stream) {
  const int s = n / 2;
  switch (variant) {
    case 0: pair<1, 0, 1, -1, true>(backend, operands(0, a, b, c, n), operands(1, a, b, c, n), s, n, stream); break;
    case 1: {
      Operand p = operands(2, a, b, c, n);
      p.d = p.e;
      pair<-1, 1, 1, 0, true>(backend, p, operands(3, a, b, c, n), s, n, stream);
      break;
    }
    case 2: pair<0, -1, 1, 1, true>(backend, operands(4, a, b, c, n), operands(5, a, b, c, n), s, n, stream); break;
    default: product<true>(6, backend, a, b, c, n, stream); break;
  }
}

// C <- AB + C by one level of classic Strassen; column-major n x n.
inline void one_level(Backend backend, Schedule schedule, const float* a, const float* b, float* c,
                      int n, cudaStream_t caller, Workspace& workspace) {
  (void)workspace;
  detail::check(bag_strassen_one_level(static_cast<int>(backend), static_cast<int>(schedule), a,
                                       b, c, n, detail::stream(caller)));
}

}  // namespace strassen_cuda
