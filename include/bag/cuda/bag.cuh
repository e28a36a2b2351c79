// Drop-in replacement for the reference's include/bag/cuda/bag.cuh
// (liuyao0322/bag): bag_cuda::Basis, Schedule, Backend, Operand, DeviceBuffer,
// local_elements, Workspace and matmul keep their names, signatures, defaults
// and error behaviour; the work runs on the B200 kernels of libbag_b200.so
// through the C ABI (include/bag_capi.h).
//
// Semantics kept (bag.cuh:247-248): C <- AB + C for distinct column-major
// N x N matrices, everything enqueued on the caller stream, no allocation, no
// host synchronisation and no cuBLAS call inside matmul.  Workspaces are not
// reentrant and must outlive the work enqueued with them.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <stdexcept>

#include "../../bag_capi.h"
#include "strassen.cuh"

namespace bag_cuda {

enum class Basis { Minimal, Full };
enum class Schedule { Serial, SevenStream, Batched };
using Backend = strassen_cuda::Backend;
using Operand = strassen_cuda::Operand;

// RAII device buffer of `count` floats.
struct DeviceBuffer {
  float* p = nullptr;
  size_t count;
  explicit DeviceBuffer(size_t elements) : count(elements) {
    if (count) strassen_cuda::checked(cudaMalloc(&p, count * sizeof(float)));
  }
  ~DeviceBuffer() {
    if (p) cudaFree(p);
  }
  DeviceBuffer(const DeviceBuffer&) = delete;
  DeviceBuffer& operator=(const DeviceBuffer&) = delete;
};

// Elements of the reference's workspace for (n, depth, basis); throws when
// depth < 1 or a level's size is not a multiple of 8.
inline size_t local_elements(int n, int depth, Basis basis) {
  size_t elements = 0;
  strassen_cuda::detail::check(bag_local_elements(n, depth, static_cast<int>(basis), &elements));
  return elements;
}

// Device workspace for one size, depth and basis.  This build rounds only the
// operands the recursion splits (and the Full basis's transformed quadrants),
// so it is smaller than the reference's and empty for Minimal at depth 1;
// output(), left() and right() all return its base (nullptr when empty).
struct Workspace {
  const int n, depth;
  const Basis basis;
  explicit Workspace(int size, int levels = 1, Basis layout = Basis::Minimal)
      : n(size), depth(levels), basis(layout) {
    strassen_cuda::detail::check(
        bag_workspace_create(size, levels, static_cast<int>(layout), &handle_));
  }
  ~Workspace() { bag_workspace_destroy(handle_); }
  float* output() const { return bag_workspace_data(handle_); }
  float* left() const { return bag_workspace_data(handle_); }
  float* right() const { return bag_workspace_data(handle_); }
  size_t bytes() const { return bag_workspace_bytes(handle_); }
  bag_workspace* handle() const { return handle_; }
  Workspace(const Workspace&) = delete;
  Workspace& operator=(const Workspace&) = delete;

 private:
  bag_workspace* handle_ = nullptr;
};

// Enqueue C <- AB + C.  A/B/C are distinct column-major N x N FP32 matrices.
//
// Leaf arithmetic: the reference's sequential-fmaf FP32 SIMT numerics by
// default.  A thread that calls bag_set_math_mode(BAG_MATH_3XTF32) before it
// creates the Workspace gets the tcgen05 3xTF32 leaves on prepared TF32
// operands, the fast path (the workspace then also holds those operands:
// bag_workspace_bytes_for(BAG_MATH_3XTF32, ...) gives its size up front).  A
// Workspace created in FFMA mode and used from a 3XTF32 thread runs the
// tensor leaves with the transforms fused into their prologue, a slower path.
// bag_last_leaf_kernel() reports which leaf kernel the last call on the
// thread ran (BAG_LEAF_KERNEL_FFMA / _TF32_FUSED / _TF32_SINGLE / _TF32_PAIR).
inline void matmul(const float* a, const float* b, float* c, int n, cudaStream_t caller,
                   Workspace& ws, Backend backend = Backend::ColumnTile8,
                   Schedule schedule = Schedule::Batched) {
  strassen_cuda::detail::check(bag_matmul(a, b, c, n, strassen_cuda::detail::stream(caller),
                                          ws.handle(), static_cast<int>(backend),
                                          static_cast<int>(schedule)));
}

}  // namespace bag_cuda
