// C-ABI harness around the reference's own header-only CUDA library -- TEST
// INFRASTRUCTURE ONLY (the checker and the measured comparator, never the
// product).
//
// Compiled by oracle/build_ref.py against the reference checkout's
// include/ directory, so the code that runs is the reference's, unmodified:
// bag_cuda::matmul (include/bag/cuda/bag.cuh:247-260) and
// strassen_cuda::one_level (include/bag/cuda/strassen.cuh:225-276).  The
// resulting oracle/_ref/libbagref.so is git-ignored and travels to the GPU
// box; nothing here reads the reference at run time.
#include <bag/cuda/bag.cuh>

#include <map>
#include <memory>
#include <string>
#include <tuple>

namespace {
thread_local std::string g_error;
std::map<std::tuple<int, int, int>, std::unique_ptr<bag_cuda::Workspace>> g_workspaces;
std::unique_ptr<strassen_cuda::Workspace> g_workers;

template <class F>
int guarded(F&& f) {
  try {
    f();
    return 0;
  } catch (const std::exception& e) {
    g_error = e.what();
    return 1;
  }
}
}  // namespace

extern "C" {

const char* ref_last_error(void) { return g_error.c_str(); }

// Allocate (once) the reference workspace for (n, depth, basis); returns bytes.
long long ref_workspace_bytes(int n, int depth, int basis) {
  long long bytes = -1;
  guarded([&] {
    auto key = std::make_tuple(n, depth, basis);
    auto& ws = g_workspaces[key];
    if (!ws)
      ws = std::make_unique<bag_cuda::Workspace>(
          n, depth, basis ? bag_cuda::Basis::Full : bag_cuda::Basis::Minimal);
    bytes = (long long)ws->bytes();
  });
  return bytes;
}

// C <- A B + C, column-major n x n, the reference's BAG.
// backend: 0 = ColumnTile8 (the default), 1 = Huge; schedule: bag.cuh:8 order.
int ref_bag_matmul(const float* a, const float* b, float* c, int n, int depth, int basis,
                   int schedule, int backend, void* stream) {
  return guarded([&] {
    if (ref_workspace_bytes(n, depth, basis) < 0) throw std::runtime_error(g_error);
    auto& ws = *g_workspaces[std::make_tuple(n, depth, basis)];
    const auto be = backend ? bag_cuda::Backend::Huge : bag_cuda::Backend::ColumnTile8;
    const auto sc = schedule == 0   ? bag_cuda::Schedule::Serial
                    : schedule == 1 ? bag_cuda::Schedule::SevenStream
                                    : bag_cuda::Schedule::Batched;
    bag_cuda::matmul(a, b, c, n, static_cast<cudaStream_t>(stream), ws, be, sc);
  });
}

// Classic Strassen one level, FourBatchedAtomic on ColumnTile8 (the schedule
// the reference benchmark times, benchmarks/cuda/bag.cu:79-81).
int ref_strassen_one_level(const float* a, const float* b, float* c, int n, void* stream) {
  return guarded([&] {
    if (!g_workers) g_workers = std::make_unique<strassen_cuda::Workspace>();
    strassen_cuda::one_level(strassen_cuda::Backend::ColumnTile8,
                             strassen_cuda::Schedule::FourBatchedAtomic, a, b, c, n,
                             static_cast<cudaStream_t>(stream), *g_workers);
  });
}

void ref_release(void) {
  g_workspaces.clear();
  g_workers.reset();
}

}  // extern "C"
