// bag_sgemm_noalloc: the BAG matmul for callers that cannot allocate device
// memory.
//
// Some callers of this library may not call cudaMalloc: a host application or
// plugin framework that owns every byte of device memory (a serving process
// with a fixed memory pool, an embedding engine whose allocator must account
// for all allocations) cannot let a library allocate on its own, and a caller
// in a latency-critical loop cannot afford an allocation that may synchronise
// the device.  Depth >= 2 (and Full-basis) plans need scratch memory for the
// operands the recursion rounds before splitting; bag_sgemm_ex takes that
// scratch from a workspace the caller creates up front, which such callers
// cannot do.  This entry point instead uses one file-scope device array of
// fixed size (kNoAllocScratchFloats floats = 16 MiB), which every GPU that
// loads this library holds until the process exits.
//
// Rules of use:
//  * The first call on each device looks up the array's device address
//    (cudaGetSymbolAddress, with that device current).  Make that first call
//    before any stream capture on the device.
//  * All calls share the one array and it keeps the previous call's contents.
//    Nothing in it needs to start at zero: every plan writes each scratch
//    block completely before any kernel reads it.  Calls that can overlap on
//    the GPU (different streams, or different host threads) race on the array
//    and must be serialised by the caller.
//  * Problems whose plan needs more scratch than the array holds are
//    rejected with BAG_ERR_WORKSPACE before anything is enqueued.
//  * Nothing here calls cudaMalloc, cudaFree or an allocating library
//    routine.
#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <string>

#include "../../include/bag_capi.h"

namespace bag_b200 {

bag_status sgemm_with_scratch(int layout, int m, int n, int k, const float* a, long long lda,
                              const float* b, long long ldb, float* c, long long ldc, float beta,
                              int depth, int basis, cudaStream_t stream, float* scratch,
                              size_t scratch_elements);
void set_last_error(const std::string& message);

namespace {

constexpr size_t kNoAllocScratchFloats = size_t(4) << 20;   // 16 MiB per device

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

// Device address of the scratch array on the current device (looked up once
// per device).  Returns nullptr and sets bag_last_error() on failure.
float* scratch_on_current_device() {
  static std::mutex mu;
  static std::map<int, float*> addresses;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_last_error(std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  auto it = addresses.find(dev);
  if (it != addresses.end()) return it->second;
  float* ptr = nullptr;
  e = cudaGetSymbolAddress(reinterpret_cast<void**>(&ptr), g_noalloc_scratch);
  if (e != cudaSuccess || ptr == nullptr) {
    set_last_error(std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
    return nullptr;
  }
  addresses[dev] = ptr;
  return ptr;
}

}  // namespace
}  // namespace bag_b200

extern "C" bag_status bag_sgemm_noalloc(int layout, int m, int n, int k, const float* a,
                                        long long lda, const float* b, long long ldb, float* c,
                                        long long ldc, float beta, int depth, int basis,
                                        bag_stream_t stream) {
  float* scratch = bag_b200::scratch_on_current_device();
  if (scratch == nullptr) return BAG_ERR_CUDA;
  return bag_b200::sgemm_with_scratch(layout, m, n, k, a, lda, b, ldb, c, ldc, beta, depth, basis,
                                      reinterpret_cast<cudaStream_t>(stream), scratch,
                                      bag_b200::kNoAllocScratchFloats);
}
