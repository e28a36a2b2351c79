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
//  * Every call looks up the array's device address on the current device
//    (cudaGetSymbolAddress, with that device current; cheap once the module is
//    loaded), so a context that was reset and re-created gets the array's new
//    address.  The first call on a device may load this library's device code
//    there; make that first call before any stream capture on the device.
//  * All calls share the one array and it keeps the previous call's contents.
//    Nothing in it needs to start at zero: every plan writes each scratch
//    block completely before any kernel reads it.  Calls that can overlap on
//    the GPU (different streams, or different host threads) race on the array
//    and must be serialised by the caller.
//  * Problems whose plan needs more scratch than the array holds are
//    rejected with BAG_ERR_WORKSPACE before anything is enqueued.  In 3xTF32
//    mode a plan whose prepared TF32 operands fit in the array uses them;
//    otherwise its leaves run the tensor kernel with the transforms fused in.
//  * Nothing here calls cudaMalloc, cudaFree or an allocating library
//    routine.
#include <cuda_runtime.h>

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

// Device address of the scratch array on the current device, looked up on
// every call.  Returns nullptr and sets bag_last_error() on failure.
float* scratch_on_current_device() {
  float* ptr = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&ptr), g_noalloc_scratch);
  if (e != cudaSuccess || ptr == nullptr) {
    set_last_error(std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
    return nullptr;
  }
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
