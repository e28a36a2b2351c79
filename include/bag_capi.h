/*
 * bag_capi.h -- C ABI of the B200-native BAG FP32 matrix multiply.
 *
 * Plain pointers, sizes and status codes; no C++ or torch types.  Every entry
 * point is asynchronous on the given stream, allocates nothing (workspaces are
 * created up front) and never throws: failures return a status and leave a
 * message in bag_last_error() (thread-local).
 *
 * Reference interfaces replaced (liuyao0322/bag, path:line):
 *   bag_workspace_create/_destroy/_bytes  bag_cuda::Workspace, include/bag/cuda/bag.cuh:34-55
 *   bag_workspace_bytes_for               bag_cuda::Workspace::bytes, bag.cuh:52 (sizing before creation)
 *   bag_local_elements                    bag_cuda::local_elements, bag.cuh:23-30
 *   bag_matmul                            bag_cuda::matmul, bag.cuh:247-260
 *   bag_valid_shape                       strassen_cuda::valid_shape, include/bag/cuda/strassen.cuh:57-66
 *   bag_primitive                         strassen_cuda::primitive, strassen.cuh:68-70 (CUDA) and
 *                                         bag_primitive, src/bag_triton/primitive.py:256-272 (gamma +-2)
 *   bag_primitive_pair                    strassen_cuda::pair, strassen.cuh:167-197
 *   bag_strassen_one_level                strassen_cuda::one_level, strassen.cuh:223-276
 *   bag_sgemm_ex / bag_sgemm_batched      new: rectangular, ragged, row-major and batched problems
 *                                         (BASELINE configs 4 and 5); no reference counterpart
 *   bag_plan_dump                         new: the host plan as JSON, for tests of the plan builder
 *   bag_sgemm_multi                       new: one process, several GPUs (row/column-band shards)
 */
#ifndef BAG_CAPI_H
#define BAG_CAPI_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same type as cudaStream_t; 0 is the legacy default stream. */
typedef struct CUstream_st* bag_stream_t;
typedef struct bag_workspace bag_workspace;

typedef enum bag_status {
  BAG_OK = 0,
  BAG_ERR_INVALID = 1,     /* bad argument (null pointer, bad enum, bad coefficient) */
  BAG_ERR_SHAPE = 2,       /* shape the algorithm or backend cannot take */
  BAG_ERR_WORKSPACE = 3,   /* workspace missing, too small or for another shape */
  BAG_ERR_UNSUPPORTED = 4, /* valid request this build does not implement */
  BAG_ERR_CUDA = 5,        /* a CUDA runtime call failed */
  BAG_ERR_INTERNAL = 6
} bag_status;

/* Basis descriptors, bag.cuh:7 (Minimal, Full); CLASSIC is Strassen-1969
 * (strassen.cuh:131-153) run through the same recursion; WINOGRAD is the
 * 15-addition Strassen-Winograd variant (new; no reference counterpart). */
enum { BAG_BASIS_MINIMAL = 0, BAG_BASIS_FULL = 1, BAG_BASIS_CLASSIC = 2, BAG_BASIS_WINOGRAD = 3 };
/* bag_cuda::Schedule, bag.cuh:8.  Every schedule runs as one grouped launch on
 * the caller stream here; the value is validated and otherwise a hint. */
enum { BAG_SCHEDULE_SERIAL = 0, BAG_SCHEDULE_SEVEN_STREAM = 1, BAG_SCHEDULE_BATCHED = 2 };
/* strassen_cuda::Schedule, strassen.cuh:165. */
enum {
  BAG_STRASSEN_SERIAL_ATOMIC = 0, BAG_STRASSEN_SERIAL_NORMAL = 1, BAG_STRASSEN_SEVEN_ATOMIC = 2,
  BAG_STRASSEN_DEPENDENCY_NORMAL = 3, BAG_STRASSEN_PAIRED_ATOMIC = 4,
  BAG_STRASSEN_PAIRED_NORMAL = 5, BAG_STRASSEN_FOUR_BATCHED_ATOMIC = 6
};
enum { BAG_LAYOUT_COL_MAJOR = 0, BAG_LAYOUT_ROW_MAJOR = 1 };
/* `depth` of bag_sgemm_ex / _batched / _noalloc, bag_workspace_create_ex and
 * bag_plan_dump: choose the recursion depth from the shape and the calling
 * thread's math mode (3XTF32: none below 4096, at least one level from 4096,
 * more while the leaves stay >= 4096; FFMA: depth 3 from 16384, 2 from 2048,
 * 1 from 1024).  New; the reference takes explicit levels. */
enum { BAG_DEPTH_AUTO = -1 };
/* Leaf arithmetic (bag_set_math_mode).  FFMA: every output a sequential fmaf
 * chain, the reference's SIMT numerics.  3XTF32: tcgen05 tensor cores on
 * hi/lo TF32 splits (hi*hi + hi*lo + lo*hi) with 32- or 64-long K chunks summed in
 * FP32 -- error below an FP32 FFMA dot product's for K >= 1024; used where
 * bag_last_leaf_path says, FFMA elsewhere. */
enum { BAG_MATH_FFMA = 0, BAG_MATH_3XTF32 = 1 };
/* Backend ids are the positions of strassen_cuda::Backend (strassen.cuh:11-16);
 * every id runs this library's kernel, valid_shape keeps its constraints. */
enum { BAG_BACKEND_LEGACY = 0, BAG_BACKEND_LARGE = 1, BAG_BACKEND_MEDIUM = 2, BAG_BACKEND_HUGE = 3,
       BAG_BACKEND_PIPE64X32 = 8, BAG_BACKEND_DEFERRED_SWIZZLE64 = 23,
       BAG_BACKEND_COLUMN_TILE8 = 37, BAG_BACKEND_COUNT = 42 };

const char* bag_last_error(void);
const char* bag_version(void);

/* Elements the reference's workspace holds (bag.cuh:23-30): throws there, returns
 * 0 and sets BAG_ERR_SHAPE here when depth < 1 or a level's size is not a multiple of 8. */
bag_status bag_local_elements(int n, int depth, int basis, size_t* elements);

/* Workspace for square n x n products at `depth` levels (bag.cuh:40-44). */
bag_status bag_workspace_create(int n, int depth, int basis, bag_workspace** out);
/* Workspace for C(m x n) += A(m x k) B(k x n), `batch` problems at once. */
bag_status bag_workspace_create_ex(int m, int n, int k, int depth, int basis, int batch,
                                   bag_workspace** out);
/* Bytes bag_workspace_create_ex would allocate for this problem when called
 * on a thread in math mode `mode` (BAG_MATH_*): in 3XTF32 mode, when every
 * leaf has K >= 1024, the workspace also holds the prepared TF32 hi/lo leaf
 * operands (without them, 3XTF32 calls run the slower fused-transform tensor
 * kernel).  No GPU needed.  New; the reference sizes its workspace with
 * local_elements (bag.cuh:23-30). */
bag_status bag_workspace_bytes_for(int mode, int m, int n, int k, int depth, int basis, int batch,
                                   size_t* bytes);
bag_status bag_workspace_destroy(bag_workspace* ws);
size_t bag_workspace_bytes(const bag_workspace* ws);
/* Device base of the workspace's rounded-operand blocks (NULL when the plan
 * needs none: Minimal basis at depth 1 fuses every transform). */
float* bag_workspace_data(const bag_workspace* ws);

/* C <- A B + C; A, B, C distinct column-major n x n, ld = n (bag.cuh:247-260).
 * Checks n == the workspace's n, the leaf against `backend`'s valid_shape, and
 * that BATCHED uses a paired backend, with the reference's error texts. */
bag_status bag_matmul(const float* a, const float* b, float* c, int n, bag_stream_t stream,
                      bag_workspace* ws, int backend, int schedule);

/* C <- A B + beta C (beta 0 or 1) for any m, n, k >= 0.  depth 0 is a plain
 * GEMM through the same kernel, BAG_DEPTH_AUTO picks one; ragged extents are
 * peeled into plain strips.
 * ws may be NULL when the plan needs no workspace (Minimal basis, depth <= 1). */
bag_status bag_sgemm_ex(int layout, int m, int n, int k, const float* a, long long lda,
                        const float* b, long long ldb, float* c, long long ldc, float beta,
                        int depth, int basis, bag_stream_t stream, bag_workspace* ws);

/* bag_sgemm_ex for callers that cannot allocate device memory -- e.g. a host
 * framework or serving process that owns a fixed device-memory pool and lets no
 * library call cudaMalloc, or a latency-critical caller that cannot afford an
 * allocation that may synchronise the device.  No counterpart in the reference.
 * Instead of a workspace it uses one built-in device scratch array of
 * 4,194,304 floats (16 MiB) that each GPU loading the library holds until the
 * process exits; problems needing more scratch (e.g. depth 2 beyond N = 1448
 * square) fail with BAG_ERR_WORKSPACE before anything is enqueued.  Every call
 * looks up the array's address on the current device (so a device reset does
 * not leave a stale address behind); the first call on a device may load the
 * library's device code there and should come before any stream capture on
 * that device.  In 3XTF32 mode the prepared TF32 operands are used when they
 * fit in the array, else the leaves run with the transforms fused in
 * (bag_last_leaf_kernel tells which).  All calls share the array, so calls
 * that can overlap on the GPU race and must be serialised by the caller.
 * Allocates nothing (no cudaMalloc/cudaFree). */
bag_status bag_sgemm_noalloc(int layout, int m, int n, int k, const float* a, long long lda,
                             const float* b, long long ldb, float* c, long long ldc, float beta,
                             int depth, int basis, bag_stream_t stream);

/* `batch` independent problems, operand i at base + i*stride (one launch). */
bag_status bag_sgemm_batched(int layout, int m, int n, int k, const float* a, long long lda,
                             long long stride_a, const float* b, long long ldb, long long stride_b,
                             float* c, long long ldc, long long stride_c, int batch, float beta,
                             int depth, int basis, bag_stream_t stream, bag_workspace* ws);

/* d (+)= gamma_d (x + delta y)(v + eps w), e likewise; column-major, x,y: m x k,
 * v,w: k x n, d,e: m x n.  delta, eps in {-1,0,1}; gamma in {-2..2}: +-1
 * accumulates (atomically when `atomic` != 0), +-2 overwrites, 0 skips. */
bag_status bag_primitive(int delta, int eps, int gamma_d, int gamma_e, int atomic,
                         const float* x, const float* y, const float* v, const float* w, float* d,
                         float* e, int m, int n, int k, long long ldx, long long ldy, long long ldv,
                         long long ldw, long long ldd, long long lde, bag_stream_t stream);

/* Two primitives with shared coefficients in one launch (strassen.cuh:167-197);
 * operand arrays are {x,y,v,w} and {d,e} for product 0 then product 1. */
bag_status bag_primitive_pair(int delta, int eps, int gamma_d, int gamma_e, int atomic,
                              const float* const operands[8], float* const outputs[4], int s,
                              long long ld, bag_stream_t stream);

/* Classic Strassen one level, C <- A B + C, column-major n x n (strassen.cuh:225-276). */
bag_status bag_strassen_one_level(int backend, int schedule, const float* a, const float* b,
                                  float* c, int n, bag_stream_t stream);

/* 1 when `s` satisfies `backend`'s tile constraint (strassen.cuh:57-66). */
bag_status bag_valid_shape(int backend, int s, int* valid);

/* Measurement hooks (new; no reference counterpart).  When set, the leaf
 * launches of later calls on this host thread are bracketed by
 * cudaEventRecord(start) / cudaEventRecord(end) on the call's stream, so a
 * caller can time the product kernel alone; NULL, NULL turns it off.
 * bag_launch_count returns how many kernels this process has launched. */
bag_status bag_profile_set_events(void* start_event, void* end_event);
/* Phase events (new): later calls of this host thread also record
 * `after_stages` once the operand materialisation launches are queued
 * (before any prepare or leaf launch) and `after_last` after the call's last
 * launch (the decode pass where there is one).  With the leaf events above
 * and an event the caller records before the call, a call splits into
 * stages | prepare | leaves | decode.  NULL, NULL turns it off. */
bag_status bag_profile_set_phase_events(void* after_stages, void* after_last);
unsigned long long bag_launch_count(void);
/* Device allocations (cudaMalloc calls) this library has made in this process:
 * workspaces, multi-GPU shard buffers, the self-test's flag.  New; diagnostic
 * (a caller can check that a call allocated nothing). */
unsigned long long bag_device_allocations(void);
/* Math mode of later calls on this host thread (like cublasSetMathMode);
 * new, no reference counterpart.  A thread starts in BAG_MATH_FFMA, or in
 * BAG_MATH_3XTF32 when the process was started with BAG_B200_MATH=3xtf32 (a
 * drop-in switch for programs that only call the reference's API). */
bag_status bag_set_math_mode(int mode);
int bag_get_math_mode(void);
/* Leaf arithmetic the last call on this host thread used (BAG_MATH_*): 3XTF32
 * only where the mode asks for it, every product has 16-byte-aligned operands
 * and every leaf K is >= 1024 (below that the FFMA path is the more accurate).
 * New; no reference counterpart. */
int bag_last_leaf_path(void);
/* Leaf kernel the last call on this host thread ran: the FFMA kernels; the
 * 3xTF32 kernel with the basis transforms fused into its prologue (no
 * prepared-operand workspace); or, on prepared operands, 128 x 256 tiles on
 * one SM or 256 x 256 tiles on a cluster of two SMs.  New; diagnostic. */
enum {
  BAG_LEAF_KERNEL_FFMA = 0,
  BAG_LEAF_KERNEL_TF32_FUSED = 1,
  BAG_LEAF_KERNEL_TF32_SINGLE = 2,
  BAG_LEAF_KERNEL_TF32_PAIR = 3
};
int bag_last_leaf_kernel(void);
/* Prepare kernel of the last call on this host thread: 1 Minimal, 2 Full,
 * 3 Classic, 4 Winograd when every operand expression matched that basis's
 * compiled-in tables (left and right operands), 0 for the kernel that reads
 * the expressions from the plan, -1 when the last call prepared nothing.
 * New; diagnostic. */
int bag_last_prepare_table(void);

/* Reads and clears the device error word (synchronous): non-zero when a
 * bounded in-kernel wait gave up instead of hanging (1) or a product reached a
 * kernel it was not planned for (2).  New; no reference counterpart. */
bag_status bag_device_error(unsigned* code);
/* Self-test of that mechanism (synchronous): one tiny launch whose only
 * thread waits, through the leaf kernels' bounded-wait routine, on an
 * mbarrier that nothing arrives on, giving up after limit_ns nanoseconds.
 * *gave_up receives 1 when the wait gave up and the kernel returned; the
 * device error word is then 1 (read it with bag_device_error).  New;
 * diagnostic. */
bag_status bag_selftest_bounded_wait(unsigned long long limit_ns, int* gave_up);
/* FP32 FFMA throughput probe (a roofline denominator): one launch of
 * 4 x SM-count CTAs x 256 threads of register-only fmaf chains; `sink` must
 * hold 1024 x SM-count floats.  *flops receives the launch's FLOP count. */
bag_status bag_ffma_probe(float* sink, int iterations, bag_stream_t stream, double* flops);

/* Several GPUs of one process (the proposed bag_sgemm_multi): C <- A B +
 * beta C with A, B, C on devices[0].  The devices form an R x S grid
 * (bag_multi_grid: 1x1, 2x1, 2x2, 4x2 for 1, 2, 4, 8 devices, else n x 1);
 * device (i, j) receives by peer copies row band i of every one of the
 * 2^depth block-rows of A (and of C when beta is 1) and column band j of every
 * block-column of B, runs the single-GPU path on those compact shards with its
 * own workspace and stream, and its C bands are copied back.  BAG combines only
 * blocks at equal offsets, so every device computes exactly the full product
 * restricted to its bands: no reduction between devices.  Needs M divisible by
 * 2^depth x R and N by 2^depth x S (of the column-major problem; row-major
 * swaps M and N).  Asynchronous: ordered after earlier work on `stream`
 * (devices[0]), and `stream` waits for every device.  The workspace is created
 * for one problem shape, device list and the calling thread's math mode, and
 * enables peer access between devices[0] and the others.  New; the reference
 * has no multi-GPU path. */
typedef struct bag_multi_workspace bag_multi_workspace;
bag_status bag_multi_grid(int ngpus, int* rows, int* cols);
bag_status bag_multi_workspace_create(int ngpus, const int* devices, int layout, int m, int n,
                                      int k, int depth, int basis, bag_multi_workspace** out);
bag_status bag_multi_workspace_destroy(bag_multi_workspace* ws);
bag_status bag_sgemm_multi(int ngpus, const int* devices, int layout, int m, int n, int k,
                           const float* a, long long lda, const float* b, long long ldb, float* c,
                           long long ldc, float beta, int depth, int basis, bag_stream_t stream,
                           bag_multi_workspace* ws);

/* Describe the plan for a column-major problem as JSON (no GPU needed).
 * Pointers are reported as {base, offset}: base 0=A, 1=B, 2=C, 3=workspace.
 * Writes at most buflen bytes; *needed receives the full length + 1. */
bag_status bag_plan_dump(int m, int n, int k, long long lda, long long ldb, long long ldc,
                         int depth, int basis, char* buf, size_t buflen, size_t* needed);

#ifdef __cplusplus
}
#endif
#endif /* BAG_CAPI_H */
