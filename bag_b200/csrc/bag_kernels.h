// Host-side entry points of the sm_100a kernels (bag_kernels.cu).
#pragma once

#include <cuda_runtime.h>

#include "bag_plan.h"

namespace bag_b200 {

enum : int {
  kTileLarge = 0,   // 128 x 128 CTA tile, 256 threads, 8 x 8 FFMA per thread, 2 CTAs/SM
  kTileSmall = 1,   // 64 x 64 CTA tile, 64 threads, for grids too small to fill 148 SMs
  kTileWide = 2,    // 128 x 256 CTA tile, 256 threads, 8 x 16 FFMA per thread, 1 CTA/SM
  kTileTall = 3,    // 256 x 128 CTA tile, 256 threads, 16 x 8 FFMA per thread, 1 CTA/SM
  kTileLarge1 = 4,  // 128 x 128 CTA tile, 256 threads, 8 x 8 per thread, 1 CTA/SM
  kTileHalf = 5,    // 128 x 64 CTA tile, 128 threads, 8 x 8 per thread, 2 CTAs/SM
  kTileTallS = 6,   // Tall with single-buffered register fragments
  kTileWS = 7,      // warp-specialised 128 x 128 kernel (bag_ws_kernel.cu), fast signatures only
  kTileMicro = 8,   // 32 x 32 CTA tile, 64 threads, 4 x 4 FFMA per thread, for tiny grids
  kTileCount = 9,
};

struct TileShape {
  int bm, bn;
};

TileShape leaf_tile_shape(int config);

// One grouped launch of every product in `plan`; grid = (plan.ntiles, batch).
// `vec` selects 128-bit loads/stores and requires every term pointer 16-byte
// aligned with ld % 4 == 0 and every block offset a multiple of 4 rows.
cudaError_t launch_leaf(const LeafPlan& plan, int config, bool vec, int batch, cudaStream_t stream);

// FP32 FFMA throughput probe over `blocks` CTAs of 256 threads; `sink` holds
// blocks*256 floats.  *flops receives the FLOPs the launch performs.
cudaError_t launch_ffma_probe(float* sink, int blocks, int iters, cudaStream_t stream,
                              double* flops);

// Warp-specialised leaf kernel (bag_ws_kernel.cu): every product must have a
// fast signature (sig != kSigGeneric) and 16-byte-aligned operands.
TileShape ws_tile_shape();
cudaError_t launch_leaf_ws(const LeafPlan& plan, int batch, cudaStream_t stream);

// 3xTF32 tcgen05 leaf kernel (bag_tc_kernel.cu).  Operand terms are read by
// TMA: a term inside one of `sources` (same ld and batch stride, block within
// its rows x cols) goes through that matrix's tensor map at the block's
// coordinates, any other term through a map of its own block.  Every operand
// must be 16-byte aligned with ld and batch stride multiples of 4.
struct TcSource {
  const float* base;
  long long ld, bstride;
  long long rows, cols;
};
TileShape tc_tile_shape();
// Whether the kernel takes a product with nl left and nr right terms (and the
// driver offers cuTensorMapEncodeTiled).
bool tc_supported(int nl, int nr);
cudaError_t launch_leaf_tc(const LeafPlan& plan, const TcSource* sources, int nsources, int batch,
                           cudaStream_t stream);
cudaError_t read_and_clear_tc_device_error(unsigned* value);

// Prepared-operand 3xTF32 path (bag_tc3_kernel.cu): prep_tree_kernel writes each
// leaf operand's TF32 hi/lo rows into a workspace region (rows of row_len k,
// row_len a multiple of prep_row_align()); the leaf kernels run the products
// on them: leaf_prep_kernel with 128 x 256 tiles on one SM each
// (kPrepLeafSingle), leaf_pair_kernel with 256 x 128 tiles on a cluster of two
// SMs (kPrepLeafPair, where the device schedules such clusters).
enum : int { kPrepLeafSingle = 0, kPrepLeafPair = 1 };
bool prep_supported();
bool prep_pair_supported();
int prep_row_align();
// prep_tree_kernel's tile: rows x k of every operand of a tree group per CTA.
constexpr int kPrepTreeRows = 16;
constexpr int kPrepTreeK = 64;
// Compiled-in operand expression tables of the tree prepare (4 bases x 2
// sides); last_tree_expr_table() is the last launch's basis (1 Minimal,
// 2 Full, 3 Classic, 4 Winograd; 0 = the plan-reading kernel).
constexpr int kTreeExprCount = 8;
int last_tree_expr_table();
// Flags the groups of `plan` whose segments hold one basis's compiled-in
// tables (TreeGroup::table) and returns that basis (1..4), 0 when none does;
// launch_prep_tree calls it, plan dumps report it.
int mark_tree_tables(PrepTreePlan& plan);
TileShape prep_tile_shape(int kind);
cudaError_t launch_prep_tree(PrepTreePlan& plan, int batch, cudaStream_t stream);  // sets group[].table
cudaError_t launch_leaf_prep(const PrepLeafPlan& plan, int kind, const float* region,
                             long long row_len, long long rows, long long region_bstride,
                             int batch, cudaStream_t stream);
cudaError_t read_and_clear_tc3_device_error(unsigned* value);
// One launch of the bounded-wait self-test (bag_tc3_kernel.cu).
cudaError_t run_wait_selftest(unsigned long long limit_ns, int* gave_up_device,
                              cudaStream_t stream);

// Reads and clears the device error word that bounded waits set on timeout.
cudaError_t read_and_clear_device_error(unsigned* value);

// The deferred inverse transform: out[t] += sum_p coef[p][t] * in[p] over
// m x n blocks (column-major, 16-byte aligned, ld % 4 == 0).
cudaError_t launch_decode(const DecodePlan& plan, int batch, cudaStream_t stream);

// One launch of every materialisation job in `plan`.
cudaError_t launch_materialize(const MatPlan& plan, int batch, cudaStream_t stream, int sm_count);

}  // namespace bag_b200
