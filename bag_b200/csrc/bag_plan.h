// Launch descriptors shared by the host plan builder and the sm_100a kernels.
//
// A BAG call is compiled on the host into two kinds of work:
//
//  * materialisation jobs ("MatPlan"): elementwise signed sums of up to four
//    input blocks, written to workspace blocks.  Only operands that the
//    reference itself rounds before recursing (bag.cuh:124-135 prepare_child,
//    bag.cuh:66-68 the Full-basis transform) are materialised; everything at
//    the deepest level is fused into the GEMM prologue.
//  * leaf products ("LeafPlan"): every one of the 7^depth sub-products (plus
//    peeling strips for ragged shapes) as one grouped launch.  A product is a
//    list of signed left terms, signed right terms and signed output targets;
//    the kernel sums the terms while staging tiles into shared memory and adds
//    +-M into every C block the inverse transform sends it to.
//
// Both plans travel by value as __grid_constant__ kernel parameters, so a call
// needs no device-side table, no upload and no allocation.
#pragma once

#include <cstdint>

namespace bag_b200 {

// One signed operand or output reference: p + batch*bstride is the block's
// first element, column-major with leading dimension ld (elements).
struct Term {
  const float* p;
  long long bstride;
  int ld;
  float coef;   // +1 / -1 for operand terms; the gamma sign for outputs
  int mode;     // outputs only: kOutAtomic / kOutAdd / kOutOverwrite
  int pad_;
};

// Output update modes of a product target.
enum : int {
  kOutAtomic = 0,     // atomicAdd (red.global) -- safe for concurrent writers
  kOutAdd = 1,        // plain read-modify-write -- single writer only
  kOutOverwrite = 2,  // store coef*M -- single writer only (gamma = +-2)
};

// Compiled main loops by (left terms, right terms); kSigGeneric runs the
// runtime-count, element-masked loop.
enum : int {
  kSigGeneric = 0, kSig11, kSig12, kSig21, kSig22, kSig33, kSig41, kSig14,
};

struct Prod {
  int m, n, k;          // extents: left is m x k, right is k x n, output m x n
  int tiles_m, tiles_n; // CTA tiles covering the output
  int tile_begin;       // first work item of this product within the launch
  short l0, nl;         // left terms  [l0, l0+nl) in LeafPlan::terms
  short r0, nr;         // right terms
  short o0, no;         // outputs
  int sig;              // kSig* main loop (fast paths need aligned, m % 4 == k % 4 == 0)
};

constexpr int kMaxProducts = 64;
constexpr int kMaxTerms = 416;
constexpr int kMaxOperandTerms = 4;   // per operand per product (fused transform)

struct LeafPlan {
  int nprod;
  int ntiles;           // total work items (grid.x)
  Prod prod[kMaxProducts];
  Term terms[kMaxTerms];
};

constexpr int kMaxJobs = 24;
constexpr int kMaxJobInputs = 4;
constexpr int kMaxJobOutputs = 4;

struct MatJob {
  int rows, cols;
  int nin, nout;
  Term in[kMaxJobInputs];     // coef unused
  Term out[kMaxJobOutputs];   // coef unused
  // expr[o][t]: signed (input index + 1) of the t-th term of output o,
  // evaluated left to right; 0 ends the list.
  signed char expr[kMaxJobOutputs][kMaxJobInputs];
};

struct MatPlan {
  int njobs;
  long long chunk_begin[kMaxJobs + 1];   // prefix sums of float4 chunks per job
  MatJob job[kMaxJobs];
};

// Prepared operands (3xTF32 path): every distinct leaf operand is written as
// TF32 hi and lo rows of `cols` k values (k contiguous, zero-padded to the
// region's row length) at rows [out_hi, out_hi + rows) and [out_hi + rows,
// out_hi + 2 rows) of the prepared region; a left operand (column-major
// rows x cols, rows contiguous) is transposed on the way, a right operand (k
// contiguous) keeps its orientation.
//
// A leaf operand is a signed sum of "mids", each mid a signed sum of source
// blocks: at the deepest recursion level the operand the reference rounds
// before its last split (prepare_child, bag.cuh:124-135; the Full-basis
// transform, bag.cuh:66-68) is a mid, evaluated in FP32 in the reference's
// order exactly as a materialisation pass would round it, and the leaf
// operand sums such mids in the fused prologue's order (the first term with
// its sign, then fmaf with +-1).  The values are therefore those of
// materialising the mids first, without their HBM round trip.  A tree group
// holds up to 16 source blocks of one shape, read once per tile, and up to 8
// segments; a segment holds up to 4 mids (codes over the group's inputs) and
// up to 8 outputs (codes over the segment's mids).  At depth 2 with the
// Minimal basis one group per side covers all 49 leaf operands: the 16
// sub-blocks of A's (B's) quadrants, one segment per outer product.  Codes
// are signed (index + 1); 0 ends a list.
constexpr int kTreeIn = 16;
constexpr int kTreeSeg = 8;
constexpr int kTreeMid = 4;
constexpr int kTreeOut = 8;
constexpr int kMaxTreeGroups = 20;

struct TreeSeg {
  int nmid, nout;
  signed char mid[kTreeMid][kMaxOperandTerms];    // per mid: its inputs
  signed char expr[kTreeOut][kMaxOperandTerms];   // per output: its mids
  int out_hi[kTreeOut];                           // lo rows at out_hi + rows
};

struct TreeGroup {
  int rows, cols;
  int transpose, nin, nseg;
  int table;                                      // 1: segments hold the launch's compiled-in tables
  Term in[kTreeIn];                               // coef unused
  TreeSeg seg[kTreeSeg];
  long long tile_begin;                           // first work item of the group
};

struct PrepTreePlan {
  int ngroups;
  int row_len;                 // floats per region row (k, padded to the tile length)
  float* region;
  long long region_bstride;    // floats between batch entries' regions
  long long ntiles;
  TreeGroup group[kMaxTreeGroups];
};

// Leaf products on prepared operands: A rows a_hi.., B rows b_hi.. of the
// region; outputs as in LeafPlan.
struct PrepProd {
  int m, n, k;
  int tiles_m, tiles_n, tile_begin;
  int a_hi, a_lo, b_hi, b_lo;
  short o0, no;
};

struct PrepLeafPlan {
  int nprod;
  int ntiles;
  PrepProd prod[kMaxProducts];
  Term outs[kMaxTerms];
};

// Deferred inverse transform (prepared 3xTF32 path, several C blocks per
// product): the leaf kernel stores each product once into its own buffer
// M_p, then one pass adds every product into its C blocks, out[t] +=
// sum_p coef[p][t] * M_p, reading each M_p once and writing each block once.
// All products and targets share the extent m x n.
constexpr int kMaxDecodeProducts = 64;
constexpr int kMaxDecodeTargets = 16;

struct DecodePlan {
  int np, nt, m, n;
  int accumulate;                  // 1: out[t] += sum; 0: out[t] = sum
  Term in[kMaxDecodeProducts];     // M_p (coef unused)
  Term out[kMaxDecodeTargets];     // C blocks (coef unused)
  // Per target, its products in plan order: +-(p + 1); count[t] of them.
  signed char list[kMaxDecodeTargets][kMaxDecodeProducts];
  int count[kMaxDecodeTargets];
};

static_assert(sizeof(LeafPlan) < 32000, "kernel parameter limit");
static_assert(sizeof(DecodePlan) < 32000, "kernel parameter limit");
static_assert(sizeof(MatPlan) < 32000, "kernel parameter limit");
static_assert(sizeof(PrepTreePlan) < 32000, "kernel parameter limit");

}  // namespace bag_b200
