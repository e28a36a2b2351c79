// C ABI and host plan builder of the B200-native BAG FP32 matmul.
//
// The builder turns one call into (a) at most a few materialisation stages and
// (b) grouped leaf launches.  It walks the recursion of the reference
// (bag.cuh:152-245): at each level an operand that is a sum of several blocks
// is first rounded into the workspace, exactly where the reference's
// prepare_child (bag.cuh:124-135) rounds it, the Full basis materialises its
// transformed quadrants where prepare<true> does (bag.cuh:66-68), and the
// seven products' operand combinations at the deepest level are fused into the
// GEMM prologue.  Outputs skip the reference's T workspace: each leaf product
// carries the signed list of C blocks the composed inverse transforms send it
// to (bag.py:530-533 for one level), so there is no decode kernel.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/bag_capi.h"
#include "bag_kernels.h"

struct bag_workspace {
  int m, n, k, depth, basis, batch;
  int device;
  float* data;
  size_t elements;
};

namespace bag_b200 {
namespace {

thread_local std::string g_last_error;

// The math mode every host thread starts in: FFMA (the reference's
// sequential-fmaf numerics) unless the environment's BAG_B200_MATH says
// "3xtf32", so a program written against the reference's headers takes the
// tensor-core leaves without a code change.  Read once per process; a value
// other than "ffma" or "3xtf32" is reported on stderr and FFMA kept.
int process_default_math_mode() {
  static const int mode = [] {
    const char* env = std::getenv("BAG_B200_MATH");
    if (!env || !*env || std::strcmp(env, "ffma") == 0) return int(BAG_MATH_FFMA);
    if (std::strcmp(env, "3xtf32") == 0) return int(BAG_MATH_3XTF32);
    std::fprintf(stderr, "bag_b200: BAG_B200_MATH=%s is not ffma or 3xtf32; using ffma\n", env);
    return int(BAG_MATH_FFMA);
  }();
  return mode;
}

thread_local int g_math_mode = process_default_math_mode();
thread_local int g_last_leaf_path = BAG_MATH_FFMA;
// Leaf kernel of the last call's prepared-operand path (BAG_LEAF_KERNEL_*).
thread_local int g_last_prep_kind = -1;
// Shortest leaf K the 3xTF32 path takes.  Its tensor-core partial sums carry a
// fixed error of about 1.4e-7 (hi/lo split and round-toward-zero
// accumulation within a 32-long chunk); an FP32 FFMA dot product's error grows
// with K and passes it near K = 256.  Measured on B200 (N(0,1) operands):
// tensor/FFMA error ratio 2.1 at K = 64, 1.07 at 256, 0.56 at 1024, 0.32 at 4096.
constexpr int kTcMinK = 1024;

// BAG_DEPTH_AUTO: the depth is chosen from the shape and this thread's math
// mode.  Measured on B200 (N(0,1) inputs, effective TFLOP/s, depths 0/1/2/3):
// 3xTF32 -- 2048^3: 148/144; 4096^3: 187/205/189; 8192^3: 227/252/247/137;
// 16384^3: 218/238/266/203; 8192x4096x16384 (m x n x k): 220/239/230/154;
// 10000^3: 212/239/233 -- so no recursion below 4096, at least one level
// from 4096, and further levels while the leaves stay >= 4096 (shorter leaves
// pay the prepare and decode passes for less saved work).  FFMA one level
// deeper per doubling from 2048 (N=4096: d1 49, d2 53; N=8192: d2 58, d3 55;
// N=16384: d2 60, d3 63).
int resolve_depth(int depth, int m, int n, int k) {
  if (depth != BAG_DEPTH_AUTO) return depth;
  const int s = std::min(m, std::min(n, k));
  if (g_math_mode == BAG_MATH_3XTF32) {
    if (s < 4096) return 0;
    int d = 1;
    while (d < 3 && (s >> (d + 1)) >= 4096) ++d;
    return d;
  }
  return s >= 16384 ? 3 : s >= 2048 ? 2 : s >= 1024 ? 1 : 0;
}
thread_local cudaEvent_t g_prof_start = nullptr;
thread_local cudaEvent_t g_prof_end = nullptr;
// Phase events: after the materialisation stages, and after the call's last
// launch (the decode pass where there is one).
thread_local cudaEvent_t g_phase_stages = nullptr;
thread_local cudaEvent_t g_phase_done = nullptr;

void record_phase(cudaEvent_t ev, cudaStream_t stream);
std::atomic<unsigned long long> g_launches{0};
// Device allocations this library has made (every cudaMalloc goes through
// device_alloc).
std::atomic<unsigned long long> g_device_allocs{0};

cudaError_t device_alloc(void** p, size_t bytes) {
  ++g_device_allocs;
  return cudaMalloc(p, bytes);
}

struct Error : std::runtime_error {
  bag_status status;
  Error(bag_status s, const std::string& what) : std::runtime_error(what), status(s) {}
};

[[noreturn]] void fail(bag_status s, const std::string& what) { throw Error(s, what); }

void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) fail(BAG_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

int sm_count_for_current_device() {
  static std::mutex mu;
  static std::map<int, int> cache;
  int dev = 0;
  cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(dev);
  if (it != cache.end()) return it->second;
  int count = 0;
  cuda_check(cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev),
             "cudaDeviceGetAttribute");
  cache[dev] = count;
  return count;
}

// ---------------------------------------------------------------------------
// Plan builder.
// ---------------------------------------------------------------------------

struct View {
  const float* p;
  long long ld;
  long long bstride;
  bool operator==(const View& o) const { return p == o.p && ld == o.ld && bstride == o.bstride; }
};

struct STerm {
  View v;
  float coef;
};
using Expr = std::vector<STerm>;

struct Target {
  View v;
  float coef;
  int mode;
};

struct HostLeaf {
  int m, n, k;
  Expr left, right;
  std::vector<Target> out;
  int prep_l = -1, prep_r = -1;   // prepared operands (Builder::prep), -1: none
};

struct HostJob {
  int rows, cols;
  std::vector<View> in;
  std::vector<View> out;
  std::vector<std::vector<int>> expr;   // signed (input index + 1)
};

enum BasisKind {
  kMinimal = BAG_BASIS_MINIMAL,
  kFull = BAG_BASIS_FULL,
  kClassic = BAG_BASIS_CLASSIC,
  kWinograd = BAG_BASIS_WINOGRAD
};

bool known_basis(int basis) {
  return basis == kMinimal || basis == kFull || basis == kClassic || basis == kWinograd;
}

// One level of each algorithm: operand combinations over quadrants
// (0=X11, 1=X12, 2=X21, 3=X22) as ordered signed terms, and the signed C
// quadrants the product is added to.
struct Combo {
  int n;
  int q[4];
  int s[4];
};
struct LevelProduct {
  Combo left, right;
  int out[4];   // coefficient per C quadrant
};

// Minimal basis: operand sums in the order the reference evaluates them
// (SA = A12 - A21 + A22 as in bag.cuh:72; SA - A11 as x + delta*y with
// x = SA, bag.cuh:118), outputs from the composed inverse transform
// C11=M4+M5, C12=M3+M5-M6-M2, C21=M1-M3-M5-M7, C22=M1+M2-M3-M5 (bag.py:530-533).
const LevelProduct kMinimal7[7] = {
    {{2, {1, 3}, {1, 1}}, {2, {1, 3}, {1, 1}}, {0, 0, 1, 1}},                     // M1
    {{2, {3, 2}, {1, -1}}, {2, {3, 2}, {1, -1}}, {0, -1, 0, 1}},                  // M2
    {{3, {1, 2, 3}, {1, -1, 1}}, {3, {1, 2, 3}, {1, -1, 1}}, {0, 1, -1, -1}},     // M3
    {{1, {0}, {1}}, {1, {0}, {1}}, {1, 0, 0, 0}},                                 // M4
    {{1, {1}, {1}}, {1, {2}, {1}}, {1, 1, -1, -1}},                               // M5
    {{4, {1, 2, 3, 0}, {1, -1, 1, -1}}, {1, {1}, {1}}, {0, -1, 0, 0}},            // M6
    {{1, {2}, {1}}, {4, {1, 2, 3, 0}, {1, -1, 1, -1}}, {0, 0, -1, 0}},            // M7
};

// Full basis: operands are x + delta*y over the transformed quadrants
// T11=X11, T12=X12-X21+X22, T21=X22-X21, T22=X12+X22 (bag.cuh:101-110, 171-189).
const LevelProduct kFull7[7] = {
    {{1, {3}, {1}}, {1, {3}, {1}}, {0, 0, 1, 1}},
    {{1, {2}, {1}}, {1, {2}, {1}}, {0, -1, 0, 1}},
    {{1, {1}, {1}}, {1, {1}, {1}}, {0, 1, -1, -1}},
    {{1, {0}, {1}}, {1, {0}, {1}}, {1, 0, 0, 0}},
    {{2, {1, 2}, {1, -1}}, {2, {3, 1}, {1, -1}}, {1, 1, -1, -1}},
    {{2, {1, 0}, {1, -1}}, {2, {1, 2}, {1, -1}}, {0, -1, 0, 0}},
    {{2, {3, 1}, {1, -1}}, {2, {1, 0}, {1, -1}}, {0, 0, -1, 0}},
};

// Classic Strassen-1969, strassen.cuh:131-153 (x + delta*y, v + eps*w order).
const LevelProduct kClassic7[7] = {
    {{2, {2, 3}, {1, 1}}, {1, {0}, {1}}, {0, 0, 1, -1}},
    {{2, {0, 1}, {1, 1}}, {1, {3}, {1}}, {-1, 1, 0, 0}},
    {{2, {2, 0}, {1, -1}}, {2, {0, 1}, {1, 1}}, {0, 0, 0, 1}},
    {{2, {1, 3}, {1, -1}}, {2, {2, 3}, {1, 1}}, {1, 0, 0, 0}},
    {{1, {0}, {1}}, {2, {1, 3}, {1, -1}}, {0, 1, 0, 1}},
    {{1, {3}, {1}}, {2, {2, 0}, {1, -1}}, {1, 0, 1, 0}},
    {{2, {0, 3}, {1, 1}}, {2, {0, 3}, {1, 1}}, {1, 0, 0, 1}},
};

// Strassen-Winograd, the 15-addition form (Winograd 1971): with
// S1 = A21+A22, S2 = S1-A11, S3 = A11-A21, S4 = A12-S2 and T1 = B12-B11,
// T2 = B22-T1, T3 = B22-B12, T4 = T2-B21, the products M1 = A11 B11,
// M2 = A12 B21, M3 = S4 B22, M4 = A22 T4, M5 = S1 T1, M6 = S2 T2, M7 = S3 T3
// give C11 = M1+M2, C12 = M1+M6+M5+M3, C21 = M1+M6+M7-M4, C22 = M1+M6+M7+M5.
// Operands are written as flat signed sums in the order the intermediates
// form them; outputs by direct decode.
const LevelProduct kWinograd7[7] = {
    {{1, {0}, {1}}, {1, {0}, {1}}, {1, 1, 1, 1}},                                  // M1
    {{1, {1}, {1}}, {1, {2}, {1}}, {1, 0, 0, 0}},                                  // M2
    {{4, {1, 2, 3, 0}, {1, -1, -1, 1}}, {1, {3}, {1}}, {0, 1, 0, 0}},              // M3
    {{1, {3}, {1}}, {4, {3, 1, 0, 2}, {1, -1, 1, -1}}, {0, 0, -1, 0}},             // M4
    {{2, {2, 3}, {1, 1}}, {2, {1, 0}, {1, -1}}, {0, 1, 0, 1}},                     // M5
    {{3, {2, 3, 0}, {1, 1, -1}}, {3, {3, 1, 0}, {1, -1, 1}}, {0, 1, 1, 1}},        // M6
    {{2, {0, 2}, {1, -1}}, {2, {3, 1}, {1, -1}}, {0, 0, 1, 1}},                    // M7
};

struct Builder {
  int basis;
  float* ws = nullptr;      // workspace base (may be a fake base for dumps)
  size_t ws_used = 0;       // elements per batch entry
  long long ws_bstride = 0; // elements between batch entries' workspaces
  struct Buf {
    const float* begin;
    const float* end;
    int stage;
  };
  std::vector<Buf> bufs;
  std::vector<std::vector<HostJob>> stages;   // stages[s-1]: jobs of stage s
  std::vector<HostLeaf> leaves;

  int stage_of(const View& v) const {
    for (const Buf& b : bufs)
      if (v.p >= b.begin && v.p < b.end) return b.stage;
    return 0;
  }

  View alloc(int rows, int cols, int stage) {
    const long long ld = std::max<long long>(4, (rows + 3) / 4 * 4);
    const size_t count = size_t(ld) * cols;
    const size_t begin = (ws_used + 63) / 64 * 64;   // 256-byte aligned
    ws_used = begin + count;
    const float* p = ws + begin;
    bufs.push_back({p, p + std::max<size_t>(count, 1), stage});
    return {p, ld, ws_bstride};
  }

  // Rounded operands of the deepest level on the prepared path stay
  // virtual: no workspace block is written for them; the prepare pass
  // evaluates them (the mids of a tree group) in the same order instead.  A
  // virtual block is a range of fake addresses far above any device pointer
  // with its definition, so a view inside it resolves to the same offset in
  // each of the definition's terms.
  bool virtual_last = false;
  struct VBuf {
    const float* begin;
    const float* end;
    long long ld;
    int rows, cols;
    Expr def;
  };
  std::vector<VBuf> vbufs;
  uintptr_t vnext = uintptr_t(1) << 50;

  const VBuf* vbuf_of(const View& v) const {
    for (const VBuf& b : vbufs)
      if (v.p >= b.begin && v.p < b.end) return &b;
    return nullptr;
  }

  // A view as a signed sum of real blocks: a virtual view is its block's
  // definition at the view's offset, any other view itself.
  Expr resolve(const View& v) const {
    const VBuf* b = vbuf_of(v);
    if (!b) return {{v, 1.f}};
    const long long off = v.p - b->begin, col = off / b->ld, row = off % b->ld;
    Expr e;
    for (const STerm& t : b->def)
      e.push_back({{t.v.p + row + col * t.v.ld, t.v.ld, t.v.bstride}, t.coef});
    return e;
  }

  // Round a signed sum of blocks into the workspace (one job output), or,
  // with `may_virtualize` on the prepared path and only real blocks in the
  // sum, define a virtual block.
  View materialize(const Expr& e, int rows, int cols, bool may_virtualize = false) {
    if (virtual_last && may_virtualize) {
      bool real = true;
      for (const STerm& t : e) real = real && vbuf_of(t.v) == nullptr;
      if (real) {
        const long long ld = std::max<long long>(4, (rows + 3) / 4 * 4);
        const float* p = reinterpret_cast<const float*>(vnext);
        const size_t count = size_t(ld) * std::max(cols, 1);
        vnext += (count * sizeof(float) + 255) / 256 * 256;
        vbufs.push_back({p, p + count, ld, rows, cols, e});
        return {p, ld, ws_bstride};
      }
    }
    int stage = 1;
    for (const STerm& t : e) stage = std::max(stage, stage_of(t.v) + 1);
    if ((int)stages.size() < stage) stages.resize(stage);
    const View out = alloc(rows, cols, stage);
    auto& jobs = stages[stage - 1];
    // Join the job that already reads most of these blocks, so one pass over
    // a quadrant set writes all of its combinations.
    HostJob* best = nullptr;
    int best_overlap = 0;
    for (HostJob& j : jobs) {
      if (j.rows != rows || j.cols != cols || (int)j.out.size() >= kMaxJobOutputs) continue;
      int overlap = 0;
      size_t fresh = 0;
      for (const STerm& t : e) {
        if (std::find(j.in.begin(), j.in.end(), t.v) != j.in.end()) ++overlap;
        else ++fresh;
      }
      if (overlap > best_overlap && j.in.size() + fresh <= size_t(kMaxJobInputs)) {
        best = &j;
        best_overlap = overlap;
      }
    }
    if (best) {
      HostJob& j = *best;
      std::vector<View>& in = j.in;
      for (const STerm& t : e)
        if (std::find(in.begin(), in.end(), t.v) == in.end()) in.push_back(t.v);
      std::vector<int> code;
      for (const STerm& t : e) {
        const int idx = int(std::find(in.begin(), in.end(), t.v) - in.begin()) + 1;
        code.push_back(t.coef > 0 ? idx : -idx);
      }
      j.out.push_back(out);
      j.expr.push_back(code);
      return out;
    }
    HostJob j;
    j.rows = rows;
    j.cols = cols;
    std::vector<int> code;
    for (const STerm& t : e) {
      j.in.push_back(t.v);
      code.push_back(t.coef > 0 ? int(j.in.size()) : -int(j.in.size()));
    }
    j.out.push_back(out);
    j.expr.push_back(code);
    jobs.push_back(j);
    return out;
  }

  // Prepared operands (3xTF32 path): every distinct leaf operand is written
  // once, as TF32 hi and lo rows of the prepared region (rows of
  // prep_row_len k values), by one HBM-speed pass; the leaf products then
  // only load and multiply.  With the tensor core the fused transform and
  // split, not the tensor core, bound a product.  An operand is a signed sum
  // of mids, each mid a signed sum of real blocks (a virtual block's
  // definition, or one block).
  using Mid = Expr;
  struct PrepOp {
    std::vector<std::pair<Mid, float>> terms;   // (mid, +-1) in the prologue's order
    int rows, cols;
    bool transpose;   // left operands: column-major rows x cols -> k-contiguous rows
    int hi_row;       // lo rows follow at hi_row + rows
  };
  std::vector<PrepOp> prep;
  int prep_rows = 0, prep_row_len = 0;
  View prep_region{nullptr, 0, 0};

  static bool same_expr(const Expr& a, const Expr& b) {
    if (a.size() != b.size()) return false;
    for (size_t i = 0; i < a.size(); ++i)
      if (!(a[i].v == b[i].v) || a[i].coef != b[i].coef) return false;
    return true;
  }

  int prep_index(const Expr& e, int rows, int cols, bool transpose) {
    std::vector<std::pair<Mid, float>> terms;
    for (const STerm& t : e) terms.push_back({resolve(t.v), t.coef});
    for (size_t i = 0; i < prep.size(); ++i) {
      const PrepOp& o = prep[i];
      if (o.rows != rows || o.cols != cols || o.transpose != transpose ||
          o.terms.size() != terms.size())
        continue;
      bool same = true;
      for (size_t t = 0; t < terms.size() && same; ++t)
        same = o.terms[t].second == terms[t].second && same_expr(o.terms[t].first, terms[t].first);
      if (same) return int(i);
    }
    prep.push_back({terms, rows, cols, transpose, prep_rows});
    prep_rows += 2 * rows;
    return int(prep.size()) - 1;
  }

  void prepare_leaf_operands(int row_align) {
    int kmax = 0;
    for (const HostLeaf& l : leaves) kmax = std::max(kmax, l.k);
    prep_row_len = std::max(row_align, (kmax + row_align - 1) / row_align * row_align);
    for (HostLeaf& l : leaves) {
      l.prep_l = prep_index(l.left, l.m, l.k, true);
      l.prep_r = prep_index(l.right, l.n, l.k, false);
    }
    prep_region = alloc(prep_row_len, std::max(prep_rows, 1), int(stages.size()) + 1);
    build_trees();
  }

  // Tree groups (prep_tree_kernel): operands of one shape whose mids fit a
  // segment (<= 4 mids, <= 8 outputs) and whose blocks fit a group (<= 16
  // inputs, <= 8 segments) are prepared together, each block read once per
  // tile.  First fit in prep order.
  struct TreeSegHost {
    std::vector<Mid> mids;
    std::vector<int> ops;                  // indices into prep
    std::vector<std::vector<int>> expr;    // per op: +-(mid index + 1)
  };
  struct TreeGroupHost {
    int rows, cols;
    bool transpose;
    std::vector<View> in;
    std::vector<TreeSegHost> segs;
    int input_code(const STerm& t) const {
      const int u = int(std::find(in.begin(), in.end(), t.v) - in.begin());
      return t.coef > 0 ? u + 1 : -(u + 1);
    }
  };
  std::vector<TreeGroupHost> trees;

  static int find_mid(const std::vector<Mid>& mids, const Mid& m) {
    for (size_t i = 0; i < mids.size(); ++i)
      if (same_expr(mids[i], m)) return int(i);
    return -1;
  }

  void build_trees() {
    trees.clear();
    for (size_t j = 0; j < prep.size(); ++j) {
      const PrepOp& o = prep[j];
      if (o.terms.empty() || o.terms.size() > size_t(kMaxOperandTerms))
        fail(BAG_ERR_INTERNAL, "prepared operand has an unsupported term count");
      std::vector<Mid> om;
      std::vector<View> oin;
      for (const auto& t : o.terms) {
        if (t.second != 1.f && t.second != -1.f)
          fail(BAG_ERR_INTERNAL, "prepared operand term coefficient is not +-1");
        if (t.first.empty() || t.first.size() > size_t(kMaxOperandTerms))
          fail(BAG_ERR_INTERNAL, "prepared operand mid has an unsupported term count");
        if (find_mid(om, t.first) < 0) om.push_back(t.first);
        for (const STerm& x : t.first) {
          if (x.coef != 1.f && x.coef != -1.f)
            fail(BAG_ERR_INTERNAL, "prepared operand block coefficient is not +-1");
          if (std::find(oin.begin(), oin.end(), x.v) == oin.end()) oin.push_back(x.v);
        }
      }
      if (om.size() > size_t(kTreeMid) || oin.size() > size_t(kTreeIn))
        fail(BAG_ERR_INTERNAL, "prepared operand too wide for a tree group");
      auto fresh_inputs = [&](const TreeGroupHost& g) {
        size_t fresh = 0;
        for (const View& v : oin)
          if (std::find(g.in.begin(), g.in.end(), v) == g.in.end()) ++fresh;
        return g.in.size() + fresh;
      };
      TreeGroupHost* home = nullptr;
      TreeSegHost* seg = nullptr;
      for (TreeGroupHost& g : trees) {
        if (g.rows != o.rows || g.cols != o.cols || g.transpose != o.transpose ||
            fresh_inputs(g) > size_t(kTreeIn))
          continue;
        for (TreeSegHost& sg : g.segs) {
          if (sg.ops.size() >= size_t(kTreeOut)) continue;
          size_t fresh = 0;
          for (const Mid& m : om) fresh += find_mid(sg.mids, m) < 0 ? 1 : 0;
          if (sg.mids.size() + fresh <= size_t(kTreeMid)) {
            home = &g;
            seg = &sg;
            break;
          }
        }
        if (seg) break;
        if (!home && g.segs.size() < size_t(kTreeSeg)) home = &g;
      }
      if (!home) {
        trees.push_back({o.rows, o.cols, o.transpose, {}, {}});
        home = &trees.back();
      }
      if (!seg) {
        home->segs.push_back({});
        seg = &home->segs.back();
      }
      for (const View& v : oin)
        if (std::find(home->in.begin(), home->in.end(), v) == home->in.end()) home->in.push_back(v);
      std::vector<int> codes;
      for (const auto& t : o.terms) {
        int mi = find_mid(seg->mids, t.first);
        if (mi < 0) {
          seg->mids.push_back(t.first);
          mi = int(seg->mids.size()) - 1;
        }
        codes.push_back(t.second > 0 ? mi + 1 : -(mi + 1));
      }
      seg->ops.push_back(int(j));
      seg->expr.push_back(codes);
    }
  }

  // Deferred inverse transform (prepared path): when products update several
  // C blocks each, every product instead stores its result once into its
  // own workspace buffer and one pass (decode_kernel) adds the buffers into
  // their C blocks -- each buffer read once, each block written once, in
  // plan order -- instead of ~4 atomic read-modify-writes per output element.
  struct Decode {
    bool on = false;
    bool overwrite = false;   // C = sum (beta 0) instead of C += sum
    int m = 0, n = 0;
    std::vector<View> targets;
    std::vector<View> buffers;                               // one per leaf
    std::vector<std::vector<std::pair<int, float>>> terms;   // per leaf: (target, coef)
  } decode;

  void defer_decode() {
    if (leaves.empty() || leaves.size() > size_t(kMaxDecodeProducts)) return;
    size_t outs = 0;
    for (const HostLeaf& l : leaves) outs += l.out.size();
    // Measured on B200: the atomic epilogue slows the leaf kernel more than
    // a store and a pass cost, from depth 1 up (one level: ~1.7 targets a
    // product; cfg5's leaves 5.1 -> 3.9 ms).
    if (outs < leaves.size()) return;
    const int m = leaves[0].m, n = leaves[0].n;
    std::vector<View> targets;
    for (const HostLeaf& l : leaves) {
      if (l.m != m || l.n != n) return;
      for (size_t i = 0; i < l.out.size(); ++i) {
        const Target& t = l.out[i];
        if (t.mode != kOutAtomic || (t.coef != 1.f && t.coef != -1.f)) return;
        for (size_t j = 0; j < i; ++j)
          if (l.out[j].v == t.v) return;   // one coefficient per (product, block)
        if (std::find(targets.begin(), targets.end(), t.v) == targets.end()) targets.push_back(t.v);
      }
    }
    if (targets.size() > size_t(kMaxDecodeTargets)) return;
    decode.on = true;
    decode.m = m;
    decode.n = n;
    decode.targets = targets;
    for (HostLeaf& l : leaves) {
      const View buf = alloc(m, n, int(stages.size()) + 1);
      std::vector<std::pair<int, float>> terms;
      for (const Target& t : l.out)
        terms.push_back({int(std::find(targets.begin(), targets.end(), t.v) - targets.begin()),
                         t.coef});
      decode.buffers.push_back(buf);
      decode.terms.push_back(terms);
      l.out = {{buf, 1.f, kOutOverwrite}};
    }
  }

  // Reduce an operand to a single unit-coefficient block.  A lone negated
  // block keeps its data; the sign moves to the outputs (exact).
  View single(const Expr& e, int rows, int cols, float* sign, bool may_virtualize = false) {
    if (e.size() == 1) {
      *sign = e[0].coef;
      return e[0].v;
    }
    *sign = 1.f;
    return materialize(e, rows, cols, may_virtualize);
  }

  static void quads(const View& v, int rows, int cols, View q[4]) {
    const long long h = rows / 2, w = (long long)(cols / 2) * v.ld;
    q[0] = {v.p, v.ld, v.bstride};
    q[1] = {v.p + w, v.ld, v.bstride};
    q[2] = {v.p + h, v.ld, v.bstride};
    q[3] = {v.p + h + w, v.ld, v.bstride};
  }

  // Full-basis transform of one operand's quadrants (bag.cuh:66-68):
  // T11 = X11 (a view), T12 = X12 - X21 + X22, T21 = X22 - X21, T22 = X12 + X22.
  void full_transform(const View q[4], int rows, int cols, View t[4], bool may_virtualize) {
    t[0] = q[0];
    t[1] = materialize({{q[1], 1.f}, {q[2], -1.f}, {q[3], 1.f}}, rows, cols, may_virtualize);
    t[2] = materialize({{q[3], 1.f}, {q[2], -1.f}}, rows, cols, may_virtualize);
    t[3] = materialize({{q[1], 1.f}, {q[3], 1.f}}, rows, cols, may_virtualize);
  }

  void expand(const Expr& L, const Expr& R, const std::vector<Target>& T, int m, int k, int n,
              int depth) {
    if (depth == 0) {
      leaves.push_back({m, n, k, L, R, T});
      return;
    }
    // At the last level the operands' quadrants become leaf operand terms, so
    // on the prepared path what this level rounds can stay virtual (the Full
    // basis transforms the quadrants first: there only the transform does).
    const bool last = depth == 1;
    float ls = 1.f, rs = 1.f;
    const View lv = single(L, m, k, &ls, last && basis != kFull);
    const View rv = single(R, k, n, &rs, last && basis != kFull);
    View lq[4], rq[4];
    quads(lv, m, k, lq);
    quads(rv, k, n, rq);
    const int h = m / 2, kk = k / 2, w = n / 2;
    const LevelProduct* table = basis == kFull       ? kFull7
                                : basis == kClassic  ? kClassic7
                                : basis == kWinograd ? kWinograd7
                                                     : kMinimal7;
    if (basis == kFull) {
      View lt[4], rt[4];
      full_transform(lq, h, kk, lt, last);
      full_transform(rq, kk, w, rt, last);
      std::copy(lt, lt + 4, lq);
      std::copy(rt, rt + 4, rq);
    }
    for (int p = 0; p < 7; ++p) {
      const LevelProduct& lp = table[p];
      Expr l, r;
      for (int i = 0; i < lp.left.n; ++i) l.push_back({lq[lp.left.q[i]], float(lp.left.s[i])});
      for (int i = 0; i < lp.right.n; ++i) r.push_back({rq[lp.right.q[i]], float(lp.right.s[i])});
      std::vector<Target> t;
      for (const Target& tg : T) {
        View cq[4];
        quads(tg.v, m, n, cq);
        for (int q = 0; q < 4; ++q)
          if (lp.out[q]) t.push_back({cq[q], tg.coef * ls * rs * float(lp.out[q]), tg.mode});
      }
      expand(l, r, t, h, kk, w, depth - 1);
    }
  }
};

struct GemmDesc {
  int m, n, k;                 // column-major C(m x n) += A(m x k) B(k x n)
  const float* a;
  long long lda, sa;
  const float* b;
  long long ldb, sb;
  float* c;
  long long ldc, sc;
  int batch;
  int depth, basis;
};

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Build the plan; ws may be a fake base when only sizes are wanted.  With
// `leaf_operands` every leaf operand is also given a prepared (TF32 hi/lo)
// copy in the workspace.
void build_plan(const GemmDesc& g, float* ws, long long ws_bstride, Builder& B,
                bool leaf_operands = false) {
  B.basis = g.basis;
  B.ws = ws;
  B.ws_bstride = ws_bstride;
  B.virtual_last = leaf_operands;
  const View A{g.a, g.lda, g.sa}, Bv{g.b, g.ldb, g.sb}, C{g.c, g.ldc, g.sc};
  if (g.m == 0 || g.n == 0) return;
  int depth = g.depth;
  // Peel so every level halves exactly and block offsets stay 16-byte aligned.
  const int align = 4 << depth;
  int mc = g.m - g.m % align, kc = g.k - g.k % align, nc = g.n - g.n % align;
  if (depth == 0 || mc == 0 || kc == 0 || nc == 0) {
    B.leaves.push_back({g.m, g.n, g.k, {{A, 1.f}}, {{Bv, 1.f}}, {{C, 1.f, kOutAtomic}}});
  } else {
    B.expand({{A, 1.f}}, {{Bv, 1.f}}, {{C, 1.f, kOutAtomic}}, mc, kc, nc, depth);
    if (kc < g.k)
      B.leaves.push_back({mc, nc, g.k - kc, {{{A.p + (long long)kc * A.ld, A.ld, A.bstride}, 1.f}},
                          {{{Bv.p + kc, Bv.ld, Bv.bstride}, 1.f}}, {{C, 1.f, kOutAtomic}}});
    if (mc < g.m)
      B.leaves.push_back({g.m - mc, g.n, g.k, {{{A.p + mc, A.ld, A.bstride}, 1.f}}, {{Bv, 1.f}},
                          {{{C.p + mc, C.ld, C.bstride}, 1.f, kOutAtomic}}});
    if (nc < g.n)
      B.leaves.push_back({mc, g.n - nc, g.k, {{A, 1.f}},
                          {{{Bv.p + (long long)nc * Bv.ld, Bv.ld, Bv.bstride}, 1.f}},
                          {{{C.p + (long long)nc * C.ld, C.ld, C.bstride}, 1.f, kOutAtomic}}});
  }
  // Last, so every leaf (peeling strips included) gets its prepared operands.
  if (leaf_operands) {
    B.prepare_leaf_operands(prep_row_align());
    B.defer_decode();
  }
}

// Workspace elements per batch entry (dry run with a fake base).
size_t plan_workspace_elements(GemmDesc g, bool leaf_operands = false) {
  static float fake;
  Builder B;
  g.a = g.b = &fake;
  g.c = &fake;
  build_plan(g, reinterpret_cast<float*>(uintptr_t(1) << 44), 0, B, leaf_operands);
  return B.ws_used;
}

// Whether math mode `mode` wants prepared leaf operands for `g`: the 3xTF32
// mode and every leaf long enough for the tensor path.
bool leaf_materialisation_wanted(GemmDesc g, int mode) {
  if (mode != BAG_MATH_3XTF32) return false;
  static float fake;
  Builder B;
  g.a = g.b = &fake;
  g.c = &fake;
  build_plan(g, reinterpret_cast<float*>(uintptr_t(1) << 44), 0, B);
  if (B.leaves.empty()) return false;
  for (const HostLeaf& l : B.leaves)
    if (l.k < kTcMinK) return false;
  return true;
}

// Tile configuration: the warp-specialised kernel where every product has a
// compiled signature and the grid fills the GPU, else the measured-fastest
// Tall tile, or smaller tiles when the grid cannot fill the GPU.
int signature(const HostLeaf& l, bool vec);

int choose_tile(const std::vector<HostLeaf>& leaves, int sm_count, bool vec) {
  bool all_fast = vec;
  for (const HostLeaf& l : leaves) all_fast = all_fast && signature(l, vec) != kSigGeneric;
  auto tiles_for = [&](int cfg) {
    const TileShape t = leaf_tile_shape(cfg);
    long long tiles = 0;
    for (const HostLeaf& l : leaves)
      tiles += (long long)((l.m + t.bm - 1) / t.bm) * ((l.n + t.bn - 1) / t.bn);
    return tiles;
  };
  if (all_fast && tiles_for(kTileWS) >= sm_count) return kTileWS;
  if (tiles_for(kTileTall) >= 2LL * sm_count) return kTileTall;
  if (tiles_for(kTileLarge) >= 2LL * sm_count) return kTileLarge;
  return tiles_for(kTileSmall) >= 2LL * sm_count ? kTileSmall : kTileMicro;
}

// The compiled main loop for a product (kSigGeneric when none applies).
int signature(const HostLeaf& l, bool vec) {
  if (!vec || l.m < 4 || l.m % 4 || l.k % 4) return kSigGeneric;
  for (const STerm& t : l.left)
    if (t.v.ld != l.left[0].v.ld) return kSigGeneric;
  for (const STerm& t : l.right)
    if (t.v.ld != l.right[0].v.ld) return kSigGeneric;
  const size_t nl = l.left.size(), nr = l.right.size();
  if (nl == 1 && nr == 1) return kSig11;
  if (nl == 1 && nr == 2) return kSig12;
  if (nl == 2 && nr == 1) return kSig21;
  if (nl == 2 && nr == 2) return kSig22;
  if (nl == 3 && nr == 3) return kSig33;
  if (nl == 4 && nr == 1) return kSig41;
  if (nl == 1 && nr == 4) return kSig14;
  return kSigGeneric;
}

void check_ld(long long ld) {
  if (ld <= 0 || ld > INT32_MAX) fail(BAG_ERR_INVALID, "leading dimension out of range");
}

Term make_term(const View& v, float coef, int mode) {
  check_ld(v.ld);
  Term t{};
  t.p = v.p;
  t.bstride = v.bstride;
  t.ld = int(v.ld);
  t.coef = coef;
  t.mode = mode;
  return t;
}

bool view_vec_ok(const View& v) { return aligned16(v.p) && v.ld % 4 == 0 && v.bstride % 4 == 0; }

// 3xTF32 leaf products on prepared operands: the prepare pass, then the leaf
// launches -- 256 x 128 tiles on clusters of two SMs where the device
// schedules them, else 128 x 256 tiles on one SM (BAG_B200_PREP_KERNEL=single
// selects the latter for comparisons).
int prep_leaf_kind() {
  const char* env = std::getenv("BAG_B200_PREP_KERNEL");
  if (env && std::strcmp(env, "single") == 0) return kPrepLeafSingle;
  return prep_pair_supported() ? kPrepLeafPair : kPrepLeafSingle;
}

// The prepare pass's launches: up to kMaxTreeGroups tree groups each.
std::vector<PrepTreePlan> tree_plans(const Builder& B) {
  static_assert(kPrepTreeK <= 64 && 64 % kPrepTreeK == 0, "rows are padded to 64 k");
  const std::vector<Builder::TreeGroupHost>& groups = B.trees;
  std::vector<PrepTreePlan> plans;
  for (size_t g0 = 0; g0 < groups.size(); g0 += kMaxTreeGroups) {
    plans.emplace_back();
    PrepTreePlan& pp = plans.back();
    std::memset(&pp, 0, sizeof(pp));
    pp.row_len = B.prep_row_len;
    pp.region = const_cast<float*>(B.prep_region.p);
    pp.region_bstride = B.ws_bstride;
    long long tiles = 0;
    for (size_t gi = g0; gi < std::min(groups.size(), g0 + kMaxTreeGroups); ++gi) {
      const Builder::TreeGroupHost& hg = groups[gi];
      TreeGroup& G = pp.group[pp.ngroups++];
      G.rows = hg.rows;
      G.cols = hg.cols;
      G.transpose = hg.transpose ? 1 : 0;
      G.nin = int(hg.in.size());
      for (int u = 0; u < G.nin; ++u) G.in[u] = make_term(hg.in[u], 1.f, 0);
      G.nseg = int(hg.segs.size());
      for (int sg = 0; sg < G.nseg; ++sg) {
        const Builder::TreeSegHost& hs = hg.segs[sg];
        TreeSeg& S = G.seg[sg];
        S.nmid = int(hs.mids.size());
        for (int i = 0; i < S.nmid; ++i)
          for (size_t q = 0; q < hs.mids[i].size(); ++q)
            S.mid[i][q] = static_cast<signed char>(hg.input_code(hs.mids[i][q]));
        S.nout = int(hs.ops.size());
        for (int o = 0; o < S.nout; ++o) {
          S.out_hi[o] = B.prep[hs.ops[o]].hi_row;
          for (size_t q = 0; q < hs.expr[o].size(); ++q)
            S.expr[o][q] = static_cast<signed char>(hs.expr[o][q]);
        }
      }
      G.tile_begin = tiles;
      tiles += (long long)((hg.rows + kPrepTreeRows - 1) / kPrepTreeRows) *
               (B.prep_row_len / kPrepTreeK);
    }
    pp.ntiles = tiles;
    if (tiles > INT32_MAX) fail(BAG_ERR_SHAPE, "problem too large");
  }
  return plans;
}

void run_prepared(Builder& B, int batch, cudaStream_t stream) {
  for (PrepTreePlan& pp : tree_plans(B)) {
    cuda_check(launch_prep_tree(pp, batch, stream), "prepare launch");
    ++g_launches;
  }
  if (g_prof_start) cuda_check(cudaEventRecord(g_prof_start, stream), "cudaEventRecord");
  const int kind = prep_leaf_kind();
  g_last_prep_kind = kind;
  const TileShape ts = prep_tile_shape(kind);
  size_t i = 0;
  while (i < B.leaves.size()) {
    PrepLeafPlan lp;
    lp.nprod = 0;
    lp.ntiles = 0;
    int nouts = 0;
    while (i < B.leaves.size() && lp.nprod < kMaxProducts) {
      const HostLeaf& l = B.leaves[i];
      if (nouts + int(l.out.size()) > kMaxTerms) break;
      PrepProd& P = lp.prod[lp.nprod];
      P.m = l.m;
      P.n = l.n;
      P.k = l.k;
      P.tiles_m = (l.m + ts.bm - 1) / ts.bm;
      P.tiles_n = (l.n + ts.bn - 1) / ts.bn;
      P.tile_begin = lp.ntiles;
      if (l.prep_l < 0 || l.prep_r < 0 || l.prep_l >= int(B.prep.size()) ||
          l.prep_r >= int(B.prep.size()))
        fail(BAG_ERR_INTERNAL, "leaf without prepared operands");
      const Builder::PrepOp& L = B.prep[l.prep_l];
      const Builder::PrepOp& R = B.prep[l.prep_r];
      P.a_hi = L.hi_row;
      P.a_lo = L.hi_row + L.rows;
      P.b_hi = R.hi_row;
      P.b_lo = R.hi_row + R.rows;
      P.o0 = short(nouts);
      P.no = short(l.out.size());
      for (const Target& t : l.out) lp.outs[nouts++] = make_term(t.v, t.coef, t.mode);
      const long long tiles = (long long)P.tiles_m * P.tiles_n;
      if (tiles > 0) {
        if ((long long)lp.ntiles + tiles > INT32_MAX) fail(BAG_ERR_SHAPE, "problem too large");
        lp.ntiles += int(tiles);
        ++lp.nprod;
      }
      ++i;
    }
    if (lp.nprod == 0 && i < B.leaves.size()) fail(BAG_ERR_INTERNAL, "plan chunking failed");
    cuda_check(launch_leaf_prep(lp, kind, B.prep_region.p, B.prep_row_len, B.prep_rows,
                                B.ws_bstride, batch, stream),
               "prepared leaf launch");
    if (lp.nprod) ++g_launches;
  }
  if (g_prof_end) cuda_check(cudaEventRecord(g_prof_end, stream), "cudaEventRecord");
  if (B.decode.on) {
    const Builder::Decode& d = B.decode;
    DecodePlan dp;
    std::memset(&dp, 0, sizeof(dp));
    dp.np = int(d.buffers.size());
    dp.nt = int(d.targets.size());
    dp.accumulate = d.overwrite ? 0 : 1;
    dp.m = d.m;
    dp.n = d.n;
    for (int p = 0; p < dp.np; ++p) {
      dp.in[p] = make_term(d.buffers[p], 1.f, 0);
      for (const auto& tc : d.terms[p]) {
        const int t = tc.first;
        dp.list[t][dp.count[t]++] = static_cast<signed char>(tc.second > 0 ? p + 1 : -(p + 1));
      }
    }
    for (int t = 0; t < dp.nt; ++t) dp.out[t] = make_term(d.targets[t], 1.f, 0);
    cuda_check(launch_decode(dp, batch, stream), "decode launch");
    ++g_launches;
  }
}

// FFMA leaves longer than kFfmaChainSplitK are split along K into chains of
// at most kFfmaChainK that add into the same C blocks (atomically), so no
// output is a sequential fmaf chain longer than 4096.  A chain's rounding
// error grows with its length; the reference's own leaves at the benchmark's
// square sizes are 2048-4096 long, and a rectangular problem with a long K
// (e.g. 8192 x 16384 x 4096 at one level: K = 8192 per leaf), which the
// reference can only run as square calls on sub-blocks (leaf K = 2048, the
// partial results added into C), then gets that composition's error.  Only
// leaves whose every output is atomic are split (plain-store and single-writer
// outputs of bag_primitive keep one chain).
constexpr int kFfmaChainSplitK = 4096;
constexpr int kFfmaChainK = 2048;

void split_long_chains(std::vector<HostLeaf>& leaves) {
  std::vector<HostLeaf> out;
  out.reserve(leaves.size());
  for (HostLeaf& l : leaves) {
    bool atomic = true;
    for (const Target& t : l.out) atomic = atomic && t.mode == kOutAtomic;
    if (l.k <= kFfmaChainSplitK || !atomic) {
      out.push_back(std::move(l));
      continue;
    }
    const int chunks = (l.k + kFfmaChainK - 1) / kFfmaChainK;
    const int step = (l.k / chunks + 3) / 4 * 4;   // multiples of 4 keep 16-byte offsets
    for (int k0 = 0; k0 < l.k; k0 += step) {
      HostLeaf c;
      c.m = l.m;
      c.n = l.n;
      c.k = std::min(step, l.k - k0);
      c.out = l.out;
      // Left operands are column-major m x k (column offset), right ones k x n
      // (row offset).
      for (const STerm& t : l.left)
        c.left.push_back({{t.v.p + (long long)k0 * t.v.ld, t.v.ld, t.v.bstride}, t.coef});
      for (const STerm& t : l.right)
        c.right.push_back({{t.v.p + k0, t.v.ld, t.v.bstride}, t.coef});
      out.push_back(std::move(c));
    }
  }
  leaves.swap(out);
}

// `sources` lists the whole operand matrices (A, B) the tensor-core path may
// address blocks of through one tensor map each; may be empty.
void execute_plan(Builder& B, int batch, cudaStream_t stream,
                  const std::vector<TcSource>& sources = {}) {
  const int sms = sm_count_for_current_device();
  // Materialisation stages.
  for (const auto& jobs : B.stages) {
    for (size_t j0 = 0; j0 < jobs.size(); j0 += kMaxJobs) {
      MatPlan mp{};
      long long chunks = 0;
      for (size_t j = j0; j < std::min(jobs.size(), j0 + kMaxJobs); ++j) {
        const HostJob& hj = jobs[j];
        MatJob& J = mp.job[mp.njobs];
        J.rows = hj.rows;
        J.cols = hj.cols;
        J.nin = int(hj.in.size());
        J.nout = int(hj.out.size());
        for (int i = 0; i < J.nin; ++i) J.in[i] = make_term(hj.in[i], 1.f, 0);
        for (int o = 0; o < J.nout; ++o) {
          J.out[o] = make_term(hj.out[o], 1.f, 0);
          for (size_t t = 0; t < hj.expr[o].size(); ++t) J.expr[o][t] = (signed char)hj.expr[o][t];
        }
        mp.chunk_begin[mp.njobs] = chunks;
        chunks += (long long)((hj.rows + 3) / 4) * hj.cols;
        ++mp.njobs;
      }
      mp.chunk_begin[mp.njobs] = chunks;
      cuda_check(launch_materialize(mp, batch, stream, sms), "materialize launch");
      ++g_launches;
    }
  }
  record_phase(g_phase_stages, stream);
  // Leaf products, grouped into as few launches as the parameter block allows.
  bool vec = true;
  for (const HostLeaf& l : B.leaves) {
    for (const STerm& t : l.left) vec = vec && view_vec_ok(t.v);
    for (const STerm& t : l.right) vec = vec && view_vec_ok(t.v);
    for (const Target& t : l.out) vec = vec && view_vec_ok(t.v);
  }
  // The tensor paths read operands by TMA, so they need aligned operands
  // (vec) but no common leading dimension among a product's terms.
  bool tensor = g_math_mode == BAG_MATH_3XTF32 && vec;
  for (const HostLeaf& l : B.leaves) tensor = tensor && l.k >= kTcMinK;
  g_last_prep_kind = -1;
  if (!B.prep.empty()) {
    // A prepared plan's deepest operands may be virtual: it runs only here.
    if (!(tensor && prep_supported()))
      fail(BAG_ERR_INTERNAL, "a prepared-operand plan cannot take the prepared path");
    g_last_leaf_path = BAG_MATH_3XTF32;
    run_prepared(B, batch, stream);
    record_phase(g_phase_done, stream);
    return;
  }
  for (const HostLeaf& l : B.leaves)
    tensor = tensor && tc_supported(int(l.left.size()), int(l.right.size()));
  if (!tensor) split_long_chains(B.leaves);
  bool all_fast = vec;
  for (const HostLeaf& l : B.leaves) all_fast = all_fast && signature(l, vec) != kSigGeneric;
  g_last_leaf_path = tensor ? BAG_MATH_3XTF32 : BAG_MATH_FFMA;
  if (g_prof_start) cuda_check(cudaEventRecord(g_prof_start, stream), "cudaEventRecord");
  const int cfg = tensor ? -1 : choose_tile(B.leaves, sms, vec);
  const TileShape ts = tensor ? tc_tile_shape() : leaf_tile_shape(cfg);
  size_t i = 0;
  while (i < B.leaves.size()) {
    LeafPlan lp;
    lp.nprod = 0;
    lp.ntiles = 0;
    int nterms = 0;
    while (i < B.leaves.size() && lp.nprod < kMaxProducts) {
      const HostLeaf& l = B.leaves[i];
      const int need = int(l.left.size() + l.right.size() + l.out.size());
      if (nterms + need > kMaxTerms) break;
      if ((int)l.left.size() > kMaxOperandTerms || (int)l.right.size() > kMaxOperandTerms)
        fail(BAG_ERR_INTERNAL, "operand has more fused terms than the kernel takes");
      Prod& P = lp.prod[lp.nprod];
      P.m = l.m;
      P.n = l.n;
      P.k = l.k;
      P.tiles_m = (l.m + ts.bm - 1) / ts.bm;
      P.tiles_n = (l.n + ts.bn - 1) / ts.bn;
      P.tile_begin = lp.ntiles;
      P.l0 = short(nterms);
      P.nl = short(l.left.size());
      for (const STerm& t : l.left) lp.terms[nterms++] = make_term(t.v, t.coef, 0);
      P.r0 = short(nterms);
      P.nr = short(l.right.size());
      for (const STerm& t : l.right) lp.terms[nterms++] = make_term(t.v, t.coef, 0);
      P.o0 = short(nterms);
      P.no = short(l.out.size());
      for (const Target& t : l.out) lp.terms[nterms++] = make_term(t.v, t.coef, t.mode);
      P.sig = signature(l, vec);
      const long long tiles = (long long)P.tiles_m * P.tiles_n;
      if (tiles > 0) {
        if ((long long)lp.ntiles + tiles > INT32_MAX) fail(BAG_ERR_SHAPE, "problem too large");
        lp.ntiles += int(tiles);
        ++lp.nprod;
      }
      ++i;
    }
    if (lp.nprod == 0 && i < B.leaves.size()) fail(BAG_ERR_INTERNAL, "plan chunking failed");
    cuda_check(tensor ? launch_leaf_tc(lp, sources.data(), int(sources.size()), batch, stream)
                      : launch_leaf(lp, cfg, vec, batch, stream),
               "leaf launch");
    if (lp.nprod) ++g_launches;
  }
  if (g_prof_end) cuda_check(cudaEventRecord(g_prof_end, stream), "cudaEventRecord");
  record_phase(g_phase_done, stream);
}

void record_phase(cudaEvent_t ev, cudaStream_t stream) {
  if (ev) cuda_check(cudaEventRecord(ev, stream), "cudaEventRecord");
}

void check_device_workspace(const bag_workspace* ws) {
  int dev = 0;
  cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
  if (ws->device != dev) fail(BAG_ERR_WORKSPACE, "workspace belongs to another device");
}

// Plans of recent calls, per host thread.  A plan holds absolute addresses
// and depends on nothing but the key's fields (the problem with every pointer,
// leading dimension and stride, beta, the math mode, the workspace and its
// size, the device), so a call equal in all of them reuses the plan as it was
// built and skips the two or three host-side builds.  Executing a plan leaves
// it unchanged (splitting long FFMA chains is idempotent).  A freed and
// reallocated buffer at the same address is the same operand to a plan.
struct PlanKey {
  GemmDesc g;
  float beta;
  int mode;
  const bag_workspace* ws;
  const float* ws_data;
  size_t ws_elements;
  int device;
  bool operator==(const PlanKey& o) const {
    return g.m == o.g.m && g.n == o.g.n && g.k == o.g.k && g.a == o.g.a && g.lda == o.g.lda &&
           g.sa == o.g.sa && g.b == o.g.b && g.ldb == o.g.ldb && g.sb == o.g.sb && g.c == o.g.c &&
           g.ldc == o.g.ldc && g.sc == o.g.sc && g.batch == o.g.batch && g.depth == o.g.depth &&
           g.basis == o.g.basis && beta == o.beta && mode == o.mode && ws == o.ws &&
           ws_data == o.ws_data && ws_elements == o.ws_elements && device == o.device;
  }
};
constexpr size_t kPlanCacheSize = 8;
struct CachedPlan {
  PlanKey key;
  Builder plan;
};
thread_local std::vector<CachedPlan> g_plan_cache;   // most recent last

Builder* cached_plan(const PlanKey& key) {
  for (size_t i = g_plan_cache.size(); i-- > 0;) {
    if (g_plan_cache[i].key == key) {
      if (i + 1 != g_plan_cache.size()) std::swap(g_plan_cache[i], g_plan_cache.back());
      return &g_plan_cache.back().plan;
    }
  }
  return nullptr;
}

void remember_plan(const PlanKey& key, Builder&& plan) {
  if (g_plan_cache.size() == kPlanCacheSize) g_plan_cache.erase(g_plan_cache.begin());
  g_plan_cache.push_back(CachedPlan{key, std::move(plan)});
}

void run_gemm(GemmDesc g, float beta, cudaStream_t stream, bag_workspace* ws) {
  if (g.m < 0 || g.n < 0 || g.k < 0) fail(BAG_ERR_SHAPE, "negative extent");
  g.depth = resolve_depth(g.depth, g.m, g.n, g.k);
  if (g.depth < 0 || g.depth > 8) fail(BAG_ERR_INVALID, "depth must be 0..8 or BAG_DEPTH_AUTO");
  if (!known_basis(g.basis)) fail(BAG_ERR_INVALID, "unknown basis");
  if (beta != 0.f && beta != 1.f) fail(BAG_ERR_UNSUPPORTED, "beta must be 0 or 1");
  if (g.batch < 0) fail(BAG_ERR_INVALID, "negative batch");
  if (g.m == 0 || g.n == 0 || g.batch == 0) return;
  if (!g.a || !g.b || !g.c) fail(BAG_ERR_INVALID, "null matrix pointer");
  if (g.lda < std::max(1, g.m) || g.ldb < std::max(1, g.k) || g.ldc < std::max(1, g.m))
    fail(BAG_ERR_INVALID, "leading dimension smaller than the row count");
  auto zero_c = [&] {
    for (int i = 0; i < g.batch; ++i)
      cuda_check(cudaMemset2DAsync(g.c + (long long)i * g.sc, size_t(g.ldc) * sizeof(float), 0,
                                   size_t(g.m) * sizeof(float), size_t(g.n), stream),
                 "cudaMemset2DAsync");
  };
  if (g.k == 0) {
    if (beta == 0.f) zero_c();
    return;
  }
  const std::vector<TcSource> sources = {{g.a, g.lda, g.sa, g.m, g.k}, {g.b, g.ldb, g.sb, g.k, g.n}};
  int device = 0;
  cuda_check(cudaGetDevice(&device), "cudaGetDevice");
  PlanKey key{g, beta, g_math_mode, ws, ws ? ws->data : nullptr, ws ? ws->elements : 0, device};
  if (Builder* hit = cached_plan(key)) {
    if (ws) check_device_workspace(ws);
    if (beta == 0.f && !hit->decode.on) zero_c();
    execute_plan(*hit, g.batch, stream, sources);
    return;
  }
  // 3xTF32 mode prepares the leaf operands when the workspace was sized for
  // it (created in that mode) and the prepared path can run (TMA available,
  // 16-byte-aligned matrices); otherwise the prologue stays fused.
  const bool aligned = aligned16(g.a) && aligned16(g.b) && aligned16(g.c) && g.lda % 4 == 0 &&
                       g.ldb % 4 == 0 && g.ldc % 4 == 0 && g.sa % 4 == 0 && g.sb % 4 == 0 &&
                       g.sc % 4 == 0;
  bool leaf_operands = aligned && leaf_materialisation_wanted(g, g_math_mode) && prep_supported();
  size_t need = plan_workspace_elements(g, leaf_operands);
  if (leaf_operands && (!ws || need * size_t(g.batch) > ws->elements)) {
    leaf_operands = false;
    need = plan_workspace_elements(g);
  }
  float* base = nullptr;
  if (need) {
    if (!ws) fail(BAG_ERR_WORKSPACE, "this plan needs a workspace");
    check_device_workspace(ws);
    if (need * size_t(g.batch) > ws->elements)
      fail(BAG_ERR_WORKSPACE, "workspace too small for this problem");
    base = ws->data;
  }
  Builder B;
  build_plan(g, base ? base : reinterpret_cast<float*>(uintptr_t(1) << 44), (long long)need, B,
             leaf_operands);
  if (B.ws_used != need) fail(BAG_ERR_INTERNAL, "plan size changed between passes");
  // With the deferred decode every C block is written once by the decode
  // pass (no peeled strips: all leaves share one shape), so C = A B needs no
  // zeroing -- the pass overwrites instead of accumulating.
  if (beta == 0.f) {
    if (B.decode.on) B.decode.overwrite = true;
    else zero_c();
  }
  execute_plan(B, g.batch, stream, sources);
  remember_plan(key, std::move(B));
}

GemmDesc make_desc(int layout, int m, int n, int k, const float* a, long long lda, long long sa,
                   const float* b, long long ldb, long long sb, float* c, long long ldc,
                   long long sc, int batch, int depth, int basis) {
  if (layout != BAG_LAYOUT_COL_MAJOR && layout != BAG_LAYOUT_ROW_MAJOR)
    fail(BAG_ERR_INVALID, "unknown layout");
  GemmDesc g{};
  if (layout == BAG_LAYOUT_COL_MAJOR) {
    g = {m, n, k, a, lda, sa, b, ldb, sb, c, ldc, sc, batch, depth, basis};
  } else {
    // Row-major C = A B is column-major C^T = B^T A^T: swap the operands.
    g = {n, m, k, b, ldb, sb, a, lda, sa, c, ldc, sc, batch, depth, basis};
  }
  return g;
}

bool valid_shape_impl(int backend, int s) {
  if (s <= 0 || s % 4) return false;
  switch (backend) {
    case BAG_BACKEND_LEGACY:
      return s % ((s <= 384) ? 16 : (s <= 1024 && s != 1024) ? 32 : (s <= 4096) ? 64 : 128) == 0;
    case BAG_BACKEND_LARGE: return s % 64 == 0;
    case BAG_BACKEND_MEDIUM: return s % 32 == 0;
    case BAG_BACKEND_HUGE: return s % 128 == 0;
    default: return true;
  }
}

bool paired_backend(int backend) {
  return backend == BAG_BACKEND_COLUMN_TILE8 || backend == BAG_BACKEND_HUGE ||
         backend == BAG_BACKEND_PIPE64X32 || backend == BAG_BACKEND_DEFERRED_SWIZZLE64;
}

void check_backend(int backend) {
  if (backend < 0 || backend >= BAG_BACKEND_COUNT) fail(BAG_ERR_INVALID, "unknown backend");
}

size_t local_elements_impl(int n, int depth, int basis) {
  if (depth < 1) fail(BAG_ERR_SHAPE, "BAG depth must be positive");
  int size = n;
  for (int level = 0; level < depth; ++level, size /= 2)
    if (size <= 0 || size % 8) fail(BAG_ERR_SHAPE, "each BAG level requires N divisible by 8");
  const size_t count = size_t(n) * n;
  return basis == BAG_BASIS_FULL ? 3 * count : count + count / 2;
}

template <class F>
bag_status guarded(F&& f) {
  try {
    f();
    return BAG_OK;
  } catch (const Error& e) {
    g_last_error = e.what();
    return e.status;
  } catch (const std::exception& e) {
    g_last_error = e.what();
    return BAG_ERR_INTERNAL;
  } catch (...) {
    g_last_error = "unknown error";
    return BAG_ERR_INTERNAL;
  }
}

// JSON dump of a plan built against fake, far-apart base pointers.
std::string dump_plan(int m, int n, int k, long long lda, long long ldb, long long ldc, int depth,
                      int basis) {
  const uintptr_t unit = uintptr_t(1) << 40;
  GemmDesc g{m, n, k, reinterpret_cast<const float*>(unit), lda, 0,
             reinterpret_cast<const float*>(2 * unit), ldb, 0,
             reinterpret_cast<float*>(3 * unit), ldc, 0, 1, depth, basis};
  Builder B;
  // In 3xTF32 mode the plan also lists the prepared (TF32 hi/lo) operands.
  build_plan(g, reinterpret_cast<float*>(4 * unit), 0, B, leaf_materialisation_wanted(g, g_math_mode));
  auto ref = [&](const View& v) {
    if (B.vbuf_of(v)) {   // a virtual block (prepared path): buffer id 4
      const long long off = (long long)((reinterpret_cast<uintptr_t>(v.p) - (uintptr_t(1) << 50)) /
                                        sizeof(float));
      return "[4," + std::to_string(off) + "," + std::to_string(v.ld) + "]";
    }
    const uintptr_t p = reinterpret_cast<uintptr_t>(v.p);
    const uintptr_t base = p / unit;
    const long long off = (long long)((p - base * unit) / sizeof(float));
    return "[" + std::to_string(int(base) - 1) + "," + std::to_string(off) + "," +
           std::to_string(v.ld) + "]";
  };
  std::string s = "{\"workspace_elements\":" + std::to_string(B.ws_used) + ",\"stages\":[";
  for (size_t si = 0; si < B.stages.size(); ++si) {
    s += si ? ",[" : "[";
    for (size_t j = 0; j < B.stages[si].size(); ++j) {
      const HostJob& hj = B.stages[si][j];
      s += j ? "," : "";
      s += "{\"rows\":" + std::to_string(hj.rows) + ",\"cols\":" + std::to_string(hj.cols) +
           ",\"in\":[";
      for (size_t i = 0; i < hj.in.size(); ++i) s += (i ? "," : "") + ref(hj.in[i]);
      s += "],\"out\":[";
      for (size_t o = 0; o < hj.out.size(); ++o) s += (o ? "," : "") + ref(hj.out[o]);
      s += "],\"expr\":[";
      for (size_t o = 0; o < hj.expr.size(); ++o) {
        s += o ? ",[" : "[";
        for (size_t t = 0; t < hj.expr[o].size(); ++t)
          s += (t ? "," : "") + std::to_string(hj.expr[o][t]);
        s += "]";
      }
      s += "]}";
    }
    s += "]";
  }
  s += "],\"leaves\":[";
  for (size_t i = 0; i < B.leaves.size(); ++i) {
    const HostLeaf& l = B.leaves[i];
    s += i ? "," : "";
    s += "{\"m\":" + std::to_string(l.m) + ",\"n\":" + std::to_string(l.n) +
         ",\"k\":" + std::to_string(l.k) + ",\"left\":[";
    for (size_t t = 0; t < l.left.size(); ++t)
      s += std::string(t ? "," : "") + "[" + ref(l.left[t].v) + "," +
           std::to_string(int(l.left[t].coef)) + "]";
    s += "],\"right\":[";
    for (size_t t = 0; t < l.right.size(); ++t)
      s += std::string(t ? "," : "") + "[" + ref(l.right[t].v) + "," +
           std::to_string(int(l.right[t].coef)) + "]";
    s += "],\"out\":[";
    for (size_t t = 0; t < l.out.size(); ++t)
      s += std::string(t ? "," : "") + "[" + ref(l.out[t].v) + "," +
           std::to_string(int(l.out[t].coef)) + "]";
    s += "],\"prep_l\":" + std::to_string(l.prep_l) + ",\"prep_r\":" + std::to_string(l.prep_r) +
         "}";
  }
  // Deferred decode: target t of C = its old value + sum over products p (in
  // plan order) of coef * buffer p, where terms[p] lists (t, coef).
  const Builder::Decode& d = B.decode;
  s += "],\"decode\":{\"deferred\":" + std::string(d.on ? "true" : "false") +
       ",\"products\":" + std::to_string(d.buffers.size()) + ",\"targets\":" +
       std::to_string(d.targets.size()) + ",\"m\":" + std::to_string(d.m) +
       ",\"n\":" + std::to_string(d.n) + ",\"target_refs\":[";
  for (size_t t = 0; t < d.targets.size(); ++t) s += (t ? "," : "") + ref(d.targets[t]);
  s += "],\"buffers\":[";
  for (size_t p = 0; p < d.buffers.size(); ++p) s += (p ? "," : "") + ref(d.buffers[p]);
  s += "],\"terms\":[";
  for (size_t p = 0; p < d.terms.size(); ++p) {
    s += p ? ",[" : "[";
    for (size_t e = 0; e < d.terms[p].size(); ++e)
      s += std::string(e ? "," : "") + "[" + std::to_string(d.terms[p][e].first) + "," +
           std::to_string(int(d.terms[p][e].second)) + "]";
    s += "]";
  }
  // Tree groups: inputs (blocks), then per segment its mids (codes over the
  // inputs), its operands (indices into "prepared") and their codes over the
  // segment's mids.
  s += "]},\"prep_groups\":[";
  auto codes = [](const std::vector<int>& c) {
    std::string r = "[";
    for (size_t t = 0; t < c.size(); ++t) r += (t ? "," : "") + std::to_string(c[t]);
    return r + "]";
  };
  for (size_t gi = 0; gi < B.trees.size(); ++gi) {
    const Builder::TreeGroupHost& g = B.trees[gi];
    s += gi ? "," : "";
    s += "{\"rows\":" + std::to_string(g.rows) + ",\"cols\":" + std::to_string(g.cols) +
         ",\"transpose\":" + std::string(g.transpose ? "true" : "false") + ",\"in\":[";
    for (size_t u = 0; u < g.in.size(); ++u) s += (u ? "," : "") + ref(g.in[u]);
    s += "],\"segs\":[";
    for (size_t sg = 0; sg < g.segs.size(); ++sg) {
      const Builder::TreeSegHost& hs = g.segs[sg];
      s += sg ? ",{\"mids\":[" : "{\"mids\":[";
      for (size_t i = 0; i < hs.mids.size(); ++i) {
        std::vector<int> c;
        for (const STerm& t : hs.mids[i]) c.push_back(g.input_code(t));
        s += (i ? "," : "") + codes(c);
      }
      s += "],\"ops\":" + codes(hs.ops) + ",\"expr\":[";
      for (size_t o = 0; o < hs.expr.size(); ++o) s += (o ? "," : "") + codes(hs.expr[o]);
      s += "]}";
    }
    s += "]}";
  }
  s += "]";
  // Virtual blocks (prepared path): what a materialisation job would have
  // written, for checkers that evaluate the leaf operands the long way.
  s += ",\"virtual\":[";
  for (size_t i = 0; i < B.vbufs.size(); ++i) {
    const Builder::VBuf& vb = B.vbufs[i];
    s += (i ? ",{\"out\":" : "{\"out\":") + ref({vb.begin, vb.ld, 0}) +
         ",\"rows\":" + std::to_string(vb.rows) + ",\"cols\":" + std::to_string(vb.cols) +
         ",\"terms\":[";
    for (size_t t = 0; t < vb.def.size(); ++t)
      s += std::string(t ? "," : "") + "[" + ref(vb.def[t].v) + "," +
           std::to_string(int(vb.def[t].coef)) + "]";
    s += "]}";
  }
  s += "]";
  // Per prepare launch: the compiled-in basis tables its kernel would use
  // (1 Minimal .. 4 Winograd, 0 none) and which of its groups take them --
  // computed by the function the launcher calls.
  s += ",\"prepare_tables\":[";
  if (!B.trees.empty()) {
    std::vector<PrepTreePlan> plans = tree_plans(B);
    for (size_t i = 0; i < plans.size(); ++i) {
      const int p = mark_tree_tables(plans[i]);
      s += std::string(i ? "," : "") + "{\"basis_tables\":" + std::to_string(p) + ",\"groups\":[";
      for (int gi = 0; gi < plans[i].ngroups; ++gi)
        s += std::string(gi ? "," : "") + std::to_string(plans[i].group[gi].table);
      s += "]}";
    }
  }
  s += "]";
  s += ",\"prepared_region\":" + (B.prep_region.p ? ref(B.prep_region) : std::string("null"));
  s += ",\"prepared_row_len\":" + std::to_string(B.prep_row_len) + ",\"prepared\":[";
  for (size_t i = 0; i < B.prep.size(); ++i) {
    const Builder::PrepOp& o = B.prep[i];
    s += i ? "," : "";
    s += "{\"rows\":" + std::to_string(o.rows) + ",\"cols\":" + std::to_string(o.cols) +
         ",\"transpose\":" + std::string(o.transpose ? "true" : "false") +
         ",\"hi_row\":" + std::to_string(o.hi_row) + ",\"terms\":[";
    // [[[block, coef], ...] (a mid), coef] per term
    for (size_t t = 0; t < o.terms.size(); ++t) {
      s += std::string(t ? "," : "") + "[[";
      for (size_t q = 0; q < o.terms[t].first.size(); ++q)
        s += std::string(q ? "," : "") + "[" + ref(o.terms[t].first[q].v) + "," +
             std::to_string(int(o.terms[t].first[q].coef)) + "]";
      s += "]," + std::to_string(int(o.terms[t].second)) + "]";
    }
    s += "]}";
  }
  s += "]}";
  return s;
}

}  // namespace
}  // namespace bag_b200

using namespace bag_b200;

extern "C" {

const char* bag_last_error(void) { return g_last_error.c_str(); }

const char* bag_version(void) { return "bag_b200 0.1.0 (sm_100a)"; }

bag_status bag_local_elements(int n, int depth, int basis, size_t* elements) {
  return guarded([&] {
    if (!elements) fail(BAG_ERR_INVALID, "null output pointer");
    *elements = 0;
    *elements = local_elements_impl(n, depth, basis);
  });
}

bag_status bag_workspace_create_ex(int m, int n, int k, int depth, int basis, int batch,
                                   bag_workspace** out) {
  return guarded([&] {
    if (!out) fail(BAG_ERR_INVALID, "null output pointer");
    *out = nullptr;
    if (m < 0 || n < 0 || k < 0 || batch < 0) fail(BAG_ERR_SHAPE, "negative extent");
    depth = resolve_depth(depth, m, n, k);
    if (depth < 0 || depth > 8) fail(BAG_ERR_INVALID, "depth must be 0..8 or BAG_DEPTH_AUTO");
    if (!known_basis(basis)) fail(BAG_ERR_INVALID, "unknown basis");
    GemmDesc g{m, n, k, nullptr, std::max(1, m), 0, nullptr, std::max(1, k), 0, nullptr,
               std::max(1, m), 0, std::max(batch, 1), depth, basis};
    // Sized for the calling thread's math mode (3xTF32 adds the prepared
    // leaf operands).
    const size_t per = plan_workspace_elements(g, leaf_materialisation_wanted(g, g_math_mode));
    const size_t total = per * size_t(std::max(batch, 1));
    auto* ws = new bag_workspace{m, n, k, depth, basis, batch, 0, nullptr, total};
    cudaError_t e = cudaGetDevice(&ws->device);
    if (e == cudaSuccess && total)
      e = device_alloc(reinterpret_cast<void**>(&ws->data), total * sizeof(float));
    if (e != cudaSuccess) {
      delete ws;
      cuda_check(e, "workspace allocation");
    }
    *out = ws;
  });
}

bag_status bag_workspace_bytes_for(int mode, int m, int n, int k, int depth, int basis, int batch,
                                   size_t* bytes) {
  return guarded([&] {
    if (!bytes) fail(BAG_ERR_INVALID, "null output pointer");
    *bytes = 0;
    if (mode != BAG_MATH_FFMA && mode != BAG_MATH_3XTF32) fail(BAG_ERR_INVALID, "unknown math mode");
    if (m < 0 || n < 0 || k < 0 || batch < 0) fail(BAG_ERR_SHAPE, "negative extent");
    const int saved = g_math_mode;   // resolve_depth reads this thread's mode
    g_math_mode = mode;
    depth = resolve_depth(depth, m, n, k);
    g_math_mode = saved;
    if (depth < 0 || depth > 8) fail(BAG_ERR_INVALID, "depth must be 0..8 or BAG_DEPTH_AUTO");
    if (!known_basis(basis)) fail(BAG_ERR_INVALID, "unknown basis");
    GemmDesc g{m, n, k, nullptr, std::max(1, m), 0, nullptr, std::max(1, k), 0, nullptr,
               std::max(1, m), 0, std::max(batch, 1), depth, basis};
    *bytes = plan_workspace_elements(g, leaf_materialisation_wanted(g, mode)) *
             size_t(std::max(batch, 1)) * sizeof(float);
  });
}

bag_status bag_workspace_create(int n, int depth, int basis, bag_workspace** out) {
  return guarded([&] {
    if (!out) fail(BAG_ERR_INVALID, "null output pointer");
    *out = nullptr;
    if (basis != kMinimal && basis != kFull) fail(BAG_ERR_INVALID, "unknown basis");
    local_elements_impl(n, depth, basis);   // the reference's shape rules (bag.cuh:23-30)
    const bag_status s = bag_workspace_create_ex(n, n, n, depth, basis, 1, out);
    if (s != BAG_OK) fail(s, g_last_error);
  });
}

bag_status bag_workspace_destroy(bag_workspace* ws) {
  return guarded([&] {
    if (!ws) return;
    if (ws->data) cudaFree(ws->data);
    delete ws;
  });
}

size_t bag_workspace_bytes(const bag_workspace* ws) {
  return ws ? ws->elements * sizeof(float) : 0;
}

float* bag_workspace_data(const bag_workspace* ws) { return ws ? ws->data : nullptr; }

bag_status bag_matmul(const float* a, const float* b, float* c, int n, bag_stream_t stream,
                      bag_workspace* ws, int backend, int schedule) {
  return guarded([&] {
    if (!ws) fail(BAG_ERR_WORKSPACE, "null workspace");
    check_backend(backend);
    if (schedule < BAG_SCHEDULE_SERIAL || schedule > BAG_SCHEDULE_BATCHED)
      fail(BAG_ERR_INVALID, "unknown schedule");
    if (n != ws->n || ws->m != ws->n || ws->k != ws->n) fail(BAG_ERR_WORKSPACE, "BAG workspace size mismatch");
    int leaf = n;
    for (int level = 0; level < ws->depth; ++level) leaf /= 2;
    if (!valid_shape_impl(backend, leaf))
      fail(BAG_ERR_SHAPE, "BAG leaf violates backend tile constraints");
    if (schedule == BAG_SCHEDULE_BATCHED && !paired_backend(backend))
      fail(BAG_ERR_UNSUPPORTED, "BAG batched schedule requires a paired backend");
    run_gemm(make_desc(BAG_LAYOUT_COL_MAJOR, n, n, n, a, n, 0, b, n, 0, c, n, 0, 1, ws->depth,
                       ws->basis),
             1.f, reinterpret_cast<cudaStream_t>(stream), ws);
  });
}

bag_status bag_sgemm_ex(int layout, int m, int n, int k, const float* a, long long lda,
                        const float* b, long long ldb, float* c, long long ldc, float beta,
                        int depth, int basis, bag_stream_t stream, bag_workspace* ws) {
  return guarded([&] {
    run_gemm(make_desc(layout, m, n, k, a, lda, 0, b, ldb, 0, c, ldc, 0, 1, depth, basis), beta,
             reinterpret_cast<cudaStream_t>(stream), ws);
  });
}

bag_status bag_sgemm_batched(int layout, int m, int n, int k, const float* a, long long lda,
                             long long stride_a, const float* b, long long ldb, long long stride_b,
                             float* c, long long ldc, long long stride_c, int batch, float beta,
                             int depth, int basis, bag_stream_t stream, bag_workspace* ws) {
  return guarded([&] {
    if (batch > 65535) fail(BAG_ERR_SHAPE, "batch must be at most 65535");
    run_gemm(make_desc(layout, m, n, k, a, lda, stride_a, b, ldb, stride_b, c, ldc, stride_c,
                       batch, depth, basis),
             beta, reinterpret_cast<cudaStream_t>(stream), ws);
  });
}

}  // extern "C"

namespace bag_b200 {
namespace {

void check_coeffs(int delta, int eps, int gd, int ge) {
  if (delta < -1 || delta > 1) fail(BAG_ERR_INVALID, "delta must be -1, 0 or 1");
  if (eps < -1 || eps > 1) fail(BAG_ERR_INVALID, "epsilon must be -1, 0 or 1");
  if (gd < -2 || gd > 2) fail(BAG_ERR_INVALID, "gamma_d must be in -2..2");
  if (ge < -2 || ge > 2) fail(BAG_ERR_INVALID, "gamma_e must be in -2..2");
}

HostLeaf primitive_leaf(int delta, int eps, int gd, int ge, int atomic, const float* x,
                        const float* y, const float* v, const float* w, float* d, float* e, int m,
                        int n, int k, long long ldx, long long ldy, long long ldv, long long ldw,
                        long long ldd, long long lde) {
  HostLeaf l;
  l.m = m;
  l.n = n;
  l.k = k;
  // An empty reduction (k == 0) reads no operand, so they may be null.
  if (k > 0 && (!x || !v)) fail(BAG_ERR_INVALID, "x and v are required");
  if (k > 0 && delta && !y) fail(BAG_ERR_INVALID, "y may be null only when delta == 0");
  if (k > 0 && eps && !w) fail(BAG_ERR_INVALID, "w may be null only when epsilon == 0");
  if (gd && !d) fail(BAG_ERR_INVALID, "d may be null only when gamma_d == 0");
  if (ge && !e) fail(BAG_ERR_INVALID, "e may be null only when gamma_e == 0");
  l.left.push_back({{x, ldx, 0}, 1.f});
  if (delta) l.left.push_back({{y, ldy, 0}, float(delta)});
  l.right.push_back({{v, ldv, 0}, 1.f});
  if (eps) l.right.push_back({{w, ldw, 0}, float(eps)});
  auto mode_of = [&](int g) {
    return (g == 2 || g == -2) ? kOutOverwrite : (atomic ? kOutAtomic : kOutAdd);
  };
  auto coef_of = [](int g) { return g > 0 ? 1.f : -1.f; };
  if (gd) l.out.push_back({{d, ldd, 0}, coef_of(gd), mode_of(gd)});
  if (ge) l.out.push_back({{e, lde, 0}, coef_of(ge), mode_of(ge)});
  return l;
}

void run_leaves(std::vector<HostLeaf> leaves, cudaStream_t stream) {
  Builder B;
  B.leaves = std::move(leaves);
  execute_plan(B, 1, stream);
}

}  // namespace

// Message for bag_last_error() from code outside this file (bag_noalloc.cu).
void set_last_error(const std::string& message) { g_last_error = message; }

// The body of bag_sgemm_noalloc (bag_noalloc.cu): the same call as
// bag_sgemm_ex, with a caller-provided device scratch region of
// `scratch_elements` floats standing in for a workspace.  Problems whose plan
// needs more scratch than that are rejected before anything is enqueued.
bag_status sgemm_with_scratch(int layout, int m, int n, int k, const float* a, long long lda,
                              const float* b, long long ldb, float* c, long long ldc, float beta,
                              int depth, int basis, cudaStream_t stream, float* scratch,
                              size_t scratch_elements) {
  return guarded([&] {
    GemmDesc g = make_desc(layout, m, n, k, a, lda, 0, b, ldb, 0, c, ldc, 0, 1, depth, basis);
    if (g.m < 0 || g.n < 0 || g.k < 0) fail(BAG_ERR_SHAPE, "negative extent");
    g.depth = resolve_depth(g.depth, g.m, g.n, g.k);
    if (g.depth < 0 || g.depth > 8) fail(BAG_ERR_INVALID, "depth must be 0..8 or BAG_DEPTH_AUTO");
    if (!known_basis(g.basis)) fail(BAG_ERR_INVALID, "unknown basis");
    const size_t need = (g.m > 0 && g.n > 0 && g.k > 0) ? plan_workspace_elements(g) : 0;
    if (need > scratch_elements)
      fail(BAG_ERR_WORKSPACE,
           "bag_sgemm_noalloc: this problem needs " + std::to_string(need) +
               " floats of scratch but the built-in scratch holds " +
               std::to_string(scratch_elements) +
               "; use bag_sgemm_ex with a workspace from bag_workspace_create_ex");
    int dev = 0;
    cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
    bag_workspace ws{g.m, g.n, g.k, g.depth, g.basis, 1, dev, scratch, scratch_elements};
    run_gemm(g, beta, stream, &ws);
  });
}

}  // namespace bag_b200

extern "C" {

bag_status bag_primitive(int delta, int eps, int gamma_d, int gamma_e, int atomic,
                         const float* x, const float* y, const float* v, const float* w, float* d,
                         float* e, int m, int n, int k, long long ldx, long long ldy, long long ldv,
                         long long ldw, long long ldd, long long lde, bag_stream_t stream) {
  return guarded([&] {
    check_coeffs(delta, eps, gamma_d, gamma_e);
    if (m < 0 || n < 0 || k < 0) fail(BAG_ERR_SHAPE, "negative extent");
    if ((gamma_d == 0 && gamma_e == 0) || m == 0 || n == 0) return;
    if (gamma_d && gamma_e && d == e && (gamma_d == 2 || gamma_d == -2 || gamma_e == 2 || gamma_e == -2))
      fail(BAG_ERR_INVALID, "overwrite modes need distinct outputs");
    auto ld_ok = [&](long long ld, int rows) { return ld >= std::max(1, rows); };
    // An empty reduction reads no operand (k == 0 only writes 0 for +-2 codes).
    const bool reads = k > 0;
    if ((reads && (!ld_ok(ldx, m) || (delta && !ld_ok(ldy, m)) || !ld_ok(ldv, k) ||
                   (eps && !ld_ok(ldw, k)))) ||
        (gamma_d && !ld_ok(ldd, m)) || (gamma_e && !ld_ok(lde, m)))
      fail(BAG_ERR_INVALID, "leading dimension smaller than the row count");
    run_leaves({primitive_leaf(delta, eps, gamma_d, gamma_e, atomic, x, y, v, w, d, e, m, n, k,
                               std::max(ldx, 1LL), std::max(ldy, 1LL), std::max(ldv, 1LL),
                               std::max(ldw, 1LL), std::max(ldd, 1LL), std::max(lde, 1LL))},
               reinterpret_cast<cudaStream_t>(stream));
  });
}

bag_status bag_primitive_pair(int delta, int eps, int gamma_d, int gamma_e, int atomic,
                              const float* const operands[8], float* const outputs[4], int s,
                              long long ld, bag_stream_t stream) {
  return guarded([&] {
    check_coeffs(delta, eps, gamma_d, gamma_e);
    if (!operands || !outputs) fail(BAG_ERR_INVALID, "null operand table");
    if (s < 0) fail(BAG_ERR_SHAPE, "negative extent");
    if (s == 0 || (gamma_d == 0 && gamma_e == 0)) return;
    if (ld < s) fail(BAG_ERR_INVALID, "leading dimension smaller than the row count");
    std::vector<HostLeaf> leaves;
    for (int p = 0; p < 2; ++p)
      leaves.push_back(primitive_leaf(delta, eps, gamma_d, gamma_e, atomic, operands[4 * p],
                                      operands[4 * p + 1], operands[4 * p + 2],
                                      operands[4 * p + 3], outputs[2 * p], outputs[2 * p + 1], s,
                                      s, s, ld, ld, ld, ld, ld, ld));
    run_leaves(std::move(leaves), reinterpret_cast<cudaStream_t>(stream));
  });
}

bag_status bag_strassen_one_level(int backend, int schedule, const float* a, const float* b,
                                  float* c, int n, bag_stream_t stream) {
  return guarded([&] {
    check_backend(backend);
    if (schedule < BAG_STRASSEN_SERIAL_ATOMIC || schedule > BAG_STRASSEN_FOUR_BATCHED_ATOMIC)
      fail(BAG_ERR_INVALID, "unknown schedule");
    if (n <= 0 || n % 8) fail(BAG_ERR_SHAPE, "one_level currently requires N divisible by 8");
    if (!valid_shape_impl(backend, n / 2))
      fail(BAG_ERR_SHAPE, "shape violates original kernel tile constraints");
    const bool normal = schedule == BAG_STRASSEN_SERIAL_NORMAL ||
                        schedule == BAG_STRASSEN_DEPENDENCY_NORMAL ||
                        schedule == BAG_STRASSEN_PAIRED_NORMAL;
    if (normal && (backend == BAG_BACKEND_LEGACY || backend == BAG_BACKEND_MEDIUM ||
                   backend == BAG_BACKEND_HUGE))
      fail(BAG_ERR_UNSUPPORTED, "selected backend requires atomic updates");
    if (schedule == BAG_STRASSEN_FOUR_BATCHED_ATOMIC && !paired_backend(backend))
      fail(BAG_ERR_UNSUPPORTED, "four-variant batching requires a paired backend");
    run_gemm(make_desc(BAG_LAYOUT_COL_MAJOR, n, n, n, a, n, 0, b, n, 0, c, n, 0, 1, 1, kClassic),
             1.f, reinterpret_cast<cudaStream_t>(stream), nullptr);
  });
}

bag_status bag_valid_shape(int backend, int s, int* valid) {
  return guarded([&] {
    if (!valid) fail(BAG_ERR_INVALID, "null output pointer");
    check_backend(backend);
    *valid = valid_shape_impl(backend, s) ? 1 : 0;
  });
}

bag_status bag_profile_set_events(void* start_event, void* end_event) {
  return guarded([&] {
    if ((start_event == nullptr) != (end_event == nullptr))
      fail(BAG_ERR_INVALID, "set both profiling events or neither");
    g_prof_start = static_cast<cudaEvent_t>(start_event);
    g_prof_end = static_cast<cudaEvent_t>(end_event);
  });
}

bag_status bag_profile_set_phase_events(void* after_stages, void* after_last) {
  return guarded([&] {
    if ((after_stages == nullptr) != (after_last == nullptr))
      fail(BAG_ERR_INVALID, "set both phase events or neither");
    g_phase_stages = static_cast<cudaEvent_t>(after_stages);
    g_phase_done = static_cast<cudaEvent_t>(after_last);
  });
}

unsigned long long bag_launch_count(void) { return g_launches.load(); }

unsigned long long bag_device_allocations(void) { return g_device_allocs.load(); }

bag_status bag_set_math_mode(int mode) {
  return guarded([&] {
    if (mode != BAG_MATH_FFMA && mode != BAG_MATH_3XTF32) fail(BAG_ERR_INVALID, "unknown math mode");
    g_math_mode = mode;
  });
}

int bag_get_math_mode(void) { return g_math_mode; }
int bag_last_leaf_path(void) { return g_last_leaf_path; }

int bag_last_leaf_kernel(void) {
  if (g_last_leaf_path != BAG_MATH_3XTF32) return BAG_LEAF_KERNEL_FFMA;
  if (g_last_prep_kind == kPrepLeafPair) return BAG_LEAF_KERNEL_TF32_PAIR;
  if (g_last_prep_kind == kPrepLeafSingle) return BAG_LEAF_KERNEL_TF32_SINGLE;
  return BAG_LEAF_KERNEL_TF32_FUSED;
}

int bag_last_prepare_table(void) { return g_last_prep_kind >= 0 ? last_tree_expr_table() : -1; }

bag_status bag_device_error(unsigned* code) {
  return guarded([&] {
    if (!code) fail(BAG_ERR_INVALID, "null output pointer");
    unsigned tc = 0, tc3 = 0;
    cuda_check(read_and_clear_tc3_device_error(&tc3), "reading the device error word");
    cuda_check(read_and_clear_device_error(code), "reading the device error word");
    cuda_check(read_and_clear_tc_device_error(&tc), "reading the device error word");
    *code |= tc | tc3;
  });
}

bag_status bag_selftest_bounded_wait(unsigned long long limit_ns, int* gave_up) {
  return guarded([&] {
    if (!gave_up) fail(BAG_ERR_INVALID, "null output pointer");
    if (limit_ns == 0 || limit_ns > 100000000ull) fail(BAG_ERR_INVALID, "limit must be in (0, 0.1 s]");
    int* flag = nullptr;
    cuda_check(device_alloc(reinterpret_cast<void**>(&flag), sizeof(int)), "cudaMalloc");
    cudaError_t e = run_wait_selftest(limit_ns, flag, nullptr);
    if (e == cudaSuccess) e = cudaStreamSynchronize(nullptr);
    int host = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&host, flag, sizeof(int), cudaMemcpyDeviceToHost);
    cudaFree(flag);
    cuda_check(e, "bounded-wait self-test");
    *gave_up = host;
  });
}

bag_status bag_ffma_probe(float* sink, int iterations, bag_stream_t stream, double* flops) {
  return guarded([&] {
    if (!sink || !flops || iterations <= 0) fail(BAG_ERR_INVALID, "bad probe arguments");
    const int blocks = 4 * sm_count_for_current_device();
    cuda_check(launch_ffma_probe(sink, blocks, iterations, reinterpret_cast<cudaStream_t>(stream),
                                 flops),
               "probe launch");
  });
}

bag_status bag_plan_dump(int m, int n, int k, long long lda, long long ldb, long long ldc,
                         int depth, int basis, char* buf, size_t buflen, size_t* needed) {
  return guarded([&] {
    if (m < 0 || n < 0 || k < 0) fail(BAG_ERR_SHAPE, "negative extent");
    depth = resolve_depth(depth, m, n, k);
    if (depth < 0 || depth > 8) fail(BAG_ERR_INVALID, "depth must be 0..8 or BAG_DEPTH_AUTO");
    if (!known_basis(basis)) fail(BAG_ERR_INVALID, "unknown basis");
    const std::string s = dump_plan(m, n, k, lda, ldb, ldc, depth, basis);
    if (needed) *needed = s.size() + 1;
    if (buf && buflen) {
      const size_t len = std::min(buflen - 1, s.size());
      std::memcpy(buf, s.data(), len);
      buf[len] = 0;
    }
  });
}

}  // extern "C"

// ---- several GPUs of one process --------------------------------------------
// bag_sgemm_multi: the devices form an R x S grid; device (i, j) computes, on
// compact copies of its shards, row band i of every one of the 2^depth
// block-rows of C and column band j of every block-column.  BAG combines only
// blocks at equal offsets (the forward transforms and the inverse transform
// act on whole blocks), so the recursion on the shards is exactly the full
// recursion restricted to those rows and columns: no reduction between
// devices.  The shards travel by 2-D peer copies from and to the caller's
// device (NVLink where peer access is available).

struct bag_multi_workspace {
  int ngpus, rows, cols;             // the R x S device grid
  int m, n, k, depth, basis;         // column-major problem (after the layout swap)
  std::vector<int> devices;
  std::vector<bag_workspace*> ws;    // one per device, for its shard problem
  std::vector<float*> a, b, c;       // shard buffers: (m/R) x k, k x (n/S), (m/R) x (n/S)
  std::vector<cudaStream_t> streams;
  std::vector<cudaEvent_t> done;
  cudaEvent_t start = nullptr;
};

namespace bag_b200 {
namespace {

void multi_grid(int ngpus, int* rows, int* cols) {
  switch (ngpus) {
    case 2: *rows = 2; *cols = 1; break;
    case 4: *rows = 2; *cols = 2; break;
    case 8: *rows = 4; *cols = 2; break;
    default: *rows = ngpus; *cols = 1; break;
  }
}

// Restores the calling thread's current device on scope exit.
struct DeviceGuard {
  int saved = 0;
  bool ok = false;
  DeviceGuard() { ok = cudaGetDevice(&saved) == cudaSuccess; }
  ~DeviceGuard() {
    if (ok) cudaSetDevice(saved);
  }
};

void multi_free(bag_multi_workspace* w) {
  if (!w) return;
  DeviceGuard guard;
  for (size_t g = 0; g < w->devices.size(); ++g) {
    cudaSetDevice(w->devices[g]);
    if (g < w->ws.size() && w->ws[g]) bag_workspace_destroy(w->ws[g]);
    if (g < w->a.size() && w->a[g]) cudaFree(w->a[g]);
    if (g < w->b.size() && w->b[g]) cudaFree(w->b[g]);
    if (g < w->c.size() && w->c[g]) cudaFree(w->c[g]);
    if (g < w->streams.size() && w->streams[g]) cudaStreamDestroy(w->streams[g]);
    if (g < w->done.size() && w->done[g]) cudaEventDestroy(w->done[g]);
  }
  if (w->start) {
    cudaSetDevice(w->devices[0]);
    cudaEventDestroy(w->start);
  }
  delete w;
}

// Copies the band rows [b0, b0 + band) of each of `blocks` row blocks of q
// rows (a column-major matrix, `ncols` columns, leading dimension ld) between
// the full matrix and a compact matrix (leading dimension blocks * band).
void copy_row_bands(float* dst, long long ldd, const float* src, long long lds, int blocks, int q,
                    int band, int b0, int ncols, bool to_compact, cudaStream_t s) {
  for (int bi = 0; bi < blocks; ++bi) {
    const long long full_row = (long long)bi * q + b0, compact_row = (long long)bi * band;
    const float* from = to_compact ? src + full_row : src + compact_row;
    float* to = to_compact ? dst + compact_row : dst + full_row;
    cuda_check(cudaMemcpy2DAsync(to, size_t(ldd) * 4, from, size_t(lds) * 4, size_t(band) * 4,
                                 size_t(ncols), cudaMemcpyDefault, s),
               "shard copy");
  }
}

}  // namespace
}  // namespace bag_b200

extern "C" {

bag_status bag_multi_grid(int ngpus, int* rows, int* cols) {
  return guarded([&] {
    if (ngpus < 1 || !rows || !cols) fail(BAG_ERR_INVALID, "bad grid arguments");
    multi_grid(ngpus, rows, cols);
  });
}

bag_status bag_multi_workspace_create(int ngpus, const int* devices, int layout, int m, int n,
                                      int k, int depth, int basis, bag_multi_workspace** out) {
  bag_multi_workspace* w = nullptr;
  const bag_status st = guarded([&] {
    if (!out) fail(BAG_ERR_INVALID, "null output pointer");
    *out = nullptr;
    if (ngpus < 1 || ngpus > 64 || !devices) fail(BAG_ERR_INVALID, "need 1..64 devices");
    if (layout != BAG_LAYOUT_COL_MAJOR && layout != BAG_LAYOUT_ROW_MAJOR)
      fail(BAG_ERR_INVALID, "unknown layout");
    if (m < 0 || n < 0 || k < 0) fail(BAG_ERR_SHAPE, "negative extent");
    if (layout == BAG_LAYOUT_ROW_MAJOR) std::swap(m, n);   // C^T = B^T A^T
    depth = resolve_depth(depth, m, n, k);
    if (depth < 0 || depth > 8) fail(BAG_ERR_INVALID, "depth must be 0..8 or BAG_DEPTH_AUTO");
    if (!known_basis(basis)) fail(BAG_ERR_INVALID, "unknown basis");
    int rows = 1, cols = 1;
    multi_grid(ngpus, &rows, &cols);
    const long long bm = (long long)rows << depth, bn = (long long)cols << depth;
    if (m % bm || n % bn)
      fail(BAG_ERR_SHAPE, "multi-GPU shards need M divisible by 2^depth x grid rows and N by "
                          "2^depth x grid columns (in the column-major problem)");
    w = new bag_multi_workspace{};
    w->ngpus = ngpus;
    w->rows = rows;
    w->cols = cols;
    w->m = m;
    w->n = n;
    w->k = k;
    w->depth = depth;
    w->basis = basis;
    w->devices.assign(devices, devices + ngpus);
    w->ws.assign(ngpus, nullptr);
    w->a.assign(ngpus, nullptr);
    w->b.assign(ngpus, nullptr);
    w->c.assign(ngpus, nullptr);
    w->streams.assign(ngpus, nullptr);
    w->done.assign(ngpus, nullptr);
    DeviceGuard guard;
    const int home = devices[0];
    const int ms = m / rows, ns = n / cols;
    for (int g = 0; g < ngpus; ++g) {
      const int dev = devices[g];
      cuda_check(cudaSetDevice(dev), "cudaSetDevice");
      if (dev != home) {
        // NVLink peer access both ways where the pair supports it; copies fall
        // back to staging through the host otherwise.
        int can = 0;
        cuda_check(cudaDeviceCanAccessPeer(&can, dev, home), "cudaDeviceCanAccessPeer");
        if (can) {
          cudaError_t e = cudaDeviceEnablePeerAccess(home, 0);
          if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled)
            cuda_check(e, "cudaDeviceEnablePeerAccess");
          cudaGetLastError();
          cuda_check(cudaSetDevice(home), "cudaSetDevice");
          e = cudaDeviceEnablePeerAccess(dev, 0);
          if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled)
            cuda_check(e, "cudaDeviceEnablePeerAccess");
          cudaGetLastError();
          cuda_check(cudaSetDevice(dev), "cudaSetDevice");
        }
      }
      cuda_check(device_alloc(reinterpret_cast<void**>(&w->a[g]), std::max<size_t>(1, size_t(ms) * k) * 4),
                 "shard allocation");
      cuda_check(device_alloc(reinterpret_cast<void**>(&w->b[g]), std::max<size_t>(1, size_t(k) * ns) * 4),
                 "shard allocation");
      cuda_check(device_alloc(reinterpret_cast<void**>(&w->c[g]), std::max<size_t>(1, size_t(ms) * ns) * 4),
                 "shard allocation");
      cuda_check(cudaStreamCreateWithFlags(&w->streams[g], cudaStreamNonBlocking), "stream");
      cuda_check(cudaEventCreateWithFlags(&w->done[g], cudaEventDisableTiming), "event");
      // The shard problem's workspace, on this device, in this thread's math mode.
      const bag_status s = bag_workspace_create_ex(ms, ns, k, depth, basis, 1, &w->ws[g]);
      if (s != BAG_OK) fail(s, g_last_error);
    }
    cuda_check(cudaSetDevice(home), "cudaSetDevice");
    cuda_check(cudaEventCreateWithFlags(&w->start, cudaEventDisableTiming), "event");
    *out = w;
  });
  if (st != BAG_OK && w && (!out || *out != w)) {
    const std::string msg = g_last_error;
    multi_free(w);
    g_last_error = msg;
  }
  return st;
}

bag_status bag_multi_workspace_destroy(bag_multi_workspace* ws) {
  return guarded([&] { multi_free(ws); });
}

bag_status bag_sgemm_multi(int ngpus, const int* devices, int layout, int m, int n, int k,
                           const float* a, long long lda, const float* b, long long ldb, float* c,
                           long long ldc, float beta, int depth, int basis, bag_stream_t stream,
                           bag_multi_workspace* ws) {
  return guarded([&] {
    if (!ws) fail(BAG_ERR_WORKSPACE, "null multi-GPU workspace");
    if (ngpus != ws->ngpus || !devices) fail(BAG_ERR_WORKSPACE, "device list differs from the workspace's");
    for (int g = 0; g < ngpus; ++g)
      if (devices[g] != ws->devices[g]) fail(BAG_ERR_WORKSPACE, "device list differs from the workspace's");
    if (beta != 0.f && beta != 1.f) fail(BAG_ERR_INVALID, "beta must be 0 or 1");
    const GemmDesc g0 = make_desc(layout, m, n, k, a, lda, 0, b, ldb, 0, c, ldc, 0, 1, depth, basis);
    const int dres = resolve_depth(depth, g0.m, g0.n, g0.k);
    if (g0.m != ws->m || g0.n != ws->n || g0.k != ws->k || dres != ws->depth || basis != ws->basis)
      fail(BAG_ERR_WORKSPACE, "problem differs from the multi-GPU workspace's");
    if (g0.k > 0 && (!g0.a || !g0.b)) fail(BAG_ERR_INVALID, "A and B are required");
    if (!g0.c) fail(BAG_ERR_INVALID, "C is required");
    if (g0.lda < std::max(1, g0.m) || g0.ldb < std::max(1, g0.k) || g0.ldc < std::max(1, g0.m))
      fail(BAG_ERR_SHAPE, "leading dimension too small");
    const int blocks = 1 << ws->depth;
    const int ms = ws->m / ws->rows, ns = ws->n / ws->cols;
    const int qm = ws->m / blocks, qn = ws->n / blocks;
    const int bandm = qm / ws->rows, bandn = qn / ws->cols;
    DeviceGuard guard;
    const cudaStream_t caller = reinterpret_cast<cudaStream_t>(stream);
    cuda_check(cudaSetDevice(ws->devices[0]), "cudaSetDevice");
    cuda_check(cudaEventRecord(ws->start, caller), "cudaEventRecord");
    for (int r = 0; r < ngpus; ++r) {
      const int i = r / ws->cols, j = r % ws->cols;
      const cudaStream_t s = ws->streams[r];
      cuda_check(cudaSetDevice(ws->devices[r]), "cudaSetDevice");
      cuda_check(cudaStreamWaitEvent(s, ws->start, 0), "cudaStreamWaitEvent");
      // A shard: row band i of each block-row, all k columns.
      if (g0.k > 0)
        copy_row_bands(ws->a[r], ms, g0.a, g0.lda, blocks, qm, bandm, i * bandm, g0.k, true, s);
      // B shard: column band j of each block-column (rows of B^T): whole
      // columns, so one 2-D copy per block-column.
      for (int bj = 0; bj < blocks && g0.k > 0; ++bj) {
        const long long col = (long long)bj * qn + (long long)j * bandn;
        cuda_check(cudaMemcpy2DAsync(ws->b[r] + (long long)bj * bandn * g0.k, size_t(g0.k) * 4,
                                     g0.b + col * g0.ldb, size_t(g0.ldb) * 4, size_t(g0.k) * 4,
                                     size_t(bandn), cudaMemcpyDefault, s),
                   "shard copy");
      }
      // C shard when it accumulates: row band i of each block-row, for each
      // column band j of each block-column.
      for (int bj = 0; bj < blocks && beta != 0.f; ++bj) {
        const long long col = (long long)bj * qn + (long long)j * bandn;
        copy_row_bands(ws->c[r] + (long long)bj * bandn * ms, ms, g0.c + col * g0.ldc, g0.ldc,
                       blocks, qm, bandm, i * bandm, bandn, true, s);
      }
      const bag_status st = bag_sgemm_ex(BAG_LAYOUT_COL_MAJOR, ms, ns, g0.k, ws->a[r], ms,
                                         ws->b[r], std::max(1, g0.k), ws->c[r], ms, beta,
                                         ws->depth, ws->basis, reinterpret_cast<bag_stream_t>(s),
                                         ws->ws[r]);
      if (st != BAG_OK) fail(st, g_last_error);
      for (int bj = 0; bj < blocks; ++bj) {
        const long long col = (long long)bj * qn + (long long)j * bandn;
        copy_row_bands(g0.c + col * g0.ldc, g0.ldc, ws->c[r] + (long long)bj * bandn * ms, ms,
                       blocks, qm, bandm, i * bandm, bandn, false, s);
      }
      cuda_check(cudaEventRecord(ws->done[r], s), "cudaEventRecord");
    }
    cuda_check(cudaSetDevice(ws->devices[0]), "cudaSetDevice");
    for (int r = 0; r < ngpus; ++r)
      cuda_check(cudaStreamWaitEvent(caller, ws->done[r], 0), "cudaStreamWaitEvent");
  });
}

}  // extern "C"
