// Consumer of the drop-in C++ API, written only against the reference's
// public names (bag_cuda::Workspace / matmul, strassen_cuda::one_level /
// primitive / pair), the way the reference's benchmarks call them
// (benchmarks/cuda/bag.cu:51-101).  Built with a plain host compiler and
// linked against libbag_b200.so; run on a GPU it checks C <- AB + C on
// exactly representable inputs against an FP64 dot product at sampled
// positions and exits non-zero on failure.  An optional argument sets n (a
// multiple of 256; default 256); after each matmul case the consumer prints
// the leaf arithmetic the library reports (bag_last_leaf_path, the one name
// it uses beyond the reference's), so a run under BAG_B200_MATH=3xtf32 can
// show the tensor-core leaves were taken without a code change.
#include <bag/cuda/bag.cuh>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <vector>

namespace {

float input(size_t i, unsigned seed) {
  // Multiples of 2^-10 in [-0.5, 0.5): products are exact in FP64.
  unsigned x = unsigned(i) * 2654435761u ^ seed;
  x ^= x >> 13;
  x *= 0x5bd1e995u;
  x ^= x >> 15;
  return float(int(x & 1023u) - 512) / 1024.0f;
}

bool check(const std::vector<float>& a, const std::vector<float>& b, const std::vector<float>& c0,
           const std::vector<float>& c, int n, int repeats, const char* what) {
  double err2 = 0, ref2 = 0;
  for (int s = 0; s < 64; ++s) {
    const int r = (s * 37) % n, col = (s * 91 + 5) % n;
    double dot = 0;
    for (int k = 0; k < n; ++k) dot += double(a[r + size_t(k) * n]) * b[k + size_t(col) * n];
    const double ref = c0[r + size_t(col) * n] + repeats * dot;
    const double d = c[r + size_t(col) * n] - ref;
    err2 += d * d;
    ref2 += ref * ref;
  }
  const double rel = std::sqrt(err2 / ref2);
  std::printf("%s rel_l2=%.3e\n", what, rel);
  return rel <= 3e-5;
}

}  // namespace

int main(int argc, char** argv) try {
  const int n = argc > 1 ? std::atoi(argv[1]) : 256;
  if (n <= 0 || n % 256) {
    std::fprintf(stderr, "n must be a positive multiple of 256\n");
    return 2;
  }
  const size_t count = size_t(n) * n;
  std::vector<float> a(count), b(count), c0(count), c(count);
  for (size_t i = 0; i < count; ++i) {
    a[i] = input(i, 11);
    b[i] = input(i, 23);
    c0[i] = input(i, 37);
  }
  cudaStream_t caller;
  strassen_cuda::checked(cudaStreamCreateWithFlags(&caller, cudaStreamNonBlocking));
  bag_cuda::DeviceBuffer da(count), db(count), dc(count);
  strassen_cuda::checked(cudaMemcpy(da.p, a.data(), count * 4, cudaMemcpyHostToDevice));
  strassen_cuda::checked(cudaMemcpy(db.p, b.data(), count * 4, cudaMemcpyHostToDevice));
  bool ok = true;
  for (auto basis : {bag_cuda::Basis::Minimal, bag_cuda::Basis::Full}) {
    for (int depth : {1, 2}) {
      bag_cuda::Workspace ws(n, depth, basis);
      strassen_cuda::checked(cudaMemcpy(dc.p, c0.data(), count * 4, cudaMemcpyHostToDevice));
      for (int r = 0; r < 3; ++r)   // accumulating calls, as the reference validates
        bag_cuda::matmul(da.p, db.p, dc.p, n, caller, ws, bag_cuda::Backend::ColumnTile8,
                         bag_cuda::Schedule::Batched);
      strassen_cuda::checked(cudaStreamSynchronize(caller));
      strassen_cuda::checked(cudaMemcpy(c.data(), dc.p, count * 4, cudaMemcpyDeviceToHost));
      ok = check(a, b, c0, c, n, 3, basis == bag_cuda::Basis::Full ? "bag_full" : "bag_minimal") && ok;
      std::printf("depth=%d leaf_path=%s\n", depth,
                  bag_last_leaf_path() == BAG_MATH_3XTF32 ? "3xtf32" : "ffma");
    }
  }
  strassen_cuda::Workspace workers;
  strassen_cuda::checked(cudaMemcpy(dc.p, c0.data(), count * 4, cudaMemcpyHostToDevice));
  strassen_cuda::one_level(strassen_cuda::Backend::ColumnTile8,
                           strassen_cuda::Schedule::FourBatchedAtomic, da.p, db.p, dc.p, n, caller,
                           workers);
  strassen_cuda::checked(cudaStreamSynchronize(caller));
  strassen_cuda::checked(cudaMemcpy(c.data(), dc.p, count * 4, cudaMemcpyDeviceToHost));
  ok = check(a, b, c0, c, n, 1, "strassen_one_level") && ok;
  // Errors surface as std::runtime_error with the reference's messages.
  try {
    bag_cuda::Workspace bad(n, 1);
    bag_cuda::matmul(da.p, db.p, dc.p, n / 2, caller, bad);
    ok = false;
  } catch (const std::runtime_error& e) {
    std::printf("rejected: %s\n", e.what());
  }
  cudaStreamDestroy(caller);
  std::printf(ok ? "DROPIN OK\n" : "DROPIN FAILED\n");
  return ok ? 0 : 1;
} catch (const std::exception& e) {
  std::fprintf(stderr, "ERROR: %s\n", e.what());
  return 2;
}
