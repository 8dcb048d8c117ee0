// Chain fusion of the B200 host layer (include/sil_b200/gpu.h), checked
// through silarray's own API: consecutive elementwise nodes of one
// evaluation run as ONE kernel launch, intermediates that are still held by
// the caller are written too, and every result equals the reference CPU
// path (sil::use_cpu()) bit for bit.  Exit status 0 = all checks passed.
#include <silarray.h>

#include <cmath>
#include <cstdio>
#include <cstring>

#include "silcu.h"

using namespace sil;

static int failures = 0;

static void expect(bool ok, const char *what) {
  std::printf("%s: %s\n", ok ? "ok  " : "FAIL", what);
  if (!ok) failures++;
}

static bool same_bits(const array<float> &g, const array<float> &c) {
  if (g.element_count() != c.element_count()) return false;
  auto *x = g.buffer_data();
  auto *y = c.buffer_data();
  return std::memcmp(x, y, g.element_count() * sizeof(float)) == 0;
}

// sigmoid and pow round like CUDA's expf / powf on the GPU and like libm on
// the CPU: equal within a few ulp, not bit for bit.
static bool close(const array<float> &g, const array<float> &c) {
  if (g.element_count() != c.element_count()) return false;
  auto *x = g.buffer_data();
  auto *y = c.buffer_data();
  for (size_t i = 0; i < g.element_count(); i++)
    if (std::abs(double(x[i]) - double(y[i])) > 2e-6 * std::abs(double(y[i])) + 1e-7) return false;
  return true;
}

template <class F>
static void check_chain(const char *what, F expr, unsigned long long want_launches, bool exact = true) {
  use_cuda();
  auto n0 = silcu_kernel_launches();
  auto g = expr();
  eval(g);
  auto launches = silcu_kernel_launches() - n0;
  use_cpu();
  auto c = expr();
  eval(c);
  use_cuda();
  char msg[256];
  std::snprintf(msg, sizeof(msg), "%s: %llu launch(es), want %llu", what, launches, want_launches);
  expect(launches == want_launches, msg);
  std::snprintf(msg, sizeof(msg), "%s: equals the CPU path %s", what, exact ? "bit for bit" : "within 2e-6");
  expect(exact ? same_bits(g, c) : close(g, c), msg);
}

int main() {
  const size_t M = 300, N = 1027;
  auto a = random({M, N});
  auto b = random({M, N});
  auto c = random({M, N}) + array<float>(0.5f);
  auto row = random({N});
  synchronize();

  check_chain("(a + b) * c - a", [&] { return (a + b) * c - a; }, 1);
  check_chain("((a * b).sigmoid() + c).relu()", [&] { return ((a * b).sigmoid() + c).relu(); }, 1, false);
  check_chain("(a + row) / c, row broadcast", [&] { return (a + row) / c; }, 1);
  check_chain("(a - b) * 2 + 1, folded affine after a node",
              [&] { return (a - b) * array<float>(2.0f) + array<float>(1.0f); }, 1);
  check_chain("a.pow(b) * c", [&] { return a.pow(b) * c; }, 1, false);

  // An intermediate the caller holds is stored as well (two outputs, one
  // launch).  (Evaluating t and u in one sil::eval(t, u) call is not used:
  // the reference's evaluator marks every root visited before its
  // depth-first walk, so u may be ordered before t there.)
  {
    use_cuda();
    auto n0 = silcu_kernel_launches();
    auto t = a + b;
    auto u = t * c;
    eval(u);
    auto launches = silcu_kernel_launches() - n0;
    use_cpu();
    auto tc = a + b;
    auto uc = tc * c;
    eval(uc);
    use_cuda();
    expect(launches == 1, "held intermediate: one launch");
    expect(same_bits(t, tc) && same_bits(u, uc), "held intermediate and result equal the CPU path");
  }

  // A chain interrupted by a reduction: the chain runs before the reduction reads it.
  {
    use_cuda();
    auto s = ((a + b) * c).sum();
    use_cpu();
    auto sc = ((a + b) * c).sum();
    use_cuda();
    double rel = std::abs(double(s) - double(sc)) / (std::abs(double(sc)) + 1.0);
    expect(rel < 1e-4, "chain feeding a whole-array sum");
  }

  // sum(axis) for axes the reference sums on the host: on the GPU in the same
  // sequential order, so bit-identical to the CPU path.
  {
    auto t3 = random({7, 300, 33});
    for (size_t axis : {size_t(1), size_t(2)}) {
      use_cuda();
      auto n0 = silcu_kernel_launches();
      auto g = t3.sum(axis);
      eval(g);
      auto launches = silcu_kernel_launches() - n0;
      use_cpu();
      auto c = t3.sum(axis);
      eval(c);
      use_cuda();
      char msg[128];
      std::snprintf(msg, sizeof(msg), "sum(axis=%zu) of [7,300,33] on the GPU, bit-identical to the CPU path", axis);
      expect(launches == 1 && same_bits(g, c), msg);
    }
    auto m2 = random({4096, 1024});
    use_cuda();
    auto g = m2.sum(1);
    eval(g);
    use_cpu();
    auto c = m2.sum(1);
    eval(c);
    use_cuda();
    expect(same_bits(g, c), "sum(axis=1) of [4096,1024], bit-identical to the CPU path");
  }

  std::printf("%s (%d failure(s))\n", failures ? "FAILED" : "PASSED", failures);
  return failures ? 1 : 0;
}
