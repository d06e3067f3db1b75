// Exhaustive check of the sampler's exp (llm-workspace_b200/csrc/pesti_exp.cuh,
// host build) against the correctly rounded value (long double expl rounded
// once to float) and against the platform expf, over every float in [lo, 0].
// Prints: "<n> <mismatch_vs_cr> <mismatch_vs_platform>" and up to 5 examples.
// Built and run by tests/test_exp_exhaustive.py.
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <vector>
#include "pesti_exp.cuh"

static float f_of(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }
static uint32_t u_of(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }

int main(int argc, char** argv) {
  const float lo = argc > 1 ? std::strtof(argv[1], nullptr) : -104.0f;
  const uint32_t lim = u_of(-lo);
  const unsigned nt = std::max(1u, std::thread::hardware_concurrency());
  std::atomic<long long> n{0}, bad_cr{0}, bad_plat{0};
  std::atomic<int> shown{0};
  std::vector<std::thread> ts;
  for (unsigned t = 0; t < nt; ++t) {
    ts.emplace_back([&, t]() {
      long long ln = 0, lb = 0, lp = 0;
      for (uint64_t m = t; m <= lim; m += nt) {
        const float x = -f_of((uint32_t)m);
        const float mine = pesti_expf(x);
        const float cr = (float)expl((long double)x);
        ++ln;
        if (u_of(mine) != u_of(cr)) {
          ++lb;
          if (shown.fetch_add(1) < 5) std::printf("x=%a mine=%a cr=%a\n", x, mine, cr);
        }
        if (u_of(mine) != u_of(expf(x))) ++lp;
      }
      n += ln; bad_cr += lb; bad_plat += lp;
    });
  }
  for (auto& th : ts) th.join();
  std::printf("%lld %lld %lld\n", n.load(), bad_cr.load(), bad_plat.load());
  return 0;
}
