// Exhaustive error measurement of pesti_expf_approx (host build of
// llm-workspace_b200/csrc/pesti_exp.cuh) against the correctly rounded f32 exp,
// over every float in [lo, 0].  Prints "<n> <max_rel_err> <count_over_bound>".
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
  std::vector<double> worst(nt, 0.0);
  std::atomic<long long> over{0}, n{0};
  const double bound = (double)PESTI_EXPF_APPROX_RELERR;
  std::vector<std::thread> ts;
  for (unsigned t = 0; t < nt; ++t) {
    ts.emplace_back([&, t]() {
      long long lo_over = 0, ln = 0;
      double w = 0.0;
      for (uint64_t m = t; m <= lim; m += nt) {
        const float x = -f_of((uint32_t)m);
        const float a = pesti_expf_approx(x);
        ++ln;
        if (!(x > -86.0f)) {  // outside the approximation's range: it must return 0
          if (a != 0.0f) ++lo_over;
          continue;
        }
        const double ex = (double)(float)expl((long double)x);  // correctly rounded f32
        const double rel = std::fabs(((double)a - ex) / ex);
        if (rel > w) w = rel;
        if (rel > bound) ++lo_over;
      }
      worst[t] = w;
      over += lo_over;
      n += ln;
    });
  }
  for (auto& th : ts) th.join();
  double w = 0.0;
  for (double v : worst) w = v > w ? v : w;
  std::printf("%lld %.6e %lld\n", n.load(), w, over.load());
  return 0;
}
