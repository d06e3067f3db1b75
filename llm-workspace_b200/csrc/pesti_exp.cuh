// Correctly rounded single-precision exp, evaluated in double precision.
//
// The reference computes exp with Rust's f32::exp (sampling.rs:127), which is
// the platform libm expf.  This routine returns the correctly rounded value
// instead: glibc's expf is a faithful (not correctly rounded) implementation,
// so no fixed algorithm reproduces it bit for bit without its private tables.
// On the domain the sampler uses (x <= 0) the two differ on about 6e-4 of the
// float inputs, by one ulp.
//
// Method (Tang's table-driven reduction, constants derived in
// gen_exp_table.py from their definitions):
//   k = rint(x * 32/ln2), r = x - k*ln2/32 (two-constant fma reduction),
//   exp(x) = 2^(k>>5) * 2^((k&31)/32) * exp(r), |r| <= ln2/64,
//   exp(r) - 1 by its degree-6 Taylor polynomial (truncation < 2^-58),
//   2^(j/32) as a double-double (T_HI + T_LO).
// The result is held as hi + lo (error ~2^-57 relative); rounding hi to float
// is correct unless hi is exactly halfway between two floats, in which case
// the sign of lo decides.  The host build of this same code agrees with the
// correctly rounded long-double value on every float x in [-104, 0]
// (tests/test_exp_exhaustive.py), and every operation below is a single IEEE
// double operation with explicit FMA, so host and device results are equal.
#pragma once
#include <stdint.h>
#include "pesti_exp_table.h"

#if defined(__CUDACC__)
#define PESTI_HD __host__ __device__ __forceinline__
#else
#define PESTI_HD inline
#endif

#if defined(__CUDA_ARCH__)
#define PX_MUL(a, b) __dmul_rn((a), (b))
#define PX_ADD(a, b) __dadd_rn((a), (b))
#define PX_FMA(a, b, c) __fma_rn((a), (b), (c))
#define PX_RINT(a) rint(a)
#define PX_D2F(a) __double2float_rn(a)
#define PX_F2BITS(f) ((uint32_t)__float_as_uint(f))
#define PX_BITS2F(u) __uint_as_float(u)
#define PX_D_FROM_BITS(u) __longlong_as_double((long long)(u))
#else
#include <cmath>
#include <cstring>
#define PX_MUL(a, b) ((a) * (b))
#define PX_ADD(a, b) ((a) + (b))
#define PX_FMA(a, b, c) std::fma((a), (b), (c))
#define PX_RINT(a) std::nearbyint(a)
#define PX_D2F(a) ((float)(a))
static inline uint32_t px_f2bits_h(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }
static inline float px_bits2f_h(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }
static inline double px_d_from_bits_h(uint64_t u) { double d; std::memcpy(&d, &u, 8); return d; }
#define PX_F2BITS(f) px_f2bits_h(f)
#define PX_BITS2F(u) px_bits2f_h(u)
#define PX_D_FROM_BITS(u) px_d_from_bits_h(u)
#endif

#if defined(__CUDACC__)
static __device__ const double pesti_exp_t_hi_d[32] = PESTI_EXP_T_HI_INIT;
static __device__ const double pesti_exp_t_lo_d[32] = PESTI_EXP_T_LO_INIT;
#endif
static const double pesti_exp_t_hi_h[32] = PESTI_EXP_T_HI_INIT;
static const double pesti_exp_t_lo_h[32] = PESTI_EXP_T_LO_INIT;

#if defined(__CUDA_ARCH__)
#define PX_T_HI(j) __ldg(&pesti_exp_t_hi_d[(j)])
#define PX_T_LO(j) __ldg(&pesti_exp_t_lo_d[(j)])
#else
#define PX_T_HI(j) pesti_exp_t_hi_h[(j)]
#define PX_T_LO(j) pesti_exp_t_lo_h[(j)]
#endif

PESTI_HD float pesti_expf(float x) {
  if (!(x == x)) return x;                    // NaN
  if (x < -110.0f) return 0.0f;               // exp < 2^-158 rounds to 0 (also -inf)
  if (x > 100.0f) return PX_BITS2F(0x7f800000u);  // overflow to +inf
  const double xd = (double)x;
  const double kd = PX_RINT(PX_MUL(xd, PESTI_EXP_INV_L));
  const int k = (int)kd;
  double r = PX_FMA(-kd, PESTI_EXP_L1, xd);
  r = PX_FMA(-kd, PESTI_EXP_L2, r);
  const int j = k & 31;
  const int n = (k - j) / 32;
  double t = PX_FMA(r, PESTI_EXP_C6, PESTI_EXP_C5);
  t = PX_FMA(r, t, PESTI_EXP_C4);
  t = PX_FMA(r, t, PESTI_EXP_C3);
  t = PX_FMA(r, t, PESTI_EXP_C2);
  const double r2 = PX_MUL(r, r);
  const double em1 = PX_FMA(r2, t, r);        // exp(r) - 1
  const double thi = PX_T_HI(j), tlo = PX_T_LO(j);
  double s = PX_FMA(tlo, em1, tlo);           // tlo * exp(r)
  s = PX_FMA(thi, em1, s);                    // + thi * (exp(r) - 1)
  double hi = PX_ADD(thi, s);
  double lo = PX_ADD(s, -PX_ADD(hi, -thi));   // exact remainder (|thi| >= |s|)
  const double scale = PX_D_FROM_BITS((uint64_t)(n + 1023) << 52);
  hi = PX_MUL(hi, scale);                     // exact: power-of-two scaling
  lo = PX_MUL(lo, scale);
  float f = PX_D2F(hi);
  const double back = (double)f;
  if (back != hi) {
    // g = the float on the other side of hi from f
    const uint32_t fb = PX_F2BITS(f);
    const float g = PX_BITS2F(hi > back ? fb + 1u : fb - 1u);
    const double mid = PX_MUL(PX_ADD(back, (double)g), 0.5);
    if (hi == mid && lo != 0.0) {
      const bool up = lo > 0.0;
      if ((g > f) == up) f = g;
    }
  }
  return f;
}

// Relative error bound of the hardware 2^y approximation (ex2.approx.ftz.f32)
// for every float y in [-200, 0] (0, flushed, allowed below -126) and -inf (0);
// tests/test_ex2_bound.py measures it exhaustively against exp2 in double and
// checks it against this value.
#define PESTI_EX2_APPROX_RELERR 0x1p-22f
