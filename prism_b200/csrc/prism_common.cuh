// Shared helpers for the Prism block-sparse attention kernels (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "../../include/prism_bsa.h"

namespace prism {

// ------------------------------------------------------------------ errors
// Thread-local last-error string (prism_last_error()).  Entry points return a
// prism_status_t and never abort the process.
void set_error(const char* fmt, ...);

#define PRISM_CHECK_ARG(cond, ...)            \
  do {                                        \
    if (!(cond)) {                            \
      ::prism::set_error(__VA_ARGS__);        \
      return PRISM_ERR_INVALID_ARG;           \
    }                                         \
  } while (0)

#define PRISM_CHECK_LAUNCH(what)                                                       \
  do {                                                                                 \
    cudaError_t e_ = cudaGetLastError();                                               \
    if (e_ != cudaSuccess) {                                                           \
      ::prism::set_error("%s: launch failed: %s", what, cudaGetErrorString(e_));       \
      return PRISM_ERR_CUDA;                                                           \
    }                                                                                  \
  } while (0)

#define PRISM_CHECK_CUDA(call, what)                                                   \
  do {                                                                                 \
    cudaError_t e_ = (call);                                                           \
    if (e_ != cudaSuccess) {                                                           \
      ::prism::set_error("%s: %s", what, cudaGetErrorString(e_));                      \
      return PRISM_ERR_CUDA;                                                           \
    }                                                                                  \
  } while (0)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline bool aligned_to(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// ------------------------------------------------------------------ shapes
// Candidate block shapes (bt, bh, bw): 7 of 64 tokens then 6 of 128 tokens
// (dynamic_block_shape.py:6-23).  The zone edge is 8 (dynamic_block_shape.py:31).
constexpr int kNumShapes = 13;
constexpr int kNumShapes64 = 7;
constexpr int kZone = 8;
constexpr int kZoneTokens = 512;
constexpr int kTile = 64;  // dynamic_block_attention.py:15
__host__ __device__ constexpr int shape_dim(int c, int d) {
  return (c == 0)    ? 4
         : (c == 1)  ? (d == 0 ? 8 : d == 1 ? 2 : 4)
         : (c == 2)  ? (d == 0 ? 8 : d == 1 ? 4 : 2)
         : (c == 3)  ? (d == 0 ? 2 : d == 1 ? 4 : 8)
         : (c == 4)  ? (d == 0 ? 2 : d == 1 ? 8 : 4)
         : (c == 5)  ? (d == 0 ? 4 : d == 1 ? 2 : 8)
         : (c == 6)  ? (d == 0 ? 4 : d == 1 ? 8 : 2)
         : (c == 7)  ? (d == 0 ? 2 : 8)
         : (c == 8)  ? (d == 0 ? 8 : d == 1 ? 2 : 8)
         : (c == 9)  ? (d == 0 ? 8 : d == 1 ? 8 : 2)
         : (c == 10) ? (d == 0 ? 4 : d == 1 ? 4 : 8)
         : (c == 11) ? (d == 0 ? 4 : d == 1 ? 8 : 4)
                     : (d == 0 ? 8 : 4);
}
__host__ __device__ constexpr int shape_tokens(int c) { return c < kNumShapes64 ? 64 : 128; }

// ------------------------------------------------------------------ bf16
__device__ __forceinline__ float bf2f(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float bfbits2f(uint16_t b) { return __uint_as_float(((uint32_t)b) << 16); }

// ----------------------------------------------------- deterministic math
// Same algorithms, written the same way, as the CPU oracle's
// oracle_det_expf / oracle_det_log2f: evaluated in double with only
// correctly-rounded + - * / (explicit _rn intrinsics, so no FMA contraction),
// then rounded once to float.
//   exp : Cody-Waite reduction x = k ln2 + r, Taylor series of e^r to r^13.
//   log2: x = 2^e m, m in [sqrt(1/2), sqrt(2)), ln m = 2 atanh((m-1)/(m+1))
//         by its power series to z^23, log2 x = e + ln m / ln 2.
__device__ __forceinline__ double dpow2_int(int k) {
  return __longlong_as_double((long long)(k + 1023) << 52);
}
#define DADD(a, b) __dadd_rn((a), (b))
#define DMUL(a, b) __dmul_rn((a), (b))
#define DDIV(a, b) __ddiv_rn((a), (b))

__device__ __forceinline__ float det_expf(float xf) {
  if (xf == -INFINITY) return 0.0f;
  if (xf < -120.0f) return 0.0f;
  if (xf > 88.0f) return INFINITY;
  const double LN2_HI = 6.93147180369123816490e-01;
  const double LN2_LO = 1.90821492927058770002e-10;
  const double INV_LN2 = 1.44269504088896338700e+00;
  double x = (double)xf;
  double kd = rint(DMUL(x, INV_LN2));
  int k = (int)kd;
  double r = DADD(DADD(x, -DMUL(kd, LN2_HI)), -DMUL(kd, LN2_LO));
  double p = DDIV(1.0, 6227020800.0);
  p = DADD(DMUL(p, r), DDIV(1.0, 479001600.0));
  p = DADD(DMUL(p, r), DDIV(1.0, 39916800.0));
  p = DADD(DMUL(p, r), DDIV(1.0, 3628800.0));
  p = DADD(DMUL(p, r), DDIV(1.0, 362880.0));
  p = DADD(DMUL(p, r), DDIV(1.0, 40320.0));
  p = DADD(DMUL(p, r), DDIV(1.0, 5040.0));
  p = DADD(DMUL(p, r), DDIV(1.0, 720.0));
  p = DADD(DMUL(p, r), DDIV(1.0, 120.0));
  p = DADD(DMUL(p, r), DDIV(1.0, 24.0));
  p = DADD(DMUL(p, r), DDIV(1.0, 6.0));
  p = DADD(DMUL(p, r), 0.5);
  p = DADD(DMUL(p, r), 1.0);
  p = DADD(DMUL(p, r), 1.0);
  return __double2float_rn(DMUL(p, dpow2_int(k)));
}

__device__ __forceinline__ float det_log2f(float xf) {
  uint32_t u = __float_as_uint(xf);
  int e = (int)((u >> 23) & 0xff) - 127;
  float mf = __uint_as_float((u & 0x007fffffu) | 0x3f800000u);
  double m = (double)mf;
  if (m > 1.4142135623730951) {
    m = DMUL(m, 0.5);
    e += 1;
  }
  double z = DDIV(DADD(m, -1.0), DADD(m, 1.0));
  double z2 = DMUL(z, z);
  double s = DDIV(1.0, 23.0);
  s = DADD(DMUL(s, z2), DDIV(1.0, 21.0));
  s = DADD(DMUL(s, z2), DDIV(1.0, 19.0));
  s = DADD(DMUL(s, z2), DDIV(1.0, 17.0));
  s = DADD(DMUL(s, z2), DDIV(1.0, 15.0));
  s = DADD(DMUL(s, z2), DDIV(1.0, 13.0));
  s = DADD(DMUL(s, z2), DDIV(1.0, 11.0));
  s = DADD(DMUL(s, z2), DDIV(1.0, 9.0));
  s = DADD(DMUL(s, z2), DDIV(1.0, 7.0));
  s = DADD(DMUL(s, z2), DDIV(1.0, 5.0));
  s = DADD(DMUL(s, z2), DDIV(1.0, 3.0));
  s = DADD(DMUL(s, z2), 1.0);
  double lnm = DMUL(DMUL(2.0, z), s);
  const double INV_LN2 = 1.44269504088896338700e+00;
  return __double2float_rn(DADD((double)e, DMUL(lnm, INV_LN2)));
}

// float arithmetic with one rounding per operation (no contraction)
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fdiv(float a, float b) { return __fdiv_rn(a, b); }

}  // namespace prism
