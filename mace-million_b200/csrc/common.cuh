// Shared device helpers of the sm_100a three-pass MACE kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/mace_b200.h"

#define MB_C 128            // channels per irrep component (the kernels are specialised for 128)
#define MB_NY 16            // spherical-harmonic components, l <= 3
#define MB_NB 8             // Bessel functions

namespace mb {

// ---------------------------------------------------------------------------------------------- error word
// Device-side checks record a bit in a status word instead of faulting; the host reads it at pass ends.
enum : unsigned {
  ST_BAD_SENDER = 1u << 0,     // pair_j outside [0, ntotal)
  ST_BAD_SPECIES = 1u << 1,    // compact species outside [0, S)
  ST_BAD_ROWPTR = 1u << 2,     // CSR row pointer not monotone / outside [0, P]
  ST_NONFINITE = 1u << 3,      // non-finite edge vector
  ST_BAD_RECEIVER = 1u << 4,   // pair_i does not match the CSR row
};
#define MB_ST_TC_TIMEOUT (1u << 5)  // a tensor-core kernel gave up waiting on its MMA barrier

__device__ __forceinline__ void set_status(unsigned* st, unsigned bit) {
  if (st) atomicOr(st, bit);
}

// ---------------------------------------------------------------------------------------------- spline rows
// Spline-coefficient loads of the edge kernels: the read-only path with L1 allocation (MB_TAB_LOAD = 0, default).
// Measured alternatives on the 1.03M-atom evaluation: no L1 allocation (1) made the layer-2 kernels 40% slower,
// L2-only caching (2) matched the default.
#ifndef MB_TAB_LOAD
#define MB_TAB_LOAD 0
#endif
__device__ __forceinline__ float4 tab_ld(const float4* p) {
#if MB_TAB_LOAD == 1
  float4 v;
  asm("ld.global.nc.L1::no_allocate.v4.f32 {%0, %1, %2, %3}, [%4];"
      : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
      : "l"(p));
  return v;
#elif MB_TAB_LOAD == 2
  return __ldcg(p);
#else
  return __ldg(p);
#endif
}

// ---------------------------------------------------------------------------------------------- reductions
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---------------------------------------------------------------------------------------------- dual numbers
// Forward-mode derivative w.r.t. the three components of the unit vector (x, y, z).
struct D3 {
  float v, dx, dy, dz;
};
__device__ __forceinline__ D3 d3c(float c) { return {c, 0.f, 0.f, 0.f}; }
__device__ __forceinline__ D3 operator+(D3 a, D3 b) { return {a.v + b.v, a.dx + b.dx, a.dy + b.dy, a.dz + b.dz}; }
__device__ __forceinline__ D3 operator-(D3 a, D3 b) { return {a.v - b.v, a.dx - b.dx, a.dy - b.dy, a.dz - b.dz}; }
__device__ __forceinline__ D3 operator*(D3 a, D3 b) {
  return {a.v * b.v, a.dx * b.v + a.v * b.dx, a.dy * b.v + a.v * b.dy, a.dz * b.v + a.v * b.dz};
}
__device__ __forceinline__ D3 operator*(float c, D3 a) { return {c * a.v, c * a.dx, c * a.dy, c * a.dz}; }
template <typename T>
__device__ __forceinline__ T d3one();
template <>
__device__ __forceinline__ float d3one<float>() { return 1.f; }
template <>
__device__ __forceinline__ D3 d3one<D3>() { return {1.f, 0.f, 0.f, 0.f}; }

// Component-normalised real spherical harmonics (l <= 3) of the unit vector (x, y, z): the homogeneous polynomial
// forms of e3nn 0.4 (sum_m Y_lm^2 = 2l + 1).  Templated so that the same code gives values (float) or values and
// gradients (D3).
template <typename T>
__device__ __forceinline__ void sh16(T x, T y, T z, T* Y) {
  const float s3 = 1.7320508075688772f, s5 = 2.23606797749979f, s15 = 3.872983346207417f;
  const float c42 = 1.0801234497346435f;   // sqrt(42) / 6
  const float c168 = 1.6201851746019651f;  // sqrt(168) / 8
  const float c7 = 2.6457513110645906f;    // sqrt(7)
  Y[0] = d3one<T>();
  Y[1] = s3 * x;
  Y[2] = s3 * y;
  Y[3] = s3 * z;
  T y2 = y * y;
  T x2z2 = x * x + z * z;
  T s20 = s15 * (x * z);
  T s24 = (0.5f * s15) * (z * z - x * x);
  Y[4] = s20;
  Y[5] = s15 * (x * y);
  Y[6] = s5 * (y2 - 0.5f * x2z2);
  Y[7] = s15 * (y * z);
  Y[8] = s24;
  Y[9] = c42 * (s20 * z + s24 * x);
  Y[10] = c7 * (s20 * y);
  Y[11] = c168 * ((4.f * y2 - x2z2) * x);
  Y[12] = (0.5f * c7) * (y * (2.f * y2 - 3.f * x2z2));
  Y[13] = c168 * (z * (4.f * y2 - x2z2));
  Y[14] = c7 * (s24 * y);
  Y[15] = c42 * (s24 * z - s20 * x);
}

// ---------------------------------------------------------------------------------------------- radial parts
struct Radial {
  float r_max, p;          // cutoff radius, polynomial cutoff order
  float r_lo, inv_h;       // spline grid: knots r_lo + k h, k = 0 .. M-1
  int M;
};

// Polynomial cutoff f(r) and f'(r) (mace PolynomialCutoff): f = 1 - (p+1)(p+2)/2 x^p + p(p+2) x^(p+1)
// - p(p+1)/2 x^(p+2), x = r / r_max, f' = -p(p+1)(p+2)/2 x^(p-1) (1 - x)^2 / r_max; zero beyond r_max.
__device__ __forceinline__ void poly_cutoff(float r, float rmax, float p, float& f, float& df) {
  float x = r / rmax;
  if (x >= 1.f) {
    f = 0.f;
    df = 0.f;
    return;
  }
  float xp1 = powf(x, p - 1.f);
  if (p == 5.f) xp1 = (x * x) * (x * x);
  float xp = xp1 * x;
  f = 1.f - 0.5f * (p + 1.f) * (p + 2.f) * xp + p * (p + 2.f) * xp * x - 0.5f * p * (p + 1.f) * xp * x * x;
  float om = 1.f - x;
  df = -0.5f * p * (p + 1.f) * (p + 2.f) * xp1 * om * om / rmax;
}

// Edge density (mace density_fn of a Density interaction block): d = sum_n w_n B_n(r) f(r), ed = tanh(d^2),
// B_n = sqrt(2 / r_max) sin(n pi r / r_max) / r.  Returns ed and d ed / dr.  wd already holds w / sqrt(8).
__device__ __forceinline__ void edge_density(float r, const float* wd, float rmax, float p, float& ed, float& ded) {
  float f, df;
  poly_cutoff(r, rmax, p, f, df);
  float th = 3.14159265358979323846f * r / rmax;
  float s1, c1;
  sincosf(th, &s1, &c1);
  float pref = sqrtf(2.f / rmax);
  float inv_r = 1.f / r;
  // sin(n th), cos(n th) by the Chebyshev recurrence
  float sp = 0.f, s = s1, cp = 1.f, c = c1;
  float d = 0.f, dd = 0.f;
#pragma unroll
  for (int n = 1; n <= MB_NB; ++n) {
    float b = pref * s * inv_r;
    float db = pref * ((float)n * 3.14159265358979323846f / rmax * c * inv_r - s * inv_r * inv_r);
    d += wd[n - 1] * b * f;
    dd += wd[n - 1] * (db * f + b * df);
    float sn = 2.f * c1 * s - sp;
    float cn = 2.f * c1 * c - cp;
    sp = s;
    s = sn;
    cp = c;
    c = cn;
  }
  float d2 = d * d;
  ed = tanhf(d2);
  ded = (1.f - ed * ed) * 2.f * d * dd;
}

// Spline coordinates: x = clamp((r - r_lo) / h, 0, M - 1 - 1e-4), interval k = floor(x), t = x - k
// (the clamp of the reference's Triton lookup, mace_onegpu/spline_w.py:19-27).
__device__ __forceinline__ void spline_coords(float r, const Radial& rd, int& k, float& t) {
  float x = (r - rd.r_lo) * rd.inv_h;
  x = fminf(fmaxf(x, 0.f), (float)(rd.M - 1) - 1e-4f);
  float kf = floorf(x);
  k = (int)kf;
  t = x - kf;
}

// Warp-wide sums of 16 per-lane values with 16 shuffles: each step exchanges half of the remaining values with the
// partner lane of one bit, so that lane L ends with the sum over the warp of v[L >> 1].
__device__ __forceinline__ float transpose_reduce16(float* v, int lane) {
#pragma unroll
  for (int h = 8, bit = 16; h >= 1; h >>= 1, bit >>= 1) {
    const bool up = lane & bit;
#pragma unroll
    for (int q = 0; q < h; ++q) {
      const float send = up ? v[q] : v[q + h];
      const float keep = up ? v[q + h] : v[q];
      v[q] = keep + __shfl_xor_sync(0xffffffffu, send, bit);
    }
  }
  return v[0] + __shfl_xor_sync(0xffffffffu, v[0], 1);
}

}  // namespace mb

// ---------------------------------------------------------------------------------------------- error plumbing
namespace mb {
void set_error(const char* fmt, ...);
int check_launch(const char* what);
}  // namespace mb
