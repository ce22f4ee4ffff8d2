// fp64 sampling of the radial TP weights and their spline tables (replaces conv_spline.build_tables /
// spline_radial._sample of the reference: mace_onegpu/conv_spline.py:230-249, mace_onegpu/spline_radial.py:237-272).
#include <math.h>

#include "common.cuh"

namespace mb {

// One CTA per sample radius (knot k, offset s in {0: r, 1: r + eps, 2: r - eps}): radial features f(r) =
// Bessel(r) * cutoff(r) in fp64, then the bias-free MLP silu(silu(silu(f A0) A1) A2) A3 (normalisation constants
// already folded into A*).  out[s][k][d] fp64.
__global__ void k_sample_mlp(const double* __restrict__ A0, const double* __restrict__ A1,
                             const double* __restrict__ A2, const double* __restrict__ A3, int n_in, int H, int D,
                             int M, double r_lo, double h, double eps, double r_max, double p, double* __restrict__ out) {
  extern __shared__ double sm[];
  double* f = sm;           // [n_in]
  double* h0 = f + n_in;    // [H]
  double* h1 = h0 + H;      // [H]
  const int k = blockIdx.x, s = blockIdx.y;
  double r = r_lo + k * h + (s == 1 ? eps : (s == 2 ? -eps : 0.0));
  if (threadIdx.x < n_in) {
    int n = threadIdx.x + 1;
    double x = r / r_max;
    double env = 0.0;
    if (x < 1.0)
      env = 1.0 - 0.5 * (p + 1.0) * (p + 2.0) * pow(x, p) + p * (p + 2.0) * pow(x, p + 1.0) -
            0.5 * p * (p + 1.0) * pow(x, p + 2.0);
    f[threadIdx.x] = sqrt(2.0 / r_max) * sin(n * M_PI / r_max * r) / r * env;
  }
  __syncthreads();
  const double* Ws[3] = {A0, A1, A2};
  double* src = f;
  double* dst = h0;
  int fan = n_in;
  for (int layer = 0; layer < 3; ++layer) {
    for (int j = threadIdx.x; j < H; j += blockDim.x) {
      double z = 0.0;
      for (int q = 0; q < fan; ++q) z += src[q] * Ws[layer][(size_t)q * H + j];
      dst[j] = z / (1.0 + exp(-z));
    }
    __syncthreads();
    src = dst;
    dst = (dst == h0) ? h1 : h0;
    fan = H;
  }
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    double z = 0.0;
    for (int q = 0; q < H; ++q) z += src[q] * A3[(size_t)q * D + d];
    out[((size_t)s * M + k) * D + d] = z;
  }
}

// Per (pair, knot, column): TV = W, TG = h dW/dr (central differences), and on each interval the cubic
// a + b t + c t^2 + d t^3 equal to the Hermite interpolant of (TV, TG) at both ends.
__global__ void k_finish_tables(const double* __restrict__ smp, const double* __restrict__ col_scale, int P, int M,
                                int D, double h, double eps, float* __restrict__ TV, float* __restrict__ TG,
                                float4* __restrict__ cubic) {
  size_t n = (size_t)P * M * D;
  for (size_t q = blockIdx.x * (size_t)blockDim.x + threadIdx.x; q < n; q += (size_t)gridDim.x * blockDim.x) {
    int d = (int)(q % D);
    size_t pk = q / D;
    int k = (int)(pk % M);
    int p = (int)(pk / M);
    double cs = col_scale ? col_scale[(size_t)p * D + d] : 1.0;
    double v0 = smp[((size_t)0 * M + k) * D + d] * cs;
    double g0 = (smp[((size_t)1 * M + k) * D + d] - smp[((size_t)2 * M + k) * D + d]) / (2.0 * eps) * h * cs;
    if (TV) TV[q] = (float)v0;
    if (TG) TG[q] = (float)g0;
    if (cubic && k < M - 1) {
      double v1 = smp[((size_t)0 * M + k + 1) * D + d] * cs;
      double g1 = (smp[((size_t)1 * M + k + 1) * D + d] - smp[((size_t)2 * M + k + 1) * D + d]) / (2.0 * eps) * h * cs;
      float4 c4;
      c4.x = (float)v0;
      c4.y = (float)g0;
      c4.z = (float)(-3.0 * v0 - 2.0 * g0 + 3.0 * v1 - g1);
      c4.w = (float)(2.0 * v0 + g0 - 2.0 * v1 + g1);
      cubic[((size_t)p * (M - 1) + k) * D + d] = c4;
    }
  }
}

}  // namespace mb

using namespace mb;

extern "C" int mace_b200_build_tables(const double* A0, const double* A1, const double* A2, const double* A3,
                                      int32_t n_in, int32_t hidden, int32_t D, const double* col_scale,
                                      int32_t n_pairs, int32_t M, double r_lo, double r_max, double p_cut, float* TV,
                                      float* TG, float* cubic, void* stream) {
  if (!A0 || !A1 || !A2 || !A3 || n_in <= 0 || n_in > 64 || hidden <= 0 || hidden > 1024 || D <= 0 || n_pairs <= 0 ||
      M < 2 || !(r_max > r_lo) || r_lo <= 0.0) {
    set_error("build_tables: bad arguments");
    return MB_E_ARG;
  }
  cudaStream_t st = (cudaStream_t)stream;
  const double h = (r_max - r_lo) / (M - 1);
  const double eps = 1e-5 * (r_max - r_lo);
  double* smp = nullptr;
  if (cudaMallocAsync(&smp, sizeof(double) * 3 * (size_t)M * D, st) != cudaSuccess) {
    set_error("build_tables: cudaMallocAsync of %zu bytes failed", sizeof(double) * 3 * (size_t)M * D);
    return MB_E_CUDA;
  }
  size_t shm = sizeof(double) * (n_in + 2 * hidden);
  k_sample_mlp<<<dim3(M, 3), 128, shm, st>>>(A0, A1, A2, A3, n_in, hidden, D, M, r_lo, h, eps, r_max, p_cut, smp);
  int rc = check_launch("k_sample_mlp");
  if (rc == 0) {
    k_finish_tables<<<1184, 256, 0, st>>>(smp, col_scale, n_pairs, M, D, h, eps, TV, TG, (float4*)cubic);
    rc = check_launch("k_finish_tables");
  }
  cudaFreeAsync(smp, st);
  return rc;
}

// ------------------------------------------------------------------------------------------------ allocation-free
// Some callers cannot allocate device memory when they (re)build tables: an MD engine that owns all device memory
// through its own pool (LAMMPS/Kokkos builds) and must not have a library allocate behind its back, or a process that
// caps its device footprint after start-up.  mace_b200_build_tables_noalloc serves them: it runs the same two kernels
// as mace_b200_build_tables, but its fp64 sample scratch is this file-scope device array instead of a
// cudaMallocAsync buffer.  Capacity: M * D <= 512 * 1280 (the largest table of the MACE-MPA-0 architecture at the
// default 512-knot grid), i.e. 3 * 655,360 doubles = 15 MiB, held by every GPU that loads the library until exit.
static constexpr size_t kNoAllocMD = 512 * 1280;
static __device__ __align__(256) double g_noalloc_samples[3 * kNoAllocMD];

extern "C" int mace_b200_build_tables_noalloc(const double* A0, const double* A1, const double* A2, const double* A3,
                                              int32_t n_in, int32_t hidden, int32_t D, const double* col_scale,
                                              int32_t n_pairs, int32_t M, double r_lo, double r_max, double p_cut,
                                              float* TV, float* TG, float* cubic, void* stream) {
  if (!A0 || !A1 || !A2 || !A3 || n_in <= 0 || n_in > 64 || hidden <= 0 || hidden > 1024 || D <= 0 || n_pairs <= 0 ||
      M < 2 || !(r_max > r_lo) || r_lo <= 0.0) {
    set_error("build_tables_noalloc: bad arguments");
    return MB_E_ARG;
  }
  if ((size_t)M * (size_t)D > kNoAllocMD) {
    set_error("build_tables_noalloc: M * D = %lld exceeds the static scratch capacity %zu (at most 512 knots x 1280 "
              "columns); use mace_b200_build_tables", (long long)M * D, kNoAllocMD);
    return MB_E_ARG;
  }
  // The symbol is only a host-side stand-in: resolve the scratch's device address on the current device (every call;
  // cudaGetSymbolAddress is cheap and no stream operation, and nothing cached goes stale after a device reset).
  double* smp = nullptr;
  cudaError_t e = cudaGetSymbolAddress((void**)&smp, g_noalloc_samples);
  if (e != cudaSuccess || !smp) {
    set_error("build_tables_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
    return MB_E_CUDA;
  }
  cudaStream_t st = (cudaStream_t)stream;
  const double h = (r_max - r_lo) / (M - 1);
  const double eps = 1e-5 * (r_max - r_lo);
  // k_sample_mlp writes every [s][k][d] entry of the scratch before k_finish_tables reads it: nothing has to start at
  // zero.  Calls that overlap on the GPU (other streams) share this scratch and race; serialise them.
  size_t shm = sizeof(double) * (n_in + 2 * hidden);
  k_sample_mlp<<<dim3(M, 3), 128, shm, st>>>(A0, A1, A2, A3, n_in, hidden, D, M, r_lo, h, eps, r_max, p_cut, smp);
  int rc = check_launch("k_sample_mlp");
  if (rc) return rc;
  k_finish_tables<<<1184, 256, 0, st>>>(smp, col_scale, n_pairs, M, D, h, eps, TV, TG, (float4*)cubic);
  return check_launch("k_finish_tables");
}
