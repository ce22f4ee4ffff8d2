// Generic fused channelwise tensor product with explicit per-edge weights: the body of FusedConvTP (replaces the
// cuEquivariance segmented polynomial of the reference, mace_onegpu/fused_conv.py:20-37):
//   out[recv_e][o][c] += sum_terms coef W[e][w][c] X[send_e][k][c] Y[e][m]
// The path table (w, k, m, o, coef) is a runtime argument, so any channelwise table works (C = 128 channels).
// Edges are visited through CSR lists built by the caller, so no kernel needs an atomic:
//   forward           one CTA per receiver, one thread per channel, the receiver's edges in its CSR row; the output
//                     row accumulates in the thread's shared-memory column;
//   backward dW, dY   one CTA per receiver: per edge, dW[e][w][c] by the channel's thread and dY[e][m] as a sum over
//                     the CTA's channels;
//   backward dX       one CTA per sender over the sender's edges (sender CSR): dX[s][k][c] in the thread's column.
// The hot path of the three passes uses the spline-fused edge kernels of edge.cu instead.
#include "common.cuh"

namespace mb {

struct TermsSmem {
  int4* t;       // (w, k, m, o)
  float* c;      // coefficients
};

__device__ __forceinline__ void load_terms(const int4* __restrict__ terms, const float* __restrict__ coef, int nT,
                                           TermsSmem s) {
  for (int q = threadIdx.x; q < nT; q += blockDim.x) {
    s.t[q] = terms[q];
    s.c[q] = coef[q];
  }
}

__global__ void __launch_bounds__(128) k_conv_tp_fwd(const float* __restrict__ X, int nX, const float* __restrict__ Y,
                                                     int nY, const float* __restrict__ W, int nW,
                                                     const int* __restrict__ snd, const int64_t* __restrict__ rowptr,
                                                     const int64_t* __restrict__ edges, int n_nodes,
                                                     const int4* __restrict__ terms, const float* __restrict__ coef,
                                                     int nT, float* __restrict__ out, int nO, unsigned* status) {
  extern __shared__ __align__(16) float sm[];
  float* acc = sm;                                          // [nO][128]
  TermsSmem ts{reinterpret_cast<int4*>(acc + (size_t)nO * MB_C), nullptr};
  ts.c = reinterpret_cast<float*>(ts.t + nT);
  const int r = blockIdx.x, c = threadIdx.x;
  load_terms(terms, coef, nT, ts);
  for (int o = 0; o < nO; ++o) acc[o * MB_C + c] = 0.f;
  __syncthreads();
  for (int64_t q = rowptr[r]; q < rowptr[r + 1]; ++q) {
    const int64_t e = edges[q];
    const int s = snd[e];
    if (s < 0 || s >= n_nodes) {
      if (c == 0) set_status(status, ST_BAD_SENDER);
      continue;
    }
    const float* xs = X + (int64_t)s * nX * MB_C + c;
    const float* we = W + e * nW * MB_C + c;
    const float* ye = Y + e * nY;
    for (int t = 0; t < nT; ++t) {
      const int4 p = ts.t[t];
      acc[p.w * MB_C + c] = fmaf(ts.c[t] * __ldg(we + p.x * MB_C) * __ldg(xs + p.y * MB_C), __ldg(ye + p.z),
                                 acc[p.w * MB_C + c]);
    }
  }
  float* orow = out + (int64_t)r * nO * MB_C + c;
  for (int o = 0; o < nO; ++o) orow[o * MB_C] = acc[o * MB_C + c];
}

// dW and dY per edge of receiver r's CSR row (g = dL/dout).
__global__ void __launch_bounds__(128) k_conv_tp_bwd_wy(const float* __restrict__ X, int nX,
                                                        const float* __restrict__ Y, int nY,
                                                        const float* __restrict__ W, int nW,
                                                        const int* __restrict__ snd,
                                                        const int64_t* __restrict__ rowptr,
                                                        const int64_t* __restrict__ edges, int n_nodes,
                                                        const int4* __restrict__ terms,
                                                        const float* __restrict__ coef, int nT,
                                                        const float* __restrict__ g, int nO, float* __restrict__ dY,
                                                        float* __restrict__ dW, unsigned* status) {
  extern __shared__ __align__(16) float sm[];
  float* gs = sm;                                           // [nO][128] the receiver's upstream gradient
  float* dwc = gs + (size_t)nO * MB_C;                      // [nW][128]
  float* pyc = dwc + (size_t)nW * MB_C;                     // [nY][128] per-channel dY partials
  float* red = pyc + (size_t)nY * MB_C;                     // [4][nY]
  TermsSmem ts{reinterpret_cast<int4*>(red + 4 * nY), nullptr};
  ts.c = reinterpret_cast<float*>(ts.t + nT);
  const int r = blockIdx.x, c = threadIdx.x, warp = c >> 5, lane = c & 31;
  load_terms(terms, coef, nT, ts);
  for (int o = 0; o < nO; ++o) gs[o * MB_C + c] = g[((int64_t)r * nO + o) * MB_C + c];
  __syncthreads();
  for (int64_t q = rowptr[r]; q < rowptr[r + 1]; ++q) {
    const int64_t e = edges[q];
    const int s = snd[e];
    const bool ok = s >= 0 && s < n_nodes;
    if (!ok && c == 0) set_status(status, ST_BAD_SENDER);
    for (int w = 0; w < nW; ++w) dwc[w * MB_C + c] = 0.f;
    for (int m = 0; m < nY; ++m) pyc[m * MB_C + c] = 0.f;
    if (ok) {
      const float* xs = X + (int64_t)s * nX * MB_C + c;
      const float* we = W + e * nW * MB_C + c;
      const float* ye = Y + e * nY;
      for (int t = 0; t < nT; ++t) {
        const int4 p = ts.t[t];
        const float gc = ts.c[t] * gs[p.w * MB_C + c];
        const float xv = __ldg(xs + p.y * MB_C), wv = __ldg(we + p.x * MB_C), yv = __ldg(ye + p.z);
        dwc[p.x * MB_C + c] = fmaf(gc * xv, yv, dwc[p.x * MB_C + c]);
        pyc[p.z * MB_C + c] = fmaf(gc * wv, xv, pyc[p.z * MB_C + c]);
      }
    }
    if (dW)
      for (int w = 0; w < nW; ++w) dW[(e * nW + w) * MB_C + c] = dwc[w * MB_C + c];
    if (dY) {
      for (int m = 0; m < nY; ++m) {
        const float v = warp_sum(pyc[m * MB_C + c]);
        if (lane == 0) red[warp * nY + m] = v;
      }
      __syncthreads();
      if (c < nY) dY[e * nY + c] = red[c] + red[nY + c] + red[2 * nY + c] + red[3 * nY + c];
      __syncthreads();
    }
  }
}

// dX of sender s over its edges (sender CSR).
__global__ void __launch_bounds__(128) k_conv_tp_bwd_x(const float* __restrict__ Y, int nY,
                                                       const float* __restrict__ W, int nW,
                                                       const int* __restrict__ rcv,
                                                       const int64_t* __restrict__ rowptr,
                                                       const int64_t* __restrict__ edges, int n_nodes,
                                                       const int4* __restrict__ terms, const float* __restrict__ coef,
                                                       int nT, const float* __restrict__ g, int nO,
                                                       float* __restrict__ dX, int nX, unsigned* status) {
  extern __shared__ __align__(16) float sm[];
  float* dxc = sm;                                          // [nX][128]
  TermsSmem ts{reinterpret_cast<int4*>(dxc + (size_t)nX * MB_C), nullptr};
  ts.c = reinterpret_cast<float*>(ts.t + nT);
  const int s = blockIdx.x, c = threadIdx.x;
  load_terms(terms, coef, nT, ts);
  for (int k = 0; k < nX; ++k) dxc[k * MB_C + c] = 0.f;
  __syncthreads();
  for (int64_t q = rowptr[s]; q < rowptr[s + 1]; ++q) {
    const int64_t e = edges[q];
    const int r = rcv[e];
    if (r < 0 || r >= n_nodes) {
      if (c == 0) set_status(status, ST_BAD_RECEIVER);
      continue;
    }
    const float* gr = g + (int64_t)r * nO * MB_C + c;
    const float* we = W + e * nW * MB_C + c;
    const float* ye = Y + e * nY;
    for (int t = 0; t < nT; ++t) {
      const int4 p = ts.t[t];
      dxc[p.y * MB_C + c] =
          fmaf(ts.c[t] * __ldg(gr + p.w * MB_C) * __ldg(we + p.x * MB_C), __ldg(ye + p.z), dxc[p.y * MB_C + c]);
    }
  }
  float* drow = dX + (int64_t)s * nX * MB_C + c;
  for (int k = 0; k < nX; ++k) drow[k * MB_C] = dxc[k * MB_C + c];
}

static int conv_args(const int32_t* terms, int nT, int nX, int nY, int nW, int nO, int n_nodes, const char* who) {
  if (!terms || nT <= 0 || nX <= 0 || nY <= 0 || nY > 64 || nW <= 0 || nO <= 0 || n_nodes < 0 ||
      (size_t)(nO + nW + nY) * MB_C * 4 + (size_t)nT * 20 + 4 * 64 * 4 > 200 * 1024) {
    set_error("%s: bad sizes (nX %d, nY %d, nW %d, nO %d, terms %d)", who, nX, nY, nW, nO, nT);
    return MB_E_ARG;
  }
  return 0;
}

}  // namespace mb

using namespace mb;

extern "C" int mace_b200_conv_tp_fwd(const float* X, int32_t nX, const float* Y, int32_t nY, const float* W,
                                     int32_t nW, const int32_t* sender, const int64_t* recv_rowptr,
                                     const int64_t* recv_edges, int32_t n_nodes, const int32_t* terms_wkmo,
                                     const float* coef, int32_t n_terms, float* out, int32_t nO, uint32_t* status,
                                     void* stream) {
  if (int rc = conv_args(terms_wkmo, n_terms, nX, nY, nW, nO, n_nodes, "conv_tp_fwd")) return rc;
  if (n_nodes == 0) return 0;
  if (!X || !Y || !W || !sender || !recv_rowptr || !recv_edges || !coef || !out) {
    set_error("conv_tp_fwd: null pointer");
    return MB_E_ARG;
  }
  const size_t shm = (size_t)nO * MB_C * 4 + (size_t)n_terms * 20;
  if (shm > 48 * 1024 && cudaFuncSetAttribute(k_conv_tp_fwd, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)shm)) {
    set_error("conv_tp_fwd: cannot reserve %zu bytes of shared memory", shm);
    return MB_E_CUDA;
  }
  k_conv_tp_fwd<<<n_nodes, MB_C, shm, (cudaStream_t)stream>>>(X, nX, Y, nY, W, nW, sender, recv_rowptr, recv_edges,
                                                              n_nodes, (const int4*)terms_wkmo, coef, n_terms, out, nO,
                                                              status);
  return check_launch("conv_tp_fwd");
}

extern "C" int mace_b200_conv_tp_bwd(const float* X, int32_t nX, const float* Y, int32_t nY, const float* W,
                                     int32_t nW, const int32_t* sender, const int32_t* receiver,
                                     const int64_t* recv_rowptr, const int64_t* recv_edges,
                                     const int64_t* send_rowptr, const int64_t* send_edges, int32_t n_nodes,
                                     const int32_t* terms_wkmo, const float* coef, int32_t n_terms, const float* g,
                                     int32_t nO, float* dX, float* dY, float* dW, uint32_t* status, void* stream) {
  if (int rc = conv_args(terms_wkmo, n_terms, nX, nY, nW, nO, n_nodes, "conv_tp_bwd")) return rc;
  if (n_nodes == 0) return 0;
  if (!X || !Y || !W || !sender || !receiver || !recv_rowptr || !recv_edges || !coef || !g ||
      (dX && (!send_rowptr || !send_edges))) {
    set_error("conv_tp_bwd: null pointer");
    return MB_E_ARG;
  }
  cudaStream_t st = (cudaStream_t)stream;
  if (dW || dY) {
    const size_t shm = (size_t)(nO + nW + nY) * MB_C * 4 + 4 * (size_t)nY * 4 + (size_t)n_terms * 20;
    if (shm > 48 * 1024 &&
        cudaFuncSetAttribute(k_conv_tp_bwd_wy, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)shm)) {
      set_error("conv_tp_bwd: cannot reserve %zu bytes of shared memory", shm);
      return MB_E_CUDA;
    }
    k_conv_tp_bwd_wy<<<n_nodes, MB_C, shm, st>>>(X, nX, Y, nY, W, nW, sender, recv_rowptr, recv_edges, n_nodes,
                                                 (const int4*)terms_wkmo, coef, n_terms, g, nO, dY, dW, status);
    if (int rc = check_launch("conv_tp_bwd_wy")) return rc;
  }
  if (dX) {
    const size_t shm = (size_t)nX * MB_C * 4 + (size_t)n_terms * 20;
    if (shm > 48 * 1024 &&
        cudaFuncSetAttribute(k_conv_tp_bwd_x, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)shm)) {
      set_error("conv_tp_bwd: cannot reserve %zu bytes of shared memory", shm);
      return MB_E_CUDA;
    }
    k_conv_tp_bwd_x<<<n_nodes, MB_C, shm, st>>>(Y, nY, W, nW, receiver, send_rowptr, send_edges, n_nodes,
                                                (const int4*)terms_wkmo, coef, n_terms, g, nO, dX, nX, status);
    if (int rc = check_launch("conv_tp_bwd_x")) return rc;
  }
  return 0;
}
