// Generic fused channelwise tensor product with explicit per-edge weights: the body of FusedConvTP
// (replaces the cuEquivariance segmented polynomial of the reference, mace_onegpu/fused_conv.py:20-37):
//   out[recv_e][o][c] += sum_terms coef W[e][w][c] X[send_e][k][c] Y[e][m]
// One CTA per edge, one thread per channel; the term table is a runtime argument (any path table), receivers need
// not be sorted (atomic scatter).  The hot path of the three passes uses the spline-fused edge kernels instead.
#include "common.cuh"

namespace mb {

__global__ void __launch_bounds__(128) k_conv_tp_fwd(const float* __restrict__ X, int nX, const float* __restrict__ Y,
                                                     int nY, const float* __restrict__ W, int nW,
                                                     const int* __restrict__ snd, const int* __restrict__ rcv,
                                                     int n_nodes, const int4* __restrict__ terms,
                                                     const float* __restrict__ coef, int nT, float* __restrict__ out,
                                                     int nO, unsigned* status) {
  const int64_t e = blockIdx.x;
  const int c = threadIdx.x;
  const int s = snd[e], r = rcv[e];
  if (s < 0 || s >= n_nodes || r < 0 || r >= n_nodes) {
    if (c == 0) set_status(status, ST_BAD_SENDER);
    return;
  }
  const float* xs = X + (int64_t)s * nX * MB_C + c;
  const float* we = W + e * nW * MB_C + c;
  const float* ye = Y + e * nY;
  float* orow = out + (int64_t)r * nO * MB_C + c;
  for (int t = 0; t < nT; ++t) {
    const int4 q = terms[t];   // (w, k, m, o)
    atomicAdd(orow + q.w * MB_C, coef[t] * we[q.x * MB_C] * xs[q.y * MB_C] * ye[q.z]);
  }
}

__global__ void __launch_bounds__(128) k_conv_tp_bwd(const float* __restrict__ X, int nX, const float* __restrict__ Y,
                                                     int nY, const float* __restrict__ W, int nW,
                                                     const int* __restrict__ snd, const int* __restrict__ rcv,
                                                     int n_nodes, const int4* __restrict__ terms,
                                                     const float* __restrict__ coef, int nT,
                                                     const float* __restrict__ g, int nO, float* __restrict__ dX,
                                                     float* __restrict__ dY, float* __restrict__ dW, unsigned* status) {
  const int64_t e = blockIdx.x;
  const int c = threadIdx.x;
  const int s = snd[e], r = rcv[e];
  if (s < 0 || s >= n_nodes || r < 0 || r >= n_nodes) {
    if (c == 0) set_status(status, ST_BAD_SENDER);
    return;
  }
  const float* xs = X + (int64_t)s * nX * MB_C + c;
  const float* we = W + e * nW * MB_C + c;
  const float* ye = Y + e * nY;
  const float* gr = g + (int64_t)r * nO * MB_C + c;
  float* dwe = dW ? dW + e * nW * MB_C + c : nullptr;
  float* dxs = dX ? dX + (int64_t)s * nX * MB_C + c : nullptr;
  for (int t = 0; t < nT; ++t) {
    const int4 q = terms[t];
    const float gc = coef[t] * gr[q.w * MB_C];
    const float xv = xs[q.y * MB_C], wv = we[q.x * MB_C], yv = ye[q.z];
    if (dwe) dwe[q.x * MB_C] += gc * xv * yv;       // this thread owns dW[e][*][c]
    if (dxs) atomicAdd(dxs + q.y * MB_C, gc * wv * yv);
    if (dY) {
      float p = warp_sum(gc * wv * xv);
      if ((c & 31) == 0) atomicAdd(dY + e * nY + q.z, p);
    }
  }
}

}  // namespace mb

using namespace mb;

extern "C" int mace_b200_conv_tp_fwd(const float* X, int32_t nX, const float* Y, int32_t nY, const float* W,
                                     int32_t nW, const int32_t* sender, const int32_t* receiver, int64_t E,
                                     int32_t n_nodes, const int32_t* terms_wkmo, const float* coef, int32_t n_terms,
                                     float* out, int32_t nO, uint32_t* status, void* stream) {
  if (E == 0) return 0;
  if (!X || !Y || !W || !sender || !receiver || !terms_wkmo || !coef || !out || E < 0 || n_terms <= 0) {
    set_error("conv_tp_fwd: bad arguments");
    return MB_E_ARG;
  }
  k_conv_tp_fwd<<<(unsigned)E, 128, 0, (cudaStream_t)stream>>>(X, nX, Y, nY, W, nW, sender, receiver, n_nodes,
                                                                (const int4*)terms_wkmo, coef, n_terms, out, nO, status);
  return check_launch("conv_tp_fwd");
}

extern "C" int mace_b200_conv_tp_bwd(const float* X, int32_t nX, const float* Y, int32_t nY, const float* W,
                                     int32_t nW, const int32_t* sender, const int32_t* receiver, int64_t E,
                                     int32_t n_nodes, const int32_t* terms_wkmo, const float* coef, int32_t n_terms,
                                     const float* g, int32_t nO, float* dX, float* dY, float* dW, uint32_t* status,
                                     void* stream) {
  if (E == 0) return 0;
  if (!X || !Y || !W || !sender || !receiver || !terms_wkmo || !coef || !g || E < 0 || n_terms <= 0) {
    set_error("conv_tp_bwd: bad arguments");
    return MB_E_ARG;
  }
  k_conv_tp_bwd<<<(unsigned)E, 128, 0, (cudaStream_t)stream>>>(X, nX, Y, nY, W, nW, sender, receiver, n_nodes,
                                                                (const int4*)terms_wkmo, coef, n_terms, g, nO, dX, dY,
                                                                dW, status);
  return check_launch("conv_tp_bwd");
}
