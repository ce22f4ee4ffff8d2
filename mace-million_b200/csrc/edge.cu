// Edge kernels of the three passes: one CTA per receiver, one thread per channel (C = 128).  Each batch of edges
// first runs a per-edge prologue (one thread per edge: length, SH, spline interval, density, SH Jacobian) into
// shared memory; then every thread walks the batch for its channel.  Replaces the reference's ConvSpline
// (mace_onegpu/conv_spline.py:38-94), SplineW (spline_w.py:30-75) and the cuEquivariance fused convolution with its
// autograd backward (fused_conv.py:33-37, mliap_threepass.py:549-581).
#include "common.cuh"
#include "tp_gen.cuh"

namespace mb {

struct EdgeCtx {
  Radial rd;
  int S, nt;
  int64_t P;
};

__device__ __forceinline__ EdgeCtx make_ctx(const mb_model_t& m, const mb_eval_t& ev) {
  EdgeCtx x;
  x.rd.r_max = m.r_max;
  x.rd.p = m.p_cut;
  x.rd.r_lo = m.r_lo;
  x.rd.inv_h = m.inv_h;
  x.rd.M = m.M;
  x.S = m.S;
  x.nt = ev.nt;
  x.P = ev.P;
  return x;
}

// Common per-edge checks and geometry.  Returns false (and records a status bit) for an edge that must be skipped.
__device__ __forceinline__ bool edge_geom(const mb_eval_t& ev, const EdgeCtx& x, int64_t e, int i, float3& v, float& r,
                                          int& j, int& pair) {
  j = ev.pair_j[e];
  const int pi = ev.pair_i[e];
  if (pi != i) {
    set_status(ev.status, ST_BAD_RECEIVER);
    return false;
  }
  if (j < 0 || j >= x.nt) {
    set_status(ev.status, ST_BAD_SENDER);
    return false;
  }
  const int ss = ev.spec[j], sr = ev.spec[i];
  if (ss < 0 || ss >= x.S || sr < 0 || sr >= x.S) {
    set_status(ev.status, ST_BAD_SPECIES);
    return false;
  }
  const double* rp = ev.rij + 3 * e;
  v = make_float3((float)rp[0], (float)rp[1], (float)rp[2]);
  r = sqrtf(v.x * v.x + v.y * v.y + v.z * v.z);
  if (!(r > 0.f) || !isfinite(r)) {
    set_status(ev.status, ST_NONFINITE);
    return false;
  }
  pair = ss * x.S + sr;
  return true;
}

// Table index of an ordered species pair (bitwise-identical per-pair tables share one table; null map = identity).
__device__ __forceinline__ int table_of(int pair, const int32_t* map) { return map ? __ldg(map + pair) : pair; }

__device__ __forceinline__ bool row_range(const mb_eval_t& ev, int i, int64_t& e0, int64_t& e1) {
  e0 = ev.rowptr[i];
  e1 = ev.rowptr[i + 1];
  if (e0 < 0 || e1 < e0 || e1 > ev.P) {
    set_status(ev.status, ST_BAD_ROWPTR);
    return false;
  }
  return true;
}

// SH values and the Jacobian dY/dv (v = r u): dY/dv = (grad_u Y - u (u . grad_u Y)) / r.
__device__ __forceinline__ void sh_jacobian(float3 u, float r, float* Y, float* J) {
  D3 ux = {u.x, 1.f, 0.f, 0.f}, uy = {u.y, 0.f, 1.f, 0.f}, uz = {u.z, 0.f, 0.f, 1.f};
  D3 Yd[16];
  sh16<D3>(ux, uy, uz, Yd);
  const float ir = 1.f / r;
#pragma unroll
  for (int q = 0; q < 16; ++q) {
    Y[q] = Yd[q].v;
    float ug = u.x * Yd[q].dx + u.y * Yd[q].dy + u.z * Yd[q].dz;
    J[3 * q + 0] = (Yd[q].dx - u.x * ug) * ir;
    J[3 * q + 1] = (Yd[q].dy - u.y * ug) * ir;
    J[3 * q + 2] = (Yd[q].dz - u.z * ug) * ir;
  }
}

__device__ __forceinline__ float cubic(float4 q, float t) { return fmaf(fmaf(fmaf(q.w, t, q.z), t, q.y), t, q.x); }

__device__ __forceinline__ float block_sum128(float v, float* red4) {
  v = warp_sum(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red4[threadIdx.x >> 5] = v;
  __syncthreads();
  return red4[0] + red4[1] + red4[2] + red4[3];
}

// ------------------------------------------------------------------------------------------------ layer 1
// Layer-1 edge kernels (pass A / C forward: s_msg[i][lm][c] = sum_e T1(r_e; pair_e)[l][c] Y_e[lm], s_rho[i];
// pass C backward: PF[e] += dL/dv_e from g = dL/dmsg1 in s_msg and s_grho): one warp per receiver, lane = channels lane + 32 j (j = 0..3, so every load and store
// of the warp is one contiguous 512-byte row); the warp's lanes run the per-edge prologue for batches of 32 edges
// into warp-private shared memory; 4 receivers per CTA, no CTA-wide barrier.  The backward forms per lane
// Q[lm] = sum_{its 4 channels} g[lm][c] T[l][c] and contracts it with the SH Jacobian once per 4 channels.
constexpr int L1_WARPS = 4;
#ifndef MB_L1_FWD_MINB
#define MB_L1_FWD_MINB 4
#endif
#ifndef MB_L1_BWD_MINB
#define MB_L1_BWD_MINB 4
#endif

__global__ void __launch_bounds__(32 * L1_WARPS, MB_L1_FWD_MINB) k_edge_l1_fwd(const mb_model_t m, const mb_eval_t ev, int a, int b) {
  __shared__ __align__(16) float sY[L1_WARPS][32][16];
  __shared__ int srow[L1_WARPS][32];
  __shared__ float st[L1_WARPS][32];
  const EdgeCtx x = make_ctx(m, ev);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int il = blockIdx.x * L1_WARPS + warp, i = a + il;
  if (i >= b) return;
  int64_t e0, e1;
  if (!row_range(ev, i, e0, e1)) return;
  const float4* tab = reinterpret_cast<const float4*>(m.tab1);
  float acc[16][4];
#pragma unroll
  for (int q = 0; q < 16; ++q) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.f;
  float rho = 0.f;
  for (int64_t base = e0; base < e1; base += 32) {
    const int n = (int)min((int64_t)32, e1 - base);
    __syncwarp();
    if (lane < n) {
      float3 v;
      float r;
      int j, pair;
      int row = -1;
      if (edge_geom(ev, x, base + lane, i, v, r, j, pair)) {
        int k;
        float t;
        spline_coords(r, x.rd, k, t);
        row = (table_of(pair, m.tab1_map) * (x.rd.M - 1) + k) * 4 * MB_C;
        st[warp][lane] = t;
        const float ir = 1.f / r;
        float Y[16];
        sh16<float>(v.x * ir, v.y * ir, v.z * ir, Y);
#pragma unroll
        for (int q = 0; q < 16; ++q) sY[warp][lane][q] = Y[q];
        float ed, ded;
        edge_density(r, m.wd1, x.rd.r_max, x.rd.p, ed, ded);
        rho += ed;
      }
      srow[warp][lane] = row;
    }
    __syncwarp();
    for (int q = 0; q < n; ++q) {
      const int row = srow[warp][q];
      if (row < 0) continue;
      const float t = st[warp][q];
      const float4* rw = tab + row + lane;
      float Y[16];
#pragma unroll
      for (int k = 0; k < 16; k += 4) {
        const float4 y4 = *reinterpret_cast<const float4*>(&sY[warp][q][k]);
        Y[k] = y4.x; Y[k + 1] = y4.y; Y[k + 2] = y4.z; Y[k + 3] = y4.w;
      }
#pragma unroll
      for (int l = 0; l < 4; ++l) {
        float T[4];
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) T[jj] = cubic(tab_ld(rw + l * MB_C + 32 * jj), t);
#pragma unroll
        for (int mm = l * l; mm < (l + 1) * (l + 1); ++mm)
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) acc[mm][jj] = fmaf(T[jj], Y[mm], acc[mm][jj]);
      }
    }
  }
  float* out = ev.s_msg + (size_t)il * 16 * MB_C + lane;
#pragma unroll
  for (int q = 0; q < 16; ++q)
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) out[q * MB_C + 32 * jj] = acc[q][jj];
  rho = warp_sum(rho);
  if (lane == 0) ev.s_rho[il] = rho;
}

__global__ void __launch_bounds__(32 * L1_WARPS, MB_L1_BWD_MINB) k_edge_l1_bwd(const mb_model_t m, const mb_eval_t ev,
                                                                              int a, int b) {
  __shared__ __align__(16) float sY[L1_WARPS][32][16];
  __shared__ __align__(16) float sred[L1_WARPS][32][17];
  __shared__ __align__(16) float sv[L1_WARPS][32][4];
  __shared__ float sgd[L1_WARPS][32];
  __shared__ int srow[L1_WARPS][32];
  __shared__ float st[L1_WARPS][32];
  const EdgeCtx x = make_ctx(m, ev);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int il = blockIdx.x * L1_WARPS + warp, i = a + il;
  if (i >= b) return;
  int64_t e0, e1;
  if (!row_range(ev, i, e0, e1)) return;
  const float4* tab = reinterpret_cast<const float4*>(m.tab1);
  float g[16][4];
  const float* gin = ev.s_msg + (size_t)il * 16 * MB_C + lane;
#pragma unroll
  for (int q = 0; q < 16; ++q)
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) g[q][jj] = gin[q * MB_C + 32 * jj];
  const float grho = ev.s_grho[il];
  for (int64_t base = e0; base < e1; base += 32) {
    const int n = (int)min((int64_t)32, e1 - base);
    __syncwarp();
    if (lane < n) {
      float3 v;
      float r;
      int j, pair;
      int row = -1;
      if (edge_geom(ev, x, base + lane, i, v, r, j, pair)) {
        int k;
        float t;
        spline_coords(r, x.rd, k, t);
        row = (table_of(pair, m.tab1_map) * (x.rd.M - 1) + k) * 4 * MB_C;
        st[warp][lane] = t;
        const float ir = 1.f / r;
        sh16<float>(v.x * ir, v.y * ir, v.z * ir, sY[warp][lane]);
        float ed, ded;
        edge_density(r, m.wd1, x.rd.r_max, x.rd.p, ed, ded);
        sv[warp][lane][0] = v.x;
        sv[warp][lane][1] = v.y;
        sv[warp][lane][2] = v.z;
        sv[warp][lane][3] = r;
        sgd[warp][lane] = grho * ded;
      }
      srow[warp][lane] = row;
    }
    __syncwarp();
    for (int q = 0; q < n; ++q) {
      const int row = srow[warp][q];
      if (row < 0) continue;
      const float t = st[warp][q];
      const float4* rw = tab + row + lane;
      float Y[16];
#pragma unroll
      for (int k = 0; k < 16; k += 4) {
        const float4 y4 = *reinterpret_cast<const float4*>(&sY[warp][q][k]);
        Y[k] = y4.x; Y[k + 1] = y4.y; Y[k + 2] = y4.z; Y[k + 3] = y4.w;
      }
      // Q[lm] = sum_c g[lm][c] T_l[c] (dE/dY, slot 0 unused: Y[0] is constant);  G_l[c] = sum_{m in l} g Y = dE/dT_l[c]
      float Q[16];
      float Sb = 0.f, Sc = 0.f, Sd = 0.f;
#pragma unroll
      for (int l = 0; l < 4; ++l) {
        float4 cq[4];
        float T[4], G[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          cq[jj] = tab_ld(rw + l * MB_C + 32 * jj);
          T[jj] = cubic(cq[jj], t);
        }
#pragma unroll
        for (int mm = l * l; mm < (l + 1) * (l + 1); ++mm) {
          float qv = 0.f;
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            qv = fmaf(g[mm][jj], T[jj], qv);
            G[jj] = fmaf(g[mm][jj], Y[mm], G[jj]);
          }
          Q[mm] = qv;
        }
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          Sb = fmaf(G[jj], cq[jj].y, Sb);
          Sc = fmaf(G[jj], cq[jj].z, Sc);
          Sd = fmaf(G[jj], cq[jj].w, Sd);
        }
      }
      Q[0] = fmaf(t, fmaf(3.f * t, Sd, 2.f * Sc), Sb);   // dE/dt of this lane's channels
      const float s = transpose_reduce16(Q, lane);
      if ((lane & 1) == 0) sred[warp][q][lane >> 1] = s;
    }
    __syncwarp();
    if (lane < n && srow[warp][lane] >= 0) {
      const float* gs = sred[warp][lane];
      const float r = sv[warp][lane][3], ir = 1.f / r;
      const float3 u = make_float3(sv[warp][lane][0] * ir, sv[warp][lane][1] * ir, sv[warp][lane][2] * ir);
      float Yj[16], J[48];
      sh_jacobian(u, r, Yj, J);
      const float gr = fmaf(gs[0], x.rd.inv_h, sgd[warp][lane]);
      float f[3] = {gr * u.x, gr * u.y, gr * u.z};
#pragma unroll
      for (int mm = 1; mm < 16; ++mm) {
        f[0] = fmaf(gs[mm], J[3 * mm + 0], f[0]);
        f[1] = fmaf(gs[mm], J[3 * mm + 1], f[1]);
        f[2] = fmaf(gs[mm], J[3 * mm + 2], f[2]);
      }
      float* pf = ev.PF + 3 * (base + lane);
#pragma unroll
      for (int d = 0; d < 3; ++d) pf[d] += f[d];
    }
  }
}

// ------------------------------------------------------------------------------------------------ layer 1, density form
// Exact density projection of layer 1 (mb_model_t.l1_density, S <= 2; derived in the reference's
// mace_onegpu/ace_layer1.py:2-16).  The layer-1 sender features depend only on the sender species and the radial
// MLP's last layer is linear, so the per-receiver densities B[s][q][m] = sum_{e: s_e = s} h_q(r_e) Y_m(e) of the 64
// hidden features h carry the whole message; the chunk's node GEMM (composite M0) maps them to x1.  One warp per
// receiver, lane = hidden features lane and lane + 32: per edge two 16-byte loads of a 64-column table (one table
// for every pair) instead of sixteen of a 512-column one, and 32 message FMAs per lane instead of 64.  The batch
// prologue orders the batch's edges by sender species (ballot prefix), so each species slot runs its own loop with
// its accumulators in registers and no per-edge branch.
constexpr int L1D_H = 64;
#ifndef MB_L1D_FWD_MINB
#define MB_L1D_FWD_MINB 4
#endif
#ifndef MB_L1D_BWD_MINB
#define MB_L1D_BWD_MINB 4
#endif


// Position of this lane's edge in the species-ordered batch (slot 0 first); returns the slot-0 count in n0 and the
// number of valid edges in nv.  Every lane of the warp calls it.
__device__ __forceinline__ int l1d_slot_order(bool ok, int slot, int lane, int& n0, int& nv) {
  const unsigned all = __ballot_sync(0xffffffffu, ok);
  const unsigned m1 = __ballot_sync(0xffffffffu, ok && slot == 1);
  const unsigned m0 = all & ~m1;
  const unsigned lt = (1u << lane) - 1u;
  n0 = __popc(m0);
  nv = __popc(all);
  return slot == 1 ? n0 + __popc(m1 & lt) : __popc(m0 & lt);
}

template <int NH>
__device__ __forceinline__ void l1d_accumulate(float (&B)[NH][16], const float (&h)[NH], const float* y) {
#pragma unroll
  for (int k = 0; k < 16; k += 4) {
    const float4 y4 = *reinterpret_cast<const float4*>(y + k);
    const float Y[4] = {y4.x, y4.y, y4.z, y4.w};
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int hh = 0; hh < NH; ++hh) B[hh][k + u] = fmaf(h[hh], Y[u], B[hh][k + u]);
  }
}

template <int NH>
__device__ __forceinline__ void l1d_fwd_edge(float (&B)[NH][16], const float4* rw, float t, const float* y) {
  float h[NH];
#pragma unroll
  for (int hh = 0; hh < NH; ++hh) h[hh] = cubic(tab_ld(rw + 32 * hh), t);
  l1d_accumulate<NH>(B, h, y);
}

__global__ void __launch_bounds__(32 * L1_WARPS, MB_L1D_FWD_MINB) k_edge_l1d_fwd(const mb_model_t m, const mb_eval_t ev,
                                                                                int a, int b) {
  constexpr int NH = 2;              // blocks of 32 hidden features per lane
  __shared__ __align__(16) float sY[L1_WARPS][32][16];
  __shared__ int srow[L1_WARPS][32];
  __shared__ float st[L1_WARPS][32];
  const EdgeCtx x = make_ctx(m, ev);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int il = blockIdx.x * L1_WARPS + warp, i = a + il;
  if (i >= b) return;
  int64_t e0, e1;
  if (!row_range(ev, i, e0, e1)) return;
  const float4* tab = reinterpret_cast<const float4*>(m.tab1) + lane;
  float B0[NH][16], B1[NH][16];      // densities of species slot 0 / 1: [hidden feature 32 hh + lane][m]
#pragma unroll
  for (int q = 0; q < 16; ++q)
#pragma unroll
    for (int hh = 0; hh < NH; ++hh) B0[hh][q] = B1[hh][q] = 0.f;
  float rho = 0.f;
  for (int64_t base = e0; base < e1; base += 32) {
    const int n = (int)min((int64_t)32, e1 - base);
    float3 v;
    float r = 0.f;
    int j, pair = 0;
    const bool ok = lane < n && edge_geom(ev, x, base + lane, i, v, r, j, pair);
    const int slot = ok ? pair / x.S : 0;
    int n0, nv;
    const int pos = l1d_slot_order(ok, slot, lane, n0, nv);
    if (ok) {
      int k;
      float t;
      spline_coords(r, x.rd, k, t);
      srow[warp][pos] = k * L1D_H;
      st[warp][pos] = t;
      const float ir = 1.f / r;
      sh16<float>(v.x * ir, v.y * ir, v.z * ir, sY[warp][pos]);
      float ed, ded;
      edge_density(r, m.wd1, x.rd.r_max, x.rd.p, ed, ded);
      rho += ed;
    }
    __syncwarp();
    for (int q = 0; q < n0; ++q) l1d_fwd_edge<NH>(B0, tab + srow[warp][q], st[warp][q], sY[warp][q]);
    for (int q = n0; q < nv; ++q) l1d_fwd_edge<NH>(B1, tab + srow[warp][q], st[warp][q], sY[warp][q]);
    __syncwarp();
  }
  float* out = ev.s_msg + (size_t)il * 16 * MB_C + lane;
#pragma unroll
  for (int q = 0; q < 16; ++q)
#pragma unroll
    for (int hh = 0; hh < NH; ++hh) {
      out[q * MB_C + 32 * hh] = B0[hh][q];
      out[q * MB_C + 64 + 32 * hh] = B1[hh][q];
    }
  rho = warp_sum(rho);
  if (lane == 0) ev.s_rho[il] = rho;
}

// One edge of the density backward: from g = dE/dB of the edge's species slot, dE/dh_q = sum_m g[q][m] Y_m (into
// the spline derivative) and this lane's share of dE/dY_m = sum_q g[q][m] h_q, reduced over the warp into sred.
// c0 / c1: this lane's two coefficient sets of the edge's table row.
__device__ __forceinline__ void l1d_edge_bwd(const float (&g)[2][16], float4 c0, float4 c1, float t, const float* y,
                                             float* sred_row, int lane) {
  const float h0 = cubic(c0, t), h1 = cubic(c1, t);
  float Y[16];
#pragma unroll
  for (int k = 0; k < 16; k += 4) {
    const float4 y4 = *reinterpret_cast<const float4*>(y + k);
    Y[k] = y4.x;
    Y[k + 1] = y4.y;
    Y[k + 2] = y4.z;
    Y[k + 3] = y4.w;
  }
  float Q[16];
  float G0a = 0.f, G0b = 0.f, G1a = 0.f, G1b = 0.f;
#pragma unroll
  for (int mm = 0; mm < 16; mm += 2) {
    G0a = fmaf(g[0][mm], Y[mm], G0a);
    G1a = fmaf(g[1][mm], Y[mm], G1a);
    G0b = fmaf(g[0][mm + 1], Y[mm + 1], G0b);
    G1b = fmaf(g[1][mm + 1], Y[mm + 1], G1b);
  }
#pragma unroll
  for (int mm = 1; mm < 16; ++mm) Q[mm] = fmaf(g[0][mm], h0, g[1][mm] * h1);
  const float G0 = G0a + G0b, G1 = G1a + G1b;
  const float Sb = fmaf(G0, c0.y, G1 * c1.y), Sc = fmaf(G0, c0.z, G1 * c1.z), Sd = fmaf(G0, c0.w, G1 * c1.w);
  Q[0] = fmaf(t, fmaf(3.f * t, Sd, 2.f * Sc), Sb);   // dE/dt of this lane's hidden features (Y_0 is constant)
  const float s = transpose_reduce16(Q, lane);
  if ((lane & 1) == 0) sred_row[lane >> 1] = s;
}

__global__ void __launch_bounds__(32 * L1_WARPS, MB_L1D_BWD_MINB) k_edge_l1d_bwd(const mb_model_t m, const mb_eval_t ev,
                                                                                int a, int b) {
  __shared__ __align__(16) float sY[L1_WARPS][32][16];
  __shared__ __align__(16) float sred[L1_WARPS][32][17];
  __shared__ __align__(16) float sv[L1_WARPS][32][4];
  __shared__ float sgd[L1_WARPS][32];
  __shared__ int srow[L1_WARPS][32];
  __shared__ int sedge[L1_WARPS][32];
  __shared__ float st[L1_WARPS][32];
  const EdgeCtx x = make_ctx(m, ev);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int il = blockIdx.x * L1_WARPS + warp, i = a + il;
  if (i >= b) return;
  int64_t e0, e1;
  if (!row_range(ev, i, e0, e1)) return;
  const float4* tab = reinterpret_cast<const float4*>(m.tab1) + lane;
  // dE/dB of this receiver, [m][slot * 64 + hh * 32 + lane]; each slot's 32 values are loaded (L1 hits after the
  // first batch) before that slot's edge loop, so that only one slot occupies registers
  const float* gin = ev.s_msg + (size_t)il * 16 * MB_C + lane;
  const float grho = ev.s_grho[il];
  for (int64_t base = e0; base < e1; base += 32) {
    const int n = (int)min((int64_t)32, e1 - base);
    float3 v;
    float r = 0.f;
    int j, pair = 0;
    const bool ok = lane < n && edge_geom(ev, x, base + lane, i, v, r, j, pair);
    const int slot = ok ? pair / x.S : 0;
    int n0, nv;
    const int pos = l1d_slot_order(ok, slot, lane, n0, nv);
    if (ok) {
      int k;
      float t;
      spline_coords(r, x.rd, k, t);
      srow[warp][pos] = k * L1D_H;
      st[warp][pos] = t;
      sedge[warp][pos] = lane;
      const float ir = 1.f / r;
      sh16<float>(v.x * ir, v.y * ir, v.z * ir, sY[warp][pos]);
      float ed, ded;
      edge_density(r, m.wd1, x.rd.r_max, x.rd.p, ed, ded);
      sv[warp][pos][0] = v.x;
      sv[warp][pos][1] = v.y;
      sv[warp][pos][2] = v.z;
      sv[warp][pos][3] = r;
      sgd[warp][pos] = grho * ded;
    }
    __syncwarp();
#pragma unroll 1
    for (int slot = 0; slot < 2; ++slot) {
      const int q0 = slot ? n0 : 0, q1 = slot ? nv : n0;
      if (q0 == q1) continue;
      float g[2][16];
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        g[0][q] = gin[q * MB_C + slot * 64];
        g[1][q] = gin[q * MB_C + slot * 64 + 32];
      }
      // the next edge's row is loaded before this edge's work, so its L2 round trip overlaps that work
      float4 c0 = tab_ld(tab + srow[warp][q0]), c1 = tab_ld(tab + srow[warp][q0] + 32);
      for (int q = q0; q < q1; ++q) {
        const int nx = srow[warp][min(q + 1, q1 - 1)];
        const float4 n0v = tab_ld(tab + nx), n1v = tab_ld(tab + nx + 32);
        l1d_edge_bwd(g, c0, c1, st[warp][q], sY[warp][q], sred[warp][q], lane);
        c0 = n0v;
        c1 = n1v;
      }
    }
    __syncwarp();
    if (lane < nv) {
      const float* gs = sred[warp][lane];
      const float r = sv[warp][lane][3], ir = 1.f / r;
      const float3 u = make_float3(sv[warp][lane][0] * ir, sv[warp][lane][1] * ir, sv[warp][lane][2] * ir);
      float Yj[16], J[48];
      sh_jacobian(u, r, Yj, J);
      const float gr = fmaf(gs[0], x.rd.inv_h, sgd[warp][lane]);
      float f[3] = {gr * u.x, gr * u.y, gr * u.z};
#pragma unroll
      for (int mm = 1; mm < 16; ++mm) {
        f[0] = fmaf(gs[mm], J[3 * mm + 0], f[0]);
        f[1] = fmaf(gs[mm], J[3 * mm + 1], f[1]);
        f[2] = fmaf(gs[mm], J[3 * mm + 2], f[2]);
      }
      float* pf = ev.PF + 3 * (base + sedge[warp][lane]);
#pragma unroll
      for (int d = 0; d < 3; ++d) pf[d] += f[d];
    }
    __syncwarp();
  }
}

// ------------------------------------------------------------------------------------------------ layer 2 forward
// Resident CTAs per SM the layer-2 kernels are compiled for (register budget 65536 / (128 x MINB) per thread).
// Forward, 1.03M-atom evaluation (128-edge batches): 4 CTAs 111.4 ms, 5: 115.5, 6: 107.2, 7 (72 registers, no
// spills): 104.9 ms.
#ifndef MB_L2_FWD_MINB
#define MB_L2_FWD_MINB 7
#endif
#ifndef MB_L2_BWD_MINB
#define MB_L2_BWD_MINB 4
#endif

// s_msg[i][o][c] = sum_e sum_(w,k,m) coef W2(r_e)[w][c] X2[j_e][k][c] Y_e[m];  s_rho[i]
// The products are formed per thread from Y_e in registers (tp2_fwd_y): keeping the 76 per-edge coefficients
// sum_m coef Y[m] in shared memory instead costs more L1 wavefronts than the extra FP32 work (125.4 against
// 107.2 ms at 6 CTAs / SM).
template <int EB>
__global__ void __launch_bounds__(128, MB_L2_FWD_MINB) k_edge_l2_fwd(const mb_model_t m, const mb_eval_t ev, int a) {
  __shared__ __align__(16) float sby[EB][16];   // SH values (the TP coefficients are formed per thread from them)
  __shared__ int srow[EB];
  __shared__ int ssend[EB];
  __shared__ float st[EB];
  __shared__ float red4[4];
  const EdgeCtx x = make_ctx(m, ev);
  const int il = blockIdx.x, i = a + il, c = threadIdx.x;
  int64_t e0, e1;
  if (!row_range(ev, i, e0, e1)) return;
  const float4* tab = reinterpret_cast<const float4*>(m.tab2);
  float acc[TP2_NO];
#pragma unroll
  for (int q = 0; q < TP2_NO; ++q) acc[q] = 0.f;
  float rho = 0.f;
  for (int64_t base = e0; base < e1; base += EB) {
    const int n = (int)min((int64_t)EB, e1 - base);
    __syncthreads();
    if (c < n) {
      float3 v;
      float r;
      int j, pair;
      int row = -1;
      if (edge_geom(ev, x, base + c, i, v, r, j, pair)) {
        int k;
        float t;
        spline_coords(r, x.rd, k, t);
        row = (table_of(pair, m.tab2_map) * (x.rd.M - 1) + k) * TP2_NW * MB_C;
        st[c] = t;
        ssend[c] = j;
        const float ir = 1.f / r;
        float Y[16];
        sh16<float>(v.x * ir, v.y * ir, v.z * ir, Y);
#pragma unroll
        for (int k = 0; k < 16; ++k) sby[c][k] = Y[k];
        float ed, ded;
        edge_density(r, m.wd2, x.rd.r_max, x.rd.p, ed, ded);
        rho += ed;
      }
      srow[c] = row;
    }
    __syncthreads();
    for (int q = 0; q < n; ++q) {
      const int row = srow[q];
      if (row < 0) continue;
      const float* xs = ev.X2 + (size_t)ssend[q] * 4 * MB_C + c;
      float X[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) X[k] = __ldg(xs + k * MB_C);
      float Y[16];
#pragma unroll
      for (int k = 0; k < 16; k += 4) {
        const float4 y4 = *reinterpret_cast<const float4*>(&sby[q][k]);
        Y[k] = y4.x; Y[k + 1] = y4.y; Y[k + 2] = y4.z; Y[k + 3] = y4.w;
      }
      tp2_fwd_y(tab + row + c, st[q], X, Y, acc);
    }
  }
  float* out = ev.s_msg + (size_t)il * TP2_NO * MB_C + c;
#pragma unroll
  for (int q = 0; q < TP2_NO; ++q) out[q * MB_C] = acc[q];
  rho = block_sum128(rho, red4);
  if (c == 0) ev.s_rho[il] = rho;
}

// ------------------------------------------------------------------------------------------------ layer 2 backward
// Pass B: given g = dE/dmsg2 (s_msg, [i][40][C]) and s_grho: PF[e] += dE/dv_e, GX2[j_e] += dE/dX2.
// Per receiver and channel the collapsed coefficients A = sum_o coef g[o] live in registers (tp2_a).  Per (edge,
// channel) the kernel forms dE/dY[1..15] and dE/dt (slot 0, Y[0] being constant); the 16 values are summed over the
// warp (transpose_reduce16) and over the 4 warps in shared memory, and one thread per edge applies the SH Jacobian
// and the spline's 1/h once.
template <int EB>
__global__ void __launch_bounds__(128, MB_L2_BWD_MINB) k_edge_l2_bwd(const mb_model_t m, const mb_eval_t ev, int a) {
  __shared__ __align__(16) float sY[EB][16];
  __shared__ __align__(16) float sv[EB][4];
  __shared__ __align__(16) float sred[EB][4 * 16 + 4];   // per edge: 4 warps x 16 slots, padded (bank spread)
  __shared__ float sgd[EB];
  __shared__ int srow[EB];
  __shared__ int ssend[EB];
  __shared__ float st[EB];
  const EdgeCtx x = make_ctx(m, ev);
  const int il = blockIdx.x, i = a + il, c = threadIdx.x, warp = c >> 5, lane = c & 31;
  int64_t e0, e1;
  if (!row_range(ev, i, e0, e1)) return;
  const float4* tab = reinterpret_cast<const float4*>(m.tab2);
  float A[TP2_NA];
  {
    float g[TP2_NO];
    const float* gin = ev.s_msg + (size_t)il * TP2_NO * MB_C + c;
#pragma unroll
    for (int q = 0; q < TP2_NO; ++q) g[q] = gin[q * MB_C];
    tp2_a(g, A);
  }
  const float grho = ev.s_grho[il];
  for (int64_t base = e0; base < e1; base += EB) {
    const int n = (int)min((int64_t)EB, e1 - base);
    __syncthreads();
    if (c < n) {
      float3 v;
      float r;
      int j, pair;
      int row = -1;
      if (edge_geom(ev, x, base + c, i, v, r, j, pair)) {
        int k;
        float t;
        spline_coords(r, x.rd, k, t);
        row = (table_of(pair, m.tab2_map) * (x.rd.M - 1) + k) * TP2_NW * MB_C;
        st[c] = t;
        ssend[c] = j;
        const float ir = 1.f / r;
        sh16<float>(v.x * ir, v.y * ir, v.z * ir, sY[c]);
        sv[c][0] = v.x;
        sv[c][1] = v.y;
        sv[c][2] = v.z;
        sv[c][3] = r;
        float ed, ded;
        edge_density(r, m.wd2, x.rd.r_max, x.rd.p, ed, ded);
        sgd[c] = grho * ded;
      }
      srow[c] = row;
    }
    __syncthreads();
    for (int q = 0; q < n; ++q) {
      const int row = srow[q];
      if (row < 0) continue;
      const int j = ssend[q];
      const float t = st[q];
      const float* xs = ev.X2 + (size_t)j * 4 * MB_C + c;
      float X[4], gX[4] = {0.f, 0.f, 0.f, 0.f}, gY[16], Y[16];
#pragma unroll
      for (int k = 0; k < 4; ++k) X[k] = __ldg(xs + k * MB_C);
#pragma unroll
      for (int k = 0; k < 16; k += 4) {
        const float4 y4 = *reinterpret_cast<const float4*>(&sY[q][k]);
        Y[k] = y4.x;
        Y[k + 1] = y4.y;
        Y[k + 2] = y4.z;
        Y[k + 3] = y4.w;
        gY[k] = gY[k + 1] = gY[k + 2] = gY[k + 3] = 0.f;
      }
      float Sb = 0.f, Sc = 0.f, Sd = 0.f;
      tp2_bwd(tab + row + c, t, X, Y, A, gX, gY, Sb, Sc, Sd);
      float* gxo = ev.GX2 + (size_t)j * 4 * MB_C + c;
#pragma unroll
      for (int k = 0; k < 4; ++k) atomicAdd(gxo + k * MB_C, gX[k]);
      gY[0] = fmaf(t, fmaf(3.f * t, Sd, 2.f * Sc), Sb);
      const float s = transpose_reduce16(gY, lane);
      if ((lane & 1) == 0) sred[q][warp * 16 + (lane >> 1)] = s;
    }
    __syncthreads();
    if (c < n && srow[c] >= 0) {
      float gs[16];
#pragma unroll
      for (int k = 0; k < 16; k += 4) {
        float4 acc4 = *reinterpret_cast<const float4*>(&sred[c][k]);
#pragma unroll
        for (int w = 1; w < 4; ++w) {
          const float4 o4 = *reinterpret_cast<const float4*>(&sred[c][w * 16 + k]);
          acc4.x += o4.x;
          acc4.y += o4.y;
          acc4.z += o4.z;
          acc4.w += o4.w;
        }
        gs[k] = acc4.x;
        gs[k + 1] = acc4.y;
        gs[k + 2] = acc4.z;
        gs[k + 3] = acc4.w;
      }
      const float r = sv[c][3], ir = 1.f / r;
      const float3 u = make_float3(sv[c][0] * ir, sv[c][1] * ir, sv[c][2] * ir);
      float Yj[16], J[48];
      sh_jacobian(u, r, Yj, J);
      const float gr = fmaf(gs[0], x.rd.inv_h, sgd[c]);
      float f[3] = {gr * u.x, gr * u.y, gr * u.z};
#pragma unroll
      for (int mm = 1; mm < 16; ++mm) {
        f[0] = fmaf(gs[mm], J[3 * mm + 0], f[0]);
        f[1] = fmaf(gs[mm], J[3 * mm + 1], f[1]);
        f[2] = fmaf(gs[mm], J[3 * mm + 2], f[2]);
      }
      float* pf = ev.PF + 3 * (base + c);
#pragma unroll
      for (int d = 0; d < 3; ++d) pf[d] += f[d];
    }
  }
}

// Edges per batch of the layer-2 kernels (one prologue, main loop and post-pass per batch).  128 covers a water
// receiver's ~90 edges in one batch, so the prologue and post-pass run on all four warps and once per receiver;
// measured on the 1.03M-atom evaluation: forward 112.9 -> 110.0 ms, backward 191.7 -> 188.3 ms (32: 114.7 / 195.6).
// The backward's static shared memory is 47 KB at 128.
#ifndef MB_L2F_EB
#define MB_L2F_EB 128
#endif
#ifndef MB_L2B_EB
#define MB_L2B_EB 128
#endif

// ------------------------------------------------------------------------------------------------ launchers
static int edge_args(const mb_model_t* m, const mb_eval_t* ev, int a, int b, const char* who) {
  if (!m || !ev || a < 0 || b > ev->nl || b < a) {
    set_error("%s: bad chunk [%d, %d)", who, a, b);
    return MB_E_ARG;
  }
  if (m->C != MB_C) {
    set_error("%s: only C = 128 is supported (got %d)", who, m->C);
    return MB_E_ARG;
  }
  if (m->l1_density && (m->S < 1 || m->S > 2)) {
    set_error("%s: the density-projection layer 1 supports 1 or 2 species (got %d)", who, m->S);
    return MB_E_ARG;
  }
  return 0;
}

}  // namespace mb

using namespace mb;

extern "C" int mace_b200_edge_l1_fwd(const mb_model_t* m, const mb_eval_t* ev, int32_t a, int32_t b, void* stream) {
  if (int rc = edge_args(m, ev, a, b, "edge_l1_fwd")) return rc;
  if (b == a) return 0;
  const int grid = (b - a + L1_WARPS - 1) / L1_WARPS;
  if (m->l1_density)
    k_edge_l1d_fwd<<<grid, 32 * L1_WARPS, 0, (cudaStream_t)stream>>>(*m, *ev, a, b);
  else
    k_edge_l1_fwd<<<grid, 32 * L1_WARPS, 0, (cudaStream_t)stream>>>(*m, *ev, a, b);
  return check_launch("edge_l1_fwd");
}

extern "C" int mace_b200_edge_l1_bwd(const mb_model_t* m, const mb_eval_t* ev, int32_t a, int32_t b, void* stream) {
  if (int rc = edge_args(m, ev, a, b, "edge_l1_bwd")) return rc;
  if (b == a) return 0;
  const int grid = (b - a + L1_WARPS - 1) / L1_WARPS;
  if (m->l1_density)
    k_edge_l1d_bwd<<<grid, 32 * L1_WARPS, 0, (cudaStream_t)stream>>>(*m, *ev, a, b);
  else
    k_edge_l1_bwd<<<grid, 32 * L1_WARPS, 0, (cudaStream_t)stream>>>(*m, *ev, a, b);
  return check_launch("edge_l1_bwd");
}

extern "C" int mace_b200_edge_l2_fwd(const mb_model_t* m, const mb_eval_t* ev, int32_t a, int32_t b, void* stream) {
  if (int rc = edge_args(m, ev, a, b, "edge_l2_fwd")) return rc;
  if (b == a) return 0;
  k_edge_l2_fwd<MB_L2F_EB><<<b - a, 128, 0, (cudaStream_t)stream>>>(*m, *ev, a);
  return check_launch("edge_l2_fwd");
}

extern "C" int mace_b200_edge_l2_bwd(const mb_model_t* m, const mb_eval_t* ev, int32_t a, int32_t b, void* stream) {
  if (int rc = edge_args(m, ev, a, b, "edge_l2_bwd")) return rc;
  if (b == a) return 0;
  k_edge_l2_bwd<MB_L2B_EB><<<b - a, 128, 0, (cudaStream_t)stream>>>(*m, *ev, a);
  return check_launch("edge_l2_bwd");
}
