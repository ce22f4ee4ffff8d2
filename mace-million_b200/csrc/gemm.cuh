// Grouped node GEMM problems: one launch serves up to kMaxGemmProblems independent problems
//   Y[atom][yoff + m][:] (+)= alpha_atom * sum_s X[atom][xoff_s + m][:] @ B_s,  N = 128, K = nseg * 128,
// rows r = t * mult + m, atom = order ? order[t] : t, alpha = 1 / (rho[atom] + 1) when rho is set.
// The CTA -> problem map is a prefix table of tile counts in the launch parameters (__grid_constant__).
#pragma once

#include "common.cuh"

namespace mb {

constexpr int kMaxGemmProblems = 16;

struct GemmProblem {
  const float* X;
  int64_t ldx;
  int xoff[4];
  int nseg;
  const float* B;      // SIMT: row-major [nseg][128 k][128 n]; tcgen05: K-major hi plane [nseg][128 n][128 k]
  int64_t plane;       // tcgen05: elements from the hi plane to the lo plane
  float* Y;
  int64_t ldy;
  int yoff;
  int mult;
  const int* order;
  int n_atoms;
  const float* rho;
  int accumulate;
};

struct GemmGroup {
  int n;
  int tile_start[kMaxGemmProblems + 1];
  GemmProblem p[kMaxGemmProblems];
  unsigned* status;
};

__device__ __forceinline__ int gemm_problem_of(const GemmGroup& grp, int tile) {
  int pi = 0;
  while (pi + 1 < grp.n && tile >= grp.tile_start[pi + 1]) ++pi;
  return pi;
}

int gemm_group_launch_simt(const GemmGroup& grp, cudaStream_t st);
void timer_begin(int kind, cudaStream_t st, int* slot);   // per-kind CUDA-event timing (passes.cu)
void timer_end(int slot, cudaStream_t st);
int gemm_group_launch_tc(const GemmGroup& grp, cudaStream_t st);

// Host-side builder: add problems, launch once (flushes automatically when full).
struct GemmBatch {
  GemmGroup g{};
  bool tc = false;
  cudaStream_t st = nullptr;

  GemmBatch(bool use_tc, unsigned* status, cudaStream_t stream) : tc(use_tc), st(stream) {
    g.n = 0;
    g.status = status;
  }

  int add(const float* X, int64_t ldx, const int32_t* xoff, int nseg, const float* B, int64_t plane, float* Y,
          int64_t ldy, int yoff, int mult, const int32_t* order, int n_atoms, const float* rho, int accumulate) {
    if (n_atoms <= 0) return 0;
    if (!X || !B || !Y || !xoff || nseg < 1 || nseg > 4 || mult < 1 || (ldx % 4) || (ldy % 4) || (tc && plane <= 0)) {
      set_error("node_gemm: bad arguments (nseg %d, mult %d)", nseg, mult);
      return MB_E_ARG;
    }
    if (g.n == kMaxGemmProblems) {
      int rc = launch();
      if (rc) return rc;
    }
    GemmProblem& p = g.p[g.n++];
    p.X = X;
    p.ldx = ldx;
    for (int s = 0; s < 4; ++s) p.xoff[s] = s < nseg ? xoff[s] : 0;
    p.nseg = nseg;
    p.B = B;
    p.plane = plane;
    p.Y = Y;
    p.ldy = ldy;
    p.yoff = yoff;
    p.mult = mult;
    p.order = order;
    p.n_atoms = n_atoms;
    p.rho = rho;
    p.accumulate = accumulate;
    return 0;
  }

  int launch() {
    if (g.n == 0) return 0;
    int slot;
    timer_begin(MB_K_NODE_GEMM, st, &slot);
    int rc = tc ? gemm_group_launch_tc(g, st) : gemm_group_launch_simt(g, st);
    timer_end(slot, st);
    g.n = 0;
    return rc;
  }
};

}  // namespace mb
