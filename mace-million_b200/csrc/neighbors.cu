// Full neighbour lists on the GPU (input preparation of the standalone driver and of the multi-GPU ghosts; the force
// evaluation itself takes the pair list as given, like the ML-IAP boundary).  Cell list with cells of at least
// r_cut, 27 candidate cells per atom, the algorithm of the reference's System.build_neighbors
// (mace_onegpu/receiver_chunk_mace.py:114-165): a count pass and a fill pass over the same candidates, one warp per
// receiver.  Candidates are visited in a fixed order (cell offsets dx, dy, dz = -1..1 nested, atoms of a cell in the
// caller's cell-sorted order), hits are compacted with ballots, so the output is deterministic.
//
// Periodic mode: orthorhombic box, minimum image, at least 3 cells per dimension (no candidate is seen twice).
// Open mode: cells over the caller's bounding box, no wrap (explicit ghost images).
// The Verlet filter keeps, per receiver, the pairs of a skin list that are within r_cut at the current positions.
#include "common.cuh"

namespace mb {

struct CellGrid {
  double lo[3], inv_w[3], box[3];
  int nc[3];
  int periodic;
};

__device__ __forceinline__ int cell_coord(double x, double lo, double inv_w, int nc) {
  int c = (int)floor((x - lo) * inv_w);
  return c < 0 ? 0 : (c >= nc ? nc - 1 : c);
}

__device__ __forceinline__ void min_image(double& d, double box, int periodic) {
  if (periodic) d -= box * rint(d / box);
}

// Visits the candidates of receiver i (one warp); fn(k_first_of_pass, hit_mask, j, dx, dy, dz) per 32-wide step.
template <typename Fn>
__device__ __forceinline__ void for_candidates(const double* __restrict__ pos, const int* __restrict__ cell_start,
                                               const int* __restrict__ cell_atoms, const CellGrid& g, int i, double r2,
                                               Fn fn) {
  const int lane = threadIdx.x & 31;
  const double xi = pos[3 * (int64_t)i], yi = pos[3 * (int64_t)i + 1], zi = pos[3 * (int64_t)i + 2];
  const int ci[3] = {cell_coord(xi, g.lo[0], g.inv_w[0], g.nc[0]), cell_coord(yi, g.lo[1], g.inv_w[1], g.nc[1]),
                     cell_coord(zi, g.lo[2], g.inv_w[2], g.nc[2])};
  for (int ox = -1; ox <= 1; ++ox)
    for (int oy = -1; oy <= 1; ++oy)
      for (int oz = -1; oz <= 1; ++oz) {
        int c3[3] = {ci[0] + ox, ci[1] + oy, ci[2] + oz};
        bool ok = true;
#pragma unroll
        for (int d = 0; d < 3; ++d) {
          if (c3[d] < 0 || c3[d] >= g.nc[d]) {
            if (!g.periodic) ok = false;
            c3[d] = (c3[d] + g.nc[d]) % g.nc[d];
          }
        }
        if (!ok) continue;
        const int c = (c3[0] * g.nc[1] + c3[1]) * g.nc[2] + c3[2];
        const int s = cell_start[c], e = cell_start[c + 1];
        for (int k0 = s; k0 < e; k0 += 32) {
          const int k = k0 + lane;
          int j = -1;
          double dx = 0.0, dy = 0.0, dz = 0.0;
          bool hit = false;
          if (k < e) {
            j = cell_atoms[k];
            dx = xi - pos[3 * (int64_t)j];
            dy = yi - pos[3 * (int64_t)j + 1];
            dz = zi - pos[3 * (int64_t)j + 2];
            min_image(dx, g.box[0], g.periodic);
            min_image(dy, g.box[1], g.periodic);
            min_image(dz, g.box[2], g.periodic);
            hit = j != i && dx * dx + dy * dy + dz * dz < r2;
          }
          fn(__ballot_sync(0xffffffffu, hit), hit, j, dx, dy, dz);
        }
      }
}

__global__ void k_nbr_count(const double* __restrict__ pos, const int* __restrict__ cell_start,
                            const int* __restrict__ cell_atoms, const CellGrid g, int n_recv, double r2,
                            int* __restrict__ counts) {
  const int i = (int)(((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  if (i >= n_recv) return;
  int cnt = 0;
  for_candidates(pos, cell_start, cell_atoms, g, i, r2,
                 [&](unsigned mask, bool, int, double, double, double) { cnt += __popc(mask); });
  if ((threadIdx.x & 31) == 0) counts[i] = cnt;
}

__global__ void k_nbr_fill(const double* __restrict__ pos, const int* __restrict__ cell_start,
                           const int* __restrict__ cell_atoms, const CellGrid g, int n_recv, double r2,
                           const int64_t* __restrict__ rowptr, int* __restrict__ pi, int* __restrict__ pj,
                           double* __restrict__ rij, unsigned* __restrict__ status) {
  const int i = (int)(((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  if (i >= n_recv) return;
  const int lane = threadIdx.x & 31;
  int64_t o = rowptr[i];
  const int64_t end = rowptr[i + 1];
  for_candidates(pos, cell_start, cell_atoms, g, i, r2,
                 [&](unsigned mask, bool hit, int j, double dx, double dy, double dz) {
                   if (hit) {
                     const int64_t q = o + __popc(mask & ((1u << lane) - 1u));
                     if (q < end) {
                       pi[q] = i;
                       pj[q] = j;
                       rij[3 * q] = dx;
                       rij[3 * q + 1] = dy;
                       rij[3 * q + 2] = dz;
                     }
                   }
                   o += __popc(mask);
                 });
  if (lane == 0 && o != end) set_status(status, ST_BAD_ROWPTR);   // positions changed between count and fill
}

// Verlet filter: pairs [vrow[i], vrow[i+1]) of receiver i (senders vj) that are within r_cut now.
template <bool FILL>
__global__ void k_verlet_filter(const double* __restrict__ pos, const CellGrid g, int n_recv,
                                const int64_t* __restrict__ vrow, const int* __restrict__ vj, double r2,
                                int* __restrict__ counts, const int64_t* __restrict__ rowptr, int* __restrict__ pi,
                                int* __restrict__ pj, double* __restrict__ rij, unsigned* __restrict__ status) {
  const int i = (int)(((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  if (i >= n_recv) return;
  const int lane = threadIdx.x & 31;
  const double xi = pos[3 * (int64_t)i], yi = pos[3 * (int64_t)i + 1], zi = pos[3 * (int64_t)i + 2];
  const int64_t s = vrow[i], e = vrow[i + 1];
  int64_t o = FILL ? rowptr[i] : 0;
  for (int64_t k0 = s; k0 < e; k0 += 32) {
    const int64_t k = k0 + lane;
    bool hit = false;
    int j = -1;
    double dx = 0.0, dy = 0.0, dz = 0.0;
    if (k < e) {
      j = vj[k];
      dx = xi - pos[3 * (int64_t)j];
      dy = yi - pos[3 * (int64_t)j + 1];
      dz = zi - pos[3 * (int64_t)j + 2];
      min_image(dx, g.box[0], g.periodic);
      min_image(dy, g.box[1], g.periodic);
      min_image(dz, g.box[2], g.periodic);
      hit = dx * dx + dy * dy + dz * dz < r2;
    }
    const unsigned mask = __ballot_sync(0xffffffffu, hit);
    if (FILL && hit) {
      const int64_t q = o + __popc(mask & ((1u << lane) - 1u));
      if (q < rowptr[i + 1]) {
        pi[q] = i;
        pj[q] = j;
        rij[3 * q] = dx;
        rij[3 * q + 1] = dy;
        rij[3 * q + 2] = dz;
      }
    }
    o += __popc(mask);
  }
  if (lane == 0) {
    if (!FILL)
      counts[i] = (int)o;
    else if (o != rowptr[i + 1])
      set_status(status, ST_BAD_ROWPTR);
  }
}

static int make_grid(const double* lo, const double* width, const int32_t* nc, const double* box, int periodic,
                     CellGrid& g, const char* who) {
  for (int d = 0; d < 3; ++d) {
    if (nc[d] < 1 || !(width[d] > 0.0) || (periodic && (nc[d] < 3 || !(box[d] > 0.0)))) {
      set_error("%s: bad cell grid (dimension %d: %d cells of %g; periodic boxes need >= 3 cells)", who, d, nc[d],
                width[d]);
      return MB_E_ARG;
    }
    g.lo[d] = lo[d];
    g.inv_w[d] = 1.0 / width[d];
    g.nc[d] = nc[d];
    g.box[d] = periodic ? box[d] : 0.0;
  }
  g.periodic = periodic ? 1 : 0;
  return 0;
}

static inline unsigned warp_blocks(int n) { return (unsigned)(((int64_t)n * 32 + 255) / 256); }

}  // namespace mb

using namespace mb;

extern "C" int mace_b200_nbr_count(const double* pos, const int32_t* cell_start, const int32_t* cell_atoms,
                                   const double* lo, const double* width, const int32_t* nc, const double* box,
                                   int32_t periodic, int32_t n_recv, double r_cut, int32_t* counts, void* stream) {
  CellGrid g;
  if (int rc = make_grid(lo, width, nc, box, periodic, g, "nbr_count")) return rc;
  if (!pos || !cell_start || !cell_atoms || !counts || n_recv < 0) {
    set_error("nbr_count: null pointer or negative size");
    return MB_E_ARG;
  }
  if (n_recv == 0) return 0;
  k_nbr_count<<<warp_blocks(n_recv), 256, 0, (cudaStream_t)stream>>>(pos, cell_start, cell_atoms, g, n_recv,
                                                                      r_cut * r_cut, counts);
  return check_launch("nbr_count");
}

extern "C" int mace_b200_nbr_fill(const double* pos, const int32_t* cell_start, const int32_t* cell_atoms,
                                  const double* lo, const double* width, const int32_t* nc, const double* box,
                                  int32_t periodic, int32_t n_recv, double r_cut, const int64_t* rowptr, int32_t* pi,
                                  int32_t* pj, double* rij, uint32_t* status, void* stream) {
  CellGrid g;
  if (int rc = make_grid(lo, width, nc, box, periodic, g, "nbr_fill")) return rc;
  if (!pos || !cell_start || !cell_atoms || !rowptr || !pi || !pj || !rij || n_recv < 0) {
    set_error("nbr_fill: null pointer or negative size");
    return MB_E_ARG;
  }
  if (n_recv == 0) return 0;
  k_nbr_fill<<<warp_blocks(n_recv), 256, 0, (cudaStream_t)stream>>>(pos, cell_start, cell_atoms, g, n_recv,
                                                                     r_cut * r_cut, rowptr, pi, pj, rij, status);
  return check_launch("nbr_fill");
}

extern "C" int mace_b200_verlet_filter(const double* pos, const double* box, int32_t periodic, int32_t n_recv,
                                       const int64_t* vrow, const int32_t* vj, double r_cut, int32_t* counts,
                                       const int64_t* rowptr, int32_t* pi, int32_t* pj, double* rij,
                                       uint32_t* status, void* stream) {
  if (!pos || !vrow || !vj || n_recv < 0 || (periodic && !box) || (!counts && !(rowptr && pi && pj && rij))) {
    set_error("verlet_filter: null pointer or negative size");
    return MB_E_ARG;
  }
  CellGrid g{};
  g.periodic = periodic ? 1 : 0;
  for (int d = 0; d < 3; ++d) g.box[d] = periodic ? box[d] : 0.0;
  if (n_recv == 0) return 0;
  const double r2 = r_cut * r_cut;
  if (counts)
    k_verlet_filter<false><<<warp_blocks(n_recv), 256, 0, (cudaStream_t)stream>>>(pos, g, n_recv, vrow, vj, r2, counts,
                                                                                  nullptr, nullptr, nullptr, nullptr,
                                                                                  status);
  else
    k_verlet_filter<true><<<warp_blocks(n_recv), 256, 0, (cudaStream_t)stream>>>(pos, g, n_recv, vrow, vj, r2, nullptr,
                                                                                 rowptr, pi, pj, rij, status);
  return check_launch("verlet_filter");
}

// ------------------------------------------------------------------------------------------------ CSR rows
// Row pointer of one receiver chunk [a, b) of a receiver-sorted pair list whose edges of the chunk are [e0, e1):
// rowptr[i] = first e in [e0, e1) with pair_i[e] >= i (e1 if none), i = a .. b.  It lets the host stream the pair
// list to the device chunk by chunk (the chunks' edge ranges come from a host binary search of the pinned pair_i)
// and verifies the sortedness that search assumed: an edge whose receiver lies outside [a, b) or below its
// predecessor's sets MB_ST_UNSORTED, and the host then evaluates again from a sorted copy.
namespace mb {
__global__ void k_csr_rows(const int32_t* __restrict__ pi, int64_t e0, int64_t e1, int a, int b,
                           int32_t* __restrict__ rowptr, unsigned* __restrict__ status) {
  const int64_t t0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x, stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t q = t0; q <= (int64_t)(b - a); q += stride) {
    const int i = a + (int)q;
    int64_t lo = e0, hi = e1;
    while (lo < hi) {
      const int64_t mid = (lo + hi) >> 1;
      if (__ldg(pi + mid) < i) lo = mid + 1;
      else hi = mid;
    }
    rowptr[i] = (int32_t)lo;
  }
  bool bad = false;
  for (int64_t e = e0 + t0; e < e1; e += stride) {
    const int p = __ldg(pi + e);
    bad |= p < a || p >= b || (e > e0 && p < __ldg(pi + e - 1));
  }
  if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) set_status(status, MB_ST_UNSORTED);
}
// Smallest and largest sender of a chunk's edges: out = (min, max) of pair_j[e0, e1), combined with atomics into
// the (INT32_MAX, -1) that k_range_init wrote (an empty range leaves those).
__global__ void k_range_init(int32_t* out) {
  out[0] = INT32_MAX;
  out[1] = -1;
}

__global__ void k_sender_range(const int32_t* __restrict__ pj, int64_t e0, int64_t e1, int32_t* out) {
  int lo = INT32_MAX, hi = -1;
  for (int64_t e = e0 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < e1; e += (int64_t)gridDim.x * blockDim.x) {
    const int j = __ldg(pj + e);
    lo = min(lo, j);
    hi = max(hi, j);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  if ((threadIdx.x & 31) == 0 && hi >= 0) {
    atomicMin(out, lo);
    atomicMax(out + 1, hi);
  }
}
}  // namespace mb

extern "C" int mace_b200_sender_range(const int32_t* pair_j, int64_t e0, int64_t e1, int32_t* out, void* stream) {
  if (!pair_j || !out || e0 < 0 || e1 < e0) {
    set_error("sender_range: bad arguments (edges [%lld, %lld))", (long long)e0, (long long)e1);
    return MB_E_ARG;
  }
  k_range_init<<<1, 1, 0, (cudaStream_t)stream>>>(out);
  if (int rc = check_launch("sender_range")) return rc;
  if (e1 == e0) return 0;
  const int64_t blocks = (e1 - e0 + 1023) / 1024 < 296 ? (e1 - e0 + 1023) / 1024 : 296;
  k_sender_range<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(pair_j, e0, e1, out);
  return check_launch("sender_range");
}

extern "C" int mace_b200_csr_rows(const int32_t* pair_i, int64_t e0, int64_t e1, int32_t a, int32_t b,
                                  int32_t* rowptr, uint32_t* status, void* stream) {
  if (!pair_i || !rowptr || !status || e0 < 0 || e1 < e0 || e1 > INT32_MAX || a < 0 || b < a) {
    set_error("csr_rows: bad arguments (edges [%lld, %lld), receivers [%d, %d))", (long long)e0, (long long)e1, a, b);
    return MB_E_ARG;
  }
  const int64_t work = (e1 - e0) > (int64_t)(b - a) + 1 ? (e1 - e0) : (int64_t)(b - a) + 1;
  const int64_t blocks = (work + 255) / 256 < 1184 ? (work + 255) / 256 : 1184;
  k_csr_rows<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(pair_i, e0, e1, a, b, rowptr, status);
  return check_launch("csr_rows");
}
