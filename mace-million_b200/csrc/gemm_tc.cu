// Node GEMM on the 5th-generation tensor cores (tcgen05, TMEM accumulator), 3xTF32 for fp32-level accuracy:
//   Y[atom][yoff + m][:] (+)= alpha_atom * sum_s X[atom][xoff_s + m][:] @ B_s
// with A = X rows gathered per (atom, m) and B given K-major and pre-split on the host into tf32 hi / lo planes
// (Bt[n][k], plane stride `plane`).  A is split on the fly: a_hi = rna_tf32(a), a_lo = rna_tf32(a - a_hi), and
// D = a_hi b_hi + a_hi b_lo + a_lo b_hi accumulates in fp32 in TMEM (the lo*lo term, ~2^-22 relative, is dropped).
//
// CTA: 256 threads, tile 128 rows x 128 columns, K blocks of 32 (one 128-byte SWIZZLE_128B atom of tf32 per row),
// two smem stages (A hi/lo + B hi/lo = 64 KB each) released by tcgen05.commit -> mbarrier.  One thread issues the
// MMAs (M = 128, N = 128, K = 8 per instruction, cta_group::1); the epilogue reads TMEM with tcgen05.ld 32x32b.
// Every mbarrier wait is bounded: on expiry the kernel records MB_ST_TC_TIMEOUT in the status word, still waits
// (bounded) for its own MMAs, frees its TMEM and exits without writing.
#include "gemm.cuh"

namespace mb {

constexpr int TC_BM = 128, TC_BN = 128, TC_BK = 32;
constexpr int TC_THREADS = 256;
constexpr int TC_TILE_BYTES = TC_BM * TC_BK * 4;          // 16 KB per operand plane
constexpr int TC_STAGE_BYTES = 4 * TC_TILE_BYTES;          // A hi, A lo, B hi, B lo
constexpr int TC_STAGES = 2;
constexpr int TC_SMEM = TC_STAGES * TC_STAGE_BYTES + 1024 + 64;   // + alignment slack + barriers
constexpr unsigned long long TC_WAIT_LIMIT = 1ull << 26;  // try_wait iterations before giving up

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// SWIZZLE_128B K-major canonical layout: 8-row groups of 1024 B, row r at (r % 8) * 128 inside its group, 16-byte
// chunk c stored at chunk position c ^ (r % 8).
__device__ __forceinline__ uint32_t sw128_offset(int row, int chunk) {
  return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((chunk ^ (row & 7)) << 4));
}

// UMMA shared-memory descriptor (sm_100): start >> 4 in [0,14), LBO (unused for swizzled K-major, 1) in [16,30),
// SBO = 1024 B between 8-row groups in [32,46), version 1 in [46,48), layout SWIZZLE_128B = 2 in [61,64).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor, kind::tf32: D fp32 (bits 4-5 = 1), A / B tf32 (bits 7-9, 10-12 = 2), both K-major,
// N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t tf32_idesc(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Bounded wait for the phase with the given parity; returns false when the limit expired.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_u32(bar);
  for (unsigned long long it = 0; it < TC_WAIT_LIMIT; ++it) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

__global__ void __launch_bounds__(TC_THREADS, 1) k_gemm_tc(const __grid_constant__ GemmGroup grp) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + TC_STAGES * TC_STAGE_BYTES);   // [2] stage barriers
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + TC_STAGES);
  __shared__ int s_failed;
  const int pi = gemm_problem_of(grp, blockIdx.x);
  const GemmProblem& g = grp.p[pi];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t nrows = (int64_t)g.n_atoms * g.mult;
  const int64_t r0 = (int64_t)(blockIdx.x - grp.tile_start[pi]) * TC_BM;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TC_BN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    for (int s = 0; s < TC_STAGES; ++s) mbar_init(&bar[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_failed = 0;
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  // A row owned by this thread (two threads per row, 16 floats = 4 chunks each of the 32-float K block)
  const int arow_i = tid >> 1, ahalf = tid & 1;
  const float* arow = nullptr;
  {
    const int64_t r = r0 + arow_i;
    if (r < nrows) {
      const int64_t t = r / g.mult;
      const int mm = (int)(r - t * g.mult);
      const int64_t at = g.order ? g.order[t] : t;
      arow = g.X + at * g.ldx + (int64_t)mm * MB_C;
    }
  }
  const int nK = g.nseg * (MB_C / TC_BK);
  const uint32_t idesc = tf32_idesc(TC_BM, TC_BN);
  // register prefetch of one K block: A (4 float4 of this thread's row half), B hi / lo (4 float4 each)
  float4 ra[4], rbh[4], rbl[4];
  auto load_block = [&](int kb) {
    const int seg = (kb * TC_BK) / MB_C, kin = kb * TC_BK - seg * MB_C;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      ra[q] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (arow) ra[q] = *reinterpret_cast<const float4*>(arow + (int64_t)g.xoff[seg] * MB_C + kin + (ahalf * 4 + q) * 4);
    }
    const float* bseg = g.B + (int64_t)seg * MB_C * MB_C + kin;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int idx = tid + q * TC_THREADS;          // 0 .. 1023 over (n, chunk)
      const float* src = bseg + (int64_t)(idx >> 3) * MB_C + (idx & 7) * 4;
      rbh[q] = __ldg(reinterpret_cast<const float4*>(src));
      rbl[q] = __ldg(reinterpret_cast<const float4*>(src + g.plane));
    }
  };
  load_block(0);
  bool ok = true;
  for (int kb = 0; kb < nK; ++kb) {
    const int s = kb & 1;
    if (kb >= TC_STAGES) {
      if (!mbar_wait(&bar[s], (uint32_t)(((kb - TC_STAGES) / TC_STAGES) & 1))) ok = false;
    }
    unsigned char* st = smem + s * TC_STAGE_BYTES;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 v = ra[q];
      float4 hi, lo;
      hi.x = tf32_rna(v.x); lo.x = tf32_rna(v.x - hi.x);
      hi.y = tf32_rna(v.y); lo.y = tf32_rna(v.y - hi.y);
      hi.z = tf32_rna(v.z); lo.z = tf32_rna(v.z - hi.z);
      hi.w = tf32_rna(v.w); lo.w = tf32_rna(v.w - hi.w);
      const uint32_t off = sw128_offset(arow_i, ahalf * 4 + q);
      *reinterpret_cast<float4*>(st + off) = hi;
      *reinterpret_cast<float4*>(st + TC_TILE_BYTES + off) = lo;
      const int idx = tid + q * TC_THREADS;
      const uint32_t boff = sw128_offset(idx >> 3, idx & 7);
      *reinterpret_cast<float4*>(st + 2 * TC_TILE_BYTES + boff) = rbh[q];
      *reinterpret_cast<float4*>(st + 3 * TC_TILE_BYTES + boff) = rbl[q];
    }
    if (kb + 1 < nK) load_block(kb + 1);             // in flight while this block is issued
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (tid == 0) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t a_hi = smem_u32(st), a_lo = a_hi + TC_TILE_BYTES;
      const uint32_t b_hi = a_hi + 2 * TC_TILE_BYTES, b_lo = a_hi + 3 * TC_TILE_BYTES;
#pragma unroll
      for (int kk = 0; kk < TC_BK / 8; ++kk) {
        const uint32_t ko = kk * 32;                 // 8 tf32 = 32 bytes along K inside the swizzle atom
        mma_tf32(tmem, sw128_desc(a_hi + ko), sw128_desc(b_hi + ko), idesc, (kb > 0 || kk > 0) ? 1u : 0u);
        mma_tf32(tmem, sw128_desc(a_hi + ko), sw128_desc(b_lo + ko), idesc, 1u);
        mma_tf32(tmem, sw128_desc(a_lo + ko), sw128_desc(b_hi + ko), idesc, 1u);
      }
      mma_commit(&bar[s]);
    }
  }
  // all MMAs done: the last commit covers every earlier tcgen05 op of the issuing thread
  {
    const int kl = nK - 1;
    if (!mbar_wait(&bar[kl & 1], (uint32_t)((kl / TC_STAGES) & 1))) ok = false;
  }
  if (!ok) s_failed = 1;
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (s_failed) {
    if (tid == 0) set_status(grp.status, MB_ST_TC_TIMEOUT);
  } else {
    // epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31 (rows), columns (w / 4) * 64 .. +63
    const int lrow = (warp & 3) * 32 + lane;
    const int col0 = (warp >> 2) * 64;
    const int64_t r = r0 + lrow;
    float v[64];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t x[32];
      const uint32_t taddr = tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)(col0 + 32 * h);
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
          "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
          : "=r"(x[0]), "=r"(x[1]), "=r"(x[2]), "=r"(x[3]), "=r"(x[4]), "=r"(x[5]), "=r"(x[6]), "=r"(x[7]),
            "=r"(x[8]), "=r"(x[9]), "=r"(x[10]), "=r"(x[11]), "=r"(x[12]), "=r"(x[13]), "=r"(x[14]), "=r"(x[15]),
            "=r"(x[16]), "=r"(x[17]), "=r"(x[18]), "=r"(x[19]), "=r"(x[20]), "=r"(x[21]), "=r"(x[22]), "=r"(x[23]),
            "=r"(x[24]), "=r"(x[25]), "=r"(x[26]), "=r"(x[27]), "=r"(x[28]), "=r"(x[29]), "=r"(x[30]), "=r"(x[31])
          : "r"(taddr));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
      for (int j = 0; j < 32; ++j) v[32 * h + j] = __uint_as_float(x[j]);
    }
    if (r < nrows) {
      const int64_t t = r / g.mult;
      const int mm = (int)(r - t * g.mult);
      const int64_t at = g.order ? g.order[t] : t;
      const float alpha = g.rho ? 1.f / (g.rho[at] + 1.f) : 1.f;
      float* y = g.Y + at * g.ldy + (int64_t)(g.yoff + mm) * MB_C + col0;
#pragma unroll
      for (int j = 0; j < 64; j += 4) {
        float4 o = make_float4(v[j] * alpha, v[j + 1] * alpha, v[j + 2] * alpha, v[j + 3] * alpha);
        float4* yp = reinterpret_cast<float4*>(y + j);
        if (g.accumulate) {
          const float4 p = *yp;
          o.x += p.x; o.y += p.y; o.z += p.z; o.w += p.w;
        }
        *yp = o;
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_BN) : "memory");
  }
}

static bool g_tc_attr_set = false;

int gemm_group_launch_tc(const GemmGroup& grp0, cudaStream_t st) {
  if (!g_tc_attr_set) {
    if (cudaFuncSetAttribute(k_gemm_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM) != cudaSuccess) {
      set_error("node_gemm_tc: cannot reserve %d bytes of shared memory", TC_SMEM);
      return MB_E_CUDA;
    }
    g_tc_attr_set = true;
  }
  GemmGroup grp = grp0;
  int tiles = 0;
  for (int q = 0; q < grp.n; ++q) {
    grp.tile_start[q] = tiles;
    tiles += (int)(((int64_t)grp.p[q].n_atoms * grp.p[q].mult + TC_BM - 1) / TC_BM);
  }
  grp.tile_start[grp.n] = tiles;
  if (tiles == 0) return 0;
  k_gemm_tc<<<tiles, TC_THREADS, TC_SMEM, st>>>(grp);
  return check_launch("node_gemm_tc");
}

}  // namespace mb

using namespace mb;

extern "C" int mace_b200_node_gemm_tc(const float* X, int64_t ldx, const int32_t* xoff, int32_t n_seg,
                                      const float* Bt_split, int64_t plane, float* Y, int64_t ldy, int32_t yoff,
                                      int32_t mult, const int32_t* order, int32_t n_atoms, const float* rho,
                                      int32_t accumulate, uint32_t* status, void* stream) {
  GemmBatch bt(true, status, (cudaStream_t)stream);
  int rc = bt.add(X, ldx, xoff, n_seg, Bt_split, plane, Y, ldy, yoff, mult, order, n_atoms, rho, accumulate);
  return rc ? rc : bt.launch();
}
