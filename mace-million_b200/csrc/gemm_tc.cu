// Node GEMM on the 5th-generation tensor cores (tcgen05, TMEM accumulator), 3xTF32 for fp32-level accuracy:
//   Y[atom][yoff + m][:] (+)= alpha_atom * sum_s X[atom][xoff_s + m][:] @ B_s
// with A = X rows gathered per (atom, m) and B given as tf32 hi / lo planes, every 128 x 128 matrix stored as four
// 16 KB K blocks that are already in the SWIZZLE_128B K-major shared-memory image (host: engine.tc_planes).  A is
// split on the fly: a_hi = rna_tf32(a), a_lo = rna_tf32(a - a_hi), and D = a_hi b_hi + a_hi b_lo + a_lo b_hi
// accumulates in fp32 in TMEM (the lo*lo term, ~2^-22 relative, is dropped).
//
// Persistent, warp-specialised CTA (one per SM; TC_PG = 2, TC_EPW = 8: 544 threads), static round-robin over the
// 128-row tiles of all problems of the group:
//   producers  TC_PG groups of 4 warps; group g makes the K blocks g, g + TC_PG, .. of the CTA's sequence, so that
//              two blocks are split at a time.  Thread p of a group owns row p of the tile: its 128-byte slice of
//              each of the group's K blocks is prefetched TC_RAW blocks ahead with cp.async into the group's padded
//              raw ring (no registers held), then split into tf32 hi / lo and written with tcgen05.st into the
//              stage's A columns of TMEM (row p = TMEM lane p); the group's thread 0 also fetches the stage's B hi /
//              lo blocks into shared memory with two 16 KB cp.async.bulk copies (no multicast).
//   epilogue   TC_EPW warps: tcgen05.ld 32x32b of the finished accumulator (warp w reads TMEM lanes 32 (w % 4) ..,
//              one row per lane; with 8 warps each takes two of the four 32-column chunks), row scale 1 / (rho + 1),
//              a transpose through shared memory so that the stores (and the loads of the previous values when
//              accumulating, eight in flight per lane) are full 128-byte row segments; then release the accumulator.
//   last warp  barrier init, TMEM allocation (two 128-column accumulators + 64 A columns per stage) and, on
//              lane 0, the MMA issue: 12 tcgen05.mma kind::tf32 (M = N = 128, K = 8, A from TMEM, B from shared
//              memory) per K block, tcgen05.commit -> stage-empty barrier, and after a tile's last block ->
//              accumulator-full barrier.
// Measured on the 1.03M-atom evaluation (node GEMMs per evaluation): A staged in shared memory beside B, 4 producer
// and 4 epilogue warps 54.4 ms (each MMA then reads 8 KB of operands from shared memory, about what the SM's shared
// memory delivers at the MMA's rate); A in TMEM 49.5-50.1 ms, where a clock64 trace showed the epilogue (about
// 11k cycles per tile) and the serial split chain of each producer warp (1.3-2.5k cycles per K block) as the
// limits; per-lane 128-byte bulk stores from the epilogue 51.2 ms (the bulk-copy issue took ~2.5k cycles per chunk).
// The two accumulators let a tile's epilogue overlap the next tile's K loop.  Every mbarrier wait is bounded: on
// expiry the kernel records MB_ST_TC_TIMEOUT, every role stops, outstanding copies and MMAs are drained (bounded),
// the TMEM is freed and the kernel exits (outputs of unfinished tiles are not written).
#include "gemm.cuh"

namespace mb {

constexpr int TC_BM = 128, TC_BN = 128, TC_BK = 32;
constexpr int TC_TILE_BYTES = TC_BM * TC_BK * 4;          // 16 KB: one operand plane of one K block
#ifndef MB_TC_STAGES
#define MB_TC_STAGES 2
#endif
#ifndef MB_TC_RAW
#define MB_TC_RAW 3
#endif
#ifndef MB_TC_PG
#define MB_TC_PG 2
#endif
#ifndef MB_TC_EPW
#define MB_TC_EPW 4
#endif
constexpr int TC_STAGES = MB_TC_STAGES;                    // operand stages (B hi / lo in shared memory, A in TMEM)
constexpr int TC_PG = MB_TC_PG;                            // producer groups of 4 warps; group g makes K blocks g, g + TC_PG, ..
constexpr int TC_EPW = MB_TC_EPW;                          // epilogue warps (4: all chunks each; 8: two per warp)
constexpr int TC_STAGE_BYTES = 2 * TC_TILE_BYTES;          // B hi, B lo
constexpr int TC_TMEM_COLS = 512;                          // two accumulators + A hi / lo (2 x 32 columns) per stage
constexpr int TC_A_COL = 2 * TC_BN;                        // first TMEM column of the A stages
constexpr int TC_RAW = MB_TC_RAW;                          // cp.async depth of each group's raw A ring, in K blocks
constexpr int TC_RAW_ROW = 144;                            // one row's 128-byte K slice + 16 bytes of bank padding
constexpr int TC_RAW_BYTES = TC_BM * TC_RAW_ROW;
constexpr int TC_EPI_ROW = 33;                             // epilogue transpose: 32 floats per row + 1 (bank spread)
constexpr int TC_EPI_WARP_BYTES = 32 * TC_EPI_ROW * 4;     // one 32-row x 32-column chunk per epilogue warp
constexpr int TC_EPI_WARP0 = 4 * TC_PG;                    // first epilogue warp
constexpr int TC_MMA_WARP = TC_EPI_WARP0 + TC_EPW;
constexpr int TC_THREADS = 32 * (TC_MMA_WARP + 1);
static_assert(TC_EPW == 4 || TC_EPW == 8, "epilogue warps");
static_assert(TC_A_COL + TC_STAGES * 2 * TC_BK <= TC_TMEM_COLS, "TMEM columns");
constexpr int TC_RAW_OFF = TC_STAGES * TC_STAGE_BYTES;
constexpr int TC_EPI_OFF = TC_RAW_OFF + TC_PG * TC_RAW * TC_RAW_BYTES;
constexpr int TC_BAR_OFF = TC_EPI_OFF + TC_EPW * TC_EPI_WARP_BYTES;
constexpr int TC_SMEM = TC_BAR_OFF + 256 + 1024;           // + barriers / TMEM slot / flag + alignment slack
static_assert(TC_SMEM <= 227 * 1024, "shared memory per CTA");
// Every mbarrier wait gives up after g_tc_wait_ns nanoseconds of %globaltimer (default 2 s; a GEMM tile takes
// microseconds).  mace_b200_tc_test_hooks shortens it and can make one producer arrival go missing, so that a test
// drives the timeout path (MB_ST_TC_TIMEOUT, drain, TMEM release) without any fault.
__device__ unsigned long long g_tc_wait_ns = 2000000000ull;
__device__ int g_tc_skip_arrival = 0;

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
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

// One MMA, A read from TMEM (tmem_a: lane 0 and the first of the 8 columns of this K step, one row per lane), B from
// a SWIZZLE_128B K-major shared-memory image (8-row groups of 1024 B, row r at (r % 8) * 128, 16-byte chunk c at
// chunk position c ^ (r % 8); the host writes B in that image, engine.tc_planes)
__device__ __forceinline__ void mma_tf32_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// 32 consecutive TMEM columns of this warp's 32 lanes from 32 registers per thread (warp-collective)
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// Bounded wait for the phase with the given parity; returns false when g_tc_wait_ns expired (the clock is read every
// 256 polls).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_u32(bar);
  unsigned long long t0 = 0;
  for (uint32_t it = 0;; ++it) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
    if ((it & 255u) == 0u) {
      const unsigned long long now = globaltimer_ns();
      if (it == 0)
        t0 = now;
      else if (now - t0 > *(volatile unsigned long long*)&g_tc_wait_ns)
        return false;
    }
  }
}

// global -> this CTA's shared memory, completing on an mbarrier transaction count (16-byte aligned, bytes % 16 == 0)
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

struct TcBars {
  uint64_t full[TC_STAGES];       // 128 producer arrivals (A hi / lo stored)
  uint64_t bfull[TC_STAGES];      // 1 arrival + 32 KB of B bulk copies
  uint64_t empty[TC_STAGES];      // tcgen05.commit after the stage's MMAs
  uint64_t acc_full[2];           // tcgen05.commit after a tile's last K block
  uint64_t acc_empty[2];          // 128 epilogue arrivals
  uint32_t tmem;
  int failed;
};

// Row geometry of tile row `row` of global tile `tile`: problem index, K blocks, whether the row exists, and its
// atom (through the optional order: the load is issued here, its value is only used later, by tc_a / tc_y, so
// that the round trip overlaps other work) and component.
struct TcRow {
  int pi;
  int nk;
  bool valid;
  int mm;
  int64_t at;
};

__device__ __forceinline__ TcRow tc_row(const GemmGroup& grp, int tile, int row) {
  TcRow o;
  o.pi = gemm_problem_of(grp, tile);
  const GemmProblem& g = grp.p[o.pi];
  o.nk = g.nseg * (MB_C / TC_BK);
  const int64_t r = (int64_t)(tile - grp.tile_start[o.pi]) * TC_BM + row;
  o.valid = r < (int64_t)g.n_atoms * g.mult;
  o.mm = 0;
  o.at = 0;
  if (o.valid) {
    const int64_t t = r / g.mult;
    o.mm = (int)(r - t * g.mult);
    o.at = g.order ? (int64_t)g.order[t] : t;
  }
  return o;
}

__device__ __forceinline__ const float* tc_a(const GemmGroup& grp, const TcRow& w) {
  const GemmProblem& g = grp.p[w.pi];
  return w.valid ? g.X + w.at * g.ldx + (int64_t)w.mm * MB_C : nullptr;
}

__device__ __forceinline__ float* tc_y(const GemmGroup& grp, const TcRow& w) {
  const GemmProblem& g = grp.p[w.pi];
  return w.valid ? g.Y + w.at * g.ldy + (int64_t)(g.yoff + w.mm) * MB_C : nullptr;
}

// Cursor over this CTA's K blocks in order (tile = blockIdx.x + k gridDim.x, then kb): the tile's row geometry,
// and the next tile's, whose order load is issued one tile ahead (tc_row).
struct TcCursor {
  int tile, kb;
  TcRow rw, next;
  __device__ __forceinline__ void init(const GemmGroup& grp, int n_tiles, int row) {
    tile = blockIdx.x;
    kb = 0;
    rw = tc_row(grp, tile, row);
    next = tile + (int)gridDim.x < n_tiles ? tc_row(grp, tile + gridDim.x, row) : rw;
  }
  __device__ __forceinline__ void step(const GemmGroup& grp, int n_tiles, int row) {
    if (++kb == rw.nk) {
      kb = 0;
      tile += gridDim.x;
      rw = next;
      if (tile + (int)gridDim.x < n_tiles) next = tc_row(grp, tile + gridDim.x, row);
    }
  }
};

__global__ void __launch_bounds__(TC_THREADS, 1) k_gemm_tc(const __grid_constant__ GemmGroup grp, int n_tiles) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  TcBars& B = *reinterpret_cast<TcBars*>(smem + TC_BAR_OFF);
  volatile int* failed = &B.failed;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (warp == TC_MMA_WARP) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&B.tmem)),
                 "r"(TC_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    if (lane == 0) {
      for (int s = 0; s < TC_STAGES; ++s) {
        mbar_init(&B.full[s], 128);
        mbar_init(&B.bfull[s], 1);
        mbar_init(&B.empty[s], 1);
      }
      for (int a = 0; a < 2; ++a) {
        mbar_init(&B.acc_full[a], 1);
        mbar_init(&B.acc_empty[a], 32 * TC_EPW);
      }
      B.failed = 0;
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = B.tmem;

  if (warp < TC_EPI_WARP0) {
    // ------------------------------------------------------------------------------------------ producers
    // Group pg (warps 4 pg .. 4 pg + 3) makes the K blocks seq = pg, pg + TC_PG, ..; thread p of a group owns
    // row p of the tile (TMEM lane p: warp w reaches lanes 32 (w % 4) ..).
    const int pg = warp >> 2, p = tid & 127;
    unsigned char* raw = smem + TC_RAW_OFF + pg * TC_RAW * TC_RAW_BYTES;
    // issue cursor, TC_RAW of this group's blocks ahead of the consumer cursor
    TcCursor ic, cc;
    ic.init(grp, n_tiles, p);
    for (int q = 0; q < pg; ++q) ic.step(grp, n_tiles, p);
    cc = ic;
    auto issue_next = [&](int slot) {
      if (ic.tile < n_tiles) {
        if (ic.rw.valid) {
          const GemmProblem& g = grp.p[ic.rw.pi];
          const int seg = (ic.kb * TC_BK) / MB_C, kin = ic.kb * TC_BK - seg * MB_C;
          const float* src = tc_a(grp, ic.rw) + (int64_t)g.xoff[seg] * MB_C + kin;
          unsigned char* dst = raw + slot * TC_RAW_BYTES + p * TC_RAW_ROW;
#pragma unroll
          for (int q = 0; q < 8; ++q) cp_async16(dst + 16 * q, src + 4 * q);
        }
        for (int q = 0; q < TC_PG; ++q) ic.step(grp, n_tiles, p);
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
    };
#pragma unroll 1
    for (int q = 0; q < TC_RAW; ++q) issue_next(q);
    int last_b[TC_STAGES];                          // last seq whose B copies this thread issued, per stage
#pragma unroll
    for (int s = 0; s < TC_STAGES; ++s) last_b[s] = -1;
    // every exit decision is warp-uniform: the loop body holds warp-collective tcgen05.st.sync.aligned
    for (int seq = pg, j = 0; cc.tile < n_tiles; seq += TC_PG, ++j) {
      if (__shfl_sync(0xffffffffu, *failed, 0)) break;
      const int s = seq % TC_STAGES, slot = j % TC_RAW, kb = cc.kb;
      const GemmProblem& g = grp.p[cc.rw.pi];
      const bool have = cc.rw.valid;
      asm volatile("cp.async.wait_group %0;" ::"n"(TC_RAW - 1) : "memory");
      float4 v[8];
      const unsigned char* src = raw + slot * TC_RAW_BYTES + p * TC_RAW_ROW;
#pragma unroll
      for (int q = 0; q < 8; ++q)
        v[q] = have ? *reinterpret_cast<const float4*>(src + 16 * q) : make_float4(0.f, 0.f, 0.f, 0.f);
      issue_next(slot);                            // the slot has been read: refill it TC_RAW blocks ahead
      uint32_t ahi[32], alo[32];                   // split before the wait, so that the wait covers it
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float c4[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float h = tf32_rna(c4[k]);
          ahi[4 * q + k] = __float_as_uint(h);
          alo[4 * q + k] = __float_as_uint(tf32_rna(c4[k] - h));
        }
      }
      // stage s free once the MMAs of its previous use completed (first use: the preceding phase counts done)
      if (!__all_sync(0xffffffffu, mbar_wait(&B.empty[s], ((seq / TC_STAGES) & 1) ^ 1))) {
        *failed = 1;
        break;
      }
      if (p == 0) {
        unsigned char* st = smem + s * TC_STAGE_BYTES;
        const int seg = (kb * TC_BK) / MB_C, kin = kb * TC_BK - seg * MB_C;
        const float* bsrc = g.B + (int64_t)seg * MB_C * MB_C + (int64_t)(kin / TC_BK) * (TC_BM * TC_BK);
        mbar_arrive_tx(&B.bfull[s], 2 * TC_TILE_BYTES);
        bulk_g2s(st, bsrc, TC_TILE_BYTES, &B.bfull[s]);
        bulk_g2s(st + TC_TILE_BYTES, bsrc + g.plane, TC_TILE_BYTES, &B.bfull[s]);
        last_b[s] = seq;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t ta = tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)(TC_A_COL + s * 2 * TC_BK);
      tmem_st32(ta, ahi);
      tmem_st32(ta + TC_BK, alo);
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      // test hook (off unless mace_b200_tc_test_hooks armed it): one arrival of CTA 0's first K block goes missing
      const bool skip = seq == 0 && p == 0 && blockIdx.x == 0 && *(volatile int*)&g_tc_skip_arrival &&
                        atomicExch(&g_tc_skip_arrival, 0);
      if (!skip) mbar_arrive(&B.full[s]);
      for (int q = 0; q < TC_PG; ++q) cc.step(grp, n_tiles, p);
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    // after a timeout: B copies this thread issued may still be landing in the stages
    if (p == 0 && *failed)
      for (int s = 0; s < TC_STAGES; ++s)
        if (last_b[s] >= 0) mbar_wait(&B.bfull[s], (last_b[s] / TC_STAGES) & 1);
  } else if (warp < TC_MMA_WARP) {
    // ------------------------------------------------------------------------------------------ epilogue
    // Warp w reads TMEM lanes 32 (w % 4) .. (one tile row per lane) and handles the 32-column chunks
    // h = (w - TC_EPI_WARP0) / 4, + TC_EPW / 4, ..; each chunk is transposed through shared memory so that the
    // output stores (and, when accumulating, the loads of the previous values, all eight issued together) are full
    // 128-byte row segments, 4 rows per warp instruction.
    const int q4 = warp & 3, row = q4 * 32 + lane, e = warp - TC_EPI_WARP0;
    float* stg = reinterpret_cast<float*>(smem + TC_EPI_OFF + e * TC_EPI_WARP_BYTES);
    // lane l stores rows 4 i + l / 8 (i = 0..7), columns 4 (l % 8) .. + 3 of the chunk
    const int srow = lane >> 3, scol = (lane & 7) * 4;
    int tc = 0;
    // every exit decision is warp-uniform: the loop body holds warp-collective tcgen05.ld.sync.aligned
    for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++tc) {
      if (__shfl_sync(0xffffffffu, *failed, 0)) break;
      const int a = tc & 1;
      const TcRow rw = tc_row(grp, tile, row);     // its loads overlap the wait
      const GemmProblem& g = grp.p[rw.pi];
      float* y = tc_y(grp, rw);
      const float rho = (rw.valid && g.rho) ? g.rho[rw.at] : 0.f;
      float* yr[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        yr[i] = reinterpret_cast<float*>(__shfl_sync(0xffffffffu, reinterpret_cast<uintptr_t>(y), 4 * i + srow));
      if (!__all_sync(0xffffffffu, mbar_wait(&B.acc_full[a], (tc >> 1) & 1))) {
        *failed = 1;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const bool acc = g.accumulate != 0;
      const float alpha = 1.f / (rho + 1.f);
#pragma unroll 1
      for (int h = e >> 2; h < 4; h += TC_EPW / 4) {
        uint32_t x[32];
        const uint32_t taddr = tmem + ((uint32_t)(q4 * 32) << 16) + (uint32_t)(a * TC_BN + 32 * h);
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
            "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
            : "=r"(x[0]), "=r"(x[1]), "=r"(x[2]), "=r"(x[3]), "=r"(x[4]), "=r"(x[5]), "=r"(x[6]), "=r"(x[7]),
              "=r"(x[8]), "=r"(x[9]), "=r"(x[10]), "=r"(x[11]), "=r"(x[12]), "=r"(x[13]), "=r"(x[14]), "=r"(x[15]),
              "=r"(x[16]), "=r"(x[17]), "=r"(x[18]), "=r"(x[19]), "=r"(x[20]), "=r"(x[21]), "=r"(x[22]), "=r"(x[23]),
              "=r"(x[24]), "=r"(x[25]), "=r"(x[26]), "=r"(x[27]), "=r"(x[28]), "=r"(x[29]), "=r"(x[30]), "=r"(x[31])
            : "r"(taddr));
        float4 prev[8];
        if (acc) {
#pragma unroll
          for (int i = 0; i < 8; ++i)
            prev[i] = yr[i] ? *reinterpret_cast<const float4*>(yr[i] + 32 * h + scol) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        __syncwarp();                                // the previous chunk's reads of the staging area are done
#pragma unroll
        for (int k = 0; k < 32; ++k) stg[lane * TC_EPI_ROW + k] = __uint_as_float(x[k]) * alpha;
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float* sv = stg + (4 * i + srow) * TC_EPI_ROW + scol;
          float4 o = make_float4(sv[0], sv[1], sv[2], sv[3]);
          if (acc) {
            o.x += prev[i].x; o.y += prev[i].y; o.z += prev[i].z; o.w += prev[i].w;
          }
          if (yr[i]) *reinterpret_cast<float4*>(yr[i] + 32 * h + scol) = o;
        }
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      mbar_arrive(&B.acc_empty[a]);
    }
  } else if (lane == 0) {
    // ------------------------------------------------------------------------------------------ MMA issue
    const uint32_t idesc = tf32_idesc(TC_BM, TC_BN);
    int seq = 0, tc = 0;
    uint64_t* last_bar = nullptr;
    uint32_t last_par = 0;
    for (int tile = blockIdx.x; tile < n_tiles && !*failed; tile += gridDim.x, ++tc) {
      const int a = tc & 1;
      if (!mbar_wait(&B.acc_empty[a], ((tc >> 1) & 1) ^ 1)) {
        *failed = 1;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int nk = grp.p[gemm_problem_of(grp, tile)].nseg * (MB_C / TC_BK);
      bool ok = true;
      for (int kb = 0; kb < nk; ++kb, ++seq) {
        const int s = seq % TC_STAGES;
        const uint32_t ph = (seq / TC_STAGES) & 1;
        if (!mbar_wait(&B.full[s], ph) || !mbar_wait(&B.bfull[s], ph)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t d = tmem + (uint32_t)(a * TC_BN);
        const uint32_t b_hi = smem_u32(smem + s * TC_STAGE_BYTES), b_lo = b_hi + TC_TILE_BYTES;
        const uint32_t a_hi = tmem + (uint32_t)(TC_A_COL + s * 2 * TC_BK), a_lo = a_hi + TC_BK;
#pragma unroll
        for (int kk = 0; kk < TC_BK / 8; ++kk) {
          const uint32_t ko = kk * 32;               // 8 tf32 = 32 bytes along K inside B's swizzle atom
          mma_tf32_ts(d, a_hi + 8 * kk, sw128_desc(b_hi + ko), idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          mma_tf32_ts(d, a_hi + 8 * kk, sw128_desc(b_lo + ko), idesc, 1u);
          mma_tf32_ts(d, a_lo + 8 * kk, sw128_desc(b_hi + ko), idesc, 1u);
        }
        mma_commit(&B.empty[s]);
        last_bar = &B.empty[s];
        last_par = ph;
      }
      if (!ok) {
        *failed = 1;
        break;
      }
      mma_commit(&B.acc_full[a]);
      last_bar = &B.acc_full[a];
      last_par = (tc >> 1) & 1;
    }
    // after a timeout: wait (bounded) for the MMAs already issued before the TMEM is freed
    if (*failed && last_bar) mbar_wait(last_bar, last_par);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  // after every role has stopped: a producer that never had to wait may finish before the MMA thread gives up
  if (tid == 0 && *failed) set_status(grp.status, MB_ST_TC_TIMEOUT);
  if (warp == TC_MMA_WARP) {
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_TMEM_COLS) : "memory");
  }
}

static int g_tc_attr_dev = -1;
static int g_tc_sms = 0;

int gemm_group_launch_tc(const GemmGroup& grp0, cudaStream_t st) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return check_launch("node_gemm_tc (device)");
  if (g_tc_attr_dev != dev) {
    if (cudaFuncSetAttribute(k_gemm_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM) != cudaSuccess) {
      set_error("node_gemm_tc: cannot reserve %d bytes of shared memory", TC_SMEM);
      return MB_E_CUDA;
    }
    if (cudaDeviceGetAttribute(&g_tc_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || g_tc_sms < 1) {
      set_error("node_gemm_tc: cannot query the SM count");
      return MB_E_CUDA;
    }
    g_tc_attr_dev = dev;
  }
  GemmGroup grp = grp0;
  int tiles = 0;
  for (int q = 0; q < grp.n; ++q) {
    const GemmProblem& p = grp.p[q];
    if ((reinterpret_cast<uintptr_t>(p.X) | reinterpret_cast<uintptr_t>(p.Y) | reinterpret_cast<uintptr_t>(p.B)) & 15 ||
        (p.plane % 4)) {
      set_error("node_gemm_tc: X, Y and B must be 16-byte aligned (and the plane stride a multiple of 4)");
      return MB_E_ARG;
    }
    grp.tile_start[q] = tiles;
    tiles += (int)(((int64_t)p.n_atoms * p.mult + TC_BM - 1) / TC_BM);
  }
  grp.tile_start[grp.n] = tiles;
  if (tiles == 0) return 0;
  const int grid = tiles < g_tc_sms ? tiles : g_tc_sms;
  k_gemm_tc<<<grid, TC_THREADS, TC_SMEM, st>>>(grp, tiles);
  return check_launch("node_gemm_tc");
}

}  // namespace mb

using namespace mb;

extern "C" int mace_b200_tc_test_hooks(uint64_t wait_ns, int32_t skip_one_arrival) {
  if (wait_ns == 0) {
    set_error("tc_test_hooks: wait_ns must be positive");
    return MB_E_ARG;
  }
  const unsigned long long w = wait_ns;
  const int k = skip_one_arrival ? 1 : 0;
  if (cudaMemcpyToSymbol(g_tc_wait_ns, &w, sizeof(w)) != cudaSuccess ||
      cudaMemcpyToSymbol(g_tc_skip_arrival, &k, sizeof(k)) != cudaSuccess) {
    set_error("tc_test_hooks: cudaMemcpyToSymbol failed");
    return MB_E_CUDA;
  }
  return 0;
}

extern "C" int mace_b200_node_gemm_tc(const float* X, int64_t ldx, const int32_t* xoff, int32_t n_seg,
                                      const float* Bt_split, int64_t plane, float* Y, int64_t ldy, int32_t yoff,
                                      int32_t mult, const int32_t* order, int32_t n_atoms, const float* rho,
                                      int32_t accumulate, uint32_t* status, void* stream) {
  GemmBatch bt(true, status, (cudaStream_t)stream);
  int rc = bt.add(X, ldx, xoff, n_seg, Bt_split, plane, Y, ldy, yoff, mult, order, n_atoms, rho, accumulate);
  return rc ? rc : bt.launch();
}
