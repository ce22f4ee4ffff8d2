// Node GEMM on the 5th-generation tensor cores (tcgen05, TMEM accumulator), 3xTF32 for fp32-level accuracy:
//   Y[atom][yoff + m][:] (+)= alpha_atom * sum_s X[atom][xoff_s + m][:] @ B_s
// with A = X rows gathered per (atom, m) and B given as tf32 hi / lo planes, every 128 x 128 matrix stored as four
// 16 KB K blocks that are already in the SWIZZLE_128B K-major shared-memory image (host: engine.tc_planes).  A is
// split on the fly: a_hi = rna_tf32(a), a_lo = rna_tf32(a - a_hi), and D = a_hi b_hi + a_hi b_lo + a_lo b_hi
// accumulates in fp32 in TMEM (the lo*lo term, ~2^-22 relative, is dropped).
//
// Persistent, warp-specialised CTA (one per SM, 288 threads), static round-robin over the 128-row tiles of all
// problems of the group:
//   warps 0-3  producers: thread p owns row p of the tile.  Its 128-byte slice of each K block is prefetched
//              TC_RAW blocks ahead with cp.async into a padded raw ring (no registers held), then split into
//              tf32 hi / lo and written with tcgen05.st into the stage's A columns of TMEM (row p = TMEM lane p);
//              thread 0 also fetches the stage's B hi / lo blocks into shared memory with two 16 KB
//              cp.async.bulk copies (no multicast).
//   warp 8     barrier init, TMEM allocation (two 128-column accumulators + 64 A columns per stage) and, on
//              lane 0, the MMA issue: 12 tcgen05.mma kind::tf32 (M = N = 128, K = 8, A from TMEM, B from shared
//              memory) per K block, tcgen05.commit -> stage-empty barrier, and after a tile's last block ->
//              accumulator-full barrier.  With A in TMEM the MMAs read half the shared-memory bytes (49.5 against
//              54.4 ms of node GEMMs per 1.03M-atom evaluation with A staged in shared memory, MB_TC_A_TMEM = 0);
//              deeper stage / raw rings (3 or 4 stages, 6 raw blocks) measured the same.
//   warps 4-7  epilogue: tcgen05.ld 32x32b of the finished accumulator (warp w reads TMEM lanes 32 (w % 4) ..,
//              one row per lane), row scale 1 / (rho + 1), then a transpose through shared memory so that the
//              optional accumulate load and the store of every 32-column chunk go out as full 128-byte row
//              segments (4 rows per warp instruction); then release the accumulator.
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
#define MB_TC_RAW 4
#endif
constexpr int TC_STAGES = MB_TC_STAGES;                    // operand stages
// A hi / lo of a stage: in TMEM (MB_TC_A_TMEM = 1; the MMA reads A from TMEM and only B from shared memory) or in
// shared memory beside B (0)
#ifndef MB_TC_A_TMEM
#define MB_TC_A_TMEM 1
#endif
#if MB_TC_A_TMEM
constexpr int TC_STAGE_BYTES = 2 * TC_TILE_BYTES;          // B hi, B lo
constexpr int TC_TMEM_COLS = 512;                          // two accumulators + A hi / lo (2 x 32 columns) per stage
#else
constexpr int TC_STAGE_BYTES = 4 * TC_TILE_BYTES;          // A hi, A lo, B hi, B lo
constexpr int TC_TMEM_COLS = 2 * TC_BN;
#endif
constexpr int TC_A_COL = 2 * TC_BN;                        // first TMEM column of the A stages
constexpr int TC_RAW = MB_TC_RAW;                          // cp.async depth of the raw A ring, in K blocks
constexpr int TC_RAW_ROW = 144;                            // one row's 128-byte K slice + 16 bytes of bank padding
constexpr int TC_RAW_BYTES = TC_BM * TC_RAW_ROW;
constexpr int TC_EPI_ROW = 33;                             // epilogue transpose: 32 floats per row + 1 (bank spread)
constexpr int TC_EPI_BYTES = 4 * 32 * TC_EPI_ROW * 4;      // one 32-row x 32-column chunk per epilogue warp
constexpr int TC_THREADS = 288;                            // 4 producer warps, 4 epilogue warps, 1 MMA warp
constexpr int TC_MMA_WARP = 8;
static_assert(!MB_TC_A_TMEM || TC_A_COL + TC_STAGES * 2 * TC_BK <= TC_TMEM_COLS, "TMEM columns");
constexpr int TC_RAW_OFF = TC_STAGES * TC_STAGE_BYTES;
constexpr int TC_EPI_OFF = TC_RAW_OFF + TC_RAW * TC_RAW_BYTES;
constexpr int TC_BAR_OFF = TC_EPI_OFF + TC_EPI_BYTES;
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

// the same with A read from TMEM (tmem_a: lane 0 and the first of the 8 columns of this K step, one row per lane)
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

// Row geometry of tile row `row` of global tile `tile`: problem index, A row pointer (null when out of range),
// output row pointer and scale.
struct TcRow {
  int pi;
  int nk;
  const float* a;
  float* y;
  float alpha;
};

__device__ __forceinline__ TcRow tc_row(const GemmGroup& grp, int tile, int row) {
  TcRow o;
  o.pi = gemm_problem_of(grp, tile);
  const GemmProblem& g = grp.p[o.pi];
  o.nk = g.nseg * (MB_C / TC_BK);
  o.a = nullptr;
  o.y = nullptr;
  o.alpha = 1.f;
  const int64_t r = (int64_t)(tile - grp.tile_start[o.pi]) * TC_BM + row;
  if (r < (int64_t)g.n_atoms * g.mult) {
    const int64_t t = r / g.mult;
    const int mm = (int)(r - t * g.mult);
    const int64_t at = g.order ? g.order[t] : t;
    o.a = g.X + at * g.ldx + (int64_t)mm * MB_C;
    o.y = g.Y + at * g.ldy + (int64_t)(g.yoff + mm) * MB_C;
    if (g.rho) o.alpha = 1.f / (g.rho[at] + 1.f);
  }
  return o;
}

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
        mbar_init(&B.acc_empty[a], 128);
      }
      B.failed = 0;
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = B.tmem;

  if (warp < 4) {
    // ------------------------------------------------------------------------------------------ producers
    const int p = tid;
    unsigned char* raw = smem + TC_RAW_OFF;
    // issue cursor (tile, kb) running TC_RAW blocks ahead of the split cursor; the next tile's row geometry is
    // computed one tile early so its dependent loads (order, rho) are off the critical path
    int it_tile = blockIdx.x, it_kb = 0;
    TcRow it_rw = tc_row(grp, it_tile, p);
    TcRow it_next = it_tile + (int)gridDim.x < n_tiles ? tc_row(grp, it_tile + gridDim.x, p) : it_rw;
    auto issue_next = [&](int slot) {
      if (it_tile < n_tiles) {
        if (it_rw.a) {
          const GemmProblem& g = grp.p[it_rw.pi];
          const int seg = (it_kb * TC_BK) / MB_C, kin = it_kb * TC_BK - seg * MB_C;
          const float* src = it_rw.a + (int64_t)g.xoff[seg] * MB_C + kin;
          unsigned char* dst = raw + slot * TC_RAW_BYTES + p * TC_RAW_ROW;
#pragma unroll
          for (int q = 0; q < 8; ++q) cp_async16(dst + 16 * q, src + 4 * q);
        }
        if (++it_kb == it_rw.nk) {
          it_kb = 0;
          it_tile += gridDim.x;
          it_rw = it_next;
          if (it_tile + (int)gridDim.x < n_tiles) it_next = tc_row(grp, it_tile + gridDim.x, p);
        }
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
    };
#pragma unroll 1
    for (int q = 0; q < TC_RAW; ++q) issue_next(q);
    int seq = 0;                                   // K blocks consumed (stage / phase counter)
    TcRow rw = tc_row(grp, blockIdx.x, p);
    // every exit decision is warp-uniform: the loop body holds warp-collective tcgen05.st.sync.aligned
    for (int tile = blockIdx.x; tile < n_tiles && !__shfl_sync(0xffffffffu, *failed, 0); tile += gridDim.x) {
      const GemmProblem& g = grp.p[rw.pi];
      const int nk = rw.nk;
      const bool have = rw.a != nullptr;
      for (int kb = 0; kb < nk; ++kb, ++seq) {
        const int s = seq % TC_STAGES, slot = seq % TC_RAW;
        asm volatile("cp.async.wait_group %0;" ::"n"(TC_RAW - 1) : "memory");
        float4 v[8];
        const unsigned char* src = raw + slot * TC_RAW_BYTES + p * TC_RAW_ROW;
#pragma unroll
        for (int q = 0; q < 8; ++q)
          v[q] = have ? *reinterpret_cast<const float4*>(src + 16 * q) : make_float4(0.f, 0.f, 0.f, 0.f);
        issue_next(slot);                          // the slot has been read: refill it TC_RAW blocks ahead
#if MB_TC_A_TMEM
        uint32_t ahi[32], alo[32];                 // split before the wait, so that the wait covers it
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float c4[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float h = tf32_rna(c4[j]);
            ahi[4 * q + j] = __float_as_uint(h);
            alo[4 * q + j] = __float_as_uint(tf32_rna(c4[j] - h));
          }
        }
#endif
        // stage s free once the MMAs of its previous use completed (first use: the preceding phase counts done)
        if (!__all_sync(0xffffffffu, mbar_wait(&B.empty[s], ((seq / TC_STAGES) & 1) ^ 1))) {
          *failed = 1;
          break;
        }
        unsigned char* st = smem + s * TC_STAGE_BYTES;
        if (p == 0) {
          const int seg = (kb * TC_BK) / MB_C, kin = kb * TC_BK - seg * MB_C;
          const float* bsrc = g.B + (int64_t)seg * MB_C * MB_C + (int64_t)(kin / TC_BK) * (TC_BM * TC_BK);
          mbar_arrive_tx(&B.bfull[s], 2 * TC_TILE_BYTES);
          bulk_g2s(st + TC_STAGE_BYTES - 2 * TC_TILE_BYTES, bsrc, TC_TILE_BYTES, &B.bfull[s]);
          bulk_g2s(st + TC_STAGE_BYTES - TC_TILE_BYTES, bsrc + g.plane, TC_TILE_BYTES, &B.bfull[s]);
        }
#if MB_TC_A_TMEM
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t ta = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(TC_A_COL + s * 2 * TC_BK);
        tmem_st32(ta, ahi);
        tmem_st32(ta + TC_BK, alo);
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
#else
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          float4 hi, lo;
          hi.x = tf32_rna(v[q].x); lo.x = tf32_rna(v[q].x - hi.x);
          hi.y = tf32_rna(v[q].y); lo.y = tf32_rna(v[q].y - hi.y);
          hi.z = tf32_rna(v[q].z); lo.z = tf32_rna(v[q].z - hi.z);
          hi.w = tf32_rna(v[q].w); lo.w = tf32_rna(v[q].w - hi.w);
          const uint32_t off = sw128_offset(p, q);
          *reinterpret_cast<float4*>(st + off) = hi;
          *reinterpret_cast<float4*>(st + TC_TILE_BYTES + off) = lo;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
#endif
        // test hook (off unless mace_b200_tc_test_hooks armed it): one arrival of CTA 0's first K block goes missing
        const bool skip = seq == 0 && p == 0 && blockIdx.x == 0 && *(volatile int*)&g_tc_skip_arrival &&
                          atomicExch(&g_tc_skip_arrival, 0);
        if (!skip) mbar_arrive(&B.full[s]);
      }
      if (tile + (int)gridDim.x < n_tiles) rw = tc_row(grp, tile + gridDim.x, p);
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    // after a timeout: B copies this thread issued may still be landing in the stages
    if (p == 0 && *failed)
      for (int s = 0; s < TC_STAGES; ++s) {
        const int last = seq - 1 - ((seq - 1 - s) % TC_STAGES + TC_STAGES) % TC_STAGES;   // last seq using stage s
        if (last >= 0) mbar_wait(&B.bfull[s], (last / TC_STAGES) & 1);
      }
  } else if (warp < TC_MMA_WARP) {
    // ------------------------------------------------------------------------------------------ epilogue
    const int q4 = warp & 3, row = q4 * 32 + lane;
    int tc = 0;
    // every exit decision is warp-uniform: the loop body holds warp-collective tcgen05.ld.sync.aligned
    for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++tc) {
      if (__shfl_sync(0xffffffffu, *failed, 0)) break;
      const int a = tc & 1;
      const TcRow rw = tc_row(grp, tile, row);     // its loads overlap the wait
      if (!__all_sync(0xffffffffu, mbar_wait(&B.acc_full[a], (tc >> 1) & 1))) {
        *failed = 1;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int acc = grp.p[rw.pi].accumulate;
      float* stg = reinterpret_cast<float*>(smem + TC_EPI_OFF) + q4 * 32 * TC_EPI_ROW;   // this warp's chunk
      // lane l stores rows 4 i + l / 8 (i = 0..7), columns 4 (l % 8) .. + 3 of the chunk: 4 rows per instruction
      const int srow = lane >> 3, scol = (lane & 7) * 4;
#pragma unroll 1
      for (int h = 0; h < 4; ++h) {
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
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        __syncwarp();                                // the previous chunk's reads of the staging area are done
#pragma unroll
        for (int j = 0; j < 32; ++j) stg[lane * TC_EPI_ROW + j] = __uint_as_float(x[j]) * rw.alpha;
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int r = 4 * i + srow;                // row of this warp's 32 (lane r of the TMEM load)
          float* yrow = reinterpret_cast<float*>(__shfl_sync(0xffffffffu, reinterpret_cast<uintptr_t>(rw.y), r));
          if (yrow) {
            const float* sv = stg + r * TC_EPI_ROW + scol;
            float4 o = make_float4(sv[0], sv[1], sv[2], sv[3]);
            float4* yp = reinterpret_cast<float4*>(yrow + 32 * h + scol);
            if (acc) {
              const float4 p4 = *yp;
              o.x += p4.x; o.y += p4.y; o.z += p4.z; o.w += p4.w;
            }
            *yp = o;
          }
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
        const uint32_t b_hi = smem_u32(smem + (s + 1) * TC_STAGE_BYTES - 2 * TC_TILE_BYTES), b_lo = b_hi + TC_TILE_BYTES;
#if MB_TC_A_TMEM
        const uint32_t a_hi = tmem + (uint32_t)(TC_A_COL + s * 2 * TC_BK), a_lo = a_hi + TC_BK;
#pragma unroll
        for (int kk = 0; kk < TC_BK / 8; ++kk) {
          const uint32_t ko = kk * 32;               // 8 tf32 = 32 bytes along K inside B's swizzle atom
          mma_tf32_ts(d, a_hi + 8 * kk, sw128_desc(b_hi + ko), idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          mma_tf32_ts(d, a_hi + 8 * kk, sw128_desc(b_lo + ko), idesc, 1u);
          mma_tf32_ts(d, a_lo + 8 * kk, sw128_desc(b_hi + ko), idesc, 1u);
        }
#else
        const uint32_t a_hi = smem_u32(smem + s * TC_STAGE_BYTES), a_lo = a_hi + TC_TILE_BYTES;
#pragma unroll
        for (int kk = 0; kk < TC_BK / 8; ++kk) {
          const uint32_t ko = kk * 32;               // 8 tf32 = 32 bytes along K inside the swizzle atom
          mma_tf32(d, sw128_desc(a_hi + ko), sw128_desc(b_hi + ko), idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          mma_tf32(d, sw128_desc(a_hi + ko), sw128_desc(b_lo + ko), idesc, 1u);
          mma_tf32(d, sw128_desc(a_lo + ko), sw128_desc(b_hi + ko), idesc, 1u);
        }
#endif
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
