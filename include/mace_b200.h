/* mace_b200.h — C ABI of the sm_100a three-pass MACE force evaluation (libmace_b200.so).
 *
 * The drop-in boundary of the reference (ShiQiaoL/mace-million, package mace_onegpu) is Python:
 * ThreePassMLIAP.compute_forces(data) (mace_onegpu/mliap_threepass.py:444-616) behind LAMMPS
 * `pair_style mliap unified`, which calls Triton kernels (conv_spline.py, spline_w.py) and cuEquivariance
 * (fused_conv.py) per receiver chunk.  This library replaces those kernels and the chunk loops.  Every entry point
 * takes plain device pointers, sizes and a cudaStream_t (passed as void*), never torch types; all device memory is
 * owned by the caller (the Python host allocates it with torch).  Each entry point returns 0 on success or a
 * negative MB_E_* code; mace_b200_last_error() gives the message of the last failure on the calling thread.
 * Kernels never trap: device-side input checks set bits in the caller's status word (MB_ST_*), read by the host
 * at pass ends.
 *
 * Layouts: features with 128 channels per irrep component are component-major, [atom][component][128] fp32
 * (h1: 4 components 0e|1o; layer-1 messages 16 components; layer-2 messages 40 components).  Pairs are sorted by
 * receiver; rowptr is the CSR row pointer over local receivers.
 */
#ifndef MACE_B200_H
#define MACE_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MB_ABI_VERSION 4

enum {
  MB_OK = 0,
  MB_E_ARG = -1,      /* bad argument (null pointer, size out of range, unsupported width) */
  MB_E_CUDA = -2,     /* a CUDA runtime call failed */
  MB_E_STATUS = -3,   /* the device status word reported an input error */
};

/* device status bits (written by kernels into mb_eval_t.status) */
enum {
  MB_ST_BAD_SENDER = 1,
  MB_ST_BAD_SPECIES = 2,
  MB_ST_BAD_ROWPTR = 4,
  MB_ST_NONFINITE = 8,
  MB_ST_BAD_RECEIVER = 16,
  MB_ST_TC_TIMEOUT = 32,      /* a tensor-core kernel gave up waiting on its MMA barrier (bounded wait) */
  MB_ST_UNSORTED = 64,        /* mace_b200_csr_rows: pair_i not receiver-sorted inside a chunk */
};

/* Folded, device-resident model (fp32 unless noted).  S = number of species present (compact indices),
 * C = 128, NT1 / NT2 = symmetric-contraction coefficient counts (mace_b200_sc_layout). */
typedef struct {
  int32_t C, S, M;             /* channels, species, spline knots */
  float r_lo, inv_h, r_max, p_cut;
  float scale;                 /* ScaleShift scale */
  const float* tab1;           /* [T1][M-1][4][C] float4 cubic coefficients of W1 * X1(sender species), T1 tables;
                                  with l1_density: [M-1][64] float4 cubic coefficients of the radial MLP's last
                                  hidden layer h(r) */
  const float* tab2;           /* [T2][M-1][5][2][C] float4 cubic coefficients of W2, T2 tables (see tab*_map):
                                  per path pair p, (a, a', b, b') then (c, c', d, d') of paths 2p and 2p + 1 */
  const float* wd1;            /* [8] layer-1 density weights / sqrt(8) */
  const float* wd2;            /* [8] layer-2 density weights / sqrt(8) */
  const float* M0;             /* [S][4][C][C]  linear_1 o skip_tp_1 per species and l; with l1_density the
                                  composite [S][4][2 x 64][C] = (last MLP layer x X1 of species slot) o M0 */
  const float* M0T;            /* transposes */
  const float* Wp1;            /* [2][C][C]     products[0].linear per l */
  const float* Wp1T;
  const float* wr0;            /* [C]           readouts[0] */
  const float* sc1;            /* [S][NT1/4][C][4]  symmetric contraction 1 (L = 0 and L = 1 outputs); coefficient t of
                                  channel c at [t / 4][c][t % 4], NT1 rounded up to a multiple of 4 with zeros */
  const float* Wup2;           /* [2][C][C]     interactions[1].linear_up per l */
  const float* Wup2T;
  const float* Wsk1;           /* [S][C][C]     interactions[1].skip_tp (0e -> 0e) per species */
  const float* Wsk1T;
  const float* Wlin2;          /* [10][C][C]    interactions[1].linear per mid entry (scaled by its group) */
  const float* Wlin2T;
  const float* sc2;            /* [S][NT2/4][C][4]  symmetric contraction 2 (L = 0), same layout */
  const float* Wp2;            /* [C][C]        products[1].linear */
  const float* Wp2T;
  const float* W1r;            /* [C][16]       readouts[1].linear_1 / sqrt(C) */
  const float* w2r;            /* [16]          readouts[1].linear_2 * cst / sqrt(16) */
  const double* e0;            /* [S]           E0 + shift per species (fp64) */
  /* tensor-core copies: the K-major form of each matrix above used as a GEMM B operand (X_tc = transpose of X),
   * split into two planes [2][...] of tf32-rounded hi and lo parts (3xTF32); used when use_tc != 0 */
  const float* M0_tc;
  const float* M0T_tc;
  const float* Wp1_tc;
  const float* Wp1T_tc;
  const float* Wup2_tc;
  const float* Wup2T_tc;
  const float* Wsk1_tc;
  const float* Wsk1T_tc;
  const float* Wlin2_tc;
  const float* Wlin2T_tc;
  const float* Wp2_tc;
  const float* Wp2T_tc;
  int32_t use_tc;              /* node GEMMs on tcgen05 (3xTF32) instead of the SIMT fp32 kernel */
  /* optional [S*S] maps from the ordered species pair (sender * S + receiver) to the table of tab1 / tab2 it reads
   * (null = identity).  Pairs whose tables are bitwise identical share one table: W2 has no species dependence in
   * an architecture without a species-pair distance transform, W1 * X1 depends on the sender species only. */
  const int32_t* tab1_map;
  const int32_t* tab2_map;
  /* exact density-projection layer 1 (S <= 2): the layer-1 edge kernels accumulate per receiver the densities
   * B[m][slot * 64 + q] = sum over edges from species `slot` of h_q(r) Y_m into the message rows of the chunk
   * (instead of msg1[m][c]) and the backward reads dE/dB there; M0 / M0T map B to x1 directly.  0 = direct. */
  int32_t l1_density;
} mb_model_t;

/* One force evaluation: the pair list (receiver-sorted), persistent per-atom state and per-chunk scratch. */
typedef struct {
  int32_t nl, nt;              /* local atoms, local + ghost atoms */
  int64_t P;                   /* pairs */
  const int32_t* pair_i;       /* [P] receivers (local), non-decreasing */
  const int32_t* pair_j;       /* [P] senders (local or ghost) */
  const double* rij;           /* [P][3] edge vectors (receiver - sender convention of the model) */
  const int32_t* rowptr;       /* [nl+1] CSR over receivers */
  const int32_t* spec;         /* [nt] compact species index */
  float* H1;                   /* [nt][4][C]  layer-1 features (ghost rows filled by the forward exchange) */
  float* X2;                   /* [nt][4][C]  linear_up(H1) of every atom */
  float* G1;                   /* [nt][4][C]  dE2/dh1 (ghost rows reverse-exchanged onto owners) */
  float* GX2;                  /* [nt][4][C]  dE2/dX2 accumulated over all chunks */
  float* PF;                   /* [P][3]      pair forces dE/drij, fp32 accumulator */
  double* eat;                 /* [nl]        per-atom energies */
  int32_t chunk;               /* receivers per chunk (scratch capacity) */
  const int32_t* order;        /* [nl] receivers of every chunk sorted by species (chunk-local indices) */
  const int32_t* spec_off;     /* HOST array [(n_chunks)*(S+1)]: species segment offsets inside each chunk */
  float* s_msg;                /* [chunk][40][C] */
  float* s_x;                  /* [chunk][16][C] */
  float* s_gx;                 /* [chunk][16][C] */
  float* s_a;                  /* [chunk][4][C]  */
  float* s_ga;                 /* [chunk][4][C]  */
  float* s_h;                  /* [chunk][C]     */
  float* s_gh;                 /* [chunk][C]     */
  float* s_sc;                 /* [chunk][C]     */
  float* s_rho;                /* [chunk] */
  float* s_grho;               /* [chunk] */
  uint32_t* status;            /* device status word */
  /* optional cache of pass A's layer-1 intermediates for pass C (null = recompute them, the reference's
   * low-memory schedule): x1 = linear_1(msg1) / (rho1 + 1) [nl][16][C] and rho1 [nl].  Pass C reads them
   * instead of re-running edge_l1_fwd and the x1 GEMMs; the values are bitwise the same (deterministic kernels). */
  float* x1_cache;
  float* rho1_cache;
  /* optional overlap of the caller's host <-> device copies with the passes (all null = off):
   * wait_ev   HOST array [n_chunks] of cudaEvent_t: pass A makes its stream wait on wait_ev[k] before chunk k's
   *           first kernel (the caller records it once chunk k's pair_j / rij rows are on the device);
   * done_ev   HOST array [n_chunks] of cudaEvent_t: right after chunk k of pass C its final pair forces are written
   *           to pf_out (fp64 [P][3] in receiver order, i.e. the caller's order for receiver-sorted input) with
   *           their max |PF| into *fmax_bits, and done_ev[k] is recorded, so the caller can copy them out while
   *           the next chunks run; mace_b200_finalize then converts no pair forces (energies only). */
  void* const* wait_ev;
  void* const* done_ev;
  double* pf_out;
  uint32_t* fmax_bits;
} mb_eval_t;

/* ---------------------------------------------------------------- library info */
int mace_b200_abi_version(void);
const char* mace_b200_last_error(void);
/* sizeof(mb_model_t), sizeof(mb_eval_t) as compiled into the library (for binding checks). */
int mace_b200_struct_sizes(int32_t* model_bytes, int32_t* eval_bytes);
/* Number of kernels this library has launched since it was loaded (all threads). */
unsigned long long mace_b200_launch_count(void);
/* Per-kind CUDA-event timing of the pass runners' edge, symmetric-contraction and grouped node-GEMM launches (the reference's
 * per-pass wall timers, mliap_threepass.py:525-585, at kernel granularity).  mace_b200_timing(enable, ms, cnt)
 * synchronises on the recorded events, writes the accumulated milliseconds and launch counts per kind
 * (MB_K_*, arrays of MB_NKINDS, either may be null), resets them and switches recording on or off. */
enum { MB_K_EDGE_L1_FWD = 0, MB_K_EDGE_L1_BWD = 1, MB_K_EDGE_L2_FWD = 2, MB_K_EDGE_L2_BWD = 3, MB_K_SYMCON = 4,
       MB_K_NODE_GEMM = 5, MB_NKINDS = 6 };
int mace_b200_timing(int enable, double* ms_out, long long* count_out);
/* Restrict recording to the kinds whose bit (1 << MB_K_*) is set in mask (default: all).  Each recorded launch
 * costs two event records on its stream, so a caller timing one kernel inside a measured region records only it. */
int mace_b200_timing_kinds(uint32_t mask);
/* FP32 FFMA issue ceiling of the current device (TFLOP/s), by an 8-chain FFMA kernel on 8 CTAs per SM (the edge
 * kernels' roofline denominator; scratch is one device float). */
int mace_b200_ffma_peak(int32_t iters, float* scratch, double* tflops, void* stream);
/* Number of symmetric-contraction coefficients per (species, channel) for block 0 (layer 1) or 1 (layer 2), and
 * the layout fingerprint the host must reproduce when it folds the weights. */
int mace_b200_sc_layout(int block, int32_t* n_coef, uint64_t* fingerprint);

/* ---------------------------------------------------------------- tables
 * Replaces conv_spline.build_tables (mace_onegpu/conv_spline.py:230-249) and spline_radial._sample
 * (mace_onegpu/spline_radial.py:237-272): per ordered species pair p = s_send * S + s_recv, the radial MLP
 * W(r) = silu(silu(silu(f(r) A0) A1) A2) A3 (f = Bessel x cutoff, fp64) sampled on M knots over [r_lo, r_max] with
 * dW/dr by central differences (eps = 1e-5 (r_max - r_lo)), times col_scale[p][d] (null = 1).  Outputs TV, TG = h dW/dr
 * ([P][M][D] fp32, the reference's table format; either may be null) and the float4 cubic form
 * cubic[P][M-1][D] (a + b t + c t^2 + d t^3 on each interval, fp32 from fp64). */
int mace_b200_build_tables(const double* A0, const double* A1, const double* A2, const double* A3, int32_t n_in,
                           int32_t hidden, int32_t D, const double* col_scale, int32_t n_pairs, int32_t M,
                           double r_lo, double r_max, double p_cut, float* TV, float* TG, float* cubic,
                           void* stream);

/* Allocation-free variant of mace_b200_build_tables (no counterpart in the reference).  For callers that must not
 * have the library allocate device memory (an MD engine that owns all device memory through its own pool, or a
 * process with a fixed device footprint): same arguments and outputs, but the fp64 sample scratch is a static device
 * array of the library, so M * D is limited to 512 * 1280 (15 MiB, held by every GPU that loads the library until
 * exit); larger tables are rejected with MB_E_ARG.  It calls no cudaMalloc / cudaFree.  Every call resolves the
 * scratch's device address (cudaGetSymbolAddress) on the current device, so the first call on a device (which loads
 * the module there) should come before any stream capture.  All calls share the scratch, so calls that overlap on the
 * GPU race: serialise them. */
int mace_b200_build_tables_noalloc(const double* A0, const double* A1, const double* A2, const double* A3,
                                   int32_t n_in, int32_t hidden, int32_t D, const double* col_scale, int32_t n_pairs,
                                   int32_t M, double r_lo, double r_max, double p_cut, float* TV, float* TG,
                                   float* cubic, void* stream);

/* ---------------------------------------------------------------- edge kernels (one receiver chunk [a, b))
 * edge_l1_fwd replaces ConvSpline.forward (mace_onegpu/conv_spline.py:294-301) and the density sum
 *   (fast_layers.py:179-183): s_msg[i][lm][c] = sum_e T1(r_e, p_e)[l][c] Y_e[lm], s_rho[i] = sum_e tanh(d_e^2).
 * edge_l2_fwd replaces FusedConvTP.forward (mace_onegpu/fused_conv.py:33-37) fed by SplineW (spline_w.py:30-50):
 *   s_msg[i][o][c] = sum_e sum_terms coef W2(r_e)[w][c] X2[j_e][k][c] Y_e[m], s_rho[i].
 * edge_l2_bwd replaces the autograd backward of pass B for the edge part (mliap_threepass.py:549-552 with
 *   spline_w.py:53-75): given s_gx = dE/dmsg (in s_msg) and s_grho, PF[e] = dE/drij, GX2[j_e] += dE/dX2.
 * edge_l1_bwd: pass C edge backward (mliap_threepass.py:576-581): PF[e] += dL/drij. */
int mace_b200_edge_l1_fwd(const mb_model_t* m, const mb_eval_t* ev, int32_t a, int32_t b, void* stream);
int mace_b200_edge_l2_fwd(const mb_model_t* m, const mb_eval_t* ev, int32_t a, int32_t b, void* stream);
int mace_b200_edge_l2_bwd(const mb_model_t* m, const mb_eval_t* ev, int32_t a, int32_t b, void* stream);
int mace_b200_edge_l1_bwd(const mb_model_t* m, const mb_eval_t* ev, int32_t a, int32_t b, void* stream);

/* ---------------------------------------------------------------- generic fused convolution (FusedConvTP)
 * Replaces the cuEquivariance fused convolution behind FusedConvTP.forward (mace_onegpu/fused_conv.py:20-37) and its
 * autograd backward: out[receiver[e]][o][:] = sum over the receiver's edges and the terms of coef W[e][w][:]
 * X[sender[e]][k][:] Y[e][m], with explicit per-edge weights W [E][nW][128], node features X [n][nX][128] and edge
 * attributes Y [E][nY]; terms_wkmo [n_terms][4] = (w, k, m, o) with coef [n_terms] (any channelwise path table).
 * Edges are visited through CSR lists the caller builds: recv_rowptr [n + 1] / recv_edges (edge ids grouped by
 * receiver), and for dX send_rowptr / send_edges (grouped by sender), so no kernel uses atomics and the results are
 * deterministic.  fwd writes every output row (no zeroing needed).  bwd: given g = dL/dout [n][nO][128] writes
 * dW [E][nW][128], dY [E][nY] and dX [n][nX][128]; any of the three may be null.  Out-of-range node indices set
 * MB_ST_BAD_SENDER / MB_ST_BAD_RECEIVER in *status (may be null) and skip the edge. */
int mace_b200_conv_tp_fwd(const float* X, int32_t nX, const float* Y, int32_t nY, const float* W, int32_t nW,
                          const int32_t* sender, const int64_t* recv_rowptr, const int64_t* recv_edges,
                          int32_t n_nodes, const int32_t* terms_wkmo, const float* coef, int32_t n_terms, float* out,
                          int32_t nO, uint32_t* status, void* stream);
int mace_b200_conv_tp_bwd(const float* X, int32_t nX, const float* Y, int32_t nY, const float* W, int32_t nW,
                          const int32_t* sender, const int32_t* receiver, const int64_t* recv_rowptr,
                          const int64_t* recv_edges, const int64_t* send_rowptr, const int64_t* send_edges,
                          int32_t n_nodes, const int32_t* terms_wkmo, const float* coef, int32_t n_terms,
                          const float* g, int32_t nO, float* dX, float* dY, float* dW, uint32_t* status, void* stream);

/* ---------------------------------------------------------------- node GEMM
 * Replaces the cuEquivariance irreps Linear and SpeciesSkip.forward (mace_onegpu/fast_layers.py:96-105):
 *   Y[atom][yoff + m][:] (+)= alpha_atom * sum_j X[atom][xoff_j + m][:] @ B_j       (m = 0 .. mult-1)
 * for n_atoms atoms (atom = order ? order[t] : t, t = 0 .. n_atoms-1), K = n_seg * 128, N = 128, B_j [128][128]
 * row-major (B = [n_seg][128][128]); alpha_atom = 1 / (rho[atom] + 1) when rho is not null.
 * ldx / ldy are the per-atom strides in floats; accumulate != 0 adds into Y. */
int mace_b200_node_gemm(const float* X, int64_t ldx, const int32_t* xoff, int32_t n_seg, const float* B,
                        float* Y, int64_t ldy, int32_t yoff, int32_t mult, const int32_t* order, int32_t n_atoms,
                        const float* rho, int32_t accumulate, void* stream);

/* The same GEMM on the 5th-generation tensor cores (tcgen05.mma kind::tf32, accumulator in TMEM), 3xTF32:
 * Bt_split = [2][n_seg][128 x 128] (K-major B split into a tf32 hi plane then a lo plane, plane = elements per
 * plane; every 128 x 128 matrix permuted into four 16 KB K blocks in the SWIZZLE_128B shared-memory image:
 * element (n, k) at (k / 32) * 4096 + (n / 8) * 256 + (n % 8) * 32 + (((k % 32) / 4) ^ (n % 8)) * 4 + k % 4).
 * X, Y, Bt_split 16-byte aligned.  Persistent kernel, one CTA per SM. 
 * A timeout of its bounded MMA-barrier wait sets MB_ST_TC_TIMEOUT in *status (may be null). */
int mace_b200_node_gemm_tc(const float* X, int64_t ldx, const int32_t* xoff, int32_t n_seg, const float* Bt_split,
                           int64_t plane, float* Y, int64_t ldy, int32_t yoff, int32_t mult, const int32_t* order,
                           int32_t n_atoms, const float* rho, int32_t accumulate, uint32_t* status, void* stream);
/* No counterpart in the reference: test hooks of the tensor-core GEMM on the current device.  wait_ns bounds every
 * mbarrier wait of k_gemm_tc (default 2 s); skip_one_arrival = 1 makes the next launch lose one producer arrival,
 * so that its waits expire and it reports MB_ST_TC_TIMEOUT after draining its copies and MMAs and freeing its TMEM
 * (the error path is exercised without any fault).  Not for production use. */
int mace_b200_tc_test_hooks(uint64_t wait_ns, int32_t skip_one_arrival);

/* ---------------------------------------------------------------- symmetric contraction
 * Replaces products[k].symmetric_contractions (mace EquivariantProductBasisBlock, correlation 3).
 * block 0: x [n][16][C] -> A [n][4][C] (L = 0 | L = 1); block 1: x [n][16][C] -> A [n][C].
 * bwd: gA -> gx [n][16][C]; when grho is not null also grho[i] = -sum(gx * x) / (rho[i] + 1). */
int mace_b200_symcon_fwd(const mb_model_t* m, int32_t block, const float* x, float* A, const int32_t* spec_local,
                         int32_t n, void* stream);
int mace_b200_symcon_bwd(const mb_model_t* m, int32_t block, const float* x, const float* gA, float* gx,
                         const int32_t* spec_local, const float* rho, float* grho, int32_t n, void* stream);

/* ---------------------------------------------------------------- three passes (chunk loops in C++)
 * pass_a: mliap_threepass.py:504-519 (H1[a:b] = layer1 for every chunk), then R1 energies.
 * x2_all: X2 = linear_up(H1) for all nt atoms (after the forward exchange); zeroes G1 and GX2.
 * pass_b: mliap_threepass.py:537-553 (layer-2 energy, PF, G1), then G1 += linear_up^T(GX2).
 * pass_c: mliap_threepass.py:564-587 (loss = E1 + G1 . h1, PF).
 * finalize: eat += E0 + shift (mliap_threepass.py:589), PFd = PF in fp64 scattered to the caller's pair order
 *   (perm = receiver-sorted position -> caller position, null = identity), and *fmax_bits (device word, zeroed by
 *   the caller) = bits of max |PF| as an fp32 (a NaN anywhere gives NaN bits), for the force guard
 *   (mliap_threepass.py:595-601). */
int mace_b200_pass_a(const mb_model_t* m, const mb_eval_t* ev, void* stream);
int mace_b200_x2_all(const mb_model_t* m, const mb_eval_t* ev, void* stream);
int mace_b200_pass_b(const mb_model_t* m, const mb_eval_t* ev, void* stream);
int mace_b200_pass_c(const mb_model_t* m, const mb_eval_t* ev, void* stream);
/* The same passes split so that a caller can overlap the halo exchanges with interior work (the reference leaves
 * the exchanges to LAMMPS between whole passes, mliap_threepass.py:522,556):
 * pass_a_chunks / pass_b_chunks / pass_c_chunks run chunks [c0, c1) (chunk k = receivers [k chunk, (k+1) chunk));
 *   pass_a_chunks adds the R1 energies of those chunks' receivers; pass_b_chunks neither zeroes PF nor folds GX2.
 * x2_rows: X2 = linear_up(H1) and zeroed G1 / GX2 for rows [r0, r1).
 * fold_g1: G1[r0:r1] += linear_up^T(GX2[r0:r1]).
 * pass_a = pass_a_chunks(all); x2_all = x2_rows(0, nt); pass_b = zero PF, pass_b_chunks(all), fold_g1(0, nt). */
int mace_b200_pass_a_chunks(const mb_model_t* m, const mb_eval_t* ev, int32_t c0, int32_t c1, void* stream);
int mace_b200_x2_rows(const mb_model_t* m, const mb_eval_t* ev, int32_t r0, int32_t r1, void* stream);
int mace_b200_pass_b_chunks(const mb_model_t* m, const mb_eval_t* ev, int32_t c0, int32_t c1, void* stream);
int mace_b200_fold_g1(const mb_model_t* m, const mb_eval_t* ev, int32_t r0, int32_t r1, void* stream);
int mace_b200_pass_c_chunks(const mb_model_t* m, const mb_eval_t* ev, int32_t c0, int32_t c1, void* stream);
int mace_b200_finalize(const mb_model_t* m, const mb_eval_t* ev, const int64_t* perm, double* PFd,
                       uint32_t* fmax_bits, void* stream);

/* ---------------------------------------------------------------- halo exchange helpers (mliap_threepass.py:40-55)
 * pack: buf[k][:] = src[idx[k]][:] (D floats per row); unpack_add: dst[idx[k]][:] += buf[k][:]. */
int mace_b200_pack_rows(const float* src, const int32_t* idx, int64_t n, int32_t D, float* buf, void* stream);
int mace_b200_unpack_add_rows(const float* buf, const int32_t* idx, int64_t n, int32_t D, float* dst, void* stream);

/* ---------------------------------------------------------------- neighbour lists (input preparation)
 * Replaces System.build_neighbors (mace_onegpu/receiver_chunk_mace.py:114-165) for the standalone driver: full
 * lists (both directions) of receivers [0, n_recv) within r_cut, one warp per receiver over the 27 candidate cells.
 * Cells: lo[3], width[3] (>= r_cut), nc[3]; cell of x = clamp(floor((x - lo) / width)), linear index
 * (cx * nc1 + cy) * nc2 + cz; cell_start [ncell + 1] and cell_atoms (atom indices grouped by cell) are the caller's.
 * periodic = 1: orthorhombic box[3], minimum image, positions wrapped into [0, box), nc >= 3 per dimension;
 * periodic = 0: no wrap (explicit ghost atoms; all atoms, receivers first, are in the cells).
 * Output order: by receiver, candidates in a fixed order (deterministic); rij = x_i - x_j (fp64).
 * nbr_count writes counts [n_recv]; the caller forms rowptr [n_recv + 1] (int64 prefix sum) and calls nbr_fill.
 * verlet_filter: pairs vrow / vj of a skin list kept when |x_i - x_j| < r_cut at the current positions; with
 * counts != null it counts, else it fills (pi, pj, rij) at rowptr.  A count / fill mismatch sets
 * MB_ST_BAD_ROWPTR in *status (may be null). */
int mace_b200_nbr_count(const double* pos, const int32_t* cell_start, const int32_t* cell_atoms, const double* lo,
                        const double* width, const int32_t* nc, const double* box, int32_t periodic, int32_t n_recv,
                        double r_cut, int32_t* counts, void* stream);
int mace_b200_nbr_fill(const double* pos, const int32_t* cell_start, const int32_t* cell_atoms, const double* lo,
                       const double* width, const int32_t* nc, const double* box, int32_t periodic, int32_t n_recv,
                       double r_cut, const int64_t* rowptr, int32_t* pi, int32_t* pj, double* rij, uint32_t* status,
                       void* stream);
int mace_b200_verlet_filter(const double* pos, const double* box, int32_t periodic, int32_t n_recv,
                            const int64_t* vrow, const int32_t* vj, double r_cut, int32_t* counts,
                            const int64_t* rowptr, int32_t* pi, int32_t* pj, double* rij, uint32_t* status,
                            void* stream);

/* ---------------------------------------------------------------- chunk-wise CSR (streamed pair lists)
 * Replaces the receiver CSR of mliap_threepass.py:468-478 (searchsorted over the whole pair_i on the device) for a
 * pair list that arrives chunk by chunk: rowptr[i] for i = a .. b from the chunk's edges [e0, e1) of a
 * receiver-sorted pair_i (first e with pair_i[e] >= i, e1 if none); an edge of the chunk whose receiver is outside
 * [a, b) or below its predecessor's sets MB_ST_UNSORTED in *status (the caller then sorts and evaluates again). */
int mace_b200_csr_rows(const int32_t* pair_i, int64_t e0, int64_t e1, int32_t a, int32_t b, int32_t* rowptr,
                       uint32_t* status, void* stream);

/* Smallest and largest sender of a chunk of a streamed pair list: out[0] = min, out[1] = max of pair_j[e0, e1)
 * ((INT32_MAX, -1) for an empty range), written on the stream.  No counterpart in the reference, whose pair list is
 * already in device memory: the engine reads the range back per chunk of a list streamed from host memory, to run
 * every pass-B chunk as soon as pass A has produced the features of all its senders while later chunks still
 * arrive. */
int mace_b200_sender_range(const int32_t* pair_j, int64_t e0, int64_t e1, int32_t* out, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* MACE_B200_H */
