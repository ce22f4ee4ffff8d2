// The three passes as native chunk loops (replacing the Python chunk loops of the reference's
// ThreePassMLIAP.compute_forces, mace_onegpu/mliap_threepass.py:504-587), plus the library's error plumbing.
//
// Per chunk [a, b) of receivers (nC = b - a) with per-chunk scratch of the eval struct:
//   pass A:  msg1, rho1 = edge_l1_fwd;  x1 = msg1 M0[s] / (rho1 + 1);  A1 = symcon1(x1);  H1[a:b] = A1 Wp1
//   pass B:  sc = h1_0e Wsk1[s];  msg2, rho2 = edge_l2_fwd(X2);  x2 = lin2(msg2) / (rho2 + 1);  A2 = symcon2(x2);
//            h2 = sc + A2 Wp2;  e2, g_h2 = readout2;  gA2 = g_h2 Wp2^T;  G1[a:b]_0e += g_h2 Wsk1[s]^T;
//            g_x2, g_rho2 = symcon2^T;  g_msg2 = g_x2 lin2^T / (rho2 + 1);  PF, GX2 += edge_l2_bwd
//            (after all chunks: G1 += GX2 Wup2^T)
//   pass C:  msg1, rho1, x1 as pass A;  g_h1 = G1r[a:b] + scale wr0;  gA1 = g_h1 Wp1^T;  g_x1, g_rho1 = symcon1^T;
//            g_msg1 = g_x1 M0[s]^T / (rho1 + 1);  PF += edge_l1_bwd
#include <stdarg.h>
#include <stdio.h>

#include "common.cuh"
#include "gemm.cuh"
#include "tp_gen.cuh"

namespace mb {

static thread_local char g_err[512] = "";
static unsigned long long g_launches = 0;       // kernels launched by this library (all threads)

// Optional per-kind CUDA-event timing of the pass runners (enabled by mace_b200_timing(1, ...)).
struct KindTimer {
  bool on = false;
  unsigned mask = ~0u;      // kinds recorded while on (bit MB_K_*)
  cudaEvent_t ev[2][8192];
  int kind[8192];
  int n = 0;
  double ms[MB_NKINDS] = {0};
  long long cnt[MB_NKINDS] = {0};
};
static KindTimer g_tm;
static bool g_tm_init = false;

void timer_begin(int kind, cudaStream_t st, int* slot) {
  *slot = -1;
  if (!g_tm.on || !((g_tm.mask >> kind) & 1u) || g_tm.n >= 8192) return;
  *slot = g_tm.n++;
  g_tm.kind[*slot] = kind;
  cudaEventRecord(g_tm.ev[0][*slot], st);
}

void timer_end(int slot, cudaStream_t st) {
  if (slot >= 0) cudaEventRecord(g_tm.ev[1][slot], st);
}

static void timer_flush() {
  if (g_tm.n == 0) return;
  cudaEventSynchronize(g_tm.ev[1][g_tm.n - 1]);
  for (int q = 0; q < g_tm.n; ++q) {
    float t = 0.f;
    if (cudaEventElapsedTime(&t, g_tm.ev[0][q], g_tm.ev[1][q]) == cudaSuccess) {
      g_tm.ms[g_tm.kind[q]] += t;
      g_tm.cnt[g_tm.kind[q]] += 1;
    }
  }
  g_tm.n = 0;
}

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int check_launch(const char* what) {
  __atomic_add_fetch(&g_launches, 1ull, __ATOMIC_RELAXED);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return MB_E_CUDA;
  }
  return 0;
}

int symcon_fwd(const mb_model_t* m, int block, const float* x, float* A, const int32_t* spec, int n, cudaStream_t st);
int symcon_fwd_sorted(const mb_model_t* m, int block, const float* x, float* A, const int32_t* rows,
                      const int32_t* so, cudaStream_t st);
int symcon_bwd_sorted(const mb_model_t* m, int block, const float* x, const float* gA, float* gx,
                      const int32_t* rows, const int32_t* so, const float* rho, float* grho, cudaStream_t st);
int symcon_bwd(const mb_model_t* m, int block, const float* x, const float* gA, float* gx, const int32_t* spec,
               const float* rho, float* grho, int n, cudaStream_t st);
int readout2(const mb_model_t* m, const float* h2, double* eat, float* gh2, int n, cudaStream_t st);
int readout1(const mb_model_t* m, const float* H1, double* eat, int n, cudaStream_t st);
int gh1(const mb_model_t* m, const float* G1, float* out, int n, cudaStream_t st);
int finalize(const mb_model_t* m, const mb_eval_t* ev, const int64_t* perm, double* PFd, unsigned* fmax_bits,
             cudaStream_t st);
int pf_range(const mb_eval_t* ev, int a, int b, cudaStream_t st);

// Species segment offsets (host, S + 1 entries) of chunk ci in its species-sorted row order.
static inline const int32_t* chunk_so(const mb_model_t* m, const mb_eval_t* ev, int ci) {
  return ev->spec_off + (size_t)ci * (m->S + 1);
}

#define TIMED(kind, call)                 \
  do {                                    \
    int _slot;                            \
    timer_begin((kind), st, &_slot);      \
    int _rc = (call);                     \
    timer_end(_slot, st);                 \
    if (_rc) return _rc;                  \
  } while (0)

#define RC(x)                 \
  do {                        \
    int _rc = (x);            \
    if (_rc) return _rc;      \
  } while (0)

// A weight matrix for the node GEMMs: SIMT fp32 row-major W, or its K-major tf32 hi / lo planes W_tc (`plane`
// elements per plane) for the tcgen05 kernel; `off` selects one 128 x 128 (or multi-segment) matrix inside both.
struct Wt {
  const float* W;
  const float* Wtc;
  int64_t plane;
};

static int add(GemmBatch& gb, Wt w, size_t off, const float* X, int64_t ldx, const int32_t* xoff, int nseg, float* Y,
               int64_t ldy, int yoff, int mult, const int32_t* order, int n, const float* rho, int acc) {
  const float* B = gb.tc ? w.Wtc + off : w.W + off;
  return gb.add(X, ldx, xoff, nseg, B, w.plane, Y, ldy, yoff, mult, order, n, rho, acc);
}

static bool use_tc(const mb_model_t* m) {
  return m->use_tc && m->M0_tc && m->M0T_tc && m->Wp1_tc && m->Wp1T_tc && m->Wup2_tc && m->Wup2T_tc && m->Wsk1_tc &&
         m->Wsk1T_tc && m->Wlin2_tc && m->Wlin2T_tc && m->Wp2_tc && m->Wp2T_tc;
}

static int check_pass_args(const mb_model_t* m, const mb_eval_t* ev, const char* who) {
  if (!m || !ev || ev->nl < 0 || ev->nt < ev->nl || ev->chunk <= 0 || m->S <= 0 || m->C != MB_C) {
    set_error("%s: bad model / eval arguments", who);
    return MB_E_ARG;
  }
  if (ev->nl > 0 && (!ev->spec_off || !ev->order || !ev->s_msg || !ev->s_x || !ev->s_gx || !ev->s_a || !ev->s_ga ||
                     !ev->s_h || !ev->s_gh || !ev->s_sc || !ev->s_rho || !ev->s_grho || !ev->H1 || !ev->rowptr)) {
    set_error("%s: missing buffer", who);
    return MB_E_ARG;
  }
  return 0;
}

static const int kOffL[2] = {0, 1};      // component offset of the 0e / 1o blocks of h1-like [4][C] rows

// x1 = msg1 M0[s] / (rho1 + 1) for one chunk: one problem per (l, species segment), one launch
static int x1_gemms(const mb_model_t* m, const mb_eval_t* ev, int a, int ci, cudaStream_t st) {
  const int C = MB_C, S = m->S;
  const int32_t* so = ev->spec_off + (size_t)ci * (S + 1);
  GemmBatch gb(use_tc(m), ev->status, st);
  static const int offs[4] = {0, 1, 4, 9};
  for (int l = 0; l < 4; ++l)
    for (int s = 0; s < S; ++s)
      RC(add(gb, {m->M0, m->M0_tc, (int64_t)S * 4 * C * C}, ((size_t)s * 4 + l) * C * C, ev->s_msg, 16 * C, &offs[l],
             1, ev->s_x, 16 * C, offs[l], 2 * l + 1, ev->order + a + so[s], so[s + 1] - so[s], ev->s_rho, 0));
  return gb.launch();
}

}  // namespace mb

using namespace mb;

extern "C" int mace_b200_abi_version(void) { return MB_ABI_VERSION; }

extern "C" int mace_b200_struct_sizes(int32_t* model_bytes, int32_t* eval_bytes) {
  if (model_bytes) *model_bytes = (int32_t)sizeof(mb_model_t);
  if (eval_bytes) *eval_bytes = (int32_t)sizeof(mb_eval_t);
  return 0;
}

extern "C" unsigned long long mace_b200_launch_count(void) { return __atomic_load_n(&g_launches, __ATOMIC_RELAXED); }

extern "C" int mace_b200_timing(int enable, double* ms_out, long long* count_out) {
  if (!g_tm_init) {
    for (int q = 0; q < 8192; ++q) {
      if (cudaEventCreate(&g_tm.ev[0][q]) != cudaSuccess || cudaEventCreate(&g_tm.ev[1][q]) != cudaSuccess) {
        set_error("timing: cudaEventCreate failed");
        return MB_E_CUDA;
      }
    }
    g_tm_init = true;
  }
  timer_flush();
  if (ms_out)
    for (int k = 0; k < MB_NKINDS; ++k) ms_out[k] = g_tm.ms[k];
  if (count_out)
    for (int k = 0; k < MB_NKINDS; ++k) count_out[k] = g_tm.cnt[k];
  for (int k = 0; k < MB_NKINDS; ++k) {
    g_tm.ms[k] = 0.0;
    g_tm.cnt[k] = 0;
  }
  g_tm.on = enable != 0;
  return 0;
}
extern "C" int mace_b200_timing_kinds(uint32_t mask) {
  g_tm.mask = mask;
  return 0;
}

extern "C" const char* mace_b200_last_error(void) { return g_err; }

// The chunk's view of the eval struct: with the layer-1 cache, x1 and rho1 live in the cache rows of the chunk.
static mb_eval_t chunk_view(const mb_eval_t* ev, int a) {
  mb_eval_t v = *ev;
  if (ev->x1_cache && ev->rho1_cache) {
    v.s_x = ev->x1_cache + (size_t)a * 16 * MB_C;
    v.s_rho = ev->rho1_cache + a;
  }
  return v;
}

static int n_chunks(const mb_eval_t* ev) { return (ev->nl + ev->chunk - 1) / ev->chunk; }

static int chunk_range_ok(const mb_eval_t* ev, int c0, int c1, const char* who) {
  if (c0 < 0 || c1 < c0 || c1 > n_chunks(ev)) {
    set_error("%s: chunk range [%d, %d) outside [0, %d)", who, c0, c1, n_chunks(ev));
    return MB_E_ARG;
  }
  return 0;
}

extern "C" int mace_b200_pass_a_chunks(const mb_model_t* m, const mb_eval_t* ev_all, int32_t c0, int32_t c1,
                                       void* stream) {
  RC(check_pass_args(m, ev_all, "pass_a"));
  RC(chunk_range_ok(ev_all, c0, c1, "pass_a"));
  cudaStream_t st = (cudaStream_t)stream;
  const int C = MB_C;
  for (int ci = c0; ci < c1; ++ci) {
    const int a = ci * ev_all->chunk;
    const mb_eval_t view = chunk_view(ev_all, a);
    const mb_eval_t* ev = &view;
    const int b = min(a + ev->chunk, ev->nl), nC = b - a;
    if (ev_all->wait_ev && ev_all->wait_ev[ci] &&
        cudaStreamWaitEvent(st, (cudaEvent_t)ev_all->wait_ev[ci], 0) != cudaSuccess) {
      set_error("pass_a: cudaStreamWaitEvent on wait_ev[%d] failed", ci);
      return MB_E_CUDA;
    }
    TIMED(MB_K_EDGE_L1_FWD, mace_b200_edge_l1_fwd(m, ev, a, b, st));
    RC(x1_gemms(m, ev, a, ci, st));
    TIMED(MB_K_SYMCON, symcon_fwd_sorted(m, 0, ev->s_x, ev->s_a, ev->order + a, chunk_so(m, ev, ci), st));
    GemmBatch gb(use_tc(m), ev->status, st);
    for (int l = 0; l < 2; ++l)
      RC(add(gb, {m->Wp1, m->Wp1_tc, 2 * C * C}, (size_t)l * C * C, ev->s_a, 4 * C, &kOffL[l], 1,
             ev->H1 + (size_t)a * 4 * C, 4 * C, kOffL[l], 2 * l + 1, nullptr, nC, nullptr, 0));
    RC(gb.launch());
  }
  const int r0 = c0 * ev_all->chunk, r1 = min(c1 * ev_all->chunk, ev_all->nl);
  return r1 > r0 ? readout1(m, ev_all->H1 + (size_t)r0 * 4 * C, ev_all->eat + r0, r1 - r0, st) : 0;
}

extern "C" int mace_b200_pass_a(const mb_model_t* m, const mb_eval_t* ev_all, void* stream) {
  RC(check_pass_args(m, ev_all, "pass_a"));
  return mace_b200_pass_a_chunks(m, ev_all, 0, n_chunks(ev_all), stream);
}

extern "C" int mace_b200_x2_rows(const mb_model_t* m, const mb_eval_t* ev, int32_t r0, int32_t r1, void* stream) {
  RC(check_pass_args(m, ev, "x2_rows"));
  if (r0 < 0 || r1 < r0 || r1 > ev->nt) {
    set_error("x2_rows: rows [%d, %d) outside [0, %d)", r0, r1, ev->nt);
    return MB_E_ARG;
  }
  if (r1 == r0) return 0;
  cudaStream_t st = (cudaStream_t)stream;
  const int C = MB_C;
  const size_t off = (size_t)r0 * 4 * C, bytes = (size_t)(r1 - r0) * 4 * C * sizeof(float);
  if (cudaMemsetAsync(ev->G1 + off, 0, bytes, st) != cudaSuccess ||
      cudaMemsetAsync(ev->GX2 + off, 0, bytes, st) != cudaSuccess) {
    set_error("x2_rows: cudaMemsetAsync failed");
    return MB_E_CUDA;
  }
  GemmBatch gb(use_tc(m), ev->status, st);
  for (int l = 0; l < 2; ++l)
    RC(add(gb, {m->Wup2, m->Wup2_tc, 2 * C * C}, (size_t)l * C * C, ev->H1 + off, 4 * C, &kOffL[l], 1,
           ev->X2 + off, 4 * C, kOffL[l], 2 * l + 1, nullptr, r1 - r0, nullptr, 0));
  return gb.launch();
}

extern "C" int mace_b200_x2_all(const mb_model_t* m, const mb_eval_t* ev, void* stream) {
  RC(check_pass_args(m, ev, "x2_all"));
  return mace_b200_x2_rows(m, ev, 0, ev->nt, stream);
}

extern "C" int mace_b200_pass_b_chunks(const mb_model_t* m, const mb_eval_t* ev, int32_t c0, int32_t c1,
                                       void* stream) {
  RC(check_pass_args(m, ev, "pass_b"));
  RC(chunk_range_ok(ev, c0, c1, "pass_b"));
  cudaStream_t st = (cudaStream_t)stream;
  const int C = MB_C, S = m->S;
  const bool tc = use_tc(m);
  const int zero = 0;
  for (int ci = c0; ci < c1; ++ci) {
    const int a = ci * ev->chunk;
    const int b = min(a + ev->chunk, ev->nl), nC = b - a;
    const int32_t* so = ev->spec_off + (size_t)ci * (S + 1);
    TIMED(MB_K_EDGE_L2_FWD, mace_b200_edge_l2_fwd(m, ev, a, b, st));
    {
      // sc = skip_tp(h1_0e, species) and x2 = linear(msg2) / (rho2 + 1) per output l over its mid copies
      GemmBatch gb(tc, ev->status, st);
      for (int s = 0; s < S; ++s)
        RC(add(gb, {m->Wsk1, m->Wsk1_tc, (int64_t)S * C * C}, (size_t)s * C * C, ev->H1 + (size_t)a * 4 * C, 4 * C,
               &zero, 1, ev->s_sc, C, 0, 1, ev->order + a + so[s], so[s + 1] - so[s], nullptr, 0));
      for (int l = 0; l < 4; ++l) {
        int xoff[4];
        for (int j = 0; j < TP2_GROUP_N[l]; ++j) xoff[j] = TP2_MID_OFF[TP2_GROUP_W0[l] + j];
        RC(add(gb, {m->Wlin2, m->Wlin2_tc, (int64_t)TP2_NW * C * C}, (size_t)TP2_GROUP_W0[l] * C * C, ev->s_msg,
               TP2_NO * C, xoff, TP2_GROUP_N[l], ev->s_x, 16 * C, l * l, 2 * l + 1, nullptr, nC, ev->s_rho, 0));
      }
      RC(gb.launch());
    }
    TIMED(MB_K_SYMCON, symcon_fwd_sorted(m, 1, ev->s_x, ev->s_a, ev->order + a, chunk_so(m, ev, ci), st));
    {
      GemmBatch gb(tc, ev->status, st);   // h2 = sc + A2 Wp2 (in s_sc)
      RC(add(gb, {m->Wp2, m->Wp2_tc, C * C}, 0, ev->s_a, C, &zero, 1, ev->s_sc, C, 0, 1, nullptr, nC, nullptr, 1));
      RC(gb.launch());
    }
    RC(readout2(m, ev->s_sc, ev->eat + a, ev->s_gh, nC, st));
    {
      GemmBatch gb(tc, ev->status, st);   // gA2 = g_h2 Wp2^T;  G1[a:b]_0e += g_h2 Wsk1[s]^T
      RC(add(gb, {m->Wp2T, m->Wp2T_tc, C * C}, 0, ev->s_gh, C, &zero, 1, ev->s_ga, C, 0, 1, nullptr, nC, nullptr, 0));
      for (int s = 0; s < S; ++s)
        RC(add(gb, {m->Wsk1T, m->Wsk1T_tc, (int64_t)S * C * C}, (size_t)s * C * C, ev->s_gh, C, &zero, 1,
               ev->G1 + (size_t)a * 4 * C, 4 * C, 0, 1, ev->order + a + so[s], so[s + 1] - so[s], nullptr, 1));
      RC(gb.launch());
    }
    TIMED(MB_K_SYMCON, symcon_bwd_sorted(m, 1, ev->s_x, ev->s_ga, ev->s_gx, ev->order + a, chunk_so(m, ev, ci),
                                         ev->s_rho, ev->s_grho, st));
    {
      GemmBatch gb(tc, ev->status, st);   // g_msg2 = g_x2 lin2^T / (rho2 + 1), one problem per mid entry
      static const int offs[4] = {0, 1, 4, 9};
      for (int l = 0; l < 4; ++l)
        for (int j = 0; j < TP2_GROUP_N[l]; ++j) {
          const int w = TP2_GROUP_W0[l] + j;
          RC(add(gb, {m->Wlin2T, m->Wlin2T_tc, (int64_t)TP2_NW * C * C}, (size_t)w * C * C, ev->s_gx, 16 * C,
                 &offs[l], 1, ev->s_msg, TP2_NO * C, TP2_MID_OFF[w], 2 * l + 1, nullptr, nC, ev->s_rho, 0));
        }
      RC(gb.launch());
    }
    TIMED(MB_K_EDGE_L2_BWD, mace_b200_edge_l2_bwd(m, ev, a, b, st));
  }
  return 0;
}

extern "C" int mace_b200_fold_g1(const mb_model_t* m, const mb_eval_t* ev, int32_t r0, int32_t r1, void* stream) {
  RC(check_pass_args(m, ev, "fold_g1"));
  if (r0 < 0 || r1 < r0 || r1 > ev->nt) {
    set_error("fold_g1: rows [%d, %d) outside [0, %d)", r0, r1, ev->nt);
    return MB_E_ARG;
  }
  if (r1 == r0) return 0;
  const int C = MB_C;
  const size_t off = (size_t)r0 * 4 * C;
  GemmBatch gb(use_tc(m), ev->status, (cudaStream_t)stream);
  for (int l = 0; l < 2; ++l)
    RC(add(gb, {m->Wup2T, m->Wup2T_tc, 2 * C * C}, (size_t)l * C * C, ev->GX2 + off, 4 * C, &kOffL[l], 1,
           ev->G1 + off, 4 * C, kOffL[l], 2 * l + 1, nullptr, r1 - r0, nullptr, 1));
  return gb.launch();
}

extern "C" int mace_b200_pass_b(const mb_model_t* m, const mb_eval_t* ev, void* stream) {
  RC(check_pass_args(m, ev, "pass_b"));
  if (ev->P > 0 && cudaMemsetAsync(ev->PF, 0, (size_t)ev->P * 3 * sizeof(float), (cudaStream_t)stream) != cudaSuccess) {
    set_error("pass_b: cudaMemsetAsync(PF) failed");
    return MB_E_CUDA;
  }
  RC(mace_b200_pass_b_chunks(m, ev, 0, n_chunks(ev), stream));
  return mace_b200_fold_g1(m, ev, 0, ev->nt, stream);
}


extern "C" int mace_b200_pass_c(const mb_model_t* m, const mb_eval_t* ev_all, void* stream) {
  RC(check_pass_args(m, ev_all, "pass_c"));
  return mace_b200_pass_c_chunks(m, ev_all, 0, n_chunks(ev_all), stream);
}

extern "C" int mace_b200_pass_c_chunks(const mb_model_t* m, const mb_eval_t* ev_all, int32_t c0, int32_t c1,
                                       void* stream) {
  RC(check_pass_args(m, ev_all, "pass_c"));
  RC(chunk_range_ok(ev_all, c0, c1, "pass_c"));
  if (ev_all->done_ev && (!ev_all->pf_out || !ev_all->fmax_bits)) {
    set_error("pass_c: done_ev needs pf_out and fmax_bits");
    return MB_E_ARG;
  }
  cudaStream_t st = (cudaStream_t)stream;
  const int C = MB_C, S = m->S;
  const bool tc = use_tc(m);
  const bool cached = ev_all->x1_cache && ev_all->rho1_cache;
  static const int offs[4] = {0, 1, 4, 9};
  for (int ci = c0; ci < c1; ++ci) {
    const int a = ci * ev_all->chunk;
    const mb_eval_t view = chunk_view(ev_all, a);
    const mb_eval_t* ev = &view;
    const int b = min(a + ev->chunk, ev->nl), nC = b - a;
    const int32_t* so = ev->spec_off + (size_t)ci * (S + 1);
    if (!cached) {
      TIMED(MB_K_EDGE_L1_FWD, mace_b200_edge_l1_fwd(m, ev, a, b, st));
      RC(x1_gemms(m, ev, a, ci, st));
    }
    RC(gh1(m, ev->G1 + (size_t)a * 4 * C, ev->s_a, nC, st));
    {
      GemmBatch gb(tc, ev->status, st);   // gA1 = g_h1 Wp1^T
      for (int l = 0; l < 2; ++l)
        RC(add(gb, {m->Wp1T, m->Wp1T_tc, 2 * C * C}, (size_t)l * C * C, ev->s_a, 4 * C, &kOffL[l], 1, ev->s_ga,
               4 * C, kOffL[l], 2 * l + 1, nullptr, nC, nullptr, 0));
      RC(gb.launch());
    }
    TIMED(MB_K_SYMCON, symcon_bwd_sorted(m, 0, ev->s_x, ev->s_ga, ev->s_gx, ev->order + a, chunk_so(m, ev, ci),
                                         ev->s_rho, ev->s_grho, st));
    {
      GemmBatch gb(tc, ev->status, st);   // g_msg1 = g_x1 M0[s]^T / (rho1 + 1)
      for (int l = 0; l < 4; ++l)
        for (int s = 0; s < S; ++s)
          RC(add(gb, {m->M0T, m->M0T_tc, (int64_t)S * 4 * C * C}, ((size_t)s * 4 + l) * C * C, ev->s_gx, 16 * C,
                 &offs[l], 1, ev->s_msg, 16 * C, offs[l], 2 * l + 1, ev->order + a + so[s], so[s + 1] - so[s],
                 ev->s_rho, 0));
      RC(gb.launch());
    }
    TIMED(MB_K_EDGE_L1_BWD, mace_b200_edge_l1_bwd(m, ev, a, b, st));
    if (ev_all->done_ev) {                     // the chunk's pair forces are final: hand them out now
      RC(pf_range(ev_all, a, b, st));
      if (cudaEventRecord((cudaEvent_t)ev_all->done_ev[ci], st) != cudaSuccess) {
        set_error("pass_c: cudaEventRecord of done_ev[%d] failed", ci);
        return MB_E_CUDA;
      }
    }
  }
  return 0;
}

extern "C" int mace_b200_finalize(const mb_model_t* m, const mb_eval_t* ev, const int64_t* perm, double* PFd,
                                  uint32_t* fmax_bits, void* stream) {
  if (!m || !ev || !PFd || !fmax_bits || !ev->PF || !ev->eat) {
    set_error("finalize: bad arguments");
    return MB_E_ARG;
  }
  return finalize(m, ev, perm, PFd, fmax_bits, (cudaStream_t)stream);
}
