// torch.ops.mace_b200.*: thin custom-op wrappers over the C ABI of libmace_b200.so (include/mace_b200.h), registered
// with TORCH_LIBRARY.  Every op takes tensors and int64 / double / bool scalars only, checks devices, dtypes, shapes
// and contiguity with TORCH_CHECK (a RuntimeError in Python), launches on torch's current CUDA stream and allocates
// its outputs with torch's caching allocator.  They are the per-kernel building blocks the reference's plugin API
// names (tables, edge kernels, symmetric contraction, node GEMM, halo pack / unpack, CSR rows, the output guard) and
// the body of FusedConvTP (mace_onegpu/fused_conv.py:20-37 in the reference).  The three-pass evaluation itself runs
// through the native pass runners (mace_b200_pass_a / _b / _c), which launch the same kernels.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <cstdio>
#include <cstring>
#include <tuple>

#include "../../include/mace_b200.h"

namespace {

using at::Tensor;

void* stream_of(const Tensor& t) { return (void*)at::cuda::getCurrentCUDAStream(t.device().index()).stream(); }

void check_rc(int rc, const char* what) {
  TORCH_CHECK(rc == 0, "mace_b200::", what, ": ", mace_b200_last_error(), " (code ", rc, ")");
}

void need(const Tensor& t, at::ScalarType dt, const char* name, const Tensor& like) {
  TORCH_CHECK(t.defined() && t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.device() == like.device(), name, " must be on ", like.device());
  TORCH_CHECK(t.scalar_type() == dt, name, " must be ", c10::toString(dt), " (got ", t.scalar_type(), ")");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

template <typename T>
const T* cptr(const Tensor& t) { return t.defined() ? t.data_ptr<T>() : nullptr; }
template <typename T>
T* mptr(const Tensor& t) { return t.defined() ? t.data_ptr<T>() : nullptr; }

// ------------------------------------------------------------------------------------------------ FusedConvTP
struct Csr {
  Tensor rowptr, edges;
};

// CSR of the edges grouped by `node` (stable: the edges of one node keep their order).
Csr csr_of(const Tensor& node, int64_t n) {
  Tensor key = node.to(at::kLong);
  Tensor edges = std::get<1>(at::sort(key, /*stable=*/true, /*dim=*/0, /*descending=*/false)).contiguous();
  Tensor bounds = at::arange(n + 1, key.options());
  Tensor rowptr = at::searchsorted(key.index_select(0, edges), bounds).to(at::kLong).contiguous();
  return {rowptr, edges};
}

struct ConvIn {
  Tensor X, Y, W, snd, rcv, terms, coef;
  int64_t n, E, nX, nY, nW, nT;
};

ConvIn conv_in(const Tensor& X, const Tensor& Y, const Tensor& W, const Tensor& edge_index, const Tensor& terms,
               const Tensor& coef) {
  ConvIn c;
  TORCH_CHECK(X.dim() == 2 && X.size(1) % 128 == 0, "node_feats must be [n, nX * 128]");
  TORCH_CHECK(W.dim() == 2 && W.size(1) % 128 == 0, "tp_weights must be [E, nW * 128]");
  TORCH_CHECK(Y.dim() == 2, "edge_attrs must be [E, nY]");
  TORCH_CHECK(edge_index.dim() == 2 && edge_index.size(0) == 2, "edge_index must be [2, E]");
  TORCH_CHECK(terms.dim() == 2 && terms.size(1) == 4, "terms must be [n_terms, 4] = (w, k, m, o)");
  c.X = X.contiguous();
  c.Y = Y.contiguous();
  c.W = W.contiguous();
  c.terms = terms.contiguous();
  c.coef = coef.contiguous();
  need(c.X, at::kFloat, "node_feats", c.X);
  need(c.Y, at::kFloat, "edge_attrs", c.X);
  need(c.W, at::kFloat, "tp_weights", c.X);
  need(c.terms, at::kInt, "terms", c.X);
  need(c.coef, at::kFloat, "coef", c.X);
  TORCH_CHECK(edge_index.device() == c.X.device(), "edge_index must be on ", c.X.device());
  c.snd = edge_index[0].to(at::kInt).contiguous();
  c.rcv = edge_index[1].to(at::kInt).contiguous();
  c.n = c.X.size(0);
  c.E = edge_index.size(1);
  TORCH_CHECK(c.Y.size(0) == c.E && c.W.size(0) == c.E, "edge_attrs / tp_weights must have E rows");
  TORCH_CHECK(c.coef.numel() == c.terms.size(0), "one coefficient per term");
  c.nX = c.X.size(1) / 128;
  c.nY = c.Y.size(1);
  c.nW = c.W.size(1) / 128;
  c.nT = c.terms.size(0);
  return c;
}

Tensor conv_tp(const Tensor& X, const Tensor& Y, const Tensor& W, const Tensor& edge_index, const Tensor& terms,
               const Tensor& coef, int64_t nO) {
  ConvIn c = conv_in(X, Y, W, edge_index, terms, coef);
  c10::cuda::CUDAGuard guard(c.X.device());
  Tensor out = at::empty({c.n, nO * 128}, c.X.options());
  if (c.n == 0) return out;
  Csr r = csr_of(c.rcv, c.n);
  Tensor status = at::zeros({1}, c.X.options().dtype(at::kInt));
  check_rc(mace_b200_conv_tp_fwd(c.X.data_ptr<float>(), (int32_t)c.nX, c.Y.data_ptr<float>(), (int32_t)c.nY,
                                 c.W.data_ptr<float>(), (int32_t)c.nW, c.snd.data_ptr<int32_t>(),
                                 r.rowptr.data_ptr<int64_t>(), r.edges.data_ptr<int64_t>(), (int32_t)c.n,
                                 c.terms.data_ptr<int32_t>(), c.coef.data_ptr<float>(), (int32_t)c.nT,
                                 out.data_ptr<float>(), (int32_t)nO, (uint32_t*)status.data_ptr<int32_t>(),
                                 stream_of(c.X)),
           "conv_tp");
  return out;
}

std::tuple<Tensor, Tensor, Tensor> conv_tp_backward(const Tensor& grad, const Tensor& X, const Tensor& Y,
                                                    const Tensor& W, const Tensor& edge_index, const Tensor& terms,
                                                    const Tensor& coef, int64_t nO, bool need_x, bool need_y,
                                                    bool need_w) {
  ConvIn c = conv_in(X, Y, W, edge_index, terms, coef);
  c10::cuda::CUDAGuard guard(c.X.device());
  Tensor g = grad.contiguous();
  need(g, at::kFloat, "grad", c.X);
  TORCH_CHECK(g.size(0) == c.n && g.size(1) == nO * 128, "grad must be [n, nO * 128]");
  Tensor dX = need_x ? at::empty_like(c.X) : Tensor();
  Tensor dY = need_y ? at::empty_like(c.Y) : Tensor();
  Tensor dW = need_w ? at::empty_like(c.W) : Tensor();
  if (c.n == 0 || c.E == 0) {
    for (Tensor* t : {&dX, &dY, &dW})
      if (t->defined()) t->zero_();
    return {dX, dY, dW};
  }
  Csr r = csr_of(c.rcv, c.n);
  Csr s = need_x ? csr_of(c.snd, c.n) : Csr{};
  Tensor status = at::zeros({1}, c.X.options().dtype(at::kInt));
  check_rc(mace_b200_conv_tp_bwd(c.X.data_ptr<float>(), (int32_t)c.nX, c.Y.data_ptr<float>(), (int32_t)c.nY,
                                 c.W.data_ptr<float>(), (int32_t)c.nW, c.snd.data_ptr<int32_t>(),
                                 c.rcv.data_ptr<int32_t>(), r.rowptr.data_ptr<int64_t>(),
                                 r.edges.data_ptr<int64_t>(), cptr<int64_t>(s.rowptr), cptr<int64_t>(s.edges),
                                 (int32_t)c.n, c.terms.data_ptr<int32_t>(), c.coef.data_ptr<float>(), (int32_t)c.nT,
                                 g.data_ptr<float>(), (int32_t)nO, mptr<float>(dX), mptr<float>(dY), mptr<float>(dW),
                                 (uint32_t*)status.data_ptr<int32_t>(), stream_of(c.X)),
           "conv_tp_backward");
  return {dX, dY, dW};
}

// ------------------------------------------------------------------------------------------------ tables
std::tuple<Tensor, Tensor, Tensor> build_tables(const Tensor& A0, const Tensor& A1, const Tensor& A2,
                                                const Tensor& A3, const c10::optional<Tensor>& col_scale,
                                                int64_t n_pairs, int64_t M, double r_lo, double r_max, double p_cut) {
  for (const Tensor* p : {&A0, &A1, &A2, &A3}) need(*p, at::kDouble, "radial MLP matrix", A0);
  TORCH_CHECK(A0.dim() == 2 && A1.dim() == 2 && A2.dim() == 2 && A3.dim() == 2, "A0..A3 must be matrices");
  const int64_t D = A3.size(1);
  Tensor cs;
  if (col_scale && col_scale->defined()) {
    cs = *col_scale;
    need(cs, at::kDouble, "col_scale", A0);
    TORCH_CHECK(cs.numel() == n_pairs * D, "col_scale must be [n_pairs, D]");
  }
  c10::cuda::CUDAGuard guard(A0.device());
  auto f32 = A0.options().dtype(at::kFloat);
  Tensor TV = at::empty({n_pairs, M, D}, f32), TG = at::empty({n_pairs, M, D}, f32);
  Tensor cub = at::empty({n_pairs, M - 1, D, 4}, f32);
  check_rc(mace_b200_build_tables(A0.data_ptr<double>(), A1.data_ptr<double>(), A2.data_ptr<double>(),
                                  A3.data_ptr<double>(), (int32_t)A0.size(0), (int32_t)A0.size(1), (int32_t)D,
                                  cptr<double>(cs), (int32_t)n_pairs, (int32_t)M, r_lo, r_max, p_cut,
                                  TV.data_ptr<float>(), TG.data_ptr<float>(), cub.data_ptr<float>(), stream_of(A0)),
           "build_tables");
  return {TV, TG, cub};
}

// ------------------------------------------------------------------------------------------------ edge kernels
struct Geo {
  mb_model_t m;
  mb_eval_t ev;
};

// The struct fields every edge kernel reads: radial constants, species count, pair list, CSR, species, status.
Geo geo(const Tensor& pair_i, const Tensor& pair_j, const Tensor& rij, const Tensor& rowptr, const Tensor& spec,
        const Tensor& status, int64_t S, int64_t M, double r_lo, double r_max, double p_cut) {
  need(pair_i, at::kInt, "pair_i", rij);
  need(pair_j, at::kInt, "pair_j", rij);
  need(rij, at::kDouble, "rij", rij);
  need(rowptr, at::kInt, "rowptr", rij);
  need(spec, at::kInt, "spec", rij);
  need(status, at::kInt, "status", rij);
  TORCH_CHECK(rij.numel() == 3 * pair_i.numel() && pair_j.numel() == pair_i.numel(), "pair arrays must agree");
  TORCH_CHECK(M >= 2 && r_max > r_lo, "bad spline grid");
  Geo g;
  std::memset(&g, 0, sizeof(g));
  g.m.C = 128;
  g.m.S = (int32_t)S;
  g.m.M = (int32_t)M;
  g.m.r_lo = (float)r_lo;
  g.m.inv_h = (float)((M - 1) / (r_max - r_lo));
  g.m.r_max = (float)r_max;
  g.m.p_cut = (float)p_cut;
  g.ev.nl = (int32_t)(rowptr.numel() - 1);
  g.ev.nt = (int32_t)spec.numel();
  g.ev.P = pair_i.numel();
  g.ev.pair_i = pair_i.data_ptr<int32_t>();
  g.ev.pair_j = pair_j.data_ptr<int32_t>();
  g.ev.rij = rij.data_ptr<double>();
  g.ev.rowptr = rowptr.data_ptr<int32_t>();
  g.ev.spec = spec.data_ptr<int32_t>();
  g.ev.status = (uint32_t*)status.data_ptr<int32_t>();
  return g;
}

void rows(const Tensor& t, int64_t nC, int64_t width, const char* name, const Tensor& like) {
  need(t, at::kFloat, name, like);
  TORCH_CHECK(t.numel() >= nC * width, name, " must hold ", nC, " rows of ", width, " floats");
}

void edge_l1(bool fwd, const Tensor& tab1, const c10::optional<Tensor>& tab1_map, const Tensor& wd1,
             int64_t l1_density, const Tensor& pair_i, const Tensor& pair_j, const Tensor& rij, const Tensor& rowptr,
             const Tensor& spec, const Tensor& s_msg, const Tensor& s_rho, const Tensor& s_grho, const Tensor& PF,
             const Tensor& status, int64_t a, int64_t b, int64_t S, int64_t M, double r_lo, double r_max,
             double p_cut) {
  c10::cuda::CUDAGuard guard(rij.device());
  Geo g = geo(pair_i, pair_j, rij, rowptr, spec, status, S, M, r_lo, r_max, p_cut);
  need(tab1, at::kFloat, "tab1", rij);
  need(wd1, at::kFloat, "wd1", rij);
  rows(s_msg, b - a, 16 * 128, "s_msg", rij);
  g.m.tab1 = tab1.data_ptr<float>();
  g.m.wd1 = wd1.data_ptr<float>();
  g.m.l1_density = (int32_t)l1_density;
  if (tab1_map && tab1_map->defined()) {
    need(*tab1_map, at::kInt, "tab1_map", rij);
    g.m.tab1_map = tab1_map->data_ptr<int32_t>();
  }
  g.ev.s_msg = s_msg.data_ptr<float>();
  if (fwd) {
    rows(s_rho, b - a, 1, "s_rho", rij);
    g.ev.s_rho = s_rho.data_ptr<float>();
    check_rc(mace_b200_edge_l1_fwd(&g.m, &g.ev, (int32_t)a, (int32_t)b, stream_of(rij)), "edge_l1_fwd");
  } else {
    rows(s_grho, b - a, 1, "s_grho", rij);
    rows(PF, g.ev.P, 3, "PF", rij);
    g.ev.s_grho = s_grho.data_ptr<float>();
    g.ev.PF = PF.data_ptr<float>();
    check_rc(mace_b200_edge_l1_bwd(&g.m, &g.ev, (int32_t)a, (int32_t)b, stream_of(rij)), "edge_l1_bwd");
  }
}

void edge_l1_fwd(const Tensor& tab1, const c10::optional<Tensor>& tab1_map, const Tensor& wd1, int64_t l1_density,
                 const Tensor& pair_i, const Tensor& pair_j, const Tensor& rij, const Tensor& rowptr,
                 const Tensor& spec, const Tensor& s_msg, const Tensor& s_rho, const Tensor& status, int64_t a,
                 int64_t b, int64_t S, int64_t M, double r_lo, double r_max, double p_cut) {
  edge_l1(true, tab1, tab1_map, wd1, l1_density, pair_i, pair_j, rij, rowptr, spec, s_msg, s_rho, Tensor(), Tensor(),
          status, a, b, S, M, r_lo, r_max, p_cut);
}

void edge_l1_bwd(const Tensor& tab1, const c10::optional<Tensor>& tab1_map, const Tensor& wd1, int64_t l1_density,
                 const Tensor& pair_i, const Tensor& pair_j, const Tensor& rij, const Tensor& rowptr,
                 const Tensor& spec, const Tensor& s_msg, const Tensor& s_grho, const Tensor& PF,
                 const Tensor& status, int64_t a, int64_t b, int64_t S, int64_t M, double r_lo, double r_max,
                 double p_cut) {
  edge_l1(false, tab1, tab1_map, wd1, l1_density, pair_i, pair_j, rij, rowptr, spec, s_msg, Tensor(), s_grho, PF,
          status, a, b, S, M, r_lo, r_max, p_cut);
}

void edge_l2(bool fwd, const Tensor& tab2, const c10::optional<Tensor>& tab2_map, const Tensor& wd2,
             const Tensor& pair_i, const Tensor& pair_j, const Tensor& rij, const Tensor& rowptr, const Tensor& spec,
             const Tensor& X2, const Tensor& s_msg, const Tensor& s_rho, const Tensor& s_grho, const Tensor& GX2,
             const Tensor& PF, const Tensor& status, int64_t a, int64_t b, int64_t S, int64_t M, double r_lo,
             double r_max, double p_cut) {
  c10::cuda::CUDAGuard guard(rij.device());
  Geo g = geo(pair_i, pair_j, rij, rowptr, spec, status, S, M, r_lo, r_max, p_cut);
  need(tab2, at::kFloat, "tab2", rij);
  need(wd2, at::kFloat, "wd2", rij);
  rows(X2, g.ev.nt, 4 * 128, "X2", rij);
  rows(s_msg, b - a, 40 * 128, "s_msg", rij);
  g.m.tab2 = tab2.data_ptr<float>();
  g.m.wd2 = wd2.data_ptr<float>();
  if (tab2_map && tab2_map->defined()) {
    need(*tab2_map, at::kInt, "tab2_map", rij);
    g.m.tab2_map = tab2_map->data_ptr<int32_t>();
  }
  g.ev.X2 = X2.data_ptr<float>();
  g.ev.s_msg = s_msg.data_ptr<float>();
  if (fwd) {
    rows(s_rho, b - a, 1, "s_rho", rij);
    g.ev.s_rho = s_rho.data_ptr<float>();
    check_rc(mace_b200_edge_l2_fwd(&g.m, &g.ev, (int32_t)a, (int32_t)b, stream_of(rij)), "edge_l2_fwd");
  } else {
    rows(s_grho, b - a, 1, "s_grho", rij);
    rows(GX2, g.ev.nt, 4 * 128, "GX2", rij);
    rows(PF, g.ev.P, 3, "PF", rij);
    g.ev.s_grho = s_grho.data_ptr<float>();
    g.ev.GX2 = GX2.data_ptr<float>();
    g.ev.PF = PF.data_ptr<float>();
    check_rc(mace_b200_edge_l2_bwd(&g.m, &g.ev, (int32_t)a, (int32_t)b, stream_of(rij)), "edge_l2_bwd");
  }
}

void edge_l2_fwd(const Tensor& tab2, const c10::optional<Tensor>& tab2_map, const Tensor& wd2, const Tensor& pair_i,
                 const Tensor& pair_j, const Tensor& rij, const Tensor& rowptr, const Tensor& spec, const Tensor& X2,
                 const Tensor& s_msg, const Tensor& s_rho, const Tensor& status, int64_t a, int64_t b, int64_t S,
                 int64_t M, double r_lo, double r_max, double p_cut) {
  edge_l2(true, tab2, tab2_map, wd2, pair_i, pair_j, rij, rowptr, spec, X2, s_msg, s_rho, Tensor(), Tensor(),
          Tensor(), status, a, b, S, M, r_lo, r_max, p_cut);
}

void edge_l2_bwd(const Tensor& tab2, const c10::optional<Tensor>& tab2_map, const Tensor& wd2, const Tensor& pair_i,
                 const Tensor& pair_j, const Tensor& rij, const Tensor& rowptr, const Tensor& spec, const Tensor& X2,
                 const Tensor& s_msg, const Tensor& s_grho, const Tensor& GX2, const Tensor& PF,
                 const Tensor& status, int64_t a, int64_t b, int64_t S, int64_t M, double r_lo, double r_max,
                 double p_cut) {
  edge_l2(false, tab2, tab2_map, wd2, pair_i, pair_j, rij, rowptr, spec, X2, s_msg, Tensor(), s_grho, GX2, PF,
          status, a, b, S, M, r_lo, r_max, p_cut);
}

// ------------------------------------------------------------------------------------------------ node side
void node_gemm(const Tensor& X, int64_t ldx, const Tensor& xoff, const Tensor& B, const Tensor& Y, int64_t ldy,
               int64_t yoff, int64_t mult, const c10::optional<Tensor>& order, int64_t n_atoms,
               const c10::optional<Tensor>& rho, bool accumulate) {
  need(X, at::kFloat, "X", X);
  need(B, at::kFloat, "B", X);
  need(Y, at::kFloat, "Y", X);
  TORCH_CHECK(xoff.device().is_cpu() && xoff.scalar_type() == at::kInt && xoff.is_contiguous(),
              "xoff must be a contiguous int32 CPU tensor (segment offsets)");
  const int64_t nseg = xoff.numel();
  TORCH_CHECK(B.numel() == nseg * 128 * 128, "B must be [n_seg, 128, 128]");
  const int32_t* ord = nullptr;
  const float* rh = nullptr;
  if (order && order->defined()) {
    need(*order, at::kInt, "order", X);
    ord = order->data_ptr<int32_t>();
  }
  if (rho && rho->defined()) {
    need(*rho, at::kFloat, "rho", X);
    rh = rho->data_ptr<float>();
  }
  c10::cuda::CUDAGuard guard(X.device());
  check_rc(mace_b200_node_gemm(X.data_ptr<float>(), ldx, xoff.data_ptr<int32_t>(), (int32_t)nseg, B.data_ptr<float>(),
                               Y.data_ptr<float>(), ldy, (int32_t)yoff, (int32_t)mult, ord, (int32_t)n_atoms, rh,
                               accumulate ? 1 : 0, stream_of(X)),
           "node_gemm");
}

mb_model_t sc_model(const Tensor& sc, int64_t block, int64_t S) {
  mb_model_t m;
  std::memset(&m, 0, sizeof(m));
  m.C = 128;
  m.S = (int32_t)S;
  if (block == 0)
    m.sc1 = sc.data_ptr<float>();
  else
    m.sc2 = sc.data_ptr<float>();
  return m;
}

Tensor symcon_fwd(const Tensor& sc, int64_t block, int64_t S, const Tensor& x, const Tensor& spec) {
  TORCH_CHECK(block == 0 || block == 1, "block must be 0 (layer 1) or 1 (layer 2)");
  need(sc, at::kFloat, "sc", x);
  need(x, at::kFloat, "x", x);
  need(spec, at::kInt, "spec", x);
  const int64_t n = spec.numel();
  TORCH_CHECK(x.numel() == n * 16 * 128, "x must be [n, 16, 128]");
  c10::cuda::CUDAGuard guard(x.device());
  Tensor A = at::empty({n, block == 0 ? 4 : 1, 128}, x.options());
  mb_model_t m = sc_model(sc, block, S);
  check_rc(mace_b200_symcon_fwd(&m, (int32_t)block, x.data_ptr<float>(), A.data_ptr<float>(), spec.data_ptr<int32_t>(),
                                (int32_t)n, stream_of(x)),
           "symcon_fwd");
  return A;
}

std::tuple<Tensor, Tensor> symcon_bwd(const Tensor& sc, int64_t block, int64_t S, const Tensor& x, const Tensor& gA,
                                      const Tensor& spec, const c10::optional<Tensor>& rho) {
  TORCH_CHECK(block == 0 || block == 1, "block must be 0 (layer 1) or 1 (layer 2)");
  need(sc, at::kFloat, "sc", x);
  need(x, at::kFloat, "x", x);
  need(gA, at::kFloat, "gA", x);
  need(spec, at::kInt, "spec", x);
  const int64_t n = spec.numel();
  TORCH_CHECK(x.numel() == n * 16 * 128 && gA.numel() == n * (block == 0 ? 4 : 1) * 128, "x / gA shapes");
  c10::cuda::CUDAGuard guard(x.device());
  Tensor gx = at::empty_like(x);
  Tensor grho;
  const float* rh = nullptr;
  if (rho && rho->defined()) {
    need(*rho, at::kFloat, "rho", x);
    rh = rho->data_ptr<float>();
    grho = at::empty({n}, x.options());
  }
  mb_model_t m = sc_model(sc, block, S);
  check_rc(mace_b200_symcon_bwd(&m, (int32_t)block, x.data_ptr<float>(), gA.data_ptr<float>(), gx.data_ptr<float>(),
                                spec.data_ptr<int32_t>(), rh, mptr<float>(grho), (int32_t)n, stream_of(x)),
           "symcon_bwd");
  return {gx, grho};
}

// ------------------------------------------------------------------------------------------------ halo, CSR, guard
Tensor pack_halo(const Tensor& src, const Tensor& idx) {
  need(src, at::kFloat, "src", src);
  need(idx, at::kInt, "idx", src);
  TORCH_CHECK(src.dim() == 2, "src must be [rows, D]");
  c10::cuda::CUDAGuard guard(src.device());
  Tensor buf = at::empty({idx.numel(), src.size(1)}, src.options());
  check_rc(mace_b200_pack_rows(src.data_ptr<float>(), idx.data_ptr<int32_t>(), idx.numel(), (int32_t)src.size(1),
                               buf.data_ptr<float>(), stream_of(src)),
           "pack_halo");
  return buf;
}

void unpack_halo_add(const Tensor& dst, const Tensor& buf, const Tensor& idx) {
  need(dst, at::kFloat, "dst", dst);
  need(buf, at::kFloat, "buf", dst);
  need(idx, at::kInt, "idx", dst);
  TORCH_CHECK(dst.dim() == 2 && buf.dim() == 2 && buf.size(1) == dst.size(1) && buf.size(0) == idx.numel(),
              "buf must be [len(idx), D] with dst [rows, D]");
  c10::cuda::CUDAGuard guard(dst.device());
  check_rc(mace_b200_unpack_add_rows(buf.data_ptr<float>(), idx.data_ptr<int32_t>(), idx.numel(),
                                     (int32_t)dst.size(1), dst.data_ptr<float>(), stream_of(dst)),
           "unpack_halo_add");
}

void csr_rows(const Tensor& pair_i, int64_t e0, int64_t e1, int64_t a, int64_t b, const Tensor& rowptr,
              const Tensor& status) {
  need(pair_i, at::kInt, "pair_i", pair_i);
  need(rowptr, at::kInt, "rowptr", pair_i);
  need(status, at::kInt, "status", pair_i);
  TORCH_CHECK(e1 <= pair_i.numel() && b < rowptr.numel(), "edge / receiver range outside the arrays");
  c10::cuda::CUDAGuard guard(pair_i.device());
  check_rc(mace_b200_csr_rows(pair_i.data_ptr<int32_t>(), e0, e1, (int32_t)a, (int32_t)b, rowptr.data_ptr<int32_t>(),
                              (uint32_t*)status.data_ptr<int32_t>(), stream_of(pair_i)),
           "csr_rows");
}

// Output guard of the ML-IAP call (mliap_threepass.py:595-601 in the reference): non-finite energies, or a pair-force
// maximum that is non-finite or not below fmax_abort, abort the call with the reference's message before LAMMPS
// would integrate the forces.  Reads device or host energies (one device -> host read for device tensors).
void guard(const Tensor& eatoms, double fmax, double fmax_abort, int64_t step) {
  const bool finite = eatoms.numel() == 0 || at::isfinite(eatoms).all().item<bool>();
  char buf[160];
  std::snprintf(buf, sizeof(buf), "(max |pair force| = %.3e eV/A, limit %g)", fmax, fmax_abort);
  TORCH_CHECK(finite && fmax == fmax && fmax < fmax_abort, "ThreePassMLIAP guard: non-finite or absurd output at call ",
              step, " ", buf,
              "; aborting before LAMMPS integrates it. The model is probably extrapolating (check the trajectory / "
              "training data).");
}

}  // namespace

TORCH_LIBRARY(mace_b200, m) {
  m.def("conv_tp(Tensor node_feats, Tensor edge_attrs, Tensor tp_weights, Tensor edge_index, Tensor terms, "
        "Tensor coef, int n_out) -> Tensor");
  m.def("conv_tp_backward(Tensor grad, Tensor node_feats, Tensor edge_attrs, Tensor tp_weights, Tensor edge_index, "
        "Tensor terms, Tensor coef, int n_out, bool need_x, bool need_y, bool need_w) -> (Tensor, Tensor, Tensor)");
  m.def("build_tables(Tensor A0, Tensor A1, Tensor A2, Tensor A3, Tensor? col_scale, int n_pairs, int M, "
        "float r_lo, float r_max, float p_cut) -> (Tensor, Tensor, Tensor)");
  m.def("edge_l1_fwd(Tensor tab1, Tensor? tab1_map, Tensor wd1, int l1_density, Tensor pair_i, Tensor pair_j, "
        "Tensor rij, Tensor rowptr, Tensor spec, Tensor(a!) s_msg, Tensor(b!) s_rho, Tensor(c!) status, int a, int b, "
        "int S, int M, float r_lo, float r_max, float p_cut) -> ()");
  m.def("edge_l1_bwd(Tensor tab1, Tensor? tab1_map, Tensor wd1, int l1_density, Tensor pair_i, Tensor pair_j, "
        "Tensor rij, Tensor rowptr, Tensor spec, Tensor s_msg, Tensor s_grho, Tensor(a!) PF, Tensor(b!) status, "
        "int a, int b, int S, int M, float r_lo, float r_max, float p_cut) -> ()");
  m.def("edge_l2_fwd(Tensor tab2, Tensor? tab2_map, Tensor wd2, Tensor pair_i, Tensor pair_j, Tensor rij, "
        "Tensor rowptr, Tensor spec, Tensor X2, Tensor(a!) s_msg, Tensor(b!) s_rho, Tensor(c!) status, int a, int b, "
        "int S, int M, float r_lo, float r_max, float p_cut) -> ()");
  m.def("edge_l2_bwd(Tensor tab2, Tensor? tab2_map, Tensor wd2, Tensor pair_i, Tensor pair_j, Tensor rij, "
        "Tensor rowptr, Tensor spec, Tensor X2, Tensor s_msg, Tensor s_grho, Tensor(a!) GX2, Tensor(b!) PF, "
        "Tensor(c!) status, int a, int b, int S, int M, float r_lo, float r_max, float p_cut) -> ()");
  m.def("node_gemm(Tensor X, int ldx, Tensor xoff, Tensor B, Tensor(a!) Y, int ldy, int yoff, int mult, "
        "Tensor? order, int n_atoms, Tensor? rho, bool accumulate) -> ()");
  m.def("symcon_fwd(Tensor sc, int block, int S, Tensor x, Tensor spec) -> Tensor");
  m.def("symcon_bwd(Tensor sc, int block, int S, Tensor x, Tensor gA, Tensor spec, Tensor? rho) -> (Tensor, Tensor)");
  m.def("pack_halo(Tensor src, Tensor idx) -> Tensor");
  m.def("unpack_halo_add(Tensor(a!) dst, Tensor buf, Tensor idx) -> ()");
  m.def("csr_rows(Tensor pair_i, int e0, int e1, int a, int b, Tensor(a!) rowptr, Tensor(b!) status) -> ()");
  m.def("guard(Tensor eatoms, float fmax, float fmax_abort, int step) -> ()");
}

TORCH_LIBRARY_IMPL(mace_b200, CUDA, m) {
  m.impl("conv_tp", &conv_tp);
  m.impl("conv_tp_backward", &conv_tp_backward);
  m.impl("build_tables", &build_tables);
  m.impl("edge_l1_fwd", &edge_l1_fwd);
  m.impl("edge_l1_bwd", &edge_l1_bwd);
  m.impl("edge_l2_fwd", &edge_l2_fwd);
  m.impl("edge_l2_bwd", &edge_l2_bwd);
  m.impl("node_gemm", &node_gemm);
  m.impl("symcon_fwd", &symcon_fwd);
  m.impl("symcon_bwd", &symcon_bwd);
  m.impl("pack_halo", &pack_halo);
  m.impl("unpack_halo_add", &unpack_halo_add);
  m.impl("csr_rows", &csr_rows);
}

// The guard reads device or host energies alike.
TORCH_LIBRARY_IMPL(mace_b200, CompositeExplicitAutograd, m) { m.impl("guard", &guard); }
