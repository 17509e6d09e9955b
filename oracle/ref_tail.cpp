// Harness over the reference's own logits tail - TEST INFRASTRUCTURE ONLY.
//
// The reference's rmsnorm is file-local to src/session.cpp, so this harness
// compiles that translation unit itself (unmodified, from the reference
// checkout) and calls, in the order of Session::Impl::batch
// (src/session.cpp:163-169) and Session::Impl::act (src/session.cpp:88-103):
// rmsnorm per row, quant_act per row for quantised heads, then matmul over a
// Pool.  oracle/Makefile links it twice: with the reference's default
// (AVX2) kernels.cpp and with kernels.cpp built as the VERBO_SCALAR option
// builds it.
#include "session.cpp"

#include <cstring>
#include <vector>

#include "oracle.h"

namespace {

// Session keeps its residual stream behind a private pointer.  An explicit
// instantiation may name a private member, so this template reads
// Session::Impl::x (the rows batch() ran, before the final rmsnorm) without
// touching the reference's sources.
template <auto M>
struct ResidualOf {
  friend const std::vector<float>* residual_of(verbo::Session& s) { return &((s.*M)->x); }
};
template struct ResidualOf<&verbo::Session::impl_>;
const std::vector<float>* residual_of(verbo::Session& s);

}  // namespace

// Loads a checkpoint with Model::load(dir, dtype), runs Session::eval_all on
// `toks` (n <= 64: one batch, so the residual holds every row) and copies out
// the final hidden rows, the reference's logits, and the head it built (its
// dtype: Q4 models keep a Q8 head, src/model.cpp:290).  meta = {dim, vocab,
// head dtype}; with x_out NULL only meta and eps are filled.
extern "C" int ref_model_tail(const char* dir, int dtype, const int* toks, int n, int threads, int* meta,
                              float* eps_out, float* x_out, float* logits_out, void* q_out, uint16_t* s_out,
                              float* norm_out) {
  using namespace verbo;
  try {
    auto m = Model::load(dir, static_cast<DType>(dtype));
    const Model::Impl& im = m->impl();
    meta[0] = im.cfg.dim;
    meta[1] = im.cfg.vocab;
    meta[2] = static_cast<int>(im.head.dt);
    *eps_out = im.cfg.eps;
    if (!x_out) return 0;
    if (n < 1 || n > 64) return -1;
    Session sess(m, 0, threads < 1 ? 1 : threads);
    const std::vector<float> all = sess.eval_all(std::vector<int>(toks, toks + n));
    std::memcpy(logits_out, all.data(), sizeof(float) * all.size());
    const std::vector<float>& x = *residual_of(sess);
    std::memcpy(x_out, x.data(), sizeof(float) * static_cast<std::size_t>(n) * im.cfg.dim);
    std::memcpy(q_out, im.head.q, im.head.qbytes());
    if (im.head.sbytes()) std::memcpy(s_out, im.head.s, im.head.sbytes());
    std::memcpy(norm_out, im.norm, sizeof(float) * im.cfg.dim);
    return 0;
  } catch (...) {
    return -1;
  }
}

extern "C" int ref_logits_tail(int dtype, int vocab, int dim, const void* q, const uint16_t* s, const float* norm,
                               float eps, const float* x, int n, long long ldx, float* out, long long ld, int8_t* xq,
                               float* xs, int threads) {
  using namespace verbo;
  if (dtype < 0 || dtype > 2 || vocab < 1 || dim < kBlk || dim % kBlk || n < 0 || ldx < dim || ld < vocab) return -1;
  if (n == 0) return 0;
  Tensor t;
  t.dt = static_cast<DType>(dtype);
  t.rows = vocab;
  t.cols = dim;
  t.q = q;
  t.s = s;
  const std::size_t nd = static_cast<std::size_t>(n) * dim;
  std::vector<float> xb(nd);
  std::vector<std::int8_t> aq(nd);
  std::vector<float> as(nd / kBlk);
  for (int i = 0; i < n; ++i) rmsnorm(x + static_cast<std::size_t>(i) * ldx, norm, xb.data() + i * dim, dim, eps);
  Act a;
  a.f = xb.data();
  a.n = n;
  a.ld = dim;
  if (t.dt != DType::F32) {
    for (int i = 0; i < n; ++i) quant_act(xb.data() + i * dim, dim, aq.data() + i * dim, as.data() + i * (dim / kBlk));
    a.q = aq.data();
    a.s = as.data();
    if (xq) std::memcpy(xq, aq.data(), nd);
    if (xs) std::memcpy(xs, as.data(), sizeof(float) * (nd / kBlk));
  }
  Pool pool(threads < 1 ? 1 : threads);
  matmul(t, a, out, static_cast<int>(ld), pool);
  return 0;
}

// Residual row of the last position of the last eval: Session::Impl::run
// splits an eval into batches of bmax rows and batch() leaves the rows of the
// last one in x, so the last position is row (n - 1) % bmax.
static const float* last_residual(verbo::Session& s, int n) {
  const int bmax = 64;  // Session::Impl::bmax (src/session.cpp:28)
  const int dim = s.model().impl().cfg.dim;
  return residual_of(s)->data() + static_cast<std::size_t>((n - 1) % bmax) * dim;
}

extern "C" int ref_decode(const char* dir, int dtype, const int* prompt, int n, const oracle_sampling* opts,
                          int max_tokens, int threads, int cap, int* ids_out, float* x_out, int* stopped) {
  using namespace verbo;
  try {
    if (!opts || opts->seed == 0 || n < 1 || cap < 1) return -1;
    auto m = Model::load(dir, static_cast<DType>(dtype));
    const int dim = m->impl().cfg.dim;
    const int nv = m->cfg().vocab;
    GenOpts go;
    go.max_tokens = max_tokens;
    go.smp.temp = opts->temp;
    go.smp.top_k = opts->top_k;
    go.smp.top_p = opts->top_p;
    go.smp.min_p = opts->min_p;
    go.smp.repeat = opts->repeat;
    go.smp.repeat_last = opts->repeat_last;
    go.smp.seed = opts->seed;
    const std::vector<int> pr(prompt, prompt + n);
    Stats st;
    {
      Session ses(m, 0, threads < 1 ? 1 : threads);
      st = generate(ses, pr, go, [](std::string_view) { return true; });
    }
    // the same loop, step by step, keeping each pick's hidden row
    Session ses(m, 0, threads < 1 ? 1 : threads);
    Sampler smp(go.smp);
    for (const int t : pr) smp.accept(t);
    const float* lg = ses.eval(pr);
    const float* xr = last_residual(ses, n);
    int picks = 0, gen = 0;
    *stopped = 0;
    while (gen < go.max_tokens) {
      const int id = smp.pick(lg, nv);
      if (picks >= cap) return -1;
      ids_out[picks] = id;
      std::memcpy(x_out + static_cast<std::size_t>(picks) * dim, xr, sizeof(float) * dim);
      ++picks;
      if (m->is_stop(id)) {
        *stopped = 1;
        break;
      }
      smp.accept(id);
      ++gen;
      if (ses.pos() >= ses.ctx() || gen >= go.max_tokens) break;
      lg = ses.eval(&id, 1);
      xr = last_residual(ses, 1);
    }
    if (gen != st.gen || *stopped != (st.stopped ? 1 : 0)) return -2;
    for (int j = 0; j < gen; ++j)
      if (ids_out[j] != st.toks[static_cast<std::size_t>(j)]) return -2;
    return picks;
  } catch (...) {
    return -1;
  }
}
