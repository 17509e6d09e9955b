// C ABI of the B200 sampler (include/verbo_cuda.h).  Mirrors the conventions
// of the reference's C ABI (src/capi.cpp): every entry point runs inside
// guard(), which turns exceptions into a -1 / NULL return and a thread-local
// message for verbo_cuda_last_error().  No compute happens here: the host
// validates arguments, plans the cluster split and launches the kernels of
// kernels.cu.  There is no CPU fallback.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>  // types only: NCCL is loaded at run time (dlopen), see Nccl below

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <deque>
#include <map>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <utility>
#include <vector>

#include "kernels.cuh"
#include "tail.cuh"
#include "verbo_cuda.h"

namespace {

thread_local std::string g_err;

template <typename F>
auto guard(F&& fn, decltype(fn()) fail) -> decltype(fn()) {
  try {
    g_err.clear();
    return fn();
  } catch (const std::exception& e) {
    g_err = e.what();
  } catch (...) {
    g_err = "verbo_cuda: unknown error";
  }
  return fail;
}

[[noreturn]] void fail(const std::string& m) { throw std::runtime_error("verbo_cuda: " + m); }

void cuda_ok(cudaError_t e, const char* what) {
  if (e != cudaSuccess) fail(std::string(what) + ": " + cudaGetErrorString(e));
}

int bitlen(unsigned long long x) {
  int b = 0;
  while (x) {
    ++b;
    x >>= 1;
  }
  return b;
}

// splitmix64, as src/sampler.cpp:11-16.
unsigned long long splitmix(unsigned long long& s) {
  unsigned long long z = (s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Sampler::reset seeding, src/sampler.cpp:26-31 (seed 0 = clock, like the reference).
void seed_state(unsigned long long seed, unsigned long long st[2]) {
  unsigned long long s = seed;
  if (s == 0) {
    const double ms =
        std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now().time_since_epoch()).count();
    s = static_cast<unsigned long long>(ms * 1000.0);
  }
  st[0] = splitmix(s);
  st[1] = splitmix(s);
}

// temp <= 0 (including -inf) is greedy, as in the reference; NaN and +inf
// would make every softmax weight NaN and are rejected.
vb::DevOpts make_opts(const verbo_sampling& s, int vocab, bool have_hist) {
  if (std::isnan(s.temp) || s.temp == INFINITY) fail("temp must not be NaN or +inf");
  vb::DevOpts o{};
  o.temp = s.temp;
  o.top_p = s.top_p;
  o.min_p = s.min_p;
  o.repeat = s.repeat;
  o.top_k = s.top_k;
  o.repeat_last = s.repeat_last;
  o.k = (s.top_k > 0 && s.top_k < vocab) ? s.top_k : vocab;
  o.greedy = s.temp <= 0.0f ? 1 : 0;
  o.penalize = (have_hist && s.repeat != 1.0f) ? 1 : 0;
  o.vocab = vocab;
  o.inv_temp = o.greedy ? 0.0 : 1.0 / static_cast<double>(s.temp);
  return o;
}

// Split `ncols` columns over a cluster of C CTAs (a power of two, at most 8)
// with slices of about 8192 columns or more; slices are multiples of 4.
void plan(int ncols, int& C, int& slice) {
  C = 1;
  while (C < 8 && static_cast<long long>(C) * 8192 < ncols) C <<= 1;
  slice = (ncols + C - 1) / C;
  slice = (slice + 3) & ~3;
}

vb::RowArgs row_args(const float* logits, int rows, int ncols, long long ld, int col_off, int vocab,
                     const int* hist, const long long* hist_off) {
  vb::RowArgs a{};
  a.logits = logits;
  a.ld = ld;
  a.rows = rows;
  a.ncols = ncols;
  a.col_off = col_off;
  a.hist = hist;
  a.hist_off = hist_off;
  a.idxbits = bitlen(static_cast<unsigned long long>(vocab - 1));
  if (a.idxbits < 1) a.idxbits = 1;
  a.fixbits = 63 - bitlen(static_cast<unsigned long long>(vocab));
  plan(ncols, a.cluster, a.slice);
  return a;
}

// Scratch of the split-row kernels, one buffer per (device, stream) so that
// calls on different streams never share it: per-slice counts and candidate
// keys, written by the streaming kernel and read by the merge kernel of the
// same call.  Allocated on first use, grown when a larger batch arrives.
struct Scratch {
  void* data = nullptr;
  size_t bytes = 0;
};
std::mutex g_scratch_mu;
std::map<std::pair<int, cudaStream_t>, Scratch> g_scratch;

void attach_split_scratch(vb::RowArgs& a, const vb::DevOpts& o, bool greedy, cudaStream_t s, bool windows = true) {
  int dev = 0;
  cuda_ok(cudaGetDevice(&dev), "cudaGetDevice");
  const int win_w = windows ? vb::split_window_width(o) : 0;
  const vb::SplitScratch l = vb::split_scratch_layout(a.rows, a.cluster, greedy, win_w);
  const size_t bytes = l.bytes;
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  Scratch& sc = g_scratch[{dev, s}];
  if (sc.bytes < bytes) {
    cuda_ok(cudaStreamSynchronize(s), "stream");  // the old buffer may still be in use
    const size_t n = std::max(bytes, 2 * sc.bytes);
    cudaFree(sc.data);
    sc.data = nullptr;
    sc.bytes = 0;
    cuda_ok(cudaMalloc(&sc.data, n), "cudaMalloc scratch");
    sc.bytes = n;
  }
  vb::split_scratch_attach(a, sc.data, l, win_w);
}

// Scratch of the streaming full-vocabulary path, one buffer per (device,
// stream): per-row state, the claim counter, the list of rows left to the
// staged kernel and the histogram slots (nucleus.cu).  Grown on demand.
std::map<std::pair<int, cudaStream_t>, Scratch> g_nuc_scratch;

void* nucleus_scratch(int rows, int ncols, cudaStream_t s) {
  int dev = 0;
  cuda_ok(cudaGetDevice(&dev), "cudaGetDevice");
  const size_t bytes = vb::nucleus_scratch_bytes(rows, ncols);
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  Scratch& sc = g_nuc_scratch[{dev, s}];
  if (sc.bytes < bytes) {
    cuda_ok(cudaStreamSynchronize(s), "stream");  // the old buffer may still be in use
    cudaFree(sc.data);
    sc.data = nullptr;
    sc.bytes = 0;
    cuda_ok(cudaMalloc(&sc.data, bytes), "cudaMalloc scratch");
    sc.bytes = bytes;
  }
  return sc.data;
}

// Slices of the split-row kernels: the fewest slices of <= kSplitSlice columns.
void plan_split(vb::RowArgs& a) {
  a.cluster = (a.ncols + vb::kSplitSlice - 1) / vb::kSplitSlice;
  a.slice = (a.ncols + a.cluster - 1) / a.cluster;
  a.slice = (a.slice + 3) & ~3;
}

// Picks the kernel for the options: the split-row kernels for greedy and
// 0 < top_k <= 256, the full-vocabulary kernel otherwise.  `ring` (batched
// streams) replaces the split kernels' scratch windows by the streams' own.
void dispatch_rows(vb::RowArgs& a, const vb::DevOpts& o, int vocab, cudaStream_t s, int* ring, int ring_w) {
  cudaError_t e;
  if (o.greedy || (o.k < vocab && o.k <= vb::kSplitMaxK)) {
    plan_split(a);
    attach_split_scratch(a, o, o.greedy != 0, s, ring == nullptr);
    if (ring) {
      a.win = ring;
      a.win_w = ring_w;
    }
    e = vb::launch_split(a, o, o.greedy ? vb::kSplitGreedy : vb::kSplitSample, s);
  } else {
    if (ring) {  // read through the CSR view; the ring is where the sampled ids go
      a.win = ring;
      a.win_w = ring_w;
    }
    if (vb::nucleus_eligible(o, vocab) && a.col_off == 0 && a.ncols == vocab)
      e = vb::launch_nucleus(a, o, nucleus_scratch(a.rows, a.ncols, s), s);
    else
      e = vb::launch_general(a, o, s);
  }
  cuda_ok(e, "kernel launch");
}

void check_hist(const int* hist, const long long* hist_off) {
  if ((hist == nullptr) != (hist_off == nullptr)) fail("hist and hist_off must both be given or both be NULL");
}

int sample_impl(const float* logits, int rows, int vocab, long long ld, const int* hist, const long long* hist_off,
                const verbo_sampling* opts, unsigned long long* rng, int* out_ids, verbo_row_stats* stats,
                cudaStream_t s) {
  if (!opts) fail("opts is NULL");
  if (rows < 0) fail("rows must be >= 0");
  if (rows == 0) return 0;
  if (!logits || !out_ids) fail("logits and out_ids must not be NULL");
  if (vocab < 1 || vocab > vb::kMaxVocab) fail("vocab must be in [1, " + std::to_string(vb::kMaxVocab) + "]");
  if (ld < vocab) fail("ld must be >= vocab");
  check_hist(hist, hist_off);
  const vb::DevOpts o = make_opts(*opts, vocab, hist != nullptr);
  if (!o.greedy && !rng) fail("rng state is required when temp > 0");
  vb::RowArgs a = row_args(logits, rows, vocab, ld, 0, vocab, hist, hist_off);
  a.rng = rng;
  a.out_ids = out_ids;
  a.stats = stats;
  dispatch_rows(a, o, vocab, s, nullptr, 0);
  return 0;
}

}  // namespace

struct verbo_cuda_sampler {
  verbo_sampling cfg{};
  int device = 0;
  cudaStream_t stream = nullptr;
  std::vector<int> hist;
  float* d_row = nullptr;
  int row_cap = 0;
  int* d_hist = nullptr;
  int hist_cap = 0;
  long long* d_off = nullptr;
  unsigned long long* d_rng = nullptr;
  int* d_out = nullptr;
  int* h_out = nullptr;  // pinned
};

namespace {

void sampler_release(verbo_cuda_sampler* s) {
  if (!s) return;
  cudaSetDevice(s->device);
  if (s->stream) cudaStreamSynchronize(s->stream);
  cudaFree(s->d_row);
  cudaFree(s->d_hist);
  cudaFree(s->d_off);
  cudaFree(s->d_rng);
  cudaFree(s->d_out);
  cudaFreeHost(s->h_out);
  if (s->stream) cudaStreamDestroy(s->stream);
}

void sampler_reset(verbo_cuda_sampler* s) {
  unsigned long long st[2];
  seed_state(s->cfg.seed, st);
  cuda_ok(cudaSetDevice(s->device), "cudaSetDevice");
  cuda_ok(cudaMemcpyAsync(s->d_rng, st, sizeof(st), cudaMemcpyHostToDevice, s->stream), "upload rng");
  cuda_ok(cudaStreamSynchronize(s->stream), "sync");
  s->hist.clear();
}

}  // namespace

extern "C" {

VERBO_CUDA_API const char* verbo_cuda_last_error(void) { return g_err.c_str(); }

VERBO_CUDA_API const char* verbo_cuda_version(void) { return "0.1.0-sm100a"; }

VERBO_CUDA_API verbo_sampling verbo_cuda_default_sampling(void) {
  verbo_sampling s;
  s.temp = 0.7f;
  s.top_k = 40;
  s.top_p = 0.9f;
  s.min_p = 0.0f;
  s.repeat = 1.0f;
  s.repeat_last = 64;
  s.seed = 0;
  return s;
}

VERBO_CUDA_API int verbo_cuda_rng_seed(unsigned long long seed, unsigned long long state[2]) {
  return guard(
      [&]() {
        if (!state) fail("state is NULL");
        seed_state(seed, state);
        return 0;
      },
      -1);
}

VERBO_CUDA_API double verbo_cuda_rng_unit(unsigned long long st[2]) {
  unsigned long long s1 = st[0];
  const unsigned long long s0 = st[1];
  const unsigned long long r = s0 + s1;
  st[0] = s0;
  s1 ^= s1 << 23;
  st[1] = s1 ^ s0 ^ (s1 >> 18) ^ (s0 >> 5);
  return static_cast<double>(r >> 11) * (1.0 / 9007199254740992.0);
}

VERBO_CUDA_API int verbo_cuda_sample(const float* logits, int rows, int vocab, long long ld, const int* hist,
                                     const long long* hist_off, const verbo_sampling* opts, unsigned long long* rng,
                                     int* out_ids, verbo_row_stats* stats, void* stream) {
  return guard(
      [&]() {
        return sample_impl(logits, rows, vocab, ld, hist, hist_off, opts, rng, out_ids, stats,
                           static_cast<cudaStream_t>(stream));
      },
      -1);
}

// Callers that cannot allocate device memory: see include/verbo_cuda.h.
// Same arguments and results as verbo_cuda_sample for greedy and
// 0 < top_k <= 256, without any cudaMalloc / cudaFree.
VERBO_CUDA_API int verbo_cuda_sample_noalloc(const float* logits, int rows, int vocab, long long ld, const int* hist,
                                             const long long* hist_off, const verbo_sampling* opts,
                                             unsigned long long* rng, int* out_ids, verbo_row_stats* stats,
                                             void* stream) {
  return guard(
      [&]() {
        if (!opts) fail("opts is NULL");
        if (rows < 0) fail("rows must be >= 0");
        if (rows == 0) return 0;
        if (!logits || !out_ids) fail("logits and out_ids must not be NULL");
        if (vocab < 1 || vocab > vb::kMaxVocab) fail("vocab must be in [1, " + std::to_string(vb::kMaxVocab) + "]");
        if (ld < vocab) fail("ld must be >= vocab");
        check_hist(hist, hist_off);
        const vb::DevOpts o = make_opts(*opts, vocab, hist != nullptr);
        if (!o.greedy && !rng) fail("rng state is required when temp > 0");
        if (!o.greedy && !(o.k < vocab && o.k <= vb::kSplitMaxK))
          fail("the allocation-free entry point needs temp <= 0 or 0 < top_k <= " +
               std::to_string(vb::kSplitMaxK) + " (and top_k < vocab)");
        vb::RowArgs a = row_args(logits, rows, vocab, ld, 0, vocab, hist, hist_off);
        a.rng = rng;
        a.out_ids = out_ids;
        a.stats = stats;
        plan_split(a);
        bool too_big = false;
        cuda_ok(vb::launch_split_noalloc(a, o, o.greedy ? vb::kSplitGreedy : vb::kSplitSample,
                                         static_cast<cudaStream_t>(stream), &too_big),
                "kernel launch");
        if (too_big) {
          // the largest row count the same layout fits (binary search, so the
          // quoted limit is exactly the one the check enforces)
          const int win_w = vb::split_window_width(o);
          long long lo = 0, hi = rows;  // lo fits, hi does not
          while (hi - lo > 1) {
            const long long mid = lo + (hi - lo) / 2;
            if (vb::split_scratch_layout(mid, a.cluster, o.greedy != 0, win_w).bytes <= vb::kNoAllocScratchBytes)
              lo = mid;
            else
              hi = mid;
          }
          fail("rows x vocab exceed the fixed scratch of " + std::to_string(vb::kNoAllocScratchBytes >> 20) +
               " MiB: at most " + std::to_string(lo) + " rows at vocab " + std::to_string(vocab) + " per call");
        }
        return 0;
      },
      -1);
}

VERBO_CUDA_API int verbo_cuda_shard_topk(const float* logits, int rows, int shard_cols, long long ld, int col_offset,
                                         int vocab, const int* hist, const long long* hist_off,
                                         const verbo_sampling* opts, int k, float* cand_val, int* cand_id,
                                         void* stream) {
  return guard(
      [&]() {
        if (!opts) fail("opts is NULL");
        if (rows < 0) fail("rows must be >= 0");
        if (rows == 0) return 0;
        if (!logits || !cand_val || !cand_id) fail("logits, cand_val and cand_id must not be NULL");
        if (k < 1 || k > vb::kSplitMaxK) fail("k must be in [1, " + std::to_string(vb::kSplitMaxK) + "]");
        if (vocab < 1 || vocab > vb::kMaxVocab) fail("vocab must be in [1, " + std::to_string(vb::kMaxVocab) + "]");
        if (shard_cols < 1 || col_offset < 0 || static_cast<long long>(col_offset) + shard_cols > vocab)
          fail("shard [col_offset, col_offset + shard_cols) must lie in [0, vocab)");
        if (ld < shard_cols) fail("ld must be >= shard_cols");
        check_hist(hist, hist_off);
        vb::DevOpts o = make_opts(*opts, vocab, hist != nullptr);
        vb::RowArgs a = row_args(logits, rows, shard_cols, ld, col_offset, vocab, hist, hist_off);
        a.cand_val = cand_val;
        a.cand_id = cand_id;
        a.cand_k = k;
        plan_split(a);
        attach_split_scratch(a, o, false, static_cast<cudaStream_t>(stream));
        cuda_ok(vb::launch_split(a, o, vb::kSplitEmit, static_cast<cudaStream_t>(stream)), "kernel launch");
        return 0;
      },
      -1);
}

VERBO_CUDA_API int verbo_cuda_merge_sample(const float* cand_val, const int* cand_id, int rows, int nshards, int k,
                                           int vocab, const verbo_sampling* opts, unsigned long long* rng,
                                           int* out_ids, verbo_row_stats* stats, void* stream) {
  return guard(
      [&]() {
        if (!opts) fail("opts is NULL");
        if (rows < 0) fail("rows must be >= 0");
        if (rows == 0) return 0;
        if (!cand_val || !cand_id || !out_ids) fail("cand_val, cand_id and out_ids must not be NULL");
        if (nshards < 1 || k < 1 || static_cast<long long>(nshards) * k > vb::kMaxMerge)
          fail("nshards * k must be in [1, " + std::to_string(vb::kMaxMerge) + "]");
        if (k > vb::kSplitMaxK) fail("k must be <= " + std::to_string(vb::kSplitMaxK));
        if (vocab < 1) fail("vocab must be >= 1");
        vb::DevOpts o = make_opts(*opts, vocab, false);
        if (!o.greedy && !(opts->top_k > 0 && opts->top_k <= k && opts->top_k < vocab))
          fail("vocab-sharded sampling needs temp <= 0 or 0 < top_k <= k");
        if (!o.greedy && !rng) fail("rng state is required when temp > 0");
        vb::MergeArgs a{};
        a.cand_val = cand_val;
        a.cand_id = cand_id;
        a.rows = rows;
        a.nshards = nshards;
        a.k = k;
        a.rng = rng;
        a.out_ids = out_ids;
        a.stats = stats;
        cuda_ok(vb::launch_merge(a, o, static_cast<cudaStream_t>(stream)), "kernel launch");
        return 0;
      },
      -1);
}

VERBO_CUDA_API int verbo_cuda_check(void* stream) {
  return guard(
      [&]() {
        unsigned st = 0;
        cuda_ok(vb::read_status(&st, true, static_cast<cudaStream_t>(stream)), "stream");
        if (st & vb::kErrLoadTimeout) fail("a row load did not complete within the wait limit");
        if (st & vb::kErrSelect) fail("a selection found no element (inconsistent input)");
        unsigned tst = 0;
        cuda_ok(vb::tail_read_status(&tst, true), "tail status");
        if (tst & vb::kErrTailWait) fail("a logits-tail pipeline wait did not complete within the wait limit");
        if (tst) fail("tail device status " + std::to_string(tst));
        if (st) fail("device status " + std::to_string(st));
        return 0;
      },
      -1);
}

VERBO_CUDA_API int verbo_cuda_full_vocab_fallbacks(void* stream) {
  return guard(
      [&]() {
        const cudaStream_t s = static_cast<cudaStream_t>(stream);
        int dev = 0;
        cuda_ok(cudaGetDevice(&dev), "cudaGetDevice");
        void* data = nullptr;
        {
          std::lock_guard<std::mutex> lk(g_scratch_mu);
          const auto it = g_nuc_scratch.find({dev, s});
          if (it != g_nuc_scratch.end()) data = it->second.data;
        }
        if (!data) return 0;
        unsigned n = 0;
        cuda_ok(vb::nucleus_fallbacks(data, s, &n), "read fallback count");
        return static_cast<int>(n);
      },
      -1);
}

VERBO_CUDA_API verbo_cuda_sampler* verbo_cuda_sampler_new(const verbo_sampling* cfg, int device) {
  return guard(
      [&]() -> verbo_cuda_sampler* {
        auto* s = new verbo_cuda_sampler();
        try {
          s->cfg = cfg ? *cfg : verbo_cuda_default_sampling();
          if (std::isnan(s->cfg.temp) || s->cfg.temp == INFINITY) fail("temp must not be NaN or +inf");
          s->device = device;
          cuda_ok(cudaSetDevice(device), "cudaSetDevice");
          cuda_ok(cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking), "cudaStreamCreate");
          cuda_ok(cudaMalloc(&s->d_rng, 2 * sizeof(unsigned long long)), "cudaMalloc");
          cuda_ok(cudaMalloc(&s->d_out, sizeof(int)), "cudaMalloc");
          cuda_ok(cudaMalloc(&s->d_off, 2 * sizeof(long long)), "cudaMalloc");
          cuda_ok(cudaMallocHost(&s->h_out, sizeof(int)), "cudaMallocHost");
          sampler_reset(s);
        } catch (...) {
          sampler_release(s);
          delete s;
          throw;
        }
        return s;
      },
      nullptr);
}

VERBO_CUDA_API void verbo_cuda_sampler_free(verbo_cuda_sampler* s) {
  if (!s) return;
  sampler_release(s);
  delete s;
}

VERBO_CUDA_API int verbo_cuda_sampler_pick(verbo_cuda_sampler* s, const float* logits, int n) {
  return guard(
      [&]() {
        if (!s || !logits) fail("sampler and logits must not be NULL");
        if (n < 1) fail("n must be >= 1");
        cuda_ok(cudaSetDevice(s->device), "cudaSetDevice");
        cudaPointerAttributes pa{};
        cuda_ok(cudaPointerGetAttributes(&pa, logits), "cudaPointerGetAttributes");
        const float* row = logits;
        if (pa.type != cudaMemoryTypeDevice && pa.type != cudaMemoryTypeManaged) {
          if (n > s->row_cap) {
            cudaFree(s->d_row);
            s->d_row = nullptr;
            s->row_cap = 0;
            cuda_ok(cudaMalloc(&s->d_row, static_cast<size_t>(n) * sizeof(float)), "cudaMalloc");
            s->row_cap = n;
          }
          cuda_ok(cudaMemcpyAsync(s->d_row, logits, static_cast<size_t>(n) * sizeof(float), cudaMemcpyHostToDevice,
                                  s->stream),
                  "upload logits");
          row = s->d_row;
        }
        // penalty window: the last repeat_last accepted ids (src/sampler.cpp:53-57)
        const int* dh = nullptr;
        const long long* doff = nullptr;
        if (s->cfg.repeat != 1.0f && !s->hist.empty()) {
          const size_t len = s->hist.size();
          const size_t from =
              (s->cfg.repeat_last > 0 && len > static_cast<size_t>(s->cfg.repeat_last)) ? len - s->cfg.repeat_last : 0;
          const int w = static_cast<int>(len - from);
          if (w > s->hist_cap) {
            cudaFree(s->d_hist);
            s->d_hist = nullptr;
            s->hist_cap = 0;
            cuda_ok(cudaMalloc(&s->d_hist, static_cast<size_t>(w) * sizeof(int)), "cudaMalloc");
            s->hist_cap = w;
          }
          const long long off[2] = {0, w};
          cuda_ok(cudaMemcpyAsync(s->d_hist, s->hist.data() + from, static_cast<size_t>(w) * sizeof(int),
                                  cudaMemcpyHostToDevice, s->stream),
                  "upload history");
          cuda_ok(cudaMemcpyAsync(s->d_off, off, sizeof(off), cudaMemcpyHostToDevice, s->stream), "upload history");
          cuda_ok(cudaStreamSynchronize(s->stream), "sync");
          dh = s->d_hist;
          doff = s->d_off;
        }
        sample_impl(row, 1, n, n, dh, doff, &s->cfg, s->d_rng, s->d_out, nullptr, s->stream);
        cuda_ok(cudaMemcpyAsync(s->h_out, s->d_out, sizeof(int), cudaMemcpyDeviceToHost, s->stream), "read id");
        cuda_ok(cudaStreamSynchronize(s->stream), "sync");
        return *s->h_out;
      },
      -1);
}

VERBO_CUDA_API int verbo_cuda_sampler_accept(verbo_cuda_sampler* s, int tok) {
  return guard(
      [&]() {
        if (!s) fail("sampler is NULL");
        // Sampler::accept (src/sampler.cpp:43-48)
        s->hist.push_back(tok);
        if (s->cfg.repeat_last > 0 && s->hist.size() > static_cast<size_t>(s->cfg.repeat_last) * 4)
          s->hist.erase(s->hist.begin(), s->hist.end() - s->cfg.repeat_last);
        return 0;
      },
      -1);
}

VERBO_CUDA_API int verbo_cuda_sampler_reset(verbo_cuda_sampler* s) {
  return guard(
      [&]() {
        if (!s) fail("sampler is NULL");
        sampler_reset(s);
        return 0;
      },
      -1);
}

VERBO_CUDA_API int verbo_cuda_sampler_cfg(const verbo_cuda_sampler* s, verbo_sampling* out) {
  return guard(
      [&]() {
        if (!s || !out) fail("sampler and out must not be NULL");
        *out = s->cfg;
        return 0;
      },
      -1);
}

// ------------------------------------------------------- batched streams --
// B generation streams whose RNG states and penalty windows stay on the device
// (the batched form of the loop in verbo::generate, src/sampler.cpp:111-181).
// Each stream's window is a ring of its last repeat_last accepted ids; the
// kernel that finishes a row appends the id it sampled, so a step is the
// sampling launch and nothing else.

}  // extern "C"

struct verbo_cuda_batch {
  verbo_sampling cfg{};
  int device = 0;
  int streams = 0;
  bool pen = false;   // repeat != 1: the streams keep windows
  int ring_len = 0;   // repeat_last
  int win_w = 0;      // ring row stride (ring_len rounded up to 4, the tail -1)
  int* d_win = nullptr;
  long long* d_pos = nullptr;
  long long* d_off = nullptr;  // CSR view of the rings for the full-vocabulary kernel
  unsigned long long* d_rng = nullptr;
  int* d_stage = nullptr;
  long long stage_cap = 0;
  // staging of verbo_cuda_batch_decode: host hidden rows in, the step's
  // logits rows, host ids / stats out
  float* d_hidden = nullptr;
  long long hidden_cap = 0;  // floats
  float* d_logits = nullptr;
  long long logits_cap = 0;  // floats
  int* d_ids = nullptr;
  verbo_row_stats* d_stats = nullptr;
};

namespace {

void batch_release(verbo_cuda_batch* b) {
  if (!b) return;
  cudaSetDevice(b->device);
  cudaDeviceSynchronize();
  cudaFree(b->d_win);
  cudaFree(b->d_pos);
  cudaFree(b->d_off);
  cudaFree(b->d_rng);
  cudaFree(b->d_stage);
  cudaFree(b->d_hidden);
  cudaFree(b->d_logits);
  cudaFree(b->d_ids);
  cudaFree(b->d_stats);
}

void batch_run(verbo_cuda_batch* b, const float* logits, int vocab, long long ld, int* out_ids,
               verbo_row_stats* stats, cudaStream_t s);

void batch_check_stream(const verbo_cuda_batch* b, int i) {
  if (!b) fail("batch is NULL");
  if (i < 0 || i >= b->streams) fail("stream index out of range");
}

// Sampler::reset of one stream (src/sampler.cpp:26-31): seed 0 takes the clock.
void batch_reset_one(verbo_cuda_batch* b, int i, unsigned long long seed, cudaStream_t s) {
  unsigned long long st[2];
  seed_state(seed, st);
  cuda_ok(cudaMemcpyAsync(b->d_rng + 2ll * i, st, sizeof(st), cudaMemcpyHostToDevice, s), "upload rng");
  if (b->pen) {
    cuda_ok(cudaMemsetAsync(b->d_win + static_cast<long long>(i) * b->win_w, 0xff, b->win_w * sizeof(int), s),
            "clear window");
    cuda_ok(cudaMemsetAsync(b->d_pos + i, 0, sizeof(long long), s), "clear count");
  }
}

}  // namespace

extern "C" {

VERBO_CUDA_API verbo_cuda_batch* verbo_cuda_batch_new(const verbo_sampling* cfg, int streams, int device) {
  return guard(
      [&]() -> verbo_cuda_batch* {
        if (!cfg) fail("cfg is NULL");
        if (streams < 1 || streams > (1 << 24)) fail("streams must be in [1, 16777216]");
        if (std::isnan(cfg->temp) || cfg->temp == INFINITY) fail("temp must not be NaN or +inf");
        const bool pen = cfg->repeat != 1.0f;
        if (pen && (cfg->repeat_last < 1 || cfg->repeat_last > vb::kWinMax))
          fail("batched streams with a repetition penalty need 1 <= repeat_last <= " + std::to_string(vb::kWinMax));
        int n = 0;
        cuda_ok(cudaGetDeviceCount(&n), "cudaGetDeviceCount");
        if (device < 0 || device >= n) fail("no CUDA device " + std::to_string(device));
        cuda_ok(cudaSetDevice(device), "cudaSetDevice");
        auto* b = new verbo_cuda_batch();
        b->cfg = *cfg;
        b->device = device;
        b->streams = streams;
        b->pen = pen;
        try {
          cuda_ok(cudaMalloc(&b->d_rng, 16ull * streams), "cudaMalloc rng");
          if (pen) {
            b->ring_len = cfg->repeat_last;
            b->win_w = (cfg->repeat_last + 3) & ~3;
            cuda_ok(cudaMalloc(&b->d_win, 4ull * b->win_w * streams), "cudaMalloc windows");
            cuda_ok(cudaMalloc(&b->d_pos, 8ull * streams), "cudaMalloc counts");
            cuda_ok(cudaMalloc(&b->d_off, 8ull * (streams + 1)), "cudaMalloc offsets");
            std::vector<long long> off(static_cast<size_t>(streams) + 1);
            for (int i = 0; i <= streams; ++i) off[i] = static_cast<long long>(i) * b->win_w;
            cuda_ok(cudaMemcpy(b->d_off, off.data(), off.size() * 8, cudaMemcpyHostToDevice), "upload offsets");
            cuda_ok(cudaMemset(b->d_win, 0xff, 4ull * b->win_w * streams), "clear windows");
            cuda_ok(cudaMemset(b->d_pos, 0, 8ull * streams), "clear counts");
          }
          // every stream starts as verbo::Sampler(cfg) does: seeded from cfg.seed
          unsigned long long st[2];
          seed_state(cfg->seed, st);
          std::vector<unsigned long long> all(2ull * streams);
          for (int i = 0; i < streams; ++i) {
            all[2ull * i] = st[0];
            all[2ull * i + 1] = st[1];
          }
          cuda_ok(cudaMemcpy(b->d_rng, all.data(), all.size() * 8, cudaMemcpyHostToDevice), "upload rng");
        } catch (...) {
          batch_release(b);
          delete b;
          throw;
        }
        return b;
      },
      nullptr);
}

VERBO_CUDA_API void verbo_cuda_batch_free(verbo_cuda_batch* b) {
  batch_release(b);
  delete b;
}

VERBO_CUDA_API int verbo_cuda_batch_reset(verbo_cuda_batch* b, int stream, unsigned long long seed, void* cuda_stream) {
  return guard(
      [&]() {
        batch_check_stream(b, stream);
        cuda_ok(cudaSetDevice(b->device), "cudaSetDevice");
        batch_reset_one(b, stream, seed, static_cast<cudaStream_t>(cuda_stream));
        return 0;
      },
      -1);
}

VERBO_CUDA_API int verbo_cuda_batch_accept(verbo_cuda_batch* b, int stream, const int* ids, int n, void* cuda_stream) {
  return guard(
      [&]() {
        batch_check_stream(b, stream);
        if (n < 0) fail("n must be >= 0");
        if (n > 0 && !ids) fail("ids is NULL");
        if (!b->pen || n == 0) return 0;  // without a penalty nothing reads the history
        cuda_ok(cudaSetDevice(b->device), "cudaSetDevice");
        const cudaStream_t s = static_cast<cudaStream_t>(cuda_stream);
        // only the last ring_len ids can reach the window
        const int skip = n > b->ring_len ? n - b->ring_len : 0;
        const int m = n - skip;
        if (b->stage_cap < m) {
          cuda_ok(cudaStreamSynchronize(s), "stream");  // the old staging may still be read
          cudaFree(b->d_stage);
          b->d_stage = nullptr;
          b->stage_cap = 0;
          cuda_ok(cudaMalloc(&b->d_stage, 4ull * b->ring_len), "cudaMalloc staging");
          b->stage_cap = b->ring_len;
        }
        cuda_ok(cudaMemcpyAsync(b->d_stage, ids + skip, 4ull * m, cudaMemcpyHostToDevice, s), "upload ids");
        // the skipped ids still count: they advance the stream's ring position
        cuda_ok(vb::launch_ring_accept(b->d_win, b->win_w, b->ring_len, b->d_pos, stream, b->d_stage, m, skip, s),
                "kernel launch");
        return 0;
      },
      -1);
}

VERBO_CUDA_API int verbo_cuda_batch_step(verbo_cuda_batch* b, const float* logits, int vocab, long long ld,
                                         int* out_ids, verbo_row_stats* stats, void* cuda_stream) {
  return guard(
      [&]() {
        if (!b) fail("batch is NULL");
        if (!logits || !out_ids) fail("logits and out_ids must not be NULL");
        if (vocab < 1 || vocab > vb::kMaxVocab) fail("vocab must be in [1, " + std::to_string(vb::kMaxVocab) + "]");
        if (ld < vocab) fail("ld must be >= vocab");
        cuda_ok(cudaSetDevice(b->device), "cudaSetDevice");
        batch_run(b, logits, vocab, ld, out_ids, stats, static_cast<cudaStream_t>(cuda_stream));
        return 0;
      },
      -1);
}

}  // extern "C"

namespace {

// One pick + accept per stream from B device rows (arguments checked).
void batch_run(verbo_cuda_batch* b, const float* logits, int vocab, long long ld, int* out_ids,
               verbo_row_stats* stats, cudaStream_t s) {
        vb::DevOpts o = make_opts(b->cfg, vocab, b->pen);
        // the rings hold exactly the windows: the CSR view (full-vocabulary
        // kernel) reads each whole ring row, -1 slots marking nothing
        if (b->pen) o.repeat_last = b->win_w;
        vb::RowArgs a = row_args(logits, b->streams, vocab, ld, 0, vocab, b->pen ? b->d_win : nullptr,
                                 b->pen ? b->d_off : nullptr);
        a.rng = b->d_rng;
        a.out_ids = out_ids;
        a.stats = stats;
        if (b->pen) {
          a.ring_pos = b->d_pos;
          a.ring_len = b->ring_len;
        }
        dispatch_rows(a, o, vocab, s, b->pen ? b->d_win : nullptr, b->win_w);
}

}  // namespace

// ---------------------------------------------------------------------------
// Logits producer tail: the head (weights, zero-padded scales, norm weight)
// resident on one device, and one scratch buffer per CUDA stream for the
// quantised activations of a call.
struct verbo_cuda_tail {
  vb::TailHead h{};
  int device = 0;
  void* d_q = nullptr;  // the tile-major head
  float* d_norm = nullptr;
  std::mutex mu;
  std::map<cudaStream_t, Scratch> scratch;
};

namespace {

void tail_run(verbo_cuda_tail* t, const float* x, int n, long long ldx, float* logits, long long ld, cudaStream_t s);

void tail_release(verbo_cuda_tail* t) {
  if (!t) return;
  cudaSetDevice(t->device);
  for (auto& kv : t->scratch) cudaFree(kv.second.data);
  cudaFree(t->d_q);
  cudaFree(t->d_norm);
  delete t;
}

}  // namespace

extern "C" {

VERBO_CUDA_API verbo_cuda_tail* verbo_cuda_tail_new(int dtype, int vocab, int dim, const void* q,
                                                    const unsigned short* s, const float* norm, float eps,
                                                    int device) {
  return guard(
      [&]() -> verbo_cuda_tail* {
        if (dtype < vb::kTailF32 || dtype > vb::kTailQ4) fail("dtype must be 0 (F32), 1 (Q8) or 2 (Q4)");
        if (vocab < 1 || vocab > vb::kTailMaxVocab)
          fail("vocab must be in [1, " + std::to_string(vb::kTailMaxVocab) + "]");
        if (dim < vb::kTailBlk || dim > vb::kTailMaxDim || dim % vb::kTailBlk)
          fail("dim must be a multiple of 32 in [32, " + std::to_string(vb::kTailMaxDim) + "]");
        if (!q || !norm) fail("q and norm must not be NULL");
        if (dtype != vb::kTailF32 && !s) fail("quantised heads need their scales s");
        int ndev = 0;
        cuda_ok(cudaGetDeviceCount(&ndev), "cudaGetDeviceCount");
        if (device < 0 || device >= ndev) fail("no CUDA device " + std::to_string(device));
        cuda_ok(cudaSetDevice(device), "cudaSetDevice");
        auto* t = new verbo_cuda_tail();
        t->device = device;
        vb::TailHead& h = t->h;
        h.dtype = dtype;
        h.vocab = vocab;
        h.dim = dim;
        h.dimp = (dim + vb::kTailChunk - 1) / vb::kTailChunk * vb::kTailChunk;
        h.nkc = h.dimp / vb::kTailChunk;
        h.ntile = (vocab + vb::kTailRows - 1) / vb::kTailRows;
        h.eps = eps;
        try {
          {
            // once per head: the tile-major, pre-swizzled form the kernels stream
            const size_t bytes = vb::tail_tiles_bytes(dtype, vocab, dim);
            std::vector<unsigned char> packed(bytes);
            vb::tail_pack_tiles(dtype, vocab, dim, q, s, packed.data());
            cuda_ok(cudaMalloc(&t->d_q, bytes), "cudaMalloc head");
            cuda_ok(cudaMemcpy(t->d_q, packed.data(), bytes, cudaMemcpyHostToDevice), "upload head");
            h.tiles = static_cast<const unsigned char*>(t->d_q);
          }
          cuda_ok(cudaMalloc(&t->d_norm, sizeof(float) * dim), "cudaMalloc norm");
          cuda_ok(cudaMemcpy(t->d_norm, norm, sizeof(float) * dim, cudaMemcpyHostToDevice), "upload norm");
        } catch (...) {
          tail_release(t);
          throw;
        }
        h.norm = t->d_norm;
        return t;
      },
      static_cast<verbo_cuda_tail*>(nullptr));
}

VERBO_CUDA_API void verbo_cuda_tail_free(verbo_cuda_tail* t) { tail_release(t); }

VERBO_CUDA_API int verbo_cuda_tail_logits(verbo_cuda_tail* t, const float* x, int n, long long ldx, float* logits,
                                          long long ld, void* stream) {
  return guard(
      [&]() {
        if (!t) fail("tail is NULL");
        if (n < 0) fail("n must be >= 0");
        if (n == 0) return 0;
        if (!x || !logits) fail("x and logits must not be NULL");
        if (ldx < t->h.dim) fail("ldx must be >= dim");
        if (ld < t->h.vocab) fail("ld must be >= vocab");
        cuda_ok(cudaSetDevice(t->device), "cudaSetDevice");
        tail_run(t, x, n, ldx, logits, ld, static_cast<cudaStream_t>(stream));
        return 0;
      },
      -1);
}

}  // extern "C"

namespace {

// n device rows of hidden state -> n device rows of logits (arguments checked).
void tail_run(verbo_cuda_tail* t, const float* x, int n, long long ldx, float* logits, long long ld, cudaStream_t s) {
        vb::TailArgs a{};
        a.x = x;
        a.ldx = ldx;
        a.n = n;
        a.logits = logits;
        a.ld = ld;
        const size_t bytes = vb::tail_scratch_bytes(t->h, n);
        std::lock_guard<std::mutex> lk(t->mu);
        Scratch& sc = t->scratch[s];
        if (sc.bytes < bytes) {
          cuda_ok(cudaStreamSynchronize(s), "stream");  // the old buffer may still be in use
          const size_t nb = std::max(bytes, 2 * sc.bytes);
          cudaFree(sc.data);
          sc.data = nullptr;
          sc.bytes = 0;
          cuda_ok(cudaMalloc(&sc.data, nb), "cudaMalloc tail scratch");
          sc.bytes = nb;
        }
        vb::tail_scratch_attach(t->h, n, sc.data, a);
        cuda_ok(vb::launch_tail(t->h, a, s), "kernel launch");
}

// Grows a device staging buffer of `count` elements (the old one may still be
// read by work queued on `s`).
template <typename T>
void grow(T*& buf, long long& cap, long long count, cudaStream_t s, const char* what) {
  if (cap >= count) return;
  cuda_ok(cudaStreamSynchronize(s), "stream");
  cudaFree(buf);
  buf = nullptr;
  cap = 0;
  cuda_ok(cudaMalloc(&buf, sizeof(T) * static_cast<size_t>(count)), what);
  cap = count;
}

bool on_device(const void* p) {
  cudaPointerAttributes pa{};
  cuda_ok(cudaPointerGetAttributes(&pa, p), "cudaPointerGetAttributes");
  return pa.type == cudaMemoryTypeDevice || pa.type == cudaMemoryTypeManaged;
}

}  // namespace

extern "C" {

VERBO_CUDA_API int verbo_cuda_batch_decode(verbo_cuda_batch* b, verbo_cuda_tail* t, const float* hidden,
                                           long long ldx, int* out_ids, verbo_row_stats* stats, void* cuda_stream) {
  return guard(
      [&]() {
        if (!b || !t) fail("batch and tail must not be NULL");
        if (!hidden || !out_ids) fail("hidden and out_ids must not be NULL");
        if (t->device != b->device) fail("the tail and the batch must live on the same device");
        const int B = b->streams, dim = t->h.dim, vocab = t->h.vocab;
        if (vocab > vb::kMaxVocab) fail("vocab must be <= " + std::to_string(vb::kMaxVocab));
        if (ldx < dim) fail("ldx must be >= dim");
        cuda_ok(cudaSetDevice(b->device), "cudaSetDevice");
        const cudaStream_t s = static_cast<cudaStream_t>(cuda_stream);
        // the hidden rows: read in place on the device, else one 2-D upload
        const float* x = hidden;
        long long lx = ldx;
        if (!on_device(hidden)) {
          grow(b->d_hidden, b->hidden_cap, static_cast<long long>(B) * dim, s, "cudaMalloc hidden rows");
          cuda_ok(cudaMemcpy2DAsync(b->d_hidden, sizeof(float) * dim, hidden, sizeof(float) * ldx, sizeof(float) * dim,
                                    B, cudaMemcpyHostToDevice, s),
                  "upload hidden rows");
          x = b->d_hidden;
          lx = dim;
        }
        grow(b->d_logits, b->logits_cap, static_cast<long long>(B) * vocab, s, "cudaMalloc logits rows");
        tail_run(t, x, B, lx, b->d_logits, vocab, s);
        // the logits stay on the device: the pick reads them where the tail wrote them
        const bool ids_host = !on_device(out_ids);
        const bool stats_host = stats && !on_device(stats);
        if (ids_host && !b->d_ids) cuda_ok(cudaMalloc(&b->d_ids, sizeof(int) * B), "cudaMalloc ids");
        if (stats_host && !b->d_stats) cuda_ok(cudaMalloc(&b->d_stats, sizeof(verbo_row_stats) * B), "cudaMalloc stats");
        batch_run(b, b->d_logits, vocab, vocab, ids_host ? b->d_ids : out_ids, stats_host ? b->d_stats : stats, s);
        if (ids_host)
          cuda_ok(cudaMemcpyAsync(out_ids, b->d_ids, sizeof(int) * B, cudaMemcpyDeviceToHost, s), "download ids");
        if (stats_host)
          cuda_ok(cudaMemcpyAsync(stats, b->d_stats, sizeof(verbo_row_stats) * B, cudaMemcpyDeviceToHost, s),
                  "download stats");
        if (ids_host || stats_host) cuda_ok(cudaStreamSynchronize(s), "stream");
        return 0;
      },
      -1);
}

}  // extern "C"

// ================================================ vocab-sharded collective ==
// The library's own communicator for the vocab-sharded pick: NCCL, loaded at
// run time (libnccl.so.2, whichever the process resolves, so a process that
// already has NCCL loaded shares that copy), so that the library has no link
// dependency on it and callers without NCCL can use everything else.
namespace {

struct Nccl {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*get_error_string)(ncclResult_t) = nullptr;
  std::string err;
};

const Nccl& nccl() {
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    if (!h) {
      const char* e = dlerror();
      n.err = e ? e : "libnccl.so.2 not found";
      return;
    }
    auto sym = [&](const char* name) {
      void* p = dlsym(h, name);
      if (!p && n.err.empty()) n.err = std::string("missing ") + name;
      return p;
    };
    n.get_unique_id = reinterpret_cast<decltype(n.get_unique_id)>(sym("ncclGetUniqueId"));
    n.comm_init_rank = reinterpret_cast<decltype(n.comm_init_rank)>(sym("ncclCommInitRank"));
    n.comm_destroy = reinterpret_cast<decltype(n.comm_destroy)>(sym("ncclCommDestroy"));
    n.comm_abort = reinterpret_cast<decltype(n.comm_abort)>(sym("ncclCommAbort"));
    n.comm_get_async_error = reinterpret_cast<decltype(n.comm_get_async_error)>(sym("ncclCommGetAsyncError"));
    n.all_gather = reinterpret_cast<decltype(n.all_gather)>(sym("ncclAllGather"));
    n.get_error_string = reinterpret_cast<decltype(n.get_error_string)>(sym("ncclGetErrorString"));
  });
  if (!n.err.empty()) fail("NCCL is not available: " + n.err);
  return n;
}

void nccl_ok(ncclResult_t r, const char* what) {
  if (r != ncclSuccess) fail(std::string(what) + ": " + nccl().get_error_string(r));
}

}  // namespace

struct verbo_cuda_comm {
  ncclComm_t comm = nullptr;
  int nranks = 0, rank = 0, device = 0;
  uint2* local = nullptr;     // this rank's candidates [rows][k], packed
  uint2* gathered = nullptr;  // every rank's [nranks][rows][k]
  size_t cap = 0;             // rows * k the buffers hold
  cudaEvent_t mark_shard = nullptr, mark_gather = nullptr;  // recorded by the next call only
  std::mutex mu;
};

extern "C" {

VERBO_CUDA_API int verbo_cuda_comm_unique_id(unsigned char id[VERBO_CUDA_UNIQUE_ID_BYTES]) {
  return guard(
      [&]() {
        static_assert(sizeof(ncclUniqueId) == VERBO_CUDA_UNIQUE_ID_BYTES, "NCCL unique id size");
        if (!id) fail("id is NULL");
        ncclUniqueId u;
        nccl_ok(nccl().get_unique_id(&u), "ncclGetUniqueId");
        std::memcpy(id, &u, sizeof(u));
        return 0;
      },
      -1);
}

VERBO_CUDA_API verbo_cuda_comm* verbo_cuda_comm_new(const unsigned char id[VERBO_CUDA_UNIQUE_ID_BYTES], int nranks,
                                                    int rank, int device) {
  return guard(
      [&]() -> verbo_cuda_comm* {
        if (!id) fail("id is NULL");
        if (nranks < 1 || rank < 0 || rank >= nranks) fail("rank must be in [0, nranks)");
        cuda_ok(cudaSetDevice(device), "cudaSetDevice");
        ncclUniqueId u;
        std::memcpy(&u, id, sizeof(u));
        auto* c = new verbo_cuda_comm;
        c->nranks = nranks;
        c->rank = rank;
        c->device = device;
        const ncclResult_t r = nccl().comm_init_rank(&c->comm, nranks, u, rank);
        if (r != ncclSuccess) {
          delete c;
          nccl_ok(r, "ncclCommInitRank");
        }
        return c;
      },
      static_cast<verbo_cuda_comm*>(nullptr));
}

VERBO_CUDA_API void verbo_cuda_comm_free(verbo_cuda_comm* c) {
  if (!c) return;
  cudaSetDevice(c->device);
  cudaDeviceSynchronize();
  if (c->comm) nccl().comm_destroy(c->comm);
  cudaFree(c->local);
  cudaFree(c->gathered);
  delete c;
}

VERBO_CUDA_API int verbo_cuda_comm_wait(verbo_cuda_comm* c, void* stream, int timeout_ms) {
  return guard(
      [&]() {
        if (!c || !c->comm) fail("communicator is NULL or aborted");
        const cudaStream_t s = static_cast<cudaStream_t>(stream);
        const auto t0 = std::chrono::steady_clock::now();
        while (true) {
          const cudaError_t q = cudaStreamQuery(s);
          if (q == cudaSuccess) break;
          if (q != cudaErrorNotReady) cuda_ok(q, "stream");
          ncclResult_t ae = ncclSuccess;
          nccl_ok(nccl().comm_get_async_error(c->comm, &ae), "ncclCommGetAsyncError");
          const bool late = std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms);
          if ((ae != ncclSuccess && ae != ncclInProgress) || late) {
            nccl().comm_abort(c->comm);
            c->comm = nullptr;
            fail(late ? "the collective did not complete within the time limit; the communicator was aborted"
                      : std::string("the collective failed (") + nccl().get_error_string(ae) +
                            "); the communicator was aborted");
          }
          std::this_thread::sleep_for(std::chrono::microseconds(50));
        }
        return 0;
      },
      -1);
}

VERBO_CUDA_API int verbo_cuda_sharded_sample(verbo_cuda_comm* c, const float* logits, int rows, int shard_cols,
                                             long long ld, int col_offset, int vocab, const int* hist,
                                             const long long* hist_off, const verbo_sampling* opts, int k,
                                             unsigned long long* rng, int* out_ids, verbo_row_stats* stats,
                                             void* stream) {
  return guard(
      [&]() {
        if (!c || !c->comm) fail("communicator is NULL or aborted");
        if (!opts) fail("opts is NULL");
        if (rows < 0) fail("rows must be >= 0");
        if (rows == 0) return 0;
        if (!logits || !out_ids) fail("logits and out_ids must not be NULL");
        if (k < 1 || k > vb::kSplitMaxK) fail("k must be in [1, " + std::to_string(vb::kSplitMaxK) + "]");
        if (static_cast<long long>(c->nranks) * k > vb::kMaxMerge)
          fail("nranks * k must be <= " + std::to_string(vb::kMaxMerge));
        if (vocab < 1 || vocab > vb::kMaxVocab) fail("vocab must be in [1, " + std::to_string(vb::kMaxVocab) + "]");
        if (shard_cols < 1 || col_offset < 0 || static_cast<long long>(col_offset) + shard_cols > vocab)
          fail("shard [col_offset, col_offset + shard_cols) must lie in [0, vocab)");
        if (ld < shard_cols) fail("ld must be >= shard_cols");
        check_hist(hist, hist_off);
        vb::DevOpts o = make_opts(*opts, vocab, hist != nullptr);
        if (!o.greedy && !(opts->top_k > 0 && opts->top_k <= k && opts->top_k < vocab))
          fail("vocab-sharded sampling needs temp <= 0 or 0 < top_k <= k");
        if (!o.greedy && !rng) fail("rng state is required when temp > 0");
        const cudaStream_t s = static_cast<cudaStream_t>(stream);
        std::lock_guard<std::mutex> lk(c->mu);
        const size_t need = static_cast<size_t>(rows) * k;
        if (c->cap < need) {
          cuda_ok(cudaStreamSynchronize(s), "stream");  // the old buffers may still be in use
          cudaFree(c->local);
          cudaFree(c->gathered);
          c->local = c->gathered = nullptr;
          c->cap = 0;
          cuda_ok(cudaMalloc(&c->local, need * sizeof(uint2)), "cudaMalloc candidates");
          cuda_ok(cudaMalloc(&c->gathered, need * c->nranks * sizeof(uint2)), "cudaMalloc candidates");
          c->cap = need;
        }
        // step 1: this shard's k best (value, global id), packed
        vb::RowArgs a = row_args(logits, rows, shard_cols, ld, col_offset, vocab, hist, hist_off);
        a.cand_packed = c->local;
        a.cand_k = k;
        plan_split(a);
        attach_split_scratch(a, o, false, s);
        cuda_ok(vb::launch_split(a, o, vb::kSplitEmit, s), "kernel launch");
        const cudaEvent_t ms = c->mark_shard, mg = c->mark_gather;
        c->mark_shard = c->mark_gather = nullptr;
        if (ms) cuda_ok(cudaEventRecord(ms, s), "cudaEventRecord");
        // step 2: one all-gather of every rank's packed candidates
        nccl_ok(nccl().all_gather(c->local, c->gathered, need, ncclUint64, c->comm, s), "ncclAllGather");
        if (mg) cuda_ok(cudaEventRecord(mg, s), "cudaEventRecord");
        // step 3: the merge and the pick, identical on every rank
        vb::MergeArgs m{};
        m.cand_packed = c->gathered;
        m.rows = rows;
        m.nshards = c->nranks;
        m.k = k;
        m.rng = rng;
        m.out_ids = out_ids;
        m.stats = stats;
        cuda_ok(vb::launch_merge(m, o, s), "kernel launch");
        return 0;
      },
      -1);
}

VERBO_CUDA_API int verbo_cuda_comm_mark_next(verbo_cuda_comm* c, void* after_shard, void* after_gather) {
  return guard(
      [&]() {
        if (!c) fail("communicator is NULL");
        std::lock_guard<std::mutex> lk(c->mu);
        c->mark_shard = static_cast<cudaEvent_t>(after_shard);
        c->mark_gather = static_cast<cudaEvent_t>(after_gather);
        return 0;
      },
      -1);
}

}  // extern "C"

// ============================================ request batching (server) ===
// Continuous batching of generation requests, each with its own sampling
// options (the reference's server maps every request's JSON options to a
// Sampling, cli/serve.cpp:149-157, and runs one request at a time behind a
// mutex, :168).  Active requests occupy rows 0..A-1 of a step, grouped by
// option set so that each group is a contiguous run of rows that one
// launch chain samples; the per-request sampler state (RNG, penalty ring)
// lives in device rows that move with the request (state_gather) when the
// rows are re-packed.
namespace {

struct ServerReq {
  long long id = 0;
  std::vector<int> prompt;
  verbo_sampling opts{};
  int max_tokens = 0;
  std::vector<int> tokens;
  bool stopped = false;
  bool finished = false;
  bool released = false;  // collected by the caller; freed once no step row lists it
};

bool same_opts(const verbo_sampling& a, const verbo_sampling& b) {
  return std::memcmp(&a.temp, &b.temp, sizeof(float)) == 0 && a.top_k == b.top_k &&
         std::memcmp(&a.top_p, &b.top_p, sizeof(float)) == 0 && std::memcmp(&a.min_p, &b.min_p, sizeof(float)) == 0 &&
         std::memcmp(&a.repeat, &b.repeat, sizeof(float)) == 0 && a.repeat_last == b.repeat_last;
}

}  // namespace

struct verbo_cuda_server {
  int device = 0, slots = 0, vocab = 0, win_w = 0;
  std::vector<int> stop;                       // the model's stop ids (Model::is_stop)
  std::deque<ServerReq*> queue;
  std::vector<ServerReq*> rows;                // row -> request of the prepared step (size A)
  std::map<long long, ServerReq*> all;         // every request not yet collected
  long long next_id = 0;
  bool prepared = false;
  // device state, double-buffered for re-packing
  unsigned long long* rng[2] = {nullptr, nullptr};
  int* win[2] = {nullptr, nullptr};
  long long* pos[2] = {nullptr, nullptr};
  int cur = 0;
  long long* off = nullptr;   // CSR view of the rings: row r at r * win_w
  int* from = nullptr;        // re-packing map (device)
  int* stage = nullptr;       // prompt ids on their way to a ring (device, win_w ints)
  int* ids = nullptr;         // the step's picks (device)
  float* host_rows = nullptr; // device copy of host logits rows
  long long host_rows_cap = 0;
  std::mutex mu;
};

namespace {

void server_release(verbo_cuda_server* v) {
  if (!v) return;
  cudaSetDevice(v->device);
  cudaDeviceSynchronize();
  for (int i = 0; i < 2; ++i) {
    cudaFree(v->rng[i]);
    cudaFree(v->win[i]);
    cudaFree(v->pos[i]);
  }
  cudaFree(v->off);
  cudaFree(v->from);
  cudaFree(v->stage);
  cudaFree(v->ids);
  cudaFree(v->host_rows);
  for (ServerReq* r : v->rows)
    if (r->released) delete r;
  for (auto& kv : v->all) delete kv.second;
  delete v;
}

}  // namespace

extern "C" {

VERBO_CUDA_API verbo_cuda_server* verbo_cuda_server_new(int slots, int vocab, int max_window, const int* stop_ids,
                                                        int n_stop, int device) {
  return guard(
      [&]() -> verbo_cuda_server* {
        if (slots < 1 || slots > (1 << 16)) fail("slots must be in [1, 65536]");
        if (vocab < 1 || vocab > vb::kMaxVocab) fail("vocab must be in [1, " + std::to_string(vb::kMaxVocab) + "]");
        if (max_window < 1 || max_window > vb::kWinMax)
          fail("max_window must be in [1, " + std::to_string(vb::kWinMax) + "]");
        if (n_stop < 0 || (n_stop > 0 && !stop_ids)) fail("stop ids: n_stop >= 0 and a pointer when n_stop > 0");
        int n = 0;
        cuda_ok(cudaGetDeviceCount(&n), "cudaGetDeviceCount");
        if (device < 0 || device >= n) fail("no CUDA device " + std::to_string(device));
        cuda_ok(cudaSetDevice(device), "cudaSetDevice");
        auto* v = new verbo_cuda_server();
        v->device = device;
        v->slots = slots;
        v->vocab = vocab;
        v->win_w = (max_window + 3) & ~3;
        v->stop.assign(stop_ids, stop_ids + n_stop);
        try {
          for (int i = 0; i < 2; ++i) {
            cuda_ok(cudaMalloc(&v->rng[i], 16ull * slots), "cudaMalloc rng");
            cuda_ok(cudaMalloc(&v->win[i], 4ull * v->win_w * slots), "cudaMalloc rings");
            cuda_ok(cudaMalloc(&v->pos[i], 8ull * slots), "cudaMalloc ring positions");
          }
          cuda_ok(cudaMalloc(&v->off, 8ull * (slots + 1)), "cudaMalloc offsets");
          cuda_ok(cudaMalloc(&v->from, 4ull * slots), "cudaMalloc map");
          cuda_ok(cudaMalloc(&v->stage, 4ull * v->win_w), "cudaMalloc staging");
          cuda_ok(cudaMalloc(&v->ids, 4ull * slots), "cudaMalloc ids");
          std::vector<long long> off(static_cast<size_t>(slots) + 1);
          for (int i = 0; i <= slots; ++i) off[i] = static_cast<long long>(i) * v->win_w;
          cuda_ok(cudaMemcpy(v->off, off.data(), off.size() * 8, cudaMemcpyHostToDevice), "upload offsets");
        } catch (...) {
          server_release(v);
          throw;
        }
        return v;
      },
      static_cast<verbo_cuda_server*>(nullptr));
}

VERBO_CUDA_API void verbo_cuda_server_free(verbo_cuda_server* v) { server_release(v); }

VERBO_CUDA_API long long verbo_cuda_server_submit(verbo_cuda_server* v, const int* prompt, int n,
                                                  const verbo_sampling* opts, int max_tokens) {
  return guard(
      [&]() -> long long {
        if (!v || !opts) fail("server and opts must not be NULL");
        if (n < 0 || (n > 0 && !prompt)) fail("prompt: n >= 0 and a pointer when n > 0");
        if (max_tokens < 0) fail("max_tokens must be >= 0");
        if (opts->seed == 0) fail("seed 0 takes the clock in the reference; give each request its own seed");
        if (std::isnan(opts->temp) || opts->temp == INFINITY) fail("temp must not be NaN or +inf");
        if (opts->repeat != 1.0f && (opts->repeat_last < 1 || opts->repeat_last > v->win_w))
          fail("a repetition penalty needs 1 <= repeat_last <= the server's window (" + std::to_string(v->win_w) + ")");
        for (int i = 0; i < n; ++i)
          if (prompt[i] < 0 || prompt[i] >= v->vocab) fail("prompt ids must be in [0, vocab)");
        std::lock_guard<std::mutex> lk(v->mu);
        auto* r = new ServerReq();
        r->id = v->next_id++;
        r->prompt.assign(prompt, prompt + n);
        r->opts = *opts;
        r->max_tokens = max_tokens;
        v->all[r->id] = r;
        if (max_tokens == 0)
          r->finished = true;
        else
          v->queue.push_back(r);
        return r->id;
      },
      -1ll);
}

// Admits queued requests into free rows, re-packs the rows by option set and
// returns the step's row -> request map (row_req[0..slots), -1 for idle
// rows).  Returns the number of active rows A (rows 0..A-1), 0 when idle.
VERBO_CUDA_API int verbo_cuda_server_prepare(verbo_cuda_server* v, long long* row_req, void* cuda_stream) {
  return guard(
      [&]() {
        if (!v || !row_req) fail("server and row_req must not be NULL");
        std::lock_guard<std::mutex> lk(v->mu);
        cuda_ok(cudaSetDevice(v->device), "cudaSetDevice");
        const cudaStream_t s = static_cast<cudaStream_t>(cuda_stream);
        // rows of the last step keep their state; new requests go to the rows after them
        std::vector<std::pair<ServerReq*, int>> live;  // request, its state row now
        for (int r = 0; r < static_cast<int>(v->rows.size()); ++r)
          if (!v->rows[r]->finished) live.emplace_back(v->rows[r], r);
        // free state rows: those not held by a live request
        std::vector<char> held(static_cast<size_t>(v->slots), 0);
        for (auto& p : live) held[p.second] = 1;
        std::vector<int> free_rows;
        for (int r = 0; r < v->slots; ++r)
          if (!held[r]) free_rows.push_back(r);
        size_t fi = 0;
        while (!v->queue.empty() && fi < free_rows.size()) {
          ServerReq* q = v->queue.front();
          v->queue.pop_front();
          const int r = free_rows[fi++];
          // Sampler(opts) with the request's seed, then accept(prompt): only
          // the last repeat_last ids can reach the window (src/sampler.cpp:26-48)
          unsigned long long st[2];
          seed_state(q->opts.seed, st);
          int* w = v->win[v->cur] + static_cast<long long>(r) * v->win_w;
          cuda_ok(cudaMemcpyAsync(v->rng[v->cur] + 2ll * r, st, sizeof(st), cudaMemcpyHostToDevice, s), "upload rng");
          cuda_ok(cudaMemsetAsync(w, 0xff, 4ull * v->win_w, s), "clear ring");
          cuda_ok(cudaMemsetAsync(v->pos[v->cur] + r, 0, 8, s), "clear ring position");
          if (q->opts.repeat != 1.0f && !q->prompt.empty()) {
            const int len = q->opts.repeat_last;
            const int np = static_cast<int>(q->prompt.size());
            const int skip = np > len ? np - len : 0;
            cuda_ok(cudaMemcpyAsync(v->stage, q->prompt.data() + skip, 4ull * (np - skip), cudaMemcpyHostToDevice, s),
                    "upload prompt");
            cuda_ok(vb::launch_ring_accept(v->win[v->cur], v->win_w, len, v->pos[v->cur], r, v->stage, np - skip, skip, s),
                    "kernel launch");
            cuda_ok(cudaStreamSynchronize(s), "stream");  // the staging buffer is reused by the next admission
          }
          live.emplace_back(q, r);
        }
        // group by option set (first appearance order), stable within a group
        std::vector<std::pair<ServerReq*, int>> order;
        std::vector<char> taken(live.size(), 0);
        for (size_t i = 0; i < live.size(); ++i) {
          if (taken[i]) continue;
          for (size_t j = i; j < live.size(); ++j)
            if (!taken[j] && same_opts(live[i].first->opts, live[j].first->opts)) {
              order.push_back(live[j]);
              taken[j] = 1;
            }
        }
        for (ServerReq* q : v->rows)
          if (q->released) delete q;  // collected while its row was still listed
        v->rows.clear();
        bool identity = true;
        std::vector<int> from(order.size());
        for (size_t r = 0; r < order.size(); ++r) {
          v->rows.push_back(order[r].first);
          from[r] = order[r].second;
          identity = identity && from[r] == static_cast<int>(r);
        }
        if (!identity) {  // move the states to their new rows
          const int nxt = v->cur ^ 1;
          cuda_ok(cudaMemcpyAsync(v->from, from.data(), 4ull * from.size(), cudaMemcpyHostToDevice, s), "upload map");
          cuda_ok(vb::launch_state_gather(v->from, static_cast<int>(from.size()), v->rng[v->cur], v->rng[nxt],
                                          v->win[v->cur], v->win[nxt], v->win_w, v->pos[v->cur], v->pos[nxt], s),
                  "kernel launch");
          cuda_ok(cudaStreamSynchronize(s), "stream");  // the map buffer is reused by the next re-packing
          v->cur = nxt;
        }
        for (int r = 0; r < v->slots; ++r)
          row_req[r] = r < static_cast<int>(v->rows.size()) ? v->rows[r]->id : -1;
        v->prepared = true;
        return static_cast<int>(v->rows.size());
      },
      -1);
}

// Samples the prepared step: `logits` holds the A active rows (row r at
// logits + r*ld, host or device memory), each sampled with its request's
// options; every request takes its id (a stop id ends it without being
// emitted, as in verbo::generate, src/sampler.cpp:156-165) and the requests
// that stop or reach max_tokens finish.  Returns the number that finished.
VERBO_CUDA_API int verbo_cuda_server_step(verbo_cuda_server* v, const float* logits, long long ld, void* cuda_stream) {
  return guard(
      [&]() {
        if (!v) fail("server is NULL");
        std::lock_guard<std::mutex> lk(v->mu);
        if (!v->prepared) fail("call verbo_cuda_server_prepare before each step");
        v->prepared = false;
        const int A = static_cast<int>(v->rows.size());
        if (A == 0) return 0;
        if (!logits) fail("logits must not be NULL");
        if (ld < v->vocab) fail("ld must be >= vocab");
        cuda_ok(cudaSetDevice(v->device), "cudaSetDevice");
        const cudaStream_t s = static_cast<cudaStream_t>(cuda_stream);
        const float* rows = logits;
        long long lr = ld;
        if (!on_device(logits)) {
          grow(v->host_rows, v->host_rows_cap, static_cast<long long>(A) * v->vocab, s, "cudaMalloc logits rows");
          cuda_ok(cudaMemcpy2DAsync(v->host_rows, 4ull * v->vocab, logits, 4ull * ld, 4ull * v->vocab, A,
                                    cudaMemcpyHostToDevice, s),
                  "upload logits rows");
          rows = v->host_rows;
          lr = v->vocab;
        }
        // one launch chain per run of rows with the same options
        for (int r0 = 0; r0 < A;) {
          int r1 = r0 + 1;
          while (r1 < A && same_opts(v->rows[r0]->opts, v->rows[r1]->opts)) ++r1;
          const verbo_sampling& so = v->rows[r0]->opts;
          const bool pen = so.repeat != 1.0f;
          vb::DevOpts o = make_opts(so, v->vocab, pen);
          if (pen) o.repeat_last = v->win_w;  // the CSR view reads whole rings; -1 slots mark nothing
          int* ring = v->win[v->cur] + static_cast<long long>(r0) * v->win_w;
          vb::RowArgs a = row_args(rows + static_cast<long long>(r0) * lr, r1 - r0, v->vocab, lr, 0, v->vocab,
                                   pen ? ring : nullptr, pen ? v->off : nullptr);
          a.rng = v->rng[v->cur] + 2ll * r0;
          a.out_ids = v->ids + r0;
          if (pen) {
            a.ring_pos = v->pos[v->cur] + r0;
            a.ring_len = so.repeat_last;
          }
          dispatch_rows(a, o, v->vocab, s, pen ? ring : nullptr, v->win_w);
          r0 = r1;
        }
        std::vector<int> got(static_cast<size_t>(A));
        cuda_ok(cudaMemcpyAsync(got.data(), v->ids, 4ull * A, cudaMemcpyDeviceToHost, s), "download ids");
        cuda_ok(cudaStreamSynchronize(s), "stream");
        int finished = 0;
        for (int r = 0; r < A; ++r) {
          ServerReq* q = v->rows[r];
          const int id = got[static_cast<size_t>(r)];
          if (std::find(v->stop.begin(), v->stop.end(), id) != v->stop.end())
            q->stopped = true;
          else
            q->tokens.push_back(id);
          if (q->stopped || static_cast<int>(q->tokens.size()) >= q->max_tokens) {
            q->finished = true;
            ++finished;
          }
        }
        return finished;
      },
      -1);
}

// A request's state: 1 finished, 0 still running or queued, -1 unknown id.
// Fills n_tokens, stopped and up to cap of its ids; a finished request is
// forgotten once collected with release = 1.
VERBO_CUDA_API int verbo_cuda_server_result(verbo_cuda_server* v, long long id, int* tokens, int cap, int* n_tokens,
                                            int* stopped, int release) {
  return guard(
      [&]() {
        if (!v) fail("server is NULL");
        std::lock_guard<std::mutex> lk(v->mu);
        auto it = v->all.find(id);
        if (it == v->all.end()) fail("unknown request id " + std::to_string(id));
        ServerReq* q = it->second;
        const int n = static_cast<int>(q->tokens.size());
        if (n_tokens) *n_tokens = n;
        if (stopped) *stopped = q->stopped ? 1 : 0;
        if (tokens && cap > 0) std::memcpy(tokens, q->tokens.data(), 4ull * std::min(n, cap));
        const int done = q->finished ? 1 : 0;
        if (done && release) {
          v->all.erase(it);
          if (std::find(v->rows.begin(), v->rows.end(), q) != v->rows.end())
            q->released = true;  // the next prepare frees it
          else
            delete q;
        }
        return done;
      },
      -1);
}

}  // extern "C"
