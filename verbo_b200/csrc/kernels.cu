// sm_100a kernels of the token-sampling path: a drop-in for the per-row work
// of verbo's Sampler::pick (src/sampler.cpp:50-109).
//
//   split_kernel    (greedy, 0 < top_k <= 256, and shard top-k)  One CTA of
//                   256 threads per (row, slice of <= 10240 columns), no
//                   clusters.  Every thread issues all of its 16-byte loads
//                   up front (10 in flight), applies the penalty from a
//                   per-slice bitmap, and reduces its columns with float
//                   compares.  Greedy publishes the slice's best key; top-k
//                   bounds the slice's top-k by a histogram of thread maxima
//                   and publishes every column above the bound.  The CTA then
//                   exits.
//   merge_slices_kernel  One CTA per row, after split_kernel on the same
//                   stream: the best key, or a radix selection of the k best
//                   of the union of candidates followed by the reference's
//                   softmax / min-p / top-p / draw in the same fp64 order
//                   (sampler.cpp:79-108).
//   general_kernel  (top_k == 0, top_k > 256 or top_k >= vocab)  One thread-
//                   block cluster per row; each CTA stages its slice in shared
//                   memory with bulk async copies.  Masses exp((v - M) / T) in
//                   64-bit fixed point (exact, order independent) go into a
//                   value-space histogram relative to the row maximum; the
//                   top-p cutoff bin and the bins the draw can reach are
//                   gathered once into every CTA and resolved there.  An exact
//                   mass-weighted radix selection over the keys handles rows
//                   whose bins are too crowded.  No full sort.
//   merge_kernel    merges per-shard candidates and runs the same tail.
#include <algorithm>
#include <mutex>
#include <utility>

#include "device.cuh"
#include "kernels.cuh"
#include "rowdev.cuh"

namespace vb {

__device__ unsigned int g_status;

__device__ __forceinline__ void raise_status(unsigned bits) { atomicOr(&g_status, bits); }

// ======================================================== shared tail (top-k)
struct TailShared {
  double sum;
  int keep;
};

// Softmax, min-p, top-p and the inverse-CDF draw over the k best candidates
// sorted in the reference order (src/sampler.cpp:79-108).  The exps run in
// parallel; every sum runs in one thread in the reference's order with
// correctly rounded fp64 operations, so the result is the reference's
// whenever the fp64 exp agrees.  The softmax sum leaves its running value in
// pre (pre[i] = pr[0] + ... + pr[i], summed from 0.0 in that order), which is
// exactly the reference's later sum of the kept candidates (pre[keep - 1])
// and the mass below the pick (pre[pick - 1]).  While thread 0 sums, warp 1
// finds the min-p cut (the first i >= 1 with pr[i] below the threshold) by
// ballots.  The sequential top-p and draw chains read their inputs eight
// ahead.  pr, q, pre: >= k doubles of shared scratch each; blockDim.x >= 64.
// rng: the row's state, written back (advanced); rng0 / rng1: its words as
// thread 0 loaded them early, off the critical path.
__device__ void tail_pick(const uint64_t* c, int k, const DevOpts& o, unsigned long long* rng, unsigned long long rng0,
                          unsigned long long rng1, int* out_id,
                          verbo_row_stats* st, double* pr, double* q, double* pre, TailShared* ts) {
  constexpr int kAhead = 8;
  const float mx = dval(c[0]);
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    const float v = dval(c[i]);
    pr[i] = exp(__ddiv_rn(static_cast<double>(__fsub_rn(v, mx)), static_cast<double>(o.temp)));
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double run = 0.0;
    for (int i0 = 0; i0 < k; i0 += kAhead) {
      double v[kAhead];
#pragma unroll
      for (int u = 0; u < kAhead; ++u) v[u] = i0 + u < k ? pr[i0 + u] : 0.0;
#pragma unroll
      for (int u = 0; u < kAhead; ++u)
        if (i0 + u < k) {
          run = __dadd_rn(run, v[u]);
          pre[i0 + u] = run;
        }
    }
    ts->sum = run;
  } else if (threadIdx.x >> 5 == 1) {
    int keep = k;
    if (o.min_p > 0.0f) {
      const int lane = threadIdx.x & 31;
      const double thr = __dmul_rn(pr[0], static_cast<double>(o.min_p));
      for (int b = 1; b < k; b += 32) {
        const int i = b + lane;
        const unsigned low = __ballot_sync(0xffffffffu, i < k && !(pr[i] >= thr));
        if (low) {
          keep = b + __ffs(low) - 1;
          break;
        }
      }
    }
    if ((threadIdx.x & 31) == 0) ts->keep = keep;
  }
  __syncthreads();
  const bool use_p = o.top_p > 0.0f && o.top_p < 1.0f;
  if (use_p)
    for (int i = threadIdx.x; i < ts->keep; i += blockDim.x) q[i] = __ddiv_rn(pr[i], ts->sum);
  __syncthreads();
  if (threadIdx.x != 0) return;
  const double inf = __longlong_as_double(0x7ff0000000000000ll);
  const double sum = ts->sum;
  int keep = ts->keep;
  double cut = inf;
  if (st && o.min_p > 0.0f) {
    const double thr = __dmul_rn(pr[0], static_cast<double>(o.min_p));
    cut = fmin(cut, (pr[keep - 1] - thr) / sum);
    if (keep < k) cut = fmin(cut, (thr - pr[keep]) / sum);
  }
  if (use_p) {
    const double tp = static_cast<double>(o.top_p);
    double acc = 0.0, prev = 0.0;
    int i = keep;  // the first index whose running mass reaches tp, else keep
    for (int i0 = 0; i0 < keep; i0 += kAhead) {
      double v[kAhead];
#pragma unroll
      for (int u = 0; u < kAhead; ++u) v[u] = i0 + u < keep ? q[i0 + u] : 0.0;
      int hit = -1;
#pragma unroll
      for (int u = 0; u < kAhead; ++u)
        if (hit < 0 && i0 + u < keep) {
          prev = acc;
          acc = __dadd_rn(acc, v[u]);
          if (acc >= tp) hit = u;
        }
      if (hit >= 0) {
        i = i0 + hit;
        break;
      }
    }
    if (i < keep) {
      cut = fmin(cut, acc - tp);
      if (i > 0) cut = fmin(cut, tp - prev);
    } else {
      cut = fmin(cut, tp - acc);
    }
    keep = keep < i + 1 ? keep : i + 1;
  }
  const double tot = pre[keep - 1];  // keep >= 1
  unsigned long long s1 = rng0, s0 = rng1;
  const double u = rng_unit(s1, s0);
  rng[0] = s1;
  rng[1] = s0;
  double r = __dmul_rn(u, tot);
  const double r0 = r;
  int pick = keep - 1;
  for (int i0 = 0; i0 < keep; i0 += kAhead) {
    double v[kAhead];
#pragma unroll
    for (int w = 0; w < kAhead; ++w) v[w] = i0 + w < keep ? pr[i0 + w] : 0.0;
    int hit = -1;
#pragma unroll
    for (int w = 0; w < kAhead; ++w)
      if (hit < 0 && i0 + w < keep) {
        r = __dsub_rn(r, v[w]);
        if (r <= 0.0) hit = w;
      }
    if (hit >= 0) {
      pick = i0 + hit;
      break;
    }
  }
  const int id = static_cast<int>(did(c[pick]));
  *out_id = id;
  if (st) {
    const double below = pick > 0 ? pre[pick - 1] : 0.0;
    double m = inf;
    if (pick > 0) m = fmin(m, r0 - below);
    if (pick < keep - 1) m = fmin(m, below + pr[pick] - r0);
    write_stats(st, sum, tot, u, m / tot, cut, k, keep, id, 0);
  }
}

// ====================================================================== top-k
struct Found {
  int bin;
  uint32_t before;
  uint32_t cnt;
};

__device__ __forceinline__ uint64_t ckey(float v, uint32_t gid, int idxbits) {
  return (static_cast<uint64_t>(~ord32(canon(v))) << idxbits) | gid;
}

// ====================================================================== merge
// A row's merge is latency-bound (a few thousand keys at most, then the
// serial sums of the pick): it places the keys by ranking them across the
// shards' sorted lists and sorts only lists that are not sorted.  Small CTAs,
// so that 512 rows run in one wave.
constexpr int kMergeThreads = 256;

__global__ void __launch_bounds__(kMergeThreads) merge_kernel(const MergeArgs a, const DevOpts o) {
  constexpr int T = kMergeThreads;
  const int row = blockIdx.x;
  unsigned long long rng0 = 0, rng1 = 0;  // read now, used by thread 0 at the draw
  if (threadIdx.x == 0 && !o.greedy) {
    rng0 = a.rng[2ll * row];
    rng1 = a.rng[2ll * row + 1];
  }
  extern __shared__ __align__(16) unsigned char smem[];
  const int total = a.nshards * a.k;
  const int P = next_pow2(max(total, 2));
  uint64_t* cand = reinterpret_cast<uint64_t*>(smem);  // P keys in input order
  uint64_t* merged = cand + P;                          // P keys in merged order
  double* pr = reinterpret_cast<double*>(merged + P);
  double* q = pr + kSplitMaxK;
  double* pre = q + kSplitMaxK;
  __shared__ uint32_t ws[T / 32];
  __shared__ TailShared ts;
  uint32_t valid = 0;
  for (int i = threadIdx.x; i < P; i += T) {
    uint64_t d = kNoKey;
    if (i < total) {
      const int s = i / a.k, j = i - s * a.k;
      const long long at = (static_cast<long long>(s) * a.rows + row) * a.k + j;
      int id;
      float val;
      if (a.cand_packed) {
        const uint2 c = a.cand_packed[at];
        id = static_cast<int>(c.y);
        val = __uint_as_float(c.x);
      } else {
        id = a.cand_id[at];
        val = id >= 0 ? a.cand_val[at] : 0.0f;
      }
      if (id >= 0) {
        d = dkey(val, static_cast<uint32_t>(id));
        ++valid;
      }
    }
    cand[i] = d;
  }
  __syncthreads();
  // Step 1 emits each shard's list in the reference order with missing slots
  // last, i.e. ascending keys.  Then the merged order is a stable merge of
  // sorted lists: a key's place is its index in its own list plus, for every
  // other list, the number of keys before it (<= for earlier lists, < for
  // later ones, so equal keys keep distinct places).  The pick reads only
  // the first min(k, valid) places (the first one when greedy), so a key
  // stops as soon as its place reaches that cap, and each search looks only
  // at the entries that could keep it below.  Every list's first r =
  // ceil(cap / nshards) keys are <= bound, the largest of the lists' r-th
  // keys: that is >= cap keys, so a key above bound has no place either.
  // The places written are the cap's first ones, each exactly once; lists
  // that are not sorted discard them and take the full sort instead.
  const int cap = o.greedy ? 1 : o.k;
  const int m = min(a.k, cap);  // keys of each list that can be placed
  const int r = (cap + a.nshards - 1) / a.nshards;
  uint64_t bound = 0;
  for (int t = 0; t < a.nshards; ++t) bound = max(bound, cand[t * a.k + r - 1]);
  bool bad = false;
  for (int i = threadIdx.x; i < total; i += T) {
    const int s = i / a.k;
    if (i > s * a.k && cand[i - 1] > cand[i]) bad = true;
  }
  // keys taken index-major, so that the few below the bound (the lists'
  // first ones) fall to different threads
  for (int x = threadIdx.x; x < a.nshards * m; x += T) {
    const int j = x / a.nshards, s = x - j * a.nshards;
    const uint64_t d = cand[s * a.k + j];
    if (d > bound) continue;  // kNoKey included
    int at = j;
    for (int t = 0; t < a.nshards && at < cap; ++t) {
      if (t == s) continue;
      const uint64_t* seg = cand + t * a.k;
      int lo = 0, hi = min(a.k, cap - at);
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        const uint64_t e = seg[mid];
        if (t < s ? e <= d : e < d) lo = mid + 1;
        else hi = mid;
      }
      at += lo;
    }
    if (at < cap) merged[at] = d;
  }
  const bool unsorted = __syncthreads_or(bad);
  valid = block_sum<uint32_t, T>(valid, ws);
  if (unsorted) bitonic_sort_u64(cand, P);
  const uint64_t* c = unsorted ? cand : merged;
  if (valid == 0) {
    if (threadIdx.x == 0) {
      raise_status(kErrSelect);
      a.out_ids[row] = -1;
    }
    return;
  }
  if (o.greedy) {
    if (threadIdx.x == 0) {
      const int id = static_cast<int>(did(c[0]));
      a.out_ids[row] = id;
      if (a.stats) write_stats(a.stats + row, 0.0, 0.0, 0.0, __longlong_as_double(0x7ff0000000000000ll),
                               __longlong_as_double(0x7ff0000000000000ll), o.vocab, 1, id, 1);
    }
    return;
  }
  const int kk = min(o.k, static_cast<int>(valid));
  tail_pick(c, kk, o, a.rng + 2ll * row, rng0, rng1, a.out_ids + row, a.stats ? a.stats + row : nullptr, pr, q, pre,
            &ts);
}

// ================================================================== general
// Staged full-vocabulary path.  Histograms have 512 bins (9-bit digits) with
// a 64-bit fixed-point mass and a 32-bit count per bin.
constexpr int kGBins = 512;
constexpr int kGDig = 9;
constexpr int kGatherCap = 256;
constexpr int kMaxGathers = 8;

struct Hist {
  unsigned long long m[kGBins];
  uint32_t c[kGBins];
};

struct Gath {
  unsigned long long key[kGatherCap];
  unsigned long long mass[kGatherCap];
};

// Value-space histogram of the nucleus path: bin = floor((M - v) * kVBins / R)
// over the row's value range R (see general_kernel).  12 KB, aliasing two Hist.
constexpr int kVBins = 1024;
constexpr int kVGatherCap = 512;
struct VHist {
  unsigned long long m[kVBins];
  uint32_t c[kVBins];
};
struct VGath {
  unsigned long long key[kVGatherCap];
  unsigned long long mass[kVGatherCap];
};
static_assert(sizeof(VHist) == 2 * sizeof(Hist), "VHist aliases two Hist");
static_assert(sizeof(VGath) == 2 * sizeof(Gath), "VGath aliases two Gath");

struct HFound {
  int bin;
  unsigned long long before_m, m, total_m;
  uint32_t before_c, c, total_c;
};

struct GenShared {
  uint64_t bar;
  uint64_t xmin[kMaxCluster];
  float xlo[kMaxCluster];
  unsigned long long xs[kMaxCluster];
  unsigned long long xz[kMaxCluster];
  alignas(16) unsigned long long my_sz[2];  // this CTA's mass-pass totals (S, Z), pulled by the others
  unsigned long long all_sz[2];              // the cluster's totals
  // value-path decisions (identical in every CTA)
  int v_gather;      // 1: resolve by one gather of bins [vb_lo, vb_hi]
  int vb_lo, vb_hi;
  unsigned long long vbase_m;  // mass of bins before vb_lo
  uint32_t vbase_c;
  unsigned long long v_tp;     // top-p target (0: no cutoff)
  unsigned long long v_ptot;   // P-set mass
  uint32_t v_pcnt;             // P-set count (positive fixed mass)
  uint32_t gcount[kMaxGathers];
  unsigned long long ws64[kWarps];
  uint32_t ws32[kWarps];
  HFound hf;
  int load_fail;
  uint32_t ng;
  // selection result
  unsigned long long r_key, r_cum_m;
  uint32_t r_cum_c;
  int r_found;
  uint32_t r_steps;  // resolve: rank + 1 of the member found among the gathered ones
  uint32_t ncrowd;   // resolve: members of the target sub-bin collected
};

__device__ HFound find_hist(const Hist* H, bool by_mass, unsigned long long target, GenShared& sh) {
  if (threadIdx.x == 0) sh.hf.bin = -1;
  const unsigned long long m = H->m[threadIdx.x];
  const uint32_t c = H->c[threadIdx.x];
  unsigned long long tm;
  uint32_t tc;
  const unsigned long long em = block_excl_scan(m, sh.ws64, &tm);
  const uint32_t ec = block_excl_scan(c, sh.ws32, &tc);
  const bool hit = by_mass ? (em < target && target <= em + m) : (ec < target && target <= ec + c);
  if (hit) {
    sh.hf.bin = threadIdx.x;
    sh.hf.before_m = em;
    sh.hf.m = m;
    sh.hf.before_c = ec;
    sh.hf.c = c;
  }
  __syncthreads();
  HFound f = sh.hf;
  f.total_m = tm;
  f.total_c = tc;
  __syncthreads();
  return f;
}

__device__ void push_hist(Hist* L, Hist* G, Hist* clr, cg::cluster_group& cl, int C) {
  const int b = threadIdx.x;  // kGBins == kThreads
  const uint32_t c = L->c[b];
  if (c) {
    const unsigned long long m = L->m[b];
    for (int r = 0; r < C; ++r) {
      atomicAdd(cl.map_shared_rank(&G->c[b], r), c);
      if (m) atomicAdd(cl.map_shared_rank(&G->m[b], r), m);
    }
    L->c[b] = 0;
    L->m[b] = 0;
  }
  if (clr) {
    clr->c[b] = 0;
    clr->m[b] = 0;
  }
}

// Sorts n <= kGatherCap (key, mass) pairs by key, in place.
__device__ void sort_pairs(unsigned long long* key, unsigned long long* mass, int P) {
  for (int k = 2; k <= P; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < P; i += kThreads) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const bool up = (i & k) == 0;
          const unsigned long long a = key[i], b = key[ixj];
          if ((a > b) == up) {
            key[i] = b;
            key[ixj] = a;
            const unsigned long long t = mass[i];
            mass[i] = mass[ixj];
            mass[ixj] = t;
          }
        }
      }
      __syncthreads();
    }
  }
}

struct GenCtx {
  const float* v;  // staged slice values (penalised), element j at v[j]
  int n;
  long long g_lo;
  int idxbits, nbits;
  float M;
  double inv_temp;
  int fixbits;      // F: masses are round(w * 2^F)
  double xcut;      // exponents below it give a fixed-point mass of 0
  bool need_w;      // min-p compares the weights themselves
  const double* T;  // T[j] = 2^(j/256), j < 256 (shared memory)
  int C, crank;
  unsigned long long kc0;  // key of the row's first element in sorted order (always kept by min-p)
};

// The min-p set (src/sampler.cpp:86-91): weights >= thr, and always the
// first element in sorted order (keep starts at 1).
__device__ __forceinline__ bool in_pset(const GenCtx& x, double m, double thr, unsigned long long kc) {
  return !(thr > 0.0) || m >= thr || kc == x.kc0;
}

// The weight w = exp((double)(v - M) / temp) of src/sampler.cpp:79-85 (with
// the division taken as a product by 1/temp) and its fixed-point mass
// round(w * 2^F).  The exponential is table driven, after P. T. P. Tang,
// "Table-driven implementation of the exponential function in IEEE
// floating-point arithmetic", ACM TOMS 15(2), 1989: x = (256 e + j) ln2/256 + r
// with |r| <= ln2/512, exp(x) = 2^e * 2^(j/256) * p(r), p the degree-4 Taylor
// polynomial (truncation below 4e-17 relative), ln2/256 split so that k * hi
// is exact.  Within a few ulp of a correctly rounded exp (tested against
// CUDA's), so sums and decisions differ from the reference's only next to a
// boundary.  Exponents below xcut (w * 2^F < 1/2) give mass 0.
__device__ __forceinline__ unsigned long long fixed_mass(const GenCtx& x, float v, double* m_out) {
  const double xx = static_cast<double>(__fsub_rn(canon(v), x.M)) * x.inv_temp;  // <= 0, -inf for NaN/-inf
  if (!(xx >= x.xcut)) {
    *m_out = x.need_w ? exp(xx) : 0.0;  // min-p may still compare tiny weights
    return 0ull;
  }
  const int k = __double2int_rn(xx * 369.3299304675746);  // 256 / ln2
  const double kd = static_cast<double>(k);
  double r = fma(-kd, 0x1.62e42ff000000p-9, xx);  // ln2/256, high part (exact product)
  r = fma(-kd, -0x1.718432a1b0e26p-43, r);        // low part
  const double p = fma(fma(fma(fma(r, 1.0 / 24.0, 1.0 / 6.0), r, 0.5), r, 1.0), r, 1.0);
  const double y = x.T[k & 255] * p;  // in [0.9986, 1.9973]
  const int e = k >> 8;               // floor(k / 256) >= -(F + 2)
  *m_out = y * __longlong_as_double(static_cast<long long>(1023 + e) << 52);
  return __double2ull_rn(y * __longlong_as_double(static_cast<long long>(1023 + x.fixbits + e) << 52));
}

// Mass- or count-weighted selection: the first element, in the reference's
// order, at which the running weight of the set {key <= klim, mass >= thr}
// reaches `target` (>= 1).  `start`, if given, is the cluster histogram of the
// first digit for that set (klim may be tighter than the set it was built
// for: only the chosen bin is affected, and it is refined with the exact set).
// Returns found=false if the set's total weight is below target.
__device__ void select_weighted(const GenCtx& x, bool by_mass, unsigned long long target, const Hist* start,
                                unsigned long long klim, double thr, Hist* L, Hist* G, Gath* gb, int& gseq, int& gbuf,
                                cg::cluster_group& cl, GenShared& sh) {
  unsigned long long prefix = 0, base_m = 0;
  uint32_t base_c = 0;
  int resolved = 0;
  const Hist* H = start;
  while (true) {
    const int shift = max(0, x.nbits - resolved - kGDig);
    const int width = x.nbits - resolved - shift;
    if (H == nullptr) {
      // histogram pass over the set restricted to the current prefix
      const int hi = x.nbits - resolved;
      const unsigned long long mask = (1ull << width) - 1;
      for (int j = threadIdx.x; j < x.n; j += kThreads) {
        const float v = x.v[j];
        const unsigned long long kc = ckey(v, static_cast<uint32_t>(x.g_lo + j), x.idxbits);
        if (kc > klim) continue;
        if (resolved > 0 && (kc >> hi) != prefix) continue;
        double m;
        const unsigned long long qm = by_mass || thr > 0.0 ? fixed_mass(x, v, &m) : 0ull;
        if (!in_pset(x, m, thr, kc)) continue;
        const int dg = static_cast<int>((kc >> shift) & mask);
        atomicAdd(&L->c[dg], 1u);
        if (by_mass && qm) atomicAdd(&L->m[dg], qm);
      }
      __syncthreads();
      Hist* Gd = G + gbuf;
      push_hist(L, Gd, G + (gbuf ^ 1), cl, x.C);
      cluster_sync_all();
      H = Gd;
      gbuf ^= 1;
    }
    const unsigned long long t = by_mass ? target - base_m : target - base_c;
    const HFound f = find_hist(H, by_mass, t, sh);
    if (f.bin < 0) {
      if (threadIdx.x == 0) sh.r_found = 0;
      __syncthreads();
      return;
    }
    prefix = (prefix << width) | static_cast<unsigned long long>(f.bin);
    resolved += width;
    base_m += f.before_m;
    base_c += f.before_c;
    if (f.c <= static_cast<uint32_t>(kGatherCap) || shift == 0) {
      // Gather the bin's members into every CTA, then scan them in order.
      const int s = gseq++ & 1;
      const int cidx = gseq - 1;
      Gath* g = gb + s;
      uint32_t* cnt0 = cl.map_shared_rank(&sh.gcount[cidx], 0);
      for (int j = threadIdx.x; j < x.n; j += kThreads) {
        const float v = x.v[j];
        const unsigned long long kc = ckey(v, static_cast<uint32_t>(x.g_lo + j), x.idxbits);
        if (kc > klim || (kc >> shift) != prefix) continue;
        double m;
        const unsigned long long qm = by_mass || thr > 0.0 ? fixed_mass(x, v, &m) : 0ull;
        if (!in_pset(x, m, thr, kc)) continue;
        const uint32_t p = atomicAdd(cnt0, 1u);
        if (p < static_cast<uint32_t>(kGatherCap))
          for (int r = 0; r < x.C; ++r) {
            *cl.map_shared_rank(&g->key[p], r) = kc;
            *cl.map_shared_rank(&g->mass[p], r) = qm;
          }
      }
      cluster_sync_all();
      if (threadIdx.x == 0) sh.ng = min(*cnt0, static_cast<uint32_t>(kGatherCap));
      __syncthreads();
      const int ng = static_cast<int>(sh.ng);
      const int P = next_pow2(max(ng, 2));
      for (int i = ng + threadIdx.x; i < P; i += kThreads) {
        g->key[i] = kNoKey;
        g->mass[i] = 0;
      }
      __syncthreads();
      sort_pairs(g->key, g->mass, P);
      if (threadIdx.x == 0) {
        unsigned long long cm = base_m;
        uint32_t cc = base_c;
        int hit = -1;
        for (int i = 0; i < ng; ++i) {
          cm += g->mass[i];
          cc += 1;
          if (by_mass ? cm >= target : cc >= target) {
            hit = i;
            break;
          }
        }
        sh.r_found = hit >= 0;
        if (hit >= 0) {
          sh.r_key = g->key[hit];
          sh.r_cum_m = cm;
          sh.r_cum_c = cc;
        }
      }
      __syncthreads();
      return;
    }
    H = nullptr;
  }
}

// One row of the staged full-vocabulary path, run by every CTA of a cluster.
__device__ __noinline__ void general_row(const RowArgs& a, const DevOpts& o, const int row) {
  cg::cluster_group cl = cg::this_cluster();
  const int C = a.cluster;
  const int crank = static_cast<int>(cl.block_rank());
  const int lo = crank * a.slice;
  const int n = max(0, min(a.ncols - lo, a.slice));
  const float* src = a.logits + static_cast<long long>(row) * a.ld + lo;
  const long long g_lo = static_cast<long long>(a.col_off) + lo;

  extern __shared__ __align__(16) unsigned char smem[];
  float* vals = reinterpret_cast<float*>(smem);
  const int vwords = ((a.slice + 4 + 3) / 4) * 4;
  uint32_t* bm = reinterpret_cast<uint32_t*>(vals + vwords);
  const int bwords = ((((a.slice >> 5) + 2) + 3) / 4) * 4;
  Hist* L = reinterpret_cast<Hist*>(bm + bwords);
  Hist* G = L + 1;   // two buffers
  // L[0..3]: radix histograms of the exact selection; the value path reuses the same bytes
  Gath* gb = reinterpret_cast<Gath*>(L + 4);  // two buffers
  double* etab = reinterpret_cast<double*>(gb + 2);  // 2^(j/256), the exponential's table
  __shared__ GenShared sh;
  for (int j = threadIdx.x; j < 256; j += kThreads) etab[j] = exp2(j * (1.0 / 256.0));

  cluster_arrive();
  // ---- stage the slice: bulk async copy of the 16-byte aligned body
  const uintptr_t addr = reinterpret_cast<uintptr_t>(src);
  int h = static_cast<int>(((16 - (addr & 15)) & 15) >> 2);
  if (h > n) h = n;
  const int nb = ((n - h) >> 2) << 2;
  const int aoff = (4 - h) & 3;
  float* v = vals + aoff;
  if (threadIdx.x == 0) {
    sh.load_fail = 0;
    for (int i = 0; i < kMaxGathers; ++i) sh.gcount[i] = 0;
    if (nb > 0) {
      mbar_init(&sh.bar, 1);
      const uint64_t pol = policy_evict_first();
      const uint32_t bytes = static_cast<uint32_t>(nb) * 4u;
      mbar_expect_tx(&sh.bar, bytes);
      for (uint32_t off = 0; off < bytes; off += 32768u)
        bulk_g2s(reinterpret_cast<char*>(v + h) + off, reinterpret_cast<const char*>(src + h) + off,
                 min(32768u, bytes - off), &sh.bar, pol);
    }
  }
  for (int j = threadIdx.x; j < h; j += kThreads) v[j] = src[j];
  for (int j = h + nb + threadIdx.x; j < n; j += kThreads) v[j] = src[j];
  for (int b = threadIdx.x; b < kGBins; b += kThreads) {
    for (int i = 0; i < 4; ++i) {
      L[i].c[b] = 0;
      L[i].m[b] = 0;
    }
  }
  // RNG: every CTA reads the row's state now; CTA 0 stores the advanced
  // state after the first cluster barrier, when all reads are done.
  unsigned long long s1 = 0, s0 = 0;
  double u = 0.0;
  if (a.rng) {
    s1 = a.rng[2ll * row];
    s0 = a.rng[2ll * row + 1];
    u = rng_unit(s1, s0);
  }
  __syncthreads();
  if (nb > 0 && !mbar_wait_bounded(&sh.bar, 0)) {
    sh.load_fail = 1;
    raise_status(kErrLoadTimeout);
  }
  __syncthreads();
  // ---- repetition penalty in place, each distinct id once
  if (o.penalize) {
    for (int i = threadIdx.x; i < bwords; i += kThreads) bm[i] = 0;
    __syncthreads();
    const long long h0 = a.hist_off[row], h1 = a.hist_off[row + 1];
    const long long len = h1 - h0;
    const long long from = (o.repeat_last > 0 && len > o.repeat_last) ? len - o.repeat_last : 0;
    for (long long j = h0 + from + threadIdx.x; j < h1; j += kThreads) {
      const long long t = static_cast<long long>(a.hist[j]) - g_lo;
      if (t >= 0 && t < n) {
        const uint32_t bit = 1u << (t & 31);
        const uint32_t old = atomicOr(&bm[t >> 5], bit);
        if (!(old & bit)) v[t] = penalize(v[t], o.repeat);
      }
    }
    __syncthreads();
  }
  // Every column of the slice once: f(value, column).  The 16-byte aligned
  // body (from v + h) is read with 16-byte shared loads, 4 consecutive columns
  // per thread and step; each thread sees its columns in increasing order.
  // Every pass below is free of visiting order (integer sums, keyed minima,
  // gathered members sorted later).
  auto each = [&](auto&& f) {
    if (static_cast<int>(threadIdx.x) < h) f(v[threadIdx.x], static_cast<int>(threadIdx.x));
    const float4* v4 = reinterpret_cast<const float4*>(v + h);
    const int n4 = (n - h) >> 2;
    for (int q = threadIdx.x; q < n4; q += kThreads) {
      const float4 t = v4[q];
      const int j = h + 4 * q;
      f(t.x, j);
      f(t.y, j + 1);
      f(t.z, j + 2);
      f(t.w, j + 3);
    }
    for (int j = h + 4 * n4 + threadIdx.x; j < n; j += kThreads) f(v[j], j);
  };
  // ---- row maximum (smallest key) across the cluster
  // (float compares: `vj > bv` keeps the lowest column on ties and never
  // takes a NaN; a thread whose columns are all -inf/NaN keeps its first)
  float bv = -__int_as_float(0x7f800000);
  int bj = -1, first = -1;
  float lo_f = __int_as_float(0x7f800000);  // smallest finite value
  each([&](float vj, int j) {
    if (first < 0) first = j;
    if (vj > bv) {
      bv = vj;
      bj = j;
    }
    if (vj > -__int_as_float(0x7f800000)) lo_f = fminf(lo_f, vj);  // NaN and -inf fail; +inf kept
  });
  if (bj < 0) bj = first;
  uint64_t best = bj >= 0 ? dkey(bv, static_cast<uint32_t>(g_lo + bj)) : kNoKey;
  best = block_min<unsigned long long>(best, sh.ws64);
  lo_f = block_min<float>(lo_f, reinterpret_cast<float*>(sh.ws64));
  cluster_wait();
  if (threadIdx.x < static_cast<unsigned>(C)) {
    *cl.map_shared_rank(&sh.xmin[crank], threadIdx.x) = best;
    *cl.map_shared_rank(&sh.xlo[crank], threadIdx.x) = lo_f;
  }
  cluster_sync_all();
  uint64_t dmin = sh.xmin[0];
  float row_lo = sh.xlo[0];
  for (int i = 1; i < C; ++i) {
    dmin = sh.xmin[i] < dmin ? sh.xmin[i] : dmin;
    row_lo = fminf(row_lo, sh.xlo[i]);
  }
  if (crank == 0 && threadIdx.x == 0 && a.rng) {
    a.rng[2ll * row] = s1;
    a.rng[2ll * row + 1] = s0;
  }

  GenCtx x;
  x.v = v;
  x.n = n;
  x.g_lo = g_lo;
  x.idxbits = a.idxbits;
  x.nbits = 32 + a.idxbits;
  x.M = dval(dmin);
  x.inv_temp = o.inv_temp;
  x.fixbits = a.fixbits;
  x.xcut = -(a.fixbits + 1) * 0.6931471805599453;
  x.need_w = o.min_p > 0.0f;
  x.T = etab;
  x.C = C;
  x.crank = crank;
  x.kc0 = ((dmin >> 32) << a.idxbits) | (dmin & 0xffffffffull);
  int gseq = 0, gbuf = 0;
  const unsigned long long kAll = ~0ull;
  const unsigned long long idmask = (1ull << a.idxbits) - 1;

  // ---- top-k limit when 0 < top_k < vocab (k above the streaming kernel's range)
  unsigned long long klim = kAll;
  if (o.k < o.vocab) {
    select_weighted(x, false, static_cast<unsigned long long>(o.k), nullptr, kAll, 0.0, L, G, gb, gseq, gbuf, cl,
                    sh);
    if (sh.r_found) klim = sh.r_key;
  }
  const bool finite_max = isfinite(x.M);
  int out_id = 0;
  double s_sum = 0.0, s_tot = 0.0;
  int s_keep = 0;
  if (!finite_max) {
    // All candidate weights are NaN in the reference: it returns buf_[keep-1]
    // with keep = 1 under min-p and k otherwise (src/sampler.cpp:86-108).
    const unsigned long long pos = o.min_p > 0.0f ? 1ull : static_cast<unsigned long long>(o.k);
    select_weighted(x, false, pos, nullptr, klim, 0.0, L, G, gb, gseq, gbuf, cl, sh);
    out_id = sh.r_found ? static_cast<int>(sh.r_key & idmask) : 0;
    s_keep = static_cast<int>(pos);
    s_sum = s_tot = __longlong_as_double(0x7ff8000000000000ll);
  } else {
    const double thr = o.min_p > 0.0f ? static_cast<double>(o.min_p) : 0.0;  // pr[0] == 1
    VHist* Lv = reinterpret_cast<VHist*>(L);      // aliases L, G[0]
    VHist* Gv = reinterpret_cast<VHist*>(L + 2);  // aliases G[1], A
    VGath* vg = reinterpret_cast<VGath*>(gb);
    if (o.k < o.vocab) {  // the k-limit selection used these buffers
      for (int b = threadIdx.x; b < kGBins; b += kThreads)
        for (int i = 0; i < 4; ++i) {
          L[i].c[b] = 0;
          L[i].m[b] = 0;
        }
      cluster_sync_all();
    }
    // Value bins: bin(v) = floor((M - v) * kVBins / R), monotone in v, over the
    // row's value range R (capped where masses fall below e^-46).
    const float R = fminf(__fsub_rn(x.M, row_lo), 46.0f * o.temp);
    const float inv_w = R > 0.0f ? static_cast<float>(kVBins) / R : 0.0f;
    auto vbin = [&](float vv) -> int {
      const float d = __fsub_rn(x.M, canon(vv));
      return static_cast<int>(fminf(__fmul_rn(d, inv_w), static_cast<float>(kVBins - 1)));
    };
    // ---- mass pass: S over the k-set; (mass, count) of the min-p set per value bin
    // The bin masses accumulate as three 16-bit limbs in 32-bit shared counters
    // (Gv's bytes, zero here) and are folded into Lv->m after the pass: 32-bit
    // shared atomics are much cheaper than 64-bit ones.  No limb sum overflows:
    // the two low limbs add < 2^16 per column over a slice of <= 40960
    // columns, and a mass is < 2^(64 - bitlen(vocab)), so the high limb adds
    // < 2^(32 - bitlen(vocab)) per column over fewer than 2^bitlen(vocab).
    uint32_t* lm0 = reinterpret_cast<uint32_t*>(Gv);
    uint32_t* lm1 = lm0 + kVBins;
    uint32_t* lm2 = lm1 + kVBins;
    unsigned long long s_local = 0, z_local = 0;
    if (klim == kAll && !(thr > 0.0)) {
      // every column is in the k-set and the min-p set: no keys needed
      each([&](float vv, int) {
        double m;
        const unsigned long long qm = fixed_mass(x, vv, &m);
        if (qm == 0) {  // below the fixed-point resolution: counted, never drawn
          ++z_local;
          return;
        }
        s_local += qm;
        const int bi = vbin(vv);
        atomicAdd(&Lv->c[bi], 1u);
        atomicAdd(&lm0[bi], static_cast<uint32_t>(qm & 0xffffu));
        atomicAdd(&lm1[bi], static_cast<uint32_t>((qm >> 16) & 0xffffu));
        atomicAdd(&lm2[bi], static_cast<uint32_t>(qm >> 32));
      });
    } else {
      each([&](float vv, int j) {
        const unsigned long long kc = ckey(vv, static_cast<uint32_t>(g_lo + j), a.idxbits);
        if (kc > klim) return;
        double m;
        const unsigned long long qm = fixed_mass(x, vv, &m);
        s_local += qm;
        if (!in_pset(x, m, thr, kc)) return;
        if (qm == 0) {  // below the fixed-point resolution: counted, never drawn
          ++z_local;
          return;
        }
        const int bi = vbin(vv);
        atomicAdd(&Lv->c[bi], 1u);
        atomicAdd(&lm0[bi], static_cast<uint32_t>(qm & 0xffffu));
        atomicAdd(&lm1[bi], static_cast<uint32_t>((qm >> 16) & 0xffffu));
        atomicAdd(&lm2[bi], static_cast<uint32_t>(qm >> 32));
      });
    }
    __syncthreads();
    for (int b = threadIdx.x; b < kVBins; b += kThreads) {
      Lv->m[b] = static_cast<unsigned long long>(lm0[b]) + (static_cast<unsigned long long>(lm1[b]) << 16) +
                 (static_cast<unsigned long long>(lm2[b]) << 32);
      lm0[b] = 0u;
      lm1[b] = 0u;
      lm2[b] = 0u;
    }
    s_local = block_sum(s_local, sh.ws64);
    z_local = block_sum(z_local, sh.ws64);
    if (threadIdx.x == 0) {
      sh.my_sz[0] = s_local;
      sh.my_sz[1] = z_local;
    }
    // Pull model: every CTA reads all local histograms with plain DSMEM loads
    // (no remote atomics).  Lv stays untouched until every CTA has pulled it.
    cluster_sync_all();
    // all remote loads are issued before any is used (16-byte vectors; bins
    // b0, b0 + 1 are adjacent)
    const int b0 = 2 * threadIdx.x;
    unsigned long long m0 = 0, m1 = 0, S = 0, Z = 0;
    uint32_t c0 = 0, c1 = 0;
    // (S, Z): thread r pulls rank r's totals, warp 0 adds them up
    if (threadIdx.x < 32) {
      ulonglong2 sz = make_ulonglong2(0ull, 0ull);
      if (threadIdx.x < static_cast<unsigned>(C))
        sz = *reinterpret_cast<const ulonglong2*>(cl.map_shared_rank(sh.my_sz, threadIdx.x));
      sz.x = warp_sum(sz.x);
      sz.y = warp_sum(sz.y);
      if (threadIdx.x == 0) {
        sh.all_sz[0] = sz.x;
        sh.all_sz[1] = sz.y;
      }
    }
#pragma unroll
    for (int r0 = 0; r0 < kMaxCluster; r0 += 4) {
      ulonglong2 pm[4];
      uint2 pc[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (r0 + q < C) {
          const VHist* Lr = cl.map_shared_rank(Lv, r0 + q);
          pm[q] = *reinterpret_cast<const ulonglong2*>(&Lr->m[b0]);
          pc[q] = *reinterpret_cast<const uint2*>(&Lr->c[b0]);
        }
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (r0 + q < C) {
          m0 += pm[q].x;
          m1 += pm[q].y;
          c0 += pc[q].x;
          c1 += pc[q].y;
        }
      }
    }
    unsigned long long tm;
    uint32_t tc;
    const unsigned long long em = block_excl_scan(m0 + m1, sh.ws64, &tm);
    const uint32_t ec = block_excl_scan(c0 + c1, sh.ws32, &tc);
    S = sh.all_sz[0];  // written before the scans' barriers
    Z = sh.all_sz[1];
    // First bin whose running mass reaches t (>= 1, <= tm): bin, mass and count before it.
    auto vfind = [&](unsigned long long t, int* bin, unsigned long long* bm_, uint32_t* bc_, uint32_t* cnt,
                     unsigned long long* mass) {
      if (em < t && t <= em + m0) {
        sh.hf.bin = b0;
        sh.hf.before_m = em;
        sh.hf.before_c = ec;
        sh.hf.c = c0;
        sh.hf.m = m0;
      } else if (em + m0 < t && t <= em + m0 + m1) {
        sh.hf.bin = b0 + 1;
        sh.hf.before_m = em + m0;
        sh.hf.before_c = ec + c0;
        sh.hf.c = c1;
        sh.hf.m = m1;
      }
      __syncthreads();
      *bin = sh.hf.bin;
      *bm_ = sh.hf.before_m;
      *bc_ = sh.hf.before_c;
      *cnt = sh.hf.c;
      *mass = sh.hf.m;
      __syncthreads();
    };
    unsigned long long tp = 0;
    if (o.top_p > 0.0f && o.top_p < 1.0f) {
      const double t = ceil(static_cast<double>(o.top_p) * static_cast<double>(S));
      tp = t < 1.0 ? 1ull : static_cast<unsigned long long>(t);
      if (tp > tm) tp = 0;  // the min-p set ends before the top-p cutoff
    }
    // Members of the min-p set with positive fixed mass and a value bin (or
    // sub-bin) accepted by `pick` are gathered, as (key, mass), into the same
    // buffer of every CTA of the cluster; after the barrier every CTA sorts its
    // copy and walks it.  Returns the member count (or cap + 1 on overflow).
    auto gather = [&](auto pick, unsigned long long* gkey, unsigned long long* gmass, int cap) -> int {
      uint32_t* cnt0 = cl.map_shared_rank(&sh.gcount[gseq++], 0);
      each([&](float vv, int j) {
        if (!pick(vv)) return;  // (cheap test first; the key only for members)
        const unsigned long long kc = ckey(vv, static_cast<uint32_t>(g_lo + j), a.idxbits);
        if (kc > klim) return;
        double m;
        const unsigned long long qm = fixed_mass(x, vv, &m);
        if (!in_pset(x, m, thr, kc) || qm == 0) return;
        const uint32_t p = atomicAdd(cnt0, 1u);
        if (p < static_cast<uint32_t>(cap))
          for (int r = 0; r < C; ++r) {
            *cl.map_shared_rank(&gkey[p], r) = kc;
            *cl.map_shared_rank(&gmass[p], r) = qm;
          }
      });
      cluster_sync_all();
      if (threadIdx.x == 0) sh.ng = *cnt0;
      __syncthreads();
      const uint32_t got = sh.ng;
      __syncthreads();
      if (got > static_cast<uint32_t>(cap)) return cap + 1;
      return static_cast<int>(got);  // unsorted: resolve() orders what it needs
    };
    // Walks sorted members from running mass `cm`: index of the first whose
    // running mass reaches t, or -1.  Run by thread 0 only.
    auto walk = [&](const unsigned long long* gmass, int ng, unsigned long long cm, unsigned long long t,
                    unsigned long long* cm_out, int* steps) {
      for (int i = 0; i < ng; ++i) {
        cm += gmass[i];
        if (cm >= t) {
          *cm_out = cm;
          *steps = i + 1;
          return i;
        }
      }
      return -1;
    };
    // Among the gathered members (gkey, gmass)[0, ng) (unsorted) of value bin
    // `bin` (its refined sub-bin `sub` when >= 0), the first in key order at
    // which base + running mass reaches t (> base): sets sh.r_found, r_key,
    // r_cum_m (running mass including it) and r_steps (its rank + 1).  The
    // members go into kThreads sub-bins by value, monotone in key order (ties
    // share a sub-bin), by a histogram and one scan in Gv; only the target
    // sub-bin's members (at most 32) are sorted, by one warp.  A crowded
    // sub-bin (ties) sorts all members and walks them instead.
    auto resolve = [&](unsigned long long* gkey, unsigned long long* gmass, int ng, int bin, int sub,
                       unsigned long long base, unsigned long long t) {
      constexpr int NS = kThreads;
      unsigned long long* sm = Gv->m;  // [NS] masses
      uint32_t* sc = Gv->c;            // [NS] counts
      uint32_t* lst = Gv->c + NS;      // [32] members of the target sub-bin
      auto sbin = [&](unsigned long long kc) -> int {
        const float vv = unord32(~static_cast<uint32_t>(kc >> a.idxbits));
        float u = __fsub_rn(__fmul_rn(__fsub_rn(x.M, vv), inv_w), static_cast<float>(bin));
        if (sub >= 0) u = __fsub_rn(__fmul_rn(u, 1024.0f), static_cast<float>(sub));
        return min(NS - 1, max(0, static_cast<int>(__fmul_rn(u, static_cast<float>(NS)))));
      };
      sm[threadIdx.x] = 0;
      sc[threadIdx.x] = 0;
      if (threadIdx.x == 0) sh.ncrowd = 0;
      __syncthreads();
      for (int i = threadIdx.x; i < ng; i += kThreads) {
        const int b = sbin(gkey[i]);
        atomicAdd(&sc[b], 1u);
        atomicAdd(&sm[b], gmass[i]);
      }
      __syncthreads();
      const unsigned long long mm = sm[threadIdx.x];
      const uint32_t cc = sc[threadIdx.x];
      unsigned long long mt;
      uint32_t ct;
      const unsigned long long em = block_excl_scan(mm, sh.ws64, &mt);
      const uint32_t ec = block_excl_scan(cc, sh.ws32, &ct);
      const unsigned long long tt = t - base;
      if (threadIdx.x == 0) sh.hf.bin = -1;
      __syncthreads();
      if (em < tt && tt <= em + mm) {
        sh.hf.bin = threadIdx.x;
        sh.hf.before_m = em;
        sh.hf.before_c = ec;
        sh.hf.c = cc;
      }
      __syncthreads();
      const int sb = sh.hf.bin;
      const unsigned long long bm = sh.hf.before_m;
      const uint32_t bcnt = sh.hf.before_c, ns = sh.hf.c;
      __syncthreads();
      if (sb < 0) {  // the members' mass does not reach t
        if (threadIdx.x == 0) sh.r_found = 0;
        __syncthreads();
        return;
      }
      if (ns <= 32u) {
        for (int i = threadIdx.x; i < ng; i += kThreads)
          if (sbin(gkey[i]) == sb) {
            const uint32_t q = atomicAdd(&sh.ncrowd, 1u);
            if (q < 32u) lst[q] = static_cast<uint32_t>(i);
          }
        __syncthreads();
        if (threadIdx.x < 32) {
          const int lane = threadIdx.x;
          const bool have = lane < static_cast<int>(ns);
          unsigned long long k = have ? gkey[lst[lane]] : kNoKey;
          unsigned long long m = have ? gmass[lst[lane]] : 0ull;
#pragma unroll
          for (int kk = 2; kk <= 32; kk <<= 1) {
#pragma unroll
            for (int j = kk >> 1; j > 0; j >>= 1) {  // ascending bitonic sort by key, mass alongside
              const unsigned long long pk = __shfl_xor_sync(0xffffffffu, k, j);
              const unsigned long long pm = __shfl_xor_sync(0xffffffffu, m, j);
              const bool take_min = ((lane & j) == 0) == ((lane & kk) == 0);
              if (take_min ? (pk < k) : (pk > k)) {
                k = pk;
                m = pm;
              }
            }
          }
          const unsigned long long inc = warp_incl_scan(m);
          const unsigned hits = __ballot_sync(0xffffffffu, lane < static_cast<int>(ns) && bm + inc >= tt);
          const int L = hits ? __ffs(hits) - 1 : 0;
          const unsigned long long kL = __shfl_sync(0xffffffffu, k, L);
          const unsigned long long iL = __shfl_sync(0xffffffffu, inc, L);
          if (lane == 0) {
            sh.r_found = hits != 0;
            sh.r_key = kL;
            sh.r_cum_m = base + bm + iL;
            sh.r_steps = bcnt + static_cast<uint32_t>(L) + 1u;
          }
        }
        __syncthreads();
        return;
      }
      const int P = next_pow2(max(ng, 2));
      for (int i = ng + threadIdx.x; i < P; i += kThreads) {
        gkey[i] = kNoKey;
        gmass[i] = 0;
      }
      __syncthreads();
      sort_pairs(gkey, gmass, P);
      if (threadIdx.x == 0) {
        unsigned long long cm = 0;
        int st = 0;
        const int i = walk(gmass, ng, base, t, &cm, &st);
        sh.r_found = i >= 0;
        if (i >= 0) {
          sh.r_key = gkey[i];
          sh.r_cum_m = cm;
          sh.r_steps = static_cast<uint32_t>(st);
        }
      }
      __syncthreads();
    };
    // the cutoff gather lands in the local histogram's space (free after the push)
    // Buffers: the cutoff gather goes to vg (nobody pulls it); the draw gather
    // goes to the Lv bytes once every CTA has passed the cutoff barrier (and
    // so finished pulling Lv), else to vg; a sub-bin histogram goes to Gv.
    constexpr int kCutCap = kVGatherCap;
    unsigned long long* ckeys = vg->key;
    unsigned long long* cmass = vg->mass;
    bool exact = true;   // resolved without the radix fallback
    unsigned long long tot_m = tm;
    uint32_t keep_c = tc + static_cast<uint32_t>(Z);
    // Gv is read by every CTA before the next barrier; zero our copy now for a
    // possible sub-bin histogram (other CTAs push into it only after that barrier).
    const unsigned long long gm0 = m0, gm1 = m1;
    const uint32_t gc0 = c0, gc1 = c1;
    (void)gm0; (void)gm1; (void)gc0; (void)gc1;
    if (tp) {
      int bc;
      unsigned long long Bc, mc;
      uint32_t Cc, nc;
      vfind(tp, &bc, &Bc, &Cc, &nc, &mc);
      const int ng = gather([&](float vv) { return vbin(vv) == bc; }, ckeys, cmass, kCutCap);
      if (ng > kCutCap) {
        exact = false;
      } else {
        resolve(ckeys, cmass, ng, bc, -1, Bc, tp);
        if (!sh.r_found) exact = false;
        tot_m = sh.r_found ? sh.r_cum_m : 0;
        keep_c = Cc + (sh.r_found ? sh.r_steps : 0u);
        __syncthreads();
      }
    }
    unsigned long long klim_keep = klim;
    if (exact) {
      // ---- the draw: target bin from the (saved) running sums of the value histogram
      const double rt = ceil(u * static_cast<double>(tot_m));
      unsigned long long t = rt < 1.0 ? 1ull : static_cast<unsigned long long>(rt);
      if (t > tot_m) t = tot_m;
      // first bin whose running mass reaches t (from the registers of the scan)
      if (threadIdx.x == 0) sh.hf.bin = -1;
      __syncthreads();
      if (em < t && t <= em + gm0) {
        sh.hf.bin = b0;
        sh.hf.before_m = em;
        sh.hf.c = gc0;
      } else if (em + gm0 < t && t <= em + gm0 + gm1) {
        sh.hf.bin = b0 + 1;
        sh.hf.before_m = em + gm0;
        sh.hf.c = gc1;
      }
      __syncthreads();
      const int bd = sh.hf.bin;
      unsigned long long base = sh.hf.before_m;
      const uint32_t nd = sh.hf.c;
      __syncthreads();
      int sub = -1;  // refined sub-bin of bd, or -1 for the whole bin
      if (nd > static_cast<uint32_t>(kVGatherCap)) {
        // refine bin bd: 1024 sub-bins of its value interval, counted into Gv
        // (local), then pulled from every CTA like the value histogram
        VHist* Ls = Gv;
        for (int b = threadIdx.x; b < kVBins; b += kThreads) {
          Ls->c[b] = 0;
          Ls->m[b] = 0;
        }
        __syncthreads();
        each([&](float vv, int j) {
          if (vbin(vv) != bd) return;
          const unsigned long long kc = ckey(vv, static_cast<uint32_t>(g_lo + j), a.idxbits);
          if (kc > klim) return;
          double m;
          const unsigned long long qm = fixed_mass(x, vv, &m);
          if (!in_pset(x, m, thr, kc) || qm == 0) return;
          const float tt = __fmul_rn(__fsub_rn(x.M, canon(vv)), inv_w);
          const int sb = min(kVBins - 1, static_cast<int>(__fmul_rn(__fsub_rn(tt, static_cast<float>(bd)), 1024.0f)));
          atomicAdd(&Ls->c[sb], 1u);
          atomicAdd(&Ls->m[sb], qm);
        });
        cluster_sync_all();
        unsigned long long s0m = 0, s1m = 0;
        uint32_t s0c = 0, s1c = 0;
        for (int r = 0; r < C; ++r) {
          const VHist* Lr = cl.map_shared_rank(Ls, r);
          s0m += Lr->m[b0];
          s1m += Lr->m[b0 + 1];
          s0c += Lr->c[b0];
          s1c += Lr->c[b0 + 1];
        }
        unsigned long long stm;
        uint32_t stc;
        const unsigned long long sem = block_excl_scan(s0m + s1m, sh.ws64, &stm);
        (void)block_excl_scan(s0c + s1c, sh.ws32, &stc);
        const unsigned long long tt = t - base;
        if (threadIdx.x == 0) sh.hf.bin = -1;
        __syncthreads();
        if (sem < tt && tt <= sem + s0m) {
          sh.hf.bin = b0;
          sh.hf.before_m = sem;
          sh.hf.c = s0c;
        } else if (sem + s0m < tt && tt <= sem + s0m + s1m) {
          sh.hf.bin = b0 + 1;
          sh.hf.before_m = sem + s0m;
          sh.hf.c = s1c;
        }
        __syncthreads();
        sub = sh.hf.bin;
        base += sh.hf.before_m;
        if (sub < 0 || sh.hf.c > static_cast<uint32_t>(kVGatherCap)) exact = false;
        __syncthreads();
      }
      if (exact) {
        unsigned long long* dkeys = tp ? reinterpret_cast<unsigned long long*>(Lv) : vg->key;
        unsigned long long* dmass = tp ? dkeys + kVGatherCap : vg->mass;
        const int ng = gather(
            [&](float vv) {
              if (vbin(vv) != bd) return false;
              if (sub < 0) return true;
              const float tt = __fmul_rn(__fsub_rn(x.M, canon(vv)), inv_w);
              return min(kVBins - 1, static_cast<int>(__fmul_rn(__fsub_rn(tt, static_cast<float>(bd)), 1024.0f))) == sub;
            },
            dkeys, dmass, kVGatherCap);
        if (ng > kVGatherCap) {
          exact = false;
        } else {
          resolve(dkeys, dmass, ng, bd, sub, base, t);
          if (sh.r_found) out_id = static_cast<int>(sh.r_key & idmask);
          else exact = false;
          __syncthreads();
        }
      }
    }
    if (!exact) {
      // ---- crowded bins (ties, skewed rows): exact mass-weighted radix
      // selection over the keys
      cluster_sync_all();  // every CTA is done with the value-path buffers
      for (int b = threadIdx.x; b < kGBins; b += kThreads)
        for (int i = 0; i < 4; ++i) {
          L[i].c[b] = 0;
          L[i].m[b] = 0;
        }
      gbuf = 0;
      cluster_sync_all();
      tot_m = tm;
      keep_c = tc + static_cast<uint32_t>(Z);
      if (tp) {
        select_weighted(x, true, tp, nullptr, klim, thr, L, G, gb, gseq, gbuf, cl, sh);
        if (sh.r_found) {
          klim_keep = sh.r_key;
          tot_m = sh.r_cum_m;
          keep_c = sh.r_cum_c;
        }
      }
      const double rt = ceil(u * static_cast<double>(tot_m));
      unsigned long long target = rt < 1.0 ? 1ull : static_cast<unsigned long long>(rt);
      if (target > tot_m) target = tot_m;
      select_weighted(x, true, target, nullptr, klim_keep, thr, L, G, gb, gseq, gbuf, cl, sh);
      if (sh.r_found) {
        out_id = static_cast<int>(sh.r_key & idmask);
      } else {
        out_id = static_cast<int>(klim_keep & idmask);
        if (threadIdx.x == 0 && crank == 0) raise_status(kErrSelect);
      }
    }
    s_sum = ldexp(static_cast<double>(S), -x.fixbits);
    s_tot = ldexp(static_cast<double>(tot_m), -x.fixbits);
    s_keep = static_cast<int>(keep_c);
  }
  if (crank == 0 && threadIdx.x == 0) {
    a.out_ids[row] = out_id;
    ring_append(a, row, out_id);  // the cluster's CTAs read the ring only at the start
    if (a.stats) {
      const double nan = __longlong_as_double(0x7ff8000000000000ll);
      write_stats(a.stats + row, s_sum, s_tot, u, nan, nan, o.k, s_keep, out_id, 0);
    }
  }
  // keep shared memory alive until no CTA reads it, and no copy is in flight
  if (sh.load_fail && threadIdx.x == 0) (void)mbar_wait_bounded(&sh.bar, 0);
  cluster_sync_all();
}

__global__ void __launch_bounds__(kThreads, 2) general_kernel(const RowArgs a, const DevOpts o) {
  general_row(a, o, static_cast<int>(blockIdx.x) / a.cluster);
}

// The rows the streaming nucleus kernel listed as not settled (list[0, *count)),
// one cluster per row at a time: a small grid whose clusters take every
// (gridDim.x / cluster)-th listed row.
__global__ void __launch_bounds__(kThreads, 2) general_list_kernel(const RowArgs a, const DevOpts o, const int* list,
                                                                    const unsigned* count) {
  const unsigned n = *count;
  const unsigned step = gridDim.x / static_cast<unsigned>(a.cluster);
  for (unsigned i = blockIdx.x / static_cast<unsigned>(a.cluster); i < n; i += step) general_row(a, o, list[i]);
}

// ================================================================ launchers
size_t general_smem(int slice) {
  const size_t vwords = static_cast<size_t>(((slice + 4 + 3) / 4) * 4);
  const size_t bwords = static_cast<size_t>(((((slice >> 5) + 2) + 3) / 4) * 4);
  return (vwords + bwords) * 4 + 4 * sizeof(Hist) + 2 * sizeof(Gath) + 256 * sizeof(double);
}
static int next_pow2_host(int x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}
static size_t merge_smem(int n) {
  return static_cast<size_t>(next_pow2_host(n < 2 ? 2 : n)) * 16 + 3 * kSplitMaxK * 8;
}

template <class K, class A>
static cudaError_t launch_cluster(K kernel, const A& args, const DevOpts& o, int grid, int cluster, size_t smem,
                                  cudaStream_t s) {
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args, o);
}

cudaError_t launch_general(const RowArgs& a, const DevOpts& o, cudaStream_t s) {
  return launch_cluster(general_kernel, a, o, a.rows * a.cluster, a.cluster, general_smem(a.slice), s);
}

cudaError_t launch_general_list(const RowArgs& a, const DevOpts& o, const int* list, const unsigned* count,
                                int max_rows, cudaStream_t s) {
  const size_t smem = general_smem(a.slice);
  cudaError_t e =
      cudaFuncSetAttribute(general_list_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(std::min(max_rows, 32) * a.cluster);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = a.cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, general_list_kernel, a, o, list, count);
}

cudaError_t launch_merge(const MergeArgs& a, const DevOpts& o, cudaStream_t s) {
  const size_t sm = merge_smem(a.nshards * a.k);
  cudaError_t e = cudaFuncSetAttribute(merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sm));
  if (e != cudaSuccess) return e;
  merge_kernel<<<a.rows, kMergeThreads, sm, s>>>(a, o);
  return cudaGetLastError();
}

cudaError_t read_status(unsigned* st, bool clear, cudaStream_t s) {
  cudaError_t e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return e;
  e = cudaMemcpyFromSymbol(st, g_status, sizeof(unsigned));
  if (e != cudaSuccess) return e;
  if (clear && *st) {
    const unsigned z = 0;
    e = cudaMemcpyToSymbol(g_status, &z, sizeof(unsigned));
    if (e != cudaSuccess) return e;
  }
  unsigned st2 = 0;
  e = read_nucleus_status(&st2, clear);
  *st |= st2;
  return e;
}


// ================================================== split-row kernels (v2) ==
// One CTA of kSplitThreads per (row, slice of <= kSplitSlice columns), no
// thread-block clusters.  Each thread issues all of its 16-byte loads before
// using any (kSplitChunks in flight per thread), applies the penalty from a
// per-slice bitmap, and reduces its columns to a tiny partial result.  The
// slice publishes that partial to global scratch; the last CTA of the row to
// finish (a per-row atomic counter after a __threadfence, no waiting) merges
// the partials and finishes the row.  Nothing waits on another CTA, so other
// rows keep streaming while a row's merge runs.
namespace split {

constexpr int NT = kSplitThreads;
constexpr int NW = NT / 32;
constexpr int kBinsS = 2048;  // 11-bit digits of the candidate key
constexpr int kUnionCap = 2048;  // union of a row's candidates staged in the merge kernel
constexpr int kAugCap = 3 * kSliceCap;  // exact keys of the (at most 3) slices whose certificate failed
// The merge's room for those keys: k <= 64 needs one slice's worth (at most 3
// bad slices of at most 64 keys), larger k three; the smaller allocation keeps
// the merge's occupancy for the common k.
__host__ __device__ constexpr int aug_cap(uint32_t k) { return k <= 64u ? kSliceCap : kAugCap; }

struct Shared {
  unsigned long long ws64[NW];
  float offer[NW];  // each full warp's q-th largest lane maximum
  uint32_t ws32[NW];
  Found found;
  uint32_t ncand;
  int last;
  int incomplete;
  TailShared tail;
};

// Loads the thread's chunks of the slice into registers: chunk i covers slice
// columns 4*q .. 4*q+3 with q = threadIdx.x + i*NT.  Columns beyond n are
// left as NaN and never used (callers test j < n).
__device__ __forceinline__ void load_regs(const float* src, int n, float4 (&x)[kSplitChunks]) {
  const bool vec = (reinterpret_cast<uintptr_t>(src) & 15) == 0;
  const float4* s4 = reinterpret_cast<const float4*>(src);
  const float nan = __int_as_float(0x7fc00000);
  const int nfull = vec ? n / (4 * NT) : 0;  // chunks that are whole for every thread (block-uniform)
#pragma unroll
  for (int i = 0; i < kSplitChunks; ++i) {
    const int q = threadIdx.x + i * NT;
    const int j0 = 4 * q;
    if (i < nfull || (vec && j0 + 3 < n)) {
      x[i] = ld_stream(s4 + q);
    } else {
      x[i].x = j0 < n ? ld_stream1(src + j0) : nan;
      x[i].y = j0 + 1 < n ? ld_stream1(src + j0 + 1) : nan;
      x[i].z = j0 + 2 < n ? ld_stream1(src + j0 + 2) : nan;
      x[i].w = j0 + 3 < n ? ld_stream1(src + j0 + 3) : nan;
    }
  }
}

// The penalty mask of a thread: bit 4*i + c stands for slice column
// 4*(thread + i*NT) + c, the c-th value of the thread's chunk i.  One 64-bit
// word per thread, so most threads (no penalised column) test one word.
static_assert(4 * kSplitChunks <= 64, "penalty mask holds 4 bits per chunk");
__device__ __forceinline__ void mask_set(unsigned long long* pm, int j) {
  const int q = j >> 2;
  atomicOr(&pm[q % NT], 1ull << (4 * (q / NT) + (j & 3)));
}
// As mask_set; true for the one call that set the bit (a window may name a
// column twice).
__device__ __forceinline__ bool mask_set_first(unsigned long long* pm, int j) {
  const int q = j >> 2;
  const unsigned long long bit = 1ull << (4 * (q / NT) + (j & 3));
  return (atomicOr(&pm[q % NT], bit) & bit) == 0ull;
}
// Penalised columns left out of the thread's registers (set to -inf): their
// penalised values come from the threads that marked them.  Selects only.
__device__ __forceinline__ void exclude_regs(float4 (&x)[kSplitChunks], unsigned long long m) {
  if (m == 0) return;
  const float ninf = -__int_as_float(0x7f800000);
#pragma unroll
  for (int i = 0; i < kSplitChunks; ++i) {
    const uint32_t nib = static_cast<uint32_t>(m >> (4 * i)) & 15u;
    if (nib) {
      if (nib & 1u) x[i].x = ninf;
      if (nib & 2u) x[i].y = ninf;
      if (nib & 4u) x[i].z = ninf;
      if (nib & 8u) x[i].w = ninf;
    }
  }
}
__device__ __forceinline__ bool mask_test(const unsigned long long* pm, int j) {
  const int q = j >> 2;
  return (pm[q % NT] >> (4 * (q / NT) + (j & 3))) & 1ull;
}
__device__ __forceinline__ void penalize_regs(float4 (&x)[kSplitChunks], unsigned long long m, float rep) {
  if (m == 0) return;
#pragma unroll
  for (int i = 0; i < kSplitChunks; ++i) {
    const uint32_t nib = static_cast<uint32_t>(m >> (4 * i)) & 15u;
    if (nib) {
      if (nib & 1u) x[i].x = penalize(x[i].x, rep);
      if (nib & 2u) x[i].y = penalize(x[i].y, rep);
      if (nib & 4u) x[i].z = penalize(x[i].z, rep);
      if (nib & 8u) x[i].w = penalize(x[i].w, rep);
    }
  }
}

// Calls f(value, j) for every valid column of the thread's registers.
template <class F>
__device__ __forceinline__ void for_regs(const float4 (&x)[kSplitChunks], int n, F&& f) {
#pragma unroll
  for (int i = 0; i < kSplitChunks; ++i) {
    const int j0 = 4 * (threadIdx.x + i * NT);
    if (j0 < n) f(x[i].x, j0);
    if (j0 + 1 < n) f(x[i].y, j0 + 1);
    if (j0 + 2 < n) f(x[i].z, j0 + 2);
    if (j0 + 3 < n) f(x[i].w, j0 + 3);
  }
}

// The thread's best column by the reference's order (value descending, lowest
// column on ties) as a 64-bit key.  Float compares do the work: `v > best`
// keeps the first (lowest) column on ties, treats -0 == +0, and never selects
// a NaN, so NaN logits rank as -inf and the NaN placeholders beyond n are
// ignored.  A thread whose valid columns are all -inf/NaN yields its lowest
// valid column with the key of -inf.
__device__ __forceinline__ unsigned long long regs_best(const float4 (&x)[kSplitChunks], int n, long long g_lo) {
  const float ninf = -__int_as_float(0x7f800000);
  float bv = ninf;
  int bj = -1;
#pragma unroll
  for (int i = 0; i < kSplitChunks; ++i) {
    const int j0 = 4 * (threadIdx.x + i * NT);
    if (x[i].x > bv) { bv = x[i].x; bj = j0; }
    if (x[i].y > bv) { bv = x[i].y; bj = j0 + 1; }
    if (x[i].z > bv) { bv = x[i].z; bj = j0 + 2; }
    if (x[i].w > bv) { bv = x[i].w; bj = j0 + 3; }
  }
  if (bj < 0) {
    if (4 * static_cast<int>(threadIdx.x) >= n) return kNoKey;
    bj = 4 * threadIdx.x;
  }
  return dkey(bv, static_cast<uint32_t>(g_lo + bj));
}

// The largest of the thread's values; NaN (logits and the placeholders beyond
// n) is ignored, so a thread without a finite or infinite value yields -inf.
__device__ __forceinline__ float regs_max(const float4 (&x)[kSplitChunks]) {
  float m = -__int_as_float(0x7f800000);
#pragma unroll
  for (int i = 0; i < kSplitChunks; ++i) m = fmaxf(fmaxf(m, fmaxf(x[i].x, x[i].y)), fmaxf(x[i].z, x[i].w));
  return m;
}

// Descending bitonic sort of one non-NaN float per lane across the warp.
__device__ __forceinline__ float warp_sort_desc(float v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      const float p = __shfl_xor_sync(0xffffffffu, v, j);
      v = (((lane & j) == 0) == ((lane & k) == 0)) ? fmaxf(v, p) : fminf(v, p);
    }
  }
  return v;
}

// The q-th largest (1 <= q <= 32, duplicates counted) of one non-NaN value
// per lane.  Small q: q rounds of warp max reductions, each retiring the lanes
// that hold the maximum; larger q: a full 32-lane sort.
__device__ __forceinline__ float warp_qth_max(float v, uint32_t q) {
  if (q > 4u) return __shfl_sync(0xffffffffu, warp_sort_desc(v), static_cast<int>(q) - 1);
  uint32_t u = ord32(canon(v));  // > 0 for every non-NaN value; 0 marks a retired lane
  uint32_t seen = 0, mx;
  while (true) {
    mx = __reduce_max_sync(0xffffffffu, u);
    seen += __popc(__ballot_sync(0xffffffffu, u == mx));
    if (seen >= q) break;
    if (u == mx) u = 0;
  }
  return unord32(mx);
}

// First bin (of kBinsS counts, kBinsS / NT per thread) where the running
// count reaches target >= 1.
__device__ Found find_bins(const uint32_t* H, uint32_t target, Shared& sh) {
  constexpr int PER = kBinsS / NT;
  static_assert(PER % 4 == 0, "bins per thread must be a multiple of 4");
  if (threadIdx.x == 0) sh.found.bin = -1;
  uint32_t v[PER];
#pragma unroll
  for (int i = 0; i < PER / 4; ++i) {
    const uint4 q = reinterpret_cast<const uint4*>(H)[(PER / 4) * threadIdx.x + i];
    v[4 * i] = q.x;
    v[4 * i + 1] = q.y;
    v[4 * i + 2] = q.z;
    v[4 * i + 3] = q.w;
  }
  uint32_t s = 0;
#pragma unroll
  for (int i = 0; i < PER; ++i) s += v[i];
  uint32_t total;
  const uint32_t ex = block_excl_scan<uint32_t, NT>(s, sh.ws32, &total);
  if (ex < target && target <= ex + s) {
    uint32_t e = ex;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      if (target <= e + v[i]) {
        sh.found.bin = PER * threadIdx.x + i;
        sh.found.before = e;
        sh.found.cnt = v[i];
        break;
      }
      e += v[i];
    }
  }
  __syncthreads();
  const Found f = sh.found;
  __syncthreads();
  return f;
}

// Exact selection of the `k` smallest keys among those produced by `each`
// (which calls its argument with every candidate key of this thread): 11-bit
// radix passes with early exit.  Returns (prefix, shift) such that the
// selected set is {key : (key >> shift) <= prefix}.  H: kBinsS zeroed counts
// (left zeroed).  nbits: significant bits of the keys.
template <class Each>
__device__ __forceinline__ void radix_select(Each&& each, uint32_t k, int nbits, uint32_t* H, Shared& sh,
                             unsigned long long* prefix_out, int* shift_out) {
  unsigned long long prefix = 0;
  int resolved = 0;
  uint32_t krem = k;
  while (true) {
    const int shift = max(0, nbits - resolved - 11);
    const int width = nbits - resolved - shift;
    const unsigned long long mask = (1ull << width) - 1;
    const int hi = nbits - resolved;
    each([&](unsigned long long key) {
      if (resolved == 0 || (key >> hi) == prefix) atomicAdd(&H[(key >> shift) & mask], 1u);
    });
    __syncthreads();
    Found f = find_bins(H, krem, sh);
    for (int b = threadIdx.x; b < kBinsS; b += NT) H[b] = 0;
    if (f.bin < 0) {  // unreachable: the set holds at least k keys
      if (threadIdx.x == 0) raise_status(kErrSelect);
      f.bin = 0;
      f.before = 0;
      f.cnt = krem;
    }
    prefix = (prefix << width) | static_cast<unsigned long long>(f.bin);
    resolved += width;
    krem -= f.before;
    if (f.cnt == krem || shift == 0) {
      *prefix_out = prefix;
      *shift_out = shift;
      __syncthreads();
      return;
    }
  }
}

}  // namespace split

namespace split {

__device__ __forceinline__ unsigned long long to_ckey(unsigned long long d, int idxbits) {
  return ((d >> 32) << idxbits) | (d & 0xffffffffull);
}

// Marks in `pm` the columns [g_lo, g_lo + n) named by the row's penalty window
// read from the CSR history (the last repeat_last ids, src/sampler.cpp:58-64;
// ids outside the slice mark nothing).  Out of line: the dense-window path is
// the common one, and this one's 64-bit indexing stays out of its registers.
__device__ __noinline__ void mark_csr_window(const RowArgs& a, const DevOpts& o, int row, long long g_lo, int n,
                                             unsigned long long* pm) {
  const long long h0 = a.hist_off[row], h1 = a.hist_off[row + 1];
  const long long len = h1 - h0;
  const long long from = (o.repeat_last > 0 && len > o.repeat_last) ? len - o.repeat_last : 0;
  for (long long j = h0 + from + threadIdx.x; j < h1; j += NT) {
    const long long t = static_cast<long long>(a.hist[j]) - g_lo;
    if (t >= 0 && t < n) mask_set(pm, static_cast<int>(t));
  }
}

// Candidates a top-k slice must certainly hold: its whole top-kl, except in
// rows of C >= 2 slices with 32 <= k <= kSplitMaxK, where the top-m with
// m = max(kTopM, ceil(k / (C - 1)), ceil(k / 4)) suffices: C - 1 full slices
// give the union at least k keys, and a slice whose threshold is above the
// union's k-th value (it then holds m of the k best, so at most
// (k - 1) / m <= 3 slices can) is resolved exactly by the merge.
__device__ __forceinline__ uint32_t split_top_m(uint32_t k, int C, uint32_t kl) {
  if (C < 2 || k < 32u || k > static_cast<uint32_t>(kSplitMaxK)) return kl;
  const uint32_t per = (k + static_cast<uint32_t>(C) - 2u) / static_cast<uint32_t>(C - 1);
  const uint32_t quarter = (k + 3u) / 4u;
  return min(kl, max(max(static_cast<uint32_t>(kTopM), per), quarter));
}

// The exact top-kl of a slice by radix selection, for slices whose bound
// admits more than kSliceCap candidates (ties, masked rows).  Rare, so it
// re-reads the slice from L2 and stays out of line: the caller's register
// copy of the slice is dead by then and its budget is not shared.
template <bool kPen>
__device__ __noinline__ void slice_exact_topk(const RowArgs& a, const DevOpts& o, const float* src, int n,
                                              long long g_lo, uint32_t kl, const unsigned long long* pm,
                                              uint32_t* H, Shared& sh, unsigned long long* out) {
  for (int b = threadIdx.x; b < kBinsS; b += NT) H[b] = 0;
  __syncthreads();
  if (threadIdx.x == 0) sh.ncand = 0;
  unsigned long long prefix;
  int shift;
  const int nbits = 32 + a.idxbits;
  auto each_col = [&](auto f) {
    for (int j = threadIdx.x; j < n; j += NT) {
      float v = ld_stream1(src + j);
      if (kPen && mask_test(pm, j)) v = penalize(v, o.repeat);
      f(v, j);
    }
  };
  radix_select(
      [&](auto f) { each_col([&](float v, int j) { f(ckey(v, static_cast<uint32_t>(g_lo + j), a.idxbits)); }); },
      kl, nbits, H, sh, &prefix, &shift);
  each_col([&](float v, int j) {
    const uint32_t gid = static_cast<uint32_t>(g_lo + j);
    if ((ckey(v, gid, a.idxbits) >> shift) <= prefix) {
      const uint32_t p = atomicAdd(&sh.ncand, 1u);
      if (p < static_cast<uint32_t>(kSliceCap)) out[p] = dkey(v, gid);
    }
  });
}

template <int kMode, bool kPen, int kLZ>
__global__ void __launch_bounds__(NT, 4) split_kernel(const RowArgs a, const DevOpts o) {
  const int C = a.cluster;
  const int row = blockIdx.x / C;
  const int s = blockIdx.x - row * C;
  const int lo = s * a.slice;
  const int n = max(0, min(a.ncols - lo, a.slice));
  const float* src = a.logits + static_cast<long long>(row) * a.ld + lo;
  const long long g_lo = static_cast<long long>(a.col_off) + lo;
  extern __shared__ __align__(16) unsigned char smem[];
  uint32_t* H = reinterpret_cast<uint32_t*>(smem);  // kBinsS counts (top-k exact fallback)
  int* wids = reinterpret_cast<int*>(smem + (kMode == kSplitGreedy ? 0 : kBinsS * 4));  // the row's window
  __shared__ Shared sh;
  __shared__ unsigned long long pm[kPen ? NT : 1];  // penalty masks, one per thread

  // The merge grid may be scheduled once every CTA of this grid has started
  // or finished: released by the last wave only, so that its CTAs fill slots
  // no split CTA is waiting for.
  if (static_cast<int>(blockIdx.x) + a.first_wave >= static_cast<int>(gridDim.x)) grid_release();
  // The dense windows come from window_kernel, which this grid may overlap
  // (programmatic launch).  CTAs of the first wave put their logits loads in
  // flight first and then wait for it; later CTAs find it finished and send
  // the window out before the logits, so it is back when they are.
  float4 x[kSplitChunks];
  auto fetch_window = [&]() {
    grid_wait();
    const int* g = a.win + static_cast<long long>(row) * a.win_w;
    for (int c = threadIdx.x; c < (a.win_w >> 2); c += NT) cp_async16(wids + 4 * c, g + 4 * c);
    cp_async_commit();
  };
  if (kPen && a.win_w > 0) {
    if (static_cast<int>(blockIdx.x) < a.first_wave) {
      load_regs(src, n, x);
      fetch_window();
    } else {
      fetch_window();
      load_regs(src, n, x);
    }
  } else {
    load_regs(src, n, x);  // all logits loads in flight before anything else
  }
  if (threadIdx.x == 0) sh.ncand = 0;
  // Lazy penalty (top-k modes, dense windows of <= NT ids, one per thread):
  // the thread that marks a column first loads that column's value itself (its
  // line is already on its way for the owner), penalises it once and supplies
  // its key; owners only leave their marked columns out, so a warp no longer
  // runs the penalty's divisions for the few lanes that need them.  The top-k
  // kernels are issue bound and gain; greedy is bound by memory latency, and
  // the extra dependent load would lengthen it, so greedy, larger windows and
  // the CSR path penalise in the owners' registers.
  constexpr int LZ = kLZ;  // window ids a thread may own on the lazy path (windows of <= LZ * NT)
  const bool lazy = kPen && kMode != kSplitGreedy && a.win_w > 0 && a.win_w <= LZ * NT;
  int pj[LZ];       // the columns this thread penalises (lazy), slice-relative, or -1
  float pv[LZ];     // their values as loaded, then penalised
#pragma unroll
  for (int e = 0; e < LZ; ++e) {
    pj[e] = -1;
    pv[e] = 0.0f;
  }
  if (kPen) {
    pm[threadIdx.x] = 0;
    if (a.win_w > 0) cp_async_wait_all();
    __syncthreads();
    // the last repeat_last ids of the row's history (src/sampler.cpp:58-64);
    // ids outside [0, vocab) and the -1 padding mark nothing
    if (a.win_w > 0) {
      const int g = static_cast<int>(g_lo);  // global ids fit in int (vocab <= kMaxVocab)
      if (lazy) {
#pragma unroll
        for (int e = 0; e < LZ; ++e) {
          const int j = threadIdx.x + e * NT;
          const int id = j < a.win_w ? wids[j] : -1;
          if (id >= g && id - g < n && mask_set_first(pm, id - g)) {  // -1 padding and ids outside fail
            pj[e] = id - g;
            pv[e] = ld_stream1(src + pj[e]);
          }
        }
      } else {
        for (int j = threadIdx.x; j < a.win_w; j += NT) {
          const int id = wids[j];
          if (id >= g && id - g < n) mask_set(pm, id - g);
        }
      }
    } else {
      mark_csr_window(a, o, row, g_lo, n, pm);
    }
  }
  __syncthreads();
  if (kPen) {
    if (lazy) {
      exclude_regs(x, pm[threadIdx.x]);
    } else {
      penalize_regs(x, pm[threadIdx.x], o.repeat);
    }
  }
#pragma unroll
  for (int e = 0; e < LZ; ++e)
    if (pj[e] >= 0) pv[e] = penalize(pv[e], o.repeat);
  const long long slot = static_cast<long long>(row) * C + s;

  if (kMode == kSplitGreedy) {
    unsigned long long best = regs_best(x, n, g_lo);
    // std::max_element returns element 0 when it is NaN: key 0 beats every other key.
    if (g_lo == 0 && threadIdx.x == 0 && n > 0 && x[0].x != x[0].x) best = 0;
    best = block_min<unsigned long long, NT>(best, sh.ws64);
    if (threadIdx.x == 0) a.slice_keys[slot] = best;
  } else {
    const uint32_t k = kMode == kSplitEmit ? static_cast<uint32_t>(min(a.cand_k, a.ncols)) : static_cast<uint32_t>(o.k);
    const uint32_t kl = min(k, static_cast<uint32_t>(n));
    const uint32_t m = split_top_m(k, C, kl);  // the slice bounds its top-m (m == kl: its whole top-k)
    float thr = -__int_as_float(0x7f800000);   // published certificate; -inf: the full top-kl was emitted
    uint32_t count = 0;
    unsigned long long* out = a.slice_keys + slot * kSliceCap;
    if (kl > 0) {
      // Value bound T: every full warp (32 lanes holding columns) offers the
      // q-th largest of its lanes' maxima, q = ceil(m / full warps), and T is
      // the lowest offer.  Each full warp then has q distinct columns >= T, so
      // the slice has at least m, and its top-m by (value desc, column asc)
      // are all among the columns >= T.
      const int wfull = min(NW, ((n + 3) >> 2) >> 5);
      const uint32_t q = wfull > 0 ? (m + wfull - 1) / static_cast<uint32_t>(wfull) : 33u;
      bool all = q > 32u;
      float tv = -__int_as_float(0x7f800000);
      if (!all) {
        const float offer = warp_qth_max(regs_max(x), q);
        if ((threadIdx.x & 31) == 0 && (threadIdx.x >> 5) < wfull) sh.offer[threadIdx.x >> 5] = offer;
        __syncthreads();
        tv = sh.offer[0];
        for (int w = 1; w < wfull; ++w) tv = fminf(tv, sh.offer[w]);
        all = !(tv > -__int_as_float(0x7f800000));
      }
      // Candidates in one pass: a shared counter hands out the slots (their
      // order is immaterial: the merge selects by key).
      if (all) {
        if (n <= kSliceCap) {
          const unsigned long long mine = lazy ? pm[threadIdx.x] : 0ull;
          for_regs(x, n, [&](float v, int j) {
            const int q4 = j >> 2;  // owners skip the columns the lazy penalty supplies
            if (!((mine >> (4 * (q4 / NT) + (j & 3))) & 1ull))
              out[atomicAdd(&sh.ncand, 1u)] = dkey(v, static_cast<uint32_t>(g_lo + j));
          });
#pragma unroll
          for (int e = 0; e < LZ; ++e)
            if (pj[e] >= 0) out[atomicAdd(&sh.ncand, 1u)] = dkey(pv[e], static_cast<uint32_t>(g_lo + pj[e]));
        }
      } else {  // NaN placeholders beyond n never pass v >= tv
#pragma unroll
        for (int e = 0; e < LZ; ++e) {
          if (pj[e] >= 0 && canon(pv[e]) >= tv) {  // (excluded from the owner's registers)
            const uint32_t p = atomicAdd(&sh.ncand, 1u);
            if (p < static_cast<uint32_t>(kSliceCap)) out[p] = dkey(pv[e], static_cast<uint32_t>(g_lo + pj[e]));
          }
        }
        auto take = [&](float v, int j) {
          if (v >= tv) {
            const uint32_t p = atomicAdd(&sh.ncand, 1u);
            if (p < static_cast<uint32_t>(kSliceCap)) out[p] = dkey(v, static_cast<uint32_t>(g_lo + j));
          }
        };
#pragma unroll
        for (int i = 0; i < kSplitChunks; ++i) {
          const int j0 = 4 * (threadIdx.x + i * NT);
          take(x[i].x, j0);
          take(x[i].y, j0 + 1);
          take(x[i].z, j0 + 2);
          take(x[i].w, j0 + 3);
        }
      }
      __syncthreads();
      const uint32_t tot = (all && n > kSliceCap) ? ~0u : sh.ncand;
      if (tot <= static_cast<uint32_t>(kSliceCap)) {
        count = tot;
        if (m < kl && !all) thr = tv;  // only the top-m is certain: the merge checks thr
      } else {
        // more than kSliceCap candidates (ties, masked rows): exact top-kl
        slice_exact_topk<kPen>(a, o, src, n, g_lo, kl, pm, H, sh, out);
        count = kl;
      }
    }
    if (threadIdx.x == 0) {
      a.slice_count[slot] = count;
      if (kMode != kSplitGreedy) a.slice_thr[slot] = thr;
    }
  }

}

// Per-row merge of the slices' partial results, launched after split_kernel
// on the same stream (so it sees every slice's stores; nothing waits).
template <int kMode>
__global__ void __launch_bounds__(NT, 6) merge_slices_kernel(const RowArgs a, const DevOpts o) {
  const int C = a.cluster;
  const int row = blockIdx.x;
  extern __shared__ __align__(16) unsigned char smem[];
  uint32_t* H = reinterpret_cast<uint32_t*>(smem);        // kBinsS counts / fp64 tail scratch
  uint64_t* U = reinterpret_cast<uint64_t*>(H + kBinsS);  // kUnionCap keys
  __shared__ Shared sh;
  // The next call's first kernel may be scheduled now; it waits for this grid.
  grid_release();
  // The row's RNG state is not written by the split grid (and the previous
  // call's merge finished before this call's first kernel went past its
  // wait): read it before waiting.
  unsigned long long rng0 = 0, rng1 = 0;
  if (kMode == kSplitSample && threadIdx.x == 0) {
    rng0 = a.rng[2ll * row];
    rng1 = a.rng[2ll * row + 1];
  }
  grid_wait();  // the split grid's partials (programmatic launch)
  if (kMode == kSplitGreedy) {
    if (threadIdx.x < 32) {
      unsigned long long m = kNoKey;
      for (int i = threadIdx.x; i < C; i += 32) {
        const unsigned long long v = a.slice_keys[static_cast<long long>(row) * C + i];
        m = v < m ? v : m;
      }
      m = warp_min(m);
      if (threadIdx.x == 0) {
        const int id = static_cast<int>(did(m));
        a.out_ids[row] = id;
        ring_append(a, row, id);
        if (a.stats) write_stats(a.stats + row, 0.0, 0.0, 0.0, __longlong_as_double(0x7ff0000000000000ll),
                                 __longlong_as_double(0x7ff0000000000000ll), o.vocab, 1, id, 1);
      }
    }
    return;
  }
  const uint32_t k = kMode == kSplitEmit ? static_cast<uint32_t>(min(a.cand_k, a.ncols)) : static_cast<uint32_t>(o.k);
  __shared__ uint32_t soff[kMaxSlices + 1];
  // counts and certificates of the row's slices, loaded together
  const uint32_t ci = threadIdx.x < static_cast<unsigned>(C) ? __ldcg(&a.slice_count[static_cast<long long>(row) * C + threadIdx.x]) : 0u;
  const float my_thr = threadIdx.x < static_cast<unsigned>(C)
                           ? __ldcg(&a.slice_thr[static_cast<long long>(row) * C + threadIdx.x])
                           : -__int_as_float(0x7f800000);
  uint32_t utot;
  const uint32_t cex = block_excl_scan<uint32_t, NT>(ci, sh.ws32, &utot);
  if (threadIdx.x < static_cast<unsigned>(C)) {
    soff[threadIdx.x] = cex;
    soff[kMaxSlices] = 0;
  }
  __shared__ uint32_t scnt[kMaxSlices];
  if (threadIdx.x < static_cast<unsigned>(C)) scnt[threadIdx.x] = ci;
  if (threadIdx.x == 0) sh.ncand = 0;
  __syncthreads();
  const unsigned long long* base = a.slice_keys + static_cast<long long>(row) * C * kSliceCap;
  uint64_t* sel = reinterpret_cast<uint64_t*>(H) + 512;  // H bytes [4 KB, 8 KB); the tail uses [0, 6 KB)
  const bool in_smem = utot <= static_cast<uint32_t>(kUnionCap);
  if (in_smem) {
    // The union's keys spread evenly over the threads (key e of the union is
    // key e - soff[i] of slice i): at most kUnionCap / NT == 8 per thread,
    // all of them in flight at once.
    static_assert(kUnionCap == 8 * NT, "eight union keys per thread");
    unsigned long long v8[8];
    int sl = 0;  // the slice of the thread's current key; keys ascend, so do slices
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int e = threadIdx.x + q * NT;
      if (e < static_cast<int>(utot)) {
        while (sl + 1 < C && static_cast<int>(soff[sl + 1]) <= e) ++sl;
        v8[q] = __ldcg(base + static_cast<long long>(sl) * kSliceCap + (e - static_cast<int>(soff[sl])));
      }
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int e = threadIdx.x + q * NT;
      if (e < static_cast<int>(utot)) U[e] = v8[q];
    }
    __syncthreads();
  }
  uint64_t* cand = sel + kSliceCap;  // the k best, sorted (sel[kSliceCap, 2 kSliceCap))
  bool done = false;
  if (in_smem) {
    // The slices' bound once more, over the union: every full warp offers the
    // q-th largest of its lanes' best values, and the lowest offer bounds the
    // union's top-k from below.  Lanes own U[t], U[t + NT], ...
    float bv = -__int_as_float(0x7f800000);
    for (uint32_t e = threadIdx.x; e < utot; e += NT) bv = fmaxf(bv, dval(U[e]));
    const int wfull = min(NW, static_cast<int>(utot >> 5));
    const uint32_t q = wfull > 0 ? (k + wfull - 1) / static_cast<uint32_t>(wfull) : 33u;
    bool all = q > 32u;
    float tv = -__int_as_float(0x7f800000);
    if (!all) {
      const float srt = warp_sort_desc(bv);
      const float offer = __shfl_sync(0xffffffffu, srt, static_cast<int>(q) - 1);
      if ((threadIdx.x & 31) == 0 && (threadIdx.x >> 5) < wfull) sh.offer[threadIdx.x >> 5] = offer;
      __syncthreads();
      tv = sh.offer[0];
      for (int w = 1; w < wfull; ++w) tv = fminf(tv, sh.offer[w]);
      all = !(tv > -__int_as_float(0x7f800000));
    }
    const uint64_t* F = U;
    uint32_t m = utot;
    if (!all) {
      for (uint32_t e = threadIdx.x; e < utot; e += NT) {
        const uint64_t d = U[e];
        if (dval(d) >= tv) {
          const uint32_t p = atomicAdd(&sh.ncand, 1u);
          if (p < static_cast<uint32_t>(kSliceCap)) sel[p] = d;
        }
      }
      __syncthreads();
      F = sel;
      m = sh.ncand;
    }
    if (m <= static_cast<uint32_t>(NT)) {
      // rank by counting: keys are distinct, so each of the k best lands at its place
      if (threadIdx.x < m) {
        const uint64_t d = F[threadIdx.x];
        uint32_t r = 0;
        for (uint32_t j = 0; j < m; ++j) r += F[j] < d ? 1u : 0u;
        if (r < k) cand[r] = d;
      }
      __syncthreads();
      done = true;
    }
  }
  if (!done) {
    // rare: the k best of the union by radix selection, then sort only those
    unsigned long long prefix;
    int shift;
    const int nbits = 32 + a.idxbits;
    __syncthreads();  // everyone has read sh.ncand
    for (int b = threadIdx.x; b < kBinsS; b += NT) H[b] = 0;
    if (threadIdx.x == 0) sh.ncand = 0;
    __syncthreads();
    auto each = [&](auto f) {
      if (in_smem) {
        for (int e = threadIdx.x; e < static_cast<int>(utot); e += NT) f(to_ckey(U[e], a.idxbits));
      } else {
        for (int e = threadIdx.x; e < C * kSliceCap; e += NT) {
          const int i = e / kSliceCap, j = e - i * kSliceCap;
          if (j < static_cast<int>(scnt[i])) f(to_ckey(__ldcg(base + e), a.idxbits));
        }
      }
    };
    radix_select(each, k, nbits, H, sh, &prefix, &shift);
    auto take = [&](unsigned long long d) {
      if ((to_ckey(d, a.idxbits) >> shift) <= prefix) {
        const uint32_t p = atomicAdd(&sh.ncand, 1u);
        if (p < static_cast<uint32_t>(kSliceCap)) sel[p] = d;
      }
    };
    if (in_smem) {
      for (int e = threadIdx.x; e < static_cast<int>(utot); e += NT) take(U[e]);
    } else {
      for (int e = threadIdx.x; e < C * kSliceCap; e += NT) {
        const int i = e / kSliceCap, j = e - i * kSliceCap;
        if (j < static_cast<int>(scnt[i])) take(__ldcg(base + e));
      }
    }
    __syncthreads();
    const int P = next_pow2(max(static_cast<int>(k), 2));
    for (int i = static_cast<int>(k) + threadIdx.x; i < P; i += NT) sel[i] = kNoKey;
    __syncthreads();
    bitonic_sort_u64(sel, P);
    for (int i = threadIdx.x; i < static_cast<int>(k); i += NT) cand[i] = sel[i];
    __syncthreads();
  }
  // ---- certificates (split_top_m): a slice that emitted only its top-m is
  // settled when its threshold is at or below the k-th value found; else it
  // holds m of the k best and may hold more: its exact top-kl replaces its
  // partial (at most (k - 1) / m slices, at most kAugCap keys in all), and
  // the k best are selected again.
  __shared__ uint32_t nbad;
  __shared__ unsigned char isbad[kMaxSlices];
  const float vk = utot >= k ? dval(cand[k - 1]) : -__int_as_float(0x7f800000);
  if (threadIdx.x == 0) nbad = 0;
  if (threadIdx.x < static_cast<unsigned>(C)) isbad[threadIdx.x] = 0;
  __syncthreads();
  if (threadIdx.x < static_cast<unsigned>(C) && my_thr > vk) {
    isbad[threadIdx.x] = 1;
    atomicAdd(&nbad, 1u);
  }
  __syncthreads();
  if (nbad > 0) {
    uint64_t* aug = U + kUnionCap;
    __shared__ unsigned long long pmk[NT];  // the bad slice's penalty masks
    uint32_t naug = 0;
    for (int sl = 0; sl < C; ++sl) {
      if (!isbad[sl]) continue;
      const int lo = sl * a.slice;
      const int n = max(0, min(a.ncols - lo, a.slice));
      const long long g_lo = static_cast<long long>(a.col_off) + lo;
      const uint32_t kl = min(k, static_cast<uint32_t>(n));
      if (naug + kl > static_cast<uint32_t>(aug_cap(k))) {  // unreachable by the bound on bad slices
        if (threadIdx.x == 0) raise_status(kErrSelect);
        break;
      }
      pmk[threadIdx.x] = 0;
      __syncthreads();
      if (o.penalize) {  // the window, as the split kernels read it
        if (a.win_w > 0) {
          for (int j = threadIdx.x; j < a.win_w; j += NT) {
            const int id = a.win[static_cast<long long>(row) * a.win_w + j];
            const long long t = static_cast<long long>(id) - g_lo;
            if (id >= 0 && t >= 0 && t < n) mask_set(pmk, static_cast<int>(t));
          }
        } else {
          mark_csr_window(a, o, row, g_lo, n, pmk);
        }
      }
      __syncthreads();
      const float* src = a.logits + static_cast<long long>(row) * a.ld + lo;
      unsigned long long* dst = reinterpret_cast<unsigned long long*>(aug + naug);
      if (o.penalize) slice_exact_topk<true>(a, o, src, n, g_lo, kl, pmk, H, sh, dst);
      else slice_exact_topk<false>(a, o, src, n, g_lo, kl, pmk, H, sh, dst);
      __syncthreads();
      naug += kl;
    }
    // the k best of the settled slices' partials and the exact lists
    unsigned long long prefix;
    int shift;
    const int nbits = 32 + a.idxbits;
    for (int b = threadIdx.x; b < kBinsS; b += NT) H[b] = 0;
    if (threadIdx.x == 0) sh.ncand = 0;
    __syncthreads();
    auto each2 = [&](auto f) {
      for (int i = 0; i < C; ++i) {
        if (isbad[i]) continue;
        for (int j = threadIdx.x; j < static_cast<int>(scnt[i]); j += NT)
          f(to_ckey(in_smem ? U[soff[i] + j] : __ldcg(base + static_cast<long long>(i) * kSliceCap + j), a.idxbits));
      }
      for (int e = threadIdx.x; e < static_cast<int>(naug); e += NT) f(to_ckey(aug[e], a.idxbits));
    };
    radix_select(each2, k, nbits, H, sh, &prefix, &shift);
    auto take2 = [&](unsigned long long d) {
      if ((to_ckey(d, a.idxbits) >> shift) <= prefix) {
        const uint32_t p = atomicAdd(&sh.ncand, 1u);
        if (p < static_cast<uint32_t>(kSliceCap)) sel[p] = d;
      }
    };
    for (int i = 0; i < C; ++i) {
      if (isbad[i]) continue;
      for (int j = threadIdx.x; j < static_cast<int>(scnt[i]); j += NT)
        take2(in_smem ? U[soff[i] + j] : __ldcg(base + static_cast<long long>(i) * kSliceCap + j));
    }
    for (int e = threadIdx.x; e < static_cast<int>(naug); e += NT) take2(aug[e]);
    __syncthreads();
    const int P = next_pow2(max(static_cast<int>(k), 2));
    for (int i = static_cast<int>(k) + threadIdx.x; i < P; i += NT) sel[i] = kNoKey;
    __syncthreads();
    bitonic_sort_u64(sel, P);
    for (int i = threadIdx.x; i < static_cast<int>(k); i += NT) cand[i] = sel[i];
    __syncthreads();
  }
  if (kMode == kSplitEmit) {
    for (int i = threadIdx.x; i < a.cand_k; i += NT) {
      const long long at = static_cast<long long>(row) * a.cand_k + i;
      const bool ok = i < static_cast<int>(k);
      const float val = ok ? dval(cand[i]) : -__int_as_float(0x7f800000);
      const int id = ok ? static_cast<int>(did(cand[i])) : -1;
      if (a.cand_packed) {
        a.cand_packed[at] = make_uint2(__float_as_uint(val), static_cast<unsigned>(id));
      } else {
        a.cand_val[at] = val;
        a.cand_id[at] = id;
      }
    }
  } else {
    // H's first 4 KB and sel (the k best are in cand now) are free: fp64
    // scratch of the tail, ending where cand starts
    double* pr = reinterpret_cast<double*>(H);
    static_assert(3 * kSplitMaxK * sizeof(double) == 512 * sizeof(uint64_t) + kSliceCap * sizeof(uint64_t),
                  "the tail's scratch is H bytes [0, 6 KB)");
    tail_pick(cand, static_cast<int>(k), o, a.rng + 2ll * row, rng0, rng1, a.out_ids + row,
              a.stats ? a.stats + row : nullptr, pr, pr + kSplitMaxK, pr + 2 * kSplitMaxK, &sh.tail);
    if (threadIdx.x == 0) ring_append(a, row, a.out_ids[row]);  // written by this thread in tail_pick
  }
}


}  // namespace split

static size_t round256(size_t b) { return (b + 255) & ~static_cast<size_t>(255); }
SplitScratch split_scratch_layout(long long rows, int slices, bool greedy, int win_w) {
  SplitScratch l;
  l.off_keys = round256(static_cast<size_t>(rows) * slices * 4);
  l.off_thr = l.off_keys + round256(static_cast<size_t>(rows) * slices * (greedy ? 1 : kSliceCap) * 8);
  l.off_win = l.off_thr + (greedy ? 0 : round256(static_cast<size_t>(rows) * slices * 4));
  l.bytes = l.off_win + static_cast<size_t>(rows) * win_w * 4;
  return l;
}
void split_scratch_attach(RowArgs& a, void* base, const SplitScratch& l, int win_w) {
  char* b = static_cast<char*>(base);
  a.slice_count = reinterpret_cast<unsigned*>(b);
  a.slice_keys = reinterpret_cast<unsigned long long*>(b + l.off_keys);
  a.slice_thr = reinterpret_cast<float*>(b + l.off_thr);
  a.win = win_w > 0 ? reinterpret_cast<int*>(b + l.off_win) : nullptr;
  a.win_w = win_w;
}
int split_window_width(const DevOpts& o) {
  if (!o.penalize || o.repeat_last <= 0 || o.repeat_last > kWinMax) return 0;
  return (o.repeat_last + 3) & ~3;
}
// Accepts skip + n ids into one stream's ring, of which only the last n
// (ids[0, n), n <= ring_len) are stored: the j-th id accepted by the stream
// occupies slot j mod ring_len, so the ring always holds the last ring_len.
__global__ void __launch_bounds__(256) ring_accept_kernel(int* win, int win_w, int ring_len, long long* pos, int row,
                                                          const int* ids, int n, int skip) {
  const long long p = pos[row] + skip;
  int* w = win + static_cast<long long>(row) * win_w;
  for (int i = threadIdx.x; i < n; i += 256) w[(p + i) % ring_len] = ids[i];
  __syncthreads();
  if (threadIdx.x == 0) pos[row] = p + n;
}
cudaError_t launch_ring_accept(int* win, int win_w, int ring_len, long long* pos, int row, const int* ids, int n,
                               int skip, cudaStream_t s) {
  ring_accept_kernel<<<1, 256, 0, s>>>(win, win_w, ring_len, pos, row, ids, n, skip);
  return cudaGetLastError();
}

// Per-row sampler state moved to new rows: row r of the output takes row
// from[r] of the input (RNG state, penalty ring and its position).  One CTA
// per output row.
__global__ void __launch_bounds__(256) state_gather_kernel(const int* from, int n, const unsigned long long* rng_in,
                                                           unsigned long long* rng_out, const int* win_in, int* win_out,
                                                           int win_w, const long long* pos_in, long long* pos_out) {
  const int r = blockIdx.x;
  if (r >= n) return;
  const int f = from[r];
  const int* src = win_in + static_cast<long long>(f) * win_w;
  int* dst = win_out + static_cast<long long>(r) * win_w;
  for (int i = threadIdx.x; i < win_w; i += 256) dst[i] = src[i];
  if (threadIdx.x == 0) {
    rng_out[2ll * r] = rng_in[2ll * f];
    rng_out[2ll * r + 1] = rng_in[2ll * f + 1];
    pos_out[r] = pos_in[f];
  }
}
cudaError_t launch_state_gather(const int* from, int n, const unsigned long long* rng_in, unsigned long long* rng_out,
                                const int* win_in, int* win_out, int win_w, const long long* pos_in,
                                long long* pos_out, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  state_gather_kernel<<<n, 256, 0, s>>>(from, n, rng_in, rng_out, win_in, win_out, win_w, pos_in, pos_out);
  return cudaGetLastError();
}

namespace split {
// Copies each row's penalty window (its last repeat_last history ids,
// src/sampler.cpp:58-64) into win[row][0, win_w), padded with -1.
__global__ void __launch_bounds__(256) window_kernel(const RowArgs a, const DevOpts o) {
  // Launched with programmatic serialization after whatever precedes it: wait
  // for that grid (e.g. the previous call's merge, which still reads the
  // scratch this call rewrites) before anything else, then let the split grid
  // start its logits loads.
  grid_wait();
  grid_release();
  const int row = blockIdx.x;
  const long long h0 = a.hist_off[row], h1 = a.hist_off[row + 1];
  const long long len = h1 - h0;
  const long long from = (o.repeat_last > 0 && len > o.repeat_last) ? len - o.repeat_last : 0;
  const long long st = h0 + from, wl = len - from;  // wl <= repeat_last <= win_w
  int* d = a.win + static_cast<long long>(row) * a.win_w;
  for (int j = threadIdx.x; j < a.win_w; j += 256) d[j] = j < wl ? a.hist[st + j] : -1;
}
}  // namespace split

// CTAs of the split kernel resident at once (SM count x CTAs per SM), looked
// up once per device and instantiation.
template <int kMode, bool kPen, int kLZ>
static cudaError_t split_first_wave(size_t smem, int* out) {
  static std::mutex mu;
  static int cache[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(mu);
  if (!cache[dev]) {
    int sms = 0, occ = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, split::split_kernel<kMode, kPen, kLZ>, split::NT, smem);
    if (e != cudaSuccess) return e;
    cache[dev] = sms * (occ > 0 ? occ : 1);
  }
  *out = cache[dev];
  return cudaSuccess;
}

// Launch with programmatic stream serialisation: the kernel may start while
// the previous kernel on the stream (one of ours, released by it) still runs,
// and waits for it with grid_wait where it needs its results.
template <class... P, class... A>
static cudaError_t launch_after(void (*k)(P...), int grid, int block, size_t smem, cudaStream_t s, A&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, std::forward<A>(args)...);
}

// kLZ: window ids each thread may penalise lazily (top-k modes; see split_kernel)
template <int kMode, bool kPen, int kLZ>
static cudaError_t launch_split_lz(const RowArgs& a0, const DevOpts& o, cudaStream_t s) {
  RowArgs a = a0;
  const bool windows = kPen && a.win_w > 0;
  const size_t sm = (kMode == kSplitGreedy ? 0 : split::kBinsS * 4) + (windows ? a.win_w * 4 : 0);
  cudaError_t e = split_first_wave<kMode, kPen, kLZ>(sm, &a.first_wave);
  if (e != cudaSuccess) return e;
  const int grid = a.rows * a.cluster;
  if (windows && !a.ring_pos) {  // batched streams keep their windows in place
    // programmatic launch: scheduled while the previous kernel drains, it
    // waits for it before touching memory
    e = launch_after(split::window_kernel, a.rows, 256, 0, s, a, o);
    if (e != cudaSuccess) return e;
    e = launch_after(split::split_kernel<kMode, kPen, kLZ>, grid, split::NT, sm, s, a, o);
  } else {
    split::split_kernel<kMode, kPen, kLZ><<<grid, split::NT, sm, s>>>(a, o);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) return e;
  // the per-row merge runs after every slice of the batch (same stream)
  if (kMode == kSplitGreedy) return launch_after(split::merge_slices_kernel<kMode>, a.rows, 32, 0, s, a, o);
  const uint32_t kk = kMode == kSplitEmit ? static_cast<uint32_t>(std::min(a.cand_k, a.ncols)) : static_cast<uint32_t>(o.k);
  return launch_after(split::merge_slices_kernel<kMode>, a.rows, split::NT,
                      static_cast<size_t>(split::kBinsS * 4 + (split::kUnionCap + split::aug_cap(kk)) * 8), s, a, o);
}
template <int kMode, bool kPen>
static cudaError_t launch_split_t(const RowArgs& a, const DevOpts& o, cudaStream_t s) {
  // windows of 257..1024 ids: four per thread on the lazy path (their register
  // cost would slow the common windows of <= 256 ids)
  if constexpr (kPen && kMode != kSplitGreedy) {
    if (a.win_w > split::NT && a.win_w <= 4 * split::NT) return launch_split_lz<kMode, kPen, 4>(a, o, s);
  }
  return launch_split_lz<kMode, kPen, 1>(a, o, s);
}
cudaError_t launch_split(const RowArgs& a, const DevOpts& o, int mode, cudaStream_t s) {
  switch (mode * 2 + (o.penalize ? 1 : 0)) {
    case 0: return launch_split_t<kSplitGreedy, false>(a, o, s);
    case 1: return launch_split_t<kSplitGreedy, true>(a, o, s);
    case 2: return launch_split_t<kSplitSample, false>(a, o, s);
    case 3: return launch_split_t<kSplitSample, true>(a, o, s);
    case 4: return launch_split_t<kSplitEmit, false>(a, o, s);
    default: return launch_split_t<kSplitEmit, true>(a, o, s);
  }
}

// ================================================ allocation-free scratch ==
// Scratch for verbo_cuda_sample_noalloc: a fixed array in the library's own
// device image instead of memory from cudaMalloc.  Every device that loads the
// library holds these kNoAllocScratchBytes until the process exits.  All calls
// share it and it keeps the last call's contents; calls that overlap on the
// GPU (different streams, or several host threads) race on it.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// The array's device address on the current device.  Host code cannot use the
// symbol itself (that is a host-side stand-in, not a device address), so the
// address is looked up with cudaGetSymbolAddress, with the device current, on
// every call: the lookup allocates nothing once the module is loaded, and a
// fresh lookup stays right after cudaDeviceReset recreates the context.  The
// first lookup on a device loads the library's module there (CUDA loads
// modules lazily): the array and the kernels' code are placed in device memory
// at that moment.
static cudaError_t noalloc_scratch_address(void** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess) return e;
  *out = p;
  return cudaSuccess;
}

cudaError_t launch_split_noalloc(RowArgs& a, const DevOpts& o, int mode, cudaStream_t s, bool* too_big) {
  const int win_w = split_window_width(o);
  const SplitScratch l = split_scratch_layout(a.rows, a.cluster, mode == kSplitGreedy, win_w);
  *too_big = l.bytes > kNoAllocScratchBytes;
  if (*too_big) return cudaSuccess;
  void* base = nullptr;
  cudaError_t e = noalloc_scratch_address(&base);
  if (e != cudaSuccess) return e;
  // Nothing in the scratch has to start at zero: the window kernel and each
  // slice write what the later kernels of the same call read, so the previous
  // call's contents are simply overwritten.
  split_scratch_attach(a, base, l, win_w);
  return launch_split(a, o, mode, s);
}
}  // namespace vb
