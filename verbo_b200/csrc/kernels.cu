// sm_100a kernels of the token-sampling path: a drop-in for the per-row work
// of verbo's Sampler::pick (src/sampler.cpp:50-109).
//
// Every kernel runs one thread-block cluster per logits row (or shard row):
// the row's columns are split into `cluster` contiguous slices, one per CTA,
// and the CTAs combine results through distributed shared memory (DSMEM).
//
//   greedy_kernel   temp <= 0.  One streaming pass: penalty from a per-slice
//                   bitmap, then the minimum of the 64-bit candidate key
//                   (= argmax with lowest-index ties, sampler.cpp:66-70).
//   topk_kernel     0 < top_k <= 1024.  One streaming pass keeping each
//                   thread's 4 best keys; a cluster-wide histogram of the
//                   thread maxima bounds the top-k from below; the candidates
//                   above the bound go to CTA 0, which sorts them and runs the
//                   reference's softmax / min-p / top-p / draw sequence in the
//                   same fp64 order (sampler.cpp:79-108).  If a thread could
//                   hold more than 4 candidates, the cluster instead runs an
//                   exact radix select by re-reading the row.  With `emit` it
//                   writes a shard's sorted top-k instead of sampling.
//   general_kernel  top_k == 0 (or > 1024, or >= vocab).  The slice is staged
//                   in shared memory with bulk async copies; the full-vocab
//                   softmax mass, min-p set, top-p cutoff and the draw are
//                   found by mass-weighted radix selection over the keys,
//                   with masses accumulated in 64-bit fixed point (exact and
//                   order-independent).  No full sort.
//   merge_kernel    merges per-shard candidates and runs the same tail as
//                   topk_kernel.
#include "device.cuh"
#include "kernels.cuh"

namespace vb {

__device__ unsigned int g_status;

__device__ __forceinline__ void raise_status(unsigned bits) { atomicOr(&g_status, bits); }

// xoroshiro128+ draw, Sampler::unit (src/sampler.cpp:33-41).
__device__ __forceinline__ double rng_unit(unsigned long long& s1_io, unsigned long long& s0_io) {
  unsigned long long s1 = s1_io;
  const unsigned long long s0 = s0_io;
  const unsigned long long r = s0 + s1;
  s1_io = s0;
  s1 ^= s1 << 23;
  s0_io = s1 ^ s0 ^ (s1 >> 18) ^ (s0 >> 5);
  return __dmul_rn(static_cast<double>(r >> 11), 1.0 / 9007199254740992.0);
}

// Penalty window of one row (src/sampler.cpp:53-57) marked in a bitmap over
// the slice [g_lo, g_lo + n) of global columns.
__device__ void build_bitmap(uint32_t* bm, int nwords, const RowArgs& a, const DevOpts& o, int row, long long g_lo,
                             int n) {
  for (int i = threadIdx.x; i < nwords; i += kThreads) bm[i] = 0;
  __syncthreads();
  const long long h0 = a.hist_off[row], h1 = a.hist_off[row + 1];
  const long long len = h1 - h0;
  const long long from = (o.repeat_last > 0 && len > o.repeat_last) ? len - o.repeat_last : 0;
  for (long long j = h0 + from + threadIdx.x; j < h1; j += kThreads) {
    const long long t = static_cast<long long>(a.hist[j]) - g_lo;
    if (t >= 0 && t < n) atomicOr(&bm[t >> 5], 1u << (t & 31));
  }
  __syncthreads();
}

template <bool kPen, class F>
__device__ __forceinline__ void consume4(float4 x, int j0, const uint32_t* bm, float rep, F& f) {
  if (kPen) {
    const uint32_t nib = (bm[j0 >> 5] >> (j0 & 31)) & 15u;
    if (nib) {
      if (nib & 1u) x.x = penalize(x.x, rep);
      if (nib & 2u) x.y = penalize(x.y, rep);
      if (nib & 4u) x.z = penalize(x.z, rep);
      if (nib & 8u) x.w = penalize(x.w, rep);
    }
  }
  f(x.x, j0);
  f(x.y, j0 + 1);
  f(x.z, j0 + 2);
  f(x.w, j0 + 3);
}

// Calls f(value_after_penalty, j) for each column j of the slice [0, n) that
// this thread owns.  16-byte loads with 4 in flight per thread when the slice
// start is 16-byte aligned; scalar loads otherwise and for the ragged tail.
template <bool kPen, class F>
__device__ __forceinline__ void stream_slice(const float* src, int n, const uint32_t* bm, float rep, F&& f) {
  const bool vec = (reinterpret_cast<uintptr_t>(src) & 15) == 0;
  const int nq = vec ? (n >> 2) : 0;
  const float4* s4 = reinterpret_cast<const float4*>(src);
  int q = threadIdx.x;
  for (; q + 3 * kThreads < nq; q += 4 * kThreads) {
    float4 x[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) x[u] = ld_stream(s4 + q + u * kThreads);
#pragma unroll
    for (int u = 0; u < 4; ++u) consume4<kPen>(x[u], 4 * (q + u * kThreads), bm, rep, f);
  }
  for (; q < nq; q += kThreads) consume4<kPen>(ld_stream(s4 + q), 4 * q, bm, rep, f);
  for (int j = 4 * nq + threadIdx.x; j < n; j += kThreads) {
    float v = ld_stream1(src + j);
    if (kPen && ((bm[j >> 5] >> (j & 31)) & 1u)) v = penalize(v, rep);
    f(v, j);
  }
}

__device__ __forceinline__ void write_stats(verbo_row_stats* st, double sum, double tot, double u, double dm,
                                            double cm, int k, int keep, int id, int greedy) {
  st->sum = sum;
  st->tot = tot;
  st->u = u;
  st->draw_margin = dm;
  st->cut_margin = cm;
  st->k = k;
  st->keep = keep;
  st->id = id;
  st->greedy = greedy;
}

// ===================================================================== greedy
template <bool kPen>
__global__ void __launch_bounds__(kThreads) greedy_kernel(const RowArgs a, const DevOpts o) {
  cg::cluster_group cl = cg::this_cluster();
  const int C = a.cluster;
  const int crank = static_cast<int>(cl.block_rank());
  const int row = blockIdx.x / C;
  const int lo = crank * a.slice;
  const int n = max(0, min(a.ncols - lo, a.slice));
  const float* src = a.logits + static_cast<long long>(row) * a.ld + lo;
  const long long g_lo = static_cast<long long>(a.col_off) + lo;

  extern __shared__ __align__(16) uint32_t bm[];
  __shared__ uint64_t slot[kMaxCluster];
  __shared__ uint64_t ws[kWarps];

  cluster_arrive();
  if (kPen)
    build_bitmap(bm, (a.slice >> 5) + 2, a, o, row, g_lo, n);
  uint64_t best = kNoKey;
  stream_slice<kPen>(src, n, bm, o.repeat, [&](float v, int j) {
    const uint64_t d = dkey(v, static_cast<uint32_t>(g_lo + j));
    best = d < best ? d : best;
  });
  best = block_min(best, ws);
  cluster_wait();
  if (threadIdx.x == 0) *cl.map_shared_rank(&slot[crank], 0) = best;
  cluster_sync_all();
  if (crank == 0 && threadIdx.x == 0) {
    uint64_t m = slot[0];
    for (int i = 1; i < C; ++i) m = slot[i] < m ? slot[i] : m;
    int id = static_cast<int>(did(m));
    // std::max_element keeps element 0 when it is NaN (nothing compares above it).
    float v0 = src[0];
    if (kPen && ((bm[0] & 1u) != 0)) v0 = penalize(v0, o.repeat);
    if (v0 != v0) id = 0;
    a.out_ids[row] = id;
    if (a.stats) write_stats(a.stats + row, 0.0, 0.0, 0.0, __longlong_as_double(0x7ff0000000000000ll),
                             __longlong_as_double(0x7ff0000000000000ll), o.vocab, 1, id, 1);
  }
}

// ======================================================== shared tail (top-k)
struct TailShared {
  double sum;
  int keep;
};

// Softmax, min-p, top-p and the inverse-CDF draw over the k best candidates
// sorted in the reference order (src/sampler.cpp:79-108).  The exps run in
// parallel; every sum runs in one thread in the reference's order with
// correctly rounded fp64 operations, so the result is the reference's
// whenever the fp64 exp agrees.  pr, q: >= k doubles of shared scratch.
__device__ void tail_pick(const uint64_t* c, int k, const DevOpts& o, unsigned long long* rng, int* out_id,
                          verbo_row_stats* st, double* pr, double* q, TailShared* ts) {
  const float mx = dval(c[0]);
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    const float v = dval(c[i]);
    pr[i] = exp(__ddiv_rn(static_cast<double>(__fsub_rn(v, mx)), static_cast<double>(o.temp)));
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double sum = 0.0;
    for (int i = 0; i < k; ++i) sum = __dadd_rn(sum, pr[i]);
    int keep = k;
    if (o.min_p > 0.0f) {
      const double thr = __dmul_rn(pr[0], static_cast<double>(o.min_p));
      keep = 1;
      while (keep < k && pr[keep] >= thr) ++keep;
    }
    ts->sum = sum;
    ts->keep = keep;
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
    int i = 0;
    for (; i < keep; ++i) {
      prev = acc;
      acc = __dadd_rn(acc, q[i]);
      if (acc >= tp) break;
    }
    if (i < keep) {
      cut = fmin(cut, acc - tp);
      if (i > 0) cut = fmin(cut, tp - prev);
    } else {
      cut = fmin(cut, tp - acc);
    }
    keep = keep < i + 1 ? keep : i + 1;
  }
  double tot = 0.0;
  for (int i = 0; i < keep; ++i) tot = __dadd_rn(tot, pr[i]);
  unsigned long long s1 = rng[0], s0 = rng[1];
  const double u = rng_unit(s1, s0);
  rng[0] = s1;
  rng[1] = s0;
  double r = __dmul_rn(u, tot);
  const double r0 = r;
  int pick = keep - 1;
  for (int i = 0; i < keep; ++i) {
    r = __dsub_rn(r, pr[i]);
    if (r <= 0.0) {
      pick = i;
      break;
    }
  }
  const int id = static_cast<int>(did(c[pick]));
  *out_id = id;
  if (st) {
    double below = 0.0;
    for (int i = 0; i < pick; ++i) below += pr[i];
    double m = inf;
    if (pick > 0) m = fmin(m, r0 - below);
    if (pick < keep - 1) m = fmin(m, below + pr[pick] - r0);
    write_stats(st, sum, tot, u, m / tot, cut, k, keep, id, 0);
  }
}

// ====================================================================== top-k
constexpr int kBins = 2048;  // 11-bit radix digits (4 per thread)
constexpr int kDig = 11;

struct Found {
  int bin;
  uint32_t before;
  uint32_t cnt;
};

struct TopkShared {
  uint32_t count;  // candidates reserved in CTA 0's buffer
  uint32_t flag;   // some thread may have dropped a candidate
  uint32_t c_total, c_flag;
  Found found;
  uint32_t ws[kWarps];
  uint64_t ws64[kWarps];
  TailShared tail;
};

// First bin (of kBins counts) at which the running count reaches target >= 1.
__device__ Found find_u32x4(const uint32_t* G, uint32_t target, TopkShared& sh) {
  if (threadIdx.x == 0) sh.found.bin = -1;
  const uint4 c = reinterpret_cast<const uint4*>(G)[threadIdx.x];
  const uint32_t s = c.x + c.y + c.z + c.w;
  uint32_t total;
  const uint32_t ex = block_excl_scan(s, sh.ws, &total);
  if (ex < target && target <= ex + s) {
    const uint32_t v[4] = {c.x, c.y, c.z, c.w};
    uint32_t e = ex;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (target <= e + v[i]) {
        sh.found.bin = 4 * threadIdx.x + i;
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

// Adds this CTA's histogram L into G of every CTA of the cluster and zeroes L
// (and, if given, the local buffer `clr` for the next pass).
__device__ void push_u32(uint32_t* L, uint32_t* G, uint32_t* clr, cg::cluster_group& cl, int C) {
  for (int b = threadIdx.x; b < kBins; b += kThreads) {
    const uint32_t v = L[b];
    if (v) {
      for (int r = 0; r < C; ++r) atomicAdd(cl.map_shared_rank(G + b, r), v);
      L[b] = 0;
    }
    if (clr) clr[b] = 0;
  }
}

__device__ __forceinline__ uint64_t ckey(float v, uint32_t gid, int idxbits) {
  return (static_cast<uint64_t>(~ord32(canon(v))) << idxbits) | gid;
}

template <bool kPen, bool kEmit>
__global__ void __launch_bounds__(kThreads) topk_kernel(const RowArgs a, const DevOpts o) {
  cg::cluster_group cl = cg::this_cluster();
  const int C = a.cluster;
  const int crank = static_cast<int>(cl.block_rank());
  const int row = blockIdx.x / C;
  const int lo = crank * a.slice;
  const int n = max(0, min(a.ncols - lo, a.slice));
  const float* src = a.logits + static_cast<long long>(row) * a.ld + lo;
  const long long g_lo = static_cast<long long>(a.col_off) + lo;

  extern __shared__ __align__(16) unsigned char smem[];
  uint32_t* L = reinterpret_cast<uint32_t*>(smem);
  uint32_t* G = L + kBins;                                     // two buffers
  uint64_t* cand = reinterpret_cast<uint64_t*>(G + 2 * kBins);  // kCandCap
  uint32_t* bm = reinterpret_cast<uint32_t*>(cand + kCandCap);
  __shared__ TopkShared sh;

  cluster_arrive();
  for (int b = threadIdx.x; b < kBins; b += kThreads) {
    L[b] = 0;
    G[b] = 0;
    G[kBins + b] = 0;
  }
  if (threadIdx.x == 0) {
    sh.count = 0;
    sh.flag = 0;
  }
  if (kPen)
    build_bitmap(bm, (a.slice >> 5) + 2, a, o, row, g_lo, n);
  else
    __syncthreads();
  const uint32_t k = kEmit ? static_cast<uint32_t>(min(a.cand_k, a.ncols)) : static_cast<uint32_t>(o.k);

  // Pass over the slice: each thread keeps its 4 smallest keys.
  uint64_t t0 = kNoKey, t1 = kNoKey, t2 = kNoKey, t3 = kNoKey;
  stream_slice<kPen>(src, n, bm, o.repeat, [&](float v, int j) {
    const uint64_t d = dkey(v, static_cast<uint32_t>(g_lo + j));
    if (d < t3) {
      if (d < t1) {
        t3 = t2;
        t2 = t1;
        if (d < t0) {
          t1 = t0;
          t0 = d;
        } else {
          t1 = d;
        }
      } else if (d < t2) {
        t3 = t2;
        t2 = d;
      } else {
        t3 = d;
      }
    }
  });

  // Histogram of thread maxima over the top 11 key bits, summed over the
  // cluster.  The first bin b* at which it reaches k holds the k-th largest
  // thread maximum, so at least k elements have a key bin <= b*: every
  // top-k element does.
  if (t0 != kNoKey) atomicAdd(&L[t0 >> 53], 1u);
  __syncthreads();
  cluster_wait();
  push_u32(L, G, nullptr, cl, C);
  cluster_sync_all();
  const Found fb = find_u32x4(G, k, sh);
  const uint64_t bstar = fb.bin >= 0 ? static_cast<uint64_t>(fb.bin) : static_cast<uint64_t>(kBins - 1);

  // This thread's keys in bins <= b* are candidates.  If its 4th key is one,
  // a 5th might have been dropped: the cluster then selects exactly.
  const bool c0 = t0 != kNoKey && (t0 >> 53) <= bstar;
  const bool c1 = c0 && t1 != kNoKey && (t1 >> 53) <= bstar;
  const bool c2 = c1 && t2 != kNoKey && (t2 >> 53) <= bstar;
  const bool c3 = c2 && t3 != kNoKey && (t3 >> 53) <= bstar;
  const int mine = int(c0) + int(c1) + int(c2) + int(c3);
  const int lane = threadIdx.x & 31;
  const int incl = warp_incl_scan(mine);
  const int wtot = __shfl_sync(0xffffffffu, incl, 31);
  uint32_t base = 0;
  if (lane == 31 && wtot) base = atomicAdd(cl.map_shared_rank(&sh.count, 0), static_cast<uint32_t>(wtot));
  base = __shfl_sync(0xffffffffu, base, 31);
  {
    uint64_t* cand0 = cl.map_shared_rank(cand, 0);
    const uint32_t pos = base + static_cast<uint32_t>(incl - mine);
    const uint64_t tk[4] = {t0, t1, t2, t3};
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (i < mine && pos + i < static_cast<uint32_t>(kCandCap)) cand0[pos + i] = tk[i];
  }
  if (c3) atomicOr(cl.map_shared_rank(&sh.flag, 0), 1u);
  cluster_sync_all();
  if (threadIdx.x == 0) {
    sh.c_total = *cl.map_shared_rank(&sh.count, 0);
    sh.c_flag = *cl.map_shared_rank(&sh.flag, 0);
  }
  __syncthreads();
  uint32_t total = sh.c_total;
  const bool fallback = sh.c_flag != 0 || total > static_cast<uint32_t>(kCandCap) || total < k;

  if (fallback) {
    // Exact radix select of the k-th smallest key, re-reading the slice.
    cluster_sync_all();  // every CTA has read CTA 0's counters
    if (crank == 0 && threadIdx.x == 0) sh.count = 0;
    const int nbits = 32 + a.idxbits;
    uint64_t prefix = 0;
    int resolved = 0;
    uint32_t krem = k;
    int g = 1;  // G[0] still holds the thread-maxima histogram; cleared in the first pass
    int sel_shift = 0;
    while (true) {
      const int shift = max(0, nbits - resolved - kDig);
      const int width = nbits - resolved - shift;
      const uint64_t mask = (1ull << width) - 1;
      const int hi = nbits - resolved;
      stream_slice<kPen>(src, n, bm, o.repeat, [&](float v, int j) {
        const uint64_t kc = ckey(v, static_cast<uint32_t>(g_lo + j), a.idxbits);
        if (resolved == 0 || (kc >> hi) == prefix) atomicAdd(&L[(kc >> shift) & mask], 1u);
      });
      __syncthreads();
      push_u32(L, G + g * kBins, G + (g ^ 1) * kBins, cl, C);
      cluster_sync_all();
      Found f = find_u32x4(G + g * kBins, krem, sh);
      if (f.bin < 0) {  // unreachable: the cluster holds at least k elements
        if (threadIdx.x == 0 && crank == 0) raise_status(kErrSelect);
        f.bin = 0;
        f.before = 0;
        f.cnt = krem;
      }
      prefix = (prefix << width) | static_cast<uint64_t>(f.bin);
      resolved += width;
      krem -= f.before;
      if (f.cnt == krem || shift == 0) {
        sel_shift = shift;
        break;
      }
      g ^= 1;
    }
    // Collect exactly the k selected elements into CTA 0's buffer.
    uint64_t* cand0 = cl.map_shared_rank(cand, 0);
    uint32_t* cnt0 = cl.map_shared_rank(&sh.count, 0);
    stream_slice<kPen>(src, n, bm, o.repeat, [&](float v, int j) {
      const uint32_t gid = static_cast<uint32_t>(g_lo + j);
      const uint64_t kc = ckey(v, gid, a.idxbits);
      if ((kc >> sel_shift) <= prefix) {
        const uint32_t p = atomicAdd(cnt0, 1u);
        if (p < static_cast<uint32_t>(kCandCap)) cand0[p] = dkey(v, gid);
      }
    });
    cluster_sync_all();
    total = k;
  }

  cluster_arrive();
  if (crank != 0) {
    cluster_wait();
    return;
  }
  const int P = next_pow2(max(static_cast<int>(total), 2));
  for (int i = static_cast<int>(total) + threadIdx.x; i < P; i += kThreads) cand[i] = kNoKey;
  __syncthreads();
  bitonic_sort_u64(cand, P);
  if (kEmit) {
    for (int i = threadIdx.x; i < a.cand_k; i += kThreads) {
      const long long at = static_cast<long long>(row) * a.cand_k + i;
      const bool ok = i < static_cast<int>(k);
      a.cand_val[at] = ok ? dval(cand[i]) : -__int_as_float(0x7f800000);
      a.cand_id[at] = ok ? static_cast<int>(did(cand[i])) : -1;
    }
  } else {
    // L and G are free now: reuse them as the tail's fp64 scratch.
    double* pr = reinterpret_cast<double*>(smem);
    double* q = pr + kMaxK;
    tail_pick(cand, static_cast<int>(k), o, a.rng + 2ll * row, a.out_ids + row, a.stats ? a.stats + row : nullptr,
              pr, q, &sh.tail);
  }
  cluster_wait();
}

// ====================================================================== merge
__global__ void __launch_bounds__(kThreads) merge_kernel(const MergeArgs a, const DevOpts o) {
  const int row = blockIdx.x;
  extern __shared__ __align__(16) unsigned char smem[];
  const int total = a.nshards * a.k;
  const int P = next_pow2(max(total, 2));
  uint64_t* cand = reinterpret_cast<uint64_t*>(smem);
  double* pr = reinterpret_cast<double*>(cand + P);
  double* q = pr + kMaxK;
  __shared__ uint32_t ws[kWarps];
  __shared__ TailShared ts;
  uint32_t valid = 0;
  for (int i = threadIdx.x; i < P; i += kThreads) {
    uint64_t d = kNoKey;
    if (i < total) {
      const int s = i / a.k, j = i - s * a.k;
      const long long at = (static_cast<long long>(s) * a.rows + row) * a.k + j;
      const int id = a.cand_id[at];
      if (id >= 0) {
        d = dkey(a.cand_val[at], static_cast<uint32_t>(id));
        ++valid;
      }
    }
    cand[i] = d;
  }
  valid = block_sum(valid, ws);
  bitonic_sort_u64(cand, P);
  if (valid == 0) {
    if (threadIdx.x == 0) {
      raise_status(kErrSelect);
      a.out_ids[row] = -1;
    }
    return;
  }
  if (o.greedy) {
    if (threadIdx.x == 0) {
      const int id = static_cast<int>(did(cand[0]));
      a.out_ids[row] = id;
      if (a.stats) write_stats(a.stats + row, 0.0, 0.0, 0.0, __longlong_as_double(0x7ff0000000000000ll),
                               __longlong_as_double(0x7ff0000000000000ll), o.vocab, 1, id, 1);
    }
    return;
  }
  const int kk = min(o.k, static_cast<int>(valid));
  tail_pick(cand, kk, o, a.rng + 2ll * row, a.out_ids + row, a.stats ? a.stats + row : nullptr, pr, q, &ts);
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

struct HFound {
  int bin;
  unsigned long long before_m, m, total_m;
  uint32_t before_c, c, total_c;
};

struct GenShared {
  uint64_t bar;
  uint64_t xmin[kMaxCluster];
  unsigned long long xs[kMaxCluster];
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
  double fscale;  // 2^fixbits
  int C, crank;
};

__device__ __forceinline__ unsigned long long fixed_mass(const GenCtx& x, float v, double* m_out) {
  const double m = exp(static_cast<double>(__fsub_rn(canon(v), x.M)) * x.inv_temp);
  *m_out = m;
  return __double2ull_rn(m * x.fscale);
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
        if (thr > 0.0 && !(m >= thr)) continue;
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
        if (thr > 0.0 && !(m >= thr)) continue;
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

__global__ void __launch_bounds__(kThreads) general_kernel(const RowArgs a, const DevOpts o) {
  cg::cluster_group cl = cg::this_cluster();
  const int C = a.cluster;
  const int crank = static_cast<int>(cl.block_rank());
  const int row = blockIdx.x / C;
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
  Hist* A = L + 3;   // saved first-digit histogram of the mass pass
  Gath* gb = reinterpret_cast<Gath*>(L + 4);  // two buffers
  __shared__ GenShared sh;

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
  // ---- row maximum (smallest key) across the cluster
  uint64_t best = kNoKey;
  for (int j = threadIdx.x; j < n; j += kThreads) {
    const uint64_t d = dkey(v[j], static_cast<uint32_t>(g_lo + j));
    best = d < best ? d : best;
  }
  best = block_min<unsigned long long>(best, sh.ws64);
  cluster_wait();
  if (threadIdx.x < static_cast<unsigned>(C)) *cl.map_shared_rank(&sh.xmin[crank], threadIdx.x) = best;
  cluster_sync_all();
  uint64_t dmin = sh.xmin[0];
  for (int i = 1; i < C; ++i) dmin = sh.xmin[i] < dmin ? sh.xmin[i] : dmin;
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
  x.fscale = ldexp(1.0, a.fixbits);
  x.C = C;
  x.crank = crank;
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
    // ---- mass pass: S over the k-set, first-digit histogram of the min-p set
    const int shift0 = max(0, x.nbits - kGDig);
    unsigned long long s_local = 0;
    for (int j = threadIdx.x; j < n; j += kThreads) {
      const float vv = v[j];
      const unsigned long long kc = ckey(vv, static_cast<uint32_t>(g_lo + j), a.idxbits);
      if (kc > klim) continue;
      double m;
      const unsigned long long qm = fixed_mass(x, vv, &m);
      s_local += qm;
      if (thr > 0.0 && !(m >= thr)) continue;
      const int dg = static_cast<int>(kc >> shift0);
      atomicAdd(&L->c[dg], 1u);
      if (qm) atomicAdd(&L->m[dg], qm);
    }
    s_local = block_sum(s_local, sh.ws64);
    Hist* Gd = G + gbuf;
    push_hist(L, Gd, G + (gbuf ^ 1), cl, C);
    if (threadIdx.x < static_cast<unsigned>(C)) *cl.map_shared_rank(&sh.xs[crank], threadIdx.x) = s_local;
    cluster_sync_all();
    gbuf ^= 1;
    unsigned long long S = 0;
    for (int i = 0; i < C; ++i) S += sh.xs[i];
    A->c[threadIdx.x] = Gd->c[threadIdx.x];
    A->m[threadIdx.x] = Gd->m[threadIdx.x];
    __syncthreads();
    const HFound tot = find_hist(A, true, ~0ull, sh);  // totals only
    unsigned long long tot_m = tot.total_m;
    uint32_t keep_c = tot.total_c;
    unsigned long long klim_keep = klim;
    // ---- top-p cutoff (src/sampler.cpp:92-100): first element whose running
    // mass reaches top_p * S within the min-p set
    if (o.top_p > 0.0f && o.top_p < 1.0f) {
      const unsigned long long tp =
          static_cast<unsigned long long>(ceil(static_cast<double>(o.top_p) * static_cast<double>(S)));
      const unsigned long long tpt = tp < 1ull ? 1ull : tp;
      if (tot_m >= tpt) {
        select_weighted(x, true, tpt, A, klim, thr, L, G, gb, gseq, gbuf, cl, sh);
        if (sh.r_found) {
          klim_keep = sh.r_key;
          tot_m = sh.r_cum_m;
          keep_c = sh.r_cum_c;
        }
      }
    }
    // ---- the draw (src/sampler.cpp:101-108): first element whose running
    // mass reaches u * tot
    double rt = ceil(u * static_cast<double>(tot_m));
    unsigned long long target = rt < 1.0 ? 1ull : static_cast<unsigned long long>(rt);
    if (target > tot_m) target = tot_m;
    select_weighted(x, true, target, A, klim_keep, thr, L, G, gb, gseq, gbuf, cl, sh);
    if (sh.r_found) {
      out_id = static_cast<int>(sh.r_key & idmask);
    } else {
      out_id = static_cast<int>(klim_keep & idmask);
      if (threadIdx.x == 0 && crank == 0) raise_status(kErrSelect);
    }
    s_sum = static_cast<double>(S) / x.fscale;
    s_tot = static_cast<double>(tot_m) / x.fscale;
    s_keep = static_cast<int>(keep_c);
  }
  if (crank == 0 && threadIdx.x == 0) {
    a.out_ids[row] = out_id;
    if (a.stats) {
      const double nan = __longlong_as_double(0x7ff8000000000000ll);
      write_stats(a.stats + row, s_sum, s_tot, u, nan, nan, o.k, s_keep, out_id, 0);
    }
  }
  // keep shared memory alive until no CTA reads it, and no copy is in flight
  if (sh.load_fail && threadIdx.x == 0) (void)mbar_wait_bounded(&sh.bar, 0);
  cluster_sync_all();
}

// ================================================================ launchers
size_t greedy_smem(int slice) { return static_cast<size_t>((slice >> 5) + 2) * 4; }
size_t topk_smem(int slice) {
  return static_cast<size_t>(3 * kBins) * 4 + static_cast<size_t>(kCandCap) * 8 +
         static_cast<size_t>((slice >> 5) + 2) * 4;
}
size_t general_smem(int slice) {
  const size_t vwords = static_cast<size_t>(((slice + 4 + 3) / 4) * 4);
  const size_t bwords = static_cast<size_t>(((((slice >> 5) + 2) + 3) / 4) * 4);
  return (vwords + bwords) * 4 + 4 * sizeof(Hist) + 2 * sizeof(Gath);
}
static int next_pow2_host(int x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}
size_t merge_smem(int n) { return static_cast<size_t>(next_pow2_host(n < 2 ? 2 : n)) * 8 + 2 * kMaxK * 8; }

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

cudaError_t launch_greedy(const RowArgs& a, const DevOpts& o, cudaStream_t s) {
  const size_t sm = greedy_smem(a.slice);
  if (o.penalize) return launch_cluster(greedy_kernel<true>, a, o, a.rows * a.cluster, a.cluster, sm, s);
  return launch_cluster(greedy_kernel<false>, a, o, a.rows * a.cluster, a.cluster, sm, s);
}

cudaError_t launch_topk(const RowArgs& a, const DevOpts& o, bool emit, cudaStream_t s) {
  const size_t sm = topk_smem(a.slice);
  const int grid = a.rows * a.cluster;
  if (emit) {
    if (o.penalize) return launch_cluster(topk_kernel<true, true>, a, o, grid, a.cluster, sm, s);
    return launch_cluster(topk_kernel<false, true>, a, o, grid, a.cluster, sm, s);
  }
  if (o.penalize) return launch_cluster(topk_kernel<true, false>, a, o, grid, a.cluster, sm, s);
  return launch_cluster(topk_kernel<false, false>, a, o, grid, a.cluster, sm, s);
}

cudaError_t launch_general(const RowArgs& a, const DevOpts& o, cudaStream_t s) {
  return launch_cluster(general_kernel, a, o, a.rows * a.cluster, a.cluster, general_smem(a.slice), s);
}

cudaError_t launch_merge(const MergeArgs& a, const DevOpts& o, cudaStream_t s) {
  const size_t sm = merge_smem(a.nshards * a.k);
  cudaError_t e = cudaFuncSetAttribute(merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sm));
  if (e != cudaSuccess) return e;
  merge_kernel<<<a.rows, kThreads, sm, s>>>(a, o);
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
  }
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
constexpr int kUnionCap = 2048;

struct Shared {
  unsigned long long ws64[NW];
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
#pragma unroll
  for (int i = 0; i < kSplitChunks; ++i) {
    const int q = threadIdx.x + i * NT;
    const int j0 = 4 * q;
    if (vec && j0 + 3 < n) {
      x[i] = ld_stream(s4 + q);
    } else {
      x[i].x = j0 < n ? ld_stream1(src + j0) : nan;
      x[i].y = j0 + 1 < n ? ld_stream1(src + j0 + 1) : nan;
      x[i].z = j0 + 2 < n ? ld_stream1(src + j0 + 2) : nan;
      x[i].w = j0 + 3 < n ? ld_stream1(src + j0 + 3) : nan;
    }
  }
}

__device__ __forceinline__ void penalize_regs(float4 (&x)[kSplitChunks], const uint32_t* bm, float rep, int n) {
#pragma unroll
  for (int i = 0; i < kSplitChunks; ++i) {
    const int j0 = 4 * (threadIdx.x + i * NT);
    if (j0 < n) {
      const uint32_t nib = (bm[j0 >> 5] >> (j0 & 31)) & 15u;
      if (nib) {
        if (nib & 1u) x[i].x = penalize(x[i].x, rep);
        if (nib & 2u) x[i].y = penalize(x[i].y, rep);
        if (nib & 4u) x[i].z = penalize(x[i].z, rep);
        if (nib & 8u) x[i].w = penalize(x[i].w, rep);
      }
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

// First bin (of kBinsS counts, 8 per thread) where the running count reaches target >= 1.
__device__ Found find_bins(const uint32_t* H, uint32_t target, Shared& sh) {
  if (threadIdx.x == 0) sh.found.bin = -1;
  const uint4 a = reinterpret_cast<const uint4*>(H)[2 * threadIdx.x];
  const uint4 b = reinterpret_cast<const uint4*>(H)[2 * threadIdx.x + 1];
  const uint32_t v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  uint32_t s = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) s += v[i];
  uint32_t total;
  const uint32_t ex = block_excl_scan<uint32_t, NT>(s, sh.ws32, &total);
  if (ex < target && target <= ex + s) {
    uint32_t e = ex;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (target <= e + v[i]) {
        sh.found.bin = 8 * threadIdx.x + i;
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

template <int kMode, bool kPen>
__global__ void __launch_bounds__(NT, 4) split_kernel(const RowArgs a, const DevOpts o) {
  const int C = a.cluster;
  const int row = blockIdx.x / C;
  const int s = blockIdx.x - row * C;
  const int lo = s * a.slice;
  const int n = max(0, min(a.ncols - lo, a.slice));
  const float* src = a.logits + static_cast<long long>(row) * a.ld + lo;
  const long long g_lo = static_cast<long long>(a.col_off) + lo;
  extern __shared__ __align__(16) unsigned char smem[];
  uint32_t* H = reinterpret_cast<uint32_t*>(smem);                          // kBinsS counts (top-k modes)
  uint64_t* U = reinterpret_cast<uint64_t*>(H + kBinsS);  // kUnionCap keys (top-k modes)
  uint32_t* bm = kMode == kSplitGreedy ? reinterpret_cast<uint32_t*>(smem) : reinterpret_cast<uint32_t*>(U + kUnionCap);
  __shared__ Shared sh;

  float4 x[kSplitChunks];
  load_regs(src, n, x);  // all loads in flight before anything else
  if (kMode != kSplitGreedy)
    for (int b = threadIdx.x; b < kBinsS; b += NT) H[b] = 0;
  if (threadIdx.x == 0) sh.ncand = 0;
  if (kPen) {
    const int nw = (a.slice >> 5) + 2;
    for (int i = threadIdx.x; i < nw; i += NT) bm[i] = 0;
    __syncthreads();
    const long long h0 = a.hist_off[row], h1 = a.hist_off[row + 1];
    const long long len = h1 - h0;
    const long long from = (o.repeat_last > 0 && len > o.repeat_last) ? len - o.repeat_last : 0;
    for (long long j = h0 + from + threadIdx.x; j < h1; j += NT) {
      const long long t = static_cast<long long>(a.hist[j]) - g_lo;
      if (t >= 0 && t < n) atomicOr(&bm[t >> 5], 1u << (t & 31));
    }
  }
  __syncthreads();
  if (kPen) penalize_regs(x, bm, o.repeat, n);
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
    // Bound from the slice's thread maxima: the first 11-bit key bin where
    // their count reaches kl has at least kl elements at or above it, so the
    // slice's top-kl lies in bins <= b*.
    const unsigned long long tmin = regs_best(x, n, g_lo);
    if (tmin != kNoKey) atomicAdd(&H[tmin >> 53], 1u);
    __syncthreads();
    uint32_t count = 0;
    unsigned long long* out = a.slice_keys + slot * kSliceCap;
    if (kl > 0) {
      const Found fb = find_bins(H, kl, sh);
      for (int b = threadIdx.x; b < kBinsS; b += NT) H[b] = 0;
      const uint32_t bstar = fb.bin >= 0 ? static_cast<uint32_t>(fb.bin) : kBinsS - 1u;
      // bins <= b*  <=>  ord32(v) >= T  <=>  v >= unord32(T) for non-NaN v.
      // T <= ord32(-inf) means every column is a candidate (-inf and NaN too).
      const uint32_t T = ~(((bstar + 1u) << 21) - 1u);
      const bool all = T <= 0x007fffffu;
      const float tv = unord32(T);
      uint32_t mine = 0;
      if (all) {
        for_regs(x, n, [&](float, int) { ++mine; });
      } else {
#pragma unroll
        for (int i = 0; i < kSplitChunks; ++i)
          mine += uint32_t(x[i].x >= tv) + uint32_t(x[i].y >= tv) + uint32_t(x[i].z >= tv) + uint32_t(x[i].w >= tv);
      }
      uint32_t tot;
      const uint32_t ex = block_excl_scan<uint32_t, NT>(mine, sh.ws32, &tot);
      if (tot <= static_cast<uint32_t>(kSliceCap) && tot >= kl) {
        uint32_t at = ex;
        for_regs(x, n, [&](float v, int j) {
          if (all || v >= tv) out[at++] = dkey(v, static_cast<uint32_t>(g_lo + j));
        });
        count = tot;
      } else {
        // more than kSliceCap candidates (ties, masked rows): exact top-kl
        unsigned long long prefix;
        int shift;
        const int nbits = 32 + a.idxbits;
        // (rare path: re-read the slice from L2 so the register copy can die)
        auto each_col = [&](auto f) {
          for (int j = threadIdx.x; j < n; j += NT) {
            float v = ld_stream1(src + j);
            if (kPen && ((bm[j >> 5] >> (j & 31)) & 1u)) v = penalize(v, o.repeat);
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
        count = kl;
      }
    }
    if (threadIdx.x == 0) a.slice_count[slot] = count;
  }

  // publish; the last slice of the row to finish merges
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) sh.last = atomicAdd(&a.counters[row], 1u) == static_cast<unsigned>(C - 1);
  __syncthreads();
  if (!sh.last) return;
  __threadfence();

  if (kMode == kSplitGreedy) {
    if (threadIdx.x < 32) {
      unsigned long long m = kNoKey;
      for (int i = threadIdx.x; i < C; i += 32) {
        const unsigned long long v = __ldcg(&a.slice_keys[static_cast<long long>(row) * C + i]);
        m = v < m ? v : m;
      }
      m = warp_min(m);
      if (threadIdx.x == 0) {
        const int id = static_cast<int>(did(m));
        a.out_ids[row] = id;
        if (a.stats) write_stats(a.stats + row, 0.0, 0.0, 0.0, __longlong_as_double(0x7ff0000000000000ll),
                                 __longlong_as_double(0x7ff0000000000000ll), o.vocab, 1, id, 1);
        a.counters[row] = 0;
      }
    }
    return;
  }

  const uint32_t k = kMode == kSplitEmit ? static_cast<uint32_t>(min(a.cand_k, a.ncols)) : static_cast<uint32_t>(o.k);
  __shared__ uint32_t soff[kMaxSlices + 1];
  const uint32_t ci = threadIdx.x < static_cast<unsigned>(C) ? __ldcg(&a.slice_count[static_cast<long long>(row) * C + threadIdx.x]) : 0u;
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
  uint32_t total;
  if (utot <= static_cast<uint32_t>(kUnionCap)) {
    for (int e = threadIdx.x; e < C * kSliceCap; e += NT) {
      const int i = e / kSliceCap, j = e - i * kSliceCap;
      if (j < static_cast<int>(scnt[i])) U[soff[i] + j] = __ldcg(base + e);
    }
    total = utot;
  } else {
    unsigned long long prefix;
    int shift;
    const int nbits = 32 + a.idxbits;
    auto each = [&](auto f) {
      for (int e = threadIdx.x; e < C * kSliceCap; e += NT) {
        const int i = e / kSliceCap, j = e - i * kSliceCap;
        if (j < static_cast<int>(scnt[i])) f(to_ckey(__ldcg(base + e), a.idxbits));
      }
    };
    radix_select(each, k, nbits, H, sh, &prefix, &shift);
    for (int e = threadIdx.x; e < C * kSliceCap; e += NT) {
      const int i = e / kSliceCap, j = e - i * kSliceCap;
      if (j < static_cast<int>(scnt[i])) {
        const unsigned long long d = __ldcg(base + e);
        if ((to_ckey(d, a.idxbits) >> shift) <= prefix) {
          const uint32_t p = atomicAdd(&sh.ncand, 1u);
          if (p < static_cast<uint32_t>(kUnionCap)) U[p] = d;
        }
      }
    }
    total = k;
  }
  __syncthreads();
  const int P = next_pow2(max(static_cast<int>(total), 2));
  for (int i = static_cast<int>(total) + threadIdx.x; i < P; i += NT) U[i] = kNoKey;
  __syncthreads();
  bitonic_sort_u64(U, P);
  if (kMode == kSplitEmit) {
    for (int i = threadIdx.x; i < a.cand_k; i += NT) {
      const long long at = static_cast<long long>(row) * a.cand_k + i;
      const bool ok = i < static_cast<int>(k);
      a.cand_val[at] = ok ? dval(U[i]) : -__int_as_float(0x7f800000);
      a.cand_id[at] = ok ? static_cast<int>(did(U[i])) : -1;
    }
  } else {
    double* pr = reinterpret_cast<double*>(H);  // H is free: fp64 scratch of the tail
    tail_pick(U, static_cast<int>(k), o, a.rng + 2ll * row, a.out_ids + row, a.stats ? a.stats + row : nullptr, pr,
              pr + kSplitMaxK, &sh.tail);
  }
  if (threadIdx.x == 0) a.counters[row] = 0;
}

}  // namespace split

size_t split_scratch_bytes(long long rows, int slices, size_t* off_count, size_t* off_keys) {
  auto up = [](size_t b) { return (b + 255) & ~static_cast<size_t>(255); };
  const size_t counters = up(static_cast<size_t>(rows) * 4);
  const size_t counts = up(static_cast<size_t>(rows) * slices * 4);
  const size_t keys = static_cast<size_t>(rows) * slices * kSliceCap * 8;
  *off_count = counters;
  *off_keys = counters + counts;
  return counters + counts + keys;
}

template <int kMode, bool kPen>
static cudaError_t launch_split_t(const RowArgs& a, const DevOpts& o, cudaStream_t s) {
  const size_t bmb = static_cast<size_t>((a.slice >> 5) + 2) * 4;
  const size_t sm = kMode == kSplitGreedy ? bmb : split::kBinsS * 4 + split::kUnionCap * 8 + bmb;
  split::split_kernel<kMode, kPen><<<a.rows * a.cluster, split::NT, sm, s>>>(a, o);
  return cudaGetLastError();
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

}  // namespace vb
