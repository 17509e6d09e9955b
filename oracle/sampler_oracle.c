/*
 * Plain-C restatement of verbo's token sampler (src/sampler.cpp) - TEST
 * INFRASTRUCTURE ONLY.  It is the checker for the CUDA library, never a
 * fallback for it.  Every step cites the reference line it restates; the
 * arithmetic is kept in the same types and the same order so that results
 * are bit-identical to the reference on the same inputs (checked against the
 * reference's own compiled Sampler by tests/test_oracle.py).
 *
 * Build: oracle/Makefile (no -ffast-math: fp32 penalty and fp64 softmax must
 * round exactly as the reference does).
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
  float v;
  int i;
} pair_t;

/* splitmix64 step: src/sampler.cpp:11-16. */
static uint64_t splitmix(uint64_t* s) {
  uint64_t z = (*s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

/* Sampler::reset seeding: src/sampler.cpp:26-31 (caller supplies a non-zero seed). */
void oracle_seed(uint64_t seed, uint64_t state[2]) {
  uint64_t s = seed;
  state[0] = splitmix(&s);
  state[1] = splitmix(&s);
}

/* Sampler::unit, xoroshiro128+: src/sampler.cpp:33-41. */
double oracle_unit(uint64_t st[2]) {
  uint64_t s1 = st[0];
  const uint64_t s0 = st[1];
  const uint64_t r = s0 + s1;
  st[0] = s0;
  s1 ^= s1 << 23;
  st[1] = s1 ^ s0 ^ (s1 >> 18) ^ (s0 >> 5);
  return (double)(r >> 11) * (1.0 / 9007199254740992.0);
}

/* The `by` order of src/sampler.cpp:71: value descending, index ascending. */
static int before(pair_t a, pair_t b) { return a.v > b.v || (a.v == b.v && a.i < b.i); }

static int cmp_by(const void* x, const void* y) {
  const pair_t a = *(const pair_t*)x, b = *(const pair_t*)y;
  return before(a, b) ? -1 : (before(b, a) ? 1 : 0);
}

static int cmp_int(const void* x, const void* y) {
  const int a = *(const int*)x, b = *(const int*)y;
  return (a > b) - (a < b);
}

/* Penalty window and dedup: src/sampler.cpp:53-59.  Returns the count of
   distinct ids written to `seen`. */
static int window_ids(const int* hist, long long beg, long long end, int repeat_last, int* seen) {
  long long len = end - beg;
  long long from = (repeat_last > 0 && len > repeat_last) ? len - repeat_last : 0;
  int n = 0;
  for (long long j = beg + from; j < end; ++j) seen[n++] = hist[j];
  qsort(seen, (size_t)n, sizeof(int), cmp_int);
  int u = 0;
  for (int j = 0; j < n; ++j)
    if (u == 0 || seen[u - 1] != seen[j]) seen[u++] = seen[j];
  return u;
}

/* v > 0 ? v / repeat : v * repeat, in fp32: src/sampler.cpp:60-64. */
static void apply_penalty(pair_t* buf, int n, int col_offset, const int* seen, int nseen, float repeat) {
  for (int j = 0; j < nseen; ++j) {
    const int t = seen[j] - col_offset;
    if (t < 0 || t >= n) continue;
    float v = buf[t].v;
    buf[t].v = v > 0.0f ? v / repeat : v * repeat;
  }
}

/* The k first elements of `buf` in `by` order, sorted (std::partial_sort at
   src/sampler.cpp:73-75; the full std::sort at :76-78 when k == n). */
static void top_sorted(pair_t* buf, int n, int k) {
  if (k >= n || k > 256) {
    qsort(buf, (size_t)n, sizeof(pair_t), cmp_by);
    return;
  }
  /* insertion into a sorted prefix of length k */
  int cnt = 0;
  for (int i = 0; i < n; ++i) {
    pair_t e = buf[i];
    if (cnt == k && !before(e, buf[k - 1])) continue;
    int p = cnt < k ? cnt : k - 1;
    while (p > 0 && before(e, buf[p - 1])) {
      buf[p] = buf[p - 1];
      --p;
    }
    buf[p] = e;
    if (cnt < k) ++cnt;
  }
}

static double dmin(double a, double b) { return a < b ? a : b; }

/* Softmax, min-p, top-p and the draw over a sorted candidate list:
   src/sampler.cpp:79-108. */
static int pick_sorted(const pair_t* buf, int k, const oracle_sampling* o, uint64_t* st, oracle_row_stats* rs) {
  if (k < 1) k = 1;
  double* pr = (double*)calloc((size_t)k, sizeof(double));
  const float mx = buf[0].v;
  double sum = 0.0;
  for (int i = 0; i < k; ++i) {
    pr[i] = exp((double)(buf[i].v - mx) / o->temp);
    sum += pr[i];
  }
  int keep = k;
  double cut_margin = INFINITY;
  if (o->min_p > 0.0f) {
    const double thr = pr[0] * o->min_p;
    keep = 1;
    while (keep < k && pr[keep] >= thr) ++keep;
    cut_margin = dmin(cut_margin, (pr[keep - 1] - thr) / sum);
    if (keep < k) cut_margin = dmin(cut_margin, (thr - pr[keep]) / sum);
  }
  if (o->top_p > 0.0f && o->top_p < 1.0f) {
    double acc = 0.0, prev = 0.0;
    int i = 0;
    for (; i < keep; ++i) {
      prev = acc;
      acc += pr[i] / sum;
      if (acc >= o->top_p) break;
    }
    if (i < keep) {
      cut_margin = dmin(cut_margin, acc - o->top_p);
      if (i > 0) cut_margin = dmin(cut_margin, o->top_p - prev);
    } else {
      cut_margin = dmin(cut_margin, o->top_p - acc);
    }
    keep = keep < i + 1 ? keep : i + 1;
  }
  double tot = 0.0;
  for (int i = 0; i < keep; ++i) tot += pr[i];
  const double u = oracle_unit(st);
  double r = u * tot;
  const double r0 = r;
  int pick = keep - 1;
  for (int i = 0; i < keep; ++i) {
    r -= pr[i];
    if (r <= 0.0) {
      pick = i;
      break;
    }
  }
  if (rs) {
    double below = 0.0;
    for (int i = 0; i < pick; ++i) below += pr[i];
    double m = INFINITY;
    if (pick > 0) m = dmin(m, r0 - below);
    if (pick < keep - 1) m = dmin(m, below + pr[pick] - r0);
    rs->sum = sum;
    rs->tot = tot;
    rs->u = u;
    rs->draw_margin = m / tot;
    rs->cut_margin = cut_margin;
    rs->k = k;
    rs->keep = keep;
    rs->id = buf[pick].i;
    rs->greedy = 0;
  }
  const int id = buf[pick].i;
  free(pr);
  return id;
}

/* Greedy argmax, lowest index on ties, as std::max_element with the
   comparator of src/sampler.cpp:66-70 (scanned in index order). */
static int pick_greedy(const pair_t* buf, int n) {
  int best = 0;
  for (int i = 1; i < n; ++i) {
    const pair_t a = buf[best], b = buf[i];
    if (a.v < b.v || (a.v == b.v && a.i > b.i)) best = i;
  }
  return buf[best].i;
}

static void greedy_stats(oracle_row_stats* rs, int id, int n) {
  if (!rs) return;
  memset(rs, 0, sizeof(*rs));
  rs->draw_margin = INFINITY;
  rs->cut_margin = INFINITY;
  rs->k = n;
  rs->keep = 1;
  rs->id = id;
  rs->greedy = 1;
}

/* Sampler::pick (src/sampler.cpp:50-109) for each row. */
int oracle_sample_rows(const float* logits, int rows, int vocab, long long ld, const int* hist,
                       const long long* hist_off, const oracle_sampling* o, uint64_t* rng_state,
                       int* out_ids, oracle_row_stats* stats) {
  pair_t* buf = (pair_t*)malloc(sizeof(pair_t) * (size_t)vocab);
  int* seen = NULL;
  long long max_h = 0;
  if (hist && hist_off)
    for (int r = 0; r < rows; ++r) {
      long long h = hist_off[r + 1] - hist_off[r];
      if (h > max_h) max_h = h;
    }
  seen = (int*)malloc(sizeof(int) * (size_t)(max_h + 1));
  for (int r = 0; r < rows; ++r) {
    const float* row = logits + (long long)r * ld;
    for (int i = 0; i < vocab; ++i) {
      buf[i].v = row[i];
      buf[i].i = i;
    }
    if (o->repeat != 1.0f && hist && hist_off && hist_off[r + 1] > hist_off[r]) {
      int ns = window_ids(hist, hist_off[r], hist_off[r + 1], o->repeat_last, seen);
      apply_penalty(buf, vocab, 0, seen, ns, o->repeat);
    }
    oracle_row_stats* rs = stats ? stats + r : NULL;
    if (o->temp <= 0.0f) {
      out_ids[r] = pick_greedy(buf, vocab);
      greedy_stats(rs, out_ids[r], vocab);
      continue;
    }
    int k = vocab;
    if (o->top_k > 0 && o->top_k < vocab) k = o->top_k;
    top_sorted(buf, vocab, k);
    out_ids[r] = pick_sorted(buf, k, o, rng_state + 2 * (long long)r, rs);
  }
  free(seen);
  free(buf);
  return 0;
}

/* Per-shard candidates: the penalty restricted to the shard's columns, then
   the shard's k best (value, global id) pairs in `by` order; missing slots
   are (-inf, -1). */
int oracle_shard_topk(const float* logits, int rows, int shard_cols, long long ld, int col_offset, int vocab,
                      const int* hist, const long long* hist_off, const oracle_sampling* o, int k,
                      float* cand_val, int* cand_id) {
  (void)vocab;
  pair_t* buf = (pair_t*)malloc(sizeof(pair_t) * (size_t)(shard_cols > 0 ? shard_cols : 1));
  long long max_h = 0;
  if (hist && hist_off)
    for (int r = 0; r < rows; ++r) {
      long long h = hist_off[r + 1] - hist_off[r];
      if (h > max_h) max_h = h;
    }
  int* seen = (int*)malloc(sizeof(int) * (size_t)(max_h + 1));
  for (int r = 0; r < rows; ++r) {
    const float* row = logits + (long long)r * ld;
    for (int i = 0; i < shard_cols; ++i) {
      buf[i].v = row[i];
      buf[i].i = col_offset + i;
    }
    if (o->repeat != 1.0f && hist && hist_off && hist_off[r + 1] > hist_off[r]) {
      int ns = window_ids(hist, hist_off[r], hist_off[r + 1], o->repeat_last, seen);
      apply_penalty(buf, shard_cols, col_offset, seen, ns, o->repeat);
    }
    int kk = k < shard_cols ? k : shard_cols;
    top_sorted(buf, shard_cols, kk);
    for (int i = 0; i < k; ++i) {
      cand_val[(long long)r * k + i] = i < kk ? buf[i].v : -INFINITY;
      cand_id[(long long)r * k + i] = i < kk ? buf[i].i : -1;
    }
  }
  free(seen);
  free(buf);
  return 0;
}

/* Merge of per-shard candidates, then the same tail as Sampler::pick.  The
   global top_k set is contained in the union of the shards' top-k sets when
   top_k <= k, so this equals pick() on the unsharded row. */
int oracle_merge_sample(const float* cand_val, const int* cand_id, int rows, int nshards, int k, int vocab,
                        const oracle_sampling* o, uint64_t* rng_state, int* out_ids, oracle_row_stats* stats) {
  pair_t* buf = (pair_t*)malloc(sizeof(pair_t) * (size_t)(nshards * k));
  for (int r = 0; r < rows; ++r) {
    int n = 0;
    for (int s = 0; s < nshards; ++s)
      for (int i = 0; i < k; ++i) {
        long long at = ((long long)s * rows + r) * k + i;
        if (cand_id[at] < 0) continue;
        buf[n].v = cand_val[at];
        buf[n].i = cand_id[at];
        ++n;
      }
    qsort(buf, (size_t)n, sizeof(pair_t), cmp_by);
    oracle_row_stats* rs = stats ? stats + r : NULL;
    if (o->temp <= 0.0f) {
      out_ids[r] = buf[0].i;
      greedy_stats(rs, out_ids[r], vocab);
      continue;
    }
    int kk = (o->top_k > 0 && o->top_k < vocab) ? o->top_k : vocab;
    if (kk > n) kk = n;
    out_ids[r] = pick_sorted(buf, kk, o, rng_state + 2 * (long long)r, rs);
  }
  free(buf);
  return 0;
}
