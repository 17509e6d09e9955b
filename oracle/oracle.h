/*
 * CPU oracle for the token-sampling path.  TEST INFRASTRUCTURE ONLY.
 *
 * This header declares two checkers with the same batched row layout as the
 * product's C ABI (include/verbo_cuda.h):
 *
 *   oracle_*  - a plain-C restatement of verbo's Sampler (src/sampler.cpp),
 *               built from sampler_oracle.c into oracle/_build/liboracle.so;
 *   ref_*     - a harness around the reference's own compiled Sampler,
 *               built from the reference sources into oracle/_ref/.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU legs may load these
 * libraries, and only to check or time the CPU side.  The CUDA library never
 * links against them and has no CPU fallback.
 *
 * Row layout (shared with the product):
 *   logits   rows x ld floats, row r at logits + r*ld, `vocab` valid columns;
 *   hist     concatenated token histories, row r owns hist[off[r] .. off[r+1]);
 *            NULL means no history for every row;
 *   window   the penalty window is the last `repeat_last` ids of a row's
 *            history (all of it when repeat_last <= 0), as Sampler::pick
 *            computes it (src/sampler.cpp:53-57);
 *   rng      2 x u64 xoroshiro128+ state per row, advanced in place by one
 *            draw per non-greedy pick (src/sampler.cpp:33-41).
 */
#ifndef VERBO_ORACLE_H
#define VERBO_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Field-for-field copy of verbo::Sampling (include/verbo/verbo.hpp:56-64). */
typedef struct {
  float temp;
  int top_k;
  float top_p;
  float min_p;
  float repeat;
  int repeat_last;
  unsigned long long seed;
} oracle_sampling;

/* Per-row diagnostics of one pick. */
typedef struct {
  double sum;         /* softmax normaliser over the k candidates (sampler.cpp:80-85)  */
  double tot;         /* mass of the kept prefix (sampler.cpp:101-102)                 */
  double u;           /* the uniform drawn for this pick (sampler.cpp:103)             */
  double draw_margin; /* distance of u to the nearest CDF boundary, in units of tot    */
  double cut_margin;  /* distance of top_p / min_p decisions to their thresholds       */
  int k;              /* candidate count (top_k or vocab)                              */
  int keep;           /* kept prefix length after min-p and top-p                      */
  int id;             /* sampled token id                                              */
  int greedy;         /* 1 when temp <= 0                                              */
} oracle_row_stats;

/* splitmix64 seeding as Sampler::reset (src/sampler.cpp:11-16, 26-31).
   seed must be non-zero (the reference seeds 0 from the clock). */
void oracle_seed(uint64_t seed, uint64_t state[2]);
/* One xoroshiro128+ draw in [0,1) as Sampler::unit (src/sampler.cpp:33-41). */
double oracle_unit(uint64_t state[2]);

/* Sampler::pick over a batch of rows (src/sampler.cpp:50-109).  Returns 0. */
int oracle_sample_rows(const float* logits, int rows, int vocab, long long ld, const int* hist,
                       const long long* hist_off, const oracle_sampling* opts, uint64_t* rng_state,
                       int* out_ids, oracle_row_stats* stats);

/* Vocab-sharded form of the same pick: per-shard top-k candidates ...        */
int oracle_shard_topk(const float* logits, int rows, int shard_cols, long long ld, int col_offset,
                      int vocab, const int* hist, const long long* hist_off, const oracle_sampling* opts,
                      int k, float* cand_val, int* cand_id);
/* ... merged across shards (layout [nshards][rows][k]) and sampled.          */
int oracle_merge_sample(const float* cand_val, const int* cand_id, int rows, int nshards, int k, int vocab,
                        const oracle_sampling* opts, uint64_t* rng_state, int* out_ids,
                        oracle_row_stats* stats);

/* Harness over the reference's compiled verbo::Sampler (oracle/_ref).
   Row r gets Sampler(opts with seed = seeds[r]); its history is fed with
   accept(); then pick() runs `steps` times on the same row, writing
   out_ids[r*steps + s].  Rows are split over `threads` std::threads. */
int ref_sample_rows(const float* logits, int rows, int vocab, long long ld, const int* hist,
                    const long long* hist_off, const oracle_sampling* opts,
                    const unsigned long long* seeds, int steps, int* out_ids, int threads);

#ifdef __cplusplus
}
#endif

#endif
