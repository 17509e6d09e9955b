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

/* ---- Logits producer tail (src/session.cpp:163-169) ----------------------
 *
 * The final RMSNorm of the last hidden states followed by the LM head:
 *   x      n rows of `dim` floats, row i at x + i*ldx;
 *   norm   dim floats (model.norm.weight), eps = rms_norm_eps;
 *   head   verbo::Tensor layout (src/kernels.hpp:13-23), `vocab` rows:
 *            dtype 0 (F32)  q = vocab x dim floats, s unused;
 *            dtype 1 (Q8)   q = vocab x dim int8, s = vocab x dim/32 fp16 bits;
 *            dtype 2 (Q4)   q = vocab x dim/2 bytes (byte i of a 32-block holds
 *                           element i in its low nibble and element i+16 in
 *                           its high nibble, each stored as value + 8), s as Q8;
 *   out    n rows of `vocab` floats, row i at out + i*ld;
 *   xq, xs optional: the activations as quant_act leaves them (Q8/Q4 heads),
 *          n x dim int8 and n x dim/32 float block scales.
 * dim must be a positive multiple of 32 (src/model.cpp:108).  Returns 0, or -1
 * on bad arguments. */
int oracle_logits_tail(int dtype, int vocab, int dim, const void* q, const uint16_t* s, const float* norm,
                       float eps, const float* x, int n, long long ldx, float* out, long long ld, int8_t* xq,
                       float* xs);

/* The same through the reference's own rmsnorm, quant_act and matmul
   (oracle/_ref/libverbo_ref_tail*.so), matmul on a Pool of `threads`. */
int ref_logits_tail(int dtype, int vocab, int dim, const void* q, const uint16_t* s, const float* norm, float eps,
                    const float* x, int n, long long ldx, float* out, long long ld, int8_t* xq, float* xs,
                    int threads);

/* Runs a checkpoint through the reference's Session (oracle/_ref tail
   harnesses): Model::load(dir, dtype), Session::eval_all(toks[0..n)), n <= 64.
   Copies out the final hidden rows x (n x dim, before the last rmsnorm), the
   reference's logits (n x vocab), its head q / s (verbo::Tensor layout, the
   head's own dtype) and the norm weight.  meta = {dim, vocab, head dtype}; with
   x_out NULL only meta and eps are filled. */
int ref_model_tail(const char* dir, int dtype, const int* toks, int n, int threads, int* meta, float* eps_out,
                   float* x_out, float* logits_out, void* q_out, uint16_t* s_out, float* norm_out);

/* The reference's decode loop on a checkpoint (oracle/_ref tail harnesses):
   verbo::generate (src/sampler.cpp:111-181) of prompt[0..n) with `opts`
   (seed must be non-zero), max_tokens, no stop text; then the same loop
   replayed on a fresh Session with the reference's Sampler, copying out for
   every pick j (at most `cap`) its id and the hidden row its logits came from
   (x_out + j*dim: the residual of the position that produced them, before the
   final rmsnorm).  The last pick is the stop id when the generation stopped
   on one (*stopped = 1).  Returns the number of picks, -1 on an error, -2
   when the replay's ids differ from generate's (Stats::toks). */
int ref_decode(const char* dir, int dtype, const int* prompt, int n, const oracle_sampling* opts, int max_tokens,
               int threads, int cap, int* ids_out, float* x_out, int* stopped);

#ifdef __cplusplus
}
#endif

#endif
