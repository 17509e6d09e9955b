/*
 * verbo_cuda.h - C ABI of the B200 (sm_100a) token sampler.
 *
 * A drop-in for verbo's Sampler (src/sampler.cpp, include/verbo/verbo.hpp:
 * 56-64 and 116-132), placed beside the reference's C ABI
 * (include/verbo/verbo.h, src/capi.cpp).  Conventions follow that ABI:
 *   - plain pointers and sizes, no C++ or torch types;
 *   - int functions return 0 (or a token id) on success and -1 on error,
 *     pointer functions return NULL on error;
 *   - the message of the last error on this thread is verbo_cuda_last_error()
 *     (as verbo_last_error, src/capi.cpp:17-30 and :46);
 *   - VERBO_CUDA_API marks every exported symbol (the library is built with
 *     -fvisibility=hidden, as CMakeLists.txt:36 does for libverbo).
 *
 * Batched entry points take DEVICE pointers and are asynchronous on the given
 * CUDA stream (NULL = legacy default stream).  The caller owns every buffer.
 * Device-side failures (a bounded wait that ran out) are recorded in a status
 * word that verbo_cuda_check() reads.
 *
 * Row layout:
 *   logits   rows x ld fp32, row r at logits + r*ld, `vocab` valid columns;
 *   hist     int32 token histories in CSR form: row r owns
 *            hist[hist_off[r] .. hist_off[r+1]); NULL hist => no history;
 *            the penalty window is the last repeat_last ids of each row
 *            (all of them when repeat_last <= 0), src/sampler.cpp:53-57;
 *   rng      2 x u64 xoroshiro128+ state per row, advanced in place by one
 *            draw per non-greedy pick (src/sampler.cpp:33-41, :103).
 */
#ifndef VERBO_CUDA_H
#define VERBO_CUDA_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(_WIN32)
#define VERBO_CUDA_API __declspec(dllexport)
#else
#define VERBO_CUDA_API __attribute__((visibility("default")))
#endif

/* verbo::Sampling, field for field (include/verbo/verbo.hpp:56-64);
   verbo_cuda_default_sampling() returns the reference defaults
   {temp 0.7, top_k 40, top_p 0.9, min_p 0, repeat 1, repeat_last 64, seed 0}. */
typedef struct {
  float temp;
  int top_k;
  float top_p;
  float min_p;
  float repeat;
  int repeat_last;
  unsigned long long seed;
} verbo_sampling;

/* Optional per-row diagnostics of one pick (device memory when passed to a
   batched call).  `sum`/`tot` are the softmax normaliser and the kept mass of
   src/sampler.cpp:80-102, `u` the uniform drawn, `keep` the kept prefix. */
typedef struct {
  double sum;
  double tot;
  double u;
  double draw_margin;
  double cut_margin;
  int k;
  int keep;
  int id;
  int greedy;
} verbo_row_stats;

/* Replaces verbo_last_error (include/verbo/verbo.h:30). */
VERBO_CUDA_API const char* verbo_cuda_last_error(void);
/* Replaces verbo_version (include/verbo/verbo.h:31). */
VERBO_CUDA_API const char* verbo_cuda_version(void);
/* The defaults of verbo::Sampling (include/verbo/verbo.hpp:56-64). */
VERBO_CUDA_API verbo_sampling verbo_cuda_default_sampling(void);

/* Seeds one xoroshiro128+ state exactly as Sampler::reset
   (src/sampler.cpp:26-31): two splitmix64 outputs of `seed`; seed 0 takes the
   clock, as the reference does.  Host memory. */
VERBO_CUDA_API int verbo_cuda_rng_seed(unsigned long long seed, unsigned long long state[2]);
/* One Sampler::unit draw on a host state (src/sampler.cpp:33-41). */
VERBO_CUDA_API double verbo_cuda_rng_unit(unsigned long long state[2]);

/* Sampler::pick (src/sampler.cpp:50-109) for `rows` device-resident rows with
   one option set.  Writes out_ids[r] (device).  rng may be NULL only when
   opts->temp <= 0 (greedy consumes no draw).  stats may be NULL.
   Limits: 1 <= vocab <= 327680, ld >= vocab, temp not NaN or +inf. */
VERBO_CUDA_API int verbo_cuda_sample(const float* logits, int rows, int vocab, long long ld, const int* hist,
                                     const long long* hist_off, const verbo_sampling* opts,
                                     unsigned long long* rng, int* out_ids, verbo_row_stats* stats,
                                     void* stream);

/* No counterpart in the reference (its sampler never touches the GPU).
   Same arguments and results as verbo_cuda_sample, for greedy and
   0 < top_k <= 256, but it allocates nothing: no cudaMalloc, cudaFree or
   allocating library call.  It is meant for callers that cannot let a library
   allocate device memory behind their back: a serving engine that reserves
   almost all of HBM for its KV cache up front and runs its own allocator,
   or a latency-sensitive decode loop that cannot afford the device-wide
   synchronisation of cudaMalloc/cudaFree (verbo_cuda_sample allocates its
   scratch on first use per stream and grows it for larger batches).
   Its scratch is a fixed 8 MiB array inside the library, held by every device
   that loads the library until the process exits: up to about 272 top-k rows
   per call at vocab 151936 (127 at the largest vocab, 327680) and about
   46,000 greedy rows; larger calls are rejected with an error.  Each call
   looks up the array's address (cudaGetSymbolAddress).  CUDA loads a
   library's device code lazily, so the first call on each device also loads
   this library's module there, placing the array and the kernels' code in
   device memory at that moment: make that first call (or run with
   CUDA_MODULE_LOADING=EAGER) before reserving the memory pool and before any
   stream capture.  All calls share the array: calls that overlap on the GPU
   (concurrent streams or host threads) race and must be serialised by the
   caller. */
VERBO_CUDA_API int verbo_cuda_sample_noalloc(const float* logits, int rows, int vocab, long long ld,
                                             const int* hist, const long long* hist_off,
                                             const verbo_sampling* opts, unsigned long long* rng, int* out_ids,
                                             verbo_row_stats* stats, void* stream);

/* Vocab-sharded sampling, step 1: for a shard holding global columns
   [col_offset, col_offset + shard_cols) of each row, apply the penalty for
   the history ids that fall in the shard and emit the shard's k best
   (value, global id) pairs in the reference's order (value descending, id
   ascending) to cand_val/cand_id [rows][k] (device).  Missing slots are
   (-inf, -1).  1 <= k <= 256. */
VERBO_CUDA_API int verbo_cuda_shard_topk(const float* logits, int rows, int shard_cols, long long ld,
                                         int col_offset, int vocab, const int* hist, const long long* hist_off,
                                         const verbo_sampling* opts, int k, float* cand_val, int* cand_id,
                                         void* stream);

/* Vocab-sharded sampling, step 2: merge the candidates of all shards, laid
   out [nshards][rows][k] (the layout of an all-gather of step-1 outputs), and
   finish the pick: softmax, min-p, top-p and the draw.  Equal to
   verbo_cuda_sample on the unsharded rows when opts->temp <= 0 or
   0 < opts->top_k <= k.  k <= 256, nshards * k <= 4096. */
VERBO_CUDA_API int verbo_cuda_merge_sample(const float* cand_val, const int* cand_id, int rows, int nshards,
                                           int k, int vocab, const verbo_sampling* opts,
                                           unsigned long long* rng, int* out_ids, verbo_row_stats* stats,
                                           void* stream);

/* ---- vocab-sharded sampling over GPUs, with the library's own collective ----
   No counterpart in the reference (its sampler runs on one host).  A row whose
   columns are split over the ranks of a job, one GPU each (the logits of a
   vocab-parallel LM head), is sampled as verbo_cuda_shard_topk, ONE all-gather
   of every rank's packed (value, id) candidates over NVLink, and
   verbo_cuda_merge_sample, all on the caller's stream; every rank gets the
   same ids.  The communicator is NCCL, loaded at run time (libnccl.so.2).
   Set-up: rank 0 makes an id with verbo_cuda_comm_unique_id, the caller hands
   the 128 bytes to every rank (MPI, a store, a file), and every rank calls
   verbo_cuda_comm_new with it (collective: all ranks must call it). */
#define VERBO_CUDA_UNIQUE_ID_BYTES 128
typedef struct verbo_cuda_comm verbo_cuda_comm;
VERBO_CUDA_API int verbo_cuda_comm_unique_id(unsigned char id[VERBO_CUDA_UNIQUE_ID_BYTES]);
VERBO_CUDA_API verbo_cuda_comm* verbo_cuda_comm_new(const unsigned char id[VERBO_CUDA_UNIQUE_ID_BYTES], int nranks,
                                                    int rank, int device);
VERBO_CUDA_API void verbo_cuda_comm_free(verbo_cuda_comm* c);
/* One vocab-sharded pick: this rank holds global columns [col_offset,
   col_offset + shard_cols) of each row (device memory, like
   verbo_cuda_shard_topk); the penalty applies to the history ids in the shard.
   k <= 256 candidates per rank, nranks * k <= 4096; needs temp <= 0 or
   0 < top_k <= k (then the global top-k lies in the union of the shards').
   rng (2 per row, the same on every rank) is advanced as in verbo_cuda_sample. */
VERBO_CUDA_API int verbo_cuda_sharded_sample(verbo_cuda_comm* c, const float* logits, int rows, int shard_cols,
                                             long long ld, int col_offset, int vocab, const int* hist,
                                             const long long* hist_off, const verbo_sampling* opts, int k,
                                             unsigned long long* rng, int* out_ids, verbo_row_stats* stats,
                                             void* stream);
/* Bounded wait for the work queued on `stream`: returns 0 once it completed;
   if it has not within timeout_ms, or the communicator reports an error, the
   communicator is aborted and -1 is returned (a rank that died turns into an
   error on the others, not a hang). */
VERBO_CUDA_API int verbo_cuda_comm_wait(verbo_cuda_comm* c, void* stream, int timeout_ms);
/* Timing of the three steps: the next verbo_cuda_sharded_sample on `c` records
   `after_shard` (a cudaEvent_t, or NULL) on its stream once the shard's top-k
   kernel is queued, and `after_gather` once the all-gather is; the caller's
   own events before and after the call close the shard-kernel and merge
   intervals.  Applies to that one call, then both are cleared. */
VERBO_CUDA_API int verbo_cuda_comm_mark_next(verbo_cuda_comm* c, void* after_shard, void* after_gather);

/* Synchronises `stream` and reports device-side failures recorded since the
   last check (then clears them): 0 if none, -1 with a message otherwise. */
VERBO_CUDA_API int verbo_cuda_check(void* stream);

/* Diagnostics of the full-vocabulary path (top_k == 0 or >= vocab, no
   penalty; no counterpart in the reference): synchronises `stream` and
   returns how many rows of the last such call on it were settled by the
   staged cluster kernel instead of the streaming one (rows whose cutoff or
   draw fell among crowded or underflow columns), or -1 on error. */
VERBO_CUDA_API int verbo_cuda_full_vocab_fallbacks(void* stream);

/* ---- Single-stream sampler object: the verbo::Sampler interface
        (include/verbo/verbo.hpp:116-132) as an opaque handle. ---- */
typedef struct verbo_cuda_sampler verbo_cuda_sampler;

/* Sampler(Sampling) (src/sampler.cpp:24): seeds the RNG, empty history.
   `device` is the CUDA device to run on. */
VERBO_CUDA_API verbo_cuda_sampler* verbo_cuda_sampler_new(const verbo_sampling* cfg, int device);
VERBO_CUDA_API void verbo_cuda_sampler_free(verbo_cuda_sampler* s);
/* Sampler::pick (src/sampler.cpp:50-109).  `logits` may be host or device
   memory; returns the token id, or -1 on error. */
VERBO_CUDA_API int verbo_cuda_sampler_pick(verbo_cuda_sampler* s, const float* logits, int n);
/* Sampler::accept (src/sampler.cpp:43-48). */
VERBO_CUDA_API int verbo_cuda_sampler_accept(verbo_cuda_sampler* s, int tok);
/* Sampler::reset (src/sampler.cpp:26-31). */
VERBO_CUDA_API int verbo_cuda_sampler_reset(verbo_cuda_sampler* s);
/* Sampler::cfg (include/verbo/verbo.hpp:123). */
VERBO_CUDA_API int verbo_cuda_sampler_cfg(const verbo_cuda_sampler* s, verbo_sampling* out);

/* ---- batched generation streams ------------------------------------------
   The loop of verbo::generate (src/sampler.cpp:111-181) for B streams at
   once, with each stream's Sampler state on the device: its xoroshiro128+
   state and its penalty window (the last repeat_last accepted ids, which is
   all Sampler::pick reads of the history).  A step samples one id per stream
   from B device rows and accepts it into the stream's window on the device,
   so the caller's decode loop moves only the ids it wants to inspect (stop
   checks and detokenisation stay on the host, as in generate).  The reference
   has one Sampler per generation and no batched form.
   With a penalty (repeat != 1) the options need 1 <= repeat_last <= 2048;
   every stream starts as verbo::Sampler(cfg) does (seeded from cfg.seed) and
   is re-seeded with verbo_cuda_batch_reset.  Calls on one batch are ordered by
   the CUDA stream they are given: use one stream per batch, or synchronise. */
typedef struct verbo_cuda_batch verbo_cuda_batch;
VERBO_CUDA_API verbo_cuda_batch* verbo_cuda_batch_new(const verbo_sampling* cfg, int streams, int device);
VERBO_CUDA_API void verbo_cuda_batch_free(verbo_cuda_batch* b);
/* Sampler::reset for stream `stream` (src/sampler.cpp:26-31) with `seed`
   (0: the clock, as in the reference): new RNG state, empty window. */
VERBO_CUDA_API int verbo_cuda_batch_reset(verbo_cuda_batch* b, int stream, unsigned long long seed,
                                          void* cuda_stream);
/* Sampler::accept of n host ids (src/sampler.cpp:43-48), e.g. the prompt. */
VERBO_CUDA_API int verbo_cuda_batch_accept(verbo_cuda_batch* b, int stream, const int* ids, int n,
                                           void* cuda_stream);
/* One pick + accept per stream: `logits` holds B device rows of `ld` floats
   (vocab used); out_ids (device, B ints) receives the ids; stats optional. */
VERBO_CUDA_API int verbo_cuda_batch_step(verbo_cuda_batch* b, const float* logits, int vocab, long long ld,
                                         int* out_ids, verbo_row_stats* stats, void* cuda_stream);

/* ---- logits producer tail ------------------------------------------------
   The end of Session::Impl::batch (src/session.cpp:163-169): the final
   RMSNorm of each output row's hidden state (model.norm.weight, eps =
   rms_norm_eps), the activation quantisation of Session::Impl::act
   (src/session.cpp:88-103) for quantised heads, and matmul with the LM head
   (lm_head.weight, or the tied embedding), writing fp32 logits rows straight
   into a device buffer that verbo_cuda_sample / verbo_cuda_batch_step read.
   The logits are bit-identical to those of the reference built with its
   VERBO_SCALAR option; its default SIMD builds sum the same terms in another
   order.  The reference computes this on the host with no device form. */
typedef struct verbo_cuda_tail verbo_cuda_tail;
/* Uploads a head to `device`.  dtype is verbo::DType (include/verbo/verbo.hpp:13):
   0 F32, 1 Q8, 2 Q4.  q and s are HOST arrays in verbo::Tensor layout
   (src/kernels.hpp:13-23): F32 vocab x dim floats (s unused, may be NULL);
   Q8 vocab x dim int8; Q4 vocab x dim/2 bytes (byte i of a 32-block: element i
   in the low nibble, element i+16 in the high one, each stored as value + 8);
   s = vocab x dim/32 fp16 scales for Q8/Q4.  norm: dim host floats.  dim must
   be a multiple of 32 in [32, 16384] (src/model.cpp:108); vocab in [1, 4194304]. */
VERBO_CUDA_API verbo_cuda_tail* verbo_cuda_tail_new(int dtype, int vocab, int dim, const void* q,
                                                    const unsigned short* s, const float* norm, float eps,
                                                    int device);
VERBO_CUDA_API void verbo_cuda_tail_free(verbo_cuda_tail* t);
/* n device rows of hidden state (row i at x + i*ldx, dim floats) -> n device
   rows of logits (row i at logits + i*ld, vocab floats), ordered on `stream`. */
VERBO_CUDA_API int verbo_cuda_tail_logits(verbo_cuda_tail* t, const float* x, int n, long long ldx, float* logits,
                                          long long ld, void* stream);

/* ---- request batching for a server -----------------------------------------
   The reference's server (cli/serve.cpp:139-218) runs one request at a time
   behind a global mutex (:168), each through verbo::generate with the
   request's own Sampling (:149-157).  A verbo_cuda_server keeps up to `slots`
   requests in flight instead, each with its own options and sampler state on
   the device: per step, verbo_cuda_server_prepare admits queued requests
   (Sampler(opts) seeded with opts.seed, then accept(prompt)) and returns which
   request each row of the step belongs to; the caller's model writes each
   active request's next logits row there; verbo_cuda_server_step samples all
   rows (one launch chain per option set) and accepts the ids, a stop id ending
   its request without being emitted and max_tokens the others, as generate
   does (src/sampler.cpp:156-165).  With a penalty, 1 <= repeat_last <=
   max_window (the device ring of the last ids).  Calls on one server are
   serialised by it; use one CUDA stream per server. */
typedef struct verbo_cuda_server verbo_cuda_server;
VERBO_CUDA_API verbo_cuda_server* verbo_cuda_server_new(int slots, int vocab, int max_window, const int* stop_ids,
                                                        int n_stop, int device);
VERBO_CUDA_API void verbo_cuda_server_free(verbo_cuda_server* v);
/* Queues a request (prompt ids host memory, opts->seed != 0); returns its id
   (>= 0) or -1. */
VERBO_CUDA_API long long verbo_cuda_server_submit(verbo_cuda_server* v, const int* prompt, int n,
                                                  const verbo_sampling* opts, int max_tokens);
/* Admits queued requests into free rows and fills row_req[0..slots) with the
   request id of each row of the next step (-1: idle); returns the number of
   active rows A (rows 0..A-1 hold them), 0 when nothing is left. */
VERBO_CUDA_API int verbo_cuda_server_prepare(verbo_cuda_server* v, long long* row_req, void* cuda_stream);
/* Samples the prepared step from A logits rows (row r at logits + r*ld, vocab
   floats, host or device memory); returns how many requests finished. */
VERBO_CUDA_API int verbo_cuda_server_step(verbo_cuda_server* v, const float* logits, long long ld, void* cuda_stream);
/* A request's ids so far (up to cap into tokens), their count and whether it
   ended on a stop id; returns 1 once it finished, 0 before; with release = 1
   a finished request is forgotten. */
VERBO_CUDA_API int verbo_cuda_server_result(verbo_cuda_server* v, long long id, int* tokens, int cap, int* n_tokens,
                                            int* stopped, int release);

/* ---- one decode step of B concurrent generations --------------------------
   The end of Session::Impl::batch (src/session.cpp:163-169) for the last row
   of each of B sessions, followed by the pick + accept of verbo::generate
   (src/sampler.cpp:156-165) for each: `hidden` holds B rows of final hidden
   state (row i, the residual of generation i's last position before the
   final norm, at hidden + i*ldx, dim floats; host or device memory) ->
   verbo_cuda_tail_logits into device rows the batch owns ->
   verbo_cuda_batch_step on them.  The logits never leave the device.
   out_ids (B ints) and stats (B rows, optional) may be host or device
   memory; with either on the host the call returns once they are written,
   otherwise it is ordered on `cuda_stream`.  `t` and `b` must live on the
   same device; B is the batch's stream count.  The reference runs one
   Session and one Sampler per generation on the host, with no batched form. */
VERBO_CUDA_API int verbo_cuda_batch_decode(verbo_cuda_batch* b, verbo_cuda_tail* t, const float* hidden,
                                           long long ldx, int* out_ids, verbo_row_stats* stats, void* cuda_stream);

#ifdef __cplusplus
}
#endif

#endif
