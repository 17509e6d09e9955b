// Launch-side view of the sampling kernels (shared by kernels.cu and capi.cpp).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "verbo_cuda.h"

namespace vb {

constexpr int kMaxSlice = 40960;  // largest per-CTA slice of a row (floats) in the staged kernel
constexpr int kMaxVocab = kMaxSlice * 8;
constexpr int kMaxMerge = 4096;   // nshards * k candidates merged per row

// Error bits recorded in the device status word (read by verbo_cuda_check).
constexpr unsigned kErrLoadTimeout = 1u;  // a bulk copy did not complete within the wait limit
constexpr unsigned kErrSelect = 2u;       // a selection found no element

// Sampling options as the kernels use them (built on the host from verbo_sampling).
struct DevOpts {
  float temp, top_p, min_p, repeat;
  int top_k, repeat_last;
  int k;         // candidate count of Sampler::pick: top_k if 0 < top_k < vocab, else vocab
  int greedy;    // temp <= 0
  int penalize;  // repeat != 1 and histories given
  int vocab;     // full vocabulary
  double inv_temp;
};

struct RowArgs {
  const float* logits;
  long long ld;
  int rows;
  int ncols;    // columns processed per row (vocab, or a shard's width)
  int col_off;  // global id of column 0 (shards)
  const int* hist;
  const long long* hist_off;
  unsigned long long* rng;  // 2 per row
  int* out_ids;
  verbo_row_stats* stats;
  float* cand_val;  // shard candidates out, [rows][cand_k]
  int* cand_id;
  uint2* cand_packed;  // or packed (x = value bits, y = id), [rows][cand_k] (used when non-null)
  int cand_k;
  int cluster;  // CTAs per row (a thread-block cluster, or independent slices in the split kernels)
  int slice;    // columns per CTA (multiple of 4)
  int idxbits;  // bits of the largest global id
  int fixbits;  // fixed-point fraction bits of the staged kernel's masses
  // Scratch of the split-row kernels (global memory, see split_scratch_layout):
  unsigned* slice_count;           // [rows * cluster]: candidates each slice published
  unsigned long long* slice_keys;  // [rows * cluster * kSliceCap]: candidate keys (greedy: 1 per slice)
  float* slice_thr;                // [rows * cluster]: top-k slices' emission thresholds (-inf: full top-k)
  int* win;                        // [rows][win_w]: dense penalty windows, -1 padded (win_w > 0)
  int win_w;
  int first_wave;  // split kernel: CTAs resident at launch (SMs x CTAs per SM), set by the launcher
  // Batched streams (verbo_cuda_batch_*): `win` is then each stream's ring of
  // its last ring_len accepted ids (slot = count mod ring_len, -1 = empty),
  // read as the dense window, and the kernel that finishes a row appends the
  // sampled id to it.  ring_pos == nullptr otherwise.
  long long* ring_pos;  // [rows]: ids accepted so far
  int ring_len;
};

// Accepts skip + n ids into row `row`'s ring (batched streams), storing the
// last n = ids[0, n) (n <= ring_len): one CTA.
cudaError_t launch_ring_accept(int* win, int win_w, int ring_len, long long* pos, int row, const int* ids, int n,
                               int skip, cudaStream_t s);
// Row r of the output state takes row from[r] of the input: the RNG state
// (2 words), the penalty ring (win_w ids) and its position.
cudaError_t launch_state_gather(const int* from, int n, const unsigned long long* rng_in, unsigned long long* rng_out,
                                const int* win_in, int* win_out, int win_w, const long long* pos_in,
                                long long* pos_out, cudaStream_t s);

// Split-row kernels: one CTA of kSplitThreads per (row, slice of <= kSplitSlice
// columns) publishes a partial result; a per-row merge kernel follows on the
// same stream.
constexpr int kSplitThreads = 256;
constexpr int kSplitChunks = 10;                                  // 16-byte chunks per thread, in registers
constexpr int kSplitSlice = kSplitThreads * kSplitChunks * 4;     // 10240 columns
constexpr int kSliceCap = 256;                                    // candidates a slice may publish
constexpr int kSplitMaxK = kSliceCap;                             // largest top_k of the split top-k kernel
constexpr int kMaxSlices = 32;
// Top-k slices of rows with >= 2 slices and 32 <= k <= kSplitMaxK emit only
// their top-m, m = max(kTopM, ceil(k / (slices - 1)), ceil(k / 4)), with their
// threshold as a certificate the merge checks (kernels.cu, merge_slices_kernel).
constexpr int kTopM = 16;

// Dense penalty windows: when every row's window (its last repeat_last ids)
// is at most kWinMax long, a small kernel copies the windows into
// [rows][win_w] ahead of the split kernel, whose CTAs then fetch their row's
// window before their logits instead of after them.
constexpr int kWinMax = 2048;
int split_window_width(const DevOpts& o);  // 0: the kernels read the CSR histories directly

// Layout of the split kernels' scratch (nothing in it needs zeroing): per-slice
// counts at offset 0, keys at off_keys (one per slice for greedy, kSliceCap
// for top-k), windows at off_win.
struct SplitScratch {
  size_t off_keys, off_thr, off_win, bytes;
};
SplitScratch split_scratch_layout(long long rows, int slices, bool greedy, int win_w);
void split_scratch_attach(RowArgs& a, void* base, const SplitScratch& l, int win_w);
cudaError_t launch_split(const RowArgs& a, const DevOpts& o, int mode, cudaStream_t s);
enum SplitMode { kSplitGreedy = 0, kSplitSample = 1, kSplitEmit = 2 };

// Allocation-free variant: the split kernel with its scratch in a fixed
// device array of kNoAllocScratchBytes (kernels.cu).  Sets *too_big (and
// launches nothing) when rows x slices need more than that.
constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
cudaError_t launch_split_noalloc(RowArgs& a, const DevOpts& o, int mode, cudaStream_t s, bool* too_big);

struct MergeArgs {
  const float* cand_val;  // [nshards][rows][k]
  const int* cand_id;
  const uint2* cand_packed;  // or packed (x = value bits, y = id), [nshards][rows][k] (used when non-null)
  int rows, nshards, k;
  unsigned long long* rng;
  int* out_ids;
  verbo_row_stats* stats;
};

// Host launchers (kernels.cu).  Return a cudaError_t.
cudaError_t launch_general(const RowArgs& a, const DevOpts& o, cudaStream_t s);
// The staged full-vocabulary kernel over the rows list[0, *count) (device
// memory, read when the kernel starts); max_rows bounds *count.
cudaError_t launch_general_list(const RowArgs& a, const DevOpts& o, const int* list, const unsigned* count,
                                int max_rows, cudaStream_t s);

// Streaming full-vocabulary path (nucleus.cu): top_k == 0 or >= vocab, no
// penalty, vocab >= kNucleusMinVocab (top-p and min-p both taken).  One persistent kernel
// reads every row once from HBM and settles almost every row; the rest go to
// the staged kernel above (launched by launch_nucleus on the same stream).
constexpr int kNucleusMinVocab = 4096;
bool nucleus_eligible(const DevOpts& o, int vocab);
size_t nucleus_scratch_bytes(int rows, int ncols);
cudaError_t launch_nucleus(const RowArgs& a, const DevOpts& o, void* scratch, cudaStream_t s);
// Rows of the last launch_nucleus on `scratch` that went to the staged kernel
// (synchronises the stream).
cudaError_t nucleus_fallbacks(const void* scratch, cudaStream_t s, unsigned* out);
// Device-side failures of the nucleus kernel (bounded waits that ran out).
cudaError_t read_nucleus_status(unsigned* st, bool clear);
cudaError_t launch_merge(const MergeArgs& a, const DevOpts& o, cudaStream_t s);
size_t general_smem(int slice);
cudaError_t read_status(unsigned* st, bool clear, cudaStream_t s);

}  // namespace vb
