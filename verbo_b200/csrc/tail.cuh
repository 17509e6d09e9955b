// Launch-side view of the logits producer tail (shared by tail.cu and capi.cpp).
//
// The tail of Session::Impl::batch (src/session.cpp:163-169): the final
// RMSNorm of the last hidden states, the activation quantisation of
// Session::Impl::act (src/session.cpp:88-103) for quantised heads, and the LM
// head matmul, writing fp32 logits rows straight into the sampler's input
// buffer.  Results are bit-identical to the reference's scalar build
// (VERBO_SCALAR) and follow its rounding step by step.
//
// Device layouts (HBM):
//   quantised head   tile-major: for each tile of kTailRows vocab rows and
//                    each K chunk of kTailChunk elements, one contiguous block
//                    of the tile's weight bytes for the chunk (row stride
//                    kTailChunk for Q8, kTailChunk/2 for Q4, 16-byte units
//                    XOR-swizzled per row) followed by its fp16 scales (4 per
//                    row).  Rows past the vocab and K past dim are zeros.  A
//                    pipeline stage is one bulk copy of such a block.
//   activations      one block per (K chunk, token tile of nt tokens), chunk
//                    major: the nt x kTailChunk int8 codes (16-byte units
//                    XOR-swizzled by (token & 7)) then their block scales as
//                    [4 blocks][nt] fp32; tokens past n are zeros.  A stage
//                    takes one such block with one bulk copy.
//   F32 head         tile-major too: for each tile of kTailRows rows and each
//                    32 floats of K, a 16 KB block (16-byte units swizzled by
//                    row & 7); its normalised rows xb are blocks of
//                    [32 floats of K][nt tokens] per (K block, token tile).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace vb {

constexpr int kTailBlk = 32;        // quantisation block (src/kernels.hpp:11)
constexpr int kTailChunk = 128;     // K elements of one pipeline stage: 4 blocks
constexpr int kTailRows = 128;      // vocab rows of one head tile
constexpr int kTailThreads = 256;
constexpr int kTailMaxDim = 16384;
constexpr int kTailMaxVocab = 1 << 22;
constexpr unsigned kErrTailWait = 4u;  // a head-kernel pipeline wait hit its time limit

enum TailDtype { kTailF32 = 0, kTailQ8 = 1, kTailQ4 = 2 };  // verbo::DType values

// A head resident in HBM.
struct TailHead {
  int dtype;
  int vocab;
  int dim;
  int dimp;                    // dim rounded up to kTailChunk
  int nkc;                     // dimp / kTailChunk
  int ntile;                   // vocab tiles of kTailRows
  const unsigned char* tiles;  // the tile-major head
  const float* norm;           // dim floats
  float eps;
};

// One call: n hidden rows in, n logits rows out.
struct TailArgs {
  const float* x;      // n rows, row i at x + i*ldx
  long long ldx;
  int n;
  int n_pad;           // n rounded up to the token tile of the head kernel
  int nt;              // token tile (quantised heads 8, 16, 32 or 64; F32 heads 2, 4, 8 or 16)
  float* logits;       // n rows, row i at logits + i*ld
  long long ld;
  unsigned char* act;  // scratch (Q8/Q4): the activation blocks
  float* xb;           // scratch (F32): the activation blocks
};

// Bytes of the tile-major form of a quantised head, and the packing itself
// (host memory to host memory) from the reference's Tensor layout.
size_t tail_tiles_bytes(int dtype, int vocab, int dim);
void tail_pack_tiles(int dtype, int vocab, int dim, const void* q, const uint16_t* s, unsigned char* out);

int tail_token_tile(const TailHead& h, int n);
size_t tail_scratch_bytes(const TailHead& h, int n);
void tail_scratch_attach(const TailHead& h, int n, void* base, TailArgs& a);
cudaError_t launch_tail(const TailHead& h, const TailArgs& a, cudaStream_t s);
// Reads (and optionally clears) the tail kernels' error bits; the caller has
// synchronised the stream.
cudaError_t tail_read_status(unsigned* st, bool clear);

}  // namespace vb
