// Launch-side view of the logits producer tail (shared by tail.cu and capi.cpp).
//
// The tail of Session::Impl::batch (src/session.cpp:163-169): the final
// RMSNorm of the last hidden states, the activation quantisation of
// Session::Impl::act (src/session.cpp:88-103) for quantised heads, and the LM
// head matmul, writing fp32 logits rows straight into the sampler's input
// buffer.  Results are bit-identical to the reference's scalar build
// (VERBO_SCALAR) and follow its rounding step by step.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace vb {

constexpr int kTailBlk = 32;        // quantisation block (src/kernels.hpp:11)
constexpr int kTailChunk = 128;     // K elements of one pipeline stage: 4 blocks
constexpr int kTailRows = 128;      // vocab rows of one CTA tile (quantised heads)
constexpr int kTailThreads = 256;
constexpr int kTailStages = 4;
constexpr int kTailMaxDim = 16384;
constexpr int kTailMaxVocab = 1 << 22;

enum TailDtype { kTailF32 = 0, kTailQ8 = 1, kTailQ4 = 2 };  // verbo::DType values

// A head resident in HBM.
struct TailHead {
  int dtype;
  int vocab;
  int dim;
  int dimp;            // dim rounded up to kTailChunk
  int nbp;             // dimp / kTailBlk: scale blocks per row, zero-padded
  const void* q;       // reference layout: F32 vocab x dim floats, Q8 vocab x dim int8, Q4 vocab x dim/2 bytes
  const uint16_t* s;   // Q8/Q4: vocab x nbp fp16 bits (the reference's scales, zero-padded per row)
  const float* norm;   // dim floats
  float eps;
};

// One call: n hidden rows in, n logits rows out.
struct TailArgs {
  const float* x;      // n rows, row i at x + i*ldx
  long long ldx;
  int n;
  float* logits;       // n rows, row i at logits + i*ld
  long long ld;
  int8_t* xq;          // scratch: n x dimp quantised activations (Q8/Q4)
  float* xs;           // scratch: n x nbp block scales (Q8/Q4)
  float* xb;           // scratch: n x dimp normalised rows (F32)
};

size_t tail_scratch_bytes(const TailHead& h, int n);
void tail_scratch_attach(const TailHead& h, int n, void* base, TailArgs& a);
cudaError_t launch_tail(const TailHead& h, const TailArgs& a, cudaStream_t s);
int tail_kernels_per_call(const TailHead& h);

}  // namespace vb
