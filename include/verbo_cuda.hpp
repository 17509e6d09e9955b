// verbo_cuda.hpp - header-only C++ face of the B200 sampler (include/verbo_cuda.h).
//
// verbo::cuda::Sampler keeps the interface of verbo::Sampler
// (include/verbo/verbo.hpp:116-132): construct from a Sampling, pick(logits, n),
// accept(tok), reset(), cfg().  Errors that the C ABI reports as -1 become
// std::runtime_error with verbo_cuda_last_error().  verbo::cuda::Sampling has
// the fields and defaults of verbo::Sampling (include/verbo/verbo.hpp:56-64).
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>

#include "verbo_cuda.h"

namespace verbo {
namespace cuda {

struct Sampling {
  float temp = 0.7f;
  int top_k = 40;
  float top_p = 0.9f;
  float min_p = 0.0f;
  float repeat = 1.0f;
  int repeat_last = 64;
  std::uint64_t seed = 0;

  verbo_sampling c() const { return verbo_sampling{temp, top_k, top_p, min_p, repeat, repeat_last, seed}; }
};

inline void check(int rc) {
  if (rc < 0) throw std::runtime_error(verbo_cuda_last_error());
}

// One generation stream's sampler on a CUDA device.  pick() accepts host or
// device logits; the RNG state and penalty history live with the object, as
// in verbo::Sampler.  Not thread-safe (neither is verbo::Sampler).
class Sampler {
 public:
  explicit Sampler(Sampling cfg = {}, int device = 0) : cfg_(cfg) {
    const verbo_sampling c = cfg.c();
    h_ = verbo_cuda_sampler_new(&c, device);
    if (!h_) throw std::runtime_error(verbo_cuda_last_error());
  }
  ~Sampler() { verbo_cuda_sampler_free(h_); }
  Sampler(const Sampler&) = delete;
  Sampler& operator=(const Sampler&) = delete;
  Sampler(Sampler&& o) noexcept : cfg_(o.cfg_), h_(o.h_) { o.h_ = nullptr; }
  Sampler& operator=(Sampler&& o) noexcept {
    if (this != &o) {
      verbo_cuda_sampler_free(h_);
      cfg_ = o.cfg_;
      h_ = o.h_;
      o.h_ = nullptr;
    }
    return *this;
  }

  int pick(const float* logits, int n) {
    const int id = verbo_cuda_sampler_pick(h_, logits, n);
    check(id);
    return id;
  }
  void accept(int tok) { check(verbo_cuda_sampler_accept(h_, tok)); }
  void reset() { check(verbo_cuda_sampler_reset(h_)); }
  const Sampling& cfg() const { return cfg_; }

 private:
  Sampling cfg_;
  verbo_cuda_sampler* h_ = nullptr;
};

// B generation streams whose Sampler state (RNG, penalty window) lives on the
// device: the batched form of the loop in verbo::generate.  step() samples
// one id per stream from B device rows and accepts it on the device.
class Batch {
 public:
  Batch(Sampling cfg, int streams, int device = 0) : cfg_(cfg) {
    const verbo_sampling c = cfg.c();
    h_ = verbo_cuda_batch_new(&c, streams, device);
    if (!h_) throw std::runtime_error(verbo_cuda_last_error());
  }
  ~Batch() { verbo_cuda_batch_free(h_); }
  Batch(const Batch&) = delete;
  Batch& operator=(const Batch&) = delete;

  void reset(int stream, std::uint64_t seed, void* cuda_stream = nullptr) {
    check(verbo_cuda_batch_reset(h_, stream, seed, cuda_stream));
  }
  void accept(int stream, const int* ids, int n, void* cuda_stream = nullptr) {
    check(verbo_cuda_batch_accept(h_, stream, ids, n, cuda_stream));
  }
  void step(const float* d_logits, int vocab, long long ld, int* d_out_ids, void* cuda_stream = nullptr) {
    check(verbo_cuda_batch_step(h_, d_logits, vocab, ld, d_out_ids, nullptr, cuda_stream));
  }
  const Sampling& cfg() const { return cfg_; }

 private:
  Sampling cfg_;
  verbo_cuda_batch* h_ = nullptr;
};

// The logits producer tail (verbo_cuda_tail_*): the final RMSNorm and LM head
// of Session::Impl::batch (src/session.cpp:163-169) on the device.  dtype is
// verbo::DType as an int (0 F32, 1 Q8, 2 Q4); q / s / norm are the host
// arrays of the loaded model's head Tensor and norm weight.
class Tail {
 public:
  Tail(int dtype, int vocab, int dim, const void* q, const unsigned short* s, const float* norm, float eps,
       int device = 0) {
    h_ = verbo_cuda_tail_new(dtype, vocab, dim, q, s, norm, eps, device);
    if (!h_) throw std::runtime_error(verbo_cuda_last_error());
  }
  ~Tail() { verbo_cuda_tail_free(h_); }
  Tail(const Tail&) = delete;
  Tail& operator=(const Tail&) = delete;

  // n device rows of hidden state (stride ldx) -> n device rows of logits (stride ld)
  void logits(const float* d_x, int n, long long ldx, float* d_logits, long long ld, void* cuda_stream = nullptr) {
    if (verbo_cuda_tail_logits(h_, d_x, n, ldx, d_logits, ld, cuda_stream) < 0)
      throw std::runtime_error(verbo_cuda_last_error());
  }

 private:
  verbo_cuda_tail* h_ = nullptr;
};

}  // namespace cuda
}  // namespace verbo
