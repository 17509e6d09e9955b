// Device helpers shared by the sampling kernels (kernels.cu, nucleus.cu):
// the reference's RNG draw, the batched streams' penalty ring, row stats.
#pragma once

#include "device.cuh"
#include "kernels.cuh"

namespace vb {

// Sampler::accept (src/sampler.cpp:43-48) of a batched stream on the device:
// the ring keeps the last ring_len ids, which is all the penalty window reads.
__device__ __forceinline__ void ring_append(const RowArgs& a, int row, int id) {
  if (!a.ring_pos) return;
  const long long p = a.ring_pos[row];
  a.win[static_cast<long long>(row) * a.win_w + p % a.ring_len] = id;
  a.ring_pos[row] = p + 1;
}

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

}  // namespace vb
