// Harness over the reference's own compiled verbo::Sampler - TEST
// INFRASTRUCTURE ONLY.  Linked with the reference's sources (compiled
// unmodified by oracle/Makefile into oracle/_ref/), it drives the stock
// Sampler exactly as verbo::generate does (src/sampler.cpp:116-158):
// construct with the options, accept() every history id, then pick().
//
// Two uses: it pins the C restatement (oracle/sampler_oracle.c) and the golden
// fixtures under tests/golden/, and it is the timed CPU baseline of bench.py.
#include <algorithm>
#include <thread>
#include <vector>

#include "oracle.h"
#include "verbo/verbo.hpp"

extern "C" int ref_sample_rows(const float* logits, int rows, int vocab, long long ld, const int* hist,
                               const long long* hist_off, const oracle_sampling* o,
                               const unsigned long long* seeds, int steps, int* out_ids, int threads) {
  if (rows <= 0) return 0;
  if (threads < 1) threads = 1;
  if (threads > rows) threads = rows;
  auto work = [&](int r0, int r1) {
    for (int r = r0; r < r1; ++r) {
      verbo::Sampling s;
      s.temp = o->temp;
      s.top_k = o->top_k;
      s.top_p = o->top_p;
      s.min_p = o->min_p;
      s.repeat = o->repeat;
      s.repeat_last = o->repeat_last;
      s.seed = seeds ? seeds[r] : 1;
      verbo::Sampler smp(s);
      if (hist && hist_off)
        for (long long j = hist_off[r]; j < hist_off[r + 1]; ++j) smp.accept(hist[j]);
      const float* row = logits + static_cast<long long>(r) * ld;
      for (int t = 0; t < steps; ++t) out_ids[static_cast<long long>(r) * steps + t] = smp.pick(row, vocab);
    }
  };
  std::vector<std::thread> pool;
  const int per = (rows + threads - 1) / threads;
  for (int t = 0; t < threads; ++t) {
    const int r0 = t * per, r1 = std::min(rows, r0 + per);
    if (r0 < r1) pool.emplace_back(work, r0, r1);
  }
  for (auto& th : pool) th.join();
  return 0;
}
