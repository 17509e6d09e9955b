// The reference's sampler known answers (tests/test_core.cpp:454-495) through
// the header-only C++ wrapper verbo::cuda::Sampler.  Exit 0 on success,
// 1 on a wrong answer, 2 if the library reported an error.
#include <cstdio>
#include <vector>

#include "verbo_cuda.hpp"

int main() {
  std::vector<float> lg = {0.1f, 3.0f, 2.9f, -1.0f, 0.0f};
  try {
    verbo::cuda::Sampling g;
    g.temp = 0.0f;
    verbo::cuda::Sampler greedy(g);
    const int a = greedy.pick(lg.data(), 5);
    verbo::cuda::Sampling rp;
    rp.temp = 0.0f;
    rp.repeat = 2.0f;
    verbo::cuda::Sampler sr(rp);
    sr.accept(1);
    const int b = sr.pick(lg.data(), 5);
    sr.reset();
    const int c = sr.pick(lg.data(), 5);
    verbo::cuda::Sampling t2;
    t2.seed = 42;
    t2.top_k = 2;
    t2.top_p = 1.0f;
    verbo::cuda::Sampler x(t2), y(t2);
    int ones = 0, agree = 1;
    for (int i = 0; i < 400; ++i) {
      const int u = x.pick(lg.data(), 5), v = y.pick(lg.data(), 5);
      agree &= u == v && (u == 1 || u == 2);
      ones += u == 1;
    }
    std::printf("ok %d %d %d %d %d\n", a, b, c, agree, ones);
    return (a == 1 && b == 2 && c == 1 && agree && ones > 150 && ones < 300) ? 0 : 1;
  } catch (const std::exception& e) {
    std::printf("error %s\n", e.what());
    return 2;
  }
}
