// set_seed / randn with the reference runtime's semantics
// (runtime/ops/elementwise.inc:30-55): one global std::mt19937, seeded from
// std::random_device until set_seed is called; randn fills row-major with
// std::normal_distribution<double>(0, 1), a fresh distribution per call.
//
// Built with the reference's flags (-O3 -ffast-math -mavx2 -mfma, as
// `dream run` compiles the runtime): the distribution is a header template
// instantiated here, and those flags decide the last bit of its output, so a
// program gets the same inputs on this runtime as on the reference.
#include <random>

#include "dream_b200.h"

static std::mt19937& rng() {
  static std::mt19937 r(std::random_device{}());
  return r;
}

extern "C" Tensor* dream_set_seed(Tensor* seed_t) {
  const unsigned seed = seed_t ? (unsigned)seed_t->data[0] : 42u;
  rng().seed(seed);
  return create_scalar((double)seed);
}

extern "C" Tensor* dream_randn(Tensor* d0, Tensor* d1) {
  Tensor* t = alloc_tensor((int)d0->data[0], (int)d1->data[0], 1, 1);
  std::normal_distribution<double> dist(0.0, 1.0);
  for (int i = 0; i < t->size; ++i) t->data[i] = dist(rng());
  return t;
}
