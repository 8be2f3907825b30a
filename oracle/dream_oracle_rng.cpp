// TEST INFRASTRUCTURE — NOT PART OF THE PRODUCT.
//
// The reference's seeded RNG, restated so tests can regenerate the exact
// inputs a Dream program gets from set_seed/randn. This file is compiled with
// the flags `dream run` compiles the runtime with (src/main.cpp:994:
// -O3 -ffast-math -mavx2 -mfma): std::normal_distribution is a header
// template instantiated in the caller's translation unit, and fast-math
// changes the last bit of some of its outputs, so other flags would give a
// stream that differs from the reference's in the final ulp.
#include <cstdint>
#include <random>

extern "C" {

// ---------------------------------------------------------------- RNG
// The reference seeds one global std::mt19937 (set_seed, runtime/ops/
// elementwise.inc:30-41) and draws std::normal_distribution<double>(0,1)
// element by element for randn (:48-55). A fresh distribution object is
// built per randn call, so no cached second normal carries across calls.
static std::mt19937& rng() {
  static std::mt19937 r(42);
  return r;
}
void orc_set_seed(unsigned seed) { rng().seed(seed); }
void orc_randn(double* out, long n) {
  std::normal_distribution<double> dist(0.0, 1.0);
  for (long i = 0; i < n; ++i) out[i] = dist(rng());
}
void orc_rand_uniform(double* out, long n, double lo, double hi) {
  std::uniform_real_distribution<double> dist(lo, hi);
  for (long i = 0; i < n; ++i) out[i] = dist(rng());
}

}  // extern "C"
