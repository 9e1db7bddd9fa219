// Host build of contract-stablehlo-mlx_b200/csrc/erff_cr.cuh for the CPU tests:
// exposes the fast+slow correctly rounded erff and the slow path alone.
#include <stdint.h>
#include "../../contract-stablehlo-mlx_b200/csrc/erff_cr.cuh"

extern "C" void erff_cr_bits(const uint32_t *in, uint32_t *out, long n) {
  for (long i = 0; i < n; i++) out[i] = shlo_erf::f2u(shlo_erf::erff_cr(shlo_erf::u2f(in[i])));
}
extern "C" void erff_slow_bits(const uint32_t *in, uint32_t *out, long n) {
  for (long i = 0; i < n; i++) out[i] = shlo_erf::f2u(shlo_erf::erff_slow(shlo_erf::u2f(in[i])));
}
#include <thread>
#include <vector>
// erff_cr of the consecutive patterns base .. base + n - 1, over nthreads threads.
extern "C" void erff_cr_range(uint32_t base, long n, uint32_t *out, int nthreads) {
  std::vector<std::thread> th;
  for (int t = 0; t < nthreads; t++)
    th.emplace_back([=] {
      for (long i = t; i < n; i += nthreads)
        out[i] = shlo_erf::f2u(shlo_erf::erff_cr(shlo_erf::u2f(base + (uint32_t)i)));
    });
  for (auto &x : th) x.join();
}
