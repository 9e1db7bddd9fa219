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
