// The register-stack mul_mat's instances (k_mul_mat_short), in a translation
// unit of their own so that the kernel instances compile in parallel.
#define SHLO_MUL_MAT_INSTANCES
#include "mul_mat.cuh"

namespace shlo {
void launch_mul_mat_short(int ng, bool epi, unsigned grid, cudaStream_t stream, const MMArgs &a) {
#define SHLO_MS(NG)                                                              \
  (epi ? k_mul_mat_short<true, NG><<<grid, ms::THREADS, 0, stream>>>(a)          \
       : k_mul_mat_short<false, NG><<<grid, ms::THREADS, 0, stream>>>(a))
  switch (ng) {
    case 1: SHLO_MS(1); break;
    case 2: SHLO_MS(2); break;
    case 3: SHLO_MS(3); break;
    default: SHLO_MS(4); break;
  }
#undef SHLO_MS
}
}  // namespace shlo
