// The TMEM-stack mul_mat's instances for tiles split over 16 CTAs (SPLIT 16), in a
// translation unit of their own so that the kernel instances compile in parallel.
#define SHLO_MUL_MAT_INSTANCES
#include "mul_mat.cuh"

namespace shlo {
template cudaError_t mul_mat_tm_attributes<16>();
template void launch_mul_mat_tm<16>(int, bool, int, unsigned, cudaStream_t, const MMArgs &, const CUtensorMap &,
                                      const CUtensorMap &);
}  // namespace shlo
