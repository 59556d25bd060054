// bc_fast_w32l4_v4.cu -- instantiates the fast NTT kernels for 32-bit words, q < 2^30, schedule variant 4.
#include "bc_kernels_fast.cuh"

namespace bc {
namespace fast {
template int dispatch_l<Arith32<true>, 4>(uint32_t L, bool gs, bool scale, const KArgs &a, cudaStream_t s);
template int dispatch_polymul_l<Arith32<true>, 4>(uint32_t L, const KArgs &a, cudaStream_t s);
template int dispatch_ntt_mul_l<Arith32<true>, 4>(uint32_t L, bool inverse, const KArgs &a, cudaStream_t s);
}  // namespace fast
}  // namespace bc
