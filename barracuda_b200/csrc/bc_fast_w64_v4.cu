// bc_fast_w64_v4.cu -- instantiates the fast NTT kernels for 64-bit words, q < 2^62, schedule variant 4.
#include "bc_kernels_fast.cuh"

namespace bc {
namespace fast {
template int dispatch_l<Arith64, 4>(uint32_t L, bool gs, bool scale, const KArgs &a, cudaStream_t s);
template int dispatch_polymul_l<Arith64, 4>(uint32_t L, const KArgs &a, cudaStream_t s);
template int dispatch_ntt_mul_l<Arith64, 4>(uint32_t L, bool inverse, const KArgs &a, cudaStream_t s);
}  // namespace fast
}  // namespace bc
