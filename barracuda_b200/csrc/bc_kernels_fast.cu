// bc_kernels_fast.cu -- selection and dispatch of the fast NTT kernels
// (templates in bc_kernels_fast.cuh, instantiated per arithmetic flavour in
// bc_fast_*.cu so that they compile in parallel).
#include <cstdint>
#include <cstdlib>

#include "bc_common.hpp"
#include "bc_kernels.hpp"

namespace bc {
namespace fast {
template <class A, int LOGE>
int dispatch_l(uint32_t L, bool gs, bool scale, const KArgs &a, cudaStream_t s);
}  // namespace fast

namespace {
// Coefficients per thread (log2) of the fast kernel for a word size and N:
// BARRACUDA_NTT_ELEMS=16|32 overrides the default for 32-bit words.
uint32_t fast_loge(Word w, uint32_t logn) {
    if (w == Word::W64) return 4;
    static const int env = [] {
        const char *e = std::getenv("BARRACUDA_NTT_ELEMS");
        return e ? std::atoi(e) : 0;
    }();
    if (env == 16 && logn <= 16) return 4;
    if (env == 32) return 5;
    // 16 coefficients per thread keep two 512-thread CTAs with their
    // staging buffers resident per SM; N = 2^17 needs 32 (cluster of 8)
    return logn <= 16 ? 4 : 5;
}

uint32_t sched_logc(uint32_t logn, uint32_t loge) {
    // local words per CTA: 2^14 for 32 coefficients per thread, 2^13 for 16
    const uint32_t cap = loge == 5 ? 14 : 13;
    return logn > cap ? logn - cap : 0;
}
}  // namespace

bool fast_supported(Word w, uint32_t logn) {
    if (w == Word::W64) return logn >= 10 && logn <= 16;
    return logn >= 10 && logn <= 17;
}

int fast_cluster_size(Word w, uint32_t logn) {
    if (!fast_supported(w, logn)) return 1;
    return 1 << sched_logc(logn, fast_loge(w, logn));
}

int launch_ntt_fast(Word w, bool gs, bool scale_last, const KArgs &a, cudaStream_t s) {
    const uint32_t loge = fast_loge(w, a.logn);
    switch (w) {
    case Word::W32Lazy4:
        return loge == 4 ? fast::dispatch_l<Arith32<true>, 4>(a.logn, gs, scale_last, a, s)
                         : fast::dispatch_l<Arith32<true>, 5>(a.logn, gs, scale_last, a, s);
    case Word::W32Lazy2:
        return loge == 4 ? fast::dispatch_l<Arith32<false>, 4>(a.logn, gs, scale_last, a, s)
                         : fast::dispatch_l<Arith32<false>, 5>(a.logn, gs, scale_last, a, s);
    default: return fast::dispatch_l<Arith64, 4>(a.logn, gs, scale_last, a, s);
    }
}

}  // namespace bc
