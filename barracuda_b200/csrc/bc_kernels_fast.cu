// bc_kernels_fast.cu -- selection and dispatch of the fast NTT kernels
// (templates in bc_kernels_fast.cuh, instantiated per arithmetic flavour in
// bc_fast_*.cu so that they compile in parallel).
#include <cstdint>
#include <cstdlib>

#include "bc_common.hpp"
#include "bc_kernels.hpp"
#include "bc_schedule.hpp"

namespace bc {
namespace fast {
template <class A, int LOGE>
int dispatch_l(uint32_t L, bool gs, bool scale, const KArgs &a, cudaStream_t s);
template <class A, int LOGE>
int dispatch_polymul_l(uint32_t L, const KArgs &a, cudaStream_t s);
template <class A, int LOGE>
int dispatch_ntt_mul_l(uint32_t L, bool inverse, const KArgs &a, cudaStream_t s);
}  // namespace fast

namespace {
// Schedule variant of the fast kernel for a word size and N (see
// gen_schedule.py): 4 = 16 coefficients per thread in 512-thread CTAs,
// 5 = 32 per thread in CTAs of up to 2^14 words, 6 = 32 per thread in
// 256-thread CTAs, 7 = 32 per thread in 128-thread CTAs.
// BARRACUDA_NTT_VARIANT=4|5|6|7 overrides the default for 32-bit words where
// that schedule exists.
int env_int(const char *name) {
    const char *e = std::getenv(name);
    return e ? std::atoi(e) : 0;
}

int fast_variant(Word w, uint32_t logn, bool inverse) {
    if (w == Word::W64) return 4;
    static const int env_all = env_int("BARRACUDA_NTT_VARIANT");
    static const int env_fwd = env_int("BARRACUDA_NTT_VARIANT_FWD");
    static const int env_inv = env_int("BARRACUDA_NTT_VARIANT_INV");
    const int L = static_cast<int>(logn);
    const int e = inverse ? (env_inv ? env_inv : env_all) : (env_fwd ? env_fwd : env_all);
    if (e && fast::sched_logc(L, e) >= 0) return e;
    // Measured on B200 (forward and inverse, ~2 GiB batches): 32 per thread
    // in one CTA of up to 2^13 words (5) wins for N <= 2^13 (0.90 of HBM at
    // 2^12 against 0.80 for 16 per thread, whose loads and stores stay
    // inlined), 256-thread CTAs of 32 per thread for 2^14..2^17 (clusters of
    // 16 at 2^17); 128-thread CTAs (7) lose at 2^16.
    if (L <= 13 && fast::sched_logc(L, 5) >= 0) return 5;
    if (fast::sched_logc(L, 6) >= 0) return 6;
    return 5;
}
}  // namespace

int fast_variant_for(Word w, uint32_t logn, bool inverse) { return fast_variant(w, logn, inverse); }

int cluster_policy() {
    static const int pol = [] {
        const int v = std::getenv("BARRACUDA_CLUSTER_POLICY") ? env_int("BARRACUDA_CLUSTER_POLICY") : 2;
        return v >= 0 && v <= 2 ? v : 2;
    }();
    return pol;
}

uint64_t fast_table_index(uint32_t L, int V, uint64_t knat, int pair) {
    if (knat == 0) return 0;
    uint32_t s = 0;
    while ((knat >> (s + 1)) != 0) ++s;  // m = 2^s butterfly groups
    const uint64_t m = 1ull << s, i = knat - m;
    const int b = static_cast<int>(L) - 1 - static_cast<int>(s);
    const int hi = fast::sched_pass_hi(static_cast<int>(L), V, b);
    const int k = hi - b;
    const uint64_t h = i >> k, j = i & ((1ull << k) - 1);
    const uint64_t H = (1ull << L) >> (hi + 1);
    if (k == 0) return m + h;
    const uint64_t P = static_cast<uint64_t>(pair);
    return m + (j / P) * (P * H) + P * h + (j % P);
}

bool fast_supported(Word w, uint32_t logn) {
    if (w == Word::W64) return logn >= 10 && logn <= 17;
    return logn >= 10 && logn <= 17;
}

int fast_cluster_size(Word w, uint32_t logn) {
    if (!fast_supported(w, logn)) return 1;
    return 1 << fast::sched_logc(static_cast<int>(logn), fast_variant(w, logn, false));
}

int launch_ntt_fast(Word w, bool gs, bool scale_last, const KArgs &a, cudaStream_t s) {
    const int v = fast_variant(w, a.logn, gs || scale_last);
    switch (w) {
    case Word::W32Lazy4:
        if (v == 4) return fast::dispatch_l<Arith32<true>, 4>(a.logn, gs, scale_last, a, s);
        if (v == 6) return fast::dispatch_l<Arith32<true>, 6>(a.logn, gs, scale_last, a, s);
        if (v == 7) return fast::dispatch_l<Arith32<true>, 7>(a.logn, gs, scale_last, a, s);
        return fast::dispatch_l<Arith32<true>, 5>(a.logn, gs, scale_last, a, s);
    case Word::W32Lazy2:
        if (v == 4) return fast::dispatch_l<Arith32<false>, 4>(a.logn, gs, scale_last, a, s);
        if (v == 6) return fast::dispatch_l<Arith32<false>, 6>(a.logn, gs, scale_last, a, s);
        if (v == 7) return fast::dispatch_l<Arith32<false>, 7>(a.logn, gs, scale_last, a, s);
        return fast::dispatch_l<Arith32<false>, 5>(a.logn, gs, scale_last, a, s);
    default: return fast::dispatch_l<Arith64, 4>(a.logn, gs, scale_last, a, s);
    }
}

int launch_ntt_mul_fast(Word w, bool inverse, const KArgs &a, cudaStream_t s) {
    const int v = fast_variant(w, a.logn, inverse);
    switch (w) {
    case Word::W32Lazy4:
        if (v == 4) return fast::dispatch_ntt_mul_l<Arith32<true>, 4>(a.logn, inverse, a, s);
        if (v == 6) return fast::dispatch_ntt_mul_l<Arith32<true>, 6>(a.logn, inverse, a, s);
        if (v == 7) return fast::dispatch_ntt_mul_l<Arith32<true>, 7>(a.logn, inverse, a, s);
        return fast::dispatch_ntt_mul_l<Arith32<true>, 5>(a.logn, inverse, a, s);
    case Word::W32Lazy2:
        if (v == 4) return fast::dispatch_ntt_mul_l<Arith32<false>, 4>(a.logn, inverse, a, s);
        if (v == 6) return fast::dispatch_ntt_mul_l<Arith32<false>, 6>(a.logn, inverse, a, s);
        if (v == 7) return fast::dispatch_ntt_mul_l<Arith32<false>, 7>(a.logn, inverse, a, s);
        return fast::dispatch_ntt_mul_l<Arith32<false>, 5>(a.logn, inverse, a, s);
    default: return fast::dispatch_ntt_mul_l<Arith64, 4>(a.logn, inverse, a, s);
    }
}

int launch_polymul_fast(Word w, const KArgs &a, cudaStream_t s) {
    const int v = fast_variant(w, a.logn, false);
    if (v != fast_variant(w, a.logn, true))
        return fail(BC_ERR_INTERNAL, "fused polymul needs one schedule for both directions");
    switch (w) {
    case Word::W32Lazy4:
        if (v == 4) return fast::dispatch_polymul_l<Arith32<true>, 4>(a.logn, a, s);
        if (v == 6) return fast::dispatch_polymul_l<Arith32<true>, 6>(a.logn, a, s);
        if (v == 7) return fast::dispatch_polymul_l<Arith32<true>, 7>(a.logn, a, s);
        return fast::dispatch_polymul_l<Arith32<true>, 5>(a.logn, a, s);
    case Word::W32Lazy2:
        if (v == 4) return fast::dispatch_polymul_l<Arith32<false>, 4>(a.logn, a, s);
        if (v == 6) return fast::dispatch_polymul_l<Arith32<false>, 6>(a.logn, a, s);
        if (v == 7) return fast::dispatch_polymul_l<Arith32<false>, 7>(a.logn, a, s);
        return fast::dispatch_polymul_l<Arith32<false>, 5>(a.logn, a, s);
    default: return fast::dispatch_polymul_l<Arith64, 4>(a.logn, a, s);
    }
}

}  // namespace bc
