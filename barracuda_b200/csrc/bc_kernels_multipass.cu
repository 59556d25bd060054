// bc_kernels_multipass.cu -- pass schedule, table layout and launches of the
// multi-pass transform (kernels in bc_kernels_multipass.cuh).
#include <atomic>
#include <cstdint>

#include "bc_common.hpp"
#include "bc_kernels.hpp"
#include "bc_kernels_multipass.cuh"

namespace bc {
namespace {

// Pass widths, lowest bits first.  A tile is 32 x 2^S words: 64 KB at most
// (S <= 9 for 32-bit words, S <= 8 for 64-bit words).  N = 2^18 with 32-bit
// words takes two passes of 9 bits (24N bytes of HBM traffic); everything
// else three passes (32N bytes).  The TOP pass needs S >= 5 and lo >= 5, the
// MID / LOW passes lo + S <= L - 5; every split below satisfies both.
struct Sched {
    int n;
    int bits[3];  // LOW, (MID,) TOP
};

Sched schedule(Word w, uint32_t L) {
    Sched s{};
    if (w != Word::W64 && L == 18) {
        s.n = 2;
        s.bits[0] = 9;
        s.bits[1] = 9;
        return s;
    }
    s.n = 3;
    const int base = static_cast<int>(L) / 3, extra = static_cast<int>(L) % 3;
    s.bits[0] = base;                       // LOW
    s.bits[1] = base + (extra >= 2 ? 1 : 0);  // MID
    s.bits[2] = base + (extra >= 1 ? 1 : 0);  // TOP
    return s;
}

bool schedule_ok(Word, uint32_t L) { return L >= 18 && L <= 24; }

int check_launch_mp(const char *what) {
    const cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) return BC_OK;
    return fail(e == cudaErrorMemoryAllocation ? BC_ERR_OUT_OF_MEMORY : BC_ERR_GPU,
                format("%s launch failed: %s", what, cudaGetErrorString(e)));
}

template <class A, bool GS, bool SCALE, int S, int ROLE>
int launch_pass(const KArgs &a, void *scratch, uint32_t lo, cudaStream_t s) {
    using W = typename A::W;
    const size_t smem = sizeof(W) * (32u << S);
    // the shared-memory attribute is set once per device (each device loads
    // its own copy of the kernel); concurrent first calls only repeat it
    static std::atomic<bool> attr_set[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 64 || !attr_set[dev].load()) {
        const cudaError_t e = cudaFuncSetAttribute(mp::k_ntt_pass<A, GS, SCALE, S, ROLE>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return cuda_fail(e, "multi-pass transform shared memory");
        if (dev < 64) attr_set[dev].store(true);
    }
    const uint32_t tile_bits = ROLE == mp::kTop ? lo - 5 : a.logn - 5 - S;
    const uint64_t blocks = (static_cast<uint64_t>(a.batch) * a.n_limbs) << tile_bits;
    if (blocks > 0x7FFFFFFFull) return fail(BC_ERR_UNSUPPORTED, "batch too large for the multi-pass transform");
    mp::k_ntt_pass<A, GS, SCALE, S, ROLE><<<static_cast<unsigned>(blocks), mp::kThreads, smem, s>>>(
        a, static_cast<W *>(scratch), lo);
    return check_launch_mp("k_ntt_pass");
}

template <class A, bool GS, bool SCALE, int ROLE>
int launch_pass_s(int S, const KArgs &a, void *scratch, uint32_t lo, cudaStream_t s) {
    switch (S) {
    case 6: return launch_pass<A, GS, SCALE, 6, ROLE>(a, scratch, lo, s);
    case 7: return launch_pass<A, GS, SCALE, 7, ROLE>(a, scratch, lo, s);
    case 8: return launch_pass<A, GS, SCALE, 8, ROLE>(a, scratch, lo, s);
    case 9:
        if constexpr (A::kBits == 32) return launch_pass<A, GS, SCALE, 9, ROLE>(a, scratch, lo, s);
        [[fallthrough]];
    default: return fail(BC_ERR_INTERNAL, format("no multi-pass tile of %d bits", S));
    }
}

template <class A, bool GS>
int run_passes(const KArgs &a, void *scratch, bool scale, cudaStream_t s, Word w) {
    const Sched sc = schedule(w, a.logn);
    // pass p covers bits [lo[p], lo[p] + bits[p]), p = 0 the lowest
    uint32_t lo[3] = {0, 0, 0};
    for (int p = 1; p < sc.n; ++p) lo[p] = lo[p - 1] + static_cast<uint32_t>(sc.bits[p - 1]);
    const int top = sc.n - 1;
    for (int k = 0; k < sc.n; ++k) {
        const int p = GS ? k : sc.n - 1 - k;  // CT from the top bits down, GS from the bottom up
        // N^-1 rides on the last stage executed: GS b = L-1 (TOP), CT b = 0 (LOW)
        int st;
        if (p == top)
            st = GS && scale ? launch_pass_s<A, GS, true, mp::kTop>(sc.bits[p], a, scratch, lo[p], s)
                             : launch_pass_s<A, GS, false, mp::kTop>(sc.bits[p], a, scratch, lo[p], s);
        else if (p == 0)
            st = !GS && scale ? launch_pass_s<A, GS, true, mp::kLow>(sc.bits[p], a, scratch, lo[p], s)
                              : launch_pass_s<A, GS, false, mp::kLow>(sc.bits[p], a, scratch, lo[p], s);
        else
            st = launch_pass_s<A, GS, false, mp::kMid>(sc.bits[p], a, scratch, lo[p], s);
        if (st) return st;
    }
    return BC_OK;
}

template <class A>
int run_word(bool gs, bool scale, const KArgs &a, void *scratch, cudaStream_t s, Word w) {
    return gs ? run_passes<A, true>(a, scratch, scale, s, w) : run_passes<A, false>(a, scratch, scale, s, w);
}

}  // namespace

bool multipass_supported(Word w, uint32_t logn) { return schedule_ok(w, logn); }

uint32_t multipass_top_lo(Word w, uint32_t logn) {
    const Sched sc = schedule(w, logn);
    return logn - static_cast<uint32_t>(sc.bits[sc.n - 1]);
}

uint64_t multipass_table_index(uint32_t L, uint32_t top_lo, uint64_t knat) {
    if (knat == 0) return 0;
    uint32_t s = 0;
    while ((knat >> (s + 1)) != 0) ++s;  // block of 2^s entries: stage b = L - 1 - s
    const uint32_t b = L - 1 - s;
    if (b >= top_lo) return knat;  // TOP stages: natural (broadcast reads)
    const uint64_t m = 1ull << s, i = knat - m;
    const uint32_t c = L - b - 6;  // i has c + 5 bits; its top five move innermost
    return m + (((i & ((1ull << c) - 1)) << 5) | (i >> c));
}

int launch_ntt_multipass(Word w, bool gs, bool scale_last, const KArgs &a, void *scratch, cudaStream_t s) {
    if (!schedule_ok(w, a.logn))
        return fail(BC_ERR_INTERNAL, format("multi-pass transform does not cover log2 N = %u", a.logn));
    switch (w) {
    case Word::W32Lazy4: return run_word<Arith32<true>>(gs, scale_last, a, scratch, s, w);
    case Word::W32Lazy2: return run_word<Arith32<false>>(gs, scale_last, a, scratch, s, w);
    default: return run_word<Arith64>(gs, scale_last, a, scratch, s, w);
    }
}

}  // namespace bc
