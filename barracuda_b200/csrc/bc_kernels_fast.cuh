// bc_kernels_fast.cuh -- the register / shared-memory / thread-block-cluster
// NTT kernels (2^10 <= N <= 2^17) for sm_100a.
//
// One polynomial per cluster of C = 2^kLogC CTAs (C = 1: a single CTA).
// Each thread keeps E = 2^LOGE coefficients in registers and runs the
// butterfly stages of one group of position bits (a "pass", see
// gen_schedule.py / bc_schedule.hpp) in registers; between passes the
// coefficients are exchanged through shared memory, and once through
// distributed shared memory when the cluster changes which CTA owns which
// positions.  HBM is read once (first pass, straight into registers, input
// reduced on the way) and written once (last pass, straight from registers,
// canonical residues), so a transform moves exactly 16N bytes of HBM.
//
// Position convention is the one of bc_kernels_basic.cu: the Cooley-Tukey
// stage flipping bit b uses table entry (N >> (b+1)) + (p >> (b+1)); CT
// reads natural order and leaves position p holding output bitrev(p), which
// the last pass stores at its natural index; GS runs the passes in reverse
// on input loaded from natural index bitrev(p).
#pragma once

#include <atomic>
#include <cstdint>
#include <cstdlib>

#include "bc_common.hpp"
#include "bc_kernels.hpp"
#include "bc_schedule.hpp"

namespace bc {
namespace fast {

// Padded shared-memory word of local index x (see gen_schedule.py): local
// bit i shifts the bank by 2^(i mod 5), and swz(a | b) = swz(a) + swz(b) for
// disjoint a, b, so register-dependent parts become immediate offsets.
__host__ __device__ constexpr uint32_t swz(uint32_t x) { return x + (x >> 5) + (x >> 10) + (x >> 15); }
__host__ __device__ constexpr uint32_t padded_words(uint32_t n) { return swz(n - 1) + 1; }

template <class S>
__host__ __device__ constexpr bool is_rank_bit(int b, int phase) {
    for (int j = 0; j < S::kLogC; ++j)
        if ((phase ? S::rank1(j) : S::rank0(j)) == b) return true;
    return false;
}

// Local index (rank bits of `phase` removed) of a set of position bits.
// Local index of position bits p in a phase: the schedule's per-phase bit
// permutation (rank bits dropped), chosen for conflict-free banks.
template <class S, int L>
__host__ __device__ constexpr uint32_t local_of(uint32_t p, int phase) {
    uint32_t out = 0;
    for (int b = 0; b < L; ++b) {
        const int k = phase ? S::local1(b) : S::local0(b);
        if (k < 0) continue;
        out |= ((p >> b) & 1u) << k;
    }
    return out;
}

template <class S, int L>
__host__ __device__ constexpr uint32_t smem_addr(uint32_t p, int phase) {
    return swz(local_of<S, L>(p, phase));
}

__host__ __device__ constexpr uint32_t brev_c(uint32_t x, int bits) {
    uint32_t r = 0;
    for (int i = 0; i < bits; ++i) r |= ((x >> i) & 1u) << (bits - 1 - i);
    return r;
}

// Position bits contributed by register index m in pass PI.
template <class S, int PI>
__host__ __device__ constexpr uint32_t reg_pos(int m) {
    uint32_t p = 0;
    for (int j = 0; j < S::pass(PI).nreg; ++j) p |= static_cast<uint32_t>((m >> j) & 1) << S::pass(PI).reg[j];
    return p;
}

// Position bits contributed by the thread (lane, warp) and the CTA rank.
template <class S, int PI>
__device__ __forceinline__ uint32_t thread_pos(uint32_t tid, uint32_t rank) {
    constexpr PassDesc P = S::pass(PI);
    uint32_t p = 0;
#pragma unroll
    for (int j = 0; j < 5; ++j) p |= ((tid >> j) & 1u) << P.lane[j];
#pragma unroll
    for (int j = 0; j < P.nwarp; ++j) p |= ((tid >> (5 + j)) & 1u) << P.warp[j];
#pragma unroll
    for (int j = 0; j < S::kLogC; ++j)
        p |= ((rank >> j) & 1u) << (P.phase ? S::rank1(j) : S::rank0(j));
    return p;
}

// Register index whose position is bit 0 (for paired 128-bit accesses), or -1.
template <class S, int PI>
__host__ __device__ constexpr int reg_of_bit0() {
    for (int j = 0; j < S::pass(PI).nreg; ++j)
        if (S::pass(PI).reg[j] == 0) return j;
    return -1;
}

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Cluster barrier without memory ordering: used where every CTA only has to
// have *consumed* (not published) shared-memory data before the next step.
__device__ __forceinline__ void cluster_sync_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t map_rank(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}

template <class W>
__device__ __forceinline__ void st_cluster(uint32_t addr, W v);
template <>
__device__ __forceinline__ void st_cluster<uint32_t>(uint32_t addr, uint32_t v) {
    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
template <>
__device__ __forceinline__ void st_cluster<uint64_t>(uint32_t addr, uint64_t v) {
    asm volatile("st.shared::cluster.u64 [%0], %1;" ::"r"(addr), "l"(v) : "memory");
}

// Keeps x in a register at this point of the program: computations that
// feed it cannot sink below, which bounds how many raw loads are live.
__device__ __forceinline__ void pin(uint32_t &x) { asm volatile("" : "+r"(x)); }
__device__ __forceinline__ void pin(uint64_t &x) { asm volatile("" : "+l"(x)); }
// Memory operations may not move across this point.
__device__ __forceinline__ void compiler_fence() { asm volatile("" ::: "memory"); }

// Twiddle loads through inline PTX: volatile, so their issue order is the
// program order below (the compiler would otherwise hoist every twiddle load
// of a pass to its start and run out of registers).  Read-only path.
__device__ __forceinline__ void ldg_tw(const uint2 *p, uint2 &a, uint2 &b) {
    asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(a.x), "=r"(a.y), "=r"(b.x), "=r"(b.y)
                 : "l"(p));
}
__device__ __forceinline__ void ldg_tw(const uint2 *p, uint2 &a) {
    asm volatile("ld.global.nc.v2.u32 {%0, %1}, [%2];" : "=r"(a.x), "=r"(a.y) : "l"(p));
}
__device__ __forceinline__ void ldg_tw(const ulonglong2 *p, ulonglong2 &a) {
    asm volatile("ld.global.nc.v2.u64 {%0, %1}, [%2];" : "=l"(a.x), "=l"(a.y) : "l"(p));
}

// Asynchronous 16-byte global -> shared copies (L2 only), per thread.
__device__ __forceinline__ void cp_async16(uint32_t saddr, const void *g) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// One-thread bulk copies (TMA, non-tensor form) global -> shared, completed
// through a transaction-counting mbarrier in shared memory.
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
// Orders this thread's earlier generic-proxy shared-memory accesses (made
// visible to it by a barrier) before its following bulk copies.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Arms the barrier's current phase for `bytes` and starts the copy; src and
// dst 16-byte aligned, bytes a multiple of 16 below 2^20.
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Waits for phase `parity` with an iteration limit (each try_wait suspends
// the thread for a hardware-bounded time); false if the limit ran out.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity) {
    for (uint32_t i = 0; i < (1u << 22); ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

// Twiddle chunks of one pass, in execution order.  Stage st of the pass
// (CT: position bits high to low, GS: low to high) uses 2^k twiddles,
// k = hi - b; they are fetched kCh at a time, each chunk `kAhead` chunks
// before the butterflies that consume it.
template <class A, class S, int PI, bool GS>
struct TwSeq {
    static constexpr PassDesc P = S::pass(PI);
    static constexpr int R = P.hi - P.lo + 1;
    static constexpr int kCh = A::kBits == 32 ? 4 : 2;
    __host__ __device__ static constexpr int t_of(int st) { return GS ? st : R - 1 - st; }
    __host__ __device__ static constexpr int k_of(int st) { return P.hi - P.lo - t_of(st); }
    __host__ __device__ static constexpr int cnt_of(int st) { return (1 << k_of(st)) < kCh ? (1 << k_of(st)) : kCh; }
    __host__ __device__ static constexpr int nch_of(int st) { return (1 << k_of(st)) / cnt_of(st); }
    __host__ __device__ static constexpr int total() {
        int n = 0;
        for (int st = 0; st < R; ++st) n += nch_of(st);
        return n;
    }
    __host__ __device__ static constexpr int stage_of(int c) {
        for (int st = 0; st < R; ++st) {
            if (c < nch_of(st)) return st;
            c -= nch_of(st);
        }
        return R - 1;
    }
    __host__ __device__ static constexpr int first_of(int c) {
        for (int st = 0; st < R; ++st) {
            if (c < nch_of(st)) return c * cnt_of(st);
            c -= nch_of(st);
        }
        return 0;
    }
};

template <class A, class S, int L, int PI, bool GS, int C>
__device__ __forceinline__ void load_chunk(typename A::Tw (&w)[TwSeq<A, S, PI, GS>::kCh], const typename A::Tw *tw,
                                           uint32_t h) {
    using Q = TwSeq<A, S, PI, GS>;
    constexpr int st = Q::stage_of(C);
    constexpr int b = Q::P.lo + Q::t_of(st);
    constexpr int k = Q::k_of(st);
    constexpr int cnt = Q::cnt_of(st);
    // The fast table stores the 2^k twiddles of group h of this stage
    // transposed, so that the lanes of a warp (different h) read adjacent
    // words: entry (h, j) at (N >> (b+1)) + (j / P)(P H) + P h + (j % P),
    // H = N >> (hi+1) groups, P = 2 for 8-byte entries (two per 16-byte
    // load) and 1 for 16-byte entries.  See fast_table_index().
    constexpr uint32_t H = (1u << L) >> (Q::P.hi + 1);
    const typename A::Tw *base = tw + ((1u << L) >> (b + 1));
    constexpr int j0 = Q::first_of(C);
    if constexpr (A::kBits == 32) {
        if constexpr (k == 0) {
            ldg_tw(base + h, w[0]);
        } else {
#pragma unroll
            for (int j = 0; j < cnt; j += 2) ldg_tw(base + (j0 + j) * H + 2 * h, w[j], w[j + 1]);
        }
    } else {
#pragma unroll
        for (int j = 0; j < cnt; ++j) ldg_tw(base + (j0 + j) * H + h, w[j]);
    }
}

template <class A, class S, int PI, bool GS, int SCALE_STAGE, int C>
__device__ __forceinline__ void compute_chunk(typename A::W (&v)[1 << S::pass(PI).nreg],
                                              const typename A::Tw (&w)[TwSeq<A, S, PI, GS>::kCh],
                                              const LimbConst &lc) {
    using W = typename A::W;
    using Q = TwSeq<A, S, PI, GS>;
    constexpr int st = Q::stage_of(C);
    constexpr int t = Q::t_of(st);
    constexpr int R = Q::R;
    constexpr int E = 1 << Q::P.nreg;
    constexpr int first = Q::first_of(C), cnt = Q::cnt_of(st);
    const W q = static_cast<W>(lc.q);
#pragma unroll
    for (int m = 0; m < E; ++m) {
        if (m & (1 << t)) continue;
        const int j = (m & ((1 << R) - 1)) >> (t + 1);
        if (j < first || j >= first + cnt) continue;
        const int m2 = m | (1 << t);
        const typename A::Tw wj = w[j - first];
        if constexpr (st == SCALE_STAGE) {
            const W s = static_cast<W>(lc.ninv), sq = static_cast<W>(lc.ninv_shoup);
            if constexpr (GS)
                A::gs_scaled(v[m], v[m2], wj.x, wj.y, s, sq, q);
            else
                A::ct_scaled(v[m], v[m2], wj.x, wj.y, s, sq, q);
        } else {
            if constexpr (GS)
                A::gs(v[m], v[m2], wj.x, wj.y, q);
            else
                A::ct(v[m], v[m2], wj.x, wj.y, q);
        }
    }
}

// Chunk C is computed while chunks C+1 .. C+AHEAD are in flight.
template <class A, class S, int L, int PI, bool GS, int SCALE_STAGE, int AHEAD, int C>
struct Chunks {
    using Q = TwSeq<A, S, PI, GS>;
    using Tw = typename A::Tw;
    static constexpr int kTotal = Q::total();
    __device__ __forceinline__ static void run(typename A::W (&v)[1 << S::pass(PI).nreg], Tw (&ring)[AHEAD + 1][Q::kCh],
                                               const Tw *tw, uint32_t h, const LimbConst &lc) {
        if constexpr (C + AHEAD < kTotal) load_chunk<A, S, L, PI, GS, C + AHEAD>(ring[(C + AHEAD) % (AHEAD + 1)], tw, h);
        compute_chunk<A, S, PI, GS, SCALE_STAGE, C>(v, ring[C % (AHEAD + 1)], lc);
        if constexpr (C + 1 < kTotal) Chunks<A, S, L, PI, GS, SCALE_STAGE, AHEAD, C + 1>::run(v, ring, tw, h, lc);
    }
};

template <class A, class S, int L, int PI, bool GS, int AHEAD, int C>
__device__ __forceinline__ void prefetch_chunks(typename A::Tw (&ring)[AHEAD + 1][TwSeq<A, S, PI, GS>::kCh],
                                                const typename A::Tw *tw, uint32_t h) {
    if constexpr (C < AHEAD && C < TwSeq<A, S, PI, GS>::total()) {
        load_chunk<A, S, L, PI, GS, C>(ring[C], tw, h);
        prefetch_chunks<A, S, L, PI, GS, AHEAD, C + 1>(ring, tw, h);
    }
}

template <int L, int LOGE>
struct Shape {
    using S = Sched<L, LOGE>;
    static constexpr int kC = 1 << S::kLogC;
    static constexpr int kT = 1 << S::kLogT;
    static constexpr int kE = 1 << S::kLogE;
    static constexpr uint32_t kLocal = 1u << (L - S::kLogC);  // words per CTA
};

// Shared memory of one CTA: the working array (padded, one word per
// coefficient) and the staging buffer (the CTA's share of the next
// polynomial as raw u64 words).
template <class A, int L, int LOGE, int PF>
struct Smem {
    static constexpr uint32_t kLocal = Shape<L, LOGE>::kLocal;
    static constexpr uint32_t kWorkBytes = ((sizeof(typename A::W) * (kLocal + (kLocal >> 5) + (kLocal >> 10) + (kLocal >> 15)) + 127) / 128) * 128;
    static constexpr uint32_t kStageBytes = PF ? 8 * kLocal : 0;
    static constexpr uint32_t kBytes = kWorkBytes + kStageBytes;
};

// CTAs per SM the launch bounds are sized for: as many as shared memory
// (228 KB per SM, 1 KB reserved per CTA) and the 2048-thread limit allow.
template <class A, int L, int LOGE, int PF>
struct Occupancy {
    static constexpr int kT = Shape<L, LOGE>::kT;
    static constexpr int kBySmem = static_cast<int>((228u * 1024u) / (Smem<A, L, LOGE, PF>::kBytes + 1024u));
    // registers: 32 data registers per thread fit 1024 threads, 16 fit 1536
    static constexpr int kDataRegs = (1 << Sched<L, LOGE>::kLogE) * (A::kBits / 32);
    static constexpr int kByThreads = (kDataRegs >= 32 ? 1024 : 1536) / kT;
    static constexpr int kMin = kBySmem < kByThreads ? kBySmem : kByThreads;
    static constexpr int kMinBlocks = kMin < 1 ? 1 : kMin;
};

// Index in the CT pass order of the pass executed at step `i`.
template <class S, bool GS>
__host__ __device__ constexpr int pass_at(int i) {
    return GS ? (S::kPasses - 1 - i) : i;
}

// Position of local index l of a CTA in `phase` (rank bits inserted, with
// the value `rank`); linear in l over GF(2) once rank is fixed.
template <class S, int L>
__host__ __device__ constexpr uint32_t expand_local(uint32_t l, int phase) {
    uint32_t p = 0;
    int k = 0;
    for (int b = 0; b < L; ++b) {
        if (is_rank_bit<S>(b, phase)) continue;
        p |= ((l >> k) & 1u) << b;
        ++k;
    }
    return p;
}

template <class S>
__device__ __forceinline__ uint32_t rank_pos(uint32_t rank, int phase) {
    uint32_t p = 0;
#pragma unroll
    for (int j = 0; j < S::kLogC; ++j) p |= ((rank >> j) & 1u) << (phase ? S::rank1(j) : S::rank0(j));
    return p;
}

// ---------------------------------------------------------------- global I/O
// Every CTA moves its share of the polynomial between HBM and its shared
// memory with fully coalesced 16-byte accesses (two coefficients per
// thread and access), independently of the pass schedule.  Element i of a
// CTA (i = 2 * (tid + j * T) for j = 0, 1, ...) is an index into the CTA's
// share of the *natural* coefficient order: natural index = position p for
// Cooley-Tukey input / Gentleman-Sande output, and bitrev(p) for CT output /
// GS input.  All index maps are linear over GF(2), so each access is a
// per-thread base XOR a compile-time constant.

// Natural index of CTA-local element i when positions are stored natural
// (`nat` = true) or bit-reversed.  The CTA owns the positions whose rank
// bits (of `phase`) equal its rank; in bit-reversed order that fixes the
// mirrored natural bits.
template <class S, int L>
__host__ __device__ constexpr uint32_t natural_of(uint32_t i, int phase, bool nat) {
    if (nat) return expand_local<S, L>(i, phase);
    // rank bit b of a position is natural bit L-1-b
    uint32_t k = 0;
    int kk = 0;
    for (int b = 0; b < L; ++b) {
        bool rb = false;
        for (int j = 0; j < S::kLogC; ++j)
            if ((phase ? S::rank1(j) : S::rank0(j)) == L - 1 - b) rb = true;
        if (rb) continue;
        k |= ((i >> kk) & 1u) << b;
        ++kk;
    }
    return k;
}

// Shared-memory word of the coefficient with natural index k (rank bits of
// k already being this CTA's).
template <class S, int L>
__host__ __device__ constexpr uint32_t smem_of_natural(uint32_t k, int phase, bool nat) {
    return smem_addr<S, L>(nat ? k : brev_c(k, L), phase);
}

template <class A, class S, int L, int T, int LOCAL, int PHASE, bool NAT>
struct Coop {
    using W = typename A::W;
    static constexpr int kIters = LOCAL / (2 * T);

    // Loads and stores are calls for the 32-coefficient schedules up to
    // N = 2^14, inlined otherwise.  As calls they keep their address
    // arithmetic out of the passes' register budget (those kernels stop
    // spilling; measured on B200: forward +10% at 2^14, +6% at 2^13), but
    // from 2^15 up, and for 16-coefficient schedules, inlined measured faster.
    static constexpr bool kIoCall = S::kLogE >= 5 && L <= 14;

    __device__ __forceinline__ static void load(W *smem, const uint64_t *src, uint32_t rank,
                                                const LimbConst &lc, uint32_t &bad) {
        if constexpr (kIoCall) load_call(smem, src, rank, lc, bad);
        else load_body(smem, src, rank, lc, bad);
    }
    __device__ __noinline__ static void load_call(W *smem, const uint64_t *src, uint32_t rank,
                                                  const LimbConst &lc, uint32_t &bad) {
        load_body(smem, src, rank, lc, bad);
    }
    __device__ __forceinline__ static void store(const W *smem, uint64_t *dst, uint32_t rank,
                                                 const LimbConst &lc) {
        if constexpr (kIoCall) store_call(smem, dst, rank, lc);
        else store_body(smem, dst, rank, lc);
    }
    __device__ __noinline__ static void store_call(const W *smem, uint64_t *dst, uint32_t rank,
                                                   const LimbConst &lc) {
        store_body(smem, dst, rank, lc);
    }

    // Loads the CTA's share of `src` straight into the working array,
    // kBatch 16-byte loads in flight per thread at a time.
    __device__ __forceinline__ static void load_body(W *smem, const uint64_t *src, uint32_t rank,
                                                     const LimbConst &lc, uint32_t &bad) {
        constexpr int kBatch = A::kBits == 32 ? 8 : 4;
        const uint32_t tid = threadIdx.x;
        const uint32_t kr = NAT ? rank_pos<S>(rank, PHASE) : (__brev(rank_pos<S>(rank, PHASE)) >> (32 - L));
        const uint32_t kt = natural_of<S, L>(2 * tid, PHASE, NAT) + kr;
        const uint32_t at = smem_of_natural<S, L>(natural_of<S, L>(2 * tid, PHASE, NAT), PHASE, NAT);
        const W q = static_cast<W>(lc.q), one_q = static_cast<W>(lc.one_shoup);
        constexpr uint32_t a1 = smem_of_natural<S, L>(natural_of<S, L>(1, PHASE, NAT), PHASE, NAT);
#pragma unroll
        for (int j0 = 0; j0 < kIters; j0 += kBatch) {
            ulonglong2 x[kBatch];
#pragma unroll
            for (int j = 0; j < kBatch && j0 + j < kIters; ++j)
                x[j] = __ldcs(reinterpret_cast<const ulonglong2 *>(
                    src + kt + natural_of<S, L>(2 * (j0 + j) * T, PHASE, NAT)));
#pragma unroll
            for (int j = 0; j < kBatch && j0 + j < kIters; ++j) {
                const uint32_t a0 = at + smem_of_natural<S, L>(natural_of<S, L>(2 * (j0 + j) * T, PHASE, NAT),
                                                               PHASE, NAT);
                smem[a0] = A::load_reduce(x[j].x, q, one_q, bad);
                smem[a0 + a1] = A::load_reduce(x[j].y, q, one_q, bad);
            }
        }
    }

    // Issues this thread's 16-byte copies of the CTA's share of `src` into
    // the staging buffer (raw u64 words, element i at stage[i]).
    __device__ __forceinline__ static void prefetch(uint64_t *stage, const uint64_t *src, uint32_t rank) {
        const uint32_t tid = threadIdx.x;
        const uint32_t kr = NAT ? rank_pos<S>(rank, PHASE) : (__brev(rank_pos<S>(rank, PHASE)) >> (32 - L));
        const uint32_t kt = natural_of<S, L>(2 * tid, PHASE, NAT) + kr;
        const uint32_t sbase = static_cast<uint32_t>(__cvta_generic_to_shared(stage)) + 16u * tid;
#pragma unroll
        for (int j = 0; j < kIters; ++j)
            cp_async16(sbase + 16u * j * T, src + kt + natural_of<S, L>(2 * j * T, PHASE, NAT));
        cp_async_commit();
    }

    // Reduces this thread's staged words to residues and writes them to
    // their positions in the working array (after its own copies landed).
    __device__ __forceinline__ static void convert(const uint64_t *stage, W *smem, uint32_t rank,
                                                   const LimbConst &lc, uint32_t &bad) {
        const uint32_t tid = threadIdx.x;
        const uint32_t at = smem_of_natural<S, L>(natural_of<S, L>(2 * tid, PHASE, NAT), PHASE, NAT);
        const W q = static_cast<W>(lc.q), one_q = static_cast<W>(lc.one_shoup);
        constexpr uint32_t a1 = smem_of_natural<S, L>(natural_of<S, L>(1, PHASE, NAT), PHASE, NAT);
        const ulonglong2 *st2 = reinterpret_cast<const ulonglong2 *>(stage) + tid;
#pragma unroll
        for (int j = 0; j < kIters; ++j) {
            const ulonglong2 x = st2[j * T];
            const uint32_t a0 = at + smem_of_natural<S, L>(natural_of<S, L>(2 * j * T, PHASE, NAT), PHASE, NAT);
            smem[a0] = A::load_reduce(x.x, q, one_q, bad);
            smem[a0 + a1] = A::load_reduce(x.y, q, one_q, bad);
        }
    }

    // Combines the CTA's share of the working array, coefficient-wise mod q,
    // with `src` (in this stage's order): OP kFuseMul multiplies (the
    // pointwise product of a fused polynomial multiplication or
    // transform-and-multiply), kFuseAdd / kFuseSub add or subtract.  `src`
    // words are reduced first (any u64 for 64-bit words; words >= 2^32 set
    // `bad` for 32-bit words, as the input loads do); results stay in the
    // working array's lazy range.  Kept out of line: inlined next to a
    // transform under the 64-register budget, it made the kernels spill
    // 460-550 bytes per thread inside the passes (ptxas -v); as a call they
    // spill at most 12.
    template <uint32_t OP>
    __device__ __noinline__ static void combine(W *smem, const uint64_t *src, uint32_t rank,
                                                const LimbConst &lc, uint32_t &bad) {
        const uint32_t tid = threadIdx.x;
        const uint32_t kr = NAT ? rank_pos<S>(rank, PHASE) : (__brev(rank_pos<S>(rank, PHASE)) >> (32 - L));
        const uint32_t kt = natural_of<S, L>(2 * tid, PHASE, NAT) + kr;
        const uint32_t at = smem_of_natural<S, L>(natural_of<S, L>(2 * tid, PHASE, NAT), PHASE, NAT);
        constexpr uint32_t a1 = smem_of_natural<S, L>(natural_of<S, L>(1, PHASE, NAT), PHASE, NAT);
        constexpr int kBatch = A::kBits == 32 ? 8 : 4;
        const W q = static_cast<W>(lc.q), one_q = static_cast<W>(lc.one_shoup);
#pragma unroll
        for (int j0 = 0; j0 < kIters; j0 += kBatch) {
            ulonglong2 x[kBatch];
#pragma unroll
            for (int j = 0; j < kBatch && j0 + j < kIters; ++j)
                x[j] = __ldcs(reinterpret_cast<const ulonglong2 *>(
                    src + kt + natural_of<S, L>(2 * (j0 + j) * T, PHASE, NAT)));
#pragma unroll
            for (int j = 0; j < kBatch && j0 + j < kIters; ++j) {
                const uint32_t a0 = at + smem_of_natural<S, L>(natural_of<S, L>(2 * (j0 + j) * T, PHASE, NAT),
                                                               PHASE, NAT);
                smem[a0] = fuse<OP>(smem[a0], A::load_reduce(x[j].x, q, one_q, bad), lc);
                smem[a0 + a1] = fuse<OP>(smem[a0 + a1], A::load_reduce(x[j].y, q, one_q, bad), lc);
            }
        }
    }

    // u (working array, lazy range) op y (a lazily reduced input word).
    template <uint32_t OP>
    __device__ __forceinline__ static W fuse(W u, W y, const LimbConst &lc) {
        if constexpr (OP == kFuseMul) {
            return mulmod_lc(u, y, lc);
        } else {
            const W q = static_cast<W>(lc.q);
            const W uc = static_cast<W>(A::canon(u, q)), yc = A::sub_if(y, q);  // both in [0, q)
            return OP == kFuseAdd ? uc + yc : uc - yc + q;                        // [0, 2q)
        }
    }

    // combine<op> for a runtime op (selected once, outside the loop).
    __device__ __forceinline__ static void combine_op(W *smem, const uint64_t *src, uint32_t rank,
                                                      const LimbConst &lc, uint32_t &bad, uint32_t op) {
        if (op == kFuseAdd)
            combine<kFuseAdd>(smem, src, rank, lc, bad);
        else if (op == kFuseSub)
            combine<kFuseSub>(smem, src, rank, lc, bad);
        else
            combine<kFuseMul>(smem, src, rank, lc, bad);
    }

    __device__ __forceinline__ static W mulmod_lc(W x, W y, const LimbConst &lc) {
        if constexpr (A::kBits == 32)
            return A::mulmod(x, y, static_cast<W>(lc.q), lc.barrett);
        else
            return A::mulmod(x, y, lc.q, lc.barrett, lc.bk);
    }

    __device__ __forceinline__ static void store_body(const W *smem, uint64_t *dst, uint32_t rank,
                                                      const LimbConst &lc) {
        const uint32_t tid = threadIdx.x;
        const uint32_t kr = NAT ? rank_pos<S>(rank, PHASE) : (__brev(rank_pos<S>(rank, PHASE)) >> (32 - L));
        const uint32_t kt = natural_of<S, L>(2 * tid, PHASE, NAT) + kr;
        const uint32_t at = smem_of_natural<S, L>(natural_of<S, L>(2 * tid, PHASE, NAT), PHASE, NAT);
        const W q = static_cast<W>(lc.q);
        constexpr uint32_t a1 = smem_of_natural<S, L>(natural_of<S, L>(1, PHASE, NAT), PHASE, NAT);
#pragma unroll
        for (int j = 0; j < kIters; ++j) {
            const uint32_t a0 = at + smem_of_natural<S, L>(natural_of<S, L>(2 * j * T, PHASE, NAT), PHASE, NAT);
            ulonglong2 x;
            x.x = A::canon(smem[a0], q);
            x.y = A::canon(smem[a0 + a1], q);
            __stcs(reinterpret_cast<ulonglong2 *>(dst + kt + natural_of<S, L>(2 * j * T, PHASE, NAT)), x);
        }
    }
};

// One step (one pass) of the transform, shared memory to shared memory.
// Recursion over the step index keeps every loop bound constant.
template <class A, int L, int LOGE, bool GS, bool SCALE, int STEP>
struct Step {
    using S = Sched<L, LOGE>;
    using W = typename A::W;
    static constexpr int PI = pass_at<S, GS>(STEP);
    static constexpr PassDesc P = S::pass(PI);
    static constexpr int NSTEP = S::kPasses;
    static constexpr int E = 1 << S::kLogE;
    static constexpr int R = P.hi - P.lo + 1;

    // Does a phase change happen between this step and the next one?
    static constexpr bool kCross =
        S::kLogC > 0 && STEP + 1 < NSTEP && S::pass(pass_at<S, GS>(STEP + 1)).phase != P.phase;
    // How this step's results reach the next step: CT pass i hands over to
    // pass i+1 (kind stored on pass i); GS runs them backwards, so step
    // PI hands over to pass PI-1 (kind stored on pass PI-1).
    static constexpr int kSync = STEP + 1 >= NSTEP ? kSyncBlock
                                 : (GS ? S::pass(PI - 1).sync_after : P.sync_after);
    // Stage (within this pass) that carries N^-1: the very last stage.
    static constexpr int kScaleStage = (SCALE && STEP == NSTEP - 1) ? R - 1 : -1;
    // Twiddle chunks in flight ahead of the butterflies; the ring has the
    // same shape in every pass of a schedule.
    static constexpr int kAhead = E >= 32 ? 1 : 2;
    using Ring = typename A::Tw[kAhead + 1][TwSeq<A, S, PI, GS>::kCh];

    // Issues this pass's first twiddle chunks.  Called by the previous pass
    // (or the kernel) before the barrier that precedes this pass, so their
    // L2 latency overlaps the barrier wait.
    __device__ __forceinline__ static void prefetch(Ring &ring, const typename A::Tw *tw, uint32_t rank) {
        const uint32_t h = thread_pos<S, PI>(threadIdx.x, rank) >> (P.hi + 1);
        prefetch_chunks<A, S, L, PI, GS, kAhead, 0>(ring, tw, h);
    }

    __device__ __forceinline__ static void run(W *smem, const typename A::Tw *tw, const LimbConst &lc,
                                               uint32_t rank, Ring &ring) {
        using Next = Step<A, L, LOGE, GS, SCALE, (STEP + 1 < NSTEP ? STEP + 1 : STEP)>;
        const uint32_t tp = thread_pos<S, PI>(threadIdx.x, rank);
        const uint32_t h = tp >> (P.hi + 1);  // group-index bits above the pass
        W v[E];
        {
            const uint32_t at = smem_addr<S, L>(tp, P.phase);
#pragma unroll
            for (int m = 0; m < E; ++m) v[m] = smem[at + smem_addr<S, L>(reg_pos<S, PI>(m), P.phase)];
        }

        Chunks<A, S, L, PI, GS, kScaleStage, kAhead, 0>::run(v, ring, tw, h, lc);

        if constexpr (kCross) {
            // ---- phase change: every CTA must be done reading its shared
            // memory before the owners of the next phase write into it.
            constexpr int nphase = S::pass(pass_at<S, GS>(STEP + 1)).phase;
            // every value read above has been consumed by the butterflies
            // (pin() forces their results to exist before the arrive), so the
            // arrival needs no release ordering
#pragma unroll
            for (int m = 0; m < E; ++m) pin(v[m]);
            cluster_sync_relaxed();
            const uint32_t base = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
#pragma unroll
            for (int m = 0; m < E; ++m) {
                const uint32_t p = tp | reg_pos<S, PI>(m);
                uint32_t dest = 0;
#pragma unroll
                for (int j = 0; j < S::kLogC; ++j)
                    dest |= ((p >> (nphase ? S::rank1(j) : S::rank0(j))) & 1u) << j;
                const uint32_t off = smem_addr<S, L>(p, nphase);
                st_cluster<W>(map_rank(base + off * sizeof(W), dest), v[m]);
            }
            if constexpr (STEP + 1 < NSTEP) Next::prefetch(ring, tw, rank);
            cluster_sync_all();
        } else {
            // ---- back to shared memory, same layout.  The base goes through
            // pin() so the read addresses are not kept alive across the
            // butterflies.
            uint32_t at = smem_addr<S, L>(tp, P.phase);
            pin(at);
#pragma unroll
            for (int m = 0; m < E; ++m) smem[at + smem_addr<S, L>(reg_pos<S, PI>(m), P.phase)] = v[m];
            if constexpr (STEP + 1 < NSTEP) Next::prefetch(ring, tw, rank);
            // warp-local exchange: the next pass reads only what this warp wrote
            if constexpr (kSync == kSyncWarp)
                __syncwarp();
            else
                __syncthreads();
        }
        if constexpr (STEP + 1 < NSTEP) Next::run(smem, tw, lc, rank, ring);
    }
};

// Persistent kernel: cluster c (of G in the grid) transforms polynomials
// c, c + G, c + 2G, ... (limb-major, so consecutive ones mostly share a
// limb's twiddles).  While polynomial i is transformed, the copies of
// polynomial i + G are already in flight into the staging buffer.
// PF = 1 issues those copies as 16-byte cp.async per thread; PF = 2 (one-CTA
// schedules only) as one bulk copy (TMA) per polynomial from one thread,
// completed through an mbarrier.
// PF = 0: one polynomial per cluster, grid = all polynomials, the CTA
// loads its share straight into the working array (more CTAs per SM).
template <class A, int L, int LOGE, bool GS, bool SCALE, int PF>
__global__ void __launch_bounds__(Shape<L, LOGE>::kT, (Occupancy<A, L, LOGE, PF>::kMinBlocks)) k_ntt_fast(KArgs a) {
    using W = typename A::W;
    using Sh = Shape<L, LOGE>;
    using S = Sched<L, LOGE>;
    using Sm = Smem<A, L, LOGE, PF>;
    constexpr int ph_in = S::pass(pass_at<S, GS>(0)).phase;
    constexpr int ph_out = S::pass(pass_at<S, GS>(S::kPasses - 1)).phase;
    // CT reads natural order, GS reads bit-reversed positions
    using In = Coop<A, S, L, Sh::kT, Sh::kLocal, ph_in, !GS>;
    using Out = Coop<A, S, L, Sh::kT, Sh::kLocal, ph_out, GS>;
    using First = Step<A, L, LOGE, GS, SCALE, 0>;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    W *work = reinterpret_cast<W *>(smem_raw);
    uint64_t *stage = reinterpret_cast<uint64_t *>(smem_raw + Sm::kWorkBytes);
    const uint32_t rank = Sh::kC > 1 ? cluster_rank() : 0u;
    const uint64_t G = gridDim.x / Sh::kC;
    const uint64_t npolys = static_cast<uint64_t>(a.batch) * a.n_limbs;
    auto base_of = [&](uint64_t cl) {
        const uint64_t limb = cl / a.batch, poly = cl % a.batch;
        return static_cast<int64_t>(limb) * a.limb_stride + static_cast<int64_t>(poly) * a.poly_stride;
    };
    uint32_t bad = 0;
    uint64_t cl = blockIdx.x / Sh::kC;
    if constexpr (!PF) {
        const uint32_t limb = static_cast<uint32_t>(cl / a.batch);
        const LimbConst &lc = a.limbs[limb];
        const typename A::Tw *tw = reinterpret_cast<const typename A::Tw *>(a.tw) + (static_cast<size_t>(limb) << L);
        In::load(work, a.in + base_of(cl), rank, lc, bad);
        if constexpr (A::kBits == 32) {
            if (__any_sync(0xffffffffu, bad != 0) && (threadIdx.x & 31) == 0) store_status(a.status, kStatusInputRange);
        }
        typename First::Ring ring;
        First::prefetch(ring, tw, rank);
        __syncthreads();
        First::run(work, tw, lc, rank, ring);
        Out::store(work, a.out + base_of(cl), rank, lc);
        return;
    }
    if constexpr (PF == 2) {
        static_assert(Sh::kC == 1, "bulk-copy staging needs the whole polynomial in one CTA");
        // One CTA holds the whole polynomial, so its share is the contiguous
        // range [0, N) and staging element i is natural index i (Coop::convert
        // reads it in that order).
        __shared__ __align__(8) uint64_t bar;
        constexpr uint32_t kBytes = 8u * Sh::kLocal;
        if (threadIdx.x == 0) mbar_init(&bar, 1);
        __syncthreads();
        uint32_t parity = 0;
        if (cl < npolys && threadIdx.x == 0) bulk_load(stage, a.in + base_of(cl), kBytes, &bar);
        for (; cl < npolys; cl += G) {
            const uint32_t limb = static_cast<uint32_t>(cl / a.batch);
            const LimbConst &lc = a.limbs[limb];
            const typename A::Tw *tw = reinterpret_cast<const typename A::Tw *>(a.tw) + (static_cast<size_t>(limb) << L);
            const bool ok = mbar_wait_bounded(&bar, parity);
            if (__syncthreads_or(!ok)) {  // a copy that never lands: report, drain once more, leave
                if (threadIdx.x == 0) store_status(a.status, kStatusWaitTimeout);
                mbar_wait_bounded(&bar, parity);
                return;
            }
            parity ^= 1u;
            In::convert(stage, work, rank, lc, bad);
            __syncthreads();  // staging consumed by every thread
            if (cl + G < npolys && threadIdx.x == 0) {
                fence_proxy_async_smem();
                bulk_load(stage, a.in + base_of(cl + G), kBytes, &bar);
            }
            typename First::Ring ring;
            First::prefetch(ring, tw, rank);
            First::run(work, tw, lc, rank, ring);
            Out::store(work, a.out + base_of(cl), rank, lc);
            __syncthreads();
        }
        if constexpr (A::kBits == 32) {
            if (__any_sync(0xffffffffu, bad != 0) && (threadIdx.x & 31) == 0) store_status(a.status, kStatusInputRange);
        }
        return;
    }
    if (cl < npolys) In::prefetch(stage, a.in + base_of(cl), rank);
    for (; cl < npolys; cl += G) {
        const uint32_t limb = static_cast<uint32_t>(cl / a.batch);
        const LimbConst &lc = a.limbs[limb];
        const typename A::Tw *tw = reinterpret_cast<const typename A::Tw *>(a.tw) + (static_cast<size_t>(limb) << L);
        cp_async_wait_all();
        In::convert(stage, work, rank, lc, bad);
        if (cl + G < npolys) In::prefetch(stage, a.in + base_of(cl + G), rank);
        typename First::Ring ring;
        First::prefetch(ring, tw, rank);
        __syncthreads();
        First::run(work, tw, lc, rank, ring);
        Out::store(work, a.out + base_of(cl), rank, lc);
        __syncthreads();
    }
    if constexpr (A::kBits == 32) {
        if (__any_sync(0xffffffffu, bad != 0) && (threadIdx.x & 31) == 0) store_status(a.status, kStatusInputRange);
    }
}

// Launch attributes of a cluster launch of kC CTAs: the cluster shape and
// the scheduling policy (none for kC = 1).
inline int cluster_attrs(cudaLaunchAttribute (&attr)[2], int kC) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(kC);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeClusterSchedulingPolicyPreference;
    attr[1].val.clusterSchedulingPolicyPreference = static_cast<cudaClusterSchedulingPolicy>(cluster_policy());
    return kC > 1 ? 2 : 0;
}

template <class A, int L, int LOGE, bool GS, bool SCALE, int PF>
int launch_one(const KArgs &a, cudaStream_t s) {
    using Sh = Shape<L, LOGE>;
    auto kern = k_ntt_fast<A, L, LOGE, GS, SCALE, PF>;
    const size_t smem = Smem<A, L, LOGE, PF>::kBytes;
    // Per device: the shared-memory attribute, and how many clusters fit
    // at once (the persistent grid size).
    static std::atomic<int> resident[64];  // zero-initialized; first calls may race harmlessly
    int dev = 0;
    cudaGetDevice(&dev);
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(Sh::kT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    cfg.attrs = attr;
    cfg.numAttrs = cluster_attrs(attr, Sh::kC);
    int nres = dev < 64 ? resident[dev].load() : 0;
    if (nres == 0) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return cuda_fail(e, "k_ntt_fast shared-memory attribute");
        if (Sh::kC > 8) {  // clusters of 16 CTAs: a non-portable size B200 supports
            e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
            if (e != cudaSuccess) return cuda_fail(e, "k_ntt_fast cluster-size attribute");
        }
        int props = 0;
        cudaDeviceGetAttribute(&props, cudaDevAttrMultiProcessorCount, dev);
        if (Sh::kC > 1) {
            cfg.gridDim = dim3(Sh::kC * 1024);
            e = cudaOccupancyMaxActiveClusters(&nres, kern, &cfg);
            if (e != cudaSuccess) return cuda_fail(e, "k_ntt_fast cluster occupancy");
        } else {
            int per_sm = 0;
            e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, Sh::kT, smem);
            if (e != cudaSuccess) return cuda_fail(e, "k_ntt_fast occupancy");
            nres = per_sm * props;
        }
        if (nres <= 0)
            return fail(BC_ERR_UNSUPPORTED, format("k_ntt_fast<%d>: no cluster of %d CTAs fits an SM set", L, Sh::kC));
        if (dev < 64) resident[dev].store(nres);
    }
    const uint64_t polys = static_cast<uint64_t>(a.batch) * a.n_limbs;
    const uint64_t clusters = (!PF || polys < static_cast<uint64_t>(nres)) ? polys : static_cast<uint64_t>(nres);
    cfg.gridDim = dim3(static_cast<unsigned>(clusters * Sh::kC));
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
    if (e != cudaSuccess) return cuda_fail(e, "k_ntt_fast launch");
    return BC_OK;
}

// Fused negacyclic polynomial product, one cluster per (limb, pair):
// C = INTT(NTT(A) * B^), where B^ = NTT(B) in natural order (a forward launch
// writes it, possibly into C itself).  The forward passes, the pointwise
// product and the inverse passes all run on the working array, so HBM sees
// A and B^ read once and C written once (24N bytes per pair).  B^ may alias
// C: every CTA reads its share of B^ before the cluster barrier of the
// inverse's phase change, and writes C only after it.
template <class A, int L, int LOGE>
__global__ void __launch_bounds__(Shape<L, LOGE>::kT, (Occupancy<A, L, LOGE, 0>::kMinBlocks))
    k_polymul_fast(KArgs a) {
    using W = typename A::W;
    using Sh = Shape<L, LOGE>;
    using S = Sched<L, LOGE>;
    using Fwd = Step<A, L, LOGE, false, false, 0>;
    using Inv = Step<A, L, LOGE, true, true, 0>;
    constexpr int ph_first = S::pass(0).phase, ph_last = S::pass(S::kPasses - 1).phase;
    using In = Coop<A, S, L, Sh::kT, Sh::kLocal, ph_first, true>;   // A, natural order
    using Mid = Coop<A, S, L, Sh::kT, Sh::kLocal, ph_last, false>;  // B^, NTT-domain order
    using Out = Coop<A, S, L, Sh::kT, Sh::kLocal, ph_first, true>;  // C, natural order
    extern __shared__ __align__(128) unsigned char smem_raw[];
    W *work = reinterpret_cast<W *>(smem_raw);
    const uint32_t rank = Sh::kC > 1 ? cluster_rank() : 0u;
    const uint64_t cl = blockIdx.x / Sh::kC;
    const uint64_t limb = cl / a.batch, poly = cl % a.batch;
    const int64_t base = static_cast<int64_t>(limb) * a.limb_stride + static_cast<int64_t>(poly) * a.poly_stride;
    const LimbConst &lc = a.limbs[limb];
    const typename A::Tw *tw = reinterpret_cast<const typename A::Tw *>(a.tw) + (limb << L);
    const typename A::Tw *tw2 = reinterpret_cast<const typename A::Tw *>(a.tw2) + (limb << L);
    uint32_t bad = 0;
    In::load(work, a.in + base, rank, lc, bad);
    typename Fwd::Ring ring_f;
    Fwd::prefetch(ring_f, tw, rank);
    __syncthreads();
    Fwd::run(work, tw, lc, rank, ring_f);  // ends with the working array complete
    Mid::template combine<kFuseMul>(work, a.in2 + base, rank, lc, bad);
    typename Inv::Ring ring_i;
    Inv::prefetch(ring_i, tw2, rank);
    __syncthreads();
    Inv::run(work, tw2, lc, rank, ring_i);
    Out::store(work, a.out + base, rank, lc);
    if constexpr (A::kBits == 32) {
        if (__any_sync(0xffffffffu, bad != 0) && (threadIdx.x & 31) == 0) store_status(a.status, kStatusInputRange);
    }
}

// Transform and pointwise step fused in one kernel, one cluster per
// (limb, polynomial), negacyclic plans; the step (a.op) is the product, the
// sum or the difference mod q:
//   INV = false: C = NTT(A) op B^, the step in the forward's epilogue;
//   INV = true:  C = INTT(A^ op B^), the step in the inverse's prologue.
// A^, B^ and the forward's C are in natural order.  B^ is read in the
// working array's order at the one point where the values sit in that order
// (after the forward passes, before the inverse passes), as in the fused
// polynomial product.  HBM sees 24N bytes per polynomial instead of the 32N
// of a transform launch followed by a pointwise launch.  C may alias A or
// B^: each CTA reads B^ (forward) exactly where it then writes C, and reads
// A^ and B^ (inverse) before the phase-change barrier that precedes every
// store.
template <class A, int L, int LOGE, bool INV>
__global__ void __launch_bounds__(Shape<L, LOGE>::kT, (Occupancy<A, L, LOGE, 0>::kMinBlocks))
    k_ntt_mul_fast(KArgs a) {
    using W = typename A::W;
    using Sh = Shape<L, LOGE>;
    using S = Sched<L, LOGE>;
    using Tr = Step<A, L, LOGE, INV, INV, 0>;  // negacyclic: CT forward, GS inverse with N^-1 folded
    constexpr int ph_in = S::pass(pass_at<S, INV>(0)).phase;
    constexpr int ph_out = S::pass(pass_at<S, INV>(S::kPasses - 1)).phase;
    using In = Coop<A, S, L, Sh::kT, Sh::kLocal, ph_in, !INV>;
    using Out = Coop<A, S, L, Sh::kT, Sh::kLocal, ph_out, INV>;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    W *work = reinterpret_cast<W *>(smem_raw);
    const uint32_t rank = Sh::kC > 1 ? cluster_rank() : 0u;
    const uint64_t cl = blockIdx.x / Sh::kC;
    const uint64_t limb = cl / a.batch, poly = cl % a.batch;
    const int64_t base = static_cast<int64_t>(limb) * a.limb_stride + static_cast<int64_t>(poly) * a.poly_stride;
    const LimbConst &lc = a.limbs[limb];
    const typename A::Tw *tw = reinterpret_cast<const typename A::Tw *>(a.tw) + (limb << L);
    uint32_t bad = 0;
    In::load(work, a.in + base, rank, lc, bad);
    // the thread multiplies the words it has just written: no barrier needed
    if constexpr (INV) In::combine_op(work, a.in2 + base, rank, lc, bad, a.op);
    typename Tr::Ring ring;
    Tr::prefetch(ring, tw, rank);
    __syncthreads();
    Tr::run(work, tw, lc, rank, ring);  // ends with the working array complete
    if constexpr (!INV) Out::combine_op(work, a.in2 + base, rank, lc, bad, a.op);
    Out::store(work, a.out + base, rank, lc);
    if constexpr (A::kBits == 32) {
        if (__any_sync(0xffffffffu, bad != 0) && (threadIdx.x & 31) == 0) store_status(a.status, kStatusInputRange);
    }
}

// One cluster of Shape<L, LOGE>::kC CTAs per (limb, polynomial).
template <class A, int L, int LOGE>
int launch_per_poly(void (*kern)(KArgs), std::atomic<bool> *attr_set, const char *name, const KArgs &a,
                    cudaStream_t s) {
    using Sh = Shape<L, LOGE>;
    const size_t smem = Smem<A, L, LOGE, 0>::kBytes;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 64 || !attr_set[dev].load()) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return cuda_fail(e, format("%s shared-memory attribute", name).c_str());
        if (Sh::kC > 8) {
            e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
            if (e != cudaSuccess) return cuda_fail(e, format("%s cluster-size attribute", name).c_str());
        }
        if (dev < 64) attr_set[dev].store(true);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(Sh::kT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    cfg.attrs = attr;
    cfg.numAttrs = cluster_attrs(attr, Sh::kC);
    const uint64_t polys = static_cast<uint64_t>(a.batch) * a.n_limbs;
    cfg.gridDim = dim3(static_cast<unsigned>(polys * Sh::kC));
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
    if (e != cudaSuccess) return cuda_fail(e, format("%s launch", name).c_str());
    return BC_OK;
}

template <class A, int L, int LOGE, bool INV>
int launch_ntt_mul_one(const KArgs &a, cudaStream_t s) {
    static std::atomic<bool> attr_set[64];
    return launch_per_poly<A, L, LOGE>(k_ntt_mul_fast<A, L, LOGE, INV>, attr_set, "k_ntt_mul_fast", a, s);
}

template <class A, int L, int LOGE>
int launch_polymul_one(const KArgs &a, cudaStream_t s) {
    using Sh = Shape<L, LOGE>;
    auto kern = k_polymul_fast<A, L, LOGE>;
    const size_t smem = Smem<A, L, LOGE, 0>::kBytes;
    static std::atomic<bool> attr_set[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 64 || !attr_set[dev].load()) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return cuda_fail(e, "k_polymul_fast shared-memory attribute");
        if (Sh::kC > 8) {
            e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
            if (e != cudaSuccess) return cuda_fail(e, "k_polymul_fast cluster-size attribute");
        }
        if (dev < 64) attr_set[dev].store(true);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(Sh::kT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    cfg.attrs = attr;
    cfg.numAttrs = cluster_attrs(attr, Sh::kC);
    const uint64_t polys = static_cast<uint64_t>(a.batch) * a.n_limbs;
    cfg.gridDim = dim3(static_cast<unsigned>(polys * Sh::kC));
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
    if (e != cudaSuccess) return cuda_fail(e, "k_polymul_fast launch");
    return BC_OK;
}

// Persistent prefetching launches are not used by default: with their
// staging buffers fewer CTAs fit an SM, and measured on B200 that loses
// more to barrier and shared-memory-queue stalls than the prefetch gains.
// BARRACUDA_NTT_PERSISTENT=1 selects them with per-thread cp.async copies,
// =2 with one bulk copy (TMA) per polynomial where one CTA holds the whole
// polynomial (N <= 2^13), cp.async otherwise.
inline int persistent_mode() {
    static const int mode = [] {
        const char *e = std::getenv("BARRACUDA_NTT_PERSISTENT");
        return e && (e[0] == '1' || e[0] == '2') ? e[0] - '0' : 0;
    }();
    return mode;
}

template <class A, int L, int LOGE, int PF>
int launch_dir(bool gs, bool scale, const KArgs &a, cudaStream_t s) {
    if (gs) return scale ? launch_one<A, L, LOGE, true, true, PF>(a, s) : launch_one<A, L, LOGE, true, false, PF>(a, s);
    return scale ? launch_one<A, L, LOGE, false, true, PF>(a, s) : launch_one<A, L, LOGE, false, false, PF>(a, s);
}

template <class A, int LOGE, int L>
int dispatch_dir(bool gs, bool scale, const KArgs &a, cudaStream_t s) {
    const int mode = persistent_mode();
    if constexpr (Shape<L, LOGE>::kC == 1) {
        if (mode == 2) return launch_dir<A, L, LOGE, 2>(gs, scale, a, s);
    }
    if (mode != 0) return launch_dir<A, L, LOGE, 1>(gs, scale, a, s);
    return launch_dir<A, L, LOGE, 0>(gs, scale, a, s);
}

template <class A, int V, int L>
int dispatch_if(bool gs, bool scale, const KArgs &a, cudaStream_t s) {
    if constexpr (sched_logc(L, V) >= 0) return dispatch_dir<A, V, L>(gs, scale, a, s);
    return fail(BC_ERR_INTERNAL, format("no fast schedule for log2 N = %d, variant %d", L, V));
}

template <class A, int V, int L>
int polymul_if(const KArgs &a, cudaStream_t s) {
    if constexpr (sched_logc(L, V) >= 0) return launch_polymul_one<A, L, V>(a, s);
    return fail(BC_ERR_INTERNAL, format("no fast schedule for log2 N = %d, variant %d", L, V));
}

template <class A, int V, int L>
int ntt_mul_if(bool inverse, const KArgs &a, cudaStream_t s) {
    if constexpr (sched_logc(L, V) >= 0)
        return inverse ? launch_ntt_mul_one<A, L, V, true>(a, s) : launch_ntt_mul_one<A, L, V, false>(a, s);
    return fail(BC_ERR_INTERNAL, format("no fast schedule for log2 N = %d, variant %d", L, V));
}

// Transform fused with a pointwise product (see k_ntt_mul_fast).
template <class A, int V>
int dispatch_ntt_mul_l(uint32_t L, bool inverse, const KArgs &a, cudaStream_t s) {
    switch (L) {
    case 10: return ntt_mul_if<A, V, 10>(inverse, a, s);
    case 11: return ntt_mul_if<A, V, 11>(inverse, a, s);
    case 12: return ntt_mul_if<A, V, 12>(inverse, a, s);
    case 13: return ntt_mul_if<A, V, 13>(inverse, a, s);
    case 14: return ntt_mul_if<A, V, 14>(inverse, a, s);
    case 15: return ntt_mul_if<A, V, 15>(inverse, a, s);
    case 16: return ntt_mul_if<A, V, 16>(inverse, a, s);
    case 17: return ntt_mul_if<A, V, 17>(inverse, a, s);
    default: break;
    }
    return fail(BC_ERR_INTERNAL, format("no fast schedule for log2 N = %u", L));
}

// Fused polymul for the fast sizes (see k_polymul_fast).
template <class A, int V>
int dispatch_polymul_l(uint32_t L, const KArgs &a, cudaStream_t s) {
    switch (L) {
    case 10: return polymul_if<A, V, 10>(a, s);
    case 11: return polymul_if<A, V, 11>(a, s);
    case 12: return polymul_if<A, V, 12>(a, s);
    case 13: return polymul_if<A, V, 13>(a, s);
    case 14: return polymul_if<A, V, 14>(a, s);
    case 15: return polymul_if<A, V, 15>(a, s);
    case 16: return polymul_if<A, V, 16>(a, s);
    case 17: return polymul_if<A, V, 17>(a, s);
    default: break;
    }
    return fail(BC_ERR_INTERNAL, format("no fast schedule for log2 N = %u", L));
}

// Template parameter LOGE of the kernels above is the schedule variant V
// (Sched<L, V>): 4, 5, 6 or 7, see gen_schedule.py.
template <class A, int V>
int dispatch_l(uint32_t L, bool gs, bool scale, const KArgs &a, cudaStream_t s) {
    switch (L) {
    case 10: return dispatch_if<A, V, 10>(gs, scale, a, s);
    case 11: return dispatch_if<A, V, 11>(gs, scale, a, s);
    case 12: return dispatch_if<A, V, 12>(gs, scale, a, s);
    case 13: return dispatch_if<A, V, 13>(gs, scale, a, s);
    case 14: return dispatch_if<A, V, 14>(gs, scale, a, s);
    case 15: return dispatch_if<A, V, 15>(gs, scale, a, s);
    case 16: return dispatch_if<A, V, 16>(gs, scale, a, s);
    case 17: return dispatch_if<A, V, 17>(gs, scale, a, s);
    default: break;
    }
    return fail(BC_ERR_INTERNAL, format("no fast schedule for log2 N = %u", L));
}

}  // namespace fast
}  // namespace bc
