// bc_kernels_multipass.cuh -- the transform for N = 2^18 .. 2^24: two or
// three passes through HBM instead of one launch per stage.
//
// Positions p in [0, N), N = 2^L, are split into bit fields.  A pass owns S
// consecutive bits [lo, lo + S) and runs every butterfly stage of those bits
// on independent sub-transforms: the positions that agree in every other
// bit.  One CTA holds a tile of 32 such sub-transforms (32 "columns" x 2^S
// "rows") in shared memory; warps take the columns as lanes, so every
// shared-memory access of a warp touches 32 distinct banks, and each pass's
// butterflies run in register rounds of 2 to 4 bits (radix 4..16) between
// barriers.
//
//   TOP pass  (bits [L - S, L)):  columns = position bits [0, 5)
//   MID / LOW (bits [lo, lo + S), lo + S <= L - 5): columns = bits [L - 5, L)
//
// Between passes the coefficients live in a scratch buffer in "sigma order":
// sigma(p) = ((p mod 2^(L-5)) << 5) | (p >> (L-5)), the top five position
// bits innermost.  A MID/LOW tile then reads and writes 32 consecutive words
// per row.  The TOP tile transposes through shared memory (an XOR swizzle of
// the column by the row's top five bits keeps both directions conflict-free)
// so that its natural-order side and its sigma side are both coalesced.  The
// LOW pass meets the bit-reversed side (Cooley-Tukey output, Gentleman-Sande
// input): with columns = the top five position bits, bitrev(p) keeps them as
// the five lowest index bits, so a warp again covers 32 consecutive words.
//
// Twiddles: stage b reads table entry (N >> (b+1)) + (p >> (b+1)), the
// convention of every transform here.  Stages of the TOP pass share a
// twiddle across all columns (broadcast loads, natural table layout).  Below
// the TOP pass each column needs its own entry, so those stages' blocks are
// stored permuted by the same sigma (multipass_table_index), and a warp reads
// 32 consecutive entries.
#pragma once

#include <cstdint>

#include "bc_kernels.hpp"

namespace bc {
namespace mp {

enum Role : int { kTop = 0, kMid = 1, kLow = 2 };

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

// Register rounds of a pass of S bits for words of WB bytes, from the lowest
// bits up, each leaving at least 8 tasks (one per warp).  32-bit words: two
// rounds of floor(S/2) and ceil(S/2) bits (radix 8 or 16 in registers) for
// S <= 8, three rounds of 3 bits for S = 9.  64-bit words, twice the
// registers per coefficient: rounds of at most 3 bits.
__host__ __device__ constexpr int round_count(int S, int WB) { return (S == 9 || (WB == 8 && S > 6)) ? 3 : 2; }
__host__ __device__ constexpr int round_width(int S, int WB, int r) {
    return round_count(S, WB) == 2 ? (r == 0 ? S / 2 : S - S / 2) : (S == 9 ? 3 : (r == 0 ? 2 : (S == 7 && r == 1 ? 2 : 3)));
}
__host__ __device__ constexpr int round_lo(int S, int WB, int r) {
    int lo = 0;
    for (int i = 0; i < r; ++i) lo += round_width(S, WB, i);
    return lo;
}

// CTAs per SM a pass is compiled for (register budget 65536 / (256 x this)):
// as many as its tile allows in shared memory (228 KB per SM) where the
// largest round still fits its registers, fewer otherwise.  ptxas -v shows
// no spills except 8-24 bytes in the 32-bit S = 8 TOP pass.
template <class A, int S>
__host__ __device__ constexpr int min_blocks() {
    if constexpr (sizeof(typename A::W) == 4)
        return S == 6 ? 6 : S == 7 ? 5 : S == 8 ? 4 : 3;  // 40 / 48 / 64 / 80 registers
    else
        return S == 8 ? 3 : 4;  // 64 / 64 / 80 registers
}

// Shared-memory word of tile element (row, col); TOP tiles swizzle the
// column by the row's top five bits.
template <int S, int ROLE>
__device__ __forceinline__ uint32_t tile_addr(uint32_t row, uint32_t col) {
    if constexpr (ROLE == kTop)
        return row * 32u + (col ^ (row >> (S - 5)));
    else
        return row * 32u + col;
}

struct Ctx {
    uint32_t L, lo;
    uint32_t t;           // tile index within the polynomial
    uint32_t lane, warp;
    uint32_t pfix;        // MID / LOW: the tile's fixed position bits (t placed around the pass)
    uint32_t blk0;        // MID / LOW: N >> (lo + 1), table block of the pass's lowest stage
    uint32_t pf0;         // MID / LOW: pfix >> (lo + 1)
};

template <class A, bool GS, bool SCALED>
__device__ __forceinline__ void bfly(typename A::W &x, typename A::W &y, const typename A::Tw &w,
                                     const LimbConst &lc) {
    using W = typename A::W;
    const W q = static_cast<W>(lc.q);
    if constexpr (SCALED) {
        const W s = static_cast<W>(lc.ninv), sq = static_cast<W>(lc.ninv_shoup);
        if constexpr (GS)
            A::gs_scaled(x, y, w.x, w.y, s, sq, q);
        else
            A::ct_scaled(x, y, w.x, w.y, s, sq, q);
    } else {
        if constexpr (GS)
            A::gs(x, y, w.x, w.y, q);
        else
            A::ct(x, y, w.x, w.y, q);
    }
}

// Stage J of a round: the butterflies of register pairs (m, m | 2^J).
// Whether N^-1 rides on it is known at compile time: the transform's last
// stage is GS b = L - 1 (the TOP pass's highest row bit) or CT b = 0 (the
// LOW pass's lowest).  Table entry of register 0 for stage b = lo + RR + J:
//   TOP:       (N >> (b+1)) + (row >> (RR+J+1)), natural layout;
//   MID / LOW: (N >> (b+1)) + (((p >> (b+1)) mod 2^(L-b-6)) << 5) + lane, the
//              sigma layout, where p >> (b+1) without the column is
//              (pfix >> (b+1)) | (row >> (RR+J+1)).
// Register m reads (m >> (J+1)) entries (TOP) or rows of 32 entries further.
template <class A, bool GS, bool SCALE, int S, int ROLE, int RR, int K, int J>
__device__ __forceinline__ void round_stage(typename A::W (&v)[1 << K], const typename A::Tw *tw, uint32_t base,
                                            const Ctx &c, const LimbConst &lc) {
    constexpr bool kScaled =
        SCALE && (GS ? (ROLE == kTop && RR + J == S - 1) : (ROLE == kLow && RR + J == 0));
    constexpr int kStride = ROLE == kTop ? 1 : 32;
    const typename A::Tw *tb;
    if constexpr (ROLE == kTop)
        tb = tw + ((1u << (S - RR - J - 1)) + (base >> (RR + J + 1)));
    else
        tb = tw + c.lane + (c.blk0 >> (RR + J)) + (((c.pf0 >> (RR + J)) | (base >> (RR + J + 1))) << 5);
#pragma unroll
    for (int m = 0; m < (1 << K); ++m) {
        if (m & (1 << J)) continue;
        const typename A::Tw w = __ldg(tb + (m >> (J + 1)) * kStride);
        bfly<A, GS, kScaled>(v[m], v[m | (1 << J)], w, lc);
    }
}

template <class A, bool GS, bool SCALE, int S, int ROLE, int RR, int K, int JJ>
__device__ __forceinline__ void round_stages(typename A::W (&v)[1 << K], const typename A::Tw *tw, uint32_t base,
                                             const Ctx &c, const LimbConst &lc) {
    // CT runs a round's stages from its top bit down, GS from its bottom up
    round_stage<A, GS, SCALE, S, ROLE, RR, K, GS ? JJ : K - 1 - JJ>(v, tw, base, c, lc);
    if constexpr (JJ + 1 < K) round_stages<A, GS, SCALE, S, ROLE, RR, K, JJ + 1>(v, tw, base, c, lc);
}

// One register round: bits [RR, RR + K) of the row (absolute position bits
// lo + RR ..).  Each thread runs the round's K stages on 2^K coefficients of
// its column (= lane) per task; a task fixes the row's other bits.  Shared-
// memory addresses are a per-task base plus compile-time offsets.
template <class A, bool GS, bool SCALE, int S, int ROLE, int RR, int K>
__device__ __forceinline__ void pass_round(typename A::W *tile, const typename A::Tw *tw, const LimbConst &lc,
                                           const Ctx &c) {
    using W = typename A::W;
    constexpr int kTasks = 1 << (S - K);
    constexpr int kPer = kTasks / kWarps;
    static_assert(kPer >= 1, "a round must give every warp a task");
    constexpr int TB = S - 5;  // TOP: the row's top five bits swizzle the column
#pragma unroll 1
    for (int it = 0; it < kPer; ++it) {
        const uint32_t g = c.warp + kWarps * it;
        const uint32_t base = ((g >> RR) << (RR + K)) | (g & ((1u << RR) - 1u));  // round bits zero
        // word of (base, lane); register m adds row m << RR
        const uint32_t lx = ROLE == kTop ? (c.lane ^ (base >> TB)) : c.lane;
        W *const t0 = tile + base * 32u;
        W v[1 << K];
#pragma unroll
        for (int m = 0; m < (1 << K); ++m) {
            const uint32_t mr = static_cast<uint32_t>(m) << RR;
            v[m] = t0[mr * 32u + (ROLE == kTop ? (lx ^ (mr >> TB)) : lx)];
        }
        round_stages<A, GS, SCALE, S, ROLE, RR, K, 0>(v, tw, base, c, lc);
#pragma unroll
        for (int m = 0; m < (1 << K); ++m) {
            const uint32_t mr = static_cast<uint32_t>(m) << RR;
            t0[mr * 32u + (ROLE == kTop ? (lx ^ (mr >> TB)) : lx)] = v[m];
        }
    }
}

template <class A, bool GS, bool SCALE, int S, int ROLE, int R>
__device__ __forceinline__ void rounds_from(typename A::W *tile, const typename A::Tw *tw, const LimbConst &lc,
                                            const Ctx &c) {
    // CT runs the rounds from the top bits down, GS from the bottom up.
    constexpr int WB = static_cast<int>(sizeof(typename A::W));
    constexpr int NR = round_count(S, WB);
    constexpr int r = GS ? R : NR - 1 - R;
    pass_round<A, GS, SCALE, S, ROLE, round_lo(S, WB, r), round_width(S, WB, r)>(tile, tw, lc, c);
    if constexpr (R + 1 < NR) {
        __syncthreads();
        rounds_from<A, GS, SCALE, S, ROLE, R + 1>(tile, tw, lc, c);
    }
}

__device__ __forceinline__ void flag_bad(uint32_t *status, uint32_t bad) {
    if (__any_sync(0xffffffffu, bad != 0) && (threadIdx.x & 31) == 0) store_status(status, kStatusInputRange);
}

// One pass over a tile of 32 sub-transforms.  Which side is the caller's
// buffer depends on the direction: Cooley-Tukey runs TOP (reads natural
// input) .. MID .. LOW (writes bit-reversed output); Gentleman-Sande runs
// LOW (reads bit-reversed input) .. MID .. TOP (writes natural output).
// Every other side is the sigma-order scratch (lazy residues of the plan's
// word width).
template <class A, bool GS, bool SCALE, int S, int ROLE>
__global__ void __launch_bounds__(kThreads, (min_blocks<A, S>())) k_ntt_pass(KArgs a, typename A::W *scratch, uint32_t lo) {
    using W = typename A::W;
    using Tw = typename A::Tw;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    W *tile = reinterpret_cast<W *>(smem_raw);
    const uint32_t L = a.logn;
    const uint32_t tile_bits = ROLE == kTop ? lo - 5 : L - 5 - S;
    const uint64_t pl = blockIdx.x >> tile_bits;  // polynomial index, limb-major
    Ctx c;
    c.L = L;
    c.lo = lo;
    c.t = blockIdx.x & ((1u << tile_bits) - 1u);
    c.lane = threadIdx.x & 31u;
    c.warp = threadIdx.x >> 5;
    c.pfix = ROLE == kTop ? 0u : (((c.t >> lo) << (lo + S)) | (c.t & ((1u << lo) - 1u)));
    c.blk0 = 1u << (L - lo - 1);
    c.pf0 = c.pfix >> (lo + 1);
    const uint32_t limb = static_cast<uint32_t>(pl / a.batch), poly = static_cast<uint32_t>(pl % a.batch);
    const LimbConst lc = a.limbs[limb];
    const W q = static_cast<W>(lc.q);
    const Tw *tw = reinterpret_cast<const Tw *>(a.tw) + (static_cast<size_t>(limb) << L);
    const int64_t ubase = static_cast<int64_t>(limb) * a.limb_stride + static_cast<int64_t>(poly) * a.poly_stride;
    W *sc = scratch + (pl << L);
    const bool reads_user = GS ? ROLE == kLow : ROLE == kTop;
    const bool writes_user = GS ? ROLE == kTop : ROLE == kLow;
    constexpr int kPerThread = (32 << S) / kThreads;  // tile elements per thread
    constexpr int kBatch = 8;
    constexpr int TB = S - 5;

    // Element i (0 <= i < kPerThread) of this thread on each side of the
    // pass, as a per-thread base plus a per-i step (every field below is
    // disjoint in bits, so ORs are adds and XORs distribute):
    //   TOP, natural (lanes = columns): row = warp + 8i, global index
    //     (row << lo) | (t << 5) | lane, word row * 32 + (lane ^ (row >> TB));
    //   TOP, sigma (lanes = the row's top five bits): row = (lane << TB) | (i >> 2),
    //     column warp | 8(i & 3), sigma index (i >> 2) << (lo + 5) | t << 10 | column << 5 | lane;
    //   MID / LOW, sigma: row = warp + 8i, sigma index pfix << 5 | row << (lo + 5) | lane;
    //   LOW, bit-reversed (lane l takes column bitrev5(l)): row = warp + 8i, global
    //     index bitrev_L(column << (L-5) | t << S | row) = kb | bitrev_L(8i).
    const uint32_t lane = c.lane, warp = c.warp;
    const uint32_t col_r = __brev(lane) >> 27;
    const unsigned long long *uin = reinterpret_cast<const unsigned long long *>(a.in) + ubase;
    unsigned long long *uout = reinterpret_cast<unsigned long long *>(a.out) + ubase;
    const uint64_t nat_base = (static_cast<uint64_t>(warp) << lo) | (c.t << 5) | lane;
    const uint64_t nat_step = static_cast<uint64_t>(kWarps) << lo;
    const uint32_t nat_lx = lane ^ (warp >> TB);
    const uint64_t sgt_base = (static_cast<uint64_t>(c.t) << 10) | (warp << 5) | lane;
    const uint64_t sgt_step = 1ull << (lo + 5);
    const uint32_t sgt_s0 = (lane << (TB + 5)), sgt_wl = warp ^ lane;
    const uint64_t sg_base = (static_cast<uint64_t>(c.pfix) << 5) | (static_cast<uint64_t>(warp) << (lo + 5)) | lane;
    const uint64_t sg_step = static_cast<uint64_t>(kWarps) << (lo + 5);
    const uint32_t br_kb = __brev((col_r << (L - 5)) | (c.t << S) | warp) >> (32 - L);
    const uint32_t br_sh = 32 - L;
    auto nat_g = [&](int i) { return nat_base + static_cast<uint64_t>(i) * nat_step; };
    auto nat_s = [&](int i) { return (warp + kWarps * i) * 32u + (nat_lx ^ ((kWarps * i) >> TB)); };
    auto sgt_g = [&](int i) {
        return sgt_base + static_cast<uint64_t>(i >> 2) * sgt_step + (static_cast<uint64_t>(kWarps * (i & 3)) << 5);
    };
    auto sgt_s = [&](int i) { return sgt_s0 + (i >> 2) * 32u + (sgt_wl ^ (kWarps * (i & 3))); };
    auto sg_g = [&](int i) { return sg_base + static_cast<uint64_t>(i) * sg_step; };
    auto sg_s = [&](int i) { return (warp + kWarps * i) * 32u + lane; };
    auto br_g = [&](int i) { return br_kb | (__brev(static_cast<uint32_t>(kWarps * i)) >> br_sh); };
    auto br_s = [&](int i) { return (warp + kWarps * i) * 32u + col_r; };

    // ---------------------------------------------------------------- load
    uint32_t bad = 0;
    const W one_q = static_cast<W>(lc.one_shoup);
#pragma unroll 1
    for (int i0 = 0; i0 < kPerThread; i0 += kBatch) {
        if constexpr (ROLE == kTop) {
            if (reads_user) {
                unsigned long long x[kBatch];
#pragma unroll
                for (int i = 0; i < kBatch; ++i) x[i] = __ldcs(uin + nat_g(i0 + i));
#pragma unroll
                for (int i = 0; i < kBatch; ++i) tile[nat_s(i0 + i)] = A::load_reduce(x[i], q, one_q, bad);
            } else {
                W x[kBatch];
#pragma unroll
                for (int i = 0; i < kBatch; ++i) x[i] = __ldcs(sc + sgt_g(i0 + i));
#pragma unroll
                for (int i = 0; i < kBatch; ++i) tile[sgt_s(i0 + i)] = x[i];
            }
        } else {
            if (reads_user) {
                unsigned long long x[kBatch];
#pragma unroll
                for (int i = 0; i < kBatch; ++i) x[i] = __ldcs(uin + br_g(i0 + i));
#pragma unroll
                for (int i = 0; i < kBatch; ++i) tile[br_s(i0 + i)] = A::load_reduce(x[i], q, one_q, bad);
            } else {
                W x[kBatch];
#pragma unroll
                for (int i = 0; i < kBatch; ++i) x[i] = __ldcs(sc + sg_g(i0 + i));
#pragma unroll
                for (int i = 0; i < kBatch; ++i) tile[sg_s(i0 + i)] = x[i];
            }
        }
    }
    if constexpr (A::kBits == 32) {
        if (reads_user) flag_bad(a.status, bad);
    }
    __syncthreads();

    // ----------------------------------------------------------- butterflies
    rounds_from<A, GS, SCALE, S, ROLE, 0>(tile, tw, lc, c);
    __syncthreads();

    // --------------------------------------------------------------- store
#pragma unroll 8
    for (int i = 0; i < kPerThread; ++i) {
        if constexpr (ROLE == kTop) {
            if (writes_user)
                __stcs(uout + nat_g(i), static_cast<unsigned long long>(A::canon(tile[nat_s(i)], q)));
            else
                __stcs(sc + sgt_g(i), tile[sgt_s(i)]);
        } else {
            if (writes_user)
                __stcs(uout + br_g(i), static_cast<unsigned long long>(A::canon(tile[br_s(i)], q)));
            else
                __stcs(sc + sg_g(i), tile[sg_s(i)]);
        }
    }
}

}  // namespace mp
}  // namespace bc
