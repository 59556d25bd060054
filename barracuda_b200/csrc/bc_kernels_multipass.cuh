// bc_kernels_multipass.cuh -- the transform for N = 2^18 .. 2^24: two or
// three passes through HBM instead of one launch per stage.
//
// Positions p in [0, N), N = 2^L, are split into bit fields.  A pass owns S
// consecutive bits [lo, lo + S) and runs every butterfly stage of those bits
// on independent sub-transforms: the positions that agree in every other
// bit.  One CTA holds a tile of 32 such sub-transforms (32 "columns" x 2^S
// "rows") in shared memory; warps take the columns as lanes, so every
// shared-memory access of a warp touches 32 distinct banks, and each pass's
// butterflies run in register rounds of up to 3 bits (radix 8) between
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

// Register rounds of a pass of S bits, from the lowest bits up: widths of
// at most 3 bits, each leaving at least 8 tasks (one per warp).
__host__ __device__ constexpr int round_count(int S) { return S <= 6 ? 2 : 3; }
__host__ __device__ constexpr int round_width(int S, int r) {
    // S = 6: 3 3 / 7: 2 2 3 / 8: 2 3 3 / 9: 3 3 3
    return S == 6 ? 3 : S == 7 ? (r == 2 ? 3 : 2) : S == 8 ? (r == 0 ? 2 : 3) : 3;
}
__host__ __device__ constexpr int round_lo(int S, int r) {
    int lo = 0;
    for (int i = 0; i < r; ++i) lo += round_width(S, i);
    return lo;
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
    int scale;            // fold N^-1 into the transform's last stage
};

template <class A>
__device__ __forceinline__ void bfly(bool gs, bool scaled, typename A::W &x, typename A::W &y,
                                     const typename A::Tw &w, const LimbConst &lc) {
    using W = typename A::W;
    const W q = static_cast<W>(lc.q);
    if (scaled) {
        const W s = static_cast<W>(lc.ninv), sq = static_cast<W>(lc.ninv_shoup);
        if (gs)
            A::gs_scaled(x, y, w.x, w.y, s, sq, q);
        else
            A::ct_scaled(x, y, w.x, w.y, s, sq, q);
    } else {
        if (gs)
            A::gs(x, y, w.x, w.y, q);
        else
            A::ct(x, y, w.x, w.y, q);
    }
}

// One register round: bits [RR, RR + K) of the row (absolute position bits
// lo + RR ..).  Each thread runs the round's K stages on 2^K coefficients of
// its column (= lane) per task; a task fixes the row's other bits.
template <class A, bool GS, int S, int ROLE, int RR, int K>
__device__ __forceinline__ void pass_round(typename A::W *tile, const typename A::Tw *tw, const LimbConst &lc,
                                      const Ctx &c) {
    using W = typename A::W;
    using Tw = typename A::Tw;
    constexpr int kTasks = 1 << (S - K);
    constexpr int kPer = kTasks / kWarps;
    static_assert(kPer >= 1, "a round must give every warp a task");
    const uint32_t L = c.L;
    // Position bits of this tile other than the pass's rows and the column
    // (MID / LOW: t splits around the pass's bits; TOP: t is bits [5, lo)).
    const uint32_t t_lo = c.t & ((1u << c.lo) - 1u), t_hi = c.t >> c.lo;
#pragma unroll 1
    for (int it = 0; it < kPer; ++it) {
        const uint32_t g = c.warp + kWarps * it;
        const uint32_t base = ((g >> RR) << (RR + K)) | (g & ((1u << RR) - 1u));
        W v[1 << K];
#pragma unroll
        for (int m = 0; m < (1 << K); ++m) {
            const uint32_t row = base | (static_cast<uint32_t>(m) << RR);
            v[m] = tile[tile_addr<S, ROLE>(row, c.lane)];
        }
#pragma unroll
        for (int jj = 0; jj < K; ++jj) {
            const int j = GS ? jj : K - 1 - jj;
            const uint32_t b = c.lo + RR + j;
            const bool scaled = c.scale && b == (GS ? L - 1 : 0u);
            // table block of stage b and this task's entry for m = 0
            const Tw *tb;
            if constexpr (ROLE == kTop) {
                tb = tw + ((1u << (L - b - 1)) + (base >> (RR + j + 1)));
            } else {
                const uint32_t pn = (t_hi << (c.lo + S)) | (base << c.lo) | t_lo;  // p without the column
                const uint32_t mask = (1u << (L - b - 6)) - 1u;
                tb = tw + ((1u << (L - b - 1)) + (((pn >> (b + 1)) & mask) << 5) + c.lane);
            }
            constexpr int kStride = ROLE == kTop ? 1 : 32;
#pragma unroll
            for (int m = 0; m < (1 << K); ++m) {
                if (m & (1 << j)) continue;
                const Tw w = __ldg(tb + (m >> (j + 1)) * kStride);
                bfly<A>(GS, scaled, v[m], v[m | (1 << j)], w, lc);
            }
        }
#pragma unroll
        for (int m = 0; m < (1 << K); ++m) {
            const uint32_t row = base | (static_cast<uint32_t>(m) << RR);
            tile[tile_addr<S, ROLE>(row, c.lane)] = v[m];
        }
    }
}

template <class A, bool GS, int S, int ROLE, int R>
__device__ __forceinline__ void rounds_from(typename A::W *tile, const typename A::Tw *tw, const LimbConst &lc,
                                            const Ctx &c) {
    // CT runs the rounds from the top bits down, GS from the bottom up.
    constexpr int NR = round_count(S);
    constexpr int r = GS ? R : NR - 1 - R;
    pass_round<A, GS, S, ROLE, round_lo(S, r), round_width(S, r)>(tile, tw, lc, c);
    if constexpr (R + 1 < NR) {
        __syncthreads();
        rounds_from<A, GS, S, ROLE, R + 1>(tile, tw, lc, c);
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
template <class A, bool GS, int S, int ROLE>
__global__ void __launch_bounds__(kThreads) k_ntt_pass(KArgs a, typename A::W *scratch, uint32_t lo,
                                                       int scale) {
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
    c.scale = scale;
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
    const uint32_t t_lo = c.t & ((1u << lo) - 1u), t_hi = c.t >> lo;

    // ---------------------------------------------------------------- load
    uint32_t bad = 0;
    if constexpr (ROLE == kTop) {
        if (reads_user) {  // natural order, lanes = columns
#pragma unroll 1
            for (int i0 = 0; i0 < kPerThread; i0 += kBatch) {
                uint64_t x[kBatch];
#pragma unroll
                for (int i = 0; i < kBatch; ++i) {
                    const uint32_t row = c.warp + kWarps * (i0 + i);
                    x[i] = __ldcs(reinterpret_cast<const unsigned long long *>(a.in) + ubase + ((static_cast<int64_t>(row) << lo) | (c.t << 5) | c.lane));
                }
#pragma unroll
                for (int i = 0; i < kBatch; ++i) {
                    const uint32_t row = c.warp + kWarps * (i0 + i);
                    tile[tile_addr<S, ROLE>(row, c.lane)] =
                        A::load_reduce(x[i], q, static_cast<W>(lc.one_shoup), bad);
                }
            }
        } else {  // sigma order, lanes = the row's top five bits
#pragma unroll 1
            for (int i0 = 0; i0 < kPerThread; i0 += kBatch) {
                W x[kBatch];
#pragma unroll
                for (int i = 0; i < kBatch; ++i) {
                    const uint32_t pr = c.warp + kWarps * (i0 + i), rlo = pr >> 5, col = pr & 31u;
                    x[i] = __ldcs(sc + ((((static_cast<uint64_t>(rlo) << lo) | (c.t << 5) | col) << 5) | c.lane));
                }
#pragma unroll
                for (int i = 0; i < kBatch; ++i) {
                    const uint32_t pr = c.warp + kWarps * (i0 + i), rlo = pr >> 5, col = pr & 31u;
                    tile[tile_addr<S, ROLE>((c.lane << (S - 5)) | rlo, col)] = x[i];
                }
            }
        }
    } else {
        if (reads_user) {  // LOW, bit-reversed order: lane l takes column bitrev5(l)
            const uint32_t col = __brev(c.lane) >> 27;
#pragma unroll 1
            for (int i0 = 0; i0 < kPerThread; i0 += kBatch) {
                uint64_t x[kBatch];
#pragma unroll
                for (int i = 0; i < kBatch; ++i) {
                    const uint32_t row = c.warp + kWarps * (i0 + i);
                    const uint32_t p = (col << (L - 5)) | (t_hi << S) | row;
                    x[i] = __ldcs(reinterpret_cast<const unsigned long long *>(a.in) + ubase + (__brev(p) >> (32 - L)));
                }
#pragma unroll
                for (int i = 0; i < kBatch; ++i) {
                    const uint32_t row = c.warp + kWarps * (i0 + i);
                    tile[tile_addr<S, ROLE>(row, col)] = A::load_reduce(x[i], q, static_cast<W>(lc.one_shoup), bad);
                }
            }
        } else {  // sigma order, lanes = columns
#pragma unroll 1
            for (int i0 = 0; i0 < kPerThread; i0 += kBatch) {
                W x[kBatch];
#pragma unroll
                for (int i = 0; i < kBatch; ++i) {
                    const uint32_t row = c.warp + kWarps * (i0 + i);
                    x[i] = __ldcs(sc + ((static_cast<uint64_t>((t_hi << (lo + S)) | (row << lo) | t_lo) << 5) | c.lane));
                }
#pragma unroll
                for (int i = 0; i < kBatch; ++i) {
                    const uint32_t row = c.warp + kWarps * (i0 + i);
                    tile[tile_addr<S, ROLE>(row, c.lane)] = x[i];
                }
            }
        }
    }
    if constexpr (A::kBits == 32) {
        if (reads_user) flag_bad(a.status, bad);
    }
    __syncthreads();

    // ----------------------------------------------------------- butterflies
    rounds_from<A, GS, S, ROLE, 0>(tile, tw, lc, c);
    __syncthreads();

    // --------------------------------------------------------------- store
    if constexpr (ROLE == kTop) {
        if (writes_user) {  // natural order, canonical residues
#pragma unroll 4
            for (int i = 0; i < kPerThread; ++i) {
                const uint32_t row = c.warp + kWarps * i;
                __stcs(reinterpret_cast<unsigned long long *>(a.out) + ubase + ((static_cast<int64_t>(row) << lo) | (c.t << 5) | c.lane),
                       static_cast<unsigned long long>(A::canon(tile[tile_addr<S, ROLE>(row, c.lane)], q)));
            }
        } else {
#pragma unroll 4
            for (int i = 0; i < kPerThread; ++i) {
                const uint32_t pr = c.warp + kWarps * i, rlo = pr >> 5, col = pr & 31u;
                __stcs(sc + ((((static_cast<uint64_t>(rlo) << lo) | (c.t << 5) | col) << 5) | c.lane),
                       tile[tile_addr<S, ROLE>((c.lane << (S - 5)) | rlo, col)]);
            }
        }
    } else {
        if (writes_user) {  // LOW, bit-reversed order
            const uint32_t col = __brev(c.lane) >> 27;
#pragma unroll 4
            for (int i = 0; i < kPerThread; ++i) {
                const uint32_t row = c.warp + kWarps * i;
                const uint32_t p = (col << (L - 5)) | (t_hi << S) | row;
                __stcs(reinterpret_cast<unsigned long long *>(a.out) + ubase + (__brev(p) >> (32 - L)),
                       static_cast<unsigned long long>(A::canon(tile[tile_addr<S, ROLE>(row, col)], q)));
            }
        } else {
#pragma unroll 4
            for (int i = 0; i < kPerThread; ++i) {
                const uint32_t row = c.warp + kWarps * i;
                __stcs(sc + ((static_cast<uint64_t>((t_hi << (lo + S)) | (row << lo) | t_lo) << 5) | c.lane),
                       tile[tile_addr<S, ROLE>(row, c.lane)]);
            }
        }
    }
}

}  // namespace mp
}  // namespace bc
