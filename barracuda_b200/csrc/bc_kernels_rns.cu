// bc_kernels_rns.cu -- Galois automorphisms (slot rotation), modulus
// switching and base-B digit decomposition: the coefficient-permuting and
// coefficient-rescaling steps around the transforms.  All three are
// HBM-bound: one read and one write per coefficient (decomposition writes
// one word per digit).
#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <string>

#include <cooperative_groups.h>

#include "bc_common.hpp"
#include "bc_kernels.hpp"

namespace bc {
namespace {

// 32-bit shared::cluster address of the word at local shared address `saddr`
// in the shared memory of cluster CTA `rank`, and a store to it.
__device__ __forceinline__ uint32_t cluster_addr(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
__device__ __forceinline__ void st_cluster_u64(uint32_t addr, uint64_t v) {
    asm volatile("st.shared::cluster.u64 [%0], %1;" ::"r"(addr), "l"(v) : "memory");
}

// Cluster barrier without memory ordering, for the barrier that only keeps
// a CTA from overwriting a peer's shared memory before the peer has read
// it: every value read before it has already been consumed by a store
// instruction, so the reads are complete, and a release would make the
// barrier wait for the HBM stores as well.
__device__ __forceinline__ void cluster_sync_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");
}

// fhe_rotate.wgsl:52-63: 0 stays 0, otherwise q - x with 64-bit wrap-around.
__device__ __forceinline__ uint64_t negate_mod(uint64_t x, uint64_t q) { return x == 0 ? 0 : q - x; }

// Automorphism X -> X^g of Z_q[X]/(X^N + 1) in gather form.  The reference
// scatters: input i goes to p = i g mod 2N, negated when p >= N.  Inverting
// that map, output j takes input t = j g^-1 mod 2N when t < N and the
// negation of input t - N otherwise (g^-1 is odd, so N g^-1 = N mod 2N and
// the two candidates differ by exactly N).  Writes are coalesced; reads are
// a permutation of one polynomial, served from L2.
// Each thread keeps kGatherILP gathers in flight (the kernel is bound by
// L2 latency, not bandwidth).  Index arithmetic is 32-bit: 2N divides 2^32.
constexpr uint32_t kGatherILP = 4;

__global__ void k_automorph_gather(KArgs a, uint32_t ginv, const CoeffConst *consts, uint64_t single_q) {
    const uint32_t L = a.logn;
    const uint32_t N = 1u << L, mask2 = 2 * N - 1;
    const uint32_t S = gridDim.x * blockDim.x;
    const uint64_t polys = static_cast<uint64_t>(a.batch) * a.n_limbs;
    for (uint64_t pl = blockIdx.y; pl < polys; pl += gridDim.y) {
        const uint64_t limb = pl / a.batch, poly = pl % a.batch;
        const uint64_t q = consts ? consts[limb].q : single_q;
        const int64_t base = static_cast<int64_t>(limb) * a.limb_stride + static_cast<int64_t>(poly) * a.poly_stride;
        const uint64_t *in = a.in + base;
        uint64_t *out = a.out + base;
        for (uint32_t j0 = blockIdx.x * blockDim.x + threadIdx.x; j0 < N; j0 += kGatherILP * S) {
            uint64_t x[kGatherILP];
            uint32_t t[kGatherILP];
#pragma unroll
            for (uint32_t k = 0; k < kGatherILP; ++k) {
                const uint32_t j = j0 + k * S;
                t[k] = (j * ginv) & mask2;
                x[k] = j < N ? __ldcg(in + (t[k] & (N - 1))) : 0;  // L2 only: L1 sees no reuse
            }
#pragma unroll
            for (uint32_t k = 0; k < kGatherILP; ++k) {
                const uint32_t j = j0 + k * S;
                if (j < N) __stcs(out + j, (t[k] >> L) ? negate_mod(x[k], q) : x[k]);
            }
        }
    }
}

// Scatter form, as the reference's shader writes it: each thread reads two
// consecutive words with one 16-byte load and stores each to its image
// p = t g mod 2N (negated in the upper half).  Reads are full sectors; the
// 8-byte writes of one sector land in four different places.
__global__ void k_automorph_scatter(KArgs a, uint32_t galois, const CoeffConst *consts, uint64_t single_q) {
    const uint32_t L = a.logn;
    const uint32_t N = 1u << L, mask2 = 2 * N - 1;
    const uint64_t polys = static_cast<uint64_t>(a.batch) * a.n_limbs;
    for (uint64_t pl = blockIdx.y; pl < polys; pl += gridDim.y) {
        const uint64_t limb = pl / a.batch, poly = pl % a.batch;
        const uint64_t q = consts ? consts[limb].q : single_q;
        const int64_t base = static_cast<int64_t>(limb) * a.limb_stride + static_cast<int64_t>(poly) * a.poly_stride;
        uint64_t *out = a.out + base;
        for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; 2 * i < N; i += gridDim.x * blockDim.x) {
            const ulonglong2 w = __ldcs(reinterpret_cast<const ulonglong2 *>(a.in + base) + i);
            const uint32_t p0 = (2 * i * galois) & mask2, p1 = ((2 * i + 1) * galois) & mask2;
            out[p0 & (N - 1)] = (p0 >> L) ? negate_mod(w.x, q) : w.x;
            out[p1 & (N - 1)] = (p1 >> L) ? negate_mod(w.y, q) : w.y;
        }
    }
}

// Same map for polynomials that fit in shared memory: one CTA stages a
// whole polynomial with coalesced loads, then gathers from shared memory.
// Consecutive outputs read words g^-1 apart (odd), so the 16 lanes of each
// 8-byte shared-memory phase hit 16 different bank pairs.
__global__ void __launch_bounds__(512) k_automorph_smem(KArgs a, uint32_t ginv, const CoeffConst *consts,
                                                        uint64_t single_q) {
    extern __shared__ uint64_t poly_s[];
    const uint32_t L = a.logn;
    const uint32_t N = 1u << L, mask2 = 2 * N - 1;
    const uint64_t polys = static_cast<uint64_t>(a.batch) * a.n_limbs;
    for (uint64_t pl = blockIdx.x; pl < polys; pl += gridDim.x) {
        const uint64_t limb = pl / a.batch, poly = pl % a.batch;
        const uint64_t q = consts ? consts[limb].q : single_q;
        const int64_t base = static_cast<int64_t>(limb) * a.limb_stride + static_cast<int64_t>(poly) * a.poly_stride;
        for (uint32_t i = threadIdx.x; i < N; i += blockDim.x) poly_s[i] = __ldcs(a.in + base + i);
        __syncthreads();
        for (uint32_t j = threadIdx.x; j < N; j += blockDim.x) {
            const uint32_t t = (j * ginv) & mask2;  // j, ginv < 2^14: no overflow
            const uint64_t x = poly_s[t & (N - 1)];
            __stcs(a.out + base + j, (t >> L) ? negate_mod(x, q) : x);
        }
        __syncthreads();
    }
}

// Polynomials of 2^14..2^17 words: one cluster of C = N / 8192 CTAs per
// polynomial, built on the low-bit structure of the map.  Write
// j = jl + C jh (jl < C).  Then t = j h mod 2N (h = g^-1) is
// r + C u with r = jl h mod C: output residue class jl (mod C) draws only on
// input residue class r, through u = (kappa + jh h) mod 2N/C, where
// kappa = (jl h - r) / C, and u >= N/C marks the negated half.  So:
//   1. CTA s loads input block s (8192 contiguous words, coalesced) and
//      sends word t to CTA t mod C at index t / C: every CTA ends up holding
//      one whole residue class in shared memory (remote stores of 64 to
//      256 contiguous bytes per warp instruction);
//   2. CTA r gathers output class jl = r g mod C from its own class (local
//      shared memory, conflict-free: consecutive jh read words h apart, h
//      odd) and sends each value to the CTA whose output block holds it,
//      stored class-major with a 16/C-word pad per class so that step 3
//      reads without bank conflicts;
//   3. CTA s writes output block s with coalesced stores.
// HBM sees one read and one write per word; four cluster barriers per
// polynomial order the exchanges, and two CTAs per SM overlap clusters.
// DIRECT skips the second exchange: each CTA stores its output class
// straight to HBM (stride C words) and L2 merges the partial sectors the C
// CTAs of the cluster write together.
constexpr uint32_t kClusterWords = 8192;
constexpr uint32_t kClusterThreads = 512;

template <int LOGC, bool DIRECT>
__global__ void __launch_bounds__(kClusterThreads, 2)
    k_automorph_cluster(KArgs a, uint32_t galois, uint32_t ginv, const CoeffConst *consts, uint64_t single_q,
                        int vec) {
    namespace cg = cooperative_groups;
    constexpr uint32_t C = 1u << LOGC, B = kClusterWords, T = kClusterThreads, kPer = B / T;
    constexpr uint32_t kCol = B / C, kStride = kCol + 16 / C;  // class-major output block
    extern __shared__ uint64_t buf[];                           // B + 16 words
    cg::cluster_group cl = cg::this_cluster();
    const uint32_t rank = cl.block_rank();
    const uint32_t sbuf = static_cast<uint32_t>(__cvta_generic_to_shared(buf));
    // this CTA's output class and the offset of its sources in its input class
    const uint32_t jl = (rank * galois) & (C - 1);
    const uint32_t kappa = (jl * ginv - rank) >> LOGC;
    const uint64_t polys = static_cast<uint64_t>(a.batch) * a.n_limbs;
    const uint64_t clusters = gridDim.x >> LOGC;
    for (uint64_t pl = blockIdx.x >> LOGC; pl < polys; pl += clusters) {
        const uint64_t limb = pl / a.batch, poly = pl % a.batch;
        const uint64_t q = consts ? consts[limb].q : single_q;
        const int64_t base = static_cast<int64_t>(limb) * a.limb_stride + static_cast<int64_t>(poly) * a.poly_stride +
                             static_cast<int64_t>(rank) * B;
        // 1. input block -> residue classes
        const uint64_t *src = a.in + base;
#pragma unroll 4
        for (uint32_t k = 0; k < kPer / 2; ++k) {
            const uint32_t e = 2 * (k * T + threadIdx.x);
            uint64_t w0, w1;
            if (vec) {
                const ulonglong2 w = __ldcs(reinterpret_cast<const ulonglong2 *>(src + e));
                w0 = w.x;
                w1 = w.y;
            } else {
                w0 = __ldcs(src + e);
                w1 = __ldcs(src + e + 1);
            }
            const uint32_t t = rank * B + e;  // t and t + 1 never share a class (C >= 2)
            st_cluster_u64(cluster_addr(sbuf + 8 * (t >> LOGC), t & (C - 1)), w0);
            st_cluster_u64(cluster_addr(sbuf + 8 * ((t + 1) >> LOGC), (t + 1) & (C - 1)), w1);
        }
        cl.sync();
        if constexpr (DIRECT) {  // output class straight to HBM (stride C words)
            uint64_t *dst = a.out + (base - static_cast<int64_t>(rank) * B) + jl;
#pragma unroll 4
            for (uint32_t k = 0; k < kPer; ++k) {
                const uint32_t jh = k * T + threadIdx.x;
                const uint32_t u = (kappa + jh * ginv) & (2 * B - 1);
                const uint64_t x = buf[u & (B - 1)];
                __stcs(dst + static_cast<size_t>(jh) * C, (u & B) ? negate_mod(x, q) : x);
            }
        } else {
            // 2. permute within the class (into registers) ...
            uint64_t v[kPer];
#pragma unroll
            for (uint32_t k = 0; k < kPer; ++k) {
                const uint32_t jh = k * T + threadIdx.x;
                const uint32_t u = (kappa + jh * ginv) & (2 * B - 1);
                const uint64_t x = buf[u & (B - 1)];
                v[k] = (u & B) ? negate_mod(x, q) : x;
            }
            cl.sync();
            // ... and send each output word to the CTA that stores its block
#pragma unroll
            for (uint32_t k = 0; k < kPer; ++k) {
                const uint32_t jh = k * T + threadIdx.x;
                st_cluster_u64(cluster_addr(sbuf + 8 * (jl * kStride + jh % kCol), jh / kCol), v[k]);
            }
            cl.sync();
            // 3. output block, coalesced
            uint64_t *dst = a.out + base;
#pragma unroll 4
            for (uint32_t k = 0; k < kPer; ++k) {
                const uint32_t p = k * T + threadIdx.x;
                __stcs(dst + p, buf[(p & (C - 1)) * kStride + (p >> LOGC)]);
            }
        }
        cluster_sync_relaxed();
    }
}

template <int LOGC, bool DIRECT>
int launch_automorph_cluster(const KArgs &a, uint32_t galois, uint32_t ginv, const CoeffConst *consts,
                             uint64_t single_q, cudaStream_t s) {
    auto kern = k_automorph_cluster<LOGC, DIRECT>;
    constexpr size_t smem = (kClusterWords + 16) * sizeof(uint64_t);
    static std::atomic<int> resident[64];
    int dev = 0;
    cudaGetDevice(&dev);
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(kClusterThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1u << LOGC;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeClusterSchedulingPolicyPreference;
    attr[1].val.clusterSchedulingPolicyPreference = static_cast<cudaClusterSchedulingPolicy>(cluster_policy());
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    int nres = dev < 64 ? resident[dev].load() : 0;
    if (nres == 0) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return cuda_fail(e, "k_automorph_cluster shared-memory attribute");
        if (LOGC > 3) {  // clusters of 16 CTAs: a non-portable size B200 supports
            e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
            if (e != cudaSuccess) return cuda_fail(e, "k_automorph_cluster cluster-size attribute");
        }
        cfg.gridDim = dim3((1u << LOGC) * 1024);
        e = cudaOccupancyMaxActiveClusters(&nres, kern, &cfg);
        if (e != cudaSuccess) return cuda_fail(e, "k_automorph_cluster occupancy");
        if (nres <= 0)
            return fail(BC_ERR_UNSUPPORTED, format("k_automorph_cluster: no cluster of %d CTAs fits", 1 << LOGC));
        if (dev < 64) resident[dev].store(nres);
    }
    const uint64_t polys = static_cast<uint64_t>(a.batch) * a.n_limbs;
    const uint64_t clusters = polys < static_cast<uint64_t>(nres) ? polys : static_cast<uint64_t>(nres);
    cfg.gridDim = dim3(static_cast<unsigned>(clusters << LOGC));
    const int vec = (reinterpret_cast<uintptr_t>(a.in) % 16 == 0 && a.limb_stride % 2 == 0 && a.poly_stride % 2 == 0)
                        ? 1 : 0;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a, galois, ginv, consts, single_q, vec);
    if (e != cudaSuccess) return cuda_fail(e, "k_automorph_cluster launch");
    return BC_OK;
}

// round(c * P / Q) mod P for any u64 c (ties up), P < Q, exactly:
//   c = a Q + b with a = floor(c / Q) (estimate floor(c m / 2^64),
//   m = floor(2^64 / Q), at most one below); then c P / Q = a P + b P / Q
//   and a P vanishes mod P.  t = floor(b P / Q) comes from the Shoup
//   constant Pp = floor(P 2^64 / Q) (at most one below), the remainder
//   b P - t Q (< 2Q, held in 65 bits) corrects it and decides the rounding.
//   t + round <= P, so the final reduction is one comparison.
__device__ __forceinline__ uint64_t modulus_switch_one(uint64_t x, const ModSwitchConst &c) {
    if (c.q_new == 0) return 0;
    uint64_t b = x;
    if (b >= c.q_old) {  // inputs are usually already below q_old
        b = x - __umul64hi(x, c.m_old) * c.q_old;
        if (b >= c.q_old) b -= c.q_old;
    }
    uint64_t t = __umul64hi(b, c.p_shoup);
    const uint64_t lo1 = b * c.q_new, lo2 = t * c.q_old;
    uint64_t rem = lo1 - lo2;
    // the remainder is below 2 q_old: 64 bits hold it unless q_old > 2^63
    const bool over = c.q_old > (1ull << 63)
                          ? (__umul64hi(b, c.q_new) - __umul64hi(t, c.q_old) - (lo1 < lo2 ? 1 : 0)) != 0
                          : false;
    if (over || rem >= c.q_old) {
        rem -= c.q_old;
        ++t;
    }
    if (rem >= c.q_old - rem) ++t;
    return t == c.q_new ? 0 : t;
}

// Two words per thread per iteration, both loads issued first.
// Four words a grid stride apart per thread and step, all loaded before any
// arithmetic, so that the loads of a thread overlap (measured on B200: the
// coefficient-wise kernels gained 10-15% of HBM bandwidth over one or two).
constexpr int kRnsUnroll = 4;

__global__ void k_modulus_switch(const uint64_t *__restrict__ in, uint64_t *__restrict__ out, size_t count,
                                 ModSwitchConst c) {
    const size_t S = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i0 = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i0 < count; i0 += kRnsUnroll * S) {
        uint64_t x[kRnsUnroll];
#pragma unroll
        for (int u = 0; u < kRnsUnroll; ++u)
            if (i0 + u * S < count) x[u] = __ldcs(in + i0 + u * S);
#pragma unroll
        for (int u = 0; u < kRnsUnroll; ++u)
            if (i0 + u * S < count) __stcs(out + i0 + u * S, modulus_switch_one(x[u], c));
    }
}

// Digit l of every coefficient, digit-major: out[l * count + i] =
// floor(in[i] / B^l) mod B.  Each division by B uses m = floor(2^64 / B):
// the estimate floor(x m / 2^64) is at most one below floor(x / B).
__global__ void k_decompose(const uint64_t *__restrict__ in, uint64_t *__restrict__ out, size_t count,
                            uint32_t base, uint32_t levels, uint64_t m) {
    const size_t S = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i0 = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i0 < count; i0 += kRnsUnroll * S) {
        uint64_t x[kRnsUnroll];
#pragma unroll
        for (int u = 0; u < kRnsUnroll; ++u)
            if (i0 + u * S < count) x[u] = __ldcs(in + i0 + u * S);
        for (uint32_t l = 0; l < levels; ++l) {
#pragma unroll
            for (int u = 0; u < kRnsUnroll; ++u) {
                if (i0 + u * S >= count) continue;
                uint64_t q = __umul64hi(x[u], m);
                uint64_t r = x[u] - q * base;
                if (r >= base) {
                    r -= base;
                    ++q;
                }
                __stcs(out + static_cast<size_t>(l) * count + i0 + u * S, r);
                x[u] = q;
            }
        }
    }
}

int check_launch_rns(const char *what) {
    const cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) return BC_OK;
    return fail(e == cudaErrorMemoryAllocation ? BC_ERR_OUT_OF_MEMORY : BC_ERR_GPU,
                format("%s launch failed: %s", what, cudaGetErrorString(e)));
}

unsigned grid_1d(uint64_t work, unsigned threads) {
    uint64_t blocks = (work + kRnsUnroll * threads - 1) / (kRnsUnroll * threads);
    const uint64_t cap = 148ull * 16;
    if (blocks > cap) blocks = cap;
    return static_cast<unsigned>(blocks ? blocks : 1);
}

// Largest log2 N staged whole in shared memory (64 KiB per CTA: three CTAs
// per SM keep loads of one polynomial in flight while another is stored).
constexpr uint32_t kAutomorphSmemMaxLogn = 13;

}  // namespace

uint32_t odd_inverse_pow2(uint32_t g, uint32_t logm) {
    // Newton's iteration x <- x (2 - g x) doubles the correct low bits of the
    // inverse of an odd g modulo 2^k (g is its own inverse modulo 8).
    uint64_t x = g;
    for (int i = 0; i < 5; ++i) x *= 2 - static_cast<uint64_t>(g) * x;
    return static_cast<uint32_t>(x & ((1ull << logm) - 1));
}

ModSwitchConst modswitch_const(uint64_t q_old, uint64_t q_new) {
    ModSwitchConst c = {};
    c.q_old = q_old;
    c.q_new = q_new;
    if (q_new != 0) {  // then q_old >= 2
        c.m_old = static_cast<uint64_t>((static_cast<unsigned __int128>(1) << 64) / q_old);
        c.p_shoup = static_cast<uint64_t>((static_cast<unsigned __int128>(q_new) << 64) / q_old);
    }
    return c;
}

int launch_automorphism(const KArgs &a, uint32_t galois, const CoeffConst *consts, uint64_t single_q,
                        cudaStream_t s) {
    const uint64_t polys = static_cast<uint64_t>(a.batch) * a.n_limbs;
    if (polys == 0) return BC_OK;
    const uint32_t ginv = odd_inverse_pow2(galois, a.logn + 1);
    const uint64_t N = 1ull << a.logn;
    if (a.logn <= kAutomorphSmemMaxLogn) {
        const unsigned T = N >= 512 ? 512 : static_cast<unsigned>(N);
        const size_t smem = N * sizeof(uint64_t);
        if (smem > 48 * 1024) {
            const cudaError_t e = cudaFuncSetAttribute(k_automorph_smem, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                       static_cast<int>(smem));
            if (e != cudaSuccess) return cuda_fail(e, "k_automorph_smem shared-memory attribute");
        }
        const uint64_t per_sm = N <= 1024 ? 4 : 3;
        const uint64_t grid = polys < 148 * per_sm * 8 ? polys : 148 * per_sm * 8;
        k_automorph_smem<<<static_cast<unsigned>(grid), T, smem, s>>>(a, ginv, consts, single_q);
        return check_launch_rns("k_automorph_smem");
    }
    // Kernel for N above the shared-memory size.  Measured on B200 (16-limb
    // batches of 2^28 words, fraction of HBM copy bandwidth):
    //   N        gather  scatter  cluster  cluster+direct
    //   2^14      0.45    0.46     0.50     0.67
    //   2^15      0.55    0.46     0.41     0.39
    //   2^16      0.55    0.40     0.33     0.35
    //   2^17      0.54    0.27     0.25     0.20
    // BARRACUDA_AUTOMORPH_KERNEL=gather|scatter|cluster|direct overrides.
    static const int forced = [] {
        const char *e = std::getenv("BARRACUDA_AUTOMORPH_KERNEL");
        if (!e) return 0;
        const std::string v(e);
        return v == "gather" ? 1 : v == "scatter" ? 2 : v == "cluster" ? 3 : v == "direct" ? 4 : 0;
    }();
    const bool aligned = reinterpret_cast<uintptr_t>(a.in) % 16 == 0 && a.limb_stride % 2 == 0 &&
                         a.poly_stride % 2 == 0;
    const bool clusterable = a.logn >= 14 && a.logn <= 17;
    const int kind = forced ? forced : (a.logn == 14 ? 4 : 1);
    if ((kind == 3 || kind == 4) && clusterable) {
        const bool direct = kind == 4;
        switch (a.logn) {  // one polynomial per cluster of 2..16 CTAs
        case 14:
            return direct ? launch_automorph_cluster<1, true>(a, galois, ginv, consts, single_q, s)
                          : launch_automorph_cluster<1, false>(a, galois, ginv, consts, single_q, s);
        case 15:
            return direct ? launch_automorph_cluster<2, true>(a, galois, ginv, consts, single_q, s)
                          : launch_automorph_cluster<2, false>(a, galois, ginv, consts, single_q, s);
        case 16:
            return direct ? launch_automorph_cluster<3, true>(a, galois, ginv, consts, single_q, s)
                          : launch_automorph_cluster<3, false>(a, galois, ginv, consts, single_q, s);
        default:
            return direct ? launch_automorph_cluster<4, true>(a, galois, ginv, consts, single_q, s)
                          : launch_automorph_cluster<4, false>(a, galois, ginv, consts, single_q, s);
        }
    }
    const unsigned T = 256;
    if (kind == 2 && aligned) {
        uint64_t bx = (N / 2 + T - 1) / T;
        if (bx > 64) bx = 64;
        const dim3 grid(static_cast<unsigned>(bx), static_cast<unsigned>(polys < 65535 ? polys : 65535));
        k_automorph_scatter<<<grid, T, 0, s>>>(a, galois, consts, single_q);
        return check_launch_rns("k_automorph_scatter");
    }
    uint64_t bx = (N + T - 1) / T;
    if (bx > 64) bx = 64;
    const dim3 grid(static_cast<unsigned>(bx), static_cast<unsigned>(polys < 65535 ? polys : 65535));
    k_automorph_gather<<<grid, T, 0, s>>>(a, ginv, consts, single_q);
    return check_launch_rns("k_automorph_gather");
}

int launch_modulus_switch(const uint64_t *in, uint64_t *out, size_t count, const ModSwitchConst &c,
                          cudaStream_t s) {
    if (count == 0) return BC_OK;
    k_modulus_switch<<<grid_1d(count, 256), 256, 0, s>>>(in, out, count, c);
    return check_launch_rns("k_modulus_switch");
}

int launch_decompose(const uint64_t *in, uint64_t *out, size_t count, uint32_t base, uint32_t levels,
                     cudaStream_t s) {
    if (count == 0 || levels == 0) return BC_OK;
    const uint64_t m = static_cast<uint64_t>((static_cast<unsigned __int128>(1) << 64) / base);
    k_decompose<<<grid_1d(count, 256), 256, 0, s>>>(in, out, count, base, levels, m);
    return check_launch_rns("k_decompose");
}

}  // namespace bc
