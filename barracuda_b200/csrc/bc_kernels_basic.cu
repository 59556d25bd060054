// bc_kernels_basic.cu -- straightforward sm_100a kernels of the FHE path:
// a stage-per-barrier shared-memory NTT (small N and fallback), the
// multi-pass global-memory NTT for N beyond shared memory, pointwise
// products, the fused shared-memory polymul, the seeded input generator and
// the digest used for cross-GPU checks.
//
// Position convention used by every transform kernel: the Cooley-Tukey
// network works in place on positions p in [0, N); the stage that flips bit
// b of p pairs (p, p | 2^b) for p with bit b clear and uses twiddle entry
// m + i of its table, where m = N / 2^(b+1) is the number of butterfly
// groups of the stage and i = p >> (b+1) the group index.  CT runs b from
// log2 N - 1 down to 0 on natural-order input and leaves position p holding
// output index bitrev(p); GS runs b upwards on bit-reversed input and
// leaves natural order.
#include <cstdint>

#include "bc_common.hpp"
#include "bc_kernels.hpp"

namespace bc {
namespace {

__device__ __forceinline__ uint32_t brev_bits(uint32_t x, uint32_t bits) {
    return __brev(x) >> (32 - bits);
}

__device__ __forceinline__ void raise_status(uint32_t *status, bool bad, uint32_t bit) {
    if (__any_sync(0xffffffffu, bad)) {
        if ((threadIdx.x & 31) == 0) store_status(status, bit);
    }
}

template <class A>
__device__ __forceinline__ void butterfly(bool gs, bool scaled, typename A::W &x,
                                          typename A::W &y, const typename A::Tw &w,
                                          const LimbConst &lc) {
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

// All log2 N stages of one transform on a shared-memory array.
template <class A, bool GS>
__device__ __forceinline__ void smem_stages(typename A::W *s, const typename A::Tw *tw,
                                            uint32_t L, bool scale_last,
                                            const LimbConst &lc) {
    using W = typename A::W;
    const uint32_t N = 1u << L, half = N >> 1;
    for (uint32_t st = 0; st < L; ++st) {
        const uint32_t b = GS ? st : (L - 1 - st);
        const uint32_t m = N >> (b + 1);
        const bool scaled = scale_last && (st == L - 1);
        for (uint32_t t = threadIdx.x; t < half; t += blockDim.x) {
            const uint32_t i = t >> b;
            const uint32_t p0 = (i << (b + 1)) | (t & ((1u << b) - 1u));
            const uint32_t p1 = p0 | (1u << b);
            W x = s[p0], y = s[p1];
            butterfly<A>(GS, scaled, x, y, tw[m + i], lc);
            s[p0] = x;
            s[p1] = y;
        }
        __syncthreads();
    }
}

template <class A, bool GS>
__global__ void __launch_bounds__(512) k_ntt_smem(KArgs a, int scale_last) {
    using W = typename A::W;
    using Tw = typename A::Tw;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    W *s = reinterpret_cast<W *>(smem_raw);
    const uint32_t limb = blockIdx.y, poly = blockIdx.x;
    const uint32_t L = a.logn, N = 1u << L;
    const LimbConst lc = a.limbs[limb];
    const W q = static_cast<W>(lc.q), one_q = static_cast<W>(lc.one_shoup);
    const int64_t base = static_cast<int64_t>(limb) * a.limb_stride +
                         static_cast<int64_t>(poly) * a.poly_stride;
    const uint64_t *src = a.in + base;
    uint64_t *dst = a.out + base;
    const Tw *tw = reinterpret_cast<const Tw *>(a.tw) + static_cast<size_t>(limb) * N;

    uint32_t bad = 0;
    for (uint32_t j = threadIdx.x; j < N; j += blockDim.x)
        s[GS ? brev_bits(j, L) : j] = A::load_reduce(src[j], q, one_q, bad);
    raise_status(a.status, bad != 0, kStatusInputRange);
    __syncthreads();
    smem_stages<A, GS>(s, tw, L, scale_last != 0, lc);
    for (uint32_t j = threadIdx.x; j < N; j += blockDim.x)
        dst[j] = A::canon(s[GS ? j : brev_bits(j, L)], q);
}

// ---- multi-pass global-memory path ----

template <class A, bool GS>
__global__ void k_glb_load(KArgs a, typename A::W *scratch) {
    using W = typename A::W;
    const uint32_t L = a.logn;
    const uint64_t N = 1ull << L;
    const uint64_t total = N * a.batch * a.n_limbs;
    uint32_t bad = 0;
    for (uint64_t g = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; g < total;
         g += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint64_t j = g & (N - 1), pl = g >> L;
        const uint32_t poly = static_cast<uint32_t>(pl % a.batch);
        const uint32_t limb = static_cast<uint32_t>(pl / a.batch);
        const LimbConst &lc = a.limbs[limb];
        const uint64_t v = a.in[static_cast<int64_t>(limb) * a.limb_stride +
                                static_cast<int64_t>(poly) * a.poly_stride + static_cast<int64_t>(j)];
        const W r = A::load_reduce(v, static_cast<W>(lc.q), static_cast<W>(lc.one_shoup), bad);
        const uint64_t pos = GS ? (__brevll(j) >> (64 - L)) : j;
        scratch[(pl << L) + pos] = r;
    }
    raise_status(a.status, bad != 0, kStatusInputRange);
}

template <class A, bool GS>
__global__ void k_glb_stage(KArgs a, typename A::W *scratch, uint32_t b, int scaled) {
    using W = typename A::W;
    using Tw = typename A::Tw;
    const uint32_t L = a.logn;
    const uint64_t N = 1ull << L, half = N >> 1;
    const uint64_t total = half * a.batch * a.n_limbs;
    for (uint64_t g = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; g < total;
         g += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint64_t t = g & (half - 1), pl = g >> (L - 1);
        const uint32_t limb = static_cast<uint32_t>(pl / a.batch);
        const LimbConst lc = a.limbs[limb];
        const uint64_t i = t >> b;
        const uint64_t p0 = (i << (b + 1)) | (t & ((1ull << b) - 1)), p1 = p0 | (1ull << b);
        const Tw *tw = reinterpret_cast<const Tw *>(a.tw) + static_cast<size_t>(limb) * N;
        W *s = scratch + (pl << L);
        W x = s[p0], y = s[p1];
        butterfly<A>(GS, scaled != 0, x, y, tw[(N >> (b + 1)) + i], lc);
        s[p0] = x;
        s[p1] = y;
    }
}

template <class A, bool GS>
__global__ void k_glb_store(KArgs a, const typename A::W *scratch) {
    const uint32_t L = a.logn;
    const uint64_t N = 1ull << L;
    const uint64_t total = N * a.batch * a.n_limbs;
    for (uint64_t g = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; g < total;
         g += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint64_t j = g & (N - 1), pl = g >> L;
        const uint32_t poly = static_cast<uint32_t>(pl % a.batch);
        const uint32_t limb = static_cast<uint32_t>(pl / a.batch);
        const uint64_t pos = GS ? j : (__brevll(j) >> (64 - L));
        a.out[static_cast<int64_t>(limb) * a.limb_stride + static_cast<int64_t>(poly) * a.poly_stride +
              static_cast<int64_t>(j)] =
            A::canon(scratch[(pl << L) + pos], static_cast<typename A::W>(a.limbs[limb].q));
    }
}

// ---- elementwise ----

// One polynomial per blockIdx.y (grid-stride over polynomials), four
// coefficients a block stride apart per thread and step, loaded before any
// arithmetic (see k_coeff).
template <class A>
__global__ void k_pointwise(KArgs a) {
    using W = typename A::W;
    constexpr int kUnroll = 4;
    const uint64_t N = 1ull << a.logn;
    const uint64_t polys = static_cast<uint64_t>(a.batch) * a.n_limbs;
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    uint32_t bad = 0;
    for (uint64_t pl = blockIdx.y; pl < polys; pl += gridDim.y) {
        const uint32_t poly = static_cast<uint32_t>(pl % a.batch);
        const uint32_t limb = static_cast<uint32_t>(pl / a.batch);
        const LimbConst lc = a.limbs[limb];
        const W q = static_cast<W>(lc.q);
        const int64_t base = static_cast<int64_t>(limb) * a.limb_stride + static_cast<int64_t>(poly) * a.poly_stride;
        const uint64_t *pa = a.in + base, *pb = a.in2 + base;
        uint64_t *pc = a.out + base;
        for (uint64_t j0 = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; j0 < N;
             j0 += kUnroll * stride) {
            uint64_t va[kUnroll], vb[kUnroll];
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                if (j0 + u * stride < N) {
                    va[u] = pa[j0 + u * stride];
                    vb[u] = pb[j0 + u * stride];
                }
            }
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                if (j0 + u * stride >= N) continue;
                W r;
                if constexpr (A::kBits == 32) {
                    bad |= static_cast<uint32_t>((va[u] | vb[u]) >> 32);
                    r = A::mulmod(static_cast<W>(va[u]), static_cast<W>(vb[u]), q, lc.barrett);
                } else {
                    const W x = A::load_reduce(va[u], q, static_cast<W>(lc.one_shoup), bad);
                    const W y = A::load_reduce(vb[u], q, static_cast<W>(lc.one_shoup), bad);
                    r = A::mulmod(x, y, q, lc.barrett, lc.bk);
                }
                pc[j0 + u * stride] = r;
            }
        }
    }
    raise_status(a.status, bad != 0, kStatusInputRange);
}

__global__ void k_mul_lo32(KArgs a) {
    const uint32_t L = a.logn;
    const uint64_t N = 1ull << L;
    const uint64_t total = N * a.batch * a.n_limbs;
    uint32_t bad = 0;
    for (uint64_t g = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; g < total;
         g += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint64_t j = g & (N - 1), pl = g >> L;
        const uint32_t poly = static_cast<uint32_t>(pl % a.batch);
        const uint32_t limb = static_cast<uint32_t>(pl / a.batch);
        const int64_t off = static_cast<int64_t>(limb) * a.limb_stride +
                            static_cast<int64_t>(poly) * a.poly_stride + static_cast<int64_t>(j);
        const uint64_t va = a.in[off], vb = a.in2[off];
        bad |= static_cast<uint32_t>((va | vb) >> 32);
        a.out[off] = static_cast<uint32_t>(va) * static_cast<uint32_t>(vb);
    }
    raise_status(a.status, bad != 0, kStatusInputRange);
}

template <class A>
__global__ void k_scale(KArgs a) {
    using W = typename A::W;
    const uint32_t L = a.logn;
    const uint64_t N = 1ull << L;
    const uint64_t total = N * a.batch * a.n_limbs;
    uint32_t bad = 0;
    for (uint64_t g = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; g < total;
         g += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint64_t j = g & (N - 1), pl = g >> L;
        const uint32_t poly = static_cast<uint32_t>(pl % a.batch);
        const uint32_t limb = static_cast<uint32_t>(pl / a.batch);
        const LimbConst lc = a.limbs[limb];
        const int64_t off = static_cast<int64_t>(limb) * a.limb_stride +
                            static_cast<int64_t>(poly) * a.poly_stride + static_cast<int64_t>(j);
        const W q = static_cast<W>(lc.q);
        const W x = A::load_reduce(a.in[off], q, static_cast<W>(lc.one_shoup), bad);
        a.out[off] = A::canon(A::mul_shoup(x, static_cast<W>(lc.ninv), static_cast<W>(lc.ninv_shoup), q), q);
    }
    raise_status(a.status, bad != 0, kStatusInputRange);
}

// ---- fused polymul in shared memory ----

template <class A, bool CYCLIC>
__global__ void __launch_bounds__(512) k_polymul_smem(KArgs a) {
    using W = typename A::W;
    using Tw = typename A::Tw;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const uint32_t L = a.logn, N = 1u << L;
    W *sa = reinterpret_cast<W *>(smem_raw);
    W *sb = sa + N;
    const uint32_t limb = blockIdx.y, poly = blockIdx.x;
    const LimbConst lc = a.limbs[limb];
    const W q = static_cast<W>(lc.q), one_q = static_cast<W>(lc.one_shoup);
    const int64_t base = static_cast<int64_t>(limb) * a.limb_stride +
                         static_cast<int64_t>(poly) * a.poly_stride;
    const Tw *twf = reinterpret_cast<const Tw *>(a.tw) + static_cast<size_t>(limb) * N;
    const Tw *twi = reinterpret_cast<const Tw *>(a.tw2) + static_cast<size_t>(limb) * N;

    uint32_t bad = 0;
    for (uint32_t j = threadIdx.x; j < N; j += blockDim.x) {
        sa[j] = A::load_reduce(a.in[base + j], q, one_q, bad);
        sb[j] = A::load_reduce(a.in2[base + j], q, one_q, bad);
    }
    raise_status(a.status, bad != 0, kStatusInputRange);
    __syncthreads();
    smem_stages<A, false>(sa, twf, L, false, lc);
    smem_stages<A, false>(sb, twf, L, false, lc);
    // product in bit-reversed order; cyclic mode also undoes the order
    for (uint32_t p = threadIdx.x; p < N; p += blockDim.x) {
        W r;
        if constexpr (A::kBits == 32)
            r = A::mulmod(sa[p], sb[p], q, lc.barrett);
        else
            r = A::mulmod(sa[p], sb[p], q, lc.barrett, lc.bk);
        sa[p] = r;
    }
    __syncthreads();
    W *sc = sa;
    if (CYCLIC) {
        for (uint32_t j = threadIdx.x; j < N; j += blockDim.x) sb[j] = sa[brev_bits(j, L)];
        __syncthreads();
        sc = sb;
        smem_stages<A, false>(sc, twi, L, true, lc);
        for (uint32_t j = threadIdx.x; j < N; j += blockDim.x)
            a.out[base + j] = A::canon(sc[brev_bits(j, L)], q);
    } else {
        smem_stages<A, true>(sc, twi, L, true, lc);
        for (uint32_t j = threadIdx.x; j < N; j += blockDim.x) a.out[base + j] = A::canon(sc[j], q);
    }
}

// ---- coefficient-wise ops ----
// Semantics (crates/barracuda/src/ops/, for any u64 inputs):
//   add: the wrapping 64-bit sum minus q at most twice (fhe_poly_add.wgsl
//        u64_add + mod_reduce), which is (a + b) mod q for a, b < q;
//   sub: a - b if a >= b, else (q - b) + a, wrapping (fhe_poly_sub.wgsl
//        modular_sub), which is (a - b) mod q for a, b < q;
//   mul: exact (a * b) mod q.  The reference's fhe_poly_mul.wgsl is exact
//        only while its product stays below 1001 q (a bounded subtraction
//        loop) and its 32x32 helper does not overflow; outside that range
//        this path keeps the exact residue.

// x mod q for any u64 x: the estimate floor(x m / 2^64) is at most two
// below floor(x / q).
__device__ __forceinline__ uint64_t reduce_any(uint64_t x, const CoeffConst &c) {
    uint64_t r = x - __umul64hi(x, c.m) * c.q;
    if (r >= c.q) r -= c.q;
    if (r >= c.q) r -= c.q;
    return r;
}

__device__ __forceinline__ uint64_t mulmod_any(uint64_t a, uint64_t b, const CoeffConst &c) {
    if (a < c.q && b < c.q) {  // operands already reduced (the usual case): no pre-reduction
        if (c.q <= 0xFFFFFFFFull) return reduce_any(a * b, c);
        if (c.k <= 62) return Arith64::mulmod_reduced(a, b, c.q, c.mu, c.k);
    }
    const uint64_t x = reduce_any(a, c), y = reduce_any(b, c);
    if (c.q <= 0xFFFFFFFFull) return reduce_any(x * y, c);  // x * y < 2^64
    if (c.k <= 62) return Arith64::mulmod(x, y, c.q, c.mu, c.k);
    const unsigned __int128 p = static_cast<unsigned __int128>(x) * y;  // q >= 2^62: rare
    return static_cast<uint64_t>(p % c.q);
}

// kCoeffAddExact / kCoeffSubExact: (x mod q +- y mod q) mod q for any u64;
// with `flag_wide`, a word >= 2^32 raises kStatusInputRange as the 32-bit
// transforms do for their inputs.
template <int OP>
__device__ __forceinline__ uint64_t coeff_op(uint64_t x, uint64_t y, const CoeffConst &c, int flag_wide,
                                             uint32_t *status) {
    uint64_t r;
    if constexpr (OP == kCoeffAddExact || OP == kCoeffSubExact) {
        if (flag_wide && ((x | y) >> 32) != 0) store_status(status, kStatusInputRange);
        const uint64_t xr = reduce_any(x, c), yr = reduce_any(y, c);
        if constexpr (OP == kCoeffAddExact) {
            r = xr + yr;  // q < 2^62: no overflow
            if (r >= c.q) r -= c.q;
        } else {
            r = xr >= yr ? xr - yr : xr + (c.q - yr);
        }
    } else if constexpr (OP == kCoeffAdd) {
        r = x + y;
        if (r >= c.q) r -= c.q;
        if (r >= c.q) r -= c.q;
    } else if constexpr (OP == kCoeffSub) {
        r = x >= y ? x - y : (c.q - y) + x;
    } else {
        r = mulmod_any(x, y, c);
    }
    return r;
}

// One polynomial per blockIdx.y (grid-stride over polynomials), elements
// over blockIdx.x / threads.  Each thread takes kUnroll elements a block
// stride apart per step and issues all their loads before any arithmetic:
// with one element per step, mul's long dependency chain left one load pair
// in flight per thread (measured on B200: 0.71-0.76 of HBM for mul).
template <int OP>
__global__ void k_coeff(KArgs a, uint64_t n, const CoeffConst *consts, CoeffConst single, int flag_wide) {
    constexpr int kUnroll = 4;
    const uint64_t polys = static_cast<uint64_t>(a.batch) * a.n_limbs;
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    for (uint64_t pl = blockIdx.y; pl < polys; pl += gridDim.y) {
        const uint64_t limb = pl / a.batch, poly = pl % a.batch;
        const CoeffConst c = consts ? consts[limb] : single;
        const int64_t base = static_cast<int64_t>(limb) * a.limb_stride + static_cast<int64_t>(poly) * a.poly_stride;
        const uint64_t *pa = a.in + base, *pb = a.in2 + base;
        uint64_t *pc = a.out + base;
        for (uint64_t j0 = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; j0 < n;
             j0 += kUnroll * stride) {
            uint64_t x[kUnroll], y[kUnroll];
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                const uint64_t j = j0 + u * stride;
                if (j < n) {
                    x[u] = __ldcs(pa + j);
                    y[u] = __ldcs(pb + j);
                }
            }
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                const uint64_t j = j0 + u * stride;
                if (j < n) __stcs(pc + j, coeff_op<OP>(x[u], y[u], c, flag_wide, a.status));
            }
        }
    }
}

// ---- synthetic inputs and digests ----

__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__global__ void k_fill_uniform(KArgs a, uint64_t seed, uint64_t first_poly, uint64_t total_polys) {
    const uint32_t L = a.logn;
    const uint64_t N = 1ull << L;
    const uint64_t total = N * a.batch * a.n_limbs;
    for (uint64_t g = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; g < total;
         g += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint64_t j = g & (N - 1), pl = g >> L;
        const uint32_t poly = static_cast<uint32_t>(pl % a.batch);
        const uint32_t limb = static_cast<uint32_t>(pl / a.batch);
        const uint64_t gi = ((limb * total_polys + first_poly + poly) << L) + j;
        const uint64_t z = splitmix64(seed + (gi + 1) * 0x9E3779B97F4A7C15ull);
        a.out[static_cast<int64_t>(limb) * a.limb_stride + static_cast<int64_t>(poly) * a.poly_stride +
              static_cast<int64_t>(j)] = __umul64hi(z, a.limbs[limb].q);
    }
}

__global__ void k_digest(const uint64_t *in, size_t count, uint64_t first, uint64_t *out) {
    uint64_t acc = 0;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        acc += splitmix64(in[i] ^ ((first + i) * 0xD1B54A32D192ED03ull));
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) atomicAdd(reinterpret_cast<unsigned long long *>(out), acc);
}

// ---- dispatch helpers ----

template <template <class> class F, class... Args>
int dispatch_word(Word w, Args &&...args) {
    switch (w) {
    case Word::W32Lazy4: return F<Arith32<true>>::run(args...);
    case Word::W32Lazy2: return F<Arith32<false>>::run(args...);
    default: return F<Arith64>::run(args...);
    }
}

size_t word_bytes(Word w) { return w == Word::W64 ? 8 : 4; }

int check_launch(const char *what) {
    const cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) return BC_OK;
    return fail(e == cudaErrorMemoryAllocation ? BC_ERR_OUT_OF_MEMORY : BC_ERR_GPU,
                format("%s launch failed: %s", what, cudaGetErrorString(e)));
}

unsigned grid_for(uint64_t work, unsigned threads) {
    uint64_t blocks = (work + threads - 1) / threads;
    const uint64_t cap = 148ull * 16;  // grid-stride beyond 16 CTAs per SM
    if (blocks > cap) blocks = cap;
    return static_cast<unsigned>(blocks ? blocks : 1);
}

template <class A>
struct SmemRun {
    static int run(bool gs, bool scale_last, const KArgs &a, cudaStream_t s) {
        const uint32_t N = 1u << a.logn;
        const size_t bytes = sizeof(typename A::W) * N;
        const unsigned threads = N / 2 < 512 ? (N / 2 < 32 ? 32 : N / 2) : 512;
        const dim3 grid(a.batch, a.n_limbs);
        auto kern = gs ? k_ntt_smem<A, true> : k_ntt_smem<A, false>;
        if (bytes > 48 * 1024)
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
        kern<<<grid, threads, bytes, s>>>(a, scale_last ? 1 : 0);
        return check_launch("k_ntt_smem");
    }
};

template <class A>
struct GlobalRun {
    static int run(bool gs, bool scale_last, const KArgs &a, void *scratch, cudaStream_t s) {
        using W = typename A::W;
        W *sc = static_cast<W *>(scratch);
        const uint64_t N = 1ull << a.logn;
        const uint64_t total = N * a.batch * a.n_limbs;
        const unsigned T = 256;
        if (gs)
            k_glb_load<A, true><<<grid_for(total, T), T, 0, s>>>(a, sc);
        else
            k_glb_load<A, false><<<grid_for(total, T), T, 0, s>>>(a, sc);
        for (uint32_t st = 0; st < a.logn; ++st) {
            const uint32_t b = gs ? st : a.logn - 1 - st;
            const int scaled = (scale_last && st == a.logn - 1) ? 1 : 0;
            if (gs)
                k_glb_stage<A, true><<<grid_for(total / 2, T), T, 0, s>>>(a, sc, b, scaled);
            else
                k_glb_stage<A, false><<<grid_for(total / 2, T), T, 0, s>>>(a, sc, b, scaled);
        }
        if (gs)
            k_glb_store<A, true><<<grid_for(total, T), T, 0, s>>>(a, sc);
        else
            k_glb_store<A, false><<<grid_for(total, T), T, 0, s>>>(a, sc);
        return check_launch("k_glb");
    }
};

template <class A>
struct PointwiseRun {
    static int run(const KArgs &a, cudaStream_t s) {
        const uint64_t N = 1ull << a.logn, polys = static_cast<uint64_t>(a.batch) * a.n_limbs;
        // four coefficients per thread and step; small N: smaller blocks
        const unsigned T = N >= 1024 ? 256u : static_cast<unsigned>(((N / 4 + 31) / 32) * 32);
        uint64_t bx = (N + 4 * T - 1) / (4 * T);
        if (bx > 64) bx = 64;
        const dim3 grid(static_cast<unsigned>(bx), static_cast<unsigned>(polys < 65535 ? polys : 65535));
        k_pointwise<A><<<grid, T, 0, s>>>(a);
        return check_launch("k_pointwise");
    }
};

template <class A>
struct ScaleRun {
    static int run(const KArgs &a, cudaStream_t s) {
        const uint64_t total = (1ull << a.logn) * a.batch * a.n_limbs;
        k_scale<A><<<grid_for(total, 256), 256, 0, s>>>(a);
        return check_launch("k_scale");
    }
};

template <class A>
struct PolymulRun {
    static int run(bool cyclic, const KArgs &a, cudaStream_t s) {
        const uint32_t N = 1u << a.logn;
        const size_t bytes = 2 * sizeof(typename A::W) * N;
        const unsigned threads = N / 2 < 512 ? (N / 2 < 32 ? 32 : N / 2) : 512;
        const dim3 grid(a.batch, a.n_limbs);
        auto kern = cyclic ? k_polymul_smem<A, true> : k_polymul_smem<A, false>;
        if (bytes > 48 * 1024)
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
        kern<<<grid, threads, bytes, s>>>(a);
        return check_launch("k_polymul_smem");
    }
};

}  // namespace

constexpr size_t kSmemLimit = 200 * 1024;

uint32_t smem_max_logn(Word w) {
    uint32_t l = 1;
    while ((word_bytes(w) << (l + 1)) <= kSmemLimit && l < 16) ++l;
    return l;
}

uint32_t polymul_smem_max_logn(Word w) {
    uint32_t l = 1;
    while ((2 * word_bytes(w) << (l + 1)) <= kSmemLimit && l < 16) ++l;
    return l;
}

int launch_ntt_smem(Word w, bool gs, bool scale_last, const KArgs &a, cudaStream_t s) {
    return dispatch_word<SmemRun>(w, gs, scale_last, a, s);
}

int launch_ntt_global(Word w, bool gs, bool scale_last, const KArgs &a, void *scratch,
                      cudaStream_t s) {
    return dispatch_word<GlobalRun>(w, gs, scale_last, a, scratch, s);
}

int launch_pointwise(Word w, const KArgs &a, cudaStream_t s) { return dispatch_word<PointwiseRun>(w, a, s); }

int launch_scale(Word w, const KArgs &a, cudaStream_t s) { return dispatch_word<ScaleRun>(w, a, s); }

int launch_mul_lo32(const KArgs &a, cudaStream_t s) {
    const uint64_t total = (1ull << a.logn) * a.batch * a.n_limbs;
    k_mul_lo32<<<grid_for(total, 256), 256, 0, s>>>(a);
    return check_launch("k_mul_lo32");
}

int launch_polymul_smem(Word w, bool cyclic, const KArgs &a, cudaStream_t s) {
    return dispatch_word<PolymulRun>(w, cyclic, a, s);
}

int launch_fill_uniform(const KArgs &a, uint64_t seed, uint64_t first_poly, uint64_t total_polys,
                        cudaStream_t s) {
    const uint64_t total = (1ull << a.logn) * a.batch * a.n_limbs;
    k_fill_uniform<<<grid_for(total, 256), 256, 0, s>>>(a, seed, first_poly, total_polys);
    return check_launch("k_fill_uniform");
}

CoeffConst coeff_const(uint64_t q) {
    CoeffConst c = {};
    c.q = q;
    c.m = ~0ull / q;
    c.k = 64 - static_cast<uint32_t>(__builtin_clzll(q));
    if (c.k > 32 && c.k <= 62)
        c.mu = static_cast<uint64_t>((static_cast<unsigned __int128>(1) << (2 * c.k)) / q);
    return c;
}

int launch_coeff_op(int op, const KArgs &a, uint64_t n, const CoeffConst *consts,
                    const CoeffConst &single, cudaStream_t s, bool flag_wide_words) {
    const uint64_t polys = static_cast<uint64_t>(a.batch) * a.n_limbs;
    if (n == 0 || polys == 0) return BC_OK;
    const unsigned T = 256;
    uint64_t bx = (n + 4 * T - 1) / (4 * T);  // four elements per thread and step (k_coeff)
    if (bx > 64) bx = 64;
    const dim3 grid(static_cast<unsigned>(bx), static_cast<unsigned>(polys < 65535 ? polys : 65535));
    switch (op) {
    case kCoeffAdd: k_coeff<kCoeffAdd><<<grid, T, 0, s>>>(a, n, consts, single, 0); break;
    case kCoeffSub: k_coeff<kCoeffSub><<<grid, T, 0, s>>>(a, n, consts, single, 0); break;
    case kCoeffMul: k_coeff<kCoeffMul><<<grid, T, 0, s>>>(a, n, consts, single, 0); break;
    case kCoeffAddExact: k_coeff<kCoeffAddExact><<<grid, T, 0, s>>>(a, n, consts, single, flag_wide_words); break;
    case kCoeffSubExact: k_coeff<kCoeffSubExact><<<grid, T, 0, s>>>(a, n, consts, single, flag_wide_words); break;
    default: return fail(BC_ERR_INTERNAL, "unknown coefficient op");
    }
    return check_launch("k_coeff");
}

int launch_digest(const uint64_t *in, size_t count, uint64_t first, uint64_t *out, cudaStream_t s) {
    cudaMemsetAsync(out, 0, sizeof(uint64_t), s);
    k_digest<<<grid_for(count, 256), 256, 0, s>>>(in, count, first, out);
    return check_launch("k_digest");
}

}  // namespace bc
