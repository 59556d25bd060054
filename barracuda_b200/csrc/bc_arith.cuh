// bc_arith.cuh -- device modular arithmetic for the NTT kernels.
//
// Two word sizes, chosen per plan from the largest modulus:
//   Arith32<LAZY4>: q < 2^31, u32 words.  Twiddle products use Shoup's
//     precomputed quotient (w' = floor(w * 2^32 / q)): one mul.hi and two
//     mul.lo.  Values between butterflies are kept lazily reduced: in
//     [0, 2q) for q < 2^31 (LAZY4 = false), in [0, 4q) for q < 2^30
//     (LAZY4 = true, Harvey's butterfly, one compare-subtract fewer).
//   Arith64: q < 2^62, u64 words, Harvey's lazy [0, 4q) butterflies with
//     w' = floor(w * 2^64 / q) and __umul64hi.
// All results are exact residues once canonicalised with `canon`.
#pragma once

#include <cstdint>

namespace bc {

// Per-limb constants, copied to the device once per plan.
struct LimbConst {
    uint64_t q;           // modulus
    uint64_t one_shoup;   // floor(2^W / q), W = word bits: Shoup quotient of w = 1
    uint64_t ninv;        // N^-1 mod q (0 when not invertible, as the reference)
    uint64_t ninv_shoup;  // Shoup quotient of ninv
    uint64_t barrett;     // 32-bit words: floor(2^64 / q); 64-bit words: floor(2^(2k) / q)
    uint32_t bk;          // 64-bit words: k = bit length of q
    uint32_t pad;
};

__device__ __forceinline__ uint32_t umin32(uint32_t a, uint32_t b) { return a < b ? a : b; }
__device__ __forceinline__ uint64_t umin64(uint64_t a, uint64_t b) { return a < b ? a : b; }

template <bool LAZY4>
struct Arith32 {
    using W = uint32_t;
    using Tw = uint2;  // {w, w'}
    static constexpr int kBits = 32;
    static constexpr bool kLazy4 = LAZY4;

    __device__ __forceinline__ static W mul_shoup(W x, W w, W wq, W q) {
        // x * w - floor(x * wq / 2^32) * q, in [0, 2q) for any x < 2^32.
        const W hi = __umulhi(x, wq);
        return x * w - hi * q;
    }
    __device__ __forceinline__ static W sub_if(W x, W m) { return umin32(x, x - m); }

    // Input coefficient -> lazy residue in [0, 2q).  Words with a non-zero
    // high half are outside the reference's exact domain; they set `bad`.
    __device__ __forceinline__ static W load_reduce(uint64_t v, W q, W one_shoup, uint32_t &bad) {
        bad |= static_cast<uint32_t>(v >> 32);
        return mul_shoup(static_cast<W>(v), 1u, one_shoup, q);
    }
    __device__ __forceinline__ static uint64_t canon(W x, W q) {
        if (LAZY4) x = sub_if(x, 2 * q);
        return sub_if(x, q);
    }

    // Cooley-Tukey: (X, Y) -> (X + wY, X - wY).
    __device__ __forceinline__ static void ct(W &x, W &y, W w, W wq, W q) {
        if (LAZY4) {  // in/out [0, 4q)
            x = sub_if(x, 2 * q);
            const W t = mul_shoup(y, w, wq, q);
            y = x - t + 2 * q;
            x = x + t;
        } else {  // in/out [0, 2q)
            x = sub_if(x, q);
            const W t = sub_if(mul_shoup(y, w, wq, q), q);
            y = x - t + q;
            x = x + t;
        }
    }
    // Cooley-Tukey with both outputs scaled by s (and w pre-scaled by s):
    // (X, Y) -> (sX + (sw)Y, sX - (sw)Y).
    __device__ __forceinline__ static void ct_scaled(W &x, W &y, W sw, W swq, W s, W sq, W q) {
        W a = mul_shoup(x, s, sq, q);  // [0, 2q)
        if (LAZY4) {
            const W t = mul_shoup(y, sw, swq, q);
            y = a - t + 2 * q;
            x = a + t;
        } else {
            a = sub_if(a, q);
            const W t = sub_if(mul_shoup(y, sw, swq, q), q);
            y = a - t + q;
            x = a + t;
        }
    }
    // Gentleman-Sande: (X, Y) -> (X + Y, (X - Y) w).  in/out [0, 2q).
    __device__ __forceinline__ static void gs(W &x, W &y, W w, W wq, W q) {
        if (LAZY4) {
            const W s = x + y;
            const W d = x - y + 2 * q;
            x = sub_if(s, 2 * q);
            y = mul_shoup(d, w, wq, q);
        } else {
            const W a = sub_if(x, q), b = sub_if(y, q);
            x = a + b;
            y = mul_shoup(a - b + q, w, wq, q);
        }
    }
    // Gentleman-Sande with the sum scaled by s: (X, Y) -> ((X + Y)s, (X - Y)(sw)).
    __device__ __forceinline__ static void gs_scaled(W &x, W &y, W sw, W swq, W s, W sq, W q) {
        if (LAZY4) {
            const W sum = sub_if(x + y, 2 * q);
            const W d = x - y + 2 * q;
            x = mul_shoup(sum, s, sq, q);
            y = mul_shoup(d, sw, swq, q);
        } else {
            const W a = sub_if(x, q), b = sub_if(y, q);
            x = mul_shoup(a + b, s, sq, q);
            y = mul_shoup(a - b + q, sw, swq, q);
        }
    }
    // General product of two words (< 2^32): exact a*b mod q in [0, q).
    // Barrett quotient qt = floor(t * m / 2^64) with m = floor(2^64 / q)
    // (2^64 - 1 for q = 1) is floor(t / q) or one less, so t - qt*q < 2q
    // fits the 32-bit word and one compare-subtract finishes the job.
    __device__ __forceinline__ static W mulmod(W a, W b, W q, uint64_t barrett) {
        const uint64_t t = static_cast<uint64_t>(a) * b;
        const uint64_t qt = __umul64hi(t, barrett);
        const W r = static_cast<W>(t) - static_cast<W>(qt) * q;
        return sub_if(r, q);
    }
};

struct Arith64 {
    using W = uint64_t;
    using Tw = ulonglong2;  // {w, w'}
    static constexpr int kBits = 64;
    static constexpr bool kLazy4 = true;

    __device__ __forceinline__ static W mul_shoup(W x, W w, W wq, W q) {
        const W hi = __umul64hi(x, wq);
        return x * w - hi * q;  // [0, 2q) for any x < 2^64
    }
    __device__ __forceinline__ static W sub_if(W x, W m) { return umin64(x, x - m); }
    __device__ __forceinline__ static W load_reduce(uint64_t v, W q, W one_shoup, uint32_t &) {
        return mul_shoup(v, 1u, one_shoup, q);
    }
    __device__ __forceinline__ static uint64_t canon(W x, W q) { return sub_if(sub_if(x, 2 * q), q); }

    __device__ __forceinline__ static void ct(W &x, W &y, W w, W wq, W q) {
        x = sub_if(x, 2 * q);
        const W t = mul_shoup(y, w, wq, q);
        y = x - t + 2 * q;
        x = x + t;
    }
    __device__ __forceinline__ static void ct_scaled(W &x, W &y, W sw, W swq, W s, W sq, W q) {
        const W a = mul_shoup(x, s, sq, q);
        const W t = mul_shoup(y, sw, swq, q);
        y = a - t + 2 * q;
        x = a + t;
    }
    __device__ __forceinline__ static void gs(W &x, W &y, W w, W wq, W q) {
        const W s = x + y;
        const W d = x - y + 2 * q;
        x = sub_if(s, 2 * q);
        y = mul_shoup(d, w, wq, q);
    }
    __device__ __forceinline__ static void gs_scaled(W &x, W &y, W sw, W swq, W s, W sq, W q) {
        const W sum = sub_if(x + y, 2 * q);
        const W d = x - y + 2 * q;
        x = mul_shoup(sum, s, sq, q);
        y = mul_shoup(d, sw, swq, q);
    }
    // Exact a*b mod q for a, b < 4q (q < 2^62, k = bit length of q):
    // Barrett with mu = floor(2^(2k) / q); quotient estimate within 2.
    __device__ __forceinline__ static W mulmod(W a, W b, W q, uint64_t mu, uint32_t k) {
        return mulmod_reduced(sub_if(sub_if(a, 2 * q), q), sub_if(sub_if(b, 2 * q), q), q, mu, k);
    }
    // The same for a, b < q.
    __device__ __forceinline__ static W mulmod_reduced(W a, W b, W q, uint64_t mu, uint32_t k) {
        const uint64_t lo = a * b, hi = __umul64hi(a, b);
        // t1 = floor(t / 2^(k-1)) fits in k+1 <= 63 bits
        const uint64_t t1 = (hi << (65 - k)) | (lo >> (k - 1));
        const uint64_t plo = t1 * mu, phi = __umul64hi(t1, mu);
        const uint64_t qt = (phi << (63 - k)) | (plo >> (k + 1));
        W r = lo - qt * q;  // true r in [0, 3q)
        r = sub_if(r, 2 * q);
        return sub_if(r, q);
    }
};

}  // namespace bc
