/* ref_poly.c -- CPU restatement of the reference's coefficient-wise FHE ops
 * (FhePolyAdd, FhePolySub, FhePolyMul).  TEST INFRASTRUCTURE ONLY: see
 * oracle.h.
 *
 * The reference computes in u32 pairs; where that emulation is a plain
 * 64-bit operation (carry into the high word, wrap-around) it is written
 * here with uint64_t.  Where the shader's arithmetic departs from exact
 * 64-bit math (FhePolyMul's 32x32 product helper and its bounded
 * reduction) the departure is restated step by step, so the tests can pin
 * both where the reference is exact and where it is not.  Paths are inside
 * crates/barracuda/src/ops/. */
#include <stdint.h>

#include "oracle.h"

/* fhe_poly_add.wgsl:106-155: wrapping 64-bit sum (u64_add drops the carry
 * out of the high word), then at most two conditional subtractions of q
 * (mod_reduce, :104-118). */
uint64_t orc_ref_poly_add1(uint64_t a, uint64_t b, uint64_t q) {
    uint64_t s = a + b;
    if (s >= q) s -= q;
    if (s >= q) s -= q;
    return s;
}

/* fhe_poly_sub.wgsl:64-74 modular_sub: a - b when a >= b, otherwise
 * (q - b) + a, both with 64-bit wrap-around. */
uint64_t orc_ref_poly_sub1(uint64_t a, uint64_t b, uint64_t q) {
    if (a >= b) return a - b;
    return (q - b) + a;
}

/* fhe_poly_mul.wgsl u32_mul_to_u64: 32x32 product from 16-bit halves where
 * the middle sum p_lh + p_hl + (p_ll >> 16) is kept in 32 bits, so it loses
 * 2^32 when it overflows (the high word then misses 2^16). */
static void mul32_by_halves(uint32_t a, uint32_t b, uint32_t *lo, uint32_t *hi) {
    const uint32_t a0 = a & 0xFFFFu, a1 = a >> 16, b0 = b & 0xFFFFu, b1 = b >> 16;
    const uint32_t p_ll = a0 * b0, p_lh = a0 * b1, p_hl = a1 * b0, p_hh = a1 * b1;
    const uint32_t mid = p_lh + p_hl + (p_ll >> 16); /* wraps in 32 bits */
    *lo = (mid << 16) | (p_ll & 0xFFFFu);
    *hi = p_hh + (mid >> 16);
}

/* fhe_poly_mul.wgsl u64_mul: the 128-bit product assembled from four
 * mul32_by_halves partial products with exact carries between them.
 * Result as four 32-bit words, least significant first. */
static void mul64_wide(uint64_t a, uint64_t b, uint32_t w[4]) {
    uint32_t p0l, p0h, p1l, p1h, p2l, p2h, p3l, p3h;
    mul32_by_halves((uint32_t)a, (uint32_t)b, &p0l, &p0h);
    mul32_by_halves((uint32_t)a, (uint32_t)(b >> 32), &p1l, &p1h);
    mul32_by_halves((uint32_t)(a >> 32), (uint32_t)b, &p2l, &p2h);
    mul32_by_halves((uint32_t)(a >> 32), (uint32_t)(b >> 32), &p3l, &p3h);
    const uint64_t mid = (uint64_t)p0h + p1l + p2l;  /* < 2^34, exact */
    const uint64_t hi = (uint64_t)p1h + p2h + (mid >> 32) + (((uint64_t)p3h << 32) | p3l);
    w[0] = p0l;
    w[1] = (uint32_t)mid;
    w[2] = (uint32_t)hi;
    w[3] = (uint32_t)(hi >> 32);
}

/* fhe_poly_mul.wgsl modular_mul with mu = u64::MAX / q (fhe_poly_mul.rs:65):
 *   - product below 2^64: subtract q while the value is >= q, at most 1000
 *     times (simple_mod_reduce), so values >= 1001 q stay unreduced;
 *   - otherwise barrett_reduce_128: quotient estimate = high 64 bits of
 *     (product >> 64) * mu, remainder = low 64 bits of the product minus the
 *     low 64 bits of q * estimate when that does not underflow (else the
 *     low 64 bits unchanged), then at most two subtractions of q. */
uint64_t orc_ref_poly_mul1(uint64_t a, uint64_t b, uint64_t q) {
    uint32_t p[4];
    mul64_wide(a, b, p);
    const uint64_t lo = ((uint64_t)p[1] << 32) | p[0], hi = ((uint64_t)p[3] << 32) | p[2];
    uint64_t r;
    if (hi == 0) {
        r = lo;
        for (int i = 0; i < 1000 && r >= q; ++i) r -= q;
        return r;
    }
    const uint64_t mu = UINT64_MAX / q;
    uint32_t e[4], f[4];
    mul64_wide(hi, mu, e);
    const uint64_t est = ((uint64_t)e[3] << 32) | e[2];
    mul64_wide(q, est, f);
    const uint64_t qe = ((uint64_t)f[1] << 32) | f[0];
    r = lo >= qe ? lo - qe : lo;
    if (r >= q) r -= q;
    if (r >= q) r -= q;
    return r;
}

void orc_ref_poly_add(const uint64_t *a, const uint64_t *b, uint64_t *c, uint32_t degree, uint64_t q) {
    for (uint32_t i = 0; i < degree; ++i) c[i] = orc_ref_poly_add1(a[i], b[i], q);
}

void orc_ref_poly_sub(const uint64_t *a, const uint64_t *b, uint64_t *c, uint32_t degree, uint64_t q) {
    for (uint32_t i = 0; i < degree; ++i) c[i] = orc_ref_poly_sub1(a[i], b[i], q);
}

void orc_ref_poly_mul(const uint64_t *a, const uint64_t *b, uint64_t *c, uint32_t degree, uint64_t q) {
    for (uint32_t i = 0; i < degree; ++i) c[i] = orc_ref_poly_mul1(a[i], b[i], q);
}

/* Exact coefficient-wise product (a * b) mod q for any u64 inputs. */
void orc_exact_poly_mul(const uint64_t *a, const uint64_t *b, uint64_t *c, uint32_t degree, uint64_t q) {
    for (uint32_t i = 0; i < degree; ++i)
        c[i] = (uint64_t)(((unsigned __int128)a[i] * b[i]) % q);
}
