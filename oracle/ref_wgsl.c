/*
 * ref_wgsl.c -- restatement of the reference's FHE NTT / INTT / pointwise
 * arithmetic, written in C from the WGSL and Rust sources.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h).
 *
 * The WGSL has no native u64: every 64-bit value is a {lo, hi} pair of u32
 * and all arithmetic is u32 with wrap-around.  This file keeps that model
 * (struct w64 below) so that every overflow the shader can have, this code
 * has too.  Shader sources: crates/barracuda/src/ops/fhe_ntt.wgsl,
 * fhe_intt.wgsl (lines 1-200 identical to fhe_ntt.wgsl apart from comments)
 * and fhe_pointwise_mul.wgsl.
 */
#include "oracle.h"

#include <stdlib.h>
#include <string.h>

typedef struct {
    uint32_t lo, hi;
} w64;

static w64 w64_of(uint64_t v) {
    w64 r = {(uint32_t)v, (uint32_t)(v >> 32)};
    return r;
}
static uint64_t w64_val(w64 v) { return ((uint64_t)v.hi << 32) | v.lo; }

/* fhe_ntt.wgsl:31-36 */
static w64 w_add(w64 a, w64 b) {
    w64 r;
    r.lo = a.lo + b.lo;
    uint32_t carry = (r.lo < a.lo) ? 1u : 0u;
    r.hi = a.hi + b.hi + carry;
    return r;
}

/* fhe_ntt.wgsl:38-43 */
static w64 w_sub(w64 a, w64 b) {
    w64 r;
    r.lo = a.lo - b.lo;
    uint32_t borrow = (a.lo < b.lo) ? 1u : 0u;
    r.hi = a.hi - b.hi - borrow;
    return r;
}

/* fhe_ntt.wgsl:45-70: the full lo*lo product from 16-bit halves, plus the
 * two cross terms into the high word; the hi*hi term is dropped, so the
 * result is the product modulo 2^64. */
static w64 w_mul(w64 a, w64 b) {
    uint32_t al0 = a.lo & 0xFFFFu, al1 = a.lo >> 16;
    uint32_t bl0 = b.lo & 0xFFFFu, bl1 = b.lo >> 16;
    uint32_t p00 = al0 * bl0, p01 = al0 * bl1, p10 = al1 * bl0, p11 = al1 * bl1;
    uint32_t mid = (p00 >> 16) + (p01 & 0xFFFFu) + (p10 & 0xFFFFu);
    w64 r;
    r.lo = (p00 & 0xFFFFu) | ((mid & 0xFFFFu) << 16);
    uint32_t hi = p11 + (p01 >> 16) + (p10 >> 16) + (mid >> 16);
    uint32_t cross = a.hi * b.lo + a.lo * b.hi;
    r.hi = hi + cross;
    return r;
}

/* fhe_ntt.wgsl:78-82 */
static int w_ge(w64 a, w64 b) {
    if (a.hi != b.hi) return a.hi > b.hi;
    return a.lo >= b.lo;
}

/* fhe_ntt.wgsl:84-110.  For m < 2^32 the value is consumed MSB first with a
 * u32 accumulator; `acc << 1` wraps once m >= 2^31.  For wider m the value
 * is reduced by at most 128 subtractions and may be left >= m. */
static w64 w_mod_simple(w64 a, w64 m) {
    if (m.hi == 0u) {
        uint32_t acc = 0u;
        for (int i = 31; i >= 0; --i) {
            acc = (acc << 1) | ((a.hi >> i) & 1u);
            if (acc >= m.lo) acc -= m.lo;
        }
        for (int i = 31; i >= 0; --i) {
            acc = (acc << 1) | ((a.lo >> i) & 1u);
            if (acc >= m.lo) acc -= m.lo;
        }
        w64 r = {acc, 0u};
        return r;
    }
    w64 r = a;
    for (int i = 0; i < 128; ++i) {
        if (w_ge(r, m))
            r = w_sub(r, m);
        else
            break;
    }
    return r;
}

uint64_t orc_wgsl_u64_mul(uint64_t a, uint64_t b) { return w64_val(w_mul(w64_of(a), w64_of(b))); }

uint64_t orc_wgsl_u64_mod_simple(uint64_t a, uint64_t m) {
    return w64_val(w_mod_simple(w64_of(a), w64_of(m)));
}

/* fhe_ntt.wgsl:152-172 */
static w64 w_mod_mul(w64 a, w64 b, w64 q) { return w_mod_simple(w_mul(a, b), q); }
static w64 w_mod_add(w64 a, w64 b, w64 q) { return w_mod_simple(w_add(a, b), q); }
static w64 w_mod_sub(w64 a, w64 b, w64 q) {
    if (w_ge(a, b)) return w_sub(a, b);
    return w_sub(w_add(a, q), b);
}

/* fhe_ntt.wgsl:201-209 */
static uint32_t bitrev_idx(uint32_t idx, uint32_t log_n) {
    uint32_t r = 0;
    for (uint32_t i = 0; i < log_n; ++i) {
        r = (r << 1) | (idx & 1u);
        idx >>= 1;
    }
    return r;
}

static uint32_t log2_u32(uint32_t n) {
    uint32_t l = 0;
    while ((1u << l) < n) ++l;
    return l;
}

/* fhe_ntt.wgsl:255-279: out[idx] <-> in[rev(idx)]. */
static void pass_bit_reverse(const w64 *in, w64 *out, uint32_t degree) {
    uint32_t log_n = log2_u32(degree);
    for (uint32_t idx = 0; idx < degree; ++idx) {
        uint32_t rev = bitrev_idx(idx, log_n);
        if (idx < rev) {
            out[idx] = in[rev];
            out[rev] = in[idx];
        } else if (idx == rev) {
            out[idx] = in[idx];
        }
    }
}

/* fhe_ntt.wgsl:212-252: one radix-2 DIT stage, stride 2^stage, twiddle
 * index local * N / (2 * stride).  u = a + w*b, v = a - w*b. */
static void pass_butterfly(const w64 *in, w64 *out, const w64 *tw, uint32_t degree,
                           uint32_t stage, w64 q) {
    uint32_t half = degree / 2u;
    uint32_t stride = 1u << stage;
    for (uint32_t bidx = 0; bidx < half; ++bidx) {
        uint32_t block = bidx / stride, local = bidx % stride;
        uint32_t ia = block * stride * 2u + local, ib = ia + stride;
        w64 a = in[ia], b = in[ib];
        w64 w = tw[local * (degree / (2u * stride))];
        w64 tb = w_mod_mul(w, b, q);
        out[ia] = w_mod_add(a, tb, q);
        out[ib] = w_mod_sub(a, tb, q);
    }
}

/* fhe_ntt/compute.rs:94-136: bit_reverse into the intermediate buffer, then
 * log2 N stages ping-ponging between intermediate and output. */
static void dit_chain(const uint64_t *in, uint64_t *out, uint32_t degree, uint64_t modulus,
                      const uint64_t *twiddles) {
    w64 *buf0 = (w64 *)malloc(sizeof(w64) * degree);
    w64 *buf1 = (w64 *)malloc(sizeof(w64) * degree);
    w64 *src = (w64 *)malloc(sizeof(w64) * degree);
    w64 *tw = (w64 *)malloc(sizeof(w64) * degree);
    for (uint32_t i = 0; i < degree; ++i) {
        src[i] = w64_of(in[i]);
        tw[i] = w64_of(twiddles[i]);
    }
    w64 q = w64_of(modulus);
    pass_bit_reverse(src, buf0, degree);
    uint32_t stages = log2_u32(degree);
    w64 *cur = buf0, *nxt = buf1;
    for (uint32_t s = 0; s < stages; ++s) {
        pass_butterfly(cur, nxt, tw, degree, s, q);
        w64 *t = cur;
        cur = nxt;
        nxt = t;
    }
    for (uint32_t i = 0; i < degree; ++i) out[i] = w64_val(cur[i]);
    free(buf0);
    free(buf1);
    free(src);
    free(tw);
}

/* ---- host-side Rust ---- */

static uint64_t mulmod_u128(uint64_t a, uint64_t b, uint64_t m) {
    return (uint64_t)(((unsigned __int128)a * b) % m);
}

/* fhe_ntt/mod.rs:174-184: power starts at 1 and is only reduced after the
 * first multiply, so out[0] == 1 even for modulus 1. */
void orc_ref_twiddles(uint32_t degree, uint64_t modulus, uint64_t root, uint64_t *out) {
    uint64_t power = 1;
    for (uint32_t k = 0; k < degree; ++k) {
        out[k] = power;
        power = mulmod_u128(power, root, modulus);
    }
}

/* fhe_ntt/mod.rs:190-204 */
uint64_t orc_ref_mod_pow(uint64_t base, uint64_t exp, uint64_t modulus) {
    if (modulus == 1) return 0;
    uint64_t result = 1;
    base %= modulus;
    while (exp > 0) {
        if (exp & 1) result = mulmod_u128(result, base, modulus);
        exp >>= 1;
        base = mulmod_u128(base, base, modulus);
    }
    return result;
}

/* fhe_ntt/mod.rs:210-242 */
uint64_t orc_ref_compute_primitive_root(uint32_t degree, uint64_t modulus) {
    uint64_t n = degree;
    if (modulus < 2 || n == 0) return 1;
    uint64_t qm1 = modulus - 1;
    if (qm1 % n != 0) return 3;
    uint64_t e = qm1 / n;
    static const uint64_t cands[] = {2, 3, 5, 7, 11, 13, 17, 19, 23, 29, 31};
    for (size_t i = 0; i < sizeof(cands) / sizeof(cands[0]); ++i) {
        uint64_t g = cands[i];
        if (g >= modulus) continue;
        uint64_t w = orc_ref_mod_pow(g, e, modulus);
        if (w == 1) continue;
        if (orc_ref_mod_pow(w, n, modulus) != 1) continue;
        if (n > 1 && n % 2 == 0 && orc_ref_mod_pow(w, n / 2, modulus) == 1) continue;
        return w;
    }
    return 3;
}

/* fhe_intt/mod.rs:177-198 (i128 extended Euclid; 0 when gcd > 1). */
uint64_t orc_ref_modinv(uint64_t a, uint64_t m) {
    __int128 t = 0, nt = 1, r = (__int128)m, nr = (__int128)a;
    while (nr != 0) {
        __int128 quo = r / nr;
        __int128 tmp = t - quo * nt;
        t = nt;
        nt = tmp;
        tmp = r - quo * nr;
        r = nr;
        nr = tmp;
    }
    if (r > 1) return 0;
    if (t < 0) t += (__int128)m;
    return (uint64_t)t;
}

/* fhe_intt/mod.rs:202-204 */
uint64_t orc_ref_compute_inverse_root(uint32_t degree, uint64_t modulus, uint64_t root) {
    (void)degree;
    return orc_ref_modinv(root, modulus);
}

/* fhe_fast_poly_mul.rs:176-197 */
uint64_t orc_ref_fastmul_modinv(uint64_t a, uint64_t m) {
    __int128 old_r = (__int128)a, r = (__int128)m, old_s = 1, s = 0;
    while (r != 0) {
        __int128 quo = old_r / r;
        __int128 tr = r;
        r = old_r - quo * r;
        old_r = tr;
        __int128 ts = s;
        s = old_s - quo * s;
        old_s = ts;
    }
    if (old_s < 0) old_s += (__int128)m;
    return (uint64_t)old_s;
}

/* FheNtt::execute (fhe_ntt/compute.rs:29-143). */
void orc_ref_ntt(const uint64_t *in, uint64_t *out, uint32_t degree, uint64_t modulus,
                 uint64_t root) {
    uint64_t *tw = (uint64_t *)malloc(sizeof(uint64_t) * degree);
    orc_ref_twiddles(degree, modulus, root, tw);
    dit_chain(in, out, degree, modulus, tw);
    free(tw);
}

/* FheIntt::execute (fhe_intt/compute.rs:27-168): the same DIT with the
 * inverse twiddles, then scale_by_n (fhe_intt.wgsl:282-303) multiplies by
 * N^-1 (compute_modular_inverse(N, q), fhe_intt/mod.rs:113) via mod_mul. */
void orc_ref_intt(const uint64_t *in, uint64_t *out, uint32_t degree, uint64_t modulus,
                  uint64_t inv_root) {
    uint64_t *tw = (uint64_t *)malloc(sizeof(uint64_t) * degree);
    uint64_t *tmp = (uint64_t *)malloc(sizeof(uint64_t) * degree);
    orc_ref_twiddles(degree, modulus, inv_root, tw);
    dit_chain(in, tmp, degree, modulus, tw);
    w64 q = w64_of(modulus), inv_n = w64_of(orc_ref_modinv(degree, modulus));
    for (uint32_t i = 0; i < degree; ++i) out[i] = w64_val(w_mod_mul(w64_of(tmp[i]), inv_n, q));
    free(tw);
    free(tmp);
}

/* ---- fhe_pointwise_mul.wgsl ---- */

/* :43-64 */
static void mul32_wide(uint32_t a, uint32_t b, uint32_t *lo_out, uint32_t *hi_out) {
    uint32_t a0 = a & 0xFFFFu, a1 = a >> 16, b0 = b & 0xFFFFu, b1 = b >> 16;
    uint32_t p0 = a0 * b0, p1 = a0 * b1, p2 = a1 * b0, p3 = a1 * b1;
    uint32_t lo = p0 + ((p1 & 0xFFFFu) << 16);
    uint32_t c1 = (lo < p0) ? 1u : 0u;
    uint32_t mid1 = (p1 >> 16) + c1;
    uint32_t prev = lo;
    lo = lo + ((p2 & 0xFFFFu) << 16);
    uint32_t c2 = (lo < prev) ? 1u : 0u;
    *lo_out = lo;
    *hi_out = p3 + (p2 >> 16) + mid1 + c2;
}

uint64_t orc_wgsl_mul32_wide(uint32_t a, uint32_t b) {
    uint32_t lo, hi;
    mul32_wide(a, b, &lo, &hi);
    return ((uint64_t)hi << 32) | lo;
}

/* :70-81 bit-serial reduce with a u32 accumulator. */
static uint32_t reduce64(uint32_t lo, uint32_t hi, uint32_t q) {
    uint32_t acc = 0u;
    for (int i = 31; i >= 0; --i) {
        acc = (acc << 1) | ((hi >> i) & 1u);
        if (acc >= q) acc -= q;
    }
    for (int i = 31; i >= 0; --i) {
        acc = (acc << 1) | ((lo >> i) & 1u);
        if (acc >= q) acc -= q;
    }
    return acc;
}

/* :87-141.  The wide path follows the shader word for word, including the
 * q_hat estimate `(w1 * mu.x) + (w0 * mu.y >> 32u)`: WGSL takes a runtime
 * shift count modulo the bit width, so `>> 32u` on a u32 is a shift by 0. */
uint64_t orc_wgsl_pointwise_mod_mul(uint64_t a, uint64_t b, uint64_t q, uint64_t mu) {
    uint32_t al = (uint32_t)a, ah = (uint32_t)(a >> 32);
    uint32_t bl = (uint32_t)b, bh = (uint32_t)(b >> 32);
    uint32_t ql = (uint32_t)q, qh = (uint32_t)(q >> 32);
    if (ah == 0u && bh == 0u && qh == 0u) {
        uint32_t lo, hi;
        mul32_wide(al, bl, &lo, &hi);
        return (uint64_t)reduce64(lo, hi, ql);
    }
    uint32_t p0l, p0h, p1l, p1h, p2l, p2h, p3l, p3h;
    mul32_wide(al, bl, &p0l, &p0h);
    mul32_wide(al, bh, &p1l, &p1h);
    mul32_wide(ah, bl, &p2l, &p2h);
    mul32_wide(ah, bh, &p3l, &p3h);
    uint32_t w0 = p0l, w1 = p0h, w2 = p3l, w3 = p3h;
    uint32_t prev = w1;
    w1 = w1 + p1l;
    uint32_t c1 = (w1 < prev) ? 1u : 0u;
    prev = w1;
    w1 = w1 + p2l;
    uint32_t c2 = (w1 < prev) ? 1u : 0u;
    uint32_t mid_carry = p1h + p2h + c1 + c2;
    prev = w2;
    w2 = w2 + mid_carry;
    w3 = w3 + ((w2 < prev) ? 1u : 0u);
    (void)w3;
    uint32_t mul_lo = (uint32_t)mu, mul_hi = (uint32_t)(mu >> 32);
    uint32_t qhat = (w1 * mul_lo) + (w0 * mul_hi); /* >> (32 mod 32) == >> 0 */
    uint32_t tl = qhat * ql, th = qhat * qh;
    uint32_t rx = w0 - tl, ry = w1 - th; /* component-wise, no borrow */
    for (int i = 0; i < 3; ++i) {
        if (ry > qh || (ry == qh && rx >= ql)) {
            if (rx < ql) ry -= 1u;
            rx -= ql;
            ry -= qh;
        }
    }
    return ((uint64_t)ry << 32) | rx;
}

/* fhe_pointwise_mul.rs:101-103 barrett_mu = u64::MAX / q (0 when q == 0). */
void orc_ref_pointwise(const uint64_t *a, const uint64_t *b, uint64_t *c, uint32_t degree,
                       uint64_t modulus) {
    uint64_t mu = modulus ? UINT64_MAX / modulus : 0;
    for (uint32_t i = 0; i < degree; ++i) c[i] = orc_wgsl_pointwise_mod_mul(a[i], b[i], modulus, mu);
}

/* fhe_fast_poly_mul.rs:122-154 */
void orc_ref_fast_poly_mul(const uint64_t *a, const uint64_t *b, uint64_t *c,
                           uint32_t degree, uint64_t modulus, uint64_t root) {
    uint64_t inv_root = orc_ref_fastmul_modinv(root, modulus);
    uint64_t *fa = (uint64_t *)malloc(sizeof(uint64_t) * degree);
    uint64_t *fb = (uint64_t *)malloc(sizeof(uint64_t) * degree);
    uint64_t *fc = (uint64_t *)malloc(sizeof(uint64_t) * degree);
    orc_ref_ntt(a, fa, degree, modulus, root);
    orc_ref_ntt(b, fb, degree, modulus, root);
    orc_ref_pointwise(fa, fb, fc, degree, modulus);
    orc_ref_intt(fc, c, degree, modulus, inv_root);
    free(fa);
    free(fb);
    free(fc);
}

/* Negacyclic forward through the reference ops: pre-twist with the
 * pointwise op, then the cyclic NTT with omega = psi^2. */
void orc_ref_negacyclic_ntt(const uint64_t *in, uint64_t *out, uint32_t degree,
                            uint64_t modulus, uint64_t psi) {
    uint64_t *tw = (uint64_t *)malloc(sizeof(uint64_t) * degree);
    uint64_t *tmp = (uint64_t *)malloc(sizeof(uint64_t) * degree);
    orc_ref_twiddles(degree, modulus, psi, tw); /* psi^j */
    orc_ref_pointwise(in, tw, tmp, degree, modulus);
    orc_ref_ntt(tmp, out, degree, modulus, mulmod_u128(psi, psi, modulus));
    free(tw);
    free(tmp);
}

/* Negacyclic inverse through the reference ops: cyclic INTT with
 * psi^-2, then post-twist by psi^-j with the pointwise op. */
void orc_ref_negacyclic_intt(const uint64_t *in, uint64_t *out, uint32_t degree,
                             uint64_t modulus, uint64_t psi) {
    uint64_t psi_inv = orc_ref_modinv(psi, modulus);
    uint64_t *tw = (uint64_t *)malloc(sizeof(uint64_t) * degree);
    uint64_t *tmp = (uint64_t *)malloc(sizeof(uint64_t) * degree);
    orc_ref_intt(in, tmp, degree, modulus, mulmod_u128(psi_inv, psi_inv, modulus));
    orc_ref_twiddles(degree, modulus, psi_inv, tw); /* psi^-j */
    orc_ref_pointwise(tmp, tw, out, degree, modulus);
    free(tw);
    free(tmp);
}
