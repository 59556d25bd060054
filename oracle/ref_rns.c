/* ref_rns.c -- CPU restatement of the reference's Galois rotation, modulus
 * switch and key switch (FheRotate, FheModulusSwitch, FheKeySwitch), plus
 * the exact versions the product computes where the reference's arithmetic
 * wraps.  TEST INFRASTRUCTURE ONLY: see oracle.h.  Paths are inside
 * crates/barracuda/src/ops/. */
#include <stdint.h>

#include "oracle.h"

/* fhe_rotate.rs:150-155: a negative rotation r becomes degree + r (so
 * r in [-degree/2, degree/2] maps into [0, degree)); galois = 2 r + 1
 * (fhe_rotate.wgsl:67-69, u32 arithmetic). */
uint32_t orc_ref_rotate_galois(uint32_t degree, int32_t rotation) {
    const uint32_t r = rotation < 0 ? (uint32_t)((int32_t)degree + rotation) : (uint32_t)rotation;
    return 2u * r + 1u;
}

/* fhe_rotate.wgsl:52-63 u64_negate_mod: 0 stays 0, otherwise m - a with
 * 64-bit wrap-around (a > m is not reduced first). */
static uint64_t negate_mod(uint64_t a, uint64_t m) {
    return a == 0 ? 0 : m - a;
}

/* fhe_rotate.wgsl:98-128 rotate_automorphism, one invocation per input
 * index i: new_power = (i * galois mod 2^32) mod 2N (u32 product, as the
 * shader computes it), out[new_power - N] = negate(in[i]) when
 * new_power >= N, else out[new_power] = in[i].  Scatter form, exactly as the
 * shader writes it; galois is odd, so every output is written once. */
void orc_ref_rotate(const uint64_t *in, uint64_t *out, uint32_t degree, int32_t rotation,
                    uint64_t modulus) {
    const uint32_t g = orc_ref_rotate_galois(degree, rotation);
    const uint32_t two_n = 2u * degree;
    for (uint32_t i = 0; i < degree; ++i) {
        const uint32_t p = (uint32_t)(i * g) % two_n;
        if (p >= degree)
            out[p - degree] = negate_mod(in[i], modulus);
        else
            out[p] = in[i];
    }
}

/* General automorphism X -> X^g (g odd) of one polynomial in
 * Z_q[X]/(X^N + 1), scatter form with exact index arithmetic and the same
 * negation as orc_ref_rotate. */
void orc_automorphism(const uint64_t *in, uint64_t *out, uint32_t degree, uint32_t galois,
                      uint64_t modulus) {
    const uint64_t two_n = 2ull * degree;
    for (uint32_t i = 0; i < degree; ++i) {
        const uint64_t p = ((uint64_t)i * galois) % two_n;
        if (p >= degree)
            out[p - degree] = negate_mod(in[i], modulus);
        else
            out[p] = in[i];
    }
}

/* fhe_modulus_switch.wgsl:103-131 scale_and_round, one coefficient:
 * scaled = coeff * q_new with 64-bit wrap-around, quotient and remainder of
 * scaled by q_old, +1 when remainder * 2 (64-bit wrap-around) >= q_old, then
 * the result mod q_new.  With q_new == 0 (allowed by the constructor when
 * q_old == 1) every step gives 0 before the final remainder, whose value is
 * then 0 under either WGSL rule for a zero divisor. */
uint64_t orc_ref_modulus_switch1(uint64_t c, uint64_t q_old, uint64_t q_new) {
    const uint64_t scaled = c * q_new;
    uint64_t result = scaled / q_old;
    const uint64_t rem = scaled % q_old;
    if (rem * 2u >= q_old) result += 1u;
    return q_new == 0 ? 0 : result % q_new;
}

/* Exact round(c * q_new / q_old) mod q_new (ties round up), for any u64 c
 * and q_new < q_old: the 128-bit product is not truncated.  Equal to
 * orc_ref_modulus_switch1 whenever c * q_new < 2^64 and q_old <= 2^63. */
uint64_t orc_exact_modulus_switch1(uint64_t c, uint64_t q_old, uint64_t q_new) {
    if (q_new == 0) return 0;
    const unsigned __int128 x = (unsigned __int128)c * q_new;
    unsigned __int128 t = x / q_old;
    const unsigned __int128 r = x % q_old;
    if (r >= (unsigned __int128)q_old - r) t += 1;
    return (uint64_t)(t % q_new);
}

void orc_ref_modulus_switch(const uint64_t *in, uint64_t *out, uint32_t degree, uint64_t q_old,
                            uint64_t q_new) {
    for (uint32_t i = 0; i < degree; ++i) out[i] = orc_ref_modulus_switch1(in[i], q_old, q_new);
}

void orc_exact_modulus_switch(const uint64_t *in, uint64_t *out, size_t count, uint64_t q_old,
                              uint64_t q_new) {
    for (size_t i = 0; i < count; ++i) out[i] = orc_exact_modulus_switch1(in[i], q_old, q_new);
}

/* fhe_key_switch.rs:178-210 FheKeySwitch::execute, both dispatches of one
 * submission in order: decompose_base_b (fhe_key_switch.wgsl:90-115) writes
 * digit 0 = (coeff mod base) as (digit, 0) into the output, then
 * accumulate_switched (:128-148) reads the INPUT buffer (binding 0) and
 * stores it unchanged over the same output words.  Both passes are restated
 * so the oracle shows the net effect instead of assuming it. */
void orc_ref_key_switch(const uint64_t *in, uint64_t *out, uint32_t degree, uint32_t decomp_base,
                        uint32_t decomp_levels) {
    (void)decomp_levels;
    for (uint32_t i = 0; i < degree; ++i) out[i] = (uint64_t)(uint32_t)(in[i] % decomp_base);
    for (uint32_t i = 0; i < degree; ++i) out[i] = in[i];
}

/* fhe_key_switch.wgsl:71-84 decompose_digit for every level: digit l of c is
 * (c / base^l) mod base, by repeated 64-by-32-bit division.  Output is
 * digit-major: out[l * count + i] = digit l of in[i]. */
void orc_decompose(const uint64_t *in, uint64_t *out, size_t count, uint32_t base, uint32_t levels) {
    for (size_t i = 0; i < count; ++i) {
        uint64_t cur = in[i];
        for (uint32_t l = 0; l < levels; ++l) {
            out[(size_t)l * count + i] = cur % base;
            cur /= base;
        }
    }
}
