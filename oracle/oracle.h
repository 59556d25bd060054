/*
 * oracle.h -- CPU restatement of barraCuda's FHE NTT path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library links, loads or
 * calls this code.  It is used by tests/, by __graft_entry__.smoke() and by
 * the cpu_baseline / --impl reference legs of bench.py, always as the
 * checker or the timed CPU baseline, never as a path that produces product
 * output.
 *
 * Three parts:
 *   1. ref_wgsl.c  -- a restatement of the reference's own algorithm: the
 *      WGSL shaders (u32-pair u64 emulation, low-64-bit multiply, bit-serial
 *      reduction, bit-reverse + log2 N radix-2 DIT passes with ping-pong
 *      buffers, separate N^-1 scale pass, pointwise mul with its 32-bit fast
 *      path and 64-bit Barrett path) and the host-side Rust around them
 *      (twiddle generation, root search, extended Euclid).  Bit-exact target
 *      for parity.  Citations are to crates/barracuda/src/ops/... of
 *      ecoPrimals/barraCuda.
 *   2. exact.c     -- exact u128 arithmetic: cyclic / negacyclic NTT and
 *      INTT, schoolbook convolutions, prime search, generators.
 *   3. baseline.c  -- a threaded driver of part 1 used as the CPU baseline.
 */
#ifndef BC_ORACLE_H
#define BC_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------- part 1: reference restatement ---------------- */

/* fhe_ntt.wgsl:45-70 u64_mul (low 64 bits via 16-bit partial products). */
uint64_t orc_wgsl_u64_mul(uint64_t a, uint64_t b);
/* fhe_ntt.wgsl:84-110 u64_mod_simple (bit-serial for m < 2^32, else <=128 subtractions). */
uint64_t orc_wgsl_u64_mod_simple(uint64_t a, uint64_t m);
/* fhe_pointwise_mul.wgsl:43-64 mul32_wide -> 64-bit product. */
uint64_t orc_wgsl_mul32_wide(uint32_t a, uint32_t b);
/* fhe_pointwise_mul.wgsl:87-141 mod_mul (fast path + 64-bit Barrett path). */
uint64_t orc_wgsl_pointwise_mod_mul(uint64_t a, uint64_t b, uint64_t q, uint64_t mu);

/* fhe_ntt/mod.rs:174-184 compute_twiddle_factors: out[k] = root^k, k < degree. */
void orc_ref_twiddles(uint32_t degree, uint64_t modulus, uint64_t root, uint64_t *out);
/* fhe_ntt/mod.rs:190-204 mod_pow. */
uint64_t orc_ref_mod_pow(uint64_t base, uint64_t exp, uint64_t modulus);
/* fhe_ntt/mod.rs:210-242 compute_primitive_root. */
uint64_t orc_ref_compute_primitive_root(uint32_t degree, uint64_t modulus);
/* fhe_intt/mod.rs:177-198 compute_modular_inverse (0 when not invertible). */
uint64_t orc_ref_modinv(uint64_t a, uint64_t m);
/* fhe_intt/mod.rs:202-204 compute_inverse_root. */
uint64_t orc_ref_compute_inverse_root(uint32_t degree, uint64_t modulus, uint64_t root);
/* fhe_fast_poly_mul.rs:176-197 private extended Euclid (no invertibility check). */
uint64_t orc_ref_fastmul_modinv(uint64_t a, uint64_t m);

/* fhe_ntt/compute.rs:29-143 + fhe_ntt.wgsl: FheNtt::execute on one polynomial.
 * degree must be a power of two >= 1; no validation here (the op API does it). */
void orc_ref_ntt(const uint64_t *in, uint64_t *out, uint32_t degree, uint64_t modulus,
                 uint64_t root);
/* fhe_intt/compute.rs:27-168 + fhe_intt.wgsl: FheIntt::execute (DIT with the
 * given inverse root, then the scale_by_n pass with N^-1 from orc_ref_modinv). */
void orc_ref_intt(const uint64_t *in, uint64_t *out, uint32_t degree, uint64_t modulus,
                  uint64_t inv_root);
/* fhe_pointwise_mul.rs:119-155 + .wgsl main: C[i] = A[i]*B[i] mod q. */
void orc_ref_pointwise(const uint64_t *a, const uint64_t *b, uint64_t *c, uint32_t degree,
                       uint64_t modulus);
/* fhe_fast_poly_mul.rs:122-154: NTT(a), NTT(b), pointwise, INTT(inv root). */
void orc_ref_fast_poly_mul(const uint64_t *a, const uint64_t *b, uint64_t *c,
                           uint32_t degree, uint64_t modulus, uint64_t root);

/* Negacyclic transforms expressed with the reference's own ops:
 *   forward = FheNtt(omega = psi^2) applied to FhePointwiseMul(a, [psi^j])
 *   inverse = FhePointwiseMul(FheIntt(A, psi^-2), [psi^-j])            */
void orc_ref_negacyclic_ntt(const uint64_t *in, uint64_t *out, uint32_t degree,
                            uint64_t modulus, uint64_t psi);
void orc_ref_negacyclic_intt(const uint64_t *in, uint64_t *out, uint32_t degree,
                             uint64_t modulus, uint64_t psi);

/* Coefficient-wise ops (ref_poly.c), reference behaviour for any u64 input:
 * fhe_poly_add.wgsl (wrapping sum, two conditional subtractions of q),
 * fhe_poly_sub.wgsl (a - b, or (q - b) + a when a < b), fhe_poly_mul.wgsl
 * (128-bit product through a 32x32 helper that can lose 2^32 in its middle
 * sum, then at most 1000 subtractions of q, or an approximate Barrett step
 * above 2^64).  orc_exact_poly_mul is the exact (a * b) mod q. */
uint64_t orc_ref_poly_add1(uint64_t a, uint64_t b, uint64_t q);
uint64_t orc_ref_poly_sub1(uint64_t a, uint64_t b, uint64_t q);
uint64_t orc_ref_poly_mul1(uint64_t a, uint64_t b, uint64_t q);
void orc_ref_poly_add(const uint64_t *a, const uint64_t *b, uint64_t *c, uint32_t degree, uint64_t q);
void orc_ref_poly_sub(const uint64_t *a, const uint64_t *b, uint64_t *c, uint32_t degree, uint64_t q);
void orc_ref_poly_mul(const uint64_t *a, const uint64_t *b, uint64_t *c, uint32_t degree, uint64_t q);
void orc_exact_poly_mul(const uint64_t *a, const uint64_t *b, uint64_t *c, uint32_t degree, uint64_t q);

/* Rotation, modulus switch and key switch (ref_rns.c).
 * orc_ref_rotate: fhe_rotate.wgsl (galois = 2r + 1 after fhe_rotate.rs maps a
 *   negative r to degree + r; out[i*g mod 2N] = in[i], negated as m - in[i]
 *   (0 stays 0) where i*g mod 2N >= N).  orc_automorphism: the same for any
 *   odd g with exact index arithmetic.
 * orc_ref_modulus_switch1: fhe_modulus_switch.wgsl scale_and_round with its
 *   64-bit wrap-around of coeff * q_new; orc_exact_modulus_switch1 the exact
 *   round(coeff * q_new / q_old) mod q_new.
 * orc_ref_key_switch: both passes of FheKeySwitch::execute (the second copies
 *   the input over the first's digits).  orc_decompose: every base-B digit,
 *   digit-major. */
uint32_t orc_ref_rotate_galois(uint32_t degree, int32_t rotation);
void orc_ref_rotate(const uint64_t *in, uint64_t *out, uint32_t degree, int32_t rotation,
                    uint64_t modulus);
void orc_automorphism(const uint64_t *in, uint64_t *out, uint32_t degree, uint32_t galois,
                      uint64_t modulus);
uint64_t orc_ref_modulus_switch1(uint64_t c, uint64_t q_old, uint64_t q_new);
uint64_t orc_exact_modulus_switch1(uint64_t c, uint64_t q_old, uint64_t q_new);
void orc_ref_modulus_switch(const uint64_t *in, uint64_t *out, uint32_t degree, uint64_t q_old,
                            uint64_t q_new);
void orc_exact_modulus_switch(const uint64_t *in, uint64_t *out, size_t count, uint64_t q_old,
                              uint64_t q_new);
void orc_ref_key_switch(const uint64_t *in, uint64_t *out, uint32_t degree, uint32_t decomp_base,
                        uint32_t decomp_levels);
void orc_decompose(const uint64_t *in, uint64_t *out, size_t count, uint32_t base, uint32_t levels);

/* ---------------- part 2: exact arithmetic ---------------- */

uint64_t orc_mulmod(uint64_t a, uint64_t b, uint64_t q);
uint64_t orc_powmod(uint64_t a, uint64_t e, uint64_t q);
int orc_is_prime(uint64_t n);
/* i-th (0-based) largest prime q < 2^bits with q == 1 mod 2N; 0 if none found. */
uint64_t orc_ntt_prime(uint32_t bits, uint32_t degree, uint32_t index);
/* smallest generator of Z_q^* (q prime). */
uint64_t orc_smallest_generator(uint64_t q);
/* psi = g^((q-1)/2N) with g the smallest generator. */
uint64_t orc_psi(uint64_t q, uint32_t degree);

/* exact cyclic transform X_k = sum_j x_j w^{jk} (any w, O(N^2), small N). */
void orc_exact_dft(const uint64_t *in, uint64_t *out, uint32_t n, uint64_t q, uint64_t w);
/* exact cyclic NTT in natural order, O(N log N); w must have w^N = 1. Inputs reduced mod q. */
void orc_exact_ntt(const uint64_t *in, uint64_t *out, uint32_t n, uint64_t q, uint64_t w);
/* exact negacyclic forward A_k = sum_j a_j psi^{j(2k+1)} (natural order). */
void orc_exact_negacyclic_ntt(const uint64_t *in, uint64_t *out, uint32_t n, uint64_t q,
                              uint64_t psi);
/* exact negacyclic inverse, a_j = N^-1 psi^-j sum_k A_k psi^{-2jk}. */
void orc_exact_negacyclic_intt(const uint64_t *in, uint64_t *out, uint32_t n, uint64_t q,
                               uint64_t psi);
/* schoolbook products mod (X^N - 1) and mod (X^N + 1). */
void orc_cyclic_convolution(const uint64_t *a, const uint64_t *b, uint64_t *c, uint32_t n,
                            uint64_t q);
void orc_negacyclic_convolution(const uint64_t *a, const uint64_t *b, uint64_t *c,
                                uint32_t n, uint64_t q);

/* Counter-based input generator shared with the product's device generator:
 * value(seed, g) = floor(splitmix64(seed + (g+1)*0x9E3779B97F4A7C15) * q / 2^64). */
uint64_t orc_seeded_value(uint64_t seed, uint64_t g, uint64_t q);
void orc_seeded_fill(uint64_t *out, size_t count, uint64_t seed, uint64_t g0, uint64_t q);
/* Order-sensitive digest of the product's verification path (bc_digest):
 * sum_i splitmix64(x_i ^ ((first_index + i) * 0xD1B54A32D192ED03)) mod 2^64.
 * A sum over global indices, so the digests of the shards of an array add up
 * to the digest of the whole array. */
uint64_t orc_digest(const uint64_t *x, size_t count, uint64_t first_index);

/* ---------------- part 3: threaded CPU baseline ---------------- */

/* Runs orc_ref_ntt (kind 0), orc_ref_intt (kind 1), orc_ref_negacyclic_ntt (2),
 * orc_ref_negacyclic_intt (3), an exact O(N log N) negacyclic forward (4) or
 * inverse (5) on
 * `count` polynomials of `degree` coefficients stored back to back, using up
 * to `threads` POSIX threads.  Polynomial p uses modulus moduli[p % n_moduli]
 * and root roots[p % n_moduli].  Returns the wall time in seconds. */
double orc_baseline_run(int kind, const uint64_t *in, uint64_t *out, uint32_t degree,
                        uint32_t count, const uint64_t *moduli, const uint64_t *roots,
                        uint32_t n_moduli, int threads);

/* Polynomial products c = a * b of `count` limb-polynomial pairs stored back
 * to back, on up to `threads` threads; pair p uses moduli[p % n_moduli] and
 * roots[p % n_moduli].  kind 0: the reference's cyclic FheFastPolyMul chain
 * (root = omega); 1: the reference ops chained into a negacyclic product
 * (root = psi); 2: exact negacyclic product (psi); 3: exact cyclic product
 * (omega).  Returns the wall time in seconds. */
double orc_batch_polymul(int kind, const uint64_t *a, const uint64_t *b, uint64_t *c, uint32_t degree,
                         uint32_t count, const uint64_t *moduli, const uint64_t *roots, uint32_t n_moduli,
                         int threads);

#ifdef __cplusplus
}
#endif
#endif
