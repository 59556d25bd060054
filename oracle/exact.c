/*
 * exact.c -- exact modular arithmetic used to check the reference
 * restatement and the product: u128 products, prime search, generators,
 * exact cyclic / negacyclic transforms and schoolbook convolutions.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h).
 */
#include "oracle.h"

#include <stdlib.h>
#include <string.h>

uint64_t orc_mulmod(uint64_t a, uint64_t b, uint64_t q) {
    return (uint64_t)(((unsigned __int128)a * b) % q);
}

uint64_t orc_powmod(uint64_t a, uint64_t e, uint64_t q) {
    uint64_t r = 1 % q;
    a %= q;
    while (e) {
        if (e & 1) r = orc_mulmod(r, a, q);
        a = orc_mulmod(a, a, q);
        e >>= 1;
    }
    return r;
}

/* Deterministic Miller-Rabin for 64-bit n (first 12 prime bases). */
int orc_is_prime(uint64_t n) {
    static const uint64_t bases[] = {2, 3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37};
    if (n < 2) return 0;
    for (size_t i = 0; i < 12; ++i) {
        if (n == bases[i]) return 1;
        if (n % bases[i] == 0) return 0;
    }
    uint64_t d = n - 1;
    int s = 0;
    while ((d & 1) == 0) {
        d >>= 1;
        ++s;
    }
    for (size_t i = 0; i < 12; ++i) {
        uint64_t x = orc_powmod(bases[i], d, n);
        if (x == 1 || x == n - 1) continue;
        int composite = 1;
        for (int r = 1; r < s; ++r) {
            x = orc_mulmod(x, x, n);
            if (x == n - 1) {
                composite = 0;
                break;
            }
        }
        if (composite) return 0;
    }
    return 1;
}

uint64_t orc_ntt_prime(uint32_t bits, uint32_t degree, uint32_t index) {
    if (bits < 2 || bits > 63) return 0;
    uint64_t step = 2ull * degree;
    uint64_t top = (1ull << bits) - 1; /* largest candidate < 2^bits */
    uint64_t q = top - ((top - 1) % step); /* largest value <= top with q == 1 mod step */
    uint32_t found = 0;
    while (q > step) {
        if (orc_is_prime(q)) {
            if (found == index) return q;
            ++found;
        }
        q -= step;
    }
    return 0;
}

static uint64_t gcd_u64(uint64_t a, uint64_t b) {
    while (b) {
        uint64_t t = a % b;
        a = b;
        b = t;
    }
    return a;
}

/* Pollard rho with Floyd cycle detection; returns a non-trivial factor of
 * the odd composite n (tries successive polynomial constants c). */
static uint64_t rho(uint64_t n) {
    if ((n & 1) == 0) return 2;
    for (uint64_t c = 1;; ++c) {
        uint64_t x = 2, y = 2, d = 1;
        while (d == 1) {
            x = (orc_mulmod(x, x, n) + c) % n;
            y = (orc_mulmod(y, y, n) + c) % n;
            y = (orc_mulmod(y, y, n) + c) % n;
            d = gcd_u64(x > y ? x - y : y - x, n);
        }
        if (d != n) return d;
    }
}

static void factor_into(uint64_t n, uint64_t *fs, int *nf) {
    if (n == 1) return;
    if (orc_is_prime(n)) {
        for (int i = 0; i < *nf; ++i)
            if (fs[i] == n) return;
        fs[(*nf)++] = n;
        return;
    }
    for (uint64_t p = 2; p < 1000; ++p) {
        if (n % p == 0) {
            factor_into(p, fs, nf);
            while (n % p == 0) n /= p;
            factor_into(n, fs, nf);
            return;
        }
    }
    uint64_t d = rho(n);
    factor_into(d, fs, nf);
    factor_into(n / d, fs, nf);
}

uint64_t orc_smallest_generator(uint64_t q) {
    if (q == 2) return 1;
    uint64_t fs[64];
    int nf = 0;
    factor_into(q - 1, fs, &nf);
    for (uint64_t g = 2; g < q; ++g) {
        int ok = 1;
        for (int i = 0; i < nf; ++i) {
            if (orc_powmod(g, (q - 1) / fs[i], q) == 1) {
                ok = 0;
                break;
            }
        }
        if (ok) return g;
    }
    return 0;
}

uint64_t orc_psi(uint64_t q, uint32_t degree) {
    uint64_t g = orc_smallest_generator(q);
    return orc_powmod(g, (q - 1) / (2ull * degree), q);
}

void orc_exact_dft(const uint64_t *in, uint64_t *out, uint32_t n, uint64_t q, uint64_t w) {
    for (uint32_t k = 0; k < n; ++k) {
        uint64_t wk = orc_powmod(w, k, q), acc = 0, wp = 1 % q;
        for (uint32_t j = 0; j < n; ++j) {
            acc = (acc + orc_mulmod(in[j] % q, wp, q)) % q;
            wp = orc_mulmod(wp, wk, q);
        }
        out[k] = acc;
    }
}

static uint32_t brev(uint32_t x, uint32_t bits) {
    uint32_t r = 0;
    for (uint32_t i = 0; i < bits; ++i) {
        r = (r << 1) | (x & 1u);
        x >>= 1;
    }
    return r;
}

void orc_exact_ntt(const uint64_t *in, uint64_t *out, uint32_t n, uint64_t q, uint64_t w) {
    uint32_t L = 0;
    while ((1u << L) < n) ++L;
    uint64_t *a = (uint64_t *)malloc(sizeof(uint64_t) * n);
    for (uint32_t i = 0; i < n; ++i) a[brev(i, L)] = in[i] % q;
    for (uint32_t len = 2; len <= n; len <<= 1) {
        uint64_t wl = orc_powmod(w, n / len, q);
        for (uint32_t i = 0; i < n; i += len) {
            uint64_t t = 1 % q;
            for (uint32_t j = 0; j < len / 2; ++j) {
                uint64_t u = a[i + j], v = orc_mulmod(a[i + j + len / 2], t, q);
                a[i + j] = (u + v) % q;
                a[i + j + len / 2] = (u + q - v) % q;
                t = orc_mulmod(t, wl, q);
            }
        }
    }
    memcpy(out, a, sizeof(uint64_t) * n);
    free(a);
}

void orc_exact_negacyclic_ntt(const uint64_t *in, uint64_t *out, uint32_t n, uint64_t q,
                              uint64_t psi) {
    uint64_t *t = (uint64_t *)malloc(sizeof(uint64_t) * n);
    uint64_t p = 1 % q;
    for (uint32_t j = 0; j < n; ++j) {
        t[j] = orc_mulmod(in[j] % q, p, q);
        p = orc_mulmod(p, psi, q);
    }
    orc_exact_ntt(t, out, n, q, orc_mulmod(psi, psi, q));
    free(t);
}

static uint64_t inv_mod(uint64_t a, uint64_t q) { return orc_powmod(a, q - 2, q); }

void orc_exact_negacyclic_intt(const uint64_t *in, uint64_t *out, uint32_t n, uint64_t q,
                               uint64_t psi) {
    uint64_t pinv = inv_mod(psi, q);
    uint64_t ninv = inv_mod(n % q, q);
    orc_exact_ntt(in, out, n, q, orc_mulmod(pinv, pinv, q));
    uint64_t p = ninv;
    for (uint32_t j = 0; j < n; ++j) {
        out[j] = orc_mulmod(out[j], p, q);
        p = orc_mulmod(p, pinv, q);
    }
}

void orc_cyclic_convolution(const uint64_t *a, const uint64_t *b, uint64_t *c, uint32_t n,
                            uint64_t q) {
    for (uint32_t k = 0; k < n; ++k) c[k] = 0;
    for (uint32_t i = 0; i < n; ++i)
        for (uint32_t j = 0; j < n; ++j) {
            uint32_t k = (i + j) % n;
            c[k] = (c[k] + orc_mulmod(a[i] % q, b[j] % q, q)) % q;
        }
}

void orc_negacyclic_convolution(const uint64_t *a, const uint64_t *b, uint64_t *c,
                                uint32_t n, uint64_t q) {
    for (uint32_t k = 0; k < n; ++k) c[k] = 0;
    for (uint32_t i = 0; i < n; ++i)
        for (uint32_t j = 0; j < n; ++j) {
            uint64_t p = orc_mulmod(a[i] % q, b[j] % q, q);
            uint32_t k = i + j;
            if (k < n)
                c[k] = (c[k] + p) % q;
            else
                c[k - n] = (c[k - n] + q - p) % q;
        }
}

static uint64_t splitmix(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

uint64_t orc_seeded_value(uint64_t seed, uint64_t g, uint64_t q) {
    uint64_t z = splitmix(seed + (g + 1) * 0x9E3779B97F4A7C15ull);
    return (uint64_t)(((unsigned __int128)z * q) >> 64);
}

void orc_seeded_fill(uint64_t *out, size_t count, uint64_t seed, uint64_t g0, uint64_t q) {
    for (size_t i = 0; i < count; ++i) out[i] = orc_seeded_value(seed, g0 + i, q);
}

uint64_t orc_digest(const uint64_t *x, size_t count, uint64_t first_index) {
    uint64_t acc = 0;
    for (size_t i = 0; i < count; ++i) acc += splitmix(x[i] ^ ((first_index + i) * 0xD1B54A32D192ED03ull));
    return acc;
}
