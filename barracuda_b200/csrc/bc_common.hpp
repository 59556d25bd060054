// bc_common.hpp -- shared host-side pieces of libbarracuda_fhe: status and
// error reporting, and exact host modular arithmetic used to build plans.
#pragma once

#include <cstdint>
#include <cstdio>
#include <string>

#include "barracuda_fhe.h"

namespace bc {

// Records `msg` as this thread's last error and returns `status`.
int fail(int status, const std::string &msg);
void clear_error();

template <typename... Args>
std::string format(const char *fmt, Args... args) {
    int n = std::snprintf(nullptr, 0, fmt, args...);
    std::string s(static_cast<size_t>(n > 0 ? n : 0), '\0');
    if (n > 0) std::snprintf(&s[0], s.size() + 1, fmt, args...);
    return s;
}

// ---- exact host arithmetic (u128 products) ----
inline uint64_t mulmod(uint64_t a, uint64_t b, uint64_t q) {
    return static_cast<uint64_t>((static_cast<unsigned __int128>(a) * b) % q);
}
uint64_t powmod(uint64_t a, uint64_t e, uint64_t q);

// crates/barracuda/src/ops/fhe_ntt/mod.rs:190-204 (mod_pow: modulus 1 -> 0).
uint64_t ref_mod_pow(uint64_t base, uint64_t exp, uint64_t modulus);
// fhe_ntt/mod.rs:210-242 compute_primitive_root.
uint64_t ref_primitive_root(uint32_t degree, uint64_t modulus);
// fhe_intt/mod.rs:177-198 compute_modular_inverse: 0 when gcd(a, m) > 1.
uint64_t ref_modinv(uint64_t a, uint64_t m);
// fhe_fast_poly_mul.rs:176-197: Bezout coefficient, no invertibility check.
uint64_t ref_fastmul_modinv(uint64_t a, uint64_t m);

bool is_prime(uint64_t n);
uint64_t ntt_prime(uint32_t bits, uint32_t degree, uint32_t index);
uint64_t smallest_generator(uint64_t q);

inline uint32_t ilog2(uint64_t n) {
    uint32_t l = 0;
    while ((uint64_t(1) << l) < n) ++l;
    return l;
}
inline bool is_pow2(uint64_t n) { return n && !(n & (n - 1)); }
inline uint32_t bitrev(uint32_t x, uint32_t bits) {
    uint32_t r = 0;
    for (uint32_t i = 0; i < bits; ++i) {
        r = (r << 1) | (x & 1u);
        x >>= 1;
    }
    return r;
}

// Shoup companions: floor(w * 2^32 / q) and floor(w * 2^64 / q), w < q.
inline uint32_t shoup32(uint32_t w, uint32_t q) {
    return static_cast<uint32_t>((static_cast<uint64_t>(w) << 32) / q);
}
inline uint64_t shoup64(uint64_t w, uint64_t q) {
    return static_cast<uint64_t>((static_cast<unsigned __int128>(w) << 64) / q);
}

}  // namespace bc
