// bc_math.cpp -- error state and exact host arithmetic for plan building.
#include <string>

#include "bc_common.hpp"

namespace bc {

namespace {
thread_local std::string g_last_error;
}

int fail(int status, const std::string &msg) {
    g_last_error = msg;
    return status;
}

void clear_error() { g_last_error.clear(); }

const char *last_error_cstr() { return g_last_error.c_str(); }

uint64_t powmod(uint64_t a, uint64_t e, uint64_t q) {
    uint64_t r = 1 % q;
    a %= q;
    while (e) {
        if (e & 1) r = mulmod(r, a, q);
        a = mulmod(a, a, q);
        e >>= 1;
    }
    return r;
}

uint64_t ref_mod_pow(uint64_t base, uint64_t exp, uint64_t modulus) {
    if (modulus == 1) return 0;
    return powmod(base, exp, modulus);
}

uint64_t ref_primitive_root(uint32_t degree, uint64_t modulus) {
    const uint64_t n = degree;
    if (modulus < 2 || n == 0) return 1;
    const uint64_t qm1 = modulus - 1;
    if (qm1 % n != 0) return 3;
    const uint64_t e = qm1 / n;
    static const uint64_t candidates[] = {2, 3, 5, 7, 11, 13, 17, 19, 23, 29, 31};
    for (uint64_t g : candidates) {
        if (g >= modulus) continue;
        const uint64_t w = ref_mod_pow(g, e, modulus);
        if (w == 1) continue;
        if (ref_mod_pow(w, n, modulus) != 1) continue;
        if (n > 1 && n % 2 == 0 && ref_mod_pow(w, n / 2, modulus) == 1) continue;
        return w;
    }
    return 3;
}

uint64_t ref_modinv(uint64_t a, uint64_t m) {
    __int128 t = 0, nt = 1, r = static_cast<__int128>(m), nr = static_cast<__int128>(a);
    while (nr != 0) {
        const __int128 quo = r / nr;
        __int128 tmp = t - quo * nt;
        t = nt;
        nt = tmp;
        tmp = r - quo * nr;
        r = nr;
        nr = tmp;
    }
    if (r > 1) return 0;
    if (t < 0) t += static_cast<__int128>(m);
    return static_cast<uint64_t>(t);
}

uint64_t ref_fastmul_modinv(uint64_t a, uint64_t m) {
    __int128 old_r = static_cast<__int128>(a), r = static_cast<__int128>(m);
    __int128 old_s = 1, s = 0;
    while (r != 0) {
        const __int128 quo = old_r / r;
        __int128 t = r;
        r = old_r - quo * r;
        old_r = t;
        t = s;
        s = old_s - quo * s;
        old_s = t;
    }
    if (old_s < 0) old_s += static_cast<__int128>(m);
    return static_cast<uint64_t>(old_s);
}

bool is_prime(uint64_t n) {
    static const uint64_t bases[] = {2, 3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37};
    if (n < 2) return false;
    for (uint64_t p : bases) {
        if (n == p) return true;
        if (n % p == 0) return false;
    }
    uint64_t d = n - 1;
    int s = 0;
    while ((d & 1) == 0) {
        d >>= 1;
        ++s;
    }
    for (uint64_t a : bases) {
        uint64_t x = powmod(a, d, n);
        if (x == 1 || x == n - 1) continue;
        bool witness = true;
        for (int r = 1; r < s && witness; ++r) {
            x = mulmod(x, x, n);
            if (x == n - 1) witness = false;
        }
        if (witness) return false;
    }
    return true;
}

uint64_t ntt_prime(uint32_t bits, uint32_t degree, uint32_t index) {
    if (bits < 2 || bits > 63 || degree == 0) return 0;
    const uint64_t step = 2ull * degree;
    const uint64_t top = (1ull << bits) - 1;
    uint64_t q = top - ((top - 1) % step);
    uint32_t found = 0;
    while (q > step) {
        if (is_prime(q)) {
            if (found == index) return q;
            ++found;
        }
        q -= step;
    }
    return 0;
}

namespace {
uint64_t gcd64(uint64_t a, uint64_t b) {
    while (b) {
        const uint64_t t = a % b;
        a = b;
        b = t;
    }
    return a;
}

// Pollard rho (Floyd); n odd composite.
uint64_t rho_factor(uint64_t n) {
    if ((n & 1) == 0) return 2;
    for (uint64_t c = 1;; ++c) {
        uint64_t x = 2, y = 2, d = 1;
        while (d == 1) {
            x = (mulmod(x, x, n) + c) % n;
            y = (mulmod(y, y, n) + c) % n;
            y = (mulmod(y, y, n) + c) % n;
            d = gcd64(x > y ? x - y : y - x, n);
        }
        if (d != n) return d;
    }
}

void distinct_prime_factors(uint64_t n, uint64_t *out, int *count) {
    if (n == 1) return;
    if (is_prime(n)) {
        for (int i = 0; i < *count; ++i)
            if (out[i] == n) return;
        out[(*count)++] = n;
        return;
    }
    for (uint64_t p = 2; p < 1024; ++p) {
        if (n % p == 0) {
            distinct_prime_factors(p, out, count);
            while (n % p == 0) n /= p;
            distinct_prime_factors(n, out, count);
            return;
        }
    }
    const uint64_t d = rho_factor(n);
    distinct_prime_factors(d, out, count);
    distinct_prime_factors(n / d, out, count);
}
}  // namespace

uint64_t smallest_generator(uint64_t q) {
    if (q < 3) return q == 2 ? 1 : 0;
    uint64_t fs[64];
    int nf = 0;
    distinct_prime_factors(q - 1, fs, &nf);
    for (uint64_t g = 2; g < q; ++g) {
        bool ok = true;
        for (int i = 0; i < nf && ok; ++i)
            if (powmod(g, (q - 1) / fs[i], q) == 1) ok = false;
        if (ok) return g;
    }
    return 0;
}

}  // namespace bc
