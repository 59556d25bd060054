// op_latency.cpp -- single-call latency of the reference op API through the
// C ABI (what a Rust or C caller of libbarracuda_fhe.so sees), at N = 4096
// with the largest prime q < 2^31, q = 1 mod 2N.  Each op writes into a
// preallocated output, as FheNtt::execute's caller would after the output
// allocation; the allocation itself is timed separately.  Prints one JSON
// line: median, 10th and 90th percentile microseconds over `calls` calls
// after 20 warm-up calls.  Run by `python bench.py --op-latency`.
//
//     bc_op_latency [calls]
#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

#include "barracuda_fhe.h"

namespace {

struct Stat {
    double p10, p50, p90;
};

template <class F>
bool measure(int calls, F fn, Stat *out) {
    for (int i = 0; i < 20; ++i)
        if (fn()) return false;
    std::vector<double> t;
    t.reserve(calls);
    for (int i = 0; i < calls; ++i) {
        const auto t0 = std::chrono::steady_clock::now();
        const int st = fn();
        const auto t1 = std::chrono::steady_clock::now();
        if (st) return false;
        t.push_back(std::chrono::duration<double, std::micro>(t1 - t0).count());
    }
    std::sort(t.begin(), t.end());
    *out = {t[calls / 10], t[calls / 2], t[(calls * 9) / 10]};
    return true;
}

}  // namespace

int main(int argc, char **argv) {
    const int calls = argc > 1 ? std::max(10, std::atoi(argv[1])) : 200;
    bc_ctx *ctx = nullptr;
    if (bc_ctx_create(0, &ctx)) {
        std::fprintf(stderr, "bc_ctx_create: %s\n", bc_last_error());
        return 1;
    }
    const uint32_t n = 4096;
    const uint64_t q = bc_ntt_prime(31, n, 0);
    const uint64_t psi = bc_negacyclic_root(q, n);
    const uint64_t w = static_cast<uint64_t>(static_cast<unsigned __int128>(psi) * psi % q);
    const uint64_t winv = bc_compute_inverse_root(n, q, w);
    std::vector<uint64_t> host(n);
    for (uint32_t i = 0; i < n; ++i) host[i] = (i * 2654435761ull + 12345) % q;
    void *a = nullptr, *b = nullptr, *o = nullptr;
    if (bc_buf_alloc(ctx, 8 * n, &a) || bc_buf_alloc(ctx, 8 * n, &b) || bc_buf_alloc(ctx, 8 * n, &o) ||
        bc_buf_h2d(ctx, a, host.data(), 8 * n) || bc_buf_h2d(ctx, b, host.data(), 8 * n)) {
        std::fprintf(stderr, "buffers: %s\n", bc_last_error());
        return 1;
    }
    auto *da = static_cast<uint64_t *>(a), *db = static_cast<uint64_t *>(b), *dout = static_cast<uint64_t *>(o);
    struct Op {
        const char *name;
        int (*run)(bc_ctx *, uint64_t *, uint64_t *, uint64_t *, uint32_t, uint64_t, uint64_t, uint64_t);
    };
    const Op ops[] = {
        {"FheNtt", [](bc_ctx *c, uint64_t *x, uint64_t *, uint64_t *y, uint32_t n, uint64_t q, uint64_t w, uint64_t) {
             return bc_fhe_ntt(c, x, 2 * n, n, q, w, y);
         }},
        {"FheIntt", [](bc_ctx *c, uint64_t *x, uint64_t *, uint64_t *y, uint32_t n, uint64_t q, uint64_t, uint64_t wi) {
             return bc_fhe_intt(c, x, 2 * n, n, q, wi, y);
         }},
        {"FhePointwiseMul", [](bc_ctx *c, uint64_t *x, uint64_t *z, uint64_t *y, uint32_t n, uint64_t q, uint64_t, uint64_t) {
             return bc_fhe_pointwise_mul(c, x, 2 * n, z, 2 * n, n, q, y);
         }},
        {"FheFastPolyMul", [](bc_ctx *c, uint64_t *x, uint64_t *z, uint64_t *y, uint32_t n, uint64_t q, uint64_t w, uint64_t) {
             return bc_fhe_fast_poly_mul(c, x, 2 * n, z, 2 * n, n, q, w, y);
         }},
    };
    std::string json = "{\"c_abi_latency\": true, \"N\": 4096, \"q_bits\": 31, \"calls\": " + std::to_string(calls) +
                       ", \"timing\": \"steady_clock per synchronous call, preallocated output\", \"ops_us\": {";
    char buf[256];
    bool first = true;
    for (const Op &op : ops) {
        Stat s;
        if (!measure(calls, [&] { return op.run(ctx, da, db, dout, n, q, w, winv); }, &s)) {
            std::fprintf(stderr, "%s: %s\n", op.name, bc_last_error());
            return 1;
        }
        std::snprintf(buf, sizeof buf, "%s\"%s\": {\"p50\": %.2f, \"p10\": %.2f, \"p90\": %.2f}", first ? "" : ", ",
                      op.name, s.p50, s.p10, s.p90);
        json += buf;
        first = false;
    }
    Stat sy, al;
    if (!measure(calls, [&] { return bc_ctx_sync(ctx); }, &sy) ||
        !measure(calls, [&] {
            void *p = nullptr;
            const int st = bc_buf_alloc(ctx, 8 * n, &p);
            return st ? st : bc_buf_free(ctx, p);
        }, &al)) {
        std::fprintf(stderr, "sync/alloc: %s\n", bc_last_error());
        return 1;
    }
    std::snprintf(buf, sizeof buf,
                  "}, \"ctx_sync_idle_us\": %.2f, \"output_alloc_and_free_us\": %.2f}", sy.p50, al.p50);
    json += buf;
    std::printf("%s\n", json.c_str());
    bc_buf_free(ctx, a);
    bc_buf_free(ctx, b);
    bc_buf_free(ctx, o);
    bc_ctx_destroy(ctx);
    return 0;
}
