/*
 * baseline.c -- threaded driver that times the reference restatement on the
 * host cores (the CPU baseline reported beside the GPU numbers).
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h).
 */
#include "oracle.h"

#include <pthread.h>
#include <stdlib.h>
#include <time.h>

typedef struct {
    int kind;
    const uint64_t *in;
    uint64_t *out;
    uint32_t degree, count, n_moduli;
    const uint64_t *moduli, *roots;
    const uint64_t *in2; /* second operand of the polynomial products */
    uint32_t next; /* shared work counter, guarded by lock */
    pthread_mutex_t lock;
} job_t;

static void run_one(const job_t *j, uint32_t p) {
    const uint64_t *src = j->in + (size_t)p * j->degree;
    uint64_t *dst = j->out + (size_t)p * j->degree;
    uint64_t q = j->moduli[p % j->n_moduli], r = j->roots[p % j->n_moduli];
    switch (j->kind) {
    case 0: orc_ref_ntt(src, dst, j->degree, q, r); break;
    case 1: orc_ref_intt(src, dst, j->degree, q, r); break;
    case 2: orc_ref_negacyclic_ntt(src, dst, j->degree, q, r); break;
    case 3: orc_ref_negacyclic_intt(src, dst, j->degree, q, r); break;
    case 5: orc_exact_negacyclic_intt(src, dst, j->degree, q, r); break;
    default: orc_exact_negacyclic_ntt(src, dst, j->degree, q, r); break;
    }
}

/* c = a * b of one limb-polynomial pair: kind 0 the reference's cyclic
 * FheFastPolyMul chain (fhe_fast_poly_mul.rs:122-154), 1 the reference ops
 * chained for a negacyclic product (psi twist, NTT, pointwise, INTT), 2 the
 * exact negacyclic product, 3 the exact cyclic product (exact transforms). */
static void run_product(const job_t *j, uint32_t p) {
    const size_t o = (size_t)p * j->degree;
    const uint64_t *a = j->in + o, *b = j->in2 + o;
    uint64_t *c = j->out + o;
    const uint32_t n = j->degree;
    uint64_t q = j->moduli[p % j->n_moduli], r = j->roots[p % j->n_moduli];
    if (j->kind == 0) {
        orc_ref_fast_poly_mul(a, b, c, n, q, r);
        return;
    }
    uint64_t *fa = (uint64_t *)malloc(sizeof(uint64_t) * n), *fb = (uint64_t *)malloc(sizeof(uint64_t) * n);
    if (j->kind == 1) {
        orc_ref_negacyclic_ntt(a, fa, n, q, r);
        orc_ref_negacyclic_ntt(b, fb, n, q, r);
        orc_ref_pointwise(fa, fb, fa, n, q);
        orc_ref_negacyclic_intt(fa, c, n, q, r);
    } else if (j->kind == 2) {
        orc_exact_negacyclic_ntt(a, fa, n, q, r);
        orc_exact_negacyclic_ntt(b, fb, n, q, r);
        for (uint32_t i = 0; i < n; ++i) fa[i] = orc_mulmod(fa[i], fb[i], q);
        orc_exact_negacyclic_intt(fa, c, n, q, r);
    } else {
        orc_exact_ntt(a, fa, n, q, r);
        orc_exact_ntt(b, fb, n, q, r);
        for (uint32_t i = 0; i < n; ++i) fa[i] = orc_mulmod(fa[i], fb[i], q);
        const uint64_t rinv = orc_powmod(r, q - 2, q), ninv = orc_powmod(n % q, q - 2, q);
        orc_exact_ntt(fa, c, n, q, rinv);
        for (uint32_t i = 0; i < n; ++i) c[i] = orc_mulmod(c[i], ninv, q);
    }
    free(fa);
    free(fb);
}

static void *worker(void *arg) {
    job_t *j = (job_t *)arg;
    for (;;) {
        pthread_mutex_lock(&j->lock);
        uint32_t p = j->next++;
        pthread_mutex_unlock(&j->lock);
        if (p >= j->count) break;
        if (j->in2)
            run_product(j, p);
        else
            run_one(j, p);
    }
    return NULL;
}

double orc_baseline_run(int kind, const uint64_t *in, uint64_t *out, uint32_t degree,
                        uint32_t count, const uint64_t *moduli, const uint64_t *roots,
                        uint32_t n_moduli, int threads) {
    job_t j;
    j.kind = kind;
    j.in = in;
    j.in2 = NULL;
    j.out = out;
    j.degree = degree;
    j.count = count;
    j.moduli = moduli;
    j.roots = roots;
    j.n_moduli = n_moduli ? n_moduli : 1;
    j.next = 0;
    pthread_mutex_init(&j.lock, NULL);
    if (threads < 1) threads = 1;
    pthread_t *tids = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)threads);
    struct timespec t0, t1;
    clock_gettime(CLOCK_MONOTONIC, &t0);
    for (int t = 0; t < threads; ++t) pthread_create(&tids[t], NULL, worker, &j);
    for (int t = 0; t < threads; ++t) pthread_join(tids[t], NULL);
    clock_gettime(CLOCK_MONOTONIC, &t1);
    free(tids);
    pthread_mutex_destroy(&j.lock);
    return (double)(t1.tv_sec - t0.tv_sec) + 1e-9 * (double)(t1.tv_nsec - t0.tv_nsec);
}

double orc_batch_polymul(int kind, const uint64_t *a, const uint64_t *b, uint64_t *c, uint32_t degree,
                         uint32_t count, const uint64_t *moduli, const uint64_t *roots, uint32_t n_moduli,
                         int threads) {
    job_t j;
    j.kind = kind;
    j.in = a;
    j.in2 = b;
    j.out = c;
    j.degree = degree;
    j.count = count;
    j.moduli = moduli;
    j.roots = roots;
    j.n_moduli = n_moduli ? n_moduli : 1;
    j.next = 0;
    pthread_mutex_init(&j.lock, NULL);
    if (threads < 1) threads = 1;
    pthread_t *tids = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)threads);
    struct timespec t0, t1;
    clock_gettime(CLOCK_MONOTONIC, &t0);
    for (int t = 0; t < threads; ++t) pthread_create(&tids[t], NULL, worker, &j);
    for (int t = 0; t < threads; ++t) pthread_join(tids[t], NULL);
    clock_gettime(CLOCK_MONOTONIC, &t1);
    free(tids);
    pthread_mutex_destroy(&j.lock);
    return (double)(t1.tv_sec - t0.tv_sec) + 1e-9 * (double)(t1.tv_nsec - t0.tv_nsec);
}
