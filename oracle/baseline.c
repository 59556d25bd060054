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
    default: orc_exact_negacyclic_ntt(src, dst, j->degree, q, r); break;
    }
}

static void *worker(void *arg) {
    job_t *j = (job_t *)arg;
    for (;;) {
        pthread_mutex_lock(&j->lock);
        uint32_t p = j->next++;
        pthread_mutex_unlock(&j->lock);
        if (p >= j->count) break;
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
