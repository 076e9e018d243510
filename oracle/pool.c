/*
 * pool.c — the reference's persistent worker pool and row split, used to time
 * the CPU baseline.  TEST INFRASTRUCTURE ONLY (see sg_oracle.h).
 *
 * worker_pool.rs:38-139: thread 0 is the caller, helpers spin on a generation
 * counter (200k polls) before parking; a `remaining` countdown ends the job.
 * smollm_chat.rs:309-349 / :447-512: the activation is quantized once on the
 * caller, then thread t of T runs rows [R*t/T, R*(t+1)/T) when the matrix has
 * at least 16K weights (PAR_MIN_WEIGHTS, :306).
 */
#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>

#include "sg_oracle.h"

#define SPIN_BEFORE_PARK 200000
#define PAR_MIN_WEIGHTS (16 * 1024)
#define MAX_THREADS 256

typedef void (*job_fn)(void *arg, int t, int n);

static struct {
    int n;
    pthread_t tid[MAX_THREADS];
    atomic_ulong generation;
    atomic_int remaining;
    atomic_int stop;
    job_fn fn;
    void *arg;
    pthread_mutex_t mu;
    pthread_cond_t cv;
} P = {.n = 0};

static void *worker(void *p)
{
    int t = (int)(intptr_t)p;
    unsigned long seen = 0;
    for (;;) {
        unsigned long g;
        int spins = 0;
        while ((g = atomic_load_explicit(&P.generation, memory_order_acquire)) == seen) {
            if (atomic_load(&P.stop)) return NULL;
            if (++spins >= SPIN_BEFORE_PARK) {
                pthread_mutex_lock(&P.mu);
                while (atomic_load(&P.generation) == seen && !atomic_load(&P.stop))
                    pthread_cond_wait(&P.cv, &P.mu);
                pthread_mutex_unlock(&P.mu);
                spins = 0;
            }
        }
        if (atomic_load(&P.stop)) return NULL;
        seen = g;
        P.fn(P.arg, t, P.n);
        atomic_fetch_sub_explicit(&P.remaining, 1, memory_order_acq_rel);
    }
}

int or_pool_create(int n)
{
    if (P.n) or_pool_destroy();
    if (n < 1) n = 1;
    if (n > MAX_THREADS) n = MAX_THREADS;
    atomic_store(&P.generation, 0);
    atomic_store(&P.stop, 0);
    pthread_mutex_init(&P.mu, NULL);
    pthread_cond_init(&P.cv, NULL);
    P.n = n;
    for (int t = 1; t < n; t++)
        if (pthread_create(&P.tid[t], NULL, worker, (void *)(intptr_t)t)) { P.n = t; break; }
    return P.n;
}

void or_pool_destroy(void)
{
    if (!P.n) return;
    atomic_store(&P.stop, 1);
    pthread_mutex_lock(&P.mu);
    pthread_cond_broadcast(&P.cv);
    pthread_mutex_unlock(&P.mu);
    for (int t = 1; t < P.n; t++) pthread_join(P.tid[t], NULL);
    pthread_mutex_destroy(&P.mu);
    pthread_cond_destroy(&P.cv);
    P.n = 0;
}

int or_pool_threads(void) { return P.n ? P.n : 1; }

/* WorkerPool::run: every thread (the caller as thread 0) runs fn(arg, t, n). */
static void pool_run(job_fn fn, void *arg)
{
    if (P.n <= 1) { fn(arg, 0, 1); return; }
    P.fn = fn;
    P.arg = arg;
    atomic_store(&P.remaining, P.n - 1);
    pthread_mutex_lock(&P.mu);
    atomic_fetch_add_explicit(&P.generation, 1, memory_order_release);
    pthread_cond_broadcast(&P.cv);
    pthread_mutex_unlock(&P.mu);
    fn(arg, 0, P.n);
    while (atomic_load_explicit(&P.remaining, memory_order_acquire) > 0) { }
}

typedef struct {
    const uint8_t *base;
    const or_mat *m;
    size_t n_vec;
    const float *const *xd;
    const int8_t *const *xs;
    const int16_t *const *xb;
    const float *const *xf;
    float *const *outs;
    int use_int;
} mv_job;

static void mv_rows(void *p, int t, int n)
{
    mv_job *j = (mv_job *)p;
    size_t rows = j->m->rows;
    size_t r0 = rows * (size_t)t / (size_t)n, r1 = rows * (size_t)(t + 1) / (size_t)n;
    if (r1 <= r0) return;
    if (j->use_int)
        or_matmul_rows(j->base, j->m, j->n_vec, j->xd, j->xs, j->xb, j->outs, r0, r1);
    else if (j->m->dtype == OR_F32) /* routers: one vector at a time (smollm_chat.rs:455-463) */
        for (size_t b = 0; b < j->n_vec; b++) or_matvec_rows(j->base, j->m, j->xf[b], j->outs[b] + r0, r0, r1 - r0);
    else
        or_matmul_rows_multi(j->base, j->m, j->n_vec, j->xf, j->outs, r0, r1);
}

/* matvec / matvec_multi (smollm_chat.rs:309-349, :447-512) on this pool. */
int or_pool_matvec_multi(const uint8_t *base, const or_mat *m, size_t n_vec, const float *xs, float *outs)
{
    if (n_vec == 0) return 0;
    size_t cols = m->cols, rows = m->rows;
    int use_int = (m->dtype == OR_Q4_K || m->dtype == OR_Q6_K) && cols && cols % 256 == 0;
    size_t nb = cols / 256;
    float *qd = NULL;
    int8_t *qs = NULL;
    int16_t *qb = NULL;
    const float **xd = calloc(n_vec, sizeof *xd);
    const int8_t **xq = calloc(n_vec, sizeof *xq);
    const int16_t **xb = calloc(n_vec, sizeof *xb);
    const float **xf = calloc(n_vec, sizeof *xf);
    float **op = calloc(n_vec, sizeof *op);
    int rc = 0;
    if (!xd || !xq || !xb || !xf || !op) { rc = -2; goto out; }
    if (use_int) {
        qd = malloc(n_vec * nb * sizeof(float));
        qs = malloc(n_vec * cols);
        qb = malloc(n_vec * nb * 16 * sizeof(int16_t));
        if (!qd || !qs || !qb) { rc = -2; goto out; }
    }
    for (size_t b = 0; b < n_vec; b++) {
        xf[b] = xs + b * cols;
        op[b] = outs + b * rows;
        if (use_int) {
            or_q8k_quantize(xs + b * cols, cols, qd + b * nb, qs + b * cols, qb + b * nb * 16);
            xd[b] = qd + b * nb;
            xq[b] = qs + b * cols;
            xb[b] = qb + b * nb * 16;
        }
    }
    mv_job j = {base, m, n_vec, xd, xq, xb, xf, op, use_int};
    if (rows * cols >= PAR_MIN_WEIGHTS) pool_run(mv_rows, &j);
    else mv_rows(&j, 0, 1);
out:
    free(qd); free(qs); free(qb);
    free(xd); free(xq); free(xb); free(xf); free(op);
    return rc;
}
