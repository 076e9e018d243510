/*
 * libm_check.c — test helper: compares spindle_b200/csrc/glibc_math.h (the
 * restatement of glibc's expf / sinf / cosf that the kernels use) with the
 * host's glibc, and checks buffers of device results against glibc.
 * TEST INFRASTRUCTURE ONLY: built by tests/test_libm.py with
 * gcc -O2 -mfma -ffp-contract=off (so every operation of the header is the
 * single rounding it names) and loaded through ctypes.
 *
 * fn: 0 = expf, 1 = sinf, 2 = cosf.  Two results agree when their bits are
 * equal or both are NaN.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <string.h>

#include "../spindle_b200/csrc/glibc_math.h"

static float from_bits(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t to_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

static float host_fn(int fn, float x) {
    volatile float v = x; /* keep the compiler from folding or vectorising the libm call */
    return fn == 0 ? expf(v) : fn == 1 ? sinf(v) : cosf(v);
}
static float mine_fn(int fn, float x) { return fn == 0 ? gm_expf(x) : fn == 1 ? gm_sinf(x) : gm_cosf(x); }

static int same(float a, float b) { return to_bits(a) == to_bits(b) || (isnan(a) && isnan(b)); }

typedef struct {
    int fn;
    uint64_t lo, hi; /* bit patterns [lo, hi) */
    uint64_t bad;
    uint32_t first_bad;
} job_t;

static void *run_job(void *p) {
    job_t *j = (job_t *)p;
    j->bad = 0;
    for (uint64_t u = j->lo; u < j->hi; u++) {
        const float x = from_bits((uint32_t)u);
        if (!same(host_fn(j->fn, x), mine_fn(j->fn, x))) {
            if (!j->bad) j->first_bad = (uint32_t)u;
            j->bad++;
        }
    }
    return NULL;
}

/* Number of bit patterns in [start, start + count) where the header and glibc
   differ; *first_bad receives the first such pattern. */
uint64_t lm_count_mismatch(int fn, uint64_t start, uint64_t count, int nthreads, uint32_t *first_bad) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    pthread_t th[256];
    job_t jobs[256];
    for (int t = 0; t < nthreads; t++) {
        jobs[t].fn = fn;
        jobs[t].lo = start + count * (uint64_t)t / (uint64_t)nthreads;
        jobs[t].hi = start + count * (uint64_t)(t + 1) / (uint64_t)nthreads;
        pthread_create(&th[t], NULL, run_job, &jobs[t]);
    }
    uint64_t bad = 0;
    uint32_t first = 0;
    for (int t = 0; t < nthreads; t++) {
        pthread_join(th[t], NULL);
        if (jobs[t].bad && !bad) first = jobs[t].first_bad;
        bad += jobs[t].bad;
    }
    if (first_bad) *first_bad = first;
    return bad;
}

typedef struct {
    int fn;
    uint64_t start, stride, lo, hi; /* entries [lo, hi) */
    const float *got;
    uint64_t bad;
    uint32_t first_bad;
} cmp_t;

static void *run_cmp(void *p) {
    cmp_t *j = (cmp_t *)p;
    j->bad = 0;
    for (uint64_t i = j->lo; i < j->hi; i++) {
        const uint32_t u = (uint32_t)(j->start + i * j->stride);
        if (!same(host_fn(j->fn, from_bits(u)), j->got[i])) {
            if (!j->bad) j->first_bad = u;
            j->bad++;
        }
    }
    return NULL;
}

/* got[i] holds f(bits start + i * stride) computed elsewhere (the GPU); the
   number of entries that differ from glibc, split over nthreads threads. */
uint64_t lm_compare_strided(int fn, uint64_t start, uint64_t stride, uint64_t count, const float *got,
                            int nthreads, uint32_t *first_bad) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    pthread_t th[256];
    cmp_t jobs[256];
    for (int t = 0; t < nthreads; t++) {
        cmp_t *j = &jobs[t];
        j->fn = fn;
        j->start = start;
        j->stride = stride;
        j->lo = count * (uint64_t)t / (uint64_t)nthreads;
        j->hi = count * (uint64_t)(t + 1) / (uint64_t)nthreads;
        j->got = got;
        pthread_create(&th[t], NULL, run_cmp, j);
    }
    uint64_t bad = 0;
    uint32_t first = 0;
    for (int t = 0; t < nthreads; t++) {
        pthread_join(th[t], NULL);
        if (jobs[t].bad && !bad) first = jobs[t].first_bad;
        bad += jobs[t].bad;
    }
    if (first_bad) *first_bad = first;
    return bad;
}

float lm_host(int fn, float x) { return host_fn(fn, x); }
float lm_mine(int fn, float x) { return mine_fn(fn, x); }
