/*
 * workload.c -- deterministic synthetic logits for the five sampler workloads.
 *
 * The sampler's input is Qwen2.5-0.5B lm_head logits, [rows][151936] f32.  No
 * model or dataset is available, so rows are drawn from seeded laws that stand
 * in for them.  Each row has its own counter-seeded stream, so any subset of
 * rows can be regenerated on its own and every consumer (GPU tests, the CPU
 * baselines, the bench) reads byte-identical data:
 *
 *   stream(cfg, seed, row, sub) = splitmix64 seeded by mix(mix(mix(cfg)^seed)^row)^sub
 *   normal                      = Box-Muller in double on two 53-bit uniforms
 *
 *   1  N(0, 2.0^2); 16 distinct peak ids set to 8 + 4j/15 (j = 0..15)
 *   2  N(0, 2.5^2) + row offset U(-1, 1); 8 peak ids set to 6 + 4j/7 + offset
 *   3  -1.1 * log(rank + 1) + N(0, 0.3^2), rank = seeded permutation of 0..V-1
 *   4  round(8 * N(0, 1.5^2)) / 8  (multiples of 0.125: heavy ties)
 *   5  as 2 (the 4096-row batch)
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static inline uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

typedef struct { uint64_t s; } zw_stream;

static inline uint64_t zw_next(zw_stream* st) {
    st->s += 0x9E3779B97F4A7C15ull;
    return mix64(st->s);
}

static inline double zw_u01(zw_stream* st) { /* [0, 1) */
    return (double)(zw_next(st) >> 11) * (1.0 / 9007199254740992.0);
}

static inline zw_stream zw_make(int cfg, uint64_t seed, int64_t row, uint64_t sub) {
    zw_stream st;
    st.s = mix64(mix64(mix64((uint64_t)cfg + 0x51ull) ^ seed) ^ (uint64_t)row) ^ sub;
    return st;
}

/* Fills out[0..n) with N(0,1) samples (pairs from Box-Muller). */
static void zw_normals(zw_stream* st, double* out, int n) {
    const double two_pi = 6.283185307179586476925286766559;
    for (int i = 0; i < n; i += 2) {
        double u1 = 1.0 - zw_u01(st); /* (0, 1] */
        double u2 = zw_u01(st);
        double r = sqrt(-2.0 * log(u1));
        out[i] = r * cos(two_pi * u2);
        if (i + 1 < n) out[i + 1] = r * sin(two_pi * u2);
    }
}

static inline uint32_t zw_bounded(zw_stream* st, uint32_t range) {
    return (uint32_t)(((unsigned __int128)zw_next(st) * range) >> 64);
}

static void zw_row(int cfg, uint64_t seed, int64_t row, int V, float* out, double* tmp,
                   uint32_t* perm) {
    zw_stream st = zw_make(cfg, seed, row, 0);
    zw_stream aux = zw_make(cfg, seed, row, 1);
    zw_normals(&st, tmp, V);
    if (cfg == 1) {
        for (int i = 0; i < V; ++i) out[i] = (float)(2.0 * tmp[i]);
        int npk = V < 16 ? V : 16;
        int ids[16];
        for (int j = 0; j < npk; ++j) {
            int id, dup;
            do {
                id = (int)zw_bounded(&aux, (uint32_t)V);
                dup = 0;
                for (int q = 0; q < j; ++q) dup |= (ids[q] == id);
            } while (dup);
            ids[j] = id;
            out[id] = (float)(8.0 + 4.0 * j / 15.0);
        }
    } else if (cfg == 2 || cfg == 5) {
        double off = 2.0 * zw_u01(&aux) - 1.0;
        for (int i = 0; i < V; ++i) out[i] = (float)(2.5 * tmp[i] + off);
        int npk = V < 8 ? V : 8;
        int ids[8];
        for (int j = 0; j < npk; ++j) {
            int id, dup;
            do {
                id = (int)zw_bounded(&aux, (uint32_t)V);
                dup = 0;
                for (int q = 0; q < j; ++q) dup |= (ids[q] == id);
            } while (dup);
            ids[j] = id;
            out[id] = (float)(6.0 + 4.0 * j / 7.0 + off);
        }
    } else if (cfg == 3) {
        for (int i = 0; i < V; ++i) perm[i] = (uint32_t)i;
        for (int i = V - 1; i > 0; --i) {
            uint32_t j = zw_bounded(&aux, (uint32_t)i + 1u);
            uint32_t t = perm[i];
            perm[i] = perm[j];
            perm[j] = t;
        }
        for (int i = 0; i < V; ++i)
            out[i] = (float)(-1.1 * log((double)perm[i] + 1.0) + 0.3 * tmp[i]);
    } else { /* cfg 4 */
        for (int i = 0; i < V; ++i) out[i] = (float)(round(8.0 * 1.5 * tmp[i]) / 8.0);
    }
}

typedef struct {
    int cfg;
    uint64_t seed;
    int64_t row0;
    int nrows, V;
    float* out;
    int64_t ld;
    int next;
    pthread_mutex_t mu;
} zw_job;

static void* zw_worker(void* arg) {
    zw_job* j = (zw_job*)arg;
    double* tmp = (double*)malloc(sizeof(double) * (size_t)(j->V + 2));
    uint32_t* perm = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)(j->V + 1));
    for (;;) {
        pthread_mutex_lock(&j->mu);
        int r = j->next++;
        pthread_mutex_unlock(&j->mu);
        if (r >= j->nrows) break;
        zw_row(j->cfg, j->seed, j->row0 + r, j->V, j->out + (int64_t)r * j->ld, tmp, perm);
    }
    free(tmp);
    free(perm);
    return NULL;
}

/* Rows row0 .. row0+nrows-1 of workload `cfg` into out (row stride ld floats). */
int zw_generate(int cfg, uint64_t seed, int64_t row0, int nrows, int V, float* out, int64_t ld,
                int nthreads) {
    if (cfg < 1 || cfg > 5 || V <= 0 || nrows < 0 || ld < V) return -1;
    zw_job j;
    j.cfg = cfg;
    j.seed = seed;
    j.row0 = row0;
    j.nrows = nrows;
    j.V = V;
    j.out = out;
    j.ld = ld;
    j.next = 0;
    pthread_mutex_init(&j.mu, NULL);
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    pthread_t th[256];
    for (int t = 1; t < nthreads; ++t) pthread_create(&th[t], NULL, zw_worker, &j);
    zw_worker(&j);
    for (int t = 1; t < nthreads; ++t) pthread_join(th[t], NULL);
    pthread_mutex_destroy(&j.mu);
    return 0;
}
