/*
 * TEST INFRASTRUCTURE ONLY -- multi-threaded CPU runner used by the tests
 * (large-batch oracle checks) and by bench.py's CPU-baseline legs.  It calls
 * a per-sample extractor -- the restated oracle, or the reference's own
 * tb_train_extract_features_cpu from oracle/_ref -- over contiguous sample
 * ranges, one POSIX thread per range.  The reference function is reentrant
 * (no globals; training.c:102-142), so this is the natural way to use all
 * host cores with it.
 */
#define _POSIX_C_SOURCE 199309L
#include <pthread.h>
#include <stdlib.h>
#include <time.h>

#include "features_oracle.h"

typedef struct {
    oracle_sample_fn fn;
    const float *obs, *mission;
    const uint8_t *cameras;
    float *out;
    size_t begin, end;
} oracle_range;

static void *oracle_range_main(void *arg) {
    const oracle_range *r = (const oracle_range *)arg;
    for (size_t i = r->begin; i < r->end; ++i)
        r->fn(r->obs + i * ORACLE_OBS_DIM, r->mission + i * ORACLE_MISSION_DIM,
              r->cameras ? r->cameras + i * ORACLE_CAMERA_BYTES : NULL,
              r->out + i * ORACLE_FEATURE_DIM);
    return NULL;
}

static double oracle_now(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

double oracle_extract_batch(oracle_sample_fn fn, const float *obs, const float *mission,
                            const uint8_t *cameras, size_t count, float *out, int threads) {
    if (!fn || !obs || !mission || !out) return -1.0;
    if (threads < 1) threads = 1;
    if ((size_t)threads > count && count > 0) threads = (int)count;
    oracle_range *ranges = (oracle_range *)calloc((size_t)threads, sizeof(*ranges));
    pthread_t *tids = (pthread_t *)calloc((size_t)threads, sizeof(*tids));
    if (!ranges || !tids) { free(ranges); free(tids); return -1.0; }
    const double t0 = oracle_now();
    int started = 0, failed = 0;
    for (int t = 0; t < threads; ++t) {
        ranges[t] = (oracle_range){fn, obs, mission, cameras, out,
                                   count * (size_t)t / (size_t)threads,
                                   count * (size_t)(t + 1) / (size_t)threads};
        if (t == threads - 1) break; /* the calling thread runs the last range */
        if (pthread_create(&tids[t], NULL, oracle_range_main, &ranges[t]) != 0) { failed = 1; break; }
        ++started;
    }
    if (!failed) oracle_range_main(&ranges[threads - 1]);
    for (int t = 0; t < started; ++t) pthread_join(tids[t], NULL);
    const double elapsed = oracle_now() - t0;
    free(ranges);
    free(tids);
    return failed ? -1.0 : elapsed;
}

double oracle_extract_batch_self(const float *obs, const float *mission,
                                 const uint8_t *cameras, size_t count, float *out,
                                 int threads) {
    return oracle_extract_batch(oracle_extract_features, obs, mission, cameras, count, out,
                                threads);
}

typedef struct {
    oracle_onboard_fn fn;
    const float *obs, *mission;
    float *out;
    size_t begin, end;
} onboard_range;

static void *onboard_range_main(void *arg) {
    const onboard_range *r = (const onboard_range *)arg;
    for (size_t i = r->begin; i < r->end; ++i)
        r->fn(r->obs + i * ORACLE_OBS_DIM, r->mission + i * ORACLE_MISSION_DIM, r->out + i * 39,
              r->out + i * 39 + 24);
    return NULL;
}

double oracle_onboard_batch(oracle_onboard_fn fn, const float *obs, const float *mission,
                            size_t count, float *out_39, int threads) {
    if (!fn || !obs || !mission || !out_39) return -1.0;
    if (threads < 1) threads = 1;
    if ((size_t)threads > count && count > 0) threads = (int)count;
    onboard_range *ranges = (onboard_range *)calloc((size_t)threads, sizeof(*ranges));
    pthread_t *tids = (pthread_t *)calloc((size_t)threads, sizeof(*tids));
    if (!ranges || !tids) { free(ranges); free(tids); return -1.0; }
    const double t0 = oracle_now();
    int started = 0, failed = 0;
    for (int t = 0; t < threads; ++t) {
        ranges[t] = (onboard_range){fn, obs, mission, out_39, count * (size_t)t / (size_t)threads,
                                    count * (size_t)(t + 1) / (size_t)threads};
        if (t == threads - 1) break;
        if (pthread_create(&tids[t], NULL, onboard_range_main, &ranges[t]) != 0) { failed = 1; break; }
        ++started;
    }
    if (!failed) onboard_range_main(&ranges[threads - 1]);
    for (int t = 0; t < started; ++t) pthread_join(tids[t], NULL);
    const double elapsed = oracle_now() - t0;
    free(ranges);
    free(tids);
    return failed ? -1.0 : elapsed;
}
