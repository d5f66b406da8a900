/* Seeded synthetic sensor batches; see tb_synth.h for the value model. */
#define _GNU_SOURCE
#include "tb_synth.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <unistd.h>

enum { OBS_DIM = 4148, MISSION_DIM = 10, CAMERA_BYTES = 16384, LIDAR_OFFSET = 48,
       LIDAR_BINS = 4096, TAIL_OFFSET = 4144 };

/* SplitMix64 (Steele, Lea & Flood, OOPSLA 2014): a Weyl sequence passed
 * through a 64-bit finaliser. */
static uint64_t synth_next(uint64_t *state) {
    uint64_t z = (*state += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* Uniform in [0, 1) with 24 random bits. */
static float synth_unit(uint64_t *state) {
    return (float)(synth_next(state) >> 40) * (1.0f / 16777216.0f);
}

static float synth_signed(uint64_t *state) {
    return 2.0f * synth_unit(state) - 1.0f;
}

uint8_t tb_synth_quantize(float v) {
    /* The simulator's rule in double: fmax(0, fmin(255, round(v * 255))). */
    return (uint8_t)fmax(0.0, fmin(255.0, round((double)v * 255.0)));
}

static void synth_sample(uint64_t seed, uint64_t index, int mode, float *o, float *m,
                         uint8_t *cam8, float *camf) {
    /* Independent stream per (seed, sample). */
    uint64_t key = seed * 0xD1B54A32D192ED03ull ^ (index + 1) * 0x9E3779B97F4A7C15ull;
    uint64_t st = synth_next(&key);

    for (int i = 0; i < LIDAR_OFFSET; ++i) o[i] = synth_signed(&st);
    for (int i = 0; i < 4; ++i) o[TAIL_OFFSET + i] = synth_signed(&st);
    for (int i = 0; i < MISSION_DIM; ++i) m[i] = synth_signed(&st);

    float *lidar = o + LIDAR_OFFSET;
    if (mode == TB_SYNTH_LIDAR_NORETURN) {
        for (int b = 0; b < LIDAR_BINS; ++b) lidar[b] = 300.0f;
    } else if (mode == TB_SYNTH_LIDAR_HALF) {
        for (int b = 0; b < LIDAR_BINS; ++b) lidar[b] = 0.5f;
    } else {
        const double log600 = log(600.0);
        for (int b = 0; b < LIDAR_BINS; ++b) {
            const uint64_t z = synth_next(&st);
            const double p = (double)(z & 0xFFFFFFu) * (1.0 / 16777216.0);
            const double u = (double)(z >> 40) * (1.0 / 16777216.0);
            lidar[b] = p < 0.05 ? 300.0f : (float)(0.5 * exp(u * log600));
        }
        if (mode == TB_SYNTH_LIDAR_DUPMIN) {
            /* Repeat each sector's minimum range in two further bins. */
            for (int sector = 0; sector < 64; ++sector) {
                const int head = sector >> 5, el_sector = (sector >> 3) & 3, az_sector = sector & 7;
                float *base = lidar + head * 2048 + el_sector * 512 + az_sector * 16;
                int best = 0;
                for (int k = 1; k < 64; ++k)
                    if (base[(k >> 4) * 128 + (k & 15)] < base[(best >> 4) * 128 + (best & 15)]) best = k;
                const float lo = base[(best >> 4) * 128 + (best & 15)];
                const int k1 = (int)(synth_next(&st) % 63u);
                const int k2 = (int)(synth_next(&st) % 62u);
                const int a = (best + 1 + k1) & 63;
                int c = (best + 1 + k2) & 63;
                if (c == a) c = (c + 1) & 63;
                if (c == best) c = (c + 1) & 63;
                base[(a >> 4) * 128 + (a & 15)] = lo;
                base[(c >> 4) * 128 + (c & 15)] = lo;
            }
        }
    }

    if (mode == TB_SYNTH_CAMERA_EXTREME) {
        const float v = (index & 1u) ? 1.0f : 0.0f;
        for (int p = 0; p < CAMERA_BYTES; ++p) {
            cam8[p] = tb_synth_quantize(v);
            if (camf) camf[p] = v;
        }
        return;
    }
    /* Horizon gradient plus Box-Muller noise (both outputs of each pair). */
    for (int p = 0; p < CAMERA_BYTES; p += 2) {
        const float u1 = fmaxf(synth_unit(&st), 1.0e-7f);
        const float u2 = synth_unit(&st);
        const float radius = sqrtf(-2.0f * logf(u1));
        float s, c;
        sincosf(6.28318530717958647692f * u2, &s, &c);
        const float noise[2] = {radius * c, radius * s};
        for (int k = 0; k < 2; ++k) {
            const int y = ((p + k) >> 6) & 63;
            float v = 0.8f - 0.6f * (float)y / 63.0f + 0.05f * noise[k];
            v = v < 0.0f ? 0.0f : (v > 1.0f ? 1.0f : v);
            cam8[p + k] = tb_synth_quantize(v);
            if (camf) camf[p + k] = v;
        }
    }
}

typedef struct {
    uint64_t seed, first;
    size_t begin, end;
    int mode;
    float *obs, *mission, *camf;
    uint8_t *cam8;
} synth_range;

static void *synth_range_main(void *arg) {
    const synth_range *r = (const synth_range *)arg;
    for (size_t i = r->begin; i < r->end; ++i)
        synth_sample(r->seed, r->first + i, r->mode, r->obs + i * OBS_DIM,
                     r->mission + i * MISSION_DIM, r->cam8 + i * CAMERA_BYTES,
                     r->camf ? r->camf + i * CAMERA_BYTES : NULL);
    return NULL;
}

int tb_synth_generate(uint64_t seed, uint64_t first, size_t count, int mode,
                      float *obs, float *mission, uint8_t *cameras_u8, float *cameras_f32,
                      int threads) {
    if (!obs || !mission || !cameras_u8 || mode < 0 || mode > TB_SYNTH_LIDAR_HALF) return 0;
    if (count == 0) return 1;
    if (threads <= 0) {
        long n = sysconf(_SC_NPROCESSORS_ONLN);
        threads = n > 0 ? (int)n : 1;
    }
    if ((size_t)threads > count) threads = (int)count;
    synth_range *ranges = (synth_range *)calloc((size_t)threads, sizeof(*ranges));
    pthread_t *tids = (pthread_t *)calloc((size_t)threads, sizeof(*tids));
    if (!ranges || !tids) { free(ranges); free(tids); return 0; }
    int started = 0;
    for (int t = 0; t < threads; ++t) {
        ranges[t] = (synth_range){seed, first, count * (size_t)t / (size_t)threads,
                                  count * (size_t)(t + 1) / (size_t)threads, mode,
                                  obs, mission, cameras_f32, cameras_u8};
        if (t == threads - 1) break;
        if (pthread_create(&tids[t], NULL, synth_range_main, &ranges[t]) != 0) {
            /* run the remaining ranges on this thread instead */
            for (int u = t; u < threads - 1; ++u) {
                ranges[u] = (synth_range){seed, first, count * (size_t)u / (size_t)threads,
                                          count * (size_t)(u + 1) / (size_t)threads, mode,
                                          obs, mission, cameras_f32, cameras_u8};
                synth_range_main(&ranges[u]);
            }
            break;
        }
        ++started;
    }
    ranges[threads - 1] = (synth_range){seed, first, count * (size_t)(threads - 1) / (size_t)threads,
                                        count, mode, obs, mission, cameras_f32, cameras_u8};
    synth_range_main(&ranges[threads - 1]);
    for (int t = 0; t < started; ++t) pthread_join(tids[t], NULL);
    free(ranges);
    free(tids);
    return 1;
}
