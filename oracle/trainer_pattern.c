/*
 * TEST INFRASTRUCTURE ONLY -- the reference trainer's feature call pattern
 * on real simulator observations, through this repository's C ABI.
 *
 * Follows the extraction sequence of run_training (reference
 * src/trainer/main.c:511-699, engine "cuda-p3000"): create a handle for the
 * batch, extract the initial observations, then per environment step
 * extract the opponents' observations when any environment is an arena
 * scenario, step the simulator, extract the next observations, and after
 * episode ends reset those environments and extract again (otherwise swap
 * the observation buffers, as the trainer does).  Actions come from the
 * simulator's reference controller (tb_reference_action_batch) instead of
 * a learner.  Every extracted batch is compared with the reference's own
 * CPU path (tb_train_extract_features_cpu): bit-exact for features 0-61 and
 * 126-141, |d| <= 1e-6 + 1e-5*|ref| for the LiDAR sector means 62-125.
 *
 * Built by oracle/Makefile into oracle/_ref/trainer_pattern from this file,
 * the reference's simulator (src/sim/{physics,sensors,c_api}.c) and
 * src/training/training.c, linked against libturbinator_cuda.so.
 *
 *   trainer_pattern <device> <batch> <steps> <seed> [dump_path [dump_batches]]
 *
 * With TB_PATTERN_BATCHED=1 in the environment the same observations go
 * through fewer calls: after each simulator step (and any resets), the next
 * observations, the post-reset observations and the next step's opponent
 * observations -- all taken from the same simulator state the reference
 * extracts them from -- are written by the simulator straight into
 * consecutive rows of one buffer and extracted in one call of up to
 * 3 x batch rows; TB_PATTERN_PINNED=1 in addition makes that buffer
 * page-locked (cudaHostAlloc), as a trainer would allocate it.
 *
 * Prints one summary line (with the wall time spent in extraction calls,
 * batching copies included); exit status 0 iff every call succeeded and every
 * sample matched.  With dump_path, the first dump_batches extracted batches
 * are written as records {int32 count; f32 obs[count*4148];
 * f32 mission[count*10]; u8 cameras[count*16384]}.
 */
#define _POSIX_C_SOURCE 200809L
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include <cuda_runtime_api.h>

#include "turbinator/c_api.h"
#include "turbinator/training/cuda_features.h"
#include "turbinator/training/training.h"

enum { OBS = 4148, MIS = 10, CAM = 16384, FEAT = 142, PRIV = 64, ACT = 15, SCENARIOS = 28 };

typedef struct {
    long calls, samples, exact_mismatches, lidar_over, failures, arena_calls, resets;
    double max_lidar_err, extract_ms;
    FILE *dump;
    int dump_left;
} tally;

static int is_arena_scenario(int s) { return s == 3 || s == 14 || s == 18 || s == 22 || s == 24 || s == 27; }

static void compare_batch(tally *t, const float *obs, const float *mission, const uint8_t *cams,
                          const float *gpu, int count) {
    float ref[FEAT];
    for (int i = 0; i < count; ++i) {
        tb_train_extract_features_cpu(obs + (size_t)i * OBS, mission + (size_t)i * MIS,
                                      cams + (size_t)i * CAM, ref);
        const float *g = gpu + (size_t)i * FEAT;
        for (int f = 0; f < FEAT; ++f) {
            if (f >= 62 && f < 126) {
                const double d = fabs((double)g[f] - (double)ref[f]);
                if (!(d <= 1e-6 + 1e-5 * fabs((double)ref[f]))) ++t->lidar_over;
                if (d > t->max_lidar_err || d != d) t->max_lidar_err = d;
            } else if (memcmp(&g[f], &ref[f], sizeof(float)) != 0) {
                ++t->exact_mismatches;
            }
        }
    }
    t->samples += count;
}

static double now_ms(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec * 1e3 + ts.tv_nsec * 1e-6;
}

static void extract_and_check(tally *t, tb_cuda_feature_batch *h, const float *obs, const float *mission,
                              const uint8_t *cams, float *features, int count) {
    ++t->calls;
    const double t0 = now_ms();
    const int ok = tb_cuda_extract_features_host(h, obs, mission, cams, (size_t)count, features);
    t->extract_ms += now_ms() - t0;
    if (!ok) {
        fprintf(stderr, "extraction failed: %s\n", tb_cuda_feature_batch_error(h));
        ++t->failures;
        return;
    }
    compare_batch(t, obs, mission, cams, features, count);
    if (t->dump && t->dump_left > 0) {
        const int32_t n = count;
        fwrite(&n, sizeof(n), 1, t->dump);
        fwrite(obs, sizeof(float), (size_t)count * OBS, t->dump);
        fwrite(mission, sizeof(float), (size_t)count * MIS, t->dump);
        fwrite(cams, 1, (size_t)count * CAM, t->dump);
        --t->dump_left;
    }
}

/* The rows of one batched call. */
typedef struct {
    float *obs, *mission, *features;
    uint8_t *cams;
    int count;
} group;

/* The next free rows of the batched call: observations are written straight
 * into them by the simulator, so nothing is copied to batch. */
static void group_slot(group *g, int count, float **obs, float **mission, uint8_t **cams) {
    *obs = g->obs + (size_t)g->count * OBS;
    *mission = g->mission + (size_t)g->count * MIS;
    *cams = g->cams + (size_t)g->count * CAM;
    g->count += count;
}

static void group_flush(tally *t, tb_cuda_feature_batch *h, group *g) {
    if (g->count) extract_and_check(t, h, g->obs, g->mission, g->cams, g->features, g->count);
    g->count = 0;
}

int main(int argc, char **argv) {
    if (argc < 5) {
        fprintf(stderr, "usage: %s device batch steps seed [dump_path [dump_batches]]\n", argv[0]);
        return 2;
    }
    const int device = atoi(argv[1]);
    const int batch = atoi(argv[2]);
    const int steps = atoi(argv[3]);
    const uint64_t seed = strtoull(argv[4], NULL, 10);
    tally t;
    memset(&t, 0, sizeof(t));
    if (argc >= 6) {
        t.dump = fopen(argv[5], "wb");
        t.dump_left = argc >= 7 ? atoi(argv[6]) : 4;
    }
    if (batch <= 0 || steps < 0) return 2;

    const size_t B = (size_t)batch;
    float *obs = calloc(B * OBS, sizeof(float)), *next_obs = calloc(B * OBS, sizeof(float));
    float *opp_obs = calloc(B * OBS, sizeof(float));
    float *mission = calloc(B * MIS, sizeof(float)), *next_mission = calloc(B * MIS, sizeof(float));
    float *opp_mission = calloc(B * MIS, sizeof(float));
    uint8_t *cams = calloc(B * CAM, 1), *next_cams = calloc(B * CAM, 1), *opp_cams = calloc(B * CAM, 1);
    float *priv = calloc(B * PRIV, sizeof(float)), *next_priv = calloc(B * PRIV, sizeof(float));
    float *actions = calloc(B * ACT, sizeof(float)), *rewards = calloc(B, sizeof(float));
    uint8_t *terminated = calloc(B, 1), *truncated = calloc(B, 1);
    float *features = calloc(B * FEAT, sizeof(float));
    int *scenario = calloc(B, sizeof(int));
    if (!obs || !next_obs || !opp_obs || !mission || !next_mission || !opp_mission || !cams || !next_cams ||
        !opp_cams || !priv || !next_priv || !actions || !rewards || !terminated || !truncated || !features ||
        !scenario)
        return 3;

    const char *batched_env = getenv("TB_PATTERN_BATCHED");
    const int batched = batched_env && atoi(batched_env) != 0;
    void *sim = tb_create(batch, seed);
    tb_cuda_feature_batch *h = tb_cuda_feature_batch_create(device, batched ? 3 * B : B);
    if (!sim || !h) {
        fprintf(stderr, "setup failed: %s\n", sim ? "feature handle" : tb_last_error());
        return 3;
    }
    /* batched mode: one call per step over the rows gathered here */
    group g = {0};
    const char *pinned_env = getenv("TB_PATTERN_PINNED");
    const int pinned = batched && pinned_env && atoi(pinned_env) != 0;
    if (batched && !pinned) {
        g.obs = calloc(3 * B * OBS, sizeof(float));
        g.mission = calloc(3 * B * MIS, sizeof(float));
        g.cams = calloc(3 * B * CAM, 1);
        g.features = calloc(3 * B * FEAT, sizeof(float));
        if (!g.obs || !g.mission || !g.cams || !g.features) return 3;
    } else if (pinned) { /* page-locked: the host ABI streams them at PCIe speed */
        if (cudaHostAlloc((void **)&g.obs, 3 * B * OBS * sizeof(float), cudaHostAllocPortable) != cudaSuccess ||
            cudaHostAlloc((void **)&g.mission, 3 * B * MIS * sizeof(float), cudaHostAllocPortable) != cudaSuccess ||
            cudaHostAlloc((void **)&g.cams, 3 * B * CAM, cudaHostAllocPortable) != cudaSuccess ||
            cudaHostAlloc((void **)&g.features, 3 * B * FEAT * sizeof(float), cudaHostAllocPortable) != cudaSuccess)
            return 3;
    }
    int any_arena = 0;
    for (int i = 0; i < batch; ++i) {
        scenario[i] = (int)((seed + (uint64_t)i) % SCENARIOS);
        any_arena |= is_arena_scenario(scenario[i]);
        if (tb_reset_one(sim, i, scenario[i], seed + (uint64_t)i)) return 3;
    }
    if (!batched) {
        if (tb_observe_training_batch(sim, obs, mission, cams, priv, NULL)) return 3;
        extract_and_check(&t, h, obs, mission, cams, features, batch);
    } else {
        float *o, *m;
        uint8_t *c;
        group_slot(&g, batch, &o, &m, &c);
        if (tb_observe_training_batch(sim, o, m, c, priv, NULL)) return 3;
        if (any_arena && steps > 0) { /* the first step's opponents, same state */
            group_slot(&g, batch, &o, &m, &c);
            if (tb_observe_opponents_training_batch(sim, o, m, c)) return 3;
            ++t.arena_calls;
        }
        group_flush(&t, h, &g);
    }

    uint64_t resets = 0;
    for (int step = 0; step < steps; ++step) {
        if (tb_reference_action_batch(sim, actions)) return 3;
        if (!batched) {
            if (tb_observe_opponents_training_batch(sim, opp_obs, opp_mission, opp_cams)) return 3;
            if (any_arena) {
                ++t.arena_calls;
                extract_and_check(&t, h, opp_obs, opp_mission, opp_cams, features, batch);
            }
        }
        if (tb_step(sim, actions, next_obs, rewards, terminated, truncated)) return 3;
        if (!batched) {
            if (tb_observe_training_batch(sim, next_obs, next_mission, next_cams, next_priv, NULL)) return 3;
            extract_and_check(&t, h, next_obs, next_mission, next_cams, features, batch);
        } else {
            float *o, *m;
            uint8_t *c;
            group_slot(&g, batch, &o, &m, &c);
            if (tb_observe_training_batch(sim, o, m, c, next_priv, NULL)) return 3;
        }
        int any_done = 0;
        for (int i = 0; i < batch; ++i) {
            if (!(terminated[i] || truncated[i])) continue;
            any_done = 1;
            ++t.resets;
            scenario[i] = (int)((seed + (uint64_t)i + ++resets) % SCENARIOS);
            if (tb_reset_one(sim, i, scenario[i], seed + (uint64_t)step + (uint64_t)i + 1)) return 3;
        }
        if (!any_done) {
            float *f = obs; obs = next_obs; next_obs = f;
            f = mission; mission = next_mission; next_mission = f;
            f = priv; priv = next_priv; next_priv = f;
            uint8_t *c = cams; cams = next_cams; next_cams = c;
        } else {
            if (!batched) {
                if (tb_observe_training_batch(sim, obs, mission, cams, priv, NULL)) return 3;
                extract_and_check(&t, h, obs, mission, cams, features, batch);
            } else {
                float *o, *m;
                uint8_t *c;
                group_slot(&g, batch, &o, &m, &c);
                if (tb_observe_training_batch(sim, o, m, c, priv, NULL)) return 3;
            }
            any_arena = 0;
            for (int i = 0; i < batch; ++i) any_arena |= is_arena_scenario(scenario[i]);
        }
        if (batched) {
            /* the next step's opponents come from this (post-reset) state,
             * which the reference reads at the top of the next step */
            if (any_arena && step + 1 < steps) {
                float *o, *m;
                uint8_t *c;
                group_slot(&g, batch, &o, &m, &c);
                if (tb_observe_opponents_training_batch(sim, o, m, c)) return 3;
                ++t.arena_calls;
            }
            group_flush(&t, h, &g);
        }
    }
    if (pinned) {
        cudaFreeHost(g.obs);
        cudaFreeHost(g.mission);
        cudaFreeHost(g.cams);
        cudaFreeHost(g.features);
    } else {
        free(g.obs);
        free(g.mission);
        free(g.cams);
        free(g.features);
    }
    tb_cuda_feature_batch_destroy(h);
    tb_destroy(sim);
    if (t.dump) fclose(t.dump);
    printf("trainer-pattern: calls=%ld samples=%ld failures=%ld exact_mismatches=%ld lidar_over_tol=%ld "
           "max_lidar_abs_err=%.3g arena_calls=%ld resets=%ld extract_ms=%.3f batched=%d pinned=%d\n",
           t.calls, t.samples, t.failures, t.exact_mismatches, t.lidar_over, t.max_lidar_err, t.arena_calls,
           t.resets, t.extract_ms, batched, pinned);
    return (t.failures || t.exact_mismatches || t.lidar_over) ? 1 : 0;
}
