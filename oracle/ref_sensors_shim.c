/*
 * TEST INFRASTRUCTURE ONLY -- runs the reference simulator's own sensor
 * renderers (Viatreen/Turbinator_C src/sim/sensors.c:28-50
 * tb_sim_render_lidar and :69-82 tb_sim_render_camera, compiled unchanged
 * from the reference tree with src/sim/physics.c and c_api.c) on
 * tb_sensor_scene records, and makes scenes from simulated episodes.
 * Built by oracle/Makefile into oracle/_ref/libtb_ref_sensors.so.
 *
 *   ref_sensors_render    unpack each scene into a simulator environment and
 *                         render it with the reference functions (threaded
 *                         over scenes; also the timed CPU baseline)
 *   ref_sensors_simulate  reset environments, fly them with the reference
 *                         controller (firing in the arena scenarios), pack each
 *                         one's scene as a caller of the GPU renderer would,
 *                         and render the environment itself -- so a test can
 *                         check both the GPU renderer and the packing
 *   ref_sensors_pack      the packing step alone (TbEnv/TbConfig -> scene)
 */
#define _POSIX_C_SOURCE 200809L
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "sim_internal.h"
#include "turbinator/sim/cuda_sensors.h"

/* The scene record of the GPU renderer, filled from simulator state. */
static void pack_scene(const TbEnv *e, const TbConfig *c, int player, int sensors, tb_sensor_scene *s) {
    memset(s, 0, sizeof *s);
    const TbAircraft *a = &e->aircraft[player], *opp = &e->aircraft[1 - player];
    s->position[0] = a->pos.x;
    s->position[1] = a->pos.y;
    s->position[2] = a->pos.z;
    s->attitude[0] = a->quat.w;
    s->attitude[1] = a->quat.x;
    s->attitude[2] = a->quat.y;
    s->attitude[3] = a->quat.z;
    s->opponent[0] = opp->pos.x;
    s->opponent[1] = opp->pos.y;
    s->opponent[2] = opp->pos.z;
    s->lidar_max = c->lidar_max;
    s->dome_radius = c->dome_radius;
    s->rng = e->rng;
    s->step_index = e->step_index;
    s->player = player;
    s->scenario = e->scenario;
    s->sensors = sensors;
    s->obstacle_count = e->obstacle_count;
    s->ball_count = e->ball_count;
    for (int i = 0; i < e->obstacle_count && i < TB_SENSOR_MAX_OBSTACLES; i++) {
        s->obstacles[i][0] = e->obstacles[i].center.x;
        s->obstacles[i][1] = e->obstacles[i].center.y;
        s->obstacles[i][2] = e->obstacles[i].center.z;
        s->obstacles[i][3] = e->obstacles[i].radius;
    }
    for (int i = 0; i < e->ball_count && i < TB_SENSOR_MAX_BALLS; i++) {
        s->balls[i][0] = e->balls[i].pos.x;
        s->balls[i][1] = e->balls[i].pos.y;
        s->balls[i][2] = e->balls[i].pos.z;
    }
}

void ref_sensors_pack(const void *env, const void *config, int player, int sensors, tb_sensor_scene *out) {
    pack_scene((const TbEnv *)env, (const TbConfig *)config, player, sensors, out);
}

/* The simulator state the renderers read, from a scene (player 0 or 1). */
static void unpack_scene(const tb_sensor_scene *s, TbEnv *e, TbConfig *c) {
    tb_config_defaults(c);
    c->lidar_max = s->lidar_max;
    c->dome_radius = s->dome_radius;
    const int p = s->player;
    e->scenario = s->scenario;
    e->rng = s->rng;
    e->step_index = s->step_index;
    e->aircraft[p].pos = tb_v(s->position[0], s->position[1], s->position[2]);
    e->aircraft[p].quat = tb_q(s->attitude[0], s->attitude[1], s->attitude[2], s->attitude[3]);
    e->aircraft[1 - p].pos = tb_v(s->opponent[0], s->opponent[1], s->opponent[2]);
    e->obstacle_count = s->obstacle_count < 0 ? 0 : (s->obstacle_count > TB_MAX_OBSTACLES ? TB_MAX_OBSTACLES : s->obstacle_count);
    e->ball_count = s->ball_count < 0 ? 0 : (s->ball_count > TB_MAX_BALLS ? TB_MAX_BALLS : s->ball_count);
    for (int i = 0; i < e->obstacle_count; i++) {
        e->obstacles[i].center = tb_v(s->obstacles[i][0], s->obstacles[i][1], s->obstacles[i][2]);
        e->obstacles[i].radius = s->obstacles[i][3];
    }
    for (int i = 0; i < e->ball_count; i++) e->balls[i].pos = tb_v(s->balls[i][0], s->balls[i][1], s->balls[i][2]);
}

typedef struct {
    const tb_sensor_scene *scenes;
    int64_t begin, end;
    float *lidar, *valid;
    int64_t lidar_stride, valid_stride;
    uint8_t *cameras, *raw;
    int ok;
} render_job;

static void *render_worker(void *arg) {
    render_job *j = (render_job *)arg;
    TbEnv *e = (TbEnv *)calloc(1, sizeof(TbEnv));
    if (!e) return NULL;
    TbConfig c;
    for (int64_t i = j->begin; i < j->end; i++) {
        const tb_sensor_scene *s = j->scenes + i;
        if (s->player != 0 && s->player != 1) continue;
        unpack_scene(s, e, &c);
        const int p = s->player;
        if (j->lidar && (s->sensors & TB_SENSOR_LIDAR)) {
            tb_sim_render_lidar(e, &c, p);
            memcpy(j->lidar + i * j->lidar_stride, e->lidar[p], sizeof(e->lidar[p]));
            if (j->valid) {
                j->valid[i * j->valid_stride] = e->lidar_valid[p][0];
                j->valid[i * j->valid_stride + 1] = e->lidar_valid[p][1];
            }
        }
        if ((j->cameras || j->raw) && (s->sensors & TB_SENSOR_CAMERA)) {
            e->capture_raw = j->raw != NULL;
            tb_sim_render_camera(e, &c, p);
            if (j->cameras) memcpy(j->cameras + i * (int64_t)TB_CAMERA_PIXELS, e->camera[p], TB_CAMERA_PIXELS);
            if (j->raw) memcpy(j->raw + i * (int64_t)TB_CAMERA_RAW_PIXELS, e->raw_camera[p], TB_CAMERA_RAW_PIXELS);
        }
    }
    free(e);
    j->ok = 1;
    return NULL;
}

static double now_seconds(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec + 1e-9 * ts.tv_nsec;
}

/* Renders scenes[0..count) with the reference renderers on `threads` host
 * threads (contiguous slices).  Returns the wall time in seconds, or -1. */
double ref_sensors_render(const tb_sensor_scene *scenes, int64_t count, float *lidar, int64_t lidar_stride,
                          float *valid, int64_t valid_stride, uint8_t *cameras, uint8_t *raw, int threads) {
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    if (threads > count) threads = (int)(count > 0 ? count : 1);
    pthread_t tid[256];
    render_job jobs[256];
    const double t0 = now_seconds();
    for (int k = 0; k < threads; k++) {
        render_job *j = &jobs[k];
        j->scenes = scenes;
        j->begin = count * k / threads;
        j->end = count * (k + 1) / threads;
        j->lidar = lidar;
        j->valid = valid;
        j->lidar_stride = lidar_stride;
        j->valid_stride = valid_stride;
        j->cameras = cameras;
        j->raw = raw;
        j->ok = 0;
        if (pthread_create(&tid[k], NULL, render_worker, j) != 0) {
            for (int m = 0; m < k; m++) pthread_join(tid[m], NULL);
            return -1;
        }
    }
    int ok = 1;
    for (int k = 0; k < threads; k++) {
        pthread_join(tid[k], NULL);
        ok &= jobs[k].ok;
    }
    const double t1 = now_seconds();
    return ok ? t1 - t0 : -1;
}

/* Simulated scenes: environment i is reset to scenarios[i] with seeds[i],
 * flown steps[i] steps by the reference controller (tb_sim_reference; in the
 * arena scenarios it also fires whenever the cannon is ready), and packed for
 * player players[i] (0 outside the arena scenarios).  The environment itself
 * is then rendered by the reference functions into lidar [count,4096],
 * valid [count,2] and cameras [count,16384].  Returns 0, or -1 on failure. */
int ref_sensors_simulate(int count, const int *scenarios, const uint64_t *seeds, const int *steps,
                         const int *players, tb_sensor_scene *scenes, float *lidar, float *valid,
                         uint8_t *cameras) {
    TbEnv *e = (TbEnv *)calloc(1, sizeof(TbEnv));
    if (!e) return -1;
    TbConfig c;
    tb_config_defaults(&c);
    for (int i = 0; i < count; i++) {
        memset(e, 0, sizeof *e);
        e->external_cameras = 1; /* no camera renders while flying; one at the end */
        tb_sim_reset_env(e, &c, scenarios[i], seeds[i]);
        const int arena = tb_is_arena(e->scenario);
        for (int k = 0; k < steps[i] && !e->terminated && !e->truncated; k++) {
            float action[TB_ACTION_DIM];
            tb_sim_reference(e, &c, NULL, action);
            if (arena) action[14] = 1.0f;
            tb_sim_step_env(e, &c, action, NULL);
        }
        const int p = arena ? (players[i] & 1) : 0;
        pack_scene(e, &c, p, TB_SENSOR_LIDAR | TB_SENSOR_CAMERA, scenes + i);
        tb_sim_render_lidar(e, &c, p);
        tb_sim_render_camera(e, &c, p);
        memcpy(lidar + (int64_t)i * TB_LIDAR_BINS, e->lidar[p], sizeof(e->lidar[p]));
        valid[2 * i] = e->lidar_valid[p][0];
        valid[2 * i + 1] = e->lidar_valid[p][1];
        memcpy(cameras + (int64_t)i * TB_CAMERA_PIXELS, e->camera[p], TB_CAMERA_PIXELS);
    }
    free(e);
    return 0;
}
