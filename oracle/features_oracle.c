/*
 * TEST INFRASTRUCTURE ONLY -- CPU oracle for the 142 sensor features.
 *
 * This file restates, in plain C11, the reference's CPU feature path
 * (Viatreen/Turbinator_C src/training/training.c:57-142,
 * `tb_train_extract_features_cpu` and its helpers).  It is the checker that
 * the CUDA library is compared against; nothing in the shipped library links
 * or calls it.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline may load it.
 *
 * Parity pin: tests/test_oracle.py checks this restatement bit-for-bit
 * against the reference's own training.c compiled into oracle/_ref/ (see
 * oracle/Makefile) and against the committed golden vectors in
 * tests/golden/, which were produced by that reference build.
 *
 * Every arithmetic step that decides the output bits is kept in the same
 * order and precision as the reference (float arithmetic, sequential sector
 * sums, IEEE division), because the tests demand bit equality with it.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>

#include "features_oracle.h"

/* Reference training.c:57-59: x < lo ? lo : (x > hi ? hi : x).
 * The comparison form (not fminf/fmaxf) decides the sign of a zero result. */
static float oracle_clamp(float x, float lo, float hi) {
    if (x < lo) return lo;
    if (x > hi) return hi;
    return x;
}

/* Reference training.c:61-63: non-finite values read as 0. */
static float oracle_finite_or_zero(float x) {
    return isfinite(x) ? x : 0.0f;
}

/* Reference training.c:70-81: the 48 proprioceptive divisors, as a table.
 * pi/4 and pi/2 are formed exactly as the reference forms them
 * (float pi divided by 4.0f / 2.0f), so the divisions round identically. */
static float oracle_scalar_divisor(int index) {
    const float pi = 3.14159265358979323846f;
    if (index <= 1) return 300.0f;            /* position x, y */
    if (index == 2) return 100.0f;            /* altitude */
    if (index <= 5) return 50.0f;             /* velocity */
    if (index >= 10 && index <= 12) return 5.0f;   /* body rates */
    if (index >= 13 && index <= 15) return 30.0f;  /* specific force */
    if (index >= 28 && index <= 31) return pi / 4.0f; /* inner gimbal */
    if (index >= 32 && index <= 39) return 5.0f;   /* gimbal rates */
    if (index == 44 || index == 45) return pi / 2.0f; /* cannon az/el */
    return 1.0f;
}

/* Reference training.c:65-68: one LiDAR bin in [-1, 1]. */
static float oracle_lidar_term(float range_m) {
    if (!isfinite(range_m) || range_m < 0.0f) return -1.0f;
    return log1pf(oracle_clamp(range_m, 0.0f, 120.0f)) / log1pf(120.0f);
}

void oracle_extract_features(const float *obs, const float *mission,
                             const uint8_t *cameras, float *out) {
    if (!obs || !mission || !out) return;

    /* f[0..47]: scaled proprioception (training.c:107). */
    for (int i = 0; i < ORACLE_SCALARS; ++i)
        out[i] = oracle_clamp(oracle_finite_or_zero(obs[i]) / oracle_scalar_divisor(i),
                              -1.0f, 1.0f);

    /* f[48..51]: LiDAR ages and valid fractions from the observation tail
     * (training.c:108). */
    for (int i = 0; i < 4; ++i)
        out[ORACLE_SCALARS + i] =
            oracle_clamp(oracle_finite_or_zero(obs[ORACLE_TAIL_OFFSET + i]), 0.0f, 1.0f);

    /* f[52..61]: mission vector; entries 7..9 hidden in arena missions
     * (training.c:109-112). */
    const int arena = oracle_finite_or_zero(mission[6]) > 0.5f;
    for (int i = 0; i < ORACLE_MISSION_DIM; ++i) {
        float v = (i >= 7 && arena) ? 0.0f : mission[i];
        out[52 + i] = oracle_clamp(oracle_finite_or_zero(v), -1.0f, 1.0f);
    }

    /* f[62..125]: 64 LiDAR sector means, each a sequential float sum over
     * 4 elevation rows x 16 azimuth bins, elevation-major
     * (training.c:114-127). */
    for (int sector = 0; sector < 64; ++sector) {
        const int head = sector >> 5;
        const int el_sector = (sector >> 3) & 3;
        const int az_sector = sector & 7;
        const float *base = obs + ORACLE_LIDAR_OFFSET + head * 2048 +
                            el_sector * 4 * 128 + az_sector * 16;
        float sum = 0.0f;
        for (int row = 0; row < 4; ++row)
            for (int bin = 0; bin < 16; ++bin)
                sum += oracle_lidar_term(base[row * 128 + bin]);
        out[62 + sector] = sum / 64.0f;
    }

    /* f[126..141]: camera quadrant byte sums / (1024 * 255)
     * (training.c:129-141).  NULL cameras give zeros. */
    for (int q = 0; q < 16; ++q) {
        const int cam = q >> 2, qy = (q >> 1) & 1, qx = q & 1;
        unsigned int sum = 0;
        if (cameras) {
            const uint8_t *tile = cameras + cam * 4096 + qy * 32 * 64 + qx * 32;
            for (int y = 0; y < 32; ++y)
                for (int x = 0; x < 32; ++x) sum += tile[y * 64 + x];
        }
        out[126 + q] = (float)sum / (1024.0f * 255.0f);
    }
}

/* The simulator's luma quantisation (reference src/sim/sensors.c:67, with
 * tb_clamp = fmax(lo, fmin(hi, v)) from src/sim/sim_internal.h:73), applied
 * to one float camera value in double arithmetic.  fmin returns the non-NaN
 * operand, so NaN quantises to 255. */
uint8_t oracle_quantize_luma(float v) {
    return (uint8_t)fmax(0.0, fmin(255.0, round((double)v * 255.0)));
}

void oracle_quantize_cameras(const float *cameras_f32, size_t count, uint8_t *out) {
    for (size_t i = 0; i < count; ++i) out[i] = oracle_quantize_luma(cameras_f32[i]);
}
