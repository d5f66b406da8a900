/*
 * Seeded synthetic sensor batches for the feature benchmarks and tests.
 *
 * The reference measures no public dataset on this path; these batches stand
 * in for the simulator's output (src/sim/sensors.c:101-120 packs the
 * observation; src/sim/c_api.c:88-103 the mission vector) with the shapes
 * and value ranges of the benchmark configurations:
 *   obs[0..47], obs[4144..4147], mission[0..9]  uniform in [-1, 1]
 *   obs[48..4143]  LiDAR, 5% no-return (300 m), else 0.5 * 600^u metres
 *   cameras        0.8 - 0.6*y/63 + N(0, 0.05), clamped to [0, 1]; the u8
 *                  form is quantised like the simulator (sensors.c:67)
 * Every sample draws from its own SplitMix64 stream keyed by (seed, sample
 * index), so any shard [first, first+count) is generated independently and
 * identically on every rank and machine.
 */
#ifndef TB_SYNTH_H
#define TB_SYNTH_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum tb_synth_mode {
    TB_SYNTH_STANDARD = 0,       /* configs 0-3 */
    TB_SYNTH_CAMERA_EXTREME = 1, /* stress quarter (a): cameras all 0.0 (even) / all 1.0 (odd) */
    TB_SYNTH_LIDAR_NORETURN = 2, /* stress quarter (b): every bin at the 300 m no-return */
    TB_SYNTH_LIDAR_DUPMIN = 3,   /* stress quarter (c): sector minimum repeated in 3 bins */
    TB_SYNTH_LIDAR_HALF = 4      /* stress quarter (d): every bin exactly 0.5 m */
};

/* Fills samples [first, first + count) into obs[count,4148],
 * mission[count,10], cameras_u8[count,16384] and, when cameras_f32 is not
 * NULL, the unquantised cameras_f32[count,16384].  threads <= 0 uses one
 * thread per online CPU.  Returns 1 on success, 0 on bad arguments. */
int tb_synth_generate(uint64_t seed, uint64_t first, size_t count, int mode,
                      float *obs, float *mission, uint8_t *cameras_u8, float *cameras_f32,
                      int threads);

/* The simulator's luma quantisation of one camera value (src/sim/sensors.c:67
 * with the clamp of src/sim/sim_internal.h:73), in double:
 * fmax(0, fmin(255, round(v * 255))); NaN gives 255. */
uint8_t tb_synth_quantize(float v);

#ifdef __cplusplus
}
#endif

#endif
