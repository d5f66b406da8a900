/* TEST INFRASTRUCTURE ONLY -- declarations of the CPU oracle and the
 * multi-threaded CPU baseline runner.  Not part of the shipped library. */
#ifndef TB_FEATURES_ORACLE_H
#define TB_FEATURES_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    ORACLE_OBS_DIM = 4148,
    ORACLE_MISSION_DIM = 10,
    ORACLE_CAMERA_BYTES = 16384,
    ORACLE_FEATURE_DIM = 142,
    ORACLE_SCALARS = 48,
    ORACLE_LIDAR_OFFSET = 48,
    ORACLE_TAIL_OFFSET = 4144
};

/* Same contract as the reference's tb_train_extract_features_cpu
 * (include/turbinator/training/training.h:55-58). */
void oracle_extract_features(const float *obs, const float *mission,
                             const uint8_t *cameras, float *out);

/* The simulator's camera quantisation of float luma values (sensors.c:67):
 * the oracle for the FP32-camera entry point quantises with this and then
 * runs the 142-feature path on the bytes.  count is a number of values. */
uint8_t oracle_quantize_luma(float v);
void oracle_quantize_cameras(const float *cameras_f32, size_t count, uint8_t *out);

/* Per-sample extractor signature shared by the oracle above and the
 * reference's own tb_train_extract_features_cpu (loaded from oracle/_ref). */
typedef void (*oracle_sample_fn)(const float *, const float *, const uint8_t *, float *);

/* Runs `fn` over samples [0, count) of a [count,4148]/[count,10]/[count,16384]
 * batch with `threads` POSIX threads over contiguous sample ranges, writing
 * [count,142] features.  cameras may be NULL.  Returns wall seconds, or a
 * negative value if a thread could not be started. */
double oracle_extract_batch(oracle_sample_fn fn, const float *obs, const float *mission,
                            const uint8_t *cameras, size_t count, float *out, int threads);

/* Convenience: oracle_extract_batch with the restated oracle. */
double oracle_extract_batch_self(const float *obs, const float *mission,
                                 const uint8_t *cameras, size_t count, float *out,
                                 int threads);

/* Per-aircraft onboard tactical(24)/prior(15) signature of the reference
 * header built for the host (oracle/_ref, tb_ref_onboard_tactical_prior). */
typedef void (*oracle_onboard_fn)(const float *, const float *, float *, float *);

/* Runs `fn` over [count,4148]/[count,10] rows with `threads` POSIX threads,
 * writing [count,39] (24 tactical then 15 prior).  Returns wall seconds or a
 * negative value on failure. */
double oracle_onboard_batch(oracle_onboard_fn fn, const float *obs, const float *mission,
                            size_t count, float *out_39, int threads);

#ifdef __cplusplus
}
#endif

#endif
