/*
 * Internal interface between the C11 host code, the CUDA launch shim and
 * the tests.  Not part of the public ABI (include/turbinator/...).
 */
#ifndef TB_FEATURES_INTERNAL_H
#define TB_FEATURES_INTERNAL_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    TB_OBS_DIM = 4148,
    TB_MISSION_DIM = 10,
    TB_CAMERA_BYTES = 16384,
    TB_FEATURE_DIM = 142
};

/* Status bits recorded by the kernels in their stream's status word:
 * a bounded pipeline wait expired; an index outside its buffer was caught
 * (only the debug build, TB_FEATURES_DEBUG, checks indices). */
enum { TB_FEATURE_STATUS_WAIT_TIMEOUT = 1u, TB_FEATURE_STATUS_BOUNDS = 2u };

typedef struct tb_features_launch_opts {
    int force_direct;                 /* 1: use the plain-load kernel even for aligned rows */
    int grid_limit;                   /* > 0: cap on staged-kernel CTAs */
    unsigned long long wait_ns;       /* 0: default (~1 s) limit on each pipeline wait */
    long long stall_sample;           /* test hook: >= 0 withholds that sample's copies so the
                                         bounded waits expire; -1 in normal use */
    int flat;                         /* u8 cameras, aligned rows: >= 0 takes the
                                         one-CTA-per-aircraft kernel (the default), -1 the
                                         staged ring kernel */
} tb_features_launch_opts;

/* Launch on the current device; same return contract as
 * tb_cuda_extract_features_device.  opts may be NULL. */
int tb_features_launch(const float *obs, const float *mission, const unsigned char *cameras,
                       float *features, size_t batch, void *stream,
                       const tb_features_launch_opts *opts);

/* As tb_features_launch; on failure *launch_error (if not NULL) receives
 * the cudaError_t of the failed step (cudaErrorInvalidValue for rejected
 * arguments). */
int tb_features_launch_checked(const float *obs, const float *mission,
                               const unsigned char *cameras, float *features, size_t batch,
                               void *stream, const tb_features_launch_opts *opts,
                               int *launch_error);

/* As tb_features_launch, with FP32 camera rows [batch,16384] quantised on
 * load with the simulator's rule. */
int tb_features_launch_f32cam(const float *obs, const float *mission, const float *cameras_f32,
                              float *features, size_t batch, void *stream,
                              const tb_features_launch_opts *opts);

/* Status word of `stream` on the current device (tb_status.cu): the device
 * address that the kernels launched on that stream receive and OR their
 * status bits into.  NULL if the device cannot be queried. */
unsigned int *tb_status_slot(void *stream);

/* Reads (via `stream`) and clears `stream`'s status word on the current
 * device.  Returns 1 if the read succeeded; *status receives the bits. */
int tb_status_take(void *stream, unsigned int *status);

/* Enqueue on `stream` an asynchronous copy of its status word into
 * host_word (page-locked), to be read after the stream drains. */
int tb_status_enqueue(void *stream, unsigned int *host_word);

/* Clear `stream`'s status word (synchronous on `stream`). */
int tb_status_clear(void *stream);

/* tb_cuda_extract_onboard_device with launch options (wait_ns and stall_sample
 * are honoured); opts may be NULL. */
int tb_onboard_launch(const float *obs, const float *mission, float *tactical, float *prior, size_t batch,
                      void *stream, const tb_features_launch_opts *opts);

/* The control law alone (the scans' results already parked in the prior
 * rows), one aircraft per thread on `stream`; with proprio_91 and mission_49
 * both non-NULL it also writes the tactical and prior values into those
 * learner rows (proprio columns 52..90, mission columns 10..48). */
int tb_onboard_control_launch(const float *obs, const float *mission, float *tactical, float *prior, size_t batch,
                              void *stream, float *proprio_91, float *mission_49);

/* The learner-input streaming kernel alone, tactical and prior already in
 * place (it copies them into the proprio and mission rows); opts may be NULL
 * (wait_ns and stall_sample are honoured). */
int tb_actor_inputs_launch(const float *obs, const float *mission, const unsigned char *cameras,
                           const float *tactical, const float *prior, float *proprio, float *mission_vec,
                           float *lidar, float *luma, size_t batch, void *stream,
                           const tb_features_launch_opts *opts);

/* The learner-input streaming kernel as tb_cuda_prepare_actor_inputs_device
 * launches it: it also runs the onboard LiDAR scans of the dodge and slalom
 * aircraft from the rows it has staged, parks their results in the prior
 * rows, and leaves the onboard columns of the proprio and mission rows to
 * tb_onboard_control_launch; opts as tb_actor_inputs_launch. */
int tb_actor_inputs_scan_launch(const float *obs, const float *mission, const unsigned char *cameras,
                                float *prior, float *proprio, float *mission_vec, float *lidar, float *luma,
                                size_t batch, void *stream, const tb_features_launch_opts *opts);

/* Launch geometry of the staged kernel on the current device. */
int tb_features_staged_config(int *blocks_per_sm, int *sms, int *smem_bytes, int *threads,
                              int *stages);

#ifdef __cplusplus
}
#endif

#endif
