/*
 * Batched 142-value sensor features on NVIDIA B200 (sm_100a).
 *
 * Drop-in replacement for the reference's C ABI
 * include/turbinator/training/cuda_features.h:1-40 (Viatreen/Turbinator_C).
 * The six reference entry points keep their names, argument meaning, return
 * values and error strings.  Entries below "Additive entry points" do not
 * exist in the reference and change nothing about the six.
 *
 * Layouts (row-major, one row per aircraft):
 *   obs       [batch, 4148] float   48 proprioception, 4096 LiDAR bins, 4 scan-status
 *   mission   [batch, 10]   float
 *   cameras   [batch, 16384] uint8  4 cameras x 64 x 64 luma
 *   features  [batch, 142]  float
 * Float pointers must be 4-byte aligned.  obs and cameras rows that start on
 * 16-byte boundaries (any cudaMalloc'd base) take the staged bulk-copy
 * kernel; other alignments take a slower kernel with the same results.
 */
#ifndef TURBINATOR_CUDA_FEATURES_H
#define TURBINATOR_CUDA_FEATURES_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Replaces cuda_features.h:14-19 (reference src/cuda/features.cu:158-169).
 * Device pointers; cameras may be NULL (camera features are then 0).
 * stream is a cudaStream_t or NULL for the legacy default stream.
 * Returns 1 if the kernel launch succeeded, 0 on NULL obs/mission/features,
 * batch 0, batch > 0x7fffffff, a float pointer that is not 4-byte aligned,
 * or a launch error.  Asynchronous: synchronize before reading features. */
int tb_cuda_extract_features_device(const float *device_obs,
                                    const float *device_mission,
                                    const unsigned char *device_cameras,
                                    float *device_features,
                                    size_t batch_size,
                                    void *stream);

/* Replaces cuda_features.h:20 (features.cu:171-173).  Returns 1 when the
 * stream drained without error.  It also returns 0 (once) when a kernel of
 * this library on the current device (features, onboard values or learner
 * inputs) gave up waiting on its staging pipeline; such a launch leaves its
 * outputs incomplete. */
int tb_cuda_synchronize(void *stream);

typedef struct tb_cuda_feature_batch tb_cuda_feature_batch;

/* Replaces cuda_features.h:26 (features.cu:27-44).  Makes device_id current
 * on the calling thread and allocates device staging for max_batch samples.
 * The reference capped max_batch at 1024; here any max_batch whose staging
 * fits in device memory is accepted (0 is still rejected).  NULL on
 * failure. */
tb_cuda_feature_batch *tb_cuda_feature_batch_create(int device_id, size_t max_batch);

/* Replaces cuda_features.h:27 (features.cu:46-56).  NULL-safe; drains the
 * handle's streams before freeing. */
void tb_cuda_feature_batch_destroy(tb_cuda_feature_batch *batch);

/* Replaces cuda_features.h:28 (features.cu:58-60).  "stage: cuda error" of
 * the last failed host call, "" after a successful one, and
 * "CUDA feature batch unavailable" for a NULL handle. */
const char *tb_cuda_feature_batch_error(const tb_cuda_feature_batch *batch);

/* Replaces cuda_features.h:29-34 (features.cu:62-88).  Host pointers;
 * cameras are required.  0 < count <= max_batch.  Copies in, extracts and
 * copies out, returning after the features are in out_features_142.
 * Page-locked host buffers are streamed in chunks so that copies and
 * kernels overlap.  Pageable buffers of 512 or more rows per device are
 * copied by up to 8 host threads per device (TB_CUDA_HOST_THREADS overrides
 * the total, read when the handle is created) through the handle's
 * page-locked staging, overlapping host copies, transfers and kernels;
 * smaller pageable calls are copied by the driver on the calling thread.
 * Returns 1, or 0 with a stage-named message in
 * tb_cuda_feature_batch_error().  A handle is not thread-safe. */
int tb_cuda_extract_features_host(tb_cuda_feature_batch *batch,
                                  const float *obs_4148,
                                  const float *mission_10,
                                  const unsigned char *cameras_16384,
                                  size_t count,
                                  float *out_features_142);

/* ---- Additive entry points ---- */

/* A handle whose calls are sharded by sample over several GPUs (no
 * counterpart in the reference, which drives one device per handle).
 * device_ids[0..device_count) (1 <= device_count <= 16; an id may repeat);
 * each device holds staging for ceil(max_batch / device_count) samples.
 * tb_cuda_extract_features_host on it splits the rows into contiguous
 * per-device slices, extracts them concurrently (one or more host threads
 * per device) and gathers the features into out_features_142 in row order.
 * tb_cuda_feature_batch_destroy and _error apply unchanged.  Makes
 * device_ids[0] current on the calling thread.  NULL on failure. */
tb_cuda_feature_batch *tb_cuda_feature_batch_create_multi(const int *device_ids,
                                                          int device_count,
                                                          size_t max_batch);

/* Largest shard_count accepted by tb_cuda_extract_features_device_sharded. */
#define TB_CUDA_MAX_SHARDS 64

/* The device entry point over several GPUs in one call (no counterpart in the
 * reference, which launches on one device per call).  Shard i is
 * tb_cuda_extract_features_device(device_obs[i], device_mission[i],
 * device_cameras ? device_cameras[i] : NULL, device_features[i],
 * batch_sizes[i], streams ? streams[i] : NULL) run with device_ids[i] current;
 * every pointer of shard i is memory of that device.  A shard with batch size
 * 0 launches nothing; an id may repeat.  The calling thread's current device
 * is restored before returning.  Returns 1 if every launch succeeded; 0 on
 * shard_count outside 1..TB_CUDA_MAX_SHARDS, a NULL array, an unknown device,
 * a NULL pointer of a non-empty shard, a batch size > 0x7fffffff, or a launch
 * error (shards before the failing one may have launched).  Asynchronous:
 * synchronize each shard's stream on its device (tb_cuda_synchronize with
 * that device current) before reading its features. */
int tb_cuda_extract_features_device_sharded(int shard_count,
                                            const int *device_ids,
                                            const float *const *device_obs,
                                            const float *const *device_mission,
                                            const unsigned char *const *device_cameras,
                                            float *const *device_features,
                                            const size_t *batch_sizes,
                                            void *const *streams);

/* Onboard tactical (24) and physics-prior (15) values per aircraft: the
 * reference's device-only src/network/onboard_features.cuh:515-519
 * (tb_onboard_tactical_prior), which its 618M learner evaluates one thread
 * per aircraft (src/network/network_gpu.cu:274-303) and which
 * tests/test_onboard_features.cu checks.  No C entry point exists for it in
 * the reference; this one follows the conventions of
 * tb_cuda_extract_features_device.  Device pointers: obs [batch,4148],
 * mission [batch,10], tactical [batch,24], prior [batch,15] (rows of 24 and
 * 15 floats).  Returns 1 if the launch succeeded, 0 on NULL pointers, batch
 * 0 or > 0x7fffffff, a pointer that is not 4-byte aligned, or a launch
 * error.  Asynchronous on `stream` (NULL = legacy default stream). */
int tb_cuda_extract_onboard_device(const float *device_obs,
                                   const float *device_mission,
                                   float *device_tactical_24,
                                   float *device_prior_15,
                                   size_t batch_size,
                                   void *stream);

/* FP32-camera variant of tb_cuda_extract_features_device (no counterpart in
 * the reference, whose ABI takes u8 cameras).  device_cameras_f32 is
 * [batch, 4*64*64] float luma, nominally in [0, 1]; each value is quantised
 * on load exactly as the simulator quantises luma for the u8 ABI
 * (src/sim/sensors.c:67: fmax(0, fmin(255, round(v * 255))) in double, so
 * NaN reads as 255), so the features equal those of
 * tb_cuda_extract_features_device on the quantised bytes.  May be NULL
 * (camera features 0).  Same return values and stream semantics. */
int tb_cuda_extract_features_device_f32cam(const float *device_obs,
                                           const float *device_mission,
                                           const float *device_cameras_f32,
                                           float *device_features,
                                           size_t batch_size,
                                           void *stream);

/* Input tensors of the reference's 618M learner, built from the same rows in
 * one call (no C entry point in the reference: its actor forward pass builds
 * them with scalar_inputs, lidar_channels and camera_luma,
 * src/network/network_gpu.cu:274-303,467-483,1446-1451).  Device pointers,
 * one row per aircraft:
 *   proprio [batch,91]    52 symlog-scaled proprioception values, then the
 *                         24 tactical and 15 prior values
 *   mission [batch,49]    mission (non-finite -> 0), tactical, prior
 *   tactical [batch,24], prior [batch,15]  as tb_cuda_extract_onboard_device
 *   lidar [batch,6,2048]  per head: inverse range, range/30, return flag
 *   luma [batch,16384]    camera byte / 255 - 0.5
 * obs, cameras, lidar and luma must be 16-byte aligned, the rest 4-byte
 * aligned; cameras are required.  Returns 1 if the launches succeeded, 0
 * otherwise; asynchronous on `stream`. */
int tb_cuda_prepare_actor_inputs_device(const float *device_obs,
                                        const float *device_mission,
                                        const unsigned char *device_cameras,
                                        float *device_proprio_91,
                                        float *device_mission_49,
                                        float *device_tactical_24,
                                        float *device_prior_15,
                                        float *device_lidar_6x2048,
                                        float *device_camera_luma,
                                        size_t batch_size,
                                        void *stream);

/* Largest count accepted by tb_cuda_extract_features_host_noalloc. */
#define TB_CUDA_NOALLOC_MAX_BATCH 64

/* No counterpart in the reference.  For callers that cannot allocate device
 * memory: an onboard control loop that forbids allocation once it is running
 * (cudaMalloc can block and synchronise the device in the middle of a tick),
 * or a process whose GPU memory is already reserved in full by a learner's
 * memory pool.  Does the work of tb_cuda_extract_features_host without a
 * handle: the rows are staged through one fixed 2,149,376-byte array that the
 * library reserves statically on every GPU that loads it (held until the
 * process exits); nothing here calls cudaMalloc or cudaFree.
 * Host pointers; cameras required; stream is a cudaStream_t or NULL; uses the
 * calling thread's current device.  Blocks until the features are in
 * out_features_142.  Returns 1 on success; -1, doing nothing, when count is 0
 * or greater than TB_CUDA_NOALLOC_MAX_BATCH; 0 on a NULL pointer or a CUDA
 * error.
 * The first call on each device is the set-up: CUDA loads this library's
 * kernel modules on first use, so that call reserves the array (and the
 * modules' code) on the device and then looks up the array's device address
 * (cudaGetSymbolAddress).  Make it at start-up, before a memory pool reserves
 * the device's memory and before any stream capture.  The address is cached
 * per device ordinal; after a cudaDeviceReset of that device it is stale, so
 * do not call this entry point on a device that was reset.
 * All calls on a device share the one array, which keeps the last call's rows:
 * calls that overlap on the GPU (several host threads at once) race.  Each
 * call overwrites every row it reads, so nothing needs clearing between
 * calls. */
int tb_cuda_extract_features_host_noalloc(const float *obs_4148,
                                          const float *mission_10,
                                          const unsigned char *cameras_16384,
                                          size_t count,
                                          float *out_features_142,
                                          void *stream);

#ifdef __cplusplus
}
#endif

#endif
