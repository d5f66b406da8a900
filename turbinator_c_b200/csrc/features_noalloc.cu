/*
 * Allocation-free host entry point for the 142 sensor features.
 *
 * Who needs it: code that must not allocate device memory while it runs --
 * an onboard control loop that forbids allocation after start-up (cudaMalloc
 * can block for milliseconds and synchronise the device mid-tick), or a
 * process whose GPU memory is already reserved in full by a learner's memory
 * pool, so that a feature handle's cudaMalloc would fail.  Such callers get
 * the same work as tb_cuda_extract_features_host without creating a handle:
 * their host rows are staged through one fixed array that this library
 * reserves statically, below, on every GPU that loads it.
 *
 * The array's name is only a host-side stand-in in host code; the device
 * address is looked up once per device with cudaGetSymbolAddress (with that
 * device current) on the first call, and that address is what the kernel
 * receives.  CUDA loads modules lazily, so that first call is also when the
 * array (and the kernels' code) is reserved on the device: callers make it at
 * start-up, before a memory pool takes the device's memory and before any
 * stream capture.  The cached address belongs to the device's context at the
 * time of the look-up and is stale after a cudaDeviceReset.  This file calls
 * no cudaMalloc, cudaFree or other allocating routine.
 */
#include <cuda_runtime.h>

#include <mutex>
#include <stddef.h>

#include "tb_features_internal.h"
#include "turbinator/training/cuda_features.h"

namespace {

constexpr size_t kMaxBatch = TB_CUDA_NOALLOC_MAX_BATCH;
constexpr size_t kObsRegion = 0;
constexpr size_t kObsBytes = kMaxBatch * TB_OBS_DIM * sizeof(float);          /* 1,061,888 */
constexpr size_t kMissionRegion = kObsRegion + kObsBytes;
constexpr size_t kMissionBytes = kMaxBatch * TB_MISSION_DIM * sizeof(float);  /* 2,560 */
constexpr size_t kCameraRegion = kMissionRegion + kMissionBytes;              /* 1,064,448 */
constexpr size_t kCameraBytes = kMaxBatch * TB_CAMERA_BYTES;                  /* 1,048,576 */
constexpr size_t kFeatureRegion = kCameraRegion + kCameraBytes;
constexpr size_t kFeatureBytes = kMaxBatch * TB_FEATURE_DIM * sizeof(float);  /* 36,352 */
constexpr size_t kScratchBytes = kFeatureRegion + kFeatureBytes;              /* 2,149,376 */

/* The staged kernel's bulk copies need 16-byte aligned rows. */
static_assert(kObsRegion % 256 == 0 && kCameraRegion % 256 == 0, "region alignment");
static_assert(kMissionRegion % 16 == 0 && kFeatureRegion % 16 == 0, "region alignment");

constexpr int kMaxDevices = 64;
std::mutex g_setup_lock;
unsigned char *g_scratch_address[kMaxDevices]; /* device address of the array, per device */

} /* namespace */

/* The fixed staging array: 2,149,376 bytes on every GPU that loads this library. */
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

/* Device address of g_noalloc_scratch on device `dev` (which must be current). */
static cudaError_t noalloc_scratch_on(int dev, unsigned char **out) {
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> hold(g_setup_lock);
    if (!g_scratch_address[dev]) {
        void *ptr = nullptr;
        const cudaError_t st = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (st != cudaSuccess) return st;
        g_scratch_address[dev] = static_cast<unsigned char *>(ptr);
    }
    *out = g_scratch_address[dev];
    return cudaSuccess;
}

extern "C" int tb_cuda_extract_features_host_noalloc(const float *obs_4148, const float *mission_10,
                                                      const unsigned char *cameras_16384,
                                                      size_t count, float *out_features_142,
                                                      void *stream) {
    if (count == 0 || count > kMaxBatch) return -1;
    if (!obs_4148 || !mission_10 || !cameras_16384 || !out_features_142) return 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    unsigned char *base = nullptr;
    if (noalloc_scratch_on(dev, &base) != cudaSuccess) return 0;

    float *d_obs = reinterpret_cast<float *>(base + kObsRegion);
    float *d_mission = reinterpret_cast<float *>(base + kMissionRegion);
    unsigned char *d_cameras = base + kCameraRegion;
    float *d_features = reinterpret_cast<float *>(base + kFeatureRegion);
    cudaStream_t s = static_cast<cudaStream_t>(stream);

    if (cudaMemcpyAsync(d_obs, obs_4148, count * TB_OBS_DIM * sizeof(float),
                        cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaMemcpyAsync(d_mission, mission_10, count * TB_MISSION_DIM * sizeof(float),
                        cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaMemcpyAsync(d_cameras, cameras_16384, count * TB_CAMERA_BYTES,
                        cudaMemcpyHostToDevice, s) != cudaSuccess) {
        cudaStreamSynchronize(s);
        return 0;
    }
    if (!tb_features_launch(d_obs, d_mission, d_cameras, d_features, count, stream, nullptr)) {
        cudaStreamSynchronize(s);
        return 0;
    }
    if (cudaMemcpyAsync(out_features_142, d_features, count * TB_FEATURE_DIM * sizeof(float),
                        cudaMemcpyDeviceToHost, s) != cudaSuccess) {
        cudaStreamSynchronize(s);
        return 0;
    }
    if (cudaStreamSynchronize(s) != cudaSuccess) return 0;
    unsigned int pipeline = 0;
    if (!tb_status_take(stream, &pipeline) || pipeline) return 0;
    return 1;
}
