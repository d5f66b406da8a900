/*
 * sm_100a kernel for the 618M learner's input tensors -- the consumer side of
 * the feature path.  The reference builds them in its actor forward pass
 * (src/network/network_gpu.cu:1427-1451) with three launches over the same
 * observation bytes: scalar_inputs (:274-303, one thread per aircraft,
 * including the onboard tactical/prior values), lidar_channels (:467-479)
 * and camera_luma (:480-483).  Exposed through the additive entry point
 * tb_cuda_prepare_actor_inputs_device.
 *
 * Per aircraft (outputs row-major, one row per aircraft):
 *   proprio[91]      52 symlog-scaled proprioception values (obs[0..47],
 *                    obs[4144..4147]), then tactical[24], then prior[15]
 *   mission_vec[49]  mission[10] with non-finite -> 0, tactical[24], prior[15]
 *   tactical[24], prior[15]  as tb_cuda_extract_onboard_device
 *   lidar[6][2048]   channel c of head c%2: c<2 inverse range, c<4 range/30
 *                    (1 if no return), else the return flag
 *   luma[16384]      camera byte / 255 - 0.5
 *
 * Design (B200): the onboard kernel (onboard_kernel.cu) produces tactical
 * and prior; this streaming kernel then reads each aircraft's LiDAR block
 * and cameras once and writes the 6 LiDAR channels and the luma plane with
 * 128-bit streaming stores, every warp store covering 512 contiguous bytes
 * (partial-line stores cost write bandwidth); each thread loads the next
 * aircraft's inputs before storing the current one's.  It moves 33,016
 * bytes in and 115,404 bytes out per aircraft, so it is bound by HBM write
 * bandwidth.  Persistent grid of exactly the resident CTAs, one aircraft per
 * 256-thread CTA iteration.
 *
 * Arithmetic follows the reference kernels' expressions (as nvcc compiles
 * them, i.e. with the multiply-add of the luma contracted), so the values
 * equal the reference's GPU output; the symlog uses CUDA's log1pf exactly
 * as the reference does.
 */
#include <cuda_runtime.h>

#include <stdint.h>

#include "tb_features_internal.h"
#include "turbinator/training/cuda_features.h"

namespace {

constexpr int kObsDim = 4148;
constexpr int kMissionDim = 10;
constexpr int kCameraBytes = 16384;
constexpr int kProprio = 91;
constexpr int kMissionVec = 49;
constexpr int kLidarBins = 2048;          /* per head */
constexpr int kThreads = 256;

/* Symlog scale of proprioceptive input i (network_gpu.cu:289-295). */
__device__ __forceinline__ float symlog_scale(int i) {
    float s = 1.0f;
    s = (i < 3) ? 0.05f : s;
    s = (i >= 3 && i < 6) ? 0.10f : s;
    s = (i >= 10 && i < 13) ? 0.20f : s;
    s = (i >= 13 && i < 16) ? 0.10f : s;
    s = (i >= 28 && i < 32) ? 0.50f : s;
    s = (i >= 32 && i < 36) ? 0.20f : s;
    return s;
}

/* One LiDAR range -> its three channel values (network_gpu.cu:473-478). */
struct LidarChannels {
    float inverse, scaled, flag;
};

__device__ __forceinline__ LidarChannels lidar_value(float range) {
    const bool valid = range > 0.0f && isfinite(range);
    const float clamped = fmaxf(0.05f, fminf(30.0f, range));
    LidarChannels c;
    c.inverse = valid ? 1.0f / fmaxf(0.2f, clamped) : 0.0f;
    c.scaled = valid ? clamped / 30.0f : 1.0f;
    c.flag = valid ? 1.0f : 0.0f;
    return c;
}

__device__ __forceinline__ float luma(uint32_t byte) {
    return __fmaf_rn(static_cast<float>(byte), 1.0f / 255.0f, -0.5f);
}

__device__ __forceinline__ float4 luma4(uint32_t w) {
    return make_float4(luma(w & 255u), luma((w >> 8) & 255u), luma((w >> 16) & 255u), luma(w >> 24));
}

/* One aircraft's inputs held in registers: LiDAR float4s q = k*256 + t and
 * camera words c = m*256 + t of this thread. */
struct RowLoads {
    float4 lidar[4];
    uint32_t cam[16];
};

__device__ __forceinline__ void load_row(RowLoads &r, const float *o, const unsigned char *cam_row, int t) {
#pragma unroll
    for (int k = 0; k < 4; ++k) r.lidar[k] = __ldg(reinterpret_cast<const float4 *>(o + 48) + k * kThreads + t);
    const uint32_t *cw = reinterpret_cast<const uint32_t *>(cam_row);
#pragma unroll
    for (int m = 0; m < 16; ++m) r.cam[m] = __ldg(cw + m * kThreads + t);
}

__global__ void __launch_bounds__(kThreads) actor_inputs_kernel(
    const float *__restrict__ obs, const float *__restrict__ mission, const unsigned char *__restrict__ cameras,
    const float *__restrict__ tactical, const float *__restrict__ prior, float *__restrict__ proprio,
    float *__restrict__ mission_vec, float *__restrict__ lidar, float *__restrict__ luma_out,
    unsigned long long batch) {
    const int t = threadIdx.x;
    unsigned long long b = blockIdx.x;
    if (b >= batch) return;
    RowLoads cur;
    load_row(cur, obs + b * kObsDim, cameras + b * kCameraBytes, t);
    for (; b < batch; b += gridDim.x) {
        /* Issue the next aircraft's loads before this one's stores. */
        const unsigned long long nb = b + gridDim.x;
        RowLoads nxt;
        if (nb < batch) load_row(nxt, obs + nb * kObsDim, cameras + nb * kCameraBytes, t);
        const float *o = obs + b * kObsDim;

        /* LiDAR: float4 q (0..1023) of the scan is head q/512, bins 4*(q%512)..;
         * it feeds channels head, 2+head and 4+head.  Each warp store covers
         * 512 contiguous bytes of one channel row. */
        float *lo = lidar + b * (6ull * kLidarBins);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int q = k * kThreads + t;
            const int head = q >> 9;
            const int bin4 = q & 511;
            const float4 r = cur.lidar[k];
            const LidarChannels a = lidar_value(r.x), bb = lidar_value(r.y), c = lidar_value(r.z),
                                d = lidar_value(r.w);
            __stcs(reinterpret_cast<float4 *>(lo + head * kLidarBins) + bin4,
                   make_float4(a.inverse, bb.inverse, c.inverse, d.inverse));
            __stcs(reinterpret_cast<float4 *>(lo + (2 + head) * kLidarBins) + bin4,
                   make_float4(a.scaled, bb.scaled, c.scaled, d.scaled));
            __stcs(reinterpret_cast<float4 *>(lo + (4 + head) * kLidarBins) + bin4,
                   make_float4(a.flag, bb.flag, c.flag, d.flag));
        }
        /* Luma: camera word c (bytes 4c..4c+3) -> output float4 c. */
        float4 *lu = reinterpret_cast<float4 *>(luma_out + b * kCameraBytes);
#pragma unroll
        for (int m = 0; m < 16; ++m) __stcs(lu + m * kThreads + t, luma4(cur.cam[m]));

        /* Scalars (network_gpu.cu:285-302). */
        float *p = proprio + b * kProprio;
        float *mv = mission_vec + b * kMissionVec;
        if (t < 52) {
            float raw = t < 48 ? o[t] : o[4144 + t - 48];
            raw = isfinite(raw) ? fmaxf(-1000.0f, fminf(1000.0f, raw)) : 0.0f;
            const float symlog = copysignf(log1pf(fabsf(raw * symlog_scale(t))), raw);
            p[t] = fmaxf(-8.0f, fminf(8.0f, symlog / sqrtf(1.0001f)));
        } else if (t < 52 + kMissionDim) {
            const float m = mission[b * kMissionDim + (t - 52)];
            mv[t - 52] = isfinite(m) ? m : 0.0f;
        } else if (t >= 64 && t < 64 + 24) {
            const float v = tactical[b * 24 + (t - 64)];
            p[52 + (t - 64)] = v;
            mv[10 + (t - 64)] = v;
        } else if (t >= 96 && t < 96 + 15) {
            const float v = prior[b * 15 + (t - 96)];
            p[76 + (t - 96)] = v;
            mv[34 + (t - 96)] = v;
        }
        if (nb < batch) cur = nxt;
    }
}

constexpr int kMaxDevices = 64;
int g_sms[kMaxDevices];
int g_blocks[kMaxDevices]; /* resident CTAs per SM of the streaming kernel */

bool aligned(const void *p, uintptr_t n) { return (reinterpret_cast<uintptr_t>(p) & (n - 1)) == 0; }

} /* namespace */

extern "C" int tb_cuda_prepare_actor_inputs_device(const float *device_obs, const float *device_mission,
                                                   const unsigned char *device_cameras, float *device_proprio_91,
                                                   float *device_mission_49, float *device_tactical_24,
                                                   float *device_prior_15, float *device_lidar_6x2048,
                                                   float *device_camera_luma, size_t batch_size, void *stream) {
    if (!device_obs || !device_mission || !device_cameras || !device_proprio_91 || !device_mission_49 ||
        !device_tactical_24 || !device_prior_15 || !device_lidar_6x2048 || !device_camera_luma ||
        batch_size == 0 || batch_size > 0x7fffffffu)
        return 0;
    /* 128-bit rows: obs (16,592 B), cameras (16,384 B), LiDAR channels, luma */
    if (!aligned(device_obs, 16) || !aligned(device_cameras, 16) || !aligned(device_lidar_6x2048, 16) ||
        !aligned(device_camera_luma, 16) || !aligned(device_mission, 4) || !aligned(device_proprio_91, 4) ||
        !aligned(device_mission_49, 4))
        return 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 0;
    if (!g_sms[dev]) {
        int sms = 0, blocks = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, actor_inputs_kernel, kThreads, 0) != cudaSuccess)
            return 0;
        g_blocks[dev] = blocks > 0 ? blocks : 1;
        g_sms[dev] = sms;
    }
    if (!tb_cuda_extract_onboard_device(device_obs, device_mission, device_tactical_24, device_prior_15,
                                        batch_size, stream))
        return 0;
    cudaGetLastError(); /* report this launch only */
    /* persistent: exactly the resident CTAs */
    unsigned long long grid = static_cast<unsigned long long>(g_sms[dev]) * g_blocks[dev];
    if (grid > batch_size) grid = batch_size;
    actor_inputs_kernel<<<static_cast<unsigned int>(grid), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        device_obs, device_mission, device_cameras, device_tactical_24, device_prior_15, device_proprio_91,
        device_mission_49, device_lidar_6x2048, device_camera_luma, batch_size);
    return cudaGetLastError() == cudaSuccess;
}
