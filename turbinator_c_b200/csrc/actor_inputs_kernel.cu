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
 * and prior; this kernel then streams every aircraft once.  It moves 33,016
 * bytes in and 115,404 bytes out per aircraft, so it is bound by HBM
 * bandwidth, mostly writes.  Inputs are staged the way the feature kernel
 * stages them: a producer warp bulk-copies each aircraft's observation row
 * and camera block (cp.async.bulk, completion counted in bytes on an
 * mbarrier) and its mission, tactical and prior rows (4-byte cp.async on the
 * same mbarrier) into a 3-stage shared-memory ring, so many aircraft are in flight without
 * holding registers; 8 consumer warps convert a staged aircraft and write
 * every output with 128-bit stores cached in L2 only (st.global.cg: 1.517
 * against 1.531 ms per 65,536 aircraft with the evict-first streaming hint),
 * each warp store covering 512
 * contiguous bytes.  Each CTA takes a run of 2 consecutive aircraft (1 when
 * the batch would not fill the resident CTAs) and the grid covers the batch
 * (2 CTAs resident per SM), so the hardware hands CTAs
 * to SMs as they free up: with a persistent grid and a fixed share per CTA
 * the launch ended with its slowest SMs, 1.75 ms against 1.47 ms at 65,536
 * aircraft (runs of 1, 3, 4 and 8: 1.52, 1.50, 1.53 and 1.58 ms).
 * Every mbarrier wait is bounded (about one second); on expiry the kernel
 * ORs a bit into the status word of the stream it was launched on
 * (tb_status.cu), which tb_cuda_synchronize(stream) reports, drains its own
 * outstanding copies (bounded again) and exits.
 *
 * Arithmetic follows the reference kernels' expressions (as nvcc compiles
 * them, i.e. with the multiply-add of the luma contracted), so the values
 * equal the reference's GPU output; the symlog uses CUDA's log1pf exactly
 * as the reference does.
 */
#include <cuda_runtime.h>

#include <stdint.h>

#include "tb_features_internal.h"
#include "tb_onboard_scan.cuh"
#include "tb_pipeline.cuh"
#include "turbinator/training/cuda_features.h"

namespace {

using namespace tb_pipe;

constexpr int kObsDim = 4148;
constexpr int kMissionDim = 10;
constexpr int kCameraBytes = 16384;
constexpr int kProprio = 91;
constexpr int kMissionVec = 49;
constexpr int kLidarBins = 2048; /* per head */
constexpr int kConsumerWarps = 8;
constexpr int kConsumers = 32 * kConsumerWarps;
constexpr int kThreads = kConsumers + 32; /* + the producer warp */

/* Ring geometry: one aircraft per stage (observation row, camera block,
 * mission row, tactical and prior rows), 3 stages of 33,280 bytes per CTA,
 * 2 CTAs per SM. */
constexpr uint32_t kObsBytes = kObsDim * 4u; /* 16,592 = 16 * 1,037 */
constexpr uint32_t kCamOff = kObsBytes;
constexpr uint32_t kMissionOff = kCamOff + kCameraBytes;
constexpr uint32_t kTacticalOff = kMissionOff + kMissionDim * 4;
constexpr uint32_t kPriorOff = kTacticalOff + 24 * 4;
constexpr uint32_t kStageBytes = (kPriorOff + 15 * 4 + 127) / 128 * 128;
constexpr int kStages = 3;
constexpr unsigned long long kMaxChunk = 2; /* aircraft per CTA */
constexpr uint32_t kBarrierRegion = 128;
/* After the ring: the scans' ray tables and per-warp partial results (about
 * 1.5 KB), used in scan mode. */
using ScanShared = tb_scan::BlockScanShared<kConsumerWarps>;
constexpr uint32_t kScanOff = kBarrierRegion + kStages * kStageBytes;
constexpr uint32_t kSmemBytes = kScanOff + (sizeof(ScanShared) + 15) / 16 * 16;
static_assert(kObsBytes % 16 == 0 && kCameraBytes % 16 == 0 && kStageBytes == 33280, "stage layout");
static_assert(2 * (kSmemBytes + 1024) <= 228 * 1024, "two CTAs per SM");
constexpr int kScanBarrier = 1; /* named barrier of the 256 consumer threads */

constexpr unsigned long long kDefaultWaitNs = 1000000000ull; /* ~1 s per wait */

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

struct ActorArgs {
    const float *obs, *mission;
    const unsigned char *cameras;
    const float *tactical, *prior;
    float *proprio, *mission_vec, *lidar, *luma;
    unsigned long long batch;
    unsigned long long chunk; /* CTA c takes aircraft [c*chunk, (c+1)*chunk) */
    unsigned long long wait_ns;
    long long stall_sample; /* test hook: withhold this aircraft's copies; -1 normally */
    unsigned int *status;   /* the launching stream's status word */
    int scan;               /* 0: copy the staged tactical / prior rows into the onboard columns;
                               1: scan the dodge / slalom aircraft's LiDAR rows, park the results in
                               `park` (the prior rows) and leave the onboard columns to the
                               control-law kernel */
    float *park;
};

/* All 256 consumer threads vote; every one of them gets the AND.  Every
 * consumer reaches it once per staged aircraft (after its own bounded wait),
 * so a wait that expired in one warp makes all of them leave together and no
 * consumer is left at a later barrier. */
__device__ __forceinline__ bool consumers_all(bool ok) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(ok)), "n"(kScanBarrier), "n"(kConsumers)
        : "memory");
    return r != 0;
}

/* Sanitised mission value: NaN -> 0, +-inf -> +-1 (onboard_features.cuh:12-14). */
__device__ __forceinline__ float mission_sane(float x) {
    return isnan(x) ? 0.0f : (isinf(x) ? copysignf(1.0f, x) : x);
}
/* Sanitised observation value: NaN -> 0, +-inf -> +-1000. */
__device__ __forceinline__ float obs_sane(float x) {
    return isnan(x) ? 0.0f : (isinf(x) ? copysignf(1000.0f, x) : x);
}

__global__ void __launch_bounds__(kThreads, 2) actor_inputs_kernel(const ActorArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    const uint32_t full_bar = smem_addr(smem);           /* kStages x 8 B */
    const uint32_t empty_bar = full_bar + 8 * kStages;   /* kStages x 8 B */
    unsigned char *stages = smem + kBarrierRegion;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(full_bar + 8 * s, 1);
            mbar_init(empty_bar + 8 * s, kConsumerWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    const unsigned long long first = static_cast<unsigned long long>(blockIdx.x) * a.chunk;
    const unsigned long long last = first + a.chunk < a.batch ? first + a.chunk : a.batch;

    if (warp == kConsumerWarps) {
        /* ---------------- producer warp ---------------- */
        const uint64_t policy = evict_first_policy();
        unsigned long long k = 0;
        bool ok = true;
        for (unsigned long long b = first; b < last; ++b, ++k) {
            const int s = static_cast<int>(k % kStages);
            const uint32_t phase = static_cast<uint32_t>((k / kStages) & 1);
            /* warp-uniform: every lane leaves together or none does */
            if (!__all_sync(0xffffffffu, mbar_wait(empty_bar + 8 * s, phase ^ 1u, a.wait_ns))) {
                ok = false;
                break;
            }
            if (static_cast<long long>(b) == a.stall_sample) continue; /* test hook */
            const uint32_t stage = smem_addr(stages + static_cast<size_t>(s) * kStageBytes);
            /* the 4-byte-aligned rows: mission, tactical, prior (49 floats) */
            if (lane < kMissionDim) async_load4(stage + kMissionOff + 4 * lane, a.mission + b * kMissionDim + lane);
            if (!a.scan) {
                if (lane < 24) async_load4(stage + kTacticalOff + 4 * lane, a.tactical + b * 24 + lane);
                if (lane < 15) async_load4(stage + kPriorOff + 4 * lane, a.prior + b * 15 + lane);
            }
            if (lane < 24) async_track(full_bar + 8 * s);
            __syncwarp();
            if (lane == 0) {
                mbar_arrive_expect_tx(full_bar + 8 * s, kObsBytes + kCameraBytes);
                bulk_load(stage, a.obs + b * kObsDim, kObsBytes, full_bar + 8 * s, policy);
                bulk_load(stage + kCamOff, a.cameras + b * kCameraBytes, kCameraBytes, full_bar + 8 * s, policy);
            }
            __syncwarp();
        }
        if (!ok) {
            if (lane == 0) atomicOr(a.status, TB_FEATURE_STATUS_WAIT_TIMEOUT);
            /* Drain this CTA's outstanding copies before exiting (bounded). */
            const unsigned long long lo = k > kStages ? k - kStages : 0;
            for (unsigned long long j = lo; j < k; ++j)
                mbar_wait(full_bar + 8 * (j % kStages), static_cast<uint32_t>((j / kStages) & 1), a.wait_ns);
        }
        return;
    }

    /* ---------------- consumer warps ---------------- */
    const int t = threadIdx.x; /* 0..255 */
    ScanShared &scan_sh = *reinterpret_cast<ScanShared *>(smem + kScanOff);
    if (a.scan) tb_scan::load_tables(scan_sh.tables, t, kConsumers); /* visible after the first vote */
    unsigned long long k = 0;
    for (unsigned long long b = first; b < last; ++b, ++k) {
        const int s = static_cast<int>(k % kStages);
        const uint32_t phase = static_cast<uint32_t>((k / kStages) & 1);
        bool ok = __all_sync(0xffffffffu, mbar_wait(full_bar + 8 * s, phase, a.wait_ns));
        if (a.scan) ok = consumers_all(ok); /* the scan below synchronises all consumer warps */
        if (!ok) {
            if (lane == 0) atomicOr(a.status, TB_FEATURE_STATUS_WAIT_TIMEOUT);
            return;
        }
        const unsigned char *stage = stages + static_cast<size_t>(s) * kStageBytes;
        const float *o = reinterpret_cast<const float *>(stage);
        const float *m = reinterpret_cast<const float *>(stage + kMissionOff);

        /* LiDAR: float4 q (0..1023) of the scan is head q/512, bins
         * 4*(q%512)..; it feeds channels head, 2+head and 4+head.  Each warp
         * store covers 512 contiguous bytes of one channel row. */
        float *lo = a.lidar + b * (6ull * kLidarBins);
        const float4 *scan = reinterpret_cast<const float4 *>(o + 48);
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
            const int q = q4 * kConsumers + t;
            const int head = q >> 9;
            const int bin4 = q & 511;
            const float4 r = scan[q];
            const LidarChannels c0 = lidar_value(r.x), c1 = lidar_value(r.y), c2 = lidar_value(r.z),
                                c3 = lidar_value(r.w);
            __stcg(reinterpret_cast<float4 *>(lo + head * kLidarBins) + bin4,
                   make_float4(c0.inverse, c1.inverse, c2.inverse, c3.inverse));
            __stcg(reinterpret_cast<float4 *>(lo + (2 + head) * kLidarBins) + bin4,
                   make_float4(c0.scaled, c1.scaled, c2.scaled, c3.scaled));
            __stcg(reinterpret_cast<float4 *>(lo + (4 + head) * kLidarBins) + bin4,
                   make_float4(c0.flag, c1.flag, c2.flag, c3.flag));
        }
        /* Luma: camera word c (bytes 4c..4c+3) -> output float4 c. */
        float4 *lu = reinterpret_cast<float4 *>(a.luma + b * kCameraBytes);
        const uint32_t *cw = reinterpret_cast<const uint32_t *>(stage + kCamOff);
#pragma unroll
        for (int w = 0; w < 16; ++w) __stcg(lu + w * kConsumers + t, luma4(cw[w * kConsumers + t]));

        /* Scalars (network_gpu.cu:285-302). */
        float *p = a.proprio + b * kProprio;
        float *mv = a.mission_vec + b * kMissionVec;
        if (t < 52) {
            float raw = t < 48 ? o[t] : o[4144 + t - 48];
            raw = isfinite(raw) ? fmaxf(-1000.0f, fminf(1000.0f, raw)) : 0.0f;
            const float symlog = copysignf(log1pf(fabsf(raw * symlog_scale(t))), raw);
            p[t] = fmaxf(-8.0f, fminf(8.0f, symlog / sqrtf(1.0001f)));
        } else if (t < 52 + kMissionDim) {
            const float mm = m[t - 52];
            mv[t - 52] = isfinite(mm) ? mm : 0.0f;
        } else if (a.scan) {
            /* the control-law kernel writes the onboard columns */
        } else if (t >= 64 && t < 64 + 24) {
            const float v = reinterpret_cast<const float *>(stage + kTacticalOff)[t - 64];
            p[52 + (t - 64)] = v;
            mv[10 + (t - 64)] = v;
        } else if (t >= 96 && t < 96 + 15) {
            const float v = reinterpret_cast<const float *>(stage + kPriorOff)[t - 96];
            p[76 + (t - 96)] = v;
            mv[34 + (t - 96)] = v;
        }

        /* Onboard LiDAR scans of a dodge or slalom aircraft (onboard_features.cuh:
         * 185-239) from its staged row, by all consumer warps; the results
         * go to the first six floats of its prior row for the control law. */
        if (a.scan) {
            const float m4 = mission_sane(m[4]), m5 = mission_sane(m[5]);
            const bool dodge = m5 > 0.75f;
            const bool slalom = m4 > 0.75f && !(m4 > 0.75f && m5 > 0.25f);
            if (dodge || slalom) { /* the same in every consumer thread */
                const tb_scan::Attitude at =
                    tb_scan::attitude_from(obs_sane(o[6]), obs_sane(o[7]), obs_sane(o[8]), obs_sane(o[9]));
                const tb_scan::RayStats st =
                    tb_scan::block_scan<kConsumerWarps>(scan_sh, o + 48, o + 48 + kLidarBins, at, obs_sane(o[1]),
                                                        dodge, slalom, warp, lane, kScanBarrier);
                if (t == 0) tb_scan::park_stats(a.park + b * 15, st);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty_bar + 8 * s);
    }
}

constexpr int kMaxDevices = 64;
int g_resident[kMaxDevices]; /* CTAs resident at once on this device (0: not set up) */

bool aligned(const void *p, uintptr_t n) { return (reinterpret_cast<uintptr_t>(p) & (n - 1)) == 0; }

} /* namespace */

/* Launches the streaming kernel; opts may be NULL (its wait_ns and
 * stall_sample fields are honoured).  scan selects the mode (ActorArgs). */
static int actor_launch(const float *obs, const float *mission, const unsigned char *cameras, const float *tactical,
                        const float *prior, float *proprio, float *mission_vec, float *lidar, float *luma,
                        size_t batch, void *stream, const tb_features_launch_opts *opts, float *park) {
    if (batch == 0 || batch > 0x7fffffffu) return 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 0;
    if (!g_resident[dev]) {
        int sms = 0, blocks = 0;
        if (cudaFuncSetAttribute(actor_inputs_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kSmemBytes)) != cudaSuccess ||
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, actor_inputs_kernel, kThreads, kSmemBytes) !=
                cudaSuccess)
            return 0;
        g_resident[dev] = sms * (blocks > 0 ? blocks : 1);
    }
    ActorArgs a;
    a.obs = obs;
    a.mission = mission;
    a.cameras = cameras;
    a.tactical = tactical;
    a.prior = prior;
    a.proprio = proprio;
    a.mission_vec = mission_vec;
    a.lidar = lidar;
    a.luma = luma;
    a.batch = batch;
    a.wait_ns = (opts && opts->wait_ns) ? opts->wait_ns : kDefaultWaitNs;
    a.stall_sample = opts ? opts->stall_sample : -1;
    a.status = tb_status_slot(stream);
    if (!a.status) return 0;
    a.scan = park != nullptr;
    a.park = park;
    cudaGetLastError(); /* report this launch only */
    /* runs of up to kMaxChunk aircraft, but no fewer CTAs than fit at once */
    const unsigned long long resident = static_cast<unsigned long long>(g_resident[dev]);
    const unsigned long long fill = (batch + resident - 1) / resident;
    a.chunk = fill < kMaxChunk ? fill : kMaxChunk;
    const unsigned long long grid = (batch + a.chunk - 1) / a.chunk;
    actor_inputs_kernel<<<static_cast<unsigned int>(grid), kThreads, kSmemBytes, static_cast<cudaStream_t>(stream)>>>(a);
    return cudaGetLastError() == cudaSuccess;
}

extern "C" int tb_actor_inputs_launch(const float *obs, const float *mission, const unsigned char *cameras,
                                      const float *tactical, const float *prior, float *proprio,
                                      float *mission_vec, float *lidar, float *luma, size_t batch, void *stream,
                                      const tb_features_launch_opts *opts) {
    if (!tactical || !prior) return 0;
    return actor_launch(obs, mission, cameras, tactical, prior, proprio, mission_vec, lidar, luma, batch, stream,
                        opts, nullptr);
}

extern "C" int tb_actor_inputs_scan_launch(const float *obs, const float *mission, const unsigned char *cameras,
                                           float *prior, float *proprio, float *mission_vec, float *lidar,
                                           float *luma, size_t batch, void *stream,
                                           const tb_features_launch_opts *opts) {
    if (!prior) return 0;
    return actor_launch(obs, mission, cameras, nullptr, nullptr, proprio, mission_vec, lidar, luma, batch, stream,
                        opts, prior);
}

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
    /* One pass over the staged rows (learner tensors, and the LiDAR scans of
     * the dodge and slalom aircraft parked in their prior rows), then the
     * control law, which writes tactical, prior and the onboard columns of
     * the proprio and mission rows. */
    if (!tb_actor_inputs_scan_launch(device_obs, device_mission, device_cameras, device_prior_15, device_proprio_91,
                                     device_mission_49, device_lidar_6x2048, device_camera_luma, batch_size, stream,
                                     nullptr))
        return 0;
    return tb_onboard_control_launch(device_obs, device_mission, device_tactical_24, device_prior_15, batch_size,
                                     stream, device_proprio_91, device_mission_49);
}
