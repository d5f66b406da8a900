/*
 * sm_100a kernels for the 142 sensor features, plus the thin extern "C"
 * launch shim that replaces the reference's device entry points
 * (Viatreen/Turbinator_C src/cuda/features.cu:90-173).
 *
 * What is computed per aircraft (reference CPU path training.c:102-142):
 *   f[0..47]    clamp(finite(obs[i]) / divisor_i, -1, 1)
 *   f[48..51]   clamp(finite(obs[4144+i]), 0, 1)
 *   f[52..61]   clamp(finite(mission[i]), -1, 1); 59..61 are 0 when
 *               finite(mission[6]) > 0.5 (arena: opponent truth hidden)
 *   f[62..125]  mean over a 4x16 LiDAR sector of
 *               (-1 if !finite(r) or r < 0, else log1p(min(r,120))/log1p(120))
 *   f[126..141] camera quadrant byte sum / (1024 * 255)
 *
 * Design (B200):
 *  - The path is a streaming reduction: 33,016 bytes in and 568 bytes out
 *    per aircraft, ~1 flop per byte.  It is bound by HBM bandwidth, so the
 *    kernel is built to keep enough bytes in flight and to touch every byte
 *    exactly once.
 *  - u8 cameras (the reference ABI): features_flat_kernel, one CTA per
 *    aircraft with 128-bit streaming loads straight into registers (below);
 *    it times at or below the staged ring at every batch size.
 *  - FP32 cameras (82 KB per aircraft) and the test hooks: the staged
 *    kernel, CTAs of one producer warp and eight consumer warps.  With u8
 *    cameras it takes runs of up to 8 consecutive aircraft over a covering
 *    grid; with FP32 cameras a persistent grid (one CTA per SM, whose ring
 *    would drain at every CTA change).  The producer streams each aircraft's
 *    observation row (16,592 B) and camera block (16,384 B) into a
 *    shared-memory ring with 1-D bulk copies (cp.async.bulk, completion
 *    counted in bytes on an mbarrier) and its 40-byte mission row with
 *    4-byte cp.async tracked on the same mbarrier.  No multicast anywhere.
 *  - The eight consumer warps reduce one staged aircraft together.  Warp w
 *    owns LiDAR rows 4w..4w+3 (one head x elevation-sector band, i.e. eight
 *    sectors) and half-camera w (camera w/2, rows 32*(w&1)..+31); all
 *    shared-memory reads are 128-bit and conflict-free.  Per-sector and
 *    per-quadrant partials are combined with warp shuffles.
 *  - Exactness: the scalar, mission and camera features are bit-identical
 *    to the reference (IEEE division, integer byte sums, the reference's
 *    compare-based clamp).  A LiDAR sector mean is computed as
 *    (n_saturated - n_invalid + K * sum log2(1 + r)) / 64 over the
 *    in-range bins, with K = 1/log2(121).  Saturated (>= 120 m) and invalid
 *    bins therefore contribute exact integers -- an all-no-return sector is
 *    exactly 1.0 and an all-invalid one exactly -1.0, as in the reference --
 *    and only in-range bins carry the lg2 approximation error (well inside
 *    the 1e-6 absolute / 1e-5 relative tolerance of the parity tests).
 *  - Every mbarrier wait is bounded (about one second of %globaltimer);
 *    on expiry the kernel ORs a bit into the status word of the stream it
 *    was launched on (tb_status.cu), which tb_cuda_synchronize(stream)
 *    reports, drains its own outstanding copies (bounded again) and exits.
 */
#include <cuda_runtime.h>

#include <atomic>
#include <stdint.h>

#include "turbinator/training/cuda_features.h"
#include "tb_features_internal.h"
#include "tb_pipeline.cuh"

namespace {

constexpr int kObsDim = 4148;
constexpr int kMissionDim = 10;
constexpr int kCameraBytes = 16384;
constexpr int kFeatureDim = 142;
constexpr int kLidarOffset = 48;
constexpr int kTailOffset = 4144;

constexpr uint32_t kObsBytes = kObsDim * 4u;                  /* 16,592 = 16 * 1,037 */
static_assert(kObsBytes % 16 == 0 && kCameraBytes % 16 == 0, "bulk copy sizes");

constexpr int kConsumerWarps = 8;
constexpr int kThreads = 32 * (kConsumerWarps + 1);
constexpr uint32_t kBarrierRegion = 128;

/* Shared-memory ring geometry per camera format.  A stage holds one
 * aircraft: observation row, camera block, mission row.  u8 cameras: 33 KB
 * stages, 3 per CTA, 2 CTAs per SM, runs of `chunk` aircraft per CTA; FP32
 * cameras: 82 KB stages, 2 per CTA, 1 persistent CTA per SM.  Either way
 * ~160-200 KB per SM are in flight. */
template <bool kF32Cam>
struct Ring {
    static constexpr uint32_t camera_bytes = kF32Cam ? 4u * kCameraBytes : kCameraBytes;
    static constexpr uint32_t cam_off = kObsBytes;
    static constexpr uint32_t mission_off = cam_off + camera_bytes;
    static constexpr uint32_t stage_bytes = (mission_off + kMissionDim * 4 + 127) / 128 * 128;
    static constexpr int stages = kF32Cam ? 2 : 3;
    static constexpr int min_blocks = kF32Cam ? 1 : 2;
    static constexpr uint32_t smem_bytes = kBarrierRegion + stages * stage_bytes;
    static constexpr unsigned long long max_chunk = kF32Cam ? 0 : 8; /* 0: persistent grid-stride */
};
static_assert(Ring<false>::stage_bytes == 33024 && Ring<true>::stage_bytes == 82176, "stage layout");

/* 1 / log2(121): a LiDAR term log1p(x)/log1p(120) equals log2(1+x) times this. */
constexpr float kInvLog2_121 = 0.14453241315894394f;

constexpr unsigned long long kDefaultWaitNs = 1000000000ull; /* ~1 s per wait */



using namespace tb_pipe; /* staging primitives, tb_pipeline.cuh */

/* Bounds checks of the debug build (compiled with TB_FEATURES_DEBUG): every
 * global load and store index of the feature kernels is compared with the
 * extent of its buffer (batch rows); an index outside ORs
 * TB_FEATURE_STATUS_BOUNDS into the launching stream's status word, which
 * tb_cuda_synchronize then reports, and the access is skipped.  In the
 * product build the check is the constant true and compiles away. */
__device__ __forceinline__ bool within(unsigned long long index, unsigned long long count, unsigned int *status) {
#ifdef TB_FEATURES_DEBUG
    if (index < count) return true;
    atomicOr(status, TB_FEATURE_STATUS_BOUNDS);
    return false;
#else
    (void)index;
    (void)count;
    (void)status;
    return true;
#endif
}

/* ------------------------------------------------------------------ */
/* Per-feature arithmetic shared by both kernels. */

/* Reference training.c:57-59 clamp; the compare form fixes zero signs. */
__device__ __forceinline__ float clamp_ref(float x, float lo, float hi) {
    return x < lo ? lo : (x > hi ? hi : x);
}

__device__ __forceinline__ float finite_or_zero(float x) {
    return isfinite(x) ? x : 0.0f;
}

/* Divisors of the 48 proprioceptive values (training.c:70-81). */
__device__ __forceinline__ float scalar_divisor(int i) {
    const float pi = 3.14159265358979323846f;
    float d = 1.0f;
    d = (i <= 1) ? 300.0f : d;
    d = (i == 2) ? 100.0f : d;
    d = (i >= 3 && i <= 5) ? 50.0f : d;
    d = (i >= 10 && i <= 12) ? 5.0f : d;
    d = (i >= 13 && i <= 15) ? 30.0f : d;
    d = (i >= 28 && i <= 31) ? pi / 4.0f : d;
    d = (i >= 32 && i <= 39) ? 5.0f : d;
    d = (i == 44 || i == 45) ? pi / 2.0f : d;
    return d;
}

/* Feature t in [0, 62) from the observation row `o` and mission row `m`. */
__device__ __forceinline__ float scalar_feature(int t, const float *o, const float *m) {
    if (t < 48) return clamp_ref(__fdiv_rn(finite_or_zero(o[t]), scalar_divisor(t)), -1.0f, 1.0f);
    if (t < 52) return clamp_ref(finite_or_zero(o[kTailOffset + t - 48]), 0.0f, 1.0f);
    const int i = t - 52;
    const bool arena = finite_or_zero(m[6]) > 0.5f;
    const float v = (i >= 7 && arena) ? 0.0f : m[i];
    return clamp_ref(finite_or_zero(v), -1.0f, 1.0f);
}

/* LiDAR sector accumulator: `sum` adds log2(1+r) over bins with
 * 0 <= r < 120; `counts` packs n_in_range (low byte) and n_saturated
 * (120 <= r < inf, second byte).  Invalid bins (NaN, +-inf, r < 0) are
 * 64 - n_in_range - n_saturated. */
__device__ __forceinline__ void lidar_bin(float r, float &sum, int &counts) {
    const bool in_range = (r >= 0.0f) && (r < 120.0f);
    const bool saturated = (r >= 120.0f) && (r < __int_as_float(0x7f800000));
    const float lg = __log2f(1.0f + r);
    sum += in_range ? lg : 0.0f;
    counts += (in_range ? 1 : 0) + (saturated ? 256 : 0);
}

__device__ __forceinline__ void lidar_bins4(const float4 v, float &sum, int &counts) {
    lidar_bin(v.x, sum, counts);
    lidar_bin(v.y, sum, counts);
    lidar_bin(v.z, sum, counts);
    lidar_bin(v.w, sum, counts);
}

/* Mean of a 64-bin sector from its reduced accumulator. */
__device__ __forceinline__ float lidar_sector_mean(float sum, int counts) {
    const int n_in = counts & 255;
    const int n_sat = counts >> 8;
    const float integral = static_cast<float>(2 * n_sat + n_in - 64); /* n_sat - n_invalid */
    return __fmaf_rn(sum, kInvLog2_121, integral) * (1.0f / 64.0f);
}

__device__ __forceinline__ float camera_feature(unsigned int sum) {
    return __fdiv_rn(static_cast<float>(sum), 1024.0f * 255.0f);
}

__device__ __forceinline__ uint32_t byte_sum4(uint32_t w, uint32_t acc) {
    return __dp4a(w, 0x01010101u, acc);
}

/* Byte sum of one camera quadrant from a warp's half image: lane holds the
 * 16-byte chunks lane, lane+32, lane+64, lane+96 of the half (chunk c in row
 * c/4, columns 16*(c%4).., so quadrant x = lane bit 1); the result is valid
 * in every lane, for the lane's quadrant. */
__device__ __forceinline__ uint32_t quadrant_bytes(const uint4 c0, const uint4 c1, const uint4 c2,
                                                   const uint4 c3) {
    uint32_t bytes = 0;
    bytes = byte_sum4(c0.x, bytes); bytes = byte_sum4(c0.y, bytes);
    bytes = byte_sum4(c0.z, bytes); bytes = byte_sum4(c0.w, bytes);
    bytes = byte_sum4(c1.x, bytes); bytes = byte_sum4(c1.y, bytes);
    bytes = byte_sum4(c1.z, bytes); bytes = byte_sum4(c1.w, bytes);
    bytes = byte_sum4(c2.x, bytes); bytes = byte_sum4(c2.y, bytes);
    bytes = byte_sum4(c2.z, bytes); bytes = byte_sum4(c2.w, bytes);
    bytes = byte_sum4(c3.x, bytes); bytes = byte_sum4(c3.y, bytes);
    bytes = byte_sum4(c3.z, bytes); bytes = byte_sum4(c3.w, bytes);
    bytes += __shfl_xor_sync(0xffffffffu, bytes, 1);
    bytes += __shfl_xor_sync(0xffffffffu, bytes, 4);
    bytes += __shfl_xor_sync(0xffffffffu, bytes, 8);
    bytes += __shfl_xor_sync(0xffffffffu, bytes, 16);
    return bytes;
}

/* Sector accumulators of a warp's four LiDAR rows: lane holds bins
 * 4*lane..4*lane+3 of each row, i.e. sector lane/4; reduced over the four
 * lanes of each sector. */
__device__ __forceinline__ void lidar_band(const float4 r0, const float4 r1, const float4 r2, const float4 r3,
                                           float &sum, int &counts) {
    sum = 0.0f;
    counts = 0;
    lidar_bins4(r0, sum, counts);
    lidar_bins4(r1, sum, counts);
    lidar_bins4(r2, sum, counts);
    lidar_bins4(r3, sum, counts);
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    counts += __shfl_xor_sync(0xffffffffu, counts, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    counts += __shfl_xor_sync(0xffffffffu, counts, 2);
}

/* The simulator's camera quantisation (reference src/sim/sensors.c:67 with
 * the clamp of src/sim/sim_internal.h:73): fmax(0, fmin(255, round(v*255)))
 * in double, so NaN gives 255.  Evaluated exactly in float, as a float byte
 * value: NaN is tested explicitly (a fused clamp would send it to 0);
 * clamping other values to [0, 1] first gives the same byte.  v*255 is formed
 * as hi + lo with lo the exact FMA residual; hi is rounded to the nearest
 * integer, ties to even, by adding and subtracting 2^23 (exact for
 * 0 <= hi <= 255).  Only when hi is itself a half-integer can that differ from
 * rounding the exact product half away from zero (half-integers below 256
 * are floats, so no other rounding boundary lies between hi and hi + lo);
 * there the byte is hi + 0.5 when lo >= 0 and hi - 0.5 when lo < 0 (an exact
 * residual of zero is +0).  Checked against round-half-away of v*255 in
 * double for every float in [0, 1]. */
__device__ __forceinline__ float luma_byte(float v) {
    const float c = fmaxf(fminf(v, 1.0f), 0.0f);
    const float hi = __fmul_rn(c, 255.0f);
    const float lo = __fmaf_rn(c, 255.0f, -hi);
    const float r = __fsub_rn(__fadd_rn(hi, 8388608.0f), 8388608.0f);
    const float q = fabsf(__fsub_rn(r, hi)) == 0.5f ? __fadd_rn(hi, copysignf(0.5f, lo)) : r;
    return v != v ? 255.0f : q;
}

__device__ __forceinline__ float luma_bytes4(const float4 v) {
    return (luma_byte(v.x) + luma_byte(v.y)) + (luma_byte(v.z) + luma_byte(v.w));
}

/* ------------------------------------------------------------------ */
/* Staged kernel: warp-specialised bulk-copy pipeline over runs of aircraft
 * (or a persistent grid-stride loop when a.chunk is 0). */

struct StagedArgs {
    const float *obs;
    const float *mission;
    const void *cameras; /* u8 or f32 camera rows; may be NULL */
    float *features;
    unsigned long long batch;
    unsigned long long chunk; /* > 0: CTA c takes aircraft [c*chunk, (c+1)*chunk); 0: grid-stride */
    unsigned long long wait_ns;
    long long stall_sample; /* test hook: >= 0 withholds that sample's copies */
    unsigned int *status;   /* the launching stream's status word */
};

template <bool kF32Cam>
__global__ void __launch_bounds__(kThreads, Ring<kF32Cam>::min_blocks)
    features_staged_kernel(const StagedArgs a) {
    using R = Ring<kF32Cam>;
    extern __shared__ __align__(128) unsigned char smem[];
    const uint32_t full_bar = smem_addr(smem);            /* R::stages x 8 B */
    const uint32_t empty_bar = full_bar + 8 * R::stages;   /* R::stages x 8 B */
    unsigned char *stages = smem + kBarrierRegion;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < R::stages; ++s) {
            mbar_init(full_bar + 8 * s, 1);
            mbar_init(empty_bar + 8 * s, kConsumerWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    unsigned long long first = blockIdx.x, last = a.batch, step = gridDim.x;
    if (a.chunk) {
        first = static_cast<unsigned long long>(blockIdx.x) * a.chunk;
        last = first + a.chunk < a.batch ? first + a.chunk : a.batch;
        step = 1;
    }

    if (warp == kConsumerWarps) {
        /* ---------------- producer warp ---------------- */
        const uint64_t policy = evict_first_policy();
        const uint32_t tx_bytes = kObsBytes + (a.cameras ? R::camera_bytes : 0u);
        const unsigned char *cameras = static_cast<const unsigned char *>(a.cameras);
        unsigned long long k = 0;
        bool ok = true;
        for (unsigned long long sample = first; sample < last; sample += step, ++k) {
            const int s = static_cast<int>(k % R::stages);
            const uint32_t phase = static_cast<uint32_t>((k / R::stages) & 1);
            /* warp-uniform: every lane leaves together or none does */
            if (!__all_sync(0xffffffffu, mbar_wait(empty_bar + 8 * s, phase ^ 1u, a.wait_ns))) {
                ok = false;
                break;
            }
            if (static_cast<long long>(sample) == a.stall_sample) continue; /* test hook */
            /* debug build: a source row outside its buffer is not copied (the
             * stage's consumers then time out and report it too) */
            if (!within((sample + 1) * kObsDim - 1, a.batch * kObsDim, a.status) ||
                !within((sample + 1) * kMissionDim - 1, a.batch * kMissionDim, a.status) ||
                (cameras && !within((sample + 1) * R::camera_bytes - 1, a.batch * R::camera_bytes, a.status)))
                continue;
            const uint32_t stage = smem_addr(stages + static_cast<size_t>(s) * R::stage_bytes);
            if (lane < kMissionDim) {
                async_load4(stage + R::mission_off + 4 * lane, a.mission + sample * kMissionDim + lane);
                async_track(full_bar + 8 * s);
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive_expect_tx(full_bar + 8 * s, tx_bytes);
                bulk_load(stage, a.obs + sample * kObsDim, kObsBytes, full_bar + 8 * s, policy);
                if (cameras)
                    bulk_load(stage + R::cam_off, cameras + sample * R::camera_bytes, R::camera_bytes,
                              full_bar + 8 * s, policy);
            }
            __syncwarp();
        }
        if (!ok) {
            if (lane == 0) atomicOr(a.status, TB_FEATURE_STATUS_WAIT_TIMEOUT);
            /* Drain this CTA's outstanding copies before exiting (bounded). */
            const unsigned long long issued = k;
            const unsigned long long lo = issued > R::stages ? issued - R::stages : 0;
            for (unsigned long long j = lo; j < issued; ++j)
                mbar_wait(full_bar + 8 * (j % R::stages), static_cast<uint32_t>((j / R::stages) & 1),
                          a.wait_ns);
        }
        return;
    }

    /* ---------------- consumer warps ---------------- */
    const int head = warp >> 2;          /* LiDAR rows 4w..4w+3 = head, elevation sector */
    const int el_sector = warp & 3;
    const int cam = warp >> 1;           /* camera half-image w */
    const int qy = warp & 1;
    unsigned long long k = 0;
    for (unsigned long long sample = first; sample < last; sample += step, ++k) {
        const int s = static_cast<int>(k % R::stages);
        const uint32_t phase = static_cast<uint32_t>((k / R::stages) & 1);
        if (!__all_sync(0xffffffffu, mbar_wait(full_bar + 8 * s, phase, a.wait_ns))) {
            if (lane == 0) atomicOr(a.status, TB_FEATURE_STATUS_WAIT_TIMEOUT);
            return;
        }
        const unsigned char *stage = stages + static_cast<size_t>(s) * R::stage_bytes;
        const float *o = reinterpret_cast<const float *>(stage);
        const float *m = reinterpret_cast<const float *>(stage + R::mission_off);

        /* LiDAR: lane covers bins 4*lane..4*lane+3 of the warp's four rows;
         * all 16 values belong to sector (head, el_sector, lane/4). */
        const float4 *rows = reinterpret_cast<const float4 *>(o + kLidarOffset) +
                             (head * 16 + el_sector * 4) * 32 + lane;
        const float4 r0 = rows[0], r1 = rows[32], r2 = rows[64], r3 = rows[96];
        float scalar = 0.0f;
        const int t = warp * 32 + lane;
        if (t < 62) scalar = scalar_feature(t, o, m);

        /* Camera half-image (camera w/2, rows 32*(w&1)..+31). */
        uint32_t bytes = 0;      /* u8: integer byte sum */
        float luma = 0.0f;       /* f32: sum of quantised bytes, exact in float */
        if constexpr (!kF32Cam) {
            /* 16-byte chunk c (c = lane, lane+32, ...) sits in row c/4,
             * columns 16*(c%4).., so quadrant x = lane bit 1. */
            uint4 c0 = make_uint4(0, 0, 0, 0), c1 = c0, c2 = c0, c3 = c0;
            if (a.cameras) {
                const uint4 *half = reinterpret_cast<const uint4 *>(stage + R::cam_off) +
                                    cam * 256 + qy * 128 + lane;
                c0 = half[0]; c1 = half[32]; c2 = half[64]; c3 = half[96];
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty_bar + 8 * s); /* stage fully read: release it */
            bytes = quadrant_bytes(c0, c1, c2, c3);
        } else {
            /* float4 chunk c (c = lane, lane+32, ...) sits in row c/16,
             * columns 4*(c%16).., so quadrant x = lane bit 3. */
            if (a.cameras) {
                const float4 *half = reinterpret_cast<const float4 *>(stage + R::cam_off) +
                                     cam * 1024 + qy * 512 + lane;
#pragma unroll 4
                for (int i = 0; i < 16; ++i) luma += luma_bytes4(half[32 * i]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty_bar + 8 * s); /* stage fully read: release it */
            luma += __shfl_xor_sync(0xffffffffu, luma, 1);
            luma += __shfl_xor_sync(0xffffffffu, luma, 2);
            luma += __shfl_xor_sync(0xffffffffu, luma, 4);
            luma += __shfl_xor_sync(0xffffffffu, luma, 16);
        }

        float sum;
        int counts;
        lidar_band(r0, r1, r2, r3, sum, counts);

        float *f = a.features + sample * kFeatureDim;
        const unsigned long long out_first = sample * kFeatureDim, out_count = a.batch * kFeatureDim;
        const int lidar_j = 62 + head * 32 + el_sector * 8 + (lane >> 2);
        if ((lane & 3) == 0 && within(out_first + lidar_j, out_count, a.status))
            f[lidar_j] = lidar_sector_mean(sum, counts);
        if constexpr (!kF32Cam) {
            const int cam_j = 126 + cam * 4 + qy * 2 + (lane >> 1);
            if ((lane == 0 || lane == 2) && within(out_first + cam_j, out_count, a.status))
                f[cam_j] = camera_feature(bytes);
        } else {
            const int cam_j = 126 + cam * 4 + qy * 2 + (lane >> 3);
            if ((lane == 0 || lane == 8) && within(out_first + cam_j, out_count, a.status))
                f[cam_j] = __fdiv_rn(luma, 1024.0f * 255.0f);
        }
        if (t < 62 && within(out_first + t, out_count, a.status)) f[t] = scalar;
    }
}

/* ------------------------------------------------------------------ */
/* Flat kernel, the u8-camera product kernel: one 256-thread CTA per aircraft
 * (grid = batch), each warp loading its share -- LiDAR rows 4w..4w+3 and
 * half-camera w, the staged kernel's consumer-warp roles -- straight into
 * registers with 128-bit streaming loads, 32 KB of the aircraft's 33 KB in
 * flight at once and 5 CTAs per SM.  The hardware hands the CTAs to SMs as
 * they free up, so the launch neither waits on ring refills nor ends with its
 * slowest SMs: 7.1 TB/s of algorithmic bytes at 65,536 aircraft (the best
 * read stream measured on this pool) and the whole of a small batch (config
 * 1) requested in the first wave.  Same arithmetic as the staged kernel; no
 * waits (the status word receives only the debug build's bounds bit). */
__global__ void __launch_bounds__(kConsumerWarps * 32) features_flat_kernel(const float *__restrict__ obs,
                                                                           const float *__restrict__ mission,
                                                                           const unsigned char *__restrict__ cameras,
                                                                           float *__restrict__ features,
                                                                           unsigned long long batch,
                                                                           unsigned int *__restrict__ status) {
    const unsigned long long sample = blockIdx.x;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int head = warp >> 2, el_sector = warp & 3; /* LiDAR rows 4w..4w+3 */
    const int cam = warp >> 1, qy = warp & 1;         /* camera half-image w */
    const float *o = obs + sample * kObsDim;
    const float *m = mission + sample * kMissionDim;

    const int chunk = (head * 16 + el_sector * 4) * 32 + lane; /* float4 of the scan: 32 per row */
    const float4 *rows = reinterpret_cast<const float4 *>(o + kLidarOffset) + chunk;
    float4 r0 = make_float4(0.0f, 0.0f, 0.0f, 0.0f), r1 = r0, r2 = r0, r3 = r0;
    if (within(sample * kObsDim + kLidarOffset + 4 * (chunk + 96) + 3, batch * kObsDim, status)) {
        r0 = __ldcs(rows);
        r1 = __ldcs(rows + 32);
        r2 = __ldcs(rows + 64);
        r3 = __ldcs(rows + 96);
    }
    uint4 c0 = make_uint4(0, 0, 0, 0), c1 = c0, c2 = c0, c3 = c0;
    const int cam_chunk = cam * 256 + qy * 128 + lane; /* uint4 of the camera block */
    if (cameras && within(sample * kCameraBytes + 16 * (cam_chunk + 96) + 15, batch * kCameraBytes, status)) {
        const uint4 *half = reinterpret_cast<const uint4 *>(cameras + sample * kCameraBytes) + cam_chunk;
        c0 = __ldcs(half);
        c1 = __ldcs(half + 32);
        c2 = __ldcs(half + 64);
        c3 = __ldcs(half + 96);
    }
    const int t = warp * 32 + lane;
    float scalar = 0.0f;
    if (t < 62 && within((sample + 1) * kObsDim - 1, batch * kObsDim, status) &&
        within((sample + 1) * kMissionDim - 1, batch * kMissionDim, status))
        scalar = scalar_feature(t, o, m);

    const uint32_t bytes = quadrant_bytes(c0, c1, c2, c3);
    float sum;
    int counts;
    lidar_band(r0, r1, r2, r3, sum, counts);

    float *f = features + sample * kFeatureDim;
    const unsigned long long out_count = batch * kFeatureDim;
    const int lidar_j = 62 + head * 32 + el_sector * 8 + (lane >> 2);
    const int cam_j = 126 + cam * 4 + qy * 2 + (lane >> 1);
    if ((lane & 3) == 0 && within(sample * kFeatureDim + lidar_j, out_count, status))
        f[lidar_j] = lidar_sector_mean(sum, counts);
    if ((lane == 0 || lane == 2) && within(sample * kFeatureDim + cam_j, out_count, status))
        f[cam_j] = camera_feature(bytes);
    if (t < 62 && within(sample * kFeatureDim + t, out_count, status)) f[t] = scalar;
}

/* ------------------------------------------------------------------ */
/* Direct kernel for rows that are not 16-byte aligned: one warp per
 * aircraft, plain loads, same arithmetic. */

template <bool kF32Cam>
__global__ void __launch_bounds__(256) features_direct_kernel(const float *obs, const float *mission,
                                                              const void *cameras, float *features,
                                                              unsigned long long batch, unsigned int *status) {
    const int lane = threadIdx.x & 31;
    const unsigned long long warps = (static_cast<unsigned long long>(gridDim.x) * blockDim.x) >> 5;
    for (unsigned long long sample = (static_cast<unsigned long long>(blockIdx.x) * blockDim.x +
                                      threadIdx.x) >> 5;
         sample < batch; sample += warps) {
        const float *o = obs + sample * kObsDim;
        const float *m = mission + sample * kMissionDim;
        float *f = features + sample * kFeatureDim;
        /* debug build: the rows this warp reads and writes lie in their buffers */
        if (!within((sample + 1) * kObsDim - 1, batch * kObsDim, status) ||
            !within((sample + 1) * kMissionDim - 1, batch * kMissionDim, status) ||
            !within((sample + 1) * kFeatureDim - 1, batch * kFeatureDim, status) ||
            (cameras && !within((sample + 1) * kCameraBytes - 1, batch * kCameraBytes, status)))
            continue;
        for (int band = 0; band < 8; ++band) { /* head * 4 + el_sector */
            float sum = 0.0f;
            int counts = 0;
            for (int row = 0; row < 4; ++row) {
                const float *bins = o + kLidarOffset + (band * 4 + row) * 128 + 4 * lane;
                lidar_bin(bins[0], sum, counts);
                lidar_bin(bins[1], sum, counts);
                lidar_bin(bins[2], sum, counts);
                lidar_bin(bins[3], sum, counts);
            }
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            counts += __shfl_xor_sync(0xffffffffu, counts, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            counts += __shfl_xor_sync(0xffffffffu, counts, 2);
            if ((lane & 3) == 0) f[62 + band * 8 + (lane >> 2)] = lidar_sector_mean(sum, counts);
        }
        for (int half = 0; half < 8; ++half) { /* camera * 2 + qy; lane covers columns 2*lane, +1 */
            float value = 0.0f;
            if constexpr (!kF32Cam) {
                unsigned int bytes = 0;
                if (cameras) {
                    const unsigned char *px = static_cast<const unsigned char *>(cameras) +
                                              sample * kCameraBytes + half * 2048 + 2 * lane;
                    for (int y = 0; y < 32; ++y) bytes += px[y * 64] + px[y * 64 + 1];
                }
                bytes += __shfl_xor_sync(0xffffffffu, bytes, 1);
                bytes += __shfl_xor_sync(0xffffffffu, bytes, 2);
                bytes += __shfl_xor_sync(0xffffffffu, bytes, 4);
                bytes += __shfl_xor_sync(0xffffffffu, bytes, 8);
                value = camera_feature(bytes);
            } else {
                float luma = 0.0f;
                if (cameras) {
                    const float *px = static_cast<const float *>(cameras) + sample * kCameraBytes +
                                      half * 2048 + 2 * lane;
                    for (int y = 0; y < 32; ++y) luma += luma_byte(px[y * 64]) + luma_byte(px[y * 64 + 1]);
                }
                luma += __shfl_xor_sync(0xffffffffu, luma, 1);
                luma += __shfl_xor_sync(0xffffffffu, luma, 2);
                luma += __shfl_xor_sync(0xffffffffu, luma, 4);
                luma += __shfl_xor_sync(0xffffffffu, luma, 8);
                value = __fdiv_rn(luma, 1024.0f * 255.0f);
            }
            if (lane == 0 || lane == 16) f[126 + half * 2 + (lane >> 4)] = value;
        }
        f[lane] = scalar_feature(lane, o, m);
        if (lane + 32 < 62) f[lane + 32] = scalar_feature(lane + 32, o, m);
    }
}

/* ------------------------------------------------------------------ */
/* Per-device launch parameters, filled on first use of each device. */

constexpr int kMaxDevices = 64;
struct DeviceInfo {
    std::atomic<int> ready{0};
    int sms = 0;
    int blocks_per_sm[2] = {0, 0}; /* staged kernel, u8 / f32 cameras */
};
DeviceInfo g_devices[kMaxDevices];

template <bool kF32Cam>
cudaError_t staged_occupancy(int *blocks) {
    cudaError_t st = cudaFuncSetAttribute(features_staged_kernel<kF32Cam>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(Ring<kF32Cam>::smem_bytes));
    if (st != cudaSuccess) return st;
    st = cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks, features_staged_kernel<kF32Cam>, kThreads,
                                                       Ring<kF32Cam>::smem_bytes);
    if (*blocks < 1) *blocks = 1;
    return st;
}

cudaError_t device_info(int dev, const DeviceInfo **out) {
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    DeviceInfo &d = g_devices[dev];
    if (!d.ready.load(std::memory_order_acquire)) {
        int sms = 0, b8 = 0, b32 = 0;
        cudaError_t st = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (st == cudaSuccess) st = staged_occupancy<false>(&b8);
        if (st == cudaSuccess) st = staged_occupancy<true>(&b32);
        if (st != cudaSuccess) return st;
        d.sms = sms;
        d.blocks_per_sm[0] = b8;
        d.blocks_per_sm[1] = b32;
        d.ready.store(1, std::memory_order_release);
    }
    *out = &d;
    return cudaSuccess;
}

bool aligned(const void *p, uintptr_t n) {
    return (reinterpret_cast<uintptr_t>(p) & (n - 1)) == 0;
}

} /* namespace */

/* ------------------------------------------------------------------ */
/* Internal launch used by the public shim and by the tests' hooks. */

template <bool kF32Cam>
static int launch_features(const float *obs, const float *mission, const void *cameras, float *features,
                           size_t batch, void *stream, const tb_features_launch_opts *opts,
                           int *launch_error) {
    if (launch_error) *launch_error = static_cast<int>(cudaErrorInvalidValue);
    if (!obs || !mission || !features || batch == 0 || batch > 0x7fffffffu) return 0;
    if (!aligned(obs, 4) || !aligned(mission, 4) || !aligned(features, 4)) return 0;
    if (kF32Cam && cameras && !aligned(cameras, 4)) return 0;
    int dev = 0;
    cudaError_t st = cudaGetDevice(&dev);
    const DeviceInfo *info = nullptr;
    if (st == cudaSuccess) st = device_info(dev, &info);
    if (st != cudaSuccess) {
        if (launch_error) *launch_error = static_cast<int>(st);
        return 0;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    /* Discard an earlier, unrelated error of this thread so that the check
     * after the launch reports this launch only (a sticky device error
     * persists and still fails it). */
    cudaGetLastError();
    const int force_direct = opts && opts->force_direct;
    const bool aligned_rows = !force_direct && aligned(obs, 16) && (!cameras || aligned(cameras, 16));
    const int flat_choice = opts ? opts->flat : 0;
    /* the test hooks (grid cap, withheld copies) act on the staged kernel */
    const bool limited_grid = opts && (opts->grid_limit > 0 || opts->stall_sample >= 0);
    /* u8 cameras take the flat kernel at every batch size (measured on B200,
     * amortised device time per launch, flat / staged: 8.45 / 10.4 us at
     * 1,024 aircraft, 24.0 / 28.8 us at 4,096, 306.7 / 312.6 us at 65,536);
     * the staged kernel serves FP32 cameras and the test hooks */
    const bool flat = !kF32Cam && aligned_rows && !limited_grid && flat_choice >= 0;
    if (flat) {
        unsigned int *status = tb_status_slot(stream);
        if (!status) {
            if (launch_error) *launch_error = static_cast<int>(cudaErrorInvalidDevice);
            return 0;
        }
        features_flat_kernel<<<static_cast<unsigned int>(batch), kConsumerWarps * 32, 0, s>>>(
            obs, mission, static_cast<const unsigned char *>(cameras), features, batch, status);
    } else if (aligned_rows) {
        unsigned int *status = tb_status_slot(stream);
        if (!status) {
            if (launch_error) *launch_error = static_cast<int>(cudaErrorInvalidDevice);
            return 0;
        }
        StagedArgs args;
        args.status = status;
        args.obs = obs;
        args.mission = mission;
        args.cameras = cameras;
        args.features = features;
        args.batch = batch;
        args.wait_ns = (opts && opts->wait_ns) ? opts->wait_ns : kDefaultWaitNs;
        args.stall_sample = opts ? opts->stall_sample : -1;
        /* runs of Ring::chunk aircraft over a covering grid, or (FP32 cameras,
         * and the ring-wraparound test hook `grid_limit`) a persistent grid */
        const bool limited = opts && opts->grid_limit > 0;
        const unsigned long long resident = static_cast<unsigned long long>(info->sms) *
                                            static_cast<unsigned long long>(info->blocks_per_sm[kF32Cam ? 1 : 0]);
        unsigned long long grid = resident;
        args.chunk = 0;
        if (!limited && Ring<kF32Cam>::max_chunk) {
            /* runs of up to max_chunk aircraft, but no fewer CTAs than fit at once */
            const unsigned long long fill = (batch + resident - 1) / resident;
            args.chunk = fill < Ring<kF32Cam>::max_chunk ? fill : Ring<kF32Cam>::max_chunk;
            grid = (batch + args.chunk - 1) / args.chunk;
        }
        if (limited && grid > static_cast<unsigned long long>(opts->grid_limit))
            grid = static_cast<unsigned long long>(opts->grid_limit);
        if (grid > batch) grid = batch;
        features_staged_kernel<kF32Cam>
            <<<static_cast<unsigned int>(grid), kThreads, Ring<kF32Cam>::smem_bytes, s>>>(args);
    } else {
        unsigned long long grid = (batch + 7) / 8; /* 8 warps of 32, one aircraft per warp */
        const unsigned long long cap = static_cast<unsigned long long>(info->sms) * 8;
        if (grid > cap) grid = cap;
        unsigned int *status = tb_status_slot(stream);
        if (!status) {
            if (launch_error) *launch_error = static_cast<int>(cudaErrorInvalidDevice);
            return 0;
        }
        features_direct_kernel<kF32Cam>
            <<<static_cast<unsigned int>(grid), 256, 0, s>>>(obs, mission, cameras, features, batch, status);
    }
    st = cudaGetLastError();
    if (launch_error) *launch_error = static_cast<int>(st);
    return st == cudaSuccess;
}

extern "C" int tb_features_launch_checked(const float *obs, const float *mission,
                                          const unsigned char *cameras, float *features,
                                          size_t batch, void *stream,
                                          const tb_features_launch_opts *opts, int *launch_error) {
    return launch_features<false>(obs, mission, cameras, features, batch, stream, opts, launch_error);
}

extern "C" int tb_features_launch_f32cam(const float *obs, const float *mission,
                                         const float *cameras_f32, float *features, size_t batch,
                                         void *stream, const tb_features_launch_opts *opts) {
    return launch_features<true>(obs, mission, cameras_f32, features, batch, stream, opts, nullptr);
}

extern "C" int tb_features_launch(const float *obs, const float *mission,
                                  const unsigned char *cameras, float *features, size_t batch,
                                  void *stream, const tb_features_launch_opts *opts) {
    return tb_features_launch_checked(obs, mission, cameras, features, batch, stream, opts, nullptr);
}

extern "C" int tb_features_staged_config(int *blocks_per_sm, int *sms, int *smem_bytes,
                                         int *threads, int *stages) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    const DeviceInfo *info = nullptr;
    if (device_info(dev, &info) != cudaSuccess) return 0;
    if (blocks_per_sm) *blocks_per_sm = info->blocks_per_sm[0];
    if (sms) *sms = info->sms;
    if (smem_bytes) *smem_bytes = static_cast<int>(Ring<false>::smem_bytes);
    if (threads) *threads = kThreads;
    if (stages) *stages = Ring<false>::stages;
    return 1;
}

/* ---- reference entry points (cuda_features.h:14-20) ---- */

extern "C" int tb_cuda_extract_features_device(const float *device_obs, const float *device_mission,
                                               const unsigned char *device_cameras,
                                               float *device_features, size_t batch_size,
                                               void *stream) {
    return tb_features_launch(device_obs, device_mission, device_cameras, device_features,
                              batch_size, stream, nullptr);
}

/* Waits for `stream`, then reads and clears the status word that the
 * kernels launched on that stream write: 0 if a pipeline wait of any of them
 * expired (reported once), or on a CUDA error. */
extern "C" int tb_cuda_synchronize(void *stream) {
    if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess) return 0;
    unsigned int status = 0;
    if (!tb_status_take(stream, &status)) return 0;
    return status == 0;
}

/* ---- additive entry point: FP32 cameras ---- */

extern "C" int tb_cuda_extract_features_device_f32cam(const float *device_obs,
                                                      const float *device_mission,
                                                      const float *device_cameras_f32,
                                                      float *device_features, size_t batch_size,
                                                      void *stream) {
    return tb_features_launch_f32cam(device_obs, device_mission, device_cameras_f32, device_features,
                                     batch_size, stream, nullptr);
}
