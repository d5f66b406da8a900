/*
 * sm_100a kernel for the onboard tactical (24) + physics-prior (15) values
 * per aircraft -- the reference's device-only header
 * src/network/onboard_features.cuh:1-521 (tb_onboard_tactical,
 * tb_onboard_prior), used by its 618M learner's scalar_inputs kernel
 * (src/network/network_gpu.cu:274-303) and tested by
 * tests/test_onboard_features.cu.  Exposed through the additive entry point
 * tb_cuda_extract_onboard_device.
 *
 * Work split (B200):
 *  - The two LiDAR passes over the 1,536 controller rays (2 heads x 6
 *    elevations x 128 azimuths) dominate.  A warp takes one aircraft at a
 *    time and 32 consecutive rays per step (one coalesced 128-byte load).
 *    Pass 1 keeps per-lane "first strictly smaller" minima (nearest range
 *    with its world offset, nearest corridor centre), merged by one warp
 *    (value, ray index) arg-min at the end, and caches each ray's corridor
 *    centre in shared memory; pass 2 reads that cache, counts members with
 *    a ballot + popcount and sums their y with an in-order shuffle walk over
 *    the ballot, so the float sum keeps the reference's ray order and
 *    rounding.
 *  - Only aircraft whose mission reads the scans (dodge, slalom) are
 *    scanned; a CTA lists them per chunk of 512 aircraft and its warps
 *    claim them from a shared counter (onboard_scan_kernel, one CTA per SM for its
 *    shared-memory staging).  The scalar control law runs in a second launch,
 *    one aircraft per thread without shared memory (onboard_control_kernel),
 *    so a 65,536-aircraft batch is one wave; a scanned aircraft's results
 *    reach it parked in its own prior row.
 *  - Ray directions (12 elevation and 128 azimuth cosines/sines, correctly
 *    rounded constants in tb_scan_tables.h) are copied once per CTA into
 *    shared memory.
 *
 * Arithmetic: this file is compiled with -fmad=false, so every float
 * multiply and add rounds separately in the reference's expression order, as
 * in the host build of the reference.  Float transcendentals are evaluated
 * in double and rounded once (correctly rounded but for vanishingly rare
 * cases).  The reference's float libm calls are not correctly rounded for a
 * sizeable share of inputs, so results equal the reference header built with
 * correctly rounded transcendentals bit for bit, and differ from the
 * glibc-built reference only by what that library's rounding does.
 */
#include <cuda_runtime.h>

#include <stddef.h>
#include <stdint.h>

#include "tb_features_internal.h"
#include "tb_onboard_scan.cuh"
#include "tb_pipeline.cuh"
#include "turbinator/training/cuda_features.h"

namespace {

constexpr int kObsDim = 4148;
constexpr int kMissionDim = 10;
constexpr int kRays = 1536;     /* 2 heads x 6 elevations x 128 azimuths */
constexpr int kWarps = 18;      /* scan warps per CTA (one CTA per SM) */
constexpr int kChunk = 512;    /* aircraft per CTA step */
constexpr int kThreads = 32 * kWarps;
constexpr unsigned kFull = 0xffffffffu;
constexpr unsigned long long kWaitNs = 1000000000ull; /* ~1 s limit on each staging wait */
constexpr uint32_t kHeadBlockBytes = 6 * 128 * 4;      /* elevation rows 0..5 of one head */

/* ---- correctly rounded float transcendentals (double, one rounding) ----
 * One out-of-line copy of each double-precision function, shared by every
 * call site: the control law calls them about 80 times, and inlined copies
 * made its code too large for the instruction caches. */
__device__ __noinline__ double d_sin(double x) { return sin(x); }
__device__ __noinline__ double d_cos(double x) { return cos(x); }
__device__ __noinline__ double d_tan(double x) { return tan(x); }
__device__ __noinline__ double d_asin(double x) { return asin(x); }
__device__ __noinline__ double d_acos(double x) { return acos(x); }
__device__ __noinline__ double d_atanh(double x) { return atanh(x); }
__device__ __noinline__ double d_tanh(double x) { return tanh(x); }
__device__ __noinline__ double d_exp(double x) { return exp(x); }
__device__ __noinline__ double d_atan2(double y, double x) { return atan2(y, x); }
__device__ __noinline__ double d_hypot(double x, double y) { return hypot(x, y); }
__device__ __noinline__ void d_sincos(double x, double *s, double *c) { sincos(x, s, c); }
__device__ __forceinline__ float cr_sin(float x) { return static_cast<float>(d_sin(static_cast<double>(x))); }
__device__ __forceinline__ float cr_cos(float x) { return static_cast<float>(d_cos(static_cast<double>(x))); }
__device__ __forceinline__ float cr_tan(float x) { return static_cast<float>(d_tan(static_cast<double>(x))); }
__device__ __forceinline__ float cr_asin(float x) { return static_cast<float>(d_asin(static_cast<double>(x))); }
__device__ __forceinline__ float cr_acos(float x) { return static_cast<float>(d_acos(static_cast<double>(x))); }
__device__ __forceinline__ float cr_atanh(float x) { return static_cast<float>(d_atanh(static_cast<double>(x))); }
__device__ __forceinline__ float cr_tanh(float x) { return static_cast<float>(d_tanh(static_cast<double>(x))); }
__device__ __forceinline__ float cr_exp(float x) { return static_cast<float>(d_exp(static_cast<double>(x))); }
__device__ __forceinline__ float cr_atan2(float y, float x) {
    return static_cast<float>(d_atan2(static_cast<double>(y), static_cast<double>(x)));
}
/* sin and cos of one argument from one call (one range reduction). */
__device__ __forceinline__ void cr_sincos(float x, float &s, float &c) {
    double ds, dc;
    d_sincos(static_cast<double>(x), &ds, &dc);
    s = static_cast<float>(ds);
    c = static_cast<float>(dc);
}
__device__ __forceinline__ float cr_hypot(float x, float y) {
    return static_cast<float>(d_hypot(static_cast<double>(x), static_cast<double>(y)));
}

/* ---- the reference's small helpers (onboard_features.cuh:6-22) ---- */

/* NaN passes through; otherwise clamp with fmaxf then fminf. */
__device__ __forceinline__ float nclamp(float x, float lo, float hi) {
    if (isnan(x)) return x;
    return fminf(hi, fmaxf(lo, x));
}
/* Observation sanitiser: NaN -> 0, +-inf -> +-1000. */
__device__ __forceinline__ float obs_value(float x) {
    return isnan(x) ? 0.0f : (isinf(x) ? copysignf(1000.0f, x) : x);
}
/* Mission sanitiser: NaN -> 0, +-inf -> +-1. */
__device__ __forceinline__ float mission_value(float x) {
    return isnan(x) ? 0.0f : (isinf(x) ? copysignf(1.0f, x) : x);
}
/* Angle difference wrapped through atan2(sin, cos). */
__device__ __forceinline__ float wrap(float target, float current) {
    const float d = target - current;
    float s, c;
    cr_sincos(d, s, c);
    return cr_atan2(s, c);
}
__device__ __forceinline__ float norm3(float x, float y, float z) { return sqrtf(x * x + y * y + z * z); }
/* Final tactical sanitiser: NaN -> 0, +-inf -> +-1. */
__device__ __forceinline__ float unit_sane(float x) {
    return isnan(x) ? 0.0f : (isinf(x) ? copysignf(1.0f, x) : x);
}

/* The scan summary, its parked form, the attitude rotation and the ray
 * direction tables are shared with the learner-input kernel
 * (tb_onboard_scan.cuh). */
using tb_scan::Attitude;
using tb_scan::RayStats;
using tb_scan::RayTables;
using tb_scan::attitude_from;
using tb_scan::park_stats;
using tb_scan::unpark_stats;

/* Per-warp shared memory: one staged LiDAR block (the 1,536 controller rays
 * of one aircraft, in ray order) and pass 1's corridor-centre x per ray (+inf
 * outside the corridor), which pass 2 reads back.  A single block per warp
 * (12 KB a warp) lets 18 warps share an SM; a warp then waits for its own
 * next copy, and the others cover the wait.  Two blocks per warp (a prefetch
 * ring, 18 KB a warp) fitted 11 warps: 0.137 / 0.362 ms against 0.115 /
 * 0.270 ms now per 65,536-aircraft call (mission mix / all scanning). */
struct alignas(16) WarpSlot {
    float ranges[kRays];
    float corridor_x[kRays];
    unsigned long long bar;
};
/* Bulk copies land at ranges and ranges + kRays / 2 of every warp's slot, and
 * need 16-byte aligned shared addresses: the slots are packed back to back
 * from a 128-byte aligned base, so the slot size must be a multiple of 16
 * (12,296 bytes unpadded would leave odd warps' slots 8-byte aligned). */
static_assert(sizeof(WarpSlot) % 16 == 0 && offsetof(WarpSlot, ranges) == 0 && (kRays / 2 * 4) % 16 == 0,
              "bulk-copy destinations must be 16-byte aligned");

using namespace tb_pipe; /* mbarriers, bounded waits, bulk copies: tb_pipeline.cuh */

/* Stage aircraft `row`'s two LiDAR blocks (heads 0 and 1, elevations 0..5)
 * into slot.ranges.  16-byte aligned rows take two 1-D bulk copies completing
 * on slot.bar (issued by lane 0); other rows are copied by the warp with
 * plain loads, and slot.bar is then just arrived on.  The warp has finished
 * reading the previous block (scan_rays ends in __syncwarp). */
__device__ __forceinline__ void stage_rays(WarpSlot &slot, const float *obs_row, bool bulk, int lane) {
    const uint32_t bar = smem_addr(&slot.bar);
    float *dst = slot.ranges;
    if (bulk) {
        if (lane == 0) {
            fence_proxy_async_shared();
            mbar_arrive_expect_tx(bar, 2u * kHeadBlockBytes);
            bulk_load(smem_addr(dst), obs_row + 48, kHeadBlockBytes, bar);
            bulk_load(smem_addr(dst + kRays / 2), obs_row + 48 + 2048, kHeadBlockBytes, bar);
        }
    } else {
        for (int i = lane; i < kRays; i += 32) dst[i] = __ldg(obs_row + 48 + (i >= kRays / 2 ? 2048 - kRays / 2 : 0) + i);
        __syncwarp();
        if (lane == 0) mbar_arrive(bar);
    }
}

/* Warp arg-min of (value, index): smallest value, then smallest index. */
__device__ __forceinline__ void warp_argmin(float &v, int &idx) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(kFull, v, off);
        const int oi = __shfl_xor_sync(kFull, idx, off);
        if (ov < v || (ov == v && oi < idx)) { v = ov; idx = oi; }
    }
}

/* Both controller LiDAR passes for one staged aircraft, by the whole warp.
 * Ray r (0..1535) is (head, el, azi) in the reference's loop order; lane l
 * owns rays with azi % 32 == l and visits them in increasing r, so its
 * running "strictly smaller" minima keep the first occurrence, and the warp
 * arg-min by (value, ray) reproduces the sequential result.  A range outside
 * (0.35, 11.5) never enters either pass, and the observation sanitiser maps
 * NaN and +-inf outside that window, so raw ranges are used directly.
 *
 * The control law reads the nearest return (min_r and its offsets) only for
 * dodge missions, and the corridor results (min_dx_c, cluster count, cluster
 * y) only for slalom missions -- and of the cluster y sum only its sign
 * (onboard_features.cuh:234-239).  `want_near` / `want_corridor`
 * (warp-uniform) select what is computed; the fields not asked for keep the
 * reference's initial values.  The sign of the reference's in-order float
 * sum is decided from a double-precision sum and a bound on the float sum's
 * rounding error ((n-1) * 2^-24 * sum|y| for n terms, doubled for margin);
 * only when that bound cannot settle the sign is the exact in-order float
 * sum formed (an in-order shuffle walk over each chunk's ballot).  Every lane
 * returns the same RayStats. */
__device__ RayStats scan_rays(const RayTables &t, WarpSlot &slot, const float *ranges,
                              const Attitude &a, float py, const float (&cos_az)[4],
                              const float (&sin_az)[4], int lane, bool want_near, bool want_corridor) {
    const float inf = __int_as_float(0x7f800000);
    float near_r = inf, near_wx = 0.0f, near_wy = 0.0f;
    int near_ray = 0x7fffffff;
    float ahead_x = inf;
    int ahead_ray = 0x7fffffff;

    /* Pass 1 (onboard_features.cuh:188-207). */
#pragma unroll 2
    for (int row = 0; row < 12; ++row) {          /* head * 6 + el */
        const int el = row >= 6 ? row - 6 : row;
        const float ce = t.cos_el[row], se = t.sin_el[row];
        const bool near_row = want_near && el < 4;
        if (!near_row && !want_corridor) continue;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int ray = row * 128 + q * 32 + lane;
            const float range = ranges[ray];
            const bool valid = range > 0.35f && range < 11.5f;
            const float rx = ce * cos_az[q], ry = ce * sin_az[q];
            const float rz = se;
            const float rwx = a.r00 * rx + a.r01 * ry + a.r02 * rz;
            const float rwy = a.r10 * rx + a.r11 * ry + a.r12 * rz;
            const float wx = rwx * range, wy = rwy * range;
            if (near_row && valid && range < near_r) {
                near_r = range;
                near_ray = ray;
                near_wx = wx;
                near_wy = wy;
            }
            if (want_corridor) {
                const float rwz = a.r20 * rx + a.r21 * ry + a.r22 * rz;
                const float wz = rwz * range;
                const float x_center = wx + rwx * 1.10f;
                const float y_center = py + wy + rwy * 1.10f;
                const bool corridor = valid && fabsf(wz) <= 2.1f && x_center >= -0.35f &&
                                      x_center <= 10.5f && fabsf(y_center) <= 3.5f;
                if (corridor && x_center < ahead_x) {
                    ahead_x = x_center;
                    ahead_ray = ray;
                }
                slot.corridor_x[ray] = corridor ? x_center : inf;
            }
        }
    }

    RayStats s = tb_scan::initial_stats();
    if (want_near) {
        const float lane_wx = near_wx, lane_wy = near_wy;
        warp_argmin(near_r, near_ray);
        if (near_r < 30.0f) {
            s.min_r = near_r;
            s.min_r_dx = __shfl_sync(kFull, lane_wx, near_ray & 31);
            s.min_r_dy = __shfl_sync(kFull, lane_wy, near_ray & 31);
        }
    }
    if (!want_corridor) return s;
    warp_argmin(ahead_x, ahead_ray);
    s.min_dx_c = ahead_x < 30.0f ? ahead_x : 30.0f;
    __syncwarp();

    /* Pass 2 (onboard_features.cuh:213-233): corridor centres within 1.4 m
     * of the nearest.  y is recomputed for member rays only. */
    const float limit = s.min_dx_c + 1.4f;
    int count = 0;
    double dsum = 0.0, dabs = 0.0;
#pragma unroll 4
    for (int base = 0; base < kRays; base += 32) {
        const int ray = base + lane;
        const bool member = slot.corridor_x[ray] <= limit;
        count += __popc(__ballot_sync(kFull, member));
        if (member) {
            const int row = ray >> 7, azi = ray & 127;
            const float ce = t.cos_el[row];
            const float rx = ce * t.cos_az[azi], ry = ce * t.sin_az[azi], rz = t.sin_el[row];
            const float rwy = a.r10 * rx + a.r11 * ry + a.r12 * rz;
            const float y = py + rwy * ranges[ray] + rwy * 1.10f;
            dsum += static_cast<double>(y);
            dabs += fabs(static_cast<double>(y));
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        dsum += __shfl_xor_sync(kFull, dsum, off);
        dabs += __shfl_xor_sync(kFull, dabs, off);
    }
    s.cluster_count = count;
    const double bound = 2.0 * static_cast<double>(count) * 0x1.0p-24 * dabs;
    /* The bound assumes no in-order float partial sum overflows: every partial
     * sum is at most sum|y| (1 + n 2^-24) in magnitude, below FLT_MAX when
     * sum|y| < 2^127 (n <= 1,536).  Larger or non-finite sums take the exact
     * path. */
    if (dabs < 0x1.0p127 && fabs(dsum) > bound) {
        /* Sign settled: the in-order float sum has the sign of dsum. */
        s.cluster_y_sum = dsum > 0.0 ? 1.0f : -1.0f;
    } else {
        /* Ambiguous sign: form the reference's in-order float sum exactly. */
        float ysum = 0.0f;
        for (int base = 0; base < kRays; base += 32) {
            const int ray = base + lane;
            unsigned mask = __ballot_sync(kFull, slot.corridor_x[ray] <= limit);
            if (mask) {
                const int row = ray >> 7, azi = ray & 127;
                const float ce = t.cos_el[row];
                const float rx = ce * t.cos_az[azi], ry = ce * t.sin_az[azi], rz = t.sin_el[row];
                const float rwy = a.r10 * rx + a.r11 * ry + a.r12 * rz;
                const float y = py + rwy * ranges[ray] + rwy * 1.10f;
                do {
                    ysum += __shfl_sync(kFull, y, __ffs(mask) - 1);
                    mask &= mask - 1;
                } while (mask);
            }
        }
        s.cluster_y_sum = ysum;
    }
    __syncwarp();
    return s;
}

/* ---- tactical values (onboard_features.cuh:25-86), raw inputs ---- */
__device__ void tactical(const float *o, const float *m, float *out) {
    const float pi = 3.14159265358979323846f;
    float t[24];
    float spool[4], fz[4], tau_z = 0.0f, spool_mean = 0.0f;
    for (int i = 0; i < 4; ++i) {
        spool[i] = nclamp(o[16 + i], 0.0f, 1.0f);
        const float thrust = 0.036f + 0.964f * spool[i];
        const float ci = cr_cos(o[28 + i]);
        fz[i] = thrust * o[24 + i] * ci;
        tau_z += thrust * o[20 + i] * ci;
        spool_mean += spool[i];
    }
    spool_mean *= 0.25f;
    t[0] = fz[1] - fz[3];
    t[1] = fz[2] - fz[0];
    t[2] = 0.5f * tau_z;
    t[3] = 0.25f * (fz[0] + fz[1] + fz[2] + fz[3]) - 0.5f;
    for (int i = 0; i < 4; ++i) t[4 + i] = 2.0f * (spool[i] - spool_mean);
    const float qw = o[6], qx = o[7], qy = o[8], qz = o[9];
    const float bz_x = 2.0f * (qx * qz + qw * qy);
    const float bz_y = 2.0f * (qy * qz - qw * qx);
    const float ct = nclamp(1.0f - 2.0f * (qx * qx + qy * qy), -1.0f, 1.0f);
    const float bx_x = 1.0f - 2.0f * (qy * qy + qz * qz);
    const float bx_y = 2.0f * (qx * qy + qw * qz);
    const float yaw = cr_atan2(bx_y, bx_x);
    float sy, cy;
    cr_sincos(yaw, sy, cy);
    t[8] = cy * bz_y - sy * bz_x;
    t[9] = -sy * bz_y - cy * bz_x;
    t[10] = ct;
    t[11] = ct < 0.20f ? 1.0f : 0.0f;
    const float rx = cr_atanh(nclamp(m[7], -0.995f, 0.995f)) * 20.0f;
    const float ry = cr_atanh(nclamp(m[8], -0.995f, 0.995f)) * 20.0f;
    const float rz = cr_atanh(nclamp(m[9], -0.995f, 0.995f)) * 20.0f;
    t[12] = cr_tanh((cy * rx + sy * ry) * 0.08f);
    t[13] = cr_tanh((-sy * rx + cy * ry) * 0.08f);
    t[14] = cr_tanh(rz * 0.12f);
    t[15] = cr_tanh(cr_hypot(rx, ry) * 0.05f);
    t[16] = cr_tanh((cy * o[3] + sy * o[4]) * 0.15f);
    t[17] = cr_tanh((-sy * o[3] + cy * o[4]) * 0.15f);
    t[18] = cr_exp(-fmaxf(o[2] - 0.62f, 0.0f));
    const float dist = fmaxf(norm3(rx, ry, rz), 1.0f);
    const float flight = dist / 20.0f;
    const float wx = rx - o[3] * 0.5f * flight;
    const float wy = ry - o[4] * 0.5f * flight;
    const float wz = rz - o[5] * 0.5f * flight + 0.5f * 9.80665f * flight * flight;
    const float ux = -qx, uy = -qy, uz = -qz;
    const float cx = uy * wz - uz * wy + qw * wx;
    const float cyq = uz * wx - ux * wz + qw * wy;
    const float cz = ux * wy - uy * wx + qw * wz;
    const float bx = wx + 2.0f * (uy * cz - uz * cyq);
    const float by = wy + 2.0f * (uz * cx - ux * cz);
    const float bz = wz + 2.0f * (ux * cyq - uy * cx);
    const float az = nclamp(cr_atan2(by, bx), pi / 12.0f, pi * 5.0f / 12.0f);
    const float el = nclamp(cr_atan2(bz, fmaxf(cr_hypot(bx, by), 0.2f)), -pi / 6.0f, pi / 6.0f);
    const float err = cr_hypot(az - o[44], el - o[45]);
    t[19] = (az - pi * 0.25f) / (pi / 6.0f);
    t[20] = el / (pi / 6.0f);
    t[21] = cr_tanh(err * 2.0f);
    t[22] = (o[46] <= 0.02f && o[47] > 0.01f && err < 0.26f && dist < 34.0f) ? 1.0f : -1.0f;
    t[23] = cr_sin(cr_atan2(ry, rx) - pi * 0.25f - yaw);
    for (int i = 0; i < 24; ++i) out[i] = unit_sane(t[i]);
}

/* ---- physics prior (onboard_features.cuh:88-513), sanitised inputs ---- */
__device__ void prior(const float *o, const float *m, const RayStats &rs, float *n) {
    const float pi = 3.14159265358979323846f;
    const float max_installed = 294.2f * 0.85f;
    const float idle_frac = 0.08f;
    const float min_thrust = max_installed * idle_frac;
    const float gravity = 9.80665f;
    const float outer_limit = 2.0f;
    const float inner_limit = pi / 4.0f;
    const float cannon_az_ctr = pi / 4.0f;
    const float cannon_az_half = pi / 6.0f;
    const float cannon_el_lim = pi / 6.0f;

    const float px = o[0], py = o[1], pz = o[2], vx = o[3], vy = o[4], vz = o[5];
    const Attitude at = attitude_from(o[6], o[7], o[8], o[9]);
    const float qw = at.qw, qx = at.qx, qy = at.qy, qz = at.qz;
    const float ox = o[10], oy = o[11], oz = o[12];
    const float omega_norm = norm3(ox, oy, oz);

    float spool[4], thrust[4], outer[4], fz[4], ft[4];
    float total_fz = 0.0f, jammed_yaw_ft = 0.0f;
    for (int i = 0; i < 4; ++i) {
        spool[i] = nclamp(o[16 + i], 0.0f, 1.0f);
        thrust[i] = max_installed * (idle_frac + (1.0f - idle_frac) * spool[i]);
        outer[i] = cr_atan2(o[20 + i], o[24 + i]);
        const float inner = o[28 + i];
        float so, co;
        cr_sincos(outer[i], so, co);
        const float ci = cr_cos(inner);
        fz[i] = thrust[i] * co * ci;
        ft[i] = thrust[i] * so * ci;
        total_fz += fz[i];
        jammed_yaw_ft += ft[i];
    }

    /* Mission decoding. */
    const bool landing = m[1] > 0.75f;
    const bool cargo = m[2] > 0.75f;
    const bool inversion = m[3] > 0.75f && m[0] < -0.25f;
    const bool turbine_out = m[3] > 0.75f && m[2] < -0.25f;
    const bool lateral = m[4] > 0.75f && m[5] > 0.25f;
    const bool slalom = m[4] > 0.75f && !lateral;
    const bool dodge = m[5] > 0.75f;
    const bool arena = m[6] > 0.75f;

    const float fuel = nclamp(o[40], 0.0f, 1.0f) * 9.0f;
    const float ammo_mass = nclamp(o[47], 0.0f, 4.0f) * 6.0f;
    const bool payload = o[41] > 0.5f;
    const float mass = (arena ? 40.0f : 43.0f) + fuel + ammo_mass + (payload ? 30.0f : 0.0f);
    const float weight = mass * gravity;
    const float r00 = at.r00, r01 = at.r01, r02 = at.r02;
    const float r10 = at.r10, r11 = at.r11, r12 = at.r12;
    const float r20 = at.r20, r21 = at.r21, r22 = at.r22;
    const float body_z_x = 2.0f * (qx * qz + qw * qy);
    const float body_z_y = 2.0f * (qy * qz - qw * qx);
    const float ct = nclamp(r22, -1.0f, 1.0f);
    const float yaw = cr_atan2(r10, r00);
    const float tau_x_actual = fz[1] - fz[3];
    const float tau_y_actual = fz[2] - fz[0];
    const float az_actual = (total_fz * ct - weight) / mass;
    const bool heavy_cargo = cargo && payload;
    const bool landing_like = landing || heavy_cargo;

    /* Target selection. */
    const float relx = cr_atanh(nclamp(m[7], -0.9995f, 0.9995f)) * 20.0f;
    const float rely = cr_atanh(nclamp(m[8], -0.9995f, 0.9995f)) * 20.0f;
    const float relz = cr_atanh(nclamp(m[9], -0.9995f, 0.9995f)) * 20.0f;
    float tx = (arena || lateral) ? px + relx : 0.0f;
    if (cargo) tx = 15.0f;
    if (slalom) tx = 36.0f;
    const float ty = (arena || lateral) ? py + rely : 0.0f;
    float tz = 8.0f;
    if (landing) tz = 0.60f;
    if (inversion) tz = 14.0f;
    if (cargo || arena) tz = pz + relz;
    float ex = tx, ey = ty, ez = tz;
    const float dx_opp = tx - px, dy_opp = ty - py;
    const float dxy = cr_hypot(dx_opp, dy_opp);
    const bool valid_d = dxy > 1.0e-3f;
    const float safe_d = valid_d ? dxy : 1.0f;
    const bool intercept = arena && m[0] > 0.75f && m[5] < -0.25f;
    const float desired_range = intercept ? 8.5f : 12.5f;
    float ax = valid_d ? tx - (dx_opp / safe_d) * desired_range : tx;
    float ay = valid_d ? ty - (dy_opp / safe_d) * desired_range : ty;
    const float scale = fminf(16.0f / fmaxf(cr_hypot(ax, ay), 1.0e-3f), 1.0f);
    ax *= scale;
    ay *= scale;
    const float pull = nclamp((cr_hypot(px, py) - 21.0f) / 10.0f, 0.0f, 1.0f);
    ax *= 1.0f - pull;
    ay *= 1.0f - pull;
    const float az = pz < 8.0f || vz < -1.0f ? 12.2f : nclamp(tz, 8.5f, 12.2f);
    if (arena) { ex = ax; ey = ay; ez = az; }
    const float errx = ex - px, erry = ey - py;
    const float horiz_dist = cr_hypot(errx, erry);

    /* Obstacle avoidance and slalom lane from the LiDAR passes. */
    float avoid_x = 0.0f, avoid_y = 0.0f, slalom_speed = 3.8f, nearest_dx = 30.0f;
    if (dodge && rs.min_r < 7.5f) {
        const float min_az = cr_atan2(rs.min_r_dy, rs.min_r_dx);
        float sa, ca;
        cr_sincos(min_az, sa, ca);
        avoid_x = -sa * 2.2f;
        avoid_y = ca * 2.2f;
    }
    const float min_dx_c = rs.min_dx_c;
    const float cluster_y = rs.cluster_y_sum / fmaxf(static_cast<float>(rs.cluster_count), 1.0f);
    const bool has_slalom_obs = slalom && horiz_dist > 2.5f && min_dx_c < 10.2f && rs.cluster_count > 0;
    if (has_slalom_obs) {
        nearest_dx = min_dx_c;
        ey = cluster_y >= 0.0f ? -1.85f : 1.85f;
    }
    const float lane_err = fabsf(py - ey);
    float speed_limit = lane_err > 0.55f ? 2.75f : 4.10f;
    if (lane_err > 1.05f) speed_limit = 1.55f;
    if (min_dx_c >= 6.6f && px > 4.0f) speed_limit = 3.10f;
    if (has_slalom_obs) slalom_speed = speed_limit;
    if (slalom && horiz_dist > 3.5f) {
        const float hill = nclamp((px - 6.0f) / 30.0f, 0.0f, 1.0f);
        ez = 2.5f * cr_sin(pi * hill) + 8.0f;
    }

    const float upx = ex - px, upy = ey - py, upz = ez - pz;
    const float up_horiz = cr_hypot(upx, upy);
    const bool active_slalom = slalom && nearest_dx < 10.2f && horiz_dist > 3.0f;

    /* Landing / cargo velocity and acceleration target. */
    const float pad_z = fmaxf(ez, 0.60f), above_pad = pz - pad_z;
    const float horiz_speed = cr_hypot(vx, vy);
    const float transit_cap = heavy_cargo ? 2.65f : 3.4f;
    const float low_cap = above_pad < 1.2f ? 0.55f : (heavy_cargo ? 1.25f : 1.6f);
    const float max_vxy_land = up_horiz > 1.8f ? transit_cap : low_cap;
    const float kp_land = heavy_cargo ? 0.75f : 1.05f;
    const float des_vx_land = nclamp(kp_land * upx, -max_vxy_land, max_vxy_land);
    const float des_vy_land = nclamp(kp_land * upy, -max_vxy_land, max_vxy_land);
    const float vz_land_touch = pz > 0.635f ? -0.16f : 0.0f;
    const float vz_land_cargo = nclamp(1.6f * (0.64f - pz), -0.30f, 0.18f);
    const float vz_land_low = cargo ? vz_land_cargo : vz_land_touch;
    const float max_desc = cargo ? -0.82f : -1.4f;
    const float vz_land_mid = nclamp(-0.70f * above_pad, max_desc, -0.25f);
    const float vz_land_align = nclamp(1.2f * (pad_z + 0.90f - pz), -0.30f, 0.60f);
    const float transit_z = heavy_cargo ? fmaxf(1.2f + 0.28f * up_horiz, 2.0f) : 2.0f;
    const float max_desc_trans = heavy_cargo ? -1.05f : -1.6f;
    const float vz_land_trans = nclamp(1.3f * (transit_z - pz), max_desc_trans, 1.4f);
    float des_vz_land = above_pad > 1.05f ? vz_land_mid : vz_land_low;
    if ((up_horiz > 0.85f || horiz_speed > 0.65f) && above_pad < 0.95f) des_vz_land = vz_land_align;
    if (up_horiz > 1.8f) des_vz_land = vz_land_trans;
    const float max_axy_land = heavy_cargo ? 2.2f : 2.6f;
    const float des_ax_land = nclamp(2.4f * (des_vx_land - vx), -max_axy_land, max_axy_land);
    const float des_ay_land = nclamp(2.4f * (des_vy_land - vy), -max_axy_land, max_axy_land);
    const float kp_az_land = heavy_cargo ? 5.0f : 4.5f;
    const float kd_az_land = heavy_cargo ? 1.0f : 0.80f;
    const float min_az_land = heavy_cargo ? -1.8f : -2.8f;
    const float des_az_land =
        nclamp(kp_az_land * (des_vz_land - vz) - kd_az_land * az_actual, min_az_land, 5.5f);

    /* Standard / agile / fault / arena flight target. */
    const float inv_max_v = up_horiz > 9.0f && fabsf(upz) < 2.5f && ct > 0.90f ? 6.2f : 4.2f;
    const float lat_vx = fabsf(upy) > 1.35f ? 1.45f : 3.8f;
    float max_vx = arena ? 3.2f : 3.0f;
    if (inversion) max_vx = inv_max_v;
    float max_vy = max_vx;
    if (lateral) { max_vx = lat_vx; max_vy = 3.4f; }
    if (slalom) max_vx = 3.5f;
    if (active_slalom) { max_vx = slalom_speed; max_vy = 3.2f; }
    const float max_vz = vz < -2.0f || inversion ? 6.5f : 2.6f;
    const float kp_xy = inversion ? 0.85f : (lateral ? 0.95f : 0.90f);
    const float kp_vx = active_slalom ? 1.25f : kp_xy;
    const float kp_vy = active_slalom ? 1.45f : (lateral ? 1.05f : kp_xy);
    const float des_vx = nclamp(kp_vx * upx + avoid_x, -max_vx, max_vx);
    const float des_vy = nclamp(kp_vy * upy + avoid_y, -max_vy, max_vy);
    float des_vz = nclamp(1.25f * upz, -2.6f, max_vz);
    if ((inversion || arena) && vz < -1.0f) des_vz = fmaxf(des_vz, 0.8f);
    const float kp_ax = active_slalom ? 3.0f : 2.4f;
    const float kp_ay = active_slalom ? 3.0f : 2.6f;
    const float des_ax_std = nclamp(kp_ax * (des_vx - vx), -3.8f, 3.8f);
    const float des_ay_std = nclamp(kp_ay * (des_vy - vy), -3.8f, 3.8f);
    const float max_az = vz < -1.8f || inversion ? 14.0f : 6.5f;
    const float des_az_std = nclamp(3.8f * (des_vz - vz) - 0.80f * az_actual, -4.0f, max_az);
    const float des_ax = landing_like ? des_ax_land : des_ax_std;
    const float des_ay = landing_like ? des_ay_land : des_ay_std;
    const float des_az = landing_like ? des_az_land : des_az_std;

    /* Collective, tilt and horizontal force allocation. */
    const float tilt = cr_acos(ct);
    const bool need_headroom = inversion || arena || ct < 0.88f;
    const bool urgent_climb = arena && (pz < 8.5f || vz < -1.2f) && ct > 0.58f;
    const float max_coll = urgent_climb ? 3.95f :
        (need_headroom ? nclamp(3.95f - 0.90f * omega_norm - 1.30f * tilt, 2.55f, 3.95f) : 3.95f);
    const float fz_des = nclamp((weight + mass * des_az) / fmaxf(ct, 0.45f),
                                0.10f * weight, max_coll * max_installed);
    const float horiz_scale = urgent_climb ? 0.0f :
        (need_headroom ? nclamp(1.0f - 1.5f * fmaxf(tilt - 0.15f, 0.0f), 0.0f, 1.0f) : 1.0f);
    const float tilt_comp = turbine_out ? 0.65f : 0.0f;
    const float damp_v = active_slalom ? 0.8f : 0.4f;
    const float fx_world = (mass * des_ax + damp_v * vx - tilt_comp * total_fz * body_z_x) * horiz_scale;
    const float fy_world = (mass * des_ay + damp_v * vy - tilt_comp * total_fz * body_z_y) * horiz_scale;
    float syw, cyw;
    cr_sincos(yaw, syw, cyw);
    const float max_fh = active_slalom ? 105.0f : (lateral ? 125.0f : (heavy_cargo ? 52.0f : 80.0f));
    const float fx_body = nclamp(cyw * fx_world + syw * fy_world, -max_fh, max_fh);
    const float fy_body = nclamp(-syw * fx_world + cyw * fy_world, -max_fh, max_fh);

    /* Tilt error vector in body axes. */
    const float cw_x = body_z_y, cw_y = -body_z_x;
    const float ux = -qx, uy = -qy, uz = -qz;
    const float tt_x = 2.0f * (-uz * cw_y), tt_y = 2.0f * (uz * cw_x);
    const float tt_z = 2.0f * (ux * cw_y - uy * cw_x);
    const float te_x = cw_x + qw * tt_x + (uy * tt_z - uz * tt_y);
    const float te_y = cw_y + qw * tt_y + (uz * tt_x - ux * tt_z);
    const float te_z = qw * tt_z + (ux * tt_y - uy * tt_x);
    const float te_norm = norm3(te_x, te_y, te_z);
    const float tilt_scale = te_norm > 1.0e-5f ? tilt / fmaxf(te_norm, 1.0e-5f) : 0.0f;
    const float e_rx = te_x * tilt_scale, e_ry = te_y * tilt_scale;

    /* Yaw target. */
    const bool inv_hold_yaw = (inversion || arena) && (pz < 6.0f || vz < -0.5f || ct < 0.88f);
    const bool opp_bearing_valid = arena && fabsf(m[1]) + fabsf(m[2]) > 0.1f;
    const float opp_bearing = cr_atan2(m[1], m[2]);
    const float raw_bearing = cr_atan2(ty - py, tx - px);
    const float target_bearing = opp_bearing_valid ? opp_bearing : raw_bearing;
    const float desired_yaw = arena && horiz_dist > 1.0f && !inv_hold_yaw ?
        target_bearing - cannon_az_ctr : (inv_hold_yaw ? yaw : 0.0f);
    const float yaw_err = wrap(desired_yaw, yaw);

    /* Torque commands and per-engine allocation. */
    const float parasite_scale = turbine_out ? 0.35f : 1.0f;
    const float tau_x_par = -0.1625f * fy_body * parasite_scale;
    const float tau_y_par = 0.1625f * fx_body * parasite_scale;
    const float tau_x_net = tau_x_actual + tau_x_par;
    const float tau_y_net = tau_y_actual + tau_y_par;
    const float max_txy = heavy_cargo ? 120.0f : 260.0f;
    const float tau_x_cmd = nclamp(95.0f * e_rx - 64.0f * ox - 0.90f * tau_x_net - tau_x_par,
                                   -max_txy, max_txy);
    const float tau_y_cmd = nclamp(95.0f * e_ry - 64.0f * oy - 0.90f * tau_y_net - tau_y_par,
                                   -max_txy, max_txy);
    const float tau_z_cmd = nclamp(22.0f * yaw_err - 18.0f * oz, -70.0f, 70.0f);
    const float fz_cmd[4] = {
        0.25f * fz_des - tau_y_cmd * 0.5f,
        0.25f * fz_des + tau_x_cmd * 0.5f,
        0.25f * fz_des + tau_y_cmd * 0.5f,
        0.25f * fz_des - tau_x_cmd * 0.5f,
    };
    const float yaw_ft = (tau_z_cmd - 0.40f * jammed_yaw_ft) * 0.25f;
    float outer_cmd[4], inner_cmd[4], throttle[4], u_raw[4];
    const float fx_outer = ft[3] - ft[1];
    const float fy_outer = ft[0] - ft[2];
    const float fx_rem = fx_body - fx_outer, fy_rem = fy_body - fy_outer;
    const float max_sin_inner = lateral ? 0.44f : (active_slalom ? 0.42f : (heavy_cargo ? 0.22f : 0.32f));
    const float spool_gain = turbine_out ? 10.5f : (heavy_cargo ? 4.5f : 2.4f);
    float max_raw = -__int_as_float(0x7f800000);
    const bool land_idle = landing && pz <= 0.638f && up_horiz < 0.85f && fabsf(vz) < 0.20f;
    for (int i = 0; i < 4; ++i) {
        const float yaw_alpha = cr_asin(nclamp(yaw_ft / fmaxf(thrust[i], 30.0f), -0.35f, 0.35f));
        outer_cmd[i] = nclamp(6.5f * wrap(yaw_alpha, outer[i]), -outer_limit, outer_limit);
        const float urx = i == 0 ? 1.0f : (i == 2 ? -1.0f : 0.0f);
        const float ury = i == 1 ? 1.0f : (i == 3 ? -1.0f : 0.0f);
        const float fr_req = 0.5f * (fx_rem * urx + fy_rem * ury);
        const float sin_in = nclamp(fr_req / fmaxf(thrust[i], 40.0f), -max_sin_inner, max_sin_inner);
        inner_cmd[i] = nclamp(cr_asin(sin_in), -inner_limit * 0.90f, inner_limit * 0.90f);
        const float nominal_cos = fmaxf(cr_cos(yaw_alpha) * cr_cos(inner_cmd[i]), 0.70f);
        float target_thrust = fmaxf(fz_cmd[i], 0.0f) / nominal_cos;
        if (land_idle) target_thrust = 0.15f * weight * 0.25f;
        const float u_des = nclamp((target_thrust - min_thrust) / (max_installed - min_thrust), 0.0f, 1.0f);
        u_raw[i] = u_des + spool_gain * (u_des - spool[i]);
        max_raw = fmaxf(max_raw, u_raw[i]);
    }
    const float excess = nclamp(max_raw - 1.0f, 0.0f, urgent_climb ? 0.10f : 0.45f);
    for (int i = 0; i < 4; ++i)
        throttle[i] = nclamp(u_raw[i] - (need_headroom ? excess : 0.0f), 0.0f, 1.0f);
    const bool inv_mode = ct < 0.20f;
    if (inv_mode) {
        const float inv_rx = te_norm > 1.0e-5f ? e_rx : tilt;
        const float tx_inv = 130.0f * inv_rx - 52.0f * ox;
        const float ty_inv = 130.0f * e_ry - 52.0f * oy;
        const float arm_mom[4] = {-ty_inv, tx_inv, ty_inv, -tx_inv};
        for (int i = 0; i < 4; ++i) {
            throttle[i] = arm_mom[i] > 12.0f ? 0.58f : 0.0f;
            outer_cmd[i] = nclamp(-outer[i] * 6.0f, -outer_limit, outer_limit);
            inner_cmd[i] = 0.0f;
        }
    }

    /* Cannon aim and fire decision. */
    const float to_x = tx - px, to_y = ty - py, to_z = tz - pz;
    const float dist = fmaxf(norm3(to_x, to_y, to_z), 1.0f);
    const float flight = dist / 20.0f;
    const float aim_x = to_x - vx * (0.65f * flight);
    const float aim_y = to_y - vy * (0.65f * flight);
    const float aim_z = to_z - vz * (0.65f * flight) + 0.53f * gravity * flight * flight;
    const float cx = uy * aim_z - uz * aim_y + qw * aim_x;
    const float cyq = uz * aim_x - ux * aim_z + qw * aim_y;
    const float cz = ux * aim_y - uy * aim_x + qw * aim_z;
    const float aim_bx = aim_x + 2.0f * (uy * cz - uz * cyq);
    const float aim_by = aim_y + 2.0f * (uz * cx - ux * cz);
    const float aim_bz = aim_z + 2.0f * (ux * cyq - uy * cx);
    const float des_cannon_az = nclamp(cr_atan2(aim_by, aim_bx), cannon_az_ctr - cannon_az_half,
                                       cannon_az_ctr + cannon_az_half);
    const float des_cannon_el = nclamp(cr_atan2(aim_bz, fmaxf(cr_hypot(aim_bx, aim_by), 0.2f)),
                                       -cannon_el_lim, cannon_el_lim);
    const float aim_err = cr_hypot(wrap(des_cannon_az, o[44]), des_cannon_el - o[45]);
    const bool fire = arena && !inv_mode && o[46] <= 0.02f && o[47] > 0.01f && aim_err < 0.28f &&
                      dist < 34.0f;
    const bool cannon = arena && !inv_mode;
    float norm_az = cannon ? nclamp((des_cannon_az - cannon_az_ctr) / cannon_az_half, -1.0f, 1.0f) : 0.0f;
    if (inv_mode) norm_az = -1.0f;
    float norm_el = cannon ? nclamp(des_cannon_el / cannon_el_lim, -1.0f, 1.0f) : 0.0f;
    float norm_fire = fire ? 0.8f : -0.8f;

    /* Blended-wing-body modes replace the multirotor allocation. */
    const bool bwb_arena = m[6] > 0.75f && m[4] < -0.25f;
    const bool bwb_cruise = m[4] > 0.75f && m[2] > 0.25f;
    const bool bwb_intercept = m[6] > 0.75f && m[5] > 0.60f;
    const bool bwb_endurance = bwb_cruise && m[0] > 0.25f;
    if (bwb_arena || bwb_cruise || bwb_intercept) {
        const float vb_x = r00 * vx + r10 * vy + r20 * vz;
        const float vb_y = r01 * vx + r11 * vy + r21 * vz;
        const float brx = cr_atanh(nclamp(m[7], -0.9999f, 0.9999f)) * 20.0f;
        const float bry = cr_atanh(nclamp(m[8], -0.9999f, 0.9999f)) * 20.0f;
        const float brz = cr_atanh(nclamp(m[9], -0.9999f, 0.9999f)) * 20.0f;
        float btx = px + brx, bty = py + bry, btz = pz + brz;
        const float rxy = cr_hypot(px, py);
        const float pull_b = nclamp((rxy - 235.0f) / 45.0f, 0.0f, 0.85f);
        if (arena && rxy > 235.0f) { btx *= 1.0f - pull_b; bty *= 1.0f - pull_b; }
        if (arena) btz = nclamp(btz, 28.0f, 135.0f);
        const float gx = btx - px, gy = bty - py, gz = btz - pz;
        const float gdist = fmaxf(norm3(gx, gy, gz), 1.0f);
        const float desired_yaw_b = cr_atan2(gy, gx);
        const float gs = cr_hypot(vx, vy);
        const float course_yaw = gs > 2.5f ? cr_atan2(vy, vx) : yaw;
        const float course_err = wrap(desired_yaw_b, course_yaw);
        const float desired_speed = bwb_endurance ? 18.5f : (arena ? (gdist > 38.0f ? 26.0f : 24.0f) : 22.4f);
        const float speed_err = desired_speed - vb_x;
        const float u_coll = nclamp((bwb_endurance ? 0.36f : 0.44f) + 0.065f * speed_err + 0.018f * gz,
                                    0.12f, 0.90f);
        const float roll_right = cr_atan2(r21, r22);
        const float desired_roll = nclamp(-1.35f * course_err, -0.55f, 0.55f);
        const float diff_u = nclamp(0.90f * (desired_roll - roll_right) - 0.34f * ox, -0.45f, 0.45f);
        const float u0 = nclamp(u_coll + diff_u, 0.05f, 1.0f);
        const float u1 = nclamp(u_coll - diff_u, 0.05f, 1.0f);
        throttle[0] = throttle[2] = u0;
        throttle[1] = throttle[3] = u1;
        const float pitch_up = cr_asin(nclamp(r20, -1.0f, 1.0f));
        const float climb_des = nclamp(0.42f * gz, -5.0f, 5.0f);
        const float climb_err = climb_des - vz;
        float sin_bank, cos_bank;
        cr_sincos(roll_right, sin_bank, cos_bank);
        const float gamma_des = cr_atan2(climb_des, fmaxf(gs, 14.0f));
        float desired_pitch = nclamp(0.062831853f + 0.75f * gamma_des +
            0.035f * climb_err + 0.09f * (1.0f - fmaxf(cos_bank, 0.5f)), -0.15f, 0.25f);
        if (vb_x < 15.5f) desired_pitch = fminf(desired_pitch, 0.02f);
        const float theta_dot = 2.20f * (desired_pitch - pitch_up);
        const float psi_dot = (gravity / fmaxf(vb_x, 12.0f)) * cr_tan(nclamp(-roll_right, -0.75f, 0.75f)) +
            0.35f * course_err;
        const float q_up = cos_bank * theta_dot - sin_bank * psi_dot;
        const float r_left = sin_bank * theta_dot + cos_bank * psi_dot;
        const float gimbal = pi / 6.0f;
        inner_cmd[0] = nclamp(0.85f * (q_up + oy) + 0.03f, -gimbal, gimbal);
        inner_cmd[1] = nclamp(-0.65f * (r_left - oz) - 0.025f * vb_y, -gimbal, gimbal);
        inner_cmd[2] = inner_cmd[3] = 0.0f;
        for (int i = 0; i < 4; ++i) outer_cmd[i] = 0.0f;
        const float oppx = brx - vx * 0.10f, oppy = bry - vy * 0.10f, oppz = brz - vz * 0.10f;
        const float bdist = fmaxf(norm3(oppx, oppy, oppz), 1.0f);
        const bool head_on = bwb_arena && btx * px + bty * py < -800.0f && bdist > 45.0f;
        const float closing = head_on ? 75.0f + 2.0f * fmaxf(vb_x, 0.0f) : 75.0f;
        const float bflight = bdist / closing;
        const float bax = oppx, bay = oppy;
        const float baz = oppz + (head_on ? -vz * (0.85f * bflight) : 0.0f) +
                          0.50f * gravity * bflight * bflight;
        const float bbx = r00 * bax + r10 * bay + r20 * baz;
        const float bby = r01 * bax + r11 * bay + r21 * baz;
        const float bbz = r02 * bax + r12 * bay + r22 * baz;
        const float b_az = nclamp(cr_atan2(bby, fmaxf(bbx, 0.2f)), -pi / 6.0f, pi / 6.0f);
        const float b_el = nclamp(cr_atan2(bbz, fmaxf(cr_hypot(bbx, bby), 0.2f)), -cannon_el_lim,
                                  cannon_el_lim);
        const float b_err = cr_hypot(wrap(b_az, o[44]), b_el - o[45]);
        const bool b_fire = arena && o[46] <= 0.02f && o[47] > 0.01f && b_err < 0.045f &&
                            bdist < 165.0f && bbx > 0.0f;
        norm_az = arena ? nclamp(b_az / (pi / 6.0f), -1.0f, 1.0f) : 0.0f;
        norm_el = arena ? nclamp(b_el / cannon_el_lim, -1.0f, 1.0f) : 0.0f;
        norm_fire = b_fire ? 0.8f : -0.8f;
    }
    for (int i = 0; i < 4; ++i) {
        n[i] = nclamp(throttle[i] * 2.0f - 1.0f, -1.0f, 1.0f);
        n[4 + i] = nclamp(outer_cmd[i] / outer_limit, -1.0f, 1.0f);
        n[8 + i] = nclamp(inner_cmd[i] / inner_limit, -1.0f, 1.0f);
    }
    n[12] = norm_az;
    n[13] = norm_el;
    n[14] = norm_fire;
}

/* ------------------------------------------------------------------ */
/* Two launches.  (1) onboard_scan_kernel, persistent with one CTA per SM:
 * each CTA owns a balanced contiguous range of aircraft and walks it kChunk
 * at a time; the aircraft whose mission reads the LiDAR scans (dodge:
 * nearest return; slalom: corridor) are listed in shared memory and the
 * warps claim those scan jobs from a shared counter, each staging a claimed
 * job's LiDAR block with bulk copies and then scanning it.  A scanned
 * aircraft's RayStats go to the first six floats of its own prior row, which
 * the second launch reads back before overwriting the row.  (2)
 * onboard_control_kernel runs the control law, one aircraft per thread, with
 * no shared memory, so every aircraft of a 65,536 batch is in one wave. */
struct ChunkState {
    unsigned short jobs[kChunk];   /* aircraft index in chunk | 0x4000 near | 0x8000 corridor */
    int job_count, next_job;
};

/* The missions that read the scans (onboard_features.cuh:201-239). */
__device__ __forceinline__ void scan_modes(const float *mrow, bool &dodge, bool &slalom) {
    const float m4 = mission_value(__ldg(mrow + 4));
    const float m5 = mission_value(__ldg(mrow + 5));
    dodge = m5 > 0.75f;
    slalom = m4 > 0.75f && !(m4 > 0.75f && m5 > 0.25f);
}

__global__ void __launch_bounds__(kThreads) onboard_scan_kernel(const float *__restrict__ obs,
                                                                const float *__restrict__ mission,
                                                                float *__restrict__ prior_out,
                                                                unsigned long long batch,
                                                                unsigned long long wait_ns,
                                                                long long stall_sample,
                                                                unsigned int *__restrict__ status) {
    __shared__ RayTables tables;
    extern __shared__ __align__(128) unsigned char dyn[];
    tb_scan::load_tables(tables, threadIdx.x, blockDim.x);
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    WarpSlot &slot = reinterpret_cast<WarpSlot *>(dyn)[warp];
    ChunkState &chunk = *reinterpret_cast<ChunkState *>(dyn + sizeof(WarpSlot) * kWarps);
    if (lane == 0) {
        mbar_init(smem_addr(&slot.bar), 1);
        fence_mbar_init();
    }
    __syncthreads();

    float cos_az[4], sin_az[4];
    for (int q = 0; q < 4; ++q) {
        cos_az[q] = tables.cos_az[q * 32 + lane];
        sin_az[q] = tables.sin_az[q * 32 + lane];
    }
    const bool bulk = (reinterpret_cast<uintptr_t>(obs) & 15) == 0;
    const unsigned long long begin = batch * blockIdx.x / gridDim.x;
    const unsigned long long end = batch * (blockIdx.x + 1) / gridDim.x;
    uint32_t seq = 0;            /* LiDAR blocks staged by this warp so far */
    bool failed = false;

    for (unsigned long long first = begin; first < end; first += kChunk) {
        const int n = static_cast<int>(end - first < kChunk ? end - first : kChunk);
        if (threadIdx.x == 0) {
            chunk.job_count = 0;
            chunk.next_job = 0;
        }
        __syncthreads();
        /* (1) scan jobs of this chunk */
        for (int i = threadIdx.x; i < n; i += kThreads) {
            bool dodge, slalom;
            scan_modes(mission + (first + i) * kMissionDim, dodge, slalom);
            if (dodge || slalom)
                chunk.jobs[atomicAdd(&chunk.job_count, 1)] =
                    static_cast<unsigned short>(i | (dodge ? 0x4000 : 0) | (slalom ? 0x8000 : 0));
        }
        __syncthreads();
        /* (2) scan jobs claimed from a shared counter, so a warp that drew
         * short scans takes more */
        const int jobs = chunk.job_count;
        while (!failed) {
            int cur = 0;
            if (lane == 0) cur = atomicAdd(&chunk.next_job, 1);
            cur = __shfl_sync(kFull, cur, 0);
            if (cur >= jobs) break;
            const int job = chunk.jobs[cur];
            const unsigned long long a = first + (job & 0x3fff);
            if (static_cast<long long>(a) != stall_sample) /* test hook: withhold a copy */
                stage_rays(slot, obs + a * kObsDim, bulk, lane);
            /* all lanes take the same branch, even if the copy lands at the deadline */
            if (!__all_sync(kFull, mbar_wait(smem_addr(&slot.bar), seq & 1, wait_ns))) {
                if (lane == 0) atomicOr(status, TB_FEATURE_STATUS_WAIT_TIMEOUT);
                failed = true;
                break;
            }
            const float *row = obs + a * kObsDim;
            const Attitude at = attitude_from(obs_value(__ldg(row + 6)), obs_value(__ldg(row + 7)),
                                              obs_value(__ldg(row + 8)), obs_value(__ldg(row + 9)));
            const RayStats st = scan_rays(tables, slot, slot.ranges, at, obs_value(__ldg(row + 1)), cos_az,
                                          sin_az, lane, (job & 0x4000) != 0, (job & 0x8000) != 0);
            if (lane == 0) park_stats(prior_out + a * 15, st);
            ++seq;
        }
        __syncthreads(); /* the job list is rewritten by the next chunk */
    }
}

constexpr int kControlThreads = 128;

/* The control law for one aircraft: the scans' parked results (or the
 * reference's initial values), then its 24 tactical and 15 prior values into
 * dst[0..39). */
__device__ __forceinline__ void control_one(const float *__restrict__ obs, const float *__restrict__ mission,
                                            const float *__restrict__ parked, unsigned long long sample,
                                            float *dst) {
    const float *row = obs + sample * kObsDim;
    const float *mrow = mission + sample * kMissionDim;
    bool dodge, slalom;
    scan_modes(mrow, dodge, slalom);
    const RayStats st = dodge || slalom ? unpark_stats(parked + sample * 15) : tb_scan::initial_stats();
    float raw_o[48], raw_m[10], o[48], m[10];
    for (int k = 0; k < 48; ++k) {
        raw_o[k] = __ldg(row + k);
        o[k] = obs_value(raw_o[k]);
    }
    for (int k = 0; k < 10; ++k) {
        raw_m[k] = __ldg(mrow + k);
        m[k] = mission_value(raw_m[k]);
    }
    tactical(raw_o, raw_m, dst);
    prior(o, m, st, dst + 24);
}

constexpr int kOnboardValues = 39; /* 24 tactical + 15 prior; an odd stride: no bank conflicts */

/* One aircraft per thread over a covering grid.  Each thread leaves its 39
 * values in shared memory; the CTA then writes its rows with coalesced
 * stores: the tactical and prior rows (contiguous for the CTA's aircraft)
 * and, with kRows, the onboard columns of the learner's input rows (proprio
 * columns 52..90, mission columns 10..48; network_gpu.cu:296-302), which the
 * learner-input kernel leaves to it when it runs the scans itself.  A
 * scanned aircraft's results are read from its prior row before the CTA's
 * barrier, and its prior row is overwritten only after it. */
template <bool kRows>
__global__ void __launch_bounds__(kControlThreads, 4) onboard_control_kernel(
    const float *__restrict__ obs, const float *__restrict__ mission, float *__restrict__ tactical_out,
    float *__restrict__ prior_out, unsigned long long batch, float *__restrict__ proprio,
    float *__restrict__ mission_vec) {
    __shared__ float vals[kControlThreads * kOnboardValues];
    const unsigned long long first = static_cast<unsigned long long>(blockIdx.x) * kControlThreads;
    const unsigned long long sample = first + threadIdx.x;
    if (sample < batch) control_one(obs, mission, prior_out, sample, vals + threadIdx.x * kOnboardValues);
    __syncthreads();
    const int rows = static_cast<int>(batch - first < kControlThreads ? batch - first : kControlThreads);
    float *tac = tactical_out + first * 24, *pri = prior_out + first * 15;
    for (int e = threadIdx.x; e < rows * 24; e += kControlThreads) tac[e] = vals[(e / 24) * kOnboardValues + e % 24];
    for (int e = threadIdx.x; e < rows * 15; e += kControlThreads)
        pri[e] = vals[(e / 15) * kOnboardValues + 24 + e % 15];
    if (kRows) {
        for (int e = threadIdx.x; e < rows * kOnboardValues; e += kControlThreads) {
            const unsigned long long r = first + static_cast<unsigned long long>(e / kOnboardValues);
            const int k = e % kOnboardValues;
            proprio[r * 91 + 52 + k] = vals[e];
            mission_vec[r * 49 + 10 + k] = vals[e];
        }
    }
}

constexpr int kMaxDevices = 64;
constexpr size_t kDynSmem = sizeof(WarpSlot) * kWarps + sizeof(ChunkState); /* about 217 KiB */
int g_sms[kMaxDevices];

} /* namespace */

static int onboard_setup(int *sms) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 0;
    if (!g_sms[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
        if (cudaFuncSetAttribute(onboard_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kDynSmem)) != cudaSuccess)
            return 0;
        g_sms[dev] = n;
    }
    *sms = g_sms[dev];
    return 1;
}

/* The control-law launch alone (the scans already parked their results in
 * the prior rows), on `stream`, one aircraft per thread.  With
 * device_proprio_91 and device_mission_49 both given, it also writes the
 * onboard columns of those learner rows.  Internal:
 * tb_cuda_prepare_actor_inputs_device runs it after the learner-input
 * kernel, which scans the LiDAR rows it has staged. */
extern "C" int tb_onboard_control_launch(const float *device_obs, const float *device_mission,
                                         float *device_tactical_24, float *device_prior_15, size_t batch_size,
                                         void *stream, float *device_proprio_91, float *device_mission_49) {
    int sms = 0;
    if (!onboard_setup(&sms)) return 0;
    if (!device_proprio_91 != !device_mission_49) return 0;
    cudaGetLastError(); /* report this launch only */
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const unsigned int grid = static_cast<unsigned int>((batch_size + kControlThreads - 1) / kControlThreads);
    if (device_proprio_91)
        onboard_control_kernel<true><<<grid, kControlThreads, 0, s>>>(
            device_obs, device_mission, device_tactical_24, device_prior_15, batch_size, device_proprio_91,
            device_mission_49);
    else
        onboard_control_kernel<false><<<grid, kControlThreads, 0, s>>>(
            device_obs, device_mission, device_tactical_24, device_prior_15, batch_size, nullptr, nullptr);
    return cudaGetLastError() == cudaSuccess;
}

/* Both launches; opts may be NULL (its wait_ns and stall_sample fields are
 * honoured: a test withholds one scanning aircraft's staging copy so the
 * bounded wait expires). */
extern "C" int tb_onboard_launch(const float *device_obs, const float *device_mission, float *device_tactical_24,
                                 float *device_prior_15, size_t batch_size, void *stream,
                                 const tb_features_launch_opts *opts) {
    if (!device_obs || !device_mission || !device_tactical_24 || !device_prior_15 || batch_size == 0 ||
        batch_size > 0x7fffffffu)
        return 0;
    const uintptr_t mis = 3;
    if ((reinterpret_cast<uintptr_t>(device_obs) & mis) || (reinterpret_cast<uintptr_t>(device_mission) & mis) ||
        (reinterpret_cast<uintptr_t>(device_tactical_24) & mis) ||
        (reinterpret_cast<uintptr_t>(device_prior_15) & mis))
        return 0;
    int sms = 0;
    if (!onboard_setup(&sms)) return 0;
    const unsigned long long wait_ns = (opts && opts->wait_ns) ? opts->wait_ns : kWaitNs;
    const long long stall_sample = opts ? opts->stall_sample : -1;
    unsigned int *status = tb_status_slot(stream);
    if (!status) return 0;
    cudaGetLastError(); /* report these launches only */
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    /* scans: one CTA per SM (shared memory admits one) */
    unsigned long long grid = static_cast<unsigned long long>(sms);
    if (grid > batch_size) grid = batch_size;
    onboard_scan_kernel<<<static_cast<unsigned int>(grid), kThreads, kDynSmem, s>>>(
        device_obs, device_mission, device_prior_15, batch_size, wait_ns, stall_sample, status);
    if (cudaGetLastError() != cudaSuccess) return 0;
    /* control law: one thread per aircraft */
    return tb_onboard_control_launch(device_obs, device_mission, device_tactical_24, device_prior_15, batch_size,
                                     stream, nullptr, nullptr);
}

extern "C" int tb_cuda_extract_onboard_device(const float *device_obs, const float *device_mission,
                                              float *device_tactical_24, float *device_prior_15,
                                              size_t batch_size, void *stream) {
    return tb_onboard_launch(device_obs, device_mission, device_tactical_24, device_prior_15, batch_size, stream,
                             nullptr);
}
