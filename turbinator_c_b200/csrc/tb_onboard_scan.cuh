/*
 * The onboard values' two controller LiDAR passes (reference
 * src/network/onboard_features.cuh:185-239), shared by the onboard kernel
 * (onboard_kernel.cu, one warp per aircraft) and the learner-input kernel
 * (actor_inputs_kernel.cu, all eight consumer warps on the aircraft they
 * have staged).
 *
 * The two files are compiled with different contraction settings (the
 * onboard file without FMA contraction, the learner-input file with it), so
 * every float product and sum here is written with an explicitly rounded
 * intrinsic (__fmul_rn, __fadd_rn, __fsub_rn, __fdiv_rn, __fsqrt_rn), which
 * the compiler never fuses: both files round every step separately, in the
 * reference's expression order.
 *
 * Contents: the per-aircraft scan summary (RayStats) and the six floats of
 * it parked in a prior row between two launches; the attitude rotation the
 * scans and the physics prior use; the ray direction tables
 * (tb_scan_tables.h); and block_scan, the two passes by a group of warps.
 */
#ifndef TB_ONBOARD_SCAN_CUH
#define TB_ONBOARD_SCAN_CUH

#include <cuda_runtime.h>

#include "tb_scan_tables.h"

namespace tb_scan {

constexpr int kRays = 1536;         /* 2 heads x 6 elevations x 128 azimuths */
constexpr int kChunks = kRays / 32; /* 32 consecutive azimuths of one elevation row */
constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ float fm(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fa(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fs(float a, float b) { return __fsub_rn(a, b); }

/* Per-aircraft summary of the two LiDAR passes (onboard_features.cuh:185-234). */
struct RayStats {
    float min_r, min_r_dx, min_r_dy;  /* nearest return in elevations 0..3 and its world x, y */
    float min_dx_c;                   /* nearest obstacle centre ahead inside the corridor */
    float cluster_y_sum;              /* sum of corridor centres' y within 1.4 m of min_dx_c, or a
                                         value of the same sign (only its sign is read) */
    int cluster_count;
};

/* The reference's initial values (onboard_features.cuh:188-199). */
__device__ __forceinline__ RayStats initial_stats() {
    RayStats s;
    s.min_r = 30.0f;
    s.min_r_dx = 0.0f;
    s.min_r_dy = 0.0f;
    s.min_dx_c = 30.0f;
    s.cluster_y_sum = 0.0f;
    s.cluster_count = 0;
    return s;
}

/* RayStats parked in the first six floats of a prior row between the scan
 * and the control-law launch. */
__device__ __forceinline__ void park_stats(float *row, const RayStats &st) {
    row[0] = st.min_r;
    row[1] = st.min_r_dx;
    row[2] = st.min_r_dy;
    row[3] = st.min_dx_c;
    row[4] = st.cluster_y_sum;
    row[5] = __int_as_float(st.cluster_count);
}

__device__ __forceinline__ RayStats unpark_stats(const float *row) {
    RayStats st;
    st.min_r = row[0];
    st.min_r_dx = row[1];
    st.min_r_dy = row[2];
    st.min_dx_c = row[3];
    st.cluster_y_sum = row[4];
    st.cluster_count = __float_as_int(row[5]);
    return st;
}

/* Body-to-world rotation of the normalised attitude quaternion
 * (onboard_features.cuh:104-137), from sanitised observations 6..9. */
struct Attitude {
    float qw, qx, qy, qz;
    float r00, r01, r02, r10, r11, r12, r20, r21, r22;
};

__device__ __forceinline__ Attitude attitude_from(const float o6, const float o7, const float o8,
                                                  const float o9) {
    Attitude a;
    float qnorm = fmaxf(__fsqrt_rn(fa(fa(fm(o6, o6), fm(o7, o7)), fm(o8, o8))), 0.0f);
    qnorm = fmaxf(__fsqrt_rn(fa(fm(qnorm, qnorm), fm(o9, o9))), 1.0e-8f);
    const float sign = o6 < 0.0f ? -1.0f : 1.0f;
    a.qw = __fdiv_rn(fm(sign, o6), qnorm);
    a.qx = __fdiv_rn(fm(sign, o7), qnorm);
    a.qy = __fdiv_rn(fm(sign, o8), qnorm);
    a.qz = __fdiv_rn(fm(sign, o9), qnorm);
    const float qw = a.qw, qx = a.qx, qy = a.qy, qz = a.qz;
    a.r00 = fs(1.0f, fm(2.0f, fa(fm(qy, qy), fm(qz, qz))));
    a.r01 = fm(2.0f, fs(fm(qx, qy), fm(qw, qz)));
    a.r02 = fm(2.0f, fa(fm(qx, qz), fm(qw, qy)));
    a.r10 = fm(2.0f, fa(fm(qx, qy), fm(qw, qz)));
    a.r11 = fs(1.0f, fm(2.0f, fa(fm(qx, qx), fm(qz, qz))));
    a.r12 = fm(2.0f, fs(fm(qy, qz), fm(qw, qx)));
    a.r20 = fm(2.0f, fs(fm(qx, qz), fm(qw, qy)));
    a.r21 = fm(2.0f, fa(fm(qy, qz), fm(qw, qx)));
    a.r22 = fs(1.0f, fm(2.0f, fa(fm(qx, qx), fm(qy, qy))));
    return a;
}

/* Ray direction tables, in tb_scan_tables.h's layout. */
struct RayTables {
    float cos_el[12], sin_el[12];     /* index head * 6 + el */
    float cos_az[128], sin_az[128];
};
static_assert(sizeof(RayTables) == TB_SCAN_TABLE_FLOATS * sizeof(float), "table layout");

/* Copy the tables into shared memory, by `count` threads numbered `tid`. */
__device__ __forceinline__ void load_tables(RayTables &t, int tid, int count) {
    float *dst = reinterpret_cast<float *>(&t);
    for (int i = tid; i < TB_SCAN_TABLE_FLOATS; i += count) dst[i] = tb_scan_tables[i];
}

/* World direction components of ray (row, azi) (onboard_features.cuh:
 * 190-196): x, y and (for the corridor) z. */
__device__ __forceinline__ void ray_world(const RayTables &t, const Attitude &a, int row, int azi, float &rwx,
                                          float &rwy, float &rwz) {
    const float ce = t.cos_el[row];
    const float rx = fm(ce, t.cos_az[azi]), ry = fm(ce, t.sin_az[azi]), rz = t.sin_el[row];
    rwx = fa(fa(fm(a.r00, rx), fm(a.r01, ry)), fm(a.r02, rz));
    rwy = fa(fa(fm(a.r10, rx), fm(a.r11, ry)), fm(a.r12, rz));
    rwz = fa(fa(fm(a.r20, rx), fm(a.r21, ry)), fm(a.r22, rz));
}

/* Scratch shared by the warps of block_scan: one entry per warp. */
struct WarpPart {
    float near_r, near_wx, near_wy, ahead_x;
    int near_ray, ahead_ray, count, pad;
    double dsum, dabs;
};

template <int kWarps>
struct BlockScanShared {
    RayTables tables;
    WarpPart part[kWarps];
    float exact_sum;
};

__device__ __forceinline__ void group_sync(int bar_id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(threads) : "memory");
}

/* Smaller (value, ray) first: the reference's "first strictly smaller" over
 * rays visited in increasing order. */
__device__ __forceinline__ bool before(float v, int ray, float ov, int oray) {
    return ov < v || (ov == v && oray < ray);
}

/* Corridor test of one ray (onboard_features.cuh:197-206): its centre x and
 * y, and whether it is in the corridor. */
__device__ __forceinline__ bool corridor_ray(const RayTables &t, const Attitude &a, int row, int azi, float range,
                                             float py, float &x_center, float &y_center) {
    const bool valid = range > 0.35f && range < 11.5f;
    float rwx, rwy, rwz;
    ray_world(t, a, row, azi, rwx, rwy, rwz);
    const float wx = fm(rwx, range), wy = fm(rwy, range), wz = fm(rwz, range);
    x_center = fa(wx, fm(rwx, 1.10f));
    y_center = fa(fa(py, wy), fm(rwy, 1.10f));
    return valid && fabsf(wz) <= 2.1f && x_center >= -0.35f && x_center <= 10.5f && fabsf(y_center) <= 3.5f;
}

/* Both passes over one aircraft's 1,536 controller rays by kWarps warps
 * (all 32 * kWarps threads call it together; they synchronise on named
 * barrier `bar_id`).  `head0` / `head1` point at elevation row 0 of the two
 * LiDAR heads (observation columns 48 and 2,096); ray r = row * 128 + azi
 * (row = head * 6 + el) reads head0[r] for rows 0..5, head1[r - 768] for rows
 * 6..11.  Warp w takes the 32-ray chunks w, w + kWarps, ... in increasing
 * order, so each lane's running minima keep the first occurrence and the
 * (value, ray) arg-min over lanes and then warps reproduces the sequential
 * result.  A range outside (0.35, 11.5) enters neither pass.  want_near
 * (dodge missions) computes the nearest return in elevations 0..3;
 * want_corridor (slalom) the corridor results.  Each lane keeps its rays'
 * corridor centres (x, and y, which pass 2 sums: the same expression) in
 * registers between the passes.  Of the cluster y sum only the sign is
 * read: it is decided from a double sum and a bound on the in-order float
 * sum's rounding ((n - 1) 2^-24 sum|y|, doubled), and only when that cannot
 * decide is the in-order float sum formed (warp 0, ray order, recomputing
 * each ray).  Returns the same RayStats in every thread. */
template <int kWarps>
__device__ RayStats block_scan(BlockScanShared<kWarps> &sh, const float *head0, const float *head1,
                               const Attitude &a, float py, bool want_near, bool want_corridor, int warp, int lane,
                               int bar_id) {
    static_assert(kChunks % kWarps == 0, "chunks split evenly over the warps");
    constexpr int kPerWarp = kChunks / kWarps;
    const int threads = 32 * kWarps;
    const float inf = __int_as_float(0x7f800000);
    const RayTables &t = sh.tables;
    float near_r = inf, near_wx = 0.0f, near_wy = 0.0f;
    int near_ray = 0x7fffffff;
    float ahead_x = inf;
    int ahead_ray = 0x7fffffff;
    float cx[kPerWarp], cy[kPerWarp]; /* this lane's corridor centres (x = +inf outside) */

    /* Pass 1 (onboard_features.cuh:188-207). */
#pragma unroll
    for (int j = 0; j < kPerWarp; ++j) {
        cx[j] = inf;
        cy[j] = 0.0f;
        const int c = warp + j * kWarps;
        const int row = c >> 2;
        const int el = row >= 6 ? row - 6 : row;
        const bool near_row = want_near && el < 4;
        if (!near_row && !want_corridor) continue;
        const int azi = ((c & 3) << 5) + lane;
        const int ray = (c << 5) + lane;
        const float range = row < 6 ? head0[ray] : head1[ray - 768];
        if (want_corridor) {
            float x_center, y_center;
            const bool corridor = corridor_ray(t, a, row, azi, range, py, x_center, y_center);
            if (corridor && x_center < ahead_x) {
                ahead_x = x_center;
                ahead_ray = ray;
            }
            if (corridor) {
                cx[j] = x_center;
                cy[j] = y_center;
            }
        }
        if (near_row && range > 0.35f && range < 11.5f && range < near_r) {
            float rwx, rwy, rwz;
            ray_world(t, a, row, azi, rwx, rwy, rwz);
            near_r = range;
            near_ray = ray;
            near_wx = fm(rwx, range);
            near_wy = fm(rwy, range);
        }
    }
    /* warp arg-mins; the nearest return's world offsets travel with it */
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(kFull, near_r, off);
        const int oi = __shfl_xor_sync(kFull, near_ray, off);
        const float ox = __shfl_xor_sync(kFull, near_wx, off);
        const float oy = __shfl_xor_sync(kFull, near_wy, off);
        if (before(near_r, near_ray, ov, oi)) {
            near_r = ov;
            near_ray = oi;
            near_wx = ox;
            near_wy = oy;
        }
        const float av = __shfl_xor_sync(kFull, ahead_x, off);
        const int ai = __shfl_xor_sync(kFull, ahead_ray, off);
        if (before(ahead_x, ahead_ray, av, ai)) {
            ahead_x = av;
            ahead_ray = ai;
        }
    }
    if (lane == 0) {
        WarpPart &p = sh.part[warp];
        p.near_r = near_r;
        p.near_ray = near_ray;
        p.near_wx = near_wx;
        p.near_wy = near_wy;
        p.ahead_x = ahead_x;
        p.ahead_ray = ahead_ray;
    }
    group_sync(bar_id, threads);
    /* block arg-mins, the same in every thread */
    for (int w = 0; w < kWarps; ++w) {
        const WarpPart &p = sh.part[w];
        if (before(near_r, near_ray, p.near_r, p.near_ray)) {
            near_r = p.near_r;
            near_ray = p.near_ray;
            near_wx = p.near_wx;
            near_wy = p.near_wy;
        }
        if (before(ahead_x, ahead_ray, p.ahead_x, p.ahead_ray)) {
            ahead_x = p.ahead_x;
            ahead_ray = p.ahead_ray;
        }
    }
    RayStats s = initial_stats();
    if (want_near && near_r < 30.0f) {
        s.min_r = near_r;
        s.min_r_dx = near_wx;
        s.min_r_dy = near_wy;
    }
    if (!want_corridor) return s;
    s.min_dx_c = ahead_x < 30.0f ? ahead_x : 30.0f;

    /* Pass 2 (onboard_features.cuh:213-233): corridor centres within 1.4 m
     * of the nearest. */
    const float limit = fa(s.min_dx_c, 1.4f);
    int count = 0;
    double dsum = 0.0, dabs = 0.0;
#pragma unroll
    for (int j = 0; j < kPerWarp; ++j) {
        const bool member = cx[j] <= limit;
        count += __popc(__ballot_sync(kFull, member));
        if (member) {
            dsum += static_cast<double>(cy[j]);
            dabs += fabs(static_cast<double>(cy[j]));
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        dsum += __shfl_xor_sync(kFull, dsum, off);
        dabs += __shfl_xor_sync(kFull, dabs, off);
    }
    if (lane == 0) { /* fields the arg-min loop above does not read */
        sh.part[warp].count = count;
        sh.part[warp].dsum = dsum;
        sh.part[warp].dabs = dabs;
    }
    group_sync(bar_id, threads);
    count = 0;
    dsum = 0.0;
    dabs = 0.0;
    for (int w = 0; w < kWarps; ++w) {
        count += sh.part[w].count;
        dsum += sh.part[w].dsum;
        dabs += sh.part[w].dabs;
    }
    s.cluster_count = count;
    const double bound = 2.0 * static_cast<double>(count) * 0x1.0p-24 * dabs;
    /* The bound assumes no in-order float partial sum overflows: each is at
     * most sum|y| (1 + n 2^-24) in magnitude, below FLT_MAX when sum|y| <
     * 2^127 (n <= 1,536).  Larger or non-finite sums take the exact path. */
    if (dabs < 0x1.0p127 && fabs(dsum) > bound) {
        s.cluster_y_sum = dsum > 0.0 ? 1.0f : -1.0f; /* the in-order float sum's sign */
        return s;
    }
    /* Ambiguous sign: warp 0 forms the reference's in-order float sum. */
    if (warp == 0) {
        float ysum = 0.0f;
        for (int c = 0; c < kChunks; ++c) {
            const int row = c >> 2, azi = ((c & 3) << 5) + lane;
            const int ray = (c << 5) + lane;
            const float range = row < 6 ? head0[ray] : head1[ray - 768];
            float x_center, y_center;
            const bool corridor = corridor_ray(t, a, row, azi, range, py, x_center, y_center);
            unsigned mask = __ballot_sync(kFull, corridor && x_center <= limit);
            while (mask) {
                ysum = fa(ysum, __shfl_sync(kFull, y_center, __ffs(mask) - 1));
                mask &= mask - 1;
            }
        }
        if (lane == 0) sh.exact_sum = ysum;
    }
    group_sync(bar_id, threads);
    s.cluster_y_sum = sh.exact_sum;
    return s;
}

} /* namespace tb_scan */

#endif
