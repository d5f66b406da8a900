/*
 * A camera pixel decided in single precision, when single precision provably
 * gives the simulator's byte (reference src/sim/sensors.c:11-26 trace,
 * :59-68 shade, rotation sim_internal.h:85).  Shared by the sensor kernel
 * (sensors_kernel.cu, compiled by nvcc) and by a test build of the CPU
 * renderer restatement (oracle/, compiled by gcc), so the same decision code
 * is checked bit for bit against the double renderer on the CPU.
 *
 * tbf_camera_pixel returns 1 and the byte when it can prove it; 0 when the
 * caller must trace the ray in double.  It handles the rays whose double
 * trace ends at the sky or the ground with every sphere missed, in units
 * whose attitude is a rotation and that have no raised shelf (the caller
 * checks those per unit), or at the arena dome (tbf_dome).
 *
 * Error bounds, u = 2^-24, all arithmetic plain float (the kernel's file is
 * built without contraction):
 *  - Direction: tb_rotate's formula with |q| = 1 (to 1e-9) and |v| = 1, in
 *    float from float copies of q and v, is within 35 u = 2.1e-6 of the
 *    double direction per component (each of the 18 operations rounds by u
 *    of a value <= 2, and the inputs by u).  TBF_ED = 8e-6 is used.
 *  - Sphere miss: b = oc.d in float is within sqrt(3) L TBF_ED + 5 u L of
 *    the double b (L = |oc|); b*b + (r^2 - L^2) is then within
 *    2.9e-5 (L^2 + r^2) of the double discriminant.  The caller's margin is
 *    1.2e-4 (L^2 + r^2): a float value below minus it proves "no hit".
 *  - Ground: the simulator tests d.z < -1e-5, then t = (0 - oz) / d.z
 *    against 0.05 and the sky distance.  d.z is decided when it clears -1e-5
 *    by TBF_ED; t in float is within rel = TBF_ED / (|dz| - TBF_ED) + 4 u
 *    (relative) of the double t, and the tests use t (1 -+ 2 rel).
 *  - Byte: round(luma * fog * 255) with luma from d.z and fog from the sky
 *    factor or from t through expf (CUDA's __expf, within 3e-7 for arguments
 *    <= 0, checked exhaustively by a GPU test; glibc's expf is closer).  The
 *    float value is within 255 (0.15 TBF_ED + 5e-7) of the double one for the
 *    sky and 255 (0.17 TBF_ED + 0.00625 e t rel + 6e-7) for the ground; the
 *    byte is taken when x + 0.5 clears an integer by that plus 8e-6 (the
 *    rounding of the addition).
 */
#ifndef TB_CAMERA_FLOAT_H
#define TB_CAMERA_FLOAT_H

#include <math.h>

#ifdef __CUDACC__
#define TBF_FN static __device__ __forceinline__
#define TBF_EXPF(x) __expf(x)
#else
#define TBF_FN static inline
#define TBF_EXPF(x) expf(x)
#endif

#define TBF_ED 8e-6f                 /* per-component bound on the float direction's error */
#define TBF_U 5.9604645e-8f          /* 2^-24 */
#define TBF_SPHERE_MARGIN 1.2e-4     /* times (L^2 + r^2): the float sphere-miss margin */

/* Per unit: the attitude and origin height in float, the sky distance and the
 * sky's shading factor. */
typedef struct tbf_unit {
    float qw, qx, qy, qz;
    float oz;
    float sky_fog;
    double best0;
    int dome;          /* the arena dome can be hit before the sky distance */
    float ox, oy;      /* origin x, y (dome test) */
    float dome_cc;     /* ox^2 + oy^2 - dome^2, rounded from the double value */
} tbf_unit;

/* The dome's exit distance td = (-qb + sqrt(qb^2 - 4 qa qc)) / (2 qa) along
 * the float direction, with qa = dx^2 + dy^2, qb = 2 (ox dx + oy dy),
 * qc = dome_cc (trace's expressions), and a bound on |td - td_double|.
 * Returns 1 with *td, *err when the dome test is decided and hit-capable,
 * 0 when it certainly returns no hit (qa <= 1e-9 or disc < 0), -1 when it
 * cannot tell.  Bounds (R = |ox| + |oy|, E = TBF_ED): qa within
 * 2.9 E + 4u, qb within 2 R (E + 4u), qc within u |qc|; the discriminant and
 * td bounds follow from those by first-order propagation, doubled. */
TBF_FN int tbf_dome(const tbf_unit *u, float dx, float dy, float *td, float *err) {
    const float qa = dx * dx + dy * dy;
    const float eqa = 2.9f * TBF_ED + 4.0f * TBF_U;
    if (qa + eqa <= 1e-9f) return 0;
    if (!(qa - eqa > 1e-9f) || !(qa > 4.0f * eqa)) return -1;
    const float R = fabsf(u->ox) + fabsf(u->oy);
    const float qb = 2.0f * (u->ox * dx + u->oy * dy);
    const float eqb = 2.0f * R * (TBF_ED + 4.0f * TBF_U);
    const float qc = u->dome_cc;
    const float eqc = TBF_U * fabsf(qc);
    const float disc = qb * qb - 4.0f * qa * qc;
    const float B = fabsf(qb), C = fabsf(qc);
    const float edisc = 2.0f * (2.0f * B * eqb + eqb * eqb + 4.0f * (qa * eqc + C * eqa + eqa * eqc) +
                                3.0f * TBF_U * (B * B + 4.0f * qa * C));
    if (disc + edisc < 0.0f) return 0;
    if (!(disc > 4.0f * edisc)) return -1;
    const float root = sqrtf(disc);
    const float eroot = edisc / root + TBF_U * root;
    const float num = -qb + root;
    const float enum_ = eqb + eroot + TBF_U * (B + root);
    if (!(fabsf(num) > 4.0f * enum_)) return -1;
    *td = num / (2.0f * qa);
    *err = 2.0f * fabsf(*td) * (enum_ / fabsf(num) + eqa / qa + 3.0f * TBF_U);
    return 1;
}

/* Per sphere: origin - centre (x, y, z) and r^2 - |origin - centre|^2 (w). */
typedef struct tbf_sphere {
    float x, y, z, w;
} tbf_sphere;

TBF_FN int tbf_camera_pixel(const tbf_unit *u, const tbf_sphere *spheres, const float *margins, int n, float vx,
                            float vy, float vz, unsigned int *byte) {
    const float qw = u->qw, qx = u->qx, qy = u->qy, qz = u->qz;
    const float cx = qy * vz - qz * vy, cy = qz * vx - qx * vz, cz = qx * vy - qy * vx;
    const float tx = cx * 2.0f, ty = cy * 2.0f, tz = cz * 2.0f;
    const float ax = vx + tx * qw, ay = vy + ty * qw, az = vz + tz * qw;
    const float dx = ax + (qy * tz - qz * ty), dy = ay + (qz * tx - qx * tz), dz = az + (qx * ty - qy * tx);
    for (int i = 0; i < n; ++i) {
        const float b = spheres[i].x * dx + spheres[i].y * dy + spheres[i].z * dz;
        if (!(b * b + spheres[i].w < -margins[i])) return 0;
    }
    int ground = 0;
    float t = 0.0f, rel = 0.0f;
    double best_lo = u->best0, best_hi = u->best0; /* trace's `best` after the ground test */
    if (dz < -1e-5f - TBF_ED) {
        t = -u->oz / dz;
        rel = TBF_ED / (-dz - TBF_ED) + 4.0f * TBF_U;
        if (!(rel < 0.01f)) return 0;
        const double lo = (double)t * (1.0 - 2.0 * rel), hi = (double)t * (1.0 + 2.0 * rel);
        if (lo > 0.05 && hi < u->best0) {
            ground = 1;
            best_lo = lo;
            best_hi = hi;
        } else if (!(hi < 0.05 || lo > u->best0)) {
            return 0; /* too close to call: the double trace decides */
        }
    } else if (!(dz > -1e-5f + TBF_ED)) {
        return 0;
    }
    /* the dome is tested after the spheres (all missed) and before the balls
     * (in the sphere list, all missed): it wins when td > 0.05 and td < best */
    int dome = 0;
    float td = 0.0f, etd = 0.0f;
    if (u->dome) {
        const int d = tbf_dome(u, dx, dy, &td, &etd);
        if (d < 0) return 0;
        if (d > 0) {
            const double lo = (double)td - etd, hi = (double)td + etd;
            if (lo > 0.05 && hi < best_lo)
                dome = 1;
            else if (!(hi < 0.05 || lo > best_hi))
                return 0;
        }
    }
    float x, m;
    if (dome) {
        const float e = TBF_EXPF(td * -0.0125f);
        x = 0.46f * (0.75f + 0.25f * e) * 255.0f;
        m = 255.0f * (0.46f * 0.25f * (e + 1e-6f) * (etd + 3.0f * TBF_U * td) * 0.0125f + 6e-7f);
    } else if (ground) {
        const float luma = 0.28f + 0.17f * fminf(1.0f, fmaxf(0.0f, -dz));
        const float e = TBF_EXPF(t * -0.0125f);
        x = luma * (0.75f + 0.25f * e) * 255.0f;
        m = 255.0f * (0.17f * TBF_ED + 0.00625f * (e + 1e-6f) * t * rel + 6e-7f);
    } else {
        x = (0.22f + 0.15f * fminf(1.0f, fmaxf(-1.0f, dz))) * u->sky_fog * 255.0f;
        m = 255.0f * (0.15f * TBF_ED + 5e-7f);
    }
    m += 8e-6f;
    const float y = x + 0.5f;
    const float k = floorf(y);
    const float r = y - k;
    if (!(r > m && r < 1.0f - m)) return 0;
    *byte = (unsigned int)fminf(255.0f, fmaxf(0.0f, k));
    return 1;
}

#endif
