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
 * whose attitude is a rotation and that have no raised shelf and no arena
 * dome within the sky distance (the caller checks those per unit).  (A float
 * dome test was written, checked bit for bit and dropped: it decided more
 * pixels but cost more time than it saved.)
 *
 * Error bounds, u = 2^-24, in float arithmetic where each multiply-add is
 * written as one fused operation (TBF_FMA, rounded once; the kernel's file
 * is otherwise built without contraction).  A fused a * b + c rounds once
 * where the separate product and sum round twice, so every bound below,
 * derived for separate roundings, holds for it too:
 *  - Direction: tb_rotate's formula with |q| = 1 (to 1e-9) and |v| = 1, in
 *    float from float copies of q and v, is within 35 u = 2.1e-6 of the
 *    double direction per component (each of at most 18 roundings is by u
 *    of a value <= 2, and the inputs by u).  TBF_ED = 8e-6 is used.
 *  - Sphere miss: b = oc.d in float is within sqrt(3) L TBF_ED + 5 u L of
 *    the double b (L = |oc|); b*b + (r^2 - L^2) is then within
 *    2.9e-5 (L^2 + r^2) of the double discriminant.  The caller's margin is
 *    1.2e-4 (L^2 + r^2): a float value below minus it proves "no hit".
 *  - Ground: the simulator tests d.z < -1e-5, then t = (0 - oz) / d.z
 *    against 0.05 and the sky distance.  d.z is decided when it clears -1e-5
 *    by TBF_ED; t in float (a division within 2 ulp) is within
 *    rel = TBF_ED / (|dz| - TBF_ED) + 6 u (relative) of the double t, and
 *    the tests use t (1 -+ 2 rel), in float with 4 u more for their own
 *    rounding, against 0.05 and the sky distance widened by 1e-6 relative.
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
#define TBF_FMA(a, b, c) __fmaf_rn((a), (b), (c))
#define TBF_FDIV(a, b) __fdividef((a), (b)) /* within 2 ulp for |b| in [2^-126, 2^126] */
#else
#define TBF_FN static inline
#define TBF_EXPF(x) expf(x)
#define TBF_FMA(a, b, c) fmaf((a), (b), (c)) /* correctly rounded, like the GPU's */
#define TBF_FDIV(a, b) ((a) / (b))
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
    float best0_lo, best0_hi; /* best0 (1 -+ 1e-6) in float: bounds for float comparisons */
} tbf_unit;

/* Per sphere: origin - centre (x, y, z) and r^2 - |origin - centre|^2 (w). */
typedef struct tbf_sphere {
    float x, y, z, w;
} tbf_sphere;

TBF_FN int tbf_camera_pixel(const tbf_unit *u, const tbf_sphere *spheres, const float *margins, int n, float vx,
                            float vy, float vz, unsigned int *byte) {
    const float qw = u->qw, qx = u->qx, qy = u->qy, qz = u->qz;
    const float cx = TBF_FMA(qy, vz, -(qz * vy)), cy = TBF_FMA(qz, vx, -(qx * vz)), cz = TBF_FMA(qx, vy, -(qy * vx));
    const float tx = cx * 2.0f, ty = cy * 2.0f, tz = cz * 2.0f;
    const float ax = TBF_FMA(tx, qw, vx), ay = TBF_FMA(ty, qw, vy), az = TBF_FMA(tz, qw, vz);
    const float dx = ax + TBF_FMA(qy, tz, -(qz * ty)), dy = ay + TBF_FMA(qz, tx, -(qx * tz)),
                dz = az + TBF_FMA(qx, ty, -(qy * tx));
    for (int i = 0; i < n; ++i) {
        const float b = TBF_FMA(spheres[i].z, dz, TBF_FMA(spheres[i].y, dy, spheres[i].x * dx));
        if (!(TBF_FMA(b, b, spheres[i].w) < -margins[i])) return 0;
    }
    int ground = 0;
    float t = 0.0f, rel = 0.0f;
    if (dz < -1e-5f - TBF_ED) {
        /* the division is within 2 ulp (CUDA's __fdividef; exact on the CPU):
         * t within rel of the double t, rel an over-estimate (1.001 covers the
         * error of its own division) */
        t = TBF_FDIV(-u->oz, dz);
        rel = 1.001f * TBF_FDIV(TBF_ED, -dz - TBF_ED) + 6.0f * TBF_U;
        if (!(rel < 0.01f)) return 0;
        /* t (1 -+ 2 rel), widened by 4 u for the products' own rounding */
        const float lo = t * (1.0f - 2.0f * rel - 4.0f * TBF_U), hi = t * (1.0f + 2.0f * rel + 4.0f * TBF_U);
        if (lo > 0.050001f && hi < u->best0_lo)
            ground = 1;
        else if (!(hi < 0.049999f || lo > u->best0_hi))
            return 0; /* too close to call: the double trace decides */
    } else if (!(dz > -1e-5f + TBF_ED)) {
        return 0;
    }
    float x, m;
    if (ground) {
        const float luma = TBF_FMA(0.17f, fminf(1.0f, fmaxf(0.0f, -dz)), 0.28f);
        const float e = TBF_EXPF(t * -0.0125f);
        x = luma * TBF_FMA(0.25f, e, 0.75f) * 255.0f;
        m = 255.0f * (0.17f * TBF_ED + 0.00625f * (e + 1e-6f) * t * rel + 6e-7f);
    } else {
        x = TBF_FMA(0.15f, fminf(1.0f, fmaxf(-1.0f, dz)), 0.22f) * u->sky_fog * 255.0f;
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
