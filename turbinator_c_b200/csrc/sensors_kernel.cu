/*
 * sm_100a ray tracer for the simulator's sensors: per scene the 2 x 2,048
 * LiDAR rays and the 4 x 4,096 camera rays, for a batch of scenes in one
 * launch (tb_cuda_render_sensors_device, include/turbinator/sim/cuda_sensors.h).
 *
 * Reference (Viatreen/Turbinator_C src/sim/sensors.c):
 *   sphere_hit :4-10, trace :11-26, tb_sim_render_lidar :28-50,
 *   camera_ray :52-58, shade :59-68, tb_sim_render_camera :69-82;
 *   helpers tb_rotate / tb_clamp / tb_is_arena / tb_is_bwb, sim_internal.h:73-88;
 *   tb_rand64 (SplitMix64), physics.c:73-78.
 *
 * Design (B200):
 *  - Work unit = a scene's two LiDAR heads (2 x 2,048 rays from two origins,
 *    both sphere lists formed in one setup, the heads rendered in turn) or
 *    one camera view (4,096 rays from one origin, rendered as two halves of
 *    32 rows) -- 5 units per scene, one CTA per unit, CTAs striding over
 *    units.  Each unit traces from a single origin, so the
 *    ray-independent sphere terms (o - c, |o - c|^2, r^2) and the dome's
 *    constant term are formed once per CTA in shared memory and read as warp
 *    broadcasts (two 128-bit and one 64-bit load per sphere).  Two
 *    shared-memory slots (pairs for LiDAR) alternate over a CTA's units, so a
 *    unit costs two CTA barriers (both while its sphere lists are formed); the LiDAR valid count is
 *    summed with shared-memory atomics and written by the last warp.
 *  - Sphere culling per unit: a sphere whose surface lies farther than the
 *    sky distance can never beat it, and a unit's rays lie in a cone (axis
 *    and half-angle per unit, from the ray tables).  A sphere that every ray
 *    of the cone misses by a margin -- the exact discriminant at most
 *    -1e-12 * max(1, L)^2 against a rounding error below 1e-14 * L^2, or the
 *    whole sphere behind the origin by more than 0.1 m -- would return "no
 *    hit" for every ray.  Either way the sphere is left out of that unit's
 *    list; the remaining spheres keep their order.  Only unit attitudes
 *    (|q|^2 within 1e-9 of 1) with finite geometry are culled; anything else
 *    keeps every sphere.  Likewise the arena dome is skipped (unit attitudes
 *    only) for a unit whose origin is so far inside it that every dome hit
 *    lies beyond the sky.  Camera units then cull again per warp: each warp
 *    renders a 16 x 16 pixel tile, tests the unit's list against its tile's
 *    own cone (the same test) and traces its pixels against the spheres left
 *    (24-89 spheres in the heaviest scenes, a few per tile).
 *  - Body-frame ray directions do not depend on the scene: they are built on
 *    the host with the C library the simulator uses (sensor_rays.c) and read
 *    from global memory (SoA, the camera's in tile order, coalesced); the
 *    kernel only rotates them.
 *  - The LiDAR noise stream is SplitMix64, whose state after k draws is
 *    seed + k * golden, so ray k hashes its own state without a sequential
 *    pass.
 *  - Everything is evaluated in double precision with the simulator's
 *    expression order and no multiply-add contraction (this file is built
 *    with -fmad=false); double division and square root are correctly
 *    rounded, so ranges equal the simulator's bit for bit.  The only
 *    transcendental per ray is the camera's exp(-d/80), evaluated once per
 *    unit for sky pixels (whose distance is the unit's constant sky distance).
 *  - Camera bytes are written four pixels per 32-bit store (a warp covers
 *    eight 16-byte row segments of its tile); the optional raw capture
 *    writes each pixel 3 x 3.
 *  The work is FP64-pipe and issue bound (no tensor-core or HBM bound
 *  applies): about 35 double operations to rotate a ray plus about 8 per
 *  sphere tested.
 */
#include <cuda_runtime.h>

#include <math.h>
#include <stdint.h>

#include <mutex>

#include "tb_camera_float.h"
#include "tb_sensor_rays.h"
#include "turbinator/sim/cuda_sensors.h"

#ifndef TB_SENSOR_THREADS
#define TB_SENSOR_THREADS 256
#endif
#ifndef TB_SENSOR_MIN_BLOCKS
#define TB_SENSOR_MIN_BLOCKS 4
#endif
#ifndef TB_SENSOR_CULL
#define TB_SENSOR_CULL 1
#endif

namespace {

constexpr int kThreads = TB_SENSOR_THREADS;
constexpr int kWarps = kThreads / 32;
constexpr int kUnitRays = 2048;
constexpr int kUnitsPerScene = 6; /* 2 LiDAR heads + 4 camera views */
constexpr int kMaxSpheres = TB_SENSOR_MAX_OBSTACLES + 1 + TB_SENSOR_MAX_BALLS;
constexpr int kSphereWarps = (kMaxSpheres + 31) / 32;
constexpr int kLidarBins = TB_SENSOR_LIDAR_BINS;
constexpr int kCameraPixels = TB_SENSOR_CAMERA_PIXELS;
constexpr unsigned long long kGolden = 0x9e3779b97f4a7c15ull;

static_assert(sizeof(tb_sensor_scene) == 2432, "scene record layout");
static_assert(kThreads >= 32 * kSphereWarps && kUnitRays % (4 * kThreads) == 0, "unit split");

/* Body-frame directions, structure of arrays. */
__device__ double g_lidar_x[kLidarBins], g_lidar_y[kLidarBins], g_lidar_z[kLidarBins];
__device__ unsigned int g_lidar_blocked[kLidarBins / 32];
/* Camera directions in tile order: entry (half * 8 + warp) * 256 + e is the
 * camera kernel's entry e of tile `warp` of view half `half` (view * 2 + top
 * or bottom; tile_pixel), so a warp's loads of its 256 rays are contiguous. */
__device__ double g_camera_x[kCameraPixels], g_camera_y[kCameraPixels], g_camera_z[kCameraPixels];
/* The same camera directions rounded to float, for the float pixel test. */
__device__ float g_camera_fx[kCameraPixels], g_camera_fy[kCameraPixels], g_camera_fz[kCameraPixels];
/* Per unit kind: body-frame cone axis (unit) and cos, sin of its half-angle
 * widened by 1e-6 rad. */
__device__ double g_cone[kUnitsPerScene][5];
/* The same per camera tile: view half (view * 2 + half), warp (the warp's
 * 16 x 16 pixels, rows 16 (w / 4) .. of the half, columns 16 (w % 4) ..). */
constexpr int kCameraHalves = 8; /* camera view halves (32 rows each) per scene: view * 2 + half */
__device__ double g_tile_cone[kCameraHalves][kThreads / 32][5];
constexpr int kTileCols = 16;                        /* a warp's tile: 256 / kTileCols rows of kTileCols */
static_assert((kThreads / 32) * 256 == 2048, "one 256-pixel tile per warp covers a camera unit's 2,048 pixels");
constexpr int kTileRows = 256 / kTileCols;
constexpr int kTilesAcross = 64 / kTileCols;
/* first pixel of view half `unit`'s (view * 2 + half) tile `warp`, and entry e's pixel */
__host__ __device__ constexpr int tile_first(int unit, int warp) {
    return (unit >> 1) * 4096 + (unit & 1) * 2048 + (warp / kTilesAcross) * kTileRows * 64 +
           (warp % kTilesAcross) * kTileCols;
}
__host__ __device__ constexpr int tile_pixel(int first, int e) { return first + (e / kTileCols) * 64 + e % kTileCols; }

struct Vec {
    double x, y, z;
};

/* tb_rotate (sim_internal.h:85): v + 2w(u x v) + u x (2(u x v)). */
__device__ __forceinline__ Vec rotate(double qw, double qx, double qy, double qz, Vec v) {
    const Vec c = {qy * v.z - qz * v.y, qz * v.x - qx * v.z, qx * v.y - qy * v.x};
    const Vec t = {c.x * 2, c.y * 2, c.z * 2};
    const Vec a = {v.x + t.x * qw, v.y + t.y * qw, v.z + t.z * qw};
    return Vec{a.x + (qy * t.z - qz * t.y), a.y + (qz * t.x - qx * t.z), a.z + (qx * t.y - qy * t.x)};
}

__device__ __forceinline__ bool is_bwb(int s) { return s >= 22 && s <= 27; }
__device__ __forceinline__ bool is_arena(int s) {
    return s == 3 || s == 14 || s == 15 || s == 16 || s == 18 || s == 22 || s == 24 || s == 27;
}

/* A unit's per-origin scalars. */
struct UnitHead {
    double q[4];
    double origin[3];
    double axis[3];   /* the unit's cone axis in the world frame */
    double best0;     /* trace()'s starting distance (also the sky distance) */
    double sky_fog;   /* shade()'s distance factor at best0 */
    double max_range; /* LiDAR clamp */
    double dome_cc;   /* o.x^2 + o.y^2 - dome^2 */
    unsigned long long seed;
    int n_obstacles, n_balls, arena; /* scene counts (clamped) */
    int dome;                        /* the dome can be hit before the sky distance */
    int cull;                        /* the attitude is a rotation: culling allowed */
    int shelf;                       /* scenario 10's raised ground at z = 9, x >= 20 */
    int float_camera;                /* camera pixels may be decided in float (tb_camera_float.h) */
};

/* One unit's scene, prepared for tracing from one origin. */
struct UnitScene {
    double2 oc_xy[kMaxSpheres]; /* origin - centre, x y */
    double2 oc_zq[kMaxSpheres]; /* origin - centre z, |origin - centre|^2 */
    double rr[kMaxSpheres];     /* radius^2 */
    float4 f_oc[kMaxSpheres];   /* float copies for the miss test: origin - centre, rr - |oc|^2 */
    float f_margin[kMaxSpheres]; /* the miss test's error margin (+inf: no float test) */
    float f_margin_ray[kMaxSpheres]; /* the same with a float ray direction (tb_camera_float.h) */
    UnitHead h;
    int kept_obstacles, kept_opponent, kept_total; /* the unit's list, in trace order */
    unsigned int keep_mask[kSphereWarps], obst_mask[kSphereWarps], opp_mask[kSphereWarps];
    int valid_count, warps_done; /* LiDAR valid rays of the unit, warps finished */
};

/* A camera tile's sphere list (camera kernel, one per warp). */
struct TileSpheres {
    float4 f_oc[kMaxSpheres];         /* UnitScene::f_oc of the listed spheres */
    float f_margin_ray[kMaxSpheres];  /* UnitScene::f_margin_ray of the listed spheres */
    unsigned char index[kMaxSpheres]; /* their places in the unit's list, increasing */
    int n_obst, n_opp;                /* listed obstacles, opponent (0 or 1) */
};

/* sphere_hit (sensors.c:4-10) with the ray-independent terms precomputed in
 * the same rounding: b = oc.d, disc = (b*b - oc.oc) + r*r.  `best` is the
 * caller's nearest hit so far: a sphere whose near intersection -b - sqrt(disc)
 * lies beyond it cannot change the result, and is dropped without the square
 * root when L = -b - best > 0 and L*L > disc by a relative 1e-9, with
 * L > 1e-6 (|b| + best).  Then sqrt(disc) < L (1 - 5e-10), so -b - sqrt(disc)
 * exceeds best by at least 5e-10 L > 4.4e-16 (|b| + best), more than the
 * rounding of L, of the square root and of the subtraction together: the
 * simulator's own arithmetic would have found t >= best (its far root is
 * larger still) and kept best. */
__device__ __forceinline__ double sphere_hit(const UnitScene &s, int i, Vec d, double best) {
    const double2 xy = s.oc_xy[i], zq = s.oc_zq[i];
    const double b = xy.x * d.x + xy.y * d.y + zq.x * d.z;
    const double disc = b * b - zq.y + s.rr[i];
    if (disc < 0) return INFINITY;
    const double lead = -b - best;
    if (lead > 1e-6 * (fabs(b) + best) && lead * lead > disc * (1 + 1e-9)) return INFINITY;
    const double root = sqrt(disc);
    double t = -b - root;
    if (t <= 0.05) t = -b + root;
    return t > 0.05 ? t : INFINITY;
}

/* True when sphere_hit would certainly find disc < 0 for ray d (no hit):
 * the discriminant evaluated in float from float copies of d and of the
 * sphere's terms lies below minus its error margin.  Error bound, with
 * u = 2^-24, L^2 = |oc|^2 and a unit ray (|d| <= 1 + 1e-8, which holds
 * whenever the unit's attitude passes the culling test; other units get an
 * infinite margin): rounding oc and d to float and forming b = oc.d with one
 * product and two FMAs puts b within 5.02 u L of oc.d; b*b is then within
 * 10.05 u L^2; rr - |oc|^2 rounded once to float adds u (|oc|^2 + rr); the
 * final FMA adds u (2 L^2 + rr).  So |disc_float - disc_exact| <= (13.1 L^2
 * + 2.01 rr) u < 2^-20 (L^2 + rr), while the double discriminant is within
 * 2^-51 (2 L^2 + rr) of disc_exact.  The margin stored is 2^-18 (L^2 + rr),
 * four times the float bound, so disc_float < -margin proves the double
 * disc < 0.  NaN fails the comparison and takes the double test. */
__device__ __forceinline__ bool certain_miss(const UnitScene &s, int i, float dx, float dy, float dz) {
    const float4 o = s.f_oc[i];
    const float b = __fmaf_rn(o.z, dz, __fmaf_rn(o.y, dy, __fmul_rn(o.x, dx)));
    return __fmaf_rn(b, b, o.w) < -s.f_margin[i];
}

/* trace (sensors.c:11-26): nearest hit along d from the unit's origin, in the
 * simulator's test order (ground, shelf, obstacles, opponent, dome, balls);
 * kind -1 sky, 0 ground, 1 obstacle, 2 opponent, 3 dome, 4 ball.  Spheres
 * that certainly miss are skipped by the float test above before the double
 * one. */
__device__ __forceinline__ double trace(const UnitScene &s, Vec d, int &kind) {
    double best = s.h.best0;
    kind = -1;
    const double ox = s.h.origin[0], oy = s.h.origin[1], oz = s.h.origin[2];
    const float dxf = __double2float_rn(d.x), dyf = __double2float_rn(d.y), dzf = __double2float_rn(d.z);
    if (d.z < -1e-5) {
        const double t = (0 - oz) / d.z;
        if (t > 0.05 && t < best) {
            best = t;
            kind = 0;
        }
        if (s.h.shelf) {
            const double t2 = (9 - oz) / d.z;
            if (t2 > 0.05 && t2 < best && ox + t2 * d.x >= 20) {
                best = t2;
                kind = 0;
            }
        }
    }
    int i = 0;
    for (; i < s.kept_obstacles; ++i) {
        if (certain_miss(s, i, dxf, dyf, dzf)) continue;
        const double t = sphere_hit(s, i, d, best);
        if (t < best) {
            best = t;
            kind = 1;
        }
    }
    if (s.h.arena) {
        if (s.kept_opponent) {
            if (!certain_miss(s, i, dxf, dyf, dzf)) {
                const double t = sphere_hit(s, i, d, best);
                if (t < best) {
                    best = t;
                    kind = 2;
                }
            }
            ++i;
        }
        if (s.h.dome) {
            const double a = d.x * d.x + d.y * d.y, b = 2 * (ox * d.x + oy * d.y);
            const double disc = b * b - 4 * a * s.h.dome_cc;
            if (a > 1e-9 && disc >= 0) {
                const double td = (-b + sqrt(disc)) / (2 * a);
                if (td > 0.05 && td < best) {
                    best = td;
                    kind = 3;
                }
            }
        }
    }
    for (; i < s.kept_total; ++i) {
        if (certain_miss(s, i, dxf, dyf, dzf)) continue;
        const double t = sphere_hit(s, i, d, best);
        if (t < best) {
            best = t;
            kind = 4;
        }
    }
    return best;
}

/* One sphere test of trace(): the float miss test, then the double one. */
__device__ __forceinline__ void tile_sphere(const UnitScene &s, int i, Vec d, float dxf, float dyf, float dzf,
                                            double &best, int &kind, int k) {
    if (certain_miss(s, i, dxf, dyf, dzf)) return;
    const double t = sphere_hit(s, i, d, best);
    if (t < best) {
        best = t;
        kind = k;
    }
}

/* trace() for the rays of one camera tile: the same tests in the same order,
 * over the tile's own sphere list (`index`: n_obst obstacles, then the
 * opponent when n_opp, then balls, n in all) -- the kept spheres that some
 * ray of the tile may hit.  The others are proved missed by every ray of the
 * tile, so skipping them leaves the nearest hit and its kind as they were. */
__device__ __forceinline__ double trace_tile(const UnitScene &s, Vec d, int &kind, const unsigned char *index,
                                             int n_obst, int n_opp, int n) {
    double best = s.h.best0;
    kind = -1;
    const double ox = s.h.origin[0], oy = s.h.origin[1], oz = s.h.origin[2];
    const float dxf = __double2float_rn(d.x), dyf = __double2float_rn(d.y), dzf = __double2float_rn(d.z);
    if (d.z < -1e-5) {
        const double t = (0 - oz) / d.z;
        if (t > 0.05 && t < best) {
            best = t;
            kind = 0;
        }
        if (s.h.shelf) {
            const double t2 = (9 - oz) / d.z;
            if (t2 > 0.05 && t2 < best && ox + t2 * d.x >= 20) {
                best = t2;
                kind = 0;
            }
        }
    }
    int k = 0;
    for (; k < n_obst; ++k) tile_sphere(s, index[k], d, dxf, dyf, dzf, best, kind, 1);
    if (s.h.arena) {
        if (n_opp) {
            tile_sphere(s, index[k], d, dxf, dyf, dzf, best, kind, 2);
            ++k;
        }
        if (s.h.dome) {
            const double a = d.x * d.x + d.y * d.y, b = 2 * (ox * d.x + oy * d.y);
            const double disc = b * b - 4 * a * s.h.dome_cc;
            if (a > 1e-9 && disc >= 0) {
                const double td = (-b + sqrt(disc)) / (2 * a);
                if (td > 0.05 && td < best) {
                    best = td;
                    kind = 3;
                }
            }
        }
    }
    for (; k < n; ++k) tile_sphere(s, index[k], d, dxf, dyf, dzf, best, kind, 4);
    return best;
}

/* shade()'s distance factor, sensors.c:66. */
__device__ __forceinline__ double fog(double distance) { return 0.75 + 0.25 * exp(-distance / 80); }

/* Distance from a half-integer beyond which the float-fog byte below is
 * certain (three times the error bound derived at shade). */
constexpr float kFogMargin = 3e-4f;

/* shade (sensors.c:59-68); the sky's factor comes precomputed.  A hit's
 * byte round(luma * fog(d) * 255) is first formed in float with
 * __expf: the argument -d/80 in float is within 2.3 u of -d/80 (u = 2^-24),
 * which moves exp by at most 2.3 u / e; __expf adds at most 3e-7 absolute for
 * arguments <= 0 (checked on every float argument in [-88, 0] by
 * tests/test_sensors_gpu.py); the FMA and two products add 4 u relative.
 * luma <= 1 and fog <= 1, so the float value x = luma * fog * 255 is within
 * 255 (0.25 * 3.6e-7 + 2.4e-7) < 1e-4 of the double expression, which is
 * itself within 2e-13 of the exact value; adding 0.5 rounds by at most
 * 7.6e-6.  When x + 0.5 lies more than kFogMargin from an integer, the double
 * expression rounds (half away from zero, x >= 0) to the same integer.
 * Otherwise -- about 0.06 % of pixels -- the double expression is evaluated. */
__device__ __forceinline__ uint32_t shade(const UnitScene &s, double distance, int kind, double dz) {
    double luma = 0.22 + 0.15 * fmax(-1.0, fmin(1.0, dz));
    if (kind == 0) luma = 0.28 + 0.17 * fmax(0.0, fmin(1.0, -dz));
    if (kind == 1) luma = 0.65;
    if (kind == 2) luma = 0.90;
    if (kind == 3) luma = 0.46;
    if (kind == 4) luma = 1.0;
    if (kind >= 0 && distance < 1e30) {
        const float e = __expf(__fmul_rn(-__double2float_rn(distance), 0.0125f));
        const float x = __fmul_rn(__fmul_rn(__double2float_rn(luma), __fmaf_rn(0.25f, e, 0.75f)), 255.0f);
        const float y = __fadd_rn(x, 0.5f);
        const float k = floorf(y);
        const float r = y - k;
        if (r > kFogMargin && r < 1.0f - kFogMargin) return static_cast<uint32_t>(fminf(255.0f, fmaxf(0.0f, k)));
    }
    luma *= kind < 0 ? s.h.sky_fog : fog(distance);
    return static_cast<uint32_t>(fmax(0.0, fmin(255.0, round(luma * 255))));
}

__device__ __forceinline__ unsigned long long splitmix(unsigned long long z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

/* cone_misses() below for any cone (world-frame unit axis, cos and sin of its
 * half-angle; the camera tiles use it) -- true when no ray of the cone from
 * the origin can take a sphere (centre at w from the origin, radius ra) as
 * its nearest hit: the sphere's surface lies beyond the
 * sky distance best0 (every hit t >= L - r), or every ray provably returns
 * "no hit" -- the sphere lies wholly behind the origin, or each ray's closest
 * approach to the centre exceeds the radius by 1e-6 * max(1, L).  NaN and
 * infinite inputs give false. */
__device__ __forceinline__ bool cone_misses_at(double wx, double wy, double wz, double ra, const double *axis,
                                               double cos_a, double sin_a, double best0) {
    const double l = sqrt(wx * wx + wy * wy + wz * wz);
    if (!(l < 1e7) || !(l > ra + 0.1)) return false; /* also rejects NaN */
    if (l - ra > best0 * (1 + 1e-9) + 1e-9) return true;
    const double cosc = fmin(1.0, fmax(-1.0, (wx * axis[0] + wy * axis[1] + wz * axis[2]) / l));
    const double sinc = sqrt(fmax(0.0, 1.0 - cosc * cosc));
    /* the smallest angle between a ray of the cone and the centre direction */
    const double sin_min = sinc * cos_a - cosc * sin_a;
    const double cos_min = cosc * cos_a + sinc * sin_a;
    if (cos_min < -1e-9 && sin_min > 0) return true; /* every ray points away */
    return sin_min > 0 && l * sin_min > ra + 1e-6 * fmax(1.0, l);
}

/* True when no ray of the unit's cone can take the sphere (centre c, radius
 * r) as its nearest hit from origin o: the sphere's surface lies beyond the
 * sky distance (every hit t >= L - r), or every ray provably returns "no
 * hit" -- the sphere lies wholly behind the origin, or each ray's closest
 * approach to the centre exceeds the radius by 1e-6 * max(1, L).  NaN and
 * infinite inputs give false. */
__device__ __forceinline__ bool cone_misses(const UnitHead &h, const double *cone, double cx, double cy, double cz,
                                            double r) {
    const double wx = cx - h.origin[0], wy = cy - h.origin[1], wz = cz - h.origin[2];
    const double l = sqrt(wx * wx + wy * wy + wz * wz);
    const double ra = fabs(r);
    if (!(l < 1e7) || !(l > ra + 0.1)) return false; /* also rejects NaN */
    if (l - ra > h.best0 * (1 + 1e-9) + 1e-9) return true;
    const double cosc = fmin(1.0, fmax(-1.0, (wx * h.axis[0] + wy * h.axis[1] + wz * h.axis[2]) / l));
    const double sinc = sqrt(fmax(0.0, 1.0 - cosc * cosc));
    const double cos_a = cone[3], sin_a = cone[4];
    /* the smallest angle between a ray of the cone and the centre direction */
    const double sin_min = sinc * cos_a - cosc * sin_a;
    const double cos_min = cosc * cos_a + sinc * sin_a;
    if (cos_min < -1e-9 && sin_min > 0) return true; /* every ray points away */
    return sin_min > 0 && l * sin_min > ra + 1e-6 * fmax(1.0, l);
}

/* The unit's per-origin scalars (computed by every thread that needs them,
 * so no thread waits for another; `fogged` also evaluates the sky factor). */
__device__ __forceinline__ void unit_head(UnitHead &h, const tb_sensor_scene *__restrict__ scene, int part,
                                          bool fogged) {
    const int scenario = scene->scenario;
    const bool bwb = is_bwb(scenario), arena = is_arena(scenario);
    const double qw = scene->attitude[0], qx = scene->attitude[1], qy = scene->attitude[2], qz = scene->attitude[3];
    h.q[0] = qw;
    h.q[1] = qx;
    h.q[2] = qy;
    h.q[3] = qz;
    /* Sensor mounts: LiDAR heads sensors.c:32, cameras :72. */
    Vec mount;
    if (part < 2) {
        mount = Vec{0.4, 0.4, part ? -0.4 : 0.4};
    } else {
        const int view = part - 2;
        mount = view < 2 ? Vec{0.42, 0.42, view == 0 ? 0.13 : 0.08} : Vec{0, 0, view == 2 ? -0.5 : 0.5};
    }
    const Vec r = rotate(qw, qx, qy, qz, mount);
    const double ox = scene->position[0] + r.x, oy = scene->position[1] + r.y, oz = scene->position[2] + r.z;
    h.origin[0] = ox;
    h.origin[1] = oy;
    h.origin[2] = oz;
    const Vec axis = rotate(qw, qx, qy, qz, Vec{g_cone[part][0], g_cone[part][1], g_cone[part][2]});
    h.axis[0] = axis.x;
    h.axis[1] = axis.y;
    h.axis[2] = axis.z;
    const double norm2 = qw * qw + qx * qx + qy * qy + qz * qz;
    h.cull = TB_SENSOR_CULL && fabs(norm2 - 1.0) < 1e-9;
    const double lidar_max = scene->lidar_max;
    h.best0 = bwb ? fmax(lidar_max, 120.0) : lidar_max;
    h.sky_fog = fogged ? fog(h.best0) : 0.0;
    h.max_range = bwb ? fmax(120.0, lidar_max) : lidar_max;
    const double dome = bwb ? 300.0 : scene->dome_radius;
    h.dome_cc = ox * ox + oy * oy - dome * dome;
    /* Inside the cylinder at horizontal radius rho, a dome hit needs a
     * horizontal run of at least dome - rho, so t >= dome - rho for rays of
     * unit length -- only when the attitude is a rotation (h.cull). */
    const double rho = sqrt(ox * ox + oy * oy);
    h.dome = !(h.cull && dome - rho > h.best0 * (1 + 1e-9) + 1e-9);
    h.shelf = scenario == 10;
    h.arena = arena;
    /* float camera pixels: a rotation, no shelf, no reachable dome, finite
     * geometry of modest size (tb_camera_float.h's bounds) */
    h.float_camera = h.cull && !h.shelf && !(arena && h.dome) && fabs(ox) < 1e6 && fabs(oy) < 1e6 &&
                     fabs(oz) < 1e6 && h.best0 < 1e6;
    h.n_obstacles = min(max(scene->obstacle_count, 0), TB_SENSOR_MAX_OBSTACLES);
    h.n_balls = min(max(scene->ball_count, 0), TB_SENSOR_MAX_BALLS);
    /* sensors.c:30: rng ^ step_index * golden ^ player * 257 */
    h.seed = scene->rng ^ (static_cast<unsigned long long>(static_cast<long long>(scene->step_index)) * kGolden) ^
             static_cast<unsigned long long>(static_cast<long long>(scene->player) * 257);
}

/* Forms unit `part0` of `scene` in s0 and, with `two`, unit part0 + 1 in s1:
 * the first kSphereWarps warps form a unit's scalars and sphere list, the
 * next kSphereWarps warps the second unit's, in the same two CTA barriers;
 * every thread returns after the second, with the units complete. */
__device__ __forceinline__ void prepare_units(UnitScene &s0, UnitScene &s1, const tb_sensor_scene *__restrict__ scene,
                                              int part0, bool two) {
    static_assert(2 * 32 * kSphereWarps <= kThreads, "two units' sphere warps");
    const bool second = two && threadIdx.x >= 32 * kSphereWarps; /* warp-uniform */
    UnitScene &s = second ? s1 : s0;
    const int part = part0 + (second ? 1 : 0);
    const int t = static_cast<int>(threadIdx.x) - (second ? 32 * kSphereWarps : 0);
    double ocx = 0, ocy = 0, ocz = 0, occ = 0, rr = 0;
    bool keep = false, float_test = false;
    int n_obst = 0, arena = 0;
    if (t < 32 * kSphereWarps) {
        UnitHead h;
        unit_head(h, scene, part, t == 0);
        if (t == 0) {
            s.h = h;
            s.valid_count = 0;
            s.warps_done = 0;
        }
        /* Spheres in trace order: obstacles, the arena opponent, balls. */
        n_obst = h.n_obstacles;
        arena = h.arena;
        const int n = n_obst + arena + h.n_balls;
        if (t < n) {
            double cx, cy, cz, radius;
            if (t < n_obst) {
                cx = scene->obstacles[t][0];
                cy = scene->obstacles[t][1];
                cz = scene->obstacles[t][2];
                radius = scene->obstacles[t][3];
            } else if (arena && t == n_obst) {
                cx = scene->opponent[0];
                cy = scene->opponent[1];
                cz = scene->opponent[2];
                radius = is_bwb(scene->scenario) ? 0.75 : 0.45;
            } else {
                const int j = t - n_obst - arena;
                cx = scene->balls[j][0];
                cy = scene->balls[j][1];
                cz = scene->balls[j][2];
                radius = 0.25;
            }
            ocx = h.origin[0] - cx;
            ocy = h.origin[1] - cy;
            ocz = h.origin[2] - cz;
            occ = ocx * ocx + ocy * ocy + ocz * ocz;
            rr = radius * radius;
            keep = !(h.cull && cone_misses(h, g_cone[part], cx, cy, cz, radius));
            float_test = h.cull && occ + rr < 1e30; /* unit rays, no float overflow (NaN fails) */
        }
        const unsigned int m = __ballot_sync(0xffffffffu, keep);
        const unsigned int obst = __ballot_sync(0xffffffffu, keep && t < n_obst);
        const unsigned int opp = __ballot_sync(0xffffffffu, keep && arena && t == n_obst);
        if ((t & 31) == 0) {
            s.keep_mask[t >> 5] = m;
            s.obst_mask[t >> 5] = obst;
            s.opp_mask[t >> 5] = opp;
        }
    }
    __syncthreads();
    if (t < 32 * kSphereWarps) {
        const int w = t >> 5;
        int pos = __popc(s.keep_mask[w] & ((1u << (t & 31)) - 1u));
        for (int k = 0; k < w; ++k) pos += __popc(s.keep_mask[k]);
        if (keep) {
            s.oc_xy[pos] = make_double2(ocx, ocy);
            s.oc_zq[pos] = make_double2(ocz, occ);
            s.rr[pos] = rr;
            s.f_oc[pos] = make_float4(__double2float_rn(ocx), __double2float_rn(ocy), __double2float_rn(ocz),
                                      __double2float_rn(rr - occ));
            s.f_margin[pos] = float_test ? __double2float_rn(0x1.0p-18 * (occ + rr)) : INFINITY;
            s.f_margin_ray[pos] = float_test ? __double2float_rn(TBF_SPHERE_MARGIN * (occ + rr)) : INFINITY;
        }
        if (t == 0) {
            int total = 0, kept_obst = 0, kept_opp = 0;
            for (int k = 0; k < kSphereWarps; ++k) {
                total += __popc(s.keep_mask[k]);
                kept_obst += __popc(s.obst_mask[k]);
                kept_opp += __popc(s.opp_mask[k]);
            }
            s.kept_total = total;
            s.kept_obstacles = kept_obst;
            s.kept_opponent = kept_opp;
        }
    }
    __syncthreads();
}

/* The LiDAR units (2 per scene: the heads) and the camera units (8 per
 * scene: each view's two halves) run as two kernels, so that each keeps only
 * its own code and registers (one kernel over all ten units spilled more and
 * ran 6-13 % slower with the float tests). */
constexpr int kLidarUnits = 2, kCameraUnits = 4;

/* LiDAR head `part` of scene `scene_index` (sensors.c:31-49). */
__device__ __forceinline__ void render_lidar(UnitScene &s, int part, unsigned long long scene_index, float *lidar,
                                             unsigned long long lidar_stride, float *lidar_valid,
                                             unsigned long long valid_stride) {
    const int t = threadIdx.x;
    const double qw = s.h.q[0], qx = s.h.q[1], qy = s.h.q[2], qz = s.h.q[3];
    float *out = lidar + scene_index * lidar_stride;
    const double max_range = s.h.max_range;
    /* SplitMix64 state before the draw of bin b is seed + (b + 1) * golden */
    unsigned long long state = s.h.seed + static_cast<unsigned long long>(part * kUnitRays + t + 1) * kGolden;
    int valid = 0;
#pragma unroll 1
    for (int k = 0; k < kUnitRays / kThreads; ++k, state += static_cast<unsigned long long>(kThreads) * kGolden) {
        const int bin = part * kUnitRays + k * kThreads + t;
        const unsigned long long hash = splitmix(state);
        const bool blocked = (g_lidar_blocked[bin >> 5] >> (bin & 31)) & 1u;
        float value = -1.0f;
        if (!(static_cast<double>(hash & 0xffff) / 65536.0 < 0.005 || blocked)) {
            const Vec rw = rotate(qw, qx, qy, qz, Vec{g_lidar_x[bin], g_lidar_y[bin], g_lidar_z[bin]});
            int kind;
            double range = trace(s, rw, kind);
            const double noise = (static_cast<double>((hash >> 16) & 0xffff) / 32768.0 - 1.0) * 0.02;
            range = fmax(0.05, fmin(max_range, range + noise));
            value = static_cast<float>(range);
            ++valid;
        }
        out[bin] = value;
    }
    if (lidar_valid) {
        /* the last warp to finish writes the head's valid fraction */
        valid = __reduce_add_sync(0xffffffffu, valid);
        if ((t & 31) == 0) {
            atomicAdd(&s.valid_count, valid);
            __threadfence_block();
            if (atomicAdd(&s.warps_done, 1) == kWarps - 1)
                lidar_valid[scene_index * valid_stride + part] =
                    static_cast<float>(atomicAdd(&s.valid_count, 0)) / 2048;
        }
    }
}

/* Camera view part - 2 of scene `scene_index` (sensors.c:71-79): 64 rows of 64, rendered as
 * two halves of 32 rows (one 16 x 16 tile of each per warp) after a single setup of the unit. */
__device__ __forceinline__ void render_camera(UnitScene &s, int part, unsigned long long scene_index,
                                              unsigned char *cameras, unsigned char *raw) {
    const int t = threadIdx.x;
    const double qw = s.h.q[0], qx = s.h.q[1], qy = s.h.q[2], qz = s.h.q[3];
    const bool float_unit = s.h.float_camera;
    tbf_unit fu;
    fu.qw = __double2float_rn(qw);
    fu.qx = __double2float_rn(qx);
    fu.qy = __double2float_rn(qy);
    fu.qz = __double2float_rn(qz);
    fu.oz = __double2float_rn(s.h.origin[2]);
    fu.sky_fog = __double2float_rn(s.h.sky_fog);
    fu.best0 = s.h.best0;
    fu.best0_lo = __double2float_rn(s.h.best0 * (1 - 1e-6));
    fu.best0_hi = __double2float_rn(s.h.best0 * (1 + 1e-6));
    const int view = part - 2;
    /* Each warp owns a 16 x 16 tile of the unit's 32 x 64 pixels (tile rows
     * w / 4, columns w % 4); entry e is tile row e / 16, column e % 16, and
     * lane l takes entries 4l..4l+3 and 128 + 4l..131 + 4l (four pixels of a
     * row each).  First the warp lists, in trace order, the kept spheres
     * that some ray of its tile may hit (the unit culling's cone test against
     * the tile's own cone, g_tile_cone), with their float terms copied beside
     * the list; then pass 1 decides its pixels in float; the undecided
     * ones go to a per-warp queue, which pass 2 traces in double one pixel
     * per lane (so a warp pays the double path only for its undecided pixels,
     * not whenever one lane has one); pass 3 writes the bytes four to a
     * 32-bit store. */
    __shared__ __align__(16) unsigned char warp_bytes[kWarps][256];
    __shared__ unsigned char warp_queue[kWarps][256];
    __shared__ TileSpheres warp_spheres[kWarps];
    const int warp = t >> 5, lane = t & 31;
    unsigned char *bytes = warp_bytes[warp];
    unsigned char *queue = warp_queue[warp];
    TileSpheres &ts = warp_spheres[warp];
#pragma unroll 1
    for (int half = 0; half < 2; ++half) {
    const int hu = view * 2 + half; /* the view half: index of the tile tables */
    int n = 0, n_obst = 0, n_opp = 0; /* the tile's list: all, obstacles, opponent (0 or 1) */
    const int first = tile_first(hu, warp); /* pixel of entry 0 */
    auto pixel_of = [first](int e) { return tile_pixel(first, e); };
    const int tbase = (hu * kWarps + warp) * 256; /* the tile's rays in the tile-ordered tables */
    if (s.kept_total > 0) {
        const double *cone = g_tile_cone[hu][warp];
        const Vec axis = rotate(qw, qx, qy, qz, Vec{cone[0], cone[1], cone[2]});
        const double ax[3] = {axis.x, axis.y, axis.z};
        for (int k = 0; k * 32 < s.kept_total; ++k) {
            const int i = k * 32 + lane;
            bool keep = i < s.kept_total;
            if (keep && s.h.cull) {
                const double2 xy = s.oc_xy[i], zq = s.oc_zq[i];
                keep = !cone_misses_at(-xy.x, -xy.y, -zq.x, sqrt(s.rr[i]), ax, cone[3], cone[4], s.h.best0);
            }
            const unsigned int m = __ballot_sync(0xffffffffu, keep);
            if (keep) {
                const int pos = n + __popc(m & ((1u << lane) - 1u));
                ts.f_oc[pos] = s.f_oc[i];
                ts.f_margin_ray[pos] = s.f_margin_ray[i];
                ts.index[pos] = static_cast<unsigned char>(i);
            }
            n += __popc(m);
            n_obst += __popc(__ballot_sync(0xffffffffu, keep && i < s.kept_obstacles));
            n_opp += __popc(__ballot_sync(0xffffffffu, keep && s.kept_opponent && i == s.kept_obstacles));
        }
    }
    if (lane == 0) { /* read back by pass 2 only */
        ts.n_obst = n_obst;
        ts.n_opp = n_opp;
    }
    __syncwarp();
    int queued = 0;
#pragma unroll 1
    for (int k = 0; k < 2; ++k) {
#pragma unroll 1
        for (int j = 0; j < 4; ++j) {
            const int e = k * 128 + 4 * lane + j;
            unsigned int byte = 0;
            const bool done = float_unit && tbf_camera_pixel(&fu, reinterpret_cast<const tbf_sphere *>(ts.f_oc),
                                                             ts.f_margin_ray, n, g_camera_fx[tbase + e],
                                                             g_camera_fy[tbase + e], g_camera_fz[tbase + e], &byte);
            if (done) bytes[e] = static_cast<unsigned char>(byte);
            const unsigned int pending = __ballot_sync(0xffffffffu, !done);
            if (!done) queue[queued + __popc(pending & ((1u << lane) - 1u))] = static_cast<unsigned char>(e);
            queued += __popc(pending);
        }
    }
    __syncwarp();
#pragma unroll 1
    for (int q = lane; q < queued; q += 32) {
        const int e = queue[q];
        const Vec dir =
            rotate(qw, qx, qy, qz, Vec{g_camera_x[tbase + e], g_camera_y[tbase + e], g_camera_z[tbase + e]});
        int kind;
        const double d = trace_tile(s, dir, kind, ts.index, ts.n_obst, ts.n_opp, n);
        bytes[e] = static_cast<unsigned char>(shade(s, d, kind, dir.z));
    }
    __syncwarp();
#pragma unroll 1
    for (int k = 0; k < 2; ++k) {
        const int e = k * 128 + 4 * lane;
        const int pixel = pixel_of(e);
        const int local = pixel - view * 4096; /* pixel in the view */
        const uint32_t word = *reinterpret_cast<const uint32_t *>(bytes + e);
        if (cameras)
            *reinterpret_cast<uint32_t *>(cameras + scene_index * kCameraPixels + pixel) = word;
        if (raw) {
            /* each pixel as a 3 x 3 block of the 192 x 192 view (sensors.c:78) */
            const uint32_t p0 = word & 255u, p1 = (word >> 8) & 255u, p2 = (word >> 16) & 255u,
                           p3 = word >> 24;
            const uint32_t w0 = p0 | p0 << 8 | p0 << 16 | p1 << 24;
            const uint32_t w1 = p1 | p1 << 8 | p2 << 16 | p2 << 24;
            const uint32_t w2 = p2 | p3 << 8 | p3 << 16 | p3 << 24;
            const int y = local >> 6, x = local & 63;
            unsigned char *base = raw + scene_index * static_cast<unsigned long long>(TB_SENSOR_CAMERA_RAW_PIXELS) +
                                  view * 36864 + 3 * x;
#pragma unroll
            for (int dy = 0; dy < 3; ++dy) {
                uint32_t *row = reinterpret_cast<uint32_t *>(base + (3 * y + dy) * 192);
                row[0] = w0;
                row[1] = w1;
                row[2] = w2;
            }
        }
    }
    __syncwarp(); /* the buffers are refilled by the next half or unit */
    }
}

template <bool kLidar>
__global__ void __launch_bounds__(kThreads, TB_SENSOR_MIN_BLOCKS)
    sensors_kernel(const tb_sensor_scene *__restrict__ scenes, unsigned long long units, float *__restrict__ lidar,
                   unsigned long long lidar_stride, float *__restrict__ lidar_valid, unsigned long long valid_stride,
                   unsigned char *__restrict__ cameras, unsigned char *__restrict__ raw) {
    /* Two slots, alternating over the units this CTA renders: a slot is
     * rewritten only after both barriers of the unit in between, which every
     * thread passes after it finished tracing from that slot. */
    __shared__ UnitScene slots[kLidar ? 4 : 2];
    /* LiDAR: one unit per scene, both heads formed in one setup (their own
     * origins, so two sphere lists) and rendered in turn */
    constexpr int kPerScene = kLidar ? 1 : kCameraUnits;
    int used = 0;
    for (unsigned long long unit = blockIdx.x; unit < units; unit += gridDim.x) {
        const unsigned long long scene_index = unit / kPerScene;
        const int part = kLidar ? 0 : static_cast<int>(unit - scene_index * kPerScene) + kLidarUnits;
        const tb_sensor_scene *scene = scenes + scene_index;
        /* the same word for every thread: a CTA-uniform skip */
        if (!(scene->sensors & (kLidar ? TB_SENSOR_LIDAR : TB_SENSOR_CAMERA))) continue;
        if constexpr (kLidar) {
            UnitScene &s0 = slots[(used & 1) * 2], &s1 = slots[(used & 1) * 2 + 1];
            ++used;
            prepare_units(s0, s1, scene, 0, true);
            render_lidar(s0, 0, scene_index, lidar, lidar_stride, lidar_valid, valid_stride);
            render_lidar(s1, 1, scene_index, lidar, lidar_stride, lidar_valid, valid_stride);
        } else {
            UnitScene &s = slots[used & 1];
            ++used;
            prepare_units(s, s, scene, part, false);
            render_camera(s, part, scene_index, cameras, raw);
        }
    }
}

constexpr int kMaxDevices = 64;
bool g_tables_ready[kMaxDevices];
int g_grid_cap[kMaxDevices];
std::mutex g_tables_mutex;


/* Cone of unit `part` over body-frame rays dirs[first .. first+count) (rays
 * with skip[i] set are never traced): unit axis, then cos and sin of the
 * largest angle to any ray widened by 1e-6 rad. */
void unit_cone(const double *x, const double *y, const double *z, int first, int count, const unsigned char *skip,
               double *cone) {
    double ax = 0, ay = 0, az = 0;
    for (int i = first; i < first + count; ++i)
        if (!skip || !skip[i]) {
            ax += x[i];
            ay += y[i];
            az += z[i];
        }
    const double n = sqrt(ax * ax + ay * ay + az * az);
    ax /= n;
    ay /= n;
    az /= n;
    double widest = 0;
    for (int i = first; i < first + count; ++i) {
        if (skip && skip[i]) continue;
        const double len = sqrt(x[i] * x[i] + y[i] * y[i] + z[i] * z[i]);
        const double c = fmin(1.0, fmax(-1.0, (x[i] * ax + y[i] * ay + z[i] * az) / len));
        widest = fmax(widest, acos(c));
    }
    widest += 1e-6;
    cone[0] = ax;
    cone[1] = ay;
    cone[2] = az;
    cone[3] = cos(widest);
    cone[4] = sin(widest);
}

/* Cone of camera tile `warp` of view half `unit` (view unit / 2, half
 * unit % 2): its 16 x 16 pixels, as the camera kernel assigns them. */
void tile_cone(const double *x, const double *y, const double *z, int unit, int warp, double *cone) {
    static double tx[256], ty[256], tz[256];
    const int first = tile_first(unit, warp);
    for (int e = 0; e < 256; ++e) {
        const int pixel = tile_pixel(first, e);
        tx[e] = x[pixel];
        ty[e] = y[pixel];
        tz[e] = z[pixel];
    }
    unit_cone(tx, ty, tz, 0, 256, nullptr, cone);
}

/* Uploads the body-frame ray tables and unit cones to the current device (once). */
bool ensure_tables(int dev) {
    std::lock_guard<std::mutex> lock(g_tables_mutex);
    if (g_tables_ready[dev]) return true;
    static double lidar_dirs[3 * kLidarBins], camera_dirs[3 * kCameraPixels];
    static unsigned char blocked[kLidarBins];
    static bool built = false;
    static double lx[kLidarBins], ly[kLidarBins], lz[kLidarBins];
    static double cx[kCameraPixels], cy[kCameraPixels], cz[kCameraPixels];
    static float cfx[kCameraPixels], cfy[kCameraPixels], cfz[kCameraPixels];
    static unsigned int mask[kLidarBins / 32];
    static double cones[kUnitsPerScene][5];
    static double tile_cones[kCameraHalves][kWarps][5];
    if (!built) {
        tb_sensor_lidar_rays(lidar_dirs, blocked);
        tb_sensor_camera_rays(camera_dirs);
        for (int i = 0; i < kLidarBins; ++i) {
            lx[i] = lidar_dirs[3 * i];
            ly[i] = lidar_dirs[3 * i + 1];
            lz[i] = lidar_dirs[3 * i + 2];
            if (blocked[i]) mask[i >> 5] |= 1u << (i & 31);
        }
        for (int i = 0; i < kCameraPixels; ++i) {
            cx[i] = camera_dirs[3 * i];
            cy[i] = camera_dirs[3 * i + 1];
            cz[i] = camera_dirs[3 * i + 2];
            cfx[i] = static_cast<float>(cx[i]);
            cfy[i] = static_cast<float>(cy[i]);
            cfz[i] = static_cast<float>(cz[i]);
        }
        for (int h = 0; h < 2; ++h) unit_cone(lx, ly, lz, h * kUnitRays, kUnitRays, blocked, cones[h]);
        for (int p = 2; p < kUnitsPerScene; ++p) unit_cone(cx, cy, cz, (p - 2) * 4096, 4096, nullptr, cones[p]);
        for (int u = 0; u < kCameraHalves; ++u)
            for (int w = 0; w < kWarps; ++w) tile_cone(cx, cy, cz, u, w, tile_cones[u][w]);
        /* the camera tables in tile order */
        static double px[kCameraPixels], py[kCameraPixels], pz[kCameraPixels];
        for (int i = 0; i < kCameraPixels; ++i) {
            px[i] = cx[i];
            py[i] = cy[i];
            pz[i] = cz[i];
        }
        for (int u = 0; u < kCameraHalves; ++u)
            for (int w = 0; w < kWarps; ++w)
                for (int e = 0; e < 256; ++e) {
                    const int k = (u * kWarps + w) * 256 + e, pixel = tile_pixel(tile_first(u, w), e);
                    cx[k] = px[pixel];
                    cy[k] = py[pixel];
                    cz[k] = pz[pixel];
                    cfx[k] = static_cast<float>(px[pixel]);
                    cfy[k] = static_cast<float>(py[pixel]);
                    cfz[k] = static_cast<float>(pz[pixel]);
                }
        built = true;
    }
    int sms = 0, blocks = 0;
    if (cudaMemcpyToSymbol(g_lidar_x, lx, sizeof lx) != cudaSuccess ||
        cudaMemcpyToSymbol(g_lidar_y, ly, sizeof ly) != cudaSuccess ||
        cudaMemcpyToSymbol(g_lidar_z, lz, sizeof lz) != cudaSuccess ||
        cudaMemcpyToSymbol(g_lidar_blocked, mask, sizeof mask) != cudaSuccess ||
        cudaMemcpyToSymbol(g_camera_x, cx, sizeof cx) != cudaSuccess ||
        cudaMemcpyToSymbol(g_camera_y, cy, sizeof cy) != cudaSuccess ||
        cudaMemcpyToSymbol(g_camera_z, cz, sizeof cz) != cudaSuccess ||
        cudaMemcpyToSymbol(g_camera_fx, cfx, sizeof cfx) != cudaSuccess ||
        cudaMemcpyToSymbol(g_camera_fy, cfy, sizeof cfy) != cudaSuccess ||
        cudaMemcpyToSymbol(g_camera_fz, cfz, sizeof cfz) != cudaSuccess ||
        cudaMemcpyToSymbol(g_cone, cones, sizeof cones) != cudaSuccess ||
        cudaMemcpyToSymbol(g_tile_cone, tile_cones, sizeof tile_cones) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, sensors_kernel<false>, kThreads, 0) != cudaSuccess)
        return false;
    /* enough CTAs for many waves; each strides over the units */
    g_grid_cap[dev] = sms * (blocks > 0 ? blocks : 1) * 64;
    g_tables_ready[dev] = true;
    return true;
}

bool aligned(const void *p, uintptr_t n) { return (reinterpret_cast<uintptr_t>(p) & (n - 1)) == 0; }

} /* namespace */

extern "C" int tb_cuda_render_sensors_device(const tb_sensor_scene *device_scenes, size_t count, float *device_lidar,
                                             size_t lidar_stride, float *device_lidar_valid, size_t valid_stride,
                                             unsigned char *device_cameras, unsigned char *device_raw_cameras,
                                             void *stream) {
    if (!device_scenes || count == 0 || count > 0x7fffffffu || !aligned(device_scenes, 8)) return 0;
    if (device_lidar && (!aligned(device_lidar, 4) || lidar_stride < static_cast<size_t>(kLidarBins))) return 0;
    if (device_lidar_valid && (!aligned(device_lidar_valid, 4) || valid_stride < 2)) return 0;
    if ((device_cameras && !aligned(device_cameras, 4)) || (device_raw_cameras && !aligned(device_raw_cameras, 4)))
        return 0;
    if (!device_lidar) device_lidar_valid = nullptr;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 0;
    if (!ensure_tables(dev)) return 0;
    cudaGetLastError(); /* report this launch only */
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const unsigned long long cap = static_cast<unsigned long long>(g_grid_cap[dev]);
    if (device_lidar) {
        const unsigned long long units = static_cast<unsigned long long>(count); /* both heads per unit */
        sensors_kernel<true><<<static_cast<unsigned int>(units < cap ? units : cap), kThreads, 0, s>>>(
            device_scenes, units, device_lidar, lidar_stride, device_lidar_valid, valid_stride, nullptr, nullptr);
    }
    if (device_cameras || device_raw_cameras) {
        const unsigned long long units = static_cast<unsigned long long>(count) * kCameraUnits;
        sensors_kernel<false><<<static_cast<unsigned int>(units < cap ? units : cap), kThreads, 0, s>>>(
            device_scenes, units, nullptr, 0, nullptr, 0, device_cameras, device_raw_cameras);
    }
    return cudaGetLastError() == cudaSuccess;
}
