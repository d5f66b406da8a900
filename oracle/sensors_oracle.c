/*
 * TEST INFRASTRUCTURE ONLY -- CPU restatement of the simulator's sensor
 * renderers, the checker for tb_cuda_render_sensors_device.  Never linked
 * into or called by the product.
 *
 * Follows Viatreen/Turbinator_C src/sim/sensors.c:
 *   ray/sphere distance  :4-10   nearest root beyond 0.05 m, else the far root
 *   scene trace          :11-26  ground z=0, scenario 10's shelf (z=9, x>=20),
 *                                obstacles, arena opponent (r 0.45, 0.75 for
 *                                the blended-wing scenarios 22-27), arena dome
 *                                (300 m for those, else dome_radius), balls
 *                                (r 0.25); the sky sits at lidar_max (at least
 *                                120 m for the blended-wing scenarios)
 *   LiDAR                :28-50  per head 16 x 128 rays; one SplitMix64 draw
 *                                per ray; dropout at (h & 0xffff)/65536 < 0.005
 *                                or where the airframe blocks the ray; range
 *                                noise ((h>>16 & 0xffff)/32768 - 1) * 0.02
 *   camera rays          :52-58  pinhole (45 deg) and fisheye (140 deg) views
 *   shading              :59-68  luma by surface kind, fogged by exp(-d/80)
 *   camera               :69-82  4 views of 64 x 64, raw capture 3 x 3 blocks
 * with the arithmetic in the simulator's order (built with
 * -ffp-contract=off), the quaternion rotation of sim_internal.h:85 and
 * SplitMix64 of physics.c:73-78.  Pinned bit for bit against the
 * reference's own renderers (oracle/ref_sensors_shim.c) by the CPU tests.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#include "turbinator/sim/cuda_sensors.h"

#define ORACLE_PI 3.14159265358979323846

typedef struct {
    double x, y, z;
} ovec;

static ovec ov(double x, double y, double z) {
    ovec r = {x, y, z};
    return r;
}
static double odot(ovec a, ovec b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
static ovec ocross(ovec a, ovec b) { return ov(a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x); }
static ovec oadd(ovec a, ovec b) { return ov(a.x + b.x, a.y + b.y, a.z + b.z); }
static ovec omul(ovec a, double s) { return ov(a.x * s, a.y * s, a.z * s); }
static ovec onormalise(ovec a) {
    double n = sqrt(odot(a, a));
    return n > 1e-12 ? omul(a, 1 / n) : ov(0, 0, 1);
}
static double oclamp(double v, double lo, double hi) { return fmax(lo, fmin(hi, v)); }

/* Rotate v by the unit quaternion q = (w, x, y, z). */
static ovec oturn(const double q[4], ovec v) {
    ovec axis = ov(q[1], q[2], q[3]);
    ovec twice = omul(ocross(axis, v), 2);
    return oadd(oadd(v, omul(twice, q[0])), ocross(axis, twice));
}

static uint64_t osplitmix_next(uint64_t *state) {
    uint64_t z = (*state += UINT64_C(0x9e3779b97f4a7c15));
    z = (z ^ (z >> 30)) * UINT64_C(0xbf58476d1ce4e5b9);
    z = (z ^ (z >> 27)) * UINT64_C(0x94d049bb133111eb);
    return z ^ (z >> 31);
}

static int obwb(int scenario) { return scenario >= 22 && scenario <= 27; }
static int oarena(int scenario) {
    switch (scenario) {
    case 3: case 14: case 15: case 16: case 18: case 22: case 24: case 27: return 1;
    default: return 0;
    }
}

/* Built with ORACLE_SQRT_SKIP (only into oracle/liboracle_skip.so, a test
 * build), a sphere is dropped without the square root under the condition
 * the product kernel uses (sphere_hit in sensors_kernel.cu): L = -along - best
 * > 1e-6 (|along| + best) and L*L > disc (1 + 1e-9).  The test renders scenes
 * with both builds and requires identical bits, i.e. that the condition only
 * fires where this function's result could not have been nearer than best;
 * oracle_sqrt_skips() counts the drops so the test can see that it fires.
 * The default build is the simulator's arithmetic unchanged. */
#ifdef ORACLE_SQRT_SKIP
static uint64_t g_sqrt_skips;
uint64_t oracle_sqrt_skips(void) { return g_sqrt_skips; }
#endif

static double osphere(ovec origin, ovec dir, ovec centre, double radius, double best) {
    ovec rel = ov(origin.x - centre.x, origin.y - centre.y, origin.z - centre.z);
    double along = odot(rel, dir);
    double disc = along * along - odot(rel, rel) + radius * radius;
    if (disc < 0) return INFINITY;
#ifdef ORACLE_SQRT_SKIP
    double lead = -along - best;
    if (lead > 1e-6 * (fabs(along) + best) && lead * lead > disc * (1 + 1e-9)) {
        ++g_sqrt_skips;
        return INFINITY;
    }
#else
    (void)best;
#endif
    double root = sqrt(disc);
    double t = -along - root;
    if (t <= 0.05) t = -along + root;
    return t > 0.05 ? t : INFINITY;
}

static int oclamp_count(int n, int max) { return n < 0 ? 0 : (n > max ? max : n); }

/* Nearest surface along dir; *kind: -1 sky, 0 ground, 1 obstacle, 2 opponent,
 * 3 dome, 4 ball. */
static double ocast(const tb_sensor_scene *s, ovec o, ovec d, int *kind) {
    const int bwb = obwb(s->scenario);
    double nearest = bwb ? fmax(s->lidar_max, 120) : s->lidar_max;
    *kind = -1;
    if (d.z < -1e-5) {
        double t = (0 - o.z) / d.z;
        if (t > 0.05 && t < nearest) { nearest = t; *kind = 0; }
    }
    if (s->scenario == 10 && d.z < -1e-5) {
        double t = (9 - o.z) / d.z;
        if (t > 0.05 && t < nearest && o.x + t * d.x >= 20) { nearest = t; *kind = 0; }
    }
    const int obstacles = oclamp_count(s->obstacle_count, TB_SENSOR_MAX_OBSTACLES);
    for (int i = 0; i < obstacles; i++) {
        const double *ob = s->obstacles[i];
        double t = osphere(o, d, ov(ob[0], ob[1], ob[2]), ob[3], nearest);
        if (t < nearest) { nearest = t; *kind = 1; }
    }
    if (oarena(s->scenario)) {
        double t = osphere(o, d, ov(s->opponent[0], s->opponent[1], s->opponent[2]), bwb ? 0.75 : 0.45, nearest);
        if (t < nearest) { nearest = t; *kind = 2; }
        double dome = bwb ? 300 : s->dome_radius;
        double qa = d.x * d.x + d.y * d.y, qb = 2 * (o.x * d.x + o.y * d.y);
        double qc = o.x * o.x + o.y * o.y - dome * dome;
        double disc = qb * qb - 4 * qa * qc;
        if (qa > 1e-9 && disc >= 0) {
            t = (-qb + sqrt(disc)) / (2 * qa);
            if (t > 0.05 && t < nearest) { nearest = t; *kind = 3; }
        }
    }
    const int balls = oclamp_count(s->ball_count, TB_SENSOR_MAX_BALLS);
    for (int i = 0; i < balls; i++) {
        double t = osphere(o, d, ov(s->balls[i][0], s->balls[i][1], s->balls[i][2]), 0.25, nearest);
        if (t < nearest) { nearest = t; *kind = 4; }
    }
    return nearest;
}

static ovec oorigin(const tb_sensor_scene *s, ovec mount) {
    return oadd(ov(s->position[0], s->position[1], s->position[2]), oturn(s->attitude, mount));
}

void oracle_render_lidar(const tb_sensor_scene *s, float *ranges, float *valid_fraction) {
    const double max_range = obwb(s->scenario) ? fmax(120, s->lidar_max) : s->lidar_max;
    uint64_t state = s->rng ^ (uint64_t)(s->step_index * UINT64_C(0x9e3779b97f4a7c15)) ^ (uint64_t)(s->player * 257);
    for (int head = 0; head < 2; head++) {
        ovec o = oorigin(s, ov(0.4, 0.4, head ? -0.4 : 0.4));
        int hits = 0;
        for (int row = 0; row < 16; row++) {
            double el = ((head ? -1 : 1) * 90.0 * row / 15.0) * ORACLE_PI / 180.0;
            double cel = cos(el), sel = sin(el);
            for (int col = 0; col < 128; col++) {
                int bin = head * 2048 + row * 128 + col;
                double az = (45.0 + 360.0 * col / 128.0) * ORACLE_PI / 180.0;
                ovec body = ov(cel * cos(az), cel * sin(az), sel);
                uint64_t h = osplitmix_next(&state);
                int blocked = body.x < -0.15 && fabs(body.z) < 0.28 && fabs(body.y) < 0.28;
                if ((double)(h & 0xffff) / 65536.0 < 0.005 || blocked) {
                    ranges[bin] = -1;
                    continue;
                }
                int kind;
                double r = ocast(s, o, oturn(s->attitude, body), &kind);
                double noise = ((double)((h >> 16) & 0xffff) / 32768.0 - 1.0) * 0.02;
                ranges[bin] = (float)oclamp(r + noise, 0.05, max_range);
                hits++;
            }
        }
        if (valid_fraction) valid_fraction[head] = (float)hits / 2048;
    }
}

static ovec oview_ray(int view, double u, double v) {
    ovec fwd = onormalise(ov(1, 1, 0)), side = onormalise(ov(1, -1, 0));
    if (view == 0) {
        double k = tan(45.0 * ORACLE_PI / 360.0);
        return onormalise(oadd(fwd, oadd(omul(side, u * k), ov(0, 0, -v * k))));
    }
    double rad = hypot(u, v), theta = oclamp(rad, 0, 1.4) * 140.0 * ORACLE_PI / 360.0;
    if (view == 1) {
        if (rad < 1e-12) return fwd;
        ovec tangent = oadd(omul(side, u / rad), ov(0, 0, -v / rad));
        return onormalise(oadd(omul(fwd, cos(theta)), omul(tangent, sin(theta))));
    }
    double phi = atan2(v, u);
    return onormalise(ov(sin(theta) * cos(phi), -sin(theta) * sin(phi), view == 3 ? cos(theta) : -cos(theta)));
}

static uint8_t oshade(double d, int kind, ovec dir) {
    static const double surface[5] = {0, 0.65, 0.90, 0.46, 1.0};
    double luma;
    if (kind == 0) luma = 0.28 + 0.17 * oclamp(-dir.z, 0, 1);
    else if (kind >= 1 && kind <= 4) luma = surface[kind];
    else luma = 0.22 + 0.15 * oclamp(dir.z, -1, 1);
    luma *= 0.75 + 0.25 * exp(-d / 80);
    return (uint8_t)oclamp(round(luma * 255), 0, 255);
}

#ifdef ORACLE_FLOAT_CAMERA
/* Built with ORACLE_FLOAT_CAMERA (only into oracle/liboracle_float.so, a test
 * build): each camera pixel is first offered to the product kernel's float
 * decision (turbinator_c_b200/csrc/tb_camera_float.h), with the same per-view
 * eligibility (a rotation, no shelf, no reachable dome, bounded geometry)
 * and every sphere of the scene in its list; only pixels it declines are
 * traced in double.  The test renders must equal the unmodified
 * restatement's bit for bit.  oracle_float_pixels() counts the pixels the
 * float decision took. */
#include "../turbinator_c_b200/csrc/tb_camera_float.h"
static uint64_t g_float_pixels;
uint64_t oracle_float_pixels(void) { return g_float_pixels; }

static int ofloat_view(const tb_sensor_scene *s, ovec o, tbf_unit *u, tbf_sphere *sp, float *margin, int *n) {
    const double *q = s->attitude;
    const int bwb = obwb(s->scenario), arena = oarena(s->scenario);
    const double best0 = bwb ? fmax(s->lidar_max, 120) : s->lidar_max;
    const double norm2 = q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3];
    if (!(fabs(norm2 - 1.0) < 1e-9) || s->scenario == 10) return 0;
    if (!(fabs(o.x) < 1e6 && fabs(o.y) < 1e6 && fabs(o.z) < 1e6 && best0 < 1e6)) return 0;
    if (arena) {
        const double dome = bwb ? 300.0 : s->dome_radius;
        const double rho = sqrt(o.x * o.x + o.y * o.y);
        if (!(dome - rho > best0 * (1 + 1e-9) + 1e-9)) return 0;
    }
    u->qw = (float)q[0]; u->qx = (float)q[1]; u->qy = (float)q[2]; u->qz = (float)q[3];
    u->oz = (float)o.z;
    u->sky_fog = (float)(0.75 + 0.25 * exp(-best0 / 80));
    u->best0 = best0;
    u->best0_lo = (float)(best0 * (1 - 1e-6));
    u->best0_hi = (float)(best0 * (1 + 1e-6));
    int k = 0;
    const int obstacles = oclamp_count(s->obstacle_count, TB_SENSOR_MAX_OBSTACLES);
    const int balls = oclamp_count(s->ball_count, TB_SENSOR_MAX_BALLS);
    double c[TB_SENSOR_MAX_OBSTACLES + 1 + TB_SENSOR_MAX_BALLS][4];
    for (int i = 0; i < obstacles; i++, k++) {
        c[k][0] = s->obstacles[i][0]; c[k][1] = s->obstacles[i][1]; c[k][2] = s->obstacles[i][2];
        c[k][3] = s->obstacles[i][3];
    }
    if (arena) {
        c[k][0] = s->opponent[0]; c[k][1] = s->opponent[1]; c[k][2] = s->opponent[2]; c[k][3] = bwb ? 0.75 : 0.45;
        k++;
    }
    for (int i = 0; i < balls; i++, k++) {
        c[k][0] = s->balls[i][0]; c[k][1] = s->balls[i][1]; c[k][2] = s->balls[i][2]; c[k][3] = 0.25;
    }
    for (int i = 0; i < k; i++) {
        const double ocx = o.x - c[i][0], ocy = o.y - c[i][1], ocz = o.z - c[i][2];
        const double occ = ocx * ocx + ocy * ocy + ocz * ocz, rr = c[i][3] * c[i][3];
        sp[i].x = (float)ocx; sp[i].y = (float)ocy; sp[i].z = (float)ocz; sp[i].w = (float)(rr - occ);
        margin[i] = occ + rr < 1e30 ? (float)(TBF_SPHERE_MARGIN * (occ + rr)) : INFINITY;
    }
    *n = k;
    return 1;
}
#endif

void oracle_render_camera(const tb_sensor_scene *s, uint8_t *pixels, uint8_t *raw) {
    for (int view = 0; view < 4; view++) {
        ovec mount = view < 2 ? ov(0.42, 0.42, view == 0 ? 0.13 : 0.08) : ov(0, 0, view == 2 ? -0.5 : 0.5);
        ovec o = oorigin(s, mount);
#ifdef ORACLE_FLOAT_CAMERA
        tbf_unit fu = {0};
        tbf_sphere fsp[TB_SENSOR_MAX_OBSTACLES + 1 + TB_SENSOR_MAX_BALLS];
        float fmargin[TB_SENSOR_MAX_OBSTACLES + 1 + TB_SENSOR_MAX_BALLS];
        int fn = 0;
        const int float_view = ofloat_view(s, o, &fu, fsp, fmargin, &fn);
#endif
        for (int y = 0; y < 64; y++)
            for (int x = 0; x < 64; x++) {
                ovec body = oview_ray(view, (x + 0.5 - 32) / 32, (y + 0.5 - 32) / 32);
#ifdef ORACLE_FLOAT_CAMERA
                unsigned int fb;
                if (float_view && tbf_camera_pixel(&fu, fsp, fmargin, fn, (float)body.x, (float)body.y, (float)body.z,
                                                   &fb)) {
                    ++g_float_pixels;
                    if (pixels) pixels[view * 4096 + y * 64 + x] = (uint8_t)fb;
                    if (raw)
                        for (int dy = 0; dy < 3; dy++) memset(raw + view * 36864 + (3 * y + dy) * 192 + 3 * x, (int)fb, 3);
                    continue;
                }
#endif
                ovec dir = oturn(s->attitude, body);
                int kind;
                double d = ocast(s, o, dir, &kind);
                uint8_t px = oshade(d, kind, dir);
                if (pixels) pixels[view * 4096 + y * 64 + x] = px;
                if (raw)
                    for (int dy = 0; dy < 3; dy++) memset(raw + view * 36864 + (3 * y + dy) * 192 + 3 * x, px, 3);
            }
    }
}

/* Batch driver following tb_cuda_render_sensors_device's output contract. */
void oracle_render_sensors(const tb_sensor_scene *scenes, int64_t count, float *lidar, int64_t lidar_stride,
                           float *valid, int64_t valid_stride, uint8_t *cameras, uint8_t *raw) {
    for (int64_t i = 0; i < count; i++) {
        const tb_sensor_scene *s = scenes + i;
        if (lidar && (s->sensors & TB_SENSOR_LIDAR))
            oracle_render_lidar(s, lidar + i * lidar_stride, valid ? valid + i * valid_stride : NULL);
        if ((cameras || raw) && (s->sensors & TB_SENSOR_CAMERA))
            oracle_render_camera(s, cameras ? cameras + i * TB_SENSOR_CAMERA_PIXELS : NULL,
                                 raw ? raw + i * (int64_t)TB_SENSOR_CAMERA_RAW_PIXELS : NULL);
    }
}

/* Byte offsets of tb_sensor_scene's fields, for the Python record layout. */
void oracle_sensor_scene_layout(int64_t *out) {
    out[0] = (int64_t)sizeof(tb_sensor_scene);
    out[1] = (int64_t)offsetof(tb_sensor_scene, position);
    out[2] = (int64_t)offsetof(tb_sensor_scene, attitude);
    out[3] = (int64_t)offsetof(tb_sensor_scene, opponent);
    out[4] = (int64_t)offsetof(tb_sensor_scene, lidar_max);
    out[5] = (int64_t)offsetof(tb_sensor_scene, dome_radius);
    out[6] = (int64_t)offsetof(tb_sensor_scene, rng);
    out[7] = (int64_t)offsetof(tb_sensor_scene, step_index);
    out[8] = (int64_t)offsetof(tb_sensor_scene, player);
    out[9] = (int64_t)offsetof(tb_sensor_scene, scenario);
    out[10] = (int64_t)offsetof(tb_sensor_scene, sensors);
    out[11] = (int64_t)offsetof(tb_sensor_scene, obstacle_count);
    out[12] = (int64_t)offsetof(tb_sensor_scene, ball_count);
    out[13] = (int64_t)offsetof(tb_sensor_scene, obstacles);
    out[14] = (int64_t)offsetof(tb_sensor_scene, balls);
}

/* The oracle's body-frame directions (same expressions as the renderers
 * above), to check the product's host-built ray tables against. */
void oracle_sensor_rays(double *lidar_dirs, uint8_t *blocked, double *camera_dirs) {
    for (int head = 0; head < 2; head++)
        for (int row = 0; row < 16; row++) {
            double el = ((head ? -1 : 1) * 90.0 * row / 15.0) * ORACLE_PI / 180.0;
            double cel = cos(el), sel = sin(el);
            for (int col = 0; col < 128; col++) {
                int bin = head * 2048 + row * 128 + col;
                double az = (45.0 + 360.0 * col / 128.0) * ORACLE_PI / 180.0;
                ovec body = ov(cel * cos(az), cel * sin(az), sel);
                lidar_dirs[3 * bin] = body.x;
                lidar_dirs[3 * bin + 1] = body.y;
                lidar_dirs[3 * bin + 2] = body.z;
                blocked[bin] = body.x < -0.15 && fabs(body.z) < 0.28 && fabs(body.y) < 0.28;
            }
        }
    for (int view = 0; view < 4; view++)
        for (int y = 0; y < 64; y++)
            for (int x = 0; x < 64; x++) {
                ovec d = oview_ray(view, (x + 0.5 - 32) / 32, (y + 0.5 - 32) / 32);
                int p = view * 4096 + y * 64 + x;
                camera_dirs[3 * p] = d.x;
                camera_dirs[3 * p + 1] = d.y;
                camera_dirs[3 * p + 2] = d.z;
            }
}
