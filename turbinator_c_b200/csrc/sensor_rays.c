/*
 * Body-frame ray directions of the simulator's sensors, evaluated once on the
 * host.  They depend only on the bin or pixel, never on the scene, so the GPU
 * renderer rotates these tables into the world frame instead of evaluating
 * sin, cos, tan, hypot and atan2 per ray.  They are computed here with the
 * host C library -- the same functions the simulator calls -- in the
 * simulator's expression order and without contraction (-std=c11 keeps
 * -ffp-contract=off), so every direction equals the simulator's bit for bit:
 *   LiDAR   reference src/sim/sensors.c:35-40 (elevation 90*el/15 degrees,
 *           up for head 0 and down for head 1; azimuth 45 + 360*az/128
 *           degrees; the airframe blocks rays with x < -0.15, |y|, |z| < 0.28)
 *   cameras sensors.c:52-58 (camera_ray: view 0 a 45-degree pinhole looking
 *           forward-left and down, view 1 a 140-degree fisheye on the same
 *           axis, views 2 and 3 140-degree fisheyes looking down and up) with
 *           pixel centres u, v = (x + 0.5 - 32)/32, sensors.c:75.
 */
#include <math.h>

#include "tb_sensor_rays.h"

#define RAY_PI 3.14159265358979323846

typedef struct {
    double x, y, z;
} vec3;

static vec3 v3(double x, double y, double z) {
    vec3 a = {x, y, z};
    return a;
}
static vec3 v3_add(vec3 a, vec3 b) { return v3(a.x + b.x, a.y + b.y, a.z + b.z); }
static vec3 v3_scale(vec3 a, double s) { return v3(a.x * s, a.y * s, a.z * s); }
/* Unit vector as the simulator forms it: multiply by 1/|a| (sim_internal.h:81). */
static vec3 v3_unit(vec3 a) {
    const double n = sqrt(a.x * a.x + a.y * a.y + a.z * a.z);
    return n > 1e-12 ? v3_scale(a, 1 / n) : v3(0, 0, 1);
}

void tb_sensor_lidar_rays(double *dirs, unsigned char *occluded) {
    for (int head = 0; head < 2; ++head) {
        const double sign = head ? -1 : 1;
        for (int el = 0; el < 16; ++el) {
            const double elevation = (sign * 90.0 * el / 15.0) * RAY_PI / 180.0;
            const double ce = cos(elevation), se = sin(elevation);
            for (int az = 0; az < 128; ++az) {
                const int bin = head * 2048 + el * 128 + az;
                const double azimuth = (45.0 + 360.0 * az / 128.0) * RAY_PI / 180.0;
                const vec3 d = v3(ce * cos(azimuth), ce * sin(azimuth), se);
                dirs[3 * bin] = d.x;
                dirs[3 * bin + 1] = d.y;
                dirs[3 * bin + 2] = d.z;
                occluded[bin] = d.x < -0.15 && fabs(d.z) < 0.28 && fabs(d.y) < 0.28;
            }
        }
    }
}

static vec3 camera_direction(int view, double u, double v) {
    const vec3 forward = v3_unit(v3(1, 1, 0)), right = v3_unit(v3(1, -1, 0));
    if (view == 0) {
        const double half = tan(45.0 * RAY_PI / 360.0);
        return v3_unit(v3_add(forward, v3_add(v3_scale(right, u * half), v3(0, 0, -v * half))));
    }
    const double radius = hypot(u, v);
    const double clamped = fmax(0, fmin(1.4, radius));
    const double theta = clamped * 140.0 * RAY_PI / 360.0;
    if (view == 1) {
        if (radius < 1e-12) return forward;
        const vec3 tangent = v3_add(v3_scale(right, u / radius), v3(0, 0, -v / radius));
        return v3_unit(v3_add(v3_scale(forward, cos(theta)), v3_scale(tangent, sin(theta))));
    }
    const double phi = atan2(v, u);
    return v3_unit(v3(sin(theta) * cos(phi), -sin(theta) * sin(phi), view == 3 ? cos(theta) : -cos(theta)));
}

void tb_sensor_camera_rays(double *dirs) {
    for (int view = 0; view < 4; ++view)
        for (int y = 0; y < 64; ++y)
            for (int x = 0; x < 64; ++x) {
                const double u = (x + 0.5 - 32) / 32, v = (y + 0.5 - 32) / 32;
                const vec3 d = camera_direction(view, u, v);
                const int pixel = view * 4096 + y * 64 + x;
                dirs[3 * pixel] = d.x;
                dirs[3 * pixel + 1] = d.y;
                dirs[3 * pixel + 2] = d.z;
            }
}
