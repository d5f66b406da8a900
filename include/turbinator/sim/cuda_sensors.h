/*
 * Simulator sensor rendering on NVIDIA B200 (sm_100a): the ray-traced LiDAR
 * and the four 64x64 cameras of one aircraft, for a whole batch of scenes in
 * one launch.
 *
 * Replaces the reference simulator's per-environment CPU renderers
 * (Viatreen/Turbinator_C src/sim/sensors.c):
 *   tb_sim_render_lidar   sensors.c:28-50  (declared sim_internal.h:101)
 *   tb_sim_render_camera  sensors.c:69-82  (declared sim_internal.h:102)
 * which tb_sim_step_env calls per player every 9th step (LiDAR) and every
 * 2nd step (cameras, unless external_cameras is set), src/sim/physics.c:
 * 376-380, and tb_sim_reset_env after a reset, physics.c:170.  The reference
 * has no GPU renderer and no C entry point taking a scene; the scene record
 * below carries exactly the simulator state those two functions read, so a
 * caller packs it from TbEnv/TbConfig and renders every environment's sensors
 * in one call, with the observations left on the device.
 *
 * Results equal the reference's CPU renderer: the LiDAR ranges, dropouts
 * and valid fractions bit for bit, and the camera bytes bit for bit except
 * where a pixel's luma*255 lies within about 1e-15 (relative) of a rounding
 * boundary, where CUDA's double exp and the host libm's may round the last
 * bit differently.  The body-frame ray directions are built once per process
 * with the host C library's sin, cos, tan, hypot and atan2, the functions the
 * simulator itself calls.
 */
#ifndef TURBINATOR_CUDA_SENSORS_H
#define TURBINATOR_CUDA_SENSORS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TB_SENSOR_MAX_OBSTACLES 24 /* TB_MAX_OBSTACLES, sim_internal.h:13 */
#define TB_SENSOR_MAX_BALLS 64     /* TB_MAX_BALLS, sim_internal.h:11 */
#define TB_SENSOR_LIDAR_BINS 4096  /* 2 heads x 16 elevations x 128 azimuths */
#define TB_SENSOR_CAMERA_PIXELS 16384     /* 4 views x 64 x 64 */
#define TB_SENSOR_CAMERA_RAW_PIXELS 147456 /* 4 views x 192 x 192 */

/* tb_sensor_scene.sensors bits */
#define TB_SENSOR_LIDAR 1
#define TB_SENSOR_CAMERA 2

/* What the renderers read for one aircraft (player) of one environment.
 * 2,432 bytes, 8-byte aligned. */
typedef struct tb_sensor_scene {
    double position[3];    /* TbAircraft.pos of the rendering player */
    double attitude[4];    /* TbAircraft.quat, w x y z */
    double opponent[3];    /* the other player's pos; read in arena scenarios */
    double lidar_max;      /* TbConfig.lidar_max (sky distance too) */
    double dome_radius;    /* TbConfig.dome_radius (arena scenarios) */
    uint64_t rng;          /* TbEnv.rng (LiDAR dropout and noise stream) */
    int32_t step_index;    /* TbEnv.step_index */
    int32_t player;        /* 0 or 1 */
    int32_t scenario;      /* TbEnv.scenario, 0..27 */
    int32_t sensors;       /* TB_SENSOR_LIDAR | TB_SENSOR_CAMERA: what to render */
    int32_t obstacle_count; /* 0..24 (values outside are clamped) */
    int32_t ball_count;     /* 0..64 (values outside are clamped) */
    double obstacles[TB_SENSOR_MAX_OBSTACLES][4]; /* center x y z, radius */
    double balls[TB_SENSOR_MAX_BALLS][3];         /* centers; radius 0.25 */
} tb_sensor_scene;

/* Renders the sensors of device_scenes[0..count) on `stream` (a
 * cudaStream_t, NULL = legacy default stream).  Device pointers:
 *   device_lidar        scene i's 4,096 ranges (metres, -1 = dropout) at
 *                       device_lidar + i*lidar_stride; lidar_stride >= 4096
 *                       floats (4148 with device_lidar = obs + 48 writes them
 *                       straight into observation rows, as tb_sim_observe
 *                       copies them, sensors.c:117)
 *   device_lidar_valid  scene i's two per-head valid fractions at
 *                       device_lidar_valid + i*valid_stride, valid_stride >= 2
 *                       (4148 with obs + 4146: observation entries 4146-4147)
 *   device_cameras      [count, 16384] bytes, view-major 4 x 64 x 64
 *   device_raw_cameras  [count, 147456] bytes, each pixel repeated 3 x 3
 *                       (the simulator's raw capture, sensors.c:78), or NULL
 * A scene renders LiDAR when its TB_SENSOR_LIDAR bit is set and
 * device_lidar is not NULL (device_lidar_valid may be NULL), and cameras when
 * its TB_SENSOR_CAMERA bit is set and device_cameras or device_raw_cameras is
 * not NULL; everything else is left unwritten, so one call can follow the
 * simulator's cadence (LiDAR every 9th step, cameras every 2nd).
 * Returns 1 if the launch succeeded, 0 on NULL scenes, count 0 or
 * > 0x7fffffff, scenes not 8-byte aligned, an output not 4-byte aligned, a
 * stride below its minimum, or a launch error.  Asynchronous.  The first call
 * on each device uploads the 480 KB of body-frame ray tables with a
 * synchronous copy; make it before any stream capture. */
int tb_cuda_render_sensors_device(const tb_sensor_scene *device_scenes,
                                  size_t count,
                                  float *device_lidar,
                                  size_t lidar_stride,
                                  float *device_lidar_valid,
                                  size_t valid_stride,
                                  unsigned char *device_cameras,
                                  unsigned char *device_raw_cameras,
                                  void *stream);

#ifdef __cplusplus
}
#endif

#endif
