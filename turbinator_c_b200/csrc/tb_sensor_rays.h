/* Body-frame ray directions of the simulator's LiDAR and cameras, built on
 * the host (sensor_rays.c) and uploaded once per device by sensors_kernel.cu. */
#ifndef TB_SENSOR_RAYS_H
#define TB_SENSOR_RAYS_H

#ifdef __cplusplus
extern "C" {
#endif

/* dirs[3*bin + k], bin = head*2048 + elevation*128 + azimuth; occluded[bin]
 * is 1 where the airframe blocks the ray. */
void tb_sensor_lidar_rays(double *dirs, unsigned char *occluded);

/* dirs[3*pixel + k], pixel = view*4096 + y*64 + x. */
void tb_sensor_camera_rays(double *dirs);

#ifdef __cplusplus
}
#endif

#endif
