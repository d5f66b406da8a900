/*
 * TEST INFRASTRUCTURE ONLY -- launches the reference's own input-preparation
 * kernels for its 618M learner, compiled from where they lie
 * (src/network/network_gpu.cu: scalar_inputs :274-303, lidar_channels
 * :467-479, camera_luma :480-483, launched as at :1446-1451).  They are
 * static to that file, so this shim includes it and adds one extern "C"
 * launcher.  Built by oracle/Makefile into oracle/_ref/; nothing of the
 * reference is copied here.  The GPU tests use it as the bit-level oracle of
 * tb_cuda_prepare_actor_inputs_device.
 */
#include "network_gpu.cu"

extern "C" int tb_ref_actor_inputs(const float *obs, const float *mission, const uint8_t *cameras,
                                   float *proprio, float *mission_vec, float *tactical, float *prior,
                                   float *lidar, float *luma, int batch) {
    scalar_inputs<<<(unsigned)((batch + 127) / 128), 128>>>(obs, mission, proprio, mission_vec, tactical, prior,
                                                             batch);
    const size_t lidar_count = (size_t)batch * 6 * 16 * 128, luma_count = (size_t)batch * 16384;
    lidar_channels<<<(unsigned)((lidar_count + 255) / 256), 256>>>(obs, lidar, lidar_count);
    camera_luma<<<(unsigned)((luma_count + 255) / 256), 256>>>(cameras, luma, luma_count);
    return cudaGetLastError() == cudaSuccess;
}
