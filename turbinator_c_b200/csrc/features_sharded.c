/*
 * tb_cuda_extract_features_device_sharded: the device entry point over
 * several GPUs in one call (C11).  No counterpart in the reference, whose ABI
 * drives one device per call (include/turbinator/training/cuda_features.h:
 * 14-19); each shard here is exactly such a call on its own device, made
 * current for the launch.  No data crosses between devices.
 */
#include <stddef.h>

#include <cuda_runtime_api.h>

#include "tb_features_internal.h"
#include "turbinator/training/cuda_features.h"

int tb_cuda_extract_features_device_sharded(int shard_count, const int *device_ids,
                                            const float *const *device_obs,
                                            const float *const *device_mission,
                                            const unsigned char *const *device_cameras,
                                            float *const *device_features, const size_t *batch_sizes,
                                            void *const *streams) {
    if (shard_count < 1 || shard_count > TB_CUDA_MAX_SHARDS || !device_ids || !device_obs || !device_mission ||
        !device_features || !batch_sizes)
        return 0;
    int devices = 0;
    if (cudaGetDeviceCount(&devices) != cudaSuccess) return 0;
    for (int i = 0; i < shard_count; ++i) {
        if (device_ids[i] < 0 || device_ids[i] >= devices) return 0;
        if (batch_sizes[i] > 0x7fffffffu) return 0;
        if (batch_sizes[i] && (!device_obs[i] || !device_mission[i] || !device_features[i])) return 0;
    }
    int caller = 0;
    if (cudaGetDevice(&caller) != cudaSuccess) return 0;
    int ok = 1;
    for (int i = 0; i < shard_count && ok; ++i) {
        if (batch_sizes[i] == 0) continue; /* an empty shard launches nothing */
        if (cudaSetDevice(device_ids[i]) != cudaSuccess) {
            cudaGetLastError();
            ok = 0;
            break;
        }
        ok = tb_features_launch(device_obs[i], device_mission[i], device_cameras ? device_cameras[i] : NULL,
                                device_features[i], batch_sizes[i], streams ? streams[i] : NULL, NULL);
    }
    if (cudaSetDevice(caller) != cudaSuccess) ok = 0;
    return ok;
}
