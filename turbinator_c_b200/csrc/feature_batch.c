/*
 * C11 host side of the batched feature ABI: the persistent staging handle
 * that the trainer's batch loop uses (reference src/cuda/features.cu:9-88;
 * call sites src/trainer/main.c:513,526,566,618,673,706).
 *
 * Differences from the reference that keep its contract:
 *  - max_batch is no longer capped at 1024; staging is sized to max_batch.
 *  - Large batches are split into chunks that alternate between two
 *    non-blocking streams, so the host->device copy of one chunk overlaps the
 *    kernel and the device->host copy of the previous one.
 *  - After the last copy the kernels' pipeline status word is checked; a
 *    timed-out pipeline fails the call with a stage-named message.
 * Error strings keep the reference's "stage: cuda error" form and stage
 * names (features.cu:20-25,70-87).
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>

#include "tb_features_internal.h"
#include "turbinator/training/cuda_features.h"

/* Samples per pipelined chunk (~270 MB of input). */
#define TB_HOST_CHUNK ((size_t)8192)
#define TB_MAX_BATCH ((size_t)0x7fffffff)

struct tb_cuda_feature_batch {
    int device_id;
    size_t max_batch;
    cudaStream_t streams[2];
    float *obs;
    float *mission;
    unsigned char *cameras;
    float *features;
    char error[192];
};

static int batch_fail(tb_cuda_feature_batch *batch, const char *stage, cudaError_t status) {
    if (batch)
        snprintf(batch->error, sizeof(batch->error), "%s: %s", stage, cudaGetErrorString(status));
    return 0;
}

/* Fail after asynchronous work was queued: let it drain first, so no copy
 * still reads the caller's buffers after we return. */
static int batch_fail_drain(tb_cuda_feature_batch *batch, const char *stage, cudaError_t status) {
    batch_fail(batch, stage, status);
    cudaStreamSynchronize(batch->streams[0]);
    cudaStreamSynchronize(batch->streams[1]);
    return 0;
}

tb_cuda_feature_batch *tb_cuda_feature_batch_create(int device_id, size_t max_batch) {
    if (max_batch == 0 || max_batch > TB_MAX_BATCH) return NULL;
    if (cudaSetDevice(device_id) != cudaSuccess) {
        cudaGetLastError(); /* a bad device id must not fail this thread's next launch */
        return NULL;
    }
    tb_cuda_feature_batch *batch = (tb_cuda_feature_batch *)calloc(1, sizeof(*batch));
    if (!batch) return NULL;
    batch->device_id = device_id;
    batch->max_batch = max_batch;
    if (cudaStreamCreateWithFlags(&batch->streams[0], cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&batch->streams[1], cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc((void **)&batch->obs, max_batch * TB_OBS_DIM * sizeof(float)) != cudaSuccess ||
        cudaMalloc((void **)&batch->mission, max_batch * TB_MISSION_DIM * sizeof(float)) != cudaSuccess ||
        cudaMalloc((void **)&batch->cameras, max_batch * TB_CAMERA_BYTES) != cudaSuccess ||
        cudaMalloc((void **)&batch->features, max_batch * TB_FEATURE_DIM * sizeof(float)) != cudaSuccess) {
        tb_cuda_feature_batch_destroy(batch);
        cudaGetLastError(); /* do not leave the allocation failure for the next launch check */
        return NULL;
    }
    return batch;
}

void tb_cuda_feature_batch_destroy(tb_cuda_feature_batch *batch) {
    if (!batch) return;
    cudaSetDevice(batch->device_id);
    for (int i = 0; i < 2; ++i)
        if (batch->streams[i]) cudaStreamSynchronize(batch->streams[i]);
    cudaFree(batch->obs);
    cudaFree(batch->mission);
    cudaFree(batch->cameras);
    cudaFree(batch->features);
    for (int i = 0; i < 2; ++i)
        if (batch->streams[i]) cudaStreamDestroy(batch->streams[i]);
    free(batch);
}

const char *tb_cuda_feature_batch_error(const tb_cuda_feature_batch *batch) {
    return batch ? batch->error : "CUDA feature batch unavailable";
}

/* 1 if `p` is page-locked (or device-visible) host memory. */
static int host_pinned(const void *p) {
    struct cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return attr.type == cudaMemoryTypeHost || attr.type == cudaMemoryTypeManaged;
}

int tb_cuda_extract_features_host(tb_cuda_feature_batch *batch, const float *obs,
                                  const float *mission, const unsigned char *cameras,
                                  size_t count, float *out_features) {
    if (!batch || !obs || !mission || !cameras || !out_features || count == 0 ||
        count > batch->max_batch)
        return 0;
    batch->error[0] = 0;
    cudaError_t status = cudaSetDevice(batch->device_id);
    if (status != cudaSuccess) return batch_fail(batch, "select device", status);

    /* Pageable destinations make each device->host copy synchronous, which
     * would serialise the chunks; those get one copy after the last kernel. */
    const int stream_out = host_pinned(out_features);
    size_t chunk_index = 0;
    for (size_t first = 0; first < count; first += TB_HOST_CHUNK, ++chunk_index) {
        const size_t n = count - first < TB_HOST_CHUNK ? count - first : TB_HOST_CHUNK;
        cudaStream_t s = batch->streams[chunk_index & 1];
        status = cudaMemcpyAsync(batch->obs + first * TB_OBS_DIM, obs + first * TB_OBS_DIM,
                                 n * TB_OBS_DIM * sizeof(float), cudaMemcpyHostToDevice, s);
        if (status != cudaSuccess) return batch_fail_drain(batch, "copy observations", status);
        status = cudaMemcpyAsync(batch->mission + first * TB_MISSION_DIM,
                                 mission + first * TB_MISSION_DIM,
                                 n * TB_MISSION_DIM * sizeof(float), cudaMemcpyHostToDevice, s);
        if (status != cudaSuccess) return batch_fail_drain(batch, "copy mission", status);
        status = cudaMemcpyAsync(batch->cameras + first * TB_CAMERA_BYTES,
                                 cameras + first * TB_CAMERA_BYTES, n * TB_CAMERA_BYTES,
                                 cudaMemcpyHostToDevice, s);
        if (status != cudaSuccess) return batch_fail_drain(batch, "copy cameras", status);
        int launch_error = 0;
        if (!tb_features_launch_checked(batch->obs + first * TB_OBS_DIM,
                                        batch->mission + first * TB_MISSION_DIM,
                                        batch->cameras + first * TB_CAMERA_BYTES,
                                        batch->features + first * TB_FEATURE_DIM, n, s, NULL,
                                        &launch_error))
            return batch_fail_drain(batch, "extract features", (cudaError_t)launch_error);
        if (stream_out) {
            status = cudaMemcpyAsync(out_features + first * TB_FEATURE_DIM,
                                     batch->features + first * TB_FEATURE_DIM,
                                     n * TB_FEATURE_DIM * sizeof(float), cudaMemcpyDeviceToHost, s);
            if (status != cudaSuccess) return batch_fail_drain(batch, "copy features", status);
        }
    }
    if (!stream_out) {
        if (chunk_index > 1) {
            /* The single copy below runs on stream 0; order it after stream 1. */
            status = cudaStreamSynchronize(batch->streams[1]);
            if (status != cudaSuccess) return batch_fail_drain(batch, "synchronize features", status);
        }
        status = cudaMemcpyAsync(out_features, batch->features, count * TB_FEATURE_DIM * sizeof(float),
                                 cudaMemcpyDeviceToHost, batch->streams[0]);
        if (status != cudaSuccess) return batch_fail_drain(batch, "copy features", status);
    }
    for (int i = 0; i < 2; ++i) {
        status = cudaStreamSynchronize(batch->streams[i]);
        if (status != cudaSuccess) return batch_fail_drain(batch, "synchronize features", status);
    }
    unsigned int pipeline = 0;
    if (!tb_features_status_take(batch->streams[0], &pipeline))
        return batch_fail(batch, "synchronize features", cudaGetLastError());
    if (pipeline) {
        snprintf(batch->error, sizeof(batch->error),
                 "synchronize features: feature pipeline wait timed out");
        return 0;
    }
    return 1;
}
