/*
 * C11 host side of the batched feature ABI: the persistent staging handle
 * that the trainer's batch loop uses (reference src/cuda/features.cu:9-88;
 * call sites src/trainer/main.c:513,526,566,618,673,706).
 *
 * Differences from the reference that keep its contract:
 *  - max_batch is no longer capped at 1024; staging is sized to max_batch.
 *  - A handle may span several GPUs (tb_cuda_feature_batch_create_multi):
 *    each call's rows are split into contiguous per-device shards.
 *  - Within a device the rows are split again into "lanes", one host thread
 *    each (the caller's and workers that the handle starts on its first call
 *    with more than one lane and keeps until it is destroyed).  Page-locked caller buffers are copied straight to the device in
 *    chunks alternating between two streams.  Large pageable calls (the
 *    trainer's calloc'd batch buffers) are copied by each lane's thread into
 *    a double-buffered page-locked staging area, so the host copy of one
 *    chunk overlaps the DMA and kernel of the previous one and several lanes
 *    copy in parallel; the driver's own pageable copy runs on one thread at
 *    a fraction of PCIe speed.  Small pageable calls use the driver's path.
 *  - After the last copy the status words of the lane's own streams are
 *    checked (each stream has its own, tb_status.cu, so another handle's or
 *    thread's timeout is never reported here); a timed-out pipeline fails
 *    the call with a stage-named message.
 * Error strings keep the reference's "stage: cuda error" form and stage
 * names (features.cu:20-25,70-87).
 */
#define _POSIX_C_SOURCE 200809L
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include <cuda_runtime_api.h>

#include "tb_features_internal.h"
#include "turbinator/training/cuda_features.h"

#define TB_MAX_BATCH ((size_t)0x7fffffff)
#define TB_MAX_DEVICES 16
#define TB_MAX_LANES 16
/* Rows per chunk when the caller's buffers are page-locked (~270 MB of input). */
#define TB_DIRECT_CHUNK ((size_t)8192)
/* Rows per page-locked staging buffer (~8.5 MB of input). */
#define TB_STAGE_ROWS ((size_t)256)
/* Pageable calls below this many rows per device let the driver copy from the
 * caller's buffers directly (faster at that size than staging on one
 * thread); larger ones are staged, one host thread per TB_STAGE_ROWS rows up
 * to the lane count. */
#ifndef TB_STAGED_MIN_ROWS
#define TB_STAGED_MIN_ROWS ((size_t)512)
#endif

#define TB_IN_ROW_BYTES (TB_OBS_DIM * sizeof(float) + TB_MISSION_DIM * sizeof(float) + TB_CAMERA_BYTES)
#define TB_OUT_ROW_BYTES (TB_FEATURE_DIM * sizeof(float))

typedef struct tb_lane {
    cudaStream_t streams[2];
    cudaEvent_t staged_free[2];   /* host->device copy out of stage b finished */
    cudaEvent_t result_ready[2];  /* features of stage b's chunk are in out_stage[b] */
    unsigned char *in_stage[2];   /* page-locked: obs | mission | cameras rows */
    float *out_stage[2];          /* page-locked features rows */
    unsigned int *status;         /* page-locked: the kernels' status word as seen by each stream */
    size_t stage_rows;
} tb_lane;

typedef struct tb_device_shard {
    int device_id;
    size_t rows;                  /* device staging capacity */
    float *obs, *mission, *features;
    unsigned char *cameras;
    int lane_count;
    tb_lane lanes[TB_MAX_LANES];
} tb_device_shard;

struct tb_lane_job;

struct tb_cuda_feature_batch {
    int device_id;                /* first device (the reference handle's device) */
    size_t max_batch;
    int device_count;
    tb_device_shard shards[TB_MAX_DEVICES];
    char error[192];
    /* Worker threads that run a call's lanes beside the calling thread; started
     * on the first call with more than one lane, kept until the handle is
     * destroyed.  A call posts its jobs and takes part itself. */
    int pool_ready;               /* lock and conditions initialised */
    int pool_size;                /* workers started */
    pthread_t pool_threads[TB_MAX_DEVICES * TB_MAX_LANES];
    pthread_mutex_t pool_lock;
    pthread_cond_t pool_work, pool_done;
    struct tb_lane_job *pool_jobs;
    int pool_job_count, pool_next, pool_finished, pool_quit;
    unsigned long pool_generation;
};

/* ------------------------------------------------------------------ */

static int batch_fail(tb_cuda_feature_batch *batch, const char *stage, cudaError_t status) {
    if (batch)
        snprintf(batch->error, sizeof(batch->error), "%s: %s", stage, cudaGetErrorString(status));
    return 0;
}

static void lane_release(tb_lane *lane) {
    for (int b = 0; b < 2; ++b) {
        if (lane->streams[b]) {
            cudaStreamSynchronize(lane->streams[b]);
            cudaStreamDestroy(lane->streams[b]);
        }
        if (lane->staged_free[b]) cudaEventDestroy(lane->staged_free[b]);
        if (lane->result_ready[b]) cudaEventDestroy(lane->result_ready[b]);
        if (lane->in_stage[b]) cudaFreeHost(lane->in_stage[b]);
        if (lane->out_stage[b]) cudaFreeHost(lane->out_stage[b]);
    }
    if (lane->status) cudaFreeHost(lane->status);
    memset(lane, 0, sizeof(*lane));
}

static void shard_release(tb_device_shard *shard) {
    if (!shard->obs && !shard->lane_count) return; /* never set up */
    if (cudaSetDevice(shard->device_id) != cudaSuccess) return;
    for (int l = 0; l < shard->lane_count; ++l) lane_release(&shard->lanes[l]);
    cudaFree(shard->obs);
    cudaFree(shard->mission);
    cudaFree(shard->cameras);
    cudaFree(shard->features);
    shard->obs = shard->mission = shard->features = NULL;
    shard->cameras = NULL;
}

static int lane_init(tb_lane *lane, size_t rows) {
    lane->stage_rows = rows < TB_STAGE_ROWS ? rows : TB_STAGE_ROWS;
    if (lane->stage_rows == 0) lane->stage_rows = 1;
    if (cudaHostAlloc((void **)&lane->status, 2 * sizeof(unsigned int), cudaHostAllocPortable) != cudaSuccess)
        return 0;
    for (int b = 0; b < 2; ++b) {
        if (cudaStreamCreateWithFlags(&lane->streams[b], cudaStreamNonBlocking) != cudaSuccess ||
            cudaEventCreateWithFlags(&lane->staged_free[b], cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&lane->result_ready[b], cudaEventDisableTiming) != cudaSuccess ||
            cudaHostAlloc((void **)&lane->in_stage[b], lane->stage_rows * TB_IN_ROW_BYTES,
                          cudaHostAllocPortable) != cudaSuccess ||
            cudaHostAlloc((void **)&lane->out_stage[b], lane->stage_rows * TB_OUT_ROW_BYTES,
                          cudaHostAllocPortable) != cudaSuccess)
            return 0;
    }
    return 1;
}

/* Host threads a handle may use per call: TB_CUDA_HOST_THREADS if set,
 * else the online CPUs, capped at 8 per device. */
static int host_threads_per_device(int device_count) {
    long n = 0;
    const char *env = getenv("TB_CUDA_HOST_THREADS");
    if (env && *env) n = strtol(env, NULL, 10);
    if (n <= 0) {
        n = sysconf(_SC_NPROCESSORS_ONLN);
        if (n <= 0) n = 1;
    }
    n /= device_count;
    if (n < 1) n = 1;
    if (n > 8) n = 8;
    return (int)n;
}

tb_cuda_feature_batch *tb_cuda_feature_batch_create_multi(const int *device_ids, int device_count,
                                                          size_t max_batch) {
    if (!device_ids || device_count < 1 || device_count > TB_MAX_DEVICES || max_batch == 0 ||
        max_batch > TB_MAX_BATCH)
        return NULL;
    /* the first device ends current on the calling thread, as in the reference */
    for (int d = device_count - 1; d >= 0; --d)
        if (cudaSetDevice(device_ids[d]) != cudaSuccess) {
            cudaGetLastError(); /* a bad device id must not fail this thread's next launch */
            return NULL;
        }
    tb_cuda_feature_batch *batch = (tb_cuda_feature_batch *)calloc(1, sizeof(*batch));
    if (!batch) return NULL;
    batch->device_id = device_ids[0];
    batch->max_batch = max_batch;
    batch->device_count = device_count;
    const int lanes = host_threads_per_device(device_count);
    int ok = 1;
    for (int d = 0; d < device_count && ok; ++d) {
        tb_device_shard *shard = &batch->shards[d];
        shard->device_id = device_ids[d];
        shard->rows = (max_batch + (size_t)device_count - 1) / (size_t)device_count;
        ok = cudaSetDevice(shard->device_id) == cudaSuccess &&
             cudaMalloc((void **)&shard->obs, shard->rows * TB_OBS_DIM * sizeof(float)) == cudaSuccess &&
             cudaMalloc((void **)&shard->mission, shard->rows * TB_MISSION_DIM * sizeof(float)) == cudaSuccess &&
             cudaMalloc((void **)&shard->cameras, shard->rows * TB_CAMERA_BYTES) == cudaSuccess &&
             cudaMalloc((void **)&shard->features, shard->rows * TB_OUT_ROW_BYTES) == cudaSuccess;
        /* extra lanes only where a call can be large enough to use them */
        const int shard_lanes = shard->rows >= 2 * TB_STAGED_MIN_ROWS ? lanes : 1;
        const size_t per_lane = (shard->rows + (size_t)shard_lanes - 1) / (size_t)shard_lanes;
        for (int l = 0; l < shard_lanes && ok; ++l) {
            shard->lane_count = l + 1;
            ok = lane_init(&shard->lanes[l], l == 0 ? shard->rows : per_lane);
        }
    }
    if (!ok) {
        tb_cuda_feature_batch_destroy(batch);
        cudaGetLastError(); /* do not leave the allocation failure for the next launch check */
        return NULL;
    }
    cudaSetDevice(device_ids[0]);
    return batch;
}

tb_cuda_feature_batch *tb_cuda_feature_batch_create(int device_id, size_t max_batch) {
    return tb_cuda_feature_batch_create_multi(&device_id, 1, max_batch);
}

static void pool_stop(tb_cuda_feature_batch *batch) {
    if (!batch->pool_ready) return;
    pthread_mutex_lock(&batch->pool_lock);
    batch->pool_quit = 1;
    pthread_cond_broadcast(&batch->pool_work);
    pthread_mutex_unlock(&batch->pool_lock);
    for (int i = 0; i < batch->pool_size; ++i) pthread_join(batch->pool_threads[i], NULL);
    pthread_cond_destroy(&batch->pool_work);
    pthread_cond_destroy(&batch->pool_done);
    pthread_mutex_destroy(&batch->pool_lock);
    batch->pool_ready = 0;
    batch->pool_size = 0;
}

void tb_cuda_feature_batch_destroy(tb_cuda_feature_batch *batch) {
    if (!batch) return;
    pool_stop(batch);
    for (int d = 0; d < batch->device_count; ++d) shard_release(&batch->shards[d]);
    cudaSetDevice(batch->device_id);
    free(batch);
}

const char *tb_cuda_feature_batch_error(const tb_cuda_feature_batch *batch) {
    return batch ? batch->error : "CUDA feature batch unavailable";
}

/* 1 if the byte at `p` is page-locked (or otherwise device-visible) host memory. */
static int host_byte_pinned(const void *p) {
    struct cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return attr.type == cudaMemoryTypeHost || attr.type == cudaMemoryTypeManaged;
}

/* 1 if the first and the last byte of [p, p + bytes) are page-locked: a buffer
 * that is page-locked only at its start takes the staged (pageable) path. */
static int host_pinned(const void *p, size_t bytes) {
    return host_byte_pinned(p) && host_byte_pinned((const unsigned char *)p + bytes - 1);
}

/* ------------------------------------------------------------------ */
/* One lane's share of a call: rows [first, first + count) of the caller's
 * arrays, processed on its shard's device into device rows starting at
 * shard_first.  Runs on its own host thread (or the caller's). */

typedef struct tb_lane_job {
    tb_device_shard *shard;
    tb_lane *lane;
    size_t first, count;          /* caller rows */
    size_t shard_first;           /* device staging rows */
    const float *obs, *mission;
    const unsigned char *cameras;
    float *out;
    int direct_in;                /* copy from the caller's buffers (page-locked, or a small call) */
    int direct_out;               /* caller's output page-locked */
    const char *stage;            /* failing stage, NULL on success */
    cudaError_t status;
} tb_lane_job;

static void job_fail(tb_lane_job *job, const char *stage, cudaError_t status) {
    if (!job->stage) {
        job->stage = stage;
        job->status = status;
    }
}

/* Launch the features of device rows [row, row + n) on stream s. */
static int job_launch(tb_lane_job *job, size_t row, size_t n, cudaStream_t s) {
    tb_device_shard *sh = job->shard;
    int launch_error = 0;
    if (!tb_features_launch_checked(sh->obs + row * TB_OBS_DIM, sh->mission + row * TB_MISSION_DIM,
                                    sh->cameras + row * TB_CAMERA_BYTES, sh->features + row * TB_FEATURE_DIM,
                                    n, s, NULL, &launch_error)) {
        job_fail(job, "extract features", (cudaError_t)launch_error);
        return 0;
    }
    return 1;
}

/* Page-locked caller buffers: chunked async copies, alternating streams. */
static void job_run_direct(tb_lane_job *job) {
    tb_device_shard *sh = job->shard;
    tb_lane *lane = job->lane;
    cudaError_t st;
    size_t chunk = 0;
    for (size_t done = 0; done < job->count; done += TB_DIRECT_CHUNK, ++chunk) {
        const size_t n = job->count - done < TB_DIRECT_CHUNK ? job->count - done : TB_DIRECT_CHUNK;
        const size_t src = job->first + done, dst = job->shard_first + done;
        cudaStream_t s = lane->streams[chunk & 1];
        if ((st = cudaMemcpyAsync(sh->obs + dst * TB_OBS_DIM, job->obs + src * TB_OBS_DIM,
                                  n * TB_OBS_DIM * sizeof(float), cudaMemcpyHostToDevice, s)) != cudaSuccess) {
            job_fail(job, "copy observations", st);
            return;
        }
        if ((st = cudaMemcpyAsync(sh->mission + dst * TB_MISSION_DIM, job->mission + src * TB_MISSION_DIM,
                                  n * TB_MISSION_DIM * sizeof(float), cudaMemcpyHostToDevice, s)) != cudaSuccess) {
            job_fail(job, "copy mission", st);
            return;
        }
        if ((st = cudaMemcpyAsync(sh->cameras + dst * TB_CAMERA_BYTES, job->cameras + src * TB_CAMERA_BYTES,
                                  n * TB_CAMERA_BYTES, cudaMemcpyHostToDevice, s)) != cudaSuccess) {
            job_fail(job, "copy cameras", st);
            return;
        }
        if (!job_launch(job, dst, n, s)) return;
        if (job->direct_out &&
            (st = cudaMemcpyAsync(job->out + src * TB_FEATURE_DIM, sh->features + dst * TB_FEATURE_DIM,
                                  n * TB_OUT_ROW_BYTES, cudaMemcpyDeviceToHost, s)) != cudaSuccess) {
            job_fail(job, "copy features", st);
            return;
        }
    }
    if (!job->direct_out) {
        /* pageable destination: one synchronous copy after every kernel */
        for (int b = 0; b < 2; ++b)
            if ((st = cudaStreamSynchronize(lane->streams[b])) != cudaSuccess) {
                job_fail(job, "synchronize features", st);
                return;
            }
        if ((st = cudaMemcpy(job->out + job->first * TB_FEATURE_DIM, sh->features + job->shard_first * TB_FEATURE_DIM,
                             job->count * TB_OUT_ROW_BYTES, cudaMemcpyDeviceToHost)) != cudaSuccess)
            job_fail(job, "copy features", st);
    }
}

/* Pageable caller buffers: the lane copies each chunk into page-locked
 * staging (double-buffered) and streams it from there. */
static void job_run_staged(tb_lane_job *job) {
    tb_device_shard *sh = job->shard;
    tb_lane *lane = job->lane;
    const size_t rows = lane->stage_rows;
    const size_t chunks = (job->count + rows - 1) / rows;
    cudaError_t st;
    for (size_t k = 0; k < chunks + 2; ++k) {
        const int b = (int)(k & 1);
        /* retire chunk k-2 from buffer b: its features to the caller */
        if (k >= 2) {
            const size_t done = (k - 2) * rows;
            const size_t n = job->count - done < rows ? job->count - done : rows;
            if ((st = cudaEventSynchronize(lane->result_ready[b])) != cudaSuccess) {
                job_fail(job, "synchronize features", st);
                return;
            }
            memcpy(job->out + (job->first + done) * TB_FEATURE_DIM, lane->out_stage[b], n * TB_OUT_ROW_BYTES);
        }
        if (k >= chunks) continue;
        const size_t done = k * rows;
        const size_t n = job->count - done < rows ? job->count - done : rows;
        const size_t src = job->first + done, dst = job->shard_first + done;
        unsigned char *stage = lane->in_stage[b];
        float *s_obs = (float *)stage;
        float *s_mission = s_obs + rows * TB_OBS_DIM;
        unsigned char *s_cam = (unsigned char *)(s_mission + rows * TB_MISSION_DIM);
        if (k >= 2 && (st = cudaEventSynchronize(lane->staged_free[b])) != cudaSuccess) {
            job_fail(job, "copy observations", st);
            return;
        }
        memcpy(s_obs, job->obs + src * TB_OBS_DIM, n * TB_OBS_DIM * sizeof(float));
        memcpy(s_mission, job->mission + src * TB_MISSION_DIM, n * TB_MISSION_DIM * sizeof(float));
        memcpy(s_cam, job->cameras + src * TB_CAMERA_BYTES, n * TB_CAMERA_BYTES);
        cudaStream_t s = lane->streams[b];
        if ((st = cudaMemcpyAsync(sh->obs + dst * TB_OBS_DIM, s_obs, n * TB_OBS_DIM * sizeof(float),
                                  cudaMemcpyHostToDevice, s)) != cudaSuccess) {
            job_fail(job, "copy observations", st);
            return;
        }
        if ((st = cudaMemcpyAsync(sh->mission + dst * TB_MISSION_DIM, s_mission,
                                  n * TB_MISSION_DIM * sizeof(float), cudaMemcpyHostToDevice, s)) != cudaSuccess) {
            job_fail(job, "copy mission", st);
            return;
        }
        if ((st = cudaMemcpyAsync(sh->cameras + dst * TB_CAMERA_BYTES, s_cam, n * TB_CAMERA_BYTES,
                                  cudaMemcpyHostToDevice, s)) != cudaSuccess) {
            job_fail(job, "copy cameras", st);
            return;
        }
        if ((st = cudaEventRecord(lane->staged_free[b], s)) != cudaSuccess) {
            job_fail(job, "copy cameras", st);
            return;
        }
        if (!job_launch(job, dst, n, s)) return;
        if ((st = cudaMemcpyAsync(lane->out_stage[b], sh->features + dst * TB_FEATURE_DIM, n * TB_OUT_ROW_BYTES,
                                  cudaMemcpyDeviceToHost, s)) != cudaSuccess ||
            (st = cudaEventRecord(lane->result_ready[b], s)) != cudaSuccess) {
            job_fail(job, "copy features", st);
            return;
        }
    }
}

static void *job_main(void *arg) {
    tb_lane_job *job = (tb_lane_job *)arg;
    cudaError_t st = cudaSetDevice(job->shard->device_id);
    if (st != cudaSuccess) {
        job_fail(job, "select device", st);
        return NULL;
    }
    if (job->direct_in)
        job_run_direct(job);
    else
        job_run_staged(job);
    /* read the kernels' status word behind this lane's work on each stream it
     * used (a job of one chunk uses stream 0 only) */
    const size_t chunk_rows = job->direct_in ? TB_DIRECT_CHUNK : job->lane->stage_rows;
    const int used = job->count > chunk_rows ? 2 : 1;
    job->lane->status[0] = job->lane->status[1] = 0;
    for (int b = 0; b < used; ++b)
        if (!job->stage && !tb_status_enqueue(job->lane->streams[b], &job->lane->status[b]))
            job_fail(job, "synchronize features", cudaGetLastError());
    /* leave nothing in flight that reads or writes the caller's buffers */
    for (int b = 0; b < used; ++b) {
        st = cudaStreamSynchronize(job->lane->streams[b]);
        if (st != cudaSuccess) job_fail(job, "synchronize features", st);
    }
    int timed_out = 0;
    for (int b = 0; b < used; ++b)
        if (job->lane->status[b]) {
            tb_status_clear(job->lane->streams[b]); /* report each expiry once */
            timed_out = 1;
        }
    if (!job->stage && timed_out) job->stage = "synchronize features: feature pipeline wait timed out";
    return NULL;
}

/* Worker loop: wait for a new call's jobs, take them one at a time. */
static void *pool_worker(void *arg) {
    tb_cuda_feature_batch *batch = (tb_cuda_feature_batch *)arg;
    unsigned long seen = 0;
    pthread_mutex_lock(&batch->pool_lock);
    for (;;) {
        while (!batch->pool_quit && batch->pool_generation == seen)
            pthread_cond_wait(&batch->pool_work, &batch->pool_lock);
        if (batch->pool_quit) break;
        seen = batch->pool_generation;
        while (batch->pool_next < batch->pool_job_count) {
            struct tb_lane_job *job = &batch->pool_jobs[batch->pool_next++];
            pthread_mutex_unlock(&batch->pool_lock);
            job_main(job);
            pthread_mutex_lock(&batch->pool_lock);
            if (++batch->pool_finished == batch->pool_job_count) pthread_cond_broadcast(&batch->pool_done);
        }
    }
    pthread_mutex_unlock(&batch->pool_lock);
    return NULL;
}

/* Start workers until `want` run (as many as the system gives). */
static void pool_grow(tb_cuda_feature_batch *batch, int want) {
    if (!batch->pool_ready) {
        if (pthread_mutex_init(&batch->pool_lock, NULL) != 0) return;
        if (pthread_cond_init(&batch->pool_work, NULL) != 0) {
            pthread_mutex_destroy(&batch->pool_lock);
            return;
        }
        if (pthread_cond_init(&batch->pool_done, NULL) != 0) {
            pthread_cond_destroy(&batch->pool_work);
            pthread_mutex_destroy(&batch->pool_lock);
            return;
        }
        batch->pool_ready = 1;
    }
    while (batch->pool_size < want &&
           pthread_create(&batch->pool_threads[batch->pool_size], NULL, pool_worker, batch) == 0)
        ++batch->pool_size;
}

/* Runs every job: on the pool's workers and the calling thread together. */
static void run_jobs(tb_cuda_feature_batch *batch, tb_lane_job *jobs, int job_count) {
    if (job_count > 1) pool_grow(batch, job_count - 1);
    if (job_count <= 1 || !batch->pool_ready) {
        for (int j = 0; j < job_count; ++j) job_main(&jobs[j]);
        return;
    }
    pthread_mutex_lock(&batch->pool_lock);
    batch->pool_jobs = jobs;
    batch->pool_job_count = job_count;
    batch->pool_next = 0;
    batch->pool_finished = 0;
    ++batch->pool_generation;
    pthread_cond_broadcast(&batch->pool_work);
    while (batch->pool_next < job_count) {
        tb_lane_job *job = &jobs[batch->pool_next++];
        pthread_mutex_unlock(&batch->pool_lock);
        job_main(job);
        pthread_mutex_lock(&batch->pool_lock);
        if (++batch->pool_finished == job_count) pthread_cond_broadcast(&batch->pool_done);
    }
    while (batch->pool_finished < job_count) pthread_cond_wait(&batch->pool_done, &batch->pool_lock);
    batch->pool_jobs = NULL;
    batch->pool_job_count = 0;
    pthread_mutex_unlock(&batch->pool_lock);
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

    const int direct_in = host_pinned(obs, count * TB_OBS_DIM * sizeof(float)) &&
                          host_pinned(mission, count * TB_MISSION_DIM * sizeof(float)) &&
                          host_pinned(cameras, count * TB_CAMERA_BYTES);
    const int direct_out = host_pinned(out_features, count * TB_OUT_ROW_BYTES);
    tb_lane_job jobs[TB_MAX_DEVICES * TB_MAX_LANES];
    int job_count = 0;
    for (int d = 0; d < batch->device_count; ++d) {
        tb_device_shard *shard = &batch->shards[d];
        const size_t first = count * (size_t)d / (size_t)batch->device_count;
        const size_t rows = count * (size_t)(d + 1) / (size_t)batch->device_count - first;
        if (rows == 0) continue;
        /* page-locked input needs no host copy, and small pageable calls go
         * through the driver: one lane; else one lane per TB_STAGE_ROWS rows */
        const int staged = !direct_in && rows >= TB_STAGED_MIN_ROWS;
        int lanes = 1;
        if (staged) {
            const size_t want = rows / TB_STAGE_ROWS;
            lanes = want < (size_t)shard->lane_count ? (int)want : shard->lane_count;
            if (lanes < 1) lanes = 1;
        }
        for (int l = 0; l < lanes; ++l) {
            const size_t a = rows * (size_t)l / (size_t)lanes, z = rows * (size_t)(l + 1) / (size_t)lanes;
            if (z == a) continue;
            tb_lane_job *job = &jobs[job_count++];
            memset(job, 0, sizeof(*job));
            job->shard = shard;
            job->lane = &shard->lanes[l];
            job->first = first + a;
            job->count = z - a;
            job->shard_first = a;
            job->obs = obs;
            job->mission = mission;
            job->cameras = cameras;
            job->out = out_features;
            job->direct_in = !staged;
            job->direct_out = direct_out;
        }
    }
    run_jobs(batch, jobs, job_count);
    cudaSetDevice(batch->device_id);
    for (int j = 0; j < job_count; ++j) {
        if (!jobs[j].stage) continue;
        if (jobs[j].status == cudaSuccess) { /* the kernels' own pipeline report */
            snprintf(batch->error, sizeof(batch->error), "%s", jobs[j].stage);
            return 0;
        }
        return batch_fail(batch, jobs[j].stage, jobs[j].status);
    }
    return 1;
}
