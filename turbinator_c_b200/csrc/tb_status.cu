/*
 * Per-stream status words of the kernels' bounded pipeline waits.
 *
 * The staged kernels (features, learner inputs, onboard scans) wait on
 * mbarriers with a time limit; a wait that expires ORs a bit into a status
 * word that the host reads behind the work.  The reference reports errors per
 * handle (src/cuda/features.cu:20-25) and synchronises per stream
 * (tb_cuda_synchronize(stream), features.cu:171-173), so a status word here
 * belongs to one stream: every launch writes the word of the stream it is
 * launched on, and tb_cuda_synchronize(stream) / a handle's lanes read and
 * clear only that word.  A timeout on one stream is therefore never reported
 * to, or cleared by, a caller that synchronises another stream.
 *
 * Layout: a fixed __device__ array of kSlots words per device (no
 * allocation).  Slot 0 is shared by streams beyond the first kSlots - 1 seen
 * on a device; slots 1.. are handed out in first-use order, keyed by the
 * stream handle's value (NULL, cudaStreamLegacy and cudaStreamPerThread are
 * keys like any other).  A handle value that is reused by a new stream after
 * the old one was destroyed keeps the old stream's slot (a bit the old
 * stream never reported would surface on the new one).  The device address of
 * the array is looked up once per device (cudaGetSymbolAddress, with that
 * device current) and cached: after a cudaDeviceReset the cache is stale, so
 * a process that resets a device must not call this library on it again.
 */
#include <cuda_runtime.h>

#include <mutex>
#include <stdint.h>

#include "tb_features_internal.h"

namespace {

constexpr int kSlots = 1024;
constexpr int kMaxDevices = 64;

__device__ unsigned int g_status_slots[kSlots];

struct DeviceSlots {
    std::mutex lock;
    unsigned int *base = nullptr;   /* device address of g_status_slots */
    uintptr_t keys[kSlots] = {};
    int used = 1;                   /* slot 0 is the shared overflow slot */
};
DeviceSlots g_devices[kMaxDevices];

/* One-entry cache per host thread: the (device, stream) of the last lookup. */
struct SlotCache {
    int dev = -1;
    uintptr_t key = 0;
    unsigned int *slot = nullptr;
};
thread_local SlotCache t_cache;

unsigned int *slot_for(int dev, uintptr_t key) {
    DeviceSlots &d = g_devices[dev];
    std::lock_guard<std::mutex> hold(d.lock);
    if (!d.base) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_status_slots) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        d.base = static_cast<unsigned int *>(p);
    }
    for (int i = 1; i < d.used; ++i)
        if (d.keys[i] == key) return d.base + i;
    if (d.used < kSlots) {
        d.keys[d.used] = key;
        return d.base + d.used++;
    }
    return d.base; /* shared overflow slot */
}

} /* namespace */

extern "C" unsigned int *tb_status_slot(void *stream) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    const uintptr_t key = reinterpret_cast<uintptr_t>(stream);
    SlotCache &c = t_cache;
    if (c.slot && c.dev == dev && c.key == key) return c.slot;
    unsigned int *slot = slot_for(dev, key);
    if (slot) {
        c.dev = dev;
        c.key = key;
        c.slot = slot;
    }
    return slot;
}

extern "C" int tb_status_take(void *stream, unsigned int *status) {
    unsigned int *slot = tb_status_slot(stream);
    if (!slot) return 0;
    unsigned int value = 0;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (cudaMemcpyAsync(&value, slot, sizeof(value), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return 0;
    if (value && (cudaMemsetAsync(slot, 0, sizeof(unsigned int), s) != cudaSuccess ||
                  cudaStreamSynchronize(s) != cudaSuccess))
        return 0;
    if (status) *status = value;
    return 1;
}

extern "C" int tb_status_enqueue(void *stream, unsigned int *host_word) {
    unsigned int *slot = tb_status_slot(stream);
    return slot && cudaMemcpyAsync(host_word, slot, sizeof(unsigned int), cudaMemcpyDeviceToHost,
                                   static_cast<cudaStream_t>(stream)) == cudaSuccess;
}

extern "C" int tb_status_clear(void *stream) {
    unsigned int *slot = tb_status_slot(stream);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    return slot && cudaMemsetAsync(slot, 0, sizeof(unsigned int), s) == cudaSuccess &&
           cudaStreamSynchronize(s) == cudaSuccess;
}
