/*
 * HBM throughput of simple float4 streams by access pattern -- the ceilings
 * the feature and learner-input kernels are read against.  Not part of the
 * library: a measurement program built beside it (../hbm_patterns).
 *
 * Each case streams rows shaped like the kernels' per-aircraft blocks:
 * 65,536 rows of 33,024 B read (the feature kernel's input bytes), and
 * 65,536 rows of 114,688 B written (about the learner-input kernel's
 * output bytes).  Three ways of dealing rows to CTAs are compared:
 *   grid-stride  a fixed grid, each thread strides over the flat buffer
 *   persistent   a fixed grid, CTA c takes rows c, c + grid, ...
 *   runs of R    a covering grid, CTA c takes rows [c*R, (c+1)*R); the
 *                hardware hands CTAs to SMs as they free up
 * plus cudaMemsetAsync and a device-to-device cudaMemcpyAsync.  Times are
 * CUDA events around one launch, best of 10, a 256 MiB memset between
 * launches to flush L2; GB/s counts bytes read plus bytes written.
 */
#include <cuda_runtime.h>

#include <cstdio>

namespace {

constexpr size_t kRows = 65536;
constexpr size_t kReadRowF4 = 2064;   /* 33,024 B */
constexpr size_t kWriteRowF4 = 7168;  /* 114,688 B */

__device__ __forceinline__ float sum4(float4 v) { return (v.x + v.y) + (v.z + v.w); }

__global__ void read_grid_stride(const float4 *p, size_t n4, float *sink) {
    float acc = 0.f;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        acc += sum4(__ldcs(p + i));
    if (acc == 1234.5f) *sink = acc; /* keeps the loads; never true for the zeroed input */
}

__global__ void read_persistent(const float4 *p, float *sink) {
    float acc = 0.f;
    for (size_t r = blockIdx.x; r < kRows; r += gridDim.x)
        for (size_t i = threadIdx.x; i < kReadRowF4; i += blockDim.x) acc += sum4(__ldcs(p + r * kReadRowF4 + i));
    if (acc == 1234.5f) *sink = acc;
}

__global__ void read_runs(const float4 *p, float *sink, size_t run) {
    float acc = 0.f;
    const size_t first = blockIdx.x * run;
    for (size_t r = first; r < first + run && r < kRows; ++r)
        for (size_t i = threadIdx.x; i < kReadRowF4; i += blockDim.x) acc += sum4(__ldcs(p + r * kReadRowF4 + i));
    if (acc == 1234.5f) *sink = acc;
}

__global__ void write_grid_stride(float4 *p, size_t n4) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const float f = static_cast<float>(i & 0xffff);
        __stcs(p + i, make_float4(f, f, f, f));
    }
}

__global__ void write_persistent(float4 *p) {
    for (size_t r = blockIdx.x; r < kRows; r += gridDim.x)
        for (size_t i = threadIdx.x; i < kWriteRowF4; i += blockDim.x) {
            const float f = static_cast<float>(i & 0xff) + static_cast<float>(r);
            __stcs(p + r * kWriteRowF4 + i, make_float4(f, f, f, f));
        }
}

__global__ void write_runs(float4 *p, size_t run) {
    const size_t first = blockIdx.x * run;
    for (size_t r = first; r < first + run && r < kRows; ++r)
        for (size_t i = threadIdx.x; i < kWriteRowF4; i += blockDim.x) {
            const float f = static_cast<float>(i & 0xff) + static_cast<float>(r);
            __stcs(p + r * kWriteRowF4 + i, make_float4(f, f, f, f));
        }
}

bool check(cudaError_t e, const char *what) {
    if (e != cudaSuccess) std::printf("%s: %s\n", what, cudaGetErrorString(e));
    return e == cudaSuccess;
}

} /* namespace */

int main() {
    const size_t read4 = kRows * kReadRowF4, write4 = kRows * kWriteRowF4;
    const size_t flush_bytes = 256u << 20;
    float4 *in = nullptr, *out = nullptr;
    float *sink = nullptr;
    void *flush = nullptr;
    if (!check(cudaMalloc(&in, read4 * 16), "cudaMalloc") || !check(cudaMalloc(&out, write4 * 16), "cudaMalloc") ||
        !check(cudaMalloc(&sink, 4), "cudaMalloc") || !check(cudaMalloc(&flush, flush_bytes), "cudaMalloc") ||
        !check(cudaMemset(in, 0, read4 * 16), "cudaMemset"))
        return 1;
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    bool ok = true;
    auto run = [&](const char *name, double bytes, auto launch) {
        for (int i = 0; i < 3; ++i) launch();
        ok = check(cudaDeviceSynchronize(), name) && ok;
        float best = 1e30f;
        for (int rep = 0; rep < 10; ++rep) {
            cudaMemsetAsync(flush, rep, flush_bytes);
            cudaEventRecord(a);
            launch();
            cudaEventRecord(b);
            cudaEventSynchronize(b);
            float ms = 0.f;
            cudaEventElapsedTime(&ms, a, b);
            if (ms < best) best = ms;
        }
        ok = check(cudaGetLastError(), name) && ok;
        std::printf("| %-44s | %8.4f | %6.0f |\n", name, best, bytes / best / 1e6);
    };
    const double rd = read4 * 16.0, wr = write4 * 16.0;
    std::printf("| case | ms | GB/s |\n|---|---|---|\n");
    run("read 2.16 GB: grid-stride, 8 x SMs CTAs x 256", rd,
        [&] { read_grid_stride<<<sms * 8, 256>>>(in, read4, sink); });
    run("read 2.16 GB: persistent, 2 x SMs CTAs x 256", rd, [&] { read_persistent<<<sms * 2, 256>>>(in, sink); });
    run("read 2.16 GB: persistent, 8 x SMs CTAs x 256", rd, [&] { read_persistent<<<sms * 8, 256>>>(in, sink); });
    run("read 2.16 GB: runs of 8 rows, CTAs of 256", rd,
        [&] { read_runs<<<kRows / 8, 256>>>(in, sink, 8); });
    run("read 2.16 GB: runs of 1 row, CTAs of 256", rd, [&] { read_runs<<<kRows, 256>>>(in, sink, 1); });
    run("read 2.16 GB: runs of 1 row, CTAs of 512", rd, [&] { read_runs<<<kRows, 512>>>(in, sink, 1); });
    run("write 7.52 GB: cudaMemsetAsync", wr, [&] { cudaMemsetAsync(out, 0, write4 * 16); });
    run("write 7.52 GB: grid-stride, 8 x SMs CTAs x 256", wr, [&] { write_grid_stride<<<sms * 8, 256>>>(out, write4); });
    run("write 7.52 GB: persistent, 2 x SMs CTAs x 256", wr, [&] { write_persistent<<<sms * 2, 256>>>(out); });
    run("write 7.52 GB: persistent, 8 x SMs CTAs x 256", wr, [&] { write_persistent<<<sms * 8, 256>>>(out); });
    run("write 7.52 GB: runs of 1 row, CTAs of 256", wr, [&] { write_runs<<<kRows, 256>>>(out, 1); });
    run("copy 2.16 GB -> 2.16 GB: cudaMemcpyAsync", 2 * rd,
        [&] { cudaMemcpyAsync(out, in, read4 * 16, cudaMemcpyDeviceToDevice); });
    cudaFree(in);
    cudaFree(out);
    cudaFree(sink);
    cudaFree(flush);
    return ok ? 0 : 1;
}
