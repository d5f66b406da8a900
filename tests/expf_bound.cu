/*
 * Largest absolute error of CUDA's __expf against its double exp over every
 * float argument a in [-88, 0] (test infrastructure for the sensor kernel's
 * float fog, turbinator_c_b200/csrc/sensors_kernel.cu: shade).  Below -88
 * both values are under 1e-38.  Prints the largest error and its argument.
 */
#include <cstdio>
#include <cuda_runtime.h>

__global__ void worst_error(unsigned int first, unsigned int count, unsigned long long *worst) {
    unsigned long long mine = 0;
    for (unsigned int i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += gridDim.x * blockDim.x) {
        const float a = __uint_as_float(first + i);
        const double err = fabs(static_cast<double>(__expf(a)) - exp(static_cast<double>(a)));
        /* error in the high 44 bits, argument bits in the low 20 bits would
         * lose the argument; keep the error's bits and report the argument
         * of the largest separately below */
        const unsigned long long bits = static_cast<unsigned long long>(__double_as_longlong(err));
        mine = bits > mine ? bits : mine;
    }
    atomicMax(worst, mine);
}

__global__ void find_argument(unsigned int first, unsigned int count, unsigned long long target,
                              unsigned int *where) {
    for (unsigned int i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += gridDim.x * blockDim.x) {
        const float a = __uint_as_float(first + i);
        const double err = fabs(static_cast<double>(__expf(a)) - exp(static_cast<double>(a)));
        if (static_cast<unsigned long long>(__double_as_longlong(err)) == target) atomicMin(where, first + i);
    }
}

int main() {
    const unsigned int first = 0x80000000u;          /* -0.0 */
    const unsigned int last = 0xC2B00000u;           /* -88.0 */
    const unsigned int count = last - first + 1;
    unsigned long long *worst = nullptr;
    unsigned int *where = nullptr;
    if (cudaMallocManaged(&worst, sizeof(*worst)) != cudaSuccess ||
        cudaMallocManaged(&where, sizeof(*where)) != cudaSuccess)
        return 2;
    *worst = 0;
    *where = 0xffffffffu;
    worst_error<<<148 * 16, 256>>>(first, count, worst);
    if (cudaDeviceSynchronize() != cudaSuccess) return 3;
    find_argument<<<148 * 16, 256>>>(first, count, *worst, where);
    if (cudaDeviceSynchronize() != cudaSuccess) return 4;
    double err;
    const unsigned long long bits = *worst;
    __builtin_memcpy(&err, &bits, sizeof(err));
    unsigned int arg_bits = *where;
    float arg;
    __builtin_memcpy(&arg, &arg_bits, sizeof(arg));
    std::printf("%.9e %.9e %u\n", err, static_cast<double>(arg), count);
    return 0;
}
