// probe_atomics.cu -- measures the 64-bit atomic-add rate that bounds the
// density scatter: 1.4M "cells" each add to an FX x FY footprint of a
// 2048 x 2048 int64 grid (rows of 2048 words) at a hashed position, the
// pattern of k_scatter's red.global.add.u64.  Prints G atomic adds per second
// per footprint shape, plus a plain-load pass over the same grid for scale.
//
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 \
//        dreamplacett_framework_b200/csrc/probe_atomics.cu -o probe_atomics && ./probe_atomics
#include <cstdint>
#include <cstdio>
#include <cuda_runtime.h>

#define CK(x)                                                                          \
    do {                                                                               \
        cudaError_t e_ = (x);                                                          \
        if (e_ != cudaSuccess) {                                                       \
            std::printf("CUDA error %s at line %d\n", cudaGetErrorString(e_), __LINE__); \
            return 1;                                                                  \
        }                                                                              \
    } while (0)

namespace {

constexpr int kSide = 2048;

__device__ __forceinline__ unsigned mix(unsigned x) {
    x ^= x >> 16; x *= 0x7feb352du; x ^= x >> 15; x *= 0x846ca68bu; x ^= x >> 16;
    return x;
}

// one thread per cell; FX x FY adds (RED = true) or loads at a hashed position
template <int FX, int FY, bool RED>
__global__ void __launch_bounds__(256) footprint(unsigned long long* g, int ncell, unsigned long long* sink) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= ncell) return;
    const unsigned h = mix((unsigned)i * 2654435761u + 17u);
    const int kx = h % (kSide - FX), ky = (h >> 11) % (kSide - FY);
    unsigned long long acc = 0;
    for (int a = 0; a < FX; ++a)
        for (int b = 0; b < FY; ++b) {
            unsigned long long* p = g + (size_t)(kx + a) * kSide + ky + b;
            if (RED) atomicAdd(p, 1ull + a + b);
            else acc += *p;
        }
    if (!RED && acc == 0x1234567ull) *sink = acc;
}

}  // namespace

int main() {
    const size_t words = (size_t)kSide * kSide;
    unsigned long long *g = nullptr, *sink = nullptr;
    CK(cudaMalloc(&g, words * sizeof(unsigned long long)));
    CK(cudaMalloc(&sink, sizeof(unsigned long long)));
    CK(cudaMemset(g, 0, words * sizeof(unsigned long long)));
    const int ncell = 1400000;
    const unsigned blocks = (ncell + 255) / 256;
    cudaEvent_t e0, e1;
    CK(cudaEventCreate(&e0));
    CK(cudaEventCreate(&e1));
    auto run = [&](const char* name, double ops, auto launch) -> int {
        for (int w = 0; w < 3; ++w) launch();
        CK(cudaEventRecord(e0));
        for (int r = 0; r < 20; ++r) launch();
        CK(cudaEventRecord(e1));
        CK(cudaEventSynchronize(e1));
        float ms = 0.0f;
        CK(cudaEventElapsedTime(&ms, e0, e1));
        const double us = ms * 1000.0 / 20.0;
        std::printf("%-12s %9.2f us  %7.1f G ops/s\n", name, us, ops / us / 1e3);
        return 0;
    };
    if (run("2x2 add", ncell * 4.0, [&] { footprint<2, 2, true><<<blocks, 256>>>(g, ncell, sink); })) return 1;
    if (run("2x3 add", ncell * 6.0, [&] { footprint<2, 3, true><<<blocks, 256>>>(g, ncell, sink); })) return 1;
    if (run("3x3 add", ncell * 9.0, [&] { footprint<3, 3, true><<<blocks, 256>>>(g, ncell, sink); })) return 1;
    if (run("3x3 load", ncell * 9.0, [&] { footprint<3, 3, false><<<blocks, 256>>>(g, ncell, sink); })) return 1;
    CK(cudaGetLastError());
    CK(cudaDeviceSynchronize());
    CK(cudaFree(g));
    CK(cudaFree(sink));
    return 0;
}
