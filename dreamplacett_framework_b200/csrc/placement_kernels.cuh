// placement_kernels.cuh -- device pieces of the global-placement loop around
// the electric-potential operator:
//
//   k_overflow   fixed-point density grid (+ initial density) -> overflow area
//                and maximum density: the per-iteration overflow metric that
//                DREAMPlace's placer evaluates (ElectricOverflow; the reference
//                reads it back per iteration in integration/run_dreamplace.py:333-370)
//   k_grad_linf  max over nodes of max(|grad_x|, |grad_y|)
//   k_descent    normalised gradient step of every node, clamped to the die
//
// Both reductions are deterministic: k_overflow reduces fixed per-block chunks
// in fp64 in a fixed order and the last block combines the block partials in
// block order; the maximum is order-independent.
#pragma once
#include <cstdint>
#include "epb_kernels.cuh"

namespace epb {

constexpr int kOvfThreads = 256;
constexpr int kOvfBinsPerThread = 8;   // bins per thread that size the block count
constexpr int kOvfMaxBlocks = 2048;

inline int ovf_blocks(int64_t nbins) {
    const int64_t per = (int64_t)kOvfThreads * kOvfBinsPerThread;
    int64_t b = (nbins + per - 1) / per;
    return (int)(b < 1 ? 1 : (b > kOvfMaxBlocks ? kOvfMaxBlocks : b));
}

// Per bin: rho = fp32(q * dscale) + init (the density-map value epb_forward
// writes), excess = max(rho - target, 0) in fp64.  out[0] = bin_area * sum of
// excess, out[1] = max rho.  With `merge`, each bin's q is then added to
// merge[bin] (another grid of the same layout, e.g. the one the forward converts).
// The grid is left zeroed for the next scatter.
__global__ void __launch_bounds__(kOvfThreads)
k_overflow(long long* __restrict__ qgrid, const float* __restrict__ init, double dscale, int64_t nbins,
           float target, double bin_area, double* __restrict__ partials, unsigned* __restrict__ counter,
           double* __restrict__ out, long long* __restrict__ merge, unsigned* __restrict__ flags) {
    __shared__ double s_sum[kOvfThreads];
    __shared__ double s_max[kOvfThreads];
    __shared__ bool is_last;
    // block b reduces bins [b*chunk, (b+1)*chunk): a fixed partition of the grid
    const int64_t chunk = (nbins + gridDim.x - 1) / gridDim.x;
    const int64_t lo = (int64_t)blockIdx.x * chunk;
    const int64_t hi = min(nbins, lo + chunk);
    double sum = 0.0;
    float mx = -INFINITY;
    unsigned sat = 0;
    for (int64_t i = lo + threadIdx.x; i < hi; i += kOvfThreads) {
        const long long q = qgrid[i];
        if (q < 0 || q >= (1ll << 62)) sat = 1;
        float v = __double2float_rn(__dmul_rn(__ll2double_rn(q), dscale));
        if (init) v = __fadd_rn(v, __ldg(init + i));
        const double ex = (double)v - (double)target;
        if (ex > 0.0) sum += ex;
        mx = fmaxf(mx, v);
    }
    // merge and re-zero after every load of this thread has been issued
    for (int64_t i = lo + threadIdx.x; i < hi; i += kOvfThreads) {
        if (merge) {
            const long long q = qgrid[i];
            if (q != 0) merge[i] += q;
        }
        qgrid[i] = 0;
    }
    if (sat) atomicOr(flags, kFlagSaturated);
    s_sum[threadIdx.x] = sum;
    s_max[threadIdx.x] = (double)mx;
    __syncthreads();
    for (int w = kOvfThreads / 2; w > 0; w >>= 1) {
        if (threadIdx.x < w) {
            s_sum[threadIdx.x] += s_sum[threadIdx.x + w];
            s_max[threadIdx.x] = fmax(s_max[threadIdx.x], s_max[threadIdx.x + w]);
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        partials[2 * blockIdx.x] = s_sum[0];
        partials[2 * blockIdx.x + 1] = s_max[0];
        __threadfence();
        const unsigned t = atomicInc(counter, gridDim.x - 1);
        is_last = (t == gridDim.x - 1);
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    double s = 0.0, m = -INFINITY;
    for (int b = threadIdx.x; b < (int)gridDim.x; b += kOvfThreads) {
        s += __ldcg(partials + 2 * b);
        m = fmax(m, __ldcg(partials + 2 * b + 1));
    }
    s_sum[threadIdx.x] = s;
    s_max[threadIdx.x] = m;
    __syncthreads();
    for (int w = kOvfThreads / 2; w > 0; w >>= 1) {
        if (threadIdx.x < w) {
            s_sum[threadIdx.x] += s_sum[threadIdx.x + w];
            s_max[threadIdx.x] = fmax(s_max[threadIdx.x], s_max[threadIdx.x + w]);
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        out[0] = s_sum[0] * bin_area;
        out[1] = s_max[0];
    }
}

// max(|gx|, |gy|) over the cells' nodes, as the bit pattern of a non-negative
// float (for those, unsigned order is float order) -> atomicMax.  Non-finite
// gradients are skipped and flagged.
__global__ void __launch_bounds__(256)
k_grad_linf(CellView c, const float* __restrict__ gx, const float* __restrict__ gy, unsigned* __restrict__ linf_bits,
            unsigned* __restrict__ flags) {
    unsigned m = 0, bad = 0;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < c.n; i += stride) {
        const int64_t node = cell_node(c, i);
        const float a = fabsf(__ldg(gx + node)), b = fabsf(__ldg(gy + node));
        if (!isfinite(a) || !isfinite(b)) { bad = 1; continue; }
        m = max(m, max(__float_as_uint(a), __float_as_uint(b)));
    }
    m = __reduce_max_sync(0xffffffffu, m);
    if ((threadIdx.x & 31) == 0 && m != 0) atomicMax(linf_bits, m);
    if (bad) atomicOr(flags, kFlagNonFinite);
}

// x <- max(min(x - (step_x / linf) * gx, xh - w), xl), and likewise y, for
// every node of the cells' ranges; no move when linf is 0.  Every operation is
// one fp32 round-to-nearest step so the CPU restatement matches bit for bit.
__global__ void __launch_bounds__(256)
k_descent(CellView c, float* __restrict__ x, float* __restrict__ y, const float* __restrict__ gx,
          const float* __restrict__ gy, const float* __restrict__ w, const float* __restrict__ h,
          const unsigned* __restrict__ linf_bits, float step_x, float step_y, float xl, float yl, float xh, float yh,
          float* __restrict__ linf_out) {
    const float linf = __uint_as_float(*linf_bits);
    if (linf_out && blockIdx.x == 0 && threadIdx.x == 0) *linf_out = linf;
    if (!(linf > 0.0f)) return;
    const float sx = __fdiv_rn(step_x, linf), sy = __fdiv_rn(step_y, linf);
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < c.n; i += stride) {
        const int64_t node = cell_node(c, i);
        const float a = __ldg(gx + node), b = __ldg(gy + node);
        if (!isfinite(a) || !isfinite(b)) continue;
        float nx = __fsub_rn(x[node], __fmul_rn(sx, a));
        float ny = __fsub_rn(y[node], __fmul_rn(sy, b));
        nx = fmaxf(fminf(nx, __fsub_rn(xh, __ldg(w + node))), xl);
        ny = fmaxf(fminf(ny, __fsub_rn(yh, __ldg(h + node))), yl);
        x[node] = nx;
        y[node] = ny;
    }
}

}  // namespace epb
