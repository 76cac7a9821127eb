// geometry.cuh -- per-cell bin footprint and overlap weights shared by the
// scatter and gather kernels.
//
// Every fp32 operation is an explicit round-to-nearest intrinsic so nvcc can
// not contract a multiply-add into an FMA: the contributions must equal the
// CPU restatement bit for bit (the fixed-point density is bit-exact).
//
// Reference semantics (paths relative to ayadavTT/DREAMPlaceTT-Framework):
//   bin index  kernels/v4_compute.cpp:85-126  floor((v - origin) * inv_bs),
//              clamped at 0, corrected so origin + k*bs <= v < origin + (k+1)*bs
//   overlap    kernels/v4_compute.cpp:128-176 max(0, min(v+s, left+bs) - max(v, left)),
//              left = origin + k*bs
#pragma once
#include <cstdint>

namespace epb {

struct GridGeom {
    int M, N;                 // bins along x (rows) and y (columns)
    float xl, yl, bsx, bsy;   // origin and fp32 bin sizes
    float ibsx, ibsy;         // fp32(1 / bin size)
};

struct CellView {
    const float* __restrict__ x;
    const float* __restrict__ y;
    const float* __restrict__ sx;
    const float* __restrict__ sy;
    const float* __restrict__ ox;   // nullable offsets
    const float* __restrict__ oy;
    const float* __restrict__ ratio; // nullable
    int64_t b0, n0;  // first range: nodes b0 .. b0+n0-1
    int64_t b1;      // second range starts at node b1
    int64_t n;       // total cells (n0 + second range length)
};

constexpr int kSelChunk = 2048;   // cells per segment of a shard's band list

__device__ __forceinline__ int64_t cell_node(const CellView& c, int64_t i) {
    return i < c.n0 ? c.b0 + i : c.b1 + (i - c.n0);
}

// Visit every cell of v with body(node), the work spread over the grid by a
// grid-stride loop.
template <typename F>
__device__ __forceinline__ void for_each_cell(const CellView& c, F&& body) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < c.n; i += stride) body(cell_node(c, i));
}

__device__ __forceinline__ int bin_floor(float v, float origin, float bs, float ibs, int nb) {
    float t = floorf(__fmul_rn(__fsub_rn(v, origin), ibs));
    if (t < 0.0f) t = 0.0f;
    if (t > (float)nb) t = (float)nb;
    int k = (int)t;
    float bl = __fadd_rn(origin, __fmul_rn((float)k, bs));
    if (bl > v) k -= 1;
    bl = __fadd_rn(origin, __fmul_rn((float)(k + 1), bs));
    if (bl <= v) k += 1;
    if (k < 0) k = 0;
    return k;
}

__device__ __forceinline__ float bin_overlap(float v, float vend, float origin, float bs, int k) {
    float left = __fadd_rn(origin, __fmul_rn((float)k, bs));
    float lo = v > left ? v : left;
    float right = __fadd_rn(left, bs);
    float hi = vend < right ? vend : right;
    float o = __fsub_rn(hi, lo);
    return o < 0.0f ? 0.0f : o;
}

struct Footprint {
    float x, y, ex, ey, r;
    int kx0, kx1, ky0, ky1;
};

// Returns -1 for a non-finite cell (skipped and flagged), 0 when the cell
// contributes nothing (non-positive size or off the die), 2 when it is outside
// the row band [row_lo, row_hi) (owner == false: its rows do not meet the band;
// owner == true: its first row is not in the band), 1 otherwise.
//
// On the whole grid every load is issued before any test (one memory round
// trip per cell).  On a row band the x data is read first, so a cell of another
// band costs three loads instead of seven; the test is uniform across the grid.
// A cell's raw inputs (offsets and ratio as given; absent ones unused).  Kept
// apart from the footprint arithmetic so a kernel can have the next cell's
// loads in flight while it works on the current one.
struct CellData {
    float x, ox, y, oy, sx, sy, r;
};

__device__ __forceinline__ CellData load_cell(const CellView& c, int64_t node) {
    CellData d;
    d.x = __ldg(c.x + node);
    d.ox = c.ox ? __ldg(c.ox + node) : 0.0f;
    d.sx = __ldg(c.sx + node);
    d.y = __ldg(c.y + node);
    d.oy = c.oy ? __ldg(c.oy + node) : 0.0f;
    d.sy = __ldg(c.sy + node);
    d.r = c.ratio ? __ldg(c.ratio + node) : 1.0f;
    return d;
}

// Footprint of a cell from its loaded inputs on the whole grid (no band), as
// cell_footprint computes it with the band [0, M): -1 for non-finite inputs, 0
// for an empty footprint, 2 for a footprint outside the grid's rows, else 1.
__device__ __forceinline__ int footprint_of(const CellView& c, const GridGeom& g, const CellData& d, Footprint& f) {
    const float x = c.ox ? __fadd_rn(d.x, d.ox) : d.x;
    const float y = c.oy ? __fadd_rn(d.y, d.oy) : d.y;
    if (!isfinite(x) || !isfinite(d.sx)) return -1;
    bool empty = !(d.sx > 0.0f);
    if (!empty) {
        f.ex = __fadd_rn(x, d.sx);
        f.kx0 = bin_floor(x, g.xl, g.bsx, g.ibsx, g.M);
        f.kx1 = min(bin_floor(f.ex, g.xl, g.bsx, g.ibsx, g.M), g.M - 1);
        empty = f.kx0 > f.kx1;
        if (!empty && (f.kx1 < 0 || f.kx0 >= g.M)) return 2;
    }
    if (!isfinite(y) || !isfinite(d.sy) || !isfinite(d.r)) return -1;
    if (empty || !(d.sy > 0.0f)) return 0;
    f.ey = __fadd_rn(y, d.sy);
    f.ky0 = bin_floor(y, g.yl, g.bsy, g.ibsy, g.N);
    f.ky1 = min(bin_floor(f.ey, g.yl, g.bsy, g.ibsy, g.N), g.N - 1);
    if (f.ky0 > f.ky1) return 0;
    f.x = x; f.y = y; f.r = d.r;
    return 1;
}

// Visit the cells of v as for_each_cell does, calling body(node, data) with the
// cell's loaded inputs; each thread loads its next cell's inputs before it
// works on the current one, so that load overlaps the body's own reads.
template <typename F>
__device__ __forceinline__ void for_each_cell_prefetched(const CellView& c, F&& body) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= c.n) return;
    CellData cur = load_cell(c, cell_node(c, i));
    for (;;) {
        const int64_t inext = i + stride;
        CellData nxt = cur;
        if (inext < c.n) nxt = load_cell(c, cell_node(c, inext));
        body(cell_node(c, i), cur);
        if (inext >= c.n) break;
        cur = nxt;
        i = inext;
    }
}

__device__ __forceinline__ int cell_footprint(const CellView& c, const GridGeom& g, int64_t node,
                                              Footprint& f, int row_lo, int row_hi, bool owner) {
    const bool banded = row_lo > 0 || row_hi < g.M;
    float x = __ldg(c.x + node);
    if (c.ox) x = __fadd_rn(x, __ldg(c.ox + node));
    const float sx = __ldg(c.sx + node);
    float y = 0.0f, sy = 0.0f, r = 1.0f;
    if (!banded) {
        y = __ldg(c.y + node);
        if (c.oy) y = __fadd_rn(y, __ldg(c.oy + node));
        sy = __ldg(c.sy + node);
        if (c.ratio) r = __ldg(c.ratio + node);
    }
    if (!isfinite(x) || !isfinite(sx)) return -1;
    bool empty = !(sx > 0.0f);
    if (!empty) {
        f.ex = __fadd_rn(x, sx);
        f.kx0 = bin_floor(x, g.xl, g.bsx, g.ibsx, g.M);
        f.kx1 = min(bin_floor(f.ex, g.xl, g.bsx, g.ibsx, g.M), g.M - 1);
        empty = f.kx0 > f.kx1;
        if (!empty && (owner ? (f.kx0 < row_lo || f.kx0 >= row_hi) : (f.kx1 < row_lo || f.kx0 >= row_hi)))
            return 2;
    }
    if (banded) {
        // the rest is read for cells of this band, and for empty cells so every
        // non-finite input is reported as on one GPU
        y = __ldg(c.y + node);
        if (c.oy) y = __fadd_rn(y, __ldg(c.oy + node));
        sy = __ldg(c.sy + node);
        if (c.ratio) r = __ldg(c.ratio + node);
    }
    if (!isfinite(y) || !isfinite(sy) || !isfinite(r)) return -1;
    if (empty || !(sy > 0.0f)) return 0;
    f.ey = __fadd_rn(y, sy);
    f.ky0 = bin_floor(y, g.yl, g.bsy, g.ibsy, g.N);
    f.ky1 = min(bin_floor(f.ey, g.yl, g.bsy, g.ibsy, g.N), g.N - 1);
    if (f.ky0 > f.ky1) return 0;
    f.x = x; f.y = y; f.r = r;
    return 1;
}

}  // namespace epb
