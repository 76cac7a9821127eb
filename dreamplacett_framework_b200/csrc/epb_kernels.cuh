// epb_kernels.cuh -- CUDA kernels of the electric-potential step.
//
//   k_scatter      cells -> int64 fixed-point density grid (atomic adds to L2)
//   k_row_fwd<L>   grid (or fp32 density) -> normalised density rho (+ initial
//                  density), then DCT-II along y of every row       -> T1
//   k_col<L>       DCT-II along x of T1 columns -> auv; spectral energy;
//                  weights wu/wv/inv; inverse transforms along x     -> Gx, Gy, Gp
//   k_row_inv<L>   inverse transforms along y of Gx, Gy, Gp rows     -> field_x,
//                  field_y, potential (+ interleaved field map for the gather)
//   k_gather       cells + interleaved fields -> per-node gradient
//
// Grid layout: [M rows = x bins][N columns = y bins], row-major, index bx*N+by
// (the reference's density layout, host/density_scatter_ttnn_server_host.cpp:458-459).
//
// Transform conventions follow the reference's matrices
// (host/density_scatter_ttnn_server_host.cpp:124-181):
//   DCT2[k,n]  = (2/L) cos(pi k (n+1/2)/L)
//   IDCT[k,n]  = n == 0 ? 1 : 2 cos(pi n (k+1/2)/L)
//   IDXST[k,n] = sin(pi n (k+1/2)/L)
// computed with L-point complex FFTs (two real sequences packed per FFT):
//   DCT2:  v = makhoul(x); V = FFT(v); a_k = (2/L) Re(exp(-i pi k/2L) V_k)
//   IDCT:  V_n = (a_n - i a_{L-n}) exp(i pi n/2L) (a_L = 0); v = IFFT(V) (unnormalised);
//          y = makhoul^-1(v)
//   IDXST: IDXST(a)_k = (-1)^k/2 * IDCT(b)_k with b_0 = 0, b_m = a_{L-m}
#pragma once
#include <cstdint>
#include "fft.cuh"
#include "geometry.cuh"

namespace epb {

constexpr int kFftThreads = 256;
constexpr unsigned kFlagNonFinite = 0x1u;
constexpr unsigned kFlagSaturated = 0x2u;

// ---------------------------------------------------------------------------
// Scatter
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
k_scatter(CellView c, GridGeom g, float qscale, unsigned long long* __restrict__ grid,
          unsigned* __restrict__ flags) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < c.n; i += stride) {
        Footprint f;
        const int st = cell_footprint(c, g, cell_node(c, i), f);
        if (st < 0) { atomicOr(flags, kFlagNonFinite); continue; }
        if (st == 0) continue;
        for (int kx = f.kx0; kx <= f.kx1; ++kx) {
            const float oxr = __fmul_rn(bin_overlap(f.x, f.ex, g.xl, g.bsx, kx), f.r);
            if (oxr == 0.0f) continue;
            unsigned long long* row = grid + (int64_t)kx * g.N;
            for (int ky = f.ky0; ky <= f.ky1; ++ky) {
                const float a = __fmul_rn(oxr, bin_overlap(f.y, f.ey, g.yl, g.bsy, ky));
                const long long q = __float2ll_rn(__fmul_rn(a, qscale));
                if (q != 0) atomicAdd(row + ky, (unsigned long long)q);
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Pass 1: conversion + forward DCT along y (rows)
// S sequences of length L = N per CTA -> 2S rows.
// ---------------------------------------------------------------------------
template <int L>
struct RowFwdCfg {
    static constexpr int S = (4096 / L) > 0 ? 4096 / L : 1;
    static constexpr int ROWS = 2 * S;
    static constexpr size_t SMEM = (size_t)S * L * sizeof(float2);
};

template <int L, bool FROM_FIXED>
__global__ void __launch_bounds__(kFftThreads)
k_row_fwd(long long* __restrict__ qgrid,            // FROM_FIXED: [M][L] int64 (zeroed after read)
          const float* __restrict__ rho_in,         // !FROM_FIXED: [M][L] fp32
          const float* __restrict__ init,           // nullable [M][L]
          double dscale, int M,
          float* __restrict__ rho_out,              // nullable
          float* __restrict__ t1,                   // [M][L]
          const float2* __restrict__ tw, const float2* __restrict__ qw,
          unsigned* __restrict__ flags) {
    using C = RowFwdCfg<L>;
    constexpr int S = C::S, T = kFftThreads;
    extern __shared__ float2 sm_rowfwd[];
    float2* buf = sm_rowfwd;
    const int row0 = blockIdx.x * C::ROWS;
    unsigned sat = 0;
    // load: element m of row (row0 + 2s + p) goes to buf[s][makhoul_pos(m)], real (p=0) or imag (p=1)
    for (int e = threadIdx.x; e < S * L; e += T) {
        const int s = e / L, m = e % L;
        float vals[2];
#pragma unroll
        for (int p = 0; p < 2; ++p) {
            const int row = row0 + 2 * s + p;
            float v = 0.0f;
            if (row < M) {
                const int64_t off = (int64_t)row * L + m;
                if (FROM_FIXED) {
                    long long q = qgrid[off];
                    qgrid[off] = 0;  // leave the grid zeroed for the next scatter
                    if (q < 0 || q >= (1ll << 62)) sat = 1;
                    v = __double2float_rn(__dmul_rn(__ll2double_rn(q), dscale));
                    if (init) v = __fadd_rn(v, __ldg(init + off));
                } else {
                    v = __ldg(rho_in + off);
                }
                if (rho_out) rho_out[off] = v;
            }
            vals[p] = v;
        }
        buf[s * L + makhoul_pos(m, L)] = make_float2(vals[0], vals[1]);
    }
    if (FROM_FIXED && sat) atomicOr(flags, kFlagSaturated);
    __syncthreads();
    fft_smem<L, S, T, false>(buf, tw);
    const float scale = 2.0f / (float)L;
    for (int e = threadIdx.x; e < S * L; e += T) {
        const int s = e / L, k = e % L;
        const float2 Z = buf[s * L + k];
        const float2 Zr = buf[s * L + ((L - k) & (L - 1))];
        // Va = (Z + conj(Zr))/2 ; Vb = -i (Z - conj(Zr))/2
        const float2 Va = make_float2(0.5f * (Z.x + Zr.x), 0.5f * (Z.y - Zr.y));
        const float2 Vb = make_float2(0.5f * (Z.y + Zr.y), -0.5f * (Z.x - Zr.x));
        const float2 q = __ldg(qw + k);  // (cos, sin)(pi k / 2L)
        const int ra = row0 + 2 * s;
        if (ra < M) t1[(int64_t)ra * L + k] = scale * (Va.x * q.x + Va.y * q.y);
        if (ra + 1 < M) t1[(int64_t)(ra + 1) * L + k] = scale * (Vb.x * q.x + Vb.y * q.y);
    }
}

// ---------------------------------------------------------------------------
// Pass 2: along x (columns).  S sequences of length L = M per CTA -> W = 2S columns.
// ---------------------------------------------------------------------------
template <int L>
struct ColCfg {
    static constexpr int S = (4096 / L) > 2 ? 4096 / L : 2;
    static constexpr int W = 2 * S;
    static constexpr size_t SMEM = (size_t)S * L * sizeof(float2) + (size_t)W * L * sizeof(float);
};

struct ColArgs {
    const float* t1;        // [M][N]
    float* gx;              // [M][N] (2 IDXST_M)(auv*wu)
    float* gy;              // [M][N] (2 IDCT_M)(auv*wv)
    float* gp;              // [M][N] IDCT_M(auv*inv)   (only when want_phi)
    const float* wu;        // [M] 2 pi u / M
    const float* wv;        // [N] 2 pi v / N * bsx/bsy
    const float2* tw;       // FFT twiddles, length M
    const float2* qw;       // quarter-wave table, length M
    double* partials;       // [gridDim.x] energy partial sums
    unsigned* counter;      // last-block counter (wraps to 0)
    double* energy_d;       // device double energy
    float* energy_out;      // nullable caller scalar
    int N;
    int want_phi;
    double energy_scale;    // M*N/4
};

__device__ __forceinline__ void spectral_weights(float wu, float wv, float& wuh, float& wvh, float& inv) {
    const float d = wu * wu + wv * wv;
    if (d == 0.0f) { wuh = wvh = inv = 0.0f; return; }
    inv = 1.0f / d;
    wuh = wu * inv * 0.5f;
    wvh = wv * inv * 0.5f;
}

template <int L>
__global__ void __launch_bounds__(kFftThreads)
k_col(ColArgs a) {
    using C = ColCfg<L>;
    constexpr int S = C::S, W = C::W, T = kFftThreads;
    extern __shared__ float2 sm_col[];
    float2* buf = sm_col;                                  // S x L complex
    float* auv = reinterpret_cast<float*>(sm_col + S * L); // W x L real (column-major per column)
    const int N = a.N;
    const int c0 = blockIdx.x * W;

    // ---- load T1 strip [L rows][W cols], Makhoul reorder along rows ----
    for (int e = threadIdx.x; e < L * (W / 4); e += T) {
        const int m = e / (W / 4), q4 = e % (W / 4);
        const int col = c0 + 4 * q4;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (col < N) v = __ldg(reinterpret_cast<const float4*>(a.t1 + (int64_t)m * N + col));
        const int pos = makhoul_pos(m, L);
        const int s0 = 2 * q4;  // columns 4q4, 4q4+1 -> seq 2q4 ; 4q4+2, 4q4+3 -> seq 2q4+1
        buf[s0 * L + pos] = make_float2(v.x, v.y);
        buf[(s0 + 1) * L + pos] = make_float2(v.z, v.w);
    }
    __syncthreads();
    fft_smem<L, S, T, false>(buf, a.tw);

    // ---- auv + energy ----
    const float scale = 2.0f / (float)L;
    double esum = 0.0;
    for (int e = threadIdx.x; e < S * L; e += T) {
        const int s = e / L, u = e % L;
        const float2 Z = buf[s * L + u];
        const float2 Zr = buf[s * L + ((L - u) & (L - 1))];
        const float2 Va = make_float2(0.5f * (Z.x + Zr.x), 0.5f * (Z.y - Zr.y));
        const float2 Vb = make_float2(0.5f * (Z.y + Zr.y), -0.5f * (Z.x - Zr.x));
        const float2 q = __ldg(a.qw + u);
        const float xa = scale * (Va.x * q.x + Va.y * q.y);
        const float xb = scale * (Vb.x * q.x + Vb.y * q.y);
        auv[(2 * s) * L + u] = xa;
        auv[(2 * s + 1) * L + u] = xb;
        const float wu = __ldg(a.wu + u);
        const double cu = u == 0 ? 1.0 : 2.0;
#pragma unroll
        for (int p = 0; p < 2; ++p) {
            const int col = c0 + 2 * s + p;
            if (col < N) {
                const float wv = __ldg(a.wv + col);
                float wuh, wvh, inv;
                spectral_weights(wu, wv, wuh, wvh, inv);
                const double x = p ? xb : xa;
                esum += cu * (col == 0 ? 1.0 : 2.0) * (double)inv * x * x;
            }
        }
    }
    __syncthreads();

    // ---- three inverse transforms along x: 0 -> gx (IDXST form), 1 -> gy, 2 -> gp ----
    const int rounds = a.want_phi ? 3 : 2;
    for (int r = 0; r < rounds; ++r) {
        // build V for seq s = columns (2s, 2s+1)
        for (int e = threadIdx.x; e < S * L; e += T) {
            const int s = e / L, n = e % L;
            float An[2], Am[2];  // A_n and A_{L-n} for the two packed columns
#pragma unroll
            for (int p = 0; p < 2; ++p) {
                const int cl = 2 * s + p;
                const int col = c0 + cl;
                const float wv = col < N ? __ldg(a.wv + col) : 0.0f;
                const float* au = auv + cl * L;
                if (r == 0) {
                    // b_n = a_{L-n} (b_0 = 0), a_u = auv_u * wu_half
                    float wuh, wvh, inv;
                    if (n == 0) {
                        An[p] = 0.0f;
                        Am[p] = 0.0f;  // b_L = 0 by definition
                    } else {
                        spectral_weights(__ldg(a.wu + (L - n)), wv, wuh, wvh, inv);
                        An[p] = au[L - n] * wuh;
                        spectral_weights(__ldg(a.wu + n), wv, wuh, wvh, inv);
                        Am[p] = au[n] * wuh;
                    }
                } else {
                    float wuh, wvh, inv;
                    spectral_weights(__ldg(a.wu + n), wv, wuh, wvh, inv);
                    An[p] = au[n] * (r == 1 ? 2.0f * wvh : inv);
                    if (n == 0) {
                        Am[p] = 0.0f;
                    } else {
                        spectral_weights(__ldg(a.wu + (L - n)), wv, wuh, wvh, inv);
                        Am[p] = au[L - n] * (r == 1 ? 2.0f * wvh : inv);
                    }
                }
            }
            // V = (A_n - i A_{L-n}) e^{i pi n / 2L} for each column; pack col p=1 as imaginary
            const float2 q = __ldg(a.qw + n);
            const float2 va = make_float2(An[0] * q.x + Am[0] * q.y, An[0] * q.y - Am[0] * q.x);
            const float2 vb = make_float2(An[1] * q.x + Am[1] * q.y, An[1] * q.y - Am[1] * q.x);
            buf[s * L + n] = make_float2(va.x - vb.y, va.y + vb.x);
        }
        __syncthreads();
        fft_smem<L, S, T, true>(buf, a.tw);
        float* out = r == 0 ? a.gx : (r == 1 ? a.gy : a.gp);
        for (int e = threadIdx.x; e < L * (W / 4); e += T) {
            const int k = e / (W / 4), q4 = e % (W / 4);
            const int col = c0 + 4 * q4;
            const int src = makhoul_pos(k, L);
            float2 v0 = buf[(2 * q4) * L + src];
            float2 v1 = buf[(2 * q4 + 1) * L + src];
            if (r == 0 && (k & 1)) { v0.x = -v0.x; v0.y = -v0.y; v1.x = -v1.x; v1.y = -v1.y; }
            if (col < N)
                *reinterpret_cast<float4*>(out + (int64_t)k * N + col) = make_float4(v0.x, v0.y, v1.x, v1.y);
        }
        __syncthreads();
    }

    // ---- deterministic energy reduction: block partial, last block sums in order ----
    double* red = reinterpret_cast<double*>(sm_col);
    red[threadIdx.x] = esum;
    __syncthreads();
    for (int w = T / 2; w > 0; w >>= 1) {
        if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
        __syncthreads();
    }
    __shared__ bool is_last;
    if (threadIdx.x == 0) {
        a.partials[blockIdx.x] = red[0];
        __threadfence();
        const unsigned t = atomicInc(a.counter, gridDim.x - 1);
        is_last = (t == gridDim.x - 1);
    }
    __syncthreads();
    if (is_last) {
        __threadfence();
        double s = 0.0;
        for (int b = threadIdx.x; b < (int)gridDim.x; b += T) s += __ldcg(a.partials + b);
        red[threadIdx.x] = s;
        __syncthreads();
        for (int w = T / 2; w > 0; w >>= 1) {
            if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
            __syncthreads();
        }
        if (threadIdx.x == 0) {
            const double e = red[0] * a.energy_scale;
            *a.energy_d = e;
            if (a.energy_out) *a.energy_out = (float)e;
        }
    }
}

// ---------------------------------------------------------------------------
// Pass 3: inverse along y (rows).  ROWS rows per CTA; sequences:
//   2j   : fx row (IDCT of Gx) + i * fy row (IDXST of Gy) for row j (j < ROWS)
//   ...  : potential rows packed in pairs (IDCT of Gp)
// ---------------------------------------------------------------------------
template <int L>
struct RowInvCfg {
    static constexpr int ROWS = (2048 / L) > 1 ? 2 * (2048 / L) : 2;
    static constexpr int S = ROWS + ROWS / 2;
    static constexpr size_t SMEM = (size_t)S * L * sizeof(float2);
};

struct RowInvArgs {
    const float* gx; const float* gy; const float* gp;  // [M][N]
    float* fx; float* fy; float* phi;                   // nullable outputs
    float2* fxy;                                        // interleaved fields [M][N]
    const float2* tw; const float2* qw;                 // length N
    int M;
    int want_phi;
};

template <int L>
__global__ void __launch_bounds__(kFftThreads)
k_row_inv(RowInvArgs a) {
    using C = RowInvCfg<L>;
    constexpr int S = C::S, ROWS = C::ROWS, T = kFftThreads;
    extern __shared__ float2 sm_rowinv[];
    float2* buf = sm_rowinv;
    const int row0 = blockIdx.x * ROWS;
    for (int e = threadIdx.x; e < S * L; e += T) {
        const int s = e / L, n = e % L;
        float An[2], Am[2];
        bool valid = true;
        if (s < ROWS) {
            const int row = row0 + s;
            valid = row < a.M;
            if (valid) {
                const float* gxr = a.gx + (int64_t)row * L;
                const float* gyr = a.gy + (int64_t)row * L;
                An[0] = __ldg(gxr + n);
                Am[0] = n == 0 ? 0.0f : __ldg(gxr + (L - n));
                // IDXST: b_0 = 0, b_m = a_{L-m}; the 1/2 factor folded in
                An[1] = n == 0 ? 0.0f : 0.5f * __ldg(gyr + (L - n));
                Am[1] = n == 0 ? 0.0f : 0.5f * __ldg(gyr + n);
            }
        } else {
            const int row = row0 + 2 * (s - ROWS);
            valid = a.want_phi && row < a.M;
            if (valid) {
#pragma unroll
                for (int p = 0; p < 2; ++p) {
                    const float* gpr = a.gp + (int64_t)(row + p) * L;
                    const bool ok = row + p < a.M;
                    An[p] = ok ? __ldg(gpr + n) : 0.0f;
                    Am[p] = (ok && n != 0) ? __ldg(gpr + (L - n)) : 0.0f;
                }
            }
        }
        if (!valid) { An[0] = An[1] = Am[0] = Am[1] = 0.0f; }
        const float2 q = __ldg(a.qw + n);
        const float2 va = make_float2(An[0] * q.x + Am[0] * q.y, An[0] * q.y - Am[0] * q.x);
        const float2 vb = make_float2(An[1] * q.x + Am[1] * q.y, An[1] * q.y - Am[1] * q.x);
        buf[s * L + n] = make_float2(va.x - vb.y, va.y + vb.x);
    }
    __syncthreads();
    fft_smem<L, S, T, true>(buf, a.tw);
    for (int e = threadIdx.x; e < S * L; e += T) {
        const int s = e / L, l = e % L;
        const float2 v = buf[s * L + makhoul_pos(l, L)];
        if (s < ROWS) {
            const int row = row0 + s;
            if (row < a.M) {
                const int64_t off = (int64_t)row * L + l;
                const float fx = v.x;
                const float fy = (l & 1) ? -v.y : v.y;
                a.fxy[off] = make_float2(fx, fy);
                if (a.fx) a.fx[off] = fx;
                if (a.fy) a.fy[off] = fy;
            }
        } else if (a.want_phi && a.phi) {
            const int row = row0 + 2 * (s - ROWS);
            if (row < a.M) a.phi[(int64_t)row * L + l] = v.x;
            if (row + 1 < a.M) a.phi[(int64_t)(row + 1) * L + l] = v.y;
        }
    }
}

// ---------------------------------------------------------------------------
// Gather: grad[node] = -g * ratio * sum (ox*oy) * field
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
k_gather(CellView c, GridGeom g, const float2* __restrict__ fxy,
         const float* __restrict__ fx, const float* __restrict__ fy,  // planar alternative when fxy == nullptr
         const float* __restrict__ grad_out, float* __restrict__ grad_x, float* __restrict__ grad_y,
         unsigned* __restrict__ flags) {
    const float gscale = grad_out ? -__ldg(grad_out) : -1.0f;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < c.n; i += stride) {
        const int64_t node = cell_node(c, i);
        Footprint f;
        const int st = cell_footprint(c, g, node, f);
        float ax = 0.0f, ay = 0.0f, r = 0.0f;
        if (st < 0) atomicOr(flags, kFlagNonFinite);
        if (st > 0) {
            r = f.r;
            for (int kx = f.kx0; kx <= f.kx1; ++kx) {
                const float ox = bin_overlap(f.x, f.ex, g.xl, g.bsx, kx);
                const int64_t rowoff = (int64_t)kx * g.N;
                for (int ky = f.ky0; ky <= f.ky1; ++ky) {
                    const float w = ox * bin_overlap(f.y, f.ey, g.yl, g.bsy, ky);
                    float2 fv;
                    if (fxy) fv = __ldg(fxy + rowoff + ky);
                    else fv = make_float2(__ldg(fx + rowoff + ky), __ldg(fy + rowoff + ky));
                    ax = fmaf(w, fv.x, ax);
                    ay = fmaf(w, fv.y, ay);
                }
            }
        }
        const float s = gscale * r;
        grad_x[node] = s * ax;
        grad_y[node] = s * ay;
    }
}

}  // namespace epb
