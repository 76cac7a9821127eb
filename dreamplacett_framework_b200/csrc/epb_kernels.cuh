// epb_kernels.cuh -- CUDA kernels of the electric-potential step.
//
//   k_scatter      cells -> int64 fixed-point density grid (atomic adds to L2)
//   k_row_fwd<L>   grid (or fp32 density) -> normalised density rho (+ initial
//                  density), then DCT-II along y of every row       -> T1
//   k_col<L>       DCT-II along x of T1 columns -> auv; spectral energy;
//                  weights wu/wv/inv; inverse transforms along x     -> Gx, Gp
//   k_row_inv<L>   inverse transforms along y of Gx, wv * Gp, Gp rows -> field_x,
//                  field_y, potential (+ interleaved field map for the gather)
//   k_gather       cells + interleaved fields -> per-node gradient
//
// Grid layout: [M rows = x bins][N columns = y bins], row-major, index bx*N+by
// (the reference's density layout, host/density_scatter_ttnn_server_host.cpp:458-459).
//
// Sharding: with P GPUs, GPU p owns the row band [p*M/P, (p+1)*M/P) and, for the
// column pass, the column band [p*N/P, (p+1)*N/P).  The kernels take the band
// and the layouts of the exchanged buffers as arguments; P = 1 is the
// single-GPU case of the same code.  Exchanged layouts (NB = N/P, RB = M/P):
//   T1 (row pass -> column pass): block q (destination) = rows of my band, columns of
//       band q: t1[q][r][c], r < RB, c < NB; after the all-to-all GPU q holds its
//       column strip as [M][NB] (source bands stacked in row order).
//   G (column pass -> row pass): g[d][o][s][r][w]: destination band d, output o
//       (0 = field_x form, 1 = potential form), column strip s of SW columns, band
//       row r, column w in the strip (local column c = s*SW + w).
//       Strip-major so every column-pass CTA writes whole contiguous blocks; after
//       the all-to-all GPU d holds g[q][o][s][r][w] from each source q.
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
#include <cuda_fp16.h>
#include "fft.cuh"
#include "geometry.cuh"

namespace epb {

constexpr unsigned kFlagNonFinite = 0x1u;
constexpr unsigned kFlagSaturated = 0x2u;
constexpr unsigned kFlagHalo = 0x4u;       // a gathered footprint reached past the field halo
constexpr unsigned kFlagTimeout = 0x8u;    // a wait for another GPU's signal gave up
constexpr int kMaxShards = 8;
// Outputs of the column pass per bin: the field_x form (IDXST_M of b*wu) and the
// potential form (IDCT_M of b).  The field_y form IDCT_M(b*wv) is not a third
// transform: wv depends on the column only, so it equals wv * IDCT_M(b), and the
// row pass applies wv when it loads the potential form.
constexpr int kColOutputs = 2;
// Minimum strip width (columns) of the exchanged column-pass layout.  The row
// pass reads a row as one run of kStripWidth floats per strip; the column pass
// writes its W columns of a strip row as one 16-byte piece.
#ifndef EPB_STRIP_WIDTH
#define EPB_STRIP_WIDTH 8
#endif
constexpr int kStripWidth = EPB_STRIP_WIDTH;

// Destination of each column block / row band of an exchanged buffer: this
// GPU's send buffer (NCCL transport) or the peer's receive buffer mapped over
// NVLink (peer transport).
struct DstTable {
    float* p[kMaxShards];
};

// Cell kernels: footprints at most kOyCache bins wide compute their column
// overlaps once per cell (compile-time knob EPB_OY_CACHE).
constexpr int kOyCache = 4;
#ifndef EPB_OY_CACHE
#define EPB_OY_CACHE 1
#endif

// Register caps of the cell kernels (0 = no bound).
#ifndef EPB_SCATTER_MINB
#define EPB_SCATTER_MINB 0
#endif
#ifndef EPB_SEL_SCATTER_SPLIT
#define EPB_SEL_SCATTER_SPLIT 8  // shard scatter: CTAs per band-list segment times the shard count
#endif
#ifndef EPB_GATHER_WAVES
#define EPB_GATHER_WAVES 1   // whole-grid gather launch: waves of resident CTAs
#endif
#ifndef EPB_GATHER_MINB
#define EPB_GATHER_MINB 5
#endif
#if EPB_SCATTER_MINB > 0
#define EPB_SCATTER_BOUNDS __launch_bounds__(256, EPB_SCATTER_MINB)
#else
#define EPB_SCATTER_BOUNDS __launch_bounds__(256)
#endif
#if EPB_GATHER_MINB > 0
#define EPB_GATHER_BOUNDS __launch_bounds__(256, EPB_GATHER_MINB)
#else
#define EPB_GATHER_BOUNDS __launch_bounds__(256)
#endif
// ---------------------------------------------------------------------------
// Scatter
// ---------------------------------------------------------------------------
// IO: c.x / c.y point into pinned host memory (read over PCIe) and every
// visited node's position is also stored to xcopy / ycopy in device memory.
// The fixed-point contributions of footprint f to rows [row0, row1) of the
// density grid (grid holds those rows): one 64-bit atomic add per bin.
__device__ __forceinline__ void deposit(const Footprint& f, const GridGeom& g, float qscale,
                                        unsigned long long* __restrict__ grid, int row0, int row1) {
    const int kxa = max(f.kx0, row0), kxb = min(f.kx1, row1 - 1);
    if (EPB_OY_CACHE && f.ky1 - f.ky0 < kOyCache) {
        // the column overlaps are the same for every row: computed once
        float oy[kOyCache];
#pragma unroll
        for (int j = 0; j < kOyCache; ++j)
            oy[j] = f.ky0 + j <= f.ky1 ? bin_overlap(f.y, f.ey, g.yl, g.bsy, f.ky0 + j) : 0.0f;
        for (int kx = kxa; kx <= kxb; ++kx) {
            const float oxr = __fmul_rn(bin_overlap(f.x, f.ex, g.xl, g.bsx, kx), f.r);
            if (oxr == 0.0f) continue;
            unsigned long long* row = grid + (int64_t)(kx - row0) * g.N + f.ky0;
#pragma unroll
            for (int j = 0; j < kOyCache; ++j) {
                if (f.ky0 + j > f.ky1) break;
                const long long q = __float2ll_rn(__fmul_rn(__fmul_rn(oxr, oy[j]), qscale));
                if (q != 0) atomicAdd(row + j, (unsigned long long)q);
            }
        }
        return;
    }
    for (int kx = kxa; kx <= kxb; ++kx) {
        const float oxr = __fmul_rn(bin_overlap(f.x, f.ex, g.xl, g.bsx, kx), f.r);
        if (oxr == 0.0f) continue;
        unsigned long long* row = grid + (int64_t)(kx - row0) * g.N;
        for (int ky = f.ky0; ky <= f.ky1; ++ky) {
            const float a = __fmul_rn(oxr, bin_overlap(f.y, f.ey, g.yl, g.bsy, ky));
            const long long q = __float2ll_rn(__fmul_rn(a, qscale));
            if (q != 0) atomicAdd(row + ky, (unsigned long long)q);
        }
    }
}

template <bool IO = false>
__global__ void EPB_SCATTER_BOUNDS
k_scatter(CellView c, GridGeom g, float qscale, unsigned long long* __restrict__ grid,
          int row0, int row1, unsigned* __restrict__ flags, float* __restrict__ xcopy = nullptr,
          float* __restrict__ ycopy = nullptr) {
    // grid holds rows [row0, row1) of the density grid; footprints are clipped to them.
    for_each_cell(c, [&](int64_t node) {
        if constexpr (IO) {
            xcopy[node] = __ldg(c.x + node);
            ycopy[node] = __ldg(c.y + node);
        }
        Footprint f;
        const int st = cell_footprint(c, g, node, f, row0, row1, false);
        if (st < 0) { atomicOr(flags, kFlagNonFinite); return; }
        if (st != 1) return;
        deposit(f, g, qscale, grid, row0, row1);
    });
}

// ---------------------------------------------------------------------------
// Pass 1: conversion + forward DCT along y (rows)
// S sequences of length L = N per CTA (two rows packed per sequence), P = L/16
// threads per sequence.
// ---------------------------------------------------------------------------
// Minimum resident CTAs per SM requested from the compiler (a register cap) for
// the three DCT passes; compile-time tuning knobs.  0 leaves the bound out:
// ptxas then picks its own register budget, which differs from an explicit 1.
#ifndef EPB_ROWFWD_MINB
#define EPB_ROWFWD_MINB 4
#endif
#ifndef EPB_COL_MINB
#define EPB_COL_MINB 2
#endif
#ifndef EPB_ROWINV_MINB
#define EPB_ROWINV_MINB 3
#endif
#if EPB_ROWFWD_MINB > 0
#define EPB_ROWFWD_BOUNDS(...) __launch_bounds__(__VA_ARGS__, EPB_ROWFWD_MINB)
#else
#define EPB_ROWFWD_BOUNDS(...) __launch_bounds__(__VA_ARGS__)
#endif

// HALF: half the sequences per CTA (at least one), for launches that would
// otherwise leave SMs idle (a shard's few rows or columns).
template <int L, bool HALF = false>
struct RowFwdCfg {
    static constexpr int P = L / 16;
    static constexpr int S0 = (4096 / L) > 0 ? 4096 / L : 1;
    static constexpr int S = HALF ? (S0 / 2 > 0 ? S0 / 2 : 1) : S0;
    static constexpr int T = P * S;
    static constexpr int ROWS = 2 * S;
    static constexpr int LP = Padded<L>::value;
    static constexpr size_t SMEM = (size_t)S * LP * sizeof(float2);
};

template <int L, bool FROM_FIXED, bool HALF = false>
__global__ void EPB_ROWFWD_BOUNDS(RowFwdCfg<L, HALF>::T)
k_row_fwd(long long* __restrict__ qgrid,            // FROM_FIXED: [M][L] int64 (zeroed after read)
          const float* __restrict__ rho_in,         // !FROM_FIXED: [M][L] fp32
          const float* __restrict__ init,           // nullable [M][L]
          double dscale, int M,
          float* __restrict__ rho_out,              // nullable
          const __grid_constant__ DstTable t1dst,   // column block q goes to t1dst.p[q][(drow0 + row) * nb + c]
          int lnb, int drow0,                       // log2 block width nb; first row of this band there
          const float2* __restrict__ tw, const float2* __restrict__ qw,
          unsigned* __restrict__ flags) {
    using C = RowFwdCfg<L, HALF>;
    constexpr int S = C::S, T = C::T, LP = C::LP, P = C::P;
    constexpr bool GS = GroupSync<L, S>::value;  // sequences run on their own barriers
    extern __shared__ float2 sm_rowfwd[];
    float2* buf = sm_rowfwd;
    const int row0 = blockIdx.x * C::ROWS;
    const int grp = threadIdx.x / P, lane = threadIdx.x % P;
    unsigned sat = 0;
    // element m of row (row0 + 2s + p) goes to sequence s at makhoul_pos(m), real (p=0) or imag (p=1);
    // with GS each group loads only its own sequence
    if constexpr (GS) {
        // a batch of U elements per thread: every load of the batch is issued
        // before any of them is used (no branch or store between them)
        constexpr int U = 4;
        static_assert((L / P) % U == 0, "whole batches");
        const int ra = row0 + 2 * grp;
        const bool ok0 = ra < M, ok1 = ra + 1 < M;
        const int64_t off0 = (int64_t)(ok0 ? ra : 0) * L, off1 = (int64_t)(ok1 ? ra + 1 : 0) * L;
        for (int m0 = lane; m0 < L; m0 += U * P) {
            float va[U], vb[U];
            if constexpr (FROM_FIXED) {
                long long qa[U], qb[U];
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    qa[u] = qgrid[off0 + m0 + u * P];
                    qb[u] = qgrid[off1 + m0 + u * P];
                }
                float ia[U], ib[U];
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    ia[u] = init ? __ldg(init + off0 + m0 + u * P) : 0.0f;
                    ib[u] = init ? __ldg(init + off1 + m0 + u * P) : 0.0f;
                }
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    if (qa[u] < 0 || qa[u] >= (1ll << 62) || qb[u] < 0 || qb[u] >= (1ll << 62)) sat = 1;
                    va[u] = __double2float_rn(__dmul_rn(__ll2double_rn(qa[u]), dscale));
                    vb[u] = __double2float_rn(__dmul_rn(__ll2double_rn(qb[u]), dscale));
                    if (init) { va[u] = __fadd_rn(va[u], ia[u]); vb[u] = __fadd_rn(vb[u], ib[u]); }
                }
            } else {
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    va[u] = __ldg(rho_in + off0 + m0 + u * P);
                    vb[u] = __ldg(rho_in + off1 + m0 + u * P);
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int m = m0 + u * P;
                if (!ok0) va[u] = 0.0f;
                if (!ok1) vb[u] = 0.0f;
                if (rho_out) {
                    if (ok0) rho_out[off0 + m] = va[u];
                    if (ok1) rho_out[off1 + m] = vb[u];
                }
                buf[grp * LP + pidx(makhoul_pos(m, L))] = make_float2(va[u], vb[u]);
            }
        }
    } else {
#pragma unroll 4
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
                    // the grid is re-zeroed after the FFT: a store right behind this
                    // load to the same address would stall the load pipeline
                    const long long q = qgrid[off];
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
        buf[s * LP + pidx(makhoul_pos(m, L))] = make_float2(vals[0], vals[1]);
    }
    }
    if (FROM_FIXED && sat) atomicOr(flags, kFlagSaturated);
    seq_sync<P, GS>(grp);
    fft_seq<L, false, GS>(buf + grp * LP, lane, tw, true, grp);
    const float scale = 2.0f / (float)L;
#pragma unroll 4
    for (int e = GS ? lane : threadIdx.x; e < (GS ? L : S * L); e += (GS ? P : T)) {
        const int s = GS ? grp : e / L, k = GS ? e : e % L;
        const float2 Z = buf[s * LP + pidx(k)];
        const float2 Zr = buf[s * LP + pidx((L - k) & (L - 1))];
        // Va = (Z + conj(Zr))/2 ; Vb = -i (Z - conj(Zr))/2
        const float2 Va = make_float2(0.5f * (Z.x + Zr.x), 0.5f * (Z.y - Zr.y));
        const float2 Vb = make_float2(0.5f * (Z.y + Zr.y), -0.5f * (Z.x - Zr.x));
        const float2 q = __ldg(qw + k);  // (cos, sin)(pi k / 2L)
        const int ra = row0 + 2 * s;
        const int nb = 1 << lnb;
        float* tb = t1dst.p[k >> lnb] + (int64_t)drow0 * nb + (k & (nb - 1));
        if (ra < M) tb[(int64_t)ra * nb] = scale * (Va.x * q.x + Va.y * q.y);
        if (ra + 1 < M) tb[(int64_t)(ra + 1) * nb] = scale * (Vb.x * q.x + Vb.y * q.y);
    }
    if (FROM_FIXED) {
        // leave the rows this CTA (GS: this group) read zeroed for the next scatter
        const int r0 = GS ? row0 + 2 * grp : row0;
        const int nrows = min(GS ? 2 : C::ROWS, M - r0);
        longlong2* g2 = reinterpret_cast<longlong2*>(qgrid + (int64_t)r0 * L);
        for (int e = GS ? lane : threadIdx.x; e < nrows * L / 2; e += (GS ? P : T)) g2[e] = make_longlong2(0ll, 0ll);
    }
}

// ---------------------------------------------------------------------------
// Pass 2: along x (columns).  S sequences of length L = M per CTA -> W = 2S columns.
// ---------------------------------------------------------------------------
template <int L, bool HALF = false>
struct ColCfg {
    static constexpr int P = L / 16;
    static constexpr int S0 = (4096 / L) > 2 ? 4096 / L : 2;
    static constexpr int S = HALF ? S0 / 2 : S0;
    static constexpr int T = P * S;
    static constexpr int W = 2 * S;
    static constexpr int LP = Padded<L>::value;
    // S forward sequences (column pairs), then W = 2S inverse sequences (one per column)
    static constexpr size_t SMEM = (size_t)W * LP * sizeof(float2);
    // the register cap applies to the 256-thread configurations (L <= 2048)
    static constexpr int MINB = T <= 256 ? EPB_COL_MINB : 1;
};

struct ColArgs {
    const float* t1;        // column strip [M][N] (N = local strip width, the row stride)
    DstTable g;             // outputs for destination band d at g.p[d][o*ostride + (c>>lsw)*(RB<<lsw) + r*SW + (c&(SW-1))]:
                            //   o = 0 (2 IDXST_M)(auv*wu_half), 1 IDCT_M(auv*inv)
    int64_t ostride;        // elements between outputs o
    int lrb;                // log2 rows per destination band (RB)
    int lsw;                // log2 strip width SW of the output layout
    int col_base;           // global index of local column 0
    float ku;               // wu = u * ku,  ku = 2 pi / M
    float kv;               // wv = v * kv,  kv = 2 pi / N * bsx / bsy
    const float2* tw;       // per-pass FFT twiddle table of length-M transforms (fft.cuh)
    const float2* qw;       // quarter-wave table, length M
    double* partials;       // [gridDim.x] energy partial sums
    unsigned* counter;      // last-block counter (wraps to 0)
    double* energy_d;       // device double energy
    float* energy_out;      // nullable caller scalar
    int N;
    double energy_scale;    // M*N/4
};

// Eigenvalue weights (host/density_scatter_ttnn_server_host.cpp:252-263 and
// DREAMPlace's inv_wu2_plus_wv2): with inv = 1/(wu^2+wv^2) (0 at (0,0)) and
// b = auv * inv, the reference's wu/(wu^2+wv^2)/2 weight is applied in the
// column pass as b*wu/2 (the field chain's left factor 2 folded into the
// IDXST), and its wv/(wu^2+wv^2)/2 weight in the row pass: (2 IDCT_M)(b*wv/2)
// = wv * IDCT_M(b) because wv is constant along a column.

// Sum over a warp in a fixed order (lane 0 receives the total).
__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
    return v;
}

// V_n = (A_n - i A_{L-n}) e^{i pi n / 2L} of two packed real sequences (p=0 real, p=1 imaginary)
__device__ __forceinline__ float2 idct_pre(float an0, float am0, float an1, float am1, float2 q) {
    const float2 va = make_float2(an0 * q.x + am0 * q.y, an0 * q.y - am0 * q.x);
    const float2 vb = make_float2(an1 * q.x + am1 * q.y, an1 * q.y - am1 * q.x);
    return make_float2(va.x - vb.y, va.y + vb.x);
}

template <int L, bool HALF = false>
__global__ void __launch_bounds__(ColCfg<L, HALF>::T, ColCfg<L, HALF>::MINB)
k_col(const __grid_constant__ ColArgs a) {
    using C = ColCfg<L, HALF>;
    constexpr int S = C::S, W = C::W, T = C::T, LP = C::LP, P = C::P;
    // CTA-wide phases: the strip's float4 loads and stores span both sequences of a CTA
    constexpr bool GS = false;
    extern __shared__ float2 sm_col[];
    // W x LP complex.  Forward: sequence s < S holds columns (2s, 2s+1) as real and
    // imaginary parts.  Inverse: sequence r*S + s holds output r of the same two
    // columns (r = 0 the field_x form, r = 1 the potential form; the two forms
    // differ in scale by up to ~1/wu, so each sequence packs one form), and
    // output 0 takes over forward sequence s in place.
    float2* buf = sm_col;
    const int N = a.N;
    const int c0 = blockIdx.x * W;
    const int grp = threadIdx.x / P;
    const int lane = threadIdx.x % P;

    // ---- load T1 strip [L rows][W cols], Makhoul reorder along rows; four columns
    //      (two sequences) per load, or two (one sequence) when W == 2 ----
    constexpr int VW = W >= 4 ? 4 : 2;
#pragma unroll 4
    for (int e = threadIdx.x; e < L * (W / VW); e += T) {
        const int m = e / (W / VW), qv = e % (W / VW);
        const int col = c0 + VW * qv;
        const int pos = pidx(makhoul_pos(m, L));
        // read once per launch: keep it out of L1, which serves the twiddle table
        if constexpr (VW == 4) {
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (col < N) v = __ldcg(reinterpret_cast<const float4*>(a.t1 + (int64_t)m * N + col));
            const int s0 = 2 * qv;  // columns 4qv, 4qv+1 -> seq 2qv ; 4qv+2, 4qv+3 -> seq 2qv+1
            buf[s0 * LP + pos] = make_float2(v.x, v.y);
            buf[(s0 + 1) * LP + pos] = make_float2(v.z, v.w);
        } else {
            float2 v = make_float2(0.f, 0.f);
            if (col < N) v = __ldcg(reinterpret_cast<const float2*>(a.t1 + (int64_t)m * N + col));
            buf[qv * LP + pos] = v;
        }
    }
    seq_sync<P, GS>(grp);
    fft_seq<L, false, GS>(buf + grp * LP, lane, a.tw, true, grp);

    // ---- auv, b = auv / (wu^2 + wv^2), energy, and the inverse inputs ----
    // One iteration handles the index pair (u, L-u) of one sequence (u = 0 handles
    // the self-paired 0 and L/2): for two real columns packed as one FFT Z,
    //   Va_u = (Z_u + conj(Z_{L-u}))/2,  Vb_u = -i (Z_u - conj(Z_{L-u}))/2,
    // Va_{L-u} = conj(Va_u), Vb_{L-u} = conj(Vb_u), and the quarter-wave factor of
    // L-u is that of u with cos and sin swapped.  The inverse inputs at n need b at
    // n and L-n, so the same iteration writes V_u and V_{L-u} of both outputs, at
    // the positions it read (no other iteration touches them).
    const float scale = 2.0f / (float)L;
    const float hku = 0.5f * a.ku;
    double esum = 0.0;
    for (int e = threadIdx.x; e < S * (L / 2); e += T) {
        const int s = e / (L / 2), u = e % (L / 2);
        const int u2 = u == 0 ? L / 2 : L - u;   // the second index of this iteration
        const float2 Z = buf[s * LP + pidx(u)];
        const float2 Zr = buf[s * LP + pidx(u == 0 ? 0 : L - u)];
        const float2 Zh = u == 0 ? buf[s * LP + pidx(L / 2)] : make_float2(0.0f, 0.0f);
        const float2 Va = make_float2(0.5f * (Z.x + Zr.x), 0.5f * (Z.y - Zr.y));
        const float2 Vb = make_float2(0.5f * (Z.y + Zr.y), -0.5f * (Z.x - Zr.x));
        const float2 q = __ldg(a.qw + u);
        const float2 q2 = __ldg(a.qw + u2);
        float x1[2], x2[2];  // [column p]: values at u and at u2
        x1[0] = scale * (Va.x * q.x + Va.y * q.y);
        x1[1] = scale * (Vb.x * q.x + Vb.y * q.y);
        if (u != 0) {
            x2[0] = scale * (Va.x * q.y - Va.y * q.x);
            x2[1] = scale * (Vb.x * q.y - Vb.y * q.x);
        } else {
            // index L/2 pairs with itself: Va = (Zh.x, 0), Vb = (Zh.y, 0)
            x2[0] = scale * (Zh.x * q2.x);
            x2[1] = scale * (Zh.y * q2.x);
        }
        const float wu1 = (float)u * a.ku, wu2 = (float)u2 * a.ku;
        const float cu1 = u == 0 ? 1.0f : 2.0f;
        float b1[2], b2[2];  // [column p]: b at u and at u2
#pragma unroll
        for (int p = 0; p < 2; ++p) {
            const int col = c0 + 2 * s + p;
            const int gcol = a.col_base + col;
            const float wv = (float)gcol * a.kv;
            const float wv2 = wv * wv;
            const float d1 = wu1 * wu1 + wv2, d2 = wu2 * wu2 + wv2;
            b1[p] = d1 == 0.0f ? 0.0f : __fdividef(x1[p], d1);
            b2[p] = __fdividef(x2[p], d2);
            // energy terms c_u c_v auv^2 / (wu^2 + wv^2), accumulated in fp64
            const float cv = gcol == 0 ? 1.0f : 2.0f;
            if (col < N) esum += (double)(cu1 * cv * (x1[p] * b1[p])) + (double)(2.0f * cv * (x2[p] * b2[p]));
        }
        // inverse inputs (Makhoul IDCT pre-twiddle of A_n, A_{L-n}, two columns packed):
        //   output 0, the IDXST form: IDCT of c_n = a_{L-n} with a_u = b_u * wu / 2 (c_0 = 0)
        //   output 1, the IDCT form: A_u = b_u (A_L = 0)
        float2* v0s = buf + s * LP;
        float2* v1s = buf + (S + s) * LP;
        if (u != 0) {
            float an[2], am[2];
#pragma unroll
            for (int p = 0; p < 2; ++p) {
                an[p] = b2[p] * ((float)u2 * hku);
                am[p] = b1[p] * ((float)u * hku);
            }
            v0s[pidx(u)] = idct_pre(an[0], am[0], an[1], am[1], q);
            v0s[pidx(u2)] = idct_pre(am[0], an[0], am[1], an[1], q2);
            v1s[pidx(u)] = idct_pre(b1[0], b2[0], b1[1], b2[1], q);
            v1s[pidx(u2)] = idct_pre(b2[0], b1[0], b2[1], b1[1], q2);
        } else {
            // V_{L/2} = (A_{L/2} - i A_{L/2}) e^{i pi / 4}
            float h[2];
#pragma unroll
            for (int p = 0; p < 2; ++p) h[p] = b2[p] * ((float)(L / 2) * hku);
            v0s[pidx(0)] = idct_pre(0.0f, 0.0f, 0.0f, 0.0f, q);
            v0s[pidx(L / 2)] = idct_pre(h[0], h[0], h[1], h[1], q2);
            v1s[pidx(0)] = idct_pre(b1[0], 0.0f, b1[1], 0.0f, q);
            v1s[pidx(L / 2)] = idct_pre(b2[0], b2[0], b2[1], b2[1], q2);
        }
    }
    // ---- deterministic energy reduction, done before the inverse rounds so the
    //      fp64 partial is not live across them: warps, then the block in warp
    //      order; the last block to finish sums the block partials in order ----
    {
        __shared__ double wred[T / 32];
        __shared__ bool is_last;
        const double v = warp_sum(esum);
        if ((threadIdx.x & 31) == 0) wred[threadIdx.x >> 5] = v;
        __syncthreads();
        if (threadIdx.x == 0) {
            double bsum = 0.0;
            for (int w = 0; w < T / 32; ++w) bsum += wred[w];
            a.partials[blockIdx.x] = bsum;
            __threadfence();
            const unsigned t = atomicInc(a.counter, gridDim.x - 1);
            is_last = (t == gridDim.x - 1);
        }
        __syncthreads();
        if (is_last) {
            __threadfence();
            double tot = 0.0;
            for (int b = threadIdx.x; b < (int)gridDim.x; b += T) tot += __ldcg(a.partials + b);
            tot = warp_sum(tot);
            if ((threadIdx.x & 31) == 0) wred[threadIdx.x >> 5] = tot;
            __syncthreads();
            if (threadIdx.x == 0) {
                double e = 0.0;
                for (int w = 0; w < T / 32; ++w) e += wred[w];
                e *= a.energy_scale;
                *a.energy_d = e;
                if (a.energy_out) *a.energy_out = (float)e;
            }
        }
    }
    seq_sync<P, GS>(grp);

    // ---- inverse transforms along x: group g takes outputs 0 and 1 of its column pair ----
    fft_seq<L, true, GS>(buf + grp * LP, lane, a.tw, true, grp);
    fft_seq<L, true, GS>(buf + (S + grp) * LP, lane, a.tw, true, grp);
    const int rbm = (1 << a.lrb) - 1;
#pragma unroll 4
    for (int e = threadIdx.x; e < L * (W / VW); e += T) {
        const int k = e / (W / VW), qv = e % (W / VW);
        const int col = c0 + VW * qv;
        const int src = pidx(makhoul_pos(k, L));
        float* dst = a.g.p[k >> a.lrb] + ((int64_t)(col >> a.lsw) << (a.lrb + a.lsw)) +
                     ((int64_t)(k & rbm) << a.lsw) + (col & ((1 << a.lsw) - 1));
        if constexpr (VW == 4) {
            // columns 4qv .. 4qv+3: pairs 2qv and 2qv+1, outputs 0 and 1
            float2 g0 = buf[(2 * qv) * LP + src], g1 = buf[(2 * qv + 1) * LP + src];
            const float2 p0 = buf[(S + 2 * qv) * LP + src], p1 = buf[(S + 2 * qv + 1) * LP + src];
            // output 0: the IDXST, the IDCT of the reversed input with odd outputs negated
            if (k & 1) { g0.x = -g0.x; g0.y = -g0.y; g1.x = -g1.x; g1.y = -g1.y; }
            if (col < N) {
                *reinterpret_cast<float4*>(dst) = make_float4(g0.x, g0.y, g1.x, g1.y);
                *reinterpret_cast<float4*>(dst + a.ostride) = make_float4(p0.x, p0.y, p1.x, p1.y);
            }
        } else {
            float2 g0 = buf[qv * LP + src];
            const float2 p0 = buf[(S + qv) * LP + src];
            if (k & 1) { g0.x = -g0.x; g0.y = -g0.y; }
            if (col < N) {
                *reinterpret_cast<float2*>(dst) = g0;
                *reinterpret_cast<float2*>(dst + a.ostride) = p0;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Pass 3: inverse along y (rows).  ROWS rows per CTA; sequences:
//   j < ROWS : fx row j (IDCT of Gx) + i * fy row j (IDXST of wv * Gp)
//   then     : potential rows packed in pairs (IDCT of Gp)
// ---------------------------------------------------------------------------
template <int L>
struct RowInvCfg {
    static constexpr int P = L / 16;
    static constexpr int ROWS = (2048 / L) > 1 ? 2 * (2048 / L) : 2;
    static constexpr int S = ROWS + ROWS / 2;
    static constexpr int T = P * S;
    static constexpr int LP = Padded<L>::value;
    static constexpr size_t SMEM = (size_t)S * LP * sizeof(float2);
    static constexpr int MINB = T <= 384 ? EPB_ROWINV_MINB : 1;
};

struct RowInvArgs {
    const float* g;          // g[q][o][r][c] from every source band q (see the layout note at the top)
    float kv;                // wv = v * kv for global column v (as in the column pass)
    int64_t ostride;         // elements between outputs o
    int64_t qstride;         // elements between source bands q
    int lnb;                 // log2 columns per band (NB)
    int lsw;                 // log2 strip width of the layout
    int lrb;                 // log2 rows per band
    float* fx; float* fy; float* phi;                   // nullable outputs, [M][N] of this band
    float2* fxy;                                        // interleaved fields [M][N] of this band
    float2* halo_dst;        // nullable: the previous band's field halo (its rows RB..), peer memory
    int halo_rows;           // rows of this band that also go to halo_dst
    const float2* tw; const float2* qw;                 // per-pass FFT twiddles, quarter-wave table (N)
    int M;                   // rows in this band
    int want_phi;
};

template <int L>
__global__ void __launch_bounds__(RowInvCfg<L>::T, RowInvCfg<L>::MINB)
k_row_inv(RowInvArgs a) {
    using C = RowInvCfg<L>;
    constexpr int S = C::S, ROWS = C::ROWS, T = C::T, LP = C::LP, P = C::P;
    constexpr bool GS = GroupSync<L, S>::value;  // sequences run on their own barriers
    extern __shared__ float2 sm_rowinv[];
    float2* buf = sm_rowinv;
    const int row0 = blockIdx.x * ROWS;
    const int grp = threadIdx.x / P, lane = threadIdx.x % P;
    // ---- stage: outputs 0 and 1 of the CTA's rows, read once as float4 (strips are
    //      at least 8 columns wide and 16-byte aligned), stored contiguously as
    //      stage[(o * ROWS + j) * L + l] at the top of the sequence buffers ----
    constexpr int NST = 2 * ROWS * L;                 // staged floats
    static_assert(NST <= 2 * S * LP, "staging fits in the sequence buffers");
    float* stage = reinterpret_cast<float*>(buf) + (2 * S * LP - NST);
    {
        constexpr int NV = NST / 4, IT = (NV + T - 1) / T;
        float4 v[IT];
#pragma unroll
        for (int i = 0; i < IT; ++i) {
            const int e = threadIdx.x + i * T;
            v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (e < NV) {
                const int l = (e % (L / 4)) * 4, oj = e / (L / 4), o = oj / ROWS, j = oj % ROWS;
                const int row = row0 + j, c = l & ((1 << a.lnb) - 1);
                if (row < a.M)
                    v[i] = __ldg(reinterpret_cast<const float4*>(
                        a.g + (int64_t)(l >> a.lnb) * a.qstride + (int64_t)o * a.ostride +
                        ((int64_t)(c >> a.lsw) << (a.lrb + a.lsw)) + ((int64_t)row << a.lsw) +
                        (c & ((1 << a.lsw) - 1))));
            }
        }
#pragma unroll
        for (int i = 0; i < IT; ++i) {
            const int e = threadIdx.x + i * T;
            if (e < NV) reinterpret_cast<float4*>(stage)[e] = v[i];
        }
    }
    __syncthreads();
    // ---- build: item (k, n) makes V_n and V_{L-n} (n = 0: V_0 and V_{L/2}) of the
    //      sequences of rows 2k, 2k+1 (fx + i fy each) and of their potential pair.
    //      The staged values of all items are read first: the sequences overwrite them. ----
    {
        constexpr int H = L / 2, NI = (ROWS / 2) * H, IT = (NI + T - 1) / T;
        const float hkv = 0.5f * a.kv;
        // [item][row p of the pair]: output 0 at n, at L-n; output 1 at n, at L-n
        float x0n[IT][2], x0m[IT][2], x1n[IT][2], x1m[IT][2];
#pragma unroll
        for (int i = 0; i < IT; ++i) {
            const int e = threadIdx.x + i * T;
            const int k = e / H, n = e % H;
            const int m = n == 0 ? H : L - n;   // n = 0 pairs with L/2
#pragma unroll
            for (int p = 0; p < 2; ++p) {
                const float* s0 = stage + (2 * k + p) * L;            // output 0, row 2k + p
                const float* s1 = stage + (ROWS + 2 * k + p) * L;     // output 1, row 2k + p
                const bool ok = e < NI;
                x0n[i][p] = ok ? s0[n] : 0.f;
                x0m[i][p] = ok ? s0[m] : 0.f;
                x1n[i][p] = ok ? s1[n] : 0.f;
                x1m[i][p] = ok ? s1[m] : 0.f;
            }
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < IT; ++i) {
            const int e = threadIdx.x + i * T;
            if (e >= NI) break;
            const int k = e / H, n = e % H;
            const float2 qn = __ldg(a.qw + n);
            float2* sp = buf + (ROWS + k) * LP;   // potential rows 2k (real), 2k + 1 (imaginary)
            if (n != 0) {
                const int nm = L - n;
                const float2 qm = __ldg(a.qw + nm);
#pragma unroll
                for (int p = 0; p < 2; ++p) {
                    // fx: IDCT of the Gx row; fy: IDXST of the Gy row = IDCT of b (b_0 = 0,
                    // b_m = a_{L-m}) with the 1/2 folded in, Gy_l = wv_l * Gp_l
                    const float an1 = x1m[i][p] * ((float)nm * hkv), am1 = x1n[i][p] * ((float)n * hkv);
                    float2* sq = buf + (2 * k + p) * LP;
                    sq[pidx(n)] = idct_pre(x0n[i][p], x0m[i][p], an1, am1, qn);
                    sq[pidx(nm)] = idct_pre(x0m[i][p], x0n[i][p], am1, an1, qm);
                }
                sp[pidx(n)] = idct_pre(x1n[i][0], x1m[i][0], x1n[i][1], x1m[i][1], qn);
                sp[pidx(nm)] = idct_pre(x1m[i][0], x1n[i][0], x1m[i][1], x1n[i][1], qm);
            } else {
                // V_0 = A_0 (A_L = 0); V_{L/2} = (A_{L/2} - i A_{L/2}) e^{i pi / 4}
                const float2 qh = __ldg(a.qw + H);
#pragma unroll
                for (int p = 0; p < 2; ++p) {
                    float2* sq = buf + (2 * k + p) * LP;
                    sq[0] = idct_pre(x0n[i][p], 0.0f, 0.0f, 0.0f, qn);
                    const float hb = x1m[i][p] * ((float)H * hkv);
                    sq[pidx(H)] = idct_pre(x0m[i][p], x0m[i][p], hb, hb, qh);
                }
                sp[0] = idct_pre(x1n[i][0], 0.0f, x1n[i][1], 0.0f, qn);
                sp[pidx(H)] = idct_pre(x1m[i][0], x1m[i][0], x1m[i][1], x1m[i][1], qh);
            }
        }
    }
    __syncthreads();  // every thread wrote into every sequence
    fft_seq<L, true, GS>(buf + grp * LP, lane, a.tw, true, grp);
#pragma unroll 2
    for (int e = GS ? lane : threadIdx.x; e < (GS ? L : S * L); e += (GS ? P : T)) {
        const int s = GS ? grp : e / L, l = GS ? e : e % L;
        const float2 v = buf[s * LP + pidx(makhoul_pos(l, L))];
        if (s < ROWS) {
            const int row = row0 + s;
            if (row < a.M) {
                const int64_t off = (int64_t)row * L + l;
                const float fx = v.x;
                const float fy = (l & 1) ? -v.y : v.y;
                a.fxy[off] = make_float2(fx, fy);
                if (row < a.halo_rows) a.halo_dst[off] = make_float2(fx, fy);
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


// Atomic-rate probe: footprint i of fw x fh bins at a hashed bin of the grid,
// one 64-bit atomic add per bin with its result unused (the scatter's
// reduction, without its loads).
__global__ void __launch_bounds__(256)
k_atomic_probe(unsigned long long* __restrict__ grid, int M, int N, int64_t n, int fw, int fh) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    // a 32-bit integer hash of the footprint index (multiply-xorshift rounds)
    uint32_t h = (uint32_t)i * 0x9e3779b9u;
    h ^= h >> 16; h *= 0x85ebca6bu; h ^= h >> 13; h *= 0xc2b2ae35u; h ^= h >> 16;
    const uint32_t wx = (uint32_t)(M - fw + 1), wy = (uint32_t)(N - fh + 1);
    const int bx = (int)(h % wx);
    const int by = (int)((h / wx) % wy);
    for (int dx = 0; dx < fw; ++dx)
        for (int dy = 0; dy < fh; ++dy)
            atomicAdd(grid + (int64_t)(bx + dx) * N + (by + dy), 1ull);
}

// ---------------------------------------------------------------------------
// Band lists of a shard (cell order): the cells whose rows meet the band widened
// by kBandMargin rows on each side, kept across calls.  Each segment of
// kSelChunk cells keeps its listed cells in increasing order at
// sel[s * kSelChunk + j], j < cnt[s], and beside each the cell's static inputs
// (sizes, offsets, ratio) copied at list time, so the scatter and the gather
// read those contiguously and gather only the positions by node.
//
// Every forward, k_band_update checks each segment: when one of its unlisted
// cells now meets the band itself, that segment alone is listed again (a
// listed cell that has left the band costs a band test and nothing else).
// Segments are independent, so the check and the listing are one kernel with
// no grid-wide step.  The static inputs are read at list time: a caller that
// changes sizes, offsets or ratio in place between calls with the same arrays
// must hand in other arrays (or a new handle).
// ---------------------------------------------------------------------------
constexpr int kBandMargin = 8;

struct BandList {
    int* sel;               // [nseg * kSelChunk] cell indices, per segment
    int* cnt;               // [nseg]
    float4* geo;            // [nseg * kSelChunk] sx, sy, ox, oy of the listed cell (0 for absent offsets)
    float* r;               // [nseg * kSelChunk] ratio (1 when absent)
    unsigned char* listed;  // [n] 1 when the cell is in the list
    unsigned* ext;          // [n] the cell's cached x extent (band_extent)
};

// A cell's static x extent relative to its position, [x + lo, x + hi] with
// lo = offset and hi = offset + width, cached per cell as two half-precision
// values rounded outward (lo down, hi up), so the check reads 4 bytes instead
// of the offset and the width: the cached extent holds the cell's true extent.
// A non-positive width caches (-inf, +inf), a cell that may reach any band; a
// non-finite offset or width caches NaN, a cell that is flagged every check
// and never listed.
__device__ __forceinline__ unsigned band_extent(float ox, float sx) {
    __half lo, hi;
    if (!isfinite(ox) || !isfinite(sx)) {
        lo = hi = __ushort_as_half((unsigned short)0x7e00);   // NaN
    } else if (!(sx > 0.0f)) {
        lo = __ushort_as_half((unsigned short)0xfc00);        // -inf
        hi = __ushort_as_half((unsigned short)0x7c00);        // +inf
    } else {
        lo = __float2half_rd(ox);
        hi = __float2half_ru(__fadd_ru(ox, sx));
    }
    return (unsigned)__half_as_ushort(lo) | ((unsigned)__half_as_ushort(hi) << 16);
}

// Whether the cached extent at position x reaches the coordinates (lo_c, hi_c)
// of a band widened by some rows, or may start past the grid's last row: a
// superset of the cells whose bin rows meet the band (an edge band's outer side
// is open, as bins clamp cells beyond the die into the first and last rows),
// decided with two additions and compares instead of bin arithmetic.
__device__ __forceinline__ bool band_reaches(float x, unsigned ext, float lo_c, float hi_c, float last_c) {
    const float xlo = __fadd_rd(x, __half2float(__ushort_as_half((unsigned short)(ext & 0xffffu))));
    const float xhi = __fadd_ru(x, __half2float(__ushort_as_half((unsigned short)(ext >> 16))));
    return xlo >= last_c || (xlo < hi_c && xhi > lo_c);
}

// The coordinate of row k's lower edge, as bin_floor computes it.
__device__ __forceinline__ float row_edge(const GridGeom& g, int k) {
    return __fadd_rn(g.xl, __fmul_rn((float)k, g.bsx));
}

constexpr int kBandThreads = 512;   // threads of a k_band_update CTA (one segment per CTA)
static_assert(kSelChunk % kBandThreads == 0, "a band-list segment splits evenly over a CTA");

// CTA s checks segment s of the cells (kSelChunk / kBandThreads cells a thread, all
// their loads issued first) and lists the segment again when an unlisted cell
// reaches the band [row0, row1) widened by one row, or when force.  A listing
// takes the cells that reach the band widened by kBandMargin rows, so a cell
// must travel that far before it makes its segment list again.  With force the
// cached extents are made from the offsets and widths; otherwise only the
// positions, the cached extents and the list flags are read.  Cells with
// non-finite data are flagged (and never listed).
__global__ void __launch_bounds__(kBandThreads)
k_band_update(CellView c, GridGeom g, int row0, int row1, BandList b, int force, unsigned* __restrict__ flags) {
    constexpr int R = kSelChunk / kBandThreads;
    const int64_t seg0 = (int64_t)blockIdx.x * kSelChunk;
    float x[R];
    unsigned ext[R];
    unsigned char was[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int64_t i = seg0 + r * kBandThreads + threadIdx.x;
        x[r] = 0.0f;
        ext[r] = 0u;
        was[r] = 1;
        if (i < c.n) {
            const int64_t node = cell_node(c, i);
            was[r] = b.listed[i];
            x[r] = __ldg(c.x + node);
            if (force) {
                ext[r] = band_extent(c.ox ? __ldg(c.ox + node) : 0.0f, __ldg(c.sx + node));
                b.ext[i] = ext[r];
            } else {
                ext[r] = b.ext[i];
            }
        }
    }
    const float last_c = row_edge(g, g.M - 1);
    const float lo1 = row0 == 0 ? -INFINITY : row_edge(g, row0 - 1);
    const float hi1 = row1 >= g.M ? INFINITY : row_edge(g, row1 + 1);
    const float loM = row0 == 0 ? -INFINITY : row_edge(g, max(row0 - kBandMargin, 0));
    const float hiM = row1 >= g.M ? INFINITY : row_edge(g, min(row1 + kBandMargin, g.M));
    bool need = false, in[R];
    unsigned bad = 0;
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int64_t i = seg0 + r * kBandThreads + threadIdx.x;
        const bool nan_ext = (ext[r] & 0x7fffu) > 0x7c00u;     // the cached NaN of a bad offset or width
        const bool ok = i < c.n && isfinite(x[r]) && !nan_ext;
        bad |= (i < c.n && !ok) ? 1u : 0u;
        need |= ok && !was[r] && band_reaches(x[r], ext[r], lo1, hi1, last_c);
        in[r] = ok && band_reaches(x[r], ext[r], loM, hiM, last_c);
    }
    if (bad) atomicOr(flags, kFlagNonFinite);
    if (!__syncthreads_or(need || force)) return;
    // list the segment again
    __shared__ int wtot[kBandThreads / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int run = 0;
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int64_t i = seg0 + r * kBandThreads + threadIdx.x;
        if (i < c.n) b.listed[i] = in[r] ? 1 : 0;
        const unsigned m = __ballot_sync(0xffffffffu, in[r]);
        if (lane == 0) wtot[warp] = __popc(m);
        __syncthreads();
        int base = 0, tot = 0;
#pragma unroll
        for (int w = 0; w < kBandThreads / 32; ++w) {
            base += w < warp ? wtot[w] : 0;
            tot += wtot[w];
        }
        if (in[r]) {
            const int64_t node = cell_node(c, i);
            const int64_t slot = seg0 + run + base + __popc(m & ((1u << lane) - 1u));
            b.sel[slot] = (int)i;
            b.geo[slot] = make_float4(__ldg(c.sx + node), __ldg(c.sy + node), c.ox ? __ldg(c.ox + node) : 0.0f,
                                      c.oy ? __ldg(c.oy + node) : 0.0f);
            b.r[slot] = c.ratio ? __ldg(c.ratio + node) : 1.0f;
        }
        run += tot;
        __syncthreads();
    }
    if (threadIdx.x == 0) b.cnt[blockIdx.x] = run;
}

// A listed cell's inputs: the positions by node, the rest from its list slot.
__device__ __forceinline__ CellData listed_cell(const CellView& c, const BandList& b, int64_t slot, int64_t node) {
    CellData d;
    const float4 q = b.geo[slot];
    d.x = __ldg(c.x + node);
    d.y = __ldg(c.y + node);
    d.sx = q.x; d.sy = q.y; d.ox = q.z; d.oy = q.w;
    d.r = b.r[slot];
    return d;
}

// Scatter of a band's listed cells into rows [row0, row1) (grid holds them).
// G consecutive CTAs share a segment when the grid has G CTAs per segment.
__global__ void EPB_SCATTER_BOUNDS
k_scatter_listed(CellView c, GridGeom g, float qscale, unsigned long long* __restrict__ grid, int row0, int row1,
                 BandList b, unsigned* __restrict__ flags) {
    const int64_t nseg = (c.n + kSelChunk - 1) / kSelChunk;
    const int64_t G = gridDim.x >= nseg ? gridDim.x / nseg : 1;
    const int64_t slots = gridDim.x / G;
    if (blockIdx.x >= slots * G) return;
    const int sub = (int)(blockIdx.x % G);
    for (int64_t s = blockIdx.x / G; s < nseg; s += slots) {
        const int cnt = b.cnt[s];
        for (int j = sub * (int)blockDim.x + threadIdx.x; j < cnt; j += (int)(G * blockDim.x)) {
            const int64_t slot = s * kSelChunk + j;
            const CellData d = listed_cell(c, b, slot, cell_node(c, b.sel[slot]));
            Footprint f;
            const int st = footprint_of(c, g, d, f);
            if (st < 0) { atomicOr(flags, kFlagNonFinite); continue; }
            if (st != 1) continue;
            deposit(f, g, qscale, grid, row0, row1);
        }
    }
}

// ---------------------------------------------------------------------------
// Gather: grad[node] = -g * ratio * sum (ox*oy) * field
// ---------------------------------------------------------------------------
// The overlap-weighted field sums (ax, ay) of footprint f over field maps that
// hold rows [row0, row1 + halo); rows past them are dropped and flagged.
__device__ __forceinline__ void gather_sum(const Footprint& f, const GridGeom& g, const float2* __restrict__ fxy,
                                           const float* __restrict__ fx, const float* __restrict__ fy, int row0,
                                           int row1, int halo, unsigned* __restrict__ flags, float& ax, float& ay) {
    int kxb = f.kx1;
    if (kxb >= row1 + halo) {
        atomicOr(flags, kFlagHalo);
        kxb = row1 + halo - 1;
    }
    if (EPB_OY_CACHE && fxy && f.ky1 - f.ky0 < kOyCache) {
        // column overlaps computed once per cell; the same products in the same order
        float oy[kOyCache];
#pragma unroll
        for (int j = 0; j < kOyCache; ++j)
            oy[j] = f.ky0 + j <= f.ky1 ? bin_overlap(f.y, f.ey, g.yl, g.bsy, f.ky0 + j) : 0.0f;
        for (int kx = f.kx0; kx <= kxb; ++kx) {
            const float ox = bin_overlap(f.x, f.ex, g.xl, g.bsx, kx);
            const float2* rowp = fxy + (int64_t)(kx - row0) * g.N + f.ky0;
#pragma unroll
            for (int j = 0; j < kOyCache; ++j) {
                if (f.ky0 + j > f.ky1) break;
                const float w = ox * oy[j];
                const float2 fv = __ldg(rowp + j);
                ax = fmaf(w, fv.x, ax);
                ay = fmaf(w, fv.y, ay);
            }
        }
        return;
    }
    for (int kx = f.kx0; kx <= kxb; ++kx) {
        const float ox = bin_overlap(f.x, f.ex, g.xl, g.bsx, kx);
        const int64_t rowoff = (int64_t)(kx - row0) * g.N;
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

// IO: the gradients are also stored to host_gx / host_gy in pinned host memory
// (written over PCIe).
template <bool IO = false>
__global__ void EPB_GATHER_BOUNDS
k_gather(CellView c, GridGeom g, const float2* __restrict__ fxy,
         const float* __restrict__ fx, const float* __restrict__ fy,  // planar alternative when fxy == nullptr
         int row0, int row1, int halo, int owned_only,
         const float* __restrict__ grad_out, float* __restrict__ grad_x, float* __restrict__ grad_y,
         unsigned* __restrict__ flags, float* __restrict__ host_gx = nullptr, float* __restrict__ host_gy = nullptr) {
    // The field maps hold rows [row0, row1 + halo).  With owned_only, only cells
    // whose first bin row lies in [row0, row1) are computed and written; other
    // entries of grad_x / grad_y are left as they are.
    const float gscale = grad_out ? -__ldg(grad_out) : -1.0f;
    // per-cell accumulation over the footprint and the gradient stores
    auto finish = [&](int64_t node, int st, const Footprint& f) {
        float ax = 0.0f, ay = 0.0f, r = 0.0f;
        if (st < 0) atomicOr(flags, kFlagNonFinite);
        if (owned_only && st != 1) return;
        if (st == 1) {
            r = f.r;
            gather_sum(f, g, fxy, fx, fy, row0, row1, halo, flags, ax, ay);
        }
        const float s = gscale * r;
        grad_x[node] = s * ax;
        grad_y[node] = s * ay;
        if constexpr (IO) {
            host_gx[node] = s * ax;
            host_gy[node] = s * ay;
        }
    };
    if (row0 == 0 && row1 >= g.M) {
        // the whole grid: a footprint from loaded inputs, the next cell's loads in
        // flight while the current cell's fields are read (one round trip per cell,
        // not two)
        for_each_cell_prefetched(c, [&](int64_t node, const CellData& d) {
            Footprint f;
            finish(node, footprint_of(c, g, d, f), f);
        });
        return;
    }
    // a band without a selection: every cell is tested against it
    for_each_cell(c, [&](int64_t node) {
        Footprint f;
        const int st = cell_footprint(c, g, node, f, row0, row1, owned_only != 0);
        finish(node, st, f);
    });
}

// Gather of a band's own listed cells (first bin row in [row0, row1)) from
// field maps holding rows [row0, row1 + halo).  One CTA
// per segment, the next listed cell's inputs loaded while the current cell's
// fields are read.  Other entries of grad_x / grad_y are left as they are.
__global__ void EPB_GATHER_BOUNDS
k_gather_listed(CellView c, GridGeom g, const float2* __restrict__ fxy, int row0, int row1, int halo,
                const float* __restrict__ grad_out, float* __restrict__ grad_x, float* __restrict__ grad_y, BandList b,
                unsigned* __restrict__ flags) {
    const float gscale = grad_out ? -__ldg(grad_out) : -1.0f;
    const int64_t nseg = (c.n + kSelChunk - 1) / kSelChunk;
    for (int64_t s = blockIdx.x; s < nseg; s += gridDim.x) {
        const int cnt = b.cnt[s];
        int j = threadIdx.x;
        if (j >= cnt) continue;
        int64_t slot = s * kSelChunk + j;
        int64_t node = cell_node(c, b.sel[slot]);
        CellData cur = listed_cell(c, b, slot, node);
        for (;;) {
            const int jn = j + (int)blockDim.x;
            int64_t nslot = slot, nnode = node;
            CellData nxt = cur;
            if (jn < cnt) {
                nslot = s * kSelChunk + jn;
                nnode = cell_node(c, b.sel[nslot]);
                nxt = listed_cell(c, b, nslot, nnode);
            }
            Footprint f;
            const int st = footprint_of(c, g, cur, f);
            if (st < 0) {
                atomicOr(flags, kFlagNonFinite);
            } else if (st == 1 && f.kx0 >= row0 && f.kx0 < row1) {
                float ax = 0.0f, ay = 0.0f;
                gather_sum(f, g, fxy, nullptr, nullptr, row0, row1, halo, flags, ax, ay);
                const float sc = gscale * f.r;
                grad_x[node] = sc * ax;
                grad_y[node] = sc * ay;
            }
            if (jn >= cnt) break;
            j = jn;
            slot = nslot;
            node = nnode;
            cur = nxt;
        }
    }
}

// ---------------------------------------------------------------------------
// Cross-GPU ordering for the peer transport.  After a producer kernel has
// stored its blocks into the peers' buffers, k_signal publishes `epoch` in
// every peer's signal slot for (stage, this shard), optionally with this
// shard's energy partial.  k_wait (one thread) then waits until every shard
// has published `epoch` for the stage, with a bounded number of polls: when
// the limit is reached it sets kFlagTimeout and returns, so a missing peer
// turns into an error status instead of a hang.
// ---------------------------------------------------------------------------
// Coalesced copy of whole blocks into peer memory: block d of `src` goes to
// `dst[d]` (16-byte loads and stores, consecutive threads on consecutive
// addresses, so every NVLink write carries full lines).
struct PushArgs {
    const float4* src[kMaxShards];
    float4* dst[kMaxShards];
    int nblocks;
    int64_t n4;   // float4 per block
};

__global__ void __launch_bounds__(256) k_push(PushArgs a) {
    const int64_t total = (int64_t)a.nblocks * a.n4;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
        const int d = (int)(i / a.n4);
        const int64_t j = i - (int64_t)d * a.n4;
        a.dst[d][j] = __ldg(a.src[d] + j);
    }
}

struct PeerSignals {
    unsigned* sig[kMaxShards];     // peer q's signal array: [stage][shard]
    double* energy[kMaxShards];    // peer q's energy partials: [shard]
};

// The epoch lives in device memory (*epoch_dev) so that a captured step replays
// with a fresh epoch: the stage-0 signal of a step (bump = 1) advances it, the
// later signals and waits of the step read it.
__global__ void k_signal(PeerSignals peers, int P, int p, int stage, unsigned* epoch_dev, int bump,
                         const double* energy) {
    if (threadIdx.x != 0) return;
    unsigned epoch = *epoch_dev;
    if (bump) *epoch_dev = ++epoch;
    __threadfence_system();
    for (int q = 0; q < P; ++q) {
        if (energy) peers.energy[q][p] = *energy;
    }
    __threadfence_system();
    for (int q = 0; q < P; ++q) {
        volatile unsigned* slot = peers.sig[q] + stage * kMaxShards + p;
        *slot = epoch;
    }
    __threadfence_system();
}

__global__ void k_wait(const unsigned* sig, int P, int stage, const unsigned* epoch_dev, unsigned epoch_add,
                       long long max_polls, const double* energy_in, double* energy_sum, float* energy_out,
                       double energy_scale, unsigned* flags) {
    if (threadIdx.x != 0) return;
    const unsigned epoch = *epoch_dev + epoch_add;
    const volatile unsigned* row = sig + stage * kMaxShards;
    for (int q = 0; q < P; ++q) {
        long long polls = 0;
        while ((int)(row[q] - epoch) < 0) {
            if (++polls > max_polls) {
                atomicOr(flags, kFlagTimeout);
                return;
            }
            __nanosleep(128);
        }
    }
    __threadfence_system();
    if (energy_sum) {
        // fixed summation order: every shard gets the same bits
        double e = 0.0;
        for (int q = 0; q < P; ++q) e += ((const volatile double*)energy_in)[q];
        *energy_sum = e;
        if (energy_out) *energy_out = (float)(e * energy_scale);
    }
}

}  // namespace epb
