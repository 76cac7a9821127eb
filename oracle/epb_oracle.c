/*
 * epb_oracle.c -- CPU restatement of the electric-potential density and
 * gather math.  TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline leg load this library as the checker and as
 * the timed CPU baseline.  The product path (dreamplacett_framework_b200)
 * never links or calls it.
 *
 * Algorithm sources (paths relative to the reference project):
 *   - bin index with exact-edge correction: kernels/v4_compute.cpp:85-126
 *     (sfpu_floor, correct_bin_idx, face_bxl/face_byl) and the numpy mirror in
 *     tools/v11_phase2_smoke.py:55-72;
 *   - 1-D overlap max(0, min(x+s, left+bs) - max(x, left)) with
 *     left = xl + k*bs: kernels/v4_compute.cpp:128-176,
 *     integration/scatter_ttnn_client.py:64-73;
 *   - contribution = (overlap_x * ratio) * overlap_y: DREAMPlace's triangle
 *     density map (external; described in
 *     integration/scatter_ttnn_client.py:619-627, ratio/offset rule in
 *     tools/v13_offset_ratio_stats.py:54-67);
 *   - density normalisation by 1/bin_area: host/density_scatter_ttnn_server_host.cpp:411-412,
 *     integration/scatter_ttnn_client.py:123-124;
 *   - initial (fixed-macro) density fold: host/density_scatter_ttnn_server_host.cpp:1770-1777.
 *
 * All fp32 arithmetic is written as separate IEEE operations and the file is
 * compiled with -ffp-contract=off, so every contribution equals the CUDA
 * kernel's bit for bit.  Contributions are quantised with round-to-nearest-even
 * to 2^-S and summed in int64, so the fixed-point grid is order independent.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* Corrected floor bin index of coordinate v (kernels/v4_compute.cpp:96-126).
 * The estimate floor((v-origin)*inv_bs) is clamped at 0, then moved so that
 * origin + k*bs <= v < origin + (k+1)*bs holds in fp32, then clamped at 0
 * again.  The extra clamp at nb only keeps the float->int conversion in range;
 * a value of nb or more means "right of the die". */
static inline int ora_bin_floor(float v, float origin, float bs, float inv_bs, int nb) {
    float t = floorf((v - origin) * inv_bs);
    if (t < 0.0f) t = 0.0f;
    if (t > (float)nb) t = (float)nb;
    int k = (int)t;
    float bl = origin + (float)k * bs;
    if (bl > v) k -= 1;
    bl = origin + (float)(k + 1) * bs;
    if (bl <= v) k += 1;
    if (k < 0) k = 0;
    return k;
}

/* Overlap of [v, v+s) with bin k: kernels/v4_compute.cpp:143-151. */
static inline float ora_overlap(float v, float vs_end, float origin, float bs, int k) {
    float left = origin + (float)k * bs;
    float lo = v > left ? v : left;
    float right = left + bs;
    float hi = vs_end < right ? vs_end : right;
    float o = hi - lo;
    return o < 0.0f ? 0.0f : o;
}

typedef struct ora_cells {
    const float* x; const float* y;
    const float* size_x; const float* size_y;
    const float* offset_x; const float* offset_y; /* nullable */
    const float* ratio;                            /* nullable */
    int64_t begin0, end0, begin1, end1;
} ora_cells;

typedef struct ora_grid {
    int M, N;            /* bins along x (rows) and y (columns) */
    float xl, yl, bsx, bsy, inv_bsx, inv_bsy;
} ora_grid;

static inline int64_t ora_node(const ora_cells* c, int64_t i) {
    int64_t n0 = c->end0 - c->begin0;
    return i < n0 ? c->begin0 + i : c->begin1 + (i - n0);
}

static inline int64_t ora_count(const ora_cells* c) {
    return (c->end0 - c->begin0) + (c->end1 - c->begin1);
}

/* Footprint of one cell.  Returns 0 when the cell contributes nothing
 * (non-finite input, non-positive size, or entirely off the die). */
typedef struct { float x, y, ex, ey, r; int kx0, kx1, ky0, ky1; } ora_fp;

static inline int ora_footprint(const ora_cells* c, const ora_grid* g, int64_t node, ora_fp* f) {
    float x = c->x[node], y = c->y[node];
    if (c->offset_x) x = x + c->offset_x[node];
    if (c->offset_y) y = y + c->offset_y[node];
    float sx = c->size_x[node], sy = c->size_y[node];
    float r = c->ratio ? c->ratio[node] : 1.0f;
    if (!isfinite(x) || !isfinite(y) || !isfinite(sx) || !isfinite(sy) || !isfinite(r)) return -1;
    if (!(sx > 0.0f) || !(sy > 0.0f)) return 0;
    float ex = x + sx, ey = y + sy;
    int kx0 = ora_bin_floor(x, g->xl, g->bsx, g->inv_bsx, g->M);
    int kx1 = ora_bin_floor(ex, g->xl, g->bsx, g->inv_bsx, g->M);
    int ky0 = ora_bin_floor(y, g->yl, g->bsy, g->inv_bsy, g->N);
    int ky1 = ora_bin_floor(ey, g->yl, g->bsy, g->inv_bsy, g->N);
    if (kx1 > g->M - 1) kx1 = g->M - 1;
    if (ky1 > g->N - 1) ky1 = g->N - 1;
    if (kx0 > kx1 || ky0 > ky1) return 0;
    f->x = x; f->y = y; f->ex = ex; f->ey = ey; f->r = r;
    f->kx0 = kx0; f->kx1 = kx1; f->ky0 = ky0; f->ky1 = ky1;
    return 1;
}

static void ora_make_grid(ora_grid* g, int M, int N, float xl, float yl, float bsx, float bsy) {
    g->M = M; g->N = N; g->xl = xl; g->yl = yl; g->bsx = bsx; g->bsy = bsy;
    g->inv_bsx = (float)(1.0 / (double)bsx);
    g->inv_bsy = (float)(1.0 / (double)bsy);
}

/* Fixed-point density: grid[kx*N+ky] += llrintf(((ox*ratio)*oy) * 2^S).
 * With nthreads > 1 each thread accumulates into its own slice of the
 * caller-owned workspace ws[(nthreads-1)*M*N] and the slices are summed in
 * parallel over bins; integer sums make the result independent of the thread
 * count.  Returns the number of cells with non-finite inputs (skipped). */
int64_t ora_density_fixed(const float* x, const float* y, const float* sx, const float* sy,
                          const float* offx, const float* offy, const float* ratio,
                          int64_t b0, int64_t e0, int64_t b1, int64_t e1,
                          int M, int N, float xl, float yl, float bsx, float bsy,
                          int S, int64_t* grid, int nthreads, int64_t* ws) {
    ora_cells c = {x, y, sx, sy, offx, offy, ratio, b0, e0, b1, e1};
    ora_grid g; ora_make_grid(&g, M, N, xl, yl, bsx, bsy);
    const float scale = ldexpf(1.0f, S);
    const int64_t n = ora_count(&c);
    const int64_t MN = (int64_t)M * (int64_t)N;
    int64_t bad = 0;
    if (nthreads < 1 || ws == NULL) nthreads = 1;
#ifdef _OPENMP
    #pragma omp parallel num_threads(nthreads) reduction(+:bad)
    {
        const int tid = omp_get_thread_num();
        const int nt = omp_get_num_threads();
        int64_t* priv = tid == 0 ? grid : ws + (int64_t)(tid - 1) * MN;
        memset(priv, 0, (size_t)MN * sizeof(int64_t));
        #pragma omp for schedule(static)
        for (int64_t i = 0; i < n; ++i) {
            ora_fp f;
            int st = ora_footprint(&c, &g, ora_node(&c, i), &f);
            if (st < 0) { bad++; continue; }
            if (st == 0) continue;
            for (int kx = f.kx0; kx <= f.kx1; ++kx) {
                float ox = ora_overlap(f.x, f.ex, g.xl, g.bsx, kx);
                float oxr = ox * f.r;
                for (int ky = f.ky0; ky <= f.ky1; ++ky) {
                    float oy = ora_overlap(f.y, f.ey, g.yl, g.bsy, ky);
                    float a = oxr * oy;
                    priv[(int64_t)kx * N + ky] += llrintf(a * scale);
                }
            }
        }
        /* implicit barrier above; merge the private slices bin-parallel */
        if (nt > 1) {
            #pragma omp for schedule(static)
            for (int64_t b = 0; b < MN; ++b) {
                int64_t s = grid[b];
                for (int t = 1; t < nt; ++t) s += ws[(int64_t)(t - 1) * MN + b];
                grid[b] = s;
            }
        }
    }
#else
    (void)ws;
    memset(grid, 0, (size_t)MN * sizeof(int64_t));
    for (int64_t i = 0; i < n; ++i) {
        ora_fp f;
        int st = ora_footprint(&c, &g, ora_node(&c, i), &f);
        if (st < 0) { bad++; continue; }
        if (st == 0) continue;
        for (int kx = f.kx0; kx <= f.kx1; ++kx) {
            float ox = ora_overlap(f.x, f.ex, g.xl, g.bsx, kx);
            float oxr = ox * f.r;
            for (int ky = f.ky0; ky <= f.ky1; ++ky) {
                float oy = ora_overlap(f.y, f.ey, g.yl, g.bsy, ky);
                grid[(int64_t)kx * N + ky] += llrintf((oxr * oy) * scale);
            }
        }
    }
#endif
    return bad;
}

/* Same footprint and fp32 contributions, accumulated in fp64 without
 * quantisation (area units, not normalised). */
int64_t ora_density_f64(const float* x, const float* y, const float* sx, const float* sy,
                        const float* offx, const float* offy, const float* ratio,
                        int64_t b0, int64_t e0, int64_t b1, int64_t e1,
                        int M, int N, float xl, float yl, float bsx, float bsy,
                        double* grid) {
    ora_cells c = {x, y, sx, sy, offx, offy, ratio, b0, e0, b1, e1};
    ora_grid g; ora_make_grid(&g, M, N, xl, yl, bsx, bsy);
    const int64_t n = ora_count(&c);
    int64_t bad = 0;
    memset(grid, 0, (size_t)M * N * sizeof(double));
    for (int64_t i = 0; i < n; ++i) {
        ora_fp f;
        int st = ora_footprint(&c, &g, ora_node(&c, i), &f);
        if (st < 0) { bad++; continue; }
        if (st == 0) continue;
        for (int kx = f.kx0; kx <= f.kx1; ++kx) {
            float oxr = ora_overlap(f.x, f.ex, g.xl, g.bsx, kx) * f.r;
            for (int ky = f.ky0; ky <= f.ky1; ++ky) {
                float oy = ora_overlap(f.y, f.ey, g.yl, g.bsy, ky);
                grid[(size_t)kx * N + ky] += (double)(oxr * oy);
            }
        }
    }
    return bad;
}

/* Fixed grid -> normalised fp32 density, plus the fp32 fold of the
 * normalised initial density (host/density_scatter_ttnn_server_host.cpp:1774-1777):
 *   rho[b] = (float)((double)grid[b] * dscale) + init[b]
 * dscale = 2^-S / bin_area (double).  Returns the number of bins whose
 * fixed value is negative or >= 2^62 (saturation). */
int64_t ora_fixed_to_density(const int64_t* grid, const float* init, int64_t MN,
                             double dscale, float* rho) {
    int64_t sat = 0;
    const int64_t lim = (int64_t)1 << 62;
    for (int64_t b = 0; b < MN; ++b) {
        int64_t q = grid[b];
        if (q < 0 || q >= lim) sat++;
        float v = (float)((double)q * dscale);
        rho[b] = init ? v + init[b] : v;
    }
    return sat;
}

/* Per-cell field gather (DREAMPlace electric_force, external; same footprint
 * and overlap weights as the scatter):
 *   grad_x[node] = -gout * ratio * sum_b (ox_b*oy_b) * field_x[b]
 * accumulated in fp64.  Nodes outside the two ranges are not written. */
int64_t ora_gather(const float* x, const float* y, const float* sx, const float* sy,
                   const float* offx, const float* offy, const float* ratio,
                   int64_t b0, int64_t e0, int64_t b1, int64_t e1,
                   int M, int N, float xl, float yl, float bsx, float bsy,
                   const float* field_x, const float* field_y, double gout,
                   float* grad_x, float* grad_y, int nthreads) {
    ora_cells c = {x, y, sx, sy, offx, offy, ratio, b0, e0, b1, e1};
    ora_grid g; ora_make_grid(&g, M, N, xl, yl, bsx, bsy);
    const int64_t n = ora_count(&c);
    int64_t bad = 0;
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
    #pragma omp parallel for num_threads(nthreads) schedule(static) reduction(+:bad)
#else
    (void)nthreads;
#endif
    for (int64_t i = 0; i < n; ++i) {
        int64_t node = ora_node(&c, i);
        ora_fp f;
        int st = ora_footprint(&c, &g, node, &f);
        double ax = 0.0, ay = 0.0;
        if (st < 0) bad++;
        if (st > 0) {
            for (int kx = f.kx0; kx <= f.kx1; ++kx) {
                float ox = ora_overlap(f.x, f.ex, g.xl, g.bsx, kx);
                for (int ky = f.ky0; ky <= f.ky1; ++ky) {
                    float oy = ora_overlap(f.y, f.ey, g.yl, g.bsy, ky);
                    double a = (double)ox * (double)oy;
                    size_t b = (size_t)kx * N + ky;
                    ax += a * (double)field_x[b];
                    ay += a * (double)field_y[b];
                }
            }
        }
        double r = st > 0 ? (double)f.r : 0.0;
        grad_x[node] = (float)(-gout * r * ax);
        grad_y[node] = (float)(-gout * r * ay);
    }
    return bad;
}

/* Bin range of one coordinate, exposed for the exact-edge known-answer tests. */
void ora_bin_range(float v, float s, float origin, float bs, int nb, int* lo, int* hi) {
    float inv = (float)(1.0 / (double)bs);
    int a = ora_bin_floor(v, origin, bs, inv, nb);
    int b = ora_bin_floor(v + s, origin, bs, inv, nb);
    if (b > nb - 1) b = nb - 1;
    *lo = a; *hi = b;
}

int ora_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
