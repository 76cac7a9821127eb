// epb_engine.cu -- host engine and C ABI of libepb200.so.
//
// Replaces the reference's out-of-process server
// (host/density_scatter_ttnn_server_host.cpp: argv parse :324-339, sizing
// :405-460, per-iteration loop :1326-1824, TTNNDCTSolver :225-306) with an
// in-process, stream-ordered engine on device pointers.  See include/epb.h for
// the per-function mapping.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/epb.h"
#include "epb_kernels.cuh"
#include "tile_kernels.cuh"
#include "wirelength.cuh"
#include "placement_kernels.cuh"

using namespace epb;

struct epb_handle {
    int dev = 0;
    int M = 0, N = 0;
    // sharding: this handle is shard p of P; it owns rows [row0, row0+RB) and,
    // in the column pass, columns [col0, col0+NB).  P = 1 for a whole grid.
    int P = 1, p = 0, RB = 0, NB = 0, row0 = 0, col0 = 0;
    double xl = 0, yl = 0, xh = 0, yh = 0;
    float bsx = 0, bsy = 0;
    int S = 0;
    double dscale = 0;          // 2^-S / bin_area
    long long* grid = nullptr;  // int64 [RB*N] (this band), kept zeroed between forwards
    long long* grid2 = nullptr; // int64 [M*N] first-range grid of epb_forward_overflow (lazy)
    bool grid_dirty = false;
    float* init = nullptr;      // normalised initial density of this band [RB*N]
    bool has_init = false;
    float* t1 = nullptr;        // [M*N] row-DCT output (P == 1 only; shards use the caller's buffers)
    float* g = nullptr;         // [kColOutputs*M*N] column-pass outputs (P == 1 only)
    float2* fxy = nullptr;      // interleaved fields of the last forward (P == 1 only)
    bool have_fields = false;
    float2 *twM = nullptr, *qwM = nullptr, *twN = nullptr, *qwN = nullptr;
    double* partials = nullptr;
    unsigned* counter = nullptr;
    double* energy_d = nullptr;
    unsigned* flags = nullptr;
    // placement-loop scratch (epb_overflow, epb_descent_step)
    double* ovf_partials = nullptr;   // [2 * kOvfMaxBlocks]
    unsigned* ovf_counter = nullptr;
    unsigned* linf_bits = nullptr;
    int sms = 1;  // streaming multiprocessors of the device
    // whole-grid gather: CTAs resident at once (k_gather<false>, k_gather<true>),
    // the grid of its cell-striding launch
    unsigned gather_grid[2] = {1, 1};
    // band lists of a shard in cell order (k_band_check / k_band_list): kept
    // across calls, with the cell view they were made from
    BandList bl{};
    int64_t bl_cap = 0;         // cells the buffers hold (grows)
    bool bl_force = true;       // the next list maintenance lists again (new buffers or cell arrays)
    bool bl_stale = false;      // epb_descent_step moved the cells since the lists were last checked
    CellView bl_key{};
    // peer transport (epb_shard_peer_buffers / epb_shard_connect)
    float* p_t1 = nullptr;      // t1_recv [M*NB]
    float* p_g = nullptr;       // g_recv [kColOutputs*M*NB]
    float* p_gsend = nullptr;   // column-pass blocks bound for other shards [kColOutputs*M*NB]
    float2* p_fxy = nullptr;    // fxy_ext [(RB+Hmax)*N]
    unsigned char* p_sig = nullptr;  // signal slots [3][kMaxShards] uint32, then energies [kMaxShards] double
    int p_halo = 0;             // halo rows this band receives (0 for the last band)
    int p_halo_max = 0;
    bool connected = false;
    unsigned* epoch_dev = nullptr;  // step epoch of the peer signals (device: captured steps replay)
    float* peer_t1[kMaxShards] = {nullptr};
    float* peer_g[kMaxShards] = {nullptr};
    float2* peer_fxy[kMaxShards] = {nullptr};
    unsigned char* peer_sig[kMaxShards] = {nullptr};
    double* energy_total = nullptr;
    long long max_polls = 40000000;  // bounded waits: ~5 s of 128 ns polls
    // cell tiles (whole-grid handles without EPB_CONFIG_CELL_ORDER): the lists,
    // kept across calls (tile_prepare), and the cell view they were made from
    bool cell_order = false;
    TileGeom tg{};
    TileBins tb{};
    int ntiles = 0;
    int64_t tb_cells = 0;       // cells the buffers hold (escape lists, grows)
    int64_t tb_cap = 0;         // listing capacity = kMaxTilesPerCell * tb_cells
    int tb_items = 0;           // work-item capacity
    bool tb_force = true;       // the next list maintenance must rebuild (new buffers or cell arrays)
    bool tb_stale = false;      // epb_descent_step moved the cells since the lists were last validated
    float* rho = nullptr;       // [M*N] density when the caller passes none
    unsigned tile_grid = 1;     // persistent CTAs of k_tile_scatter / k_tile_gather
    unsigned tile_grid_ovf = 1; // persistent CTAs of k_tile_scatter<true> (two limb sets)
    unsigned long long* esc_grid0 = nullptr;  // [M*N] escape sums of the overflow cells (lazy)
    double* tile_ovf_part = nullptr;          // [2 * ntiles]
    unsigned* tile_ovf_counter = nullptr;
    bool tb_valid = false;
    CellView tb_key{};
    // stage timing (epb_profile_start/stop)
    struct Span { int stage, a, b; };
    bool prof_on = false;
    int prof_calls_left = 0;
    std::vector<cudaEvent_t> prof_events;
    int prof_used = 0;
    std::vector<Span> prof_spans;
    std::string err;
};

namespace {

struct DeviceGuard {
    int prev = -1;
    bool ok = true;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

int fail(epb_handle* h, int code, const std::string& msg) {
    if (h) h->err = msg;
    return code;
}

int cuda_fail(epb_handle* h, cudaError_t e, const char* what) {
    return fail(h, EPB_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

#define EPB_CUDA(h, call)                                                  \
    do {                                                                   \
        cudaError_t e_ = (call);                                           \
        if (e_ != cudaSuccess) return cuda_fail((h), e_, #call);           \
    } while (0)

#define EPB_LAUNCHED(h, what)                                              \
    do {                                                                   \
        cudaError_t e_ = cudaGetLastError();                               \
        if (e_ != cudaSuccess) return cuda_fail((h), e_, what);            \
    } while (0)

bool pow2_in_range(int v) { return v >= 16 && v <= 4096 && (v & (v - 1)) == 0; }

GridGeom geom(const epb_handle* h) {
    GridGeom g;
    g.M = h->M; g.N = h->N;
    g.xl = (float)h->xl; g.yl = (float)h->yl;
    g.bsx = h->bsx; g.bsy = h->bsy;
    g.ibsx = (float)(1.0 / (double)h->bsx);
    g.ibsy = (float)(1.0 / (double)h->bsy);
    return g;
}

int make_view(epb_handle* h, const epb_cells* c, CellView& v) {
    if (!c) return fail(h, EPB_EINVAL, "cells is NULL");
    const int64_t n0 = c->end0 - c->begin0, n1 = c->end1 - c->begin1;
    if (c->begin0 < 0 || c->begin1 < 0 || n0 < 0 || n1 < 0)
        return fail(h, EPB_EINVAL, "cell ranges must satisfy 0 <= begin <= end");
    if (n0 + n1 > 0 && (!c->x || !c->y || !c->size_x || !c->size_y))
        return fail(h, EPB_EINVAL, "x, y, size_x and size_y must be non-NULL");
    v.x = c->x; v.y = c->y; v.sx = c->size_x; v.sy = c->size_y;
    v.ox = c->offset_x; v.oy = c->offset_y; v.ratio = c->ratio;
    v.b0 = c->begin0; v.n0 = n0; v.b1 = c->begin1; v.n = n0 + n1;
    return EPB_OK;
}

unsigned cell_blocks(int64_t n);

// Whole-grid gather: one wave of CTAs striding over the cells (fewer when
// there are fewer cells than threads).
unsigned gather_blocks(const epb_handle* h, int64_t n, bool io) {
    return std::min(cell_blocks(n), h->gather_grid[io ? 1 : 0]);
}

unsigned cell_blocks(int64_t n) {
    int64_t b = (n + 255) / 256;
    if (b < 1) b = 1;
    if (b > (1 << 20)) b = 1 << 20;  // grid-stride beyond this
    return (unsigned)b;
}

// FFT twiddles in the per-pass [r][k] layout the device FFT reads (fft.cuh):
// entry (pass NS, r, k) = exp(-2 pi i r k STEP / L), STEP = L / (NS R); and the
// quarter-wave table (cos, sin)(pi k / 2L).  fp64 -> fp32.
void host_tables(int L, std::vector<float2>& tw, std::vector<float2>& qw) {
    std::vector<float2> w(L);
    qw.resize(L);
    for (int t = 0; t < L; ++t) {
        const double a = 2.0 * M_PI * (double)t / (double)L;
        w[t] = make_float2((float)std::cos(a), (float)(-std::sin(a)));
        const double b = M_PI * (double)t / (2.0 * (double)L);
        qw[t] = make_float2((float)std::cos(b), (float)std::sin(b));
    }
    tw.assign(std::max(1, tw_table_size(L)), make_float2(1.0f, 0.0f));
    for (int ns = 16; ns < L; ns *= 16) {
        const int R = L / ns >= 16 ? 16 : L / ns;
        const int step = L / (ns * R);
        for (int r = 0; r < R; ++r)
            for (int k = 0; k < ns; ++k) tw[tw_offset(L, ns) + r * ns + k] = w[(int64_t)r * k * step];
    }
}

template <typename T>
int dev_alloc(epb_handle* h, T** p, size_t count) {
    cudaError_t e = cudaMalloc((void**)p, count * sizeof(T));
    if (e != cudaSuccess) { *p = nullptr; return cuda_fail(h, e, "cudaMalloc"); }
    return EPB_OK;
}

void free_all(epb_handle* h) {
    void* ptrs[] = {h->grid, h->grid2, h->init, h->t1, h->g, h->fxy, h->twM, h->qwM,
                    h->twN, h->qwN, h->partials, h->counter, h->energy_d, h->flags,
                    h->ovf_partials, h->ovf_counter, h->linf_bits, h->bl.sel, h->bl.cnt,
                    h->bl.geo, h->bl.r, h->bl.listed, h->bl.ext, h->rho, h->tb.cnt, h->tb.cur, h->tb.start, h->tb.nown,
                    h->tb.first_item, h->tb.items, h->tb.arrive, h->tb.part, h->tb.meta, h->tb.stat, h->tb.key,
                    h->tb.geo, h->tb.bins, h->tb.esc_dyn, h->tb.esc_static, h->tb.esc_grid, h->esc_grid0,
                    h->tile_ovf_part, h->tile_ovf_counter};
    for (void* p : ptrs)
        if (p) cudaFree(p);
    for (int q = 0; q < kMaxShards; ++q) {
        if (q == h->p) continue;
        if (h->peer_t1[q]) cudaIpcCloseMemHandle(h->peer_t1[q]);
        if (h->peer_g[q]) cudaIpcCloseMemHandle(h->peer_g[q]);
        if (h->peer_fxy[q]) cudaIpcCloseMemHandle(h->peer_fxy[q]);
        if (h->peer_sig[q]) cudaIpcCloseMemHandle(h->peer_sig[q]);
    }
    void* own[] = {h->p_t1, h->p_g, h->p_gsend, h->p_fxy, h->p_sig, h->energy_total, h->epoch_dev};
    for (void* p : own)
        if (p) cudaFree(p);
    for (cudaEvent_t e : h->prof_events) cudaEventDestroy(e);
    h->prof_events.clear();
}

// ----- kernel dispatch on the transform length -----

template <int L>
int set_smem(epb_handle* h, const void* fn, size_t bytes) {
    if (bytes > 48 * 1024) EPB_CUDA(h, cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    return EPB_OK;
}

int ilog2(int v) {
    int l = 0;
    while ((1 << l) < v) ++l;
    return l;
}

// Row pass over this handle's RB rows: t1 receives the blocked layout (block
// width NB, RB*NB elements per block); for P == 1 that is plain [M][N].
template <int L, bool HALF>
int launch_row_fwd_v(epb_handle* h, bool from_fixed, const float* rho_in, float* rho_out, const DstTable& t1,
                     int drow0, cudaStream_t st) {
    using C = RowFwdCfg<L, HALF>;
    const unsigned blocks = (unsigned)((h->RB + C::ROWS - 1) / C::ROWS);
    const float* init = h->has_init && from_fixed ? h->init : nullptr;
    const int lnb = ilog2(h->NB);
    if (from_fixed) {
        auto fn = k_row_fwd<L, true, HALF>;
        if (int rc = set_smem<L>(h, (const void*)fn, C::SMEM)) return rc;
        fn<<<blocks, C::T, C::SMEM, st>>>(h->grid, nullptr, init, h->dscale, h->RB, rho_out, t1, lnb, drow0,
                                          h->twN, h->qwN, h->flags);
    } else {
        auto fn = k_row_fwd<L, false, HALF>;
        if (int rc = set_smem<L>(h, (const void*)fn, C::SMEM)) return rc;
        fn<<<blocks, C::T, C::SMEM, st>>>(nullptr, rho_in, nullptr, h->dscale, h->RB, rho_out, t1, lnb, drow0,
                                          h->twN, h->qwN, h->flags);
    }
    EPB_LAUNCHED(h, "k_row_fwd launch");
    return EPB_OK;
}

// Half-size CTAs when the default launch has fewer CTAs than the GPU has SMs
// (a shard's band of a few hundred rows, a strip of a few hundred columns).
template <int L>
int launch_row_fwd_t(epb_handle* h, bool from_fixed, const float* rho_in, float* rho_out, const DstTable& t1,
                     int drow0, cudaStream_t st) {
    if ((h->RB + RowFwdCfg<L>::ROWS - 1) / RowFwdCfg<L>::ROWS < h->sms)
        return launch_row_fwd_v<L, true>(h, from_fixed, rho_in, rho_out, t1, drow0, st);
    return launch_row_fwd_v<L, false>(h, from_fixed, rho_in, rho_out, t1, drow0, st);
}

template <int L, bool HALF>
int launch_col_v(epb_handle* h, const ColArgs& a, cudaStream_t st) {
    using C = ColCfg<L, HALF>;
    const unsigned blocks = (unsigned)((a.N + C::W - 1) / C::W);
    auto fn = k_col<L, HALF>;
    if (int rc = set_smem<L>(h, (const void*)fn, C::SMEM)) return rc;
    fn<<<blocks, C::T, C::SMEM, st>>>(a);
    EPB_LAUNCHED(h, "k_col launch");
    return EPB_OK;
}

template <int L>
int launch_col_t(epb_handle* h, const ColArgs& a, cudaStream_t st) {
    if ((a.N + ColCfg<L>::W - 1) / ColCfg<L>::W < h->sms) return launch_col_v<L, true>(h, a, st);
    return launch_col_v<L, false>(h, a, st);
}

template <int L>
int launch_row_inv_t(epb_handle* h, const RowInvArgs& a, cudaStream_t st) {
    using C = RowInvCfg<L>;
    const unsigned blocks = (unsigned)((a.M + C::ROWS - 1) / C::ROWS);
    auto fn = k_row_inv<L>;
    if (int rc = set_smem<L>(h, (const void*)fn, C::SMEM)) return rc;
    fn<<<blocks, C::T, C::SMEM, st>>>(a);
    EPB_LAUNCHED(h, "k_row_inv launch");
    return EPB_OK;
}

#define EPB_DISPATCH_L(Lval, CALL)                                          \
    switch (Lval) {                                                         \
        case 16: return CALL(16);                                           \
        case 32: return CALL(32);                                           \
        case 64: return CALL(64);                                           \
        case 128: return CALL(128);                                         \
        case 256: return CALL(256);                                         \
        case 512: return CALL(512);                                         \
        case 1024: return CALL(1024);                                       \
        case 2048: return CALL(2048);                                       \
        case 4096: return CALL(4096);                                       \
        default: return fail(h, EPB_EINVAL, "unsupported transform length"); \
    }

int launch_row_fwd(epb_handle* h, bool from_fixed, const float* rho_in, float* rho_out, const DstTable& t1,
                   int drow0, cudaStream_t st) {
#define CALL_RF(L) launch_row_fwd_t<L>(h, from_fixed, rho_in, rho_out, t1, drow0, st)
    EPB_DISPATCH_L(h->N, CALL_RF)
#undef CALL_RF
}

int launch_col(epb_handle* h, const ColArgs& a, cudaStream_t st) {
#define CALL_C(L) launch_col_t<L>(h, a, st)
    EPB_DISPATCH_L(h->M, CALL_C)
#undef CALL_C
}

int launch_row_inv(epb_handle* h, const RowInvArgs& a, cudaStream_t st) {
#define CALL_RI(L) launch_row_inv_t<L>(h, a, st)
    EPB_DISPATCH_L(h->N, CALL_RI)
#undef CALL_RI
}

int col_width(int M) {
    switch (M) {
        case 16: return ColCfg<16>::W;
        case 32: return ColCfg<32>::W;
        case 64: return ColCfg<64>::W;
        case 128: return ColCfg<128>::W;
        case 256: return ColCfg<256>::W;
        case 512: return ColCfg<512>::W;
        case 1024: return ColCfg<1024>::W;
        case 2048: return ColCfg<2048>::W;
        default: return ColCfg<4096>::W;
    }
}

// Columns per strip of the column-pass output layout: at least the column
// kernel's width (so a CTA writes inside one strip) and kStripWidth (so the row
// pass reads whole sectors), at most the column band.
int strip_width(const epb_handle* h) {
    return std::min(std::max(col_width(h->M), kStripWidth), h->NB);
}

int col_blocks(int M, int N) {
    int W = 4;
    switch (M) {
        case 16: W = ColCfg<16>::W; break;
        case 32: W = ColCfg<32>::W; break;
        case 64: W = ColCfg<64>::W; break;
        case 128: W = ColCfg<128>::W; break;
        case 256: W = ColCfg<256>::W; break;
        case 512: W = ColCfg<512>::W; break;
        case 1024: W = ColCfg<1024>::W; break;
        case 2048: W = ColCfg<2048>::W; break;
        case 4096: W = ColCfg<4096>::W; break;
    }
    return (N + W - 1) / W;
}

// Profiling: a mark is an event recorded on the stream between two kernels.
struct ProfCall {
    epb_handle* h;
    cudaStream_t st;
    bool on;
    int last = -1;
    ProfCall(epb_handle* h_, cudaStream_t s) : h(h_), st(s) {
        on = h->prof_on && h->prof_calls_left > 0;
        if (on) h->prof_calls_left--;
    }
    int mark() {
        if (!on || h->prof_used >= (int)h->prof_events.size()) return -1;
        const int i = h->prof_used++;
        if (cudaEventRecord(h->prof_events[i], st) != cudaSuccess) return -1;
        return i;
    }
    void begin() { last = mark(); }
    void end_stage(int stage) {
        const int m = mark();
        if (last >= 0 && m >= 0) h->prof_spans.push_back({stage, last, m});
        last = m;
    }
};

// Destination table of a local send buffer laid out in P blocks of `block` elements.
DstTable blocked(float* base, int64_t block, int P) {
    DstTable t;
    for (int q = 0; q < kMaxShards; ++q) t.p[q] = q < P ? base + q * block : nullptr;
    return t;
}

// Column pass: t1 = column strip [M][NB] of this handle's column band; g =
// outputs laid out g[d][o][r][c] (d destination row band).  The energy of the
// strip (times MN/4) lands in h->energy_d and, when given, energy_out.
int launch_columns(epb_handle* h, const float* t1, const DstTable& g, float* energy_out, cudaStream_t st) {
    ColArgs ca;
    ca.t1 = t1;
    ca.g = g;
    ca.ostride = (int64_t)h->RB * h->NB;
    ca.lrb = ilog2(h->RB);
    ca.lsw = ilog2(strip_width(h));
    ca.col_base = h->col0;
    ca.ku = (float)(2.0 * M_PI / h->M);
    ca.kv = (float)(2.0 * M_PI / h->N * (double)(h->bsx / h->bsy));
    ca.tw = h->twM; ca.qw = h->qwM;
    ca.partials = h->partials; ca.counter = h->counter; ca.energy_d = h->energy_d;
    ca.energy_out = energy_out; ca.N = h->NB;
    ca.energy_scale = (double)h->M * (double)h->N / 4.0;
    return launch_col(h, ca, st);
}

// Row inverses of this handle's RB rows from g[q][o][r][c] (q source column band).
int launch_rows_inverse(epb_handle* h, const float* g, float* potential, float* field_x, float* field_y,
                        float2* fxy, bool want_phi, cudaStream_t st, float2* halo_dst = nullptr, int halo_rows = 0) {
    RowInvArgs ra;
    ra.g = g;
    ra.ostride = (int64_t)h->RB * h->NB;
    ra.qstride = kColOutputs * (int64_t)h->RB * h->NB;
    ra.kv = (float)(2.0 * M_PI / h->N * (double)(h->bsx / h->bsy));
    ra.lnb = ilog2(h->NB);
    ra.lsw = ilog2(strip_width(h));
    ra.lrb = ilog2(h->RB);
    ra.fx = field_x; ra.fy = field_y; ra.phi = want_phi ? potential : nullptr; ra.fxy = fxy;
    ra.halo_dst = halo_dst; ra.halo_rows = halo_dst ? halo_rows : 0;
    ra.tw = h->twN; ra.qw = h->qwN; ra.M = h->RB; ra.want_phi = want_phi;
    return launch_row_inv(h, ra, st);
}

// DCT solve from the state in t1 (after the row-forward pass), single-grid handles.
int solve_from_t1(epb_handle* h, cudaStream_t st, float* potential, float* field_x, float* field_y,
                  float* energy, ProfCall& pc) {
    const bool want_phi = potential != nullptr;
    if (int rc = launch_columns(h, h->t1, blocked(h->g, 0, 1), energy, st)) return rc;
    pc.end_stage(EPB_STAGE_COLUMN);
    if (int rc = launch_rows_inverse(h, h->g, potential, field_x, field_y, h->fxy, want_phi, st)) return rc;
    pc.end_stage(EPB_STAGE_ROW_INV);
    h->have_fields = true;
    return EPB_OK;
}

// Same cell arrays and ranges: the lists made from one view serve the other.
bool same_cells(const CellView& a, const CellView& b) {
    return a.x == b.x && a.ox == b.ox && a.sx == b.sx && a.b0 == b.b0 && a.n0 == b.n0 && a.b1 == b.b1 && a.n == b.n;
}

bool same_view(const CellView& a, const CellView& b);

// Band-list buffers for n cells (grown when more cells come; that call
// synchronises the stream and allocates, and the lists are made again).
int band_list_reserve(epb_handle* h, int64_t n, cudaStream_t st) {
    if (n <= h->bl_cap) return EPB_OK;
    EPB_CUDA(h, cudaStreamSynchronize(st));
    void** bufs[] = {(void**)&h->bl.sel, (void**)&h->bl.cnt, (void**)&h->bl.geo, (void**)&h->bl.r,
                     (void**)&h->bl.listed, (void**)&h->bl.ext};
    for (void** b : bufs) {
        if (*b) cudaFree(*b);
        *b = nullptr;
    }
    h->bl_cap = 0;
    const int64_t nseg = (n + kSelChunk - 1) / kSelChunk;
    if (int rc = dev_alloc(h, &h->bl.sel, (size_t)(nseg * kSelChunk))) return rc;
    if (int rc = dev_alloc(h, &h->bl.cnt, (size_t)nseg)) return rc;
    if (int rc = dev_alloc(h, &h->bl.geo, (size_t)(nseg * kSelChunk))) return rc;
    if (int rc = dev_alloc(h, &h->bl.r, (size_t)(nseg * kSelChunk))) return rc;
    if (int rc = dev_alloc(h, &h->bl.listed, (size_t)n)) return rc;
    if (int rc = dev_alloc(h, &h->bl.ext, (size_t)n)) return rc;
    EPB_CUDA(h, cudaMemset(h->bl.listed, 0, (size_t)n));
    h->bl_cap = n;
    h->bl_force = true;
    return EPB_OK;
}

// On a shard (P > 1) in cell order: check the band's list against the
// positions of v, segment by segment, and list a segment again when a cell
// came into the band (on the device); every segment when the buffers or the
// cell arrays are new.
int band_list_prepare(epb_handle* h, const CellView& v, cudaStream_t st) {
    if (int rc = band_list_reserve(h, std::max<int64_t>(v.n, 1), st)) return rc;
    if (!same_view(h->bl_key, v)) h->bl_force = true;
    const int row1 = h->row0 + h->RB;
    const int64_t nseg = (v.n + kSelChunk - 1) / kSelChunk;
    k_band_update<<<(unsigned)std::max<int64_t>(nseg, 1), kBandThreads, 0, st>>>(v, geom(h), h->row0, row1, h->bl,
                                                                                 h->bl_force ? 1 : 0, h->flags);
    EPB_LAUNCHED(h, "k_band_update launch");
    h->bl_force = false;
    h->bl_stale = false;
    h->bl_key = v;
    return EPB_OK;
}

int scatter_into(epb_handle* h, const CellView& v0, cudaStream_t st, long long* grid) {
    if (v0.n == 0) return EPB_OK;
    if (v0.n >= ((int64_t)1 << 31)) return fail(h, EPB_EINVAL, "at most 2^31 - 1 cells");
    const float qscale = ldexpf(1.0f, h->S);
    const CellView& v = v0;
    if (h->P > 1) {
        if (int rc = band_list_prepare(h, v, st)) return rc;
        // a band lists about 1/P of a segment's cells: CTAs per segment so that a
        // thread has about one cell, as in the whole-grid scatter
        const int64_t split = std::max(1, EPB_SEL_SCATTER_SPLIT / h->P);
        const unsigned blocks = (unsigned)(((v.n + kSelChunk - 1) / kSelChunk) * split);
        k_scatter_listed<<<blocks, 256, 0, st>>>(v, geom(h), qscale, (unsigned long long*)grid, h->row0,
                                                 h->row0 + h->RB, h->bl, h->flags);
        EPB_LAUNCHED(h, "k_scatter_listed launch");
        return EPB_OK;
    }
    k_scatter<false><<<cell_blocks(v.n), 256, 0, st>>>(v, geom(h), qscale, (unsigned long long*)grid, h->row0,
                                                      h->row0 + h->RB, h->flags);
    EPB_LAUNCHED(h, "k_scatter launch");
    return EPB_OK;
}

// Gather of a shard's own cells (first bin row in the band) from fields holding
// rows [row0, row0 + RB + halo).
int tile_gather(epb_handle* h, const CellView& v, const float2* fxy, int halo, int owned_only, const float* grad_out,
                float* grad_x, float* grad_y, cudaStream_t st);

int shard_gather(epb_handle* h, const CellView& v0, const float2* fxy, int halo, const float* grad_out,
                 float* grad_x, float* grad_y, cudaStream_t st) {
    if (!h->cell_order) return tile_gather(h, v0, fxy, halo, 1, grad_out, grad_x, grad_y, st);
    const CellView& v = v0;
    if (h->P > 1) {
        if (v.n == 0) return EPB_OK;
        // the forward's list, checked again when the cells or their positions may differ
        if (h->bl_force || h->bl_stale || !same_view(h->bl_key, v))
            if (int rc = band_list_prepare(h, v, st)) return rc;
        const unsigned blocks = (unsigned)((v.n + kSelChunk - 1) / kSelChunk);   // one CTA per segment
        k_gather_listed<<<blocks, 256, 0, st>>>(v, geom(h), fxy, h->row0, h->row0 + h->RB, halo, grad_out, grad_x,
                                                grad_y, h->bl, h->flags);
        EPB_LAUNCHED(h, "k_gather_listed launch");
        return EPB_OK;
    }
    k_gather<false><<<cell_blocks(v.n), 256, 0, st>>>(v, geom(h), fxy, nullptr, nullptr, h->row0, h->row0 + h->RB,
                                                     halo, 1, grad_out, grad_x, grad_y, h->flags);
    EPB_LAUNCHED(h, "k_gather launch");
    return EPB_OK;
}

// ----- cell tiles ------------------------------------------------------------

// Bins the listings are widened by on a whole grid: a cell may move this far
// between rebuilds of the lists (a shard rebuilds its band's lists every call).
constexpr int kTileMargin = kGatherLo;

unsigned fixed_blocks(const epb_handle* h) { return (unsigned)(8 * h->sms); }

// Listing and escape buffers for n cells (grown when more cells come; that
// call synchronises the stream and allocates, and the lists are rebuilt).
int tile_reserve(epb_handle* h, int64_t n, cudaStream_t st) {
    if (n <= h->tb_cells) return EPB_OK;
    if (n > (int64_t)kNodeMask / kMaxTilesPerCell) return fail(h, EPB_EINVAL, "too many cells for the tile lists");
    EPB_CUDA(h, cudaStreamSynchronize(st));
    void** bufs[] = {(void**)&h->tb.stat, (void**)&h->tb.key, (void**)&h->tb.geo, (void**)&h->tb.bins,
                     (void**)&h->tb.esc_dyn, (void**)&h->tb.esc_static, (void**)&h->tb.items, (void**)&h->tb.part};
    for (void** b : bufs) {
        if (*b) cudaFree(*b);
        *b = nullptr;
    }
    h->tb_cells = 0;
    h->tb_valid = false;
    const int64_t cap = (int64_t)kMaxTilesPerCell * n;
    const int64_t items = h->ntiles + cap / kChunk + 1;
    if (int rc = dev_alloc(h, &h->tb.stat, (size_t)cap)) return rc;
    if (int rc = dev_alloc(h, &h->tb.key, (size_t)cap)) return rc;
    if (int rc = dev_alloc(h, &h->tb.geo, (size_t)cap)) return rc;
    if (int rc = dev_alloc(h, &h->tb.bins, (size_t)cap)) return rc;
    if (int rc = dev_alloc(h, &h->tb.esc_dyn, (size_t)n)) return rc;
    if (int rc = dev_alloc(h, &h->tb.esc_static, (size_t)n)) return rc;
    if (int rc = dev_alloc(h, &h->tb.items, (size_t)items)) return rc;
    if (int rc = dev_alloc(h, &h->tb.part, (size_t)items * 2 * kTileBinsMax)) return rc;
    h->tb_cells = n;
    h->tb_cap = cap;
    h->tb_items = (int)items;
    h->tb_force = true;
    return EPB_OK;
}

bool same_view(const CellView& a, const CellView& b) {
    return same_cells(a, b) && a.y == b.y && a.oy == b.oy && a.sy == b.sy && a.ratio == b.ratio;
}

// The list maintenance of a forward: rebuild when needed (on the device: the
// kernels return at once otherwise), then validate the lists against the
// positions now.  A view other than the lists' forces a rebuild.
int tile_prepare(epb_handle* h, const CellView& v, cudaStream_t st) {
    if (int rc = tile_reserve(h, std::max<int64_t>(v.n, 1), st)) return rc;
    for (int64_t e : {v.b0 + v.n0, v.b1 + (v.n - v.n0)})
        if (e > (int64_t)kNodeMask) return fail(h, EPB_EINVAL, "node indices must be below 2^30");
    // a shard rebuilds its band's lists every call: a cell may have moved in from
    // another band, which this band's lists cannot see
    const bool force = h->P > 1 || h->tb_force || !h->tb_valid || !same_view(h->tb_key, v);
    k_tile_decide<<<1, 32, 0, st>>>(h->tb, force ? 1 : 0);
    EPB_LAUNCHED(h, "k_tile_decide launch");
    const GridGeom g = geom(h);
    k_rebuild_count<<<fixed_blocks(h), 256, 0, st>>>(v, g, h->tg, h->tb, h->flags);
    EPB_LAUNCHED(h, "k_rebuild_count launch");
    k_rebuild_scan<<<1, kScanThreads, 0, st>>>(h->ntiles, h->tb);
    EPB_LAUNCHED(h, "k_rebuild_scan launch");
    k_rebuild_fill<<<fixed_blocks(h), 256, 0, st>>>(v, g, h->tg, h->tb);
    EPB_LAUNCHED(h, "k_rebuild_fill launch");
    k_validate<<<fixed_blocks(h), 256, 0, st>>>(v, g, h->tb);
    EPB_LAUNCHED(h, "k_validate launch");
    h->tb_force = false;
    h->tb_stale = false;
    h->tb_key = v;
    h->tb_valid = true;
    return EPB_OK;
}

// Overflow request of a tile scatter: the overflow cells are the nodes of the
// two ranges set0; their map's overflow terms go to out[2].
struct TileOverflow {
    int64_t set0[4];
    float target;
    double* out;
};

// Density of the listed cells (plus the initial density) into rho [band rows * N]
// (nullable with an overflow request).
int tile_scatter(epb_handle* h, const CellView& v, float* rho, cudaStream_t st, const TileOverflow* ovf = nullptr) {
    if (ovf && !h->esc_grid0) {
        // scratch of the overflow variant (allocated once; the first call synchronises)
        EPB_CUDA(h, cudaStreamSynchronize(st));
        const size_t MN = (size_t)h->RB * h->N;
        if (int rc = dev_alloc(h, &h->esc_grid0, MN)) return rc;
        if (int rc = dev_alloc(h, &h->tile_ovf_part, 2 * (size_t)h->ntiles)) return rc;
        if (int rc = dev_alloc(h, &h->tile_ovf_counter, 1)) return rc;
        EPB_CUDA(h, cudaMemset(h->esc_grid0, 0, MN * sizeof(unsigned long long)));
        EPB_CUDA(h, cudaMemset(h->tile_ovf_counter, 0, sizeof(unsigned)));
    }
    const int64_t* s0 = ovf ? ovf->set0 : nullptr;
    k_esc_scatter<<<(unsigned)(2 * h->sms), 256, 0, st>>>(v, geom(h), h->tg, ldexpf(1.0f, h->S), h->tb,
                                                          ovf ? h->esc_grid0 : nullptr, s0 ? s0[0] : 0, s0 ? s0[1] : 0,
                                                          s0 ? s0[2] : 0, s0 ? s0[3] : 0);
    EPB_LAUNCHED(h, "k_esc_scatter launch");
    TileScatterArgs a;
    a.g = geom(h);
    a.t = h->tg;
    a.b = h->tb;
    a.qscale = ldexpf(1.0f, h->S);
    a.dscale = h->dscale;
    a.init = h->has_init ? h->init : nullptr;
    a.rho = rho;
    a.flags = h->flags;
    if (ovf) {
        for (int k = 0; k < 4; ++k) a.set0[k] = ovf->set0[k];
        a.target = ovf->target;
        a.bin_area = (double)h->bsx * (double)h->bsy;
        a.ovf_part = h->tile_ovf_part;
        a.ovf_counter = h->tile_ovf_counter;
        a.ovf_out = ovf->out;
        a.esc_grid0 = h->esc_grid0;
        k_tile_scatter<true><<<h->tile_grid_ovf, kTileThreads, 0, st>>>(a);
    } else {
        k_tile_scatter<false><<<h->tile_grid, kTileThreads, 0, st>>>(a);
    }
    EPB_LAUNCHED(h, "k_tile_scatter launch");
    return EPB_OK;
}

// Gradients of the cells of v from the interleaved fields fxy (rows [row0,
// row0 + RB + halo)): the positions of the last forward on the same cell
// arrays; other arrays are listed first.  owned_only: only the cells whose
// first bin row is in the band are written (a shard).
int tile_gather(epb_handle* h, const CellView& v, const float2* fxy, int halo, int owned_only, const float* grad_out,
                float* grad_x, float* grad_y, cudaStream_t st) {
    if (!h->tb_valid || h->tb_stale || !same_view(h->tb_key, v))
        if (int rc = tile_prepare(h, v, st)) return rc;
    TileGatherArgs a;
    a.g = geom(h);
    a.t = h->tg;
    a.b = h->tb;
    a.fxy = fxy;
    a.halo = halo;
    a.grad_out = grad_out;
    a.grad_x = grad_x;
    a.grad_y = grad_y;
    a.flags = h->flags;
    EPB_CUDA(h, cudaMemsetAsync(h->tb.meta + kMetaWorkGather, 0, sizeof(int), st));
    k_tile_gather<<<h->tile_grid, kTileThreads, 0, st>>>(a);
    EPB_LAUNCHED(h, "k_tile_gather launch");
    k_esc_gather<<<(unsigned)(2 * h->sms), 256, 0, st>>>(v, geom(h), h->tg, h->tb, fxy, halo, owned_only, grad_out,
                                                         grad_x, grad_y, h->flags);
    EPB_LAUNCHED(h, "k_esc_gather launch");
    return EPB_OK;
}

}  // namespace

extern "C" {

const char* epb_version(void) { return "epb200 1.0 (sm_100a)"; }

const char* epb_status_string(int s) {
    switch (s) {
        case EPB_OK: return "ok";
        case EPB_EINVAL: return "invalid argument";
        case EPB_ECUDA: return "CUDA error";
        case EPB_ENCCL: return "NCCL error";
        case EPB_ETIMEOUT: return "timeout";
        case EPB_EOVERFLOW: return "fixed-point density saturated";
        case EPB_ENOSTATE: return "no forward state";
        default: return "unknown status";
    }
}

}  // extern "C"

namespace {

// Shared by epb_create and epb_create_shard.
int create_handle(const epb_config* cfg, int P, int p, epb_handle** out) {
    if (!out) return EPB_EINVAL;
    *out = nullptr;
    if (!cfg) return EPB_EINVAL;
    if (!pow2_in_range(cfg->num_bins_x) || !pow2_in_range(cfg->num_bins_y)) return EPB_EINVAL;
    if (!(cfg->xh > cfg->xl) || !(cfg->yh > cfg->yl) || !std::isfinite(cfg->xl) || !std::isfinite(cfg->xh) ||
        !std::isfinite(cfg->yl) || !std::isfinite(cfg->yh))
        return EPB_EINVAL;
    if ((cfg->flags & ~(EPB_CONFIG_CELL_ORDER | EPB_CONFIG_TILES)) != 0 ||
        (cfg->flags & EPB_CONFIG_CELL_ORDER) && (cfg->flags & EPB_CONFIG_TILES) || cfg->fixed_point_bits > 60)
        return EPB_EINVAL;
    // shards: P a power of two, each band at least 16 rows / columns
    if (P < 1 || p < 0 || p >= P || (P & (P - 1)) != 0) return EPB_EINVAL;
    if (cfg->num_bins_x / P < 16 || cfg->num_bins_y / P < 16) return EPB_EINVAL;
    epb_handle* h = new epb_handle();
    h->dev = cfg->device;
    h->M = cfg->num_bins_x; h->N = cfg->num_bins_y;
    h->P = P; h->p = p;
    h->RB = h->M / P; h->NB = h->N / P;
    h->row0 = p * h->RB; h->col0 = p * h->NB;
    h->xl = cfg->xl; h->yl = cfg->yl; h->xh = cfg->xh; h->yh = cfg->yh;
    // fp32 bin sizes as the reference server computes them (host:411)
    h->bsx = ((float)cfg->xh - (float)cfg->xl) / (float)h->M;
    h->bsy = ((float)cfg->yh - (float)cfg->yl) / (float)h->N;
    if (cfg->fixed_point_bits > 0) {
        h->S = cfg->fixed_point_bits;
    } else {
        const double area = (cfg->xh - cfg->xl) * (cfg->yh - cfg->yl);
        int ib = (int)std::ceil(std::log2(area > 1.0 ? area : 1.0)) + 1;
        if (ib < 32) ib = 32;
        h->S = 63 - ib;
    }
    h->dscale = std::ldexp(1.0, -h->S) / ((double)h->bsx * (double)h->bsy);
    // cell order unless the tiles are asked for (measured faster on one GPU and on shards)
    h->cell_order = (cfg->flags & EPB_CONFIG_TILES) == 0;
    h->tg.ltx = ilog2(std::min(kTileMax, h->RB));
    h->tg.lty = ilog2(std::min(kTileMax, h->N));
    h->tg.ntx = h->RB >> h->tg.ltx;
    h->tg.nty = h->N >> h->tg.lty;
    h->tg.row0 = h->row0;
    h->tg.rows = h->RB;
    h->tg.margin = P == 1 ? kTileMargin : 0;
    h->ntiles = h->tg.ntx * h->tg.nty;

    DeviceGuard guard(h->dev);
    if (!guard.ok) { delete h; return EPB_ECUDA; }
    const size_t MN = (size_t)h->M * h->N;
    const size_t band = (size_t)h->RB * h->N;
    int rc = EPB_OK;
    const int ncolb = col_blocks(h->M, h->N);
    if (!rc) rc = dev_alloc(h, &h->grid, band);
    if (!rc) rc = dev_alloc(h, &h->init, band);
    if (P == 1) {
        if (!rc) rc = dev_alloc(h, &h->t1, MN);
        if (!rc) rc = dev_alloc(h, &h->g, kColOutputs * MN);
        if (!rc) rc = dev_alloc(h, &h->fxy, MN);
    }
    if (!rc) rc = dev_alloc(h, &h->twM, (size_t)std::max(1, tw_table_size(h->M)));
    if (!rc) rc = dev_alloc(h, &h->qwM, (size_t)h->M);
    if (!rc) rc = dev_alloc(h, &h->twN, (size_t)std::max(1, tw_table_size(h->N)));
    if (!rc) rc = dev_alloc(h, &h->qwN, (size_t)h->N);
    if (!rc) rc = dev_alloc(h, &h->partials, 2 * (size_t)ncolb);  // room for the half-size column CTAs
    if (!rc) rc = dev_alloc(h, &h->counter, 1);
    if (!rc) rc = dev_alloc(h, &h->energy_d, 1);
    if (!rc) rc = dev_alloc(h, &h->flags, 1);
    if (!rc) rc = dev_alloc(h, &h->ovf_partials, 2 * (size_t)kOvfMaxBlocks);
    if (!rc) rc = dev_alloc(h, &h->ovf_counter, 1);
    if (!rc) rc = dev_alloc(h, &h->linf_bits, 1);
    if (!h->cell_order) {
        if (!rc) rc = dev_alloc(h, &h->tb.cnt, (size_t)h->ntiles * kCounterStride);
        if (!rc) rc = dev_alloc(h, &h->tb.cur, (size_t)h->ntiles * kCounterStride);
        if (!rc) rc = dev_alloc(h, &h->tb.start, (size_t)h->ntiles + 1);
        if (!rc) rc = dev_alloc(h, &h->tb.nown, (size_t)h->ntiles);
        if (!rc) rc = dev_alloc(h, &h->tb.first_item, (size_t)h->ntiles);
        if (!rc) rc = dev_alloc(h, &h->tb.arrive, (size_t)h->ntiles);
        if (!rc) rc = dev_alloc(h, &h->tb.meta, (size_t)kMetaWords);
        if (!rc) rc = dev_alloc(h, &h->tb.esc_grid, band);
        if (!rc) rc = dev_alloc(h, &h->rho, band);
    }
    if (rc) { free_all(h); delete h; return rc; }

    std::vector<float2> tw, qw;
    cudaError_t e = cudaSuccess;
    host_tables(h->M, tw, qw);
    if (e == cudaSuccess) e = cudaMemcpy(h->twM, tw.data(), tw.size() * sizeof(float2), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(h->qwM, qw.data(), qw.size() * sizeof(float2), cudaMemcpyHostToDevice);
    host_tables(h->N, tw, qw);
    if (e == cudaSuccess) e = cudaMemcpy(h->twN, tw.data(), tw.size() * sizeof(float2), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(h->qwN, qw.data(), qw.size() * sizeof(float2), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemset(h->grid, 0, band * sizeof(long long));
    if (e == cudaSuccess) e = cudaMemset(h->counter, 0, sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMemset(h->ovf_counter, 0, sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMemset(h->flags, 0, sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMemset(h->energy_d, 0, sizeof(double));
    if (!h->cell_order) {
        if (e == cudaSuccess) e = cudaMemset(h->tb.cnt, 0, (size_t)h->ntiles * kCounterStride * sizeof(int));
        if (e == cudaSuccess) e = cudaMemset(h->tb.arrive, 0, (size_t)h->ntiles * sizeof(unsigned));
        if (e == cudaSuccess) e = cudaMemset(h->tb.meta, 0, kMetaWords * sizeof(int));
        if (e == cudaSuccess) e = cudaMemset(h->tb.esc_grid, 0, band * sizeof(unsigned long long));
    }
    int sms = 0, occ0 = 0, occ1 = 0;
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, h->dev);
    h->sms = std::max(1, sms);
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ0, k_gather<false>, 256, 0);
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ1, k_gather<true>, 256, 0);
    h->gather_grid[0] = (unsigned)std::max(1, sms * occ0 * EPB_GATHER_WAVES);
    h->gather_grid[1] = (unsigned)std::max(1, sms * occ1 * EPB_GATHER_WAVES);
    int occ_ts = 0, occ_tg = 0, occ_to = 0;
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ_ts, k_tile_scatter<false>, kTileThreads, 0);
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ_tg, k_tile_gather, kTileThreads, 0);
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ_to, k_tile_scatter<true>, kTileThreads, 0);
    h->tile_grid = (unsigned)std::max(1, sms * std::max(1, std::min(occ_ts, occ_tg)));
    h->tile_grid_ovf = (unsigned)std::max(1, sms * std::max(1, occ_to));
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) { free_all(h); delete h; return EPB_ECUDA; }
    *out = h;
    return EPB_OK;
}

int whole_grid_only(epb_handle* h) {
    if (h->P != 1) return fail(h, EPB_EINVAL, "this entry point needs a whole-grid handle (epb_create); "
                                              "use the epb_shard_* stages on a shard handle");
    return EPB_OK;
}

}  // namespace

extern "C" {

int epb_create(const epb_config* cfg, epb_handle** out) { return create_handle(cfg, 1, 0, out); }

int epb_create_shard(const epb_config* cfg, int32_t num_shards, int32_t shard, epb_handle** out) {
    return create_handle(cfg, num_shards, shard, out);
}

int epb_destroy(epb_handle* h) {
    if (!h) return EPB_EINVAL;
    {
        DeviceGuard guard(h->dev);
        cudaDeviceSynchronize();
        free_all(h);
    }
    delete h;
    return EPB_OK;
}

const char* epb_last_error(const epb_handle* h) { return h ? h->err.c_str() : "null handle"; }

int epb_geometry(const epb_handle* h, float* bsx, float* bsy, int32_t* bits) {
    if (!h) return EPB_EINVAL;
    if (bsx) *bsx = h->bsx;
    if (bsy) *bsy = h->bsy;
    if (bits) *bits = h->S;
    return EPB_OK;
}

int epb_set_initial_density(epb_handle* h, const float* init_norm, epb_stream stream) {
    if (!h) return EPB_EINVAL;
    DeviceGuard guard(h->dev);
    if (!init_norm) { h->has_init = false; return EPB_OK; }
    // a shard keeps only its own rows of the [M][N] map
    EPB_CUDA(h, cudaMemcpyAsync(h->init, init_norm + (size_t)h->row0 * h->N, (size_t)h->RB * h->N * sizeof(float),
                                cudaMemcpyDeviceToDevice, (cudaStream_t)stream));
    h->has_init = true;
    return EPB_OK;
}

int epb_forward(epb_handle* h, const epb_cells* cells, epb_stream stream, float* density, float* potential,
                float* field_x, float* field_y, float* energy) {
    if (!h) return EPB_EINVAL;
    if (int rc = whole_grid_only(h)) return rc;
    CellView v;
    if (int rc = make_view(h, cells, v)) return rc;
    DeviceGuard guard(h->dev);
    cudaStream_t st = (cudaStream_t)stream;
    if (!h->cell_order) {
        // cell tiles: bin, then every tile writes its finished density bins
        ProfCall pc(h, st);
        pc.begin();
        if (int rc = tile_prepare(h, v, st)) return rc;
        pc.end_stage(EPB_STAGE_BIN);
        float* rho = density ? density : h->rho;
        if (int rc = tile_scatter(h, v, rho, st)) return rc;
        pc.end_stage(EPB_STAGE_SCATTER);
        if (int rc = launch_row_fwd(h, false, rho, nullptr, blocked(h->t1, 0, 1), 0, st)) return rc;
        pc.end_stage(EPB_STAGE_ROW_FWD);
        return solve_from_t1(h, st, potential, field_x, field_y, energy, pc);
    }
    if (h->grid_dirty) {
        EPB_CUDA(h, cudaMemsetAsync(h->grid, 0, (size_t)h->M * h->N * sizeof(long long), st));
        h->grid_dirty = false;
    }
    h->grid_dirty = true;  // until the row pass has consumed and re-zeroed it
    ProfCall pc(h, st);
    pc.begin();
    if (int rc = scatter_into(h, v, st, h->grid)) return rc;
    pc.end_stage(EPB_STAGE_SCATTER);
    if (int rc = launch_row_fwd(h, true, nullptr, density, blocked(h->t1, 0, 1), 0, st)) return rc;
    pc.end_stage(EPB_STAGE_ROW_FWD);
    h->grid_dirty = false;
    return solve_from_t1(h, st, potential, field_x, field_y, energy, pc);
}

int epb_backward(epb_handle* h, const epb_cells* cells, const float* grad_out, epb_stream stream,
                 float* grad_x, float* grad_y) {
    if (!h) return EPB_EINVAL;
    if (int rc = whole_grid_only(h)) return rc;
    if (!h->have_fields) return fail(h, EPB_ENOSTATE, "epb_backward before epb_forward");
    CellView v;
    if (int rc = make_view(h, cells, v)) return rc;
    if (v.n > 0 && (!grad_x || !grad_y)) return fail(h, EPB_EINVAL, "grad_x/grad_y must be non-NULL");
    if (v.n == 0) return EPB_OK;
    DeviceGuard guard(h->dev);
    ProfCall pc(h, (cudaStream_t)stream);
    pc.begin();
    if (!h->cell_order) {
        if (int rc = tile_gather(h, v, h->fxy, 0, 0, grad_out, grad_x, grad_y, (cudaStream_t)stream)) return rc;
        pc.end_stage(EPB_STAGE_GATHER);
        return EPB_OK;
    }
    k_gather<false><<<gather_blocks(h, v.n, false), 256, 0, (cudaStream_t)stream>>>(v, geom(h), h->fxy, nullptr, nullptr, 0, h->M, 0, 0,
                                                               grad_out, grad_x, grad_y, h->flags);
    EPB_LAUNCHED(h, "k_gather launch");
    pc.end_stage(EPB_STAGE_GATHER);
    return EPB_OK;
}

int epb_scatter_fixed(epb_handle* h, const epb_cells* cells, epb_stream stream, int64_t* grid) {
    if (!h) return EPB_EINVAL;
    if (int rc = whole_grid_only(h)) return rc;
    if (!grid) return fail(h, EPB_EINVAL, "grid is NULL");
    CellView v;
    if (int rc = make_view(h, cells, v)) return rc;
    DeviceGuard guard(h->dev);
    cudaStream_t st = (cudaStream_t)stream;
    EPB_CUDA(h, cudaMemsetAsync(grid, 0, (size_t)h->M * h->N * sizeof(int64_t), st));
    ProfCall pc(h, st);
    pc.begin();
    if (int rc = scatter_into(h, v, st, (long long*)grid)) return rc;
    pc.end_stage(EPB_STAGE_SCATTER);
    return EPB_OK;
}

int epb_dct_solve(epb_handle* h, const float* density, epb_stream stream, float* potential, float* field_x,
                  float* field_y, float* energy) {
    if (!h) return EPB_EINVAL;
    if (int rc = whole_grid_only(h)) return rc;
    if (!density) return fail(h, EPB_EINVAL, "density is NULL");
    DeviceGuard guard(h->dev);
    cudaStream_t st = (cudaStream_t)stream;
    ProfCall pc(h, st);
    pc.begin();
    if (int rc = launch_row_fwd(h, false, density, nullptr, blocked(h->t1, 0, 1), 0, st)) return rc;
    pc.end_stage(EPB_STAGE_ROW_FWD);
    return solve_from_t1(h, st, potential, field_x, field_y, energy, pc);
}

int epb_gather(epb_handle* h, const epb_cells* cells, const float* field_x, const float* field_y,
               const float* grad_out, epb_stream stream, float* grad_x, float* grad_y) {
    if (!h) return EPB_EINVAL;
    if (int rc = whole_grid_only(h)) return rc;
    if (!field_x || !field_y) return fail(h, EPB_EINVAL, "field maps must be non-NULL");
    CellView v;
    if (int rc = make_view(h, cells, v)) return rc;
    if (v.n > 0 && (!grad_x || !grad_y)) return fail(h, EPB_EINVAL, "grad_x/grad_y must be non-NULL");
    if (v.n == 0) return EPB_OK;
    DeviceGuard guard(h->dev);
    k_gather<false><<<gather_blocks(h, v.n, false), 256, 0, (cudaStream_t)stream>>>(v, geom(h), nullptr, field_x, field_y, 0, h->M, 0, 0,
                                                               grad_out, grad_x, grad_y, h->flags);
    EPB_LAUNCHED(h, "k_gather launch");
    return EPB_OK;
}

namespace {

// The column pass and the row inverse move the exchanged blocks as float4.
bool aligned(const void* p, uintptr_t bytes) { return (reinterpret_cast<uintptr_t>(p) & (bytes - 1)) == 0; }

// Device address of a pinned host buffer (EINVAL when it is not pinned).
int host_device_ptr(epb_handle* h, const void* host, void** dev) {
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, host) != cudaSuccess || at.type != cudaMemoryTypeHost || !at.devicePointer) {
        cudaGetLastError();  // clear the sticky-free error of a failed query
        return fail(h, EPB_EINVAL, "host buffers must be pinned (page-locked) host memory");
    }
    *dev = at.devicePointer;
    return EPB_OK;
}

}  // namespace

int epb_forward_host(epb_handle* h, const epb_cells* cells, const float* host_x, const float* host_y,
                     epb_stream stream, float* density, float* potential, float* field_x, float* field_y,
                     float* energy) {
    if (!h) return EPB_EINVAL;
    if (int rc = whole_grid_only(h)) return rc;
    if (!host_x || !host_y) return fail(h, EPB_EINVAL, "host_x and host_y must be non-NULL");
    CellView v;
    if (int rc = make_view(h, cells, v)) return rc;
    DeviceGuard guard(h->dev);
    cudaStream_t st = (cudaStream_t)stream;
    void *hx = nullptr, *hy = nullptr;
    if (int rc = host_device_ptr(h, host_x, &hx)) return rc;
    if (int rc = host_device_ptr(h, host_y, &hy)) return rc;
    if (!h->cell_order) {
        // the positions of the two node ranges are copied into cells->x / cells->y,
        // then the device path runs on them
        ProfCall pc(h, st);
        pc.begin();
        const int64_t rb[2][2] = {{v.b0, v.n0}, {v.b1, v.n - v.n0}};
        for (const auto& r : rb) {
            if (r[1] == 0) continue;
            EPB_CUDA(h, cudaMemcpyAsync(const_cast<float*>(cells->x) + r[0], host_x + r[0], (size_t)r[1] * sizeof(float),
                                        cudaMemcpyHostToDevice, st));
            EPB_CUDA(h, cudaMemcpyAsync(const_cast<float*>(cells->y) + r[0], host_y + r[0], (size_t)r[1] * sizeof(float),
                                        cudaMemcpyHostToDevice, st));
        }
        if (int rc = tile_prepare(h, v, st)) return rc;
        pc.end_stage(EPB_STAGE_BIN);
        float* rho = density ? density : h->rho;
        if (int rc = tile_scatter(h, v, rho, st)) return rc;
        pc.end_stage(EPB_STAGE_SCATTER);
        if (int rc = launch_row_fwd(h, false, rho, nullptr, blocked(h->t1, 0, 1), 0, st)) return rc;
        pc.end_stage(EPB_STAGE_ROW_FWD);
        return solve_from_t1(h, st, potential, field_x, field_y, energy, pc);
    }
    if (h->grid_dirty) {
        EPB_CUDA(h, cudaMemsetAsync(h->grid, 0, (size_t)h->M * h->N * sizeof(long long), st));
        h->grid_dirty = false;
    }
    h->grid_dirty = true;
    ProfCall pc(h, st);
    pc.begin();
    if (v.n > 0) {
        // positions read straight from host memory over PCIe and kept in cells->x / cells->y
        CellView vh = v;
        vh.x = static_cast<const float*>(hx);
        vh.y = static_cast<const float*>(hy);
        k_scatter<true><<<cell_blocks(v.n), 256, 0, st>>>(vh, geom(h), ldexpf(1.0f, h->S),
                                                          (unsigned long long*)h->grid, 0, h->M, h->flags,
                                                          const_cast<float*>(cells->x), const_cast<float*>(cells->y));
        EPB_LAUNCHED(h, "k_scatter launch");
    }
    pc.end_stage(EPB_STAGE_SCATTER);
    if (int rc = launch_row_fwd(h, true, nullptr, density, blocked(h->t1, 0, 1), 0, st)) return rc;
    pc.end_stage(EPB_STAGE_ROW_FWD);
    h->grid_dirty = false;
    return solve_from_t1(h, st, potential, field_x, field_y, energy, pc);
}

int epb_backward_host(epb_handle* h, const epb_cells* cells, const float* grad_out, epb_stream stream,
                      float* grad_x, float* grad_y, float* host_grad_x, float* host_grad_y) {
    if (!h) return EPB_EINVAL;
    if (int rc = whole_grid_only(h)) return rc;
    if (!h->have_fields) return fail(h, EPB_ENOSTATE, "epb_backward_host before a forward");
    if (!grad_x || !grad_y || !host_grad_x || !host_grad_y)
        return fail(h, EPB_EINVAL, "grad_x, grad_y, host_grad_x and host_grad_y must be non-NULL");
    CellView v;
    if (int rc = make_view(h, cells, v)) return rc;
    DeviceGuard guard(h->dev);
    cudaStream_t st = (cudaStream_t)stream;
    void *hgx = nullptr, *hgy = nullptr;
    if (int rc = host_device_ptr(h, host_grad_x, &hgx)) return rc;
    if (int rc = host_device_ptr(h, host_grad_y, &hgy)) return rc;
    if (v.n == 0) return EPB_OK;
    ProfCall pc(h, st);
    pc.begin();
    if (!h->cell_order) {
        // gradients into the device arrays, then each node range to host memory
        if (int rc = tile_gather(h, v, h->fxy, 0, 0, grad_out, grad_x, grad_y, st)) return rc;
        const int64_t rb[2][2] = {{v.b0, v.n0}, {v.b1, v.n - v.n0}};
        for (const auto& r : rb) {
            if (r[1] == 0) continue;
            EPB_CUDA(h, cudaMemcpyAsync(host_grad_x + r[0], grad_x + r[0], (size_t)r[1] * sizeof(float),
                                        cudaMemcpyDeviceToHost, st));
            EPB_CUDA(h, cudaMemcpyAsync(host_grad_y + r[0], grad_y + r[0], (size_t)r[1] * sizeof(float),
                                        cudaMemcpyDeviceToHost, st));
        }
        pc.end_stage(EPB_STAGE_GATHER);
        return EPB_OK;
    }
    k_gather<true><<<gather_blocks(h, v.n, true), 256, 0, st>>>(v, geom(h), h->fxy, nullptr, nullptr, 0, h->M, 0, 0, grad_out,
                                                     grad_x, grad_y, h->flags, static_cast<float*>(hgx),
                                                     static_cast<float*>(hgy));
    EPB_LAUNCHED(h, "k_gather launch");
    pc.end_stage(EPB_STAGE_GATHER);
    return EPB_OK;
}

int epb_overflow(epb_handle* h, const epb_cells* cells, float target_density, epb_stream stream, double* out) {
    if (!h) return EPB_EINVAL;
    if (!out) return fail(h, EPB_EINVAL, "out is NULL");
    if (!std::isfinite(target_density)) return fail(h, EPB_EINVAL, "target_density must be finite");
    CellView v;
    if (int rc = make_view(h, cells, v)) return rc;
    DeviceGuard guard(h->dev);
    cudaStream_t st = (cudaStream_t)stream;
    if (!h->cell_order) {
        // every cell given is an overflow cell; no density map is written
        if (int rc = tile_prepare(h, v, st)) return rc;
        TileOverflow ov{{v.b0, v.b0 + v.n0, v.b1, v.b1 + (v.n - v.n0)}, target_density, out};
        return tile_scatter(h, v, nullptr, st, &ov);
    }
    const int64_t nbins = (int64_t)h->RB * h->N;
    if (h->grid_dirty) {
        EPB_CUDA(h, cudaMemsetAsync(h->grid, 0, (size_t)nbins * sizeof(long long), st));
        h->grid_dirty = false;
    }
    h->grid_dirty = true;  // until k_overflow has consumed and re-zeroed it
    if (int rc = scatter_into(h, v, st, h->grid)) return rc;
    k_overflow<<<ovf_blocks(nbins), kOvfThreads, 0, st>>>(h->grid, h->has_init ? h->init : nullptr, h->dscale, nbins,
                                                          target_density, (double)h->bsx * (double)h->bsy,
                                                          h->ovf_partials, h->ovf_counter, out, nullptr, h->flags);
    EPB_LAUNCHED(h, "k_overflow launch");
    h->grid_dirty = false;
    return EPB_OK;
}

int epb_forward_overflow(epb_handle* h, const epb_cells* cells, float target_density, epb_stream stream,
                         double* overflow, float* density, float* potential, float* field_x, float* field_y,
                         float* energy) {
    if (!h) return EPB_EINVAL;
    if (int rc = whole_grid_only(h)) return rc;
    if (!overflow) return fail(h, EPB_EINVAL, "overflow is NULL");
    if (!std::isfinite(target_density)) return fail(h, EPB_EINVAL, "target_density must be finite");
    CellView v;
    if (int rc = make_view(h, cells, v)) return rc;
    DeviceGuard guard(h->dev);
    cudaStream_t st = (cudaStream_t)stream;
    if (!h->cell_order) {
        // one set of lists for both ranges; the tiles sum the first range apart for its overflow
        ProfCall pc(h, st);
        pc.begin();
        if (int rc = tile_prepare(h, v, st)) return rc;
        pc.end_stage(EPB_STAGE_BIN);
        float* rho = density ? density : h->rho;
        TileOverflow ov{{v.b0, v.b0 + v.n0, 0, 0}, target_density, overflow};
        if (int rc = tile_scatter(h, v, rho, st, &ov)) return rc;
        pc.end_stage(EPB_STAGE_SCATTER);
        if (int rc = launch_row_fwd(h, false, rho, nullptr, blocked(h->t1, 0, 1), 0, st)) return rc;
        pc.end_stage(EPB_STAGE_ROW_FWD);
        return solve_from_t1(h, st, potential, field_x, field_y, energy, pc);
    }
    const int64_t nbins = (int64_t)h->M * h->N;
    if (!h->grid2) {
        // second grid for the first range (allocated once; the first call synchronises)
        EPB_CUDA(h, cudaStreamSynchronize(st));
        if (int rc = dev_alloc(h, &h->grid2, (size_t)nbins)) return rc;
        EPB_CUDA(h, cudaMemset(h->grid2, 0, (size_t)nbins * sizeof(long long)));
    }
    if (h->grid_dirty) {
        EPB_CUDA(h, cudaMemsetAsync(h->grid, 0, (size_t)nbins * sizeof(long long), st));
        EPB_CUDA(h, cudaMemsetAsync(h->grid2, 0, (size_t)nbins * sizeof(long long), st));
        h->grid_dirty = false;
    }
    h->grid_dirty = true;  // until the row pass has consumed and re-zeroed the grids
    // first range -> grid2 (its overflow), second range -> grid; then grid += grid2
    CellView v0 = v, v1 = v;
    v0.n = v.n0;
    v1.b0 = v.b1; v1.n0 = v.n - v.n0; v1.n = v.n - v.n0;
    ProfCall pc(h, st);
    pc.begin();
    if (int rc = scatter_into(h, v0, st, h->grid2)) return rc;
    if (int rc = scatter_into(h, v1, st, h->grid)) return rc;
    k_overflow<<<ovf_blocks(nbins), kOvfThreads, 0, st>>>(h->grid2, h->has_init ? h->init : nullptr, h->dscale, nbins,
                                                          target_density, (double)h->bsx * (double)h->bsy,
                                                          h->ovf_partials, h->ovf_counter, overflow, h->grid,
                                                          h->flags);
    EPB_LAUNCHED(h, "k_overflow launch");
    pc.end_stage(EPB_STAGE_SCATTER);
    if (int rc = launch_row_fwd(h, true, nullptr, density, blocked(h->t1, 0, 1), 0, st)) return rc;
    pc.end_stage(EPB_STAGE_ROW_FWD);
    h->grid_dirty = false;
    return solve_from_t1(h, st, potential, field_x, field_y, energy, pc);
}

int epb_descent_step(epb_handle* h, const epb_cells* cells, float* x, float* y, const float* grad_x,
                     const float* grad_y, const float* width, const float* height, float step_bins,
                     epb_stream stream, float* grad_linf) {
    if (!h) return EPB_EINVAL;
    CellView v;
    if (int rc = make_view(h, cells, v)) return rc;
    if (!std::isfinite(step_bins) || step_bins < 0.0f) return fail(h, EPB_EINVAL, "step_bins must be finite and >= 0");
    if (v.n > 0 && (!x || !y || !grad_x || !grad_y || !width || !height))
        return fail(h, EPB_EINVAL, "x, y, grad_x, grad_y, width and height must be non-NULL");
    DeviceGuard guard(h->dev);
    cudaStream_t st = (cudaStream_t)stream;
    EPB_CUDA(h, cudaMemsetAsync(h->linf_bits, 0, sizeof(unsigned), st));
    h->bl_stale = true;    // positions move: a gather before the next forward checks the band list first
    // the tile lists stay (every forward validates them against the positions it is
    // given); a gather before the next forward validates them first
    h->tb_stale = true;
    if (v.n > 0) {
        k_grad_linf<<<cell_blocks(v.n), 256, 0, st>>>(v, grad_x, grad_y, h->linf_bits, h->flags);
        EPB_LAUNCHED(h, "k_grad_linf launch");
    }
    // the step lengths as fp32 products, the same rounding as the CPU restatement
    const float step_x = step_bins * h->bsx, step_y = step_bins * h->bsy;
    k_descent<<<cell_blocks(v.n), 256, 0, st>>>(v, x, y, grad_x, grad_y, width, height, h->linf_bits, step_x, step_y,
                                                (float)h->xl, (float)h->yl, (float)h->xh, (float)h->yh, grad_linf);
    EPB_LAUNCHED(h, "k_descent launch");
    return EPB_OK;
}

int epb_error_flags(epb_handle* h, epb_stream stream, uint32_t* flags) {
    if (!h) return EPB_EINVAL;
    DeviceGuard guard(h->dev);
    unsigned f = 0;
    cudaStream_t st = (cudaStream_t)stream;
    EPB_CUDA(h, cudaMemcpyAsync(&f, h->flags, sizeof(unsigned), cudaMemcpyDeviceToHost, st));
    EPB_CUDA(h, cudaStreamSynchronize(st));
    EPB_CUDA(h, cudaMemsetAsync(h->flags, 0, sizeof(unsigned), st));
    EPB_CUDA(h, cudaStreamSynchronize(st));
    if (flags) *flags = f;
    if (f & EPB_FLAG_TIMEOUT) return fail(h, EPB_ETIMEOUT, "a wait for another GPU's signal gave up");
    if (f & EPB_FLAG_SATURATED) return fail(h, EPB_EOVERFLOW, "fixed-point density saturated");
    return EPB_OK;
}

int epb_shard_geometry(const epb_handle* h, int32_t* num_shards, int32_t* shard, int32_t* rows_per_band,
                       int32_t* cols_per_band) {
    if (!h) return EPB_EINVAL;
    if (num_shards) *num_shards = h->P;
    if (shard) *shard = h->p;
    if (rows_per_band) *rows_per_band = h->RB;
    if (cols_per_band) *cols_per_band = h->NB;
    return EPB_OK;
}

int epb_shard_rows_forward(epb_handle* h, const epb_cells* cells, epb_stream stream, float* density_band,
                           float* t1_send) {
    if (!h) return EPB_EINVAL;
    if (!t1_send) return fail(h, EPB_EINVAL, "t1_send is NULL");
    CellView v;
    if (int rc = make_view(h, cells, v)) return rc;
    DeviceGuard guard(h->dev);
    cudaStream_t st = (cudaStream_t)stream;
    if (!h->cell_order) {
        // the band's cell tiles: its density, then the row DCT blocks
        ProfCall pc(h, st);
        pc.begin();
        if (int rc = tile_prepare(h, v, st)) return rc;
        pc.end_stage(EPB_STAGE_BIN);
        float* rho = density_band ? density_band : h->rho;
        if (int rc = tile_scatter(h, v, rho, st)) return rc;
        pc.end_stage(EPB_STAGE_SCATTER);
        if (int rc = launch_row_fwd(h, false, rho, nullptr, blocked(t1_send, (int64_t)h->RB * h->NB, h->P), 0, st))
            return rc;
        pc.end_stage(EPB_STAGE_ROW_FWD);
        return EPB_OK;
    }
    if (h->grid_dirty) {
        EPB_CUDA(h, cudaMemsetAsync(h->grid, 0, (size_t)h->RB * h->N * sizeof(long long), st));
        h->grid_dirty = false;
    }
    h->grid_dirty = true;
    ProfCall pc(h, st);
    pc.begin();
    if (int rc = scatter_into(h, v, st, h->grid)) return rc;
    pc.end_stage(EPB_STAGE_SCATTER);
    if (int rc = launch_row_fwd(h, true, nullptr, density_band, blocked(t1_send, (int64_t)h->RB * h->NB, h->P), 0,
                                st))
        return rc;
    pc.end_stage(EPB_STAGE_ROW_FWD);
    h->grid_dirty = false;
    return EPB_OK;
}

int epb_shard_columns(epb_handle* h, const float* t1_recv, epb_stream stream, float* g_send, int32_t want_potential,
                      double* energy_partial) {
    if (!h) return EPB_EINVAL;
    if (!t1_recv || !g_send) return fail(h, EPB_EINVAL, "t1_recv and g_send must be non-NULL");
    if (!aligned(t1_recv, 16) || !aligned(g_send, 16))
        return fail(h, EPB_EINVAL, "t1_recv and g_send must be 16-byte aligned");
    DeviceGuard guard(h->dev);
    cudaStream_t st = (cudaStream_t)stream;
    ProfCall pc(h, st);
    pc.begin();
    (void)want_potential;  // the column pass produces the potential form in every case
    if (int rc = launch_columns(h, t1_recv, blocked(g_send, kColOutputs * (int64_t)h->RB * h->NB, h->P), nullptr, st))
        return rc;
    pc.end_stage(EPB_STAGE_COLUMN);
    if (energy_partial)
        EPB_CUDA(h, cudaMemcpyAsync(energy_partial, h->energy_d, sizeof(double), cudaMemcpyDeviceToDevice, st));
    return EPB_OK;
}

int epb_shard_rows_inverse(epb_handle* h, const float* g_recv, epb_stream stream, float* potential_band,
                           float* field_x_band, float* field_y_band, float* fxy_band) {
    if (!h) return EPB_EINVAL;
    if (!g_recv || !fxy_band) return fail(h, EPB_EINVAL, "g_recv and fxy_band must be non-NULL");
    if (!aligned(g_recv, 16) || !aligned(fxy_band, 8))
        return fail(h, EPB_EINVAL, "g_recv must be 16-byte and fxy_band 8-byte aligned");
    DeviceGuard guard(h->dev);
    cudaStream_t st = (cudaStream_t)stream;
    ProfCall pc(h, st);
    pc.begin();
    if (int rc = launch_rows_inverse(h, g_recv, potential_band, field_x_band, field_y_band,
                                     reinterpret_cast<float2*>(fxy_band), potential_band != nullptr, st))
        return rc;
    pc.end_stage(EPB_STAGE_ROW_INV);
    return EPB_OK;
}

int epb_shard_gather(epb_handle* h, const epb_cells* cells, const float* fxy_ext, int32_t halo_rows,
                     const float* grad_out, epb_stream stream, float* grad_x, float* grad_y) {
    if (!h) return EPB_EINVAL;
    if (!fxy_ext) return fail(h, EPB_EINVAL, "fxy_ext is NULL");
    if (halo_rows < 0 || h->row0 + h->RB + halo_rows > h->M)
        return fail(h, EPB_EINVAL, "halo_rows must keep the extended band inside the grid");
    CellView v;
    if (int rc = make_view(h, cells, v)) return rc;
    if (v.n > 0 && (!grad_x || !grad_y)) return fail(h, EPB_EINVAL, "grad_x/grad_y must be non-NULL");
    if (v.n == 0) return EPB_OK;
    DeviceGuard guard(h->dev);
    cudaStream_t st = (cudaStream_t)stream;
    ProfCall pc(h, st);
    pc.begin();
    if (int rc = shard_gather(h, v, reinterpret_cast<const float2*>(fxy_ext), halo_rows, grad_out, grad_x, grad_y, st))
        return rc;
    pc.end_stage(EPB_STAGE_GATHER);
    return EPB_OK;
}

// ---- peer transport -------------------------------------------------------

int epb_shard_peer_buffers(epb_handle* h, int32_t halo_rows, void* handles_out) {
    if (!h || !handles_out) return EPB_EINVAL;
    if (h->P > kMaxShards) return fail(h, EPB_EINVAL, "at most 8 shards");
    if (halo_rows < 0 || halo_rows > h->RB) return fail(h, EPB_EINVAL, "halo_rows must be in [0, rows per band]");
    if (h->p_t1) return fail(h, EPB_EINVAL, "peer buffers already created");
    DeviceGuard guard(h->dev);
    const size_t strip = (size_t)h->M * h->NB;
    h->p_halo_max = halo_rows;
    h->p_halo = h->p == h->P - 1 ? 0 : halo_rows;
    const size_t sig_bytes = 3 * kMaxShards * sizeof(unsigned) + kMaxShards * sizeof(double) + 64;
    int rc = EPB_OK;
    if (!rc) rc = dev_alloc(h, &h->p_t1, strip);
    if (!rc) rc = dev_alloc(h, &h->p_g, kColOutputs * strip);
    if (!rc && h->P > 1) rc = dev_alloc(h, &h->p_gsend, kColOutputs * strip);
    if (!rc) rc = dev_alloc(h, &h->p_fxy, (size_t)(h->RB + halo_rows) * h->N);
    if (!rc) rc = dev_alloc(h, &h->p_sig, sig_bytes);
    if (!rc) rc = dev_alloc(h, &h->energy_total, 1);
    if (!rc) rc = dev_alloc(h, &h->epoch_dev, 1);
    if (rc) return rc;
    EPB_CUDA(h, cudaMemset(h->p_sig, 0, sig_bytes));
    EPB_CUDA(h, cudaMemset(h->epoch_dev, 0, sizeof(unsigned)));
    EPB_CUDA(h, cudaMemset(h->p_fxy, 0, (size_t)(h->RB + halo_rows) * h->N * sizeof(float2)));
    cudaIpcMemHandle_t* out = static_cast<cudaIpcMemHandle_t*>(handles_out);
    EPB_CUDA(h, cudaIpcGetMemHandle(&out[0], h->p_t1));
    EPB_CUDA(h, cudaIpcGetMemHandle(&out[1], h->p_g));
    EPB_CUDA(h, cudaIpcGetMemHandle(&out[2], h->p_fxy));
    EPB_CUDA(h, cudaIpcGetMemHandle(&out[3], h->p_sig));
    EPB_CUDA(h, cudaDeviceSynchronize());
    return EPB_OK;
}

int epb_shard_connect(epb_handle* h, const void* all_handles) {
    if (!h || !all_handles) return EPB_EINVAL;
    if (!h->p_t1) return fail(h, EPB_ENOSTATE, "epb_shard_peer_buffers first");
    DeviceGuard guard(h->dev);
    const cudaIpcMemHandle_t* hs = static_cast<const cudaIpcMemHandle_t*>(all_handles);
    for (int q = 0; q < h->P; ++q) {
        if (q == h->p) {
            h->peer_t1[q] = h->p_t1; h->peer_g[q] = h->p_g; h->peer_fxy[q] = h->p_fxy; h->peer_sig[q] = h->p_sig;
            continue;
        }
        void* ptr = nullptr;
        EPB_CUDA(h, cudaIpcOpenMemHandle(&ptr, hs[4 * q + 0], cudaIpcMemLazyEnablePeerAccess));
        h->peer_t1[q] = static_cast<float*>(ptr);
        EPB_CUDA(h, cudaIpcOpenMemHandle(&ptr, hs[4 * q + 1], cudaIpcMemLazyEnablePeerAccess));
        h->peer_g[q] = static_cast<float*>(ptr);
        EPB_CUDA(h, cudaIpcOpenMemHandle(&ptr, hs[4 * q + 2], cudaIpcMemLazyEnablePeerAccess));
        h->peer_fxy[q] = static_cast<float2*>(ptr);
        EPB_CUDA(h, cudaIpcOpenMemHandle(&ptr, hs[4 * q + 3], cudaIpcMemLazyEnablePeerAccess));
        h->peer_sig[q] = static_cast<unsigned char*>(ptr);
    }
    h->connected = true;
    return EPB_OK;
}

int epb_shard_set_timeout(epb_handle* h, int64_t max_polls) {
    if (!h || max_polls < 1) return EPB_EINVAL;
    h->max_polls = max_polls;
    return EPB_OK;
}

namespace {

PeerSignals peer_signals(epb_handle* h) {
    PeerSignals ps;
    for (int q = 0; q < kMaxShards; ++q) {
        ps.sig[q] = q < h->P ? reinterpret_cast<unsigned*>(h->peer_sig[q]) : nullptr;
        ps.energy[q] = q < h->P ? reinterpret_cast<double*>(h->peer_sig[q] + 3 * kMaxShards * sizeof(unsigned))
                                : nullptr;
    }
    return ps;
}

int signal_and_wait(epb_handle* h, int stage, cudaStream_t st, const double* energy = nullptr,
                    float* energy_out = nullptr) {
    k_signal<<<1, 32, 0, st>>>(peer_signals(h), h->P, h->p, stage, h->epoch_dev, stage == 0 ? 1 : 0, energy);
    EPB_LAUNCHED(h, "k_signal launch");
    const double* my_energy = reinterpret_cast<const double*>(h->p_sig + 3 * kMaxShards * sizeof(unsigned));
    k_wait<<<1, 32, 0, st>>>(reinterpret_cast<const unsigned*>(h->p_sig), h->P, stage, h->epoch_dev, 0u,
                             h->max_polls, my_energy, energy ? h->energy_total : nullptr, energy_out, 1.0, h->flags);
    EPB_LAUNCHED(h, "k_wait launch");
    return EPB_OK;
}

}  // namespace

int epb_shard_forward_peer(epb_handle* h, const epb_cells* cells, epb_stream stream, float* density_band,
                           float* potential_band, float* field_x_band, float* field_y_band, float* energy) {
    if (!h) return EPB_EINVAL;
    if (!h->connected) return fail(h, EPB_ENOSTATE, "epb_shard_connect first");
    CellView v;
    if (int rc = make_view(h, cells, v)) return rc;
    DeviceGuard guard(h->dev);
    cudaStream_t st = (cudaStream_t)stream;
    ProfCall pc(h, st);
    pc.begin();
    // row DCT blocks go straight into every shard's column strip
    DstTable t1;
    for (int q = 0; q < kMaxShards; ++q) t1.p[q] = q < h->P ? h->peer_t1[q] : nullptr;
    if (!h->cell_order) {
        if (int rc = tile_prepare(h, v, st)) return rc;
        pc.end_stage(EPB_STAGE_BIN);
        float* rho = density_band ? density_band : h->rho;
        if (int rc = tile_scatter(h, v, rho, st)) return rc;
        pc.end_stage(EPB_STAGE_SCATTER);
        if (int rc = launch_row_fwd(h, false, rho, nullptr, t1, h->row0, st)) return rc;
        pc.end_stage(EPB_STAGE_ROW_FWD);
    } else {
        if (h->grid_dirty) {
            EPB_CUDA(h, cudaMemsetAsync(h->grid, 0, (size_t)h->RB * h->N * sizeof(long long), st));
            h->grid_dirty = false;
        }
        h->grid_dirty = true;
        if (int rc = scatter_into(h, v, st, h->grid)) return rc;
        pc.end_stage(EPB_STAGE_SCATTER);
        if (int rc = launch_row_fwd(h, true, nullptr, density_band, t1, h->row0, st)) return rc;
        pc.end_stage(EPB_STAGE_ROW_FWD);
        h->grid_dirty = false;
    }
    if (int rc = signal_and_wait(h, 0, st)) return rc;
    pc.last = pc.mark();
    // column outputs: this band's block in place, the other bands' blocks staged
    // locally (each row of a strip is only 4 columns wide) and pushed as whole
    // contiguous blocks into the peers' row-band buffers
    const int64_t gblock = kColOutputs * (int64_t)h->RB * h->NB;
    DstTable g;
    for (int q = 0; q < kMaxShards; ++q)
        g.p[q] = q >= h->P ? nullptr : (q == h->p ? h->p_g + h->p * gblock : h->p_gsend + q * gblock);
    const bool want_phi = potential_band != nullptr;
    if (int rc = launch_columns(h, h->p_t1, g, nullptr, st)) return rc;
    if (h->P > 1) {
        PushArgs pa;
        pa.nblocks = 0;
        pa.n4 = gblock / 4;
        for (int q = 0; q < h->P; ++q) {
            if (q == h->p) continue;
            pa.src[pa.nblocks] = reinterpret_cast<const float4*>(h->p_gsend + q * gblock);
            pa.dst[pa.nblocks] = reinterpret_cast<float4*>(h->peer_g[q] + h->p * gblock);
            pa.nblocks++;
        }
        k_push<<<148 * 8, 256, 0, st>>>(pa);
        EPB_LAUNCHED(h, "k_push launch");
    }
    pc.end_stage(EPB_STAGE_COLUMN);
    if (int rc = signal_and_wait(h, 1, st, h->energy_d, energy)) return rc;
    pc.last = pc.mark();
    // row inverses; the first halo rows also go to the previous band's halo
    float2* halo_dst = h->p > 0 ? h->peer_fxy[h->p - 1] + (int64_t)h->RB * h->N : nullptr;
    if (int rc = launch_rows_inverse(h, h->p_g, potential_band, field_x_band, field_y_band, h->p_fxy, want_phi, st,
                                     halo_dst, h->p_halo_max))
        return rc;
    pc.end_stage(EPB_STAGE_ROW_INV);
    return signal_and_wait(h, 2, st);
}

int epb_shard_backward_peer(epb_handle* h, const epb_cells* cells, const float* grad_out, epb_stream stream,
                            float* grad_x, float* grad_y) {
    if (!h) return EPB_EINVAL;
    if (!h->connected) return fail(h, EPB_ENOSTATE, "epb_shard_connect first");
    CellView v;
    if (int rc = make_view(h, cells, v)) return rc;
    if (v.n > 0 && (!grad_x || !grad_y)) return fail(h, EPB_EINVAL, "grad_x/grad_y must be non-NULL");
    if (v.n == 0) return EPB_OK;
    DeviceGuard guard(h->dev);
    cudaStream_t st = (cudaStream_t)stream;
    ProfCall pc(h, st);
    pc.begin();
    if (int rc = shard_gather(h, v, h->p_fxy, h->p_halo, grad_out, grad_x, grad_y, st)) return rc;
    pc.end_stage(EPB_STAGE_GATHER);
    return EPB_OK;
}

int epb_shard_wait_test(epb_handle* h, epb_stream stream, int64_t max_polls) {
    if (!h || max_polls < 1) return EPB_EINVAL;
    if (!h->p_sig) return fail(h, EPB_ENOSTATE, "epb_shard_peer_buffers first");
    DeviceGuard guard(h->dev);
    // an epoch no shard has published: the wait must run out and flag a timeout
    k_wait<<<1, 32, 0, (cudaStream_t)stream>>>(reinterpret_cast<const unsigned*>(h->p_sig), h->P, 0, h->epoch_dev,
                                                0x40000000u, (long long)max_polls, nullptr, nullptr, nullptr, 1.0,
                                                h->flags);
    EPB_LAUNCHED(h, "k_wait launch");
    return EPB_OK;
}

int epb_profile_start(epb_handle* h, int32_t max_calls) {
    if (!h) return EPB_EINVAL;
    if (max_calls < 1 || max_calls > 200000) return fail(h, EPB_EINVAL, "max_calls must be in [1, 200000]");
    DeviceGuard guard(h->dev);
    for (cudaEvent_t e : h->prof_events) cudaEventDestroy(e);
    h->prof_events.clear();
    h->prof_spans.clear();
    h->prof_used = 0;
    const size_t n = (size_t)max_calls * 8;
    h->prof_events.resize(n);
    for (size_t i = 0; i < n; ++i) {
        cudaError_t e = cudaEventCreate(&h->prof_events[i]);
        if (e != cudaSuccess) {
            for (size_t j = 0; j < i; ++j) cudaEventDestroy(h->prof_events[j]);
            h->prof_events.clear();
            return cuda_fail(h, e, "cudaEventCreate");
        }
    }
    h->prof_calls_left = max_calls;
    h->prof_on = true;
    return EPB_OK;
}

int epb_atomic_probe(epb_handle* h, int64_t n_cells, int32_t fw, int32_t fh, epb_stream stream, double* ms) {
    if (!h) return EPB_EINVAL;
    if (!ms || n_cells < 0 || n_cells >= ((int64_t)1 << 31) || fw < 1 || fw > 8 || fh < 1 || fh > 8 || fw > h->M ||
        fh > h->N)
        return fail(h, EPB_EINVAL, "ms must be non-NULL, 0 <= n_cells < 2^31, footprints 1..8 and within the grid");
    if (h->P > 1) return fail(h, EPB_EINVAL, "the probe runs on a whole-grid handle");
    DeviceGuard guard(h->dev);
    if (!guard.ok) return fail(h, EPB_ECUDA, "cudaSetDevice failed");
    cudaStream_t st = (cudaStream_t)stream;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    cudaError_t e = cudaEventCreate(&e0);
    if (e == cudaSuccess) e = cudaEventCreate(&e1);
    if (e == cudaSuccess) e = cudaEventRecord(e0, st);
    if (e == cudaSuccess && n_cells > 0) {
        k_atomic_probe<<<(unsigned)((n_cells + 255) / 256), 256, 0, st>>>((unsigned long long*)h->grid, h->M, h->N,
                                                                          n_cells, fw, fh);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaEventRecord(e1, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(h->grid, 0, sizeof(long long) * (size_t)h->M * h->N, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    float t = 0.0f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&t, e0, e1);
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    if (e != cudaSuccess) return fail(h, EPB_ECUDA, std::string("atomic probe: ") + cudaGetErrorString(e));
    *ms = t;
    return EPB_OK;
}

int epb_profile_stop(epb_handle* h, double* stage_ms, int32_t* stage_launches) {
    if (!h) return EPB_EINVAL;
    DeviceGuard guard(h->dev);
    double ms[EPB_NUM_STAGES] = {0};
    int32_t cnt[EPB_NUM_STAGES] = {0};
    int rc = EPB_OK;
    if (h->prof_used > 0) {
        cudaError_t e = cudaEventSynchronize(h->prof_events[h->prof_used - 1]);
        if (e != cudaSuccess) rc = cuda_fail(h, e, "cudaEventSynchronize");
    }
    for (const auto& sp : h->prof_spans) {
        if (rc) break;
        float t = 0.f;
        cudaError_t e = cudaEventElapsedTime(&t, h->prof_events[sp.a], h->prof_events[sp.b]);
        if (e != cudaSuccess) { rc = cuda_fail(h, e, "cudaEventElapsedTime"); break; }
        ms[sp.stage] += t;
        cnt[sp.stage] += 1;
    }
    for (cudaEvent_t e : h->prof_events) cudaEventDestroy(e);
    h->prof_events.clear();
    h->prof_spans.clear();
    h->prof_used = 0;
    h->prof_on = false;
    h->prof_calls_left = 0;
    for (int i = 0; i < EPB_NUM_STAGES; ++i) {
        if (stage_ms) stage_ms[i] = ms[i];
        if (stage_launches) stage_launches[i] = cnt[i];
    }
    return rc;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free density map (epb_density_noalloc).  For callers that may not
// allocate device memory: their memory belongs to another allocator, or
// cudaMalloc's device-wide synchronisation is not acceptable on their path.
// The accumulation grid is this file-scope device array; its device address
// is looked up once per device with cudaGetSymbolAddress (host code must not
// use the symbol itself as a pointer).  The word right after a call's nbins
// map words holds the scatter's flag word; each call clears both.
// ---------------------------------------------------------------------------
static __device__ __align__(256) long long g_noalloc_grid[EPB_NOALLOC_MAX_BINS + 32];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {nullptr};

// fp32 density = fp32(q * dscale) (+ init), the same operations as k_row_fwd's load phase
__global__ void __launch_bounds__(256)
k_fixed_to_density(const long long* __restrict__ q, const float* __restrict__ init, double dscale,
                   int64_t nbins, float* __restrict__ out) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; b < nbins; b += stride) {
        float v = __double2float_rn(__dmul_rn(__ll2double_rn(q[b]), dscale));
        if (init) v = __fadd_rn(v, __ldg(init + b));
        out[b] = v;
    }
}

int noalloc_fail(char* err, int32_t len, int code, const std::string& msg) {
    if (err && len > 0) {
        std::strncpy(err, msg.c_str(), (size_t)len - 1);
        err[len - 1] = '\0';
    }
    return code;
}

}  // namespace

extern "C" int epb_density_noalloc(const epb_config* cfg, const epb_cells* cells, const float* init_norm,
                                   epb_stream stream, float* density, char* err, int32_t err_len) {
    if (!cfg || !cells || !density) return noalloc_fail(err, err_len, EPB_EINVAL, "cfg, cells and density must be non-NULL");
    if (cfg->num_bins_x < 1 || cfg->num_bins_y < 1)
        return noalloc_fail(err, err_len, EPB_EINVAL, "num_bins_x and num_bins_y must be positive");
    const int64_t nbins = (int64_t)cfg->num_bins_x * cfg->num_bins_y;
    if (nbins > EPB_NOALLOC_MAX_BINS)
        return noalloc_fail(err, err_len, EPB_EINVAL,
                            "grid of " + std::to_string(cfg->num_bins_x) + "x" + std::to_string(cfg->num_bins_y) +
                                " bins exceeds the allocation-free limit of " + std::to_string(EPB_NOALLOC_MAX_BINS) +
                                " bins; use epb_create/epb_forward");
    if (!std::isfinite(cfg->xl) || !std::isfinite(cfg->xh) || !std::isfinite(cfg->yl) || !std::isfinite(cfg->yh) ||
        !(cfg->xh > cfg->xl) || !(cfg->yh > cfg->yl) || cfg->fixed_point_bits > 60 || cfg->flags != 0)
        return noalloc_fail(err, err_len, EPB_EINVAL, "invalid die box (bounds must be finite, xh > xl, yh > yl), "
                                                      "fixed_point_bits or flags");
    if (cfg->device < 0 || cfg->device >= kMaxDevices) return noalloc_fail(err, err_len, EPB_EINVAL, "bad device");
    CellView v;
    if (int rc = make_view(nullptr, cells, v)) return noalloc_fail(err, err_len, rc, "invalid cell ranges or NULL arrays");

    DeviceGuard guard(cfg->device);
    if (!guard.ok) return noalloc_fail(err, err_len, EPB_ECUDA, "cudaSetDevice failed");
    void* base = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        if (!g_noalloc_ptr[cfg->device]) {
            cudaError_t e = cudaGetSymbolAddress(&g_noalloc_ptr[cfg->device], g_noalloc_grid);
            if (e != cudaSuccess) {
                g_noalloc_ptr[cfg->device] = nullptr;
                return noalloc_fail(err, err_len, EPB_ECUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
            }
        }
        base = g_noalloc_ptr[cfg->device];
    }
    long long* grid = static_cast<long long*>(base);
    unsigned* flags = reinterpret_cast<unsigned*>(grid + nbins);  // cleared with the map below

    // geometry exactly as epb_create resolves it
    epb_handle g;
    g.M = cfg->num_bins_x; g.N = cfg->num_bins_y;
    g.xl = cfg->xl; g.yl = cfg->yl; g.xh = cfg->xh; g.yh = cfg->yh;
    g.bsx = ((float)cfg->xh - (float)cfg->xl) / (float)g.M;
    g.bsy = ((float)cfg->yh - (float)cfg->yl) / (float)g.N;
    if (cfg->fixed_point_bits > 0) {
        g.S = cfg->fixed_point_bits;
    } else {
        const double area = (cfg->xh - cfg->xl) * (cfg->yh - cfg->yl);
        int ib = (int)std::ceil(std::log2(area > 1.0 ? area : 1.0)) + 1;
        if (ib < 32) ib = 32;
        g.S = 63 - ib;
    }
    const double dscale = std::ldexp(1.0, -g.S) / ((double)g.bsx * (double)g.bsy);
    cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e = cudaMemsetAsync(grid, 0, (size_t)(nbins + 32) * sizeof(long long), st);
    if (e != cudaSuccess) return noalloc_fail(err, err_len, EPB_ECUDA, std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
    if (v.n > 0) {
        k_scatter<false><<<cell_blocks(v.n), 256, 0, st>>>(v, geom(&g), ldexpf(1.0f, g.S), (unsigned long long*)grid, 0, g.M,
                                                    flags);
        e = cudaGetLastError();
        if (e != cudaSuccess) return noalloc_fail(err, err_len, EPB_ECUDA, std::string("k_scatter: ") + cudaGetErrorString(e));
    }
    int64_t blocks = (nbins + 255) / 256;
    if (blocks > 4096) blocks = 4096;
    k_fixed_to_density<<<(unsigned)blocks, 256, 0, st>>>(grid, init_norm, dscale, nbins, density);
    e = cudaGetLastError();
    if (e != cudaSuccess) return noalloc_fail(err, err_len, EPB_ECUDA, std::string("k_fixed_to_density: ") + cudaGetErrorString(e));
    return EPB_OK;
}

// ---------------------------------------------------------------------------
// Wirelength (allocation-free; csrc/wirelength.cuh)
// ---------------------------------------------------------------------------
extern "C" size_t epb_wirelength_scratch_bytes(int32_t num_pins) {
    return kWlPinGradOffset + 2 * sizeof(float2) * (size_t)std::max<int32_t>(num_pins, 0);
}

extern "C" int epb_wirelength(const epb_netlist* nl, const float* x, const float* y, float gamma, epb_stream stream,
                              void* scratch, size_t scratch_bytes, double* out, float* grad_x, float* grad_y,
                              uint32_t* flags, char* err, int32_t err_len) {
    if (!nl || !out || !scratch) return noalloc_fail(err, err_len, EPB_EINVAL, "nl, out and scratch must be non-NULL");
    if (nl->num_nets < 0 || nl->num_pins < 0 || nl->num_nodes < 0)
        return noalloc_fail(err, err_len, EPB_EINVAL, "netlist counts must be >= 0");
    if (!nl->net_start || (nl->num_pins > 0 && (!nl->net_pins || !nl->pin_node || !nl->pin_offset_x ||
                                                 !nl->pin_offset_y)))
        return noalloc_fail(err, err_len, EPB_EINVAL, "net_start, net_pins, pin_node and pin offsets must be non-NULL");
    const bool want_grad = grad_x || grad_y;
    if (want_grad && (!nl->node_pin_start || (nl->num_pins > 0 && !nl->node_pins)))
        return noalloc_fail(err, err_len, EPB_EINVAL, "a gradient needs node_pin_start and node_pins");
    if (nl->num_nodes > 0 && nl->num_pins > 0 && (!x || !y))
        return noalloc_fail(err, err_len, EPB_EINVAL, "x and y must be non-NULL");
    if (!std::isfinite(gamma) || !(gamma > 0.0f)) return noalloc_fail(err, err_len, EPB_EINVAL, "gamma must be finite and > 0");
    if (scratch_bytes < epb_wirelength_scratch_bytes(nl->num_pins) || (reinterpret_cast<uintptr_t>(scratch) & 15))
        return noalloc_fail(err, err_len, EPB_EINVAL, "scratch must be 16-byte aligned and epb_wirelength_scratch_bytes long");
    DeviceGuard guard(nl->device);
    if (!guard.ok) return noalloc_fail(err, err_len, EPB_ECUDA, "cudaSetDevice failed");
    cudaStream_t st = (cudaStream_t)stream;
    NetlistView v;
    v.net_start = nl->net_start; v.net_pins = nl->net_pins; v.pin_node = nl->pin_node;
    v.pin_ox = nl->pin_offset_x; v.pin_oy = nl->pin_offset_y; v.net_weight = nl->net_weight;
    v.node_pin_start = nl->node_pin_start; v.node_pins = nl->node_pins;
    v.E = nl->num_nets; v.P = nl->num_pins; v.V = nl->num_nodes; v.ignore_degree = nl->ignore_net_degree;
    char* base = static_cast<char*>(scratch);
    unsigned* counter = reinterpret_cast<unsigned*>(base);
    double* partials = reinterpret_cast<double*>(base + kWlPartialsOffset);
    float2* pin_grad = reinterpret_cast<float2*>(base + kWlPinGradOffset);
    float2* slot_pos = pin_grad + v.P;
    cudaError_t e = cudaMemsetAsync(counter, 0, sizeof(unsigned), st);
    if (e != cudaSuccess) return noalloc_fail(err, err_len, EPB_ECUDA, std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
    // pin positions by net-list slot, a thread each
    if (v.P > 0) {
        const int64_t per_block = (int64_t)kWlThreads * kWlPinsPerThread;
        const int pb = (int)(((int64_t)v.P + per_block - 1) / per_block);
        k_wa_pins<<<pb, kWlThreads, 0, st>>>(v, x, y, slot_pos, flags);
        e = cudaGetLastError();
        if (e != cudaSuccess) return noalloc_fail(err, err_len, EPB_ECUDA, std::string("k_wa_pins: ") + cudaGetErrorString(e));
    }
    // windows of 32 nets, a warp each, over a fixed grid (one wave of resident
    // blocks on a B200; the same partition of the windows, so the same bits, on
    // every device); the last block adds up the block partials
    const int64_t windows = ((int64_t)v.E + 31) / 32;
    const int nb = (int)std::min<int64_t>(std::max<int64_t>((windows + kWlWarps - 1) / kWlWarps, 1), kWlWindowBlocks);
    const float inv_gamma = 1.0f / gamma;
    const float ig2 = (float)(1.4426950408889634 / (double)gamma);   // log2(e) / gamma
    k_wa_windows<<<nb, kWlThreads, 0, st>>>(v, inv_gamma, ig2, pin_grad, slot_pos, partials, counter, out, flags);
    e = cudaGetLastError();
    if (e != cudaSuccess) return noalloc_fail(err, err_len, EPB_ECUDA, std::string("k_wa_windows: ") + cudaGetErrorString(e));
    if (want_grad && v.V > 0) {
        const int gb = (int)(((int64_t)v.V + kWlThreads - 1) / kWlThreads);
        k_wa_nodes<<<gb, kWlThreads, 0, st>>>(v, pin_grad, grad_x, grad_y, flags);
        e = cudaGetLastError();
        if (e != cudaSuccess) return noalloc_fail(err, err_len, EPB_ECUDA, std::string("k_wa_nodes: ") + cudaGetErrorString(e));
    }
    return EPB_OK;
}
