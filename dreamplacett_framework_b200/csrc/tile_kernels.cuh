// tile_kernels.cuh -- the cell-tile density scatter and field gather.
//
// The grid (or a shard's row band) is cut into tiles of TX x TY bins (32 x 32
// on grids of 32 bins or more per axis).  Each cell is listed in every tile
// that its footprint, widened by `margin` bins on each side, meets.  A tile's
// CTA owns all of its bins: it sums the contributions of its listings exactly
// in shared memory and writes the finished fp32 density (fixed-point total ->
// fp32, plus the initial density) with plain stores -- no global atomics and
// no int64 grid round trip.
//
// The lists persist across calls.  Every forward validates them: k_validate
// re-reads each listed cell's position, computes its footprint and checks
// that it still lies inside the widened footprint the cell was listed with
// (then every tile it reaches lists it).  A cell that moved further takes the
// escape path for this call (global atomics into an int64 escape grid that the
// tiles fold in) and makes the next forward rebuild the lists.  The rebuild
// kernels are launched by every forward and return at once unless the device
// flag asks for a rebuild, so a captured step replays correctly whatever the
// cells do.
//
//   k_tile_decide   one thread: this forward rebuilds when the host forces it
//                   (new cell arrays, new buffers) or the last forward saw an
//                   escape; per-call counters are reset
//   k_rebuild_count cells -> listings and owner listings per tile (padded
//                   counters: no two tiles share a 32-byte sector); cells that
//                   cannot be listed (non-finite, empty, off the grid, or whose
//                   widened footprint meets more than kMaxTilesPerCell tiles)
//                   go to the static escape list
//   k_rebuild_scan  one CTA: tile starts, owner counts, work items (tile, chunk
//                   of at most kChunk listings), fill cursors
//   k_rebuild_fill  cells -> listing records (offsets, sizes, ratio, node,
//                   widened footprint), the owner listings first in each tile
//   k_validate      listings -> current footprint, or the cell escapes
//   k_esc_scatter   escape cells -> int64 escape grid
//   k_tile_scatter  work items -> density.  A tile with more than kChunk
//                   listings (a hot tile) is split over several items whose
//                   integer partial sums the last item to finish adds up in
//                   chunk order: the GPU form of the reference's hot-tile shard
//                   table (host/v11_tile_ownership.h:98-163,
//                   kernels/v11_accum_dm.cpp:315-369), with the count of each
//                   rebuild as its histogram.  Optionally (OVF) the cells of two
//                   node ranges are also summed apart for their overflow.
//   k_tile_gather   work items -> gradients of the owner listings (the tile
//                   that held the cell's first bin when it was listed), from
//                   the tile's field region staged in shared memory; a
//                   footprint beyond the region reads the field map in global
//                   memory
//   k_esc_gather    escape cells -> gradients (global field reads)
//
// Exactness: a contribution is q = round(fp32(a) * 2^S), summed as an integer
// with the operations of k_scatter; shared memory holds each bin's sum in three
// 32-bit limbs of 21, 21 and 22 bits (q mod 2^64 = l0 + l1 2^21 + l2 2^42).  A
// work item holds at most kChunk = 1024 listings and a cell adds at most once
// to a bin, so every limb sum stays below 1024 * 2^22 = 2^32: the limb sums are
// exact and a bin's total mod 2^64 equals the int64 sum of the atomic scatter.
// The density is bit-identical to k_scatter + k_row_fwd's conversion whatever
// the order of the listings, and so is the gather's gradient (the same fp32
// operations per cell).
#pragma once
#include <cstdint>
#include "epb_kernels.cuh"

namespace epb {

constexpr int kTileMax = 32;          // tile side (bins) on grids of >= 32 bins per axis
constexpr int kTileBinsMax = kTileMax * kTileMax;
constexpr int kChunk = 1024;          // listings per work item (limb exactness bound)
constexpr int kMaxTilesPerCell = 4;   // cells whose widened footprint meets more take the escape path
constexpr int kTileThreads = 256;
constexpr int kCounterStride = 8;     // ints per tile counter (32 bytes)
constexpr int kGatherLo = 2;          // gather region: rows / columns staged before the tile
constexpr int kGatherHi = 4;          //                and after it
constexpr int kRegionMax = (kTileMax + kGatherLo + kGatherHi) * (kTileMax + kGatherLo + kGatherHi);
constexpr unsigned kOwnerBit = 0x80000000u;    // this listing computes the cell's gradient
constexpr unsigned kPrimaryBit = 0x40000000u;  // this listing enqueues the cell when it escapes
constexpr unsigned kNodeMask = 0x3fffffffu;

// Device counters of the tile lists.
enum TileMeta : int {
    kMetaItems = 0,      // work items of the current lists
    kMetaWorkScatter,    // next item for k_tile_scatter
    kMetaWorkGather,     // next item for k_tile_gather
    kMetaEscDyn,         // cells that escaped in this call
    kMetaEscStatic,      // cells the lists do not hold
    kMetaListings,       // listings of the current lists
    kMetaUnused,
    kMetaEscaped,        // set by k_validate: an escape happened; rebuild at the next forward
    kMetaRebuild,        // this forward rebuilds (k_tile_decide)
    kMetaValid,          // the lists have been built at least once
    kMetaRebuilds,       // rebuilds so far (diagnostic)
    kMetaWords = 16
};

struct TileGeom {
    int ltx, lty;        // log2 tile rows / columns
    int ntx, nty;        // tiles along x (rows) and y (columns) of the band
    int row0;            // first grid row of the band (0 on a whole grid)
    int rows;            // rows of the band
    int margin;          // bins the footprints are widened by for listing
};

struct TileBins {
    int* cnt;            // [ntiles * kCounterStride] listings (0) and owner listings (1) per tile
    int* cur;            // [ntiles * kCounterStride] fill cursors: owners (0), others (1)
    int* start;          // [ntiles + 1] first listing of each tile
    int* nown;           // [ntiles] owner listings of each tile (the first ones of its range)
    int* first_item;     // [ntiles] first work item of each tile
    int2* items;         // [max_items] (tile, chunk)
    unsigned* arrive;    // [ntiles] finished items of multi-item tiles (zeroed by the scan)
    long long* part;     // [max_items][2][kTileBinsMax] partial sums of multi-item tiles
    int* meta;           // [kMetaWords]
    // listing records, [capacity] each
    float4* stat;        // offset_x, offset_y, size_x, size_y (written by the rebuild)
    int4* key;           // node | owner / primary bits, widened box lo (kx | ky << 16), hi, ratio bits
    float4* geo;         // x + offset_x, y + offset_y, ex, ey (k_validate; x is NaN: the cell escaped)
    short4* bins;        // kx0, kx1, ky0, ky1 of the footprint (k_validate)
    int* esc_dyn;        // [cells] cells that escaped in this call (node | owner bit)
    int* esc_static;     // [cells] cells the lists do not hold
    unsigned long long* esc_grid;  // [band rows * N] int64 escape sums, zero outside a call
};

__device__ __forceinline__ int pack_box(int kx, int ky) { return (kx & 0xFFFF) | (ky << 16); }
__device__ __forceinline__ int box_x(int v) { return v & 0xFFFF; }
__device__ __forceinline__ int box_y(int v) { return (int)((unsigned)v >> 16); }

// ---------------------------------------------------------------------------
// Rebuild
// ---------------------------------------------------------------------------
__global__ void k_tile_decide(TileBins b, int force) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    int* m = b.meta;
    const int rebuild = (force | m[kMetaEscaped] | (m[kMetaValid] == 0)) ? 1 : 0;
    m[kMetaRebuild] = rebuild;
    m[kMetaEscaped] = 0;
    m[kMetaEscDyn] = 0;
    m[kMetaWorkScatter] = 0;
    m[kMetaWorkGather] = 0;
    if (rebuild) {
        m[kMetaEscStatic] = 0;
        m[kMetaRebuilds] += 1;
    }
}

// Listing of a cell on the band: the tiles (band tile coordinates txa..txb,
// tya..tyb) its widened footprint meets and the widened box (blo, bhi).  False
// when the band does not list it; *esc then tells whether it goes to this
// band's static escape list instead.
__device__ __forceinline__ bool listing_of(const CellView& c, const GridGeom& g, const TileGeom& t,
                                          const CellData& d, Footprint& f, int& st, int& txa, int& txb, int& tya,
                                          int& tyb, int& blo, int& bhi, bool& esc) {
    esc = false;
    st = footprint_of(c, g, d, f);
    if (st != 1) {
        // it contributes nothing now: the band holding row 0 keeps it (it reports
        // non-finite data and, on a whole grid, writes the cell's zero gradient)
        esc = t.row0 == 0;
        return false;
    }
    const int m = t.margin;
    const int xlo = max(f.kx0 - m, 0), xhi = min(f.kx1 + m, g.M - 1);
    const int ylo = max(f.ky0 - m, 0), yhi = min(f.ky1 + m, g.N - 1);
    const int r0 = t.row0, r1 = t.row0 + t.rows - 1;
    if (xhi < r0 || xlo > r1) return false;   // another band's cell
    txa = (max(xlo, r0) - r0) >> t.ltx; txb = (min(xhi, r1) - r0) >> t.ltx;
    tya = ylo >> t.lty; tyb = yhi >> t.lty;
    blo = pack_box(xlo, ylo);
    bhi = pack_box(xhi, yhi);
    if ((txb - txa + 1) * (tyb - tya + 1) > kMaxTilesPerCell) {
        esc = true;
        return false;
    }
    return true;
}

// On a band (a shard's rows), whether a cell can matter to it from its x data
// alone: its rows, widened by the margin, meet the band, or its x data does
// not give a footprint (the band holding row 0 then keeps it).  The y data is
// read only for those; on a whole grid every cell passes.
__device__ __forceinline__ bool band_may_list(const CellView& c, const GridGeom& g, const TileGeom& t, int64_t node) {
    if (t.rows == g.M) return true;
    float x = __ldg(c.x + node);
    if (c.ox) x = __fadd_rn(x, __ldg(c.ox + node));
    const float sx = __ldg(c.sx + node);
    if (!isfinite(x) || !isfinite(sx) || !(sx > 0.0f)) return t.row0 == 0;
    const int kx0 = bin_floor(x, g.xl, g.bsx, g.ibsx, g.M);
    const int kx1 = min(bin_floor(__fadd_rn(x, sx), g.xl, g.bsx, g.ibsx, g.M), g.M - 1);
    if (kx0 > kx1) return t.row0 == 0;
    return !(kx1 + t.margin < t.row0 || kx0 - t.margin >= t.row0 + t.rows);
}

__global__ void __launch_bounds__(256)
k_rebuild_count(CellView c, GridGeom g, TileGeom t, TileBins b, unsigned* __restrict__ flags) {
    if (b.meta[kMetaRebuild] == 0) return;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    unsigned bad = 0;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < c.n; i += stride) {
        const int64_t node = cell_node(c, i);
        if (!band_may_list(c, g, t, node)) continue;
        Footprint f;
        int st, txa, txb, tya, tyb, blo, bhi;
        bool esc;
        if (!listing_of(c, g, t, load_cell(c, node), f, st, txa, txb, tya, tyb, blo, bhi, esc)) {
            if (st < 0) bad = 1;
            if (esc) b.esc_static[atomicAdd(b.meta + kMetaEscStatic, 1)] = (int)node;
            continue;
        }
        const int ox = f.kx0 - t.row0;   // the owner tile holds the first bin
        for (int tx = txa; tx <= txb; ++tx)
            for (int ty = tya; ty <= tyb; ++ty) {
                const int tile = tx * t.nty + ty;
                atomicAdd(b.cnt + tile * kCounterStride, 1);
                if (ox >= 0 && (ox >> t.ltx) == tx && (f.ky0 >> t.lty) == ty)
                    atomicAdd(b.cnt + tile * kCounterStride + 1, 1);
            }
    }
    if (bad) atomicOr(flags, kFlagNonFinite);
}

constexpr int kScanThreads = 1024;

// Exclusive scan of (a, b) pairs over the CTA; total receives the sums.
__device__ __forceinline__ int2 block_exclusive_scan2(int2 v, int2* s_warp, int2& total) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int2 inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int ax = __shfl_up_sync(0xffffffffu, inc.x, o), ay = __shfl_up_sync(0xffffffffu, inc.y, o);
        if (lane >= o) { inc.x += ax; inc.y += ay; }
    }
    if (lane == 31) s_warp[w] = inc;
    __syncthreads();
    if (w == 0) {
        int2 s = lane < nw ? s_warp[lane] : make_int2(0, 0);
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int ax = __shfl_up_sync(0xffffffffu, s.x, o), ay = __shfl_up_sync(0xffffffffu, s.y, o);
            if (lane >= o) { s.x += ax; s.y += ay; }
        }
        if (lane < nw) s_warp[lane] = s;
    }
    __syncthreads();
    const int2 before = w > 0 ? s_warp[w - 1] : make_int2(0, 0);
    total = s_warp[nw - 1];
    __syncthreads();
    return make_int2(before.x + inc.x - v.x, before.y + inc.y - v.y);
}

// One CTA; each thread takes ntiles / kScanThreads consecutive tiles (at least
// one), sums them, then one CTA-wide scan of the sums.
__global__ void __launch_bounds__(kScanThreads)
k_rebuild_scan(int ntiles, TileBins b) {
    if (b.meta[kMetaRebuild] == 0) return;
    __shared__ int2 s_warp[kScanThreads / 32];
    const int per = (ntiles + kScanThreads - 1) / kScanThreads;
    const int t0 = threadIdx.x * per;
    int2 loc = make_int2(0, 0);
    for (int k = 0; k < per && t0 + k < ntiles; ++k) {
        const int cnt = b.cnt[(t0 + k) * kCounterStride];
        loc.x += cnt;
        loc.y += max(1, (cnt + kChunk - 1) / kChunk);
    }
    int2 tot;
    int2 ex = block_exclusive_scan2(loc, s_warp, tot);
    for (int k = 0; k < per && t0 + k < ntiles; ++k) {
        const int tile = t0 + k;
        const int cnt = b.cnt[tile * kCounterStride], own = b.cnt[tile * kCounterStride + 1];
        const int nit = max(1, (cnt + kChunk - 1) / kChunk);
        b.start[tile] = ex.x;
        b.nown[tile] = own;
        b.first_item[tile] = ex.y;
        b.cur[tile * kCounterStride] = ex.x;
        b.cur[tile * kCounterStride + 1] = ex.x + own;
        for (int it = 0; it < nit; ++it) b.items[ex.y + it] = make_int2(tile, it);
        b.cnt[tile * kCounterStride] = 0;
        b.cnt[tile * kCounterStride + 1] = 0;
        b.arrive[tile] = 0u;
        ex.x += cnt;
        ex.y += nit;
    }
    if (threadIdx.x == 0) {
        b.start[ntiles] = tot.x;
        b.meta[kMetaItems] = tot.y;
        b.meta[kMetaListings] = tot.x;
        b.meta[kMetaValid] = 1;
    }
}

__global__ void __launch_bounds__(256)
k_rebuild_fill(CellView c, GridGeom g, TileGeom t, TileBins b) {
    if (b.meta[kMetaRebuild] == 0) return;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < c.n; i += stride) {
        const int64_t node = cell_node(c, i);
        if (!band_may_list(c, g, t, node)) continue;
        const CellData d = load_cell(c, node);
        Footprint f;
        int st, txa, txb, tya, tyb, blo, bhi;
        bool esc;
        if (!listing_of(c, g, t, d, f, st, txa, txb, tya, tyb, blo, bhi, esc)) continue;
        const float4 sv = make_float4(d.ox, d.oy, d.sx, d.sy);
        const int ox = f.kx0 - t.row0;
        for (int tx = txa; tx <= txb; ++tx)
            for (int ty = tya; ty <= tyb; ++ty) {
                const int tile = tx * t.nty + ty;
                const bool owner = ox >= 0 && (ox >> t.ltx) == tx && (f.ky0 >> t.lty) == ty;
                const bool primary = tx == txa && ty == tya;
                const int slot = atomicAdd(b.cur + tile * kCounterStride + (owner ? 0 : 1), 1);
                const unsigned tag = (unsigned)node | (owner ? kOwnerBit : 0u) | (primary ? kPrimaryBit : 0u);
                b.stat[slot] = sv;
                b.key[slot] = make_int4((int)tag, blo, bhi, __float_as_int(d.r));
            }
    }
}

// ---------------------------------------------------------------------------
// Per call: validate, escape scatter
// ---------------------------------------------------------------------------
// Each listing: the cell's footprint from its position now.  Inside the listed
// box: geo and bins.  Outside (or no longer contributing): the cell escapes
// for this call; its primary listing enqueues it once (with the owner bit when
// this band holds its owner listing) and every listing of it is marked.
__global__ void __launch_bounds__(256)
k_validate(CellView c, GridGeom g, TileBins b) {
    const int n = b.meta[kMetaListings];
    const int stride = gridDim.x * blockDim.x;
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < n; j += stride) {
        const int4 k = b.key[j];
        const float4 sv = b.stat[j];
        const unsigned tag = (unsigned)k.x;
        const int64_t node = (int64_t)(tag & kNodeMask);
        CellData d;
        d.x = __ldg(c.x + node);
        d.y = __ldg(c.y + node);
        d.ox = sv.x; d.oy = sv.y; d.sx = sv.z; d.sy = sv.w;
        d.r = __int_as_float(k.w);
        Footprint f;
        const int st = footprint_of(c, g, d, f);
        if (st == 1 && f.kx0 >= box_x(k.y) && f.kx1 <= box_x(k.z) && f.ky0 >= box_y(k.y) && f.ky1 <= box_y(k.z)) {
            b.geo[j] = make_float4(f.x, f.y, f.ex, f.ey);
            b.bins[j] = make_short4((short)f.kx0, (short)f.kx1, (short)f.ky0, (short)f.ky1);
            continue;
        }
        b.geo[j] = make_float4(__int_as_float(0x7fc00000), 0.0f, 0.0f, 0.0f);
        if (tag & kPrimaryBit)
            b.esc_dyn[atomicAdd(b.meta + kMetaEscDyn, 1)] = (int)((unsigned)node | (tag & kOwnerBit));
        b.meta[kMetaEscaped] = 1;
    }
}

// Escape cells (the static list, then this call's) into the int64 escape grid
// of the band, footprints clipped to its rows.  With grid0, the nodes of the
// two ranges set0 go to grid0 instead (the overflow cells of k_tile_scatter<true>).
__global__ void __launch_bounds__(256)
k_esc_scatter(CellView c, GridGeom g, TileGeom t, float qscale, TileBins b, unsigned long long* __restrict__ grid0,
              int64_t s00, int64_t s01, int64_t s02, int64_t s03) {
    const int ns = b.meta[kMetaEscStatic], nd = b.meta[kMetaEscDyn];
    const int stride = gridDim.x * blockDim.x;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < ns + nd; i += stride) {
        const int64_t node = i < ns ? (int64_t)b.esc_static[i] : (int64_t)((unsigned)b.esc_dyn[i - ns] & kNodeMask);
        Footprint f;
        if (footprint_of(c, g, load_cell(c, node), f) != 1) continue;
        const bool to0 = grid0 && ((node >= s00 && node < s01) || (node >= s02 && node < s03));
        unsigned long long* base = to0 ? grid0 : b.esc_grid;
        const int kxa = max(f.kx0, t.row0), kxb = min(f.kx1, t.row0 + t.rows - 1);
        for (int kx = kxa; kx <= kxb; ++kx) {
            const float oxr = __fmul_rn(bin_overlap(f.x, f.ex, g.xl, g.bsx, kx), f.r);
            if (oxr == 0.0f) continue;
            unsigned long long* row = base + (int64_t)(kx - t.row0) * g.N;
            for (int ky = f.ky0; ky <= f.ky1; ++ky) {
                const float a = __fmul_rn(oxr, bin_overlap(f.y, f.ey, g.yl, g.bsy, ky));
                const long long q = __float2ll_rn(__fmul_rn(a, qscale));
                if (q != 0) atomicAdd(row + ky, (unsigned long long)q);
            }
        }
    }
}

// Next work item of a CTA (hot tiles' items and the others balance over the
// SMs); -1 when none is left.
__device__ __forceinline__ int next_item(int* counter, int nitems) {
    __shared__ int s_item;
    if (threadIdx.x == 0) s_item = atomicAdd(counter, 1);
    __syncthreads();
    const int it = s_item;
    __syncthreads();
    return it < nitems ? it : -1;
}

// ---------------------------------------------------------------------------
// Tile scatter
// ---------------------------------------------------------------------------
struct TileScatterArgs {
    GridGeom g;
    TileGeom t;
    TileBins b;
    float qscale;            // 2^S
    double dscale;           // 2^-S / bin_area
    const float* init;       // nullable [band rows * N] normalised initial density
    float* rho;              // [band rows * N] density out (nullable with OVF: the overflow only)
    unsigned* flags;
    // OVF: the listings of nodes in [set0[0], set0[1]) or [set0[2], set0[3]) (the
    // overflow cells) are also summed apart, for the overflow metric of their map
    int64_t set0[4];
    float target;
    double bin_area;
    double* ovf_part;        // [2 * ntiles] per-tile excess sum and maximum
    unsigned* ovf_counter;   // tiles finished (wraps to 0)
    double* ovf_out;         // [2]: bin_area * sum max(rho0 - target, 0), max rho0
    unsigned long long* esc_grid0;   // escape sums of the overflow cells
};

// Sum of a double and max of a float over the CTA in a fixed order (warps,
// then warp totals in warp order); thread 0 receives both.
__device__ __forceinline__ void block_sum_max(double& s, float& m) {
    __shared__ double s_s[kTileThreads / 32];
    __shared__ float s_m[kTileThreads / 32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        s += __shfl_down_sync(0xffffffffu, s, o);
        m = fmaxf(m, __shfl_down_sync(0xffffffffu, m, o));
    }
    if ((threadIdx.x & 31) == 0) { s_s[threadIdx.x >> 5] = s; s_m[threadIdx.x >> 5] = m; }
    __syncthreads();
    if (threadIdx.x == 0) {
        s = 0.0; m = -INFINITY;
        for (int w = 0; w < kTileThreads / 32; ++w) { s += s_s[w]; m = fmaxf(m, s_m[w]); }
    }
    __syncthreads();
}

__device__ __forceinline__ unsigned long long limb_total(const unsigned* l0, const unsigned* l1, const unsigned* l2,
                                                         int e) {
    return (unsigned long long)l0[e] + ((unsigned long long)l1[e] << 21) + ((unsigned long long)l2[e] << 42);
}

// Limb sets: one, or with OVF two (0: the overflow cells, 1: the others).
// Limb sets: one, or with OVF two (0: the overflow cells, 1: the others).
template <bool OVF>
__global__ void __launch_bounds__(kTileThreads)
k_tile_scatter(const __grid_constant__ TileScatterArgs a) {
    constexpr int NS = OVF ? 2 : 1;
    __shared__ unsigned s_limb[NS][3][kTileBinsMax];
    __shared__ bool s_last, s_last_tile;
    const GridGeom& g = a.g;
    const TileBins& b = a.b;
    const int TX = 1 << a.t.ltx, TY = 1 << a.t.lty, TB = TX * TY;
    const int ntiles = a.t.ntx * a.t.nty;
    const int nitems = b.meta[kMetaItems];
    const bool any_esc = b.meta[kMetaEscStatic] + b.meta[kMetaEscDyn] > 0;
    unsigned sat = 0;
    for (int item = next_item(b.meta + kMetaWorkScatter, nitems); item >= 0;
         item = next_item(b.meta + kMetaWorkScatter, nitems)) {
        const int2 it = b.items[item];
        const int tile = it.x;
        const int tx0 = a.t.row0 + ((tile / a.t.nty) << a.t.ltx), ty0 = (tile % a.t.nty) << a.t.lty;
        const int s0 = b.start[tile], s1 = b.start[tile + 1];
        const int nit = max(1, (s1 - s0 + kChunk - 1) / kChunk);
        const int lo = s0 + it.y * kChunk, hi = min(s1, lo + kChunk);
        for (int e = threadIdx.x; e < TB; e += kTileThreads) {
#pragma unroll
            for (int k = 0; k < NS; ++k) { s_limb[k][0][e] = 0u; s_limb[k][1][e] = 0u; s_limb[k][2][e] = 0u; }
        }
        __syncthreads();
        for (int j = lo + threadIdx.x; j < hi; j += kTileThreads) {
            const float4 gv = b.geo[j];
            if (gv.x != gv.x) continue;   // escaped: the escape grid has it
            const short4 bn = b.bins[j];
            const int4 k = b.key[j];
            int set = 0;
            if constexpr (OVF) {
                const int64_t node = (int64_t)((unsigned)k.x & kNodeMask);
                set = ((node >= a.set0[0] && node < a.set0[1]) || (node >= a.set0[2] && node < a.set0[3])) ? 0 : 1;
            }
            const float r = __int_as_float(k.w);
            const int kxa = max((int)bn.x, tx0), kxb = min((int)bn.y, tx0 + TX - 1);
            const int kya = max((int)bn.z, ty0), kyb = min((int)bn.w, ty0 + TY - 1);
            unsigned* L0 = s_limb[set][0];
            unsigned* L1 = s_limb[set][1];
            unsigned* L2 = s_limb[set][2];
            // q = round(fp32((ox * ratio) * oy) * 2^S) into the limbs of bin e
            auto add = [&](int e, float oxr, float ov) {
                const long long q = __float2ll_rn(__fmul_rn(__fmul_rn(oxr, ov), a.qscale));
                if (q == 0) return;
                const unsigned lo32 = (unsigned)q, hi32 = (unsigned)((unsigned long long)q >> 32);
                atomicAdd(L0 + e, lo32 & 0x1FFFFFu);
                atomicAdd(L1 + e, __funnelshift_r(lo32, hi32, 21) & 0x1FFFFFu);
                if (hi32 >> 10) atomicAdd(L2 + e, hi32 >> 10);
            };
            if (kyb - kya < kOyCache) {
                // column overlaps of the clipped footprint, once per listing
                float oy[kOyCache];
#pragma unroll
                for (int jj = 0; jj < kOyCache; ++jj)
                    oy[jj] = kya + jj <= kyb ? bin_overlap(gv.y, gv.w, g.yl, g.bsy, kya + jj) : 0.0f;
                for (int kx = kxa; kx <= kxb; ++kx) {
                    const float oxr = __fmul_rn(bin_overlap(gv.x, gv.z, g.xl, g.bsx, kx), r);
                    if (oxr == 0.0f) continue;
                    const int rowb = (kx - tx0) * TY + (kya - ty0);
#pragma unroll
                    for (int jj = 0; jj < kOyCache; ++jj) {
                        if (kya + jj > kyb) break;
                        add(rowb + jj, oxr, oy[jj]);
                    }
                }
            } else {
                for (int kx = kxa; kx <= kxb; ++kx) {
                    const float oxr = __fmul_rn(bin_overlap(gv.x, gv.z, g.xl, g.bsx, kx), r);
                    if (oxr == 0.0f) continue;
                    const int rowb = (kx - tx0) * TY - ty0;
                    for (int ky = kya; ky <= kyb; ++ky) add(rowb + ky, oxr, bin_overlap(gv.y, gv.w, g.yl, g.bsy, ky));
                }
            }
        }
        __syncthreads();
        bool finish = nit == 1;
        if (!finish) {
            // a hot tile: publish this item's partial sums; the last item of the
            // tile to finish adds them up in chunk order
            long long* part = b.part + (int64_t)item * 2 * kTileBinsMax;
            for (int e = threadIdx.x; e < TB; e += kTileThreads)
#pragma unroll
                for (int k = 0; k < NS; ++k)
                    part[k * kTileBinsMax + e] = (long long)limb_total(s_limb[k][0], s_limb[k][1], s_limb[k][2], e);
            __threadfence();
            __syncthreads();
            if (threadIdx.x == 0) {
                s_last = atomicAdd(b.arrive + tile, 1u) == (unsigned)(nit - 1);
                // the last item resets the count for the next call (every other item of
                // the tile has counted by now)
                if (s_last) b.arrive[tile] = 0u;
            }
            __syncthreads();
            finish = s_last;
            if (finish) __threadfence();
        }
        if (finish) {
            const int item0 = b.first_item[tile];
            double ex_sum = 0.0;
            float mx = -INFINITY;
            constexpr int PER = kTileBinsMax / kTileThreads;
            // every bin's initial density loaded before any is used
            float ini[PER];
#pragma unroll
            for (int u = 0; u < PER; ++u) {
                const int e = threadIdx.x + u * kTileThreads;
                ini[u] = 0.0f;
                if (a.init && e < TB) ini[u] = __ldg(a.init + (int64_t)(tx0 - a.t.row0 + e / TY) * g.N + ty0 + e % TY);
            }
#pragma unroll
            for (int u = 0; u < PER; ++u) {
                const int e = threadIdx.x + u * kTileThreads;
                if (e >= TB) break;
                unsigned long long q[NS];
#pragma unroll
                for (int k = 0; k < NS; ++k) {
                    if (nit == 1) {
                        q[k] = limb_total(s_limb[k][0], s_limb[k][1], s_limb[k][2], e);
                    } else {
                        q[k] = 0ull;
                        for (int cc = 0; cc < nit; ++cc)
                            q[k] += (unsigned long long)__ldcg(b.part + ((int64_t)(item0 + cc) * 2 + k) * kTileBinsMax + e);
                    }
                }
                const int64_t gb = (int64_t)(tx0 - a.t.row0 + e / TY) * g.N + ty0 + e % TY;
                if (any_esc) {
                    q[NS - 1] += b.esc_grid[gb];
                    b.esc_grid[gb] = 0ull;
                    if constexpr (OVF) {
                        q[0] += a.esc_grid0[gb];
                        a.esc_grid0[gb] = 0ull;
                    }
                }
                if constexpr (OVF) {
                    // the overflow cells' map, with the operations of k_overflow
                    const long long q0 = (long long)q[0];
                    if (q0 < 0 || q0 >= (1ll << 62)) sat = 1;
                    float v0 = __double2float_rn(__dmul_rn(__ll2double_rn(q0), a.dscale));
                    if (a.init) v0 = __fadd_rn(v0, ini[u]);
                    const double ex = (double)v0 - (double)a.target;
                    if (ex > 0.0) ex_sum += ex;
                    mx = fmaxf(mx, v0);
                }
                if (a.rho) {
                    unsigned long long qt = q[0];
                    if constexpr (OVF) qt += q[1];
                    const long long qs = (long long)qt;
                    if (qs < 0 || qs >= (1ll << 62)) sat = 1;
                    float v = __double2float_rn(__dmul_rn(__ll2double_rn(qs), a.dscale));
                    if (a.init) v = __fadd_rn(v, ini[u]);
                    a.rho[gb] = v;
                }
            }
            if constexpr (OVF) {
                // per-tile partials, then the last tile to finish combines them in tile order
                block_sum_max(ex_sum, mx);
                if (threadIdx.x == 0) {
                    a.ovf_part[2 * tile] = ex_sum;
                    a.ovf_part[2 * tile + 1] = (double)mx;
                    __threadfence();
                    s_last_tile = atomicInc(a.ovf_counter, (unsigned)(ntiles - 1)) == (unsigned)(ntiles - 1);
                }
                __syncthreads();
                if (s_last_tile) {
                    __threadfence();
                    double s = 0.0;
                    float m = -INFINITY;
                    for (int tt = threadIdx.x; tt < ntiles; tt += kTileThreads) {
                        s += __ldcg(a.ovf_part + 2 * tt);
                        m = fmaxf(m, (float)__ldcg(a.ovf_part + 2 * tt + 1));
                    }
                    block_sum_max(s, m);
                    if (threadIdx.x == 0) {
                        a.ovf_out[0] = s * a.bin_area;
                        a.ovf_out[1] = (double)m;
                    }
                }
            }
        }
        __syncthreads();
    }
    if (sat) atomicOr(a.flags, kFlagSaturated);
}

// ---------------------------------------------------------------------------
// Gather
// ---------------------------------------------------------------------------
// Per-cell accumulation (the arithmetic of k_gather: w = ox * oy, fmaf into ax,
// ay, rows then columns) over rows kx0..kxb.  fv(kx, ky) returns the field pair.
template <typename FV>
__device__ __forceinline__ void gather_sum(const GridGeom& g, float x, float ex, float y, float ey, int kx0, int kxb,
                                           int ky0, int ky1, FV&& fv, float& ax, float& ay) {
    ax = 0.0f; ay = 0.0f;
    if (ky1 - ky0 < kOyCache) {
        float oy[kOyCache];
#pragma unroll
        for (int j = 0; j < kOyCache; ++j)
            oy[j] = ky0 + j <= ky1 ? bin_overlap(y, ey, g.yl, g.bsy, ky0 + j) : 0.0f;
        for (int kx = kx0; kx <= kxb; ++kx) {
            const float ox = bin_overlap(x, ex, g.xl, g.bsx, kx);
#pragma unroll
            for (int j = 0; j < kOyCache; ++j) {
                if (ky0 + j > ky1) break;
                const float w = ox * oy[j];
                const float2 v = fv(kx, ky0 + j);
                ax = fmaf(w, v.x, ax);
                ay = fmaf(w, v.y, ay);
            }
        }
        return;
    }
    for (int kx = kx0; kx <= kxb; ++kx) {
        const float ox = bin_overlap(x, ex, g.xl, g.bsx, kx);
        for (int ky = ky0; ky <= ky1; ++ky) {
            const float w = ox * bin_overlap(y, ey, g.yl, g.bsy, ky);
            const float2 v = fv(kx, ky);
            ax = fmaf(w, v.x, ax);
            ay = fmaf(w, v.y, ay);
        }
    }
}

struct TileGatherArgs {
    GridGeom g;
    TileGeom t;
    TileBins b;
    const float2* fxy;       // interleaved fields of rows [row0, row0 + rows + halo)
    int halo;                // field rows past the band
    const float* grad_out;   // nullable scalar
    float* grad_x;
    float* grad_y;
    unsigned* flags;
};

__global__ void __launch_bounds__(kTileThreads)
k_tile_gather(const __grid_constant__ TileGatherArgs a) {
    __shared__ float2 s_f[kRegionMax];
    const GridGeom& g = a.g;
    const TileBins& b = a.b;
    const int TX = 1 << a.t.ltx, TY = 1 << a.t.lty;
    const int RY = TY + kGatherLo + kGatherHi;
    const int nitems = b.meta[kMetaItems];
    const int xend = a.t.row0 + a.t.rows + a.halo;   // field rows available: [row0, xend)
    const float gscale = a.grad_out ? -__ldg(a.grad_out) : -1.0f;
    for (int item = next_item(b.meta + kMetaWorkGather, nitems); item >= 0;
         item = next_item(b.meta + kMetaWorkGather, nitems)) {
        const int2 it = b.items[item];
        const int tile = it.x;
        const int tx0 = a.t.row0 + ((tile / a.t.nty) << a.t.ltx), ty0 = (tile % a.t.nty) << a.t.lty;
        const int s0 = b.start[tile];
        const int lo = s0 + it.y * kChunk, hi = min(s0 + b.nown[tile], lo + kChunk);
        if (lo >= hi) continue;   // no owner listings in this item (uniform across the CTA)
        // staged region: rows rx0 .. rx1-1, columns ry0 .. ry1-1
        const int rx0 = max(tx0 - kGatherLo, a.t.row0), rx1 = min(tx0 + TX + kGatherHi, xend);
        const int ry0 = max(ty0 - kGatherLo, 0), ry1 = min(ty0 + TY + kGatherHi, g.N);
        const int nrx = rx1 - rx0, nry = ry1 - ry0;
        for (int e = threadIdx.x; e < nrx * RY; e += kTileThreads) {
            const int i = e / RY, jj = e % RY;
            if (jj < nry) s_f[e] = __ldg(a.fxy + (int64_t)(rx0 + i - a.t.row0) * g.N + ry0 + jj);
        }
        __syncthreads();
        for (int jl = lo + threadIdx.x; jl < hi; jl += kTileThreads) {
            const float4 gv = b.geo[jl];
            if (gv.x != gv.x) continue;   // escaped: k_esc_gather has it
            const short4 bn = b.bins[jl];
            const int4 k = b.key[jl];
            const int64_t node = (int64_t)((unsigned)k.x & kNodeMask);
            const float r = __int_as_float(k.w);
            int kxb = bn.y;
            if (kxb >= xend) {
                atomicOr(a.flags, kFlagHalo);
                kxb = xend - 1;
            }
            float ax, ay;
            if (bn.x >= rx0 && kxb < rx1 && bn.z >= ry0 && bn.w < ry1)
                gather_sum(g, gv.x, gv.z, gv.y, gv.w, bn.x, kxb, bn.z, bn.w,
                           [&](int kx, int ky) { return s_f[(kx - rx0) * RY + (ky - ry0)]; }, ax, ay);
            else
                gather_sum(g, gv.x, gv.z, gv.y, gv.w, bn.x, kxb, bn.z, bn.w,
                           [&](int kx, int ky) { return __ldg(a.fxy + (int64_t)(kx - a.t.row0) * g.N + ky); }, ax, ay);
            const float s = gscale * r;
            a.grad_x[node] = s * ax;
            a.grad_y[node] = s * ay;
        }
        __syncthreads();
    }
}

// Gradients of the escape cells from the field map in global memory.  On a
// whole grid every escape cell gets its gradient (zero when it contributes
// nothing); on a band only the cells whose first bin row is in the band
// (owned_only), as in the cell-order gather.
__global__ void __launch_bounds__(256)
k_esc_gather(CellView c, GridGeom g, TileGeom t, TileBins b, const float2* __restrict__ fxy, int halo,
             int owned_only, const float* __restrict__ grad_out, float* __restrict__ grad_x,
             float* __restrict__ grad_y, unsigned* __restrict__ flags) {
    const int ns = b.meta[kMetaEscStatic], nd = b.meta[kMetaEscDyn];
    const float gscale = grad_out ? -__ldg(grad_out) : -1.0f;
    const int xend = t.row0 + t.rows + halo;
    const int stride = gridDim.x * blockDim.x;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < ns + nd; i += stride) {
        const int64_t node = i < ns ? (int64_t)b.esc_static[i] : (int64_t)((unsigned)b.esc_dyn[i - ns] & kNodeMask);
        Footprint f;
        const int st = footprint_of(c, g, load_cell(c, node), f);
        if (st < 0) atomicOr(flags, kFlagNonFinite);
        if (owned_only && (st != 1 || f.kx0 < t.row0 || f.kx0 >= t.row0 + t.rows)) continue;
        float ax = 0.0f, ay = 0.0f, r = 0.0f;
        if (st == 1) {
            r = f.r;
            int kxb = f.kx1;
            if (kxb >= xend) {
                atomicOr(flags, kFlagHalo);
                kxb = xend - 1;
            }
            gather_sum(g, f.x, f.ex, f.y, f.ey, f.kx0, kxb, f.ky0, f.ky1,
                       [&](int kx, int ky) { return __ldg(fxy + (int64_t)(kx - t.row0) * g.N + ky); }, ax, ay);
        }
        const float s = gscale * r;
        grad_x[node] = s * ax;
        grad_y[node] = s * ay;
    }
}

}  // namespace epb
