/*
 * epb.h -- C ABI of the B200 electric-potential engine (libepb200.so).
 *
 * One handle owns the device state of one placement grid: fixed-point
 * density grid, DCT scratch, twiddle tables, the fields of the last forward.
 * All array pointers passed to these functions are DEVICE pointers on the
 * handle's device (torch.Tensor.data_ptr() works), caller-owned; the engine
 * allocates only its internal scratch, at epb_create.  Work is stream-ordered
 * on the caller's cudaStream_t (0 = legacy default stream); no call blocks the
 * host except epb_create, epb_destroy and epb_error_flags.  A handle is not
 * thread-safe: use one handle per host thread / stream.
 *
 * Every function returns an epb_status; epb_last_error() gives the message of
 * the last failure on a handle.
 *
 * What each entry point replaces in the reference project
 * (ayadavTT/DREAMPlaceTT-Framework, paths relative to its root):
 *   epb_create        host/density_scatter_ttnn_server_host.cpp:324-460 (server argv
 *                     "M N NC_max ipc_dir xl yl xh yh", sizing) and :1252-1254
 *                     (TTNNDCTSolver::init); integration/scatter_ttnn_client.py:293-390
 *                     (ScatterTTNNClient.start).
 *   epb_destroy       integration/scatter_ttnn_client.py:392-407 (stop: QUIT + wait).
 *   epb_set_initial_density
 *                     integration/scatter_ttnn_client.py:786-795 (one-time upload of
 *                     initial_density_map / bin_area) and the fold at
 *                     host/density_scatter_ttnn_server_host.cpp:1770-1777.
 *   epb_forward       integration/scatter_ttnn_client.py:411-509 (ScatterTTNNClient.call)
 *                     and the server iteration host/density_scatter_ttnn_server_host.cpp:
 *                     1326-1824 (scatter, accumulate, fold, TTNNDCTSolver::solve :272-305),
 *                     plus DREAMPlace's potential/energy (returned as 0 by the reference,
 *                     scatter_ttnn_client.py:860).
 *   epb_backward      DREAMPlace ElectricPotentialFunction.backward / electric_force
 *                     (external; reads ctx.field_map_x/y saved at
 *                     integration/scatter_ttnn_client.py:831-855).
 *   epb_scatter_fixed the scatter + accumulate programs alone (kernels/v11_scatter_dm.cpp,
 *                     kernels/v11_accum_dm.cpp; host:1630-1678) with the grid exposed
 *                     for bit-exact checks (the reference's EXPORT_DENSITY_PATH dump,
 *                     host:1687-1695).
 *   epb_dct_solve     TTNNDCTSolver::solve alone (host:272-305), as used by the
 *                     CPU_DCT=1 diagnostic split (scatter_ttnn_client.py:804-829).
 *   epb_gather        the gather half of DREAMPlace's backward on given field maps.
 *   epb_error_flags   the drop counter read-back (host:1633-1659); here it reports
 *                     skipped non-finite cells and fixed-point saturation instead.
 *   epb_profile_start / epb_profile_stop
 *                     the server's per-stage hrclock spans written to the shm header
 *                     (host:1343-1812, timing keys at integration/scatter_ttnn_client.py:492-507),
 *                     here as CUDA events on the caller's stream around each kernel.
 */
#ifndef EPB_H
#define EPB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct epb_handle epb_handle;

/* Opaque stream: pass a cudaStream_t (or torch.cuda.Stream.cuda_stream). */
typedef void* epb_stream;

typedef enum epb_status {
    EPB_OK = 0,
    EPB_EINVAL = 1,     /* bad argument (size, null pointer, unsupported grid) */
    EPB_ECUDA = 2,      /* a CUDA runtime call failed */
    EPB_ENCCL = 3,      /* reserved for the multi-GPU exchange */
    EPB_ETIMEOUT = 4,   /* a bounded wait gave up */
    EPB_EOVERFLOW = 5,  /* fixed-point density saturated (see epb_error_flags) */
    EPB_ENOSTATE = 6    /* backward called before any forward */
} epb_status;

/* Bits of the device error word returned by epb_error_flags. */
#define EPB_FLAG_NONFINITE_CELL 0x1u  /* a cell had a non-finite coordinate/size/ratio; it was skipped */
#define EPB_FLAG_SATURATED      0x2u  /* a fixed-point bin left [0, 2^62) */

/* epb_config.flags selects how the cells reach the grid:
 * EPB_CONFIG_CELL_ORDER (the default, also when flags is 0): one 64-bit
 *   global atomic add per (cell, bin) into an int64 grid, and a gather that
 *   reads the fields per cell in node order.  A shard keeps a list of the
 *   cells that meet its band widened by 8 rows, with their sizes, offsets and
 *   ratio copied beside it; every forward checks the unlisted cells against
 *   the band and lists again (on the device) when one came in.  The sizes,
 *   offsets and ratio are read when the list is made: change them in place
 *   and the shard needs other arrays (or a new handle);
 * EPB_CONFIG_TILES: cell tiles -- each cell listed in the 32 x 32-bin tiles its
 *   footprint (widened by 2 bins) meets, the lists kept across calls and
 *   validated against the positions of every forward (a shard rebuilds its
 *   band's lists every call), each tile summed exactly in shared memory and
 *   written once, its gradients read from the tile's field region in shared
 *   memory.  Measured slower than cell order on B200 (the list upkeep costs
 *   more than the atomics it saves); kept for comparison.
 * Both give the same density bit for bit and the same gradients bit for bit.
 * With the tiles, epb_backward gives the gradient at the positions of the
 * last forward on the same cell arrays (positions moved by epb_descent_step
 * since are read again). */
#define EPB_CONFIG_CELL_ORDER 0x1
#define EPB_CONFIG_TILES 0x2

typedef struct epb_config {
    int32_t num_bins_x;        /* M: bins along x = grid rows (power of two, 16..4096) */
    int32_t num_bins_y;        /* N: bins along y = grid columns (power of two, 16..4096) */
    double xl, yl, xh, yh;     /* die box; bin size = fp32((xh-xl)/M), fp32((yh-yl)/N) */
    int32_t fixed_point_bits;  /* S, fraction bits of the int64 density; <=0 selects
                                  63 - max(32, ceil(log2(die area)) + 1) */
    int32_t device;            /* CUDA device ordinal */
    int32_t flags;             /* 0, EPB_CONFIG_CELL_ORDER or EPB_CONFIG_TILES */
    int32_t reserved;
} epb_config;

/* Cells in DREAMPlace's node layout.  Cell i (0 <= i < n0 + n1, n0 = end0-begin0,
 * n1 = end1-begin1) is node  i < n0 ? begin0 + i : begin1 + (i - n0).
 * DREAMPlace orders nodes [movable | fixed terminals | fillers]; the two ranges
 * select movable and fillers so terminals (already in the initial density) are
 * skipped, as integration/scatter_ttnn_client.py:611-649 does by concatenation.
 * The cell box used for binning is [x+offset_x, x+offset_x+size_x) and likewise
 * in y; its contribution to a bin is (overlap_x * ratio) * overlap_y. */
typedef struct epb_cells {
    const float* x;          /* [num nodes] lower-left x (pos[0:num_nodes] in DREAMPlace) */
    const float* y;          /* [num nodes] lower-left y (pos[num_nodes:2*num_nodes]) */
    const float* size_x;     /* [num nodes] sizes used for binning (node_size_x_clamped) */
    const float* size_y;
    const float* offset_x;   /* nullable [num nodes]: added to x before binning */
    const float* offset_y;   /* nullable */
    const float* ratio;      /* nullable [num nodes]: per-node density scale (1 when NULL) */
    int64_t begin0, end0;    /* first node range */
    int64_t begin1, end1;    /* second node range; may be empty (begin1 == end1) */
} epb_cells;

const char* epb_version(void);
const char* epb_status_string(int status);

int epb_create(const epb_config* cfg, epb_handle** out);
int epb_destroy(epb_handle* h);
const char* epb_last_error(const epb_handle* h);

/* Geometry the handle resolved: bin sizes (fp32), fixed-point bits. */
int epb_geometry(const epb_handle* h, float* bin_size_x, float* bin_size_y, int32_t* fixed_point_bits);

/* Store the normalised fixed-cell density (initial_density_map / bin_area,
 * fp32 [M*N] device array) that every forward adds to the scattered density.
 * NULL clears it.  The array is copied (stream-ordered). */
int epb_set_initial_density(epb_handle* h, const float* init_norm, epb_stream stream);

/* Electric-potential forward: scatter -> normalised density (+ initial
 * density) -> DCT Poisson solve -> potential, fields, energy.  Output arrays
 * are nullable [M*N] fp32 device arrays (row-major, index bx*N + by);
 * energy is a nullable fp32 device scalar.  The fields are also kept inside
 * the handle for epb_backward. */
int epb_forward(epb_handle* h, const epb_cells* cells, epb_stream stream,
                float* density, float* potential, float* field_x, float* field_y,
                float* energy);

/* Per-cell density gradient from the fields of the last epb_forward:
 *   grad_x[node] = -g * ratio * sum_bins (overlap_x*overlap_y) * field_x[bin]
 * with g = *grad_out (device scalar) or 1 when grad_out is NULL.  Only nodes in
 * the cell ranges are written. */
int epb_backward(epb_handle* h, const epb_cells* cells, const float* grad_out,
                 epb_stream stream, float* grad_x, float* grad_y);

/* Scatter only: overwrite grid[M*N] (int64 device array) with the fixed-point
 * density sum of round_nearest_even(contribution * 2^S). */
int epb_scatter_fixed(epb_handle* h, const epb_cells* cells, epb_stream stream, int64_t* grid);

/* DCT solve only, from a normalised density map (fp32 [M*N], initial density
 * NOT added).  Outputs nullable as in epb_forward. */
int epb_dct_solve(epb_handle* h, const float* density, epb_stream stream,
                  float* potential, float* field_x, float* field_y, float* energy);

/* Gather only, from caller-supplied field maps. */
int epb_gather(epb_handle* h, const epb_cells* cells, const float* field_x, const float* field_y,
               const float* grad_out, epb_stream stream, float* grad_x, float* grad_y);

/* Synchronise the stream, return the accumulated EPB_FLAG_* word and clear
 * it.  Returns EPB_EOVERFLOW when EPB_FLAG_SATURATED is set. */
int epb_error_flags(epb_handle* h, epb_stream stream, uint32_t* flags);

/* ---- One grid over P GPUs -------------------------------------------------
 * The reference runs on one device (a unit mesh, host/density_scatter_ttnn_server_host.cpp:399)
 * and has no multi-device counterpart; these entry points split epb_forward /
 * epb_backward into the stages between which the caller moves data between GPUs
 * (NCCL all-to-all, all-reduce, point-to-point).  P is a power of two; shard p
 * owns grid rows [p*RB, (p+1)*RB) and, in the column pass, columns
 * [p*NB, (p+1)*NB), RB = M/P, NB = N/P.  Buffers are caller-owned device arrays:
 *   t1_send  RB*N floats  block q = [RB][NB] rows of this band, columns of band q
 *   t1_recv  M*NB floats  after all-to-all(t1_send): block q = rows of band q (= [M][NB])
 *   g_send   2*M*NB       block d = [2][RB][NB]: outputs (field_x form, potential
 *                          form) for band d's rows, columns of this band
 *   g_recv   2*M*NB       after all-to-all(g_send): block q = [2][RB][NB] from band q
 *   fxy_ext  (RB+halo)*N*2 floats: interleaved (field_x, field_y) of this band,
 *                          then `halo` rows of the next band (point-to-point)
 * t1_recv, g_send and g_recv are moved as float4 and must be 16-byte aligned,
 * fxy_band 8-byte aligned (EPB_EINVAL otherwise).
 * Every cell that overlaps the band is scattered (clipped to it), so the
 * fixed-point density of every bin is the same integer as on one GPU.  The
 * gather computes the cells whose first bin row is in the band and leaves
 * other gradient entries untouched; a footprint reaching past the halo sets
 * EPB_FLAG_HALO and is clipped.  The band list's buffers are allocated by the
 * first call with a given cell count (that call synchronises the stream), so
 * make one eager call before capturing a step into a CUDA graph. */
#define EPB_FLAG_HALO 0x4u
int epb_create_shard(const epb_config* cfg, int32_t num_shards, int32_t shard, epb_handle** out);
int epb_shard_geometry(const epb_handle* h, int32_t* num_shards, int32_t* shard, int32_t* rows_per_band,
                       int32_t* cols_per_band);
/* scatter into this band + density band (nullable, [RB][N]) + row DCT-II -> t1_send */
int epb_shard_rows_forward(epb_handle* h, const epb_cells* cells, epb_stream stream, float* density_band,
                           float* t1_send);
/* column DCT-II, weights, column inverses -> g_send; this strip's share of the
 * energy (double, device scalar, nullable) to be summed over shards.  Both
 * outputs are produced whatever want_potential says (the field_y chain is
 * derived from the potential form); the argument is kept for the caller's
 * symmetry with epb_shard_rows_inverse. */
int epb_shard_columns(epb_handle* h, const float* t1_recv, epb_stream stream, float* g_send, int32_t want_potential,
                      double* energy_partial);
/* row inverses of this band from g_recv -> potential / field_x / field_y bands
 * (nullable, [RB][N]) and the first RB rows of fxy_band; want_potential must
 * match the epb_shard_columns call (non-NULL potential_band) */
int epb_shard_rows_inverse(epb_handle* h, const float* g_recv, epb_stream stream, float* potential_band,
                           float* field_x_band, float* field_y_band, float* fxy_band);
/* gradient of the cells whose first bin row lies in this band (other entries
 * of grad_x / grad_y are left as they are).  Given the same cell arrays and
 * ranges as the shard's last forward (and no epb_descent_step since), the
 * gather uses the band list that forward checked; otherwise it checks the
 * list first.  The positions must be the ones the forward saw, as in the
 * reference, whose backward reads the pos the forward saved
 * (integration/scatter_ttnn_client.py:833). */
int epb_shard_gather(epb_handle* h, const epb_cells* cells, const float* fxy_ext, int32_t halo_rows,
                     const float* grad_out, epb_stream stream, float* grad_x, float* grad_y);

/* Peer transport: the same stages with the exchanges fused into the kernels.
 * The row pass stores its blocks directly into every shard's column strip, the
 * column pass its outputs directly into every shard's row-band buffer and the
 * row-inverse pass its first halo rows into the previous shard's field halo,
 * all as plain stores to peer memory over NVLink (CUDA IPC mappings; no
 * multicast).  After each producer a one-thread kernel publishes an epoch in
 * every shard's signal slots; a one-thread kernel waits for all shards'
 * epochs before the consumer runs, with a bounded number of polls (about 5 s
 * by default, epb_shard_set_timeout): when the bound is hit it sets
 * EPB_FLAG_TIMEOUT and returns, and epb_error_flags reports EPB_ETIMEOUT.
 * Every shard must call the peer forward (and backward) the same number of
 * times.  Buffers live in the engine; set-up is:
 *   epb_shard_peer_buffers(h, halo_rows, handles)  -> 4 cudaIpcMemHandle_t (256 bytes)
 *   (exchange the handles of all shards, in shard order)
 *   epb_shard_connect(h, all_handles)              <- P x 256 bytes
 * The energy output of epb_shard_forward_peer is the total over all shards. */
#define EPB_FLAG_TIMEOUT 0x8u
int epb_shard_peer_buffers(epb_handle* h, int32_t halo_rows, void* handles_out);
int epb_shard_connect(epb_handle* h, const void* all_handles);
int epb_shard_set_timeout(epb_handle* h, int64_t max_polls);
int epb_shard_forward_peer(epb_handle* h, const epb_cells* cells, epb_stream stream, float* density_band,
                           float* potential_band, float* field_x_band, float* field_y_band, float* energy);
int epb_shard_backward_peer(epb_handle* h, const epb_cells* cells, const float* grad_out, epb_stream stream,
                            float* grad_x, float* grad_y);
/* Test hook: waits for an epoch nobody publishes, so the bounded wait runs out
 * after max_polls polls and EPB_FLAG_TIMEOUT is set (no GPU fault, no hang). */
int epb_shard_wait_test(epb_handle* h, epb_stream stream, int64_t max_polls);

/* ---- Host buffers ------------------------------------------------------
 * The reference's client hands the server host arrays every iteration
 * (integration/scatter_ttnn_client.py:411-509: px, py, sx, sy written to shared
 * memory, field maps read back).  These two entry points take and return
 * pinned (page-locked) host buffers with no separate copy: the kernels access
 * host memory over PCIe themselves, so the transfer and the cell work overlap.
 *   epb_forward_host: the scatter reads the node positions from host_x /
 *     host_y and stores those of the nodes in the cell ranges into the device
 *     arrays cells->x / cells->y (for the backward); then it continues exactly
 *     as epb_forward (same results).
 *   epb_backward_host: as epb_backward into grad_x / grad_y (device), each
 *     gradient also stored to host_grad_x / host_grad_y; they are complete once
 *     `stream` has been synchronised.
 * Non-pinned host buffers are rejected with EPB_EINVAL.  Whole-grid handles
 * only.  No reference counterpart as entry points. */
int epb_forward_host(epb_handle* h, const epb_cells* cells, const float* host_x, const float* host_y,
                     epb_stream stream, float* density, float* potential, float* field_x, float* field_y,
                     float* energy);
int epb_backward_host(epb_handle* h, const epb_cells* cells, const float* grad_out, epb_stream stream,
                      float* grad_x, float* grad_y, float* host_grad_x, float* host_grad_y);

/* ---- Global-placement loop pieces (the operator's callers) -------------
 *
 * Overflow metric.  Replaces the per-iteration overflow that the reference
 * reads back from DREAMPlace's EvalMetrics on the host
 * (integration/run_dreamplace.py:333-370; DREAMPlace computes it with its
 * ElectricOverflow operator, which is not in the reference tree).  The cells
 * (normally the movable range alone) are scattered exactly as by epb_forward,
 * the normalised initial density is added, and with rho_b the resulting
 * density-map value of bin b:
 *   out[0] = bin_area * sum_b max(rho_b - target_density, 0)   (area units)
 *   out[1] = max_b rho_b
 * as two device doubles.  Overflow as the placer reports it is out[0] divided
 * by the total movable area.  The sum is reduced in fp64 over a fixed
 * partition of the grid (deterministic).  On a shard handle both cover the
 * band's rows; combine the ranks with a sum and a max.  Stream-ordered, no
 * host synchronisation; uses the handle's grid, so calls on one handle must
 * not overlap with its forward. */
int epb_overflow(epb_handle* h, const epb_cells* cells, float target_density, epb_stream stream, double* out);

/* epb_forward with the overflow of the first cell range folded in: the cells
 * of the first range (DREAMPlace's movable nodes) are scattered into a second
 * fixed-point grid, those of the second range (fillers) into the forward's
 * grid; out[0..1] receive the first range's overflow exactly as epb_overflow
 * reports it for that range alone; the second grid is then added into the
 * first (integer sums: the density is bit-for-bit epb_forward's for both
 * ranges) and the forward continues as epb_forward.  One scatter of every
 * cell per placement iteration instead of two.  The first call allocates the
 * second grid (M*N int64) and synchronises: make it before stream capture.
 * Whole-grid handles only. */
int epb_forward_overflow(epb_handle* h, const epb_cells* cells, float target_density, epb_stream stream,
                         double* overflow, float* density, float* potential, float* field_x, float* field_y,
                         float* energy);

/* One normalised density-descent step of every node in the cells' ranges:
 *   linf = max over those nodes of max(|grad_x|, |grad_y|)
 *   x <- max(min(x - (step_bins * bin_size_x / linf) * grad_x, xh - width), xl)
 *   y <- max(min(y - (step_bins * bin_size_y / linf) * grad_y, yh - height), yl)
 * with each fp32 operation rounded once (no contraction).  Nodes with a
 * non-finite gradient stay put and set EPB_FLAG_NONFINITE_CELL; nothing moves
 * when linf is 0.  x, y, grad_*, width, height are node-indexed device arrays
 * (DREAMPlace's pos[:n], pos[n:], its gradient halves and the unstretched node
 * sizes).  grad_linf (nullable, device) receives linf.  This is the position
 * update of the benchmark's 200-step density loop: the step that the
 * reference's placer (DREAMPlace's Nesterov optimiser, driven from
 * integration/run_dreamplace.py:315-331) takes between operator calls, reduced
 * to its density term. */
int epb_descent_step(epb_handle* h, const epb_cells* cells, float* x, float* y, const float* grad_x,
                     const float* grad_y, const float* width, const float* height, float step_bins,
                     epb_stream stream, float* grad_linf);

/* Stage timing.  Stages, in launch order: */
#define EPB_STAGE_SCATTER   0  /* cells -> density sums (tiles: -> fp32 density map) */
#define EPB_STAGE_ROW_FWD   1  /* density (+ initial density) -> row DCT-II          */
#define EPB_STAGE_COLUMN    2  /* column DCT-II, spectral weights, column inverses   */
#define EPB_STAGE_ROW_INV   3  /* row inverses -> potential, fields                  */
#define EPB_STAGE_GATHER    4  /* fields -> per-cell gradient                        */
#define EPB_STAGE_BIN       5  /* cells -> tile lists (cell-tile path: count, scan, fill) */
#define EPB_NUM_STAGES      6
/* After epb_profile_start, the next max_calls forward/backward calls record a
 * CUDA event between consecutive kernels on the caller's stream (no host
 * synchronisation).  epb_profile_stop synchronises on those events and
 * returns, per stage, the summed milliseconds and the number of launches
 * timed; it releases the events.  Calls beyond max_calls are not timed. */
int epb_profile_start(epb_handle* h, int32_t max_calls);
int epb_profile_stop(epb_handle* h, double* stage_ms, int32_t* stage_launches);

/* Diagnostic (no reference counterpart): the device's rate of the scatter's
 * atomics, measured beside the scatter.  n_cells synthetic footprints of
 * fw x fh bins (1..8 each) at hashed positions of the handle's grid, one
 * 64-bit atomic add per (footprint, bin) with its result unused, as the
 * scatter issues them; timed with CUDA events on `stream` around that kernel
 * alone.  The grid is zeroed again afterwards, as a forward expects it.
 * Whole-grid handles only.  Synchronises the stream.  *ms = the kernel's
 * time; the rate is n_cells * fw * fh / ms.  Not for use inside a graph
 * capture. */
int epb_atomic_probe(epb_handle* h, int64_t n_cells, int32_t fw, int32_t fh, epb_stream stream, double* ms);

/* Allocation-free density map.  This entry point has no counterpart in the
 * reference; it exists for callers that cannot allocate device memory: code
 * whose device memory is owned by another allocator (a framework's caching
 * allocator or a fixed memory pool that must account for every byte), and
 * code on a latency-critical path where cudaMalloc/cudaFree, which can
 * synchronise the whole device, are not acceptable.
 *
 * It computes exactly the `density` output of epb_forward (fixed-point
 * scatter, normalisation, plus the optional normalised initial density
 * init_norm[M*N]) into the caller's density[M*N], without a handle.  The
 * int64 accumulation grid lives in a fixed device array inside the library,
 * EPB_NOALLOC_MAX_BINS bins (8 MiB), which every GPU that loads the library
 * holds until the process exits.  Grids with M*N > EPB_NOALLOC_MAX_BINS are
 * rejected with EPB_EINVAL and a message in err[err_len] (nullable).
 * cfg->device selects the GPU; the first call on a device looks up the
 * array's device address there, so make that first call before any stream
 * capture.  All calls share the one array and clear it before use: calls that
 * overlap on the GPU (different streams, or different host threads) race and
 * corrupt each other's result; serialise them.  Non-finite cells are skipped;
 * saturation is not reported by this entry point (use epb_error_flags on a
 * handle for that). */
#define EPB_NOALLOC_MAX_BINS (1024 * 1024)
int epb_density_noalloc(const epb_config* cfg, const epb_cells* cells, const float* init_norm,
                        epb_stream stream, float* density, char* err, int32_t err_len);

/* ---- Wirelength of the placement objective --------------------------------
 * The other half of the objective DREAMPlace minimises around the electric
 * potential: the weighted-average (WA) wirelength with its gradient, and the
 * HPWL that EvalMetrics reports.  In the reference both come from DREAMPlace
 * (absent from the reference tree): benchmarks/configs/adaptec1_2048.json
 * selects "wirelength": "weighted_average", gamma 4.0, ignore_net_degree 100,
 * and integration/run_dreamplace.py:315-370 reads hpwl (and overflow, see
 * epb_overflow) every iteration.  These entry points replace those ops on the
 * device.
 *
 * The netlist uses DREAMPlace's flat maps, as device int32 / fp32 arrays:
 *   net_start[E+1], net_pins[P]   pins of net e: net_pins[net_start[e] .. net_start[e+1])
 *                                 (netpin_start / flat_netpin); every pin listed once
 *   pin_node[P]                   pin2node_map
 *   pin_offset_x/y[P]             pin offset from the node's lower-left corner
 *   net_weight[E]                 nullable (1)
 *   node_pin_start[V+1], node_pins[P]  pins of node v, in increasing pin order
 *                                 (flat_node2pin_start_map / flat_node2pin_map)
 *   ignore_net_degree             nets with more pins are left out of the WA
 *                                 wirelength and its gradient, not of the HPWL
 * Per net and axis, with pin coordinates v (node corner + offset, fp32):
 *   WA = sum v e^(v/g) / sum e^(v/g) - sum v e^(-v/g) / sum e^(-v/g), HPWL = max v - min v,
 * both times the net weight; nets with fewer than 2 pins contribute nothing. */
typedef struct {
    const int32_t* net_start;
    const int32_t* net_pins;
    const int32_t* pin_node;
    const float* pin_offset_x;
    const float* pin_offset_y;
    const float* net_weight;      /* nullable */
    const int32_t* node_pin_start;
    const int32_t* node_pins;
    int32_t num_nets, num_pins, num_nodes;
    int32_t ignore_net_degree;
    int32_t device;               /* CUDA device of the arrays */
} epb_netlist;

#define EPB_FLAG_BAD_INDEX 0x10u  /* a netlist index was out of range; that entry was skipped */

/* Bytes of device scratch one epb_wirelength call needs (16-byte aligned). */
size_t epb_wirelength_scratch_bytes(int32_t num_pins);

/* WA wirelength and HPWL of the netlist at node positions x[V], y[V]
 * (lower-left corners), gamma > 0 in layout units (DREAMPlace derives it from
 * params.gamma, the bin size and the overflow).  out: device double[2] =
 * {WA, HPWL}; grad_x/grad_y: nullable device float[V], the WA gradient of
 * every node (0 for nodes without pins).  Allocation-free: scratch is the
 * caller's, at least epb_wirelength_scratch_bytes(num_pins); calls sharing
 * one scratch must not overlap on the GPU.  flags: nullable device uint32,
 * EPB_FLAG_BAD_INDEX / EPB_FLAG_NONFINITE_CELL are OR-ed in (a net with a bad
 * index or a non-finite pin is skipped).  Deterministic: the same inputs give
 * the same bits.  err[err_len] (nullable) receives the message of an
 * EPB_EINVAL. */
int epb_wirelength(const epb_netlist* nl, const float* x, const float* y, float gamma, epb_stream stream,
                   void* scratch, size_t scratch_bytes, double* out, float* grad_x, float* grad_y,
                   uint32_t* flags, char* err, int32_t err_len);

#ifdef __cplusplus
}
#endif

#endif /* EPB_H */
