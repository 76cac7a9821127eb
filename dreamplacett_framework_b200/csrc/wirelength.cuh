// wirelength.cuh -- weighted-average (WA) wirelength, its gradient and the HPWL
// of a netlist: the wirelength half of the placement objective around the
// electric potential (DREAMPlace's "weighted_average" wirelength, selected in
// the reference's benchmarks/configs/adaptec1_2048.json, and the hpwl that
// integration/run_dreamplace.py:315-370 reads from EvalMetrics every iteration).
//
// For a net and one axis, with pin coordinates v_i, m = max v, n = min v:
//   a_i = exp((v_i - m)/g), b = sum a_i, f = sum v_i a_i / b
//   c_i = exp((n - v_i)/g), d = sum c_i, h = sum v_i c_i / d
//   WA = f - h,  dWA/dv_i = (a_i/b)(1 + (v_i - f)/g) - (c_i/d)(1 - (v_i - h)/g)
// (Hsu, Chang and Balabanov, DAC 2011), HPWL = m - n; both times the net weight.
//
// The exponentials are 2^(v log2 e) by the ex2.approx.ftz instruction (about
// 2^-22 relative error), well inside the 1e-5 parity bar against the float64
// restatement.
//
// Determinism: one thread computes a small net in pin order, a warp a big net
// in a fixed lane order; the node gradient sums the node's pin gradients in
// the order of the node-to-pin list; the totals are fp64 sums over a fixed
// partition.  Every run gives the same bits.
#pragma once
#include <cstdint>
#include "epb_kernels.cuh"

namespace epb {

constexpr unsigned kFlagBadIndex = 0x10u;   // an index out of range (entry skipped)
constexpr int kWlThreads = 256;
constexpr int kWlMaxBlocks = 1184;          // 148 SMs x 8
constexpr int kWlWarpDegree = 32;           // nets with more pins get a whole warp

// Scratch of one call: the block counter, the block partials,
// the pin gradients [P] (by pin), the pin positions [P] (by net-list slot).
constexpr size_t kWlPartialsOffset = 16;
constexpr size_t kWlPinGradOffset = kWlPartialsOffset + 2 * sizeof(double) * kWlMaxBlocks;

struct NetlistView {
    const int* net_start;       // [E + 1]
    const int* net_pins;        // [P] pins of each net, net by net
    const int* pin_node;        // [P]
    const float* pin_ox;        // [P] offset from the node's lower-left corner
    const float* pin_oy;
    const float* net_weight;    // nullable [E]
    const int* node_pin_start;  // [V + 1]
    const int* node_pins;       // [P] pins of each node, node by node
    int E, P, V, ignore_degree;
};

__device__ __forceinline__ double wl_warp_sum(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
    return v;
}

// exp(v) = 2^(v log2 e): callers pass v log2 e (the scale folded into their
// 1/gamma) to the ex2.approx.ftz instruction (relative error near 2^-22; a
// result below the smallest normal float is 0, as the pin's weight is then).
__device__ __forceinline__ float wl_exp2(float x) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

// Block totals in warp order: lane 0 of each warp holds its warp's sums.
__device__ __forceinline__ void wl_block_partials(double wa, double hp, double* partials) {
    __shared__ double red[2][kWlThreads / 32];
    const double a = wl_warp_sum(wa), b = wl_warp_sum(hp);
    if ((threadIdx.x & 31) == 0) {
        red[0][threadIdx.x >> 5] = a;
        red[1][threadIdx.x >> 5] = b;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        double sa = 0.0, sb = 0.0;
        for (int w = 0; w < kWlThreads / 32; ++w) { sa += red[0][w]; sb += red[1][w]; }
        partials[2 * blockIdx.x] = sa;
        partials[2 * blockIdx.x + 1] = sb;
    }
}

// Pin pass: slot_pos[k] = position of the pin in net-list slot k, one thread
// per slot: coalesced, independent loads, so the pin, node and position levels
// of every slot are in flight at once.  A bad index gives NaN and a flag; a
// non-finite position stays as it is and raises a flag.  The net passes skip a
// net with a non-finite pin.
constexpr int kWlPinsPerThread = 4;

__global__ void __launch_bounds__(kWlThreads)
k_wa_pins(NetlistView nl, const float* __restrict__ x, const float* __restrict__ y, float2* __restrict__ slot_pos,
          unsigned* __restrict__ flags) {
    unsigned bad = 0;
    const int64_t chunk = (int64_t)kWlThreads * kWlPinsPerThread;
    for (int64_t k0 = (int64_t)blockIdx.x * chunk + threadIdx.x; k0 < nl.P; k0 += (int64_t)gridDim.x * chunk) {
        // each level of loads for all kWlPinsPerThread slots before the next level
        int pin[kWlPinsPerThread], node[kWlPinsPerThread];
#pragma unroll
        for (int i = 0; i < kWlPinsPerThread; ++i) {
            const int64_t k = k0 + i * kWlThreads;
            pin[i] = k < nl.P ? __ldg(nl.net_pins + k) : -1;
        }
#pragma unroll
        for (int i = 0; i < kWlPinsPerThread; ++i) {
            node[i] = -1;
            if (pin[i] >= 0 && pin[i] < nl.P) node[i] = __ldg(nl.pin_node + pin[i]);
        }
#pragma unroll
        for (int i = 0; i < kWlPinsPerThread; ++i) {
            const int64_t k = k0 + i * kWlThreads;
            if (k >= nl.P) break;
            float px = __int_as_float(0x7fc00000), py = px;
            if (node[i] < 0 || node[i] >= nl.V) {
                bad |= kFlagBadIndex;   // a bad pin index or a bad node index
            } else {
                px = __fadd_rn(__ldg(x + node[i]), __ldg(nl.pin_ox + pin[i]));
                py = __fadd_rn(__ldg(y + node[i]), __ldg(nl.pin_oy + pin[i]));
                if (!isfinite(px) || !isfinite(py)) bad |= kFlagNonFinite;
            }
            slot_pos[k] = make_float2(px, py);
        }
    }
    if (bad && flags) atomicOr(flags, bad);
}

// Net pass: warp w takes the windows w, w + W, ... of 32 consecutive nets
// (W warps in the grid, a fixed partition, so the totals' bits never change).
//  1. lane l holds net base + l; the small nets' pins (at most kWlWarpDegree)
//     are numbered 0..T-1 across the window by a warp scan of their degrees;
//  2. the lanes copy those T pins' positions and pin indices from slot_pos and
//     net_pins to shared memory, 32 at a time (coalesced, independent loads);
//  3. lane l computes its net from shared memory in pin order (max, min, the
//     exponential sums, WA and HPWL) and leaves the net's terms in shared memory;
//  4. the lanes walk the T pins again and write each pin's gradient;
//  5. the window's big nets, one after the other, the whole warp on each.
// A window whose small nets hold more than kWlWinCap pins reads them from
// slot_pos and net_pins instead of shared memory.
constexpr int kWlWarps = kWlThreads / 32;
constexpr int kWlWinCap = 256;
constexpr int kWlWindowBlocks = 592;        // 148 SMs x 4 blocks (64 registers, 41 KB shared memory each)

struct WlNetTerms {
    float4 mm[32];   // xmax, xmin, ymax, ymin
    float4 fh[32];   // fx, hx, fy, hy
    float4 rr[32];   // 1/b, 1/d per axis: rbx, rdx, rby, rdy
    float2 wf[32];   // net weight, 1 when the net is in the WA sum (else 0)
};

// The window's pin number j (0 <= j < T) -> its net's lane, by a binary search
// over the lanes' exclusive offsets (every lane of the warp takes part).
__device__ __forceinline__ int wl_lane_of(int off, int j) {
    int n = 0;
#pragma unroll
    for (int step = 16; step > 0; step >>= 1) {
        const int v = __shfl_sync(0xffffffffu, off, n + step);
        if (v <= j) n += step;
    }
    return n;
}

// One big net (more than kWlWarpDegree pins) by the whole warp: its lanes over
// the slots, butterfly sums (every lane ends with the same totals).  WA and
// HPWL go to lane 0's sums.
__device__ __forceinline__ void wa_big_net(const NetlistView& nl, float inv_gamma, float ig2, int e, int s, int t,
                                           int lane,
                                           float2* __restrict__ pin_grad, const float2* __restrict__ slot_pos,
                                           double& wa_sum, double& hp_sum) {
    const float w = nl.net_weight ? __ldg(nl.net_weight + e) : 1.0f;
    bool ok = true;
    float xmax = -INFINITY, xmin = INFINITY, ymax = -INFINITY, ymin = INFINITY;
#pragma unroll 4
    for (int k = s + lane; k < t; k += 32) {
        const float2 pp = slot_pos[k];
        ok &= isfinite(pp.x) && isfinite(pp.y);
        xmax = fmaxf(xmax, pp.x); xmin = fminf(xmin, pp.x);
        ymax = fmaxf(ymax, pp.y); ymin = fminf(ymin, pp.y);
    }
    ok = __all_sync(0xffffffffu, ok);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        xmax = fmaxf(xmax, __shfl_xor_sync(0xffffffffu, xmax, o));
        xmin = fminf(xmin, __shfl_xor_sync(0xffffffffu, xmin, o));
        ymax = fmaxf(ymax, __shfl_xor_sync(0xffffffffu, ymax, o));
        ymin = fminf(ymin, __shfl_xor_sync(0xffffffffu, ymin, o));
    }
    if (ok && lane == 0) hp_sum += (double)(w * ((xmax - xmin) + (ymax - ymin)));
    const bool in_wa = ok && t - s <= nl.ignore_degree;
    float fx = 0.0f, hx = 0.0f, fy = 0.0f, hy = 0.0f, rbx = 1.0f, rdx = 1.0f, rby = 1.0f, rdy = 1.0f;
    if (in_wa) {
        float sax = 0.0f, scx = 0.0f, say = 0.0f, scy = 0.0f;
        float bx = 0.0f, dx = 0.0f, by = 0.0f, dy = 0.0f;
#pragma unroll 4
        for (int k = s + lane; k < t; k += 32) {
            const float2 pp = slot_pos[k];
            const float px = pp.x, py = pp.y;
            const float ax = wl_exp2((px - xmax) * ig2), cx = wl_exp2((xmin - px) * ig2);
            const float ay = wl_exp2((py - ymax) * ig2), cy = wl_exp2((ymin - py) * ig2);
            bx += ax; dx += cx; sax += px * ax; scx += px * cx;
            by += ay; dy += cy; say += py * ay; scy += py * cy;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            bx += __shfl_xor_sync(0xffffffffu, bx, o); dx += __shfl_xor_sync(0xffffffffu, dx, o);
            sax += __shfl_xor_sync(0xffffffffu, sax, o); scx += __shfl_xor_sync(0xffffffffu, scx, o);
            by += __shfl_xor_sync(0xffffffffu, by, o); dy += __shfl_xor_sync(0xffffffffu, dy, o);
            say += __shfl_xor_sync(0xffffffffu, say, o); scy += __shfl_xor_sync(0xffffffffu, scy, o);
        }
        rbx = 1.0f / bx; rdx = 1.0f / dx; rby = 1.0f / by; rdy = 1.0f / dy;
        fx = sax * rbx; hx = scx * rdx;
        fy = say * rby; hy = scy * rdy;
        if (lane == 0) wa_sum += (double)(w * ((fx - hx) + (fy - hy)));
    }
#pragma unroll 4
    for (int k = s + lane; k < t; k += 32) {
        const int pin = __ldg(nl.net_pins + k);
        if (pin < 0 || pin >= nl.P) continue;
        float2 gp = make_float2(0.0f, 0.0f);
        if (in_wa) {
            const float2 pp = slot_pos[k];
            const float px = pp.x, py = pp.y;
            const float ax = wl_exp2((px - xmax) * ig2), cx = wl_exp2((xmin - px) * ig2);
            const float ay = wl_exp2((py - ymax) * ig2), cy = wl_exp2((ymin - py) * ig2);
            gp.x = w * ((ax * rbx) * (1.0f + (px - fx) * inv_gamma) - (cx * rdx) * (1.0f - (px - hx) * inv_gamma));
            gp.y = w * ((ay * rby) * (1.0f + (py - fy) * inv_gamma) - (cy * rdy) * (1.0f - (py - hy) * inv_gamma));
        }
        pin_grad[pin] = gp;
    }
}

__global__ void __launch_bounds__(kWlThreads)
k_wa_windows(NetlistView nl, float inv_gamma, float ig2, float2* __restrict__ pin_grad, const float2* __restrict__ slot_pos,
             double* __restrict__ partials, unsigned* __restrict__ counter, double* __restrict__ out,
             unsigned* __restrict__ flags) {
    __shared__ float2 s_pos[kWlWarps][kWlWinCap];
    __shared__ int s_pin[kWlWarps][kWlWinCap];
    __shared__ unsigned char s_lane[kWlWarps][kWlWinCap];
    __shared__ WlNetTerms s_net[kWlWarps];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    float2* const wpos = s_pos[wid];
    int* const wpin = s_pin[wid];
    unsigned char* const wlane = s_lane[wid];
    WlNetTerms& nt = s_net[wid];
    const int nwarps = gridDim.x * kWlWarps;
    const int nwin = (nl.E + 31) >> 5;
    double wa_sum = 0.0, hp_sum = 0.0;
    unsigned bad = 0;
    int win = blockIdx.x * kWlWarps + wid;
    // the window's net bounds, loaded one window ahead
    int s_next = 0, t_next = 0;
    if (win < nwin && win * 32 + lane < nl.E) {
        s_next = __ldg(nl.net_start + win * 32 + lane);
        t_next = __ldg(nl.net_start + win * 32 + lane + 1);
    }
    for (; win < nwin; win += nwarps) {
        const int e = win * 32 + lane;
        int s = s_next, t = t_next;
        const float w = (e < nl.E && nl.net_weight) ? __ldg(nl.net_weight + e) : 1.0f;
        s_next = t_next = 0;
        if (win + nwarps < nwin && e + nwarps * 32 < nl.E) {
            s_next = __ldg(nl.net_start + e + nwarps * 32);
            t_next = __ldg(nl.net_start + e + nwarps * 32 + 1);
        }
        if (e < nl.E && (s < 0 || t < s || t > nl.P)) { bad |= kFlagBadIndex; s = t = 0; }
        const int deg = t - s;
        const bool big = deg > kWlWarpDegree;
        const int dsm = big ? 0 : deg;
        // exclusive scan of the small degrees: lane l's pins are [off, off + dsm)
        int inc = dsm;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += v;
        }
        const int off = inc - dsm;
        const int T = __shfl_sync(0xffffffffu, inc, 31);
        const bool in_smem = T <= kWlWinCap;
        // 2. the small nets' pins into shared memory
        if (in_smem) {
#pragma unroll 4
            for (int j0 = 0; j0 < T; j0 += 32) {
                const int j = j0 + lane;
                const int n = wl_lane_of(off, j);
                const int ns = __shfl_sync(0xffffffffu, s, n), noff = __shfl_sync(0xffffffffu, off, n);
                if (j < T) {
                    const int k = ns + (j - noff);
                    wpos[j] = slot_pos[k];
                    wpin[j] = __ldg(nl.net_pins + k);
                    wlane[j] = (unsigned char)n;
                }
            }
        }
        __syncwarp();
        // 3. lane l computes net e from its pins in pin order
        {
            const float2* src = in_smem ? wpos + off : slot_pos + s;
            bool ok = dsm >= 2;
            float xmax = -INFINITY, xmin = INFINITY, ymax = -INFINITY, ymin = INFINITY;
            for (int i = 0; i < dsm; ++i) {
                const float2 pp = src[i];
                ok &= isfinite(pp.x) && isfinite(pp.y);
                xmax = fmaxf(xmax, pp.x); xmin = fminf(xmin, pp.x);
                ymax = fmaxf(ymax, pp.y); ymin = fminf(ymin, pp.y);
            }
            if (ok) hp_sum += (double)(w * ((xmax - xmin) + (ymax - ymin)));
            const bool in_wa = ok && dsm <= nl.ignore_degree;
            float fx = 0.0f, hx = 0.0f, fy = 0.0f, hy = 0.0f, rbx = 1.0f, rdx = 1.0f, rby = 1.0f, rdy = 1.0f;
            if (in_wa) {
                float sax = 0.0f, scx = 0.0f, say = 0.0f, scy = 0.0f;
                float bx = 0.0f, dx = 0.0f, by = 0.0f, dy = 0.0f;
                for (int i = 0; i < dsm; ++i) {
                    const float2 pp = src[i];
                    const float px = pp.x, py = pp.y;
                    const float ax = wl_exp2((px - xmax) * ig2), cx = wl_exp2((xmin - px) * ig2);
                    const float ay = wl_exp2((py - ymax) * ig2), cy = wl_exp2((ymin - py) * ig2);
                    bx += ax; dx += cx; sax += px * ax; scx += px * cx;
                    by += ay; dy += cy; say += py * ay; scy += py * cy;
                }
                rbx = 1.0f / bx; rdx = 1.0f / dx; rby = 1.0f / by; rdy = 1.0f / dy;
                fx = sax * rbx; hx = scx * rdx;
                fy = say * rby; hy = scy * rdy;
                wa_sum += (double)(w * ((fx - hx) + (fy - hy)));
            }
            nt.mm[lane] = make_float4(xmax, xmin, ymax, ymin);
            nt.fh[lane] = make_float4(fx, hx, fy, hy);
            nt.rr[lane] = make_float4(rbx, rdx, rby, rdy);
            nt.wf[lane] = make_float2(w, in_wa ? 1.0f : 0.0f);
        }
        __syncwarp();
        // 4. pin gradients of the small nets (zero for a net left out)
#pragma unroll 4
        for (int j0 = 0; j0 < T; j0 += 32) {
            const int j = j0 + lane;
            int n, k = 0;
            if (in_smem) {
                n = j < T ? wlane[j] : 0;
            } else {
                n = wl_lane_of(off, j);
                const int ns = __shfl_sync(0xffffffffu, s, n), noff = __shfl_sync(0xffffffffu, off, n);
                k = ns + (j - noff);
            }
            if (j < T) {
                const int pin = in_smem ? wpin[j] : __ldg(nl.net_pins + k);
                if (pin >= 0 && pin < nl.P) {
                    float2 gp = make_float2(0.0f, 0.0f);
                    const float2 wf = nt.wf[n];
                    if (wf.y != 0.0f) {
                        const float2 pp = in_smem ? wpos[j] : slot_pos[k];
                        const float px = pp.x, py = pp.y;
                        const float4 mm = nt.mm[n], fh = nt.fh[n], rr = nt.rr[n];
                        const float ax = wl_exp2((px - mm.x) * ig2), cx = wl_exp2((mm.y - px) * ig2);
                        const float ay = wl_exp2((py - mm.z) * ig2), cy = wl_exp2((mm.w - py) * ig2);
                        gp.x = wf.x * ((ax * rr.x) * (1.0f + (px - fh.x) * inv_gamma) -
                                       (cx * rr.y) * (1.0f - (px - fh.y) * inv_gamma));
                        gp.y = wf.x * ((ay * rr.z) * (1.0f + (py - fh.z) * inv_gamma) -
                                       (cy * rr.w) * (1.0f - (py - fh.w) * inv_gamma));
                    }
                    pin_grad[pin] = gp;
                }
            }
        }
        // 5. the window's big nets, in net order
        unsigned bigs = __ballot_sync(0xffffffffu, big);
        while (bigs) {
            const int n = __ffs(bigs) - 1;
            bigs &= bigs - 1;
            const int bs = __shfl_sync(0xffffffffu, s, n), bt = __shfl_sync(0xffffffffu, t, n);
            wa_big_net(nl, inv_gamma, ig2, win * 32 + n, bs, bt, lane, pin_grad, slot_pos, wa_sum, hp_sum);
        }
        __syncwarp();   // the next window reuses this warp's shared memory
    }
    if (bad && flags) atomicOr(flags, bad);
    wl_block_partials(wa_sum, hp_sum, partials);
    // the last block adds the block partials in block order
    __shared__ bool is_last;
    if (threadIdx.x == 0) {
        __threadfence();
        is_last = atomicInc(counter, gridDim.x - 1) == gridDim.x - 1;
    }
    __syncthreads();
    if (is_last && threadIdx.x == 0) {
        __threadfence();
        double sa = 0.0, sb = 0.0;
        for (unsigned i = 0; i < gridDim.x; ++i) {
            sa += __ldcg(partials + 2 * i);
            sb += __ldcg(partials + 2 * i + 1);
        }
        out[0] = sa;
        out[1] = sb;
    }
}

// Node pass: grad[v] = sum of the gradients of v's pins, in node-to-pin order.
__global__ void __launch_bounds__(kWlThreads)
k_wa_nodes(NetlistView nl, const float2* __restrict__ pin_grad, float* __restrict__ grad_x,
           float* __restrict__ grad_y, unsigned* __restrict__ flags) {
    unsigned bad = 0;
    for (int v = blockIdx.x * blockDim.x + threadIdx.x; v < nl.V; v += gridDim.x * blockDim.x) {
        const int s = __ldg(nl.node_pin_start + v), t = __ldg(nl.node_pin_start + v + 1);
        float gx = 0.0f, gy = 0.0f;
        if (s < 0 || t < s || t > nl.P) {
            bad |= kFlagBadIndex;
        } else {
#pragma unroll 4
            for (int k = s; k < t; ++k) {
                const int pin = __ldg(nl.node_pins + k);
                if (pin < 0 || pin >= nl.P) { bad |= kFlagBadIndex; continue; }
                const float2 gp = pin_grad[pin];
                gx += gp.x;
                gy += gp.y;
            }
        }
        if (grad_x) grad_x[v] = gx;
        if (grad_y) grad_y[v] = gy;
    }
    if (bad && flags) atomicOr(flags, bad);
}

}  // namespace epb
