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
// Determinism: one thread computes a whole net in pin order; the node gradient
// sums the node's pin gradients in the order of the node-to-pin list; the
// totals are fp64 sums over a fixed partition.  Every run gives the same bits.
#pragma once
#include <cstdint>
#include "epb_kernels.cuh"

namespace epb {

constexpr unsigned kFlagBadIndex = 0x10u;   // an index out of range (entry skipped)
constexpr int kWlThreads = 256;
constexpr int kWlMaxBlocks = 1184;          // 148 SMs x 8: the thread-per-net pass
constexpr int kWlBigBlocks = 592;           // 148 SMs x 4: the warp-per-net pass
constexpr int kWlWarpDegree = 32;           // nets with more pins get a whole warp

// Scratch of one call: the block counter, the block partials of both passes,
// the pin gradients [P] (by pin), the pin positions [P] (by net-list slot).
constexpr size_t kWlPartialsOffset = 16;
constexpr size_t kWlPinGradOffset = kWlPartialsOffset + 2 * sizeof(double) * (kWlMaxBlocks + kWlBigBlocks);

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

// Pin coordinates of net e's k-th entry; false for a bad index or a
// non-finite position (then the net is skipped).
__device__ __forceinline__ bool wl_pin(const NetlistView& nl, const float* x, const float* y, int k, int& pin,
                                       float& px, float& py, unsigned& bad) {
    px = py = 0.0f;
    pin = __ldg(nl.net_pins + k);
    if (pin < 0 || pin >= nl.P) { bad |= kFlagBadIndex; return false; }
    const int node = __ldg(nl.pin_node + pin);
    if (node < 0 || node >= nl.V) { bad |= kFlagBadIndex; return false; }
    px = __fadd_rn(__ldg(x + node), __ldg(nl.pin_ox + pin));
    py = __fadd_rn(__ldg(y + node), __ldg(nl.pin_oy + pin));
    if (!isfinite(px) || !isfinite(py)) { bad |= kFlagNonFinite; return false; }
    return true;
}

__device__ __forceinline__ double wl_warp_sum(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
    return v;
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

// Warp pass (runs first): the nets of more than kWlWarpDegree pins, one warp
// per net, its lanes over the pins; block partials into big_partials.
__global__ void __launch_bounds__(kWlThreads)
k_wa_big_nets(NetlistView nl, const float* __restrict__ x, const float* __restrict__ y, float inv_gamma,
              float2* __restrict__ pin_grad, float2* __restrict__ slot_pos, double* __restrict__ big_partials,
              unsigned* __restrict__ flags) {
    const int lane = threadIdx.x & 31;
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, nwarps = (gridDim.x * blockDim.x) >> 5;
    double wa_sum = 0.0, hp_sum = 0.0;
    unsigned bad = 0;
    for (int base = warp * 32; base < nl.E; base += nwarps * 32) {
        // lane l looks at net base + l; the warp then takes the big ones in turn
        const int el = base + lane;
        int deg = 0;
        if (el < nl.E) deg = __ldg(nl.net_start + el + 1) - __ldg(nl.net_start + el);
        unsigned big = __ballot_sync(0xffffffffu, deg > kWlWarpDegree);
        while (big) {
            const int j = __ffs(big) - 1;
            big &= big - 1;
            const int e = base + j;
            const int s = __ldg(nl.net_start + e), t = __ldg(nl.net_start + e + 1);
            if (s < 0 || t > nl.P) { bad |= kFlagBadIndex; continue; }
            const float w = nl.net_weight ? __ldg(nl.net_weight + e) : 1.0f;
            bool ok = true;
            float xmax = -INFINITY, xmin = INFINITY, ymax = -INFINITY, ymin = INFINITY;
            for (int k = s + lane; k < t; k += 32) {
                int pin;
                float px, py;
                ok &= wl_pin(nl, x, y, k, pin, px, py, bad);
                slot_pos[k] = make_float2(px, py);   // read back by this lane in the later passes
                xmax = fmaxf(xmax, px); xmin = fminf(xmin, px);
                ymax = fmaxf(ymax, py); ymin = fminf(ymin, py);
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
            float fx = 0.0f, hx = 0.0f, fy = 0.0f, hy = 0.0f, bx = 1.0f, dx = 1.0f, by = 1.0f, dy = 1.0f;
            if (in_wa) {
                float sax = 0.0f, scx = 0.0f, say = 0.0f, scy = 0.0f;
                bx = dx = by = dy = 0.0f;
                for (int k = s + lane; k < t; k += 32) {
                    const float2 pp = slot_pos[k];
                    const float px = pp.x, py = pp.y;
                    const float ax = expf((px - xmax) * inv_gamma), cx = expf((xmin - px) * inv_gamma);
                    const float ay = expf((py - ymax) * inv_gamma), cy = expf((ymin - py) * inv_gamma);
                    bx += ax; dx += cx; sax += px * ax; scx += px * cx;
                    by += ay; dy += cy; say += py * ay; scy += py * cy;
                }
                // butterfly sums: every lane ends with the same totals
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    bx += __shfl_xor_sync(0xffffffffu, bx, o); dx += __shfl_xor_sync(0xffffffffu, dx, o);
                    sax += __shfl_xor_sync(0xffffffffu, sax, o); scx += __shfl_xor_sync(0xffffffffu, scx, o);
                    by += __shfl_xor_sync(0xffffffffu, by, o); dy += __shfl_xor_sync(0xffffffffu, dy, o);
                    say += __shfl_xor_sync(0xffffffffu, say, o); scy += __shfl_xor_sync(0xffffffffu, scy, o);
                }
                fx = sax / bx; hx = scx / dx;
                fy = say / by; hy = scy / dy;
                if (lane == 0) wa_sum += (double)(w * ((fx - hx) + (fy - hy)));
            }
            for (int k = s + lane; k < t; k += 32) {
                const int pin = __ldg(nl.net_pins + k);
                if (pin < 0 || pin >= nl.P) continue;
                float2 gp = make_float2(0.0f, 0.0f);
                if (in_wa) {
                    const float2 pp = slot_pos[k];
                    const float px = pp.x, py = pp.y;
                    const float ax = expf((px - xmax) * inv_gamma), cx = expf((xmin - px) * inv_gamma);
                    const float ay = expf((py - ymax) * inv_gamma), cy = expf((ymin - py) * inv_gamma);
                    gp.x = w * ((ax / bx) * (1.0f + (px - fx) * inv_gamma) - (cx / dx) * (1.0f - (px - hx) * inv_gamma));
                    gp.y = w * ((ay / by) * (1.0f + (py - fy) * inv_gamma) - (cy / dy) * (1.0f - (py - hy) * inv_gamma));
                }
                pin_grad[pin] = gp;
            }
        }
    }
    if (bad && flags) atomicOr(flags, bad);
    wl_block_partials(wa_sum, hp_sum, big_partials);
}

// Thread pass: the nets of at most kWlWarpDegree pins, one thread per net in
// pin order; per-pin WA gradients into pin_grad[pin] (zero for pins of nets
// that contribute nothing).  Its last block writes out[0] = WA, out[1] = HPWL:
// the warp pass's block partials, then this pass's, each in block order.
// Nets of at most kWlSmall pins take a register path: every level of loads
// (pins, then nodes and offsets, then positions) is issued for all pins at
// once, and each pin's exponentials are computed once.  The operations and
// their order are those of the general loops, so both give the same bits.
constexpr int kWlSmall = 4;

__device__ __forceinline__ void wa_small_net(const NetlistView& nl, const float* __restrict__ x,
                                             const float* __restrict__ y, float inv_gamma, int s, int deg, float w,
                                             float2* __restrict__ pin_grad, double& wa_sum, double& hp_sum,
                                             unsigned& bad) {
    int pin[kWlSmall], node[kWlSmall];
    float px[kWlSmall], py[kWlSmall];
    bool ok = deg >= 2;
#pragma unroll
    for (int j = 0; j < kWlSmall; ++j) pin[j] = j < deg ? __ldg(nl.net_pins + s + j) : 0;
#pragma unroll
    for (int j = 0; j < kWlSmall; ++j) {
        node[j] = 0;
        if (j < deg) {
            if (pin[j] < 0 || pin[j] >= nl.P) { bad |= kFlagBadIndex; ok = false; pin[j] = -1; }
            else node[j] = __ldg(nl.pin_node + pin[j]);
        }
    }
    float ox[kWlSmall], oy[kWlSmall];
#pragma unroll
    for (int j = 0; j < kWlSmall; ++j) {
        ox[j] = oy[j] = 0.0f;
        if (j < deg && pin[j] >= 0) {
            if (node[j] < 0 || node[j] >= nl.V) { bad |= kFlagBadIndex; ok = false; node[j] = -1; }
            else { ox[j] = __ldg(nl.pin_ox + pin[j]); oy[j] = __ldg(nl.pin_oy + pin[j]); }
        }
    }
    float xmax = -INFINITY, xmin = INFINITY, ymax = -INFINITY, ymin = INFINITY;
#pragma unroll
    for (int j = 0; j < kWlSmall; ++j) {
        px[j] = py[j] = 0.0f;
        if (j < deg && pin[j] >= 0 && node[j] >= 0) {
            px[j] = __fadd_rn(__ldg(x + node[j]), ox[j]);
            py[j] = __fadd_rn(__ldg(y + node[j]), oy[j]);
            if (!isfinite(px[j]) || !isfinite(py[j])) { bad |= kFlagNonFinite; ok = false; px[j] = py[j] = 0.0f; }
        }
        if (j < deg) {
            xmax = fmaxf(xmax, px[j]); xmin = fminf(xmin, px[j]);
            ymax = fmaxf(ymax, py[j]); ymin = fminf(ymin, py[j]);
        }
    }
    if (ok) hp_sum += (double)(w * ((xmax - xmin) + (ymax - ymin)));
    const bool in_wa = ok && deg <= nl.ignore_degree;
    float ax[kWlSmall], cx[kWlSmall], ay[kWlSmall], cy[kWlSmall];
    float fx = 0.0f, hx = 0.0f, fy = 0.0f, hy = 0.0f, bx = 1.0f, dx = 1.0f, by = 1.0f, dy = 1.0f;
    if (in_wa) {
        float sax = 0.0f, scx = 0.0f, say = 0.0f, scy = 0.0f;
        bx = dx = by = dy = 0.0f;
#pragma unroll
        for (int j = 0; j < kWlSmall; ++j) {
            if (j >= deg) break;
            ax[j] = expf((px[j] - xmax) * inv_gamma); cx[j] = expf((xmin - px[j]) * inv_gamma);
            ay[j] = expf((py[j] - ymax) * inv_gamma); cy[j] = expf((ymin - py[j]) * inv_gamma);
            bx += ax[j]; dx += cx[j]; sax += px[j] * ax[j]; scx += px[j] * cx[j];
            by += ay[j]; dy += cy[j]; say += py[j] * ay[j]; scy += py[j] * cy[j];
        }
        fx = sax / bx; hx = scx / dx;
        fy = say / by; hy = scy / dy;
        wa_sum += (double)(w * ((fx - hx) + (fy - hy)));
    }
#pragma unroll
    for (int j = 0; j < kWlSmall; ++j) {
        if (j >= deg) break;
        if (pin[j] < 0) continue;
        float2 gp = make_float2(0.0f, 0.0f);
        if (in_wa) {
            gp.x = w * ((ax[j] / bx) * (1.0f + (px[j] - fx) * inv_gamma) -
                        (cx[j] / dx) * (1.0f - (px[j] - hx) * inv_gamma));
            gp.y = w * ((ay[j] / by) * (1.0f + (py[j] - fy) * inv_gamma) -
                        (cy[j] / dy) * (1.0f - (py[j] - hy) * inv_gamma));
        }
        pin_grad[pin[j]] = gp;
    }
}

__global__ void __launch_bounds__(kWlThreads)
k_wa_nets(NetlistView nl, const float* __restrict__ x, const float* __restrict__ y, float inv_gamma,
          float2* __restrict__ pin_grad, float2* __restrict__ slot_pos, double* __restrict__ partials,
          const double* __restrict__ big_partials,
          int big_blocks, unsigned* __restrict__ counter, double* __restrict__ out, unsigned* __restrict__ flags) {
    double wa_sum = 0.0, hp_sum = 0.0;
    unsigned bad = 0;
    for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < nl.E; e += gridDim.x * blockDim.x) {
        const int s = __ldg(nl.net_start + e), t = __ldg(nl.net_start + e + 1);
        if (s < 0 || t < s || t > nl.P) { bad |= kFlagBadIndex; continue; }
        if (t - s > kWlWarpDegree) continue;        // the warp pass's net
        const float w = nl.net_weight ? __ldg(nl.net_weight + e) : 1.0f;
        if (t - s <= kWlSmall) {
            wa_small_net(nl, x, y, inv_gamma, s, t - s, w, pin_grad, wa_sum, hp_sum, bad);
            continue;
        }
        bool ok = t - s >= 2;
        float xmax = -INFINITY, xmin = INFINITY, ymax = -INFINITY, ymin = INFINITY;
#pragma unroll 4
        for (int k = s; k < t; ++k) {
            int pin;
            float px, py;
            ok &= wl_pin(nl, x, y, k, pin, px, py, bad);
            slot_pos[k] = make_float2(px, py);   // read back by this thread in the later passes
            xmax = fmaxf(xmax, px); xmin = fminf(xmin, px);
            ymax = fmaxf(ymax, py); ymin = fminf(ymin, py);
        }
        if (ok) hp_sum += (double)(w * ((xmax - xmin) + (ymax - ymin)));
        const bool in_wa = ok && t - s <= nl.ignore_degree;
        float fx = 0.0f, hx = 0.0f, fy = 0.0f, hy = 0.0f, bx = 1.0f, dx = 1.0f, by = 1.0f, dy = 1.0f;
        if (in_wa) {
            float sax = 0.0f, scx = 0.0f, say = 0.0f, scy = 0.0f;
            bx = dx = by = dy = 0.0f;
#pragma unroll 4
            for (int k = s; k < t; ++k) {
                const float2 pp = slot_pos[k];
                const float px = pp.x, py = pp.y;
                const float ax = expf((px - xmax) * inv_gamma), cx = expf((xmin - px) * inv_gamma);
                const float ay = expf((py - ymax) * inv_gamma), cy = expf((ymin - py) * inv_gamma);
                bx += ax; dx += cx; sax += px * ax; scx += px * cx;
                by += ay; dy += cy; say += py * ay; scy += py * cy;
            }
            fx = sax / bx; hx = scx / dx;
            fy = say / by; hy = scy / dy;
            wa_sum += (double)(w * ((fx - hx) + (fy - hy)));
        }
        // pin gradients (zero when the net is left out)
#pragma unroll 4
        for (int k = s; k < t; ++k) {
            const int pin = __ldg(nl.net_pins + k);
            if (pin < 0 || pin >= nl.P) continue;
            float2 gp = make_float2(0.0f, 0.0f);
            if (in_wa) {
                const float2 pp = slot_pos[k];
                const float px = pp.x, py = pp.y;
                const float ax = expf((px - xmax) * inv_gamma), cx = expf((xmin - px) * inv_gamma);
                const float ay = expf((py - ymax) * inv_gamma), cy = expf((ymin - py) * inv_gamma);
                gp.x = w * ((ax / bx) * (1.0f + (px - fx) * inv_gamma) - (cx / dx) * (1.0f - (px - hx) * inv_gamma));
                gp.y = w * ((ay / by) * (1.0f + (py - fy) * inv_gamma) - (cy / dy) * (1.0f - (py - hy) * inv_gamma));
            }
            pin_grad[pin] = gp;
        }
    }
    if (bad && flags) atomicOr(flags, bad);
    wl_block_partials(wa_sum, hp_sum, partials);
    __shared__ bool is_last;
    if (threadIdx.x == 0) {
        __threadfence();
        is_last = atomicInc(counter, gridDim.x - 1) == gridDim.x - 1;
    }
    __syncthreads();
    if (is_last && threadIdx.x == 0) {
        __threadfence();
        double sa = 0.0, sb = 0.0;
        for (int i = 0; i < big_blocks; ++i) {
            sa += __ldcg(big_partials + 2 * i);
            sb += __ldcg(big_partials + 2 * i + 1);
        }
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
