// fft.cuh -- shared-memory complex FFT used by the DCT-family kernels.
//
// A CTA of T threads transforms S contiguous length-L sequences held in
// shared memory (sequence s at buf + s*L), in place, natural order in and
// out.  The schedule is Stockham autosort with radix-4 stages and one closing
// radix-2 stage when log2(L) is odd (formulation of E. Bainville, "OpenCL
// Fast Fourier Transform", 2010: stage stride Ns, output index
// expand(j, Ns, R) = (j / Ns) * Ns * R + j % Ns).  Each stage reads all of a
// thread's butterfly inputs into registers, synchronises, then writes: the
// permutation is a bijection, so the in-place update is race free.
//
// Twiddles come from a table tw[t] = exp(-2*pi*i*t/L), t < L, computed in
// float64 on the host and rounded once to fp32 (no device sincosf).
// INV selects exp(+...) (unnormalised inverse DFT).
#pragma once
#include <cstdint>

namespace epb {

__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
    return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}
__device__ __forceinline__ float2 cmulc(float2 a, float2 b) {  // a * conj(b)
    return make_float2(a.x * b.x + a.y * b.y, a.y * b.x - a.x * b.y);
}
__device__ __forceinline__ float2 cadd(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
__device__ __forceinline__ float2 csub(float2 a, float2 b) { return make_float2(a.x - b.x, a.y - b.y); }

template <int L>
struct Log2 { static constexpr int value = 1 + Log2<L / 2>::value; };
template <>
struct Log2<1> { static constexpr int value = 0; };

template <int L, int S, int T, bool INV>
__device__ __forceinline__ void fft_smem(float2* buf, const float2* __restrict__ tw) {
    constexpr int LOG = Log2<L>::value;
    constexpr int NR4 = LOG / 2;
    constexpr int J4 = L / 4;                      // butterflies per sequence, radix-4
    constexpr int TOT4 = S * J4;
    constexpr int BPT4 = (TOT4 + T - 1) / T;
    const int tid = threadIdx.x;

    int Ns = 1;
#pragma unroll 1
    for (int st = 0; st < NR4; ++st) {
        float2 v[BPT4][4];
#pragma unroll
        for (int b = 0; b < BPT4; ++b) {
            const int idx = tid + b * T;
            if (TOT4 % T == 0 || idx < TOT4) {
                const int s = idx / J4, j = idx % J4;
                const float2* in = buf + s * L;
#pragma unroll
                for (int r = 0; r < 4; ++r) v[b][r] = in[j + r * J4];
            }
        }
        __syncthreads();
#pragma unroll
        for (int b = 0; b < BPT4; ++b) {
            const int idx = tid + b * T;
            if (TOT4 % T == 0 || idx < TOT4) {
                const int s = idx / J4, j = idx % J4;
                const int k = j & (Ns - 1);
                const int ts = k * (L / (4 * Ns));
                float2 a0 = v[b][0], a1, a2, a3;
                if (INV) {
                    a1 = cmulc(v[b][1], __ldg(tw + ts));
                    a2 = cmulc(v[b][2], __ldg(tw + 2 * ts));
                    a3 = cmulc(v[b][3], __ldg(tw + 3 * ts));
                } else {
                    a1 = cmul(v[b][1], __ldg(tw + ts));
                    a2 = cmul(v[b][2], __ldg(tw + 2 * ts));
                    a3 = cmul(v[b][3], __ldg(tw + 3 * ts));
                }
                const float2 b0 = cadd(a0, a2), b1 = csub(a0, a2);
                const float2 b2 = cadd(a1, a3), b3 = csub(a1, a3);
                // forward: X1 = b1 - i*b3, X3 = b1 + i*b3; inverse swaps the signs
                const float2 ib3 = make_float2(-b3.y, b3.x);  // i * b3
                float2* out = buf + s * L + (j / Ns) * Ns * 4 + k;
                out[0] = cadd(b0, b2);
                out[2 * Ns] = csub(b0, b2);
                if (INV) {
                    out[Ns] = cadd(b1, ib3);
                    out[3 * Ns] = csub(b1, ib3);
                } else {
                    out[Ns] = csub(b1, ib3);
                    out[3 * Ns] = cadd(b1, ib3);
                }
            }
        }
        __syncthreads();
        Ns *= 4;
    }
    if (LOG & 1) {
        constexpr int J2 = L / 2;
        constexpr int TOT2 = S * J2;
        constexpr int BPT2 = (TOT2 + T - 1) / T;
        float2 v[BPT2][2];
#pragma unroll
        for (int b = 0; b < BPT2; ++b) {
            const int idx = tid + b * T;
            if (TOT2 % T == 0 || idx < TOT2) {
                const int s = idx / J2, j = idx % J2;
                v[b][0] = buf[s * L + j];
                v[b][1] = buf[s * L + j + J2];
            }
        }
        __syncthreads();
#pragma unroll
        for (int b = 0; b < BPT2; ++b) {
            const int idx = tid + b * T;
            if (TOT2 % T == 0 || idx < TOT2) {
                const int s = idx / J2, j = idx % J2;
                // last stage: Ns == L/2, so k == j and the twiddle index is j
                const float2 w = __ldg(tw + j);
                const float2 a1 = INV ? cmulc(v[b][1], w) : cmul(v[b][1], w);
                buf[s * L + j] = cadd(v[b][0], a1);
                buf[s * L + j + J2] = csub(v[b][0], a1);
            }
        }
        __syncthreads();
    }
}

// Makhoul (1980) even/odd reordering used by both directions:
// v[n] = x[2n], v[L-1-n] = x[2n+1].  position_of(m) is where x[m] goes.
__device__ __forceinline__ int makhoul_pos(int m, int L) {
    return (m & 1) ? (L - 1 - (m >> 1)) : (m >> 1);
}

}  // namespace epb
