// fft.cuh -- shared-memory complex FFT used by the DCT-family kernels.
//
// One length-L sequence (L = 2^p, 16 <= L <= 4096) is transformed by
// P = L/16 threads of a CTA; a CTA holds several sequences, one per group of P
// consecutive threads, and all of them run the passes in lock step (each
// pass ends in __syncthreads, so every thread of the CTA must call).
//
// Schedule: Stockham autosort (natural order in and out) with radix-16
// passes and one closing radix-2/4/8 pass when p is not a multiple of 4.
// In a pass of radix R with stride Ns, butterfly b reads in[b + r*L/R],
// multiplies element r by w_{Ns*R}^{r*(b mod Ns)}, takes an R-point DFT in
// registers and writes out[(b / Ns)*Ns*R + b mod Ns + r*Ns] (E. Bainville,
// "OpenCL Fast Fourier Transform", 2010).  Every thread owns 16 values per
// pass (16/R butterflies), reads all of them, synchronises, then writes: the
// pass is a bijection, so it runs in place.
//
// Shared-memory layout: logical element p of a sequence lives at
// p + p/16 (one float2 of padding per 16), so the stride-16 writes of the
// first pass and the stride-R reads of later passes spread over all banks.
//
// Twiddles: pass (R, NS) multiplies element r of butterfly b by w^(r*k*STEP),
// k = b mod NS, STEP = L/(NS*R), w = exp(-2 pi i / L).  They are read from a
// table laid out per pass as [r][k] (k fastest) so the lanes of a warp, which
// hold consecutive k, read consecutive entries; the entries are the fp32
// roundings of the float64 values computed on the host (no device sincosf).
// INV selects exp(+...) (unnormalised inverse DFT) by conjugation.
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
// multiply by -i (forward) or +i (inverse)
template <bool INV>
__device__ __forceinline__ float2 mul_mi(float2 a) {
    return INV ? make_float2(-a.y, a.x) : make_float2(a.y, -a.x);
}

// Offset of pass NS's twiddle block in the per-pass table of length-L
// transforms (passes NS = 16, 256, ... carry twiddles; block size R*NS).
__host__ __device__ constexpr int tw_offset(int L, int NS) {
    int off = 0;
    for (int ns = 16; ns < NS; ns *= 16) off += (L / ns >= 16 ? 16 : L / ns) * ns;
    return off;
}
// Entries of the whole per-pass twiddle table of a length-L transform.
__host__ __device__ constexpr int tw_table_size(int L) { return tw_offset(L, L); }

template <int L>
struct Log2 { static constexpr int value = 1 + Log2<L / 2>::value; };
template <>
struct Log2<1> { static constexpr int value = 0; };

// padded shared-memory index and sequence stride
__device__ __forceinline__ int pidx(int p) { return p + (p >> 4); }
template <int L>
struct Padded { static constexpr int value = L + L / 16; };

// Barrier of one sequence's P threads (named barrier 1 + group) when GROUP,
// else of the whole CTA.  With per-sequence barriers the sequences of a CTA
// drift apart, so one group's loads overlap another group's arithmetic.
template <int P, bool GROUP>
__device__ __forceinline__ void seq_sync(int group) {
    if constexpr (GROUP) {
        asm volatile("bar.sync %0, %1;" ::"r"(group + 1), "r"(P) : "memory");
    } else {
        __syncthreads();
    }
}

// Per-sequence barriers need whole warps per sequence and at most 15 groups.
template <int L, int S>
struct GroupSync { static constexpr bool value = (L / 16) % 32 == 0 && S <= 15; };

// ---- small DFTs in registers, natural order in and out ----
template <bool INV>
__device__ __forceinline__ void dft2(float2* v) {
    const float2 a = v[0];
    v[0] = cadd(a, v[1]);
    v[1] = csub(a, v[1]);
}

template <bool INV>
__device__ __forceinline__ void dft4(float2& a0, float2& a1, float2& a2, float2& a3) {
    const float2 b0 = cadd(a0, a2), b1 = csub(a0, a2);
    const float2 b2 = cadd(a1, a3), b3 = mul_mi<INV>(csub(a1, a3));
    a0 = cadd(b0, b2);
    a2 = csub(b0, b2);
    a1 = cadd(b1, b3);
    a3 = csub(b1, b3);
}

template <bool INV>
__device__ __forceinline__ void dft4(float2* v) { dft4<INV>(v[0], v[1], v[2], v[3]); }

template <bool INV>
__device__ __forceinline__ void dft8(float2* v) {
    // even/odd split: X_k = E_k + w8^k O_k, X_{k+4} = E_k - w8^k O_k
    float2 e0 = v[0], e1 = v[2], e2 = v[4], e3 = v[6];
    float2 o0 = v[1], o1 = v[3], o2 = v[5], o3 = v[7];
    dft4<INV>(e0, e1, e2, e3);
    dft4<INV>(o0, o1, o2, o3);
    const float h = 0.70710678118654752440f;
    o1 = cmul(o1, make_float2(h, INV ? h : -h));
    o2 = mul_mi<INV>(o2);
    o3 = cmul(o3, make_float2(-h, INV ? h : -h));
    v[0] = cadd(e0, o0); v[4] = csub(e0, o0);
    v[1] = cadd(e1, o1); v[5] = csub(e1, o1);
    v[2] = cadd(e2, o2); v[6] = csub(e2, o2);
    v[3] = cadd(e3, o3); v[7] = csub(e3, o3);
}

template <bool INV>
__device__ __forceinline__ void dft16(float2* x) {
    // n = 4 n1 + n2, k = k1 + 4 k2:
    // Y[n2][k1] = DFT4_n1(x[4 n1 + n2]) * w16^(n2 k1);  X[k1 + 4 k2] = DFT4_n2(Y[n2][k1])
#pragma unroll
    for (int n2 = 0; n2 < 4; ++n2) dft4<INV>(x[n2], x[4 + n2], x[8 + n2], x[12 + n2]);
    // after this, x[4 k1 + n2] holds Y[n2][k1]
    const float c1 = 0.92387953251128675613f, s1 = 0.38268343236508977173f;
    const float h = 0.70710678118654752440f;
    const float sg = INV ? 1.0f : -1.0f;
    // twiddles w16^j, j = n2*k1 in {1,2,3,2,4,6,3,6,9}
    x[5] = cmul(x[5], make_float2(c1, sg * s1));     // n2=1,k1=1: j=1
    x[9] = cmul(x[9], make_float2(h, sg * h));       // n2=1,k1=2: j=2
    x[13] = cmul(x[13], make_float2(s1, sg * c1));   // n2=1,k1=3: j=3
    x[6] = cmul(x[6], make_float2(h, sg * h));       // n2=2,k1=1: j=2
    x[10] = mul_mi<INV>(x[10]);                      // n2=2,k1=2: j=4
    x[14] = cmul(x[14], make_float2(-h, sg * h));    // n2=2,k1=3: j=6
    x[7] = cmul(x[7], make_float2(s1, sg * c1));     // n2=3,k1=1: j=3
    x[11] = cmul(x[11], make_float2(-h, sg * h));    // n2=3,k1=2: j=6
    x[15] = cmul(x[15], make_float2(-c1, -sg * s1)); // n2=3,k1=3: j=9
#pragma unroll
    for (int k1 = 0; k1 < 4; ++k1) dft4<INV>(x[4 * k1], x[4 * k1 + 1], x[4 * k1 + 2], x[4 * k1 + 3]);
    // now x[4 k1 + k2] holds X[k1 + 4 k2]; transpose to natural order
    float2 t[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) t[i] = x[i];
#pragma unroll
    for (int k1 = 0; k1 < 4; ++k1)
#pragma unroll
        for (int k2 = 0; k2 < 4; ++k2) x[k1 + 4 * k2] = t[4 * k1 + k2];
}

template <int R, bool INV>
__device__ __forceinline__ void dft(float2* v) {
    if constexpr (R == 2) dft2<INV>(v);
    else if constexpr (R == 4) dft4<INV>(v);
    else if constexpr (R == 8) dft8<INV>(v);
    else dft16<INV>(v);
}

template <int L, int R, int NS, bool INV, bool GROUP>
__device__ __forceinline__ void fft_pass(float2* seq, int lane, const float2* __restrict__ tw, bool active, int group) {
    constexpr int NB = L / R;      // butterflies per sequence
    constexpr int P = L / 16;      // threads per sequence
    constexpr int BPT = NB / P;    // butterflies per thread (16 / R)
    float2 v[BPT][R];
    if (active) {
#pragma unroll
        for (int bb = 0; bb < BPT; ++bb) {
            const int b = lane + bb * P;
#pragma unroll
            for (int r = 0; r < R; ++r) v[bb][r] = seq[pidx(b + r * NB)];
        }
    }
    seq_sync<P, GROUP>(group);
#pragma unroll
    for (int bb = 0; bb < BPT; ++bb) {
        if (!active) break;
        const int b = lane + bb * P;
        const int k = b & (NS - 1);
        if (NS > 1) {
            const float2* __restrict__ twp = tw + tw_offset(L, NS) + k;
#pragma unroll
            for (int r = 1; r < R; ++r) {
                const float2 w = __ldg(twp + r * NS);
                v[bb][r] = INV ? cmulc(v[bb][r], w) : cmul(v[bb][r], w);
            }
        }
        dft<R, INV>(v[bb]);
        const int base = (b / NS) * NS * R + k;
#pragma unroll
        for (int r = 0; r < R; ++r) seq[pidx(base + r * NS)] = v[bb][r];
    }
    seq_sync<P, GROUP>(group);
}

template <int L, int NS, bool INV, bool GROUP>
__device__ __forceinline__ void fft_passes(float2* seq, int lane, const float2* __restrict__ tw, bool active,
                                           int group) {
    if constexpr (NS < L) {
        constexpr int REM = L / NS;
        constexpr int R = REM >= 16 ? 16 : REM;
        fft_pass<L, R, NS, INV, GROUP>(seq, lane, tw, active, group);
        fft_passes<L, NS * R, INV, GROUP>(seq, lane, tw, active, group);
    }
}

// Transform the padded sequence at `seq` in place; lane in [0, L/16).  Threads
// with active == false skip the arithmetic but still meet every barrier.
// GROUP selects per-sequence barriers (group = sequence index); the caller's
// own phases around the FFT must then touch only this group's sequence.
template <int L, bool INV, bool GROUP = false>
__device__ __forceinline__ void fft_seq(float2* seq, int lane, const float2* __restrict__ tw, bool active = true,
                                        int group = 0) {
    static_assert(L >= 16 && (L & (L - 1)) == 0, "power-of-two length >= 16");
    fft_passes<L, 1, INV, GROUP>(seq, lane, tw, active, group);
}

// Makhoul (1980) even/odd reordering used by both directions:
// v[n] = x[2n], v[L-1-n] = x[2n+1].  makhoul_pos(m) is where x[m] goes.
__device__ __forceinline__ int makhoul_pos(int m, int L) {
    return (m & 1) ? (L - 1 - (m >> 1)) : (m >> 1);
}

}  // namespace epb
