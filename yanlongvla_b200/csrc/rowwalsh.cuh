// Row transform helpers shared by the rotation kernels (rotate.cu) and the decode-GEMV with its pre fused
// (trellis.cu): the block Walsh of one token row, the per-token INT8 quantizer and the input loaders.
//
// A row of width K (multiple of 16, <= 16384) is the concatenation of descending power-of-two blocks
// (tcq_format.py:26-30); each block gets the FP32 Walsh transform with stages h = 1, 2, 4, ... and the scale
// (float)(1 / sqrt(w)) (tcq_format.py:44-55); every kernel that includes this header computes it the same way, so
// their results agree bit for bit.
//
// A thread holds CH contiguous elements of the row (a chunk; CH = 4 or 16). CH = 16 gives every thread more
// independent work (many-row launches, bound by throughput); CH = 4 puts four times as many threads on a row, so a
// launch of a few rows (bound by the latency of each thread's instruction stream) finishes sooner. The arithmetic is
// the same for both: only which thread performs an addition changes, never its operands or their order.
#pragma once
#include <type_traits>

#include "tcq_common.cuh"

namespace tcq {

// ---------------------------------------------------------------------------------------------------- row transform
template <int R, class Fin>
__device__ __forceinline__ void walsh_pass(float* buf, int off, int w, int S, bool last, Fin& fin) {
    const int G = w >> R;
    const float c = wscale(w);
#pragma unroll 1
    for (int g = threadIdx.x; g < G; g += blockDim.x) {
        const int low = g & (S - 1);
        const int base = off + (((g - low) << R) | low);
        // S is a multiple of 128 and swz only permutes bits 2..3 by bits 5..6, so swz(base + k S) = swz(base) + k S.
        float* p = buf + swz(base);
        float v[1 << R];
#pragma unroll
        for (int k = 0; k < (1 << R); ++k) v[k] = p[k * S];
        bfly<R>(v);
        if (last) {
#pragma unroll
            for (int k = 0; k < (1 << R); ++k) fin(base + k * S, v[k] * c);
        } else {
#pragma unroll
            for (int k = 0; k < (1 << R); ++k) p[k * S] = v[k];
        }
    }
}

template <int CH>
struct ChunkLog {
    static constexpr int value = CH == 16 ? 4 : 2;
};

// ldc(c, v): the CH inputs of chunk c (indices CH c .. CH c + CH - 1). fin(i, value): called exactly once per index
// with the finished, scaled value (by the thread that owns index i in that pass; it may write buf[swz(i)]).
// finc(i0, v): the same for the CH finished values of a whole chunk i0 .. i0 + CH - 1 at once (blocks of up to
// 32 CH, finished in registers), so that callers load their per-index operands and store their results in vectors.
// Ends with a __syncthreads() so that values fin / finc stored to buf are visible to the whole block.
//
// Stages h = 1 .. CH/2 run in registers on a thread's CH contiguous inputs; h = CH .. 16 CH across the 32 lanes of a
// warp, which hold 32 consecutive chunks (lane partner = lane ^ h/CH: the lower lane keeps a + b, the upper
// b' = a - b, the reference's operands in its order; both as one rounding of (+-1) * own + partner); blocks of up to
// 32 CH are then done. Wider blocks finish with radix-16 passes through shared memory at stride 32 CH (then 16 times
// that). Threads per row are a multiple of 32, so a warp's chunks are consecutive; blocks are aligned to their width,
// so a stage never pairs chunks of different blocks. The cross-lane stages are a rolled loop (less code to fetch).
// A thread with several chunks (rows wider than its block's threads hold at once) loads the inputs of NP of them
// before transforming any, so that their global-memory round trips overlap instead of following one another. ldc
// only reads (the same thread's chunks may be rewritten by finc afterwards).
template <int CH, int NP = (CH == 4 ? 2 : 1), class Ldc, class Finc, class Fin>
__device__ __forceinline__ void row_walshc(float* buf, int K, Ldc ldc, Finc finc, Fin fin) {
    constexpr int LC = ChunkLog<CH>::value;
    const int nch = K >> LC, lane = threadIdx.x & 31;
#pragma unroll 1
    for (int cg = threadIdx.x - lane; cg < nch; cg += NP * blockDim.x) {     // warp-uniform
        float vv[NP][CH];
#pragma unroll
        for (int j = 0; j < NP; ++j) {
            const int c = cg + j * (int)blockDim.x + lane;
            if (c < nch) {
                ldc(c, vv[j]);
            } else {
#pragma unroll
                for (int k = 0; k < CH; ++k) vv[j][k] = 0.f;
            }
        }
#pragma unroll
        for (int j = 0; j < NP; ++j) {
            const int c0 = cg + j * (int)blockDim.x;
            if (c0 >= nch) break;                                              // warp-uniform
            const int c = c0 + lane;
            float* v = vv[j];
            int w = 0;                                                         // width of this chunk's block
            if (c < nch) {
                bfly<LC>(v);
                w = block_of(c << LC, K);
            }
#pragma unroll 1
            for (int hc = 1; hc < 32; hc <<= 1) {                             // stage h = CH hc
                if (!__any_sync(0xffffffffu, w > CH * hc)) break;
                const bool act = w > CH * hc;
                const float sg = (lane & hc) ? -1.f : 1.f;                     // upper lane: partner - own
#pragma unroll
                for (int k = 0; k < CH; ++k) {
                    const float p = __shfl_xor_sync(0xffffffffu, v[k], hc);
                    if (act) v[k] = __fmaf_rn(sg, v[k], p);
                }
            }
            if (c < nch) {
                const int i0 = c << LC;
                if (w <= 32 * CH) {
                    const float sc = wscale(w);
#pragma unroll
                    for (int k = 0; k < CH; ++k) v[k] = v[k] * sc;
                    finc(i0, v);
                } else {
                    float4* b4 = reinterpret_cast<float4*>(buf);
#pragma unroll
                    for (int q = 0; q < CH / 4; ++q) b4[swz(i0 + 4 * q) >> 2] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
                }
            }
        }
    }
    __syncthreads();
#pragma unroll 1
    for (int S = 32 * CH;; S <<= 4) {
        bool work = false;
        int off = 0;
#pragma unroll 1
        for (int rem = K; rem;) {
            const int w = 1 << (31 - __clz(rem));
            if (w > S) {
                work = true;
                const int L = 31 - __clz(w / S);
                const bool last = L <= 4;
                switch (last ? L : 4) {
                    case 4: walsh_pass<4>(buf, off, w, S, last, fin); break;
                    case 3: walsh_pass<3>(buf, off, w, S, last, fin); break;
                    case 2: walsh_pass<2>(buf, off, w, S, last, fin); break;
                    default: walsh_pass<1>(buf, off, w, S, last, fin); break;
                }
            }
            off += w;
            rem -= w;
        }
        __syncthreads();
        if (!work) break;
    }
}

// The transform with a per-index finisher only.
template <int CH, class Ldc, class Fin>
__device__ __forceinline__ void row_walsh(float* buf, int K, Ldc ldc, Fin fin) {
    row_walshc<CH>(buf, K, ldc, [&](int i0, const float* v) {
#pragma unroll
        for (int k = 0; k < CH; ++k) fin(i0 + k, v[k]);
    }, fin);
}

// finc of a pass whose result is the finished row in buf (at swz(i)) plus its absolute maximum.
template <int CH>
__device__ __forceinline__ void store_chunk(float* buf, int i0, const float* v, float& mx) {
    float4* b4 = reinterpret_cast<float4*>(buf);
#pragma unroll
    for (int q = 0; q < CH / 4; ++q) {
        b4[swz(i0 + 4 * q) >> 2] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
#pragma unroll
        for (int k = 0; k < 4; ++k) mx = fmaxf(mx, fabsf(v[4 * q + k]));
    }
}

__device__ __forceinline__ float block_max(float mx, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    float r = 0.f;
    const int warps = (blockDim.x + 31) >> 5;
    for (int i = 0; i < warps; ++i) r = fmaxf(r, red[i]);
    return r;
}

// Per-token INT8 quantizer (tcq_format.py:119-122; kernels.py:164-184): s = amax / 127 (IEEE division, 1 when
// amax = 0), q = clamp(rint(v / s), -127, 127). q (M, K) row-major and/or q4 (K/4, ldq) words, token = column.
//
// rint(v / s) without a division per element, by a guard band around the rounding boundaries: with rs = 1 / s
// (IEEE, once per row) the product a = v * rs is within |v / s| * 2^-23 (two roundings of 2^-24) of the true
// quotient, i.e. within 1.52e-5 for |v / s| <= 127.5. When a lies more than 3.1e-5 from the nearest half-integer,
// the quotient lies on the same side of it (more than 1.52e-5 away), so rint(a) = rint(v / s); otherwise -- and for
// NaN, infinities and an overflowing reciprocal, where the test is false -- the quotient is computed by division.
// Either way the result is rint of the correctly rounded quotient, bit for bit.
__device__ __forceinline__ int q8(float v, float s, float rs) {
    const float a = v * rs;
    float r = rintf(a);
    if (!(fabsf(fabsf(a - r) - 0.5f) > 3.1e-5f)) r = rintf(v / s);
    r = fminf(fmaxf(r, -127.f), 127.f);
    return (int)r;
}

// One q4 word (four values) per thread and step, so that every thread of the block takes part.
__device__ __forceinline__ void quantize_store(const float* buf, float mx, float* red, int8_t* q, int* q4, float* scale,
                                               int tok, int K, int ldq) {
    mx = block_max(mx, red);
    const float s = mx > 0.f ? mx / 127.f : 1.f, rs = 1.f / s;
    if (threadIdx.x == 0) scale[tok] = s;
    const float4* b4 = reinterpret_cast<const float4*>(buf);
#pragma unroll 1
    for (int g = threadIdx.x; g < (K >> 2); g += blockDim.x) {
        const float4 v = b4[swz(4 * g) >> 2];
        const u32 w = (u32)(q8(v.x, s, rs) & 0xff) | ((u32)(q8(v.y, s, rs) & 0xff) << 8) | ((u32)(q8(v.z, s, rs) & 0xff) << 16) |
                      ((u32)(q8(v.w, s, rs) & 0xff) << 24);
        if (q) reinterpret_cast<u32*>(q + (size_t)tok * K)[g] = w;
        if (q4) q4[(size_t)g * ldq + tok] = (int)w;
    }
}

// ---------------------------------------------------------------------------------------------------- chunk I/O
template <int CH>
__device__ __forceinline__ void pack_bf16c(const float* v, u32* w) {
#pragma unroll
    for (int k = 0; k < CH / 2; ++k) w[k] = f2bf2(v[2 * k], v[2 * k + 1]);
}

// CH packed BF16 values (2 CH bytes) to p, aligned to 2 CH bytes (global or shared): vector stores.
template <int CH>
__device__ __forceinline__ void store_bf16c(u16* p, const u32* w) {
    if (CH == 16) {
        store16_bf16(p, w);
    } else {
        *reinterpret_cast<uint2*>(p) = make_uint2(w[0], w[1]);
    }
}

// The same for a destination of unknown alignment (a caller's output view): vector stores when p allows them.
template <int CH>
__device__ __forceinline__ void store_bf16c_any(u16* p, const u32* w) {
    if ((reinterpret_cast<uintptr_t>(p) & (2 * CH - 1)) == 0) {
        store_bf16c<CH>(p, w);
    } else {
#pragma unroll
        for (int k = 0; k < CH / 2; ++k) {
            p[2 * k] = (u16)(w[k] & 0xffffu);
            p[2 * k + 1] = (u16)(w[k] >> 16);
        }
    }
}

// ---------------------------------------------------------------------------------------------------- loaders
// NB bytes (4, 8 or a multiple of 16) from p, aligned to min(NB, 16), as 32-bit words. G: p is global memory the
// kernel only reads (__ldg); otherwise p may be in any address space (plain loads).
template <int NB, bool G>
__device__ __forceinline__ void ldw(const void* p, u32* w) {
    if (NB >= 16) {
        const uint4* u = reinterpret_cast<const uint4*>(p);
#pragma unroll
        for (int q = 0; q < NB / 16; ++q) {
            const uint4 a = G ? __ldg(u + q) : u[q];
            w[4 * q] = a.x; w[4 * q + 1] = a.y; w[4 * q + 2] = a.z; w[4 * q + 3] = a.w;
        }
    } else if (NB == 8) {
        const uint2 a = G ? __ldg(reinterpret_cast<const uint2*>(p)) : *reinterpret_cast<const uint2*>(p);
        w[0] = a.x; w[1] = a.y;
    } else {
        w[0] = G ? __ldg(reinterpret_cast<const u32*>(p)) : *reinterpret_cast<const u32*>(p);
    }
}

// CH inputs of a row (BF16 / F16 / F32) from global memory.
template <int DT, int CH>
__device__ __forceinline__ void loadc(const void* p, float* v) {
    if (DT == TCQ_DT_F32) {
        u32 w[CH];
        ldw<4 * CH, true>(p, w);
#pragma unroll
        for (int k = 0; k < CH; ++k) v[k] = __uint_as_float(w[k]);
    } else {
        u32 w[CH / 2];
        ldw<2 * CH, true>(p, w);
#pragma unroll
        for (int k = 0; k < CH / 2; ++k) {
            if (DT == TCQ_DT_BF16) {
                v[2 * k] = __uint_as_float(w[k] << 16);
                v[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
            } else {
                v[2 * k] = h2f((u16)(w[k] & 0xffff));
                v[2 * k + 1] = h2f((u16)(w[k] >> 16));
            }
        }
    }
}

// CH BF16 values from p (global or shared; plain loads).
template <int CH>
__device__ __forceinline__ void load_bf16c_any(const u16* p, float* v) {
    u32 w[CH / 2];
    ldw<2 * CH, false>(p, w);
#pragma unroll
    for (int k = 0; k < CH / 2; ++k) {
        v[2 * k] = __uint_as_float(w[k] << 16);
        v[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
    }
}

// CH signs (+-1 as int8) as floats; G as in ldw.
template <int CH, bool G>
__device__ __forceinline__ void load_signsc(const i8* p, float* sg) {
    u32 w[CH / 4];
    ldw<CH, G>(p, w);
#pragma unroll
    for (int k = 0; k < CH; ++k) sg[k] = (float)(i8)((w[k >> 2] >> (8 * (k & 3))) & 0xff);
}

// CH FP32 values; G as in ldw.
template <int CH, bool G>
__device__ __forceinline__ void load_f32c(const float* p, float* v) {
    u32 w[CH];
    ldw<4 * CH, G>(p, w);
#pragma unroll
    for (int k = 0; k < CH; ++k) v[k] = __uint_as_float(w[k]);
}

// Scaled accumulator inputs z = SCALE(acc): I32 ((float)a * s) * rs, F32 a, BF16 bf2f(a) * rs (kernels.py:545).
// rs may be a shared-memory copy (stage_const).
template <int AT, int CH>
__device__ __forceinline__ void load_scaledc(const void* acc, size_t idx, float s, const float* rs, float* v) {
    if (AT == TCQ_DT_I32) {
        float r[CH];
        load_f32c<CH, false>(rs, r);
        u32 a[CH];
        ldw<4 * CH, true>(reinterpret_cast<const int*>(acc) + idx, a);
#pragma unroll
        for (int k = 0; k < CH; ++k) v[k] = ((float)(int)a[k] * s) * r[k];
    } else if (AT == TCQ_DT_F32) {
        load_f32c<CH, true>(reinterpret_cast<const float*>(acc) + idx, v);
    } else {
        float r[CH];
        load_f32c<CH, false>(rs, r);
        loadc<TCQ_DT_BF16, CH>(reinterpret_cast<const u16*>(acc) + idx, v);
#pragma unroll
        for (int k = 0; k < CH; ++k) v[k] = v[k] * r[k];
    }
}

// ---------------------------------------------------------------------------------------------------- windowed transform
// The block Walsh of one power-of-two row of D = 2^NL elements (1024 .. 16384) held by D / 32 threads, 32 elements
// each, in register windows: a thread's 32 elements are V consecutive ones (V = 2 from 4096 wide, 4 below) times the
// 2^(5 - log2 V) values of a window of index bits; the window's new butterfly stages run in registers in the
// definition's order (h = 1, 2, 4, ...), so the sums are the row transform's bit for bit; between windows the row
// passes through shared memory as groups of V floats with one padding group per 2^(5 - log2 V) (conflict-free).
template <int NL, int V>
struct Win2 {
    static_assert(V == 2 || V == 4, "exchange vectors of 2 or 4 floats");
    static constexpr int VB = V == 2 ? 1 : 2, WB = 5 - VB;
    static constexpr int P = 1 + (NL - 5 + WB - 1) / WB;                                 // windows
    static constexpr int first(int p) { return p == 0 ? 0 : 5 + WB * (p - 1); }        // first index bit new in window p
    static constexpr int lo(int p) { return p == 0 ? VB : (first(p) + WB <= NL ? first(p) : NL - WB); }
};

template <int NL>
constexpr int rot_vec() { return NL >= 12 ? 2 : 4; }

// The windowed block Walsh of one power-of-two row of D = 2^NL elements held by D / 32 threads, 32 each: on entry v is
// the thread's window 0 (its 32 consecutive elements 32 t .. 32 t + 31); on return v is the unscaled transform in the
// last window's layout (register V q + k holds element win_elem<NL>(t, q, k)). buf: D + D / 2^WB floats of shared
// memory for the exchanges. REUSE: buf may still be read by another thread's previous use, so the first exchange
// waits for the whole block first. Contains __syncthreads().
// Barrier of the threads that run a windowed transform. BAR 0: the whole block (__syncthreads); 1: the whole block in
// the unaligned form, for code where the threads take different branches that each execute the same number of
// barriers (two power-of-two blocks of one row); 2: only the first NT threads (named barrier 1), for a transform run
// by part of a larger block.
template <int BAR, int NT = 0>
__device__ __forceinline__ void blk_sync() {
    if constexpr (BAR == 0) __syncthreads();
    else if constexpr (BAR == 1) asm volatile("barrier.sync 0;" ::: "memory");
    else asm volatile("barrier.sync 1, %0;" ::"n"(NT) : "memory");
}

template <int NL, bool REUSE, int BAR = 0>
__device__ __forceinline__ void win_walsh(float (&v)[32], float* buf, int t) {
    constexpr int V = rot_vec<NL>();
    using W = Win2<NL, V>;
    constexpr int VB = W::VB, WB = W::WB, G = 1 << WB;
    static_assert(NL >= 2 * WB + VB, "every window after the first needs lo - log2 V >= WB");
    using VecT = typename std::conditional<V == 2, float2, float4>::type;
    VecT* bv = reinterpret_cast<VecT*>(buf);
    // element of register r in window p: (r % V) | thread bits at VB .. lo - 1 | (r / V) << lo | thread bits >= lo + WB
    auto ebase = [&](int lo) { return ((t & ((1 << (lo - VB)) - 1)) << VB) | ((t >> (lo - VB)) << (lo + WB)); };
#pragma unroll
    for (int p = 0; p < W::P; ++p) {
        const int lo = W::lo(p);
        const int g0 = ebase(lo) >> VB, ph0 = g0 + (g0 >> WB);       // padded group of register group 0
        // padded step between register groups (window 0: consecutive groups within one padding period)
        const int gstep = p == 0 ? 1 : (1 << (lo - VB)) + (1 << (lo - VB - WB));
        if (p > 0) {
#pragma unroll
            for (int q = 0; q < G; ++q) {
                const VecT a = bv[ph0 + q * gstep];
                if constexpr (V == 2) {
                    v[2 * q] = a.x; v[2 * q + 1] = a.y;
                } else {
                    v[4 * q] = a.x; v[4 * q + 1] = a.y; v[4 * q + 2] = a.z; v[4 * q + 3] = a.w;
                }
            }
        }
#pragma unroll
        for (int sb = 0; sb < 5; ++sb) {
            const int bit = sb < VB ? sb : lo + sb - VB;
            if (bit < W::first(p) || (p > 0 && sb < VB)) continue;
            const int hh = 1 << sb;
#pragma unroll
            for (int k = 0; k < 32; ++k)
                if (!(k & hh)) {
                    const float a = v[k], b = v[k + hh];
                    v[k] = a + b;
                    v[k + hh] = a - b;
                }
        }
        if (p + 1 < W::P) {
            if (p > 0 || REUSE) blk_sync<BAR, (1 << NL) / 32>();       // every thread has read buf before it is overwritten
#pragma unroll
            for (int q = 0; q < G; ++q) {
                if constexpr (V == 2) bv[ph0 + q * gstep] = make_float2(v[2 * q], v[2 * q + 1]);
                else bv[ph0 + q * gstep] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
            }
            blk_sync<BAR, (1 << NL) / 32>();
        }
    }
}

// Element of register V q + k of thread t after win_walsh (the last window's layout).
template <int NL>
__device__ __forceinline__ int win_elem(int t, int q, int k) {
    constexpr int V = rot_vec<NL>();
    using W = Win2<NL, V>;
    constexpr int VB = W::VB, WB = W::WB, LO = W::lo(W::P - 1);
    return (((t & ((1 << (LO - VB)) - 1)) << VB) | ((t >> (LO - VB)) << (LO + WB))) + (q << LO) + k;
}

// Back to window 0 through buf: v in the last window's layout -> the thread's 32 consecutive elements (buf as in
// win_walsh; waits for the block before writing and after).
template <int NL, int BAR = 0>
__device__ __forceinline__ void win_relayout(float (&v)[32], float* buf, int t) {
    constexpr int V = rot_vec<NL>();
    constexpr int WB = Win2<NL, V>::WB, G = 1 << WB;
    using VecT = typename std::conditional<V == 2, float2, float4>::type;
    VecT* bv = reinterpret_cast<VecT*>(buf);
    auto ph = [](int g) { return g + (g >> WB); };
    blk_sync<BAR, (1 << NL) / 32>();
#pragma unroll
    for (int q = 0; q < G; ++q) {
        const int g = win_elem<NL>(t, q, 0) / V;
        if constexpr (V == 2) bv[ph(g)] = make_float2(v[2 * q], v[2 * q + 1]);
        else bv[ph(g)] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    }
    blk_sync<BAR, (1 << NL) / 32>();
    const int p0 = ph(t << WB);                                      // window 0: 2^WB consecutive groups, one period
#pragma unroll
    for (int q = 0; q < G; ++q) {
        const VecT a = bv[p0 + q];
        if constexpr (V == 2) {
            v[2 * q] = a.x; v[2 * q + 1] = a.y;
        } else {
            v[4 * q] = a.x; v[4 * q + 1] = a.y; v[4 * q + 2] = a.z; v[4 * q + 3] = a.w;
        }
    }
}


}  // namespace tcq
