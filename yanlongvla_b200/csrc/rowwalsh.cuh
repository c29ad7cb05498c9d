// Row transform helpers shared by the rotation kernels (rotate.cu) and the decode-GEMV with its pre fused
// (trellis.cu): the block Walsh of one token row, the per-token INT8 quantizer and the input loaders.
//
// A row of width K (multiple of 16, <= 16384) is the concatenation of descending power-of-two blocks
// (tcq_format.py:26-30); each block gets the FP32 Walsh transform with stages h = 1, 2, 4, ... and the scale
// (float)(1 / sqrt(w)) (tcq_format.py:44-55); every kernel that includes this header computes it the same way, so
// their results agree bit for bit.
#pragma once
#include "tcq_common.cuh"

namespace tcq {

// ---------------------------------------------------------------------------------------------------- row transform
template <int R, class Fin>
__device__ __forceinline__ void walsh_pass(float* buf, int off, int w, int S, bool last, Fin& fin) {
    const int G = w >> R;
    const float c = wscale(w);
    for (int g = threadIdx.x; g < G; g += blockDim.x) {
        const int low = g & (S - 1);
        const int base = off + (((g - low) << R) | low);
        float v[1 << R];
#pragma unroll
        for (int k = 0; k < (1 << R); ++k) v[k] = buf[swz(base + k * S)];
        bfly<R>(v);
        if (last) {
#pragma unroll
            for (int k = 0; k < (1 << R); ++k) fin(base + k * S, v[k] * c);
        } else {
#pragma unroll
            for (int k = 0; k < (1 << R); ++k) buf[swz(base + k * S)] = v[k];
        }
    }
}

// ld16(c, v): the 16 inputs of chunk c (indices 16c .. 16c+15). fin(i, value): called exactly once per index with the
// finished, scaled value (by the thread that owns index i in that pass; it may write buf[swz(i)]). fin16(i0, v): the
// same for the 16 finished values of a whole chunk i0 .. i0+15 at once (blocks of up to 512, finished in registers),
// so that callers can load their per-index operands and store their results 16 bytes at a time.
// Ends with a __syncthreads() so that values fin / fin16 stored to buf are visible to the whole block.
//
// Stages h = 1..8 run in registers on a thread's 16 contiguous inputs; h = 16..256 across the 32 lanes of a warp,
// which hold 32 consecutive chunks (lane partner = lane ^ h/16: the lower lane keeps a + b, the upper b' = a - b, the
// reference's operands in its order; both as one rounding of (+-1) * own + partner); blocks of up to 512 are then
// done. Wider blocks finish with radix-16 passes through shared memory at stride 512 (and 8192). Threads per row are
// a multiple of 32, so a warp's chunks are consecutive; blocks are aligned to their width, so a stage never pairs
// chunks of different blocks. The cross-lane stages are a rolled loop: row kernels run once per launch and are bound
// by instruction fetch, not by the loop overhead.
template <class Ld16, class Fin16, class Fin>
__device__ __forceinline__ void row_walsh16(float* buf, int K, Ld16 ld16, Fin16 fin16, Fin fin) {
    const int nch = K >> 4, lane = threadIdx.x & 31;
    for (int c0 = threadIdx.x - lane; c0 < nch; c0 += blockDim.x) {        // warp-uniform
        const int c = c0 + lane;
        float v[16];
        int w = 0;                                                             // width of this chunk's block
        if (c < nch) {
            ld16(c, v);
            bfly<4>(v);
            w = block_of(c << 4, K);
        } else {
#pragma unroll
            for (int k = 0; k < 16; ++k) v[k] = 0.f;
        }
#pragma unroll 1
        for (int hc = 1; hc < 32; hc <<= 1) {                                 // stage h = 16 hc
            if (!__any_sync(0xffffffffu, w > 16 * hc)) break;
            const bool act = w > 16 * hc;
            const float sg = (lane & hc) ? -1.f : 1.f;                         // upper lane: partner - own
#pragma unroll
            for (int k = 0; k < 16; ++k) {
                const float p = __shfl_xor_sync(0xffffffffu, v[k], hc);
                if (act) v[k] = __fmaf_rn(sg, v[k], p);
            }
        }
        if (c < nch) {
            const int i0 = c << 4;
            if (w <= 512) {
                const float sc = wscale(w);
#pragma unroll
                for (int k = 0; k < 16; ++k) v[k] = v[k] * sc;
                fin16(i0, v);
            } else {
                float4* b4 = reinterpret_cast<float4*>(buf);
#pragma unroll
                for (int q = 0; q < 4; ++q) b4[swz(i0 + 4 * q) >> 2] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
            }
        }
    }
    __syncthreads();
    for (int S = 512;; S <<= 4) {
        bool work = false;
        int off = 0;
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

template <class Ld16, class Fin>
__device__ __forceinline__ void row_walsh(float* buf, int K, Ld16 ld16, Fin fin) {
    row_walsh16(buf, K, ld16, [&](int i0, const float* v) {
#pragma unroll
        for (int k = 0; k < 16; ++k) fin(i0 + k, v[k]);
    }, fin);
}

// fin16 of a pass whose result is the finished row in buf (at swz(i)) plus its absolute maximum: four 16-byte stores.
__device__ __forceinline__ void store_chunk(float* buf, int i0, const float* v, float& mx) {
    float4* b4 = reinterpret_cast<float4*>(buf);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
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
__device__ __forceinline__ int q8(float v, float s) {
    float r = rintf(v / s);
    r = fminf(fmaxf(r, -127.f), 127.f);
    return (int)r;
}

__device__ __forceinline__ void quantize_store(const float* buf, float mx, float* red, int8_t* q, int* q4, float* scale,
                                               int tok, int K, int ldq) {
    mx = block_max(mx, red);
    const float s = mx > 0.f ? mx / 127.f : 1.f;
    if (threadIdx.x == 0) scale[tok] = s;
    // Four values (one q4 word) per step, in a rolled loop: the division's code is fetched once, not sixteen times.
    const float4* b4 = reinterpret_cast<const float4*>(buf);
    for (int c = threadIdx.x; c < (K >> 4); c += blockDim.x) {
#pragma unroll 1
        for (int g = 0; g < 4; ++g) {
            const float4 v = b4[swz(16 * c + 4 * g) >> 2];
            const u32 w = (u32)(q8(v.x, s) & 0xff) | ((u32)(q8(v.y, s) & 0xff) << 8) | ((u32)(q8(v.z, s) & 0xff) << 16) |
                          ((u32)(q8(v.w, s) & 0xff) << 24);
            if (q) reinterpret_cast<u32*>(q + (size_t)tok * K + 16 * c)[g] = w;
            if (q4) q4[(size_t)(4 * c + g) * ldq + tok] = (int)w;
        }
    }
}

// ---------------------------------------------------------------------------------------------------- chunk I/O
// The same for a destination of unknown alignment (a caller's output view): 16-byte stores when p allows them.
__device__ __forceinline__ void store16_bf16_any(u16* p, const u32* w) {
    if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) {
        store16_bf16(p, w);
    } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            p[2 * k] = (u16)(w[k] & 0xffffu);
            p[2 * k + 1] = (u16)(w[k] >> 16);
        }
    }
}

// 16 finished FP32 values of chunk i0 into the row buffer at swz(i0 + k): four 16-byte stores.
__device__ __forceinline__ void store16_f32_swz(float* buf, int i0, const float* v) {
    float4* b4 = reinterpret_cast<float4*>(buf);
#pragma unroll
    for (int q = 0; q < 4; ++q) b4[swz(i0 + 4 * q) >> 2] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
}

// 16 BF16 values from p (16-byte aligned, global or shared; generic loads).
__device__ __forceinline__ void load_bf16x16_any(const u16* p, float* v) {
    const uint4* u = reinterpret_cast<const uint4*>(p);
    const uint4 a = u[0], b = u[1];
    const u32 w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        v[2 * k] = __uint_as_float(w[k] << 16);
        v[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
    }
}

// ---------------------------------------------------------------------------------------------------- loaders
// 16 inputs of a row (BF16 / F16 / F32), 16-byte aligned.
template <int DT>
__device__ __forceinline__ void load16(const void* p, float* v) {
    if (DT == TCQ_DT_F32) {
        const float4* f = reinterpret_cast<const float4*>(p);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float4 a = __ldg(f + q);
            v[4 * q] = a.x; v[4 * q + 1] = a.y; v[4 * q + 2] = a.z; v[4 * q + 3] = a.w;
        }
    } else {
        const uint4* u = reinterpret_cast<const uint4*>(p);
        const uint4 a = __ldg(u), b = __ldg(u + 1);
        const u32 w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int k = 0; k < 8; ++k) {
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

__device__ __forceinline__ void load_signs16(const i8* p, float* sg) {
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(p));
    const u32 w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int k = 0; k < 16; ++k) sg[k] = (float)(i8)((w[k >> 2] >> (8 * (k & 3))) & 0xff);
}

// The same for a vector that may be a shared-memory copy (stage_const): plain, generic loads.
__device__ __forceinline__ void load_signs16_any(const i8* p, float* sg) {
    const uint4 a = *reinterpret_cast<const uint4*>(p);
    const u32 w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int k = 0; k < 16; ++k) sg[k] = (float)(i8)((w[k >> 2] >> (8 * (k & 3))) & 0xff);
}

__device__ __forceinline__ void load_f16x(const float* p, float* v) {
    const float4* f = reinterpret_cast<const float4*>(p);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const float4 a = __ldg(f + q);
        v[4 * q] = a.x; v[4 * q + 1] = a.y; v[4 * q + 2] = a.z; v[4 * q + 3] = a.w;
    }
}

__device__ __forceinline__ void load_f16x_any(const float* p, float* v) {
    const float4* f = reinterpret_cast<const float4*>(p);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const float4 a = f[q];
        v[4 * q] = a.x; v[4 * q + 1] = a.y; v[4 * q + 2] = a.z; v[4 * q + 3] = a.w;
    }
}

// Scaled accumulator inputs z = SCALE(acc): I32 ((float)a * s) * rs, F32 a, BF16 bf2f(a) * rs (kernels.py:545).
// rs may be a shared-memory copy (stage_const).
template <int AT>
__device__ __forceinline__ void load_scaled16(const void* acc, size_t idx, float s, const float* rs, float* v) {
    if (AT == TCQ_DT_I32) {
        const int4* a4 = reinterpret_cast<const int4*>(reinterpret_cast<const int*>(acc) + idx);
        float r[16];
        load_f16x_any(rs, r);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int4 a = __ldg(a4 + q);
            v[4 * q] = ((float)a.x * s) * r[4 * q];
            v[4 * q + 1] = ((float)a.y * s) * r[4 * q + 1];
            v[4 * q + 2] = ((float)a.z * s) * r[4 * q + 2];
            v[4 * q + 3] = ((float)a.w * s) * r[4 * q + 3];
        }
    } else if (AT == TCQ_DT_F32) {
        load_f16x(reinterpret_cast<const float*>(acc) + idx, v);
    } else {
        float r[16];
        load_f16x_any(rs, r);
        load16<TCQ_DT_BF16>(reinterpret_cast<const u16*>(acc) + idx, v);
#pragma unroll
        for (int k = 0; k < 16; ++k) v[k] = v[k] * r[k];
    }
}

}  // namespace tcq
