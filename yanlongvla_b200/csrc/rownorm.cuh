// Row norm core shared by tcq_add_norm (norm.cu) and the fused post -> add -> norm -> pre chain (rotate.cu).
//
// A thread block owns one row of width D (a multiple of 16); thread t holds the 16-element chunks c = t + k * blockDim
// (k < kNormMaxChunks) in registers. Row sums run in a fixed order: each thread's elements in index order, a
// butterfly over the warp (every lane ends with the same sum: floating-point addition is commutative), then the
// warps' sums in warp order. Both kernels launch norm_threads(D) threads per row, so they reduce identically and
// their outputs agree bit for bit.
#pragma once
#include "tcq_common.cuh"

namespace tcq {

constexpr int kNormMaxChunks = 4;      // rows up to 16 * 4 * 512 = 32768 wide
constexpr int kStageMaxBytes = 64 * 1024;   // layer constants staged in shared memory per block (stage_const), at most
constexpr int kStageMaxSmem = 200 * 1024;   // and the block's whole dynamic shared memory with them

__host__ __device__ inline int norm_threads(int D) {
    int t = ((D >> 4) + 31) & ~31;
    if (t < 32) t = 32;
    if (t > 512) t = 512;
    return t;
}

__device__ __forceinline__ float bf16_round(float f) { return bf2f(f2bf(f)); }

// h = BF16(x + y) on a chunk, in place in x (FP32 add, one rounding); the packed BF16 words go to hout when given.
__device__ __forceinline__ void add_round_chunk(float* x, const float* y, u16* hout) {
    float t[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) t[i] = x[i] + y[i];
    u32 w[8];
    pack_bf16x16(t, w);
    unpack_bf16w(w, x);
    if (hout) store16_bf16(hout, w);
}

// Sum over the block in a fixed order; every thread receives the same value. `red` holds one float per warp.
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();                               // red may still be read by a previous reduction
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.f;
    const int warps = (blockDim.x + 31) >> 5;
    for (int i = 0; i < warps; ++i) t += red[i];
    return t;
}

__device__ __forceinline__ void unpack_bf16x16(const uint4& a, const uint4& b, float* v) {
    const u32 w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        v[2 * i] = bf2f((u16)(w[i] & 0xffffu));
        v[2 * i + 1] = bf2f((u16)(w[i] >> 16));
    }
}

__device__ __forceinline__ void load_bf16x16(const u16* p, float* v) {
    const uint4* u = reinterpret_cast<const uint4*>(p);
    unpack_bf16x16(__ldg(u), __ldg(u + 1), v);
}

__device__ __forceinline__ void store_bf16x16(u16* p, const float* v) {
    u32 w[8];
    pack_bf16x16(v, w);
    store16_bf16(p, w);
}

// Element j of an FP32 or BF16 parameter vector, in global memory or a shared-memory copy (stage_const).
template <bool WBF16>
__device__ __forceinline__ float ldp(const void* p, int j) {
    if (WBF16) return bf2f(reinterpret_cast<const u16*>(p)[j]);
    return reinterpret_cast<const float*>(p)[j];
}

// Elements j0 .. j0+15 of an FP32 or BF16 parameter vector (global or a shared-memory copy): 16-byte loads when the
// address allows them.
template <bool WBF16>
__device__ __forceinline__ void ldp16(const void* p, int j0, float* v) {
    const char* a = reinterpret_cast<const char*>(p) + (size_t)j0 * (WBF16 ? 2 : 4);
    if ((reinterpret_cast<uintptr_t>(a) & 15) == 0) {
        const uint4* u = reinterpret_cast<const uint4*>(a);
        if (WBF16) {
            const uint4 x = u[0], y = u[1];
            const u32 w[8] = {x.x, x.y, x.z, x.w, y.x, y.y, y.z, y.w};
            unpack_bf16w(w, v);
        } else {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint4 x = u[q];
                v[4 * q] = __uint_as_float(x.x); v[4 * q + 1] = __uint_as_float(x.y);
                v[4 * q + 2] = __uint_as_float(x.z); v[4 * q + 3] = __uint_as_float(x.w);
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = ldp<WBF16>(p, j0 + i);
    }
}

// Modulation values of a thread's first chunk, loaded early (with the row's other inputs) into registers: BF16
// pairs, element i of the chunk in the low (even i) or high (odd i) half of word i / 2.
struct ModChunk {
    u32 s[8], h[8];
    bool on;
};

__device__ __forceinline__ void load_mod_chunk(ModChunk& m, const u16* ms, const u16* mh) {
    const uint4* a = reinterpret_cast<const uint4*>(ms);
    const uint4* b = reinterpret_cast<const uint4*>(mh);
    const uint4 a0 = __ldg(a), a1 = __ldg(a + 1), b0 = __ldg(b), b1 = __ldg(b + 1);
    m.s[0] = a0.x; m.s[1] = a0.y; m.s[2] = a0.z; m.s[3] = a0.w; m.s[4] = a1.x; m.s[5] = a1.y; m.s[6] = a1.z; m.s[7] = a1.w;
    m.h[0] = b0.x; m.h[1] = b0.y; m.h[2] = b0.z; m.h[3] = b0.w; m.h[4] = b1.x; m.h[5] = b1.y; m.h[6] = b1.z; m.h[7] = b1.w;
    m.on = true;
}

// The same from shared memory (a copy made with cp_async16), 16-byte aligned.
__device__ __forceinline__ void load_mod_chunk_smem(ModChunk& m, const u16* ms, const u16* mh) {
    const uint4* a = reinterpret_cast<const uint4*>(ms);
    const uint4* b = reinterpret_cast<const uint4*>(mh);
    const uint4 a0 = a[0], a1 = a[1], b0 = b[0], b1 = b[1];
    m.s[0] = a0.x; m.s[1] = a0.y; m.s[2] = a0.z; m.s[3] = a0.w; m.s[4] = a1.x; m.s[5] = a1.y; m.s[6] = a1.z; m.s[7] = a1.w;
    m.h[0] = b0.x; m.h[1] = b0.y; m.h[2] = b0.z; m.h[3] = b0.w; m.h[4] = b1.x; m.h[5] = b1.y; m.h[6] = b1.z; m.h[7] = b1.w;
    m.on = true;
}

__device__ __forceinline__ float bf_half(u32 w, int i) { return __uint_as_float((i & 1) ? (w & 0xffff0000u) : (w << 16)); }

// The norm of the row held in v (the residual sum h, already rounded to BF16), in place, unrounded:
// KIND 0 (RMSNorm):   n = (h * r) * w,                r = rsqrt(sum(h^2) / D + eps)
// KIND 1 (LayerNorm): n = ((h - mu) * r) * w + b,     mu = sum(h) / D, r = rsqrt(sum((h - mu)^2) / D + eps)
// w / b optional (NULL = 1 / 0), FP32 or (WBF16) BF16, in global memory or a shared-memory copy; ms / mh (BF16,
// NULL = none): n = n * (1 + ms) + mh, the thread's first chunk from m0 when m0.on.
// Every thread of the block must call it (it synchronizes).
// NC: chunks per thread the caller holds (1 when D <= 16 * blockDim, else kNormMaxChunks).
template <int KIND, bool WBF16, int NC>
__device__ __forceinline__ void norm_chunks(float (&v)[NC][16], int D, const void* w, const void* b,
                                            const u16* ms, const u16* mh, float eps, float* red, const ModChunk& m0) {
    const int nch = D >> 4;
    float part = 0.f;
#pragma unroll
    for (int k = 0; k < NC; ++k) {
        const int c = threadIdx.x + k * blockDim.x;
        if (c < nch) {
#pragma unroll
            for (int i = 0; i < 16; ++i) part += KIND == 0 ? v[k][i] * v[k][i] : v[k][i];
        }
    }
    const float tot = block_sum(part, red);
    float mu = 0.f, r;
    if (KIND == 0) {
        r = rsqrtf(tot / (float)D + eps);
    } else {
        mu = tot / (float)D;
        float p2 = 0.f;
#pragma unroll
        for (int k = 0; k < NC; ++k) {
            const int c = threadIdx.x + k * blockDim.x;
            if (c < nch) {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float d = v[k][i] - mu;
                    p2 += d * d;
                }
            }
        }
        r = rsqrtf(block_sum(p2, red) / (float)D + eps);
    }
#pragma unroll
    for (int k = 0; k < NC; ++k) {
        const int c = threadIdx.x + k * blockDim.x;
        if (c < nch) {
            float wv[16], bv[16];
            if (w) ldp16<WBF16>(w, 16 * c, wv);
            if (b) ldp16<WBF16>(b, 16 * c, bv);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int j = 16 * c + i;
                float t = KIND == 0 ? v[k][i] * r : (v[k][i] - mu) * r;
                if (w) t = t * wv[i];
                if (b) t = t + bv[i];
                if (ms) {
                    const float a = k == 0 && m0.on ? bf_half(m0.s[i >> 1], i) : bf2f(__ldg(ms + j));
                    const float c = k == 0 && m0.on ? bf_half(m0.h[i >> 1], i) : bf2f(__ldg(mh + j));
                    t = t * (1.f + a) + c;
                }
                v[k][i] = t;
            }
        }
    }
}

}  // namespace tcq
