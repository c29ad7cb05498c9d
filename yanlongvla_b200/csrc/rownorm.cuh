// Row norm core shared by tcq_add_norm (norm.cu) and the fused post -> add -> norm -> pre chain (rotate.cu).
//
// A thread block owns one row of width D (a multiple of 16); thread t holds the CH-element chunks c = t + k * blockDim
// (k < NC) in registers: CH = 16 (NC = 1 up to 8192 wide, kNormMaxChunks above), or CH = 4 for rows up to 2048 wide
// in launches of few rows (four times the threads per row: such launches are bound by each thread's instruction
// latency). Row sums run in one fixed order whatever the chunking: the canonical order of 16-element chunks, one per
// thread of norm_threads(D) threads -- each chunk's elements summed in index order from 0 (CH = 4 continues the
// running sum across the four lanes of a chunk), then a butterfly over the 32 chunks of a warp (every lane ends with
// the same sum: floating-point addition is commutative), then the warps' sums in warp order. tcq_add_norm and the
// chain therefore agree bit for bit, and a row's norm does not depend on how many rows the launch has.
#pragma once
#include "rowwalsh.cuh"

namespace tcq {

constexpr int kNormMaxChunks = 4;           // rows up to 16 * 4 * 512 = 32768 wide
constexpr int kStageMaxBytes = 64 * 1024;   // layer constants staged in shared memory per block (stage_const), at most
constexpr int kStageMaxSmem = 200 * 1024;   // and the block's whole dynamic shared memory with them

// Threads of a row with chunks of CH elements (CH = 4 only for D <= 2048).
__host__ __device__ inline int norm_threads(int D, int CH = 16) {
    int t = ((D / CH) + 31) & ~31;
    if (t < 32) t = 32;
    if (t > 512) t = 512;
    return t;
}

// Chunks of 16 per thread: one up to 8192 wide, kNormMaxChunks above.
__host__ __device__ inline int norm_nc(int D) { return D <= 8192 ? 1 : kNormMaxChunks; }

// h = BF16(x + y) on a chunk, in place in x (FP32 add, one rounding); the packed BF16 words go to hout when given
// (aligned to 2 CH bytes).
template <int CH>
__device__ __forceinline__ void add_round_chunk(float* x, const float* y, u16* hout) {
    float t[CH];
#pragma unroll
    for (int i = 0; i < CH; ++i) t[i] = x[i] + y[i];
    u32 w[CH / 2];
    pack_bf16c<CH>(t, w);
#pragma unroll
    for (int k = 0; k < CH / 2; ++k) {
        x[2 * k] = __uint_as_float(w[k] << 16);
        x[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
    }
    if (hout) store_bf16c<CH>(hout, w);
}

// The canonical row sum for CH = 4 (rows up to 2048 wide; blockDim = norm_threads(D, 4)): `part` is this thread's
// 4-element partial term list, summed here in the canonical order. The running sum of a 16-element chunk passes from
// lane to lane (4 j, 4 j + 1, 4 j + 2, 4 j + 3); the chunk sums then go through shared memory to the warps of the
// CH = 16 layout (norm_threads(D) threads), whose butterflies and warp-ordered total are block_sum's.
template <int KIND>
__device__ __forceinline__ float chunk4_sum(const float (&t)[4], int D, float* red) {
    __shared__ float gs[128];                      // one sum per 16-element chunk (D <= 2048)
    const int lane = threadIdx.x & 31, nch16 = D >> 4, c16 = threadIdx.x >> 2;
    float acc = 0.f;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const float in = __shfl_up_sync(0xffffffffu, acc, 1);
        if ((lane & 3) == r) {
            float a = r == 0 ? 0.f : in;
#pragma unroll
            for (int i = 0; i < 4; ++i) a += t[i];
            acc = a;
        }
    }
    const int t16 = norm_threads(D);
    __syncthreads();                               // gs / red may still be read by a previous reduction
    if ((lane & 3) == 3 && c16 < nch16) gs[c16] = acc;
    for (int i = nch16 + threadIdx.x; i < t16; i += blockDim.x) gs[i] = 0.f;   // the padding chunks of the last warp
    __syncthreads();
    if ((int)threadIdx.x < t16) {
        float v = gs[threadIdx.x];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) red[threadIdx.x >> 5] = v;
    }
    __syncthreads();
    float tot = 0.f;
    for (int i = 0; i < (t16 >> 5); ++i) tot += red[i];
    return tot;
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

// Element j of an FP32 or BF16 parameter vector, in global memory or a shared-memory copy (stage_const).
template <bool WBF16>
__device__ __forceinline__ float ldp(const void* p, int j) {
    if (WBF16) return bf2f(reinterpret_cast<const u16*>(p)[j]);
    return reinterpret_cast<const float*>(p)[j];
}

// Elements j0 .. j0 + CH - 1 of a parameter vector (global or a shared-memory copy): vector loads when the address
// allows them.
template <bool WBF16, int CH>
__device__ __forceinline__ void ldpc(const void* p, int j0, float* v) {
    constexpr int NB = CH * (WBF16 ? 2 : 4);
    const char* a = reinterpret_cast<const char*>(p) + (size_t)j0 * (WBF16 ? 2 : 4);
    if ((reinterpret_cast<uintptr_t>(a) & ((NB < 16 ? NB : 16) - 1)) == 0) {
        if (WBF16) {
            load_bf16c_any<CH>(reinterpret_cast<const u16*>(a), v);
        } else {
            load_f32c<CH, false>(reinterpret_cast<const float*>(a), v);
        }
    } else {
#pragma unroll
        for (int i = 0; i < CH; ++i) v[i] = ldp<WBF16>(p, j0 + i);
    }
}

// Modulation values of a thread's first chunk, loaded early (with the row's other inputs) into registers: BF16
// pairs, element i of the chunk in the low (even i) or high (odd i) half of word i / 2.
template <int CH>
struct ModChunk {
    u32 s[CH / 2], h[CH / 2];
    bool on;
};

// G: ms / mh are global (__ldg); otherwise shared-memory copies. Aligned to 2 CH bytes.
template <int CH, bool G>
__device__ __forceinline__ void load_mod_chunk(ModChunk<CH>& m, const u16* ms, const u16* mh) {
    ldw<2 * CH, G>(ms, m.s);
    ldw<2 * CH, G>(mh, m.h);
    m.on = true;
}

__device__ __forceinline__ float bf_half(u32 w, int i) { return __uint_as_float((i & 1) ? (w & 0xffff0000u) : (w << 16)); }

// The norm of the row held in v (the residual sum h, already rounded to BF16), in place, unrounded:
// KIND 0 (RMSNorm):   n = (h * r) * w,                r = rsqrt(sum(h^2) / D + eps)
// KIND 1 (LayerNorm): n = ((h - mu) * r) * w + b,     mu = sum(h) / D, r = rsqrt(sum((h - mu)^2) / D + eps)
// w / b optional (NULL = 1 / 0), FP32 or (WBF16) BF16, in global memory or a shared-memory copy; ms / mh (BF16,
// NULL = none): n = n * (1 + ms) + mh, the thread's first chunk from m0 when m0.on.
// Every thread of the block must call it (it synchronizes). CH = 16 with NC = norm_nc(D), or CH = 4 with NC = 1.
template <int KIND, bool WBF16, int NC, int CH>
__device__ __forceinline__ void norm_chunks(float (&v)[NC][CH], int D, const void* w, const void* b,
                                            const u16* ms, const u16* mh, float eps, float* red, const ModChunk<CH>& m0) {
    static_assert(CH == 16 || NC == 1, "chunks of 4: one per thread");
    const int nch = D / CH;
    float tot;
    if (CH == 4) {
        float t[4] = {0.f, 0.f, 0.f, 0.f};
        if ((int)threadIdx.x < nch) {
#pragma unroll
            for (int i = 0; i < 4; ++i) t[i] = KIND == 0 ? v[0][i] * v[0][i] : v[0][i];
        }
        tot = chunk4_sum<KIND>(t, D, red);
    } else {
        float part = 0.f;
#pragma unroll
        for (int k = 0; k < NC; ++k) {
            const int c = threadIdx.x + k * blockDim.x;
            if (c < nch) {
#pragma unroll
                for (int i = 0; i < CH; ++i) part += KIND == 0 ? v[k][i] * v[k][i] : v[k][i];
            }
        }
        tot = block_sum(part, red);
    }
    float mu = 0.f, r;
    if (KIND == 0) {
        r = rsqrtf(tot / (float)D + eps);
    } else {
        mu = tot / (float)D;
        float p2;
        if (CH == 4) {
            float t[4] = {0.f, 0.f, 0.f, 0.f};
            if ((int)threadIdx.x < nch) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float d = v[0][i] - mu;
                    t[i] = d * d;
                }
            }
            p2 = chunk4_sum<KIND>(t, D, red);
        } else {
            p2 = 0.f;
#pragma unroll
            for (int k = 0; k < NC; ++k) {
                const int c = threadIdx.x + k * blockDim.x;
                if (c < nch) {
#pragma unroll
                    for (int i = 0; i < CH; ++i) {
                        const float d = v[k][i] - mu;
                        p2 += d * d;
                    }
                }
            }
            p2 = block_sum(p2, red);
        }
        r = rsqrtf(p2 / (float)D + eps);
    }
#pragma unroll
    for (int k = 0; k < NC; ++k) {
        const int c = threadIdx.x + k * blockDim.x;
        if (c < nch) {
            float wv[CH], bv[CH];
            if (w) ldpc<WBF16, CH>(w, CH * c, wv);
            if (b) ldpc<WBF16, CH>(b, CH * c, bv);
#pragma unroll
            for (int i = 0; i < CH; ++i) {
                const int j = CH * c + i;
                float t = KIND == 0 ? v[k][i] * r : (v[k][i] - mu) * r;
                if (w) t = t * wv[i];
                if (b) t = t + bv[i];
                if (ms) {
                    const float a = k == 0 && m0.on ? bf_half(m0.s[i >> 1], i) : bf2f(__ldg(ms + j));
                    const float cc = k == 0 && m0.on ? bf_half(m0.h[i >> 1], i) : bf2f(__ldg(mh + j));
                    t = t * (1.f + a) + cc;
                }
                v[k][i] = t;
            }
        }
    }
}

}  // namespace tcq
