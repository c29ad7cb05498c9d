// W2 float-activation products (the reference's k_gemmf_w8 / k_gemmf_tcq, kernels.py:430-489, 677-696): BF16
// activations in the rotated space, INT8-table weights, FP32 accumulation, z (M, N) = (sum_k w[n][k] h[m][k]) * rs[n].
//
// hT (K, ldh) BF16 is the transposed rotated activation written by tcq_pre_h (token = column). One warp per output
// row: lanes stride over the row's 16-column tiles (trellis) or 16-byte chunks (INT8), multiply-add in FP32 in index
// order, then a butterfly over the warp; the sum order is fixed, so results are reproducible run to run (they are not
// bit-identical to the float64 definition: this path is held to a tolerance, as in the reference). At most 16 tokens
// per launch; the host entry points loop over token chunks of 16.
#include "trellis_common.cuh"

namespace {

using namespace tcq;

constexpr int kThreads = 512;      // 16 warps: one tile row (16 output rows) per step

// Per-lane replicated table with BF16-valued entries built from the INT8 table: low half BF16(v0) (sign bit flipped
// for keys >= 512, the negated first coordinate), high half BF16(v1). INT8 values are exact in BF16.
__device__ __forceinline__ void fill_table_bf16_from_i8(u32* tab, const u16* pairs) {
    uint4* t4 = reinterpret_cast<uint4*>(tab);
    const int slot = threadIdx.x & 7, kstep = blockDim.x >> 3;
    for (int k = threadIdx.x >> 3; k < 512; k += kstep) {
        const u32 pr = pairs[k];
        const float v0 = (float)(i8)(pr & 0xffu), v1 = (float)(i8)(pr >> 8);
        const u32 ep = (u32)f2bf(v0) | ((u32)f2bf(v1) << 16), en = ep ^ 0x8000u;
        t4[k * 8 + slot] = make_uint4(ep, ep, ep, ep);
        t4[(k + 512) * 8 + slot] = make_uint4(en, en, en, en);
    }
}

template <int MT>
__device__ __forceinline__ void finish_row(float (&acc)[MT], int lane, int row, int M, int N, const float* rs, float* z) {
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        float v = acc[m];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0 && m < M) z[(size_t)m * N + row] = v * __ldg(rs + row);
    }
}

// Fused trellis decode + W2 product. CTA c takes tile rows [R c / G, R (c + 1) / G); the table is rebuilt when the
// layer slot changes (layer bounds nb0 / nb1 in tile rows, per-layer tables of 1 KB in t8).
template <int MT>
__global__ void __launch_bounds__(kThreads, 1)
k_gemmf_tcq(const u16* __restrict__ bits, const i8* __restrict__ t8, const u16* __restrict__ hT, const float* __restrict__ rs,
            float* __restrict__ z, int M, int N, int K, int ldh, int nb0, int nb1) {
    extern __shared__ __align__(128) u32 tab[];
    __shared__ __align__(16) u16 pairs[512];
    pdl_launch_dependents();
    const int R = N >> 4, tiles = K >> 4, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tr0 = (int)((long long)R * blockIdx.x / gridDim.x), tr1 = (int)((long long)R * (blockIdx.x + 1) / gridDim.x);
    const u32 lane4 = 4u * lane;
    int slot = -1;
    bool waited = false;
    for (int tr = tr0; tr < tr1; ++tr) {
        const int sl = (tr >= nb0) + (tr >= nb1);
        if (sl != slot) {                           // uniform over the block
            __syncthreads();                        // the previous table is no longer read
            if (threadIdx.x < 64)
                reinterpret_cast<uint4*>(pairs)[threadIdx.x] = ldg_table_v4(reinterpret_cast<const uint4*>(t8 + 1024 * sl) + threadIdx.x);
            __syncthreads();
            fill_table_bf16_from_i8(tab, pairs);
            __syncthreads();
            slot = sl;
        }
        if (!waited) {
            pdl_wait();                             // the activations come from the previous kernel
            waited = true;
        }
        const int row = tr * 16 + warp;
        float acc[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[m] = 0.f;
        for (int j = lane; j < tiles; j += 32) {
            const u32* tw = reinterpret_cast<const u32*>(bits + ((size_t)tr * tiles + j) * 32);
            u32 e[8];
            row_entries(rowA(__ldg(tw + warp)), rowA(__ldg(tw + ((warp + 1) & 15))), tab, lane4, e);
            const u16* hk = hT + (size_t)16 * j * ldh;
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                const float wv = __uint_as_float((c & 1) ? (e[c >> 1] & 0xffff0000u) : (e[c >> 1] << 16));
#pragma unroll
                for (int m = 0; m < MT; ++m)
                    if (m < M) acc[m] = __fmaf_rn(wv, bf2f(__ldg(hk + (size_t)c * ldh + m)), acc[m]);
            }
        }
        finish_row<MT>(acc, lane, row, M, N, rs, z);
    }
    if (!waited) pdl_wait();
}

// INT8-resident weights W (N, K): one warp per row, lanes over 16-byte chunks of the row.
template <int MT>
__global__ void __launch_bounds__(kThreads) k_gemmf_w8(const i8* __restrict__ W, const u16* __restrict__ hT,
                                                       const float* __restrict__ rs, float* __restrict__ z, int M, int N, int K,
                                                       int ldh) {
    pdl_launch_dependents();
    pdl_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, row = blockIdx.x * 16 + warp;
    if (row >= N) return;
    float acc[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m] = 0.f;
    const i8* wr = W + (size_t)row * K;
    for (int k0 = 16 * lane; k0 < K; k0 += 512) {
        const uint4 wv4 = __ldg(reinterpret_cast<const uint4*>(wr + k0));
        const u32 w[4] = {wv4.x, wv4.y, wv4.z, wv4.w};
        const u16* hk = hT + (size_t)k0 * ldh;
#pragma unroll
        for (int c = 0; c < 16; ++c) {
            const float wv = (float)(i8)((w[c >> 2] >> (8 * (c & 3))) & 0xffu);
#pragma unroll
            for (int m = 0; m < MT; ++m)
                if (m < M) acc[m] = __fmaf_rn(wv, bf2f(__ldg(hk + (size_t)c * ldh + m)), acc[m]);
        }
    }
    finish_row<MT>(acc, lane, row, M, N, rs, z);
}

int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    }
    return n;
}

template <class Kern, class... Args>
int launch(Kern kern, int grid, int smem, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...) == cudaSuccess ? TCQ_OK : TCQ_ERR_LAUNCH;
}

template <int MT>
int gemmf_tcq_chunk(const u16* bits, const i8* t8, const u16* hT, const float* rs, float* z, int M, int N, int K, int ldh,
                    int nb0, int nb1, cudaStream_t st) {
    auto kern = k_gemmf_tcq<MT>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kTabBytes) != cudaSuccess) return TCQ_ERR_LAUNCH;
    const int R = N >> 4, grid = R < sm_count() ? R : sm_count();
    return launch(kern, grid, kTabBytes, st, bits, t8, hT, rs, z, M, N, K, ldh, nb0, nb1);
}

template <int MT>
int gemmf_w8_chunk(const i8* W, const u16* hT, const float* rs, float* z, int M, int N, int K, int ldh, cudaStream_t st) {
    return launch(k_gemmf_w8<MT>, (N + 15) / 16, 0, st, W, hT, rs, z, M, N, K, ldh);
}

}  // namespace

extern "C" {

int tcq_gemmf_tcq(const uint16_t* bits, const int8_t* t8, const uint16_t* hT, const float* rs, float* z, int M, int N, int K,
                  int ldh, int nb0, int nb1, void* stream) {
    if (!bits || !t8 || !hT || !rs || !z) return TCQ_ERR_ARG;
    if (M <= 0 || N <= 0 || K <= 0 || (N & 15) || (K & 15) || ldh < M) return TCQ_ERR_SHAPE;
    if (!tcq_aligned(bits, 4) || !tcq_aligned(t8, 16)) return TCQ_ERR_ALIGN;
    cudaStream_t st = (cudaStream_t)stream;
    for (int c0 = 0; c0 < M; c0 += 16) {
        const int m = M - c0 < 16 ? M - c0 : 16;
        const u16* h = reinterpret_cast<const u16*>(hT) + c0;
        float* zc = z + (size_t)c0 * N;
        const u16* b = reinterpret_cast<const u16*>(bits);
        const i8* t = reinterpret_cast<const i8*>(t8);
        int e;
        if (m == 1) e = gemmf_tcq_chunk<1>(b, t, h, rs, zc, m, N, K, ldh, nb0, nb1, st);
        else if (m == 2) e = gemmf_tcq_chunk<2>(b, t, h, rs, zc, m, N, K, ldh, nb0, nb1, st);
        else if (m <= 4) e = gemmf_tcq_chunk<4>(b, t, h, rs, zc, m, N, K, ldh, nb0, nb1, st);
        else if (m <= 8) e = gemmf_tcq_chunk<8>(b, t, h, rs, zc, m, N, K, ldh, nb0, nb1, st);
        else e = gemmf_tcq_chunk<16>(b, t, h, rs, zc, m, N, K, ldh, nb0, nb1, st);
        if (e) return e;
    }
    return TCQ_OK;
}

int tcq_gemmf_w8(const int8_t* W, const uint16_t* hT, const float* rs, float* z, int M, int N, int K, int ldh, void* stream) {
    if (!W || !hT || !rs || !z) return TCQ_ERR_ARG;
    if (M <= 0 || N <= 0 || K <= 0 || (K & 15) || ldh < M) return TCQ_ERR_SHAPE;
    if (!tcq_aligned(W, 16)) return TCQ_ERR_ALIGN;
    cudaStream_t st = (cudaStream_t)stream;
    for (int c0 = 0; c0 < M; c0 += 16) {
        const int m = M - c0 < 16 ? M - c0 : 16;
        const u16* h = reinterpret_cast<const u16*>(hT) + c0;
        float* zc = z + (size_t)c0 * N;
        const i8* w = reinterpret_cast<const i8*>(W);
        int e;
        if (m == 1) e = gemmf_w8_chunk<1>(w, h, rs, zc, m, N, K, ldh, st);
        else if (m == 2) e = gemmf_w8_chunk<2>(w, h, rs, zc, m, N, K, ldh, st);
        else if (m <= 4) e = gemmf_w8_chunk<4>(w, h, rs, zc, m, N, K, ldh, st);
        else if (m <= 8) e = gemmf_w8_chunk<8>(w, h, rs, zc, m, N, K, ldh, st);
        else e = gemmf_w8_chunk<16>(w, h, rs, zc, m, N, K, ldh, st);
        if (e) return e;
    }
    return TCQ_OK;
}

}  // extern "C"
