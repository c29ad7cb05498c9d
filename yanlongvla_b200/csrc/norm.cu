// Row kernels for the policy's glue around the quantized layers: residual add + RMSNorm / LayerNorm (+ the DiT's
// AdaLN modulation) in one pass, and the rotary position embedding.
//
// One thread block per token row. A thread owns chunks c = threadIdx.x + k * blockDim.x of 4 or 16 elements of the
// row and keeps them in registers; row sums are taken in a fixed order (each thread's elements in index order,
// then a butterfly over the warp, then the warps' sums in warp order), so a row's result does not depend on timing.
// The policy runs every runtime (the PyTorch reference runtime included) through these kernels, so the runtimes
// agree bit for bit; tests compare them with a PyTorch FP32 restatement within BF16 rounding.
#include "rownorm.cuh"

namespace {

using namespace tcq;

// h = x (+ y, rounded to BF16 as a BF16 tensor add does); written to hout when given; out = BF16(norm_chunks(h)).
// Modulation vectors: row group g = row / mod_rows (rows of one sample), row stride ld_mod.
// stage: the norm weights are copied into shared memory before the dependency wait (dynamic shared memory holds
// them); the modulation values of the first chunk are loaded with x and y.
template <int KIND, bool WBF16, int NC, int CH>
__global__ void __launch_bounds__(512, 1) k_addnorm(const u16* __restrict__ x, const u16* __restrict__ y, u16* __restrict__ hout,
                                                 u16* __restrict__ nout, const void* __restrict__ w, const void* __restrict__ b,
                                                 const u16* __restrict__ mscale, const u16* __restrict__ mshift, int mod_rows,
                                                 int ld_mod, float eps, int D, int stage) {
    extern __shared__ __align__(16) char cst[];
    __shared__ float red[32];
    pdl_launch_dependents();
    char* sp = cst;
    const void* ws = stage_const(sp, w, (WBF16 ? 2 : 4) * D, stage != 0);
    const void* bs = stage_const(sp, b, (WBF16 ? 2 : 4) * D, stage != 0);
    __syncthreads();
    pdl_wait();
    const int row = blockIdx.x, nch = D / CH;
    const size_t base = (size_t)row * D;
    const u16* ms = mscale ? mscale + (size_t)(row / mod_rows) * ld_mod : nullptr;
    const u16* mh = mscale ? mshift + (size_t)(row / mod_rows) * ld_mod : nullptr;
    ModChunk<CH> m0{};
    if (ms && (((uintptr_t)ms | (uintptr_t)mh) & 15) == 0 && (int)threadIdx.x < nch)
        load_mod_chunk<CH, true>(m0, ms + CH * threadIdx.x, mh + CH * threadIdx.x);
    float v[NC][CH];
#pragma unroll
    for (int k = 0; k < NC; ++k) {
        const int c = threadIdx.x + k * blockDim.x;
        if (c < nch) {
            loadc<TCQ_DT_BF16, CH>(x + base + CH * c, v[k]);
            if (y) {
                float t[CH];
                loadc<TCQ_DT_BF16, CH>(y + base + CH * c, t);
                add_round_chunk<CH>(v[k], t, hout ? hout + base + CH * c : nullptr);
            }
        }
    }
    norm_chunks<KIND, WBF16, NC, CH>(v, D, ws, bs, ms, mh, eps, red, m0);
#pragma unroll
    for (int k = 0; k < NC; ++k) {
        const int c = threadIdx.x + k * blockDim.x;
        if (c < nch) {
            u32 wn[CH / 2];
            pack_bf16c<CH>(v[k], wn);
            store_bf16c<CH>(nout + base + CH * c, wn);
        }
    }
}

// Rotary embedding, half-split form, on rows of `heads` heads of width D (row r is position r % T):
// out[a] = BF16(a * cos - b * sin), out[b] = BF16(a * sin + b * cos) for the pair (a, b) = (x[j], x[j + D/2]) of each
// head, FP32 arithmetic in that order. cos / sin: (T, D / 2) FP32.
__global__ void __launch_bounds__(256) k_rope(const u16* __restrict__ x, u16* __restrict__ out, const float* __restrict__ cs,
                                              const float* __restrict__ sn, int T, int heads, int D, int ldx, int ldo) {
    pdl_launch_dependents();
    pdl_wait();
    const int row = blockIdx.x, half = D >> 1, t = row % T;
    const u16* xr = x + (size_t)row * ldx;
    u16* orow = out + (size_t)row * ldo;
    for (int i = threadIdx.x; i < heads * half; i += blockDim.x) {
        const int h = i / half, j = i - h * half;
        const float a = bf2f(xr[h * D + j]), bb = bf2f(xr[h * D + half + j]);
        const float c = __ldg(cs + (size_t)t * half + j), s = __ldg(sn + (size_t)t * half + j);
        const float p = a * c, q = bb * s, u = a * s, v = bb * c;
        orow[h * D + j] = f2bf(p - q);
        orow[h * D + half + j] = f2bf(u + v);
    }
}

template <class Kern, class... Args>
int launch_rows(Kern kern, int rows, int threads, int smem, void* stream, Args... args) {
    if (smem > 46 * 1024 && cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
        return TCQ_ERR_LAUNCH;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(rows);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...) == cudaSuccess ? TCQ_OK : TCQ_ERR_LAUNCH;
}

}  // namespace

extern "C" {

int tcq_add_norm(const uint16_t* x, const uint16_t* y, uint16_t* h, uint16_t* out, const void* w, const void* b, int wb_dtype,
                 const uint16_t* mod_scale, const uint16_t* mod_shift, int mod_rows, int ld_mod, float eps, int kind, int M,
                 int D, void* stream) {
    if (!x || !out || (h && !y) || (!mod_scale != !mod_shift)) return TCQ_ERR_ARG;
    if (kind != 0 && kind != 1) return TCQ_ERR_ARG;
    if (wb_dtype != TCQ_DT_F32 && wb_dtype != TCQ_DT_BF16) return TCQ_ERR_DTYPE;
    if (M <= 0 || D <= 0 || (D & 15) || D > 16 * kNormMaxChunks * 512) return TCQ_ERR_SHAPE;
    if (mod_scale && (mod_rows <= 0 || ld_mod < D)) return TCQ_ERR_ARG;
    if (!tcq_aligned(x, 16) || !tcq_aligned(out, 16) || (y && !tcq_aligned(y, 16)) || (h && !tcq_aligned(h, 16)))
        return TCQ_ERR_ALIGN;
    // Chunks of 4 for a few rows up to 2048 wide (the sum order does not depend on the chunking), else 16: one chunk
    // per thread up to 8192 wide.
    const bool c4 = D <= 2048 && (long long)M * norm_threads(D, 4) <= (long long)tcq_sm_count() * 512;
    const int T = norm_threads(D, c4 ? 4 : 16);
    const bool wb = wb_dtype == TCQ_DT_BF16;
    auto pick = [&](auto k0, auto k1, auto k2) { return c4 ? k0 : D <= 8192 ? k1 : k2; };
#define TCQ_ADDNORM(KD, WB) pick(k_addnorm<KD, WB, 1, 4>, k_addnorm<KD, WB, 1, 16>, k_addnorm<KD, WB, kNormMaxChunks, 16>)
    auto kern = kind == 0 ? (wb ? TCQ_ADDNORM(0, true) : TCQ_ADDNORM(0, false)) : (wb ? TCQ_ADDNORM(1, true) : TCQ_ADDNORM(1, false));
#undef TCQ_ADDNORM
    const int cbytes = ((w ? 1 : 0) + (b ? 1 : 0)) * (wb ? 2 : 4) * D;
    const int stage = cbytes > 0 && tcq_stage_rows(M, cbytes, kStageMaxBytes);
    return launch_rows(kern, M, T, stage ? cbytes : 0, stream, (const u16*)x, (const u16*)y, (u16*)h, (u16*)out, w, b,
                       (const u16*)mod_scale, (const u16*)mod_shift, mod_rows, ld_mod, eps, D, stage);
}

int tcq_rope(const uint16_t* x, uint16_t* out, const float* cos_t, const float* sin_t, int rows, int T, int heads, int D,
             int ldx, int ldo, void* stream) {
    if (!x || !out || !cos_t || !sin_t) return TCQ_ERR_ARG;
    if (rows <= 0 || T <= 0 || heads <= 0 || D <= 0 || (D & 1) || ldx < heads * D || ldo < heads * D) return TCQ_ERR_SHAPE;
    return launch_rows(k_rope, rows, 256, 0, stream, (const u16*)x, (u16*)out, cos_t, sin_t, T, heads, D, ldx, ldo);
}

}  // extern "C"
