// Randomized block-Walsh rotation, per-token INT8 quantizer and the scale epilogue on sm_100a.
//
// One thread block per token row. A row of width K (multiple of 16, <= 16384) is the concatenation of descending
// power-of-two blocks (tcq_format.py:26-30); each block gets the FP32 Walsh transform with stages h = 1, 2, 4, ...
// and the scale (float)(1 / sqrt(w)) (tcq_format.py:44-55). The transform runs as radix-16 passes: the first pass
// takes 16 contiguous inputs per thread straight from global memory (128-bit loads) and performs stages 1..8 in
// registers; the later passes (stride 16, 256, 4096) go through shared memory in an XOR-swizzled layout that keeps
// every 128-bit store and every 32-float warp access conflict-free. A radix-2^R pass performs exactly the additions
// of R consecutive radix-2 stages in the same order, so the sums are bit-identical to the reference.
#include <type_traits>

#include "rownorm.cuh"
#include "rowwalsh.cuh"
#include "tcq_common.cuh"

namespace {

using namespace tcq;

constexpr int kMaxWidth = 16384;

// ---------------------------------------------------------------------------------------------------- kernels
// CH: elements per thread chunk (4 or 16, see rowwalsh.cuh); the host picks it per launch (rows_ch) and launches
// threads_for(K, CH) threads per row.
template <int DT, int CH>
__global__ void __launch_bounds__(512, 1) k_pre(const void* __restrict__ x, const i8* __restrict__ su, int8_t* __restrict__ q,
                                             int* __restrict__ q4, float* __restrict__ scale, int M, int K, int ldq) {
    extern __shared__ __align__(16) float buf[];
    __shared__ float red[32];
    pdl_launch_dependents();
    pdl_wait();
    const int tok = blockIdx.x;
    const size_t es = DT == TCQ_DT_F32 ? 4 : 2;
    const char* xr = reinterpret_cast<const char*>(x) + (size_t)tok * K * es;
    float mx = 0.f;
    row_walshc<CH>(buf, K,
                   [&](int c, float* v) {
                       float sg[CH];
                       loadc<DT, CH>(xr + (size_t)CH * c * es, v);
                       load_signsc<CH, true>(su + CH * c, sg);
#pragma unroll
                       for (int k = 0; k < CH; ++k) v[k] = v[k] * sg[k];
                   },
                   [&](int i0, const float* v) { store_chunk<CH>(buf, i0, v, mx); },
                   [&](int i, float v) { buf[swz(i)] = v; mx = fmaxf(mx, fabsf(v)); });
    quantize_store(buf, mx, red, q, q4, scale, tok, K, ldq);
}

template <int CH>
__global__ void __launch_bounds__(512, 1) k_pre2(const u16* __restrict__ g, const u16* __restrict__ u, const i8* __restrict__ su,
                                              int8_t* __restrict__ q, int* __restrict__ q4, float* __restrict__ scale, int M,
                                              int K, int ldq) {
    extern __shared__ __align__(16) float buf[];
    __shared__ float red[32];
    pdl_launch_dependents();
    pdl_wait();
    const int tok = blockIdx.x;
    const size_t base = (size_t)tok * K;
    float mx = 0.f;
    row_walshc<CH>(buf, K,
                   [&](int c, float* v) {
                       float gv[CH], uv[CH], sg[CH];
                       loadc<TCQ_DT_BF16, CH>(g + base + CH * c, gv);
                       loadc<TCQ_DT_BF16, CH>(u + base + CH * c, uv);
                       load_signsc<CH, true>(su + CH * c, sg);
#pragma unroll
                       for (int k = 0; k < CH; ++k) v[k] = bf2f(f2bf(gv[k] * uv[k])) * sg[k];
                   },
                   [&](int i0, const float* v) { store_chunk<CH>(buf, i0, v, mx); },
                   [&](int i, float v) { buf[swz(i)] = v; mx = fmaxf(mx, fabsf(v)); });
    quantize_store(buf, mx, red, q, q4, scale, tok, K, ldq);
}

template <int DT, int CH>
__global__ void __launch_bounds__(512, 1) k_pre_h(const void* __restrict__ x, const i8* __restrict__ su, u16* __restrict__ h,
                                               u16* __restrict__ hT, int M, int K, int ldh) {
    extern __shared__ __align__(16) float buf[];
    pdl_launch_dependents();
    pdl_wait();
    const int tok = blockIdx.x;
    const size_t es = DT == TCQ_DT_F32 ? 4 : 2;
    const char* xr = reinterpret_cast<const char*>(x) + (size_t)tok * K * es;
    row_walshc<CH>(buf, K,
                   [&](int c, float* v) {
                       float sg[CH];
                       loadc<DT, CH>(xr + (size_t)CH * c * es, v);
                       load_signsc<CH, true>(su + CH * c, sg);
#pragma unroll
                       for (int k = 0; k < CH; ++k) v[k] = v[k] * sg[k];
                   },
                   [&](int i0, const float* v) {
                       u32 w[CH / 2];
                       pack_bf16c<CH>(v, w);
                       if (h) store_bf16c_any<CH>(h + (size_t)tok * K + i0, w);
                       if (hT) {
#pragma unroll
                           for (int k = 0; k < CH; ++k)
                               hT[(size_t)(i0 + k) * ldh + tok] = (u16)((k & 1) ? (w[k >> 1] >> 16) : (w[k >> 1] & 0xffffu));
                       }
                   },
                   [&](int i, float v) {
                       const u16 b = f2bf(v);
                       if (h) h[(size_t)tok * K + i] = b;
                       if (hT) hT[(size_t)i * ldh + tok] = b;
                   });
}

template <int DT, int OT, int CH>
__global__ void __launch_bounds__(512, 1) k_rotate(const void* __restrict__ x, const i8* __restrict__ sg, void* __restrict__ y,
                                                int M, int D, int inverse) {
    extern __shared__ __align__(16) float buf[];
    pdl_launch_dependents();
    pdl_wait();
    const int tok = blockIdx.x;
    const size_t es = DT == TCQ_DT_F32 ? 4 : 2;
    const char* xr = reinterpret_cast<const char*>(x) + (size_t)tok * D * es;
    row_walshc<CH>(buf, D,
                   [&](int c, float* v) {
                       loadc<DT, CH>(xr + (size_t)CH * c * es, v);
                       if (!inverse) {
                           float s16[CH];
                           load_signsc<CH, true>(sg + CH * c, s16);
#pragma unroll
                           for (int k = 0; k < CH; ++k) v[k] = v[k] * s16[k];
                       }
                   },
                   [&](int i0, const float* vin) {
                       float v[CH];
#pragma unroll
                       for (int k = 0; k < CH; ++k) v[k] = vin[k];
                       if (inverse) {
                           float s16[CH];
                           load_signsc<CH, true>(sg + i0, s16);
#pragma unroll
                           for (int k = 0; k < CH; ++k) v[k] = v[k] * s16[k];
                       }
                       if (OT == TCQ_DT_F32) {
                           float4* o = reinterpret_cast<float4*>(reinterpret_cast<float*>(y) + (size_t)tok * D + i0);
#pragma unroll
                           for (int q = 0; q < CH / 4; ++q) o[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
                       } else {
                           u32 w[CH / 2];
                           pack_bf16c<CH>(v, w);
                           store_bf16c<CH>(reinterpret_cast<u16*>(y) + (size_t)tok * D + i0, w);
                       }
                   },
                   [&](int i, float v) {
                       if (inverse) v = v * (float)sg[i];
                       if (OT == TCQ_DT_F32) reinterpret_cast<float*>(y)[(size_t)tok * D + i] = v;
                       else reinterpret_cast<u16*>(y)[(size_t)tok * D + i] = f2bf(v);
                   });
}

// The rotation op on power-of-two widths D = 2^NL (1024 .. 16384: benchmark config 2), one row per CTA of D / 32
// threads. A thread holds 32 elements at a time: V consecutive ones (index bits 0 .. log2 V - 1) times the 2^WB values
// of a WB-bit window of index bits [lo, lo + WB), WB = 5 - log2 V (the first window is bits 0..4, i.e. 32 consecutive
// elements). The butterfly stages of the window's new bits run in registers (low slot a + b, high slot a - b, in the
// order h = 1, 2, 4, ...: the definition's order, so the sums are bit-identical). Windows after the first take WB new
// bits each in increasing order (the last one slides down to end at bit NL - 1 and skips bits already done). Between
// windows the row passes through shared memory as groups of V floats, with one group of padding after every 2^WB
// groups (group g at g + g / 2^WB): window 0's threads start 2^WB + 1 groups apart and every later window has
// lo - log2 V >= WB, so every access of every window is conflict-free (16 lanes per 128-byte phase for V = 2, 8 for
// V = 4), at the thread's base plus an immediate. The last window stores V consecutive outputs at a time.
// V = 2 (WB = 4) takes two exchanges at D = 4096 and 8192 where V = 4 (WB = 3) takes three (16 instead of 24 bytes
// of shared-memory traffic per element: 4096 x 4096 in 20.0 instead of 23.0 us), and at 16384 three either way but
// wins 2 % there; at 1024 and 2048 the counts are equal and V = 4 moves them with half the instructions.
template <int DT, int OT, int NL>
__global__ void __launch_bounds__((1 << NL) / 32) k_rotate_p2(const void* __restrict__ x, const i8* __restrict__ sg,
                                                            void* __restrict__ y, int inverse) {
    constexpr int D = 1 << NL, V = rot_vec<NL>();
    constexpr int WB = Win2<NL, V>::WB, G = 1 << WB;
    extern __shared__ __align__(16) float buf[];
    i8* ssg = reinterpret_cast<i8*>(buf + D + (D >> WB));          // inverse: the row's signs, for the last window
    pdl_launch_dependents();
    const int t = threadIdx.x;
    if (inverse) {                                                  // 32 signs per thread (read after a barrier below)
        const uint4* src = reinterpret_cast<const uint4*>(sg) + 2 * t;
        uint4* dst = reinterpret_cast<uint4*>(ssg) + 2 * t;
        dst[0] = __ldg(src);
        dst[1] = __ldg(src + 1);
    }
    pdl_wait();
    const size_t row = blockIdx.x;
    float v[32];
    {
        const size_t es = DT == TCQ_DT_F32 ? 4 : 2;
        loadc<DT, 32>(reinterpret_cast<const char*>(x) + (row * D + 32 * t) * es, v);
        if (!inverse) {
            float s32[32];
            load_signsc<32, true>(sg + 32 * t, s32);
#pragma unroll
            for (int k = 0; k < 32; ++k) v[k] = v[k] * s32[k];
        }
    }
    win_walsh<NL, false>(v, buf, t);
    // the last window: scale, signs (inverse), V consecutive outputs per store
    const float sc = wscale(D);
#pragma unroll
    for (int q = 0; q < G; ++q) {
        const int e = win_elem<NL>(t, q, 0);
        float o[V];
#pragma unroll
        for (int k = 0; k < V; ++k) o[k] = v[V * q + k] * sc;
        if (inverse) {
            const u32 sw = V == 2 ? (u32)*reinterpret_cast<const u16*>(ssg + e) : *reinterpret_cast<const u32*>(ssg + e);
#pragma unroll
            for (int k = 0; k < V; ++k) o[k] = o[k] * (float)(i8)((sw >> (8 * k)) & 0xffu);
        }
        if constexpr (V == 2) {
            if (OT == TCQ_DT_F32) *reinterpret_cast<float2*>(reinterpret_cast<float*>(y) + row * D + e) = make_float2(o[0], o[1]);
            else *reinterpret_cast<u32*>(reinterpret_cast<u16*>(y) + row * D + e) = f2bf2(o[0], o[1]);
        } else {
            if (OT == TCQ_DT_F32) {
                *reinterpret_cast<float4*>(reinterpret_cast<float*>(y) + row * D + e) = make_float4(o[0], o[1], o[2], o[3]);
            } else {
                *reinterpret_cast<uint2*>(reinterpret_cast<u16*>(y) + row * D + e) = make_uint2(f2bf2(o[0], o[1]), f2bf2(o[2], o[3]));
            }
        }
    }
}

// Epilogue of one layer on one token: SCALE(acc[base + i]) -> block Walsh -> * sv -> + bias -> BF16 (-> act).
// out(i, b): one BF16 result; outc(i0, w): the CH results of chunk i0 as CH / 2 packed words (element i0 + k in the
// low half of w[k / 2] for even k). sv / bias / rs may be shared-memory copies.
template <int AT, int CH, class Out, class Outc>
__device__ __forceinline__ void post_row(float* buf, const void* acc, size_t base, float s, const float* rs, const i8* sv,
                                         const float* bias, int N, Out out, Outc outc) {
    row_walshc<CH>(buf, N, [&](int c, float* v) { load_scaledc<AT, CH>(acc, base + CH * c, s, rs ? rs + CH * c : nullptr, v); },
                   [&](int i0, const float* vin) {
                       float v[CH], sg[CH];
                       load_signsc<CH, false>(sv + i0, sg);
#pragma unroll
                       for (int k = 0; k < CH; ++k) v[k] = vin[k] * sg[k];
                       if (bias) {
                           float bb[CH];
                           load_f32c<CH, false>(bias + i0, bb);
#pragma unroll
                           for (int k = 0; k < CH; ++k) v[k] = v[k] + bb[k];
                       }
                       u32 w[CH / 2];
                       pack_bf16c<CH>(v, w);
                       outc(i0, w);
                   },
                   [&](int i, float v) {
                       v = v * (float)sv[i];
                       if (bias) v = v + bias[i];
                       out(i, f2bf(v));
                   });
}

template <int AT, int CH>
__global__ void __launch_bounds__(512, 2) k_post(const void* __restrict__ acc, const float* __restrict__ s, const float* __restrict__ rs,
                                              const i8* __restrict__ sv, const float* __restrict__ bias, u16* __restrict__ y, int M,
                                              int N, int lda, int col0, int stage) {
    extern __shared__ __align__(16) float buf[];
    pdl_launch_dependents();
    char* sp = reinterpret_cast<char*>(buf + N);    // layer constants (tcq_post sizes the same set)
    const float* rsc = static_cast<const float*>(stage_const(sp, AT != TCQ_DT_F32 ? rs : nullptr, 4 * N, stage != 0));
    const float* biasc = static_cast<const float*>(stage_const(sp, bias, 4 * N, stage != 0));
    const i8* svc = static_cast<const i8*>(stage_const(sp, sv, N, stage != 0));
    __syncthreads();
    pdl_wait();
    const int tok = blockIdx.x;
    u16* yo = y + (size_t)tok * N;
    post_row<AT, CH>(buf, acc, (size_t)tok * lda + col0, s ? s[tok] : 1.f, rsc, svc, biasc, N, [&](int i, u16 b) { yo[i] = b; },
                     [&](int i0, const u32* w) { store_bf16c_any<CH>(yo + i0, w); });
}

// Several layers sharing the accumulator row. grid.y == 1: the layers one after another in one block (post3);
// grid.y == number of layers: one block per (token, layer) (postg). act0: activation table on layer 0's output.
template <int AT, int CH>
__global__ void __launch_bounds__(512, 1) k_post_multi(const void* __restrict__ acc, const float* __restrict__ s,
                                                    const float* __restrict__ rs, const i8* __restrict__ sv,
                                                    const float* __restrict__ bias, const u16* __restrict__ lut, u16* y0, u16* y1,
                                                    u16* y2, int M, int n0, int n1, int n2, int lda, int act0, int nmax,
                                                    int stage) {
    extern __shared__ __align__(16) float buf[];
    pdl_launch_dependents();
    const int seg_begin = gridDim.y == 1 ? 0 : blockIdx.y, seg_end = gridDim.y == 1 ? 3 : blockIdx.y + 1;
    // The constants of this block's columns [cs, ce) into shared memory (after the nmax-float Walsh buffer).
    const int cs = seg_begin == 0 ? 0 : seg_begin == 1 ? n0 : n0 + n1;
    const int ce = seg_end == 1 ? n0 : seg_end == 2 ? n0 + n1 : n0 + n1 + n2;
    char* sp = reinterpret_cast<char*>(buf + nmax);
    const bool on = stage != 0;
    const float* rsc = static_cast<const float*>(stage_const(sp, AT != TCQ_DT_F32 && rs ? rs + cs : nullptr, 4 * (ce - cs), on));
    const float* biasc = static_cast<const float*>(stage_const(sp, bias ? bias + cs : nullptr, 4 * (ce - cs), on));
    const i8* svc = static_cast<const i8*>(stage_const(sp, sv + cs, ce - cs, on));
    __syncthreads();
    pdl_wait();
    const int tok = blockIdx.x;
    for (int seg = seg_begin; seg < seg_end; ++seg) {
        const int N = seg == 0 ? n0 : seg == 1 ? n1 : n2;
        if (N == 0) continue;
        const int c0 = seg == 0 ? 0 : seg == 1 ? n0 : n0 + n1;
        u16* yo = (seg == 0 ? y0 : seg == 1 ? y1 : y2) + (size_t)tok * N;
        const bool act = act0 && seg == 0;
        post_row<AT, CH>(buf, acc, (size_t)tok * lda + c0, s ? s[tok] : 1.f, rsc ? rsc + (c0 - cs) : nullptr, svc + (c0 - cs),
                         biasc ? biasc + (c0 - cs) : nullptr, N, [&](int i, u16 b) { yo[i] = act ? lut[b] : b; },
                         [&](int i0, const u32* w) {
                             if (act) {
                                 u32 a[CH / 2];
#pragma unroll
                                 for (int k = 0; k < CH / 2; ++k) a[k] = (u32)lut[w[k] & 0xffffu] | ((u32)lut[w[k] >> 16] << 16);
                                 store_bf16c_any<CH>(yo + i0, a);
                             } else {
                                 store_bf16c_any<CH>(yo + i0, w);
                             }
                         });
    }
}

// Fused chain of one token row across a residual block boundary: one layer's post, the model's residual add and
// norm, and the next layer's pre, without the BF16 round trips between them (four launches become one):
//   y = post(acc)        as k_post: SCALE(acc) -> block Walsh -> * sv -> + bias -> BF16          (acc != NULL)
//       or y = yg        a BF16 tensor                                                            (yg != NULL)
//   h = BF16(x + y)      written to hout (h = x when there is no y)
//   n = norm(h)          norm_chunks: the same arithmetic and sum order as tcq_add_norm; BF16(n) written to nout
//                        when given
//   q / q4, scale        = pre(BF16(n), su) as k_pre on a BF16 input                             (su != NULL)
// Each step is bit-identical to the separate kernel. Shared memory: N floats (Walsh buffer) + N BF16 (y, then n),
// then the staged constants and the copy area of the row inputs.
template <int AT, int KIND, bool WBF16, int NC, int CH>
__global__ void __launch_bounds__(512, 1) k_chain(const void* __restrict__ acc, const float* __restrict__ s, const float* __restrict__ rs,
                                               const i8* __restrict__ sv, const float* __restrict__ bias, int lda, int col0,
                                               const u16* __restrict__ yg, const u16* __restrict__ x, u16* __restrict__ hout,
                                               u16* __restrict__ nout, const void* __restrict__ w, const void* __restrict__ b,
                                               const u16* __restrict__ mscale, const u16* __restrict__ mshift, int mod_rows,
                                               int ld_mod, float eps, const i8* __restrict__ su, int8_t* __restrict__ q,
                                               int* __restrict__ q4, float* __restrict__ scale, int ldq, int N, int stage) {
    extern __shared__ __align__(16) float buf[];
    __shared__ float red[32];
    u16* yb = reinterpret_cast<u16*>(buf + N);
    pdl_launch_dependents();
    // Layer constants into shared memory while the previous kernel drains (tcq_chain sizes the same set).
    char* sp = reinterpret_cast<char*>(yb + N);
    const bool on = stage != 0;
    const float* rsc = static_cast<const float*>(stage_const(sp, acc && AT != TCQ_DT_F32 ? rs : nullptr, 4 * N, on));
    const float* biasc = static_cast<const float*>(stage_const(sp, acc ? bias : nullptr, 4 * N, on));
    const i8* svc = static_cast<const i8*>(stage_const(sp, acc ? sv : nullptr, N, on));
    const void* wc = stage_const(sp, w, (WBF16 ? 2 : 4) * N, on);
    const void* bc = stage_const(sp, b, (WBF16 ? 2 : 4) * N, on);
    const i8* suc = static_cast<const i8*>(stage_const(sp, su, N, on));
    __syncthreads();
    pdl_wait();
    const int tok = blockIdx.x, nch = N / CH;
    const size_t base = (size_t)tok * N;
    // With staging on, the thread's first chunk of x (and of y / the modulation) is copied into shared memory
    // asynchronously now, with the accumulator loads in flight, so that the residual add and the norm find it there
    // (the copy area follows the constants: x, then y when added from a tensor, then the two modulation vectors).
    // Chunks of CH = 4 are 8 bytes: two threads' chunks form one 16-byte copy, issued by the even thread.
    const bool first = (int)threadIdx.x < nch;
    const u16* ms = mscale ? mscale + (size_t)(tok / mod_rows) * ld_mod : nullptr;
    const u16* mh = mscale ? mshift + (size_t)(tok / mod_rows) * ld_mod : nullptr;
    const bool ycopy = !acc && yg, mcopy = ms && (((uintptr_t)ms | (uintptr_t)mh) & 15) == 0;
    u16* xs = reinterpret_cast<u16*>(sp);
    u16* ys = xs + N;
    u16* mss = ys + (ycopy ? N : 0);
    u16* mhs = mss + N;
    if (on) {
        for (int o = 8 * threadIdx.x; o < (nch < (int)blockDim.x ? nch : (int)blockDim.x) * CH; o += 8 * blockDim.x) {
            cp_async16(xs + o, x + base + o);
            if (ycopy) cp_async16(ys + o, yg + base + o);
            if (mcopy) {
                cp_async16(mss + o, ms + o);
                cp_async16(mhs + o, mh + o);
            }
        }
    }
    if (acc)                                        // ends with a block barrier: yb complete
        post_row<AT, CH>(buf, acc, (size_t)tok * lda + col0, s ? s[tok] : 1.f, rsc, svc, biasc, N, [&](int i, u16 v) { yb[i] = v; },
                         [&](int i0, const u32* ww) { store_bf16c<CH>(yb + i0, ww); });
    ModChunk<CH> m0{};
    if (on) {
        cp_async_wait_all();
        __syncthreads();                            // copies of 16 bytes span the chunks of two threads
        if (mcopy && first) load_mod_chunk<CH, false>(m0, mss + CH * threadIdx.x, mhs + CH * threadIdx.x);
    }
    float v[NC][CH];
#pragma unroll
    for (int k = 0; k < NC; ++k) {
        const int c = threadIdx.x + k * blockDim.x;
        if (c < nch) {
            if (k == 0 && on) load_bf16c_any<CH>(xs + CH * c, v[k]);
            else loadc<TCQ_DT_BF16, CH>(x + base + CH * c, v[k]);
            if (acc || yg) {
                float t[CH];
                if (acc) load_bf16c_any<CH>(yb + CH * c, t);
                else if (k == 0 && on) load_bf16c_any<CH>(ys + CH * c, t);
                else loadc<TCQ_DT_BF16, CH>(yg + base + CH * c, t);
                add_round_chunk<CH>(v[k], t, hout ? hout + base + CH * c : nullptr);
            }
        }
    }
    norm_chunks<KIND, WBF16, NC, CH>(v, N, wc, bc, ms, mh, eps, red, m0);   // synchronizes: all reads of yb are done
#pragma unroll
    for (int k = 0; k < NC; ++k) {
        const int c = threadIdx.x + k * blockDim.x;
        if (c < nch) {
            u32 wn[CH / 2];
            pack_bf16c<CH>(v[k], wn);
            if (nout) store_bf16c<CH>(nout + base + CH * c, wn);
            store_bf16c<CH>(yb + CH * c, wn);
        }
    }
    if (!su) {
        if (!q && !q4) return;
        // No rotation: the per-token INT8 quantization of BF16(n) itself (the W8A8 layers' quantizer, tcq_quantize's
        // arithmetic). quantize_store's block maximum synchronizes before any thread reads another's values.
        float mx = 0.f;
#pragma unroll
        for (int k = 0; k < NC; ++k) {
            const int c = threadIdx.x + k * blockDim.x;
            if (c < nch) {
                float nv[CH];
                load_bf16c_any<CH>(yb + CH * c, nv);
                store_chunk<CH>(buf, CH * c, nv, mx);
            }
        }
        quantize_store(buf, mx, red, q, q4, scale, tok, N, ldq);
        return;
    }
    __syncthreads();
    float mx = 0.f;
    row_walshc<CH>(buf, N,
                   [&](int c, float* vv) {
                       float sg[CH], nb[CH];
                       load_signsc<CH, false>(suc + CH * c, sg);
                       load_bf16c_any<CH>(yb + CH * c, nb);
#pragma unroll
                       for (int i = 0; i < CH; ++i) vv[i] = nb[i] * sg[i];
                   },
                   [&](int i0, const float* vv) { store_chunk<CH>(buf, i0, vv, mx); },
                   [&](int i, float val) { buf[swz(i)] = val; mx = fmaxf(mx, fabsf(val)); });
    quantize_store(buf, mx, red, q, q4, scale, tok, N, ldq);
}

// The finished row in buf as the next transform's input chunk c.
template <int CH>
__device__ __forceinline__ void buf_chunk(const float* buf, int c, float* v) {
    const float4* b4 = reinterpret_cast<const float4*>(buf);
#pragma unroll
    for (int g = 0; g < CH / 4; ++g) {
        const float4 a = b4[swz(CH * c + 4 * g) >> 2];
        v[4 * g] = a.x; v[4 * g + 1] = a.y; v[4 * g + 2] = a.z; v[4 * g + 3] = a.w;
    }
}

// Gated-MLP middle (kernels.py:263-278): g = lut(BF16(post(gate))), u = BF16(post(up)), x = BF16(g * u) * su,
// block Walsh, INT8. Shared memory: N floats + N BF16.
template <int AT, int CH>
__global__ void __launch_bounds__(512, 2) k_mid2(const void* __restrict__ acc, const float* __restrict__ s, const float* __restrict__ rs,
                                              const i8* __restrict__ sv, const u16* __restrict__ lut, const i8* __restrict__ su,
                                              int8_t* __restrict__ q, int* __restrict__ q4, float* __restrict__ scale, int M, int N,
                                              int lda, int ldq, int stage) {
    extern __shared__ __align__(16) float buf[];
    __shared__ float red[32];
    u16* gb = reinterpret_cast<u16*>(buf + N);
    pdl_launch_dependents();
    char* sp = reinterpret_cast<char*>(gb + N);     // layer constants of the gate and up layers and the next pre
    const bool on = stage != 0;
    const float* rsc = static_cast<const float*>(stage_const(sp, AT != TCQ_DT_F32 ? rs : nullptr, 8 * N, on));
    const i8* svc = static_cast<const i8*>(stage_const(sp, sv, 2 * N, on));
    const i8* suc = static_cast<const i8*>(stage_const(sp, su, N, on));
    __syncthreads();
    pdl_wait();
    const int tok = blockIdx.x;
    const size_t base = (size_t)tok * lda;
    const float st = s ? s[tok] : 1.f;
    row_walsh<CH>(buf, N, [&](int c, float* v) { load_scaledc<AT, CH>(acc, base + CH * c, st, rsc ? rsc + CH * c : nullptr, v); },
                  [&](int i, float v) { gb[i] = lut[f2bf(v * (float)svc[i])]; });
    row_walsh<CH>(buf, N, [&](int c, float* v) { load_scaledc<AT, CH>(acc, base + N + CH * c, st, rsc ? rsc + N + CH * c : nullptr, v); },
                  [&](int i, float v) {
                      const u16 u = f2bf(v * (float)svc[N + i]);
                      buf[swz(i)] = bf2f(f2bf(bf2f(gb[i]) * bf2f(u))) * (float)suc[i];
                  });
    float mx = 0.f;
    row_walshc<CH>(buf, N, [&](int c, float* v) { buf_chunk<CH>(buf, c, v); },
                   [&](int i0, const float* v) { store_chunk<CH>(buf, i0, v, mx); },
                   [&](int i, float v) { buf[swz(i)] = v; mx = fmaxf(mx, fabsf(v)); });
    quantize_store(buf, mx, red, q, q4, scale, tok, N, ldq);
}

// The gated-MLP middle on a power-of-two width N = 2^NL (1024 .. 16384: the LLM's 8192): the same arithmetic as
// k_mid2, each of its three block Walsh transforms done by win_walsh (32 elements per thread, register windows,
// two or three shared-memory exchanges) instead of the general row transform. The gate and up transforms end in the
// same register layout, so g * u is formed in registers; one exchange brings the product back to window 0 for the
// third transform; the finished row goes through shared memory to quantize_store (the common quantizer).
template <int AT, int NL>
__global__ void __launch_bounds__((1 << NL) / 32) k_mid2_p2(const void* __restrict__ acc, const float* __restrict__ s,
                                                          const float* __restrict__ rs, const i8* __restrict__ sv,
                                                          const u16* __restrict__ lut, const i8* __restrict__ su,
                                                          int8_t* __restrict__ q, int* __restrict__ q4, float* __restrict__ scale,
                                                          int lda, int ldq) {
    constexpr int N = 1 << NL, V = rot_vec<NL>();
    constexpr int WB = Win2<NL, V>::WB, G = 1 << WB;
    extern __shared__ __align__(16) float buf[];
    __shared__ float red[32];
    // sv of both layers and su staged in shared memory before the dependency wait (layer constants)
    i8* ssv = reinterpret_cast<i8*>(buf + N + (N >> WB));
    i8* ssu = ssv + 2 * N;
    pdl_launch_dependents();
    const int t = threadIdx.x;
    for (int i = t; i < 2 * N / 16; i += N / 32) reinterpret_cast<uint4*>(ssv)[i] = __ldg(reinterpret_cast<const uint4*>(sv) + i);
    for (int i = t; i < N / 16; i += N / 32) reinterpret_cast<uint4*>(ssu)[i] = __ldg(reinterpret_cast<const uint4*>(su) + i);
    pdl_wait();
    const int tok = blockIdx.x;
    const size_t base = (size_t)tok * lda;
    const float st = s ? s[tok] : 1.f;
    const float sc = wscale(N);
    float v[32];
    auto load_half = [&](int off) {                 // window 0 of z = SCALE(acc[base + off + i])
        const float* r = rs ? rs + off + 32 * t : nullptr;
        load_scaledc<AT, 16>(acc, base + off + 32 * t, st, r, v);
        load_scaledc<AT, 16>(acc, base + off + 32 * t + 16, st, r ? r + 16 : nullptr, v + 16);
    };
    // gate: g = lut(BF16(post(gate))), kept as BF16 pairs in registers; the up half's 128 bytes per thread (and its
    // row scales) are requested into L1 now, to be read after the gate transform
    load_half(0);
    asm volatile("prefetch.global.L1 [%0];" ::"l"(static_cast<const char*>(acc) + (base + N + 32 * t) * 4));
    if (rs) asm volatile("prefetch.global.L1 [%0];" ::"l"(rs + N + 32 * t));
    __syncthreads();                                // the staged constants are complete
    win_walsh<NL, false>(v, buf, t);
    u32 gw[16];
#pragma unroll
    for (int qq = 0; qq < G; ++qq) {
        const int e = win_elem<NL>(t, qq, 0);
#pragma unroll
        for (int k = 0; k < V; k += 2) {
            const int r = V * qq + k;
            const u16 g0 = __ldg(lut + f2bf((v[r] * sc) * (float)ssv[e + k]));
            const u16 g1 = __ldg(lut + f2bf((v[r + 1] * sc) * (float)ssv[e + k + 1]));
            gw[r >> 1] = (u32)g0 | ((u32)g1 << 16);
        }
    }
    // up, then x = BF16(g * u) * su in registers
    load_half(N);
    win_walsh<NL, true>(v, buf, t);
#pragma unroll
    for (int qq = 0; qq < G; ++qq) {
        const int e = win_elem<NL>(t, qq, 0);
#pragma unroll
        for (int k = 0; k < V; ++k) {
            const int r = V * qq + k;
            const u16 u = f2bf((v[r] * sc) * (float)ssv[N + e + k]);
            const u16 g = (u16)(gw[r >> 1] >> (16 * (r & 1)));
            v[r] = bf2f(f2bf(bf2f(g) * bf2f(u))) * (float)ssu[e + k];
        }
    }
    // the next layer's pre: block Walsh of x, INT8 (quantize_store reads the finished row at swz positions)
    win_relayout<NL>(v, buf, t);
    win_walsh<NL, true>(v, buf, t);
    __syncthreads();                                // every thread has read buf in the last window
    float mx = 0.f;
#pragma unroll
    for (int qq = 0; qq < G; ++qq) {
        const int e = win_elem<NL>(t, qq, 0);
#pragma unroll
        for (int k = 0; k < V; ++k) {
            const float o = v[V * qq + k] * sc;
            buf[swz(e + k)] = o;
            mx = fmaxf(mx, fabsf(o));
        }
    }
    quantize_store(buf, mx, red, q, q4, scale, tok, N, ldq);
}

// One row transform on a width of one or two power-of-two blocks (as k_mid1_2b): load(e0, v) fills the 32 inputs
// e0 .. e0 + 31 of a thread's window 0, fin(e, v, sc, V) takes V finished unscaled outputs e .. e + V - 1 and the
// block's scale. A block-wide barrier separates the transform's last shared-memory reads from fin, which may rewrite
// buf. buf: the exchange areas of both blocks (as k_mid1_2b). Every thread of the row's block calls this.
template <int NL0, int NL1, class Load, class Fin>
__device__ __forceinline__ void row2b_transform(float* buf, int t, Load load, Fin fin) {
    constexpr int NLB = NL1 ? NL1 : NL0, N0 = 1 << NL0, T0 = N0 / 32;
    constexpr int WB0 = Win2<NL0, rot_vec<NL0>()>::WB;
    static_assert(!NL1 || (NL1 < NL0 && Win2<NL0, rot_vec<NL0>()>::P == Win2<NLB, rot_vec<NLB>()>::P),
                  "the two blocks' transforms execute the same barriers");
    auto run = [&](auto nlc, int tb, int off, float* bb) {
        constexpr int NL = decltype(nlc)::value, V = rot_vec<NL>(), G = 1 << Win2<NL, V>::WB;
        float v[32];
        load(off + 32 * tb, v);
        win_walsh<NL, true, 1>(v, bb, tb);
        blk_sync<1>();
        const float sc = wscale(1 << NL);
#pragma unroll
        for (int qq = 0; qq < G; ++qq) fin(off + win_elem<NL>(tb, qq, 0), v + V * qq, sc, std::integral_constant<int, V>{});
    };
    if (t < T0) run(std::integral_constant<int, NL0>{}, t, 0, buf);
    else if constexpr (NL1 != 0) run(std::integral_constant<int, NLB>{}, t - T0, N0, buf + N0 + (N0 >> WB0));
}

// Shared memory of row2b_transform's exchange areas, in floats.
template <int NL0, int NL1>
constexpr int row2b_floats() {
    constexpr int NLB = NL1 ? NL1 : NL0;
    return (1 << NL0) + ((1 << NL0) >> Win2<NL0, rot_vec<NL0>()>::WB) +
           (NL1 ? (1 << NLB) + ((1 << NLB) >> Win2<NLB, rot_vec<NLB>()>::WB) : 0);
}

// pre (k_pre's arithmetic) on widths of one or two power-of-two blocks, for latency-bound launches.
template <int DT, int NL0, int NL1>
__global__ void __launch_bounds__(((1 << NL0) + (NL1 ? (1 << NL1) : 0)) / 32)
k_pre_2b(const void* __restrict__ x, const i8* __restrict__ su, int8_t* __restrict__ q, int* __restrict__ q4,
         float* __restrict__ scale, int ldq) {
    constexpr int K = (1 << NL0) + (NL1 ? (1 << NL1) : 0);
    extern __shared__ __align__(16) float buf[];
    __shared__ float red[32];
    pdl_launch_dependents();
    pdl_wait();
    const int tok = blockIdx.x;
    const size_t es = DT == TCQ_DT_F32 ? 4 : 2;
    const char* xr = reinterpret_cast<const char*>(x) + (size_t)tok * K * es;
    float mx = 0.f;
    row2b_transform<NL0, NL1>(buf, threadIdx.x,
        [&](int e0, float* v) {
            float sg[32];
            loadc<DT, 32>(xr + (size_t)e0 * es, v);
            load_signsc<32, true>(su + e0, sg);
#pragma unroll
            for (int k = 0; k < 32; ++k) v[k] = v[k] * sg[k];
        },
        [&](int e, const float* v, float sc, auto vc) {
#pragma unroll
            for (int k = 0; k < decltype(vc)::value; ++k) {
                const float o = v[k] * sc;
                buf[swz(e + k)] = o;
                mx = fmaxf(mx, fabsf(o));
            }
        });
    quantize_store(buf, mx, red, q, q4, scale, tok, K, ldq);
}

// post (k_post's arithmetic) on widths of one or two power-of-two blocks, for latency-bound launches; sv and bias
// staged before the dependency wait.
template <int AT, int NL0, int NL1>
__global__ void __launch_bounds__(((1 << NL0) + (NL1 ? (1 << NL1) : 0)) / 32)
k_post_2b(const void* __restrict__ acc, const float* __restrict__ s, const float* __restrict__ rs, const i8* __restrict__ sv,
          const float* __restrict__ bias, u16* __restrict__ y, int lda, int col0) {
    constexpr int N = (1 << NL0) + (NL1 ? (1 << NL1) : 0);
    extern __shared__ __align__(16) float buf[];
    float* sbias = buf + row2b_floats<NL0, NL1>();
    i8* ssv = reinterpret_cast<i8*>(sbias + (bias ? N : 0));
    pdl_launch_dependents();
    const int t = threadIdx.x, nt = N / 32;
    for (int i = t; i < N / 16; i += nt) reinterpret_cast<uint4*>(ssv)[i] = __ldg(reinterpret_cast<const uint4*>(sv) + i);
    if (bias)
        for (int i = t; i < N / 4; i += nt) reinterpret_cast<float4*>(sbias)[i] = __ldg(reinterpret_cast<const float4*>(bias) + i);
    __syncthreads();
    pdl_wait();
    const int tok = blockIdx.x;
    const size_t base = (size_t)tok * lda + col0;
    const float st = s ? s[tok] : 1.f;
    u16* yo = y + (size_t)tok * N;
    row2b_transform<NL0, NL1>(buf, t,
        [&](int e0, float* v) {
            const float* r = rs ? rs + e0 : nullptr;
            load_scaledc<AT, 16>(acc, base + e0, st, r, v);
            load_scaledc<AT, 16>(acc, base + e0 + 16, st, r ? r + 16 : nullptr, v + 16);
        },
        [&](int e, const float* v, float sc, auto vc) {
            constexpr int V = decltype(vc)::value;
            u16 o[V];
#pragma unroll
            for (int k = 0; k < V; ++k) {
                float z = (v[k] * sc) * (float)ssv[e + k];
                if (bias) z = z + sbias[e + k];
                o[k] = f2bf(z);
            }
            if constexpr (V == 2) {
                *reinterpret_cast<u32*>(yo + e) = (u32)o[0] | ((u32)o[1] << 16);
            } else {
                *reinterpret_cast<uint2*>(yo + e) = make_uint2((u32)o[0] | ((u32)o[1] << 16), (u32)o[2] | ((u32)o[3] << 16));
            }
        });
}

// f(integral_constant NL0, integral_constant NL1) for the widths the two-block kernels take; -1 otherwise.
template <class F>
int with_2b(int N, F f) {
    using std::integral_constant;
    switch (N) {
        case 1536: return f(integral_constant<int, 10>{}, integral_constant<int, 9>{});
        case 3072: return f(integral_constant<int, 11>{}, integral_constant<int, 10>{});
        case 6144: return f(integral_constant<int, 12>{}, integral_constant<int, 11>{});
        case 12288: return f(integral_constant<int, 13>{}, integral_constant<int, 12>{});
        case 1024: return f(integral_constant<int, 10>{}, integral_constant<int, 0>{});
        case 2048: return f(integral_constant<int, 11>{}, integral_constant<int, 0>{});
        case 4096: return f(integral_constant<int, 12>{}, integral_constant<int, 0>{});
        case 8192: return f(integral_constant<int, 13>{}, integral_constant<int, 0>{});
        case 16384: return f(integral_constant<int, 14>{}, integral_constant<int, 0>{});
        default: return -1;
    }
}

// The plain-MLP middle on widths of one or two power-of-two blocks, N = 2^NL0 (+ 2^NL1), whose windowed transforms
// take the same number of windows (6144 = 4096 + 2048, the DiT's; 1536, 3072, 12288; powers of two 1024 .. 16384):
// the arithmetic of k_mid1, each block's two transforms done by win_walsh on its own 2^NL / 32 threads. The two
// blocks' threads run different code that executes the same barriers the same number of times, so the barriers
// there are the unaligned form. Layer constants (sv, su, bias) are staged before the dependency wait.
template <int AT, int NL0, int NL1>
__global__ void __launch_bounds__(((1 << NL0) + (NL1 ? (1 << NL1) : 0)) / 32)
k_mid1_2b(const void* __restrict__ acc, const float* __restrict__ s, const float* __restrict__ rs, const i8* __restrict__ sv,
          const float* __restrict__ bias, const u16* __restrict__ lut, const i8* __restrict__ su, int8_t* __restrict__ q,
          int* __restrict__ q4, float* __restrict__ scale, int lda, int ldq) {
    constexpr int NLB = NL1 ? NL1 : NL0;                          // (the second block's parameters when there is one)
    constexpr int N0 = 1 << NL0, N1 = NL1 ? 1 << NL1 : 0, N = N0 + N1, T0 = N0 / 32;
    constexpr int WB0 = Win2<NL0, rot_vec<NL0>()>::WB, WB1 = Win2<NLB, rot_vec<NLB>()>::WB;
    static_assert(!NL1 || (NL1 < NL0 && Win2<NL0, rot_vec<NL0>()>::P == Win2<NLB, rot_vec<NLB>()>::P),
                  "the two blocks' transforms execute the same barriers");
    extern __shared__ __align__(16) float buf[];
    float* buf0 = buf;
    float* buf1 = buf + N0 + (N0 >> WB0);
    float* sbias = buf1 + (NL1 ? N1 + (N1 >> WB1) : 0);
    i8* ssv = reinterpret_cast<i8*>(sbias + (bias ? N : 0));
    i8* ssu = ssv + N;
    __shared__ float red[32];
    pdl_launch_dependents();
    const int t = threadIdx.x, nt = N / 32;
    for (int i = t; i < N / 16; i += nt) {
        reinterpret_cast<uint4*>(ssv)[i] = __ldg(reinterpret_cast<const uint4*>(sv) + i);
        reinterpret_cast<uint4*>(ssu)[i] = __ldg(reinterpret_cast<const uint4*>(su) + i);
    }
    if (bias)
        for (int i = t; i < N / 4; i += nt) reinterpret_cast<float4*>(sbias)[i] = __ldg(reinterpret_cast<const float4*>(bias) + i);
    __syncthreads();
    pdl_wait();
    const int tok = blockIdx.x;
    const size_t base = (size_t)tok * lda;
    const float st = s ? s[tok] : 1.f;
    float mx = 0.f;
    auto run_block = [&](auto nlc, int tb, int off, float* bb) {
        constexpr int NL = decltype(nlc)::value, V = rot_vec<NL>(), G = 1 << Win2<NL, V>::WB;
        const float sc = wscale(1 << NL);
        float v[32];
        const float* r = rs ? rs + off + 32 * tb : nullptr;
        load_scaledc<AT, 16>(acc, base + off + 32 * tb, st, r, v);
        load_scaledc<AT, 16>(acc, base + off + 32 * tb + 16, st, r ? r + 16 : nullptr, v + 16);
        win_walsh<NL, false, 1>(v, bb, tb);
#pragma unroll
        for (int qq = 0; qq < G; ++qq) {
            const int e = off + win_elem<NL>(tb, qq, 0);
#pragma unroll
            for (int k = 0; k < V; ++k) {
                float y = (v[V * qq + k] * sc) * (float)ssv[e + k];
                if (bias) y = y + sbias[e + k];
                v[V * qq + k] = bf2f(__ldg(lut + f2bf(y))) * (float)ssu[e + k];
            }
        }
        win_relayout<NL, 1>(v, bb, tb);
        win_walsh<NL, true, 1>(v, bb, tb);
        blk_sync<1>();                          // both blocks' last reads are done: buf is rewritten below
#pragma unroll
        for (int qq = 0; qq < G; ++qq) {
            const int e = off + win_elem<NL>(tb, qq, 0);
#pragma unroll
            for (int k = 0; k < V; ++k) {
                const float o = v[V * qq + k] * sc;
                buf[swz(e + k)] = o;
                mx = fmaxf(mx, fabsf(o));
            }
        }
    };
    if (t < T0) run_block(std::integral_constant<int, NL0>{}, t, 0, buf0);
    else if constexpr (NL1 != 0) run_block(std::integral_constant<int, NLB>{}, t - T0, N0, buf1);
    quantize_store(buf, mx, red, q, q4, scale, tok, N, ldq);
}

// Plain-MLP middle (kernels.py:280-292): x = lut(BF16(post(acc) + bias)) * su, block Walsh, INT8.
template <int AT, int CH>
__global__ void __launch_bounds__(512, 2) k_mid1(const void* __restrict__ acc, const float* __restrict__ s, const float* __restrict__ rs,
                                              const i8* __restrict__ sv, const float* __restrict__ bias, const u16* __restrict__ lut,
                                              const i8* __restrict__ su, int8_t* __restrict__ q, int* __restrict__ q4,
                                              float* __restrict__ scale, int M, int N, int lda, int ldq, int stage) {
    extern __shared__ __align__(16) float buf[];
    __shared__ float red[32];
    pdl_launch_dependents();
    char* sp = reinterpret_cast<char*>(buf + N);    // layer constants
    const bool on = stage != 0;
    const float* rsc = static_cast<const float*>(stage_const(sp, AT != TCQ_DT_F32 ? rs : nullptr, 4 * N, on));
    const float* biasc = static_cast<const float*>(stage_const(sp, bias, 4 * N, on));
    const i8* svc = static_cast<const i8*>(stage_const(sp, sv, N, on));
    const i8* suc = static_cast<const i8*>(stage_const(sp, su, N, on));
    __syncthreads();
    pdl_wait();
    const int tok = blockIdx.x;
    const size_t base = (size_t)tok * lda;
    const float st = s ? s[tok] : 1.f;
    row_walsh<CH>(buf, N, [&](int c, float* v) { load_scaledc<AT, CH>(acc, base + CH * c, st, rsc ? rsc + CH * c : nullptr, v); },
                  [&](int i, float v) {
                      v = v * (float)svc[i];
                      if (biasc) v = v + biasc[i];
                      buf[swz(i)] = bf2f(lut[f2bf(v)]) * (float)suc[i];
                  });
    float mx = 0.f;
    row_walshc<CH>(buf, N, [&](int c, float* v) { buf_chunk<CH>(buf, c, v); },
                   [&](int i0, const float* v) { store_chunk<CH>(buf, i0, v, mx); },
                   [&](int i, float v) { buf[swz(i)] = v; mx = fmaxf(mx, fabsf(v)); });
    quantize_store(buf, mx, red, q, q4, scale, tok, N, ldq);
}


// Per-token INT8 quantizer without rotation (the W8A8 layers of config 3 / the vision tower): x (M, K) -> q (M, K),
// scale (M,) = absmax / 127 (tcq_format.py:119-122). One block per token row; the row is read twice (max, quantize)
// and stays in L1 / L2 between the two passes.
template <int DT>
__global__ void __launch_bounds__(256) k_quant(const void* __restrict__ x, int8_t* __restrict__ q, float* __restrict__ scale, int M,
                                               int K) {
    __shared__ float red[32];
    pdl_launch_dependents();
    pdl_wait();
    const int tok = blockIdx.x;
    const size_t es = DT == TCQ_DT_F32 ? 4 : 2;
    const char* xr = reinterpret_cast<const char*>(x) + (size_t)tok * K * es;
    float mx = 0.f;
    for (int c = threadIdx.x; c < (K >> 4); c += blockDim.x) {
        float v[16];
        loadc<DT, 16>(xr + (size_t)16 * c * es, v);
#pragma unroll
        for (int k = 0; k < 16; ++k) mx = fmaxf(mx, fabsf(v[k]));
    }
    mx = block_max(mx, red);
    const float s = mx > 0.f ? mx / 127.f : 1.f, rs = 1.f / s;
    if (threadIdx.x == 0) scale[tok] = s;
    for (int c = threadIdx.x; c < (K >> 4); c += blockDim.x) {
        float v[16];
        loadc<DT, 16>(xr + (size_t)16 * c * es, v);
        u32 w[4];
#pragma unroll
        for (int g = 0; g < 4; ++g)
            w[g] = (u32)(q8(v[4 * g], s, rs) & 0xff) | ((u32)(q8(v[4 * g + 1], s, rs) & 0xff) << 8) |
                   ((u32)(q8(v[4 * g + 2], s, rs) & 0xff) << 16) | ((u32)(q8(v[4 * g + 3], s, rs) & 0xff) << 24);
        *reinterpret_cast<uint4*>(q + (size_t)tok * K + 16 * c) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// ---------------------------------------------------------------------------------------------------- host side
int threads_for(int K, int CH) {
    int t = ((K / CH) + 31) & ~31;
    if (t < 32) t = 32;
    if (t > 512) t = 512;
    return t;
}

// Elements per thread chunk of a launch of M rows of width K: 4 while the launch's threads at that chunking fit on the
// machine at once (at most `per_sm` threads per SM; each thread's instruction latency bounds such a launch, so more
// threads per row finish it sooner), 16 otherwise (more rows: throughput, fewer threads per row).
int rows_ch(int M, int K, int per_sm) {
    return (long long)M * threads_for(K, 4) <= (long long)tcq_sm_count() * per_sm ? 4 : 16;
}
constexpr int kLightPerSm = 1024;   // row kernels of at most 64 registers a thread (pre, rotate, post, middles)
constexpr int kHeavyPerSm = 512;    // row kernels with the epilogue's operands in registers (chain, post_multi)

// Threads per row of the heavy row kernels (80-96 registers a thread: one 512-thread block fills an SM's register
// file): more rows than SMs get at most 256 threads a row (two chunks a thread on the widest rows), so that two rows
// share an SM and 160 rows still run as one wave instead of two.
int heavy_threads(int M, int N, int CH) {
    const int t = threads_for(N, CH);
    return M > tcq_sm_count() && t > 256 ? 256 : t;
}

// Threads per row of the row kernels of at most 64 registers a thread (post, MLP middles): two 512-thread rows fit on
// an SM, so up to twice as many rows as SMs take the whole width's threads and still run as one wave; beyond that the
// launch is throughput-bound and rows get at most 256 threads (more chunks per thread, fewer barriers per element).
int light_threads(int M, int N, int CH) {
    const int t = threads_for(N, CH);
    return M > 2 * tcq_sm_count() && t > 256 ? 256 : t;
}

// f(std::integral_constant<int, CH>{}) for the chunk width ch (4 or 16).
template <class F>
int with_ch(int ch, F f) {
    return ch == 4 ? f(std::integral_constant<int, 4>{}) : f(std::integral_constant<int, 16>{});
}

bool width_ok(int K) { return K > 0 && (K & 15) == 0 && K <= kMaxWidth; }

template <class Kern, class... Args>
int launch(Kern kern, dim3 grid, int threads, size_t smem, void* stream, Args... args) {
    // Opt in above 46 KB of dynamic shared memory: the kernels also use up to 1 KB of static shared memory, and the
    // default per-block limit (48 KB) covers both.
    if (smem > 46 * 1024 && cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return TCQ_ERR_LAUNCH;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
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

bool acc_aligned(const void* acc, int acc_dtype, int lda, int col0) {
    const int vec = acc_dtype == TCQ_DT_BF16 ? 8 : 4;   // elements per 16 bytes
    return tcq_aligned(acc, 16) && lda % vec == 0 && col0 % vec == 0;
}

}  // namespace

namespace {
template <int NL>
int launch_rotate_p2(const void* x, int x_dtype, const int8_t* signs, void* y, bool of, int M, int inv, void* stream) {
    constexpr int WB = Win2<NL, rot_vec<NL>()>::WB;
    const size_t smem = (size_t)4 * ((1 << NL) + ((1 << NL) >> WB)) + (1 << NL);
    const int T = (1 << NL) / 32;
    auto go = [&](auto kern) { return launch(kern, dim3(M), T, smem, stream, x, (const i8*)signs, y, inv); };
    switch (x_dtype) {
        case TCQ_DT_BF16: return of ? go(k_rotate_p2<TCQ_DT_BF16, TCQ_DT_F32, NL>) : go(k_rotate_p2<TCQ_DT_BF16, TCQ_DT_BF16, NL>);
        case TCQ_DT_F16: return of ? go(k_rotate_p2<TCQ_DT_F16, TCQ_DT_F32, NL>) : go(k_rotate_p2<TCQ_DT_F16, TCQ_DT_BF16, NL>);
        case TCQ_DT_F32: return of ? go(k_rotate_p2<TCQ_DT_F32, TCQ_DT_F32, NL>) : go(k_rotate_p2<TCQ_DT_F32, TCQ_DT_BF16, NL>);
        default: return (int)TCQ_ERR_DTYPE;
    }
}

}  // namespace

extern "C" {

int tcq_abi_version(void) { return TCQ_ABI_VERSION; }

const char* tcq_status_string(int status) {
    switch (status) {
        case TCQ_OK: return "ok";
        case TCQ_ERR_SHAPE: return "unsupported shape";
        case TCQ_ERR_ALIGN: return "misaligned pointer or leading dimension (16-byte alignment required)";
        case TCQ_ERR_DTYPE: return "unknown dtype";
        case TCQ_ERR_ARG: return "invalid argument";
        case TCQ_ERR_LAUNCH: return "CUDA launch failed";
        case TCQ_ERR_DEVICE: return "no usable sm_100 device";
        case TCQ_ERR_WORKSPACE: return "workspace missing or too small";
        default: return "unknown status";
    }
}


int tcq_quantize(const void* x, int x_dtype, int8_t* q, float* scale, int M, int K, void* stream) {
    if (!x || !q || !scale) return TCQ_ERR_ARG;
    if (M <= 0 || K <= 0 || (K & 15)) return TCQ_ERR_SHAPE;
    if (!tcq_aligned(x, 16) || !tcq_aligned(q, 16)) return TCQ_ERR_ALIGN;
    int T = ((K >> 4) + 31) & ~31;
    if (T > 256) T = 256;
    switch (x_dtype) {
        case TCQ_DT_BF16: return launch(k_quant<TCQ_DT_BF16>, dim3(M), T, 0, stream, x, q, scale, M, K);
        case TCQ_DT_F16: return launch(k_quant<TCQ_DT_F16>, dim3(M), T, 0, stream, x, q, scale, M, K);
        case TCQ_DT_F32: return launch(k_quant<TCQ_DT_F32>, dim3(M), T, 0, stream, x, q, scale, M, K);
        default: return TCQ_ERR_DTYPE;
    }
}

int tcq_pre(const void* x, int x_dtype, const int8_t* su, int8_t* q, int32_t* q4, float* scale, int M, int K, int ldq,
            void* stream) {
    if (!x || !su || !scale || (!q && !q4)) return TCQ_ERR_ARG;
    if (M <= 0 || !width_ok(K)) return TCQ_ERR_SHAPE;
    if (q4 && ldq < M) return TCQ_ERR_ARG;
    if (!tcq_aligned(x, 16) || !tcq_aligned(su, 16) || (q && !tcq_aligned(q, 16))) return TCQ_ERR_ALIGN;
    // Widths of one or two power-of-two blocks in a latency-bound launch: the register-window transform (k_pre_2b).
    if (M <= 2 * tcq_sm_count() && (x_dtype == TCQ_DT_BF16 || x_dtype == TCQ_DT_F16 || x_dtype == TCQ_DT_F32)) {
        const int e = with_2b(K, [&](auto n0, auto n1) {
            constexpr int NL0 = decltype(n0)::value, NL1 = decltype(n1)::value;
            constexpr int T = ((1 << NL0) + (NL1 ? (1 << NL1) : 0)) / 32;
            const size_t sm = (size_t)4 * row2b_floats<NL0, NL1>();
            auto kern = x_dtype == TCQ_DT_BF16 ? k_pre_2b<TCQ_DT_BF16, NL0, NL1>
                        : x_dtype == TCQ_DT_F16 ? k_pre_2b<TCQ_DT_F16, NL0, NL1> : k_pre_2b<TCQ_DT_F32, NL0, NL1>;
            return launch(kern, dim3(M), T, sm, stream, x, (const i8*)su, q, (int*)q4, scale, ldq);
        });
        if (e >= 0) return e;
    }
    const size_t smem = (size_t)4 * K;
    return with_ch(rows_ch(M, K, kLightPerSm), [&](auto C) {
        constexpr int CH = decltype(C)::value;
        const int T = threads_for(K, CH);
        switch (x_dtype) {
            case TCQ_DT_BF16: return launch(k_pre<TCQ_DT_BF16, CH>, dim3(M), T, smem, stream, x, (const i8*)su, q, (int*)q4, scale, M, K, ldq);
            case TCQ_DT_F16: return launch(k_pre<TCQ_DT_F16, CH>, dim3(M), T, smem, stream, x, (const i8*)su, q, (int*)q4, scale, M, K, ldq);
            case TCQ_DT_F32: return launch(k_pre<TCQ_DT_F32, CH>, dim3(M), T, smem, stream, x, (const i8*)su, q, (int*)q4, scale, M, K, ldq);
            default: return (int)TCQ_ERR_DTYPE;
        }
    });
}

int tcq_pre2(const uint16_t* g, const uint16_t* u, const int8_t* su, int8_t* q, int32_t* q4, float* scale, int M, int K,
             int ldq, void* stream) {
    if (!g || !u || !su || !scale || (!q && !q4)) return TCQ_ERR_ARG;
    if (M <= 0 || !width_ok(K)) return TCQ_ERR_SHAPE;
    if (q4 && ldq < M) return TCQ_ERR_ARG;
    if (!tcq_aligned(g, 16) || !tcq_aligned(u, 16) || !tcq_aligned(su, 16) || (q && !tcq_aligned(q, 16))) return TCQ_ERR_ALIGN;
    return with_ch(rows_ch(M, K, kLightPerSm), [&](auto C) {
        constexpr int CH = decltype(C)::value;
        return launch(k_pre2<CH>, dim3(M), threads_for(K, CH), (size_t)4 * K, stream, (const u16*)g, (const u16*)u, (const i8*)su,
                      q, (int*)q4, scale, M, K, ldq);
    });
}

int tcq_pre_h(const void* x, int x_dtype, const int8_t* su, uint16_t* h, uint16_t* hT, int M, int K, int ldh, void* stream) {
    if (!x || !su || (!h && !hT)) return TCQ_ERR_ARG;
    if (M <= 0 || !width_ok(K)) return TCQ_ERR_SHAPE;
    if (hT && ldh < M) return TCQ_ERR_ARG;
    if (!tcq_aligned(x, 16) || !tcq_aligned(su, 16)) return TCQ_ERR_ALIGN;
    const size_t smem = (size_t)4 * K;
    return with_ch(rows_ch(M, K, kLightPerSm), [&](auto C) {
        constexpr int CH = decltype(C)::value;
        const int T = threads_for(K, CH);
        switch (x_dtype) {
            case TCQ_DT_BF16: return launch(k_pre_h<TCQ_DT_BF16, CH>, dim3(M), T, smem, stream, x, (const i8*)su, (u16*)h, (u16*)hT, M, K, ldh);
            case TCQ_DT_F16: return launch(k_pre_h<TCQ_DT_F16, CH>, dim3(M), T, smem, stream, x, (const i8*)su, (u16*)h, (u16*)hT, M, K, ldh);
            case TCQ_DT_F32: return launch(k_pre_h<TCQ_DT_F32, CH>, dim3(M), T, smem, stream, x, (const i8*)su, (u16*)h, (u16*)hT, M, K, ldh);
            default: return (int)TCQ_ERR_DTYPE;
        }
    });
}

int tcq_rotate(const void* x, int x_dtype, const int8_t* signs, void* y, int y_dtype, int M, int D, int inverse,
               void* stream) {
    if (!x || !signs || !y) return TCQ_ERR_ARG;
    if (M <= 0 || !width_ok(D)) return TCQ_ERR_SHAPE;
    if (!tcq_aligned(x, 16) || !tcq_aligned(signs, 16)) return TCQ_ERR_ALIGN;
    const size_t smem = (size_t)4 * D;
    const int inv = inverse ? 1 : 0;
    if (y_dtype != TCQ_DT_F32 && y_dtype != TCQ_DT_BF16) return TCQ_ERR_DTYPE;
    if (!tcq_aligned(y, 16)) return TCQ_ERR_ALIGN;
    const bool of = y_dtype == TCQ_DT_F32;
    switch (D) {                                           // power-of-two widths: the register-window kernel
        case 1024: return launch_rotate_p2<10>(x, x_dtype, signs, y, of, M, inv, stream);
        case 2048: return launch_rotate_p2<11>(x, x_dtype, signs, y, of, M, inv, stream);
        case 4096: return launch_rotate_p2<12>(x, x_dtype, signs, y, of, M, inv, stream);
        case 8192: return launch_rotate_p2<13>(x, x_dtype, signs, y, of, M, inv, stream);
        case 16384: return launch_rotate_p2<14>(x, x_dtype, signs, y, of, M, inv, stream);
        default: break;
    }
    return with_ch(rows_ch(M, D, kLightPerSm), [&](auto C) {
        constexpr int CH = decltype(C)::value;
        const int T = threads_for(D, CH);
        switch (x_dtype) {
            case TCQ_DT_BF16:
                return of ? launch(k_rotate<TCQ_DT_BF16, TCQ_DT_F32, CH>, dim3(M), T, smem, stream, x, (const i8*)signs, y, M, D, inv)
                          : launch(k_rotate<TCQ_DT_BF16, TCQ_DT_BF16, CH>, dim3(M), T, smem, stream, x, (const i8*)signs, y, M, D, inv);
            case TCQ_DT_F16:
                return of ? launch(k_rotate<TCQ_DT_F16, TCQ_DT_F32, CH>, dim3(M), T, smem, stream, x, (const i8*)signs, y, M, D, inv)
                          : launch(k_rotate<TCQ_DT_F16, TCQ_DT_BF16, CH>, dim3(M), T, smem, stream, x, (const i8*)signs, y, M, D, inv);
            case TCQ_DT_F32:
                return of ? launch(k_rotate<TCQ_DT_F32, TCQ_DT_F32, CH>, dim3(M), T, smem, stream, x, (const i8*)signs, y, M, D, inv)
                          : launch(k_rotate<TCQ_DT_F32, TCQ_DT_BF16, CH>, dim3(M), T, smem, stream, x, (const i8*)signs, y, M, D, inv);
            default: return (int)TCQ_ERR_DTYPE;
        }
    });
}

int tcq_post(const void* acc, int acc_dtype, const float* s, const float* rs, const int8_t* sv, const float* bias,
             uint16_t* y, int M, int N, int lda, int col0, void* stream) {
    if (!acc || !sv || !y) return TCQ_ERR_ARG;
    if (acc_dtype == TCQ_DT_I32 && (!s || !rs)) return TCQ_ERR_ARG;
    if (acc_dtype == TCQ_DT_BF16 && !rs) return TCQ_ERR_ARG;
    if (M <= 0 || !width_ok(N) || col0 < 0 || lda < col0 + N) return TCQ_ERR_SHAPE;
    if (!acc_aligned(acc, acc_dtype, lda, col0) || (rs && !tcq_aligned(rs, 16))) return TCQ_ERR_ALIGN;
    // Widths of one or two power-of-two blocks in a latency-bound launch: the register-window transform (k_post_2b).
    if (M <= 2 * tcq_sm_count() && (acc_dtype == TCQ_DT_I32 || acc_dtype == TCQ_DT_F32) && tcq_aligned(sv, 16) &&
        (!bias || tcq_aligned(bias, 16)) && tcq_aligned(y, 16)) {
        const int e = with_2b(N, [&](auto n0, auto n1) {
            constexpr int NL0 = decltype(n0)::value, NL1 = decltype(n1)::value;
            constexpr int NN = (1 << NL0) + (NL1 ? (1 << NL1) : 0);
            const size_t sm = (size_t)4 * row2b_floats<NL0, NL1>() + (bias ? (size_t)4 * NN : 0) + NN;
            auto kern = acc_dtype == TCQ_DT_I32 ? k_post_2b<TCQ_DT_I32, NL0, NL1> : k_post_2b<TCQ_DT_F32, NL0, NL1>;
            return launch(kern, dim3(M), NN / 32, sm, stream, acc, s, rs, (const i8*)sv, bias, (u16*)y, lda, col0);
        });
        if (e >= 0) return e;
    }
    // Staged layer constants (as k_post stages them): rs (I32 / BF16 accumulators), bias, sv.
    const size_t cb = (size_t)(acc_dtype != TCQ_DT_F32 && rs ? 4 * N : 0) + (bias ? 4 * N : 0) + N;
    const int st = tcq_stage_rows(M, cb, kStageMaxBytes);
    const size_t smem = (size_t)4 * N + (st ? cb : 0);
    return with_ch(rows_ch(M, N, kLightPerSm), [&](auto C) {
        constexpr int CH = decltype(C)::value;
        const int T = light_threads(M, N, CH);
        switch (acc_dtype) {
            case TCQ_DT_I32: return launch(k_post<TCQ_DT_I32, CH>, dim3(M), T, smem, stream, acc, s, rs, (const i8*)sv, bias, (u16*)y, M, N, lda, col0, st);
            case TCQ_DT_F32: return launch(k_post<TCQ_DT_F32, CH>, dim3(M), T, smem, stream, acc, s, rs, (const i8*)sv, bias, (u16*)y, M, N, lda, col0, st);
            case TCQ_DT_BF16: return launch(k_post<TCQ_DT_BF16, CH>, dim3(M), T, smem, stream, acc, s, rs, (const i8*)sv, bias, (u16*)y, M, N, lda, col0, st);
            default: return (int)TCQ_ERR_DTYPE;
        }
    });
}

int tcq_chain(const void* acc, int acc_dtype, const float* s, const float* rs, const int8_t* sv, const float* bias, int lda,
              int col0, const uint16_t* y, const uint16_t* x, uint16_t* h, uint16_t* n, const void* w, const void* b,
              int wb_dtype, const uint16_t* mod_scale, const uint16_t* mod_shift, int mod_rows, int ld_mod, float eps,
              int kind, const int8_t* su, int8_t* q, int32_t* q4, float* scale, int ldq, int M, int N, void* stream) {
    if (!x || (acc && y) || (!n && !su && !q && !q4) || (!mod_scale != !mod_shift)) return TCQ_ERR_ARG;
    if (kind != 0 && kind != 1) return TCQ_ERR_ARG;
    if (wb_dtype != TCQ_DT_F32 && wb_dtype != TCQ_DT_BF16) return TCQ_ERR_DTYPE;
    if (M <= 0 || !width_ok(N)) return TCQ_ERR_SHAPE;
    if (acc) {
        if (!sv) return TCQ_ERR_ARG;
        if (acc_dtype != TCQ_DT_I32 && acc_dtype != TCQ_DT_F32) return TCQ_ERR_DTYPE;
        if (acc_dtype == TCQ_DT_I32 && (!s || !rs)) return TCQ_ERR_ARG;
        if (col0 < 0 || lda < col0 + N) return TCQ_ERR_SHAPE;
        if (!acc_aligned(acc, acc_dtype, lda, col0) || (rs && !tcq_aligned(rs, 16))) return TCQ_ERR_ALIGN;
    }
    if ((su || q || q4) && (!scale || (!q && !q4) || (q4 && ldq < M))) return TCQ_ERR_ARG;
    if (mod_scale && (mod_rows <= 0 || ld_mod < N)) return TCQ_ERR_ARG;
    if (!tcq_aligned(x, 16) || (y && !tcq_aligned(y, 16)) || (h && !tcq_aligned(h, 16)) || (n && !tcq_aligned(n, 16)) ||
        (su && !tcq_aligned(su, 16)) || (q && !tcq_aligned(q, 16)))
        return TCQ_ERR_ALIGN;
    // Chunks of 4 for a few rows up to 2048 wide (the norm's sum order does not depend on the chunking), else 16.
    const bool c4 = N <= 2048 && rows_ch(M, N, kHeavyPerSm) == 4;
    const int T = norm_threads(N, c4 ? 4 : 16);
    const bool wb = wb_dtype == TCQ_DT_BF16, i32 = acc && acc_dtype == TCQ_DT_I32;
    // Layer constants staged by the kernel (the same set, in bytes): rs (I32 accumulators), bias, sv, w, b, su.
    const size_t cb = (acc ? (size_t)(i32 ? 4 * N : 0) + (bias ? 4 * N : 0) + N : 0) + (size_t)(w ? 1 : 0) * (wb ? 2 : 4) * N +
                      (size_t)(b ? 1 : 0) * (wb ? 2 : 4) * N + (su ? N : 0);
    // With staging on, also the copy area of x (and y, the two modulation vectors) for the first chunks.
    const size_t pb = (size_t)2 * N * (1 + (!acc && y ? 1 : 0) + (mod_scale ? 2 : 0));
    const int stage = tcq_stage_rows(M, cb, kStageMaxBytes) && (size_t)6 * N + cb + pb <= (size_t)kStageMaxSmem;
    const size_t smem = (size_t)6 * N + (stage ? cb + pb : 0);
    auto pick = [&](auto k0, auto k1, auto k2) { return c4 ? k0 : N <= 8192 ? k1 : k2; };
#define TCQ_CHAIN(AT_, K_, WB_) \
    pick(k_chain<AT_, K_, WB_, 1, 4>, k_chain<AT_, K_, WB_, 1, 16>, k_chain<AT_, K_, WB_, kNormMaxChunks, 16>)
    auto kern = kind == 0 ? (i32 ? (wb ? TCQ_CHAIN(TCQ_DT_I32, 0, true) : TCQ_CHAIN(TCQ_DT_I32, 0, false))
                                 : (wb ? TCQ_CHAIN(TCQ_DT_F32, 0, true) : TCQ_CHAIN(TCQ_DT_F32, 0, false)))
                          : (i32 ? (wb ? TCQ_CHAIN(TCQ_DT_I32, 1, true) : TCQ_CHAIN(TCQ_DT_I32, 1, false))
                                 : (wb ? TCQ_CHAIN(TCQ_DT_F32, 1, true) : TCQ_CHAIN(TCQ_DT_F32, 1, false)));
#undef TCQ_CHAIN
    return launch(kern, dim3(M), T, smem, stream, acc, s, rs, (const i8*)sv, bias, lda, col0, (const u16*)y, (const u16*)x,
                  (u16*)h, (u16*)n, w, b, (const u16*)mod_scale, (const u16*)mod_shift, mod_rows, ld_mod, eps, (const i8*)su, q,
                  (int*)q4, scale, ldq, N, stage);
}

static int post_multi(const void* acc, int acc_dtype, const float* s, const float* rs, const int8_t* sv, const float* bias,
                      const uint16_t* lut, uint16_t* y0, uint16_t* y1, uint16_t* y2, int M, int n0, int n1, int n2, int lda,
                      int act0, int per_layer_blocks, void* stream) {
    if (!acc || !sv || !y0) return TCQ_ERR_ARG;
    if (acc_dtype == TCQ_DT_I32 && (!s || !rs)) return TCQ_ERR_ARG;
    if (acc_dtype == TCQ_DT_BF16 && !rs) return TCQ_ERR_ARG;
    if (act0 && !lut) return TCQ_ERR_ARG;
    if ((n1 && !y1) || (n2 && !y2)) return TCQ_ERR_ARG;
    if (M <= 0 || !width_ok(n0) || (n1 && !width_ok(n1)) || (n2 && !width_ok(n2)) || n1 < 0 || n2 < 0) return TCQ_ERR_SHAPE;
    if (n2 && !n1) return TCQ_ERR_SHAPE;
    if (lda < n0 + n1 + n2) return TCQ_ERR_SHAPE;
    if (!acc_aligned(acc, acc_dtype, lda, 0) || (rs && !tcq_aligned(rs, 16))) return TCQ_ERR_ALIGN;
    const int nmax = n0 > n1 ? (n0 > n2 ? n0 : n2) : (n1 > n2 ? n1 : n2);
    const int layers = 1 + (n1 > 0) + (n2 > 0);
    const dim3 grid(M, per_layer_blocks ? layers : 1);
    // Staged layer constants of a block's columns (at most all n0 + n1 + n2 of them): rs, bias, sv.
    const size_t ntot = (size_t)n0 + n1 + n2;
    const size_t cb = ntot * ((acc_dtype != TCQ_DT_F32 && rs ? 4 : 0) + (bias ? 4 : 0) + 1);
    const int st = tcq_stage_rows(M, cb, kStageMaxBytes);
    const size_t smem = (size_t)4 * nmax + (st ? cb : 0);
    return with_ch(rows_ch(M * (int)grid.y, nmax, kHeavyPerSm), [&](auto C) {
        constexpr int CH = decltype(C)::value;
        const int T = heavy_threads(M * (int)grid.y, nmax, CH);
        switch (acc_dtype) {
            case TCQ_DT_I32: return launch(k_post_multi<TCQ_DT_I32, CH>, grid, T, smem, stream, acc, s, rs, (const i8*)sv, bias, (const u16*)lut, (u16*)y0, (u16*)y1, (u16*)y2, M, n0, n1, n2, lda, act0, nmax, st);
            case TCQ_DT_F32: return launch(k_post_multi<TCQ_DT_F32, CH>, grid, T, smem, stream, acc, s, rs, (const i8*)sv, bias, (const u16*)lut, (u16*)y0, (u16*)y1, (u16*)y2, M, n0, n1, n2, lda, act0, nmax, st);
            case TCQ_DT_BF16: return launch(k_post_multi<TCQ_DT_BF16, CH>, grid, T, smem, stream, acc, s, rs, (const i8*)sv, bias, (const u16*)lut, (u16*)y0, (u16*)y1, (u16*)y2, M, n0, n1, n2, lda, act0, nmax, st);
            default: return (int)TCQ_ERR_DTYPE;
        }
    });
}

int tcq_post3(const void* acc, int acc_dtype, const float* s, const float* rs, const int8_t* sv, const float* bias,
              uint16_t* y0, uint16_t* y1, uint16_t* y2, int M, int n0, int n1, int n2, int lda, void* stream) {
    return post_multi(acc, acc_dtype, s, rs, sv, bias, nullptr, y0, y1, y2, M, n0, n1, n2, lda, 0, 0, stream);
}

int tcq_postg(const void* acc, int acc_dtype, const float* s, const float* rs, const int8_t* sv, const float* bias,
              const uint16_t* lut, uint16_t* y0, uint16_t* y1, uint16_t* y2, int M, int n0, int n1, int n2, int lda, int act0,
              void* stream) {
    return post_multi(acc, acc_dtype, s, rs, sv, bias, lut, y0, y1, y2, M, n0, n1, n2, lda, act0, 1, stream);
}

int tcq_mid2(const void* acc, int acc_dtype, const float* s, const float* rs, const int8_t* sv, const uint16_t* lut,
             const int8_t* su, int8_t* q, int32_t* q4, float* scale, int M, int N, int lda, int ldq, void* stream) {
    if (!acc || !sv || !lut || !su || !scale || (!q && !q4)) return TCQ_ERR_ARG;
    if (acc_dtype == TCQ_DT_I32 && (!s || !rs)) return TCQ_ERR_ARG;
    if (acc_dtype == TCQ_DT_BF16 && !rs) return TCQ_ERR_ARG;
    if (M <= 0 || !width_ok(N) || lda < 2 * N) return TCQ_ERR_SHAPE;
    if (q4 && ldq < M) return TCQ_ERR_ARG;
    if (!acc_aligned(acc, acc_dtype, lda, N) || (rs && !tcq_aligned(rs, 16)) || !tcq_aligned(su, 16) || (q && !tcq_aligned(q, 16)))
        return TCQ_ERR_ALIGN;
    // Power-of-two widths in a latency-bound launch (at most two rows per SM; sv 16-byte aligned): the register-window transforms
    // (k_mid2_p2), one row of N / 32 threads per block. Many-row launches keep k_mid2, whose 64 registers a thread let
    // twice as many rows share an SM.
    if ((N & (N - 1)) == 0 && N >= 1024 && N <= 16384 && (acc_dtype == TCQ_DT_I32 || acc_dtype == TCQ_DT_F32) &&
        M <= 2 * tcq_sm_count() && tcq_aligned(sv, 16)) {
        auto go = [&](auto nl) {
            constexpr int NL = decltype(nl)::value;
            constexpr int WB = Win2<NL, rot_vec<NL>()>::WB;
            const size_t smem = (size_t)4 * ((1 << NL) + ((1 << NL) >> WB)) + 3 * (1 << NL);   // + staged sv, su
            auto kern = acc_dtype == TCQ_DT_I32 ? k_mid2_p2<TCQ_DT_I32, NL> : k_mid2_p2<TCQ_DT_F32, NL>;
            return launch(kern, dim3(M), (1 << NL) / 32, smem, stream, acc, s, rs, (const i8*)sv, (const u16*)lut, (const i8*)su, q,
                          (int*)q4, scale, lda, ldq);
        };
        switch (N) {
            case 1024: return go(std::integral_constant<int, 10>{});
            case 2048: return go(std::integral_constant<int, 11>{});
            case 4096: return go(std::integral_constant<int, 12>{});
            case 8192: return go(std::integral_constant<int, 13>{});
            default: return go(std::integral_constant<int, 14>{});
        }
    }
    // Staged layer constants (as k_mid2 stages them): rs of both layers (I32 / BF16 accumulators), sv of both, su.
    const size_t cb = (size_t)(acc_dtype != TCQ_DT_F32 && rs ? 8 * N : 0) + 2 * N + N;
    const int st = tcq_stage_rows(M, cb, kStageMaxBytes);
    const size_t smem = (size_t)6 * N + (st ? cb : 0);
    return with_ch(rows_ch(M, N, kLightPerSm), [&](auto C) {
        constexpr int CH = decltype(C)::value;
        const int T = light_threads(M, N, CH);
        switch (acc_dtype) {
            case TCQ_DT_I32: return launch(k_mid2<TCQ_DT_I32, CH>, dim3(M), T, smem, stream, acc, s, rs, (const i8*)sv, (const u16*)lut, (const i8*)su, q, (int*)q4, scale, M, N, lda, ldq, st);
            case TCQ_DT_F32: return launch(k_mid2<TCQ_DT_F32, CH>, dim3(M), T, smem, stream, acc, s, rs, (const i8*)sv, (const u16*)lut, (const i8*)su, q, (int*)q4, scale, M, N, lda, ldq, st);
            case TCQ_DT_BF16: return launch(k_mid2<TCQ_DT_BF16, CH>, dim3(M), T, smem, stream, acc, s, rs, (const i8*)sv, (const u16*)lut, (const i8*)su, q, (int*)q4, scale, M, N, lda, ldq, st);
            default: return (int)TCQ_ERR_DTYPE;
        }
    });
}

int tcq_mid1(const void* acc, int acc_dtype, const float* s, const float* rs, const int8_t* sv, const float* bias,
             const uint16_t* lut, const int8_t* su, int8_t* q, int32_t* q4, float* scale, int M, int N, int lda, int ldq,
             void* stream) {
    if (!acc || !sv || !lut || !su || !scale || (!q && !q4)) return TCQ_ERR_ARG;
    if (acc_dtype == TCQ_DT_I32 && (!s || !rs)) return TCQ_ERR_ARG;
    if (acc_dtype == TCQ_DT_BF16 && !rs) return TCQ_ERR_ARG;
    if (M <= 0 || !width_ok(N) || lda < N) return TCQ_ERR_SHAPE;
    if (q4 && ldq < M) return TCQ_ERR_ARG;
    if (!acc_aligned(acc, acc_dtype, lda, 0) || (rs && !tcq_aligned(rs, 16)) || !tcq_aligned(su, 16) || (q && !tcq_aligned(q, 16)))
        return TCQ_ERR_ALIGN;
    // Widths of one or two power-of-two blocks with equal window counts, in a latency-bound launch (at most two rows
    // per SM): the register-window transforms (k_mid1_2b).
    if ((acc_dtype == TCQ_DT_I32 || acc_dtype == TCQ_DT_F32) && M <= 2 * tcq_sm_count() && tcq_aligned(sv, 16) &&
        (!bias || tcq_aligned(bias, 16))) {
        auto go = [&](auto n0, auto n1) {
            constexpr int NL0 = decltype(n0)::value, NL1 = decltype(n1)::value, NLB = NL1 ? NL1 : NL0;
            constexpr int NN = (1 << NL0) + (NL1 ? 1 << NL1 : 0);
            const size_t smem = (size_t)4 * ((1 << NL0) + ((1 << NL0) >> Win2<NL0, rot_vec<NL0>()>::WB)) +
                                (NL1 ? (size_t)4 * ((1 << NLB) + ((1 << NLB) >> Win2<NLB, rot_vec<NLB>()>::WB)) : 0) +
                                (bias ? (size_t)4 * NN : 0) + 2 * (size_t)NN;
            auto kern = acc_dtype == TCQ_DT_I32 ? k_mid1_2b<TCQ_DT_I32, NL0, NL1> : k_mid1_2b<TCQ_DT_F32, NL0, NL1>;
            return launch(kern, dim3(M), NN / 32, smem, stream, acc, s, rs, (const i8*)sv, bias, (const u16*)lut, (const i8*)su, q,
                          (int*)q4, scale, lda, ldq);
        };
        using std::integral_constant;
        switch (N) {
            case 1536: return go(integral_constant<int, 10>{}, integral_constant<int, 9>{});
            case 3072: return go(integral_constant<int, 11>{}, integral_constant<int, 10>{});
            case 6144: return go(integral_constant<int, 12>{}, integral_constant<int, 11>{});
            case 12288: return go(integral_constant<int, 13>{}, integral_constant<int, 12>{});
            case 1024: return go(integral_constant<int, 10>{}, integral_constant<int, 0>{});
            case 2048: return go(integral_constant<int, 11>{}, integral_constant<int, 0>{});
            case 4096: return go(integral_constant<int, 12>{}, integral_constant<int, 0>{});
            case 8192: return go(integral_constant<int, 13>{}, integral_constant<int, 0>{});
            case 16384: return go(integral_constant<int, 14>{}, integral_constant<int, 0>{});
            default: break;
        }
    }
    // Staged layer constants (as k_mid1 stages them): rs (I32 / BF16 accumulators), bias, sv, su.
    const size_t cb = (size_t)(acc_dtype != TCQ_DT_F32 && rs ? 4 * N : 0) + (bias ? 4 * N : 0) + N + N;
    const int st = tcq_stage_rows(M, cb, kStageMaxBytes);
    const size_t smem = (size_t)4 * N + (st ? cb : 0);
    return with_ch(rows_ch(M, N, kLightPerSm), [&](auto C) {
        constexpr int CH = decltype(C)::value;
        const int T = light_threads(M, N, CH);
        switch (acc_dtype) {
            case TCQ_DT_I32: return launch(k_mid1<TCQ_DT_I32, CH>, dim3(M), T, smem, stream, acc, s, rs, (const i8*)sv, bias, (const u16*)lut, (const i8*)su, q, (int*)q4, scale, M, N, lda, ldq, st);
            case TCQ_DT_F32: return launch(k_mid1<TCQ_DT_F32, CH>, dim3(M), T, smem, stream, acc, s, rs, (const i8*)sv, bias, (const u16*)lut, (const i8*)su, q, (int*)q4, scale, M, N, lda, ldq, st);
            case TCQ_DT_BF16: return launch(k_mid1<TCQ_DT_BF16, CH>, dim3(M), T, smem, stream, acc, s, rs, (const i8*)sv, bias, (const u16*)lut, (const i8*)su, q, (int*)q4, scale, M, N, lda, ldq, st);
            default: return (int)TCQ_ERR_DTYPE;
        }
    });
}

}  // extern "C"
