// Shared device helpers of the sm_100a trellis-coded W2A8 kernels.
//
// Bit-exactness contract (the same as the reference definition, deploy/tcq_kernels/tcq_format.py and kernels.py:8-10):
// FP32 butterflies in stage order h = 1, 2, 4, ... with (a + b, a - b) pairs, block scale as an FP32 multiply by
// (float)(1 / sqrt((double)w)), true FP32 division and round-half-even in the activation quantizer, the product
// epilogue ((float)acc * s) * rs, BF16 by round-to-nearest-even. Every file is compiled with -fmad=false, so no
// a * b + c is contracted into an FMA.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "../../include/tcq_b200.h"

typedef unsigned short u16;
typedef unsigned int u32;
typedef signed char i8;
typedef unsigned long long u64;

#define TCQ_HD __device__ __forceinline__

// ---------------------------------------------------------------------------------------------------- BF16 / FP16
TCQ_HD float bf2f(u16 b) { return __uint_as_float(((u32)b) << 16); }

// FP32 -> BF16, round to nearest even; NaN -> 0x7fc0 (the c10::BFloat16 scalar rule, kernels.py:20-25).
TCQ_HD u16 f2bf(float f) {
    u32 u = __float_as_uint(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (u16)0x7fc0;
    u += 0x7fffu + ((u >> 16) & 1u);
    return (u16)(u >> 16);
}

// Two values at once: the hardware round-to-nearest-even conversion (identical to f2bf for every non-NaN input,
// infinities, overflow to infinity and subnormals included), lo in the low half; a pair holding a NaN is redone with
// f2bf for the NaN rule.
TCQ_HD u32 f2bf2(float lo, float hi) {
    u32 r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    if (lo != lo || hi != hi) r = (u32)f2bf(lo) | ((u32)f2bf(hi) << 16);
    return r;
}

// Two 16-byte stores of 8 packed words (p 16-byte aligned: global or shared).
TCQ_HD void store16_bf16(u16* p, const u32* w) {
    uint4* u = reinterpret_cast<uint4*>(p);
    u[0] = make_uint4(w[0], w[1], w[2], w[3]);
    u[1] = make_uint4(w[4], w[5], w[6], w[7]);
}

TCQ_HD float h2f(u16 h) {
    float f;
    asm("{ .reg .b16 t; mov.b16 t, %1; cvt.f32.f16 %0, t; }" : "=f"(f) : "h"(h));
    return f;
}

// ---------------------------------------------------------------------------------------------------- Walsh helpers
// FP32 block scale of a power-of-two width w = 2^k: (float)(1 / sqrt((double)w)) (tcq_format.py:36-41), built from
// its bits instead of FP64 arithmetic. Even k: exactly 2^(-k/2). Odd k: sqrt((double)2^k) = 2^((k-1)/2) * RN(sqrt 2)
// and the quotient and the FP32 rounding scale by the same power of two, so the result is (float)(1 / sqrt(2.0)) =
// 0x3F3504F3 (the FP32 rounding of 0.70710678...) times 2^(-(k-1)/2): its exponent field lowered by (k - 1) / 2.
TCQ_HD float wscale(int w) {
#ifdef __CUDA_ARCH__
    const int k = 31 - __clz(w);
#else
    const int k = 31 - __builtin_clz((unsigned)w);
#endif
    const u32 b = (k & 1) ? 0x3F3504F3u - ((u32)(k >> 1) << 23) : (127u - (u32)(k >> 1)) << 23;
#ifdef __CUDA_ARCH__
    return __uint_as_float(b);
#else
    float f;
    memcpy(&f, &b, 4);
    return f;
#endif
}

// R radix-2 stages on 2^R values in registers: stage s pairs slot k with k + 2^s, low slot gets a + b, high slot a - b.
template <int R>
TCQ_HD void bfly(float* v) {
#pragma unroll
    for (int s = 0; s < R; ++s) {
        const int hh = 1 << s;
#pragma unroll
        for (int k = 0; k < (1 << R); ++k)
            if (!(k & hh)) {
                const float a = v[k], b = v[k + hh];
                v[k] = a + b;
                v[k + hh] = a - b;
            }
    }
}

// Width of the power-of-two block of a row of width K (K % 16 == 0, descending binary decomposition) that contains
// index i < K: the highest bit in which i and K differ (i agrees with K above it and has a 0 there).
TCQ_HD int block_of(int i, int K) { return 1 << (31 - __clz(i ^ K)); }

// Shared-memory layout of a row being transformed: element i lives at swz(i). The XOR permutes the four 16-byte
// granules of each 16-element chunk so that 32 lanes storing 16 contiguous floats each (4 x st.shared.v4) hit all 32
// banks; 32 consecutive indices still map to 32 distinct banks.
TCQ_HD int swz(int i) { return i ^ (((i >> 5) & 3) << 2); }

// ---------------------------------------------------------------------------------------------------- division
// Exact n / d for 0 <= n < 2^31 by a multiply-high and a shift (Granlund and Montgomery, "Division by invariant
// integers using multiplication", 1994): with l = ceil(log2 d) and m = ceil(2^(31+l) / d) < 2^32, the error of
// n * m / 2^(31+l) against n / d stays below 1/d as long as n * d < 2^(31+l), which n < 2^31 guarantees.
struct FastDiv {
    unsigned d, m, sh;    // d == 1: the identity
};

static inline FastDiv make_fastdiv(unsigned d) {
    FastDiv f{d, 0u, 0u};
    if (d > 1) {
        int l = 0;
        while ((1ull << l) < d) ++l;
        f.m = (unsigned)(((1ull << (31 + l)) + d - 1) / d);
        f.sh = (unsigned)(l - 1);
    }
    return f;
}

TCQ_HD unsigned fdiv(unsigned n, const FastDiv& f) { return f.d == 1 ? n : __umulhi(n, f.m) >> f.sh; }

// ---------------------------------------------------------------------------------------------------- loads
// L2 eviction priorities of the decode kernels' two kinds of input: the weight stream is read once per launch (evict
// first); the per-layer 1 KB decode tables are read by every CTA of every launch of their layer (evict last), so they
// stay in L2 while the weight streams of the layers in between pass through.
TCQ_HD u64 l2_evict_first() {
    u64 pol;
    asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
TCQ_HD u64 l2_evict_last() {
    u64 pol;
    asm("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// Streaming load of the weight stream: no L1 allocation, L2 evict-first.
TCQ_HD uint4 ldg_stream_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p), "l"(l2_evict_first()));
    return r;
}

// Load of a decode table: L2 evict-last.
TCQ_HD uint4 ldg_table_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p), "l"(l2_evict_last()));
    return r;
}

// Bulk prefetch of [p, p + bytes) into L2 (no register or shared-memory destination); p and bytes multiples of 16.
TCQ_HD void prefetch_l2_bulk(const void* p, unsigned bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// ---------------------------------------------------------------------------------------------------- PDL
// Programmatic dependent launch: a kernel launched with the programmatic-serialization attribute may start while its
// predecessor drains; it must call pdl_wait() before touching anything the predecessor writes.
TCQ_HD void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
TCQ_HD void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

// Asynchronous 16-byte global -> shared copy (L2 only), both addresses 16-byte aligned; the issuing thread sees the
// data after cp_async_wait_all() (other threads after a block barrier as well).
TCQ_HD void cp_async16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((u32)__cvta_generic_to_shared(smem)), "l"(gmem) : "memory");
}
TCQ_HD void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Shared-memory copy of a layer-constant vector (a parameter no kernel of the stream writes: signs, row scales,
// biases, norm weights), made by the whole block BEFORE pdl_wait(): a launched-early kernel then reads its constants
// from shared memory instead of paying a global round trip for each of them after the dependency is released.
// `bytes` is a multiple of 16 and `sp` advances by it (so it stays 16-byte aligned). Returns a generic pointer to the
// copy, or src itself when src is NULL or `on` is false; either way it must be read with plain loads (never __ldg).
// The caller synchronizes the block before the copy is read.
TCQ_HD const void* stage_const(char*& sp, const void* src, int bytes, bool on) {
    if (!src || !on) return src;
    char* dst = sp;
    sp += bytes;
    if ((reinterpret_cast<uintptr_t>(src) & 15) == 0) {
        for (int i = threadIdx.x; i < (bytes >> 4); i += blockDim.x)
            reinterpret_cast<uint4*>(dst)[i] = __ldg(reinterpret_cast<const uint4*>(src) + i);
    } else {
        for (int i = threadIdx.x; i < bytes; i += blockDim.x) dst[i] = __ldg(reinterpret_cast<const char*>(src) + i);
    }
    return dst;
}

// ---------------------------------------------------------------------------------------------------- host helpers
#define TCQ_CHECK_LAUNCH()                                        \
    do {                                                          \
        cudaError_t e_ = cudaGetLastError();                      \
        if (e_ != cudaSuccess) return TCQ_ERR_LAUNCH;             \
    } while (0)

static inline bool tcq_aligned(const void* p, size_t a) { return (((uintptr_t)p) & (a - 1)) == 0; }

// Streaming multiprocessors of the current device (queried once per translation unit; 148, a B200's, if the query
// fails).
static inline int tcq_sm_count() {
    static int n = 0;
    if (n <= 0) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
            n <= 0)
            n = 148;
    }
    return n;
}

// Row kernels (one block per token row) stage their layer constants in shared memory (stage_const) when the launch
// is latency-bound: at most a few rows per SM, so the extra shared memory costs no occupancy. Many-row launches read
// the constants through L1, where the blocks of an SM share them.
static inline bool tcq_stage_rows(int rows, size_t const_bytes, size_t max_bytes) {
    return const_bytes <= max_bytes && rows <= 4 * tcq_sm_count();
}
