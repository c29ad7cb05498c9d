// W8A8 INT8 GEMM on sm_100a: TMA -> 128B-swizzled shared memory -> tcgen05.mma.kind::i8 -> TMEM INT32 accumulators ->
// tcgen05.ld epilogue with the per-token / per-channel scales.
//
// acc[t][c] = sum_k q[t][k] * W[c][k] (exact INT32), the product of the reference's prefill path
// (torch._int_mm(q, W.t()), modules.py:86; tcq_format.py:110-116). Epilogues: raw INT32 (drop-in for _int_mm),
// FP32 z = ((float)acc * s_tok[t]) * s_ch[c], or BF16(z) (tcq_format.py:135).
//
// Tiling: the UMMA M side is 128 output channels (rows of W), the UMMA N side BN tokens (32..256), K in 128-byte
// stages (four K=32 MMAs per stage). One CTA per SM, persistent over tiles. Warp roles:
//   warp 0    one thread issues the TMA loads (no multicast) into a STAGES-deep ring,
//   warp 1    allocates TMEM; one thread issues tcgen05.mma and commits stage / accumulator barriers,
//   warps 2-5 epilogue: tcgen05.ld of their 32-lane quarter, scale, coalesced stores; TMEM double-buffered so the
//             epilogue of tile i overlaps the MMAs of tile i + 1.
// Every mbarrier wait is bounded (about 2 s): on expiry the kernel sets a device error flag, stops, waits (bounded)
// for its copies and MMAs in flight, frees TMEM and returns; tcq_device_error() reports the flag.
#include <algorithm>
#include "tma.cuh"
#include "trellis_common.cuh"

__device__ int g_tcq_device_error;

namespace {

using namespace tcq;

constexpr int BM = 128;           // channels per tile
constexpr int BK = 128;           // K bytes per stage

// Bounded wait that reports through this file's device error flag.
__device__ __forceinline__ bool mbar_wait(u32 bar, u32 parity, volatile int* abort_flag, unsigned long long limit = kWaitNs) {
    return mbar_wait_bounded(bar, parity, abort_flag, &g_tcq_device_error, limit);
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: rows of 128 bytes, 8-row groups 1024 bytes apart
// (SBO = 1024), LBO unused (1), descriptor version 1, layout type 2 (SWIZZLE_128B). The tile base is 1024-aligned, so
// advancing along K inside the swizzle row is a plain add of 32 bytes to the start address.
__device__ __forceinline__ u64 sw128_desc(u32 addr) {
    return (u64)((addr >> 4) & 0x3FFF) | ((u64)1 << 16) | ((u64)(1024 >> 4) << 32) | ((u64)1 << 46) | ((u64)2 << 61);
}

// Instruction descriptor of tcgen05.mma.kind::i8: D s32, A and B signed int8, both K-major, N = bn, M = 128.
__host__ __device__ constexpr u32 idesc_i8(int bn) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((u32)(bn >> 3) << 17) | ((u32)(BM >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(u32 d_tmem, u64 adesc, u64 bdesc, u32 idesc, u32 accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(u32 bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tmem_ld32(u32 taddr, u32 (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
          "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

enum { OUT_I32 = 0, OUT_F32 = 1, OUT_BF16 = 2 };

// Epilogue warps of the GEMMs (warps 2 .., after the TMA and MMA warps): sixteen for BF16 output, four per TMEM lane
// quarter (its scaling and paired conversion are the heaviest epilogue work; a single-tile CTA waits for all of it),
// eight otherwise. Each warp stages one 32-token x 32-channel box of the output.
constexpr int epi_warps(int mode) { return mode == OUT_BF16 ? 16 : 8; }
constexpr int epi_threads(int mode) { return 64 + 32 * epi_warps(mode); }
constexpr int epi_box_bytes(int mode) { return mode == OUT_BF16 ? 32 * 32 * 2 : 32 * 32 * 4; }

// One epilogue step of a warp: TMEM column group v of its lane's channel ch0 + lane, tokens t0 .. t0 + 31, into the
// output: INT32 as is, or z = ((float)acc * s_tok[t]) * s_ch[n] as FP32 or BF16 (BF16 then + bias as a BF16 tensor add,
// then the activation table: the PyTorch ops of a biased layer, bit for bit). stv: lane l's token scale s_tok[t0 + l]
// (0 past M), loaded by the caller before it waits for the accumulator (the load's latency hides behind the MMAs);
// the scales go round the warp by shuffles. tma: the values are written token-major into the warp's staging box and one
// TMA store writes the box (rows past M, columns past N clipped by the tensor map), instead of 32 two- or four-byte
// stores per lane with stride N.
template <int MODE, bool SPLIT>
__device__ __forceinline__ void epi_chunk(const u32 (&v)[32], int lane, int ch0, int t0, int M, int N, float sc, float bb,
                                          float stv, const u16* __restrict__ bias, const u16* __restrict__ lut,
                                          void* __restrict__ out, uint8_t* stage, const CUtensorMap* tmO, bool tma) {
    const int ch = ch0 + lane;
    auto value = [&](int j, float st) -> u32 {
        if (MODE == OUT_I32) return v[j];
        const float z = ((float)(int)v[j] * st) * sc;
        if (MODE == OUT_F32) return __float_as_uint(z);
        u16 y = f2bf(z);
        if (bias) y = f2bf(bf2f(y) + bb);
        if (lut) y = lut[y];
        return y;
    };
    if (tma && !SPLIT) {
        if (lane == 0) bulk_wait_read_all();       // the warp's previous box has left the staging area
        __syncwarp();
        if (MODE == OUT_BF16) {
            // Two tokens at a time: one paired round-to-nearest conversion (f2bf2) for the product and one for the
            // bias add, the same roundings as f2bf on each value.
            u16* st16 = reinterpret_cast<u16*>(stage);
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
                const float s0 = __shfl_sync(0xffffffffu, stv, j), s1 = __shfl_sync(0xffffffffu, stv, j + 1);
                u32 w = f2bf2(((float)(int)v[j] * s0) * sc, ((float)(int)v[j + 1] * s1) * sc);
                if (bias) w = f2bf2(__uint_as_float(w << 16) + bb, __uint_as_float(w & 0xffff0000u) + bb);
                if (lut) w = (u32)lut[w & 0xffffu] | ((u32)lut[w >> 16] << 16);
                st16[j * 32 + lane] = (u16)(w & 0xffffu);
                st16[(j + 1) * 32 + lane] = (u16)(w >> 16);
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const float st = __shfl_sync(0xffffffffu, stv, j);
                reinterpret_cast<u32*>(stage)[j * 32 + lane] = value(j, st);
            }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // generic-proxy writes -> the TMA store
        __syncwarp();
        if (lane == 0 && ch0 < N && t0 < M) {
            tma_store_2d(tmO, smem_u32(stage), ch0, t0);
            bulk_commit_group();
        }
        return;
    }
    const bool chok = ch < N;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        const float st = __shfl_sync(0xffffffffu, stv, j);
        const int tok = t0 + j;
        if (chok && tok < M) {
            const size_t o = (size_t)tok * N + ch;
            const u32 y = value(j, st);
            if (MODE == OUT_I32) {
                if (!SPLIT) reinterpret_cast<int*>(out)[o] = (int)y;
                else atomicAdd(reinterpret_cast<int*>(out) + o, (int)y);
            } else if (MODE == OUT_F32) {
                reinterpret_cast<u32*>(out)[o] = y;
            } else {
                reinterpret_cast<u16*>(out)[o] = (u16)y;
            }
        }
    }
}

template <int BN, int STAGES, int MODE, bool SPLIT>
__global__ void __launch_bounds__(epi_threads(MODE), 1)
k_gemm_i8(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmQ, void* __restrict__ out,
          const float* __restrict__ s_tok, const float* __restrict__ s_ch, int M, int N, int K, int ks,
          const u16* __restrict__ bias, const u16* __restrict__ lut, const __grid_constant__ CUtensorMap tmO, int tma) {
    constexpr int A_BYTES = BM * BK, B_BYTES = BN * BK;
    constexpr u32 TMEM_COLS = 2 * BN;          // two accumulator buffers; BN in {32, 64, 128, 256} -> power of two
    constexpr u32 IDESC = idesc_i8(BN);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * A_BYTES;
    uint8_t* sE = sB + STAGES * B_BYTES;                     // epilogue staging boxes (warps 2..9)
    u64* bars = reinterpret_cast<u64*>(sE + epi_warps(MODE) * epi_box_bytes(MODE));
    u32* tmem_slot = reinterpret_cast<u32*>(bars + 2 * STAGES + 4);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const u32 full0 = smem_u32(bars), empty0 = smem_u32(bars + STAGES), tfull0 = smem_u32(bars + 2 * STAGES),
              tempty0 = smem_u32(bars + 2 * STAGES + 2);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Work item = (channel tile, token tile, K split); with ks > 1 (INT32 output only) the splits add their partial
    // sums into the zero-filled output with integer atomics (exact).
    const int tiles_n = (N + BM - 1) / BM, tiles_m = (M + BN - 1) / BN, tiles = tiles_n * tiles_m * ks;
    const int KB = (K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(tfull0 + 8 * a, 1);
            mbar_init(tempty0 + 8 * a, 32 * epi_warps(MODE));    // every thread of the epilogue warps
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)), "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const u32 tmem = *tmem_slot;
    pdl_launch_dependents();
    pdl_wait();

    if (warp == 0) {
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&tmW) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(&tmQ) : "memory");
            int stage = 0;
            u32 phase = 0;
            u32 armed[STAGES];
            for (int s = 0; s < STAGES; ++s) armed[s] = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
                const int sp = tile % ks, tt = tile / ks, tn = tt % tiles_n, tm = tt / tiles_n;
                const int kb0 = KB * sp / ks, kb1 = KB * (sp + 1) / ks;
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, abort_flag)) { ok = false; break; }
                    mbar_expect_tx(full0 + 8 * stage, A_BYTES + B_BYTES);
                    tma_load_2d(smem_u32(sA + stage * A_BYTES), &tmW, full0 + 8 * stage, kb * BK, tn * BM);
                    tma_load_2d(smem_u32(sB + stage * B_BYTES), &tmQ, full0 + 8 * stage, kb * BK, tm * BN);
                    armed[stage] += 1;
                    if (++stage == STAGES) { stage = 0; phase ^= 1; }
                }
            }
            if (!ok) {
                // Drain: wait (bounded) for the last load issued into every stage before shared memory goes away.
                for (int s = 0; s < STAGES; ++s)
                    if (armed[s]) { volatile int never = 0; mbar_wait(full0 + 8 * s, (armed[s] - 1) & 1, &never, 100000000ull); }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int stage = 0, it = 0;
            u32 phase = 0;
            bool ok = true;
            int committed = -1;
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++it) {
                const int sp = tile % ks;
                const int kb0 = KB * sp / ks, kb1 = KB * (sp + 1) / ks;
                const int a = it & 1;
                const u32 aph = (it >> 1) & 1;
                if (!mbar_wait(tempty0 + 8 * a, aph ^ 1, abort_flag)) { ok = false; break; }
                tc_fence_after();
                const u32 d = tmem + a * BN;
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait(full0 + 8 * stage, phase, abort_flag)) { ok = false; break; }
                    tc_fence_after();
                    const u32 aaddr = smem_u32(sA + stage * A_BYTES), baddr = smem_u32(sB + stage * B_BYTES);
#pragma unroll
                    for (int k = 0; k < BK / 32; ++k)
                        mma_i8(d, sw128_desc(aaddr + 32 * k), sw128_desc(baddr + 32 * k), IDESC, (kb > kb0 || k > 0) ? 1u : 0u);
                    mma_commit(empty0 + 8 * stage);
                    if (++stage == STAGES) { stage = 0; phase ^= 1; }
                }
                if (!ok) break;
                mma_commit(tfull0 + 8 * a);
                committed = it;
            }
            if (!ok && committed >= 0) {
                // MMAs already issued must finish before TMEM is freed: wait (bounded) for the last commit.
                volatile int never = 0;
                mbar_wait(tfull0 + 8 * (committed & 1), (committed >> 1) & 1, &never, 100000000ull);
            }
        }
    } else {
        const int q = warp & 3;                  // TMEM lane quarter this warp may access
        constexpr int GW = epi_warps(MODE) / 4;  // warps per lane quarter: each takes every GW-th 32-token column group
        const int grp = (warp - 2) >> 2;
        constexpr int NCW = (BN / 32 + GW - 1) / GW;   // column groups of a warp, at most
        int it = 0;
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++it) {
            const int a = it & 1;
            const u32 aph = (it >> 1) & 1;
            // The tile's channel and token scales first: their loads complete while the MMAs still run.
            const int tt = tile / ks, tn = tt % tiles_n, tm = tt / tiles_n;
            const int ch0 = tn * BM + 32 * q, ch = ch0 + lane, m0 = tm * BN;
            const bool chok = ch < N;
            const float sc = (MODE != OUT_I32 && chok) ? s_ch[ch] : 0.f;
            const float bb = (MODE == OUT_BF16 && bias && chok) ? bf2f(bias[ch]) : 0.f;
            float stv[NCW];
#pragma unroll
            for (int i = 0; i < NCW; ++i) {
                const int t = m0 + 32 * (grp + GW * i) + lane;
                stv[i] = MODE != OUT_I32 && grp + GW * i < BN / 32 && t < M ? s_tok[t] : 0.f;
            }
            if (!mbar_wait(tfull0 + 8 * a, aph, abort_flag)) break;
            tc_fence_after();
#pragma unroll 1
            for (int i = 0; i < NCW; ++i) {
                const int c = grp + GW * i;
                if (c >= BN / 32) break;
                float st = stv[0];
#pragma unroll
                for (int j = 1; j < NCW; ++j) st = i == j ? stv[j] : st;
                u32 v[32];
                tmem_ld32(tmem + ((u32)(32 * q) << 16) + (u32)(a * BN + 32 * c), v);
                epi_chunk<MODE, SPLIT>(v, lane, ch0, m0 + 32 * c, M, N, sc, bb, st, bias, lut, out,
                                       sE + (warp - 2) * epi_box_bytes(MODE), &tmO, tma != 0);
            }
            tc_fence_before();
            mbar_arrive(tempty0 + 8 * a);
        }
        if (tma && lane == 0) bulk_wait_all();      // the TMA stores are complete before the CTA exits
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
}


// ------------------------------------------------------------------------------------------------ self-test
// One thread waits, through the kernels' bounded wait, on a barrier that nothing ever arrives at: the wait must give up
// after limit_ns, raise the device error flag and let the kernel return (a failure path tested without a fault).
__global__ void k_wait_expiry(unsigned long long limit_ns) {
    __shared__ __align__(8) u64 bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&bar), 1);
        abort_flag = 0;
        mbar_init_fence();
    }
    __syncthreads();
    if (threadIdx.x == 0) mbar_wait(smem_u32(&bar), 0, &abort_flag, limit_ns);
}

// ------------------------------------------------------------------------------------------------ two-SM INT8 GEMM
// Large products: a cluster of two CTAs on an SM pair computes a 256-channel x 256-token tile with
// tcgen05.mma.cta_group::2 (M = 256, N = 256). Each CTA loads only its own 128 weight rows and its own 128 tokens per
// K stage (32 KB) with plain TMA loads (no multicast) whose bytes complete on the leader CTA's stage barrier; the pair
// exchanges the token halves inside the MMA, so each SM streams a third less operand data from L2 per MMA than the
// single-SM 128 x 256 tile. The leader's thread issues the MMAs; its commits arrive on the barriers of both CTAs
// (tcgen05.commit multicast); each CTA's epilogue reads its own 128 accumulator lanes (channels) x 256 columns
// (tokens) from its own TMEM and releases the buffer on the leader's barrier with a remote arrive.
constexpr int kStages2 = 6;
constexpr int kHalf = 128;                                   // channels / tokens per CTA of the pair

__device__ __forceinline__ u32 cluster_rank() {
    u32 r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ u32 map_to_rank(u32 addr, u32 rank) {
    u32 r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void remote_arrive(u32 cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// TMA load into this CTA's shared memory whose bytes complete on a barrier of the pair (the leader's).
__device__ __forceinline__ void tma_load_2d_pair(u32 dst, const CUtensorMap* map, u32 bar_cluster, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(map), "r"(bar_cluster), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void mma_i8_pair(u32 d_tmem, u64 adesc, u64 bdesc, u32 idesc, u32 accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u)
        : "memory");
}
// Commit the pair's outstanding MMAs to the barrier at this offset in both CTAs.
__device__ __forceinline__ void mma_commit_pair(u32 bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
                 "h"((unsigned short)3)
                 : "memory");
}

constexpr u32 idesc_i8_pair() {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((u32)(256 >> 3) << 17) | ((u32)(256 >> 4) << 24);
}

template <int MODE>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(epi_threads(MODE), 1)
k_gemm_i8_2sm(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmQ, void* __restrict__ out,
              const float* __restrict__ s_tok, const float* __restrict__ s_ch, int M, int N, int K,
              const u16* __restrict__ bias, const u16* __restrict__ lut, const __grid_constant__ CUtensorMap tmO, int tma) {
    constexpr int A_BYTES = kHalf * BK, B_BYTES = kHalf * BK;
    constexpr u32 TMEM_COLS = 512;                           // two 256-column accumulators
    constexpr u32 IDESC = idesc_i8_pair();
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* sA = smem;
    uint8_t* sB = smem + kStages2 * A_BYTES;
    uint8_t* sE = sB + kStages2 * B_BYTES;                   // epilogue staging boxes (warps 2..9)
    u64* bars = reinterpret_cast<u64*>(sE + epi_warps(MODE) * epi_box_bytes(MODE));
    u32* tmem_slot = reinterpret_cast<u32*>(bars + 2 * kStages2 + 4);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const u32 full0 = smem_u32(bars), empty0 = smem_u32(bars + kStages2), tfull0 = smem_u32(bars + 2 * kStages2),
              tempty0 = smem_u32(bars + 2 * kStages2 + 2);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const u32 rank = cluster_rank();
    const bool leader = rank == 0;
    const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
    const int tiles_n = (N + 255) / 256, tiles_m = (M + 255) / 256, tiles = tiles_n * tiles_m;
    const int KB = (K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int st = 0; st < kStages2; ++st) {
            mbar_init(full0 + 8 * st, 1);                    // the leader's producer arrives; both CTAs' bytes complete
            mbar_init(empty0 + 8 * st, 1);                   // the leader's MMA commit (multicast)
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(tfull0 + 8 * a, 1);                    // the leader's MMA commit (multicast)
            mbar_init(tempty0 + 8 * a, 2 * epi_warps(MODE));     // the epilogue warps of both CTAs (used in the leader)
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {                                         // the same warp of both CTAs allocates the pair's TMEM
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)), "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    cluster_sync();                                          // barriers of both CTAs initialized, TMEM allocated
    tc_fence_after();
    const u32 tmem = *tmem_slot;
    pdl_launch_dependents();
    pdl_wait();

    if (warp == 0) {
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&tmW) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(&tmQ) : "memory");
            int stage = 0;
            u32 phase = 0;
            bool ok = true;
            for (int tile = pair; tile < tiles && ok; tile += pairs) {
                const int tn = tile % tiles_n, tm = tile / tiles_n;
                for (int kb = 0; kb < KB; ++kb) {
                    if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, abort_flag)) { ok = false; break; }
                    const u32 fb = map_to_rank(full0 + 8 * stage, 0);
                    if (leader) mbar_expect_tx(full0 + 8 * stage, 2 * (A_BYTES + B_BYTES));
                    tma_load_2d_pair(smem_u32(sA + stage * A_BYTES), &tmW, fb, kb * BK, tn * 256 + (int)rank * kHalf);
                    tma_load_2d_pair(smem_u32(sB + stage * B_BYTES), &tmQ, fb, kb * BK, tm * 256 + (int)rank * kHalf);
                    if (++stage == kStages2) { stage = 0; phase ^= 1; }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            int stage = 0, it = 0;
            u32 phase = 0;
            bool ok = true;
            int committed = -1;
            for (int tile = pair; tile < tiles && ok; tile += pairs, ++it) {
                const int a = it & 1;
                const u32 aph = (it >> 1) & 1;
                if (!mbar_wait(tempty0 + 8 * a, aph ^ 1, abort_flag)) { ok = false; break; }
                tc_fence_after();
                const u32 d = tmem + a * 256;
                for (int kb = 0; kb < KB; ++kb) {
                    if (!mbar_wait(full0 + 8 * stage, phase, abort_flag)) { ok = false; break; }
                    tc_fence_after();
                    const u32 aaddr = smem_u32(sA + stage * A_BYTES), baddr = smem_u32(sB + stage * B_BYTES);
#pragma unroll
                    for (int k = 0; k < BK / 32; ++k)
                        mma_i8_pair(d, sw128_desc(aaddr + 32 * k), sw128_desc(baddr + 32 * k), IDESC, (kb > 0 || k > 0) ? 1u : 0u);
                    mma_commit_pair(empty0 + 8 * stage);
                    if (++stage == kStages2) { stage = 0; phase ^= 1; }
                }
                if (!ok) break;
                mma_commit_pair(tfull0 + 8 * a);
                committed = it;
            }
            if (!ok && committed >= 0) {
                volatile int never = 0;
                mbar_wait(tfull0 + 8 * (committed & 1), (committed >> 1) & 1, &never, 100000000ull);
            }
        }
    } else {
        const int q = warp & 3;                              // TMEM lane quarter this warp may access
        constexpr int NCW = 256 / 32 / (epi_warps(MODE) / 4);   // 32-token column groups of a warp
        const int c0 = ((warp - 2) >> 2) * NCW;              // its share of the tile's column groups
        const u32 tempty_leader = map_to_rank(tempty0, 0);
        int it = 0;
        for (int tile = pair; tile < tiles; tile += pairs, ++it) {
            const int a = it & 1;
            const u32 aph = (it >> 1) & 1;
            // The tile's channel and token scales first: their loads complete while the MMAs still run.
            const int tn = tile % tiles_n, tm = tile / tiles_n;
            const int ch0 = tn * 256 + (int)rank * kHalf + 32 * q, ch = ch0 + lane, m0 = tm * 256;
            const bool chok = ch < N;
            const float sc = (MODE != OUT_I32 && chok) ? s_ch[ch] : 0.f;
            const float bb = (MODE == OUT_BF16 && bias && chok) ? bf2f(bias[ch]) : 0.f;
            float stv[NCW];
#pragma unroll
            for (int i = 0; i < NCW; ++i) {
                const int t = m0 + 32 * (c0 + i) + lane;
                stv[i] = MODE != OUT_I32 && t < M ? s_tok[t] : 0.f;
            }
            if (!mbar_wait(tfull0 + 8 * a, aph, abort_flag)) break;
            tc_fence_after();
#pragma unroll 1
            for (int i = 0; i < NCW; ++i) {
                const int c = c0 + i;
                float st = stv[0];
#pragma unroll
                for (int j = 1; j < NCW; ++j) st = i == j ? stv[j] : st;
                u32 v[32];
                tmem_ld32(tmem + ((u32)(32 * q) << 16) + (u32)(a * 256 + 32 * c), v);
                epi_chunk<MODE, false>(v, lane, ch0, m0 + 32 * c, M, N, sc, bb, st, bias, lut, out,
                                       sE + (warp - 2) * epi_box_bytes(MODE), &tmO, tma != 0);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) remote_arrive(tempty_leader + 8 * a);
        }
        if (tma && lane == 0) bulk_wait_all();      // the TMA stores are complete before the CTA exits
    }
    tc_fence_before();
    cluster_sync();                                          // every MMA done, every TMEM read done in both CTAs
    tc_fence_after();
    if (warp == 1) {
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
}

// ------------------------------------------------------------------------------------------------ fused decode-GEMM
// z (M, N) FP32 = ((float)(q W^T) * s[t]) * rs[n] with W decoded from the trellis stream straight into shared memory:
// the decoded weights never leave the SM. One CTA = one 128-channel tile (8 tile rows) x one K range; per 128-byte K
// stage, 16 decoder warps write the 128 x 128 INT8 A tile in the 128B-swizzled K-major UMMA layout (512 threads x 2
// tile rows), TMA brings the BN x 128 activation tile, one thread issues four tcgen05.mma.kind::i8 (M = 128, N = BN,
// K = 32) into TMEM. Epilogue: the 16 decoder warps copy the accumulator from TMEM into shared memory (the decode
// table's space, dead by then); without a K split the CTA scales and writes z from there; the K splits of a channel
// tile run as one thread-block cluster, and every rank sums one slice of the tile over all ranks' shared memory and
// writes it. Only when no cluster fits do the splits store INT32 partials into their own workspace slices (plain
// stores), and the CTA whose arrival completes a channel tile sums them, writes z and zeroes the slices again.
constexpr int kTcDecWarps = 16;
constexpr int kTcKsMax = 4;         // K splits per channel tile, at most (the finishing CTA sums that many slices)
constexpr int kTcPrefetch = 4;      // K stages of weight words a decoder thread has in flight
constexpr int kTcThreads = 64 + 32 * kTcDecWarps;

struct TcParts {
    int ct;         // channel tiles
    int ks;         // K splits per channel tile
    int kb;         // 128-byte K stages
    int nb0, nb1;   // layer bounds in tile rows (multiples of 8)
    int cl;         // the K splits of a channel tile are one thread-block cluster
    int zvec;       // z is 16-byte aligned: the finished outputs leave as 16-byte stores
};

// 16 bytes of a cluster peer's (or this CTA's) shared memory.
__device__ __forceinline__ int4 ld_cluster_v4(u32 addr) {
    int4 v;
    asm volatile("ld.shared::cluster.v4.s32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr) : "memory");
    return v;
}

__device__ __forceinline__ int ld_cluster_s32(u32 addr) {
    int v;
    asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
    return v;
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(kTcThreads, 1)
k_gemm_tcq_tc(const __grid_constant__ CUtensorMap tmQ, const u16* __restrict__ bits, const i8* __restrict__ t8,
              const float* __restrict__ s_tok, const float* __restrict__ rs, float* __restrict__ z, int M, int N, int K,
              TcParts P, int* __restrict__ ws_acc, int* __restrict__ ws_cnt) {
    constexpr int A_BYTES = BM * BK, B_BYTES = BN * BK;
    constexpr u32 TMEM_COLS = BN < 32 ? 32 : BN;
    // The MMA's N covers the tokens only (M rounded up to 16, a valid UMMA N), not the whole BN-wide token tile: rows
    // past M of the activation tile are zero-filled and would only cost tensor time (160 tokens in a 256 tile: 3/8).
    const u32 IDESC = idesc_i8(min(BN, (M + 15) & ~15));
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    char* tab = reinterpret_cast<char*>(smem);                       // 64 KB decode table (16-bit entries)
    uint8_t* sA = smem + tcq::kTab16Bytes;
    uint8_t* sB = sA + STAGES * A_BYTES;
    u16* pairs = reinterpret_cast<u16*>(sB + STAGES * B_BYTES);       // 1 KB staging of t8 (1024-byte aligned)
    u64* bars = reinterpret_cast<u64*>(sB + STAGES * B_BYTES + 1024);
    u32* tmem_slot = reinterpret_cast<u32*>(bars + 2 * STAGES + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* last_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);
    const u32 full0 = smem_u32(bars), empty0 = smem_u32(bars + STAGES), tfull = smem_u32(bars + 2 * STAGES);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ct = blockIdx.x / P.ks, ksi = blockIdx.x % P.ks;
    const int kb0 = (int)((long long)P.kb * ksi / P.ks), kb1 = (int)((long long)P.kb * (ksi + 1) / P.ks);
    const int tr0 = ct * 8, tiles_k = K >> 4, tiles_n = N >> 4;
    const int slot = (tr0 >= P.nb0) + (tr0 >= P.nb1);

    if (threadIdx.x == 0) {
        for (int st = 0; st < STAGES; ++st) {
            mbar_init(full0 + 8 * st, kTcDecWarps + 1);        // one arrival per decoder warp + the TMA
            mbar_init(empty0 + 8 * st, 1);
        }
        mbar_init(tfull, 1);
        *abort_flag = 0;
        *last_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)), "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    pdl_launch_dependents();
    // Decoder thread d -> tile (i, j) = (d >> 6, (d >> 3) & 7) of a K stage, tile rows 2g, 2g + 1 (g = d & 7). Its
    // words of the first kTcPrefetch stages are requested before the table build (their DRAM latency hides under
    // it); while stage kb is decoded, stage kb + kTcPrefetch is requested (a stage decodes in a fraction of the load
    // latency, so one stage of look-ahead left the decoders waiting on every stage).
    const int dd = threadIdx.x - 64;
    const int di = dd >> 6, dj = (dd >> 3) & 7, dg = dd & 7;
    const bool drow_ok = warp >= 2 && tr0 + di < tiles_n;
    auto load_words = [&](int kb, u32& a, u32& b, u32& c) {
        const int tc = kb * 8 + dj;
        a = b = c = 0;
        if (drow_ok && kb < kb1 && tc < tiles_k) {
            const u32* tw = reinterpret_cast<const u32*>(bits + ((size_t)(tr0 + di) * tiles_k + tc) * 32);
            a = __ldg(tw + 2 * dg);
            b = __ldg(tw + 2 * dg + 1);
            c = __ldg(tw + ((2 * dg + 2) & 15));
        }
    };
    u32 pw[kTcPrefetch][3];
#pragma unroll
    for (int p = 0; p < kTcPrefetch; ++p) load_words(kb0 + p, pw[p][0], pw[p][1], pw[p][2]);
    if (threadIdx.x < 8 && tr0 + (int)threadIdx.x < tiles_n && kb1 - kb0 > 1) {   // later stages: into L2 now
        const int t0 = (kb0 + 1) * 8, t1 = kb1 * 8 < tiles_k ? kb1 * 8 : tiles_k;
        if (t1 > t0)
            prefetch_l2_bulk(bits + ((size_t)(tr0 + threadIdx.x) * tiles_k + t0) * 32, (unsigned)(t1 - t0) * 64u);
    }
    tcq::build_table16(tab, pairs, t8 + 1024 * slot);                // weights only: before the dependency wait
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const u32 tmem = *tmem_slot;
    // The dependency wait is per role: the token tiles (TMA), the MMAs that consume them and everything the epilogue
    // reads or writes in global memory come after it; the decoders run ahead of it through the first STAGES K stages
    // (the weights and the table are layer constants; those stages' ring slots start free, so nothing waits on a
    // barrier before the predecessor has finished and every bounded wait keeps its meaning), so a launch that starts
    // while its predecessor runs has its first stages decoded by the time the activations are ready.

    if (warp == 0) {
        pdl_wait();
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&tmQ) : "memory");
            int st = 0;
            u32 ph = 0;
            for (int kb = kb0; kb < kb1; ++kb) {
                if (!mbar_wait(empty0 + 8 * st, ph ^ 1, abort_flag)) break;
                mbar_expect_tx(full0 + 8 * st, B_BYTES);
                tma_load_2d(smem_u32(sB + st * B_BYTES), &tmQ, full0 + 8 * st, kb * BK, 0);
                if (++st == STAGES) { st = 0; ph ^= 1; }
            }
        }
    } else if (warp == 1) {
        pdl_wait();
        if (lane == 0) {
            int st = 0;
            u32 ph = 0;
            bool ok = true;
            for (int kb = kb0; kb < kb1; ++kb) {
                if (!mbar_wait(full0 + 8 * st, ph, abort_flag)) { ok = false; break; }
                tc_fence_after();
                const u32 aaddr = smem_u32(sA + st * A_BYTES), baddr = smem_u32(sB + st * B_BYTES);
#pragma unroll
                for (int k = 0; k < BK / 32; ++k)
                    mma_i8(tmem, sw128_desc(aaddr + 32 * k), sw128_desc(baddr + 32 * k), IDESC, (kb > kb0 || k > 0) ? 1u : 0u);
                mma_commit(empty0 + 8 * st);
                if (++st == STAGES) { st = 0; ph ^= 1; }
            }
            (void)ok;
            mma_commit(tfull);   // also on an early stop: it arrives once every MMA issued so far has finished
        }
    } else {
        // ---- decoders (tile (di, dj), tile rows 2 dg, 2 dg + 1 of each stage; see load_words)
        const int i = di, j = dj, g = dg;
        const u32 lane4 = 4u * lane;
        int st = 0;
        u32 ph = 0;
        for (int kb = kb0; kb < kb1; ++kb) {
            if (kb == kb0 + STAGES) pdl_wait();      // beyond the free ring slots: wait for the predecessor first
            const int tc = kb * 8 + j;
            const u32 w0 = pw[0][0], w1 = pw[0][1], w2 = pw[0][2];
            const bool ok = drow_ok && tc < tiles_k;
#pragma unroll
            for (int p = 0; p + 1 < kTcPrefetch; ++p) {
                pw[p][0] = pw[p + 1][0];
                pw[p][1] = pw[p + 1][1];
                pw[p][2] = pw[p + 1][2];
            }
            load_words(kb + kTcPrefetch, pw[kTcPrefetch - 1][0], pw[kTcPrefetch - 1][1], pw[kTcPrefetch - 1][2]);
            if (!mbar_wait(empty0 + 8 * st, ph ^ 1, abort_flag)) break;
            uint8_t* a = sA + st * A_BYTES;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int row = 16 * i + 2 * g + h;
                u32 wd[4] = {0, 0, 0, 0};
                if (ok) tcq::row_words16(tcq::rowA(h ? w1 : w0), tcq::rowA(h ? w2 : w1), tab, lane4, wd);
                *reinterpret_cast<uint4*>(a + row * 128 + ((j ^ (row & 7)) << 4)) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // generic-proxy stores -> tensor-core reads
            __syncwarp();
            if (lane == 0) mbar_arrive(full0 + 8 * st);
            if (++st == STAGES) { st = 0; ph ^= 1; }
        }
        pdl_wait();                                  // the epilogue reads the token scales and writes z / the workspace
        // ---- epilogue
        if (P.ks == 1 || P.cl) {
            // Every decoder warp moves part of the accumulator from TMEM (its lane quarter warp & 3, column groups
            // (warp - 2) / 4, + 4, ...) into shared memory, token-major [token][128 channels], in the space of the
            // decode table: once the last MMA has completed, every decoder has arrived on its last stage, so no
            // table lookup is left. Stores are unconditional (rows past M are never read).
            if (mbar_wait(tfull, 0, abort_flag) && !*abort_flag) {
                tc_fence_after();
                const int q = warp & 3;
                int* sp = reinterpret_cast<int*>(smem) + 32 * q + lane;
                const int chunks = (M + 31) >> 5;
#pragma unroll 1
                for (int c = (warp - 2) >> 2; c < chunks; c += 4) {
                    u32 v[32];
                    tmem_ld32(tmem + ((u32)(32 * q) << 16) + (u32)(32 * c), v);
#pragma unroll
                    for (int jj = 0; jj < 32; ++jj) sp[(32 * c + jj) * BM] = (int)v[jj];
                }
            }
        } else if (warp >= 4 && warp < 8) {
            // K split without a cluster: decoder warps 2..5 (warp index 4..7), one TMEM lane quarter each, store the
            // INT32 partials into this split's own slice of the workspace (plain stores, no atomics)
            const int q = warp & 3;
            const int ch = ct * BM + 32 * q + lane;
            const bool chok = ch < N;
            if (mbar_wait(tfull, 0, abort_flag)) {
                tc_fence_after();
                int* part = ws_acc + (size_t)ksi * M * N;
#pragma unroll 1
                for (int c = 0; c < (M + 31) / 32; ++c) {
                    u32 v[32];
                    tmem_ld32(tmem + ((u32)(32 * q) << 16) + (u32)(32 * c), v);
                    if (chok) {
#pragma unroll
                        for (int jj = 0; jj < 32; ++jj) {
                            const int tok = 32 * c + jj;
                            if (tok < M) part[(size_t)tok * N + ch] = (int)v[jj];
                        }
                    }
                }
            }
        }
    }
    if (P.ks == 1 || P.cl) {
        // Scale and write z. Without a K split, from this CTA's shared memory. With one, the K splits of the channel
        // tile are a cluster and each rank finishes one slice of the tile's (token, channel) elements, summing the
        // ranks' partials through distributed shared memory (integers: exact in any order); the second cluster
        // barrier keeps every rank's shared memory alive until all have read it. Every thread reaches the barriers.
        // The tile's row scales and the token scales go to shared memory (the A stages, free once the last MMA has
        // completed) before the barrier, so the reduction below reads every operand on chip.
        // (at the end of the operand ring: the accumulator staging, up to 256 x 128 INT32, spans the table and the
        // first stages)
        float* s_rs = reinterpret_cast<float*>(sB + STAGES * B_BYTES) - (BM + 256);
        float* s_st = s_rs + BM;
        if (!*abort_flag && warp >= 2) {
            for (int i = threadIdx.x - 64; i < BM + M; i += 32 * kTcDecWarps) {
                if (i < BM) s_rs[i] = ct * BM + i < N ? rs[ct * BM + i] : 0.f;
                else s_st[i - BM] = s_tok[i - BM];
            }
        }
        if (P.cl) cluster_sync(); else __syncthreads();
        if (!*abort_flag && warp >= 2) {
            const int R = P.cl ? P.ks : 1, rank = P.cl ? (int)cluster_rank() : 0;
            // groups of 4 consecutive channels of one token: one 16-byte load per rank and group, U groups in flight
            const int G = M * (BM / 4), g_end = (int)((long long)G * (rank + 1) / R);
            u32 peer[8];
#pragma unroll
            for (int r = 0; r < 8; ++r) peer[r] = r < R ? (P.cl ? map_to_rank(smem_u32(smem), r) : smem_u32(smem)) : 0u;
            constexpr int NT = 32 * kTcDecWarps, U = 4;
            for (int g0 = (int)((long long)G * rank / R) + (int)threadIdx.x - 64; g0 < g_end; g0 += U * NT) {
                int4 sum[U];
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int g = g0 + u * NT;
                    sum[u] = make_int4(0, 0, 0, 0);
                    if (g < g_end) {
                        if (!P.cl) {
                            sum[u] = reinterpret_cast<const int4*>(smem)[g];     // no cluster: this CTA's own staging
                        } else {
#pragma unroll
                            for (int r = 0; r < 8; ++r)
                                if (r < R) {
                                    const int4 a = ld_cluster_v4(peer[r] + 16u * g);
                                    sum[u].x += a.x; sum[u].y += a.y; sum[u].z += a.z; sum[u].w += a.w;
                                }
                        }
                    }
                }
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int g = g0 + u * NT, tok = g >> 5, c = 4 * (g & 31);
                    if (g < g_end && ct * BM + c < N) {
                        const float st = s_st[tok];
                        const float4 o = make_float4(((float)sum[u].x * st) * s_rs[c], ((float)sum[u].y * st) * s_rs[c + 1],
                                                     ((float)sum[u].z * st) * s_rs[c + 2], ((float)sum[u].w * st) * s_rs[c + 3]);
                        float* zo = z + (size_t)tok * N + ct * BM + c;
                        if (P.zvec) {
                            *reinterpret_cast<float4*>(zo) = o;
                        } else {
                            zo[0] = o.x; zo[1] = o.y; zo[2] = o.z; zo[3] = o.w;
                        }
                    }
                }
            }
        }
        if (P.cl) cluster_sync();
    }
    // Split K without a cluster: every CTA has stored its partials; the one whose arrival completes the channel tile
    // finishes it. The decision sits between two CTA-wide barriers that every thread reaches on every path.
    __syncthreads();
    if (P.ks > 1 && !P.cl && threadIdx.x == 0) {
        int done = 0;
        if (!*abort_flag) {
            int old;
            asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(old) : "l"(ws_cnt + ct) : "memory");
            done = old + 1 == P.ks;
            if (done) ws_cnt[ct] = 0;
        }
        *last_flag = done;
    }
    __syncthreads();
    if (P.ks > 1 && !P.cl && *last_flag && warp >= 2) {
        // The CTA that completes the channel tile sums its ks slices (exact integers, slice order), clears them for the
        // next call and writes z. All 16 decoder warps take part, 8 elements (tok, channel) per thread and step with
        // every load of the step issued before any is used; consecutive threads take consecutive channels.
        const int t = threadIdx.x - 64;
        for (int e0 = t; e0 < M * BM; e0 += 8 * 32 * kTcDecWarps) {
            int vals[8][kTcKsMax];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int e = e0 + u * 32 * kTcDecWarps, tok = e / BM, ch = ct * BM + e % BM;
                const bool ok = e < M * BM && ch < N;
#pragma unroll
                for (int k = 0; k < kTcKsMax; ++k)
                    vals[u][k] = ok && k < P.ks ? __ldcg(ws_acc + ((size_t)k * M + tok) * N + ch) : 0;
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int e = e0 + u * 32 * kTcDecWarps, tok = e / BM, ch = ct * BM + e % BM;
                if (e < M * BM && ch < N) {
                    int sum = 0;
#pragma unroll
                    for (int k = 0; k < kTcKsMax; ++k)
                        if (k < P.ks) {
                            sum += vals[u][k];
                            ws_acc[((size_t)k * M + tok) * N + ch] = 0;
                        }
                    z[(size_t)tok * N + ch] = ((float)sum * s_tok[tok]) * rs[ch];
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        if (*abort_flag && lane == 0) {
            // MMAs already issued must finish before TMEM is freed: wait (bounded) for the final commit.
            volatile int never = 0;
            mbar_wait(tfull, 0, &never, 100000000ull);
        }
        __syncwarp();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
}

// ------------------------------------------------------------------------------------------------ host side
int g_sms_i8 = 0;
int sms() {
    if (!g_sms_i8) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&g_sms_i8, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || g_sms_i8 <= 0) g_sms_i8 = 148;
    }
    return g_sms_i8;
}

// 2-D int8 tensor map over a row-major (rows, K) matrix: box = 128 bytes of K x box_rows rows, 128-byte swizzle,
// out-of-bounds elements read as zero (exact for integer products).
bool make_map(CUtensorMap* map, const void* base, int rows, int K, int box_rows) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)K};
    const cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The output as a TMA store target: (M, N) INT32 / FP32 / BF16 row-major, 32 x 32 boxes, no swizzle. False when the
// address or the row pitch is not a multiple of 16 bytes (the epilogue then stores directly).
bool make_out_map(CUtensorMap* map, void* out, int M, int N, int mode) {
    EncodeTiledFn enc = encode_fn();
    const size_t es = mode == OUT_BF16 ? 2 : 4;
    if (!enc || !tcq_aligned(out, 16) || ((size_t)N * es) % 16) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)M};
    const cuuint64_t strides[1] = {(cuuint64_t)N * es};
    const cuuint32_t box[2] = {32, 32};
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt = mode == OUT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                   : mode == OUT_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_INT32;
    return enc(map, dt, 2, out, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
               CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, int STAGES, int MODE, bool SPLIT = false>
int launch_i8(const int8_t* q, const int8_t* W, void* out, const float* s_tok, const float* s_ch, int M, int N, int K, int ks,
              cudaStream_t st, const u16* bias = nullptr, const u16* lut = nullptr) {
    CUtensorMap tmW, tmQ;
    if (!make_map(&tmW, W, N, K, BM) || !make_map(&tmQ, q, M, K, BN)) return TCQ_ERR_ARG;
    CUtensorMap tmO = {};
    const int tma = !SPLIT && make_out_map(&tmO, out, M, N, MODE) ? 1 : 0;
    auto kern = k_gemm_i8<BN, STAGES, MODE, SPLIT>;
    const int smem = 1024 + STAGES * (BM + BN) * BK + epi_warps(MODE) * epi_box_bytes(MODE) + (2 * STAGES + 4) * 8 + 16;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return TCQ_ERR_LAUNCH;
    if (ks > 1 && cudaMemsetAsync(out, 0, (size_t)M * N * sizeof(int), st) != cudaSuccess) return TCQ_ERR_LAUNCH;
    const int tiles = ((N + BM - 1) / BM) * ((M + BN - 1) / BN) * ks;
    const int grid = tiles < sms() ? tiles : sms();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(epi_threads(MODE));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, tmW, tmQ, out, s_tok, s_ch, M, N, K, ks, bias, lut, tmO, tma) == cudaSuccess ? TCQ_OK
                                                                                                          : TCQ_ERR_LAUNCH;
}

template <int MODE>
int launch_i8_2sm(const int8_t* q, const int8_t* W, void* out, const float* s_tok, const float* s_ch, int M, int N, int K,
                  cudaStream_t st, const u16* bias = nullptr, const u16* lut = nullptr) {
    CUtensorMap tmW, tmQ;
    if (!make_map(&tmW, W, N, K, kHalf) || !make_map(&tmQ, q, M, K, kHalf)) return TCQ_ERR_ARG;
    CUtensorMap tmO = {};
    const int tma = make_out_map(&tmO, out, M, N, MODE) ? 1 : 0;
    auto kern = k_gemm_i8_2sm<MODE>;
    const int smem = 1024 + kStages2 * 2 * kHalf * BK + epi_warps(MODE) * epi_box_bytes(MODE) + (2 * kStages2 + 4) * 8 + 16;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return TCQ_ERR_LAUNCH;
    const int tiles = ((N + 255) / 256) * ((M + 255) / 256);
    int pairs = sms() / 2;
    if (pairs > tiles) pairs = tiles;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs);
    cfg.blockDim = dim3(epi_threads(MODE));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, tmW, tmQ, out, s_tok, s_ch, M, N, K, bias, lut, tmO, tma) == cudaSuccess ? TCQ_OK
                                                                                                     : TCQ_ERR_LAUNCH;
}

// Above that, token-tile width: 256 while that still gives a quarter of the SMs a tile (wide tiles re-read the weights least);
// otherwise the widest of 128 / 64 / 32 that fills half the SMs, so small-M products do not run on a handful of SMs.
// An INT32 product with too few tiles even at 32 is split along K as well (integer atomics into the zeroed output).
template <int MODE>
int dispatch(const int8_t* q, const int8_t* W, void* out, const float* s_tok, const float* s_ch, int M, int N, int K,
             cudaStream_t st, const u16* bias = nullptr, const u16* lut = nullptr) {
    const int ct = (N + BM - 1) / BM, half = sms() / 2, KB = (K + BK - 1) / BK;
    auto tiles = [&](int bn) { return ct * ((M + bn - 1) / bn); };
    // Large products: the two-SM 256 x 256 tile once every SM pair gets a tile, unless its last round is so partial
    // that one-SM 128 x 128 tiles fill the rounds far better (wave efficiency = tiles / (rounds x slots)); the one-SM
    // tile runs at a lower rate per SM, so smaller differences keep the two-SM tile (measured: 4096 x 4304 -> 1152,
    // 0.54 against 0.97, 35.0 -> 32.6 us; 1024 x 2048 -> 6144, 0.65 against 0.86, 19.4 -> 22.5 us).
    auto wave = [](long long t, long long slots) { return (double)t / (double)(((t + slots - 1) / slots) * slots); };
    const long long t2 = (long long)((N + 255) / 256) * ((M + 255) / 256);
    if (M >= 512 && t2 >= half) {
        if (wave(tiles(128), sms()) > wave(t2, half) + 0.3) return launch_i8<128, 6, MODE>(q, W, out, s_tok, s_ch, M, N, K, 1, st, bias, lut);
        return launch_i8_2sm<MODE>(q, W, out, s_tok, s_ch, M, N, K, st, bias, lut);
    }
    // Token tiles of 256 on at most half the SMs: tiles of 128 instead while they still fit in one round (twice the
    // SMs at half the work each; measured faster at every such shape of 256-1024 tokens).
    if (M > 128 && tiles(256) >= sms() / 4 && tiles(256) <= half && tiles(128) <= sms())
        return launch_i8<128, 6, MODE>(q, W, out, s_tok, s_ch, M, N, K, 1, st, bias, lut);
    if (M > 128 && tiles(256) >= sms() / 4) return launch_i8<256, 4, MODE>(q, W, out, s_tok, s_ch, M, N, K, 1, st, bias, lut);
    if (M > 64 && tiles(128) >= half) return launch_i8<128, 6, MODE>(q, W, out, s_tok, s_ch, M, N, K, 1, st, bias, lut);
    if (M > 32 && tiles(64) >= half) return launch_i8<64, 8, MODE>(q, W, out, s_tok, s_ch, M, N, K, 1, st, bias, lut);
    if (MODE == OUT_I32 && tiles(32) < half) {
        int ks = sms() / tiles(32);
        if (ks > KB / 2) ks = KB / 2;
        if (ks > 1) return launch_i8<32, 8, MODE, true>(q, W, out, s_tok, s_ch, M, N, K, ks, st, bias, lut);
    }
    return launch_i8<32, 8, MODE>(q, W, out, s_tok, s_ch, M, N, K, 1, st, bias, lut);
}

// Clusters of `size` CTAs of `kern` (smem bytes each) that can be resident at once (cached per kernel and size).
template <class Kern>
int max_clusters(Kern kern, int smem, int size) {
    static int cache[9] = {0};
    static const void* cached_for = nullptr;
    if (size < 2 || size > 8) return 0;
    if (cached_for != reinterpret_cast<const void*>(kern)) {
        for (int& c : cache) c = 0;
        cached_for = reinterpret_cast<const void*>(kern);
    }
    if (cache[size] == 0) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(size * 64);
        cfg.blockDim = dim3(kTcThreads);
        cfg.dynamicSmemBytes = smem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = size;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        cache[size] = cudaOccupancyMaxActiveClusters(&n, kern, &cfg) == cudaSuccess && n > 0 ? n : -1;
    }
    return cache[size];
}

template <int BN, int STAGES>
int launch_tc(const uint16_t* bits, const int8_t* t8, const int8_t* q, const float* s, const float* rs, float* z, int M, int N,
              int K, int nb0, int nb1, int* ws, cudaStream_t st) {
    CUtensorMap tmQ;
    if (!make_map(&tmQ, q, M, K, BN)) return TCQ_ERR_ARG;
    auto kern = k_gemm_tcq_tc<BN, STAGES>;
    const int smem = 1024 + tcq::kTab16Bytes + STAGES * (BM + BN) * BK + (2 * STAGES + 1) * 8 + 16 + 1024;
    static_assert(tcq::kTab16Bytes + STAGES * (BM + BN) * BK - (BM + 256) * 4 >= 256 * BM * 4 || BN < 256,
                  "the accumulator staging and the staged scales fit in the table and the ring");
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return TCQ_ERR_LAUNCH;
    TcParts P;
    P.ct = (N + BM - 1) / BM;
    P.kb = (K + BK - 1) / BK;
    // K splits: the splits of a channel tile form a cluster (at most 8, a portable size) that reduces in distributed
    // shared memory, each rank finishing one slice of the tile: the largest split whose clusters are all resident at
    // once (one CTA fills an SM, so clusters pack into the GPCs only so far), with about 4 K stages per CTA for 32-token
    // tiles from 12 stages on (measured at 17 tokens: 4 splits beat 6 and 8 at 12 and 16 stages, 8 beat 6 at 48), at
    // least 3 below that, and at least 2 for wider token tiles. When no cluster of 2 or more fits, the splits reduce
    // through workspace slices (at most kTcKsMax).
    int ks = 1;
    bool cl = false;
    {
        const int want = BN == 32 ? (P.kb >= 12 ? std::max(4, (P.kb + 3) / 4) : (P.kb + 2) / 3) : P.kb / 2;
        int c = std::min({8, sms() / P.ct, P.kb, want});
        for (; c >= 2; --c)
            if (P.ct <= max_clusters(kern, smem, c)) break;
        if (c >= 2) {
            ks = c;
            cl = true;
        }
    }
    if (!cl) ks = std::max(1, std::min({kTcKsMax, sms() / P.ct, P.kb}));
    P.ks = ks;
    P.cl = cl ? 1 : 0;
    P.zvec = tcq_aligned(z, 16) ? 1 : 0;
    P.nb0 = nb0;
    P.nb1 = nb1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(P.ct * P.ks);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = P.cl ? P.ks : 1;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = P.cl ? 2 : 1;
    // Workspace: the channel tiles' arrival counters, then kTcKsMax slices of (M, N) INT32 partial sums.
    int* cnt = ws;
    int* part = ws + ((P.ct + 31) & ~31);
    return cudaLaunchKernelEx(&cfg, kern, tmQ, reinterpret_cast<const u16*>(bits), reinterpret_cast<const i8*>(t8), s, rs, z, M, N,
                              K, P, part, cnt) == cudaSuccess ? TCQ_OK : TCQ_ERR_LAUNCH;
}

int check_args(const int8_t* q, const int8_t* W, const void* out, int M, int N, int K) {
    if (!q || !W || !out) return TCQ_ERR_ARG;
    if (M <= 0 || N <= 0 || K <= 0 || (K & 15)) return TCQ_ERR_SHAPE;
    if (!tcq_aligned(q, 16) || !tcq_aligned(W, 16)) return TCQ_ERR_ALIGN;
    return TCQ_OK;
}

}  // namespace

extern "C" {

int tcq_int_mm(const int8_t* q, const int8_t* W, int32_t* acc, int M, int N, int K, void* stream) {
    const int e = check_args(q, W, acc, M, N, K);
    if (e) return e;
    return dispatch<OUT_I32>(q, W, acc, nullptr, nullptr, M, N, K, (cudaStream_t)stream);
}

int tcq_int8_gemm_bias(const int8_t* q, const int8_t* W, const float* s_tok, const float* s_ch, const uint16_t* bias,
                       const uint16_t* act_lut, uint16_t* out, int M, int N, int K, void* stream) {
    const int e = check_args(q, W, out, M, N, K);
    if (e) return e;
    if (!s_tok || !s_ch) return TCQ_ERR_ARG;
    return dispatch<OUT_BF16>(q, W, out, s_tok, s_ch, M, N, K, (cudaStream_t)stream, reinterpret_cast<const u16*>(bias),
                              reinterpret_cast<const u16*>(act_lut));
}

int tcq_int8_gemm(const int8_t* q, const int8_t* W, const float* s_tok, const float* s_ch, void* out, int out_dtype, int M,
                  int N, int K, void* stream) {
    const int e = check_args(q, W, out, M, N, K);
    if (e) return e;
    if (!s_tok || !s_ch) return TCQ_ERR_ARG;
    if (out_dtype == TCQ_DT_BF16) return dispatch<OUT_BF16>(q, W, out, s_tok, s_ch, M, N, K, (cudaStream_t)stream);
    if (out_dtype == TCQ_DT_F32) return dispatch<OUT_F32>(q, W, out, s_tok, s_ch, M, N, K, (cudaStream_t)stream);
    return TCQ_ERR_DTYPE;
}


size_t tcq_gemm_tcq_tc_workspace(int M, int N) {
    if (M <= 0 || N <= 0) return 0;
    return ((size_t)kTcKsMax * M * N + (size_t)(((N + BM - 1) / BM + 31) & ~31)) * sizeof(int);
}

int tcq_gemm_tcq_tc(const uint16_t* bits, const int8_t* t8, const int8_t* q, const float* s, const float* rs, float* z, int M, int N,
                    int K, int nb0, int nb1, void* workspace, size_t workspace_bytes, void* stream) {
    if (!bits || !t8 || !q || !s || !rs || !z) return TCQ_ERR_ARG;
    if (M < 1 || M > 256 || N <= 0 || K <= 0 || (N & 15) || (K & 15)) return TCQ_ERR_SHAPE;
    const int R = N >> 4;
    if ((nb0 < R && (nb0 & 7)) || (nb1 < R && (nb1 & 7)) || nb0 < 0 || nb1 < 0) return TCQ_ERR_SHAPE;   // layers on 128-row tiles
    if (!tcq_aligned(bits, 16) || !tcq_aligned(q, 16) || !tcq_aligned(t8, 16)) return TCQ_ERR_ALIGN;
    if (!workspace || workspace_bytes < tcq_gemm_tcq_tc_workspace(M, N)) return TCQ_ERR_WORKSPACE;
    int* ws = reinterpret_cast<int*>(workspace);
    cudaStream_t st = (cudaStream_t)stream;
    if (M <= 32) return launch_tc<32, 6>(bits, t8, q, s, rs, z, M, N, K, nb0, nb1, ws, st);
    if (M <= 64) return launch_tc<64, 5>(bits, t8, q, s, rs, z, M, N, K, nb0, nb1, ws, st);
    if (M <= 128) return launch_tc<128, 4>(bits, t8, q, s, rs, z, M, N, K, nb0, nb1, ws, st);
    return launch_tc<256, 3>(bits, t8, q, s, rs, z, M, N, K, nb0, nb1, ws, st);
}

int tcq_selftest_wait_expiry(unsigned limit_us, void* stream) {
    if (limit_us == 0 || limit_us > 1000000) return TCQ_ERR_ARG;
    k_wait_expiry<<<1, 32, 0, (cudaStream_t)stream>>>((unsigned long long)limit_us * 1000ull);
    return cudaGetLastError() == cudaSuccess ? TCQ_OK : TCQ_ERR_LAUNCH;
}

int tcq_device_error(int reset) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_tcq_device_error, sizeof(int)) != cudaSuccess) return -1;
    if (reset) {
        const int z = 0;
        if (cudaMemcpyToSymbol(g_tcq_device_error, &z, sizeof(int)) != cudaSuccess) return -1;
    }
    return v;
}

}  // extern "C"
