// Bitshift-trellis 2-bit weights (L = 16, K = 2, V = 2, 16 x 16 tiles, 512 x 2 hashed table) on sm_100a:
// dense decode, decode fused into the small-M product, and the INT8-resident small-M product.
//
// Format (tcq_format.py:3-12, 58-71): a tile is 32 uint16 words = 512 bits, MSB first; the state of weight pair p
// (0..7) of tile row r (0..15) is bits [32 r + 4 p, 32 r + 4 p + 16) of the tile's stream (tail-biting). A state s
// decodes to the pair t8[h], h = ((s + 1) s >> 6) & 511, first coordinate negated when bit 15 of (s + 1) s is set.
//
// Decoding on sm_100a is integer-ALU and shared-memory-port bound, not HBM bound (0.25 bytes of stream per weight),
// so the per-pair work is cut to the bone:
//   * bits 6..15 of x = (s + 1) s, i.e. table index AND sign, are one 10-bit key; the shared-memory table holds all
//     1024 (index, sign) variants, so the sign costs nothing;
//   * the key is taken straight out of 2x = s * (2 s) + 2 s (one IMAD) with a single AND that also yields the byte
//     offset key * 128; states are read from 32-bit funnel shifts of the tile row and need no masking (junk above
//     bit 16 only reaches bits >= 17 of 2x);
//   * the table is replicated once per lane (1024 keys x 32 lanes x 4 bytes = 128 KB), lane l reading bank l, so the
//     random lookups of a warp never conflict;
//   * decoded pairs are packed with one byte_perm per two pairs and consumed by dp4a in registers.
#include <mutex>

#include <algorithm>

#include "rowwalsh.cuh"
#include "trellis_common.cuh"

namespace {

using namespace tcq;

constexpr int kThreads = 512;

// ------------------------------------------------------------------------------------------------------ dense decode
// One thread per tile: its 64 bytes arrive with four 16-byte loads (the next tile of the thread is fetched while this
// one decodes), and its 16 rows leave as 16-byte stores; consecutive threads take consecutive tiles of a tile row, so
// every store instruction of a warp writes 512 contiguous bytes. The grid is persistent (one 128 KB table per CTA).
template <int OUT_BYTES>    // 1: INT8 weights, 2: BF16 weights
__device__ __forceinline__ void decode_tiles(const u16* __restrict__ bits, void* __restrict__ out, int m, int n, const u32* tab) {
    const u32 lane4 = 4u * (threadIdx.x & 31);
    const int tiles = n >> 4;
    const long long total = (long long)(m >> 4) * tiles;
    const long long step = (long long)gridDim.x * blockDim.x;
    long long it = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    u32 Wn[17];
    if (it < total) load_tile_rows<16>(bits, (size_t)it, 0, Wn);
    for (; it < total; it += step) {
        u32 W[17];
#pragma unroll
        for (int a = 0; a < 17; ++a) W[a] = Wn[a];
        if (it + step < total) load_tile_rows<16>(bits, (size_t)(it + step), 0, Wn);
        const int tr = (int)(it / tiles), tc = (int)(it % tiles);
#pragma unroll
        for (int r = 0; r < 16; ++r) {
            const size_t row = (size_t)tr * 16 + r;
            if (OUT_BYTES == 1) {
                u32 w[4];
                row_words_i8(rowA(W[r]), rowA(W[r + 1]), tab, lane4, w);
                *reinterpret_cast<uint4*>(reinterpret_cast<int8_t*>(out) + row * n + 16 * tc) = make_uint4(w[0], w[1], w[2], w[3]);
            } else {
                u32 e[8];
                row_entries(rowA(W[r]), rowA(W[r + 1]), tab, lane4, e);
                uint4* o = reinterpret_cast<uint4*>(reinterpret_cast<u16*>(out) + row * n + 16 * tc);
                o[0] = make_uint4(e[0], e[1], e[2], e[3]);
                o[1] = make_uint4(e[4], e[5], e[6], e[7]);
            }
        }
    }
}

__global__ void __launch_bounds__(kThreads, 1)
k_decode_i8(const u16* __restrict__ bits, const i8* __restrict__ t8, int8_t* __restrict__ out, int m, int n) {
    extern __shared__ __align__(128) u32 tab[];
    __shared__ __align__(16) u16 pairs[512];
    pdl_launch_dependents();
    build_table_i8(tab, pairs, t8);
    __syncthreads();
    pdl_wait();
    decode_tiles<1>(bits, out, m, n, tab);
}

__global__ void __launch_bounds__(kThreads, 1)
k_decode_bf16(const u16* __restrict__ bits, const u16* __restrict__ tb, u16* __restrict__ out, int m, int n) {
    extern __shared__ __align__(128) u32 tab[];
    __shared__ __align__(16) u32 pairs[512];
    pdl_launch_dependents();
    build_table_bf16(tab, pairs, tb);
    __syncthreads();
    pdl_wait();
    decode_tiles<2>(bits, out, m, n, tab);
}

// ------------------------------------------------------------------------------------------------------ fused decode-GEMV
// Work unit = (tile row, K segment of TPU tiles), one warp per unit. Lane (t, g) of a unit decodes rows
// g*RPT .. g*RPT+RPT-1 of tile t and keeps RPT x MT int32 accumulators. Units are split evenly over a persistent grid
// (stream-K). Each CTA sums its units' partial rows in shared memory (integer atomics); a tile row that straddles two
// CTAs is summed in the workspace with global integer atomics, and the CTA that completes it (its arrival brings the
// row's unit count to S) writes z and zeroes the workspace again. Integer sums are exact and associative, so the
// result does not depend on the split. Each warp's first tile is fetched before the table build so the DRAM latency
// hides under it; later tiles are fetched one unit ahead.
struct Parts {
    int n;          // layers with rows (1..3)
    int cta0[4];    // first CTA of layer l; cta0[n] = grid
    int tr0[4];     // first tile row of layer l; tr0[n] = N / 16
    int slot[3];    // table slot (0..2) of layer l in t8
    int uq[3];      // units of layer l per CTA: CTA c of the layer takes uq + (c < ur) units, c * uq + min(c, ur) first
    int ur[3];
    FastDiv fS;     // division by S, the units per tile row
    int pf_lead;    // > 0 (one layer only): CTA c prefetches into L2 the stream of CTA c + pf_lead
};

constexpr int kMaxRows = 24;
constexpr int kUnitBytes = 32 * 64;    // one warp's unit of one-lane-per-tile work: 32 tiles
constexpr int kFxMaxSmem = 220 * 1024; // dynamic shared memory of the decode-GEMV with its pre fused (table + staging + row)
    // tile rows one CTA may touch (the launcher bounds the units per CTA accordingly)

// Sum V = RPT x MT accumulators over the lanes that hold the same row group (lanes differing in bits >= log2(LT)) by
// recursive halving: each exchange step sends half of the remaining values and keeps the other half (16 values over
// 32 lanes: 8 + 4 + 2 + 1 + 1 shuffles instead of 80). On return lane l holds KEEP values; value i is element
// out_index(l, i) (= a * MT + m) of its row group's accumulator array; lanes with writer(l) hold distinct sums.
template <int V, int LT>
struct LaneReduce {
    static constexpr int LOGV = V == 16 ? 4 : V == 8 ? 3 : V == 4 ? 2 : V == 2 ? 1 : 0;
    static constexpr int LOGP = LT == 1 ? 5 : LT == 2 ? 4 : LT == 4 ? 3 : LT == 8 ? 2 : 1;
    static constexpr int STEPS = LOGV < LOGP ? LOGV : LOGP;
    static constexpr int KEEP = V >> STEPS;
    __device__ __forceinline__ static void run(int (&v)[V], int lane) {
#pragma unroll
        for (int j = 0; j < STEPS; ++j) {
            const int o = 16 >> j, half = V >> (j + 1);
            const bool up = (lane & o) != 0;
#pragma unroll
            for (int i = 0; i < half; ++i) {
                const int send = up ? v[i] : v[i + half];
                const int keep = up ? v[i + half] : v[i];
                v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
            }
        }
#pragma unroll
        for (int j = STEPS; j < LOGP; ++j)
#pragma unroll
            for (int i = 0; i < KEEP; ++i) v[i] += __shfl_xor_sync(0xffffffffu, v[i], 16 >> j);
    }
    __device__ __forceinline__ static int out_index(int lane, int i) {
        int idx = i;
#pragma unroll
        for (int j = 0; j < STEPS; ++j)
            if (lane & (16 >> j)) idx += V >> (j + 1);
        return idx;
    }
    __device__ __forceinline__ static bool writer(int lane) {
        int mask = 0;
#pragma unroll
        for (int j = STEPS; j < LOGP; ++j) mask |= 16 >> j;
        return (lane & mask) == 0;
    }
};

__device__ __forceinline__ int atom_add_acq_rel_gpu(int* p, int v) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// FX (M <= 4): the layer's pre runs in the kernel: after the dependency wait every CTA rotates and quantizes the M
// activation rows x (BF16 / F16 / F32) itself (the same transform and quantize_store as the pre kernels, so the same
// bits) into shared memory, and the decode loop reads its activations and token scales from there; the separate pre
// launch and its global round trip disappear. With one token and a power-of-two K the transform's threads start at
// once while the others build the table.
template <int MT, int LT, bool FX>
__global__ void __launch_bounds__(kThreads, 1)
k_gemm_tcq(const u16* __restrict__ bits, const i8* __restrict__ t8, const int* __restrict__ q4, const float* __restrict__ s,
           const float* __restrict__ rs, float* __restrict__ z, int M, int N, int K, Parts parts, int* __restrict__ ws_acc,
           int* __restrict__ ws_cnt, int act_vec, const void* __restrict__ xin, int xdt, const i8* __restrict__ su) {
    constexpr int RPT = 16 / LT;    // tile rows per lane (LT lanes share a tile)
    constexpr int TPU = 32 / LT;    // tiles per unit
    constexpr int RV = 16 * MT;     // partial sums per tile row
    constexpr int V = RPT * MT;     // accumulators per lane
    using Red = LaneReduce<V, LT>;
    extern __shared__ __align__(128) u32 tab[];
    __shared__ __align__(16) u16 pairs[512];
    __shared__ int racc[kMaxRows * RV];
    __shared__ float srs[kMaxRows * 16];           // row scales of this CTA's tile rows
    __shared__ float ss[MT];                       // token scales
    __shared__ float red[32];                      // FX: the quantizer's block maximum
    pdl_launch_dependents();
    // This CTA's layer (selected without dynamic indexing of the parameter arrays).
    int cb = parts.cta0[0], tb = parts.tr0[0], slot = parts.slot[0], uq = parts.uq[0], ur = parts.ur[0];
    if (parts.n > 1 && (int)blockIdx.x >= parts.cta0[1]) {
        cb = parts.cta0[1]; tb = parts.tr0[1]; slot = parts.slot[1]; uq = parts.uq[1]; ur = parts.ur[1];
    }
    if (parts.n > 2 && (int)blockIdx.x >= parts.cta0[2]) {
        cb = parts.cta0[2]; tb = parts.tr0[2]; slot = parts.slot[2]; uq = parts.uq[2]; ur = parts.ur[2];
    }
    // Units (tile row, TPU-tile segment) u = row * S + segment; this CTA takes [ub, ue). No divisions: the split
    // comes from the launcher's quotient / remainder, rows from a multiply-high.
    const int tiles = K >> 4, S = (int)parts.fS.d;
    const int c = blockIdx.x - cb;
    const int ub = c * uq + (c < ur ? c : ur), ue = ub + uq + (c < ur ? 1 : 0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const int tin = lane / LT, rg = lane % LT;
    const u32 lane4 = 4u * lane;
    const int row_first = (int)fdiv(ub, parts.fS);
    const int nrows = ub < ue ? (int)fdiv(ue - 1, parts.fS) - row_first + 1 : 0;

    // FX with one token and a power-of-two K (1024 .. 8192): the first K / 32 threads (the pre threads) start the pre's
    // transform at once, waiting only for the previous kernel, while the other threads request the table and fill it;
    // the two halves meet at the quantizer. Otherwise every thread builds the table, then waits, then runs the pre.
    const int nl = FX && (K & (K - 1)) == 0 && K >= 1024 && K <= 8192 ? 31 - __clz(K) : 0;
    const int PT = nl && M == 1 ? K / 32 : 0;
    const int tq = (int)threadIdx.x - PT;          // index among the threads that build the table
    // The 1 KB table is the CTA's first memory request: the table build waits for it, and under a full HBM stream
    // a request queued behind this CTA's weight loads returns about a microsecond later.
    uint4 t8v = make_uint4(0, 0, 0, 0);
    if (tq >= 0 && tq < 64) t8v = ldg_table_v4(reinterpret_cast<const uint4*>(t8 + 1024 * slot) + tq);
    // The CTAs of a launch start one by one, in index order, as the previous launch's CTAs leave their SMs (over
    // about one launch time). When each CTA has little work, CTA c asks L2 for the stream of CTA c + pf_lead, which
    // starts about a DRAM latency later and then finds its weights in L2 instead of waiting on DRAM.
    if (parts.pf_lead && threadIdx.x == 0) {
        const int c2 = c + parts.pf_lead;
        if (c2 < parts.cta0[1] - parts.cta0[0]) {
            const int b2 = c2 * uq + (c2 < ur ? c2 : ur), e2 = b2 + uq + (c2 < ur ? 1 : 0);
            const int r0 = (int)fdiv(b2, parts.fS), r1 = (int)fdiv(e2 - 1, parts.fS);
            const long long t0 = (long long)(tb + r0) * tiles + (b2 - r0 * S) * TPU;
            const long long t1 = (long long)(tb + r1) * tiles + std::min(tiles, (e2 - 1 - r1 * S) * TPU + TPU);
            const char* p0 = reinterpret_cast<const char*>(bits) + t0 * 64;
            for (long long o = 0; o < (t1 - t0) * 64; o += 65536)
                prefetch_l2_bulk(p0 + o, (unsigned)std::min((t1 - t0) * 64 - o, 65536ll));
        }
    }
    int u = ub + warp;
    int rrel = (int)fdiv(u, parts.fS), seg = u - rrel * S;    // this warp's unit, relative tile row and segment
    // CO (one lane per tile): a warp loads its unit's 2 KB with row-contiguous 16-byte loads (4 cache lines per
    // instruction instead of 16, which would hold up the table request in the load/store pipeline) and turns it
    // into one tile per lane through a 2 KB staging area in shared memory. The staging layout keeps 16-byte chunk c
    // of tile t at chunk c ^ ((t >> 1) & 3): both the row-contiguous stores and the per-tile reads are conflict-free.
    constexpr bool CO = LT == 1;
    char* stage = reinterpret_cast<char*>(tab + kTabBytes / 4) + warp * kUnitBytes;
    auto load_unit = [&](int r, int sg, uint4 (&L)[4]) {
        const uint4* base = reinterpret_cast<const uint4*>(bits + ((size_t)(tb + r) * tiles + (size_t)sg * TPU) * 32);
#pragma unroll
        for (int j = 0; j < 4; ++j)
            L[j] = sg * TPU + 8 * j + (lane >> 2) < tiles ? ldg_stream_v4(base + 32 * j + lane) : make_uint4(0, 0, 0, 0);
    };
    // CO: a unit's 2 KB (Ln, as loaded) -> this lane's tile words W through the warp's staging area.
    auto stage_unit = [&](const uint4 (&L)[4], u32 (&W)[RPT + 1]) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int t = 8 * j + (lane >> 2), c = lane & 3;
            *reinterpret_cast<uint4*>(stage + 64 * t + 16 * (c ^ ((t >> 1) & 3))) = L[j];
        }
        __syncwarp();
        const char* mine = stage + 64 * lane;
        const int x = (lane >> 1) & 3;
        const uint4 c0 = *reinterpret_cast<const uint4*>(mine + 16 * (0 ^ x)), c1 = *reinterpret_cast<const uint4*>(mine + 16 * (1 ^ x)),
                    c2 = *reinterpret_cast<const uint4*>(mine + 16 * (2 ^ x)), c3 = *reinterpret_cast<const uint4*>(mine + 16 * (3 ^ x));
        __syncwarp();
        const u32 all[16] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w, c2.x, c2.y, c2.z, c2.w, c3.x, c3.y, c3.z, c3.w};
#pragma unroll
        for (int a = 0; a <= RPT; ++a) W[a] = all[a & 15];
    };
    u32 Wn[RPT + 1];
    uint4 Ln[4];
    if (u < ue) {
        const int tc = seg * TPU + tin;
        if (CO) load_unit(rrel, seg, Ln);                                      // weights: before the wait
        else if (tc < tiles) load_tile_rows<RPT>(bits, (size_t)(tb + rrel) * tiles + tc, rg, Wn);
    }
    for (int i = threadIdx.x; i < nrows * RV; i += blockDim.x) racc[i] = 0;
    // Epilogue operands are fetched now and held in registers until the decode is done, so that their latency hides
    // behind it: the row scales (layer constants) before the dependency wait, the token scales right after it.
    const int nrs = nrows * 16;                    // <= kMaxRows * 16 <= kThreads
    const float rsv = (int)threadIdx.x < nrs ? __ldg(rs + (size_t)(tb + row_first) * 16 + threadIdx.x) : 0.f;
    // FX: the pre of the M rows into shared memory (Walsh buffer, then q4 words (K/4, M) and ss).
    float* sbuf = reinterpret_cast<float*>(reinterpret_cast<char*>(tab + kTabBytes / 4) + (CO ? (kThreads / 32) * kUnitBytes : 0));
    int* sq4 = reinterpret_cast<int*>(sbuf + K + K / 8);   // (the windowed transform's exchange area: K + K / 8 floats)
    const size_t es = xdt == TCQ_DT_F32 ? 4 : 2;
    float mx = 0.f;
    // Power-of-two widths: the register-window transform of token row m on the first K / 32 threads (a named barrier
    // among them): the scaled result into sbuf, its absolute maximum into mx.
    auto pre_win_row = [&](int m) {
        const char* xr = reinterpret_cast<const char*>(xin) + (size_t)m * K * es;
        auto pre_win = [&](auto nlc) {
            constexpr int NL = decltype(nlc)::value, V = rot_vec<NL>(), G = 1 << Win2<NL, V>::WB;
            const int t = threadIdx.x;
            if (t < (1 << NL) / 32) {
                float v[32], sg[32];
                if (xdt == TCQ_DT_BF16) loadc<TCQ_DT_BF16, 32>(xr + (size_t)32 * t * es, v);
                else if (xdt == TCQ_DT_F16) loadc<TCQ_DT_F16, 32>(xr + (size_t)32 * t * es, v);
                else loadc<TCQ_DT_F32, 32>(xr + (size_t)32 * t * es, v);
                load_signsc<32, true>(su + 32 * t, sg);
#pragma unroll
                for (int k = 0; k < 32; ++k) v[k] = v[k] * sg[k];
                win_walsh<NL, true, 2>(v, sbuf, t);
                blk_sync<2, (1 << NL) / 32>();          // the transform's last reads of sbuf are done
                const float sc = wscale(1 << NL);
#pragma unroll
                for (int qq = 0; qq < G; ++qq) {
                    const int e = win_elem<NL>(t, qq, 0);
#pragma unroll
                    for (int k = 0; k < V; ++k) {
                        const float o = v[V * qq + k] * sc;
                        sbuf[swz(e + k)] = o;
                        mx = fmaxf(mx, fabsf(o));
                    }
                }
            }
        };
        switch (nl) {
            case 10: pre_win(std::integral_constant<int, 10>{}); break;
            case 11: pre_win(std::integral_constant<int, 11>{}); break;
            case 12: pre_win(std::integral_constant<int, 12>{}); break;
            default: pre_win(std::integral_constant<int, 13>{}); break;
        }
    };
    if (PT == 0) {
        if (threadIdx.x < 64) reinterpret_cast<uint4*>(pairs)[threadIdx.x] = t8v;
        __syncthreads();
        fill_table_i8_nt<kThreads>(tab, pairs);
    } else if ((int)threadIdx.x < PT) {
        if constexpr (FX) {
            pdl_wait();                            // the activations come from the previous kernel
            pre_win_row(0);
        }
    } else {
        if (tq < 64) reinterpret_cast<uint4*>(pairs)[tq] = t8v;
        asm volatile("barrier.sync 2, %0;" ::"r"(kThreads - PT) : "memory");
        fill_table_i8_span(tab, pairs, tq, kThreads - PT);
    }
    __syncthreads();
    pdl_wait();                                    // activations / scales come from the previous kernel
    const float sv = !FX && (int)threadIdx.x < M && threadIdx.x < MT ? s[threadIdx.x] : 0.f;
    if constexpr (FX) {
        if (PT) {
            quantize_store(sbuf, mx, red, nullptr, sq4, ss, 0, K, M);
            __syncthreads();                       // sq4 / ss complete
        }
        for (int m = 0; m < M && !PT; ++m) {
            const char* xr = reinterpret_cast<const char*>(xin) + (size_t)m * K * es;
            mx = 0.f;
            if (nl) {
                pre_win_row(m);                    // the other threads wait at the quantizer's block barrier
                quantize_store(sbuf, mx, red, nullptr, sq4, ss, m, K, M);
                __syncthreads();                   // sbuf is rewritten by the next row; sq4 / ss complete
                continue;
            }
            // Chunks of 4: a few rows on 512 threads, where per-thread latency bounds the transform.
            row_walshc<4>(sbuf, K,
                          [&](int cc, float* v) {
                              float sg[4];
                              if (xdt == TCQ_DT_BF16) loadc<TCQ_DT_BF16, 4>(xr + (size_t)4 * cc * es, v);
                              else if (xdt == TCQ_DT_F16) loadc<TCQ_DT_F16, 4>(xr + (size_t)4 * cc * es, v);
                              else loadc<TCQ_DT_F32, 4>(xr + (size_t)4 * cc * es, v);
                              load_signsc<4, true>(su + 4 * cc, sg);
#pragma unroll
                              for (int k = 0; k < 4; ++k) v[k] = v[k] * sg[k];
                          },
                          [&](int i0, const float* v) { store_chunk<4>(sbuf, i0, v, mx); },
                          [&](int i, float v) { sbuf[swz(i)] = v; mx = fmaxf(mx, fabsf(v)); });
            quantize_store(sbuf, mx, red, nullptr, sq4, ss, m, K, M);
            __syncthreads();                       // sbuf is rewritten by the next row; sq4 / ss complete
        }
    }
    const int* qsrc = FX ? sq4 : q4;
    for (; u < ue; u += nw) {
        const int tc = seg * TPU + tin;
        u32 W[RPT + 1];
        int rn = rrel, sn = seg + nw;              // the warp's next unit
        while (sn >= S) { sn -= S; ++rn; }
        if constexpr (CO) {
            stage_unit(Ln, W);
            if (u + nw < ue) load_unit(rn, sn, Ln);
        } else {
#pragma unroll
            for (int a = 0; a <= RPT; ++a) W[a] = Wn[a];
            if (u + nw < ue) {
                const int tcn = sn * TPU + tin;
                if (tcn < tiles) load_tile_rows<RPT>(bits, (size_t)(tb + rn) * tiles + tcn, rg, Wn);
            }
        }
        int acc[V];
#pragma unroll
        for (int i = 0; i < V; ++i) acc[i] = 0;
        // CO: tiles past the end of the tile row hold zero words and get zero activations, so the decode runs on
        // every lane without a branch (their products add nothing).
        if (CO || tc < tiles) {
            int act[4][MT];
            const int* qa = qsrc + (size_t)4 * tc * M;
            if (MT == 1 && act_vec) {
                int4 v = make_int4(0, 0, 0, 0);
                if (!CO || tc < tiles) v = FX ? *reinterpret_cast<const int4*>(qa) : __ldg(reinterpret_cast<const int4*>(qa));
                act[0][0] = v.x; act[1][0] = v.y; act[2][0] = v.z; act[3][0] = v.w;
            } else {
#pragma unroll
                for (int e = 0; e < 4; ++e)
#pragma unroll
                    for (int m = 0; m < MT; ++m)
                        act[e][m] = (m < M && tc < tiles) ? (FX ? qa[e * M + m] : __ldg(qa + e * M + m)) : 0;
            }
#pragma unroll
            for (int a = 0; a < RPT; ++a) {
                u32 w[4];
                row_words_i8(rowA(W[a]), rowA(W[a + 1]), tab, lane4, w);
#pragma unroll
                for (int e = 0; e < 4; ++e)
#pragma unroll
                    for (int m = 0; m < MT; ++m) acc[a * MT + m] = __dp4a((int)w[e], act[e][m], acc[a * MT + m]);
            }
        }
        Red::run(acc, lane);
        if (Red::writer(lane)) {
            int* ra = racc + (rrel - row_first) * RV + rg * RPT * MT;
#pragma unroll
            for (int i = 0; i < Red::KEEP; ++i) {
                const int idx = Red::out_index(lane, i);
                if (idx % MT < M) atomicAdd(ra + idx, acc[i]);
            }
        }
        rrel = rn;
        seg = sn;
    }
    if ((int)threadIdx.x < nrs) srs[threadIdx.x] = rsv;
    if (!FX && threadIdx.x < MT) ss[threadIdx.x] = sv;
    __syncthreads();
    for (int r = warp; r < nrows; r += nw) {
        const int rrel = row_first + r, trow = tb + rrel;
        const int a0 = rrel * S, a1 = a0 + S;
        const int* src = racc + r * RV;
        const float* rsr = srs + r * 16;
        if (a0 >= ub && a1 <= ue) {                // the whole tile row was summed here
            for (int i = lane; i < RV; i += 32) {
                const int rr = i / MT, m = i % MT, row = trow * 16 + rr;
                if (m < M) z[(size_t)m * N + row] = ((float)src[i] * ss[m]) * rsr[rr];
            }
            continue;
        }
        // A tile row split between CTAs: add this CTA's part in the workspace; the CTA whose arrival completes the
        // row's S units finishes it. Release / acquire on the arrival counter orders the sums (no full fence).
        const int mine = (a1 < ue ? a1 : ue) - (a0 > ub ? a0 : ub);
        for (int i = lane; i < RV; i += 32) {
            const int rr = i / MT, m = i % MT;
            if (m < M) atomicAdd(ws_acc + (size_t)m * N + trow * 16 + rr, src[i]);
        }
        __syncwarp();
        int last = 0;
        if (lane == 0) last = atom_add_acq_rel_gpu(ws_cnt + trow, mine) + mine == S;
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
            constexpr int IT = (RV + 31) / 32;
            int v[IT];
#pragma unroll
            for (int j = 0; j < IT; ++j) {                // read and clear: all of a lane's requests in flight at once
                const int i = lane + 32 * j, rr = i / MT, m = i % MT;
                v[j] = i < RV && m < M ? atomicExch(ws_acc + (size_t)m * N + trow * 16 + rr, 0) : 0;
            }
#pragma unroll
            for (int j = 0; j < IT; ++j) {
                const int i = lane + 32 * j, rr = i / MT, m = i % MT;
                if (i < RV && m < M) z[(size_t)m * N + trow * 16 + rr] = ((float)v[j] * ss[m]) * rsr[rr];
            }
            if (lane == 0) ws_cnt[trow] = 0;
        }
    }
}

// ------------------------------------------------------------------------------------------------------ INT8-resident GEMV
// One warp per RPW output rows; lanes stride over K in 16-byte chunks, UNR chunks per lane per step with all weight
// loads issued before the products; the activations are staged in shared memory token-major (sq[m][K/4]) so that a
// lane's 16 inputs of one token are one conflict-free 16-byte load.
template <int MT, int RPW>
__global__ void __launch_bounds__(256)
k_gemm_w8(const int8_t* __restrict__ W, const int* __restrict__ q4, const float* __restrict__ s, const float* __restrict__ rs,
          float* __restrict__ z, int M, int N, int K) {
    constexpr int UNR = 4;
    extern __shared__ __align__(16) int sq[];
    const int words = K >> 2;
    const int lane = threadIdx.x & 31;
    const int row0 = (blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * RPW;
    const int chunks = K >> 4;
    pdl_launch_dependents();
    pdl_wait();                     // W itself may come from the previous kernel (per-chunk decode of the hybrid runtime)
    uint4 w[UNR][RPW];
#pragma unroll
    for (int u = 0; u < UNR; ++u)
#pragma unroll
        for (int a = 0; a < RPW; ++a) {
            const int j = lane + 32 * u;
            w[u][a] = (row0 + a < N && j < chunks) ? ldg_stream_v4(W + (size_t)(row0 + a) * K + 16 * j) : make_uint4(0, 0, 0, 0);
        }
    for (int i = threadIdx.x; i < words * M; i += blockDim.x) {
        const int j = i / M, m = i % M;
        sq[m * words + j] = q4[i];
    }
    __syncthreads();
    if (row0 >= N) return;
    int acc[RPW][MT];
#pragma unroll
    for (int a = 0; a < RPW; ++a)
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[a][m] = 0;
    for (int j0 = lane; j0 < chunks; j0 += 32 * UNR) {
        uint4 cur[UNR][RPW];
#pragma unroll
        for (int u = 0; u < UNR; ++u)
#pragma unroll
            for (int a = 0; a < RPW; ++a) cur[u][a] = w[u][a];
#pragma unroll
        for (int u = 0; u < UNR; ++u)
#pragma unroll
            for (int a = 0; a < RPW; ++a) {
                const int j = j0 + 32 * UNR + 32 * u;
                w[u][a] = (row0 + a < N && j < chunks) ? ldg_stream_v4(W + (size_t)(row0 + a) * K + 16 * j) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
        for (int u = 0; u < UNR; ++u) {
            const int j = j0 + 32 * u;
            if (j < chunks) {
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                    if (m < M) {
                        const int4 x = *reinterpret_cast<const int4*>(sq + m * words + 4 * j);
#pragma unroll
                        for (int a = 0; a < RPW; ++a) {
                            acc[a][m] = __dp4a((int)cur[u][a].x, x.x, acc[a][m]);
                            acc[a][m] = __dp4a((int)cur[u][a].y, x.y, acc[a][m]);
                            acc[a][m] = __dp4a((int)cur[u][a].z, x.z, acc[a][m]);
                            acc[a][m] = __dp4a((int)cur[u][a].w, x.w, acc[a][m]);
                        }
                    }
                }
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int a = 0; a < RPW; ++a)
#pragma unroll
            for (int m = 0; m < MT; ++m) acc[a][m] += __shfl_xor_sync(0xffffffffu, acc[a][m], o);
    if (lane == 0) {
#pragma unroll
        for (int a = 0; a < RPW; ++a)
#pragma unroll
            for (int m = 0; m < MT; ++m)
                if (m < M && row0 + a < N) z[(size_t)m * N + row0 + a] = ((float)acc[a][m] * s[m]) * rs[row0 + a];
    }
}

int g_sms = 0;

int num_sms() {
    if (g_sms == 0) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess) return 148;
        if (cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || g_sms <= 0) g_sms = 148;
    }
    return g_sms;
}

template <class Kern>
int set_smem(Kern k, int bytes) {
    return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) == cudaSuccess ? 0 : TCQ_ERR_LAUNCH;
}

template <class Kern, class... Args>
int launch_pdl(Kern kern, int grid, int smem, cudaStream_t st, Args... args) {
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

int decode_grid(int m, int n) {
    const long long tiles = (long long)(m >> 4) * (n >> 4);
    long long grid = (tiles + kThreads - 1) / kThreads;
    return (int)(grid < num_sms() ? grid : num_sms());
}

template <int MT, int LT>
int launch_gemm_tcq(const uint16_t* bits, const int8_t* t8, const int32_t* q4, const float* s, const float* rs, float* z,
                    int M, int N, int K, int nb0, int nb1, int* ws, cudaStream_t st, const void* xin = nullptr, int xdt = 0,
                    const int8_t* su = nullptr) {
    const int TPU = 32 / LT, tiles = K >> 4, S = (tiles + TPU - 1) / TPU, R = N >> 4;
    Parts p{};
    int bounds[4] = {0, nb0 < R ? nb0 : R, nb1 < R ? nb1 : R, R};
    if (bounds[2] < bounds[1]) bounds[2] = bounds[1];
    int nl = 0;
    int rows[3];
    for (int l = 0; l < 3; ++l) rows[l] = bounds[l + 1] - bounds[l];
    const int sms = num_sms();
    const long long U = (long long)R * S;
    if (U >= (1ll << 31)) return TCQ_ERR_SHAPE;
    int cta = 0;
    for (int l = 0; l < 3; ++l) {
        if (rows[l] <= 0) continue;
        const long long Ul = (long long)rows[l] * S;
        long long g = (sms * Ul + U - 1) / U;
        // Whole tile rows per CTA need no cross-CTA finish; take that split when its imbalance against the even
        // stream-K split is at most 20 %.
        const long long rows_per = (rows[l] + g - 1) / g;
        if (rows_per * g * 5 <= (long long)rows[l] * 6 && rows_per <= kMaxRows) g = (rows[l] + rows_per - 1) / rows_per;
        const long long gmin = (Ul + (long long)(kMaxRows - 2) * S - 1) / ((long long)(kMaxRows - 2) * S);   // rows per CTA <= kMaxRows
        if (g < gmin) g = gmin;
        if (g < 1) g = 1;
        if (g > Ul) g = Ul;
        p.cta0[nl] = cta;
        p.tr0[nl] = bounds[l];
        p.slot[nl] = l;
        p.uq[nl] = (int)(Ul / g);
        p.ur[nl] = (int)(Ul % g);
        cta += (int)g;
        ++nl;
    }
    p.n = nl;
    p.cta0[nl] = cta;
    p.tr0[nl] = R;
    p.fS = make_fastdiv((unsigned)S);
    int max_units = 0;
    for (int l = 0; l < nl; ++l) max_units = std::max(max_units, p.uq[l] + (p.ur[l] > 0 ? 1 : 0));
    p.pf_lead = nl == 1 && max_units <= 2 * (kThreads / 32) ? std::max(1, (cta * 5) / 16) : 0;
    const bool fx = xin != nullptr;
    auto kern = fx ? k_gemm_tcq<MT, LT, (MT <= 4)> : k_gemm_tcq<MT, LT, false>;
    const int smem = kTabBytes + (LT == 1 ? (kThreads / 32) * kUnitBytes : 0) + (fx ? K * 4 + K / 2 + K * MT : 0);
    if (fx && (MT > 4 || smem > kFxMaxSmem)) return TCQ_ERR_SHAPE;
    if (set_smem(kern, smem)) return TCQ_ERR_LAUNCH;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cta);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int* ws_acc = ws;
    int* ws_cnt = ws + (size_t)M * N;
    const int act_vec = fx || tcq_aligned(q4, 16) ? 1 : 0;
    if (cudaLaunchKernelEx(&cfg, kern, reinterpret_cast<const u16*>(bits), reinterpret_cast<const i8*>(t8), q4, s, rs, z,
                           M, N, K, p, ws_acc, ws_cnt, act_vec, xin, xdt, reinterpret_cast<const i8*>(su)) != cudaSuccess)
        return TCQ_ERR_LAUNCH;
    return TCQ_OK;
}

// Lanes per tile: for M = 1, one lane per tile (fewest instructions per weight) once the layer has at least 3/4 as
// many tiles as the machine has threads (4096 x 4096 and up); on smaller layers two or four lanes split a tile's
// rows so that every warp still gets work. M <= 4: 4 lanes; larger M: one lane per token slot (MT lanes).
int dispatch_gemm_tcq(const uint16_t* bits, const int8_t* t8, const int32_t* q4, const float* s, const float* rs, float* z, int M,
                      int N, int K, int nb0, int nb1, int* ws, cudaStream_t st, const void* xin = nullptr, int xdt = 0,
                      const int8_t* su = nullptr) {
    const long long tiles = (long long)(N >> 4) * (K >> 4), lanes = (long long)num_sms() * kThreads;
#define TCQ_GEMV(MT, LT) launch_gemm_tcq<MT, LT>(bits, t8, q4, s, rs, z, M, N, K, nb0, nb1, ws, st, xin, xdt, su)
    if (M == 1 && tiles * 4 >= lanes * 3) return TCQ_GEMV(1, 1);
    if (M == 1 && tiles * 8 >= lanes * 3) return TCQ_GEMV(1, 2);
    if (M == 1) return TCQ_GEMV(1, 4);
    if (M == 2) return TCQ_GEMV(2, 4);
    if (M <= 4) return TCQ_GEMV(4, 4);
    if (M <= 8) return TCQ_GEMV(8, 8);
    return TCQ_GEMV(16, 16);
#undef TCQ_GEMV
}

template <int MT, int RPW>
int launch_gemm_w8(const int8_t* W, const int32_t* q4, const float* s, const float* rs, float* z, int M, int N, int K,
                   cudaStream_t st) {
    auto kern = k_gemm_w8<MT, RPW>;
    const int smem = K * M;
    if (smem > 46 * 1024 && set_smem(kern, smem)) return TCQ_ERR_LAUNCH;
    const int rows_per_cta = (256 / 32) * RPW;
    const int grid = (N + rows_per_cta - 1) / rows_per_cta;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, W, q4, s, rs, z, M, N, K) == cudaSuccess ? TCQ_OK : TCQ_ERR_LAUNCH;
}


// ------------------------------------------------------------------------------------------------------ no-allocation variant
// Scratch of tcq_gemm_tcq_noalloc: a fixed file-scope device array (every GPU that loads this library holds it, about
// 2 MiB, until the process exits) instead of a caller-provided workspace. Host code must not pass the array's name to
// a kernel (on the host it is only a stand-in symbol); the device address is looked up once per device with
// cudaGetSymbolAddress, with that device current.
constexpr int kNoAllocMaxMN = 16 * 32768;   // M * N limit (M <= 16, N <= 32768)
constexpr int kNoAllocMaxN = 32768;
static __device__ __align__(256) int g_gemv_scratch[kNoAllocMaxMN + kNoAllocMaxN / 16];

constexpr int kMaxDevices = 64;
int* g_scratch_addr[kMaxDevices];
std::mutex g_scratch_mu;

// The address is looked up again on every call whose stream is not capturing (a host-side lookup once the module is
// loaded), so a device reset that reloads the module never leaves a stale address behind; during a capture the last
// address looked up on this device is used.
int scratch_for_current_device(int** out, cudaStream_t st) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return TCQ_ERR_DEVICE;
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cap) != cudaSuccess) return TCQ_ERR_DEVICE;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_addr[dev] || cap == cudaStreamCaptureStatusNone) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_gemv_scratch) != cudaSuccess || !p) return TCQ_ERR_DEVICE;
        g_scratch_addr[dev] = reinterpret_cast<int*>(p);
    }
    *out = g_scratch_addr[dev];
    return TCQ_OK;
}
}  // namespace

extern "C" {

int tcq_decode(const uint16_t* bits, const int8_t* t8, int8_t* out, int m, int n, void* stream) {
    if (!bits || !t8 || !out) return TCQ_ERR_ARG;
    if (m <= 0 || n <= 0 || (m & 15) || (n & 15)) return TCQ_ERR_SHAPE;
    if (!tcq_aligned(bits, 16) || !tcq_aligned(out, 16) || !tcq_aligned(t8, 16)) return TCQ_ERR_ALIGN;
    if (set_smem(k_decode_i8, kTabBytes)) return TCQ_ERR_LAUNCH;
    return launch_pdl(k_decode_i8, decode_grid(m, n), kTabBytes, (cudaStream_t)stream, reinterpret_cast<const u16*>(bits),
                      reinterpret_cast<const i8*>(t8), out, m, n);
}

int tcq_decode_bf16(const uint16_t* bits, const uint16_t* tb, uint16_t* out, int m, int n, void* stream) {
    if (!bits || !tb || !out) return TCQ_ERR_ARG;
    if (m <= 0 || n <= 0 || (m & 15) || (n & 15)) return TCQ_ERR_SHAPE;
    if (!tcq_aligned(bits, 16) || !tcq_aligned(out, 16) || !tcq_aligned(tb, 16)) return TCQ_ERR_ALIGN;
    if (set_smem(k_decode_bf16, kTabBytes)) return TCQ_ERR_LAUNCH;
    return launch_pdl(k_decode_bf16, decode_grid(m, n), kTabBytes, (cudaStream_t)stream, reinterpret_cast<const u16*>(bits), tb,
                      out, m, n);
}

size_t tcq_gemm_tcq_workspace(int M, int N) {
    if (M <= 0 || N <= 0) return 0;
    return ((size_t)M * N + (size_t)(N >> 4)) * sizeof(int);
}

int tcq_gemm_tcq(const uint16_t* bits, const int8_t* t8, const int32_t* q4, const float* s, const float* rs, float* z,
                 int M, int N, int K, int nb0, int nb1, void* workspace, size_t workspace_bytes, void* stream) {
    if (!bits || !t8 || !q4 || !s || !rs || !z) return TCQ_ERR_ARG;
    if (M < 1 || M > 16 || N <= 0 || K <= 0 || (N & 15) || (K & 15)) return TCQ_ERR_SHAPE;
    if (!tcq_aligned(bits, 16) || !tcq_aligned(q4, 4) || !tcq_aligned(t8, 16)) return TCQ_ERR_ALIGN;
    if (!workspace || workspace_bytes < tcq_gemm_tcq_workspace(M, N)) return TCQ_ERR_WORKSPACE;
    if (nb0 < 0 || nb1 < 0) return TCQ_ERR_ARG;
    int* ws = reinterpret_cast<int*>(workspace);
    cudaStream_t st = (cudaStream_t)stream;
    return dispatch_gemm_tcq(bits, t8, q4, s, rs, z, M, N, K, nb0, nb1, ws, st);
}

int tcq_gemm_tcq_x(const uint16_t* bits, const int8_t* t8, const void* x, int x_dtype, const int8_t* su, const float* rs,
                   float* z, int M, int N, int K, int nb0, int nb1, void* workspace, size_t workspace_bytes, void* stream) {
    if (!bits || !t8 || !x || !su || !rs || !z) return TCQ_ERR_ARG;
    if (x_dtype != TCQ_DT_BF16 && x_dtype != TCQ_DT_F16 && x_dtype != TCQ_DT_F32) return TCQ_ERR_DTYPE;
    if (M < 1 || M > 4 || N <= 0 || K <= 0 || (N & 15) || (K & 15) || K > 8192) return TCQ_ERR_SHAPE;
    if (!tcq_aligned(bits, 16) || !tcq_aligned(t8, 16) || !tcq_aligned(x, 16) || !tcq_aligned(su, 16)) return TCQ_ERR_ALIGN;
    if (!workspace || workspace_bytes < tcq_gemm_tcq_workspace(M, N)) return TCQ_ERR_WORKSPACE;
    if (nb0 < 0 || nb1 < 0) return TCQ_ERR_ARG;
    return dispatch_gemm_tcq(bits, t8, nullptr, nullptr, rs, z, M, N, K, nb0, nb1, reinterpret_cast<int*>(workspace),
                             (cudaStream_t)stream, x, x_dtype, su);
}

int tcq_gemm_w8(const int8_t* W, const int32_t* q4, const float* s, const float* rs, float* z, int M, int N, int K,
                void* stream) {
    if (!W || !q4 || !s || !rs || !z) return TCQ_ERR_ARG;
    if (M < 1 || M > 16 || N <= 0 || K <= 0 || (K & 15)) return TCQ_ERR_SHAPE;
    if ((size_t)K * M > 200 * 1024) return TCQ_ERR_SHAPE;
    if (!tcq_aligned(W, 16) || !tcq_aligned(q4, 4)) return TCQ_ERR_ALIGN;
    cudaStream_t st = (cudaStream_t)stream;
    if (M == 1) return launch_gemm_w8<1, 2>(W, q4, s, rs, z, M, N, K, st);
    if (M == 2) return launch_gemm_w8<2, 2>(W, q4, s, rs, z, M, N, K, st);
    if (M <= 4) return launch_gemm_w8<4, 2>(W, q4, s, rs, z, M, N, K, st);
    if (M <= 8) return launch_gemm_w8<8, 1>(W, q4, s, rs, z, M, N, K, st);
    return launch_gemm_w8<16, 1>(W, q4, s, rs, z, M, N, K, st);
}

size_t tcq_gemm_tcq_noalloc_max_elements(void) { return (size_t)kNoAllocMaxMN; }

// Fused decode-GEMV for callers that cannot allocate device memory: identical arguments and results to tcq_gemm_tcq,
// without the workspace. Callers in this position are, for example, a robot's real-time control loop that must not
// call cudaMalloc (it may synchronize the device and take an unbounded time in the middle of an action step), or a
// host framework's plugin interface that owns every device buffer and hands the plugin only its inputs and outputs.
// The stream-K scratch is the fixed array g_gemv_scratch; its device address is looked up on every call outside a
// stream capture, and a call inside a capture uses the address of the last call on that device (so the first call on
// a device should come before any stream capture). Limits: 1 <= M <= 16, N <= 32768, M * N <= 524288; larger shapes
// return TCQ_ERR_SHAPE. All calls share the one array per device: the used part is cleared (cudaMemsetAsync, no
// allocation) on the caller's stream before the kernel, and calls that overlap on the GPU (other streams, other host
// threads) race on it. If the kernel launch itself then fails (TCQ_ERR_LAUNCH), that clear is already queued; it
// touches only the library's own array. Allocates nothing: no cudaMalloc / cudaFree / library allocation.
int tcq_gemm_tcq_noalloc(const uint16_t* bits, const int8_t* t8, const int32_t* q4, const float* s, const float* rs, float* z,
                         int M, int N, int K, int nb0, int nb1, void* stream) {
    if (!bits || !t8 || !q4 || !s || !rs || !z) return TCQ_ERR_ARG;
    if (M < 1 || M > 16 || N <= 0 || K <= 0 || (N & 15) || (K & 15)) return TCQ_ERR_SHAPE;
    if (N > kNoAllocMaxN || (long long)M * N > kNoAllocMaxMN) return TCQ_ERR_SHAPE;
    if (!tcq_aligned(bits, 16) || !tcq_aligned(q4, 4) || !tcq_aligned(t8, 16)) return TCQ_ERR_ALIGN;
    if (nb0 < 0 || nb1 < 0) return TCQ_ERR_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    int* ws = nullptr;
    const int e = scratch_for_current_device(&ws, st);
    if (e) return e;
    if (cudaMemsetAsync(ws, 0, tcq_gemm_tcq_workspace(M, N), st) != cudaSuccess) return TCQ_ERR_LAUNCH;
    return dispatch_gemm_tcq(bits, t8, q4, s, rs, z, M, N, K, nb0, nb1, ws, st);
}

}  // extern "C"

