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

#include "tcq_common.cuh"

namespace {

constexpr int kTabBytes = 1024 * 32 * 4;   // per-lane replicated decode table
constexpr int kThreads = 512;

// Table entry for key k (bits 6..15 of x): pair index k & 511, sign k >> 9.
// INT8 entry: byte 0 = (sign ? -v0 : v0), byte 1 = v1. The 1 KB source table is staged through shared memory with one
// 16-byte load per thread (one memory round trip), then the 128 KB replicated table is written with consecutive
// 16-byte stores (lanes of a warp cover 512 contiguous bytes: no bank conflicts).
__device__ __forceinline__ void stage_pairs(u16* pairs, const void* __restrict__ src) {
    if (threadIdx.x < 64) reinterpret_cast<uint4*>(pairs)[threadIdx.x] = __ldg(reinterpret_cast<const uint4*>(src) + threadIdx.x);
    __syncthreads();
}

__device__ __forceinline__ void build_table_i8(u32* tab, u16* pairs, const i8* __restrict__ t8) {
    stage_pairs(pairs, t8);
    uint4* t4 = reinterpret_cast<uint4*>(tab);
    for (int i = threadIdx.x; i < 1024 * 8; i += blockDim.x) {
        const int k = i >> 3;
        const u32 pr = pairs[k & 511];
        const u32 v0 = (k >> 9) ? ((0u - pr) & 0xffu) : (pr & 0xffu);
        const u32 e = v0 | (pr & 0xff00u);
        t4[i] = make_uint4(e, e, e, e);
    }
}

// BF16 entry: low half = BF16(v0) with the sign bit flipped for sign keys, high half = BF16(v1) (kernels.py:320-337).
// pairs: 512 staged (v0, v1) BF16 pairs (2 KB, staged with one 16-byte load by each of 128 threads).
__device__ __forceinline__ void build_table_bf16(u32* tab, u32* pairs, const u16* __restrict__ tb) {
    if (threadIdx.x < 128) reinterpret_cast<uint4*>(pairs)[threadIdx.x] = __ldg(reinterpret_cast<const uint4*>(tb) + threadIdx.x);
    __syncthreads();
    uint4* t4 = reinterpret_cast<uint4*>(tab);
    for (int i = threadIdx.x; i < 1024 * 8; i += blockDim.x) {
        const int k = i >> 3;
        const u32 e = pairs[k & 511] ^ ((u32)(k >> 9) << 15);
        t4[i] = make_uint4(e, e, e, e);
    }
}

// Table lookup of this lane's copy: byte offset (key * 128) | (4 * lane) from the shared table `tab` (the key offset
// has bits 7..16, the lane offset bits 2..6, so one OR joins them; the constant shared base is added by the compiler).
__device__ __forceinline__ u32 lut(const u32* tab, u32 lane4, u32 off) {
    return *reinterpret_cast<const u32*>(reinterpret_cast<const char*>(tab) + (off | lane4));
}

// Byte offset key * 128 of the state in the upper half of F: v = F >> 16 taken as the high word of F * 2^16 (multiply
// pipe), 2x = v * 2v + 2v, bits 7..16 of 2x = bits 6..15 of x = key.
__device__ __forceinline__ u32 off_hi(u32 F) {
    const u32 v = __umulhi(F, 65536u), u = v * 2u;
    return (v * u + u) & 0x1FF80u;
}
// Byte offset of the state in the lower half of F (bits above 16 are junk and drop out of bits 7..16 of 2x).
__device__ __forceinline__ u32 off_lo(u32 F) {
    const u32 u = F * 2u;
    return (F * u + u) & 0x1FF80u;
}

// The 8 table entries of one tile row. A = (w[2r] << 16) | w[2r+1], B = (w[2r+2] << 16) | w[2r+3] (words mod 32):
// F_p = bits [4p, 4p + 32) of the row's window, so its upper half is state p and its lower half state p + 4.
__device__ __forceinline__ void row_entries(u32 A, u32 B, const u32* tab, u32 lane4, u32 (&e)[8]) {
    const u32 F1 = __funnelshift_l(B, A, 4), F2 = __funnelshift_l(B, A, 8), F3 = __funnelshift_l(B, A, 12);
    e[0] = lut(tab, lane4, off_hi(A));
    e[1] = lut(tab, lane4, off_hi(F1));
    e[2] = lut(tab, lane4, off_hi(F2));
    e[3] = lut(tab, lane4, off_hi(F3));
    e[4] = lut(tab, lane4, off_lo(A));
    e[5] = lut(tab, lane4, off_lo(F1));
    e[6] = lut(tab, lane4, off_lo(F2));
    e[7] = lut(tab, lane4, off_lo(F3));
}

// INT8 weights of one tile row as 4 little-endian words (columns 4j .. 4j+3 in word j).
__device__ __forceinline__ void row_words_i8(u32 A, u32 B, const u32* tab, u32 lane4, u32 (&w)[4]) {
    u32 e[8];
    row_entries(A, B, tab, lane4, e);
#pragma unroll
    for (int j = 0; j < 4; ++j) w[j] = __byte_perm(e[2 * j], e[2 * j + 1], 0x5410);
}

// Tile row r's A word from the tile's 32-bit words: swap the two uint16 halves (memory is little endian, the stream
// is MSB first).
__device__ __forceinline__ u32 rowA(u32 word) { return __byte_perm(word, 0, 0x1032); }

// Words rg*RPT .. rg*RPT+RPT (mod 16) of a tile: row a of the lane's row group is (W[a], W[a + 1]).
template <int RPT>
__device__ __forceinline__ void load_tile_rows(const u16* __restrict__ bits, size_t tile, int rg, u32 (&W)[RPT + 1]) {
    const u32* tw = reinterpret_cast<const u32*>(bits + tile * 32);
    if (RPT == 16) {
        const uint4* tp = reinterpret_cast<const uint4*>(tw);
        const uint4 a0 = ldg_stream_v4(tp), a1 = ldg_stream_v4(tp + 1), a2 = ldg_stream_v4(tp + 2), a3 = ldg_stream_v4(tp + 3);
        const u32 all[16] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w, a2.x, a2.y, a2.z, a2.w, a3.x, a3.y, a3.z, a3.w};
#pragma unroll
        for (int a = 0; a <= RPT; ++a) W[a] = all[a & 15];
    } else {
#pragma unroll
        for (int a = 0; a <= RPT; ++a) W[a] = __ldg(tw + ((rg * RPT + a) & 15));
    }
}

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
};

constexpr int kMaxRows = 24;    // tile rows one CTA may touch (the launcher bounds the units per CTA accordingly)

// Sum RPT x MT accumulators over the lanes that hold the same row group (lanes differing in bits >= log2(LT)) by
// recursive halving: each exchange step sends half of the remaining values and keeps the other half, so 16 values
// need 8 + 4 + 2 + 1 shuffles instead of 16 per step. On return lane l holds KEEP values; value i is the flattened
// index out_index(l, i) = a * MT + m of its row group's accumulator array.
template <int MT>
struct LaneReduce {
    static constexpr int LT = MT;
    static constexpr int P = 32 / LT;                       // lanes sharing a row group
    static constexpr int LOGP = P == 32 ? 5 : P == 16 ? 4 : P == 8 ? 3 : P == 4 ? 2 : 1;
    static constexpr int STEPS = LOGP < 4 ? LOGP : 4;       // halving steps (16 values)
    static constexpr int KEEP = 16 >> STEPS;
    __device__ __forceinline__ static void run(int (&v)[16], int lane) {
#pragma unroll
        for (int j = 0; j < STEPS; ++j) {
            const int o = 16 >> j, half = 8 >> j;
            const bool up = (lane & o) != 0;
#pragma unroll
            for (int i = 0; i < half; ++i) {
                const int send = up ? v[i] : v[i + half];
                const int keep = up ? v[i + half] : v[i];
                v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
            }
        }
        if (LOGP == 5) v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
    }
    __device__ __forceinline__ static int out_index(int lane, int i) {
        int idx = i;
#pragma unroll
        for (int j = 0; j < STEPS; ++j)
            if (lane & (16 >> j)) idx += 8 >> j;
        return idx;
    }
    // lanes that write: all, except the duplicate odd lanes of the 32-lane case
    __device__ __forceinline__ static bool writer(int lane) { return LOGP != 5 || (lane & 1) == 0; }
};

__device__ __forceinline__ int atom_add_acq_rel_gpu(int* p, int v) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

template <int MT>
__global__ void __launch_bounds__(kThreads, 1)
k_gemm_tcq(const u16* __restrict__ bits, const i8* __restrict__ t8, const int* __restrict__ q4, const float* __restrict__ s,
           const float* __restrict__ rs, float* __restrict__ z, int M, int N, int K, Parts parts, int* __restrict__ ws_acc,
           int* __restrict__ ws_cnt, int act_vec) {
    constexpr int LT = MT;          // lanes per tile
    constexpr int RPT = 16 / MT;    // tile rows per lane
    constexpr int TPU = 32 / LT;    // tiles per unit
    constexpr int RV = 16 * MT;     // partial sums per tile row
    using Red = LaneReduce<MT>;
    extern __shared__ __align__(128) u32 tab[];
    __shared__ __align__(16) u16 pairs[512];
    __shared__ int racc[kMaxRows * RV];
    pdl_launch_dependents();
    // This CTA's layer (selected without dynamic indexing of the parameter arrays).
    int cb = parts.cta0[0], ce = parts.cta0[1], tb = parts.tr0[0], te = parts.tr0[1], slot = parts.slot[0];
    if (parts.n > 1 && (int)blockIdx.x >= parts.cta0[1]) {
        cb = parts.cta0[1]; ce = parts.cta0[2]; tb = parts.tr0[1]; te = parts.tr0[2]; slot = parts.slot[1];
    }
    if (parts.n > 2 && (int)blockIdx.x >= parts.cta0[2]) {
        cb = parts.cta0[2]; ce = parts.cta0[3]; tb = parts.tr0[2]; te = parts.tr0[3]; slot = parts.slot[2];
    }
    const int tiles = K >> 4, S = (tiles + TPU - 1) / TPU;
    const int U = (te - tb) * S;                   // < 2^31: checked by the launcher
    const int G = ce - cb, c = blockIdx.x - cb;
    const int ub = (int)((long long)U * c / G), ue = (int)((long long)U * (c + 1) / G);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const int tin = lane / LT, rg = lane % LT;
    const u32 lane4 = 4u * lane;
    const int row_first = ub / S;
    const int nrows = ub < ue ? (ue - 1) / S - row_first + 1 : 0;

    int u = ub + warp;
    u32 Wn[RPT + 1];
    if (u < ue) {
        const int tc = (u % S) * TPU + tin;
        if (tc < tiles) load_tile_rows<RPT>(bits, (size_t)(tb + u / S) * tiles + tc, rg, Wn);   // weights: before the wait
    }
    for (int i = threadIdx.x; i < nrows * RV; i += blockDim.x) racc[i] = 0;
    build_table_i8(tab, pairs, t8 + 1024 * slot);
    __syncthreads();
    pdl_wait();                                    // activations / scales come from the previous kernel
    for (; u < ue; u += nw) {
        const int rrel = u / S, tc = (u - rrel * S) * TPU + tin;
        u32 W[RPT + 1];
#pragma unroll
        for (int a = 0; a <= RPT; ++a) W[a] = Wn[a];
        const int un = u + nw;
        if (un < ue) {
            const int rn = un / S, tcn = (un - rn * S) * TPU + tin;
            if (tcn < tiles) load_tile_rows<RPT>(bits, (size_t)(tb + rn) * tiles + tcn, rg, Wn);
        }
        int acc[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[i] = 0;
        if (tc < tiles) {
            int act[4][MT];
            const int* qa = q4 + (size_t)4 * tc * M;
            if (MT == 1 && act_vec) {
                const int4 v = __ldg(reinterpret_cast<const int4*>(qa));
                act[0][0] = v.x; act[1][0] = v.y; act[2][0] = v.z; act[3][0] = v.w;
            } else {
#pragma unroll
                for (int e = 0; e < 4; ++e)
#pragma unroll
                    for (int m = 0; m < MT; ++m) act[e][m] = (m < M) ? __ldg(qa + e * M + m) : 0;
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
    }
    __syncthreads();
    for (int r = warp; r < nrows; r += nw) {
        const int rrel = row_first + r, trow = tb + rrel;
        const int a0 = rrel * S, a1 = a0 + S;
        const int* src = racc + r * RV;
        if (a0 >= ub && a1 <= ue) {                // the whole tile row was summed here
            for (int i = lane; i < RV; i += 32) {
                const int rr = i / MT, m = i % MT, row = trow * 16 + rr;
                if (m < M) z[(size_t)m * N + row] = ((float)src[i] * s[m]) * rs[row];
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
            for (int i = lane; i < RV; i += 32) {
                const int rr = i / MT, m = i % MT, row = trow * 16 + rr;
                if (m < M) {
                    const size_t o = (size_t)m * N + row;
                    const int v = atomicExch(ws_acc + o, 0);      // read and clear; lanes issue these in parallel
                    z[o] = ((float)v * s[m]) * rs[row];
                }
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

template <int MT>
int launch_gemm_tcq(const uint16_t* bits, const int8_t* t8, const int32_t* q4, const float* s, const float* rs, float* z,
                    int M, int N, int K, int nb0, int nb1, int* ws, cudaStream_t st) {
    auto kern = k_gemm_tcq<MT>;
    if (set_smem(kern, kTabBytes)) return TCQ_ERR_LAUNCH;
    const int TPU = 32 / MT, tiles = K >> 4, S = (tiles + TPU - 1) / TPU, R = N >> 4;
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
        const long long gmin = (Ul + (long long)(kMaxRows - 2) * S - 1) / ((long long)(kMaxRows - 2) * S);   // rows per CTA <= kMaxRows
        if (g < gmin) g = gmin;
        if (g < 1) g = 1;
        if (g > Ul) g = Ul;
        p.cta0[nl] = cta;
        p.tr0[nl] = bounds[l];
        p.slot[nl] = l;
        cta += (int)g;
        ++nl;
    }
    p.n = nl;
    p.cta0[nl] = cta;
    p.tr0[nl] = R;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cta);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kTabBytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int* ws_acc = ws;
    int* ws_cnt = ws + (size_t)M * N;
    const int act_vec = tcq_aligned(q4, 16) ? 1 : 0;
    if (cudaLaunchKernelEx(&cfg, kern, reinterpret_cast<const u16*>(bits), reinterpret_cast<const i8*>(t8), q4, s, rs, z,
                           M, N, K, p, ws_acc, ws_cnt, act_vec) != cudaSuccess)
        return TCQ_ERR_LAUNCH;
    return TCQ_OK;
}

template <int MT, int RPW>
int launch_gemm_w8(const int8_t* W, const int32_t* q4, const float* s, const float* rs, float* z, int M, int N, int K,
                   cudaStream_t st) {
    auto kern = k_gemm_w8<MT, RPW>;
    const int smem = K * M;
    if (smem > 48 * 1024 && set_smem(kern, smem)) return TCQ_ERR_LAUNCH;
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

int scratch_for_current_device(int** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return TCQ_ERR_DEVICE;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_addr[dev]) {
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
    if (M == 1) return launch_gemm_tcq<1>(bits, t8, q4, s, rs, z, M, N, K, nb0, nb1, ws, st);
    if (M == 2) return launch_gemm_tcq<2>(bits, t8, q4, s, rs, z, M, N, K, nb0, nb1, ws, st);
    if (M <= 4) return launch_gemm_tcq<4>(bits, t8, q4, s, rs, z, M, N, K, nb0, nb1, ws, st);
    if (M <= 8) return launch_gemm_tcq<8>(bits, t8, q4, s, rs, z, M, N, K, nb0, nb1, ws, st);
    return launch_gemm_tcq<16>(bits, t8, q4, s, rs, z, M, N, K, nb0, nb1, ws, st);
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
// The stream-K scratch is the fixed array g_gemv_scratch; its device address is resolved on the first call on each
// device (so that first call should come before any stream capture). Limits: 1 <= M <= 16, N <= 32768,
// M * N <= 524288; larger shapes return TCQ_ERR_SHAPE. All calls share the one array per device: the used part is
// cleared (cudaMemsetAsync, no allocation) on the caller's stream before the kernel, and calls that overlap on the GPU
// (other streams, other host threads) race on it. Allocates nothing: no cudaMalloc / cudaFree / library allocation.
int tcq_gemm_tcq_noalloc(const uint16_t* bits, const int8_t* t8, const int32_t* q4, const float* s, const float* rs, float* z,
                         int M, int N, int K, int nb0, int nb1, void* stream) {
    if (!bits || !t8 || !q4 || !s || !rs || !z) return TCQ_ERR_ARG;
    if (M < 1 || M > 16 || N <= 0 || K <= 0 || (N & 15) || (K & 15)) return TCQ_ERR_SHAPE;
    if (N > kNoAllocMaxN || (long long)M * N > kNoAllocMaxMN) return TCQ_ERR_SHAPE;
    if (!tcq_aligned(bits, 16) || !tcq_aligned(q4, 4) || !tcq_aligned(t8, 16)) return TCQ_ERR_ALIGN;
    if (nb0 < 0 || nb1 < 0) return TCQ_ERR_ARG;
    int* ws = nullptr;
    const int e = scratch_for_current_device(&ws);
    if (e) return e;
    cudaStream_t st = (cudaStream_t)stream;
    if (cudaMemsetAsync(ws, 0, tcq_gemm_tcq_workspace(M, N), st) != cudaSuccess) return TCQ_ERR_LAUNCH;
    if (M == 1) return launch_gemm_tcq<1>(bits, t8, q4, s, rs, z, M, N, K, nb0, nb1, ws, st);
    if (M == 2) return launch_gemm_tcq<2>(bits, t8, q4, s, rs, z, M, N, K, nb0, nb1, ws, st);
    if (M <= 4) return launch_gemm_tcq<4>(bits, t8, q4, s, rs, z, M, N, K, nb0, nb1, ws, st);
    if (M <= 8) return launch_gemm_tcq<8>(bits, t8, q4, s, rs, z, M, N, K, nb0, nb1, ws, st);
    return launch_gemm_tcq<16>(bits, t8, q4, s, rs, z, M, N, K, nb0, nb1, ws, st);
}

}  // extern "C"

