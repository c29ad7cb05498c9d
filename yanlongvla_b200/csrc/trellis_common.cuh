// Trellis decode helpers shared by the SIMT kernels (trellis.cu) and the tensor-core decode-GEMM (gemm_i8.cu).
//
// Format (tcq_format.py:3-12, 58-71): a tile is 32 uint16 words = 512 bits, MSB first; the state of weight pair p
// (0..7) of tile row r (0..15) is bits [32 r + 4 p, 32 r + 4 p + 16) of the tile's stream (tail-biting). A state s
// decodes to the pair t8[h], h = ((s + 1) s >> 6) & 511, first coordinate negated when bit 15 of (s + 1) s is set.
#pragma once
#include "tcq_common.cuh"

namespace tcq {

constexpr int kTabBytes = 1024 * 32 * 4;   // per-lane replicated decode table

// Table entry for key k (bits 6..15 of x): pair index k & 511, sign k >> 9.
// INT8 entry: byte 0 = (sign ? -v0 : v0), byte 1 = v1. The 1 KB source table is staged through shared memory with one
// 16-byte load per thread (one memory round trip), then the 128 KB replicated table is written with consecutive
// 16-byte stores (lanes of a warp cover 512 contiguous bytes: no bank conflicts).
__device__ __forceinline__ void stage_pairs(u16* pairs, const void* __restrict__ src) {
    if (threadIdx.x < 64) reinterpret_cast<uint4*>(pairs)[threadIdx.x] = ldg_table_v4(reinterpret_cast<const uint4*>(src) + threadIdx.x);
    __syncthreads();
}

__device__ __forceinline__ void fill_table_i8(u32* tab, const u16* pairs) {
    // Thread t writes 16-byte slot (t & 7) of keys k and k + 512 (the same pair, first coordinate negated) for
    // k = t >> 3, + blockDim / 8, ...: one shared load per two stores.
    uint4* t4 = reinterpret_cast<uint4*>(tab);
    const int slot = threadIdx.x & 7, kstep = blockDim.x >> 3;
    for (int k = threadIdx.x >> 3; k < 512; k += kstep) {
        const u32 pr = pairs[k];
        const u32 ep = pr & 0xffffu, en = ((0u - pr) & 0xffu) | (pr & 0xff00u);
        t4[k * 8 + slot] = make_uint4(ep, ep, ep, ep);
        t4[(k + 512) * 8 + slot] = make_uint4(en, en, en, en);
    }
}

// The same fill for a block of exactly NT threads: all shared loads first, then the stores (no load -> store chain
// per iteration).
template <int NT>
__device__ __forceinline__ void fill_table_i8_nt(u32* tab, const u16* pairs) {
    constexpr int IT = 512 / (NT / 8);
    uint4* t4 = reinterpret_cast<uint4*>(tab);
    const int slot = threadIdx.x & 7, k0 = threadIdx.x >> 3;
    u32 pr[IT];
#pragma unroll
    for (int j = 0; j < IT; ++j) pr[j] = pairs[k0 + j * (NT / 8)];
#pragma unroll
    for (int j = 0; j < IT; ++j) {
        const int k = k0 + j * (NT / 8);
        const u32 ep = pr[j] & 0xffffu, en = ((0u - pr[j]) & 0xffu) | (pr[j] & 0xff00u);
        t4[k * 8 + slot] = make_uint4(ep, ep, ep, ep);
        t4[(k + 512) * 8 + slot] = make_uint4(en, en, en, en);
    }
}

// The same fill by nt threads (a multiple of 8) of index i = 0 .. nt - 1 of the block.
__device__ __forceinline__ void fill_table_i8_span(u32* tab, const u16* pairs, int i, int nt) {
    uint4* t4 = reinterpret_cast<uint4*>(tab);
    const int slot = i & 7;
#pragma unroll 4
    for (int k = i >> 3; k < 512; k += nt >> 3) {
        const u32 p = pairs[k];
        const u32 ep = p & 0xffffu, en = ((0u - p) & 0xffu) | (p & 0xff00u);
        t4[k * 8 + slot] = make_uint4(ep, ep, ep, ep);
        t4[(k + 512) * 8 + slot] = make_uint4(en, en, en, en);
    }
}

__device__ __forceinline__ void build_table_i8(u32* tab, u16* pairs, const i8* __restrict__ t8) {
    stage_pairs(pairs, t8);
    fill_table_i8(tab, pairs);
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

// Table lookup of this lane's copy: byte offset (key * 128) | (4 * lane) from the shared table `tab`: the key offset
// is bits 7..16 of t (below), the lane offset bits 2..6, so one three-input logic op (t & 0x1FF80) | lane4 forms the
// address (written as one lop3 so that the mask and the lane always fuse); the constant shared base is added by the
// compiler.
__device__ __forceinline__ u32 lut(const u32* tab, u32 lane4, u32 t) {
    u32 off;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(off) : "r"(t), "n"(0x1FF80), "r"(lane4));   // (a & b) | c
    return *reinterpret_cast<const u32*>(reinterpret_cast<const char*>(tab) + off);
}

// 2x for the state in the upper half of F: v = F >> 16 taken as the high word of F * 2^16 (multiply pipe),
// 2x = v * 2v + 2v; bits 7..16 of 2x = bits 6..15 of x = key.
__device__ __forceinline__ u32 off_hi(u32 F) {
    const u32 v = __umulhi(F, 65536u), u = v * 2u;
    return v * u + u;
}
// 2x for the state in the lower half of F (bits above 16 are junk and drop out of bits 7..16 of 2x).
__device__ __forceinline__ u32 off_lo(u32 F) {
    const u32 u = F * 2u;
    return F * u + u;
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

// The same table with 16-bit entries (byte 0 = the sign-applied first value, byte 1 = the second), 64 KB: key k of
// lane l at byte (k >> 1) * 128 + 4 l + 2 (k & 1), so lane l still always reads bank l (a warp's random lookups never
// conflict) at one more instruction per pair than the 32-bit form. For kernels that need the other 64 KB of shared
// memory more than that instruction (the tensor-core decode-GEMM's operand ring).
constexpr int kTab16Bytes = 1024 * 32 * 2;

// Word (row j, any lane) = entry(2j) | entry(2j + 1) << 16; rows 256.. hold the sign keys (first bytes negated).
__device__ __forceinline__ void build_table16(char* tab, u16* pairs, const i8* __restrict__ t8) {
    stage_pairs(pairs, t8);
    const u32* p32 = reinterpret_cast<const u32*>(pairs);
    uint4* t4 = reinterpret_cast<uint4*>(tab);
    for (int i = threadIdx.x; i < 512 * 8; i += blockDim.x) {
        const int j = i >> 3;
        u32 v = p32[j & 255];
        if (j >= 256) {
            const u32 n0 = (0u - v) & 0xffu, n2 = (0u - (v >> 16)) & 0xffu;
            v = (v & 0xff00ff00u) | n0 | (n2 << 16);
        }
        t4[i] = make_uint4(v, v, v, v);
    }
}

// Lookup of x = (s + 1) s in the 16-bit table: (x & 0xFF80) | 4 l | ((x >> 5) & 2).
__device__ __forceinline__ u32 lut16(const char* tab, u32 lane4, u32 x) {
    return *reinterpret_cast<const u16*>(tab + ((x & 0xFF80u) | lane4 | ((x >> 5) & 2u)));
}

// INT8 weights of one tile row as 4 words from the 16-bit table (A, B as in row_entries: the upper half of F_p is
// state p, its lower half state p + 4; junk above bit 16 of a state never reaches bits 6..15 of (s + 1) s).
__device__ __forceinline__ void row_words16(u32 A, u32 B, const char* tab, u32 lane4, u32 (&w)[4]) {
    const u32 Fs[4] = {A, __funnelshift_l(B, A, 4), __funnelshift_l(B, A, 8), __funnelshift_l(B, A, 12)};
    u32 e[8];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const u32 v = __umulhi(Fs[p], 65536u);
        e[p] = lut16(tab, lane4, v * v + v);
        e[p + 4] = lut16(tab, lane4, Fs[p] * Fs[p] + Fs[p]);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) w[j] = __byte_perm(e[2 * j], e[2 * j + 1], 0x5410);
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


}  // namespace tcq
