// mbarrier and TMA helpers shared by the tensor-core GEMMs (gemm_i8.cu) and the decode-GEMV (trellis.cu).
//
// Only loads without cluster multicast are issued. Every wait is bounded by the global timer: a wait that expires
// raises the caller's device error flag and the CTA's abort flag instead of spinning forever.
#pragma once
#include <cuda.h>

#include "tcq_common.cuh"

namespace tcq {

constexpr unsigned long long kWaitNs = 2000000000ull;    // 2 s

__device__ __forceinline__ u32 smem_u32(const void* p) { return (u32)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(u32 bar, u32 count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
// Make initialized barriers visible to the async proxy (TMA) and to the other threads after a CTA barrier.
__device__ __forceinline__ void mbar_init_fence() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(u32 bar, u32 bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(u32 bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try(u32 bar, u32 parity) {
    u32 ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ unsigned long long gtime() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait for the phase of parity `parity` to complete. Returns false when the CTA was aborted or the wait
// expired (then *err gets bit 1 and the CTA abort flag is raised).
__device__ __forceinline__ bool mbar_wait_bounded(u32 bar, u32 parity, volatile int* abort_flag, int* err,
                                                  unsigned long long limit = kWaitNs) {
    if (mbar_try(bar, parity)) return true;
    const unsigned long long t0 = gtime();
    for (u32 i = 1;; ++i) {
        if (mbar_try(bar, parity)) return true;
        if ((i & 127) == 0) {
            if (*abort_flag) return false;
            if (gtime() - t0 > limit) {
                atomicOr(err, 1);
                *abort_flag = 1;
                return false;
            }
        }
    }
}

__device__ __forceinline__ void tma_load_2d(u32 dst, const CUtensorMap* map, u32 bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(map), "r"(bar), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(u32 dst, const CUtensorMap* map, u32 bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
        "l"(map), "r"(bar), "r"(x), "r"(y), "r"(z)
        : "memory");
}

// Tiled TMA store of a shared-memory box to global memory (bulk-group completion). x is the innermost coordinate; the
// caller keeps x * element size a multiple of 16 bytes and never starts a store at a negative coordinate.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, u32 src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(map), "r"(src), "r"(x), "r"(y)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until the thread's committed bulk stores have finished reading their shared-memory sources.
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Wait until the thread's committed bulk stores are complete.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// cuTensorMapEncodeTiled is a driver entry point; it is resolved through the runtime at first use so that the library
// does not link libcuda (it loads on machines without a driver, where only the host-side validation is exercised).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                                  const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static inline EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

}  // namespace tcq
