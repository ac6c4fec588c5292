// qsa_tma.cuh -- tensor-memory-accelerator (TMA) loads into this CTA's shared memory, non-blocking
// mbarrier probes, and the host-side tensor-map encoder (cuTensorMapEncodeTiled through the
// runtime's driver entry-point query, so the library does not link the driver library).
#pragma once
#include <cuda.h>          // CUtensorMap and its enums

#include "qsa_common.cuh"

namespace qsa {

// Tiled tensor loads global -> this CTA's shared memory (no multicast), completing on `bar`.  The
// innermost coordinate times the element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap * map, int x, int y, uint64_t * bar) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                 :: "r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap * map, int x, int y, int z, uint64_t * bar) {
    asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
                 :: "r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap * map, int w, uint64_t * bar) {
    asm volatile("cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %2, %2, %3}], [%4];"
                 :: "r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(w), "r"(smem_u32(bar)) : "memory");
}
// non-blocking probe of a phase (an MMA thread polls two streams of work with it)
__device__ __forceinline__ bool mbar_test(uint64_t * bar, uint32_t parity) {
    uint32_t done;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(done) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return done != 0;
}
// Bounded wait by polling (no suspension): a thread suspended on a phase that other threads'
// arrivals complete was seen to resume microseconds late, so loaders poll.
__device__ __forceinline__ bool mbar_poll_bounded(uint64_t * bar, uint32_t parity, uint32_t * status) {
    if (mbar_test(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (int k = 1;; k++) {
        if (mbar_test(bar, parity)) return true;
        if ((k & 63) == 0 && global_timer_ns() - t0 > 2000000000ull) break;
    }
    set_status(status, DEV_TIMEOUT);
    return false;
}

// cuTensorMapEncodeTiled, reached through the runtime's driver entry-point query
typedef CUresult (*encode_tiled_fn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                    const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
inline encode_tiled_fn tensor_map_encoder() {
    static encode_tiled_fn fn = nullptr;
    if (!fn) {
        void * f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<encode_tiled_fn>(f);
    }
    return fn;
}

}  // namespace qsa
