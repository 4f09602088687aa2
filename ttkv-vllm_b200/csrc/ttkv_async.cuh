// Asynchronous-copy plumbing shared by the sm_100a kernels: mbarriers with bounded waits, 16-byte
// cp.async, 2-D tiled TMA loads (never with cluster multicast), and the host encoder of a TMA map.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

namespace ttkv {

constexpr long long kWaitCycles = 4000000000LL;   // ~2 s at 2 GHz: the bound of every mbarrier wait

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Order this thread's generic-proxy shared-memory writes before later async-proxy reads (TMA,
// tcgen05) of the same bytes.
__device__ __forceinline__ void fence_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(bar)), "r"(count));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}

// Bounded wait for an mbarrier phase: false after ~2 s. The clock is read only when the first
// test finds the phase still open.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try(bar, parity))
        if (clock64() - t0 > kWaitCycles) return false;
    return true;
}

// The one arrival of a TMA phase, announcing the bytes its copies will deliver.
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(smem_u32(smem)), "l"(gmem) : "memory");
}

// Arrive on `bar` once every earlier cp.async of this thread has landed (no pending-count
// increment: the barrier is initialised with one arrival per thread).
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" :: "r"(smem_u32(bar)) : "memory");
}

// Fetch a TMA map's descriptor ahead of its first use.
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled TMA load of the box at element (x, y) of `map` into this CTA's shared memory, its bytes
// counted on `bar`. No multicast. x times the element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        :: "r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// Untiled bulk copy of `bytes` (a multiple of 16, both addresses 16-byte aligned) from global
// memory into this CTA's shared memory, its bytes counted on `bar`. No multicast.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

// Programmatic dependent launch. A kernel launched with programmatic stream serialization may
// start while the kernel before it runs: pdl_wait() blocks until that kernel has completed and
// its memory is visible (it returns at once when there is no such dependency); pdl_trigger()
// lets the next kernel of the stream launch before this one ends.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// A 2-D TMA map: `rows` rows of `d0` elements of `dt`, `stride` bytes apart; boxes of b0 x b1
// elements, swizzled by `box_bytes` (the box's inner width when it is 32, 64 or 128 bytes; any
// other value: no swizzle). False if the driver's encoder is unavailable or refuses the tensor.
inline bool encode_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* ptr, uint64_t d0, uint64_t rows,
                      uint64_t stride, uint32_t b0, uint32_t b1, int box_bytes) {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
        cudaGetLastError();
    });
    if (!encode || rows < 1) return false;
    const CUtensorMapSwizzle sw = box_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                : box_bytes == 64  ? CU_TENSOR_MAP_SWIZZLE_64B
                                : box_bytes == 32  ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_NONE;
    const cuuint64_t dims[2] = {d0, rows};
    const cuuint64_t strides[1] = {stride};
    const cuuint32_t box[2] = {b0, b1};
    const cuuint32_t estr[2] = {1, 1};
    return encode(m, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  sw, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace ttkv
