// C-ABI plumbing: the thread-local error message, the layout constructor, the version.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <utility>
#include <vector>

#include "ttkv_common.cuh"

namespace ttkv {

static thread_local char g_err[1024] = "";

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return code;
}

int check_launch(const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(TTKV_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return TTKV_OK;
}

int raise_smem_limit(const void* kernel, const char* what) {
    static std::mutex mu;
    static std::vector<std::pair<int, const void*>> done;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) { cudaGetLastError(); return fail(TTKV_ERR_CUDA, "cudaGetDevice"); }
    std::lock_guard<std::mutex> lock(mu);
    for (const auto& d : done)
        if (d.first == dev && d.second == kernel) return TTKV_OK;
    int optin = 0;
    cudaFuncAttributes fa{};
    if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
        cudaFuncGetAttributes(&fa, kernel) != cudaSuccess ||
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             optin - int(fa.sharedSizeBytes)) != cudaSuccess) {
        const cudaError_t e = cudaGetLastError();
        return fail(TTKV_ERR_CUDA, "%s: raising the shared-memory limit: %s", what, cudaGetErrorString(e));
    }
    done.emplace_back(dev, kernel);
    return TTKV_OK;
}

}  // namespace ttkv

using namespace ttkv;

static int32_t align_up(int32_t n, int32_t a) { return a <= 1 ? n : ((n + a - 1) / a) * a; }

extern "C" const char* ttkv_last_error(void) { return g_err; }

extern "C" int32_t ttkv_abi_version(void) { return TTKV_ABI_VERSION; }

extern "C" int ttkv_layout_init(ttkv_layout_t* lay, int32_t H, int32_t d, int32_t r1,
                                int32_t qbits, int32_t res_k, int32_t res_bits, int32_t v_lanes,
                                int32_t v_bits, int32_t align) {
    g_err[0] = 0;
    if (!lay) return fail(TTKV_ERR_ARG, "layout pointer is null");
    if (H < 1 || d < 8 || r1 < 1 || qbits < 1 || res_k < 0 || v_lanes < 1 || align < 1)
        return fail(TTKV_ERR_LAYOUT, "layout H=%d d=%d r1=%d qbits=%d res_k=%d v_lanes=%d align=%d "
                    "has a non-positive field", H, d, r1, qbits, res_k, v_lanes, align);
    if (d % 8)
        return fail(TTKV_ERR_LAYOUT, "head dim %d is not a multiple of 8; the lane bitmap is d/8 "
                    "bytes per row", d);
    if (res_k > d) return fail(TTKV_ERR_LAYOUT, "res_k=%d exceeds d=%d", res_k, d);
    if (v_lanes > d) return fail(TTKV_ERR_LAYOUT, "v_lanes=%d exceeds d=%d", v_lanes, d);
    if ((r1 * qbits) % 8)
        return fail(TTKV_ERR_LAYOUT, "r1=%d at qbits=%d is not a whole number of bytes", r1, qbits);
    if (res_bits < 1 || res_bits > 8 || v_bits < 1 || v_bits > 8)
        return fail(TTKV_ERR_LAYOUT, "code widths res_bits=%d v_bits=%d outside 1..8", res_bits, v_bits);
    lay->H = H; lay->d = d; lay->r1 = r1; lay->qbits = qbits; lay->res_k = res_k;
    lay->res_bits = res_bits; lay->v_lanes = v_lanes; lay->v_bits = v_bits; lay->align = align;
    lay->coeff_bytes = r1 * qbits / 8;
    lay->k_row_bytes = d / 8 + packed_row_bytes(res_k, res_bits) + 2;
    lay->v_row_bytes = d / 8 + packed_row_bytes(v_lanes, v_bits) + 2;
    lay->k_slot_bytes = align_up(lay->coeff_bytes + 2 + H * lay->k_row_bytes, align);
    lay->v_slot_bytes = align_up(H * lay->v_row_bytes, align);
    lay->v_offset = lay->k_slot_bytes;
    lay->blob_bytes = lay->k_slot_bytes + lay->v_slot_bytes;
    return TTKV_OK;
}

// ---------------------------------------------------------------- memory shared through CUDA IPC
extern "C" size_t ttkv_ipc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int ttkv_ipc_alloc(size_t bytes, void** ptr, void* handle) {
    if (!ptr || !handle || bytes == 0) return fail(TTKV_ERR_ARG, "ipc alloc: null pointer or zero bytes");
    *ptr = nullptr;
    cudaError_t e = cudaMalloc(ptr, bytes);
    if (e == cudaSuccess) e = cudaMemset(*ptr, 0, bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), *ptr);
    if (e != cudaSuccess) {
        cudaGetLastError();
        if (*ptr) cudaFree(*ptr);
        *ptr = nullptr;
        return fail(TTKV_ERR_CUDA, "ipc alloc of %zu bytes: %s", bytes, cudaGetErrorString(e));
    }
    return TTKV_OK;
}

extern "C" int ttkv_ipc_open(const void* handle, void** ptr) {
    if (!ptr || !handle) return fail(TTKV_ERR_ARG, "ipc open: null pointer");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
        cudaGetLastError();
        *ptr = nullptr;
        return fail(TTKV_ERR_CUDA, "ipc open: %s", cudaGetErrorString(e));
    }
    return TTKV_OK;
}

extern "C" int ttkv_ipc_close(void* ptr) {
    if (!ptr) return TTKV_OK;
    const cudaError_t e = cudaIpcCloseMemHandle(ptr);
    if (e != cudaSuccess) { cudaGetLastError(); return fail(TTKV_ERR_CUDA, "ipc close: %s", cudaGetErrorString(e)); }
    return TTKV_OK;
}

extern "C" int ttkv_ipc_free(void* ptr) {
    if (!ptr) return TTKV_OK;
    const cudaError_t e = cudaFree(ptr);
    if (e != cudaSuccess) { cudaGetLastError(); return fail(TTKV_ERR_CUDA, "ipc free: %s", cudaGetErrorString(e)); }
    return TTKV_OK;
}
