// C-ABI plumbing: error reporting, cross-process receive buffers (CUDA IPC),
// and the host-mapped device status word.
//
// The receive buffers replace ThunderKittens' TKParallelTensor allocation used
// by the reference (flash_ulysses/context.py:63-90): each rank allocates its
// own buffer with cudaMalloc, exports a CUDA IPC handle, and maps every peer's
// handle.  The caller moves the 64-byte handles between processes, which
// removes the reference's fixed-name IPC broker.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "flash_ulysses_b200.h"
#include "fu_internal.h"

namespace fu {
static thread_local std::string g_last_error;

int set_error(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

EncodeTiledFn encode_tiled_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        void* ptr = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    });
    return fn;
}

namespace {
struct DeviceGuard {
    int prev = -1;
    bool changed = false;
    explicit DeviceGuard(int device) {
        if (cudaGetDevice(&prev) == cudaSuccess && prev != device) {
            changed = cudaSetDevice(device) == cudaSuccess;
        }
    }
    ~DeviceGuard() {
        if (changed) cudaSetDevice(prev);
    }
};

int cuda_fail(const char* what, cudaError_t e) {
    return set_error(FU_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}
}  // namespace
}  // namespace fu

using namespace fu;

extern "C" const char* fu_last_error(void) { return g_last_error.c_str(); }

extern "C" int fu_version(void) { return 1; }

extern "C" int fu_buffer_alloc(int device, size_t bytes, void** ptr) {
    if (ptr == nullptr || bytes == 0) return set_error(FU_ERR_INVALID, "bad buffer request");
    DeviceGuard g(device);
    cudaError_t e = cudaMalloc(ptr, bytes);
    if (e != cudaSuccess) return cuda_fail("cudaMalloc", e);
    return FU_OK;
}

extern "C" int fu_buffer_free(int device, void* ptr) {
    DeviceGuard g(device);
    cudaError_t e = cudaFree(ptr);
    if (e != cudaSuccess) return cuda_fail("cudaFree", e);
    return FU_OK;
}

extern "C" int fu_buffer_export(int device, void* ptr, unsigned char handle[FU_IPC_HANDLE_BYTES]) {
    static_assert(sizeof(cudaIpcMemHandle_t) == FU_IPC_HANDLE_BYTES, "IPC handle size");
    DeviceGuard g(device);
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, ptr);
    if (e != cudaSuccess) return cuda_fail("cudaIpcGetMemHandle", e);
    std::memcpy(handle, &h, sizeof(h));
    return FU_OK;
}

extern "C" int fu_buffer_import(int device, const unsigned char handle[FU_IPC_HANDLE_BYTES],
                                void** peer_ptr) {
    DeviceGuard g(device);
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    cudaError_t e = cudaIpcOpenMemHandle(peer_ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail("cudaIpcOpenMemHandle", e);
    return FU_OK;
}

extern "C" int fu_buffer_close(int device, void* peer_ptr) {
    DeviceGuard g(device);
    cudaError_t e = cudaIpcCloseMemHandle(peer_ptr);
    if (e != cudaSuccess) return cuda_fail("cudaIpcCloseMemHandle", e);
    return FU_OK;
}

extern "C" int fu_status_alloc(int32_t** host_ptr, int32_t** device_ptr) {
    if (host_ptr == nullptr || device_ptr == nullptr) return set_error(FU_ERR_INVALID, "null");
    void* h = nullptr;
    cudaError_t e = cudaHostAlloc(&h, 64, cudaHostAllocMapped | cudaHostAllocPortable);
    if (e != cudaSuccess) return cuda_fail("cudaHostAlloc", e);
    std::memset(h, 0, 64);
    void* d = nullptr;
    e = cudaHostGetDevicePointer(&d, h, 0);
    if (e != cudaSuccess) {
        cudaFreeHost(h);
        return cuda_fail("cudaHostGetDevicePointer", e);
    }
    *host_ptr = static_cast<int32_t*>(h);
    *device_ptr = static_cast<int32_t*>(d);
    return FU_OK;
}

extern "C" int fu_status_free(int32_t* host_ptr) {
    cudaError_t e = cudaFreeHost(host_ptr);
    if (e != cudaSuccess) return cuda_fail("cudaFreeHost", e);
    return FU_OK;
}
