// tk_host.cuh — host-side helpers shared by the C-ABI entry points: device
// capability checks, cached device properties, and the driver entry point for
// tensor-map encoding (fetched at run time so the library has no link-time
// dependency on libcuda).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <mutex>

namespace tk {
namespace host {

constexpr int kMaxDevices = 64;

struct DeviceInfo {
    std::atomic<int> state{0};  // 0 unknown, 1 ok (cc 10.0), 2 unsupported
    int sm_count = 0;
};

inline DeviceInfo& device_info(int device) {
    static DeviceInfo infos[kMaxDevices];
    return infos[device];
}

// Returns cudaSuccess when the current device is a compute capability 10.0 part.
// Touches no pending error on success.
inline cudaError_t current_device(int* device_out, int* sm_count_out) {
    int device = 0;
    cudaError_t err = cudaGetDevice(&device);
    if (err != cudaSuccess) return err;
    if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
    DeviceInfo& info = device_info(device);
    int state = info.state.load(std::memory_order_acquire);
    if (state == 0) {
        int major = 0, minor = 0, sms = 0;
        err = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
        if (err != cudaSuccess) return err;
        err = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
        if (err != cudaSuccess) return err;
        err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
        if (err != cudaSuccess) return err;
        info.sm_count = sms;
        state = (major == 10 && minor == 0) ? 1 : 2;
        info.state.store(state, std::memory_order_release);
    }
    if (state != 1) return cudaErrorInvalidDeviceFunction;
    if (device_out) *device_out = device;
    if (sm_count_out) *sm_count_out = info.sm_count;
    return cudaSuccess;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
        } else {
            static_cast<void>(cudaGetLastError());
        }
    });
    return fn;
}

// Row-major 2D (or 3D with a batch dimension) binary16 tensor map with a
// 128-byte swizzle. dims/strides innermost first; strides in bytes for dims >= 1.
inline bool make_map_f16(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                         const uint64_t* strides_bytes, const uint32_t* box) {
    EncodeTiledFn fn = encode_tiled();
    if (fn == nullptr) return false;
    cuuint64_t d[5];
    cuuint64_t s[4];
    cuuint32_t b[5];
    cuuint32_t e[5];
    for (int i = 0; i < rank; ++i) {
        d[i] = dims[i];
        b[i] = box[i];
        e[i] = 1;
        if (i + 1 < rank) s[i] = strides_bytes[i];
    }
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, static_cast<cuuint32_t>(rank),
                    const_cast<void*>(base), d, s, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Stream-ordered scratch from a private per-device memory pool that keeps its
// memory (release threshold = max), so repeated calls reuse the same pages instead
// of mapping and unmapping them around every call. The pool is the library's own;
// the process's default pool is left untouched. It is created by the first call
// on a device that needs scratch.
struct ScratchPools {
    std::mutex mu;
    cudaMemPool_t pools[kMaxDevices] = {};
};

inline ScratchPools& scratch_pools() {
    static ScratchPools p;
    return p;
}

inline cudaError_t scratch_alloc(void** ptr, size_t bytes, int device, cudaStream_t stream) {
    ScratchPools& sp = scratch_pools();
    cudaMemPool_t pool;
    {
        std::lock_guard<std::mutex> lock(sp.mu);
        if (sp.pools[device] == nullptr) {
            cudaMemPoolProps props{};
            props.allocType = cudaMemAllocationTypePinned;
            props.location.type = cudaMemLocationTypeDevice;
            props.location.id = device;
            cudaMemPool_t created = nullptr;
            cudaError_t err = cudaMemPoolCreate(&created, &props);
            if (err != cudaSuccess) return err;
            uint64_t keep = UINT64_MAX;
            err = cudaMemPoolSetAttribute(created, cudaMemPoolAttrReleaseThreshold, &keep);
            if (err != cudaSuccess) {
                static_cast<void>(cudaMemPoolDestroy(created));
                return err;
            }
            sp.pools[device] = created;
        }
        pool = sp.pools[device];
    }
    return cudaMallocFromPoolAsync(ptr, bytes, pool, stream);
}

// Bytes the scratch pool of `device` has reserved from the driver and has handed
// out to allocations not yet freed (both 0 while no call has created the pool).
inline cudaError_t scratch_pool_bytes(int device, uint64_t* reserved, uint64_t* used) {
    ScratchPools& sp = scratch_pools();
    std::lock_guard<std::mutex> lock(sp.mu);
    *reserved = 0;
    *used = 0;
    if (sp.pools[device] == nullptr) return cudaSuccess;
    cudaError_t err = cudaMemPoolGetAttribute(sp.pools[device], cudaMemPoolAttrReservedMemCurrent, reserved);
    if (err != cudaSuccess) return err;
    return cudaMemPoolGetAttribute(sp.pools[device], cudaMemPoolAttrUsedMemCurrent, used);
}

inline bool ranges_overlap(const void* a, size_t a_bytes, const void* b, size_t b_bytes) {
    const uintptr_t a0 = reinterpret_cast<uintptr_t>(a), b0 = reinterpret_cast<uintptr_t>(b);
    return a0 < b0 + b_bytes && b0 < a0 + a_bytes;
}

}  // namespace host
}  // namespace tk
