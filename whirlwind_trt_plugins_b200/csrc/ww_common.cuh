// ww_common.cuh -- status handling, launch-error reporting and the per-device
// property cache shared by every entry point of libww_trt_plugins.so.
#pragma once

#include "../../include/ww_trt_plugins.h"

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>

namespace ww {

// Mirrors the reference's lastLaunchError (src/common/cuda_check.hpp:15-23):
// report the pending launch error on stderr with the same prefix and turn it
// into a status.  `where` is the launching function.
inline int launch_status(const char* where) noexcept
{
    const cudaError_t err = cudaPeekAtLastError();
    if (err != cudaSuccess) {
        std::fprintf(stderr, "[ww_trt_plugins] %s: CUDA launch failed: %s\n", where,
                     cudaGetErrorString(err));
        return WW_ERR_LAUNCH;
    }
    return WW_SUCCESS;
}

// Streaming-multiprocessor count and opt-in shared memory of the current
// device, cached per device ordinal.  (The reference caches per host thread,
// corr_volume_kernel.cu:26-40, which returns the wrong count when one thread
// drives several devices.)
struct DeviceInfo {
    int sm_count = 0;
    int smem_optin = 0;
    int cc_major = 0;
    int cc_minor = 0;
};

int current_device_info(DeviceInfo* out) noexcept;

// Device-side error word set by bounded waits (see umma.cuh).  Codes:
constexpr int kErrMbarTimeout = 0x100;  // | site

__device__ __forceinline__ void record_device_error(int* slot, int code)
{
    atomicCAS(slot, 0, code);
}

int* device_error_slot() noexcept;  // device address of the error word (current device)

__host__ __device__ __forceinline__ int64_t i64(int v) { return static_cast<int64_t>(v); }

}  // namespace ww
