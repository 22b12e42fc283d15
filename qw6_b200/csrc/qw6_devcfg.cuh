// qw6_devcfg.cuh -- one-time, per-device launch configuration (host side).
//
// cudaFuncSetAttribute applies to the CURRENT device only, and a process may
// drive several GPUs (one qw6cu_ctx per device, or the allocation-free entry
// point on whichever device is current).  So the "already configured" state
// of a kernel is kept per device: one atomic slot per device ordinal, set
// after the attribute call succeeded on that device.  Two host threads that
// configure the same kernel on the same device at once both make the (cheap,
// idempotent) attribute call; neither can observe the flag before the call
// has returned in the thread that set it.
#pragma once

#include <atomic>

#include <cuda_runtime.h>

#include "qw6_launch.h"

namespace qw6 {

using DevFlags = std::atomic<int>[QW6K_MAX_DEVICES];

// Current device ordinal, or -1 if it cannot be had or is out of range.
inline int current_device() {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= QW6K_MAX_DEVICES) return -1;
    return dev;
}

// Allow `bytes` of dynamic shared memory for kernel k on the current device
// (once per device and value; a larger request later raises it).  0 or
// QW6K_ERR_CUDA.
template <typename Kern>
inline int smem_optin(DevFlags& flags, Kern k, int bytes) {
    const int dev = current_device();
    if (dev < 0) return QW6K_ERR_CUDA;
    if (flags[dev].load(std::memory_order_acquire) >= bytes) return 0;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
        return QW6K_ERR_CUDA;
    int cur = flags[dev].load(std::memory_order_relaxed);
    while (cur < bytes && !flags[dev].compare_exchange_weak(cur, bytes, std::memory_order_release)) {
    }
    return 0;
}

// Streaming multiprocessors of the current device (cached per device).
inline int device_sms() {
    static std::atomic<int> sms[QW6K_MAX_DEVICES];
    const int dev = current_device();
    if (dev < 0) return 148;
    int n = sms[dev].load(std::memory_order_acquire);
    if (n <= 0) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        sms[dev].store(n, std::memory_order_release);
    }
    return n;
}

}  // namespace qw6
