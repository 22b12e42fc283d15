// k_static.cu -- fixed device scratch for the allocation-free MoE entry point
// (qw6cu_moe_decode_noalloc in qw6_cuda.h).
//
// The scratch is a file-scope __device__ array, so the module loader reserves
// it on every GPU that loads this library and keeps it until the process
// exits; no call ever allocates.  In host code the array's name is only a
// host-side stand-in, never a device address, so the address handed to the
// kernels comes from cudaGetSymbolAddress, looked up once per device with
// that device current.
#include <atomic>

#include <cuda_runtime.h>

#include "qw6_launch.h"

static __device__ __align__(256) unsigned char g_qw6_static_scratch[QW6K_STATIC_SCRATCH_BYTES];

// One slot per device ordinal.  The address is published with release order
// after the device's set-up succeeded and read with acquire order, so a
// thread that sees a non-null slot also sees a finished set-up; two threads
// racing on a device's first call both do the set-up (it is idempotent) and
// store the same value.
static std::atomic<void*> g_scratch_addr[QW6K_MAX_DEVICES];

// First call on a device: the array's device address, and every decode
// kernel configured and loaded (qw6k_moe_decode_setup), so that later calls
// only enqueue launches.
extern "C" int qw6k_static_scratch(void** ptr, size_t* bytes) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= QW6K_MAX_DEVICES) return QW6K_ERR_CUDA;
    void* p = g_scratch_addr[dev].load(std::memory_order_acquire);
    if (!p) {
        if (cudaGetSymbolAddress(&p, g_qw6_static_scratch) != cudaSuccess || !p) return QW6K_ERR_CUDA;
        if (qw6k_moe_decode_setup() != 0) return QW6K_ERR_CUDA;
        g_scratch_addr[dev].store(p, std::memory_order_release);
    }
    *ptr = p;
    *bytes = QW6K_STATIC_SCRATCH_BYTES;
    return 0;
}
