// k_static.cu -- fixed device scratch for the allocation-free MoE entry point
// (qw6cu_moe_decode_noalloc in qw6_cuda.h).
//
// The scratch is a file-scope __device__ array, so the module loader reserves
// it on every GPU that loads this library and keeps it until the process
// exits; no call ever allocates.  In host code the array's name is only a
// host-side stand-in, never a device address, so the address handed to the
// kernels comes from cudaGetSymbolAddress, looked up once per device with
// that device current.
#include <cuda_runtime.h>

#include "qw6_launch.h"

static __device__ __align__(256) unsigned char g_qw6_static_scratch[QW6K_STATIC_SCRATCH_BYTES];

extern "C" int qw6k_static_scratch(void** ptr, size_t* bytes) {
    static void* addr[QW6K_MAX_DEVICES];
    static int ready[QW6K_MAX_DEVICES];
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= QW6K_MAX_DEVICES) return QW6K_ERR_CUDA;
    if (!ready[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_qw6_static_scratch) != cudaSuccess || !p) return QW6K_ERR_CUDA;
        addr[dev] = p;
        ready[dev] = 1;
    }
    *ptr = addr[dev];
    *bytes = QW6K_STATIC_SCRATCH_BYTES;
    return 0;
}
