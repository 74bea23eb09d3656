// smem_attr.cuh -- raise a kernel's dynamic shared-memory limit once per GPU.
//
// cudaFuncSetAttribute acts on the kernel's instance in the CURRENT device's
// context, so a process that drives several GPUs (one context per device)
// must raise the limit on each of them.  A SmemAttr kept beside the kernel
// remembers, per device ordinal, the largest size already granted.
#pragma once
#include <cuda_runtime.h>

#include <atomic>

namespace velo {

constexpr int kMaxDevices = 64;

struct SmemAttr {
    std::atomic<int> granted[kMaxDevices];
    SmemAttr() {
        for (auto& g : granted) g.store(0, std::memory_order_relaxed);
    }
};

// Ensure `kernel` may launch with `bytes` of dynamic shared memory on the
// current device.  Sizes up to the default 48 KB need nothing.  Two threads
// racing on the first launch may both set the attribute: harmless.
template <typename Kernel>
inline cudaError_t ensure_smem(SmemAttr& s, Kernel* kernel, int bytes) {
    if (bytes <= 48 * 1024) return cudaSuccess;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const bool cached = dev >= 0 && dev < kMaxDevices;
    if (cached && s.granted[dev].load(std::memory_order_acquire) >= bytes) return cudaSuccess;
    e = cudaFuncSetAttribute(reinterpret_cast<const void*>(kernel),
                             cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess || !cached) return e;
    int cur = s.granted[dev].load(std::memory_order_relaxed);
    while (cur < bytes && !s.granted[dev].compare_exchange_weak(cur, bytes, std::memory_order_release)) {
    }
    return cudaSuccess;
}

}  // namespace velo
