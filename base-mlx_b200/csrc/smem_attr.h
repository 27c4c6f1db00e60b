// Per-device opt-in to large dynamic shared memory.
//
// cudaFuncAttributeMaxDynamicSharedMemorySize is a property of a kernel on
// one device: raising it on device 0 leaves device 1 at the 48 KB default.
// ensure_max_dyn_smem raises it the first time a kernel is launched with a
// given size on the calling thread's current device, under a lock, so that
// host threads and devices that share the library never launch a kernel
// whose opt-in is missing.
#pragma once
#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <utility>

namespace qw {

inline cudaError_t ensure_max_dyn_smem_fn(const void* func, int bytes) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, int> done;  // (kernel, device) -> bytes already allowed
    std::lock_guard<std::mutex> lk(mu);
    const auto key = std::make_pair(func, dev);
    const auto it = done.find(key);
    if (it != done.end() && it->second >= bytes) return cudaSuccess;
    e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) done[key] = bytes;
    return e;
}

template <typename Kernel>
cudaError_t ensure_max_dyn_smem(Kernel* kernel, int bytes) {
    return ensure_max_dyn_smem_fn(reinterpret_cast<const void*>(kernel), bytes);
}

}  // namespace qw
