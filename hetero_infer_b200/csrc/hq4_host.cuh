// Host-side helpers shared by the launchers: per-device one-time set-up that
// is safe when several host threads call into the library at once.
#pragma once
#include <atomic>
#include <mutex>

#include <cuda_runtime.h>

namespace hq4 {

constexpr int kMaxDevices = 64;

// A set-up step (a function attribute, a symbol address) that must run once
// on every device before its first use there.  The fast path is one acquire
// load; the first callers on a device serialise on a mutex, and a step that
// fails is retried by the next call.
class PerDeviceOnce {
public:
    template <class F>
    cudaError_t run(F&& step) {
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
        if (done_[dev].load(std::memory_order_acquire)) return cudaSuccess;
        std::lock_guard<std::mutex> lock(mu_);
        if (done_[dev].load(std::memory_order_relaxed)) return cudaSuccess;
        e = step(dev);
        if (e == cudaSuccess) done_[dev].store(true, std::memory_order_release);
        return e;
    }

private:
    std::mutex mu_;
    std::atomic<bool> done_[kMaxDevices] = {};
};

// Raise a kernel's dynamic shared-memory limit once per device.
template <class Kern>
inline cudaError_t smem_opt_in(PerDeviceOnce& once, Kern kern, int bytes) {
    return once.run([&](int) { return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes); });
}

}  // namespace hq4
