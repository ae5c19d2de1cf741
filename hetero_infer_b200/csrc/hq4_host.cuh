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

// Split-K factor for `tiles` output tiles of `kern` (one CTA per tile and
// split, the splits of a tile launched as one 1 x ks x 1 cluster): the ks in
// [1, kmax] with the most splits per wave, the fewer splits on a tie.  A
// cluster's CTAs share one GPC, so a device holds fewer clusters of ks than
// SMs / ks (28 clusters of 5 do not fit 148 SMs at one CTA per SM); the
// device's own count (cudaOccupancyMaxActiveClusters) is cached per
// (device, kernel, ks, threads, shared memory).  `smem_limit` is the
// kernel's dynamic shared-memory opt-in, the same value its launcher sets.
class SplitPicker {
public:
    int pick(const void* kern, int threads, size_t smem, int smem_limit, int tiles, int kmax) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || tiles <= 0) return 1;
        int best = 1;
        double best_score = 0.0;
        for (int ks = 1; ks <= kmax; ks++) {
            const int cap = capacity(dev, kern, threads, smem, smem_limit, ks);
            if (cap <= 0) continue;
            const int waves = (tiles + cap - 1) / cap;
            const double score = (double)ks / waves;
            if (score > best_score) {
                best_score = score;
                best = ks;
            }
        }
        return best;
    }

    // Clusters of ks CTAs (1 x ks x 1) of `kern` the current device holds at
    // once; 0 when the query fails.
    int capacity(const void* kern, int threads, size_t smem, int smem_limit, int ks) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess) return 0;
        return capacity(dev, kern, threads, smem, smem_limit, ks);
    }

private:
    struct Entry {
        int dev, threads, ks, cap;
        const void* kern;
        size_t smem;
    };
    int capacity(int dev, const void* kern, int threads, size_t smem, int smem_limit, int ks) {
        std::lock_guard<std::mutex> lock(mu_);
        for (int i = 0; i < n_; i++) {
            const Entry& e = cache_[i];
            if (e.dev == dev && e.kern == kern && e.threads == threads && e.smem == smem && e.ks == ks) return e.cap;
        }
        int cap = 0;
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_limit) == cudaSuccess) {
            cudaLaunchAttribute a;
            a.id = cudaLaunchAttributeClusterDimension;
            a.val.clusterDim.x = 1;
            a.val.clusterDim.y = (unsigned)ks;
            a.val.clusterDim.z = 1;
            cudaLaunchConfig_t lc = {};
            lc.gridDim = dim3(1, (unsigned)ks, 1);
            lc.blockDim = dim3((unsigned)threads);
            lc.dynamicSmemBytes = smem;
            lc.attrs = &a;
            lc.numAttrs = 1;
            if (cudaOccupancyMaxActiveClusters(&cap, kern, &lc) != cudaSuccess) cap = 0;
        }
        if (cap <= 0) {
            (void)cudaGetLastError();  // a refused query leaves no sticky error
            return 0;
        }
        if (n_ < kCache) cache_[n_++] = Entry{dev, threads, ks, cap, kern, smem};
        return cap;
    }
    static constexpr int kCache = 256;
    std::mutex mu_;
    Entry cache_[kCache];
    int n_ = 0;
};

}  // namespace hq4
