// Kernel launch with programmatic dependent launch enabled.
#pragma once

#include <cuda_runtime.h>

#include <mutex>

namespace cl {

// ---------------------------------------------------------------------------
// Per-device launch set-up.  A kernel's dynamic shared-memory limit
// (cudaFuncSetAttribute) and the SM count belong to the device that is
// current when they are set or read, so both are cached per device: one
// process may drive several GPUs (one host thread per device, or one thread
// switching devices), and each device is configured the first time a launch
// runs with it current.
// ---------------------------------------------------------------------------
constexpr int kMaxDevices = 64;

// SM count of the current device (cached per device).
inline cudaError_t device_sm_count(int* count) {
    static std::mutex mu;
    static int cache[kMaxDevices] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(mu);
    if (cache[dev] == 0) {
        e = cudaDeviceGetAttribute(&cache[dev], cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
    }
    *count = cache[dev];
    return cudaSuccess;
}

// The dynamic shared-memory limit one kernel has been raised to, per device.
// One instance per kernel (a function-local static beside the launch).
class SmemLimit {
public:
    template <typename Kernel>
    cudaError_t ensure(Kernel kernel, int bytes) {
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
        std::lock_guard<std::mutex> lock(mu_);
        if (bytes > set_[dev]) {
            e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
            if (e != cudaSuccess) return e;
            set_[dev] = bytes;
        }
        return cudaSuccess;
    }

private:
    std::mutex mu_;
    int set_[kMaxDevices] = {};
};

// Process-wide switch (cl_set_pdl): kernels always call griddepcontrol.wait,
// which is a no-op when the launch carries no programmatic edge, so turning
// the attribute off only removes the overlap, never the ordering.
extern int g_pdl_enabled;

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = g_pdl_enabled ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

}  // namespace cl
