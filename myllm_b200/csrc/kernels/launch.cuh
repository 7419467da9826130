// Kernel launch with programmatic dependent launch enabled.
#pragma once

#include <cuda_runtime.h>

namespace cl {

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
