/* Programmatic dependent launch for the layer kernels (kda.cu, mla.cu).
 *
 * A kernel launched behind another on the same stream with the
 * programmatic-serialisation attribute may start once every CTA of that
 * kernel has run launch_dependents (or exited). Its wait returns when that
 * kernel has finished and its writes are visible. So a kernel reads only
 * constants, or data final before the kernel ahead began, before its wait.
 * Both instructions are no-ops in a kernel launched without the attribute,
 * so the same kernel serves both kinds of launch. */
#pragma once

#include <cuda_runtime.h>

namespace wc_pdl {

__device__ __forceinline__ void trigger() { asm volatile("griddepcontrol.launch_dependents;"); }
__device__ __forceinline__ void wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                   bool pdl, Args... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

} /* namespace wc_pdl */
