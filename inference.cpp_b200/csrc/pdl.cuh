// Programmatic dependent launch (PDL) between the kernels of one decode step.
//
// A kernel launched with programmatic stream serialization may start while the
// previous kernel on the stream is still running.  Such a kernel must execute
// pdl_wait() before it touches anything the previous kernel writes or reads
// (activations, caches, positions); work on data that is constant while the
// previous kernel runs (weight prefetch; KV-cache rows that earlier steps wrote) may
// run before it.  pdl_launch_dependents() lets the next kernel start early; it
// changes scheduling only, never visibility: the next kernel's pdl_wait() still
// returns only after this grid has completed and its writes are visible.  Both
// are no-ops for a kernel launched without the attribute.
#pragma once
#include <cuda_runtime.h>

namespace ib {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

}  // namespace ib
