// launch.cuh — kernel launches with optional programmatic dependent launch.
//
// With PDL on, a kernel may start while the previous kernel on the stream is
// still running. Every kernel therefore calls pdl_wait() before it reads
// anything an earlier kernel wrote or writes anything an earlier kernel
// reads; only reads of constant data (weights) may come before it. Each
// kernel calls pdl_trigger() early so that its successor can be scheduled.
#pragma once

#include <cuda_runtime.h>

#include <utility>

#include "kernels.h"

template <class... KArgs, class... Args>
static inline cudaError_t fbk_launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                     Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    if (fbk_pdl_enabled()) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}
