// Kernel launch with programmatic dependent launch (PDL).
//
// launch_k() launches like <<<grid, block, smem, st>>> but, while g_pdl is
// set, with cudaLaunchAttributeProgrammaticStreamSerialization: the kernel
// may be scheduled as soon as every CTA of the previous kernel in the stream
// has executed dep_launch() (common.cuh), so its launch latency and its
// prologue (barrier setup, TMEM allocation, weight loads) overlap the tail of
// the previous kernel. Every kernel launched this way calls dep_wait() before
// it touches data of other kernels. Inside stream capture the attribute
// becomes a programmatic edge of the CUDA graph.
#pragma once

#include <cuda_runtime.h>

#include <utility>

namespace n550 {

extern bool g_pdl;

template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                     Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = g_pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace n550
