// stage_host.cu — host-pointer decode without copy-engine round trips.
//
// leap_attn_decode_host (the call an engine that keeps its activations on
// the host makes per layer, in place of src/inference/FloatTransformer.cpp:
// 404-662) moves q | k_new | v_new in and the output out through the
// context's pinned staging buffer.  Instead of two cudaMemcpyAsync calls it
// launches three kernels chained by programmatic dependent launch:
//   stage_in   reads q|k|v from pinned host memory (mapped, unified address)
//              into the device staging buffer;
//   decode     starts its K/V tile copies while stage_in runs and reads q/k/v
//              after griddepcontrol.wait (it never reads them before);
//   stage_out  waits for the decode grid, then writes out | error word into
//              pinned host memory with plain stores.
// The caller synchronizes the stream once.
#include "common.cuh"
#include "ctx.h"

namespace leap {
namespace {

template <bool WAIT>
__global__ void __launch_bounds__(256) stage_copy_kernel(const float4 *__restrict__ src,
                                                         float4 *__restrict__ dst, int n4) {
    if (WAIT) grid_dependency_wait();  // src is written by the previous grid
    grid_launch_dependents();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += gridDim.x * blockDim.x)
        dst[i] = src[i];
}

}  // namespace

// n4 float4s from pinned host memory to device memory, ordered after all
// earlier work on the stream (no programmatic overlap with what precedes).
int launch_stage_in(cudaStream_t st, const float *h_src, float *d_dst, int n4) {
    stage_copy_kernel<false><<<(n4 + 255) / 256, 256, 0, st>>>(
        reinterpret_cast<const float4 *>(h_src), reinterpret_cast<float4 *>(d_dst), n4);
    return cuda_status(cudaGetLastError(), "stage_in launch");
}

// n4 float4s from device memory to pinned host memory once the previous
// grid (launched with programmatic serialization) has completed.
int launch_stage_out(cudaStream_t st, const float *d_src, float *h_dst, int n4) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((n4 + 255) / 256);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_status(cudaLaunchKernelEx(&cfg, stage_copy_kernel<true>,
                                          reinterpret_cast<const float4 *>(d_src),
                                          reinterpret_cast<float4 *>(h_dst), n4),
                       "stage_out launch");
}

}  // namespace leap
