// stage_host.cu — host-pointer decode without copy-engine round trips.
//
// leap_attn_decode_host (the call an engine that keeps its activations on
// the host makes per layer, in place of src/inference/FloatTransformer.cpp:
// 404-662) moves q | k_new | v_new in and the output out through the
// context's pinned staging buffer.  Instead of two cudaMemcpyAsync calls it
// launches two kernels chained by programmatic dependent launch:
//   stage_in   reads q|k|v from pinned host memory (mapped, unified address)
//              into the device staging buffer;
//   decode     starts its K/V tile copies while stage_in runs, reads q/k/v
//              after griddepcontrol.wait (it never reads them before), and
//              stores the output, and an error code if a wait gives up,
//              straight into the mapped pinned buffer.
// The caller synchronizes the stream once.  (A third kernel copying the
// output back cost a launch: 33.2 -> 28.5 us per call at ctx 256.)
#include "common.cuh"
#include "ctx.h"

namespace leap {
namespace {

__global__ void __launch_bounds__(256) stage_copy_kernel(const float4 *__restrict__ src,
                                                         float4 *__restrict__ dst, int n4) {
    grid_launch_dependents();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += gridDim.x * blockDim.x)
        dst[i] = src[i];
}

}  // namespace

// n4 float4s from pinned host memory to device memory, ordered after all
// earlier work on the stream (no programmatic overlap with what precedes).
int launch_stage_in(cudaStream_t st, const float *h_src, float *d_dst, int n4) {
    stage_copy_kernel<<<(n4 + 255) / 256, 256, 0, st>>>(
        reinterpret_cast<const float4 *>(h_src), reinterpret_cast<float4 *>(d_dst), n4);
    return cuda_status(cudaGetLastError(), "stage_in launch");
}

}  // namespace leap
