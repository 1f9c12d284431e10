// f3s_probe.cu -- throughput of the tensor-core instruction the fused kernel
// uses (mma.sync.m16n8k16, f16 x f16 -> f32), measured on the current device:
// the tensor-side roofline denominator of k_fused3s.  Every warp of every SM
// runs independent accumulator chains back to back (no memory traffic).
#include <cuda_runtime.h>
#include "f3s_internal.cuh"

namespace f3s {

constexpr int kProbeChains = 8;

// Sink for the probe's sums (keeps the chains live).
static __device__ float g_probe_sink;

__global__ void k_probe_mma(int iters) {
    const uint32_t lane = threadIdx.x & 31;
    uint32_t a[4] = {0x3c003c00u ^ lane, 0x3c013c00u ^ lane, 0x3c003c01u ^ lane, 0x3c013c01u ^ lane};
    const uint32_t b0 = 0x3c003c00u + lane, b1 = b0 + 7;
    float acc[kProbeChains][4];
#pragma unroll
    for (int j = 0; j < kProbeChains; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    for (int i = 0; i < iters; ++i) {
#pragma unroll
        for (int j = 0; j < kProbeChains; ++j) mma_16816(acc[j], a, b0, b1);
    }
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < kProbeChains; ++j) s += acc[j][0] + acc[j][1] + acc[j][2] + acc[j][3];
    if (blockIdx.x == 0 && threadIdx.x == 0) g_probe_sink = s;
}

static int probe_mma_sync(int warps_per_sm, int iters, double* tflops, cudaStream_t stream) {
    if (warps_per_sm < 1 || warps_per_sm > 32 || iters < 1 || !tflops) return F3S_ERR_INVALID_VALUE;
    const int sms = num_sms_of_current_device();
    const int block = 32 * warps_per_sm;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    F3S_CUDA_TRY(cudaEventCreate(&e0));
    cudaError_t e = cudaEventCreate(&e1);
    if (e != cudaSuccess) {
        cudaEventDestroy(e0);
        note_cuda_error(e);
        return F3S_ERR_CUDA;
    }
    float ms = 0.f;
    k_probe_mma<<<sms, block, 0, stream>>>(16);  // warm-up
    e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaEventRecord(e0, stream);
    if (e == cudaSuccess) {
        k_probe_mma<<<sms, block, 0, stream>>>(iters);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaEventRecord(e1, stream);
    if (e == cudaSuccess) e = cudaEventSynchronize(e1);
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (e != cudaSuccess) {
        note_cuda_error(e);
        return F3S_ERR_CUDA;
    }
    const double flops = (double)sms * warps_per_sm * iters * kProbeChains * 16.0 * 8.0 * 16.0 * 2.0;
    *tflops = ms > 0.f ? flops / (ms * 1e-3) / 1e12 : 0.0;
    return F3S_SUCCESS;
}

}  // namespace f3s

extern "C" {

int f3s_probe_mma_sync(int32_t warps_per_sm, int32_t iters, double* h_tflops, f3s_stream_t stream) {
    return f3s::probe_mma_sync(warps_per_sm, iters, h_tflops, (cudaStream_t)stream);
}

}  // extern "C"
