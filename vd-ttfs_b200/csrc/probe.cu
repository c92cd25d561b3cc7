// probe.cu -- measured denominators for the integrators' roofline on the GPU
// the bench runs on, at its current clocks: FP32 FMA throughput (the
// integrators' arithmetic: one FMA per fetched synapse) and the L2-to-SM read
// bandwidth (every fetched synapse reads one 4-byte weight from L1 or L2).
// No counterpart in the reference; measurement helpers only.
#include <algorithm>

#include "vdt_internal.h"

namespace vdt {
namespace {

constexpr int kChains = 8;     // independent packed accumulator pairs per thread

// kChains independent fma.rn.f32x2 chains (2 FMAs each) per thread, iters
// times: 2 * kChains * iters FMAs per thread.
__global__ void k_probe_fma(float* out, int iters, float a, float b) {
    float x[2 * kChains];
#pragma unroll
    for (int j = 0; j < 2 * kChains; ++j) x[j] = (float)(threadIdx.x + j) * 1e-3f;
    for (int i = 0; i < iters; ++i) {
#pragma unroll
        for (int j = 0; j < kChains; ++j) {
            asm volatile("{\n\t"
                         ".reg .b64 p, q, r;\n\t"
                         "mov.b64 p, {%0, %1};\n\t"
                         "mov.b64 q, {%2, %2};\n\t"
                         "mov.b64 r, {%3, %3};\n\t"
                         "fma.rn.f32x2 p, p, q, r;\n\t"
                         "mov.b64 {%0, %1}, p;\n\t"
                         "}"
                         : "+f"(x[2 * j]), "+f"(x[2 * j + 1])
                         : "f"(a), "f"(b));
        }
    }
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < 2 * kChains; ++j) s += x[j];
    if (s == 12345.678f) out[blockIdx.x] = s;            // keeps the chains live
}

constexpr int kL2Unroll = 4;   // independent 16-byte loads in flight per thread

// Every thread reads 16-byte vectors of an L2-resident buffer, cached in L2
// only (ld.global.cg), kL2Unroll independent loads at a time, `reps` passes
// over its CTA's slice (a whole number of blockDim * kL2Unroll vectors).
__global__ void k_probe_l2(const float4* __restrict__ buf, long long per_cta, int reps, float* out) {
    const float4* p = buf + per_cta * blockIdx.x;
    float s = 0.0f;
    for (int r = 0; r < reps; ++r) {
        for (long long i = threadIdx.x; i < per_cta; i += (long long)blockDim.x * kL2Unroll) {
            float4 v[kL2Unroll];
#pragma unroll
            for (int u = 0; u < kL2Unroll; ++u)
                asm volatile("ld.global.cg.v4.f32 {%0, %1, %2, %3}, [%4];"
                             : "=f"(v[u].x), "=f"(v[u].y), "=f"(v[u].z), "=f"(v[u].w)
                             : "l"(p + i + (long long)u * blockDim.x));
#pragma unroll
            for (int u = 0; u < kL2Unroll; ++u) s += v[u].x + v[u].y + v[u].z + v[u].w;
        }
    }
    if (s == 12345.678f) out[blockIdx.x] = s;
}

}  // namespace
}  // namespace vdt

using namespace vdt;

extern "C" int vdt_measure_peaks(int device, double* fma_per_s, double* l2_read_bytes_per_s) {
    api_clear_error();
    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return api_cuda_fail(e, "cudaSetDevice");
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    const size_t l2_bytes = 32u << 20;                   // resident in B200's 126 MB L2
    float* buf = nullptr;
    float* out = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    double best_fma = 0.0, best_l2 = 0.0;
    e = cudaMalloc(&buf, l2_bytes);
    if (e == cudaSuccess) e = cudaMalloc(&out, 65536 * sizeof(float));
    if (e == cudaSuccess) e = cudaMemset(buf, 0, l2_bytes);
    if (e == cudaSuccess) e = cudaEventCreate(&e0);
    if (e == cudaSuccess) e = cudaEventCreate(&e1);
    const int fma_blocks = sms * 8, fma_threads = 256, iters = 4096;
    const int l2_blocks = sms * 4, l2_threads = 512, reps = 64;   // 2048 threads per SM
    for (int trial = 0; trial < 4 && e == cudaSuccess; ++trial) {
        float ms = 0.0f;
        cudaEventRecord(e0);
        k_probe_fma<<<fma_blocks, fma_threads>>>(out, iters, 0.999f, 1e-7f);
        cudaEventRecord(e1);
        e = cudaEventSynchronize(e1);
        if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, e0, e1);
        if (e == cudaSuccess && trial > 0)
            best_fma = std::max(best_fma, 2.0 * kChains * iters * (double)fma_blocks * fma_threads / (ms * 1e-3));
        if (e != cudaSuccess) break;
        const long long n_vec = (long long)(l2_bytes / sizeof(float4));
        const long long chunk = (long long)l2_threads * kL2Unroll;
        const long long per_cta = n_vec / l2_blocks / chunk * chunk;
        cudaEventRecord(e0);
        k_probe_l2<<<l2_blocks, l2_threads>>>(reinterpret_cast<const float4*>(buf), per_cta, reps, out);
        cudaEventRecord(e1);
        e = cudaEventSynchronize(e1);
        if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, e0, e1);
        const double moved = (double)per_cta * l2_blocks * sizeof(float4) * reps;
        if (e == cudaSuccess && trial > 0) best_l2 = std::max(best_l2, moved / (ms * 1e-3));
    }
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    cudaFree(buf);
    cudaFree(out);
    if (prev >= 0) cudaSetDevice(prev);
    if (e != cudaSuccess) return api_cuda_fail(e, "peak probes");
    if (fma_per_s) *fma_per_s = best_fma;
    if (l2_read_bytes_per_s) *l2_read_bytes_per_s = best_l2;
    return VDT_OK;
}
