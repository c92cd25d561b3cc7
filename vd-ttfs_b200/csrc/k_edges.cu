// k_edges.cu -- the small kernels on either side of the integrator:
//   * k_build_luts   update_LUTs (t1:208-216, t2:236-243) for every layer of a
//                    model in one launch (grid.y = layer).  The exponent is
//                    evaluated in double precision and rounded once to fp32
//                    (a correctly rounded exp for these arguments); the
//                    argument itself is formed in fp32 exactly like the
//                    reference: -((float)t - td) / tc.
//   * k_encode       k_encode_image's log encoder (t1:32-42, t2:32-42) and the
//                    linear t = floor((1 - x) * T) encoder.
//   * k_pool_min     k_pooling (t1:164-181, t2:192-209), 4 channels per thread.
//   * k_layer_vmem   k_layer_vmem (t2:172-190): one warp per image, lanes over
//                    output channels, the input vector staged in shared memory.
//   * k_readout      the host argmin/argmax loops of t1:313-315, t2:391-392,
//                    t3:295-296, one thread per image.
#include "vdt_internal.h"

namespace vdt {
namespace {

__device__ __forceinline__ void build_lut_pair(const LutJob& j, int T, int decay_len, float vth) {
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < decay_len || t < T;
         t += gridDim.x * blockDim.x) {
        if (t < decay_len) {
            const float x = __fdiv_rn(-__fsub_rn((float)t, j.td_integ), j.tc_integ);
            j.decay[t] = (float)exp((double)x);
        }
        if (t < T) {
            const float x = __fdiv_rn(-__fsub_rn((float)t, j.td_fire), j.tc_fire);
            j.th[t] = __fmul_rn(vth, (float)exp((double)x));
        }
    }
}

__global__ void k_build_luts(const LutJob* jobs, int T, int decay_len, float vth) {
    build_lut_pair(jobs[blockIdx.y], T, decay_len, vth);
}

__global__ void k_build_lut_one(LutJob j, int T, int decay_len, float vth) {
    build_lut_pair(j, T, decay_len, vth);
}

__global__ void k_encode(const float* __restrict__ px, float* __restrict__ out, long long n,
                         int encoder, float tc, float td, int T, float inf_time) {
    chain_release();
    chain_wait();
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        out[i] = encode_pixel(__ldg(px + i), encoder, tc, td, T, inf_time);
    }
}

__global__ void k_pool_min(const float* __restrict__ in, float* __restrict__ out, int B,
                           int H_in, int W_in, int C, float inf_time) {
    chain_release();
    chain_wait();
    const int H_out = H_in / 2, W_out = W_in / 2, C4 = C / 4;
    const long long n = (long long)B * H_out * W_out * C4;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const int c4 = (int)(i % C4);
        long long r = i / C4;
        const int w = (int)(r % W_out);
        r /= W_out;
        const int h = (int)(r % H_out);
        const long long b = r / H_out;
        float4 m = make_float4(inf_time, inf_time, inf_time, inf_time);
#pragma unroll
        for (int dy = 0; dy < 2; ++dy)
#pragma unroll
            for (int dx = 0; dx < 2; ++dx) {
                const float4 t = __ldg(reinterpret_cast<const float4*>(
                    in + ((b * H_in + 2 * h + dy) * W_in + 2 * w + dx) * C) + c4);
                if (t.x < m.x) m.x = t.x;
                if (t.y < m.y) m.y = t.y;
                if (t.z < m.z) m.z = t.z;
                if (t.w < m.w) m.w = t.w;
            }
        reinterpret_cast<float4*>(out)[i] = m;
    }
}

__global__ void k_pool_min_scalar(const float* __restrict__ in, float* __restrict__ out, int B,
                                  int H_in, int W_in, int C, float inf_time) {
    chain_release();
    chain_wait();
    const int H_out = H_in / 2, W_out = W_in / 2;
    const long long n = (long long)B * H_out * W_out * C;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const int c = (int)(i % C);
        long long r = i / C;
        const int w = (int)(r % W_out);
        r /= W_out;
        const int h = (int)(r % H_out);
        const long long b = r / H_out;
        float m = inf_time;
        for (int dy = 0; dy < 2; ++dy)
            for (int dx = 0; dx < 2; ++dx) {
                const float t = __ldg(in + ((b * H_in + 2 * h + dy) * W_in + 2 * w + dx) * C + c);
                if (t < m) m = t;
            }
        out[i] = m;
    }
}

// is value v a strict improvement on m for readout `mode`?
__device__ __forceinline__ bool readout_better(float v, float m, int mode) {
    return mode == VDT_READ_ARGMAX ? v > m : v < m;
}

__global__ void k_layer_vmem(const float* __restrict__ in, const float* __restrict__ W,
                             const float* __restrict__ bias, const float* __restrict__ lut,
                             int B, int C_in, int C_out, int T, float tfs, float inf_time,
                             float* __restrict__ out, int32_t* __restrict__ pred, int mode) {
    extern __shared__ float s_in[];                  // [warps][C_in] values, then flags
    chain_release();
    chain_wait();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const long long img = (long long)blockIdx.x * (blockDim.x >> 5) + warp;
    if (img >= B) return;
    float* x = s_in + warp * C_in;
    unsigned char* use = reinterpret_cast<unsigned char*>(s_in + (blockDim.x >> 5) * C_in) + warp * C_in;
    for (int i = lane; i < C_in; i += 32) {
        const float t = __ldg(in + img * C_in + i);
        const bool u = t < inf_time && (t - tfs) <= (float)T;
        float lv = 0.0f;
        if (u) {
            int ti = (int)t;
            ti = ti < 0 ? 0 : (ti > T ? T : ti);
            lv = __ldg(lut + ti);
        }
        x[i] = lv;
        use[i] = u ? 1 : 0;
    }
    __syncwarp();
    // the readout fused in: each lane scans its own outputs in increasing
    // index order from k_readout's start value (for ARGMIN_LOWEST: lane 0
    // starts at output 0, the other lanes at +infinity), then the lanes'
    // bests merge, a lower index winning a tie -- k_readout's sequential scan
    // keeps the first index of the best value
    float m = mode == VDT_READ_ARGMAX ? -1e9f : (mode == VDT_READ_ARGMIN_FIRST ? inf_time : __int_as_float(0x7f800000));
    int pbest = -1;
    for (int c = lane; c < C_out; c += 32) {
        float acc = 0.0f;
        for (int i = 0; i < C_in; ++i)
            if (use[i]) acc = fmaf(__ldg(W + (long long)i * C_out + c), x[i], acc);
        const float v = acc + __ldg(bias + c);
        out[img * C_out + c] = v;
        if (mode == VDT_READ_ARGMIN_LOWEST && c == 0) { m = v; pbest = 0; }
        else if (readout_better(v, m, mode)) { m = v; pbest = c; }
    }
    if (pred) {
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) {
            const float m2 = __shfl_down_sync(0xffffffffu, m, d);
            const int p2 = __shfl_down_sync(0xffffffffu, pbest, d);
            const bool take = p2 >= 0 && (pbest < 0 || readout_better(m2, m, mode) || (m2 == m && p2 < pbest));
            if (take) { m = m2; pbest = p2; }
        }
        if (lane == 0) pred[img] = pbest;
    }
}

__global__ void k_readout(const float* __restrict__ out, int B, int K, int mode, float inf_time,
                          int32_t* __restrict__ pred) {
    chain_release();
    chain_wait();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    const float* o = out + (long long)b * K;
    int p;
    if (mode == VDT_READ_ARGMIN_FIRST) {
        float m = inf_time; p = -1;
        for (int i = 0; i < K; ++i) { const float v = o[i]; if (v < m) { m = v; p = i; } }
    } else if (mode == VDT_READ_ARGMIN_LOWEST) {
        float m = o[0]; p = 0;
        for (int i = 1; i < K; ++i) { const float v = o[i]; if (v < m) { m = v; p = i; } }
    } else {
        float m = -1e9f; p = -1;
        for (int i = 0; i < K; ++i) { const float v = o[i]; if (v > m) { m = v; p = i; } }
    }
    pred[b] = p;
}

unsigned grid_for(long long n, int threads) {
    long long g = (n + threads - 1) / threads;
    const long long cap = 148LL * 16;                // 16 resident CTAs per SM
    return (unsigned)(g < 1 ? 1 : (g > cap ? cap : g));
}

}  // namespace

cudaError_t launch_build_luts(const LutJob* d_jobs, int n_jobs, int T, int decay_len, float vth,
                              cudaStream_t s) {
    if (n_jobs <= 0) return cudaSuccess;
    const int n = decay_len > T ? decay_len : T;
    dim3 grid((n + 127) / 128, n_jobs);
    k_build_luts<<<grid, 128, 0, s>>>(d_jobs, T, decay_len, vth);
    return cudaGetLastError();
}

cudaError_t launch_build_lut_one(const LutJob& j, int T, int decay_len, float vth, cudaStream_t s) {
    const int n = decay_len > T ? decay_len : T;
    k_build_lut_one<<<(n + 127) / 128, 128, 0, s>>>(j, T, decay_len, vth);
    return cudaGetLastError();
}

cudaError_t launch_encode(const float* px, float* out, long long n, int encoder, float tc, float td,
                          int T, float inf_time, cudaStream_t s) {
    if (n <= 0) return cudaSuccess;
    return launch_chain(k_encode, dim3(grid_for(n, 256)), dim3(256), 0, s, px, out, n, encoder, tc, td, T,
                        inf_time);
}

cudaError_t launch_pool_min(const float* in, float* out, int B, int H_in, int W_in, int C,
                            float inf_time, cudaStream_t s) {
    const long long n = (long long)B * (H_in / 2) * (W_in / 2) * C;
    if (n <= 0) return cudaSuccess;
    const bool vec = (C % 4 == 0) && ((uintptr_t)in % 16 == 0) && ((uintptr_t)out % 16 == 0);
    if (vec)
        return launch_chain(k_pool_min, dim3(grid_for(n / 4, 256)), dim3(256), 0, s, in, out, B, H_in, W_in, C,
                            inf_time);
    return launch_chain(k_pool_min_scalar, dim3(grid_for(n, 256)), dim3(256), 0, s, in, out, B, H_in, W_in, C,
                        inf_time);
}

cudaError_t launch_layer_vmem(const float* in, const float* W, const float* bias,
                              const float* lut_decay, int B, int C_in, int C_out, int T,
                              float tfs, float inf_time, float* out, cudaStream_t s,
                              int32_t* pred, int readout) {
    if (B <= 0) return cudaSuccess;
    const int warps = 4;
    const size_t smem = (size_t)warps * C_in * (sizeof(float) + 1);
    if (smem > 48 * 1024) return cudaErrorInvalidValue;
    return launch_chain(k_layer_vmem, dim3((B + warps - 1) / warps), dim3(warps * 32), smem, s, in, W, bias,
                        lut_decay, B, C_in, C_out, T, tfs, inf_time, out, pred, readout);
}

cudaError_t launch_readout(const float* out, int B, int K, int mode, float inf_time, int32_t* pred,
                           cudaStream_t s) {
    if (B <= 0) return cudaSuccess;
    return launch_chain(k_readout, dim3((B + 127) / 128), dim3(128), 0, s, out, B, K, mode, inf_time, pred);
}

}  // namespace vdt
