// vdt_internal.h -- declarations shared by the engine's kernel files and the
// host runtime (not part of the public ABI; see include/vdttfs.h).
#pragma once

#include <cuda_runtime.h>
#include <cstdint>
#include <initializer_list>
#include <utility>

#include "vdttfs.h"

namespace vdt {

// error reporting shared by every C entry point (vdt_last_error)
void api_clear_error();
int api_fail(int status, const char* msg);
int api_cuda_fail(cudaError_t e, const char* what);
int api_check_cfg(const vdt_time_cfg* c);
// every non-null pointer is device memory of `dev` (< 0: the current device)
int api_check_buffers(int dev, std::initializer_list<const void*> ptrs);

// ------------------------------------------------------- launch overlap (PDL)
// Kernels of the layer chain are launched with programmatic stream
// serialization: a kernel's CTAs may start while its predecessor's last wave
// drains.  Every chained kernel signals chain_release() first and calls
// chain_wait() before it reads anything a predecessor wrote or writes any
// global memory; before that it may only read model constants (weights,
// LUTs) and use shared memory.  griddepcontrol.wait returns once the
// predecessor grid has completed and its writes are visible (immediately
// when the kernel was launched without the attribute).
bool overlap_enabled();

__device__ __forceinline__ void chain_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void chain_release() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_chain(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = overlap_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------- bucketize
struct BktParams {
    const float* in;
    long long n_cols;
    int c_in;
    int layout;        // VDT_LAYOUT_NHWC / VDT_LAYOUT_NCHW
    long long hw;      // sites per image (NCHW)
    int T, delta, NC;  // NC = ceil(T / delta)
    float tfs;         // TIME_FIRE_START
    int tb_mode;       // VDT_TB_FLOOR_STAGGER / VDT_TB_TRUNC
    float inf_time;
    int* off;          // [n_cols, NC + 1]
    int* cin;          // [n_cols, c_in]
    float* tin;        // [n_cols, c_in]
    unsigned long long* events;  // optional event counter (may be null)
};
cudaError_t launch_bucketize(const BktParams& p, cudaStream_t s);

// ---------------------------------------------------------------- integrate
struct IntegParams {
    const int* off;
    const int* cin;
    const float* tin;
    const float* W;          // HWIO [K, K, C_in, C_out] or [C_in, C_out]
    const float* bias;       // [C_out]
    const float* lut_decay;  // [decay_len]
    const float* lut_th;     // [T]
    float* out;              // NHWC [B, H_out, W_out, C_out]
    int B, H_in, W_in, C_in, H_out, W_out, C_out, K, pad, is_fc;
    int T, delta, NC, t_min, lut_mode, decay_len;
    float tfs, inf_time;
    unsigned long long* fetched;  // optional synapse counter (may be null)
    // task-3 CuLIF layers (launch_culif): constant current decay and threshold;
    // out_nchw = 1 writes the output map NCHW [B, C_out, H_out, W_out]
    float culif_decay, culif_th;
    int out_nchw;
    int in_nchw;   // launch_dense_culif: the input spike map is NCHW [B, C_in, H_in, W_in]
    // k_dense / k_sorted (LIF conv layers): when set, the layer's 2x2 min pool
    // [B, H_out / 2, W_out / 2, C_out] is written here instead of the map
    // (`out` is not written); the caller fills it with the bytes 0x7F first
    float* pool_out;
    // k_dense (LIF): the input map holds pixels, encoded with encode_pixel
    // as they are read (VDT_ENC_NONE: spike times)
    int encoder;
    float enc_tc, enc_td;
};

// k_encode_image's log encoder (t1:32-42, t2:32-42) and the linear
// t = floor((1 - x) * T) encoder for one pixel value; shared by k_encode and
// the first layer's fused read, so both give the same bits
__device__ __forceinline__ float encode_pixel(float x, int encoder, float tc, float td, int T, float inf_time) {
    if (encoder == VDT_ENC_LOG) {
        if (x < 1e-5) return inf_time;
        float tf = fmaf(-tc, logf(x), td);
        if (tf < 0.0f) tf = 0.0f;
        const float ts = ceilf(tf);
        return ts > (float)T ? inf_time : ts;
    }
    if (x < 1e-5f) return inf_time;
    const float ts = floorf(__fmul_rn(__fsub_rn(1.0f, x), (float)T));
    return ts > (float)T ? inf_time : ts;
}
cudaError_t launch_integrate(const IntegParams& p, cudaStream_t s);
// true when launch_integrate supports this (K, delta, C_out) combination
bool integrate_supported(int K, int is_fc, int delta, int C_out, int T, int decay_len);

// Integrator fused with the bucketing for small per-pixel fan-in: reads the
// NHWC spike map `in` directly (same results as bucketize + integrate).
cudaError_t launch_dense(const IntegParams& p, const float* in, cudaStream_t s);
bool dense_supported(int K, int is_fc, int C_in, int C_out, int T, int decay_len);
// The same for task-3 CuLIF conv layers (conv_bucketed_early t3:109-143 fused
// with its k_bucketize_conv, t3:70-89): reads the spike map (NHWC or NCHW),
// scans every step up to NC * delta.  Supported where dense_supported is.
cudaError_t launch_dense_culif(const IntegParams& p, const float* in, cudaStream_t s);

// One thread per output pixel for narrow conv layers (K*K*C_in <= 32,
// C_out <= 16): reads the NHWC spike map directly, same results.
cudaError_t launch_thread(const IntegParams& p, const float* in, cudaStream_t s);
// The same with the layer's 2x2 min pool fused in: p.out is the pooled map
// [B, H_out / 2, W_out / 2, C_out] (H_out, W_out >= 2).
cudaError_t launch_thread_pooled(const IntegParams& p, const float* in, cudaStream_t s);
bool thread_supported(int K, int is_fc, int C_in, int C_out, int T, int decay_len);

// Chunk integrator with per-chunk slot sorting (reference bucket layout,
// same results as launch_integrate, fewer instructions per event).
cudaError_t launch_sorted(const IntegParams& p, cudaStream_t s);
// chunk width the runtime buckets k_sorted layers at (outside counting passes)
constexpr int kSortedDelta = 8;

// Task-3 bucketed CuLIF layer (conv_bucketed_early t3:109-143 with K = 3,
// fc2_bucketed_early t3:203-225 with is_fc): k_sorted's event path with the
// CuLIF step; buckets by tb = (int)t (VDT_TB_TRUNC), weights HWIO / [in, out].
cudaError_t launch_culif(const IntegParams& p, cudaStream_t s);
bool culif_supported(int K, int is_fc, int delta, int C_in, int C_out, int T);

// Task-3 layers that are not bucketed integrators (k_culif.cu)
bool culif_conv1_supported(int C_in, int C_out, int K, int delta);
cudaError_t launch_culif_conv1(const float* frames, const float* w_oihw, float* out, int N, int C_in, int C_out,
                               int H, int W, int K, int T, int delta, float decay, float th, cudaStream_t s);
cudaError_t launch_culif_pool(const float* in, float* out, int N, int C, int H_in, int W_in, int layout,
                              int T, int delta, float decay, float th, cudaStream_t s);
// scratch: the feed-forward sums' buffer (culif_fc1_scratch_bytes; 0 = not
// used for this shape); NULL allocates it stream-ordered
cudaError_t launch_culif_fc1_rec(const int* off, const int* cin, const float* tin, const float* w_t,
                                 const float* wrec_t, float* out, int N, int F_in, int F_out, int T, int delta,
                                 float decay, float th, cudaStream_t s, float* scratch);
size_t culif_fc1_scratch_bytes(int N, int F_out, int T, int delta);
cudaError_t launch_oihw_to_hwio(const float* src, float* dst, int O, int I, int K, cudaStream_t s);
bool sorted_supported(int K, int is_fc, int delta, int C_in, int C_out, int T, int decay_len);

// -------------------------------------------------------------- edges / LUT
struct LutJob {            // one layer's table pair
    float tc_integ, td_integ, tc_fire, td_fire;
    float* decay;          // [decay_len]
    float* th;             // [T]
};
cudaError_t launch_build_luts(const LutJob* d_jobs, int n_jobs, int T, int decay_len,
                              float vth_init, cudaStream_t s);
cudaError_t launch_build_lut_one(const LutJob& j, int T, int decay_len, float vth_init,
                                 cudaStream_t s);
cudaError_t launch_encode(const float* px, float* out, long long n, int encoder, float tc,
                          float td, int T, float inf_time, cudaStream_t s);
cudaError_t launch_pool_min(const float* in, float* out, int B, int H_in, int W_in, int C,
                            float inf_time, cudaStream_t s);
// pred (may be null): the readout (VDT_READ_* mode) of the outputs, fused in
cudaError_t launch_layer_vmem(const float* in, const float* W, const float* bias,
                              const float* lut_decay, int B, int C_in, int C_out, int T,
                              float tfs, float inf_time, float* out, cudaStream_t s,
                              int32_t* pred = nullptr, int readout = VDT_READ_ARGMAX);
cudaError_t launch_readout(const float* out, int B, int K, int mode, float inf_time,
                           int32_t* pred, cudaStream_t s);

}  // namespace vdt
