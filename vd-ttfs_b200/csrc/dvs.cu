// dvs.cu -- C entry points of the task-3 (DVS gesture, CuLIF) stages.
#include <cstdio>

#include "vdt_internal.h"

using namespace vdt;

namespace {

int cuda_status(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return VDT_OK;
    if (e == cudaErrorInvalidValue) return api_fail(VDT_ERR_UNSUPPORTED, what);
    return api_cuda_fail(e, what);
}

bool culif_ok(int T, int delta) { return T >= 1 && T <= 4096 && delta >= 1 && delta <= 64; }

}  // namespace

extern "C" int vdt_dvs_conv1_raw(const float* d_frames, const float* d_w_oihw, int N, int C_in, int C_out,
                                 int H, int W, int K, int T, int delta, float decay, float th, float* d_out,
                                 vdt_stream stream) {
    api_clear_error();
    if (!d_frames || !d_w_oihw || !d_out || N < 0 || C_in <= 0 || C_out <= 0 || H <= 0 || W <= 0 || K <= 0 ||
        K % 2 == 0 || !culif_ok(T, delta))
        return api_fail(VDT_ERR_INVALID, "bad conv1_raw arguments");
    if (!culif_conv1_supported(C_in, C_out, K, delta))
        return api_fail(VDT_ERR_UNSUPPORTED, "conv1_raw needs delta in {8,16,32}, C_out <= 128, C_in*K*K <= 32");
    if (int s = api_check_buffers(-1, {d_frames, d_w_oihw, d_out})) return s;
    return cuda_status(launch_culif_conv1(d_frames, d_w_oihw, d_out, N, C_in, C_out, H, W, K, T, delta, decay, th,
                                          static_cast<cudaStream_t>(stream)),
                       "conv1_raw launch");
}

extern "C" int vdt_dvs_conv_bucketed(const int* d_off, const int* d_cin, const float* d_tin,
                                     const float* d_w_hwio, int N, int C_in, int C_out, int H, int W, int K,
                                     int T, int delta, float decay, float th, int out_layout, float* d_out,
                                     vdt_stream stream) {
    api_clear_error();
    if (!d_off || !d_cin || !d_tin || !d_w_hwio || !d_out || N < 0 || C_in <= 0 || C_out <= 0 || H <= 0 ||
        W <= 0 || K <= 0 || K % 2 == 0 || !culif_ok(T, delta))
        return api_fail(VDT_ERR_INVALID, "bad conv_bucketed_early arguments");
    if (out_layout != VDT_LAYOUT_NHWC && out_layout != VDT_LAYOUT_NCHW) return api_fail(VDT_ERR_INVALID, "out_layout");
    if (!culif_supported(K, 0, delta, C_in, C_out, T))
        return api_fail(VDT_ERR_UNSUPPORTED, "delta must be a power of two <= 64 and K*K <= 32");
    if (int s = api_check_buffers(-1, {d_off, d_cin, d_tin, d_w_hwio, d_out})) return s;
    IntegParams ip{};
    ip.off = d_off; ip.cin = d_cin; ip.tin = d_tin; ip.W = d_w_hwio; ip.out = d_out;
    ip.B = N; ip.H_in = H; ip.W_in = W; ip.C_in = C_in; ip.H_out = H; ip.W_out = W; ip.C_out = C_out;
    ip.K = K; ip.pad = K / 2; ip.is_fc = 0;
    ip.T = T; ip.delta = delta; ip.NC = (T + delta - 1) / delta;
    ip.inf_time = 9999.0f; ip.culif_decay = decay; ip.culif_th = th;
    ip.out_nchw = out_layout == VDT_LAYOUT_NCHW;
    return cuda_status(launch_culif(ip, static_cast<cudaStream_t>(stream)), "conv_bucketed_early launch");
}

extern "C" int vdt_dvs_conv_dense(const float* d_in, int in_layout, const float* d_w_hwio, int N, int C_in,
                                  int C_out, int H, int W, int K, int T, int delta, float decay, float th,
                                  int out_layout, float* d_out, vdt_stream stream) {
    api_clear_error();
    if (!d_in || !d_w_hwio || !d_out || N < 0 || C_in <= 0 || C_out <= 0 || H <= 0 || W <= 0 || K <= 0 ||
        K % 2 == 0 || !culif_ok(T, delta))
        return api_fail(VDT_ERR_INVALID, "bad conv_dense arguments");
    if ((in_layout != VDT_LAYOUT_NHWC && in_layout != VDT_LAYOUT_NCHW) ||
        (out_layout != VDT_LAYOUT_NHWC && out_layout != VDT_LAYOUT_NCHW))
        return api_fail(VDT_ERR_INVALID, "in_layout / out_layout");
    if (!dense_supported(K, 0, C_in, C_out, T, 0))
        return api_fail(VDT_ERR_UNSUPPORTED, "conv_dense needs K*K*C_in <= 1152 and K*K <= 32");
    if (int s = api_check_buffers(-1, {d_in, d_w_hwio, d_out})) return s;
    IntegParams ip{};
    ip.W = d_w_hwio; ip.out = d_out;
    ip.B = N; ip.H_in = H; ip.W_in = W; ip.C_in = C_in; ip.H_out = H; ip.W_out = W; ip.C_out = C_out;
    ip.K = K; ip.pad = K / 2; ip.is_fc = 0;
    ip.T = T; ip.delta = delta; ip.NC = (T + delta - 1) / delta;
    ip.inf_time = 9999.0f; ip.culif_decay = decay; ip.culif_th = th;
    ip.out_nchw = out_layout == VDT_LAYOUT_NCHW;
    ip.in_nchw = in_layout == VDT_LAYOUT_NCHW;
    return cuda_status(launch_dense_culif(ip, d_in, static_cast<cudaStream_t>(stream)), "conv_dense launch");
}

extern "C" int vdt_dvs_fc2(const int* d_off, const int* d_cin, const float* d_tin, const float* d_w_t, int N,
                           int F_in, int F_out, int T, int delta, float decay, float th, float* d_out,
                           vdt_stream stream) {
    api_clear_error();
    if (!d_off || !d_cin || !d_tin || !d_w_t || !d_out || N < 0 || F_in <= 0 || F_out <= 0 || !culif_ok(T, delta))
        return api_fail(VDT_ERR_INVALID, "bad fc2_bucketed_early arguments");
    if (!culif_supported(1, 1, delta, F_in, F_out, T))
        return api_fail(VDT_ERR_UNSUPPORTED, "delta must be a power of two <= 64");
    if (int s = api_check_buffers(-1, {d_off, d_cin, d_tin, d_w_t, d_out})) return s;
    IntegParams ip{};
    ip.off = d_off; ip.cin = d_cin; ip.tin = d_tin; ip.W = d_w_t; ip.out = d_out;
    ip.B = N; ip.H_in = 1; ip.W_in = 1; ip.C_in = F_in; ip.H_out = 1; ip.W_out = 1; ip.C_out = F_out;
    ip.K = 1; ip.pad = 0; ip.is_fc = 1;
    ip.T = T; ip.delta = delta; ip.NC = (T + delta - 1) / delta;
    ip.inf_time = 9999.0f; ip.culif_decay = decay; ip.culif_th = th;
    return cuda_status(launch_culif(ip, static_cast<cudaStream_t>(stream)), "fc2_bucketed_early launch");
}

extern "C" int vdt_dvs_pool(const float* d_in, float* d_out, int N, int C, int H_in, int W_in, int layout, int T,
                            int delta, float decay, float th, vdt_stream stream) {
    api_clear_error();
    if (!d_in || !d_out || N < 0 || C <= 0 || H_in < 2 || W_in < 2 || !culif_ok(T, delta) ||
        (layout != VDT_LAYOUT_NHWC && layout != VDT_LAYOUT_NCHW))
        return api_fail(VDT_ERR_INVALID, "bad pool_chunk_early arguments");
    if (int s = api_check_buffers(-1, {d_in, d_out})) return s;
    return cuda_status(launch_culif_pool(d_in, d_out, N, C, H_in, W_in, layout, T, delta, decay, th,
                                         static_cast<cudaStream_t>(stream)),
                       "pool_chunk_early launch");
}

namespace {
int fc1_checks(const int* d_off, const int* d_cin, const float* d_tin, const float* d_w_t, const float* d_wrec_t,
               int N, int F_in, int F_out, int T, int delta, const float* d_out) {
    if (!d_off || !d_cin || !d_tin || !d_w_t || !d_wrec_t || !d_out || N < 0 || F_in <= 0 || F_out <= 0 ||
        !culif_ok(T, delta))
        return api_fail(VDT_ERR_INVALID, "bad fc1_bucketed_recurrent arguments");
    if (F_out % 32 != 0 || F_out > 1024)
        return api_fail(VDT_ERR_UNSUPPORTED, "F_out must be a multiple of 32, at most 1024");
    return VDT_OK;
}
}  // namespace

extern "C" int vdt_dvs_fc1_recurrent(const int* d_off, const int* d_cin, const float* d_tin, const float* d_w_t,
                                     const float* d_wrec_t, int N, int F_in, int F_out, int T, int delta,
                                     float decay, float th, float* d_out, vdt_stream stream) {
    api_clear_error();
    if (int st = fc1_checks(d_off, d_cin, d_tin, d_w_t, d_wrec_t, N, F_in, F_out, T, delta, d_out)) return st;
    if (int s = api_check_buffers(-1, {d_off, d_cin, d_tin, d_w_t, d_wrec_t, d_out})) return s;
    return cuda_status(launch_culif_fc1_rec(d_off, d_cin, d_tin, d_w_t, d_wrec_t, d_out, N, F_in, F_out, T, delta,
                                            decay, th, static_cast<cudaStream_t>(stream), nullptr),
                       "fc1_bucketed_recurrent launch");
}

extern "C" size_t vdt_dvs_fc1_scratch_bytes(int N, int F_out, int T, int delta) {
    return culif_fc1_scratch_bytes(N, F_out, T, delta);
}

extern "C" int vdt_dvs_fc1_recurrent_ws(const int* d_off, const int* d_cin, const float* d_tin, const float* d_w_t,
                                        const float* d_wrec_t, int N, int F_in, int F_out, int T, int delta,
                                        float decay, float th, float* d_out, void* d_scratch, size_t scratch_bytes,
                                        vdt_stream stream) {
    api_clear_error();
    if (int st = fc1_checks(d_off, d_cin, d_tin, d_w_t, d_wrec_t, N, F_in, F_out, T, delta, d_out)) return st;
    const size_t need = culif_fc1_scratch_bytes(N, F_out, T, delta);
    if (need > 0 && (!d_scratch || scratch_bytes < need)) {
        char msg[160];
        snprintf(msg, sizeof(msg), "scratch of %zu bytes, the call needs %zu (vdt_dvs_fc1_scratch_bytes)",
                 scratch_bytes, need);
        return api_fail(VDT_ERR_CAPACITY, msg);
    }
    if (need > 0 && (reinterpret_cast<uintptr_t>(d_scratch) & 15))
        return api_fail(VDT_ERR_INVALID, "d_scratch must be 16-byte aligned");
    if (int s = api_check_buffers(-1, {d_off, d_cin, d_tin, d_w_t, d_wrec_t, d_out, need ? d_scratch : nullptr}))
        return s;
    return cuda_status(launch_culif_fc1_rec(d_off, d_cin, d_tin, d_w_t, d_wrec_t, d_out, N, F_in, F_out, T, delta,
                                            decay, th, static_cast<cudaStream_t>(stream),
                                            need ? static_cast<float*>(d_scratch) : nullptr),
                       "fc1_bucketed_recurrent launch");
}

extern "C" int vdt_oihw_to_hwio(const float* d_src, float* d_dst, int O, int I, int K, vdt_stream stream) {
    api_clear_error();
    if (!d_src || !d_dst || O <= 0 || I <= 0 || K <= 0) return api_fail(VDT_ERR_INVALID, "bad permute arguments");
    if (int s = api_check_buffers(-1, {d_src, d_dst})) return s;
    return cuda_status(launch_oihw_to_hwio(d_src, d_dst, O, I, K, static_cast<cudaStream_t>(stream)),
                       "weight permute launch");
}
