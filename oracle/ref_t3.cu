// ref_t3.cu -- build harness that compiles the reference's own Task-3 (DVS,
// CuLIF) vdttfs_cuda program unmodified and exposes its kernels over a C ABI,
// so tests can pin the CPU oracle against the reference itself.
//
// TEST INFRASTRUCTURE ONLY (output: oracle/_ref/libref_t3.so, git-ignored).
// The reference source is #included from REF_SRC at build time.
// conv1_raw_early and fc1_bucketed_recurrent hard-code the reference's shapes
// (2x32x32 input, 64 conv1 channels, T=160 time stride, 128 hidden neurons),
// so they can only be driven at those shapes.
#define main vdt_ref_t3_main
#include REF_SRC
#undef main

extern "C" {

int ref_t3_info(int* T, int* chunk, int* classes, float* decay_conv, float* decay_fc,
                float* th_conv, float* th_fc) {
    *T = T_TOTAL; *chunk = CHUNK_SIZE; *classes = NUM_CLASSES;
    *decay_conv = decay_syn_conv; *decay_fc = decay_syn_fc;
    *th_conv = v_th_conv; *th_fc = v_th_fc;
    return 0;
}

// frames [N, 2, 32, 32, 160]; w [64, 2, 3, 3]; out [N, 64, 32, 32]
int ref_t3_conv1(const float* d_frames, float* d_out, const float* d_w, int N) {
    int n = N * 64 * 32 * 32;
    conv1_raw_early<<<GET_BLOCKS(n), 256>>>(d_frames, d_out, d_w, N, decay_syn_conv, v_th_conv);
    return (int)cudaDeviceSynchronize();
}

int ref_t3_bucketize_conv(const float* d_in, int N, int C, int H, int W, int* d_cin, float* d_tin, int* d_off) {
    k_bucketize_conv<<<GET_BLOCKS(N * H * W), 256>>>(d_in, N, C, H, W, d_cin, d_tin, d_off);
    return (int)cudaDeviceSynchronize();
}

int ref_t3_bucketize_fc(const float* d_in, int N, int F, int* d_cin, float* d_tin, int* d_off) {
    k_bucketize_fc<<<GET_BLOCKS(N), 256>>>(d_in, N, F, d_cin, d_tin, d_off);
    return (int)cudaDeviceSynchronize();
}

int ref_t3_conv(const int* d_cin, const float* d_tin, const int* d_off, float* d_out, const float* d_w,
                int N, int C_in, int C_out, int H, int W) {
    int n = N * C_out * H * W;
    conv_bucketed_early<<<GET_BLOCKS(n), 256>>>(d_cin, d_tin, d_off, d_out, d_w, N, C_in, C_out, H, W,
                                                decay_syn_conv, v_th_conv);
    return (int)cudaDeviceSynchronize();
}

int ref_t3_pool(const float* d_in, float* d_out, int N, int C, int H_in, int W_in) {
    int n = N * C * (H_in / 2) * (W_in / 2);
    pool_chunk_early<<<GET_BLOCKS(n), 256>>>(d_in, d_out, N, C, H_in, W_in, decay_syn_conv, v_th_conv);
    return (int)cudaDeviceSynchronize();
}

// 128 hidden neurons (one 128-thread CTA per sample, t3:171-200)
int ref_t3_fc1(const int* d_cin, const float* d_tin, const int* d_off, float* d_out,
               const float* d_w, const float* d_w_rec, int N, int F_in) {
    fc1_bucketed_recurrent<<<N, 128>>>(d_cin, d_tin, d_off, d_out, d_w, d_w_rec, N, F_in, 128,
                                       decay_syn_fc, v_th_fc);
    return (int)cudaDeviceSynchronize();
}

int ref_t3_fc2(const int* d_cin, const float* d_tin, const int* d_off, float* d_out, const float* d_w,
               int N, int F_in, int F_out) {
    int n = N * F_out;
    fc2_bucketed_early<<<GET_BLOCKS(n), 256>>>(d_cin, d_tin, d_off, d_out, d_w, N, F_in, F_out,
                                               decay_syn_fc, v_th_fc);
    return (int)cudaDeviceSynchronize();
}

}  // extern "C"
