// ref_t1.cu -- build harness that compiles the reference's own Task-1 (LeNet)
// vdttfs_cuda program unmodified and exposes its kernels and host helpers over
// a C ABI, so tests can pin the CPU oracle against the reference itself.
//
// TEST INFRASTRUCTURE ONLY (output: oracle/_ref/libref_t1.so, git-ignored).
// The reference source is #included from REF_SRC at build time; nothing of it
// is copied into this repository.
#define main vdt_ref_t1_main
#include REF_SRC
#undef main

extern "C" {

int ref_t1_info(int* T, int* chunk, float* tfs, float* vth, float* inf_time) {
    *T = TIME_WINDOW; *chunk = CHUNK; *tfs = TIME_FIRE_START;
    *vth = VTH_INIT; *inf_time = INF_TIME;
    return 0;
}

int ref_t1_update_luts(float* d_decay, float* d_th, float tc_i, float td_i, float tc_f, float td_f) {
    update_LUTs(d_decay, d_th, tc_i, td_i, tc_f, td_f);
    return (int)cudaDeviceSynchronize();
}

int ref_t1_encode(const float* d_img, float* d_out, int n, float tc, float td) {
    k_encode_image<<<(n + 255) / 256, 256>>>(d_img, d_out, n, tc, td);
    return (int)cudaDeviceSynchronize();
}

int ref_t1_bucketize(const float* d_in, int n_cols, int c_in, int* d_cin, float* d_tin, int* d_off) {
    k_bucketize<<<(n_cols + 255) / 256, 256>>>(d_in, n_cols, c_in, d_cin, d_tin, d_off);
    return (int)cudaDeviceSynchronize();
}

int ref_t1_conv_bucketed(float* d_out, const int* d_cin, const float* d_tin, const int* d_off,
                         const float* d_kernel, const float* d_bias,
                         const float* d_decay, const float* d_th, int t_min, int B,
                         int H_in, int W_in, int C_in, int H_out, int W_out, int C_out,
                         int K_h, int K_w, int is_fc) {
    int n = B * H_out * W_out * C_out;
    k_conv_bucketed<<<(n + 255) / 256, 256>>>(d_out, d_cin, d_tin, d_off, d_kernel, d_bias,
        d_decay, d_th, t_min, B, H_in, W_in, C_in, H_out, W_out, C_out, K_h, K_w, is_fc != 0);
    return (int)cudaDeviceSynchronize();
}

int ref_t1_pooling(const float* d_in, float* d_out, int B, int H_in, int W_in, int C) {
    int n = B * (H_in / 2) * (W_in / 2) * C;
    k_pooling<<<(n + 255) / 256, 256>>>(d_in, d_out, B, H_in, W_in, C);
    return (int)cudaDeviceSynchronize();
}

// A LeNet-style network driven through the reference's own launch_layer /
// launch_pool / update_LUTs (t1:222-240, flow t1:290-305) on host spike
// times.  Per layer i: shape[i*7 + 0..6] = {H_in, W_in, C_in, H_out, W_out,
// C_out, K}; is_fc[i]; pool[i].  d_kernels/d_biases hold each layer's device
// tensors; tc/td its fire constants.  One repetition = H2D copy of the spike
// times, all layers (with the reference's syncs), D2H copy of the last
// layer's first-spike times and the host argmin (t1:313-315).
int ref_t1_run_net(int B, int L, const int* shape, const int* is_fc, const int* pool,
                   float* const* d_kernels, float* const* d_biases, const float* tc,
                   const float* td, float tc_in, float td_in, const float* h_spikes,
                   float* h_out, int* h_pred, int reps, float* ms) {
    std::vector<LayerWeights> layers(L);
    size_t max_map = 0, max_elems = 0, max_cols = 0;
    for (int i = 0; i < L; ++i) {
        const int* s = shape + 7 * i;
        layers[i].d_kernel = d_kernels[i]; layers[i].d_bias = d_biases[i];
        layers[i].tc_fire = tc[i]; layers[i].td = td[i];
        layers[i].k_h = layers[i].k_w = s[6];
        layers[i].c_in = s[2]; layers[i].c_out = s[5];
        size_t in_elems = (size_t)B * s[0] * s[1] * s[2];
        size_t out_elems = (size_t)B * s[3] * s[4] * s[5];
        max_map = std::max(max_map, std::max(in_elems, out_elems));
        max_elems = std::max(max_elems, in_elems);
        max_cols = std::max(max_cols, is_fc[i] ? (size_t)B : (size_t)B * s[0] * s[1]);
    }
    const size_t f = sizeof(float);
    float* bufs[3];
    for (auto& b : bufs) cudaMalloc(&b, max_map * f);
    cudaMalloc(&g_bkt_cin, max_elems * sizeof(int));
    cudaMalloc(&g_bkt_tin, max_elems * sizeof(float));
    cudaMalloc(&g_bkt_off, max_cols * OFF_STRIDE * sizeof(int));
    float *d_LUT_decay, *d_LUT_th;
    cudaMalloc(&d_LUT_decay, TIME_WINDOW * f); cudaMalloc(&d_LUT_th, TIME_WINDOW * f);
    const int* last = shape + 7 * (L - 1);
    const int K = last[5];
    std::vector<float> h((size_t)B * K);
    cudaEvent_t e0, e1; cudaEventCreate(&e0); cudaEventCreate(&e1);
    cudaEventRecord(e0);
    for (int r = 0; r < reps; ++r) {
        cudaMemcpy(bufs[0], h_spikes, (size_t)B * shape[0] * shape[1] * shape[2] * f, cudaMemcpyHostToDevice);
        int xi = 0;
        for (int i = 0; i < L; ++i) {
            const int* s = shape + 7 * i;
            float tci = i ? layers[i - 1].tc_fire : tc_in, tdi = i ? layers[i - 1].td : td_in;
            update_LUTs(d_LUT_decay, d_LUT_th, tci, tdi, layers[i].tc_fire, layers[i].td);
            int yi = (xi + 1) % 3, zi = (xi + 2) % 3;
            launch_layer(bufs[xi], bufs[yi], s[0], s[1], s[2], s[3], s[4], s[5], i,
                         d_LUT_decay, d_LUT_th, layers, B, is_fc[i] != 0);
            if (pool[i]) { launch_pool(bufs[yi], bufs[zi], s[3], s[4], s[5], B); yi = zi; }
            xi = yi;
        }
        cudaMemcpy(h.data(), bufs[xi], (size_t)B * K * f, cudaMemcpyDeviceToHost);
        for (int bi = 0; bi < B; ++bi) {
            float mt = INF_TIME; int p = -1;
            for (int k = 0; k < K; ++k) { float t = h[(size_t)bi * K + k]; if (t < mt) { mt = t; p = k; } }
            h_pred[bi] = p;
        }
    }
    cudaEventRecord(e1); cudaEventSynchronize(e1);
    cudaEventElapsedTime(ms, e0, e1);
    memcpy(h_out, h.data(), (size_t)B * K * f);
    int err = (int)cudaGetLastError();
    for (auto b : bufs) cudaFree(b);
    cudaFree(d_LUT_decay); cudaFree(d_LUT_th);
    cudaFree(g_bkt_cin); cudaFree(g_bkt_tin); cudaFree(g_bkt_off);
    g_bkt_cin = nullptr; g_bkt_tin = nullptr; g_bkt_off = nullptr;
    cudaEventDestroy(e0); cudaEventDestroy(e1);
    return err;
}

}  // extern "C"
