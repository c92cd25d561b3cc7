// dvs_net.cu -- the task-3 (DVS gesture, CuLIF) network as one engine model:
// the flat weight blob loader and the per-batch stage sequence of the
// reference's main (t3:234-296), run by the same vdt_ctx machinery as the
// task-1/2 networks (ctx-owned workspace, one captured CUDA graph per batch
// size, the host and pipelined host entry points).
//
// Stages (NCHW spike-time maps between them, as in the reference):
//   conv1  conv1_raw_early over the dense frames          t3:30-65
//   conv2  conv_bucketed_early (+ its k_bucketize_conv)    t3:70-90, :109-143
//   pool1  pool_chunk_early                               t3:146-168
//   conv3  conv_bucketed_early (+ its k_bucketize_conv)
//   pool2  pool_chunk_early
//   fc1    k_bucketize_fc + fc1_bucketed_recurrent         t3:93-106, :171-200
//   fc2    k_bucketize_fc + fc2_bucketed_early             t3:203-225
//   readout  argmin with class 0 as the start              t3:295-296
// A conv stage whose per-pixel fan-in fits k_dense (K*K*C_in <= 1152) reads
// its input map itself (bucketing fused in); otherwise it is bucketized
// first.  Every stage after conv1 runs at chunk width 8 when the configured
// width and 8 both divide T: each neuron then sees the same per-step inputs
// in the same order and its scan still ends at T, so the results are the
// same bit for bit, with narrower per-chunk tables.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <vector>

#include "engine_types.h"
#include "vdt_internal.h"

namespace vdt {

int dvs_internal_delta(const vdt_dvs_desc& d) {
    return (d.T % d.delta == 0 && d.T % 8 == 0) ? 8 : d.delta;
}

void dvs_stage_sizes(const vdt_dvs_desc& d, size_t out[DVS_STAGES]) {
    const size_t hw = (size_t)d.H * d.W;
    out[DVS_CONV1] = (size_t)d.c1 * hw;
    out[DVS_CONV2] = (size_t)d.c2 * hw;
    out[DVS_POOL1] = (size_t)d.c2 * hw / 4;
    out[DVS_CONV3] = (size_t)d.c3 * hw / 4;
    out[DVS_POOL2] = (size_t)d.c3 * hw / 16;
    out[DVS_FC1] = (size_t)d.hidden;
    out[DVS_FC2] = (size_t)d.classes;
}

namespace {

size_t fc1_in(const vdt_dvs_desc& d) { return (size_t)d.c3 * (d.H / 4) * (d.W / 4); }

bool conv_dense(const vdt_dvs_desc& d, int c_in, int c_out) {
    return dense_supported(d.k, 0, c_in, c_out, d.T, 0);
}

}  // namespace

DvsSizes dvs_sizes(const vdt_model* m, long long B) {
    const vdt_dvs_desc& d = m->dvs;
    DvsSizes z;
    size_t st[DVS_STAGES];
    dvs_stage_sizes(d, st);
    for (size_t v : st) z.act = std::max(z.act, (size_t)B * v);
    const int di = dvs_internal_delta(d);
    const size_t OS = (size_t)(d.T + di - 1) / di + 1;
    const size_t hw = (size_t)d.H * d.W;
    // bucket lists of the bucketed stages: FC1 and FC2 rows, and a conv stage
    // that k_dense cannot take
    z.bkt = std::max((size_t)B * fc1_in(d), (size_t)B * d.hidden);
    z.off = (size_t)B * OS;
    if (!conv_dense(d, d.c1, d.c2)) { z.bkt = std::max(z.bkt, (size_t)B * hw * d.c1); z.off = std::max(z.off, (size_t)B * hw * OS); }
    if (!conv_dense(d, d.c2, d.c3)) { z.bkt = std::max(z.bkt, (size_t)B * hw / 4 * d.c2); z.off = std::max(z.off, (size_t)B * hw / 4 * OS); }
    z.scratch_bytes = culif_fc1_scratch_bytes((int)B, d.hidden, d.T, di);
    return z;
}

namespace {

// A CuLIF conv stage on an NCHW map x -> NCHW map y (same-pad, K = d.k).
cudaError_t conv_stage(vdt_ctx* c, int stage, const float* x, float* y, const float* w_hwio, int B, int c_in,
                       int c_out, int H, int W, int di) {
    const vdt_dvs_desc& d = c->m->dvs;
    IntegParams ip{};
    ip.W = w_hwio; ip.out = y;
    ip.B = B; ip.H_in = H; ip.W_in = W; ip.C_in = c_in; ip.H_out = H; ip.W_out = W; ip.C_out = c_out;
    ip.K = d.k; ip.pad = d.k / 2; ip.is_fc = 0;
    ip.T = d.T; ip.delta = di; ip.NC = (d.T + di - 1) / di;
    ip.inf_time = 9999.0f; ip.culif_decay = d.decay_conv; ip.culif_th = d.th_conv;
    ip.out_nchw = 1;
    if (conv_dense(d, c_in, c_out)) {
        ip.in_nchw = 1;
        StageTimer st(c, stage, 1);
        return launch_dense_culif(ip, x, c->stream);
    }
    BktParams bp{};
    bp.in = x; bp.n_cols = (long long)B * H * W; bp.c_in = c_in;
    bp.layout = VDT_LAYOUT_NCHW; bp.hw = (long long)H * W;
    bp.T = d.T; bp.delta = di; bp.NC = ip.NC; bp.tfs = 0.0f; bp.tb_mode = VDT_TB_TRUNC; bp.inf_time = 9999.0f;
    bp.off = c->off; bp.cin = c->cin; bp.tin = c->tin;
    {
        StageTimer st(c, stage, 0);
        cudaError_t e = launch_bucketize(bp, c->stream);
        if (e != cudaSuccess) return e;
    }
    ip.off = c->off; ip.cin = c->cin; ip.tin = c->tin;
    StageTimer st(c, stage, 1);
    return launch_culif(ip, c->stream);
}

// Buckets of [B, F] feature rows (k_bucketize_fc) into the ctx's lists.
cudaError_t bucketize_rows(vdt_ctx* c, int stage, const float* x, int B, int F, int di) {
    const vdt_dvs_desc& d = c->m->dvs;
    BktParams bp{};
    bp.in = x; bp.n_cols = B; bp.c_in = F; bp.layout = VDT_LAYOUT_NHWC; bp.hw = 1;
    bp.T = d.T; bp.delta = di; bp.NC = (d.T + di - 1) / di; bp.tfs = 0.0f; bp.tb_mode = VDT_TB_TRUNC;
    bp.inf_time = 9999.0f;
    bp.off = c->off; bp.cin = c->cin; bp.tin = c->tin;
    StageTimer st(c, stage, 0);
    return launch_bucketize(bp, c->stream);
}

}  // namespace

int dvs_enqueue(vdt_ctx* c, const float* d_frames, int B, float* d_out, int32_t* d_pred, float* const* trace) {
    const vdt_model* m = c->m;
    const vdt_dvs_desc& d = m->dvs;
    const DvsWeights& w = m->dw;
    cudaStream_t s = c->stream;
    const int di = dvs_internal_delta(d);
    const int H = d.H, W = d.W, H2 = d.H / 2, W2 = d.W / 2;
    size_t st_size[DVS_STAGES];
    dvs_stage_sizes(d, st_size);
    float* const A = c->act[0];
    float* const Bm = c->act[1];
    float* const Cm = c->act[2];
    cudaError_t e = cudaSuccess;
    // copies a stage's map to the caller's trace buffer
    auto keep = [&](int stage, const float* y) -> cudaError_t {
        if (!trace || !trace[stage]) return cudaSuccess;
        return cudaMemcpyAsync(trace[stage], y, (size_t)B * st_size[stage] * sizeof(float), cudaMemcpyDeviceToDevice, s);
    };
#define VDT_STAGE(call)                                            \
    do {                                                           \
        e = (call);                                                \
        if (e != cudaSuccess) return api_cuda_fail(e, #call);      \
    } while (0)
    {   // conv1 over the raw frames, at the configured chunk width (its frame windows)
        StageTimer t(c, DVS_CONV1, 1);
        VDT_STAGE(launch_culif_conv1(d_frames, w.conv1, A, B, d.in_c, d.c1, H, W, d.k, d.T, d.delta, d.decay_conv,
                                     d.th_conv, s));
    }
    VDT_STAGE(keep(DVS_CONV1, A));
    VDT_STAGE(conv_stage(c, DVS_CONV2, A, Bm, w.conv2, B, d.c1, d.c2, H, W, di));
    VDT_STAGE(keep(DVS_CONV2, Bm));
    {
        StageTimer t(c, DVS_POOL1, 1);
        VDT_STAGE(launch_culif_pool(Bm, Cm, B, d.c2, H, W, VDT_LAYOUT_NCHW, d.T, di, d.decay_conv, d.th_conv, s));
    }
    VDT_STAGE(keep(DVS_POOL1, Cm));
    VDT_STAGE(conv_stage(c, DVS_CONV3, Cm, A, w.conv3, B, d.c2, d.c3, H2, W2, di));
    VDT_STAGE(keep(DVS_CONV3, A));
    {
        StageTimer t(c, DVS_POOL2, 1);
        VDT_STAGE(launch_culif_pool(A, Bm, B, d.c3, H2, W2, VDT_LAYOUT_NCHW, d.T, di, d.decay_conv, d.th_conv, s));
    }
    VDT_STAGE(keep(DVS_POOL2, Bm));
    const int F = (int)fc1_in(d);
    VDT_STAGE(bucketize_rows(c, DVS_FC1, Bm, B, F, di));
    {
        StageTimer t(c, DVS_FC1, 1);
        VDT_STAGE(launch_culif_fc1_rec(c->off, c->cin, c->tin, w.fc1_t, w.rec_t, Cm, B, F, d.hidden, d.T, di,
                                       d.decay_fc, d.th_fc, s, c->scratch_bytes ? c->scratch : nullptr));
    }
    VDT_STAGE(keep(DVS_FC1, Cm));
    VDT_STAGE(bucketize_rows(c, DVS_FC2, Cm, B, d.hidden, di));
    {
        IntegParams ip{};
        ip.off = c->off; ip.cin = c->cin; ip.tin = c->tin; ip.W = w.fc2_t; ip.out = d_out;
        ip.B = B; ip.H_in = 1; ip.W_in = 1; ip.C_in = d.hidden; ip.H_out = 1; ip.W_out = 1; ip.C_out = d.classes;
        ip.K = 1; ip.pad = 0; ip.is_fc = 1;
        ip.T = d.T; ip.delta = di; ip.NC = (d.T + di - 1) / di;
        ip.inf_time = 9999.0f; ip.culif_decay = d.decay_fc; ip.culif_th = d.th_fc;
        StageTimer t(c, DVS_FC2, 1);
        VDT_STAGE(launch_culif(ip, s));
    }
    VDT_STAGE(keep(DVS_FC2, d_out));
    if (d_pred) VDT_STAGE(launch_readout(d_out, B, d.classes, VDT_READ_ARGMIN_LOWEST, 9999.0f, d_pred, s));
#undef VDT_STAGE
    if (c->profiling) c->prof_batches++;
    return VDT_OK;
}

}  // namespace vdt

using namespace vdt;

namespace {

int check_dvs_desc(const vdt_dvs_desc* d) {
    if (!d) return api_fail(VDT_ERR_INVALID, "DVS descriptor is NULL");
    if (d->in_c <= 0 || d->H <= 0 || d->W <= 0 || d->c1 <= 0 || d->c2 <= 0 || d->c3 <= 0 || d->hidden <= 0 ||
        d->classes <= 0 || d->k <= 0 || d->k % 2 == 0)
        return api_fail(VDT_ERR_INVALID, "DVS descriptor: sizes must be positive, k odd");
    if (d->H % 4 || d->W % 4) return api_fail(VDT_ERR_INVALID, "DVS descriptor: H and W must be multiples of 4 (two 2x2 pools)");
    if (d->T < 1 || d->T > 4096 || d->delta < 1 || d->delta > 64)
        return api_fail(VDT_ERR_INVALID, "DVS descriptor: T in [1, 4096], delta in [1, 64]");
    if (!culif_conv1_supported(d->in_c, d->c1, d->k, d->delta))
        return api_fail(VDT_ERR_UNSUPPORTED, "conv1 needs delta in {8,16,32}, c1 <= 128, in_c*k*k <= 32");
    const int di = dvs_internal_delta(*d);
    if (!dense_supported(d->k, 0, d->c1, d->c2, d->T, 0) && !culif_supported(d->k, 0, di, d->c1, d->c2, d->T))
        return api_fail(VDT_ERR_UNSUPPORTED, "conv2: no integrator takes this shape");
    if (!dense_supported(d->k, 0, d->c2, d->c3, d->T, 0) && !culif_supported(d->k, 0, di, d->c2, d->c3, d->T))
        return api_fail(VDT_ERR_UNSUPPORTED, "conv3: no integrator takes this shape");
    if (d->hidden % 32 || d->hidden > 1024) return api_fail(VDT_ERR_UNSUPPORTED, "hidden must be a multiple of 32, at most 1024");
    if (!culif_supported(1, 1, di, d->hidden, d->classes, d->T))
        return api_fail(VDT_ERR_UNSUPPORTED, "fc2: no integrator takes this shape");
    const double fin = (double)d->c3 * (d->H / 4) * (d->W / 4);
    if (fin * d->hidden >= 2147483647.0) return api_fail(VDT_ERR_UNSUPPORTED, "FC1 above 2^31 weights");
    return VDT_OK;
}

}  // namespace

extern "C" int vdt_model_load_dvs_flat(const void* blob, size_t nbytes, const vdt_dvs_desc* d, int device,
                                       vdt_model** out) {
    api_clear_error();
    if (!out) return api_fail(VDT_ERR_INVALID, "out is NULL");
    *out = nullptr;
    if (!blob) return api_fail(VDT_ERR_INVALID, "blob is NULL");
    if (int s = check_dvs_desc(d)) return s;
    const size_t k2 = (size_t)d->k * d->k, F = fc1_in(*d), hid = d->hidden;
    // flat blob order (the reference's dvsgesture_weights_meta.txt, t3:237-241):
    // conv1, conv2, conv3 (OIHW), fc1 recurrent [hidden, hidden], fc1
    // [hidden, F_in], fc2 [classes, hidden]
    const size_t n_c1 = (size_t)d->c1 * d->in_c * k2, n_c2 = (size_t)d->c2 * d->c1 * k2,
                 n_c3 = (size_t)d->c3 * d->c2 * k2, n_rec = hid * hid, n_fc1 = hid * F,
                 n_fc2 = (size_t)d->classes * hid;
    const size_t total = n_c1 + n_c2 + n_c3 + n_rec + n_fc1 + n_fc2;
    // the reference reads a fixed-size file and never touches floats past the
    // last layer, so a longer blob is accepted
    if (nbytes / sizeof(float) < total) {
        char msg[160];
        snprintf(msg, sizeof msg, "DVS blob holds %zu floats, the network needs %zu", nbytes / sizeof(float), total);
        return api_fail(VDT_ERR_BLOB, msg);
    }
    const float* src = static_cast<const float*>(blob);
    std::vector<float> h(total);
    const float* p = src;
    float* q = h.data();
    memcpy(q, p, n_c1 * sizeof(float));                      // conv1 stays OIHW
    p += n_c1; q += n_c1;
    auto oihw_to_hwio = [&](int O, int I) {
        for (int o = 0; o < O; ++o)
            for (int i = 0; i < I; ++i)
                for (size_t t = 0; t < k2; ++t) q[(t * I + i) * O + o] = p[((size_t)o * I + i) * k2 + t];
        p += (size_t)O * I * k2; q += (size_t)O * I * k2;
    };
    oihw_to_hwio(d->c2, d->c1);
    oihw_to_hwio(d->c3, d->c2);
    auto transpose = [&](size_t rows, size_t cols) {       // [rows, cols] -> [cols, rows]
        for (size_t r = 0; r < rows; ++r)
            for (size_t cc = 0; cc < cols; ++cc) q[cc * rows + r] = p[r * cols + cc];
        p += rows * cols; q += rows * cols;
    };
    float* const h_rec = q;
    transpose(hid, hid);
    float* const h_fc1 = q;
    transpose(hid, F);
    float* const h_fc2 = q;
    transpose((size_t)d->classes, hid);

    auto m = new vdt_model();
    m->device = device;
    m->is_dvs = true;
    m->dvs = *d;
    m->n_classes = d->classes;
    m->in_elems = (size_t)d->in_c * d->H * d->W * d->T;
    m->cfg.T = d->T;
    m->cfg.delta = d->delta;
    m->cfg.inf_time = 9999.0f;
    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    cudaError_t e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaMalloc(&m->arena, total * sizeof(float));
    if (e == cudaSuccess) e = cudaMemcpy(m->arena, h.data(), total * sizeof(float), cudaMemcpyHostToDevice);
    if (prev >= 0) cudaSetDevice(prev);
    if (e != cudaSuccess) {
        if (m->arena) cudaFree(m->arena);
        delete m;
        return api_cuda_fail(e, "DVS weight upload");
    }
    m->weight_bytes = total * sizeof(float);
    float* a = m->arena;
    m->dw.conv1 = a;
    m->dw.conv2 = a + n_c1;
    m->dw.conv3 = a + n_c1 + n_c2;
    m->dw.rec_t = a + (h_rec - h.data());
    m->dw.fc1_t = a + (h_fc1 - h.data());
    m->dw.fc2_t = a + (h_fc2 - h.data());
    *out = m;
    return VDT_OK;
}
