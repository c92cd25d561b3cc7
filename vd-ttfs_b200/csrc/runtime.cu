// runtime.cu -- host runtime of the engine and the C ABI (include/vdttfs.h).
//
//  * vdt_model: parses the reference's weight blob (load_weights, t1:185-206 /
//    t2:213-234) against an explicit topology, uploads all weights into one
//    device allocation and builds every layer's LUT pair once (the reference
//    rebuilds them on the host and re-uploads them with blocking copies before
//    every layer of every batch, t2:343-384).
//  * vdt_ctx: the per-stream workspace (ping-pong activation maps, bucket
//    lists) and a cache of captured CUDA graphs, one per (batch, input kind,
//    counting) -- the reference synchronises the device after every launch
//    (t2:260,273,280,286); here a batch is one graph launch.
//  * the per-stage entry points wrap single kernels for drop-in use.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <initializer_list>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "engine_types.h"
#include "vdt_internal.h"

using namespace vdt;

namespace {

thread_local std::string g_last_error;

int fail(int status, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return status;
}

int cuda_fail(cudaError_t e, const char* what) {
    if (e == cudaErrorMemoryAllocation)
        return fail(VDT_ERR_OOM, "%s: %s", what, cudaGetErrorString(e));
    return fail(VDT_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define VDT_CUDA(call)                                      \
    do {                                                    \
        cudaError_t e_ = (call);                            \
        if (e_ != cudaSuccess) return cuda_fail(e_, #call); \
    } while (0)

// Restores the caller's current device on scope exit.
struct DeviceGuard {
    int prev = -1;
    bool ok = false;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) {
            prev = -1;
            cudaGetLastError();  // leave no error behind for other libraries
            return;
        }
        if (dev < 0 || cudaSetDevice(dev) == cudaSuccess) ok = true;
        else cudaGetLastError();
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

int check_cfg(const vdt_time_cfg* c) {
    if (!c) return fail(VDT_ERR_INVALID, "time config is NULL");
    if (c->T < 1 || c->T > 4096) return fail(VDT_ERR_INVALID, "T=%d out of range [1, 4096]", c->T);
    if (c->delta < 1 || c->delta > 64)
        return fail(VDT_ERR_INVALID, "delta=%d out of range [1, 64]", c->delta);
    if (c->lut_mode != VDT_LUT_BY_TB && c->lut_mode != VDT_LUT_BY_TIN)
        return fail(VDT_ERR_INVALID, "lut_mode=%d", c->lut_mode);
    const int need = c->lut_mode == VDT_LUT_BY_TIN ? c->T + 1 : c->T;
    if (c->decay_len < need)
        return fail(VDT_ERR_INVALID, "decay_len=%d < %d required by lut_mode %d", c->decay_len,
                    need, c->lut_mode);
    if (c->lut_source != VDT_LUT_DEVICE && c->lut_source != VDT_LUT_HOST_LIBM)
        return fail(VDT_ERR_INVALID, "lut_source=%d", c->lut_source);
    return VDT_OK;
}

// Device buffers handed to a call must live on the device the call runs on
// (or be managed memory): a buffer of another GPU would otherwise be read by
// the kernels as a bad address.  dev < 0 means the current device.
int check_device_buffers(int dev, std::initializer_list<const void*> ptrs) {
    if (dev < 0 && cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return fail(VDT_ERR_CUDA, "no current device");
    }
    for (const void* p : ptrs) {
        if (!p) continue;
        cudaPointerAttributes a{};
        if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
            cudaGetLastError();
            return fail(VDT_ERR_INVALID, "buffer %p is not a CUDA allocation", p);
        }
        if (a.type == cudaMemoryTypeManaged) continue;
        if (a.type != cudaMemoryTypeDevice)
            return fail(VDT_ERR_INVALID, "buffer %p is host memory, a device buffer is required", p);
        if (a.device != dev)
            return fail(VDT_ERR_INVALID, "buffer %p lives on device %d, the call runs on device %d", p,
                        a.device, dev);
    }
    return VDT_OK;
}

// launch overlap (programmatic dependent launch): off by default -- on the
// VGG-16 B=256 step it measured 9.83 ms against 9.62 ms without it
std::atomic<int> g_overlap{0};

}  // namespace

extern "C" int vdt_set_launch_overlap(int enable) { return g_overlap.exchange(enable != 0 ? 1 : 0); }

namespace vdt {
bool overlap_enabled() { return g_overlap.load(std::memory_order_relaxed) != 0; }
void api_clear_error() { g_last_error.clear(); }
int api_check_buffers(int dev, std::initializer_list<const void*> ptrs) { return check_device_buffers(dev, ptrs); }
int api_fail(int status, const char* msg) { return fail(status, "%s", msg); }
int api_cuda_fail(cudaError_t e, const char* what) { return cuda_fail(e, what); }
int api_check_cfg(const vdt_time_cfg* c) { return check_cfg(c); }
}  // namespace vdt

namespace {

// Blob reader with bounds checks (the reference's load_weights has none).
struct Reader {
    const unsigned char* p;
    size_t n, off = 0;
    bool i32(int* v) {
        if (off + 4 > n) return false;
        memcpy(v, p + off, 4);
        off += 4;
        return true;
    }
    const float* f32(size_t count) {
        if (count > (n - off) / 4) return nullptr;
        const float* r = reinterpret_cast<const float*>(p + off);
        off += 4 * count;
        return r;
    }
};

}  // namespace

namespace {
// which integrator runs a layer: k_thread for narrow conv layers (a warp per
// pixel would leave most lanes idle), k_dense (bucketing fused in) up to
// dense_max_fan inputs per pixel, else k_sorted, else k_dense if it takes the
// layer, else the generic chunk integrator
int layer_kernel(const vdt_ctx* c, int li, const vdt_time_cfg& cfg) {
    const Layer& ly = c->m->layers[li];
    if (ly.d.out == VDT_OUT_VMEM) return VDT_KERNEL_VMEM;
    if (li < (int)c->kernel_override.size() && c->kernel_override[li] >= 0) return c->kernel_override[li];
    const int fc = ly.d.kind == VDT_FC;
    const int K = fc ? 1 : ly.d.k;
    const int fan = K * K * ly.C_in;
    if (thread_supported(ly.d.k, fc, ly.C_in, ly.C_out, cfg.T, cfg.decay_len) &&
        dense_supported(ly.d.k, fc, ly.C_in, ly.C_out, cfg.T, cfg.decay_len))
        return VDT_KERNEL_THREAD;
    const bool dense_ok = dense_supported(ly.d.k, fc, ly.C_in, ly.C_out, cfg.T, cfg.decay_len);
    if (fan <= c->dense_max_fan && dense_ok) return VDT_KERNEL_DENSE;
    if (sorted_supported(K, fc, kSortedDelta, ly.C_in, ly.C_out, cfg.T, cfg.decay_len)) return VDT_KERNEL_SORTED;
    return dense_ok ? VDT_KERNEL_DENSE : VDT_KERNEL_CHUNK;
}

}  // namespace

// ----------------------------------------------------------------- metadata
extern "C" const char* vdt_version(void) { return "vdttfs-b200 0.1 (sm_100a)"; }

extern "C" const char* vdt_strerror(int s) {
    switch (s) {
        case VDT_OK: return "ok";
        case VDT_ERR_INVALID: return "invalid argument";
        case VDT_ERR_BLOB: return "malformed weight blob";
        case VDT_ERR_CUDA: return "CUDA error";
        case VDT_ERR_OOM: return "out of device memory";
        case VDT_ERR_UNSUPPORTED: return "unsupported configuration";
        case VDT_ERR_CAPACITY: return "batch exceeds context capacity";
        default: return "unknown status";
    }
}

extern "C" const char* vdt_last_error(void) { return g_last_error.c_str(); }

// -------------------------------------------------------------------- model
static int host_luts(const vdt_time_cfg& c, float tci, float tdi, float tcf, float tdf,
                     std::vector<float>& d, std::vector<float>& th) {
    // update_LUTs' host loop (t1:210-213, t2:239-240), libm expf
    d.resize(c.decay_len);
    th.resize(c.T);
    for (int t = 0; t < c.decay_len; ++t) d[t] = expf(-((float)t - tdi) / tci);
    for (int t = 0; t < c.T; ++t) th[t] = c.vth_init * expf(-((float)t - tdf) / tcf);
    return VDT_OK;
}

extern "C" int vdt_model_load_blob(const void* blob, size_t nbytes, const vdt_layer_desc* descs,
                                   int n_layers, const vdt_net_desc* net, const vdt_time_cfg* cfg,
                                   int device, vdt_model** out) {
    g_last_error.clear();
    if (!out) return fail(VDT_ERR_INVALID, "out is NULL");
    *out = nullptr;
    if (!blob || !descs || !net || n_layers <= 0)
        return fail(VDT_ERR_INVALID, "blob/layers/net missing");
    if (int s = check_cfg(cfg)) return s;
    if (net->in_h <= 0 || net->in_w <= 0 || net->in_c <= 0)
        return fail(VDT_ERR_INVALID, "bad input shape");
    if (net->encoder < VDT_ENC_NONE || net->encoder > VDT_ENC_LINEAR)
        return fail(VDT_ERR_INVALID, "encoder=%d", net->encoder);
    if (net->readout < VDT_READ_ARGMIN_FIRST || net->readout > VDT_READ_ARGMAX)
        return fail(VDT_ERR_INVALID, "readout=%d", net->readout);

    Reader r{static_cast<const unsigned char*>(blob), nbytes};
    int L;
    if (!r.i32(&L)) return fail(VDT_ERR_BLOB, "blob shorter than its header");
    if (L != n_layers) return fail(VDT_ERR_BLOB, "blob has %d layers, topology has %d", L, n_layers);

    auto m = new vdt_model();
    m->device = device;
    m->cfg = *cfg;
    m->net = *net;
    std::vector<const float*> hk, hb;
    int h = net->in_h, w = net->in_w, c = net->in_c;
    for (int i = 0; i < L; ++i) {
        Layer ly{};
        ly.d = descs[i];
        int nd;
        if (!r.i32(&nd) || (nd != 2 && nd != 4)) { delete m; return fail(VDT_ERR_BLOB, "layer %d: kernel ndim", i); }
        int shp[4] = {1, 1, 1, 1};
        size_t ksz = 1;
        for (int k = 0; k < nd; ++k) {
            if (!r.i32(&shp[k]) || shp[k] <= 0) { delete m; return fail(VDT_ERR_BLOB, "layer %d: kernel shape", i); }
            ksz *= (size_t)shp[k];
        }
        const float* kp = r.f32(ksz);
        if (!kp) { delete m; return fail(VDT_ERR_BLOB, "layer %d: truncated kernel", i); }
        int nb, bsz, tmp, tcs, tds;
        if (!r.i32(&nb) || !r.i32(&bsz) || bsz <= 0) { delete m; return fail(VDT_ERR_BLOB, "layer %d: bias header", i); }
        const float* bp = r.f32((size_t)bsz);
        if (!bp) { delete m; return fail(VDT_ERR_BLOB, "layer %d: truncated bias", i); }
        const float* tcp; const float* tdp;
        if (!r.i32(&tmp) || !r.i32(&tcs) || tcs < 1 || !(tcp = r.f32((size_t)tcs)))
            { delete m; return fail(VDT_ERR_BLOB, "layer %d: tc_fire", i); }
        if (!r.i32(&tmp) || !r.i32(&tds) || tds < 1 || !(tdp = r.f32((size_t)tds)))
            { delete m; return fail(VDT_ERR_BLOB, "layer %d: td", i); }
        ly.tc_fire = tcp[0];
        ly.td = tdp[0];
        int t_min = (int)ceilf(ly.td);
        ly.t_min = t_min < 0 ? 0 : t_min;
        const bool last = (i == L - 1);
        if (ly.d.out == VDT_OUT_VMEM && !last) { delete m; return fail(VDT_ERR_INVALID, "layer %d: VMEM output only on the last layer", i); }
        if (ly.d.kind == VDT_CONV) {
            if (nd != 4) { delete m; return fail(VDT_ERR_BLOB, "layer %d: conv needs an HWIO kernel", i); }
            if (shp[0] != shp[1] || shp[0] != ly.d.k) { delete m; return fail(VDT_ERR_BLOB, "layer %d: kernel %dx%d, topology k=%d", i, shp[0], shp[1], ly.d.k); }
            if (shp[2] != c) { delete m; return fail(VDT_ERR_BLOB, "layer %d: C_in %d, map has %d", i, shp[2], c); }
            if (ly.d.out == VDT_OUT_VMEM) { delete m; return fail(VDT_ERR_UNSUPPORTED, "layer %d: VMEM readout on a conv", i); }
            ly.H_in = h; ly.W_in = w; ly.C_in = c;
            if (ly.d.pad == VDT_PAD_SAME) { ly.H_out = h; ly.W_out = w; }
            else { ly.H_out = h - ly.d.k + 1; ly.W_out = w - ly.d.k + 1; }
            if (ly.H_out <= 0 || ly.W_out <= 0) { delete m; return fail(VDT_ERR_INVALID, "layer %d: empty output map", i); }
            ly.C_out = shp[3];
        } else if (ly.d.kind == VDT_FC) {
            const int f = h * w * c;
            const int cin = nd == 2 ? shp[0] : shp[0] * shp[1] * shp[2];
            if (cin != f) { delete m; return fail(VDT_ERR_BLOB, "layer %d: FC C_in %d, flattened map %d", i, cin, f); }
            ly.H_in = ly.W_in = 1; ly.C_in = f;
            ly.H_out = ly.W_out = 1; ly.C_out = shp[nd - 1];
            ly.d.k = 1; ly.d.pad = VDT_PAD_VALID;
            if (ly.d.pool_after) { delete m; return fail(VDT_ERR_INVALID, "layer %d: pool after FC", i); }
        } else {
            delete m; return fail(VDT_ERR_INVALID, "layer %d: kind %d", i, ly.d.kind);
        }
        if (bsz != ly.C_out) { delete m; return fail(VDT_ERR_BLOB, "layer %d: bias %d != C_out %d", i, bsz, ly.C_out); }
        if (ly.d.out == VDT_OUT_FIRE &&
            !integrate_supported(ly.d.kind == VDT_CONV ? ly.d.k : 1, ly.d.kind == VDT_FC, cfg->delta,
                                 ly.C_out, cfg->T, cfg->decay_len)) {
            delete m;
            return fail(VDT_ERR_UNSUPPORTED, "layer %d: integrator needs delta in {1,2,4,...,64} and K*K <= 32", i);
        }
        if ((double)ly.d.k * ly.d.k * ly.C_in * ly.C_out >= 2147483647.0) {
            delete m; return fail(VDT_ERR_UNSUPPORTED, "layer %d: kernel above 2^31 elements", i);
        }
        h = ly.H_out; w = ly.W_out; c = ly.C_out;
        if (ly.d.pool_after) {
            h /= 2; w /= 2;
            if (h <= 0 || w <= 0) { delete m; return fail(VDT_ERR_INVALID, "layer %d: pool of a 1-wide map", i); }
        }
        m->layers.push_back(ly);
        hk.push_back(kp);
        hb.push_back(bp);
    }
    if (r.off != r.n) { delete m; return fail(VDT_ERR_BLOB, "blob has %zu trailing bytes", r.n - r.off); }
    // the output is the last map, flattened (an FC layer's [classes]; a conv
    // layer's pooled or unpooled [H, W, C])
    m->n_classes = h * w * c;
    m->in_elems = (size_t)net->in_h * net->in_w * net->in_c;

    DeviceGuard g(device);
    if (!g.ok) { delete m; return fail(VDT_ERR_CUDA, "cannot select device %d", device); }
    // one arena: weights, biases, LUT pairs (each segment 16-byte aligned)
    auto al = [](size_t n) { return (n + 3) & ~size_t(3); };
    size_t total = 0;
    for (auto& ly : m->layers)
        total += al((size_t)ly.d.k * ly.d.k * ly.C_in * ly.C_out) + al(ly.C_out) +
                 al(cfg->decay_len) + al(cfg->T);
    cudaError_t e = cudaMalloc(&m->arena, total * sizeof(float));
    if (e != cudaSuccess) { delete m; return cuda_fail(e, "cudaMalloc(model arena)"); }
    m->weight_bytes = total * sizeof(float);
    float* cur = m->arena;
    std::vector<LutJob> jobs;
    std::vector<float> hd, hth;
    for (size_t i = 0; i < m->layers.size(); ++i) {
        Layer& ly = m->layers[i];
        const size_t kn = (size_t)ly.d.k * ly.d.k * ly.C_in * ly.C_out;
        ly.W = cur; cur += al(kn);
        ly.bias = cur; cur += al(ly.C_out);
        ly.decay = cur; cur += al(cfg->decay_len);
        ly.th = cur; cur += al(cfg->T);
        e = cudaMemcpy(ly.W, hk[i], kn * sizeof(float), cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(ly.bias, hb[i], ly.C_out * sizeof(float), cudaMemcpyHostToDevice);
        const float tci = i ? m->layers[i - 1].tc_fire : net->tc_in;
        const float tdi = i ? m->layers[i - 1].td : net->td_in;
        if (e == cudaSuccess && cfg->lut_source == VDT_LUT_HOST_LIBM) {
            host_luts(*cfg, tci, tdi, ly.tc_fire, ly.td, hd, hth);
            e = cudaMemcpy(ly.decay, hd.data(), hd.size() * sizeof(float), cudaMemcpyHostToDevice);
            if (e == cudaSuccess) e = cudaMemcpy(ly.th, hth.data(), hth.size() * sizeof(float), cudaMemcpyHostToDevice);
        }
        jobs.push_back(LutJob{tci, tdi, ly.tc_fire, ly.td, ly.decay, ly.th});
        if (e != cudaSuccess) { cudaFree(m->arena); delete m; return cuda_fail(e, "weight upload"); }
    }
    if (cfg->lut_source == VDT_LUT_DEVICE) {
        LutJob* dj = nullptr;
        e = cudaMalloc(&dj, jobs.size() * sizeof(LutJob));
        if (e == cudaSuccess) e = cudaMemcpy(dj, jobs.data(), jobs.size() * sizeof(LutJob), cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = launch_build_luts(dj, (int)jobs.size(), cfg->T, cfg->decay_len, cfg->vth_init, 0);
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (dj) cudaFree(dj);
        if (e != cudaSuccess) { cudaFree(m->arena); delete m; return cuda_fail(e, "LUT build"); }
    }
    *out = m;
    return VDT_OK;
}

extern "C" void vdt_model_destroy(vdt_model* m) {
    if (!m) return;
    DeviceGuard g(m->device);
    cudaFree(m->arena);
    delete m;
}

extern "C" int vdt_model_info(const vdt_model* m, int* n_layers, int* n_classes, size_t* wbytes) {
    if (!m) return fail(VDT_ERR_INVALID, "model is NULL");
    if (n_layers) *n_layers = model_stages(m);
    if (n_classes) *n_classes = m->n_classes;
    if (wbytes) *wbytes = m->weight_bytes;
    return VDT_OK;
}

extern "C" int vdt_model_luts(const vdt_model* m, int layer, float* h_decay, float* h_th) {
    if (m && m->is_dvs) return fail(VDT_ERR_UNSUPPORTED, "a task-3 network has no LUTs");
    if (!m || layer < 0 || layer >= (int)m->layers.size()) return fail(VDT_ERR_INVALID, "bad layer");
    DeviceGuard g(m->device);
    const Layer& ly = m->layers[layer];
    if (h_decay) VDT_CUDA(cudaMemcpy(h_decay, ly.decay, m->cfg.decay_len * sizeof(float), cudaMemcpyDeviceToHost));
    if (h_th) VDT_CUDA(cudaMemcpy(h_th, ly.th, m->cfg.T * sizeof(float), cudaMemcpyDeviceToHost));
    return VDT_OK;
}

// ---------------------------------------------------------------------- ctx
namespace {

struct Sizes {
    size_t act = 0, off = 0, bkt = 0;
};

Sizes ctx_sizes(const vdt_model* m, long long B) {
    Sizes s;
    const int dmin = std::min(m->cfg.delta, kSortedDelta);
    const int OS = (m->cfg.T + dmin - 1) / dmin + 1;
    if (m->is_dvs) {
        const DvsSizes d = dvs_sizes(m, B);
        s.act = d.act; s.off = d.off; s.bkt = d.bkt;
        return s;
    }
    s.act = (size_t)B * m->in_elems;
    for (auto& ly : m->layers) {
        const size_t in = (size_t)B * ly.H_in * ly.W_in * ly.C_in;
        const size_t out = (size_t)B * ly.H_out * ly.W_out * ly.C_out;
        s.act = std::max(s.act, std::max(in, out));
        if (ly.d.out == VDT_OUT_FIRE) {
            const size_t cols = ly.d.kind == VDT_FC ? (size_t)B : (size_t)B * ly.H_in * ly.W_in;
            s.off = std::max(s.off, cols * OS);
            s.bkt = std::max(s.bkt, in);
        }
    }
    return s;
}

void ctx_free(vdt_ctx* c) {
    for (auto& mk : c->marks) { cudaEventDestroy(mk.a); cudaEventDestroy(mk.b); }
    for (auto e : c->spare_events) cudaEventDestroy(e);
    c->marks.clear();
    c->spare_events.clear();
    for (auto& kv : c->cache) cudaGraphExecDestroy(kv.second);
    c->cache.clear();
    for (auto& a : c->act) cudaFree(a);
    cudaFree(c->in_slot); cudaFree(c->out_slot); cudaFree(c->pred_slot);
    cudaFree(c->in_slot2); cudaFree(c->out_slot2); cudaFree(c->pred_slot2);
    for (int i = 0; i < 2; ++i) {
        if (c->ev_h2d[i]) cudaEventDestroy(c->ev_h2d[i]);
        if (c->ev_done[i]) cudaEventDestroy(c->ev_done[i]);
    }
    for (auto e : c->ev_part)
        if (e) cudaEventDestroy(e);
    if (c->copy_stream) cudaStreamDestroy(c->copy_stream);
    for (auto& w : c->sub) {
        for (auto& a : w.act) cudaFree(a);
        cudaFree(w.off); cudaFree(w.cin); cudaFree(w.tin);
        if (w.join) cudaEventDestroy(w.join);
        if (w.stream) cudaStreamDestroy(w.stream);
    }
    c->sub.clear();
    if (c->ev_fork) cudaEventDestroy(c->ev_fork);
    cudaFree(c->off); cudaFree(c->cin); cudaFree(c->tin); cudaFree(c->scratch); cudaFree(c->counters);
}

// Enqueue one batch: the reference's per-batch layer sequence.
int enqueue(vdt_ctx* c, const float* d_input, int pixels, int B, float* d_out, int32_t* d_pred,
            float* const* trace) {
    const vdt_model* m = c->m;
    if (m->is_dvs) return dvs_enqueue(c, d_input, B, d_out, d_pred, trace);
    const vdt_time_cfg& cfg = m->cfg;
    cudaStream_t s = c->stream;
    const float* x = d_input;
    int ai = 0;
    // pixels: a first layer on k_dense encodes them as it reads its windows
    // (unless counting, whose bucket pass needs the spike times); otherwise
    // one encode pass writes the spike times first
    const bool encode_fused = pixels && m->net.encoder != VDT_ENC_NONE && !c->counting &&
                              layer_kernel(c, 0, cfg) == VDT_KERNEL_DENSE;
    if (pixels && m->net.encoder != VDT_ENC_NONE && !encode_fused) {
        const long long n = (long long)B * m->net.in_h * m->net.in_w * m->net.in_c;
        VDT_CUDA(launch_encode(d_input, c->act[0], n, m->net.encoder, m->net.tc_in, m->net.td_in,
                               cfg.T, cfg.inf_time, s));
        x = c->act[0];
        ai = 1;
    }
    bool readout_done = false;                               // the readout ran fused into the last layer
    const int L = (int)m->layers.size();
    for (int i = 0; i < L; ++i) {
        const Layer& ly = m->layers[i];
        // layer i counts into counters[2i] (events) and [2i + 1] (fetched synapses)
        unsigned long long* ev = c->counting ? c->counters + 2 * i : nullptr;
        unsigned long long* fe = c->counting ? c->counters + 2 * i + 1 : nullptr;
        const bool last = i == L - 1;
        float* y = (last && !ly.d.pool_after) ? d_out : c->act[ai];
        if (trace && trace[i] && !last) y = trace[i];
        if (trace && trace[i] && last && ly.d.pool_after) y = trace[i];
        bool pooled = false;                                 // the layer's pool ran fused into it
        if (ly.d.out == VDT_OUT_VMEM) {
            // the membrane readout (last layer only) with the argmax fused in
            int32_t* fused_pred = last ? d_pred : nullptr;
            StageTimer st(c, i, 1);
            VDT_CUDA(launch_layer_vmem(x, ly.W, ly.bias, ly.decay, B, ly.C_in, ly.C_out, cfg.T,
                                       cfg.fire_start, cfg.inf_time, y, s, fused_pred, m->net.readout));
            readout_done = fused_pred != nullptr;
        } else {
            const bool fc = ly.d.kind == VDT_FC;
            // small fan-in: the integrator reads the spike map itself (no
            // bucket pass); otherwise bucketize, then integrate
            IntegParams ip{};
            ip.off = c->off; ip.cin = c->cin; ip.tin = c->tin;
            ip.W = ly.W; ip.bias = ly.bias; ip.lut_decay = ly.decay; ip.lut_th = ly.th;
            ip.out = y;
            ip.B = B; ip.H_in = ly.H_in; ip.W_in = ly.W_in; ip.C_in = ly.C_in;
            ip.H_out = ly.H_out; ip.W_out = ly.W_out; ip.C_out = ly.C_out;
            ip.K = ly.d.k;
            ip.pad = (!fc && ly.d.pad == VDT_PAD_SAME) ? ly.d.k / 2 : 0;
            ip.is_fc = fc;
            const int kern = layer_kernel(c, i, cfg);
            // k_sorted buckets at its own chunk width (results do not depend
            // on it); the counting pass keeps the configured width, which
            // defines the reference's fetched-synapse accounting
            const int kd = (kern == VDT_KERNEL_SORTED && !ev) ? kSortedDelta : cfg.delta;
            const int knc = (cfg.T + kd - 1) / kd;
            ip.T = cfg.T; ip.delta = kd; ip.NC = knc; ip.t_min = ly.t_min;
            ip.lut_mode = cfg.lut_mode; ip.decay_len = cfg.decay_len;
            ip.tfs = cfg.fire_start; ip.inf_time = cfg.inf_time;
            ip.fetched = fe;
            if (i == 0 && encode_fused) {
                ip.encoder = m->net.encoder; ip.enc_tc = m->net.tc_in; ip.enc_td = m->net.td_in;
            }
            const bool dense = kern == VDT_KERNEL_DENSE || kern == VDT_KERNEL_THREAD;
            if (!dense || ev) {
                // the dense path needs no buckets; they are still built when
                // counting, for the event counter
                BktParams bp{};
                bp.in = x;
                bp.n_cols = fc ? B : (long long)B * ly.H_in * ly.W_in;
                bp.c_in = ly.C_in;
                bp.layout = VDT_LAYOUT_NHWC;
                bp.hw = 1;
                bp.T = cfg.T;
                bp.delta = kd;
                bp.NC = knc;
                bp.tfs = cfg.fire_start;
                bp.tb_mode = VDT_TB_FLOOR_STAGGER;
                bp.inf_time = cfg.inf_time;
                bp.off = c->off; bp.cin = c->cin; bp.tin = c->tin;
                bp.events = ev;
                StageTimer st(c, i, 0);
                VDT_CUDA(launch_bucketize(bp, s));
            }
            // k_dense and k_sorted write the pooled map themselves when nobody
            // asks for the layer's own map (not traced): an integer min of
            // each output into its cell, the cells pre-filled with 0x7F bytes
            // (the times' bits order like their values only when the no-spike
            // time is positive, as it is in every reference configuration)
            if (ly.d.pool_after && !(trace && trace[i]) && ly.H_out >= 2 && ly.W_out >= 2 && cfg.inf_time > 0.0f &&
                (kern == VDT_KERNEL_DENSE || kern == VDT_KERNEL_SORTED)) {
                float* z = last ? d_out : y;
                StageTimer sp(c, i, 2);
                VDT_CUDA(cudaMemsetAsync(z, 0x7F, (size_t)B * (ly.H_out / 2) * (ly.W_out / 2) * ly.C_out * sizeof(float),
                                         s));
                ip.pool_out = z;
                pooled = true;
            }
            StageTimer st(c, i, 1);
            if (kern == VDT_KERNEL_THREAD && !fe) {
                // k_thread writes the pooled map itself when nobody asks for
                // the layer's own map (not traced)
                if (ly.d.pool_after && !(trace && trace[i]) && ly.H_out >= 2 && ly.W_out >= 2) {
                    if (last) ip.out = d_out;
                    VDT_CUDA(launch_thread_pooled(ip, x, s));
                    pooled = true;
                } else {
                    VDT_CUDA(launch_thread(ip, x, s));
                }
            } else if (dense) VDT_CUDA(launch_dense(ip, x, s));
            else if (kern == VDT_KERNEL_SORTED) VDT_CUDA(launch_sorted(ip, s));
            else VDT_CUDA(launch_integrate(ip, s));
        }
        if (pooled) {                                        // y (or d_out) holds the pooled map
            x = last ? d_out : y;
            if (!last && y == c->act[ai]) ai = (ai + 1) % 3;
            continue;
        }
        if (trace && trace[i] && y != trace[i])
            VDT_CUDA(cudaMemcpyAsync(trace[i], y, (size_t)B * ly.H_out * ly.W_out * ly.C_out * sizeof(float),
                                     cudaMemcpyDeviceToDevice, s));
        x = y;
        if (y == c->act[ai]) ai = (ai + 1) % 3;
        if (ly.d.pool_after) {
            float* z = last ? d_out : c->act[ai];
            StageTimer st(c, i, 2);
            VDT_CUDA(launch_pool_min(x, z, B, ly.H_out, ly.W_out, ly.C_out, cfg.inf_time, s));
            x = z;
            if (z == c->act[ai]) ai = (ai + 1) % 3;
        }
    }
    if (d_pred && !readout_done)
        VDT_CUDA(launch_readout(x, B, m->n_classes, m->net.readout, cfg.inf_time, d_pred, s));
    if (c->profiling) c->prof_batches++;
    return VDT_OK;
}

// One batch, split into n_sub parts on n_sub streams when sub-batches are
// on (part 0 on the ctx stream, part k on sub[k - 1]'s stream with its
// workspace; each part is an independent run of the same per-batch body, so
// the results are those of one run).  Counting and profiling passes run
// whole.
int enqueue_split(vdt_ctx* c, const float* d_input, int pixels, int B, float* d_out, int32_t* d_pred) {
    const int n = std::min(c->n_sub, B);
    if (n < 2 || c->counting || c->profiling) return enqueue(c, d_input, pixels, B, d_out, d_pred, nullptr);
    const vdt_model* m = c->m;
    const size_t in_row = m->in_elems;
    cudaStream_t s = c->stream;
    VDT_CUDA(cudaEventRecord(c->ev_fork, s));
    auto swap_ws = [c](vdt_ctx::SubWs& w) {
        std::swap(c->stream, w.stream);
        for (int i = 0; i < 3; ++i) std::swap(c->act[i], w.act[i]);
        std::swap(c->off, w.off);
        std::swap(c->cin, w.cin);
        std::swap(c->tin, w.tin);
    };
    int b0 = 0;
    for (int k = 0; k < n; ++k) {
        const int bk = B / n + (k < B % n ? 1 : 0);
        const float* in = d_input + (size_t)b0 * in_row;
        float* out = d_out + (size_t)b0 * m->n_classes;
        int32_t* pred = d_pred ? d_pred + b0 : nullptr;
        if (k == 0) {
            if (int st = enqueue(c, in, pixels, bk, out, pred, nullptr)) return st;
        } else {
            vdt_ctx::SubWs& w = c->sub[k - 1];
            VDT_CUDA(cudaStreamWaitEvent(w.stream, c->ev_fork, 0));
            swap_ws(w);
            const int st = enqueue(c, in, pixels, bk, out, pred, nullptr);
            swap_ws(w);
            if (st) return st;
            VDT_CUDA(cudaEventRecord(w.join, w.stream));
            VDT_CUDA(cudaStreamWaitEvent(s, w.join, 0));
        }
        b0 += bk;
    }
    return VDT_OK;
}

}  // namespace

extern "C" int vdt_ctx_set_sub_batches(vdt_ctx* c, int n) {
    g_last_error.clear();
    if (!c) return fail(VDT_ERR_INVALID, "ctx is NULL");
    if (n < 1 || n > VDT_MAX_SUB_BATCHES) return fail(VDT_ERR_INVALID, "n=%d (1 to %d)", n, VDT_MAX_SUB_BATCHES);
    if (c->m->is_dvs && n != 1) return fail(VDT_ERR_UNSUPPORTED, "a task-3 network runs whole batches");
    DeviceGuard g(c->m->device);
    if (!c->ev_fork) VDT_CUDA(cudaEventCreateWithFlags(&c->ev_fork, cudaEventDisableTiming));
    const Sizes z = ctx_sizes(c->m, (c->max_batch + n - 1) / n);
    while ((int)c->sub.size() < n - 1) {                     // workspaces made once, kept
        vdt_ctx::SubWs w;
        cudaError_t e = cudaSuccess;
        for (auto& a : w.act) if (e == cudaSuccess) e = cudaMalloc(&a, z.act * sizeof(float));
        if (e == cudaSuccess) e = cudaMalloc(&w.off, std::max<size_t>(z.off, 1) * sizeof(int));
        if (e == cudaSuccess) e = cudaMalloc(&w.cin, std::max<size_t>(z.bkt, 1) * sizeof(int));
        if (e == cudaSuccess) e = cudaMalloc(&w.tin, std::max<size_t>(z.bkt, 1) * sizeof(float));
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&w.join, cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&w.stream, cudaStreamNonBlocking);
        c->sub.push_back(w);                                 // freed with the ctx, even on failure
        if (e != cudaSuccess) return cuda_fail(e, "sub-batch workspace");
    }
    if (c->n_sub != n) {
        VDT_CUDA(cudaStreamSynchronize(c->stream));
        for (auto& kv : c->cache) cudaGraphExecDestroy(kv.second);   // captured with the old split
        c->cache.clear();
        c->n_sub = n;
    }
    return VDT_OK;
}

extern "C" int vdt_ctx_create(const vdt_model* m, int max_batch, vdt_stream stream, vdt_ctx** out) {
    g_last_error.clear();
    if (!out) return fail(VDT_ERR_INVALID, "out is NULL");
    *out = nullptr;
    if (!m || max_batch <= 0) return fail(VDT_ERR_INVALID, "model NULL or max_batch <= 0");
    DeviceGuard g(m->device);
    auto c = new vdt_ctx();
    c->m = m;
    c->device = m->device;
    c->max_batch = max_batch;
    c->stream = static_cast<cudaStream_t>(stream);
    const Sizes z = ctx_sizes(m, max_batch);
    const size_t in_n = (size_t)max_batch * m->in_elems;
    cudaError_t e = cudaSuccess;
    for (auto& a : c->act) if (e == cudaSuccess) e = cudaMalloc(&a, z.act * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&c->in_slot, in_n * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&c->out_slot, (size_t)max_batch * m->n_classes * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&c->pred_slot, (size_t)max_batch * sizeof(int32_t));
    if (e == cudaSuccess) e = cudaMalloc(&c->off, std::max<size_t>(z.off, 1) * sizeof(int));
    if (e == cudaSuccess) e = cudaMalloc(&c->cin, std::max<size_t>(z.bkt, 1) * sizeof(int));
    if (e == cudaSuccess) e = cudaMalloc(&c->tin, std::max<size_t>(z.bkt, 1) * sizeof(float));
    if (e == cudaSuccess && m->is_dvs) {
        c->scratch_bytes = dvs_sizes(m, max_batch).scratch_bytes;
        if (c->scratch_bytes) e = cudaMalloc(&c->scratch, c->scratch_bytes);
    }
    const size_t n_counters = 2 * std::max<size_t>(1, m->layers.size());
    if (e == cudaSuccess) e = cudaMalloc(&c->counters, n_counters * sizeof(unsigned long long));
    if (e == cudaSuccess) e = cudaMemset(c->counters, 0, n_counters * sizeof(unsigned long long));
    if (e != cudaSuccess) {
        ctx_free(c);
        delete c;
        return cuda_fail(e, "ctx workspace allocation");
    }
    *out = c;
    return VDT_OK;
}

extern "C" void vdt_ctx_destroy(vdt_ctx* c) {
    if (!c) return;
    DeviceGuard g(c->device);
    if (c->stream) cudaStreamSynchronize(c->stream); else cudaDeviceSynchronize();
    ctx_free(c);
    delete c;
}

extern "C" int vdt_ctx_set_graphs(vdt_ctx* c, int enable) {
    if (!c) return fail(VDT_ERR_INVALID, "ctx is NULL");
    c->graphs = enable != 0;
    return VDT_OK;
}

extern "C" int vdt_ctx_set_counting(vdt_ctx* c, int enable) {
    if (!c) return fail(VDT_ERR_INVALID, "ctx is NULL");
    c->counting = enable != 0;
    return VDT_OK;
}

// Per-layer counts since the last read, then zeroed.
static int read_counters(vdt_ctx* c, std::vector<unsigned long long>& h) {
    DeviceGuard g(c->m->device);
    h.assign(2 * std::max<size_t>(1, c->m->layers.size()), 0ull);
    VDT_CUDA(cudaStreamSynchronize(c->stream));
    VDT_CUDA(cudaMemcpy(h.data(), c->counters, h.size() * sizeof(unsigned long long), cudaMemcpyDeviceToHost));
    VDT_CUDA(cudaMemset(c->counters, 0, h.size() * sizeof(unsigned long long)));
    return VDT_OK;
}

extern "C" int vdt_ctx_counters(vdt_ctx* c, unsigned long long* events, unsigned long long* fetched) {
    g_last_error.clear();
    if (!c) return fail(VDT_ERR_INVALID, "ctx is NULL");
    std::vector<unsigned long long> h;
    if (int s = read_counters(c, h)) return s;
    unsigned long long ev = 0, fe = 0;
    for (size_t i = 0; i + 1 < h.size(); i += 2) { ev += h[i]; fe += h[i + 1]; }
    if (events) *events = ev;
    if (fetched) *fetched = fe;
    return VDT_OK;
}

extern "C" int vdt_ctx_layer_counters(vdt_ctx* c, int n_layers, unsigned long long* events,
                                      unsigned long long* fetched) {
    g_last_error.clear();
    if (!c) return fail(VDT_ERR_INVALID, "ctx is NULL");
    if (c->m->is_dvs) return fail(VDT_ERR_UNSUPPORTED, "a task-3 network has no event counters");
    if (n_layers != (int)c->m->layers.size()) return fail(VDT_ERR_INVALID, "n_layers mismatch");
    std::vector<unsigned long long> h;
    if (int s = read_counters(c, h)) return s;
    for (int i = 0; i < n_layers; ++i) {
        if (events) events[i] = h[2 * i];
        if (fetched) fetched[i] = h[2 * i + 1];
    }
    return VDT_OK;
}

extern "C" int vdt_ctx_set_profiling(vdt_ctx* c, int enable) {
    if (!c) return fail(VDT_ERR_INVALID, "ctx is NULL");
    c->profiling = enable != 0;
    return VDT_OK;
}

extern "C" int vdt_ctx_layer_times(vdt_ctx* c, int n_layers, float* bkt_ms, float* int_ms,
                                   float* pool_ms, int* batches) {
    if (!c) return fail(VDT_ERR_INVALID, "ctx is NULL");
    if (n_layers != model_stages(c->m)) return fail(VDT_ERR_INVALID, "n_layers mismatch");
    DeviceGuard g(c->m->device);
    VDT_CUDA(cudaStreamSynchronize(c->stream));
    float* dst[3] = {bkt_ms, int_ms, pool_ms};
    for (auto* d : dst) if (d) for (int i = 0; i < n_layers; ++i) d[i] = 0.0f;
    for (auto& mk : c->marks) {
        float ms = 0.0f;
        VDT_CUDA(cudaEventElapsedTime(&ms, mk.a, mk.b));
        if (dst[mk.stage]) dst[mk.stage][mk.layer] += ms;
        c->spare_events.push_back(mk.a);
        c->spare_events.push_back(mk.b);
    }
    c->marks.clear();
    if (batches) *batches = c->prof_batches;
    c->prof_batches = 0;
    return VDT_OK;
}

extern "C" int vdt_ctx_layer_kernels(const vdt_ctx* c, int n_layers, int* kernels) {
    g_last_error.clear();
    if (!c || !kernels) return fail(VDT_ERR_INVALID, "ctx or kernels is NULL");
    if (c->m->is_dvs) return fail(VDT_ERR_UNSUPPORTED, "a task-3 network has no per-layer integrator choice");
    if (n_layers != (int)c->m->layers.size()) return fail(VDT_ERR_INVALID, "n_layers mismatch");
    for (int i = 0; i < n_layers; ++i) kernels[i] = layer_kernel(c, i, c->m->cfg);
    return VDT_OK;
}

extern "C" int vdt_ctx_set_layer_kernel(vdt_ctx* c, int layer, int kernel) {
    g_last_error.clear();
    if (!c) return fail(VDT_ERR_INVALID, "ctx is NULL");
    if (c->m->is_dvs) return fail(VDT_ERR_UNSUPPORTED, "a task-3 network has no per-layer integrator choice");
    if (layer < 0 || layer >= (int)c->m->layers.size()) return fail(VDT_ERR_INVALID, "layer=%d", layer);
    const Layer& ly = c->m->layers[layer];
    const vdt_time_cfg& cfg = c->m->cfg;
    const int fc = ly.d.kind == VDT_FC;
    const int K = fc ? 1 : ly.d.k;
    bool ok = false;
    switch (kernel) {
        case -1: ok = true; break;
        case VDT_KERNEL_CHUNK: ok = ly.d.out != VDT_OUT_VMEM && integrate_supported(K, fc, cfg.delta, ly.C_out, cfg.T, cfg.decay_len); break;
        case VDT_KERNEL_SORTED: ok = ly.d.out != VDT_OUT_VMEM && sorted_supported(K, fc, kSortedDelta, ly.C_in, ly.C_out, cfg.T, cfg.decay_len); break;
        case VDT_KERNEL_DENSE: ok = ly.d.out != VDT_OUT_VMEM && dense_supported(K, fc, ly.C_in, ly.C_out, cfg.T, cfg.decay_len); break;
        case VDT_KERNEL_VMEM: ok = ly.d.out == VDT_OUT_VMEM; break;
        case VDT_KERNEL_THREAD:   // counting passes run the layer through k_dense
            ok = ly.d.out != VDT_OUT_VMEM && thread_supported(K, fc, ly.C_in, ly.C_out, cfg.T, cfg.decay_len) &&
                 dense_supported(K, fc, ly.C_in, ly.C_out, cfg.T, cfg.decay_len);
            break;
        default: return fail(VDT_ERR_INVALID, "kernel=%d", kernel);
    }
    if (!ok) return fail(VDT_ERR_UNSUPPORTED, "kernel %d cannot run layer %d", kernel, layer);
    if (c->kernel_override.size() != c->m->layers.size()) c->kernel_override.assign(c->m->layers.size(), -1);
    if (c->kernel_override[layer] != kernel) {
        DeviceGuard g(c->m->device);
        VDT_CUDA(cudaStreamSynchronize(c->stream));
        for (auto& kv : c->cache) cudaGraphExecDestroy(kv.second);   // captured with the old choice
        c->cache.clear();
        c->kernel_override[layer] = kernel;
    }
    return VDT_OK;
}

// Run one batch from the ctx's input slot `slot` (0: in_slot, 1: in_slot2)
// into the matching output slots, through a cached CUDA graph when enabled.
// The executable graph cached under key, captured on first use from what
// enqueue_fn() enqueues on c->stream (pointed at a private capture stream
// meanwhile: the legacy default stream can't be captured).
template <class F>
static int cached_graph(vdt_ctx* c, const GraphKey& key, F&& enqueue_fn, cudaGraphExec_t* ex) {
    auto it = c->cache.find(key);
    if (it == c->cache.end()) {
        cudaStream_t cap;
        VDT_CUDA(cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking));
        cudaStream_t user = c->stream;
        c->stream = cap;
        cudaGraph_t graph = nullptr;
        cudaError_t e = cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal);
        int st = VDT_OK;
        if (e == cudaSuccess) st = enqueue_fn();
        cudaError_t e2 = cudaStreamEndCapture(cap, &graph);
        c->stream = user;
        cudaStreamDestroy(cap);
        if (e != cudaSuccess) return cuda_fail(e, "cudaStreamBeginCapture");
        if (st != VDT_OK) { if (graph) cudaGraphDestroy(graph); return st; }
        if (e2 != cudaSuccess) return cuda_fail(e2, "cudaStreamEndCapture");
        cudaGraphExec_t x;
        e = cudaGraphInstantiate(&x, graph, 0);
        cudaGraphDestroy(graph);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGraphInstantiate");
        it = c->cache.emplace(key, x).first;
    }
    *ex = it->second;
    return VDT_OK;
}

static int run_slots(vdt_ctx* c, int pixels, int batch, int slot = 0) {
    float* in = slot ? c->in_slot2 : c->in_slot;
    float* out = slot ? c->out_slot2 : c->out_slot;
    int32_t* pred = slot ? c->pred_slot2 : c->pred_slot;
    if (!c->graphs || c->profiling) return enqueue_split(c, in, pixels, batch, out, pred);
    cudaGraphExec_t ex = nullptr;
    const GraphKey key{batch, pixels, c->counting ? 1 : 0, slot, 0};
    if (int st = cached_graph(c, key, [&] { return enqueue_split(c, in, pixels, batch, out, pred); }, &ex))
        return st;
    VDT_CUDA(cudaGraphLaunch(ex, c->stream));
    return VDT_OK;
}

static int ensure_copy_stream(vdt_ctx* c) {
    if (c->copy_stream) return VDT_OK;
    cudaStream_t cs = nullptr;
    VDT_CUDA(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking));
    c->copy_stream = cs;
    return VDT_OK;
}

// One batch from host memory as its sub-batches, each overlapping the
// others' copies: part k's input crosses on the copy stream (the parts in
// order), its graph (part k alone, on its workspace) runs on its own stream
// once that input has landed, and its outputs cross back on the same stream.
// Part 0 computes while part 1's input is still crossing.  Same kernels and
// results as the whole-batch graph.
static int infer_host_parts(vdt_ctx* c, const float* h_input, int pixels, int batch, float* h_out,
                            int32_t* h_pred) {
    const vdt_model* m = c->m;
    const int n = std::min(c->n_sub, batch);
    if (int st = ensure_copy_stream(c)) return st;
    for (int k = 0; k < n; ++k)
        if (!c->ev_part[k]) VDT_CUDA(cudaEventCreateWithFlags(&c->ev_part[k], cudaEventDisableTiming));
    const size_t in_row = m->in_elems;
    cudaStream_t cs = c->copy_stream;
    // the inputs may land once earlier work on the ctx stream is done with the slot
    VDT_CUDA(cudaEventRecord(c->ev_fork, c->stream));
    VDT_CUDA(cudaStreamWaitEvent(cs, c->ev_fork, 0));
    int b0 = 0;
    for (int k = 0; k < n; ++k) {
        const int bk = batch / n + (k < batch % n ? 1 : 0);
        VDT_CUDA(cudaMemcpyAsync(c->in_slot + (size_t)b0 * in_row, h_input + (size_t)b0 * in_row,
                                 (size_t)bk * in_row * sizeof(float), cudaMemcpyHostToDevice, cs));
        VDT_CUDA(cudaEventRecord(c->ev_part[k], cs));
        b0 += bk;
    }
    b0 = 0;
    for (int k = 0; k < n; ++k) {
        const int bk = batch / n + (k < batch % n ? 1 : 0);
        const float* in = c->in_slot + (size_t)b0 * in_row;
        float* out = c->out_slot + (size_t)b0 * m->n_classes;
        int32_t* pred = c->pred_slot + b0;
        cudaStream_t sk = k == 0 ? c->stream : c->sub[k - 1].stream;
        cudaGraphExec_t ex = nullptr;
        const GraphKey key{bk, pixels, 0, 0, k + 1};
        auto part = [&] {
            if (k == 0) return enqueue(c, in, pixels, bk, out, pred, nullptr);
            vdt_ctx::SubWs& w = c->sub[k - 1];                // this part's workspace
            auto swap_ws = [&] {
                for (int i = 0; i < 3; ++i) std::swap(c->act[i], w.act[i]);
                std::swap(c->off, w.off);
                std::swap(c->cin, w.cin);
                std::swap(c->tin, w.tin);
            };
            swap_ws();
            const int st = enqueue(c, in, pixels, bk, out, pred, nullptr);
            swap_ws();
            return st;
        };
        if (int st = cached_graph(c, key, part, &ex)) return st;
        VDT_CUDA(cudaStreamWaitEvent(sk, c->ev_part[k], 0));
        VDT_CUDA(cudaGraphLaunch(ex, sk));
        if (h_out)
            VDT_CUDA(cudaMemcpyAsync(h_out + (size_t)b0 * m->n_classes, out, (size_t)bk * m->n_classes * sizeof(float),
                                     cudaMemcpyDeviceToHost, sk));
        if (h_pred)
            VDT_CUDA(cudaMemcpyAsync(h_pred + b0, pred, (size_t)bk * sizeof(int32_t), cudaMemcpyDeviceToHost, sk));
        if (k > 0) {
            VDT_CUDA(cudaEventRecord(c->sub[k - 1].join, sk));
            VDT_CUDA(cudaStreamWaitEvent(c->stream, c->sub[k - 1].join, 0));
        }
        b0 += bk;
    }
    VDT_CUDA(cudaStreamSynchronize(c->stream));
    return VDT_OK;
}

static int check_batch(vdt_ctx* c, int batch) {
    if (!c) return fail(VDT_ERR_INVALID, "ctx is NULL");
    if (batch <= 0) return fail(VDT_ERR_INVALID, "batch=%d", batch);
    if (batch > c->max_batch) return fail(VDT_ERR_CAPACITY, "batch %d > max_batch %d", batch, c->max_batch);
    return VDT_OK;
}

extern "C" int vdt_infer(vdt_ctx* c, const float* d_input, int input_is_pixels, int batch,
                         float* d_out, int32_t* d_pred) {
    g_last_error.clear();
    if (int s = check_batch(c, batch)) return s;
    if (!d_input || !d_out) return fail(VDT_ERR_INVALID, "d_input/d_out is NULL");
    if (int s = check_device_buffers(c->m->device, {d_input, d_out, d_pred})) return s;
    DeviceGuard g(c->m->device);
    const vdt_model* m = c->m;
    const size_t in_n = (size_t)batch * m->in_elems;
    if (!c->graphs || c->profiling) return enqueue_split(c, d_input, input_is_pixels, batch, d_out, d_pred);
    VDT_CUDA(cudaMemcpyAsync(c->in_slot, d_input, in_n * sizeof(float), cudaMemcpyDeviceToDevice, c->stream));
    if (int s = run_slots(c, input_is_pixels, batch)) return s;
    VDT_CUDA(cudaMemcpyAsync(d_out, c->out_slot, (size_t)batch * m->n_classes * sizeof(float),
                             cudaMemcpyDeviceToDevice, c->stream));
    if (d_pred)
        VDT_CUDA(cudaMemcpyAsync(d_pred, c->pred_slot, (size_t)batch * sizeof(int32_t),
                                 cudaMemcpyDeviceToDevice, c->stream));
    return VDT_OK;
}

extern "C" int vdt_infer_host(vdt_ctx* c, const float* h_input, int input_is_pixels, int batch,
                              float* h_out, int32_t* h_pred) {
    g_last_error.clear();
    if (int s = check_batch(c, batch)) return s;
    if (!h_input) return fail(VDT_ERR_INVALID, "h_input is NULL");
    DeviceGuard g(c->m->device);
    const vdt_model* m = c->m;
    if (c->graphs && !c->profiling && !c->counting && std::min(c->n_sub, batch) >= 2)
        return infer_host_parts(c, h_input, input_is_pixels, batch, h_out, h_pred);
    const size_t in_n = (size_t)batch * m->in_elems;
    VDT_CUDA(cudaMemcpyAsync(c->in_slot, h_input, in_n * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    if (c->graphs) {
        if (int s = run_slots(c, input_is_pixels, batch)) return s;
    } else {
        if (int s = enqueue_split(c, c->in_slot, input_is_pixels, batch, c->out_slot, c->pred_slot)) return s;
    }
    if (h_out)
        VDT_CUDA(cudaMemcpyAsync(h_out, c->out_slot, (size_t)batch * m->n_classes * sizeof(float),
                                 cudaMemcpyDeviceToHost, c->stream));
    if (h_pred)
        VDT_CUDA(cudaMemcpyAsync(h_pred, c->pred_slot, (size_t)batch * sizeof(int32_t),
                                 cudaMemcpyDeviceToHost, c->stream));
    VDT_CUDA(cudaStreamSynchronize(c->stream));
    return VDT_OK;
}

// Resources of the pipelined host path, made once per ctx (each only if
// missing, so a call after a failed one retries without leaking).
static int ensure_pipeline(vdt_ctx* c) {
    const vdt_model* m = c->m;
    const size_t in_n = (size_t)c->max_batch * m->in_elems;
    cudaError_t e = cudaSuccess;
    if (!c->in_slot2) e = cudaMalloc(&c->in_slot2, in_n * sizeof(float));
    if (e == cudaSuccess && !c->out_slot2)
        e = cudaMalloc(&c->out_slot2, (size_t)c->max_batch * m->n_classes * sizeof(float));
    if (e == cudaSuccess && !c->pred_slot2) e = cudaMalloc(&c->pred_slot2, (size_t)c->max_batch * sizeof(int32_t));
    for (int i = 0; i < 2 && e == cudaSuccess; ++i) {
        if (!c->ev_h2d[i]) e = cudaEventCreateWithFlags(&c->ev_h2d[i], cudaEventDisableTiming);
        if (e == cudaSuccess && !c->ev_done[i]) e = cudaEventCreateWithFlags(&c->ev_done[i], cudaEventDisableTiming);
    }
    if (e != cudaSuccess) return cuda_fail(e, "pipelined host path resources");
    return ensure_copy_stream(c);
}

extern "C" int vdt_infer_host_batches(vdt_ctx* c, int n_batches, const float* const* h_inputs,
                                      int input_is_pixels, int batch, float* const* h_outs,
                                      int32_t* const* h_preds) {
    g_last_error.clear();
    if (int s = check_batch(c, batch)) return s;
    if (n_batches < 0 || (n_batches > 0 && !h_inputs)) return fail(VDT_ERR_INVALID, "n_batches / h_inputs");
    for (int i = 0; i < n_batches; ++i)
        if (!h_inputs[i]) return fail(VDT_ERR_INVALID, "h_inputs[%d] is NULL", i);
    if (n_batches == 0) return VDT_OK;
    DeviceGuard g(c->m->device);
    if (int s = ensure_pipeline(c)) return s;
    const vdt_model* m = c->m;
    const size_t in_bytes = (size_t)batch * m->in_elems * sizeof(float);
    const size_t out_bytes = (size_t)batch * m->n_classes * sizeof(float);
    const size_t pred_bytes = (size_t)batch * sizeof(int32_t);
    float* const ins[2] = {c->in_slot, c->in_slot2};
    float* const outs[2] = {c->out_slot, c->out_slot2};
    int32_t* const preds[2] = {c->pred_slot, c->pred_slot2};
    cudaStream_t cs = c->copy_stream;
    // batch i uses slot i % 2.  Copy stream: H2D(0), H2D(1), then per batch
    // i: D2H(i) after its compute, H2D(i + 2) once compute(i) has released
    // the slot.  The ctx stream runs compute(i) once H2D(i) has landed.
    VDT_CUDA(cudaMemcpyAsync(ins[0], h_inputs[0], in_bytes, cudaMemcpyHostToDevice, cs));
    VDT_CUDA(cudaEventRecord(c->ev_h2d[0], cs));
    for (int i = 0; i < n_batches; ++i) {
        const int s = i & 1;
        VDT_CUDA(cudaStreamWaitEvent(c->stream, c->ev_h2d[s], 0));
        if (int st = run_slots(c, input_is_pixels, batch, s)) return st;
        VDT_CUDA(cudaEventRecord(c->ev_done[s], c->stream));
        if (i + 1 < n_batches) {                             // next input, overlapping compute(i)
            const int s1 = (i + 1) & 1;
            if (i >= 1) VDT_CUDA(cudaStreamWaitEvent(cs, c->ev_done[s1], 0));   // compute(i - 1) left the slot
            VDT_CUDA(cudaMemcpyAsync(ins[s1], h_inputs[i + 1], in_bytes, cudaMemcpyHostToDevice, cs));
            VDT_CUDA(cudaEventRecord(c->ev_h2d[s1], cs));
        }
        VDT_CUDA(cudaStreamWaitEvent(cs, c->ev_done[s], 0));
        if (h_outs && h_outs[i]) VDT_CUDA(cudaMemcpyAsync(h_outs[i], outs[s], out_bytes, cudaMemcpyDeviceToHost, cs));
        if (h_preds && h_preds[i])
            VDT_CUDA(cudaMemcpyAsync(h_preds[i], preds[s], pred_bytes, cudaMemcpyDeviceToHost, cs));
    }
    VDT_CUDA(cudaStreamSynchronize(cs));
    VDT_CUDA(cudaStreamSynchronize(c->stream));
    return VDT_OK;
}

extern "C" int vdt_infer_trace(vdt_ctx* c, const float* d_input, int input_is_pixels, int batch,
                               float* const* d_layer_out, float* d_out, int32_t* d_pred) {
    g_last_error.clear();
    if (int s = check_batch(c, batch)) return s;
    if (!d_input || !d_out || !d_layer_out) return fail(VDT_ERR_INVALID, "NULL buffer");
    if (int s = check_device_buffers(c->m->device, {d_input, d_out, d_pred})) return s;
    for (int i = 0; i < model_stages(c->m); ++i)
        if (int s = check_device_buffers(c->m->device, {d_layer_out[i]})) return s;
    DeviceGuard g(c->m->device);
    return enqueue(c, d_input, input_is_pixels, batch, d_out, d_pred, d_layer_out);
}

// ------------------------------------------------------- per-stage entries
extern "C" int vdt_build_luts(int T, int decay_len, float tc_integ, float td_integ, float tc_fire,
                              float td_fire, float vth_init, float* d_decay, float* d_th,
                              vdt_stream stream) {
    g_last_error.clear();
    if (T < 1 || decay_len < 1 || !d_decay || !d_th) return fail(VDT_ERR_INVALID, "bad LUT arguments");
    if (int s = check_device_buffers(-1, {d_decay, d_th})) return s;
    const LutJob j{tc_integ, td_integ, tc_fire, td_fire, d_decay, d_th};
    VDT_CUDA(launch_build_lut_one(j, T, decay_len, vth_init, static_cast<cudaStream_t>(stream)));
    return VDT_OK;
}

extern "C" int vdt_encode(const float* d_pixels, float* d_spikes, int64_t n, int encoder, float tc,
                          float td, int T, float inf_time, vdt_stream stream) {
    g_last_error.clear();
    if (!d_pixels || !d_spikes || n < 0) return fail(VDT_ERR_INVALID, "bad encode arguments");
    if (int s = check_device_buffers(-1, {d_pixels, d_spikes})) return s;
    if (encoder != VDT_ENC_LOG && encoder != VDT_ENC_LINEAR) return fail(VDT_ERR_INVALID, "encoder=%d", encoder);
    VDT_CUDA(launch_encode(d_pixels, d_spikes, n, encoder, tc, td, T, inf_time, static_cast<cudaStream_t>(stream)));
    return VDT_OK;
}

extern "C" int vdt_bucketize(const float* d_in, int64_t n_cols, int c_in, int layout, int64_t hw,
                             const vdt_time_cfg* cfg, int tb_mode, int* d_off, int* d_cin,
                             float* d_tin, vdt_stream stream) {
    g_last_error.clear();
    if (int s = check_cfg(cfg)) return s;
    if (!d_in || !d_off || !d_cin || !d_tin || n_cols < 0 || c_in <= 0)
        return fail(VDT_ERR_INVALID, "bad bucketize arguments");
    if (layout == VDT_LAYOUT_NCHW && (hw <= 0 || n_cols % hw != 0))
        return fail(VDT_ERR_INVALID, "NCHW needs hw > 0 dividing n_cols");
    if (tb_mode != VDT_TB_FLOOR_STAGGER && tb_mode != VDT_TB_TRUNC) return fail(VDT_ERR_INVALID, "tb_mode");
    if (int s = check_device_buffers(-1, {d_in, d_off, d_cin, d_tin})) return s;
    BktParams p{};
    p.in = d_in; p.n_cols = n_cols; p.c_in = c_in; p.layout = layout; p.hw = hw < 1 ? 1 : hw;
    p.T = cfg->T; p.delta = cfg->delta; p.NC = (cfg->T + cfg->delta - 1) / cfg->delta;
    p.tfs = cfg->fire_start; p.tb_mode = tb_mode; p.inf_time = cfg->inf_time;
    p.off = d_off; p.cin = d_cin; p.tin = d_tin; p.events = nullptr;
    cudaError_t e = launch_bucketize(p, static_cast<cudaStream_t>(stream));
    if (e == cudaErrorInvalidValue) return fail(VDT_ERR_UNSUPPORTED, "too many chunks for the counters");
    VDT_CUDA(e);
    return VDT_OK;
}

extern "C" int vdt_conv_bucketed(const int* d_off, const int* d_cin, const float* d_tin,
                                 const float* d_kernel, const float* d_bias, const float* d_decay,
                                 const float* d_th, int t_min, int B, int H_in, int W_in, int C_in,
                                 int H_out, int W_out, int C_out, int K, int pad, int is_fc,
                                 const vdt_time_cfg* cfg, float* d_out, vdt_stream stream) {
    g_last_error.clear();
    if (int s = check_cfg(cfg)) return s;
    if (!d_off || !d_cin || !d_tin || !d_kernel || !d_bias || !d_decay || !d_th || !d_out)
        return fail(VDT_ERR_INVALID, "NULL buffer");
    if (B < 0 || C_in <= 0 || C_out <= 0 || (!is_fc && (H_out <= 0 || W_out <= 0 || K <= 0)))
        return fail(VDT_ERR_INVALID, "bad shape");
    if (!integrate_supported(K, is_fc, cfg->delta, C_out, cfg->T, cfg->decay_len))
        return fail(VDT_ERR_UNSUPPORTED, "delta must be a power of two <= 64 and K*K <= 32");
    if (int s = check_device_buffers(-1, {d_off, d_cin, d_tin, d_kernel, d_bias, d_decay, d_th, d_out})) return s;
    IntegParams ip{};
    ip.off = d_off; ip.cin = d_cin; ip.tin = d_tin;
    ip.W = d_kernel; ip.bias = d_bias; ip.lut_decay = d_decay; ip.lut_th = d_th; ip.out = d_out;
    ip.B = B; ip.H_in = is_fc ? 1 : H_in; ip.W_in = is_fc ? 1 : W_in; ip.C_in = C_in;
    ip.H_out = is_fc ? 1 : H_out; ip.W_out = is_fc ? 1 : W_out; ip.C_out = C_out;
    ip.K = is_fc ? 1 : K; ip.pad = is_fc ? 0 : pad; ip.is_fc = is_fc != 0;
    ip.T = cfg->T; ip.delta = cfg->delta; ip.NC = (cfg->T + cfg->delta - 1) / cfg->delta;
    ip.t_min = t_min; ip.lut_mode = cfg->lut_mode; ip.decay_len = cfg->decay_len;
    ip.tfs = cfg->fire_start; ip.inf_time = cfg->inf_time; ip.fetched = nullptr;
    VDT_CUDA(launch_integrate(ip, static_cast<cudaStream_t>(stream)));
    return VDT_OK;
}

extern "C" int vdt_layer_vmem(const float* d_in, const float* d_kernel, const float* d_bias,
                              const float* d_decay, int B, int C_in, int C_out,
                              const vdt_time_cfg* cfg, float* d_out, vdt_stream stream) {
    g_last_error.clear();
    if (int s = check_cfg(cfg)) return s;
    if (!d_in || !d_kernel || !d_bias || !d_decay || !d_out || B < 0 || C_in <= 0 || C_out <= 0)
        return fail(VDT_ERR_INVALID, "bad vmem arguments");
    if (int s = check_device_buffers(-1, {d_in, d_kernel, d_bias, d_decay, d_out})) return s;
    cudaError_t e = launch_layer_vmem(d_in, d_kernel, d_bias, d_decay, B, C_in, C_out, cfg->T,
                                      cfg->fire_start, cfg->inf_time, d_out, static_cast<cudaStream_t>(stream));
    if (e == cudaErrorInvalidValue) return fail(VDT_ERR_UNSUPPORTED, "C_in too large for the vmem kernel");
    VDT_CUDA(e);
    return VDT_OK;
}

extern "C" int vdt_pool_min(const float* d_in, float* d_out, int B, int H_in, int W_in, int C,
                            float inf_time, vdt_stream stream) {
    g_last_error.clear();
    if (!d_in || !d_out || B < 0 || H_in < 2 || W_in < 2 || C <= 0) return fail(VDT_ERR_INVALID, "bad pool arguments");
    if (int s = check_device_buffers(-1, {d_in, d_out})) return s;
    VDT_CUDA(launch_pool_min(d_in, d_out, B, H_in, W_in, C, inf_time, static_cast<cudaStream_t>(stream)));
    return VDT_OK;
}

extern "C" int vdt_readout(const float* d_out, int B, int K, int mode, float inf_time, int32_t* d_pred,
                           vdt_stream stream) {
    g_last_error.clear();
    if (!d_out || !d_pred || B < 0 || K <= 0) return fail(VDT_ERR_INVALID, "bad readout arguments");
    if (mode < VDT_READ_ARGMIN_FIRST || mode > VDT_READ_ARGMAX) return fail(VDT_ERR_INVALID, "mode=%d", mode);
    if (int s = check_device_buffers(-1, {d_out, d_pred})) return s;
    VDT_CUDA(launch_readout(d_out, B, K, mode, inf_time, d_pred, static_cast<cudaStream_t>(stream)));
    return VDT_OK;
}
