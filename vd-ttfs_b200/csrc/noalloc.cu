// noalloc.cu -- one fire layer (bucketize + integrate) that allocates nothing.
//
// Some callers cannot let a library allocate device memory while they run:
// inference servers that plan every byte of device memory up front, loops
// that cannot take cudaMalloc's device-wide synchronisation, and plugin hosts
// that own the device allocator.  vdt_conv_layer_noalloc serves them.  Its
// only scratch -- the bucket lists between the counting sort and the
// integrator -- lives in the file-scope device array below: one copy of
// VDT_NOALLOC_SCRATCH_BYTES per GPU, created with the module and held until
// the process exits.  The caller passes every input and output.
//
// In host code the array's name is only a stand-in for the device symbol, so
// its device address is looked up with cudaGetSymbolAddress, with the device
// current, on the first call on each device (the caller's current device);
// that first call should come before any stream capture.  The address
// belongs to the module as loaded into one CUDA context: after
// cudaDeviceReset the device gets a new context, the module is loaded again
// and the array may move, so the cached address is keyed by the id of the
// context it was looked up in (cuCtxGetId, unique for the life of the
// process) and looked up again when the current context's id differs.  All
// calls on one device share the array, so calls that can overlap on the GPU
// race on it.  Nothing in it has to start at zero: the counting sort writes
// every chunk offset the integrator reads, and the integrator reads only list
// entries those offsets cover, written by the sort of the same call.
#include <cuda.h>   // CUcontext / CUresult of the two driver entry points below

#include <mutex>

#include "vdt_internal.h"

using namespace vdt;

namespace {

constexpr size_t kScratchBytes = VDT_NOALLOC_SCRATCH_BYTES;
__device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
struct ScratchSlot {
    unsigned long long ctx_id = 0;   // context the address was looked up in
    void* addr = nullptr;
};
ScratchSlot g_scratch[kMaxDevices];

// cuCtxGetCurrent / cuCtxGetId, reached through the runtime (the library
// links the runtime only)
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);
CtxGetCurrentFn g_ctx_current = nullptr;
CtxGetIdFn g_ctx_id = nullptr;

// id of the calling thread's current context; 0 when there is none yet
cudaError_t current_context_id(unsigned long long* id) {
    *id = 0;
    if (!g_ctx_current || !g_ctx_id) {
        cudaDriverEntryPointQueryResult q1 = cudaDriverEntryPointSymbolNotFound, q2 = q1;
        void* f1 = nullptr;
        void* f2 = nullptr;
        cudaError_t e = cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &f1, 12000, cudaEnableDefault, &q1);
        if (e == cudaSuccess) e = cudaGetDriverEntryPointByVersion("cuCtxGetId", &f2, 12000, cudaEnableDefault, &q2);
        if (e != cudaSuccess) return e;
        if (q1 != cudaDriverEntryPointSuccess || q2 != cudaDriverEntryPointSuccess || !f1 || !f2)
            return cudaErrorNotSupported;
        g_ctx_current = reinterpret_cast<CtxGetCurrentFn>(f1);
        g_ctx_id = reinterpret_cast<CtxGetIdFn>(f2);
    }
    CUcontext ctx = nullptr;
    if (g_ctx_current(&ctx) != CUDA_SUCCESS) return cudaErrorContextIsDestroyed;
    if (ctx && g_ctx_id(ctx, id) != CUDA_SUCCESS) return cudaErrorContextIsDestroyed;
    return cudaSuccess;
}

// device address of the scratch array in the current device's current context
cudaError_t scratch_address(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    unsigned long long id = 0;
    if ((e = current_context_id(&id)) != cudaSuccess) return e;
    ScratchSlot& slot = g_scratch[dev];
    if (!slot.addr || id == 0 || slot.ctx_id != id) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);    // also makes the context current
        if (e != cudaSuccess) return e;
        if (id == 0 && (e = current_context_id(&id)) != cudaSuccess) return e;
        slot.ctx_id = id;
        slot.addr = p;
    }
    *out = slot.addr;
    return cudaSuccess;
}

size_t round256(size_t n) { return (n + 255) & ~size_t(255); }

}  // namespace

extern "C" size_t vdt_noalloc_scratch_bytes(void) { return kScratchBytes; }

extern "C" int vdt_conv_layer_noalloc(const float* d_in, int tb_mode, const float* d_kernel,
                                      const float* d_bias, const float* d_decay, const float* d_th,
                                      int t_min, int B, int H_in, int W_in, int C_in, int H_out,
                                      int W_out, int C_out, int K, int pad, int is_fc,
                                      const vdt_time_cfg* cfg, float* d_out, vdt_stream stream) {
    api_clear_error();
    if (int s = api_check_cfg(cfg)) return s;
    if (!d_in || !d_kernel || !d_bias || !d_decay || !d_th || !d_out)
        return api_fail(VDT_ERR_INVALID, "NULL buffer");
    if (B < 0 || C_in <= 0 || C_out <= 0 ||
        (!is_fc && (H_in <= 0 || W_in <= 0 || H_out <= 0 || W_out <= 0 || K <= 0)))
        return api_fail(VDT_ERR_INVALID, "bad shape");
    if (tb_mode != VDT_TB_FLOOR_STAGGER && tb_mode != VDT_TB_TRUNC)
        return api_fail(VDT_ERR_INVALID, "tb_mode");
    if (!integrate_supported(K, is_fc, cfg->delta, C_out, cfg->T, cfg->decay_len))
        return api_fail(VDT_ERR_UNSUPPORTED, "delta must be a power of two <= 64 and K*K <= 32");

    const int NC = (cfg->T + cfg->delta - 1) / cfg->delta;
    const size_t n_cols = is_fc ? (size_t)B : (size_t)B * (size_t)H_in * (size_t)W_in;
    // scratch layout: [chunk offsets | channel lists | time lists]
    const size_t off_bytes = round256(n_cols * (size_t)(NC + 1) * sizeof(int));
    const size_t list_bytes = round256(n_cols * (size_t)C_in * sizeof(int));
    if (off_bytes + 2 * list_bytes > kScratchBytes)
        return api_fail(VDT_ERR_CAPACITY, "layer needs more bucket scratch than VDT_NOALLOC_SCRATCH_BYTES");
    if (B == 0) return VDT_OK;
    if (int s = api_check_buffers(-1, {d_in, d_kernel, d_bias, d_decay, d_th, d_out})) return s;

    void* base = nullptr;
    cudaError_t e = scratch_address(&base);
    if (e != cudaSuccess) return api_cuda_fail(e, "cudaGetSymbolAddress(noalloc scratch)");
    unsigned char* sb = static_cast<unsigned char*>(base);
    int* d_off = reinterpret_cast<int*>(sb);
    int* d_cin = reinterpret_cast<int*>(sb + off_bytes);
    float* d_tin = reinterpret_cast<float*>(sb + off_bytes + list_bytes);
    cudaStream_t s = static_cast<cudaStream_t>(stream);

    BktParams bp{};
    bp.in = d_in; bp.n_cols = (long long)n_cols; bp.c_in = C_in;
    bp.layout = VDT_LAYOUT_NHWC; bp.hw = 1;
    bp.T = cfg->T; bp.delta = cfg->delta; bp.NC = NC;
    bp.tfs = cfg->fire_start; bp.tb_mode = tb_mode; bp.inf_time = cfg->inf_time;
    bp.off = d_off; bp.cin = d_cin; bp.tin = d_tin; bp.events = nullptr;
    e = launch_bucketize(bp, s);
    if (e == cudaErrorInvalidValue) return api_fail(VDT_ERR_UNSUPPORTED, "too many chunks for the counters");
    if (e != cudaSuccess) return api_cuda_fail(e, "launch_bucketize");

    IntegParams ip{};
    ip.off = d_off; ip.cin = d_cin; ip.tin = d_tin;
    ip.W = d_kernel; ip.bias = d_bias; ip.lut_decay = d_decay; ip.lut_th = d_th; ip.out = d_out;
    ip.B = B; ip.H_in = is_fc ? 1 : H_in; ip.W_in = is_fc ? 1 : W_in; ip.C_in = C_in;
    ip.H_out = is_fc ? 1 : H_out; ip.W_out = is_fc ? 1 : W_out; ip.C_out = C_out;
    ip.K = is_fc ? 1 : K; ip.pad = is_fc ? 0 : pad; ip.is_fc = is_fc != 0;
    ip.T = cfg->T; ip.delta = cfg->delta; ip.NC = NC;
    ip.t_min = t_min; ip.lut_mode = cfg->lut_mode; ip.decay_len = cfg->decay_len;
    ip.tfs = cfg->fire_start; ip.inf_time = cfg->inf_time; ip.fetched = nullptr;
    e = launch_integrate(ip, s);
    if (e != cudaSuccess) return api_cuda_fail(e, "launch_integrate");
    return VDT_OK;
}
