// k_culif.cu -- task-3 (DVS gesture) CuLIF layers that are not bucketed
// integrators: the raw-frame first convolution, the spiking 2x2 pool and the
// recurrent FC1.  Same results as the reference kernels, bit for bit:
//   conv1_raw_early        t3:30-65
//   pool_chunk_early       t3:146-168
//   fc1_bucketed_recurrent t3:171-200
// (the bucketed conv / fc2 layers run on k_sorted, launch_culif).
//
// CuLIF step (every kernel): I = fma(I, decay, in[t]); V += I; fire at the
// first t with V >= th.  The scan covers whole chunks (t < NC*delta, no t < T
// guard, as in the reference).
#include "lanes.h"
#include "vdt_internal.h"

namespace vdt {
namespace {

// ------------------------------------------------------------ conv1 (raw) --
// One warp per output pixel (n, y, x), lane l owns output channels
// l*V .. l*V+V-1.  Per chunk the pixel's K*K*C_in input frame windows (delta
// time bins each, contiguous in memory: frames are [N, C_in, H, W, T]) are
// staged in shared memory and lane t marks the taps with a nonzero value in
// bin t.  Each step then walks its marked taps in the reference's order
// (c_in, ky, kx) with one FMA each: a zero frame value (and an out-of-range
// tap, which the reference skips) leaves the FMA chain unchanged, since
// fma(w, 0, acc) = acc for finite w and an accumulator that is never -0.
// Frames past T read as 0.
constexpr int C1_WARPS = 4;

template <int V, int DELTA>
__global__ void __launch_bounds__(C1_WARPS * 32) k_culif_conv1(const float* __restrict__ frames,
                                                               const float* __restrict__ w_oihw,
                                                               float* __restrict__ out, int N, int C_in,
                                                               int C_out, int H, int W, int K, int T,
                                                               int NC, float decay, float th) {
    extern __shared__ float c1_sm[];
    __shared__ long long s_toff[32];                          // per tap: frame offset from the pixel's own
    __shared__ int s_tdy[32], s_tdx[32];                      // per tap: row / column offset
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int taps = C_in * K * K;                            // <= 32
    float* s_w = c1_sm;                                       // [taps][C_out]
    float* s_f = c1_sm + taps * C_out + warp * taps * DELTA;  // [taps][DELTA]
    for (int i = threadIdx.x; i < taps * C_out; i += blockDim.x) {
        const int q = i / C_out, co = i - q * C_out;
        s_w[i] = __ldg(w_oihw + (long long)co * taps + q);
    }
    if (threadIdx.x < taps) {                                 // tap q = (c_in, ky, kx), the reference's order
        const int q = threadIdx.x, ci = q / (K * K), r = q - ci * K * K, ky = r / K, kx = r - ky * K;
        s_tdy[q] = ky - K / 2;
        s_tdx[q] = kx - K / 2;
        s_toff[q] = (((long long)ci * H + (ky - K / 2)) * W + (kx - K / 2)) * T;
    }
    __syncthreads();
    const long long gw = (long long)blockIdx.x * C1_WARPS + warp;
    if (gw >= (long long)N * H * W) return;
    const int x = (int)(gw % W);
    const int y = (int)((gw / W) % H);
    const long long n = gw / ((long long)W * H);
    const int c0 = lane * V;
    const bool lane_ok = c0 < C_out;
    const float* wl = s_w + (lane_ok ? c0 : 0);

    CulifLanes<V> nu;
    nu.init(lane_ok, 9999.0f);
    const CulifCfg cc{decay, th};
    // the pixel's own frame row: frames[n][0][y][x][0]
    const float* fpix = frames + ((n * C_in * H + y) * (long long)W + x) * T;
    for (int tau = 0; tau < NC; ++tau) {
        const int base = tau * DELTA;
        // lane l stages bin l % DELTA of taps l / DELTA, l / DELTA + 32 / DELTA, ...
        // and marks the nonzero ones; OR over the lanes of one bin gives its mask
        unsigned mask = 0;                                    // lane t: taps with input in bin t
        for (int i = lane; i < taps * DELTA; i += 32) {
            const int q = i / DELTA, t = i - q * DELTA;      // DELTA is a power of two
            float v = 0.0f;
            if ((unsigned)(y + s_tdy[q]) < (unsigned)H && (unsigned)(x + s_tdx[q]) < (unsigned)W && base + t < T)
                v = __ldg(fpix + s_toff[q] + base + t);
            s_f[i] = v;
            mask |= (v != 0.0f ? 1u : 0u) << q;
        }
#pragma unroll
        for (int o = DELTA; o < 32; o <<= 1) mask |= __shfl_xor_sync(FULL_MASK, mask, o);
        __syncwarp();
#pragma unroll 4
        for (int t = 0; t < DELTA; ++t) {
            unsigned m = __shfl_sync(FULL_MASK, mask, t);
            float in[V];
#pragma unroll
            for (int v = 0; v < V; ++v) in[v] = 0.0f;
            while (m) {                                       // warp-uniform
                const int q = __ffs(m) - 1;
                m &= m - 1;
                const float f = s_f[q * DELTA + t];
#pragma unroll
                for (int v = 0; v < V; ++v) in[v] = fmaf(wl[q * C_out + v], f, in[v]);
            }
            nu.step_all(base + t, in, cc);
        }
        __syncwarp();
        if (!__any_sync(FULL_MASK, nu.any())) break;
    }
    if (lane_ok) {
#pragma unroll
        for (int v = 0; v < V; ++v)
            out[((n * C_out + c0 + v) * H + y) * (long long)W + x] = nu.res[v];
    }
}

// ------------------------------------------------------------------ pool --
// One thread per output neuron; in[t] = 1 at each of the 4 inputs' spike
// bins (set, not added).  layout: VDT_LAYOUT_NCHW or VDT_LAYOUT_NHWC.
__global__ void k_culif_pool(const float* __restrict__ in, float* __restrict__ out, int N, int C, int H_in,
                             int W_in, int layout, int delta, int NC, float decay, float th) {
    const int H_out = H_in / 2, W_out = W_in / 2;
    const long long total = (long long)N * C * H_out * W_out;
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += stride) {
        long long n;
        int c, yo, xo;
        if (layout == VDT_LAYOUT_NCHW) {
            xo = (int)(idx % W_out);
            yo = (int)((idx / W_out) % H_out);
            c = (int)((idx / ((long long)W_out * H_out)) % C);
            n = idx / ((long long)W_out * H_out * C);
        } else {
            c = (int)(idx % C);
            xo = (int)((idx / C) % W_out);
            yo = (int)((idx / ((long long)C * W_out)) % H_out);
            n = idx / ((long long)C * W_out * H_out);
        }
        float tf[4];
#pragma unroll
        for (int d = 0; d < 4; ++d) {
            const int yy = yo * 2 + (d >> 1), xx = xo * 2 + (d & 1);
            const long long at = layout == VDT_LAYOUT_NCHW ? ((n * C + c) * H_in + yy) * (long long)W_in + xx
                                                            : ((n * H_in + yy) * (long long)W_in + xx) * C + c;
            tf[d] = __ldg(in + at);
        }
        float I = 0.0f, V = 0.0f, res = 9999.0f;
        // before the first input spike I and V stay exactly 0 (fma(0, d, 0) = 0,
        // 0 + 0 = 0), so with th > 0 nothing can fire there: start at the
        // chunk holding the earliest spike of the scan (none: never fires)
        int tau0 = 0;
        if (th > 0.0f) {
            float tmin = 3.0e38f;
#pragma unroll
            for (int d = 0; d < 4; ++d)
                if (tf[d] >= 0.0f && tf[d] < (float)(NC * delta)) tmin = fminf(tmin, tf[d]);
            tau0 = tmin < 3.0e38f ? (int)tmin / delta : NC;
        }
        for (int tau = tau0; tau < NC; ++tau) {
            const int base = tau * delta;
            unsigned long long set = 0;                      // bins of this chunk holding a spike
#pragma unroll
            for (int d = 0; d < 4; ++d)
                if (tf[d] >= (float)base && tf[d] < (float)(base + delta)) set |= 1ull << ((int)tf[d] - base);
            bool fired = false;
            for (int t = 0; t < delta; ++t) {
                I = fmaf(I, decay, (set >> t) & 1ull ? 1.0f : 0.0f);
                V += I;
                if (V >= th) { res = (float)(base + t); fired = true; break; }
            }
            if (fired) break;
        }
        out[idx] = res;
    }
}

// -------------------------------------------------------------- FC1 (rec) --
// One CTA per sample, one thread per output neuron (F_out <= 1024).  Per
// chunk the feed-forward input in_ff[t][i] is summed in shared memory in the
// reference's order (the sample's bucket, ascending j inside a chunk), then
// the chunk's steps run in lock-step: the recurrent input of neuron i sums
// W_rec[i][j] over the neurons j that fired on the previous step (ascending
// j), I = fma(I, decay, in_ff) + in_rec, V += I; a neuron fires once and
// its V is reset to -10000.  No early exit.  Weights are transposed:
// w_t[j][i] = W_fc1[i][j], wrec_t[j][i] = W_rec[i][j].
// FC1's feed-forward input, event-parallel: one warp per (sample, step,
// group of 128 neurons), lane l owns neurons 4l..4l+3 of the group and sums
// them in registers.  The warp scans its chunk's bucket list 32 events at a
// time and takes the events of its own step (ballot, lowest lane first), so
// per (step, neuron) the additions run in bucket order: the reference's
// in_ff[tt - base] += w chain (t3:186).  Up to 8 weight rows load at once.
// Output ff[n][t][i] for t < NC * delta.
constexpr int FF_WARPS = 4;

__global__ void __launch_bounds__(FF_WARPS * 32) k_fc1_ff(const int* __restrict__ off, const int* __restrict__ bcin,
                                                          const float* __restrict__ btin,
                                                          const float* __restrict__ w_t, float* __restrict__ ff,
                                                          int N, int F_in, int F_out, int delta, int NC) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = F_out / 128, TS = NC * delta;
    const long long item = (long long)blockIdx.x * FF_WARPS + warp;
    if (item >= (long long)N * TS * G) return;               // warp-uniform
    const int g = (int)(item % G);
    const int t = (int)((item / G) % TS);
    const long long n = item / ((long long)G * TS);
    const int ch = t / delta, OS = NC + 1;
    const int s = __ldg(off + n * OS + ch), e = __ldg(off + n * OS + ch + 1);
    const int* sc = bcin + n * F_in;
    const float* st = btin + n * F_in;
    const float* wl = w_t + g * 128 + lane * 4;
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (int p0 = s; p0 < e; p0 += 32) {
        int j = 0;
        bool mine = false;
        if (p0 + lane < e) {
            j = __ldg(sc + p0 + lane);
            mine = (int)__ldg(st + p0 + lane) == t;
        }
        unsigned m = __ballot_sync(FULL_MASK, mine);
        while (m) {                                          // warp-uniform
            float4 w[8];
            int cnt = 0;
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                if (m) {
                    const int b = __ffs(m) - 1;
                    m &= m - 1;
                    const int jq = __shfl_sync(FULL_MASK, j, b);
                    w[u] = __ldg(reinterpret_cast<const float4*>(wl + (long long)jq * F_out));
                    cnt = u + 1;
                }
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                if (u < cnt) { acc.x += w[u].x; acc.y += w[u].y; acc.z += w[u].z; acc.w += w[u].w; }
            }
        }
    }
    *reinterpret_cast<float4*>(ff + (n * TS + t) * F_out + g * 128 + lane * 4) = acc;
}

// With ff (k_fc1_ff's feed-forward sums) each chunk reads those sums;
// without, each neuron sums its own events.
__global__ void k_culif_fc1_rec(const int* __restrict__ off, const int* __restrict__ bcin,
                                const float* __restrict__ btin, const float* __restrict__ w_t,
                                const float* __restrict__ wrec_t, const float* __restrict__ ff,
                                float* __restrict__ out, int F_in, int F_out, int delta, int NC, float decay,
                                float th) {
    extern __shared__ float f1_sm[];
    float* s_ff = f1_sm;                                     // [delta][F_out]
    unsigned* s_prev = reinterpret_cast<unsigned*>(s_ff + (size_t)delta * F_out);   // fired bitmap
    const int i = threadIdx.x;
    const long long n = blockIdx.x;
    const int words = (F_out + 31) / 32;
    for (int k = i; k < words; k += blockDim.x) s_prev[k] = 0u;
    float I = 0.0f, V = 0.0f, fire = 9999.0f;
    bool has = false;
    const int OS = NC + 1;
    const int* sc = bcin + n * F_in;
    const float* st = btin + n * F_in;
    for (int ch = 0; ch < NC; ++ch) {
        const int base = ch * delta;
        if (ff) {
            const float* fr = ff + (n * NC * delta + base) * F_out + i;
            for (int t = 0; t < delta; ++t) s_ff[t * F_out + i] = __ldg(fr + (long long)t * F_out);
        } else {
            for (int t = 0; t < delta; ++t) s_ff[t * F_out + i] = 0.0f;
            const int s = __ldg(off + n * OS + ch), e = __ldg(off + n * OS + ch + 1);
            for (int p = s; p < e; ++p) {
                const int j = __ldg(sc + p);
                const int tt = (int)__ldg(st + p);
                s_ff[(tt - base) * F_out + i] += __ldg(w_t + (long long)j * F_out + i);
            }
        }
        for (int t = 0; t < delta; ++t) {
            __syncthreads();                                 // previous step's bitmap complete
            float in_rec = 0.0f;
            for (int k = 0; k < words; ++k) {
                unsigned m = s_prev[k];
                while (m) {
                    const int b = __ffs(m) - 1;
                    m &= m - 1;
                    in_rec += __ldg(wrec_t + (long long)(k * 32 + b) * F_out + i);
                }
            }
            I = fmaf(I, decay, s_ff[t * F_out + i]) + in_rec;
            V += I;
            bool now = false;
            if (V >= th && !has) { now = true; has = true; fire = (float)(base + t); V = -10000.0f; }
            __syncthreads();                                 // everyone read the old bitmap
            const unsigned bits = __ballot_sync(FULL_MASK, now);
            if ((i & 31) == 0) s_prev[i >> 5] = bits;
        }
    }
    out[n * F_out + i] = fire;
}

// OIHW -> HWIO ([K][K][C_in][C_out]) weight permutation
__global__ void k_oihw_to_hwio(const float* __restrict__ src, float* __restrict__ dst, int O, int I, int K) {
    const long long total = (long long)O * I * K * K;
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long d = (long long)blockIdx.x * blockDim.x + threadIdx.x; d < total; d += stride) {
        const int o = (int)(d % O);
        long long r = d / O;
        const int ci = (int)(r % I);
        r /= I;
        const int kx = (int)(r % K), ky = (int)(r / K);
        dst[d] = src[(((long long)o * I + ci) * K + ky) * K + kx];
    }
}

unsigned grid_1d(long long n, int threads) {
    long long b = (n + threads - 1) / threads;
    const long long cap = 148LL * 32;
    return (unsigned)(b < 1 ? 1 : (b > cap ? cap : b));
}

template <int V, int DELTA>
cudaError_t launch_conv1_vd(const float* frames, const float* w, float* out, int N, int C_in, int C_out, int H,
                            int W, int K, int T, int NC, float decay, float th, cudaStream_t s) {
    const size_t smem = ((size_t)C1_WARPS * DELTA + C_out) * C_in * K * K * sizeof(float);
    auto kern = k_culif_conv1<V, DELTA>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    const long long warps = (long long)N * H * W;
    kern<<<(unsigned)((warps + C1_WARPS - 1) / C1_WARPS), C1_WARPS * 32, smem, s>>>(
        frames, w, out, N, C_in, C_out, H, W, K, T, NC, decay, th);
    return cudaGetLastError();
}

template <int V>
cudaError_t launch_conv1_v(const float* frames, const float* w, float* out, int N, int C_in, int C_out, int H,
                           int W, int K, int T, int delta, float decay, float th, cudaStream_t s) {
    const int NC = (T + delta - 1) / delta;
    switch (delta) {
        case 8: return launch_conv1_vd<V, 8>(frames, w, out, N, C_in, C_out, H, W, K, T, NC, decay, th, s);
        case 16: return launch_conv1_vd<V, 16>(frames, w, out, N, C_in, C_out, H, W, K, T, NC, decay, th, s);
        case 32: return launch_conv1_vd<V, 32>(frames, w, out, N, C_in, C_out, H, W, K, T, NC, decay, th, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

bool culif_conv1_supported(int C_in, int C_out, int K, int delta) {
    if (delta != 8 && delta != 16 && delta != 32) return false;
    if (C_out > 128 || C_in * K * K > 32) return false;       // tap mask in one word
    return ((size_t)C1_WARPS * delta + C_out) * C_in * K * K * sizeof(float) <= 200 * 1024;
}

cudaError_t launch_culif_conv1(const float* frames, const float* w_oihw, float* out, int N, int C_in, int C_out,
                               int H, int W, int K, int T, int delta, float decay, float th, cudaStream_t s) {
    if (!culif_conv1_supported(C_in, C_out, K, delta)) return cudaErrorInvalidValue;
    if (N <= 0) return cudaSuccess;
    if (C_out <= 32) return launch_conv1_v<1>(frames, w_oihw, out, N, C_in, C_out, H, W, K, T, delta, decay, th, s);
    if (C_out <= 64) return launch_conv1_v<2>(frames, w_oihw, out, N, C_in, C_out, H, W, K, T, delta, decay, th, s);
    return launch_conv1_v<4>(frames, w_oihw, out, N, C_in, C_out, H, W, K, T, delta, decay, th, s);
}

cudaError_t launch_culif_pool(const float* in, float* out, int N, int C, int H_in, int W_in, int layout,
                              int T, int delta, float decay, float th, cudaStream_t s) {
    if (delta < 1 || delta > 64) return cudaErrorInvalidValue;
    const long long total = (long long)N * C * (H_in / 2) * (W_in / 2);
    if (total <= 0) return cudaSuccess;
    const int NC = (T + delta - 1) / delta;
    k_culif_pool<<<grid_1d(total, 256), 256, 0, s>>>(in, out, N, C, H_in, W_in, layout, delta, NC, decay, th);
    return cudaGetLastError();
}

size_t culif_fc1_scratch_bytes(int N, int F_out, int T, int delta) {
    if (N <= 0 || F_out % 128 != 0 || delta < 1) return 0;
    const int NC = (T + delta - 1) / delta;
    return (size_t)N * NC * delta * F_out * sizeof(float);
}

cudaError_t launch_culif_fc1_rec(const int* off, const int* cin, const float* tin, const float* w_t,
                                 const float* wrec_t, float* out, int N, int F_in, int F_out, int T, int delta,
                                 float decay, float th, cudaStream_t s, float* scratch) {
    if (F_out < 1 || F_out > 1024 || F_out % 32 != 0 || delta < 1) return cudaErrorInvalidValue;
    if (N <= 0) return cudaSuccess;
    const int NC = (T + delta - 1) / delta;
    const size_t smem = (size_t)delta * F_out * sizeof(float) + (size_t)(F_out / 32) * sizeof(unsigned);
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(k_culif_fc1_rec, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    // feed-forward sums first, event-parallel, where the neurons split into
    // groups of 128 and the per-warp step table fits: into the caller's
    // scratch, else a stream-ordered allocation freed after the launch
    float* ff = nullptr;
    bool own = false;
    if (culif_fc1_scratch_bytes(N, F_out, T, delta) > 0) {
        cudaError_t e = cudaSuccess;
        if (scratch) {
            ff = scratch;
        } else {
            e = cudaMallocAsync(&ff, culif_fc1_scratch_bytes(N, F_out, T, delta), s);
            if (e != cudaSuccess) return e;
            own = true;
        }
        const long long items = (long long)N * NC * delta * (F_out / 128);
        if ((items + FF_WARPS - 1) / FF_WARPS >= (1ll << 31)) e = cudaErrorInvalidValue;
        if (e == cudaSuccess) {
            k_fc1_ff<<<(unsigned)((items + FF_WARPS - 1) / FF_WARPS), FF_WARPS * 32, 0, s>>>(
                off, cin, tin, w_t, ff, N, F_in, F_out, delta, NC);
            e = cudaGetLastError();
        }
        if (e != cudaSuccess) {
            if (own) cudaFreeAsync(ff, s);
            return e;
        }
    }
    k_culif_fc1_rec<<<N, F_out, smem, s>>>(off, cin, tin, w_t, wrec_t, ff, out, F_in, F_out, delta, NC, decay, th);
    cudaError_t e = cudaGetLastError();
    if (own) {
        const cudaError_t e2 = cudaFreeAsync(ff, s);
        if (e == cudaSuccess) e = e2;
    }
    return e;
}

cudaError_t launch_oihw_to_hwio(const float* src, float* dst, int O, int I, int K, cudaStream_t s) {
    const long long total = (long long)O * I * K * K;
    if (total <= 0) return cudaSuccess;
    k_oihw_to_hwio<<<grid_1d(total, 256), 256, 0, s>>>(src, dst, O, I, K);
    return cudaGetLastError();
}

}  // namespace vdt
