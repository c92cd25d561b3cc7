// k_dense.cu -- integrator fused with the bucketing for layers whose
// per-pixel fan-in (K*K*C_in) is small: same results as k_bucketize +
// k_conv_bucketed (t1:45-162, t2:45-170), bit for bit.
//
// One warp integrates one output pixel for 32*V output channels:
//   1. read: the pixel's K*K*C_in input spike times, straight from the NHWC
//      spike map (lanes over the flattened (tap, channel) index, coalesced per
//      tap); an input is an event iff t < INF and tb = max(0, floor(t - TFS)) < T
//      (the bucketize rule, t1:57-59 / t2:58-60);
//   2. sort: a stable counting sort of the events by tb in shared memory
//      (warp-aggregated histogram with __match_any_sync, exclusive scan over the
//      T steps, ranked scatter).  The input order is (tap, channel), so inside
//      each step the list keeps exactly the reference's FMA-chain order;
//   3. stream: per event one broadcast LDS.64, one V-wide weight load, V FMAs
//      into a single accumulator per neuron; when the step changes, the step is
//      closed (carry += acc, threshold test) and steps without input are closed
//      in O(1) per neuron (non-increasing threshold tables: a constant carry
//      can fire in a run only if it reaches the run's last valid threshold).
//      The warp stops once all its neurons fired.
// The fetched-synapse counter keeps the reference's chunk accounting (events
// of every chunk a neuron entered alive).
#include "vdt_internal.h"

namespace vdt {
namespace {

constexpr unsigned FULL = 0xffffffffu;
constexpr int DW = 4;        // warps per CTA
constexpr int DSUB = 8;      // weight rows in flight per streamed batch
constexpr int DENSE_WIN = 36; // largest fan-in handled: 36 windows of 32 inputs

template <int V>
__device__ __forceinline__ void ldw(const float* p, float (&w)[V]) {
    if constexpr (V == 1) {
        w[0] = __ldg(p);
    } else if constexpr (V == 2) {
        const float2 v = __ldg(reinterpret_cast<const float2*>(p));
        w[0] = v.x; w[1] = v.y;
    } else {
        const float4 v = __ldg(reinterpret_cast<const float4*>(p));
        w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
    }
}

template <int V>
__device__ __forceinline__ void stw(float* p, const float (&r)[V]) {
    if constexpr (V == 1) {
        *p = r[0];
    } else if constexpr (V == 2) {
        *reinterpret_cast<float2*>(p) = make_float2(r[0], r[1]);
    } else {
        *reinterpret_cast<float4*>(p) = make_float4(r[0], r[1], r[2], r[3]);
    }
}

// shared words per warp: list (int2 per input), step bins (T + 1, padded),
// tap column bases (64-bit)
__host__ __device__ inline int dense_words(int fan_in, int T, int ntaps) {
    return ((2 * fan_in + 3) & ~3) + ((T + 1 + 3) & ~3) + ((2 * ntaps + 3) & ~3);
}

template <int V>
struct DLane {
    float carry[V], res[V], acc[V];
    bool alive[V];
    __device__ __forceinline__ bool any() const {
        bool a = false;
#pragma unroll
        for (int v = 0; v < V; ++v) a |= alive[v];
        return a;
    }
    __device__ __forceinline__ int live() const {
        int n = 0;
#pragma unroll
        for (int v = 0; v < V; ++v) n += alive[v] ? 1 : 0;
        return n;
    }
    __device__ __forceinline__ void close_step(int s, const float* s_th, int t_min) {
        const float th = s_th[s];
#pragma unroll
        for (int v = 0; v < V; ++v) {
            if (alive[v]) {
                carry[v] += acc[v];
                if (s >= t_min && carry[v] >= th && th >= 1e-5f) {
                    res[v] = (float)s;
                    alive[v] = false;
                }
            }
            acc[v] = 0.0f;
        }
    }
    __device__ __forceinline__ void close_empty(int a, int b, const float* s_th, int t_min, int t_floor,
                                                bool monotone) {
        if (a >= b) return;
        if (monotone) {
            const int lo = max(a, t_min), hi = min(b, t_floor);
            if (lo >= hi) return;
            const float mn = s_th[hi - 1];
#pragma unroll
            for (int v = 0; v < V; ++v) {
                if (alive[v] && carry[v] >= mn) {
                    // thresholds are non-increasing: the first step whose
                    // threshold the constant carry reaches, by bisection
                    int l = lo, h = hi - 1;
                    while (l < h) {
                        const int mid = (l + h) >> 1;
                        if (carry[v] >= s_th[mid]) h = mid; else l = mid + 1;
                    }
                    res[v] = (float)l;
                    alive[v] = false;
                }
            }
        } else {
            for (int t = a; t < b; ++t) {
                const float th = s_th[t];
#pragma unroll
                for (int v = 0; v < V; ++v)
                    if (alive[v] && t >= t_min && carry[v] >= th && th >= 1e-5f) {
                        res[v] = (float)t;
                        alive[v] = false;
                    }
            }
        }
    }
};

// flattened input index f = tap * C_in + c -> tap, via a float estimate and
// one exact correction (f < 2^20, so the estimate is off by at most one)
__device__ __forceinline__ int tap_of(int f, int C_in, float inv) {
    int j = __float2int_rz((float)f * inv);
    if (j * C_in > f) --j;
    else if ((j + 1) * C_in <= f) ++j;
    return j;
}

template <int V, int R, int MINB>
__global__ void __launch_bounds__(DW * 32, MINB) k_dense(IntegParams p, const float* __restrict__ in,
                                                         int n_warps, int groups) {
    extern __shared__ __align__(16) int sm[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntaps = p.is_fc ? 1 : p.K * p.K;
    const int fan = ntaps * p.C_in;
    const int words = dense_words(fan, p.T, ntaps);
    int* wb = sm + warp * words;
    int2* s_list = reinterpret_cast<int2*>(wb);
    int* s_bin = wb + ((2 * fan + 3) & ~3);                  // [T + 1]
    long long* s_col = reinterpret_cast<long long*>(s_bin + ((p.T + 1 + 3) & ~3));
    float* s_decay = reinterpret_cast<float*>(sm + DW * words);
    float* s_th = s_decay + p.decay_len;
    __shared__ int s_floor, s_mono;
    for (int i = threadIdx.x; i < p.decay_len; i += blockDim.x) s_decay[i] = p.lut_decay[i];
    for (int i = threadIdx.x; i < p.T; i += blockDim.x) s_th[i] = p.lut_th[i];
    if (threadIdx.x == 0) { s_floor = p.T; s_mono = 1; }
    __syncthreads();
    for (int t = threadIdx.x; t < p.T; t += blockDim.x) {
        if (!(s_th[t] >= 1e-5f)) atomicMin(&s_floor, t);
        if (t + 1 < p.T && !(s_th[t + 1] <= s_th[t])) s_mono = 0;
    }
    __syncthreads();
    const bool monotone = s_mono != 0;
    const int t_floor = s_floor;

    const int gw = blockIdx.x * DW + warp;
    if (gw >= n_warps) return;                               // warp-uniform
    const unsigned pix = (unsigned)gw / (unsigned)groups;
    const int grp = gw - (int)pix * groups;
    const int c0 = (grp * 32 + lane) * V;
    const bool lane_ok = c0 < p.C_out;
    int w_out = 0, h_out = 0;
    long long img = pix;
    if (!p.is_fc) {
        const unsigned r = pix / (unsigned)p.W_out;
        w_out = (int)(pix - r * (unsigned)p.W_out);
        const unsigned q = r / (unsigned)p.H_out;
        h_out = (int)(r - q * (unsigned)p.H_out);
        img = q;
    }
    if (lane < ntaps) {
        long long col = -1;
        if (p.is_fc) {
            col = img;
        } else {
            const int kh = lane / p.K, kw = lane - (lane / p.K) * p.K;
            const int h_in = h_out - p.pad + kh, w_in = w_out - p.pad + kw;
            if (h_in >= 0 && h_in < p.H_in && w_in >= 0 && w_in < p.W_in)
                col = (img * p.H_in + h_in) * p.W_in + w_in;
        }
        s_col[lane] = col < 0 ? -1 : col * p.C_in;
    }
    for (int i = lane; i <= p.T; i += 32) s_bin[i] = 0;
    __syncwarp();

    const float inv = 1.0f / (float)p.C_in;
    const unsigned lt = (1u << lane) - 1u;
    // all of the pixel's inputs in one round trip: input f = r*32 + lane
    float tv[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int f = r * 32 + lane;
        tv[r] = p.inf_time;
        if (f < fan) {
            const int j = tap_of(f, p.C_in, inv);
            const long long cb = s_col[j];
            if (cb >= 0) tv[r] = __ldg(in + cb + (f - j * p.C_in));
        }
    }
    // input value -> its step tb (or -1) and LUT value (bucketize rule)
    auto decode = [&](float t, int& tb, float& lv) {
        tb = -1;
        if (!(t < p.inf_time)) return;
        int b = (int)floorf(t - p.tfs);
        if (b < 0) b = 0;
        if (b >= p.T) return;
        int ti;
        if (p.lut_mode == VDT_LUT_BY_TB) {
            ti = b;
        } else {
            ti = (int)t;
            ti = ti < 0 ? 0 : (ti > p.T ? p.T : ti);
        }
        tb = b;
        lv = s_decay[ti];
    };
    // 1. histogram by step
#pragma unroll
    for (int r = 0; r < R; ++r) {
        int tb;
        float lv;
        decode(tv[r], tb, lv);
        const unsigned g = __match_any_sync(FULL, tb);
        if (tb >= 0 && lane == __ffs(g) - 1) s_bin[tb] += __popc(g);
        __syncwarp();
    }
    // 2. exclusive scan over steps, then the stable scatter
    int run = 0;
    for (int b0 = 0; b0 < p.T; b0 += 32) {
        const int b = b0 + lane;
        const int v = b < p.T ? s_bin[b] : 0;
        int x = v;
#pragma unroll
        for (int dd = 1; dd < 32; dd <<= 1) {
            const int u = __shfl_up_sync(FULL, x, dd);
            if (lane >= dd) x += u;
        }
        if (b < p.T) s_bin[b] = run + x - v;
        run += __shfl_sync(FULL, x, 31);
    }
    const int n = run;
    __syncwarp();
#pragma unroll
    for (int r = 0; r < R; ++r) {
        int tb;
        float lv;
        decode(tv[r], tb, lv);
        const unsigned g = __match_any_sync(FULL, tb);
        int pos = 0;
        if (tb >= 0) pos = s_bin[tb] + __popc(g & lt);
        __syncwarp();
        if (tb >= 0) {
            s_list[pos] = make_int2((r * 32 + lane) | (tb << 20), __float_as_int(lv));
            if (lane == __ffs(g) - 1) s_bin[tb] += __popc(g);
        }
        __syncwarp();
    }

    // 3. stream the step-ordered list
    DLane<V> nu;
#pragma unroll
    for (int v = 0; v < V; ++v) {
        nu.carry[v] = lane_ok ? __ldg(p.bias + c0 + v) : 0.0f;
        nu.res[v] = p.inf_time;
        nu.acc[v] = 0.0f;
        nu.alive[v] = lane_ok;
    }
    const float* Wl = p.W + (lane_ok ? c0 : 0);
    const int C_out = p.C_out;
    // fetched synapses, reference chunk accounting: the chunk sizes come from
    // the scattered bins (s_bin[tb] now holds the end of step tb's run)
    unsigned long long fetched = 0;
    int next_chunk = 0;
    auto step_end = [&](int t) { return t <= 0 ? 0 : s_bin[t - 1]; };   // events with tb < t
    auto account_one = [&]() {
        const int a = next_chunk * p.delta, b = min(p.T, a + p.delta);
        fetched += (unsigned long long)(step_end(b) - step_end(a)) * nu.live();
        ++next_chunk;
    };
    auto close_run = [&](int a, int b) {
        if (p.fetched) {
            while (next_chunk < p.NC && next_chunk * p.delta < b) {
                const int cs = max(a, next_chunk * p.delta);
                nu.close_empty(a, cs, s_th, p.t_min, t_floor, monotone);
                a = cs;
                account_one();
            }
        }
        nu.close_empty(a, b, s_th, p.t_min, t_floor, monotone);
    };

    // runs of equal step: stream the run into acc, then close the step
    int k = 0, next_t = 0;
    while (k < n) {
        const int tb = s_list[k].x >> 20;                     // warp-uniform
        const int end = s_bin[tb];                            // end of tb's run
        close_run(next_t, tb);
        if (p.fetched) {
            while (next_chunk < p.NC && next_chunk * p.delta <= tb) account_one();
        }
        if (!__any_sync(FULL, nu.any())) { next_t = p.T; break; }
        const bool lane_live = nu.any();
        float w[DSUB][V];
        for (; k + DSUB <= end; k += DSUB) {
            int2 e[DSUB];
#pragma unroll
            for (int u = 0; u < DSUB; ++u) e[u] = s_list[k + u];
            if (lane_live) {
#pragma unroll
                for (int u = 0; u < DSUB; ++u) ldw<V>(Wl + (e[u].x & 0xfffff) * C_out, w[u]);
            }
#pragma unroll
            for (int u = 0; u < DSUB; ++u) {
                const float lq = __int_as_float(e[u].y);
#pragma unroll
                for (int v = 0; v < V; ++v) nu.acc[v] = fmaf(w[u][v], lq, nu.acc[v]);
            }
        }
        for (; k < end; ++k) {
            const int2 e = s_list[k];
            if (lane_live) ldw<V>(Wl + (e.x & 0xfffff) * C_out, w[0]);
            const float lq = __int_as_float(e.y);
#pragma unroll
            for (int v = 0; v < V; ++v) nu.acc[v] = fmaf(w[0][v], lq, nu.acc[v]);
        }
        nu.close_step(tb, s_th, p.t_min);
        next_t = tb + 1;
    }
    close_run(next_t, p.T);
    if (p.fetched) {
        while (next_chunk < p.NC) account_one();
    }
    if (lane_ok) stw<V>(p.out + (long long)pix * p.C_out + c0, nu.res);
    if (p.fetched) {
#pragma unroll
        for (int dd = 16; dd > 0; dd >>= 1) fetched += __shfl_down_sync(FULL, fetched, dd);
        if (lane == 0 && fetched) atomicAdd(p.fetched, fetched);
    }
}

int pick_v_dense(int C_out) {
    if (C_out % 4 == 0 && C_out >= 128) return 4;
    if (C_out % 2 == 0 && C_out >= 64) return 2;
    return 1;
}

template <int V, int R>
cudaError_t launch_dense_vr(const IntegParams& p, const float* in, cudaStream_t s, int n_warps,
                            int groups) {
    const int ntaps = p.is_fc ? 1 : p.K * p.K;
    const size_t smem = (size_t)DW * dense_words(ntaps * p.C_in, p.T, ntaps) * sizeof(int) +
                        (size_t)(p.decay_len + p.T) * sizeof(float);
    constexpr int REGS = DSUB * V + 4 * V + R + 56;
    constexpr int MINB = (65536 / (DW * 32 * REGS)) > 8 ? 8 : (65536 / (DW * 32 * REGS));
    auto kern = k_dense<V, R, MINB>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    kern<<<(n_warps + DW - 1) / DW, DW * 32, smem, s>>>(p, in, n_warps, groups);
    return cudaGetLastError();
}

template <int V>
cudaError_t launch_dense_v(const IntegParams& p, const float* in, cudaStream_t s) {
    const int groups = (p.C_out + 32 * V - 1) / (32 * V);
    const long long pixels = p.is_fc ? (long long)p.B : (long long)p.B * p.H_out * p.W_out;
    const long long n_warps = pixels * groups;
    if (n_warps <= 0) return cudaSuccess;
    if (n_warps >= (1ll << 31)) return cudaErrorInvalidValue;   // 32-bit work index
    const int fan = (p.is_fc ? 1 : p.K * p.K) * p.C_in;
    const int w = (fan + 31) / 32;                          // 32-input windows per pixel
    if (w <= 1) return launch_dense_vr<V, 1>(p, in, s, (int)n_warps, groups);
    if (w <= 4) return launch_dense_vr<V, 4>(p, in, s, (int)n_warps, groups);
    if (w <= 9) return launch_dense_vr<V, 9>(p, in, s, (int)n_warps, groups);
    if (w <= 18) return launch_dense_vr<V, 18>(p, in, s, (int)n_warps, groups);
    return launch_dense_vr<V, DENSE_WIN>(p, in, s, (int)n_warps, groups);
}

}  // namespace

bool dense_supported(int K, int is_fc, int C_in, int T, int decay_len) {
    const int ntaps = is_fc ? 1 : K * K;
    const int fan = ntaps * C_in;
    if (ntaps > 32 || fan > DENSE_WIN * 32 || T >= 2048) return false;   // inputs held in registers
    return (size_t)DW * dense_words(fan, T, ntaps) * sizeof(int) + (size_t)(decay_len + T) * sizeof(float) <=
           160 * 1024;
}

cudaError_t launch_dense(const IntegParams& p, const float* in, cudaStream_t s) {
    switch (pick_v_dense(p.C_out)) {
        case 4: return launch_dense_v<4>(p, in, s);
        case 2: return launch_dense_v<2>(p, in, s);
        default: return launch_dense_v<1>(p, in, s);
    }
}

}  // namespace vdt
