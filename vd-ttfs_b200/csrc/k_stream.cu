// k_stream.cu -- the fused path's integrator over time-sorted buckets.
//
// Same result as k_conv_bucketed (t1:83-162, t2:84-170), bit for bit, but fed
// by buckets sorted at delta = 1 (a full stable counting sort by arrival step
// tb; vdt_bucketize with delta 1): per input column, fine offsets foff[tb]
// (T + 1 of them) and the events in (tb, channel) order.  The reference's
// chunk offsets at any delta are foff[c * delta].
//
// Each warp integrates one output pixel for 32*V output channels.  Per chunk
// (width DELTA) it builds, from the taps' fine offsets, one event stream in
// (step, tap, channel) order: for every step s the events are met exactly in
// the reference's FMA-chain order (tap, then channel), and all of step s's
// events are contiguous.  So one accumulator register per neuron suffices:
//     acc = fmaf(W[tap][cin][c], LUT_decay[ti], acc)   for the events of step s
//     carry += acc; fire if carry >= LUT_th[s] ...      when the step ends
// with no per-event dispatch on the step.  Weight rows are loaded EB at a time
// into registers, double-buffered (the next batch's rows are in flight while
// the current batch is applied), and the event records of the stream are
// decoded 32 at a time, one per lane.  The warp stops as soon as every one of
// its neurons has fired -- at step granularity, so it fetches no more
// synapses than the chunk-granular reference.
#include "vdt_internal.h"

namespace vdt {
namespace {

constexpr unsigned FULL = 0xffffffffu;
constexpr int SW = 4;      // warps per CTA
constexpr int EBS = 8;     // weight rows per batch

template <int V>
__device__ __forceinline__ void ldv(const float* p, float (&w)[V]) {
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
__device__ __forceinline__ void stv(float* p, const float (&r)[V]) {
    if constexpr (V == 1) {
        *p = r[0];
    } else if constexpr (V == 2) {
        *reinterpret_cast<float2*>(p) = make_float2(r[0], r[1]);
    } else {
        *reinterpret_cast<float4*>(p) = make_float4(r[0], r[1], r[2], r[3]);
    }
}

struct SEv {
    int step;    // absolute step tb of the event (-1: none)
    int wo;      // weight row offset
    float lv;    // LUT_decay value
};

// Neuron state of one lane (V neurons) and the step-finalisation rule.
template <int V>
struct Neurons {
    float carry[V], res[V], acc[V];
    bool alive[V];
    // close steps [from, to): the first gets this step's accumulated delta,
    // every step gets the threshold test (t1:150-157, t2:158-165).
    __device__ __forceinline__ void close(int from, int to, const float* s_th, int t_min, bool has_acc) {
        if (from >= to) return;
        if (has_acc) {
#pragma unroll
            for (int v = 0; v < V; ++v) {
                if (alive[v]) carry[v] += acc[v];
                acc[v] = 0.0f;
            }
        }
        for (int t = from; t < to; ++t) {
            const float th = s_th[t];
#pragma unroll
            for (int v = 0; v < V; ++v) {
                if (alive[v] && t >= t_min && carry[v] >= th && th >= 1e-5f) {
                    res[v] = (float)t;
                    alive[v] = false;
                }
            }
        }
    }
};

template <int DELTA, int V>
__global__ void __launch_bounds__(SW * 32, 4) k_stream(IntegParams p, const int* __restrict__ foff,
                                                       long long n_warps, int groups) {
    extern __shared__ __align__(16) int ssm[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntaps = p.is_fc ? 1 : p.K * p.K;
    const int cells = DELTA * ntaps;                      // (step, tap) cells per chunk
    int* s_P = ssm + warp * 2 * cells;                    // stream start of each cell
    int* s_O = s_P + cells;                               // bucket start of each cell
    float* s_decay = reinterpret_cast<float*>(ssm + SW * 2 * cells);
    float* s_th = s_decay + p.decay_len;
    for (int i = threadIdx.x; i < p.decay_len; i += blockDim.x) s_decay[i] = p.lut_decay[i];
    for (int i = threadIdx.x; i < p.T; i += blockDim.x) s_th[i] = p.lut_th[i];
    __syncthreads();

    const long long gw = (long long)blockIdx.x * SW + warp;
    if (gw >= n_warps) return;                            // warp-uniform
    const long long pix = gw / groups;
    const int grp = (int)(gw - pix * groups);
    const int c0 = (grp * 32 + lane) * V;
    const bool lane_ok = c0 < p.C_out;

    int w_out = 0, h_out = 0;
    long long img = pix;
    if (!p.is_fc) {
        w_out = (int)(pix % p.W_out);
        const long long r = pix / p.W_out;
        h_out = (int)(r % p.H_out);
        img = r / p.H_out;
    }
    const int FS = p.T + 1;                               // fine offsets per column
    long long my_col = -1;
    if (lane < ntaps) {
        if (p.is_fc) {
            my_col = img;
        } else {
            const int kh = lane / p.K, kw = lane - (lane / p.K) * p.K;
            const int h_in = h_out - p.pad + kh, w_in = w_out - p.pad + kw;
            if (h_in >= 0 && h_in < p.H_in && w_in >= 0 && w_in < p.W_in)
                my_col = (img * p.H_in + h_in) * p.W_in + w_in;
        }
    }
    const int* fo = my_col >= 0 ? foff + my_col * FS : nullptr;

    Neurons<V> nu;
#pragma unroll
    for (int v = 0; v < V; ++v) {
        nu.carry[v] = lane_ok ? __ldg(p.bias + c0 + v) : 0.0f;
        nu.res[v] = p.inf_time;
        nu.acc[v] = 0.0f;
        nu.alive[v] = lane_ok;
    }
    unsigned long long fetched = 0;
    const float* Wl = p.W + (lane_ok ? c0 : 0);

    // fine offsets of the next chunk, one chunk ahead
    int onx[DELTA + 1];
#pragma unroll
    for (int i = 0; i <= DELTA; ++i) onx[i] = (fo && i <= p.T) ? __ldg(fo + min(i, p.T)) : 0;

    bool done = false;
    for (int tau = 0; tau < p.NC && !done; ++tau) {
        const int base = tau * DELTA;
        const int steps = min(DELTA, p.T - base);
        int o[DELTA + 1];
#pragma unroll
        for (int i = 0; i <= DELTA; ++i) o[i] = onx[i];
        if (tau + 1 < p.NC) {
#pragma unroll
            for (int i = 0; i <= DELTA; ++i) {
                const int t = base + DELTA + i;
                onx[i] = (fo && t <= p.T) ? __ldg(fo + t) : 0;
            }
        }
        // stream layout: cell (s, j) in step-major order
        int run = 0;
#pragma unroll
        for (int s = 0; s < DELTA; ++s) {
            const int c = (s < steps && fo) ? o[s + 1] - o[s] : 0;
            int inc = c;
#pragma unroll
            for (int dd = 1; dd < 32; dd <<= 1) {
                const int u = __shfl_up_sync(FULL, inc, dd);
                if (lane >= dd) inc += u;
            }
            if (lane < ntaps) { s_P[s * ntaps + lane] = run + inc - c; s_O[s * ntaps + lane] = o[s]; }
            run += __shfl_sync(FULL, inc, 31);
        }
        const int total = run;
        int n_live = 0;
#pragma unroll
        for (int v = 0; v < V; ++v) n_live += nu.alive[v] ? 1 : 0;
        if (p.fetched) fetched += (unsigned long long)total * n_live;
        __syncwarp();

        int cur = base;                                   // first step not closed yet
        bool has_acc = false;
        for (int p0 = 0; p0 < total && !done; p0 += 32) {
            // decode event p0 + lane of the stream
            SEv ev{-1, 0, 0.0f};
            const int pos = p0 + lane;
            if (pos < total) {
                int lo = 0, hi = cells - 1;
                while (lo < hi) {
                    const int mid = (lo + hi + 1) >> 1;
                    if (s_P[mid] <= pos) lo = mid; else hi = mid - 1;
                }
                const int s = lo / ntaps, j = lo - s * ntaps;
                long long col;
                if (p.is_fc) {
                    col = img;
                } else {
                    const int kh = j / p.K, kw = j - kh * p.K;
                    col = (img * p.H_in + (h_out - p.pad + kh)) * p.W_in + (w_out - p.pad + kw);
                }
                const long long at = col * p.C_in + s_O[lo] + (pos - s_P[lo]);
                const int ci = __ldg(p.cin + at);
                int ti;
                if (p.lut_mode == VDT_LUT_BY_TB) {
                    ti = base + s;
                } else {
                    const float t = __ldg(p.tin + at);
                    ti = (int)t;
                    ti = ti < 0 ? 0 : (ti > p.T ? p.T : ti);
                }
                ev.step = base + s;
                ev.lv = s_decay[ti];
                ev.wo = ((p.is_fc ? 0 : j * p.C_in) + ci) * p.C_out;
            }
            const int nb = min(32, total - p0);
            bool lane_live = false;
#pragma unroll
            for (int v = 0; v < V; ++v) lane_live |= nu.alive[v];

            float wa[EBS][V], wb[EBS][V];
            auto fetch = [&](float (&w)[EBS][V], int q0) {
#pragma unroll
                for (int u = 0; u < EBS; ++u) {
                    const int woq = __shfl_sync(FULL, ev.wo, (q0 + u) & 31);
                    if (lane_live && q0 + u < nb) {
                        ldv<V>(Wl + woq, w[u]);
                    } else {
#pragma unroll
                        for (int v = 0; v < V; ++v) w[u][v] = 0.0f;
                    }
                }
            };
            auto apply = [&](const float (&w)[EBS][V], int q0) {
#pragma unroll
                for (int u = 0; u < EBS; ++u) {
                    const int st = __shfl_sync(FULL, ev.step, (q0 + u) & 31);
                    const float lq = __shfl_sync(FULL, ev.lv, (q0 + u) & 31);
                    if (q0 + u < nb) {
                        if (st != cur) {                   // a new step begins
                            nu.close(cur, st, s_th, p.t_min, has_acc);
                            cur = st;
                        }
                        has_acc = true;
#pragma unroll
                        for (int v = 0; v < V; ++v) nu.acc[v] = fmaf(w[u][v], lq, nu.acc[v]);
                    }
                }
            };
            fetch(wa, 0);
            for (int q0 = 0; q0 < nb; q0 += 2 * EBS) {
                if (q0 + EBS < nb) fetch(wb, q0 + EBS);
                apply(wa, q0);
                if (q0 + 2 * EBS < nb) fetch(wa, q0 + 2 * EBS);
                if (q0 + EBS < nb) apply(wb, q0 + EBS);
            }
            // every neuron of the warp fired: stop fetching synapses
            bool any = false;
#pragma unroll
            for (int v = 0; v < V; ++v) any |= nu.alive[v];
            if (!__any_sync(FULL, any)) done = true;
        }
        __syncwarp();
        if (!done) {
            nu.close(cur, base + steps, s_th, p.t_min, has_acc);
            bool any = false;
#pragma unroll
            for (int v = 0; v < V; ++v) any |= nu.alive[v];
            if (!__any_sync(FULL, any)) done = true;
        }
    }
    if (lane_ok) stv<V>(p.out + pix * p.C_out + c0, nu.res);
    if (p.fetched) {
#pragma unroll
        for (int dd = 16; dd > 0; dd >>= 1) fetched += __shfl_down_sync(FULL, fetched, dd);
        if (lane == 0 && fetched) atomicAdd(p.fetched, fetched);
    }
}

int pick_vs(int C_out) {
    if (C_out % 4 == 0 && C_out >= 128) return 4;
    if (C_out % 2 == 0 && C_out >= 64) return 2;
    return 1;
}

template <int DELTA, int V>
cudaError_t launch_sv(const IntegParams& p, const int* foff, cudaStream_t s, long long n_warps, int groups) {
    const int ntaps = p.is_fc ? 1 : p.K * p.K;
    const size_t smem = (size_t)SW * 2 * DELTA * ntaps * sizeof(int) + (size_t)(p.decay_len + p.T) * sizeof(float);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(k_stream<DELTA, V>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    const long long blocks = (n_warps + SW - 1) / SW;
    k_stream<DELTA, V><<<(unsigned)blocks, SW * 32, smem, s>>>(p, foff, n_warps, groups);
    return cudaGetLastError();
}

template <int DELTA>
cudaError_t launch_sd(const IntegParams& p, const int* foff, cudaStream_t s) {
    int V = pick_vs(p.C_out);
    if (DELTA > 8 && V == 4) V = 2;          // keep o[]/onx[] + weights in registers
    const int groups = (p.C_out + 32 * V - 1) / (32 * V);
    const long long pixels = p.is_fc ? (long long)p.B : (long long)p.B * p.H_out * p.W_out;
    const long long n_warps = pixels * groups;
    if (n_warps <= 0) return cudaSuccess;
    switch (V) {
        case 4: return launch_sv<DELTA, (DELTA > 8 ? 2 : 4)>(p, foff, s, n_warps, groups);
        case 2: return launch_sv<DELTA, 2>(p, foff, s, n_warps, groups);
        default: return launch_sv<DELTA, 1>(p, foff, s, n_warps, groups);
    }
}

}  // namespace

bool stream_supported(int K, int is_fc, int delta, int T, int decay_len) {
    const int ntaps = is_fc ? 1 : K * K;
    if (ntaps > 32) return false;
    if (delta != 4 && delta != 8 && delta != 16) return false;
    return (size_t)SW * 2 * delta * ntaps * sizeof(int) + (size_t)(decay_len + T) * sizeof(float) <= 200 * 1024;
}

cudaError_t launch_stream(const IntegParams& p, const int* foff, cudaStream_t s) {
    switch (p.delta) {
        case 4: return launch_sd<4>(p, foff, s);
        case 8: return launch_sd<8>(p, foff, s);
        case 16: return launch_sd<16>(p, foff, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace vdt
