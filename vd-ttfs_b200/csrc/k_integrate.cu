// k_integrate.cu -- the chunked early-exit integrator (the reference's
// k_conv_bucketed, t1:83-162 / t2:84-170) for sm_100a.
//
// Work mapping.  One warp integrates one output pixel for 32*V consecutive
// output channels: lane l owns channels c0 = (group*32 + l)*V .. c0+V-1, so a
// synaptic event's weight row W[(tap*C_in + cin)*C_out + c0 ..] is one
// coalesced V-wide vector load per lane (512 B per warp at V = 4), and all
// lanes share the pixel's events.
//
// Per chunk tau (width DELTA):
//   * lanes 0..ntaps-1 fetch the [start, end) offsets of their tap's input
//     column in one coalesced step;
//   * per tap, events are read 32 at a time, one per lane (cin, t_in ->
//     slot = tb - tau*DELTA, LUT_decay value from shared memory, weight-row
//     offset);
//   * the batch is then consumed slot by slot: for each (unrolled) slot s,
//     __ballot_sync gives the lanes whose event falls in s, and those events
//     are applied in lane order with one vector weight load + V FFMAs into
//     delta[s][*].  `s` is a compile-time index, so delta[DELTA][V] stays in
//     registers (the reference's dynamically indexed delta[CHUNK] spills to
//     local memory at CHUNK = 16).
//   Within a slot, events are applied in (tap, bucket position) order -- the
//   reference's order -- and each delta[s] is the same chain of fmaf(W, LUT,
//   delta) the reference's `delta[tb - base_t] += kernel[..] * LUT_decay[ti]`
//   compiles to, so results are bit-identical.
//   * the threshold scan then adds delta[i] to the carry step by step and
//     records the first t >= t_min with carry >= LUT_th[t] >= 1e-5
//     (t1:150-157, t2:158-165);
//   * __any_sync over the lanes' live neurons ends the warp's chunk loop as
//     soon as every neuron fired: later chunks (and their synapses) are never
//     fetched.  Lanes whose neurons all fired stop issuing weight loads.
//
// LUT_decay / LUT_th are staged in shared memory once per CTA.
#include "vdt_internal.h"

namespace vdt {
namespace {

constexpr unsigned FULL = 0xffffffffu;

template <int V> struct VecT;
template <> struct VecT<1> { typedef float type; };
template <> struct VecT<2> { typedef float2 type; };
template <> struct VecT<4> { typedef float4 type; };

template <int V>
__device__ __forceinline__ void load_vec(const float* p, float (&w)[V]) {
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
__device__ __forceinline__ void store_vec(float* p, const float (&r)[V]) {
    if constexpr (V == 1) {
        *p = r[0];
    } else if constexpr (V == 2) {
        *reinterpret_cast<float2*>(p) = make_float2(r[0], r[1]);
    } else {
        *reinterpret_cast<float4*>(p) = make_float4(r[0], r[1], r[2], r[3]);
    }
}

template <int DELTA, int V>
__global__ void __launch_bounds__(256, 2) k_integrate(IntegParams p, long long n_warps, int groups) {
    extern __shared__ float s_lut[];
    float* s_decay = s_lut;
    float* s_th = s_lut + p.decay_len;
    for (int i = threadIdx.x; i < p.decay_len; i += blockDim.x) s_decay[i] = p.lut_decay[i];
    for (int i = threadIdx.x; i < p.T; i += blockDim.x) s_th[i] = p.lut_th[i];
    __syncthreads();

    const int lane = threadIdx.x & 31;
    const long long gw = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (gw >= n_warps) return;                        // warp-uniform
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
    const int ntaps = p.is_fc ? 1 : p.K * p.K;
    const int OS = p.NC + 1;

    // lane j < ntaps owns tap j's input column (or none if out of range)
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

    float carry[V], res[V];
    bool alive[V];
#pragma unroll
    for (int v = 0; v < V; ++v) {
        carry[v] = lane_ok ? __ldg(p.bias + c0 + v) : 0.0f;
        res[v] = p.inf_time;
        alive[v] = lane_ok;
    }
    unsigned long long fetched = 0;
    const float* Wl = p.W + (lane_ok ? c0 : 0);

    for (int tau = 0; tau < p.NC; ++tau) {
        const int base = tau * DELTA;
        float d[DELTA][V];
#pragma unroll
        for (int i = 0; i < DELTA; ++i)
#pragma unroll
            for (int v = 0; v < V; ++v) d[i][v] = 0.0f;

        int n_live = 0;
#pragma unroll
        for (int v = 0; v < V; ++v) n_live += alive[v] ? 1 : 0;
        const bool lane_live = n_live > 0;

        int my_s = 0, my_e = 0;
        if (my_col >= 0) {
            const int* o = p.off + my_col * OS + tau;
            my_s = __ldg(o);
            my_e = __ldg(o + 1);
        }
        for (int j = 0; j < ntaps; ++j) {
            const int s = __shfl_sync(FULL, my_s, j);
            const int e = __shfl_sync(FULL, my_e, j);
            if (s >= e) continue;                     // warp-uniform
            const long long col = p.is_fc ? img
                : (img * p.H_in + (h_out - p.pad + j / p.K)) * p.W_in + (w_out - p.pad + j % p.K);
            const int wrow0 = p.is_fc ? 0 : j * p.C_in;
            const int* bc = p.cin + col * p.C_in;
            const float* bt = p.tin + col * p.C_in;
            for (int p0 = s; p0 < e; p0 += 32) {
                const int idx = p0 + lane;
                int slot = -1, wo = 0;
                float lv = 0.0f;
                if (idx < e) {
                    const int ci = __ldg(bc + idx);
                    const float t = __ldg(bt + idx);
                    int tb = (int)floorf(t - p.tfs);
                    if (tb < 0) tb = 0;
                    int ti;
                    if (p.lut_mode == VDT_LUT_BY_TB) {
                        ti = tb;
                    } else {
                        ti = (int)t;
                        ti = ti < 0 ? 0 : (ti > p.T ? p.T : ti);
                    }
                    slot = tb - base;
                    lv = s_decay[ti];
                    wo = (wrow0 + ci) * p.C_out;
                }
                if (p.fetched) fetched += (unsigned long long)__popc(__ballot_sync(FULL, idx < e)) * n_live;
#pragma unroll
                for (int sl = 0; sl < DELTA; ++sl) {
                    unsigned m = __ballot_sync(FULL, slot == sl);
                    while (m) {
                        const int q = __ffs(m) - 1;
                        m &= m - 1;
                        const int woq = __shfl_sync(FULL, wo, q);
                        const float lq = __shfl_sync(FULL, lv, q);
                        float w[V];
                        if (lane_live) {
                            load_vec<V>(Wl + woq, w);
                        } else {
#pragma unroll
                            for (int v = 0; v < V; ++v) w[v] = 0.0f;
                        }
#pragma unroll
                        for (int v = 0; v < V; ++v) d[sl][v] = fmaf(w[v], lq, d[sl][v]);
                    }
                }
            }
        }
        // integrate this chunk; first crossing wins (t1:150-157, t2:158-165)
#pragma unroll
        for (int i = 0; i < DELTA; ++i) {
            const int t = base + i;
            if (t < p.T) {
                const float th = s_th[t];
#pragma unroll
                for (int v = 0; v < V; ++v) {
                    if (alive[v]) {
                        carry[v] += d[i][v];
                        if (t >= p.t_min && carry[v] >= th && th >= 1e-5f) {
                            res[v] = (float)t;
                            alive[v] = false;
                        }
                    }
                }
            }
        }
        bool any_alive = false;
#pragma unroll
        for (int v = 0; v < V; ++v) any_alive |= alive[v];
        if (!__any_sync(FULL, any_alive)) break;
    }
    if (lane_ok) store_vec<V>(p.out + pix * p.C_out + c0, res);
    if (p.fetched) {
#pragma unroll
        for (int dd = 16; dd > 0; dd >>= 1) fetched += __shfl_down_sync(FULL, fetched, dd);
        if (lane == 0 && fetched) atomicAdd(p.fetched, fetched);
    }
}

// V (output channels per lane) for a layer: the widest of 4/2/1 that divides
// C_out and keeps the per-lane delta[DELTA][V] block at <= 64 registers.
int pick_v(int C_out, int delta) {
    if (C_out % 4 == 0 && C_out >= 128 && delta * 4 <= 64) return 4;
    if (C_out % 2 == 0 && C_out >= 64 && delta * 2 <= 64) return 2;
    return 1;
}

template <int DELTA>
cudaError_t launch_delta(const IntegParams& p, cudaStream_t s) {
    const int V = pick_v(p.C_out, DELTA);
    const int groups = (p.C_out + 32 * V - 1) / (32 * V);
    const long long pixels = p.is_fc ? (long long)p.B : (long long)p.B * p.H_out * p.W_out;
    const long long n_warps = pixels * groups;
    if (n_warps <= 0) return cudaSuccess;
    const int warps_per_cta = 8;
    const long long blocks = (n_warps + warps_per_cta - 1) / warps_per_cta;
    const size_t smem = (size_t)(p.decay_len + p.T) * sizeof(float);
    switch (V) {
        case 4: k_integrate<DELTA, (DELTA <= 16 ? 4 : 1)><<<(unsigned)blocks, 256, smem, s>>>(p, n_warps, groups); break;
        case 2: k_integrate<DELTA, (DELTA <= 32 ? 2 : 1)><<<(unsigned)blocks, 256, smem, s>>>(p, n_warps, groups); break;
        default: k_integrate<DELTA, 1><<<(unsigned)blocks, 256, smem, s>>>(p, n_warps, groups); break;
    }
    return cudaGetLastError();
}

}  // namespace

bool integrate_supported(int K, int is_fc, int delta, int C_out, int T, int decay_len) {
    if (!is_fc && (K < 1 || K * K > 32)) return false;
    if (delta != 1 && delta != 2 && delta != 4 && delta != 8 && delta != 16 && delta != 32 && delta != 64)
        return false;
    if ((size_t)(decay_len + T) * sizeof(float) > 48 * 1024) return false;
    return C_out > 0;
}

cudaError_t launch_integrate(const IntegParams& p, cudaStream_t s) {
    switch (p.delta) {
        case 1: return launch_delta<1>(p, s);
        case 2: return launch_delta<2>(p, s);
        case 4: return launch_delta<4>(p, s);
        case 8: return launch_delta<8>(p, s);
        case 16: return launch_delta<16>(p, s);
        case 32: return launch_delta<32>(p, s);
        case 64: return launch_delta<64>(p, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace vdt
