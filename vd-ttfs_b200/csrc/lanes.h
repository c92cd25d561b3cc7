// lanes.h -- per-lane neuron state shared by the integrators (k_dense,
// k_sorted): V output channels per lane, the membrane carry, the open step's
// accumulator and the first-spike result.
//
// Step semantics follow k_conv_bucketed (t1:150-157, t2:158-165): at the end
// of step s the step's input (a per-step FMA chain, accumulated in `acc`) is
// added to the carry with one separate add, and the neuron fires at s if
// s >= t_min, LUT_th[s] >= 1e-5 and carry >= LUT_th[s].
#pragma once

#include "vdt_internal.h"

namespace vdt {

constexpr unsigned FULL_MASK = 0xffffffffu;

// Staged threshold tables: s_th = LUT_th, s_thx = LUT_th where a spike may be
// recorded (s >= t_min and LUT_th >= 1e-5), NaN elsewhere (every comparison
// with NaN is false); t_floor = first step with LUT_th < 1e-5 (or T) and
// monotone = thresholds non-increasing.  Built by the whole CTA.
struct ThTables {
    const float* th;
    const float* thx;
    int t_min, t_floor;
    bool monotone;
};

__device__ __forceinline__ ThTables stage_thresholds(const IntegParams& p, float* s_th, float* s_thx,
                                                     int* s_floor, int* s_mono) {
    for (int i = threadIdx.x; i < p.T; i += blockDim.x) {
        const float th = p.lut_th[i];
        s_th[i] = th;
        s_thx[i] = (i >= p.t_min && th >= 1e-5f) ? th : __int_as_float(0x7fffffff);
    }
    if (threadIdx.x == 0) { *s_floor = p.T; *s_mono = 1; }
    __syncthreads();
    for (int t = threadIdx.x; t < p.T; t += blockDim.x) {
        if (!(s_th[t] >= 1e-5f)) atomicMin(s_floor, t);
        if (t + 1 < p.T && !(s_th[t + 1] <= s_th[t])) *s_mono = 0;
    }
    __syncthreads();
    return ThTables{s_th, s_thx, p.t_min, *s_floor, *s_mono != 0};
}

template <int V>
struct Lanes {
    float carry[V], res[V], acc[V];
    bool alive[V];

    __device__ __forceinline__ void init(const float* bias, int c0, bool lane_ok, float inf_time) {
#pragma unroll
        for (int v = 0; v < V; ++v) {
            carry[v] = lane_ok ? __ldg(bias + c0 + v) : 0.0f;
            res[v] = inf_time;
            acc[v] = 0.0f;
            alive[v] = lane_ok;
        }
    }
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
    __device__ __forceinline__ void fma(const float (&w)[V], float lv) {
#pragma unroll
        for (int v = 0; v < V; ++v) acc[v] = fmaf(w[v], lv, acc[v]);
    }
    // end of step s with input: carry += acc, threshold test, acc = 0
    __device__ __forceinline__ void close_step(int s, const ThTables& tt) {
        const float th = tt.thx[s];
#pragma unroll
        for (int v = 0; v < V; ++v) {
            if (alive[v]) {
                carry[v] += acc[v];
                if (carry[v] >= th) {
                    res[v] = (float)s;
                    alive[v] = false;
                }
            }
            acc[v] = 0.0f;
        }
    }
    // branch-free forms of the two closes (no per-lane divergence): a dead
    // neuron's carry is never read again, so it is updated unconditionally
    __device__ __forceinline__ void close_step_bf(int s, const ThTables& tt) {
        const float th = tt.thx[s];
#pragma unroll
        for (int v = 0; v < V; ++v) {
            carry[v] += acc[v];
            const bool fire = alive[v] && carry[v] >= th;
            res[v] = fire ? (float)s : res[v];
            alive[v] = alive[v] && !fire;
            acc[v] = 0.0f;
        }
    }
    // steps [a, b) without input, non-increasing thresholds: the first step
    // t in [lo, hi) with carry >= LUT_th[t] by a bisection whose trip count
    // depends only on the (warp-uniform) run length
    __device__ __forceinline__ void close_empty_bf(int a, int b, const ThTables& tt) {
        if (a >= b) return;
        if (!tt.monotone) { close_empty(a, b, tt); return; }
        const int lo = max(a, tt.t_min), hi = min(b, tt.t_floor);
        if (lo >= hi) return;
        const float mn = tt.th[hi - 1];
        int top = 1;
        while (top * 2 <= hi - lo) top *= 2;
#pragma unroll
        for (int v = 0; v < V; ++v) {
            // pos = last step in [lo - 1, hi - 1) whose threshold is above the carry
            int pos = lo - 1;
            for (int step = top; step > 0; step >>= 1) {
                const int q = pos + step;
                pos = (q < hi && tt.th[q] > carry[v]) ? q : pos;
            }
            const bool fire = alive[v] && carry[v] >= mn;
            res[v] = fire ? (float)(pos + 1) : res[v];
            alive[v] = alive[v] && !fire;
        }
    }
    // steps [a, b) without input: the carry is constant, so with
    // non-increasing thresholds a neuron fires in the run iff it reaches the
    // run's last valid threshold, at the first step found by bisection
    __device__ __forceinline__ void close_empty(int a, int b, const ThTables& tt) {
        if (a >= b) return;
        if (tt.monotone) {
            const int lo = max(a, tt.t_min), hi = min(b, tt.t_floor);
            if (lo >= hi) return;
            const float mn = tt.th[hi - 1];
#pragma unroll
            for (int v = 0; v < V; ++v) {
                if (alive[v] && carry[v] >= mn) {
                    int l = lo, h = hi - 1;
                    while (l < h) {
                        const int mid = (l + h) >> 1;
                        if (carry[v] >= tt.th[mid]) h = mid; else l = mid + 1;
                    }
                    res[v] = (float)l;
                    alive[v] = false;
                }
            }
        } else {
            for (int t = a; t < b; ++t) {
                const float th = tt.thx[t];
#pragma unroll
                for (int v = 0; v < V; ++v)
                    if (alive[v] && carry[v] >= th) {
                        res[v] = (float)t;
                        alive[v] = false;
                    }
            }
        }
    }
};

// CuLIF neurons of task 3 (conv_bucketed_early t3:109-143, fc2_bucketed_early
// t3:203-225): every step t updates I = fma(I, decay, in[t]); V += I and the
// neuron fires at the first t with V >= th.  A step without input has
// in[t] = 0, so no step can be skipped.
struct CulifCfg {
    float decay, th;
};

template <int V>
struct CulifLanes {
    float I[V], Vm[V], res[V], acc[V];
    bool alive[V];

    __device__ __forceinline__ void init(bool lane_ok, float inf_time) {
#pragma unroll
        for (int v = 0; v < V; ++v) {
            I[v] = 0.0f;
            Vm[v] = 0.0f;
            res[v] = inf_time;
            acc[v] = 0.0f;
            alive[v] = lane_ok;
        }
    }
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
    __device__ __forceinline__ void step(int s, float in, int v, const CulifCfg& c) {
        I[v] = fmaf(I[v], c.decay, in);
        Vm[v] += I[v];
        const bool fire = alive[v] && Vm[v] >= c.th;
        res[v] = fire ? (float)s : res[v];
        alive[v] = alive[v] && !fire;
    }
    // step s of every channel with inputs in[]: channel pairs update I and V
    // with packed fma.rn.f32x2 / add.rn.f32x2 (two independent
    // round-to-nearest operations, the same results as fmaf and +)
    __device__ __forceinline__ void step_all(int s, const float (&in)[V], const CulifCfg& c) {
#pragma unroll
        for (int v = 0; v + 1 < V; v += 2) {
            asm("{\n\t"
                ".reg .b64 i, d, x, m;\n\t"
                "mov.b64 i, {%0, %1};\n\t"
                "mov.b64 d, {%4, %4};\n\t"
                "mov.b64 x, {%5, %6};\n\t"
                "fma.rn.f32x2 i, i, d, x;\n\t"
                "mov.b64 m, {%2, %3};\n\t"
                "add.rn.f32x2 m, m, i;\n\t"
                "mov.b64 {%0, %1}, i;\n\t"
                "mov.b64 {%2, %3}, m;\n\t"
                "}"
                : "+f"(I[v]), "+f"(I[v + 1]), "+f"(Vm[v]), "+f"(Vm[v + 1])
                : "f"(c.decay), "f"(in[v]), "f"(in[v + 1]));
        }
        if constexpr (V % 2 == 1) {
            I[V - 1] = fmaf(I[V - 1], c.decay, in[V - 1]);
            Vm[V - 1] += I[V - 1];
        }
#pragma unroll
        for (int v = 0; v < V; ++v) {
            const bool fire = alive[v] && Vm[v] >= c.th;
            res[v] = fire ? (float)s : res[v];
            alive[v] = alive[v] && !fire;
        }
    }
    // step s with input acc (the step's in[] sum), then acc = 0
    __device__ __forceinline__ void close_step_bf(int s, const CulifCfg& c) {
        step_all(s, acc, c);
#pragma unroll
        for (int v = 0; v < V; ++v) acc[v] = 0.0f;
    }
    // steps [a, b) without input
    __device__ __forceinline__ void close_empty(int a, int b, const CulifCfg& c) {
        float zero[V];
#pragma unroll
        for (int v = 0; v < V; ++v) zero[v] = 0.0f;
        for (int t = a; t < b; ++t) step_all(t, zero, c);
    }
};

template <int V>
__device__ __forceinline__ void load_row(const float* p, float (&w)[V]);

// one record {weight offset, LUT value} from a 32-bit shared-memory address
__device__ __forceinline__ int2 lds_rec(unsigned sa) {
    int2 e;
    asm volatile("ld.shared.v2.s32 {%0, %1}, [%2];" : "=r"(e.x), "=r"(e.y) : "r"(sa));
    return e;
}

// acc[v] = fma(w[v], lv, acc[v]) for every v; pairs use the packed
// fma.rn.f32x2 (two independent round-to-nearest fp32 FMAs, the same
// results as two fmaf calls)
template <int V>
__device__ __forceinline__ void fma_lanes(float (&acc)[V], const float (&w)[V], float lv) {
    if constexpr (V == 1) {
        acc[0] = fmaf(w[0], lv, acc[0]);
    } else {
#pragma unroll
        for (int v = 0; v < V; v += 2) {
            asm("{\n\t"
                ".reg .b64 a, b, c;\n\t"
                "mov.b64 a, {%0, %1};\n\t"
                "mov.b64 b, {%2, %3};\n\t"
                "mov.b64 c, {%4, %4};\n\t"
                "fma.rn.f32x2 a, b, c, a;\n\t"
                "mov.b64 {%0, %1}, a;\n\t"
                "}"
                : "+f"(acc[v]), "+f"(acc[v + 1])
                : "f"(w[v]), "f"(w[v + 1]), "f"(lv));
        }
    }
}

// U records {element offset of the event's weight row, LUT value bits}:
// U weight loads in flight, then the U FMAs of each neuron's chain in order
template <int V, int U>
__device__ __forceinline__ void stream_block(Lanes<V>& nu, const int2* rec, const float* Wl) {
    int2 e[U];
    float w[U][V];
#pragma unroll
    for (int u = 0; u < U; ++u) e[u] = rec[u];
#pragma unroll
    for (int u = 0; u < U; ++u) load_row<V>(Wl + (unsigned)e[u].x, w[u]);
#pragma unroll
    for (int u = 0; u < U; ++u) fma_lanes<V>(nu.acc, w[u], __int_as_float(e[u].y));
}

// the same from a 32-bit shared address (no generic-pointer arithmetic)
template <int V, int U, class L>
__device__ __forceinline__ void stream_block_sa(L& nu, unsigned sa, const float* Wl) {
    int2 e[U];
    float w[U][V];
#pragma unroll
    for (int u = 0; u < U; ++u) e[u] = lds_rec(sa + 8u * u);
#pragma unroll
    for (int u = 0; u < U; ++u) load_row<V>(Wl + (unsigned)e[u].x, w[u]);
#pragma unroll
    for (int u = 0; u < U; ++u) fma_lanes<V>(nu.acc, w[u], __int_as_float(e[u].y));
}

// The records [k, end) of one run: full blocks of FS records without any
// test, then the tail (fewer than FS records) as one block of its exact
// size, reached by a switch (one indexed jump instead of a test per
// power-of-two piece).
template <int V, int FS, class L>
__device__ __forceinline__ void stream_run_records(L& nu, unsigned sa0, int k, int end, const float* Wl) {
    static_assert(FS >= 1 && FS <= 8, "a run's tail (< FS records) is covered by blocks of 1 to 7");
    for (; k + FS <= end; k += FS) stream_block_sa<V, FS>(nu, sa0 + 8u * k, Wl);
    switch (end - k) {
        case 7: stream_block_sa<V, 7>(nu, sa0 + 8u * k, Wl); break;
        case 6: stream_block_sa<V, 6>(nu, sa0 + 8u * k, Wl); break;
        case 5: stream_block_sa<V, 5>(nu, sa0 + 8u * k, Wl); break;
        case 4: stream_block_sa<V, 4>(nu, sa0 + 8u * k, Wl); break;
        case 3: stream_block_sa<V, 3>(nu, sa0 + 8u * k, Wl); break;
        case 2: stream_block_sa<V, 2>(nu, sa0 + 8u * k, Wl); break;
        case 1: stream_block_sa<V, 1>(nu, sa0 + 8u * k, Wl); break;
        default: break;
    }
}

// Stream step-sorted records through their runs: runs[j] = {end index of
// run j in rec, its step}, runs in increasing step order, the records of one
// run in FMA-chain order.  Each run ends with the close of its step
// (input-free steps before it are closed first).  Returns false once every
// neuron of the warp has fired (the caller may stop).
template <int V, int FS, class L, class TT>
__device__ __forceinline__ bool stream_runs(L& nu, const int2* rec, int k, const int2* runs,
                                            int nruns, const float* Wl, int& next_t,
                                            const TT& tt) {
    const unsigned sa0 = (unsigned)__cvta_generic_to_shared(rec);
    for (int j = 0; j < nruns; ++j) {
        const int2 rn = runs[j];
        stream_run_records<V, FS>(nu, sa0, k, rn.x, Wl);
        k = rn.x;
        nu.close_empty(next_t, rn.y, tt);
        nu.close_step_bf(rn.y, tt);
        next_t = rn.y + 1;
        if (!__any_sync(FULL_MASK, nu.any())) return false;
    }
    return true;
}

// The same for several pixels per warp: each lane follows its own pixel's
// records and runs (rec, runs, nruns differ between lane groups); jmax is
// the warp's largest run count.  The groups share one pass of the run loop;
// the all-fired vote is taken by the whole warp once per run index.
template <int V, int FS, class L, class TT>
__device__ __forceinline__ bool stream_runs_grouped(L& nu, const int2* rec, const int2* runs, int nruns,
                                                    int jmax, const float* Wl, int& next_t, const TT& tt) {
    const unsigned sa0 = (unsigned)__cvta_generic_to_shared(rec);
    int k = 0;
    for (int j = 0; j < jmax; ++j) {
        if (j < nruns) {
            const int2 rn = runs[j];
            stream_run_records<V, FS>(nu, sa0, k, rn.x, Wl);
            k = rn.x;
            nu.close_empty(next_t, rn.y, tt);
            nu.close_step_bf(rn.y, tt);
            next_t = rn.y + 1;
        }
        if (!__any_sync(FULL_MASK, nu.any())) return false;
    }
    return true;
}

// Compact the non-empty bins into runs: bins [0, nb) with exclusive ends
// end[b] (start of bin b = end[b - 1], 0 for b = 0); runs[j] = {end, base + b}.
// Returns the number of runs.  Whole warp.
__device__ __forceinline__ int compact_runs(const int* end, int nb, int base, int2* runs) {
    const int lane = threadIdx.x & 31;
    const unsigned lt = (1u << lane) - 1u;
    int n = 0;
    for (int b0 = 0; b0 < nb; b0 += 32) {
        const int b = b0 + lane;
        bool ne = false;
        int e = 0;
        if (b < nb) {
            e = end[b];
            ne = e > (b == 0 ? 0 : end[b - 1]);
        }
        const unsigned m = __ballot_sync(FULL_MASK, ne);
        if (ne) runs[n + __popc(m & lt)] = make_int2(e, base + b);
        n += __popc(m);
    }
    __syncwarp();
    return n;
}

template <int V>
__device__ __forceinline__ void load_row(const float* p, float (&w)[V]) {
    if constexpr (V == 1) {
        w[0] = __ldg(p);
    } else if constexpr (V == 2) {
        const float2 v = __ldg(reinterpret_cast<const float2*>(p));
        w[0] = v.x; w[1] = v.y;
    } else {
        static_assert(V == 4, "V is 1, 2 or 4");
        const float4 v = __ldg(reinterpret_cast<const float4*>(p));
        w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
    }
}

// The layer's 2x2 min pool fused into its integrator (k_pool_min's result,
// t1:164-181 / t2:192-209): output pixel (img, h, w) takes part in pooled
// cell (h / 2, w / 2) -- none if it lies in the last row or column of an odd
// map -- by an integer min on the float bits of its V results.  Spike times
// and the no-spike time are non-negative, so their bits order like their
// values; the cell starts at the bytes 0x7F (about 3.4e38, above every time)
// and ends as the minimum of its four outputs, which is what k_pool_min
// writes (its start value, the no-spike time, is never below them).
template <int V>
__device__ __forceinline__ void pool_store(float* pooled, long long img, int h, int w, int H, int W, int C,
                                           int c0, const float (&r)[V]) {
    const int Hp = H >> 1, Wp = W >> 1;
    if ((h >> 1) >= Hp || (w >> 1) >= Wp) return;
    int* dst = reinterpret_cast<int*>(pooled) + ((img * Hp + (h >> 1)) * Wp + (w >> 1)) * (long long)C + c0;
#pragma unroll
    for (int v = 0; v < V; ++v) atomicMin(dst + v, __float_as_int(r[v]));
}

template <int V>
__device__ __forceinline__ void store_res(float* p, const float (&r)[V]) {
    if constexpr (V == 1) {
        *p = r[0];
    } else if constexpr (V == 2) {
        *reinterpret_cast<float2*>(p) = make_float2(r[0], r[1]);
    } else {
        *reinterpret_cast<float4*>(p) = make_float4(r[0], r[1], r[2], r[3]);
    }
}

}  // namespace vdt
