// k_sorted.cu -- chunked early-exit integrator with per-chunk slot sorting
// (same contract and bit-identical results as k_conv_bucketed, t1:83-162 /
// t2:84-170; input: the reference bucket layout).
//
// One warp integrates one output pixel for 32*V output channels (lane l owns
// channels (group*32 + l)*V .. +V-1, so each synaptic event's weight row is a
// coalesced V-wide load).  For each chunk tau with input:
//   1. decode (event-parallel, one event per lane): the chunk's events of all
//      taps, in tap order and bucket order -- the reference's FMA-chain order --
//      become {weight row = tap*C_in + cin, slot = tb - tau*DELTA, LUT_decay}
//      records in shared memory, and a warp-aggregated histogram counts them
//      per slot (__match_any_sync, one shared-memory add per distinct slot);
//   2. an exclusive scan turns the counts into slot offsets, and a stable
//      scatter (rank = popc(group & lanemask_lt)) groups the records by slot,
//      keeping their chain order inside each slot;
//   3. a loop over the slots, unrolled so every delta[slot] index is a
//      compile-time constant (registers, no dispatch), streams each slot's run:
//      per event one broadcast LDS.64, one weight load, V FMAs
//          delta[slot] = fmaf(W[row][c], LUT_decay[ti], delta[slot]).
//   The threshold scan over the chunk's steps, the early exit (warp vote once
//   every neuron fired; later chunks are never fetched) and the event-free
//   chunk shortcut are those of k_integrate.  Chunks with more events than the
//   per-warp record buffer are processed in segments; the delta[] chains simply
//   continue across segments.
#include "vdt_internal.h"

namespace vdt {
namespace {

constexpr unsigned FULL = 0xffffffffu;
constexpr int SWARPS = 4;    // warps per CTA
constexpr int SEG = 256;     // records per warp-segment
constexpr int SUB = 4;       // weight rows in flight per streamed batch

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

// shared words per warp: records (tmp + sorted, int2 each), slot counters /
// starts / cursors, tap tables (64-bit column base, weight row, list start,
// bucket start) and every tap's chunk offsets
__host__ __device__ inline int sorted_words(int ntaps, int OS) {
    return 2 * SEG * 2 + 3 * 96 + 64 + 3 * 32 + ((ntaps * OS + 3) & ~3);
}

// delta[S] += the run [a, b) of sorted records (chain order kept)
template <int DELTA, int V, int S>
__device__ __forceinline__ void stream_slot(float (&d)[DELTA][V], const int2* rec, int a, int b,
                                            const float* Wl, int C_out, bool lane_live) {
    int k = a;
    for (; k + SUB <= b; k += SUB) {
        int2 e[SUB];
        float w[SUB][V];
#pragma unroll
        for (int u = 0; u < SUB; ++u) e[u] = rec[k + u];
#pragma unroll
        for (int u = 0; u < SUB; ++u) {
            if (lane_live) ldw<V>(Wl + e[u].x * C_out, w[u]);
            else {
#pragma unroll
                for (int v = 0; v < V; ++v) w[u][v] = 0.0f;
            }
        }
#pragma unroll
        for (int u = 0; u < SUB; ++u) {
            const float lv = __int_as_float(e[u].y);
#pragma unroll
            for (int v = 0; v < V; ++v) d[S][v] = fmaf(w[u][v], lv, d[S][v]);
        }
    }
    for (; k < b; ++k) {
        const int2 e = rec[k];
        float w[V];
        if (lane_live) ldw<V>(Wl + e.x * C_out, w);
        else {
#pragma unroll
            for (int v = 0; v < V; ++v) w[v] = 0.0f;
        }
        const float lv = __int_as_float(e.y);
#pragma unroll
        for (int v = 0; v < V; ++v) d[S][v] = fmaf(w[v], lv, d[S][v]);
    }
}

template <int DELTA, int V, int S = 0>
__device__ __forceinline__ void stream_all(float (&d)[DELTA][V], const int2* rec, const int* start,
                                           const float* Wl, int C_out, bool lane_live) {
    if constexpr (S < DELTA) {
        const int a = start[S], b = start[S + 1];
        if (a < b) stream_slot<DELTA, V, S>(d, rec, a, b, Wl, C_out, lane_live);
        stream_all<DELTA, V, S + 1>(d, rec, start, Wl, C_out, lane_live);
    }
}

template <int DELTA, int V, int MINB>
__global__ void __launch_bounds__(SWARPS * 32, MINB) k_sorted(IntegParams p, long long n_warps, int groups) {
    extern __shared__ __align__(16) int sm[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntaps = p.is_fc ? 1 : p.K * p.K;
    const int OS = p.NC + 1;
    const int words = sorted_words(ntaps, OS);
    int* wb = sm + warp * words;
    int2* s_tmp = reinterpret_cast<int2*>(wb);               // [SEG] arrival order
    int2* s_rec = s_tmp + SEG;                               // [SEG] slot order
    int* s_cnt = wb + 4 * SEG;                               // [96] counts, then cursors
    int* s_start = s_cnt + 96;                               // [96] slot starts (+ end)
    long long* s_cbase = reinterpret_cast<long long*>(s_start + 2 * 96);
    int* s_wrow = s_start + 2 * 96 + 64;
    int* s_pre = s_wrow + 32;
    int* s_st = s_pre + 32;
    int* s_off = s_st + 32;                                  // [ntaps][OS]
    float* s_decay = reinterpret_cast<float*>(sm + SWARPS * words);
    float* s_th = s_decay + p.decay_len;
    float* s_min = s_th + p.T;
    for (int i = threadIdx.x; i < p.decay_len; i += blockDim.x) s_decay[i] = p.lut_decay[i];
    for (int i = threadIdx.x; i < p.T; i += blockDim.x) s_th[i] = p.lut_th[i];
    __syncthreads();
    for (int c = threadIdx.x; c < p.NC; c += blockDim.x) {
        float mn = __int_as_float(0x7f800000);
        for (int t = c * DELTA; t < min(p.T, (c + 1) * DELTA); ++t) {
            const float th = s_th[t];
            if (t >= p.t_min && th >= 1e-5f && th < mn) mn = th;
        }
        s_min[c] = mn;
    }
    __syncthreads();

    const long long gw = (long long)blockIdx.x * SWARPS + warp;
    if (gw >= n_warps) return;                               // warp-uniform
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
        s_cbase[lane] = col;
        s_wrow[lane] = p.is_fc ? 0 : lane * p.C_in;
    }
    __syncwarp();
    for (int i = lane; i < ntaps * OS; i += 32) {
        const int j = i / OS, c = i - j * OS;
        const long long col = s_cbase[j];
        s_off[i] = col < 0 ? 0 : __ldg(p.off + col * OS + c);
    }
    __syncwarp();
    if (lane < ntaps) {
        const long long col = s_cbase[lane];
        s_cbase[lane] = col < 0 ? 0 : col * p.C_in;
    }
    __syncwarp();

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
    const unsigned lt = (1u << lane) - 1u;

    for (int tau = 0; tau < p.NC; ++tau) {
        const int base = tau * DELTA;
        int cnt = 0, st = 0;
        if (lane < ntaps) {
            st = s_off[lane * OS + tau];
            cnt = s_off[lane * OS + tau + 1] - st;
        }
        int inc = cnt;
#pragma unroll
        for (int dd = 1; dd < 32; dd <<= 1) {
            const int u = __shfl_up_sync(FULL, inc, dd);
            if (lane >= dd) inc += u;
        }
        const int total = __shfl_sync(FULL, inc, 31);
        int n_live = 0;
#pragma unroll
        for (int v = 0; v < V; ++v) n_live += alive[v] ? 1 : 0;
        if (p.fetched) fetched += (unsigned long long)total * n_live;

        if (total == 0) {
            // no input in this chunk: constant carry, fires iff it reaches the
            // chunk's lowest firing threshold
            const float mn = s_min[tau];
#pragma unroll
            for (int v = 0; v < V; ++v) {
                if (alive[v] && carry[v] >= mn) {
                    for (int t = base; t < min(p.T, base + DELTA); ++t) {
                        const float th = s_th[t];
                        if (t >= p.t_min && carry[v] >= th && th >= 1e-5f) {
                            res[v] = (float)t;
                            alive[v] = false;
                            break;
                        }
                    }
                }
            }
        } else {
            if (lane < ntaps) { s_pre[lane] = inc - cnt; s_st[lane] = st; }
            __syncwarp();
            float d[DELTA][V];
#pragma unroll
            for (int i = 0; i < DELTA; ++i)
#pragma unroll
                for (int v = 0; v < V; ++v) d[i][v] = 0.0f;
            const bool lane_live = n_live > 0;
            for (int s0 = 0; s0 < total; s0 += SEG) {
                const int segn = min(SEG, total - s0);
                for (int i = lane; i < DELTA; i += 32) s_cnt[i] = 0;
                __syncwarp();
                // 1. decode + per-slot histogram
                for (int w0 = 0; w0 < segn; w0 += 32) {
                    const int q = w0 + lane;
                    int slot = -1;
                    if (q < segn) {
                        const int pidx = s0 + q;
                        int lo = 0, hi = ntaps - 1;
                        while (lo < hi) {
                            const int mid = (lo + hi + 1) >> 1;
                            if (s_pre[mid] <= pidx) lo = mid; else hi = mid - 1;
                        }
                        const long long at = s_cbase[lo] + s_st[lo] + (pidx - s_pre[lo]);
                        const int ci = __ldg(p.cin + at);
                        const float t = __ldg(p.tin + at);
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
                        s_tmp[q] = make_int2((s_wrow[lo] + ci) | (slot << 24), __float_as_int(s_decay[ti]));
                    }
                    const unsigned g = __match_any_sync(FULL, slot);
                    if (slot >= 0 && lane == __ffs(g) - 1) s_cnt[slot] += __popc(g);
                    __syncwarp();
                }
                // 2. slot offsets, then the stable scatter into slot order
                for (int c = 0; c < DELTA; c += 32) {
                    const int i = c + lane;
                    const int v = i < DELTA ? s_cnt[i] : 0;
                    int x = v;
#pragma unroll
                    for (int dd = 1; dd < 32; dd <<= 1) {
                        const int u = __shfl_up_sync(FULL, x, dd);
                        if (lane >= dd) x += u;
                    }
                    const int prev = c == 0 ? 0 : s_start[c];
                    if (i < DELTA) { s_start[i] = prev + x - v; s_cnt[i] = prev + x - v; }
                    if (lane == 31) s_start[min(c + 32, DELTA)] = prev + x;
                    __syncwarp();
                }
                for (int w0 = 0; w0 < segn; w0 += 32) {
                    const int q = w0 + lane;
                    int slot = -1;
                    int2 e = make_int2(0, 0);
                    if (q < segn) { e = s_tmp[q]; slot = e.x >> 24; }
                    const unsigned g = __match_any_sync(FULL, slot);
                    int pos = 0;
                    if (slot >= 0) pos = s_cnt[slot] + __popc(g & lt);
                    __syncwarp();
                    if (slot >= 0) {
                        s_rec[pos] = make_int2(e.x & 0xffffff, e.y);
                        if (lane == __ffs(g) - 1) s_cnt[slot] += __popc(g);
                    }
                    __syncwarp();
                }
                // 3. stream every slot's run into its own delta register
                stream_all<DELTA, V>(d, s_rec, s_start, Wl, p.C_out, lane_live);
                __syncwarp();
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
        }
        bool any_alive = false;
#pragma unroll
        for (int v = 0; v < V; ++v) any_alive |= alive[v];
        if (!__any_sync(FULL, any_alive)) break;
    }
    if (lane_ok) stw<V>(p.out + pix * p.C_out + c0, res);
    if (p.fetched) {
#pragma unroll
        for (int dd = 16; dd > 0; dd >>= 1) fetched += __shfl_down_sync(FULL, fetched, dd);
        if (lane == 0 && fetched) atomicAdd(p.fetched, fetched);
    }
}

int pick_v_sorted(int C_out, int delta) {
    if (C_out % 4 == 0 && C_out >= 128 && delta * 4 <= 32) return 4;
    if (C_out % 2 == 0 && C_out >= 64 && delta * 2 <= 32) return 2;
    return 1;
}

template <int DELTA, int V>
cudaError_t launch_sorted_dv(const IntegParams& p, cudaStream_t s, long long n_warps, int groups) {
    const int ntaps = p.is_fc ? 1 : p.K * p.K;
    const size_t smem = (size_t)SWARPS * sorted_words(ntaps, p.NC + 1) * sizeof(int) +
                        (size_t)(p.decay_len + p.T + p.NC) * sizeof(float);
    constexpr int REGS = DELTA * V + SUB * V + 48;
    constexpr int MINB = (65536 / (SWARPS * 32 * REGS)) > 8 ? 8 : (65536 / (SWARPS * 32 * REGS));
    auto kern = k_sorted<DELTA, V, MINB>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    kern<<<(unsigned)((n_warps + SWARPS - 1) / SWARPS), SWARPS * 32, smem, s>>>(p, n_warps, groups);
    return cudaGetLastError();
}

template <int DELTA>
cudaError_t launch_sorted_d(const IntegParams& p, cudaStream_t s) {
    const int V = pick_v_sorted(p.C_out, DELTA);
    const int groups = (p.C_out + 32 * V - 1) / (32 * V);
    const long long pixels = p.is_fc ? (long long)p.B : (long long)p.B * p.H_out * p.W_out;
    const long long n_warps = pixels * groups;
    if (n_warps <= 0) return cudaSuccess;
    switch (V) {
        case 4: return launch_sorted_dv<DELTA, (DELTA <= 8 ? 4 : 1)>(p, s, n_warps, groups);
        case 2: return launch_sorted_dv<DELTA, (DELTA <= 16 ? 2 : 1)>(p, s, n_warps, groups);
        default: return launch_sorted_dv<DELTA, 1>(p, s, n_warps, groups);
    }
}

}  // namespace

bool sorted_supported(int K, int is_fc, int delta, int C_in, int T, int decay_len) {
    const int ntaps = is_fc ? 1 : K * K;
    if (ntaps > 32) return false;
    if (delta != 1 && delta != 2 && delta != 4 && delta != 8 && delta != 16 && delta != 32 && delta != 64)
        return false;
    if ((long long)ntaps * C_in >= (1 << 24)) return false;          // 24-bit weight row in a record
    const int OS = (T + delta - 1) / delta + 1;
    return (size_t)SWARPS * sorted_words(ntaps, OS) * sizeof(int) + (size_t)(decay_len + T + OS) * sizeof(float) <=
           200 * 1024;
}

cudaError_t launch_sorted(const IntegParams& p, cudaStream_t s) {
    switch (p.delta) {
        case 1: return launch_sorted_d<1>(p, s);
        case 2: return launch_sorted_d<2>(p, s);
        case 4: return launch_sorted_d<4>(p, s);
        case 8: return launch_sorted_d<8>(p, s);
        case 16: return launch_sorted_d<16>(p, s);
        case 32: return launch_sorted_d<32>(p, s);
        case 64: return launch_sorted_d<64>(p, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace vdt
