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
//      each step the list keeps exactly the reference's FMA-chain order; the
//      non-empty steps become a run table;
//   3. stream (stream_runs): per event one broadcast LDS.64, one V-wide weight
//      load, V FMAs into a single accumulator per neuron; each run ends with
//      the close of its step, steps without input are closed in O(log T).
//      The warp stops once all its neurons fired.
// The fetched-synapse counter keeps the reference's chunk accounting (events
// of every chunk a neuron entered alive).
//
// Layers with at most 16 output channels run k_dense_pair instead (outside
// counting passes): two pixels per warp, sorted one after the other by the
// whole warp, streamed by one half-warp each.
#include <type_traits>

#include "lanes.h"
#include "vdt_internal.h"

namespace vdt {
namespace {

constexpr int DW = 4;         // warps per CTA
constexpr int FS = 8;         // weight rows in flight per streamed block
constexpr int DENSE_WIN = 36; // largest fan-in handled: 36 windows of 32 inputs

// shared words per warp: event records (int2 per input), step bins (T + 1),
// tap column bases (64-bit), runs (int2 per non-empty step)
__host__ __device__ inline int dense_words(int fan_in, int T, int ntaps) {
    const int runs = fan_in < T ? fan_in : T;
    return ((2 * fan_in + 3) & ~3) + ((T + 1 + 3) & ~3) + ((2 * ntaps + 3) & ~3) + 2 * runs;
}

// flattened input index f = tap * C_in + c -> tap, via a float estimate and
// one exact correction (f < 2^20, so the estimate is off by at most one)
__device__ __forceinline__ int tap_of(int f, int C_in, float inv) {
    int j = __float2int_rz((float)f * inv);
    if (j * C_in > f) --j;
    else if ((j + 1) * C_in <= f) ++j;
    return j;
}

size_t dense_smem(int fan, int T, int ntaps, int decay_len, int P) {
    return (size_t)DW * P * dense_words(fan, T, ntaps) * sizeof(int) + (size_t)(decay_len + 2 * T) * sizeof(float);
}

// Sort one output pixel's events into its region (whole warp): reads the
// K*K*C_in input times, stable counting sort by step, records {element
// offset of the weight row, LUT value} in s_list and the run table in
// s_runs; s_bin[tb] ends as the end of step tb's run.  Returns the number of
// runs (warp-uniform).
// CULIF: the task-3 rule (tb = (int)t, kept iff 0 <= tb < T, t3:79; the
// record's LUT value is 1, so the chain adds the weight exactly) and the
// input map may be NCHW (p.in_nchw).
template <int R, bool CULIF, bool ENC = false>
__device__ __forceinline__ int sort_pixel(const IntegParams& p, const float* __restrict__ in, unsigned pix,
                                          int fan, int ntaps, int* wb, const float* s_decay) {
    const int lane = threadIdx.x & 31;
    int2* s_list = reinterpret_cast<int2*>(wb);
    int* s_bin = wb + ((2 * fan + 3) & ~3);                  // [T + 1]
    long long* s_col = reinterpret_cast<long long*>(s_bin + ((p.T + 1 + 3) & ~3));
    int2* s_runs = reinterpret_cast<int2*>(reinterpret_cast<int*>(s_col) + ((2 * ntaps + 3) & ~3));
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
            col = img * p.C_in;                              // one column of C_in features
        } else {
            const int kh = lane / p.K, kw = lane - (lane / p.K) * p.K;
            const int h_in = h_out - p.pad + kh, w_in = w_out - p.pad + kw;
            if (h_in >= 0 && h_in < p.H_in && w_in >= 0 && w_in < p.W_in) {
                if (CULIF && p.in_nchw) col = ((img * p.C_in) * p.H_in + h_in) * p.W_in + w_in;
                else col = ((img * p.H_in + h_in) * p.W_in + w_in) * p.C_in;
            }
        }
        s_col[lane] = col;
    }
    for (int i = lane; i <= p.T; i += 32) s_bin[i] = 0;
    __syncwarp();

    // channel stride of the input map: 1 (NHWC) or H*W (NCHW, CuLIF layers)
    const long long cs = (CULIF && p.in_nchw) ? (long long)p.H_in * p.W_in : 1;
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
            if (cb >= 0) {
                const float v = __ldg(in + cb + (f - j * p.C_in) * cs);
                // ENC: a first layer reading pixels encodes each one as it is read
                if constexpr (ENC) tv[r] = encode_pixel(v, p.encoder, p.enc_tc, p.enc_td, p.T, p.inf_time);
                else tv[r] = v;
            }
        }
    }
    // input value -> key = tb | LUT index << 16 (bucketize rule), -1 if no event
    int key[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const float t = tv[r];
        key[r] = -1;
        if constexpr (CULIF) {
            if (t < p.inf_time) {
                const int b = (int)t;
                if (b >= 0 && b < p.T) key[r] = b;
            }
        } else if (t < p.inf_time) {
            int b = (int)floorf(t - p.tfs);
            if (b < 0) b = 0;
            if (b < p.T) {
                int ti;
                if (p.lut_mode == VDT_LUT_BY_TB) {
                    ti = b;
                } else {
                    ti = (int)t;
                    ti = ti < 0 ? 0 : (ti > p.T ? p.T : ti);
                }
                key[r] = b | (ti << 16);
            }
        }
    }
    // 1. histogram by step (shared-memory atomics)
#pragma unroll
    for (int r = 0; r < R; ++r) {
        if (key[r] >= 0) atomicAdd(&s_bin[key[r] & 0xffff], 1);   // counts only: order is free
    }
    __syncwarp();
    // 2. exclusive scan over steps, then the stable scatter of records
    //    {element offset of the weight row, LUT value}
    int run = 0;
    for (int b0 = 0; b0 < p.T; b0 += 32) {
        const int b = b0 + lane;
        const int v = b < p.T ? s_bin[b] : 0;
        int x = v;
#pragma unroll
        for (int dd = 1; dd < 32; dd <<= 1) {
            const int u = __shfl_up_sync(FULL_MASK, x, dd);
            if (lane >= dd) x += u;
        }
        if (b < p.T) s_bin[b] = run + x - v;
        run += __shfl_sync(FULL_MASK, x, 31);
    }
    __syncwarp();
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int tb = key[r] < 0 ? -1 : (key[r] & 0xffff);
        const unsigned g = __match_any_sync(FULL_MASK, tb);
        int pos = 0;
        if (tb >= 0) pos = s_bin[tb] + __popc(g & lt);
        __syncwarp();
        if (tb >= 0) {
            s_list[pos] = make_int2((r * 32 + lane) * p.C_out,
                                    CULIF ? __float_as_int(1.0f) : __float_as_int(s_decay[key[r] >> 16]));
            if (lane == __ffs(g) - 1) s_bin[tb] += __popc(g);
        }
        __syncwarp();
    }
    // s_bin[tb] is now the end of step tb's run
    return compact_runs(s_bin, p.T, 0, s_runs);
}

// CULIF: the task-3 conv_bucketed_early neuron (t3:109-143) fed straight
// from the spike map: CulifLanes, every step scanned up to NC * delta (the
// reference scans whole chunks), output NHWC or NCHW (p.out_nchw).
template <int V, int R, int MINB, bool COUNT, bool CULIF, bool ENC = false>
__global__ void __launch_bounds__(DW * 32, MINB) k_dense(IntegParams p, const float* __restrict__ in,
                                                         int n_warps, int groups) {
    static_assert(!(COUNT && CULIF), "no counters on CuLIF layers");
    static_assert(!(ENC && (COUNT || CULIF)), "the fused encoder is for a LIF first layer outside counting passes");
    extern __shared__ __align__(16) int sm[];
    __shared__ int s_floor, s_mono;
    chain_release();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntaps = p.is_fc ? 1 : p.K * p.K;
    const int fan = ntaps * p.C_in;
    const int words = dense_words(fan, p.T, ntaps);
    int* wb = sm + warp * words;
    int2* s_list = reinterpret_cast<int2*>(wb);
    int* s_bin = wb + ((2 * fan + 3) & ~3);                  // [T + 1]
    int2* s_runs = reinterpret_cast<int2*>(s_bin + ((p.T + 1 + 3) & ~3) + ((2 * ntaps + 3) & ~3));
    float* s_decay = reinterpret_cast<float*>(sm + DW * words);
    float* s_th = s_decay + p.decay_len;
    float* s_thx = s_th + p.T;
    ThTables tt{};
    if constexpr (!CULIF) {
        for (int i = threadIdx.x; i < p.decay_len; i += blockDim.x) s_decay[i] = p.lut_decay[i];
        tt = stage_thresholds(p, s_th, s_thx, &s_floor, &s_mono);
    }
    const CulifCfg cc{p.culif_decay, p.culif_th};
    chain_wait();                                            // the input map is complete

    const int gw = blockIdx.x * DW + warp;
    if (gw >= n_warps) return;                               // warp-uniform
    const unsigned pix = (unsigned)gw / (unsigned)groups;
    const int grp = gw - (int)pix * groups;
    const int c0 = (grp * 32 + lane) * V;
    const bool lane_ok = c0 < p.C_out;
    const int nruns = sort_pixel<R, CULIF, ENC>(p, in, pix, fan, ntaps, wb, s_decay);

    // 3. stream the runs
    std::conditional_t<CULIF, CulifLanes<V>, Lanes<V>> nu;
    if constexpr (CULIF) nu.init(lane_ok, p.inf_time);
    else nu.init(p.bias, c0, lane_ok, p.inf_time);
    const float* Wl = p.W + (lane_ok ? c0 : 0);
    int next_t = 0;
    if constexpr (CULIF) {
        if (stream_runs<V, FS>(nu, s_list, 0, s_runs, nruns, Wl, next_t, cc))
            nu.close_empty(next_t, p.NC * p.delta, cc);
        if (lane_ok && p.out_nchw) {
            const unsigned r = pix / (unsigned)p.W_out, q = r / (unsigned)p.H_out;
            const long long plane = (long long)p.H_out * p.W_out;
            const long long site = (long long)(r - q * (unsigned)p.H_out) * p.W_out + (pix - r * (unsigned)p.W_out);
#pragma unroll
            for (int v = 0; v < V; ++v) p.out[((long long)q * p.C_out + c0 + v) * plane + site] = nu.res[v];
            return;
        }
    } else if constexpr (!COUNT) {
        if (stream_runs<V, FS>(nu, s_list, 0, s_runs, nruns, Wl, next_t, tt))
            nu.close_empty(next_t, p.T, tt);
    } else {
        // fetched synapses, reference chunk accounting: chunk c counts its
        // events once per neuron still alive when the chunk starts
        unsigned long long fetched = 0;
        int next_chunk = 0;
        auto step_end = [&](int t) { return t <= 0 ? 0 : s_bin[min(t, p.T) - 1]; };
        auto account_to = [&](int t) {                       // every chunk starting at or before t
            while (next_chunk < p.NC && next_chunk * p.delta <= t) {
                const int cs = next_chunk * p.delta;
                nu.close_empty(next_t, cs, tt);
                next_t = max(next_t, cs);
                fetched += (unsigned long long)(step_end(cs + p.delta) - step_end(cs)) * nu.live();
                ++next_chunk;
            }
        };
        int k = 0;
        for (int j = 0; j < nruns; ++j) {
            const int2 rn = s_runs[j];
            account_to(rn.y);
            for (; k < rn.x; ++k) stream_block<V, 1>(nu, s_list + k, Wl);
            nu.close_empty(next_t, rn.y, tt);
            nu.close_step(rn.y, tt);
            next_t = rn.y + 1;
        }
        nu.close_empty(next_t, p.T, tt);
#pragma unroll
        for (int dd = 16; dd > 0; dd >>= 1) fetched += __shfl_down_sync(FULL_MASK, fetched, dd);
        if (lane == 0 && fetched) atomicAdd(p.fetched, fetched);
    }
    if (lane_ok) {
        if (p.pool_out) {
            const unsigned r = pix / (unsigned)p.W_out, q = r / (unsigned)p.H_out;
            pool_store<V>(p.pool_out, q, (int)(r - q * (unsigned)p.H_out), (int)(pix - r * (unsigned)p.W_out),
                          p.H_out, p.W_out, p.C_out, c0, nu.res);
        } else {
            store_res<V>(p.out + (long long)pix * p.C_out + c0, nu.res);
        }
    }
}

// Two output pixels per warp for layers with at most 16 output channels
// (a warp per pixel would leave half of its lanes idle): the whole warp
// sorts both pixels, one after the other, into two shared regions
// (sort_pixel), then lanes 0-15 stream the first pixel and lanes 16-31 the
// second, one channel per lane, sharing each run's loop, close and vote
// instructions (stream_runs_grouped).  Outside counting passes only.
template <int R, int MINB>
__global__ void __launch_bounds__(DW * 32, MINB) k_dense_pair(IntegParams p, const float* __restrict__ in,
                                                              int n_warps, long long n_pix) {
    extern __shared__ __align__(16) int sm[];
    __shared__ int s_floor, s_mono;
    chain_release();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntaps = p.is_fc ? 1 : p.K * p.K;
    const int fan = ntaps * p.C_in;
    const int words = dense_words(fan, p.T, ntaps);
    float* s_decay = reinterpret_cast<float*>(sm + DW * 2 * words);
    float* s_th = s_decay + p.decay_len;
    float* s_thx = s_th + p.T;
    for (int i = threadIdx.x; i < p.decay_len; i += blockDim.x) s_decay[i] = p.lut_decay[i];
    const ThTables tt = stage_thresholds(p, s_th, s_thx, &s_floor, &s_mono);
    chain_wait();                                            // the input map is complete

    const int gw = blockIdx.x * DW + warp;
    if (gw >= n_warps) return;                               // warp-uniform
    int nr[2];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        const long long pix = 2ll * gw + q;
        nr[q] = pix < n_pix ? sort_pixel<R, false>(p, in, (unsigned)pix, fan, ntaps, sm + (warp * 2 + q) * words, s_decay)
                            : 0;
    }
    const int g = lane >> 4;
    const long long pix = 2ll * gw + g;
    const int* wb = sm + (warp * 2 + g) * words;
    const int2* s_list = reinterpret_cast<const int2*>(wb);
    const int2* s_runs = reinterpret_cast<const int2*>(wb + ((2 * fan + 3) & ~3) + ((p.T + 1 + 3) & ~3) +
                                                       ((2 * ntaps + 3) & ~3));
    const int c0 = lane & 15;
    const bool lane_ok = c0 < p.C_out && pix < n_pix;
    Lanes<1> nu;
    nu.init(p.bias, c0, lane_ok, p.inf_time);
    const float* Wl = p.W + (lane_ok ? c0 : 0);
    int next_t = 0;
    if (stream_runs_grouped<1, FS>(nu, s_list, s_runs, g ? nr[1] : nr[0], max(nr[0], nr[1]), Wl, next_t, tt))
        nu.close_empty(next_t, p.T, tt);
    if (lane_ok) p.out[pix * p.C_out + c0] = nu.res[0];
}

template <int R>
cudaError_t launch_pair_r(const IntegParams& p, const float* in, cudaStream_t s, long long pixels) {
    const long long n_warps = (pixels + 1) / 2;
    if (n_warps <= 0) return cudaSuccess;
    if (n_warps >= (1ll << 31)) return cudaErrorInvalidValue;   // 32-bit work index
    const int ntaps = p.is_fc ? 1 : p.K * p.K;
    const size_t smem = dense_smem(ntaps * p.C_in, p.T, ntaps, p.decay_len, 2);
    constexpr int REGS = FS + 2 * FS + 4 + R;
    constexpr int MINB = (65536 / (DW * 32 * REGS)) > 8 ? 8 : (65536 / (DW * 32 * REGS));
    auto kern = k_dense_pair<R, MINB>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    return launch_chain(kern, dim3((unsigned)((n_warps + DW - 1) / DW)), dim3(DW * 32), smem, s, p, in,
                        (int)n_warps, pixels);
}

cudaError_t launch_pair(const IntegParams& p, const float* in, cudaStream_t s) {
    const long long pixels = p.is_fc ? (long long)p.B : (long long)p.B * p.H_out * p.W_out;
    const int w = ((p.is_fc ? 1 : p.K * p.K) * p.C_in + 31) / 32;
    if (w <= 1) return launch_pair_r<1>(p, in, s, pixels);
    if (w <= 4) return launch_pair_r<4>(p, in, s, pixels);
    if (w <= 9) return launch_pair_r<9>(p, in, s, pixels);
    if (w <= 18) return launch_pair_r<18>(p, in, s, pixels);
    return launch_pair_r<DENSE_WIN>(p, in, s, pixels);
}

int pick_v_dense(int C_out) {
    if (C_out % 4 == 0 && C_out >= 128) return 4;
    if (C_out % 2 == 0 && C_out >= 64) return 2;
    return 1;
}

template <int V, int R, bool CULIF>
cudaError_t launch_dense_vr(const IntegParams& p, const float* in, cudaStream_t s, int n_warps,
                            int groups) {
    const int ntaps = p.is_fc ? 1 : p.K * p.K;
    const size_t smem = (size_t)DW * dense_words(ntaps * p.C_in, p.T, ntaps) * sizeof(int) +
                        (size_t)(p.decay_len + 2 * p.T) * sizeof(float);
    // register budget tuned for occupancy (the kernel is latency-bound): the
    // streamed block, lane state and the sort's input registers, at most 8
    // CTAs per SM; measured exceptions: one 32-input window runs 16 CTAs (32
    // registers), and 18 windows at 4 channels per lane 9 CTAs (56 registers,
    // the shared-memory limit at 576 inputs; 2 channels per lane stay at 8)
    constexpr int REGS = FS * V + 2 * FS + (CULIF ? 5 : 4) * V + R;
    constexpr int MINB0 = (65536 / (DW * 32 * REGS)) > 8 ? 8 : (65536 / (DW * 32 * REGS));
    constexpr int MINB = CULIF ? MINB0 : (R == 18 && V == 4) ? 9 : (R == 1 ? 16 : MINB0);
    auto kern = CULIF ? k_dense<V, R, MINB, false, true>
                      : (p.fetched ? k_dense<V, R, MINB, true, false>
                                   : (p.encoder ? k_dense<V, R, MINB, false, false, true> : k_dense<V, R, MINB, false, false>));
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    return launch_chain(kern, dim3((n_warps + DW - 1) / DW), dim3(DW * 32), smem, s, p, in, n_warps, groups);
}

template <int V, bool CULIF>
cudaError_t launch_dense_v(const IntegParams& p, const float* in, cudaStream_t s) {
    const int groups = (p.C_out + 32 * V - 1) / (32 * V);
    const long long pixels = p.is_fc ? (long long)p.B : (long long)p.B * p.H_out * p.W_out;
    const long long n_warps = pixels * groups;
    if (n_warps <= 0) return cudaSuccess;
    if (n_warps >= (1ll << 31)) return cudaErrorInvalidValue;   // 32-bit work index
    const int nw = (int)n_warps;
    const int fan = (p.is_fc ? 1 : p.K * p.K) * p.C_in;
    const int w = (fan + 31) / 32;                          // 32-input windows per pixel
    if (w <= 1) return launch_dense_vr<V, 1, CULIF>(p, in, s, nw, groups);
    if (w <= 4) return launch_dense_vr<V, 4, CULIF>(p, in, s, nw, groups);
    if (w <= 9) return launch_dense_vr<V, 9, CULIF>(p, in, s, nw, groups);
    if (w <= 18) return launch_dense_vr<V, 18, CULIF>(p, in, s, nw, groups);
    return launch_dense_vr<V, DENSE_WIN, CULIF>(p, in, s, nw, groups);
}

}  // namespace

bool dense_supported(int K, int is_fc, int C_in, int C_out, int T, int decay_len) {
    const int ntaps = is_fc ? 1 : K * K;
    const int fan = ntaps * C_in;
    if (ntaps > 32 || fan > DENSE_WIN * 32) return false;   // inputs held in registers
    if ((long long)fan * C_out >= (1ll << 31)) return false; // 31-bit weight offsets
    if (T > 0xffff) return false;                           // 16-bit step keys
    return (size_t)DW * dense_words(fan, T, ntaps) * sizeof(int) + (size_t)(decay_len + 2 * T) * sizeof(float) <=
           160 * 1024;
}

cudaError_t launch_dense(const IntegParams& p, const float* in, cudaStream_t s) {
    const int ntaps = p.is_fc ? 1 : p.K * p.K;
    if (!p.fetched && !p.pool_out && !p.encoder && p.C_out <= 16 &&
        dense_smem(ntaps * p.C_in, p.T, ntaps, p.decay_len, 2) <= 160 * 1024)
        return launch_pair(p, in, s);
    switch (pick_v_dense(p.C_out)) {
        case 4: return launch_dense_v<4, false>(p, in, s);
        case 2: return launch_dense_v<2, false>(p, in, s);
        default: return launch_dense_v<1, false>(p, in, s);
    }
}

cudaError_t launch_dense_culif(const IntegParams& p, const float* in, cudaStream_t s) {
    switch (pick_v_dense(p.C_out)) {
        case 4: return launch_dense_v<4, true>(p, in, s);
        case 2: return launch_dense_v<2, true>(p, in, s);
        default: return launch_dense_v<1, true>(p, in, s);
    }
}

}  // namespace vdt
