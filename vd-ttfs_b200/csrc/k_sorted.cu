// k_sorted.cu -- chunked early-exit integrator over reference-layout bucket
// lists (same contract and bit-identical results as k_conv_bucketed,
// t1:83-162 / t2:84-170).
//
// One warp integrates one output pixel for 32*V output channels (lane l owns
// channels (group*32 + l)*V .. +V-1, so each synaptic event's weight row is a
// coalesced V-wide load).  When a pixel has 2 or 4 channel groups, their
// warps sit in one CTA as a team that shares the pixel's tap tables, record
// buffers and sort.  For each chunk tau with input:
//   1. decode (event-parallel, one event per lane, each warp of the team a
//      contiguous share): the chunk's events of all taps, in tap order and
//      bucket order -- the reference's FMA-chain order -- become {weight row =
//      tap*C_in + cin, slot = tb - tau*DELTA, LUT_decay} records in shared
//      memory, counted per slot and warp (shared-memory atomics);
//   2. one warp turns the counts into slot offsets and per-warp cursors (a
//      warp's share follows the shares before it), each warp scatters its
//      share stably (rank = popc(group & lanemask_lt)), so the records are
//      grouped by slot with their chain order inside each slot, and the
//      non-empty slots become a run table;
//   3. every warp streams the chunk's records for its own channels into a
//      single accumulator per neuron (one broadcast LDS.64, one weight load,
//      V FMAs per event; blocks of 8 records run branch-free) and closes the
//      step at the end of each run.  Steps without input are closed lazily
//      in O(log T) (Lanes::close_empty), input-free chunks cost nothing.
//   The team stops once all its neurons fired (later chunks are never
//   fetched); a warp whose neurons have all fired keeps sorting for the
//   others.  A chunk with more events than the record buffer is sorted and
//   streamed in segments of half a buffer; each slot's partial sum carries
//   over between segments in shared memory (the chain order is the same),
//   and the chunk's steps close after its last segment.
#include <type_traits>

#include "lanes.h"
#include "vdt_internal.h"

namespace vdt {
namespace {

constexpr int SWARPS = 4;    // warps per CTA
constexpr int FS = 8;        // records per streamed block
constexpr int MAXS = 64;     // slots per chunk (DELTA <= 64)
constexpr int ROW_MASK = 0xffffff;      // decoded record.x: row | slot << 24
constexpr int META_NRUNS = SWARPS;      // s_meta: [0, G) alive flags, then the run count

// records per team buffer: 256 for one warp per pixel (so that 8 CTAs fit
// in shared memory), 512 for teams of 2 or 4 warps
__host__ __device__ constexpr int seg_records(int G) { return G == 1 ? 256 : 512; }

// shared words per team of G warps: records (arrival order + slot order,
// int2 each), per-warp slot counts and cursors, slot starts (+ end), tap
// tables (64-bit column base, weight row, list start, bucket start), the
// chunk's runs (int2 per slot), per-warp alive flags and the run count, and
// every tap's chunk offsets
__host__ __device__ inline int sorted_words(int ntaps, int OS, int G) {
    const int SEG = seg_records(G);
    return 2 * SEG * 2 + 2 * G * MAXS + 96 + 64 + 3 * 32 + 2 * MAXS + 8 + ((ntaps * OS + 3) & ~3);
}

template <int V>
__device__ __forceinline__ void load_row_shared(const float* p, float (&w)[V]) {
    if constexpr (V == 1) {
        w[0] = *p;
    } else if constexpr (V == 2) {
        const float2 v = *reinterpret_cast<const float2*>(p);
        w[0] = v.x; w[1] = v.y;
    } else {
        const float4 v = *reinterpret_cast<const float4*>(p);
        w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
    }
}

// barrier of the G warps of one team (named barrier team + 1; G = 1: the warp)
template <int G>
__device__ __forceinline__ void team_sync(int team) {
    if constexpr (G == 1) {
        __syncwarp();
    } else if constexpr (G == SWARPS) {
        asm volatile("bar.sync 1, %0;" ::"n"(G * 32) : "memory");
    } else {
        static_assert(SWARPS / G == 2, "two teams per CTA");
        if (team == 0) asm volatile("bar.sync 1, %0;" ::"n"(G * 32) : "memory");
        else asm volatile("bar.sync 2, %0;" ::"n"(G * 32) : "memory");
    }
}

// CULIF selects the task-3 neuron (CulifLanes, no LUT, every step scanned).
// G warps (a team) share one output pixel: warp rank r of the team owns its
// channel group r, and the team decodes and sorts each chunk once.
template <int DELTA, int V, int MINB, bool CULIF, int G>
__global__ void __launch_bounds__(SWARPS * 32, MINB) k_sorted(IntegParams p, int n_warps, int groups) {
    static_assert(SWARPS % G == 0, "teams tile the CTA");
    constexpr int SEG = seg_records(G);
    extern __shared__ __align__(16) int sm[];
    __shared__ int s_floor, s_mono;
    chain_release();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int team = warp / G, rank = warp - team * G;
    const int ntaps = p.is_fc ? 1 : p.K * p.K;
    const int OS = p.NC + 1;
    const int words = sorted_words(ntaps, OS, G);
    int* wb = sm + team * words;
    int2* s_tmp = reinterpret_cast<int2*>(wb);               // [SEG] arrival order
    int2* s_rec = s_tmp + SEG;                               // [SEG] slot order
    int* s_cnt = wb + 4 * SEG;                               // [G][MAXS] per-warp slot counts
    int* s_cur = s_cnt + G * MAXS;                           // [G][MAXS] per-warp slot cursors
    int* s_start = s_cur + G * MAXS;                         // [96] slot starts (+ end)
    long long* s_cbase = reinterpret_cast<long long*>(s_start + 96);
    int* s_wrow = s_start + 96 + 64;
    int* s_pre = s_wrow + 32;
    int* s_st = s_pre + 32;
    int2* s_runs = reinterpret_cast<int2*>(s_st + 32);      // [MAXS] chunk runs
    int* s_meta = s_st + 32 + 2 * MAXS;                      // [G] alive flags, [META_NRUNS] run count
    int* s_off = s_meta + 8;                                 // [ntaps][OS]
    float* s_decay = reinterpret_cast<float*>(sm + (SWARPS / G) * words);
    float* s_th = s_decay + p.decay_len;
    float* s_thx = s_th + p.T;
    ThTables tt{};
    if constexpr (!CULIF) {
        for (int i = threadIdx.x; i < p.decay_len; i += blockDim.x) s_decay[i] = p.lut_decay[i];
        tt = stage_thresholds(p, s_th, s_thx, &s_floor, &s_mono);
    }
    const CulifCfg cc{p.culif_decay, p.culif_th};
    chain_wait();                                            // the bucket lists are complete

    const int gw = blockIdx.x * SWARPS + warp;
    if (gw >= n_warps) return;   // whole teams: with G > 1, n_warps is a multiple of G = groups
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
    if (rank == 0) {                                         // the team's tap tables
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
    }
    team_sync<G>(team);

    std::conditional_t<CULIF, CulifLanes<V>, Lanes<V>> nu;
    if constexpr (CULIF) nu.init(lane_ok, p.inf_time);
    else nu.init(p.bias, c0, lane_ok, p.inf_time);
    unsigned long long fetched = 0;
    const float* Wl = p.W + (lane_ok ? c0 : 0);
    const unsigned lt = (1u << lane) - 1u;
    int next_t = 0;                                          // steps < next_t are closed
    bool done = false;                                       // every neuron of this warp fired
    int base = 0;

    // decode of the chunk's event pidx (tap order, then bucket order): its
    // slot and record {weight row (+ slot << 24), LUT value}
    auto decode = [&](int pidx, int& slot) -> int2 {
        int lo = 0, hi = ntaps - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (s_pre[mid] <= pidx) lo = mid; else hi = mid - 1;
        }
        const long long at = s_cbase[lo] + s_st[lo] + (pidx - s_pre[lo]);
        const int ci = __ldg(p.cin + at);
        const float t = __ldg(p.tin + at);
        float lv = 1.0f;                                     // CuLIF: in[t] += w exactly
        int tb;
        if constexpr (CULIF) {
            tb = (int)t;
        } else {
            tb = (int)floorf(t - p.tfs);
            if (tb < 0) tb = 0;
            int ti;
            if (p.lut_mode == VDT_LUT_BY_TB) {
                ti = tb;
            } else {
                ti = (int)t;
                ti = ti < 0 ? 0 : (ti > p.T ? p.T : ti);
            }
            lv = s_decay[ti];
        }
        slot = tb - base;
        return make_int2((s_wrow[lo] + ci) | (slot << 24), __float_as_int(lv));
    };
    // the chunk's events [s0, s0 + n) whose slot is in [p0, p0 + nb), into
    // s_rec grouped by slot, chain order kept inside each slot (the whole
    // team): each warp decodes a contiguous share of the events into dec and
    // counts them per slot; one warp turns the counts into slot starts, each
    // warp's cursors (its share follows the shares before it) and the runs
    // {end, rbase + slot}; each warp scatters its share stably
    // (rank = popc(group & lanemask_lt)).  Returns the run count.
    auto sort_slots = [&](int2* dec, int s0, int n, int p0, int nb, int rbase) -> int {
        int* my_cnt = s_cnt + rank * MAXS;
        int* my_cur = s_cur + rank * MAXS;
        for (int i = lane; i < nb; i += 32) my_cnt[i] = 0;
        __syncwarp();
        const int per = (n + G * 32 - 1) / (G * 32) * 32;
        const int lo = min(n, rank * per), hi = min(n, lo + per);
        for (int w0 = lo; w0 < hi; w0 += 32) {
            const int q = w0 + lane;
            int slot = -1;
            if (q < hi) dec[q] = decode(s0 + q, slot);
            slot -= p0;
            if (slot >= 0 && slot < nb) atomicAdd(&my_cnt[slot], 1);   // counts only: order is free
        }
        team_sync<G>(team);
        if (rank == 0) {
            int prev = 0;
            for (int c = 0; c < nb; c += 32) {
                const int i = c + lane;
                int v = 0;
                if (i < nb) {
#pragma unroll
                    for (int r = 0; r < G; ++r) v += s_cnt[r * MAXS + i];
                }
                int x = v;
#pragma unroll
                for (int dd = 1; dd < 32; dd <<= 1) {
                    const int u = __shfl_up_sync(FULL_MASK, x, dd);
                    if (lane >= dd) x += u;
                }
                if (i < nb) {
                    int at = prev + x - v;
                    s_start[i] = at;
#pragma unroll
                    for (int r = 0; r < G; ++r) { s_cur[r * MAXS + i] = at; at += s_cnt[r * MAXS + i]; }
                }
                prev += __shfl_sync(FULL_MASK, x, 31);
            }
            if (lane == 0) s_start[nb] = prev;
            __syncwarp();
            const int nr = compact_runs(s_start + 1, nb, rbase, s_runs);
            if (lane == 0) s_meta[META_NRUNS] = nr;
        }
        team_sync<G>(team);
        for (int w0 = lo; w0 < hi; w0 += 32) {
            const int q = w0 + lane;
            int slot = -1;
            int2 e = make_int2(0, 0);
            if (q < hi) {
                e = dec[q];
                slot = (e.x >> 24) - p0;
                if (slot >= nb) slot = -1;
                e.x = (e.x & ROW_MASK) * p.C_out;            // element offset of the weight row
            }
            const unsigned g = __match_any_sync(FULL_MASK, slot);
            int pos = 0;
            if (slot >= 0) pos = my_cur[slot] + __popc(g & lt);
            __syncwarp();
            if (slot >= 0) {
                s_rec[pos] = e;
                if (lane == __ffs(g) - 1) my_cur[slot] += __popc(g);
            }
            __syncwarp();
        }
        team_sync<G>(team);
        return s_meta[META_NRUNS];
    };

    for (int tau = 0; tau < p.NC; ++tau) {
        base = tau * DELTA;
        int cnt = 0, st = 0;
        if (lane < ntaps) {
            st = s_off[lane * OS + tau];
            cnt = s_off[lane * OS + tau + 1] - st;
        }
        int inc = cnt;
#pragma unroll
        for (int dd = 1; dd < 32; dd <<= 1) {
            const int u = __shfl_up_sync(FULL_MASK, inc, dd);
            if (lane >= dd) inc += u;
        }
        const int total = __shfl_sync(FULL_MASK, inc, 31);  // the same in every warp of the team
        if constexpr (CULIF) {
            if (total == 0) {                                // every step still integrates
                if (!done) {
                    nu.close_empty(next_t, base + DELTA, cc);
                    next_t = base + DELTA;
                    done = !__any_sync(FULL_MASK, nu.any());
                }
                continue;
            }
        } else {
            if (total == 0) continue;                        // closed lazily
            if (!done) {
                nu.close_empty(next_t, base, tt);            // input-free steps before the chunk
                next_t = base;
            }
        }
        if (p.fetched) fetched += (unsigned long long)total * nu.live();
        done = done || !__any_sync(FULL_MASK, nu.any());
        // the team goes on while any of its warps has a neuron alive
        if (lane == 0) s_meta[rank] = done ? 0 : 1;
        if (rank == 0 && lane < ntaps) { s_pre[lane] = inc - cnt; s_st[lane] = st; }
        team_sync<G>(team);
        int alive = 0;
#pragma unroll
        for (int r = 0; r < G; ++r) alive |= s_meta[r];
        if (!alive) break;
        if (total <= SEG) {
            const int nruns = sort_slots(s_tmp, 0, total, 0, DELTA, base);
            if (!done) {
                if constexpr (CULIF) {
                    done = !stream_runs<V, FS>(nu, s_rec, 0, s_runs, nruns, Wl, next_t, cc);
                    if (!done) {
                        nu.close_empty(next_t, base + DELTA, cc);    // the chunk's remaining steps
                        next_t = base + DELTA;
                        done = !__any_sync(FULL_MASK, nu.any());
                    }
                } else {
                    done = !stream_runs<V, FS>(nu, s_rec, 0, s_runs, nruns, Wl, next_t, tt);
                }
            }
        } else {
            // more events than the record buffer: segments of SEG / 2 events,
            // each sorted by slot like a chunk that fits (decoded into the
            // upper half of s_rec, scattered into the lower half); every
            // slot's partial sum carries over between segments in this
            // warp's share of the s_tmp words, so each slot's chain keeps the
            // event order.  Then the chunk's steps close in order (the CuLIF
            // scan has no t < T guard, t3:137-141).
            constexpr int HS = SEG / 2;
            constexpr int SPW = 2 * SEG / (32 * V * G) > 0 ? 2 * SEG / (32 * V * G) : 1;
            constexpr int SPP = SPW < DELTA ? SPW : DELTA;  // slots per pass: the team's sums fill s_tmp
            float* s_acc = reinterpret_cast<float*>(s_tmp) + rank * SPP * V * 32 + lane * V;
            int2* s_dec = s_rec + HS;
            const unsigned sa_rec = (unsigned)__cvta_generic_to_shared(s_rec);
            const float zero[V] = {};
            for (int p0 = 0; p0 < DELTA; p0 += SPP) {
#pragma unroll
                for (int i = 0; i < SPP; ++i) store_res<V>(s_acc + i * 32 * V, zero);
                for (int s0 = 0; s0 < total; s0 += HS) {
                    const int segn = min(HS, total - s0);
                    team_sync<G>(team);                      // every warp is done with s_rec
                    const int nruns = sort_slots(s_dec, s0, segn, p0, SPP, 0);
                    if (!done) {
                        int k = 0;
                        for (int j = 0; j < nruns; ++j) {
                            const int2 rn = s_runs[j];
                            load_row_shared<V>(s_acc + rn.y * 32 * V, nu.acc);
                            stream_run_records<V, FS>(nu, sa_rec, k, rn.x, Wl);
                            store_res<V>(s_acc + rn.y * 32 * V, nu.acc);
                            k = rn.x;
                        }
                    }
                }
                if (!done) {
                    for (int i = 0; i < SPP; ++i) {
                        if (!CULIF && base + p0 + i >= p.T) break;
                        load_row_shared<V>(s_acc + i * 32 * V, nu.acc);
                        if constexpr (CULIF) nu.close_step_bf(base + p0 + i, cc);
                        else nu.close_step(base + p0 + i, tt);
                    }
                }
                __syncwarp();
            }
            if (!done) {
                next_t = CULIF ? base + DELTA : min(p.T, base + DELTA);
                done = !__any_sync(FULL_MASK, nu.any());
            }
        }
    }
    if constexpr (!CULIF) {
        if (!done) nu.close_empty(next_t, p.T, tt);
    }
    if (lane_ok) {
        if (p.pool_out) {
            pool_store<V>(p.pool_out, img, h_out, w_out, p.H_out, p.W_out, p.C_out, c0, nu.res);
        } else if (p.out_nchw) {
            const long long plane = (long long)p.H_out * p.W_out;
            const long long site = (long long)h_out * p.W_out + w_out;
#pragma unroll
            for (int v = 0; v < V; ++v) p.out[(img * p.C_out + c0 + v) * plane + site] = nu.res[v];
        } else {
            store_res<V>(p.out + (long long)pix * p.C_out + c0, nu.res);
        }
    }
    if (p.fetched) {
#pragma unroll
        for (int dd = 16; dd > 0; dd >>= 1) fetched += __shfl_down_sync(FULL_MASK, fetched, dd);
        if (lane == 0 && fetched) atomicAdd(p.fetched, fetched);
    }
}

int pick_v_sorted(int C_out, int delta) {
    if (C_out % 4 == 0 && C_out >= 128 && delta * 4 <= 32) return 4;
    if (C_out % 2 == 0 && C_out >= 64 && delta * 2 <= 32) return 2;
    return 1;
}

template <int DELTA, int V, bool CULIF, int G>
cudaError_t launch_sorted_dvg(const IntegParams& p, cudaStream_t s, int n_warps, int groups) {
    const int ntaps = p.is_fc ? 1 : p.K * p.K;
    const size_t smem = (size_t)(SWARPS / G) * sorted_words(ntaps, p.NC + 1, G) * sizeof(int) +
                        (CULIF ? 0 : (size_t)(p.decay_len + 2 * p.T) * sizeof(float));
    // occupancy: 8 CTAs of 4 warps per SM (64 registers, a few bytes of
    // spill; about 24 KB of shared memory per CTA for 3x3 taps: two teams of
    // two warps, or four single warps with half-size record buffers)
    constexpr int MINB = 8;
    auto kern = k_sorted<DELTA, V, MINB, CULIF, G>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    return launch_chain(kern, dim3((n_warps + SWARPS - 1) / SWARPS), dim3(SWARPS * 32), smem, s, p, n_warps,
                        groups);
}

// 2 or 4 channel groups: the group warps of a pixel form a team in one CTA
template <int DELTA, int V, bool CULIF>
cudaError_t launch_sorted_dv(const IntegParams& p, cudaStream_t s, int n_warps, int groups) {
    switch (groups) {
        case 2: return launch_sorted_dvg<DELTA, V, CULIF, 2>(p, s, n_warps, groups);
        case 4: return launch_sorted_dvg<DELTA, V, CULIF, 4>(p, s, n_warps, groups);
        default: return launch_sorted_dvg<DELTA, V, CULIF, 1>(p, s, n_warps, groups);
    }
}

template <int DELTA, bool CULIF>
cudaError_t launch_sorted_d(const IntegParams& p, cudaStream_t s) {
    const int V = pick_v_sorted(p.C_out, DELTA);
    const int groups = (p.C_out + 32 * V - 1) / (32 * V);
    const long long pixels = p.is_fc ? (long long)p.B : (long long)p.B * p.H_out * p.W_out;
    const long long n_warps = pixels * groups;
    if (n_warps <= 0) return cudaSuccess;
    if (n_warps >= (1ll << 31)) return cudaErrorInvalidValue;   // 32-bit work index
    const int nw = (int)n_warps;
    switch (V) {
        case 4: return launch_sorted_dv<DELTA, (DELTA <= 8 ? 4 : 1), CULIF>(p, s, nw, groups);
        case 2: return launch_sorted_dv<DELTA, (DELTA <= 16 ? 2 : 1), CULIF>(p, s, nw, groups);
        default: return launch_sorted_dv<DELTA, 1, CULIF>(p, s, nw, groups);
    }
}

template <bool CULIF>
cudaError_t launch_sorted_any(const IntegParams& p, cudaStream_t s) {
    switch (p.delta) {
        case 1: return launch_sorted_d<1, CULIF>(p, s);
        case 2: return launch_sorted_d<2, CULIF>(p, s);
        case 4: return launch_sorted_d<4, CULIF>(p, s);
        case 8: return launch_sorted_d<8, CULIF>(p, s);
        case 16: return launch_sorted_d<16, CULIF>(p, s);
        case 32: return launch_sorted_d<32, CULIF>(p, s);
        case 64: return launch_sorted_d<64, CULIF>(p, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

bool sorted_supported(int K, int is_fc, int delta, int C_in, int C_out, int T, int decay_len) {
    const int ntaps = is_fc ? 1 : K * K;
    if (ntaps > 32) return false;
    if ((long long)ntaps * C_in * C_out >= (1ll << 31)) return false;   // 31-bit weight offsets
    if (delta != 1 && delta != 2 && delta != 4 && delta != 8 && delta != 16 && delta != 32 && delta != 64)
        return false;
    if ((long long)ntaps * C_in >= (1 << 24)) return false;          // 24-bit weight row in a record
    const int OS = (T + delta - 1) / delta + 1;
    return (size_t)SWARPS * sorted_words(ntaps, OS, 1) * sizeof(int) + (size_t)(decay_len + 2 * T) * sizeof(float) <=
           200 * 1024;
}

cudaError_t launch_sorted(const IntegParams& p, cudaStream_t s) { return launch_sorted_any<false>(p, s); }

bool culif_supported(int K, int is_fc, int delta, int C_in, int C_out, int T) {
    return sorted_supported(K, is_fc, delta, C_in, C_out, T, 0);
}

cudaError_t launch_culif(const IntegParams& p, cudaStream_t s) { return launch_sorted_any<true>(p, s); }

}  // namespace vdt
