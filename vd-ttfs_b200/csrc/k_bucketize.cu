// k_bucketize.cu -- lossless counting sort of spike events into arrival chunks
// (the reference's k_bucketize, t1:45-80 / t2:45-81, and k_bucketize_conv /
// k_bucketize_fc, t3:70-106).
//
// Output layout is exactly the reference's: per column, off[col*(NC+1) + c]
// are exclusive chunk offsets (off[..+NC] = event count), and cin/tin[col*c_in
// + p] list the kept events, stable (increasing channel) within each chunk.
//
// Two kernels:
//  * k_bucketize_warp  -- one warp per column (NHWC, c_in >= 32).  Lanes read
//    32 consecutive channels per step (coalesced), group equal chunk bins with
//    __match_any_sync (warp-aggregated histogram: one shared-memory add per
//    distinct bin per step), an exclusive warp scan turns counts into offsets,
//    and the scatter ranks each lane inside its bin group with
//    popc(group & lanemask_lt), so equal-bin events keep channel order.
//    Channel values stay in registers between the two passes (c_in <= 512).
//  * k_bucketize_rows  -- one CTA per long column (NHWC, c_in > 512), RW warps
//    over contiguous segments with chunk-major segment offsets.
//  * k_bucketize_thread -- one thread per column for narrow columns (c_in < 32)
//    and for NCHW sites, where adjacent threads read adjacent addresses; its
//    chunk counters live in shared memory laid out [bin][thread] (no bank
//    conflicts) instead of the reference's local-memory arrays.
#include "vdt_internal.h"

namespace vdt {
namespace {

constexpr unsigned FULL = 0xffffffffu;

// chunk bin of a spike time, or -1 when the event is not kept (t1:57-59,
// t2:58-60 for tb_mode 0; t3:79 for tb_mode 1)
__device__ __forceinline__ int chunk_bin(float t, const BktParams& p) {
    if (!(t < p.inf_time)) return -1;
    int tb;
    if (p.tb_mode == VDT_TB_FLOOR_STAGGER) {
        tb = (int)floorf(t - p.tfs);
        if (tb < 0) tb = 0;
        if (tb >= p.T) return -1;
    } else {
        tb = (int)t;
        if (tb < 0 || tb >= p.T) return -1;
    }
    return tb / p.delta;
}

template <int MAXR>
__global__ void __launch_bounds__(256) k_bucketize_warp(BktParams p) {
    extern __shared__ int s_bins[];                 // [warps][NC]
    chain_release();
    chain_wait();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const long long col = (long long)blockIdx.x * (blockDim.x >> 5) + warp;
    if (col >= p.n_cols) return;                    // warp-uniform
    int* cnt = s_bins + warp * p.NC;
    for (int c = lane; c < p.NC; c += 32) cnt[c] = 0;
    __syncwarp();

    const float* src = p.in + col * p.c_in;
    const int nb = (p.c_in + 31) >> 5;
    float tv[MAXR];
    // pass 1: per-chunk counts (shared-memory atomics)
#pragma unroll
    for (int j = 0; j < MAXR; ++j) {
        if (j < nb) {
            const int ch = j * 32 + lane;
            const float t = ch < p.c_in ? __ldg(src + ch) : p.inf_time;
            tv[j] = t;
            const int b = chunk_bin(t, p);
            if (b >= 0) atomicAdd(&cnt[b], 1);          // counts only: order is free
        }
    }
    __syncwarp();
    // exclusive scan of the NC counters -> offsets; cnt becomes the cursor
    int* off = p.off + col * (long long)(p.NC + 1);
    int run = 0;
    for (int c0 = 0; c0 < p.NC; c0 += 32) {
        const int c = c0 + lane;
        const int v = c < p.NC ? cnt[c] : 0;
        int inc = v;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int u = __shfl_up_sync(FULL, inc, d);
            if (lane >= d) inc += u;
        }
        const int exc = run + inc - v;
        if (c < p.NC) { off[c] = exc; cnt[c] = exc; }
        run += __shfl_sync(FULL, inc, 31);
    }
    if (lane == 0) off[p.NC] = run;
    if (p.events && lane == 0) atomicAdd(p.events, (unsigned long long)run);
    __syncwarp();

    // pass 2: stable scatter
    int* dc = p.cin + col * p.c_in;
    float* dt = p.tin + col * p.c_in;
    const unsigned lt = (1u << lane) - 1u;
#pragma unroll
    for (int j = 0; j < MAXR; ++j) {
        if (j < nb) {
            const int ch = j * 32 + lane;
            const float t = tv[j];
            const int b = chunk_bin(t, p);
            const unsigned grp = __match_any_sync(FULL, b);
            int pos = 0;
            if (b >= 0) pos = cnt[b] + __popc(grp & lt);
            __syncwarp();
            if (b >= 0) {
                dc[pos] = ch;
                dt[pos] = t;
                if (lane == __ffs(grp) - 1) cnt[b] += __popc(grp);
            }
            __syncwarp();
        }
    }
}

__global__ void __launch_bounds__(128) k_bucketize_thread(BktParams p) {
    chain_release();
    chain_wait();
    extern __shared__ int s_cnt[];                  // [NC][blockDim]
    const long long col = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const bool live = col < p.n_cols;
    const int stride = blockDim.x;
    int* cnt = s_cnt + threadIdx.x;
    for (int c = 0; c < p.NC; ++c) cnt[c * stride] = 0;
    const float* src;
    long long cs;
    if (p.layout == VDT_LAYOUT_NHWC) { src = p.in + col * p.c_in; cs = 1; }
    else { const long long n = col / p.hw, s = col % p.hw; src = p.in + n * p.c_in * p.hw + s; cs = p.hw; }
    int run = 0;
    if (live) {
        for (int i = 0; i < p.c_in; ++i) {
            const int b = chunk_bin(__ldg(src + i * cs), p);
            if (b >= 0) cnt[b * stride]++;
        }
        int* off = p.off + col * (long long)(p.NC + 1);
        for (int c = 0; c < p.NC; ++c) {
            const int v = cnt[c * stride];
            off[c] = run;
            cnt[c * stride] = run;
            run += v;
        }
        off[p.NC] = run;
        int* dc = p.cin + col * p.c_in;
        float* dt = p.tin + col * p.c_in;
        for (int i = 0; i < p.c_in; ++i) {
            const float t = __ldg(src + i * cs);
            const int b = chunk_bin(t, p);
            if (b >= 0) {
                const int pos = cnt[b * stride]++;
                dc[pos] = i;
                dt[pos] = t;
            }
        }
    }
    if (p.events) {
        // one atomic per warp
        unsigned long long v = (unsigned long long)run;
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) v += __shfl_down_sync(FULL, v, d);
        if ((threadIdx.x & 31) == 0 && v) atomicAdd(p.events, v);
    }
}

}  // namespace

// One CTA per long column (NHWC rows with c_in > 512, e.g. a flattened FC
// input): each of the RW warps owns a contiguous segment of the row.  Pass 1
// counts the segment's events per chunk (warp-aggregated), the CTA turns the
// [chunk][warp] counts into exclusive offsets (chunk-major, so segments keep
// channel order inside a chunk), and pass 2 re-reads each segment and
// scatters it stably with the same in-window ranking as k_bucketize_warp.
constexpr int RW = 8;

__global__ void __launch_bounds__(RW * 32) k_bucketize_rows(BktParams p) {
    extern __shared__ int s_cnt[];                  // [RW][NC] counts, then cursors
    chain_release();
    chain_wait();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const long long col = blockIdx.x;
    const int seg = ((p.c_in + RW * 32 - 1) / (RW * 32)) * 32;
    const int c_lo = warp * seg, c_hi = min(p.c_in, c_lo + seg);
    int* cnt = s_cnt + warp * p.NC;
    for (int c = lane; c < p.NC; c += 32) cnt[c] = 0;
    __syncwarp();
    const float* src = p.in + col * p.c_in;
    const unsigned lt = (1u << lane) - 1u;
    for (int c0 = c_lo; c0 < c_hi; c0 += 32) {
        const int ch = c0 + lane;
        const float t = ch < c_hi ? __ldg(src + ch) : p.inf_time;
        const int b = chunk_bin(t, p);
        const unsigned grp = __match_any_sync(FULL, b);
        if (b >= 0 && lane == __ffs(grp) - 1) cnt[b] += __popc(grp);
        __syncwarp();
    }
    __syncthreads();
    // chunk totals -> exclusive chunk offsets (warp 0), then every warp's
    // cursor = chunk offset + counts of the earlier segments in that chunk
    int* off = p.off + col * (long long)(p.NC + 1);
    if (warp == 0) {
        int run = 0;
        for (int c0 = 0; c0 < p.NC; c0 += 32) {
            const int c = c0 + lane;
            int v = 0;
            if (c < p.NC)
                for (int w = 0; w < RW; ++w) v += s_cnt[w * p.NC + c];
            int inc = v;
#pragma unroll
            for (int d = 1; d < 32; d <<= 1) {
                const int u = __shfl_up_sync(FULL, inc, d);
                if (lane >= d) inc += u;
            }
            if (c < p.NC) {
                int base = run + inc - v;
                off[c] = base;
                for (int w = 0; w < RW; ++w) {
                    const int k = s_cnt[w * p.NC + c];
                    s_cnt[w * p.NC + c] = base;
                    base += k;
                }
            }
            run += __shfl_sync(FULL, inc, 31);
        }
        if (lane == 0) {
            off[p.NC] = run;
            if (p.events) atomicAdd(p.events, (unsigned long long)run);
        }
    }
    __syncthreads();
    int* dc = p.cin + col * p.c_in;
    float* dt = p.tin + col * p.c_in;
    for (int c0 = c_lo; c0 < c_hi; c0 += 32) {
        const int ch = c0 + lane;
        const float t = ch < c_hi ? __ldg(src + ch) : p.inf_time;
        const int b = chunk_bin(t, p);
        const unsigned grp = __match_any_sync(FULL, b);
        int pos = 0;
        if (b >= 0) pos = cnt[b] + __popc(grp & lt);
        __syncwarp();
        if (b >= 0) {
            dc[pos] = ch;
            dt[pos] = t;
            if (lane == __ffs(grp) - 1) cnt[b] += __popc(grp);
        }
        __syncwarp();
    }
}

cudaError_t launch_bucketize(const BktParams& p, cudaStream_t s) {
    if (p.n_cols <= 0) return cudaSuccess;
    if (p.layout == VDT_LAYOUT_NHWC && p.c_in > 512 && p.NC <= 1024) {
        const size_t smem = (size_t)RW * p.NC * sizeof(int);
        if (smem > 48 * 1024) {
            cudaError_t e = cudaFuncSetAttribute(k_bucketize_rows, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)smem);
            if (e != cudaSuccess) return e;
        }
        if (p.n_cols >= (1ll << 31)) return cudaErrorInvalidValue;
        return launch_chain(k_bucketize_rows, dim3((unsigned)p.n_cols), dim3(RW * 32), smem, s, p);
    }
    if (p.layout == VDT_LAYOUT_NHWC && p.c_in >= 32 && p.c_in <= 512) {
        const int warps = 8;
        const size_t smem = (size_t)warps * p.NC * sizeof(int);
        const long long blocks = (p.n_cols + warps - 1) / warps;
        if (p.c_in <= 128)
            return launch_chain(k_bucketize_warp<4>, dim3((unsigned)blocks), dim3(warps * 32), smem, s, p);
        return launch_chain(k_bucketize_warp<16>, dim3((unsigned)blocks), dim3(warps * 32), smem, s, p);
    }
    const int threads = 128;
    const size_t smem = (size_t)threads * p.NC * sizeof(int);
    if (smem > 227 * 1024) return cudaErrorInvalidValue;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(k_bucketize_thread,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    const long long blocks = (p.n_cols + threads - 1) / threads;
    return launch_chain(k_bucketize_thread, dim3((unsigned)blocks), dim3(threads), smem, s, p);
}

}  // namespace vdt
