// k_thread.cu -- integrator for narrow conv layers (C_out <= 16, K*K*C_in <=
// 255 inputs per pixel): one thread per output pixel, all of its output
// channels.  Same results as k_bucketize + k_conv_bucketed (t1:45-162,
// t2:45-170), bit for bit.
//
// A warp of 32 pixels replaces 32 warps of k_dense, which for a 6-channel
// layer would leave 26 of 32 lanes idle.  With at most 32 inputs per pixel
// the thread turns its pixel's events into keys (step << 18 | input index <<
// 13 | LUT index), so increasing key order is the reference's order: by
// step, and inside a step by (tap, channel) -- each neuron's FMA chain.  The
// keys are appended to the thread's own shared-memory column and sorted by
// insertion over the events only (a pixel has few events; a fully unrolled
// sorting network was slower, its code overflowing the instruction cache).
// The thread then walks its sorted events, adds w[input][c] * LUT to every
// channel's open step, and closes a step when the next key leaves it
// (lanes.h closes; input-free steps by bisection).  Wider pixels order their
// events by per-step lists instead (WIDE below).
#include "lanes.h"
#include "vdt_internal.h"

namespace vdt {
namespace {

constexpr int TW = 4;             // warps per CTA
constexpr int TKEYS = 32;         // inputs per pixel at most (keys per thread column)
constexpr int NT = TW * 32;
constexpr int LIST_END = 0xff;    // wide form: end of a step's event list (inputs 0..254)

// weight row stride in floats: past CO, to the next multiple of the vector
// width (4, or 2 when CO is not a multiple of 4) that is an odd number of
// vectors, so that the rows of different inputs read by one phase of a
// vector load start in different bank groups (a CO-float row would put them
// in one or two)
__host__ __device__ constexpr int row_stride(int CO) {
    return CO % 4 == 0 ? ((CO / 4) % 2 == 0 ? CO + 4 : CO + 8) : ((CO / 2) % 2 == 0 ? CO + 2 : CO + 4);
}

// floats of a weight table of n rows, rounded up to a multiple of 4 (the
// int4 table after it stays 16-byte aligned)
__host__ __device__ constexpr int w_floats(int n, int sw) { return (n * sw + 3) & ~3; }

// acc[c] = fma(w[f][c], lv, acc[c]) for the CO channels of weight row f
template <int CO, int SW>
__device__ __forceinline__ void add_row(Lanes<CO>& nu, const float* s_w, int f, float lv) {
    static_assert(CO % 2 == 0 && SW % (CO % 4 == 0 ? 4 : 2) == 0, "row vectors");
    if constexpr (CO % 4 == 0) {
        const float4* wr = reinterpret_cast<const float4*>(s_w + f * SW);
#pragma unroll
        for (int q = 0; q < CO / 4; ++q) {
            const float4 w4 = wr[q];
            const float w[4] = {w4.x, w4.y, w4.z, w4.w};
            float a[4] = {nu.acc[4 * q], nu.acc[4 * q + 1], nu.acc[4 * q + 2], nu.acc[4 * q + 3]};
            fma_lanes<4>(a, w, lv);
#pragma unroll
            for (int j = 0; j < 4; ++j) nu.acc[4 * q + j] = a[j];
        }
    } else {
        const float2* wr = reinterpret_cast<const float2*>(s_w + f * SW);
#pragma unroll
        for (int q = 0; q < CO / 2; ++q) {
            const float2 w2 = wr[q];
            const float w[2] = {w2.x, w2.y};
            float a[2] = {nu.acc[2 * q], nu.acc[2 * q + 1]};
            fma_lanes<2>(a, w, lv);
            nu.acc[2 * q] = a[0];
            nu.acc[2 * q + 1] = a[1];
        }
    }
}

// a thread's byte column in shared memory, word-interleaved across the CTA:
// byte k of thread t at ((k / 4) * NT + t) * 4 + k % 4, so every lane of a
// warp reads its own bank whatever entry it wants
struct ByteCol {
    unsigned char* base;                                     // column start of the CTA
    __device__ __forceinline__ unsigned char& operator[](int k) const {
        return base[(((k >> 2) * NT + (int)threadIdx.x) << 2) + (k & 3)];
    }
};
__host__ __device__ constexpr size_t col_bytes(int n) { return (size_t)((n + 3) / 4) * NT * 4; }

// POOL: the layer's 2x2 min pool (k_pooling t1:164-181, t2:192-209) fused
// in: thread t integrates pixel (2 ph + (t & 3) / 2, 2 pw + (t & 1)) of
// pooled position t / 4, the four lanes of a quad take the minimum of their
// first-spike times by shuffles and one writes the pooled map p.out
// [B, H_out / 2, W_out / 2, C_out]; a last odd row or column is not computed
// (no pooled output reads it).  n_thr counts threads (pixels, or 4 per pooled
// position).
//
// WIDE (33 to 255 inputs per pixel): the events are ordered by one list per
// step instead of sorted keys.  A single pass over the inputs, from the last
// to the first, pushes each event's input index onto its step's list (byte
// columns: a head per step, a link per input, and for LUTs indexed by t_in
// the event's LUT index), so each list runs in input order -- the
// reference's chain order inside the step; the walk takes the steps in
// order and follows each list.
template <int CO, int MINB, bool POOL, bool WIDE>
__global__ void __launch_bounds__(TW * 32, MINB) k_thread(IntegParams p, const float* __restrict__ in,
                                                          long long n_thr) {
    extern __shared__ __align__(16) float tsm[];
    __shared__ int s_floor, s_mono;
    chain_release();
    constexpr int SW = row_stride(CO);
    const int fan = p.K * p.K * p.C_in;
    const int NF = WIDE ? fan : TKEYS;                       // weight rows
    const int NTAP = WIDE ? p.K * p.K : TKEYS;               // tap rows: per tap (wide), per input
    // weights padded to CO columns (zeros past C_out), one row per input
    float* s_w = tsm;                                        // [NF][SW]
    // (the weight table rounded up to 16 bytes: SW = 10 with an odd row count
    // would leave the int4 table misaligned)
    int4* s_tap = reinterpret_cast<int4*>(s_w + w_floats(NF, SW));   // kh - pad, kw - pad, offset
    float* s_decay = reinterpret_cast<float*>(s_tap + NTAP);
    float* s_th = s_decay + p.decay_len;
    float* s_thx = s_th + p.T;
    // per-thread columns after the tables: narrow, fan int keys; wide, byte
    // columns of list heads [T], list links [fan] and LUT indices [fan], each
    // word-interleaved (ByteCol)
    int* s_keys = reinterpret_cast<int*>(s_thx + p.T);      // [fan][NT]
    unsigned char* s_head = reinterpret_cast<unsigned char*>(s_thx + p.T);
    unsigned char* s_next = s_head + col_bytes(p.T);
    unsigned char* s_lut = s_next + col_bytes(fan);         // LUT by t_in only
    for (int i = threadIdx.x; i < NF * SW; i += blockDim.x) {
        const int f = i / SW, c = i - f * SW;
        s_w[i] = (f < fan && c < p.C_out) ? p.W[f * p.C_out + c] : 0.0f;
    }
    for (int f = threadIdx.x; f < NTAP; f += blockDim.x) {
        const int tap = WIDE ? f : f / p.C_in, c = WIDE ? 0 : f - tap * p.C_in;
        const int kh = tap / p.K, kw = tap - kh * p.K;
        s_tap[f] = make_int4(kh - p.pad, kw - p.pad, (kh * p.W_in + kw) * p.C_in + c, 0);
    }
    for (int i = threadIdx.x; i < p.decay_len; i += blockDim.x) s_decay[i] = p.lut_decay[i];
    const ThTables tt = stage_thresholds(p, s_th, s_thx, &s_floor, &s_mono);   // ends with __syncthreads
    chain_wait();                                            // the input map is complete

    const long long thr = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    // a pooled run keeps every thread to the end (the quads' shuffles); others
    // leave at once past the last pixel
    if (!POOL && thr >= n_thr) return;
    const bool valid = thr < n_thr;
    int w_out, h_out;
    long long img, pq = 0;
    if constexpr (POOL) {
        const int PW = p.W_out / 2, PH = p.H_out / 2;
        pq = valid ? thr >> 2 : 0;
        const int sub = (int)(thr & 3);
        const int pw = (int)(pq % PW);
        const long long rq = pq / PW;
        w_out = 2 * pw + (sub & 1);
        h_out = 2 * (int)(rq % PH) + (sub >> 1);
        img = rq / PH;
    } else {
        w_out = (int)(thr % p.W_out);
        const long long r = thr / p.W_out;
        h_out = (int)(r % p.H_out);
        img = r / p.H_out;
    }
    const long long pix = (img * p.H_out + h_out) * p.W_out + w_out;
    // input (kh, kw, c) sits at base + offset when its row and column are inside the map
    const long long base = ((img * p.H_in + (h_out - p.pad)) * p.W_in + (w_out - p.pad)) * p.C_in;

    // the event of the input at spike time t, or -1: its step and LUT index
    auto event_at = [&](float t, int& ti) -> int {
        if (!(t < p.inf_time)) return -1;
        int b = (int)floorf(t - p.tfs);
        if (b < 0) b = 0;
        if (b >= p.T) return -1;
        if (p.lut_mode == VDT_LUT_BY_TB) {
            ti = b;
        } else {
            ti = (int)t;
            ti = ti < 0 ? 0 : (ti > p.T ? p.T : ti);
        }
        return b;
    };
    // the same for input f (per-input tap table); a pixel whose whole window
    // lies inside the map (every pixel of a valid convolution) skips the
    // per-input row and column tests
    const bool inside = h_out >= p.pad && h_out - p.pad + p.K <= p.H_in && w_out >= p.pad &&
                        w_out - p.pad + p.K <= p.W_in;
    auto event_of = [&](int f, int& ti) -> int {
        const int4 tp = s_tap[f];
        if (!inside && ((unsigned)(h_out + tp.x) >= (unsigned)p.H_in || (unsigned)(w_out + tp.y) >= (unsigned)p.W_in))
            return -1;
        return event_at(__ldg(in + (base + tp.z)), ti);
    };
    const ByteCol head{s_head}, next{s_next}, lut{s_lut};
    if constexpr (WIDE) {
        // one list per step, linked through the input indices; inputs are
        // pushed from the last to the first, so each list runs in input order
        unsigned* hw = reinterpret_cast<unsigned*>(s_head) + threadIdx.x;
        for (int w = 0; w < (p.T + 3) / 4; ++w) hw[w * NT] = 0xffffffffu;   // LIST_END
        for (int tap = (valid ? NTAP : 0) - 1; tap >= 0; --tap) {
            const int4 tp = s_tap[tap];
            if ((unsigned)(h_out + tp.x) >= (unsigned)p.H_in || (unsigned)(w_out + tp.y) >= (unsigned)p.W_in) continue;
            const float* src = in + (base + tp.z);
            for (int c = p.C_in - 1; c >= 0; --c) {
                int ti = 0;
                const int b = event_at(__ldg(src + c), ti);
                if (b >= 0) {
                    const int f = tap * p.C_in + c;
                    next[f] = head[b];
                    head[b] = (unsigned char)f;
                    if (p.lut_mode != VDT_LUT_BY_TB) lut[f] = (unsigned char)ti;
                }
            }
        }
    }
    int n_ev = 0;
    if constexpr (!WIDE) {
        // the pixel's events as keys in the thread's own shared-memory column:
        // appended without a branch in input order (a non-event's key lands
        // past the last event and is overwritten or ignored), then sorted by
        // insertion over the events only (keys are distinct: the input index
        // is part of each; a step's keys are already in input order)
        int* col = s_keys + threadIdx.x;                     // entry e at col[e * NT]
        const int fan_t = valid ? fan : 0;
#pragma unroll 4
        for (int f = 0; f < fan_t; ++f) {                    // n_ev <= f < fan <= TKEYS
            int ti = 0;
            const int b = event_of(f, ti);
            col[n_ev * NT] = (int)(((unsigned)b << 18) | (unsigned)(f << 13) | (unsigned)ti);
            n_ev += b >= 0 ? 1 : 0;
        }
        for (int e = 1; e < n_ev; ++e) {
            const int key = col[e * NT];
            int pos = e;
            while (pos > 0) {
                const int prev = col[(pos - 1) * NT];
                if (prev < key) break;
                col[pos * NT] = prev;
                --pos;
            }
            col[pos * NT] = key;
        }
    }

    Lanes<CO> nu;
#pragma unroll
    for (int c = 0; c < CO; ++c) {
        nu.carry[c] = c < p.C_out ? __ldg(p.bias + c) : 0.0f;
        nu.res[c] = p.inf_time;
        nu.acc[c] = 0.0f;
        nu.alive[c] = valid && c < p.C_out;
    }
    if constexpr (WIDE) {
        int next_t = 0;
        for (int b = 0; b < p.T && nu.any(); ++b) {
            int f = head[b];
            if (f == LIST_END) continue;
            nu.close_empty(next_t, b, tt);
            do {
                const int ti = p.lut_mode == VDT_LUT_BY_TB ? b : lut[f];
                add_row<CO, SW>(nu, s_w, f, s_decay[ti]);
                f = next[f];
            } while (f != LIST_END);
            nu.close_step_bf(b, tt);
            next_t = b + 1;
        }
        if (nu.any()) nu.close_empty(next_t, p.T, tt);
    } else {
        int cur = -1, next_t = 0;
        for (int e = 0; e < n_ev; ++e) {
            const int m = s_keys[e * (TW * 32) + threadIdx.x];
            const int tb = m >> 18;
            if (tb != cur) {
                if (cur >= 0) {
                    nu.close_empty(next_t, cur, tt);
                    nu.close_step_bf(cur, tt);
                    next_t = cur + 1;
                    if (!nu.any()) break;                    // (cur stays closed)
                }
                cur = tb;
            }
            add_row<CO, SW>(nu, s_w, (m >> 13) & 31, s_decay[m & 0x1fff]);
        }
        if (cur >= 0 && nu.any()) {
            nu.close_empty(next_t, cur, tt);
            nu.close_step_bf(cur, tt);
            next_t = cur + 1;
        }
        if (nu.any()) nu.close_empty(next_t, p.T, tt);
    }
    if constexpr (POOL) {
#pragma unroll
        for (int c = 0; c < CO; ++c) {
            float m = nu.res[c];
            m = fminf(m, __shfl_xor_sync(FULL_MASK, m, 1));
            m = fminf(m, __shfl_xor_sync(FULL_MASK, m, 2));
            nu.res[c] = fminf(p.inf_time, m);                // k_pooling starts from INF_TIME
        }
        if (valid && (thr & 3) == 0) {
            float* o = p.out + pq * p.C_out;
#pragma unroll
            for (int c = 0; c < CO; ++c)
                if (c < p.C_out) o[c] = nu.res[c];
        }
    } else {
        float* o = p.out + pix * p.C_out;
#pragma unroll
        for (int c = 0; c < CO; ++c)
            if (c < p.C_out) o[c] = nu.res[c];
    }
}

// shared memory of one CTA: tables, then the per-thread columns
size_t thread_smem(int CO, int K, int fan, int T, int decay_len, bool wide, bool lut_tin) {
    const int nf = wide ? fan : TKEYS, ntap = wide ? K * K : TKEYS;
    size_t b = (size_t)w_floats(nf, row_stride(CO)) * sizeof(float) + (size_t)ntap * sizeof(int4) + (size_t)(decay_len + 2 * T) * sizeof(float);
    if (wide) b += col_bytes(T) + col_bytes(fan) + (lut_tin ? col_bytes(fan) : 0);
    else b += (size_t)fan * NT * sizeof(int);                // a key per input at most
    return b;
}

template <int CO, bool POOL, bool WIDE>
cudaError_t launch_thread_cw(const IntegParams& p, const float* in, cudaStream_t s, long long n_thr) {
    const int fan = p.K * p.K * p.C_in;
    const size_t smem = thread_smem(CO, p.K, fan, p.T, p.decay_len, WIDE, p.lut_mode != VDT_LUT_BY_TB);
    // registers: narrow, the keys' build plus lane state; wide, lane state
    // (96 for 16 channels: 5 CTAs per SM, which a 150-input layer's shared
    // memory also allows)
    // (42 for a 6-channel narrow layer: 12 CTAs per SM, which its shared
    // memory, a key column sized by the fan-in, also allows; the few spills
    // cost less than the added warps gain)
    constexpr int REGS = WIDE ? 4 * CO + 32 : (CO <= 6 ? 42 : CO <= 8 ? TKEYS + 2 * CO + 16 : TKEYS + 4 * CO);
    constexpr int MINB = (65536 / (TW * 32 * REGS)) > 12 ? 12 : (65536 / (TW * 32 * REGS));
    auto kern = k_thread<CO, MINB, POOL, WIDE>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    const long long blocks = (n_thr + TW * 32 - 1) / (TW * 32);
    if (blocks >= (1ll << 31)) return cudaErrorInvalidValue;
    return launch_chain(kern, dim3((unsigned)blocks), dim3(TW * 32), smem, s, p, in, n_thr);
}

template <bool POOL>
cudaError_t launch_thread_any(const IntegParams& p, const float* in, cudaStream_t s, long long n_thr) {
    // channel lanes: 6, 8, 12 or 16 (the layer's C_out rounded up)
    if (p.K * p.K * p.C_in > TKEYS) {
        if (p.C_out <= 6) return launch_thread_cw<6, POOL, true>(p, in, s, n_thr);
        if (p.C_out <= 8) return launch_thread_cw<8, POOL, true>(p, in, s, n_thr);
        if (p.C_out <= 12) return launch_thread_cw<12, POOL, true>(p, in, s, n_thr);
        return launch_thread_cw<16, POOL, true>(p, in, s, n_thr);
    }
    if (p.C_out <= 6) return launch_thread_cw<6, POOL, false>(p, in, s, n_thr);
    if (p.C_out <= 8) return launch_thread_cw<8, POOL, false>(p, in, s, n_thr);
    if (p.C_out <= 12) return launch_thread_cw<12, POOL, false>(p, in, s, n_thr);
    return launch_thread_cw<16, POOL, false>(p, in, s, n_thr);
}

}  // namespace

bool thread_supported(int K, int is_fc, int C_in, int C_out, int T, int decay_len) {
    if (is_fc || C_out > 16) return false;
    const int fan = K * K * C_in;
    if (fan <= TKEYS) {
        if (T >= (1 << 13)) return false;                      // 13-bit step / LUT index in the key
        return thread_smem(16, K, fan, T, decay_len, false, true) <= 48 * 1024;
    }
    // wide: byte counters, input and LUT indices (255 at most each)
    if (fan > 255 || T > 255 || decay_len > 256) return false;
    return thread_smem(16, K, fan, T, decay_len, true, true) <= 100 * 1024;
}

cudaError_t launch_thread(const IntegParams& p, const float* in, cudaStream_t s) {
    const long long n_pix = (long long)p.B * p.H_out * p.W_out;
    if (n_pix <= 0) return cudaSuccess;
    return launch_thread_any<false>(p, in, s, n_pix);
}

cudaError_t launch_thread_pooled(const IntegParams& p, const float* in, cudaStream_t s) {
    if (p.H_out < 2 || p.W_out < 2) return cudaErrorInvalidValue;
    const long long n_thr = 4ll * p.B * (p.H_out / 2) * (p.W_out / 2);
    if (n_thr <= 0) return cudaSuccess;
    return launch_thread_any<true>(p, in, s, n_thr);
}

}  // namespace vdt
