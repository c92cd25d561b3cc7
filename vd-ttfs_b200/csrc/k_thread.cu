// k_thread.cu -- integrator for narrow conv layers (K*K*C_in <= 32 inputs per
// pixel, C_out <= 16): one thread per output pixel, all of its output
// channels.  Same results as k_bucketize + k_conv_bucketed (t1:45-162,
// t2:45-170), bit for bit.
//
// A warp of 32 pixels replaces 32 warps of k_dense, which for a 6-channel
// layer would leave 26 of 32 lanes idle.  The thread turns its pixel's events
// into keys (step << 18 | input index << 13 | LUT index), so increasing key
// order is the reference's order: by step, and inside a step by (tap,
// channel) -- each neuron's FMA chain.  Each key is inserted in order into
// the thread's own shared-memory column as it is made (a pixel has few
// events; a fully unrolled sorting network was slower, its code overflowing
// the instruction cache).  The thread then walks its sorted events, adds
// w[input][c] * LUT to every channel's open step, and closes a step when the
// next key leaves it (lanes.h closes; input-free steps by bisection).
#include "lanes.h"
#include "vdt_internal.h"

namespace vdt {
namespace {

constexpr int TW = 4;             // warps per CTA
constexpr int TKEYS = 32;         // inputs per pixel at most (keys per thread column)

// POOL: the layer's 2x2 min pool (k_pooling t1:164-181, t2:192-209) fused
// in: thread t integrates pixel (2 ph + (t & 3) / 2, 2 pw + (t & 1)) of
// pooled position t / 4, the four lanes of a quad take the minimum of their
// first-spike times by shuffles and one writes the pooled map p.out
// [B, H_out / 2, W_out / 2, C_out]; a last odd row or column is not computed
// (no pooled output reads it).  n_thr counts threads (pixels, or 4 per pooled
// position).
template <int CO, int MINB, bool POOL>
__global__ void __launch_bounds__(TW * 32, MINB) k_thread(IntegParams p, const float* __restrict__ in,
                                                          long long n_thr) {
    extern __shared__ __align__(16) float tsm[];
    __shared__ int s_floor, s_mono;
    chain_release();
    const int fan = p.K * p.K * p.C_in;
    // weights padded to CO columns (zeros past C_out), one row per input
    float* s_w = tsm;                                        // [TKEYS][CO]
    int4* s_tap = reinterpret_cast<int4*>(s_w + TKEYS * CO); // per input: kh - pad, kw - pad, offset
    int* s_keys = reinterpret_cast<int*>(s_tap + TKEYS);    // [TKEYS][TW * 32]: a column per thread
    float* s_decay = reinterpret_cast<float*>(s_keys + TKEYS * TW * 32);
    float* s_th = s_decay + p.decay_len;
    float* s_thx = s_th + p.T;
    for (int i = threadIdx.x; i < TKEYS * CO; i += blockDim.x) {
        const int f = i / CO, c = i - f * CO;
        s_w[i] = (f < fan && c < p.C_out) ? p.W[f * p.C_out + c] : 0.0f;
    }
    for (int f = threadIdx.x; f < TKEYS; f += blockDim.x) {
        const int tap = f / p.C_in, c = f - tap * p.C_in;
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

    // the pixel's events as keys, inserted in order into the thread's own
    // shared-memory column (keys are distinct: the input index is part of
    // each; inputs come in index order, so a key of an already seen step
    // lands at the end at once)
    int* col = s_keys + threadIdx.x;                         // entry e at col[e * TW * 32]
    int n_ev = 0;
    const int fan_t = valid ? fan : 0;
#pragma unroll 4
    for (int f = 0; f < fan_t; ++f) {
        const int4 tp = s_tap[f];
        if ((unsigned)(h_out + tp.x) < (unsigned)p.H_in && (unsigned)(w_out + tp.y) < (unsigned)p.W_in) {
            const float t = __ldg(in + (base + tp.z));
            if (t < p.inf_time) {
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
                    const int key = (b << 18) | (f << 13) | ti;
                    int pos = n_ev;
                    while (pos > 0) {
                        const int prev = col[(pos - 1) * (TW * 32)];
                        if (prev < key) break;
                        col[pos * (TW * 32)] = prev;
                        --pos;
                    }
                    col[pos * (TW * 32)] = key;
                    ++n_ev;
                }
            }
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
    int cur = -1, next_t = 0;
    for (int e = 0; e < n_ev && nu.any(); ++e) {
        const int m = s_keys[e * (TW * 32) + threadIdx.x];
        const int tb = m >> 18;
        if (tb != cur) {
            if (cur >= 0) {
                nu.close_empty(next_t, cur, tt);
                nu.close_step_bf(cur, tt);
                next_t = cur + 1;
            }
            cur = tb;
        }
        const float lv = s_decay[m & 0x1fff];
        const float4* wr = reinterpret_cast<const float4*>(s_w + ((m >> 13) & 31) * CO);
#pragma unroll
        for (int q = 0; q < CO / 4; ++q) {
            const float4 w4 = wr[q];
            const float w[4] = {w4.x, w4.y, w4.z, w4.w};
            float a[4] = {nu.acc[4 * q], nu.acc[4 * q + 1], nu.acc[4 * q + 2], nu.acc[4 * q + 3]};
            fma_lanes<4>(a, w, lv);
#pragma unroll
            for (int j = 0; j < 4; ++j) nu.acc[4 * q + j] = a[j];
        }
    }
    if (cur >= 0 && nu.any()) {
        nu.close_empty(next_t, cur, tt);
        nu.close_step_bf(cur, tt);
        next_t = cur + 1;
    }
    if (nu.any()) nu.close_empty(next_t, p.T, tt);
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

size_t thread_smem(int CO, int T, int decay_len) {
    return (size_t)TKEYS * CO * sizeof(float) + TKEYS * sizeof(int4) + (size_t)TKEYS * TW * 32 * sizeof(int) +
           (size_t)(decay_len + 2 * T) * sizeof(float);
}

template <int CO, bool POOL>
cudaError_t launch_thread_c(const IntegParams& p, const float* in, cudaStream_t s, long long n_thr) {
    const size_t smem = thread_smem(CO, p.T, p.decay_len);
    constexpr int REGS = CO <= 8 ? TKEYS + 2 * CO + 16 : TKEYS + 4 * CO;   // keys + lane state
    constexpr int MINB = (65536 / (TW * 32 * REGS)) > 8 ? 8 : (65536 / (TW * 32 * REGS));
    auto kern = k_thread<CO, MINB, POOL>;
    const long long blocks = (n_thr + TW * 32 - 1) / (TW * 32);
    if (blocks >= (1ll << 31)) return cudaErrorInvalidValue;
    return launch_chain(kern, dim3((unsigned)blocks), dim3(TW * 32), smem, s, p, in, n_thr);
}

}  // namespace

bool thread_supported(int K, int is_fc, int C_in, int C_out, int T, int decay_len) {
    if (is_fc || K * K * C_in > TKEYS || C_out > 16) return false;
    if (T >= (1 << 13)) return false;                          // 13-bit step / LUT index in the key
    return thread_smem(16, T, decay_len) <= 48 * 1024;
}

cudaError_t launch_thread(const IntegParams& p, const float* in, cudaStream_t s) {
    const long long n_pix = (long long)p.B * p.H_out * p.W_out;
    if (n_pix <= 0) return cudaSuccess;
    if (p.C_out <= 8) return launch_thread_c<8, false>(p, in, s, n_pix);
    return launch_thread_c<16, false>(p, in, s, n_pix);
}

cudaError_t launch_thread_pooled(const IntegParams& p, const float* in, cudaStream_t s) {
    if (p.H_out < 2 || p.W_out < 2) return cudaErrorInvalidValue;
    const long long n_thr = 4ll * p.B * (p.H_out / 2) * (p.W_out / 2);
    if (n_thr <= 0) return cudaSuccess;
    if (p.C_out <= 8) return launch_thread_c<8, true>(p, in, s, n_thr);
    return launch_thread_c<16, true>(p, in, s, n_thr);
}

}  // namespace vdt
