/*
 * vdt_oracle.c -- CPU restatement of the VD-TTFS `vdttfs_cuda` hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker that the CUDA engine is
 * compared against; it is never linked into, loaded by, or called from the
 * product library (libvdttfs.so).  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / `--impl reference` legs of bench.py may load it.
 *
 * Every function restates one reference kernel or host helper, in the same
 * per-neuron operation order, so that fp32 results are bit-identical to the
 * reference's device code:
 *   - `a += w * l` in device code is contracted by nvcc into one FFMA; here it
 *     is written as fmaf(w, l, a).  The file is compiled with
 *     -ffp-contract=off so that no other expression is contracted.
 *   - sequential `carry += delta[i]`, `V += I` stay plain fp32 adds.
 *   - the LUTs use the host libm expf, exactly like update_LUTs does.
 *
 * Reference files (paths inside the Xarlley/VD-TTFS project):
 *   t1 = task1_lenet_mnist/vdttfs_cuda/snn_timesorted_earlyexit.cu
 *   t2 = task2_vgg16_cifar10/vdttfs_cuda/bench_vgg_eventdriven_timesorted_earlyexit.cu
 *   t3 = task3_dvsgesture/vdttfs_cuda/snn_inference_timesorted.cu
 *
 * Generalisations over the reference (all are compile-time macros or
 * hard-coded shapes there): T, delta (chunk width), the inter-layer stagger
 * TFS, the spatial shapes, channel counts and the padding are parameters.
 * One deliberate deviation, documented in orc_dvs_conv1: frames past T read
 * as zero (the reference reads the next pixel's frames when delta does not
 * divide T).
 *
 * Parallelism: the per-neuron loops carry `omp parallel for`; each neuron is
 * computed independently in the reference order, so the thread count never
 * changes a result.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_MAX_DELTA 1024

/* ------------------------------------------------------------------------ */
/* a1: update_LUTs  (t1:208-216, t2:236-243)                                 */
/* LUT_decay[t] = expf(-((float)t - td_integ) / tc_integ), t in [0, n_decay) */
/* LUT_th[t]    = vth * expf(-((float)t - td_fire) / tc_fire), t in [0, T)   */
/* n_decay is T (task 1) or T+1 (task 2).                                    */
/* ------------------------------------------------------------------------ */
void orc_update_luts(int T, int n_decay, float tc_integ, float td_integ,
                     float tc_fire, float td_fire, float vth_init,
                     float* lut_decay, float* lut_th) {
    for (int t = 0; t < n_decay; ++t)
        lut_decay[t] = expf(-((float)t - td_integ) / tc_integ);
    for (int t = 0; t < T; ++t)
        lut_th[t] = vth_init * expf(-((float)t - td_fire) / tc_fire);
}

/* ------------------------------------------------------------------------ */
/* a6: k_encode_image (t1:32-42, t2:32-42), logarithmic TTFS encoder.        */
/* The device version uses CUDA logf; this one uses libm logf, so the two    */
/* can differ only where td - tc*ln(x) lies within an ulp of an integer.      */
/* ------------------------------------------------------------------------ */
void orc_encode_log(const float* img, float* out, long n, float tc, float td,
                    int T, float inf_time) {
#pragma omp parallel for schedule(static)
    for (long i = 0; i < n; ++i) {
        float x = img[i];
        if (x < 1e-5) { out[i] = inf_time; continue; }
        float tf = fmaf(-tc, logf(x), td);
        if (tf < 0.0f) tf = 0.0f;
        float ts = ceilf(tf);
        out[i] = (ts > (float)T) ? inf_time : ts;
    }
}

/* Linear TTFS encoder of the synthetic workloads: t = floor((1 - x) * T);   */
/* x < 1e-5 (the zeroed pixels) never spikes, mirroring a6's cut-off.        */
void orc_encode_linear(const float* img, float* out, long n, int T, float inf_time) {
#pragma omp parallel for schedule(static)
    for (long i = 0; i < n; ++i) {
        float x = img[i];
        if (x < 1e-5f) { out[i] = inf_time; continue; }
        float t = floorf((1.0f - x) * (float)T);
        out[i] = (t > (float)T) ? inf_time : t;
    }
}

/* ------------------------------------------------------------------------ */
/* a2 / a7: k_bucketize (t1:45-80, t2:45-81), k_bucketize_conv (t3:70-90),   */
/* k_bucketize_fc (t3:93-106).                                               */
/*                                                                          */
/* Column `col` holds c_in channels.  layout 0 (NHWC / [N,F]): channel i of   */
/* column col is in[col*c_in + i].  layout 1 (NCHW): col = n*hw + s and       */
/* channel i is in[n*c_in*hw + i*hw + s].                                    */
/* tb_mode 0 (tasks 1/2): tb = max(0, (int)floorf(t - tfs)), kept iff tb < T. */
/* tb_mode 1 (task 3):    tb = (int)t, kept iff 0 <= tb < T.                  */
/* Outputs: off[col*(NC+1) + c] exclusive chunk offsets, off[..+NC] = total; */
/* cin/tin[col*c_in + p] the kept events in increasing channel order within  */
/* each chunk (stable counting sort).  Returns the total event count.        */
/* ------------------------------------------------------------------------ */
static inline int orc_tb(float t, float tfs, int tb_mode, int T, float inf_time, int* ok) {
    *ok = 0;
    if (!(t < inf_time)) return 0;
    int tb;
    if (tb_mode == 0) {
        tb = (int)floorf(t - tfs);
        if (tb < 0) tb = 0;
        if (tb < T) *ok = 1;
    } else {
        tb = (int)t;
        if (tb >= 0 && tb < T) *ok = 1;
    }
    return tb;
}

long long orc_bucketize(const float* in, long n_cols, int c_in, int layout, long hw,
                        int T, int delta, float tfs, int tb_mode, float inf_time,
                        int* off, int* cin, float* tin) {
    const int NC = (T + delta - 1) / delta, OS = NC + 1;
    if (delta < 1 || delta > ORC_MAX_DELTA || NC > ORC_MAX_DELTA) return -1;
    long long total = 0;
#pragma omp parallel for schedule(static) reduction(+:total)
    for (long col = 0; col < n_cols; ++col) {
        const float* src;
        long cs;
        if (layout == 0) { src = in + col * (long)c_in; cs = 1; }
        else { long n = col / hw, s = col % hw; src = in + n * (long)c_in * hw + s; cs = hw; }
        int cnt[ORC_MAX_DELTA + 1];
        int cur[ORC_MAX_DELTA + 1];
        for (int c = 0; c < NC; ++c) cnt[c] = 0;
        for (int i = 0; i < c_in; ++i) {
            int ok; int tb = orc_tb(src[i * cs], tfs, tb_mode, T, inf_time, &ok);
            if (ok) cnt[tb / delta]++;
        }
        int run = 0;
        for (int c = 0; c < NC; ++c) { off[col * OS + c] = run; cur[c] = run; run += cnt[c]; }
        off[col * OS + NC] = run;
        total += run;
        int* dc = cin + col * (long)c_in;
        float* dt = tin + col * (long)c_in;
        for (int i = 0; i < c_in; ++i) {
            float t = src[i * cs];
            int ok; int tb = orc_tb(t, tfs, tb_mode, T, inf_time, &ok);
            if (ok) { int p = cur[tb / delta]++; dc[p] = i; dt[p] = t; }
        }
    }
    return total;
}

/* ------------------------------------------------------------------------ */
/* a3: k_conv_bucketed (t1:83-162, t2:84-170).                               */
/* Neuron nid = ((img*H_out + h)*W_out + w)*C_out + c_out (NHWC output).      */
/* Conv taps read input column (img, h - pad_h + kh, w - pad_w + kw) and skip */
/* out-of-range taps (t2:136-141; t1 is the pad=0 "valid" case).  is_fc uses  */
/* one column per image and kernel [C_in, C_out].                            */
/* lut_mode 0: LUT_decay index = tb (t1:128,144).  lut_mode 1: index =        */
/* clamp((int)t_in, 0, T) (t2:132,150).                                      */
/* fetched counts inner-loop executions like task2 macs/stat_timesorted_macs */
/* .cu:136,155 (`my_macs`).                                                  */
/* ------------------------------------------------------------------------ */
long long orc_conv_bucketed(const int* off, const int* bcin, const float* btin,
                            const float* kernel, const float* bias,
                            const float* lut_decay, const float* lut_th, int t_min,
                            int B, int H_in, int W_in, int C_in,
                            int H_out, int W_out, int C_out, int K_h, int K_w,
                            int pad_h, int pad_w, int is_fc,
                            int T, int delta, float tfs, int lut_mode, float inf_time,
                            float* out) {
    const int NC = (T + delta - 1) / delta, OS = NC + 1;
    const long total = (long)B * H_out * W_out * C_out;
    if (delta < 1 || delta > ORC_MAX_DELTA) return -1;
    long long fetched = 0;
#pragma omp parallel for schedule(dynamic, 4096) reduction(+:fetched)
    for (long nid = 0; nid < total; ++nid) {
        int c_out = (int)(nid % C_out);
        long r = nid / C_out;
        int w_out = 0, h_out = 0; long img;
        if (is_fc) { img = r; }
        else { w_out = (int)(r % W_out); r /= W_out; h_out = (int)(r % H_out); img = r / H_out; }
        float carry = bias[c_out];
        float result = inf_time;
        float d[ORC_MAX_DELTA];
        for (int tau = 0; tau < NC; ++tau) {
            for (int i = 0; i < delta; ++i) d[i] = 0.0f;
            const int base = tau * delta;
            for (int kh = 0; kh < (is_fc ? 1 : K_h); ++kh) {
                int h_in = h_out - pad_h + kh;
                if (!is_fc && (h_in < 0 || h_in >= H_in)) continue;
                for (int kw = 0; kw < (is_fc ? 1 : K_w); ++kw) {
                    int w_in = w_out - pad_w + kw;
                    if (!is_fc && (w_in < 0 || w_in >= W_in)) continue;
                    long col = is_fc ? img : ((img * H_in + h_in) * W_in + w_in);
                    int s = off[col * OS + tau], e = off[col * OS + tau + 1];
                    const int* bc = bcin + col * (long)C_in;
                    const float* bt = btin + col * (long)C_in;
                    long wbase = is_fc ? 0 : (long)(kh * K_w + kw) * C_in;
                    for (int idx = s; idx < e; ++idx) {
                        int ci = bc[idx]; float t_in = bt[idx];
                        int tb = (int)floorf(t_in - tfs); if (tb < 0) tb = 0;
                        int ti;
                        if (lut_mode == 0) ti = tb;
                        else { ti = (int)t_in; if (ti < 0) ti = 0; else if (ti > T) ti = T; }
                        d[tb - base] = fmaf(kernel[(wbase + ci) * C_out + c_out], lut_decay[ti], d[tb - base]);
                        ++fetched;
                    }
                }
            }
            for (int i = 0; i < delta; ++i) {
                int t = base + i;
                if (t >= T) break;
                carry += d[i];
                float th = lut_th[t];
                if (t >= t_min && carry >= th && th >= 1e-5f) { result = (float)t; break; }
            }
            if (result < inf_time) break;
        }
        out[nid] = result;
    }
    return fetched;
}

/* ------------------------------------------------------------------------ */
/* a4: k_layer_vmem (t2:172-190).  Dense membrane readout of the last layer. */
/* ------------------------------------------------------------------------ */
void orc_layer_vmem(const float* in, const float* kernel, const float* bias,
                    const float* lut_decay, int B, int C_in, int C_out,
                    int T, float tfs, float inf_time, float* out) {
#pragma omp parallel for schedule(static)
    for (long id = 0; id < (long)B * C_out; ++id) {
        long img = id / C_out; int c = (int)(id % C_out);
        float acc = 0.0f;
        for (int i = 0; i < C_in; ++i) {
            float t = in[img * C_in + i];
            if (t < inf_time && (t - tfs) <= (float)T) {
                int ti = (int)t; if (ti < 0) ti = 0; else if (ti > T) ti = T;
                acc = fmaf(kernel[(long)i * C_out + c], lut_decay[ti], acc);
            }
        }
        out[id] = acc + bias[c];
    }
}

/* ------------------------------------------------------------------------ */
/* a5: k_pooling (t1:164-181, t2:192-209): 2x2 stride-2 min, NHWC.           */
/* ------------------------------------------------------------------------ */
void orc_pool_min(const float* in, float* out, int B, int H_in, int W_in, int C, float inf_time) {
    const int H_out = H_in / 2, W_out = W_in / 2;
#pragma omp parallel for schedule(static)
    for (long idx = 0; idx < (long)B * H_out * W_out * C; ++idx) {
        long b = idx / ((long)H_out * W_out * C);
        long li = idx % ((long)H_out * W_out * C);
        int c = (int)(li % C), w = (int)((li / C) % W_out), h = (int)(li / C / W_out);
        float m = inf_time;
        for (int i = 0; i < 2; ++i)
            for (int j = 0; j < 2; ++j) {
                int ch = h * 2 + i, cw = w * 2 + j;
                if (ch < H_in && cw < W_in) {
                    float t = in[b * ((long)H_in * W_in * C) + ((long)ch * W_in + cw) * C + c];
                    if (t < m) m = t;
                }
            }
        out[idx] = m;
    }
}

/* ------------------------------------------------------------------------ */
/* Readouts.  argmin_first: t1:313-315 (strict <, starts at INF, -1 if no   */
/* class fires).  argmin_lowest: t3:295-296 (starts at class 0, strict <).   */
/* argmax: t2:391-392 (strict >, starts at -1e9, -1 if all <= -1e9).         */
/* ------------------------------------------------------------------------ */
void orc_readout(const float* out, int B, int K, int mode, float inf_time, int* pred) {
    for (long b = 0; b < B; ++b) {
        const float* o = out + b * (long)K;
        int p;
        if (mode == 0) {
            float m = inf_time; p = -1;
            for (int i = 0; i < K; ++i) if (o[i] < m) { m = o[i]; p = i; }
        } else if (mode == 1) {
            float m = o[0]; p = 0;
            for (int i = 1; i < K; ++i) if (o[i] < m) { m = o[i]; p = i; }
        } else {
            float m = -1e9f; p = -1;
            for (int i = 0; i < K; ++i) if (o[i] > m) { m = o[i]; p = i; }
        }
        pred[b] = p;
    }
}

/* ======================================================================== */
/* Task 3 (CuLIF, no LUT).  decay/threshold are passed in (t3:24-27).        */
/* ======================================================================== */

/* conv1_raw_early (t3:30-65): dense multi-spike 3x3 conv over raw frames    */
/* [N, C_in, H, W, T] (time innermost), OIHW weights, output NCHW.  Per      */
/* chunk: in_val[t] = fma(w, frame, in_val[t]) over c_in, ky, kx; then the   */
/* CuLIF scan I = fma(I, decay, in_val[t]); V += I; fire at V >= th.  The    */
/* scan has no t < T guard (t3:59-62).  Frames at t >= T read as 0 here.     */
void orc_dvs_conv1(const float* frames, const float* w, int N, int C_in, int C_out,
                   int H, int W, int K, int T, int delta, float decay, float th, float* out) {
    const int pad = K / 2;
    const long total = (long)N * C_out * H * W;
#pragma omp parallel for schedule(dynamic, 1024)
    for (long idx = 0; idx < total; ++idx) {
        long n = idx / ((long)C_out * H * W);
        long rem = idx % ((long)C_out * H * W);
        int co = (int)(rem / ((long)H * W)), y = (int)((rem / W) % H), x = (int)(rem % W);
        float I = 0.0f, V = 0.0f, res = 9999.0f;
        float iv[ORC_MAX_DELTA];
        int done = 0;
        for (int chunk = 0; chunk < T && !done; chunk += delta) {
            for (int t = 0; t < delta; ++t) iv[t] = 0.0f;
            for (int ci = 0; ci < C_in; ++ci)
                for (int ky = 0; ky < K; ++ky) {
                    int iy = y + ky - pad; if (iy < 0 || iy >= H) continue;
                    for (int kx = 0; kx < K; ++kx) {
                        int ix = x + kx - pad; if (ix < 0 || ix >= W) continue;
                        float wv = w[(((long)co * C_in + ci) * K + ky) * K + kx];
                        const float* f = frames + ((((n * C_in + ci) * H + iy) * (long)W + ix) * T);
                        for (int t = 0; t < delta; ++t) {
                            float v = (chunk + t < T) ? f[chunk + t] : 0.0f;
                            iv[t] = fmaf(wv, v, iv[t]);
                        }
                    }
                }
            for (int t = 0; t < delta; ++t) {
                I = fmaf(I, decay, iv[t]); V += I;
                if (V >= th) { res = (float)(chunk + t); done = 1; break; }
            }
        }
        out[idx] = res;
    }
}

/* conv_bucketed_early (t3:109-143): NCHW single-spike input bucketed by site */
/* (orc_bucketize layout 1, tb_mode 1).  in_val[tt-base] += w (no LUT, plain  */
/* add), weights OIHW, then the same CuLIF scan.                             */
long long orc_dvs_conv(const int* off, const int* bcin, const float* btin, const float* w,
                       int N, int C_in, int C_out, int H, int W, int K,
                       int T, int delta, float decay, float th, float* out) {
    const int NC = (T + delta - 1) / delta, OS = NC + 1, pad = K / 2;
    const long total = (long)N * C_out * H * W;
    long long fetched = 0;
#pragma omp parallel for schedule(dynamic, 1024) reduction(+:fetched)
    for (long idx = 0; idx < total; ++idx) {
        long n = idx / ((long)C_out * H * W);
        long rem = idx % ((long)C_out * H * W);
        int co = (int)(rem / ((long)H * W)), y = (int)((rem / W) % H), x = (int)(rem % W);
        float I = 0.0f, V = 0.0f, res = 9999.0f;
        float iv[ORC_MAX_DELTA];
        int done = 0;
        for (int ch = 0; ch < NC && !done; ++ch) {
            const int base = ch * delta;
            for (int t = 0; t < delta; ++t) iv[t] = 0.0f;
            for (int ky = 0; ky < K; ++ky) {
                int iy = y + ky - pad; if (iy < 0 || iy >= H) continue;
                for (int kx = 0; kx < K; ++kx) {
                    int ix = x + kx - pad; if (ix < 0 || ix >= W) continue;
                    long site = (n * H + iy) * (long)W + ix;
                    int s = off[site * OS + ch], e = off[site * OS + ch + 1];
                    const int* sc = bcin + site * (long)C_in;
                    const float* st = btin + site * (long)C_in;
                    for (int p = s; p < e; ++p) {
                        int ci = sc[p]; int tt = (int)st[p];
                        iv[tt - base] += w[(((long)co * C_in + ci) * K + ky) * K + kx];
                        ++fetched;
                    }
                }
            }
            for (int t = 0; t < delta; ++t) {
                I = fmaf(I, decay, iv[t]); V += I;
                if (V >= th) { res = (float)(base + t); done = 1; break; }
            }
        }
        out[idx] = res;
    }
    return fetched;
}

/* pool_chunk_early (t3:146-168): spiking 2x2 pool, NCHW.  A CuLIF neuron    */
/* driven by 1.0 at each input's spike time (set, not added), early exit.    */
void orc_dvs_pool(const float* in, float* out, int N, int C, int H_in, int W_in,
                  int T, int delta, float decay, float th) {
    const int H_out = H_in / 2, W_out = W_in / 2;
    const long total = (long)N * C * H_out * W_out;
#pragma omp parallel for schedule(static)
    for (long idx = 0; idx < total; ++idx) {
        long n = idx / ((long)C * H_out * W_out);
        long rem = idx % ((long)C * H_out * W_out);
        int c = (int)(rem / ((long)H_out * W_out)), yo = (int)((rem / W_out) % H_out), xo = (int)(rem % W_out);
        float I = 0.0f, V = 0.0f, res = 9999.0f;
        long base = (n * C + c) * (long)H_in * W_in;
        float iv[ORC_MAX_DELTA];
        int done = 0;
        for (int chunk = 0; chunk < T && !done; chunk += delta) {
            for (int t = 0; t < delta; ++t) iv[t] = 0.0f;
            for (int dy = 0; dy < 2; ++dy)
                for (int dx = 0; dx < 2; ++dx) {
                    float tf = in[base + (long)(yo * 2 + dy) * W_in + (xo * 2 + dx)];
                    if (tf >= (float)chunk && tf < (float)(chunk + delta)) iv[(int)tf - chunk] = 1.0f;
                }
            for (int t = 0; t < delta; ++t) {
                I = fmaf(I, decay, iv[t]); V += I;
                if (V >= th) { res = (float)(chunk + t); done = 1; break; }
            }
        }
        out[idx] = res;
    }
}

/* fc1_bucketed_recurrent (t3:171-200): one sample, F_out neurons stepping   */
/* in lock-step.  Feed-forward events in_ff[tt-base] += W[i*F_in + j]; each  */
/* step in_rec = sum over neurons j that fired on the previous step of       */
/* W_rec[i*F_out + j] (j ascending), I = fma(I, decay, in_ff[t]) + in_rec,   */
/* V += I; first crossing records base+t and sets V = -10000.  No early exit.*/
void orc_dvs_fc1_rec(const int* off, const int* bcin, const float* btin,
                     const float* w, const float* w_rec, int N, int F_in, int F_out,
                     int T, int delta, float decay, float th, float* out) {
    const int NC = (T + delta - 1) / delta, OS = NC + 1;
#pragma omp parallel for schedule(dynamic, 1)
    for (long n = 0; n < N; ++n) {
        float* I = (float*)malloc(sizeof(float) * F_out * 3);
        float* V = I + F_out;
        float* fire = V + F_out;
        unsigned char* has = (unsigned char*)calloc((size_t)F_out * 2, 1);
        unsigned char* prev = has + F_out;
        float* ff = (float*)malloc(sizeof(float) * (size_t)F_out * delta);
        unsigned char* now = (unsigned char*)malloc((size_t)F_out);
        for (int i = 0; i < F_out; ++i) { I[i] = 0.0f; V[i] = 0.0f; fire[i] = 9999.0f; }
        const int* sc = bcin + n * (long)F_in;
        const float* st = btin + n * (long)F_in;
        for (int ch = 0; ch < NC; ++ch) {
            const int base = ch * delta;
            int s = off[n * OS + ch], e = off[n * OS + ch + 1];
            for (int i = 0; i < F_out; ++i) {
                float* f = ff + (long)i * delta;
                for (int t = 0; t < delta; ++t) f[t] = 0.0f;
                for (int p = s; p < e; ++p) { int j = sc[p]; int tt = (int)st[p]; f[tt - base] += w[(long)i * F_in + j]; }
            }
            for (int t = 0; t < delta; ++t) {
                for (int i = 0; i < F_out; ++i) {
                    float in_rec = 0.0f;
                    for (int j = 0; j < F_out; ++j) if (prev[j]) in_rec += w_rec[(long)i * F_out + j];
                    I[i] = fmaf(I[i], decay, ff[(long)i * delta + t]) + in_rec;
                    V[i] += I[i];
                    now[i] = 0;
                    if (V[i] >= th && !has[i]) { now[i] = 1; has[i] = 1; fire[i] = (float)(base + t); V[i] = -10000.0f; }
                }
                memcpy(prev, now, (size_t)F_out);
            }
        }
        for (int i = 0; i < F_out; ++i) out[n * (long)F_out + i] = fire[i];
        free(I); free(has); free(ff); free(now);
    }
}

/* fc2_bucketed_early (t3:203-225): bucketed FC, weights [F_out, F_in].      */
long long orc_dvs_fc2(const int* off, const int* bcin, const float* btin, const float* w,
                      int N, int F_in, int F_out, int T, int delta, float decay, float th,
                      float* out) {
    const int NC = (T + delta - 1) / delta, OS = NC + 1;
    long long fetched = 0;
#pragma omp parallel for schedule(static) reduction(+:fetched)
    for (long idx = 0; idx < (long)N * F_out; ++idx) {
        long n = idx / F_out; int i = (int)(idx % F_out);
        float I = 0.0f, V = 0.0f, res = 9999.0f;
        const int* sc = bcin + n * (long)F_in;
        const float* st = btin + n * (long)F_in;
        float iv[ORC_MAX_DELTA];
        int done = 0;
        for (int ch = 0; ch < NC && !done; ++ch) {
            const int base = ch * delta;
            for (int t = 0; t < delta; ++t) iv[t] = 0.0f;
            int s = off[n * OS + ch], e = off[n * OS + ch + 1];
            for (int p = s; p < e; ++p) { int j = sc[p]; int tt = (int)st[p]; iv[tt - base] += w[(long)i * F_in + j]; ++fetched; }
            for (int t = 0; t < delta; ++t) {
                I = fmaf(I, decay, iv[t]); V += I;
                if (V >= th) { res = (float)(base + t); done = 1; break; }
            }
        }
        out[idx] = res;
    }
    return fetched;
}

int orc_max_delta(void) { return ORC_MAX_DELTA; }

/* OpenMP worker count for every later call (launchers such as torchrun set
   OMP_NUM_THREADS=1 per process; the CPU baselines use all host cores). */
#ifdef _OPENMP
#include <omp.h>
#endif
int orc_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
    return omp_get_max_threads();
#else
    (void)n;
    return 1;
#endif
}
