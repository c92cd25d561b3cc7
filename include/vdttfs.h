/*
 * vdttfs.h -- C ABI of the B200-native VD-TTFS engine (libvdttfs.so).
 *
 * Drop-in for the `vdttfs_cuda` path of Xarlley/VD-TTFS.  The reference has no
 * library: each task is one .cu program whose `main` hard-codes the network,
 * and whose per-stage kernels/host helpers are what this header replaces.
 * File references below are paths inside the reference project:
 *   t1 = task1_lenet_mnist/vdttfs_cuda/snn_timesorted_earlyexit.cu
 *   t2 = task2_vgg16_cifar10/vdttfs_cuda/bench_vgg_eventdriven_timesorted_earlyexit.cu
 *   t3 = task3_dvsgesture/vdttfs_cuda/snn_inference_timesorted.cu
 *
 * Conventions
 *   - Every call returns an int status (VDT_OK = 0); the library never exits
 *     the process.  vdt_strerror() names a status; vdt_last_error() returns a
 *     per-thread message with details of the last failure.
 *   - "d_" pointers are device memory owned by the caller; "h_" pointers are
 *     host memory.  Calls taking a stream are asynchronous on it (NULL = the
 *     legacy default stream); the vdt_*_host calls are synchronous.
 *   - A vdt_model is immutable after load and may be shared by threads; a
 *     vdt_ctx (workspace + captured CUDA graphs) belongs to one thread/stream.
 *   - Spike times are fp32; inf_time (9999 in the reference) means "no spike".
 *   - Compile-time macros of the reference (TIME_WINDOW, CHUNK,
 *     TIME_FIRE_START, VTH_INIT, INF_TIME) are runtime fields of vdt_time_cfg.
 */
#ifndef VDTTFS_H
#define VDTTFS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct vdt_model vdt_model;
typedef struct vdt_ctx vdt_ctx;
typedef void* vdt_stream; /* cudaStream_t */

enum vdt_status {
    VDT_OK = 0,
    VDT_ERR_INVALID = 1,     /* bad argument / shape / descriptor */
    VDT_ERR_BLOB = 2,        /* malformed or truncated weight blob */
    VDT_ERR_CUDA = 3,        /* a CUDA runtime call failed */
    VDT_ERR_OOM = 4,         /* device allocation failed */
    VDT_ERR_UNSUPPORTED = 5, /* valid request outside what the kernels implement */
    VDT_ERR_CAPACITY = 6     /* batch above the ctx's max_batch */
};

/* layer kinds / padding / output kind (topology lives in each reference main) */
enum { VDT_CONV = 0, VDT_FC = 1 };
enum { VDT_PAD_VALID = 0, VDT_PAD_SAME = 1 };  /* t1 valid conv; t2 pad = K/2 */
enum { VDT_OUT_FIRE = 0, VDT_OUT_VMEM = 1 };   /* k_conv_bucketed / k_layer_vmem */
/* LUT_decay index: tb (t1:128,144) or clamp((int)t_in, 0, T) (t2:132,150) */
enum { VDT_LUT_BY_TB = 0, VDT_LUT_BY_TIN = 1 };
/* where the tables come from: a device kernel (exp in double, rounded) or
   the host libm expf exactly like update_LUTs (bit-identical tables) */
enum { VDT_LUT_DEVICE = 0, VDT_LUT_HOST_LIBM = 1 };
/* readouts: t1:313-315 argmin (-1 if nothing fires), t3:295-296 argmin with
   class 0 as the start, t2:391-392 argmax of the membrane */
enum { VDT_READ_ARGMIN_FIRST = 0, VDT_READ_ARGMIN_LOWEST = 1, VDT_READ_ARGMAX = 2 };
/* input encoders: none (spike times given), k_encode_image's log encoder
   (t1:32-42, t2:32-42), or the linear t = floor((1 - x) * T) */
enum { VDT_ENC_NONE = 0, VDT_ENC_LOG = 1, VDT_ENC_LINEAR = 2 };
/* bucket index: tb = max(0, floor(t - fire_start)) (t1:58, t2:59) or
   tb = (int)t with 0 <= tb < T (t3:79,99) */
enum { VDT_TB_FLOOR_STAGGER = 0, VDT_TB_TRUNC = 1 };
/* column layout for vdt_bucketize: NHWC / [N, F] rows (t1, t2, t3 fc) or
   NCHW sites with channel stride H*W (t3:70-90) */
enum { VDT_LAYOUT_NHWC = 0, VDT_LAYOUT_NCHW = 1 };

typedef struct {
    int T;            /* TIME_WINDOW, or the truncated window T' */
    int delta;        /* CHUNK: arrival-chunk width */
    float fire_start; /* TIME_FIRE_START: inter-layer stagger (0 t1, 40 t2) */
    float vth_init;   /* VTH_INIT */
    float inf_time;   /* INF_TIME */
    int lut_mode;     /* VDT_LUT_BY_TB | VDT_LUT_BY_TIN */
    int decay_len;    /* LUT_decay length: T (t1:209) or T + 1 (t2:238) */
    int lut_source;   /* VDT_LUT_DEVICE | VDT_LUT_HOST_LIBM */
} vdt_time_cfg;

typedef struct {
    int kind;       /* VDT_CONV | VDT_FC */
    int k;          /* square kernel size (conv; ignored for fc) */
    int pad;        /* VDT_PAD_VALID | VDT_PAD_SAME */
    int pool_after; /* 2x2 stride-2 min pool after this layer (k_pooling) */
    int out;        /* VDT_OUT_FIRE | VDT_OUT_VMEM (last layer only) */
} vdt_layer_desc;

typedef struct {
    int in_h, in_w, in_c; /* input map, NHWC */
    float tc_in, td_in;   /* input encoding constants (t1:283, t2:335) */
    int encoder;          /* applied when vdt_infer is given pixels */
    int readout;          /* VDT_READ_* */
} vdt_net_desc;

const char* vdt_version(void);
/* Launch overlap (no counterpart in the reference): 1 lets each kernel of a
   batch start while its predecessor's last CTAs finish (CUDA programmatic
   dependent launch; every kernel still waits for its inputs), 0 (default)
   launches them one after the other.  Process-wide; returns the previous
   setting.  Results do not change.  Graphs already captured keep the
   setting they were captured with. */
int vdt_set_launch_overlap(int enable);
const char* vdt_strerror(int status);
const char* vdt_last_error(void);

/* ------------------------------------------------------------------------
 * Model: replaces load_weights (t1:185-206, t2:213-234) + the per-batch
 * update_LUTs calls (t1:208-216, t2:236-243; tables are built once here).
 * `blob` is the reference's weight-blob bytes; `layers` the topology that the
 * reference's main hard-codes.  Shapes are checked against the blob.
 * ---------------------------------------------------------------------- */
int vdt_model_load_blob(const void* blob, size_t nbytes, const vdt_layer_desc* layers,
                        int n_layers, const vdt_net_desc* net, const vdt_time_cfg* cfg,
                        int device, vdt_model** out);
void vdt_model_destroy(vdt_model* m);
int vdt_model_info(const vdt_model* m, int* n_layers, int* n_classes, size_t* weight_bytes);
/* copy layer `layer`'s tables to host: decay_len and T floats */
int vdt_model_luts(const vdt_model* m, int layer, float* h_decay, float* h_th);

/* Task-3 (DVS gesture) CuLIF network: the topology and constants the
   reference's task-3 main hard-codes (t3:18-27 and its stage list :267-284;
   the reference: 2x32x32 input, T 160, delta 32, channels 64/128/128,
   k 3, hidden 128, 10 classes, decay exp(-1/5) / exp(-1/60), th 5 / 10). */
typedef struct {
    int in_c, H, W;       /* sensor polarities and size; H, W multiples of 4 */
    int T, delta;         /* T_TOTAL and CHUNK */
    int c1, c2, c3;       /* conv1 (raw frames), conv2, conv3 output channels */
    int k;                /* conv kernel size (odd, same padding) */
    int hidden, classes;  /* recurrent FC1 width (multiple of 32, <= 1024), FC2 outputs */
    float decay_conv, th_conv, decay_fc, th_fc;
} vdt_dvs_desc;

/* Replaces the task-3 main's weight read (t3:237-241): `blob` is the flat
   little-endian float32 array in the order of the reference's
   dvsgesture_weights_meta.txt -- conv1, conv2, conv3 (OIHW), FC1 recurrent
   [hidden, hidden], FC1 [hidden, c3*(H/4)*(W/4)], FC2 [classes, hidden] --
   at the offsets those sizes give (1,288,576 floats for the reference's
   shapes, FC2 at float 1,287,296); a longer blob is accepted (the reference
   reads a fixed 1,292,032 floats), a shorter one is VDT_ERR_BLOB.  The returned model is used with
   vdt_ctx_create and the whole-network calls below: vdt_infer,
   vdt_infer_host, vdt_infer_host_batches and vdt_infer_trace take frames
   [batch, in_c, H, W, T] (time innermost, the reference's raw input; the
   input_is_pixels flag is ignored), write FC2's first-spike times
   [batch, classes] and the argmin readout with class 0 as the start
   (t3:295-296), and run each batch as one captured CUDA graph with the
   ctx's workspace.  vdt_infer_trace's d_layer_out[0..6] receive the seven
   stage maps (conv1, conv2, pool1, conv3, pool2 NCHW; fc1 [batch, hidden];
   fc2); profiling times the same seven stages.  Per-layer integrator
   choice, LUTs, counting and sub-batches do not apply (VDT_ERR_UNSUPPORTED
   or no effect). */
int vdt_model_load_dvs_flat(const void* blob, size_t nbytes, const vdt_dvs_desc* desc, int device,
                            vdt_model** out);

/* ------------------------------------------------------------------------
 * Context: workspace (activations, bucket lists) for batches <= max_batch,
 * bound to one stream.  Replaces the reference's cudaMalloc'd g_bkt_* statics
 * (t1:218-220, t2:245-248) and activation buffers.
 * ---------------------------------------------------------------------- */
/* The model must outlive every ctx created from it. */
int vdt_ctx_create(const vdt_model* m, int max_batch, vdt_stream stream, vdt_ctx** out);
void vdt_ctx_destroy(vdt_ctx* c);
/* 1 = launch the per-batch layer sequence as a captured CUDA graph (default) */
int vdt_ctx_set_graphs(vdt_ctx* c, int enable);
/* 1 = count events and fetched synapses (k_conv_bucketed's inner-loop
   executions, as counted by task2 macs/stat_timesorted_macs.cu:136,155) */
int vdt_ctx_set_counting(vdt_ctx* c, int enable);
int vdt_ctx_counters(vdt_ctx* c, unsigned long long* events, unsigned long long* fetched);
/* The same per layer (n_layers entries each, either array may be NULL): the
   events kept by the layer's bucketing and the synapses its integrator
   fetched.  Each read, by either call, returns the counts since the previous
   read and zeroes them. */
int vdt_ctx_layer_counters(vdt_ctx* c, int n_layers, unsigned long long* events, unsigned long long* fetched);
/* 1 = time every stage with CUDA events on the ctx stream (forces the eager,
   non-graph path while on); vdt_ctx_layer_times then returns, per layer, the
   milliseconds accumulated since the last read by its bucketize, integrate
   (or membrane readout) and pool launches, and the number of batches run. */
int vdt_ctx_set_profiling(vdt_ctx* c, int enable);
int vdt_ctx_layer_times(vdt_ctx* c, int n_layers, float* bucketize_ms, float* integrate_ms,
                        float* pool_ms, int* batches);

/* Integrator each layer runs (no counterpart in the reference, which has one
   kernel).  A layer with VDT_KERNEL_DENSE or VDT_KERNEL_THREAD launches no
   bucketize pass unless counting is on (counting passes run a
   VDT_KERNEL_THREAD layer through k_dense, which keeps the reference's
   fetched-synapse accounting). */
enum {
    VDT_KERNEL_CHUNK = 0,   /* k_integrate: chunk-bucket integrator (t2:84-170 order) */
    VDT_KERNEL_SORTED = 1,  /* k_sorted: per-chunk slot-sorted buckets, same results */
    VDT_KERNEL_DENSE = 2,   /* k_dense: bucketing fused, reads the spike map */
    VDT_KERNEL_VMEM = 3,    /* k_layer_vmem membrane readout */
    VDT_KERNEL_THREAD = 4   /* k_thread: one thread per output pixel, bucketing
                               fused; conv layers with C_out <= 16 and K*K*C_in
                               <= 32 (T < 8192), or 33..255 inputs with T <= 255
                               and decay_len <= 256 */
};
int vdt_ctx_layer_kernels(const vdt_ctx* c, int n_layers, int* kernels);
/* Force the integrator of one layer (-1 = automatic choice); results are the
   same with every kernel, only speed differs.  VDT_ERR_UNSUPPORTED if that
   kernel cannot run the layer.  Drops the ctx's captured graphs. */
int vdt_ctx_set_layer_kernel(vdt_ctx* c, int layer, int kernel);

/* n in [1, VDT_MAX_SUB_BATCHES]: every batch runs as n near-equal parts on n
   streams (the ctx stream and n - 1 of the ctx's own, each with an
   activation / bucket workspace sized for max_batch / n, made once and kept),
   so one part's small late layers overlap the other parts' work; n = 1
   (default): one run.  Results are the same either way (each image's
   computation does not depend on the rest of its batch).  Counting,
   profiling and vdt_infer_trace run whole batches.  Drops the ctx's captured
   graphs.  No reference counterpart. */
#define VDT_MAX_SUB_BATCHES 4
int vdt_ctx_set_sub_batches(vdt_ctx* c, int n);

/* ------------------------------------------------------------------------
 * Whole-network inference: the per-batch body of the reference's main
 * (t1:290-315, t2:341-392).  d_input is [batch, in_h, in_w, in_c]: spike
 * times (input_is_pixels = 0) or pixels encoded with net->encoder.
 * d_out receives the last layer's output [batch, classes] (first-spike times,
 * or membrane values for a VDT_OUT_VMEM layer); d_pred (may be NULL) the
 * readout.  Asynchronous on the ctx stream.
 * ---------------------------------------------------------------------- */
int vdt_infer(vdt_ctx* c, const float* d_input, int input_is_pixels, int batch,
              float* d_out, int32_t* d_pred);
/* Same, end to end from host buffers: H2D copy of the input, the network,
   D2H copy of outputs; synchronous.  With sub-batches (and graphs on) each
   part runs as its own graph on its own stream as soon as its share of the
   input has landed (the parts' inputs cross in order on a copy stream), and
   copies its outputs back on that stream: part 0 computes while part 1's
   input is still crossing.  h_pred may be NULL. */
int vdt_infer_host(vdt_ctx* c, const float* h_input, int input_is_pixels, int batch,
                   float* h_out, int32_t* h_pred);
/* n_batches batches of `batch` images each, end to end from host buffers,
   pipelined: batch i+1's H2D copy (a second input slot, a copy stream) runs
   while batch i computes, and batch i's D2H copy while batch i+1 computes.
   h_inputs[i] (pinned host memory for the overlap to happen) must stay valid
   until the call returns; h_outs / h_preds (or any entry of them) may be
   NULL.  Same results as n_batches calls of vdt_infer_host; synchronous.
   The serving loop around the reference's per-batch body (t1:290-315,
   t2:341-392), which copies, computes and copies back in turn. */
int vdt_infer_host_batches(vdt_ctx* c, int n_batches, const float* const* h_inputs, int input_is_pixels,
                           int batch, float* const* h_outs, int32_t* const* h_preds);
/* Same as vdt_infer, also writing every layer's output map (before its pool)
   into d_layer_out[i] (device buffers sized [batch, H_out, W_out, C_out]). */
int vdt_infer_trace(vdt_ctx* c, const float* d_input, int input_is_pixels, int batch,
                    float* const* d_layer_out, float* d_out, int32_t* d_pred);

/* ------------------------------------------------------------------------
 * Per-stage entry points (the reference's kernels, as drop-ins)
 * ---------------------------------------------------------------------- */

/* update_LUTs (t1:208-216, t2:236-243) as a device kernel:
   d_decay[t] = exp(-((float)t - td_integ) / tc_integ), t < decay_len;
   d_th[t] = vth_init * exp(-((float)t - td_fire) / tc_fire), t < T. */
int vdt_build_luts(int T, int decay_len, float tc_integ, float td_integ, float tc_fire,
                   float td_fire, float vth_init, float* d_decay, float* d_th,
                   vdt_stream stream);

/* k_encode_image (t1:32-42, t2:32-42) / linear encoder; n elements. */
int vdt_encode(const float* d_pixels, float* d_spikes, int64_t n, int encoder, float tc,
               float td, int T, float inf_time, vdt_stream stream);

/* k_bucketize (t1:45-80, t2:45-81), k_bucketize_conv / k_bucketize_fc
   (t3:70-106): lossless counting sort of each column's spikes into
   NC = ceil(T/delta) arrival chunks.  Output layout identical to the
   reference: d_off [n_cols, NC+1] exclusive offsets (last = count),
   d_cin / d_tin [n_cols, c_in] channel index and spike time, stable
   (increasing channel) within each chunk.  NHWC: column col holds
   d_in[col*c_in + i]; NCHW: col = n*hw + s holds d_in[n*c_in*hw + i*hw + s]. */
int vdt_bucketize(const float* d_in, int64_t n_cols, int c_in, int layout, int64_t hw,
                  const vdt_time_cfg* cfg, int tb_mode, int* d_off, int* d_cin,
                  float* d_tin, vdt_stream stream);

/* k_conv_bucketed (t1:83-162, t2:84-170): chunked early-exit integrator over
   reference-layout buckets.  Weights HWIO [K, K, C_in, C_out] (conv) or
   [C_in, C_out] (is_fc); output NHWC first-spike times [B, H_out, W_out,
   C_out].  pad: taps at (h - pad + kh, w - pad + kw), out-of-range skipped. */
int vdt_conv_bucketed(const int* d_off, const int* d_cin, const float* d_tin,
                      const float* d_kernel, const float* d_bias, const float* d_decay,
                      const float* d_th, int t_min, int B, int H_in, int W_in, int C_in,
                      int H_out, int W_out, int C_out, int K, int pad, int is_fc,
                      const vdt_time_cfg* cfg, float* d_out, vdt_stream stream);

/* k_layer_vmem (t2:172-190): membrane readout of a non-firing last layer. */
int vdt_layer_vmem(const float* d_in, const float* d_kernel, const float* d_bias,
                   const float* d_decay, int B, int C_in, int C_out,
                   const vdt_time_cfg* cfg, float* d_out, vdt_stream stream);

/* k_pooling (t1:164-181, t2:192-209): 2x2 stride-2 min of spike times, NHWC. */
int vdt_pool_min(const float* d_in, float* d_out, int B, int H_in, int W_in, int C,
                 float inf_time, vdt_stream stream);

/* host readout loops (t1:313-315, t2:391-392, t3:295-296) on the device */
int vdt_readout(const float* d_out, int B, int K, int mode, float inf_time,
                int32_t* d_pred, vdt_stream stream);

/* ------------------------------------------------------------------------
 * Task 3 (DVS gesture) CuLIF stages.  Every neuron steps
 * I = fma(I, decay, in[t]); V += I and fires at the first t with V >= th;
 * the scan covers whole chunks (t < ceil(T/delta)*delta, as the reference).
 * Spike maps are fp32 spike times (9999 = none).  Buckets come from
 * vdt_bucketize with VDT_TB_TRUNC (NCHW sites for convs, per-sample rows for
 * FC layers).
 * ---------------------------------------------------------------------- */

/* conv1_raw_early (t3:30-65): dense frames [N, C_in, H, W, T] (time
   innermost), weights OIHW [C_out, C_in, K, K], same-pad conv; output NCHW.
   in[t] sums w * frame in (c_in, ky, kx) order with FMAs; frames past T
   read as 0.  delta in {8, 16, 32}, C_out <= 128. */
int vdt_dvs_conv1_raw(const float* d_frames, const float* d_w_oihw, int N, int C_in, int C_out,
                      int H, int W, int K, int T, int delta, float decay, float th, float* d_out,
                      vdt_stream stream);

/* conv_bucketed_early (t3:109-143): in[tt - base] += w over the chunk's
   events in (ky, kx, bucket) order.  Weights HWIO [K, K, C_in, C_out]
   (vdt_oihw_to_hwio converts the reference's OIHW); output NCHW or NHWC. */
int vdt_dvs_conv_bucketed(const int* d_off, const int* d_cin, const float* d_tin,
                          const float* d_w_hwio, int N, int C_in, int C_out, int H, int W, int K,
                          int T, int delta, float decay, float th, int out_layout, float* d_out,
                          vdt_stream stream);

/* k_bucketize_conv (t3:70-90) and conv_bucketed_early (t3:109-143) in one
   launch: reads the layer's input spike map (d_in, NCHW or NHWC per
   in_layout) instead of bucket lists, same results as
   vdt_bucketize (VDT_TB_TRUNC) + vdt_dvs_conv_bucketed bit for bit (each
   step's input summed in (ky, kx, channel) order, every step scanned up to
   ceil(T / delta) * delta).  VDT_ERR_UNSUPPORTED unless K*K*C_in <= 1152
   and K*K <= 32. */
int vdt_dvs_conv_dense(const float* d_in, int in_layout, const float* d_w_hwio, int N, int C_in, int C_out,
                       int H, int W, int K, int T, int delta, float decay, float th, int out_layout,
                       float* d_out, vdt_stream stream);

/* pool_chunk_early (t3:146-168): spiking 2x2 pool, in[t] = 1 at each input
   spike's bin; layout VDT_LAYOUT_NCHW or VDT_LAYOUT_NHWC (in and out). */
int vdt_dvs_pool(const float* d_in, float* d_out, int N, int C, int H_in, int W_in, int layout,
                 int T, int delta, float decay, float th, vdt_stream stream);

/* fc1_bucketed_recurrent (t3:171-200): feed-forward in_ff from the sample's
   buckets plus, every step, the recurrent input of the neurons that fired
   on the previous step (ascending j); I = fma(I, decay, in_ff) + in_rec; a
   neuron fires once (V reset to -10000); no early exit.  Transposed weights:
   d_w_t[j][i] = W_fc1[i][j] ([F_in, F_out]), d_wrec_t[j][i] = W_rec[i][j].
   F_out a multiple of 32, at most 1024. */
int vdt_dvs_fc1_recurrent(const int* d_off, const int* d_cin, const float* d_tin,
                          const float* d_w_t, const float* d_wrec_t, int N, int F_in, int F_out,
                          int T, int delta, float decay, float th, float* d_out, vdt_stream stream);
/* Where F_out is a multiple of 128, the feed-forward sums of every
   (sample, step, neuron) are built first by an event-parallel kernel into a
   scratch buffer of vdt_dvs_fc1_scratch_bytes(N, F_out, T, delta) bytes (0:
   none used for this shape); vdt_dvs_fc1_recurrent allocates it
   stream-ordered per call, vdt_dvs_fc1_recurrent_ws takes it from the caller
   (device memory, 16-byte aligned; VDT_ERR_CAPACITY when smaller).  Same
   results either way.  No reference counterpart (the reference sums each
   neuron's events inside the recurrent kernel). */
size_t vdt_dvs_fc1_scratch_bytes(int N, int F_out, int T, int delta);
int vdt_dvs_fc1_recurrent_ws(const int* d_off, const int* d_cin, const float* d_tin,
                             const float* d_w_t, const float* d_wrec_t, int N, int F_in, int F_out,
                             int T, int delta, float decay, float th, float* d_out, void* d_scratch,
                             size_t scratch_bytes, vdt_stream stream);

/* fc2_bucketed_early (t3:203-225): bucketed FC, transposed weights
   d_w_t[j][i] = W_fc2[i][j] ([F_in, F_out]); output [N, F_out]. */
int vdt_dvs_fc2(const int* d_off, const int* d_cin, const float* d_tin, const float* d_w_t, int N,
                int F_in, int F_out, int T, int delta, float decay, float th, float* d_out,
                vdt_stream stream);

/* OIHW [O, I, K, K] -> HWIO [K, K, I, O] weight permutation (device). */
int vdt_oihw_to_hwio(const float* d_src, float* d_dst, int O, int I, int K, vdt_stream stream);

/* ------------------------------------------------------------------------
 * Allocation-free layer step (no counterpart in the reference)
 * ---------------------------------------------------------------------- */

/* Bytes of the library's fixed per-device scratch array. */
#define VDT_NOALLOC_SCRATCH_BYTES (32u << 20)
size_t vdt_noalloc_scratch_bytes(void);

/* One fire layer -- vdt_bucketize (NHWC, tb_mode) followed by
   vdt_conv_bucketed, same arguments and same results -- for callers that
   cannot let a library allocate device memory while they run (servers that
   plan all device memory up front, loops that cannot take cudaMalloc's
   device-wide synchronisation, hosts that own the allocator).  It allocates
   nothing: the bucket lists live in a static device array of
   VDT_NOALLOC_SCRATCH_BYTES per GPU.  A layer whose lists need more
   (n_cols*(NC+1) + 2*n_cols*C_in 4-byte words, each of the three parts rounded
   up to 256 bytes; n_cols = B*H_in*W_in, or B for is_fc) returns
   VDT_ERR_CAPACITY and launches nothing: 54 maps of 32x32x64 fit at T=80,
   delta=4 (58 at delta=8), one 224x224x64 map at delta >= 4.  The first
   call on each device looks the array's address up (with that device
   current) and should precede any stream capture; the address is cached per
   device and CUDA context, so a call after cudaDeviceReset looks it up
   again.  Calls on one device share the array, so calls that can
   overlap on the GPU (unordered streams or threads) race; order them.
   Nothing in the array needs to start zeroed. */
int vdt_conv_layer_noalloc(const float* d_in, int tb_mode, const float* d_kernel,
                           const float* d_bias, const float* d_decay, const float* d_th,
                           int t_min, int B, int H_in, int W_in, int C_in, int H_out,
                           int W_out, int C_out, int K, int pad, int is_fc,
                           const vdt_time_cfg* cfg, float* d_out, vdt_stream stream);

/* ------------------------------------------------------------------------
 * Measurement helper (no counterpart in the reference)
 * ---------------------------------------------------------------------- */

/* Measures, on `device` at its current clocks, the FP32 FMA throughput
   (FMAs per second over independent packed fma.rn.f32x2 chains on every SM)
   and the L2-to-SM read bandwidth (bytes per second, 16-byte L2-only loads of
   a 32 MiB L2-resident buffer): the integrators' two limits, one FMA and one
   4-byte weight read per fetched synapse.  Allocates and frees 32 MiB; runs
   on the legacy default stream and synchronises it. */
int vdt_measure_peaks(int device, double* fma_per_s, double* l2_read_bytes_per_s);

#ifdef __cplusplus
}
#endif
#endif /* VDTTFS_H */
