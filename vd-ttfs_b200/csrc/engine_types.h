// engine_types.h -- the model and context objects behind the C ABI's opaque
// vdt_model / vdt_ctx handles, shared by the host runtime (runtime.cu) and the
// task-3 network runner (dvs_net.cu).  Not part of the public ABI.
#pragma once

#include <map>
#include <tuple>
#include <vector>

#include "vdt_internal.h"

namespace vdt {

// One layer of a task-1/2 network: its descriptor, shapes, time constants
// and pointers into the model's weight arena.
struct Layer {
    vdt_layer_desc d;
    int H_in, W_in, C_in, H_out, W_out, C_out;
    float tc_fire, td;
    int t_min;
    float* W = nullptr;      // into the model's weight arena
    float* bias = nullptr;
    float* decay = nullptr;  // [decay_len]
    float* th = nullptr;     // [T]
};

// Task-3 CuLIF network weights in the kernels' layouts (one device arena).
struct DvsWeights {
    float* conv1 = nullptr;  // OIHW [c1, in_c, k, k] (conv1_raw reads it as is)
    float* conv2 = nullptr;  // HWIO [k, k, c1, c2]
    float* conv3 = nullptr;  // HWIO [k, k, c2, c3]
    float* fc1_t = nullptr;  // [F_in, hidden]
    float* rec_t = nullptr;  // [hidden, hidden], rec_t[j][i] = W_rec[i][j]
    float* fc2_t = nullptr;  // [hidden, classes]
};

// Stages of the task-3 network (the reference main's order, t3:267-284);
// per-stage profiling and vdt_infer_trace index them like layers.
enum DvsStage { DVS_CONV1 = 0, DVS_CONV2, DVS_POOL1, DVS_CONV3, DVS_POOL2, DVS_FC1, DVS_FC2, DVS_STAGES };

}  // namespace vdt

struct vdt_model {
    int device = 0;
    vdt_time_cfg cfg{};
    vdt_net_desc net{};
    std::vector<vdt::Layer> layers;
    float* arena = nullptr;
    size_t weight_bytes = 0;
    int n_classes = 0;       // output values per sample (the last map, flattened)
    size_t in_elems = 0;     // input floats per sample
    // task-3 network (vdt_model_load_dvs_flat): no layer list, the stages of
    // dvs_net.cu run instead
    bool is_dvs = false;
    vdt_dvs_desc dvs{};
    vdt::DvsWeights dw{};
};

// part 0: a whole batch (its sub-batches forked and joined inside the
// graph); part k + 1: sub-batch k alone, on its workspace (the host path)
struct GraphKey {
    int batch, pixels, counting, slot, part;
    bool operator<(const GraphKey& o) const {
        return std::tie(batch, pixels, counting, slot, part) <
               std::tie(o.batch, o.pixels, o.counting, o.slot, o.part);
    }
};

struct vdt_ctx {
    const vdt_model* m = nullptr;  // must outlive the ctx
    int device = 0;
    int max_batch = 0;
    cudaStream_t stream = nullptr;
    float* act[3] = {nullptr, nullptr, nullptr};
    float* in_slot = nullptr;    // [max_batch, in_elems]
    float* out_slot = nullptr;   // [max_batch, classes]
    int32_t* pred_slot = nullptr;
    // copy stream of the host paths and the per-part input events of
    // vdt_infer_host, made on first use
    cudaStream_t copy_stream = nullptr;
    cudaEvent_t ev_part[VDT_MAX_SUB_BATCHES] = {};
    // second input/output slot and events of the pipelined host path
    // (vdt_infer_host_batches), made on its first call
    float* in_slot2 = nullptr;
    float* out_slot2 = nullptr;
    int32_t* pred_slot2 = nullptr;
    cudaEvent_t ev_h2d[2] = {nullptr, nullptr}, ev_done[2] = {nullptr, nullptr};
    // sub-batches (vdt_ctx_set_sub_batches): parts 1.. of a batch run on
    // their own streams with their own activation and bucket workspaces
    struct SubWs {
        float* act[3] = {nullptr, nullptr, nullptr};
        int* off = nullptr;
        int* cin = nullptr;
        float* tin = nullptr;
        cudaStream_t stream = nullptr;
        cudaEvent_t join = nullptr;
    };
    int n_sub = 1;
    std::vector<SubWs> sub;                  // n_sub - 1 entries once made
    cudaEvent_t ev_fork = nullptr;
    int* off = nullptr;
    int* cin = nullptr;
    float* tin = nullptr;
    float* scratch = nullptr;                // task 3: FC1 feed-forward sums
    size_t scratch_bytes = 0;
    unsigned long long* counters = nullptr;  // [events, fetched]
    bool graphs = true;
    bool counting = false;
    bool profiling = false;
    // layers with K*K*C_in up to this use k_dense: its per-pixel window fits
    // 8 CTAs per SM in shared memory (wider windows run k_sorted, which does)
    int dense_max_fan = 576;
    std::vector<int> kernel_override;  // per layer: -1 automatic, else VDT_KERNEL_*
    std::map<GraphKey, cudaGraphExec_t> cache;
    // profiling: (layer, stage, start, stop) per timed launch, read back lazily
    struct Mark { int layer, stage; cudaEvent_t a, b; };
    std::vector<Mark> marks;
    std::vector<cudaEvent_t> spare_events;
    int prof_batches = 0;
};

namespace vdt {

inline cudaEvent_t take_event(vdt_ctx* c) {
    if (!c->spare_events.empty()) {
        cudaEvent_t e = c->spare_events.back();
        c->spare_events.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

// Records a start/stop event pair around one stage when the ctx profiles
// (stage 0 = bucketize, 1 = integrate / compute, 2 = pool).
struct StageTimer {
    vdt_ctx* c; int layer, stage; cudaEvent_t a = nullptr;
    StageTimer(vdt_ctx* c_, int l, int s) : c(c_), layer(l), stage(s) {
        if (c->profiling) { a = take_event(c); cudaEventRecord(a, c->stream); }
    }
    ~StageTimer() {
        if (a) {
            cudaEvent_t b = take_event(c);
            cudaEventRecord(b, c->stream);
            c->marks.push_back({layer, stage, a, b});
        }
    }
};

// Number of profiled / traced stages: the layers of a task-1/2 network, the
// DvsStage list of a task-3 network.
inline int model_stages(const vdt_model* m) { return m->is_dvs ? (int)DVS_STAGES : (int)m->layers.size(); }

// ------------------------------------------------------ task 3 (dvs_net.cu)
// Workspace sizes (floats / ints) of a ctx for batches up to B.
struct DvsSizes {
    size_t act = 0, off = 0, bkt = 0, scratch_bytes = 0;
};
DvsSizes dvs_sizes(const vdt_model* m, long long B);
// Enqueue one batch of frames [B, in_c, H, W, T] on c->stream: every stage,
// the readout; trace[i] (when given) receives stage i's output map.
int dvs_enqueue(vdt_ctx* c, const float* d_frames, int B, float* d_out, int32_t* d_pred, float* const* trace);
// Chunk width the stages after conv1 run at (results do not depend on it).
int dvs_internal_delta(const vdt_dvs_desc& d);
// The stage output sizes (floats per sample), in DvsStage order.
void dvs_stage_sizes(const vdt_dvs_desc& d, size_t out[DVS_STAGES]);

}  // namespace vdt
