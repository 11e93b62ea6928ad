// The B200 engine's Model: one graph bound to one GPU and one concrete input
// shape, mirroring nert::Model (include/nert/executor.hpp:57-122,
// src/executor.cpp:202-560) with three B200-first differences:
//   * a peephole fuses Relu / residual Add(+Relu) / Sigmoid*Mul (SiLU) and
//     MatMul+Add(bias) into the Conv/Gemm that produces them, and the arena is
//     planned over the fused graph (groups are single nodes for liveness);
//   * weights are uploaded once and Conv/Gemm weights are pre-split into the
//     tf32 hi/lo K-major layout the tensor-core kernel reads;
//   * a Run is one CUDA-graph replay of every row on the device's stream
//     (no per-node synchronisation, no per-node host work).
#pragma once

#include "../runtime.hpp"
#include "graph.hpp"

#include <cuda_runtime.h>

#include <functional>
#include <map>
#include <string>
#include <vector>

namespace nb2 {
namespace eng {

// kNchwOnly keeps every activation NCHW (no channels-last trunk);
// kNoAttention runs attention chains as their MatMul / Softmax rows.
enum ModelFlags : int { kNoFusion = 1, kNoGraph = 2, kNchwOnly = 4, kNoAttention = 8 };

struct IOInfo {
    std::string name;
    DType dtype;
    std::vector<int64_t> dims;
    void* dev = nullptr;
    int64_t bytes = 0;
};

class Model {
  public:
    Model(const uint8_t* onnx, size_t size, const std::map<std::string, std::vector<int64_t>>& input_dims,
          int ordinal, int flags);
    ~Model();
    Model(const Model&) = delete;
    Model& operator=(const Model&) = delete;

    // End to end: host inputs -> device, run, device -> host outputs, synchronised.
    void run_host(const std::vector<const void*>& inputs, const std::vector<void*>& outputs);
    // The same, queued on the device stream without the final synchronise.
    void enqueue_host(const std::vector<const void*>& inputs, const std::vector<void*>& outputs);
    // Device-resident run: inputs already in the input buffers; asynchronous.
    void launch();
    void synchronize();

    const std::vector<IOInfo>& inputs() const { return inputs_; }
    const std::vector<IOInfo>& outputs() const { return outputs_; }
    int64_t kernels_per_run() const { return launches_; }
    int64_t arena_bytes() const { return arena_bytes_; }
    int64_t weight_bytes() const { return weight_bytes_; }
    int64_t fused_groups() const { return fused_groups_; }
    int64_t exec_nodes() const { return static_cast<int64_t>(steps_.size()); }
    int64_t nhwc_tensors() const { return nhwc_tensors_; }
    nb2_device* device() const { return dev_; }
    // Per-step device time of one eager pass (ms), with the step labels.
    std::vector<std::pair<std::string, float>> profile();

  private:
    struct Step {
        std::string label;
        int launches = 1;
        std::function<void()> run;
    };
    void build(const std::map<std::string, std::vector<int64_t>>& input_dims, int flags);
    void run_steps();

    nb2_device* dev_ = nullptr;
    Graph g_;
    std::map<std::string, TensorInfo> shapes_;
    std::vector<Step> steps_;
    std::vector<IOInfo> inputs_, outputs_;
    std::vector<void*> allocations_;
    void* scratch_ = nullptr;
    void* xform_ = nullptr; // NHWC copy of an NCHW Conv input (shared by the steps)
    int64_t arena_bytes_ = 0, weight_bytes_ = 0, launches_ = 0, fused_groups_ = 0, nhwc_tensors_ = 0;
    bool use_graph_ = true;
    cudaGraphExec_t exec_ = nullptr;
    int exec_precision_ = -1;
    // Host-input pipeline of enqueue_host: the next run's inputs are copied
    // from host memory into one of two staging buffers on a copy stream, so
    // the transfer overlaps the run in flight; the run then moves its staged
    // inputs into the input buffers on the device stream (device-to-device).
    cudaStream_t copy_stream_ = nullptr;
    uint8_t* stage_[2] = {nullptr, nullptr};
    cudaEvent_t staged_[2] = {nullptr, nullptr}; // staging k filled (copy stream)
    cudaEvent_t freed_[2] = {nullptr, nullptr};  // staging k consumed (device stream)
    uint64_t pipe_runs_ = 0;
    void release_pipeline();
};

} // namespace eng
} // namespace nb2
