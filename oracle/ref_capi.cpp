// TEST INFRASTRUCTURE ONLY — never part of the product path.
//
// A small C ABI over the reference NERT library (compiled from the reference
// sources by oracle/Makefile into oracle/_ref/libnert_ref.so). It lets the
// pytest suite, __graft_entry__.smoke() and bench.py's cpu_baseline leg drive
// the reference's own loader, shape inference, planner and executor:
//
//   nert::LoadGraphFromFile   include/nert/model_loader.hpp:30
//   nert::Model / RunTyped    include/nert/executor.hpp:57-76, src/executor.cpp:202,300
//   nert::CpuDevice()         include/nert/device.hpp:80 (the oracle kernels)
//
// A caller may also pass any other `const nert::Device*` (for example the B200
// device handle exported by libnert_b200_device.so through nb2_nert_device);
// that is how the drop-in test runs the reference's unmodified executor on the
// new device. Errors never cross the C boundary as exceptions: every entry
// point returns 0 on success and a negative code otherwise, with the message
// kept on the session (or in a thread-local buffer when there is none).

#include "nert/constant_folding.hpp"
#include "nert/device.hpp"
#include "nert/executor.hpp"
#include "nert/graph.hpp"
#include "nert/model_loader.hpp"

#include <chrono>
#include <cstdint>
#include <cstring>
#include <exception>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace {

thread_local std::string g_error;

struct Session {
    nert::Graph graph;
    std::unique_ptr<nert::Model> model;
    nert::HostTensorMap outputs;
    std::vector<std::string> output_names;
    std::string error;
    double last_run_ms = 0.0;
};

nert::DataType ToDtype(int code) {
    switch (code) {
    case 0:
        return nert::DataType::Float32;
    case 1:
        return nert::DataType::Int64;
    case 2:
        return nert::DataType::Bool;
    default:
        return nert::DataType::Unknown;
    }
}

int FromDtype(nert::DataType dtype) {
    switch (dtype) {
    case nert::DataType::Float32:
        return 0;
    case nert::DataType::Int64:
        return 1;
    case nert::DataType::Bool:
        return 2;
    default:
        return -1;
    }
}

} // namespace

extern "C" {

const char* nref_last_error(void* session) {
    if (session != nullptr) {
        return static_cast<Session*>(session)->error.c_str();
    }
    return g_error.c_str();
}

// Loads `onnx_path` with the reference loader and binds it with concrete input
// shapes to `device` (a `const nert::Device*`; null selects nert::CpuDevice()).
// `dims_flat` holds every input's dims back to back; `ranks[i]` says how many
// belong to input i. Returns a session or null (see nref_last_error(null)).
void* nref_open(const char* onnx_path, int n_inputs, const char* const* names, const int64_t* dims_flat,
                const int* ranks, const void* device) {
    auto session = std::make_unique<Session>();
    try {
        session->graph = nert::LoadGraphFromFile(onnx_path);
        nert::ShapeMap shapes;
        int64_t at = 0;
        for (int i = 0; i < n_inputs; ++i) {
            std::vector<int64_t> dims(dims_flat + at, dims_flat + at + ranks[i]);
            at += ranks[i];
            shapes.emplace(names[i], dims);
        }
        const nert::Device& dev =
            device != nullptr ? *static_cast<const nert::Device*>(device) : nert::CpuDevice();
        session->model = std::make_unique<nert::Model>(session->graph, shapes, dev);
        for (const auto& out : session->graph.outputs) {
            session->output_names.push_back(out.first);
        }
    } catch (const std::exception& e) {
        g_error = e.what();
        return nullptr;
    }
    return session.release();
}

// nref_open with the reference's load-time constant folding first:
// nert::FoldConstants(graph, *fold_device) (include/nert/constant_folding.hpp:22),
// which runs every all-constant node with that device's rows on the
// initializers' host bytes; *folded receives the number of nodes it folded.
// The Model then runs on `device` (CpuDevice when null).
void* nref_open_folded(const char* onnx_path, int n_inputs, const char* const* names, const int64_t* dims_flat,
                       const int* ranks, const void* fold_device, const void* device, int* folded) {
    auto session = std::make_unique<Session>();
    try {
        session->graph = nert::LoadGraphFromFile(onnx_path);
        const nert::Device& fdev =
            fold_device != nullptr ? *static_cast<const nert::Device*>(fold_device) : nert::CpuDevice();
        *folded = nert::FoldConstants(session->graph, fdev);
        nert::ShapeMap shapes;
        int64_t at = 0;
        for (int i = 0; i < n_inputs; ++i) {
            std::vector<int64_t> dims(dims_flat + at, dims_flat + at + ranks[i]);
            at += ranks[i];
            shapes.emplace(names[i], dims);
        }
        const nert::Device& dev =
            device != nullptr ? *static_cast<const nert::Device*>(device) : nert::CpuDevice();
        session->model = std::make_unique<nert::Model>(session->graph, shapes, dev);
        for (const auto& out : session->graph.outputs) {
            session->output_names.push_back(out.first);
        }
    } catch (const std::exception& e) {
        g_error = e.what();
        return nullptr;
    }
    return session.release();
}

void nref_close(void* session) { delete static_cast<Session*>(session); }

// Runs the bound model once through Model::RunTyped. `dtypes` uses 0=float32,
// 1=int64, 2=bool; `nbytes[i]` is the byte size of `data[i]`.
int nref_run(void* handle, int n_inputs, const char* const* names, const int* dtypes, const void* const* data,
             const int64_t* nbytes) {
    auto* session = static_cast<Session*>(handle);
    try {
        nert::HostTensorMap inputs;
        for (int i = 0; i < n_inputs; ++i) {
            nert::HostTensor t;
            t.dtype = ToDtype(dtypes[i]);
            t.dims = session->model->shapes().tensors.at(names[i]).dims;
            const auto* bytes = static_cast<const uint8_t*>(data[i]);
            t.bytes.assign(bytes, bytes + nbytes[i]);
            inputs.emplace(names[i], std::move(t));
        }
        const auto t0 = std::chrono::steady_clock::now();
        session->outputs = session->model->RunTyped(inputs);
        const auto t1 = std::chrono::steady_clock::now();
        session->last_run_ms = std::chrono::duration<double, std::milli>(t1 - t0).count();
    } catch (const std::exception& e) {
        session->error = e.what();
        return -1;
    }
    return 0;
}

double nref_last_run_ms(void* handle) { return static_cast<Session*>(handle)->last_run_ms; }

int nref_num_outputs(void* handle) { return static_cast<int>(static_cast<Session*>(handle)->output_names.size()); }

const char* nref_output_name(void* handle, int i) {
    return static_cast<Session*>(handle)->output_names.at(static_cast<size_t>(i)).c_str();
}

// Reports output i's dtype code, rank and dims (dims must hold 8 entries).
int nref_output_info(void* handle, int i, int* dtype, int* rank, int64_t* dims) {
    auto* session = static_cast<Session*>(handle);
    const auto it = session->outputs.find(session->output_names.at(static_cast<size_t>(i)));
    if (it == session->outputs.end()) {
        session->error = "output not produced";
        return -1;
    }
    *dtype = FromDtype(it->second.dtype);
    *rank = static_cast<int>(it->second.dims.size());
    for (size_t d = 0; d < it->second.dims.size() && d < 8; ++d) {
        dims[d] = it->second.dims[d];
    }
    return 0;
}

// Copies output i's bytes into `dst` (capacity `cap`); returns the byte count.
int64_t nref_output_copy(void* handle, int i, void* dst, int64_t cap) {
    auto* session = static_cast<Session*>(handle);
    const auto it = session->outputs.find(session->output_names.at(static_cast<size_t>(i)));
    if (it == session->outputs.end()) {
        session->error = "output not produced";
        return -1;
    }
    const int64_t n = static_cast<int64_t>(it->second.bytes.size());
    if (n > cap) {
        session->error = "destination too small";
        return -1;
    }
    std::memcpy(dst, it->second.bytes.data(), static_cast<size_t>(n));
    return n;
}

// The arena size the reference planner chose (memory_planner.cpp:79-225).
int64_t nref_arena_bytes(void* handle) { return static_cast<Session*>(handle)->model->plan().arena_size; }

} // extern "C"

#ifdef NREF_WITH_CUDA
// The reference's own CUDA device (cuDNN Conv, cuBLAS Gemm/MatMul, its CUDA
// kernel table), for the GPU baseline: src/cuda_device.cpp:98-102.
extern "C" const void* nref_cuda_device() {
    try {
        return &nert::CudaDevice();
    } catch (const std::exception& e) {
        g_error = e.what();
        return nullptr;
    }
}
#endif
