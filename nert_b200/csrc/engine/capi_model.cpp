// extern "C" entry points of the B200 engine (declared in include/nert_b200.h).

#include "../../../include/nert_b200.h"
#include "model.hpp"

#include <cstring>
#include <memory>

using nb2::eng::Model;

struct nb2_model {
    std::unique_ptr<Model> m;
};

namespace {

template <typename F>
int guard(F&& f) {
    try {
        f();
        return NB2_OK;
    } catch (const nb2::Error& e) {
        nb2::set_last_error(e.what());
        return e.code;
    } catch (const nb2::eng::LoadError& e) {
        nb2::set_last_error(e.what());
        return NB2_ERR_INVALID;
    } catch (const nb2::eng::RunError& e) {
        nb2::set_last_error(e.what());
        const std::string w = e.what();
        return w.find("device error") != std::string::npos ? NB2_ERR_DEVICE : NB2_ERR_INVALID;
    } catch (const std::bad_alloc&) {
        nb2::set_last_error("out of host memory");
        return NB2_ERR_NOMEM;
    } catch (const std::exception& e) {
        nb2::set_last_error(e.what());
        return NB2_ERR_INVALID;
    }
}

} // namespace

extern "C" {

int nb2_model_create(const void* onnx, int64_t size, int n_inputs, const char* const* names,
                     const int64_t* dims_flat, const int* ranks, int ordinal, int flags, nb2_model** out) {
    return guard([&] {
        if (out == nullptr || onnx == nullptr || size <= 0) {
            throw nb2::eng::LoadError("nb2_model_create: bad arguments");
        }
        *out = nullptr;
        std::map<std::string, std::vector<int64_t>> dims;
        int64_t at = 0;
        for (int i = 0; i < n_inputs; ++i) {
            dims[names[i]] = std::vector<int64_t>(dims_flat + at, dims_flat + at + ranks[i]);
            at += ranks[i];
        }
        auto h = std::make_unique<nb2_model>();
        h->m = std::make_unique<Model>(static_cast<const uint8_t*>(onnx), static_cast<size_t>(size), dims, ordinal,
                                       flags);
        *out = h.release();
    });
}

int nb2_model_destroy(nb2_model* m) {
    return guard([&] { delete m; });
}

int nb2_model_num_io(const nb2_model* m, int* n_inputs, int* n_outputs) {
    return guard([&] {
        *n_inputs = static_cast<int>(m->m->inputs().size());
        *n_outputs = static_cast<int>(m->m->outputs().size());
    });
}

int nb2_model_io(const nb2_model* m, int is_output, int i, const char** name, int* dtype, int* rank, int64_t* dims8,
                 void** device_ptr) {
    return guard([&] {
        const auto& v = is_output ? m->m->outputs() : m->m->inputs();
        if (i < 0 || i >= static_cast<int>(v.size())) {
            throw nb2::eng::RunError("io index out of range");
        }
        const auto& io = v[static_cast<size_t>(i)];
        *name = io.name.c_str();
        *dtype = static_cast<int>(io.dtype);
        *rank = static_cast<int>(io.dims.size());
        for (size_t d = 0; d < io.dims.size() && d < 8; ++d) {
            dims8[d] = io.dims[d];
        }
        *device_ptr = io.dev;
    });
}

int nb2_model_run(nb2_model* m, const void* const* host_inputs, void* const* host_outputs) {
    return guard([&] {
        std::vector<const void*> in(host_inputs, host_inputs + m->m->inputs().size());
        std::vector<void*> out(host_outputs, host_outputs + m->m->outputs().size());
        m->m->run_host(in, out);
    });
}

int nb2_model_run_async(nb2_model* m, const void* const* host_inputs, void* const* host_outputs) {
    return guard([&] {
        std::vector<const void*> in(host_inputs, host_inputs + m->m->inputs().size());
        std::vector<void*> out(host_outputs, host_outputs + m->m->outputs().size());
        m->m->enqueue_host(in, out);
    });
}

int nb2_model_launch(nb2_model* m) {
    return guard([&] { m->m->launch(); });
}

int nb2_model_synchronize(nb2_model* m) {
    return guard([&] { m->m->synchronize(); });
}

int nb2_model_stats(const nb2_model* m, int64_t* kernels_per_run, int64_t* arena_bytes, int64_t* weight_bytes,
                    int64_t* fused_groups, int64_t* exec_nodes) {
    return guard([&] {
        *kernels_per_run = m->m->kernels_per_run();
        *arena_bytes = m->m->arena_bytes();
        *weight_bytes = m->m->weight_bytes();
        *fused_groups = m->m->fused_groups();
        *exec_nodes = m->m->exec_nodes();
    });
}

int nb2_model_profile(nb2_model* m, int max_steps, char* labels, int label_len, float* ms, int* count) {
    return guard([&] {
        const auto prof = m->m->profile();
        const int n = std::min<int>(max_steps, static_cast<int>(prof.size()));
        for (int i = 0; i < n; ++i) {
            std::strncpy(labels + static_cast<size_t>(i) * label_len, prof[i].first.c_str(), label_len - 1);
            labels[static_cast<size_t>(i) * label_len + label_len - 1] = 0;
            ms[i] = prof[i].second;
        }
        *count = static_cast<int>(prof.size());
    });
}

int nb2_model_stream(const nb2_model* m, void** stream) {
    return guard([&] { *stream = m->m->device()->stream; });
}

int nb2_host_alloc(int64_t bytes, void** out) {
    return guard([&] {
        *out = nullptr;
        if (bytes > 0) {
            nb2::check_cuda(cudaMallocHost(out, static_cast<size_t>(bytes)), "cudaMallocHost");
        }
    });
}

int nb2_host_free(void* p) {
    return guard([&] {
        if (p) {
            nb2::check_cuda(cudaFreeHost(p), "cudaFreeHost");
        }
    });
}

} // extern "C"

namespace nb2 {
namespace eng {
std::string analyze_json(const uint8_t* onnx, size_t size, const std::map<std::string, std::vector<int64_t>>& dims,
                         int flags);
}
} // namespace nb2

extern "C" int nb2_graph_analyze(const void* onnx, int64_t size, int n_inputs, const char* const* names,
                                 const int64_t* dims_flat, const int* ranks, int flags, char* buf, int64_t cap,
                                 int64_t* needed) {
    return guard([&] {
        std::map<std::string, std::vector<int64_t>> dims;
        int64_t at = 0;
        for (int i = 0; i < n_inputs; ++i) {
            dims[names[i]] = std::vector<int64_t>(dims_flat + at, dims_flat + at + ranks[i]);
            at += ranks[i];
        }
        const std::string js =
            nb2::eng::analyze_json(static_cast<const uint8_t*>(onnx), static_cast<size_t>(size), dims, flags);
        *needed = static_cast<int64_t>(js.size()) + 1;
        if (buf != nullptr && cap >= *needed) {
            std::memcpy(buf, js.c_str(), js.size() + 1);
        }
    });
}
