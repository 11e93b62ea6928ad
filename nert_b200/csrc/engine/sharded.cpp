// Batch-sharded execution over several GPUs (include/nert_b200.h,
// nb2_sharded_*): the same graph is planned once per GPU for that GPU's slice
// of the batch, each slice runs on its own host thread and stream, and the
// slices are scattered from / gathered into the caller's host buffers at
// offset (first image of the slice) x (bytes per image).
//
// The reference has one process-wide CudaDevice and one Model bound to it
// (src/cuda_device.cpp:98-102, src/executor.cpp:202-225); every op on the
// path is per image once BatchNormalization is folded, so no data crosses
// between GPUs and there is no collective.

#include "../../../include/nert_b200.h"
#include "model.hpp"

#include <condition_variable>
#include <exception>
#include <memory>
#include <mutex>
#include <thread>

namespace nb2 {
namespace eng {

// Contiguous slices of `batch` images over `n` shards: the first batch % n
// shards take one image more. A shard may be empty when batch < n.
void shard_plan(int64_t batch, int n, int64_t* offsets, int64_t* counts) {
    const int64_t base = batch / n, extra = batch % n;
    int64_t at = 0;
    for (int i = 0; i < n; ++i) {
        counts[i] = base + (i < extra ? 1 : 0);
        offsets[i] = at;
        at += counts[i];
    }
}

} // namespace eng
} // namespace nb2

using nb2::eng::Model;

struct nb2_sharded {
    struct Shard {
        int ordinal = 0;
        int64_t offset = 0, count = 0;
        std::unique_ptr<Model> model;
        std::thread worker;
        std::exception_ptr error;
    };
    std::vector<Shard> shards;
    std::vector<int64_t> in_image_bytes, out_image_bytes;
    std::vector<nb2::eng::IOInfo> inputs, outputs; // global shapes
    // one generation per run; workers wait for a new generation, run their
    // slice and count themselves done
    std::mutex mu;
    std::condition_variable cv_start, cv_done;
    uint64_t generation = 0;
    int pending = 0;
    bool stop = false;
    const void* const* host_in = nullptr;
    void* const* host_out = nullptr;

    void work(size_t i);
    void run(const void* const* in, void* const* out);
    ~nb2_sharded();
};

void nb2_sharded::work(size_t i) {
    uint64_t seen = 0;
    Shard& s = shards[i];
    while (true) {
        {
            std::unique_lock<std::mutex> lock(mu);
            cv_start.wait(lock, [&] { return stop || generation != seen; });
            if (stop) {
                return;
            }
            seen = generation;
        }
        try {
            std::vector<const void*> in(inputs.size());
            std::vector<void*> out(outputs.size());
            for (size_t k = 0; k < in.size(); ++k) {
                in[k] = static_cast<const uint8_t*>(host_in[k]) + s.offset * in_image_bytes[k];
            }
            for (size_t k = 0; k < out.size(); ++k) {
                out[k] = static_cast<uint8_t*>(host_out[k]) + s.offset * out_image_bytes[k];
            }
            s.model->run_host(in, out);
        } catch (...) {
            s.error = std::current_exception();
        }
        std::lock_guard<std::mutex> lock(mu);
        if (--pending == 0) {
            cv_done.notify_all();
        }
    }
}

void nb2_sharded::run(const void* const* in, void* const* out) {
    std::unique_lock<std::mutex> lock(mu);
    host_in = in;
    host_out = out;
    int active = 0;
    for (auto& s : shards) {
        s.error = nullptr;
        active += s.model ? 1 : 0;
    }
    pending = active;
    ++generation;
    cv_start.notify_all();
    cv_done.wait(lock, [&] { return pending == 0; });
    for (auto& s : shards) {
        if (s.error) {
            std::rethrow_exception(s.error);
        }
    }
}

nb2_sharded::~nb2_sharded() {
    {
        std::lock_guard<std::mutex> lock(mu);
        stop = true;
    }
    cv_start.notify_all();
    for (auto& s : shards) {
        if (s.worker.joinable()) {
            s.worker.join();
        }
    }
}

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

int64_t tail_bytes(const nb2::eng::IOInfo& io) {
    int64_t n = nb2::eng::dtype_size(io.dtype);
    for (size_t d = 1; d < io.dims.size(); ++d) {
        n *= io.dims[d];
    }
    return n;
}

} // namespace

extern "C" {

int nb2_shard_plan(int64_t batch, int n_shards, int64_t* offsets, int64_t* counts) {
    return guard([&] {
        if (batch < 0 || n_shards <= 0 || offsets == nullptr || counts == nullptr) {
            throw nb2::eng::LoadError("nb2_shard_plan: bad arguments");
        }
        nb2::eng::shard_plan(batch, n_shards, offsets, counts);
    });
}

int nb2_sharded_create(const void* onnx, int64_t size, int n_inputs, const char* const* names,
                       const int64_t* dims_flat, const int* ranks, const int* ordinals, int n_shards, int flags,
                       nb2_sharded** out) {
    return guard([&] {
        if (out == nullptr || onnx == nullptr || size <= 0 || n_inputs <= 0 || ordinals == nullptr ||
            n_shards <= 0) {
            throw nb2::eng::LoadError("nb2_sharded_create: bad arguments");
        }
        *out = nullptr;
        std::map<std::string, std::vector<int64_t>> dims;
        int64_t at = 0, batch = -1;
        for (int i = 0; i < n_inputs; ++i) {
            std::vector<int64_t> d(dims_flat + at, dims_flat + at + ranks[i]);
            at += ranks[i];
            if (d.empty() || d[0] <= 0 || (batch >= 0 && d[0] != batch)) {
                throw nb2::eng::LoadError("nb2_sharded_create: every input must lead with the same batch dimension");
            }
            batch = d[0];
            dims[names[i]] = d;
        }
        if (flags & nb2::eng::kNoGraph) {
            // eager rows of two models on one stream could interleave between
            // a split-K launch and its reduction; graph replays cannot
            for (int i = 0; i < n_shards; ++i) {
                for (int j = 0; j < i; ++j) {
                    if (ordinals[i] == ordinals[j]) {
                        throw nb2::eng::LoadError("nb2_sharded_create: shards that share a GPU need CUDA-graph replay");
                    }
                }
            }
        }
        auto h = std::make_unique<nb2_sharded>();
        h->shards.resize(static_cast<size_t>(n_shards));
        std::vector<int64_t> offs(n_shards), counts(n_shards);
        nb2::eng::shard_plan(batch, n_shards, offs.data(), counts.data());
        for (int i = 0; i < n_shards; ++i) {
            auto& s = h->shards[i];
            s.ordinal = ordinals[i];
            s.offset = offs[i];
            s.count = counts[i];
            if (s.count == 0) {
                continue;
            }
            auto local = dims;
            for (auto& kv : local) {
                kv.second[0] = s.count;
            }
            // built one after another on this thread; each model's first
            // launch captures its CUDA graph here, on zeroed inputs, so the
            // worker threads only ever replay
            s.model = std::make_unique<Model>(static_cast<const uint8_t*>(onnx), static_cast<size_t>(size), local,
                                              s.ordinal, flags);
            for (const auto& io : s.model->outputs()) {
                if (io.dims.empty() || io.dims[0] != s.count) {
                    throw nb2::eng::LoadError("nb2_sharded_create: output '" + io.name +
                                              "' does not lead with the batch dimension");
                }
            }
            nb2_device* dev = s.model->device();
            dev->make_current();
            for (const auto& io : s.model->inputs()) {
                nb2::check_cuda(cudaMemsetAsync(io.dev, 0, static_cast<size_t>(io.bytes), dev->stream),
                                "cudaMemsetAsync(shard input)");
            }
            s.model->launch();
            dev->take_device_error(); // warm-up on zeros: its device errors mean nothing
        }
        const Model* first = nullptr;
        for (auto& s : h->shards) {
            if (s.model) {
                first = s.model.get();
                break;
            }
        }
        for (auto io : first->inputs()) {
            io.dims[0] = batch;
            h->in_image_bytes.push_back(tail_bytes(io));
            h->inputs.push_back(io);
        }
        for (auto io : first->outputs()) {
            io.dims[0] = batch;
            h->out_image_bytes.push_back(tail_bytes(io));
            h->outputs.push_back(io);
        }
        for (size_t i = 0; i < h->shards.size(); ++i) {
            if (h->shards[i].model) {
                nb2_sharded* raw = h.get();
                h->shards[i].worker = std::thread([raw, i] { raw->work(i); });
            }
        }
        *out = h.release();
    });
}

int nb2_sharded_destroy(nb2_sharded* s) {
    return guard([&] { delete s; });
}

int nb2_sharded_num_io(const nb2_sharded* s, int* n_inputs, int* n_outputs) {
    return guard([&] {
        if (s == nullptr) {
            throw nb2::eng::LoadError("null sharded model");
        }
        if (n_inputs) {
            *n_inputs = static_cast<int>(s->inputs.size());
        }
        if (n_outputs) {
            *n_outputs = static_cast<int>(s->outputs.size());
        }
    });
}

int nb2_sharded_io(const nb2_sharded* s, int is_output, int i, const char** name, int* dtype, int* rank,
                   int64_t* dims8) {
    return guard([&] {
        if (s == nullptr) {
            throw nb2::eng::LoadError("null sharded model");
        }
        const auto& v = is_output ? s->outputs : s->inputs;
        if (i < 0 || i >= static_cast<int>(v.size())) {
            throw nb2::eng::LoadError("io index out of range");
        }
        const auto& io = v[static_cast<size_t>(i)];
        if (name) {
            *name = io.name.c_str();
        }
        if (dtype) {
            *dtype = static_cast<int>(io.dtype);
        }
        if (rank) {
            *rank = static_cast<int>(io.dims.size());
        }
        if (dims8) {
            for (size_t d = 0; d < io.dims.size() && d < 8; ++d) {
                dims8[d] = io.dims[d];
            }
        }
    });
}

int nb2_sharded_shard(const nb2_sharded* s, int i, int* ordinal, int64_t* batch_offset, int64_t* batch_count) {
    return guard([&] {
        if (s == nullptr || i < 0 || i >= static_cast<int>(s->shards.size())) {
            throw nb2::eng::LoadError("shard index out of range");
        }
        const auto& sh = s->shards[static_cast<size_t>(i)];
        if (ordinal) {
            *ordinal = sh.ordinal;
        }
        if (batch_offset) {
            *batch_offset = sh.offset;
        }
        if (batch_count) {
            *batch_count = sh.count;
        }
    });
}

int nb2_sharded_run(nb2_sharded* s, const void* const* host_inputs, void* const* host_outputs) {
    return guard([&] {
        if (s == nullptr || host_inputs == nullptr || host_outputs == nullptr) {
            throw nb2::eng::RunError("nb2_sharded_run: bad arguments");
        }
        s->run(host_inputs, host_outputs);
    });
}

} // extern "C"
