// Per-GPU contexts, scratch workspace, device error word and host<->device
// copies of the B200 layer (see runtime.hpp).

#include "runtime.hpp"

#include <cuda.h>

#include <array>
#include <cstring>
#include <memory>

namespace nb2 {

namespace {
thread_local std::string g_last_error;
std::mutex g_devices_mu;
std::array<std::unique_ptr<nb2_device>, 64> g_devices;
} // namespace

void set_last_error(const std::string& msg) { g_last_error = msg; }
const char* last_error() { return g_last_error.c_str(); }

void fail(int code, const std::string& msg) { throw Error(code, msg); }

void check_cuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        fail(kStatusCuda, std::string(what) + ": " + cudaGetErrorString(e));
    }
}

EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        check_cuda(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q),
                   "cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)");
        if (p == nullptr || q != cudaDriverEntryPointSuccess) {
            fail(kStatusCuda, "cuTensorMapEncodeTiled is unavailable");
        }
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

EncodeIm2colFn encode_im2col() {
    static EncodeIm2colFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        check_cuda(cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &p, cudaEnableDefault, &q),
                   "cudaGetDriverEntryPoint(cuTensorMapEncodeIm2col)");
        if (p == nullptr || q != cudaDriverEntryPointSuccess) {
            fail(kStatusCuda, "cuTensorMapEncodeIm2col is unavailable");
        }
        return reinterpret_cast<EncodeIm2colFn>(p);
    }();
    return fn;
}

nb2_device* device(int ordinal) {
    if (ordinal < 0 || ordinal >= 64) {
        fail(kStatusInvalid, "device ordinal out of range");
    }
    std::lock_guard<std::mutex> lock(g_devices_mu);
    if (!g_devices[ordinal]) {
        int count = 0;
        check_cuda(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
        if (ordinal >= count) {
            fail(kStatusInvalid, "no CUDA device " + std::to_string(ordinal));
        }
        cudaDeviceProp prop{};
        check_cuda(cudaGetDeviceProperties(&prop, ordinal), "cudaGetDeviceProperties");
        if (prop.major != 10) {
            fail(kStatusUnsupported, std::string("the B200 layer needs an sm_100 GPU, found ") + prop.name);
        }
        auto dev = std::make_unique<nb2_device>();
        dev->ordinal = ordinal;
        dev->num_sms = prop.multiProcessorCount;
        check_cuda(cudaSetDevice(ordinal), "cudaSetDevice");
        check_cuda(cudaStreamCreateWithFlags(&dev->stream, cudaStreamNonBlocking), "cudaStreamCreate");
        check_cuda(cudaMalloc(&dev->err_word, 256), "cudaMalloc(error word)");
        check_cuda(cudaMemsetAsync(dev->err_word, 0, 256, dev->stream), "cudaMemsetAsync(error word)");
        check_cuda(cudaStreamSynchronize(dev->stream), "cudaStreamSynchronize");
        if (const char* env = std::getenv("NERT_B200_PRECISION")) {
            if (std::strcmp(env, "1xtf32") == 0 || std::strcmp(env, "1") == 0) {
                dev->precision = kPrec1xTF32;
            }
        }
        g_devices[ordinal] = std::move(dev);
    }
    return g_devices[ordinal].get();
}

} // namespace nb2

nb2_device::nb2_device() : wait_bound(nb2::kDefaultWaitBoundCycles) {}

void nb2_device::make_current() const { nb2::check_cuda(cudaSetDevice(ordinal), "cudaSetDevice"); }

void* nb2_device::scratch(size_t bytes) {
    bytes = (bytes + 255) & ~size_t(255);
    if (bytes <= workspace_bytes) {
        return workspace;
    }
    if (capturing) {
        nb2::fail(nb2::kStatusInvalid, "workspace must be sized before CUDA-graph capture");
    }
    nb2::check_cuda(cudaStreamSynchronize(stream), "cudaStreamSynchronize(workspace grow)");
    if (workspace != nullptr) {
        nb2::check_cuda(cudaFree(workspace), "cudaFree(workspace)");
        workspace = nullptr;
        workspace_bytes = 0;
    }
    const size_t grow = std::max(bytes, workspace_bytes * 2);
    nb2::check_cuda(cudaMalloc(&workspace, grow), "cudaMalloc(workspace)");
    workspace_bytes = grow;
    return workspace;
}

void* nb2_device::split_scratch(size_t bytes) {
    bytes = (bytes + 255) & ~size_t(255);
    if (no_grow) {
        return nullptr; // a no-allocation call never depends on this shared buffer
    }
    if (bytes <= split_ws_bytes) {
        return split_ws;
    }
    if (capturing) {
        return nullptr; // the caller then runs the contraction unsplit
    }
    const size_t grow = std::max(bytes, split_ws_bytes * 2);
    void* fresh = nullptr;
    nb2::check_cuda(cudaMalloc(&fresh, grow), "cudaMalloc(split workspace)");
    if (split_ws != nullptr) {
        retired_split.push_back(split_ws);
    }
    split_ws = fresh;
    split_ws_bytes = grow;
    return split_ws;
}

int nb2_device::take_device_error() {
    int code = 0;
    nb2::check_cuda(cudaMemcpyAsync(&code, err_word, sizeof(int), cudaMemcpyDeviceToHost, stream),
                    "cudaMemcpyAsync(error word)");
    nb2::check_cuda(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
    if (code != 0) {
        nb2::check_cuda(cudaMemsetAsync(err_word, 0, sizeof(int), stream), "cudaMemsetAsync(error word)");
        nb2::check_cuda(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
    }
    return code;
}
