// nb2_conv2d_noalloc: the Conv row for callers that must not allocate.
//
// nb2_conv2d packs (splits and reorders) the weight into the device
// workspace, which grows with cudaMalloc on first use of a larger layer.
// Some callers cannot allow that: a host framework that owns all device
// memory and forbids allocation once it is running (a plug-in executed from
// a framework's enqueue callback), or a service held to a fixed memory budget.
// This entry point keeps its scratch in one file-scope __device__ array of a
// fixed size instead, so a call allocates nothing; the caller still provides
// every input and output buffer.
//
// Rules of the array:
//   * kNoAllocScratchBytes (8 MiB) per GPU, held by every GPU that loads this
//     library until the process exits;
//   * its address is resolved once per device, with that device current, by
//     the first call on that device (cudaGetSymbolAddress may load the module
//     on the GPU), so make the first call on each device before any stream
//     capture begins;
//   * every call shares the array and leaves its contents behind: each call
//     rewrites every byte it reads (packed weights including their zero
//     padding, and the tap table), so nothing has to start at zero;
//   * calls whose kernels could overlap on the same GPU would race on the
//     array; calls on one device are issued in order on that device's single
//     stream.
// A weight whose packed form exceeds the array is rejected with
// NB2_ERR_INVALID and a message giving both sizes.

#include "../../include/nert_b200.h"
#include "igemm.cuh"
#include "runtime.hpp"

#include <mutex>
#include <new>
#include <string>

namespace nb2 {
ConvGeom conv_geom_from_c(const nb2_conv_geom* c); // capi.cu (validation shared with nb2_conv2d)
}

namespace {

constexpr size_t kNoAllocScratchBytes = 8u << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_addr_mu;
void* g_addr[64] = {};

// Device address of g_noalloc_scratch on `dev` (the host-side symbol is only a
// stand-in and must never be passed to a kernel). Resolved once per device.
void* scratch_address(nb2_device* dev) {
    std::lock_guard<std::mutex> lock(g_addr_mu);
    void*& slot = g_addr[dev->ordinal];
    if (slot == nullptr) {
        dev->make_current();
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr) {
            nb2::fail(nb2::kStatusCuda, std::string("cudaGetSymbolAddress(no-alloc scratch): ") + cudaGetErrorString(e));
        }
        slot = p;
    }
    return slot;
}

} // namespace

extern "C" int nb2_conv2d_noalloc(nb2_device* dev, const nb2_conv_geom* g, const float* x, const float* w,
                                  const float* bias, const float* residual, int act, float* y) {
    try {
        const nb2::ConvGeom geom = nb2::conv_geom_from_c(g);
        if (dev == nullptr || x == nullptr || w == nullptr || y == nullptr) {
            nb2::fail(nb2::kStatusInvalid, "Conv: null buffer");
        }
        const size_t need = nb2::conv_packed_bytes(geom);
        if (need > kNoAllocScratchBytes) {
            nb2::fail(nb2::kStatusInvalid, "Conv (no-alloc): packed weight needs " + std::to_string(need) +
                                               " bytes, above the " + std::to_string(kNoAllocScratchBytes) +
                                               "-byte static scratch; use nb2_conv2d");
        }
        dev->make_current();
        void* scratch = scratch_address(dev);
        // no split K here: the split-K workspace is shared, growable and
        // freed by nothing this call controls, so a layer that would split K
        // runs unsplit (same results, one kernel)
        struct NoGrow {
            nb2_device* d;
            int prev;
            ~NoGrow() { d->no_grow = prev; }
        } guard{dev, dev->no_grow};
        dev->no_grow = 1;
        nb2::conv_pack(dev, geom, w, scratch);
        nb2::Epilogue ep;
        ep.bias = bias;
        ep.res = residual;
        ep.act = act;
        nb2::conv_run(dev, geom, x, scratch, y, ep);
        return NB2_OK;
    } catch (const nb2::Error& e) {
        nb2::set_last_error(e.what());
        return e.code;
    } catch (const std::bad_alloc&) {
        nb2::set_last_error("out of host memory");
        return NB2_ERR_NOMEM;
    } catch (const std::exception& e) {
        nb2::set_last_error(e.what());
        return NB2_ERR_INVALID;
    }
}

extern "C" int64_t nb2_conv2d_noalloc_capacity(void) { return static_cast<int64_t>(kNoAllocScratchBytes); }
