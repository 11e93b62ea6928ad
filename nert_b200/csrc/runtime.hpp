// Per-GPU runtime state of the B200 execution layer.
//
// One `nb2_device` per CUDA ordinal, created on first use and kept for the
// life of the process (the reference's CudaDevice() is a process singleton,
// src/cuda_device.cpp:98-102; here there is one per GPU). Each owns:
//   * a non-blocking stream on which every row of that GPU is launched, so
//     rows return without synchronising (the reference syncs after each row,
//     e.g. src/cuda/relu.cu:68);
//   * a grow-only scratch workspace for per-call packing (no per-call
//     cudaMalloc);
//   * a device error word that kernels set instead of trapping (an index out
//     of range, a bounded wait that gave up), read at synchronisation points;
//   * a pinned bounce buffer so host->device copies can be asynchronous while
//     the caller's memory may be freed as soon as the call returns.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

struct nb2_device;

namespace nb2 {

// Thrown inside the library; converted to a status code at the C boundary.
struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

constexpr int kStatusInvalid = -1;
constexpr int kStatusCuda = -2;
constexpr int kStatusDevice = -3;
constexpr int kStatusUnsupported = -4;
constexpr int kStatusNoMem = -5;

[[noreturn]] void fail(int code, const std::string& msg);
void check_cuda(cudaError_t e, const char* what);
void set_last_error(const std::string& msg);

// Default bound of a tensor-core kernel's mbarrier waits, in clock64 ticks
// (about one second at the B200's SM clock).
constexpr long long kDefaultWaitBoundCycles = 2000000000LL;

// 0 = 3xTF32 (fp32-accurate, the default), 1 = 1xTF32 (opt-in).
enum Precision : int { kPrec3xTF32 = 0, kPrec1xTF32 = 1 };

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled();

using EncodeIm2colFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const int*, const int*, cuuint32_t, cuuint32_t,
                                    const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeIm2colFn encode_im2col();

} // namespace nb2

struct nb2_device {
    int ordinal = 0;
    cudaStream_t stream = nullptr;
    int* err_word = nullptr; // device int
    void* workspace = nullptr;
    size_t workspace_bytes = 0;
    void* pinned = nullptr;
    size_t pinned_bytes = 0;
    void* split_ws = nullptr; // split-K partial sums (grow-only)
    size_t split_ws_bytes = 0;
    // Split-K buffers outgrown by a later call. They are kept, not freed, for
    // the life of the process: a CUDA graph captured by an engine model may
    // still hold their address, and freeing them would let its replays write
    // into memory handed out again.
    std::vector<void*> retired_split;
    int precision = nb2::kPrec3xTF32;
    int capturing = 0; // inside a CUDA-graph capture: the workspace may not grow
    int no_grow = 0;   // inside a call that must not allocate: contractions never split K
    int num_sms = 148;
    // clock64 ticks after which a tensor-core kernel's mbarrier wait gives
    // up, records a device error and unwinds (default about one second)
    long long wait_bound;
    // schedule of the most recent contraction launch on this device (what
    // the host chose; read back by tests to confirm a case took its path)
    struct Schedule {
        int tile_n = 0;   // output tile width (64 or 128 columns)
        int alt = 0;      // 1: two tiles in flight, MMA issuers on alternate tiles
        int ksplit = 0;   // K slices (1 = unsplit)
        int a_mode = 0;   // how A reaches shared memory / TMEM
        int grid = 0;     // CTAs launched
        int64_t tiles = 0; // output tiles (before K slicing)
    } last_sched;
    std::mutex mu;

    nb2_device();

    // Makes this device current for the calling thread.
    void make_current() const;
    // Returns a workspace of at least `bytes` (256-B aligned). Growing it
    // synchronises the stream first, so pointers from earlier calls stay
    // valid until the kernels that use them have finished.
    void* scratch(size_t bytes);
    // Buffer for split-K partial sums of at least `bytes`, or nullptr inside a
    // call that must not allocate, or when it would have to grow inside a
    // CUDA-graph capture (the caller then runs without splitting K). Growing
    // synchronises the stream first and retires (keeps) the old buffer.
    void* split_scratch(size_t bytes);
    // Reads and clears the device error word (synchronises the stream).
    int take_device_error();
};

namespace nb2 {
nb2_device* device(int ordinal);
} // namespace nb2
