// Data-movement and selection rows (ops_move.cu, ops_topk.cu) and the engine
// hook that turns one graph node of those kinds into a launchable step.
#pragma once

#include "engine/graph.hpp"
#include "runtime.hpp"

#include <cstdint>
#include <functional>
#include <map>
#include <string>
#include <vector>

namespace nb2 {

// Copy `rows` rows of `row_bytes` between pitched buffers, for up to 64
// segments in one launch (Concat / Split: one segment per input / output).
struct CopySeg {
    const uint8_t* src;
    uint8_t* dst;
    int64_t src_pitch, dst_pitch, row_bytes, rows;
};
void segment_copy(nb2_device* dev, const std::vector<CopySeg>& segs);

// General permutation (rank <= 8), element size 1/4/8 bytes.
void transpose(nb2_device* dev, const void* x, void* y, const std::vector<int64_t>& in_dims,
               const std::vector<int64_t>& perm, int elem_bytes);

// Strided slice: y[i] = x[start + i*step] per axis.
void slice(nb2_device* dev, const void* x, void* y, const std::vector<int64_t>& in_dims,
           const std::vector<int64_t>& out_dims, const std::vector<int64_t>& starts, const std::vector<int64_t>& steps,
           int elem_bytes);

// Gather along one axis of [outer, axis_len, inner] by int64 indices;
// negative indices wrap, out-of-range ones set device error 2 and write 0.
void gather(nb2_device* dev, const void* x, const int64_t* idx, void* y, int64_t outer, int64_t axis_len,
            int64_t inner, int64_t n_idx, int elem_bytes);

// Resize by per-axis source tables (lower index, upper index, upper weight).
struct ResizeTables {
    int rank;
    std::vector<int64_t> in_dims, out_dims;
    std::vector<int64_t> lower, upper; // concatenated per axis
    std::vector<double> weight;
    std::vector<int64_t> axis_off;     // start of each axis in the tables
};
// near2: 1 / 0 when the caller knows whether this is a nearest resize of the
// last two axes only (every leading axis the identity); -1 = decide from the
// host copy of the tables in `t`.
void resize(nb2_device* dev, const void* x, void* y, const ResizeTables& t, const void* dev_tables, bool is_f32,
            int near2 = -1);

// Resize with the per-axis tables built on the device into `scratch`
// (resize_table_bytes(out_dims) bytes) — for callers without host tables.
size_t resize_table_bytes(const std::vector<int64_t>& out_dims);
void resize_on_device_tables(nb2_device* dev, const void* x, void* y, const std::vector<int64_t>& in_dims,
                             const std::vector<int64_t>& out_dims, const std::vector<double>& scales, int linear,
                             int transform, int nearest, bool is_f32, void* scratch);

void cast(nb2_device* dev, const void* x, int from, void* y, int to, int64_t n);

// TopK (largest, sorted) along the last axis of [rows, L]: values and int64
// indices ordered by (value desc, index asc). Long rows are split over many
// CTAs and need `scratch` of topk_scratch_bytes(rows, L, k) bytes (0 for
// short rows).
size_t topk_scratch_bytes(int64_t rows, int64_t L, int64_t k);
// kernels one topk() call launches
int topk_launches(int64_t rows, int64_t L, int64_t k);
void topk(nb2_device* dev, const float* x, float* values, int64_t* indices, int64_t rows, int64_t L, int64_t k,
          void* scratch);

namespace eng {
struct MoveStep {
    std::function<void(nb2_device*)> run;
    int launches = 1;
};
// Builds the step for Transpose/Concat/Split/Slice/Gather/TopK/Resize/Cast;
// `run` is empty for any other op. `nhwc`: the node's 4-D tensors are held
// channels-last ([N,H,W,C] in memory for the logical [N,C,H,W]); only
// Concat, Split and Resize accept it.
MoveStep build_move_step(const Node& n, const Graph& g, const std::map<std::string, TensorInfo>& shapes,
                         const std::function<void*(const std::string&)>& ptr,
                         const std::function<uint8_t*(int64_t)>& dmalloc, bool nhwc = false);
} // namespace eng

} // namespace nb2
