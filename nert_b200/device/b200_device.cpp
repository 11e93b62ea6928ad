// nert::b200::Device(ordinal) — the B200 layer behind NERT's device seam.
//
// Implements the seam of include/nert/device.hpp:22-77 unchanged, so a graph
// loaded by NERT's own loader runs on a B200 through the reference's own
// nert::Model (src/executor.cpp:202-560) by passing this handle instead of
// nert::CudaDevice() (src/cuda_device.cpp:98-102):
//
//   nert::Graph g = nert::LoadGraphFromFile("model.onnx");
//   nert::Model m(g, {{"input", {64, 3, 224, 224}}}, nert::b200::Device(0));
//   auto out = m.Run({{"input", pixels}});
//
// Every KernelFn row validates the node like the reference CPU row, then
// calls the C ABI of include/nert_b200.h, which launches on the GPU's stream
// and returns without synchronising (the reference rows sync after every op,
// e.g. src/cuda/relu.cu:68). Results reach the host through
// Transfer::device_to_host, which synchronises and reports device-recorded
// errors (a Gather index out of range, a bounded wait that expired) as
// nert::InferenceException.
//
// KernelFn carries no device, so KernelTable::find — which the executor calls
// on the same thread immediately before each kernel (src/executor.cpp:485) —
// records the table's GPU in a thread-local that the rows read.
//
// Small host->device uploads (<= 4 KB: Reshape shapes, Split sizes, TopK K,
// Slice bounds, Resize scales/sizes, ReduceMean axes) are mirrored on the
// host, so the rows read those constants without a device->host round trip
// (the reference rows read them back with cudaMemcpy, e.g. top_k.cu:112).

#include "nert/device.hpp"
#include "nert/graph.hpp"
#include "nert_b200.h"

#include <algorithm>
#include <array>
#include <cmath>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

namespace nert {
namespace b200 {

const ::nert::Device& Device(int ordinal);

namespace {

thread_local nb2_device* tl_device = nullptr;
thread_local std::map<const void*, std::vector<uint8_t>>* tl_mirror = nullptr;
struct DeviceState;
thread_local DeviceState* tl_state = nullptr;

// The tensor-core layout of a resident weight, packed on first use and kept
// until the weight's memory is released or written again (defined with the
// seam objects below). Returns null when `w` is not a resident upload (then
// the caller packs per call).
const void* cached_pack(const void* w, int64_t w_bytes, const std::string& key, int64_t packed_bytes,
                        const std::function<int(void*)>& pack, const std::string& ctx);

[[noreturn]] void fail(const std::string& ctx, const std::string& msg) { throw InferenceException(ctx + ": " + msg); }

void check(int status, const std::string& ctx) {
    if (status != NB2_OK) {
        fail(ctx, nb2_last_error());
    }
}

nb2_device* current(const std::string& ctx) {
    if (tl_device == nullptr) {
        fail(ctx, "no B200 device bound to this thread (call through the device's kernel table)");
    }
    return tl_device;
}

std::string context(const Node& node) { return node.op_type + " (node '" + node.name + "')"; }

int64_t count_of(const std::vector<int64_t>& dims) {
    int64_t n = 1;
    for (int64_t d : dims) {
        n *= d;
    }
    return n;
}

int elem_bytes(DataType t) {
    switch (t) {
    case DataType::Float32:
        return 4;
    case DataType::Int64:
        return 8;
    case DataType::Bool:
        return 1;
    default:
        return 0;
    }
}

const Attribute* find_attr(const Node& node, const std::string& name) {
    for (const Attribute& a : node.attributes) {
        if (a.name == name) {
            return &a;
        }
    }
    return nullptr;
}

int64_t int_attr(const Node& node, const std::string& name, int64_t def) {
    const Attribute* a = find_attr(node, name);
    if (a == nullptr) {
        return def;
    }
    const int64_t* v = std::get_if<int64_t>(&a->value);
    if (v == nullptr) {
        fail(context(node), "attribute '" + name + "' must be an integer");
    }
    return *v;
}

float float_attr(const Node& node, const std::string& name, float def) {
    const Attribute* a = find_attr(node, name);
    if (a == nullptr) {
        return def;
    }
    const float* v = std::get_if<float>(&a->value);
    if (v == nullptr) {
        fail(context(node), "attribute '" + name + "' must be a float");
    }
    return *v;
}

std::string str_attr(const Node& node, const std::string& name, const std::string& def) {
    const Attribute* a = find_attr(node, name);
    if (a == nullptr) {
        return def;
    }
    const std::string* v = std::get_if<std::string>(&a->value);
    if (v == nullptr) {
        fail(context(node), "attribute '" + name + "' must be a string");
    }
    return *v;
}

std::vector<int64_t> ints_attr(const Node& node, const std::string& name) {
    const Attribute* a = find_attr(node, name);
    if (a == nullptr) {
        return {};
    }
    const auto* v = std::get_if<std::vector<int64_t>>(&a->value);
    if (v == nullptr) {
        fail(context(node), "attribute '" + name + "' must be an int list");
    }
    return *v;
}

// The host bytes of a small device operand: the mirror of its upload, or a
// synchronising device->host read when it was computed on the device.
std::vector<uint8_t> host_bytes(const TensorView& v, const std::string& ctx) {
    const int64_t n = count_of(v.dims) * elem_bytes(v.dtype);
    if (n == 0) {
        return {};
    }
    if (v.data == nullptr) {
        fail(ctx, "null buffer");
    }
    if (tl_mirror != nullptr) {
        auto it = tl_mirror->find(v.data);
        if (it != tl_mirror->end() && static_cast<int64_t>(it->second.size()) >= n) {
            return std::vector<uint8_t>(it->second.begin(), it->second.begin() + n);
        }
    }
    std::vector<uint8_t> out(static_cast<size_t>(n));
    check(nb2_memcpy_d2h(current(ctx), out.data(), v.data, n), ctx);
    return out;
}

std::vector<int64_t> host_ints(const TensorView& v, const std::string& ctx) {
    const std::vector<uint8_t> b = host_bytes(v, ctx);
    std::vector<int64_t> out(static_cast<size_t>(count_of(v.dims)));
    if (v.dtype == DataType::Int64) {
        std::memcpy(out.data(), b.data(), out.size() * 8);
    } else if (v.dtype == DataType::Float32) {
        for (size_t i = 0; i < out.size(); ++i) {
            float f;
            std::memcpy(&f, b.data() + 4 * i, 4);
            out[i] = static_cast<int64_t>(f);
        }
    } else {
        fail(ctx, "expected an int64 operand");
    }
    return out;
}

std::vector<float> host_floats(const TensorView& v, const std::string& ctx) {
    if (v.dtype != DataType::Float32) {
        fail(ctx, "expected a float32 operand");
    }
    const std::vector<uint8_t> b = host_bytes(v, ctx);
    std::vector<float> out(static_cast<size_t>(count_of(v.dims)));
    std::memcpy(out.data(), b.data(), out.size() * 4);
    return out;
}

void expect_io(const Node& node, const std::vector<TensorView>& in, const std::vector<TensorView>& out, size_t in_min,
               size_t in_max, size_t out_n) {
    if (in.size() < in_min || in.size() > in_max || out.size() < out_n) {
        fail(context(node), "unexpected number of inputs or outputs");
    }
}

void expect_f32(const Node& node, const TensorView& v) {
    if (v.dtype != DataType::Float32) {
        fail(context(node), "tensors must be float32");
    }
}

// ---- window geometry (reference ResolvePads / WindowOutput, conv.cpp:78-135)

void resolve_pads(const Node& node, const std::vector<int64_t>& in_sp, const std::vector<int64_t>& k,
                  const std::vector<int64_t>& d, const std::vector<int64_t>& s, std::vector<int64_t>& pb,
                  std::vector<int64_t>& pe) {
    const size_t r = in_sp.size();
    pb.assign(r, 0);
    pe.assign(r, 0);
    const std::string ap = str_attr(node, "auto_pad", "NOTSET");
    if (ap == "VALID") {
        return;
    }
    if (ap == "SAME_UPPER" || ap == "SAME_LOWER") {
        for (size_t i = 0; i < r; ++i) {
            const int64_t out = (in_sp[i] + s[i] - 1) / s[i];
            const int64_t total = std::max<int64_t>(0, (out - 1) * s[i] + d[i] * (k[i] - 1) + 1 - in_sp[i]);
            if (ap == "SAME_UPPER") {
                pb[i] = total / 2;
                pe[i] = total - pb[i];
            } else {
                pe[i] = total / 2;
                pb[i] = total - pe[i];
            }
        }
        return;
    }
    const std::vector<int64_t> pads = ints_attr(node, "pads");
    if (pads.empty()) {
        return;
    }
    if (pads.size() != 2 * r) {
        fail(context(node), "pads must have two entries per spatial dimension");
    }
    for (size_t i = 0; i < r; ++i) {
        pb[i] = pads[i];
        pe[i] = pads[r + i];
    }
}

int64_t window_out(const Node& node, int64_t in, int64_t k, int64_t d, int64_t pb, int64_t pe, int64_t s, bool ceil_mode) {
    const int64_t numer = in + pb + pe - (d * (k - 1) + 1);
    if (numer < 0) {
        fail(context(node), "window is larger than the padded input");
    }
    return (ceil_mode ? (numer + s - 1) / s : numer / s) + 1;
}

// ---- rows ------------------------------------------------------------------

void Conv(const Node& node, const std::vector<TensorView>& in, const std::vector<TensorView>& out) {
    const std::string ctx = context(node);
    expect_io(node, in, out, 2, 3, 1);
    const TensorView& x = in[0];
    const TensorView& w = in[1];
    const TensorView& y = out[0];
    expect_f32(node, x);
    expect_f32(node, w);
    expect_f32(node, y);
    const bool has_bias = in.size() == 3 && in[2].data != nullptr;
    if (has_bias) {
        expect_f32(node, in[2]);
    }
    const size_t rank = x.dims.size();
    if (rank != 3 && rank != 4) {
        fail(ctx, rank == 5 ? "3-D convolution has no B200 row" : "input must be rank 3 or 4");
    }
    if (w.dims.size() != rank) {
        fail(ctx, "weight rank must match the input rank");
    }
    const size_t sp = rank - 2;
    const int64_t group = int_attr(node, "group", 1);
    if (group <= 0) {
        fail(ctx, "group must be positive");
    }
    if (x.dims[1] % group != 0) {
        fail(ctx, "input channels are not divisible by group");
    }
    if (w.dims[1] != x.dims[1] / group) {
        fail(ctx, "weight channel dimension does not match input/group");
    }
    std::vector<int64_t> s = ints_attr(node, "strides"), d = ints_attr(node, "dilations");
    if (s.empty()) {
        s.assign(sp, 1);
    }
    if (d.empty()) {
        d.assign(sp, 1);
    }
    if (s.size() != sp || d.size() != sp) {
        fail(ctx, "stride and dilation must have one entry per spatial dimension");
    }
    std::vector<int64_t> in_sp(x.dims.begin() + 2, x.dims.end()), k(w.dims.begin() + 2, w.dims.end()), pb, pe;
    resolve_pads(node, in_sp, k, d, s, pb, pe);
    std::vector<int64_t> expected = {x.dims[0], w.dims[0]};
    for (size_t i = 0; i < sp; ++i) {
        expected.push_back(window_out(node, in_sp[i], k[i], d[i], pb[i], pe[i], s[i], false));
    }
    if (y.dims != expected) {
        fail(ctx, "output shape does not match the convolution");
    }
    if (has_bias && (in[2].dims.size() != 1 || in[2].dims[0] != w.dims[0])) {
        fail(ctx, "bias must be rank-1 of length M");
    }
    const bool one = sp == 1;
    nb2_conv_geom g{};
    g.n = x.dims[0];
    g.c = x.dims[1];
    g.h = one ? 1 : x.dims[2];
    g.w = one ? x.dims[2] : x.dims[3];
    g.m = w.dims[0];
    g.kh = one ? 1 : w.dims[2];
    g.kw = one ? w.dims[2] : w.dims[3];
    g.oh = one ? 1 : y.dims[2];
    g.ow = one ? y.dims[2] : y.dims[3];
    g.stride_h = one ? 1 : s[0];
    g.stride_w = one ? s[0] : s[1];
    g.pad_top = one ? 0 : pb[0];
    g.pad_bottom = one ? 0 : pe[0];
    g.pad_left = one ? pb[0] : pb[1];
    g.pad_right = one ? pe[0] : pe[1];
    g.dil_h = one ? 1 : d[0];
    g.dil_w = one ? d[0] : d[1];
    g.group = group;
    nb2_device* dev = current(ctx);
    const float* bias = has_bias ? static_cast<const float*>(in[2].data) : nullptr;
    int64_t pbytes = 0;
    check(nb2_conv2d_packed_size(&g, &pbytes), ctx);
    // the weights of a loaded graph are resident uploads: split and reorder
    // them for the tensor cores once, not on every Run
    const std::string key = "conv:" + std::to_string(g.c) + "," + std::to_string(g.h) + "," + std::to_string(g.w) +
                            "," + std::to_string(g.m) + "," + std::to_string(g.kh) + "," + std::to_string(g.kw) +
                            "," + std::to_string(g.dil_h) + "," + std::to_string(g.dil_w) + "," +
                            std::to_string(g.group);
    const void* packed = cached_pack(
        w.data, count_of(w.dims) * 4, key, pbytes,
        [&](void* dst) { return nb2_conv2d_pack(dev, &g, static_cast<const float*>(w.data), dst); }, ctx);
    if (packed != nullptr) {
        check(nb2_conv2d_run_packed(dev, &g, static_cast<const float*>(x.data), packed, bias, nullptr, NB2_ACT_NONE,
                                    static_cast<float*>(y.data)),
              ctx);
        return;
    }
    check(nb2_conv2d(dev, &g, static_cast<const float*>(x.data), static_cast<const float*>(w.data), bias, nullptr,
                     NB2_ACT_NONE, static_cast<float*>(y.data)),
          ctx);
}

// ConvTranspose (src/kernels/conv_transpose.cpp:76-145): explicit pads
// (auto_pad NOTSET or VALID), output_padding, dilations, groups, bias [M].
void ConvTranspose(const Node& node, const std::vector<TensorView>& in, const std::vector<TensorView>& out) {
    const std::string ctx = context(node);
    expect_io(node, in, out, 2, 3, 1);
    const TensorView &x = in[0], &w = in[1], &y = out[0];
    expect_f32(node, x);
    expect_f32(node, w);
    if (x.dims.size() != 4 || w.dims.size() != 4) {
        fail(ctx, "input and weight must be rank 4 (NCHW)");
    }
    const int64_t group = int_attr(node, "group", 1);
    if (group <= 0 || x.dims[1] % group != 0 || w.dims[0] != x.dims[1]) {
        fail(ctx, "weight channels do not match the input and group");
    }
    std::vector<int64_t> s = ints_attr(node, "strides"), d = ints_attr(node, "dilations"),
                         op = ints_attr(node, "output_padding"), p = ints_attr(node, "pads");
    if (s.empty()) {
        s = {1, 1};
    }
    if (d.empty()) {
        d = {1, 1};
    }
    if (op.empty()) {
        op = {0, 0};
    }
    if (p.empty() || str_attr(node, "auto_pad", "NOTSET") == "VALID") {
        p = {0, 0, 0, 0};
    }
    if (s.size() != 2 || d.size() != 2 || op.size() != 2 || p.size() != 4) {
        fail(ctx, "strides, dilations, output_padding, and pads must be 2-D");
    }
    const bool has_bias = in.size() == 3 && in[2].data != nullptr;
    const int64_t m = w.dims[1] * group;
    if (has_bias && (in[2].dims.size() != 1 || in[2].dims[0] != m)) {
        fail(ctx, "bias must be rank-1 of length M");
    }
    nb2_convt_geom g{};
    g.n = x.dims[0];
    g.c = x.dims[1];
    g.h = x.dims[2];
    g.w = x.dims[3];
    g.m = m;
    g.kh = w.dims[2];
    g.kw = w.dims[3];
    g.oh = y.dims.size() == 4 ? y.dims[2] : -1;
    g.ow = y.dims.size() == 4 ? y.dims[3] : -1;
    g.stride_h = s[0];
    g.stride_w = s[1];
    g.pad_top = p[0];
    g.pad_left = p[1];
    g.pad_bottom = p[2];
    g.pad_right = p[3];
    g.dil_h = d[0];
    g.dil_w = d[1];
    g.out_pad_h = op[0];
    g.out_pad_w = op[1];
    g.group = group;
    check(nb2_conv_transpose2d(current(ctx), &g, static_cast<const float*>(x.data), static_cast<const float*>(w.data),
                               has_bias ? static_cast<const float*>(in[2].data) : nullptr,
                               static_cast<float*>(y.data)),
          ctx);
}

void Gemm(const Node& node, const std::vector<TensorView>& in, const std::vector<TensorView>& out) {
    const std::string ctx = context(node);
    expect_io(node, in, out, 2, 3, 1);
    const TensorView &a = in[0], &b = in[1], &y = out[0];
    expect_f32(node, a);
    expect_f32(node, b);
    if (a.dims.size() != 2 || b.dims.size() != 2) {
        fail(ctx, "A and B must be rank-2");
    }
    const int64_t ta = int_attr(node, "transA", 0), tb = int_attr(node, "transB", 0);
    const float alpha = float_attr(node, "alpha", 1.0f), beta = float_attr(node, "beta", 1.0f);
    const int64_t m = ta ? a.dims[1] : a.dims[0], k = ta ? a.dims[0] : a.dims[1];
    const int64_t kb = tb ? b.dims[1] : b.dims[0], n = tb ? b.dims[0] : b.dims[1];
    if (k != kb) {
        fail(ctx, "contraction dimension mismatch");
    }
    if (y.dims != std::vector<int64_t>{m, n}) {
        fail(ctx, "output shape does not match the operands");
    }
    int c_rank = 0;
    const float* c = nullptr;
    if (in.size() == 3 && in[2].data != nullptr) {
        const TensorView& cv = in[2];
        expect_f32(node, cv);
        if (cv.dims.size() == 1 && cv.dims[0] == n) {
            c_rank = 1;
        } else if (cv.dims.size() == 2 && cv.dims[0] == m && cv.dims[1] == n) {
            c_rank = 2;
        } else {
            fail(ctx, "bias shape must be [N] or [M,N]");
        }
        c = static_cast<const float*>(cv.data);
    }
    nb2_device* dev = current(ctx);
    int64_t pbytes = 0;
    check(nb2_gemm_packed_size(n, k, &pbytes), ctx);
    const void* packed = cached_pack(
        b.data, count_of(b.dims) * 4, "gemm:" + std::to_string(n) + "," + std::to_string(k) + "," + std::to_string(tb),
        pbytes,
        [&](void* dst) { return nb2_gemm_pack(dev, static_cast<const float*>(b.data), n, k, static_cast<int>(tb), dst); },
        ctx);
    if (packed != nullptr) {
        check(nb2_gemm_run_packed(dev, static_cast<const float*>(a.data), packed, c, c_rank,
                                  static_cast<float*>(y.data), m, n, k, static_cast<int>(ta), alpha, beta,
                                  NB2_ACT_NONE),
              ctx);
        return;
    }
    check(nb2_gemm(dev, static_cast<const float*>(a.data), static_cast<const float*>(b.data), c, c_rank,
                   static_cast<float*>(y.data), m, n, k, static_cast<int>(ta), static_cast<int>(tb), alpha, beta,
                   NB2_ACT_NONE),
          ctx);
}

void MatMul(const Node& node, const std::vector<TensorView>& in, const std::vector<TensorView>& out) {
    const std::string ctx = context(node);
    expect_io(node, in, out, 2, 2, 1);
    expect_f32(node, in[0]);
    expect_f32(node, in[1]);
    const TensorView &a = in[0], &b = in[1];
    if (b.dims.size() == 2 && a.dims.size() >= 2 && a.dims.back() == b.dims[0]) {
        // a rank-2 B (a linear layer's weight) shared by every batch: one
        // contraction over all of A's rows with B packed once
        nb2_device* dev = current(ctx);
        const int64_t k = b.dims[0], n = b.dims[1], m = count_of(a.dims) / k;
        std::vector<int64_t> want(a.dims.begin(), a.dims.end() - 1);
        want.push_back(n);
        if (out[0].dims != want) {
            fail(ctx, "output shape does not match the operands");
        }
        int64_t pbytes = 0;
        check(nb2_gemm_packed_size(n, k, &pbytes), ctx);
        const void* packed = cached_pack(
            b.data, count_of(b.dims) * 4, "gemm:" + std::to_string(n) + "," + std::to_string(k) + ",0", pbytes,
            [&](void* dst) { return nb2_gemm_pack(dev, static_cast<const float*>(b.data), n, k, 0, dst); }, ctx);
        if (packed != nullptr && m > 0) {
            check(nb2_gemm_run_packed(dev, static_cast<const float*>(a.data), packed, nullptr, 0,
                                      static_cast<float*>(out[0].data), m, n, k, 0, 1.0f, 1.0f, NB2_ACT_NONE),
                  ctx);
            return;
        }
    }
    check(nb2_matmul(current(ctx), static_cast<const float*>(in[0].data), in[0].dims.data(),
                     static_cast<int>(in[0].dims.size()), static_cast<const float*>(in[1].data), in[1].dims.data(),
                     static_cast<int>(in[1].dims.size()), static_cast<float*>(out[0].data)),
          ctx);
}

template <int OP>
void Unary(const Node& node, const std::vector<TensorView>& in, const std::vector<TensorView>& out) {
    const std::string ctx = context(node);
    expect_io(node, in, out, 1, 1, 1);
    expect_f32(node, in[0]);
    expect_f32(node, out[0]);
    const int64_t n = count_of(out[0].dims);
    if (count_of(in[0].dims) != n) {
        fail(ctx, "element-count mismatch");
    }
    check(nb2_unary(current(ctx), OP, static_cast<const float*>(in[0].data), static_cast<float*>(out[0].data), n),
          ctx);
}

template <int OP>
void Binary(const Node& node, const std::vector<TensorView>& in, const std::vector<TensorView>& out) {
    const std::string ctx = context(node);
    expect_io(node, in, out, 2, 2, 1);
    if (in[0].dtype != in[1].dtype || in[0].dtype != out[0].dtype) {
        fail(ctx, "operands must share one dtype");
    }
    int dt;
    if (in[0].dtype == DataType::Float32) {
        dt = NB2_F32;
    } else if (in[0].dtype == DataType::Int64 && OP != NB2_BINARY_POW) {
        dt = NB2_I64;
    } else {
        fail(ctx, "tensors must be float32 or int64");
    }
    check(nb2_binary(current(ctx), OP, dt, in[0].data, in[0].dims.data(), static_cast<int>(in[0].dims.size()),
                     in[1].data, in[1].dims.data(), static_cast<int>(in[1].dims.size()), out[0].data,
                     out[0].dims.data(), static_cast<int>(out[0].dims.size())),
          ctx);
}

void MaxPool(const Node& node, const std::vector<TensorView>& in, const std::vector<TensorView>& out) {
    const std::string ctx = context(node);
    expect_io(node, in, out, 1, 1, 1);
    const TensorView &x = in[0], &y = out[0];
    expect_f32(node, x);
    if (x.dims.size() != 4) {
        fail(ctx, "input must be rank 4 (NCHW)");
    }
    if (out.size() > 1 && out[1].data != nullptr) {
        fail(ctx, "the Indices output has no B200 row");
    }
    const std::vector<int64_t> k = ints_attr(node, "kernel_shape");
    if (k.size() != 2) {
        fail(ctx, k.empty() ? "kernel_shape is required" : "kernel_shape must have two spatial entries");
    }
    std::vector<int64_t> s = ints_attr(node, "strides"), d = ints_attr(node, "dilations");
    if (s.empty()) {
        s = {1, 1};
    }
    if (d.empty()) {
        d = {1, 1};
    }
    const bool ceil_mode = int_attr(node, "ceil_mode", 0) != 0;
    std::vector<int64_t> pb, pe;
    resolve_pads(node, {x.dims[2], x.dims[3]}, k, d, s, pb, pe);
    const std::vector<int64_t> expected = {x.dims[0], x.dims[1],
                                           window_out(node, x.dims[2], k[0], d[0], pb[0], pe[0], s[0], ceil_mode),
                                           window_out(node, x.dims[3], k[1], d[1], pb[1], pe[1], s[1], ceil_mode)};
    if (y.dims != expected) {
        fail(ctx, "output shape does not match the pooling window");
    }
    const int64_t pads[4] = {pb[0], pb[1], pe[0], pe[1]};
    check(nb2_maxpool2d(current(ctx), static_cast<const float*>(x.data), x.dims.data(), static_cast<float*>(y.data),
                        y.dims.data(), k.data(), s.data(), pads, d.data()),
          ctx);
}

// AveragePool (src/kernels/average_pool.cpp:128-225): dilations fixed at 1,
// count_include_pad selects the divisor.
void AveragePool(const Node& node, const std::vector<TensorView>& in, const std::vector<TensorView>& out) {
    const std::string ctx = context(node);
    expect_io(node, in, out, 1, 1, 1);
    const TensorView &x = in[0], &y = out[0];
    expect_f32(node, x);
    expect_f32(node, y);
    if (x.dims.size() != 4) {
        fail(ctx, "input must be rank 4 (NCHW)");
    }
    const std::vector<int64_t> k = ints_attr(node, "kernel_shape");
    if (k.size() != 2) {
        fail(ctx, "kernel_shape must have two spatial entries");
    }
    std::vector<int64_t> s = ints_attr(node, "strides");
    if (s.empty()) {
        s = {1, 1};
    }
    if (s.size() != 2) {
        fail(ctx, "strides must have two spatial entries");
    }
    const std::vector<int64_t> d = {1, 1};
    const bool ceil_mode = int_attr(node, "ceil_mode", 0) != 0;
    std::vector<int64_t> pb, pe;
    resolve_pads(node, {x.dims[2], x.dims[3]}, k, d, s, pb, pe);
    const std::vector<int64_t> expected = {x.dims[0], x.dims[1],
                                           window_out(node, x.dims[2], k[0], 1, pb[0], pe[0], s[0], ceil_mode),
                                           window_out(node, x.dims[3], k[1], 1, pb[1], pe[1], s[1], ceil_mode)};
    if (y.dims != expected) {
        fail(ctx, "output shape does not match the pooling window");
    }
    const int64_t pads[4] = {pb[0], pb[1], pe[0], pe[1]};
    check(nb2_avgpool2d(current(ctx), static_cast<const float*>(x.data), x.dims.data(), static_cast<float*>(y.data),
                        y.dims.data(), k.data(), s.data(), pads, int_attr(node, "count_include_pad", 0) != 0 ? 1 : 0),
          ctx);
}

void GlobalAveragePool(const Node& node, const std::vector<TensorView>& in, const std::vector<TensorView>& out) {
    const std::string ctx = context(node);
    expect_io(node, in, out, 1, 1, 1);
    expect_f32(node, in[0]);
    if (in[0].dims.size() < 2) {
        fail(ctx, "input must have batch and channel axes (rank at least 2)");
    }
    const int64_t rows = in[0].dims[0] * in[0].dims[1];
    const int64_t inner = rows == 0 ? 0 : count_of(in[0].dims) / rows;
    check(nb2_row_mean(current(ctx), static_cast<const float*>(in[0].data), rows, std::max<int64_t>(inner, 1),
                       static_cast<float*>(out[0].data)),
          ctx);
}

void ReduceMean(const Node& node, const std::vector<TensorView>& in, const std::vector<TensorView>& out) {
    const std::string ctx = context(node);
    expect_f32(node, in[0]);
    const int64_t r = static_cast<int64_t>(in[0].dims.size());
    std::vector<int64_t> axes;
    if (node.schema_version != 0 && node.schema_version < 18) {
        axes = ints_attr(node, "axes");
    } else if (in.size() > 1 && in[1].data != nullptr) {
        axes = host_ints(in[1], ctx);
    } else {
        axes = ints_attr(node, "axes");
    }
    std::vector<bool> red(static_cast<size_t>(r), axes.empty());
    for (int64_t a : axes) {
        if (a < -r || a >= r) {
            fail(ctx, "axis out of range");
        }
        red[static_cast<size_t>(a < 0 ? a + r : a)] = true;
    }
    int64_t first = r;
    for (int64_t i = 0; i < r; ++i) {
        if (red[static_cast<size_t>(i)]) {
            first = std::min(first, i);
        }
    }
    for (int64_t i = first; i < r; ++i) {
        if (!red[static_cast<size_t>(i)]) {
            fail(ctx, "only trailing-axis means have a B200 row");
        }
    }
    int64_t rows = 1, inner = 1;
    for (int64_t i = 0; i < r; ++i) {
        (i < first ? rows : inner) *= in[0].dims[static_cast<size_t>(i)];
    }
    check(nb2_row_mean(current(ctx), static_cast<const float*>(in[0].data), rows, inner,
                       static_cast<float*>(out[0].data)),
          ctx);
}

void Softmax(const Node& node, const std::vector<TensorView>& in, const std::vector<TensorView>& out) {
    const std::string ctx = context(node);
    expect_io(node, in, out, 1, 1, 1);
    expect_f32(node, in[0]);
    const int64_t r = static_cast<int64_t>(in[0].dims.size());
    const bool legacy = node.schema_version != 0 && node.schema_version < 13;
    int64_t axis = int_attr(node, "axis", legacy ? 1 : -1);
    if (axis < -r || axis >= r) {
        fail(ctx, "axis out of range");
    }
    if (axis < 0) {
        axis += r;
    }
    int64_t outer = 1, len = 1, inner = 1;
    for (int64_t i = 0; i < r; ++i) {
        const int64_t v = in[0].dims[static_cast<size_t>(i)];
        if (legacy) {
            (i < axis ? outer : len) *= v; // 2-D coercion (src/softmax_form.hpp)
        } else {
            (i < axis ? outer : i == axis ? len : inner) *= v;
        }
    }
    check(nb2_softmax(current(ctx), static_cast<const float*>(in[0].data), static_cast<float*>(out[0].data), outer,
                      len, inner),
          ctx);
}

void LayerNormalization(const Node& node, const std::vector<TensorView>& in, const std::vector<TensorView>& out) {
    const std::string ctx = context(node);
    expect_io(node, in, out, 2, 3, 1);
    expect_f32(node, in[0]);
    const int64_t r = static_cast<int64_t>(in[0].dims.size());
    int64_t axis = int_attr(node, "axis", -1);
    if (axis < -r || axis >= r) {
        fail(ctx, "axis out of range");
    }
    if (axis < 0) {
        axis += r;
    }
    int64_t rows = 1, d = 1;
    for (int64_t i = 0; i < r; ++i) {
        (i < axis ? rows : d) *= in[0].dims[static_cast<size_t>(i)];
    }
    if (count_of(in[1].dims) != d) {
        fail(ctx, "scale must cover the normalised axes");
    }
    const float* bias = in.size() > 2 && in[2].data != nullptr ? static_cast<const float*>(in[2].data) : nullptr;
    float* mean = out.size() > 1 ? static_cast<float*>(out[1].data) : nullptr;
    float* inv = out.size() > 2 ? static_cast<float*>(out[2].data) : nullptr;
    check(nb2_layernorm(current(ctx), static_cast<const float*>(in[0].data), static_cast<const float*>(in[1].data),
                        bias, static_cast<float*>(out[0].data), mean, inv, rows, d,
                        float_attr(node, "epsilon", 1e-5f)),
          ctx);
}

// Flatten / Reshape / Squeeze / Unsqueeze / Identity: the output is its own
// arena slice, so the bytes move once (device to device, on the stream).
void CopyView(const Node& node, const std::vector<TensorView>& in, const std::vector<TensorView>& out) {
    const std::string ctx = context(node);
    if (in.empty() || out.size() != 1) {
        fail(ctx, "expected one data input and one output");
    }
    const int64_t n = count_of(out[0].dims) * elem_bytes(out[0].dtype);
    if (count_of(in[0].dims) * elem_bytes(in[0].dtype) != n) {
        fail(ctx, "element-count mismatch");
    }
    check(nb2_memcpy_d2d(current(ctx), out[0].data, in[0].data, n), ctx);
}

int64_t norm_axis(const std::string& ctx, int64_t a, int64_t r) {
    if (a < -r || a >= r) {
        fail(ctx, "axis out of range");
    }
    return a < 0 ? a + r : a;
}

void Transpose(const Node& node, const std::vector<TensorView>& in, const std::vector<TensorView>& out) {
    const std::string ctx = context(node);
    expect_io(node, in, out, 1, 1, 1);
    const int64_t r = static_cast<int64_t>(in[0].dims.size());
    std::vector<int64_t> perm = ints_attr(node, "perm");
    if (perm.empty()) {
        for (int64_t i = 0; i < r; ++i) {
            perm.push_back(r - 1 - i);
        }
    }
    if (static_cast<int64_t>(perm.size()) != r) {
        fail(ctx, "perm must list every axis");
    }
    for (auto& p : perm) {
        p = norm_axis(ctx, p, r);
    }
    check(nb2_transpose(current(ctx), in[0].data, out[0].data, in[0].dims.data(), perm.data(), static_cast<int>(r),
                        elem_bytes(in[0].dtype)),
          ctx);
}

void ConcatSplit(const Node& node, const TensorView& whole, const std::vector<const TensorView*>& parts, bool concat) {
    const std::string ctx = context(node);
    const int64_t r = static_cast<int64_t>(whole.dims.size());
    const int64_t axis = norm_axis(ctx, int_attr(node, "axis", 0), r);
    int64_t outer = 1, inner = 1;
    for (int64_t i = 0; i < axis; ++i) {
        outer *= whole.dims[static_cast<size_t>(i)];
    }
    for (int64_t i = axis + 1; i < r; ++i) {
        inner *= whole.dims[static_cast<size_t>(i)];
    }
    std::vector<void*> ptrs;
    std::vector<int64_t> lens;
    for (const TensorView* p : parts) {
        if (p->dtype != whole.dtype || p->dims.size() != whole.dims.size()) {
            fail(ctx, "parts must share the dtype and rank");
        }
        ptrs.push_back(p->data);
        lens.push_back(p->dims[static_cast<size_t>(axis)]);
    }
    check(nb2_concat_split(current(ctx), concat ? 1 : 0, whole.data, ptrs.data(), lens.data(),
                           static_cast<int>(ptrs.size()), outer, inner, elem_bytes(whole.dtype)),
          ctx);
}

void Concat(const Node& node, const std::vector<TensorView>& in, const std::vector<TensorView>& out) {
    std::vector<const TensorView*> parts;
    for (const auto& v : in) {
        parts.push_back(&v);
    }
    ConcatSplit(node, out.at(0), parts, true);
}

void Split(const Node& node, const std::vector<TensorView>& in, const std::vector<TensorView>& out) {
    std::vector<const TensorView*> parts;
    for (const auto& v : out) {
        parts.push_back(&v);
    }
    ConcatSplit(node, in.at(0), parts, false);
}

void Slice(const Node& node, const std::vector<TensorView>& in, const std::vector<TensorView>& out) {
    const std::string ctx = context(node);
    expect_io(node, in, out, 3, 5, 1);
    const TensorView& x = in[0];
    const int64_t r = static_cast<int64_t>(x.dims.size());
    const std::vector<int64_t> starts = host_ints(in[1], ctx);
    std::vector<int64_t> axes, steps;
    if (in.size() > 3 && in[3].data != nullptr) {
        axes = host_ints(in[3], ctx);
    } else {
        for (size_t i = 0; i < starts.size(); ++i) {
            axes.push_back(static_cast<int64_t>(i));
        }
    }
    if (in.size() > 4 && in[4].data != nullptr) {
        steps = host_ints(in[4], ctx);
    } else {
        steps.assign(starts.size(), 1);
    }
    std::vector<int64_t> s0(static_cast<size_t>(r), 0), sp(static_cast<size_t>(r), 1);
    for (size_t i = 0; i < starts.size(); ++i) {
        const int64_t a = norm_axis(ctx, axes[i], r);
        const int64_t dim = x.dims[static_cast<size_t>(a)];
        if (steps[i] == 0) {
            fail(ctx, "step must be non-zero");
        }
        int64_t s = starts[i] < 0 ? starts[i] + dim : starts[i];
        s = steps[i] > 0 ? std::clamp<int64_t>(s, 0, dim) : std::clamp<int64_t>(s, 0, dim - 1);
        s0[static_cast<size_t>(a)] = s;
        sp[static_cast<size_t>(a)] = steps[i];
    }
    if (count_of(out[0].dims) == 0) {
        return;
    }
    check(nb2_slice(current(ctx), x.data, out[0].data, x.dims.data(), out[0].dims.data(), s0.data(), sp.data(),
                    static_cast<int>(r), elem_bytes(x.dtype)),
          ctx);
}

void Gather(const Node& node, const std::vector<TensorView>& in, const std::vector<TensorView>& out) {
    const std::string ctx = context(node);
    expect_io(node, in, out, 2, 2, 1);
    if (in[1].dtype != DataType::Int64) {
        fail(ctx, "indices must be int64");
    }
    const int64_t r = static_cast<int64_t>(in[0].dims.size());
    const int64_t axis = norm_axis(ctx, int_attr(node, "axis", 0), r);
    int64_t outer = 1, inner = 1;
    for (int64_t i = 0; i < axis; ++i) {
        outer *= in[0].dims[static_cast<size_t>(i)];
    }
    for (int64_t i = axis + 1; i < r; ++i) {
        inner *= in[0].dims[static_cast<size_t>(i)];
    }
    check(nb2_gather(current(ctx), in[0].data, static_cast<const int64_t*>(in[1].data), out[0].data, outer,
                     in[0].dims[static_cast<size_t>(axis)], inner, count_of(in[1].dims), elem_bytes(in[0].dtype)),
          ctx);
}

void TopK(const Node& node, const std::vector<TensorView>& in, const std::vector<TensorView>& out) {
    const std::string ctx = context(node);
    expect_io(node, in, out, 2, 2, 2);
    expect_f32(node, in[0]);
    if (int_attr(node, "largest", 1) != 1 || int_attr(node, "sorted", 1) != 1) {
        fail(ctx, "only largest=1 and sorted=1 are supported");
    }
    const int64_t r = static_cast<int64_t>(in[0].dims.size());
    if (norm_axis(ctx, int_attr(node, "axis", -1), r) != r - 1) {
        fail(ctx, "the B200 TopK row selects along the last axis");
    }
    const std::vector<int64_t> kv = host_ints(in[1], ctx);
    if (kv.size() != 1) {
        fail(ctx, "K must be a single int64");
    }
    const int64_t len = in[0].dims.back();
    const int64_t rows = len == 0 ? 0 : count_of(in[0].dims) / len;
    check(nb2_topk(current(ctx), static_cast<const float*>(in[0].data), static_cast<float*>(out[0].data),
                   static_cast<int64_t*>(out[1].data), rows, len, kv[0]),
          ctx);
}

void Resize(const Node& node, const std::vector<TensorView>& in, const std::vector<TensorView>& out) {
    const std::string ctx = context(node);
    expect_io(node, in, out, 1, 4, 1);
    const std::string mode = str_attr(node, "mode", "nearest");
    if (mode != "nearest" && mode != "linear") {
        fail(ctx, "Resize 'mode' must be 'nearest' or 'linear' here");
    }
    const std::string tr = str_attr(node, "coordinate_transformation_mode", "half_pixel");
    const std::string nm = str_attr(node, "nearest_mode", "round_prefer_floor");
    static const std::map<std::string, int> trs = {
        {"half_pixel", 0}, {"pytorch_half_pixel", 1}, {"align_corners", 2}, {"asymmetric", 3}};
    static const std::map<std::string, int> nms = {
        {"round_prefer_floor", 0}, {"round_prefer_ceil", 1}, {"floor", 2}, {"ceil", 3}};
    if (!trs.count(tr)) {
        fail(ctx, "unsupported coordinate_transformation_mode '" + tr + "'");
    }
    if (!nms.count(nm)) {
        fail(ctx, "unsupported nearest_mode '" + nm + "'");
    }
    const TensorView &x = in[0], &y = out[0];
    const size_t rank = x.dims.size();
    std::vector<double> scales(rank, 1.0);
    const bool has_sizes = in.size() > 3 && in[3].data != nullptr;
    const bool has_scales = in.size() > 2 && in[2].data != nullptr && count_of(in[2].dims) > 0;
    if (has_sizes == has_scales) {
        fail(ctx, "Resize takes exactly one of scales and sizes");
    }
    if (has_sizes) {
        const std::vector<int64_t> sizes = host_ints(in[3], ctx);
        if (sizes.size() != rank || sizes != y.dims) {
            fail(ctx, "output shape does not match the sizes input");
        }
        for (size_t i = 0; i < rank; ++i) {
            scales[i] = static_cast<double>(static_cast<float>(sizes[i]) / static_cast<float>(x.dims[i]));
        }
    } else {
        const std::vector<float> sc = host_floats(in[2], ctx);
        if (sc.size() != rank) {
            fail(ctx, "Resize scales rank must match the input rank");
        }
        for (size_t i = 0; i < rank; ++i) {
            scales[i] = static_cast<double>(sc[i]);
            if (static_cast<int64_t>(std::floor(static_cast<double>(x.dims[i]) * scales[i])) != y.dims[i]) {
                fail(ctx, "output shape does not match the scaled input");
            }
        }
    }
    const int dt = x.dtype == DataType::Float32 ? NB2_F32 : x.dtype == DataType::Int64 ? NB2_I64 : -1;
    check(nb2_resize(current(ctx), x.data, y.data, x.dims.data(), y.dims.data(), scales.data(), static_cast<int>(rank),
                     mode == "linear" ? 1 : 0, trs.at(tr), nms.at(nm), dt),
          ctx);
}

void Cast(const Node& node, const std::vector<TensorView>& in, const std::vector<TensorView>& out) {
    const std::string ctx = context(node);
    expect_io(node, in, out, 1, 1, 1);
    auto code = [&](DataType t) {
        switch (t) {
        case DataType::Float32:
            return NB2_F32;
        case DataType::Int64:
            return NB2_I64;
        case DataType::Bool:
            return NB2_BOOL;
        default:
            fail(ctx, "unsupported dtype");
        }
    };
    check(nb2_cast(current(ctx), in[0].data, code(in[0].dtype), out[0].data, code(out[0].dtype),
                   count_of(in[0].dims)),
          ctx);
}

// Every row runs through this wrapper: views whose memory kernels cannot read
// (pageable host memory) are staged through device buffers, inputs copied in
// before the row and outputs copied back after it. The executor only passes
// arena and resident views (no staging); the reference's FoldConstants passes
// the initializers' own host bytes to whatever device it is given
// (src/constant_folding.cpp:32-95), and then this makes the row work anyway.
template <KernelFn F>
void HostSafe(const Node& node, const std::vector<TensorView>& in, const std::vector<TensorView>& out) {
    bool host = false;
    for (const auto* vs : {&in, &out}) {
        for (const TensorView& v : *vs) {
            host = host || (v.data != nullptr && nb2_pointer_on_device(v.data) == 0);
        }
    }
    if (!host) {
        F(node, in, out);
        return;
    }
    const std::string ctx = context(node);
    nb2_device* dev = current(ctx);
    std::vector<void*> owned;
    auto stage = [&](const std::vector<TensorView>& vs, bool upload) {
        std::vector<TensorView> d = vs;
        for (TensorView& v : d) {
            if (v.data == nullptr || nb2_pointer_on_device(v.data) != 0) {
                continue;
            }
            const int64_t bytes = count_of(v.dims) * elem_bytes(v.dtype);
            void* p = nullptr;
            if (bytes > 0) {
                check(nb2_device_malloc(dev, bytes, &p), ctx);
                owned.push_back(p);
                if (upload) {
                    check(nb2_memcpy_h2d(dev, p, v.data, bytes), ctx);
                }
            }
            v.data = p;
        }
        return d;
    };
    try {
        const std::vector<TensorView> din = stage(in, true), dout = stage(out, false);
        F(node, din, dout);
        for (size_t i = 0; i < out.size(); ++i) {
            if (out[i].data != nullptr && dout[i].data != out[i].data) {
                check(nb2_memcpy_d2h(dev, out[i].data, dout[i].data, count_of(out[i].dims) * elem_bytes(out[i].dtype)),
                      ctx);
            }
        }
    } catch (...) {
        for (void* p : owned) {
            nb2_device_free(dev, p);
        }
        throw;
    }
    for (void* p : owned) {
        nb2_device_free(dev, p);
    }
}

// ---- seam objects ------------------------------------------------------------

struct DeviceState {
    int ordinal = 0;
    nb2_device* dev = nullptr;
    std::map<const void*, std::vector<uint8_t>> mirror;
    std::multimap<int64_t, void*> pool; // released buffers kept for reuse, by size
    std::unordered_map<void*, int64_t> sizes;
    // bytes written by host_to_device at each destination since it was last
    // (re)allocated: the executor uploads every initializer into a buffer of
    // its own once per Model (src/executor.cpp:390-413)
    std::map<const void*, int64_t> uploads;
    // packed tensor-core layouts of resident weights, by weight address
    struct Packed {
        std::string key;
        void* buf = nullptr;
    };
    std::map<const void*, Packed> packs;
    std::mutex mu;

    // Drops uploads and packs whose address lies in [lo, lo + bytes); the
    // caller holds `mu`.
    void forget(const void* lo, int64_t bytes) {
        const auto* b = static_cast<const uint8_t*>(lo);
        for (auto it = packs.lower_bound(lo); it != packs.end() && static_cast<const uint8_t*>(it->first) < b + bytes;) {
            nb2_device_free(dev, it->second.buf);
            it = packs.erase(it);
        }
        for (auto it = uploads.lower_bound(lo);
             it != uploads.end() && static_cast<const uint8_t*>(it->first) < b + bytes;) {
            it = uploads.erase(it);
        }
    }
};

const void* cached_pack(const void* w, int64_t w_bytes, const std::string& key, int64_t packed_bytes,
                        const std::function<int(void*)>& pack, const std::string& ctx) {
    DeviceState* st = tl_state;
    if (st == nullptr || w == nullptr) {
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(st->mu);
    auto up = st->uploads.find(w);
    if (up == st->uploads.end() || up->second < w_bytes) {
        return nullptr; // not a resident upload (an activation, or a partial write)
    }
    auto it = st->packs.find(w);
    if (it != st->packs.end()) {
        if (it->second.key == key) {
            return it->second.buf;
        }
        nb2_device_free(st->dev, it->second.buf); // the same weight seen with another geometry
        st->packs.erase(it);
    }
    void* buf = nullptr;
    if (nb2_device_malloc(st->dev, packed_bytes, &buf) != NB2_OK || buf == nullptr) {
        return nullptr; // no room: pack per call in the workspace instead
    }
    if (pack(buf) != NB2_OK) {
        nb2_device_free(st->dev, buf);
        fail(ctx, nb2_last_error());
    }
    st->packs[w] = DeviceState::Packed{key, buf};
    return buf;
}

class B200Allocator final : public Allocator {
  public:
    explicit B200Allocator(DeviceState* s) : s_(s) {}
    // Device memory for the arena, resident weights and staged inputs. The
    // reference executor stages every graph input with allocate/release per
    // run (src/executor.cpp:470); released buffers are kept and reused by
    // size, so steady-state runs call no cudaMalloc.
    void* allocate(int64_t bytes) override {
        if (bytes <= 0) {
            return nullptr;
        }
        std::lock_guard<std::mutex> lock(s_->mu);
        auto it = s_->pool.find(bytes);
        if (it != s_->pool.end()) {
            void* p = it->second;
            s_->pool.erase(it);
            return p;
        }
        void* p = nullptr;
        if (nb2_device_malloc(s_->dev, bytes, &p) != NB2_OK) {
            return nullptr;
        }
        s_->sizes[p] = bytes;
        return p;
    }
    void release(void* buffer) override {
        if (buffer == nullptr) {
            return;
        }
        std::lock_guard<std::mutex> lock(s_->mu);
        s_->mirror.erase(buffer);
        auto it = s_->sizes.find(buffer);
        if (it == s_->sizes.end()) {
            return;
        }
        s_->forget(buffer, it->second);
        // queued work may still read the buffer: wait before it is reused
        nb2_device_synchronize(s_->dev);
        s_->pool.emplace(it->second, buffer);
    }

  private:
    DeviceState* s_;
};

class B200Transfer final : public Transfer {
  public:
    explicit B200Transfer(DeviceState* s) : s_(s) {}
    void host_to_device(void* dst, const void* src, int64_t bytes) override {
        if (bytes == 0) {
            return;
        }
        {
            std::lock_guard<std::mutex> lock(s_->mu);
            if (bytes <= 4096) {
                const auto* b = static_cast<const uint8_t*>(src);
                s_->mirror[dst].assign(b, b + bytes);
            } else {
                s_->mirror.erase(dst);
            }
            // new contents: any packed layout of these bytes is stale
            s_->forget(dst, bytes);
            s_->uploads[dst] = bytes;
        }
        if (nb2_memcpy_h2d(s_->dev, dst, src, bytes) != NB2_OK) {
            throw InferenceException(std::string("B200 transfer: ") + nb2_last_error());
        }
    }
    void device_to_host(void* dst, const void* src, int64_t bytes) override {
        if (bytes == 0) {
            return;
        }
        if (nb2_memcpy_d2h(s_->dev, dst, src, bytes) != NB2_OK) {
            throw InferenceException(std::string("B200 transfer: ") + nb2_last_error());
        }
    }

  private:
    DeviceState* s_;
};

class B200Table final : public KernelTable {
  public:
    explicit B200Table(DeviceState* s) : s_(s) {
        rows_ = {{"Conv", HostSafe<Conv>},
                 {"Gemm", HostSafe<Gemm>},
                 {"ConvTranspose", HostSafe<ConvTranspose>},
                 {"MatMul", HostSafe<MatMul>},
                 {"Relu", HostSafe<Unary<NB2_UNARY_RELU>>},
                 {"Sigmoid", HostSafe<Unary<NB2_UNARY_SIGMOID>>},
                 {"Erf", HostSafe<Unary<NB2_UNARY_ERF>>},
                 {"Sqrt", HostSafe<Unary<NB2_UNARY_SQRT>>},
                 {"Neg", HostSafe<Unary<NB2_UNARY_NEG>>},
                 {"Abs", HostSafe<Unary<NB2_UNARY_ABS>>},
                 {"Exp", HostSafe<Unary<NB2_UNARY_EXP>>},
                 {"Tanh", HostSafe<Unary<NB2_UNARY_TANH>>},
                 {"Add", HostSafe<Binary<NB2_BINARY_ADD>>},
                 {"Sub", HostSafe<Binary<NB2_BINARY_SUB>>},
                 {"Mul", HostSafe<Binary<NB2_BINARY_MUL>>},
                 {"Div", HostSafe<Binary<NB2_BINARY_DIV>>},
                 {"Pow", HostSafe<Binary<NB2_BINARY_POW>>},
                 {"MaxPool", HostSafe<MaxPool>},
                 {"AveragePool", HostSafe<AveragePool>},
                 {"GlobalAveragePool", HostSafe<GlobalAveragePool>},
                 {"ReduceMean", HostSafe<ReduceMean>},
                 {"Softmax", HostSafe<Softmax>},
                 {"LayerNormalization", HostSafe<LayerNormalization>},
                 {"Flatten", HostSafe<CopyView>},
                 {"Reshape", HostSafe<CopyView>},
                 {"Squeeze", HostSafe<CopyView>},
                 {"Unsqueeze", HostSafe<CopyView>},
                 {"Identity", HostSafe<CopyView>},
                 {"Transpose", HostSafe<Transpose>},
                 {"Concat", HostSafe<Concat>},
                 {"Split", HostSafe<Split>},
                 {"Slice", HostSafe<Slice>},
                 {"Gather", HostSafe<Gather>},
                 {"TopK", HostSafe<TopK>},
                 {"Resize", HostSafe<Resize>},
                 {"Cast", HostSafe<Cast>}};
    }
    // Returns the row (null when this device has none, as the reference
    // tables do) and binds this GPU to the calling thread for it.
    KernelFn find(const std::string& op_type) const override {
        tl_device = s_->dev;
        tl_mirror = &s_->mirror;
        tl_state = s_;
        auto it = rows_.find(op_type);
        return it == rows_.end() ? nullptr : it->second;
    }

  private:
    DeviceState* s_;
    std::unordered_map<std::string, KernelFn> rows_;
};

class B200Device final : public ::nert::Device {
  public:
    explicit B200Device(int ordinal) : alloc_(&state_), xfer_(&state_), table_(&state_) {
        state_.ordinal = ordinal;
        name_ = "b200:" + std::to_string(ordinal);
        if (nb2_device_open(ordinal, &state_.dev) != NB2_OK) {
            throw InferenceException(std::string("B200 device: ") + nb2_last_error());
        }
    }
    const char* name() const override { return name_.c_str(); }
    Allocator& allocator() override { return alloc_; }
    Transfer& transfer() override { return xfer_; }
    const KernelTable& kernels() const override { return table_; }
    bool is_host() const override { return false; }
    bool supports_arena_offsets() const override { return true; }

  private:
    DeviceState state_;
    B200Allocator alloc_;
    B200Transfer xfer_;
    B200Table table_;
    std::string name_;
};

std::mutex g_mu;
std::array<std::unique_ptr<B200Device>, 64> g_devices;

} // namespace

// The process-lifetime device handle of GPU `ordinal`.
const ::nert::Device& Device(int ordinal) {
    if (ordinal < 0 || ordinal >= 64) {
        throw InferenceException("B200 device: ordinal out of range");
    }
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_devices[ordinal]) {
        g_devices[ordinal] = std::make_unique<B200Device>(ordinal);
    }
    return *g_devices[ordinal];
}

} // namespace b200
} // namespace nert

// C-linkage accessor for FFI callers and tests: the `const nert::Device*` of
// GPU `ordinal` as an opaque pointer, or null (message in nb2_last_error()).
extern "C" const void* nb2_nert_device(int ordinal) {
    try {
        return &nert::b200::Device(ordinal);
    } catch (const std::exception& e) {
        return nullptr;
    }
}
