// Static shape inference for the B200 engine (the ONNX rules NERT applies in
// src/shape_inference.cpp, for the operators this engine executes). Constant
// int64/float operands (Reshape shape, Split sizes, Slice bounds, TopK K,
// Resize scales/sizes, Unsqueeze/Squeeze axes) must be initializers or
// Constant nodes, as in the reference's static context.

#include "graph.hpp"

#include <algorithm>
#include <cmath>
#include <set>

namespace nb2 {
namespace eng {

namespace {

[[noreturn]] void fail(const Node& n, const std::string& msg) { throw LoadError(n.where() + ": " + msg); }

int64_t norm_axis(const Node& n, int64_t axis, int64_t rank) {
    if (axis < -rank || axis >= rank) {
        fail(n, "axis out of range");
    }
    return axis < 0 ? axis + rank : axis;
}

std::vector<int64_t> broadcast(const Node& n, const std::vector<int64_t>& a, const std::vector<int64_t>& b) {
    const size_t r = std::max(a.size(), b.size());
    std::vector<int64_t> out(r);
    for (size_t i = 0; i < r; ++i) {
        const int64_t x = i + a.size() >= r ? a[i + a.size() - r] : 1;
        const int64_t y = i + b.size() >= r ? b[i + b.size() - r] : 1;
        if (x != y && x != 1 && y != 1) {
            fail(n, "operand shapes do not broadcast");
        }
        out[i] = x == 1 ? y : x;
    }
    return out;
}

struct Ctx {
    const Graph& g;
    std::map<std::string, TensorInfo>& t;
    const TensorInfo& in(const Node& n, size_t i) const {
        if (i >= n.inputs.size() || n.inputs[i].empty()) {
            fail(n, "missing input " + std::to_string(i));
        }
        auto it = t.find(n.inputs[i]);
        if (it == t.end()) {
            fail(n, "input '" + n.inputs[i] + "' has no shape");
        }
        return it->second;
    }
    bool present(const Node& n, size_t i) const { return i < n.inputs.size() && !n.inputs[i].empty(); }
    const Constant& constant(const Node& n, size_t i) const {
        auto it = g.constants.find(n.inputs[i]);
        if (it == g.constants.end()) {
            fail(n, "operand '" + n.inputs[i] + "' must be a constant");
        }
        return it->second;
    }
};

void window(const Node& n, const std::vector<int64_t>& in_sp, const std::vector<int64_t>& k,
            std::vector<int64_t>& out, bool ceil_mode) {
    const size_t r = in_sp.size();
    std::vector<int64_t> s = n.getints("strides"), d = n.getints("dilations"), pads = n.getints("pads");
    if (s.empty()) {
        s.assign(r, 1);
    }
    if (d.empty()) {
        d.assign(r, 1);
    }
    const std::string ap = n.gets("auto_pad", "NOTSET");
    out.assign(r, 0);
    for (size_t i = 0; i < r; ++i) {
        if (ap == "SAME_UPPER" || ap == "SAME_LOWER") {
            out[i] = (in_sp[i] + s[i] - 1) / s[i];
            continue;
        }
        int64_t pb = 0, pe = 0;
        if (ap != "VALID" && !pads.empty()) {
            if (pads.size() != 2 * r) {
                fail(n, "pads must have two entries per spatial dimension");
            }
            pb = pads[i];
            pe = pads[r + i];
        }
        const int64_t numer = in_sp[i] + pb + pe - (d[i] * (k[i] - 1) + 1);
        if (numer < 0) {
            fail(n, "window is larger than the padded input");
        }
        out[i] = (ceil_mode ? (numer + s[i] - 1) / s[i] : numer / s[i]) + 1;
    }
}

std::vector<TensorInfo> infer_node(Ctx& c, const Node& n, int64_t opset) {
    const std::string& op = n.op;
    static const std::set<std::string> unary = {"Relu", "Sigmoid", "Erf", "Sqrt", "Neg", "Abs", "Exp", "Tanh",
                                                "Identity", "Softmax", "Floor"};
    if (unary.count(op)) {
        return {c.in(n, 0)};
    }
    if (op == "Add" || op == "Sub" || op == "Mul" || op == "Div" || op == "Pow") {
        const TensorInfo& a = c.in(n, 0);
        const TensorInfo& b = c.in(n, 1);
        return {TensorInfo{a.dtype, broadcast(n, a.dims, b.dims)}};
    }
    if (op == "Conv") {
        const TensorInfo& x = c.in(n, 0);
        const TensorInfo& w = c.in(n, 1);
        if (x.dims.size() < 3 || x.dims.size() > 4 || w.dims.size() != x.dims.size()) {
            fail(n, "the B200 Conv row takes rank-3 or rank-4 NCHW inputs with a matching weight rank");
        }
        std::vector<int64_t> in_sp(x.dims.begin() + 2, x.dims.end()), k(w.dims.begin() + 2, w.dims.end()), o;
        window(n, in_sp, k, o, false);
        std::vector<int64_t> out = {x.dims[0], w.dims[0]};
        out.insert(out.end(), o.begin(), o.end());
        return {TensorInfo{DType::F32, out}};
    }
    if (op == "ConvTranspose") {
        // src/kernels/conv_transpose.cpp: s*(in-1) + output_padding + d*(k-1) + 1 - pads
        const TensorInfo& x = c.in(n, 0);
        const TensorInfo& w = c.in(n, 1);
        if (x.dims.size() != 4 || w.dims.size() != 4) {
            fail(n, "input and weight must be rank 4 (NCHW)");
        }
        if (n.has("output_shape")) {
            fail(n, "output_shape is not supported");
        }
        const std::string ap = n.gets("auto_pad", "NOTSET");
        if (ap != "NOTSET" && ap != "VALID") {
            fail(n, "auto_pad " + ap + " is not supported");
        }
        auto list = [&](const char* k, int64_t def, size_t len) {
            std::vector<int64_t> v = n.getints(k);
            if (v.empty() || (std::string(k) == "pads" && ap == "VALID")) {
                v.assign(len, def);
            }
            if (v.size() != len) {
                fail(n, std::string(k) + " has the wrong length");
            }
            return v;
        };
        const auto s = list("strides", 1, 2), d = list("dilations", 1, 2), op2 = list("output_padding", 0, 2),
                   p = list("pads", 0, 4);
        const int64_t g = n.geti("group", 1);
        if (g <= 0 || x.dims[1] % g != 0 || w.dims[0] != x.dims[1]) {
            fail(n, "weight channels do not match the input and group");
        }
        std::vector<int64_t> out = {x.dims[0], w.dims[1] * g};
        for (int i = 0; i < 2; ++i) {
            const int64_t o = s[i] * (x.dims[2 + i] - 1) + op2[i] + d[i] * (w.dims[2 + i] - 1) + 1 - p[i] - p[2 + i];
            if (o <= 0) {
                fail(n, "computes a non-positive output dimension");
            }
            out.push_back(o);
        }
        return {TensorInfo{DType::F32, out}};
    }
    if (op == "MaxPool" || op == "AveragePool") {
        const TensorInfo& x = c.in(n, 0);
        if (x.dims.size() != 4) {
            fail(n, "input must be rank 4 (NCHW)");
        }
        std::vector<int64_t> in_sp(x.dims.begin() + 2, x.dims.end()), o;
        window(n, in_sp, n.getints("kernel_shape"), o, n.geti("ceil_mode", 0) != 0);
        return {TensorInfo{DType::F32, {x.dims[0], x.dims[1], o[0], o[1]}}};
    }
    if (op == "BatchNormalization") {
        // after fold_batchnorm: (input, per-channel scale, per-channel shift)
        const TensorInfo& x = c.in(n, 0);
        if (x.dims.size() < 2) {
            fail(n, "input must have batch and channel axes");
        }
        return {TensorInfo{DType::F32, x.dims}};
    }
    if (op == "GlobalAveragePool") {
        const TensorInfo& x = c.in(n, 0);
        std::vector<int64_t> out = {x.dims[0], x.dims[1]};
        out.insert(out.end(), x.dims.size() - 2, 1);
        return {TensorInfo{DType::F32, out}};
    }
    if (op == "ReduceMean") {
        const TensorInfo& x = c.in(n, 0);
        std::vector<int64_t> axes = opset >= 18 ? (c.present(n, 1) ? c.constant(n, 1).as_i64() : std::vector<int64_t>{})
                                                : n.getints("axes");
        const bool keep = n.geti("keepdims", 1) != 0;
        const int64_t r = static_cast<int64_t>(x.dims.size());
        std::set<int64_t> ax;
        if (axes.empty()) {
            for (int64_t i = 0; i < r; ++i) {
                ax.insert(i);
            }
        }
        for (int64_t a : axes) {
            ax.insert(norm_axis(n, a, r));
        }
        std::vector<int64_t> out;
        for (int64_t i = 0; i < r; ++i) {
            if (ax.count(i)) {
                if (keep) {
                    out.push_back(1);
                }
            } else {
                out.push_back(x.dims[i]);
            }
        }
        return {TensorInfo{DType::F32, out}};
    }
    if (op == "Flatten") {
        const TensorInfo& x = c.in(n, 0);
        const int64_t r = static_cast<int64_t>(x.dims.size());
        int64_t axis = n.geti("axis", 1);
        if (axis < 0) {
            axis += r;
        }
        if (axis < 0 || axis > r) {
            fail(n, "axis out of range");
        }
        int64_t a = 1, b = 1;
        for (int64_t i = 0; i < r; ++i) {
            (i < axis ? a : b) *= x.dims[i];
        }
        return {TensorInfo{x.dtype, {a, b}}};
    }
    if (op == "Reshape") {
        const TensorInfo& x = c.in(n, 0);
        std::vector<int64_t> shape = c.constant(n, 1).as_i64();
        const bool allowzero = n.geti("allowzero", 0) != 0;
        int64_t known = 1, infer = -1;
        for (size_t i = 0; i < shape.size(); ++i) {
            if (shape[i] == 0 && !allowzero) {
                if (i >= x.dims.size()) {
                    fail(n, "0 in shape refers past the input rank");
                }
                shape[i] = x.dims[i];
            }
            if (shape[i] == -1) {
                if (infer >= 0) {
                    fail(n, "more than one -1 in shape");
                }
                infer = static_cast<int64_t>(i);
            } else {
                known *= shape[i];
            }
        }
        const int64_t total = numel(x.dims);
        if (infer >= 0) {
            if (known == 0 || total % known != 0) {
                fail(n, "cannot infer the -1 dimension");
            }
            shape[infer] = total / known;
        }
        if (numel(shape) != total) {
            fail(n, "shape does not preserve the element count");
        }
        return {TensorInfo{x.dtype, shape}};
    }
    if (op == "Gemm") {
        const TensorInfo& a = c.in(n, 0);
        const TensorInfo& b = c.in(n, 1);
        if (a.dims.size() != 2 || b.dims.size() != 2) {
            fail(n, "A and B must be rank-2");
        }
        const int64_t m = n.geti("transA", 0) ? a.dims[1] : a.dims[0];
        const int64_t k = n.geti("transA", 0) ? a.dims[0] : a.dims[1];
        const int64_t kb = n.geti("transB", 0) ? b.dims[1] : b.dims[0];
        const int64_t nn = n.geti("transB", 0) ? b.dims[0] : b.dims[1];
        if (k != kb) {
            fail(n, "contraction dimension mismatch");
        }
        return {TensorInfo{DType::F32, {m, nn}}};
    }
    if (op == "MatMul") {
        std::vector<int64_t> a = c.in(n, 0).dims, b = c.in(n, 1).dims;
        const bool a1 = a.size() == 1, b1 = b.size() == 1;
        if (a1) {
            a.insert(a.begin(), 1);
        }
        if (b1) {
            b.push_back(1);
        }
        if (a[a.size() - 1] != b[b.size() - 2]) {
            fail(n, "contraction dimension mismatch");
        }
        std::vector<int64_t> ab(a.begin(), a.end() - 2), bb(b.begin(), b.end() - 2);
        std::vector<int64_t> out = broadcast(n, ab, bb);
        if (!a1) {
            out.push_back(a[a.size() - 2]);
        }
        if (!b1) {
            out.push_back(b.back());
        }
        return {TensorInfo{DType::F32, out}};
    }
    if (op == "LayerNormalization") {
        const TensorInfo& x = c.in(n, 0);
        std::vector<TensorInfo> outs = {x};
        const int64_t r = static_cast<int64_t>(x.dims.size());
        const int64_t axis = norm_axis(n, n.geti("axis", -1), r);
        std::vector<int64_t> stat = x.dims;
        for (int64_t i = axis; i < r; ++i) {
            stat[i] = 1;
        }
        for (size_t i = 1; i < n.outputs.size(); ++i) {
            outs.push_back(TensorInfo{DType::F32, stat});
        }
        return outs;
    }
    if (op == "Transpose") {
        const TensorInfo& x = c.in(n, 0);
        std::vector<int64_t> perm = n.getints("perm");
        const size_t r = x.dims.size();
        if (perm.empty()) {
            for (size_t i = 0; i < r; ++i) {
                perm.push_back(static_cast<int64_t>(r - 1 - i));
            }
        }
        if (perm.size() != r) {
            fail(n, "perm must list every axis");
        }
        std::vector<int64_t> out(r);
        for (size_t i = 0; i < r; ++i) {
            out[i] = x.dims[norm_axis(n, perm[i], static_cast<int64_t>(r))];
        }
        return {TensorInfo{x.dtype, out}};
    }
    if (op == "Concat") {
        const TensorInfo& x0 = c.in(n, 0);
        const int64_t r = static_cast<int64_t>(x0.dims.size());
        const int64_t axis = norm_axis(n, n.geti("axis", 0), r);
        std::vector<int64_t> out = x0.dims;
        out[axis] = 0;
        for (size_t i = 0; i < n.inputs.size(); ++i) {
            const TensorInfo& xi = c.in(n, i);
            if (static_cast<int64_t>(xi.dims.size()) != r) {
                fail(n, "inputs must share a rank");
            }
            for (int64_t d = 0; d < r; ++d) {
                if (d != axis && xi.dims[d] != x0.dims[d]) {
                    fail(n, "inputs differ off the concat axis");
                }
            }
            out[axis] += xi.dims[axis];
        }
        return {TensorInfo{x0.dtype, out}};
    }
    if (op == "Split") {
        const TensorInfo& x = c.in(n, 0);
        const int64_t r = static_cast<int64_t>(x.dims.size());
        const int64_t axis = norm_axis(n, n.geti("axis", 0), r);
        std::vector<int64_t> sizes;
        if (opset >= 13 && c.present(n, 1)) {
            sizes = c.constant(n, 1).as_i64();
        } else if (opset < 13) {
            sizes = n.getints("split");
        }
        const int64_t parts = static_cast<int64_t>(n.outputs.size());
        if (sizes.empty()) {
            const int64_t dim = x.dims[axis];
            const int64_t each = (dim + parts - 1) / parts;
            for (int64_t i = 0; i < parts; ++i) {
                sizes.push_back(std::min(each, dim - i * each));
            }
        }
        if (static_cast<int64_t>(sizes.size()) != parts) {
            fail(n, "split sizes must match the output count");
        }
        int64_t tot = 0;
        std::vector<TensorInfo> outs;
        for (int64_t s : sizes) {
            TensorInfo t = x;
            t.dims[axis] = s;
            tot += s;
            outs.push_back(t);
        }
        if (tot != x.dims[axis]) {
            fail(n, "split sizes must sum to the axis length");
        }
        return outs;
    }
    if (op == "Slice") {
        const TensorInfo& x = c.in(n, 0);
        const int64_t r = static_cast<int64_t>(x.dims.size());
        const std::vector<int64_t> starts = c.constant(n, 1).as_i64();
        const std::vector<int64_t> ends = c.constant(n, 2).as_i64();
        std::vector<int64_t> axes, steps;
        if (c.present(n, 3)) {
            axes = c.constant(n, 3).as_i64();
        } else {
            for (size_t i = 0; i < starts.size(); ++i) {
                axes.push_back(static_cast<int64_t>(i));
            }
        }
        if (c.present(n, 4)) {
            steps = c.constant(n, 4).as_i64();
        } else {
            steps.assign(starts.size(), 1);
        }
        std::vector<int64_t> out = x.dims;
        for (size_t i = 0; i < starts.size(); ++i) {
            const int64_t a = norm_axis(n, axes[i], r);
            const int64_t dim = x.dims[a];
            const int64_t st = steps[i];
            if (st == 0) {
                fail(n, "step must be non-zero");
            }
            int64_t s = starts[i] < 0 ? starts[i] + dim : starts[i];
            int64_t e = ends[i] < 0 ? ends[i] + dim : ends[i];
            if (st > 0) {
                s = std::clamp<int64_t>(s, 0, dim);
                e = std::clamp<int64_t>(e, 0, dim);
                out[a] = e > s ? (e - s + st - 1) / st : 0;
            } else {
                s = std::clamp<int64_t>(s, 0, dim - 1);
                e = std::clamp<int64_t>(e, -1, dim - 1);
                out[a] = s > e ? (s - e + (-st) - 1) / (-st) : 0;
            }
        }
        return {TensorInfo{x.dtype, out}};
    }
    if (op == "Gather") {
        const TensorInfo& x = c.in(n, 0);
        const TensorInfo& idx = c.in(n, 1);
        const int64_t r = static_cast<int64_t>(x.dims.size());
        const int64_t axis = norm_axis(n, n.geti("axis", 0), r);
        std::vector<int64_t> out(x.dims.begin(), x.dims.begin() + axis);
        out.insert(out.end(), idx.dims.begin(), idx.dims.end());
        out.insert(out.end(), x.dims.begin() + axis + 1, x.dims.end());
        return {TensorInfo{x.dtype, out}};
    }
    if (op == "TopK") {
        const TensorInfo& x = c.in(n, 0);
        const int64_t k = c.constant(n, 1).as_i64().at(0);
        const int64_t r = static_cast<int64_t>(x.dims.size());
        const int64_t axis = norm_axis(n, n.geti("axis", -1), r);
        if (k < 0 || k > x.dims[axis]) {
            fail(n, "K is out of range");
        }
        std::vector<int64_t> out = x.dims;
        out[axis] = k;
        return {TensorInfo{x.dtype, out}, TensorInfo{DType::I64, out}};
    }
    if (op == "Resize") {
        const TensorInfo& x = c.in(n, 0);
        const size_t r = x.dims.size();
        const bool has_scales = c.present(n, 2) && c.constant(n, 2).count() > 0;
        const bool has_sizes = c.present(n, 3);
        if (has_sizes) {
            std::vector<int64_t> sizes = c.constant(n, 3).as_i64();
            if (sizes.size() != r) {
                fail(n, "sizes rank must match the input rank");
            }
            return {TensorInfo{x.dtype, sizes}};
        }
        if (!has_scales) {
            fail(n, "Resize requires a scales input");
        }
        const Constant& sc = c.constant(n, 2);
        if (sc.dtype != DType::F32 || static_cast<size_t>(sc.count()) != r) {
            fail(n, "scales must be float32 with one entry per axis");
        }
        std::vector<int64_t> out(r);
        for (size_t i = 0; i < r; ++i) {
            out[i] = static_cast<int64_t>(std::floor(static_cast<double>(x.dims[i]) * static_cast<double>(sc.f32()[i])));
        }
        return {TensorInfo{x.dtype, out}};
    }
    if (op == "Unsqueeze" || op == "Squeeze") {
        const TensorInfo& x = c.in(n, 0);
        std::vector<int64_t> axes = opset >= 13 ? (c.present(n, 1) ? c.constant(n, 1).as_i64() : std::vector<int64_t>{})
                                                : n.getints("axes");
        std::vector<int64_t> out;
        if (op == "Unsqueeze") {
            const int64_t r = static_cast<int64_t>(x.dims.size() + axes.size());
            std::set<int64_t> ax;
            for (int64_t a : axes) {
                ax.insert(norm_axis(n, a, r));
            }
            size_t j = 0;
            for (int64_t i = 0; i < r; ++i) {
                out.push_back(ax.count(i) ? 1 : x.dims[j++]);
            }
        } else {
            const int64_t r = static_cast<int64_t>(x.dims.size());
            std::set<int64_t> ax;
            for (int64_t a : axes) {
                ax.insert(norm_axis(n, a, r));
            }
            for (int64_t i = 0; i < r; ++i) {
                if (axes.empty() ? x.dims[i] == 1 : ax.count(i) != 0) {
                    continue;
                }
                out.push_back(x.dims[i]);
            }
        }
        return {TensorInfo{x.dtype, out}};
    }
    if (op == "Cast") {
        const TensorInfo& x = c.in(n, 0);
        const int64_t to = n.geti("to", 1);
        return {TensorInfo{to == 7 ? DType::I64 : to == 9 ? DType::Bool : DType::F32, x.dims}};
    }
    fail(n, "op '" + op + "' has no row on the B200 device");
}

} // namespace

std::map<std::string, TensorInfo> infer_shapes(const Graph& g,
                                               const std::map<std::string, std::vector<int64_t>>& input_dims) {
    std::map<std::string, TensorInfo> t;
    for (const auto& kv : g.constants) {
        t[kv.first] = TensorInfo{kv.second.dtype, kv.second.dims};
    }
    for (const auto& in : g.inputs) {
        auto it = input_dims.find(in.first);
        if (it == input_dims.end()) {
            throw LoadError("no shape given for graph input '" + in.first + "'");
        }
        for (int64_t d : it->second) {
            if (d <= 0) {
                throw LoadError("graph input '" + in.first + "' has a non-positive dimension");
            }
        }
        t[in.first] = TensorInfo{in.second.dtype == DType::Unknown ? DType::F32 : in.second.dtype, it->second};
    }
    Ctx c{g, t};
    for (const Node& n : g.nodes) {
        std::vector<TensorInfo> outs = infer_node(c, n, g.opset);
        if (outs.size() < n.outputs.size()) {
            fail(n, "produces fewer outputs than declared");
        }
        for (size_t i = 0; i < n.outputs.size(); ++i) {
            if (!n.outputs[i].empty()) {
                t[n.outputs[i]] = outs[i];
            }
        }
    }
    for (const auto& out : g.outputs) {
        if (t.count(out.first) == 0) {
            throw LoadError("graph output '" + out.first + "' is never produced");
        }
    }
    return t;
}

} // namespace eng
} // namespace nb2
