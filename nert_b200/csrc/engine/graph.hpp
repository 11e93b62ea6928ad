// The B200 engine's graph IR and ONNX reader.
//
// Mirrors the reference IR (include/nert/graph.hpp:21-141: nodes in execution
// order, a value table, embedded constants, declared inputs/outputs, the
// declared opset) closely enough that the same ONNX file means the same graph
// to both. Tensors are float32, int64 or bool, as in the reference.
#pragma once

#include <cstdint>
#include <map>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace nb2 {
namespace eng {

enum class DType : int { F32 = 0, I64 = 1, Bool = 2, Unknown = 3 };

inline int64_t dtype_size(DType t) {
    switch (t) {
    case DType::F32:
        return 4;
    case DType::I64:
        return 8;
    case DType::Bool:
        return 1;
    default:
        return 0;
    }
}

// Load-time problems (malformed file, unsupported graph): reference
// ModelLoadException, include/nert/graph.hpp:25-28.
struct LoadError : std::runtime_error {
    using std::runtime_error::runtime_error;
};
// Run-time problems (bad inputs, shapes): reference InferenceException,
// include/nert/graph.hpp:31-34.
struct RunError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

struct TensorInfo {
    DType dtype = DType::Unknown;
    std::vector<int64_t> dims;
};

struct Constant {
    DType dtype = DType::Unknown;
    std::vector<int64_t> dims;
    std::vector<uint8_t> bytes; // little-endian elements
    int64_t count() const {
        int64_t n = 1;
        for (int64_t d : dims) {
            n *= d;
        }
        return n;
    }
    const float* f32() const { return reinterpret_cast<const float*>(bytes.data()); }
    const int64_t* i64() const { return reinterpret_cast<const int64_t*>(bytes.data()); }
    std::vector<int64_t> as_i64() const; // int64 (or float) constant as a vector
};

struct Attr {
    enum Kind { kNone, kInt, kFloat, kString, kInts, kFloats, kTensor } kind = kNone;
    int64_t i = 0;
    float f = 0.0f;
    std::string s;
    std::vector<int64_t> ints;
    std::vector<float> floats;
    Constant t;
};

struct Node {
    std::string name;
    std::string op;
    std::vector<std::string> inputs;
    std::vector<std::string> outputs;
    std::map<std::string, Attr> attrs;

    bool has(const std::string& k) const { return attrs.count(k) != 0; }
    int64_t geti(const std::string& k, int64_t def) const;
    float getf(const std::string& k, float def) const;
    std::string gets(const std::string& k, const std::string& def) const;
    std::vector<int64_t> getints(const std::string& k) const;
    std::string where() const { return op + " (node '" + name + "')"; }
};

struct Graph {
    std::vector<Node> nodes;
    std::map<std::string, Constant> constants; // initializers
    std::vector<std::pair<std::string, TensorInfo>> inputs;
    std::vector<std::pair<std::string, TensorInfo>> outputs;
    int64_t opset = 0;
};

// Parse ONNX ModelProto bytes (the subset NERT's loader accepts,
// src/model_loader.cpp:2020-2284). Constant nodes become constants.
Graph parse_onnx(const uint8_t* data, size_t size);

// Inference BatchNormalization with constant statistics: folded into the
// producing Conv where it is that output's only use, else kept as a
// three-input node (input, per-channel scale, per-channel shift).
void fold_batchnorm(Graph& g);

// Static shapes for one concrete input shape (reference InferShapes,
// src/shape_inference.cpp:3022). Returns the table for every tensor.
std::map<std::string, TensorInfo> infer_shapes(const Graph& g, const std::map<std::string, std::vector<int64_t>>& input_dims);

int64_t numel(const std::vector<int64_t>& d);

} // namespace eng
} // namespace nb2
