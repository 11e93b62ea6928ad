// Inference BatchNormalization at load time.
//
// The reference has no BatchNormalization row and its loader rejects the op
// (src/model_loader.cpp:1677-1690); its exporters fold BN into the Conv
// before export (tools/provision_resnet18.py:70-71). Graphs exported without
// that fold still load here: with every statistic constant, a BN whose input
// is the only use of a Conv output is folded into that Conv
// (W' = W * a, b' = b * a + beta - mean * a per output channel, with
// a = gamma / sqrt(var + epsilon), computed in double and rounded once);
// any other BN stays a node that the engine runs as y = x * a[c] + s[c]
// (channel_affine) with a and s folded the same way.

#include "graph.hpp"

#include <cmath>
#include <cstring>
#include <iterator>

namespace nb2 {
namespace eng {

namespace {

const Constant* constant_of(const Graph& g, const std::string& name) {
    auto it = g.constants.find(name);
    return it == g.constants.end() ? nullptr : &it->second;
}

std::vector<double> f64(const Constant& c) {
    std::vector<double> v(static_cast<size_t>(c.count()));
    for (size_t i = 0; i < v.size(); ++i) {
        v[i] = c.f32()[i];
    }
    return v;
}

Constant f32_constant(const std::vector<int64_t>& dims, const std::vector<double>& v) {
    Constant c;
    c.dtype = DType::F32;
    c.dims = dims;
    c.bytes.resize(v.size() * 4);
    for (size_t i = 0; i < v.size(); ++i) {
        const float f = static_cast<float>(v[i]);
        std::memcpy(c.bytes.data() + 4 * i, &f, 4);
    }
    return c;
}

} // namespace

void fold_batchnorm(Graph& g) {
    std::map<std::string, int> uses;
    for (const Node& n : g.nodes) {
        for (const auto& in : n.inputs) {
            if (!in.empty()) {
                ++uses[in];
            }
        }
    }
    for (const auto& o : g.outputs) {
        ++uses[o.first];
    }
    bool any = false;
    for (const Node& n : g.nodes) {
        any = any || n.op == "BatchNormalization";
    }
    if (!any) {
        return;
    }
    std::vector<Node> kept;
    kept.reserve(g.nodes.size());
    for (Node& n : g.nodes) {
        if (n.op != "BatchNormalization") {
            kept.push_back(std::move(n));
            continue;
        }
        if (n.inputs.size() != 5 || n.geti("training_mode", 0) != 0) {
            throw LoadError(n.where() + ": only inference BatchNormalization (five inputs) is supported");
        }
        for (size_t o = 1; o < n.outputs.size(); ++o) {
            if (!n.outputs[o].empty() && uses[n.outputs[o]] > 0) {
                throw LoadError(n.where() + ": the running-statistics outputs are not supported");
            }
        }
        const Constant* sc = constant_of(g, n.inputs[1]);
        const Constant* bi = constant_of(g, n.inputs[2]);
        const Constant* mu = constant_of(g, n.inputs[3]);
        const Constant* va = constant_of(g, n.inputs[4]);
        if (!sc || !bi || !mu || !va) {
            throw LoadError(n.where() + ": scale, bias, mean and variance must be constants");
        }
        const int64_t C = sc->count();
        for (const Constant* c : {sc, bi, mu, va}) {
            if (c->dtype != DType::F32 || c->count() != C) {
                throw LoadError(n.where() + ": statistics must be float32 vectors of one length");
            }
        }
        const double eps = n.getf("epsilon", 1e-5f);
        const std::vector<double> gamma = f64(*sc), beta = f64(*bi), mean = f64(*mu), var = f64(*va);
        std::vector<double> a(static_cast<size_t>(C)), s(static_cast<size_t>(C));
        for (int64_t c = 0; c < C; ++c) {
            a[c] = gamma[c] / std::sqrt(var[c] + eps);
            s[c] = beta[c] - mean[c] * a[c];
        }
        // the producing Conv, when this BN is the only use of its output
        Node* conv = nullptr;
        for (auto it = kept.rbegin(); it != kept.rend(); ++it) {
            if (!it->outputs.empty() && it->outputs[0] == n.inputs[0]) {
                conv = &*it;
                break;
            }
        }
        const Constant* w = conv && conv->op == "Conv" && conv->inputs.size() >= 2 ? constant_of(g, conv->inputs[1])
                                                                                 : nullptr;
        const Constant* cb = conv && conv->inputs.size() > 2 && !conv->inputs[2].empty()
                                 ? constant_of(g, conv->inputs[2])
                                 : nullptr;
        const bool has_bias = conv && conv->inputs.size() > 2 && !conv->inputs[2].empty();
        if (w && uses[n.inputs[0]] == 1 && w->dtype == DType::F32 && !w->dims.empty() && w->dims[0] == C &&
            (!has_bias || (cb && cb->dtype == DType::F32 && cb->count() == C))) {
            const int64_t per = w->count() / C;
            std::vector<double> wv = f64(*w), bv(static_cast<size_t>(C), 0.0);
            if (cb) {
                bv = f64(*cb);
            }
            for (int64_t c = 0; c < C; ++c) {
                for (int64_t i = 0; i < per; ++i) {
                    wv[c * per + i] *= a[c];
                }
                bv[c] = bv[c] * a[c] + s[c];
            }
            const std::string wname = conv->name + "/bn_folded.weight", bname = conv->name + "/bn_folded.bias";
            g.constants[wname] = f32_constant(w->dims, wv);
            g.constants[bname] = f32_constant({C}, bv);
            conv->inputs.resize(3);
            conv->inputs[1] = wname;
            conv->inputs[2] = bname;
            conv->outputs[0] = n.outputs[0];
            continue;
        }
        // stays a node: the engine applies the folded per-channel affine
        const std::string aname = n.name + "/bn.scale", sname = n.name + "/bn.shift";
        g.constants[aname] = f32_constant({C}, a);
        g.constants[sname] = f32_constant({C}, s);
        n.inputs = {n.inputs[0], aname, sname};
        n.outputs.resize(1);
        kept.push_back(std::move(n));
    }
    g.nodes = std::move(kept);
    // drop the constants nothing reads any more (the unfolded weights and
    // statistics), so they are not uploaded
    std::map<std::string, int> read;
    for (const Node& n : g.nodes) {
        for (const auto& in : n.inputs) {
            read[in] = 1;
        }
    }
    for (const auto& o : g.outputs) {
        read[o.first] = 1;
    }
    for (auto it = g.constants.begin(); it != g.constants.end();) {
        it = read.count(it->first) ? std::next(it) : g.constants.erase(it);
    }
}

} // namespace eng
} // namespace nb2
