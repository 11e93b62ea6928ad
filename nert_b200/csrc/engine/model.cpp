// B200 engine Model: fusion peephole, arena planning, weight residency and
// packing, and CUDA-graph execution (see model.hpp).

#include "model.hpp"

#include "../igemm.cuh"
#include "../ops.cuh"
#include "../ops_move.cuh"
#include "../ops_norm.cuh"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <list>
#include <set>

namespace nb2 {
namespace eng {

namespace {

constexpr int64_t kAlign = 256;

int64_t align_up(int64_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

// One executable unit after fusion: a node, or a Conv/Gemm/MatMul that
// absorbed its epilogue consumers.
struct ExecNode {
    const Node* node = nullptr;
    std::string op;
    std::vector<std::string> ins;  // every tensor read (for liveness)
    std::vector<std::string> outs; // tensors produced
    std::string out;               // the fused group's visible output (outs[0] for plain nodes)
    std::string residual;          // fused residual Add operand
    std::string bias;              // fused MatMul bias (Add of a constant [N])
    int act = kActNone;
    float act_a = 0.f, act_b = 0.f, act_c = 0.f; // GELU constants
    float alpha = 1.f;                           // fused scale (Div / Mul by a power of two)
    int pos = 0;
    bool alias = false; // output is a view of input 0
    int group = 1;      // nodes in the group
    int pool_k = 0, chain = 0; // SPPF: window and cascade length
    // Attention: scale applied to Q K^T (0 none, 1 Mul, 2 Div) and whether the
    // head-merge Transpose + Reshape were absorbed ([B, T, H*D] output)
    int attn_mode = 0;
    float attn_scale = 1.f;
    bool attn_merged = false;
    // a MatMul whose (Reshape +) Transpose consumer was absorbed: the
    // contraction writes its result straight into the transposed layout
    std::vector<int64_t> view, perm;
};

// Output map of a contraction with z slices of R x C results viewed as
// `view` (a split of [Z, R, C] into at most two axes each) and permuted by
// `perm`: each view axis gets its stride in the permuted, contiguous
// tensor. False when the view does not split Z, R and C that way or a
// two-axis column split has an inner extent that is not a multiple of 16.
bool make_out_map(const std::vector<int64_t>& view, const std::vector<int64_t>& perm, int64_t Z, int64_t R,
                  int64_t C, OutMap* m) {
    const size_t r = view.size();
    if (perm.size() != r || r == 0) {
        return false;
    }
    std::vector<int64_t> tstride(r, 1), vstride(r, 0);
    for (size_t j = r - 1; j > 0; --j) {
        tstride[j - 1] = tstride[j] * view[static_cast<size_t>(perm[j])];
    }
    std::vector<bool> seen(r, false);
    for (size_t j = 0; j < r; ++j) {
        if (perm[j] < 0 || perm[j] >= static_cast<int64_t>(r) || seen[static_cast<size_t>(perm[j])]) {
            return false;
        }
        seen[static_cast<size_t>(perm[j])] = true;
        vstride[static_cast<size_t>(perm[j])] = tstride[j];
    }
    // consume view axes (skipping size-1 axes) whose product is `want`,
    // at most two of them: (outer, inner) -> radix and strides
    size_t i = 0;
    auto take = [&](int64_t want, int64_t& x2, int64_t& s1, int64_t& s2, int64_t round) -> bool {
        std::vector<size_t> ax;
        int64_t prod = 1;
        while (i < r && prod < want) {
            if (view[i] != 1) {
                ax.push_back(i);
                prod *= view[i];
            }
            ++i;
        }
        while (i < r && view[i] == 1 && want == 1) {
            ++i;
        }
        if (prod != want || ax.size() > 2) {
            return false;
        }
        if (ax.empty()) {
            x2 = 1, s1 = 0, s2 = 0;
        } else if (ax.size() == 1) {
            x2 = (want + round - 1) / round * round, s1 = 0, s2 = vstride[ax[0]];
        } else {
            x2 = view[ax[1]], s1 = vstride[ax[0]], s2 = vstride[ax[1]];
        }
        return true;
    };
    OutMap o;
    o.on = true;
    if (!take(Z, o.z2, o.zs1, o.zs2, 1) || !take(R, o.r2, o.rs1, o.rs2, 1) || !take(C, o.c2, o.cs1, o.cs2, 16)) {
        return false;
    }
    while (i < r && view[i] == 1) {
        ++i;
    }
    if (i != r || o.c2 % 16 != 0) {
        return false;
    }
    *m = o;
    return true;
}

// Z, R, C of a MatMul as the contraction kernel runs it: a B without batch
// (rank 2, or leading dimensions of 1) folds every leading dimension of A
// into the rows, else the batch is z.
void matmul_zrc(const std::vector<int64_t>& out, const std::vector<int64_t>& b, int64_t& Z, int64_t& R, int64_t& C) {
    C = out.back();
    Z = 1;
    R = 1;
    const size_t r = out.size();
    int64_t b_count = 1;
    for (size_t i = 0; i + 2 < b.size(); ++i) {
        b_count *= b[i];
    }
    if (b_count == 1) {
        for (size_t i = 0; i + 1 < r; ++i) {
            R *= out[i];
        }
    } else {
        for (size_t i = 0; i + 2 < r; ++i) {
            Z *= out[i];
        }
        R = r >= 2 ? out[r - 2] : 1;
    }
}

bool is_alias_op(const std::string& op) {
    return op == "Flatten" || op == "Reshape" || op == "Squeeze" || op == "Unsqueeze" || op == "Identity";
}

std::vector<ExecNode> fuse(const Graph& g, const std::map<std::string, TensorInfo>& shapes, bool enable,
                           int64_t& fused_groups, bool attention_on) {
    std::map<std::string, std::vector<int>> consumers;
    for (int i = 0; i < static_cast<int>(g.nodes.size()); ++i) {
        for (const auto& in : g.nodes[i].inputs) {
            if (!in.empty()) {
                consumers[in].push_back(i);
            }
        }
    }
    std::set<std::string> outputs;
    for (const auto& o : g.outputs) {
        outputs.insert(o.first);
    }
    std::vector<bool> absorbed(g.nodes.size(), false);
    // the single, not yet fused consumer of `t` (t not a graph output), else -1
    auto single = [&](const std::string& t) -> int {
        if (outputs.count(t)) {
            return -1;
        }
        auto it = consumers.find(t);
        if (it == consumers.end() || it->second.size() != 1 || absorbed[it->second[0]]) {
            return -1;
        }
        return it->second[0];
    };
    std::vector<ExecNode> list;
    fused_groups = 0;
    // SPPF: a Concat over channels of [t, m1, ..., mL] where m_l is a k x k,
    // stride-1, pad k/2 MaxPool of m_{l-1} (m0 = t) read only by the next pool
    // and the Concat becomes one pass over t (sppf_nchw); the pools are
    // absorbed into the Concat's node
    std::map<int, std::pair<std::string, std::pair<int64_t, int64_t>>> sppf; // concat -> (t, (k, L))
    if (enable) {
        std::map<std::string, int> producer;
        for (int i = 0; i < static_cast<int>(g.nodes.size()); ++i) {
            for (const auto& o : g.nodes[i].outputs) {
                producer[o] = i;
            }
        }
        auto same_pool = [&](const Node& p, int64_t& k) {
            const std::vector<int64_t> ks = p.getints("kernel_shape"), st = p.getints("strides"),
                                       dl = p.getints("dilations"), pd = p.getints("pads");
            if (p.op != "MaxPool" || p.outputs.size() != 1 || ks.size() != 2 || ks[0] != ks[1] || ks[0] % 2 == 0 ||
                p.gets("auto_pad", "NOTSET") != "NOTSET") {
                return false;
            }
            k = ks[0];
            const int64_t r = k / 2;
            const bool s1 = st.empty() || (st.size() == 2 && st[0] == 1 && st[1] == 1);
            const bool d1 = dl.empty() || (dl.size() == 2 && dl[0] == 1 && dl[1] == 1);
            const bool pr = pd.size() == 4 && pd[0] == r && pd[1] == r && pd[2] == r && pd[3] == r;
            return s1 && d1 && (pr || (r == 0 && pd.empty()));
        };
        for (int i = 0; i < static_cast<int>(g.nodes.size()); ++i) {
            const Node& cat = g.nodes[i];
            if (cat.op != "Concat" || cat.inputs.size() < 2 || cat.outputs.size() != 1) {
                continue;
            }
            const std::string& t = cat.inputs[0];
            const auto td = shapes.find(t);
            const int64_t axis = cat.geti("axis", 0);
            if (td == shapes.end() || td->second.dims.size() != 4 || td->second.dtype != DType::F32 ||
                (axis != 1 && axis != -3) || td->second.dims[2] * td->second.dims[3] > kSppfMaxPlane) {
                continue;
            }
            int64_t k = 0;
            bool ok = true;
            std::vector<int> pools;
            for (size_t l = 1; l < cat.inputs.size() && ok; ++l) {
                const std::string& m = cat.inputs[l];
                auto pi = producer.find(m);
                int64_t kl = 0;
                ok = pi != producer.end() && same_pool(g.nodes[pi->second], kl) && (l == 1 || kl == k) &&
                     g.nodes[pi->second].inputs[0] == cat.inputs[l - 1] && !outputs.count(m);
                if (!ok) {
                    break;
                }
                k = kl;
                // read by the Concat once and, before the last, by the next pool
                const auto& cs = consumers[m];
                const bool last = l + 1 == cat.inputs.size();
                ok = last ? (cs.size() == 1 && cs[0] == i)
                          : (cs.size() == 2 && ((cs[0] == i && producer[cat.inputs[l + 1]] == cs[1]) ||
                                                (cs[1] == i && producer[cat.inputs[l + 1]] == cs[0])));
                pools.push_back(pi->second);
            }
            if (!ok) {
                continue;
            }
            for (int p : pools) {
                absorbed[p] = true;
            }
            sppf[i] = {t, {k, static_cast<int64_t>(pools.size())}};
        }
    }
    // Attention: MatMul(q, k) [-> Div / Mul by a float scalar] -> Softmax over
    // the last axis -> MatMul(., v) [-> Transpose(0, 2, 1, 3) -> Reshape to
    // [B, T, H*D]] with q, v [B, H, T, 64], k [B, H, 64, T], T <= 208 and every
    // intermediate read only by the next node: one fused step (ops_attn.cu)
    struct AttnMatch {
        std::string q, k, v, out;
        int mode;
        float scale;
        bool merged;
    };
    std::map<int, AttnMatch> attn; // index of the chain's last node -> match
    if (enable && attention_on) {
        std::map<std::string, int> producer;
        for (int i = 0; i < static_cast<int>(g.nodes.size()); ++i) {
            for (const auto& o : g.nodes[i].outputs) {
                producer[o] = i;
            }
        }
        auto only_reader = [&](const std::string& t) -> int {
            if (outputs.count(t)) {
                return -1;
            }
            auto it = consumers.find(t);
            return it == consumers.end() || it->second.size() != 1 ? -1 : it->second[0];
        };
        auto dims_of = [&](const std::string& t) -> const std::vector<int64_t>* {
            auto it = shapes.find(t);
            return it == shapes.end() || it->second.dtype != DType::F32 ? nullptr : &it->second.dims;
        };
        for (int i = 0; i < static_cast<int>(g.nodes.size()); ++i) {
            const Node& sm = g.nodes[i];
            if (sm.op != "Softmax" || sm.inputs.empty() || sm.outputs.size() != 1 || absorbed[i]) {
                continue;
            }
            const std::vector<int64_t>* sd = dims_of(sm.inputs[0]);
            if (!sd || sd->size() != 4) {
                continue;
            }
            const int64_t axis = sm.geti("axis", g.opset >= 13 ? -1 : 1);
            if (axis != -1 && axis != 3) {
                continue;
            }
            // producer chain upstream of the Softmax
            auto pi = producer.find(sm.inputs[0]);
            if (pi == producer.end() || only_reader(sm.inputs[0]) != i) {
                continue;
            }
            int scale_node = -1, mode = 0;
            float scale = 1.f;
            int qk = pi->second;
            if (g.nodes[qk].op == "Div" || g.nodes[qk].op == "Mul") {
                const Node& dv = g.nodes[qk];
                auto c = g.constants.find(dv.inputs.size() == 2 ? dv.inputs[1] : std::string());
                if (c == g.constants.end() || c->second.dtype != DType::F32 || c->second.count() != 1) {
                    continue;
                }
                std::memcpy(&scale, c->second.bytes.data(), 4);
                mode = dv.op == "Mul" ? 1 : 2;
                if (mode == 2 && scale == 0.f) {
                    continue;
                }
                scale_node = qk;
                auto pq = producer.find(dv.inputs[0]);
                if (pq == producer.end() || only_reader(dv.inputs[0]) != qk) {
                    continue;
                }
                qk = pq->second;
            }
            const Node& mq = g.nodes[qk];
            if (mq.op != "MatMul" || absorbed[qk] || g.constants.count(mq.inputs[0]) ||
                g.constants.count(mq.inputs[1])) {
                continue;
            }
            const int av = only_reader(sm.outputs[0]);
            if (av < 0 || g.nodes[av].op != "MatMul" || g.nodes[av].inputs[0] != sm.outputs[0] ||
                g.constants.count(g.nodes[av].inputs[1])) {
                continue;
            }
            const std::vector<int64_t>*qd = dims_of(mq.inputs[0]), *kd = dims_of(mq.inputs[1]),
                                 *vd = dims_of(g.nodes[av].inputs[1]), *od = dims_of(g.nodes[av].outputs[0]);
            if (!qd || !kd || !vd || !od || qd->size() != 4) {
                continue;
            }
            const int64_t B = (*qd)[0], H = (*qd)[1], T = (*qd)[2], D = (*qd)[3];
            if (D != 64 || T < 1 || T > kAttnMaxT || *kd != std::vector<int64_t>{B, H, D, T} ||
                *vd != std::vector<int64_t>{B, H, T, D} || *od != std::vector<int64_t>{B, H, T, D}) {
                continue;
            }
            AttnMatch m{mq.inputs[0], mq.inputs[1], g.nodes[av].inputs[1], g.nodes[av].outputs[0], mode, scale, false};
            int last = av;
            // the head merge: Transpose(0, 2, 1, 3) -> Reshape [B, T, H*D]
            const int tr = only_reader(m.out);
            if (tr >= 0 && g.nodes[tr].op == "Transpose" &&
                g.nodes[tr].getints("perm") == std::vector<int64_t>{0, 2, 1, 3}) {
                const int rs = only_reader(g.nodes[tr].outputs[0]);
                const std::vector<int64_t>* rd = rs >= 0 ? dims_of(g.nodes[rs].outputs[0]) : nullptr;
                if (rs >= 0 && g.nodes[rs].op == "Reshape" && g.nodes[rs].inputs[0] == g.nodes[tr].outputs[0] && rd &&
                    *rd == std::vector<int64_t>{B, T, H * D}) {
                    absorbed[tr] = absorbed[rs] = true;
                    m.out = g.nodes[rs].outputs[0];
                    m.merged = true;
                    last = rs;
                }
            }
            absorbed[qk] = absorbed[i] = absorbed[av] = true;
            if (scale_node >= 0) {
                absorbed[scale_node] = true;
            }
            attn[last] = m;
        }
    }
    // the chain's output is produced where its last node was
    for (auto& kv : attn) {
        absorbed[kv.first] = false;
    }
    for (int i = 0; i < static_cast<int>(g.nodes.size()); ++i) {
        if (absorbed[i]) {
            continue;
        }
        if (attn.count(i)) {
            const AttnMatch& m = attn[i];
            ExecNode e;
            e.node = &g.nodes[i];
            e.op = "Attention";
            e.pos = i;
            e.ins = {m.q, m.k, m.v};
            e.outs = {m.out};
            e.out = m.out;
            e.attn_mode = m.mode;
            e.attn_scale = m.scale;
            e.attn_merged = m.merged;
            e.group = 3 + (m.mode != 0 ? 1 : 0) + (m.merged ? 2 : 0);
            ++fused_groups;
            list.push_back(std::move(e));
            continue;
        }
        if (sppf.count(i)) {
            const Node& cat = g.nodes[i];
            ExecNode e;
            e.node = &cat;
            e.op = "SPPF";
            e.pos = i;
            e.ins = {sppf[i].first};
            e.outs = cat.outputs;
            e.out = cat.outputs[0];
            e.pool_k = static_cast<int>(sppf[i].second.first);
            e.chain = static_cast<int>(sppf[i].second.second);
            e.group = e.chain + 1;
            ++fused_groups;
            list.push_back(std::move(e));
            continue;
        }
        const Node& n = g.nodes[i];
        ExecNode e;
        e.node = &n;
        e.op = n.op;
        e.pos = i;
        for (const auto& in : n.inputs) {
            if (!in.empty()) {
                e.ins.push_back(in);
            }
        }
        e.outs = n.outputs;
        e.out = n.outputs.empty() ? "" : n.outputs[0];
        e.alias = is_alias_op(n.op);
        const bool mm_const_b = n.op == "MatMul" && g.constants.count(n.inputs[1]) &&
                                g.constants.at(n.inputs[1]).dims.size() == 2 &&
                                shapes.at(n.inputs[0]).dims.size() >= 2;
        const bool mm = n.op == "MatMul" && shapes.at(n.inputs[0]).dims.size() >= 2 &&
                        shapes.at(n.inputs[1]).dims.size() >= 2;
        // a float scalar constant
        auto scalar_of = [&](const std::string& t, float& v) {
            auto c = g.constants.find(t);
            if (c == g.constants.end() || c->second.dtype != DType::F32 || c->second.count() != 1) {
                return false;
            }
            std::memcpy(&v, c->second.bytes.data(), 4);
            return true;
        };
        if (enable && (n.op == "Conv" || n.op == "Gemm" || mm)) {
            std::string cur = e.out;
            if (mm && !mm_const_b) {
                // QK^T / sqrt(d): a Div (or Mul) by a power of two is exact as
                // the epilogue's alpha
                const int j = single(cur);
                float c = 0.f;
                if (j >= 0 && (g.nodes[j].op == "Div" || g.nodes[j].op == "Mul") && g.nodes[j].inputs[0] == cur &&
                    scalar_of(g.nodes[j].inputs[1], c) && c != 0.f) {
                    int ex = 0;
                    const float m = std::frexp(c, &ex);
                    if (m == 0.5f || m == -0.5f) {
                        e.alpha = g.nodes[j].op == "Div" ? 1.0f / c : c;
                        absorbed[j] = true;
                        e.pos = j;
                        e.group++;
                        cur = g.nodes[j].outputs[0];
                    }
                }
            }
            if (mm_const_b) {
                const int j = single(cur);
                if (j >= 0 && g.nodes[j].op == "Add") {
                    const Node& a = g.nodes[j];
                    const std::string other = a.inputs[0] == cur ? a.inputs[1] : a.inputs[0];
                    const int64_t N = g.constants.at(n.inputs[1]).dims[1];
                    auto c = g.constants.find(other);
                    if (c != g.constants.end() && c->second.dtype == DType::F32 && c->second.count() == N &&
                        shapes.at(a.outputs[0]).dims == shapes.at(cur).dims) {
                        e.bias = other;
                        e.ins.push_back(other);
                        absorbed[j] = true;
                        e.pos = j;
                        e.group++;
                        cur = a.outputs[0];
                    }
                }
            }
            int j = single(cur);
            if (j >= 0 && g.nodes[j].op == "Add") {
                const Node& a = g.nodes[j];
                const std::string other = a.inputs[0] == cur ? a.inputs[1] : a.inputs[0];
                if (other != cur && shapes.at(other).dims == shapes.at(cur).dims &&
                    shapes.at(other).dtype == DType::F32) {
                    e.residual = other;
                    e.ins.push_back(other);
                    absorbed[j] = true;
                    e.pos = j;
                    e.group++;
                    cur = a.outputs[0];
                    j = single(cur);
                }
            }
            if (j >= 0 && g.nodes[j].op == "Relu") {
                e.act = kActRelu;
                absorbed[j] = true;
                e.pos = j;
                e.group++;
                cur = g.nodes[j].outputs[0];
            } else if (!outputs.count(cur) && consumers.count(cur) && consumers[cur].size() == 2 &&
                       (g.nodes[consumers[cur][0]].op == "Div" || g.nodes[consumers[cur][1]].op == "Div")) {
                // GELU, erf form: Div(cur, a) -> Erf -> Add(., b) -> Mul(cur, .) -> Mul(., c)
                const int c0 = consumers[cur][0], c1 = consumers[cur][1];
                const int dv = g.nodes[c0].op == "Div" ? c0 : c1;
                const int m1 = dv == c0 ? c1 : c0;
                float a = 0.f, b = 0.f, c = 0.f;
                const Node& div = g.nodes[dv];
                const int ef = div.inputs[0] == cur && scalar_of(div.inputs[1], a) && a != 0.f ? single(div.outputs[0])
                                                                                              : -1;
                const int ad = ef >= 0 && g.nodes[ef].op == "Erf" ? single(g.nodes[ef].outputs[0]) : -1;
                int mu = -1;
                if (ad >= 0 && g.nodes[ad].op == "Add") {
                    const Node& add = g.nodes[ad];
                    const std::string eo = g.nodes[ef].outputs[0];
                    const std::string other = add.inputs[0] == eo ? add.inputs[1] : add.inputs[0];
                    if (scalar_of(other, b)) {
                        mu = single(add.outputs[0]);
                    }
                }
                int m2 = -1;
                if (mu == m1 && !absorbed[m1] && g.nodes[m1].op == "Mul") {
                    const Node& mul = g.nodes[m1];
                    const std::string ao = g.nodes[ad].outputs[0];
                    const bool pair = (mul.inputs[0] == cur && mul.inputs[1] == ao) ||
                                      (mul.inputs[1] == cur && mul.inputs[0] == ao);
                    m2 = pair ? single(mul.outputs[0]) : -1;
                }
                if (m2 >= 0 && g.nodes[m2].op == "Mul") {
                    const Node& h = g.nodes[m2];
                    const std::string mo = g.nodes[m1].outputs[0];
                    const std::string other = h.inputs[0] == mo ? h.inputs[1] : h.inputs[0];
                    if (scalar_of(other, c) && !absorbed[dv] && !absorbed[ef] && !absorbed[ad] && !absorbed[m2]) {
                        e.act = kActGeluErf;
                        e.act_a = a;
                        e.act_b = b;
                        e.act_c = c;
                        absorbed[dv] = absorbed[ef] = absorbed[ad] = absorbed[m1] = absorbed[m2] = true;
                        e.pos = std::max({dv, ef, ad, m1, m2});
                        e.group += 5;
                        cur = h.outputs[0];
                    }
                }
            } else if (!outputs.count(cur) && consumers.count(cur) && consumers[cur].size() == 2) {
                // SiLU: Sigmoid(cur) feeding only Mul(cur, sigmoid)
                const int c0 = consumers[cur][0], c1 = consumers[cur][1];
                const int s = g.nodes[c0].op == "Sigmoid" ? c0 : g.nodes[c1].op == "Sigmoid" ? c1 : -1;
                const int m = s == c0 ? c1 : c0;
                if (s >= 0 && g.nodes[m].op == "Mul" && !absorbed[s] && !absorbed[m]) {
                    const std::string sig = g.nodes[s].outputs[0];
                    const Node& mul = g.nodes[m];
                    const bool pair = (mul.inputs[0] == cur && mul.inputs[1] == sig) ||
                                      (mul.inputs[1] == cur && mul.inputs[0] == sig);
                    if (pair && single(sig) == m && m > s) {
                        e.act = kActSilu;
                        absorbed[s] = absorbed[m] = true;
                        e.pos = m;
                        e.group += 2;
                        cur = mul.outputs[0];
                    }
                }
            }
            if (mm && e.residual.empty()) {
                // a head split / merge: MatMul -> [Reshape ->] Transpose,
                // written straight into the transposed layout
                const int r0 = single(cur);
                int rs = -1, tr = r0;
                std::vector<int64_t> view = shapes.at(cur).dims;
                if (r0 >= 0 && g.nodes[r0].op == "Reshape") {
                    rs = r0;
                    view = shapes.at(g.nodes[r0].outputs[0]).dims;
                    tr = single(g.nodes[r0].outputs[0]);
                }
                if (tr >= 0 && g.nodes[tr].op == "Transpose") {
                    std::vector<int64_t> perm = g.nodes[tr].getints("perm");
                    if (perm.empty()) {
                        for (int64_t a = static_cast<int64_t>(view.size()) - 1; a >= 0; --a) {
                            perm.push_back(a);
                        }
                    }
                    int64_t Z = 1, R = 1, C = 1;
                    matmul_zrc(shapes.at(cur).dims, shapes.at(n.inputs[1]).dims, Z, R, C);
                    OutMap om;
                    if (make_out_map(view, perm, Z, R, C, &om)) {
                        e.view = view;
                        e.perm = perm;
                        if (rs >= 0) {
                            absorbed[rs] = true;
                            e.group++;
                        }
                        absorbed[tr] = true;
                        e.group++;
                        e.pos = tr;
                        cur = g.nodes[tr].outputs[0];
                    }
                }
            }
            if (e.group > 1) {
                ++fused_groups;
                e.out = cur;
                e.outs = {cur};
            }
        }
        list.push_back(std::move(e));
    }
    std::stable_sort(list.begin(), list.end(), [](const ExecNode& a, const ExecNode& b) { return a.pos < b.pos; });
    return list;
}

ConvGeom conv_geom(const Node& n, const TensorInfo& x, const TensorInfo& w, const TensorInfo& y) {
    const bool one_d = x.dims.size() == 3;
    ConvGeom g{};
    g.N = x.dims[0];
    g.C = x.dims[1];
    g.H = one_d ? 1 : x.dims[2];
    g.W = one_d ? x.dims[2] : x.dims[3];
    g.M = w.dims[0];
    g.KH = one_d ? 1 : w.dims[2];
    g.KW = one_d ? w.dims[2] : w.dims[3];
    g.OH = one_d ? 1 : y.dims[2];
    g.OW = one_d ? y.dims[2] : y.dims[3];
    const size_t r = x.dims.size() - 2;
    std::vector<int64_t> s = n.getints("strides"), d = n.getints("dilations"), pads = n.getints("pads");
    if (s.empty()) {
        s.assign(r, 1);
    }
    if (d.empty()) {
        d.assign(r, 1);
    }
    std::vector<int64_t> pb(r, 0);
    const std::string ap = n.gets("auto_pad", "NOTSET");
    std::vector<int64_t> in_sp(x.dims.begin() + 2, x.dims.end()), k(w.dims.begin() + 2, w.dims.end());
    for (size_t i = 0; i < r; ++i) {
        if (ap == "SAME_UPPER" || ap == "SAME_LOWER") {
            const int64_t out = (in_sp[i] + s[i] - 1) / s[i];
            const int64_t total = std::max<int64_t>(0, (out - 1) * s[i] + d[i] * (k[i] - 1) + 1 - in_sp[i]);
            pb[i] = ap == "SAME_UPPER" ? total / 2 : total - total / 2;
        } else if (ap != "VALID" && !pads.empty()) {
            pb[i] = pads[i];
        }
    }
    g.sh = one_d ? 1 : s[0];
    g.sw = one_d ? s[0] : s[1];
    g.dh = one_d ? 1 : d[0];
    g.dw = one_d ? d[0] : d[1];
    g.ph = one_d ? 0 : pb[0];
    g.pw = one_d ? pb[0] : pb[1];
    g.group = n.geti("group", 1);
    // the end padding that the output extent implies (the last window's end)
    g.pb = (g.OH - 1) * g.sh + g.dh * (g.KH - 1) + 1 - g.H - g.ph;
    g.pr = (g.OW - 1) * g.sw + g.dw * (g.KW - 1) + 1 - g.W - g.pw;
    if (g.group <= 0 || g.C % g.group != 0 || g.M % g.group != 0 || w.dims[1] != g.C / g.group) {
        throw LoadError(n.where() + ": weight channel dimension does not match input/group");
    }
    return g;
}

} // namespace

Model::Model(const uint8_t* onnx, size_t size, const std::map<std::string, std::vector<int64_t>>& input_dims,
             int ordinal, int flags)
    : dev_(nb2::device(ordinal)), g_(parse_onnx(onnx, size)) {
    dev_->make_current();
    try {
        build(input_dims, flags);
    } catch (...) {
        if (exec_) {
            cudaGraphExecDestroy(exec_);
            exec_ = nullptr;
        }
        cudaStreamSynchronize(dev_->stream);
        release_pipeline();
        for (void* p : allocations_) {
            cudaFree(p);
        }
        allocations_.clear();
        throw;
    }
}

void Model::release_pipeline() {
    if (copy_stream_) {
        cudaStreamSynchronize(copy_stream_);
        cudaStreamDestroy(copy_stream_);
        copy_stream_ = nullptr;
    }
    for (int k = 0; k < 2; ++k) {
        if (staged_[k]) {
            cudaEventDestroy(staged_[k]);
            staged_[k] = nullptr;
        }
        if (freed_[k]) {
            cudaEventDestroy(freed_[k]);
            freed_[k] = nullptr;
        }
    }
}

Model::~Model() {
    cudaSetDevice(dev_->ordinal);
    if (exec_) {
        cudaGraphExecDestroy(exec_);
    }
    cudaStreamSynchronize(dev_->stream);
    release_pipeline();
    for (void* p : allocations_) {
        cudaFree(p);
    }
}

namespace {

// Host-only half of Model construction: shapes, fusion, liveness and the
// arena plan. Needs no GPU (nb2_graph_analyze exposes it for tests).
struct PlanResult {
    std::map<std::string, TensorInfo> shapes;
    std::vector<ExecNode> ex;
    std::map<std::string, std::string> root;
    std::map<std::string, int64_t> offset;
    std::map<std::string, int> last_use;
    int64_t arena = 0;
    int64_t fused_groups = 0;
    std::set<std::string> nhwc; // activations kept channels-last
};

// Channels-last trunk: a 4-D fp32 activation is stored NHWC when every node
// touching it can work in that layout and at least one Conv produces a tensor
// of its layout class. Conv reads either layout (TMA im2col for NHWC, C % 32 ==
// 0) and writes either; MaxPool, unary and same-shape binary rows are layout
// preserving (one class); GlobalAveragePool reads either layout and writes
// [N, C, 1, 1], which is the same in both. Graph inputs and outputs, aliased
// views and every other row stay NCHW, so the boundary layout is the
// reference's.
std::set<std::string> assign_nhwc(const Graph& g, const std::map<std::string, TensorInfo>& shapes,
                                  const std::vector<ExecNode>& ex);


PlanResult plan_graph(const Graph& g_, const std::map<std::string, std::vector<int64_t>>& input_dims, int flags) {
    PlanResult pr;
    pr.shapes = infer_shapes(g_, input_dims);
    const auto& shapes_ = pr.shapes;
    std::vector<ExecNode>& ex = pr.ex;
    ex = fuse(g_, shapes_, (flags & kNoFusion) == 0, pr.fused_groups, (flags & kNoAttention) == 0);

    // ---- liveness over the fused list (aliases share their root's buffer)
    std::map<std::string, std::string> root;
    auto root_of = [&](const std::string& t) -> std::string {
        auto it = root.find(t);
        return it == root.end() ? t : it->second;
    };
    std::set<std::string> graph_inputs, graph_outputs;
    for (const auto& in : g_.inputs) {
        graph_inputs.insert(in.first);
    }
    for (const auto& o : g_.outputs) {
        graph_outputs.insert(o.first);
    }
    const int n_exec = static_cast<int>(ex.size());
    std::map<std::string, int> last_use;
    for (int i = 0; i < n_exec; ++i) {
        if (ex[i].alias) {
            root[ex[i].out] = root_of(ex[i].ins[0]);
        }
        for (const auto& in : ex[i].ins) {
            last_use[root_of(in)] = i;
        }
    }
    for (const auto& o : graph_outputs) {
        last_use[root_of(o)] = n_exec + 1;
    }

    // ---- arena plan: first fit over live blocks, outputs placed before the
    // node's dying inputs are released (an output never aliases its inputs).
    std::map<std::string, int64_t> offset;
    std::list<std::pair<int64_t, std::pair<int64_t, std::string>>> live; // offset -> (size, root)
    int64_t arena = 0;
    auto place = [&](const std::string& t, int64_t bytes) {
        bytes = align_up(std::max<int64_t>(bytes, 1));
        int64_t at = 0;
        auto it = live.begin();
        for (; it != live.end(); ++it) {
            if (it->first - at >= bytes) {
                break;
            }
            at = std::max(at, it->first + it->second.first);
        }
        live.insert(it, {at, {bytes, t}});
        offset[t] = at;
        arena = std::max(arena, at + bytes);
    };
    for (int i = 0; i < n_exec; ++i) {
        if (!ex[i].alias) {
            for (const auto& o : ex[i].outs) {
                if (o.empty() || graph_inputs.count(o) || g_.constants.count(o)) {
                    continue;
                }
                const TensorInfo& ti = shapes_.at(o);
                place(o, numel(ti.dims) * dtype_size(ti.dtype));
            }
        }
        for (auto it = live.begin(); it != live.end();) {
            const std::string& r = it->second.second;
            auto lu = last_use.find(r);
            const int until = lu == last_use.end() ? i : lu->second;
            if (until <= i) {
                it = live.erase(it);
            } else {
                ++it;
            }
        }
    }
    pr.root = root;
    pr.offset = offset;
    pr.last_use = last_use;
    pr.arena = arena;
    if ((flags & kNchwOnly) == 0) {
        pr.nhwc = assign_nhwc(g_, shapes_, ex);
    }
    return pr;
}

std::set<std::string> assign_nhwc(const Graph& g, const std::map<std::string, TensorInfo>& shapes,
                                  const std::vector<ExecNode>& ex) {
    std::set<std::string> io;
    for (const auto& in : g.inputs) {
        io.insert(in.first);
    }
    for (const auto& o : g.outputs) {
        io.insert(o.first);
    }
    auto candidate = [&](const std::string& t) {
        if (t.empty() || io.count(t) || g.constants.count(t)) {
            return false;
        }
        auto it = shapes.find(t);
        return it != shapes.end() && it->second.dtype == DType::F32 && it->second.dims.size() == 4;
    };
    // union-find over tensor names: members of a class share one layout
    std::map<std::string, std::string> parent;
    std::function<std::string(const std::string&)> find = [&](const std::string& t) -> std::string {
        auto it = parent.find(t);
        if (it == parent.end() || it->second == t) {
            return t;
        }
        const std::string r = find(it->second);
        parent[t] = r;
        return r;
    };
    auto unite = [&](const std::string& a, const std::string& b) {
        const std::string ra = find(a), rb = find(b);
        if (ra != rb) {
            parent[ra] = rb;
        }
    };
    std::set<std::string> bad, conv_out, touched;
    for (const auto& e : ex) {
        const Node& n = *e.node;
        for (const auto& t : e.ins) {
            touched.insert(t);
        }
        for (const auto& t : e.outs) {
            touched.insert(t);
        }
        if (e.op == "Conv") {
            const auto& x = shapes.at(n.inputs[0]);
            if (x.dims.size() == 4) {
                const ConvGeom cg = conv_geom(n, x, shapes.at(n.inputs[1]), shapes.at(n.outputs[0]));
                if (!cg.nhwc_in_place().nhwc_input_ok()) {
                    bad.insert(n.inputs[0]);
                }
                if (direct_conv_ok(cg)) { // the CUDA-core path reads and writes NCHW
                    bad.insert(n.inputs[0]);
                    bad.insert(e.out);
                }
            } else {
                bad.insert(n.inputs[0]);
            }
            for (size_t i = 1; i < n.inputs.size(); ++i) {
                bad.insert(n.inputs[i]);
            }
            if (!e.bias.empty()) {
                bad.insert(e.bias);
            }
            if (!e.residual.empty()) {
                unite(e.residual, e.out);
            }
            conv_out.insert(e.out);
        } else if (e.op == "MaxPool" && n.outputs.size() == 1) {
            unite(n.inputs[0], n.outputs[0]);
        } else if (e.op == "Concat" || e.op == "Split" ||
                   (e.op == "Resize" && shapes.at(n.inputs[0]).dims.size() == 4)) {
            // the channels-last forms cut and move along the same logical
            // axes; every 4-D tensor of the node shares one layout
            // (Split's sizes and Resize's roi / scales / sizes are
            // operands, not data)
            const std::string& first = n.inputs[0];
            if (e.op == "Concat") {
                for (const auto& t : n.inputs) {
                    unite(t, first);
                }
            }
            for (const auto& t : n.outputs) {
                unite(t, first);
            }
        } else if (e.op == "GlobalAveragePool") {
            bad.insert(n.outputs[0]);
        } else if (e.op == "Relu" || e.op == "Sigmoid" || e.op == "Erf" || e.op == "Sqrt" || e.op == "Neg" ||
                   e.op == "Abs" || e.op == "Exp" || e.op == "Tanh") {
            unite(n.inputs[0], n.outputs[0]);
        } else if ((e.op == "Add" || e.op == "Sub" || e.op == "Mul" || e.op == "Div" || e.op == "Pow") &&
                   shapes.at(n.inputs[0]).dims == shapes.at(n.outputs[0]).dims &&
                   shapes.at(n.inputs[1]).dims == shapes.at(n.outputs[0]).dims) {
            unite(n.inputs[0], n.outputs[0]);
            unite(n.inputs[1], n.outputs[0]);
        } else {
            for (const auto& t : e.ins) {
                bad.insert(t);
            }
            for (const auto& t : e.outs) {
                bad.insert(t);
            }
        }
    }
    std::set<std::string> bad_class, has_conv;
    for (const auto& t : touched) {
        if (bad.count(t) || !candidate(t)) {
            bad_class.insert(find(t));
        }
        if (conv_out.count(t)) {
            has_conv.insert(find(t));
        }
    }
    std::set<std::string> out;
    for (const auto& t : touched) {
        const std::string r = find(t);
        if (!bad_class.count(r) && has_conv.count(r)) {
            out.insert(t);
        }
    }
    return out;
}

} // namespace

void Model::build(const std::map<std::string, std::vector<int64_t>>& input_dims, int flags) {
    use_graph_ = (flags & kNoGraph) == 0;
    PlanResult pr = plan_graph(g_, input_dims, flags);
    shapes_ = pr.shapes;
    fused_groups_ = pr.fused_groups;
    const std::vector<ExecNode>& ex = pr.ex;
    const std::map<std::string, std::string>& root = pr.root;
    auto root_of = [&](const std::string& t) -> std::string {
        auto it = root.find(t);
        return it == root.end() ? t : it->second;
    };
    const std::map<std::string, int64_t>& offset = pr.offset;
    const std::set<std::string>& nhwc = pr.nhwc;
    nhwc_tensors_ = static_cast<int64_t>(nhwc.size());
    arena_bytes_ = pr.arena;

    // ---- device buffers: arena, graph inputs, constants, packed weights
    auto dmalloc = [&](int64_t bytes) -> uint8_t* {
        if (bytes <= 0) {
            return nullptr;
        }
        void* p = nullptr;
        if (cudaMalloc(&p, static_cast<size_t>(bytes)) != cudaSuccess) {
            cudaGetLastError();
            throw RunError("executor: could not allocate " + std::to_string(bytes) + " bytes on the device");
        }
        allocations_.push_back(p);
        return static_cast<uint8_t*>(p);
    };
    uint8_t* arena_ptr = dmalloc(arena_bytes_);
    std::map<std::string, void*> ptr;
    for (const auto& in : g_.inputs) {
        const TensorInfo& ti = shapes_.at(in.first);
        IOInfo io{in.first, ti.dtype, ti.dims, nullptr, numel(ti.dims) * dtype_size(ti.dtype)};
        io.dev = dmalloc(align_up(io.bytes));
        ptr[in.first] = io.dev;
        inputs_.push_back(io);
    }
    // constants read by kernels as data (not shape operands, not packed weights)
    std::set<std::string> packed_conv, packed_gemm, raw_needed;
    for (const auto& e : ex) {
        const Node& n = *e.node;
        auto data_in = [&](size_t i) {
            if (i < n.inputs.size() && g_.constants.count(n.inputs[i])) {
                raw_needed.insert(n.inputs[i]);
            }
        };
        if (e.op == "Conv") {
            if (g_.constants.count(n.inputs[1])) {
                packed_conv.insert(n.inputs[1]);
            } else {
                data_in(1);
            }
            data_in(0);
            data_in(2);
        } else if (e.op == "Gemm" || e.op == "MatMul") {
            data_in(0);
            if (g_.constants.count(n.inputs[1])) {
                packed_gemm.insert(n.inputs[1]);
            }
            data_in(2);
            data_in(1); // raw copy also kept (simple; weights are small next to 180 GB)
        } else if (e.op == "Reshape" || e.op == "Squeeze" || e.op == "Unsqueeze" || e.op == "Split" ||
                   e.op == "Slice" || e.op == "TopK" || e.op == "Resize" || e.op == "ReduceMean") {
            data_in(0);
        } else {
            for (size_t i = 0; i < n.inputs.size(); ++i) {
                data_in(i);
            }
        }
        if (!e.residual.empty()) {
            data_in(0);
            if (g_.constants.count(e.residual)) {
                raw_needed.insert(e.residual);
            }
        }
        if (!e.bias.empty()) {
            raw_needed.insert(e.bias);
        }
    }
    int64_t wbytes = 0;
    std::map<std::string, int64_t> woff;
    for (const auto& name : raw_needed) {
        woff[name] = wbytes;
        wbytes += align_up(static_cast<int64_t>(g_.constants.at(name).bytes.size()));
    }
    uint8_t* wptr = dmalloc(wbytes);
    for (const auto& name : raw_needed) {
        const Constant& c = g_.constants.at(name);
        if (!c.bytes.empty()) {
            // Ordered on the device stream: a plain cudaMemcpy from pageable
            // memory may return before its DMA lands, and the packing kernels
            // below run on the (non-blocking) device stream.
            check_cuda(cudaMemcpyAsync(wptr + woff[name], c.bytes.data(), c.bytes.size(), cudaMemcpyHostToDevice,
                                       dev_->stream),
                       "cudaMemcpyAsync(weights)");
        }
        ptr[name] = wptr + woff[name];
    }
    weight_bytes_ = wbytes;
    for (const auto& kv : offset) {
        ptr[kv.first] = arena_ptr + kv.second;
    }
    auto P = [&](const std::string& t) -> void* {
        if (t.empty()) {
            return nullptr;
        }
        auto it = ptr.find(root_of(t));
        if (it == ptr.end()) {
            throw RunError("executor: tensor '" + t + "' has no device buffer");
        }
        return it->second;
    };
    auto F = [&](const std::string& t) { return static_cast<float*>(P(t)); };
    auto dims = [&](const std::string& t) -> const std::vector<int64_t>& { return shapes_.at(t).dims; };

    // ---- steps
    int64_t scratch_need = 0;
    int64_t xform_need = 0; // shared buffer for NCHW -> NHWC copies of Conv inputs
    std::vector<std::function<void(void*)>> pending; // steps needing the scratch pointer
    for (const auto& e : ex) {
        const Node& n = *e.node;
        if (e.alias) {
            continue;
        }
        Step st;
        st.label = n.op + (e.group > 1 ? "+fused" : "") + ":" + n.name;
        if (e.op == "Conv") {
            ConvGeom geom = conv_geom(n, shapes_.at(n.inputs[0]), shapes_.at(n.inputs[1]), shapes_.at(n.outputs[0]));
            if (nhwc.count(n.inputs[0]) > 0) {
                geom = geom.nhwc_in_place();
            }
            geom.out_nhwc = nhwc.count(e.out) > 0;
            if (geom.in_nhwc || geom.out_nhwc) {
                st.label += geom.in_nhwc ? (geom.out_nhwc ? "[nhwc]" : "[nhwc>nchw]") : "[nchw>nhwc]";
            }
            // An NCHW input outside the channels-last trunk (packed weights
            // only) is converted to NHWC in front of the contraction: up to 16
            // channels padded to 4, 8 or 16 (each tap one to four 16-byte
            // loads); a spatial filter over more channels padded to a multiple
            // of 32 and read through TMA im2col.
            const bool direct = direct_conv_ok(geom);
            const bool convertible = (flags & kNchwOnly) == 0 && !geom.in_nhwc &&
                                     packed_conv.count(n.inputs[1]) > 0 && geom.group == 1 && !direct;
            if (convertible) {
                geom = nchw_input_layout(geom);
            }
            Epilogue ep;
            ep.bias = n.inputs.size() > 2 ? F(n.inputs[2]) : nullptr;
            ep.res = e.residual.empty() ? nullptr : F(e.residual);
            ep.act = e.act;
            ep.act_a = e.act_a;
            ep.act_b = e.act_b;
            ep.act_c = e.act_c;
            const float* x = F(n.inputs[0]);
            float* y = F(e.out);
            if (direct) {
                // narrow output: the CUDA-core direct kernel on the raw weights
                const float* w = nullptr;
                if (packed_conv.count(n.inputs[1])) {
                    const Constant& wc = g_.constants.at(n.inputs[1]);
                    uint8_t* wd = dmalloc(align_up(static_cast<int64_t>(wc.bytes.size())));
                    check_cuda(cudaMemcpyAsync(wd, wc.bytes.data(), wc.bytes.size(), cudaMemcpyHostToDevice,
                                               dev_->stream),
                               "cudaMemcpyAsync(weight)");
                    check_cuda(cudaStreamSynchronize(dev_->stream), "weight upload sync");
                    weight_bytes_ += static_cast<int64_t>(wc.bytes.size());
                    w = reinterpret_cast<const float*>(wd);
                } else {
                    w = F(n.inputs[1]);
                }
                nb2_device* dev = dev_;
                st.label += "[direct]";
                st.launches = 1;
                st.run = [=] { conv_direct(dev, geom, x, w, y, ep); };
                launches_ += st.launches;
                steps_.push_back(std::move(st));
                continue;
            }
            const int64_t pbytes = static_cast<int64_t>(conv_packed_bytes(geom));
            // the contraction kernel, plus a reduce launch when it splits K
            const int conv_k = contraction_launches(dev_, geom.N * geom.OH * geom.OW, geom.Mg(), geom.K(), geom.group);
            st.launches = conv_k;
            if (packed_conv.count(n.inputs[1])) {
                // pack once at load from a temporary upload of the raw weight
                uint8_t* packed = dmalloc(align_up(pbytes));
                const Constant& wc = g_.constants.at(n.inputs[1]);
                void* tmp = nullptr;
                check_cuda(cudaMalloc(&tmp, wc.bytes.size()), "cudaMalloc(weight staging)");
                check_cuda(cudaMemcpyAsync(tmp, wc.bytes.data(), wc.bytes.size(), cudaMemcpyHostToDevice,
                                           dev_->stream),
                           "cudaMemcpyAsync(weight)");
                conv_pack(dev_, geom, static_cast<const float*>(tmp), packed);
                check_cuda(cudaStreamSynchronize(dev_->stream), "pack sync");
                cudaFree(tmp);
                weight_bytes_ += pbytes;
                nb2_device* dev = dev_;
                if (geom.converts_input()) {
                    // the converted input lives in the shared transform buffer
                    const int64_t cp = geom.Cin();
                    xform_need = std::max(xform_need, geom.N * cp * geom.H * geom.W * 4);
                    void** xp = &xform_;
                    st.label += geom.cvec == 4 ? "[c4]" : (geom.cvec ? "[c" + std::to_string(geom.cvec) + "]"
                                                                     : "[t>nhwc]");
                    st.launches = conv_k + 1;
                    st.run = [=] {
                        nchw_to_nhwc_pad(dev, x, static_cast<float*>(*xp), geom.N, geom.C, geom.H, geom.W, cp);
                        conv_run(dev, geom, static_cast<const float*>(*xp), packed, y, ep);
                    };
                } else {
                    st.run = [=] { conv_run(dev, geom, x, packed, y, ep); };
                }
            } else {
                const float* w = F(n.inputs[1]);
                scratch_need = std::max(scratch_need, pbytes);
                nb2_device* dev = dev_;
                void** sp = &scratch_;
                st.launches = conv_k + (geom.tap_major() ? 1 : 2);
                st.run = [=] {
                    conv_pack(dev, geom, w, *sp);
                    conv_run(dev, geom, x, *sp, y, ep);
                };
            }
        } else if (e.op == "Gemm" || e.op == "MatMul") {
            GemmGeom gg{};
            Epilogue ep;
            const auto& ad = dims(n.inputs[0]);
            const auto& bd = dims(n.inputs[1]);
            if (e.op == "Gemm") {
                gg.trans_a = static_cast<int>(n.geti("transA", 0));
                gg.trans_b = static_cast<int>(n.geti("transB", 0));
                gg.M = gg.trans_a ? ad[1] : ad[0];
                gg.K = gg.trans_a ? ad[0] : ad[1];
                gg.N = gg.trans_b ? bd[0] : bd[1];
                gg.lda = ad[1];
                gg.ldb = bd[1];
                gg.ldc = gg.N;
                ep.alpha = n.getf("alpha", 1.0f);
                const float beta = n.getf("beta", 1.0f);
                if (n.inputs.size() > 2 && !n.inputs[2].empty()) {
                    const auto& cd = dims(n.inputs[2]);
                    if (cd.size() == 1 && cd[0] == gg.N) {
                        ep.bias = F(n.inputs[2]);
                        ep.bias_scale = beta;
                    } else if (cd.size() == 2 && cd[0] == gg.M && cd[1] == gg.N) {
                        ep.res = F(n.inputs[2]);
                        ep.res_scale = beta;
                    } else {
                        throw LoadError(n.where() + ": bias shape must be [N] or [M,N]");
                    }
                }
                if (!e.residual.empty()) {
                    if (ep.res) {
                        throw LoadError(n.where() + ": cannot fuse a residual into a Gemm with an [M,N] bias");
                    }
                    ep.res = F(e.residual);
                }
            } else {
                // MatMul (src/kernels/mat_mul.cpp:79-169)
                std::vector<int64_t> a = ad, b = bd;
                if (a.size() == 1) {
                    a.insert(a.begin(), 1);
                }
                if (b.size() == 1) {
                    b.push_back(1);
                }
                const int64_t M = a[a.size() - 2], K = a.back(), N = b.back();
                int64_t batch = 1, a_count = 1, b_count = 1;
                const auto& yd = dims(n.outputs[0]);
                (void)yd;
                std::vector<int64_t> ab(a.begin(), a.end() - 2), bb(b.begin(), b.end() - 2);
                const size_t r = std::max(ab.size(), bb.size());
                ab.insert(ab.begin(), r - ab.size(), 1);
                bb.insert(bb.begin(), r - bb.size(), 1);
                for (size_t i = 0; i < r; ++i) {
                    batch *= std::max(ab[i], bb[i]);
                    a_count *= ab[i];
                    b_count *= bb[i];
                }
                if ((a_count != batch && a_count != 1) || (b_count != batch && b_count != 1)) {
                    throw LoadError(n.where() + ": partial batch broadcasting is not supported");
                }
                gg.N = N;
                gg.K = K;
                gg.lda = K;
                gg.ldb = N;
                gg.ldc = N;
                if (b_count == 1) {
                    gg.M = M * batch;
                } else {
                    gg.M = M;
                    gg.batch = batch;
                    gg.a_zstride = a_count == 1 ? 0 : M * K;
                    gg.b_zstride = K * N;
                    gg.c_zstride = M * N;
                }
                if (!e.bias.empty()) {
                    ep.bias = F(e.bias);
                }
                if (!e.residual.empty()) {
                    ep.res = F(e.residual);
                }
                if (!e.perm.empty()) {
                    int64_t Z = 1, R = 1, C = 1;
                    matmul_zrc(yd, bd, Z, R, C);
                    if (Z != gg.batch || R != gg.M || C != gg.N || !make_out_map(e.view, e.perm, Z, R, C, &gg.omap)) {
                        throw LoadError(n.where() + ": transposed output does not match the contraction");
                    }
                }
            }
            ep.act = e.act;
            ep.act_a = e.act_a;
            ep.act_b = e.act_b;
            ep.act_c = e.act_c;
            ep.alpha *= e.alpha;
            const float* A = F(n.inputs[0]);
            float* y = F(e.out);
            const int64_t pbytes = static_cast<int64_t>(gemm_packed_bytes(gg));
            nb2_device* dev = dev_;
            const int gemm_k = contraction_launches(dev_, gg.M, gg.N, gg.K, gg.batch);
            st.launches = gemm_k;
            if (packed_gemm.count(n.inputs[1])) {
                uint8_t* packed = dmalloc(align_up(pbytes));
                gemm_pack_b(dev_, gg, F(n.inputs[1]), packed);
                check_cuda(cudaStreamSynchronize(dev_->stream), "pack sync");
                weight_bytes_ += pbytes;
                st.run = [=] { gemm_run(dev, gg, A, packed, y, ep); };
            } else {
                const float* B = F(n.inputs[1]);
                scratch_need = std::max(scratch_need, pbytes);
                void** sp = &scratch_;
                st.launches = gemm_k + 1;
                st.run = [=] {
                    gemm_pack_b(dev, gg, B, *sp);
                    gemm_run(dev, gg, A, *sp, y, ep);
                };
            }
        } else if (e.op == "Relu" || e.op == "Sigmoid" || e.op == "Erf" || e.op == "Sqrt" || e.op == "Neg" ||
                   e.op == "Abs" || e.op == "Exp" || e.op == "Tanh") {
            static const std::map<std::string, int> codes = {{"Relu", kURelu}, {"Sigmoid", kUSigmoid},
                                                             {"Erf", kUErf},   {"Sqrt", kUSqrt},
                                                             {"Neg", kUNeg},   {"Abs", kUAbs},
                                                             {"Exp", kUExp},   {"Tanh", kUTanh}};
            const int code = codes.at(e.op);
            const float* x = F(n.inputs[0]);
            float* y = F(n.outputs[0]);
            const int64_t cnt = numel(dims(n.outputs[0]));
            nb2_device* dev = dev_;
            st.run = [=] { unary(dev, code, x, y, cnt); };
        } else if (e.op == "Add" || e.op == "Sub" || e.op == "Mul" || e.op == "Div" || e.op == "Pow") {
            static const std::map<std::string, int> codes = {
                {"Add", kBAdd}, {"Sub", kBSub}, {"Mul", kBMul}, {"Div", kBDiv}, {"Pow", kBPow}};
            const int code = codes.at(e.op);
            const TensorInfo& ta = shapes_.at(n.inputs[0]);
            const int dt = ta.dtype == DType::I64 ? kI64 : kF32;
            const void* a = P(n.inputs[0]);
            const void* b = P(n.inputs[1]);
            void* y = P(n.outputs[0]);
            const auto ad = dims(n.inputs[0]), bd = dims(n.inputs[1]), yd = dims(n.outputs[0]);
            nb2_device* dev = dev_;
            st.run = [=] { binary(dev, code, dt, a, ad, b, bd, y, yd); };
        } else if (e.op == "Attention") {
            const auto& qd = dims(e.ins[0]);
            const int64_t B = qd[0], H = qd[1], T = qd[2], D = qd[3];
            AttnGeom ag{};
            ag.B = B;
            ag.H = H;
            ag.T = T;
            ag.qb = H * T * D, ag.qh = T * D, ag.qt = D, ag.qj = 1;
            ag.kb = H * D * T, ag.kh = D * T, ag.kt = 1, ag.kj = T; // K^T [B, H, D, T]
            ag.vb = H * T * D, ag.vh = T * D, ag.vt = D, ag.vj = 1;
            if (e.attn_merged) {
                ag.ob = T * H * D, ag.oh = D, ag.ot = H * D; // [B, T, H*D]
            } else {
                ag.ob = H * T * D, ag.oh = T * D, ag.ot = D;
            }
            ag.scale_mode = e.attn_mode;
            ag.scale = e.attn_scale;
            const float* q = F(e.ins[0]);
            const float* k = F(e.ins[1]);
            const float* v = F(e.ins[2]);
            float* y = F(e.out);
            nb2_device* dev = dev_;
            st.label = std::string("Attention:") + n.name;
            st.run = [=] { attention(dev, ag, q, k, v, y); };
        } else if (e.op == "SPPF") {
            const auto& xd = dims(e.ins[0]);
            const SppfGeom sg{xd[0], xd[1], xd[2], xd[3], e.pool_k, e.chain};
            const float* x = F(e.ins[0]);
            float* y = F(e.out);
            nb2_device* dev = dev_;
            st.label = "SPPF:" + n.name;
            st.run = [=] { sppf_nchw(dev, sg, x, y); };
        } else if (e.op == "MaxPool") {
            const auto& xd = dims(n.inputs[0]);
            const auto& yd = dims(n.outputs[0]);
            std::vector<int64_t> k = n.getints("kernel_shape"), s = n.getints("strides"), d = n.getints("dilations"),
                                 pads = n.getints("pads");
            if (s.empty()) {
                s = {1, 1};
            }
            if (d.empty()) {
                d = {1, 1};
            }
            if (pads.empty()) {
                pads = {0, 0, 0, 0};
            }
            if (n.gets("auto_pad", "NOTSET") != "NOTSET" || n.outputs.size() > 1) {
                throw LoadError(n.where() + ": auto_pad and the Indices output are not supported on B200");
            }
            PoolGeom pg{xd[0], xd[1], xd[2], xd[3], yd[2], yd[3], k[0], k[1], s[0], s[1], pads[0], pads[1], d[0], d[1]};
            const float* x = F(n.inputs[0]);
            float* y = F(n.outputs[0]);
            nb2_device* dev = dev_;
            if (nhwc.count(n.inputs[0])) {
                st.label += "[nhwc]";
                st.run = [=] { maxpool2d_nhwc(dev, pg, x, y); };
            } else {
                st.run = [=] { maxpool2d(dev, pg, x, y); };
            }
        } else if (e.op == "ConvTranspose") {
            // a stride-1 Conv over the zero-inserted input (ops_convt.cu); the
            // weight is transposed, flipped and packed once here
            const auto& xd = dims(n.inputs[0]);
            const auto& wd = dims(n.inputs[1]);
            const auto& yd = dims(n.outputs[0]);
            auto list = [&](const char* k, int64_t def, size_t len) {
                std::vector<int64_t> v = n.getints(k);
                if (v.empty() || (std::string(k) == "pads" && n.gets("auto_pad", "NOTSET") == "VALID")) {
                    v.assign(len, def);
                }
                return v;
            };
            const auto s2 = list("strides", 1, 2), d2 = list("dilations", 1, 2), op2 = list("output_padding", 0, 2),
                       p4 = list("pads", 0, 4);
            const int64_t grp = n.geti("group", 1);
            const ConvTGeom t{xd[0], xd[1], xd[2], xd[3], wd[1] * grp, wd[2], wd[3], yd[2], yd[3], s2[0], s2[1],
                              p4[0], p4[1], p4[2], p4[3], d2[0], d2[1], op2[0], op2[1], grp};
            ConvGeom geom = convt_as_conv(t);
            if ((flags & kNchwOnly) == 0) {
                geom = nchw_input_layout(geom);
            }
            if (!g_.constants.count(n.inputs[1])) {
                throw LoadError(n.where() + ": the weight must be a constant on B200");
            }
            const Constant& wc = g_.constants.at(n.inputs[1]);
            const int64_t pbytes = static_cast<int64_t>(conv_packed_bytes(geom));
            uint8_t* packed = dmalloc(align_up(pbytes));
            void* tmp = nullptr;
            check_cuda(cudaMalloc(&tmp, 2 * wc.bytes.size()), "cudaMalloc(weight staging)");
            check_cuda(cudaMemcpyAsync(tmp, wc.bytes.data(), wc.bytes.size(), cudaMemcpyHostToDevice, dev_->stream),
                       "cudaMemcpyAsync(weight)");
            float* w2 = reinterpret_cast<float*>(static_cast<uint8_t*>(tmp) + wc.bytes.size());
            convt_flip_weights(dev_, t, static_cast<const float*>(tmp), w2);
            conv_pack(dev_, geom, w2, packed);
            check_cuda(cudaStreamSynchronize(dev_->stream), "pack sync");
            cudaFree(tmp);
            weight_bytes_ += pbytes;
            const size_t zb = convt_zero_insert_bytes(t);
            float* xz = zb ? reinterpret_cast<float*>(dmalloc(align_up(static_cast<int64_t>(zb)))) : nullptr;
            if (geom.converts_input()) {
                xform_need = std::max(xform_need, geom.N * geom.Cin() * geom.H * geom.W * 4);
            }
            Epilogue ep;
            ep.bias = n.inputs.size() > 2 && !n.inputs[2].empty() ? F(n.inputs[2]) : nullptr;
            const float* x = F(n.inputs[0]);
            float* y = F(n.outputs[0]);
            nb2_device* dev = dev_;
            void** xp = &xform_;
            st.launches = contraction_launches(dev_, geom.N * geom.OH * geom.OW, geom.Mg(), geom.K(), geom.group) +
                          (zb ? 1 : 0) + (geom.converts_input() ? 1 : 0);
            st.run = [=] {
                const float* src = x;
                if (xz) {
                    convt_zero_insert(dev, t, x, xz);
                    src = xz;
                }
                if (geom.converts_input()) {
                    nchw_to_nhwc_pad(dev, src, static_cast<float*>(*xp), geom.N, geom.C, geom.H, geom.W, geom.Cin());
                    conv_run(dev, geom, static_cast<const float*>(*xp), packed, y, ep);
                } else {
                    conv_run(dev, geom, src, packed, y, ep);
                }
            };
        } else if (e.op == "BatchNormalization") {
            // a BN the load-time fold could not merge into a Conv
            const auto& xd = dims(n.inputs[0]);
            int64_t inner = 1;
            for (size_t d = 2; d < xd.size(); ++d) {
                inner *= xd[d];
            }
            const int64_t outer = xd[0], C = xd[1];
            const float* x = F(n.inputs[0]);
            const float* a = F(n.inputs[1]);
            const float* sh = F(n.inputs[2]);
            float* y = F(n.outputs[0]);
            nb2_device* dev = dev_;
            st.run = [=] { channel_affine(dev, x, a, sh, y, outer, C, inner); };
        } else if (e.op == "AveragePool") {
            const auto& xd = dims(n.inputs[0]);
            const auto& yd = dims(n.outputs[0]);
            std::vector<int64_t> k = n.getints("kernel_shape"), s = n.getints("strides"), pads = n.getints("pads");
            if (s.empty()) {
                s = {1, 1};
            }
            if (pads.empty()) {
                pads = {0, 0, 0, 0};
            }
            if (n.gets("auto_pad", "NOTSET") != "NOTSET") {
                throw LoadError(n.where() + ": auto_pad is not supported on B200");
            }
            const AvgPoolGeom ag{xd[0], xd[1], xd[2], xd[3], yd[2], yd[3], k[0], k[1], s[0], s[1],
                                 pads[0], pads[1], pads[2], pads[3],
                                 n.geti("count_include_pad", 0) != 0 ? 1 : 0};
            const float* x = F(n.inputs[0]);
            float* y = F(n.outputs[0]);
            nb2_device* dev = dev_;
            st.run = [=] { avgpool2d(dev, ag, x, y); };
        } else if (e.op == "GlobalAveragePool" || e.op == "ReduceMean") {
            const auto& xd = dims(n.inputs[0]);
            int64_t rows = 1, inner = 1;
            if (e.op == "GlobalAveragePool") {
                rows = xd[0] * xd[1];
                inner = numel(xd) / rows;
            } else {
                std::vector<int64_t> axes = g_.opset >= 18
                                                ? (n.inputs.size() > 1 && !n.inputs[1].empty()
                                                       ? g_.constants.at(n.inputs[1]).as_i64()
                                                       : std::vector<int64_t>{})
                                                : n.getints("axes");
                const int64_t r = static_cast<int64_t>(xd.size());
                std::set<int64_t> ax;
                for (int64_t a : axes) {
                    ax.insert(a < 0 ? a + r : a);
                }
                if (axes.empty()) {
                    for (int64_t i = 0; i < r; ++i) {
                        ax.insert(i);
                    }
                }
                const int64_t first = *ax.begin();
                if (*ax.rbegin() != r - 1 || static_cast<int64_t>(ax.size()) != r - first) {
                    throw LoadError(n.where() + ": only trailing-axis means are implemented on B200");
                }
                for (int64_t i = 0; i < r; ++i) {
                    (i < first ? rows : inner) *= xd[i];
                }
            }
            const float* x = F(n.inputs[0]);
            float* y = F(n.outputs[0]);
            nb2_device* dev = dev_;
            if (e.op == "GlobalAveragePool" && nhwc.count(n.inputs[0])) {
                const int64_t N = xd[0], C = xd[1];
                st.label += "[nhwc]";
                st.run = [=] { mean_nhwc(dev, x, y, N, inner, C); };
            } else {
                st.run = [=] { row_mean(dev, x, y, rows, inner); };
            }
        } else if (e.op == "Softmax") {
            const auto& xd = dims(n.inputs[0]);
            const int64_t r = static_cast<int64_t>(xd.size());
            int64_t axis = n.geti("axis", g_.opset >= 13 ? -1 : 1);
            if (axis < 0) {
                axis += r;
            }
            int64_t outer = 1, L = 1, inner = 1;
            if (g_.opset >= 13) {
                for (int64_t i = 0; i < r; ++i) {
                    (i < axis ? outer : i == axis ? L : inner) *= xd[i];
                }
            } else { // legacy 2-D coercion (src/softmax_form.hpp)
                for (int64_t i = 0; i < r; ++i) {
                    (i < axis ? outer : L) *= xd[i];
                }
            }
            const float* x = F(n.inputs[0]);
            float* y = F(n.outputs[0]);
            nb2_device* dev = dev_;
            st.run = [=] { softmax(dev, x, y, outer, L, inner); };
        } else if (e.op == "LayerNormalization") {
            const auto& xd = dims(n.inputs[0]);
            const int64_t r = static_cast<int64_t>(xd.size());
            int64_t axis = n.geti("axis", -1);
            if (axis < 0) {
                axis += r;
            }
            int64_t rows = 1, D = 1;
            for (int64_t i = 0; i < r; ++i) {
                (i < axis ? rows : D) *= xd[i];
            }
            const float eps = n.getf("epsilon", 1e-5f);
            const float* x = F(n.inputs[0]);
            const float* sc = F(n.inputs[1]);
            const float* bi = n.inputs.size() > 2 ? F(n.inputs[2]) : nullptr;
            float* y = F(n.outputs[0]);
            float* mo = n.outputs.size() > 1 && !n.outputs[1].empty() ? F(n.outputs[1]) : nullptr;
            float* io = n.outputs.size() > 2 && !n.outputs[2].empty() ? F(n.outputs[2]) : nullptr;
            nb2_device* dev = dev_;
            st.run = [=] { layernorm(dev, x, sc, bi, y, mo, io, rows, D, eps); };
        } else {
            const bool cl = (e.op == "Concat" || e.op == "Split" || e.op == "Resize") && nhwc.count(n.outputs[0]) > 0;
            if (cl) {
                st.label += "[nhwc]";
            }
            MoveStep ms = build_move_step(n, g_, shapes_, P, dmalloc, cl);
            if (!ms.run) {
                throw LoadError(n.where() + ": op '" + n.op + "' has no row on the B200 device");
            }
            nb2_device* dev = dev_;
            auto run = ms.run;
            st.launches = ms.launches;
            st.run = [=] { run(dev); };
        }
        launches_ += st.launches;
        steps_.push_back(std::move(st));
    }
    if (xform_need > 0) {
        xform_ = dmalloc(align_up(xform_need));
    }
    if (scratch_need > 0) {
        scratch_ = dmalloc(align_up(scratch_need));
    }
    for (const auto& o : g_.outputs) {
        const TensorInfo& ti = shapes_.at(o.first);
        IOInfo io{o.first, ti.dtype, ti.dims, P(o.first), numel(ti.dims) * dtype_size(ti.dtype)};
        outputs_.push_back(io);
    }
    check_cuda(cudaStreamSynchronize(dev_->stream), "model build sync");
}

void Model::run_steps() {
    for (auto& s : steps_) {
        s.run();
    }
}

void Model::launch() {
    dev_->make_current();
    if (!use_graph_) {
        run_steps();
        return;
    }
    if (exec_ == nullptr || exec_precision_ != dev_->precision) {
        if (exec_) {
            check_cuda(cudaGraphExecDestroy(exec_), "cudaGraphExecDestroy");
            exec_ = nullptr;
        }
        // eager warm-up pass (sets kernel attributes, builds tensor maps)
        run_steps();
        check_cuda(cudaStreamSynchronize(dev_->stream), "warm-up sync");
        cudaGraph_t graph = nullptr;
        dev_->capturing = 1;
        check_cuda(cudaStreamBeginCapture(dev_->stream, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
        try {
            run_steps();
        } catch (...) {
            cudaStreamEndCapture(dev_->stream, &graph);
            if (graph) {
                cudaGraphDestroy(graph);
            }
            dev_->capturing = 0;
            throw;
        }
        check_cuda(cudaStreamEndCapture(dev_->stream, &graph), "cudaStreamEndCapture");
        dev_->capturing = 0;
        check_cuda(cudaGraphInstantiate(&exec_, graph, 0), "cudaGraphInstantiate");
        cudaGraphDestroy(graph);
        exec_precision_ = dev_->precision;
    }
    check_cuda(cudaGraphLaunch(exec_, dev_->stream), "cudaGraphLaunch");
}

void Model::synchronize() {
    dev_->make_current();
    const int code = dev_->take_device_error();
    if (code != 0) {
        throw RunError("a kernel reported device error " + std::to_string(code) +
                       (code == 2 ? " (index out of range)" : code == 1 ? " (bounded wait expired)" : ""));
    }
}

void Model::run_host(const std::vector<const void*>& in, const std::vector<void*>& out) {
    enqueue_host(in, out);
    synchronize();
}

void Model::enqueue_host(const std::vector<const void*>& in, const std::vector<void*>& out) {
    if (in.size() != inputs_.size() || out.size() != outputs_.size()) {
        throw RunError("executor: expected " + std::to_string(inputs_.size()) + " inputs and " +
                       std::to_string(outputs_.size()) + " outputs");
    }
    dev_->make_current();
    if (copy_stream_ == nullptr) {
        int64_t total = 0;
        for (const auto& io : inputs_) {
            total += align_up(io.bytes);
        }
        check_cuda(cudaStreamCreateWithFlags(&copy_stream_, cudaStreamNonBlocking), "cudaStreamCreate(copy)");
        for (int k = 0; k < 2; ++k) {
            void* p = nullptr;
            check_cuda(cudaMalloc(&p, static_cast<size_t>(std::max<int64_t>(total, 256))), "cudaMalloc(staging)");
            allocations_.push_back(p);
            stage_[k] = static_cast<uint8_t*>(p);
            check_cuda(cudaEventCreateWithFlags(&staged_[k], cudaEventDisableTiming), "cudaEventCreate");
            check_cuda(cudaEventCreateWithFlags(&freed_[k], cudaEventDisableTiming), "cudaEventCreate");
            check_cuda(cudaEventRecord(freed_[k], dev_->stream), "cudaEventRecord");
        }
    }
    // host -> staging k on the copy stream, once run pipe_runs_ - 2 has moved
    // its inputs out of it; this run waits for the copy, moves the inputs into
    // place and releases the staging buffer
    const int k = static_cast<int>(pipe_runs_ & 1);
    check_cuda(cudaStreamWaitEvent(copy_stream_, freed_[k], 0), "cudaStreamWaitEvent");
    int64_t off = 0;
    for (size_t i = 0; i < in.size(); ++i) {
        if (inputs_[i].bytes > 0) {
            check_cuda(cudaMemcpyAsync(stage_[k] + off, in[i], static_cast<size_t>(inputs_[i].bytes),
                                       cudaMemcpyHostToDevice, copy_stream_),
                       "cudaMemcpyAsync(input)");
        }
        off += align_up(inputs_[i].bytes);
    }
    check_cuda(cudaEventRecord(staged_[k], copy_stream_), "cudaEventRecord");
    check_cuda(cudaStreamWaitEvent(dev_->stream, staged_[k], 0), "cudaStreamWaitEvent");
    off = 0;
    for (size_t i = 0; i < in.size(); ++i) {
        if (inputs_[i].bytes > 0) {
            check_cuda(cudaMemcpyAsync(inputs_[i].dev, stage_[k] + off, static_cast<size_t>(inputs_[i].bytes),
                                       cudaMemcpyDeviceToDevice, dev_->stream),
                       "cudaMemcpyAsync(stage)");
        }
        off += align_up(inputs_[i].bytes);
    }
    check_cuda(cudaEventRecord(freed_[k], dev_->stream), "cudaEventRecord");
    ++pipe_runs_;
    launch();
    for (size_t i = 0; i < out.size(); ++i) {
        if (outputs_[i].bytes > 0) {
            check_cuda(cudaMemcpyAsync(out[i], outputs_[i].dev, static_cast<size_t>(outputs_[i].bytes),
                                       cudaMemcpyDeviceToHost, dev_->stream),
                       "cudaMemcpyAsync(output)");
        }
    }
}

std::vector<std::pair<std::string, float>> Model::profile() {
    dev_->make_current();
    std::vector<std::pair<std::string, float>> out;
    std::vector<cudaEvent_t> ev(steps_.size() + 1);
    for (auto& e : ev) {
        check_cuda(cudaEventCreate(&e), "cudaEventCreate");
    }
    run_steps(); // warm
    check_cuda(cudaEventRecord(ev[0], dev_->stream), "cudaEventRecord");
    for (size_t i = 0; i < steps_.size(); ++i) {
        steps_[i].run();
        check_cuda(cudaEventRecord(ev[i + 1], dev_->stream), "cudaEventRecord");
    }
    check_cuda(cudaStreamSynchronize(dev_->stream), "profile sync");
    for (size_t i = 0; i < steps_.size(); ++i) {
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, ev[i], ev[i + 1]);
        out.emplace_back(steps_[i].label, ms);
    }
    for (auto& e : ev) {
        cudaEventDestroy(e);
    }
    return out;
}

} // namespace eng
} // namespace nb2

namespace nb2 {
namespace eng {

namespace {
std::string jstr(const std::string& s) {
    std::string o = "\"";
    for (char c : s) {
        if (c == '"' || c == '\\') {
            o += '\\';
        }
        o += c;
    }
    return o + "\"";
}
std::string jdims(const std::vector<int64_t>& d) {
    std::string o = "[";
    for (size_t i = 0; i < d.size(); ++i) {
        o += (i ? "," : "") + std::to_string(d[i]);
    }
    return o + "]";
}
} // namespace

std::string analyze_json(const uint8_t* onnx, size_t size, const std::map<std::string, std::vector<int64_t>>& dims,
                         int flags) {
    const Graph g = parse_onnx(onnx, size);
    const PlanResult pr = plan_graph(g, dims, flags);
    auto root_of = [&](const std::string& t) {
        auto it = pr.root.find(t);
        return it == pr.root.end() ? t : it->second;
    };
    std::string o = "{\"arena\":" + std::to_string(pr.arena) + ",\"fused_groups\":" +
                    std::to_string(pr.fused_groups) + ",\"opset\":" + std::to_string(g.opset) + ",\"exec\":[";
    for (size_t i = 0; i < pr.ex.size(); ++i) {
        const ExecNode& e = pr.ex[i];
        o += (i ? "," : "") + std::string("{\"op\":") + jstr(e.op) + ",\"name\":" + jstr(e.node->name) +
             ",\"act\":" + std::to_string(e.act) + ",\"group\":" + std::to_string(e.group) +
             ",\"alias\":" + (e.alias ? "true" : "false") + ",\"residual\":" + jstr(e.residual) +
             ",\"bias\":" + jstr(e.bias) + ",\"perm\":[";
        for (size_t j = 0; j < e.perm.size(); ++j) {
            o += (j ? "," : "") + std::to_string(e.perm[j]);
        }
        o += "],\"ins\":[";
        for (size_t j = 0; j < e.ins.size(); ++j) {
            o += (j ? "," : "") + jstr(e.ins[j]);
        }
        o += "],\"outs\":[";
        for (size_t j = 0; j < e.outs.size(); ++j) {
            o += (j ? "," : "") + jstr(e.outs[j]);
        }
        o += "]}";
    }
    o += "],\"tensors\":{";
    bool first = true;
    for (const auto& kv : pr.shapes) {
        if (g.constants.count(kv.first)) {
            continue;
        }
        const std::string r = root_of(kv.first);
        auto off = pr.offset.find(r);
        auto lu = pr.last_use.find(r);
        o += std::string(first ? "" : ",") + jstr(kv.first) + ":{\"dims\":" + jdims(kv.second.dims) +
             ",\"dtype\":" + std::to_string(static_cast<int>(kv.second.dtype)) + ",\"root\":" + jstr(r) +
             ",\"offset\":" + (off == pr.offset.end() ? std::string("-1") : std::to_string(off->second)) +
             ",\"bytes\":" + std::to_string(numel(kv.second.dims) * dtype_size(kv.second.dtype)) +
             ",\"last_use\":" + (lu == pr.last_use.end() ? std::string("-1") : std::to_string(lu->second)) +
             ",\"nhwc\":" + (pr.nhwc.count(kv.first) ? "true" : "false") + "}";
        first = false;
    }
    return o + "}}";
}

} // namespace eng
} // namespace nb2
