// ONNX protobuf reader for the B200 engine (a hand-written wire decoder, as in
// the reference's src/wire_reader.cpp; field numbers from the public ONNX
// schema, the same ones the reference decodes at src/model_loader.cpp:41-97).

#include "graph.hpp"

#include <cstring>

namespace nb2 {
namespace eng {

namespace {

struct Reader {
    const uint8_t* p;
    const uint8_t* end;
    Reader(const uint8_t* d, size_t n) : p(d), end(d + n) {}
    bool done() const { return p >= end; }
    uint64_t varint() {
        uint64_t v = 0;
        int shift = 0;
        while (true) {
            if (p >= end || shift > 63) {
                throw LoadError("malformed protobuf varint");
            }
            const uint8_t b = *p++;
            v |= static_cast<uint64_t>(b & 0x7F) << shift;
            if ((b & 0x80) == 0) {
                return v;
            }
            shift += 7;
        }
    }
    void tag(int& field, int& wire) {
        const uint64_t k = varint();
        field = static_cast<int>(k >> 3);
        wire = static_cast<int>(k & 7);
    }
    std::pair<const uint8_t*, size_t> bytes() {
        const uint64_t n = varint();
        if (n > static_cast<uint64_t>(end - p)) {
            throw LoadError("malformed protobuf length");
        }
        const uint8_t* s = p;
        p += n;
        return {s, static_cast<size_t>(n)};
    }
    std::string str() {
        auto b = bytes();
        return std::string(reinterpret_cast<const char*>(b.first), b.second);
    }
    uint32_t fixed32() {
        if (end - p < 4) {
            throw LoadError("malformed protobuf fixed32");
        }
        uint32_t v;
        std::memcpy(&v, p, 4);
        p += 4;
        return v;
    }
    void skip(int wire) {
        switch (wire) {
        case 0:
            varint();
            break;
        case 1:
            if (end - p < 8) {
                throw LoadError("malformed protobuf fixed64");
            }
            p += 8;
            break;
        case 2:
            bytes();
            break;
        case 5:
            fixed32();
            break;
        default:
            throw LoadError("unsupported protobuf wire type");
        }
    }
};

void read_ints(Reader& r, int wire, std::vector<int64_t>& out) {
    if (wire == 0) {
        out.push_back(static_cast<int64_t>(r.varint()));
        return;
    }
    auto b = r.bytes();
    Reader sub(b.first, b.second);
    while (!sub.done()) {
        out.push_back(static_cast<int64_t>(sub.varint()));
    }
}

void read_floats(Reader& r, int wire, std::vector<float>& out) {
    auto push = [&](uint32_t bits) {
        float f;
        std::memcpy(&f, &bits, 4);
        out.push_back(f);
    };
    if (wire == 5) {
        push(r.fixed32());
        return;
    }
    auto b = r.bytes();
    Reader sub(b.first, b.second);
    while (!sub.done()) {
        push(sub.fixed32());
    }
}

DType dtype_of(int64_t code) {
    switch (code) {
    case 1:
        return DType::F32;
    case 7:
        return DType::I64;
    case 9:
        return DType::Bool;
    default:
        return DType::Unknown;
    }
}

std::pair<std::string, Constant> read_tensor(const uint8_t* d, size_t n) {
    Reader r(d, n);
    std::string name;
    Constant c;
    int64_t code = 1;
    std::vector<float> floats;
    std::vector<int64_t> ints;
    bool have_raw = false;
    while (!r.done()) {
        int f, w;
        r.tag(f, w);
        switch (f) {
        case 1:
            read_ints(r, w, c.dims);
            break;
        case 2:
            code = static_cast<int64_t>(r.varint());
            break;
        case 4:
            read_floats(r, w, floats);
            break;
        case 5: // int32_data (bool payloads)
        case 7:
            read_ints(r, w, ints);
            break;
        case 8:
            name = r.str();
            break;
        case 9: {
            auto b = r.bytes();
            c.bytes.assign(b.first, b.first + b.second);
            have_raw = true;
            break;
        }
        case 13:
            throw LoadError("tensor '" + name + "': external data is not supported by the B200 engine loader");
        default:
            r.skip(w);
        }
    }
    c.dtype = dtype_of(code);
    if (c.dtype == DType::Unknown) {
        throw LoadError("tensor '" + name + "': unsupported element type " + std::to_string(code));
    }
    if (!have_raw) {
        if (c.dtype == DType::F32) {
            c.bytes.resize(floats.size() * 4);
            std::memcpy(c.bytes.data(), floats.data(), c.bytes.size());
        } else if (c.dtype == DType::I64) {
            c.bytes.resize(ints.size() * 8);
            std::memcpy(c.bytes.data(), ints.data(), c.bytes.size());
        } else {
            c.bytes.resize(ints.size());
            for (size_t i = 0; i < ints.size(); ++i) {
                c.bytes[i] = ints[i] != 0;
            }
        }
    }
    if (static_cast<int64_t>(c.bytes.size()) != c.count() * dtype_size(c.dtype)) {
        throw LoadError("tensor '" + name + "': payload size does not match its dims");
    }
    return {name, std::move(c)};
}

Attr read_attr(const uint8_t* d, size_t n, std::string& name) {
    Reader r(d, n);
    Attr a;
    int64_t type = 0;
    while (!r.done()) {
        int f, w;
        r.tag(f, w);
        switch (f) {
        case 1:
            name = r.str();
            break;
        case 2: {
            const uint32_t bits = r.fixed32();
            std::memcpy(&a.f, &bits, 4);
            a.kind = Attr::kFloat;
            break;
        }
        case 3:
            a.i = static_cast<int64_t>(r.varint());
            a.kind = Attr::kInt;
            break;
        case 4:
            a.s = r.str();
            a.kind = Attr::kString;
            break;
        case 5: {
            auto b = r.bytes();
            a.t = read_tensor(b.first, b.second).second;
            a.kind = Attr::kTensor;
            break;
        }
        case 7:
            read_floats(r, w, a.floats);
            break;
        case 8:
            read_ints(r, w, a.ints);
            break;
        case 20:
            type = static_cast<int64_t>(r.varint());
            break;
        default:
            r.skip(w);
        }
    }
    if (type == 6) {
        a.kind = Attr::kFloats;
    } else if (type == 7) {
        a.kind = Attr::kInts;
    } else if (a.kind == Attr::kNone && !a.ints.empty()) {
        a.kind = Attr::kInts;
    } else if (a.kind == Attr::kNone && !a.floats.empty()) {
        a.kind = Attr::kFloats;
    } else if (a.kind == Attr::kNone && type == 7) {
        a.kind = Attr::kInts;
    }
    return a;
}

std::pair<std::string, TensorInfo> read_value_info(const uint8_t* d, size_t n) {
    Reader r(d, n);
    std::string name;
    TensorInfo info;
    while (!r.done()) {
        int f, w;
        r.tag(f, w);
        if (f == 1) {
            name = r.str();
        } else if (f == 2) {
            auto tb = r.bytes();
            Reader tr(tb.first, tb.second);
            while (!tr.done()) {
                int f2, w2;
                tr.tag(f2, w2);
                if (f2 != 1) {
                    tr.skip(w2);
                    continue;
                }
                auto tt = tr.bytes();
                Reader ttr(tt.first, tt.second);
                while (!ttr.done()) {
                    int f3, w3;
                    ttr.tag(f3, w3);
                    if (f3 == 1) {
                        info.dtype = dtype_of(static_cast<int64_t>(ttr.varint()));
                    } else if (f3 == 2) {
                        auto sb = ttr.bytes();
                        Reader sr(sb.first, sb.second);
                        while (!sr.done()) {
                            int f4, w4;
                            sr.tag(f4, w4);
                            if (f4 != 1) {
                                sr.skip(w4);
                                continue;
                            }
                            auto db = sr.bytes();
                            Reader dr(db.first, db.second);
                            int64_t dim = -1;
                            while (!dr.done()) {
                                int f5, w5;
                                dr.tag(f5, w5);
                                if (f5 == 1) {
                                    dim = static_cast<int64_t>(dr.varint());
                                } else {
                                    dr.skip(w5);
                                }
                            }
                            info.dims.push_back(dim);
                        }
                    } else {
                        ttr.skip(w3);
                    }
                }
            }
        } else {
            r.skip(w);
        }
    }
    return {name, info};
}

} // namespace

std::vector<int64_t> Constant::as_i64() const {
    std::vector<int64_t> out(static_cast<size_t>(count()));
    if (dtype == DType::I64) {
        std::memcpy(out.data(), bytes.data(), out.size() * 8);
    } else if (dtype == DType::F32) {
        for (size_t i = 0; i < out.size(); ++i) {
            out[i] = static_cast<int64_t>(f32()[i]);
        }
    } else {
        for (size_t i = 0; i < out.size(); ++i) {
            out[i] = bytes[i];
        }
    }
    return out;
}

int64_t Node::geti(const std::string& k, int64_t def) const {
    auto it = attrs.find(k);
    if (it == attrs.end()) {
        return def;
    }
    if (it->second.kind != Attr::kInt) {
        throw RunError(where() + ": attribute '" + k + "' must be an integer");
    }
    return it->second.i;
}

float Node::getf(const std::string& k, float def) const {
    auto it = attrs.find(k);
    if (it == attrs.end()) {
        return def;
    }
    if (it->second.kind != Attr::kFloat) {
        throw RunError(where() + ": attribute '" + k + "' must be a float");
    }
    return it->second.f;
}

std::string Node::gets(const std::string& k, const std::string& def) const {
    auto it = attrs.find(k);
    if (it == attrs.end()) {
        return def;
    }
    return it->second.s;
}

std::vector<int64_t> Node::getints(const std::string& k) const {
    auto it = attrs.find(k);
    if (it == attrs.end()) {
        return {};
    }
    if (it->second.kind != Attr::kInts) {
        throw RunError(where() + ": attribute '" + k + "' must be an int list");
    }
    return it->second.ints;
}

int64_t numel(const std::vector<int64_t>& d) {
    int64_t n = 1;
    for (int64_t v : d) {
        n *= v;
    }
    return n;
}

Graph parse_onnx(const uint8_t* data, size_t size) {
    Graph g;
    Reader r(data, size);
    std::pair<const uint8_t*, size_t> graph_bytes{nullptr, 0};
    while (!r.done()) {
        int f, w;
        r.tag(f, w);
        if (f == 7 && w == 2) {
            graph_bytes = r.bytes();
        } else if (f == 8 && w == 2) {
            auto ob = r.bytes();
            Reader orr(ob.first, ob.second);
            std::string domain;
            int64_t version = -1;
            while (!orr.done()) {
                int f2, w2;
                orr.tag(f2, w2);
                if (f2 == 1) {
                    domain = orr.str();
                } else if (f2 == 2) {
                    version = static_cast<int64_t>(orr.varint());
                } else {
                    orr.skip(w2);
                }
            }
            if (domain.empty() || domain == "ai.onnx") {
                g.opset = version;
            }
        } else {
            r.skip(w);
        }
    }
    if (graph_bytes.first == nullptr) {
        throw LoadError("model carries no graph");
    }
    if (g.opset < 11) {
        throw LoadError("model does not declare an ONNX-domain opset of 11 or above");
    }
    Reader gr(graph_bytes.first, graph_bytes.second);
    std::vector<std::pair<std::string, TensorInfo>> declared_inputs;
    while (!gr.done()) {
        int f, w;
        gr.tag(f, w);
        if (f == 1 && w == 2) {
            auto nb = gr.bytes();
            Reader nr(nb.first, nb.second);
            Node node;
            while (!nr.done()) {
                int f2, w2;
                nr.tag(f2, w2);
                switch (f2) {
                case 1:
                    node.inputs.push_back(nr.str());
                    break;
                case 2:
                    node.outputs.push_back(nr.str());
                    break;
                case 3:
                    node.name = nr.str();
                    break;
                case 4:
                    node.op = nr.str();
                    break;
                case 5: {
                    auto ab = nr.bytes();
                    std::string an;
                    Attr a = read_attr(ab.first, ab.second, an);
                    node.attrs[an] = std::move(a);
                    break;
                }
                case 7: {
                    const std::string dom = nr.str();
                    if (!dom.empty() && dom != "ai.onnx") {
                        throw LoadError("node '" + node.name + "': domain '" + dom + "' is not supported");
                    }
                    break;
                }
                default:
                    nr.skip(w2);
                }
            }
            if (node.op.empty()) {
                throw LoadError("node '" + node.name + "' is missing op_type");
            }
            if (node.op == "Constant") {
                auto it = node.attrs.find("value");
                if (it == node.attrs.end() || it->second.kind != Attr::kTensor || node.outputs.size() != 1) {
                    throw LoadError("Constant node '" + node.name + "' needs a tensor 'value'");
                }
                g.constants[node.outputs[0]] = it->second.t;
            } else {
                g.nodes.push_back(std::move(node));
            }
        } else if (f == 5 && w == 2) {
            auto tb = gr.bytes();
            auto t = read_tensor(tb.first, tb.second);
            g.constants[t.first] = std::move(t.second);
        } else if (f == 11 && w == 2) {
            auto vb = gr.bytes();
            declared_inputs.push_back(read_value_info(vb.first, vb.second));
        } else if (f == 12 && w == 2) {
            auto vb = gr.bytes();
            g.outputs.push_back(read_value_info(vb.first, vb.second));
        } else {
            gr.skip(w);
        }
    }
    for (auto& in : declared_inputs) {
        if (g.constants.count(in.first) == 0) {
            g.inputs.push_back(in);
        }
    }
    if (g.nodes.empty()) {
        throw LoadError("graph has no nodes");
    }
    fold_batchnorm(g);
    return g;
}

} // namespace eng
} // namespace nb2
