// The extern "C" boundary (include/nert_b200.h): validation, then a launch on
// the device's stream. C++ exceptions never cross it.

#include "../../include/nert_b200.h"
#include "igemm.cuh"
#include "ops.cuh"
#include "ops_move.cuh"
#include "ops_norm.cuh"
#include "runtime.hpp"

#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

namespace nb2 {
const char* last_error();
}

using namespace nb2;

namespace {

template <typename F>
int guard(F&& f) {
    try {
        f();
        return NB2_OK;
    } catch (const Error& e) {
        set_last_error(e.what());
        return e.code;
    } catch (const std::bad_alloc&) {
        set_last_error("out of host memory");
        return NB2_ERR_NOMEM;
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return NB2_ERR_INVALID;
    }
}

void need(bool ok, const std::string& msg) {
    if (!ok) {
        fail(kStatusInvalid, msg);
    }
}

nb2_device* bind(nb2_device* dev) {
    need(dev != nullptr, "null device");
    dev->make_current();
    return dev;
}

ConvGeom to_geom(const nb2_conv_geom* c) {
    need(c != nullptr, "Conv: null geometry");
    ConvGeom g{};
    g.N = c->n;
    g.C = c->c;
    g.H = c->h;
    g.W = c->w;
    g.M = c->m;
    g.KH = c->kh;
    g.KW = c->kw;
    g.OH = c->oh;
    g.OW = c->ow;
    g.sh = c->stride_h;
    g.sw = c->stride_w;
    g.ph = c->pad_top;
    g.pw = c->pad_left;
    g.dh = c->dil_h;
    g.dw = c->dil_w;
    g.group = c->group;
    // Same checks and output formula as the reference Conv row
    // (src/kernels/conv.cpp:151-218, WindowOutput :122-135).
    need(g.N > 0 && g.C > 0 && g.H > 0 && g.W > 0 && g.M > 0 && g.KH > 0 && g.KW > 0,
         "Conv: non-positive dimension");
    need(g.group > 0, "Conv: group must be positive");
    need(g.C % g.group == 0, "Conv: input channels are not divisible by group");
    need(g.M % g.group == 0, "Conv: output channels are not divisible by group");
    need(g.sh > 0 && g.sw > 0 && g.dh > 0 && g.dw > 0, "Conv: stride and dilation must be positive");
    need(c->pad_top >= 0 && c->pad_left >= 0 && c->pad_bottom >= 0 && c->pad_right >= 0,
         "Conv: pads must be non-negative");
    auto out_dim = [](int64_t in, int64_t k, int64_t d, int64_t pb, int64_t pe, int64_t s) {
        const int64_t numer = in + pb + pe - (d * (k - 1) + 1);
        return numer < 0 ? int64_t{-1} : numer / s + 1;
    };
    const int64_t oh = out_dim(g.H, g.KH, g.dh, c->pad_top, c->pad_bottom, g.sh);
    const int64_t ow = out_dim(g.W, g.KW, g.dw, c->pad_left, c->pad_right, g.sw);
    need(oh > 0 && ow > 0, "Conv: window is larger than the padded input");
    need(oh == g.OH && ow == g.OW, "Conv: output shape does not match the convolution");
    need(g.KH * g.dh < 32768 && g.KW * g.dw < 32768, "Conv: kernel extent too large");
    return g;
}

struct HostStage {
    // pinned bounce buffer per device, grown on demand
    static void* get(nb2_device* dev, size_t bytes) {
        if (bytes > dev->pinned_bytes) {
            check_cuda(cudaStreamSynchronize(dev->stream), "cudaStreamSynchronize");
            if (dev->pinned) {
                check_cuda(cudaFreeHost(dev->pinned), "cudaFreeHost");
                dev->pinned = nullptr;
                dev->pinned_bytes = 0;
            }
            const size_t sz = std::max<size_t>(bytes, 1 << 20);
            check_cuda(cudaMallocHost(&dev->pinned, sz), "cudaMallocHost");
            dev->pinned_bytes = sz;
        }
        return dev->pinned;
    }
};

} // namespace

namespace {

// Bytes of the NHWC copy a converted NCHW input needs (0 when none).
size_t nhwc_copy_bytes(const ConvGeom& g) {
    return g.converts_input() ? static_cast<size_t>(g.N * g.Cin() * g.H * g.W * 4) : 0;
}

// A Conv whose input arrives NCHW: converted to NHWC first when its layout
// asks for it (into `xbuf`, or the device workspace when null), then run.
void run_nchw_conv(nb2_device* dev, const ConvGeom& g, const float* x, const void* packed, float* y,
                   const Epilogue& ep, void* xbuf) {
    if (g.converts_input()) {
        float* xp = static_cast<float*>(xbuf != nullptr ? xbuf : dev->scratch(nhwc_copy_bytes(g)));
        nchw_to_nhwc_pad(dev, x, xp, g.N, g.C, g.H, g.W, g.Cin());
        conv_run(dev, g, xp, packed, y, ep);
        return;
    }
    conv_run(dev, g, x, packed, y, ep);
}

} // namespace

namespace nb2 {
// The validated geometry of a C-ABI Conv description (shared by every Conv
// entry point).
ConvGeom conv_geom_from_c(const nb2_conv_geom* c) { return to_geom(c); }
} // namespace nb2

extern "C" {

const char* nb2_last_error(void) { return nb2::last_error(); }

int nb2_device_open(int ordinal, nb2_device** out) {
    return guard([&] {
        need(out != nullptr, "null output pointer");
        *out = nb2::device(ordinal);
    });
}

int nb2_device_ordinal(const nb2_device* dev) { return dev ? dev->ordinal : -1; }

void* nb2_device_stream(nb2_device* dev) { return dev ? static_cast<void*>(dev->stream) : nullptr; }

int nb2_device_set_precision(nb2_device* dev, int precision) {
    return guard([&] {
        need(dev != nullptr, "null device");
        need(precision == NB2_PREC_3XTF32 || precision == NB2_PREC_1XTF32, "unknown precision");
        dev->precision = precision;
    });
}

int nb2_device_get_precision(const nb2_device* dev) { return dev ? dev->precision : -1; }

int nb2_device_set_wait_bound(nb2_device* dev, int64_t cycles) {
    return guard([&] {
        need(dev != nullptr, "null device");
        dev->wait_bound = cycles > 0 ? static_cast<long long>(cycles) : kDefaultWaitBoundCycles;
    });
}

int64_t nb2_device_get_wait_bound(const nb2_device* dev) { return dev ? dev->wait_bound : -1; }

int nb2_device_last_contraction(const nb2_device* dev, int* tile_n, int* two_in_flight, int* k_slices, int* a_mode,
                                int64_t* tiles) {
    return guard([&] {
        need(dev != nullptr, "null device");
        const nb2_device::Schedule& s = dev->last_sched;
        if (tile_n) {
            *tile_n = s.tile_n;
        }
        if (two_in_flight) {
            *two_in_flight = s.alt;
        }
        if (k_slices) {
            *k_slices = s.ksplit;
        }
        if (a_mode) {
            *a_mode = s.a_mode;
        }
        if (tiles) {
            *tiles = s.tiles;
        }
    });
}

int nb2_device_synchronize(nb2_device* dev) {
    return guard([&] {
        bind(dev);
        const int code = dev->take_device_error();
        if (code != 0) {
            fail(kStatusDevice, "a kernel reported device error " + std::to_string(code) +
                                    (code == 1 ? " (bounded wait expired)" : code == 2 ? " (index out of range)" : ""));
        }
    });
}

int nb2_pointer_on_device(const void* ptr) {
    if (ptr == nullptr) {
        return 0;
    }
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, ptr) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged || a.type == cudaMemoryTypeHost ? 1 : 0;
}

int nb2_device_malloc(nb2_device* dev, int64_t bytes, void** out) {
    return guard([&] {
        need(out != nullptr, "null output pointer");
        *out = nullptr;
        if (bytes <= 0) {
            return;
        }
        bind(dev);
        if (cudaMalloc(out, static_cast<size_t>(bytes)) != cudaSuccess) {
            cudaGetLastError();
            *out = nullptr;
            fail(kStatusNoMem, "cudaMalloc of " + std::to_string(bytes) + " bytes failed");
        }
    });
}

int nb2_device_free(nb2_device* dev, void* ptr) {
    return guard([&] {
        if (ptr == nullptr) {
            return;
        }
        bind(dev);
        check_cuda(cudaStreamSynchronize(dev->stream), "cudaStreamSynchronize");
        check_cuda(cudaFree(ptr), "cudaFree");
    });
}

int nb2_memcpy_h2d(nb2_device* dev, void* dst, const void* src, int64_t bytes) {
    return guard([&] {
        if (bytes == 0) {
            return;
        }
        need(bytes > 0 && dst != nullptr && src != nullptr, "h2d: bad arguments");
        bind(dev);
        std::lock_guard<std::mutex> lock(dev->mu);
        cudaPointerAttributes attr{};
        const bool known = cudaPointerGetAttributes(&attr, src) == cudaSuccess;
        if (!known) {
            cudaGetLastError();
        }
        if (!known || attr.type == cudaMemoryTypeUnregistered) {
            // pageable memory: the driver stages it through its own pinned
            // buffers, pipelined, and returns once `src` has been read
            check_cuda(cudaMemcpyAsync(dst, src, static_cast<size_t>(bytes), cudaMemcpyHostToDevice, dev->stream),
                       "cudaMemcpyAsync(H2D)");
            return;
        }
        // Pinned (or device-visible) memory would be read asynchronously:
        // chunked through our pinned buffer so the caller may free `src` as
        // soon as we return, while the copy stays ordered on the stream.
        const size_t chunk = 64u << 20;
        const auto* s = static_cast<const uint8_t*>(src);
        auto* d = static_cast<uint8_t*>(dst);
        size_t left = static_cast<size_t>(bytes);
        void* pin = HostStage::get(dev, std::min(left, chunk));
        while (left > 0) {
            const size_t n = std::min(left, chunk);
            check_cuda(cudaStreamSynchronize(dev->stream), "cudaStreamSynchronize");
            std::memcpy(pin, s, n);
            check_cuda(cudaMemcpyAsync(d, pin, n, cudaMemcpyHostToDevice, dev->stream), "cudaMemcpyAsync(H2D)");
            s += n;
            d += n;
            left -= n;
        }
        check_cuda(cudaStreamSynchronize(dev->stream), "cudaStreamSynchronize");
    });
}

int nb2_memcpy_d2h(nb2_device* dev, void* dst, const void* src, int64_t bytes) {
    return guard([&] {
        if (bytes == 0) {
            return;
        }
        need(bytes > 0 && dst != nullptr && src != nullptr, "d2h: bad arguments");
        bind(dev);
        check_cuda(cudaMemcpyAsync(dst, src, static_cast<size_t>(bytes), cudaMemcpyDeviceToHost, dev->stream),
                   "cudaMemcpyAsync(D2H)");
        const int code = dev->take_device_error();
        if (code != 0) {
            fail(kStatusDevice, "a kernel reported device error " + std::to_string(code));
        }
    });
}

int nb2_memcpy_d2d(nb2_device* dev, void* dst, const void* src, int64_t bytes) {
    return guard([&] {
        need(bytes >= 0, "d2d: negative size");
        bind(dev);
        nb2::copy(dev, src, dst, bytes);
    });
}

int nb2_conv2d_packed_size(const nb2_conv_geom* g, int64_t* bytes) {
    return guard([&] {
        need(bytes != nullptr, "null output pointer");
        *bytes = static_cast<int64_t>(conv_packed_bytes(nchw_input_layout(to_geom(g))));
    });
}

int nb2_conv2d_pack(nb2_device* dev, const nb2_conv_geom* g, const float* w, void* packed) {
    return guard([&] {
        const ConvGeom geom = nchw_input_layout(to_geom(g));
        need(w != nullptr && packed != nullptr, "Conv: null buffer");
        bind(dev);
        conv_pack(dev, geom, w, packed);
    });
}

int nb2_conv2d_run_packed(nb2_device* dev, const nb2_conv_geom* g, const float* x, const void* packed,
                          const float* bias, const float* residual, int act, float* y) {
    return guard([&] {
        const ConvGeom geom = nchw_input_layout(to_geom(g));
        need(x != nullptr && packed != nullptr && y != nullptr, "Conv: null buffer");
        bind(dev);
        Epilogue ep;
        ep.bias = bias;
        ep.res = residual;
        ep.act = act;
        run_nchw_conv(dev, geom, x, packed, y, ep, nullptr);
    });
}

int nb2_conv2d(nb2_device* dev, const nb2_conv_geom* g, const float* x, const float* w, const float* bias,
               const float* residual, int act, float* y) {
    return guard([&] {
        const ConvGeom plain = to_geom(g);
        need(x != nullptr && w != nullptr && y != nullptr, "Conv: null buffer");
        if (direct_conv_ok(plain)) {
            // narrow output (<= 32 channels): the CUDA-core direct kernel
            bind(dev);
            Epilogue ep;
            ep.bias = bias;
            ep.res = residual;
            ep.act = act;
            conv_direct(dev, plain, x, w, y, ep);
            return;
        }
        const ConvGeom geom = nchw_input_layout(plain);
        bind(dev);
        const size_t pbytes = (conv_packed_bytes(geom) + 255) & ~size_t(255);
        uint8_t* ws = static_cast<uint8_t*>(dev->scratch(pbytes + nhwc_copy_bytes(geom)));
        conv_pack(dev, geom, w, ws);
        Epilogue ep;
        ep.bias = bias;
        ep.res = residual;
        ep.act = act;
        run_nchw_conv(dev, geom, x, ws, y, ep, ws + pbytes);
    });
}

int nb2_conv_transpose2d(nb2_device* dev, const nb2_convt_geom* c, const float* x, const float* w,
                         const float* bias, float* y) {
    return guard([&] {
        need(c != nullptr, "ConvTranspose: null geometry");
        // the reference row's checks (src/kernels/conv_transpose.cpp:78-145)
        need(c->n > 0 && c->c > 0 && c->h > 0 && c->w > 0 && c->m > 0 && c->kh > 0 && c->kw > 0,
             "ConvTranspose: non-positive dimension");
        need(c->group > 0 && c->c % c->group == 0 && c->m % c->group == 0,
             "ConvTranspose: weight channels do not match the input and group");
        need(c->stride_h > 0 && c->stride_w > 0 && c->dil_h > 0 && c->dil_w > 0,
             "ConvTranspose: strides and dilations must be positive");
        need(c->pad_top >= 0 && c->pad_left >= 0 && c->pad_bottom >= 0 && c->pad_right >= 0 && c->out_pad_h >= 0 &&
                 c->out_pad_w >= 0,
             "ConvTranspose: pads and output_padding must be non-negative");
        const int64_t oh = c->stride_h * (c->h - 1) + c->out_pad_h + c->dil_h * (c->kh - 1) + 1 - c->pad_top -
                           c->pad_bottom;
        const int64_t ow = c->stride_w * (c->w - 1) + c->out_pad_w + c->dil_w * (c->kw - 1) + 1 - c->pad_left -
                           c->pad_right;
        need(oh > 0 && ow > 0 && oh == c->oh && ow == c->ow, "ConvTranspose: output shape does not match the transposed window");
        need(x != nullptr && w != nullptr && y != nullptr, "ConvTranspose: null buffer");
        bind(dev);
        const ConvTGeom t{c->n, c->c, c->h, c->w, c->m, c->kh, c->kw, c->oh, c->ow, c->stride_h, c->stride_w,
                          c->pad_top, c->pad_left, c->pad_bottom, c->pad_right, c->dil_h, c->dil_w,
                          c->out_pad_h, c->out_pad_w, c->group};
        const ConvGeom g = nchw_input_layout(convt_as_conv(t));
        auto al = [](size_t v) { return (v + 255) & ~size_t(255); };
        const size_t zb = al(convt_zero_insert_bytes(t));
        const size_t wb = al(static_cast<size_t>(t.M * (t.C / t.group) * t.KH * t.KW * 4));
        const size_t pb = al(conv_packed_bytes(g));
        uint8_t* ws = static_cast<uint8_t*>(dev->scratch(zb + wb + pb + nhwc_copy_bytes(g)));
        float* w2 = reinterpret_cast<float*>(ws + zb);
        convt_flip_weights(dev, t, w, w2);
        conv_pack(dev, g, w2, ws + zb + wb);
        const float* src = x;
        if (zb > 0) {
            convt_zero_insert(dev, t, x, reinterpret_cast<float*>(ws));
            src = reinterpret_cast<const float*>(ws);
        }
        Epilogue ep;
        ep.bias = bias;
        run_nchw_conv(dev, g, src, ws + zb + wb, y, ep, ws + zb + wb + pb);
    });
}

int nb2_gemm(nb2_device* dev, const float* a, const float* b, const float* c, int c_rank, float* y, int64_t m,
             int64_t n, int64_t k, int trans_a, int trans_b, float alpha, float beta, int act) {
    return guard([&] {
        need(m > 0 && n > 0 && k > 0, "Gemm: non-positive dimension");
        need(a != nullptr && b != nullptr && y != nullptr, "Gemm: null buffer");
        need(c_rank >= 0 && c_rank <= 2, "Gemm: bias shape must be [N] or [M,N]");
        need(c_rank == 0 || c != nullptr, "Gemm: null buffer");
        bind(dev);
        GemmGeom g{};
        g.M = m;
        g.N = n;
        g.K = k;
        g.trans_a = trans_a;
        g.trans_b = trans_b;
        g.lda = trans_a ? m : k;
        g.ldb = trans_b ? k : n;
        g.ldc = n;
        void* packed = dev->scratch(gemm_packed_bytes(g));
        gemm_pack_b(dev, g, b, packed);
        Epilogue ep;
        ep.alpha = alpha;
        if (c_rank == 1) {
            ep.bias = c;
            ep.bias_scale = beta;
        } else if (c_rank == 2) {
            ep.res = c;
            ep.res_scale = beta;
        }
        ep.act = act;
        gemm_run(dev, g, a, packed, y, ep);
    });
}

int nb2_gemm_packed_size(int64_t n, int64_t k, int64_t* bytes) {
    return guard([&] {
        need(n > 0 && k > 0 && bytes != nullptr, "Gemm: bad packed-size arguments");
        GemmGeom g{};
        g.N = n;
        g.K = k;
        g.batch = 1;
        *bytes = static_cast<int64_t>(gemm_packed_bytes(g));
    });
}

int nb2_gemm_pack(nb2_device* dev, const float* b, int64_t n, int64_t k, int trans_b, void* packed) {
    return guard([&] {
        need(n > 0 && k > 0, "Gemm: non-positive dimension");
        need(b != nullptr && packed != nullptr, "Gemm: null buffer");
        bind(dev);
        GemmGeom g{};
        g.N = n;
        g.K = k;
        g.batch = 1;
        g.trans_b = trans_b;
        g.ldb = trans_b ? k : n;
        gemm_pack_b(dev, g, b, packed);
    });
}

int nb2_gemm_run_packed(nb2_device* dev, const float* a, const void* packed_b, const float* c, int c_rank, float* y,
                        int64_t m, int64_t n, int64_t k, int trans_a, float alpha, float beta, int act) {
    return guard([&] {
        need(m > 0 && n > 0 && k > 0, "Gemm: non-positive dimension");
        need(a != nullptr && packed_b != nullptr && y != nullptr, "Gemm: null buffer");
        need(c_rank >= 0 && c_rank <= 2, "Gemm: bias shape must be [N] or [M,N]");
        need(c_rank == 0 || c != nullptr, "Gemm: null buffer");
        bind(dev);
        GemmGeom g{};
        g.M = m;
        g.N = n;
        g.K = k;
        g.batch = 1;
        g.trans_a = trans_a;
        g.lda = trans_a ? m : k;
        g.ldc = n;
        Epilogue ep;
        ep.alpha = alpha;
        if (c_rank == 1) {
            ep.bias = c;
            ep.bias_scale = beta;
        } else if (c_rank == 2) {
            ep.res = c;
            ep.res_scale = beta;
        }
        ep.act = act;
        gemm_run(dev, g, a, packed_b, y, ep);
    });
}

int nb2_matmul(nb2_device* dev, const float* a, const int64_t* a_dims, int a_rank, const float* b,
               const int64_t* b_dims, int b_rank, float* y) {
    return guard([&] {
        need(a_rank >= 1 && b_rank >= 1 && a_rank <= 8 && b_rank <= 8, "MatMul: operand rank must be 1..8");
        need(a != nullptr && b != nullptr && y != nullptr, "MatMul: null buffer");
        std::vector<int64_t> ad(a_dims, a_dims + a_rank), bd(b_dims, b_dims + b_rank);
        // 1-D promotion (src/kernels/mat_mul.cpp:79-169)
        if (ad.size() == 1) {
            ad.insert(ad.begin(), 1);
        }
        if (bd.size() == 1) {
            bd.push_back(1);
        }
        const int64_t M = ad[ad.size() - 2], K = ad.back();
        const int64_t K2 = bd[bd.size() - 2], N = bd.back();
        need(K == K2, "MatMul: contraction dimension mismatch");
        need(M > 0 && N > 0 && K > 0, "MatMul: non-positive dimension");
        std::vector<int64_t> abatch(ad.begin(), ad.end() - 2), bbatch(bd.begin(), bd.end() - 2);
        const size_t r = std::max(abatch.size(), bbatch.size());
        abatch.insert(abatch.begin(), r - abatch.size(), 1);
        bbatch.insert(bbatch.begin(), r - bbatch.size(), 1);
        int64_t batch = 1, a_count = 1, b_count = 1;
        for (size_t i = 0; i < r; ++i) {
            need(abatch[i] == bbatch[i] || abatch[i] == 1 || bbatch[i] == 1, "MatMul: batch dims do not broadcast");
            batch *= std::max(abatch[i], bbatch[i]);
            a_count *= abatch[i];
            b_count *= bbatch[i];
        }
        need((a_count == batch || a_count == 1) && (b_count == batch || b_count == 1),
             "MatMul: partial batch broadcasting is not supported");
        bind(dev);
        GemmGeom g{};
        g.N = N;
        g.K = K;
        g.trans_a = 0;
        g.trans_b = 0;
        g.lda = K;
        g.ldb = N;
        g.ldc = N;
        if (b_count == 1) {
            // B shared by every batch: fold the batch into M (one GEMM).
            g.M = M * batch;
            g.batch = 1;
        } else {
            g.M = M;
            g.batch = batch;
            g.a_zstride = a_count == 1 ? 0 : M * K;
            g.b_zstride = K * N;
            g.c_zstride = M * N;
        }
        void* packed = dev->scratch(gemm_packed_bytes(g));
        gemm_pack_b(dev, g, b, packed);
        gemm_run(dev, g, a, packed, y, Epilogue{});
    });
}

int nb2_unary(nb2_device* dev, int op, const float* x, float* y, int64_t count) {
    return guard([&] {
        need(count >= 0, "unary: negative count");
        need(op >= 0 && op <= kUGeluErf, "unary: unknown op");
        need(count == 0 || (x != nullptr && y != nullptr), "unary: null buffer");
        bind(dev);
        unary(dev, op, x, y, count);
    });
}

int nb2_binary(nb2_device* dev, int op, int dtype, const void* a, const int64_t* a_dims, int a_rank, const void* b,
               const int64_t* b_dims, int b_rank, void* y, const int64_t* y_dims, int y_rank) {
    return guard([&] {
        need(op >= 0 && op <= kBPow, "binary: unknown op");
        need(a_rank >= 0 && b_rank >= 0 && y_rank >= 0 && y_rank <= kMaxRank, "binary: bad rank");
        std::vector<int64_t> ad(a_dims, a_dims + a_rank), bd(b_dims, b_dims + b_rank), yd(y_dims, y_dims + y_rank);
        // the output must be the broadcast of the inputs
        const size_t r = std::max(ad.size(), bd.size());
        need(yd.size() == r, "binary: output rank does not match the broadcast");
        for (size_t i = 0; i < r; ++i) {
            const int64_t x1 = i + ad.size() >= r ? ad[i + ad.size() - r] : 1;
            const int64_t x2 = i + bd.size() >= r ? bd[i + bd.size() - r] : 1;
            need(x1 == x2 || x1 == 1 || x2 == 1, "binary: shapes do not broadcast");
            need(yd[i] == std::max(x1, x2), "binary: output shape does not match the broadcast");
        }
        bind(dev);
        binary(dev, op, dtype, a, ad, b, bd, y, yd);
    });
}

int nb2_maxpool2d(nb2_device* dev, const float* x, const int64_t x_dims[4], float* y, const int64_t y_dims[4],
                  const int64_t kernel[2], const int64_t strides[2], const int64_t pads[4],
                  const int64_t dilations[2]) {
    return guard([&] {
        PoolGeom g{x_dims[0], x_dims[1], x_dims[2], x_dims[3], y_dims[2], y_dims[3], kernel[0], kernel[1],
                   strides[0], strides[1], pads[0], pads[1], dilations[0], dilations[1]};
        need(y_dims[0] == g.N && y_dims[1] == g.C, "MaxPool: output shape does not match the pooling window");
        need(g.KH > 0 && g.KW > 0, "MaxPool: kernel dimensions must be positive");
        need(g.sh > 0 && g.sw > 0 && g.dh > 0 && g.dw > 0, "MaxPool: stride and dilation must be positive");
        need(x != nullptr && y != nullptr, "MaxPool: null buffer");
        bind(dev);
        maxpool2d(dev, g, x, y);
    });
}

int nb2_attention(nb2_device* dev, const float* q, const float* k, const float* v, float* out, int64_t batch,
                  int64_t heads, int64_t tokens, int64_t head_dim, const int64_t q_strides[4],
                  const int64_t k_strides[4], const int64_t v_strides[4], const int64_t out_strides[3],
                  int scale_mode, float scale) {
    return guard([&] {
        need(q && k && v && out && q_strides && k_strides && v_strides && out_strides, "Attention: null argument");
        need(batch >= 0 && heads >= 0, "Attention: negative dimension");
        need(head_dim == 64, "Attention: the fused kernel takes a head dimension of 64");
        need(tokens >= 1 && tokens <= kAttnMaxT, "Attention: between 1 and 208 tokens");
        need(scale_mode >= 0 && scale_mode <= 2, "Attention: scale_mode is 0, 1 or 2");
        need(scale_mode != 2 || scale != 0.0f, "Attention: division by zero scale");
        const AttnGeom g{batch,        heads,        tokens,       q_strides[0], q_strides[1], q_strides[2],
                         q_strides[3], k_strides[0], k_strides[1], k_strides[2], k_strides[3], v_strides[0],
                         v_strides[1], v_strides[2], v_strides[3], out_strides[0], out_strides[1],
                         out_strides[2], scale_mode,   scale};
        bind(dev);
        attention(dev, g, q, k, v, out);
    });
}

int nb2_sppf(nb2_device* dev, const float* x, const int64_t x_dims[4], float* y, int64_t k, int64_t chain) {
    return guard([&] {
        need(x_dims != nullptr && x != nullptr && y != nullptr, "SPPF: null argument");
        const SppfGeom g{x_dims[0], x_dims[1], x_dims[2], x_dims[3], k, chain};
        need(g.N >= 0 && g.C >= 0 && g.H >= 0 && g.W >= 0, "SPPF: negative dimension");
        need(k > 0 && k % 2 == 1 && chain >= 1, "SPPF: the window must be odd and the cascade at least one pool");
        need(g.H * g.W <= kSppfMaxPlane, "SPPF: plane larger than 6144 elements");
        bind(dev);
        sppf_nchw(dev, g, x, y);
    });
}

int nb2_avgpool2d(nb2_device* dev, const float* x, const int64_t x_dims[4], float* y, const int64_t y_dims[4],
                  const int64_t kernel[2], const int64_t strides[2], const int64_t pads[4], int count_include_pad) {
    return guard([&] {
        need(x_dims != nullptr && y_dims != nullptr && kernel != nullptr && strides != nullptr && pads != nullptr,
             "AveragePool: null argument");
        AvgPoolGeom g{x_dims[0], x_dims[1], x_dims[2], x_dims[3], y_dims[2], y_dims[3], kernel[0], kernel[1],
                      strides[0], strides[1], pads[0], pads[1], pads[2], pads[3], count_include_pad ? 1 : 0};
        need(g.N > 0 && g.C > 0 && g.H > 0 && g.W > 0, "AveragePool: non-positive dimension");
        need(g.KH > 0 && g.KW > 0 && g.sh > 0 && g.sw > 0, "AveragePool: kernel and stride must be positive");
        need(g.pt >= 0 && g.pl >= 0 && g.pb >= 0 && g.pr >= 0, "AveragePool: pads must be non-negative");
        need(y_dims[0] == g.N && y_dims[1] == g.C && g.OH > 0 && g.OW > 0,
             "AveragePool: output shape does not match the pooling window");
        need(x != nullptr && y != nullptr, "AveragePool: null buffer");
        bind(dev);
        avgpool2d(dev, g, x, y);
    });
}

int nb2_row_mean(nb2_device* dev, const float* x, int64_t rows, int64_t inner, float* y) {
    return guard([&] {
        need(rows >= 0 && inner > 0, "mean: bad extents");
        need(rows == 0 || (x != nullptr && y != nullptr), "mean: null buffer");
        bind(dev);
        row_mean(dev, x, y, rows, inner);
    });
}

int nb2_softmax(nb2_device* dev, const float* x, float* y, int64_t outer, int64_t len, int64_t inner) {
    return guard([&] {
        need(outer >= 0 && len >= 0 && inner >= 0, "Softmax: negative extent");
        need(outer * len * inner == 0 || (x != nullptr && y != nullptr), "Softmax: null buffer");
        bind(dev);
        softmax(dev, x, y, outer, len, inner);
    });
}

int nb2_layernorm(nb2_device* dev, const float* x, const float* scale, const float* bias, float* y, float* mean,
                  float* inv_std, int64_t rows, int64_t d, float epsilon) {
    return guard([&] {
        need(rows >= 0 && d > 0, "LayerNormalization: bad extents");
        need(rows == 0 || (x != nullptr && scale != nullptr && y != nullptr), "LayerNormalization: null buffer");
        bind(dev);
        layernorm(dev, x, scale, bias, y, mean, inv_std, rows, d, epsilon);
    });
}

int nb2_transpose(nb2_device* dev, const void* x, void* y, const int64_t* dims, const int64_t* perm, int rank,
                  int elem_bytes) {
    return guard([&] {
        need(rank >= 0 && rank <= 8, "Transpose: rank must be 0..8");
        need(elem_bytes == 1 || elem_bytes == 4 || elem_bytes == 8, "Transpose: element size must be 1, 4 or 8");
        std::vector<int64_t> d(dims, dims + rank), p(perm, perm + rank);
        std::vector<bool> seen(static_cast<size_t>(rank), false);
        for (int64_t a : p) {
            need(a >= 0 && a < rank && !seen[static_cast<size_t>(a)], "Transpose: perm is not a permutation");
            seen[static_cast<size_t>(a)] = true;
        }
        bind(dev);
        transpose(dev, x, y, d, p, elem_bytes);
    });
}

int nb2_concat_split(nb2_device* dev, int concat, void* whole, void* const* parts, const int64_t* parts_len,
                     int n_parts, int64_t outer, int64_t inner, int elem_bytes) {
    return guard([&] {
        need(n_parts > 0 && outer >= 0 && inner >= 0 && elem_bytes > 0, "Concat/Split: bad extents");
        int64_t total = 0;
        for (int i = 0; i < n_parts; ++i) {
            need(parts_len[i] >= 0, "Concat/Split: negative part length");
            total += parts_len[i];
        }
        const int64_t pitch = total * inner * elem_bytes;
        std::vector<CopySeg> segs;
        int64_t at = 0;
        for (int i = 0; i < n_parts; ++i) {
            const int64_t rb = parts_len[i] * inner * elem_bytes;
            auto* w = static_cast<uint8_t*>(whole) + at;
            auto* p = static_cast<uint8_t*>(parts[i]);
            segs.push_back(concat ? CopySeg{p, w, rb, pitch, rb, outer} : CopySeg{w, p, pitch, rb, rb, outer});
            at += rb;
        }
        bind(dev);
        segment_copy(dev, segs);
    });
}

int nb2_slice(nb2_device* dev, const void* x, void* y, const int64_t* in_dims, const int64_t* out_dims,
              const int64_t* starts, const int64_t* steps, int rank, int elem_bytes) {
    return guard([&] {
        need(rank >= 1 && rank <= 8, "Slice: rank must be 1..8");
        bind(dev);
        slice(dev, x, y, std::vector<int64_t>(in_dims, in_dims + rank), std::vector<int64_t>(out_dims, out_dims + rank),
              std::vector<int64_t>(starts, starts + rank), std::vector<int64_t>(steps, steps + rank), elem_bytes);
    });
}

int nb2_gather(nb2_device* dev, const void* x, const int64_t* indices, void* y, int64_t outer, int64_t axis_len,
               int64_t inner, int64_t n_indices, int elem_bytes) {
    return guard([&] {
        need(outer >= 0 && axis_len >= 0 && inner >= 0 && n_indices >= 0, "Gather: negative extent");
        bind(dev);
        gather(dev, x, indices, y, outer, axis_len, inner, n_indices, elem_bytes);
    });
}

int nb2_topk(nb2_device* dev, const float* x, float* values, int64_t* indices, int64_t rows, int64_t len, int64_t k) {
    return guard([&] {
        need(rows >= 0 && len >= 0 && k >= 0, "TopK: negative extent");
        need(k <= len, "TopK: K is larger than the axis");
        bind(dev);
        const size_t sb = topk_scratch_bytes(rows, len, k);
        topk(dev, x, values, indices, rows, len, k, sb ? dev->scratch(sb) : nullptr);
    });
}

int nb2_resize(nb2_device* dev, const void* x, void* y, const int64_t* in_dims, const int64_t* out_dims,
               const double* scales, int rank, int mode, int transform, int nearest_mode, int dtype) {
    return guard([&] {
        need(rank >= 1 && rank <= 8, "Resize: rank must be 1..8");
        need(mode == 0 || mode == 1, "Resize: mode must be nearest (0) or linear (1)");
        need(transform >= 0 && transform <= 3 && nearest_mode >= 0 && nearest_mode <= 3, "Resize: unknown mode");
        need(dtype == NB2_F32 || (dtype == NB2_I64 && mode == 0), "Resize: tensors must be float32 (or int64 for nearest)");
        std::vector<int64_t> in(in_dims, in_dims + rank), out(out_dims, out_dims + rank);
        for (int d = 0; d < rank; ++d) {
            need(in[d] > 0 && out[d] > 0, "Resize: non-positive dimension");
        }
        bind(dev);
        void* tables = dev->scratch(resize_table_bytes(out));
        resize_on_device_tables(dev, x, y, in, out, std::vector<double>(scales, scales + rank), mode, transform,
                                nearest_mode, dtype == NB2_F32, tables);
    });
}

int nb2_cast(nb2_device* dev, const void* x, int from_dtype, void* y, int to_dtype, int64_t count) {
    return guard([&] {
        need(from_dtype >= 0 && from_dtype <= 2 && to_dtype >= 0 && to_dtype <= 2, "Cast: unknown dtype");
        need(count >= 0, "Cast: negative count");
        bind(dev);
        cast(dev, x, from_dtype, y, to_dtype, count);
    });
}

} // extern "C"
