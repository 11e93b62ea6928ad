// ConvTranspose on the tensor-core Conv engine.
//
// Reference row: src/kernels/conv_transpose.cpp (input [N,C,H,W], weight
// [C, M/group, KH, KW], explicit pads, output_padding, dilations, groups; out
// size s*(in-1) + output_padding + d*(k-1) + 1 - pad_begin - pad_end; a float32
// scatter). Here it is the equivalent gather: the input with s-1 zeros inserted
// between neighbours (when s > 1), then an ordinary stride-1 Conv with the
// weight transposed per group and flipped in both spatial axes, dilation d and
// pads d*(k-1) - pad_begin (begin) and d*(k-1) - pad_end + output_padding (end).
// Pads above d*(k-1) (which would crop) are rejected.

#include "igemm.cuh"
#include "ops.cuh"

namespace nb2 {

namespace {

// xz[nc][r][c] = x[nc][r / sh][c / sw] where both divide, else 0.
__global__ void zero_insert_kernel(const float* __restrict__ x, float* __restrict__ xz, int64_t H, int64_t W,
                                   int64_t Hz, int64_t Wz, int sh, int sw, int64_t total) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t c = i % Wz;
        const int64_t t = i / Wz;
        const int64_t r = t % Hz;
        const int64_t nc = t / Hz;
        float v = 0.0f;
        if (r % sh == 0 && c % sw == 0) {
            v = __ldg(x + (nc * H + r / sh) * W + c / sw);
        }
        xz[i] = v;
    }
}

// w2[g*Mg + m][c][kh][kw] = w[g*Cg + c][m][KH-1-kh][KW-1-kw]
__global__ void flip_weights_kernel(const float* __restrict__ w, float* __restrict__ w2, int64_t Cg, int64_t Mg,
                                    int64_t KH, int64_t KW, int64_t total) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t kw = i % KW;
        int64_t t = i / KW;
        const int64_t kh = t % KH;
        t /= KH;
        const int64_t c = t % Cg;
        t /= Cg; // g * Mg + m
        const int64_t m = t % Mg, g = t / Mg;
        w2[i] = __ldg(w + (((g * Cg + c) * Mg + m) * KH + (KH - 1 - kh)) * KW + (KW - 1 - kw));
    }
}

unsigned blocks_of(nb2_device* dev, int64_t n) {
    return static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, dev->num_sms * 32)));
}

} // namespace

ConvGeom convt_as_conv(const ConvTGeom& t) {
    if (t.ph > t.dh * (t.KH - 1) || t.pb > t.dh * (t.KH - 1) || t.pw > t.dw * (t.KW - 1) ||
        t.pr > t.dw * (t.KW - 1)) {
        fail(kStatusUnsupported, "ConvTranspose: pads larger than dilation*(kernel-1) are not supported on B200");
    }
    ConvGeom g{};
    g.N = t.N;
    g.C = t.C;
    g.H = (t.H - 1) * t.sh + 1;
    g.W = (t.W - 1) * t.sw + 1;
    g.M = t.M;
    g.KH = t.KH;
    g.KW = t.KW;
    g.OH = t.OH;
    g.OW = t.OW;
    g.sh = 1;
    g.sw = 1;
    g.ph = t.dh * (t.KH - 1) - t.ph;
    g.pw = t.dw * (t.KW - 1) - t.pw;
    g.pb = t.dh * (t.KH - 1) - t.pb + t.oph;
    g.pr = t.dw * (t.KW - 1) - t.pr + t.opw;
    g.dh = t.dh;
    g.dw = t.dw;
    g.group = t.group;
    return g;
}

size_t convt_zero_insert_bytes(const ConvTGeom& t) {
    if (t.sh == 1 && t.sw == 1) {
        return 0;
    }
    return static_cast<size_t>(t.N * t.C * ((t.H - 1) * t.sh + 1) * ((t.W - 1) * t.sw + 1) * 4);
}

void convt_zero_insert(nb2_device* dev, const ConvTGeom& t, const float* x, float* xz) {
    const int64_t Hz = (t.H - 1) * t.sh + 1, Wz = (t.W - 1) * t.sw + 1;
    const int64_t total = t.N * t.C * Hz * Wz;
    zero_insert_kernel<<<blocks_of(dev, total), 256, 0, dev->stream>>>(x, xz, t.H, t.W, Hz, Wz,
                                                                       static_cast<int>(t.sh),
                                                                       static_cast<int>(t.sw), total);
    check_cuda(cudaGetLastError(), "zero_insert launch");
}

void convt_flip_weights(nb2_device* dev, const ConvTGeom& t, const float* w, float* w2) {
    const int64_t Cg = t.C / t.group, Mg = t.M / t.group;
    const int64_t total = t.M * Cg * t.KH * t.KW;
    flip_weights_kernel<<<blocks_of(dev, total), 256, 0, dev->stream>>>(w, w2, Cg, Mg, t.KH, t.KW, total);
    check_cuda(cudaGetLastError(), "flip_weights launch");
}

} // namespace nb2
