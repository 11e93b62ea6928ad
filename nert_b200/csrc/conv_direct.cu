// Direct convolution on the CUDA cores for narrow outputs.
//
// Reference row: src/kernels/conv.cpp:138-295 (NCHW in and out, the sum over
// input channels and filter taps per output element, bias added). A layer
// with at most 32 output channels (YOLO's 16- and 32-channel layers at
// 320x320 and 160x160, its DFL 1x1 with one output channel) leaves most of a
// 64-wide tensor-core tile empty and does a handful of FLOPs per byte: it is
// bound by reading its input and writing its output. Here a thread owns one
// output pixel and all M <= 32 output channels in registers, reads each of
// its C x KH x KW input taps once (neighbouring threads share them through
// L1) and multiplies by the weights broadcast from shared memory; the sum runs
// in fp32 FMAs in (channel, kh, kw) order, the reference's loop order, with
// exact fp32 products. The engine's fused epilogue (bias, residual Add,
// activation) is applied before the one store per output.

#include "igemm.cuh"
#include "ops.cuh"

namespace nb2 {

namespace {

constexpr int kDirectThreads = 128;
// shared weights: C*KH*KW rows of MT floats
constexpr int64_t kDirectSmemFloats = 12288;

struct DirectArgs {
    const float* x;
    const float* w; // [M][C][KH][KW]
    float* y;
    const float* bias;
    const float* res;
    int C, H, W, M, KH, KW, OH, OW, sh, sw, ph, pw, dh, dw;
    float alpha, bias_scale, res_scale;
    int act;
    float act_a, act_b, act_c;
};

template <int ACT>
__device__ __forceinline__ float direct_act(float v, const DirectArgs& a) {
    if constexpr (ACT == kActRelu) {
        return v > 0.0f ? v : 0.0f;
    } else if constexpr (ACT == kActSilu) {
        return v * (1.0f / (1.0f + expf(-v)));
    } else if constexpr (ACT == kActSigmoid) {
        return 1.0f / (1.0f + expf(-v));
    } else if constexpr (ACT == kActGeluErf) {
        return (v * (erff(v / a.act_a) + a.act_b)) * a.act_c;
    } else {
        return v;
    }
}

template <int MT, int ACT>
__device__ __forceinline__ void direct_store(const DirectArgs& a, const float (&acc)[MT], float* yn, const float* rn,
                                             int opix) {
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        if (m < a.M) {
            const float bb = a.bias ? a.bias_scale * __ldg(a.bias + m) : 0.0f;
            const float rv = rn ? __ldg(rn + (int64_t)m * opix) : 0.0f;
            yn[(int64_t)m * opix] = direct_act<ACT>(fmaf(a.res_scale, rv, fmaf(a.alpha, acc[m], bb)), a);
        }
    }
}

// The taps of one input channel for KT x KT filters (KT = 1 or 3, known at
// compile time and unrolled) or any filter (KT = 0); BOUNDED = false when the
// whole window lies inside the input (no per-tap test).
template <int MT, int KT, bool BOUNDED>
__device__ __forceinline__ void direct_channel(const DirectArgs& a, const float* xc, const float4* w4, int c, int ih0,
                                               int iw0, float (&acc)[MT]) {
    const int KH = KT ? KT : a.KH, KW = KT ? KT : a.KW;
#pragma unroll
    for (int kh = 0; kh < KH; ++kh) {
        const int ih = ih0 + kh * a.dh;
        const bool hok = !BOUNDED || (ih >= 0 && ih < a.H);
        const int krow = (c * KH + kh) * KW;
        const float* xr = xc + (int64_t)ih * a.W;
#pragma unroll
        for (int kw = 0; kw < KW; ++kw) {
            const int iw = iw0 + kw * a.dw;
            const float xv = (!BOUNDED || (hok && iw >= 0 && iw < a.W)) ? __ldg(xr + iw) : 0.0f;
            const float4* wk = w4 + (krow + kw) * (MT / 4);
#pragma unroll
            for (int q = 0; q < MT / 4; ++q) {
                const float4 wv = wk[q];
                acc[4 * q] = fmaf(wv.x, xv, acc[4 * q]);
                acc[4 * q + 1] = fmaf(wv.y, xv, acc[4 * q + 1]);
                acc[4 * q + 2] = fmaf(wv.z, xv, acc[4 * q + 2]);
                acc[4 * q + 3] = fmaf(wv.w, xv, acc[4 * q + 3]);
            }
        }
    }
}

template <int MT, int KT>
__global__ void __launch_bounds__(kDirectThreads) conv_direct_kernel(const __grid_constant__ DirectArgs a) {
    extern __shared__ float4 direct_smem4[];
    float* ws = reinterpret_cast<float*>(direct_smem4); // ws[(c*KH + kh)*KW + kw][m], MT per row
    const int taps = a.C * a.KH * a.KW;
    for (int i = threadIdx.x; i < taps * MT; i += blockDim.x) {
        const int k = i / MT, m = i - k * MT;
        ws[i] = m < a.M ? __ldg(a.w + (int64_t)m * taps + k) : 0.0f;
    }
    __syncthreads();
    const int n = blockIdx.y;
    const int p = blockIdx.x * kDirectThreads + threadIdx.x;
    const int opix = a.OH * a.OW;
    if (p >= opix) {
        return;
    }
    const int oh = p / a.OW, ow = p - oh * a.OW;
    const int ih0 = oh * a.sh - a.ph, iw0 = ow * a.sw - a.pw;
    const float* xn = a.x + (int64_t)n * a.C * a.H * a.W;
    float acc[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        acc[m] = 0.0f;
    }
    const float4* w4 = reinterpret_cast<const float4*>(ws);
    // a window wholly inside the input (most pixels) skips the per-tap tests
    const bool inside = ih0 >= 0 && ih0 + (a.KH - 1) * a.dh < a.H && iw0 >= 0 && iw0 + (a.KW - 1) * a.dw < a.W;
    if (inside) {
        for (int c = 0; c < a.C; ++c) {
            direct_channel<MT, KT, false>(a, xn + (int64_t)c * a.H * a.W, w4, c, ih0, iw0, acc);
        }
    } else {
        for (int c = 0; c < a.C; ++c) {
            direct_channel<MT, KT, true>(a, xn + (int64_t)c * a.H * a.W, w4, c, ih0, iw0, acc);
        }
    }
    float* yn = a.y + (int64_t)n * a.M * opix + p;
    const float* rn = a.res ? a.res + (int64_t)n * a.M * opix + p : nullptr;
    switch (a.act) {
    case kActRelu:
        direct_store<MT, kActRelu>(a, acc, yn, rn, opix);
        break;
    case kActSilu:
        direct_store<MT, kActSilu>(a, acc, yn, rn, opix);
        break;
    case kActSigmoid:
        direct_store<MT, kActSigmoid>(a, acc, yn, rn, opix);
        break;
    case kActGeluErf:
        direct_store<MT, kActGeluErf>(a, acc, yn, rn, opix);
        break;
    default:
        direct_store<MT, kActNone>(a, acc, yn, rn, opix);
        break;
    }
}

int direct_width(int64_t M) { return M <= 4 ? 4 : (M <= 8 ? 8 : (M <= 16 ? 16 : 32)); }

template <int MT, int KT>
void launch_direct(dim3 grid, size_t smem, nb2_device* dev, const DirectArgs& a) {
    conv_direct_kernel<MT, KT><<<grid, kDirectThreads, smem, dev->stream>>>(a);
}

} // namespace

bool direct_conv_ok(const ConvGeom& g) {
    if (g.group != 1 || g.M > 32 || g.in_nhwc || g.out_nhwc || g.cvec || g.cpad) {
        return false;
    }
    const int64_t taps = g.C * g.KH * g.KW;
    // Only where a pixel needs few multiply-adds (taps x M <= 2560): there the
    // layer is bound by its bytes and this kernel beats the tensor-core tile
    // (measured at YOLO b16: the 3->16 3x3/2 stem 396 -> 125 µs, the 1-channel
    // DFL 1x1 84 -> under 10 µs); at 4608 and more (16->32 3x3, 32->32 3x3) the
    // CUDA-core FMAs are the limit and the tensor cores win.
    // (end padding needs nothing: taps outside the input read as zero)
    return taps * g.M <= 2560 && taps * direct_width(g.M) <= kDirectSmemFloats && g.N <= 65535 &&
           g.OH * g.OW < (int64_t(1) << 31) && g.C * g.H * g.W < (int64_t(1) << 31);
}

void conv_direct(nb2_device* dev, const ConvGeom& g, const float* x, const float* w, float* y, const Epilogue& ep) {
    if (!direct_conv_ok(g)) {
        fail(kStatusUnsupported, "Conv: geometry outside the direct (CUDA-core) path");
    }
    if (g.N == 0 || g.OH * g.OW == 0 || g.M == 0) {
        return;
    }
    DirectArgs a{};
    a.x = x;
    a.w = w;
    a.y = y;
    a.bias = ep.bias;
    a.res = ep.res;
    a.C = static_cast<int>(g.C), a.H = static_cast<int>(g.H), a.W = static_cast<int>(g.W);
    a.M = static_cast<int>(g.M), a.KH = static_cast<int>(g.KH), a.KW = static_cast<int>(g.KW);
    a.OH = static_cast<int>(g.OH), a.OW = static_cast<int>(g.OW);
    a.sh = static_cast<int>(g.sh), a.sw = static_cast<int>(g.sw), a.ph = static_cast<int>(g.ph);
    a.pw = static_cast<int>(g.pw), a.dh = static_cast<int>(g.dh), a.dw = static_cast<int>(g.dw);
    a.alpha = ep.alpha, a.bias_scale = ep.bias_scale, a.res_scale = ep.res_scale;
    a.act = ep.act, a.act_a = ep.act_a, a.act_b = ep.act_b, a.act_c = ep.act_c;
    const int mt = direct_width(g.M);
    const size_t smem = static_cast<size_t>(g.C * g.KH * g.KW * mt) * sizeof(float);
    const dim3 grid(static_cast<unsigned>((g.OH * g.OW + kDirectThreads - 1) / kDirectThreads),
                    static_cast<unsigned>(g.N));
    // 1x1 and 3x3 filters unrolled at compile time, any other shape generic
    const int kt = (g.KH == 1 && g.KW == 1) ? 1 : ((g.KH == 3 && g.KW == 3) ? 3 : 0);
    switch (mt * 10 + kt) {
    case 40: launch_direct<4, 0>(grid, smem, dev, a); break;
    case 41: launch_direct<4, 1>(grid, smem, dev, a); break;
    case 43: launch_direct<4, 3>(grid, smem, dev, a); break;
    case 80: launch_direct<8, 0>(grid, smem, dev, a); break;
    case 81: launch_direct<8, 1>(grid, smem, dev, a); break;
    case 83: launch_direct<8, 3>(grid, smem, dev, a); break;
    case 160: launch_direct<16, 0>(grid, smem, dev, a); break;
    case 161: launch_direct<16, 1>(grid, smem, dev, a); break;
    case 163: launch_direct<16, 3>(grid, smem, dev, a); break;
    case 320: launch_direct<32, 0>(grid, smem, dev, a); break;
    case 321: launch_direct<32, 1>(grid, smem, dev, a); break;
    default: launch_direct<32, 3>(grid, smem, dev, a); break;
    }
    check_cuda(cudaGetLastError(), "conv_direct launch");
}

} // namespace nb2
