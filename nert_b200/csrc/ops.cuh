// Bandwidth-bound rows of the B200 layer (elementwise, pooling, reductions,
// normalisation, data movement, selection). All launch on the device's
// stream and return without synchronising.
#pragma once

#include "runtime.hpp"

#include <cstdint>
#include <vector>

namespace nb2 {

enum UnaryOp : int {
    kURelu = 0,
    kUSigmoid = 1,
    kUErf = 2,
    kUSqrt = 3,
    kUNeg = 4,
    kUAbs = 5,
    kUExp = 6,
    kUTanh = 7,
    kUIdentity = 8,
    kUSilu = 9,
    kUGeluErf = 10, // 0.5*x*(1+erf(x/sqrt(2))) — the fused form of the Erf chain
};

enum BinaryOp : int { kBAdd = 0, kBSub = 1, kBMul = 2, kBDiv = 3, kBPow = 4 };

// dtype codes shared with the C ABI
enum Dtype : int { kF32 = 0, kI64 = 1, kBool = 2 };

constexpr int kMaxRank = 8;

void unary(nb2_device* dev, int op, const float* x, float* y, int64_t n);
// y[o][c][i] = x[o][c][i] * a[c] + b[c] over an [outer, C, inner] view: an
// inference BatchNormalization whose scale and shift were folded on the host.
void channel_affine(nb2_device* dev, const float* x, const float* a, const float* b, float* y, int64_t outer,
                    int64_t C, int64_t inner);
// y = a (op) b with NumPy broadcasting; a/b/y dims given explicitly.
void binary(nb2_device* dev, int op, int dtype, const void* a, const std::vector<int64_t>& ad, const void* b,
            const std::vector<int64_t>& bd, void* y, const std::vector<int64_t>& yd);
void copy(nb2_device* dev, const void* src, void* dst, int64_t bytes);

struct PoolGeom {
    int64_t N, C, H, W, OH, OW, KH, KW, sh, sw, ph, pw, dh, dw;
};
void maxpool2d(nb2_device* dev, const PoolGeom& g, const float* x, float* y);
// AveragePool 2-D (src/kernels/average_pool.cpp): begin pads (pt, pl), end
// pads (pb, pr); include_pad selects count_include_pad.
struct AvgPoolGeom {
    int64_t N, C, H, W, OH, OW, KH, KW, sh, sw, pt, pl, pb, pr;
    int include_pad;
};
void avgpool2d(nb2_device* dev, const AvgPoolGeom& g, const float* x, float* y);
// Fused attention out = Softmax(scale(Q K^T)) V per (batch, head) with head
// dim 64 and T <= kAttnMaxT tokens; element (token t, dim j) of head (b, h)
// sits at b*xb + h*xh + t*xt + j*xj for x = q, k, v; the output row at
// b*ob + h*oh + t*ot with its 64 values contiguous. scale_mode: 0 none,
// 1 multiply by `scale`, 2 divide by `scale` (the graph's Mul / Div).
constexpr int64_t kAttnMaxT = 208;
struct AttnGeom {
    int64_t B, H, T;
    int64_t qb, qh, qt, qj;
    int64_t kb, kh, kt, kj;
    int64_t vb, vh, vt, vj;
    int64_t ob, oh, ot;
    int scale_mode;
    float scale;
};
void attention(nb2_device* dev, const AttnGeom& g, const float* q, const float* k, const float* v, float* out);
size_t attention_smem_bytes(int T);
// SPPF: y[n] = Concat over axis 1 of [x, m1, ..., m_chain] with m_l the
// k x k, stride-1, pad k/2 MaxPool of m_{l-1} (m0 = x); x is [N][C][H][W] and
// y [N][(chain+1)*C][H][W]. One read of each plane, kept in shared memory
// (H*W <= kSppfMaxPlane) while the cascade runs.
constexpr int64_t kSppfMaxPlane = 6144;
struct SppfGeom {
    int64_t N, C, H, W, k, chain;
};
void sppf_nchw(nb2_device* dev, const SppfGeom& g, const float* x, float* y);
// The same window over channels-last x[N][H][W][C] -> y[N][OH][OW][C].
void maxpool2d_nhwc(nb2_device* dev, const PoolGeom& g, const float* x, float* y);
// y[n][c] = mean over the hw pixels of channels-last x[n][hw][c]
void mean_nhwc(nb2_device* dev, const float* x, float* y, int64_t n, int64_t hw, int64_t c);
// x[N][C][H][W] -> y[N][H][W][Cp], channels zero padded to Cp (4, 8, 16 or a
// multiple of 32): the input forms of the narrow-channel and TMA im2col Conv
// paths for tensors that arrive NCHW.
void nchw_to_nhwc_pad(nb2_device* dev, const float* x, float* y, int64_t N, int64_t C, int64_t H, int64_t W,
                      int64_t Cp);
// mean over the trailing `inner` elements of each of `rows` rows
void row_mean(nb2_device* dev, const float* x, float* y, int64_t rows, int64_t inner);

} // namespace nb2
