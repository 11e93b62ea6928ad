// Pooling rows: MaxPool 2-D and spatial means (GlobalAveragePool / the
// ReduceMean form of global pooling).
//
// Reference semantics: MaxPool takes the max over in-range taps only, -inf when
// none is in range (src/kernels/max_pool.cpp:207-235); GlobalAveragePool sums
// in double and divides by the spatial size (global_average_pool.cpp:59-67).
// The reference CUDA rows use one thread per output / per row
// (src/cuda/max_pool.cu:101-128, global_average_pool.cu:36-44).

#include "ops.cuh"

#include <cfloat>

namespace nb2 {

namespace {

// One thread per output element, consecutive threads along the output row so
// the window reads of a warp stay within a few cache lines.
__global__ void maxpool2d_kernel(const float* __restrict__ x, float* __restrict__ y, PoolGeom g, int64_t total) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t ow = i % g.OW;
        int64_t t = i / g.OW;
        const int64_t oh = t % g.OH;
        t /= g.OH; // n*C + c
        const float* plane = x + t * g.H * g.W;
        const int64_t h0 = oh * g.sh - g.ph;
        const int64_t w0 = ow * g.sw - g.pw;
        float best = -INFINITY;
        for (int64_t kh = 0; kh < g.KH; ++kh) {
            const int64_t ih = h0 + kh * g.dh;
            if (ih < 0 || ih >= g.H) {
                continue;
            }
            const float* row = plane + ih * g.W;
            for (int64_t kw = 0; kw < g.KW; ++kw) {
                const int64_t iw = w0 + kw * g.dw;
                if (iw < 0 || iw >= g.W) {
                    continue;
                }
                const float v = __ldg(row + iw);
                if (v > best) {
                    best = v;
                }
            }
        }
        y[i] = best;
    }
}

// NCHW max pool over a fixed KH x KW window without dilation (YOLO's SPPF
// 5x5/1): 32-bit indices, all taps' loads issued together (an out-of-image
// tap reads as -inf, which never wins the comparison the generic kernel
// makes); neighbouring threads share their windows through L1.
template <int KH, int KW>
__global__ void maxpool2d_fixed_kernel(const float* __restrict__ x, float* __restrict__ y, int H, int W, int OH,
                                       int OW, int sh, int sw, int ph, int pw, uint32_t total) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const int ow = static_cast<int>(i % OW);
        const uint32_t t = i / OW;
        const int oh = static_cast<int>(t % OH);
        const float* plane = x + (size_t)(t / OH) * H * W;
        const int h0 = oh * sh - ph, w0 = ow * sw - pw;
        float v[KH * KW];
#pragma unroll
        for (int kh = 0; kh < KH; ++kh) {
#pragma unroll
            for (int kw = 0; kw < KW; ++kw) {
                const int ih = h0 + kh, iw = w0 + kw;
                v[kh * KW + kw] = ((unsigned)ih < (unsigned)H && (unsigned)iw < (unsigned)W)
                                      ? __ldg(plane + ih * W + iw)
                                      : -INFINITY;
            }
        }
        float best = -INFINITY;
#pragma unroll
        for (int k = 0; k < KH * KW; ++k) {
            best = v[k] > best ? v[k] : best;
        }
        y[i] = best;
    }
}

// Warp per row, double accumulation, for short rows (e.g. 7x7 = 49).
__global__ void row_mean_warp_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t rows, int64_t inner) {
    const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= rows) {
        return;
    }
    const float* r = x + warp * inner;
    double s = 0.0;
    for (int64_t k = lane; k < inner; k += 32) {
        s += static_cast<double>(__ldg(r + k));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        s += __shfl_xor_sync(0xffffffffu, s, o);
    }
    if (lane == 0) {
        y[warp] = static_cast<float>(s / static_cast<double>(inner));
    }
}

// Short rows (inner <= 64, e.g. 7x7 = 49): a block stages 128 whole rows
// (one contiguous span of the input) in shared memory with 16-byte loads, then
// each thread sums one row in double. Rows of 49 floats break 16-byte
// alignment row by row, so a warp per row would issue short, misaligned loads.
constexpr int kMeanRows = 128;
constexpr int kMeanInner = 64;
__global__ void __launch_bounds__(kMeanRows) row_mean_staged_kernel(const float* __restrict__ x,
                                                                    float* __restrict__ y, int64_t rows,
                                                                    int inner) {
    __shared__ __align__(16) float sm[kMeanRows * kMeanInner];
    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kMeanRows;
    const int64_t left = rows - r0;
    const int nrows = left < kMeanRows ? static_cast<int>(left) : kMeanRows;
    const int n = nrows * inner;
    const float* src = x + r0 * inner;
    const int n4 = ((reinterpret_cast<uintptr_t>(src) & 15) == 0) ? n / 4 : 0;
    const float4* s4 = reinterpret_cast<const float4*>(src);
    float4* d4 = reinterpret_cast<float4*>(sm);
    // every 16-byte load of the thread (at most 16) in flight before the
    // shared stores
    constexpr int kPer = kMeanRows * kMeanInner / 4 / kMeanRows;
    float4 v[kPer];
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        const int i4 = threadIdx.x + j * kMeanRows;
        if (i4 < n4) {
            v[j] = __ldg(s4 + i4);
        }
    }
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        const int i4 = threadIdx.x + j * kMeanRows;
        if (i4 < n4) {
            d4[i4] = v[j];
        }
    }
    for (int i = n4 * 4 + threadIdx.x; i < n; i += blockDim.x) {
        sm[i] = __ldg(src + i);
    }
    __syncthreads();
    if (threadIdx.x < nrows) {
        const float* row = sm + threadIdx.x * inner;
        double acc = 0.0;
        if (inner & 1) {
            // odd row strides put the lanes on distinct banks: sum in order
            for (int k = 0; k < inner; ++k) {
                acc += static_cast<double>(row[k]);
            }
        } else {
            // even strides: lane-rotated start so the lanes spread over banks
            const int rot = threadIdx.x & 31;
            for (int k = 0; k < inner; ++k) {
                int q = k + rot;
                q = q >= inner ? q - inner : q;
                acc += static_cast<double>(row[q]);
            }
        }
        y[r0 + threadIdx.x] = static_cast<float>(acc / static_cast<double>(inner));
    }
}

// Block per row for long rows.
__global__ void row_mean_block_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t inner) {
    __shared__ double part[32];
    const float* r = x + blockIdx.x * inner;
    double s = 0.0;
    if ((reinterpret_cast<uintptr_t>(r) & 15) == 0 && inner % 4 == 0) {
        const float4* r4 = reinterpret_cast<const float4*>(r);
        for (int64_t k = threadIdx.x; k < inner / 4; k += blockDim.x) {
            const float4 v = __ldg(r4 + k);
            s += (double)v.x + (double)v.y + (double)v.z + (double)v.w;
        }
    } else {
        for (int64_t k = threadIdx.x; k < inner; k += blockDim.x) {
            s += static_cast<double>(__ldg(r + k));
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        s += __shfl_xor_sync(0xffffffffu, s, o);
    }
    if ((threadIdx.x & 31) == 0) {
        part[threadIdx.x >> 5] = s;
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        s = threadIdx.x < blockDim.x / 32 ? part[threadIdx.x] : 0.0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            s += __shfl_xor_sync(0xffffffffu, s, o);
        }
        if (threadIdx.x == 0) {
            y[blockIdx.x] = static_cast<float>(s / static_cast<double>(inner));
        }
    }
}

// 32-bit geometry of a channels-last pool (every extent and index < 2^31).
struct PoolGeom32 {
    int C4, H, W, OH, OW, KH, KW, sh, sw, ph, pw, dh, dw;
};

// Channels-last max pool: one thread per (output pixel, 4 channels), so a
// warp reads 512 contiguous bytes of one input pixel per tap (C % 4 == 0).
__global__ void maxpool2d_nhwc4_kernel(const float4* __restrict__ x, float4* __restrict__ y, PoolGeom32 g,
                                       uint32_t total) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const uint32_t c4 = i % g.C4;
        uint32_t t = i / g.C4;
        const int ow = static_cast<int>(t % g.OW);
        t /= g.OW;
        const int oh = static_cast<int>(t % g.OH);
        const uint32_t n = t / g.OH;
        const int h0 = oh * g.sh - g.ph;
        const int w0 = ow * g.sw - g.pw;
        float4 best = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
        for (int kh = 0; kh < g.KH; ++kh) {
            const int ih = h0 + kh * g.dh;
            if (ih < 0 || ih >= g.H) {
                continue;
            }
            const float4* row = x + ((size_t)(n * g.H + ih) * g.W) * g.C4 + c4;
            for (int kw = 0; kw < g.KW; ++kw) {
                const int iw = w0 + kw * g.dw;
                if (iw < 0 || iw >= g.W) {
                    continue;
                }
                const float4 v = __ldg(row + iw * g.C4);
                best.x = v.x > best.x ? v.x : best.x;
                best.y = v.y > best.y ? v.y : best.y;
                best.z = v.z > best.z ? v.z : best.z;
                best.w = v.w > best.w ? v.w : best.w;
            }
        }
        y[i] = best;
    }
}

// The same for a fixed KH x KW window without dilation: fully unrolled, so
// all taps' loads are in flight together (an out-of-image tap reads as
// -inf, which never wins the same comparison the generic kernel makes).
template <int KH, int KW>
__global__ void maxpool2d_nhwc4_fixed_kernel(const float4* __restrict__ x, float4* __restrict__ y, PoolGeom32 g,
                                             uint32_t total) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const uint32_t c4 = i % g.C4;
        uint32_t t = i / g.C4;
        const int ow = static_cast<int>(t % g.OW);
        t /= g.OW;
        const int oh = static_cast<int>(t % g.OH);
        const uint32_t n = t / g.OH;
        const int h0 = oh * g.sh - g.ph;
        const int w0 = ow * g.sw - g.pw;
        const float4* base = x + (size_t)n * g.H * g.W * g.C4 + c4;
        float4 v[KH * KW];
#pragma unroll
        for (int kh = 0; kh < KH; ++kh) {
#pragma unroll
            for (int kw = 0; kw < KW; ++kw) {
                const int ih = h0 + kh, iw = w0 + kw;
                const bool ok = (unsigned)ih < (unsigned)g.H && (unsigned)iw < (unsigned)g.W;
                v[kh * KW + kw] = ok ? __ldg(base + ((size_t)ih * g.W + iw) * g.C4)
                                     : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
            }
        }
        float4 best = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
#pragma unroll
        for (int k = 0; k < KH * KW; ++k) {
            best.x = v[k].x > best.x ? v[k].x : best.x;
            best.y = v[k].y > best.y ? v[k].y : best.y;
            best.z = v[k].z > best.z ? v[k].z : best.z;
            best.w = v[k].w > best.w ? v[k].w : best.w;
        }
        y[i] = best;
    }
}

__global__ void maxpool2d_nhwc1_kernel(const float* __restrict__ x, float* __restrict__ y, PoolGeom g, int64_t total) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t c = i % g.C;
        int64_t t = i / g.C;
        const int64_t ow = t % g.OW;
        t /= g.OW;
        const int64_t oh = t % g.OH;
        const int64_t n = t / g.OH;
        const int64_t h0 = oh * g.sh - g.ph;
        const int64_t w0 = ow * g.sw - g.pw;
        float best = -INFINITY;
        for (int64_t kh = 0; kh < g.KH; ++kh) {
            const int64_t ih = h0 + kh * g.dh;
            if (ih < 0 || ih >= g.H) {
                continue;
            }
            for (int64_t kw = 0; kw < g.KW; ++kw) {
                const int64_t iw = w0 + kw * g.dw;
                if (iw < 0 || iw >= g.W) {
                    continue;
                }
                const float v = __ldg(x + ((n * g.H + ih) * g.W + iw) * g.C + c);
                best = v > best ? v : best;
            }
        }
        y[i] = best;
    }
}

// Channels-last spatial mean: a 32 x 8 block owns 32 channels of one image;
// threadIdx.y strides the pixels, the 8 partial double sums meet in shared
// memory. Reads are 128-byte coalesced along the channels.
__global__ void mean_nhwc_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t hw, int64_t C) {
    __shared__ double part[8][33];
    const int64_t c = blockIdx.x * 32 + threadIdx.x;
    const int64_t n = blockIdx.y;
    double s = 0.0;
    if (c < C) {
        const float* p = x + n * hw * C + c;
        for (int64_t q = threadIdx.y; q < hw; q += 8) {
            s += static_cast<double>(__ldg(p + q * C));
        }
    }
    part[threadIdx.y][threadIdx.x] = s;
    __syncthreads();
    if (threadIdx.y == 0 && c < C) {
        double t = 0.0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            t += part[j][threadIdx.x];
        }
        y[n * C + c] = static_cast<float>(t / static_cast<double>(hw));
    }
}

} // namespace

void maxpool2d_nhwc(nb2_device* dev, const PoolGeom& g, const float* x, float* y) {
    const bool v4 = g.C % 4 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0;
    const int64_t total = g.N * g.OH * g.OW * (v4 ? g.C / 4 : g.C);
    if (total <= 0) {
        return;
    }
    const int64_t blocks = std::min<int64_t>((total + 255) / 256, static_cast<int64_t>(dev->num_sms) * 32);
    if (v4 && total < (int64_t(1) << 31) && g.N * g.H * g.W * g.C < (int64_t(1) << 33)) {
        const PoolGeom32 g32{static_cast<int>(g.C / 4), static_cast<int>(g.H), static_cast<int>(g.W),
                             static_cast<int>(g.OH), static_cast<int>(g.OW), static_cast<int>(g.KH),
                             static_cast<int>(g.KW), static_cast<int>(g.sh), static_cast<int>(g.sw),
                             static_cast<int>(g.ph), static_cast<int>(g.pw), static_cast<int>(g.dh),
                             static_cast<int>(g.dw)};
        const auto* x4 = reinterpret_cast<const float4*>(x);
        auto* y4 = reinterpret_cast<float4*>(y);
        const auto tot = static_cast<uint32_t>(total);
        const auto nb = static_cast<unsigned>(blocks);
        const bool plain = g.dh == 1 && g.dw == 1;
        if (plain && g.KH == 3 && g.KW == 3) {
            maxpool2d_nhwc4_fixed_kernel<3, 3><<<nb, 256, 0, dev->stream>>>(x4, y4, g32, tot);
        } else if (plain && g.KH == 5 && g.KW == 5) {
            maxpool2d_nhwc4_fixed_kernel<5, 5><<<nb, 256, 0, dev->stream>>>(x4, y4, g32, tot);
        } else if (plain && g.KH == 2 && g.KW == 2) {
            maxpool2d_nhwc4_fixed_kernel<2, 2><<<nb, 256, 0, dev->stream>>>(x4, y4, g32, tot);
        } else {
            maxpool2d_nhwc4_kernel<<<nb, 256, 0, dev->stream>>>(x4, y4, g32, tot);
        }
    } else {
        const int64_t total1 = g.N * g.OH * g.OW * g.C;
        const int64_t blocks1 = std::min<int64_t>((total1 + 255) / 256, static_cast<int64_t>(dev->num_sms) * 32);
        maxpool2d_nhwc1_kernel<<<static_cast<unsigned>(blocks1), 256, 0, dev->stream>>>(x, y, g, total1);
    }
    check_cuda(cudaGetLastError(), "maxpool_nhwc launch");
}

void mean_nhwc(nb2_device* dev, const float* x, float* y, int64_t n, int64_t hw, int64_t c) {
    if (n <= 0 || c <= 0 || hw <= 0) {
        return;
    }
    if (n > 65535) {
        fail(kStatusUnsupported, "GlobalAveragePool: batch above 65535 in channels-last form");
    }
    const dim3 grid(static_cast<unsigned>((c + 31) / 32), static_cast<unsigned>(n), 1);
    mean_nhwc_kernel<<<grid, dim3(32, 8), 0, dev->stream>>>(x, y, hw, c);
    check_cuda(cudaGetLastError(), "mean_nhwc launch");
}

namespace {

// One thread per output, NCHW. Same window clipping, float summation order
// (rows, then columns) and divisor as the reference row
// (src/kernels/average_pool.cpp:198-225), so results are bit-identical.
__global__ void avgpool2d_kernel(const float* __restrict__ x, float* __restrict__ y, AvgPoolGeom g, int64_t total) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t ow = i % g.OW;
        int64_t t = i / g.OW;
        const int64_t oh = t % g.OH;
        t /= g.OH; // n * C + c
        const float* xc = x + t * g.H * g.W;
        const int64_t hs = oh * g.sh - g.pt, he = min(hs + g.KH, g.H + g.pb);
        const int64_t ws = ow * g.sw - g.pl, we = min(ws + g.KW, g.W + g.pr);
        const int64_t h0 = hs > 0 ? hs : 0, h1 = min(he, g.H);
        const int64_t w0 = ws > 0 ? ws : 0, w1 = min(we, g.W);
        float sum = 0.0f;
        for (int64_t ih = h0; ih < h1; ++ih) {
            for (int64_t iw = w0; iw < w1; ++iw) {
                sum += __ldg(xc + ih * g.W + iw);
            }
        }
        const int64_t div = g.include_pad ? (he - hs) * (we - ws) : (h1 - h0) * (w1 - w0);
        y[i] = div > 0 ? sum / static_cast<float>(div) : 0.0f;
    }
}

} // namespace

void avgpool2d(nb2_device* dev, const AvgPoolGeom& g, const float* x, float* y) {
    const int64_t total = g.N * g.C * g.OH * g.OW;
    if (total == 0) {
        return;
    }
    const int64_t blocks = std::min<int64_t>((total + 255) / 256, static_cast<int64_t>(dev->num_sms) * 32);
    avgpool2d_kernel<<<static_cast<unsigned>(blocks), 256, 0, dev->stream>>>(x, y, g, total);
    check_cuda(cudaGetLastError(), "avgpool launch");
}

namespace {

// One CTA per (n, c) plane at a time: the plane is read once into shared
// memory, then each pool of the cascade is a row pass (max over the in-range
// columns w-r..w+r) and a column pass (rows h-r..h+r) between two shared
// buffers; the column pass writes its slice of the Concat. Max over in-range
// taps of a separable window is the max of row maxima, so every slice equals
// the reference's one-window-at-a-time MaxPool (src/kernels/max_pool.cpp:207-235:
// `v > best` from -inf, NaN never taken).
__global__ void __launch_bounds__(128) sppf_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t planes,
                                                   int64_t C, int H, int W, int r, int chain) {
    extern __shared__ float sppf_smem[];
    const int hw = H * W;
    float* a = sppf_smem;
    float* b = sppf_smem + hw;
    const int64_t slice = C * hw;
    for (int64_t p = blockIdx.x; p < planes; p += gridDim.x) {
        const int64_t n = p / C, c = p % C;
        const float* xp = x + p * hw;
        float* yp = y + (n * (chain + 1) * C + c) * hw;
        __syncthreads(); // the previous plane's readers of a are done
        for (int i = threadIdx.x; i < hw; i += blockDim.x) {
            const float v = __ldg(xp + i);
            a[i] = v;
            yp[i] = v;
        }
        for (int l = 1; l <= chain; ++l) {
            __syncthreads();
            for (int i = threadIdx.x; i < hw; i += blockDim.x) {
                const int h = i / W, w = i - h * W;
                const int w0 = w - r < 0 ? 0 : w - r, w1 = w + r >= W ? W - 1 : w + r;
                const float* row = a + h * W;
                float best = -INFINITY;
                for (int q = w0; q <= w1; ++q) {
                    best = row[q] > best ? row[q] : best;
                }
                b[i] = best;
            }
            __syncthreads();
            float* ys = yp + l * slice;
            for (int i = threadIdx.x; i < hw; i += blockDim.x) {
                const int h = i / W, w = i - h * W;
                const int h0 = h - r < 0 ? 0 : h - r, h1 = h + r >= H ? H - 1 : h + r;
                float best = -INFINITY;
                for (int q = h0; q <= h1; ++q) {
                    const float v = b[q * W + w];
                    best = v > best ? v : best;
                }
                a[i] = best;
                ys[i] = best;
            }
        }
    }
}

} // namespace

void sppf_nchw(nb2_device* dev, const SppfGeom& g, const float* x, float* y) {
    if (g.H * g.W > kSppfMaxPlane || g.k % 2 == 0 || g.k < 1 || g.chain < 1) {
        fail(kStatusInvalid, "SPPF: needs an odd window and a plane of at most 6144 elements");
    }
    const int64_t planes = g.N * g.C;
    if (planes == 0 || g.H * g.W == 0) {
        return;
    }
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>(planes, static_cast<int64_t>(dev->num_sms) * 16));
    const size_t smem = static_cast<size_t>(2 * g.H * g.W) * sizeof(float);
    sppf_kernel<<<grid, 128, smem, dev->stream>>>(x, y, planes, g.C, static_cast<int>(g.H), static_cast<int>(g.W),
                                                  static_cast<int>(g.k / 2), static_cast<int>(g.chain));
    check_cuda(cudaGetLastError(), "sppf launch");
}

void maxpool2d(nb2_device* dev, const PoolGeom& g, const float* x, float* y) {
    const int64_t total = g.N * g.C * g.OH * g.OW;
    if (total <= 0) {
        return;
    }
    const int64_t blocks = std::min<int64_t>((total + 255) / 256, static_cast<int64_t>(dev->num_sms) * 32);
    const bool small = total < (int64_t(1) << 31) && g.N * g.C * g.H * g.W < (int64_t(1) << 31);
    const bool plain = small && g.dh == 1 && g.dw == 1;
    const auto nb = static_cast<unsigned>(blocks);
    const int H = static_cast<int>(g.H), W = static_cast<int>(g.W), OH = static_cast<int>(g.OH),
              OW = static_cast<int>(g.OW), sh = static_cast<int>(g.sh), sw = static_cast<int>(g.sw),
              ph = static_cast<int>(g.ph), pw = static_cast<int>(g.pw);
    const auto tot = static_cast<uint32_t>(total);
    if (plain && g.KH == 5 && g.KW == 5) {
        maxpool2d_fixed_kernel<5, 5><<<nb, 256, 0, dev->stream>>>(x, y, H, W, OH, OW, sh, sw, ph, pw, tot);
    } else if (plain && g.KH == 3 && g.KW == 3) {
        maxpool2d_fixed_kernel<3, 3><<<nb, 256, 0, dev->stream>>>(x, y, H, W, OH, OW, sh, sw, ph, pw, tot);
    } else if (plain && g.KH == 2 && g.KW == 2) {
        maxpool2d_fixed_kernel<2, 2><<<nb, 256, 0, dev->stream>>>(x, y, H, W, OH, OW, sh, sw, ph, pw, tot);
    } else {
        maxpool2d_kernel<<<nb, 256, 0, dev->stream>>>(x, y, g, total);
    }
    check_cuda(cudaGetLastError(), "maxpool launch");
}

void row_mean(nb2_device* dev, const float* x, float* y, int64_t rows, int64_t inner) {
    if (rows <= 0 || inner <= 0) {
        return;
    }
    if (inner <= kMeanInner) {
        const int64_t blocks = (rows + kMeanRows - 1) / kMeanRows;
        row_mean_staged_kernel<<<static_cast<unsigned>(blocks), kMeanRows, 0, dev->stream>>>(
            x, y, rows, static_cast<int>(inner));
    } else if (inner <= 1024) {
        const int64_t blocks = (rows * 32 + 255) / 256;
        row_mean_warp_kernel<<<static_cast<unsigned>(blocks), 256, 0, dev->stream>>>(x, y, rows, inner);
    } else {
        row_mean_block_kernel<<<static_cast<unsigned>(rows), 256, 0, dev->stream>>>(x, y, inner);
    }
    check_cuda(cudaGetLastError(), "row_mean launch");
}

} // namespace nb2
