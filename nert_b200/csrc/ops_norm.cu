// Softmax and LayerNormalization rows.
//
// Reference semantics: Softmax subtracts the axis max, exponentiates and
// normalises (src/kernels/softmax.cpp:47-120, double sums); LayerNormalization
// takes the population mean and variance over the trailing axes from `axis`,
// y = (x - mean) / sqrt(var + eps) * scale + bias, with optional Mean and
// InvStdDev outputs (src/kernels/layer_normalization.cpp:77-160, double).
// The reference CUDA rows run one thread per row in three passes
// (src/cuda/softmax.cu:39-59, layer_normalization.cu:78-107). Here a warp (or a
// block for long rows) owns a row, keeps it in registers and reduces with
// shuffles, so every element is read once and written once.

#include "ops.cuh"
#include "ops_norm.cuh"

#include <cfloat>

namespace nb2 {

namespace {

constexpr int kWarpRowMax = 1024; // warp-per-row path up to this row length (32 regs/lane)

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    }
    return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        v += __shfl_xor_sync(0xffffffffu, v, o);
    }
    return v;
}

__device__ __forceinline__ double warp_sumd(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        v += __shfl_xor_sync(0xffffffffu, v, o);
    }
    return v;
}

// Warp per row, row length L <= 1024, values held in registers.
template <int PER_LANE>
__global__ void softmax_warp_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t rows, int L) {
    const int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= rows) {
        return;
    }
    const float* r = x + row * L;
    float v[PER_LANE];
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i) {
        const int k = lane + i * 32;
        v[i] = k < L ? __ldg(r + k) : -INFINITY;
        m = fmaxf(m, v[i]);
    }
    m = warp_max(m);
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i) {
        const int k = lane + i * 32;
        v[i] = k < L ? expf(v[i] - m) : 0.0f;
        s += v[i];
    }
    s = warp_sum(s);
    const float inv = 1.0f / s;
    float* o = y + row * L;
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i) {
        const int k = lane + i * 32;
        if (k < L) {
            o[k] = v[i] * inv;
        }
    }
}

// Block per row for long rows: three passes over the row (L1/L2 resident).
__global__ void softmax_block_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t L) {
    __shared__ float red[32];
    const float* r = x + blockIdx.x * L;
    float m = -INFINITY;
    for (int64_t k = threadIdx.x; k < L; k += blockDim.x) {
        m = fmaxf(m, __ldg(r + k));
    }
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) {
        red[threadIdx.x >> 5] = m;
    }
    __syncthreads();
    m = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : -INFINITY;
    m = warp_max(m);
    __syncthreads();
    if (threadIdx.x == 0) {
        red[0] = m;
    }
    __syncthreads();
    m = red[0];
    __syncthreads();
    float s = 0.0f;
    for (int64_t k = threadIdx.x; k < L; k += blockDim.x) {
        s += expf(__ldg(r + k) - m);
    }
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) {
        red[threadIdx.x >> 5] = s;
    }
    __syncthreads();
    s = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.0f;
    s = warp_sum(s);
    const float inv = 1.0f / __shfl_sync(0xffffffffu, s, 0);
    __syncthreads();
    if (threadIdx.x == 0) {
        red[0] = inv;
    }
    __syncthreads();
    const float iv = red[0];
    float* o = y + blockIdx.x * L;
    for (int64_t k = threadIdx.x; k < L; k += blockDim.x) {
        o[k] = expf(__ldg(r + k) - m) * iv;
    }
}

// Softmax along a non-innermost axis: thread per (outer, inner) column,
// consecutive threads on consecutive inner positions (coalesced).
__global__ void softmax_strided_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t outer, int64_t L,
                                       int64_t inner) {
    const int64_t total = outer * inner;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t o = t / inner, i = t - o * inner;
        const float* r = x + o * L * inner + i;
        float m = -INFINITY;
        for (int64_t k = 0; k < L; ++k) {
            m = fmaxf(m, __ldg(r + k * inner));
        }
        float s = 0.0f;
        for (int64_t k = 0; k < L; ++k) {
            s += expf(__ldg(r + k * inner) - m);
        }
        const float inv = 1.0f / s;
        float* w = y + o * L * inner + i;
        for (int64_t k = 0; k < L; ++k) {
            w[k * inner] = expf(__ldg(r + k * inner) - m) * inv;
        }
    }
}

// The same for short axes (L <= LMAX, e.g. YOLO's 16 DFL bins): the column
// is loaded once into registers with all L loads in flight, then max, sum
// and output exactly as above (same order, same expressions).
template <int LMAX>
__global__ void softmax_strided_reg_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t outer, int L,
                                           int64_t inner) {
    const int64_t total = outer * inner;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t o = t / inner, i = t - o * inner;
        const float* r = x + o * L * inner + i;
        float v[LMAX];
#pragma unroll
        for (int k = 0; k < LMAX; ++k) {
            v[k] = k < L ? __ldg(r + k * inner) : -INFINITY;
        }
        float m = -INFINITY;
#pragma unroll
        for (int k = 0; k < LMAX; ++k) {
            m = k < L ? fmaxf(m, v[k]) : m;
        }
        float s = 0.0f;
#pragma unroll
        for (int k = 0; k < LMAX; ++k) {
            if (k < L) {
                v[k] = expf(v[k] - m);
                s += v[k];
            }
        }
        const float inv = 1.0f / s;
        float* w = y + o * L * inner + i;
#pragma unroll
        for (int k = 0; k < LMAX; ++k) {
            if (k < L) {
                w[k * inner] = v[k] * inv;
            }
        }
    }
}

// Warp per row LayerNorm, D <= 1024; two-pass mean/variance in double.
template <int PER_LANE>
__global__ void layernorm_warp_kernel(const float* __restrict__ x, const float* __restrict__ scale,
                                      const float* __restrict__ bias, float* __restrict__ y, float* __restrict__ mean_out,
                                      float* __restrict__ inv_out, int64_t rows, int D, float eps) {
    const int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= rows) {
        return;
    }
    const float* r = x + row * D;
    float v[PER_LANE];
    double s = 0.0;
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i) {
        const int k = lane + i * 32;
        v[i] = k < D ? __ldg(r + k) : 0.0f;
        s += v[i];
    }
    const double mean = warp_sumd(s) / D;
    double q = 0.0;
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i) {
        const int k = lane + i * 32;
        const double d = k < D ? (double)v[i] - mean : 0.0;
        q += d * d;
    }
    const double var = warp_sumd(q) / D;
    const double inv = 1.0 / sqrt(var + (double)eps);
    float* o = y + row * D;
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i) {
        const int k = lane + i * 32;
        if (k < D) {
            double t = ((double)v[i] - mean) * inv * (double)__ldg(scale + k);
            if (bias) {
                t += (double)__ldg(bias + k);
            }
            o[k] = (float)t;
        }
    }
    if (lane == 0) {
        if (mean_out) {
            mean_out[row] = (float)mean;
        }
        if (inv_out) {
            inv_out[row] = (float)inv;
        }
    }
}

// Warp per row LayerNorm for D % 128 == 0 (D <= 1024): 16-byte loads and
// stores, two-pass mean / centred variance in fp32 from registers (the
// reference's double sums differ from these by rounding far below the fp32
// output's own precision).
// Up to D = 768 the kernel is held to 48 registers so five 256-thread blocks
// fit an SM and a ViT-B row count (6304 rows at b32) runs in one wave.
template <int V4>
__global__ void __launch_bounds__(256, V4 <= 6 ? 5 : 1) layernorm_warp4_kernel(const float4* __restrict__ x, const float4* __restrict__ scale,
                                       const float4* __restrict__ bias, float4* __restrict__ y,
                                       float* __restrict__ mean_out, float* __restrict__ inv_out, uint32_t rows,
                                       float eps) {
    const uint32_t row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= rows) {
        return;
    }
    constexpr int D = V4 * 128;
    const float4* r = x + (size_t)row * (D / 4);
    float4 v[V4];
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < V4; ++i) {
        v[i] = __ldg(r + lane + 32 * i);
        s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    }
    const float mean = warp_sum(s) * (1.0f / D);
    float q = 0.0f;
#pragma unroll
    for (int i = 0; i < V4; ++i) {
        const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
        q += (a * a + b * b) + (c * c + d * d);
    }
    const float inv = 1.0f / sqrtf(warp_sum(q) * (1.0f / D) + eps);
    float4* o = y + (size_t)row * (D / 4);
#pragma unroll
    for (int i = 0; i < V4; ++i) {
        const float4 g = __ldg(scale + lane + 32 * i);
        const float4 b = bias ? __ldg(bias + lane + 32 * i) : make_float4(0.f, 0.f, 0.f, 0.f);
        float4 w;
        w.x = (v[i].x - mean) * inv * g.x + b.x;
        w.y = (v[i].y - mean) * inv * g.y + b.y;
        w.z = (v[i].z - mean) * inv * g.z + b.z;
        w.w = (v[i].w - mean) * inv * g.w + b.w;
        o[lane + 32 * i] = w;
    }
    if (lane == 0) {
        if (mean_out) {
            mean_out[row] = mean;
        }
        if (inv_out) {
            inv_out[row] = inv;
        }
    }
}

// Block per row LayerNorm for D > 1024 (row re-read from L1/L2).
__global__ void layernorm_block_kernel(const float* __restrict__ x, const float* __restrict__ scale,
                                       const float* __restrict__ bias, float* __restrict__ y,
                                       float* __restrict__ mean_out, float* __restrict__ inv_out, int64_t D, float eps) {
    __shared__ double red[32];
    __shared__ double stat[2];
    const float* r = x + blockIdx.x * D;
    double s = 0.0;
    for (int64_t k = threadIdx.x; k < D; k += blockDim.x) {
        s += __ldg(r + k);
    }
    s = warp_sumd(s);
    if ((threadIdx.x & 31) == 0) {
        red[threadIdx.x >> 5] = s;
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        double t = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.0;
        t = warp_sumd(t);
        if (threadIdx.x == 0) {
            stat[0] = t / (double)D;
        }
    }
    __syncthreads();
    const double mean = stat[0];
    double q = 0.0;
    for (int64_t k = threadIdx.x; k < D; k += blockDim.x) {
        const double d = (double)__ldg(r + k) - mean;
        q += d * d;
    }
    q = warp_sumd(q);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) {
        red[threadIdx.x >> 5] = q;
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        double t = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.0;
        t = warp_sumd(t);
        if (threadIdx.x == 0) {
            stat[1] = 1.0 / sqrt(t / (double)D + (double)eps);
        }
    }
    __syncthreads();
    const double inv = stat[1];
    float* o = y + blockIdx.x * D;
    for (int64_t k = threadIdx.x; k < D; k += blockDim.x) {
        double t = ((double)__ldg(r + k) - mean) * inv * (double)__ldg(scale + k);
        if (bias) {
            t += (double)__ldg(bias + k);
        }
        o[k] = (float)t;
    }
    if (threadIdx.x == 0) {
        if (mean_out) {
            mean_out[blockIdx.x] = (float)mean;
        }
        if (inv_out) {
            inv_out[blockIdx.x] = (float)inv;
        }
    }
}

} // namespace

void softmax(nb2_device* dev, const float* x, float* y, int64_t outer, int64_t L, int64_t inner) {
    if (outer * L * inner <= 0) {
        return;
    }
    if (inner == 1 && L <= kWarpRowMax) {
        const unsigned blocks = static_cast<unsigned>((outer * 32 + 255) / 256);
        if (L <= 32) {
            softmax_warp_kernel<1><<<blocks, 256, 0, dev->stream>>>(x, y, outer, static_cast<int>(L));
        } else if (L <= 128) {
            softmax_warp_kernel<4><<<blocks, 256, 0, dev->stream>>>(x, y, outer, static_cast<int>(L));
        } else if (L <= 256) {
            softmax_warp_kernel<8><<<blocks, 256, 0, dev->stream>>>(x, y, outer, static_cast<int>(L));
        } else if (L <= 512) {
            softmax_warp_kernel<16><<<blocks, 256, 0, dev->stream>>>(x, y, outer, static_cast<int>(L));
        } else {
            softmax_warp_kernel<32><<<blocks, 256, 0, dev->stream>>>(x, y, outer, static_cast<int>(L));
        }
    } else if (inner == 1) {
        softmax_block_kernel<<<static_cast<unsigned>(outer), 256, 0, dev->stream>>>(x, y, L);
    } else {
        const int64_t total = outer * inner;
        const unsigned blocks = static_cast<unsigned>(std::min<int64_t>((total + 255) / 256, dev->num_sms * 32));
        if (L <= 8) {
            softmax_strided_reg_kernel<8><<<blocks, 256, 0, dev->stream>>>(x, y, outer, static_cast<int>(L), inner);
        } else if (L <= 16) {
            softmax_strided_reg_kernel<16><<<blocks, 256, 0, dev->stream>>>(x, y, outer, static_cast<int>(L), inner);
        } else if (L <= 32) {
            softmax_strided_reg_kernel<32><<<blocks, 256, 0, dev->stream>>>(x, y, outer, static_cast<int>(L), inner);
        } else {
            softmax_strided_kernel<<<blocks, 256, 0, dev->stream>>>(x, y, outer, L, inner);
        }
    }
    check_cuda(cudaGetLastError(), "softmax launch");
}

void layernorm(nb2_device* dev, const float* x, const float* scale, const float* bias, float* y, float* mean,
               float* inv_std, int64_t rows, int64_t D, float eps) {
    if (rows <= 0 || D <= 0) {
        return;
    }
    const bool al = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(scale) |
                      reinterpret_cast<uintptr_t>(bias) | reinterpret_cast<uintptr_t>(y)) & 15) == 0;
    if (D % 128 == 0 && D <= kWarpRowMax && al && rows < (int64_t(1) << 26)) {
        const unsigned blocks = static_cast<unsigned>((rows * 32 + 255) / 256);
        const auto* x4 = reinterpret_cast<const float4*>(x);
        const auto* s4 = reinterpret_cast<const float4*>(scale);
        const auto* b4 = reinterpret_cast<const float4*>(bias);
        auto* y4 = reinterpret_cast<float4*>(y);
        const auto r = static_cast<uint32_t>(rows);
        switch (D / 128) {
        case 1:
            layernorm_warp4_kernel<1><<<blocks, 256, 0, dev->stream>>>(x4, s4, b4, y4, mean, inv_std, r, eps);
            break;
        case 2:
            layernorm_warp4_kernel<2><<<blocks, 256, 0, dev->stream>>>(x4, s4, b4, y4, mean, inv_std, r, eps);
            break;
        case 3:
            layernorm_warp4_kernel<3><<<blocks, 256, 0, dev->stream>>>(x4, s4, b4, y4, mean, inv_std, r, eps);
            break;
        case 4:
            layernorm_warp4_kernel<4><<<blocks, 256, 0, dev->stream>>>(x4, s4, b4, y4, mean, inv_std, r, eps);
            break;
        case 5:
            layernorm_warp4_kernel<5><<<blocks, 256, 0, dev->stream>>>(x4, s4, b4, y4, mean, inv_std, r, eps);
            break;
        case 6:
            layernorm_warp4_kernel<6><<<blocks, 256, 0, dev->stream>>>(x4, s4, b4, y4, mean, inv_std, r, eps);
            break;
        case 7:
            layernorm_warp4_kernel<7><<<blocks, 256, 0, dev->stream>>>(x4, s4, b4, y4, mean, inv_std, r, eps);
            break;
        default:
            layernorm_warp4_kernel<8><<<blocks, 256, 0, dev->stream>>>(x4, s4, b4, y4, mean, inv_std, r, eps);
            break;
        }
    } else if (D <= kWarpRowMax) {
        const unsigned blocks = static_cast<unsigned>((rows * 32 + 255) / 256);
        const int d = static_cast<int>(D);
        if (D <= 256) {
            layernorm_warp_kernel<8><<<blocks, 256, 0, dev->stream>>>(x, scale, bias, y, mean, inv_std, rows, d, eps);
        } else if (D <= 512) {
            layernorm_warp_kernel<16><<<blocks, 256, 0, dev->stream>>>(x, scale, bias, y, mean, inv_std, rows, d, eps);
        } else if (D <= 768) {
            layernorm_warp_kernel<24><<<blocks, 256, 0, dev->stream>>>(x, scale, bias, y, mean, inv_std, rows, d, eps);
        } else {
            layernorm_warp_kernel<32><<<blocks, 256, 0, dev->stream>>>(x, scale, bias, y, mean, inv_std, rows, d, eps);
        }
    } else {
        layernorm_block_kernel<<<static_cast<unsigned>(rows), 256, 0, dev->stream>>>(x, scale, bias, y, mean, inv_std,
                                                                                     D, eps);
    }
    check_cuda(cudaGetLastError(), "layernorm launch");
}

} // namespace nb2
