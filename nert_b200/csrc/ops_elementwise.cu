// Elementwise rows: unary ops and NumPy-broadcast binaries.
//
// Reference semantics: Relu max(0,x) (src/kernels/relu.cpp:52), Sigmoid
// 1/(1+exp(-x)) in float (src/kernels/sigmoid.cpp:52), Erf std::erf in float
// (src/kernels/erf.cpp:48), broadcast binaries in float32 per element
// (src/kernels/add.cpp:96-130, mul.cpp, sub.cpp, div.cpp; int64 Div truncates
// toward zero, div.cpp:96-115). The reference CUDA rows run one thread per
// element with div/mod stride math (src/cuda/add.cu:90-104); here the same-shape
// case moves 128-bit vectors and only true broadcasts take the stride path.

#include "ops.cuh"

#include <cmath>

namespace nb2 {

namespace {

__device__ __forceinline__ float unary_f(int op, float x) {
    switch (op) {
    case kURelu:
        return x > 0.0f ? x : 0.0f;
    case kUSigmoid:
        return 1.0f / (1.0f + expf(-x));
    case kUErf:
        return erff(x);
    case kUSqrt:
        return sqrtf(x);
    case kUNeg:
        return -x;
    case kUAbs:
        return fabsf(x);
    case kUExp:
        return expf(x);
    case kUTanh:
        return tanhf(x);
    case kUSilu:
        return x * (1.0f / (1.0f + expf(-x)));
    case kUGeluErf:
        return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
    default:
        return x;
    }
}

__global__ void unary_vec4_kernel(int op, const float4* __restrict__ x, float4* __restrict__ y, int64_t n4) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
        float4 v = x[i];
        v.x = unary_f(op, v.x);
        v.y = unary_f(op, v.y);
        v.z = unary_f(op, v.z);
        v.w = unary_f(op, v.w);
        y[i] = v;
    }
}

__global__ void unary_kernel(int op, const float* __restrict__ x, float* __restrict__ y, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        y[i] = unary_f(op, x[i]);
    }
}

__device__ __forceinline__ float binary_f(int op, float a, float b) {
    switch (op) {
    case kBAdd:
        return a + b;
    case kBSub:
        return a - b;
    case kBMul:
        return a * b;
    case kBDiv:
        return a / b;
    default:
        return powf(a, b);
    }
}

__device__ __forceinline__ long long binary_i(int op, long long a, long long b, int* err) {
    switch (op) {
    case kBAdd:
        return a + b;
    case kBSub:
        return a - b;
    case kBMul:
        return a * b;
    case kBDiv:
        if (b == 0) {
            atomicExch(err, 3);
            return 0;
        }
        return a / b; // C++ division truncates toward zero
    default:
        return 0;
    }
}

__global__ void binary_same_vec4_kernel(int op, const float4* __restrict__ a, const float4* __restrict__ b,
                                        float4* __restrict__ y, int64_t n4) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
        const float4 u = a[i], v = b[i];
        y[i] = make_float4(binary_f(op, u.x, v.x), binary_f(op, u.y, v.y), binary_f(op, u.z, v.z),
                           binary_f(op, u.w, v.w));
    }
}

// Two-axis broadcast after collapsing: y is [outer][inner] with inner % 4 ==
// 0; each operand is full (0), repeats a row of `inner` (1), holds one value
// per row (2) or is a scalar (3). 32-bit indices.
template <int M>
__device__ __forceinline__ float4 bload(const float* __restrict__ p, uint32_t i4, uint32_t inner4) {
    if constexpr (M == 0) {
        return reinterpret_cast<const float4*>(p)[i4];
    } else if constexpr (M == 1) {
        return reinterpret_cast<const float4*>(p)[i4 % inner4];
    } else if constexpr (M == 2) {
        const float v = p[i4 / inner4];
        return make_float4(v, v, v, v);
    } else {
        const float v = p[0];
        return make_float4(v, v, v, v);
    }
}

template <int MA, int MB>
__global__ void bcast2_vec4_kernel(int op, const float* __restrict__ a, const float* __restrict__ b,
                                   float4* __restrict__ y, uint32_t n4, uint32_t inner4) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += gridDim.x * blockDim.x) {
        const float4 u = bload<MA>(a, i, inner4), v = bload<MB>(b, i, inner4);
        y[i] = make_float4(binary_f(op, u.x, v.x), binary_f(op, u.y, v.y), binary_f(op, u.z, v.z),
                           binary_f(op, u.w, v.w));
    }
}

template <int MA>
void launch_bcast2(int mb, dim3 grid, cudaStream_t st, int op, const float* a, const float* b, float4* y, uint32_t n4,
                   uint32_t inner4) {
    switch (mb) {
    case 0:
        bcast2_vec4_kernel<MA, 0><<<grid, 256, 0, st>>>(op, a, b, y, n4, inner4);
        break;
    case 1:
        bcast2_vec4_kernel<MA, 1><<<grid, 256, 0, st>>>(op, a, b, y, n4, inner4);
        break;
    case 2:
        bcast2_vec4_kernel<MA, 2><<<grid, 256, 0, st>>>(op, a, b, y, n4, inner4);
        break;
    default:
        bcast2_vec4_kernel<MA, 3><<<grid, 256, 0, st>>>(op, a, b, y, n4, inner4);
        break;
    }
}

struct BStrides {
    int rank;
    int64_t ydims[kMaxRank];
    int64_t as[kMaxRank];
    int64_t bs[kMaxRank];
};

template <typename T>
__global__ void binary_bcast_kernel(int op, const T* __restrict__ a, const T* __restrict__ b, T* __restrict__ y,
                                    int64_t n, BStrides s, int* err) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t rem = i, ao = 0, bo = 0;
        for (int d = s.rank - 1; d >= 0; --d) {
            const int64_t c = rem % s.ydims[d];
            rem /= s.ydims[d];
            ao += c * s.as[d];
            bo += c * s.bs[d];
        }
        if constexpr (sizeof(T) == 8) {
            y[i] = binary_i(op, a[ao], b[bo], err);
        } else {
            y[i] = binary_f(op, a[ao], b[bo]);
        }
    }
}

unsigned grid_for(nb2_device* dev, int64_t n, int threads = 256) {
    const int64_t blocks = (n + threads - 1) / threads;
    const int64_t cap = static_cast<int64_t>(dev->num_sms) * 16;
    return static_cast<unsigned>(std::max<int64_t>(1, std::min(blocks, cap)));
}

} // namespace

void unary(nb2_device* dev, int op, const float* x, float* y, int64_t n) {
    if (n <= 0) {
        return;
    }
    if ((reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0 && n % 4 == 0) {
        unary_vec4_kernel<<<grid_for(dev, n / 4), 256, 0, dev->stream>>>(
            op, reinterpret_cast<const float4*>(x), reinterpret_cast<float4*>(y), n / 4);
    } else {
        unary_kernel<<<grid_for(dev, n), 256, 0, dev->stream>>>(op, x, y, n);
    }
    check_cuda(cudaGetLastError(), "unary launch");
}

void binary(nb2_device* dev, int op, int dtype, const void* a, const std::vector<int64_t>& ad, const void* b,
            const std::vector<int64_t>& bd, void* y, const std::vector<int64_t>& yd) {
    int64_t n = 1;
    for (int64_t d : yd) {
        n *= d;
    }
    if (n <= 0) {
        return;
    }
    if (yd.size() > kMaxRank) {
        fail(kStatusUnsupported, "broadcast rank above 8");
    }
    if (dtype == kF32 && ad == yd && bd == yd && n % 4 == 0 && ((reinterpret_cast<uintptr_t>(a) |
        reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(y)) & 15) == 0) {
        binary_same_vec4_kernel<<<grid_for(dev, n / 4), 256, 0, dev->stream>>>(
            op, static_cast<const float4*>(a), static_cast<const float4*>(b), static_cast<float4*>(y), n / 4);
        check_cuda(cudaGetLastError(), "binary launch");
        return;
    }
    if (dtype == kF32 && n < (int64_t(1) << 31)) {
        // collapse to y[outer][inner] and classify each operand
        const int r = static_cast<int>(yd.size());
        std::vector<int64_t> ys, as, bs;
        auto stride_of = [&](const std::vector<int64_t>& dims, int d, int64_t run) {
            const int src = d - (r - static_cast<int>(dims.size()));
            return (src < 0 || dims[src] == 1) ? int64_t(0) : run;
        };
        int64_t arun = 1, brun = 1;
        std::vector<int64_t> a_st(r), b_st(r);
        for (int d = r - 1; d >= 0; --d) {
            a_st[d] = stride_of(ad, d, arun);
            b_st[d] = stride_of(bd, d, brun);
            const int sa = d - (r - static_cast<int>(ad.size())), sb = d - (r - static_cast<int>(bd.size()));
            arun *= sa >= 0 ? ad[sa] : 1;
            brun *= sb >= 0 ? bd[sb] : 1;
        }
        for (int d = 0; d < r; ++d) {
            if (yd[d] == 1) {
                continue;
            }
            if (!ys.empty() && as.back() == a_st[d] * yd[d] && bs.back() == b_st[d] * yd[d]) {
                ys.back() *= yd[d];
                as.back() = a_st[d];
                bs.back() = b_st[d];
                continue;
            }
            ys.push_back(yd[d]);
            as.push_back(a_st[d]);
            bs.push_back(b_st[d]);
        }
        if (ys.size() == 1) {
            ys.insert(ys.begin(), 1);
            as.insert(as.begin(), 0);
            bs.insert(bs.begin(), 0);
        }
        if (ys.size() == 2 && ys[1] % 4 == 0) {
            const int64_t inner = ys[1];
            auto mode = [&](int64_t so, int64_t si) {
                if (si == 1) {
                    return (so == inner || ys[0] == 1) ? 0 : (so == 0 ? 1 : -1);
                }
                if (si == 0) {
                    return so == 0 ? 3 : (so == 1 ? 2 : -1);
                }
                return -1;
            };
            const int ma = mode(as[0], as[1]), mb = mode(bs[0], bs[1]);
            auto vec_ok = [](int m, const void* p) {
                return m >= 2 || (reinterpret_cast<uintptr_t>(p) & 15) == 0;
            };
            if (ma >= 0 && mb >= 0 && vec_ok(ma, a) && vec_ok(mb, b) && (reinterpret_cast<uintptr_t>(y) & 15) == 0) {
                const uint32_t n4 = static_cast<uint32_t>(n / 4), inner4 = static_cast<uint32_t>(inner / 4);
                const dim3 grid(grid_for(dev, n4));
                const float* fa = static_cast<const float*>(a);
                const float* fb = static_cast<const float*>(b);
                float4* fy = static_cast<float4*>(y);
                switch (ma) {
                case 0:
                    launch_bcast2<0>(mb, grid, dev->stream, op, fa, fb, fy, n4, inner4);
                    break;
                case 1:
                    launch_bcast2<1>(mb, grid, dev->stream, op, fa, fb, fy, n4, inner4);
                    break;
                case 2:
                    launch_bcast2<2>(mb, grid, dev->stream, op, fa, fb, fy, n4, inner4);
                    break;
                default:
                    launch_bcast2<3>(mb, grid, dev->stream, op, fa, fb, fy, n4, inner4);
                    break;
                }
                check_cuda(cudaGetLastError(), "binary launch");
                return;
            }
        }
    }
    BStrides s{};
    s.rank = static_cast<int>(yd.size());
    auto strides_for = [&](const std::vector<int64_t>& dims, int64_t* out) {
        // right-align dims against the output, stride 0 on broadcast axes
        const int off = s.rank - static_cast<int>(dims.size());
        int64_t st = 1;
        for (int d = s.rank - 1; d >= 0; --d) {
            const int src = d - off;
            if (src < 0) {
                out[d] = 0;
                continue;
            }
            out[d] = dims[src] == 1 ? 0 : st;
            st *= dims[src];
        }
    };
    for (int d = 0; d < s.rank; ++d) {
        s.ydims[d] = yd[d];
    }
    strides_for(ad, s.as);
    strides_for(bd, s.bs);
    if (dtype == kF32) {
        binary_bcast_kernel<float><<<grid_for(dev, n), 256, 0, dev->stream>>>(
            op, static_cast<const float*>(a), static_cast<const float*>(b), static_cast<float*>(y), n, s,
            dev->err_word);
    } else if (dtype == kI64) {
        binary_bcast_kernel<long long><<<grid_for(dev, n), 256, 0, dev->stream>>>(
            op, static_cast<const long long*>(a), static_cast<const long long*>(b), static_cast<long long*>(y), n, s,
            dev->err_word);
    } else {
        fail(kStatusUnsupported, "binary: unsupported dtype");
    }
    check_cuda(cudaGetLastError(), "binary launch");
}

void copy(nb2_device* dev, const void* src, void* dst, int64_t bytes) {
    if (bytes <= 0 || src == dst) {
        return;
    }
    check_cuda(cudaMemcpyAsync(dst, src, static_cast<size_t>(bytes), cudaMemcpyDeviceToDevice, dev->stream),
               "cudaMemcpyAsync(D2D)");
}

namespace {
__global__ void channel_affine_kernel(const float* __restrict__ x, const float* __restrict__ a,
                                      const float* __restrict__ b, float* __restrict__ y, int64_t C, int64_t inner,
                                      int64_t total) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t c = (i / inner) % C;
        y[i] = fmaf(__ldg(x + i), __ldg(a + c), __ldg(b + c));
    }
}
} // namespace

void channel_affine(nb2_device* dev, const float* x, const float* a, const float* b, float* y, int64_t outer,
                    int64_t C, int64_t inner) {
    const int64_t total = outer * C * inner;
    if (total == 0) {
        return;
    }
    const int64_t blocks = std::min<int64_t>((total + 255) / 256, static_cast<int64_t>(dev->num_sms) * 32);
    channel_affine_kernel<<<static_cast<unsigned>(blocks), 256, 0, dev->stream>>>(x, a, b, y, C, inner, total);
    check_cuda(cudaGetLastError(), "channel_affine launch");
}

} // namespace nb2
