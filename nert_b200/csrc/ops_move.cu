// Data-movement rows: Concat / Split (pitched segment copies in one launch),
// Transpose, Slice, Gather, Resize (nearest / linear through per-axis tables),
// Cast.
//
// Reference semantics: Concat/Split copy contiguous blocks along the axis
// (src/kernels/concat.cpp:64, split.cpp:65; the reference CUDA rows issue one
// cudaMemcpy per block from a host loop, src/cuda/concat.cu:63); Transpose
// permutes (transpose.cpp:54); Gather wraps negative indices and rejects
// out-of-range ones (gather.cpp:49-129); Resize samples per-axis tables built
// with the ONNX coordinate transform and nearest rounding
// (resize.cpp:62-158); Cast truncates float->int64 toward zero (cast.cpp).

#include "ops_move.cuh"
#include "ops.cuh"

#include <algorithm>
#include <cmath>
#include <cstring>

namespace nb2 {

namespace {

constexpr int kMaxSegs = 64;

struct SegTable {
    CopySeg s[kMaxSegs];
    int n;
};

// blockIdx.y = segment; grid-stride over rows x (row_bytes / unit). I is
// the index type (32-bit whenever every segment fits, which keeps the
// per-element divide cheap).
template <typename U, typename I>
__global__ void segment_copy_kernel(SegTable t) {
    const CopySeg s = t.s[blockIdx.y];
    const I per_row = static_cast<I>(s.row_bytes / static_cast<int64_t>(sizeof(U)));
    const I total = per_row * static_cast<I>(s.rows);
    for (I i = blockIdx.x * (I)blockDim.x + threadIdx.x; i < total; i += (I)gridDim.x * blockDim.x) {
        const I r = i / per_row, c = i - r * per_row;
        reinterpret_cast<U*>(s.dst + (int64_t)r * s.dst_pitch)[c] =
            reinterpret_cast<const U*>(s.src + (int64_t)r * s.src_pitch)[c];
    }
}

struct Dims8 {
    int64_t d[8];
};

template <typename T>
__global__ void transpose_kernel(const T* __restrict__ x, T* __restrict__ y, int rank, Dims8 out_dims,
                                 Dims8 in_stride_of_out_axis, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t rem = i, src = 0;
        for (int d = rank - 1; d >= 0; --d) {
            const int64_t c = rem % out_dims.d[d];
            rem /= out_dims.d[d];
            src += c * in_stride_of_out_axis.d[d];
        }
        y[i] = x[src];
    }
}

// Permutes whose innermost axis stays innermost: rows of `L` contiguous
// elements move as a block (16-byte vectors when L % 4 == 0). The row index
// decomposes over the collapsed output axes (32-bit math).
struct RowPerm {
    int rank;         // output axes other than the innermost
    uint32_t od[7];   // their extents
    int64_t ist[7];   // input stride (elements) of each
};

template <typename V>
__global__ void permute_rows_kernel(const V* __restrict__ x, V* __restrict__ y, RowPerm p, uint32_t rows,
                                    uint32_t L) {
    const uint32_t total = rows * L;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const uint32_t row = i / L, c = i - row * L;
        uint32_t rem = row;
        int64_t src = 0;
        for (int d = p.rank - 1; d >= 0; --d) {
            const uint32_t q = rem / p.od[d];
            src += (int64_t)(rem - q * p.od[d]) * p.ist[d];
            rem = q;
        }
        y[i] = x[src + c];
    }
}

// General 2-D tiled permute: u = the input's innermost axis (contiguous in x),
// v = the output's innermost axis (contiguous in y); the other axes form the
// batch (blockIdx.z, decomposed once per block).
struct TilePerm {
    int nb;            // batch axes
    int64_t bd[6];     // extents
    int64_t bin[6];    // input strides
    int64_t bout[6];   // output strides
    int64_t U, V;      // tile axis extents
    int64_t in_v;      // input stride of v
    int64_t out_u;     // output stride of u
};

// A 32 (u) x 64 (v) tile per block and pass: each thread has eight loads in
// flight (rows v) before the shared-memory exchange, then eight stores
// (two 32-wide v halves of four u rows).
__global__ void permute_tile_kernel(const float* __restrict__ x, float* __restrict__ y, TilePerm p, int64_t batches) {
    __shared__ float tile[64][33];
    for (int64_t b = blockIdx.z; b < batches; b += gridDim.z) {
        int64_t rem = b, ib = 0, ob = 0;
        for (int d = p.nb - 1; d >= 0; --d) {
            const int64_t c = rem % p.bd[d];
            rem /= p.bd[d];
            ib += c * p.bin[d];
            ob += c * p.bout[d];
        }
        const int64_t u0 = blockIdx.x * 32, v0 = blockIdx.y * 64;
        const int64_t u = u0 + threadIdx.x;
        float r[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int64_t v = v0 + threadIdx.y + 8 * j;
            r[j] = (u < p.U && v < p.V) ? __ldg(x + ib + v * p.in_v + u) : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            tile[threadIdx.y + 8 * j][threadIdx.x] = r[j];
        }
        __syncthreads();
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int64_t uu = u0 + threadIdx.y + 8 * (j & 3);
            const int vl = threadIdx.x + 32 * (j >> 2);
            const int64_t v = v0 + vl;
            if (uu < p.U && v < p.V) {
                y[ob + uu * p.out_u + v] = tile[vl][threadIdx.y + 8 * (j & 3)];
            }
        }
        __syncthreads();
    }
}

// Batched 2-D transpose [B, R, C] -> [B, C, R] through a 32x33 smem tile.
template <typename T>
__global__ void transpose_last2_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t R, int64_t C) {
    __shared__ T tile[32][33];
    const int64_t b = blockIdx.z;
    const int64_t r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
    const T* xb = x + b * R * C;
    T* yb = y + b * R * C;
    for (int i = threadIdx.y; i < 32; i += 8) {
        const int64_t r = r0 + i, c = c0 + threadIdx.x;
        if (r < R && c < C) {
            tile[i][threadIdx.x] = xb[r * C + c];
        }
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += 8) {
        const int64_t c = c0 + i, r = r0 + threadIdx.x;
        if (r < R && c < C) {
            yb[c * R + r] = tile[threadIdx.x][i];
        }
    }
}

template <typename T>
__global__ void slice_kernel(const T* __restrict__ x, T* __restrict__ y, int rank, Dims8 out_dims, Dims8 in_strides,
                             Dims8 starts, Dims8 steps, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t rem = i, src = 0;
        for (int d = rank - 1; d >= 0; --d) {
            const int64_t c = rem % out_dims.d[d];
            rem /= out_dims.d[d];
            src += (starts.d[d] + c * steps.d[d]) * in_strides.d[d];
        }
        y[i] = x[src];
    }
}

template <typename T>
__global__ void gather_kernel(const T* __restrict__ x, const int64_t* __restrict__ idx, T* __restrict__ y,
                              int64_t outer, int64_t axis_len, int64_t inner, int64_t n_idx, int* err) {
    const int64_t total = outer * n_idx * inner;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t in_i = i % inner;
        const int64_t t = i / inner;
        const int64_t j = t % n_idx;
        const int64_t o = t / n_idx;
        int64_t k = idx[j];
        if (k < 0) {
            k += axis_len;
        }
        if (k < 0 || k >= axis_len) {
            atomicExch(err, 2);
            y[i] = T(0);
            continue;
        }
        y[i] = x[(o * axis_len + k) * inner + in_i];
    }
}

// Nearest resize of the last two axes only (every leading axis copied
// through): y[o][oh][ow] = x[o][lh[oh]][lw[ow]], 32-bit indices, one
// coalesced store per thread (YOLO's x2 up-sampling).
template <typename T>
__global__ void resize_nearest2_kernel(const T* __restrict__ x, T* __restrict__ y, const int64_t* __restrict__ lh,
                                       const int64_t* __restrict__ lw, uint32_t H, uint32_t W, uint32_t OH,
                                       uint32_t OW, uint32_t n) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const uint32_t ow = i % OW;
        const uint32_t t = i / OW;
        const uint32_t oh = t % OH, o = t / OH;
        y[i] = x[((size_t)o * H + static_cast<uint32_t>(__ldg(lh + oh))) * W + static_cast<uint32_t>(__ldg(lw + ow))];
    }
}

// Nearest resize of a channels-last image ([N,H,W,C] in memory, C and N
// unchanged): each output pixel's C floats are the source pixel's, moved as
// 16-byte vectors; lh / lw are the H and W axes' source-index tables.
__global__ void resize_nearest_rows_kernel(const float4* __restrict__ x, float4* __restrict__ y,
                                           const int64_t* __restrict__ lh, const int64_t* __restrict__ lw,
                                           uint32_t H, uint32_t W, uint32_t OH, uint32_t OW, uint32_t C4,
                                           uint32_t n4) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += gridDim.x * blockDim.x) {
        const uint32_t q = i % C4;
        uint32_t t = i / C4;
        const uint32_t ow = t % OW;
        t /= OW;
        const uint32_t oh = t % OH, img = t / OH;
        y[i] = x[((img * H + static_cast<uint32_t>(lh[oh])) * W + static_cast<uint32_t>(lw[ow])) * C4 + q];
    }
}

// resize_nearest2_kernel for float rows with OW % 4 == 0: four outputs of one
// row per thread and one 16-byte store (the gathers of a quad share one input
// row).
__global__ void resize_nearest2_vec4_kernel(const float* __restrict__ x, float4* __restrict__ y,
                                            const int64_t* __restrict__ lh, const int64_t* __restrict__ lw,
                                            uint32_t H, uint32_t W, uint32_t OH, uint32_t OW4, uint32_t n4) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += gridDim.x * blockDim.x) {
        const uint32_t q = i % OW4;
        const uint32_t t = i / OW4;
        const uint32_t oh = t % OH, o = t / OH;
        const float* row = x + ((size_t)o * H + static_cast<uint32_t>(__ldg(lh + oh))) * W;
        const int64_t* c = lw + 4 * q;
        float4 v;
        v.x = __ldg(row + __ldg(c));
        v.y = __ldg(row + __ldg(c + 1));
        v.z = __ldg(row + __ldg(c + 2));
        v.w = __ldg(row + __ldg(c + 3));
        y[i] = v;
    }
}

struct ResizeDev {
    int rank;
    int64_t in_dims[8], out_dims[8], in_strides[8], axis_off[8];
    const int64_t* lower;
    const int64_t* upper;
    const double* weight;
};

template <typename T>
__global__ void resize_kernel(const T* __restrict__ x, T* __restrict__ y, ResizeDev r, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t rem = i;
        int64_t coord[8];
        for (int d = r.rank - 1; d >= 0; --d) {
            coord[d] = rem % r.out_dims[d];
            rem /= r.out_dims[d];
        }
        int64_t base = 0;
        int lin_axes[8];
        int nlin = 0;
        for (int d = 0; d < r.rank; ++d) {
            const int64_t t = r.axis_off[d] + coord[d];
            base += r.lower[t] * r.in_strides[d];
            if (r.weight[t] != 0.0) {
                lin_axes[nlin++] = d;
            }
        }
        if (nlin == 0) {
            y[i] = x[base];
            continue;
        }
        double acc = 0.0;
        for (int tap = 0; tap < (1 << nlin); ++tap) {
            int64_t off = base;
            double w = 1.0;
            for (int q = 0; q < nlin; ++q) {
                const int d = lin_axes[q];
                const int64_t t = r.axis_off[d] + coord[d];
                if (tap & (1 << q)) {
                    off += (r.upper[t] - r.lower[t]) * r.in_strides[d];
                    w *= r.weight[t];
                } else {
                    w *= 1.0 - r.weight[t];
                }
            }
            acc += w * static_cast<double>(x[off]);
        }
        y[i] = static_cast<T>(acc);
    }
}

__global__ void cast_kernel(const void* x, int from, void* y, int to, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        double v;
        if (from == 0) {
            v = static_cast<const float*>(x)[i];
        } else if (from == 1) {
            v = static_cast<double>(static_cast<const long long*>(x)[i]);
        } else {
            v = static_cast<const uint8_t*>(x)[i] ? 1.0 : 0.0;
        }
        if (to == 0) {
            static_cast<float*>(y)[i] = from == 1 ? static_cast<float>(static_cast<const long long*>(x)[i])
                                                  : static_cast<float>(v);
        } else if (to == 1) {
            static_cast<long long*>(y)[i] =
                from == 1 ? static_cast<const long long*>(x)[i] : static_cast<long long>(trunc(v));
        } else {
            static_cast<uint8_t*>(y)[i] = v != 0.0 ? 1 : 0;
        }
    }
}

unsigned blocks_for(nb2_device* dev, int64_t n) {
    return static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, dev->num_sms * 16)));
}

// NCHW -> NHWC with the channels zero padded to CP (4, 8 or 16): one thread
// per pixel; channel planes are read coalesced along the pixels and the
// pixel's CP channels written as CP/4 16-byte vectors.
template <int CP>
__global__ void nchw_to_nhwc_narrow_kernel(const float* __restrict__ x, float4* __restrict__ y, uint32_t C,
                                           uint32_t HW, uint32_t total) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const uint32_t n = i / HW, p = i - n * HW;
        const float* src = x + (size_t)n * C * HW + p;
        float v[CP];
#pragma unroll
        for (int c = 0; c < CP; ++c) {
            v[c] = (uint32_t)c < C ? __ldg(src + (size_t)c * HW) : 0.0f;
        }
#pragma unroll
        for (int q = 0; q < CP / 4; ++q) {
            y[(size_t)i * (CP / 4) + q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        }
    }
}

// NCHW -> NHWC with the channels zero padded to Cp (a multiple of 32): 32 x 32
// (channel x pixel) tiles through shared memory, both sides coalesced.
__global__ void nchw_to_nhwc_tile_kernel(const float* __restrict__ x, float* __restrict__ y, int C, int Cp,
                                         int64_t HW) {
    __shared__ float tile[32][33];
    const int64_t n = blockIdx.z;
    const int c0 = blockIdx.y * 32;
    const int64_t p0 = blockIdx.x * 32;
    for (int i = threadIdx.y; i < 32; i += 8) {
        const int c = c0 + i;
        const int64_t p = p0 + threadIdx.x;
        tile[i][threadIdx.x] = (c < C && p < HW) ? __ldg(x + (n * C + c) * HW + p) : 0.0f;
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += 8) {
        const int64_t p = p0 + i;
        const int c = c0 + threadIdx.x;
        if (p < HW) {
            y[(n * HW + p) * Cp + c] = tile[threadIdx.x][i];
        }
    }
}

} // namespace

void nchw_to_nhwc_pad(nb2_device* dev, const float* x, float* y, int64_t N, int64_t C, int64_t H, int64_t W,
                      int64_t Cp) {
    const int64_t HW = H * W, total = N * HW;
    if (total <= 0) {
        return;
    }
    if (C < 1 || C > Cp || total >= (int64_t(1) << 31)) {
        fail(kStatusUnsupported, "nchw_to_nhwc_pad: needs 1 <= C <= Cp and fewer than 2^31 pixels");
    }
    if (Cp == 4 || Cp == 8 || Cp == 16) {
        const auto c = static_cast<uint32_t>(C), hw = static_cast<uint32_t>(HW), t = static_cast<uint32_t>(total);
        auto* y4 = reinterpret_cast<float4*>(y);
        const unsigned g = blocks_for(dev, total);
        if (Cp == 4) {
            nchw_to_nhwc_narrow_kernel<4><<<g, 256, 0, dev->stream>>>(x, y4, c, hw, t);
        } else if (Cp == 8) {
            nchw_to_nhwc_narrow_kernel<8><<<g, 256, 0, dev->stream>>>(x, y4, c, hw, t);
        } else {
            nchw_to_nhwc_narrow_kernel<16><<<g, 256, 0, dev->stream>>>(x, y4, c, hw, t);
        }
    } else if (Cp % 32 == 0 && N <= 65535 && Cp / 32 <= 65535) {
        const dim3 grid(static_cast<unsigned>((HW + 31) / 32), static_cast<unsigned>(Cp / 32),
                        static_cast<unsigned>(N));
        nchw_to_nhwc_tile_kernel<<<grid, dim3(32, 8), 0, dev->stream>>>(x, y, static_cast<int>(C),
                                                                         static_cast<int>(Cp), HW);
    } else {
        fail(kStatusUnsupported, "nchw_to_nhwc_pad: Cp must be 4, 8, 16 or a multiple of 32");
    }
    check_cuda(cudaGetLastError(), "nchw_to_nhwc_pad launch");
}

void segment_copy(nb2_device* dev, const std::vector<CopySeg>& segs) {
    for (size_t base = 0; base < segs.size(); base += kMaxSegs) {
        SegTable t{};
        t.n = static_cast<int>(std::min<size_t>(kMaxSegs, segs.size() - base));
        uintptr_t bits = 0;
        int64_t most = 0;
        for (int i = 0; i < t.n; ++i) {
            t.s[i] = segs[base + i];
            bits |= reinterpret_cast<uintptr_t>(t.s[i].src) | reinterpret_cast<uintptr_t>(t.s[i].dst) |
                    static_cast<uintptr_t>(t.s[i].src_pitch) | static_cast<uintptr_t>(t.s[i].dst_pitch) |
                    static_cast<uintptr_t>(t.s[i].row_bytes);
            most = std::max(most, t.s[i].row_bytes * t.s[i].rows);
        }
        if (most == 0) {
            continue;
        }
        const bool narrow = most < (int64_t(1) << 31);
        if ((bits & 15) == 0) {
            const dim3 grid(blocks_for(dev, most / 16), t.n);
            narrow ? segment_copy_kernel<uint4, uint32_t><<<grid, 256, 0, dev->stream>>>(t)
                   : segment_copy_kernel<uint4, int64_t><<<grid, 256, 0, dev->stream>>>(t);
        } else if ((bits & 3) == 0) {
            const dim3 grid(blocks_for(dev, most / 4), t.n);
            narrow ? segment_copy_kernel<uint32_t, uint32_t><<<grid, 256, 0, dev->stream>>>(t)
                   : segment_copy_kernel<uint32_t, int64_t><<<grid, 256, 0, dev->stream>>>(t);
        } else {
            const dim3 grid(blocks_for(dev, most), t.n);
            narrow ? segment_copy_kernel<uint8_t, uint32_t><<<grid, 256, 0, dev->stream>>>(t)
                   : segment_copy_kernel<uint8_t, int64_t><<<grid, 256, 0, dev->stream>>>(t);
        }
        check_cuda(cudaGetLastError(), "segment copy launch");
    }
}

void transpose(nb2_device* dev, const void* x, void* y, const std::vector<int64_t>& in_dims,
               const std::vector<int64_t>& perm, int elem_bytes) {
    const int rank = static_cast<int>(in_dims.size());
    if (rank > 8) {
        fail(kStatusUnsupported, "Transpose: rank above 8");
    }
    int64_t n = 1;
    for (int64_t d : in_dims) {
        n *= d;
    }
    if (n == 0) {
        return;
    }
    std::vector<int64_t> in_strides(rank, 1);
    for (int d = rank - 2; d >= 0; --d) {
        in_strides[d] = in_strides[d + 1] * in_dims[d + 1];
    }
    if (elem_bytes == 4) {
        // collapse: drop unit axes, merge input axes that stay adjacent and in
        // order in the output
        std::vector<int64_t> cd;  // collapsed input extents
        std::vector<int> cperm;   // collapsed permutation
        {
            std::vector<int> keep;
            for (int d = 0; d < rank; ++d) {
                if (in_dims[d] != 1) {
                    keep.push_back(d);
                }
            }
            std::vector<int> p2; // output order over kept input axes
            for (int d = 0; d < rank; ++d) {
                if (in_dims[perm[d]] != 1) {
                    p2.push_back(static_cast<int>(perm[d]));
                }
            }
            // groups: maximal runs in p2 of consecutive kept input axes
            std::vector<std::vector<int>> groups;
            for (size_t i = 0; i < p2.size(); ++i) {
                const auto pos = std::find(keep.begin(), keep.end(), p2[i]) - keep.begin();
                if (!groups.empty()) {
                    const int last = groups.back().back();
                    const auto lpos = std::find(keep.begin(), keep.end(), last) - keep.begin();
                    if (pos == lpos + 1) {
                        groups.back().push_back(p2[i]);
                        continue;
                    }
                }
                groups.push_back({p2[i]});
            }
            // collapsed input axes are the groups ordered by their first input axis
            std::vector<int> order(groups.size());
            for (size_t i = 0; i < order.size(); ++i) {
                order[i] = static_cast<int>(i);
            }
            std::sort(order.begin(), order.end(), [&](int a, int b) { return groups[a][0] < groups[b][0]; });
            std::vector<int> in_index(groups.size());
            for (size_t j = 0; j < order.size(); ++j) {
                in_index[order[j]] = static_cast<int>(j);
                int64_t ext = 1;
                for (int a : groups[order[j]]) {
                    ext *= in_dims[a];
                }
                cd.push_back(ext);
            }
            for (size_t i = 0; i < groups.size(); ++i) {
                cperm.push_back(in_index[i]);
            }
        }
        const int cr = static_cast<int>(cd.size());
        std::vector<int64_t> cst(cr, 1);
        for (int d = cr - 2; d >= 0; --d) {
            cst[d] = cst[d + 1] * cd[d + 1];
        }
        if (cr <= 1) {
            copy(dev, x, y, n * 4);
            return;
        }
        if (cr <= 8 && cperm[cr - 1] == cr - 1 && n < (int64_t(1) << 31)) {
            // innermost axis stays: move rows
            RowPerm rp{};
            rp.rank = cr - 1;
            for (int d = 0; d < cr - 1; ++d) {
                rp.od[d] = static_cast<uint32_t>(cd[cperm[d]]);
                rp.ist[d] = cst[cperm[d]];
            }
            const int64_t L = cd[cr - 1];
            const int64_t rows = n / L;
            const bool v4 = L % 4 == 0 && ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0;
            if (v4) {
                for (int d = 0; d < rp.rank; ++d) {
                    rp.ist[d] /= 4;
                }
                permute_rows_kernel<float4><<<blocks_for(dev, n / 4), 256, 0, dev->stream>>>(
                    static_cast<const float4*>(x), static_cast<float4*>(y), rp, static_cast<uint32_t>(rows),
                    static_cast<uint32_t>(L / 4));
            } else {
                permute_rows_kernel<float><<<blocks_for(dev, n), 256, 0, dev->stream>>>(
                    static_cast<const float*>(x), static_cast<float*>(y), rp, static_cast<uint32_t>(rows),
                    static_cast<uint32_t>(L));
            }
            check_cuda(cudaGetLastError(), "transpose launch");
            return;
        }
        if (cr <= 8) {
            // tiled: u = input axis cr-1, v = the output's innermost axis
            const int v_in = cperm[cr - 1];
            int u_out = 0;
            for (int d = 0; d < cr; ++d) {
                if (cperm[d] == cr - 1) {
                    u_out = d;
                }
            }
            std::vector<int64_t> ost(cr, 1); // output strides by output axis
            for (int d = cr - 2; d >= 0; --d) {
                ost[d] = ost[d + 1] * cd[cperm[d + 1]];
            }
            TilePerm tp{};
            tp.U = cd[cr - 1];
            tp.V = cd[v_in];
            tp.in_v = cst[v_in];
            tp.out_u = ost[u_out];
            int64_t batches = 1;
            for (int d = 0; d < cr; ++d) {
                if (d == u_out || d == cr - 1) {
                    continue;
                }
                tp.bd[tp.nb] = cd[cperm[d]];
                tp.bin[tp.nb] = cst[cperm[d]];
                tp.bout[tp.nb] = ost[d];
                batches *= cd[cperm[d]];
                ++tp.nb;
            }
            const int64_t gx = (tp.U + 31) / 32, gy = (tp.V + 63) / 64;
            if (gy <= 65535) {
                const dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(gy),
                                static_cast<unsigned>(std::min<int64_t>(batches, 65535)));
                permute_tile_kernel<<<grid, dim3(32, 8), 0, dev->stream>>>(static_cast<const float*>(x),
                                                                            static_cast<float*>(y), tp, batches);
                check_cuda(cudaGetLastError(), "transpose launch");
                return;
            }
        }
    }
    // fast path: swap of the last two axes, leading axes in order
    bool last2 = rank >= 2 && perm[rank - 1] == rank - 2 && perm[rank - 2] == rank - 1;
    for (int d = 0; d < rank - 2 && last2; ++d) {
        last2 = perm[d] == d;
    }
    if (last2 && elem_bytes == 4) {
        const int64_t R = in_dims[rank - 2], C = in_dims[rank - 1];
        const int64_t B = n / (R * C);
        if (B <= 65535) {
            const dim3 grid(static_cast<unsigned>((C + 31) / 32), static_cast<unsigned>((R + 31) / 32),
                            static_cast<unsigned>(B));
            transpose_last2_kernel<float><<<grid, dim3(32, 8), 0, dev->stream>>>(static_cast<const float*>(x),
                                                                                 static_cast<float*>(y), R, C);
            check_cuda(cudaGetLastError(), "transpose launch");
            return;
        }
    }
    Dims8 od{}, st{};
    for (int d = 0; d < rank; ++d) {
        od.d[d] = in_dims[perm[d]];
        st.d[d] = in_strides[perm[d]];
    }
    const unsigned g = blocks_for(dev, n);
    if (elem_bytes == 4) {
        transpose_kernel<float><<<g, 256, 0, dev->stream>>>(static_cast<const float*>(x), static_cast<float*>(y), rank,
                                                            od, st, n);
    } else if (elem_bytes == 8) {
        transpose_kernel<long long><<<g, 256, 0, dev->stream>>>(static_cast<const long long*>(x),
                                                                static_cast<long long*>(y), rank, od, st, n);
    } else {
        transpose_kernel<uint8_t><<<g, 256, 0, dev->stream>>>(static_cast<const uint8_t*>(x),
                                                              static_cast<uint8_t*>(y), rank, od, st, n);
    }
    check_cuda(cudaGetLastError(), "transpose launch");
}

void slice(nb2_device* dev, const void* x, void* y, const std::vector<int64_t>& in_dims,
           const std::vector<int64_t>& out_dims, const std::vector<int64_t>& starts, const std::vector<int64_t>& steps,
           int elem_bytes) {
    const int rank = static_cast<int>(in_dims.size());
    if (rank > 8) {
        fail(kStatusUnsupported, "Slice: rank above 8");
    }
    int64_t n = 1;
    for (int64_t d : out_dims) {
        n *= d;
    }
    if (n == 0) {
        return;
    }
    Dims8 od{}, ist{}, s0{}, sp{};
    int64_t st = 1;
    for (int d = rank - 1; d >= 0; --d) {
        ist.d[d] = st;
        st *= in_dims[d];
        od.d[d] = out_dims[d];
        s0.d[d] = starts[d];
        sp.d[d] = steps[d];
    }
    const unsigned g = blocks_for(dev, n);
    if (elem_bytes == 4) {
        slice_kernel<float><<<g, 256, 0, dev->stream>>>(static_cast<const float*>(x), static_cast<float*>(y), rank, od,
                                                        ist, s0, sp, n);
    } else if (elem_bytes == 8) {
        slice_kernel<long long><<<g, 256, 0, dev->stream>>>(static_cast<const long long*>(x),
                                                            static_cast<long long*>(y), rank, od, ist, s0, sp, n);
    } else {
        slice_kernel<uint8_t><<<g, 256, 0, dev->stream>>>(static_cast<const uint8_t*>(x), static_cast<uint8_t*>(y),
                                                          rank, od, ist, s0, sp, n);
    }
    check_cuda(cudaGetLastError(), "slice launch");
}

void gather(nb2_device* dev, const void* x, const int64_t* idx, void* y, int64_t outer, int64_t axis_len,
            int64_t inner, int64_t n_idx, int elem_bytes) {
    const int64_t total = outer * n_idx * inner;
    if (total == 0) {
        return;
    }
    const unsigned g = blocks_for(dev, total);
    if (elem_bytes == 4) {
        gather_kernel<float><<<g, 256, 0, dev->stream>>>(static_cast<const float*>(x), idx, static_cast<float*>(y),
                                                         outer, axis_len, inner, n_idx, dev->err_word);
    } else if (elem_bytes == 8) {
        gather_kernel<long long><<<g, 256, 0, dev->stream>>>(static_cast<const long long*>(x), idx,
                                                             static_cast<long long*>(y), outer, axis_len, inner,
                                                             n_idx, dev->err_word);
    } else {
        gather_kernel<uint8_t><<<g, 256, 0, dev->stream>>>(static_cast<const uint8_t*>(x), idx,
                                                           static_cast<uint8_t*>(y), outer, axis_len, inner, n_idx,
                                                           dev->err_word);
    }
    check_cuda(cudaGetLastError(), "gather launch");
}

namespace {
// a 4-D nearest resize that keeps axes 0 and 3 (a channels-last image) with
// 16-byte channel rows
bool near_rows(const ResizeTables& t, const void* x, const void* y, int64_t n, int64_t in_numel) {
    if (t.rank != 4 || t.in_dims[3] % 4 != 0 || n >= (int64_t(1) << 31) || in_numel >= (int64_t(1) << 31) ||
        ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) != 0) {
        return false;
    }
    for (double w : t.weight) {
        if (w != 0.0) {
            return false;
        }
    }
    for (int d : {0, 3}) {
        if (t.in_dims[d] != t.out_dims[d]) {
            return false;
        }
        for (int64_t i = 0; i < t.out_dims[d]; ++i) {
            if (t.lower[t.axis_off[d] + i] != i) {
                return false;
            }
        }
    }
    return true;
}
} // namespace

void resize(nb2_device* dev, const void* x, void* y, const ResizeTables& t, const void* dev_tables, bool is_f32,
            int near2_hint) {
    ResizeDev r{};
    r.rank = t.rank;
    int64_t st = 1, n = 1;
    for (int d = t.rank - 1; d >= 0; --d) {
        r.in_strides[d] = st;
        st *= t.in_dims[d];
        r.in_dims[d] = t.in_dims[d];
        r.out_dims[d] = t.out_dims[d];
        r.axis_off[d] = t.axis_off[d];
        n *= t.out_dims[d];
    }
    const int64_t total = static_cast<int64_t>(t.lower.size());
    r.lower = static_cast<const int64_t*>(dev_tables);
    r.upper = r.lower + total;
    r.weight = reinterpret_cast<const double*>(r.upper + total);
    if (n == 0) {
        return;
    }
    const unsigned g = blocks_for(dev, n);
    // nearest, leading axes unchanged: the two-axis gather kernel
    bool near2 = t.rank >= 2 && n < (int64_t(1) << 31) && st < (int64_t(1) << 31);
    if (near2_hint >= 0) {
        near2 = near2 && near2_hint == 1;
    } else {
        for (double w : t.weight) {
            near2 = near2 && w == 0.0;
        }
        for (int d = 0; near2 && d + 2 < t.rank; ++d) {
            near2 = t.in_dims[d] == t.out_dims[d];
            for (int64_t i = 0; near2 && i < t.out_dims[d]; ++i) {
                near2 = t.lower[t.axis_off[d] + i] == i;
            }
        }
    }
    if (near2) {
        const int a = t.rank - 2, b = t.rank - 1;
        const auto H = static_cast<uint32_t>(t.in_dims[a]), W = static_cast<uint32_t>(t.in_dims[b]);
        const auto OH = static_cast<uint32_t>(t.out_dims[a]), OW = static_cast<uint32_t>(t.out_dims[b]);
        const int64_t* lh = r.lower + t.axis_off[a];
        const int64_t* lw = r.lower + t.axis_off[b];
        if (is_f32 && OW % 4 == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0) {
            const uint32_t n4 = static_cast<uint32_t>(n / 4);
            resize_nearest2_vec4_kernel<<<blocks_for(dev, n4), 256, 0, dev->stream>>>(
                static_cast<const float*>(x), static_cast<float4*>(y), lh, lw, H, W, OH, OW / 4, n4);
        } else if (is_f32) {
            resize_nearest2_kernel<float><<<g, 256, 0, dev->stream>>>(
                static_cast<const float*>(x), static_cast<float*>(y), lh, lw, H, W, OH, OW, static_cast<uint32_t>(n));
        } else {
            resize_nearest2_kernel<long long><<<g, 256, 0, dev->stream>>>(static_cast<const long long*>(x),
                                                                          static_cast<long long*>(y), lh, lw, H, W,
                                                                          OH, OW, static_cast<uint32_t>(n));
        }
    } else if (is_f32 && near_rows(t, x, y, n, st)) {
        const uint32_t n4 = static_cast<uint32_t>(n / 4);
        resize_nearest_rows_kernel<<<blocks_for(dev, n4), 256, 0, dev->stream>>>(
            static_cast<const float4*>(x), static_cast<float4*>(y), r.lower + t.axis_off[1], r.lower + t.axis_off[2],
            static_cast<uint32_t>(t.in_dims[1]), static_cast<uint32_t>(t.in_dims[2]),
            static_cast<uint32_t>(t.out_dims[1]), static_cast<uint32_t>(t.out_dims[2]),
            static_cast<uint32_t>(t.in_dims[3] / 4), n4);
    } else if (is_f32) {
        resize_kernel<float><<<g, 256, 0, dev->stream>>>(static_cast<const float*>(x), static_cast<float*>(y), r, n);
    } else {
        resize_kernel<long long><<<g, 256, 0, dev->stream>>>(static_cast<const long long*>(x),
                                                             static_cast<long long*>(y), r, n);
    }
    check_cuda(cudaGetLastError(), "resize launch");
}

namespace {

struct TableArgs {
    int rank;
    int64_t in_dims[8], out_dims[8], axis_off[8];
    double scale[8];
    int linear, transform, nearest;
    int64_t total;
};

// Per-axis sampling tables on the device: the same double-precision formulas
// as the reference (src/kernels/resize.cpp:62-107) and as the engine's
// host-built tables.
__global__ void resize_tables_kernel(TableArgs a, int64_t* lower, int64_t* upper, double* weight) {
    const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (t >= a.total) {
        return;
    }
    int d = 0;
    while (d + 1 < a.rank && t >= a.axis_off[d + 1]) {
        ++d;
    }
    const int64_t o = t - a.axis_off[d];
    const int64_t in_len = a.in_dims[d], out_len = a.out_dims[d];
    const double x = static_cast<double>(o), scale = a.scale[d];
    double xs;
    switch (a.transform) {
    case 0:
        xs = (x + 0.5) / scale - 0.5;
        break;
    case 1:
        xs = out_len > 1 ? (x + 0.5) / scale - 0.5 : 0.0;
        break;
    case 2:
        xs = out_len == 1 ? 0.0 : x * static_cast<double>(in_len - 1) / static_cast<double>(out_len - 1);
        break;
    default:
        xs = x / scale;
    }
    if (!a.linear) {
        int64_t idx;
        if (a.nearest == 0) {
            const double f = floor(xs);
            idx = static_cast<int64_t>(xs - f == 0.5 ? f : round(xs));
        } else if (a.nearest == 1) {
            idx = static_cast<int64_t>(round(xs));
        } else if (a.nearest == 2) {
            idx = static_cast<int64_t>(floor(xs));
        } else {
            idx = static_cast<int64_t>(ceil(xs));
        }
        idx = idx < 0 ? 0 : (idx > in_len - 1 ? in_len - 1 : idx);
        lower[t] = upper[t] = idx;
        weight[t] = 0.0;
        return;
    }
    const double cl = fmin(fmax(xs, 0.0), static_cast<double>(in_len - 1));
    const int64_t lo = static_cast<int64_t>(floor(cl));
    const int64_t hi = lo + 1 < in_len - 1 ? lo + 1 : in_len - 1;
    lower[t] = lo;
    upper[t] = hi;
    weight[t] = hi == lo ? 0.0 : cl - static_cast<double>(lo);
}

} // namespace

size_t resize_table_bytes(const std::vector<int64_t>& out_dims) {
    int64_t total = 0;
    for (int64_t d : out_dims) {
        total += d;
    }
    return static_cast<size_t>(total * 24);
}

void resize_on_device_tables(nb2_device* dev, const void* x, void* y, const std::vector<int64_t>& in_dims,
                             const std::vector<int64_t>& out_dims, const std::vector<double>& scales, int linear,
                             int transform, int nearest, bool is_f32, void* scratch) {
    const int rank = static_cast<int>(in_dims.size());
    if (rank > 8) {
        fail(kStatusUnsupported, "Resize: rank above 8");
    }
    TableArgs a{};
    a.rank = rank;
    a.linear = linear;
    a.transform = transform;
    a.nearest = nearest;
    ResizeTables t;
    t.rank = rank;
    t.in_dims = in_dims;
    t.out_dims = out_dims;
    int64_t total = 0;
    for (int d = 0; d < rank; ++d) {
        a.in_dims[d] = in_dims[d];
        a.out_dims[d] = out_dims[d];
        a.axis_off[d] = total;
        a.scale[d] = scales[d];
        t.axis_off.push_back(total);
        total += out_dims[d];
    }
    a.total = total;
    t.lower.resize(static_cast<size_t>(total)); // sizes only: the kernel reads the device tables
    int64_t* lower = static_cast<int64_t*>(scratch);
    resize_tables_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, dev->stream>>>(
        a, lower, lower + total, reinterpret_cast<double*>(lower + 2 * total));
    check_cuda(cudaGetLastError(), "resize tables launch");
    // a nearest resize whose leading axes keep their length at scale 1 maps
    // them to themselves under every coordinate transform and rounding (an
    // integer source coordinate rounds to itself): the two-axis kernel
    int near2 = linear == 0 ? 1 : 0;
    for (int d = 0; near2 && d + 2 < rank; ++d) {
        near2 = (in_dims[d] == out_dims[d] && scales[d] == 1.0) ? 1 : 0;
    }
    resize(dev, x, y, t, scratch, is_f32, near2);
}

void cast(nb2_device* dev, const void* x, int from, void* y, int to, int64_t n) {
    if (n == 0) {
        return;
    }
    cast_kernel<<<blocks_for(dev, n), 256, 0, dev->stream>>>(x, from, y, to, n);
    check_cuda(cudaGetLastError(), "cast launch");
}

// ---- engine hook -------------------------------------------------------------

namespace eng {

namespace {

int64_t naxis(const Node& n, int64_t a, int64_t r) {
    if (a < -r || a >= r) {
        throw LoadError(n.where() + ": axis out of range");
    }
    return a < 0 ? a + r : a;
}

// Reference Resize coordinate helpers (src/kernels/resize.cpp:62-107).
double source_coord(const std::string& mode, int64_t o, int64_t in_len, int64_t out_len, double scale) {
    const double x = static_cast<double>(o);
    if (mode == "half_pixel") {
        return (x + 0.5) / scale - 0.5;
    }
    if (mode == "pytorch_half_pixel") {
        return out_len > 1 ? (x + 0.5) / scale - 0.5 : 0.0;
    }
    if (mode == "align_corners") {
        return out_len == 1 ? 0.0 : x * static_cast<double>(in_len - 1) / static_cast<double>(out_len - 1);
    }
    if (mode == "asymmetric") {
        return x / scale;
    }
    throw LoadError("Resize: unsupported coordinate_transformation_mode '" + mode + "'");
}

int64_t nearest_index(const std::string& mode, double x, int64_t in_len) {
    int64_t index = 0;
    if (mode == "round_prefer_floor") {
        const double f = std::floor(x);
        index = static_cast<int64_t>(x - f == 0.5 ? f : std::round(x));
    } else if (mode == "round_prefer_ceil") {
        index = static_cast<int64_t>(std::round(x));
    } else if (mode == "floor") {
        index = static_cast<int64_t>(std::floor(x));
    } else if (mode == "ceil") {
        index = static_cast<int64_t>(std::ceil(x));
    } else {
        throw LoadError("Resize: unsupported nearest_mode '" + mode + "'");
    }
    return std::min(std::max(index, int64_t{0}), in_len - 1);
}

} // namespace

MoveStep build_move_step(const Node& n, const Graph& g, const std::map<std::string, TensorInfo>& shapes,
                         const std::function<void*(const std::string&)>& ptr,
                         const std::function<uint8_t*(int64_t)>& dmalloc, bool nhwc) {
    MoveStep st;
    const auto& sh = [&](const std::string& t) -> const TensorInfo& { return shapes.at(t); };
    if (nhwc && n.op != "Concat" && n.op != "Split" && n.op != "Resize") {
        throw LoadError(n.where() + ": no channels-last form of '" + n.op + "'");
    }
    // logical axis held at memory position p of a channels-last 4-D tensor
    constexpr int kLogicalAt[4] = {0, 2, 3, 1};
    auto mem_dims = [&](const std::vector<int64_t>& d) {
        if (!nhwc) {
            return d;
        }
        if (d.size() != 4) {
            throw LoadError(n.where() + ": a channels-last tensor must be 4-D");
        }
        return std::vector<int64_t>{d[0], d[2], d[3], d[1]};
    };
    auto constant = [&](size_t i) -> const Constant& {
        auto it = g.constants.find(n.inputs.at(i));
        if (it == g.constants.end()) {
            throw LoadError(n.where() + ": operand '" + n.inputs[i] + "' must be a constant");
        }
        return it->second;
    };
    if (n.op == "Transpose") {
        const TensorInfo& x = sh(n.inputs[0]);
        std::vector<int64_t> perm = n.getints("perm");
        const int64_t r = static_cast<int64_t>(x.dims.size());
        if (perm.empty()) {
            for (int64_t i = 0; i < r; ++i) {
                perm.push_back(r - 1 - i);
            }
        }
        for (auto& p : perm) {
            p = naxis(n, p, r);
        }
        const void* xp = ptr(n.inputs[0]);
        void* yp = ptr(n.outputs[0]);
        const auto dims = x.dims;
        const int eb = static_cast<int>(dtype_size(x.dtype));
        st.run = [=](nb2_device* dev) { transpose(dev, xp, yp, dims, perm, eb); };
    } else if (n.op == "Concat" || n.op == "Split") {
        const bool concat = n.op == "Concat";
        const TensorInfo& whole = concat ? sh(n.outputs[0]) : sh(n.inputs[0]);
        const int64_t r = static_cast<int64_t>(whole.dims.size());
        int64_t axis = naxis(n, n.geti("axis", 0), r);
        if (nhwc) { // the same cut in memory order: the channel axis is innermost
            axis = axis == 0 ? 0 : axis == 1 ? 3 : axis - 1;
        }
        const std::vector<int64_t> wd = mem_dims(whole.dims);
        int64_t outer = 1, inner = 1;
        for (int64_t i = 0; i < axis; ++i) {
            outer *= wd[i];
        }
        for (int64_t i = axis + 1; i < r; ++i) {
            inner *= wd[i];
        }
        const int64_t es = dtype_size(whole.dtype);
        const int64_t pitch = wd[axis] * inner * es;
        std::vector<CopySeg> segs;
        int64_t at = 0;
        uint8_t* wp = static_cast<uint8_t*>(ptr(concat ? n.outputs[0] : n.inputs[0]));
        const size_t parts = concat ? n.inputs.size() : n.outputs.size();
        for (size_t i = 0; i < parts; ++i) {
            const std::string& t = concat ? n.inputs[i] : n.outputs[i];
            const int64_t len = mem_dims(sh(t).dims)[axis];
            const int64_t rb = len * inner * es;
            uint8_t* part = static_cast<uint8_t*>(ptr(t));
            CopySeg s{};
            if (concat) {
                s = CopySeg{part, wp + at, rb, pitch, rb, outer};
            } else {
                s = CopySeg{wp + at, part, pitch, rb, rb, outer};
            }
            segs.push_back(s);
            at += rb;
        }
        st.run = [=](nb2_device* dev) { segment_copy(dev, segs); };
        st.launches = static_cast<int>((segs.size() + 63) / 64);
    } else if (n.op == "Slice") {
        const TensorInfo& x = sh(n.inputs[0]);
        const TensorInfo& y = sh(n.outputs[0]);
        const int64_t r = static_cast<int64_t>(x.dims.size());
        const std::vector<int64_t> starts = constant(1).as_i64();
        std::vector<int64_t> axes, steps;
        if (n.inputs.size() > 3 && !n.inputs[3].empty()) {
            axes = constant(3).as_i64();
        } else {
            for (size_t i = 0; i < starts.size(); ++i) {
                axes.push_back(static_cast<int64_t>(i));
            }
        }
        if (n.inputs.size() > 4 && !n.inputs[4].empty()) {
            steps = constant(4).as_i64();
        } else {
            steps.assign(starts.size(), 1);
        }
        std::vector<int64_t> s0(r, 0), sp(r, 1);
        for (size_t i = 0; i < starts.size(); ++i) {
            const int64_t a = naxis(n, axes[i], r);
            const int64_t dim = x.dims[a];
            int64_t s = starts[i] < 0 ? starts[i] + dim : starts[i];
            s = steps[i] > 0 ? std::clamp<int64_t>(s, 0, dim) : std::clamp<int64_t>(s, 0, dim - 1);
            s0[a] = s;
            sp[a] = steps[i];
        }
        const void* xp = ptr(n.inputs[0]);
        void* yp = ptr(n.outputs[0]);
        const auto xd = x.dims, yd = y.dims;
        const int eb = static_cast<int>(dtype_size(x.dtype));
        st.run = [=](nb2_device* dev) { slice(dev, xp, yp, xd, yd, s0, sp, eb); };
    } else if (n.op == "Gather") {
        const TensorInfo& x = sh(n.inputs[0]);
        const TensorInfo& idx = sh(n.inputs[1]);
        if (idx.dtype != DType::I64) {
            throw LoadError(n.where() + ": indices must be int64");
        }
        const int64_t r = static_cast<int64_t>(x.dims.size());
        const int64_t axis = naxis(n, n.geti("axis", 0), r);
        int64_t outer = 1, inner = 1;
        for (int64_t i = 0; i < axis; ++i) {
            outer *= x.dims[i];
        }
        for (int64_t i = axis + 1; i < r; ++i) {
            inner *= x.dims[i];
        }
        const int64_t alen = x.dims[axis], nidx = numel(idx.dims);
        const void* xp = ptr(n.inputs[0]);
        const int64_t* ip = static_cast<const int64_t*>(ptr(n.inputs[1]));
        void* yp = ptr(n.outputs[0]);
        const int eb = static_cast<int>(dtype_size(x.dtype));
        st.run = [=](nb2_device* dev) { gather(dev, xp, ip, yp, outer, alen, inner, nidx, eb); };
    } else if (n.op == "TopK") {
        const TensorInfo& x = sh(n.inputs[0]);
        const int64_t r = static_cast<int64_t>(x.dims.size());
        const int64_t axis = naxis(n, n.geti("axis", -1), r);
        if (axis != r - 1) {
            throw LoadError(n.where() + ": the B200 TopK row selects along the last axis");
        }
        if (n.geti("largest", 1) != 1 || n.geti("sorted", 1) != 1) {
            throw LoadError(n.where() + ": only largest=1, sorted=1 are supported (src/kernels/top_k.cpp:74-79)");
        }
        if (x.dtype != DType::F32) {
            throw LoadError(n.where() + ": input must be float32");
        }
        const int64_t k = constant(1).as_i64().at(0);
        const int64_t L = x.dims[axis];
        const int64_t rows = numel(x.dims) / std::max<int64_t>(L, 1);
        const float* xp = static_cast<const float*>(ptr(n.inputs[0]));
        float* vp = static_cast<float*>(ptr(n.outputs[0]));
        int64_t* ip = static_cast<int64_t*>(ptr(n.outputs[1]));
        const size_t sb = topk_scratch_bytes(rows, L, k);
        uint8_t* scratch = sb ? dmalloc(static_cast<int64_t>(sb)) : nullptr;
        st.launches = topk_launches(rows, L, k);
        st.run = [=](nb2_device* dev) { topk(dev, xp, vp, ip, rows, L, k, scratch); };
    } else if (n.op == "Resize") {
        const TensorInfo& x = sh(n.inputs[0]);
        const TensorInfo& y = sh(n.outputs[0]);
        const std::string mode = n.gets("mode", "nearest");
        if (mode != "nearest" && mode != "linear") {
            throw LoadError(n.where() + ": Resize 'mode' must be 'nearest' or 'linear'");
        }
        const bool linear = mode == "linear";
        const std::string transform = n.gets("coordinate_transformation_mode", "half_pixel");
        const std::string nearest = n.gets("nearest_mode", "round_prefer_floor");
        const int64_t rank = static_cast<int64_t>(x.dims.size());
        std::vector<double> scale(rank, 1.0);
        const bool has_sizes = n.inputs.size() > 3 && !n.inputs[3].empty();
        if (has_sizes) {
            for (int64_t i = 0; i < rank; ++i) {
                scale[i] = static_cast<double>(static_cast<float>(y.dims[i]) / static_cast<float>(x.dims[i]));
            }
        } else {
            const Constant& sc = constant(2);
            for (int64_t i = 0; i < rank; ++i) {
                scale[i] = static_cast<double>(sc.f32()[i]);
            }
        }
        ResizeTables t;
        t.rank = static_cast<int>(rank);
        t.in_dims = mem_dims(x.dims);
        t.out_dims = mem_dims(y.dims);
        // one table per axis, in memory order
        for (int64_t p = 0; p < rank; ++p) {
            const int64_t d = nhwc ? kLogicalAt[p] : p;
            t.axis_off.push_back(static_cast<int64_t>(t.lower.size()));
            for (int64_t o = 0; o < y.dims[d]; ++o) {
                const double xs = source_coord(transform, o, x.dims[d], y.dims[d], scale[d]);
                if (!linear) {
                    const int64_t idx = nearest_index(nearest, xs, x.dims[d]);
                    t.lower.push_back(idx);
                    t.upper.push_back(idx);
                    t.weight.push_back(0.0);
                    continue;
                }
                const double cl = std::min(std::max(xs, 0.0), static_cast<double>(x.dims[d] - 1));
                const int64_t lo = static_cast<int64_t>(std::floor(cl));
                const int64_t hi = std::min(lo + 1, x.dims[d] - 1);
                t.lower.push_back(lo);
                t.upper.push_back(hi);
                t.weight.push_back(hi == lo ? 0.0 : cl - static_cast<double>(lo));
            }
        }
        const int64_t tn = static_cast<int64_t>(t.lower.size());
        uint8_t* tables = dmalloc(tn * 24);
        std::vector<uint8_t> host(static_cast<size_t>(tn * 24));
        std::memcpy(host.data(), t.lower.data(), tn * 8);
        std::memcpy(host.data() + tn * 8, t.upper.data(), tn * 8);
        std::memcpy(host.data() + tn * 16, t.weight.data(), tn * 8);
        check_cuda(cudaMemcpy(tables, host.data(), host.size(), cudaMemcpyHostToDevice), "cudaMemcpy(resize tables)");
        // a pageable cudaMemcpy may return before its DMA (on the legacy
        // stream) lands; the rows run on the non-blocking device stream
        check_cuda(cudaStreamSynchronize(0), "cudaStreamSynchronize(legacy)");
        const void* xp = ptr(n.inputs[0]);
        void* yp = ptr(n.outputs[0]);
        const bool f32 = x.dtype == DType::F32;
        st.run = [=](nb2_device* dev) { resize(dev, xp, yp, t, tables, f32); };
    } else if (n.op == "Cast") {
        const TensorInfo& x = sh(n.inputs[0]);
        const TensorInfo& y = sh(n.outputs[0]);
        const void* xp = ptr(n.inputs[0]);
        void* yp = ptr(n.outputs[0]);
        const int from = static_cast<int>(x.dtype), to = static_cast<int>(y.dtype);
        const int64_t cnt = numel(x.dims);
        st.run = [=](nb2_device* dev) { cast(dev, xp, from, yp, to, cnt); };
    }
    return st;
}

} // namespace eng

} // namespace nb2
