// TopK row (largest=1, sorted=1): block-level radix select + bitonic sort.
//
// Reference semantics (src/kernels/top_k.cpp:53-142): the k largest values of
// each row along the last axis, ordered by (value desc, index asc), with int64
// indices. The reference CUDA row runs one thread per row with O(k^2 * L)
// repeated selection (src/cuda/top_k.cu:49-77) and reads K back with a
// device->host copy (:112); here K is a load-time constant.
//
// One CTA per row:
//   1. floats map to order-preserving uint32 keys (-0 folded onto +0 so equal
//      values tie and fall back to index order, as in the reference);
//   2. four 8-bit radix passes find the exact key T of the k-th largest value
//      and how many elements equal to T are needed;
//   3. one pass collects every key > T, and the needed keys == T in index
//      order (block prefix counts per tile), so ties keep the smallest indices;
//   4. a shared-memory bitonic sort orders the k winners.

#include "ops_move.cuh"

namespace nb2 {

namespace {

constexpr int kThreads = 1024;
constexpr int kMaxK = 1024;

__device__ __forceinline__ uint32_t key_of(float f) {
    uint32_t u = __float_as_uint(f);
    if (u == 0x80000000u) {
        u = 0; // -0 == +0
    }
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__global__ void __launch_bounds__(kThreads) topk_kernel(const float* __restrict__ x, float* __restrict__ values,
                                                         int64_t* __restrict__ indices, int64_t L, int k, int sort_n) {
    __shared__ uint32_t hist[256];
    __shared__ uint32_t s_prefix, s_mask;
    __shared__ int s_need, s_gt_count, s_eq_base;
    __shared__ uint32_t cand_key[kMaxK];
    __shared__ int64_t cand_idx[kMaxK];
    __shared__ int warp_counts[kThreads / 32];

    const float* row = x + blockIdx.x * L;
    const int tid = threadIdx.x;
    if (tid == 0) {
        s_prefix = 0;
        s_mask = 0;
        s_need = k;
    }
    __syncthreads();

    // ---- radix select
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = tid; i < 256; i += kThreads) {
            hist[i] = 0;
        }
        __syncthreads();
        const uint32_t prefix = s_prefix, mask = s_mask;
        for (int64_t i = tid; i < L; i += kThreads) {
            const uint32_t key = key_of(__ldg(row + i));
            if ((key & mask) == prefix) {
                atomicAdd(&hist[(key >> shift) & 255u], 1u);
            }
        }
        __syncthreads();
        if (tid == 0) {
            int need = s_need;
            uint32_t cum = 0;
            int sel = 0;
            for (int d = 255; d >= 0; --d) {
                if (cum + hist[d] >= static_cast<uint32_t>(need)) {
                    sel = d;
                    break;
                }
                cum += hist[d];
            }
            s_need = need - static_cast<int>(cum);
            s_prefix = prefix | (static_cast<uint32_t>(sel) << shift);
            s_mask = mask | (255u << shift);
        }
        __syncthreads();
    }
    const uint32_t T = s_prefix;
    const int need_eq = s_need;  // how many keys == T to take (smallest indices)
    const int gt_total = k - need_eq;
    if (tid == 0) {
        s_gt_count = 0;
        s_eq_base = 0;
    }
    __syncthreads();

    // ---- collect: keys > T anywhere; keys == T in index order
    const int lane = tid & 31, warp = tid >> 5;
    for (int64_t base = 0; base < L; base += kThreads) {
        const int64_t i = base + tid;
        uint32_t key = 0;
        bool valid = i < L;
        if (valid) {
            key = key_of(__ldg(row + i));
        }
        if (valid && key > T) {
            const int slot = atomicAdd(&s_gt_count, 1);
            cand_key[slot] = key;
            cand_idx[slot] = i;
        }
        const bool eq = valid && key == T;
        const unsigned ballot = __ballot_sync(0xffffffffu, eq);
        if (lane == 0) {
            warp_counts[warp] = __popc(ballot);
        }
        __syncthreads();
        const int eq_base = s_eq_base;
        if (eq && eq_base < need_eq) {
            int before = __popc(ballot & ((1u << lane) - 1u));
            for (int w = 0; w < warp; ++w) {
                before += warp_counts[w];
            }
            const int r = eq_base + before;
            if (r < need_eq) {
                cand_key[gt_total + r] = key;
                cand_idx[gt_total + r] = i;
            }
        }
        __syncthreads();
        if (tid == 0) {
            int tot = 0;
            for (int w = 0; w < kThreads / 32; ++w) {
                tot += warp_counts[w];
            }
            s_eq_base = eq_base + tot;
        }
        __syncthreads();
    }

    // ---- bitonic sort of sort_n (power of two >= k) entries, padded below everything
    for (int i = k + tid; i < sort_n; i += kThreads) {
        cand_key[i] = 0;
        cand_idx[i] = INT64_MAX;
    }
    __syncthreads();
    for (int size = 2; size <= sort_n; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = tid; i < sort_n; i += kThreads) {
                const int j = i ^ stride;
                if (j > i) {
                    const bool desc = (i & size) == 0; // this block sorted "best first"
                    const uint32_t ki = cand_key[i], kj = cand_key[j];
                    const int64_t ii = cand_idx[i], ij = cand_idx[j];
                    // "a before b" means larger key, or equal key and smaller index
                    const bool j_first = kj > ki || (kj == ki && ij < ii);
                    if (j_first == desc) {
                        cand_key[i] = kj;
                        cand_key[j] = ki;
                        cand_idx[i] = ij;
                        cand_idx[j] = ii;
                    }
                }
            }
            __syncthreads();
        }
    }
    for (int i = tid; i < k; i += kThreads) {
        const int64_t idx = cand_idx[i];
        values[blockIdx.x * (int64_t)k + i] = row[idx];
        indices[blockIdx.x * (int64_t)k + i] = idx;
    }
}

} // namespace

void topk(nb2_device* dev, const float* x, float* values, int64_t* indices, int64_t rows, int64_t L, int64_t k) {
    if (rows == 0 || k == 0) {
        return;
    }
    if (k > kMaxK) {
        fail(kStatusUnsupported, "TopK: K above 1024 is not supported on B200");
    }
    if (k > L) {
        fail(kStatusInvalid, "TopK: K is larger than the axis");
    }
    if (rows > 2147483647LL) {
        fail(kStatusUnsupported, "TopK: too many rows");
    }
    int sort_n = 1;
    while (sort_n < k) {
        sort_n <<= 1;
    }
    topk_kernel<<<static_cast<unsigned>(rows), kThreads, 0, dev->stream>>>(x, values, indices, L, static_cast<int>(k),
                                                                            sort_n);
    check_cuda(cudaGetLastError(), "topk launch");
}

} // namespace nb2
