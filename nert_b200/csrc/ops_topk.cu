// TopK row (largest=1, sorted=1): radix select + bitonic sort.
//
// Reference semantics (src/kernels/top_k.cpp:53-142): the k largest values of
// each row along the last axis, ordered by (value desc, index asc), with int64
// indices. The reference CUDA row runs one thread per row with O(k^2 * L)
// repeated selection (src/cuda/top_k.cu:49-77) and reads K back with a
// device->host copy (:112); here K is a load-time constant.
//
// Floats map to order-preserving uint32 keys (-0 folded onto +0 so equal
// values tie and fall back to index order, as in the reference). The exact
// key T of the k-th largest value is found digit by digit (11, 11, 10 bits);
// every key > T is selected, and of the keys == T only the `need` smallest
// indices (chunks are visited in index order), so ties resolve exactly as the
// reference's stable order does. The k winners are then bitonic-sorted in
// shared memory.
//
// Short rows (L < kSplitMin) use one 1024-thread CTA per row. Long rows (the
// detector's 8400*80 scores) are split over many CTAs per row: each digit pass
// is a grid-wide histogram with warp-aggregated shared-memory atomics, and the
// digit selection is recomputed from the histograms by every CTA of the next
// pass, so no separate selection launch is needed.

#include "ops_move.cuh"

namespace nb2 {

namespace {

constexpr int kThreads = 1024;
constexpr int kMaxK = 1024;
constexpr int64_t kSplitMin = 16384;
constexpr int kChunk = 8192;     // elements per CTA in the split path
constexpr int kBins = 2048;

__device__ __forceinline__ uint32_t key_of(float f) {
    uint32_t u = __float_as_uint(f);
    if (u == 0x80000000u) {
        u = 0; // -0 == +0
    }
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Sorts cand_key/cand_idx[0..sort_n) best-first: larger key, then smaller index.
__device__ void bitonic_best_first(uint32_t* cand_key, int64_t* cand_idx, int sort_n) {
    for (int size = 2; size <= sort_n; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < sort_n; i += blockDim.x) {
                const int j = i ^ stride;
                if (j > i) {
                    const bool desc = (i & size) == 0;
                    const uint32_t ki = cand_key[i], kj = cand_key[j];
                    const int64_t ii = cand_idx[i], ij = cand_idx[j];
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
}

// ---- single-CTA path ---------------------------------------------------------

__global__ void __launch_bounds__(kThreads) topk_row_kernel(const float* __restrict__ x, float* __restrict__ values,
                                                             int64_t* __restrict__ indices, int64_t L, int k,
                                                             int sort_n) {
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
            const int need = s_need;
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
    const int need_eq = s_need;
    const int gt_total = k - need_eq;
    if (tid == 0) {
        s_gt_count = 0;
        s_eq_base = 0;
    }
    __syncthreads();
    const int lane = tid & 31, warp = tid >> 5;
    for (int64_t base = 0; base < L; base += kThreads) {
        const int64_t i = base + tid;
        const bool valid = i < L;
        const uint32_t key = valid ? key_of(__ldg(row + i)) : 0u;
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
    for (int i = k + tid; i < sort_n; i += kThreads) {
        cand_key[i] = 0;
        cand_idx[i] = INT64_MAX;
    }
    __syncthreads();
    bitonic_best_first(cand_key, cand_idx, sort_n);
    for (int i = tid; i < k; i += kThreads) {
        const int64_t idx = cand_idx[i];
        values[blockIdx.x * (int64_t)k + i] = row[idx];
        indices[blockIdx.x * (int64_t)k + i] = idx;
    }
}

// ---- split path ----------------------------------------------------------------

// Digit passes: bits [21,32), [10,21), [0,10).
__device__ __forceinline__ int digit_shift(int pass) { return pass == 0 ? 21 : pass == 1 ? 10 : 0; }
__device__ __forceinline__ uint32_t digit_mask(int pass) { return pass == 2 ? 1023u : 2047u; }

// Replays the digit selection of passes [0, pass) from the row's histograms:
// returns the key prefix, its mask and how many keys equal to the prefix are
// still needed. Deterministic, so every CTA of a row agrees.
// Block-parallel: each of the 512 threads owns 4 bins; a suffix sum over the
// threads (warp shuffles + one shared-memory pass) locates the bin holding
// the need-th largest key.
__device__ void select_prefix(const uint32_t* __restrict__ hist_row, int pass, int k, uint32_t& prefix,
                              uint32_t& mask, int& need) {
    __shared__ uint32_t s_prefix, s_mask;
    __shared__ int s_need;
    __shared__ uint32_t warp_tot[16];
    __shared__ int s_sel, s_cum;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) {
        s_prefix = 0;
        s_mask = 0;
        s_need = k;
    }
    __syncthreads();
    for (int q = 0; q < pass; ++q) {
        const uint32_t* h = hist_row + q * kBins;
        const int nbins = static_cast<int>(digit_mask(q)) + 1;
        uint32_t c[4];
        uint32_t mine = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int bin = tid * 4 + j;
            c[j] = bin < nbins ? __ldg(h + bin) : 0u;
            mine += c[j];
        }
        // inclusive suffix sum over lanes (higher lanes own higher bins)
        uint32_t suf = mine;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t v = __shfl_down_sync(0xffffffffu, suf, o);
            if (lane + o < 32) {
                suf += v;
            }
        }
        if (lane == 0) {
            warp_tot[warp] = suf;
        }
        __syncthreads();
        uint32_t above = suf - mine; // bins of higher lanes in this warp
        for (int w = warp + 1; w < static_cast<int>(blockDim.x / 32); ++w) {
            above += warp_tot[w];
        }
        const int nd = s_need;
        if (above < static_cast<uint32_t>(nd) && above + mine >= static_cast<uint32_t>(nd)) {
            uint32_t cum = above;
#pragma unroll
            for (int j = 3; j >= 0; --j) {
                if (cum + c[j] >= static_cast<uint32_t>(nd)) {
                    s_sel = tid * 4 + j;
                    s_cum = static_cast<int>(cum);
                    break;
                }
                cum += c[j];
            }
        }
        __syncthreads();
        if (tid == 0) {
            s_need = nd - s_cum;
            s_prefix |= static_cast<uint32_t>(s_sel) << digit_shift(q);
            s_mask |= digit_mask(q) << digit_shift(q);
        }
        __syncthreads();
    }
    prefix = s_prefix;
    mask = s_mask;
    need = s_need;
}

// grid (chunks, rows): histogram of digit `pass` over keys matching the
// prefix chosen by the earlier passes.
__global__ void __launch_bounds__(512) topk_hist_kernel(const float* __restrict__ x, int64_t L, int k, int pass,
                                                         uint32_t* __restrict__ hist) {
    __shared__ uint32_t h[kBins];
    const int64_t row = blockIdx.y;
    uint32_t* hist_row = hist + row * 3 * kBins;
    for (int i = threadIdx.x; i < kBins; i += blockDim.x) {
        h[i] = 0;
    }
    uint32_t prefix, mask;
    int need;
    select_prefix(hist_row, pass, k, prefix, mask, need);
    const int sh = digit_shift(pass);
    const uint32_t dm = digit_mask(pass);
    const float* r = x + row * L;
    const int64_t begin = static_cast<int64_t>(blockIdx.x) * kChunk;
    const int64_t end = min(begin + kChunk, L);
    // four loads in flight per thread (coalesced across the block), then
    // their histogram updates
    const int64_t step = blockDim.x;
    for (int64_t i0 = begin + threadIdx.x; i0 < end; i0 += 4 * step) {
        float v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t i = i0 + u * step;
            v[u] = i < end ? __ldg(r + i) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const bool in = i0 + u * step < end;
            const uint32_t key = key_of(v[u]);
            if (in && (key & mask) == prefix) {
                const uint32_t bin = (key >> sh) & dm;
                // warp-aggregated increment: one atomic per distinct bin in the warp
                const unsigned active = __activemask();
                const unsigned peers = __match_any_sync(active, bin);
                if ((__ffs(peers) - 1) == static_cast<int>(threadIdx.x & 31)) {
                    atomicAdd(&h[bin], static_cast<uint32_t>(__popc(peers)));
                }
            }
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < kBins; i += blockDim.x) {
        if (h[i]) {
            atomicAdd(&hist_row[pass * kBins + i], h[i]);
        }
    }
}

// grid (chunks, rows): how many keys of each chunk equal T.
__global__ void __launch_bounds__(512) topk_eqcount_kernel(const float* __restrict__ x, int64_t L, int k,
                                                            const uint32_t* __restrict__ hist,
                                                            int* __restrict__ eq_counts, int chunks) {
    __shared__ int s_count;
    const int64_t row = blockIdx.y;
    uint32_t T, mask;
    int need;
    select_prefix(hist + row * 3 * kBins, 3, k, T, mask, need);
    if (threadIdx.x == 0) {
        s_count = 0;
    }
    __syncthreads();
    const float* r = x + row * L;
    const int64_t begin = static_cast<int64_t>(blockIdx.x) * kChunk;
    const int64_t end = min(begin + kChunk, L);
    int c = 0;
    const int64_t step = blockDim.x;
    for (int64_t i0 = begin + threadIdx.x; i0 < end; i0 += 4 * step) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t i = i0 + u * step;
            c += (i < end && key_of(__ldg(r + i)) == T) ? 1 : 0;
        }
    }
    c = __reduce_add_sync(0xffffffffu, c);
    if ((threadIdx.x & 31) == 0 && c) {
        atomicAdd(&s_count, c);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        eq_counts[row * chunks + blockIdx.x] = s_count;
    }
}

// grid (chunks, rows): every key > T, and the keys == T whose rank in index
// order is below `need`, go to the row's candidate list.
__global__ void __launch_bounds__(512) topk_collect_kernel(const float* __restrict__ x, int64_t L, int k,
                                                            const uint32_t* __restrict__ hist,
                                                            const int* __restrict__ eq_counts, int chunks,
                                                            int* __restrict__ gt_count, uint32_t* __restrict__ cand_key,
                                                            int64_t* __restrict__ cand_idx) {
    __shared__ int warp_counts[16];
    __shared__ int s_base;
    const int64_t row = blockIdx.y;
    uint32_t T, mask;
    int need;
    select_prefix(hist + row * 3 * kBins, 3, k, T, mask, need);
    const int gt_total = k - need;
    if (threadIdx.x == 0) {
        int b = 0;
        for (int c = 0; c < static_cast<int>(blockIdx.x); ++c) {
            b += eq_counts[row * chunks + c];
        }
        s_base = b;
    }
    __syncthreads();
    int eq_base = s_base;
    const float* r = x + row * L;
    uint32_t* ck = cand_key + row * k;
    int64_t* ci = cand_idx + row * k;
    const int64_t begin = static_cast<int64_t>(blockIdx.x) * kChunk;
    const int64_t end = min(begin + kChunk, L);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int64_t base = begin; base < end; base += blockDim.x) {
        const int64_t i = base + threadIdx.x;
        const bool valid = i < end;
        const uint32_t key = valid ? key_of(__ldg(r + i)) : 0u;
        if (valid && key > T) {
            const int slot = atomicAdd(&gt_count[row], 1);
            ck[slot] = key;
            ci[slot] = i;
        }
        const bool eq = valid && key == T;
        const unsigned ballot = __ballot_sync(0xffffffffu, eq);
        if (lane == 0) {
            warp_counts[warp] = __popc(ballot);
        }
        __syncthreads();
        if (eq) {
            int before = __popc(ballot & ((1u << lane) - 1u));
            for (int w = 0; w < warp; ++w) {
                before += warp_counts[w];
            }
            const int rk = eq_base + before;
            if (rk < need) {
                ck[gt_total + rk] = key;
                ci[gt_total + rk] = i;
            }
        }
        int tot = 0;
        for (int w = 0; w < static_cast<int>(blockDim.x / 32); ++w) {
            tot += warp_counts[w];
        }
        eq_base += tot;
        __syncthreads();
    }
}

// grid rows: sort the k candidates and write values / indices.
__global__ void __launch_bounds__(kThreads) topk_sort_kernel(const float* __restrict__ x, int64_t L, int k,
                                                              int sort_n, const uint32_t* __restrict__ cand_key,
                                                              const int64_t* __restrict__ cand_idx,
                                                              float* __restrict__ values,
                                                              int64_t* __restrict__ indices) {
    __shared__ uint32_t sk[kMaxK];
    __shared__ int64_t si[kMaxK];
    const int64_t row = blockIdx.x;
    for (int i = threadIdx.x; i < sort_n; i += blockDim.x) {
        sk[i] = i < k ? cand_key[row * k + i] : 0u;
        si[i] = i < k ? cand_idx[row * k + i] : INT64_MAX;
    }
    __syncthreads();
    bitonic_best_first(sk, si, sort_n);
    for (int i = threadIdx.x; i < k; i += blockDim.x) {
        values[row * k + i] = x[row * L + si[i]];
        indices[row * k + i] = si[i];
    }
}

} // namespace

size_t topk_scratch_bytes(int64_t rows, int64_t L, int64_t k) {
    if (L < kSplitMin) {
        return 0;
    }
    const int64_t chunks = (L + kChunk - 1) / kChunk;
    const size_t hist = static_cast<size_t>(rows) * 3 * kBins * 4;
    const size_t eq = static_cast<size_t>(rows * chunks) * 4;
    const size_t gt = static_cast<size_t>(rows) * 4;
    const size_t cand = static_cast<size_t>(rows * k) * 12;
    return ((hist + eq + gt + 255) / 256) * 256 + cand + 256;
}

void topk(nb2_device* dev, const float* x, float* values, int64_t* indices, int64_t rows, int64_t L, int64_t k,
          void* scratch) {
    if (rows == 0 || k == 0) {
        return;
    }
    if (k > kMaxK) {
        fail(kStatusUnsupported, "TopK: K above 1024 is not supported on B200");
    }
    if (k > L) {
        fail(kStatusInvalid, "TopK: K is larger than the axis");
    }
    if (rows > 65535) {
        fail(kStatusUnsupported, "TopK: more than 65535 rows");
    }
    int sort_n = 1;
    while (sort_n < k) {
        sort_n <<= 1;
    }
    if (L < kSplitMin) {
        topk_row_kernel<<<static_cast<unsigned>(rows), kThreads, 0, dev->stream>>>(x, values, indices, L,
                                                                                   static_cast<int>(k), sort_n);
        check_cuda(cudaGetLastError(), "topk launch");
        return;
    }
    if (scratch == nullptr) {
        fail(kStatusInvalid, "TopK: long rows need scratch memory");
    }
    const int chunks = static_cast<int>((L + kChunk - 1) / kChunk);
    auto* hist = static_cast<uint32_t*>(scratch);
    int* eq_counts = reinterpret_cast<int*>(hist + rows * 3 * kBins);
    int* gt_count = eq_counts + rows * chunks;
    const size_t head = ((static_cast<size_t>(rows) * 3 * kBins * 4 + static_cast<size_t>(rows * chunks) * 4 +
                          static_cast<size_t>(rows) * 4 + 255) / 256) * 256;
    auto* cand_idx = reinterpret_cast<int64_t*>(static_cast<uint8_t*>(scratch) + head);
    auto* cand_key = reinterpret_cast<uint32_t*>(cand_idx + rows * k);
    check_cuda(cudaMemsetAsync(scratch, 0, head, dev->stream), "topk scratch clear");
    const dim3 grid(static_cast<unsigned>(chunks), static_cast<unsigned>(rows));
    const int ki = static_cast<int>(k);
    for (int pass = 0; pass < 3; ++pass) {
        topk_hist_kernel<<<grid, 512, 0, dev->stream>>>(x, L, ki, pass, hist);
    }
    topk_eqcount_kernel<<<grid, 512, 0, dev->stream>>>(x, L, ki, hist, eq_counts, chunks);
    topk_collect_kernel<<<grid, 512, 0, dev->stream>>>(x, L, ki, hist, eq_counts, chunks, gt_count, cand_key,
                                                       cand_idx);
    topk_sort_kernel<<<static_cast<unsigned>(rows), kThreads, 0, dev->stream>>>(x, L, ki, sort_n, cand_key,
                                                                                cand_idx, values, indices);
    check_cuda(cudaGetLastError(), "topk launch");
}

} // namespace nb2
