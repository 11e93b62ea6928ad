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
// detector's 8400*80 scores) first take the sampled-threshold path: one read
// of the row keeps every key at or above a threshold drawn from a sample, and
// the few thousand survivors are ranked exactly. A row for which that cannot
// be exact (fewer than k survivors, or more than the candidate list holds,
// e.g. a flood of equal values) is redone by the radix passes: each digit
// pass is a grid-wide histogram with warp-aggregated shared-memory atomics,
// and the digit selection is recomputed from the histograms by every CTA of
// the next pass, so no separate selection launch is needed.

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
                                                         uint32_t* __restrict__ hist, const int* __restrict__ done) {
    __shared__ uint32_t h[kBins];
    const int64_t row = blockIdx.y;
    if (done != nullptr && done[row]) {
        return; // finished by the sampled-threshold path
    }
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
                                                            int* __restrict__ eq_counts, int chunks,
                                                            const int* __restrict__ done) {
    __shared__ int s_count;
    const int64_t row = blockIdx.y;
    if (done != nullptr && done[row]) {
        return;
    }
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
                                                            int64_t* __restrict__ cand_idx,
                                                            const int* __restrict__ done) {
    __shared__ int warp_counts[16];
    __shared__ int s_base;
    const int64_t row = blockIdx.y;
    if (done != nullptr && done[row]) {
        return;
    }
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
                                                              int64_t* __restrict__ indices,
                                                              const int* __restrict__ done) {
    __shared__ uint32_t sk[kMaxK];
    __shared__ int64_t si[kMaxK];
    const int64_t row = blockIdx.x;
    if (done != nullptr && done[row]) {
        return;
    }
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


// grid (ceil(k / 256), rows), 256 threads: K above kMaxK. Each thread places
// one of the row's k candidates at its rank in (key desc, index asc) order,
// counting the candidates that precede it (staged through shared memory).
__global__ void __launch_bounds__(256) topk_rank_kernel(const float* __restrict__ x, int64_t L, int k,
                                                         const uint32_t* __restrict__ cand_key,
                                                         const int64_t* __restrict__ cand_idx,
                                                         float* __restrict__ values, int64_t* __restrict__ indices) {
    __shared__ uint32_t sk[1024];
    __shared__ int64_t si[1024];
    const int64_t row = blockIdx.y;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t* ck = cand_key + row * k;
    const int64_t* ci = cand_idx + row * k;
    const uint32_t mk = i < k ? ck[i] : 0u;
    const int64_t mi = i < k ? ci[i] : 0;
    int rank = 0;
    for (int base = 0; base < k; base += 1024) {
        const int n = min(1024, k - base);
        __syncthreads();
        for (int q = threadIdx.x; q < n; q += blockDim.x) {
            sk[q] = ck[base + q];
            si[q] = ci[base + q];
        }
        __syncthreads();
        for (int q = 0; q < n; ++q) {
            rank += (sk[q] > mk || (sk[q] == mk && si[q] < mi)) ? 1 : 0;
        }
    }
    if (i < k) {
        values[row * k + rank] = x[row * L + mi];
        indices[row * k + rank] = mi;
    }
}

// ---- sampled-threshold path for long rows --------------------------------------
//
// One read of the row instead of five: a threshold t is taken from a sample
// of the row (kSampleBlocks contiguous blocks spread over it) as its j-th
// largest key, with j sized so that about 4k keys of the full row reach t;
// every key >= t is appended to a candidate list; the candidates are sorted
// by (key desc, index asc) and the first k written. Exact whenever at least k
// keys reach t (then the k-th largest key T >= t, so every key >= T, ties
// included, is a candidate) and the list did not overflow; a row for which
// either fails is flagged and redone by the radix passes above.

constexpr int kSampleBlocks = 32;
constexpr int kSampleBlock = 1024;
constexpr int kSample = kSampleBlocks * kSampleBlock;
constexpr int kCandCap = 2048;
constexpr int kSampledMaxK = 384; // largest k the sampled path takes
constexpr int kFilterChunk = 16384;

__device__ __forceinline__ int64_t sample_pos(int64_t L, int i) {
    const int b = i / kSampleBlock;
    const int64_t start = (L - kSampleBlock) * b / (kSampleBlocks - 1);
    return start + (i - b * kSampleBlock);
}

// Exact key of rank j (1 = largest) among keys[0..n) in shared memory, by
// three digit passes over a 2048-bin histogram (warp-aggregated atomics).
// Every thread of the block calls it; returns the key and how many keys
// greater than it there are.
__device__ uint32_t block_kth_key(const uint32_t* keys, int n, int j, uint32_t* hist, int* n_greater) {
    __shared__ uint32_t s_prefix, s_mask;
    __shared__ int s_need;
    __shared__ uint32_t lane_tot[32];
    const int tid = threadIdx.x;
    if (tid == 0) {
        s_prefix = 0;
        s_mask = 0;
        s_need = j;
    }
    for (int pass = 0; pass < 3; ++pass) {
        for (int i = tid; i < kBins; i += blockDim.x) {
            hist[i] = 0;
        }
        __syncthreads();
        const uint32_t prefix = s_prefix, mask = s_mask;
        const int sh = digit_shift(pass);
        const uint32_t dm = digit_mask(pass);
        for (int base = 0; base < n; base += blockDim.x) {
            const int i = base + tid;
            const bool in = i < n && (keys[i] & mask) == prefix;
            const uint32_t bin = in ? (keys[i] >> sh) & dm : 0xFFFFFFFFu;
            const unsigned peers = __match_any_sync(0xffffffffu, bin);
            if (in && (__ffs(peers) - 1) == (tid & 31)) {
                atomicAdd(&hist[bin], static_cast<uint32_t>(__popc(peers)));
            }
        }
        __syncthreads();
        {
            // Block-parallel bin search: each thread owns kBins / blockDim.x
            // consecutive bins; a suffix sum over the threads (larger keys in
            // higher bins) finds the one thread whose range holds the bin
            // where the count from the top reaches `need`.
            const int lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
            const int per = kBins / static_cast<int>(blockDim.x);
            const int b0 = tid * per;
            const uint32_t need = static_cast<uint32_t>(s_need);
            uint32_t mine = 0;
            for (int b = 0; b < per; ++b) {
                mine += hist[b0 + b];
            }
            uint32_t suf = mine; // inclusive suffix within the warp
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t v = __shfl_down_sync(0xffffffffu, suf, o);
                suf += lane + o < 32 ? v : 0u;
            }
            if (lane == 0) {
                lane_tot[warp] = suf; // the warp's total
            }
            __syncthreads();
            uint32_t above_w = 0;
            for (int w = warp + 1; w < nwarps; ++w) {
                above_w += lane_tot[w];
            }
            const uint32_t incl = suf + above_w, excl = incl - mine;
            if (excl < need && need <= incl) {
                uint32_t above = excl;
                int sel = b0;
                for (int b = b0 + per - 1; b >= b0; --b) {
                    if (above + hist[b] >= need) {
                        sel = b;
                        break;
                    }
                    above += hist[b];
                }
                s_need = static_cast<int>(need - above);
                s_prefix |= static_cast<uint32_t>(sel) << sh;
                s_mask |= dm << sh;
            }
        }
        __syncthreads();
    }
    *n_greater = j - s_need;
    return s_prefix;
}

// grid rows, 1024 threads: thread i takes the i-th element of every sample
// block (kSampleBlocks values spread over the row) and keeps their largest
// key; thresh[row] = the j-th largest of those 1024 maxima. At least j
// sampled keys reach it, and a sampled key seldom shares its thread with
// another top one, so about j * L / kSample keys of the row reach it.
__global__ void __launch_bounds__(kThreads) topk_sample_kernel(const float* __restrict__ x, int64_t L, int j,
                                                                uint32_t* __restrict__ thresh) {
    __shared__ uint32_t keys[kThreads];
    __shared__ uint32_t hist[kBins];
    const float* r = x + blockIdx.x * L;
    const int tid = threadIdx.x;
    uint32_t best = 0;
#pragma unroll 8
    for (int q = 0; q < kSampleBlocks; ++q) {
        best = max(best, key_of(__ldg(r + sample_pos(L, q * kThreads + tid))));
    }
    keys[tid] = best;
    __syncthreads();
    int greater = 0;
    const uint32_t t = block_kth_key(keys, kThreads, j, hist, &greater);
    if (tid == 0) {
        thresh[blockIdx.x] = t;
    }
}

// grid (chunks, rows), 256 threads: append every key >= thresh[row] with its
// index (one atomic per warp and load round).
__global__ void __launch_bounds__(256) topk_filter_kernel(const float* __restrict__ x, int64_t L,
                                                           const uint32_t* __restrict__ thresh,
                                                           int* __restrict__ count, uint32_t* __restrict__ cand_key,
                                                           int64_t* __restrict__ cand_idx, int vec4) {
    const int64_t row = blockIdx.y;
    const uint32_t t = thresh[row];
    const float* r = x + row * L;
    const int64_t begin = static_cast<int64_t>(blockIdx.x) * kFilterChunk;
    const int64_t end = min(begin + kFilterChunk, L);
    const int lane = threadIdx.x & 31;
    uint32_t* ck = cand_key + row * kCandCap;
    int64_t* ci = cand_idx + row * kCandCap;
    auto emit = [&](bool hit, uint32_t key, int64_t i) {
        const unsigned ballot = __ballot_sync(0xffffffffu, hit);
        if (ballot == 0u) {
            return;
        }
        int base = 0;
        if (lane == 0) {
            base = atomicAdd(&count[row], __popc(ballot));
        }
        base = __shfl_sync(0xffffffffu, base, 0);
        if (hit) {
            const int slot = base + __popc(ballot & ((1u << lane) - 1u));
            if (slot < kCandCap) {
                ck[slot] = key;
                ci[slot] = i;
            }
        }
    };
    if (vec4) {
        const float4* r4 = reinterpret_cast<const float4*>(r);
        // four float4 per thread in flight per round
        for (int64_t q0 = begin / 4 + threadIdx.x; q0 * 4 < end; q0 += 4 * blockDim.x) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int64_t q = q0 + u * blockDim.x;
                v[u] = q * 4 < end ? __ldg(r4 + q) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int64_t q = q0 + u * blockDim.x;
                const bool in = q * 4 < end;
                const float f[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
                const bool any = in && (key_of(f[0]) >= t || key_of(f[1]) >= t || key_of(f[2]) >= t ||
                                        key_of(f[3]) >= t);
                if (__ballot_sync(0xffffffffu, any) == 0u) {
                    continue; // nearly every round: nothing in this warp reaches t
                }
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const uint32_t key = key_of(f[c]);
                    emit(in && key >= t, key, q * 4 + c);
                }
            }
        }
    } else {
        for (int64_t i0 = begin + threadIdx.x; i0 < end; i0 += blockDim.x) {
            const uint32_t key = key_of(__ldg(r + i0));
            emit(key >= t, key, i0);
        }
    }
}

// grid rows: the first k candidates in (key desc, index asc) order; flags rows
// whose list is short of k or overflowed (done[row] = 0) for the radix passes.
// T = the k-th largest candidate key; every key > T is taken, and of the keys
// == T the ones with the smallest indices; the k taken are placed by counting
// how many of them precede each.
__global__ void __launch_bounds__(kThreads) topk_final_kernel(const float* __restrict__ x, int64_t L, int k,
                                                               const int* __restrict__ count,
                                                               const uint32_t* __restrict__ cand_key,
                                                               const int64_t* __restrict__ cand_idx,
                                                               float* __restrict__ values,
                                                               int64_t* __restrict__ indices, int* __restrict__ done) {
    __shared__ uint32_t sk[kCandCap];
    __shared__ int64_t si[kCandCap];
    __shared__ uint32_t hist[kBins];
    __shared__ uint32_t tk[kSampledMaxK];
    __shared__ int64_t ti[kSampledMaxK];
    __shared__ int s_taken, s_ties;
    __shared__ int tie_pos[kCandCap]; // positions in sk / si of the keys == T
    const int64_t row = blockIdx.x;
    const int n = count[row];
    if (n < k || n > kCandCap) {
        if (threadIdx.x == 0) {
            done[row] = 0;
        }
        return;
    }
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        sk[i] = cand_key[row * kCandCap + i];
        si[i] = cand_idx[row * kCandCap + i];
    }
    if (threadIdx.x == 0) {
        s_taken = 0;
        s_ties = 0;
    }
    __syncthreads();
    int greater = 0;
    const uint32_t T = block_kth_key(sk, n, k, hist, &greater);
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        if (sk[i] > T) {
            const int slot = atomicAdd(&s_taken, 1);
            tk[slot] = sk[i];
            ti[slot] = si[i];
        } else if (sk[i] == T) {
            tie_pos[atomicAdd(&s_ties, 1)] = i;
        }
    }
    __syncthreads();
    const int ties = s_ties;
    const int need = k - greater;
    for (int i = threadIdx.x; i < ties; i += blockDim.x) {
        const int64_t me = si[tie_pos[i]];
        int r = 0;
        for (int q = 0; q < ties; ++q) {
            r += si[tie_pos[q]] < me ? 1 : 0;
        }
        if (r < need) {
            tk[greater + r] = T;
            ti[greater + r] = me;
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < k; i += blockDim.x) {
        const uint32_t ki = tk[i];
        const int64_t ii = ti[i];
        int rank = 0;
        for (int q = 0; q < k; ++q) {
            rank += (tk[q] > ki || (tk[q] == ki && ti[q] < ii)) ? 1 : 0;
        }
        values[row * k + rank] = x[row * L + ii];
        indices[row * k + rank] = ii;
    }
    if (threadIdx.x == 0) {
        done[row] = 1;
    }
}

} // namespace

// Sizes of the sampled-threshold path's sample and of its j (see above), or
// 0 when a row is too short or k too large for it (radix passes only).
static int sample_rank(int64_t L, int64_t k) {
    if (L < 65536 || k > kSampledMaxK) {
        return 0;
    }
    const int64_t j = (4 * k * kSample + L - 1) / L;
    return (j >= 32 && j <= kThreads / 4) ? static_cast<int>(j) : 0;
}

namespace {
struct TopkScratch {
    uint32_t* hist;
    int* eq_counts;
    int* gt_count;
    int64_t* cand_idx;
    uint32_t* cand_key;
    uint32_t* thresh;
    int* count;
    int* done;
    uint32_t* fkey;
    int64_t* fidx;
    size_t head;  // bytes cleared before the radix passes
    size_t fhead; // bytes cleared before the filter (thresh, count, done)
    size_t total;
};

TopkScratch topk_layout(void* base, int64_t rows, int64_t L, int64_t k) {
    auto al = [](size_t v) { return (v + 255) / 256 * 256; };
    const int64_t chunks = (L + kChunk - 1) / kChunk;
    TopkScratch t{};
    uint8_t* p = static_cast<uint8_t*>(base);
    size_t at = 0;
    t.hist = reinterpret_cast<uint32_t*>(p + at);
    t.eq_counts = reinterpret_cast<int*>(p + at + static_cast<size_t>(rows) * 3 * kBins * 4);
    t.gt_count = t.eq_counts + rows * chunks;
    t.head = al(static_cast<size_t>(rows) * 3 * kBins * 4 + static_cast<size_t>(rows * chunks) * 4 +
                static_cast<size_t>(rows) * 4);
    at += t.head;
    t.cand_idx = reinterpret_cast<int64_t*>(p + at);
    at += al(static_cast<size_t>(rows * k) * 8);
    t.cand_key = reinterpret_cast<uint32_t*>(p + at);
    at += al(static_cast<size_t>(rows * k) * 4);
    t.thresh = reinterpret_cast<uint32_t*>(p + at);
    t.count = reinterpret_cast<int*>(p + at + rows * 4);
    t.done = t.count + rows;
    t.fhead = al(static_cast<size_t>(rows) * 12);
    const size_t fat = at;
    at += t.fhead;
    if (sample_rank(L, k) > 0) {
        t.fkey = reinterpret_cast<uint32_t*>(p + at);
        at += al(static_cast<size_t>(rows) * kCandCap * 4);
        t.fidx = reinterpret_cast<int64_t*>(p + at);
        at += al(static_cast<size_t>(rows) * kCandCap * 8);
    }
    (void)fat;
    t.total = at;
    return t;
}
} // namespace

size_t topk_scratch_bytes(int64_t rows, int64_t L, int64_t k) {
    if (L < kSplitMin && k <= kMaxK) {
        return 0;
    }
    return topk_layout(nullptr, rows, L, k).total;
}

int topk_launches(int64_t rows, int64_t L, int64_t k) {
    (void)rows;
    if (L < kSplitMin && k <= kMaxK) {
        return 1;
    }
    return (sample_rank(L, k) > 0 ? 3 : 0) + 6;
}

void topk(nb2_device* dev, const float* x, float* values, int64_t* indices, int64_t rows, int64_t L, int64_t k,
          void* scratch) {
    if (rows == 0 || k == 0) {
        return;
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
    if (k >= (int64_t(1) << 30)) {
        fail(kStatusUnsupported, "TopK: K too large");
    }
    if (L < kSplitMin && k <= kMaxK) {
        topk_row_kernel<<<static_cast<unsigned>(rows), kThreads, 0, dev->stream>>>(x, values, indices, L,
                                                                                   static_cast<int>(k), sort_n);
        check_cuda(cudaGetLastError(), "topk launch");
        return;
    }
    if (scratch == nullptr) {
        fail(kStatusInvalid, "TopK: long rows need scratch memory");
    }
    const TopkScratch t = topk_layout(scratch, rows, L, k);
    const int chunks = static_cast<int>((L + kChunk - 1) / kChunk);
    const int ki = static_cast<int>(k);
    const int j = sample_rank(L, k);
    const int* done = nullptr;
    if (j > 0) {
        check_cuda(cudaMemsetAsync(t.thresh, 0, t.fhead, dev->stream), "topk scratch clear");
        topk_sample_kernel<<<static_cast<unsigned>(rows), kThreads, 0, dev->stream>>>(x, L, j, t.thresh);
        const int vec4 = (L % 4 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0) ? 1 : 0;
        const dim3 fgrid(static_cast<unsigned>((L + kFilterChunk - 1) / kFilterChunk), static_cast<unsigned>(rows));
        topk_filter_kernel<<<fgrid, 256, 0, dev->stream>>>(x, L, t.thresh, t.count, t.fkey, t.fidx, vec4);
        topk_final_kernel<<<static_cast<unsigned>(rows), kThreads, 0, dev->stream>>>(x, L, ki, t.count, t.fkey, t.fidx,
                                                                                    values, indices, t.done);
        done = t.done;
    }
    // radix passes: every row when the sampled path does not apply, else
    // only the rows it flagged (the others return at once)
    check_cuda(cudaMemsetAsync(scratch, 0, t.head, dev->stream), "topk scratch clear");
    const dim3 grid(static_cast<unsigned>(chunks), static_cast<unsigned>(rows));
    for (int pass = 0; pass < 3; ++pass) {
        topk_hist_kernel<<<grid, 512, 0, dev->stream>>>(x, L, ki, pass, t.hist, done);
    }
    topk_eqcount_kernel<<<grid, 512, 0, dev->stream>>>(x, L, ki, t.hist, t.eq_counts, chunks, done);
    topk_collect_kernel<<<grid, 512, 0, dev->stream>>>(x, L, ki, t.hist, t.eq_counts, chunks, t.gt_count, t.cand_key,
                                                       t.cand_idx, done);
    if (k <= kMaxK) {
        topk_sort_kernel<<<static_cast<unsigned>(rows), kThreads, 0, dev->stream>>>(x, L, ki, sort_n, t.cand_key,
                                                                                    t.cand_idx, values, indices, done);
    } else {
        // the sampled path never takes K above kSampledMaxK, so every row is here
        const dim3 rgrid(static_cast<unsigned>((k + 255) / 256), static_cast<unsigned>(rows));
        topk_rank_kernel<<<rgrid, 256, 0, dev->stream>>>(x, L, ki, t.cand_key, t.cand_idx, values, indices);
    }
    check_cuda(cudaGetLastError(), "topk launch");
}

} // namespace nb2
