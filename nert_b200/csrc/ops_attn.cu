// Fused attention on the tensor cores: O = Softmax(scale(Q K^T)) V for every
// (batch, head), one CTA per (batch, head).
//
// Replaces the reference's three rows for this chain: MatMul Q x K^T
// (src/kernels/mat_mul.cpp:79-169), the Div by sqrt(d) (src/kernels/div.cpp),
// Softmax over the last axis (src/kernels/softmax.cpp:47-120: exp(x - max) /
// sum) and MatMul P x V, plus the head-merge Transpose when the graph has one.
// The products use the same 3xTF32 split as the contraction kernel
// (hi = tf32(x), lo = x - hi; a_lo*b_hi + a_hi*b_lo + a_hi*b_hi, fp32
// accumulation in TMEM), the softmax runs in fp32 with expf.
//
// Layout of one CTA (256 threads = 8 warps; warps w and w + 4 both own TMEM
// lanes 32*w .. 32*w + 31, i.e. query rows of the current 128-row block, and
// split the columns of those rows between them):
//   shared memory: K as the B operand of S = Q K^T (rows = keys, K-major over
//   the head dim, two 32-wide slabs) and V^T as the B operand of O = P V
//   (rows = head dims, K-major over the keys, 32-key slabs), each as tf32 hi
//   and lo planes in the 128-byte swizzled layout the MMA descriptor reads;
//   keys past T are zero.
//   TMEM (512 columns): S accumulator [0, Np) (Np = T rounded up to 16),
//   Q hi/lo [Np, Np + 128) while S is computed, then P hi in place of S and
//   P lo in [Np, 2 Np), O accumulator at max(2 Np, Np + 128).
// Limits: head dim 64, T <= 208 keys (shared memory for the K and V^T
// planes); ViT-B/16 at 224x224 has T = 197.

#include "ops.cuh"
#include "ptx.cuh"

#include <cmath>

namespace nb2 {

namespace {

constexpr int kAttnD = 64;
constexpr int kAttnThreads = 256;

__device__ __forceinline__ void split_store(uint8_t* hi_slab, uint8_t* lo_slab, uint32_t off, float x) {
    const float h = to_tf32(x);
    *reinterpret_cast<float*>(hi_slab + off) = h;
    *reinterpret_cast<float*>(lo_slab + off) = x - h;
}

} // namespace

size_t attention_smem_bytes(int T) {
    const int np = (T + 15) / 16 * 16;
    const int vslabs = (np + 31) / 32;
    // K hi/lo: 2 slabs of np rows; V^T hi/lo: vslabs slabs of 64 rows; the
    // two column halves' row maxima and sums; barrier, TMEM slot, abort flag;
    // + 1 KB for the 1024-byte alignment of the slabs
    return static_cast<size_t>(4 * np * 128 + 2 * vslabs * 64 * 128 + 4 * 128 * 4 + 64 + 1024);
}

namespace {

struct AttnArgs {
    AttnGeom g;
    const float* q;
    const float* k;
    const float* v;
    float* out;
    int* err;
    long long wait_bound;
};

template <int MODE>
__device__ __forceinline__ float attn_scale(float c, float s) {
    return MODE == 1 ? s * c : (MODE == 2 ? __fdiv_rn(s, c) : s);
}

// Byte offset of (row, k) in a 128-byte swizzled K-major slab (32 fp32 per
// row, 8-row groups of 1024 bytes, the 16-byte chunk index XORed with row & 7):
// the row part is computed once per row.
struct SwzRow {
    uint32_t base;
    int r7;
    __device__ __forceinline__ explicit SwzRow(int row)
        : base(static_cast<uint32_t>((row >> 3) * 1024 + (row & 7) * 128)), r7(row & 7) {}
    __device__ __forceinline__ uint32_t at(int k) const {
        return base + static_cast<uint32_t>(((((k >> 2) ^ r7) & 7) << 4) + (k & 3) * 4);
    }
};


template <int MODE>
__global__ void __launch_bounds__(kAttnThreads, 1) attention_kernel(AttnArgs a) {
    extern __shared__ uint8_t attn_smem_raw[];
    const AttnGeom& g = a.g;
    const int T = static_cast<int>(g.T);
    const int np = (T + 15) & ~15;
    const int vslabs = (np + 31) / 32;
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(attn_smem_raw) + 1023) & ~uintptr_t(1023));
    const int kslab = np * 128; // bytes of one K slab (np rows x 128 B)
    uint8_t* k_hi = base;                 // slabs 0, 1
    uint8_t* k_lo = base + 2 * kslab;     // slabs 0, 1
    uint8_t* v_hi = base + 4 * kslab;     // vslabs x 8 KB
    uint8_t* v_lo = v_hi + vslabs * 8192; // vslabs x 8 KB
    float* red_max = reinterpret_cast<float*>(v_lo + vslabs * 8192); // [2][128]
    float* red_sum = red_max + 256;                                  // [2][128]
    uint64_t* bar = reinterpret_cast<uint64_t*>(red_sum + 256);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int quarter = warp & 3, half = warp >> 2;
    const int row = quarter * 32 + lane; // query row within the block = TMEM lane
    const int64_t z = blockIdx.x;
    const int64_t b = z / g.H, h = z - b * g.H;
    const float* qz = a.q + b * g.qb + h * g.qh;
    const float* kz = a.k + b * g.kb + h * g.kh;
    const float* vz = a.v + b * g.vb + h * g.vh;
    float* oz = a.out + b * g.ob + h * g.oh;

    if (tid == 0) {
        mbar_init(bar, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }

    // ---- K (rows = keys, K-major over d) and V^T (rows = d, K-major over
    // keys) into shared memory as tf32 hi/lo planes, zero past T. Each loop
    // walks the operand's contiguous axis across the threads and keeps eight
    // loads in flight per thread.
    if (g.kt == 1) { // K^T in memory ([d][T]): thread = key, loop over d
        const int t = tid;
        const SwzRow sr(t);
#pragma unroll 1
        for (int j0 = 0; j0 < kAttnD; j0 += 32) { // 32 loads in flight per thread
            float x[32];
#pragma unroll
            for (int u = 0; u < 32; ++u) {
                x[u] = t < T ? __ldg(kz + t + (j0 + u) * g.kj) : 0.0f;
            }
            if (t < np) {
#pragma unroll
                for (int u = 0; u < 32; ++u) {
                    split_store(k_hi, k_lo, static_cast<uint32_t>((j0 >> 5) * kslab) + sr.at(u), x[u]);
                }
            }
        }
    } else { // [T][d]: thread = (d, key mod 4), loop over keys
        const int j = tid & 63;
        for (int t0 = tid >> 6; t0 < np; t0 += 32) {
            float x[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int t = t0 + 4 * u;
                x[u] = t < T ? __ldg(kz + t * g.kt + j * g.kj) : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int t = t0 + 4 * u;
                if (t < np) {
                    split_store(k_hi, k_lo, static_cast<uint32_t>((j >> 5) * kslab) + SwzRow(t).at(j & 31), x[u]);
                }
            }
        }
    }
    const int tv = vslabs * 32; // keys held for V^T (zero past T)
    if (g.vj == 1) { // [T][d]: thread = (d, key mod 4), loop over keys
        const int j = tid & 63;
        const SwzRow sr(j);
#pragma unroll 1
        for (int t0 = tid >> 6; t0 < tv; t0 += 128) { // 32 loads in flight per thread
            float x[32];
#pragma unroll
            for (int u = 0; u < 32; ++u) {
                const int t = t0 + 4 * u;
                x[u] = t < T ? __ldg(vz + t * g.vt + j) : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < 32; ++u) {
                const int t = t0 + 4 * u;
                if (t < tv) {
                    split_store(v_hi, v_lo, static_cast<uint32_t>((t >> 5) * 8192) + sr.at(t & 31), x[u]);
                }
            }
        }
    } else { // thread = key, loop over d
        const int t = tid;
        for (int j0 = 0; j0 < kAttnD; j0 += 8) {
            float x[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                x[u] = t < T ? __ldg(vz + t * g.vt + (j0 + u) * g.vj) : 0.0f;
            }
            if (t < tv) {
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int j = j0 + u;
                    split_store(v_hi, v_lo, static_cast<uint32_t>((t >> 5) * 8192) + SwzRow(j).at(t & 31), x[u]);
                }
            }
        }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t qcol = static_cast<uint32_t>(np);
    const uint32_t ocol = static_cast<uint32_t>(np + 128 > 2 * np ? np + 128 : 2 * np);
    // this warp's share of the S / P columns: chunks of 16 in [c0, c1)
    const int nch = np / 16;
    const int c0 = half == 0 ? 0 : (nch + 1) / 2, c1 = half == 0 ? (nch + 1) / 2 : nch;
    // with a positive scale (or none) the row max of the scaled scores is the
    // scaled max of the raw ones (rounding is monotonic)
    const float sc = g.scale;
    const bool scale_after_max = MODE == 0 || sc > 0.0f;
    uint32_t uses = 0; // completed phases of `bar`
    bool ok = true;

    // block-uniform bounded wait on the next phase of `bar`
    auto wait_bar = [&]() -> bool {
        bool w = mbar_wait(bar, uses & 1u, abort_flag, a.err, a.wait_bound);
        ++uses;
        w = __syncthreads_and(w) != 0;
        tc_fence_after();
        return w;
    };

    for (int q0 = 0; q0 < T && ok; q0 += 128) {
        const int t = q0 + row;
        // ---- Q row -> TMEM hi [qcol, qcol+64) and lo [qcol+64, qcol+128);
        // this warp's half of the head dim
        {
            const float* qr = qz + static_cast<int64_t>(t) * g.qt + static_cast<int64_t>(half * 32) * g.qj;
            const bool vec = g.qj == 1 && ((reinterpret_cast<uintptr_t>(qr)) & 15) == 0;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                float x[16], hi[16], lo[16];
                if (t < T && vec) {
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float4 f = __ldg(reinterpret_cast<const float4*>(qr + c * 16) + i);
                        x[4 * i] = f.x, x[4 * i + 1] = f.y, x[4 * i + 2] = f.z, x[4 * i + 3] = f.w;
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        x[i] = t < T ? __ldg(qr + (c * 16 + i) * g.qj) : 0.0f;
                    }
                }
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    hi[i] = to_tf32(x[i]);
                    lo[i] = x[i] - hi[i];
                }
                const uint32_t col = qcol + static_cast<uint32_t>(half * 32 + c * 16);
                tmem_st16(tmem + lane_base + col, hi);
                tmem_st16(tmem + lane_base + col + 64, lo);
            }
            tmem_wait_st();
        }
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        // ---- S = Q K^T: M = 128 query rows, N = np keys, K = 64 (two slabs)
        if (tid == 0) {
            const uint32_t idesc = idesc_tf32(128, np);
#pragma unroll
            for (int s = 0; s < 2; ++s) {
                const uint64_t bh = sdesc_k128(smem_u32(k_hi + s * kslab));
                const uint64_t bl = sdesc_k128(smem_u32(k_lo + s * kslab));
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const uint32_t col = static_cast<uint32_t>(s * 32 + kk * 8);
                    const uint32_t first = (s == 0 && kk == 0) ? 0u : 1u;
                    mma_tf32_ta(tmem, tmem + qcol + 64 + col, bh + 2 * kk, idesc, first);
                    mma_tf32_ta(tmem, tmem + qcol + col, bl + 2 * kk, idesc, 1u);
                    mma_tf32_ta(tmem, tmem + qcol + col, bh + 2 * kk, idesc, 1u);
                }
            }
            mma_commit(bar);
        }
        __syncwarp();
        if (!wait_bar()) {
            ok = false;
            break;
        }
        // ---- softmax of row `row` over keys [0, T): this warp's columns,
        // the two halves combined through shared memory
        const uint32_t srow = tmem + lane_base;
        // chunks wholly below T skip the per-key test
        float m = -INFINITY;
        for (int c = c0; c < c1; ++c) {
            float v[16];
            tmem_ld16(srow + c * 16, v);
            if (c * 16 + 16 <= T) {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    m = fmaxf(m, scale_after_max ? v[i] : attn_scale<MODE>(sc, v[i]));
                }
            } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float s = scale_after_max ? v[i] : attn_scale<MODE>(sc, v[i]);
                    m = c * 16 + i < T ? fmaxf(m, s) : m;
                }
            }
        }
        red_max[half * 128 + row] = m;
        __syncthreads();
        m = fmaxf(red_max[row], red_max[128 + row]);
        if (scale_after_max) {
            m = attn_scale<MODE>(sc, m);
        }
        float sum = 0.0f;
        for (int c = c0; c < c1; ++c) {
            float v[16];
            tmem_ld16(srow + c * 16, v);
            if (c * 16 + 16 <= T) {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    v[i] = expf(attn_scale<MODE>(sc, v[i]) - m);
                    sum += v[i];
                }
            } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    v[i] = c * 16 + i < T ? expf(attn_scale<MODE>(sc, v[i]) - m) : 0.0f;
                    sum += v[i];
                }
            }
            tmem_st16(srow + c * 16, v);
        }
        red_sum[half * 128 + row] = sum;
        tmem_wait_st();
        __syncthreads();
        const float inv = 1.0f / (red_sum[row] + red_sum[128 + row]);
        for (int c = c0; c < c1; ++c) {
            float v[16], hi[16], lo[16];
            tmem_ld16(srow + c * 16, v);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const float p = v[i] * inv;
                hi[i] = to_tf32(p);
                lo[i] = p - hi[i];
            }
            tmem_st16(srow + c * 16, hi);
            tmem_st16(srow + qcol + c * 16, lo);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        // ---- O = P V: M = 128, N = 64, K = np keys (32-key slabs of V^T)
        if (tid == 0) {
            const uint32_t idesc = idesc_tf32(128, kAttnD);
            for (int s = 0; s < vslabs; ++s) {
                const uint64_t bh = sdesc_k128(smem_u32(v_hi + s * 8192));
                const uint64_t bl = sdesc_k128(smem_u32(v_lo + s * 8192));
                for (int kk = 0; kk < 4 && s * 32 + kk * 8 < np; ++kk) {
                    const uint32_t col = static_cast<uint32_t>(s * 32 + kk * 8);
                    const uint32_t first = (s == 0 && kk == 0) ? 0u : 1u;
                    mma_tf32_ta(tmem + ocol, tmem + qcol + col, bh + 2 * kk, idesc, first);
                    mma_tf32_ta(tmem + ocol, tmem + col, bl + 2 * kk, idesc, 1u);
                    mma_tf32_ta(tmem + ocol, tmem + col, bh + 2 * kk, idesc, 1u);
                }
            }
            mma_commit(bar);
        }
        __syncwarp();
        if (!wait_bar()) {
            ok = false;
            break;
        }
        // ---- epilogue: this warp's 32 of the row's 64 output values
        {
            float* orow = oz + static_cast<int64_t>(t) * g.ot + half * 32;
            const bool vec = ((reinterpret_cast<uintptr_t>(orow)) & 15) == 0;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                float v[16];
                tmem_ld16(tmem + lane_base + ocol + static_cast<uint32_t>(half * 32 + c * 16), v);
                if (t < T) {
                    if (vec) {
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            reinterpret_cast<float4*>(orow + c * 16)[i] =
                                make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            orow[c * 16 + i] = v[i];
                        }
                    }
                }
            }
        }
        // the next block's Q overwrites TMEM columns the MMAs just read
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
    }
    if (!ok && tid == 0) {
        // MMAs already issued complete on their own: let them land before
        // the columns are freed
        const long long t0 = clock64();
        while (!mbar_try_wait(bar, (uses - 1) & 1u) && clock64() - t0 < kWaitBoundCycles) {
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

} // namespace

void attention(nb2_device* dev, const AttnGeom& g, const float* q, const float* k, const float* v, float* out) {
    if (g.T < 1 || g.T > kAttnMaxT) {
        fail(kStatusUnsupported, "Attention: between 1 and 208 keys are supported by the fused kernel");
    }
    if (g.B * g.H == 0) {
        return;
    }
    if (g.B * g.H > 0x7fffffff) {
        fail(kStatusUnsupported, "Attention: too many (batch, head) pairs");
    }
    const size_t smem = attention_smem_bytes(static_cast<int>(g.T));
    static size_t attr_bytes[64] = {};
    if (attr_bytes[dev->ordinal] < smem) {
        for (auto fn : {attention_kernel<0>, attention_kernel<1>, attention_kernel<2>}) {
            check_cuda(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)),
                       "cudaFuncSetAttribute(attention)");
        }
        attr_bytes[dev->ordinal] = smem;
    }
    AttnArgs a{g, q, k, v, out, dev->err_word, dev->wait_bound};
    // a division by a power of two is the multiplication by its exact
    // reciprocal (both are the correctly rounded s / c)
    if (a.g.scale_mode == 2) {
        int e = 0;
        const float m = std::frexp(a.g.scale, &e);
        if (m == 0.5f || m == -0.5f) {
            const float r = 1.0f / a.g.scale;
            if (std::isfinite(r) && r != 0.0f && std::frexp(r, &e) == m) {
                a.g.scale_mode = 1;
                a.g.scale = r;
            }
        }
    }
    const unsigned grid = static_cast<unsigned>(g.B * g.H);
    if (a.g.scale_mode == 1) {
        attention_kernel<1><<<grid, kAttnThreads, smem, dev->stream>>>(a);
    } else if (a.g.scale_mode == 2) {
        attention_kernel<2><<<grid, kAttnThreads, smem, dev->stream>>>(a);
    } else {
        attention_kernel<0><<<grid, kAttnThreads, smem, dev->stream>>>(a);
    }
    check_cuda(cudaGetLastError(), "attention launch");
}

} // namespace nb2
