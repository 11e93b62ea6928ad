// tcgen05 contraction engine for Conv / Gemm / MatMul on sm_100a.
//
// Replaces the reference's cuDNN Conv row (src/cuda/conv.cu:230-530, FP32 FMA
// math, no tensor cores) and cuBLAS Gemm/MatMul rows (src/cuda/gemm.cu:84-166,
// src/cuda/mat_mul.cu:94-198, pedantic FP32). The reference CPU oracle
// accumulates in double and rounds once (src/kernels/conv.cpp:263-289,
// gemm.cpp:122-136); this engine keeps fp32 accuracy on tf32 tensor cores with
// the 3xTF32 split of Ootomo & Yokota (2022): x = hi + lo with hi = tf32(x),
// and D += A_lo*B_hi + A_hi*B_lo + A_hi*B_hi accumulated in fp32 in TMEM
// (A_lo*B_lo, ~2^-22 relative, is dropped). 1xTF32 keeps only A_hi*B_hi.
//
// CTA = 10 warps, one 128 x BN output tile, BK = 32 fp32 (one 128-byte
// swizzle row) per pipeline stage:
//   warps 0-7  gather A (im2col / dense), split hi/lo, write the 128B-swizzled
//              K-major tile; then the epilogue (TMEM -> registers -> global);
//   warp 8     TMA loads of the pre-split B planes;
//   warp 9     one thread issues tcgen05.mma (M=128, N=BN, K=8) into TMEM.
// Every mbarrier wait is bounded (ptx.cuh); a timeout sets the device error
// word and the CTA unwinds, frees its TMEM and returns.

#include "igemm.cuh"
#include "ptx.cuh"

#include <algorithm>
#include <cstring>

namespace nb2 {

int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

namespace {

// kADenseTma: row-major A whose rows are 16-byte aligned; TMA brings the raw
// fp32 tile into shared memory and the producer warps split it in place.
// kAConvNhwc: Conv over NHWC activations (C % 4 == 0; K padded to a multiple
// of 32 channels a tap); TMA im2col brings the raw fp32 tile for one (filter
// tap, 32-channel block) per K block, the channels past C read as zeros.
// kAConvCvec: Conv over x[N][H][W][cv] with cv = 4, 8 or 16 channels (C <= cv,
// zero padded; e.g. a stem's RGB image); K ordered (tap, channel), so a
// thread's 16 K values are 16 / cv taps of 16-byte vector loads.
enum AMode : int {
    kAConvTap = 0,
    kAConvGeneric = 1,
    kADenseK = 2,
    kADenseM = 3,
    kADenseTma = 4,
    kAConvNhwc = 5,
    kAConvCvec = 6
};

struct Args {
    int M, N, K, nkb;
    // split K: work unit = (tile, K slice); slice ks covers K blocks
    // [ks*kper, min(nkb, (ks+1)*kper)); with ksplit > 1 the epilogue writes
    // raw fp32 partial sums to part[((ks*zcount + z)*M + row)*N + col] and a
    // second kernel reduces them and applies the real epilogue
    int ksplit, kper;
    // balanced split (stream > 0): the (tile, K block) pairs in tile-major
    // order, sk_total of them, are cut into equal spans of sk_span, one per
    // CTA; a unit is the part of one tile inside a CTA's span. Units that
    // cover a whole tile take the normal epilogue; the others write raw
    // partials to part[(cta * 2 + slot) * 128 * BN] (slot 0: the span's first
    // unit, 1: its last) and streamk_reduce_kernel finishes those tiles.
    int stream, sk_span, sk_total;
    float* part;
    int zcount; // batch / group slices
    int mode;
    const float* a;
    int64_t a_zstride;
    int64_t lda;
    int vec4; // dense K-major rows are 16-byte aligned with K % 4 == 0
    int a_zrows; // kADenseTma: A-map row offset per z slice
    // conv geometry
    int C, H, W, OH, OW, KH, KW, sh, sw, ph, pw, dh, dw, Cg;
    int64_t HW, OHW, img_stride;
    const int2* ktab;
    int ktab_smem; // copy the tap table into shared memory
    // B
    int b_zrows;
    // epilogue
    float* out;
    int64_t out_zstride, out_img_stride, ldc;
    int conv_out;
    int vec_out; // rows are 16-byte aligned and contiguous in n (and so are bias / res)
    // permuted output (OutMap): offsets from (z, row, col) by two-level
    // mixed radices; the epilogue then takes path 0 (lanes over rows) or,
    // when cs2 == 1, path 1 (16 contiguous columns per chunk)
    // 128-wide tiles with several tiles per CTA: two tiles in flight with
    // one accumulator each, the MMA issuers taking alternate tiles (the
    // epilogue of one tile overlaps the next tile's main loop)
    int alt;
    int omap;
    int oz2, or2, oc2;
    int64_t ozs1, ozs2, ors1, ors2, ocs1, ocs2;
    const float* bias;
    int bias_zstride;
    float bias_scale;
    const float* res;
    float res_scale;
    float alpha;
    int act;
    float act_a, act_b, act_c; // GELU (erf form) constants
    int* err;
    long long wait_bound; // clock64 ticks before a pipeline wait gives up
};

constexpr int pow2_at_least(int v) {
    int p = 32;
    while (p < v) {
        p *= 2;
    }
    return p;
}

// TMA_A: the raw A tile arrives by TMA (dense row-major A, NHWC Conv) and
// four converter warps split it; otherwise eight producer warps gather A.
template <int BN, bool THREE, bool TMA_A>
struct Cfg {
    // A lives in tensor memory: the producers write the tf32 hi/lo planes of
    // A with tcgen05.st and the MMA reads A from TMEM, B from shared memory.
    // An MMA that reads both from shared memory needs 128 B/clock at N = 128
    // (all of shared memory's bandwidth, starving the producers and the TMA
    // writes); with A in TMEM it reads 64.
    static constexpr int kAPlane = 128 * 128;
    static constexpr int kBPlane = BN * 128;
    static constexpr int kPlanes = THREE ? 2 : 1;
    static constexpr int kBStageBytes = kBPlane * kPlanes;
    // shared-memory stage: a raw A tile (TMA_A modes only; released by the
    // converter once read) and the B hi / lo planes (released by the MMA).
    // The gather modes take no raw A space: the shared memory they leave
    // unclaimed stays L1, which holds the overlapping filter windows their
    // loads re-read.
    static constexpr int kAStageBytes = TMA_A ? kAPlane : 0;
    static constexpr int kStageBytes = kAStageBytes + kBStageBytes;
    static constexpr int kStagesRaw = (200 * 1024) / kStageBytes;
    // two accumulators per tile (even / odd K blocks, one per MMA issuer) x
    // kAccBufs tiles in flight: two for BN = 64 (the epilogue overlaps the
    // next tile's MMAs), one for BN = 128 (the other 256 columns hold the A
    // stages). Measured: one issuer per tile with two 128-wide tiles in
    // flight is slower wherever an SM gets one or two tiles (the issuer's
    // wake-ups between K blocks are then exposed).
    static constexpr int kAccs = 2;
    static constexpr int kAccBufs = BN <= 64 ? 2 : 1;
    static constexpr int kAccCols = kAccBufs * kAccs * BN;
    static constexpr int kAStageCols = 32 * kPlanes; // hi plane, then lo plane
    static constexpr int kTStagesRaw = (512 - kAccCols) / kAStageCols;
    static constexpr int kMin3(int a, int b, int c) { return a < b ? (a < c ? a : c) : (b < c ? b : c); }
    // TMEM A stage t == shared-memory stage s, so one MMA commit frees both
    static constexpr int kStages = kMin3(kStagesRaw, kTStagesRaw, 8);
    static constexpr int kTmemCols = pow2_at_least(kAccCols + kStages * kAStageCols);
    static constexpr int kRingBytes = kStages * kStageBytes;
    static_assert(kTmemCols <= 512, "TMEM budget");
    static_assert(BN == 64 || BN == 128, "tile widths");
    // Warp roles. Epilogue warps: w -> TMEM lane quarter w & 3, column part
    // w >> 2; eight of them where the accumulator is single buffered and A
    // needs no gathering (the epilogue is then on the critical path). A
    // producers: lane quarter w & 3 and a K half (gather), or two 4-warp
    // converter groups taking alternate K blocks (TMA_A). One thread issues
    // at most one TMA copy every few hundred cycles, and one tcgen05.mma per
    // ~50 cycles whatever its width, so the copies of a K block come from
    // three warps and the MMAs from two threads (even and odd K blocks,
    // which feed separate accumulators).
    static constexpr int kEpiWarps = (TMA_A && BN == 128) ? 8 : 4;
    static constexpr int kProdWarps = 8;
    static constexpr int kGroupWarps = TMA_A ? 4 : 8; // producer warps per K block
    static constexpr int kTmaWarp = kEpiWarps + kProdWarps; // B hi plane
    static constexpr int kMmaWarp = kTmaWarp + 1;           // even K blocks
    static constexpr int kTmaAWarp = kTmaWarp + 2;          // raw A tile (TMA_A)
    static constexpr int kTmaBloWarp = kTmaWarp + 3;        // B lo plane (3xTF32)
    static constexpr int kMma2Warp = kTmaWarp + 4;          // odd K blocks
    static constexpr int kThreads = (kTmaWarp + 5) * 32;
    // epilogue staging: one 32 x 17 fp32 tile per epilogue warp (row-major
    // outputs whose rows are not 16-byte aligned leave as 64-byte pieces).
    // Measured: staging 16-byte rows the same way is slower than storing
    // one 16-byte vector per row directly.
    static constexpr int kEpiTileFloats = 32 * 17;
    static constexpr int kEpiBytes = kEpiWarps * kEpiTileFloats * 4;
    static constexpr int kSmemBytes = kRingBytes + 1024 + 512 + kEpiBytes;
};

template <int A>
struct ActTag {
    static constexpr int value = A;
};

// Fused activation, resolved at compile time. The GELU form is the ONNX
// export's op sequence, kept in order so the fused value equals the unfused
// rows': ((x * (erf(x / a) + b)) * c).
template <int ACT>
__device__ __forceinline__ float act_of(float v, const Args& p) {
    if constexpr (ACT == kActGeluErf) {
        return (v * (erff(v / p.act_a) + p.act_b)) * p.act_c;
    } else if constexpr (ACT == kActRelu) {
        return v > 0.0f ? v : 0.0f;
    } else if constexpr (ACT == kActSilu) {
        return v * (1.0f / (1.0f + expf(-v)));
    } else if constexpr (ACT == kActSigmoid) {
        return 1.0f / (1.0f + expf(-v));
    } else {
        return v;
    }
}

// Per-thread producer state: one output row (pixel / matrix row) of the tile
// and one 16-wide half of every 32-wide K block.
struct RowState {
    bool ok;
    const float* base; // mode-dependent base pointer
    int ih0, iw0;      // conv: top-left input coordinate of the window
    int m;
    // conv tap-major running position
    int cin, kh, kw;
};

// Narrow-channel gather: the half's 16 K values are 16 / CV whole filter
// taps of CV channels (one to four 16-byte loads per tap). tab[tap] = (kh*dh,
// kw*dw, 16-byte offset of the tap from the window's top-left pixel); past
// the last tap x is far out of range, so the bounds test rejects it.
template <int CV>
__device__ __forceinline__ void gather_cvec(const Args& p, const RowState& rs, int kb, int half, const int4* tab,
                                            float (&v)[16]) {
    constexpr int kTaps = 16 / CV;
    constexpr int kVec = CV / 4;
    const int t0 = (kb * 32 + half * 16) / CV;
    const float4* base = reinterpret_cast<const float4*>(rs.base);
#pragma unroll
    for (int t = 0; t < kTaps; ++t) {
        const int4 e = tab[t0 + t];
        const bool ok = rs.ok & ((unsigned)(rs.ih0 + e.x) < (unsigned)p.H) & ((unsigned)(rs.iw0 + e.y) < (unsigned)p.W);
#pragma unroll
        for (int q = 0; q < kVec; ++q) {
            const float4 f = ok ? __ldg(base + e.z + q) : make_float4(0.f, 0.f, 0.f, 0.f);
            const int o = (t * kVec + q) * 4;
            v[o] = f.x;
            v[o + 1] = f.y;
            v[o + 2] = f.z;
            v[o + 3] = f.w;
        }
    }
}

template <int MODE>
__device__ __forceinline__ void gather16(const Args& p, RowState& rs, int kb, int half, const int2* ktab,
                                         float (&v)[16]) {
    if constexpr (MODE == kAConvTap) {
        // K ordered (kh, kw, cin) with Cg % 32 == 0: the whole 32-wide block
        // sits on one filter tap, so validity is one test per block.
        const int ih = rs.ih0 + rs.kh * p.dh;
        const int iw = rs.iw0 + rs.kw * p.dw;
        const bool ok = rs.ok && (unsigned)ih < (unsigned)p.H && (unsigned)iw < (unsigned)p.W;
        const float* src = rs.base + (int64_t)(rs.cin + half * 16) * p.HW + (int64_t)ih * p.W + iw;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            v[i] = ok ? __ldg(src + (int64_t)i * p.HW) : 0.0f;
        }
        // advance to the next block
        rs.cin += 32;
        if (rs.cin >= p.Cg) {
            rs.cin = 0;
            if (++rs.kw == p.KW) {
                rs.kw = 0;
                ++rs.kh;
            }
        }
    } else if constexpr (MODE == kAConvCvec) {
        const int4* tab = reinterpret_cast<const int4*>(ktab);
        if (p.Cg == 4) {
            gather_cvec<4>(p, rs, kb, half, tab, v);
        } else if (p.Cg == 8) {
            gather_cvec<8>(p, rs, kb, half, tab, v);
        } else {
            gather_cvec<16>(p, rs, kb, half, tab, v);
        }
    } else if constexpr (MODE == kAConvGeneric) {
        // per-k tap table (shared memory when it fits); branch-free: an
        // out-of-window tap loads from a valid address and is zeroed after
        const int k0 = kb * 32 + half * 16;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int2 e = ktab[k0 + i];
            const int dhk = e.y >> 16;
            const int dwk = e.y & 0xFFFF;
            const bool ok = rs.ok & (e.y >= 0) & ((unsigned)(rs.ih0 + dhk) < (unsigned)p.H) &
                            ((unsigned)(rs.iw0 + dwk) < (unsigned)p.W);
            const float t = __ldg(ok ? rs.base + e.x : p.a);
            v[i] = ok ? t : 0.0f;
        }
    } else if constexpr (MODE == kADenseK) {
        const int k0 = kb * 32 + half * 16;
        if (p.vec4) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int k = k0 + q * 4;
                float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
                if (rs.ok && k < p.K) {
                    t = __ldg(reinterpret_cast<const float4*>(rs.base + k));
                }
                v[q * 4 + 0] = t.x;
                v[q * 4 + 1] = t.y;
                v[q * 4 + 2] = t.z;
                v[q * 4 + 3] = t.w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int k = k0 + i;
                v[i] = (rs.ok && k < p.K) ? __ldg(rs.base + k) : 0.0f;
            }
        }
    } else { // kADenseM: A stored [K][M] (transposed), row m is a column
        const int k0 = kb * 32 + half * 16;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int k = k0 + i;
            v[i] = (rs.ok && k < p.K) ? __ldg(rs.base + (int64_t)k * p.lda) : 0.0f;
        }
    }
}

// All 32 lanes wait; the outcome is made warp-uniform.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err,
                                          long long bound) {
    const bool ok = mbar_wait(bar, parity, abort_flag, err, bound);
    return __all_sync(0xffffffffu, ok);
}

// tf32 hi/lo planes of 16 consecutive K values of one A row into TMEM:
// columns [col, col+16) of the hi plane and [col+32, col+48) of the lo plane,
// lane = the thread's row (the warp's lane quarter is fixed by its id).
template <bool THREE>
__device__ __forceinline__ void store16_tmem(uint32_t taddr, const float (&v)[16]) {
    float h[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        h[i] = to_tf32(v[i]);
    }
    tmem_st16(taddr, h);
    if (THREE) {
        float l[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            l[i] = v[i] - h[i];
        }
        tmem_st16(taddr + 32, l);
    }
}

// Publishes a TMEM A stage to the MMA issuer (one arrive per warp).
__device__ __forceinline__ void publish_tmem(uint64_t* bar, int lane) {
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
        mbar_arrive(bar);
    }
}

// Persistent, warp-specialised contraction kernel: one CTA per SM walks the
// output tiles (m fastest, so concurrent CTAs share the B tile in L2). With
// two TMEM accumulator buffers (BN = 64) the epilogue of one tile overlaps
// the main loop of the next.
template <int MODE>
__host__ __device__ constexpr bool tma_a_mode() {
    return MODE == kADenseTma || MODE == kAConvNhwc;
}

template <int BN, bool THREE, int MODE, bool STREAM>
// 17 or 21 warps: an SM sub-partition has 16K registers and holds 5 or 6 of
// them, so a thread may use at most 96 or 80 registers (the launch bound
// makes the compiler keep to that). STREAM: the balanced split's unit walk
// and partial tiles (a separate instance, so the other schedules keep their
// registers).
__global__ void __launch_bounds__(Cfg<BN, THREE, tma_a_mode<MODE>()>::kThreads, 1)
    igemm_kernel(const __grid_constant__ Args p, const __grid_constant__ CUtensorMap tm_hi,
                 const __grid_constant__ CUtensorMap tm_lo, const __grid_constant__ CUtensorMap tm_a) {
    constexpr bool kTmaA = tma_a_mode<MODE>();
    using C = Cfg<BN, THREE, kTmaA>;
    constexpr int S = C::kStages;
    constexpr int ST = C::kStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    // full_a = raw A landed (TMA_A), empty_a = raw A read (converter warps),
    // full_b = B landed, t_full = TMEM A stage written (producer warps),
    // empty = B stage and TMEM A stage consumed (MMA commit).
    uint64_t* full_a = reinterpret_cast<uint64_t*>(smem + C::kRingBytes);
    uint64_t* full_b = full_a + S;
    uint64_t* empty = full_b + S;
    uint64_t* empty_a = empty + S;
    uint64_t* t_full = empty_a + S;
    uint64_t* acc_full = t_full + ST;  // [2]
    uint64_t* acc_empty = acc_full + 2; // [2]
    uint64_t* mma_done = acc_empty + 2;
    // alternate tiles: the issuer of tile i arrives once it has seen its
    // last K block ready; the issuer of tile i + 1 waits for that before
    // its first, so each waits on every A stage's phases in order
    uint64_t* mma_turn = mma_done + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_turn + 1);
    // accumulator buffers: BN = 64: kAccBufs x (even, odd); BN = 128: one
    // tile x (even, odd), or (alt) two tiles x one
    const bool alt = BN == 128 && p.alt != 0;
    const int nbuf = alt ? 2 : C::kAccBufs;
    auto acc_col = [&](int b) { return static_cast<uint32_t>(alt ? b * BN : b * C::kAccs * BN); };
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    // the raw A ring (S x 16 KB, TMA_A modes), then the B ring (S x [B hi][B lo])
    auto a_raw = [&](int s) { return smem + s * C::kAPlane; };
    auto b_hi = [&](int s) { return smem + S * C::kAStageBytes + s * C::kBStageBytes; };
    auto b_lo = [&](int s) { return b_hi(s) + C::kBPlane; };

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int nkb = p.nkb;
    const int num_m = (p.M + 127) / 128;
    const int num_n = (p.N + BN - 1) / BN;
    const int tiles_per_z = num_m * num_n;
    const int num_tiles = tiles_per_z * p.zcount * p.ksplit; // work units

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full_a[s], 1);
            mbar_init(&full_b[s], THREE ? 2 : 1); // the B hi and B lo TMA threads
            mbar_init(&empty[s], 1);
            mbar_init(&empty_a[s], C::kGroupWarps);
        }
        for (int t = 0; t < ST; ++t) {
            mbar_init(&t_full[t], C::kGroupWarps);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], alt ? 1 : 2); // the issuers that feed a tile commit
            mbar_init(&acc_empty[b], C::kEpiWarps);
        }
        mbar_init(mma_done, 2);
        mbar_init(mma_turn, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    // generic conv gather: tap table into shared memory when it fits
    const int2* ktab = p.ktab;
    if constexpr (MODE == kAConvGeneric) {
        if (p.ktab_smem) {
            int2* t = reinterpret_cast<int2*>(smem + C::kRingBytes + 512 + C::kEpiBytes);
            for (int k = threadIdx.x; k < nkb * 32; k += blockDim.x) {
                t[k] = p.ktab[k];
            }
            ktab = t;
        }
    } else if constexpr (MODE == kAConvCvec) {
        // per-tap filter offsets, built here (32 / cv taps per K block)
        int4* t = reinterpret_cast<int4*>(smem + C::kRingBytes + 512 + C::kEpiBytes);
        const int taps = p.KH * p.KW;
        for (int k = threadIdx.x; k < nkb * (32 / p.Cg); k += blockDim.x) {
            const int kh = k / p.KW, dy = kh * p.dh, dx = (k - kh * p.KW) * p.dw;
            t[k] = k < taps ? make_int4(dy, dx, (dy * p.W + dx) * (p.Cg >> 2), 0) : make_int4(-(1 << 24), 0, 0, 0);
        }
        ktab = reinterpret_cast<const int2*>(t);
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, C::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // tile t -> (z, n_tile, m_tile), m fastest
    // unit t -> (K slice, z, n tile, m tile), m fastest; kb0 / kcnt = the
    // slice's first K block and block count
    // this CTA's units: [u_first, u_end), stepping by u_next
    constexpr bool stream = STREAM;
    const int u_first = stream ? static_cast<int>(blockIdx.x) * p.sk_span : static_cast<int>(blockIdx.x);
    const int u_end = stream ? min(u_first + p.sk_span, p.sk_total) : num_tiles;
    auto decode = [&](int t, int& z, int& m0, int& n0) {
        const int u = stream ? t / nkb : t % (tiles_per_z * p.zcount);
        z = u / tiles_per_z;
        const int r = u - z * tiles_per_z;
        const int nt = r / num_m;
        m0 = (r - nt * num_m) * 128;
        n0 = nt * BN;
    };
    auto kslice = [&](int t, int& kb0, int& kcnt) {
        if (stream) {
            kb0 = t % nkb;
            kcnt = min(nkb - kb0, u_end - t);
            return;
        }
        kb0 = (t / (tiles_per_z * p.zcount)) * p.kper;
        kcnt = min(nkb - kb0, p.kper);
    };
    auto u_next = [&](int t) -> int {
        return stream ? min((t / nkb + 1) * nkb, u_end) : t + static_cast<int>(gridDim.x);
    };

    if (warp >= C::kEpiWarps && warp < C::kEpiWarps + C::kProdWarps) {
        // ---------------- A producers ----------------
        const int pw = warp - C::kEpiWarps;
        const int r = (pw & 3) * 32 + lane;
        const int half = pw >> 2;
        if constexpr (kTmaA) {
            // Converter: two 4-warp groups take alternate K blocks, so one
            // group's TMEM stores overlap the other's loads. Thread = row r
            // (its warp's lane quarter), all 32 K values: eight swizzled
            // 16-byte chunks of the raw tile -> tf32 hi / lo planes in TMEM.
            // Even ring depth: every use of a stage falls to one group, which
            // waits on its phases in order.
            static_assert(S % 2 == 0, "converter groups need an even ring depth");
            uint32_t items = 0;
            for (int t = u_first; t < u_end; t = u_next(t)) {
                int kb0, kcnt;
                kslice(t, kb0, kcnt);
                items += static_cast<uint32_t>(kcnt);
            }
            const uint32_t tq = tmem + (static_cast<uint32_t>((pw & 3) * 32) << 16) + C::kAccCols;
            for (uint32_t g = static_cast<uint32_t>(pw >> 2); g < items; g += 2) {
                const int s = static_cast<int>(g % S);
                const int t = static_cast<int>(g % ST);
                if (!warp_wait(&full_a[s], (g / S) & 1u, abort_flag, p.err, p.wait_bound)) {
                    break;
                }
                const uint32_t row = smem_u32(a_raw(s)) + r * 128;
                float v[32];
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                                 : "=f"(v[4 * c]), "=f"(v[4 * c + 1]), "=f"(v[4 * c + 2]), "=f"(v[4 * c + 3])
                                 : "r"(row + ((c ^ (r & 7)) << 4))
                                 : "memory");
                }
                // TMEM stage t == s is free once the MMA released stage s
                if (!warp_wait(&empty[t], ((g / ST) & 1u) ^ 1u, abort_flag, p.err, p.wait_bound)) {
                    break;
                }
                const uint32_t ta = tq + t * C::kAStageCols;
                store16_tmem<THREE>(ta, *reinterpret_cast<const float(*)[16]>(&v[0]));
                store16_tmem<THREE>(ta + 16, *reinterpret_cast<const float(*)[16]>(&v[16]));
                // The raw tile has been read (its values went into the TMEM
                // stores); order those generic-proxy reads before the next
                // TMA (async-proxy) write into the stage, then release it.
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&empty_a[s]);
                }
                // B landed too, so the MMA issuer waits on t_full alone
                if (!warp_wait(&full_b[s], (g / S) & 1u, abort_flag, p.err, p.wait_bound)) {
                    break;
                }
                publish_tmem(&t_full[t], lane);
            }
        } else {
        // The (tile, K block) items of this CTA form one stream: the gather
        // cursor runs two items ahead of the stores, across tile boundaries,
        // so short-K layers also keep loads in flight.
        int ct = u_first; // cursor unit
        int ckb = 0;         // cursor K block
        int ckb_end = 0;     // end of the cursor unit's K slice
        RowState rs;
        auto start_tile = [&](int t) {
            int z, m0, n0, kb0, kcnt;
            decode(t, z, m0, n0);
            kslice(t, kb0, kcnt);
            ckb = kb0;
            ckb_end = kb0 + kcnt;
            rs.m = m0 + r;
            rs.ok = rs.m < p.M;
            // tap-major running position of the slice's first K block
            const int k0 = kb0 * 32;
            const int tap = p.Cg > 0 ? k0 / p.Cg : 0;
            rs.cin = k0 - tap * p.Cg;
            rs.kh = p.KW > 0 ? tap / p.KW : 0;
            rs.kw = tap - rs.kh * p.KW;
            const float* az = p.a + (int64_t)z * p.a_zstride;
            if constexpr (MODE == kAConvTap || MODE == kAConvGeneric || MODE == kAConvCvec) {
                const int mm = rs.ok ? rs.m : 0;
                const int n_img = mm / (int)p.OHW;
                const int pix = mm - n_img * (int)p.OHW;
                const int oh = pix / p.OW;
                const int ow = pix - oh * p.OW;
                rs.ih0 = oh * p.sh - p.ph;
                rs.iw0 = ow * p.sw - p.pw;
                const float* img = az + (int64_t)n_img * p.img_stride;
                // generic: the window's top-left pixel of each channel plane;
                // narrow channels: that pixel's vector (either may lie
                // outside the image: only in-window taps are read)
                rs.base = (MODE == kAConvGeneric) ? img + (int64_t)rs.ih0 * p.W + rs.iw0
                          : (MODE == kAConvCvec)  ? img + ((int64_t)rs.ih0 * p.W + rs.iw0) * p.Cg
                                                  : img;
            } else if constexpr (MODE == kADenseK) {
                rs.base = az + (int64_t)(rs.ok ? rs.m : 0) * p.lda;
            } else {
                rs.base = az + (rs.ok ? rs.m : 0);
            }
        };
        if (ct < u_end) {
            start_tile(ct);
        }
        auto next = [&](float (&buf)[16]) -> bool {
            if (ct >= u_end) {
                return false;
            }
            gather16<MODE>(p, rs, ckb, half, ktab, buf);
            if (++ckb == ckb_end) {
                ct = u_next(ct);
                if (ct < u_end) {
                    start_tile(ct);
                }
            }
            return true;
        };
        uint32_t g = 0; // global K-block counter (the smem ring spans tiles)
        const uint32_t tq = tmem + (static_cast<uint32_t>((pw & 3) * 32) << 16) + C::kAccCols + half * 16;
        auto produce = [&](const float (&v)[16]) -> bool {
            const int t = static_cast<int>(g % ST);
            if (!warp_wait(&empty[t], ((g / ST) & 1u) ^ 1u, abort_flag, p.err, p.wait_bound)) {
                return false;
            }
            store16_tmem<THREE>(tq + t * C::kAStageCols, v);
            publish_tmem(&t_full[t], lane);
            return true;
        };
        float b0[16], b1[16], b2[16];
        bool h0 = next(b0);
        bool h1 = next(b1);
        while (true) {
            const bool h2 = next(b2);
            if (!h0 || !produce(b0)) {
                break;
            }
            ++g;
            h0 = next(b0);
            if (!h1 || !produce(b1)) {
                break;
            }
            ++g;
            h1 = next(b1);
            if (!h2 || !produce(b2)) {
                break;
            }
            ++g;
        }
        }
    } else if (warp < C::kEpiWarps) {
        // ---------------- epilogue ----------------
        // The activation is a template argument of the tile loop (one switch
        // per launch, not per element); per-element work is two FMAs, the
        // activation and the store.
        const int quarter = warp & 3;                  // TMEM lanes quarter*32 .. +31
        constexpr int kCols = BN / (C::kEpiWarps / 4); // columns per warp
        const int col_lo = (warp >> 2) * kCols;
        float* const stile = reinterpret_cast<float*>(smem + C::kRingBytes + 512) + warp * C::kEpiTileFloats;
        // 0: NCHW conv output, 1: row-major with 16-byte rows, 2: other row-major
        const int path = p.conv_out ? 0 : (p.vec_out ? 1 : 2);
        auto tiles = [&](auto act_tag) {
            constexpr int ACT = decltype(act_tag)::value;
            int i = 0;
            for (int t = u_first; t < u_end; t = u_next(t), ++i) {
                int z, m0, n0;
                decode(t, z, m0, n0);
                const int b = i % nbuf;
                if (!warp_wait(&acc_full[b], (i / nbuf) & 1, abort_flag, p.err, p.wait_bound)) {
                    break;
                }
                tc_fence_after();
                const int row = m0 + quarter * 32 + lane;
                const bool row_ok = row < p.M;
                int64_t row_off;
                int64_t col_stride;
                if (p.omap) {
                    const int rr = row_ok ? row : 0;
                    row_off = (int64_t)(z / p.oz2) * p.ozs1 + (int64_t)(z % p.oz2) * p.ozs2 +
                              (int64_t)(rr / p.or2) * p.ors1 + (int64_t)(rr % p.or2) * p.ors2;
                    col_stride = p.ocs2; // within one column block (oc2 % 16 == 0)
                } else if (path == 0) {
                    const int mm = row_ok ? row : 0;
                    const int n_img = mm / (int)p.OHW;
                    const int pix = mm - n_img * (int)p.OHW;
                    row_off = (int64_t)z * p.out_zstride + (int64_t)n_img * p.out_img_stride + pix;
                    col_stride = p.OHW;
                } else {
                    row_off = (int64_t)z * p.out_zstride + (int64_t)(row_ok ? row : 0) * p.ldc;
                    col_stride = 1;
                }
                const float* __restrict__ bias = p.bias ? p.bias + (int64_t)z * p.bias_zstride : nullptr;
                const float* __restrict__ res = p.res;
                float* __restrict__ out = p.out;
                const float alpha = p.alpha, bsc = p.bias_scale, rsc = p.res_scale;
                const uint32_t acc0 = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + acc_col(b);
                int kb0, kcnt;
                kslice(t, kb0, kcnt);
                const bool two = !alt && kcnt > 1; // odd-block accumulator in use
                const bool piece = stream && !(kb0 == 0 && kcnt == nkb);
                if (piece) {
                    // balanced split, part of a tile: raw partials into this
                    // CTA's slot (0: its span's first unit, 1: its last), a
                    // 128 x BN tile, all rows
                    const int slot = t == u_first ? 0 : 1;
                    float* prow = p.part + (((int64_t)blockIdx.x * 2 + slot) * 128 + quarter * 32 + lane) * BN;
#pragma unroll 1
                    for (int cc = col_lo; cc < col_lo + kCols; cc += 16) {
                        float v[16], v1[16];
                        tmem_ld16(acc0 + cc, v);
                        if (two) {
                            tmem_ld16(acc0 + BN + cc, v1);
#pragma unroll
                            for (int j = 0; j < 16; ++j) {
                                v[j] += v1[j];
                            }
                        }
#pragma unroll
                        for (int j = 0; j < 16; j += 4) {
                            *reinterpret_cast<float4*>(prow + cc + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                        }
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(&acc_empty[b]);
                    }
                    continue;
                } else if (p.ksplit > 1) {
                    // raw partial sums of this K slice, row-major [M][N]
                    float* prow = p.part + ((int64_t)(kb0 / p.kper) * p.zcount + z) * p.M * p.N + (int64_t)row * p.N;
#pragma unroll 1
                    for (int cc = col_lo; cc < col_lo + kCols; cc += 16) {
                        if (n0 + cc >= p.N) {
                            break;
                        }
                        float v[16], v1[16];
                        tmem_ld16(acc0 + cc, v);
                        if (two) {
                            tmem_ld16(acc0 + BN + cc, v1);
                        }
                        if (two) {
#pragma unroll
                            for (int j = 0; j < 16; ++j) {
                                v[j] += v1[j];
                            }
                        }
                        if (row_ok && (p.N & 3) == 0 && n0 + cc + 16 <= p.N) {
                            // N % 4 == 0: the partial rows are 16-byte aligned
#pragma unroll
                            for (int j = 0; j < 16; j += 4) {
                                *reinterpret_cast<float4*>(prow + n0 + cc + j) =
                                    make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                            }
                        } else if (row_ok) {
#pragma unroll
                            for (int j = 0; j < 16; ++j) {
                                if (n0 + cc + j < p.N) {
                                    prow[n0 + cc + j] = v[j];
                                }
                            }
                        }
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(&acc_empty[b]);
                    }
                    continue;
                }
#pragma unroll 1
                for (int cc = col_lo; cc < col_lo + kCols; cc += 16) {
                    if (n0 + cc >= p.N) {
                        break; // warp-uniform: the rest is padding
                    }
                    float v[16];
                    {
                        float v1[16];
                        tmem_ld16(acc0 + cc, v);
                        if (two) {
                            tmem_ld16(acc0 + BN + cc, v1);
#pragma unroll
                            for (int j = 0; j < 16; ++j) {
                                v[j] += v1[j];
                            }
                        }
                    }
                    if (path == 2) {
                        // rows not 16-byte aligned: through this warp's shared
                        // tile, so a store writes two 64-byte row pieces
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            stile[lane * 17 + j] = v[j];
                        }
                        __syncwarp();
                        const int jj = lane & 15, hr = lane >> 4;
                        const int col = n0 + cc + jj;
                        const bool col_ok = col < p.N;
                        const float bl = (bias && col_ok) ? bsc * __ldg(bias + col) : 0.0f;
                        const int lim = p.M - (m0 + quarter * 32) - hr; // rows 2*rr + hr < M
                        const int64_t base = (int64_t)z * p.out_zstride + (int64_t)(m0 + quarter * 32 + hr) * p.ldc + col;
                        float* o = out + base;
                        const float* ro = res ? res + base : nullptr;
                        const int ld2 = 2 * static_cast<int>(p.ldc);
                        const float* sp = stile + hr * 17 + jj;
                        if (col_ok) {
                            if (ro) {
#pragma unroll
                                for (int rr = 0; rr < 16; ++rr) {
                                    if (2 * rr < lim) {
                                        const float x = fmaf(rsc, __ldg(ro + rr * ld2), fmaf(alpha, sp[rr * 34], bl));
                                        o[rr * ld2] = act_of<ACT>(x, p);
                                    }
                                }
                            } else {
#pragma unroll
                                for (int rr = 0; rr < 16; ++rr) {
                                    if (2 * rr < lim) {
                                        o[rr * ld2] = act_of<ACT>(fmaf(alpha, sp[rr * 34], bl), p);
                                    }
                                }
                            }
                        }
                        __syncwarp();
                    } else if (path == 1) {
                        // 16-byte rows: four vector stores per thread
                        if (row_ok && n0 + cc + 16 <= p.N) {
                            const int c0 = n0 + cc;
                            const int64_t o = row_off + (p.omap ? (int64_t)(c0 / p.oc2) * p.ocs1 + (c0 % p.oc2) : c0);
#pragma unroll
                            for (int j = 0; j < 16; j += 4) {
                                float4 bb = make_float4(0.f, 0.f, 0.f, 0.f), rv = bb;
                                if (bias) {
                                    bb = __ldg(reinterpret_cast<const float4*>(bias + n0 + cc + j));
                                }
                                if (res) {
                                    rv = __ldg(reinterpret_cast<const float4*>(res + o + j));
                                }
                                float4 w;
                                w.x = act_of<ACT>(fmaf(rsc, rv.x, fmaf(alpha, v[j], bsc * bb.x)), p);
                                w.y = act_of<ACT>(fmaf(rsc, rv.y, fmaf(alpha, v[j + 1], bsc * bb.y)), p);
                                w.z = act_of<ACT>(fmaf(rsc, rv.z, fmaf(alpha, v[j + 2], bsc * bb.z)), p);
                                w.w = act_of<ACT>(fmaf(rsc, rv.w, fmaf(alpha, v[j + 3], bsc * bb.w)), p);
                                *reinterpret_cast<float4*>(out + o + j) = w;
                            }
                        } else if (row_ok) {
                            for (int j = 0; j < 16 && n0 + cc + j < p.N; ++j) {
                                const int n = n0 + cc + j;
                                const int64_t o = row_off + (p.omap ? (int64_t)(n / p.oc2) * p.ocs1 + (n % p.oc2) : n);
                                const float bb = bias ? __ldg(bias + n) : 0.0f;
                                const float rv = res ? __ldg(res + o) : 0.0f;
                                out[o] = act_of<ACT>(fmaf(rsc, rv, fmaf(alpha, v[j], bsc * bb)), p);
                            }
                        }
                    } else {
                        // NCHW: a lane's row is a pixel, so each store covers 32
                        // consecutive pixels of one channel
                        // (a permuted output: the chunk lies in one column
                        // block, whose columns are col_stride apart)
                        const int c0 = n0 + cc;
                        const int64_t cb = row_off + (p.omap ? (int64_t)(c0 / p.oc2) * p.ocs1 + (int64_t)(c0 % p.oc2) * p.ocs2
                                                              : (int64_t)c0 * col_stride);
                        float rv[16];
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const int n = c0 + j;
                            rv[j] = (res && row_ok && n < p.N) ? __ldg(res + cb + (int64_t)j * col_stride) : 0.0f;
                        }
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const int n = c0 + j;
                            if (row_ok && n < p.N) {
                                const float bb = bias ? __ldg(bias + n) : 0.0f;
                                out[cb + (int64_t)j * col_stride] =
                                    act_of<ACT>(fmaf(rsc, rv[j], fmaf(alpha, v[j], bsc * bb)), p);
                            }
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&acc_empty[b]);
                }
            }
        };
        switch (p.act) {
        case kActRelu:
            tiles(ActTag<kActRelu>{});
            break;
        case kActSilu:
            tiles(ActTag<kActSilu>{});
            break;
        case kActSigmoid:
            tiles(ActTag<kActSigmoid>{});
            break;
        case kActGeluErf:
            tiles(ActTag<kActGeluErf>{});
            break;
        default:
            tiles(ActTag<kActNone>{});
            break;
        }
    } else if (warp == C::kTmaWarp || warp == C::kTmaAWarp || warp == C::kTmaBloWarp) {
        // ---------------- TMA issuers: B hi, raw A, B lo ----------------
        const int role = warp == C::kTmaWarp ? 0 : warp == C::kTmaAWarp ? 1 : 2;
        const bool active = role == 0 || (role == 1 && kTmaA) || (role == 2 && THREE);
        uint64_t* const my_full = role == 1 ? full_a : full_b;
        if (lane == 0 && active) {
            const CUtensorMap* map = role == 0 ? &tm_hi : role == 1 ? &tm_a : &tm_lo;
            prefetch_tmap(map);
            uint32_t g = 0;
            bool alive = true;
            for (int t = u_first; t < u_end && alive; t = u_next(t)) {
                int z, m0, n0;
                decode(t, z, m0, n0);
                const int row = n0 + z * p.b_zrows;
                int nn0 = 0, nh0 = 0, nw0 = 0; // kAConvNhwc: window start of the tile's first pixel
                if constexpr (MODE == kAConvNhwc) {
                    nn0 = m0 / (int)p.OHW;
                    const int pix = m0 - nn0 * (int)p.OHW;
                    const int oh = pix / p.OW;
                    nh0 = oh * p.sh - p.ph;
                    nw0 = (pix - oh * p.OW) * p.sw - p.pw;
                }
                int kb0, kcnt;
                kslice(t, kb0, kcnt);
                for (int kb = kb0; kb < kb0 + kcnt; ++kb, ++g) {
                    const int s = static_cast<int>(g % S);
                    const uint32_t ph = (g / S) & 1u;
                    uint64_t* free_bar = role == 1 ? &empty_a[s] : &empty[s];
                    if (!mbar_wait(free_bar, ph ^ 1u, abort_flag, p.err, p.wait_bound)) {
                        alive = false;
                        break;
                    }
                    if (role == 1) {
                        mbar_arrive_expect_tx(&my_full[s], C::kAPlane);
                        if constexpr (MODE == kADenseTma) {
                            tma_load_2d(a_raw(s), &tm_a, kb * 32, z * p.a_zrows + m0, &my_full[s]);
                        } else if constexpr (MODE == kAConvNhwc) {
                            // K ordered (kh, kw, cin): block kb = (tap, 32-channel block)
                            const int cblocks = p.Cg >> 5;
                            const int tap = kb / cblocks;
                            const int c0 = (kb - tap * cblocks) * 32;
                            const int kh = tap / p.KW, kw = tap - (tap / p.KW) * p.KW;
                            tma_load_im2col_4d(a_raw(s), &tm_a, c0, nw0, nh0, nn0, static_cast<uint16_t>(kw * p.dw),
                                               static_cast<uint16_t>(kh * p.dh), &my_full[s]);
                        }
                    } else {
                        mbar_arrive_expect_tx(&full_b[s], C::kBPlane);
                        tma_load_2d(role == 0 ? b_hi(s) : b_lo(s), map, kb * 32, row, &full_b[s]);
                    }
                }
            }
            // never leave with a bulk copy still landing in shared memory
            const uint32_t issued = g;
            for (uint32_t q = issued > S ? issued - S : 0; q < issued; ++q) {
                const long long t0 = clock64();
                while (!mbar_try_wait(&my_full[q % S], (q / S) & 1u) && clock64() - t0 < kWaitBoundCycles) {
                }
            }
        }
        __syncwarp();
    } else if (warp == C::kMmaWarp || warp == C::kMma2Warp) {
        // ---------------- MMA issuers: even / odd K blocks ----------------
        if (lane == 0) {
            const int par = warp == C::kMmaWarp ? 0 : 1;
            constexpr uint32_t idesc = idesc_tf32(128, BN);
            uint32_t g = 0;
            int i = 0;
            bool alive = true;
            for (int t = u_first; t < u_end && alive; t = u_next(t), ++i) {
                int kb0, kcnt;
                kslice(t, kb0, kcnt);
                if (alt && (i & 1) != par) {
                    g += static_cast<uint32_t>(kcnt); // the other issuer's tile
                    continue;
                }
                const int b = i % nbuf;
                if (!mbar_wait(&acc_empty[b], ((i / nbuf) & 1) ^ 1, abort_flag, p.err, p.wait_bound) ||
                    (alt && i > 0 && !mbar_wait(mma_turn, (i - 1) & 1, abort_flag, p.err, p.wait_bound))) {
                    break;
                }
                tc_fence_after();
                const uint32_t d0 = tmem + acc_col(b);
                for (int j = 0; j < kcnt; ++j, ++g) { // j = K block within the slice
                    if (!alt && (j & 1) != par) {
                        continue; // the other issuer's K block
                    }
                    const int s = static_cast<int>(g % S); // smem B stage == TMEM A stage
                    const uint32_t ph = (g / S) & 1u;
                    // TMA-fed A: the converter publishes only after B landed
                    if (!mbar_wait(&t_full[s], ph, abort_flag, p.err, p.wait_bound) ||
                        (!kTmaA && !mbar_wait(&full_b[s], ph, abort_flag, p.err, p.wait_bound))) {
                        alive = false;
                        break;
                    }
                    if (alt && j == kcnt - 1) {
                        mbar_arrive(mma_turn); // the next tile's issuer may start waiting
                    }
                    tc_fence_after();
                    const uint32_t d = d0 + static_cast<uint32_t>(alt ? 0 : (j & 1) * BN);
                    const uint32_t at = tmem + C::kAccCols + static_cast<uint32_t>(s * C::kAStageCols);
                    // a K step of 8 tf32 is 32 bytes: +2 in the descriptor's address field
                    const uint64_t bdh0 = sdesc_k128(smem_u32(b_hi(s))), bdl0 = sdesc_k128(smem_u32(b_lo(s)));
                    // the first K block into an accumulator overwrites it
                    const uint32_t first = (alt ? j == 0 : j < 2) ? 0u : 1u;
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint32_t acc = kk == 0 ? first : 1u;
                        if (THREE) {
                            mma_tf32_ta(d, at + 32 + kk * 8, bdh0 + 2 * kk, idesc, acc);
                            mma_tf32_ta(d, at + kk * 8, bdl0 + 2 * kk, idesc, 1u);
                            mma_tf32_ta(d, at + kk * 8, bdh0 + 2 * kk, idesc, 1u);
                        } else {
                            mma_tf32_ta(d, at + kk * 8, bdh0 + 2 * kk, idesc, acc);
                        }
                    }
                    mma_commit(&empty[s]);
                }
                if (alive) {
                    mma_commit(&acc_full[b]);
                }
            }
            // every MMA of this CTA must finish before TMEM is freed
            mma_commit(mma_done);
            const long long t0 = clock64();
            while (!mbar_try_wait(mma_done, 0) && clock64() - t0 < kWaitBoundCycles) {
            }
        }
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, C::kTmemCols);
    }
}

// ---- packing -------------------------------------------------------------

enum BLayout : int { kBRowsK = 0, kBKRows = 1, kBConvTap = 2 };

// out[z*rows + row][k] = hi/lo split of B(row, k), zero for k >= K.
// 32x32 tiles through shared memory so both the read and the write coalesce.
__global__ void pack_b_kernel(const float* __restrict__ src, int layout, int rows, int K, int Kpad, int64_t ld,
                              int64_t zstride, int Cg, int KHKW, int Cpad, float* __restrict__ hi,
                              float* __restrict__ lo) {
    __shared__ float tile[32][33];
    const int k0 = blockIdx.x * 32;
    const int r0 = blockIdx.y * 32;
    const int z = blockIdx.z;
    const float* s = src + (int64_t)z * zstride;
    const int tx = threadIdx.x, ty = threadIdx.y; // 32 x 8
    for (int i = ty; i < 32; i += 8) {
        if (layout == kBKRows) {
            // consecutive threads walk rows (contiguous in src)
            const int k = k0 + i, row = r0 + tx;
            tile[tx][i] = (k < K && row < rows) ? s[(int64_t)k * ld + row] : 0.0f;
        } else {
            const int k = k0 + tx, row = r0 + i;
            float v = 0.0f;
            if (k < K && row < rows) {
                if (layout == kBRowsK) {
                    v = s[(int64_t)row * ld + k];
                } else { // conv weight [M][Cg][KHKW], k = tap*Cpad + cin (zero for cin >= Cg)
                    const int tap = k / Cpad, cin = k - tap * Cpad;
                    v = cin < Cg ? s[((int64_t)row * Cg + cin) * KHKW + tap] : 0.0f;
                }
            }
            tile[i][tx] = v;
        }
    }
    __syncthreads();
    for (int i = ty; i < 32; i += 8) {
        const int row = r0 + i, k = k0 + tx;
        if (row < rows && k < Kpad) {
            const float v = tile[i][tx];
            uint32_t h;
            asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(v));
            const float hv = __uint_as_float(h);
            const int64_t o = ((int64_t)z * rows + row) * Kpad + k;
            hi[o] = hv;
            lo[o] = v - hv;
        }
    }
}

// Per-k tap table for the generic conv gather: x = cin*H*W + kh*dh*W + kw*dw,
// y = (kh*dh << 16) | kw*dw, or y = -1 for the zero padding k >= K.
__global__ void conv_ktab_kernel(int2* tab, int K, int Kpad, int KHKW, int KW, int dh, int dw, int64_t HW, int W) {
    const int k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= Kpad) {
        return;
    }
    if (k >= K) {
        tab[k] = make_int2(0, -1);
        return;
    }
    const int cin = k / KHKW;
    const int t = k - cin * KHKW;
    const int kh = t / KW, kw = t - kh * KW;
    tab[k] = make_int2(static_cast<int>(cin * HW + (int64_t)kh * dh * W + (int64_t)kw * dw), ((kh * dh) << 16) | (kw * dw));
}

__device__ __forceinline__ float act_rt(float v, const Args& p) {
    switch (p.act) {
    case kActRelu:
        return act_of<kActRelu>(v, p);
    case kActSilu:
        return act_of<kActSilu>(v, p);
    case kActSigmoid:
        return act_of<kActSigmoid>(v, p);
    case kActGeluErf:
        return act_of<kActGeluErf>(v, p);
    default:
        return v;
    }
}

// Split K: sums the K slices' partials in slice order (deterministic) and
// applies the contraction's epilogue and output layout.
__global__ void splitk_reduce_kernel(const __grid_constant__ Args p) {
    const int64_t total = (int64_t)p.zcount * p.M * p.N;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int col = static_cast<int>(i % p.N);
        const int64_t t = i / p.N;
        const int row = static_cast<int>(t % p.M);
        const int z = static_cast<int>(t / p.M);
        float acc = 0.0f;
        for (int ks = 0; ks < p.ksplit; ++ks) {
            acc += p.part[(int64_t)ks * total + i];
        }
        int64_t off;
        if (p.conv_out) {
            const int n_img = row / (int)p.OHW;
            const int pix = row - n_img * (int)p.OHW;
            off = (int64_t)z * p.out_zstride + (int64_t)n_img * p.out_img_stride + pix + (int64_t)col * p.OHW;
        } else {
            off = (int64_t)z * p.out_zstride + (int64_t)row * p.ldc + col;
        }
        const float bb = p.bias ? p.bias[(int64_t)z * p.bias_zstride + col] : 0.0f;
        const float rv = p.res ? p.res[off] : 0.0f;
        p.out[off] = act_rt(fmaf(p.res_scale, rv, fmaf(p.alpha, acc, p.bias_scale * bb)), p);
    }
}

// Balanced split: each tile whose K blocks crossed a CTA span boundary sums
// its pieces in CTA order (deterministic) and applies the epilogue. Blocks
// (tile, y): a thread takes four consecutive columns of one row, loads the
// pieces' 16-byte vectors, then writes the four outputs; tiles done whole by
// one CTA return at once.
template <int BN>
__global__ void __launch_bounds__(256) streamk_reduce_kernel(const __grid_constant__ Args p) {
    const int tile = blockIdx.x;
    const int nkb = p.nkb, span = p.sk_span;
    const int g0 = tile * nkb, g1 = g0 + nkb;
    const int c_first = g0 / span, c_last = (g1 - 1) / span;
    if (c_first == c_last) {
        return;
    }
    const int num_m = (p.M + 127) / 128;
    const int num_n = (p.N + BN - 1) / BN;
    const int tiles_per_z = num_m * num_n;
    const int z = tile / tiles_per_z;
    const int r = tile - z * tiles_per_z;
    const int nt = r / num_m;
    const int m0 = (r - nt * num_m) * 128, n0 = nt * BN;
    for (int q = blockIdx.y * blockDim.x + threadIdx.x; q < 128 * BN / 4; q += gridDim.y * blockDim.x) {
        const int e = q * 4;
        const int lr = e / BN, lc = e - lr * BN;
        const int row = m0 + lr;
        if (row >= p.M || n0 + lc >= p.N) {
            continue;
        }
        // up to four pieces loaded before the sum (a tile spans at most
        // ceil(nkb / span) + 1 CTAs), then any further ones; CTA order kept
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        float4 v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int c = c_first + j;
            if (c <= c_last) {
                const int slot = (c * span >= g0) ? 0 : 1;
                v[j] = __ldg(reinterpret_cast<const float4*>(p.part + ((int64_t)c * 2 + slot) * 128 * BN + e));
            }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if (c_first + j <= c_last) {
                acc.x += v[j].x, acc.y += v[j].y, acc.z += v[j].z, acc.w += v[j].w;
            }
        }
        for (int c = c_first + 4; c <= c_last; ++c) {
            const float4 w = __ldg(reinterpret_cast<const float4*>(p.part + ((int64_t)c * 2) * 128 * BN + e));
            acc.x += w.x, acc.y += w.y, acc.z += w.z, acc.w += w.w;
        }
        const float a4[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int col = n0 + lc + j;
            if (col >= p.N) {
                break;
            }
            int64_t off;
            if (p.omap) { // the permuted output map of the main epilogue
                off = (int64_t)(z / p.oz2) * p.ozs1 + (int64_t)(z % p.oz2) * p.ozs2 +
                      (int64_t)(row / p.or2) * p.ors1 + (int64_t)(row % p.or2) * p.ors2 +
                      (int64_t)(col / p.oc2) * p.ocs1 + (int64_t)(col % p.oc2) * p.ocs2;
            } else if (p.conv_out) {
                const int n_img = row / (int)p.OHW;
                const int pix = row - n_img * (int)p.OHW;
                off = (int64_t)z * p.out_zstride + (int64_t)n_img * p.out_img_stride + pix + (int64_t)col * p.OHW;
            } else {
                off = (int64_t)z * p.out_zstride + (int64_t)row * p.ldc + col;
            }
            const float bb = p.bias ? p.bias[(int64_t)z * p.bias_zstride + col] : 0.0f;
            const float rv = p.res ? p.res[off] : 0.0f;
            p.out[off] = act_rt(fmaf(p.res_scale, rv, fmaf(p.alpha, a4[j], p.bias_scale * bb)), p);
        }
    }
}

// 2-D fp32 map over [rows][inner] (row stride `ld` elements) with 32 x
// box_rows boxes in the 128-byte swizzle; out-of-range boxes read zeros.
void make_tmap(CUtensorMap* map, const float* base, int64_t inner, int64_t rows, int box_rows, int64_t ld = -1) {
    if (ld < 0) {
        ld = inner;
    }
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 4)};
    const cuuint32_t box[2] = {32, static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode_tiled()(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides,
                                      box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        fail(kStatusCuda, "cuTensorMapEncodeTiled failed (" + std::to_string(static_cast<int>(r)) + ")");
    }
}

template <int BN, bool THREE, int MODE, bool STREAM>
void launch_variant(nb2_device* dev, const Args& a, dim3 grid, const CUtensorMap& hi, const CUtensorMap& lo,
                    const CUtensorMap& am) {
    using C = Cfg<BN, THREE, tma_a_mode<MODE>()>;
    const int smem = C::kSmemBytes + (a.ktab_smem ? a.nkb * 32 * 8 : 0);
    static int attr_bytes[64] = {};
    if (attr_bytes[dev->ordinal] < smem) {
        check_cuda(cudaFuncSetAttribute(igemm_kernel<BN, THREE, MODE, STREAM>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                   "cudaFuncSetAttribute(igemm)");
        attr_bytes[dev->ordinal] = smem;
    }
    igemm_kernel<BN, THREE, MODE, STREAM><<<grid, C::kThreads, smem, dev->stream>>>(a, hi, lo, am);
    check_cuda(cudaGetLastError(), "igemm launch");
}

template <int BN, bool THREE, int MODE>
void launch_mode(nb2_device* dev, const Args& a, dim3 grid, const CUtensorMap& hi, const CUtensorMap& lo,
                 const CUtensorMap& am) {
    if constexpr (BN == 128) {
        if (a.stream) {
            launch_variant<BN, THREE, MODE, true>(dev, a, grid, hi, lo, am);
            return;
        }
    }
    launch_variant<BN, THREE, MODE, false>(dev, a, grid, hi, lo, am);
}

template <int BN, bool THREE>
void launch_bn(nb2_device* dev, const Args& a, dim3 grid, const CUtensorMap& hi, const CUtensorMap& lo,
               const CUtensorMap& am) {
    switch (a.mode) {
    case kAConvTap:
        launch_mode<BN, THREE, kAConvTap>(dev, a, grid, hi, lo, am);
        break;
    case kAConvGeneric:
        launch_mode<BN, THREE, kAConvGeneric>(dev, a, grid, hi, lo, am);
        break;
    case kADenseK:
        launch_mode<BN, THREE, kADenseK>(dev, a, grid, hi, lo, am);
        break;
    case kADenseTma:
        launch_mode<BN, THREE, kADenseTma>(dev, a, grid, hi, lo, am);
        break;
    case kAConvNhwc:
        launch_mode<BN, THREE, kAConvNhwc>(dev, a, grid, hi, lo, am);
        break;
    case kAConvCvec:
        launch_mode<BN, THREE, kAConvCvec>(dev, a, grid, hi, lo, am);
        break;
    default:
        launch_mode<BN, THREE, kADenseM>(dev, a, grid, hi, lo, am);
        break;
    }
}

} // namespace

int split_k_slices(const nb2_device* dev, int64_t tiles, int nkb, int* kper) {
    *kper = nkb;
    if (tiles * 2 > dev->num_sms || nkb < 8) {
        return 1;
    }
    int ks = static_cast<int>(std::min<int64_t>(nkb / 4, (dev->num_sms + tiles - 1) / tiles));
    *kper = (nkb + ks - 1) / ks;
    return (nkb + *kper - 1) / *kper;
}

// Tile width: 64 for narrow outputs; for short K (<= 4 blocks) 64 as well,
// since a 64-wide tile's double-buffered accumulator lets the epilogue
// overlap the next tile (measured 10-12% faster on 1x1 convs with K = 64,
// 128), unless every CTA gets at least four 128-wide tiles, which then keep
// two tiles in flight too.
int tile_width(const nb2_device* dev, int64_t M, int64_t n_per_z, int nkb, int64_t z) {
    if (n_per_z <= 64) {
        return 64;
    }
    if (nkb > 4) {
        return 128;
    }
    const int64_t t128 = ((M + 127) / 128) * ((n_per_z + 127) / 128) * z;
    return t128 >= 4 * static_cast<int64_t>(dev->num_sms) ? 128 : 64;
}

// Balanced split for 128-wide tiles whose count leaves the last wave short
// (e.g. 52, 100 or 196 tiles on 148 SMs): every CTA takes an equal span of
// the (tile, K block) pairs. Cost model in K-block times: a unit costs its K
// blocks plus ~9 for the single-buffered accumulator's drain, a reduce ~11;
// compared with the unsplit tiles or, where those apply, equal K slices.
// Taken when it saves at least 10%; returns the span (0: not taken).
// Measured on ResNet-18 bs64 layers 3 and 4 (196 and 100 tiles): 103 -> 78
// µs per contraction kernel plus 6-15 µs of reduce.
int64_t balanced_span(const nb2_device* dev, int64_t tiles, int nkb, int bn) {
    if (bn != 128 || nkb < 8 || dev->no_grow || tiles * nkb >= (1LL << 30)) {
        return 0;
    }
    const int64_t G = dev->num_sms, E = 9, R = 11;
    int64_t other = (tiles + G - 1) / G * (nkb + E); // unsplit
    int kper = nkb;
    const int ks = split_k_slices(dev, tiles, nkb, &kper);
    if (ks > 1) { // equal K slices
        other = (tiles * ks + G - 1) / G * (kper + E) + R;
    }
    const int64_t span = (tiles * nkb + G - 1) / G;
    const int64_t balanced = span + ((span + nkb - 1) / nkb + 1) * E + R;
    // (with no margin ViT-B/16 fc1, 1200 tiles of 24 K blocks, and several
    // ResNet-50 layers took it and lost 2-8% against two tiles in flight or
    // the unsplit tiles: the model leaves out the epilogue overlap they have)
    return balanced * 10 < other * 9 ? span : 0;
}

int contraction_launches(const nb2_device* dev, int64_t M, int64_t n_per_z, int64_t K, int64_t z) {
    const int nkb = static_cast<int>((K + 31) / 32);
    const int bn = tile_width(dev, M, n_per_z, nkb, z);
    const int64_t tiles = ((M + 127) / 128) * ((n_per_z + bn - 1) / bn) * z;
    int kper = 0;
    return (balanced_span(dev, tiles, nkb, bn) > 0 || split_k_slices(dev, tiles, nkb, &kper) > 1) ? 2 : 1;
}

namespace {

void launch(nb2_device* dev, Args& a, int64_t n_per_z, int64_t z, const float* packed, int64_t rows_total,
            const CUtensorMap* a_map = nullptr) {
    const int64_t kpad = static_cast<int64_t>(a.nkb) * 32;
    const int bn = tile_width(dev, a.M, n_per_z, a.nkb, z);
    CUtensorMap hi, lo;
    make_tmap(&hi, packed, kpad, rows_total, bn);
    make_tmap(&lo, packed + rows_total * kpad, kpad, rows_total, bn);
    a.err = dev->err_word;
    a.wait_bound = dev->wait_bound;
    a.zcount = static_cast<int>(z);
    auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    a.vec_out = (!a.conv_out && a.ldc % 4 == 0 && a.out_zstride % 4 == 0 && al16(a.out) &&
                 (a.res == nullptr || al16(a.res)) && (a.bias == nullptr || (al16(a.bias) && a.bias_zstride % 4 == 0)))
                    ? 1
                    : 0;
    if (a.omap) {
        // 16 contiguous columns per chunk when the block stride is 1 and
        // every offset keeps 16-byte alignment; else lanes over rows
        const bool v = a.ocs2 == 1 && a.oc2 % 16 == 0 && a.N % 16 == 0 && a.ozs1 % 4 == 0 && a.ozs2 % 4 == 0 &&
                       a.ors1 % 4 == 0 && a.ors2 % 4 == 0 && a.ocs1 % 4 == 0 && al16(a.out) &&
                       (a.bias == nullptr || al16(a.bias));
        a.vec_out = v ? 1 : 0;
        a.conv_out = v ? 0 : 1;
    }
    a.ktab_smem = ((a.mode == kAConvGeneric && kpad * 8 <= 16384) || a.mode == kAConvCvec) ? 1 : 0;
    if (a.mode == kAConvCvec && kpad * 8 > 16384) {
        fail(kStatusUnsupported, "Conv: filter too large for the narrow-channel input path");
    }
    // row-major A with 16-byte rows: TMA it (a zero stride broadcasts one A)
    CUtensorMap am = a_map ? *a_map : hi;
    if (a.mode == kADenseK && a.vec4 && (a.a_zstride % a.lda) == 0) {
        a.mode = kADenseTma;
        a.a_zrows = static_cast<int>(a.a_zstride / a.lda);
        const int64_t a_rows = a.a_zstride == 0 ? a.M : static_cast<int64_t>(a.a_zrows) * (z - 1) + a.M;
        make_tmap(&am, a.a, a.K, a_rows, 128, a.lda);
    }
    const int64_t tiles = ((a.M + 127) / 128) * ((n_per_z + bn - 1) / bn) * z;
    if (tiles >= (1LL << 31)) {
        fail(kStatusUnsupported, "igemm: too many tiles");
    }
    // Split K when the tiles would leave most SMs idle and K is long: each
    // (tile, K slice) is a work unit, slices keep >= 4 K blocks.
    a.ksplit = 1;
    a.kper = a.nkb;
    a.part = nullptr;
    int kper = a.nkb;
    // the equal-slice reduce writes row-major or NCHW, not through an output map
    const int64_t bspan = balanced_span(dev, tiles, a.nkb, bn);
    const int ks = (a.omap || bspan > 0) ? 1 : split_k_slices(dev, tiles, a.nkb, &kper);
    if (ks > 1) {
        const size_t bytes = static_cast<size_t>(ks) * static_cast<size_t>(z) * a.M * n_per_z * sizeof(float);
        float* part = static_cast<float*>(dev->split_scratch(bytes));
        if (part != nullptr) {
            a.ksplit = ks;
            a.kper = kper;
            a.part = part;
        }
    }
    a.stream = 0;
    if (bspan > 0) {
        const size_t bytes = static_cast<size_t>(dev->num_sms) * 2 * 128 * bn * sizeof(float);
        float* part = static_cast<float*>(dev->split_scratch(bytes));
        if (part != nullptr) {
            a.stream = 1;
            a.sk_span = static_cast<int>(bspan);
            a.sk_total = static_cast<int>(tiles * a.nkb);
            a.part = part;
        }
    }
    // persistent: one CTA per SM (shared memory admits exactly one)
    const dim3 grid(static_cast<unsigned>(a.stream ? std::min<int64_t>((a.sk_total + a.sk_span - 1) / a.sk_span,
                                                                          dev->num_sms)
                                                   : std::min<int64_t>(tiles * a.ksplit, dev->num_sms)),
                    1, 1);
    // two 128-wide tiles in flight once every CTA has several short-K
    // tiles (with one or two tiles per CTA, or long K, the single issuer's
    // gaps between K blocks cost more than the epilogue overlap saves:
    // measured 10-15% slower on 4096^3)
    a.alt = (bn == 128 && a.ksplit == 1 && !a.stream && a.nkb <= 32 && tiles >= 4 * static_cast<int64_t>(grid.x))
                ? 1
                : 0;
    dev->last_sched.tile_n = bn;
    dev->last_sched.alt = a.alt;
    dev->last_sched.ksplit = a.stream ? 0 : a.ksplit;
    dev->last_sched.a_mode = a.mode;
    dev->last_sched.grid = static_cast<int>(grid.x);
    dev->last_sched.tiles = tiles;
    const bool three = dev->precision == kPrec3xTF32;
    if (bn == 64) {
        three ? launch_bn<64, true>(dev, a, grid, hi, lo, am) : launch_bn<64, false>(dev, a, grid, hi, lo, am);
    } else {
        three ? launch_bn<128, true>(dev, a, grid, hi, lo, am) : launch_bn<128, false>(dev, a, grid, hi, lo, am);
    }
    if (a.stream) {
        streamk_reduce_kernel<128><<<dim3(static_cast<unsigned>(tiles), 16), 256, 0, dev->stream>>>(a);
        check_cuda(cudaGetLastError(), "balanced-split reduce launch");
    }
    if (a.ksplit > 1) {
        const int64_t total = z * a.M * static_cast<int64_t>(n_per_z);
        const unsigned blocks = static_cast<unsigned>(std::min<int64_t>((total + 255) / 256, dev->num_sms * 8));
        splitk_reduce_kernel<<<blocks, 256, 0, dev->stream>>>(a);
        check_cuda(cudaGetLastError(), "split-K reduce launch");
    }
}

void fill_epilogue(Args& a, const Epilogue& ep) {
    a.alpha = ep.alpha;
    a.act_a = ep.act_a;
    a.act_b = ep.act_b;
    a.act_c = ep.act_c;
    a.bias = ep.bias;
    a.bias_scale = ep.bias_scale;
    a.res = ep.res;
    a.res_scale = ep.res_scale;
    a.act = ep.act;
}

} // namespace

// ---- Conv ------------------------------------------------------------------

ConvGeom nchw_input_layout(const ConvGeom& g) {
    if (g.group != 1 || g.in_nhwc || g.cvec || g.cpad) {
        return g;
    }
    ConvGeom r = g;
    if (g.C <= 16) {
        r.cvec = g.C <= 4 ? 4 : (g.C <= 8 ? 8 : 16);
        return r;
    }
    if (g.KH * g.KW > 1 && g.H * g.W > 1) {
        r.cpad = round_up(g.C, 32);
        r.in_nhwc = true;
        if (r.nhwc_input_ok()) {
            return r;
        }
    }
    return g;
}

size_t conv_packed_bytes(const ConvGeom& g) {
    const int64_t kpad = round_up(g.K(), 32);
    size_t bytes = static_cast<size_t>(2 * g.M * kpad * 4);
    if (!g.tap_major()) {
        bytes += static_cast<size_t>(kpad * 8);
    }
    return bytes;
}

void conv_pack(nb2_device* dev, const ConvGeom& g, const float* w, void* packed) {
    const int64_t K = g.K(), kpad = round_up(K, 32);
    float* hi = static_cast<float*>(packed);
    float* lo = hi + g.M * kpad;
    const int layout = g.tap_major() ? kBConvTap : kBRowsK;
    const dim3 grid(static_cast<unsigned>(kpad / 32), static_cast<unsigned>((g.M + 31) / 32), 1);
    pack_b_kernel<<<grid, dim3(32, 8), 0, dev->stream>>>(w, layout, static_cast<int>(g.M), static_cast<int>(K),
                                                        static_cast<int>(kpad), K, 0, static_cast<int>(g.Cg()),
                                                        static_cast<int>(g.KH * g.KW), static_cast<int>(g.Cpad()),
                                                        hi, lo);
    check_cuda(cudaGetLastError(), "pack_b launch");
    if (!g.tap_major()) {
        int2* tab = reinterpret_cast<int2*>(lo + g.M * kpad);
        conv_ktab_kernel<<<static_cast<unsigned>((kpad + 255) / 256), 256, 0, dev->stream>>>(
            tab, static_cast<int>(K), static_cast<int>(kpad), static_cast<int>(g.KH * g.KW), static_cast<int>(g.KW),
            static_cast<int>(g.dh), static_cast<int>(g.dw), g.H * g.W, static_cast<int>(g.W));
        check_cuda(cudaGetLastError(), "ktab launch");
    }
}

void conv_run(nb2_device* dev, const ConvGeom& g, const float* x, const void* packed, float* y, const Epilogue& ep) {
    const int64_t K = g.K(), kpad = round_up(K, 32);
    const int64_t ohw = g.OH * g.OW;
    const int64_t m_total = g.N * ohw;
    if (m_total >= (1LL << 31) || g.C * g.H * g.W >= (1LL << 31) || ohw * g.M >= (1LL << 31)) {
        fail(kStatusUnsupported, "Conv: tensor too large for 32-bit tile indexing");
    }
    Args a{};
    a.M = static_cast<int>(m_total);
    a.N = static_cast<int>(g.Mg());
    a.K = static_cast<int>(K);
    a.nkb = static_cast<int>(kpad / 32);
    // NHWC inputs always take TMA im2col: measured, gathering the same
    // channels-last rows with 16-byte loads from the producer warps is
    // 20-50% slower per layer even where one im2col copy per K block
    // (~850 cycles) bounds the main loop
    a.mode = g.cvec ? kAConvCvec : g.in_nhwc ? kAConvNhwc : g.tap_major() ? kAConvTap : kAConvGeneric;
    if (g.in_nhwc && !g.nhwc_input_ok()) {
        fail(kStatusUnsupported, "Conv: NHWC input needs group 1, C % 4 == 0 (K padded to 32 channels a tap) "
                                 "and strides <= 8");
    }
    if (g.cvec && (!g.cvec_input_ok(g.cvec) || g.in_nhwc)) {
        fail(kStatusUnsupported, "Conv: the narrow-channel input form needs group 1, C <= cv, cv in {4, 8, 16}");
    }
    a.a = x;
    a.a_zstride = g.Cg() * g.H * g.W;
    a.C = static_cast<int>(g.C);
    a.H = static_cast<int>(g.H);
    a.W = static_cast<int>(g.W);
    a.OH = static_cast<int>(g.OH);
    a.OW = static_cast<int>(g.OW);
    a.KH = static_cast<int>(g.KH);
    a.KW = static_cast<int>(g.KW);
    a.sh = static_cast<int>(g.sh);
    a.sw = static_cast<int>(g.sw);
    a.ph = static_cast<int>(g.ph);
    a.pw = static_cast<int>(g.pw);
    a.dh = static_cast<int>(g.dh);
    a.dw = static_cast<int>(g.dw);
    a.Cg = static_cast<int>(g.Cpad()); // channels per tap in the K layout
    a.HW = g.H * g.W;
    a.OHW = ohw;
    a.img_stride = g.Cin() * g.H * g.W;
    const float* hi = static_cast<const float*>(packed);
    a.ktab = g.tap_major() ? nullptr : reinterpret_cast<const int2*>(hi + 2 * g.M * kpad);
    a.b_zrows = static_cast<int>(g.Mg());
    a.out = y;
    if (g.out_nhwc) {
        // rows are pixels, columns channels: y[pixel][M]; a group is a channel offset
        a.conv_out = 0;
        a.ldc = g.M;
        a.out_zstride = g.Mg();
    } else {
        a.out_zstride = g.Mg() * ohw;
        a.out_img_stride = g.M * ohw;
        a.conv_out = 1;
    }
    a.bias_zstride = static_cast<int>(g.Mg());
    fill_epilogue(a, ep);
    if (g.in_nhwc) {
        // im2col map over x[N][H][W][C]: window starts from -pad to the last
        // start (the upper corner is pad_end - dil*(k-1), relative to the far
        // edge); 128 pixels x 32 channels per load, 128-byte swizzle.
        CUtensorMap am;
        const int64_t ci = g.Cin(); // channels held by the NHWC input (C, or padded)
        const cuuint64_t dims[4] = {static_cast<cuuint64_t>(ci), static_cast<cuuint64_t>(g.W),
                                    static_cast<cuuint64_t>(g.H), static_cast<cuuint64_t>(g.N)};
        const cuuint64_t strides[3] = {static_cast<cuuint64_t>(ci * 4), static_cast<cuuint64_t>(g.W * ci * 4),
                                       static_cast<cuuint64_t>(g.H * g.W * ci * 4)};
        const int64_t pb = g.pad_bottom(), pr = g.pad_right();
        const int lower[2] = {static_cast<int>(-g.pw), static_cast<int>(-g.ph)};
        const int upper[2] = {static_cast<int>(pr - g.dw * (g.KW - 1)), static_cast<int>(pb - g.dh * (g.KH - 1))};
        const cuuint32_t estr[4] = {1, static_cast<cuuint32_t>(g.sw), static_cast<cuuint32_t>(g.sh), 1};
        const CUresult r = encode_im2col()(&am, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float*>(x), dims,
                                           strides, lower, upper, 32, 128, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) {
            fail(kStatusCuda, "cuTensorMapEncodeIm2col failed (" + std::to_string(static_cast<int>(r)) + ")");
        }
        launch(dev, a, g.Mg(), g.group, hi, g.M, &am);
        return;
    }
    launch(dev, a, g.Mg(), g.group, hi, g.M);
}

// ---- Gemm / MatMul -----------------------------------------------------------

size_t gemm_packed_bytes(const GemmGeom& g) {
    const int64_t kpad = round_up(g.K, 32);
    return static_cast<size_t>(2 * g.batch * g.N * kpad * 4);
}

void gemm_pack_b(nb2_device* dev, const GemmGeom& g, const float* b, void* packed) {
    const int64_t kpad = round_up(g.K, 32);
    float* hi = static_cast<float*>(packed);
    float* lo = hi + g.batch * g.N * kpad;
    // op(B) is [K,N]; packed rows are the N columns. transB=1 stores B as
    // [N,K] (rows already K-major); transB=0 stores [K,N].
    const int layout = g.trans_b ? kBRowsK : kBKRows;
    const dim3 grid(static_cast<unsigned>(kpad / 32), static_cast<unsigned>((g.N + 31) / 32),
                    static_cast<unsigned>(g.batch));
    pack_b_kernel<<<grid, dim3(32, 8), 0, dev->stream>>>(b, layout, static_cast<int>(g.N), static_cast<int>(g.K),
                                                        static_cast<int>(kpad), g.ldb, g.b_zstride, 1, 1, 1, hi, lo);
    check_cuda(cudaGetLastError(), "pack_b launch");
}

void gemm_run(nb2_device* dev, const GemmGeom& g, const float* a_ptr, const void* packed_b, float* y,
              const Epilogue& ep) {
    if (g.M >= (1LL << 31) || g.N >= (1LL << 31) || g.K >= (1LL << 31)) {
        fail(kStatusUnsupported, "Gemm: dimension too large");
    }
    const int64_t kpad = round_up(g.K, 32);
    Args a{};
    a.M = static_cast<int>(g.M);
    a.N = static_cast<int>(g.N);
    a.K = static_cast<int>(g.K);
    a.nkb = static_cast<int>(kpad / 32);
    a.mode = g.trans_a ? kADenseM : kADenseK;
    a.a = a_ptr;
    a.a_zstride = g.a_zstride;
    a.lda = g.lda;
    a.vec4 = (!g.trans_a && g.K % 4 == 0 && g.lda % 4 == 0 && (reinterpret_cast<uintptr_t>(a_ptr) & 15) == 0 &&
              (g.a_zstride % 4) == 0)
                 ? 1
                 : 0;
    a.b_zrows = static_cast<int>(g.N);
    a.out = y;
    a.out_zstride = g.c_zstride;
    a.ldc = g.ldc;
    a.conv_out = 0;
    a.bias_zstride = 0;
    if (g.omap.on) {
        if (g.omap.c2 % 16 != 0 || g.omap.z2 < 1 || g.omap.r2 < 1 || ep.res != nullptr) {
            fail(kStatusUnsupported, "Gemm: permuted output needs column blocks of 16k and no residual");
        }
        a.omap = 1;
        a.oz2 = static_cast<int>(g.omap.z2);
        a.or2 = static_cast<int>(g.omap.r2);
        a.oc2 = static_cast<int>(g.omap.c2);
        a.ozs1 = g.omap.zs1;
        a.ozs2 = g.omap.zs2;
        a.ors1 = g.omap.rs1;
        a.ors2 = g.omap.rs2;
        a.ocs1 = g.omap.cs1;
        a.ocs2 = g.omap.cs2;
    }
    fill_epilogue(a, ep);
    launch(dev, a, g.N, g.batch, static_cast<const float*>(packed_b), g.batch * g.N);
}

} // namespace nb2
