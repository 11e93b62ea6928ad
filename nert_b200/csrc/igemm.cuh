// Host-facing interface of the tcgen05 contraction engine (igemm.cu).
//
// One kernel serves Conv (implicit GEMM on NCHW), Gemm and batched MatMul:
//     D[z][M x N] = A[z][M x K] * B[z][N x K]^T, then a fused epilogue
//     v = alpha*acc + bias_scale*bias[n] + res_scale*res[off]; act(v).
// A is gathered by producer warps straight from the fp32 source (im2col
// addressing for Conv, row- or column-major for dense operands) and split into
// tf32 hi/lo planes in shared memory; B is a pre-packed, pre-split K-major
// matrix [rows][Kpad] (hi plane, then lo plane) fetched by TMA.
#pragma once

#include "runtime.hpp"

#include <cstdint>

namespace nb2 {

// kActGeluErf: ((x * (erf(x / act_a) + act_b)) * act_c), the erf form of GELU
// as exported to ONNX (Div, Erf, Add, Mul, Mul).
enum Act : int { kActNone = 0, kActRelu = 1, kActSilu = 2, kActSigmoid = 3, kActGeluErf = 4 };

struct Epilogue {
    float alpha = 1.0f;
    const float* bias = nullptr; // per output column n (per output channel for Conv)
    float bias_scale = 1.0f;
    const float* res = nullptr; // same layout as the output
    float res_scale = 1.0f;
    int act = kActNone;
    float act_a = 0.f, act_b = 0.f, act_c = 0.f;
};

// 2-D convolution geometry (1-D convolutions use H = KH = 1).
struct ConvGeom {
    int64_t N, C, H, W;  // input
    int64_t M, KH, KW;   // weight [M, C/group, KH, KW]
    int64_t OH, OW;      // output
    int64_t sh, sw, ph, pw, dh, dw, group;
    static constexpr int64_t kPadUnset = INT64_MIN;
    int64_t pb = kPadUnset, pr = kPadUnset; // bottom / right padding (unset: as top / left)
    // Physical layouts (the engine keeps ResNet-style trunks in NHWC; the
    // C ABI and the nert::Device rows are NCHW). An NHWC input needs
    // nhwc_input_ok(): A is then brought in by TMA im2col.
    bool in_nhwc = false, out_nhwc = false;
    // Narrow input given as x[N][H][W][cvec] (C <= cvec channels zero padded,
    // cvec = 4, 8 or 16; e.g. a stem's image): K ordered (tap, channel).
    int64_t cvec = 0;
    // NHWC input holding cpad >= C channels (zero padded to a multiple of 32
    // for the TMA im2col form); 0 = exactly C.
    int64_t cpad = 0;
    // cpad pads only the packed K layout: the NHWC input holds exactly C
    // channels (C % 4 == 0, 16-byte pixels) and the TMA im2col copy of the
    // last channel block reads the channels past C as zeros.
    bool cpad_k_only = false;
    int64_t Cg() const { return C / group; }
    int64_t Mg() const { return M / group; }
    // channels per pixel of the input tensor
    int64_t Cin() const { return cvec ? cvec : (cpad && !cpad_k_only ? cpad : C); }
    // the NCHW input is first copied to a padded NHWC buffer
    bool converts_input() const { return cvec != 0 || (cpad != 0 && !cpad_k_only); }
    // this geometry with its input read channels-last where it lies
    ConvGeom nhwc_in_place() const {
        ConvGeom r = *this;
        r.in_nhwc = true;
        if (group == 1 && C % 32 != 0 && cvec == 0 && cpad == 0) {
            r.cpad = (C + 31) / 32 * 32;
            r.cpad_k_only = true;
        }
        return r;
    }
    // channels per filter tap in the packed K layout
    int64_t Cpad() const { return cvec ? cvec : (cpad ? cpad : Cg()); }
    int64_t K() const { return Cpad() * KH * KW; }
    bool tap_major() const { return cvec || cpad || Cg() % 32 == 0; }
    bool cvec_input_ok(int64_t cv) const { return group == 1 && C <= cv && (cv == 4 || cv == 8 || cv == 16); }
    int64_t pad_bottom() const { return pb == kPadUnset ? ph : pb; }
    int64_t pad_right() const { return pr == kPadUnset ? pw : pr; }
    // TMA im2col limits for a 4-D map: traversal strides 1..8, box corners in
    // [-128, 127] and filter offsets in [0, 255] (kept well inside here).
    bool nhwc_input_ok() const {
        return group == 1 && Cpad() % 32 == 0 && Cin() % 4 == 0 && sh >= 1 && sh <= 8 && sw >= 1 && sw <= 8 && ph <= 64 && pw <= 64 &&
               pad_bottom() >= -64 && pad_bottom() <= 64 && pad_right() >= -64 && pad_right() <= 64 &&
               dh * (KH - 1) <= 64 && dw * (KW - 1) <= 64;
    }
};

int64_t round_up(int64_t v, int64_t m);

// ConvTranspose geometry (NCHW): x [N,C,H,W], w [C, M/group, KH, KW],
// y [N,M,OH,OW]; begin pads (ph, pw), end pads (pb, pr), output_padding
// (oph, opw).
struct ConvTGeom {
    int64_t N, C, H, W, M, KH, KW, OH, OW, sh, sw, ph, pw, pb, pr, dh, dw, oph, opw, group;
};
// The stride-1 Conv over the zero-inserted input that equals it (ops_convt.cu).
ConvGeom convt_as_conv(const ConvTGeom& t);
size_t convt_zero_insert_bytes(const ConvTGeom& t); // 0 when both strides are 1
void convt_zero_insert(nb2_device* dev, const ConvTGeom& t, const float* x, float* xz);
// w [C, M/group, KH, KW] -> w2 [M, C/group, KH, KW], transposed per group and flipped.
void convt_flip_weights(nb2_device* dev, const ConvTGeom& t, const float* w, float* w2);

// The layout a Conv over an NCHW input runs in once that input is converted
// to NHWC in front of the contraction (group 1 only): up to 16 channels
// padded to 4, 8 or 16 (each filter tap one to four 16-byte loads); a spatial
// filter over more channels padded to a multiple of 32 and read through TMA
// im2col; otherwise the geometry unchanged (gathered straight from NCHW).
ConvGeom nchw_input_layout(const ConvGeom& g);

// K slices the contraction kernel uses for a problem with `tiles` output
// tiles and `nkb` 32-wide K blocks (1 = no split; >1 adds a reduce launch);
// *kper = K blocks per slice.
int split_k_slices(const nb2_device* dev, int64_t tiles, int nkb, int* kper);
// Kernel launches of one contraction (1, or 2 with split K): M rows, N
// columns per z slice, K, z slices.
int contraction_launches(const nb2_device* dev, int64_t M, int64_t n_per_z, int64_t K, int64_t z);

// Bytes of the packed weight buffer of a Conv: hi and lo planes of
// [M][Kpad] fp32, then (generic layout only) a Kpad-entry int2 tap table.
// Direct convolution on the CUDA cores (conv_direct.cu) for narrow outputs:
// group 1, M <= 32, NCHW in and out, the shared weight tile within 48 KB;
// raw fp32 weights [M][C][KH][KW], fp32 FMAs, the same epilogue.
bool direct_conv_ok(const ConvGeom& g);
void conv_direct(nb2_device* dev, const ConvGeom& g, const float* x, const float* w, float* y, const Epilogue& ep);
size_t conv_packed_bytes(const ConvGeom& g);
void conv_pack(nb2_device* dev, const ConvGeom& g, const float* w, void* packed);
void conv_run(nb2_device* dev, const ConvGeom& g, const float* x, const void* packed, float* y, const Epilogue& ep);

// Dense GEMM: Y[M,N] = op(A)[M,K] * op(B)[K,N]; lda/ldb are the row strides of
// A and B as stored. B is packed per call into `packed` (see gemm_packed_bytes).
// Output placement of a contraction written straight into a permuted
// layout (e.g. a linear layer's [B*T, H*D] result stored as [B, H, T, D]):
// element (z, row, col) goes to
//   (z / z2) * zs1 + (z % z2) * zs2 + (row / r2) * rs1 + (row % r2) * rs2
//   + (col / c2) * cs1 + (col % c2) * cs2,
// with c2 % 16 == 0. Off (on = false) for plain row-major output.
struct OutMap {
    bool on = false;
    int64_t z2 = 1, zs1 = 0, zs2 = 0;
    int64_t r2 = 1, rs1 = 0, rs2 = 0;
    int64_t c2 = 1, cs1 = 0, cs2 = 0;
};

struct GemmGeom {
    int64_t M, N, K;
    int trans_a, trans_b;
    int64_t lda, ldb, ldc;
    int64_t batch = 1;                  // batched MatMul: z slices
    int64_t a_zstride = 0, b_zstride = 0, c_zstride = 0;
    OutMap omap;                        // permuted output (no residual, no split K)
};

size_t gemm_packed_bytes(const GemmGeom& g);
void gemm_pack_b(nb2_device* dev, const GemmGeom& g, const float* b, void* packed);
void gemm_run(nb2_device* dev, const GemmGeom& g, const float* a, const void* packed_b, float* y,
              const Epilogue& ep);

} // namespace nb2
