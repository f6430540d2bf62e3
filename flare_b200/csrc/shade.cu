// shade.cu -- per-hit decode and front-to-back compositing, forward and backward, plus the multi-pass
// drivers.  Replaces the reference kernels
//   Forward_training_CUDA_kernel      (CPyOptiXFLARERenderer_CUDA_Forward_training.cu:497-945)
//   Forward_inference_CUDA_kernel     (CPyOptiXFLARERenderer_CUDA_Forward_inference.cu:501-928)
//   GetMedianDepth_CUDA_kernel        (CPyOptiXFLARERenderer_CUDA_GetMedianDepth.cu:497-878)
//   Backward_CUDA_kernel              (CPyOptiXFLARERenderer_CUDA_Backward.cu:1300-2234)
//   and their *_base twins (constant colour, no decoder)
// and the host pass loops (e.g. Forward_training.cu:949-1132), whose thrust compaction and per-pass
// reduce are replaced by an in-kernel warp-aggregated append to the next pass's ray list.
//
// Decoder on the 5th-generation tensor core.  A CTA of 128 threads owns 128 rays, one per thread; for
// each of the 16 hit slots of a pass the CTA decodes one hit per ray as a 128-row tile:
//   X (128 x 128 f16: LUT 8 | view encoding 24 | descriptor 96) is written to shared memory row by row
//   (each thread its own row), then one elected thread issues tcgen05.mma
//     Y1 = X  W1^T (128x64, K=128)   -> TMEM, epilogue Hardswish -> f16 H1 in shared memory
//     Y2 = H1 W2^T (128x64, K=64)    -> TMEM, epilogue Hardswish -> f16 H2
//     Y3 = H2 W3^T (128x16, K=64)    -> TMEM, each thread reads its own row's 4 outputs
// TMEM lane r of the accumulator is row r, i.e. thread r's hit, so no fragment shuffles are needed.
// The backward recomputes the forward tile, forms delta3 from the compositing gradient and runs the
// chain on the tensor core as well:
//   G2 = d3 W3 (K=16), G1 = d2 W2 (K=64), dX = d1 W1 (K=64; only the LUT and descriptor columns),
// while the weight gradients accumulate in TMEM across all tiles a CTA processes (M=64 accumulators in
// the two half-subpartitions: dW1|db1 in lanes 0-15, dW2|dW3^T|db2|db3 in lanes 16-31 of each warp),
// and are flushed once per CTA.  Backward operands are f16 with a per-call power-of-two gradient scale
// (from max |dL/dI|) so small image gradients do not underflow.
#include <cuda_fp16.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "renderer.cuh"
#include "umma.cuh"

namespace flare {

// ------------------------------------------------------------------------------------------------
// shared-memory layout of the decoder kernels (bytes)
// ------------------------------------------------------------------------------------------------
constexpr int SM_W1 = 0;                  // 64x128 f16, K chunk stride 1024
constexpr int SM_W2 = SM_W1 + 16384;      // 64x64 f16, K chunk stride 1024
constexpr int SM_W3 = SM_W2 + 8192;       // 16x64 f16, K chunk stride 256
constexpr int SM_BIAS = SM_W3 + 2048;     // b1 64, b2 64, b3 16 floats
#ifndef FLARE_FWD_LUT_SMEM
#define FLARE_FWD_LUT_SMEM 0  // 1: the forward stages the LUT in shared memory; 0: reads it through L1 (3 CTAs/SM fit)
#endif
#ifndef FLARE_FWD_CTAS
#define FLARE_FWD_CTAS 3      // resident forward CTAs per SM the grid is sized for
#endif
constexpr int SM_FWD_LUT = SM_BIAS + 1024;                    // 13154 floats
constexpr int SM_FWD_TILE = ((SM_FWD_LUT + (FLARE_FWD_LUT_SMEM ? LUT * 4 : 0) + 1023) / 1024) * 1024;  // 128x128 f16
constexpr int SM_FWD_MISC = SM_FWD_TILE + 32768;
constexpr int SM_FWD_BYTES = SM_FWD_MISC + 64;

constexpr int SM_BWD_X = ((SM_BIAS + 1024 + 1023) / 1024) * 1024;  // 128x128 f16 (X)
constexpr int SM_BWD_D3 = SM_BWD_X + 32768;   // 128x16 f16 (delta3, scaled), followed by >= 14 KB of tiles
constexpr int SM_BWD_ONES = SM_BWD_D3 + 4096; // 128x8 f16 ones column
constexpr int SM_BWD_H1 = SM_BWD_ONES + 2048; // 128x64 f16 (H1, later delta1)
constexpr int SM_BWD_H2 = SM_BWD_H1 + 16384;  // 128x64 f16 (H2, later delta2)
constexpr int SM_BWD_MISC = SM_BWD_H2 + 16384;
constexpr int SM_BWD_BYTES = SM_BWD_MISC + 64;

constexpr int TM_FWD_COLS = 128;
constexpr int TM_BWD_COLS = 256;
constexpr int TM_DW = 128;  // backward: weight-gradient region starts at this column
// backward TMEM map: transients [0,128): Y1 [0,64), Y2 [64,128) kept until delta2 is formed, Y3 / G2 / G1
// at [0,64), dX at [0,112).  Weight gradients [128,256): lanes 0-15 of each warp (half 0) dW1 (64x128);
// lanes 16-31 (half 1) dW2 [0,64), dW3^T hi|lo [64,72), db2 [72], db3 hi|lo rows [80], db1 [88].

// The 6577-cell LUT receives 32 gradient atomics per hit; one table shared by every CTA serialises them
// in L2, so each CTA accumulates into its own copy (L2-resident) and one kernel sums the copies.
constexpr int LUT_PRIV_STRIDE = LUT_PRIV_FLOATS;

// dense weight-gradient accumulator layout in renderer->dw (floats)
constexpr int DW_W1 = 0, DW_B1 = 8192, DW_W2 = 8256, DW_B2 = 12352, DW_W3 = 12416, DW_B3 = 13440;
constexpr int DW_TOTAL = 13456;

// ------------------------------------------------------------------------------------------------
struct SceneP {
    const float *m, *s, *q, *RGBA, *k;
    const uint4 *cond;  // (N, 12) 16-byte chunks of the f16 descriptor
    const float *features;
    const __half *A1, *A2, *A3;
    const float *b1, *b2, *b3;
    const float *override_colors;
    int n;
};

struct PassP {
    const float *O, *v;
    const int *list_in;
    int count;
    const float *hit_t;
    const int *hit_idx;
    float *T, *t_min;
    float *hint;           // per ray: the next pass collects hits at t < hint only (null: unbounded passes)
    float bound_f;         // bound of a pass after a full one: t_K + bound_f (t_K - t_{K/2})
    unsigned char *flags;  // per list slot: the ray stays active (compacted in list order after the pass)
    int *work;             // next unclaimed list slot (zeroed before each launch that claims rays)
    int *status;
    unsigned long long *stats;
    float bg0, bg1, bg2, T_thr;
};

// Bounded later passes.  A pass that filled all K_PASS slots sets the ray's next pass to collect only hits
// at t < hint = t_K + 3 (t_K - t_{K/2}): about three times the depth the second half of its buffer spanned.
// From its first node visit that pass prunes every subtree beyond the bound instead of exploring with an
// unbounded K-th distance until its buffer fills (a restarted packet's lanes start deep inside the scene at
// different t_min).  A bounded pass that found fewer than K_PASS hits has every hit below the bound, so the
// ray continues at t_min = hint with an unbounded pass: the sequence of hits is the same, only the pass
// boundaries move.  (t_K, t_{K/2}: the K-th and (K/2)-th hit of the pass.)
struct PassEnd {
    bool more;        // hits beyond this pass may exist
    float t_min, hint;
};
__device__ __forceinline__ PassEnd pass_end(bool full, float t_K, float t_half, float hint_cur, float bound_f) {
    PassEnd e;
    if (full) {
        e.more = true;
        e.t_min = nextafterf(t_K, INFINITY);
        const float h = __fadd_rn(t_K, __fmul_rn(bound_f, __fsub_rn(t_K, t_half)));
        e.hint = h > e.t_min ? h : INFINITY;
    } else if (hint_cur < INFINITY) {
        e.more = true;
        e.t_min = hint_cur;
        e.hint = INFINITY;
    } else {
        e.more = false;
        e.t_min = INFINITY;
        e.hint = INFINITY;
    }
    return e;
}

struct FwdOut {
    float *bitmap, *dacc, *nacc, *normal, *alpha, *edn, *med;
    const float *surface_normal;
    float reg_a, reg_b;
    const unsigned char *shadow;  // FWD_VIEWER: per hit slot (slot-major like the hit lists), lit = 0
    float shadow_mult;
};

struct BwdIO {
    float *I;
    const float *dL_dI;
    float *dRGB, *dA, *dk, *dm, *ds, *dq, *dcond, *dfeat;
    float *dw;  // dense MLP gradient accumulators (DW_*)
    float *dfeat_priv;  // per-CTA private LUT gradients (pair-major, LUT_PRIV_STRIDE floats per CTA), reduced at the end
    float *pgrad;       // packed per-primitive gradients (PGRAD_FLOATS per primitive), scattered at the end
    const float *dacc;
    float *prefix;
    const float *surface_normal;
    float lambda_depth, reg_a, reg_b, lambda_normal;
    const float *gscale;  // [0] = scale applied to delta3 operands
    int vec4;             // dq is 16-byte aligned: use vector reductions
};

// dst[0..3] += (a, b, c, d): one vector reduction when 16-byte aligned, else four scalar atomics.
__device__ __forceinline__ void red_add4(float *dst, bool vec, float a, float b, float c, float d);

// ------------------------------------------------------------------------------------------------
// per-hit geometry (reference Forward_training.cu:719-783 and Backward.cu:1527-1608)
// ------------------------------------------------------------------------------------------------
struct Geo {
    float sx, sy;            // e^{-s}
    float U[3], V[3], N[3];  // rotation columns (N unnormalised by the same S as U, V)
    float S;                 // 2 / |q|^2
    float q[4];
    float d[3];              // P - m
    float u, w;              // local coordinates
    float kraw, kappa, kinv;
    float r2, pk, r2k, G;    // r^2, (r^2)^(kappa-1), (r^2)^kappa, exp(-r2k / (2 kappa))
};

template <int DK>
struct Dec;
template <>
struct Dec<0> {
    static constexpr int LEVELS = 4, COND = 96, COND_CHUNKS = 12, FEATS = LUT;
};
template <>
struct Dec<1> {
    static constexpr int LEVELS = 8, COND = 32, COND_CHUNKS = 4, FEATS = GRID_FEATS;
};

__device__ __forceinline__ void prefetch_l2(const void *p) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// Pulls the per-primitive rows the next hit slot reads into L2 while the current slot's tiles run.
template <int DK = 0>
__device__ __forceinline__ void prefetch_hit(const SceneP &sc, int idx) {
    if (idx < 0) return;
    prefetch_l2(sc.m + 3 * (size_t)idx);
    prefetch_l2(sc.s + 2 * (size_t)idx);
    prefetch_l2(sc.q + 4 * (size_t)idx);
    prefetch_l2(sc.k + idx);
    prefetch_l2(sc.RGBA + 4 * (size_t)idx);
    if (sc.cond) {  // the 192-byte descriptor row spans two 128-byte lines (the 64-byte one, one)
        const char *c = reinterpret_cast<const char *>(sc.cond + (size_t)idx * Dec<DK>::COND_CHUNKS);
        prefetch_l2(c);
        if (DK == 0) prefetch_l2(c + 128);
    }
}

// A hit's raw primitive parameters, loaded one slot ahead by the forward kernel (load_raw) so that their
// latency hides behind the current slot's tensor-core waits.
struct Raw {
    float2 s;
    float4 q;
    float k;
    float m[3];
    float4 rgba;
};
__device__ __forceinline__ Raw load_raw(const SceneP &sc, int idx) {
    Raw r;
    r.s = __ldg(reinterpret_cast<const float2 *>(sc.s) + idx);
    r.q = __ldg(reinterpret_cast<const float4 *>(sc.q) + idx);
    r.k = __ldg(sc.k + idx);
    const float *m = sc.m + 3 * (size_t)idx;
    r.m[0] = __ldg(m);
    r.m[1] = __ldg(m + 1);
    r.m[2] = __ldg(m + 2);
    r.rgba = __ldg(reinterpret_cast<const float4 *>(sc.RGBA) + idx);
    return r;
}

__device__ __forceinline__ void prefetch_l1(const void *p) {
    asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}

// geometry() on parameters already in registers (same operations, same results).
__device__ __forceinline__ void geometry_raw(const Raw &r, float t, float3 O, float3 v, Geo &g) {
    const float2 s = r.s;
    const float4 q = r.q;
    g.sx = expf(-s.x);
    g.sy = expf(-s.y);
    g.q[0] = q.x; g.q[1] = q.y; g.q[2] = q.z; g.q[3] = q.w;
    float aa = q.x * q.x, bb = q.y * q.y, cc = q.z * q.z, dd = q.w * q.w;
    float S = __fdiv_rn(2.0f, aa + bb + cc + dd);
    g.S = S;
    float bs = q.y * S, cs = q.z * S, ds = q.w * S;
    float ab = q.x * bs, ac = q.x * cs, ad = q.x * ds;
    bb *= S;
    float bc = q.y * cs, bd = q.y * ds;
    cc *= S;
    float cd = q.z * ds;
    dd *= S;
    g.U[0] = 1.0f - cc - dd; g.U[1] = bc + ad; g.U[2] = bd - ac;
    g.V[0] = bc - ad; g.V[1] = 1.0f - bb - dd; g.V[2] = cd + ab;
    g.N[0] = bd + ac; g.N[1] = cd - ab; g.N[2] = 1.0f - bb - cc;
    g.kraw = r.k;
    g.kappa = 1.0f + log1pf(expf(g.kraw));
    g.kinv = 1.0f / g.kappa;
    g.d[0] = __fmaf_rn(v.x, t, O.x) - r.m[0];
    g.d[1] = __fmaf_rn(v.y, t, O.y) - r.m[1];
    g.d[2] = __fmaf_rn(v.z, t, O.z) - r.m[2];
    g.u = g.sx * __fmaf_rn(g.U[0], g.d[0], __fmaf_rn(g.U[1], g.d[1], g.U[2] * g.d[2]));
    g.w = g.sy * __fmaf_rn(g.V[0], g.d[0], __fmaf_rn(g.V[1], g.d[1], g.V[2] * g.d[2]));
    g.r2 = __fmaf_rn(g.u, g.u, g.w * g.w);
    float pk = __powf(g.r2, g.kappa - 1.0f);
    if (isnan(pk)) pk = 0.0f;
    g.pk = pk;
    g.r2k = g.r2 * pk;
    g.G = __expf(-0.5f * g.kinv * g.r2k);
}

__device__ __forceinline__ void geometry(const SceneP &sc, int idx, float t, float3 O, float3 v, Geo &g) {
    float2 s = __ldg(reinterpret_cast<const float2 *>(sc.s) + idx);
    float4 q = __ldg(reinterpret_cast<const float4 *>(sc.q) + idx);
    // accurate exp / division: the LUT interpolation has cell boundaries, so the local coordinates are
    // kept within an ulp or two of the exact value (fast-math intrinsics drift several ulp)
    g.sx = expf(-s.x);
    g.sy = expf(-s.y);
    g.q[0] = q.x; g.q[1] = q.y; g.q[2] = q.z; g.q[3] = q.w;
    float aa = q.x * q.x, bb = q.y * q.y, cc = q.z * q.z, dd = q.w * q.w;
    float S = __fdiv_rn(2.0f, aa + bb + cc + dd);
    g.S = S;
    float bs = q.y * S, cs = q.z * S, ds = q.w * S;
    float ab = q.x * bs, ac = q.x * cs, ad = q.x * ds;
    bb *= S;
    float bc = q.y * cs, bd = q.y * ds;
    cc *= S;
    float cd = q.z * ds;
    dd *= S;
    g.U[0] = 1.0f - cc - dd; g.U[1] = bc + ad; g.U[2] = bd - ac;
    g.V[0] = bc - ad; g.V[1] = 1.0f - bb - dd; g.V[2] = cd + ab;
    g.N[0] = bd + ac; g.N[1] = cd - ab; g.N[2] = 1.0f - bb - cc;
    g.kraw = __ldg(sc.k + idx);
    g.kappa = 1.0f + log1pf(expf(g.kraw));
    g.kinv = 1.0f / g.kappa;
    const float *m = sc.m + 3 * (size_t)idx;
    g.d[0] = __fmaf_rn(v.x, t, O.x) - __ldg(m);
    g.d[1] = __fmaf_rn(v.y, t, O.y) - __ldg(m + 1);
    g.d[2] = __fmaf_rn(v.z, t, O.z) - __ldg(m + 2);
    g.u = g.sx * __fmaf_rn(g.U[0], g.d[0], __fmaf_rn(g.U[1], g.d[1], g.U[2] * g.d[2]));
    g.w = g.sy * __fmaf_rn(g.V[0], g.d[0], __fmaf_rn(g.V[1], g.d[1], g.V[2] * g.d[2]));
    g.r2 = __fmaf_rn(g.u, g.u, g.w * g.w);
    float pk = __powf(g.r2, g.kappa - 1.0f);
    if (isnan(pk)) pk = 0.0f;
    g.pk = pk;
    g.r2k = g.r2 * pk;
    g.G = __expf(-0.5f * g.kinv * g.r2k);
}

__device__ __forceinline__ float hswish(float y) { return (y * fmaxf(fminf(y + 3.0f, 6.0f), 0.0f)) * (1.0f / 6.0f); }
__device__ __forceinline__ float hswish_d(float y) {
    float xu = y + 3.0f, xc = fmaxf(fminf(xu, 6.0f), 0.0f);
    return (xc + ((xu == xc) ? y : 0.0f)) * (1.0f / 6.0f);
}
__device__ __forceinline__ float sigm(float x) { return 1.0f / (1.0f + __expf(-x)); }

// Decoder kinds (flare_scene::decoder).  Both fill the same 128-wide f16 input row and run the same
// 128->64->64->16 tensor-core tiles; they differ in the row's contents, the hidden activation and the
// colour head.
//   0 (FLARE_DECODER_LUT_PE, the reference's compiled decoder, Forward_training.cu:198-373):
//     [LUT 4 levels x 2 | sin/cos view encoding 24 | descriptor 96], Hardswish, colour = relu(y) * RGB.
//   1 (FLARE_DECODER_GRID_SH, the BASELINE config-0 encoder): [dense grid 8 levels x 2 | real spherical
//     harmonics of the view direction, degree 3 (16) | descriptor 32 | zeros 64], ReLU, colour =
//     sigmoid(y) * RGB.  W1 keeps its (64, 128) shape; columns 64..127 meet zero inputs.
template <int DK>
__device__ __forceinline__ float act(float y) {
    return DK ? fmaxf(y, 0.0f) : hswish(y);
}
template <int DK>
__device__ __forceinline__ float act_d(float y) {
    return DK ? (y > 0.0f ? 1.0f : 0.0f) : hswish_d(y);
}

// LUT levels (reference Forward_training.cu:240-263): res {16,25,40,64}, float2 offsets {0,256,881,2481}
__device__ __forceinline__ int lut_res(int l) { return l == 0 ? 16 : (l == 1 ? 25 : (l == 2 ? 40 : 64)); }
__device__ __forceinline__ int lut_off(int l) { return l == 0 ? 0 : (l == 1 ? 256 : (l == 2 ? 881 : 2481)); }

// Dense grid levels of decoder 1: resolution floor(4 * 1.5^l) vertices per side, l = 0..7 (every level
// has fewer than 2^16 vertices, so the multiresolution table addresses them row-major, unhashed), float2
// offsets = running sums of res^2.
__device__ __forceinline__ int grid_res(int l) {
    return l < 4 ? (l == 0 ? 4 : (l == 1 ? 6 : (l == 2 ? 9 : 13))) : (l == 4 ? 20 : (l == 5 ? 30 : (l == 6 ? 45 : 68)));
}
__device__ __forceinline__ int grid_off(int l) {
    return l < 4 ? (l == 0 ? 0 : (l == 1 ? 16 : (l == 2 ? 52 : 133))) : (l == 4 ? 302 : (l == 5 ? 702 : (l == 6 ? 1602 : 3627)));
}

struct LutCell {
    int i00;        // float2 index of the (x0, y0) corner
    int R;
    float fx, fy;
};
template <int DK = 0>
__device__ __forceinline__ LutCell lut_cell(int l, float cu, float cw) {
    LutCell c;
    int R = DK ? grid_res(l) : lut_res(l);
    float xs = __saturatef((cu + 1.0f) * 0.5f), ys = __saturatef((cw + 1.0f) * 0.5f);
    float scale = (float)R - 1.0f;
    float px = xs * scale, py = ys * scale;
    int ix = min(__float2int_rd(px), R - 2), iy = min(__float2int_rd(py), R - 2);
    c.fx = px - (float)ix;
    c.fy = py - (float)iy;
    c.R = R;
    c.i00 = (DK ? grid_off(l) : lut_off(l)) + iy * R + ix;
    return c;
}

// Real spherical harmonics of a unit direction, degrees 0..3 (16 values, the standard real basis with
// the Condon-Shortley phase, as the Instant-NGP / 3DGS view encodings use).
__device__ __forceinline__ void sh_deg3(float x, float y, float z, float out[16]) {
    const float xx = x * x, yy = y * y, zz = z * z;
    out[0] = 0.28209479177387814f;
    out[1] = -0.48860251190291987f * y;
    out[2] = 0.48860251190291987f * z;
    out[3] = -0.48860251190291987f * x;
    out[4] = 1.0925484305920792f * x * y;
    out[5] = -1.0925484305920792f * y * z;
    out[6] = 0.94617469575755997f * zz - 0.31539156525251999f;
    out[7] = -1.0925484305920792f * x * z;
    out[8] = 0.54627421529603959f * (xx - yy);
    out[9] = 0.59004358992664352f * y * (-3.0f * xx + yy);
    out[10] = 2.8906114426405538f * x * y * z;
    out[11] = 0.45704579946446572f * y * (1.0f - 5.0f * zz);
    out[12] = 0.3731763325901154f * z * (5.0f * zz - 3.0f);
    out[13] = 0.45704579946446572f * x * (1.0f - 5.0f * zz);
    out[14] = 1.4453057213202769f * z * (xx - yy);
    out[15] = 0.59004358992664352f * x * (-xx + 3.0f * yy);
}

// Writes one 128-wide f16 decoder input row into a K-major interleaved tile (row r).  Returns the
// LUT values through lut8 for reuse.
template <int DK = 0>
__device__ __forceinline__ void write_x_row(char *tile, int r, const float2 *lut2, const SceneP &sc, int idx,
                                            float cu, float cw, float3 v, bool zero) {
    uint4 *T = reinterpret_cast<uint4 *>(tile);
    if (zero) {
#pragma unroll
        for (int kc = 0; kc < 16; ++kc) T[kc * 128 + r] = make_uint4(0, 0, 0, 0);
        return;
    }
    if constexpr (DK == 1) {
        // Each of the 32 grid / spherical-harmonics inputs x is split into an f16 hi part (chunks 0-3) and
        // the f16 remainder x - hi (chunks 8-11, met by a copy of W1's columns 0..31): the layer-1
        // pre-activations see x to ~22 bits instead of f16's 11, so the sign of a ReLU input near zero --
        // which gates the whole layer-1 gradient -- does not hang on the f16 rounding of x.
        // chunks 0-1 / 8-9: grid levels 0-7 (level l -> elements 2l, 2l+1); one chunk at a time keeps the
        // corner loads in flight to 16 float2
#pragma unroll 1
        for (int hc = 0; hc < 2; ++hc) {
            __half2 h[4], lo[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                LutCell c = lut_cell<1>(4 * hc + q, cu, cw);
                float2 f00 = lut2[c.i00], f10 = lut2[c.i00 + 1], f01 = lut2[c.i00 + c.R], f11 = lut2[c.i00 + c.R + 1];
                float ux = c.fx, vx = 1.0f - ux;
                float r0x = __fmaf_rn(f00.x, vx, f10.x * ux), r0y = __fmaf_rn(f00.y, vx, f10.y * ux);
                float r1x = __fmaf_rn(f01.x, vx, f11.x * ux), r1y = __fmaf_rn(f01.y, vx, f11.y * ux);
                float uy = c.fy, vy = 1.0f - uy;
                const float gx = __fmaf_rn(r0x, vy, r1x * uy), gy = __fmaf_rn(r0y, vy, r1y * uy);
                h[q] = __floats2half2_rn(gx, gy);
                const float2 hf = __half22float2(h[q]);
                lo[q] = __floats2half2_rn(gx - hf.x, gy - hf.y);
            }
            T[hc * 128 + r] = *reinterpret_cast<uint4 *>(h);
            T[(8 + hc) * 128 + r] = *reinterpret_cast<uint4 *>(lo);
        }
        // chunks 2-3 / 10-11: spherical harmonics of v
        float shv[16];
        sh_deg3(v.x, v.y, v.z, shv);
#pragma unroll
        for (int hc = 0; hc < 2; ++hc) {
            __half2 h[4], lo[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float a0 = shv[8 * hc + 2 * q], a1 = shv[8 * hc + 2 * q + 1];
                h[q] = __floats2half2_rn(a0, a1);
                const float2 hf = __half22float2(h[q]);
                lo[q] = __floats2half2_rn(a0 - hf.x, a1 - hf.y);
            }
            T[(2 + hc) * 128 + r] = *reinterpret_cast<uint4 *>(h);
            T[(10 + hc) * 128 + r] = *reinterpret_cast<uint4 *>(lo);
        }
        // chunks 4-7: the 32-wide descriptor row (f16 already); 12-15: zero
        const uint4 *cr = sc.cond + (size_t)idx * 4;
#pragma unroll
        for (int j = 0; j < 4; ++j) T[(4 + j) * 128 + r] = __ldg(cr + j);
#pragma unroll
        for (int kc = 12; kc < 16; ++kc) T[kc * 128 + r] = make_uint4(0, 0, 0, 0);
    } else {
    // chunk 0: LUT (level l -> elements 2l, 2l+1)
    __half2 h[4];
#pragma unroll
    for (int l = 0; l < 4; ++l) {
        LutCell c = lut_cell(l, cu, cw);
        float2 f00 = lut2[c.i00], f10 = lut2[c.i00 + 1], f01 = lut2[c.i00 + c.R], f11 = lut2[c.i00 + c.R + 1];
        float ux = c.fx, vx = 1.0f - ux;
        float r0x = __fmaf_rn(f00.x, vx, f10.x * ux), r0y = __fmaf_rn(f00.y, vx, f10.y * ux);
        float r1x = __fmaf_rn(f01.x, vx, f11.x * ux), r1y = __fmaf_rn(f01.y, vx, f11.y * ux);
        float uy = c.fy, vy = 1.0f - uy;
        h[l] = __floats2half2_rn(__fmaf_rn(r0x, vy, r1x * uy), __fmaf_rn(r0y, vy, r1y * uy));
    }
    T[0 * 128 + r] = *reinterpret_cast<uint4 *>(h);
    // chunks 1..3: view-direction encoding, axis a -> chunk 1+a, octave f -> (sin, cos) at 2f, 2f+1
    float va[3] = {v.x, v.y, v.z};
#pragma unroll
    for (int a = 0; a < 3; ++a) {
        __half2 e[4];
#pragma unroll
        for (int f = 0; f < 4; ++f) {
            float sn, cs;
            __sincosf(3.14159265358979f * (float)(1 << f) * va[a], &sn, &cs);
            e[f] = __floats2half2_rn(sn, cs);
        }
        T[(1 + a) * 128 + r] = *reinterpret_cast<uint4 *>(e);
    }
    // chunks 4..15: the descriptor row, 12 x 16 bytes
    const uint4 *cr = sc.cond + (size_t)idx * 12;
#pragma unroll
    for (int j = 0; j < 12; ++j) T[(4 + j) * 128 + r] = __ldg(cr + j);
    }
}

// Writes 64 f16 values (8 chunks) as row r of a K-major interleaved 128-row tile.
__device__ __forceinline__ void write_row64(char *tile, int r, const float *x) {
    uint4 *T = reinterpret_cast<uint4 *>(tile);
#pragma unroll
    for (int kc = 0; kc < 8; ++kc) {
        __half2 h[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) h[e] = __floats2half2_rn(x[8 * kc + 2 * e], x[8 * kc + 2 * e + 1]);
        T[kc * 128 + r] = *reinterpret_cast<uint4 *>(h);
    }
}

// Writes 16 values as K chunks kc0, kc0+1 of row r of a K-major interleaved 128-row tile.
__device__ __forceinline__ void write_row16(char *tile, int r, int kc0, const float *x) {
    uint4 *T = reinterpret_cast<uint4 *>(tile);
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        __half2 h[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) h[e] = __floats2half2_rn(x[8 * c + 2 * e], x[8 * c + 2 * e + 1]);
        T[(kc0 + c) * 128 + r] = *reinterpret_cast<uint4 *>(h);
    }
}

// As write_row16, split into f16 hi = rn(x) (tile_hi) and lo = rn(x - hi) (tile_lo).
__device__ __forceinline__ void write_row16_split(char *tile_hi, char *tile_lo, int r, int kc0, const float *x) {
    uint4 *H = reinterpret_cast<uint4 *>(tile_hi);
    uint4 *L = reinterpret_cast<uint4 *>(tile_lo);
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        __half2 h[4], l[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float a0 = x[8 * c + 2 * e], a1 = x[8 * c + 2 * e + 1];
            h[e] = __floats2half2_rn(a0, a1);
            const float2 hf = __half22float2(h[e]);
            l[e] = __floats2half2_rn(a0 - hf.x, a1 - hf.y);
        }
        H[(kc0 + c) * 128 + r] = *reinterpret_cast<uint4 *>(h);
        L[(kc0 + c) * 128 + r] = *reinterpret_cast<uint4 *>(l);
    }
}

// Loads the decoder weights, biases (and optionally the LUT) into shared memory.
// grid_lo (decoder 1): W1 columns 0..31 are copied into columns 64..95, which that decoder does not use, so
// the f16 lo parts of its grid and spherical-harmonics inputs (X columns 64..95, see write_x_row) meet the
// same weights as their hi parts.
__device__ void load_decoder(char *smem, const SceneP &sc, bool with_lut, bool dup_w3 = false, bool grid_lo = false) {
    const int tid = threadIdx.x, nt = blockDim.x;
    const uint4 *A1 = reinterpret_cast<const uint4 *>(sc.A1);
    const uint4 *A2 = reinterpret_cast<const uint4 *>(sc.A2);
    const uint4 *A3 = reinterpret_cast<const uint4 *>(sc.A3);
    for (int c = tid; c < 64 * 16; c += nt) {  // W1: row o, chunk kc
        int o = c >> 4, kc = c & 15;
        const int src = (grid_lo && kc >= 8 && kc < 12) ? c - 8 : c;
        *reinterpret_cast<uint4 *>(smem + SM_W1 + kc * 1024 + o * 16) = __ldg(A1 + src);
    }
    for (int c = tid; c < 64 * 8; c += nt) {
        int o = c >> 3, kc = c & 7;
        *reinterpret_cast<uint4 *>(smem + SM_W2 + kc * 1024 + o * 16) = __ldg(A2 + c);
    }
    for (int c = tid; c < 16 * 8; c += nt) {
        int o = c >> 3, kc = c & 7;
        // rows 4..15 of A3 are padding (only outputs 0..3 are used); the backward stores a copy of rows
        // 0..3 in rows 4..7 so a delta3 split into f16 hi (K 0..3) + lo (K 4..7) parts multiplies W3 twice
        int src = (dup_w3 && o >= 4 && o < 8) ? c - 32 : c;
        *reinterpret_cast<uint4 *>(smem + SM_W3 + kc * 256 + o * 16) = __ldg(A3 + src);
    }
    float *bias = reinterpret_cast<float *>(smem + SM_BIAS);
    for (int i = tid; i < 144; i += nt) bias[i] = i < 64 ? __ldg(sc.b1 + i) : (i < 128 ? __ldg(sc.b2 + i - 64) : __ldg(sc.b3 + i - 128));
    if (with_lut) {
        float2 *lut = reinterpret_cast<float2 *>(smem + SM_FWD_LUT);
        const float2 *src = reinterpret_cast<const float2 *>(sc.features);
        for (int i = tid; i < LUT / 2; i += nt) lut[i] = __ldg(src + i);
    }
}

// One elected thread issues the three forward layers; the others wait on the mbarrier.
struct Mma {
    uint32_t tmem;   // accumulator base
    uint32_t parity;
    void *mbar;
    int *abort;
};

__device__ __forceinline__ bool mma_wait(Mma &mm) {
    bool ok = (*(volatile int *)mm.abort == 0) && mbar_wait(mm.mbar, mm.parity);
    mm.parity ^= 1u;
    if (!ok) atomicExch(mm.abort, 1);
    tc_fence_after();
    return ok;
}

// Issue helpers (called by thread 0 after a CTA barrier).
__device__ __forceinline__ void issue_l1(uint32_t d, uint32_t x_addr, uint32_t w1_addr) {
    const uint32_t id = idesc_f16(128, 64);
#pragma unroll
    for (int ks = 0; ks < 8; ++ks)
        mma_f16_ss(d, sdesc(x_addr + ks * 4096, 2048, 128), sdesc(w1_addr + ks * 2048, 1024, 128), id, ks > 0);
}
__device__ __forceinline__ void issue_l2(uint32_t d, uint32_t h_addr, uint32_t w2_addr) {
    const uint32_t id = idesc_f16(128, 64);
#pragma unroll
    for (int ks = 0; ks < 4; ++ks)
        mma_f16_ss(d, sdesc(h_addr + ks * 4096, 2048, 128), sdesc(w2_addr + ks * 2048, 1024, 128), id, ks > 0);
}
__device__ __forceinline__ void issue_l3(uint32_t d, uint32_t h_addr, uint32_t w3_addr) {
    const uint32_t id = idesc_f16(128, 16);
#pragma unroll
    for (int ks = 0; ks < 4; ++ks)
        mma_f16_ss(d, sdesc(h_addr + ks * 4096, 2048, 128), sdesc(w3_addr + ks * 512, 256, 128), id, ks > 0);
}

// Reads 64 accumulator columns [col, col+64) of this thread's TMEM lane.
__device__ __forceinline__ void tmem_row64(uint32_t tmem, int col, float *y) {
    uint32_t lane = (uint32_t)((threadIdx.x & ~31) << 16);
    tmem_ld16(tmem + lane + col, y);
    tmem_ld16(tmem + lane + col + 16, y + 16);
    tmem_ld16(tmem + lane + col + 32, y + 32);
    tmem_ld16(tmem + lane + col + 48, y + 48);
    tmem_wait_ld();
}

// Forward MLP of the tile in `tile` (X already written, fence + barrier done by the caller).
// Leaves h1/h2 in `tile` at the end (h2), returns y[0..3] (+ b3) for this thread's row.
// If keep_d1 is non-null the layer-1 Hardswish derivatives are stored there (fp32).  Layer 2 accumulates
// into TMEM columns [y2col, y2col+64): the backward keeps them there to form delta2 exactly.
// With DK == 1 (ReLU) the derivatives are 0 / 1 and go to the 64-bit mask keep_m1 instead (bit o = z1[o] > 0).
template <int DK = 0>
__device__ __forceinline__ bool mlp_forward_tile(char *smem, char *x_tile, char *h1_tile, char *h2_tile, Mma &mm,
                                                 float *y4, float *keep_d1, int y2col,
                                                 unsigned long long *keep_m1 = nullptr) {
    const float *bias = reinterpret_cast<const float *>(smem + SM_BIAS);
    const int r = threadIdx.x;
    float y[64];
    if (r == 0) {
        tc_fence_after();
        issue_l1(mm.tmem, smem_u32(x_tile), smem_u32(smem + SM_W1));
        mma_commit(mm.mbar);
    }
    bool ok = mma_wait(mm);
    tmem_row64(mm.tmem, 0, y);
#pragma unroll
    for (int o = 0; o < 64; o += 2) {
        const float z0 = y[o] + bias[o], z1 = y[o + 1] + bias[o + 1];
        if (keep_d1) {
            keep_d1[o] = act_d<DK>(z0);
            keep_d1[o + 1] = act_d<DK>(z1);
        }
        if (keep_m1)
            *keep_m1 |= ((unsigned long long)(z0 > 0.0f) << o) | ((unsigned long long)(z1 > 0.0f) << (o + 1));
        y[o] = act<DK>(z0);
        y[o + 1] = act<DK>(z1);
    }
    write_row64(h1_tile, r, y);
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (r == 0) {
        tc_fence_after();
        issue_l2(mm.tmem + y2col, smem_u32(h1_tile), smem_u32(smem + SM_W2));
        mma_commit(mm.mbar);
    }
    ok = mma_wait(mm) && ok;
    tmem_row64(mm.tmem, y2col, y);
#pragma unroll
    for (int o = 0; o < 64; o += 2) {
        const float z0 = y[o] + bias[64 + o], z1 = y[o + 1] + bias[64 + o + 1];
        y[o] = act<DK>(z0);
        y[o + 1] = act<DK>(z1);
    }
    write_row64(h2_tile, r, y);
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (r == 0) {
        tc_fence_after();
        issue_l3(mm.tmem, smem_u32(h2_tile), smem_u32(smem + SM_W3));
        mma_commit(mm.mbar);
    }
    ok = mma_wait(mm) && ok;
    {
        float y16[16];
        uint32_t lane = (uint32_t)((threadIdx.x & ~31) << 16);
        tmem_ld16(mm.tmem + lane, y16);
        tmem_wait_ld();
#pragma unroll
        for (int o = 0; o < 4; ++o) y4[o] = y16[o] + bias[128 + o];
    }
    tc_fence_before();
    return ok;
}

// ================================================================================================
// Forward
// ================================================================================================
template <bool DEC, int MODE, int DK>
__global__ void __launch_bounds__(128) shade_fwd_kernel(SceneP sc, PassP pp, FwdOut fo) {
    extern __shared__ __align__(1024) char smem[];
    __shared__ int s_abort;
    const int tid = threadIdx.x;
    Mma mm{};
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + SM_FWD_MISC + 8);
    if (DEC) {
        if (tid == 0) {
            mbar_init(smem + SM_FWD_MISC, 1);
            fence_mbar_init();
            s_abort = 0;
        }
        if (tid < 32) tmem_alloc(tmem_slot, TM_FWD_COLS);
        load_decoder(smem, sc, FLARE_FWD_LUT_SMEM, false, DK == 1);
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        mm.tmem = *tmem_slot;
        mm.parity = 0;
        mm.mbar = smem + SM_FWD_MISC;
        mm.abort = &s_abort;
    }
    const float2 *lut2 = FLARE_FWD_LUT_SMEM ? reinterpret_cast<const float2 *>(smem + SM_FWD_LUT)
                                            : reinterpret_cast<const float2 *>(sc.features);
    char *tile = smem + SM_FWD_TILE;
    unsigned long long nhits = 0, ntiles = 0;
    const int nchunks = (pp.count + 127) / 128;
    // Chunks of 128 list slots are claimed in list order by whichever CTA is free (decoder path: the grid is
    // the resident CTAs), so CTAs that drew cheap chunks take more instead of idling at the end of the pass.
    __shared__ int s_chunk;
    int chunk = blockIdx.x;
    if (DEC) {
        if (tid == 0) s_chunk = atomicAdd(pp.work, 1);
        __syncthreads();
        chunk = s_chunk;
    }
    for (; chunk < nchunks;) {
        const int slot = chunk * 128 + tid;
        const bool have = slot < pp.count;
        const int ray = have ? pp.list_in[slot] : -1;
        float3 O = make_float3(0, 0, 0), v = make_float3(0, 0, 1);
        float T = 0.0f;
        float rgb[3] = {0, 0, 0}, dacc[4] = {0, 0, 0, 0}, nacc = 0.0f, nrm[3] = {0, 0, 0}, edn = 0.0f;
        float Nm[3] = {0, 0, 0};
        bool nvalid = false;
        float med_t = 0.0f, med_i = 0.0f;
        bool med_set = false;
        if (have) {
            O = make_float3(pp.O[3 * (size_t)ray], pp.O[3 * (size_t)ray + 1], pp.O[3 * (size_t)ray + 2]);
            v = make_float3(pp.v[3 * (size_t)ray], pp.v[3 * (size_t)ray + 1], pp.v[3 * (size_t)ray + 2]);
            T = pp.T[ray];
            if (MODE != FLARE_FWD_MEDIAN)
                for (int c = 0; c < 3; ++c) rgb[c] = fo.bitmap[3 * (size_t)ray + c];
            if (MODE == FLARE_FWD_TRAINING) {
                for (int c = 0; c < 4; ++c) dacc[c] = fo.dacc[4 * (size_t)ray + c];
                nacc = fo.nacc[4 * (size_t)ray];
                for (int c = 0; c < 3; ++c) Nm[c] = fo.surface_normal[3 * (size_t)ray + c];
                nvalid = __fmaf_rn(Nm[0], Nm[0], __fmaf_rn(Nm[1], Nm[1], Nm[2] * Nm[2])) > 0.0f;
            }
            if (MODE == FLARE_FWD_INFERENCE_GEOMETRY) {
                if (fo.normal)
                    for (int c = 0; c < 3; ++c) nrm[c] = fo.normal[3 * (size_t)ray + c];
                if (fo.edn) edn = fo.edn[ray];
            }
        }
        int ind = -1;
        float t_hit = 0.0f;
        // Software pipeline over the hit slots: slot h+1's list entry is read at the top of slot h and its
        // primitive parameters are loaded (and its descriptor row prefetched into L1) before slot h's
        // tensor-core chain, whose waits hide their latency.
        int ind_nx = have ? pp.hit_idx[slot] : -1;
        float t_nx = have ? pp.hit_t[slot] : 0.0f;
        Raw raw_nx{};
        if (ind_nx >= 0) raw_nx = load_raw(sc, ind_nx);
        for (int h = 0; h < K_PASS; ++h) {
            ind = ind_nx;
            t_hit = t_nx;
            const Raw raw = raw_nx;
            ind_nx = (ind >= 0 && h + 1 < K_PASS) ? pp.hit_idx[(size_t)(h + 1) * pp.count + slot] : -1;
            t_nx = ind_nx >= 0 ? pp.hit_t[(size_t)(h + 1) * pp.count + slot] : 0.0f;
            bool valid = ind >= 0 && T >= pp.T_thr;
            if (MODE == FLARE_FWD_MEDIAN) valid = valid && (T > 0.5f);
            const int idc = ind >= 0 ? ind : 0;
            Geo g;
            if (ind >= 0) geometry_raw(raw, t_hit, O, v, g);
            else g = Geo{};
            float y4[4] = {0, 0, 0, 0};
            if (DEC) {
                // this barrier also closes the previous slot: its TMEM reads are done before the next
                // layer-1 MMA is issued, and an abort raised in its waits is seen by every thread here
                const bool any = __syncthreads_or(valid);
                if (s_abort) goto done;
                if (!any) continue;  // uniform: no ray of this CTA needs slot h
                ++ntiles;
                write_x_row<DK>(tile, tid, lut2, sc, idc, g.u * LUT_SCALE, g.w * LUT_SCALE, v, !valid);
                fence_async_smem();
                tc_fence_before();
                __syncthreads();
                if (ind_nx >= 0 && valid) {
                    raw_nx = load_raw(sc, ind_nx);
                    const char *c = reinterpret_cast<const char *>(sc.cond + (size_t)ind_nx * Dec<DK>::COND_CHUNKS);
                    prefetch_l1(c);
                    if (DK == 0) prefetch_l1(c + 128);
                }
                mlp_forward_tile<DK>(smem, tile, tile, tile, mm, y4, nullptr, 0);
            } else if (ind_nx >= 0) {
                raw_nx = load_raw(sc, ind_nx);
            }
            if (!valid) continue;
            {
                const float4 rgba = raw.rgba;
                float sig_y = DEC ? sigm(y4[3]) : 1.0f;
                float opa1 = sigm(rgba.w);
                float alpha = opa1 * g.G * sig_y;
                float o = T * alpha;
                ++nhits;
                if (MODE == FLARE_FWD_MEDIAN) {
                    med_t = t_hit;
                    med_i = __int_as_float(ind);
                    med_set = true;
                    T = T - o;
                    continue;
                }
                float c0 = rgba.x, c1 = rgba.y, c2 = rgba.z;
                if (DEC) {
                    c0 *= DK ? sigm(y4[0]) : fmaxf(y4[0], 0.0f);
                    c1 *= DK ? sigm(y4[1]) : fmaxf(y4[1], 0.0f);
                    c2 *= DK ? sigm(y4[2]) : fmaxf(y4[2], 0.0f);
                }
                if (MODE == FWD_VIEWER && fo.shadow[(size_t)h * pp.count + slot]) {
                    c0 *= fo.shadow_mult;
                    c1 *= fo.shadow_mult;
                    c2 *= fo.shadow_mult;
                }
                if (MODE == FLARE_FWD_PCA && sc.override_colors) {
                    c0 = sc.override_colors[3 * (size_t)ind];
                    c1 = sc.override_colors[3 * (size_t)ind + 1];
                    c2 = sc.override_colors[3 * (size_t)ind + 2];
                }
                rgb[0] = __fmaf_rn(c0, o, rgb[0]);
                rgb[1] = __fmaf_rn(c1, o, rgb[1]);
                rgb[2] = __fmaf_rn(c2, o, rgb[2]);
                float sgn = (__fmaf_rn(g.N[0], v.x, __fmaf_rn(g.N[1], v.y, g.N[2] * v.z)) > 0.0f) ? -1.0f : 1.0f;
                if (MODE == FLARE_FWD_INFERENCE_GEOMETRY) {
                    nrm[0] = __fmaf_rn(sgn * g.N[0], o, nrm[0]);
                    nrm[1] = __fmaf_rn(sgn * g.N[1], o, nrm[1]);
                    nrm[2] = __fmaf_rn(sgn * g.N[2], o, nrm[2]);
                    edn = __fmaf_rn(t_hit, o, edn);
                }
                T = T - o;
                if (MODE == FLARE_FWD_TRAINING) {
                    float tt = __saturatef(__fdividef(fo.reg_a, t_hit) + fo.reg_b);
                    float oacc = dacc[1], toacc = dacc[2];
                    float Ld = o * __fmaf_rn(tt, oacc, -toacc);
                    dacc[0] = __fmaf_rn(4.0f, Ld, dacc[0]);
                    dacc[1] = oacc + o;
                    dacc[2] = __fmaf_rn(tt, o, toacc);
                    dacc[3] = __fmaf_rn(t_hit, o, dacc[3]);
                    float nd = sgn * __fmaf_rn(Nm[0], g.N[0], __fmaf_rn(Nm[1], g.N[1], Nm[2] * g.N[2]));
                    if (nvalid) nacc += o * (1.0f - nd);
                }
            }
        }
        {
            PassEnd pe{ind >= 0, ind >= 0 ? nextafterf(t_hit, INFINITY) : INFINITY, INFINITY};
            if (pp.hint && have)
                pe = pass_end(ind >= 0, t_hit, ind >= 0 ? pp.hit_t[(size_t)(K_PASS / 2 - 1) * pp.count + slot] : 0.0f,
                              pp.hint[ray], pp.bound_f);
            bool active = have && pe.more && T >= pp.T_thr;
            if (MODE == FLARE_FWD_MEDIAN) active = active && (T > 0.5f);
            if (have) {
                if (MODE != FLARE_FWD_MEDIAN) {
                    if (!active && MODE != FWD_VIEWER) {
                        rgb[0] = __fmaf_rn(pp.bg0, T, rgb[0]);
                        rgb[1] = __fmaf_rn(pp.bg1, T, rgb[1]);
                        rgb[2] = __fmaf_rn(pp.bg2, T, rgb[2]);
                    }
                    for (int c = 0; c < 3; ++c) fo.bitmap[3 * (size_t)ray + c] = rgb[c];
                }
                if (MODE == FLARE_FWD_TRAINING) {
                    for (int c = 0; c < 4; ++c) fo.dacc[4 * (size_t)ray + c] = dacc[c];
                    fo.nacc[4 * (size_t)ray] = nacc;
                }
                if (MODE == FLARE_FWD_INFERENCE_GEOMETRY) {
                    if (fo.normal)
                        for (int c = 0; c < 3; ++c) fo.normal[3 * (size_t)ray + c] = nrm[c];
                    if (fo.alpha) fo.alpha[ray] = 1.0f - T;
                    if (fo.edn) fo.edn[ray] = edn;
                }
                if (MODE == FLARE_FWD_MEDIAN && med_set) {
                    fo.med[2 * (size_t)ray] = med_t;
                    fo.med[2 * (size_t)ray + 1] = med_i;
                }
                pp.t_min[ray] = pe.t_min;
                if (pp.hint) pp.hint[ray] = pe.hint;
                pp.T[ray] = T;
            }
            if (have) pp.flags[slot] = active;
        }
        if (DEC) {
            __syncthreads();  // every row has read s_chunk
            if (tid == 0) s_chunk = atomicAdd(pp.work, 1);
            __syncthreads();
            chunk = s_chunk;
        } else {
            chunk += gridDim.x;
        }
    }
done:
    for (int o = 16; o > 0; o >>= 1) nhits += __shfl_xor_sync(0xffffffffu, nhits, o);
    if ((tid & 31) == 0 && nhits) atomicAdd(pp.stats + ST_HITS, nhits);
    if (tid == 0 && ntiles) atomicAdd(pp.stats + ST_TILES, ntiles);
    if (DEC) {
        if (s_abort && tid == 0) atomicOr(pp.status, ERR_MBAR);
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (tid < 32) tmem_dealloc(mm.tmem, TM_FWD_COLS);
    }
}

// ================================================================================================
// Backward
// ================================================================================================
// vector reduction into global memory (sm_90+)
__device__ __forceinline__ void red_add_v4(float *addr, float a, float b, float c, float d) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
                 : "memory");
}

// scalar gradient accumulation into global memory
__device__ __forceinline__ void gadd(float *dst, float v) {
    atomicAdd(dst, v);
}

__device__ __forceinline__ void red_add4(float *dst, bool vec, float a, float b, float c, float d) {
    if (vec) {
        red_add_v4(dst, a, b, c, d);
    } else {
        atomicAdd(dst, a);
        atomicAdd(dst + 1, b);
        atomicAdd(dst + 2, c);
        atomicAdd(dst + 3, d);
    }
}

// Per-primitive gradients of one hit, in the order of the PG_* slots below.
enum { PG_M = 0, PG_S = 3, PG_Q = 5, PG_RGB = 9, PG_A = 12, PG_K = 13, PG_N = 14 };
static_assert(PG_N <= PGRAD_FLOATS, "packed layout");

__device__ __forceinline__ float *pg_dst(const BwdIO &bo, int prim, int j) {
    if (j < PG_S) return bo.dm + 3 * (size_t)prim + j;
    if (j < PG_Q) return bo.ds + 2 * (size_t)prim + (j - PG_S);
    if (j < PG_RGB) return bo.dq + 4 * (size_t)prim + (j - PG_Q);
    if (j < PG_A) return bo.dRGB + 3 * (size_t)prim + (j - PG_RGB);
    if (j == PG_A) return bo.dA + prim;
    return bo.dk + prim;
}

// Geometry gradients (dm, ds, dq) from dL/du, dL/dw and dL/dt (restates Backward.cu:1587-1608, 2033-2216).
__device__ __forceinline__ void geom_grads(const Geo &g, float3 v, float gu, float gw, float dLdt_depth, float ow,
                                           float sgn, bool nvalid, const float Nm[3], float lambda_normal,
                                           float pg[PG_N]) {
            // ---- primitive geometry gradients from dL/du, dL/dw and dL/dt (depth) ----
            float ndv = __fmaf_rn(g.N[0], v.x, __fmaf_rn(g.N[1], v.y, g.N[2] * v.z));
            float inv_ndv = 1.0f / ndv;
            float Uv = __fmaf_rn(g.U[0], v.x, __fmaf_rn(g.U[1], v.y, g.U[2] * v.z));
            float Vv = __fmaf_rn(g.V[0], v.x, __fmaf_rn(g.V[1], v.y, g.V[2] * v.z));
            // total dL/dt through u, w (P = O + t v) and the depth regulariser
            float dLdt = __fmaf_rn(gu * g.sx, Uv, __fmaf_rn(gw * g.sy, Vv, dLdt_depth));
            float kt = dLdt * inv_ndv;
            // dL/dm = dL/dt N/(N.v) - (gu e^-sx U + gw e^-sy V)
            float su = gu * g.sx, sw = gw * g.sy;
            pg[PG_M] = kt * g.N[0] - (su * g.U[0] + sw * g.V[0]);
            pg[PG_M + 1] = kt * g.N[1] - (su * g.U[1] + sw * g.V[1]);
            pg[PG_M + 2] = kt * g.N[2] - (su * g.U[2] + sw * g.V[2]);
            // dL/ds = -u dL/du (u = e^-s U.(P - m))
            pg[PG_S] = -g.u * gu;
            pg[PG_S + 1] = -g.w * gw;
            // dL/dR for R = [U V N]: G_U = gu e^-sx (P-m), G_V = gw e^-sy (P-m),
            // G_N = -dL/dt (P-m)/(N.v) - lambda_n o sgn N_target (the normal regulariser's opacity is held)
            float ln = nvalid ? lambda_normal * (-ow * sgn) : 0.0f;
            const float a = g.q[0], b = g.q[1], c = g.q[2], d = g.q[3], S = g.S;
            // The reference forms the depth regulariser's share of dL/dq from a dt/dq that lacks the factor
            // S = 2/|q|^2 (Backward.cu:2096-2110, Backward_base.cu:496-510: dt_dq is built from (dN/dq) / S
            // and, unlike du_dq and dv_dq, never scaled by S), so that share is (exact share) / S; it is
            // reproduced here.  dm and the other shares of dq are exact.
            const float kq = __fmaf_rn(dLdt_depth * inv_ndv, __fdiv_rn(1.0f, S) - 1.0f, kt);
            float Gm[3][3];
#pragma unroll
            for (int i = 0; i < 3; ++i) {
                Gm[i][0] = su * g.d[i];
                Gm[i][1] = sw * g.d[i];
                Gm[i][2] = -kq * g.d[i] + ln * Nm[i];
            }
            // R = I + S M(q) with S = 2/|q|^2; dR/dq_k = S (dM/dq_k - S q_k M)
            float GM = Gm[0][0] * (-(c * c + d * d)) + Gm[0][1] * (b * c - a * d) + Gm[0][2] * (b * d + a * c) +
                       Gm[1][0] * (b * c + a * d) + Gm[1][1] * (-(b * b + d * d)) + Gm[1][2] * (c * d - a * b) +
                       Gm[2][0] * (b * d - a * c) + Gm[2][1] * (c * d + a * b) + Gm[2][2] * (-(b * b + c * c));
            float dMa = -d * Gm[0][1] + c * Gm[0][2] + d * Gm[1][0] - b * Gm[1][2] - c * Gm[2][0] + b * Gm[2][1];
            float dMb = c * Gm[0][1] + d * Gm[0][2] + c * Gm[1][0] - 2.0f * b * Gm[1][1] - a * Gm[1][2] +
                        d * Gm[2][0] + a * Gm[2][1] - 2.0f * b * Gm[2][2];
            float dMc = -2.0f * c * Gm[0][0] + b * Gm[0][1] + a * Gm[0][2] + b * Gm[1][0] + d * Gm[1][2] -
                        a * Gm[2][0] + d * Gm[2][1] - 2.0f * c * Gm[2][2];
            float dMd = -2.0f * d * Gm[0][0] - a * Gm[0][1] + b * Gm[0][2] + a * Gm[1][0] - 2.0f * d * Gm[1][1] +
                        c * Gm[1][2] + b * Gm[2][0] + c * Gm[2][1];
            pg[PG_Q] = S * (dMa - S * a * GM);
            pg[PG_Q + 1] = S * (dMb - S * b * GM);
            pg[PG_Q + 2] = S * (dMc - S * c * GM);
            pg[PG_Q + 3] = S * (dMd - S * d * GM);
}

// One hit's per-primitive gradients straight into the caller's arrays (decoder-free path).
__device__ __forceinline__ void flush_prim_direct(const BwdIO &bo, int prim, const float pg[PG_N]) {
#pragma unroll
    for (int j = 0; j < PG_N; ++j)
        if (j < PG_Q || j >= PG_RGB) gadd(pg_dst(bo, prim, j), pg[j]);
    red_add4(bo.dq + 4 * (size_t)prim, bo.vec4, pg[PG_Q], pg[PG_Q + 1], pg[PG_Q + 2], pg[PG_Q + 3]);
}

// Asynchronous bulk reduction of `bytes` (a multiple of 16, both addresses 16-byte aligned) from shared
// to global memory: the copy engine performs the adds, so one instruction replaces a row of per-lane
// vector reductions.  The issuing thread waits (wait_bulk_read) before the source is overwritten.
__device__ __forceinline__ void bulk_red_add_f32(float *gdst, const float *ssrc, uint32_t bytes) {
    asm volatile("cp.reduce.async.bulk.global.shared::cta.bulk_group.add.f32 [%0], [%1], %2;" ::"l"(gdst),
                 "r"(smem_u32(ssrc)), "r"(bytes)
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void wait_bulk_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void wait_bulk_done() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Per-lane staging rows: the PGRAD_FLOATS packed primitive gradients then the 64 layer-1 deltas
// (row stride an odd number of 16-byte chunks so the lanes' vector stores hit distinct banks); warps 0-1
// use the X tile, 2-3 the H1-H2 tiles, which are free between the last tensor-core stage of a slot and the
// next slot's X row.
constexpr int DC_ROW = 84;
static_assert(DC_ROW >= PROW_FLOATS && (DC_ROW / 4) % 2 == 1, "staging row");
static_assert(2 * 32 * DC_ROW * 4 <= 32768, "two warps' rows fit the X tile and the H1-H2 tiles");

template <bool DEC, int DK>
__global__ void __launch_bounds__(128) shade_bwd_kernel(SceneP sc, PassP pp, BwdIO bo) {
    extern __shared__ __align__(1024) char smem[];
    __shared__ int s_abort;
    __shared__ int s_first;
    const int tid = threadIdx.x;
    Mma mm{};
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + SM_BWD_MISC + 8);
    void *mbar2 = smem + SM_BWD_MISC + 16;  // completion of a slot's layer-1 weight-gradient MMAs
    uint32_t par2 = 0;
    float gscale = 1.0f, ginv = 1.0f;
    if (DEC) {
        if (tid == 0) {
            mbar_init(smem + SM_BWD_MISC, 1);
            mbar_init(smem + SM_BWD_MISC + 16, 1);  // second barrier: the layer-1 weight-gradient MMAs
            fence_mbar_init();
            s_abort = 0;
            s_first = 1;
        }
        if (tid < 32) tmem_alloc(tmem_slot, TM_BWD_COLS);
        load_decoder(smem, sc, false, true, DK == 1);
        {   // ones column tile (128 rows x 8, element 0 = 1)
            uint4 *ones = reinterpret_cast<uint4 *>(smem + SM_BWD_ONES);
            __half2 h[4] = {__floats2half2_rn(1.0f, 0.0f), __floats2half2_rn(0.0f, 0.0f), __floats2half2_rn(0.0f, 0.0f),
                            __floats2half2_rn(0.0f, 0.0f)};
            ones[tid] = *reinterpret_cast<uint4 *>(h);
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        mm.tmem = *tmem_slot;
        mm.parity = 0;
        mm.mbar = smem + SM_BWD_MISC;
        mm.abort = &s_abort;
        gscale = bo.gscale[0];
        ginv = 1.0f / gscale;
    }
    const float2 *lut2 = reinterpret_cast<const float2 *>(sc.features);
    char *xt = smem + SM_BWD_X, *d3t = smem + SM_BWD_D3, *h1t = smem + SM_BWD_H1, *h2t = smem + SM_BWD_H2;
    // Each row (thread) works through rays of the pass list, one hit slot per iteration; when its ray
    // finishes the pass (a slot that no longer composites, or all K_PASS slots done) the row claims the
    // next ray, so the tiles stay full instead of idling until the tile's slowest ray is done.
    int slot = -1, ray = 0, h = 0;
    bool have = false, exhausted = false;
    float3 O = make_float3(0, 0, 0), v = make_float3(0, 0, 1);
    float T = 0.0f;
    float dLdI[3] = {0, 0, 0}, run[3] = {0, 0, 0};  // run = -(colour from this hit onwards, incl. bg)
    float D[4] = {0, 0, 0, 0}, P[4] = {0, 0, 0, 0};
    float Nm[3] = {0, 0, 0};
    bool nvalid = false;
    int ind = -1, ind_next = -1;
    float t_hit = 0.0f, t_next = 0.0f;
    Raw raw_next{};
    bool raw_ok = false;  // raw_next / t_next hold this row's next slot
    unsigned long long ntiles = 0;
    bool bulk_pending = false;  // this thread's last bulk reduction may still be reading its staging row
    // Each warp reserves list slots 32 at a time (one atomic), reads their ray ids and pulls the rays'
    // state and first hit into L2 when it reserves them, and reserves the next 32 once half are used: a
    // row that claims a ray then waits for one L2 round trip, not for an atomic, the id and the state in
    // turn (a claim stalls the whole tile at the next barrier, and some row of a tile claims most slots).
    int res_base = -1, res_used = 32, nx_base = -1;  // warp-uniform
    int res_id = -1, nx_id = -1;                      // per lane: ray id of slot base + lane (-1: past the list)
    auto fetch_reserve = [&](int &b, int &id) {
        int x = 0;
        if ((tid & 31) == 0) x = atomicAdd(pp.work, 32);
        b = __shfl_sync(0xffffffffu, x, 0);
        const int s_ = b + (tid & 31);
        id = s_ < pp.count ? pp.list_in[s_] : -1;
        if (id >= 0) {
            prefetch_l2(pp.O + 3 * (size_t)id);
            prefetch_l2(pp.v + 3 * (size_t)id);
            prefetch_l2(pp.T + id);
            prefetch_l2(bo.dL_dI + 3 * (size_t)id);
            prefetch_l2(bo.I + 3 * (size_t)id);
            prefetch_l2(bo.dacc + 4 * (size_t)id);
            prefetch_l2(bo.prefix + 4 * (size_t)id);
            prefetch_l2(bo.surface_normal + 3 * (size_t)id);
            prefetch_l2(pp.hit_idx + s_);
            prefetch_l2(pp.hit_t + s_);
        }
    };
    while (true) {
        {   // rows without a ray claim the next ones from the warp's reserve of list slots
            const bool need = !have && !exhausted;
            const unsigned nm = __ballot_sync(0xffffffffu, need);
            const int ln = tid & 31;
            if (nm) {
                const int k = __popc(nm);
                // the reserve runs out with this claim: the next one must be there before the swap below
                if (res_used + k >= 32 && nx_base < 0) fetch_reserve(nx_base, nx_id);
                const int e = res_used + __popc(nm & ((1u << ln) - 1u));
                const int id_r = __shfl_sync(0xffffffffu, res_id, e & 31);
                const int id_n = __shfl_sync(0xffffffffu, nx_id, e & 31);
                const int s_ = e < 32 ? res_base + e : nx_base + e - 32;
                const int rid = e < 32 ? id_r : id_n;
                res_used += k;
                if (res_used >= 32) {
                    res_base = nx_base;
                    res_id = nx_id;
                    res_used -= 32;
                    nx_base = -1;
                }
                if (need) {
                    if (s_ < pp.count && s_ >= 0 && rid >= 0) {
                        slot = s_;
                        have = true;
                        h = 0;
                        ray = rid;
                        O = make_float3(pp.O[3 * (size_t)ray], pp.O[3 * (size_t)ray + 1], pp.O[3 * (size_t)ray + 2]);
                        v = make_float3(pp.v[3 * (size_t)ray], pp.v[3 * (size_t)ray + 1], pp.v[3 * (size_t)ray + 2]);
                        T = pp.T[ray];
                        for (int c = 0; c < 3; ++c) {
                            dLdI[c] = bo.dL_dI[3 * (size_t)ray + c];
                            run[c] = -bo.I[3 * (size_t)ray + c];
                        }
                        for (int c = 0; c < 4; ++c) {
                            D[c] = bo.dacc[4 * (size_t)ray + c];
                            P[c] = bo.prefix[4 * (size_t)ray + c];
                        }
                        for (int c = 0; c < 3; ++c) Nm[c] = bo.surface_normal[3 * (size_t)ray + c];
                        nvalid = __fmaf_rn(Nm[0], Nm[0], __fmaf_rn(Nm[1], Nm[1], Nm[2] * Nm[2])) > 0.0f;
                        ind_next = pp.hit_idx[slot];
                    } else {
                        exhausted = true;
                    }
                }
            }
            if (nx_base < 0 && res_used >= 16) fetch_reserve(nx_base, nx_id);  // the next 32 slots, ahead
        }
        {
            ind = have ? ind_next : -1;
            // this slot's parameters: loaded during the previous slot when the row kept its ray (the same
            // software pipeline as the forward), else now
            t_hit = have ? (raw_ok ? t_next : pp.hit_t[(size_t)h * pp.count + slot]) : 0.0f;
            const Raw raw = (raw_ok || ind < 0) ? raw_next : load_raw(sc, ind);
            ind_next = (have && ind >= 0 && h + 1 < K_PASS) ? pp.hit_idx[(size_t)(h + 1) * pp.count + slot] : -1;
            raw_ok = false;
            const bool valid = ind >= 0 && T >= pp.T_thr;
            const int idc = ind >= 0 ? ind : 0;
            Geo g;
            if (ind >= 0) geometry_raw(raw, t_hit, O, v, g);
            else g = Geo{};
            const float cu = g.u * LUT_SCALE, cw = g.w * LUT_SCALE;
            float y4[4] = {0, 0, 0, 0};
            // layer-1 activation derivatives: fp32 for the Hardswish decoder (then the layer-1 deltas, kept for
            // the per-primitive row); decoder 1's ReLU needs only a bit each, and its deltas are re-read from
            // TMEM, where G1 stays because that decoder's dX goes to columns 64..79
            constexpr int HD1 = DK == 1 ? 1 : 64;
            constexpr uint32_t DXCOL = DK == 1 ? 64u : 0u;  // TMEM column of dX (y2's, free by then)
            float hd1[HD1];
            unsigned long long m1 = 0ull;
            float pg[PG_N];  // this hit's per-primitive gradients (layout PG_*)
#pragma unroll
            for (int e = 0; e < PG_N; ++e) pg[e] = 0.0f;
            // The slot's first barrier.  It also closes the previous slot: that slot's staging rows have
            // been read by its bulk reductions (the issuing threads waited) before the X and H1 tiles are
            // written again, and an abort raised in its waits is seen by every thread here.  A valid row
            // has a ray, so whether any row still has one is asked only when no row composites.
            if (DEC && bulk_pending) {  // the staging rows are overwritten after this barrier
                wait_bulk_read();
                bulk_pending = false;
            }
            const bool any_valid = DEC ? __syncthreads_or(valid) : false;  // uniform
            if (DEC && s_abort) goto done;
            if (!any_valid && !__syncthreads_or(have)) break;
            if (any_valid && tid == 0) ++ntiles;
            if (DEC && any_valid) {
                write_x_row<DK>(xt, tid, lut2, sc, idc, cu, cw, v, !valid);
                fence_async_smem();
                tc_fence_before();
                __syncthreads();
                if (valid && ind_next >= 0) {  // the next slot of this ray: its parameters now, its row into L2
                    raw_next = load_raw(sc, ind_next);
                    t_next = pp.hit_t[(size_t)(h + 1) * pp.count + slot];
                    raw_ok = true;
                    const char *c = reinterpret_cast<const char *>(sc.cond + (size_t)ind_next * Dec<DK>::COND_CHUNKS);
                    prefetch_l2(c);
                    if (DK == 0) prefetch_l2(c + 128);
                }
                mlp_forward_tile<DK>(smem, xt, h1t, h2t, mm, y4, DK == 1 ? nullptr : hd1, 64, DK == 1 ? &m1 : nullptr);
            }
            // ---- compositing gradient (restates Backward.cu:1700-1900) ----
            float gu = 0.0f, gw = 0.0f, dLdt_depth = 0.0f, ow = 0.0f, sgn = 1.0f;
            float d3[4] = {0, 0, 0, 0};
            if (valid) {
                const float4 rgba = raw.rgba;
                float z3[3] = {1.0f, 1.0f, 1.0f}, sig_y = 1.0f, dz3[4] = {1.0f, 1.0f, 1.0f, 0.0f};
                if (DEC) {
#pragma unroll
                    for (int c = 0; c < 3; ++c) {
                        if (DK) {
                            z3[c] = sigm(y4[c]);
                            dz3[c] = z3[c] * (1.0f - z3[c]);
                        } else {
                            z3[c] = fmaxf(y4[c], 0.0f);
                            dz3[c] = y4[c] >= 0.0f ? 1.0f : 0.0f;
                        }
                    }
                    sig_y = sigm(y4[3]);
                    dz3[3] = sig_y * (1.0f - sig_y);
                }
                const float opa1 = sigm(rgba.w);
                const float aG = opa1 * g.G;     // sigma(A) G
                const float alpha = aG * sig_y;  // opacity of this hit
                const float T_prev = T;
                float a_eff = alpha;
                T = T - T * alpha;
                float tu = __fdividef(bo.reg_a, t_hit) + bo.reg_b;
                float tt = __saturatef(tu);
                float o = T_prev * alpha;
                float oacc = P[1], toacc = P[2];
                float dLdo = 2.0f * (__fmaf_rn(tt, __fmaf_rn(2.0f, oacc, -D[1]), -2.0f * toacc) + D[2]);
                float dLdt = 2.0f * o * __fmaf_rn(2.0f, oacc, o - D[1]);
                dLdt *= __fdividef(-bo.reg_a, t_hit * t_hit);
                if (tt != tu) dLdt = 0.0f;
                sgn = (__fmaf_rn(g.N[0], v.x, __fmaf_rn(g.N[1], v.y, g.N[2] * v.z)) > 0.0f) ? -1.0f : 1.0f;
                float nd = sgn * __fmaf_rn(Nm[0], g.N[0], __fmaf_rn(Nm[1], g.N[1], Nm[2] * g.N[2]));
                float dLn_do = nvalid ? 1.0f - nd : 0.0f;
                P[0] = __fmaf_rn(o, dLdo, P[0]);
                P[1] = oacc + o;
                P[2] = __fmaf_rn(tt, o, toacc);
                P[3] = __fmaf_rn(o, dLn_do, P[3]);
                float dLdalpha = (T >= pp.T_thr) ? __fdividef(P[0] - D[0], 1.0f - alpha) : 0.0f;
                dLdalpha = bo.lambda_depth * __fmaf_rn(dLdo, T_prev, dLdalpha);
                dLdt_depth = dLdt * bo.lambda_depth;
                if (T < pp.T_thr) {
                    run[0] = -T_prev * pp.bg0;
                    run[1] = -T_prev * pp.bg1;
                    run[2] = -T_prev * pp.bg2;
                    a_eff = 0.0f;
                }
                float cc0 = z3[0] * rgba.x, cc1 = z3[1] * rgba.y, cc2 = z3[2] * rgba.z;
                float partial = __fdividef(
                    __fmaf_rn(dLdI[0], __fmaf_rn(cc0, T_prev, run[0]),
                              __fmaf_rn(dLdI[1], __fmaf_rn(cc1, T_prev, run[1]), dLdI[2] * __fmaf_rn(cc2, T_prev, run[2]))),
                    1.0f - a_eff);
                float gsum = partial + dLdalpha;  // dL/d(alpha) of this hit
                float w_eff = a_eff * T_prev;
                float dRGB0 = z3[0] * w_eff, dRGB1 = z3[1] * w_eff, dRGB2 = z3[2] * w_eff;
                run[0] = __fmaf_rn(dRGB0, rgba.x, run[0]);
                run[1] = __fmaf_rn(dRGB1, rgba.y, run[1]);
                run[2] = __fmaf_rn(dRGB2, rgba.z, run[2]);
                // kappa = 1 + softplus(k): dG/dkappa (Backward.cu:1882-1894)
                float dk = alpha * gsum * 0.5f * g.r2k * sigm(g.kraw) * g.kinv * (g.kinv - __logf(g.r2));
                if (isnan(dk)) dk = 0.0f;
                pg[PG_RGB] = dRGB0 * dLdI[0];
                pg[PG_RGB + 1] = dRGB1 * dLdI[1];
                pg[PG_RGB + 2] = dRGB2 * dLdI[2];
                pg[PG_A] = alpha * (1.0f - opa1) * gsum;
                pg[PG_K] = dk;
                // delta3: gradients of the layer-3 pre-activations
                d3[0] = dLdI[0] * rgba.x * alpha * T_prev * dz3[0];
                d3[1] = dLdI[1] * rgba.y * alpha * T_prev * dz3[1];
                d3[2] = dLdI[2] * rgba.z * alpha * T_prev * dz3[2];
                d3[3] = aG * gsum * dz3[3];
                // opacity path of dL/du, dL/dw: d alpha/du = -alpha (r^2)^(kappa-1) u
                float apk = alpha * gsum * g.pk;
                gu = -apk * g.u;
                gw = -apk * g.w;
                ow = o;
            }
            // ---- decoder backward on the tensor core ----
            if (DEC && any_valid) {
                {   // delta3 tile row, scaled into the f16 range and split into hi (columns 0..3) and
                    // lo = delta3 - hi (columns 4..7); zero for rows that do not contribute
                    uint4 *T3 = reinterpret_cast<uint4 *>(d3t);
                    __half2 hh[4];
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const float a0 = d3[2 * e] * gscale, a1 = d3[2 * e + 1] * gscale;
                        hh[e] = __floats2half2_rn(a0, a1);
                        const float2 hf = __half22float2(hh[e]);
                        hh[2 + e] = __floats2half2_rn(a0 - hf.x, a1 - hf.y);
                    }
                    T3[tid] = *reinterpret_cast<uint4 *>(hh);
                    T3[128 + tid] = make_uint4(0, 0, 0, 0);
                }
                fence_async_smem();
                tc_fence_before();
                __syncthreads();
                if (s_abort) goto done;  // raised in the forward tile's waits
                const uint32_t acc0 = s_first ? 0u : 1u;
                const uint32_t dwreg = mm.tmem + TM_DW;
                const uint32_t half1 = 16u << 16;
                if (tid == 0) {
                    tc_fence_after();
                    // G2 = d3 W3 : M=128, N=64 (h2 features), K=16; B = W3 read MN-major
                    mma_f16_ss(mm.tmem, sdesc(smem_u32(d3t), 2048, 128), sdesc(smem_u32(smem + SM_W3), 128, 256),
                               idesc_f16(128, 64, 0, 1), 0);
                    // dW3^T += H2^T d3 : M=64 (h2 features), N=8, K=128 hits; both operands MN-major
                    for (int ks = 0; ks < 8; ++ks)
                        mma_f16_ss(dwreg + half1 + 64, sdesc(smem_u32(h2t) + ks * 256, 128, 2048),
                                   sdesc(smem_u32(d3t) + ks * 256, 128, 2048), idesc_f16(64, 8, 1, 1),
                                   (ks > 0) | acc0);
                    // db3 += d3^T 1 : M=64 (rows >= 16 are not used), N=8
                    for (int ks = 0; ks < 8; ++ks)
                        mma_f16_ss(dwreg + half1 + 80, sdesc(smem_u32(d3t) + ks * 256, 128, 2048),
                                   sdesc(smem_u32(smem + SM_BWD_ONES) + ks * 256, 128, 2048), idesc_f16(64, 8, 1, 1),
                                   (ks > 0) | acc0);
                    mma_commit(mm.mbar);
                }
                mma_wait(mm);
                const uint32_t lane = (uint32_t)((threadIdx.x & ~31) << 16);
                {   // delta2 = G2 * hswish'(y2 + b2), y2 re-read in fp32 from TMEM -> H2 tile (free: dW3 done)
                    const float *b2s = reinterpret_cast<const float *>(smem + SM_BIAS) + 64;
#pragma unroll
                    for (int cb = 0; cb < 4; ++cb) {
                        float gv[16], yv[16];
                        tmem_ld16(mm.tmem + lane + 16 * cb, gv);
                        tmem_ld16(mm.tmem + lane + 64 + 16 * cb, yv);
                        tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 16; ++e) gv[e] *= act_d<DK>(yv[e] + b2s[16 * cb + e]);
                        write_row16(h2t, tid, 2 * cb, gv);
                    }
                }
                fence_async_smem();
                tc_fence_before();
                __syncthreads();
                if (tid == 0) {
                    tc_fence_after();
                    // G1 = d2 W2 : M=128, N=64 (h1 features), K=64
                    for (int ks = 0; ks < 4; ++ks)
                        mma_f16_ss(mm.tmem, sdesc(smem_u32(h2t) + ks * 4096, 2048, 128),
                                   sdesc(smem_u32(smem + SM_W2) + ks * 256, 128, 1024), idesc_f16(128, 64, 0, 1),
                                   ks > 0);
                    // dW2 += d2^T H1 : M=64 (out), N=64 (h1 features), K=128 hits
                    for (int ks = 0; ks < 8; ++ks)
                        mma_f16_ss(dwreg + half1, sdesc(smem_u32(h2t) + ks * 256, 128, 2048),
                                   sdesc(smem_u32(h1t) + ks * 256, 128, 2048), idesc_f16(64, 64, 1, 1),
                                   (ks > 0) | acc0);
                    // db2 += d2^T 1
                    for (int ks = 0; ks < 8; ++ks)
                        mma_f16_ss(dwreg + half1 + 72, sdesc(smem_u32(h2t) + ks * 256, 128, 2048),
                                   sdesc(smem_u32(smem + SM_BWD_ONES) + ks * 256, 128, 2048), idesc_f16(64, 8, 1, 1),
                                   (ks > 0) | acc0);
                    mma_commit(mm.mbar);
                }
                mma_wait(mm);
                // delta1 = G1 * hswish'(y1): hi -> H1 tile, lo -> H2 tile (both free now)
#pragma unroll
                for (int cb = 0; cb < 4; ++cb) {
                    float gv[16];
                    tmem_ld16(mm.tmem + lane + 16 * cb, gv);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        if constexpr (DK == 1) {
                            gv[e] = ((m1 >> (16 * cb + e)) & 1ull) ? gv[e] : 0.0f;
                        } else {
                            gv[e] *= hd1[16 * cb + e];
                            hd1[16 * cb + e] = gv[e];  // delta1, kept for the per-primitive row
                        }
                    }
                    write_row16_split(h1t, h2t, tid, 2 * cb, gv);
                }
                fence_async_smem();
                tc_fence_before();
                __syncthreads();
                if (tid == 0) {
                    tc_fence_after();
                    // dX[:, 0:16) = d1 W1[:, 0:16) (hi and lo parts of d1).  The descriptor columns of dX
                    // are not formed per hit: dX[:, 32:128) = d1 W1[:, 32:128) is linear in d1, so each
                    // primitive's sum of d1 is reduced instead and multiplied by W1 once per primitive.
                    for (int ks = 0; ks < 4; ++ks)
                        mma_f16_ss(mm.tmem + DXCOL, sdesc(smem_u32(h1t) + ks * 4096, 2048, 128),
                                   sdesc(smem_u32(smem + SM_W1) + ks * 256, 128, 1024), idesc_f16(128, 16, 0, 1),
                                   ks > 0);
                    for (int ks = 0; ks < 4; ++ks)
                        mma_f16_ss(mm.tmem + DXCOL, sdesc(smem_u32(h2t) + ks * 4096, 2048, 128),
                                   sdesc(smem_u32(smem + SM_W1) + ks * 256, 128, 1024), idesc_f16(128, 16, 0, 1), 1);
                    // dX is all the rest of the slot waits for: a barrier of its own, so the LUT and geometry
                    // gradients start while the weight-gradient MMAs below still run (they only read the
                    // tiles, which nothing writes before the second barrier is waited for)
                    mma_commit(mm.mbar);
                    // dW1 += d1^T X : M=64, N=128, K=128 hits (hi and lo parts of d1)
                    for (int ks = 0; ks < 8; ++ks)
                        mma_f16_ss(dwreg, sdesc(smem_u32(h1t) + ks * 256, 128, 2048),
                                   sdesc(smem_u32(xt) + ks * 256, 128, 2048), idesc_f16(64, 128, 1, 1),
                                   (ks > 0) | acc0);
                    for (int ks = 0; ks < 8; ++ks)
                        mma_f16_ss(dwreg, sdesc(smem_u32(h2t) + ks * 256, 128, 2048),
                                   sdesc(smem_u32(xt) + ks * 256, 128, 2048), idesc_f16(64, 128, 1, 1), 1);
                    // db1 += d1^T 1
                    for (int ks = 0; ks < 8; ++ks)
                        mma_f16_ss(dwreg + half1 + 88, sdesc(smem_u32(h1t) + ks * 256, 128, 2048),
                                   sdesc(smem_u32(smem + SM_BWD_ONES) + ks * 256, 128, 2048), idesc_f16(64, 8, 1, 1),
                                   (ks > 0) | acc0);
                    for (int ks = 0; ks < 8; ++ks)
                        mma_f16_ss(dwreg + half1 + 88, sdesc(smem_u32(h2t) + ks * 256, 128, 2048),
                                   sdesc(smem_u32(smem + SM_BWD_ONES) + ks * 256, 128, 2048), idesc_f16(64, 8, 1, 1),
                                   1);
                    mma_commit(mbar2);
                }
                mma_wait(mm);  // dX
                const int wid = tid >> 5;
                float *dcrow = reinterpret_cast<float *>(wid < 2 ? xt : h1t) + ((wid & 1) * 32 + (tid & 31)) * DC_ROW;
                float dx16[16];
                tmem_ld16(mm.tmem + lane + DXCOL, dx16);
                tmem_wait_ld();
                float dxu = 0.0f, dxw = 0.0f;
                if (valid) {
                    // LUT: dX element 2l+f -> feature gradients of level l and the coordinate gradient
                    // groups of four levels, one group at a time (decoder 1 has two)
#pragma unroll 1
                    for (int hb = 0; hb < Dec<DK>::LEVELS / 4; ++hb)
#pragma unroll
                    for (int lq = 0; lq < 4; ++lq) {
                        const int l = 4 * hb + lq;
                        LutCell c = lut_cell<DK>(l, cu, cw);
                        float dx_ = (hb ? dx16[8 + 2 * lq] : dx16[2 * lq]) * ginv,
                              dy_ = (hb ? dx16[9 + 2 * lq] : dx16[2 * lq + 1]) * ginv;
                        float ux = c.fx, vx = 1.0f - ux, uy = c.fy, vy = 1.0f - uy;
                        float2 f00 = __ldg(lut2 + c.i00), f10 = __ldg(lut2 + c.i00 + 1),
                               f01 = __ldg(lut2 + c.i00 + c.R), f11 = __ldg(lut2 + c.i00 + c.R + 1);
                        float dfx_x = __fmaf_rn(f10.x - f00.x, vy, (f11.x - f01.x) * uy);
                        float dfx_y = __fmaf_rn(f10.y - f00.y, vy, (f11.y - f01.y) * uy);
                        float dfy_x = __fmaf_rn(f01.x - f00.x, vx, (f11.x - f10.x) * ux);
                        float dfy_y = __fmaf_rn(f01.y - f00.y, vx, (f11.y - f10.y) * ux);
                        float sc_ = 0.5f * LUT_SCALE * ((float)c.R - 1.0f);
                        dxu += sc_ * __fmaf_rn(dx_, dfx_x, dy_ * dfx_y);
                        dxw += sc_ * __fmaf_rn(dx_, dfy_x, dy_ * dfy_y);
                        float *F = bo.dfeat_priv + (size_t)blockIdx.x * LUT_PRIV_STRIDE + 4 * (size_t)c.i00;
                        red_add_v4(F, dx_ * vx * vy, dy_ * vx * vy, dx_ * ux * vy, dy_ * ux * vy);
                        red_add_v4(F + 4 * c.R, dx_ * vx * uy, dy_ * vx * uy, dx_ * ux * uy, dy_ * ux * uy);
                    }
                }
                gu += dxu;
                gw += dxw;
                if (valid) geom_grads(g, v, gu, gw, dLdt_depth, ow, sgn, nvalid, Nm, bo.lambda_normal, pg);
                // the weight-gradient MMAs have read the X / H1 / H2 tiles: the staging rows may overwrite them
                if (!mbar_wait(mbar2, par2)) atomicExch(&s_abort, 1);
                par2 ^= 1u;
                if constexpr (DK == 1) {  // delta1 = G1 (still in TMEM columns 0..63) gated by the ReLU mask
#pragma unroll
                    for (int cb = 0; cb < 4; ++cb) {
                        float gv[16];
                        tmem_ld16(mm.tmem + lane + 16 * cb, gv);
                        tmem_wait_ld();
                        if (valid) {
#pragma unroll
                            for (int e = 0; e < 16; e += 4) {
                                float d[4];
#pragma unroll
                                for (int q = 0; q < 4; ++q)
                                    d[q] = ((m1 >> (16 * cb + e + q)) & 1ull) ? gv[e + q] * ginv : 0.0f;
                                *reinterpret_cast<float4 *>(dcrow + PGRAD_FLOATS + 16 * cb + e) =
                                    make_float4(d[0], d[1], d[2], d[3]);
                            }
                        }
                    }
                } else if (valid) {  // delta1 into the staging row
#pragma unroll
                    for (int e = 0; e < 64; e += 4)
                        *reinterpret_cast<float4 *>(dcrow + PGRAD_FLOATS + e) =
                            make_float4(hd1[e] * ginv, hd1[e + 1] * ginv, hd1[e + 2] * ginv, hd1[e + 3] * ginv);
                }
                if (valid) {
                    // this hit's row [packed primitive gradients | delta1] -> one bulk reduction
#pragma unroll
                    for (int e = 0; e < PG_N; e += 2)
                        *reinterpret_cast<float2 *>(dcrow + e) = make_float2(pg[e], pg[e + 1]);
#pragma unroll
                    for (int e = PG_N; e < PGRAD_FLOATS; e += 2)
                        *reinterpret_cast<float2 *>(dcrow + e) = make_float2(0.0f, 0.0f);
                    fence_async_smem();
                    bulk_red_add_f32(bo.pgrad + (size_t)ind * PROW_FLOATS, dcrow, PROW_FLOATS * 4);
                }
                bulk_pending = valid;  // its staging row is read before the next slot's first barrier
                tc_fence_before();
                if (tid == 0) s_first = 0;
            }
            if (!DEC && valid) {  // decoder-free path: straight into the caller's arrays
                geom_grads(g, v, gu, gw, dLdt_depth, ow, sgn, nvalid, Nm, bo.lambda_normal, pg);
                flush_prim_direct(bo, ind, pg);
            }
            if (have) {
                ++h;
                if (!valid || h == K_PASS) {  // this ray's pass is done: write its state back
                    // full: all K_PASS slots composited; a bounded pass that ended early continues too
                    const bool full = valid && h == K_PASS;
                    PassEnd pe{full, full ? nextafterf(t_hit, INFINITY) : INFINITY, INFINITY};
                    if (pp.hint)
                        pe = pass_end(full, t_hit, full ? pp.hit_t[(size_t)(K_PASS / 2 - 1) * pp.count + slot] : 0.0f,
                                      pp.hint[ray], pp.bound_f);
                    const bool active = pe.more && T >= pp.T_thr;
                    for (int c = 0; c < 3; ++c) bo.I[3 * (size_t)ray + c] = -run[c];
                    for (int c = 0; c < 4; ++c) bo.prefix[4 * (size_t)ray + c] = P[c];
                    pp.t_min[ray] = active ? pe.t_min : INFINITY;
                    if (pp.hint) pp.hint[ray] = pe.hint;
                    pp.T[ray] = T;
                    pp.flags[slot] = active;
                    have = false;
                }
            }
        }
    }
done:
    if (tid == 0 && ntiles) atomicAdd(pp.stats + ST_TILES, ntiles);
    if (DEC) {
        wait_bulk_done();
        if (s_abort && tid == 0) atomicOr(pp.status, ERR_MBAR);
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        // flush this CTA's weight-gradient accumulators (all lanes load the same columns)
        if (!s_first && !s_abort) {
            const int w = tid >> 5, l = tid & 31;
            const uint32_t lane = (uint32_t)((w * 32) << 16);
            const int mrow = 16 * w + (l & 15);
#pragma unroll 1
            for (int b = 0; b < 8; ++b) {
                float vals[16];
                tmem_ld16(mm.tmem + lane + TM_DW + 16 * b, vals);
                tmem_wait_ld();
                for (int e = 0; e < 16; ++e) {
                    const int col = 16 * b + e;
                    const float x = vals[e] * ginv;
                    if (l < 16) {  // half 0: dW1 row mrow (decoder 1: columns 64..95 hold the lo inputs' share of
                                   // columns 0..31)
                        atomicAdd(bo.dw + DW_W1 + mrow * 128 + ((DK == 1 && col >= 64 && col < 96) ? col - 64 : col), x);
                    } else {       // half 1: dW2 row mrow | dW3^T row mrow | db2 | db3 | db1
                        if (col < 64) atomicAdd(bo.dw + DW_W2 + mrow * 64 + col, x);
                        else if (col < 72) atomicAdd(bo.dw + DW_W3 + ((col - 64) & 3) * 64 + mrow, x);
                        else if (col == 72) atomicAdd(bo.dw + DW_B2 + mrow, x);
                        else if (col == 80 && mrow < 8) atomicAdd(bo.dw + DW_B3 + (mrow & 3), x);
                        else if (col == 88) atomicAdd(bo.dw + DW_B1 + mrow, x);
                    }
                }
            }
        }
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (tid < 32) tmem_dealloc(mm.tmem, TM_BWD_COLS);
    }
}

// ================================================================================================
// helpers: init, gradient scale, dW packing into the reference fragment layout
// ================================================================================================
__global__ void init_rays_kernel(int R, float *T, float *t_min, int *list, float *med, float *hint) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= R) return;
    T[i] = 1.0f;
    t_min[i] = 0.0f;
    if (hint) hint[i] = INFINITY;
    list[i] = i;
    if (med) {
        med[2 * (size_t)i] = INFINITY;
        med[2 * (size_t)i + 1] = __int_as_float(-1);
    }
}

__global__ void grad_scale_kernel(const float *dL_dI, int n3, float lambda_depth, float *scale_out) {
    __shared__ float red[32];
    float mx = fabsf(lambda_depth);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n3; i += gridDim.x * blockDim.x) mx = fmaxf(mx, fabsf(dL_dI[i]));
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    if (threadIdx.x < 32) {
        mx = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (threadIdx.x == 0) atomicMax(reinterpret_cast<int *>(scale_out), __float_as_int(mx));
    }
}

// max |dL/dI| (stored as float bits) -> power-of-two scale with max * scale ~ 2^4
__global__ void grad_scale_finish_kernel(float *scale) {
    float mx = scale[0];
    int e = 0;
    if (mx > 0.0f && isfinite(mx)) {
        frexpf(mx, &e);
        e = 4 - e;
        e = max(-100, min(100, e));
    }
    scale[0] = ldexpf(1.0f, e);
}

// dfeat[i] += sum over the per-CTA copies
// Sums the per-CTA pair-major copies: feature i of cell c = i / 2 is the cell's own slot plus the
// right-neighbour slot of cell c - 1 (a bilinear row never spans two rows or levels, so that slot is
// zero wherever c - 1 is not a left corner of c).
__global__ void reduce_lut_kernel(const float *__restrict__ priv, int copies, float *__restrict__ dfeat, int nfeat) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nfeat) return;
    const int cell = i >> 1, f = i & 1;
    float acc = 0.0f;
    for (int c = 0; c < copies; ++c) {
        const float *P = priv + (size_t)c * LUT_PRIV_STRIDE;
        acc += P[4 * cell + f];
        if (cell > 0) acc += P[4 * (cell - 1) + 2 + f];
    }
    dfeat[i] += acc;
}

// Adds the per-primitive rows of the decoder backward into the caller's arrays, one warp per primitive:
// the packed gradients (layout PG_*) directly, and the descriptor gradient dcond = W1[:, 32:128)^T d1,
// d1 being the primitive's summed layer-1 deltas (W1 (64, 128) f16, row = output); cdim = the descriptor
// width (96 or 32).
__global__ void __launch_bounds__(256) scatter_prow_kernel(const float *__restrict__ prow, int n,
                                                           const __half *__restrict__ A1, float *dm, float *ds,
                                                           float *dq, float *dRGB, float *dA, float *dk,
                                                           float *dcond, int cdim) {
    __shared__ float w[64 * 96];  // w[k * 96 + j] = W1[k][32 + j], j < cdim
    __shared__ float rows[8][64];
    for (int i = threadIdx.x; i < 64 * 96; i += blockDim.x)
        w[i] = (i % 96) < cdim ? __half2float(A1[(i / 96) * 128 + 32 + i % 96]) : 0.0f;
    __syncthreads();
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int nw = gridDim.x * 8;
    for (int p = blockIdx.x * 8 + wib; p < n; p += nw) {
        const float *r = prow + (size_t)p * PROW_FLOATS;
        const float a = r[lane], b = r[32 + lane], c = lane < 16 ? r[64 + lane] : 0.0f;
        if (!__any_sync(0xffffffffu, a != 0.0f || b != 0.0f || c != 0.0f)) continue;  // not hit
        if (lane < PG_N) {
            float *dst;
            if (lane < PG_S) dst = dm + 3 * (size_t)p + lane;
            else if (lane < PG_Q) dst = ds + 2 * (size_t)p + (lane - PG_S);
            else if (lane < PG_RGB) dst = dq + 4 * (size_t)p + (lane - PG_Q);
            else if (lane < PG_A) dst = dRGB + 3 * (size_t)p + (lane - PG_RGB);
            else if (lane == PG_A) dst = dA + p;
            else dst = dk + p;
            *dst += a;
        }
        if (dcond) {
            if (lane >= PGRAD_FLOATS) rows[wib][lane - PGRAD_FLOATS] = a;
            rows[wib][16 + lane] = b;
            if (lane < 16) rows[wib][48 + lane] = c;
            __syncwarp();
            float o0 = 0.0f, o1 = 0.0f, o2 = 0.0f;
#pragma unroll 8
            for (int k = 0; k < 64; ++k) {
                const float d = rows[wib][k];
                o0 = __fmaf_rn(w[k * 96 + lane], d, o0);
                o1 = __fmaf_rn(w[k * 96 + 32 + lane], d, o1);
                o2 = __fmaf_rn(w[k * 96 + 64 + lane], d, o2);
            }
            __syncwarp();
            float *dc = dcond + (size_t)p * cdim;
            dc[lane] += o0;
            if (cdim == 96) {
                dc[32 + lane] += o1;
                dc[64 + lane] += o2;
            }
        }
    }
}

// Adds the dense MLP gradients into row 0 of the reference's fragment-layout buffers
// (layout decoded from train.py:754-790).
__global__ void pack_dw_kernel(const float *dw, float *dw1, float *db1, float *dw2, float *db2, float *dw3,
                               float *db3) {
    int t = blockIdx.x * blockDim.x + threadIdx.x;
    // dW1: flat[(i*16 + j)*64 + c*32 + lane] = W1g[8i + lane/4][8j + 2(lane%4) + c]
    if (t < 8192) {
        int lane = t & 31, c = (t >> 5) & 1, ij = t >> 6, i = ij >> 4, j = ij & 15;
        int row = 8 * i + (lane >> 2), col = 8 * j + 2 * (lane & 3) + c;
        if (dw1) dw1[t] += dw[DW_W1 + row * 128 + col];
    }
    if (t < 4096) {
        int lane = t & 31, c = (t >> 5) & 1, ij = t >> 6, i = ij >> 3, j = ij & 7;
        int row = 8 * i + (lane >> 2), col = 8 * j + 2 * (lane & 3) + c;
        if (dw2) dw2[t] += dw[DW_W2 + row * 64 + col];
    }
    if (t < 512) {
        int lane = t & 31, c = (t >> 5) & 1, j = t >> 6;
        int row = lane >> 2, col = 8 * j + 2 * (lane & 3) + c;
        if (dw3 && row < 4) dw3[t] += dw[DW_W3 + row * 64 + col];
        // db1/db2: flat[j*64 + c*32 + lane] summed into b[8j + lane/4]; put it at c = 0, lane%4 = 0
        if (c == 0 && (lane & 3) == 0) {
            if (db1) db1[t] += dw[DW_B1 + 8 * j + (lane >> 2)];
            if (db2) db2[t] += dw[DW_B2 + 8 * j + (lane >> 2)];
        }
    }
    if (t < 64) {
        int lane = t & 31, c = (t >> 5) & 1;
        int row = lane >> 2;
        if (db3 && c == 0 && (lane & 3) == 0 && row < 4) db3[t] += dw[DW_B3 + row];
    }
}

// ================================================================================================
// host drivers
// ================================================================================================
static SceneP scene_params(const flare_scene *sc, const float *override_colors) {
    SceneP p;
    p.m = sc->m; p.s = sc->s; p.q = sc->q; p.RGBA = sc->RGBA; p.k = sc->k;
    p.cond = reinterpret_cast<const uint4 *>(sc->cond);
    p.features = sc->features;
    p.A1 = reinterpret_cast<const __half *>(sc->A1);
    p.A2 = reinterpret_cast<const __half *>(sc->A2);
    p.A3 = reinterpret_cast<const __half *>(sc->A3);
    p.b1 = sc->b1; p.b2 = sc->b2; p.b3 = sc->b3;
    p.override_colors = override_colors;
    p.n = sc->n;
    return p;
}

template <bool DEC, int MODE, int DK = 0>
static int launch_fwd(flare_renderer *r, const SceneP &sp, const PassP &pp, const FwdOut &fo, cudaStream_t st) {
    auto kern = shade_fwd_kernel<DEC, MODE, DK>;
    int smem = DEC ? SM_FWD_BYTES : 0;
    if (DEC) FLARE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    int chunks = (pp.count + 127) / 128;
    int grid = DEC ? std::min(chunks, r->num_sms * FLARE_FWD_CTAS) : chunks;
    if (DEC) FLARE_CUDA_TRY(cudaMemsetAsync(pp.work, 0, sizeof(int), st));
    kern<<<grid, 128, smem, st>>>(sp, pp, fo);
    FLARE_CUDA_TRY(cudaGetLastError());
    return FLARE_OK;
}

template <bool DEC, int DK = 0>
static int launch_fwd_mode(flare_renderer *r, int mode, const SceneP &sp, const PassP &pp, const FwdOut &fo,
                           cudaStream_t st) {
    switch (mode) {
        case FLARE_FWD_TRAINING: return launch_fwd<DEC, FLARE_FWD_TRAINING, DK>(r, sp, pp, fo, st);
        case FLARE_FWD_INFERENCE: return launch_fwd<DEC, FLARE_FWD_INFERENCE, DK>(r, sp, pp, fo, st);
        case FLARE_FWD_INFERENCE_GEOMETRY: return launch_fwd<DEC, FLARE_FWD_INFERENCE_GEOMETRY, DK>(r, sp, pp, fo, st);
        case FLARE_FWD_PCA: return launch_fwd<DEC, FLARE_FWD_PCA, DK>(r, sp, pp, fo, st);
        case FLARE_FWD_MEDIAN: return launch_fwd<DEC, FLARE_FWD_MEDIAN, DK>(r, sp, pp, fo, st);
    }
    set_error("unknown forward mode %d", mode);
    return FLARE_E_INVALID;
}

// One pass of the secondary-ray path: decode + composite the hit lists of `count` rays (list `lin`)
// into bitmap, with shadowed hits darkened; per-ray T and t_min are the generation's own arrays.  The
// per-slot still-active flags land in r->pass_flags for the compaction.
int launch_shade_viewer(flare_renderer *r, const flare_scene *sc, const float *O, const float *v, const int *lin,
                        int count, const float *ht, const int *hi, const unsigned char *shadow, float shadow_mult,
                        float *T, float *t_min, float *bitmap, float T_thr, cudaStream_t st);

// ------------------------------------------------------------------------------------------------
// Hit cache.  A Backward re-walks exactly the passes of the Forward_training that produced its image
// (same rays, geometry and parameters give the same active rays and the same 16-hit lists per pass), so
// the forward keeps each pass's active-ray list and hit lists and a matching backward replays them
// instead of tracing again.  "Matching" is checked by a pointer/size signature and by a checksum of the
// contents of every input the pass sequence depends on (rays, primitive parameters, decoder).
// ------------------------------------------------------------------------------------------------
struct HashBufs {
    const unsigned *p[16];
    unsigned long long n[16];
    int count;
};

__device__ __forceinline__ unsigned long long hash_word(unsigned w, unsigned long long i, int b) {
    unsigned long long x = ((unsigned long long)w << 32) ^ (i * 0x9E3779B97F4A7C15ull) ^ (unsigned long long)b;
    x ^= x >> 33;
    x *= 0xff51afd7ed558ccdull;
    x ^= x >> 33;
    return x;
}

// Sum over every 32-bit word of every buffer of hash_word(word, index, buffer).  The words before the first
// 16-byte boundary and after the last are read one by one; the body as 16-byte vectors, four per thread in
// flight, so that the read runs near HBM bandwidth (a buffer can be a slice at any 4-byte offset).
__global__ void checksum_kernel(HashBufs hb, unsigned long long *out) {
    unsigned long long acc = 0;
    const unsigned long long tid = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x;
    const unsigned long long stride = (unsigned long long)gridDim.x * blockDim.x;
    for (int b = 0; b < hb.count; ++b) {
        const unsigned *p = hb.p[b];
        const unsigned long long n = hb.n[b];
        unsigned long long head = ((16u - ((unsigned)(uintptr_t)p & 15u)) & 15u) / 4u;
        if (head > n) head = n;
        const unsigned long long nv = (n - head) / 4;
        const uint4 *pv = reinterpret_cast<const uint4 *>(p + head);
        const unsigned long long tail0 = head + nv * 4;
        for (unsigned long long t = tid; t < head; t += stride) acc += hash_word(__ldg(p + t), t, b);
        for (unsigned long long t = tail0 + tid; t < n; t += stride) acc += hash_word(__ldg(p + t), t, b);
        unsigned long long j = tid;
        for (; j + 3 * stride < nv; j += 4 * stride) {
            uint4 w[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) w[u] = __ldg(pv + j + u * stride);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const unsigned long long i0 = head + 4 * (j + u * stride);
                acc += hash_word(w[u].x, i0, b) + hash_word(w[u].y, i0 + 1, b) + hash_word(w[u].z, i0 + 2, b) +
                       hash_word(w[u].w, i0 + 3, b);
            }
        }
        for (; j < nv; j += stride) {
            const uint4 w = __ldg(pv + j);
            const unsigned long long i0 = head + 4 * j;
            acc += hash_word(w.x, i0, b) + hash_word(w.y, i0 + 1, b) + hash_word(w.z, i0 + 2, b) +
                   hash_word(w.w, i0 + 3, b);
        }
    }
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) atomicAdd(out, acc);
}

static int input_checksum(flare_renderer *r, const flare_scene *sc, const float *O, const float *v, int R,
                          unsigned long long *out, cudaStream_t st) {
    HashBufs hb{};
    auto add = [&](const void *p, size_t bytes) {
        if (p && bytes >= 4 && hb.count < 16) {
            hb.p[hb.count] = static_cast<const unsigned *>(p);
            hb.n[hb.count] = bytes / 4;
            ++hb.count;
        }
    };
    const size_t n = (size_t)sc->n;
    add(O, (size_t)R * 12);
    add(v, (size_t)R * 12);
    add(sc->m, n * 12);
    add(sc->s, n * 8);
    add(sc->q, n * 16);
    add(sc->RGBA, n * 16);
    add(sc->k, n * 4);
    if (sc->cond) {
        add(sc->cond, n * (sc->decoder ? Dec<1>::COND : Dec<0>::COND) * 2);
        add(sc->features, (size_t)(sc->decoder ? Dec<1>::FEATS : Dec<0>::FEATS) * 4);
        add(sc->A1, 64 * 128 * 2);
        add(sc->A2, 64 * 64 * 2);
        add(sc->A3, 16 * 64 * 2);
        add(sc->b1, 64 * 4);
        add(sc->b2, 64 * 4);
        add(sc->b3, 16 * 4);
    }
    FLARE_CUDA_TRY(cudaMemsetAsync(out, 0, sizeof(unsigned long long), st));
    checksum_kernel<<<r->num_sms * 4, 256, 0, st>>>(hb, out);
    FLARE_CUDA_TRY(cudaGetLastError());
    return FLARE_OK;
}

static void cache_key(const flare_scene *sc, const float *O, const float *v, int R, float T_thr, unsigned long long geom,
                      unsigned long long *key) {
    key[0] = (unsigned long long)(uintptr_t)O;
    key[1] = (unsigned long long)(uintptr_t)v;
    key[2] = (unsigned long long)R;
    key[3] = (unsigned long long)sc->n;
    key[4] = (unsigned long long)(uintptr_t)sc->m;
    key[5] = (unsigned long long)(uintptr_t)sc->s;
    key[6] = (unsigned long long)(uintptr_t)sc->q;
    key[7] = (unsigned long long)(uintptr_t)sc->RGBA;
    key[8] = (unsigned long long)(uintptr_t)sc->k;
    key[9] = (unsigned long long)(uintptr_t)sc->cond;
    key[10] = (unsigned long long)(uintptr_t)sc->A1;
    key[11] = geom;
    unsigned tb = 0;
    memcpy(&tb, &T_thr, 4);
    key[12] = tb;
    key[13] = key[14] = key[15] = 0;
}

// Grows the cache to the ray-passes the last uncached forward needed, within a device-memory budget
// (FLARE_HIT_CACHE_MB, default half of the free memory).  Runs before any pass, never inside the loop.
static void grow_cache(flare_renderer *r) {
    if (r->hc_need <= r->hc_cap) return;
    size_t want = r->hc_need + r->hc_need / 8 + 1024;
    size_t bytes = want * (4 + (size_t)K_PASS * 8);
    size_t freeb = 0, total = 0;
    cudaMemGetInfo(&freeb, &total);
    size_t budget = freeb / 2;
    if (const char *e = getenv("FLARE_HIT_CACHE_MB")) budget = (size_t)atoll(e) << 20;
    r->hc_need = 0;
    if (bytes > budget) return;
    cudaFree(r->hc_list); cudaFree(r->hc_t); cudaFree(r->hc_idx);
    r->hc_list = nullptr; r->hc_t = nullptr; r->hc_idx = nullptr; r->hc_cap = 0;
    if (cudaMalloc(&r->hc_list, want * 4) != cudaSuccess || cudaMalloc(&r->hc_t, want * K_PASS * 4) != cudaSuccess ||
        cudaMalloc(&r->hc_idx, want * K_PASS * 4) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(r->hc_list); cudaFree(r->hc_t); cudaFree(r->hc_idx);
        r->hc_list = nullptr; r->hc_t = nullptr; r->hc_idx = nullptr;
        return;
    }
    r->hc_cap = want;
}

// Bounded later passes (pass_end above); FLARE_PASS_BOUND=0 turns them off.
// FLARE_PASS_BOUND_F: the factor of the bound (default 3; the pass-exact parity test assumes 3).
static float pass_bound_factor() {
    static const float f = [] {
        const char *e = getenv("FLARE_PASS_BOUND_F");
        return e ? (float)atof(e) : 3.0f;
    }();
    return f;
}

static bool pass_bound_on() {
    static const bool on = [] {
        const char *e = getenv("FLARE_PASS_BOUND");
        return !(e && strcmp(e, "0") == 0);
    }();
    return on;
}

// Runs the pass loop: trace -> shade -> compaction, until no ray is active.
template <typename ShadeFn>
static int pass_loop(flare_renderer *r, const float *O, const float *v, int R, cudaStream_t st, int shade_kind,
                     ShadeFn shade, bool cache = false) {
    int count = R;
    int cur = 0;
    long long passes = 0;
    size_t off = 0;
    bool cached = cache;
    const long long max_passes = (long long)(r->n / K_PASS) + 4;
    while (count > 0) {
        if (passes > max_passes) {
            set_error("pass loop did not terminate after %lld passes", passes);
            return FLARE_E_DEVICE;
        }
        float *ht = r->hit_t;
        int *hi = r->hit_idx;
        if (cached && (off + count > r->hc_cap || passes >= flare_renderer::HC_MAX_PASSES)) cached = false;
        if (cached) {  // hits go straight into the cache; the active list is copied beside them
            ht = r->hc_t + (size_t)K_PASS * off;
            hi = r->hc_idx + (size_t)K_PASS * off;
            FLARE_CUDA_TRY(cudaMemcpyAsync(r->hc_list + off, r->list[cur], (size_t)count * sizeof(int),
                                           cudaMemcpyDeviceToDevice, st));
            r->hc_off[passes] = off;
            r->hc_cnt[passes] = count;
        }
        off += count;
        int slot = prof_begin(r, PK_TRACE, st);
        int e = launch_trace(r, O, v, r->t_min, r->list[cur], count, ht, hi, count, st, K_PASS,
                             pass_bound_on() ? r->hint : nullptr, passes == 0);
        prof_end(r, slot, st);
        if (e) return e;
        slot = prof_begin(r, shade_kind, st);
        e = shade(r->list[cur], count, ht, hi);
        prof_end(r, slot, st);
        if (e) return e;
        e = compact_active(r, r->list[cur], count, r->list[cur ^ 1], st);
        if (e) return e;
        FLARE_CUDA_TRY(cudaMemcpyAsync(r->h_count, r->counters, sizeof(int), cudaMemcpyDeviceToHost, st));
        FLARE_CUDA_TRY(cudaStreamSynchronize(st));
#ifdef FLARE_PASS_TRACE
        if (r->prof_on && r->prof_n >= 2) {
            float tms = 0.0f, sms = 0.0f;
            cudaEventElapsedTime(&tms, r->prof_ev[2 * (r->prof_n - 2)], r->prof_ev[2 * (r->prof_n - 2) + 1]);
            cudaEventElapsedTime(&sms, r->prof_ev[2 * (r->prof_n - 1)], r->prof_ev[2 * (r->prof_n - 1) + 1]);
            static unsigned long long last[ST_NSTATS];
            unsigned long long h[ST_NSTATS];
            cudaMemcpy(h, r->dstats, sizeof(h), cudaMemcpyDeviceToHost);
            fprintf(stderr, "pass %lld rays %d trace %.3f ms shade %.3f ms nodes %llu prims %llu hits %llu\n", passes,
                    count, tms, sms, h[ST_NODES] - last[ST_NODES], h[ST_PRIM_TESTS] - last[ST_PRIM_TESTS],
                    h[ST_HITS] - last[ST_HITS]);
            fprintf(stderr, "   max nodes per walk %llu\n", h[5]);
            cudaMemset(r->dstats + 5, 0, 8);
            memcpy(last, h, sizeof(h));
        }
#endif
        prof_collect(r);
        count = *r->h_count;
        cur ^= 1;
        ++passes;
    }
    if (cache) {
        r->hc_valid = cached;
        r->hc_npass = cached ? (int)passes : 0;
        if (!cached) r->hc_need = off;  // the next forward grows the cache before its first pass
    }
    unsigned long long p = (unsigned long long)passes;
    FLARE_CUDA_TRY(cudaMemcpyAsync(r->dstats + ST_PASSES, &p, sizeof(p), cudaMemcpyHostToDevice, st));
    FLARE_CUDA_TRY(cudaStreamSynchronize(st));
    return FLARE_OK;
}

static PassP make_pass(flare_renderer *r, const float *O, const float *v, float bg0, float bg1, float bg2,
                       float T_thr) {
    PassP pp{};
    pp.hint = pass_bound_on() ? r->hint : nullptr;
    pp.bound_f = pass_bound_factor();
    pp.O = O; pp.v = v;
    pp.hit_t = r->hit_t; pp.hit_idx = r->hit_idx;
    pp.T = r->T; pp.t_min = r->t_min;
    pp.flags = r->pass_flags;
    pp.work = r->counters + 1;
    pp.status = r->dstatus;
    pp.stats = r->dstats;
    pp.bg0 = bg0; pp.bg1 = bg1; pp.bg2 = bg2;
    pp.T_thr = T_thr;
    return pp;
}

int run_forward(flare_renderer *r, const flare_scene *sc, const flare_forward_args *a, cudaStream_t st) {
    const int R = a->n_rays;
    if (R <= 0) return FLARE_OK;
    const bool dec = sc->cond != nullptr;
    SceneP sp = scene_params(sc, a->override_colors);
    FwdOut fo{};
    fo.bitmap = a->bitmap; fo.dacc = a->depth_reg_accums; fo.nacc = a->normal_reg_accums;
    fo.normal = a->normal; fo.alpha = a->alpha; fo.edn = a->expected_depth_numerator;
    fo.med = a->depth_and_index; fo.surface_normal = a->surface_normal;
    fo.reg_a = a->reg_a; fo.reg_b = a->reg_b;
    init_rays_kernel<<<(R + 255) / 256, 256, 0, st>>>(R, r->T, r->t_min, r->list[0],
                                                       a->mode == FLARE_FWD_MEDIAN ? a->depth_and_index : nullptr,
                                                       pass_bound_on() ? r->hint : nullptr);
    FLARE_CUDA_TRY(cudaGetLastError());
    {
        int e = order_rays(r, a->O, a->v, R, r->list[0], st);
        if (e) return e;
    }
    PassP base = make_pass(r, a->O, a->v, a->bg[0], a->bg[1], a->bg[2], a->T_threshold);
    const bool cache = a->mode == FLARE_FWD_TRAINING;
    r->hc_valid = false;
    if (cache) {
        grow_cache(r);
        cache_key(sc, a->O, a->v, R, a->T_threshold, r->geom_version, r->hc_key);
        int e = input_checksum(r, sc, a->O, a->v, R, r->hc_sum, st);
        if (e) return e;
    }
    return pass_loop(
        r, a->O, a->v, R, st, PK_SHADE_FWD,
        [&](const int *lin, int count, const float *ht, const int *hi) -> int {
            PassP pp = base;
            pp.list_in = lin;
            pp.count = count;
                pp.hit_t = ht;
            pp.hit_idx = hi;
            if (!dec) return launch_fwd_mode<false>(r, a->mode, sp, pp, fo, st);
            return sc->decoder ? launch_fwd_mode<true, 1>(r, a->mode, sp, pp, fo, st)
                               : launch_fwd_mode<true, 0>(r, a->mode, sp, pp, fo, st);
        },
        cache);
}

int run_backward(flare_renderer *r, const flare_scene *sc, const flare_backward_args *a, cudaStream_t st) {
    const int R = a->n_rays;
    if (R <= 0) return FLARE_OK;
    const bool dec = sc->cond != nullptr;
    SceneP sp = scene_params(sc, nullptr);
    BwdIO bo{};
    bo.I = a->I; bo.dL_dI = a->dL_dI;
    bo.dRGB = a->dL_dRGB; bo.dA = a->dL_dA; bo.dk = a->dL_dk; bo.dm = a->dL_dm; bo.ds = a->dL_ds; bo.dq = a->dL_dq;
    bo.dcond = a->dL_dcond; bo.dfeat = a->dL_dfeatures;
    bo.dw = r->dw;
    bo.dacc = a->depth_reg_accums; bo.prefix = a->depth_normal_reg_prefix_sums;
    bo.surface_normal = a->surface_normal;
    bo.lambda_depth = a->lambda_depth; bo.reg_a = a->reg_a; bo.reg_b = a->reg_b; bo.lambda_normal = a->lambda_normal;
    bo.gscale = r->gscale;
    bo.dfeat_priv = r->dfeat_priv;
    const bool rows_out = dec && a->prim_rows != nullptr;  // caller-owned rows, scattered by the caller
    if (dec && !rows_out && (size_t)sc->n > r->pgrad_cap) {
        cudaFree(r->pgrad);
        r->pgrad = nullptr;
        r->pgrad_cap = 0;
        FLARE_CUDA_TRY(cudaMalloc(&r->pgrad, (size_t)sc->n * PROW_FLOATS * sizeof(float)));
        r->pgrad_cap = sc->n;
    }
    bo.pgrad = rows_out ? a->prim_rows : r->pgrad;
    bo.vec4 = (reinterpret_cast<uintptr_t>(a->dL_dq) & 15) == 0;
    init_rays_kernel<<<(R + 255) / 256, 256, 0, st>>>(R, r->T, r->t_min, r->list[0], nullptr,
                                                       pass_bound_on() ? r->hint : nullptr);
    FLARE_CUDA_TRY(cudaGetLastError());
    if (dec) {
        FLARE_CUDA_TRY(cudaMemsetAsync(r->dw, 0, DW_TOTAL * sizeof(float), st));
        FLARE_CUDA_TRY(cudaMemsetAsync(r->gscale, 0, sizeof(float), st));
        grad_scale_kernel<<<std::min((3 * R + 255) / 256, 1024), 256, 0, st>>>(a->dL_dI, 3 * R, a->lambda_depth,
                                                                             r->gscale);
        grad_scale_finish_kernel<<<1, 1, 0, st>>>(r->gscale);
        FLARE_CUDA_TRY(cudaMemsetAsync(r->dfeat_priv, 0, (size_t)r->num_sms * 2 * LUT_PRIV_STRIDE * sizeof(float), st));
        if (sc->n > 0 && !rows_out)
            FLARE_CUDA_TRY(cudaMemsetAsync(r->pgrad, 0, (size_t)sc->n * PROW_FLOATS * sizeof(float), st));
        FLARE_CUDA_TRY(cudaFuncSetAttribute(shade_bwd_kernel<true, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            SM_BWD_BYTES));
        FLARE_CUDA_TRY(cudaFuncSetAttribute(shade_bwd_kernel<true, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            SM_BWD_BYTES));
    }
    PassP base = make_pass(r, a->O, a->v, a->bg[0], a->bg[1], a->bg[2], a->T_threshold);
    auto shade = [&](const int *lin, int count, const float *ht, const int *hi) -> int {
        PassP pp = base;
        pp.list_in = lin;
        pp.count = count;
        pp.hit_t = ht;
        pp.hit_idx = hi;
        int chunks = (count + 127) / 128;
        FLARE_CUDA_TRY(cudaMemsetAsync(pp.work, 0, sizeof(int), st));
        if (dec) {
            int grid = std::min(chunks, r->num_sms * 2);
            if (sc->decoder)
                shade_bwd_kernel<true, 1><<<grid, 128, SM_BWD_BYTES, st>>>(sp, pp, bo);
            else
                shade_bwd_kernel<true, 0><<<grid, 128, SM_BWD_BYTES, st>>>(sp, pp, bo);
        } else {
            shade_bwd_kernel<false, 0><<<chunks, 128, 0, st>>>(sp, pp, bo);
        }
        FLARE_CUDA_TRY(cudaGetLastError());
        return FLARE_OK;
    };
    bool replay = false;
    if (r->hc_valid) {
        unsigned long long key[16];
        cache_key(sc, a->O, a->v, R, a->T_threshold, r->geom_version, key);
        if (memcmp(key, r->hc_key, sizeof(key)) == 0) {
            int e = input_checksum(r, sc, a->O, a->v, R, r->hc_sum + 1, st);
            if (e) return e;
            unsigned long long h[2];
            FLARE_CUDA_TRY(cudaMemcpyAsync(h, r->hc_sum, sizeof(h), cudaMemcpyDeviceToHost, st));
            FLARE_CUDA_TRY(cudaStreamSynchronize(st));
            replay = h[0] == h[1];
        }
    }
    int e = FLARE_OK;
    if (replay) {  // the forward's passes, back to back, without tracing or host round trips
        for (int p = 0; p < r->hc_npass && !e; ++p) {
            int slot = prof_begin(r, PK_SHADE_BWD, st);
            const size_t off = r->hc_off[p];
            e = shade(r->hc_list + off, r->hc_cnt[p], r->hc_t + (size_t)K_PASS * off, r->hc_idx + (size_t)K_PASS * off);
            prof_end(r, slot, st);
        }
        unsigned long long np = (unsigned long long)r->hc_npass;
        FLARE_CUDA_TRY(cudaMemcpyAsync(r->dstats + ST_PASSES, &np, sizeof(np), cudaMemcpyHostToDevice, st));
        FLARE_CUDA_TRY(cudaStreamSynchronize(st));
        prof_collect(r);
    } else {  // no matching forward: trace again, from the coherence order of the rays
        e = order_rays(r, a->O, a->v, R, r->list[0], st);
        if (!e) e = pass_loop(r, a->O, a->v, R, st, PK_SHADE_BWD, shade);
    }
    if (e) return e;
    if (dec) {
        pack_dw_kernel<<<32, 256, 0, st>>>(r->dw, a->dL_dw1, a->dL_db1, a->dL_dw2, a->dL_db2, a->dL_dw3, a->dL_db3);
        const int nfeat = sc->decoder ? Dec<1>::FEATS : Dec<0>::FEATS;
        reduce_lut_kernel<<<(nfeat + 255) / 256, 256, 0, st>>>(r->dfeat_priv, r->num_sms * 2, a->dL_dfeatures, nfeat);
        if (sc->n > 0 && !rows_out)
            scatter_prow_kernel<<<std::min((sc->n + 7) / 8, r->num_sms * 8), 256, 0, st>>>(
                r->pgrad, sc->n, static_cast<const __half *>(sc->A1), a->dL_dm, a->dL_ds, a->dL_dq, a->dL_dRGB,
                a->dL_dA, a->dL_dk, a->dL_dcond, sc->decoder ? Dec<1>::COND : Dec<0>::COND);
        FLARE_CUDA_TRY(cudaGetLastError());
    }
    return FLARE_OK;
}

int run_scatter_rows(const float *rows, int n, const void *A1, int decoder, float *dRGB, float *dA, float *dk,
                     float *dm, float *ds, float *dq, float *dcond, cudaStream_t st) {
    if (n <= 0) return FLARE_OK;
    int dev = 0, sms = 148;
    FLARE_CUDA_TRY(cudaGetDevice(&dev));
    FLARE_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    scatter_prow_kernel<<<std::min((n + 7) / 8, sms * 8), 256, 0, st>>>(
        rows, n, static_cast<const __half *>(A1), dm, ds, dq, dRGB, dA, dk, dcond, decoder ? Dec<1>::COND : Dec<0>::COND);
    FLARE_CUDA_TRY(cudaGetLastError());
    return FLARE_OK;
}

// ------------------------------------------------------------------------------------------------
// self-test: the forward MLP tile on caller-provided rows
// ------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(128) selftest_mlp_kernel(const uint4 *X, int rows, SceneP sc, float *Y, int *status) {
    extern __shared__ __align__(1024) char smem[];
    __shared__ int s_abort;
    const int tid = threadIdx.x;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + SM_FWD_MISC + 8);
    if (tid == 0) {
        mbar_init(smem + SM_FWD_MISC, 1);
        fence_mbar_init();
        s_abort = 0;
    }
    if (tid < 32) tmem_alloc(tmem_slot, TM_FWD_COLS);
    load_decoder(smem, sc, false);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    Mma mm{*tmem_slot, 0u, smem + SM_FWD_MISC, &s_abort};
    char *tile = smem + SM_FWD_TILE;
    for (int base = blockIdx.x * 128; base < rows; base += gridDim.x * 128) {
        int row = base + tid;
        uint4 *T = reinterpret_cast<uint4 *>(tile);
        for (int kc = 0; kc < 16; ++kc) T[kc * 128 + tid] = row < rows ? X[(size_t)row * 16 + kc] : make_uint4(0, 0, 0, 0);
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        float y4[4];
        mlp_forward_tile(smem, tile, tile, tile, mm, y4, nullptr, 0);
        __syncthreads();
        if (s_abort) break;
        if (row < rows)
            for (int o = 0; o < 16; ++o) Y[(size_t)row * 16 + o] = o < 4 ? y4[o] : 0.0f;
    }
    if (s_abort && tid == 0) atomicOr(status, ERR_MBAR);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid < 32) tmem_dealloc(mm.tmem, TM_FWD_COLS);
}

int selftest_mlp(const void *X, int rows, const void *A1, const float *b1, const void *A2, const float *b2,
                 const void *A3, const float *b3, float *Y, cudaStream_t st, int *status) {
    if (rows <= 0) return FLARE_OK;
    SceneP sp{};
    sp.A1 = reinterpret_cast<const __half *>(A1);
    sp.A2 = reinterpret_cast<const __half *>(A2);
    sp.A3 = reinterpret_cast<const __half *>(A3);
    sp.b1 = b1; sp.b2 = b2; sp.b3 = b3;
    FLARE_CUDA_TRY(cudaFuncSetAttribute(selftest_mlp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SM_FWD_BYTES));
    int grid = std::max(1, std::min((rows + 127) / 128, 148));
    selftest_mlp_kernel<<<grid, 128, SM_FWD_BYTES, st>>>(reinterpret_cast<const uint4 *>(X), rows, sp, Y, status);
    FLARE_CUDA_TRY(cudaGetLastError());
    return FLARE_OK;
}

// One pass of the secondary-ray path (declared above the hit cache).
int launch_shade_viewer(flare_renderer *r, const flare_scene *sc, const float *O, const float *v, const int *lin,
                        int count, const float *ht, const int *hi, const unsigned char *shadow, float shadow_mult,
                        float *T, float *t_min, float *bitmap, float T_thr, cudaStream_t st) {
    if (count <= 0) return FLARE_OK;
    SceneP sp = scene_params(sc, nullptr);
    PassP pp = make_pass(r, O, v, 0.0f, 0.0f, 0.0f, T_thr);
    pp.hint = nullptr;  // the viewer bounds its passes by the nearest sphere instead
    pp.T = T;
    pp.t_min = t_min;
    pp.list_in = lin;
    pp.count = count;
    pp.hit_t = ht;
    pp.hit_idx = hi;
    FwdOut fo{};
    fo.bitmap = bitmap;
    fo.shadow = shadow;
    fo.shadow_mult = shadow_mult;
    if (!sc->cond) return launch_fwd<false, FWD_VIEWER>(r, sp, pp, fo, st);
    return sc->decoder ? launch_fwd<true, FWD_VIEWER, 1>(r, sp, pp, fo, st)
                       : launch_fwd<true, FWD_VIEWER, 0>(r, sp, pp, fo, st);
}

}  // namespace flare
