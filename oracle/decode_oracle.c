/*
 * decode_oracle.c -- CPU restatement of FlaRe's per-hit decode and front-to-back compositing.
 *
 * TEST INFRASTRUCTURE ONLY (checker and timed CPU baseline).  The product never links or calls it.
 *
 * Restates, per composited hit (reference paths relative to the FlaRe repository,
 * source/renderer/CPyOptiXFLARERenderer_CUDA_*.cu):
 *   - local coordinates (u, w) = e^-s * [U; V] . (O + t v - m)            Forward_training.cu:719-777
 *   - 4-level dense LUT encoding of 0.2968928 * (u, w), res {16,25,40,64}  Forward_training.cu:114-194,240-263
 *   - sin/cos view-direction encoding, 4 octaves                           Forward_training.cu:198-209,266-280
 *   - decoder input order [LUT 8 | PE 24 | descriptor 96], fp16            Forward_training.cu:213-292
 *   - MLP 128->64->64->16, Hardswish, fp16 activations, fp32 accumulate     Forward_training.cu:296-493
 *   - colour = RGB_base * relu(y[0:3]); alpha = sigma(A) G(r) sigmoid(y3)   Forward_training.cu:846-878
 *   - compositing while T >= T_thr, background at termination               Forward_training.cu:854-928
 *   - depth / normal regulariser accumulators                              Forward_training.cu:884-908
 *   - inference geometry outputs and override colours                      Forward_inference.cu:866-917
 *   - median depth (last hit while T > 0.5)                                GetMedianDepth.cu:852-867
 *   - base model (constant colour, alpha = sigma(A) G(r))                  Forward_training_base.cu:21-257
 * and the grid/SH decoder variant (decoder = 1, BASELINE config 0's encoder; no compiled reference code):
 *   - 8-level dense grid of the same (u, w) coordinates, res floor(4 * 1.5^l), row-major vertices
 *     (scripts/encoding_2d_benchmark.py:107-163 GridLevel / MultiResolutionEncoding with 2^16 entries)
 *   - degree-3 real spherical harmonics of v (16), descriptor 32, zeros 64; ReLU hidden layers;
 *     colour = RGB_base * sigmoid(y[0:3])
 * Transcendentals use libm (expf, logf, powf, sinf, cosf); the reference's fast intrinsics differ by a
 * few ulp, far inside the 1e-3 parity tolerance.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <omp.h>

#define K_HITS 16
#define LUT_SCALE 0.29689279887990428378374198030042f

enum { M_TRAIN = 0, M_INFER = 1, M_GEOM = 2, M_PCA = 3, M_MEDIAN = 4 };

typedef struct {
    const float *m, *s, *q, *RGBA, *k;
    const _Float16 *cond; /* NULL = base model */
    const float *features;
    const _Float16 *A1, *A2, *A3;
    const float *b1, *b2, *b3;
    const float *override_colors;
    int decoder; /* 0: LUT / sin-cos / 96 (reference); 1: grid / SH / 32 */
} oscene;

typedef struct {
    int mode;
    float bg[3];
    float T_thr, reg_a, reg_b;
} oparams;

/* Per-ray state carried across passes (the reference keeps these in the output buffers). */
typedef struct {
    float T;
    float rgb[3];
    float dacc[4];     /* depth_reg_accums */
    float nacc[4];     /* normal_reg_accums */
    float normal[3];
    float edn;         /* expected depth numerator */
    float med_t;
    int med_idx;
    int hits;          /* composited hits (statistics) */
} oray;

static inline float sat(float x) { return x < 0.0f ? 0.0f : (x > 1.0f ? 1.0f : x); }
static inline float hswish(float y) {
    float c = y + 3.0f;
    c = c < 0.0f ? 0.0f : (c > 6.0f ? 6.0f : c);
    return (y * c) * (1.0f / 6.0f);
}

static const int lut_res[4] = {16, 25, 40, 64};
static const int lut_off[4] = {0, 256, 881, 2481}; /* in float2 units */

static const int grid_res[8] = {4, 6, 9, 13, 20, 30, 45, 68};
static const int grid_off[8] = {0, 16, 52, 133, 302, 702, 1602, 3627}; /* in float2 units */

/* One bilinear lookup per level: nl levels of resolution res[l] at float2 offset off[l]. */
static void grid_encode(const float *features, float cu, float cw, int nl, const int *res, const int *off,
                        float *out) {
    for (int l = 0; l < nl; ++l) {
        int R = res[l];
        float xs = sat((cu + 1.0f) * 0.5f), ys = sat((cw + 1.0f) * 0.5f);
        float scale = (float)R - 1.0f;
        float px = xs * scale, py = ys * scale;
        int ix = (int)floorf(px), iy = (int)floorf(py);
        if (ix > R - 2) ix = R - 2;
        if (iy > R - 2) iy = R - 2;
        float fx = px - (float)ix, fy = py - (float)iy;
        const float *F = features + 2 * off[l];
        for (int f = 0; f < 2; ++f) {
            float f00 = F[2 * (iy * R + ix) + f], f10 = F[2 * (iy * R + ix + 1) + f];
            float f01 = F[2 * ((iy + 1) * R + ix) + f], f11 = F[2 * ((iy + 1) * R + ix + 1) + f];
            float r0 = fmaf(f00, 1.0f - fx, f10 * fx);
            float r1 = fmaf(f01, 1.0f - fx, f11 * fx);
            out[2 * l + f] = fmaf(r0, 1.0f - fy, r1 * fy);
        }
    }
}

static void lut_encode(const float *features, float cu, float cw, float *out8) {
    grid_encode(features, cu, cw, 4, lut_res, lut_off, out8);
}

/* Real spherical harmonics of degrees 0..3 of a unit direction (standard real basis, Condon-Shortley
   phase; the normalisation constants sqrt((2l+1)/(4 pi) (l-|m|)!/(l+|m|)!) times the usual factors). */
static void sh_deg3(float x, float y, float z, float *o) {
    float xx = x * x, yy = y * y, zz = z * z;
    o[0] = 0.28209479177387814f;
    o[1] = -0.48860251190291987f * y;
    o[2] = 0.48860251190291987f * z;
    o[3] = -0.48860251190291987f * x;
    o[4] = 1.0925484305920792f * x * y;
    o[5] = -1.0925484305920792f * y * z;
    o[6] = 0.94617469575755997f * zz - 0.31539156525251999f;
    o[7] = -1.0925484305920792f * x * z;
    o[8] = 0.54627421529603959f * (xx - yy);
    o[9] = 0.59004358992664352f * y * (-3.0f * xx + yy);
    o[10] = 2.8906114426405538f * x * y * z;
    o[11] = 0.45704579946446572f * y * (1.0f - 5.0f * zz);
    o[12] = 0.3731763325901154f * z * (5.0f * zz - 3.0f);
    o[13] = 0.45704579946446572f * x * (1.0f - 5.0f * zz);
    o[14] = 1.4453057213202769f * z * (xx - yy);
    o[15] = 0.59004358992664352f * x * (-xx + 3.0f * yy);
}

static inline float relu(float y) { return y > 0.0f ? y : 0.0f; }

/* Decoder: returns y[0..3] (pre-activation outputs 0..3 of layer 3). */
static void decode(const oscene *S, int idx, float cu, float cw, const float *v, float *y4) {
    float x[128];
    if (S->decoder == 1) {
        float enc[16], sh[16];
        grid_encode(S->features, cu, cw, 8, grid_res, grid_off, enc);
        sh_deg3(v[0], v[1], v[2], sh);
        for (int i = 0; i < 16; ++i) {  /* fed as f16 hi + lo parts (~22 bits): not rounded to f16 */
            x[i] = enc[i];
            x[16 + i] = sh[i];
        }
        for (int j = 0; j < 32; ++j) x[32 + j] = (float)S->cond[(long)idx * 32 + j];
        for (int j = 64; j < 128; ++j) x[j] = 0.0f;
    } else {
        float lut[8];
        lut_encode(S->features, cu, cw, lut);
        for (int i = 0; i < 8; ++i) x[i] = (float)(_Float16)lut[i];
        for (int a = 0; a < 3; ++a)
            for (int f = 0; f < 4; ++f) {
                float arg = (float)M_PI * (float)(1 << f) * v[a];
                x[8 + 8 * a + 2 * f] = (float)(_Float16)sinf(arg);
                x[9 + 8 * a + 2 * f] = (float)(_Float16)cosf(arg);
            }
        for (int j = 0; j < 96; ++j) x[32 + j] = (float)S->cond[(long)idx * 96 + j];
    }
    float h1[64], h2[64];
    for (int o = 0; o < 64; ++o) {
        float acc = S->b1[o];
        for (int kk = 0; kk < 128; ++kk) acc = fmaf((float)S->A1[o * 128 + kk], x[kk], acc);
        h1[o] = (float)(_Float16)(S->decoder == 1 ? relu(acc) : hswish(acc));
    }
    for (int o = 0; o < 64; ++o) {
        float acc = S->b2[o];
        for (int kk = 0; kk < 64; ++kk) acc = fmaf((float)S->A2[o * 64 + kk], h1[kk], acc);
        h2[o] = (float)(_Float16)(S->decoder == 1 ? relu(acc) : hswish(acc));
    }
    for (int o = 0; o < 4; ++o) {
        float acc = S->b3[o];
        for (int kk = 0; kk < 64; ++kk) acc = fmaf((float)S->A3[o * 64 + kk], h2[kk], acc);
        y4[o] = acc;
    }
}

/* Shades one pass (up to 16 hits, ascending t) of one ray.  Returns 1 if the ray stays active.
   `last_valid` is whether slot 16 held a hit (reference: is_active = ind16 != -1 && T >= thr). */
static int shade_pass(const oscene *S, const oparams *P, const float *O, const float *v, const float *ts,
                      const int *ids, int nh, const float *surface_normal, oray *st, int *count) {
    float T = st->T;
    int last_valid = (nh == K_HITS) && ids[K_HITS - 1] >= 0;
    float Nm[3] = {0, 0, 0};
    int nvalid = 0;
    if (surface_normal) {
        Nm[0] = surface_normal[0]; Nm[1] = surface_normal[1]; Nm[2] = surface_normal[2];
        nvalid = fmaf(Nm[0], Nm[0], fmaf(Nm[1], Nm[1], Nm[2] * Nm[2])) > 0.0f;
    }
    for (int h = 0; h < nh; ++h) {
        int idx = ids[h];
        if (idx < 0) break;
        int median = P->mode == M_MEDIAN;
        if (!(T >= P->T_thr) || (median && !(T > 0.5f))) break;
        float t = ts[h];
        const float *q = S->q + 4 * idx;
        float sx = expf(-S->s[2 * idx]), sy = expf(-S->s[2 * idx + 1]);
        float aa = q[0] * q[0], bb = q[1] * q[1], cc = q[2] * q[2], dd = q[3] * q[3];
        float Sq = 2.0f / (aa + bb + cc + dd);
        float bs = q[1] * Sq, cs = q[2] * Sq, ds = q[3] * Sq;
        float ab = q[0] * bs, ac = q[0] * cs, ad = q[0] * ds;
        bb = bb * Sq;
        float bc = q[1] * cs, bd = q[1] * ds;
        cc = cc * Sq;
        float cd = q[2] * ds;
        dd = dd * Sq;
        float Q11 = sx * (1.0f - cc - dd), Q12 = sx * (bc + ad), Q13 = sx * (bd - ac);
        float Q21 = sy * (bc - ad), Q22 = sy * (1.0f - bb - dd), Q23 = sy * (cd + ab);
        float N1 = bd + ac, N2 = cd - ab, N3 = 1.0f - bb - cc;
        float kap = 1.0f + logf(1.0f + expf(S->k[idx]));
        float kinv = 1.0f / kap;
        const float *m = S->m + 3 * idx;
        float dx = fmaf(v[0], t, O[0]) - m[0], dy = fmaf(v[1], t, O[1]) - m[1], dz = fmaf(v[2], t, O[2]) - m[2];
        float u = fmaf(Q11, dx, fmaf(Q12, dy, Q13 * dz));
        float w = fmaf(Q21, dx, fmaf(Q22, dy, Q23 * dz));
        const float *rgba = S->RGBA + 4 * idx;
        float sig_y = 1.0f, crgb[3] = {rgba[0], rgba[1], rgba[2]};
        if (S->cond) {
            float y[4];
            decode(S, idx, u * LUT_SCALE, w * LUT_SCALE, v, y);
            sig_y = 1.0f / (1.0f + expf(-y[3]));
            for (int c = 0; c < 3; ++c)
                crgb[c] = rgba[c] * (S->decoder == 1 ? 1.0f / (1.0f + expf(-y[c])) : (y[c] > 0.0f ? y[c] : 0.0f));
        }
        if (P->mode == M_PCA && S->override_colors)
            for (int c = 0; c < 3; ++c) crgb[c] = S->override_colors[3 * idx + c];
        float opa1 = 1.0f / (1.0f + expf(-rgba[3]));
        float r2 = fmaf(u, u, w * w);
        float pk = powf(r2, kap - 1.0f);
        if (isnan(pk)) pk = 0.0f;
        float r2k = r2 * pk;
        float alpha = opa1 * expf(-0.5f * kinv * r2k) * sig_y;
        float o = T * alpha;
        (*count)++;
        st->hits++;
        if (median) {
            st->med_t = t;
            st->med_idx = idx;
            T = T - o;
            continue;
        }
        for (int c = 0; c < 3; ++c) st->rgb[c] = fmaf(crgb[c], o, st->rgb[c]);
        float sgn = (fmaf(N1, v[0], fmaf(N2, v[1], N3 * v[2])) > 0.0f) ? -1.0f : 1.0f;
        if (P->mode == M_GEOM) {
            st->normal[0] = fmaf(sgn * N1, o, st->normal[0]);
            st->normal[1] = fmaf(sgn * N2, o, st->normal[1]);
            st->normal[2] = fmaf(sgn * N3, o, st->normal[2]);
            st->edn = fmaf(t, o, st->edn);
        }
        T = T - o;
        if (P->mode == M_TRAIN) {
            float tt = sat(P->reg_a / t + P->reg_b);
            float oacc = st->dacc[1], toacc = st->dacc[2];
            float Ld = o * fmaf(tt, oacc, -toacc);
            st->dacc[0] = fmaf(4.0f, Ld, st->dacc[0]);
            st->dacc[1] = oacc + o;
            st->dacc[2] = fmaf(tt, o, toacc);
            st->dacc[3] = fmaf(t, o, st->dacc[3]);
            float nd = sgn * fmaf(Nm[0], N1, fmaf(Nm[1], N2, Nm[2] * N3));
            if (nvalid) st->nacc[0] += o * (1.0f - nd);
        }
    }
    st->T = T;
    int active = last_valid && (T >= P->T_thr);
    if (P->mode == M_MEDIAN) active = active && (T > 0.5f);
    return active;
}

static void finish_ray(const oparams *P, oray *st) {
    if (P->mode == M_MEDIAN) return;
    for (int c = 0; c < 3; ++c) st->rgb[c] = fmaf(P->bg[c], st->T, st->rgb[c]);
}

/*
 * Forward over per-ray hit lists in CSR form: ray r's hits, ascending in t, are hit_t/hit_idx
 * [off[r], off[r+1]), grouped in passes of 16 (a pass that ends with fewer than 16 entries, or a
 * trailing -1, ends the ray).  Outputs (all may be NULL except rgb):
 *   rgb (R,3), dacc (R,4), nacc (R,4), normal (R,3), alpha (R), edn (R), med (R,2 floats: t, idx bits),
 *   Tout (R), nhits (R).
 * Returns the total number of composited hits.
 */
long oracle_shade_csr(const float *m, const float *s, const float *q, const float *RGBA, const float *k,
                      const void *cond, const float *features, const void *A1, const float *b1, const void *A2,
                      const float *b2, const void *A3, const float *b3, const float *override_colors, int mode,
                      const float *bg, float T_thr, float reg_a, float reg_b, const float *O, const float *v,
                      const float *surface_normal, int R, const long *off, const float *hit_t,
                      const int *hit_idx, float *rgb, float *dacc, float *nacc, float *normal, float *alpha,
                      float *edn, float *med, float *Tout, int *nhits, int decoder) {
    oscene S = {m, s, q, RGBA, k, (const _Float16 *)cond, features, (const _Float16 *)A1, (const _Float16 *)A2,
                (const _Float16 *)A3, b1, b2, b3, override_colors, decoder};
    oparams P;
    P.mode = mode;
    P.bg[0] = bg[0]; P.bg[1] = bg[1]; P.bg[2] = bg[2];
    P.T_thr = T_thr; P.reg_a = reg_a; P.reg_b = reg_b;
    long total = 0;
#pragma omp parallel for schedule(dynamic, 64) reduction(+ : total)
    for (int r = 0; r < R; ++r) {
        oray st;
        memset(&st, 0, sizeof(st));
        st.T = 1.0f;
        st.med_t = INFINITY;
        st.med_idx = -1;
        int cnt = 0;
        long b = off[r], e = off[r + 1];
        for (long p = b; p < e; p += K_HITS) {
            int nh = (int)((e - p) < K_HITS ? (e - p) : K_HITS);
            int act = shade_pass(&S, &P, O + 3 * r, v + 3 * r, hit_t + p, hit_idx + p, nh,
                                 surface_normal ? surface_normal + 3 * r : NULL, &st, &cnt);
            if (!act) break;
        }
        finish_ray(&P, &st);
        total += cnt;
        for (int c = 0; c < 3; ++c) rgb[3 * r + c] = st.rgb[c];
        if (dacc) for (int c = 0; c < 4; ++c) dacc[4 * r + c] = st.dacc[c];
        if (nacc) for (int c = 0; c < 4; ++c) nacc[4 * r + c] = st.nacc[c];
        if (normal) for (int c = 0; c < 3; ++c) normal[3 * r + c] = st.normal[c];
        if (alpha) alpha[r] = 1.0f - st.T;
        if (edn) edn[r] = st.edn;
        if (med) {
            med[2 * r] = st.med_t;
            memcpy(&med[2 * r + 1], &st.med_idx, 4);
        }
        if (Tout) Tout[r] = st.T;
        if (nhits) nhits[r] = st.hits;
    }
    return total;
}

/* The LUT encoding alone, for the golden-vector test: out (n, 8) for coordinates (cu, cw). */
void oracle_lut(const float *features, const float *cu, const float *cw, int n, float *out) {
    for (int i = 0; i < n; ++i) lut_encode(features, cu[i], cw[i], out + 8 * i);
}

/* The decoder-1 grid encoding alone: out (n, 16). */
void oracle_grid(const float *features, const float *cu, const float *cw, int n, float *out) {
    for (int i = 0; i < n; ++i) grid_encode(features, cu[i], cw[i], 8, grid_res, grid_off, out + 16 * i);
}

/* Degree-3 spherical harmonics of n directions: out (n, 16). */
void oracle_sh(const float *v, int n, float *out) {
    for (int i = 0; i < n; ++i) sh_deg3(v[3 * i], v[3 * i + 1], v[3 * i + 2], out + 16 * i);
}

/*
 * Secondary-ray compositing (viewer path, CPyOptiXFLAREVIEWERRenderer_CUDA_Forward.cu:695-897): the
 * hits of ray ray[j] are hit_t / hit_idx [off[j], off[j+1]) ascending; a shadowed hit (flag != 0)
 * contributes its colour times shadow_mult; no background.  T (by ray id) and rgb (R,3, by ray id) are
 * read and updated.  RGBA = [RGB | A logit].  Returns the number of composited hits.
 */
long oracle_viewer_composite(const float *m, const float *s, const float *q, const float *RGBA, const float *k,
                             const void *cond, const float *features, const void *A1, const float *b1, const void *A2,
                             const float *b2, const void *A3, const float *b3, float T_thr, float shadow_mult,
                             const float *O, const float *v, const int *ray, int n, const long *off,
                             const float *hit_t, const int *hit_idx, const unsigned char *shadow, float *T_io,
                             float *rgb_io, int decoder) {
    oscene S = {m, s, q, RGBA, k, (const _Float16 *)cond, features, (const _Float16 *)A1, (const _Float16 *)A2,
                (const _Float16 *)A3, b1, b2, b3, NULL, decoder};
    long total = 0;
#pragma omp parallel for schedule(dynamic, 64) reduction(+ : total)
    for (int j = 0; j < n; ++j) {
        int r = ray[j];
        float T = T_io[r];
        float rgb[3] = {rgb_io[3 * (long)r], rgb_io[3 * (long)r + 1], rgb_io[3 * (long)r + 2]};
        const float *o = O + 3 * (long)r, *d = v + 3 * (long)r;
        for (long h = off[j]; h < off[j + 1]; ++h) {
            int idx = hit_idx[h];
            if (idx < 0 || !(T >= T_thr)) break;
            float t = hit_t[h];
            const float *qq = S.q + 4 * (long)idx;
            float sx = expf(-S.s[2 * (long)idx]), sy = expf(-S.s[2 * (long)idx + 1]);
            float aa = qq[0] * qq[0], bb = qq[1] * qq[1], cc = qq[2] * qq[2], dd = qq[3] * qq[3];
            float Sq = 2.0f / (aa + bb + cc + dd);
            float bs = qq[1] * Sq, cs = qq[2] * Sq, ds = qq[3] * Sq;
            float ab = qq[0] * bs, ac = qq[0] * cs, ad = qq[0] * ds;
            bb = bb * Sq;
            float bc = qq[1] * cs, bd = qq[1] * ds;
            cc = cc * Sq;
            float cd = qq[2] * ds;
            dd = dd * Sq;
            float Q11 = sx * (1.0f - cc - dd), Q12 = sx * (bc + ad), Q13 = sx * (bd - ac);
            float Q21 = sy * (bc - ad), Q22 = sy * (1.0f - bb - dd), Q23 = sy * (cd + ab);
            float kap = 1.0f + logf(1.0f + expf(S.k[idx]));
            float kinv = 1.0f / kap;
            const float *mm = S.m + 3 * (long)idx;
            float dx = fmaf(d[0], t, o[0]) - mm[0], dy = fmaf(d[1], t, o[1]) - mm[1], dz = fmaf(d[2], t, o[2]) - mm[2];
            float u = fmaf(Q11, dx, fmaf(Q12, dy, Q13 * dz));
            float w = fmaf(Q21, dx, fmaf(Q22, dy, Q23 * dz));
            const float *rgba = S.RGBA + 4 * (long)idx;
            float sig_y = 1.0f, crgb[3] = {rgba[0], rgba[1], rgba[2]};
            if (S.cond) {
                float y[4];
                decode(&S, idx, u * LUT_SCALE, w * LUT_SCALE, d, y);
                sig_y = 1.0f / (1.0f + expf(-y[3]));
                for (int c = 0; c < 3; ++c)
                crgb[c] = rgba[c] * (S.decoder == 1 ? 1.0f / (1.0f + expf(-y[c])) : (y[c] > 0.0f ? y[c] : 0.0f));
            }
            if (shadow[h])
                for (int c = 0; c < 3; ++c) crgb[c] *= shadow_mult;
            float opa1 = 1.0f / (1.0f + expf(-rgba[3]));
            float r2 = fmaf(u, u, w * w);
            float pk = powf(r2, kap - 1.0f);
            if (isnan(pk)) pk = 0.0f;
            float alpha = opa1 * expf(-0.5f * kinv * (r2 * pk)) * sig_y;
            float oo = T * alpha;
            for (int c = 0; c < 3; ++c) rgb[c] = fmaf(crgb[c], oo, rgb[c]);
            T = T - oo;
            ++total;
        }
        T_io[r] = T;
        for (int c = 0; c < 3; ++c) rgb_io[3 * (long)r + c] = rgb[c];
    }
    return total;
}

/*
 * The whole forward of the reference on the CPU (the timed CPU baseline): per ray, passes of
 * 16-nearest queries on the CPU hierarchy (oracle_bvh_build) restarting at nextafter(t_16)
 * (Forward_training.cu:1004-1131), each shaded by shade_pass until the ray terminates.  OpenMP over
 * rays.  Outputs as oracle_shade_csr; the composited hits of ray r go to hit_t / hit_idx
 * [r * cap, r * cap + nhits[r]) (cap >= nhits or the excess is dropped from the list, not the image).
 * times[0] / times[1]: thread-seconds spent in traversal / shading.
 */
void oracle_bvh_hits_one(const void *h, int nsides, const float *pc, const float *ps, const float *O, const float *v,
                         float t_min, float *tb, int *ib);
void oracle_polygon_constants(int nsides, float *c, float *s);

long oracle_render_bvh(const void *bvh, int nsides, const float *m, const float *s, const float *q, const float *RGBA,
                       const float *k, const void *cond, const float *features, const void *A1, const float *b1,
                       const void *A2, const float *b2, const void *A3, const float *b3, int mode, const float *bg,
                       float T_thr, float reg_a, float reg_b, const float *O, const float *v, int R, int cap,
                       float *hit_t, int *hit_idx, float *rgb, float *Tout, int *nhits, double *times, int decoder) {
    oscene S = {m, s, q, RGBA, k, (const _Float16 *)cond, features, (const _Float16 *)A1, (const _Float16 *)A2,
                (const _Float16 *)A3, b1, b2, b3, NULL, decoder};
    oparams P;
    P.mode = mode;
    P.bg[0] = bg[0]; P.bg[1] = bg[1]; P.bg[2] = bg[2];
    P.T_thr = T_thr; P.reg_a = reg_a; P.reg_b = reg_b;
    float pc[64], ps[64];
    oracle_polygon_constants(nsides, pc, ps);
    long total = 0;
    double t_trace = 0.0, t_shade = 0.0;
#pragma omp parallel for schedule(dynamic, 16) reduction(+ : total, t_trace, t_shade)
    for (int r = 0; r < R; ++r) {
        oray st;
        memset(&st, 0, sizeof(st));
        st.T = 1.0f;
        st.med_t = INFINITY;
        st.med_idx = -1;
        int cnt = 0, kept = 0;
        float t_min = 0.0f;
        for (;;) {
            float tb[K_HITS];
            int ib[K_HITS];
            const double w0 = omp_get_wtime();
            oracle_bvh_hits_one(bvh, nsides, pc, ps, O + 3 * r, v + 3 * r, t_min, tb, ib);
            const double w1 = omp_get_wtime();
            const int before = st.hits;
            const int act = shade_pass(&S, &P, O + 3 * r, v + 3 * r, tb, ib, K_HITS, NULL, &st, &cnt);
            t_trace += w1 - w0;
            t_shade += omp_get_wtime() - w1;
            for (int h = 0; h < st.hits - before && kept < cap; ++h, ++kept) {
                hit_t[(long)r * cap + kept] = tb[h];
                hit_idx[(long)r * cap + kept] = ib[h];
            }
            if (!act) break;
            t_min = nextafterf(tb[K_HITS - 1], INFINITY);
        }
        finish_ray(&P, &st);
        total += cnt;
        for (int c = 0; c < 3; ++c) rgb[3 * r + c] = st.rgb[c];
        if (Tout) Tout[r] = st.T;
        nhits[r] = kept;
    }
    times[0] = t_trace;
    times[1] = t_shade;
    return total;
}
