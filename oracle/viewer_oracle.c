/*
 * viewer_oracle.c -- CPU restatement of the secondary-ray (viewer) path, analytic spheres standing in
 * for the reference viewer's triangle meshes.
 *
 * TEST INFRASTRUCTURE ONLY (checker and timed CPU baseline).  The product never links or calls it.
 *
 * Restates (reference paths in source/viewer_renderer/):
 *   - k-nearest passes that end at the nearest mesh hit              shaders.cu:545-586 (mesh any-hit)
 *   - shadow test of every buffered hit towards each light           shaders.cu:86-122 (mask 15: meshes)
 *   - compositing, colour of a shadowed hit x shadow multiplier       CPyOptiXFLAREVIEWERRenderer_CUDA_Forward.cu:876-897
 *   - shading at the mesh: Fresnel (Schlick), refraction / TIR,      shaders.cu:180-230, 234-490
 *     ambient, diffuse and specular with shadow rays, the split into
 *     the in-place and the pushed child
 * with the departures of the product (spheres hit analytically, normal (P - c) / |P - c|, IEEE
 * operations in place of the approximate rcp / sqrt / rsqrt, a ray whose T fell below the threshold
 * inside a generation ends with background * T).  The operation sequence follows the CUDA kernels
 * (flare_b200/csrc/viewer.cu) one rounding at a time (built with -ffp-contract=off), so ray
 * generations and hit lists agree bit for bit.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static float sphere_t(const float *c, const float *O, const float *v, float t_min) {
    float ox = O[0] - c[0], oy = O[1] - c[1], oz = O[2] - c[2];
    float a = fmaf(v[0], v[0], fmaf(v[1], v[1], v[2] * v[2]));
    float b = fmaf(ox, v[0], fmaf(oy, v[1], oz * v[2]));
    float cc = fmaf(ox, ox, fmaf(oy, oy, fmaf(oz, oz, -(c[3] * c[3]))));
    float disc = fmaf(b, b, -(a * cc));
    if (!(disc >= 0.0f)) return INFINITY;
    float sq = sqrtf(disc);
    float t0 = (-b - sq) / a, t1 = (-b + sq) / a;
    if (t0 > t_min) return t0;
    if (t1 > t_min) return t1;
    return INFINITY;
}

static int lit(const float *sph, int S, const float *light, const float *P, float eps) {
    float d[3] = {-light[3], -light[4], -light[5]};
    for (int s = 0; s < S; ++s)
        if (sphere_t(sph + 4 * s, P, d, eps) < INFINITY) return 0;
    return 1;
}

/* nearest sphere beyond t_min for each of R rays */
void oracle_sphere_nearest(const float *sph, int S, const float *O, const float *v, const float *tmin, int R,
                           float *t_out, int *id_out) {
    for (int r = 0; r < R; ++r) {
        float best = INFINITY;
        int id = -1;
        for (int s = 0; s < S; ++s) {
            float t = sphere_t(sph + 4 * s, O + 3 * r, v + 3 * r, tmin[r]);
            if (t < best) {
                best = t;
                id = s;
            }
        }
        t_out[r] = best;
        id_out[r] = id;
    }
}

/* shadow flag (1 = some light blocked) of H hits: hit h of ray ray[h] at t[h] */
void oracle_shadow_flags(const float *sph, int S, const float *lights, int L, float eps, const float *O,
                         const float *v, const int *ray, const float *t, long H, unsigned char *flag) {
#pragma omp parallel for schedule(static)
    for (long h = 0; h < H; ++h) {
        const float *o = O + 3 * (long)ray[h], *d = v + 3 * (long)ray[h];
        float P[3] = {fmaf(d[0], t[h], o[0]), fmaf(d[1], t[h], o[1]), fmaf(d[2], t[h], o[2])};
        unsigned char f = 0;
        for (int l = 0; l < L && !f; ++l) f = !lit(sph, S, lights + 6 * l, P, eps);
        flag[h] = f;
    }
}

static float fresnel(float cos1, float eta, float cos2) {
    float t1 = (1.0f - eta) / (1.0f + eta);
    float R0 = t1 * t1;
    float t2 = 1.0f - (eta <= 1.0f ? cos2 : cos1);
    float t3 = t2 * t2;
    t3 = t3 * t3;
    t3 = t2 * t3;
    return fmaf(1.0f - R0, t3, R0);
}

static int cos_theta2(float cos1, float n_inv, float *cos2) {
    float s2 = fmaf(-cos1, cos1, 1.0f);
    if (s2 < 0.0f) s2 = 0.0f;
    float c2 = fmaf(-(n_inv * n_inv), s2, 1.0f);
    if (c2 < 0.0f) return 1;
    *cos2 = sqrtf(c2);
    return 0;
}

static float dot3(const float *a, const float *b) { return fmaf(a[0], b[0], fmaf(a[1], b[1], a[2] * b[2])); }
static float sat(float x) { return x < 0.0f ? 0.0f : (x > 1.0f ? 1.0f : x); }

/*
 * End of a ray generation for the rays ray[0..n).  Arrays O, v, T, tmin are the generation's (indexed by
 * ray id) and receive the in-place child; pO.. receive the pushed child; act_in / act_push per list
 * position.  bitmap (R,3) indexed by ray id.
 */
void oracle_sphere_shade(const float *sph, const float *mat, int S, const float *lights, int L, float eps,
                         float shadow_unused, float T_thr, const float *Ia, const float *bg, const int *ray, int n,
                         float *O, float *v, float *T, float *tmin, const float *t_sph, const int *sph_id,
                         float *bitmap, float *pO, float *pv, float *pT, float *ptmin, unsigned char *act_in,
                         unsigned char *act_push) {
    (void)shadow_unused;
    for (int j = 0; j < n; ++j) {
        int r = ray[j];
        float T_old = T[r], ts = t_sph[r];
        float *px = bitmap + 3 * (long)r;
        if (!(T_old >= T_thr) || !(ts < INFINITY)) {
            for (int c = 0; c < 3; ++c) px[c] = fmaf(bg[c], T_old, px[c]);
            act_in[j] = 0;
            act_push[j] = 0;
            continue;
        }
        int s = sph_id[r];
        const float *o = O + 3 * (long)r, *d = v + 3 * (long)r;
        float vv[3] = {d[0], d[1], d[2]};
        float P[3] = {fmaf(d[0], ts, o[0]), fmaf(d[1], ts, o[1]), fmaf(d[2], ts, o[2])};
        float N[3] = {P[0] - sph[4 * s], P[1] - sph[4 * s + 1], P[2] - sph[4 * s + 2]};
        float ninv = 1.0f / sqrtf(dot3(N, N));
        for (int c = 0; c < 3; ++c) N[c] = N[c] * ninv;
        const float *m = mat + 6 * s;
        float kd_old = m[3], eta_old = m[4], nsh = m[5];
        float eta_old_inv = 1.0f / eta_old;
        float cos1 = dot3(N, vv);
        float c2m = -2.0f * cos1;
        float Rv[3] = {fmaf(N[0], c2m, vv[0]), fmaf(N[1], c2m, vv[1]), fmaf(N[2], c2m, vv[2])};
        float eta_inv, kd;
        if (cos1 <= 0.0f) {
            eta_inv = eta_old_inv;
            kd = kd_old;
        } else {
            eta_inv = eta_old;
            kd = 0.0f;
        }
        float cos2 = 0.0f;
        int tir = cos_theta2(cos1, eta_inv, &cos2);
        float Tv[3] = {0.0f, 0.0f, 0.0f};
        float F1 = 1.0f;
        if (!tir) {
            float tmp = fmaf(-cos1, eta_inv, copysignf(cos2, cos1));
            for (int c = 0; c < 3; ++c) Tv[c] = (vv[c] * eta_inv) + (N[c] * tmp);
            F1 = fresnel(cos1, eta_inv, cos2);
        }
        float T_R = T_old * F1;
        float T_T = (T_old * (1.0f - F1)) * (1.0f - kd);
        float col[3] = {0.0f, 0.0f, 0.0f};
        if (cos1 < 0.0f) {
            float w = (1.0f - F1) * kd_old;
            for (int c = 0; c < 3; ++c) col[c] = fmaf(m[c] * w, Ia[c], col[c]);
        }
        for (int l = 0; l < L; ++l) {
            const float *lt = lights + 6 * l;
            int is_lit = lit(sph, S, lt, P, eps);
            float Ld[3] = {lt[3], lt[4], lt[5]};
            float linv = 1.0f / sqrtf(dot3(Ld, Ld));
            for (int c = 0; c < 3; ++c) Ld[c] = Ld[c] * linv;
            float cl = dot3(N, Ld);
            float ei = cl <= 0.0f ? eta_old_inv : eta_old;
            float c2l = 0.0f;
            float F2 = cos_theta2(cl, ei, &c2l) ? 1.0f : fresnel(cl, ei, c2l);
            float diffuse = (((1.0f - F1) * (1.0f - F2)) * kd_old) * sat(-cl);
            float H[3] = {vv[0] + Ld[0], vv[1] + Ld[1], vv[2] + Ld[2]};
            float hinv = 1.0f / sqrtf(dot3(H, H));
            for (int c = 0; c < 3; ++c) H[c] = H[c] * hinv;
            float ch = sat(-dot3(N, H));
            float specular = (F2 * ch) / fmaf(nsh, 1.0f - ch, ch);
            if (!is_lit) {
                diffuse = 0.0f;
                specular = 0.0f;
            }
            for (int c = 0; c < 3; ++c) col[c] = fmaf(lt[c], fmaf(m[c], diffuse, specular), col[c]);
        }
        for (int c = 0; c < 3; ++c) px[c] = sat(fmaf(T_old, col[c], px[c]));
        int refl_first = T_T <= T_R;
        float T1 = refl_first ? T_R : T_T, T2 = refl_first ? T_T : T_R;
        const float *v1 = refl_first ? Rv : Tv, *v2 = refl_first ? Tv : Rv;
        for (int c = 0; c < 3; ++c) {
            O[3 * (long)r + c] = P[c];
            v[3 * (long)r + c] = v1[c];
            pO[3 * (long)r + c] = P[c];
            pv[3 * (long)r + c] = v2[c];
        }
        T[r] = T1;
        tmin[r] = eps;
        pT[r] = T2;
        ptmin[r] = eps;
        act_in[j] = T1 >= T_thr;
        act_push[j] = T2 >= T_thr;
    }
}
