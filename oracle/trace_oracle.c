/*
 * trace_oracle.c -- CPU restatement of the FlaRe proxy geometry and k-nearest hit search.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (flare_b200/) links, loads or calls this file;
 * only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg use it, as the checker.
 *
 * What it restates (reference paths relative to the FlaRe repository):
 *   - proxy radius and frame per primitive: source/renderer/CPyOptiXFLARERenderer_CUDA_Core.cu:553-622
 *     (quaternion -> rotation with S = 2/|q|^2, rho = max(0, kappa*(11.3449 + 2 ln sigma))^(1/(2 kappa)),
 *     columns [U e^sx rho, V e^sy rho, N, m]);
 *   - the proxy polygon: Core.cu:322-339 (n vertices on the unit circle at angles 2 pi j / n);
 *   - the k-buffer: source/renderer/shaders.cu:145-189 (16 smallest t, sorted ascending) and the raygen
 *     writes of shaders.cu:63-76 (slot-major (16,R), padding +inf / -1).
 *   - the pass restart t_min = nextafter(t_16, +inf): CPyOptiXFLARERenderer_CUDA_Forward_training.cu:929.
 *
 * The hit test itself is defined by this build (OptiX's triangle intersector is closed and not
 * available): a ray hits primitive i at t = N.(m-O) / N.v when t >= t_min and the hit point lies inside
 * the polygon in the primitive's scaled (a, b) frame.  The exact fp32 operation sequence below is the
 * one the CUDA traversal kernel executes (fmaf, then correctly rounded * / + -), so hit lists are
 * bit-identical given identical frames.  Ties in t are broken by the smaller primitive index.
 *
 * Build: see oracle/Makefile (-O2 -ffp-contract=off, no fast-math).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <stdlib.h>
#include <omp.h>

#define K_HITS 16

/* Edge half-plane constants of the regular n-gon with a vertex at angle 0 and circumradius 1:
   inside <=> fmaf(c_j, a, s_j * b) <= 1 for every edge j (normal angle (2j+1) pi / n, divided by the
   apothem cos(pi / n)).  Computed in double and rounded once. */
void oracle_polygon_constants(int nsides, float *c, float *s) {
    double ap = cos(M_PI / nsides);
    for (int j = 0; j < nsides; ++j) {
        double phi = (2.0 * j + 1.0) * M_PI / nsides;
        c[j] = (float)(cos(phi) / ap);
        s[j] = (float)(sin(phi) / ap);
    }
}

/* Frame of each primitive from the activated SetGeometry inputs (Core.cu:553-622).
   frames (n,12) = [m.xyz, N.xyz, U/(sx rho), V/(sy rho)] with sx = scale.x, sy = scale.y. */
void oracle_prep_frames(const float *m, const float *scale, const float *q, const float *opacity,
                        const float *kappa, int n, float *frames) {
    for (int i = 0; i < n; ++i) {
        float qa = q[4 * i + 0], qb = q[4 * i + 1], qc = q[4 * i + 2], qd = q[4 * i + 3];
        float aa = qa * qa, bb = qb * qb, cc = qc * qc, dd = qd * qd;
        float S = 2.0f / (aa + bb + cc + dd);
        float bs = qb * S, cs = qc * S, ds = qd * S;
        float ab = qa * bs, ac = qa * cs, ad = qa * ds;
        bb = bb * S;
        float bc = qb * cs, bd = qb * ds;
        cc = cc * S;
        float cd = qc * ds;
        dd = dd * S;
        float kap = kappa[i];
        float power = kap * (11.3449f + 2.0f * logf(opacity[i]));
        if (power < 0.0f) power = 0.0f;
        float rho = powf(power, 1.0f / (2.0f * kap));
        float sx = scale[2 * i + 0] * rho, sy = scale[2 * i + 1] * rho;
        float Ux = 1.0f - cc - dd, Uy = bc + ad, Uz = bd - ac;
        float Vx = bc - ad, Vy = 1.0f - bb - dd, Vz = cd + ab;
        float Nx = bd + ac, Ny = cd - ab, Nz = 1.0f - bb - cc;
        float *f = frames + 12 * i;
        f[0] = m[3 * i + 0]; f[1] = m[3 * i + 1]; f[2] = m[3 * i + 2];
        f[3] = Nx; f[4] = Ny; f[5] = Nz;
        f[6] = Ux / sx; f[7] = Uy / sx; f[8] = Uz / sx;
        f[9] = Vx / sy; f[10] = Vy / sy; f[11] = Vz / sy;
    }
}

/* Exact hit test.  Returns 1 and writes *t_out when the ray (O, v) hits the polygon of frame f at
   t >= t_min. */
static inline int hit_test(const float *f, const float *O, const float *v, float t_min, int nsides,
                           const float *pc, const float *ps, float *t_out) {
    float dx = f[0] - O[0], dy = f[1] - O[1], dz = f[2] - O[2];
    float num = fmaf(f[3], dx, fmaf(f[4], dy, f[5] * dz));
    float den = fmaf(f[3], v[0], fmaf(f[4], v[1], f[5] * v[2]));
    float t = num / den;
    if (!(t >= t_min)) return 0;
    float ex = fmaf(v[0], t, O[0]) - f[0];
    float ey = fmaf(v[1], t, O[1]) - f[1];
    float ez = fmaf(v[2], t, O[2]) - f[2];
    float a = fmaf(f[6], ex, fmaf(f[7], ey, f[8] * ez));
    float b = fmaf(f[9], ex, fmaf(f[10], ey, f[11] * ez));
    for (int j = 0; j < nsides; ++j)
        if (!(fmaf(pc[j], a, ps[j] * b) <= 1.0f)) return 0;
    *t_out = t;
    return 1;
}

/* Brute-force k-nearest: for each ray r, the K_HITS smallest (t, idx) with t >= t_min[r].
   t_out / idx_out are slot-major (K_HITS, R).  Optionally returns the count of hits found. */
static void kbuf_push(float *tb, int *ib, float t, int i) {
    if (!(t < tb[K_HITS - 1] || (t == tb[K_HITS - 1] && i < ib[K_HITS - 1]))) return;
    float ct = t;
    int ci = i;
    for (int k = 0; k < K_HITS; ++k) {
        int sw = (ct < tb[k]) || (ct == tb[k] && ci < ib[k]);
        if (sw) {
            float tt = tb[k]; int ii = ib[k];
            tb[k] = ct; ib[k] = ci;
            ct = tt; ci = ii;
        }
    }
}

/* Few rays: the primitives are split over the threads, each keeps its own buffer, the buffers merge. */
static void oracle_hits_few(const float *frames, int n, const float *O, const float *v, const float *t_min, int R,
                            int nsides, const float *pc, const float *ps, float *t_out, int *idx_out) {
    for (int r = 0; r < R; ++r) {
        float tb[K_HITS];
        int ib[K_HITS];
        for (int k = 0; k < K_HITS; ++k) { tb[k] = INFINITY; ib[k] = 0x7fffffff; }
        const float *o = O + 3 * r, *d = v + 3 * r;
#pragma omp parallel
        {
            float lt[K_HITS];
            int li[K_HITS];
            for (int k = 0; k < K_HITS; ++k) { lt[k] = INFINITY; li[k] = 0x7fffffff; }
#pragma omp for schedule(static)
            for (int i = 0; i < n; ++i) {
                float t;
                if (hit_test(frames + 12 * (long)i, o, d, t_min[r], nsides, pc, ps, &t)) kbuf_push(lt, li, t, i);
            }
#pragma omp critical
            for (int k = 0; k < K_HITS; ++k)
                if (li[k] != 0x7fffffff) kbuf_push(tb, ib, lt[k], li[k]);
        }
        for (int k = 0; k < K_HITS; ++k) {
            int valid = ib[k] != 0x7fffffff;
            t_out[(long)k * R + r] = valid ? tb[k] : INFINITY;
            idx_out[(long)k * R + r] = valid ? ib[k] : -1;
        }
    }
}

void oracle_hits(const float *frames, int n, const float *O, const float *v, const float *t_min, int R,
                 int nsides, float *t_out, int *idx_out) {
    float pc[64], ps[64];
    oracle_polygon_constants(nsides, pc, ps);
    if (R < 64 && n > 4096) {
        oracle_hits_few(frames, n, O, v, t_min, R, nsides, pc, ps, t_out, idx_out);
        return;
    }
#pragma omp parallel for schedule(dynamic, 16)
    for (int r = 0; r < R; ++r) {
        float tb[K_HITS];
        int ib[K_HITS];
        for (int k = 0; k < K_HITS; ++k) { tb[k] = INFINITY; ib[k] = 0x7fffffff; }
        const float *o = O + 3 * r, *d = v + 3 * r;
        for (int i = 0; i < n; ++i) {
            float t;
            if (!hit_test(frames + 12 * (long)i, o, d, t_min[r], nsides, pc, ps, &t)) continue;
            if (!(t < tb[K_HITS - 1] || (t == tb[K_HITS - 1] && i < ib[K_HITS - 1]))) continue;
            float ct = t;
            int ci = i;
            for (int k = 0; k < K_HITS; ++k) {
                int sw = (ct < tb[k]) || (ct == tb[k] && ci < ib[k]);
                if (sw) {
                    float tt = tb[k]; int ii = ib[k];
                    tb[k] = ct; ib[k] = ci;
                    ct = tt; ci = ii;
                }
            }
        }
        for (int k = 0; k < K_HITS; ++k) {
            int valid = ib[k] != 0x7fffffff;
            t_out[(long)k * R + r] = valid ? tb[k] : INFINITY;
            idx_out[(long)k * R + r] = valid ? ib[k] : -1;
        }
    }
}

/* Next-pass restart value used by the multi-pass driver (Forward_training.cu:929). */
float oracle_next_tmin(float t16) { return nextafterf(t16, INFINITY); }

/* As oracle_hits, with each ray's hits restricted to t < t_max[r] (the viewer path's nearest sphere). */
void oracle_hits_tmax(const float *frames, int n, const float *O, const float *v, const float *t_min,
                      const float *t_max, int R, int nsides, float *t_out, int *idx_out) {
    float pc[64], ps[64];
    oracle_polygon_constants(nsides, pc, ps);
#pragma omp parallel for schedule(dynamic, 16)
    for (int r = 0; r < R; ++r) {
        float tb[K_HITS];
        int ib[K_HITS];
        for (int k = 0; k < K_HITS; ++k) { tb[k] = INFINITY; ib[k] = 0x7fffffff; }
        const float *o = O + 3 * r, *d = v + 3 * r;
        for (int i = 0; i < n; ++i) {
            float t;
            if (!hit_test(frames + 12 * (long)i, o, d, t_min[r], nsides, pc, ps, &t)) continue;
            if (!(t < t_max[r])) continue;
            kbuf_push(tb, ib, t, i);
        }
        for (int k = 0; k < K_HITS; ++k) {
            int valid = ib[k] != 0x7fffffff;
            t_out[(long)k * R + r] = valid ? tb[k] : INFINITY;
            idx_out[(long)k * R + r] = valid ? ib[k] : -1;
        }
    }
}

/* Every hit of each ray with t >= t_min[r], ascending by (t, index): the whole sequence the multi-pass
   k-buffer restarts walk through (shaders.cu:166-188 per pass, Forward_training.cu:929 between passes),
   found in one brute-force sweep per ray for the full-size parity tests (a few hundred rays).  Ray r's
   hits go to t_out / idx_out [r * cap, r * cap + counts[r]); returns the largest count, which exceeds
   cap (and truncates that ray's list) when cap was too small. */
static int cmp_hit(const void *pa, const void *pb) {
    const float ta = ((const float *)pa)[0], tb = ((const float *)pb)[0];
    if (ta < tb) return -1;
    if (ta > tb) return 1;
    const int ia = ((const int *)pa)[1], ib = ((const int *)pb)[1];
    return (ia > ib) - (ia < ib);
}

int oracle_all_hits(const float *frames, int n, const float *O, const float *v, const float *t_min, int R,
                    int nsides, int cap, int *counts, float *t_out, int *idx_out) {
    float pc[64], ps[64];
    oracle_polygon_constants(nsides, pc, ps);
    const int nthr = omp_get_max_threads() < 64 ? omp_get_max_threads() : 64;
    const size_t slice = (size_t)2 * cap;  /* floats per thread slice: (t, index bits) pairs */
    float *buf = (float *)malloc(sizeof(float) * slice * nthr);
    float *all = (float *)malloc(sizeof(float) * slice * nthr);
    int worst = 0;
    /* few rays, many primitives: the primitives are split over the threads, each appends to its own
       slice; the slices are concatenated and sorted */
    for (int r = 0; r < R; ++r) {
        const float *o = O + 3 * r, *d = v + 3 * r;
        int cnt_thr[64] = {0};
#pragma omp parallel num_threads(nthr)
        {
            const int tid = omp_get_thread_num();
            float *mine = buf + slice * tid;
            int c = 0;
#pragma omp for schedule(static)
            for (int i = 0; i < n; ++i) {
                float t;
                if (hit_test(frames + 12 * (long)i, o, d, t_min[r], nsides, pc, ps, &t)) {
                    if (c < cap) {
                        mine[2 * c] = t;
                        memcpy(mine + 2 * c + 1, &i, sizeof(int));
                    }
                    ++c;
                }
            }
            cnt_thr[tid] = c;
        }
        int total = 0, kept = 0;
        for (int th = 0; th < nthr; ++th) {
            const int c = cnt_thr[th] < cap ? cnt_thr[th] : cap;
            memcpy(all + 2 * (size_t)kept, buf + slice * th, sizeof(float) * 2 * c);
            kept += c;
            total += cnt_thr[th];
        }
        qsort(all, kept, 2 * sizeof(float), cmp_hit);
        const int keep = kept < cap ? kept : cap;
        for (int k = 0; k < keep; ++k) {
            t_out[(long)r * cap + k] = all[2 * k];
            memcpy(idx_out + (long)r * cap + k, all + 2 * k + 1, sizeof(int));
        }
        counts[r] = keep;
        if (total > worst) worst = total;
    }
    free(all);
    free(buf);
    return worst;
}
