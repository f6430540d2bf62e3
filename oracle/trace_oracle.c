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

/* ------------------------------------------------------------------------------------------------
 * CPU bounding-volume hierarchy for the timed CPU baseline (bench.py) and the large-scene oracle runs:
 * the same k-nearest query as oracle_hits, culled by a binary hierarchy over conservative primitive
 * boxes.  Culling is conservative and the hit test is the exact one above, so the hits equal the
 * brute-force search bit for bit (tests/test_oracle.py checks it).
 *
 * Build: primitives sorted by a 30-bit Morton code of their centres, then ranges split at the highest
 * differing code bit (at the middle when the codes are equal) down to leaves of at most 4 primitives;
 * boxes bottom-up.  Box of a primitive: the polygon lies in the ellipse m + a U' + b V' (a^2 + b^2 <= 1)
 * with U' = Ua / |Ua|^2, V' = Va / |Va|^2 (Ua, Va the frame's scaled in-plane axes), whose extent along
 * axis x is sqrt(U'x^2 + V'x^2); the box is padded by a relative 1e-4 and 1e-6.
 * ------------------------------------------------------------------------------------------------ */
typedef struct {
    float lo[3], hi[3];
    int left, right;   /* internal: child nodes; leaf: left = -1 - first sorted position, right = count */
} obvh_node;

typedef struct {
    int n, n_nodes;
    obvh_node *nodes;
    int *order;        /* sorted position -> primitive index */
    const float *frames;
} obvh;

static unsigned spread3(unsigned v) {
    v &= 1023u;
    v = (v | (v << 16)) & 0x030000FFu;
    v = (v | (v << 8)) & 0x0300F00Fu;
    v = (v | (v << 4)) & 0x030C30C3u;
    v = (v | (v << 2)) & 0x09249249u;
    return v;
}

typedef struct { unsigned key; int idx; } okey;
static int cmp_okey(const void *a, const void *b) {
    const okey *x = (const okey *)a, *y = (const okey *)b;
    if (x->key != y->key) return x->key < y->key ? -1 : 1;
    return (x->idx > y->idx) - (x->idx < y->idx);
}

static void prim_box(const float *f, float *lo, float *hi) {
    const float *Ua = f + 6, *Va = f + 9;
    const double uu = (double)Ua[0] * Ua[0] + (double)Ua[1] * Ua[1] + (double)Ua[2] * Ua[2];
    const double vv = (double)Va[0] * Va[0] + (double)Va[1] * Va[1] + (double)Va[2] * Va[2];
    for (int a = 0; a < 3; ++a) {
        const double up = uu > 0 ? Ua[a] / uu : 1e30, vp = vv > 0 ? Va[a] / vv : 1e30;
        double ext = sqrt(up * up + vp * vp);
        ext = ext * (1.0 + 1e-4) + 1e-6;
        lo[a] = (float)(f[a] - ext);
        hi[a] = (float)(f[a] + ext);
        if (!(lo[a] <= hi[a])) { lo[a] = -INFINITY; hi[a] = INFINITY; }  /* degenerate frame: never culled */
    }
}

static int build_range(obvh *b, const okey *keys, int first, int last, const float *pbox) {
    const int id = b->n_nodes++;
    obvh_node *nd = &b->nodes[id];
    if (last - first + 1 <= 4) {
        nd->left = -1 - first;
        nd->right = last - first + 1;
        for (int a = 0; a < 3; ++a) { nd->lo[a] = INFINITY; nd->hi[a] = -INFINITY; }
        for (int p = first; p <= last; ++p)
            for (int a = 0; a < 3; ++a) {
                const float *bx = pbox + 6 * (size_t)keys[p].idx;
                if (bx[a] < nd->lo[a]) nd->lo[a] = bx[a];
                if (bx[3 + a] > nd->hi[a]) nd->hi[a] = bx[3 + a];
            }
        return id;
    }
    int split = (first + last) / 2;
    const unsigned kf = keys[first].key, kl = keys[last].key;
    if (kf != kl) {
        const int bit = 31 - __builtin_clz(kf ^ kl);
        int lo = first, hi = last;  /* last position whose key has that bit clear */
        while (lo < hi) {
            const int mid = (lo + hi + 1) / 2;
            if ((keys[mid].key >> bit) & 1u) hi = mid - 1; else lo = mid;
        }
        split = lo;
    }
    const int l = build_range(b, keys, first, split, pbox);
    const int r = build_range(b, keys, split + 1, last, pbox);
    nd = &b->nodes[id];
    nd->left = l;
    nd->right = r;
    for (int a = 0; a < 3; ++a) {
        nd->lo[a] = fminf(b->nodes[l].lo[a], b->nodes[r].lo[a]);
        nd->hi[a] = fmaxf(b->nodes[l].hi[a], b->nodes[r].hi[a]);
    }
    return id;
}

void *oracle_bvh_build(const float *frames, int n) {
    obvh *b = (obvh *)calloc(1, sizeof(obvh));
    b->n = n;
    b->frames = frames;
    if (n == 0) return b;
    float *pbox = (float *)malloc(sizeof(float) * 6 * (size_t)n);
    float clo[3] = {INFINITY, INFINITY, INFINITY}, chi[3] = {-INFINITY, -INFINITY, -INFINITY};
#pragma omp parallel for schedule(static)
    for (int i = 0; i < n; ++i) prim_box(frames + 12 * (size_t)i, pbox + 6 * (size_t)i, pbox + 6 * (size_t)i + 3);
    for (int i = 0; i < n; ++i)
        for (int a = 0; a < 3; ++a) {
            const float c = frames[12 * (size_t)i + a];
            if (c < clo[a]) clo[a] = c;
            if (c > chi[a]) chi[a] = c;
        }
    okey *keys = (okey *)malloc(sizeof(okey) * (size_t)n);
#pragma omp parallel for schedule(static)
    for (int i = 0; i < n; ++i) {
        unsigned code = 0;
        for (int a = 0; a < 3; ++a) {
            const float ext = chi[a] - clo[a];
            float x = ext > 0 ? (frames[12 * (size_t)i + a] - clo[a]) / ext : 0.5f;
            int q = (int)(x * 1023.0f);
            q = q < 0 ? 0 : (q > 1023 ? 1023 : q);
            code |= spread3((unsigned)q) << (2 - a);
        }
        keys[i].key = code;
        keys[i].idx = i;
    }
    qsort(keys, n, sizeof(okey), cmp_okey);
    b->nodes = (obvh_node *)malloc(sizeof(obvh_node) * (size_t)(2 * n + 1));
    b->order = (int *)malloc(sizeof(int) * (size_t)n);
    for (int i = 0; i < n; ++i) b->order[i] = keys[i].idx;
    build_range(b, keys, 0, n - 1, pbox);
    free(keys);
    free(pbox);
    return b;
}

void oracle_bvh_free(void *h) {
    obvh *b = (obvh *)h;
    if (!b) return;
    free(b->nodes);
    free(b->order);
    free(b);
}

static inline int box_hit(const obvh_node *nd, const float *O, const float *iv, float tlo, float thi, float *tn) {
    float t0 = tlo, t1 = thi;
    for (int a = 0; a < 3; ++a) {
        float ta = (nd->lo[a] - O[a]) * iv[a], tb = (nd->hi[a] - O[a]) * iv[a];
        if (ta > tb) { float x = ta; ta = tb; tb = x; }
        if (ta > t0) t0 = ta;
        if (tb < t1) t1 = tb;
    }
    *tn = t0;
    return t0 <= t1;
}

/* The K_HITS nearest hits of one ray at or beyond t_min (slot order, +inf / -1 padding). */
static void bvh_hits16(const obvh *b, int nsides, const float *pc, const float *ps, const float *O, const float *v,
                       float t_min, float *tb, int *ib) {
    for (int k = 0; k < K_HITS; ++k) { tb[k] = INFINITY; ib[k] = 0x7fffffff; }
    if (b->n == 0 || !(t_min < INFINITY)) goto out;
    {
        float iv[3];
        for (int a = 0; a < 3; ++a) iv[a] = 1.0f / (fabsf(v[a]) > 1e-30f ? v[a] : copysignf(1e-30f, v[a]));
        const float tlo = t_min - fabsf(t_min) * 1e-5f;
        int stack[256], sp = 0;
        stack[sp++] = 0;
        while (sp) {
            const obvh_node *nd = &b->nodes[stack[--sp]];
            const float bk = tb[K_HITS - 1];
            float tn;
            if (!box_hit(nd, O, iv, tlo, bk + fabsf(bk) * 1e-5f, &tn)) continue;
            if (nd->left < 0) {
                const int first = -1 - nd->left;
                for (int p = first; p < first + nd->right; ++p) {
                    const int i = b->order[p];
                    float t;
                    if (hit_test(b->frames + 12 * (size_t)i, O, v, t_min, nsides, pc, ps, &t)) kbuf_push(tb, ib, t, i);
                }
                continue;
            }
            float tl, tr;
            const int hl = box_hit(&b->nodes[nd->left], O, iv, tlo, bk + fabsf(bk) * 1e-5f, &tl);
            const int hr = box_hit(&b->nodes[nd->right], O, iv, tlo, bk + fabsf(bk) * 1e-5f, &tr);
            if (sp + 2 > 256) continue;  /* cannot happen: depth <= 2 * 32 code bits + leaf levels */
            if (hl && hr) {
                if (tl <= tr) { stack[sp++] = nd->right; stack[sp++] = nd->left; }
                else { stack[sp++] = nd->left; stack[sp++] = nd->right; }
            } else if (hl) stack[sp++] = nd->left;
            else if (hr) stack[sp++] = nd->right;
        }
    }
out:
    for (int k = 0; k < K_HITS; ++k)
        if (ib[k] == 0x7fffffff) { tb[k] = INFINITY; ib[k] = -1; }
}

/* One ray's 16-nearest query for the CPU renderer in decode_oracle.c. */
void oracle_bvh_hits_one(const void *h, int nsides, const float *pc, const float *ps, const float *O, const float *v,
                         float t_min, float *tb, int *ib) {
    bvh_hits16((const obvh *)h, nsides, pc, ps, O, v, t_min, tb, ib);
}

void oracle_bvh_hits(const void *h, const float *O, const float *v, const float *t_min, int R, int nsides,
                     float *t_out, int *idx_out) {
    const obvh *b = (const obvh *)h;
    float pc[64], ps[64];
    oracle_polygon_constants(nsides, pc, ps);
#pragma omp parallel for schedule(dynamic, 16)
    for (int r = 0; r < R; ++r) {
        float tb[K_HITS];
        int ib[K_HITS];
        bvh_hits16(b, nsides, pc, ps, O + 3 * r, v + 3 * r, t_min[r], tb, ib);
        for (int k = 0; k < K_HITS; ++k) {
            t_out[(long)k * R + r] = tb[k];
            idx_out[(long)k * R + r] = ib[k];
        }
    }
}
