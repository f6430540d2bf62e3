// api.cu -- the extern "C" entry points of include/flare_b200.h: renderer lifetime, argument checks,
// error reporting, GenerateRays, and dispatch into bvh.cu / trace.cu / shade.cu.
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "renderer.cuh"

namespace flare {

static thread_local char g_err[1024] = "";

void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

int check_status(flare_renderer *r, cudaStream_t st, const char *what) {
    int h = 0;
    FLARE_CUDA_TRY(cudaMemcpyAsync(&h, r->dstatus, sizeof(int), cudaMemcpyDeviceToHost, st));
    FLARE_CUDA_TRY(cudaStreamSynchronize(st));
    if (h) {
        FLARE_CUDA_TRY(cudaMemsetAsync(r->dstatus, 0, sizeof(int), st));
        set_error("%s: device reported error bits 0x%x (%s%s%s)", what, h, (h & ERR_STACK) ? "traversal stack overflow " : "",
                  (h & ERR_MBAR) ? "tensor-core wait timeout " : "", (h & ERR_INDEX) ? "index out of range" : "");
        return FLARE_E_DEVICE;
    }
    return FLARE_OK;
}

int prof_begin(flare_renderer *r, int kind, cudaStream_t st) {
    if (!r->prof_on) return -1;
    if (r->prof_n >= flare_renderer::PROF_SLOTS) {
        cudaStreamSynchronize(st);
        prof_collect(r);
    }
    int slot = r->prof_n++;
    r->prof_kind[slot] = kind;
    cudaEventRecord(r->prof_ev[2 * slot], st);
    return slot;
}

void prof_end(flare_renderer *r, int slot, cudaStream_t st) {
    if (slot < 0) return;
    cudaEventRecord(r->prof_ev[2 * slot + 1], st);
}

void prof_collect(flare_renderer *r) {
    for (int i = 0; i < r->prof_n; ++i) {
        float ms = 0.0f;
        if (cudaEventElapsedTime(&ms, r->prof_ev[2 * i], r->prof_ev[2 * i + 1]) == cudaSuccess) {
            r->prof_ms[r->prof_kind[i]] += ms;
            r->prof_launches[r->prof_kind[i]] += 1;
        }
    }
    r->prof_n = 0;
}

int selftest_mlp(const void *X, int rows, const void *A1, const float *b1, const void *A2, const float *b2,
                 const void *A3, const float *b3, float *Y, cudaStream_t st, int *status);

// GenerateRays (reference GenerateRays.cu:6-39): v = R (a_x x + b_x) + D (a_y y + b_y) + F
__global__ void generate_rays_kernel(const float *Rp, const float *Dp, const float *Fp, int width, int height,
                                     float ttx, float tty, float *out) {
    int tid = blockIdx.x * blockDim.x + threadIdx.x;
    if (tid >= width * height) return;
    float3 R = make_float3(Rp[0], Rp[1], Rp[2]), D = make_float3(Dp[0], Dp[1], Dp[2]), F = make_float3(Fp[0], Fp[1], Fp[2]);
    int x = tid % width, y = tid / width;
    float a_x = ttx / width, b_x = 0.5f * ttx * ((1.0f / width) - 1.0f);
    float a_y = tty / height, b_y = 0.5f * tty * ((1.0f / height) - 1.0f);
    float dx = __fmaf_rn(a_x, (float)x, b_x), dy = __fmaf_rn(a_y, (float)y, b_y);
    out[3 * (size_t)tid + 0] = __fmaf_rn(R.x, dx, __fmaf_rn(D.x, dy, F.x));
    out[3 * (size_t)tid + 1] = __fmaf_rn(R.y, dx, __fmaf_rn(D.y, dy, F.y));
    out[3 * (size_t)tid + 2] = __fmaf_rn(R.z, dx, __fmaf_rn(D.z, dy, F.z));
}

}  // namespace flare

using namespace flare;

#define CHECK_ARG(cond, ...)          \
    do {                              \
        if (!(cond)) {                \
            set_error(__VA_ARGS__);   \
            return FLARE_E_INVALID;   \
        }                             \
    } while (0)

static inline cudaStream_t S(void *s) { return reinterpret_cast<cudaStream_t>(s); }

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

extern "C" {

const char *flare_last_error(void) { return g_err; }
const char *flare_version(void) { return "flare_b200 0.1 (sm_100a)"; }

int flare_create(int number_of_sides, float chi_square_squared_radius, int max_batch_size, int device,
                 flare_renderer **out) {
    g_err[0] = 0;
    CHECK_ARG(out, "flare_create: out is NULL");
    CHECK_ARG(number_of_sides >= 3 && number_of_sides <= MAX_SIDES, "flare_create: number_of_sides %d not in [3, %d]",
              number_of_sides, MAX_SIDES);
    CHECK_ARG(max_batch_size >= 0, "flare_create: max_batch_size %d < 0", max_batch_size);
    *out = nullptr;
    int ndev = 0;
    FLARE_CUDA_TRY(cudaGetDeviceCount(&ndev));
    CHECK_ARG(device >= 0 && device < ndev, "flare_create: device %d not in [0, %d)", device, ndev);
    DeviceGuard dg(device);
    flare_renderer *r = new flare_renderer();
    r->device = device;
    r->nsides = number_of_sides;
    r->chi2 = chi_square_squared_radius;
    r->max_rays = max_batch_size;
    cudaDeviceGetAttribute(&r->num_sms, cudaDevAttrMultiProcessorCount, device);
    r->poly.n = number_of_sides;
    {
        const double ap = std::cos(M_PI / number_of_sides);
        for (int j = 0; j < number_of_sides; ++j) {
            const double phi = (2.0 * j + 1.0) * M_PI / number_of_sides;
            r->poly.c[j] = (float)(std::cos(phi) / ap);
            r->poly.s[j] = (float)(std::sin(phi) / ap);
        }
        // fmaf(-c, a, (-s) * b) == -fmaf(c, a, s * b) exactly, so opposite edges fold into one |.| test
        // whenever the rounded constants are exactly antisymmetric
        bool sym = number_of_sides % 2 == 0;
        for (int j = 0; sym && j < number_of_sides / 2; ++j)
            sym = r->poly.c[j + number_of_sides / 2] == -r->poly.c[j] && r->poly.s[j + number_of_sides / 2] == -r->poly.s[j];
        r->poly.half = sym ? number_of_sides / 2 : 0;
    }
    size_t R = (size_t)(max_batch_size > 0 ? max_batch_size : 1);
    cudaError_t e = cudaSuccess;
#define ALLOC(p, bytes) \
    if (e == cudaSuccess) e = cudaMalloc(&(p), (bytes))
    ALLOC(r->t_min, R * sizeof(float));
    ALLOC(r->hint, R * sizeof(float));
    ALLOC(r->chunk_tk, (R / 256 + 2) * sizeof(float));
    ALLOC(r->T, R * sizeof(float));
    ALLOC(r->list[0], R * sizeof(int));
    ALLOC(r->list[1], R * sizeof(int));
    ALLOC(r->hit_t, R * K_PASS * sizeof(float));
    ALLOC(r->hit_idx, R * K_PASS * sizeof(int));
    ALLOC(r->counters, 64 * sizeof(int));
    ALLOC(r->dw, 16384 * sizeof(float));
    ALLOC(r->gscale, 64);
    ALLOC(r->hc_sum, 64);
    ALLOC(r->dfeat_priv, (size_t)r->num_sms * 2 * LUT_PRIV_FLOATS * sizeof(float));
    ALLOC(r->bounds, 128);
    ALLOC(r->ray_keys, 2 * R * sizeof(unsigned long long));
    ALLOC(r->ray_ids_tmp, R * sizeof(int));
    if (e == cudaSuccess) {
        r->ray_sort_tmp_bytes = ray_sort_temp_bytes((int)R);
        e = cudaMalloc(&r->ray_sort_tmp, r->ray_sort_tmp_bytes);
    }
    ALLOC(r->pass_flags, R);
    if (e == cudaSuccess) {
        r->select_tmp_bytes = select_temp_bytes((int)R);
        e = cudaMalloc(&r->select_tmp, r->select_tmp_bytes);
    }
    ALLOC(r->dstatus, 64);
    ALLOC(r->dstats, ST_NSTATS * sizeof(unsigned long long));
#undef ALLOC
    if (e == cudaSuccess) e = cudaMallocHost(&r->h_count, 64);
    if (e == cudaSuccess) e = cudaMemset(r->dstatus, 0, 64);
    if (e == cudaSuccess) e = cudaMemset(r->dstats, 0, ST_NSTATS * sizeof(unsigned long long));
    if (e != cudaSuccess) {
        set_error("flare_create: %s", cudaGetErrorString(e));
        flare_destroy(r);
        return FLARE_E_CUDA;
    }
    *out = r;
    return FLARE_OK;
}

int flare_destroy(flare_renderer *r) {
    if (!r) return FLARE_OK;
    DeviceGuard dg(r->device);
    for (int i = 0; i < 2 * flare_renderer::PROF_SLOTS; ++i)
        if (r->prof_ev[i]) cudaEventDestroy(r->prof_ev[i]);
    void *ptrs[] = {r->frames, r->rec, r->aabb, r->morton, r->morton_sorted, r->ids, r->ids_sorted, r->nodes,
                    r->parent, r->refit_flag, r->bounds, r->sort_tmp, r->t_min, r->hint, r->chunk_tk, r->T, r->list[0], r->list[1],
                    r->hit_t, r->hit_idx, r->ray_aux, r->counters, r->dfeat_priv, r->pgrad, r->vw_buf, r->ray_keys, r->ray_ids_tmp, r->ray_sort_tmp, r->pass_flags, r->select_tmp, r->dw, r->gscale, r->hc_sum, r->hc_list, r->hc_t, r->hc_idx, r->dstatus, r->dstats,
                    r->ploc_scratch, r->nodes4, r->bvh4_scratch, r->nodesL};
    for (void *p : ptrs)
        if (p) cudaFree(p);
    if (r->h_count) cudaFreeHost(r->h_count);
    delete r;
    return FLARE_OK;
}

int flare_set_geometry(flare_renderer *r, const float *m, const float *scale, const float *q, const float *opacity,
                       const float *kappa, int n, void *stream) {
    g_err[0] = 0;
    CHECK_ARG(r, "flare_set_geometry: renderer is NULL");
    CHECK_ARG(n >= 0, "flare_set_geometry: n = %d < 0", n);
    CHECK_ARG(n == 0 || (m && scale && q && opacity && kappa), "flare_set_geometry: NULL tensor");
    CHECK_ARG(((reinterpret_cast<uintptr_t>(q) & 15) | (reinterpret_cast<uintptr_t>(scale) & 7)) == 0,
              "flare_set_geometry: q must be 16-byte aligned and scale 8-byte aligned");
    DeviceGuard dg(r->device);
    int slot = prof_begin(r, PK_BUILD, S(stream));
    ++r->geom_version;
    r->hc_valid = false;
    int e = build_geometry(r, m, scale, q, opacity, kappa, n, S(stream));
    prof_end(r, slot, S(stream));
    if (e) return e;
    e = check_status(r, S(stream), "flare_set_geometry");
    prof_collect(r);
    return e;
}

int flare_render_hits(flare_renderer *r, const float *O, const float *v, const float *t_min, int n_rays, float *t_out,
                      int *idx_out, void *stream) {
    g_err[0] = 0;
    CHECK_ARG(r, "flare_render_hits: renderer is NULL");
    CHECK_ARG(n_rays >= 0, "flare_render_hits: n_rays < 0");
    if (n_rays == 0) return FLARE_OK;
    CHECK_ARG(O && v && t_min && t_out && idx_out, "flare_render_hits: NULL tensor");
    DeviceGuard dg(r->device);
    int e = launch_trace(r, O, v, t_min, nullptr, n_rays, t_out, idx_out, n_rays, S(stream));
    if (e) return e;
    return check_status(r, S(stream), "flare_render_hits");
}

int flare_generate_rays(const float *R, const float *D, const float *F, int width, int height, float fov_x, float fov_y,
                        float *out, void *stream) {
    g_err[0] = 0;
    CHECK_ARG(R && D && F && out, "flare_generate_rays: NULL tensor");
    CHECK_ARG(width > 0 && height > 0, "flare_generate_rays: bad size %dx%d", width, height);
    float ttx = 2.0f * tanf(0.5f * fov_x), tty = 2.0f * tanf(0.5f * fov_y);
    int n = width * height;
    generate_rays_kernel<<<(n + 63) / 64, 64, 0, S(stream)>>>(R, D, F, width, height, ttx, tty, out);
    FLARE_CUDA_TRY(cudaGetLastError());
    return FLARE_OK;
}

static int check_scene(flare_renderer *r, const flare_scene *sc, const char *who) {
    CHECK_ARG(sc, "%s: scene is NULL", who);
    CHECK_ARG(sc->n == r->n, "%s: scene has %d primitives but the last SetGeometry had %d", who, sc->n, r->n);
    CHECK_ARG(sc->n == 0 || (sc->m && sc->s && sc->q && sc->RGBA && sc->k), "%s: NULL primitive tensor", who);
    CHECK_ARG(sc->decoder == FLARE_DECODER_LUT_PE || sc->decoder == FLARE_DECODER_GRID_SH,
              "%s: unknown decoder kind %d", who, sc->decoder);
    if (sc->cond)
        CHECK_ARG(sc->features && sc->A1 && sc->A2 && sc->A3 && sc->b1 && sc->b2 && sc->b3,
                  "%s: decoder tensors missing", who);
    // the kernels read q and RGBA as float4, s and the LUT as float2, the descriptor and weights in
    // 16-byte chunks (as the reference's casts do)
    auto al = [](const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; };
    CHECK_ARG(al(sc->q, 16) && al(sc->RGBA, 16) && al(sc->s, 8), "%s: q and RGBA must be 16-byte aligned, s 8-byte",
              who);
    if (sc->cond)
        CHECK_ARG(al(sc->cond, 16) && al(sc->A1, 16) && al(sc->A2, 16) && al(sc->A3, 16) && al(sc->features, 8),
                  "%s: descriptor and weights must be 16-byte aligned, features 8-byte", who);
    return FLARE_OK;
}

int flare_forward(flare_renderer *r, const flare_scene *sc, const flare_forward_args *a, void *stream) {
    g_err[0] = 0;
    CHECK_ARG(r && a, "flare_forward: NULL argument");
    int e = check_scene(r, sc, "flare_forward");
    if (e) return e;
    CHECK_ARG(a->n_rays >= 0 && a->n_rays <= r->max_rays, "flare_forward: n_rays %d exceeds max_batch_size %d",
              a->n_rays, r->max_rays);
    CHECK_ARG(a->mode >= 0 && a->mode <= FLARE_FWD_MEDIAN, "flare_forward: bad mode %d", a->mode);
    if (a->n_rays == 0) return FLARE_OK;
    CHECK_ARG(a->O && a->v, "flare_forward: NULL rays");
    if (a->mode != FLARE_FWD_MEDIAN) CHECK_ARG(a->bitmap, "flare_forward: bitmap is NULL");
    if (a->mode == FLARE_FWD_TRAINING)
        CHECK_ARG(a->depth_reg_accums && a->normal_reg_accums && a->surface_normal,
                  "flare_forward: training mode needs depth_reg_accums, normal_reg_accums, surface_normal");
    if (a->mode == FLARE_FWD_MEDIAN) CHECK_ARG(a->depth_and_index, "flare_forward: depth_and_index is NULL");
    if (a->mode == FLARE_FWD_PCA) CHECK_ARG(a->override_colors, "flare_forward: override_colors is NULL");
    DeviceGuard dg(r->device);
    FLARE_CUDA_TRY(cudaMemsetAsync(r->dstats, 0, ST_NSTATS * sizeof(unsigned long long), S(stream)));
    r->last_stream = S(stream);
    e = run_forward(r, sc, a, S(stream));
    if (e) return e;
    return check_status(r, S(stream), "flare_forward");
}

int flare_adam_step(const flare_adam_args *a, void *stream) {
    g_err[0] = 0;
    CHECK_ARG(a, "flare_adam_step: NULL argument");
    CHECK_ARG(a->n_segments >= 0 && a->n_segments <= FLARE_ADAM_MAX_SEGMENTS, "flare_adam_step: %d segments (max %d)",
              a->n_segments, FLARE_ADAM_MAX_SEGMENTS);
    CHECK_ARG(a->step >= 1, "flare_adam_step: step %d < 1", a->step);
    for (int i = 0; i < a->n_segments; ++i) {
        const flare_adam_segment &s = a->seg[i];
        CHECK_ARG(s.param && s.grad && s.exp_avg && s.exp_avg_sq, "flare_adam_step: segment %d has a NULL buffer", i);
        CHECK_ARG(s.rows >= 0 && s.width >= 1 && s.p_offset >= 0 && s.p_offset + s.width <= s.p_stride,
                  "flare_adam_step: segment %d: rows %lld width %d stride %d offset %d", i, s.rows, s.width, s.p_stride,
                  s.p_offset);
        CHECK_ARG(s.scale_reg == 0.0f || s.width == 2, "flare_adam_step: segment %d: scale_reg needs width 2", i);
    }
    int e = run_adam(a, S(stream));
    if (e) return e;
    return FLARE_OK;
}

int flare_gather_rows(const flare_gather_tensor *t, int n_tensors, const int *src_row, int n_out, int alt_begin,
                      int alt_end, void *stream) {
    g_err[0] = 0;
    CHECK_ARG(n_tensors >= 0 && n_tensors <= FLARE_GATHER_MAX_TENSORS, "flare_gather_rows: %d tensors (max %d)",
              n_tensors, FLARE_GATHER_MAX_TENSORS);
    CHECK_ARG(n_out >= 0 && (n_out == 0 || src_row), "flare_gather_rows: NULL row map");
    for (int i = 0; i < n_tensors; ++i)
        CHECK_ARG(t && t[i].src && t[i].dst && t[i].row_bytes > 0 && (t[i].row_bytes & 3) == 0,
                  "flare_gather_rows: tensor %d: NULL buffer or row of %d bytes (multiple of 4 required)", i,
                  t ? t[i].row_bytes : 0);
    return run_gather_rows(t, n_tensors, src_row, n_out, alt_begin, alt_end, S(stream));
}

int flare_viewer_forward(flare_renderer *r, const flare_scene *sc, const flare_viewer_args *a, void *stream) {
    g_err[0] = 0;
    CHECK_ARG(r && a, "flare_viewer_forward: NULL argument");
    int e = check_scene(r, sc, "flare_viewer_forward");
    if (e) return e;
    CHECK_ARG(a->n_rays >= 0 && a->n_rays <= r->max_rays, "flare_viewer_forward: n_rays %d exceeds max_batch_size %d",
              a->n_rays, r->max_rays);
    if (a->n_rays == 0) return FLARE_OK;
    CHECK_ARG(a->O && a->v && a->bitmap, "flare_viewer_forward: NULL rays / bitmap");
    CHECK_ARG((a->n_spheres == 0 || (a->spheres && a->materials)) && (a->n_lights == 0 || a->lights),
              "flare_viewer_forward: NULL sphere / material / light table");
    DeviceGuard dg(r->device);
    FLARE_CUDA_TRY(cudaMemsetAsync(r->dstats, 0, ST_NSTATS * sizeof(unsigned long long), S(stream)));
    r->last_stream = S(stream);
    e = run_viewer_forward(r, sc, a, S(stream));
    if (e) return e;
    return check_status(r, S(stream), "flare_viewer_forward");
}

int flare_backward(flare_renderer *r, const flare_scene *sc, const flare_backward_args *a, void *stream) {
    g_err[0] = 0;
    CHECK_ARG(r && a, "flare_backward: NULL argument");
    int e = check_scene(r, sc, "flare_backward");
    if (e) return e;
    CHECK_ARG(a->n_rays >= 0 && a->n_rays <= r->max_rays, "flare_backward: n_rays %d exceeds max_batch_size %d",
              a->n_rays, r->max_rays);
    if (a->n_rays == 0) return FLARE_OK;
    CHECK_ARG(a->O && a->v && a->I && a->dL_dI, "flare_backward: NULL rays / image");
    CHECK_ARG(a->dL_dRGB && a->dL_dA && a->dL_dk && a->dL_dm && a->dL_ds && a->dL_dq, "flare_backward: NULL gradient");
    CHECK_ARG(a->depth_reg_accums && a->depth_normal_reg_prefix_sums && a->surface_normal,
              "flare_backward: NULL regulariser buffer");
    if (sc->cond)
        CHECK_ARG(a->dL_dcond && a->dL_dfeatures, "flare_backward: NULL decoder gradient");
    CHECK_ARG(!a->prim_rows || (reinterpret_cast<uintptr_t>(a->prim_rows) & 15) == 0,
              "flare_backward: prim_rows must be 16-byte aligned");
    DeviceGuard dg(r->device);
    FLARE_CUDA_TRY(cudaMemsetAsync(r->dstats, 0, ST_NSTATS * sizeof(unsigned long long), S(stream)));
    r->last_stream = S(stream);
    e = run_backward(r, sc, a, S(stream));
    if (e) return e;
    return check_status(r, S(stream), "flare_backward");
}

static_assert(PROW_FLOATS == FLARE_PRIM_ROW_FLOATS, "the header's row width must match the build's");

int flare_scatter_prim_rows(const float *rows, int n, const void *A1, int decoder, float *dL_dRGB, float *dL_dA,
                            float *dL_dk, float *dL_dm, float *dL_ds, float *dL_dq, float *dL_dcond, void *stream) {
    g_err[0] = 0;
    CHECK_ARG(n >= 0, "flare_scatter_prim_rows: n < 0");
    CHECK_ARG(decoder == FLARE_DECODER_LUT_PE || decoder == FLARE_DECODER_GRID_SH,
              "flare_scatter_prim_rows: unknown decoder %d", decoder);
    if (n == 0) return FLARE_OK;
    CHECK_ARG(rows && A1 && dL_dRGB && dL_dA && dL_dk && dL_dm && dL_ds && dL_dq && dL_dcond,
              "flare_scatter_prim_rows: NULL argument");
    return run_scatter_rows(rows, n, A1, decoder, dL_dRGB, dL_dA, dL_dk, dL_dm, dL_ds, dL_dq, dL_dcond, S(stream));
}

int flare_get_stats(flare_renderer *r, flare_stats *out) {
    g_err[0] = 0;
    CHECK_ARG(r && out, "flare_get_stats: NULL argument");
    DeviceGuard dg(r->device);
    unsigned long long h[ST_NSTATS];
    FLARE_CUDA_TRY(cudaMemcpyAsync(h, r->dstats, sizeof(h), cudaMemcpyDeviceToHost, r->last_stream));
    FLARE_CUDA_TRY(cudaStreamSynchronize(r->last_stream));
    out->passes = (long long)h[ST_PASSES];
    out->hits_composited = (long long)h[ST_HITS];
    out->prim_tests = (long long)h[ST_PRIM_TESTS];
    out->decoder_tiles = (long long)h[ST_TILES];
    out->node_visits = (long long)h[ST_NODES];
    out->rays = 0;
    return FLARE_OK;
}

int flare_profile(flare_renderer *r, int enable) {
    g_err[0] = 0;
    CHECK_ARG(r, "flare_profile: renderer is NULL");
    DeviceGuard dg(r->device);
    if (enable && !r->prof_ev[0]) {
        for (int i = 0; i < 2 * flare_renderer::PROF_SLOTS; ++i)
            FLARE_CUDA_TRY(cudaEventCreate(&r->prof_ev[i]));
    }
    r->prof_on = enable != 0;
    r->prof_n = 0;
    for (int k = 0; k < 4; ++k) {
        r->prof_ms[k] = 0.0;
        r->prof_launches[k] = 0;
    }
    return FLARE_OK;
}

int flare_get_kernel_times(flare_renderer *r, flare_kernel_times *out) {
    g_err[0] = 0;
    CHECK_ARG(r && out, "flare_get_kernel_times: NULL argument");
    DeviceGuard dg(r->device);
    if (r->prof_n) {
        FLARE_CUDA_TRY(cudaDeviceSynchronize());
        prof_collect(r);
    }
    for (int k = 0; k < 4; ++k) {
        out->ms[k] = r->prof_ms[k];
        out->launches[k] = r->prof_launches[k];
    }
    return FLARE_OK;
}

int flare_get_frames(flare_renderer *r, float *frames_out, void *stream) {
    g_err[0] = 0;
    CHECK_ARG(r && frames_out, "flare_get_frames: NULL argument");
    if (r->n == 0) return FLARE_OK;
    DeviceGuard dg(r->device);
    FLARE_CUDA_TRY(cudaMemcpyAsync(frames_out, r->frames, (size_t)r->n * 12 * sizeof(float), cudaMemcpyDeviceToDevice,
                                   S(stream)));
    FLARE_CUDA_TRY(cudaStreamSynchronize(S(stream)));
    return FLARE_OK;
}

static_assert(K_PASS == FLARE_PASS_SLOTS, "the header's pass size must match the build's");

int flare_get_pass_hits(flare_renderer *r, int pass, int *count, int *ray_ids, float *t_out, int *idx_out,
                        void *stream) {
    g_err[0] = 0;
    CHECK_ARG(r && count, "flare_get_pass_hits: NULL argument");
    if (!r->hc_valid) {
        set_error("flare_get_pass_hits: no cached Forward_training passes (the first Forward_training on a "
                  "renderer only sizes the cache; the cache was dropped, or a Backward consumed it)");
        return FLARE_E_STATE;
    }
    if (pass < 0) {
        *count = r->hc_npass;
        return FLARE_OK;
    }
    CHECK_ARG(pass < r->hc_npass, "flare_get_pass_hits: pass out of range");
    *count = r->hc_cnt[pass];
    if (!ray_ids && !t_out && !idx_out) return FLARE_OK;
    CHECK_ARG(ray_ids && t_out && idx_out, "flare_get_pass_hits: NULL output");
    DeviceGuard dg(r->device);
    const size_t off = r->hc_off[pass], c = (size_t)r->hc_cnt[pass];
    FLARE_CUDA_TRY(cudaMemcpyAsync(ray_ids, r->hc_list + off, c * sizeof(int), cudaMemcpyDeviceToDevice, S(stream)));
    FLARE_CUDA_TRY(cudaMemcpyAsync(t_out, r->hc_t + (size_t)K_PASS * off, c * K_PASS * sizeof(float),
                                   cudaMemcpyDeviceToDevice, S(stream)));
    FLARE_CUDA_TRY(cudaMemcpyAsync(idx_out, r->hc_idx + (size_t)K_PASS * off, c * K_PASS * sizeof(int),
                                   cudaMemcpyDeviceToDevice, S(stream)));
    FLARE_CUDA_TRY(cudaStreamSynchronize(S(stream)));
    return FLARE_OK;
}

int flare_selftest_mlp(const void *X, int rows, const void *A1, const float *b1, const void *A2, const float *b2,
                       const void *A3, const float *b3, float *Y, void *stream) {
    g_err[0] = 0;
    CHECK_ARG(X && A1 && b1 && A2 && b2 && A3 && b3 && Y, "flare_selftest_mlp: NULL argument");
    CHECK_ARG(rows >= 0, "flare_selftest_mlp: rows < 0");
    int *status = nullptr;
    FLARE_CUDA_TRY(cudaMalloc(&status, sizeof(int)));
    cudaMemsetAsync(status, 0, sizeof(int), S(stream));
    int e = selftest_mlp(X, rows, A1, b1, A2, b2, A3, b3, Y, S(stream), status);
    int h = 0;
    if (!e) {
        cudaMemcpyAsync(&h, status, sizeof(int), cudaMemcpyDeviceToHost, S(stream));
        cudaError_t ce = cudaStreamSynchronize(S(stream));
        if (ce != cudaSuccess) {
            set_error("flare_selftest_mlp: %s", cudaGetErrorString(ce));
            e = FLARE_E_CUDA;
        } else if (h) {
            set_error("flare_selftest_mlp: device reported error bits 0x%x", h);
            e = FLARE_E_DEVICE;
        }
    }
    cudaFree(status);
    return e;
}

}  // extern "C"
