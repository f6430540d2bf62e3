// viewer.cu -- secondary rays: the reference viewer's recursive forward (reflection, refraction, shadows)
// with analytic spheres in place of its triangle meshes.
//
// Reference (source/viewer_renderer/): per ray generation, the k-nearest passes over the primitives end
// at the closest mesh hit (shaders.cu:545-586, the mesh any-hit truncates the k-buffer), every buffered
// primitive hit gets a shadow test towards each directional light against the meshes only (shaders.cu:
// 86-122, instance masks 240 / 15), shadowed hits are composited with their colour times the shadow
// multiplier (Forward.cu:876-897), and when the generation's passes are done each ray that reached a
// mesh is shaded there (Fresnel / refraction / TIR, ambient, diffuse and specular with shadow rays,
// shaders.cu:180-490) and splits into a reflected and a refracted ray: the one carrying more
// transmittance continues in place, the other is pushed on a stack of ray sets (host loop, Forward.cu:
// 995-1276).  Rays that reach no mesh take the background times their transmittance.
//
// Departures, each forced by the sphere stand-in or chosen for exact CPU restatement: spheres are hit
// analytically (nearest root beyond the generation's t_min), their normal is (P - c) normalised; the
// reference's approximate rcp / sqrt / rsqrt are IEEE operations here; a ray whose transmittance fell
// below the threshold inside the generation ends there (background times its remaining T) instead of
// being shaded when the mesh happened to sit in its last 16-entry buffer.
#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_select.cuh>

#include "renderer.cuh"

namespace flare {

int launch_shade_viewer(flare_renderer *r, const flare_scene *sc, const float *O, const float *v, const int *lin,
                        int count, const float *ht, const int *hi, const unsigned char *shadow, float shadow_mult,
                        float *T, float *t_min, float *bitmap, float T_thr, cudaStream_t st);

struct ViewerConst {
    int S, L;
    float sph[FLARE_VIEWER_MAX_SPHERES][4];  // centre xyz, radius
    float mat[FLARE_VIEWER_MAX_SPHERES][6];  // Id rgb, kd, eta, n
    float light[FLARE_VIEWER_MAX_LIGHTS][6];  // Is rgb, direction L (the light travels along L)
    float eps, shadow_mult, T_thr;
    float Ia[3], bg[3];
};

// Nearest root of |O + t v - c| = r beyond t_min (INFINITY if none).
__device__ __forceinline__ float sphere_t(const float *c, float3 O, float3 v, float t_min) {
    const float ox = __fsub_rn(O.x, c[0]), oy = __fsub_rn(O.y, c[1]), oz = __fsub_rn(O.z, c[2]);
    const float a = __fmaf_rn(v.x, v.x, __fmaf_rn(v.y, v.y, __fmul_rn(v.z, v.z)));
    const float b = __fmaf_rn(ox, v.x, __fmaf_rn(oy, v.y, __fmul_rn(oz, v.z)));
    const float cc = __fmaf_rn(ox, ox, __fmaf_rn(oy, oy, __fmaf_rn(oz, oz, -__fmul_rn(c[3], c[3]))));
    const float disc = __fmaf_rn(b, b, -__fmul_rn(a, cc));
    if (!(disc >= 0.0f)) return INFINITY;
    const float sq = __fsqrt_rn(disc);
    const float t0 = __fdiv_rn(__fsub_rn(-b, sq), a), t1 = __fdiv_rn(__fadd_rn(-b, sq), a);
    if (t0 > t_min) return t0;
    if (t1 > t_min) return t1;
    return INFINITY;
}

// Does the point P see light j (no sphere along -L beyond eps)?
__device__ __forceinline__ bool lit(const ViewerConst &vc, float3 P, int j) {
    const float3 d = make_float3(-vc.light[j][3], -vc.light[j][4], -vc.light[j][5]);
    for (int s = 0; s < vc.S; ++s)
        if (sphere_t(vc.sph[s], P, d, vc.eps) < INFINITY) return false;
    return true;
}

__global__ void sphere_nearest_kernel(const ViewerConst vc, const int *__restrict__ list, int count,
                                      const float *__restrict__ O_, const float *__restrict__ v_,
                                      const float *__restrict__ tmin_, float *__restrict__ t_sph,
                                      int *__restrict__ sph_id) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= count) return;
    const int ray = list[j];
    const float3 O = make_float3(O_[3 * (size_t)ray], O_[3 * (size_t)ray + 1], O_[3 * (size_t)ray + 2]);
    const float3 v = make_float3(v_[3 * (size_t)ray], v_[3 * (size_t)ray + 1], v_[3 * (size_t)ray + 2]);
    const float tmin = tmin_[ray];
    float best = INFINITY;
    int id = -1;
    for (int s = 0; s < vc.S; ++s) {
        const float t = sphere_t(vc.sph[s], O, v, tmin);
        if (t < best) {
            best = t;
            id = s;
        }
    }
    t_sph[ray] = best;
    sph_id[ray] = id;
}

// Shadow flag of every buffered hit of the pass (slot-major, like the hit lists): 1 when some light is
// blocked by a sphere.
__global__ void shadow_flags_kernel(const ViewerConst vc, const int *__restrict__ list, int count, int K,
                                    const float *__restrict__ O_, const float *__restrict__ v_,
                                    const float *__restrict__ ht, const int *__restrict__ hi,
                                    unsigned char *__restrict__ shadow) {
    const size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= (size_t)count * K) return;
    const int j = (int)(e % count);
    unsigned char f = 0;
    if (hi[e] >= 0 && vc.L > 0) {
        const int ray = list[j];
        const float t = ht[e];
        const float3 P = make_float3(__fmaf_rn(v_[3 * (size_t)ray], t, O_[3 * (size_t)ray]),
                                     __fmaf_rn(v_[3 * (size_t)ray + 1], t, O_[3 * (size_t)ray + 1]),
                                     __fmaf_rn(v_[3 * (size_t)ray + 2], t, O_[3 * (size_t)ray + 2]));
        for (int l = 0; l < vc.L && !f; ++l) f = !lit(vc, P, l);
    }
    shadow[e] = f;
}

__device__ __forceinline__ float fresnel(float cos1, float eta, float cos2) {
    const float t1 = __fdiv_rn(__fsub_rn(1.0f, eta), __fadd_rn(1.0f, eta));
    const float R0 = __fmul_rn(t1, t1);
    const float t2 = __fsub_rn(1.0f, eta <= 1.0f ? cos2 : cos1);
    float t3 = __fmul_rn(t2, t2);
    t3 = __fmul_rn(t3, t3);
    t3 = __fmul_rn(t2, t3);
    return __fmaf_rn(__fsub_rn(1.0f, R0), t3, R0);
}

// cos(theta_2)^2 = 1 - n_inv^2 (1 - cos1^2); returns true on total internal reflection.
__device__ __forceinline__ bool cos_theta2(float cos1, float n_inv, float &cos2) {
    float s2 = __fmaf_rn(-cos1, cos1, 1.0f);
    if (s2 < 0.0f) s2 = 0.0f;
    const float c2 = __fmaf_rn(-__fmul_rn(n_inv, n_inv), s2, 1.0f);
    if (c2 < 0.0f) return true;
    cos2 = __fsqrt_rn(c2);
    return false;
}

__device__ __forceinline__ float dot3(float3 a, float3 b) {
    return __fmaf_rn(a.x, b.x, __fmaf_rn(a.y, b.y, __fmul_rn(a.z, b.z)));
}

__device__ __forceinline__ float3 scale3(float3 a, float s) {
    return make_float3(__fmul_rn(a.x, s), __fmul_rn(a.y, s), __fmul_rn(a.z, s));
}

// End of a ray generation.  A ray that composited everything before its sphere with T >= threshold is
// shaded at the sphere and split (in-place child into the generation's own arrays, the other into the
// push set); every other ray takes background * T.  Flags per list position: child still active.
__global__ void sphere_shade_kernel(const ViewerConst vc, const int *__restrict__ list, int count,
                                    float *__restrict__ O_, float *__restrict__ v_, float *__restrict__ T_,
                                    float *__restrict__ tmin_, const float *__restrict__ t_sph,
                                    const int *__restrict__ sph_id, float *__restrict__ bitmap,
                                    float *__restrict__ pO, float *__restrict__ pv, float *__restrict__ pT,
                                    float *__restrict__ ptmin, unsigned char *__restrict__ act_in,
                                    unsigned char *__restrict__ act_push) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= count) return;
    const int ray = list[j];
    const float T_old = T_[ray];
    const float ts = t_sph[ray];
    float *px = bitmap + 3 * (size_t)ray;
    if (!(T_old >= vc.T_thr) || !(ts < INFINITY)) {
        px[0] = __fmaf_rn(vc.bg[0], T_old, px[0]);
        px[1] = __fmaf_rn(vc.bg[1], T_old, px[1]);
        px[2] = __fmaf_rn(vc.bg[2], T_old, px[2]);
        act_in[j] = 0;
        act_push[j] = 0;
        return;
    }
    const int s = sph_id[ray];
    const float3 O = make_float3(O_[3 * (size_t)ray], O_[3 * (size_t)ray + 1], O_[3 * (size_t)ray + 2]);
    const float3 v = make_float3(v_[3 * (size_t)ray], v_[3 * (size_t)ray + 1], v_[3 * (size_t)ray + 2]);
    const float3 P = make_float3(__fmaf_rn(v.x, ts, O.x), __fmaf_rn(v.y, ts, O.y), __fmaf_rn(v.z, ts, O.z));
    float3 N = make_float3(__fsub_rn(P.x, vc.sph[s][0]), __fsub_rn(P.y, vc.sph[s][1]), __fsub_rn(P.z, vc.sph[s][2]));
    N = scale3(N, __fdiv_rn(1.0f, __fsqrt_rn(dot3(N, N))));
    const float Id[3] = {vc.mat[s][0], vc.mat[s][1], vc.mat[s][2]};
    const float kd_old = vc.mat[s][3], eta_old = vc.mat[s][4], nsh = vc.mat[s][5];
    const float eta_old_inv = __fdiv_rn(1.0f, eta_old);
    float cos1 = dot3(N, v);
    const float c2m = -2.0f * cos1;
    const float3 Rv = make_float3(__fmaf_rn(N.x, c2m, v.x), __fmaf_rn(N.y, c2m, v.y), __fmaf_rn(N.z, c2m, v.z));
    float eta_inv, kd;
    if (cos1 <= 0.0f) {
        eta_inv = eta_old_inv;
        kd = kd_old;
    } else {
        eta_inv = eta_old;
        kd = 0.0f;
    }
    float cos2 = 0.0f;
    const bool tir = cos_theta2(cos1, eta_inv, cos2);
    float3 Tv = make_float3(0.0f, 0.0f, 0.0f);
    float F1 = 1.0f;
    if (!tir) {
        const float tmp = __fmaf_rn(-cos1, eta_inv, copysignf(cos2, cos1));
        Tv = make_float3(__fadd_rn(__fmul_rn(v.x, eta_inv), __fmul_rn(N.x, tmp)),
                         __fadd_rn(__fmul_rn(v.y, eta_inv), __fmul_rn(N.y, tmp)),
                         __fadd_rn(__fmul_rn(v.z, eta_inv), __fmul_rn(N.z, tmp)));
        F1 = fresnel(cos1, eta_inv, cos2);
    }
    const float T_R = __fmul_rn(T_old, F1);
    const float T_T = __fmul_rn(__fmul_rn(T_old, __fsub_rn(1.0f, F1)), __fsub_rn(1.0f, kd));
    float col[3] = {0.0f, 0.0f, 0.0f};
    if (cos1 < 0.0f) {
        const float w = __fmul_rn(__fsub_rn(1.0f, F1), kd_old);
        for (int c = 0; c < 3; ++c) col[c] = __fmaf_rn(__fmul_rn(Id[c], w), vc.Ia[c], col[c]);
    }
    for (int l = 0; l < vc.L; ++l) {
        const bool is_lit = lit(vc, P, l);
        float3 L = make_float3(vc.light[l][3], vc.light[l][4], vc.light[l][5]);
        L = scale3(L, __fdiv_rn(1.0f, __fsqrt_rn(dot3(L, L))));
        const float cl = dot3(N, L);
        const float ei = cl <= 0.0f ? eta_old_inv : eta_old;
        float c2l = 0.0f;
        const float F2 = cos_theta2(cl, ei, c2l) ? 1.0f : fresnel(cl, ei, c2l);
        float diffuse = __fmul_rn(__fmul_rn(__fmul_rn(__fsub_rn(1.0f, F1), __fsub_rn(1.0f, F2)), kd_old),
                                  __saturatef(-cl));
        float3 H = make_float3(__fadd_rn(v.x, L.x), __fadd_rn(v.y, L.y), __fadd_rn(v.z, L.z));
        H = scale3(H, __fdiv_rn(1.0f, __fsqrt_rn(dot3(H, H))));
        const float ch = __saturatef(-dot3(N, H));
        float specular = __fdiv_rn(__fmul_rn(F2, ch), __fmaf_rn(nsh, __fsub_rn(1.0f, ch), ch));
        if (!is_lit) {
            diffuse = 0.0f;
            specular = 0.0f;
        }
        for (int c = 0; c < 3; ++c) col[c] = __fmaf_rn(vc.light[l][c], __fmaf_rn(Id[c], diffuse, specular), col[c]);
    }
    for (int c = 0; c < 3; ++c) px[c] = __saturatef(__fmaf_rn(T_old, col[c], px[c]));
    // the child with more transmittance continues in place; the other goes to the push set
    const bool refl_first = T_T <= T_R;
    const float T1 = refl_first ? T_R : T_T, T2 = refl_first ? T_T : T_R;
    const float3 v1 = refl_first ? Rv : Tv, v2 = refl_first ? Tv : Rv;
    O_[3 * (size_t)ray] = P.x; O_[3 * (size_t)ray + 1] = P.y; O_[3 * (size_t)ray + 2] = P.z;
    v_[3 * (size_t)ray] = v1.x; v_[3 * (size_t)ray + 1] = v1.y; v_[3 * (size_t)ray + 2] = v1.z;
    T_[ray] = T1;
    tmin_[ray] = vc.eps;
    pO[3 * (size_t)ray] = P.x; pO[3 * (size_t)ray + 1] = P.y; pO[3 * (size_t)ray + 2] = P.z;
    pv[3 * (size_t)ray] = v2.x; pv[3 * (size_t)ray + 1] = v2.y; pv[3 * (size_t)ray + 2] = v2.z;
    pT[ray] = T2;
    ptmin[ray] = vc.eps;
    act_in[j] = T1 >= vc.T_thr;
    act_push[j] = T2 >= vc.T_thr;
}

__global__ void iota_kernel(int *a, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) a[i] = i;
}

__global__ void fill_kernel(float *a, float x, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) a[i] = x;
}

// Sort key of a generation's rays: octahedral direction Morton code above the origin's (the origins of
// secondary rays are the sphere points they left from), so rays that travel together share packets.
__global__ void gen_key_kernel(const int *__restrict__ list, int count, const float *__restrict__ O_,
                               const float *__restrict__ v_, unsigned long long *__restrict__ keys,
                               int *__restrict__ vals) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= count) return;
    const int ray = list[j];
    auto spread16 = [](unsigned x) {
        unsigned long long v = x & 0xFFFFu;
        v = (v | (v << 8)) & 0x00FF00FFull;
        v = (v | (v << 4)) & 0x0F0F0F0Full;
        v = (v | (v << 2)) & 0x33333333ull;
        v = (v | (v << 1)) & 0x55555555ull;
        return v;
    };
    auto spread10 = [](unsigned v) {
        v = (v * 0x00010001u) & 0xFF0000FFu;
        v = (v * 0x00000101u) & 0x0F00F00Fu;
        v = (v * 0x00000011u) & 0xC30C30C3u;
        v = (v * 0x00000005u) & 0x49249249u;
        return v;
    };
    const float dx = v_[3 * (size_t)ray], dy = v_[3 * (size_t)ray + 1], dz = v_[3 * (size_t)ray + 2];
    const float l1 = fabsf(dx) + fabsf(dy) + fabsf(dz);
    float px = l1 > 0.0f ? dx / l1 : 0.0f, py = l1 > 0.0f ? dy / l1 : 0.0f;
    if (dz < 0.0f) {
        const float qx = (1.0f - fabsf(py)) * copysignf(1.0f, px), qy = (1.0f - fabsf(px)) * copysignf(1.0f, py);
        px = qx;
        py = qy;
    }
    const unsigned ux = (unsigned)fminf(fmaxf((px * 0.5f + 0.5f) * 65536.0f, 0.0f), 65535.0f);
    const unsigned uy = (unsigned)fminf(fmaxf((py * 0.5f + 0.5f) * 65536.0f, 0.0f), 65535.0f);
    unsigned oc = 0;
    for (int a = 0; a < 3; ++a) {  // origins in [-4, 4]^3 (the scene cube and cameras on a radius-3 sphere)
        const float x = (O_[3 * (size_t)ray + a] + 4.0f) * 0.125f;
        oc |= spread10((unsigned)fminf(fmaxf(x * 1024.0f, 0.0f), 1023.0f)) << (2 - a);
    }
    keys[j] = ((spread16(ux) << 1 | spread16(uy)) << 30) | oc;
    vals[j] = ray;
}

namespace {
struct RaySet {
    float *O = nullptr, *v = nullptr, *T = nullptr, *tmin = nullptr;
    int *list = nullptr;
    int count = 0;
    bool processed = false;
};
}  // namespace

static int viewer_alloc(flare_renderer *r, int sets) {
    const size_t R = (size_t)r->max_rays;
    if (r->vw_sets >= sets) return FLARE_OK;
    cudaFree(r->vw_buf);
    r->vw_buf = nullptr;
    r->vw_sets = 0;
    // per set: O 3, v 3, T 1, tmin 1 floats + list 1 int; shared: t_sph, sph_id, 2 flag arrays, shadow flags,
    // a compaction output list
    const size_t per_set = R * 9 * 4;
    const size_t shared = R * 4 * 3 + R * 2 + (size_t)K_PASS * R + R * 4;
    FLARE_CUDA_TRY(cudaMalloc(&r->vw_buf, per_set * sets + shared + 4096));
    r->vw_sets = sets;
    return FLARE_OK;
}

int run_viewer_forward(flare_renderer *r, const flare_scene *sc, const flare_viewer_args *a, cudaStream_t st) {
    const int R = a->n_rays;
    if (R <= 0) return FLARE_OK;
    if (a->n_spheres < 0 || a->n_spheres > FLARE_VIEWER_MAX_SPHERES || a->n_lights < 0 ||
        a->n_lights > FLARE_VIEWER_MAX_LIGHTS || a->max_recursion_depth < 0 || a->max_recursion_depth > 64) {
        set_error("flare_viewer_forward: %d spheres (max %d), %d lights (max %d), depth %d (max 64)", a->n_spheres,
                  FLARE_VIEWER_MAX_SPHERES, a->n_lights, FLARE_VIEWER_MAX_LIGHTS, a->max_recursion_depth);
        return FLARE_E_INVALID;
    }
    ViewerConst vc{};
    vc.S = a->n_spheres;
    vc.L = a->n_lights;
    for (int s = 0; s < vc.S; ++s) {
        for (int c = 0; c < 4; ++c) vc.sph[s][c] = a->spheres[4 * s + c];
        for (int c = 0; c < 6; ++c) vc.mat[s][c] = a->materials[6 * s + c];
    }
    for (int l = 0; l < vc.L; ++l)
        for (int c = 0; c < 6; ++c) vc.light[l][c] = a->lights[6 * l + c];
    vc.eps = a->epsilon;
    vc.shadow_mult = a->shadow_multiplier;
    vc.T_thr = a->T_threshold;
    for (int c = 0; c < 3; ++c) {
        vc.Ia[c] = a->ambient[c];
        vc.bg[c] = a->bg[c];
    }
    const int D = a->max_recursion_depth;
    const int nsets = D + 2;  // the primary set + push sets 0..D
    int e = viewer_alloc(r, nsets);
    if (e) return e;
    const size_t Rm = (size_t)r->max_rays;
    char *p = static_cast<char *>(r->vw_buf);
    RaySet sets[66];
    for (int i = 0; i < nsets; ++i) {
        sets[i].O = reinterpret_cast<float *>(p); p += Rm * 12;
        sets[i].v = reinterpret_cast<float *>(p); p += Rm * 12;
        sets[i].T = reinterpret_cast<float *>(p); p += Rm * 4;
        sets[i].tmin = reinterpret_cast<float *>(p); p += Rm * 4;
        sets[i].list = reinterpret_cast<int *>(p); p += Rm * 4;
    }
    float *t_sph = reinterpret_cast<float *>(p); p += Rm * 4;
    int *sph_id = reinterpret_cast<int *>(p); p += Rm * 4;
    int *tmp_list = reinterpret_cast<int *>(p); p += Rm * 4;
    unsigned char *act_in = reinterpret_cast<unsigned char *>(p); p += Rm;
    unsigned char *act_push = reinterpret_cast<unsigned char *>(p); p += Rm;
    unsigned char *shadow = reinterpret_cast<unsigned char *>(p); p += (size_t)K_PASS * Rm;
    const int B = 256;
    const int G = (R + B - 1) / B;
    // primary set: the caller's rays (copied: secondary generations overwrite origins and directions)
    RaySet *cur = &sets[0];
    FLARE_CUDA_TRY(cudaMemcpyAsync(cur->O, a->O, (size_t)R * 12, cudaMemcpyDeviceToDevice, st));
    FLARE_CUDA_TRY(cudaMemcpyAsync(cur->v, a->v, (size_t)R * 12, cudaMemcpyDeviceToDevice, st));
    fill_kernel<<<G, B, 0, st>>>(cur->T, 1.0f, R);
    fill_kernel<<<G, B, 0, st>>>(cur->tmin, 0.0f, R);
    iota_kernel<<<G, B, 0, st>>>(cur->list, R);
    FLARE_CUDA_TRY(cudaGetLastError());
    cur->count = R;
    RaySet *stack = &sets[1];
    int ss = 0;
    long long generations = 0, passes = 0;
    auto count_of = [&](int *out) -> int {
        FLARE_CUDA_TRY(cudaMemcpyAsync(r->h_count, r->counters, sizeof(int), cudaMemcpyDeviceToHost, st));
        FLARE_CUDA_TRY(cudaStreamSynchronize(st));
        *out = *r->h_count;
        return FLARE_OK;
    };
    const long long max_generations = 1ll << 20;
    while (true) {
        if (++generations > max_generations) {
            set_error("flare_viewer_forward: ray recursion did not end");
            return FLARE_E_DEVICE;
        }
        const int n0 = cur->count;
        if (n0 > 0) {
            const int g0 = (n0 + B - 1) / B;
            sphere_nearest_kernel<<<g0, B, 0, st>>>(vc, cur->list, n0, cur->O, cur->v, cur->tmin, t_sph, sph_id);
            // coherence order of this generation's rays into r->list[0]
            gen_key_kernel<<<g0, B, 0, st>>>(cur->list, n0, cur->O, cur->v, r->ray_keys, r->ray_ids_tmp);
            size_t tb = r->ray_sort_tmp_bytes;
            FLARE_CUDA_TRY(cub::DeviceRadixSort::SortPairs(r->ray_sort_tmp, tb, r->ray_keys, r->ray_keys + r->max_rays,
                                                           r->ray_ids_tmp, r->list[0], n0, 0, 64, st));
            int count = n0, c = 0;
            while (count > 0) {
                if (passes++ > (long long)(r->n / K_PASS) + 4 + 64 * generations) {
                    set_error("flare_viewer_forward: pass loop did not terminate");
                    return FLARE_E_DEVICE;
                }
                int slot = prof_begin(r, PK_TRACE, st);
                e = launch_trace(r, cur->O, cur->v, cur->tmin, r->list[c], count, r->hit_t, r->hit_idx, count, st,
                                 K_PASS, t_sph);
                prof_end(r, slot, st);
                if (e) return e;
                const size_t nh = (size_t)count * K_PASS;
                shadow_flags_kernel<<<(unsigned)((nh + B - 1) / B), B, 0, st>>>(vc, r->list[c], count, K_PASS, cur->O,
                                                                                cur->v, r->hit_t, r->hit_idx, shadow);
                FLARE_CUDA_TRY(cudaGetLastError());
                slot = prof_begin(r, PK_SHADE_FWD, st);
                e = launch_shade_viewer(r, sc, cur->O, cur->v, r->list[c], count, r->hit_t, r->hit_idx, shadow,
                                        vc.shadow_mult, cur->T, cur->tmin, a->bitmap, vc.T_thr, st);
                prof_end(r, slot, st);
                if (e) return e;
                e = compact_active(r, r->list[c], count, r->list[c ^ 1], st);
                if (e) return e;
                e = count_of(&count);
                if (e) return e;
                prof_collect(r);
                c ^= 1;
            }
        }
        // end of the generation: sphere shading and the split (push set = stack[ss])
        RaySet *push = &stack[ss];
        if (n0 > 0) {
            sphere_shade_kernel<<<(n0 + B - 1) / B, B, 0, st>>>(vc, cur->list, n0, cur->O, cur->v, cur->T, cur->tmin,
                                                                 t_sph, sph_id, a->bitmap, push->O, push->v, push->T,
                                                                 push->tmin, act_in, act_push);
            FLARE_CUDA_TRY(cudaGetLastError());
        }
        int n_push = 0, n_in = 0;
        if (n0 > 0) {
            size_t tb = r->select_tmp_bytes;
            FLARE_CUDA_TRY(cub::DeviceSelect::Flagged(r->select_tmp, tb, cur->list, act_push, push->list, r->counters, n0,
                                                      st));
            e = count_of(&n_push);
            if (e) return e;
            FLARE_CUDA_TRY(cub::DeviceSelect::Flagged(r->select_tmp, tb, cur->list, act_in, tmp_list, r->counters, n0,
                                                      st));
            e = count_of(&n_in);
            if (e) return e;
            FLARE_CUDA_TRY(cudaMemcpyAsync(cur->list, tmp_list, (size_t)n_in * 4, cudaMemcpyDeviceToDevice, st));
        }
        bool pop = false;
        if (n_push > 0) {
            if (ss < D) {  // keep the pushed rays for later, continue with the in-place children
                push->count = n_push;
                push->processed = false;
                ++ss;
                cur->count = n_in;
            } else {
                pop = true;  // depth limit: this generation's children end here
            }
        } else {
            cur->count = n_in;
            pop = n_in == 0;
        }
        if (pop) {
            do {
                --ss;
            } while (ss >= 0 && stack[ss].processed);
            if (ss < 0) break;
            cur = &stack[ss];
            stack[ss].processed = true;
            ++ss;
        }
    }
    unsigned long long gp[2] = {(unsigned long long)passes, (unsigned long long)generations};
    FLARE_CUDA_TRY(cudaMemcpyAsync(r->dstats + ST_PASSES, gp, sizeof(unsigned long long), cudaMemcpyHostToDevice, st));
    FLARE_CUDA_TRY(cudaStreamSynchronize(st));
    r->vw_generations = generations;
    return FLARE_OK;
}

}  // namespace flare
