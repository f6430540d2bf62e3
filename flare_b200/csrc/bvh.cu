// bvh.cu -- proxy frames and the LBVH over the polygon proxies (replaces the reference's
// GenerateInstances kernel + OptiX IAS build, CPyOptiXFLARERenderer_CUDA_Core.cu:532-816).
//
// Every flare_set_geometry call rebuilds from scratch, as the reference rebuilds its IAS every step:
//   1. prep: per primitive, the frame of its polygon proxy (Core.cu:553-622: rotation from the
//      quaternion with S = 2/|q|^2, radius rho = max(0, kappa (11.3449 + 2 ln sigma))^(1/(2 kappa)))
//      stored as [m, N, U/(e^sx rho), V/(e^sy rho)], plus a conservative AABB and the centre;
//   2. scene bounds of the centres (ordered-int atomics);
//   3. 32-bit extended Morton codes (centre + size class), CUB radix sort of (code, index) pairs;
//   4. Karras (2012) radix-tree hierarchy, one thread per internal node;
//   5. bottom-up box refit with one atomic flag per node; child boxes are stored in the parent so one
//      64-byte node fetch tests both children.
// Primitive records used by the traversal are gathered into Morton order (48 B each, 3 x 16 B loads).
#include <cub/device/device_radix_sort.cuh>

#include <cstdlib>
#include <cstring>

#include "renderer.cuh"

namespace flare {

__device__ __forceinline__ int f2ord(float f) {
    int i = __float_as_int(f);
    return i >= 0 ? i : i ^ 0x7FFFFFFF;
}
__device__ __forceinline__ float ord2f(int i) { return __int_as_float(i >= 0 ? i : i ^ 0x7FFFFFFF); }

// Frame of one primitive; explicit round-to-nearest intrinsics keep nvcc from contracting products
// into FMAs so the values follow the plain fp32 expression order.
__global__ void prep_kernel(const float *__restrict__ m, const float *__restrict__ scale,
                            const float *__restrict__ q, const float *__restrict__ opacity,
                            const float *__restrict__ kappa, int n, float *__restrict__ frames,
                            float *__restrict__ aabb, int *__restrict__ bounds) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    float cmin[3] = {INFINITY, INFINITY, INFINITY}, cmax[3] = {-INFINITY, -INFINITY, -INFINITY};
    if (i < n) {
        float4 qq = reinterpret_cast<const float4 *>(q)[i];
        float aa = __fmul_rn(qq.x, qq.x), bb = __fmul_rn(qq.y, qq.y), cc = __fmul_rn(qq.z, qq.z),
              dd = __fmul_rn(qq.w, qq.w);
        float S = __fdiv_rn(2.0f, __fadd_rn(__fadd_rn(__fadd_rn(aa, bb), cc), dd));
        float bs = __fmul_rn(qq.y, S), cs = __fmul_rn(qq.z, S), ds = __fmul_rn(qq.w, S);
        float ab = __fmul_rn(qq.x, bs), ac = __fmul_rn(qq.x, cs), ad = __fmul_rn(qq.x, ds);
        bb = __fmul_rn(bb, S);
        float bc = __fmul_rn(qq.y, cs), bd = __fmul_rn(qq.y, ds);
        cc = __fmul_rn(cc, S);
        float cd = __fmul_rn(qq.z, ds);
        dd = __fmul_rn(dd, S);
        float kap = kappa[i];
        float power = __fmul_rn(kap, __fadd_rn(11.3449f, __fmul_rn(2.0f, logf(opacity[i]))));
        if (power < 0.0f) power = 0.0f;
        float rho = powf(power, __fdiv_rn(1.0f, __fmul_rn(2.0f, kap)));
        float2 sc = reinterpret_cast<const float2 *>(scale)[i];
        float sx = __fmul_rn(sc.x, rho), sy = __fmul_rn(sc.y, rho);
        float Ux = __fsub_rn(__fsub_rn(1.0f, cc), dd), Uy = __fadd_rn(bc, ad), Uz = __fsub_rn(bd, ac);
        float Vx = __fsub_rn(bc, ad), Vy = __fsub_rn(__fsub_rn(1.0f, bb), dd), Vz = __fadd_rn(cd, ab);
        float Nx = __fadd_rn(bd, ac), Ny = __fsub_rn(cd, ab), Nz = __fsub_rn(__fsub_rn(1.0f, bb), cc);
        float mx = m[3 * i], my = m[3 * i + 1], mz = m[3 * i + 2];
        float *f = frames + 12 * (size_t)i;
        f[0] = mx; f[1] = my; f[2] = mz;
        f[3] = Nx; f[4] = Ny; f[5] = Nz;
        f[6] = __fdiv_rn(Ux, sx); f[7] = __fdiv_rn(Uy, sx); f[8] = __fdiv_rn(Uz, sx);
        f[9] = __fdiv_rn(Vx, sy); f[10] = __fdiv_rn(Vy, sy); f[11] = __fdiv_rn(Vz, sy);
        // The polygon is inscribed in the ellipse m + sx cos(th) U + sy sin(th) V; its box bounds the polygon.
        float hx = sqrtf(sx * sx * Ux * Ux + sy * sy * Vx * Vx);
        float hy = sqrtf(sx * sx * Uy * Uy + sy * sy * Vy * Vy);
        float hz = sqrtf(sx * sx * Uz * Uz + sy * sy * Vz * Vz);
        float pad = 1e-5f * (fabsf(mx) + fabsf(my) + fabsf(mz)) + 1e-6f;
        hx = hx * 1.0001f + pad; hy = hy * 1.0001f + pad; hz = hz * 1.0001f + pad;
        if (!(hx < INFINITY)) hx = 0.0f;  // degenerate (zero-radius / NaN) primitives never hit
        if (!(hy < INFINITY)) hy = 0.0f;
        if (!(hz < INFINITY)) hz = 0.0f;
        float *bx = aabb + 6 * (size_t)i;
        bx[0] = mx - hx; bx[1] = my - hy; bx[2] = mz - hz;
        bx[3] = mx + hx; bx[4] = my + hy; bx[5] = mz + hz;
        cmin[0] = cmax[0] = mx; cmin[1] = cmax[1] = my; cmin[2] = cmax[2] = mz;
    }
    // block-reduce the centre bounds, then one atomic per block
#pragma unroll
    for (int a = 0; a < 3; ++a) {
        for (int o = 16; o > 0; o >>= 1) {
            cmin[a] = fminf(cmin[a], __shfl_xor_sync(0xffffffffu, cmin[a], o));
            cmax[a] = fmaxf(cmax[a], __shfl_xor_sync(0xffffffffu, cmax[a], o));
        }
    }
    if ((threadIdx.x & 31) == 0 && cmin[0] <= cmax[0]) {
        for (int a = 0; a < 3; ++a) {
            atomicMin(bounds + a, f2ord(cmin[a]));
            atomicMax(bounds + 3 + a, f2ord(cmax[a]));
        }
    }
}

__global__ void init_bounds_kernel(int *bounds) {
    if (threadIdx.x < 3) bounds[threadIdx.x] = 0x7FFFFFFF;            // +max ordered
    else if (threadIdx.x < 6) bounds[threadIdx.x] = (int)0x80000000;  // -max ordered
}

__device__ __forceinline__ unsigned expand_bits10(unsigned v) {
    v = (v * 0x00010001u) & 0xFF0000FFu;
    v = (v * 0x00000101u) & 0x0F00F00Fu;
    v = (v * 0x00000011u) & 0xC30C30C3u;
    v = (v * 0x00000005u) & 0x49249249u;
    return v;
}

// Sort key = extended Morton code: the top EMC_P bits of the 30-bit centre code, then EMC_S bits of
// box-size class, then the next centre bits.  Primitives of very different sizes are separated just
// below the top levels, so small primitives' nodes are not inflated by large overlapping neighbours
// (cf. Vinkler et al. 2017, "Extended Morton codes for high performance bounding volume hierarchy
// construction").  The size class splits log2(box extent / scene diagonal) over [EMC_LO, EMC_HI) evenly;
// boxes outside clamp to the end classes, so scenes of uniformly small primitives get a plain Morton order.
#ifndef FLARE_EMC_S
#define FLARE_EMC_S 2
#endif
#ifndef FLARE_EMC_P
#define FLARE_EMC_P 6
#endif
#ifndef FLARE_EMC_LO
#define FLARE_EMC_LO -10.0f
#endif
#ifndef FLARE_EMC_HI
#define FLARE_EMC_HI -3.0f
#endif
// Hierarchy builder: the Karras radix tree (default), or locally-ordered clustering (ploc.cu) when the
// environment sets FLARE_BVH=ploc -- a slightly better tree for a ~3x longer build (config 3: traversal
// -3.5 %, build +5 ms; config 2: no net gain).
// 4-wide traversal hierarchy (collapsed from the binary one after every build) with FLARE_BVH4=1.  Off by
// default: on the 6M-primitive workload its traversal measured 569 ms per step against 512 ms for the
// binary one (same hits), so the dependent node-fetch chain it halves is not what bounds the traversal.
static bool use_bvh4() {
    static const bool on = [] {
        const char *e = getenv("FLARE_BVH4");
        return e && strcmp(e, "1") == 0;
    }();
    return on;
}

// Traversal nodes with inline leaf records (NodeL), built after every hierarchy build, with
// FLARE_TRACE_INLINE=1.  Off by default: same hits, but the exact test of every leaf child a packet reaches
// costs more than the box cull plus dependent record fetch it replaces (config 2 traversal 41.0 vs 38.1 ms,
// config 3 508 vs 478 ms per step).
bool use_inline_leaves() {
    static const bool on = [] {
        const char *e = getenv("FLARE_TRACE_INLINE");
        return e && strcmp(e, "1") == 0;
    }();
    return on;
}

// Node i of the binary hierarchy with each leaf child's record copied in (layout: NodeL).
__global__ void pack_inline_kernel(const Node *__restrict__ nodes, const float4 *__restrict__ rec, int n_internal,
                                   NodeL *__restrict__ out) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_internal) return;
    const Node nd = nodes[i];
    float4 c[8];
    const int link[2] = {nd.d.x, nd.d.y}, pid[2] = {nd.d.z, nd.d.w};
    const float box[2][6] = {{nd.a.x, nd.a.y, nd.a.z, nd.a.w, nd.b.x, nd.b.y},
                             {nd.b.z, nd.b.w, nd.c.x, nd.c.y, nd.c.z, nd.c.w}};
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        if (link[j] < 0) {
            const size_t p = (size_t)(~link[j]);
            c[4 * j] = rec[3 * p];
            c[4 * j + 1] = rec[3 * p + 1];
            c[4 * j + 2] = rec[3 * p + 2];
        } else {
            c[4 * j] = make_float4(box[j][0], box[j][1], box[j][2], box[j][3]);
            c[4 * j + 1] = make_float4(box[j][4], box[j][5], 0.0f, 0.0f);
            c[4 * j + 2] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
        c[4 * j + 3] = make_float4(__int_as_float(link[j]), __int_as_float(pid[j]), 0.0f, 0.0f);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) out[i].c[k] = c[k];
}

static bool use_ploc() {
    static const bool on = [] {
        const char *e = getenv("FLARE_BVH");
        return e && strcmp(e, "ploc") == 0;
    }();
    return on;
}
constexpr int MORTON_END_BIT = FLARE_EMC_S ? 32 : 30;

__global__ void morton_kernel(const float *__restrict__ m, const float *__restrict__ aabb, int n,
                              const int *__restrict__ bounds, unsigned *__restrict__ codes, int *__restrict__ ids) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    unsigned c = 0;
    float diag2 = 0.0f;
#pragma unroll
    for (int a = 0; a < 3; ++a) {
        float lo = ord2f(bounds[a]), hi = ord2f(bounds[3 + a]);
        float ext = hi - lo;
        diag2 += ext * ext;
        float x = ext > 0.0f ? (m[3 * i + a] - lo) / ext : 0.5f;
        unsigned q = (unsigned)fminf(fmaxf(x * 1024.0f, 0.0f), 1023.0f);
        c |= expand_bits10(q) << (2 - a);
    }
    if (FLARE_EMC_S) {
        const float *bx = aabb + 6 * (size_t)i;
        float e = fmaxf(fmaxf(bx[3] - bx[0], bx[4] - bx[1]), bx[5] - bx[2]);
        float rel = e * rsqrtf(fmaxf(diag2, 1e-30f));
        // size class: log2 of the box extent over the scene diagonal, [LO, HI) in 2^S steps
        float l = (log2f(fmaxf(rel, 1e-30f)) - FLARE_EMC_LO) * ((float)(1 << FLARE_EMC_S) / (FLARE_EMC_HI - FLARE_EMC_LO));
        unsigned sz = (unsigned)fminf(fmaxf(l, 0.0f), (float)((1 << FLARE_EMC_S) - 1));
        constexpr int P = FLARE_EMC_P, S = FLARE_EMC_S, L = 32 - P - S;
        unsigned hi = P ? (c >> (30 - P)) : 0u;
        unsigned lo = (L >= 30 - P) ? ((c << (L - (30 - P))) & ((1u << L) - 1u)) : ((c >> ((30 - P) - L)) & ((1u << L) - 1u));
        c = (P ? (hi << (32 - P)) : 0u) | (sz << L) | lo;
    }
    codes[i] = c;
    ids[i] = i;
}

// Common-prefix length of sorted keys i and j (index breaks ties), -1 when j is out of range.
__device__ __forceinline__ int delta(const unsigned *codes, int n, int i, int j) {
    if (j < 0 || j >= n) return -1;
    unsigned a = codes[i], b = codes[j];
    if (a == b) return 32 + __clz((unsigned)(i ^ j));
    return __clz(a ^ b);
}

__global__ void karras_kernel(const unsigned *__restrict__ codes, const int *__restrict__ ids_sorted, int n,
                              Node *__restrict__ nodes, int *__restrict__ parent) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n - 1) return;
    int d = (delta(codes, n, i, i + 1) - delta(codes, n, i, i - 1)) >= 0 ? 1 : -1;
    int dmin = delta(codes, n, i, i - d);
    int lmax = 2;
    while (delta(codes, n, i, i + lmax * d) > dmin) lmax <<= 1;
    int l = 0;
    for (int t = lmax >> 1; t >= 1; t >>= 1)
        if (delta(codes, n, i, i + (l + t) * d) > dmin) l += t;
    int j = i + l * d;
    int dnode = delta(codes, n, i, j);
    int s = 0;
    int t = l;
    do {
        t = (t + 1) >> 1;
        if (delta(codes, n, i, i + (s + t) * d) > dnode) s += t;
    } while (t > 1);
    int gamma = i + s * d + min(d, 0);
    int lo = min(i, j), hi = max(i, j);
    int c0 = (lo == gamma) ? ~gamma : gamma;
    int c1 = (hi == gamma + 1) ? ~(gamma + 1) : gamma + 1;
    // links, then the original index of each leaf child (the traversal reads it with the node)
    nodes[i].d = make_int4(c0, c1, c0 < 0 ? ids_sorted[gamma] : -1, c1 < 0 ? ids_sorted[gamma + 1] : -1);
    if (c0 >= 0) parent[c0] = i; else parent[(n - 1) + gamma] = i;
    if (c1 >= 0) parent[c1] = i; else parent[(n - 1) + gamma + 1] = i;
}

__device__ __forceinline__ void write_slot(Node *nd, int slot, const float *bx) {
    float *f = reinterpret_cast<float *>(nd);
    // slot 0: floats 0..5, slot 1: floats 6..11 (lo.xyz, hi.xyz)
#pragma unroll
    for (int k = 0; k < 6; ++k) __stcg(f + 6 * slot + k, bx[k]);
}

// Bottom-up refit: leaf threads climb; the second arrival at a node merges its two child boxes.
__global__ void refit_kernel(int n, const int *__restrict__ ids_sorted, const float *__restrict__ aabb,
                             Node *__restrict__ nodes, const int *__restrict__ parent, unsigned *__restrict__ flag,
                             float4 *__restrict__ rec, const float *__restrict__ frames, int *__restrict__ status) {
    int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= n) return;
    int pid = ids_sorted[j];
    // gather the traversal record in sorted order
    const float *f = frames + 12 * (size_t)pid;
    rec[3 * (size_t)j + 0] = make_float4(f[0], f[1], f[2], f[3]);
    rec[3 * (size_t)j + 1] = make_float4(f[4], f[5], f[6], f[7]);
    rec[3 * (size_t)j + 2] = make_float4(f[8], f[9], f[10], f[11]);
    if (n < 2) return;
    float bx[6];
#pragma unroll
    for (int k = 0; k < 6; ++k) bx[k] = aabb[6 * (size_t)pid + k];
    int p = parent[(n - 1) + j];
    int child = ~j;
    for (int depth = 0; depth < 256; ++depth) {  // a radix tree over 32+32-bit keys is < 128 deep
        Node *nd = nodes + p;
        int4 links = nd->d;
        write_slot(nd, links.x == child ? 0 : 1, bx);
        __threadfence();
        unsigned old = atomicAdd(flag + p, 1u);
        if (old == 0) return;  // sibling not done yet; it will continue upwards
        __threadfence();
        const float *nf = reinterpret_cast<const float *>(nd);
        float s[12];
#pragma unroll
        for (int k = 0; k < 12; ++k) s[k] = __ldcg(nf + k);
        bx[0] = fminf(s[0], s[6]); bx[1] = fminf(s[1], s[7]); bx[2] = fminf(s[2], s[8]);
        bx[3] = fmaxf(s[3], s[9]); bx[4] = fmaxf(s[4], s[10]); bx[5] = fmaxf(s[5], s[11]);
        if (p == 0) return;
        child = p;
        p = parent[p];
        if (p < 0 || p >= n - 1) break;
    }
    atomicOr(status, ERR_INDEX);
}

static int grow(flare_renderer *r, int n, cudaStream_t st) {
    if (n <= r->cap_n) return FLARE_OK;
    cudaFree(r->frames); cudaFree(r->rec); cudaFree(r->aabb); cudaFree(r->morton); cudaFree(r->morton_sorted);
    cudaFree(r->ids); cudaFree(r->ids_sorted); cudaFree(r->nodes); cudaFree(r->parent); cudaFree(r->refit_flag);
    cudaFree(r->sort_tmp);
    cudaFree(r->ploc_scratch);
    r->ploc_scratch = nullptr;
    cudaFree(r->nodes4);
    cudaFree(r->bvh4_scratch);
    r->nodes4 = nullptr;
    r->bvh4_scratch = nullptr;
    r->frames = nullptr; r->rec = nullptr; r->aabb = nullptr; r->morton = r->morton_sorted = nullptr;
    r->ids = r->ids_sorted = nullptr; r->nodes = nullptr; r->parent = nullptr; r->refit_flag = nullptr;
    r->sort_tmp = nullptr; r->cap_n = 0;
    size_t N = (size_t)n;
    FLARE_CUDA_TRY(cudaMalloc(&r->frames, N * 12 * sizeof(float)));
    FLARE_CUDA_TRY(cudaMalloc(&r->rec, N * 3 * sizeof(float4)));
    FLARE_CUDA_TRY(cudaMalloc(&r->aabb, N * 6 * sizeof(float)));
    FLARE_CUDA_TRY(cudaMalloc(&r->morton, N * sizeof(unsigned)));
    FLARE_CUDA_TRY(cudaMalloc(&r->morton_sorted, N * sizeof(unsigned)));
    FLARE_CUDA_TRY(cudaMalloc(&r->ids, N * sizeof(int)));
    FLARE_CUDA_TRY(cudaMalloc(&r->ids_sorted, N * sizeof(int)));
    FLARE_CUDA_TRY(cudaMalloc(&r->nodes, (N > 1 ? N - 1 : 1) * sizeof(Node)));
    FLARE_CUDA_TRY(cudaMalloc(&r->parent, (2 * N) * sizeof(int)));
    FLARE_CUDA_TRY(cudaMalloc(&r->refit_flag, (N > 1 ? N - 1 : 1) * sizeof(unsigned)));
    size_t tmp = 0;
    cub::DeviceRadixSort::SortPairs(nullptr, tmp, r->morton, r->morton_sorted, r->ids, r->ids_sorted, n, 0, MORTON_END_BIT, st);
    FLARE_CUDA_TRY(cudaMalloc(&r->sort_tmp, tmp));
    if (use_ploc()) FLARE_CUDA_TRY(cudaMalloc(&r->ploc_scratch, ploc_scratch_bytes(n)));
    cudaFree(r->nodesL);
    r->nodesL = nullptr;
    if (use_inline_leaves()) FLARE_CUDA_TRY(cudaMalloc(&r->nodesL, (N > 1 ? N - 1 : 1) * sizeof(NodeL)));
    if (use_bvh4()) {
        FLARE_CUDA_TRY(cudaMalloc(&r->nodes4, (N > 1 ? N - 1 : 1) * sizeof(Node4)));
        FLARE_CUDA_TRY(cudaMalloc(&r->bvh4_scratch, bvh4_scratch_bytes(n)));
    }
    r->sort_tmp_bytes = tmp;
    r->cap_n = n;
    return FLARE_OK;
}

int build_geometry(flare_renderer *r, const float *m, const float *scale, const float *q, const float *opacity,
                   const float *kappa, int n, cudaStream_t st) {
    r->n = 0;
    if (n == 0) return FLARE_OK;
    int e = grow(r, n, st);
    if (e) return e;
    const int B = 256;
    int G = (n + B - 1) / B;
    init_bounds_kernel<<<1, 32, 0, st>>>(reinterpret_cast<int *>(r->bounds));
    prep_kernel<<<G, B, 0, st>>>(m, scale, q, opacity, kappa, n, r->frames, r->aabb,
                                 reinterpret_cast<int *>(r->bounds));
    morton_kernel<<<G, B, 0, st>>>(m, r->aabb, n, reinterpret_cast<int *>(r->bounds), r->morton, r->ids);
    size_t tmp = r->sort_tmp_bytes;
    FLARE_CUDA_TRY(cub::DeviceRadixSort::SortPairs(r->sort_tmp, tmp, r->morton, r->morton_sorted, r->ids,
                                                   r->ids_sorted, n, 0, MORTON_END_BIT, st));
    if (use_ploc()) {
        e = build_hierarchy_ploc(n, r->ids_sorted, r->aabb, r->frames, r->nodes, r->rec, r->ploc_scratch,
                                 reinterpret_cast<unsigned long long *>(r->h_count), st);
        if (e) return e;
    } else {
        if (n > 1) {
            FLARE_CUDA_TRY(cudaMemsetAsync(r->refit_flag, 0, (size_t)(n - 1) * sizeof(unsigned), st));
            karras_kernel<<<(n - 1 + B - 1) / B, B, 0, st>>>(r->morton_sorted, r->ids_sorted, n, r->nodes, r->parent);
        }
        refit_kernel<<<G, B, 0, st>>>(n, r->ids_sorted, r->aabb, r->nodes, r->parent, r->refit_flag, r->rec,
                                      r->frames, r->dstatus);
    }
    if (r->nodesL && n > 1)
        pack_inline_kernel<<<(n - 1 + B - 1) / B, B, 0, st>>>(r->nodes, r->rec, n - 1, r->nodesL);
    if (r->nodes4) {
        e = build_bvh4(r->nodes, n, r->nodes4, r->bvh4_scratch, r->dstatus, st);
        if (e) return e;
    }
    FLARE_CUDA_TRY(cudaGetLastError());
    r->n = n;
    return FLARE_OK;
}

// The same build over an explicit buffer set (used by the allocation-free entry point in noalloc.cu).
int build_geometry_into(const GeomBufs &g, const float *m, const float *scale, const float *q, const float *opacity,
                        const float *kappa, int n, cudaStream_t st) {
    if (n == 0) return FLARE_OK;
    const int B = 256;
    int G = (n + B - 1) / B;
    init_bounds_kernel<<<1, 32, 0, st>>>(reinterpret_cast<int *>(g.bounds));
    prep_kernel<<<G, B, 0, st>>>(m, scale, q, opacity, kappa, n, g.frames, g.aabb, reinterpret_cast<int *>(g.bounds));
    morton_kernel<<<G, B, 0, st>>>(m, g.aabb, n, reinterpret_cast<int *>(g.bounds), g.morton, g.ids);
    size_t tmp = g.sort_tmp_bytes;
    FLARE_CUDA_TRY(cub::DeviceRadixSort::SortPairs(g.sort_tmp, tmp, g.morton, g.morton_sorted, g.ids, g.ids_sorted, n,
                                                   0, MORTON_END_BIT, st));
    if (n > 1) {
        FLARE_CUDA_TRY(cudaMemsetAsync(g.refit_flag, 0, (size_t)(n - 1) * sizeof(unsigned), st));
        karras_kernel<<<(n - 1 + B - 1) / B, B, 0, st>>>(g.morton_sorted, g.ids_sorted, n, g.nodes, g.parent);
    }
    refit_kernel<<<G, B, 0, st>>>(n, g.ids_sorted, g.aabb, g.nodes, g.parent, g.refit_flag, g.rec, g.frames, g.status);
    FLARE_CUDA_TRY(cudaGetLastError());
    return FLARE_OK;
}

size_t geometry_sort_temp_bytes(int n) {
    size_t tmp = 0;
    cub::DeviceRadixSort::SortPairs(nullptr, tmp, (unsigned *)nullptr, (unsigned *)nullptr, (int *)nullptr,
                                    (int *)nullptr, n, 0, MORTON_END_BIT, (cudaStream_t)0);
    return tmp;
}

}  // namespace flare

