// trace.cu -- k-nearest proxy traversal (replaces the reference's OptiX raygen + any-hit programs,
// source/renderer/shaders.cu:81-189, and the diagnostic raygen used by Render, shaders.cu:19-77).
//
// A warp walks the LBVH for a packet of 32 coherent rays (a whole warp per ray once a pass is sparse),
// nearer child first, and each ray keeps the K smallest (t, primitive index) hits with t >= t_min in a
// register-resident sorted buffer (the reference's any-hit insertion sort, shaders.cu:166-188, with ties
// broken by the smaller index so the result is independent of traversal order).  A subtree is pruned
// when its box entry lies beyond the ray's current K-th hit.  Nodes are 64-byte records read as four
// 16-byte loads; primitive records are 48 bytes in Morton order read as three 16-byte loads.
//
// The hit test is exact fp32 with explicit rounding intrinsics; oracle/trace_oracle.c executes the
// identical sequence, which is what makes hit lists bit-comparable.
#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_select.cuh>

#include <cstdlib>

#include "renderer.cuh"

#ifndef FLARE_TRACE_MIN_BLOCKS
#define FLARE_TRACE_MIN_BLOCKS 4  // resident 128-thread blocks per SM the register budget aims for
#endif

namespace flare {

template <int K>
struct KBuf {
    float t[K];
    int i[K];
};

template <int K>
__device__ __forceinline__ void kbuf_insert(KBuf<K> &b, float t, int id) {
    // Sorted by (t, index).  Slot k takes the old slot k-1 when (t, id) precedes both old entries, the
    // new entry when it precedes only old slot k, else keeps its own.  Every comparison reads the old
    // buffer (slots are rewritten from the top down), so the K steps are independent instead of one
    // serial compare-and-swap chain.
    bool lt_k = t < b.t[K - 1] || (t == b.t[K - 1] && id < b.i[K - 1]);
#pragma unroll
    for (int k = K - 1; k > 0; --k) {
        const float tp = b.t[k - 1];
        const int ip = b.i[k - 1];
        const bool lt_p = t < tp || (t == tp && id < ip);
        b.t[k] = lt_k ? (lt_p ? tp : t) : b.t[k];
        b.i[k] = lt_k ? (lt_p ? ip : id) : b.i[k];
        lt_k = lt_p;
    }
    b.t[0] = lt_k ? t : b.t[0];
    b.i[0] = lt_k ? id : b.i[0];
}

#ifdef FLARE_TRACE_WHY
__device__ unsigned long long g_why[4];  // diagnostic build only: why primitive tests fail
#endif

// Exact hit test against one 48-byte primitive record (same operation order as the oracle).
__device__ __forceinline__ bool hit_rec(float4 r0, float4 r1, float4 r2, float3 O, float3 v, float t_min,
                                        const PolyConst &c_poly, float &t_out, float t_max = INFINITY) {
    // r0 = m.xyz N.x, r1 = N.yz Ua.xy, r2 = Ua.z Va.xyz
    float dx = __fsub_rn(r0.x, O.x), dy = __fsub_rn(r0.y, O.y), dz = __fsub_rn(r0.z, O.z);
    float num = __fmaf_rn(r0.w, dx, __fmaf_rn(r1.x, dy, __fmul_rn(r1.y, dz)));
    float den = __fmaf_rn(r0.w, v.x, __fmaf_rn(r1.x, v.y, __fmul_rn(r1.y, v.z)));
    float t = __fdiv_rn(num, den);
    if (!(t >= t_min) || t > t_max) {  // beyond the K-th buffered hit: cannot enter the buffer
#ifdef FLARE_TRACE_WHY
        atomicAdd(g_why + (t >= t_min ? 1 : 0), 1ull);  // 0: before t_min, 1: beyond the K-th hit
#endif
        return false;
    }
    float ex = __fsub_rn(__fmaf_rn(v.x, t, O.x), r0.x);
    float ey = __fsub_rn(__fmaf_rn(v.y, t, O.y), r0.y);
    float ez = __fsub_rn(__fmaf_rn(v.z, t, O.z), r0.z);
    float a = __fmaf_rn(r1.z, ex, __fmaf_rn(r1.w, ey, __fmul_rn(r2.x, ez)));
    float b = __fmaf_rn(r2.y, ex, __fmaf_rn(r2.z, ey, __fmul_rn(r2.w, ez)));
    if (c_poly.half == 4) {  // octagon (the renderer's default): the same tests, unrolled
#pragma unroll
        for (int j = 0; j < 4; ++j)
            if (!(fabsf(__fmaf_rn(c_poly.c[j], a, __fmul_rn(c_poly.s[j], b))) <= 1.0f)) {
#ifdef FLARE_TRACE_WHY
                atomicAdd(g_why + 2, 1ull);  // outside the polygon
#endif
                return false;
            }
    } else if (c_poly.half) {
        for (int j = 0; j < c_poly.half; ++j)
            if (!(fabsf(__fmaf_rn(c_poly.c[j], a, __fmul_rn(c_poly.s[j], b))) <= 1.0f)) {
#ifdef FLARE_TRACE_WHY
                atomicAdd(g_why + 2, 1ull);  // outside the polygon
#endif
                return false;
            }
    } else {
        for (int j = 0; j < c_poly.n; ++j)
            if (!(__fmaf_rn(c_poly.c[j], a, __fmul_rn(c_poly.s[j], b)) <= 1.0f)) return false;
    }
    t_out = t;
    return true;
}

// Exact hit test on the record of sorted primitive p.
__device__ __forceinline__ bool hit_prim(const float4 *__restrict__ rec, int p, float3 O, float3 v, float t_min,
                                         const PolyConst &c_poly, float &t_out, float t_max = INFINITY) {
    return hit_rec(__ldg(rec + 3 * (size_t)p), __ldg(rec + 3 * (size_t)p + 1), __ldg(rec + 3 * (size_t)p + 2), O, v,
                   t_min, c_poly, t_out, t_max);
}

__device__ __forceinline__ bool slab(float lx, float ly, float lz, float hx, float hy, float hz, float3 O, float3 iv,
                                     float tlo, float thi, float &tnear) {
    float tx0 = (lx - O.x) * iv.x, tx1 = (hx - O.x) * iv.x;
    float ty0 = (ly - O.y) * iv.y, ty1 = (hy - O.y) * iv.y;
    float tz0 = (lz - O.z) * iv.z, tz1 = (hz - O.z) * iv.z;
    float tn = fmaxf(fmaxf(fminf(tx0, tx1), fminf(ty0, ty1)), fmaxf(fminf(tz0, tz1), tlo));
    float tf = fminf(fminf(fmaxf(tx0, tx1), fmaxf(ty0, ty1)), fminf(fmaxf(tz0, tz1), thi));
    tnear = tn;
    return tn <= tf;
}

// The slab distances as fma(bound, 1/v, -O/v): one instruction per plane instead of a subtract and a
// multiply (traversal -2.4 % on the 6M-primitive workload).  The boxes are padded well beyond that
// rounding (prep_kernel), so the culling stays conservative; FLARE_SLAB_FMA=0 builds the two-step form.
#ifndef FLARE_SLAB_FMA
#define FLARE_SLAB_FMA 1
#endif
__device__ __forceinline__ bool slab_fma(float lx, float ly, float lz, float hx, float hy, float hz, float3 niv,
                                         float3 iv, float tlo, float thi, float &tnear) {
    float tx0 = __fmaf_rn(lx, iv.x, niv.x), tx1 = __fmaf_rn(hx, iv.x, niv.x);
    float ty0 = __fmaf_rn(ly, iv.y, niv.y), ty1 = __fmaf_rn(hy, iv.y, niv.y);
    float tz0 = __fmaf_rn(lz, iv.z, niv.z), tz1 = __fmaf_rn(hz, iv.z, niv.z);
    float tn = fmaxf(fmaxf(fminf(tx0, tx1), fminf(ty0, ty1)), fmaxf(fminf(tz0, tz1), tlo));
    float tf = fminf(fminf(fmaxf(tx0, tx1), fmaxf(ty0, ty1)), fminf(fmaxf(tz0, tz1), thi));
    tnear = tn;
    return tn <= tf;
}

// Traversal kernel: the 32 rays of a warp share one traversal stack (in shared memory) and every node
// fetch; each lane keeps its own k-buffer and interval [t_min, t_16], and a child is entered when any
// lane's interval overlaps its box (lane masks ride on the stack).  Control flow is warp-uniform, so
// the per-ray divergence of the one-thread-per-ray walk disappears; coherent rays (sorted by origin and
// direction before the first pass) share most of their node visits.  The hit set is the same exact
// k-nearest set as any other traversal order.
template <bool STATS, int K>
__global__ void __launch_bounds__(128, FLARE_TRACE_MIN_BLOCKS) trace_packet_kernel(
    const float *__restrict__ O_, const float *__restrict__ v_, const float *__restrict__ tmin_,
    const int *__restrict__ ray_ids, int count, const Node *__restrict__ nodes, const float4 *__restrict__ rec,
    const int *__restrict__ ids, int n, float *__restrict__ t_out, int *__restrict__ idx_out, int stride,
    const PolyConst poly, int *__restrict__ status, unsigned long long *__restrict__ stats,
    const float *__restrict__ tmax_ = nullptr) {
    __shared__ int s_node[4][TRACE_STACK];
    __shared__ unsigned s_mask[4][TRACE_STACK];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    const bool live = j < count;
    unsigned long long nprim = 0, nnode = 0;
    int ray = live ? (ray_ids ? ray_ids[j] : j) : 0;
    float3 O = make_float3(0, 0, 0), v = make_float3(0, 0, 1);
    float t_min = INFINITY, tcap = INFINITY;
    if (live) {
        O = make_float3(O_[3 * (size_t)ray], O_[3 * (size_t)ray + 1], O_[3 * (size_t)ray + 2]);
        v = make_float3(v_[3 * (size_t)ray], v_[3 * (size_t)ray + 1], v_[3 * (size_t)ray + 2]);
        t_min = tmin_[ray];
        if (tmax_) tcap = nextafterf(tmax_[ray], -INFINITY);  // hits must lie before t_max
    }
    KBuf<K> kb;
#pragma unroll
    for (int k = 0; k < K; ++k) {
        kb.t[k] = INFINITY;
        kb.i[k] = 0x7fffffff;
    }
    const float3 iv = make_float3(1.0f / (fabsf(v.x) > 1e-30f ? v.x : copysignf(1e-30f, v.x)),
                                  1.0f / (fabsf(v.y) > 1e-30f ? v.y : copysignf(1e-30f, v.y)),
                                  1.0f / (fabsf(v.z) > 1e-30f ? v.z : copysignf(1e-30f, v.z)));
    const float tlo = __fmaf_rn(-fabsf(t_min), 1e-5f, t_min);
    const bool want = live && t_min < INFINITY;
    if (n == 1) {
        float t;
        if (want) {
            ++nprim;
            if (hit_prim(rec, 0, O, v, t_min, poly, t, tcap)) kbuf_insert(kb, t, ids[0]);
        }
    } else if (n > 1) {
        unsigned mask = __ballot_sync(0xffffffffu, want);
        int node = 0, sp = 0;
        const unsigned long long max_visits = 2ull * (unsigned long long)n + 64ull;
        while (mask) {
            if (++nnode > max_visits) {
                if (lane == 0) atomicOr(status, ERR_INDEX);
                break;
            }
            const bool in = (mask >> lane) & 1u;
            const float4 *np = reinterpret_cast<const float4 *>(nodes + node);
            const float4 a = __ldg(np), b = __ldg(np + 1), c = __ldg(np + 2);
            const int4 d = __ldg(reinterpret_cast<const int4 *>(np + 3));
            const float bk = fminf(kb.t[K - 1], tcap);
            const float thi = __fmaf_rn(fabsf(bk), 1e-5f, bk);
            float t0 = 0.0f, t1 = 0.0f;
            bool h0 = in && slab(a.x, a.y, a.z, a.w, b.x, b.y, O, iv, tlo, thi, t0);
            bool h1 = in && slab(b.z, b.w, c.x, c.y, c.z, c.w, O, iv, tlo, thi, t1);
            if (d.x < 0) {  // warp-uniform: leaf child 0
                if (h0) {
                    float t;
                    ++nprim;
                    if (hit_prim(rec, ~d.x, O, v, t_min, poly, t, bk)) {
                        const int pid = d.z;
                        if (t < kb.t[K - 1] || (t == kb.t[K - 1] && pid < kb.i[K - 1]))
                            kbuf_insert(kb, t, pid);
                    }
                }
                h0 = false;
            }
            if (d.y < 0) {
                if (h1) {
                    float t;
                    ++nprim;
                    if (hit_prim(rec, ~d.y, O, v, t_min, poly, t, bk)) {
                        const int pid = d.w;
                        if (t < kb.t[K - 1] || (t == kb.t[K - 1] && pid < kb.i[K - 1]))
                            kbuf_insert(kb, t, pid);
                    }
                }
                h1 = false;
            }
            const unsigned m0 = __ballot_sync(0xffffffffu, h0), m1 = __ballot_sync(0xffffffffu, h1);
            if (m0 && m1) {
                // nearer child first by lane vote (lanes that hit only one child vote for it)
                const unsigned v0 = __ballot_sync(0xffffffffu, h0 && (!h1 || t0 <= t1));
                const bool first0 = __popc(v0) * 2 >= __popc(m0 | m1);
                if (sp < TRACE_STACK) {
                    if (lane == 0) {
                        s_node[wib][sp] = first0 ? d.y : d.x;
                        s_mask[wib][sp] = first0 ? m1 : m0;
                    }
                    ++sp;
                } else if (lane == 0) {
                    atomicOr(status, ERR_STACK);
                }
                node = first0 ? d.x : d.y;
                mask = first0 ? m0 : m1;
                __syncwarp();
                continue;
            }
            if (m0) { node = d.x; mask = m0; continue; }
            if (m1) { node = d.y; mask = m1; continue; }
            __syncwarp();
            if (sp == 0) break;
            --sp;
            node = s_node[wib][sp];
            mask = s_mask[wib][sp];
        }
    }
    if (live) {
#pragma unroll
        for (int k = 0; k < K; ++k) {
            const bool valid = kb.i[k] != 0x7fffffff;
            t_out[(size_t)k * stride + j] = valid ? kb.t[k] : INFINITY;
            idx_out[(size_t)k * stride + j] = valid ? kb.i[k] : -1;
        }
    }
    if (STATS) {
        for (int o = 16; o > 0; o >>= 1) nprim += __shfl_xor_sync(0xffffffffu, nprim, o);
        if (lane == 0 && (nprim | nnode)) {
            atomicAdd(stats + ST_PRIM_TESTS, nprim);
            atomicAdd(stats + ST_NODES, nnode);
        }
    }
}


// Per-lane k-buffer as a max-heap in shared memory ([slot][thread] layout: every lane reads its own
// column, so accesses are bank-conflict free).  An accepted hit replaces the root (the current K-th
// nearest) and sifts down about log2 K levels instead of shifting a sorted register array; the heap is
// sorted once when the pass ends.  Frees the ~2K registers of the register buffer.
// Bound of a first-pass chunk: its phase-1 neighbours' largest K-th hit distance times this factor.
#ifndef FLARE_FIRST_BOUND_F
#define FLARE_FIRST_BOUND_F 1.0f
#endif
constexpr float FIRST_BOUND_F = FLARE_FIRST_BOUND_F;

__device__ __forceinline__ bool key_greater(float ta, int ia, float tb, int ib) {
    return ta > tb || (ta == tb && ia > ib);
}

template <int K>
struct HeapBuf {
    float *t;  // t[k * 128 + lane]
    int *i;
    float rt;  // root key (the current K-th nearest), cached
    int ri;
};
template <int K>
__device__ __forceinline__ void heap_init(HeapBuf<K> &h, unsigned char *smem) {
    h.t = reinterpret_cast<float *>(smem);
    h.i = reinterpret_cast<int *>(smem + (size_t)K * 128 * sizeof(float));
    for (int k = 0; k < K; ++k) {
        h.t[k * 128 + threadIdx.x] = INFINITY;
        h.i[k * 128 + threadIdx.x] = 0x7fffffff;
    }
    h.rt = INFINITY;
    h.ri = 0x7fffffff;
}
template <int K>
__device__ __forceinline__ bool heap_accepts(const HeapBuf<K> &h, float t, int id) {
    return t < h.rt || (t == h.rt && id < h.ri);
}
template <int K>
__device__ __forceinline__ float heap_root_t(const HeapBuf<K> &h) { return h.rt; }

template <int K>
__device__ __forceinline__ void heap_sift(HeapBuf<K> &h, int size, float t, int id) {
    const int c = threadIdx.x;
    int pos = 0;
    while (true) {
        const int l = 2 * pos + 1;
        if (l >= size) break;
        float tc = h.t[l * 128 + c];
        int ic = h.i[l * 128 + c];
        int ch = l;
        if (l + 1 < size) {
            const float tr = h.t[(l + 1) * 128 + c];
            const int ir = h.i[(l + 1) * 128 + c];
            if (key_greater(tr, ir, tc, ic)) {
                tc = tr;
                ic = ir;
                ch = l + 1;
            }
        }
        if (!key_greater(tc, ic, t, id)) break;
        h.t[pos * 128 + c] = tc;
        h.i[pos * 128 + c] = ic;
        pos = ch;
    }
    h.t[pos * 128 + c] = t;
    h.i[pos * 128 + c] = id;
}

template <int K>
__device__ __forceinline__ void heap_insert(HeapBuf<K> &h, float t, int id) {
    heap_sift(h, K, t, id);
    h.rt = h.t[threadIdx.x];
    h.ri = h.i[threadIdx.x];
}
// Writes the K entries in ascending order (slot-major, +inf / -1 padding); destroys the heap.
template <int K>
__device__ __forceinline__ void heap_emit(HeapBuf<K> &h, float *t_out, int *idx_out, int stride, int j) {
    for (int k = K - 1; k >= 0; --k) {  // the largest key leaves first, into the last slot
        const float tk = h.t[threadIdx.x];
        const int ik = h.i[threadIdx.x];
        const bool valid = ik != 0x7fffffff;
        t_out[(size_t)k * stride + j] = valid ? tk : INFINITY;
        idx_out[(size_t)k * stride + j] = valid ? ik : -1;
        if (k > 0) heap_sift(h, k, h.t[k * 128 + threadIdx.x], h.i[k * 128 + threadIdx.x]);
    }
}

template <bool STATS, int K, bool PERSIST>
__global__ void __launch_bounds__(128, 5) trace_heap_kernel(
    const float *__restrict__ O_, const float *__restrict__ v_, const float *__restrict__ tmin_,
    const int *__restrict__ ray_ids, int count, const Node *__restrict__ nodes, const float4 *__restrict__ rec,
    const int *__restrict__ ids, int n, float *__restrict__ t_out, int *__restrict__ idx_out, int stride,
    const PolyConst poly, int *__restrict__ status, unsigned long long *__restrict__ stats,
    const float *__restrict__ tmax_ = nullptr, int *__restrict__ chunk_ctr = nullptr, int phase = 0,
    float *__restrict__ chunk_tk = nullptr, float *__restrict__ hint_out = nullptr) {
    __shared__ int s_node[4][TRACE_STACK];
    __shared__ unsigned s_mask[4][TRACE_STACK];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    unsigned long long nprim = 0, nnode = 0;
    // PERSIST: the grid holds as many blocks as fit at once and every warp claims the next 32 rays of
    // the list until it is exhausted, so a warp slot frees as soon as its rays are done instead of
    // when the slowest warp of its block is (dense and sparse rays share blocks).
    // First-pass phases (phase 1, then 2): phase 1 traces every FIRST_STRIDE-th 32-ray chunk of the list
    // and records, per chunk, the largest K-th hit distance of its rays (+inf if one of them found fewer
    // than K hits); phase 2 traces the other chunks, each bounded by its two phase-1 neighbours' record
    // (coherent rays: the neighbouring packets of the ray order), the bound also going to hint_out so that
    // a ray that finds fewer than K hits below it continues there (the bounded-pass rule).
    constexpr int FIRST_STRIDE = 8;
    const int nchunks = (count + 31) / 32;
    int base = blockIdx.x * blockDim.x + (threadIdx.x & ~31);
    while (true) {
    int chunk = 0;
    if (PERSIST) {
        int b = 0;
        if (lane == 0) b = atomicAdd(chunk_ctr, phase ? 1 : 32);
        b = __shfl_sync(0xffffffffu, b, 0);
        if (phase == 1) chunk = b * FIRST_STRIDE;
        else if (phase == 2) chunk = (b / (FIRST_STRIDE - 1)) * FIRST_STRIDE + b % (FIRST_STRIDE - 1) + 1;
        else chunk = b / 32;
        base = chunk * 32;
        if (chunk >= nchunks) break;
    }
    const int j = base + lane;
    const bool live = j < count;
    int ray = live ? (ray_ids ? ray_ids[j] : j) : 0;
    float3 O = make_float3(0, 0, 0), v = make_float3(0, 0, 1);
    float t_min = INFINITY, tcap = INFINITY;
    if (live) {
        O = make_float3(O_[3 * (size_t)ray], O_[3 * (size_t)ray + 1], O_[3 * (size_t)ray + 2]);
        v = make_float3(v_[3 * (size_t)ray], v_[3 * (size_t)ray + 1], v_[3 * (size_t)ray + 2]);
        t_min = tmin_[ray];
        if (tmax_) tcap = nextafterf(tmax_[ray], -INFINITY);  // hits must lie before t_max
    }
    if (PERSIST && phase == 2) {
        const int a = chunk / FIRST_STRIDE;
        float bnd = __ldcg(chunk_tk + a);
        if ((a + 1) * FIRST_STRIDE < nchunks) bnd = fmaxf(bnd, __ldcg(chunk_tk + a + 1));
        bnd = __fmul_rn(bnd, FIRST_BOUND_F);
        if (bnd < INFINITY && live && t_min < bnd) {
            tcap = fminf(tcap, nextafterf(bnd, -INFINITY));
            hint_out[ray] = bnd;
        }
    }
    extern __shared__ __align__(16) unsigned char heap_smem[];
    HeapBuf<K> kb;
    heap_init(kb, heap_smem);
    const float3 iv = make_float3(1.0f / (fabsf(v.x) > 1e-30f ? v.x : copysignf(1e-30f, v.x)),
                                  1.0f / (fabsf(v.y) > 1e-30f ? v.y : copysignf(1e-30f, v.y)),
                                  1.0f / (fabsf(v.z) > 1e-30f ? v.z : copysignf(1e-30f, v.z)));
    const float tlo = __fmaf_rn(-fabsf(t_min), 1e-5f, t_min);
#if FLARE_SLAB_FMA
    const float3 niv = make_float3(-O.x * iv.x, -O.y * iv.y, -O.z * iv.z);
#endif
    const bool want = live && t_min < INFINITY;
    if (n == 1) {
        float t;
        if (want) {
            ++nprim;
            if (hit_prim(rec, 0, O, v, t_min, poly, t, tcap)) heap_insert(kb, t, ids[0]);
        }
    } else if (n > 1) {
        unsigned mask = __ballot_sync(0xffffffffu, want);
        int node = 0, sp = 0;
        const unsigned long long max_visits = 2ull * (unsigned long long)n + 64ull;
        // The next node's fetch is issued as soon as the box tests decide it, ahead of this node's leaf
        // tests, so its L2 latency overlaps the primitive-record fetches and hit tests.
        const float4 *np = reinterpret_cast<const float4 *>(nodes);
        float4 a = __ldg(np), b = __ldg(np + 1), c = __ldg(np + 2);
        int4 d = __ldg(reinterpret_cast<const int4 *>(np + 3));
        while (mask) {
            if (++nnode > max_visits) {
                if (lane == 0) atomicOr(status, ERR_INDEX);
                break;
            }
            const bool in = (mask >> lane) & 1u;
            const bool leaf0 = d.x < 0, leaf1 = d.y < 0;  // warp-uniform
            const float bk = fminf(heap_root_t(kb), tcap);
            const float thi = __fmaf_rn(fabsf(bk), 1e-5f, bk);
            float t0 = 0.0f, t1 = 0.0f;
#if FLARE_SLAB_FMA
            const bool h0 = in && slab_fma(a.x, a.y, a.z, a.w, b.x, b.y, niv, iv, tlo, thi, t0);
            const bool h1 = in && slab_fma(b.z, b.w, c.x, c.y, c.z, c.w, niv, iv, tlo, thi, t1);
#else
            const bool h0 = in && slab(a.x, a.y, a.z, a.w, b.x, b.y, O, iv, tlo, thi, t0);
            const bool h1 = in && slab(b.z, b.w, c.x, c.y, c.z, c.w, O, iv, tlo, thi, t1);
#endif
            const bool i0 = h0 && !leaf0, i1 = h1 && !leaf1;
            const unsigned m0 = __ballot_sync(0xffffffffu, i0), m1 = __ballot_sync(0xffffffffu, i1);
            int next = -1;
            unsigned nmask = 0;
            if (m0 && m1) {
                // nearer child first by lane vote (lanes that hit only one child vote for it)
                const unsigned v0 = __ballot_sync(0xffffffffu, i0 && (!i1 || t0 <= t1));
                const bool first0 = __popc(v0) * 2 >= __popc(m0 | m1);
                if (sp < TRACE_STACK) {
                    if (lane == 0) {
                        s_node[wib][sp] = first0 ? d.y : d.x;
                        s_mask[wib][sp] = first0 ? m1 : m0;
                    }
                    ++sp;
                } else if (lane == 0) {
                    atomicOr(status, ERR_STACK);
                }
                next = first0 ? d.x : d.y;
                nmask = first0 ? m0 : m1;
            } else if (m0) {
                next = d.x;
                nmask = m0;
            } else if (m1) {
                next = d.y;
                nmask = m1;
            } else {
                __syncwarp();
                if (sp > 0) {
                    --sp;
                    next = s_node[wib][sp];
                    nmask = s_mask[wib][sp];
                }
            }
            float4 na = a, nb = b, nc = c;
            int4 nd = d;
            if (next >= 0) {
                const float4 *nq = reinterpret_cast<const float4 *>(nodes + next);
                na = __ldg(nq);
                nb = __ldg(nq + 1);
                nc = __ldg(nq + 2);
                nd = __ldg(reinterpret_cast<const int4 *>(nq + 3));
            }
            if (leaf0 && h0) {
                float t;
                ++nprim;
                if (hit_prim(rec, ~d.x, O, v, t_min, poly, t, bk)) {
                    const int pid = d.z;
                    if (heap_accepts(kb, t, pid)) heap_insert(kb, t, pid);
                }
            }
            if (leaf1 && h1) {
                float t;
                ++nprim;
                if (hit_prim(rec, ~d.y, O, v, t_min, poly, t, bk)) {
                    const int pid = d.w;
                    if (heap_accepts(kb, t, pid)) heap_insert(kb, t, pid);
                }
            }
            __syncwarp();
            if (next < 0) break;
            node = next;
            mask = nmask;
            a = na;
            b = nb;
            c = nc;
            d = nd;
        }
    }
    if (PERSIST && phase == 1) {  // this chunk's largest K-th hit distance (+inf: a ray found fewer)
        float tk = live ? (kb.ri != 0x7fffffff ? kb.rt : INFINITY) : -INFINITY;
        for (int o = 16; o > 0; o >>= 1) tk = fmaxf(tk, __shfl_xor_sync(0xffffffffu, tk, o));
        if (lane == 0) __stcg(chunk_tk + chunk / FIRST_STRIDE, tk);
    }
    if (live) {  // heap sort into ascending slots
        heap_emit(kb, t_out, idx_out, stride, j);
    }
    __syncwarp();
    if (!PERSIST) break;
    }
    if (STATS) {
        for (int o = 16; o > 0; o >>= 1) nprim += __shfl_xor_sync(0xffffffffu, nprim, o);
        if (lane == 0 && (nprim | nnode)) {
            atomicAdd(stats + ST_PRIM_TESTS, nprim);
            atomicAdd(stats + ST_NODES, nnode);
        }
    }
}


// The persistent heap traversal over nodes with inline leaf records (NodeL): one 128-byte line per visit
// carries both child boxes or, for a leaf child, the primitive's whole record, so the exact hit test of a
// leaf needs no further fetch.  A leaf child is tested by every lane still tracing the node (the exact
// test rejects on t and on the polygon, so it subsumes the leaf box the 64-byte layout tests first); the
// next node's fetch is issued before the leaf tests.  Same hits, same order as trace_heap_kernel.
template <bool STATS, int K>
__global__ void __launch_bounds__(128, 5) trace_heapL_kernel(
    const float *__restrict__ O_, const float *__restrict__ v_, const float *__restrict__ tmin_,
    const int *__restrict__ ray_ids, int count, const NodeL *__restrict__ nodes, const float4 *__restrict__ rec,
    const int *__restrict__ ids, int n, float *__restrict__ t_out, int *__restrict__ idx_out, int stride,
    const PolyConst poly, int *__restrict__ status, unsigned long long *__restrict__ stats,
    const float *__restrict__ tmax_, int *__restrict__ chunk_ctr) {
    __shared__ int s_node[4][TRACE_STACK];
    __shared__ unsigned s_mask[4][TRACE_STACK];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    unsigned long long nprim = 0, nnode = 0;
    extern __shared__ __align__(16) unsigned char heap_smem[];
    while (true) {
        int b0 = 0;
        if (lane == 0) b0 = atomicAdd(chunk_ctr, 32);
        const int base = __shfl_sync(0xffffffffu, b0, 0);
        if (base >= count) break;
        const int j = base + lane;
        const bool live = j < count;
        int ray = live ? (ray_ids ? ray_ids[j] : j) : 0;
        float3 O = make_float3(0, 0, 0), v = make_float3(0, 0, 1);
        float t_min = INFINITY, tcap = INFINITY;
        if (live) {
            O = make_float3(O_[3 * (size_t)ray], O_[3 * (size_t)ray + 1], O_[3 * (size_t)ray + 2]);
            v = make_float3(v_[3 * (size_t)ray], v_[3 * (size_t)ray + 1], v_[3 * (size_t)ray + 2]);
            t_min = tmin_[ray];
            if (tmax_) tcap = nextafterf(tmax_[ray], -INFINITY);  // hits must lie before t_max
        }
        HeapBuf<K> kb;
        heap_init(kb, heap_smem);
        const float3 iv = make_float3(1.0f / (fabsf(v.x) > 1e-30f ? v.x : copysignf(1e-30f, v.x)),
                                      1.0f / (fabsf(v.y) > 1e-30f ? v.y : copysignf(1e-30f, v.y)),
                                      1.0f / (fabsf(v.z) > 1e-30f ? v.z : copysignf(1e-30f, v.z)));
        const float tlo = __fmaf_rn(-fabsf(t_min), 1e-5f, t_min);
        const bool want = live && t_min < INFINITY;
        if (n == 1) {
            float t;
            if (want) {
                ++nprim;
                if (hit_prim(rec, 0, O, v, t_min, poly, t, tcap)) heap_insert(kb, t, ids[0]);
            }
        } else if (n > 1) {
            unsigned mask = __ballot_sync(0xffffffffu, want);
            int sp = 0;
            const unsigned long long max_visits = 2ull * (unsigned long long)n + 64ull;
            float4 c[8];
            {
                const float4 *np = nodes[0].c;
#pragma unroll
                for (int k = 0; k < 8; ++k) c[k] = __ldg(np + k);
            }
            while (mask) {
                if (++nnode > max_visits) {
                    if (lane == 0) atomicOr(status, ERR_INDEX);
                    break;
                }
                const bool in = (mask >> lane) & 1u;
                const int link0 = __float_as_int(c[3].x), link1 = __float_as_int(c[7].x);
                const bool leaf0 = link0 < 0, leaf1 = link1 < 0;  // warp-uniform
                const float bk = fminf(heap_root_t(kb), tcap);
                const float thi = __fmaf_rn(fabsf(bk), 1e-5f, bk);
                float t0 = 0.0f, t1 = 0.0f;
                const bool i0 = in && !leaf0 && slab(c[0].x, c[0].y, c[0].z, c[0].w, c[1].x, c[1].y, O, iv, tlo, thi, t0);
                const bool i1 = in && !leaf1 && slab(c[4].x, c[4].y, c[4].z, c[4].w, c[5].x, c[5].y, O, iv, tlo, thi, t1);
                const unsigned m0 = __ballot_sync(0xffffffffu, i0), m1 = __ballot_sync(0xffffffffu, i1);
                int next = -1;
                unsigned nmask = 0;
                if (m0 && m1) {
                    const unsigned v0 = __ballot_sync(0xffffffffu, i0 && (!i1 || t0 <= t1));
                    const bool first0 = __popc(v0) * 2 >= __popc(m0 | m1);
                    if (sp < TRACE_STACK) {
                        if (lane == 0) {
                            s_node[wib][sp] = first0 ? link1 : link0;
                            s_mask[wib][sp] = first0 ? m1 : m0;
                        }
                        ++sp;
                    } else if (lane == 0) {
                        atomicOr(status, ERR_STACK);
                    }
                    next = first0 ? link0 : link1;
                    nmask = first0 ? m0 : m1;
                } else if (m0) {
                    next = link0;
                    nmask = m0;
                } else if (m1) {
                    next = link1;
                    nmask = m1;
                } else {
                    __syncwarp();
                    if (sp > 0) {
                        --sp;
                        next = s_node[wib][sp];
                        nmask = s_mask[wib][sp];
                    }
                }
                float4 nc[8];
                if (next >= 0) {
                    const float4 *nq = nodes[next].c;
#pragma unroll
                    for (int k = 0; k < 8; ++k) nc[k] = __ldg(nq + k);
                } else {
#pragma unroll
                    for (int k = 0; k < 8; ++k) nc[k] = c[k];
                }
                if (leaf0 && in) {
                    float t;
                    ++nprim;
                    if (hit_rec(c[0], c[1], c[2], O, v, t_min, poly, t, bk)) {
                        const int pid = __float_as_int(c[3].y);
                        if (heap_accepts(kb, t, pid)) heap_insert(kb, t, pid);
                    }
                }
                if (leaf1 && in) {
                    float t;
                    ++nprim;
                    if (hit_rec(c[4], c[5], c[6], O, v, t_min, poly, t, bk)) {
                        const int pid = __float_as_int(c[7].y);
                        if (heap_accepts(kb, t, pid)) heap_insert(kb, t, pid);
                    }
                }
                __syncwarp();
                if (next < 0) break;
                mask = nmask;
#pragma unroll
                for (int k = 0; k < 8; ++k) c[k] = nc[k];
            }
        }
        if (live) {  // heap sort into ascending slots
            heap_emit(kb, t_out, idx_out, stride, j);
        }
        __syncwarp();
    }
    if (STATS) {
        for (int o = 16; o > 0; o >>= 1) nprim += __shfl_xor_sync(0xffffffffu, nprim, o);
        if (lane == 0 && (nprim | nnode)) {
            atomicAdd(stats + ST_PRIM_TESTS, nprim);
            atomicAdd(stats + ST_NODES, nnode);
        }
    }
}


// The heap traversal over the 4-wide hierarchy: one 128-byte line per visit, four box tests per lane;
// entered internal children are visited nearest first (by the warp's nearest entry distance), the
// others pushed; the next node's fetch is issued before this node's leaf tests.  The stack holds node
// indices only: a popped node is tested by every lane still tracing (a lane that missed its box misses
// its children too, the children's boxes lying inside it).
__device__ __forceinline__ bool slab4(float lx, float ly, float lz, float hx, float hy, float hz, float3 O, float3 iv,
                                      float tlo, float thi, float &tnear) {
    return slab(lx, ly, lz, hx, hy, hz, O, iv, tlo, thi, tnear);
}

template <bool STATS, int K>
__global__ void __launch_bounds__(128, 5) trace_heap4_kernel(
    const float *__restrict__ O_, const float *__restrict__ v_, const float *__restrict__ tmin_,
    const int *__restrict__ ray_ids, int count, const Node4 *__restrict__ nodes, const float4 *__restrict__ rec,
    const int *__restrict__ ids, int n, float *__restrict__ t_out, int *__restrict__ idx_out, int stride,
    const PolyConst poly, int *__restrict__ status, unsigned long long *__restrict__ stats,
    const float *__restrict__ tmax_ = nullptr) {
    constexpr int STACK4 = 128;
    __shared__ int s_node[4][STACK4];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    const bool live = j < count;
    unsigned long long nprim = 0, nnode = 0;
    int ray = live ? (ray_ids ? ray_ids[j] : j) : 0;
    float3 O = make_float3(0, 0, 0), v = make_float3(0, 0, 1);
    float t_min = INFINITY, tcap = INFINITY;
    if (live) {
        O = make_float3(O_[3 * (size_t)ray], O_[3 * (size_t)ray + 1], O_[3 * (size_t)ray + 2]);
        v = make_float3(v_[3 * (size_t)ray], v_[3 * (size_t)ray + 1], v_[3 * (size_t)ray + 2]);
        t_min = tmin_[ray];
        if (tmax_) tcap = nextafterf(tmax_[ray], -INFINITY);  // hits must lie before t_max
    }
    extern __shared__ __align__(16) unsigned char heap_smem[];
    HeapBuf<K> kb;
    heap_init(kb, heap_smem);
    const float3 iv = make_float3(1.0f / (fabsf(v.x) > 1e-30f ? v.x : copysignf(1e-30f, v.x)),
                                  1.0f / (fabsf(v.y) > 1e-30f ? v.y : copysignf(1e-30f, v.y)),
                                  1.0f / (fabsf(v.z) > 1e-30f ? v.z : copysignf(1e-30f, v.z)));
    const float tlo = __fmaf_rn(-fabsf(t_min), 1e-5f, t_min);
    const bool want = live && t_min < INFINITY;
    if (n == 1) {
        float t;
        if (want) {
            ++nprim;
            if (hit_prim(rec, 0, O, v, t_min, poly, t, tcap)) heap_insert(kb, t, ids[0]);
        }
    } else if (n > 1) {
        const unsigned all = __ballot_sync(0xffffffffu, want);
        unsigned mask = all;
        int sp = 0;
        const unsigned long long max_visits = 2ull * (unsigned long long)n + 64ull;
        const float4 *np = reinterpret_cast<const float4 *>(nodes);
        float4 lx = __ldg(np), ly = __ldg(np + 1), lz = __ldg(np + 2), hx = __ldg(np + 3), hy = __ldg(np + 4),
               hz = __ldg(np + 5);
        int4 ln = __ldg(reinterpret_cast<const int4 *>(np + 6)), pd = __ldg(reinterpret_cast<const int4 *>(np + 7));
        while (mask) {
            if (++nnode > max_visits) {
                if (lane == 0) atomicOr(status, ERR_INDEX);
                break;
            }
            const bool in = (mask >> lane) & 1u;
            const float bk = fminf(heap_root_t(kb), tcap);
            const float thi = __fmaf_rn(fabsf(bk), 1e-5f, bk);
            const float clx[4] = {lx.x, lx.y, lx.z, lx.w}, cly[4] = {ly.x, ly.y, ly.z, ly.w},
                        clz[4] = {lz.x, lz.y, lz.z, lz.w}, chx[4] = {hx.x, hx.y, hx.z, hx.w},
                        chy[4] = {hy.x, hy.y, hy.z, hy.w}, chz[4] = {hz.x, hz.y, hz.z, hz.w};
            const int link[4] = {ln.x, ln.y, ln.z, ln.w};
            bool h[4];
            unsigned key[4], im[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                float tn = 0.0f;
                h[c] = in && link[c] != NODE4_EMPTY && slab4(clx[c], cly[c], clz[c], chx[c], chy[c], chz[c], O, iv, tlo, thi, tn);
                const bool ic = h[c] && link[c] >= 0;  // empty slots never have h set
                im[c] = __ballot_sync(0xffffffffu, ic);
                // nearest entry among the lanes entering the child (entries are >= 0 here, so their bit
                // patterns order like the values)
                key[c] = im[c] ? __reduce_min_sync(0xffffffffu, ic ? __float_as_uint(fmaxf(tn, 0.0f)) : 0xffffffffu)
                               : 0xffffffffu;
            }
            // order the entered internal children by key: push all but the nearest, farthest first
            int order[4] = {0, 1, 2, 3};
#pragma unroll
            for (int a = 0; a < 3; ++a)
#pragma unroll
                for (int b = 0; b < 3 - a; ++b)
                    if (key[order[b]] < key[order[b + 1]]) {  // descending: farthest first
                        const int tmp = order[b];
                        order[b] = order[b + 1];
                        order[b + 1] = tmp;
                    }
            int next = -1;
            unsigned nmask = 0;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int c = order[q];
                if (!im[c]) continue;
                if (next >= 0) {  // the previous nearer candidate goes to the stack
                    if (sp < STACK4) {
                        if (lane == 0) s_node[wib][sp] = next;
                        ++sp;
                    } else if (lane == 0) {
                        atomicOr(status, ERR_STACK);
                    }
                }
                next = link[c];
                nmask = im[c];
            }
            if (next < 0) {
                __syncwarp();
                if (sp > 0) {
                    --sp;
                    next = s_node[wib][sp];
                    nmask = all;
                }
            }
            const int4 pid = pd;
            float4 nlx = lx, nly = ly, nlz = lz, nhx = hx, nhy = hy, nhz = hz;
            int4 nln = ln, npd = pd;
            if (next >= 0) {
                const float4 *q = reinterpret_cast<const float4 *>(nodes + next);
                nlx = __ldg(q); nly = __ldg(q + 1); nlz = __ldg(q + 2);
                nhx = __ldg(q + 3); nhy = __ldg(q + 4); nhz = __ldg(q + 5);
                nln = __ldg(reinterpret_cast<const int4 *>(q + 6));
                npd = __ldg(reinterpret_cast<const int4 *>(q + 7));
            }
            const int pids[4] = {pid.x, pid.y, pid.z, pid.w};
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                if (link[c] < 0 && h[c]) {
                    float t;
                    ++nprim;
                    if (hit_prim(rec, ~link[c], O, v, t_min, poly, t, bk)) {
                        const int p = pids[c];
                        if (heap_accepts(kb, t, p)) heap_insert(kb, t, p);
                    }
                }
            }
            __syncwarp();
            if (next < 0) break;
            mask = nmask;
            lx = nlx; ly = nly; lz = nlz; hx = nhx; hy = nhy; hz = nhz;
            ln = nln; pd = npd;
        }
    }
    if (live) {  // heap sort into ascending slots
        heap_emit(kb, t_out, idx_out, stride, j);
    }
    if (STATS) {
        for (int o = 16; o > 0; o >>= 1) nprim += __shfl_xor_sync(0xffffffffu, nprim, o);
        if (lane == 0 && (nprim | nnode)) {
            atomicAdd(stats + ST_PRIM_TESTS, nprim);
            atomicAdd(stats + ST_NODES, nnode);
        }
    }
}

// Group-per-ray traversal for sparse late passes: once few rays remain, a pass lasts as long as its
// longest single walk, so G lanes (a quarter, half or whole warp) split one ray's walk.  Each step the
// group pops up to G nodes of its shared stack, tests their children and pushes the entered internal
// ones; a leaf is tested by the lane that met it, into that lane's own K-buffer.  The pruning bound is
// the group minimum of the lanes' K-th hits: the ray's K-th nearest hit over all lanes lies no farther
// than any one lane's K-th.  At the end a group merge emits the K nearest (t, index) entries in order.
constexpr int WIDE_WARP_STACK = 2048;  // stack entries per warp, split evenly between its rays

__device__ __forceinline__ bool key_less(float ta, int ia, float tb, int ib) {
    return ta < tb || (ta == tb && ia < ib);
}

template <int K, int G>
__global__ void __launch_bounds__(128) trace_group_kernel(
    const float *__restrict__ O_, const float *__restrict__ v_, const float *__restrict__ tmin_,
    const int *__restrict__ ray_ids, int count, const Node *__restrict__ nodes, const float4 *__restrict__ rec,
    const int *__restrict__ ids, int n, float *__restrict__ t_out, int *__restrict__ idx_out, int stride,
    const PolyConst poly, int *__restrict__ status, unsigned long long *__restrict__ stats,
    const float *__restrict__ tmax_ = nullptr) {
    static_assert(G == 8 || G == 16 || G == 32, "group of 8, 16 or 32 lanes");
    constexpr int CAP = WIDE_WARP_STACK * G / 32;
    __shared__ int s_stack[4][WIDE_WARP_STACK];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int gl = lane % G, gid = lane / G;                 // lane within the group, group within the warp
    const unsigned gmask = (G == 32 ? 0xffffffffu : ((1u << G) - 1u) << (gid * G));
    const int j = (blockIdx.x * 4 + wib) * (32 / G) + gid;  // this group's ray slot
    const bool live = j < count;
    const unsigned lt_mask = (1u << gl) - 1u;
    const int ray = live ? (ray_ids ? ray_ids[j] : j) : 0;
    float3 O = make_float3(0, 0, 0), v = make_float3(0, 0, 1);
    float t_min = INFINITY, tcap = INFINITY;
    if (live) {
        O = make_float3(O_[3 * (size_t)ray], O_[3 * (size_t)ray + 1], O_[3 * (size_t)ray + 2]);
        v = make_float3(v_[3 * (size_t)ray], v_[3 * (size_t)ray + 1], v_[3 * (size_t)ray + 2]);
        t_min = tmin_[ray];
        if (tmax_) tcap = nextafterf(tmax_[ray], -INFINITY);  // hits must lie before t_max
    }
    unsigned long long nprim = 0, nnode = 0;
    KBuf<K> kb;
#pragma unroll
    for (int k = 0; k < K; ++k) {
        kb.t[k] = INFINITY;
        kb.i[k] = 0x7fffffff;
    }
    const float3 iv = make_float3(1.0f / (fabsf(v.x) > 1e-30f ? v.x : copysignf(1e-30f, v.x)),
                                  1.0f / (fabsf(v.y) > 1e-30f ? v.y : copysignf(1e-30f, v.y)),
                                  1.0f / (fabsf(v.z) > 1e-30f ? v.z : copysignf(1e-30f, v.z)));
    const float tlo = __fmaf_rn(-fabsf(t_min), 1e-5f, t_min);
    if (n == 1) {
        float t;
        if (gl == 0 && t_min < INFINITY) {
            ++nprim;
            if (hit_prim(rec, 0, O, v, t_min, poly, t, tcap)) kbuf_insert(kb, t, ids[0]);
        }
    } else if (n > 1) {
        int *stack = s_stack[wib] + gid * CAP;
        int sp = t_min < INFINITY ? 1 : 0;  // uniform within the group
        if (gl == 0) stack[0] = 0;
        const unsigned long long max_steps = 2ull * (unsigned long long)n + 64ull;
        unsigned long long steps = 0;
        __syncwarp();
        // the whole warp steps together (shuffles and ballots span it); a group with an empty stack idles
        while (__any_sync(0xffffffffu, sp > 0)) {
            if (++steps > max_steps) {
                if (lane == 0) atomicOr(status, ERR_INDEX);
                break;
            }
            const int take = min(G, sp);
            const int node = gl < take ? stack[sp - 1 - gl] : -1;
            sp -= take;
            float bound = fminf(kb.t[K - 1], tcap);
#pragma unroll
            for (int o = G / 2; o > 0; o >>= 1) bound = fminf(bound, __shfl_xor_sync(0xffffffffu, bound, o));
            bool push_near = false, push_far = false;
            int near_c = 0, far_c = 0;
            if (node >= 0) {
                ++nnode;
                const float thi = __fmaf_rn(fabsf(bound), 1e-5f, bound);
                const float4 *np = reinterpret_cast<const float4 *>(nodes + node);
                const float4 a = __ldg(np), b = __ldg(np + 1), c = __ldg(np + 2);
                const int4 d = __ldg(reinterpret_cast<const int4 *>(np + 3));
                float t0 = 0.0f, t1 = 0.0f;
                bool h0 = slab(a.x, a.y, a.z, a.w, b.x, b.y, O, iv, tlo, thi, t0);
                bool h1 = slab(b.z, b.w, c.x, c.y, c.z, c.w, O, iv, tlo, thi, t1);
                if (d.x < 0) {
                    if (h0) {
                        float t;
                        ++nprim;
                        if (hit_prim(rec, ~d.x, O, v, t_min, poly, t, bound)) {
                            const int pid = d.z;
                            if (key_less(t, pid, kb.t[K - 1], kb.i[K - 1])) kbuf_insert(kb, t, pid);
                        }
                    }
                    h0 = false;
                }
                if (d.y < 0) {
                    if (h1) {
                        float t;
                        ++nprim;
                        if (hit_prim(rec, ~d.y, O, v, t_min, poly, t, bound)) {
                            const int pid = d.w;
                            if (key_less(t, pid, kb.t[K - 1], kb.i[K - 1])) kbuf_insert(kb, t, pid);
                        }
                    }
                    h1 = false;
                }
                // the nearer child goes on top of the stack (pushed last)
                const bool first0 = !h1 || (h0 && t0 <= t1);
                push_near = h0 || h1;
                push_far = h0 && h1;
                near_c = first0 ? d.x : d.y;
                far_c = first0 ? d.y : d.x;
            }
            const unsigned bf = (__ballot_sync(0xffffffffu, push_far) & gmask) >> (gid * G);
            const unsigned bn = (__ballot_sync(0xffffffffu, push_near) & gmask) >> (gid * G);
            const int nf = __popc(bf), nn = __popc(bn);
            if (sp + nf + nn > CAP) {
                if (gl == 0) atomicOr(status, ERR_STACK);
                sp = 0;  // this ray's list is incomplete; the error bit reports it
            } else {
                if (push_far) stack[sp + __popc(bf & lt_mask)] = far_c;
                if (push_near) stack[sp + nf + __popc(bn & lt_mask)] = near_c;
                sp += nf + nn;
            }
            __syncwarp();
        }
    }
    // merge: K rounds of a group argmin over the lanes' buffer heads
    for (int k = 0; k < K; ++k) {
        float bt = kb.t[0];
        int bi = kb.i[0];
#pragma unroll
        for (int o = G / 2; o > 0; o >>= 1) {
            const float ot = __shfl_xor_sync(0xffffffffu, bt, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (key_less(ot, oi, bt, bi)) {
                bt = ot;
                bi = oi;
            }
        }
        if (gl == 0 && live) {
            const bool valid = bi != 0x7fffffff;
            t_out[(size_t)k * stride + j] = valid ? bt : INFINITY;
            idx_out[(size_t)k * stride + j] = valid ? bi : -1;
        }
        if (bi != 0x7fffffff && kb.i[0] == bi && kb.t[0] == bt) {  // the winning lane drops its head
#pragma unroll
            for (int q = 0; q < K - 1; ++q) {
                kb.t[q] = kb.t[q + 1];
                kb.i[q] = kb.i[q + 1];
            }
            kb.t[K - 1] = INFINITY;
            kb.i[K - 1] = 0x7fffffff;
        }
    }
    if (stats) {
        for (int o = 16; o > 0; o >>= 1) {
            nprim += __shfl_xor_sync(0xffffffffu, nprim, o);
            nnode += __shfl_xor_sync(0xffffffffu, nnode, o);
        }
        if (lane == 0 && (nprim | nnode)) {
            atomicAdd(stats + ST_PRIM_TESTS, nprim);
            atomicAdd(stats + ST_NODES, nnode);
        }
    }
}

// ------------------------------------------------------------------------------------------------
// Ray ordering: rays are visited in the order of a 64-bit key, origin Morton code (30 bits, within the
// batch's origin bounds) above the Morton code of the octahedral direction (2 x 16 bits), so the 32 rays
// of a packet are neighbours in origin and direction whatever order the caller passed them in.
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ int ord_f(float f) {
    int i = __float_as_int(f);
    return i >= 0 ? i : i ^ 0x7FFFFFFF;
}
__device__ __forceinline__ float ord_inv(int i) { return __int_as_float(i >= 0 ? i : i ^ 0x7FFFFFFF); }

__global__ void origin_bounds_kernel(const float *__restrict__ O, int R, int *__restrict__ bounds) {
    float lo[3] = {INFINITY, INFINITY, INFINITY}, hi[3] = {-INFINITY, -INFINITY, -INFINITY};
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < R; i += gridDim.x * blockDim.x)
        for (int a = 0; a < 3; ++a) {
            float x = O[3 * (size_t)i + a];
            lo[a] = fminf(lo[a], x);
            hi[a] = fmaxf(hi[a], x);
        }
    for (int a = 0; a < 3; ++a)
        for (int o = 16; o > 0; o >>= 1) {
            lo[a] = fminf(lo[a], __shfl_xor_sync(0xffffffffu, lo[a], o));
            hi[a] = fmaxf(hi[a], __shfl_xor_sync(0xffffffffu, hi[a], o));
        }
    if ((threadIdx.x & 31) == 0 && lo[0] <= hi[0])
        for (int a = 0; a < 3; ++a) {
            atomicMin(bounds + a, ord_f(lo[a]));
            atomicMax(bounds + 3 + a, ord_f(hi[a]));
        }
}

__device__ __forceinline__ unsigned long long spread16(unsigned x) {
    unsigned long long v = x & 0xFFFFu;
    v = (v | (v << 8)) & 0x00FF00FFull;
    v = (v | (v << 4)) & 0x0F0F0F0Full;
    v = (v | (v << 2)) & 0x33333333ull;
    v = (v | (v << 1)) & 0x55555555ull;
    return v;
}
__device__ __forceinline__ unsigned spread10(unsigned v) {
    v = (v * 0x00010001u) & 0xFF0000FFu;
    v = (v * 0x00000101u) & 0x0F00F00Fu;
    v = (v * 0x00000011u) & 0xC30C30C3u;
    v = (v * 0x00000005u) & 0x49249249u;
    return v;
}

__global__ void ray_key_kernel(const float *__restrict__ O, const float *__restrict__ v, int R,
                               const int *__restrict__ bounds, unsigned long long *__restrict__ keys,
                               int *__restrict__ ids) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= R) return;
    unsigned oc = 0;
    for (int a = 0; a < 3; ++a) {
        float lo = ord_inv(bounds[a]), hi = ord_inv(bounds[3 + a]);
        float x = hi > lo ? (O[3 * (size_t)i + a] - lo) / (hi - lo) : 0.5f;
        oc |= spread10((unsigned)fminf(fmaxf(x * 1024.0f, 0.0f), 1023.0f)) << (2 - a);
    }
    float dx = v[3 * (size_t)i], dy = v[3 * (size_t)i + 1], dz = v[3 * (size_t)i + 2];
    float l1 = fabsf(dx) + fabsf(dy) + fabsf(dz);
    float px = l1 > 0.0f ? dx / l1 : 0.0f, py = l1 > 0.0f ? dy / l1 : 0.0f;
    if (dz < 0.0f) {  // octahedral fold of the lower hemisphere
        float qx = (1.0f - fabsf(py)) * copysignf(1.0f, px), qy = (1.0f - fabsf(px)) * copysignf(1.0f, py);
        px = qx;
        py = qy;
    }
    unsigned ux = (unsigned)fminf(fmaxf((px * 0.5f + 0.5f) * 65536.0f, 0.0f), 65535.0f);
    unsigned uy = (unsigned)fminf(fmaxf((py * 0.5f + 0.5f) * 65536.0f, 0.0f), 65535.0f);
    keys[i] = ((unsigned long long)oc << 32) | (spread16(ux) << 1) | spread16(uy);
    ids[i] = i;
}

__global__ void init_bounds6_kernel(int *b) {
    if (threadIdx.x < 3) b[threadIdx.x] = 0x7FFFFFFF;
    else if (threadIdx.x < 6) b[threadIdx.x] = (int)0x80000000;
}

int order_rays(flare_renderer *r, const float *O, const float *v, int R, int *list_out, cudaStream_t st) {
    if (R <= 1) return FLARE_OK;
    int *bounds = reinterpret_cast<int *>(r->bounds) + 8;
    init_bounds6_kernel<<<1, 32, 0, st>>>(bounds);
    origin_bounds_kernel<<<std::min((R + 255) / 256, 1184), 256, 0, st>>>(O, R, bounds);
    ray_key_kernel<<<(R + 255) / 256, 256, 0, st>>>(O, v, R, bounds, r->ray_keys, r->ray_ids_tmp);
    size_t tmp = r->ray_sort_tmp_bytes;
    FLARE_CUDA_TRY(cub::DeviceRadixSort::SortPairs(r->ray_sort_tmp, tmp, r->ray_keys, r->ray_keys + r->max_rays,
                                                   r->ray_ids_tmp, list_out, R, 0, 64, st));
    FLARE_CUDA_TRY(cudaGetLastError());
    return FLARE_OK;
}

// Keeps the active rays of a pass in list order (a stable select on the shading kernel's per-slot
// flags), so each 32-ray traversal packet of the next pass is a run of the first pass's coherence order;
// the count goes to r->counters[0].
int compact_active(flare_renderer *r, const int *list_in, int count, int *list_out, cudaStream_t st) {
    size_t tmp = r->select_tmp_bytes;
    FLARE_CUDA_TRY(cub::DeviceSelect::Flagged(r->select_tmp, tmp, list_in, r->pass_flags, list_out, r->counters, count,
                                              st));
    FLARE_CUDA_TRY(cudaGetLastError());
    return FLARE_OK;
}

size_t select_temp_bytes(int max_rays) {
    size_t tmp = 0;
    cub::DeviceSelect::Flagged(nullptr, tmp, (const int *)nullptr, (const unsigned char *)nullptr, (int *)nullptr,
                               (int *)nullptr, max_rays, (cudaStream_t)0);
    return tmp;
}

size_t ray_sort_temp_bytes(int max_rays) {
    size_t tmp = 0;
    cub::DeviceRadixSort::SortPairs(nullptr, tmp, (unsigned long long *)nullptr, (unsigned long long *)nullptr,
                                    (int *)nullptr, (int *)nullptr, max_rays, 0, 64, (cudaStream_t)0);
    return tmp;
}

static int getenv_int(const char *name, int dflt) {
    const char *e = getenv(name);
    return e ? atoi(e) : dflt;
}

int launch_trace(flare_renderer *r, const float *O, const float *v, const float *t_min, const int *ray_ids,
                 int count, float *t_out, int *idx_out, int out_stride, cudaStream_t st, int k,
                 const float *t_max, bool first) {
    if (count <= 0) return FLARE_OK;
    const int B = 128;
    // Sparse passes: G lanes per ray, G chosen so the pass still spreads over the whole GPU
    static const int g32_max = getenv_int("FLARE_TRACE_G32_MAX", 16384);
    static const int g16_max = getenv_int("FLARE_TRACE_G16_MAX", 0);
    static const int g8_max = getenv_int("FLARE_TRACE_G8_MAX", 0);
    if (k == K_PASS && K_PASS != K_HITS && (count <= g32_max || count <= g16_max || count <= g8_max)) {
        if (count <= g32_max)
            trace_group_kernel<K_PASS, 32><<<(count + 3) / 4, B, 0, st>>>(
                O, v, t_min, ray_ids, count, r->nodes, r->rec, r->ids_sorted, r->n, t_out, idx_out, out_stride, r->poly,
                r->dstatus, r->dstats, t_max);
        else if (count <= g16_max)
            trace_group_kernel<K_PASS, 16><<<(count + 7) / 8, B, 0, st>>>(
                O, v, t_min, ray_ids, count, r->nodes, r->rec, r->ids_sorted, r->n, t_out, idx_out, out_stride, r->poly,
                r->dstatus, r->dstats, t_max);
        else
            trace_group_kernel<K_PASS, 8><<<(count + 15) / 16, B, 0, st>>>(
                O, v, t_min, ray_ids, count, r->nodes, r->rec, r->ids_sorted, r->n, t_out, idx_out, out_stride, r->poly,
                r->dstatus, r->dstats, t_max);
        FLARE_CUDA_TRY(cudaGetLastError());
        return FLARE_OK;
    }
    // Internal passes keep each ray's K_PASS-entry buffer as a shared-memory heap (FLARE_TRACE_HEAP=0: the
    // sorted register buffer of the packet kernel).
    static const bool heap = getenv_int("FLARE_TRACE_HEAP", 1) != 0;
    if (k == K_PASS && K_PASS != K_HITS && heap && r->nodes4) {
        const size_t smem = (size_t)K_PASS * 128 * 8;
        FLARE_CUDA_TRY(cudaFuncSetAttribute(trace_heap4_kernel<true, K_PASS>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        trace_heap4_kernel<true, K_PASS><<<(count + B - 1) / B, B, smem, st>>>(
            O, v, t_min, ray_ids, count, r->nodes4, r->rec, r->ids_sorted, r->n, t_out, idx_out, out_stride, r->poly,
            r->dstatus, r->dstats, t_max);
        FLARE_CUDA_TRY(cudaGetLastError());
        return FLARE_OK;
    }
    static const bool persist = getenv_int("FLARE_TRACE_PERSIST", 1) != 0;
    if (k == K_PASS && K_PASS != K_HITS && heap && persist && r->nodesL) {
        const size_t smem = (size_t)K_PASS * 128 * 8;
        FLARE_CUDA_TRY(cudaFuncSetAttribute(trace_heapL_kernel<true, K_PASS>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        int per_sm = 0;
        FLARE_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, trace_heapL_kernel<true, K_PASS>, B,
                                                                     smem));
        const int grid = std::max(1, std::min((count + B - 1) / B, r->num_sms * std::max(per_sm, 1)));
        FLARE_CUDA_TRY(cudaMemsetAsync(r->counters + 2, 0, sizeof(int), st));
        trace_heapL_kernel<true, K_PASS><<<grid, B, smem, st>>>(
            O, v, t_min, ray_ids, count, r->nodesL, r->rec, r->ids_sorted, r->n, t_out, idx_out, out_stride, r->poly,
            r->dstatus, r->dstats, t_max, r->counters + 2);
        FLARE_CUDA_TRY(cudaGetLastError());
        return FLARE_OK;
    }
    if (k == K_PASS && K_PASS != K_HITS && heap && persist) {
        const size_t smem = (size_t)K_PASS * 128 * 8;
        FLARE_CUDA_TRY(cudaFuncSetAttribute(trace_heap_kernel<true, K_PASS, true>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        int per_sm = 0;
        FLARE_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, trace_heap_kernel<true, K_PASS, true>, B,
                                                                     smem));
        const int grid = std::max(1, std::min((count + B - 1) / B, r->num_sms * std::max(per_sm, 1)));
        static const bool first_phases = getenv_int("FLARE_FIRST_BOUND", 1) != 0;
        if (first && t_max && first_phases && count >= 65536 && r->chunk_tk) {
            // a first pass in two phases (see trace_heap_kernel): sparse chunks, then the rest bounded
            for (int phase = 1; phase <= 2; ++phase) {
                FLARE_CUDA_TRY(cudaMemsetAsync(r->counters + 2, 0, sizeof(int), st));
                trace_heap_kernel<true, K_PASS, true><<<grid, B, smem, st>>>(
                    O, v, t_min, ray_ids, count, r->nodes, r->rec, r->ids_sorted, r->n, t_out, idx_out, out_stride,
                    r->poly, r->dstatus, r->dstats, t_max, r->counters + 2, phase, r->chunk_tk,
                    const_cast<float *>(t_max));
                FLARE_CUDA_TRY(cudaGetLastError());
            }
            return FLARE_OK;
        }
        FLARE_CUDA_TRY(cudaMemsetAsync(r->counters + 2, 0, sizeof(int), st));
        trace_heap_kernel<true, K_PASS, true><<<grid, B, smem, st>>>(
            O, v, t_min, ray_ids, count, r->nodes, r->rec, r->ids_sorted, r->n, t_out, idx_out, out_stride, r->poly,
            r->dstatus, r->dstats, t_max, r->counters + 2);
        FLARE_CUDA_TRY(cudaGetLastError());
        return FLARE_OK;
    }
    if (k == K_PASS && K_PASS != K_HITS && heap) {
        const size_t smem = (size_t)K_PASS * 128 * 8;
        FLARE_CUDA_TRY(cudaFuncSetAttribute(trace_heap_kernel<true, K_PASS, false>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        trace_heap_kernel<true, K_PASS, false><<<(count + B - 1) / B, B, smem, st>>>(
            O, v, t_min, ray_ids, count, r->nodes, r->rec, r->ids_sorted, r->n, t_out, idx_out, out_stride, r->poly,
            r->dstatus, r->dstats, t_max);
        FLARE_CUDA_TRY(cudaGetLastError());
        return FLARE_OK;
    }
    if (k == K_PASS && K_PASS != K_HITS) {
        trace_packet_kernel<true, K_PASS><<<(count + B - 1) / B, B, 0, st>>>(O, v, t_min, ray_ids, count, r->nodes,
                                                                             r->rec, r->ids_sorted, r->n, t_out,
                                                                             idx_out, out_stride, r->poly, r->dstatus,
                                                                             r->dstats, t_max);
        FLARE_CUDA_TRY(cudaGetLastError());
        return FLARE_OK;
    }
    trace_packet_kernel<true, K_HITS><<<(count + B - 1) / B, B, 0, st>>>(O, v, t_min, ray_ids, count, r->nodes, r->rec,
                                                           r->ids_sorted, r->n, t_out, idx_out, out_stride, r->poly,
                                                           r->dstatus, r->dstats, t_max);
    FLARE_CUDA_TRY(cudaGetLastError());
    return FLARE_OK;
}

// The same traversal over explicit geometry (used by the allocation-free entry point in noalloc.cu).
int launch_trace_geom(const Node *nodes, const float4 *rec, const int *ids_sorted, int n, const PolyConst &poly,
                      const float *O, const float *v, const float *t_min, int count, float *t_out, int *idx_out,
                      int *status, cudaStream_t st) {
    if (count <= 0) return FLARE_OK;
    const int B = 128;
    trace_packet_kernel<false, K_HITS><<<(count + B - 1) / B, B, 0, st>>>(O, v, t_min, nullptr, count, nodes, rec, ids_sorted,
                                                                   n, t_out, idx_out, count, poly, status, nullptr);
    FLARE_CUDA_TRY(cudaGetLastError());
    return FLARE_OK;
}

}  // namespace flare


#ifdef FLARE_TRACE_WHY
// Diagnostic build only (-DFLARE_TRACE_WHY): failed primitive tests by reason since the last reset:
// [0] t before t_min, [1] t beyond the current K-th hit, [2] outside the polygon.
extern "C" int flare_debug_why(unsigned long long *out, int reset) {
    FLARE_CUDA_TRY(cudaDeviceSynchronize());
    FLARE_CUDA_TRY(cudaMemcpyFromSymbol(out, flare::g_why, 3 * sizeof(unsigned long long)));
    if (reset) {
        unsigned long long z[4] = {0, 0, 0, 0};
        FLARE_CUDA_TRY(cudaMemcpyToSymbol(flare::g_why, z, sizeof(z)));
    }
    return 0;
}
#endif
