// trace.cu -- k-nearest proxy traversal (replaces the reference's OptiX raygen + any-hit programs,
// source/renderer/shaders.cu:81-189, and the diagnostic raygen used by Render, shaders.cu:19-77).
//
// One thread per ray walks the LBVH with a short local stack, nearer child first, and keeps the 16
// smallest (t, primitive index) hits with t >= t_min in a register-resident sorted buffer (the
// reference's any-hit insertion sort, shaders.cu:166-188, with ties broken by the smaller index so
// the result is independent of traversal order).  A subtree is pruned when its box entry lies beyond
// the current 16th hit.  Nodes are 64-byte records read as four 16-byte loads; primitive records are
// 48 bytes in Morton order read as three 16-byte loads.
//
// The hit test is exact fp32 with explicit rounding intrinsics; oracle/trace_oracle.c executes the
// identical sequence, which is what makes hit lists bit-comparable.
#include "renderer.cuh"

namespace flare {

struct KBuf {
    float t[K_HITS];
    int i[K_HITS];
};

__device__ __forceinline__ void kbuf_insert(KBuf &b, float t, int id) {
    float ct = t;
    int ci = id;
#pragma unroll
    for (int k = 0; k < K_HITS; ++k) {
        bool sw = (ct < b.t[k]) || (ct == b.t[k] && ci < b.i[k]);
        float tt = b.t[k];
        int ii = b.i[k];
        b.t[k] = sw ? ct : tt;
        b.i[k] = sw ? ci : ii;
        ct = sw ? tt : ct;
        ci = sw ? ii : ci;
    }
}

// Exact hit test on the record of sorted primitive p (same operation order as the oracle).
__device__ __forceinline__ bool hit_prim(const float4 *__restrict__ rec, int p, float3 O, float3 v, float t_min,
                                         const PolyConst &c_poly, float &t_out) {
    float4 r0 = __ldg(rec + 3 * (size_t)p), r1 = __ldg(rec + 3 * (size_t)p + 1), r2 = __ldg(rec + 3 * (size_t)p + 2);
    // r0 = m.xyz N.x, r1 = N.yz Ua.xy, r2 = Ua.z Va.xyz
    float dx = __fsub_rn(r0.x, O.x), dy = __fsub_rn(r0.y, O.y), dz = __fsub_rn(r0.z, O.z);
    float num = __fmaf_rn(r0.w, dx, __fmaf_rn(r1.x, dy, __fmul_rn(r1.y, dz)));
    float den = __fmaf_rn(r0.w, v.x, __fmaf_rn(r1.x, v.y, __fmul_rn(r1.y, v.z)));
    float t = __fdiv_rn(num, den);
    if (!(t >= t_min)) return false;
    float ex = __fsub_rn(__fmaf_rn(v.x, t, O.x), r0.x);
    float ey = __fsub_rn(__fmaf_rn(v.y, t, O.y), r0.y);
    float ez = __fsub_rn(__fmaf_rn(v.z, t, O.z), r0.z);
    float a = __fmaf_rn(r1.z, ex, __fmaf_rn(r1.w, ey, __fmul_rn(r2.x, ez)));
    float b = __fmaf_rn(r2.y, ex, __fmaf_rn(r2.z, ey, __fmul_rn(r2.w, ez)));
    const int ns = c_poly.n;
    for (int j = 0; j < ns; ++j)
        if (!(__fmaf_rn(c_poly.c[j], a, __fmul_rn(c_poly.s[j], b)) <= 1.0f)) return false;
    t_out = t;
    return true;
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

template <bool STATS>
__global__ void __launch_bounds__(128) trace_kernel(const float *__restrict__ O_, const float *__restrict__ v_,
                                                    const float *__restrict__ tmin_, const int *__restrict__ ray_ids,
                                                    int count, const Node *__restrict__ nodes,
                                                    const float4 *__restrict__ rec, const int *__restrict__ ids,
                                                    int n, float *__restrict__ t_out, int *__restrict__ idx_out,
                                                    int stride, const PolyConst poly, int *__restrict__ status,
                                                    unsigned long long *__restrict__ stats) {
    int j = blockIdx.x * blockDim.x + threadIdx.x;
    unsigned long long nprim = 0, nnode = 0;
    if (j < count) {
        int ray = ray_ids ? ray_ids[j] : j;
        float3 O = make_float3(O_[3 * (size_t)ray], O_[3 * (size_t)ray + 1], O_[3 * (size_t)ray + 2]);
        float3 v = make_float3(v_[3 * (size_t)ray], v_[3 * (size_t)ray + 1], v_[3 * (size_t)ray + 2]);
        float t_min = tmin_[ray];
        KBuf kb;
#pragma unroll
        for (int k = 0; k < K_HITS; ++k) {
            kb.t[k] = INFINITY;
            kb.i[k] = 0x7fffffff;
        }
        float3 iv = make_float3(1.0f / (fabsf(v.x) > 1e-30f ? v.x : copysignf(1e-30f, v.x)),
                                1.0f / (fabsf(v.y) > 1e-30f ? v.y : copysignf(1e-30f, v.y)),
                                1.0f / (fabsf(v.z) > 1e-30f ? v.z : copysignf(1e-30f, v.z)));
        const float tlo = __fmaf_rn(-fabsf(t_min), 1e-5f, t_min);  // culling slack; the exact test decides hits
        if (n == 1) {
            float t;
            ++nprim;
            if (hit_prim(rec, 0, O, v, t_min, poly, t)) kbuf_insert(kb, t, ids[0]);
        } else if (n > 1) {
            int stk[TRACE_STACK];
            float stt[TRACE_STACK];
            int sp = 0;
            int node = 0;
            const unsigned long long max_visits = 2ull * (unsigned long long)n + 64ull;
            while (true) {
                if (++nnode > max_visits) {  // malformed hierarchy: report instead of spinning
                    atomicOr(status, ERR_INDEX);
                    break;
                }
                const float4 *np = reinterpret_cast<const float4 *>(nodes + node);
                float4 a = __ldg(np), b = __ldg(np + 1), c = __ldg(np + 2);
                int4 d = __ldg(reinterpret_cast<const int4 *>(np + 3));
                float thi = __fmaf_rn(fabsf(kb.t[K_HITS - 1]), 1e-5f, kb.t[K_HITS - 1]);
                float t0, t1;
                bool h0 = slab(a.x, a.y, a.z, a.w, b.x, b.y, O, iv, tlo, thi, t0);
                bool h1 = slab(b.z, b.w, c.x, c.y, c.z, c.w, O, iv, tlo, thi, t1);
                if (h0 && d.x < 0) {
                    float t;
                    ++nprim;
                    if (hit_prim(rec, ~d.x, O, v, t_min, poly, t)) {
                        int pid = __ldg(ids + ~d.x);
                        if (t < kb.t[K_HITS - 1] || (t == kb.t[K_HITS - 1] && pid < kb.i[K_HITS - 1]))
                            kbuf_insert(kb, t, pid);
                    }
                    h0 = false;
                }
                if (h1 && d.y < 0) {
                    float t;
                    ++nprim;
                    if (hit_prim(rec, ~d.y, O, v, t_min, poly, t)) {
                        int pid = __ldg(ids + ~d.y);
                        if (t < kb.t[K_HITS - 1] || (t == kb.t[K_HITS - 1] && pid < kb.i[K_HITS - 1]))
                            kbuf_insert(kb, t, pid);
                    }
                    h1 = false;
                }
                if (h0 && h1) {
                    bool first0 = t0 <= t1;
                    int far = first0 ? d.y : d.x;
                    float tfar = first0 ? t1 : t0;
                    node = first0 ? d.x : d.y;
                    if (sp < TRACE_STACK) {
                        stk[sp] = far;
                        stt[sp] = tfar;
                        ++sp;
                    } else {
                        atomicOr(status, ERR_STACK);
                    }
                    continue;
                }
                if (h0) { node = d.x; continue; }
                if (h1) { node = d.y; continue; }
                // pop, skipping subtrees whose entry is now beyond the 16th hit
                bool found = false;
                while (sp > 0) {
                    --sp;
                    if (stt[sp] <= __fmaf_rn(fabsf(kb.t[K_HITS - 1]), 1e-5f, kb.t[K_HITS - 1])) {
                        node = stk[sp];
                        found = true;
                        break;
                    }
                }
                if (!found) break;
            }
        }
#pragma unroll
        for (int k = 0; k < K_HITS; ++k) {
            bool valid = kb.i[k] != 0x7fffffff;
            t_out[(size_t)k * stride + j] = valid ? kb.t[k] : INFINITY;
            idx_out[(size_t)k * stride + j] = valid ? kb.i[k] : -1;
        }
    }
    if (STATS) {
        for (int o = 16; o > 0; o >>= 1) {
            nprim += __shfl_xor_sync(0xffffffffu, nprim, o);
            nnode += __shfl_xor_sync(0xffffffffu, nnode, o);
        }
        if ((threadIdx.x & 31) == 0 && (nprim | nnode)) {
            atomicAdd(stats + ST_PRIM_TESTS, nprim);
            atomicAdd(stats + ST_NODES, nnode);
        }
    }
}

int launch_trace(flare_renderer *r, const float *O, const float *v, const float *t_min, const int *ray_ids,
                 int count, float *t_out, int *idx_out, int out_stride, cudaStream_t st) {
    if (count <= 0) return FLARE_OK;
    const int B = 128;
    trace_kernel<true><<<(count + B - 1) / B, B, 0, st>>>(O, v, t_min, ray_ids, count, r->nodes, r->rec,
                                                           r->ids_sorted, r->n, t_out, idx_out, out_stride, r->poly,
                                                           r->dstatus, r->dstats);
    FLARE_CUDA_TRY(cudaGetLastError());
    return FLARE_OK;
}

}  // namespace flare
