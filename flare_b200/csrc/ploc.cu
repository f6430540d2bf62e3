// ploc.cu -- bottom-up hierarchy by parallel locally-ordered clustering (Meister & Bittner 2018, "Parallel
// Locally-Ordered Clustering for Bounding Volume Hierarchy Construction"), an alternative to the Karras
// radix tree over the same sorted primitives.
//
// Clusters start as the primitives in extended-Morton order.  Each iteration every cluster finds, among
// the PLOC_R clusters on either side in that order, the one whose merged box has the smallest surface
// area; mutual nearest neighbours merge into a new node (the left one keeps the merged cluster, the right
// one drops out) and the survivors are compacted in order.  Ties are broken by the pair's indices, so the
// globally closest pair is always mutual and every iteration merges at least once.  Node indices count
// down from n-2 in creation order, so the last merge -- the root -- is node 0, and nodes made in the same
// iteration sit together in Morton order.  Nodes are written in the traversal's format (both child boxes
// plus links), so no refit pass is needed.
#include <cub/device/device_scan.cuh>

#include "renderer.cuh"

namespace flare {

#ifndef FLARE_PLOC_R
#define FLARE_PLOC_R 16
#endif
constexpr int PLOC_R = FLARE_PLOC_R;
constexpr int PLOC_B = 256;

struct Box6 {
    float lx, ly, lz, hx, hy, hz;
};

__device__ __forceinline__ float merged_area(const Box6 &a, const Box6 &b) {
    const float ex = fmaxf(a.hx, b.hx) - fminf(a.lx, b.lx);
    const float ey = fmaxf(a.hy, b.hy) - fminf(a.ly, b.ly);
    const float ez = fmaxf(a.hz, b.hz) - fminf(a.lz, b.lz);
    return ex * ey + ey * ez + ez * ex;
}

__device__ __forceinline__ unsigned long long pair_key(int i, int j) {
    return ((unsigned long long)min(i, j) << 32) | (unsigned)max(i, j);
}

__device__ __forceinline__ Box6 load_box(const float *b, int i) {
    const float *p = b + 6 * (size_t)i;
    return Box6{p[0], p[1], p[2], p[3], p[4], p[5]};
}

// Leaf clusters: box of sorted primitive j, link ~j.
__global__ void ploc_init_kernel(int n, const int *__restrict__ ids_sorted, const float *__restrict__ aabb,
                                 float *__restrict__ cbox, int *__restrict__ cid) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= n) return;
    const int pid = ids_sorted[j];
#pragma unroll
    for (int k = 0; k < 6; ++k) cbox[6 * (size_t)j + k] = aabb[6 * (size_t)pid + k];
    cid[j] = ~j;
}

// Nearest neighbour (smallest merged surface area) within +-PLOC_R positions; key (area, lo, hi index).
__global__ void __launch_bounds__(PLOC_B) ploc_nn_kernel(int m, const float *__restrict__ cbox, int *__restrict__ nn) {
    __shared__ Box6 s[PLOC_B + 2 * PLOC_R];
    const int base = blockIdx.x * PLOC_B;
    for (int t = threadIdx.x; t < PLOC_B + 2 * PLOC_R; t += PLOC_B) {
        const int g = base - PLOC_R + t;
        if (g >= 0 && g < m) s[t] = load_box(cbox, g);
    }
    __syncthreads();
    const int i = base + threadIdx.x;
    if (i >= m) return;
    const Box6 me = s[threadIdx.x + PLOC_R];
    float best = INFINITY;
    int bj = -1;
#pragma unroll 4
    for (int d = -PLOC_R; d <= PLOC_R; ++d) {
        const int j = i + d;
        if (d == 0 || j < 0 || j >= m) continue;
        const float a = merged_area(me, s[threadIdx.x + PLOC_R + d]);
        // ties: the pair with the smaller (low, high) index wins -- the same rule seen from either end
        if (a < best || (a == best && bj >= 0 && pair_key(i, j) < pair_key(i, bj))) {
            best = a;
            bj = j;
        }
    }
    nn[i] = bj;
}

// Per cluster: keeps (1 in the low 32 bits) unless absorbed by a merge to its left; merge leaders add
// 1 in the high 32 bits.  One 64-bit exclusive scan then gives both output positions and node ranks.
__global__ void ploc_flags_kernel(int m, const int *__restrict__ nn, unsigned long long *__restrict__ flags) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= m) return;
    const int j = nn[i];
    const bool mutual = j >= 0 && nn[j] == i;
    const bool leader = mutual && i < j;
    const bool keep = !mutual || leader;
    flags[i] = (keep ? 1ull : 0ull) | (leader ? (1ull << 32) : 0ull);
}

__global__ void ploc_merge_kernel(int m, int n, int created, const int *__restrict__ nn,
                                  const unsigned long long *__restrict__ flags,
                                  const unsigned long long *__restrict__ scan, const float *__restrict__ cbox,
                                  const int *__restrict__ cid, float *__restrict__ cbox_out, int *__restrict__ cid_out,
                                  Node *__restrict__ nodes, const int *__restrict__ ids_sorted) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= m) return;
    const unsigned long long f = flags[i];
    if (!(f & 0xffffffffull)) return;  // absorbed into the cluster on its left
    const int pos = (int)(scan[i] & 0xffffffffull);
    Box6 b = load_box(cbox, i);
    int id = cid[i];
    if (f >> 32) {  // merge leader: node (this cluster, its right neighbour)
        const int j = nn[i];
        const Box6 o = load_box(cbox, j);
        const int node = (n - 2) - (created + (int)(scan[i] >> 32));
        float *nf = reinterpret_cast<float *>(nodes + node);
        nf[0] = b.lx; nf[1] = b.ly; nf[2] = b.lz; nf[3] = b.hx; nf[4] = b.hy; nf[5] = b.hz;
        nf[6] = o.lx; nf[7] = o.ly; nf[8] = o.lz; nf[9] = o.hx; nf[10] = o.hy; nf[11] = o.hz;
        const int cj = cid[j];
        nodes[node].d = make_int4(id, cj, id < 0 ? ids_sorted[~id] : -1, cj < 0 ? ids_sorted[~cj] : -1);
        b = Box6{fminf(b.lx, o.lx), fminf(b.ly, o.ly), fminf(b.lz, o.lz),
                 fmaxf(b.hx, o.hx), fmaxf(b.hy, o.hy), fmaxf(b.hz, o.hz)};
        id = node;
    }
    float *q = cbox_out + 6 * (size_t)pos;
    q[0] = b.lx; q[1] = b.ly; q[2] = b.lz; q[3] = b.hx; q[4] = b.hy; q[5] = b.hz;
    cid_out[pos] = id;
}

// Traversal records in sorted order (the hierarchy's leaves refer to sorted positions).
__global__ void gather_rec_kernel(int n, const int *__restrict__ ids_sorted, const float *__restrict__ frames,
                                  float4 *__restrict__ rec) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= n) return;
    const float4 *f = reinterpret_cast<const float4 *>(frames + 12 * (size_t)ids_sorted[j]);
    rec[3 * (size_t)j] = f[0];
    rec[3 * (size_t)j + 1] = f[1];
    rec[3 * (size_t)j + 2] = f[2];
}

size_t ploc_scratch_bytes(int n) {
    size_t scan_tmp = 0;
    cub::DeviceScan::ExclusiveSum(nullptr, scan_tmp, (unsigned long long *)nullptr, (unsigned long long *)nullptr, n,
                                  (cudaStream_t)0);
    const size_t N = (size_t)n;
    return 2 * N * 6 * sizeof(float) + 2 * N * sizeof(int) + N * sizeof(int) + 2 * N * sizeof(unsigned long long) +
           scan_tmp + 4096;
}

// Builds nodes[0 .. n-2] over the n sorted primitives; `scratch` holds ploc_scratch_bytes(n) bytes.
int build_hierarchy_ploc(int n, const int *ids_sorted, const float *aabb, const float *frames, Node *nodes,
                         float4 *rec, void *scratch, unsigned long long *h_total, cudaStream_t st) {
    const size_t N = (size_t)n;
    char *p = static_cast<char *>(scratch);
    auto take = [&](size_t bytes) {
        char *q = p;
        p += (bytes + 255) & ~size_t(255);
        return q;
    };
    float *cbox[2] = {reinterpret_cast<float *>(take(N * 6 * sizeof(float))),
                      reinterpret_cast<float *>(take(N * 6 * sizeof(float)))};
    int *cid[2] = {reinterpret_cast<int *>(take(N * sizeof(int))), reinterpret_cast<int *>(take(N * sizeof(int)))};
    int *nn = reinterpret_cast<int *>(take(N * sizeof(int)));
    unsigned long long *flags = reinterpret_cast<unsigned long long *>(take(N * sizeof(unsigned long long)));
    unsigned long long *scan = reinterpret_cast<unsigned long long *>(take(N * sizeof(unsigned long long)));
    size_t scan_tmp = 0;
    cub::DeviceScan::ExclusiveSum(nullptr, scan_tmp, flags, scan, n, st);
    void *tmp = take(scan_tmp);
    const int B = 256;
    gather_rec_kernel<<<(n + B - 1) / B, B, 0, st>>>(n, ids_sorted, frames, rec);
    if (n < 2) {
        FLARE_CUDA_TRY(cudaGetLastError());
        return FLARE_OK;
    }
    ploc_init_kernel<<<(n + B - 1) / B, B, 0, st>>>(n, ids_sorted, aabb, cbox[0], cid[0]);
    int m = n, cur = 0, created = 0;
    for (int it = 0; m > 1; ++it) {
        if (it > n) {
            set_error("hierarchy build did not converge");
            return FLARE_E_DEVICE;
        }
        const int G = (m + B - 1) / B;
        ploc_nn_kernel<<<(m + PLOC_B - 1) / PLOC_B, PLOC_B, 0, st>>>(m, cbox[cur], nn);
        ploc_flags_kernel<<<G, B, 0, st>>>(m, nn, flags);
        size_t t = scan_tmp;
        FLARE_CUDA_TRY(cub::DeviceScan::ExclusiveSum(tmp, t, flags, scan, m, st));
        ploc_merge_kernel<<<G, B, 0, st>>>(m, n, created, nn, flags, scan, cbox[cur], cid[cur], cbox[cur ^ 1],
                                           cid[cur ^ 1], nodes, ids_sorted);
        // totals = last exclusive prefix + last flag
        FLARE_CUDA_TRY(cudaMemcpyAsync(h_total, scan + (m - 1), sizeof(unsigned long long), cudaMemcpyDeviceToHost, st));
        FLARE_CUDA_TRY(cudaMemcpyAsync(h_total + 1, flags + (m - 1), sizeof(unsigned long long),
                                       cudaMemcpyDeviceToHost, st));
        FLARE_CUDA_TRY(cudaStreamSynchronize(st));
        const unsigned long long tot = h_total[0] + h_total[1];
        const int kept = (int)(tot & 0xffffffffull), merged = (int)(tot >> 32);
        if (merged == 0) {
            set_error("hierarchy build made no progress");
            return FLARE_E_DEVICE;
        }
        created += merged;
        m = kept;
        cur ^= 1;
    }
    FLARE_CUDA_TRY(cudaGetLastError());
    return FLARE_OK;
}

}  // namespace flare
