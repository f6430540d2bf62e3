// bvh4.cu -- 4-wide hierarchy collapsed from the binary one (either builder): every binary node at even
// depth becomes a 4-wide node whose children are its grandchildren through internal children (and its
// leaf children directly).  A traversal step then fetches one 128-byte line and tests four boxes, so a
// root-to-leaf walk takes half as many dependent fetches.
//
// Node4 layout: the four child boxes as structure of arrays (lo.x[4] lo.y[4] lo.z[4] hi.x[4] hi.y[4]
// hi.z[4]), the four links (internal >= 0: 4-wide node index, leaf: ~sorted position, NODE4_EMPTY: no
// child) and the four leaf children's original indices.  A missing child also gets lo = +inf, hi = -inf, but
// the slab test orders each axis' two planes, so the traversal skips it by its link, not by its box.
#include <cub/device/device_scan.cuh>

#include "renderer.cuh"

namespace flare {

__global__ void bin_parent_kernel(const Node *__restrict__ nodes, int m, int *__restrict__ par) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= m) return;
    const int4 d = nodes[i].d;
    if (d.x >= 0) par[d.x] = i;
    if (d.y >= 0) par[d.y] = i;
    if (i == 0) par[0] = -1;
}

// 1 for internal nodes at even depth (root = depth 0)
__global__ void even_depth_kernel(const int *__restrict__ par, int m, int *__restrict__ flag,
                                  int *__restrict__ status) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= m) return;
    int depth = 0, p = i;
    while (p > 0 && depth < 4096) {
        p = par[p];
        ++depth;
        if (p < 0 || p >= m) {
            atomicOr(status, ERR_INDEX);
            break;
        }
    }
    flag[i] = (depth & 1) == 0;
}

__global__ void collapse_kernel(const Node *__restrict__ nodes, int m, const int *__restrict__ flag,
                                const int *__restrict__ idx4, Node4 *__restrict__ out) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= m || !flag[i]) return;
    float lo[3][4], hi[3][4];
    int link[4], pid[4];
    int n4 = 0;
    const Node b = nodes[i];
    const float *bs = reinterpret_cast<const float *>(&b);
    const int bl[2] = {b.d.x, b.d.y}, bp[2] = {b.d.z, b.d.w};
    for (int c = 0; c < 2; ++c) {
        if (bl[c] < 0) {  // leaf child of the even node
            for (int a = 0; a < 3; ++a) {
                lo[a][n4] = bs[6 * c + a];
                hi[a][n4] = bs[6 * c + 3 + a];
            }
            link[n4] = bl[c];
            pid[n4] = bp[c];
            ++n4;
        } else {  // internal (odd depth): its two children
            const Node o = nodes[bl[c]];
            const float *os = reinterpret_cast<const float *>(&o);
            const int ol[2] = {o.d.x, o.d.y}, op[2] = {o.d.z, o.d.w};
            for (int g = 0; g < 2; ++g) {
                for (int a = 0; a < 3; ++a) {
                    lo[a][n4] = os[6 * g + a];
                    hi[a][n4] = os[6 * g + 3 + a];
                }
                link[n4] = ol[g] < 0 ? ol[g] : idx4[ol[g]];
                pid[n4] = ol[g] < 0 ? op[g] : -1;
                ++n4;
            }
        }
    }
    for (; n4 < 4; ++n4) {
        for (int a = 0; a < 3; ++a) {
            lo[a][n4] = INFINITY;
            hi[a][n4] = -INFINITY;
        }
        link[n4] = NODE4_EMPTY;
        pid[n4] = -1;
    }
    Node4 q;
    q.lox = make_float4(lo[0][0], lo[0][1], lo[0][2], lo[0][3]);
    q.loy = make_float4(lo[1][0], lo[1][1], lo[1][2], lo[1][3]);
    q.loz = make_float4(lo[2][0], lo[2][1], lo[2][2], lo[2][3]);
    q.hix = make_float4(hi[0][0], hi[0][1], hi[0][2], hi[0][3]);
    q.hiy = make_float4(hi[1][0], hi[1][1], hi[1][2], hi[1][3]);
    q.hiz = make_float4(hi[2][0], hi[2][1], hi[2][2], hi[2][3]);
    q.link = make_int4(link[0], link[1], link[2], link[3]);
    q.pid = make_int4(pid[0], pid[1], pid[2], pid[3]);
    out[idx4[i]] = q;
}

size_t bvh4_scratch_bytes(int n) {
    size_t tmp = 0;
    cub::DeviceScan::ExclusiveSum(nullptr, tmp, (int *)nullptr, (int *)nullptr, n, (cudaStream_t)0);
    return (size_t)n * 3 * sizeof(int) + tmp + 1024;  // + alignment of the scan workspace
}

// Collapses nodes[0 .. n-2] into nodes4 (room for n - 1 nodes); scratch holds bvh4_scratch_bytes(n).
int build_bvh4(const Node *nodes, int n, Node4 *nodes4, void *scratch, int *status, cudaStream_t st) {
    if (n < 2) return FLARE_OK;
    const int m = n - 1;
    char *p = static_cast<char *>(scratch);
    int *par = reinterpret_cast<int *>(p);
    int *flag = par + n;
    int *idx4 = flag + n;
    void *tmp = reinterpret_cast<void *>((reinterpret_cast<uintptr_t>(idx4 + n) + 255) & ~uintptr_t(255));
    size_t tb = 0;
    cub::DeviceScan::ExclusiveSum(nullptr, tb, flag, idx4, m, st);
    const int B = 256, G = (m + B - 1) / B;
    bin_parent_kernel<<<G, B, 0, st>>>(nodes, m, par);
    even_depth_kernel<<<G, B, 0, st>>>(par, m, flag, status);
    FLARE_CUDA_TRY(cub::DeviceScan::ExclusiveSum(tmp, tb, flag, idx4, m, st));
    collapse_kernel<<<G, B, 0, st>>>(nodes, m, flag, idx4, nodes4);
    FLARE_CUDA_TRY(cudaGetLastError());
    return FLARE_OK;
}

}  // namespace flare
