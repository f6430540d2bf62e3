// noalloc.cu -- flare_render_hits_noalloc: the proxy-hierarchy build and the 16-nearest-hit query of
// flare_set_geometry + flare_render_hits in one call that allocates no device memory.
//
// Who needs it: callers that cannot allocate device memory when they call in -- hosts that hand this
// library a fixed device-memory budget and forbid it to grow, and plugins loaded into processes whose own
// allocator owns every device byte.  The renderer object allocates its scratch in flare_create and grows it in
// flare_set_geometry; this entry point instead keeps all scratch -- polygon frames, boxes, Morton keys,
// the radix-sort workspace, the hierarchy and the traversal records -- in one file-scope static device
// array sized for at most FLARE_NOALLOC_MAX_PRIMS primitives.  The caller passes inputs and outputs.
//
// Set-up: the first call on a device resolves the array's device address with cudaGetSymbolAddress
// (that device current) and checks the sort workspace fits; a failed resolution is not cached, so the
// next call retries it.  Later calls on the device reuse the address.  Each call synchronises `stream`
// to read the status word.  The array keeps the last call's contents; each
// call clears what must start at zero (status word, refit flags).  Calls that overlap on the GPU (two
// streams, or two host threads on one device) share the array and race: serialise them.
#include <cmath>
#include <mutex>

#include "renderer.cuh"

namespace {

constexpr int MAX_P = FLARE_NOALLOC_MAX_PRIMS;
constexpr size_t al256(size_t x) { return (x + 255) & ~(size_t)255; }

// byte offsets of the scratch regions
constexpr size_t OFF_FRAMES = 0;
constexpr size_t OFF_REC = OFF_FRAMES + al256((size_t)MAX_P * 12 * sizeof(float));
constexpr size_t OFF_AABB = OFF_REC + al256((size_t)MAX_P * 3 * sizeof(float4));
constexpr size_t OFF_MORTON = OFF_AABB + al256((size_t)MAX_P * 6 * sizeof(float));
constexpr size_t OFF_MORTON_S = OFF_MORTON + al256((size_t)MAX_P * sizeof(unsigned));
constexpr size_t OFF_IDS = OFF_MORTON_S + al256((size_t)MAX_P * sizeof(unsigned));
constexpr size_t OFF_IDS_S = OFF_IDS + al256((size_t)MAX_P * sizeof(int));
constexpr size_t OFF_NODES = OFF_IDS_S + al256((size_t)MAX_P * sizeof(int));
constexpr size_t OFF_PARENT = OFF_NODES + al256((size_t)MAX_P * sizeof(flare::Node));
constexpr size_t OFF_FLAGS = OFF_PARENT + al256((size_t)2 * MAX_P * sizeof(int));
constexpr size_t OFF_BOUNDS = OFF_FLAGS + al256((size_t)MAX_P * sizeof(unsigned));
constexpr size_t OFF_STATUS = OFF_BOUNDS + 256;
constexpr size_t OFF_SORT = OFF_STATUS + 256;
constexpr size_t SORT_BYTES = (size_t)4 << 20;  // radix-sort workspace, checked at set-up
constexpr size_t SCRATCH_BYTES = OFF_SORT + SORT_BYTES;

}  // namespace

// The scratch: every GPU that loads the library holds it (about 11 MB) until the process exits.  In host
// code this name is only a host-side stand-in; kernels get the address from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[SCRATCH_BYTES];

namespace {

struct DeviceSetup {
    bool done = false;
    unsigned char *ptr = nullptr;
};
std::mutex g_setup_mu;
DeviceSetup g_setup[64];

// edge constants of the regular n-gon, computed as flare_create computes them
flare::PolyConst poly_for(int nsides) {
    flare::PolyConst p{};
    p.n = nsides;
    const double ap = std::cos(M_PI / nsides);
    for (int j = 0; j < nsides; ++j) {
        const double phi = (2.0 * j + 1.0) * M_PI / nsides;
        p.c[j] = (float)(std::cos(phi) / ap);
        p.s[j] = (float)(std::sin(phi) / ap);
    }
    bool sym = nsides % 2 == 0;
    for (int j = 0; sym && j < nsides / 2; ++j) sym = p.c[j + nsides / 2] == -p.c[j] && p.s[j + nsides / 2] == -p.s[j];
    p.half = sym ? nsides / 2 : 0;
    return p;
}

}  // namespace

using namespace flare;

extern "C" int flare_render_hits_noalloc(int number_of_sides, const float *m, const float *scale, const float *q,
                                         const float *opacity, const float *kappa, int n_prims, const float *O,
                                         const float *v, const float *t_min, int n_rays, float *t_out, int *idx_out,
                                         void *stream) {
    if (number_of_sides < 3 || number_of_sides > MAX_SIDES) {
        set_error("flare_render_hits_noalloc: number_of_sides %d not in [3, %d]", number_of_sides, MAX_SIDES);
        return FLARE_E_INVALID;
    }
    if (n_prims < 0 || n_prims > MAX_P) {
        set_error("flare_render_hits_noalloc: %d primitives; this entry point holds at most %d (use the renderer "
                  "object for larger scenes)", n_prims, MAX_P);
        return FLARE_E_INVALID;
    }
    if (n_rays < 0) {
        set_error("flare_render_hits_noalloc: n_rays < 0");
        return FLARE_E_INVALID;
    }
    if (n_rays == 0) return FLARE_OK;
    if (!O || !v || !t_min || !t_out || !idx_out || (n_prims > 0 && (!m || !scale || !q || !opacity || !kappa))) {
        set_error("flare_render_hits_noalloc: NULL pointer argument");
        return FLARE_E_INVALID;
    }
    if (((reinterpret_cast<uintptr_t>(q) & 15) | (reinterpret_cast<uintptr_t>(scale) & 7)) != 0) {
        set_error("flare_render_hits_noalloc: q must be 16-byte aligned and scale 8-byte aligned");
        return FLARE_E_INVALID;
    }
    int dev = 0;
    FLARE_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) {
        set_error("flare_render_hits_noalloc: device %d out of range", dev);
        return FLARE_E_INVALID;
    }
    unsigned char *base = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_setup_mu);
        DeviceSetup &s = g_setup[dev];
        if (!s.done) {  // once per device, with that device current
            if (geometry_sort_temp_bytes(MAX_P) > SORT_BYTES) {  // deterministic: a build-time sizing fault
                set_error("flare_render_hits_noalloc: the radix-sort workspace does not fit its %zu-byte region",
                          SORT_BYTES);
                return FLARE_E_STATE;
            }
            void *p = nullptr;
            const cudaError_t err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
            if (err != cudaSuccess || !p) {  // not cached: a later call retries the resolution
                cudaGetLastError();
                set_error("flare_render_hits_noalloc: set-up on device %d failed: %s", dev, cudaGetErrorString(err));
                return FLARE_E_CUDA;
            }
            s.ptr = static_cast<unsigned char *>(p);
            s.done = true;
        }
        base = s.ptr;
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    GeomBufs g;
    g.frames = reinterpret_cast<float *>(base + OFF_FRAMES);
    g.rec = reinterpret_cast<float4 *>(base + OFF_REC);
    g.aabb = reinterpret_cast<float *>(base + OFF_AABB);
    g.morton = reinterpret_cast<unsigned *>(base + OFF_MORTON);
    g.morton_sorted = reinterpret_cast<unsigned *>(base + OFF_MORTON_S);
    g.ids = reinterpret_cast<int *>(base + OFF_IDS);
    g.ids_sorted = reinterpret_cast<int *>(base + OFF_IDS_S);
    g.nodes = reinterpret_cast<Node *>(base + OFF_NODES);
    g.parent = reinterpret_cast<int *>(base + OFF_PARENT);
    g.refit_flag = reinterpret_cast<unsigned *>(base + OFF_FLAGS);  // cleared by the build
    g.bounds = reinterpret_cast<float *>(base + OFF_BOUNDS);          // initialised by the build
    g.sort_tmp = base + OFF_SORT;
    g.sort_tmp_bytes = SORT_BYTES;
    g.status = reinterpret_cast<int *>(base + OFF_STATUS);
    FLARE_CUDA_TRY(cudaMemsetAsync(g.status, 0, sizeof(int), st));
    int e = build_geometry_into(g, m, scale, q, opacity, kappa, n_prims, st);
    if (e) return e;
    e = launch_trace_geom(g.nodes, g.rec, g.ids_sorted, n_prims, poly_for(number_of_sides), O, v, t_min, n_rays,
                          t_out, idx_out, g.status, st);
    if (e) return e;
    int h = 0;
    FLARE_CUDA_TRY(cudaMemcpyAsync(&h, g.status, sizeof(int), cudaMemcpyDeviceToHost, st));
    FLARE_CUDA_TRY(cudaStreamSynchronize(st));
    if (h) {
        set_error("flare_render_hits_noalloc: device reported error bits 0x%x", h);
        return FLARE_E_DEVICE;
    }
    return FLARE_OK;
}
