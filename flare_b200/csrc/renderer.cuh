// renderer.cuh -- the renderer object and the host-side launchers shared by the library's .cu files.
#pragma once
#include "common.cuh"

struct flare_renderer {
    int device = 0;
    int nsides = 8;
    float chi2 = 11.3449f;
    int max_rays = 0;
    int num_sms = 148;
    flare::PolyConst poly{};

    // ---- geometry (rebuilt by every flare_set_geometry) ----
    int n = 0;              // primitives
    int cap_n = 0;          // capacity of the geometry buffers
    float *frames = nullptr;     // (n,12) prim order: m, N, U/(sx rho), V/(sy rho)
    float4 *rec = nullptr;       // (n,3) float4 sorted order: (m.xyz,N.x) (N.yz,Ua.xy) (Ua.z,Va.xyz)
    float *aabb = nullptr;       // (n,6) prim order
    unsigned *morton = nullptr, *morton_sorted = nullptr;
    int *ids = nullptr, *ids_sorted = nullptr;  // sorted position -> primitive index
    flare::Node *nodes = nullptr;               // n-1 internal nodes, node 0 is the root
    int *parent = nullptr;                      // parent of internal node i (n-1) then of leaf j (n)
    unsigned *refit_flag = nullptr;
    float *bounds = nullptr;                    // 6 floats (scene centre bounds, ordered-int encoded)
    void *sort_tmp = nullptr;
    void *ploc_scratch = nullptr;               // clustering build scratch (ploc.cu)
    flare::Node4 *nodes4 = nullptr;             // 4-wide collapse of nodes (bvh4.cu), null when not used
    flare::NodeL *nodesL = nullptr;             // nodes with inline leaf records (bvh.cu), null when not used
    void *bvh4_scratch = nullptr;
    size_t sort_tmp_bytes = 0;

    // ---- per-ray scratch, sized max_rays ----
    float *t_min = nullptr;
    float *hint = nullptr;   // per ray: bound of its next pass (hits at t < hint), +inf = unbounded
    float *chunk_tk = nullptr;  // two-phase first pass: largest K-th hit distance per sparse 32-ray chunk
    float *T = nullptr;
    int *list[2] = {nullptr, nullptr};
    float *hit_t = nullptr;   // (16, max_rays)
    int *hit_idx = nullptr;   // (16, max_rays)
    float *ray_aux = nullptr; // (max_rays, 4) per-ray carried state (backward running colour, median)
    int *counters = nullptr;  // [0] next active count, [1..] scratch
    unsigned long long *ray_keys = nullptr;  // (2, max_rays) ray-ordering keys (trace.cu)
    int *ray_ids_tmp = nullptr;              // (max_rays)
    void *ray_sort_tmp = nullptr;
    size_t ray_sort_tmp_bytes = 0;
    unsigned char *pass_flags = nullptr;     // (max_rays) per list slot: still active after the pass
    void *select_tmp = nullptr;              // stable compaction of the active list
    size_t select_tmp_bytes = 0;
    int *h_count = nullptr;   // pinned host mirror of counters[0]

    // ---- decoder scratch ----
    float *dw = nullptr;      // dense weight-gradient accumulators (see shade.cu)
    float *gscale = nullptr;  // backward gradient scale (1 float)
    float *dfeat_priv = nullptr;  // per-CTA LUT gradient copies (2 * num_sms * LUT_PRIV_FLOATS floats)
    float *pgrad = nullptr;       // per-primitive rows of the decoder backward (PROW_FLOATS each)
    size_t pgrad_cap = 0;         // primitives pgrad holds
    void *vw_buf = nullptr;       // secondary-ray path: ray sets and per-generation scratch (viewer.cu)
    int vw_sets = 0;
    long long vw_generations = 0; // ray generations of the last flare_viewer_forward

    // ---- hit cache: the passes of the last Forward_training, replayed by a matching Backward ----
    unsigned long long geom_version = 0;  // bumped by every flare_set_geometry
    int *hc_list = nullptr;               // per pass: the active ray ids
    float *hc_t = nullptr;                // per pass: (16, count) slot-major hits
    int *hc_idx = nullptr;
    size_t hc_cap = 0;                    // capacity in ray-passes
    size_t hc_need = 0;                   // ray-passes the last uncached forward needed
    bool hc_valid = false;
    int hc_npass = 0;
    static constexpr int HC_MAX_PASSES = 4096;
    size_t hc_off[HC_MAX_PASSES] = {};
    int hc_cnt[HC_MAX_PASSES] = {};
    unsigned long long hc_key[16] = {};    // pointer / size signature of the cached forward
    unsigned long long *hc_sum = nullptr; // device: [0] forward input checksum, [1] backward input checksum

    // ---- optional per-kernel timing (CUDA events on the launching stream) ----
    bool prof_on = false;
    static constexpr int PROF_SLOTS = 256;
    cudaEvent_t prof_ev[2 * PROF_SLOTS] = {};
    int prof_kind[PROF_SLOTS] = {};
    int prof_n = 0;
    double prof_ms[4] = {0, 0, 0, 0};
    long long prof_launches[4] = {0, 0, 0, 0};

    // ---- status / statistics ----
    int *dstatus = nullptr;               // device status bits
    unsigned long long *dstats = nullptr; // flare::ST_* counters
    cudaStream_t last_stream = nullptr;
};

namespace flare {

// bvh.cu: the geometry buffers of one build over caller-chosen memory (allocation-free entry point)
struct GeomBufs {
    float *frames;
    float4 *rec;
    float *aabb;
    unsigned *morton, *morton_sorted;
    int *ids, *ids_sorted;
    Node *nodes;
    int *parent;
    unsigned *refit_flag;
    float *bounds;
    void *sort_tmp;
    size_t sort_tmp_bytes;
    int *status;
};
int build_geometry_into(const GeomBufs &g, const float *m, const float *scale, const float *q, const float *opacity,
                        const float *kappa, int n, cudaStream_t st);
size_t geometry_sort_temp_bytes(int n);
size_t ploc_scratch_bytes(int n);
size_t bvh4_scratch_bytes(int n);
int build_bvh4(const Node *nodes, int n, Node4 *nodes4, void *scratch, int *status, cudaStream_t st);
int build_hierarchy_ploc(int n, const int *ids_sorted, const float *aabb, const float *frames, Node *nodes,
                         float4 *rec, void *scratch, unsigned long long *h_total, cudaStream_t st);
int launch_trace_geom(const Node *nodes, const float4 *rec, const int *ids_sorted, int n, const PolyConst &poly,
                      const float *O, const float *v, const float *t_min, int count, float *t_out, int *idx_out,
                      int *status, cudaStream_t st);
// bvh.cu
int build_geometry(flare_renderer *r, const float *m, const float *scale, const float *q, const float *opacity,
                   const float *kappa, int n, cudaStream_t st);

// trace.cu: traces `count` rays.  Ray j is ray_ids[j] (or j when ray_ids is null); t_min is indexed by
// ray id; outputs (16, out_stride) slot-major at column j.
int launch_trace(flare_renderer *r, const float *O, const float *v, const float *t_min, const int *ray_ids,
                 int count, float *t_out, int *idx_out, int out_stride, cudaStream_t st, int k = K_HITS,
                 const float *t_max = nullptr,  // t_max: optional per-ray bound, hits at t >= t_max[ray] excluded
                 bool first = false);  // first pass of a bounded pass loop: t_max is the pass-bound array
                                       // (all +inf), which the traversal may set (two-phase first pass)

// trace.cu: writes the coherence order of R rays into list_out
int order_rays(flare_renderer *r, const float *O, const float *v, int R, int *list_out, cudaStream_t st);
size_t ray_sort_temp_bytes(int max_rays);
int compact_active(flare_renderer *r, const int *list_in, int count, int *list_out, cudaStream_t st);
size_t select_temp_bytes(int max_rays);

// shade.cu
int run_forward(flare_renderer *r, const flare_scene *sc, const flare_forward_args *a, cudaStream_t st);
int run_backward(flare_renderer *r, const flare_scene *sc, const flare_backward_args *a, cudaStream_t st);
int run_viewer_forward(flare_renderer *r, const flare_scene *sc, const flare_viewer_args *a, cudaStream_t st);
int run_scatter_rows(const float *rows, int n, const void *A1, int decoder, float *dRGB, float *dA, float *dk,
                     float *dm, float *ds, float *dq, float *dcond, cudaStream_t st);
int run_adam(const flare_adam_args *a, cudaStream_t st);
int run_gather_rows(const flare_gather_tensor *t, int n_tensors, const int *src_row, int n_out, int alt_begin,
                    int alt_end, cudaStream_t st);
int selftest_mlp(const void *X, int rows, const void *A1, const float *b1, const void *A2, const float *b2,
                 const void *A3, const float *b3, float *Y, cudaStream_t st);

// api.cu: per-kernel timing; begin returns a slot (or -1 when profiling is off), collect needs the
// stream synchronised.
enum { PK_BUILD = 0, PK_TRACE = 1, PK_SHADE_FWD = 2, PK_SHADE_BWD = 3 };
int prof_begin(flare_renderer *r, int kind, cudaStream_t st);
void prof_end(flare_renderer *r, int slot, cudaStream_t st);
void prof_collect(flare_renderer *r);

// api.cu: reads the device status word after a call and turns set bits into an error.
int check_status(flare_renderer *r, cudaStream_t st, const char *what);

}  // namespace flare
