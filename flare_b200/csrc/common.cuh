// common.cuh -- shared definitions of the FlaRe B200 render-path library.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "../../include/flare_b200.h"

namespace flare {

constexpr int K_HITS = FLARE_HIT_BUFFER_SIZE;  // 16: hits per Render call (the reference's k-buffer)
#ifndef FLARE_K_PASS
#define FLARE_K_PASS FLARE_PASS_SLOTS
#endif
// Hits gathered per pass inside Forward / Backward.  The composited result does not depend on it (hits
// are consumed in (t, index) order either way); it trades traversal restarts against the per-ray heap in
// shared memory: 42 entries (42 KB per 128-ray block + the stack) is the most that keeps 5 traversal
// blocks per SM.
constexpr int K_PASS = FLARE_K_PASS;
constexpr int COND = FLARE_COND_DIM;           // 96
constexpr int LUT = FLARE_LUT_SIZE;            // 13154 floats
constexpr int MAX_SIDES = 64;
constexpr int TRACE_STACK = 64;
// Per-CTA LUT-gradient copy in the backward, "pair-major": 4 floats per cell hold the (x, y) gradient of
// the cell and of its right neighbour, so the two corners of a bilinear row are one 16-byte reduction.
constexpr int GRID_FEATS = FLARE_GRID_SIZE;   // 16502 floats (decoder 1's dense 8-level grid)
// per-CTA pair-major feature-gradient copy: 4 floats per cell of the larger table (4 * 16502 / 2 = 33004),
// rounded up to 128 floats
constexpr int LUT_PRIV_FLOATS = 33024;
// Packed per-primitive gradient of the decoder backward: dm 3, ds 2, dq 4, dRGB 3, dA 1, dk 1, 2 pad.
constexpr int PGRAD_FLOATS = 16;
constexpr int PROW_FLOATS = PGRAD_FLOATS + 64;  // decoder backward row per primitive: packed gradients | layer-1 deltas
constexpr float LUT_SCALE = 0.29689279887990428378374198030042f;  // 1/sqrt(11.3449)

// Internal forward mode of the secondary-ray (viewer) path: colour of a shadowed hit times the shadow
// multiplier, no background at the end of a pass (added when the ray generation ends).
constexpr int FWD_VIEWER = 100;

// Device status word bits (first word of renderer->dstatus).
enum : int {
    ERR_STACK = 1,     // traversal stack overflow (hits may be incomplete)
    ERR_MBAR = 2,      // a tensor-core completion wait timed out
    ERR_INDEX = 4,     // out-of-range primitive index met
};

// Counters in renderer->dstats (unsigned long long each).
enum { ST_PASSES = 0, ST_HITS = 1, ST_PRIM_TESTS = 2, ST_NODES = 3, ST_TILES = 4, ST_NSTATS = 8 };

// BVH2 node: both child boxes plus child links; a negative link ~p is a leaf holding sorted primitive p.
struct __align__(16) Node {
    float4 a;  // lo0.x lo0.y lo0.z hi0.x
    float4 b;  // hi0.y hi0.z lo1.x lo1.y
    float4 c;  // lo1.z hi1.x hi1.y hi1.z
    int4 d;    // c0 c1 (internal >= 0, leaf = ~sorted position), pid0 pid1 (original index of a leaf child)
};

// 4-wide node (bvh4.cu): child boxes as structure of arrays, links (internal >= 0: 4-wide node index,
// leaf: ~sorted position) and each leaf child's original index; 128 bytes, one line per visit.
constexpr int NODE4_EMPTY = (int)0x80000000;  // link of an unused child slot (never ~position, positions < n)
struct __align__(128) Node4 {
    float4 lox, loy, loz, hix, hiy, hiz;
    int4 link, pid;
};

// Traversal node with inline leaves (128 bytes, one cache line per visit): child j owns c[4j .. 4j+3].
// Internal child: c[4j] = (lo.xyz, hi.x), c[4j+1] = (hi.y, hi.z, -, -), c[4j+3].x = link (>= 0).
// Leaf child: c[4j .. 4j+2] = the primitive's 48-byte traversal record (m, N, U/(e^sx rho), V/(e^sy rho)),
// c[4j+3] = (link = ~sorted position, original index, -, -).  A leaf is tested straight from the node:
// no second, dependent fetch of its record.
struct __align__(128) NodeL {
    float4 c[8];
};

// Polygon edge constants for the hit test (host computes them once per renderer).
struct PolyConst {
    int n;
    int half;  // n even and edge j+n/2 == -(edge j) exactly: test |c a + s b| <= 1 for j < n/2 only
    float c[MAX_SIDES];
    float s[MAX_SIDES];
};

}  // namespace flare

// internal host-side helpers (implemented in api.cu)
namespace flare {
void set_error(const char *fmt, ...);
}

#define FLARE_CUDA_TRY(call)                                                                   \
    do {                                                                                       \
        cudaError_t e_ = (call);                                                               \
        if (e_ != cudaSuccess) {                                                               \
            flare::set_error("%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, __LINE__); \
            return FLARE_E_CUDA;                                                               \
        }                                                                                      \
    } while (0)
