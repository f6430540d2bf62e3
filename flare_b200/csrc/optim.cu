// optim.cu -- the optimizer step after the backward: one fused Adam launch over every parameter group.
//
// Replaces train.py:833-860 + the torch.optim.Adam of scene/gaussian_model.py:318-336 (16 parameter
// groups with their own learning rates, default betas / eps, no weight decay) and the scale regulariser
// the reference adds to the s gradient (train.py:850-852: (lambda / N) * s2 / sqrt(sum_row s2), s2 =
// exp(s)^2).  Every group is a segment: a rows x width block of its fp32 master (strided, so RGB and A can
// live side by side in one (N,4) tensor and w1_uv / w1_v / w1_conditioning in one (64,128) matrix), a
// dense gradient of the same shape and the two moment buffers; an optional fp16 mirror at the same
// addresses receives the updated value (the descriptor rows and weights the renderer reads in fp16).
// The update restates torch's Adam step: m += (1 - b1)(g - m); v = b2 v + (1 - b2) g^2;
// p -= (lr / (1 - b1^t)) m / (sqrt(v) / sqrt(1 - b2^t) + eps).
#include <cuda_fp16.h>

#include <algorithm>

#include "renderer.cuh"

namespace flare {

struct AdamSeg {
    float *p;
    const float *g;
    float *m, *v;
    __half *h;
    long long rows, count;  // count = rows * width
    int width, p_stride, p_off;
    int block_begin;        // first block of the launch that works on this segment
    float step_size, scale_reg;
};

struct AdamArgs {
    int n;
    AdamSeg seg[FLARE_ADAM_MAX_SEGMENTS];
    float beta1, beta2, eps, bc2_sqrt;
};

constexpr int ADAM_THREADS = 256, ADAM_PER_THREAD = 8;  // elements per block: 2048

__device__ __forceinline__ void adam_update(const AdamArgs &a, const AdamSeg &sg, long long local, long long pi,
                                            float g) {
    float m = sg.m[local], v = sg.v[local];
    m = m + (1.0f - a.beta1) * (g - m);
    v = v * a.beta2 + (1.0f - a.beta2) * g * g;
    sg.m[local] = m;
    sg.v[local] = v;
    const float denom = sqrtf(v) / a.bc2_sqrt + a.eps;
    const float p = sg.p[pi] - sg.step_size * (m / denom);
    sg.p[pi] = p;
    if (sg.h) sg.h[pi] = __float2half_rn(p);
}

// Each block updates 2048 consecutive elements of one segment (blocks are laid out segment by segment).
__global__ void __launch_bounds__(ADAM_THREADS) adam_kernel(const AdamArgs a) {
    int s = 0;
    while (s + 1 < a.n && (int)blockIdx.x >= a.seg[s + 1].block_begin) ++s;
    const AdamSeg &sg = a.seg[s];
    const long long base = (long long)(blockIdx.x - sg.block_begin) * (ADAM_THREADS * ADAM_PER_THREAD);
    const bool dense = sg.p_stride == sg.width && sg.p_off == 0;
#pragma unroll
    for (int k = 0; k < ADAM_PER_THREAD; ++k) {
        const long long local = base + (long long)k * ADAM_THREADS + threadIdx.x;
        if (local >= sg.count) break;
        if (dense) {
            adam_update(a, sg, local, local, sg.g[local]);
            continue;
        }
        const long long row = local / sg.width;
        const int col = (int)(local - row * sg.width);
        const long long pi = row * sg.p_stride + sg.p_off + col;
        if (sg.scale_reg > 0.0f) {
            // s rows (width 2): the reference's scale regulariser needs both old values of the row, so the
            // thread of column 0 updates the whole row
            if (col != 0) continue;
            const float ex = expf(sg.p[pi]), ey = expf(sg.p[pi + 1]);
            const float sx = ex * ex, sy = ey * ey;
            const float rs = sqrtf(sx + sy);
            adam_update(a, sg, local, pi, sg.g[local] + sg.scale_reg * (sx / rs));
            adam_update(a, sg, local + 1, pi + 1, sg.g[local + 1] + sg.scale_reg * (sy / rs));
            continue;
        }
        adam_update(a, sg, local, pi, sg.g[local]);
    }
}

int run_adam(const flare_adam_args *in, cudaStream_t st) {
    AdamArgs a{};
    a.n = in->n_segments;
    a.beta1 = in->beta1;
    a.beta2 = in->beta2;
    a.eps = in->eps;
    const double bc1 = 1.0 - pow((double)in->beta1, (double)in->step);
    const double bc2 = 1.0 - pow((double)in->beta2, (double)in->step);
    a.bc2_sqrt = (float)sqrt(bc2);
    long long blocks = 0;
    const long long per_block = ADAM_THREADS * ADAM_PER_THREAD;
    for (int i = 0; i < a.n; ++i) {
        const flare_adam_segment &s = in->seg[i];
        AdamSeg &d = a.seg[i];
        d.p = s.param;
        d.g = s.grad;
        d.m = s.exp_avg;
        d.v = s.exp_avg_sq;
        d.h = reinterpret_cast<__half *>(s.param_f16);
        d.rows = s.rows;
        d.width = s.width;
        d.count = s.rows * s.width;
        d.p_stride = s.p_stride;
        d.p_off = s.p_offset;
        d.step_size = (float)((double)s.lr / bc1);
        d.scale_reg = s.scale_reg;
        d.block_begin = (int)blocks;
        // a scale-regularised segment must not split a row between blocks (2048 is even: rows never do)
        blocks += (d.count + per_block - 1) / per_block;
    }
    if (blocks == 0) return FLARE_OK;
    if (blocks > 0x7fffffffll) {
        set_error("flare_adam_step: %lld blocks exceed one launch", blocks);
        return FLARE_E_INVALID;
    }
    adam_kernel<<<(unsigned)blocks, ADAM_THREADS, 0, st>>>(a);
    FLARE_CUDA_TRY(cudaGetLastError());
    return FLARE_OK;
}

// ------------------------------------------------------------------------------------------------
// Row gather for densification / pruning (reference train.py:955-1240): every per-primitive tensor
// (parameters and their Adam moments) is rebuilt in one launch from a map out-row -> source row; rows
// [alt_begin, alt_end) read a tensor's alternative source when it has one (the split primitives' first
// copies take the centre and moments from before the optimizer step).  One warp per output row.
// ------------------------------------------------------------------------------------------------
struct GatherT {
    const char *src, *alt;
    char *dst;
    int row_bytes;
};
struct GatherArgs {
    int n;
    GatherT t[FLARE_GATHER_MAX_TENSORS];
};

__global__ void gather_rows_kernel(const GatherArgs a, const int *__restrict__ src_row, int n_out, int alt_begin,
                                   int alt_end) {
    const int lane = threadIdx.x & 31;
    for (long long r = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < n_out;
         r += ((long long)gridDim.x * blockDim.x) >> 5) {
        const long long sr = src_row[r];
        const bool use_alt = r >= alt_begin && r < alt_end;
        for (int i = 0; i < a.n; ++i) {
            const GatherT &t = a.t[i];
            const char *s = (use_alt && t.alt ? t.alt : t.src) + sr * t.row_bytes;
            char *d = t.dst + r * t.row_bytes;
            if ((t.row_bytes & 15) == 0 && ((reinterpret_cast<uintptr_t>(s) | reinterpret_cast<uintptr_t>(d)) & 15) == 0) {
                for (int b = lane * 16; b < t.row_bytes; b += 32 * 16)
                    *reinterpret_cast<uint4 *>(d + b) = *reinterpret_cast<const uint4 *>(s + b);
            } else {
                for (int b = lane * 4; b < t.row_bytes; b += 32 * 4)
                    *reinterpret_cast<unsigned *>(d + b) = *reinterpret_cast<const unsigned *>(s + b);
            }
        }
    }
}

int run_gather_rows(const flare_gather_tensor *t, int n_tensors, const int *src_row, int n_out, int alt_begin,
                    int alt_end, cudaStream_t st) {
    GatherArgs a{};
    a.n = n_tensors;
    for (int i = 0; i < n_tensors; ++i) {
        a.t[i].src = static_cast<const char *>(t[i].src);
        a.t[i].alt = static_cast<const char *>(t[i].src_alt);
        a.t[i].dst = static_cast<char *>(t[i].dst);
        a.t[i].row_bytes = t[i].row_bytes;
    }
    if (n_out <= 0) return FLARE_OK;
    const int B = 256;
    const long long blocks = std::min<long long>(((long long)n_out * 32 + B - 1) / B, 148 * 64);
    gather_rows_kernel<<<(unsigned)blocks, B, 0, st>>>(a, src_row, n_out, alt_begin, alt_end);
    FLARE_CUDA_TRY(cudaGetLastError());
    return FLARE_OK;
}

}  // namespace flare
