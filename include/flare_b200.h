/*
 * flare_b200.h -- C ABI of the B200-native FlaRe render path.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream handle (cudaStream_t passed
 * as void*; NULL means the legacy default stream), returns 0 on success and a non-zero FLARE_E_* code
 * on failure, and leaves a human-readable message in a thread-local buffer read by
 * flare_last_error().  No entry point synchronises the device except where stated; results are
 * ready when the stream has drained.
 *
 * The entry points replace the methods of the reference PyTorch extension `PYOPTIXFLARERENDERER`
 * (source/renderer/PyOptiXFLARERenderer.cpp:12-74 binds them, source/renderer/CPyOptiXFLARERenderer.h
 * declares them).  Each declaration below names the reference method(s) it stands in for.
 *
 * Tensor layouts follow the reference exactly (all contiguous, row-major):
 *   rays      O, v            (R,3)  f32      one origin / direction per ray
 *   geometry  m (N,3) f32, s (N,2) f32 log-scale, q (N,4) f32 (w,x,y,z order as stored, unnormalised),
 *             RGBA (N,4) f32 = [base RGB, opacity logit], k (N,1) f32 raw shape (kappa = 1 + softplus(k))
 *   decoder   cond (N,96) f16, features (13154) f32 LUT, A1 (64,128) f16, b1 (64) f32,
 *             A2 (64,64) f16, b2 (64) f32, A3 (16,64) f16, b3 (16) f32
 * Outputs are accumulated (+=) into caller-zeroed buffers, as in the reference, except where stated.
 */
#ifndef FLARE_B200_H
#define FLARE_B200_H

#ifdef __cplusplus
extern "C" {
#endif

#define FLARE_OK 0
#define FLARE_E_INVALID 1   /* bad argument (null pointer, size out of range) */
#define FLARE_E_CUDA 2      /* a CUDA runtime call failed */
#define FLARE_E_DEVICE 3    /* a kernel reported an error through the device status word */
#define FLARE_E_STATE 4     /* call made in the wrong state (e.g. render before SetGeometry) */

#define FLARE_HIT_BUFFER_SIZE 16 /* k of the k-nearest hit buffer (reference constants.h:2) */
#define FLARE_LUT_SIZE 13154     /* 2 * (16^2 + 25^2 + 40^2 + 64^2), reference Forward_training.cu:608 */
#define FLARE_COND_DIM 96        /* reference Forward_training.cu:32 */
#define FLARE_GRID_SIZE 16502    /* decoder 1: 2 * sum over l < 8 of floor(4 * 1.5^l)^2 */
#define FLARE_GRID_COND_DIM 32   /* decoder 1 descriptor width */

/* Decoder kinds (flare_scene.decoder).  FLARE_DECODER_LUT_PE is the reference's compiled decoder.
   FLARE_DECODER_GRID_SH is BASELINE config 0's encoder: a dense multiresolution grid of the local (u, v)
   coordinates (8 levels of floor(4 * 1.5^l) vertices per side, 2 features each, row-major like the
   reference's MultiResolutionEncoding when a level fits its 2^16-entry table), the degree-3 real
   spherical harmonics of the view direction, a 32-wide descriptor and ReLU hidden layers; colour =
   sigmoid(y) * RGB.  Its layouts: cond (N,32) f16, features (16502) f32 (level-major, vertex row-major,
   2 floats per vertex), A1 (64,128) f16 of which columns 64..127 are unused (their gradient is 0). */
#define FLARE_DECODER_LUT_PE 0
#define FLARE_DECODER_GRID_SH 1

typedef struct flare_renderer flare_renderer;

/* Thread-local message of the last failing call on this thread ("" if none). */
const char *flare_last_error(void);

/* Library version string. */
const char *flare_version(void);

/*
 * Replaces CPyOptiXFLARERenderer::CPyOptiXFLARERenderer(number_of_sides, chi_square_squared_radius,
 * max_batch_size) (CPyOptiXFLARERenderer.cpp:10-15 -> CPyOptiXFLARERenderer_CUDA_Core.cu:43-526).
 * Scratch for max_batch_size rays is allocated here, on `device`.  number_of_sides in [3, 64].
 * chi_square_squared_radius is stored but, as in the reference (Core.cu:583), the proxy radius uses
 * the constant 11.3449.
 */
int flare_create(int number_of_sides, float chi_square_squared_radius, int max_batch_size, int device,
                 flare_renderer **out);

/* Frees everything the renderer owns.  Accepts NULL. */
int flare_destroy(flare_renderer *r);

/*
 * Replaces CPyOptiXFLARERenderer::SetGeometry(m, scale, q, opacity, kappa)
 * (CPyOptiXFLARERenderer.cpp:19-30 -> Core.cu:687-816).  Inputs are the ACTIVATED parameters, as the
 * reference callers pass them (train.py:449): scale = exp(s) (N,2), opacity = sigmoid(A) (N),
 * kappa = 1 + softplus(k) (N).  Builds the polygon frames and the LBVH on `stream`.
 */
int flare_set_geometry(flare_renderer *r, const float *m, const float *scale, const float *q,
                       const float *opacity, const float *kappa, int n, void *stream);

/*
 * Replaces CPyOptiXFLARERenderer::Render(O, v, t_min, size) (CPyOptiXFLARERenderer.cpp:34-61 ->
 * Core.cu:820-858 -> shaders.cu:19-77): for each ray, the 16 nearest proxy hits with t >= t_min[ray],
 * ascending by (t, primitive index).  t_out and idx_out are (16, n_rays) slot-major; unused slots
 * hold t = +inf, idx = -1.
 */
int flare_render_hits(flare_renderer *r, const float *O, const float *v, const float *t_min, int n_rays,
                      float *t_out, int *idx_out, void *stream);

/*
 * Replaces the module function GenerateRays(R, D, F, width, height, fov_x, fov_y)
 * (GenerateRays.cpp:6-28 -> GenerateRays.cu:6-72): out (H*W, 3) f32, v = R*dx + D*dy + F, not
 * normalised.
 */
int flare_generate_rays(const float *R, const float *D, const float *F, int width, int height, float fov_x,
                        float fov_y, float *out, void *stream);

/* Which forward product a flare_forward call computes. */
enum flare_forward_mode {
    FLARE_FWD_TRAINING = 0,           /* Forward_training(_base): RGB + depth/normal-reg accumulators */
    FLARE_FWD_INFERENCE = 1,          /* Forward_inference(_base): RGB */
    FLARE_FWD_INFERENCE_GEOMETRY = 2, /* Forward_inference(_base)_with_geometry: RGB, normal, alpha, E[t] numerator */
    FLARE_FWD_PCA = 3,                /* Forward_pca: RGB from override colours */
    FLARE_FWD_MEDIAN = 4              /* GetMedianDepth(_base): (t, idx) of the last hit with T > 0.5 */
};

/* Scene parameters shared by forward and backward.  Decoder pointers are NULL for the base model. */
typedef struct flare_scene {
    const float *m, *s, *q, *RGBA, *k;       /* (N,3) (N,2) (N,4) (N,4) (N,1) raw parameters */
    int n;                                   /* N; must equal the N of the last flare_set_geometry */
    const void *cond;                        /* (N,96) f16 or NULL (base model) */
    const float *features;                   /* (13154) f32 LUT */
    const void *A1, *A2, *A3;                /* f16 weights (64,128) (64,64) (16,64) */
    const float *b1, *b2, *b3;               /* f32 biases (64) (64) (16) */
    int decoder;                             /* FLARE_DECODER_*; 0 unless the grid/SH variant is used */
} flare_scene;

typedef struct flare_forward_args {
    int mode;                                /* enum flare_forward_mode */
    const float *O, *v;                      /* (R,3) */
    int n_rays;
    float bg[3];
    float T_threshold;
    float *bitmap;                           /* (R,3) accumulated; not used by MEDIAN */
    /* TRAINING */
    float *depth_reg_accums;                 /* (R,4) (L_d, sum w, sum w t~, sum w t) accumulated */
    float reg_a, reg_b;
    float *depth_and_index;                  /* (R,2): MEDIAN output; unused by TRAINING (as in reference) */
    const float *surface_normal;             /* (R,3) normal-reg target, zero vector = no target */
    float *normal_reg_accums;                /* (R,4) .x accumulated */
    /* INFERENCE_GEOMETRY (each may be NULL) */
    float *normal;                           /* (R,3) accumulated */
    float *alpha;                            /* (R) written: 1 - T */
    float *expected_depth_numerator;         /* (R) accumulated */
    /* PCA */
    const float *override_colors;            /* (N,3) */
} flare_forward_args;

/*
 * Replaces CPyOptiXFLARERenderer::{Forward_training, Forward_inference, Forward_pca,
 * Forward_inference_with_geometry, GetMedianDepth} (CPyOptiXFLARERenderer.cpp:451-720 ->
 * *_Forward_training.cu:949-1132, *_Forward_inference.cu:932-1104, *_GetMedianDepth.cu:882-1046) when
 * scene->cond != NULL, and their _base twins (CPyOptiXFLARERenderer.cpp:66-450 ->
 * *_Forward_training_base.cu, *_Forward_inference_base.cu, *_GetMedianDepth_base.cu) when it is NULL.
 */
int flare_forward(flare_renderer *r, const flare_scene *scene, const flare_forward_args *a, void *stream);

typedef struct flare_backward_args {
    const float *O, *v;                      /* (R,3) */
    int n_rays;
    float bg[3];
    float T_threshold;
    float *I;                                /* (R,3) final (clamped) image; OVERWRITTEN, as in reference */
    const float *dL_dI;                      /* (R,3) */
    /* gradients, accumulated (+=) into caller-zeroed buffers */
    float *dL_dRGB, *dL_dA, *dL_dk, *dL_dm, *dL_ds, *dL_dq;   /* (N,3) (N,1) (N,1) (N,3) (N,2) (N,4) */
    float *dL_dcond;                         /* (N,96) f32 (decoder only) */
    float *dL_dfeatures;                     /* (13154) f32 (decoder only) */
    /* MLP weight gradients in the reference's per-warp fragment layout (train.py:704-790); the fully
       reduced gradient is added into row 0, other rows are untouched.  Sizes in floats per row:
       dw1 8192, db1 512, dw2 4096, db2 512, dw3 512, db3 64. */
    float *dL_dw1, *dL_db1, *dL_dw2, *dL_db2, *dL_dw3, *dL_db3;
    /* regularisers (reference Backward.cu:1753-1817) */
    const float *depth_reg_accums;           /* (R,4) from the forward */
    float *depth_normal_reg_prefix_sums;     /* (R,4) caller-zeroed scratch (written) */
    float lambda_depth, reg_a, reg_b;
    const float *surface_normal;             /* (R,3) */
    float lambda_normal;
    /* Decoder path only, optional (NULL: off).  When set, the per-primitive gradients are ACCUMULATED
       (+=) into these caller-zeroed rows (N, FLARE_PRIM_ROW_FLOATS), 16-byte aligned, and dL_dRGB, dL_dA,
       dL_dk, dL_dm, dL_ds, dL_dq and dL_dcond are left untouched; flare_scatter_prim_rows turns the rows
       into them.  Data-parallel callers sum the rows over ranks first: a row is 80 floats where the
       outputs it expands to are 14 + the descriptor width (110 for the reference decoder). */
    float *prim_rows;
} flare_backward_args;

/*
 * Replaces CPyOptiXFLARERenderer::Backward (CPyOptiXFLARERenderer.cpp:722-873 ->
 * *_Backward.cu:2238-2453) when scene->cond != NULL and Backward_base
 * (CPyOptiXFLARERenderer.cpp:345-450 -> *_Backward_base.cu:641-804) when it is NULL.
 */
int flare_backward(flare_renderer *r, const flare_scene *scene, const flare_backward_args *a, void *stream);

/*
 * Per-primitive gradient rows of the decoder backward (flare_backward_args.prim_rows): row p =
 * [dm 3, ds 2, dq 4, dRGB 3, dA 1, dk 1, 0 0 | d1 64], d1 = the sum over p's hits of the gradient of
 * layer 1's pre-activations.  The descriptor gradient is linear in d1 (dcond = W1[:, 32:32+C]^T d1,
 * C the descriptor width), so rows summed over data-parallel ranks expand to the summed gradients.
 * flare_scatter_prim_rows adds row p's parts into dm / ds / dq / dRGB / dA / dk and W1[:, 32:]^T d1
 * into dcond (all (N, .) f32 device arrays, accumulated), for n rows; A1 is the (64,128) f16 weight,
 * decoder a FLARE_DECODER_* kind.  Rows that are all zero are skipped.  No reference counterpart (the
 * reference writes its per-hit gradients straight into the outputs, Backward.cu:1300-2234).
 */
#define FLARE_PRIM_ROW_FLOATS 80
int flare_scatter_prim_rows(const float *rows, int n, const void *A1, int decoder, float *dL_dRGB, float *dL_dA,
                            float *dL_dk, float *dL_dm, float *dL_ds, float *dL_dq, float *dL_dcond, void *stream);

/*
 * Secondary rays (replaces CPyOptiXFLAREVIEWERRenderer::Forward, source/viewer_renderer/
 * CPyOptiXFLAREVIEWERRenderer.cpp -> *_CUDA_Forward.cu:912-1276 and shaders.cu, with analytic spheres
 * standing in for its triangle-mesh instances).  Per ray generation: k-nearest passes over the
 * primitives up to the nearest sphere, shadow tests of every buffered hit towards each directional
 * light, compositing with shadowed colours times shadow_multiplier; then each ray that reached a sphere
 * with T >= T_threshold is shaded there (Fresnel, refraction / total internal reflection, ambient,
 * diffuse and specular) and splits: the child with more transmittance continues, the other is pushed;
 * max_recursion_depth bounds the pushes like the reference's stack.  Rays reaching no sphere add
 * bg * T.  scene->RGBA = [RGB | A]: the viewer's RGB (N,3) colours and A (N) opacity logits.
 */
#define FLARE_VIEWER_MAX_SPHERES 16
#define FLARE_VIEWER_MAX_LIGHTS 8
typedef struct flare_viewer_args {
    const float *O, *v;          /* (R,3) primary rays, directions normalised (device) */
    float *bitmap;               /* (R,3) accumulated (device, caller-zeroed) */
    int n_rays;
    float bg[3];
    float T_threshold;
    const float *spheres;        /* HOST (S,4): centre xyz, radius */
    const float *materials;      /* HOST (S,6): Id rgb, kd, eta, n -- the reference's material rows */
    int n_spheres;
    const float *lights;         /* HOST (L,6): Is rgb, direction L (light travels along L) */
    int n_lights;
    float epsilon;               /* t_min of secondary and shadow rays */
    float shadow_multiplier;
    float ambient[3];            /* Ia */
    int max_recursion_depth;
} flare_viewer_args;
int flare_viewer_forward(flare_renderer *r, const flare_scene *scene, const flare_viewer_args *a, void *stream);

/*
 * The optimizer step (replaces torch.optim.Adam over the reference's 16 parameter groups,
 * scene/gaussian_model.py:318-336, and the scale regulariser added to the s gradient, train.py:850-852):
 * one launch over all segments.  Segment i updates param[row * p_stride + p_offset + col] for
 * row < rows, col < width from the dense grad / exp_avg / exp_avg_sq [row * width + col] (moments
 * zero-initialised by the caller) with learning rate lr; param_f16 (optional) receives the updated value
 * at the same address in fp16; scale_reg > 0 (width-2 s rows only) adds scale_reg * exp(s)^2 /
 * sqrt(sum_row exp(s)^2) to the gradient.  step is Adam's step count t >= 1 (bias corrections).
 */
#define FLARE_ADAM_MAX_SEGMENTS 24
typedef struct flare_adam_segment {
    float *param;
    const float *grad;
    float *exp_avg, *exp_avg_sq;
    void *param_f16;
    long long rows;
    int width, p_stride, p_offset;
    float lr, scale_reg;
} flare_adam_segment;
typedef struct flare_adam_args {
    int n_segments;
    flare_adam_segment seg[FLARE_ADAM_MAX_SEGMENTS];
    float beta1, beta2, eps;
    int step;
} flare_adam_args;
int flare_adam_step(const flare_adam_args *a, void *stream);

/*
 * Densification / pruning support (replaces the per-tensor index / cat sequence of train.py:955-1240):
 * builds every output tensor in one launch, dst row r = source row src_row[r] (r < n_out); rows
 * [alt_begin, alt_end) read src_alt instead of src when src_alt != NULL.  Rows are row_bytes long
 * (multiple of 4); sources and destinations are device memory and must not overlap.
 */
#define FLARE_GATHER_MAX_TENSORS 32
typedef struct flare_gather_tensor {
    const void *src, *src_alt;
    void *dst;
    int row_bytes;
} flare_gather_tensor;
int flare_gather_rows(const flare_gather_tensor *tensors, int n_tensors, const int *src_row, int n_out, int alt_begin,
                      int alt_end, void *stream);

/* Statistics of the last forward/backward call (counted on the device; reading them synchronises the
   stream of that call): rays, passes, composited hits, primitive tests, BVH node visits. */
typedef struct flare_stats {
    long long rays, passes, hits_composited, prim_tests, node_visits;
    long long decoder_tiles;  /* 128-row tensor-core tiles the decoder kernels ran (forward + backward);
                                 hits_composited / (128 * decoder_tiles) is their row utilisation */
} flare_stats;
int flare_get_stats(flare_renderer *r, flare_stats *out);

/*
 * Per-kernel device time, measured with CUDA events recorded on the caller's stream around every
 * launch while profiling is enabled (flare_profile(r, 1) enables and zeroes the counters).  Index 0
 * LBVH build (whole flare_set_geometry), 1 traversal, 2 forward shading, 3 backward shading.  No
 * reference counterpart (the reference logs wall-clock FPS only, train.py:1459-1491).
 */
typedef struct flare_kernel_times {
    double ms[4];
    long long launches[4];
} flare_kernel_times;
int flare_profile(flare_renderer *r, int enable);
int flare_get_kernel_times(flare_renderer *r, flare_kernel_times *out);

/*
 * Exposes the per-primitive polygon frames built by the last flare_set_geometry, for the bit-exact
 * hit-list test: frames (N,12) f32 = [m.xyz, N.xyz, U/(e^sx rho).xyz, V/(e^sy rho).xyz] in primitive
 * order.  Device pointer to caller storage; synchronous on `stream`.
 */
int flare_get_frames(flare_renderer *r, float *frames_out, void *stream);

/*
 * Diagnostic read-out of the traversal passes of the last Forward_training (the hit cache a following
 * Backward replays; valid from the second Forward_training on a renderer, which the first one sizes).
 * pass < 0: *count = number of cached passes.  Otherwise *count = rays of that pass and, when the
 * outputs are non-NULL, ray_ids (count) receives the pass's ray ids and t_out / idx_out
 * (FLARE_PASS_SLOTS, count) slot-major its hit lists, ascending by (t, index), +inf / -1 padded.
 * Device pointers; synchronous on `stream`.  Used by the full-size hit-list parity tests.  No
 * reference counterpart (the reference's per-pass buffers are private to its pass loop,
 * CPyOptiXFLARERenderer_CUDA_Forward_training.cu:1004-1131).
 */
#ifndef FLARE_PASS_SLOTS
#define FLARE_PASS_SLOTS 42 /* hits per internal pass; a build with another FLARE_K_PASS sets it too */
#endif
int flare_get_pass_hits(flare_renderer *r, int pass, int *count, int *ray_ids, float *t_out, int *idx_out,
                        void *stream);

/*
 * Allocation-free 16-nearest-hit query.  No counterpart in the reference, whose renderer allocates its
 * scratch in the constructor and in SetGeometry.  For callers that cannot allocate device memory when
 * they call (under a fixed device-memory budget, or as a plugin in a process whose allocator owns the
 * device): builds the proxy hierarchy for n_prims <=
 * FLARE_NOALLOC_MAX_PRIMS primitives from SetGeometry's activated inputs and writes the same (16, n_rays)
 * t / idx as flare_set_geometry + flare_render_hits, with all scratch (about 11 MB) in a static device
 * array that every GPU loading the library holds until exit.  Larger scenes return FLARE_E_INVALID.
 * The first call on a device resolves the array's address (a failed resolution is retried by the next
 * call).  Calls
 * share the array, so calls that overlap on the GPU race and must be serialised by the caller.  The
 * call synchronises `stream` to read its status word.
 */
#define FLARE_NOALLOC_MAX_PRIMS 32768
int flare_render_hits_noalloc(int number_of_sides, const float *m, const float *scale, const float *q,
                              const float *opacity, const float *kappa, int n_prims, const float *O, const float *v,
                              const float *t_min, int n_rays, float *t_out, int *idx_out, void *stream);

/*
 * Decoder self-test: runs the renderer's tensor-core MLP on `rows` fp16 input rows X (rows,128) and
 * writes the 16 fp32 layer-3 outputs per row to Y (rows,16).  Used by the tests to check the MLP
 * tiles against a host reference independently of tracing.
 */
int flare_selftest_mlp(const void *X, int rows, const void *A1, const float *b1, const void *A2,
                       const float *b2, const void *A3, const float *b3, float *Y, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* FLARE_B200_H */
