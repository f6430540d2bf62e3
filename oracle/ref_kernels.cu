// ref_kernels.cu -- launch wrappers around the reference renderer's own decode / composite / backward
// kernels, compiled from the reference sources where they lie (test infrastructure: oracle/_ref).
//
// Each build of this file includes ONE reference translation unit (REF_SRC, e.g.
// CPyOptiXFLARERenderer_CUDA_Forward_training.cu) and exports
//   ref_launch(args, number_of_rays, sm_count, stream)
// which launches that file's static __global__ kernel (REF_KERNEL) exactly as the reference's pass loop
// does (for example source/renderer/CPyOptiXFLARERenderer_CUDA_Forward_training.cu:1064: grid
// min(ceil(R / threads_per_block), SM_count), the file's threads_per_block, REF_SMEM bytes of dynamic
// shared memory, the persistent-warp counter zeroed first).  `args` is the kernel's argument array
// (cudaLaunchKernel convention: one pointer per parameter, in the kernel's parameter order).
//
// The OptiX traversal is not part of this build: the test driver (oracle/ref_kernels.py) supplies each
// pass's 16-nearest hit lists, as the reference's optixLaunch would.  OptiX's headers are replaced by the
// declarations in oracle/ref_stub/.
#define STR2(x) #x
#define STR(x) STR2(x)
#include STR(REF_SRC)

OptixResult optixLaunch(OptixPipeline, CUstream, CUdeviceptr, size_t, const OptixShaderBindingTable *, unsigned,
                        unsigned, unsigned) {
    return OPTIX_ERROR_NOT_SUPPORTED;
}

extern "C" int ref_threads_per_block() { return threads_per_block; }

extern "C" int ref_launch(void **args, int number_of_rays, int sm_count, void *stream) {
    cudaStream_t st = (cudaStream_t)stream;
    const int smem = REF_SMEM;
    cudaError_t e;
    if (smem > 48 * 1024) {
        e = cudaFuncSetAttribute(REF_KERNEL, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return (int)e;
    }
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(counter, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return (int)e;
    if (number_of_rays <= 0) return 0;
    int grid = (number_of_rays + threads_per_block - 1) / threads_per_block;
    if (grid > sm_count) grid = sm_count;
    e = cudaLaunchKernel((const void *)REF_KERNEL, dim3(grid), dim3(threads_per_block), args, smem, st);
    if (e != cudaSuccess) return (int)e;
    e = cudaStreamSynchronize(st);  // the host copy of `zero` above must outlive the copy
    return (int)e;
}
