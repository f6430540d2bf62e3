/* Minimal stand-in for the OptiX SDK host header, so that the reference renderer's plain-CUDA decode /
 * composite / backward kernels (which include Header.cuh -> optix_host.h) compile without the SDK.  It
 * declares only the type and constant names those translation units mention; nothing here traces rays.
 * The host methods that call optixLaunch are compiled but never called by the ref_kernels.cu wrappers.
 * Test infrastructure only (oracle/_ref). */
#pragma once
#include <cuda.h>
#include <cstddef>

typedef int OptixResult;
#define OPTIX_SUCCESS 0
#define OPTIX_ERROR_NOT_SUPPORTED 7806
#define OPTIX_SBT_RECORD_ALIGNMENT 16
#define OPTIX_SBT_RECORD_HEADER_SIZE 32
typedef unsigned long long OptixTraversableHandle;
typedef struct OptixDeviceContext_t *OptixDeviceContext;
typedef struct OptixModule_t *OptixModule;
typedef struct OptixProgramGroup_t *OptixProgramGroup;
typedef struct OptixPipeline_t *OptixPipeline;
typedef struct OptixShaderBindingTable {
    CUdeviceptr raygenRecord;
} OptixShaderBindingTable;

/* Defined in ref_kernels.cu to return OPTIX_ERROR_NOT_SUPPORTED: the wrappers never trace through OptiX. */
OptixResult optixLaunch(OptixPipeline pipeline, CUstream stream, CUdeviceptr pipelineParams,
                        size_t pipelineParamsSize, const OptixShaderBindingTable *sbt, unsigned width,
                        unsigned height, unsigned depth);
