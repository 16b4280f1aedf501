// Resolves the one CUDA driver entry point the GEMM kernels' host code calls
// (TMA descriptor encoding) through the runtime ONCE and caches it.
//
// The CUTLASS host adapter is built with CUTLASS_ENABLE_DIRECT_CUDA_DRIVER_CALL, so it
// calls cuTensorMapEncodeTiled directly instead of looking the entry point up on every
// GEMM launch.  This definition satisfies that call without linking libcuda (the
// library must still import on machines without a driver), and its hidden
// visibility keeps it private to this library.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

namespace {

PFN_cuTensorMapEncodeTiled_v12000 resolve_encode_tiled() {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult status;
  if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &status) !=
          cudaSuccess ||
      status != cudaDriverEntryPointSuccess)
    return nullptr;
  return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
}

}  // namespace

extern "C" __attribute__((visibility("hidden"))) CUresult CUDAAPI cuTensorMapEncodeTiled(
    CUtensorMap* tensorMap, CUtensorMapDataType tensorDataType, cuuint32_t tensorRank, void* globalAddress,
    const cuuint64_t* globalDim, const cuuint64_t* globalStrides, const cuuint32_t* boxDim,
    const cuuint32_t* elementStrides, CUtensorMapInterleave interleave, CUtensorMapSwizzle swizzle,
    CUtensorMapL2promotion l2Promotion, CUtensorMapFloatOOBfill oobFill) {
  static const PFN_cuTensorMapEncodeTiled_v12000 fn = resolve_encode_tiled();
  if (fn == nullptr) return CUDA_ERROR_NOT_INITIALIZED;
  return fn(tensorMap, tensorDataType, tensorRank, globalAddress, globalDim, globalStrides, boxDim, elementStrides,
            interleave, swizzle, l2Promotion, oobFill);
}
