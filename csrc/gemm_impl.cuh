// bf16 GEMMs on the 5th-generation tensor cores, built from the CUTLASS sm100
// collectives (tcgen05.mma issued by one thread per CTA pair, TMA-fed shared
// memory stages, TMEM accumulators, fused epilogues).  Each exported variant is
// instantiated in its own translation unit so they compile in parallel.
//
// Conventions (all packed, row-major unless noted):
//   "tn"    D[M,N] = A[M,K] . B[N,K]^T            (forward: X W^T)
//   "nn"    D[M,N] = A[M,K] . B[K,N]              (data gradient: dY W)
//   "wgrad" D[M,N] = A[K,M]^T . B[K,N]            (weight gradient: dY^T X)
#pragma once

#include <atomic>

#include <cutlass/cutlass.h>
#include <cute/tensor.hpp>
#include <cutlass/epilogue/collective/collective_builder.hpp>
#include <cutlass/epilogue/fusion/operations.hpp>
#include <cutlass/epilogue/thread/activation.h>
#include <cutlass/gemm/collective/collective_builder.hpp>
#include <cutlass/gemm/device/gemm_universal_adapter.h>
#include <cutlass/gemm/kernel/gemm_universal.hpp>
#include <cutlass/util/packed_stride.hpp>

#include "kernels.h"

namespace pra {
namespace gemm {

using namespace cute;
using BF16 = cutlass::bfloat16_t;

// ---- erf GELU for the GEMM epilogues ------------------------------------------------
// The MLP GEMMs have a short reduction (K = d_model), so their epilogue math competes with
// the tensor-core main loop; with one warp per scheduler doing it, a full-precision erf made
// the GELU GEMMs epilogue bound (about twice the time of the same GEMM with a bias epilogue).
// erf here follows Abramowitz & Stegun, Handbook of Mathematical Functions, formula 7.1.26:
//   erf(x) = 1 - (a1 t + a2 t^2 + a3 t^3 + a4 t^4 + a5 t^5) e^{-x^2},  t = 1 / (1 + p x),  x >= 0,
// |error| <= 1.5e-7 (odd extension below 0): one reciprocal and one exponential on the special
// function unit plus six fused multiply-adds, far below the bf16 output's 2^-8 resolution.
// The GELU and its derivative share e^{-z^2/2}, which is both the formula's e^{-x^2} (x = z/sqrt2)
// and the normal density's kernel.
struct ErfAS7126 {
  static constexpr float p = 0.3275911f;
  static constexpr float a1 = 0.254829592f, a2 = -0.284496736f, a3 = 1.421413741f, a4 = -1.453152027f,
                         a5 = 1.061405429f;
};

CUTLASS_HOST_DEVICE float gelu_exp(float x) {
#if defined(__CUDA_ARCH__)
  return __expf(x);
#else
  return std::exp(x);
#endif
}

CUTLASS_HOST_DEVICE float gelu_rcp(float x) {
#if defined(__CUDA_ARCH__)
  return __fdividef(1.f, x);
#else
  return 1.f / x;
#endif
}

// Phi(z) = (1 + erf(z / sqrt2)) / 2 given e = e^{-z^2/2}.
CUTLASS_HOST_DEVICE float gelu_cdf(float z, float e) {
  const float x = fabsf(z) * 0.70710678118654752f;
  const float t = gelu_rcp(1.f + ErfAS7126::p * x);
  const float poly =
      t * (ErfAS7126::a1 + t * (ErfAS7126::a2 + t * (ErfAS7126::a3 + t * (ErfAS7126::a4 + t * ErfAS7126::a5))));
  const float erf_abs = 1.f - poly * e;
  return 0.5f + copysignf(0.5f * erf_abs, z);
}

// The forward GELU needs no e^{-z^2/2}, so it takes Abramowitz & Stegun formula 7.1.28 instead:
//   erf(x) = 1 - (1 + a1 x + a2 x^2 + a3 x^3 + a4 x^4 + a5 x^5 + a6 x^6)^(-16),  x >= 0,
// |error| <= 3e-7: one reciprocal (the 16th power by four squarings; for large x it overflows to
// infinity and the reciprocal to 0, i.e. erf = 1).  The streaming GELU pass is bound by the
// special function unit, so one operation per element instead of two.
struct ErfAS7128 {
  static constexpr float a1 = 0.0705230784f, a2 = 0.0422820123f, a3 = 0.0092705272f, a4 = 0.0001520143f,
                         a5 = 0.0002765672f, a6 = 0.0000430638f;
};

CUTLASS_HOST_DEVICE float gelu_cdf_7128(float z) {
  const float x = fabsf(z) * 0.70710678118654752f;
  float p = 1.f + x * (ErfAS7128::a1 +
                       x * (ErfAS7128::a2 + x * (ErfAS7128::a3 + x * (ErfAS7128::a4 + x * (ErfAS7128::a5 +
                                                                                             x * ErfAS7128::a6)))));
  p = p * p;  // ^2
  p = p * p;  // ^4
  p = p * p;  // ^8
  p = p * p;  // ^16
  const float erf_abs = 1.f - gelu_rcp(p);
  return 0.5f + copysignf(0.5f * erf_abs, z);
}

// gelu(z) = z Phi(z)
template <typename T>
struct GeluErf {
  static const bool kIsHeavy = true;
  CUTLASS_HOST_DEVICE T operator()(T const& z_t) const {
    const float z = float(z_t);
    return T(z * gelu_cdf_7128(z));
  }
};

template <typename T, int N>
struct GeluErf<cutlass::Array<T, N>> {
  static const bool kIsHeavy = true;
  CUTLASS_HOST_DEVICE cutlass::Array<T, N> operator()(cutlass::Array<T, N> const& z) const {
    cutlass::Array<T, N> out;
    GeluErf<T> op;
    CUTLASS_PRAGMA_UNROLL
    for (int i = 0; i < N; ++i) out[i] = op(z[i]);
    return out;
  }
};

// Derivative of the erf GELU: d/dz [z Phi(z)] = Phi(z) + z phi(z), phi(z) = e^{-z^2/2} / sqrt(2 pi).
template <typename T>
struct GeluErfGrad {
  static const bool kIsHeavy = true;
  CUTLASS_HOST_DEVICE T operator()(T const& d_t, T const& z_t) const {
    const float z = float(z_t);
    const float e = gelu_exp(-0.5f * z * z);
    return T(float(d_t) * (gelu_cdf(z, e) + z * 0.39894228040143268f * e));
  }
};

template <typename T, int N>
struct GeluErfGrad<cutlass::Array<T, N>> {
  static const bool kIsHeavy = true;
  CUTLASS_HOST_DEVICE cutlass::Array<T, N> operator()(cutlass::Array<T, N> const& d_t,
                                                      cutlass::Array<T, N> const& z) const {
    cutlass::Array<T, N> out;
    GeluErfGrad<T> op;
    CUTLASS_PRAGMA_UNROLL
    for (int i = 0; i < N; ++i) out[i] = op(d_t[i], z[i]);
    return out;
  }
};

// One-SM tcgen05 tiles, cluster of one CTA: every CTA issues its own TMA loads (the
// library is also used by multi-GPU runs, which must not issue cluster-shared loads).
inline int sm_count() {
  static int cached[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 0;
  if (cached[dev] == 0) cudaDeviceGetAttribute(&cached[dev], cudaDevAttrMultiProcessorCount, dev);
  return cached[dev];
}

// Scheduler: void (persistent data-parallel tiles) or cutlass::gemm::StreamKScheduler (the
// K loop of the remaining tiles is split across idle SMs: skinny decode GEMMs).
template <class LayoutA, class LayoutB, class ElementD, class FusionOp, class TileShape = Shape<_128, _256, _64>,
          class Scheduler = void>
struct Gemm {
  using ClusterShape = Shape<_1, _1, _1>;
  using LayoutD = cutlass::layout::RowMajor;
  static constexpr int AlignAB = 8;
  static constexpr int AlignD = 128 / cutlass::sizeof_bits<ElementD>::value;
  using Epilogue = typename cutlass::epilogue::collective::CollectiveBuilder<
      cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, TileShape, ClusterShape,
      cutlass::epilogue::collective::EpilogueTileAuto, float, float, ElementD, LayoutD, AlignD, ElementD, LayoutD,
      AlignD, cutlass::epilogue::TmaWarpSpecialized1Sm, FusionOp>::CollectiveOp;
  using Mainloop = typename cutlass::gemm::collective::CollectiveBuilder<
      cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, BF16, LayoutA, AlignAB, BF16, LayoutB, AlignAB, float,
      TileShape, ClusterShape,
      cutlass::gemm::collective::StageCountAutoCarveout<static_cast<int>(sizeof(typename Epilogue::SharedStorage))>,
      cutlass::gemm::KernelTmaWarpSpecialized1SmSm100>::CollectiveOp;
  using Kernel = cutlass::gemm::kernel::GemmUniversal<Shape<int, int, int, int>, Mainloop, Epilogue, Scheduler>;
  using Device = cutlass::gemm::device::GemmUniversalAdapter<Kernel>;
  using StrideA = typename Kernel::StrideA;
  using StrideB = typename Kernel::StrideB;
  using StrideC = typename Kernel::StrideC;
  using StrideD = typename Kernel::StrideD;

  template <class FusionArgs>
  static cudaError_t run(const void* A, const void* B, const void* C, void* D, int M, int N, int K,
                         FusionArgs fusion, void* workspace, size_t workspace_bytes, cudaStream_t st) {
    if (M == 0 || N == 0) return cudaSuccess;
    typename Device::Arguments args{
        cutlass::gemm::GemmUniversalMode::kGemm,
        {M, N, K, 1},
        {static_cast<const BF16*>(A), cutlass::make_cute_packed_stride(StrideA{}, {M, K, 1}),
         static_cast<const BF16*>(B), cutlass::make_cute_packed_stride(StrideB{}, {N, K, 1})},
        {fusion, static_cast<const ElementD*>(C), cutlass::make_cute_packed_stride(StrideC{}, {M, N, 1}),
         static_cast<ElementD*>(D), cutlass::make_cute_packed_stride(StrideD{}, {M, N, 1})}};
    cudaGetDevice(&args.hw_info.device_id);
    args.hw_info.sm_count = sm_count();
    Device op;
    if (op.can_implement(args) != cutlass::Status::kSuccess) return cudaErrorNotSupported;
    if (Device::get_workspace_size(args) > workspace_bytes) return cudaErrorMemoryAllocation;
    // The full initialize() also sets the kernel's shared-memory attribute, which lasts for the
    // process: do it on the first call per device, then only the per-call parts (workspace
    // set-up and kernel parameters).
    static std::atomic<uint64_t> configured{0};
    const uint64_t bit = 1ull << (args.hw_info.device_id & 63);
    if (!(configured.load(std::memory_order_acquire) & bit)) {
      if (op.initialize(args, workspace, st) != cutlass::Status::kSuccess) return cudaErrorLaunchFailure;
      configured.fetch_or(bit, std::memory_order_acq_rel);
    } else {
      if (Kernel::initialize_workspace(args, workspace, st, nullptr) != cutlass::Status::kSuccess)
        return cudaErrorLaunchFailure;
      if (op.update(args, workspace) != cutlass::Status::kSuccess) return cudaErrorLaunchFailure;
    }
    if (op.run(st) != cutlass::Status::kSuccess) return cudaErrorLaunchFailure;
    return cudaGetLastError();
  }

  static size_t workspace(int M, int N, int K) {
    typename Device::Arguments args{cutlass::gemm::GemmUniversalMode::kGemm, {M, N, K, 1}, {}, {}};
    return Device::get_workspace_size(args);
  }
};

}  // namespace gemm
}  // namespace pra
