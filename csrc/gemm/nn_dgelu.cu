// D[M,N] = gelu'(Z) * (A[M,K] . B[K,N])   with Z the stored pre-activation (MLP backward)
#include "../gemm_impl.cuh"
using namespace pra::gemm;
using Op = cutlass::epilogue::fusion::LinCombDeEltAct<cutlass::layout::RowMajor, GeluErfGrad, BF16, float, BF16, BF16,
                                                      float>;
using G = Gemm<cutlass::layout::RowMajor, cutlass::layout::RowMajor, BF16, Op>;

cudaError_t pra_gemm_nn_dgelu(const GemmArgs& g, cudaStream_t st) {
  typename G::Epilogue::FusionCallbacks::Arguments fusion{};
  fusion.alpha = g.alpha;
  fusion.beta = 0.f;
  fusion.aux_ptr = static_cast<const BF16*>(g.aux);
  fusion.dAux = cutlass::make_cute_packed_stride(typename decltype(fusion)::StrideAux{}, {g.M, g.N, 1});
  return G::run(g.A, g.B, nullptr, g.D, g.M, g.N, g.K, fusion, g.workspace, g.workspace_bytes, st);
}
