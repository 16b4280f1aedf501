// D[M,N] = alpha * A[M,K] . B[K,N] + beta * C   (data gradient; 2-SM 256 x 256 tiles)
#include "../gemm_impl.cuh"
using namespace pra::gemm;
using Op = cutlass::epilogue::fusion::LinearCombination<BF16, float, BF16, float>;
using G = Gemm<cutlass::layout::RowMajor, cutlass::layout::RowMajor, BF16, Op, Shape<_256, _256, _64>, void, true>;

cudaError_t pra_gemm_nn_2sm(const GemmArgs& g, cudaStream_t st) {
  typename G::Epilogue::FusionCallbacks::Arguments fusion{};
  fusion.alpha = g.alpha;
  fusion.beta = g.beta;
  fusion.alpha_ptr = g.alpha_ptr;
  return G::run(g.A, g.B, g.C, g.D, g.M, g.N, g.K, fusion, g.workspace, g.workspace_bytes, st);
}
