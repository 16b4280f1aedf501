// D[M,N] = alpha * A[K,M]^T . B[K,N] + beta * C   (weight gradient, stream-K over 128 x 256 tiles)
//
// Weight gradients reduce over the token dimension (K = tokens, thousands) into small outputs
// (d_model x d_model-sized): with 128 x 256 tiles there are fewer tiles than SMs, so the
// stream-K scheduler splits the remaining K loops across idle SMs instead of shrinking the tile.
#include "../gemm_impl.cuh"
using namespace pra::gemm;
using Op = cutlass::epilogue::fusion::LinearCombination<BF16, float, BF16, float>;
using G = Gemm<cutlass::layout::ColumnMajor, cutlass::layout::RowMajor, BF16, Op, Shape<_128, _256, _64>,
               cutlass::gemm::StreamKScheduler>;

cudaError_t pra_gemm_wgrad_sk(const GemmArgs& g, cudaStream_t st) {
  typename G::Epilogue::FusionCallbacks::Arguments fusion{};
  fusion.alpha = g.alpha;
  fusion.beta = g.beta;
  fusion.alpha_ptr = g.alpha_ptr;
  return G::run(g.A, g.B, g.C, g.D, g.M, g.N, g.K, fusion, g.workspace, g.workspace_bytes, st);
}
