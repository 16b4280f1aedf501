// D[M,N] = alpha * A[M,K] . B[K,N] + beta * C   (data gradient, stream-K over 128 x 256 tiles)
//
// For long reductions into few output tiles (the LM head's data gradient: K = vocabulary,
// 8,192 x 768 outputs = 192 tiles on 148 SMs) the stream-K scheduler balances the K loops.
#include "../gemm_impl.cuh"
using namespace pra::gemm;
using Op = cutlass::epilogue::fusion::LinearCombination<BF16, float, BF16, float>;
using G = Gemm<cutlass::layout::RowMajor, cutlass::layout::RowMajor, BF16, Op, Shape<_128, _256, _64>,
               cutlass::gemm::StreamKScheduler>;

cudaError_t pra_gemm_nn_sk(const GemmArgs& g, cudaStream_t st) {
  typename G::Epilogue::FusionCallbacks::Arguments fusion{};
  fusion.alpha = g.alpha;
  fusion.beta = g.beta;
  fusion.alpha_ptr = g.alpha_ptr;
  return G::run(g.A, g.B, g.C, g.D, g.M, g.N, g.K, fusion, g.workspace, g.workspace_bytes, st);
}
