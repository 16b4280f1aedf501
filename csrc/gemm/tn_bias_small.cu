// D[M,N] = alpha * A[M,K] . B[N,K]^T + bias[N] + beta * C[M,N] for small M (decode: one
// token per row): 128x64 tiles with a stream-K schedule, so every SM streams weights even
// when there are fewer output tiles than SMs.
#include "../gemm_impl.cuh"
using namespace pra::gemm;
using Op = cutlass::epilogue::fusion::LinCombPerColBias<BF16, float, BF16, BF16, float>;
using G = Gemm<cutlass::layout::RowMajor, cutlass::layout::ColumnMajor, BF16, Op, Shape<_128, _64, _64>,
               cutlass::gemm::StreamKScheduler>;

cudaError_t pra_gemm_tn_bias_small(const GemmArgs& g, cudaStream_t st) {
  typename G::Epilogue::FusionCallbacks::Arguments fusion{};
  fusion.alpha = g.alpha;
  fusion.beta = g.beta;
  fusion.alpha_ptr = g.alpha_ptr;
  fusion.bias_ptr = static_cast<const BF16*>(g.bias);
  return G::run(g.A, g.B, g.C, g.D, g.M, g.N, g.K, fusion, g.workspace, g.workspace_bytes, st);
}
