// D[M,N] = alpha * A[M,K] . B[N,K]^T + bias[N] + beta * C[M,N] for narrow outputs (N <= 1024,
// e.g. the d_model-wide projections): 128x128 tiles give twice the CTAs of 128x256 and fill
// the 148 SMs evenly for token counts in the thousands.
#include "../gemm_impl.cuh"
using namespace pra::gemm;
using Op = cutlass::epilogue::fusion::LinCombPerColBias<BF16, float, BF16, BF16, float>;
using G = Gemm<cutlass::layout::RowMajor, cutlass::layout::ColumnMajor, BF16, Op, Shape<_128, _128, _64>>;

cudaError_t pra_gemm_tn_bias_narrow(const GemmArgs& g, cudaStream_t st) {
  typename G::Epilogue::FusionCallbacks::Arguments fusion{};
  fusion.alpha = g.alpha;
  fusion.beta = g.beta;
  fusion.alpha_ptr = g.alpha_ptr;
  fusion.bias_ptr = static_cast<const BF16*>(g.bias);
  return G::run(g.A, g.B, g.C, g.D, g.M, g.N, g.K, fusion, g.workspace, g.workspace_bytes, st);
}
