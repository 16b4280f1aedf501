// D[M,N] = alpha * A[M,K] . B[N,K]^T + bias[N] + beta * C[M,N]   (bf16 out; 2-SM 256 x 256 tiles)
#include "../gemm_impl.cuh"
using namespace pra::gemm;
using Op = cutlass::epilogue::fusion::LinCombPerColBias<BF16, float, BF16, BF16, float>;
using G = Gemm<cutlass::layout::RowMajor, cutlass::layout::ColumnMajor, BF16, Op, Shape<_256, _256, _64>, void, true>;

cudaError_t pra_gemm_tn_bias_2sm(const GemmArgs& g, cudaStream_t st) {
  typename G::Epilogue::FusionCallbacks::Arguments fusion{};
  fusion.alpha = g.alpha;
  fusion.beta = g.beta;
  fusion.alpha_ptr = g.alpha_ptr;
  fusion.bias_ptr = static_cast<const BF16*>(g.bias);
  return G::run(g.A, g.B, g.C, g.D, g.M, g.N, g.K, fusion, g.workspace, g.workspace_bytes, st);
}
