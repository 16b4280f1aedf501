// D[M,N] = alpha * A[M,K] . B[N,K]^T   (fp32 out; routing scores of normalised queries x gists)
#include "../gemm_impl.cuh"
using namespace pra::gemm;
using Op = cutlass::epilogue::fusion::LinearCombination<float, float, float, float>;
using G = Gemm<cutlass::layout::RowMajor, cutlass::layout::ColumnMajor, float, Op>;

cudaError_t pra_gemm_tn_f32(const GemmArgs& g, cudaStream_t st) {
  typename G::Epilogue::FusionCallbacks::Arguments fusion{};
  fusion.alpha = g.alpha;
  fusion.beta = 0.f;
  return G::run(g.A, g.B, nullptr, g.D, g.M, g.N, g.K, fusion, g.workspace, g.workspace_bytes, st);
}
