// D[M,N] = alpha * A[K,M]^T . B[K,N] + beta * C   (weight gradient dY^T X)
#include "../gemm_impl.cuh"
using namespace pra::gemm;
using Op = cutlass::epilogue::fusion::LinearCombination<BF16, float, BF16, float>;
// 128x64 tiles: weight gradients have few output tiles (d_out x d_in) and a long K (tokens), so
// narrower tiles put more CTAs to work
using G = Gemm<cutlass::layout::ColumnMajor, cutlass::layout::RowMajor, BF16, Op, Shape<_128, _64, _64>>;

cudaError_t pra_gemm_wgrad(const GemmArgs& g, cudaStream_t st) {
  typename G::Epilogue::FusionCallbacks::Arguments fusion{};
  fusion.alpha = g.alpha;
  fusion.beta = g.beta;
  fusion.alpha_ptr = g.alpha_ptr;
  return G::run(g.A, g.B, g.C, g.D, g.M, g.N, g.K, fusion, g.workspace, g.workspace_bytes, st);
}
