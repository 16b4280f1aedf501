// Which tcgen05 GEMM instantiation runs a training / prefill product, from its shape.
//
// Measured on one B200 (python -m pdattention_b200.profiling gemm-train-shapes, TinyGPT-PRA-163M
// shapes): 1-SM tiles for every product except two long reductions into few output tiles,
// where the stream-K schedule keeps the SMs busy: the LM head's data gradient (K = vocabulary,
// 8,192 x 768 outputs: 723 -> 551 us) and its weight gradient (a 50,304 x 768 output: 650 ->
// 618 us).  Stream-K measured slower on every d_model-sized reduction.
#include <cstdint>

#include "kernels.h"

namespace {

int64_t tiles(int64_t m, int64_t n, int tm, int tn) { return ((m + tm - 1) / tm) * ((n + tn - 1) / tn); }

bool long_reduction(const GemmArgs& g) { return g.K >= 16384 && tiles(g.M, g.N, 128, 256) < 4 * 148; }

}  // namespace

cudaError_t pra_gemm_tn_auto(const GemmArgs& g, cudaStream_t st) {
  if (g.M <= 128) return pra_gemm_tn_bias_small(g, st);
  return g.N <= 1024 ? pra_gemm_tn_bias_narrow(g, st) : pra_gemm_tn_bias(g, st);
}

cudaError_t pra_gemm_nn_auto(const GemmArgs& g, cudaStream_t st) {
  return long_reduction(g) ? pra_gemm_nn_sk(g, st) : pra_gemm_nn(g, st);
}

cudaError_t pra_gemm_wgrad_auto(const GemmArgs& g, cudaStream_t st) {
  return (int64_t)g.M * g.N >= (16 << 20) ? pra_gemm_wgrad_sk(g, st) : pra_gemm_wgrad(g, st);
}
