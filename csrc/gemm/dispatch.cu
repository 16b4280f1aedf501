// Which tcgen05 GEMM instantiation runs a training / prefill product, from its shape.
//
// Measured on one B200 (python -m pdattention_b200.profiling gemm-train-shapes, TinyGPT-PRA-163M
// shapes): the 2-SM kernels (one MMA across an SM pair, 256-row tiles) beat the 1-SM tiles
// whenever their pair tiles fill the GPU's 74 SM pairs in nearly whole waves (forward QKV
// 29.0 -> 23.9 us, fc1 37.4 -> 31.1 us, LM head 518 -> 430 us; weight gradients 39-40 -> 27-29 us);
// with few pair tiles (an 8,192 x 768 output in 96 pair tiles, 1.3 waves) the 1-SM tiles win.
// The LM head's data gradient (K = vocabulary into 192 tiles) stays on stream-K.
#include <cstdint>

#include "kernels.h"

namespace {

constexpr int kPairs = 74;  // SM pairs of a 148-SM B200

int64_t tiles(int64_t m, int64_t n, int tm, int tn) { return ((m + tm - 1) / tm) * ((n + tn - 1) / tn); }

// Fraction of the pair slots the last wave keeps busy, over all waves.
double wave_fill(int64_t t, int slots) {
  const int64_t waves = (t + slots - 1) / slots;
  return waves == 0 ? 0.0 : (double)t / (double)(waves * slots);
}

bool long_reduction(const GemmArgs& g) { return g.K >= 16384 && tiles(g.M, g.N, 128, 256) < 4 * 148; }

}  // namespace

cudaError_t pra_gemm_tn_auto(const GemmArgs& g, cudaStream_t st) {
  if (g.M <= 128) return pra_gemm_tn_bias_small(g, st);
  if (wave_fill(tiles(g.M, g.N, 256, 256), kPairs) >= 0.8) return pra_gemm_tn_bias_2sm(g, st);
  return g.N <= 1024 ? pra_gemm_tn_bias_narrow(g, st) : pra_gemm_tn_bias(g, st);
}

cudaError_t pra_gemm_nn_auto(const GemmArgs& g, cudaStream_t st) {
  if (long_reduction(g)) return pra_gemm_nn_sk(g, st);
  return pra_gemm_nn_2sm(g, st);
}

cudaError_t pra_gemm_wgrad_auto(const GemmArgs& g, cudaStream_t st) {
  if (tiles(g.M, g.N, 256, 128) >= 48) return pra_gemm_wgrad_2sm(g, st);
  return pra_gemm_wgrad(g, st);
}
