// Token + learned position embedding lookup (TinyGPT-PRA input layer), bf16 out:
//   x[m] = tok[ids[m]] + pos[positions ? positions[m] : m % period]
// The sum is formed in fp32 and rounded once (like adding the two fp32 rows and casting).
#include "common.cuh"

namespace pra {
namespace embed {

__global__ void embed_add_kernel(const int* __restrict__ ids, const int* __restrict__ positions, int period,
                                 const __nv_bfloat16* __restrict__ tok, const __nv_bfloat16* __restrict__ pos,
                                 int64_t M, int D, __nv_bfloat16* __restrict__ out) {
  const int64_t m = blockIdx.x;
  if (m >= M) return;
  const int64_t t = ids[m];
  const int64_t p = positions ? positions[m] : (int)(m % period);
  const __nv_bfloat162* a = reinterpret_cast<const __nv_bfloat162*>(tok + t * D);
  const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(pos + p * D);
  __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(out + m * D);
  for (int j = threadIdx.x; j < D / 2; j += blockDim.x) {
    const float2 x = __bfloat1622float2(a[j]), y = __bfloat1622float2(b[j]);
    o[j] = __floats2bfloat162_rn(x.x + y.x, x.y + y.y);
  }
}

}  // namespace embed
}  // namespace pra

cudaError_t pra_embed_add(const int* ids, const int* positions, int period, const __nv_bfloat16* tok,
                          const __nv_bfloat16* pos, int64_t M, int D, __nv_bfloat16* out, cudaStream_t st) {
  if (M == 0) return cudaSuccess;
  if (D % 2 || (positions == nullptr && period <= 0)) return cudaErrorInvalidValue;
  pra::embed::embed_add_kernel<<<(unsigned)M, 128, 0, st>>>(ids, positions, period, tok, pos, M, D, out);
  return cudaGetLastError();
}
