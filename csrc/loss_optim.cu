// Fused softmax cross-entropy and the fused AdamW step.
//
// Cross-entropy: one CTA per row of bf16 logits [M, ld] (only the first V
// columns are real classes).  Writes the per-row loss (0 for ignored rows) and,
// in place of the logits, the unscaled gradient softmax - onehot (zero for
// ignored rows); the backward GEMMs apply grad_out / count as a device scalar.
//
// AdamW (decoupled weight decay, bias-corrected moments) over a flat fp32
// master buffer with bf16 or fp32 gradients, global-norm clipping computed on
// the device (no host synchronisation), and the bf16 compute copy written in the
// same pass.
#include <algorithm>

#include "common.cuh"

namespace pra {
namespace lo {

constexpr int NT = 512;

__global__ void __launch_bounds__(NT) ce_kernel(__nv_bfloat16* __restrict__ logits, int64_t ld, int V,
                                                const int64_t* __restrict__ labels, int ignore_index,
                                                float* __restrict__ row_loss, float* __restrict__ row_valid) {
  __shared__ float scratch[32];
  const int64_t row = blockIdx.x;
  __nv_bfloat16* lr = logits + row * ld;
  const int64_t label = labels[row];
  const bool valid = label != ignore_index && label >= 0 && label < V;
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < V; i += NT) mx = fmaxf(mx, __bfloat162float(lr[i]));
  mx = block_max(mx, scratch);
  float se = 0.f;
  for (int i = threadIdx.x; i < V; i += NT) se += __expf(__bfloat162float(lr[i]) - mx);
  se = block_sum(se, scratch);
  const float lse = mx + __logf(se);
  const float target = valid ? __bfloat162float(lr[label]) : 0.f;
  __syncthreads();  // every thread has read lr[label] before it is overwritten
  const float inv = 1.f / se;
  for (int i = threadIdx.x; i < ld; i += NT) {
    float g = 0.f;
    if (valid && i < V) g = __expf(__bfloat162float(lr[i]) - mx) * inv - (i == label ? 1.f : 0.f);
    lr[i] = __float2bfloat16(g);
  }
  if (threadIdx.x == 0) {
    row_loss[row] = valid ? lse - target : 0.f;
    row_valid[row] = valid ? 1.f : 0.f;
  }
}

// Sum of squares of a flat gradient buffer into per-CTA partials.
template <typename G>
__global__ void sumsq_kernel(const G* __restrict__ g, int64_t n, float* __restrict__ part) {
  __shared__ float scratch[32];
  float acc = 0.f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = to_f32(g[i]);
    acc += v * v;
  }
  acc = block_sum(acc, scratch);
  if (threadIdx.x == 0) part[blockIdx.x] = acc;
}

// norm_out[0] = sqrt(sum part); coef_out[0] = min(1, max_norm / (norm + 1e-6)) (1 when max_norm <= 0).
__global__ void finish_norm_kernel(const float* __restrict__ part, int P, float max_norm, float* __restrict__ norm_out,
                                   float* __restrict__ coef_out) {
  __shared__ float scratch[32];
  float acc = 0.f;
  for (int i = threadIdx.x; i < P; i += blockDim.x) acc += part[i];
  acc = block_sum(acc, scratch);
  if (threadIdx.x == 0) {
    const float norm = sqrtf(acc);
    norm_out[0] = norm;
    coef_out[0] = max_norm > 0.f ? fminf(1.f, max_norm / (norm + 1e-6f)) : 1.f;
  }
}

template <typename G>
__global__ void adamw_kernel(float* __restrict__ param, __nv_bfloat16* __restrict__ shadow, const G* __restrict__ grad,
                             float* __restrict__ m, float* __restrict__ v, int64_t n, float lr, float beta1, float beta2,
                             float eps, float weight_decay, float bc1, float bc2_sqrt, const float* __restrict__ coef,
                             float grad_scale) {
  const float c = (coef ? coef[0] : 1.f) * grad_scale;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float g = to_f32(grad[i]) * c;
    float p = param[i];
    p *= 1.f - lr * weight_decay;
    const float mi = beta1 * m[i] + (1.f - beta1) * g;
    const float vi = beta2 * v[i] + (1.f - beta2) * g * g;
    m[i] = mi;
    v[i] = vi;
    p -= (lr / bc1) * mi / (sqrtf(vi) / bc2_sqrt + eps);
    param[i] = p;
    if (shadow) shadow[i] = __float2bfloat16(p);
  }
}

__global__ void cast_kernel(const float* __restrict__ src, __nv_bfloat16* __restrict__ dst, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = __float2bfloat16(src[i]);
}

}  // namespace lo
}  // namespace pra

cudaError_t pra_cross_entropy(__nv_bfloat16* logits, int64_t M, int64_t ld, int V, const int64_t* labels,
                              int ignore_index, float* row_loss, float* row_valid, cudaStream_t st) {
  if (M == 0) return cudaSuccess;
  pra::lo::ce_kernel<<<(unsigned)M, pra::lo::NT, 0, st>>>(logits, ld, V, labels, ignore_index, row_loss, row_valid);
  return cudaGetLastError();
}

constexpr int kNormParts = 592;  // 4 x 148 SMs
int pra_grad_norm_parts() { return kNormParts; }

cudaError_t pra_grad_norm(const void* grad, bool grad_bf16, int64_t n, float max_norm, float* part, float* norm_out,
                          float* coef_out, cudaStream_t st) {
  if (grad_bf16)
    pra::lo::sumsq_kernel<__nv_bfloat16><<<kNormParts, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(grad), n, part);
  else
    pra::lo::sumsq_kernel<float><<<kNormParts, 256, 0, st>>>(static_cast<const float*>(grad), n, part);
  PRA_RETURN_IF_ERROR(cudaGetLastError());
  pra::lo::finish_norm_kernel<<<1, 1024, 0, st>>>(part, kNormParts, max_norm, norm_out, coef_out);
  return cudaGetLastError();
}

cudaError_t pra_adamw(float* param, __nv_bfloat16* shadow, const void* grad, bool grad_bf16, float* m, float* v,
                      int64_t n, float lr, float beta1, float beta2, float eps, float weight_decay, int step,
                      const float* coef, float grad_scale, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  const float bc1 = 1.f - powf(beta1, (float)step);
  const float bc2_sqrt = sqrtf(1.f - powf(beta2, (float)step));
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, 148 * 16);
  if (grad_bf16)
    pra::lo::adamw_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(param, shadow, static_cast<const __nv_bfloat16*>(grad),
                                                                  m, v, n, lr, beta1, beta2, eps, weight_decay, bc1,
                                                                  bc2_sqrt, coef, grad_scale);
  else
    pra::lo::adamw_kernel<float><<<blocks, 256, 0, st>>>(param, shadow, static_cast<const float*>(grad), m, v, n, lr,
                                                          beta1, beta2, eps, weight_decay, bc1, bc2_sqrt, coef,
                                                          grad_scale);
  return cudaGetLastError();
}

cudaError_t pra_cast_f32_bf16(const float* src, __nv_bfloat16* dst, int64_t n, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, 148 * 16);
  pra::lo::cast_kernel<<<blocks, 256, 0, st>>>(src, dst, n);
  return cudaGetLastError();
}
