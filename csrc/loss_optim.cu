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

// Same outputs as ce_kernel with the row read from global memory once: 16-byte loads stage
// the row (ld bf16 values, ld % 8 == 0) in shared memory while each thread keeps an online
// (max, sum of exp) pair; the pairs are merged across the block, then the gradient is written
// from the staged copy.  Global traffic: one read and one write of the row.
__device__ __forceinline__ void merge_max_sum(float& m, float& s, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  if (mn == -INFINITY) return;
  s = s * __expf(m - mn) + s2 * __expf(m2 - mn);
  m = mn;
}

__global__ void __launch_bounds__(NT) ce_staged_kernel(__nv_bfloat16* __restrict__ logits, int64_t ld, int V,
                                                       const int64_t* __restrict__ labels, int ignore_index,
                                                       float* __restrict__ row_loss, float* __restrict__ row_valid) {
  extern __shared__ __align__(16) __nv_bfloat16 srow[];
  __shared__ float wm[NT / 32], ws[NT / 32];
  const int64_t row = blockIdx.x;
  __nv_bfloat16* lr = logits + row * ld;
  const int64_t label = labels[row];
  const bool valid = label != ignore_index && label >= 0 && label < V;
  const int nvec = (int)(ld / 8);
  float m = -INFINITY, s = 0.f;
  for (int v = threadIdx.x; v < nvec; v += NT) {
    const uint4 raw = reinterpret_cast<const uint4*>(lr)[v];
    reinterpret_cast<uint4*>(srow)[v] = raw;
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
    float x[8], mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      x[k] = v * 8 + k < V ? __bfloat162float(e[k]) : -INFINITY;
      mx = fmaxf(mx, x[k]);
    }
    if (mx == -INFINITY) continue;
    float add = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) add += __expf(x[k] - mx);
    merge_max_sum(m, s, mx, add);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    merge_max_sum(m, s, m2, s2);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    wm[warp] = m;
    ws[warp] = s;
  }
  __syncthreads();  // also: the staged row is complete
  m = wm[0];
  s = ws[0];
  for (int w = 1; w < NT / 32; ++w) merge_max_sum(m, s, wm[w], ws[w]);
  const float lse = m + __logf(s);
  const float target = valid ? __bfloat162float(srow[label]) : 0.f;
  const float inv = 1.f / s;
  for (int v = threadIdx.x; v < nvec; v += NT) {
    const uint4 raw = reinterpret_cast<const uint4*>(srow)[v];
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
    uint4 out;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
    for (int k = 0; k < 8; k += 2) {
      float g[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int i = v * 8 + k + u;
        g[u] = (valid && i < V) ? __expf(__bfloat162float(e[k + u]) - m) * inv - (i == label ? 1.f : 0.f) : 0.f;
      }
      ow[k / 2] = pack_bf16(g[0], g[1]);
    }
    reinterpret_cast<uint4*>(lr)[v] = out;
  }
  if (threadIdx.x == 0) {
    row_loss[row] = valid ? lse - target : 0.f;
    row_valid[row] = valid ? 1.f : 0.f;
  }
}

// Sum of squares of a bf16 buffer into per-CTA partials with 16-byte loads (n % 8 == 0,
// 16-byte aligned); same partial layout as sumsq_kernel.
__global__ void sumsq_bf16x8_kernel(const __nv_bfloat16* __restrict__ g, int64_t n, float* __restrict__ part) {
  __shared__ float scratch[32];
  float acc = 0.f;
  const int64_t nv = n / 8;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 raw = reinterpret_cast<const uint4*>(g)[i];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 v = __bfloat1622float2(h[k]);
      acc += v.x * v.x + v.y * v.y;
    }
  }
  acc = block_sum(acc, scratch);
  if (threadIdx.x == 0) part[blockIdx.x] = acc;
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
  const size_t staged = (size_t)ld * sizeof(__nv_bfloat16);
  if (ld % 8 == 0 && (reinterpret_cast<uintptr_t>(logits) & 15) == 0 && staged <= 200 * 1024) {
    PRA_RETURN_IF_ERROR(pra::set_max_dynamic_smem(reinterpret_cast<const void*>(pra::lo::ce_staged_kernel), (int)staged));
    pra::lo::ce_staged_kernel<<<(unsigned)M, pra::lo::NT, staged, st>>>(logits, ld, V, labels, ignore_index, row_loss,
                                                                         row_valid);
    return cudaGetLastError();
  }
  pra::lo::ce_kernel<<<(unsigned)M, pra::lo::NT, 0, st>>>(logits, ld, V, labels, ignore_index, row_loss, row_valid);
  return cudaGetLastError();
}

constexpr int kNormParts = 592;  // 4 x 148 SMs
int pra_grad_norm_parts() { return kNormParts; }

cudaError_t pra_grad_norm(const void* grad, bool grad_bf16, int64_t n, float max_norm, float* part, float* norm_out,
                          float* coef_out, cudaStream_t st) {
  if (grad_bf16)
    if (n % 8 == 0 && (reinterpret_cast<uintptr_t>(grad) & 15) == 0)
      pra::lo::sumsq_bf16x8_kernel<<<kNormParts, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(grad), n, part);
    else
      pra::lo::sumsq_kernel<__nv_bfloat16><<<kNormParts, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(grad), n,
                                                                      part);
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
