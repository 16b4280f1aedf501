// Counter-based dropout for the vanilla and mixed blocks' residual and MLP branches.
//
// Element e of a stream (seed, offset) draws word e % 4 of the Philox4x32-10 block e / 4
// (common.cuh): the mask is a pure function of (seed, offset, e), so the backward
// regenerates it instead of storing it, and any kernel (the attention kernels included)
// can draw the same bits.  Each thread handles 8 consecutive bf16 elements (two Philox
// blocks) with 16-byte loads when the pointers allow it.
#include <cmath>

#include "common.cuh"

namespace pra {
namespace dropout {

constexpr int NT = 256;

template <bool ADD>
__global__ void __launch_bounds__(NT) dropout_kernel(const __nv_bfloat16* res, const __nv_bfloat16* x,
                                                     __nv_bfloat16* y, int64_t n,
                                                     uint32_t thresh, float scale, uint64_t seed, uint64_t offset,
                                                     bool vec) {
  const int64_t i0 = ((int64_t)blockIdx.x * NT + threadIdx.x) * 8;
  if (i0 >= n) return;
  const uint4 r0 = dropout_block(seed, offset, i0 >> 2);
  const uint4 r1 = dropout_block(seed, offset, (i0 >> 2) + 1);
  const uint32_t words[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
  if (vec && i0 + 8 <= n) {
    uint4 xv = *reinterpret_cast<const uint4*>(x + i0);
    uint4 rv = make_uint4(0, 0, 0, 0);
    if (ADD) rv = *reinterpret_cast<const uint4*>(res + i0);
    const __nv_bfloat162* xp = reinterpret_cast<const __nv_bfloat162*>(&xv);
    const __nv_bfloat162* rp = reinterpret_cast<const __nv_bfloat162*>(&rv);
    uint32_t out[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = __bfloat1622float2(xp[j]);
      f.x = (words[2 * j] >> 8) >= thresh ? f.x * scale : 0.f;
      f.y = (words[2 * j + 1] >> 8) >= thresh ? f.y * scale : 0.f;
      if (ADD) {
        const float2 a = __bfloat1622float2(rp[j]);
        f.x += a.x;
        f.y += a.y;
      }
      out[j] = pack_bf16(f.x, f.y);
    }
    *reinterpret_cast<uint4*>(y + i0) = make_uint4(out[0], out[1], out[2], out[3]);
    return;
  }
  for (int j = 0; j < 8 && i0 + j < n; ++j) {
    float v = __bfloat162float(x[i0 + j]);
    v = (words[j] >> 8) >= thresh ? v * scale : 0.f;
    if (ADD) v += __bfloat162float(res[i0 + j]);
    y[i0 + j] = __float2bfloat16(v);
  }
}

}  // namespace dropout
}  // namespace pra

uint32_t pra_dropout_threshold(double p) {
  if (!(p > 0.0)) return 0;
  const double t = std::nearbyint(p * 16777216.0);
  return t >= 16777216.0 ? 16777216u : (uint32_t)t;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

cudaError_t pra_dropout(const __nv_bfloat16* x, __nv_bfloat16* y, int64_t n, uint32_t thresh, float scale,
                        uint64_t seed, uint64_t offset, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  const bool vec = aligned16(x) && aligned16(y);
  const unsigned blocks = (unsigned)((n + 8LL * pra::dropout::NT - 1) / (8LL * pra::dropout::NT));
  pra::dropout::dropout_kernel<false><<<blocks, pra::dropout::NT, 0, st>>>(nullptr, x, y, n, thresh, scale, seed,
                                                                           offset, vec);
  return cudaGetLastError();
}

cudaError_t pra_dropout_add(const __nv_bfloat16* res, const __nv_bfloat16* x, __nv_bfloat16* y, int64_t n,
                            uint32_t thresh, float scale, uint64_t seed, uint64_t offset, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  const bool vec = aligned16(x) && aligned16(y) && aligned16(res);
  const unsigned blocks = (unsigned)((n + 8LL * pra::dropout::NT - 1) / (8LL * pra::dropout::NT));
  pra::dropout::dropout_kernel<true><<<blocks, pra::dropout::NT, 0, st>>>(res, x, y, n, thresh, scale, seed, offset,
                                                                          vec);
  return cudaGetLastError();
}
