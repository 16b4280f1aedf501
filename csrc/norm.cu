// LayerNorm / RMSNorm forward and backward on bf16 rows (fp32 statistics).
//
// Forward: y = (x - mean) * rstd * w (+ b)   [RMSNorm: mean = 0, rstd = 1/sqrt(mean(x^2)+eps)]
// Backward: dx = rstd * (w*dy - mean(w*dy) - xhat * mean(w*dy*xhat)) (+ residual grad),
//           dw/db accumulated per CTA into fp32 partials and reduced by a second kernel.
#include "common.cuh"

namespace pra {
namespace norm {

constexpr int NT = 256;
constexpr int MAXV = 8;  // up to 8 bf16x2 pairs per thread: D <= 4096

template <bool RMS>
__global__ void __launch_bounds__(NT) fwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                                                 const __nv_bfloat16* __restrict__ b, __nv_bfloat16* __restrict__ y,
                                                 float* __restrict__ mean_out, float* __restrict__ rstd_out, int M,
                                                 int D, float eps) {
  __shared__ float scratch[32];
  pdl_launch_dependents();
  pdl_wait();
  const int row = blockIdx.x;
  if (row >= M) return;
  const __nv_bfloat162* xr = reinterpret_cast<const __nv_bfloat162*>(x + (int64_t)row * D);
  float2 vals[MAXV];
  float s = 0.f, ss = 0.f;
  int n = 0;
  for (int i = threadIdx.x; i < D / 2; i += NT, ++n) {
    vals[n] = __bfloat1622float2(xr[i]);
    s += vals[n].x + vals[n].y;
    ss += vals[n].x * vals[n].x + vals[n].y * vals[n].y;
  }
  float mean = 0.f, var;
  if (RMS) {
    var = block_sum(ss, scratch) / D;
  } else {
    mean = block_sum(s, scratch) / D;
    float dev = 0.f;
    for (int j = 0; j < n; ++j) {
      const float a = vals[j].x - mean, c = vals[j].y - mean;
      dev += a * a + c * c;
    }
    var = block_sum(dev, scratch) / D;
  }
  const float rstd = rsqrtf(var + eps);
  const __nv_bfloat162* wr = reinterpret_cast<const __nv_bfloat162*>(w);
  const __nv_bfloat162* br = reinterpret_cast<const __nv_bfloat162*>(b);
  __nv_bfloat162* yr = reinterpret_cast<__nv_bfloat162*>(y + (int64_t)row * D);
  n = 0;
  for (int i = threadIdx.x; i < D / 2; i += NT, ++n) {
    const float2 wv = __bfloat1622float2(wr[i]);
    const float2 bv = b ? __bfloat1622float2(br[i]) : make_float2(0.f, 0.f);
    yr[i] = __floats2bfloat162_rn((vals[n].x - mean) * rstd * wv.x + bv.x, (vals[n].y - mean) * rstd * wv.y + bv.y);
  }
  if (threadIdx.x == 0) {
    if (mean_out) mean_out[row] = mean;
    rstd_out[row] = rstd;
  }
}

// Warp-per-row variants for D <= 1024 (every TinyGPT width): 16-byte loads, shuffle-only
// reductions, 8 rows per 256-thread CTA.  Lane l owns the 8-element chunks l, l + 32, ...
constexpr int WCH = 4;  // chunks of 8 per lane: D <= 32 * 8 * WCH = 1024

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float* f) {
  const uint4 raw = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 v = __bfloat1622float2(h[i]);
    f[2 * i] = v.x;
    f[2 * i + 1] = v.y;
  }
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float* f) {
  uint4 raw;
  uint32_t* r = reinterpret_cast<uint32_t*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) r[i] = pack_bf16(f[2 * i], f[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = raw;
}

template <bool RMS>
__global__ void __launch_bounds__(256) fwd_warp_kernel(const __nv_bfloat16* __restrict__ x,
                                                       const __nv_bfloat16* __restrict__ w,
                                                       const __nv_bfloat16* __restrict__ b, __nv_bfloat16* __restrict__ y,
                                                       float* __restrict__ mean_out, float* __restrict__ rstd_out,
                                                       int M, int D, float eps) {
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= M) return;
  const int C = D / 8;
  const __nv_bfloat16* xr = x + (int64_t)row * D;
  float v[WCH][8];
  float s = 0.f, ss = 0.f;
#pragma unroll
  for (int j = 0; j < WCH; ++j) {
    const int c = lane + 32 * j;
    if (c < C) {
      load8(xr + 8 * c, v[j]);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        s += v[j][e];
        ss += v[j][e] * v[j][e];
      }
    }
  }
  float mean = 0.f, var;
  if (RMS) {
    var = warp_sum(ss) / D;
  } else {
    mean = warp_sum(s) / D;
    float dev = 0.f;
#pragma unroll
    for (int j = 0; j < WCH; ++j)
      if (lane + 32 * j < C)
#pragma unroll
        for (int e = 0; e < 8; ++e) dev += (v[j][e] - mean) * (v[j][e] - mean);
    var = warp_sum(dev) / D;
  }
  const float rstd = rsqrtf(var + eps);
#pragma unroll
  for (int j = 0; j < WCH; ++j) {
    const int c = lane + 32 * j;
    if (c < C) {
      float wv[8], bv[8], o[8];
      load8(w + 8 * c, wv);
      if (b) load8(b + 8 * c, bv);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = (v[j][e] - mean) * rstd * wv[e] + (b ? bv[e] : 0.f);
      store8(y + (int64_t)row * D + 8 * c, o);
    }
  }
  if (lane == 0) {
    if (mean_out) mean_out[row] = mean;
    rstd_out[row] = rstd;
  }
}

// Backward, warp per row; each warp keeps its columns' dw/db sums in registers, the CTA
// combines its 8 warps in a fixed order (deterministic) and writes one partial row.
template <bool RMS>
__global__ void __launch_bounds__(256) bwd_warp_kernel(const __nv_bfloat16* __restrict__ dy,
                                                       const __nv_bfloat16* __restrict__ x,
                                                       const __nv_bfloat16* __restrict__ w,
                                                       const float* __restrict__ mean_in,
                                                       const float* __restrict__ rstd_in,
                                                       const __nv_bfloat16* __restrict__ dres,
                                                       __nv_bfloat16* __restrict__ dx, float* __restrict__ dw_part,
                                                       float* __restrict__ db_part, int M, int D, int rows_per_cta) {
  extern __shared__ float red[];  // [8][2][D]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int C = D / 8;
  float aw[WCH][8], ab[WCH][8];
#pragma unroll
  for (int j = 0; j < WCH; ++j)
#pragma unroll
    for (int e = 0; e < 8; ++e) aw[j][e] = ab[j][e] = 0.f;
  const int r0 = blockIdx.x * rows_per_cta, r1 = min(r0 + rows_per_cta, M);
  // x / dy of the warp's next row are loaded while the current row is reduced
  uint4 xr[WCH], gr[WCH];
  float mean_n = 0.f, rstd_n = 0.f;
  auto fetch = [&](int row) {
#pragma unroll
    for (int j = 0; j < WCH; ++j) {
      const int c = lane + 32 * j;
      if (c < C) {
        xr[j] = *reinterpret_cast<const uint4*>(x + (int64_t)row * D + 8 * c);
        gr[j] = *reinterpret_cast<const uint4*>(dy + (int64_t)row * D + 8 * c);
      }
    }
    mean_n = RMS ? 0.f : mean_in[row];
    rstd_n = rstd_in[row];
  };
  if (r0 + warp < r1) fetch(r0 + warp);
  for (int row = r0 + warp; row < r1; row += 8) {
    const float mean = mean_n, rstd = rstd_n;
    uint4 xc[WCH], gc[WCH];
#pragma unroll
    for (int j = 0; j < WCH; ++j) {
      xc[j] = xr[j];
      gc[j] = gr[j];
    }
    if (row + 8 < r1) fetch(row + 8);
    float xh[WCH][8], wg[WCH][8];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int j = 0; j < WCH; ++j) {
      const int c = lane + 32 * j;
      if (c < C) {
        float xv[8], gv[8], wv[8];
        load8(reinterpret_cast<const __nv_bfloat16*>(&xc[j]), xv);
        load8(reinterpret_cast<const __nv_bfloat16*>(&gc[j]), gv);
        load8(w + 8 * c, wv);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          xh[j][e] = (xv[e] - mean) * rstd;
          wg[j][e] = gv[e] * wv[e];
          s1 += wg[j][e];
          s2 += wg[j][e] * xh[j][e];
          aw[j][e] += gv[e] * xh[j][e];
          ab[j][e] += gv[e];
        }
      }
    }
    const float m1 = RMS ? 0.f : warp_sum(s1) / D;
    const float m2 = warp_sum(s2) / D;
#pragma unroll
    for (int j = 0; j < WCH; ++j) {
      const int c = lane + 32 * j;
      if (c < C) {
        float o[8], rv[8];
        if (dres) load8(dres + (int64_t)row * D + 8 * c, rv);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = rstd * (wg[j][e] - m1 - xh[j][e] * m2) + (dres ? rv[e] : 0.f);
        store8(dx + (int64_t)row * D + 8 * c, o);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < WCH; ++j) {
    const int c = lane + 32 * j;
    if (c < C)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        red[(warp * 2) * D + 8 * c + e] = aw[j][e];
        red[(warp * 2 + 1) * D + 8 * c + e] = ab[j][e];
      }
  }
  __syncthreads();
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float sw = 0.f, sb = 0.f;
    for (int q = 0; q < 8; ++q) {
      sw += red[(q * 2) * D + d];
      sb += red[(q * 2 + 1) * D + d];
    }
    dw_part[(int64_t)blockIdx.x * D + d] = sw;
    if (db_part) db_part[(int64_t)blockIdx.x * D + d] = sb;
  }
}

// Each CTA handles `rows_per_cta` rows; writes fp32 partial dw/db [gridDim.x, D].
template <bool RMS>
__global__ void __launch_bounds__(NT) bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                                 const __nv_bfloat16* __restrict__ w, const float* __restrict__ mean_in,
                                                 const float* __restrict__ rstd_in,
                                                 const __nv_bfloat16* __restrict__ dres, __nv_bfloat16* __restrict__ dx,
                                                 float* __restrict__ dw_part, float* __restrict__ db_part, int M, int D,
                                                 int rows_per_cta) {
  __shared__ float scratch[32];
  float2 accw[MAXV], accb[MAXV];
#pragma unroll
  for (int j = 0; j < MAXV; ++j) accw[j] = accb[j] = make_float2(0.f, 0.f);
  const __nv_bfloat162* wr = reinterpret_cast<const __nv_bfloat162*>(w);
  const int r0 = blockIdx.x * rows_per_cta;
  const int r1 = min(r0 + rows_per_cta, M);
  for (int row = r0; row < r1; ++row) {
    const __nv_bfloat162* xr = reinterpret_cast<const __nv_bfloat162*>(x + (int64_t)row * D);
    const __nv_bfloat162* gr = reinterpret_cast<const __nv_bfloat162*>(dy + (int64_t)row * D);
    const float mean = RMS ? 0.f : mean_in[row];
    const float rstd = rstd_in[row];
    float2 xh[MAXV], wg[MAXV];
    float s1 = 0.f, s2 = 0.f;
    int n = 0;
    for (int i = threadIdx.x; i < D / 2; i += NT, ++n) {
      const float2 xv = __bfloat1622float2(xr[i]);
      const float2 gv = __bfloat1622float2(gr[i]);
      const float2 wv = __bfloat1622float2(wr[i]);
      xh[n] = make_float2((xv.x - mean) * rstd, (xv.y - mean) * rstd);
      wg[n] = make_float2(gv.x * wv.x, gv.y * wv.y);
      s1 += wg[n].x + wg[n].y;
      s2 += wg[n].x * xh[n].x + wg[n].y * xh[n].y;
      accw[n].x += gv.x * xh[n].x;
      accw[n].y += gv.y * xh[n].y;
      accb[n].x += gv.x;
      accb[n].y += gv.y;
    }
    const float m1 = RMS ? 0.f : block_sum(s1, scratch) / D;
    const float m2 = block_sum(s2, scratch) / D;
    __nv_bfloat162* out = reinterpret_cast<__nv_bfloat162*>(dx + (int64_t)row * D);
    const __nv_bfloat162* rr = dres ? reinterpret_cast<const __nv_bfloat162*>(dres + (int64_t)row * D) : nullptr;
    n = 0;
    for (int i = threadIdx.x; i < D / 2; i += NT, ++n) {
      float gx = rstd * (wg[n].x - m1 - xh[n].x * m2);
      float gy = rstd * (wg[n].y - m1 - xh[n].y * m2);
      if (rr) {
        const float2 rv = __bfloat1622float2(rr[i]);
        gx += rv.x;
        gy += rv.y;
      }
      out[i] = __floats2bfloat162_rn(gx, gy);
    }
  }
  int n = 0;
  for (int i = threadIdx.x; i < D / 2; i += NT, ++n) {
    dw_part[(int64_t)blockIdx.x * D + 2 * i] = accw[n].x;
    dw_part[(int64_t)blockIdx.x * D + 2 * i + 1] = accw[n].y;
    if (db_part) {
      db_part[(int64_t)blockIdx.x * D + 2 * i] = accb[n].x;
      db_part[(int64_t)blockIdx.x * D + 2 * i + 1] = accb[n].y;
    }
  }
}

// out[d] = sum_p part[p, d] (fp32 -> out dtype).  A block of 256 threads takes 32 columns:
// warp w sums partial rows w, w + 8, ... (one coalesced 128-byte row segment per load), then
// the eight warp sums are added in a fixed order (deterministic).
template <typename T>
__global__ void __launch_bounds__(256) column_reduce_kernel(const float* __restrict__ part, int P, int D,
                                                            T* __restrict__ out) {
  __shared__ float red[8][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int d = blockIdx.x * 32 + tx;
  float acc = 0.f;
  if (d < D) {
#pragma unroll 4
    for (int p = ty; p < P; p += 8) acc += part[(int64_t)p * D + d];
  }
  red[ty][tx] = acc;
  __syncthreads();
  if (ty == 0 && d < D) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s += red[i][tx];
    out[d] = from_f32<T>(s);
  }
}

}  // namespace norm
}  // namespace pra

cudaError_t pra_norm_fwd(const __nv_bfloat16* x, const __nv_bfloat16* w, const __nv_bfloat16* b, __nv_bfloat16* y,
                         float* mean, float* rstd, int M, int D, float eps, bool rms, cudaStream_t st) {
  using namespace pra::norm;
  if (D % 2 || D / 2 > NT * MAXV) return cudaErrorInvalidValue;
  if (M == 0) return cudaSuccess;
  if (D % 8 == 0 && D <= 32 * 8 * WCH) {
    const int blocks = (M + 7) / 8;
    const __nv_bfloat16* no_bias = nullptr;
    float* no_mean = nullptr;
    if (rms)
      return pra_launch_pdl(fwd_warp_kernel<true>, dim3(blocks), dim3(256), 0, st, x, w, no_bias, y, no_mean, rstd, M, D,
                            eps);
    return pra_launch_pdl(fwd_warp_kernel<false>, dim3(blocks), dim3(256), 0, st, x, w, b, y, mean, rstd, M, D, eps);
  }
  const __nv_bfloat16* no_bias = nullptr;
  float* no_mean = nullptr;
  if (rms) return pra_launch_pdl(fwd_kernel<true>, dim3(M), dim3(NT), 0, st, x, w, no_bias, y, no_mean, rstd, M, D, eps);
  return pra_launch_pdl(fwd_kernel<false>, dim3(M), dim3(NT), 0, st, x, w, b, y, mean, rstd, M, D, eps);
}

// 16 rows per CTA (two per warp, twice the warps per SM of 32-row CTAs): an 8,192 x 768
// LayerNorm backward measured 28.6 -> 25.1 us.
int pra_norm_bwd_partials(int M) { return M == 0 ? 1 : (M + 15) / 16 > 592 ? 592 : (M + 15) / 16; }

cudaError_t pra_norm_bwd(const __nv_bfloat16* dy, const __nv_bfloat16* x, const __nv_bfloat16* w, const float* mean,
                         const float* rstd, const __nv_bfloat16* dres, __nv_bfloat16* dx, float* dw_part,
                         float* db_part, __nv_bfloat16* dw, __nv_bfloat16* db, int M, int D, bool rms,
                         cudaStream_t st) {
  using namespace pra::norm;
  if (D % 2 || D / 2 > NT * MAXV) return cudaErrorInvalidValue;
  const int parts = pra_norm_bwd_partials(M);
  const int rows = M == 0 ? 0 : (M + parts - 1) / parts;
  if (D % 8 == 0 && D <= 32 * 8 * WCH) {
    const size_t smem = (size_t)16 * D * sizeof(float);
    if (rms) {
      PRA_RETURN_IF_ERROR(pra::set_max_dynamic_smem(reinterpret_cast<const void*>(bwd_warp_kernel<true>), (int)smem));
      bwd_warp_kernel<true><<<parts, 256, smem, st>>>(dy, x, w, nullptr, rstd, dres, dx, dw_part, nullptr, M, D, rows);
    } else {
      PRA_RETURN_IF_ERROR(pra::set_max_dynamic_smem(reinterpret_cast<const void*>(bwd_warp_kernel<false>), (int)smem));
      bwd_warp_kernel<false><<<parts, 256, smem, st>>>(dy, x, w, mean, rstd, dres, dx, dw_part, db_part, M, D, rows);
    }
  } else if (rms) {
    bwd_kernel<true><<<parts, NT, 0, st>>>(dy, x, w, nullptr, rstd, dres, dx, dw_part, nullptr, M, D, rows);
  } else {
    bwd_kernel<false><<<parts, NT, 0, st>>>(dy, x, w, mean, rstd, dres, dx, dw_part, db_part, M, D, rows);
  }
  PRA_RETURN_IF_ERROR(cudaGetLastError());
  column_reduce_kernel<__nv_bfloat16><<<(D + 31) / 32, 256, 0, st>>>(dw_part, parts, D, dw);
  if (!rms && db) column_reduce_kernel<__nv_bfloat16><<<(D + 31) / 32, 256, 0, st>>>(db_part, parts, D, db);
  return cudaGetLastError();
}

// Column sums of a bf16 matrix [M, N] (bias gradients): two-stage, deterministic.
namespace pra {
namespace norm {
__global__ void colsum_partial_kernel(const __nv_bfloat16* __restrict__ g, int M, int N, int rows_per_cta,
                                      float* __restrict__ part) {
  const int col2 = blockIdx.y * blockDim.x + threadIdx.x;  // bf16x2 column
  if (col2 * 2 >= N) return;
  const int r0 = blockIdx.x * rows_per_cta, r1 = min(r0 + rows_per_cta, M);
  float ax = 0.f, ay = 0.f;
  for (int r = r0; r < r1; ++r) {
    const float2 v = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(g + (int64_t)r * N)[col2]);
    ax += v.x;
    ay += v.y;
  }
  part[(int64_t)blockIdx.x * N + 2 * col2] = ax;
  part[(int64_t)blockIdx.x * N + 2 * col2 + 1] = ay;
}
}  // namespace norm
}  // namespace pra

int pra_colsum_partials(int M) { return M == 0 ? 1 : ((M + 63) / 64 > 256 ? 256 : (M + 63) / 64); }

cudaError_t pra_colsum(const __nv_bfloat16* g, int M, int N, float* part, __nv_bfloat16* out, cudaStream_t st) {
  using namespace pra::norm;
  if (N % 2) return cudaErrorInvalidValue;
  const int parts = pra_colsum_partials(M);
  const int rows = M == 0 ? 0 : (M + parts - 1) / parts;
  dim3 grid(parts, (N / 2 + 255) / 256);
  colsum_partial_kernel<<<grid, 256, 0, st>>>(g, M, N, rows, part);
  PRA_RETURN_IF_ERROR(cudaGetLastError());
  column_reduce_kernel<__nv_bfloat16><<<(N + 31) / 32, 256, 0, st>>>(part, parts, N, out);
  return cudaGetLastError();
}
