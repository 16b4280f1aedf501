// Chunk routing-gist construction on the device (cache build hot op).
//
// mean:   gist_k[c] = mean of the chunk's K rows, gist_v[c] = mean of its V rows,
//         gist_n[c] = gist_k[c] / max(||gist_k[c]||, 1e-12)   (routing copy).
// kmeans: one CTA per chunk: Lloyd in (optionally L2-normalised) key space,
//         kmeans++ or sampled initialisation driven by a precomputed random
//         stream (the draws a seeded CPU generator would make), farthest-point
//         reseed of empty clusters, then key / value gists as the means of the
//         original rows over the same assignments (occupied clusters only).
// K/V rows live in a token pool [tokens, D] (bf16); chunk c owns rows
// [start[c], start[c] + len[c]).
#include "common.cuh"

namespace pra {
namespace gist {

constexpr int NT = 256;
constexpr float EPS = 1e-12f;

__global__ void __launch_bounds__(NT) mean_kernel(const __nv_bfloat16* __restrict__ pk, const __nv_bfloat16* __restrict__ pv,
                                                  int64_t row_stride, const int* __restrict__ start,
                                                  const int* __restrict__ len, int D, float* __restrict__ gk,
                                                  float* __restrict__ gv, float* __restrict__ gn) {
  __shared__ float scratch[32];
  const int c = blockIdx.x;
  const int s = start[c], n = len[c];
  const float inv_n = n > 0 ? 1.f / n : 0.f;
  float sq = 0.f;
  for (int d = threadIdx.x; d < D; d += NT) {
    float ak = 0.f, av = 0.f;
    for (int i = 0; i < n; ++i) {
      ak += __bfloat162float(pk[(int64_t)(s + i) * row_stride + d]);
      av += __bfloat162float(pv[(int64_t)(s + i) * row_stride + d]);
    }
    ak *= inv_n;
    av *= inv_n;
    gk[(int64_t)c * D + d] = ak;
    gv[(int64_t)c * D + d] = av;
    sq += ak * ak;
  }
  const float inv = 1.f / fmaxf(sqrtf(block_sum(sq, scratch)), EPS);
  for (int d = threadIdx.x; d < D; d += NT) gn[(int64_t)c * D + d] = gk[(int64_t)c * D + d] * inv;
}

struct KMeansArgs {
  const __nv_bfloat16* pk;
  const __nv_bfloat16* pv;
  int64_t row_stride;
  const int* start;
  const int* len;
  int D, G, max_iters;
  float tol;
  bool normalize, kmeanspp, farthest;
  const int* init_first;      // [C] kmeans++ first index, or offset into init_idx for sampled init
  const int* init_idx;        // flat sampled indices
  const float* exp_draws;     // flat Exp(1) draws
  const int64_t* exp_off;     // [C] offset of this chunk's [G-1, N] draws
  float* gk;                  // [C, G, D]
  float* gv;                  // [C, G, D]
  int* count;                 // [C] occupied clusters
  int* occupancy;             // [C, G]
  int* iterations;            // [C]
  int* status;                // [C] 0 ok, 1 empty-cluster error
};

constexpr int MAXN = 1024;
constexpr int MAXG = 8;

// squared distance from (optionally normalised) point i to each of `nc` centres.
__device__ void point_dists(const KMeansArgs& a, int s, int i, const float* inv_norm, const float* centers, int nc,
                            float* out) {
  const int lane = threadIdx.x & 31;
  float acc[MAXG];
#pragma unroll
  for (int c = 0; c < MAXG; ++c) acc[c] = 0.f;
  const float sc = a.normalize ? inv_norm[i] : 1.f;
  for (int d = lane; d < a.D; d += 32) {
    const float w = __bfloat162float(a.pk[(int64_t)(s + i) * a.row_stride + d]) * sc;
#pragma unroll
    for (int c = 0; c < MAXG; ++c) {
      if (c < nc) {
        const float diff = w - centers[c * a.D + d];
        acc[c] += diff * diff;
      }
    }
  }
#pragma unroll
  for (int c = 0; c < MAXG; ++c) {
    if (c < nc) {
      const float v = warp_sum(acc[c]);
      if (lane == 0) out[c] = v;
    }
  }
}

__global__ void __launch_bounds__(NT) kmeans_kernel(KMeansArgs a) {
  extern __shared__ __align__(16) float sm[];
  float* centers = sm;                       // [G, D]
  float* next = centers + a.G * a.D;         // [G, D]
  float* inv_norm = next + a.G * a.D;        // [MAXN]
  float* dmin = inv_norm + MAXN;             // [MAXN]
  float* dist = dmin + MAXN;                 // [MAXN, MAXG]
  int* assign = reinterpret_cast<int*>(dist + MAXN * MAXG);  // [MAXN]
  __shared__ int members[MAXG];
  __shared__ int chosen[MAXG];
  __shared__ float scratch[32];
  __shared__ int pick;

  const int c = blockIdx.x;
  const int s = a.start[c], n = min(a.len[c], MAXN);
  const int G = min(a.G, n);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = NT / 32;
  const int D = a.D;
  if (threadIdx.x == 0) a.status[c] = 0;
  if (G == 0) {
    if (threadIdx.x == 0) {
      a.count[c] = 0;
      a.iterations[c] = 0;
    }
    return;
  }
  // row norms of the keys (normalised working space)
  for (int i = warp; i < n; i += nwarps) {
    float acc = 0.f;
    for (int d = lane; d < D; d += 32) {
      const float v = __bfloat162float(a.pk[(int64_t)(s + i) * a.row_stride + d]);
      acc += v * v;
    }
    acc = warp_sum(acc);
    if (lane == 0) inv_norm[i] = 1.f / fmaxf(sqrtf(acc), EPS);
  }
  __syncthreads();
  auto work = [&](int i, int d) {
    const float v = __bfloat162float(a.pk[(int64_t)(s + i) * a.row_stride + d]);
    return a.normalize ? v * inv_norm[i] : v;
  };
  // ---- initialisation ----
  if (a.kmeanspp) {
    if (threadIdx.x == 0) chosen[0] = a.init_first[c];
    __syncthreads();
    for (int d = threadIdx.x; d < D; d += NT) centers[d] = work(chosen[0], d);
    __syncthreads();
    for (int j = 1; j < G; ++j) {
      for (int i = warp; i < n; i += nwarps) {
        point_dists(a, s, i, inv_norm, centers, j, dist + i * MAXG);
      }
      __syncthreads();
      float part = 0.f;
      for (int i = threadIdx.x; i < n; i += NT) {
        float m = INFINITY;
        for (int q = 0; q < j; ++q) m = fminf(m, dist[i * MAXG + q]);
        bool taken = false;
        for (int q = 0; q < j; ++q) taken |= (chosen[q] == i);
        dmin[i] = taken ? 0.f : m;
        part += dmin[i];
      }
      const float total = block_sum(part, scratch);
      if (threadIdx.x == 0) {
        int nxt = -1;
        if (total > 0.f) {
          const float* e = a.exp_draws + a.exp_off[c] + (int64_t)(j - 1) * n;
          float best = -INFINITY;
          for (int i = 0; i < n; ++i) {
            const float q = (dmin[i] / total) / e[i];
            if (q > best) {
              best = q;
              nxt = i;
            }
          }
        }
        bool dup = nxt < 0;
        for (int q = 0; q < j && !dup; ++q) dup = (chosen[q] == nxt);
        if (dup) {
          for (int i = 0; i < n; ++i) {
            bool used = false;
            for (int q = 0; q < j; ++q) used |= (chosen[q] == i);
            if (!used) {
              nxt = i;
              break;
            }
          }
        }
        chosen[j] = nxt;
      }
      __syncthreads();
      for (int d = threadIdx.x; d < D; d += NT) centers[j * D + d] = work(chosen[j], d);
      __syncthreads();
    }
  } else {
    for (int j = 0; j < G; ++j)
      for (int d = threadIdx.x; d < D; d += NT) centers[j * D + d] = work(a.init_idx[a.init_first[c] + j], d);
    __syncthreads();
  }
  // ---- Lloyd iterations ----
  int it = 0;
  for (it = 1; it <= a.max_iters; ++it) {
    for (int i = warp; i < n; i += nwarps) point_dists(a, s, i, inv_norm, centers, G, dist + i * MAXG);
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += NT) {
      int bi = 0;
      float bd = dist[i * MAXG];
      for (int q = 1; q < G; ++q)
        if (dist[i * MAXG + q] < bd) {
          bd = dist[i * MAXG + q];
          bi = q;
        }
      assign[i] = bi;
      dmin[i] = bd;
    }
    if (threadIdx.x < MAXG) members[threadIdx.x] = 0;
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int i = 0; i < n; ++i) members[assign[i]]++;
      int far = 0;
      for (int i = 1; i < n; ++i)
        if (dmin[i] > dmin[far]) far = i;
      pick = far;
      for (int q = 0; q < G; ++q)
        if (members[q] == 0 && !a.farthest) a.status[c] = 1;
    }
    __syncthreads();
    for (int q = 0; q < G; ++q) {
      for (int d = threadIdx.x; d < D; d += NT) {
        float v;
        if (members[q] == 0) {
          v = work(pick, d);
        } else {
          float acc = 0.f;
          for (int i = 0; i < n; ++i)
            if (assign[i] == q) acc += work(i, d);
          v = acc / members[q];
        }
        next[q * D + d] = v;
      }
    }
    __syncthreads();
    float shift = 0.f;
    for (int q = 0; q < G; ++q) {
      float part = 0.f;
      for (int d = threadIdx.x; d < D; d += NT) {
        const float df = next[q * D + d] - centers[q * D + d];
        part += df * df;
      }
      shift = fmaxf(shift, sqrtf(block_sum(part, scratch)));
    }
    for (int i = threadIdx.x; i < G * D; i += NT) centers[i] = next[i];
    __syncthreads();
    if (shift <= a.tol) break;
  }
  if (it > a.max_iters) it = a.max_iters;
  // ---- final assignment and paired means over original rows ----
  for (int i = warp; i < n; i += nwarps) point_dists(a, s, i, inv_norm, centers, G, dist + i * MAXG);
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += NT) {
    int bi = 0;
    float bd = dist[i * MAXG];
    for (int q = 1; q < G; ++q)
      if (dist[i * MAXG + q] < bd) {
        bd = dist[i * MAXG + q];
        bi = q;
      }
    assign[i] = bi;
  }
  if (threadIdx.x < MAXG) members[threadIdx.x] = 0;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 0; i < n; ++i) members[assign[i]]++;
    int slot = 0;
    for (int q = 0; q < G; ++q) {
      chosen[q] = members[q] ? slot : -1;
      if (members[q]) a.occupancy[c * a.G + slot++] = members[q];
    }
    a.count[c] = slot;
    a.iterations[c] = it;
  }
  __syncthreads();
  for (int q = 0; q < G; ++q) {
    const int slot = chosen[q];
    if (slot < 0) continue;
    float part = 0.f;
    for (int d = threadIdx.x; d < D; d += NT) {
      float ak = 0.f, av = 0.f;
      for (int i = 0; i < n; ++i) {
        if (assign[i] != q) continue;
        ak += __bfloat162float(a.pk[(int64_t)(s + i) * a.row_stride + d]);
        av += __bfloat162float(a.pv[(int64_t)(s + i) * a.row_stride + d]);
      }
      ak /= members[q];
      av /= members[q];
      a.gk[((int64_t)c * a.G + slot) * D + d] = ak;
      a.gv[((int64_t)c * a.G + slot) * D + d] = av;
      part += ak * ak;
    }
    if (a.normalize) {
      const float inv = 1.f / fmaxf(sqrtf(block_sum(part, scratch)), EPS);
      for (int d = threadIdx.x; d < D; d += NT) a.gk[((int64_t)c * a.G + slot) * D + d] *= inv;
    }
    __syncthreads();
  }
}

}  // namespace gist
}  // namespace pra

cudaError_t pra_gist_mean(const __nv_bfloat16* pk, const __nv_bfloat16* pv, int64_t row_stride, const int* start,
                          const int* len, int C, int D, float* gk, float* gv, float* gn, cudaStream_t st) {
  if (C == 0) return cudaSuccess;
  pra::gist::mean_kernel<<<C, pra::gist::NT, 0, st>>>(pk, pv, row_stride, start, len, D, gk, gv, gn);
  return cudaGetLastError();
}

cudaError_t pra_gist_kmeans(const __nv_bfloat16* pk, const __nv_bfloat16* pv, int64_t row_stride, const int* start,
                            const int* len, int C, int D, int G, int max_iters, float tol, bool normalize,
                            bool kmeanspp, bool farthest, const int* init_first, const int* init_idx,
                            const float* exp_draws, const int64_t* exp_off, float* gk, float* gv, int* count,
                            int* occupancy, int* iterations, int* status, cudaStream_t st) {
  using namespace pra::gist;
  if (C == 0) return cudaSuccess;
  if (G > MAXG) return cudaErrorInvalidValue;
  KMeansArgs a{pk, pv, row_stride, start, len, D, G, max_iters, tol, normalize, kmeanspp, farthest, init_first,
               init_idx, exp_draws, exp_off, gk, gv, count, occupancy, iterations, status};
  const size_t smem = (size_t)(2 * G * D + 2 * MAXN + MAXN * MAXG) * sizeof(float) + MAXN * sizeof(int);
  PRA_RETURN_IF_ERROR(cudaFuncSetAttribute(kmeans_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  kmeans_kernel<<<C, NT, smem, st>>>(a);
  return cudaGetLastError();
}
