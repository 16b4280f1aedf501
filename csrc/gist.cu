// Chunk routing-gist construction on the device (cache build hot op).
//
// Both kernels run one CTA per (chunk, layer): grid (C, L).  Layer l's K/V
// rows live in a token pool at pk + l * layer_stride (bf16, row stride
// `row_stride`); chunk c owns rows [start[c], start[c] + len[c]).  Results are
// written straight into the cache's per-layer gist tables at chunk slot
// dest[c] (identity when dest is null):
//   gk/gv/gn  [L, S, G, D] fp32   key gist, value gist, routing copy (gk / ||gk||)
//   count     [L, S]       int    occupied gist slots of the chunk
//
// mean:   gk = mean of the chunk's K rows, gv = mean of its V rows, one slot.
// kmeans: Lloyd in (optionally L2-normalised) key space with kmeans++ or sampled
//         initialisation driven by a precomputed random stream (the draws a
//         seeded CPU generator would make), farthest-point reseed of empty
//         clusters, then key / value gists as the means of the original rows
//         over the final assignment (occupied clusters only, in cluster order).
//         The chunk's keys are staged once in shared memory (bf16) when they
//         fit, so every Lloyd iteration reads on-chip data; each thread owns a
//         4-column slice of the feature dimension and accumulates all clusters
//         for it in registers (no atomics, no per-cluster passes).
// Semantics follow pra_torch/gists/strategies.py (kmeans_gists) and
// pra_torch/gists/common.py (assignment + paired means).
#include "common.cuh"

namespace pra {
namespace gist {

constexpr int NT = 256;
constexpr int NWARPS = NT / 32;
constexpr int MAXG = 8;
constexpr int MAXN = 1024;
constexpr float EPS = 1e-12f;

struct Quad {
  float x, y, z, w;
};

__device__ __forceinline__ Quad load_quad(const __nv_bfloat16* p) {
  const uint2 raw = *reinterpret_cast<const uint2*>(p);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
  return {a.x, a.y, b.x, b.y};
}

__device__ __forceinline__ int dest_of(const GistArgs& a, int c) { return a.dest ? a.dest[c] : c; }

// Sums v[0..G) (G <= MG) over the block in place (all threads see the totals).  red holds
// NWARPS * MAXG floats.
template <int MG = MAXG>
__device__ __forceinline__ void block_sum_vec(float* v, int G, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int q = 0; q < MG; ++q)
    if (q < G) v[q] = warp_sum(v[q]);
  __syncthreads();
  if (lane == 0) {
#pragma unroll
    for (int q = 0; q < MG; ++q)
      if (q < G) red[warp * MAXG + q] = v[q];
  }
  __syncthreads();
#pragma unroll
  for (int q = 0; q < MG; ++q) {
    if (q < G) {
      float s = 0.f;
      for (int w = 0; w < NWARPS; ++w) s += red[w * MAXG + q];
      v[q] = s;
    }
  }
  __syncthreads();
}

// Block argmax with the lowest index winning ties; returns the index (-1 if every value is -inf).
__device__ __forceinline__ int block_argmax(float v, int i, float* rv, int* ri) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (ov > v || (ov == v && oi >= 0 && (i < 0 || oi < i))) {
      v = ov;
      i = oi;
    }
  }
  __syncthreads();
  if (lane == 0) {
    rv[warp] = v;
    ri[warp] = i;
  }
  __syncthreads();
  float bv = rv[0];
  int bi = ri[0];
  for (int w = 1; w < NWARPS; ++w) {
    if (rv[w] > bv || (rv[w] == bv && ri[w] >= 0 && (bi < 0 || ri[w] < bi))) {
      bv = rv[w];
      bi = ri[w];
    }
  }
  __syncthreads();
  return bi;
}

// ---------------------------------------------------------------- mean
__global__ void __launch_bounds__(NT) mean_kernel(GistArgs a) {
  __shared__ float red[NWARPS * MAXG];
  const int c = blockIdx.x, layer = blockIdx.y;
  const int s = a.start[c], n = a.len[c];
  const int D = a.D, D4 = D / 4;
  const __nv_bfloat16* pk = a.pk + layer * a.layer_stride + (int64_t)s * a.row_stride;
  const __nv_bfloat16* pv = a.pv + layer * a.layer_stride + (int64_t)s * a.row_stride;
  const int64_t out = layer * a.out_layer_stride + (int64_t)dest_of(a, c) * a.G * D;
  const float inv_n = n > 0 ? 1.f / n : 0.f;
  float sq[1] = {0.f};
  for (int j = threadIdx.x; j < D4; j += NT) {
    Quad k{0.f, 0.f, 0.f, 0.f}, v{0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
    for (int i = 0; i < n; ++i) {
      const Quad kk = load_quad(pk + (int64_t)i * a.row_stride + 4 * j);
      const Quad vv = load_quad(pv + (int64_t)i * a.row_stride + 4 * j);
      k.x += kk.x; k.y += kk.y; k.z += kk.z; k.w += kk.w;
      v.x += vv.x; v.y += vv.y; v.z += vv.z; v.w += vv.w;
    }
    k = {k.x * inv_n, k.y * inv_n, k.z * inv_n, k.w * inv_n};
    v = {v.x * inv_n, v.y * inv_n, v.z * inv_n, v.w * inv_n};
    *reinterpret_cast<float4*>(a.gk + out + 4 * j) = make_float4(k.x, k.y, k.z, k.w);
    *reinterpret_cast<float4*>(a.gv + out + 4 * j) = make_float4(v.x, v.y, v.z, v.w);
    sq[0] += k.x * k.x + k.y * k.y + k.z * k.z + k.w * k.w;
  }
  block_sum_vec(sq, 1, red);
  const float inv = 1.f / fmaxf(sqrtf(sq[0]), EPS);
  for (int j = threadIdx.x; j < D4; j += NT) {
    const float4 k = *reinterpret_cast<const float4*>(a.gk + out + 4 * j);
    *reinterpret_cast<float4*>(a.gn + out + 4 * j) = make_float4(k.x * inv, k.y * inv, k.z * inv, k.w * inv);
  }
  if (threadIdx.x == 0) a.count[layer * a.count_layer_stride + dest_of(a, c)] = n > 0 ? 1 : 0;
}

// ---------------------------------------------------------------- kmeans
// MG: compile-time bound on the number of centres (>= a.G); the per-point loops run over it.
template <bool STAGED, int MG>
__global__ void __launch_bounds__(NT) kmeans_kernel(GistArgs a) {
  extern __shared__ __align__(16) float sm[];
  const int D = a.D, D4 = D / 4, nmax = a.nmax;
  float* centers = sm;                                    // [G, D]
  float* inv_norm = centers + a.G * D;                    // [nmax]
  float* dmin = inv_norm + nmax;                          // [nmax]
  float* dist = dmin + nmax;                              // [nmax, MAXG]
  int* assign = reinterpret_cast<int*>(dist + nmax * MAXG);  // [nmax]
  __nv_bfloat16* stage = reinterpret_cast<__nv_bfloat16*>(assign + nmax);  // [nmax, D] when STAGED
  __shared__ int members[MAXG];
  __shared__ int chosen[MAXG];
  __shared__ int slot_of[MAXG];
  __shared__ float red[NWARPS * MAXG];
  __shared__ float rv[NWARPS];
  __shared__ int ri[NWARPS];
  __shared__ int pick;
  __shared__ int stop;

  const int c = blockIdx.x, layer = blockIdx.y;
  const int s = a.start[c], n = min(a.len[c], nmax);
  const int G = min(a.G, n);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int dst = dest_of(a, c);
  const int64_t status_at = (int64_t)layer * a.C + c;
  const __nv_bfloat16* gkey = a.pk + layer * a.layer_stride + (int64_t)s * a.row_stride;
  const __nv_bfloat16* gval = a.pv + layer * a.layer_stride + (int64_t)s * a.row_stride;
  const int64_t out = layer * a.out_layer_stride + (int64_t)dst * a.G * D;
  if (threadIdx.x == 0) {
    if (a.status) a.status[status_at] = a.len[c] > nmax ? 2 : 0;
    a.count[layer * a.count_layer_stride + dst] = 0;
    if (a.iterations) a.iterations[status_at] = 0;
  }
  if (G == 0) return;

  // Keys: staged copy (row stride D) or the pool itself.
  const __nv_bfloat16* keys = gkey;
  int64_t kstride = a.row_stride;
  if constexpr (STAGED) {
    for (int e = threadIdx.x; e < n * D4; e += NT) {
      const int i = e / D4, j = e - i * D4;
      *reinterpret_cast<uint2*>(stage + (int64_t)i * D + 4 * j) =
          *reinterpret_cast<const uint2*>(gkey + (int64_t)i * a.row_stride + 4 * j);
    }
    keys = stage;
    kstride = D;
    __syncthreads();
  }
  // Row norms (working space is the normalised keys when requested).
  for (int i = warp; i < n; i += NWARPS) {
    float acc = 0.f;
    for (int j = lane; j < D4; j += 32) {
      const Quad k = load_quad(keys + (int64_t)i * kstride + 4 * j);
      acc += k.x * k.x + k.y * k.y + k.z * k.z + k.w * k.w;
    }
    acc = warp_sum(acc);
    if (lane == 0) inv_norm[i] = a.normalize ? 1.f / fmaxf(sqrtf(acc), EPS) : 1.f;
  }
  __syncthreads();

  auto set_center = [&](int q, int i) {
    for (int j = threadIdx.x; j < D4; j += NT) {
      const Quad k = load_quad(keys + (int64_t)i * kstride + 4 * j);
      const float sc = inv_norm[i];
      *reinterpret_cast<float4*>(centers + q * D + 4 * j) = make_float4(k.x * sc, k.y * sc, k.z * sc, k.w * sc);
    }
  };
  // Squared distances from every point to centres [0, nc): warp per point.
  auto distances = [&](int nc) {
    for (int i = warp; i < n; i += NWARPS) {
      float acc[MG];
#pragma unroll
      for (int q = 0; q < MG; ++q) acc[q] = 0.f;
      const float sc = inv_norm[i];
      for (int j = lane; j < D4; j += 32) {
        const Quad k = load_quad(keys + (int64_t)i * kstride + 4 * j);
        const float wx = k.x * sc, wy = k.y * sc, wz = k.z * sc, ww = k.w * sc;
#pragma unroll
        for (int q = 0; q < MG; ++q) {
          if (q < nc) {
            const float4 cc = *reinterpret_cast<const float4*>(centers + q * D + 4 * j);
            const float dx = wx - cc.x, dy = wy - cc.y, dz = wz - cc.z, dw = ww - cc.w;
            acc[q] += dx * dx + dy * dy + dz * dz + dw * dw;
          }
        }
      }
#pragma unroll
      for (int q = 0; q < MG; ++q) {
        if (q < nc) {
          const float v = warp_sum(acc[q]);
          if (lane == 0) dist[i * MAXG + q] = v;
        }
      }
    }
    __syncthreads();
  };
  // Nearest centre per point (first minimum), member counts, farthest point.
  auto assign_points = [&](bool want_far) {
    if (threadIdx.x < MAXG) members[threadIdx.x] = 0;
    __syncthreads();
    float far_v = -INFINITY;
    int far_i = -1;
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
      atomicAdd(&members[bi], 1);
      if (bd > far_v) {
        far_v = bd;
        far_i = i;
      }
    }
    if (want_far) {
      const int far = block_argmax(far_v, far_i, rv, ri);
      if (threadIdx.x == 0) pick = far < 0 ? 0 : far;
    }
    __syncthreads();
  };

  // ---- initialisation ----
  if (a.kmeanspp) {
    if (threadIdx.x == 0) chosen[0] = a.init_first[c];
    __syncthreads();
    set_center(0, chosen[0]);
    __syncthreads();
    for (int j = 1; j < G; ++j) {
      distances(j);
      float part[1] = {0.f};
      for (int i = threadIdx.x; i < n; i += NT) {
        float m = INFINITY;
        bool taken = false;
        for (int q = 0; q < j; ++q) {
          m = fminf(m, dist[i * MAXG + q]);
          taken |= (chosen[q] == i);
        }
        dmin[i] = taken ? 0.f : m;
        part[0] += dmin[i];
      }
      block_sum_vec<1>(part, 1, red);
      const float total = part[0];
      float best = -INFINITY;
      int best_i = -1;
      if (total > 0.f) {
        const float* e = a.exp_draws + a.exp_off[c] + (int64_t)(j - 1) * n;
        for (int i = threadIdx.x; i < n; i += NT) {
          const float q = (dmin[i] / total) / e[i];
          if (q > best) {
            best = q;
            best_i = i;
          }
        }
      }
      const int nxt0 = block_argmax(best, best_i, rv, ri);
      if (threadIdx.x == 0) {
        int nxt = nxt0;
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
      set_center(j, chosen[j]);
      __syncthreads();
    }
  } else {
    for (int q = 0; q < G; ++q) set_center(q, a.init_idx[a.init_first[c] + q]);
    __syncthreads();
  }

  // ---- Lloyd iterations ----
  int it = 0;
  for (it = 1; it <= a.max_iters; ++it) {
    distances(G);
    assign_points(true);
    if (threadIdx.x == 0 && !a.farthest && a.status) {
      for (int q = 0; q < G; ++q)
        if (members[q] == 0) a.status[status_at] = 1;
    }
    // new centres: each thread owns 4 columns and accumulates every cluster
    float shift[MG];
#pragma unroll
    for (int q = 0; q < MG; ++q) shift[q] = 0.f;
    for (int j = threadIdx.x; j < D4; j += NT) {
      float acc[MG][4];
#pragma unroll
      for (int q = 0; q < MG; ++q) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.f;
      for (int i = 0; i < n; ++i) {
        const Quad k = load_quad(keys + (int64_t)i * kstride + 4 * j);
        const float sc = inv_norm[i];
        const int qi = assign[i];
#pragma unroll
        for (int q = 0; q < MG; ++q) {
          if (q == qi) {
            acc[q][0] += k.x * sc;
            acc[q][1] += k.y * sc;
            acc[q][2] += k.z * sc;
            acc[q][3] += k.w * sc;
          }
        }
      }
      const Quad fk = load_quad(keys + (int64_t)pick * kstride + 4 * j);
      const float fsc = inv_norm[pick];
#pragma unroll
      for (int q = 0; q < MG; ++q) {
        if (q < G) {
          float4 nv;
          if (members[q] == 0) {
            nv = make_float4(fk.x * fsc, fk.y * fsc, fk.z * fsc, fk.w * fsc);
          } else {
            const float m = (float)members[q];
            nv = make_float4(acc[q][0] / m, acc[q][1] / m, acc[q][2] / m, acc[q][3] / m);
          }
          float4* cp = reinterpret_cast<float4*>(centers + q * D + 4 * j);
          const float4 old = *cp;
          const float dx = nv.x - old.x, dy = nv.y - old.y, dz = nv.z - old.z, dw = nv.w - old.w;
          shift[q] += dx * dx + dy * dy + dz * dz + dw * dw;
          *cp = nv;
        }
      }
    }
    block_sum_vec<MG>(shift, G, red);
    if (threadIdx.x == 0) {
      float m = 0.f;
      for (int q = 0; q < G; ++q) m = fmaxf(m, sqrtf(shift[q]));
      stop = m <= a.tol;
    }
    __syncthreads();
    if (stop) break;
  }
  if (it > a.max_iters) it = a.max_iters;

  // ---- final assignment and paired means over the original rows ----
  distances(G);
  assign_points(false);
  if (threadIdx.x == 0) {
    int slot = 0;
    for (int q = 0; q < G; ++q) {
      slot_of[q] = members[q] ? slot : -1;
      if (members[q] && a.occupancy) a.occupancy[status_at * a.G + slot] = members[q];
      if (members[q]) ++slot;
    }
    a.count[layer * a.count_layer_stride + dst] = slot;
    if (a.iterations) a.iterations[status_at] = it;
  }
  __syncthreads();
  // keys (raw, not normalised) then values; each thread keeps its columns for the norms
  float norm1[MG], norm2[MG];
#pragma unroll
  for (int q = 0; q < MG; ++q) norm1[q] = norm2[q] = 0.f;
  for (int pass = 0; pass < 2; ++pass) {
    const __nv_bfloat16* src = pass == 0 ? keys : gval;
    const int64_t stride = pass == 0 ? kstride : a.row_stride;
    float* dstp = pass == 0 ? a.gk : a.gv;
    for (int j = threadIdx.x; j < D4; j += NT) {
      float acc[MG][4];
#pragma unroll
      for (int q = 0; q < MG; ++q) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.f;
      for (int i = 0; i < n; ++i) {
        const Quad k = load_quad(src + (int64_t)i * stride + 4 * j);
        const int qi = assign[i];
#pragma unroll
        for (int q = 0; q < MG; ++q) {
          if (q == qi) {
            acc[q][0] += k.x;
            acc[q][1] += k.y;
            acc[q][2] += k.z;
            acc[q][3] += k.w;
          }
        }
      }
#pragma unroll
      for (int q = 0; q < MG; ++q) {
        if (q < G && slot_of[q] >= 0) {
          const float m = (float)members[q];
          const float4 v = make_float4(acc[q][0] / m, acc[q][1] / m, acc[q][2] / m, acc[q][3] / m);
          *reinterpret_cast<float4*>(dstp + out + (int64_t)slot_of[q] * D + 4 * j) = v;
          if (pass == 0) norm1[q] += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
      }
    }
  }
  // gk is L2-normalised when the working space is; gn = gk / ||gk|| is the routing copy.
  block_sum_vec<MG>(norm1, G, red);
  for (int j = threadIdx.x; j < D4; j += NT) {
#pragma unroll
    for (int q = 0; q < MG; ++q) {
      if (q < G && slot_of[q] >= 0) {
        float4* p = reinterpret_cast<float4*>(a.gk + out + (int64_t)slot_of[q] * D + 4 * j);
        float4 v = *p;
        if (a.normalize) {
          const float inv = 1.f / fmaxf(sqrtf(norm1[q]), EPS);
          v = make_float4(v.x * inv, v.y * inv, v.z * inv, v.w * inv);
          *p = v;
        }
        norm2[q] += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      }
    }
  }
  block_sum_vec<MG>(norm2, G, red);
  for (int j = threadIdx.x; j < D4; j += NT) {
#pragma unroll
    for (int q = 0; q < MG; ++q) {
      if (q < G && slot_of[q] >= 0) {
        const int64_t o = out + (int64_t)slot_of[q] * D + 4 * j;
        const float4 v = *reinterpret_cast<const float4*>(a.gk + o);
        const float inv = 1.f / fmaxf(sqrtf(norm2[q]), EPS);
        *reinterpret_cast<float4*>(a.gn + o) = make_float4(v.x * inv, v.y * inv, v.z * inv, v.w * inv);
      }
    }
  }
}

size_t kmeans_fixed_smem(const GistArgs& a) {
  return (size_t)a.G * a.D * sizeof(float) + (size_t)a.nmax * (2 * sizeof(float) + MAXG * sizeof(float) + sizeof(int));
}

}  // namespace gist
}  // namespace pra

static cudaError_t check_gist_args(const GistArgs& a) {
  if (a.D % 4 != 0 || a.row_stride % 4 != 0 || a.layer_stride % 4 != 0) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(a.pk) | reinterpret_cast<uintptr_t>(a.pv)) & 7) return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(a.gk) & 15 || reinterpret_cast<uintptr_t>(a.gv) & 15 ||
      reinterpret_cast<uintptr_t>(a.gn) & 15)
    return cudaErrorInvalidValue;
  return cudaSuccess;
}

cudaError_t pra_gist_mean(const GistArgs& a, int layers, cudaStream_t st) {
  if (a.C == 0 || layers == 0) return cudaSuccess;
  PRA_RETURN_IF_ERROR(check_gist_args(a));
  pra::gist::mean_kernel<<<dim3(a.C, layers), pra::gist::NT, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t pra_gist_kmeans(const GistArgs& a, int layers, cudaStream_t st) {
  using namespace pra::gist;
  if (a.C == 0 || layers == 0) return cudaSuccess;
  if (a.G < 1 || a.G > MAXG || a.nmax < 1 || a.nmax > MAXN) return cudaErrorInvalidValue;
  PRA_RETURN_IF_ERROR(check_gist_args(a));
  const size_t fixed = kmeans_fixed_smem(a);
  const size_t staged = fixed + (size_t)a.nmax * a.D * sizeof(__nv_bfloat16);
  // Stage when two CTAs still fit on one SM (2 x 110 KB of the 228 KB per SM).
  const bool stage = staged <= 110 * 1024;
  if (!stage && fixed > 200 * 1024) return cudaErrorInvalidValue;
  const size_t smem = stage ? staged : fixed;
  auto go = [&](auto kernel) -> cudaError_t {
    PRA_RETURN_IF_ERROR(pra::set_max_dynamic_smem(reinterpret_cast<const void*>(kernel), (int)smem));
    kernel<<<dim3(a.C, layers), NT, smem, st>>>(a);
    return cudaSuccess;
  };
  if (a.G <= 2) PRA_RETURN_IF_ERROR(stage ? go(kmeans_kernel<true, 2>) : go(kmeans_kernel<false, 2>));
  else if (a.G <= 4) PRA_RETURN_IF_ERROR(stage ? go(kmeans_kernel<true, 4>) : go(kmeans_kernel<false, 4>));
  else PRA_RETURN_IF_ERROR(stage ? go(kmeans_kernel<true, MAXG>) : go(kmeans_kernel<false, MAXG>));
  return cudaGetLastError();
}
