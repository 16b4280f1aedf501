// Fused row-local routing + selection + materialisation plan (one CTA per query row).
//
// For query row b, over the chunks of its own namespace only:
//   1. cosine score of the normalised query against every L2-normalised gist,
//      reduced over the chunk's gist set (max / mean / logsumexp), keeping the
//      winning gist index and score;
//   2. URI scores = the same reduction over each URI's chunk scores;
//   3. hierarchical selection: top URIs ordered (-score, uri rank), then inside
//      each the top chunks ordered (-score, chunk-id rank);
//   4. optional full-reference expansion, score threshold, greedy whole-chunk
//      budget in (-score, uri, chunk-id) order, then materialisation order
//      (uri, token_start, chunk-id) with overlap already covered by the same URI
//      stripped;
//   5. the memory key list for the attention kernel: pool row indices
//      (mem_idx[b, :mem_len[b]]) plus a per-selection trace record.
// No host synchronisation is needed: every tensor stays on the device.
#include "common.cuh"

namespace pra {
namespace route {

constexpr int NT = 256;
constexpr int MAX_ROW_CHUNKS = 8192;
constexpr int MAX_ROW_REFS = 2048;
constexpr int MAX_SEL = 256;
constexpr float EPS = 1e-12f;

__device__ __forceinline__ float reduce_set(const float* v, int n, int mode) {
  if (n <= 0) return -INFINITY;
  if (mode == 0) {
    float m = -INFINITY;
    for (int i = 0; i < n; ++i) m = fmaxf(m, v[i]);
    return m;
  }
  if (mode == 1) {
    float s = 0.f;
    for (int i = 0; i < n; ++i) s += v[i];
    return s / n;
  }
  float m = -INFINITY;
  for (int i = 0; i < n; ++i) m = fmaxf(m, v[i]);
  if (m == -INFINITY) return -INFINITY;
  float s = 0.f;
  for (int i = 0; i < n; ++i) s += __expf(v[i] - m);
  return m + __logf(s);
}

// Is (s1, r1) ranked before (s2, r2) under (-score, rank)?
__device__ __forceinline__ bool before(float s1, int r1, float s2, int r2) {
  return s1 > s2 || (s1 == s2 && r1 < r2);
}

__global__ void __launch_bounds__(NT) route_kernel(RouteParams p) {
  extern __shared__ __align__(16) float smem[];
  float* qn = smem;                                   // [D]
  float* cscore = qn + p.D;                           // [MAX_ROW_CHUNKS]
  float* wscore = cscore + MAX_ROW_CHUNKS;            // [MAX_ROW_CHUNKS]
  int* widx = reinterpret_cast<int*>(wscore + MAX_ROW_CHUNKS);  // [MAX_ROW_CHUNKS]
  float* rscore = reinterpret_cast<float*>(widx + MAX_ROW_CHUNKS);  // [MAX_ROW_REFS]
  __shared__ float scratch[32];
  __shared__ int sel_chunk[MAX_SEL], sel_rrank[MAX_SEL], sel_crank[MAX_SEL], sel_keep[MAX_SEL];
  __shared__ float sel_rscore[MAX_SEL], sel_cscore[MAX_SEL];
  __shared__ int top_ref[64];
  __shared__ int n_sel;

  const int b = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = NT / 32;
  const int c0 = p.row_pos_off[b], c1 = p.row_pos_off[b + 1];
  const int r0 = p.row_ref_off[b], r1 = p.row_ref_off[b + 1];
  const int nc = c1 - c0, nr = r1 - r0;
  if (threadIdx.x == 0) {
    p.mem_len[b] = 0;
    p.sel_count[b] = 0;
    p.status[b] = (nc > MAX_ROW_CHUNKS || nr > MAX_ROW_REFS) ? 1 : 0;
  }
  if (nc <= 0 || nr <= 0 || nc > MAX_ROW_CHUNKS || nr > MAX_ROW_REFS || p.k_ref <= 0 || p.k_chunk <= 0) return;

  // 1. normalised query
  float sq = 0.f;
  for (int d = threadIdx.x; d < p.D; d += NT) {
    const float v = __bfloat162float(p.query[(int64_t)b * p.query_stride + d]);
    qn[d] = v;
    sq += v * v;
  }
  const float inv = 1.f / fmaxf(sqrtf(block_sum(sq, scratch)), EPS);
  for (int d = threadIdx.x; d < p.D; d += NT) qn[d] *= inv;
  __syncthreads();

  // 2. chunk scores (warp per chunk)
  for (int i = warp; i < nc; i += nwarps) {
    const int c = p.pos_chunk[c0 + i];
    const int g_n = p.gist_count[c];
    float sc[8];
    for (int g = 0; g < p.G; ++g) {
      float acc = 0.f;
      if (g < g_n) {
        const float* gv = p.gists + ((int64_t)c * p.G + g) * p.D;
        for (int d = lane; d < p.D; d += 32) acc += qn[d] * gv[d];
        acc = warp_sum(acc);
      }
      sc[g] = acc;
    }
    if (lane == 0) {
      int wi = 0;
      float ws = -INFINITY;
      for (int g = 0; g < g_n; ++g)
        if (sc[g] > ws) {
          ws = sc[g];
          wi = g;
        }
      cscore[i] = p.gist_agg == 0 ? ws : reduce_set(sc, g_n, p.gist_agg);
      wscore[i] = ws;
      widx[i] = wi;
    }
  }
  __syncthreads();
  // 3. URI scores (thread per ref; chunks of a ref are contiguous)
  for (int r = threadIdx.x; r < nr; r += NT) {
    const int a = p.ref_pos_off[r0 + r] - c0, z = p.ref_pos_off[r0 + r + 1] - c0;
    rscore[r] = reduce_set(cscore + a, z - a, p.ref_agg);
  }
  __syncthreads();

  // 4. selection (single thread: k_ref * k_chunk items)
  if (threadIdx.x == 0) {
    const int kr = min(min(p.k_ref, nr), 64);
    for (int j = 0; j < kr; ++j) {
      int best = -1;
      for (int r = 0; r < nr; ++r) {
        bool used = false;
        for (int q = 0; q < j; ++q) used |= (top_ref[q] == r);
        if (used) continue;
        if (best < 0 || before(rscore[r], r, rscore[best], best)) best = r;
      }
      top_ref[j] = best;
    }
    int count = 0;
    for (int j = 0; j < kr && count < MAX_SEL; ++j) {
      const int r = top_ref[j];
      const int a = p.ref_pos_off[r0 + r] - c0, z = p.ref_pos_off[r0 + r + 1] - c0;
      if (p.full_reference) {
        for (int i = a; i < z && count < MAX_SEL; ++i) {
          sel_chunk[count] = i;
          sel_rrank[count] = j + 1;
          sel_crank[count] = i - a + 1;
          sel_rscore[count] = rscore[r];
          sel_cscore[count] = -INFINITY;  // filled below from the first routed hit
          ++count;
        }
        // the expanded chunks all carry the score of the URI's best routed chunk
        int first = -1;
        for (int i = a; i < z; ++i)
          if (first < 0 || before(cscore[i], p.pos_rank[c0 + i], cscore[first], p.pos_rank[c0 + first])) first = i;
        for (int q = count - (z - a); q < count; ++q) sel_cscore[q] = cscore[first];
        continue;
      }
      const int kc = min(p.k_chunk, z - a);
      for (int t = 0; t < kc && count < MAX_SEL; ++t) {
        int best = -1;
        for (int i = a; i < z; ++i) {
          bool used = false;
          for (int q = count - t; q < count; ++q) used |= (sel_chunk[q] == i);
          if (used) continue;
          if (best < 0 || before(cscore[i], p.pos_rank[c0 + i], cscore[best], p.pos_rank[c0 + best])) best = i;
        }
        sel_chunk[count] = best;
        sel_rrank[count] = j + 1;
        sel_crank[count] = t + 1;
        sel_rscore[count] = rscore[r];
        sel_cscore[count] = cscore[best];
        ++count;
      }
    }
    // threshold
    for (int q = 0; q < count; ++q) sel_keep[q] = sel_cscore[q] >= p.threshold ? 1 : 0;
    // greedy budget in (-score, uri rank, chunk rank) order
    int remaining = p.budget_rows ? p.budget_rows[b] : p.budget;
    for (int pass = 0; pass < count; ++pass) {
      int best = -1;
      for (int q = 0; q < count; ++q) {
        if (sel_keep[q] != 1) continue;
        if (best < 0) {
          best = q;
          continue;
        }
        const int rq = p.pos_ref[c0 + sel_chunk[q]], rb = p.pos_ref[c0 + sel_chunk[best]];
        const bool better = sel_cscore[q] > sel_cscore[best] ||
                            (sel_cscore[q] == sel_cscore[best] &&
                             (rq < rb || (rq == rb && p.pos_rank[c0 + sel_chunk[q]] < p.pos_rank[c0 + sel_chunk[best]])));
        if (better) best = q;
      }
      if (best < 0) break;
      const int cost = p.gist_only ? 1 : p.chunk_len[c0 + sel_chunk[best]];
      if (cost <= remaining) {
        remaining -= cost;
        sel_keep[best] = 2;  // retained
      } else {
        sel_keep[best] = 3;  // rejected by the budget
      }
    }
    // trace records (retained, in selection order)
    int kept = 0;
    for (int q = 0; q < count; ++q) {
      if (sel_keep[q] != 2) continue;
      const int c = p.pos_chunk[c0 + sel_chunk[q]];
      const int64_t o = (int64_t)b * p.max_sel + kept;
      if (kept < p.max_sel) {
        p.sel_chunk[o] = c;
        p.sel_ref_rank[o] = sel_rrank[q];
        p.sel_chunk_rank[o] = sel_crank[q];
        p.sel_ref_score[o] = sel_rscore[q];
        p.sel_chunk_score[o] = sel_cscore[q];
        p.sel_win_index[o] = widx[sel_chunk[q]];
        p.sel_win_score[o] = wscore[sel_chunk[q]];
      }
      ++kept;
    }
    p.sel_count[b] = min(kept, p.max_sel);
    p.routing_candidates[b] = count;
    // materialisation order: (uri rank, token_start, chunk rank); strip covered overlap
    int written = 0, duplicates = 0;
    int last_ref = -1, covered = 0;
    for (int pass = 0; pass < count; ++pass) {
      int best = -1;
      for (int q = 0; q < count; ++q) {
        if (sel_keep[q] != 2) continue;
        if (best < 0) {
          best = q;
          continue;
        }
        const int pq = c0 + sel_chunk[q], pb = c0 + sel_chunk[best];
        const int cq = p.pos_chunk[pq], cb = p.pos_chunk[pb];
        const int rq = p.pos_ref[pq], rb = p.pos_ref[pb];
        const bool earlier = rq < rb || (rq == rb && (p.chunk_start[cq] < p.chunk_start[cb] ||
                                                      (p.chunk_start[cq] == p.chunk_start[cb] &&
                                                       p.pos_rank[pq] < p.pos_rank[pb])));
        if (earlier) best = q;
      }
      if (best < 0) break;
      sel_keep[best] = 4;
      const int c = p.pos_chunk[c0 + sel_chunk[best]];
      if (p.gist_only) {
        if (written < p.max_mem) p.mem_idx[(int64_t)b * p.max_mem + written] = c * p.G + widx[sel_chunk[best]];
        ++written;
        continue;
      }
      const int ref = p.pos_ref[c0 + sel_chunk[best]];
      const int tstart = p.chunk_start[c], n = p.chunk_len[c];
      int strip = 0;
      const int end = (ref == last_ref) ? covered : tstart;
      if (ref != last_ref) covered = tstart;
      strip = min(max(end - tstart, 0), n);
      duplicates += strip;
      if (!p.deduplicate) strip = 0;
      for (int t = strip; t < n; ++t) {
        if (written < p.max_mem) p.mem_idx[(int64_t)b * p.max_mem + written] = p.chunk_pool_row[c] + t;
        ++written;
      }
      covered = max(end, tstart + n);
      last_ref = ref;
    }
    p.mem_len[b] = min(written, p.max_mem);
    p.duplicate_tokens[b] = duplicates;
    if (written > p.max_mem) p.status[b] = 2;
  }
}

}  // namespace route
}  // namespace pra

cudaError_t pra_route(const RouteParams& p, cudaStream_t st) {
  using namespace pra::route;
  if (p.B == 0) return cudaSuccess;
  if (p.G > 8) return cudaErrorInvalidValue;
  const size_t smem = (size_t)p.D * sizeof(float) + (size_t)MAX_ROW_CHUNKS * (2 * sizeof(float) + sizeof(int)) +
                      (size_t)MAX_ROW_REFS * sizeof(float);
  PRA_RETURN_IF_ERROR(cudaFuncSetAttribute(route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  route_kernel<<<p.B, NT, smem, st>>>(p);
  return cudaGetLastError();
}
