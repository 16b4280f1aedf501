// Fused row-local routing + selection + materialisation plan (one CTA per query row).
//
// For query row b, over the chunks of its own namespace only:
//   1. cosine score of the normalised query against every L2-normalised gist,
//      reduced over the chunk's gist set (max / mean / logsumexp), keeping the
//      winning gist index and score;
//   2. URI scores = the same reduction over each URI's chunk scores;
//   3. hierarchical selection: top URIs ordered (-score, uri rank), then inside
//      each the top chunks ordered (-score, chunk-id rank); or (global_chunks) every
//      chunk ranked by (-score, uri rank, chunk-id rank) and taken greedily while its
//      URI has fewer than k_chunk picks and the distinct URIs stay within k_ref;
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
constexpr int MAX_SEL = 256;  // must not exceed NT (one trace item per thread)
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

// Exclusive prefix sum over the block of one int per thread (NT threads); returns the
// thread's offset and writes the total to *total.
__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_tot, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  __syncthreads();
  if (lane == 31) warp_tot[warp] = x;
  __syncthreads();
  int base = 0, all = 0;
  for (int w = 0; w < NT / 32; ++w) {
    if (w < warp) base += warp_tot[w];
    all += warp_tot[w];
  }
  if (threadIdx.x == 0) *total = all;
  __syncthreads();
  return base + x - v;
}

__global__ void __launch_bounds__(NT) route_kernel(RouteParams p) {
  extern __shared__ __align__(16) float smem[];
  float* qn = smem;                                   // [D]
  float* cscore = qn + p.D;                           // [MAX_ROW_CHUNKS]
  float* wscore = cscore + MAX_ROW_CHUNKS;            // [MAX_ROW_CHUNKS]
  int* widx = reinterpret_cast<int*>(wscore + MAX_ROW_CHUNKS);  // [MAX_ROW_CHUNKS]
  int* crank = widx + MAX_ROW_CHUNKS;                 // [MAX_ROW_CHUNKS] lexical chunk rank (pos_rank)
  float* rscore = reinterpret_cast<float*>(crank + MAX_ROW_CHUNKS);  // [MAX_ROW_REFS]
  int* ref_taken = reinterpret_cast<int*>(rscore + MAX_ROW_REFS);    // [MAX_ROW_REFS]
  int* cref = ref_taken + MAX_ROW_REFS;                              // [MAX_ROW_CHUNKS] global mode: URI of a chunk
  int* rslot = cref + MAX_ROW_CHUNKS;                                // [MAX_ROW_REFS] global mode: URI pick order
  __shared__ float scratch[32];
  __shared__ int warp_tot[NT / 32];
  __shared__ float red_v[NT / 32];
  __shared__ int red_i[NT / 32];
  // per-selection item state (selection order)
  __shared__ int it_pos[MAX_SEL], it_rrank[MAX_SEL], it_crank[MAX_SEL], it_keep[MAX_SEL];
  __shared__ int it_ref[MAX_SEL], it_lex[MAX_SEL], it_chunk[MAX_SEL], it_start[MAX_SEL], it_len[MAX_SEL];
  __shared__ float it_rscore[MAX_SEL], it_cscore[MAX_SEL];
  __shared__ int by_budget[MAX_SEL], by_place[MAX_SEL], place_off[MAX_SEL], place_strip[MAX_SEL];
  __shared__ int top_ref[64], ref_base[65], ref_first[64];
  __shared__ int n_sel, n_kept, n_written, n_total;

  const int b = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = NT / 32;
  const int c0 = p.row_pos_off[b], c1 = p.row_pos_off[b + 1];
  const int r0 = p.row_ref_off[b], r1 = p.row_ref_off[b + 1];
  const int nc = c1 - c0, nr = r1 - r0;
  // unused trace slots read as "no selection"
  for (int i = threadIdx.x; i < p.max_sel; i += NT) {
    const int64_t o = (int64_t)b * p.max_sel + i;
    p.sel_chunk[o] = p.sel_ref_rank[o] = p.sel_chunk_rank[o] = p.sel_win_index[o] = -1;
    p.sel_ref_score[o] = p.sel_chunk_score[o] = p.sel_win_score[o] = 0.f;
  }
  if (threadIdx.x == 0) {
    p.mem_len[b] = 0;
    p.sel_count[b] = 0;
    p.routing_candidates[b] = 0;
    p.duplicate_tokens[b] = 0;
    p.status[b] = (nc > MAX_ROW_CHUNKS || nr > MAX_ROW_REFS) ? 1 : 0;
  }
  if (nc <= 0 || nr <= 0 || nc > MAX_ROW_CHUNKS || nr > MAX_ROW_REFS || p.k_ref <= 0 || p.k_chunk <= 0) return;

  // 1. normalised query
  const __nv_bfloat16* qrow =
      p.query + (int64_t)b * p.query_stride + (p.query_row ? (int64_t)p.query_row[b] * p.query_row_stride : 0);
  float sq = 0.f;
  for (int d = threadIdx.x; d < p.D; d += NT) {
    const float v = __bfloat162float(qrow[d]);
    qn[d] = v;
    sq += v * v;
  }
  const float inv = 1.f / fmaxf(sqrtf(block_sum(sq, scratch)), EPS);
  for (int d = threadIdx.x; d < p.D; d += NT) qn[d] *= inv;
  __syncthreads();

  // 2. chunk scores (warp per chunk, float4 gist reads)
  const int D4 = p.D / 4;
  for (int i = warp; i < nc; i += nwarps) {
    const int c = p.pos_chunk[c0 + i];
    const int g_n = p.gist_count[c];
    float sc[8];
    for (int g = 0; g < p.G; ++g) {
      float acc = 0.f;
      if (g < g_n) {
        const float4* gv = reinterpret_cast<const float4*>(p.gists + ((int64_t)c * p.G + g) * p.D);
        for (int j = lane; j < D4; j += 32) {
          const float4 x = gv[j];
          acc += qn[4 * j] * x.x + qn[4 * j + 1] * x.y + qn[4 * j + 2] * x.z + qn[4 * j + 3] * x.w;
        }
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
      crank[i] = p.pos_rank[c0 + i];
    }
  }
  __syncthreads();
  // 3. URI scores (thread per ref; chunks of a ref are contiguous)
  for (int r = threadIdx.x; r < nr; r += NT) {
    const int a = p.ref_pos_off[r0 + r] - c0, z = p.ref_pos_off[r0 + r + 1] - c0;
    rscore[r] = reduce_set(cscore + a, z - a, p.ref_agg);
    ref_taken[r] = 0;
  }
  __syncthreads();

  if (p.global_chunks) {
    // 4g. global chunk ranking (-score, uri rank, chunk rank) taken greedily: a chunk is
    // eligible while its URI has fewer than k_chunk picks and the URI is already picked or
    // fewer than k_ref URIs are (the constraints only tighten, so the greedy over the global
    // order is repeated block argmax over the eligible chunks)
    for (int r = threadIdx.x; r < nr; r += NT) {
      const int a = p.ref_pos_off[r0 + r] - c0, z = p.ref_pos_off[r0 + r + 1] - c0;
      for (int i = a; i < z; ++i) cref[i] = r;
      ref_taken[r] = 0;  // picks of URI r
      rslot[r] = -1;
    }
    __shared__ int n_refs_picked;
    if (threadIdx.x == 0) {
      n_refs_picked = 0;
      n_sel = 0;
    }
    __syncthreads();
    const int limit = min(min(p.k_ref, 64) * p.k_chunk, MAX_SEL);
    constexpr int kTaken = 1 << 30;
    for (int q = 0; q < limit; ++q) {
      float bv = -INFINITY;
      int bi = -1, br = 0, bc = 0;
      for (int i = threadIdx.x; i < nc; i += NT) {
        const int r = cref[i];
        if (r & kTaken) continue;
        if (ref_taken[r] >= p.k_chunk || (rslot[r] < 0 && n_refs_picked >= p.k_ref)) continue;
        const float v = cscore[i];
        if (bi < 0 || v > bv || (v == bv && (r < br || (r == br && crank[i] < bc)))) {
          bv = v;
          bi = i;
          br = r;
          bc = crank[i];
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        const int orr = __shfl_xor_sync(0xffffffffu, br, o);
        const int oc = __shfl_xor_sync(0xffffffffu, bc, o);
        if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && (orr < br || (orr == br && oc < bc))))) {
          bv = ov;
          bi = oi;
          br = orr;
          bc = oc;
        }
      }
      if (lane == 0) {
        red_v[warp] = bv;
        red_i[warp] = bi;
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        int i = -1;
        float v = -INFINITY;
        for (int w = 0; w < nwarps; ++w) {
          const int wi = red_i[w];
          if (wi < 0) continue;
          const float wv = red_v[w];
          if (i < 0 || wv > v ||
              (wv == v && (cref[wi] < cref[i] || (cref[wi] == cref[i] && crank[wi] < crank[i])))) {
            v = wv;
            i = wi;
          }
        }
        if (i >= 0) {
          const int r = cref[i];
          if (rslot[r] < 0) rslot[r] = n_refs_picked++;
          ref_taken[r] += 1;
          it_pos[q] = i;
          it_rrank[q] = rslot[r] + 1;
          it_crank[q] = ref_taken[r];
          it_rscore[q] = rscore[r];
          it_cscore[q] = cscore[i];
          cref[i] = r | kTaken;
          n_sel = q + 1;
        }
        red_i[0] = i;  // broadcast "found"
      }
      __syncthreads();
      const bool found = red_i[0] >= 0;
      __syncthreads();
      if (!found) break;
    }
  } else {
    // 4a. top URIs under (-score, uri rank): rank counting when every ref has its own
    // thread, otherwise repeated block argmax
    const int kr = min(min(p.k_ref, nr), 64);
    if (nr <= NT) {
      if (threadIdx.x < nr) {
        const int r = threadIdx.x;
        int rank = 0;
        for (int o = 0; o < nr; ++o) rank += before(rscore[o], o, rscore[r], r) ? 1 : 0;
        if (rank < kr) top_ref[rank] = r;
      }
    } else {
      for (int j = 0; j < kr; ++j) {
        float bv = -INFINITY;
        int bi = -1;
        for (int r = threadIdx.x; r < nr; r += NT)
          if (!ref_taken[r] && (bi < 0 || before(rscore[r], r, bv, bi))) {
            bv = rscore[r];
            bi = r;
          }
  #pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (oi >= 0 && (bi < 0 || before(ov, oi, bv, bi))) {
            bv = ov;
            bi = oi;
          }
        }
        if (lane == 0) {
          red_v[warp] = bv;
          red_i[warp] = bi;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
          float v = red_v[0];
          int i = red_i[0];
          for (int w = 1; w < nwarps; ++w)
            if (red_i[w] >= 0 && (i < 0 || before(red_v[w], red_i[w], v, i))) {
              v = red_v[w];
              i = red_i[w];
            }
          top_ref[j] = i;
          ref_taken[i] = 1;
        }
        __syncthreads();
      }
    }
    __syncthreads();
    // 4b. items per selected URI, their offsets, and each URI's best chunk
    if (threadIdx.x == 0) {
      int acc = 0;
      for (int j = 0; j < kr; ++j) {
        const int r = top_ref[j];
        const int len = p.ref_pos_off[r0 + r + 1] - p.ref_pos_off[r0 + r];
        ref_base[j] = acc;
        acc += p.full_reference ? len : min(p.k_chunk, len);
      }
      ref_base[kr] = acc;
      n_sel = min(acc, MAX_SEL);
    }
    __syncthreads();
    for (int j = warp; j < kr; j += nwarps) {
      const int r = top_ref[j];
      const int a = p.ref_pos_off[r0 + r] - c0, z = p.ref_pos_off[r0 + r + 1] - c0;
      if (p.full_reference) {
        // best chunk of the URI (its score is carried by every expanded chunk)
        float bv = -INFINITY;
        int bi = -1, br = 0;
        for (int i = a + lane; i < z; i += 32)
          if (bi < 0 || before(cscore[i], crank[i], bv, br)) {
            bv = cscore[i];
            bi = i;
            br = crank[i];
          }
  #pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          const int orr = __shfl_xor_sync(0xffffffffu, br, o);
          if (oi >= 0 && (bi < 0 || before(ov, orr, bv, br))) {
            bv = ov;
            bi = oi;
            br = orr;
          }
        }
        if (lane == 0) ref_first[j] = bi;
        __syncwarp();
        for (int i = a + lane; i < z; i += 32) {
          const int q = ref_base[j] + (i - a);
          if (q >= MAX_SEL) continue;
          it_pos[q] = i;
          it_rrank[q] = j + 1;
          it_crank[q] = i - a + 1;
          it_rscore[q] = rscore[r];
          it_cscore[q] = cscore[bi];
        }
      } else {
        const int kc = min(p.k_chunk, z - a);
        for (int i = a + lane; i < z; i += 32) {
          int rank = 0;
          for (int o = a; o < z; ++o) rank += before(cscore[o], crank[o], cscore[i], crank[i]) ? 1 : 0;
          const int q = ref_base[j] + rank;
          if (rank < kc && q < MAX_SEL) {
            it_pos[q] = i;
            it_rrank[q] = j + 1;
            it_crank[q] = rank + 1;
            it_rscore[q] = rscore[r];
            it_cscore[q] = cscore[i];
          }
        }
      }
    }
    __syncthreads();
  }
  const int count = n_sel;
  // item attributes (threshold, namespace order, source span)
  for (int q = threadIdx.x; q < count; q += NT) {
    const int pos = c0 + it_pos[q];
    const int c = p.pos_chunk[pos];
    it_keep[q] = it_cscore[q] >= p.threshold ? 1 : 0;
    it_ref[q] = p.pos_ref[pos];
    it_lex[q] = crank[it_pos[q]];
    it_chunk[q] = c;
    it_start[q] = p.chunk_start[c];
    it_len[q] = p.chunk_len[c];
  }
  __syncthreads();
  // 4c. budget order (-score, uri, chunk rank, selection index) and materialisation order
  // (uri, token start, chunk rank, selection index) among the threshold survivors
  for (int q = threadIdx.x; q < count; q += NT) {
    if (!it_keep[q]) continue;
    int rb = 0, rp = 0;
    for (int o = 0; o < count; ++o) {
      if (!it_keep[o] || o == q) continue;
      const bool ob = it_cscore[o] > it_cscore[q] ||
                      (it_cscore[o] == it_cscore[q] &&
                       (it_ref[o] < it_ref[q] ||
                        (it_ref[o] == it_ref[q] && (it_lex[o] < it_lex[q] || (it_lex[o] == it_lex[q] && o < q)))));
      const bool op = it_ref[o] < it_ref[q] ||
                      (it_ref[o] == it_ref[q] &&
                       (it_start[o] < it_start[q] ||
                        (it_start[o] == it_start[q] && (it_lex[o] < it_lex[q] || (it_lex[o] == it_lex[q] && o < q)))));
      rb += ob ? 1 : 0;
      rp += op ? 1 : 0;
    }
    by_budget[rb] = q;
    by_place[rp] = q;
  }
  __syncthreads();
  // 4d. greedy whole-chunk budget (sequential by definition), then placement offsets
  if (threadIdx.x == 0) {
    int survivors = 0;
    for (int q = 0; q < count; ++q) survivors += it_keep[q];
    int remaining = p.budget_rows ? p.budget_rows[b] : p.budget;
    for (int k = 0; k < survivors; ++k) {
      const int q = by_budget[k];
      const int cost = p.gist_only ? 1 : it_len[q];
      if (cost <= remaining) {
        remaining -= cost;
        it_keep[q] = 2;  // retained
      } else {
        it_keep[q] = 3;  // rejected by the budget
      }
    }
    // materialisation walk over retained items: overlap already covered by the same URI is stripped
    int written = 0, duplicates = 0, last_ref = -1, covered = 0, placed = 0;
    for (int k = 0; k < survivors; ++k) {
      const int q = by_place[k];
      if (it_keep[q] != 2) continue;
      by_place[placed++] = q;
      if (p.gist_only) {
        place_off[q] = written;
        place_strip[q] = 0;
        ++written;
        continue;
      }
      const int tstart = it_start[q], n = it_len[q];
      const int end = (it_ref[q] == last_ref) ? covered : tstart;
      if (it_ref[q] != last_ref) covered = tstart;
      int strip = min(max(end - tstart, 0), n);
      duplicates += strip;
      if (!p.deduplicate) strip = 0;
      place_off[q] = written;
      place_strip[q] = strip;
      written += n - strip;
      covered = max(end, tstart + n);
      last_ref = it_ref[q];
    }
    n_kept = placed;
    n_written = written;
    p.routing_candidates[b] = count;
    p.mem_len[b] = min(written, p.max_mem);
    p.duplicate_tokens[b] = duplicates;
    if (written > p.max_mem) p.status[b] = 2;
  }
  __syncthreads();
  // 4e. trace records: retained items in selection order
  {
    const int q = threadIdx.x;
    const int flag = (q < count && it_keep[q] == 2) ? 1 : 0;
    // count may exceed NT only when MAX_SEL > NT
    int kept = block_exclusive_scan(flag, warp_tot, &n_total);
    if (flag && kept < p.max_sel) {
      const int64_t o = (int64_t)b * p.max_sel + kept;
      const int i = it_pos[q];
      p.sel_chunk[o] = it_chunk[q];
      p.sel_ref_rank[o] = it_rrank[q];
      p.sel_chunk_rank[o] = it_crank[q];
      p.sel_ref_score[o] = it_rscore[q];
      p.sel_chunk_score[o] = it_cscore[q];
      p.sel_win_index[o] = widx[i];
      p.sel_win_score[o] = wscore[i];
    }
    if (threadIdx.x == 0) p.sel_count[b] = min(n_total, p.max_sel);
  }
  // 4f. the memory key list, filled in parallel
  const int kept_items = n_kept;
  for (int k = warp; k < kept_items; k += nwarps) {
    const int q = by_place[k];
    const int c = it_chunk[q];
    if (p.gist_only) {
      if (lane == 0 && place_off[q] < p.max_mem)
        p.mem_idx[(int64_t)b * p.max_mem + place_off[q]] = c * p.G + widx[it_pos[q]];
      continue;
    }
    const int base_row = p.chunk_pool_row[c];
    for (int t = place_strip[q] + lane; t < it_len[q]; t += 32) {
      const int at = place_off[q] + t - place_strip[q];
      if (at < p.max_mem) p.mem_idx[(int64_t)b * p.max_mem + at] = base_row + t;
    }
  }
}

}  // namespace route
}  // namespace pra

cudaError_t pra_route(const RouteParams& p, cudaStream_t st) {
  using namespace pra::route;
  if (p.B == 0) return cudaSuccess;
  if (p.G > 8) return cudaErrorInvalidValue;
  if (p.D % 4 != 0 || (reinterpret_cast<uintptr_t>(p.gists) & 15)) return cudaErrorInvalidValue;
  const size_t smem = (size_t)p.D * sizeof(float) + (size_t)MAX_ROW_CHUNKS * (2 * sizeof(float) + 3 * sizeof(int)) +
                      (size_t)MAX_ROW_REFS * (sizeof(float) + 2 * sizeof(int));
  PRA_RETURN_IF_ERROR(pra::set_max_dynamic_smem(reinterpret_cast<const void*>(route_kernel), (int)smem));
  route_kernel<<<p.B, NT, smem, st>>>(p);
  return cudaGetLastError();
}
