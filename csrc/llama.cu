// Hot ops of the PRA Llama-family engine (Llama 3 / Mistral / Qwen2) on sm_100a.
//
//  * rope_copy      rotary positions (HF rotate_half layout, fp32 cos/sin tables built in
//                   fp64 on the host) applied while copying head rows to a destination row
//                   (in place for queries, into the KV cache / chunk pool for keys); with a
//                   null position table it is a plain row copy (values).
//  * decode_prologue one launch per decode step: token embeddings (with the first folded
//                   RMSNorm's sums of squares), rotary positions, cache rows, new lengths.
//  * silu_mul       SwiGLU activation over a fused [gate | up] GEMM output (halves, or the
//                   runs-of-64 interleave the decode GEMM's SwiGLU epilogue reads).
//  * decode attention: split-K flash decoding for grouped-query heads.  One CTA per
//                   (row, kv head, key split) computes the unnormalised partial
//                   (max, sum, out) of the group's query heads over its keys; keys are
//                   [selected memory rows (gathered through a row list) ; local cache
//                   rows], all visible to the token being decoded.  The splits can be laid
//                   out as memory-only and local-only ranges launched separately (the local
//                   ones before routing has run), and a persistent grid can walk them.  A
//                   second kernel merges the splits (and optionally exports the merged
//                   partial for a cross-GPU combine).
//  * route_topk     exact top-k routing per row: radix-select of the candidates from
//                   tensor-core scores, fp32 cosine rescoring of the candidates, ties by
//                   chunk id, greedy token budget, and the memory row list in chunk order.
#include <algorithm>
#include <climits>

#include "common.cuh"
#include "tcgen05.cuh"

namespace pra {
namespace llama {

// ---------------------------------------------------------------- rope / copy
__global__ void rope_copy_kernel(RopeCopyArgs a) {
  const int m = blockIdx.x;
  const int half = a.head_dim / 2;
  const int pairs = a.heads * half;
  const __nv_bfloat16* src = a.src + (int64_t)m * a.src_stride;
  const int64_t drow = a.dst_rows ? a.dst_rows[m] : m;
  __nv_bfloat16* dst = a.dst + drow * a.dst_stride;
  const int pos = a.pos ? a.pos[m] : 0;
  for (int e = blockIdx.y * blockDim.x + threadIdx.x; e < pairs; e += gridDim.y * blockDim.x) {
    const int h = e / half, i = e - h * half;
    const int c0 = h * a.head_dim + i, c1 = c0 + half;
    const float x0 = __bfloat162float(src[c0]), x1 = __bfloat162float(src[c1]);
    if (a.cos_t == nullptr) {
      dst[c0] = src[c0];
      dst[c1] = src[c1];
    } else {
      const float c = a.cos_t[(int64_t)pos * half + i], s = a.sin_t[(int64_t)pos * half + i];
      dst[c0] = __float2bfloat16(x0 * c - x1 * s);
      dst[c1] = __float2bfloat16(x1 * c + x0 * s);
    }
  }
}

// ---------------------------------------------------------------- decode step prologue
// One CTA per batch row: the token's embedding row (16-byte copies), its rotary position
// (cache length + position offset), the cache row it is written to (b * max_len + cache length)
// and the row's new cache length.  Token ids outside the vocabulary read row 0 and are reported
// through the bounds status when checking is on.
__global__ void decode_prologue_kernel(DecodePrologueArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.x;
  int64_t id = a.ids[b];
  if (id < 0 || id >= a.vocab) {
    if (threadIdx.x == 0 && a.bounds) bounds_fail(a.bounds, PRA_BOUNDS_DECODE_TOKEN, id, a.vocab);
    id = 0;
  }
  const uint4* src = reinterpret_cast<const uint4*>(a.embed + id * a.d);
  uint4* dst = reinterpret_cast<uint4*>(a.x + (int64_t)b * a.d);
  float ss = 0.f;
  for (int64_t c = threadIdx.x; c < a.d / 8; c += blockDim.x) {
    const uint4 v = src[c];
    dst[c] = v;
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      ss += f.x * f.x + f.y * f.y;
    }
  }
  if (a.ss_out != nullptr) {  // the first folded RMSNorm's sum of squares (fixed summation order)
    __shared__ float warp_ss[32];
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) warp_ss[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.f;
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += warp_ss[w];
      a.ss_out[b] = t;
    }
  }
  if (threadIdx.x == 0) {
    const int len = a.cache_len[b];
    a.pos[b] = len + (a.pos_offset ? a.pos_offset[b] : 0);
    a.rows[b] = b * a.max_len + len;
    a.new_len[b] = len + 1;
  }
}

// ---------------------------------------------------------------- swiglu
__global__ void silu_mul_kernel(const __nv_bfloat16* __restrict__ gu, int64_t M, int F, int block,
                                __nv_bfloat16* __restrict__ out) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t pairs = M * (F / 2);
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < pairs; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = e / (F / 2);
    const int j = 2 * (int)(e - m * (F / 2));
    const int gc = block > 0 ? (j / block) * 2 * block + j % block : j;  // gate column of feature j
    const int uc = block > 0 ? gc + block : F + j;
    const float2 g = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(gu + m * 2 * F + gc));
    const float2 u = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(gu + m * 2 * F + uc));
    const float a = g.x / (1.f + __expf(-g.x)) * u.x;
    const float b = g.y / (1.f + __expf(-g.y)) * u.y;
    *reinterpret_cast<__nv_bfloat162*>(out + m * F + j) = __floats2bfloat162_rn(a, b);
  }
}

// ---------------------------------------------------------------- decode attention
constexpr int DT = 128;   // threads (4 warps, 16 keys each per block of 64)
constexpr int DBN = 64;   // keys per block
constexpr int DSTAGES = 2;  // cp.async pipeline depth (blocks in flight per CTA)
constexpr float LOG2E = 1.4426950408889634f;

template <int D>
struct DSmem {
  static constexpr int LD = D + 8;
};

constexpr int kBadRow = INT_MIN;  // checked variant: a key whose row failed its bounds check

template <int D, bool CHECK>
__global__ void __launch_bounds__(DT) decode_kernel(DecodeAttnParams p) {
  constexpr int LD = DSmem<D>::LD;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __nv_bfloat16* sq = reinterpret_cast<__nv_bfloat16*>(smem_raw);  // [16][LD]
  __nv_bfloat16* sk = sq + 16 * LD;                                 // [STAGES][DBN][LD]
  __nv_bfloat16* sv = sk + DSTAGES * DBN * LD;                      // [STAGES][DBN][LD]
  float* red = reinterpret_cast<float*>(sk);                        // [4][16][D + 2], after the key loop
  int* srow = reinterpret_cast<int*>(sv + DSTAGES * DBN * LD);      // [split_keys] key row (>= 0: memory pool)

  const int G = p.H / p.Hkv;
  const int b = blockIdx.x / p.Hkv, kvh = blockIdx.x % p.Hkv;
  const int split = p.split_lo + blockIdx.y;
  const bool local_only = p.mem_splits > 0 && split >= p.mem_splits;
  const bool mem_only = p.mem_splits > 0 && split < p.mem_splits;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int mem_len = (!local_only && p.mem_len) ? p.mem_len[b] : 0;
  int loc_len = (!mem_only && p.loc_len) ? p.loc_len[b] : 0;
  if constexpr (CHECK) {  // lengths past their buffers: record, then clamp (the extra keys are skipped)
    if (mem_len < 0 || mem_len > p.mem_max) {
      if (threadIdx.x == 0) bounds_fail(p.bounds, PRA_BOUNDS_DECODE_MEM_LEN, mem_len, p.mem_max);
      mem_len = max(0, min(mem_len, p.mem_max));
    }
    if (loc_len < 0 || (p.loc_k != nullptr && loc_len > p.loc_cap)) {
      if (threadIdx.x == 0) bounds_fail(p.bounds, PRA_BOUNDS_DECODE_LOC_LEN, loc_len, p.loc_cap);
      loc_len = max(0, min(loc_len, p.loc_cap));
    }
  }
  const int total = mem_len + loc_len;
  const int keys = mem_only && p.mem_split_keys > 0 ? p.mem_split_keys : p.split_keys;
  const int k0 = (local_only ? split - p.mem_splits : split) * keys, k1 = min(total, k0 + keys);
  const int64_t part = ((int64_t)b * p.H + kvh * G) * p.n_split + split;  // first head of the group

  // queries of the group (rows >= G are zero)
  for (int c = threadIdx.x; c < 16 * (D / 8); c += DT) {
    const int r = c / (D / 8), col = (c % (D / 8)) * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < G) v = *reinterpret_cast<const uint4*>(p.q + (int64_t)b * p.q_row + (kvh * G + r) * D + col);
    *reinterpret_cast<uint4*>(sq + r * LD + col) = v;
  }
  // key rows of this split, resolved once: memory keys -> pool row, local keys -> -(t + 1)
  for (int j = k0 + threadIdx.x; j < k1; j += DT) {
    int r = j < mem_len ? p.mem_idx[(int64_t)b * p.mem_max + j] : -(j - mem_len + 1);
    if constexpr (CHECK) {
      if (j < mem_len && (r < 0 || r >= p.mem_rows)) {
        bounds_fail(p.bounds, PRA_BOUNDS_DECODE_MEM_ROW, r, p.mem_rows);
        r = kBadRow;  // never loaded, scored -inf
      }
    }
    srow[j - k0] = r;
  }
  __syncthreads();
  auto key_addr = [&](int j, bool value) -> const __nv_bfloat16* {
    const int r = srow[j - k0];
    if (r >= 0) return (value ? p.mem_v : p.mem_k) + (int64_t)r * p.mem_row + kvh * D;
    return (value ? p.loc_v : p.loc_k) + (int64_t)b * p.loc_batch + (int64_t)(-r - 1) * p.loc_row + kvh * D;
  };
  auto load_block = [&](int start, int buf) {
    for (int c = threadIdx.x; c < DBN * (D / 8); c += DT) {
      const int r = c / (D / 8), col = (c % (D / 8)) * 8;
      const int j = start + r;
      const bool ok = j < k1 && (!CHECK || srow[j - k0] != kBadRow);
      cp_async16(sk + (buf * DBN + r) * LD + col, ok ? key_addr(j, false) + col : p.q, ok);
      cp_async16(sv + (buf * DBN + r) * LD + col, ok ? key_addr(j, true) + col : p.q, ok);
    }
    cp_async_commit();
  };

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  const float sl2 = p.scale * LOG2E;
  const int n_blocks = k1 > k0 ? (k1 - k0 + DBN - 1) / DBN : 0;
#pragma unroll
  for (int st = 0; st < DSTAGES - 1; ++st) {
    if (st < n_blocks) load_block(k0 + st * DBN, st);
    else cp_async_commit();  // empty group keeps the wait counts uniform
  }
  for (int it = 0; it < n_blocks; ++it) {
    const int buf = it % DSTAGES;
    cp_async_wait<DSTAGES - 2>();
    __syncthreads();  // block `it` landed; every warp is done with block it - 1
    if (it + DSTAGES - 1 < n_blocks) load_block(k0 + (it + DSTAGES - 1) * DBN, (it + DSTAGES - 1) % DSTAGES);
    else cp_async_commit();
    // S = Q[16 x D] . K[16 keys of this warp]^T
    float s[2][4];
#pragma unroll
    for (int i = 0; i < 2; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
    const __nv_bfloat16* kb = sk + (buf * DBN + warp * 16) * LD;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t a[4], bb[4];
      ldmatrix_x4(a, smem_u32(sq + (lane & 15) * LD + kk * 16 + (lane >> 4) * 8));
      const int row = ((lane >> 4) & 1) * 8 + (lane & 7);
      ldmatrix_x4(bb, smem_u32(kb + row * LD + kk * 16 + ((lane >> 3) & 1) * 8));
      mma_bf16_16816(s[0], a, bb);
      mma_bf16_16816(s[1], a, bb + 2);
    }
    const int key_base = k0 + it * DBN + warp * 16;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nb = 0; nb < 2; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = key_base + nb * 8 + (lane & 3) * 2 + (e & 1);
        if (key >= k1 || (CHECK && srow[key - k0] == kBadRow)) s[nb][e] = -INFINITY;
        mx[e >> 1] = fmaxf(mx[e >> 1], s[nb][e]);
      }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float m_new = fmaxf(m_run[r], mx[r]);
      const float corr = (m_new == -INFINITY) ? 1.f : exp2f((m_run[r] - m_new) * sl2);
      m_run[r] = m_new;
      l_run[r] *= corr;
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        o[i][2 * r] *= corr;
        o[i][2 * r + 1] *= corr;
      }
    }
#pragma unroll
    for (int nb = 0; nb < 2; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = e >> 1;
        const float v = (m_run[r] == -INFINITY) ? 0.f : exp2f((s[nb][e] - m_run[r]) * sl2);
        s[nb][e] = v;
        l_run[r] += v;
      }
    // O += P[16 x 16] . V[16 keys x D]
    uint32_t a[4];
    a[0] = pack_bf16(s[0][0], s[0][1]);
    a[1] = pack_bf16(s[0][2], s[0][3]);
    a[2] = pack_bf16(s[1][0], s[1][1]);
    a[3] = pack_bf16(s[1][2], s[1][3]);
    const __nv_bfloat16* vb = sv + (buf * DBN + warp * 16) * LD;
#pragma unroll
    for (int np = 0; np < D / 16; ++np) {
      uint32_t bb[4];
      const int mm = lane >> 3;
      const int row = (mm & 1) * 8 + (lane & 7);
      ldmatrix_x4_trans(bb, smem_u32(vb + row * LD + np * 16 + (mm >> 1) * 8));
      mma_bf16_16816(o[2 * np], a, bb);
      mma_bf16_16816(o[2 * np + 1], a, bb + 2);
    }
  }
  cp_async_wait<0>();
  __syncthreads();  // the staging area becomes the warp-merge buffer
  // merge the four warps' partials (rows: lane >> 2 and + 8)
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 1);
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 2);
  }
  constexpr int RS = D + 2;  // per (warp, row): o[D], m, l
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = (lane >> 2) + 8 * r;
    float* dst = red + (warp * 16 + row) * RS;
#pragma unroll
    for (int nb = 0; nb < D / 8; ++nb) {
      const int col = nb * 8 + (lane & 3) * 2;
      dst[col] = o[nb][2 * r];
      dst[col + 1] = o[nb][2 * r + 1];
    }
    if ((lane & 3) == 0) {
      dst[D] = m_run[r];
      dst[D + 1] = l_run[r];
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < G * D; e += DT) {
    const int row = e / D, col = e % D;
    float M = -INFINITY;
    for (int w = 0; w < 4; ++w) M = fmaxf(M, red[(w * 16 + row) * RS + D]);
    float acc = 0.f, L = 0.f;
    for (int w = 0; w < 4; ++w) {
      const float* src = red + (w * 16 + row) * RS;
      const float f = (src[D] == -INFINITY) ? 0.f : exp2f((src[D] - M) * sl2);
      acc += src[col] * f;
      L += src[D + 1] * f;
    }
    const int64_t at = part + (int64_t)row * p.n_split;
    p.part_o[at * D + col] = acc;
    if (col == 0) {
      p.part_ml[at * 2] = M == -INFINITY ? -INFINITY : M * p.scale;  // natural-log units
      p.part_ml[at * 2 + 1] = L;
    }
  }
}

// ---------------------------------------------------------------- decode attention, TMA-fed
// The same split-K GQA flash decoding as decode_kernel, with the key / value blocks brought in
// by the tensor-memory accelerator: a 64-key block of one KV head is a 64-row x D-column box of
// the local cache or of the memory pool (a selected chunk is 64 consecutive pool rows), so one
// thread issues 2 * D / 64 tile copies per block against an mbarrier instead of every thread
// issuing 16-byte copies and resolving row addresses.  Blocks whose memory rows are not one
// contiguous run (partial chunks, or a block straddling memory and local keys) are gathered
// with cp.async into the same 128-byte-swizzled layout.  The tiles are read with ldmatrix at
// swizzled addresses; scores, softmax and the warp merge are decode_kernel's.
constexpr int TST_DEFAULT = 2;   // pipeline stages (blocks in flight per CTA): 3 CTAs per SM
constexpr int TBOX = 64 * 64 * 2;  // one 64-key x 64-column bf16 box (8 KB, 128-byte rows)
constexpr int TMAX_BLOCKS = 64;  // split_keys <= 4096
constexpr long long TWAIT_CYCLES = 4000000000LL;  // about two seconds at the boost clock

template <int D>
struct TLayout {
  static constexpr int NBOX = D / 64;
  static constexpr int TILE = NBOX * TBOX;  // K (or V) tile of one block
  static constexpr int STAGE = 2 * TILE;
  static constexpr int QLD = D + 8;
};

// Byte offset of (row r, column c) of a swizzled 64-row tile: 64-column boxes of 128-byte rows,
// 16-byte chunk k of row r stored at chunk k ^ (r % 8).
__device__ __forceinline__ uint32_t sw_off(int r, int c) {
  return (uint32_t)((c >> 6) * TBOX + r * 128 + ((((c & 63) >> 3) ^ (r & 7)) << 4) + ((c & 7) << 1));
}

template <int D, int TST>
__global__ void __launch_bounds__(DT) decode_tma_kernel(const __grid_constant__ CUtensorMap map_mk,
                                                        const __grid_constant__ CUtensorMap map_mv,
                                                        const __grid_constant__ CUtensorMap map_lk,
                                                        const __grid_constant__ CUtensorMap map_lv,
                                                        DecodeAttnParams p) {
  using Lay = TLayout<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* stages = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __nv_bfloat16* sq = reinterpret_cast<__nv_bfloat16*>(stages + TST * Lay::STAGE);  // [16][QLD]
  int* srow = reinterpret_cast<int*>(sq + 16 * Lay::QLD);                          // [split_keys]
  int* blk_mode = srow + p.split_keys;   // per block: 0 TMA memory, 1 TMA local, 2 gathered
  int* blk_y = blk_mode + TMAX_BLOCKS;   // TMA row coordinate
  uint64_t* full = reinterpret_cast<uint64_t*>(blk_y + TMAX_BLOCKS);  // [TST] (8-byte aligned: even int count)
  __shared__ int s_fail;
  float* red = reinterpret_cast<float*>(stages);  // [4][16][D + 2], after the key loop

  const int G = p.H / p.Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < TST; ++s) mbar_init(full + s, 1);
    s_fail = 0;
    tc::fence_mbarrier_init();
    asm volatile("prefetch.tensormap [%0];\n" ::"l"(&map_lk) : "memory");
    asm volatile("prefetch.tensormap [%0];\n" ::"l"(&map_lv) : "memory");
  }
  pdl_launch_dependents();
  pdl_wait();  // q, the new cache row and the routed row lists come from the kernels before
  uint32_t phase = 0;  // bit s: parity the next TMA completion of stage s shows (kept across items)
  // Work items are (row, KV head, split).  The ordinary grid runs one item per CTA; a persistent
  // grid (p.max_ctas) walks items with a stride, leaving the rest of each SM to other kernels.
  const int n_items = p.B * p.Hkv * (p.split_count > 0 ? p.split_count : p.n_split);
  for (int item = blockIdx.y * gridDim.x + blockIdx.x; item < n_items; item += gridDim.x * gridDim.y) {
  const int bh = item % (p.B * p.Hkv);
  const int b = bh / p.Hkv, kvh = bh % p.Hkv;
  const int split = p.split_lo + item / (p.B * p.Hkv);
  const bool local_only = p.mem_splits > 0 && split >= p.mem_splits;
  const bool mem_only = p.mem_splits > 0 && split < p.mem_splits;
  const int mem_len = (!local_only && p.mem_len) ? p.mem_len[b] : 0;
  const int total = mem_len + ((!mem_only && p.loc_len) ? p.loc_len[b] : 0);
  const int keys = mem_only && p.mem_split_keys > 0 ? p.mem_split_keys : p.split_keys;
  const int k0 = (local_only ? split - p.mem_splits : split) * keys, k1 = min(total, k0 + keys);
  const int64_t part = ((int64_t)b * p.H + kvh * G) * p.n_split + split;
  const int loc_rows = (int)(p.loc_batch / p.loc_row);  // cache rows per batch row

  for (int c = threadIdx.x; c < 16 * (D / 8); c += DT) {
    const int r = c / (D / 8), col = (c % (D / 8)) * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < G) v = *reinterpret_cast<const uint4*>(p.q + (int64_t)b * p.q_row + (kvh * G + r) * D + col);
    *reinterpret_cast<uint4*>(sq + r * Lay::QLD + col) = v;
  }
  for (int j = k0 + threadIdx.x; j < k1; j += DT)
    srow[j - k0] = j < mem_len ? p.mem_idx[(int64_t)b * p.mem_max + j] : -(j - mem_len + 1);
  __syncthreads();
  const int n_blocks = k1 > k0 ? (k1 - k0 + DBN - 1) / DBN : 0;
  // classify the blocks (warp per block): one contiguous run of rows -> one TMA box per 64 columns
  for (int blk = warp; blk < n_blocks; blk += DT / 32) {
    const int j0 = k0 + blk * DBN, n = min(DBN, k1 - j0);
    int mode = 2, y = 0;
    if (j0 >= mem_len) {
      mode = 1;
      y = b * loc_rows + (j0 - mem_len);
    } else if (j0 + n <= mem_len) {
      const int r0 = srow[j0 - k0];
      bool run = true;
      for (int i = lane; i < n; i += 32) run = run && srow[j0 - k0 + i] == r0 + i;
      run = __all_sync(0xffffffffu, run);
      if (run) {
        mode = 0;
        y = r0;
      }
    }
    if (lane == 0) {
      blk_mode[blk] = mode;
      blk_y[blk] = y;
    }
  }
  __syncthreads();
  auto key_addr = [&](int j, bool value) -> const __nv_bfloat16* {
    const int r = srow[j - k0];
    if (r >= 0) return (value ? p.mem_v : p.mem_k) + (int64_t)r * p.mem_row + kvh * D;
    return (value ? p.loc_v : p.loc_k) + (int64_t)b * p.loc_batch + (int64_t)(-r - 1) * p.loc_row + kvh * D;
  };
  auto issue = [&](int blk, int buf) {
    uint8_t* st = stages + buf * Lay::STAGE;
    const int mode = blk_mode[blk];
    if (mode < 2) {
      if (threadIdx.x == 0) {
        expect_tx(full + buf, Lay::STAGE);
        const CUtensorMap* mk = mode == 0 ? &map_mk : &map_lk;
        const CUtensorMap* mv = mode == 0 ? &map_mv : &map_lv;
#pragma unroll
        for (int bx = 0; bx < Lay::NBOX; ++bx) {
          tma_load(st + bx * TBOX, mk, kvh * D + bx * 64, blk_y[blk], full + buf);
          tma_load(st + Lay::TILE + bx * TBOX, mv, kvh * D + bx * 64, blk_y[blk], full + buf);
        }
      }
    } else {
      const int j0 = k0 + blk * DBN;
      for (int c = threadIdx.x; c < DBN * (D / 8); c += DT) {
        const int r = c / (D / 8), col = (c % (D / 8)) * 8;
        const int j = j0 + r;
        const bool ok = j < k1;
        cp_async16(st + sw_off(r, col), ok ? key_addr(j, false) + col : p.q, ok);
        cp_async16(st + Lay::TILE + sw_off(r, col), ok ? key_addr(j, true) + col : p.q, ok);
      }
    }
    cp_async_commit();  // one group per block (empty for TMA blocks) keeps the wait counts uniform
  };

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  const float sl2 = p.scale * LOG2E;
#pragma unroll
  for (int st = 0; st < TST - 1; ++st) {
    if (st < n_blocks) issue(st, st);
    else cp_async_commit();
  }
  int it = 0;
  for (; it < n_blocks; ++it) {
    const int buf = it % TST;
    cp_async_wait<TST - 2>();
    if (blk_mode[it] < 2) {
      if (!tc::mbar_wait_cycles(full + buf, (phase >> buf) & 1u, TWAIT_CYCLES)) s_fail = 1;
      phase ^= 1u << buf;
    }
    __syncthreads();  // block `it` landed for every thread; every warp is done with block it - 1
    if (s_fail) break;
    if (it + TST - 1 < n_blocks) issue(it + TST - 1, (it + TST - 1) % TST);
    else cp_async_commit();
    const uint32_t kst = smem_u32(stages + buf * Lay::STAGE), vst = kst + Lay::TILE;
    float s[2][4];
#pragma unroll
    for (int i = 0; i < 2; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t a[4], bb[4];
      ldmatrix_x4(a, smem_u32(sq + (lane & 15) * Lay::QLD + kk * 16 + (lane >> 4) * 8));
      const int row = warp * 16 + ((lane >> 4) & 1) * 8 + (lane & 7);
      ldmatrix_x4(bb, kst + sw_off(row, kk * 16 + ((lane >> 3) & 1) * 8));
      mma_bf16_16816(s[0], a, bb);
      mma_bf16_16816(s[1], a, bb + 2);
    }
    const int key_base = k0 + it * DBN + warp * 16;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nb = 0; nb < 2; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = key_base + nb * 8 + (lane & 3) * 2 + (e & 1);
        if (key >= k1) s[nb][e] = -INFINITY;
        mx[e >> 1] = fmaxf(mx[e >> 1], s[nb][e]);
      }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float m_new = fmaxf(m_run[r], mx[r]);
      const float corr = (m_new == -INFINITY) ? 1.f : exp2f((m_run[r] - m_new) * sl2);
      m_run[r] = m_new;
      l_run[r] *= corr;
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        o[i][2 * r] *= corr;
        o[i][2 * r + 1] *= corr;
      }
    }
#pragma unroll
    for (int nb = 0; nb < 2; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = e >> 1;
        const float v = (m_run[r] == -INFINITY) ? 0.f : exp2f((s[nb][e] - m_run[r]) * sl2);
        s[nb][e] = v;
        l_run[r] += v;
      }
    uint32_t a[4];
    a[0] = pack_bf16(s[0][0], s[0][1]);
    a[1] = pack_bf16(s[0][2], s[0][3]);
    a[2] = pack_bf16(s[1][0], s[1][1]);
    a[3] = pack_bf16(s[1][2], s[1][3]);
#pragma unroll
    for (int np = 0; np < D / 16; ++np) {
      uint32_t bb[4];
      const int mm = lane >> 3;
      const int row = warp * 16 + (mm & 1) * 8 + (lane & 7);
      ldmatrix_x4_trans(bb, vst + sw_off(row, np * 16 + (mm >> 1) * 8));
      mma_bf16_16816(o[2 * np], a, bb);
      mma_bf16_16816(o[2 * np + 1], a, bb + 2);
    }
  }
  cp_async_wait<0>();
  if (s_fail) {  // a copy never completed: wait (bounded) for every TMA block still in flight
    for (int k = it; k < min(n_blocks, it + TST - 1); ++k) {
      const int buf = k % TST;
      if (blk_mode[k] < 2 && threadIdx.x == 0) {
        tc::mbar_wait_cycles(full + buf, (phase >> buf) & 1u, TWAIT_CYCLES);
        phase ^= 1u << buf;
      }
    }
    if (threadIdx.x == 0 && p.status) atomicExch(p.status, 1);
    __syncthreads();
    return;
  }
  __syncthreads();  // the staging area becomes the warp-merge buffer
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 1);
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 2);
  }
  constexpr int RS = D + 2;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = (lane >> 2) + 8 * r;
    float* dst = red + (warp * 16 + row) * RS;
#pragma unroll
    for (int nb = 0; nb < D / 8; ++nb) {
      const int col = nb * 8 + (lane & 3) * 2;
      dst[col] = o[nb][2 * r];
      dst[col + 1] = o[nb][2 * r + 1];
    }
    if ((lane & 3) == 0) {
      dst[D] = m_run[r];
      dst[D + 1] = l_run[r];
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < G * D; e += DT) {
    const int row = e / D, col = e % D;
    float M = -INFINITY;
    for (int w = 0; w < 4; ++w) M = fmaxf(M, red[(w * 16 + row) * RS + D]);
    float acc = 0.f, L = 0.f;
    for (int w = 0; w < 4; ++w) {
      const float* src = red + (w * 16 + row) * RS;
      const float f = (src[D] == -INFINITY) ? 0.f : exp2f((src[D] - M) * sl2);
      acc += src[col] * f;
      L += src[D + 1] * f;
    }
    const int64_t at = part + (int64_t)row * p.n_split;
    p.part_o[at * D + col] = acc;
    if (col == 0) {
      p.part_ml[at * 2] = M == -INFINITY ? -INFINITY : M * p.scale;
      p.part_ml[at * 2 + 1] = L;
    }
  }
  __syncthreads();  // the merge buffer (staging area), q and the row list are the next item's
  }  // work items
}

// Merge the splits of each (row, head): out = sum_s o_s e^{m_s - M} / sum_s l_s e^{m_s - M}.
// With export_ml the merged (M, L) and unnormalised out are also written (cross-GPU combine).
__global__ void decode_merge_kernel(DecodeAttnParams p, int D) {
  pdl_launch_dependents();
  pdl_wait();
  const int bh = blockIdx.x;
  const int b = bh / p.H, h = bh % p.H;
  const int64_t base = (int64_t)bh * p.n_split;
  float M = -INFINITY;
  for (int s = 0; s < p.n_split; ++s) M = fmaxf(M, p.part_ml[(base + s) * 2]);
  float L = 0.f;
  for (int s = 0; s < p.n_split; ++s) {
    const float m = p.part_ml[(base + s) * 2];
    L += m == -INFINITY ? 0.f : p.part_ml[(base + s) * 2 + 1] * __expf(m - M);
  }
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < p.n_split; ++s) {
      const float m = p.part_ml[(base + s) * 2];
      if (m != -INFINITY) acc += p.part_o[(base + s) * D + d] * __expf(m - M);
    }
    if (p.out) p.out[(int64_t)b * p.out_row + h * D + d] = __float2bfloat16(L > 0.f ? acc / L : 0.f);
    if (p.export_o) p.export_o[(int64_t)bh * D + d] = acc;
  }
  if (threadIdx.x == 0 && p.export_ml) {
    p.export_ml[bh * 2] = M;
    p.export_ml[bh * 2 + 1] = L;
  }
}

// ---------------------------------------------------------------- routing top-k
constexpr int RT = 1024;
constexpr int MAX_CAND = 512;
constexpr int STAGE_N = 8192;  // chunk scores of one segment staged in shared memory

__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Exclusive prefix sum of one int per thread over an RT-thread block; *total gets the sum.
__device__ __forceinline__ int block_scan_int(int v, int* tmp, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  __syncthreads();
  if (lane == 31) tmp[warp] = x;
  __syncthreads();
  int base = 0, all = 0;
  for (int w = 0; w < RT / 32; ++w) {
    if (w < warp) base += tmp[w];
    all += tmp[w];
  }
  *total = all;
  return base + x - v;
}

// Ranks candidates by (-score, chunk id) and keeps the best k.  Local mode (cand_score set):
// writes them in rank order (global ids = id + id_offset; -inf / -1 padding) and stops.
// Otherwise applies the greedy token budget in rank order, sorts the kept chunks by id and
// writes the selection and the memory row list (all threads of the CTA take part).
template <bool CHECK>
__device__ void finish_selection(const float* cscore, const int* cand, int nc, int b, int k_req, int budget,
                                 const int* chunk_len, const int* chunk_row0, int* mem_idx, int mem_max,
                                 int* mem_len, int* sel_out, float* cand_score, int* cand_id, int id_offset,
                                 int* picked, int* sel_chunk, int* sel_off, int* n_sel, int64_t pool_rows,
                                 BoundsStatus* bounds) {
  const int k = min(k_req, nc);
  for (int i = threadIdx.x; i < nc; i += blockDim.x) {
    int rank = 0;
    for (int j = 0; j < nc; ++j)
      rank += (cscore[j] > cscore[i] || (cscore[j] == cscore[i] && cand[j] < cand[i])) ? 1 : 0;
    picked[i] = rank;  // ranks are unique
  }
  __syncthreads();
  if (cand_score != nullptr) {
    for (int i = threadIdx.x; i < nc; i += blockDim.x) {
      if (picked[i] < k) {
        cand_score[(int64_t)b * k_req + picked[i]] = cscore[i];
        cand_id[(int64_t)b * k_req + picked[i]] = cand[i] + id_offset;
      }
    }
    for (int r = k + threadIdx.x; r < k_req; r += blockDim.x) {
      cand_score[(int64_t)b * k_req + r] = -INFINITY;
      cand_id[(int64_t)b * k_req + r] = -1;
    }
    return;
  }
  // the top-k candidates' ids, lengths and first pool rows in rank order, loaded in parallel
  // (the greedy budget below is sequential; dependent global loads there cost microseconds)
  __shared__ int s_cid[64], s_len[64], s_row0[64], sel_row0[64];
  const int kk = min(k, 64);
  for (int i = threadIdx.x; i < nc; i += blockDim.x) {
    const int r = picked[i];
    if (r < kk) {
      const int c = cand[i];
      s_cid[r] = c;
      s_len[r] = chunk_len[c];
      s_row0[r] = chunk_row0[c];
    }
  }
  __syncthreads();
  // greedy token budget in rank order (sequential by definition; shared-memory only).  Without
  // a budget every ranked candidate is kept, so the loop is skipped.
  __shared__ int s_keep[64], sel_len[64];
  if (budget < 0) {
    if (threadIdx.x < kk) s_keep[threadIdx.x] = 1;
    if (threadIdx.x == 0) *n_sel = kk;
  } else if (threadIdx.x == 0) {
    int used = 0, chosen = 0;
    for (int r = 0; r < kk; ++r) {
      const int len = s_len[r];
      const bool keep = used + len <= budget;
      if (keep) {
        used += len;
        ++chosen;
      }
      s_keep[r] = keep;
    }
    *n_sel = chosen;
  }
  __syncthreads();
  // the kept chunks in chunk-id order: each finds its place by counting smaller kept ids
  const int chosen = *n_sel;
  if (threadIdx.x < kk && s_keep[threadIdx.x]) {
    const int r = threadIdx.x, c = s_cid[r];
    int pos = 0;
    for (int o = 0; o < kk; ++o) pos += (s_keep[o] && s_cid[o] < c) ? 1 : 0;
    sel_chunk[pos] = c;
    sel_len[pos] = s_len[r];
    sel_row0[pos] = s_row0[r];
  }
  __syncthreads();
  if (threadIdx.x < 32) {  // row offsets by a warp prefix sum, two chunks per lane (chunks held
                           // elsewhere, row0 < 0, add no rows here)
    const int lane = threadIdx.x;
    const int i0 = 2 * lane, i1 = 2 * lane + 1;
    const int n0 = i0 < chosen && sel_row0[i0] >= 0 ? sel_len[i0] : 0;
    const int n1 = i1 < chosen && sel_row0[i1] >= 0 ? sel_len[i1] : 0;
    int incl = n0 + n1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const int excl = incl - n0 - n1;
    if (i0 <= chosen) sel_off[i0] = excl;
    if (i1 <= chosen) sel_off[i1] = excl + n0;
    if (lane == 31) {
      sel_off[chosen] = incl;  // == the total once every lane is summed
      mem_len[b] = min(incl, mem_max);
    }
  }
  for (int i = threadIdx.x; i < k_req && sel_out; i += blockDim.x)
    sel_out[(int64_t)b * k_req + i] = i < chosen ? sel_chunk[i] : -1;
  __syncthreads();
  // the memory row list, one row per thread: row t belongs to the last chunk whose offset <= t
  const int rows_out = min(sel_off[chosen], mem_max);
  for (int t = threadIdx.x; t < rows_out; t += blockDim.x) {
    int lo = 0, hi = chosen - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (sel_off[mid] <= t) lo = mid;
      else hi = mid - 1;
    }
    int row = sel_row0[lo] + (t - sel_off[lo]);
    if constexpr (CHECK) {
      if (pool_rows >= 0 && (int64_t)row >= pool_rows) {  // the chunk's rows run past the pool: record, mark the key bad
        bounds_fail(bounds, PRA_BOUNDS_ROUTE_POOL_ROW, row, pool_rows);
        row = -1;
      }
    }
    mem_idx[(int64_t)b * mem_max + t] = row;
  }
}

__device__ __forceinline__ void signal_release(uint32_t* addr, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(addr), "r"(v) : "memory");
}

template <bool CHECK, bool EXCH>
__global__ void __launch_bounds__(RT) route_topk_kernel(RouteTopkArgs a, RouteExchangeArgs x) {
  __shared__ uint32_t hist[256];
  __shared__ uint32_t prefix, prefix_mask;
  __shared__ int need;
  __shared__ int n_cand;
  __shared__ int cand[MAX_CAND];
  __shared__ float cscore[MAX_CAND];
  __shared__ int picked[MAX_CAND];
  __shared__ float red[32];
  __shared__ int scan_tmp[RT / 32];
  __shared__ float seg_scores[STAGE_N];
  __shared__ int sel_chunk[64], sel_off[65];
  __shared__ int n_sel;
  // CTA = (query row, segment): with several segments each CTA selects among one slice
  // of the row's chunks and writes local candidates that a merge pass combines
  pdl_launch_dependents();
  pdl_wait();  // the scores and the routing query come from the GEMMs before
  const int S = a.segments > 0 ? a.segments : 1;
  const int b = blockIdx.x;
  const int qb = b / S, seg = b % S;
  const int seg0 = S > 1 ? seg * a.seg_len : 0;
  int c0 = S > 1 ? max(a.ns_start[qb], seg0) : a.ns_start[qb];
  int c1 = S > 1 ? min(a.ns_end[qb], seg0 + a.seg_len) : a.ns_end[qb];
  if constexpr (CHECK) {  // namespace outside the chunk table: record, then clamp it into the table
    if (c1 > c0 && (c0 < 0 || c1 > a.n_chunks)) {
      if (threadIdx.x == 0) bounds_fail(a.bounds, PRA_BOUNDS_ROUTE_NAMESPACE, c0 < 0 ? c0 : c1, a.n_chunks);
      c0 = max(c0, 0);
      c1 = min(c1, a.n_chunks);
    }
  }
  const int n = max(c1 - c0, 0);
  const float* row = a.scores + (int64_t)qb * a.score_stride;
  // chunk id of namespace position c0 + i: through the row's page table (a paged chunk cache,
  // whose rows read scattered pages), else the contiguous range itself
  const int* pages = a.page_table ? a.page_table + (int64_t)qb * a.page_stride : nullptr;
  auto phys = [&](int i) -> int { return pages ? pages[c0 + i] : c0 + i; };
  const int G = a.G > 0 ? a.G : 1;
  // a chunk's score is the best of its G gists' scores (gist aggregation "max")
  auto chunk_score = [&](int c) -> float {
    if (G == 1) return row[c];
    float m = row[(int64_t)c * G];
    for (int g = 1; g < G; ++g) m = fmaxf(m, row[(int64_t)c * G + g]);
    return m;
  };
  // the segment's chunk scores are staged in shared memory once: every radix pass and the
  // candidate scans then read on-chip data (rows longer than STAGE_N read global memory)
  const bool staged = n <= STAGE_N;
  if (staged)
    for (int i = threadIdx.x; i < n; i += RT) seg_scores[i] = chunk_score(phys(i));
  auto score_at = [&](int i) -> float { return staged ? seg_scores[i] : chunk_score(phys(i)); };
  const int kc = min(a.k_cand, min(n, MAX_CAND));
  if (threadIdx.x == 0) {
    prefix = 0;
    prefix_mask = 0;
    need = kc;
    n_cand = 0;
  }
  __syncthreads();
  // phase timestamps of CTA 0 (profiling aid, off unless a trace buffer is given)
  auto mark = [&](int k) {
    if (a.trace != nullptr && blockIdx.x == 0 && threadIdx.x == 0) a.trace[k] = clock64();
  };
  mark(0);
  // 1. radix select (MSB first, 8-bit digits): the kc-th largest approximate score
  for (int shift = 24; shift >= 0 && kc > 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += RT) hist[i] = 0;
    __syncthreads();
    // warp-aggregated histogram: cosine scores share their top bits, so plain per-thread
    // atomics would serialise on one or two bins
    const int lane = threadIdx.x & 31;
    for (int base = threadIdx.x - lane; base < n; base += RT) {
      const int i = base + lane;
      uint32_t digit = 256u;  // "no digit" for lanes past the end or outside the prefix
      if (i < n) {
        const uint32_t key = order_key(score_at(i));
        if ((key & prefix_mask) == prefix) digit = (key >> shift) & 255u;
      }
      const unsigned peers = __match_any_sync(0xffffffffu, digit);
      if (digit < 256u && lane == __ffs(peers) - 1) atomicAdd(&hist[digit], (uint32_t)__popc(peers));
    }
    __syncthreads();
    if (threadIdx.x < 32) {
      // warp 0 finds the digit holding the need-th largest: lane l owns bins 255-8l .. 248-8l
      const int ln = threadIdx.x;
      uint32_t mine = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) mine += hist[255 - 8 * ln - j];
      uint32_t incl = mine;  // inclusive prefix from the top bins down
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (ln >= o) incl += y;
      }
      const int want = need;
      const unsigned hit = __ballot_sync(0xffffffffu, (int)incl >= want);
      const int owner = hit ? __ffs(hit) - 1 : 31;  // the top-down walk always ends by lane 31
      if (ln == owner) {
        int remaining = want - (int)(incl - mine);
        int digit = 255 - 8 * ln;
        for (int j = 0; j < 7; ++j, --digit) {
          if ((int)hist[digit] >= remaining) break;
          remaining -= hist[digit];
        }
        prefix |= (uint32_t)digit << shift;
        prefix_mask |= 255u << shift;
        need = remaining;
      }
    }
    __syncthreads();
  }
  mark(1);
  // 2. candidates: every chunk strictly above the threshold, then ties at it (lowest ids first)
  const uint32_t thr = prefix;
  for (int i = threadIdx.x; i < n && kc > 0; i += RT) {
    if (order_key(score_at(i)) > thr) {
      const int slot = atomicAdd(&n_cand, 1);
      if (slot < MAX_CAND) cand[slot] = phys(i);
    }
  }
  __syncthreads();
  {
    // ties at the threshold, lowest chunk ids first: each thread scans a contiguous segment
    const int above = min(n_cand, MAX_CAND);
    const int seg = (n + RT - 1) / RT;
    const int s0 = min(n, threadIdx.x * seg), s1 = min(n, s0 + seg);
    int mine = 0;
    for (int i = s0; i < s1 && kc > 0; ++i) mine += order_key(score_at(i)) == thr ? 1 : 0;
    int total = 0;
    const int before = block_scan_int(mine, scan_tmp, &total);
    const int want = kc - above;
    int slot = above + before;
    for (int i = s0; i < s1 && kc > 0 && slot < above + want; ++i)
      if (order_key(score_at(i)) == thr) cand[slot++] = phys(i);
    __syncthreads();
    if (threadIdx.x == 0) n_cand = kc > 0 ? above + min(want, total) : 0;
    __syncthreads();
  }
  const int nc = n_cand;
  mark(2);
  // 3. exact fp32 cosine of the candidates: the query staged in shared memory (over the staged
  // scores, no longer read), each warp one candidate at a time with independent 16-byte gist loads
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* qs = seg_scores;
  float sq = 0.f;
  for (int d = threadIdx.x; d < a.D; d += RT) {
    const float v = a.query_bf16 ? __bfloat162float(a.query_bf16[(int64_t)qb * a.query_stride + d])
                                 : a.query[(int64_t)qb * a.query_stride + d];
    qs[d] = v;
    sq += v * v;
  }
  sq = warp_sum(sq);
  if (lane == 0) red[warp] = sq;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < RT / 32; ++w) t += red[w];
    red[0] = 1.f / fmaxf(sqrtf(t), 1e-12f);
  }
  __syncthreads();
  const float qinv = red[0];
  const bool vec = (a.D & 3) == 0 && (reinterpret_cast<uintptr_t>(a.gists) & 15) == 0;
  for (int i = warp; i < nc; i += RT / 32) {
    float best = -INFINITY;
    for (int gi = 0; gi < G; ++gi) {
      const float* g = a.gists + ((int64_t)cand[i] * G + gi) * a.D;
      float acc = 0.f;
      if (vec) {
        const float4* g4 = reinterpret_cast<const float4*>(g);
        const float4* q4 = reinterpret_cast<const float4*>(qs);
#pragma unroll 8
        for (int j = lane; j < a.D / 4; j += 32) {
          const float4 gv = __ldg(g4 + j), qv = q4[j];
          acc += gv.x * qv.x + gv.y * qv.y + gv.z * qv.z + gv.w * qv.w;
        }
      } else {
        for (int d = lane; d < a.D; d += 32) acc += qs[d] * g[d];
      }
      best = fmaxf(best, warp_sum(acc));
    }
    if (lane == 0) cscore[i] = best * qinv;
  }
  __syncthreads();
  if constexpr (EXCH) {
    // 4x. this rank's exact top-k (rank order, global ids) -> every rank; then merge all ranks'
    __shared__ float lcs[64];
    __shared__ int lci[64];
    __shared__ uint32_t s_ep;
    __shared__ int s_ok;
    finish_selection<false>(cscore, cand, nc, 0, a.k, -1, nullptr, nullptr, nullptr, 0, nullptr, nullptr, lcs, lci,
                            a.id_offset, picked, sel_chunk, sel_off, &n_sel, -1, nullptr);
    if (threadIdx.x == 0) {
      s_ep = x.epochs[qb] + 1;
      x.epochs[qb] = s_ep;
      s_ok = 1;
    }
    __syncthreads();
    const uint32_t ep = s_ep;
    const int half = (int)(ep & 1u), K2 = 2 * a.k;
    for (int t = threadIdx.x; t < x.world * K2; t += RT) {
      const int pr = t / K2, i = t % K2;
      const float v = i < a.k ? lcs[i] : __int_as_float(lci[i - a.k]);
      x.recv[pr][(((int64_t)half * x.B_max + qb) * x.world + x.rank) * K2 + i] = v;
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x < x.world) {
      signal_release(x.flags[threadIdx.x] + qb * x.world + x.rank, ep);
      if (!bounded_wait_geq(x.flags[x.rank] + qb * x.world + threadIdx.x, ep, x.max_spins)) {
        s_ok = 0;
        atomicExch(x.error, 1);
      }
    }
    if (threadIdx.x == 0) n_cand = 0;
    __syncthreads();
    if (!s_ok) {  // a peer never delivered: no memory for this row (the error flag tells the host)
      if (threadIdx.x == 0) a.mem_len[qb] = 0;
      for (int i = threadIdx.x; i < a.k && a.sel_out; i += RT) a.sel_out[(int64_t)qb * a.k + i] = -1;
      return;
    }
    for (int t = threadIdx.x; t < x.world * a.k; t += RT) {
      const int pr = t / a.k, i = t % a.k;
      const float* src = x.recv[x.rank] + (((int64_t)half * x.B_max + qb) * x.world + pr) * K2;
      const int id = __float_as_int(__ldcv(src + a.k + i));
      if (id >= 0) {
        const int slot = atomicAdd(&n_cand, 1);
        cand[slot] = id;
        cscore[slot] = __ldcv(src + i);
      }
    }
    __syncthreads();
    finish_selection<CHECK>(cscore, cand, n_cand, qb, a.k, a.budget, x.global_len, x.global_row0, a.mem_idx,
                            a.mem_max, a.mem_len, a.sel_out, nullptr, nullptr, 0, picked, sel_chunk, sel_off, &n_sel,
                            a.pool_rows, a.bounds);
    return;
  }
  mark(3);
  // 4. top-k by (-score, chunk id) (+ greedy budget, chunk order and the row list)
  finish_selection<CHECK>(cscore, cand, nc, b, a.k, a.budget, a.chunk_len, a.chunk_row0, a.mem_idx, a.mem_max,
                          a.mem_len, a.sel_out, a.cand_score, a.cand_id, a.id_offset, picked, sel_chunk, sel_off,
                          &n_sel, a.pool_rows, a.bounds);
  mark(4);
}

// Cross-GPU merge of the per-rank candidates: row b holds world blocks of [k scores | k ids
// (int bits)] (rank-major, as the column all-gather leaves them).
template <bool CHECK>
__global__ void __launch_bounds__(256) route_merge_kernel(RouteMergeArgs a) {
  __shared__ int cand[MAX_CAND];
  __shared__ float cscore[MAX_CAND];
  __shared__ int picked[MAX_CAND];
  __shared__ int sel_chunk[64], sel_off[65];
  __shared__ int n_sel;
  __shared__ int nc_s;
  const int b = blockIdx.x;
  const float* row = a.cands + (int64_t)b * a.row_stride;
  if (threadIdx.x == 0) nc_s = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < a.world * a.k; i += blockDim.x) {
    const int r = i / a.k, j = i % a.k;
    const float sc = row[r * 2 * a.k + j];
    const int id = __float_as_int(row[r * 2 * a.k + a.k + j]);
    if (CHECK && id >= a.n_chunks) {  // a rank sent a chunk id outside the table: record, drop it
      bounds_fail(a.bounds, PRA_BOUNDS_ROUTE_CHUNK, id, a.n_chunks);
      continue;
    }
    if (id >= 0) {
      const int slot = atomicAdd(&nc_s, 1);
      if (slot < MAX_CAND) {
        cand[slot] = id;
        cscore[slot] = sc;
      }
    }
  }
  __syncthreads();
  const int nc = min(nc_s, MAX_CAND);
  finish_selection<CHECK>(cscore, cand, nc, b, a.k, a.budget, a.chunk_len, a.chunk_row0, a.mem_idx, a.mem_max,
                          a.mem_len, a.sel_out, a.cand_score, a.cand_id, 0, picked, sel_chunk, sel_off, &n_sel,
                          a.pool_rows, a.bounds);
}

// Combine per-rank attention partials: parts [B, world, H, D + 2] (unnormalised out, max,
// sum; max in natural-log units) -> out [B, H * D] bf16.
__global__ void combine_partials_kernel(const float* __restrict__ parts, int world, int H, int D,
                                        __nv_bfloat16* __restrict__ out) {
  const int b = blockIdx.x / H, h = blockIdx.x % H;
  const int64_t stride_r = (int64_t)H * (D + 2);
  const float* base = parts + (int64_t)b * world * stride_r + (int64_t)h * (D + 2);
  float M = -INFINITY;
  for (int r = 0; r < world; ++r) M = fmaxf(M, base[r * stride_r + D]);
  float L = 0.f;
  for (int r = 0; r < world; ++r) {
    const float m = base[r * stride_r + D];
    if (m != -INFINITY) L += base[r * stride_r + D + 1] * __expf(m - M);
  }
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
    for (int r = 0; r < world; ++r) {
      const float m = base[r * stride_r + D];
      if (m != -INFINITY) acc += base[r * stride_r + d] * __expf(m - M);
    }
    out[(int64_t)b * H * D + h * D + d] = __float2bfloat16(L > 0.f ? acc / L : 0.f);
  }
}

}  // namespace llama
}  // namespace pra

cudaError_t pra_rope_copy(const RopeCopyArgs& a, cudaStream_t st) {
  if (a.M == 0) return cudaSuccess;
  const int pairs = a.heads * (a.head_dim / 2);
  const int threads = 256;
  dim3 grid(a.M, (pairs + threads - 1) / threads);
  pra::llama::rope_copy_kernel<<<grid, threads, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t pra_decode_prologue(const DecodePrologueArgs& a, cudaStream_t st) {
  if (a.B == 0) return cudaSuccess;
  if (a.d % 8 || (reinterpret_cast<uintptr_t>(a.embed) | reinterpret_cast<uintptr_t>(a.x)) & 15)
    return cudaErrorInvalidValue;
  return pra_launch_pdl(pra::llama::decode_prologue_kernel, dim3(a.B), dim3(128), 0, st, a);
}

cudaError_t pra_silu_mul(const __nv_bfloat16* gate_up, int64_t M, int F, int block, __nv_bfloat16* out,
                         cudaStream_t st) {
  if (M == 0) return cudaSuccess;
  if (F % 2) return cudaErrorInvalidValue;
  const int64_t pairs = M * (F / 2);
  const int64_t want = (pairs + 255) / 256;
  const int blocks = (int)(want < 148 * 16 ? want : 148 * 16);
  if (block < 0 || (block > 0 && (F % block || block % 2))) return cudaErrorInvalidValue;
  PRA_RETURN_IF_ERROR(
      pra_launch_pdl(pra::llama::silu_mul_kernel, dim3(blocks), dim3(256), 0, st, gate_up, M, F, block, out));
  return cudaGetLastError();
}

template <int D>
static cudaError_t launch_decode(DecodeAttnParams p, cudaStream_t st) {
  using namespace pra::llama;
  constexpr int LD = DSmem<D>::LD;
  static_assert(2 * DSTAGES * DBN * LD * sizeof(__nv_bfloat16) >= 4 * 16 * (D + 2) * sizeof(float),
                "merge buffer must fit in the staging area");
  const size_t smem = (size_t)(16 + 2 * DSTAGES * DBN) * LD * sizeof(__nv_bfloat16) + (size_t)p.split_keys * sizeof(int);
  const dim3 grid(p.B * p.Hkv, p.split_count > 0 ? p.split_count : p.n_split);
  if (p.phase != 2) {
    if (p.bounds != nullptr) {
      PRA_RETURN_IF_ERROR(pra::set_max_dynamic_smem(reinterpret_cast<const void*>(decode_kernel<D, true>), (int)smem));
      decode_kernel<D, true><<<grid, DT, smem, st>>>(p);
    } else {
      PRA_RETURN_IF_ERROR(pra::set_max_dynamic_smem(reinterpret_cast<const void*>(decode_kernel<D, false>), (int)smem));
      decode_kernel<D, false><<<grid, DT, smem, st>>>(p);
    }
    PRA_RETURN_IF_ERROR(cudaGetLastError());
  }
  if (p.phase != 1) decode_merge_kernel<<<p.B * p.H, 128, 0, st>>>(p, D);
  return cudaGetLastError();
}

static int g_decode_tma = 1;
static int g_pdl = 1;
void pra_set_pdl(int on) { g_pdl = on ? 1 : 0; }
int pra_pdl_enabled() { return g_pdl; }
static thread_local int g_launch_priority = 0;
void pra_set_launch_priority(int high) {
  int least = 0, greatest = 0;
  if (high && cudaDeviceGetStreamPriorityRange(&least, &greatest) == cudaSuccess) g_launch_priority = greatest;
  else g_launch_priority = 0;
}
int pra_launch_priority() { return g_launch_priority; }
static int g_decode_stages = pra::llama::TST_DEFAULT;
void pra_decode_set_tma(int on) { g_decode_tma = on; }
void pra_decode_set_stages(int stages) { g_decode_stages = stages; }

template <int D, int TST>
static cudaError_t launch_decode_tma_stages(const DecodeAttnParams& p, const CUtensorMap* mk, const CUtensorMap* mv,
                                            const CUtensorMap* lk, const CUtensorMap* lv, cudaStream_t st) {
  using namespace pra::llama;
  using Lay = TLayout<D>;
  const size_t smem = 1024 + (size_t)TST * Lay::STAGE + 16 * Lay::QLD * 2 + (size_t)(p.split_keys + 2 * TMAX_BLOCKS) * 4 +
                      TST * 8;
  PRA_RETURN_IF_ERROR(pra::set_max_dynamic_smem(reinterpret_cast<const void*>(decode_tma_kernel<D, TST>), (int)smem));
  const int count = p.split_count > 0 ? p.split_count : p.n_split;
  const int items = p.B * p.Hkv * count;
  const dim3 grid = p.max_ctas > 0 ? dim3(std::min(items, p.max_ctas)) : dim3(p.B * p.Hkv, count);
  PRA_RETURN_IF_ERROR(pra_launch_pdl(decode_tma_kernel<D, TST>, grid, dim3(DT), smem, st, *mk, *mv, *lk, *lv, p));
  return cudaGetLastError();
}

// The TMA-fed kernel, or cudaErrorNotSupported when a layout or option rules it out.
template <int D>
static cudaError_t launch_decode_tma(const DecodeAttnParams& p, cudaStream_t st) {
  using namespace pra::llama;
  const auto aligned = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  const bool has_mem = p.mem_idx != nullptr;
  if (!g_decode_tma || p.bounds != nullptr || p.loc_k == nullptr || p.loc_row % 8 || p.loc_batch % p.loc_row ||
      !aligned(p.loc_k) || !aligned(p.loc_v) || (has_mem && (!p.mem_on_device || p.mem_row % 8 || !aligned(p.mem_k) ||
                                                               !aligned(p.mem_v) || p.mem_rows <= 0)))
    return cudaErrorNotSupported;
  const int64_t width = (int64_t)p.Hkv * D;
  const int64_t loc_rows = (int64_t)p.B * (p.loc_batch / p.loc_row);
  const CUtensorMap* lk = pra_tile_map_bf16(p.loc_k, width, loc_rows, p.loc_row, DBN);
  const CUtensorMap* lv = pra_tile_map_bf16(p.loc_v, width, loc_rows, p.loc_row, DBN);
  const CUtensorMap* mk = has_mem ? pra_tile_map_bf16(p.mem_k, width, p.mem_rows, p.mem_row, DBN) : lk;
  const CUtensorMap* mv = has_mem ? pra_tile_map_bf16(p.mem_v, width, p.mem_rows, p.mem_row, DBN) : lv;
  if (!lk || !lv || !mk || !mv) return cudaErrorNotSupported;
  if (p.phase != 2) {
    if (g_decode_stages == 2) PRA_RETURN_IF_ERROR((launch_decode_tma_stages<D, 2>(p, mk, mv, lk, lv, st)));
    else if (g_decode_stages == 4) PRA_RETURN_IF_ERROR((launch_decode_tma_stages<D, 4>(p, mk, mv, lk, lv, st)));
    else PRA_RETURN_IF_ERROR((launch_decode_tma_stages<D, 3>(p, mk, mv, lk, lv, st)));
  }
  if (p.phase != 1) PRA_RETURN_IF_ERROR(pra_launch_pdl(decode_merge_kernel, dim3(p.B * p.H), dim3(128), 0, st, p, D));
  return cudaGetLastError();
}

cudaError_t pra_decode_attention(const DecodeAttnParams& p, int head_dim, cudaStream_t st) {
  if (p.B == 0) return cudaSuccess;
  if (p.H % p.Hkv || p.H / p.Hkv > 16 || p.split_keys % pra::llama::DBN || p.split_keys > 4096)
    return cudaErrorInvalidValue;
  const int count = p.split_count > 0 ? p.split_count : p.n_split;
  if (p.mem_splits < 0 || p.mem_splits > p.n_split || p.split_lo < 0 || p.split_lo + count > p.n_split ||
      p.phase < 0 || p.phase > 2 || p.mem_split_keys < 0 || p.mem_split_keys % pra::llama::DBN ||
      p.mem_split_keys > p.split_keys)
    return cudaErrorInvalidValue;
  cudaError_t e = cudaErrorNotSupported;
  if (head_dim == 128) e = launch_decode_tma<128>(p, st);
  else if (head_dim == 64) e = launch_decode_tma<64>(p, st);
  if (e != cudaErrorNotSupported) return e;
  switch (head_dim) {
    case 64: return launch_decode<64>(p, st);
    case 128: return launch_decode<128>(p, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t pra_combine_partials(const float* parts, int B, int world, int H, int D, __nv_bfloat16* out,
                                 cudaStream_t st) {
  if (B == 0) return cudaSuccess;
  pra::llama::combine_partials_kernel<<<B * H, 128, 0, st>>>(parts, world, H, D, out);
  return cudaGetLastError();
}

cudaError_t pra_route_merge(const RouteMergeArgs& a, cudaStream_t st) {
  if (a.B == 0) return cudaSuccess;
  if (a.k > 64 || a.world * a.k > pra::llama::MAX_CAND) return cudaErrorInvalidValue;
  if (a.bounds != nullptr) pra::llama::route_merge_kernel<true><<<a.B, 256, 0, st>>>(a);
  else pra::llama::route_merge_kernel<false><<<a.B, 256, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t pra_route_topk(const RouteTopkArgs& a, cudaStream_t st) {
  if (a.B == 0) return cudaSuccess;
  if (a.k > 64 || a.k_cand > pra::llama::MAX_CAND || a.D > pra::llama::STAGE_N) return cudaErrorInvalidValue;
  const int S = a.segments > 0 ? a.segments : 1;
  if (S > 1 && (a.cand_score == nullptr || a.seg_len <= 0)) return cudaErrorInvalidValue;  // segments need a merge
  const RouteExchangeArgs none{};
  if (a.bounds != nullptr)
    PRA_RETURN_IF_ERROR(pra_launch_pdl(pra::llama::route_topk_kernel<true, false>, dim3(a.B * S), dim3(pra::llama::RT),
                                       0, st, a, none));
  else
    PRA_RETURN_IF_ERROR(pra_launch_pdl(pra::llama::route_topk_kernel<false, false>, dim3(a.B * S),
                                       dim3(pra::llama::RT), 0, st, a, none));
  return cudaGetLastError();
}

cudaError_t pra_route_topk_exchange(const RouteTopkArgs& a, const RouteExchangeArgs& x, cudaStream_t st) {
  if (a.B == 0) return cudaSuccess;
  if (a.k > 64 || a.k_cand > pra::llama::MAX_CAND || a.D > pra::llama::STAGE_N || a.segments > 1 || x.world < 2 ||
      x.world > TP_MAX_RANKS ||
      x.world * a.k > pra::llama::MAX_CAND || a.B > x.B_max || x.rank < 0 || x.rank >= x.world || !x.epochs ||
      !x.error || !x.global_len || !x.global_row0 || !a.mem_idx || !a.mem_len)
    return cudaErrorInvalidValue;
  for (int p = 0; p < x.world; ++p)
    if (!x.recv[p] || !x.flags[p]) return cudaErrorInvalidValue;
  if (a.bounds != nullptr)
    PRA_RETURN_IF_ERROR(pra_launch_pdl(pra::llama::route_topk_kernel<true, true>, dim3(a.B), dim3(pra::llama::RT), 0,
                                       st, a, x));
  else
    PRA_RETURN_IF_ERROR(pra_launch_pdl(pra::llama::route_topk_kernel<false, true>, dim3(a.B), dim3(pra::llama::RT), 0,
                                       st, a, x));
  return cudaGetLastError();
}
