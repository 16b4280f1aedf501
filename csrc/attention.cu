// Ragged native-K/V attention for PRA: one softmax over
//   [ selected memory keys (gathered from a token pool, fully visible) ;
//     local keys (causal, optional key-padding mask) ]
// Forward (with log-sum-exp) and a deterministic two-kernel backward
// (dQ over all key blocks; dK/dV over local key blocks, each warp owning 16
// keys), bf16 tensor-core tiles with fp32 softmax / accumulators.
//
// Layouts: q/k/v/o rows are tokens ([B, T] rows with arbitrary row stride, heads
// contiguous at h*Dh), the memory pools are [tokens, Hkv*Dh] rows addressed by
// a per-row index list (mem_idx[b, j], j < mem_len[b]).  GQA maps query head h
// to kv head h / (H / Hkv).
#include "common.cuh"

namespace pra {
namespace attn {

constexpr int BM = 64;   // queries per CTA (16 per warp)
constexpr int BN = 64;   // keys per block
constexpr int NT = 128;  // threads per CTA
constexpr float LOG2E = 1.4426950408889634f;

using Params = AttnParams;

template <int D>
struct Smem {
  static constexpr int LD = D + 8;  // padded row (16 bytes) against ldmatrix bank conflicts
};

// Load `rows` x D bf16 rows into smem (row pitch LD); row r's global address from `addr(r)`.
template <int D, typename AddrFn>
__device__ __forceinline__ void load_tile(__nv_bfloat16* smem, const __nv_bfloat16* safe, AddrFn addr) {
  constexpr int LD = Smem<D>::LD;
  constexpr int CHUNKS = BN * D / 8;  // 16-byte chunks
#pragma unroll
  for (int c = threadIdx.x; c < CHUNKS; c += NT) {
    const int r = c / (D / 8), col = (c % (D / 8)) * 8;
    const __nv_bfloat16* src = addr(r);
    cp_async16(smem + r * LD + col, src ? src + col : safe, src != nullptr);
  }
}

// Warp computes acc[16 x 64] += A[16 x D] * B[64 x D]^T with A rows at `a_sm`
// (warp's 16 rows) and B rows at `b_sm` (64 rows); both row-major in smem.
template <int D>
__device__ __forceinline__ void mma_abt(float (&acc)[8][4], const __nv_bfloat16* a_sm, const __nv_bfloat16* b_sm) {
  constexpr int LD = Smem<D>::LD;
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    uint32_t a[4];
    ldmatrix_x4(a, smem_u32(a_sm + (lane & 15) * LD + kk * 16 + (lane >> 4) * 8));
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      uint32_t b[4];
      const int row = np * 16 + ((lane >> 4) & 1) * 8 + (lane & 7);
      ldmatrix_x4(b, smem_u32(b_sm + row * LD + kk * 16 + ((lane >> 3) & 1) * 8));
      mma_bf16_16816(acc[2 * np], a, b);
      mma_bf16_16816(acc[2 * np + 1], a, b + 2);
    }
  }
}

// Warp computes out[16 x D] += P[16 x 64] * B[64 x D], P given as fp32 accumulator
// fragments (converted to bf16 A fragments), B rows (64 keys) row-major in smem.
template <int D>
__device__ __forceinline__ void mma_pb(float (&out)[D / 8][4], const float (&p)[8][4], const __nv_bfloat16* b_sm) {
  constexpr int LD = Smem<D>::LD;
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int kc = 0; kc < 4; ++kc) {
    uint32_t a[4];
    a[0] = pack_bf16(p[2 * kc][0], p[2 * kc][1]);
    a[1] = pack_bf16(p[2 * kc][2], p[2 * kc][3]);
    a[2] = pack_bf16(p[2 * kc + 1][0], p[2 * kc + 1][1]);
    a[3] = pack_bf16(p[2 * kc + 1][2], p[2 * kc + 1][3]);
#pragma unroll
    for (int np = 0; np < D / 16; ++np) {
      uint32_t b[4];
      const int m = lane >> 3;
      const int row = kc * 16 + (m & 1) * 8 + (lane & 7);
      ldmatrix_x4_trans(b, smem_u32(b_sm + row * LD + np * 16 + (m >> 1) * 8));
      mma_bf16_16816(out[2 * np], a, b);
      mma_bf16_16816(out[2 * np + 1], a, b + 2);
    }
  }
}

struct KeyBlock {
  bool memory;
  int start;  // first key index (memory position or local token)
};

__device__ __forceinline__ KeyBlock key_block(int i, int n_mem_blocks) {
  return i < n_mem_blocks ? KeyBlock{true, i * BN} : KeyBlock{false, (i - n_mem_blocks) * BN};
}

// svalid: the block's key-padding mask staged in shared memory (null without a mask).
__device__ __forceinline__ bool key_visible(const Params& p, const KeyBlock& kb, int key_off, int query, int mem_len,
                                            const uint8_t* svalid) {
  const int key = kb.start + key_off;
  if (kb.memory) return key < mem_len;
  if (key >= p.T || key > query) return false;
  return svalid == nullptr || svalid[key_off] != 0;
}

// True when every key of the block is visible to every query row >= q0 (no masking needed).
__device__ __forceinline__ bool block_unmasked(const Params& p, const KeyBlock& kb, int q0, int mem_len) {
  if (kb.memory) return kb.start + BN <= mem_len;
  return p.key_valid == nullptr && kb.start + BN - 1 <= q0 && kb.start + BN <= p.T;
}

template <int D>
__device__ __forceinline__ void load_keys(const Params& p, __nv_bfloat16* sk, __nv_bfloat16* sv, uint8_t* svalid,
                                          int b, int kvh, const KeyBlock& kb, int mem_len) {
  if (!kb.memory && p.key_valid != nullptr && threadIdx.x < BN) {
    const int t = kb.start + threadIdx.x;
    svalid[threadIdx.x] = t < p.T ? p.key_valid[(int64_t)b * p.T + t] : 0;
  }
  if (kb.memory) {
    const int* idx = p.mem_idx + (int64_t)b * p.mem_max;
    load_tile<D>(sk, p.mem_k, [&](int r) -> const __nv_bfloat16* {
      const int j = kb.start + r;
      return j < mem_len ? p.mem_k + (int64_t)idx[j] * p.mem_row + kvh * D : nullptr;
    });
    load_tile<D>(sv, p.mem_v, [&](int r) -> const __nv_bfloat16* {
      const int j = kb.start + r;
      return j < mem_len ? p.mem_v + (int64_t)idx[j] * p.mem_row + kvh * D : nullptr;
    });
  } else {
    load_tile<D>(sk, p.k, [&](int r) -> const __nv_bfloat16* {
      const int t = kb.start + r;
      return t < p.T ? p.k + b * p.k_batch + t * p.k_row + kvh * D : nullptr;
    });
    load_tile<D>(sv, p.v, [&](int r) -> const __nv_bfloat16* {
      const int t = kb.start + r;
      return t < p.T ? p.v + b * p.v_batch + t * p.v_row + kvh * D : nullptr;
    });
  }
}

// Dropout element id of probability (b, h, query q, local key t): a flat index over [B, H, T, T].
__device__ __forceinline__ uint64_t drop_elem(const Params& p, int b, int h, int q, int t) {
  return (((uint64_t)b * p.H + h) * p.T + q) * p.T + t;
}

template <int D>
__global__ void __launch_bounds__(NT) fwd_kernel(Params p) {
  constexpr int LD = Smem<D>::LD;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __nv_bfloat16* sq = reinterpret_cast<__nv_bfloat16*>(smem_raw);
  __nv_bfloat16* sk = sq + BM * LD;   // [2][BN][LD]
  __nv_bfloat16* sv = sk + 2 * BN * LD;
  uint8_t* svalid = reinterpret_cast<uint8_t*>(sv + 2 * BN * LD);  // [2][BN]

  // grid (H * B, query blocks): the longest (last, causal) query blocks are scheduled first
  const int h = blockIdx.x % p.H, b = blockIdx.x / p.H;
  const int qb = gridDim.y - 1 - blockIdx.y;
  const int kvh = h / (p.H / p.Hkv);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = qb * BM;
  const int mem_len = p.mem_len ? p.mem_len[b] : 0;
  const int n_mem = (mem_len + BN - 1) / BN;
  const int q_last = min(q0 + BM, p.T) - 1;
  const int n_loc = q_last / BN + 1;
  const int n_blocks = n_mem + n_loc;

  load_tile<D>(sq, p.q, [&](int r) -> const __nv_bfloat16* {
    const int t = q0 + r;
    return t < p.T ? p.q + b * p.q_batch + t * p.q_row + h * D : nullptr;
  });
  load_keys<D>(p, sk, sv, svalid, b, kvh, key_block(0, n_mem), mem_len);
  cp_async_commit();

  float o_acc[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o_acc[i][0] = o_acc[i][1] = o_acc[i][2] = o_acc[i][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  const float sl2 = p.scale * LOG2E;
  const int row_a = q0 + warp * 16 + (lane >> 2);

  for (int it = 0; it < n_blocks; ++it) {
    const int buf = it & 1;
    if (it + 1 < n_blocks) {
      load_keys<D>(p, sk + (buf ^ 1) * BN * LD, sv + (buf ^ 1) * BN * LD, svalid + (buf ^ 1) * BN, b, kvh,
                   key_block(it + 1, n_mem), mem_len);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const KeyBlock kb = key_block(it, n_mem);
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
    mma_abt<D>(s, sq + warp * 16 * LD, sk + buf * BN * LD);
    float mx[2] = {-INFINITY, -INFINITY};
    const bool unmasked = block_unmasked(p, kb, q0, mem_len);
    const uint8_t* valid = p.key_valid ? svalid + buf * BN : nullptr;
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int q = row_a + (e >> 1) * 8;
        const int key_off = nb * 8 + (lane & 3) * 2 + (e & 1);
        if (!unmasked && !key_visible(p, kb, key_off, q, mem_len, valid)) s[nb][e] = -INFINITY;
        mx[e >> 1] = fmaxf(mx[e >> 1], s[nb][e]);
      }
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
        o_acc[i][2 * r] *= corr;
        o_acc[i][2 * r + 1] *= corr;
      }
    }
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = e >> 1;
        const float v = (m_run[r] == -INFINITY) ? 0.f : exp2f((s[nb][e] - m_run[r]) * sl2);
        s[nb][e] = v;
        rs[r] += v;
      }
    }
    l_run[0] += rs[0];
    l_run[1] += rs[1];
    if (p.drop_thresh != 0) {  // the normaliser keeps every probability; P V uses the dropped ones
#pragma unroll
      for (int nb = 0; nb < 8; ++nb)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int q = row_a + (e >> 1) * 8;
          const int t = kb.start + nb * 8 + (lane & 3) * 2 + (e & 1);
          const bool keep = q < p.T && t < p.T &&
                            dropout_keep(p.drop_seed, p.drop_offset, drop_elem(p, b, h, q, t), p.drop_thresh);
          s[nb][e] = keep ? s[nb][e] * p.drop_scale : 0.f;
        }
    }
    mma_pb<D>(o_acc, s, sv + buf * BN * LD);
    __syncthreads();
  }

#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 1);
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 2);
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int t = row_a + r * 8;
    if (t >= p.T) continue;
    const float inv = l_run[r] > 0.f ? 1.f / l_run[r] : 0.f;
    __nv_bfloat16* dst = p.o + b * p.o_batch + t * p.o_row + h * D;
#pragma unroll
    for (int nb = 0; nb < D / 8; ++nb) {
      const int col = nb * 8 + (lane & 3) * 2;
      *reinterpret_cast<__nv_bfloat162*>(dst + col) =
          __floats2bfloat162_rn(o_acc[nb][2 * r] * inv, o_acc[nb][2 * r + 1] * inv);
    }
    if ((lane & 3) == 0) {
      p.lse[((int64_t)b * p.H + h) * p.T + t] =
          l_run[r] > 0.f ? m_run[r] * p.scale + logf(l_run[r]) : -INFINITY;
    }
  }
}

// delta[b,h,t] = sum_d dO * O with 16-byte loads: D / 8 consecutive lanes cover one head
// (D / 8 <= 32), so a warp covers 256 / D (b, t, h) rows; reduction within each lane group.
template <int D>
__global__ void delta_vec_kernel(Params p) {
  constexpr int L = D / 8;  // lanes per (b, t, h) row
  const int64_t gt = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = (int64_t)p.B * p.T * p.H;
  const int64_t item = gt / L;
  const int part = (int)(gt % L);
  float acc = 0.f;
  if (item < total) {
    const int h = item % p.H, t = (item / p.H) % p.T, b = item / ((int64_t)p.H * p.T);
    const uint4 ov = *reinterpret_cast<const uint4*>(p.o + b * p.o_batch + (int64_t)t * p.o_row + h * D + part * 8);
    const uint4 gv = *reinterpret_cast<const uint4*>(p.dout + b * p.do_batch + (int64_t)t * p.do_row + h * D + part * 8);
    const __nv_bfloat162* oh = reinterpret_cast<const __nv_bfloat162*>(&ov);
    const __nv_bfloat162* gh = reinterpret_cast<const __nv_bfloat162*>(&gv);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 a = __bfloat1622float2(oh[k]), c = __bfloat1622float2(gh[k]);
      acc += a.x * c.x + a.y * c.y;
    }
  }
#pragma unroll
  for (int o = L / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (item < total && part == 0) {
    const int h = item % p.H, t = (item / p.H) % p.T, b = item / ((int64_t)p.H * p.T);
    p.delta[((int64_t)b * p.H + h) * p.T + t] = acc;
  }
}

// delta[b,h,t] = sum_d dO * O   (one warp per (b, t, h))
template <int D>
__global__ void delta_kernel(Params p) {
  const int64_t gw = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int64_t total = (int64_t)p.B * p.T * p.H;
  if (gw >= total) return;
  const int h = gw % p.H, t = (gw / p.H) % p.T, b = gw / ((int64_t)p.H * p.T);
  const __nv_bfloat16* o = p.o + b * p.o_batch + t * p.o_row + h * D;
  const __nv_bfloat16* g = p.dout + b * p.do_batch + t * p.do_row + h * D;
  float acc = 0.f;
  for (int d = lane * 2; d < D; d += 64) {
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(o + d));
    const float2 c = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(g + d));
    acc += a.x * c.x + a.y * c.y;
  }
  acc = warp_sum(acc);
  if (lane == 0) p.delta[((int64_t)b * p.H + h) * p.T + t] = acc;
}

template <int D>
__global__ void __launch_bounds__(NT) bwd_dq_kernel(Params p) {
  constexpr int LD = Smem<D>::LD;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __nv_bfloat16* sq = reinterpret_cast<__nv_bfloat16*>(smem_raw);
  __nv_bfloat16* sdo = sq + BM * LD;
  __nv_bfloat16* sk = sdo + BM * LD;  // [2][BN][LD]
  __nv_bfloat16* sv = sk + 2 * BN * LD;
  uint8_t* svalid = reinterpret_cast<uint8_t*>(sv + 2 * BN * LD);  // [2][BN]

  // grid (H * B, query blocks): the longest (last, causal) query blocks are scheduled first
  const int h = blockIdx.x % p.H, b = blockIdx.x / p.H;
  const int qb = gridDim.y - 1 - blockIdx.y;
  const int kvh = h / (p.H / p.Hkv);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = qb * BM;
  const int mem_len = p.mem_len ? p.mem_len[b] : 0;
  const int n_mem = (mem_len + BN - 1) / BN;
  const int n_loc = (min(q0 + BM, p.T) - 1) / BN + 1;
  const int n_blocks = n_mem + n_loc;
  load_tile<D>(sq, p.q, [&](int r) -> const __nv_bfloat16* {
    const int t = q0 + r;
    return t < p.T ? p.q + b * p.q_batch + t * p.q_row + h * D : nullptr;
  });
  load_tile<D>(sdo, p.dout, [&](int r) -> const __nv_bfloat16* {
    const int t = q0 + r;
    return t < p.T ? p.dout + b * p.do_batch + t * p.do_row + h * D : nullptr;
  });
  load_keys<D>(p, sk, sv, svalid, b, kvh, key_block(0, n_mem), mem_len);
  cp_async_commit();

  const int row_a = q0 + warp * 16 + (lane >> 2);
  float lse2[2], dlt[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int t = row_a + r * 8;
    const int64_t at = ((int64_t)b * p.H + h) * p.T + t;
    lse2[r] = t < p.T ? p.lse[at] * LOG2E : -INFINITY;
    dlt[r] = t < p.T ? p.delta[at] : 0.f;
  }
  const float sl2 = p.scale * LOG2E;
  float dq[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;

  for (int it = 0; it < n_blocks; ++it) {
    const int buf = it & 1;
    if (it + 1 < n_blocks) {
      load_keys<D>(p, sk + (buf ^ 1) * BN * LD, sv + (buf ^ 1) * BN * LD, svalid + (buf ^ 1) * BN, b, kvh,
                   key_block(it + 1, n_mem), mem_len);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const KeyBlock kb = key_block(it, n_mem);
    float s[8][4], dp[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
      dp[i][0] = dp[i][1] = dp[i][2] = dp[i][3] = 0.f;
    }
    mma_abt<D>(s, sq + warp * 16 * LD, sk + buf * BN * LD);
    mma_abt<D>(dp, sdo + warp * 16 * LD, sv + buf * BN * LD);
    const bool unmasked = block_unmasked(p, kb, q0, mem_len);
    const uint8_t* valid = p.key_valid ? svalid + buf * BN : nullptr;
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = e >> 1;
        const int q = row_a + r * 8;
        const int key_off = nb * 8 + (lane & 3) * 2 + (e & 1);
        const bool vis = (unmasked || key_visible(p, kb, key_off, q, mem_len, valid)) && lse2[r] != -INFINITY;
        const float pr = vis ? exp2f(s[nb][e] * sl2 - lse2[r]) : 0.f;
        float dpv = dp[nb][e];
        if (p.drop_thresh != 0) {  // dP of the dropped probabilities -> dP of the kept ones
          const int t = kb.start + key_off;
          const bool keep = vis && dropout_keep(p.drop_seed, p.drop_offset, drop_elem(p, b, h, q, t), p.drop_thresh);
          dpv = keep ? dpv * p.drop_scale : 0.f;
        }
        s[nb][e] = pr * (dpv - dlt[r]);  // dS (unscaled)
      }
    }
    mma_pb<D>(dq, s, sk + buf * BN * LD);
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int t = row_a + r * 8;
    if (t >= p.T) continue;
    __nv_bfloat16* dst = p.dq + b * p.dq_batch + t * p.dq_row + h * D;
#pragma unroll
    for (int nb = 0; nb < D / 8; ++nb) {
      const int col = nb * 8 + (lane & 3) * 2;
      *reinterpret_cast<__nv_bfloat162*>(dst + col) =
          __floats2bfloat162_rn(dq[nb][2 * r] * p.scale, dq[nb][2 * r + 1] * p.scale);
    }
  }
}

// dK/dV for one 64-key block of the local sequence; iterates query blocks that
// can see it (causal).  Each warp owns 16 keys.  MHA only (H == Hkv).
template <int D>
__global__ void __launch_bounds__(NT) bwd_dkdv_kernel(Params p) {
  constexpr int LD = Smem<D>::LD;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __nv_bfloat16* sk = reinterpret_cast<__nv_bfloat16*>(smem_raw);
  __nv_bfloat16* sv = sk + BN * LD;
  __nv_bfloat16* sq = sv + BN * LD;    // [2][BM][LD]
  __nv_bfloat16* sdo = sq + 2 * BM * LD;
  float* s_lse = reinterpret_cast<float*>(sdo + 2 * BM * LD);  // [2][BM]
  float* s_dlt = s_lse + 2 * BM;

  // grid (H * B, key blocks): the first key blocks (seen by the most queries) are scheduled first
  const int h = blockIdx.x % p.H, b = blockIdx.x / p.H;
  const int kblk = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int k0 = kblk * BN;
  const int n_q = (p.T + BM - 1) / BM;
  const int first_q = k0 / BM;
  load_tile<D>(sk, p.k, [&](int r) -> const __nv_bfloat16* {
    const int t = k0 + r;
    return t < p.T ? p.k + b * p.k_batch + t * p.k_row + h * D : nullptr;
  });
  load_tile<D>(sv, p.v, [&](int r) -> const __nv_bfloat16* {
    const int t = k0 + r;
    return t < p.T ? p.v + b * p.v_batch + t * p.v_row + h * D : nullptr;
  });
  auto load_q = [&](int qi, int buf) {
    const int qs = qi * BM;
    load_tile<D>(sq + buf * BM * LD, p.q, [&](int r) -> const __nv_bfloat16* {
      const int t = qs + r;
      return t < p.T ? p.q + b * p.q_batch + t * p.q_row + h * D : nullptr;
    });
    load_tile<D>(sdo + buf * BM * LD, p.dout, [&](int r) -> const __nv_bfloat16* {
      const int t = qs + r;
      return t < p.T ? p.dout + b * p.do_batch + t * p.do_row + h * D : nullptr;
    });
    for (int r = threadIdx.x; r < BM; r += NT) {
      const int t = qs + r;
      const int64_t at = ((int64_t)b * p.H + h) * p.T + t;
      s_lse[buf * BM + r] = t < p.T ? p.lse[at] * LOG2E : -INFINITY;
      s_dlt[buf * BM + r] = t < p.T ? p.delta[at] : 0.f;
    }
  };
  load_q(first_q, 0);
  cp_async_commit();

  const float sl2 = p.scale * LOG2E;
  float dk[D / 8][4], dv[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) {
    dk[i][0] = dk[i][1] = dk[i][2] = dk[i][3] = 0.f;
    dv[i][0] = dv[i][1] = dv[i][2] = dv[i][3] = 0.f;
  }
  const int key_a = k0 + warp * 16 + (lane >> 2);  // this thread's key rows: key_a, key_a + 8
  bool key_ok[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int key = key_a + r * 8;
    key_ok[r] = key < p.T && (p.key_valid == nullptr || p.key_valid[(int64_t)b * p.T + key] != 0);
  }
  for (int qi = first_q; qi < n_q; ++qi) {
    const int buf = (qi - first_q) & 1;
    __syncthreads();
    if (qi + 1 < n_q) {
      load_q(qi + 1, buf ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const __nv_bfloat16* q_sm = sq + buf * BM * LD;
    const __nv_bfloat16* do_sm = sdo + buf * BM * LD;
    float st[8][4], dpt[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      st[i][0] = st[i][1] = st[i][2] = st[i][3] = 0.f;
      dpt[i][0] = dpt[i][1] = dpt[i][2] = dpt[i][3] = 0.f;
    }
    mma_abt<D>(st, sk + warp * 16 * LD, q_sm);    // S^T: keys x queries
    mma_abt<D>(dpt, sv + warp * 16 * LD, do_sm);  // dP^T
    const int qs = qi * BM;
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = e >> 1;
        const int qoff = nb * 8 + (lane & 3) * 2 + (e & 1);
        const int q = qs + qoff;
        const int key = key_a + r * 8;
        const float l2 = s_lse[buf * BM + qoff];
        const bool vis = key_ok[r] && q < p.T && key <= q && l2 != -INFINITY;
        const float pr = vis ? exp2f(st[nb][e] * sl2 - l2) : 0.f;
        float dpv = dpt[nb][e], pd = pr;
        if (p.drop_thresh != 0) {  // dV takes the dropped P; dS the kept-scaled dP
          const bool keep = vis && dropout_keep(p.drop_seed, p.drop_offset, drop_elem(p, b, h, q, key), p.drop_thresh);
          dpv = keep ? dpv * p.drop_scale : 0.f;
          pd = keep ? pr * p.drop_scale : 0.f;
        }
        st[nb][e] = pd;                                         // P^T (dropped)
        dpt[nb][e] = pr * (dpv - s_dlt[buf * BM + qoff]);       // dS^T (unscaled)
      }
    }
    mma_pb<D>(dv, st, do_sm);
    mma_pb<D>(dk, dpt, q_sm);
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int t = key_a + r * 8;
    if (t >= p.T) continue;
    __nv_bfloat16* kd = p.dk + b * p.dk_batch + t * p.dk_row + h * D;
    __nv_bfloat16* vd = p.dv + b * p.dv_batch + t * p.dv_row + h * D;
#pragma unroll
    for (int nb = 0; nb < D / 8; ++nb) {
      const int col = nb * 8 + (lane & 3) * 2;
      *reinterpret_cast<__nv_bfloat162*>(kd + col) =
          __floats2bfloat162_rn(dk[nb][2 * r] * p.scale, dk[nb][2 * r + 1] * p.scale);
      *reinterpret_cast<__nv_bfloat162*>(vd + col) = __floats2bfloat162_rn(dv[nb][2 * r], dv[nb][2 * r + 1]);
    }
  }
}

template <int D>
cudaError_t launch_fwd(const Params& p, cudaStream_t st) {
  constexpr int LD = Smem<D>::LD;
  const size_t smem = (size_t)(BM + 4 * BN) * LD * sizeof(__nv_bfloat16) + 2 * BN;
  PRA_RETURN_IF_ERROR(pra::set_max_dynamic_smem(reinterpret_cast<const void*>(fwd_kernel<D>), (int)smem));
  dim3 grid(p.H * p.B, (p.T + BM - 1) / BM);
  fwd_kernel<D><<<grid, NT, smem, st>>>(p);
  return cudaGetLastError();
}

template <int D>
cudaError_t launch_bwd(const Params& p, cudaStream_t st) {
  constexpr int LD = Smem<D>::LD;
  {
    const int64_t rows = (int64_t)p.B * p.T * p.H;
    const bool vec = D % 8 == 0 && D / 8 <= 32 && p.o_row % 8 == 0 && p.o_batch % 8 == 0 && p.do_row % 8 == 0 &&
                     p.do_batch % 8 == 0 && (reinterpret_cast<uintptr_t>(p.o) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(p.dout) & 15) == 0;
    if (vec) delta_vec_kernel<D><<<(unsigned)((rows * (D / 8) + 255) / 256), 256, 0, st>>>(p);
    else delta_kernel<D><<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(p);
    PRA_RETURN_IF_ERROR(cudaGetLastError());
  }
  cudaError_t tc_dq = cudaErrorNotSupported;
  const bool tc_ok = pra_attention_get_impl() && p.T > 64 && p.drop_thresh == 0;  // dropout: mma.sync kernels
  if (tc_ok) tc_dq = pra_attention_bwd_dq_tc(p, D, st);
  if (tc_dq != cudaErrorNotSupported) {
    PRA_RETURN_IF_ERROR(tc_dq);
  } else {
    const size_t smem = (size_t)(2 * BM + 4 * BN) * LD * sizeof(__nv_bfloat16) + 2 * BN;
    PRA_RETURN_IF_ERROR(pra::set_max_dynamic_smem(reinterpret_cast<const void*>(bwd_dq_kernel<D>), (int)smem));
    dim3 grid(p.H * p.B, (p.T + BM - 1) / BM);
    bwd_dq_kernel<D><<<grid, NT, smem, st>>>(p);
    PRA_RETURN_IF_ERROR(cudaGetLastError());
  }
  if (tc_ok) {
    const cudaError_t e = pra_attention_bwd_dkdv_tc(p, D, st);
    if (e != cudaErrorNotSupported) return e;
  }
  {
    const size_t smem = (size_t)(2 * BN + 4 * BM) * LD * sizeof(__nv_bfloat16) + 4 * BM * sizeof(float);
    PRA_RETURN_IF_ERROR(pra::set_max_dynamic_smem(reinterpret_cast<const void*>(bwd_dkdv_kernel<D>), (int)smem));
    dim3 grid(p.H * p.B, (p.T + BN - 1) / BN);
    bwd_dkdv_kernel<D><<<grid, NT, smem, st>>>(p);
    return cudaGetLastError();
  }
}

}  // namespace attn
}  // namespace pra

// ---------------------------------------------------------------------------
static int g_attn_tcgen05 = 1;
void pra_attention_set_impl(int tcgen05) { g_attn_tcgen05 = tcgen05; }
int pra_attention_get_impl() { return g_attn_tcgen05; }

cudaError_t pra_attention_fwd(const AttnParams& p, int head_dim, cudaStream_t st) {
  using namespace pra::attn;
  if (p.B * p.T == 0) return cudaSuccess;
  // tcgen05: 128-query tiles, or two sequences per tile for <= 64 tokens at head dim 64; other
  // short sequences keep the 64-query mma.sync tiles, which waste no rows there.
  if (p.drop_thresh != 0 && (p.mem_len != nullptr || p.H != p.Hkv)) return cudaErrorInvalidValue;
  if (g_attn_tcgen05 && (p.T > 64 || head_dim == 64) && p.drop_thresh == 0) {
    const cudaError_t e = pra_attention_fwd_tc(p, head_dim, st);
    if (e != cudaErrorNotSupported) return e;
  }
  switch (head_dim) {
    case 16: return launch_fwd<16>(p, st);
    case 32: return launch_fwd<32>(p, st);
    case 64: return launch_fwd<64>(p, st);
    case 128: return launch_fwd<128>(p, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t pra_attention_bwd(const AttnParams& p, int head_dim, cudaStream_t st) {
  using namespace pra::attn;
  if (p.B * p.T == 0) return cudaSuccess;
  switch (head_dim) {
    case 16: return launch_bwd<16>(p, st);
    case 32: return launch_bwd<32>(p, st);
    case 64: return launch_bwd<64>(p, st);
    case 128: return launch_bwd<128>(p, st);
    default: return cudaErrorInvalidValue;
  }
}
