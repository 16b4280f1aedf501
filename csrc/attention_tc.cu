// Ragged native-K/V attention forward on the 5th-generation tensor cores (tcgen05, TMEM).
//
// Same operation and outputs as the mma.sync forward in attention.cu: one softmax over
//   [ selected memory keys (gathered from a token pool through mem_idx, fully visible) ;
//     local keys (causal, optional key-padding mask) ]
// writing O (bf16) and the natural-log LSE per query row.
//
// One CTA of 256 threads owns a tile of 128 queries of one (batch row, head); query row r is
// TMEM lane r of both accumulators and is owned by two threads (warps w and w + 4 may both
// access lanes 32 (w % 4) ... + 31), each taking half of the S and O columns:
//   S = Q K^T    (M=128, N=BN, K=D)   -> TMEM columns [0, BN)
//   O += P V     (M=128, N=D,  K=BN)  -> TMEM columns [BN, BN + D)
// Thread 0 issues the MMAs and commits them to one mbarrier; all threads stage K/V with
// cp.async (memory keys are gathered row by row, which a tiled TMA box cannot express),
// read their half S row with tcgen05.ld, apply the mask and the online softmax in registers
// (row maxima and sums combined with the partner thread through shared memory; 3-input max)
// and write their half P row (bf16, two per 32-bit column) back into TMEM, where the second
// MMA takes it as its A operand:
//   O += P V     (A = P from TMEM columns [BN + D, BN + D + BN / 2), B = V from shared memory)
// O stays in TMEM for the whole key loop: a row's running maximum is only raised (and its O
// row rescaled in TMEM) when a block's maximum exceeds it by more than 2^8 in exp2 units, so
// P <= 256 and the final O / l and LSE = m * scale + log(l) stay exact.
//
// Per iteration j: wait S_j (its commit also covers P V_{j-1}); prefetch K/V_{j+1} into the
// other stage (freed by P V_{j-1}); softmax of S_j into P; wait for K_{j+1}; thread 0 issues
// P V_j and S_{j+1} back to back.  Two CTAs share an SM (81 KB / 97 KB shared memory for
// head dim 64 / 128, 256 TMEM columns each), so one CTA's softmax overlaps the other's MMAs.
//
// Every mbarrier wait is bounded (about two seconds of SM clock); a CTA that times out sets
// *status, stops issuing MMAs, waits (bounded) for the ones in flight, frees its TMEM and
// returns.
//
// Reference behaviour: native_kv_attention (src/pra_torch/memory_batching.py:216, called from
// src/pra_torch/attention.py:443): memory keys before the causal local window, one softmax.
#include "tcgen05.cuh"

namespace pra {
namespace attn_tc {

constexpr int BM = 128;
constexpr int NT = 256;  // two threads per query row: warps w and w + 4 share TMEM lanes 32 (w % 4) ...
constexpr uint32_t TMEM_COLS = 256;
constexpr float LOG2E = 1.4426950408889634f;
constexpr float RESCALE_LOG2 = 8.f;
constexpr long long WAIT_CYCLES = 4000000000LL;

template <int D>
struct Cfg {
  static constexpr int BN = D == 64 ? 128 : 64;
  static constexpr int HB = BN / 2;  // S columns per thread
  static constexpr int HD = D / 2;   // O columns per thread
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;  // one K or V tile
  static constexpr int OFF_K = Q_BYTES;  // stage s: K at OFF_K + 2 s KV, V after it
  static constexpr int OFF_RED = OFF_K + 4 * KV_BYTES;    // [2][BM] floats: partner exchange
  static constexpr int OFF_VALID = OFF_RED + 2 * BM * 4;  // [2][BN] key-padding mask
  static constexpr int OFF_BAR = OFF_VALID + 2 * BN;
  static constexpr int SMEM = OFF_BAR + 16;
  // TMEM columns: S fp32 [0, BN), O fp32 [BN, BN + D), P bf16 pairs [BN + D, BN + D + BN / 2)
  static constexpr int O_COL = BN, P_COL = BN + D;
  static_assert(P_COL + BN / 2 <= (int)TMEM_COLS, "accumulators exceed the TMEM allocation");
  static_assert(OFF_BAR % 8 == 0, "mbarrier alignment");
  static_assert(HB % 32 == 0 && HD % 32 == 0, "32-column TMEM accesses");
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float m;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(m) : "f"(a), "f"(b), "f"(c));
  return m;
}

// (a.x * b.x + c.x, a.y * b.y + c.y).
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  return make_float2(fmaf(a.x, b.x, c.x), fmaf(a.y, b.y, c.y));
}

__device__ __forceinline__ float2 add2(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }

// Pair barrier of the two warps (w, w + 4) that own the same 32 query rows.
__device__ __forceinline__ void pair_sync(int warp) {
  switch (warp & 3) {  // immediate barrier ids 1..4 (barrier 0 is __syncthreads)
    case 0: asm volatile("bar.sync 1, 64;\n" ::: "memory"); break;
    case 1: asm volatile("bar.sync 2, 64;\n" ::: "memory"); break;
    case 2: asm volatile("bar.sync 3, 64;\n" ::: "memory"); break;
    default: asm volatile("bar.sync 4, 64;\n" ::: "memory"); break;
  }
}

// Rows of a block staged by this thread: with i = it * NT + tid, row (i / (8 * C)) * 8 + i % 8
// for it = 0 .. ROWS - 1 (C = D / 8 sixteen-byte chunks per row); the same rows for K and V.
template <int D, int BN>
struct Rows {
  static constexpr int C = D / 8;
  static constexpr int ROWS = BN * C / NT;
  static __device__ __forceinline__ int row(int it) {
    const int i = it * NT + threadIdx.x;
    return (i / (8 * C)) * 8 + (i & 7);
  }
  static __device__ __forceinline__ int chunk() { return (threadIdx.x >> 3) % C; }
};

// What the loads of one key block need from global memory before they can be issued: the
// pool row of each of this thread's memory keys (-1 past the end) and the padding mask byte
// of key threadIdx.x for local blocks.  Fetched one block ahead so the latency is hidden.
template <int D, int BN>
struct BlockMeta {
  int pool_row[Rows<D, BN>::ROWS];
  uint8_t valid;
};

template <int D, int BN>
__device__ __forceinline__ void fetch_meta(const AttnParams& p, BlockMeta<D, BN>& m, int b, bool memory, int start,
                                           int mem_len) {
  if (memory) {
    const int* idx = p.mem_idx + (int64_t)b * p.mem_max;
#pragma unroll
    for (int it = 0; it < Rows<D, BN>::ROWS; ++it) {
      const int j = start + Rows<D, BN>::row(it);
      m.pool_row[it] = j < mem_len ? __ldg(idx + j) : -1;
    }
  } else if (p.key_valid != nullptr && threadIdx.x < BN) {
    const int t = start + threadIdx.x;
    m.valid = t < p.T ? __ldg(p.key_valid + (int64_t)b * p.T + t) : 0;
  }
}

// Stage a block of BN keys: K and V rows into chunk-major core-matrix tiles (zeros past the
// end), the key-padding mask for local blocks.
template <int D, int BN>
__device__ __forceinline__ void load_block(const AttnParams& p, const BlockMeta<D, BN>& m, uint8_t* sk, uint8_t* sv,
                                           uint8_t* svalid, int b, int kvh, bool memory, int start) {
  if (!memory && p.key_valid != nullptr && threadIdx.x < BN) svalid[threadIdx.x] = m.valid;
  const int c = Rows<D, BN>::chunk();
#pragma unroll
  for (int it = 0; it < Rows<D, BN>::ROWS; ++it) {
    const int r = Rows<D, BN>::row(it);
    const __nv_bfloat16* ks = p.k;
    const __nv_bfloat16* vs = p.v;
    bool ok;
    if (memory) {
      ok = m.pool_row[it] >= 0;
      if (ok) {
        const int64_t off = (int64_t)m.pool_row[it] * p.mem_row + kvh * D + c * 8;
        ks = p.mem_k + off;
        vs = p.mem_v + off;
      }
    } else {
      const int t = start + r;
      ok = t < p.T;
      if (ok) {
        ks = p.k + b * p.k_batch + (int64_t)t * p.k_row + kvh * D + c * 8;
        vs = p.v + b * p.v_batch + (int64_t)t * p.v_row + kvh * D + c * 8;
      }
    }
    const uint32_t o = tc::core_off(r, c, BN);
    cp_async16(sk + o, ks, ok);
    cp_async16(sv + o, vs, ok);
  }
}

// Stage BM query rows (t = q0 .. q0 + BM - 1 of head h) of `src` into a chunk-major tile.
template <int D>
__device__ __forceinline__ void load_query_rows(uint8_t* tile, const __nv_bfloat16* src, int64_t row_stride,
                                                int64_t batch_stride, int b, int h, int q0, int T) {
#pragma unroll
  for (int it = 0; it < BM * (D / 8) / NT; ++it) {
    const int i = it * NT + threadIdx.x;
    const int c = (i >> 3) % (D / 8), r = (i / D) * 8 + (i & 7), t = q0 + r;
    const bool ok = t < T;
    cp_async16(tile + tc::core_off(r, c, BM), ok ? src + b * batch_stride + (int64_t)t * row_stride + h * D + c * 8 : src,
               ok);
  }
}

template <int D>
__global__ void __launch_bounds__(NT, 2) fwd_kernel(AttnParams p) {
  using C = Cfg<D>;
  constexpr int BN = C::BN, HB = C::HB, HD = C::HD;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* sq = smem;
  float* red = reinterpret_cast<float*>(smem + C::OFF_RED);
  uint8_t* svalid = smem + C::OFF_VALID;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + C::OFF_BAR + 8);
  int* s_abort = reinterpret_cast<int*>(smem + C::OFF_BAR + 12);
  auto stage_k = [&](int s) { return smem + C::OFF_K + s * 2 * C::KV_BYTES; };
  auto stage_v = [&](int s) { return smem + C::OFF_K + s * 2 * C::KV_BYTES + C::KV_BYTES; };

  // grid (H * B, query tiles): the longest (last, causal) query tiles are scheduled first
  const int h = blockIdx.x % p.H, b = blockIdx.x / p.H;
  const int qb = gridDim.y - 1 - blockIdx.y;
  const int kvh = h / (p.H / p.Hkv);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int row = tid & (BM - 1), half = tid >> 7;
  const int q0 = qb * BM;
  const int mem_len = p.mem_len ? p.mem_len[b] : 0;
  const int n_mem = (mem_len + BN - 1) / BN;
  const int q_last = min(q0 + BM, p.T) - 1;
  const int n_blocks = n_mem + q_last / BN + 1;

  if (warp == 0) {
    tc::alloc(s_tmem, TMEM_COLS);
    tc::relinquish();
  }
  if (tid == 0) {
    mbar_init(bar, 1);
    *s_abort = 0;
    tc::fence_mbarrier_init();
  }
  load_query_rows<D>(sq, p.q, p.q_row, p.q_batch, b, h, q0, p.T);
  auto block_start = [&](int j) { return j < n_mem ? j * BN : (j - n_mem) * BN; };
  BlockMeta<D, BN> meta;
  fetch_meta<D, BN>(p, meta, b, n_mem > 0, 0, mem_len);
  load_block<D, BN>(p, meta, stage_k(0), stage_v(0), svalid, b, kvh, n_mem > 0, 0);
  cp_async_commit();
  if (n_blocks > 1) fetch_meta<D, BN>(p, meta, b, 1 < n_mem, block_start(1), mem_len);
  cp_async_wait<0>();
  fence_proxy_async_smem();
  tc::fence_before();
  __syncthreads();
  tc::fence_after();

  const uint32_t tmem = *s_tmem;
  const uint32_t lane = (uint32_t)((warp & 3) * 32) << 16;
  const uint32_t t_s = tmem + lane + half * HB;                // this thread's S columns
  const uint32_t t_o = tmem + lane + C::O_COL + half * HD;     // this thread's O columns
  const uint32_t t_p = tmem + lane + C::P_COL + half * HB / 2;  // this thread's P columns
  constexpr uint32_t ID_S = tc::idesc_bf16(BM, BN, false);
  constexpr uint32_t ID_O = tc::idesc_bf16(BM, D, true);
  constexpr uint32_t Q_LBO = (BM / 8) * 128, KV_LBO = (BN / 8) * 128;
  const uint32_t q_addr = smem_u32(sq);

  // S = Q K^T: A = Q (K-major over D), B = K tile (K-major over D); 16 features per MMA.
  auto issue_s = [&](int s) {
    const uint32_t k_addr = smem_u32(stage_k(s));
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk)
      tc::mma_bf16(tmem, tc::smem_desc(q_addr + kk * 2 * Q_LBO, Q_LBO, 128),
                   tc::smem_desc(k_addr + kk * 2 * KV_LBO, KV_LBO, 128), ID_S, kk > 0);
  };
  // O (+)= P V: A = P in TMEM (8 columns per 16 keys), B = V tile (MN-major: D contiguous).
  auto issue_o = [&](int s, bool acc) {
    const uint32_t v_addr = smem_u32(stage_v(s));
#pragma unroll
    for (int kk = 0; kk < BN / 16; ++kk)
      tc::mma_bf16_ts(tmem + C::O_COL, tmem + C::P_COL + kk * 8, tc::smem_desc(v_addr + kk * 2 * 128, 128, KV_LBO),
                      ID_O, (acc || kk > 0) ? 1u : 0u);
  };

  if (tid == 0) {
    issue_s(0);
    tc::commit(bar);
  }

  const float sl2 = p.scale * LOG2E;
  const int q = q0 + row;
  float m_run = -INFINITY, l_run = 0.f;  // l_run: this thread's columns only
  bool aborted = false;

  for (int j = 0; j < n_blocks; ++j) {
    const int s = j & 1;
    if (!tc::mbar_wait_cycles(bar, (uint32_t)(j & 1), WAIT_CYCLES)) *s_abort = 1;
    const bool memory = j < n_mem;
    const int start = block_start(j);
    if (j + 1 < n_blocks) {
      load_block<D, BN>(p, meta, stage_k(s ^ 1), stage_v(s ^ 1), svalid + (s ^ 1) * BN, b, kvh, j + 1 < n_mem,
                    block_start(j + 1));
      cp_async_commit();
      if (j + 2 < n_blocks) fetch_meta<D, BN>(p, meta, b, j + 2 < n_mem, block_start(j + 2), mem_len);
    }

    // visible keys of this thread's columns: [0, lim) (and the padding mask for local blocks)
    const int col0 = half * HB;
    int lim;
    const uint8_t* valid = nullptr;
    if (memory) {
      lim = mem_len - start - col0;
    } else {
      lim = min(p.T, q + 1) - start - col0;
      if (p.key_valid != nullptr) valid = svalid + s * BN + col0;
    }
    const bool masked = lim < HB || valid != nullptr;
    // This thread's HB S columns (HB = 32 or 64, one TMEM load), masked keys at -inf.  S is
    // read twice from TMEM: here for the row maximum, below (32 columns at a time) for the
    // exponentials.
    auto load_s = [&](float (&sv)[HB]) {
      uint32_t r[HB];
      if constexpr (HB == 64) tc::ld64(t_s, r);
      else tc::ld32(t_s, r);
      if (!masked) {
#pragma unroll
        for (int i = 0; i < HB; ++i) sv[i] = __uint_as_float(r[i]);
      } else {
#pragma unroll
        for (int i = 0; i < HB; ++i) {
          const bool vis = i < lim && (valid == nullptr || valid[i] != 0);
          sv[i] = vis ? __uint_as_float(r[i]) : -INFINITY;
        }
      }
    };
    float mx = -INFINITY;
    {
      float sv[HB];
      load_s(sv);
#pragma unroll
      for (int i = 0; i < HB; i += 2) mx = max3(mx, sv[i], sv[i + 1]);
    }
    red[half * BM + row] = mx;
    pair_sync(warp);
    mx = fmaxf(mx, red[(half ^ 1) * BM + row]);

    // running maximum, raised lazily; O rows rescaled in TMEM when it moves
    float corr = 1.f;
    bool rescale = false;
    if (mx > m_run) {
      if (m_run == -INFINITY) {
        m_run = mx;  // nothing accumulated yet: l = 0 and the row of O is zero (or not yet written)
      } else if ((mx - m_run) * sl2 > RESCALE_LOG2) {
        corr = ex2((m_run - mx) * sl2);
        l_run *= corr;
        m_run = mx;
        rescale = true;
      }
    }
    if (j > 0 && __any_sync(0xffffffffu, rescale)) {
#pragma unroll
      for (int c0 = 0; c0 < HD; c0 += 32) {
        uint32_t r[32];
        tc::ld32(t_o + c0, r);
#pragma unroll
        for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * corr);
        tc::st32(t_o + c0, r);
      }
    }
    const float ms = m_run == -INFINITY ? 0.f : m_run * sl2;
    const float2 sl2x2 = make_float2(sl2, sl2), nms = make_float2(-ms, -ms);
    float2 acc = make_float2(0.f, 0.f);
#pragma unroll
    for (int c0 = 0; c0 < HB; c0 += 32) {
      uint32_t r[32];
      tc::ld32(t_s + c0, r);
      uint32_t w[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        float2 sv = make_float2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
        if (masked) {
          const int c = c0 + 2 * i;
          if (!(c < lim && (valid == nullptr || valid[c] != 0))) sv.x = -INFINITY;
          if (!(c + 1 < lim && (valid == nullptr || valid[c + 1] != 0))) sv.y = -INFINITY;
        }
        float2 x = fma2(sv, sl2x2, nms);
        x.x = ex2(x.x);
        x.y = ex2(x.y);
        acc = add2(acc, x);
        w[i] = pack_bf16(x.x, x.y);
      }
      tc::st16(t_p + c0 / 2, w);
    }
    l_run += acc.x + acc.y;

    if (j + 1 < n_blocks) cp_async_wait<0>();
    fence_proxy_async_smem();  // cp.async data -> the tensor core's (async proxy) reads
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    if (*s_abort) {
      aborted = true;
      break;
    }
    if (tid == 0) {
      issue_o(s, j > 0);
      if (j + 1 < n_blocks) issue_s(s ^ 1);
      tc::commit(bar);
    }
  }

  if (!aborted) {
    if (!tc::mbar_wait_cycles(bar, (uint32_t)(n_blocks & 1), WAIT_CYCLES)) aborted = true;
  }
  aborted = __syncthreads_or(aborted);  // uniform: the epilogue's TMEM loads are warp-collective
  red[half * BM + row] = l_run;
  pair_sync(warp);
  const float l_tot = l_run + red[(half ^ 1) * BM + row];
  if (!aborted) {
    const float inv = l_tot > 0.f ? 1.f / l_tot : 0.f;
    __nv_bfloat16* dst = p.o + b * p.o_batch + (int64_t)q * p.o_row + h * D + half * HD;
#pragma unroll
    for (int c0 = 0; c0 < HD; c0 += 32) {
      uint32_t r[32];
      tc::ld32(t_o + c0, r);
      if (q < p.T) {
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          uint4 w;
          w.x = pack_bf16(__uint_as_float(r[i + 0]) * inv, __uint_as_float(r[i + 1]) * inv);
          w.y = pack_bf16(__uint_as_float(r[i + 2]) * inv, __uint_as_float(r[i + 3]) * inv);
          w.z = pack_bf16(__uint_as_float(r[i + 4]) * inv, __uint_as_float(r[i + 5]) * inv);
          w.w = pack_bf16(__uint_as_float(r[i + 6]) * inv, __uint_as_float(r[i + 7]) * inv);
          *reinterpret_cast<uint4*>(dst + c0 + i) = w;
        }
      }
    }
    if (q < p.T && half == 0)
      p.lse[((int64_t)b * p.H + h) * p.T + q] = l_tot > 0.f ? m_run * p.scale + logf(l_tot) : -INFINITY;
  } else {
    // Stop: record the failure, give the MMAs in flight a bounded time to finish, free TMEM.
    if (tid == 0 && p.status != nullptr) atomicExch(p.status, 1);
    cp_async_wait<0>();
    tc::mbar_wait_cycles(bar, (uint32_t)(n_blocks & 1), WAIT_CYCLES);
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after();
    tc::dealloc(tmem, TMEM_COLS);
  }
}

// ---- backward: dQ -------------------------------------------------------------------------
// dQ of a 128-query tile over every key block it sees, head dim 64, blocks of 64 keys:
//   S  = Q K^T  -> TMEM [0, 64)       dP = dO V^T -> TMEM [64, 128)
//   dS = P (dP - delta) with P = exp2(S scale log2e - lse log2e), bf16 pairs -> TMEM [192, 224)
//   dQ += dS K  (A = dS from TMEM, B = K tile MN-major) -> TMEM [128, 192)
// Two threads per query row (32 S/dP columns each), the same staging, prefetch and bounded
// waits as the forward.  dQ = scale * (dS K).
struct DqCfg {
  static constexpr int D = 64, BN = 64, HB = 32;
  static constexpr int Q_BYTES = BM * D * 2, KV_BYTES = BN * D * 2;
  static constexpr int OFF_DO = Q_BYTES, OFF_K = 2 * Q_BYTES;  // stage s: K at OFF_K + 2 s KV, V after it
  static constexpr int OFF_VALID = OFF_K + 4 * KV_BYTES;
  static constexpr int OFF_BAR = OFF_VALID + 2 * BN;
  static constexpr int SMEM = OFF_BAR + 16;
  static constexpr int S_COL = 0, DP_COL = 64, DQ_COL = 128, DS_COL = 192;
};

__global__ void __launch_bounds__(NT, 2) bwd_dq_kernel(AttnParams p) {
  using C = DqCfg;
  constexpr int D = C::D, BN = C::BN, HB = C::HB;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* sq = smem;
  uint8_t* sdo = smem + C::OFF_DO;
  uint8_t* svalid = smem + C::OFF_VALID;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + C::OFF_BAR + 8);
  int* s_abort = reinterpret_cast<int*>(smem + C::OFF_BAR + 12);
  auto stage_k = [&](int s) { return smem + C::OFF_K + s * 2 * C::KV_BYTES; };
  auto stage_v = [&](int s) { return smem + C::OFF_K + s * 2 * C::KV_BYTES + C::KV_BYTES; };

  const int h = blockIdx.x % p.H, b = blockIdx.x / p.H;
  const int qb = gridDim.y - 1 - blockIdx.y;
  const int kvh = h / (p.H / p.Hkv);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int row = tid & (BM - 1), half = tid >> 7;
  const int q0 = qb * BM;
  const int mem_len = p.mem_len ? p.mem_len[b] : 0;
  const int n_mem = (mem_len + BN - 1) / BN;
  const int q_last = min(q0 + BM, p.T) - 1;
  const int n_blocks = n_mem + q_last / BN + 1;

  if (warp == 0) {
    tc::alloc(s_tmem, TMEM_COLS);
    tc::relinquish();
  }
  if (tid == 0) {
    mbar_init(bar, 1);
    *s_abort = 0;
    tc::fence_mbarrier_init();
  }
  load_query_rows<D>(sq, p.q, p.q_row, p.q_batch, b, h, q0, p.T);
  load_query_rows<D>(sdo, p.dout, p.do_row, p.do_batch, b, h, q0, p.T);
  auto block_start = [&](int j) { return j < n_mem ? j * BN : (j - n_mem) * BN; };
  BlockMeta<D, BN> meta;
  fetch_meta<D, BN>(p, meta, b, n_mem > 0, 0, mem_len);
  load_block<D, BN>(p, meta, stage_k(0), stage_v(0), svalid, b, kvh, n_mem > 0, 0);
  cp_async_commit();
  if (n_blocks > 1) fetch_meta<D, BN>(p, meta, b, 1 < n_mem, block_start(1), mem_len);
  const int q = q0 + row;
  const int64_t at = ((int64_t)b * p.H + h) * p.T + q;
  const float lse2 = q < p.T ? p.lse[at] * LOG2E : -INFINITY;
  const float dlt = q < p.T ? p.delta[at] : 0.f;
  cp_async_wait<0>();
  fence_proxy_async_smem();
  tc::fence_before();
  __syncthreads();
  tc::fence_after();

  const uint32_t tmem = *s_tmem;
  const uint32_t lane = (uint32_t)((warp & 3) * 32) << 16;
  constexpr uint32_t ID_S = tc::idesc_bf16(BM, BN, false);
  constexpr uint32_t ID_DQ = tc::idesc_bf16(BM, D, true);
  constexpr uint32_t Q_LBO = (BM / 8) * 128, KV_LBO = (BN / 8) * 128;
  const uint32_t q_addr = smem_u32(sq), do_addr = smem_u32(sdo);

  // S = Q K^T and dP = dO V^T for the block in stage s (both operands K-major over D).
  auto issue_s_dp = [&](int s) {
    const uint32_t k_addr = smem_u32(stage_k(s)), v_addr = smem_u32(stage_v(s));
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk)
      tc::mma_bf16(tmem + C::S_COL, tc::smem_desc(q_addr + kk * 2 * Q_LBO, Q_LBO, 128),
                   tc::smem_desc(k_addr + kk * 2 * KV_LBO, KV_LBO, 128), ID_S, kk > 0);
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk)
      tc::mma_bf16(tmem + C::DP_COL, tc::smem_desc(do_addr + kk * 2 * Q_LBO, Q_LBO, 128),
                   tc::smem_desc(v_addr + kk * 2 * KV_LBO, KV_LBO, 128), ID_S, kk > 0);
  };
  // dQ (+)= dS K: A = dS in TMEM (8 columns per 16 keys), B = K tile MN-major (D contiguous).
  auto issue_dq = [&](int s, bool acc) {
    const uint32_t k_addr = smem_u32(stage_k(s));
#pragma unroll
    for (int kk = 0; kk < BN / 16; ++kk)
      tc::mma_bf16_ts(tmem + C::DQ_COL, tmem + C::DS_COL + kk * 8, tc::smem_desc(k_addr + kk * 2 * 128, 128, KV_LBO),
                      ID_DQ, (acc || kk > 0) ? 1u : 0u);
  };

  if (tid == 0) {
    issue_s_dp(0);
    tc::commit(bar);
  }

  const float sl2 = p.scale * LOG2E;
  const float2 sl2x2 = make_float2(sl2, sl2), nlse = make_float2(-lse2, -lse2), ndlt = make_float2(-dlt, -dlt);
  const bool row_live = lse2 != -INFINITY;
  bool aborted = false;
  for (int j = 0; j < n_blocks; ++j) {
    const int s = j & 1;
    if (!tc::mbar_wait_cycles(bar, (uint32_t)(j & 1), WAIT_CYCLES)) *s_abort = 1;
    const bool memory = j < n_mem;
    const int start = block_start(j);
    if (j + 1 < n_blocks) {
      load_block<D, BN>(p, meta, stage_k(s ^ 1), stage_v(s ^ 1), svalid + (s ^ 1) * BN, b, kvh, j + 1 < n_mem,
                        block_start(j + 1));
      cp_async_commit();
      if (j + 2 < n_blocks) fetch_meta<D, BN>(p, meta, b, j + 2 < n_mem, block_start(j + 2), mem_len);
    }
    const int col0 = half * HB;
    int lim;
    const uint8_t* valid = nullptr;
    if (memory) {
      lim = mem_len - start - col0;
    } else {
      lim = min(p.T, q + 1) - start - col0;
      if (p.key_valid != nullptr) valid = svalid + s * BN + col0;
    }
    const bool masked = lim < HB || valid != nullptr || !row_live;
    uint32_t rs[32], rdp[32];
    tc::ld32(tmem + lane + C::S_COL + col0, rs);
    tc::ld32(tmem + lane + C::DP_COL + col0, rdp);
    uint32_t w[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float2 sv = make_float2(__uint_as_float(rs[2 * i]), __uint_as_float(rs[2 * i + 1]));
      if (masked) {
        const int c = 2 * i;
        if (!(row_live && c < lim && (valid == nullptr || valid[c] != 0))) sv.x = -INFINITY;
        if (!(row_live && c + 1 < lim && (valid == nullptr || valid[c + 1] != 0))) sv.y = -INFINITY;
      }
      float2 pr = fma2(sv, sl2x2, nlse);
      pr.x = ex2(pr.x);
      pr.y = ex2(pr.y);
      const float2 g = add2(make_float2(__uint_as_float(rdp[2 * i]), __uint_as_float(rdp[2 * i + 1])), ndlt);
      w[i] = pack_bf16(pr.x * g.x, pr.y * g.y);
    }
    tc::st16(tmem + lane + C::DS_COL + half * (HB / 2), w);

    if (j + 1 < n_blocks) cp_async_wait<0>();
    fence_proxy_async_smem();
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    if (*s_abort) {
      aborted = true;
      break;
    }
    if (tid == 0) {
      issue_dq(s, j > 0);
      if (j + 1 < n_blocks) issue_s_dp(s ^ 1);
      tc::commit(bar);
    }
  }

  if (!aborted) {
    if (!tc::mbar_wait_cycles(bar, (uint32_t)(n_blocks & 1), WAIT_CYCLES)) aborted = true;
  }
  aborted = __syncthreads_or(aborted);
  if (!aborted) {
    uint32_t r[32];
    tc::ld32(tmem + lane + C::DQ_COL + half * 32, r);
    if (q < p.T) {
      __nv_bfloat16* dst = p.dq + b * p.dq_batch + (int64_t)q * p.dq_row + h * D + half * 32;
#pragma unroll
      for (int i = 0; i < 32; i += 8) {
        uint4 v;
        v.x = pack_bf16(__uint_as_float(r[i + 0]) * p.scale, __uint_as_float(r[i + 1]) * p.scale);
        v.y = pack_bf16(__uint_as_float(r[i + 2]) * p.scale, __uint_as_float(r[i + 3]) * p.scale);
        v.z = pack_bf16(__uint_as_float(r[i + 4]) * p.scale, __uint_as_float(r[i + 5]) * p.scale);
        v.w = pack_bf16(__uint_as_float(r[i + 6]) * p.scale, __uint_as_float(r[i + 7]) * p.scale);
        *reinterpret_cast<uint4*>(dst + i) = v;
      }
    }
  } else {
    if (tid == 0 && p.status != nullptr) atomicExch(p.status, 1);
    cp_async_wait<0>();
    tc::mbar_wait_cycles(bar, (uint32_t)(n_blocks & 1), WAIT_CYCLES);
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after();
    tc::dealloc(tmem, TMEM_COLS);
  }
}

// ---- backward: dK, dV of the local keys ---------------------------------------------------
// One CTA owns 128 local keys of one (batch row, head) (TMEM lane = key) and walks the query
// blocks of 32 that can see them (causal), head dim 64, MHA:
//   S^T = K Q^T, dP^T = V dO^T        -> TMEM buffer x = block parity: [64 x, 64 x + 32), [64 x + 32, 64 x + 64)
//   P^T = exp2(S^T scale log2e - lse log2e), dS^T = P^T (dP^T - delta), written as bf16 pairs
//         over the first half of each thread's own S^T / dP^T columns
//   dV += P^T dO, dK += dS^T Q         -> TMEM [128, 192), [192, 256)
// The two S^T / dP^T buffers alternate, so the next block's MMAs never write columns that the
// previous block's dV / dK MMAs read (tcgen05 MMAs into different accumulators are not
// ordered); a buffer is reused two blocks later, after the commit that covers those reads.
// Two threads per key row (16 query columns each); lse and delta of a block staged in shared
// memory.  dK = scale * (dS^T Q).
struct DkvCfg {
  static constexpr int D = 64, BK = 128, BQ = 32, HQ = 16;
  static constexpr int KV_BYTES = BK * D * 2, QB_BYTES = BQ * D * 2;
  static constexpr int OFF_V = KV_BYTES, OFF_Q = 2 * KV_BYTES;  // stage s: Q at OFF_Q + 2 s QB, dO after it
  static constexpr int OFF_LSE = OFF_Q + 4 * QB_BYTES;           // [2][BQ] lse * log2e, then [2][BQ] delta
  static constexpr int OFF_BAR = OFF_LSE + 4 * BQ * 4;
  static constexpr int SMEM = OFF_BAR + 16;
  static constexpr int DV_COL = 128, DK_COL = 192;
};

__global__ void __launch_bounds__(NT, 2) bwd_dkdv_kernel(AttnParams p) {
  using C = DkvCfg;
  constexpr int D = C::D, BK = C::BK, BQ = C::BQ, HQ = C::HQ;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* sk = smem;
  uint8_t* sv = smem + C::OFF_V;
  float* s_lse = reinterpret_cast<float*>(smem + C::OFF_LSE);
  float* s_dlt = s_lse + 2 * BQ;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + C::OFF_BAR + 8);
  int* s_abort = reinterpret_cast<int*>(smem + C::OFF_BAR + 12);
  auto stage_q = [&](int s) { return smem + C::OFF_Q + s * 2 * C::QB_BYTES; };
  auto stage_do = [&](int s) { return smem + C::OFF_Q + s * 2 * C::QB_BYTES + C::QB_BYTES; };

  // grid (H * B, key tiles): the first key tiles (seen by the most queries) are scheduled first
  const int h = blockIdx.x % p.H, b = blockIdx.x / p.H;
  const int k0 = blockIdx.y * BK;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int row = tid & (BK - 1), half = tid >> 7;
  const int first_q = k0 / BQ;
  const int n_blocks = (p.T + BQ - 1) / BQ - first_q;

  if (warp == 0) {
    tc::alloc(s_tmem, TMEM_COLS);
    tc::relinquish();
  }
  if (tid == 0) {
    mbar_init(bar, 1);
    *s_abort = 0;
    tc::fence_mbarrier_init();
  }
  load_query_rows<D>(sk, p.k, p.k_row, p.k_batch, b, h, k0, p.T);  // 128 key rows, same tile shape as a query tile
  load_query_rows<D>(sv, p.v, p.v_row, p.v_batch, b, h, k0, p.T);
  // Q / dO rows of query block qi (32 rows x 8 chunks: one 16-byte chunk per thread each) and its lse / delta
  auto load_qblock = [&](int qi, int s) {
    const int qs = qi * BQ;
    const int c = (tid >> 3) & 7, r = (tid >> 6) * 8 + (tid & 7), t = qs + r;
    const bool ok = t < p.T;
    const uint32_t o = tc::core_off(r, c, BQ);
    cp_async16(stage_q(s) + o, ok ? p.q + b * p.q_batch + (int64_t)t * p.q_row + h * D + c * 8 : p.q, ok);
    cp_async16(stage_do(s) + o, ok ? p.dout + b * p.do_batch + (int64_t)t * p.do_row + h * D + c * 8 : p.dout, ok);
    if (tid < BQ) {
      const int tq = qs + tid;
      const int64_t at = ((int64_t)b * p.H + h) * p.T + tq;
      s_lse[s * BQ + tid] = tq < p.T ? p.lse[at] * LOG2E : -INFINITY;
      s_dlt[s * BQ + tid] = tq < p.T ? p.delta[at] : 0.f;
    }
  };
  load_qblock(first_q, 0);
  cp_async_commit();
  const int key = k0 + row;
  const bool key_ok = key < p.T && (p.key_valid == nullptr || p.key_valid[(int64_t)b * p.T + key] != 0);
  cp_async_wait<0>();
  fence_proxy_async_smem();
  tc::fence_before();
  __syncthreads();
  tc::fence_after();

  const uint32_t tmem = *s_tmem;
  const uint32_t lane = (uint32_t)((warp & 3) * 32) << 16;
  constexpr uint32_t ID_ST = tc::idesc_bf16(BK, BQ, false);
  constexpr uint32_t ID_G = tc::idesc_bf16(BK, D, true);
  constexpr uint32_t K_LBO = (BK / 8) * 128, QB_LBO = (BQ / 8) * 128;
  const uint32_t k_addr = smem_u32(sk), v_addr = smem_u32(sv);
  auto st_col = [&](int x) { return (uint32_t)(64 * x); };
  auto dpt_col = [&](int x) { return (uint32_t)(64 * x + 32); };

  // S^T = K Q^T and dP^T = V dO^T for the query block in stage s (all operands K-major over D).
  auto issue_st = [&](int s, int x) {
    const uint32_t q_addr = smem_u32(stage_q(s)), do_addr = smem_u32(stage_do(s));
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk)
      tc::mma_bf16(tmem + st_col(x), tc::smem_desc(k_addr + kk * 2 * K_LBO, K_LBO, 128),
                   tc::smem_desc(q_addr + kk * 2 * QB_LBO, QB_LBO, 128), ID_ST, kk > 0);
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk)
      tc::mma_bf16(tmem + dpt_col(x), tc::smem_desc(v_addr + kk * 2 * K_LBO, K_LBO, 128),
                   tc::smem_desc(do_addr + kk * 2 * QB_LBO, QB_LBO, 128), ID_ST, kk > 0);
  };
  // dV += P^T dO, dK += dS^T Q: A from TMEM (query columns 16 kk .. 16 kk + 15 packed at column
  // 16 kk of the thread pair's buffer), B = dO / Q stage MN-major (D contiguous).
  auto issue_grad = [&](int s, int x, bool acc) {
    const uint32_t q_addr = smem_u32(stage_q(s)), do_addr = smem_u32(stage_do(s));
#pragma unroll
    for (int kk = 0; kk < BQ / 16; ++kk)
      tc::mma_bf16_ts(tmem + C::DV_COL, tmem + st_col(x) + kk * 16,
                      tc::smem_desc(do_addr + kk * 2 * 128, 128, QB_LBO), ID_G, (acc || kk > 0) ? 1u : 0u);
#pragma unroll
    for (int kk = 0; kk < BQ / 16; ++kk)
      tc::mma_bf16_ts(tmem + C::DK_COL, tmem + dpt_col(x) + kk * 16,
                      tc::smem_desc(q_addr + kk * 2 * 128, 128, QB_LBO), ID_G, (acc || kk > 0) ? 1u : 0u);
  };

  if (tid == 0) {
    issue_st(0, 0);
    tc::commit(bar);
  }

  const float sl2 = p.scale * LOG2E;
  const float2 sl2x2 = make_float2(sl2, sl2);
  bool aborted = false;
  for (int j = 0; j < n_blocks; ++j) {
    const int s = j & 1, x = j & 1;
    const int qs = (first_q + j) * BQ;
    if (!tc::mbar_wait_cycles(bar, (uint32_t)(j & 1), WAIT_CYCLES)) *s_abort = 1;
    if (j + 1 < n_blocks) {
      load_qblock(first_q + j + 1, s ^ 1);
      cp_async_commit();
    }
    const int c0 = half * HQ;  // this thread's query columns c0 .. c0 + 15
    uint32_t rs[16], rdp[16];
    tc::ld16(tmem + lane + st_col(x) + c0, rs);
    tc::ld16(tmem + lane + dpt_col(x) + c0, rdp);
    const float* lse_b = s_lse + s * BQ + c0;
    const float* dlt_b = s_dlt + s * BQ + c0;
    uint32_t wp[8], wd[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int c = 2 * i;
      const int qa = qs + c0 + c;
      const bool va = key_ok && qa < p.T && key <= qa && lse_b[c] != -INFINITY;
      const bool vb = key_ok && qa + 1 < p.T && key <= qa + 1 && lse_b[c + 1] != -INFINITY;
      float2 sv = make_float2(va ? __uint_as_float(rs[c]) : -INFINITY, vb ? __uint_as_float(rs[c + 1]) : -INFINITY);
      float2 pr = fma2(sv, sl2x2, make_float2(va ? -lse_b[c] : 0.f, vb ? -lse_b[c + 1] : 0.f));
      pr.x = ex2(pr.x);
      pr.y = ex2(pr.y);
      const float2 g = add2(make_float2(__uint_as_float(rdp[c]), __uint_as_float(rdp[c + 1])),
                            make_float2(-dlt_b[c], -dlt_b[c + 1]));
      wp[i] = pack_bf16(pr.x, pr.y);
      wd[i] = pack_bf16(pr.x * g.x, pr.y * g.y);
    }
    tc::st8(tmem + lane + st_col(x) + c0, wp);
    tc::st8(tmem + lane + dpt_col(x) + c0, wd);

    if (j + 1 < n_blocks) cp_async_wait<0>();
    fence_proxy_async_smem();
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    if (*s_abort) {
      aborted = true;
      break;
    }
    if (tid == 0) {
      issue_grad(s, x, j > 0);
      if (j + 1 < n_blocks) issue_st(s ^ 1, x ^ 1);
      tc::commit(bar);
    }
  }

  if (!aborted) {
    if (!tc::mbar_wait_cycles(bar, (uint32_t)(n_blocks & 1), WAIT_CYCLES)) aborted = true;
  }
  aborted = __syncthreads_or(aborted);
  if (!aborted) {
    uint32_t rv[32], rk[32];
    tc::ld32(tmem + lane + C::DV_COL + half * 32, rv);
    tc::ld32(tmem + lane + C::DK_COL + half * 32, rk);
    if (key < p.T) {
      __nv_bfloat16* vd = p.dv + b * p.dv_batch + (int64_t)key * p.dv_row + h * D + half * 32;
      __nv_bfloat16* kd = p.dk + b * p.dk_batch + (int64_t)key * p.dk_row + h * D + half * 32;
#pragma unroll
      for (int i = 0; i < 32; i += 8) {
        uint4 a, c;
        a.x = pack_bf16(__uint_as_float(rv[i + 0]), __uint_as_float(rv[i + 1]));
        a.y = pack_bf16(__uint_as_float(rv[i + 2]), __uint_as_float(rv[i + 3]));
        a.z = pack_bf16(__uint_as_float(rv[i + 4]), __uint_as_float(rv[i + 5]));
        a.w = pack_bf16(__uint_as_float(rv[i + 6]), __uint_as_float(rv[i + 7]));
        c.x = pack_bf16(__uint_as_float(rk[i + 0]) * p.scale, __uint_as_float(rk[i + 1]) * p.scale);
        c.y = pack_bf16(__uint_as_float(rk[i + 2]) * p.scale, __uint_as_float(rk[i + 3]) * p.scale);
        c.z = pack_bf16(__uint_as_float(rk[i + 4]) * p.scale, __uint_as_float(rk[i + 5]) * p.scale);
        c.w = pack_bf16(__uint_as_float(rk[i + 6]) * p.scale, __uint_as_float(rk[i + 7]) * p.scale);
        *reinterpret_cast<uint4*>(vd + i) = a;
        *reinterpret_cast<uint4*>(kd + i) = c;
      }
    }
  } else {
    if (tid == 0 && p.status != nullptr) atomicExch(p.status, 1);
    cp_async_wait<0>();
    tc::mbar_wait_cycles(bar, (uint32_t)(n_blocks & 1), WAIT_CYCLES);
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after();
    tc::dealloc(tmem, TMEM_COLS);
  }
}

// ---- forward, two short sequences per tile -----------------------------------------------
// Sequences of <= 64 tokens (chunk encodes), head dim 64: batch rows b0 = 2 blockIdx.y and
// b0 + 1 share one 128-query tile (rows 0-63: b0, rows 64-127: b0 + 1).  Every key block holds
// 64 keys of each sequence (K/V rows 0-63 / 64-127): memory blocks j = 0 .. n_mem - 1 take
// memory keys 64 j .. 64 j + 63 of each row's own list, then one local block.  A query row
// only sees its own sequence's 64 columns; the other half of its P row is zero (written once),
// so the single S and P V MMAs per block serve both sequences.  Otherwise as fwd_kernel<64>.
struct PackCfg {
  static constexpr int D = 64, BN = 128, KB = 64, HB = 32;
  static constexpr int Q_BYTES = BM * D * 2, KV_BYTES = BN * D * 2;
  static constexpr int OFF_K = Q_BYTES;
  static constexpr int OFF_RED = OFF_K + 4 * KV_BYTES;
  static constexpr int OFF_VALID = OFF_RED + 2 * BM * 4;
  static constexpr int OFF_BAR = OFF_VALID + 2 * BN;
  static constexpr int SMEM = OFF_BAR + 16;
  static constexpr int O_COL = BN, P_COL = BN + D;  // as Cfg<64>
};

__global__ void __launch_bounds__(NT, 2) fwd_packed_kernel(AttnParams p) {
  using C = PackCfg;
  constexpr int D = C::D, BN = C::BN, KB = C::KB, HB = C::HB;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* sq = smem;
  float* red = reinterpret_cast<float*>(smem + C::OFF_RED);
  uint8_t* svalid = smem + C::OFF_VALID;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + C::OFF_BAR + 8);
  int* s_abort = reinterpret_cast<int*>(smem + C::OFF_BAR + 12);
  auto stage_k = [&](int s) { return smem + C::OFF_K + s * 2 * C::KV_BYTES; };
  auto stage_v = [&](int s) { return smem + C::OFF_K + s * 2 * C::KV_BYTES + C::KV_BYTES; };

  const int h = blockIdx.x;
  const int b0 = 2 * blockIdx.y;
  const int kvh = h / (p.H / p.Hkv);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int row = tid & (BM - 1), half = tid >> 7;
  const int seq = row >> 6, t = row & 63;
  const int b = b0 + seq;
  const bool row_seq = b < p.B;  // the second sequence may not exist (odd B)
  const int mlen0 = p.mem_len != nullptr ? p.mem_len[b0] : 0;
  const int mlen1 = (p.mem_len != nullptr && b0 + 1 < p.B) ? p.mem_len[b0 + 1] : 0;
  const int n_mem = (max(mlen0, mlen1) + KB - 1) / KB;
  const int n_blocks = n_mem + 1;

  if (warp == 0) {
    tc::alloc(s_tmem, TMEM_COLS);
    tc::relinquish();
  }
  if (tid == 0) {
    mbar_init(bar, 1);
    *s_abort = 0;
    tc::fence_mbarrier_init();
  }
  // Q rows: tile row r -> (b0 + r / 64, token r % 64)
#pragma unroll
  for (int it = 0; it < BM * (D / 8) / NT; ++it) {
    const int i = it * NT + tid;
    const int c = (i >> 3) % (D / 8), r = (i / D) * 8 + (i & 7);
    const int bb = b0 + (r >> 6), tt = r & 63;
    const bool ok = bb < p.B && tt < p.T;
    cp_async16(sq + tc::core_off(r, c, BM), ok ? p.q + bb * p.q_batch + (int64_t)tt * p.q_row + h * D + c * 8 : p.q,
               ok);
  }
  // K/V block j: tile row r -> key (r % 64) of block j of sequence r / 64
  auto load_block_packed = [&](int j, int s) {
    const bool memory = j < n_mem;
    uint8_t* sk = stage_k(s);
    uint8_t* sv = stage_v(s);
    if (!memory && p.key_valid != nullptr && tid < BN) {
      const int bb = b0 + (tid >> 6), tt = tid & 63;
      svalid[s * BN + tid] = (bb < p.B && tt < p.T) ? p.key_valid[(int64_t)bb * p.T + tt] : 0;
    }
    const int c = (tid >> 3) % (D / 8);
#pragma unroll
    for (int it = 0; it < BN * (D / 8) / NT; ++it) {
      const int i = it * NT + tid;
      const int r = (i / D) * 8 + (i & 7);
      const int sq_ = r >> 6, kk = r & 63, bb = b0 + sq_;
      const __nv_bfloat16* ks = p.k;
      const __nv_bfloat16* vs = p.v;
      bool ok = false;
      if (bb < p.B) {
        if (memory) {
          const int jj = j * KB + kk;
          ok = jj < (sq_ ? mlen1 : mlen0);
          if (ok) {
            const int64_t off = (int64_t)__ldg(p.mem_idx + (int64_t)bb * p.mem_max + jj) * p.mem_row + kvh * D + c * 8;
            ks = p.mem_k + off;
            vs = p.mem_v + off;
          }
        } else {
          ok = kk < p.T;
          if (ok) {
            ks = p.k + bb * p.k_batch + (int64_t)kk * p.k_row + kvh * D + c * 8;
            vs = p.v + bb * p.v_batch + (int64_t)kk * p.v_row + kvh * D + c * 8;
          }
        }
      }
      const uint32_t o = tc::core_off(r, c, BN);
      cp_async16(sk + o, ks, ok);
      cp_async16(sv + o, vs, ok);
    }
  };
  load_block_packed(0, 0);
  cp_async_commit();
  cp_async_wait<0>();
  fence_proxy_async_smem();
  tc::fence_before();
  __syncthreads();
  tc::fence_after();

  const uint32_t tmem = *s_tmem;
  const uint32_t lane = (uint32_t)((warp & 3) * 32) << 16;
  const int col0 = seq * KB + half * HB;  // this thread's 32 S columns (its own sequence's keys)
  const uint32_t t_s = tmem + lane + col0;
  const uint32_t t_o = tmem + lane + C::O_COL + half * (D / 2);
  const uint32_t t_p = tmem + lane + C::P_COL + col0 / 2;
  {
    // the other sequence's half of this row's P stays zero for the whole loop
    uint32_t z[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) z[i] = 0u;
    tc::st16(tmem + lane + C::P_COL + ((1 - seq) * KB + half * HB) / 2, z);
  }
  constexpr uint32_t ID_S = tc::idesc_bf16(BM, BN, false);
  constexpr uint32_t ID_O = tc::idesc_bf16(BM, D, true);
  constexpr uint32_t Q_LBO = (BM / 8) * 128, KV_LBO = (BN / 8) * 128;
  const uint32_t q_addr = smem_u32(sq);
  auto issue_s = [&](int s) {
    const uint32_t k_addr = smem_u32(stage_k(s));
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk)
      tc::mma_bf16(tmem, tc::smem_desc(q_addr + kk * 2 * Q_LBO, Q_LBO, 128),
                   tc::smem_desc(k_addr + kk * 2 * KV_LBO, KV_LBO, 128), ID_S, kk > 0);
  };
  auto issue_o = [&](int s, bool acc) {
    const uint32_t v_addr = smem_u32(stage_v(s));
#pragma unroll
    for (int kk = 0; kk < BN / 16; ++kk)
      tc::mma_bf16_ts(tmem + C::O_COL, tmem + C::P_COL + kk * 8, tc::smem_desc(v_addr + kk * 2 * 128, 128, KV_LBO),
                      ID_O, (acc || kk > 0) ? 1u : 0u);
  };
  tc::fence_before();
  __syncthreads();  // P zeros stored before the first P V MMA
  tc::fence_after();
  if (tid == 0) {
    issue_s(0);
    tc::commit(bar);
  }

  const float sl2 = p.scale * LOG2E;
  float m_run = -INFINITY, l_run = 0.f;
  bool aborted = false;
  for (int j = 0; j < n_blocks; ++j) {
    const int s = j & 1;
    if (!tc::mbar_wait_cycles(bar, (uint32_t)(j & 1), WAIT_CYCLES)) *s_abort = 1;
    const bool memory = j < n_mem;
    if (j + 1 < n_blocks) {
      load_block_packed(j + 1, s ^ 1);
      cp_async_commit();
    }
    // visible keys among this thread's 32 columns (key index k = half * 32 + c in its sequence)
    int lim;
    const uint8_t* valid = nullptr;
    if (!row_seq) {
      lim = 0;
    } else if (memory) {
      lim = (seq ? mlen1 : mlen0) - j * KB - half * HB;
    } else {
      lim = min(p.T, t + 1) - half * HB;
      if (p.key_valid != nullptr) valid = svalid + s * BN + col0;
    }
    const bool masked = lim < HB || valid != nullptr;
    float mx = -INFINITY;
    uint32_t r[32];
    tc::ld32(t_s, r);
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      if (masked && !(i < lim && (valid == nullptr || valid[i] != 0))) r[i] = __float_as_uint(-INFINITY);
    }
#pragma unroll
    for (int i = 0; i < 32; i += 2) mx = max3(mx, __uint_as_float(r[i]), __uint_as_float(r[i + 1]));
    red[half * BM + row] = mx;
    pair_sync(warp);
    mx = fmaxf(mx, red[(half ^ 1) * BM + row]);
    float corr = 1.f;
    bool rescale = false;
    if (mx > m_run) {
      if (m_run == -INFINITY) {
        m_run = mx;
      } else if ((mx - m_run) * sl2 > RESCALE_LOG2) {
        corr = ex2((m_run - mx) * sl2);
        l_run *= corr;
        m_run = mx;
        rescale = true;
      }
    }
    if (j > 0 && __any_sync(0xffffffffu, rescale)) {
      uint32_t o[32];
      tc::ld32(t_o, o);
#pragma unroll
      for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * corr);
      tc::st32(t_o, o);
    }
    const float ms = m_run == -INFINITY ? 0.f : m_run * sl2;
    const float2 sl2x2 = make_float2(sl2, sl2), nms = make_float2(-ms, -ms);
    float2 acc = make_float2(0.f, 0.f);
    uint32_t w[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float2 x = fma2(make_float2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1])), sl2x2, nms);
      x.x = ex2(x.x);
      x.y = ex2(x.y);
      acc = add2(acc, x);
      w[i] = pack_bf16(x.x, x.y);
    }
    tc::st16(t_p, w);
    l_run += acc.x + acc.y;

    if (j + 1 < n_blocks) cp_async_wait<0>();
    fence_proxy_async_smem();
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    if (*s_abort) {
      aborted = true;
      break;
    }
    if (tid == 0) {
      issue_o(s, j > 0);
      if (j + 1 < n_blocks) issue_s(s ^ 1);
      tc::commit(bar);
    }
  }

  if (!aborted) {
    if (!tc::mbar_wait_cycles(bar, (uint32_t)(n_blocks & 1), WAIT_CYCLES)) aborted = true;
  }
  aborted = __syncthreads_or(aborted);
  red[half * BM + row] = l_run;
  pair_sync(warp);
  const float l_tot = l_run + red[(half ^ 1) * BM + row];
  if (!aborted) {
    const float inv = l_tot > 0.f ? 1.f / l_tot : 0.f;
    uint32_t o[32];
    tc::ld32(t_o, o);
    if (row_seq && t < p.T) {
      __nv_bfloat16* dst = p.o + b * p.o_batch + (int64_t)t * p.o_row + h * D + half * (D / 2);
#pragma unroll
      for (int i = 0; i < 32; i += 8) {
        uint4 v;
        v.x = pack_bf16(__uint_as_float(o[i + 0]) * inv, __uint_as_float(o[i + 1]) * inv);
        v.y = pack_bf16(__uint_as_float(o[i + 2]) * inv, __uint_as_float(o[i + 3]) * inv);
        v.z = pack_bf16(__uint_as_float(o[i + 4]) * inv, __uint_as_float(o[i + 5]) * inv);
        v.w = pack_bf16(__uint_as_float(o[i + 6]) * inv, __uint_as_float(o[i + 7]) * inv);
        *reinterpret_cast<uint4*>(dst + i) = v;
      }
      if (half == 0)
        p.lse[((int64_t)b * p.H + h) * p.T + t] = l_tot > 0.f ? m_run * p.scale + logf(l_tot) : -INFINITY;
    }
  } else {
    if (tid == 0 && p.status != nullptr) atomicExch(p.status, 1);
    cp_async_wait<0>();
    tc::mbar_wait_cycles(bar, (uint32_t)(n_blocks & 1), WAIT_CYCLES);
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after();
    tc::dealloc(tmem, TMEM_COLS);
  }
}

template <int D>
cudaError_t launch(const AttnParams& p, cudaStream_t st) {
  constexpr int smem = Cfg<D>::SMEM;
  PRA_RETURN_IF_ERROR(pra::set_max_dynamic_smem(reinterpret_cast<const void*>(fwd_kernel<D>), smem));
  dim3 grid(p.H * p.B, (p.T + BM - 1) / BM);
  fwd_kernel<D><<<grid, NT, smem, st>>>(p);
  return cudaGetLastError();
}

}  // namespace attn_tc
}  // namespace pra

// dQ of the backward on tcgen05 (head dim 64, 16-byte aligned rows); cudaErrorNotSupported
// otherwise.  Needs p.delta (sum_d dO * O per row) computed first.
cudaError_t pra_attention_bwd_dq_tc(const AttnParams& p, int head_dim, cudaStream_t st) {
  using namespace pra::attn_tc;
  auto aligned = [](const void* ptr, int64_t a, int64_t b_) {
    return (reinterpret_cast<uintptr_t>(ptr) % 16) == 0 && a % 8 == 0 && b_ % 8 == 0;
  };
  if (head_dim != 64 || !aligned(p.q, p.q_row, p.q_batch) || !aligned(p.k, p.k_row, p.k_batch) ||
      !aligned(p.v, p.v_row, p.v_batch) || !aligned(p.dout, p.do_row, p.do_batch) ||
      !aligned(p.dq, p.dq_row, p.dq_batch))
    return cudaErrorNotSupported;
  if (p.mem_idx != nullptr && (!aligned(p.mem_k, p.mem_row, 0) || !aligned(p.mem_v, p.mem_row, 0)))
    return cudaErrorNotSupported;
  constexpr int smem = DqCfg::SMEM;
  PRA_RETURN_IF_ERROR(pra::set_max_dynamic_smem(reinterpret_cast<const void*>(bwd_dq_kernel), smem));
  dim3 grid(p.H * p.B, (p.T + BM - 1) / BM);
  bwd_dq_kernel<<<grid, NT, smem, st>>>(p);
  return cudaGetLastError();
}

// dK / dV of the local keys on tcgen05 (head dim 64, MHA, 16-byte aligned rows);
// cudaErrorNotSupported otherwise.  Needs p.delta.
cudaError_t pra_attention_bwd_dkdv_tc(const AttnParams& p, int head_dim, cudaStream_t st) {
  using namespace pra::attn_tc;
  auto aligned = [](const void* ptr, int64_t a, int64_t b_) {
    return (reinterpret_cast<uintptr_t>(ptr) % 16) == 0 && a % 8 == 0 && b_ % 8 == 0;
  };
  if (head_dim != 64 || p.H != p.Hkv || !aligned(p.q, p.q_row, p.q_batch) || !aligned(p.k, p.k_row, p.k_batch) ||
      !aligned(p.v, p.v_row, p.v_batch) || !aligned(p.dout, p.do_row, p.do_batch) ||
      !aligned(p.dk, p.dk_row, p.dk_batch) || !aligned(p.dv, p.dv_row, p.dv_batch))
    return cudaErrorNotSupported;
  constexpr int smem = DkvCfg::SMEM;
  PRA_RETURN_IF_ERROR(pra::set_max_dynamic_smem(reinterpret_cast<const void*>(bwd_dkdv_kernel), smem));
  dim3 grid(p.H * p.B, (p.T + DkvCfg::BK - 1) / DkvCfg::BK);
  bwd_dkdv_kernel<<<grid, NT, smem, st>>>(p);
  return cudaGetLastError();
}

// The tcgen05 forward takes head dims 64 and 128 with 16-byte aligned rows; returns
// cudaErrorNotSupported for anything else so the caller can use the mma.sync kernel.
cudaError_t pra_attention_fwd_tc(const AttnParams& p, int head_dim, cudaStream_t st) {
  using namespace pra::attn_tc;
  auto aligned = [](const void* ptr, int64_t a, int64_t b_) {
    return (reinterpret_cast<uintptr_t>(ptr) % 16) == 0 && a % 8 == 0 && b_ % 8 == 0;
  };
  if (!aligned(p.q, p.q_row, p.q_batch) || !aligned(p.k, p.k_row, p.k_batch) || !aligned(p.v, p.v_row, p.v_batch) ||
      !aligned(p.o, p.o_row, p.o_batch))
    return cudaErrorNotSupported;
  if (p.mem_idx != nullptr && (!aligned(p.mem_k, p.mem_row, 0) || !aligned(p.mem_v, p.mem_row, 0)))
    return cudaErrorNotSupported;
  if (head_dim == 64 && p.T <= 64) {  // two sequences per 128-query tile
    constexpr int smem = PackCfg::SMEM;
    PRA_RETURN_IF_ERROR(pra::set_max_dynamic_smem(reinterpret_cast<const void*>(fwd_packed_kernel), smem));
    dim3 grid(p.H, (p.B + 1) / 2);
    fwd_packed_kernel<<<grid, NT, smem, st>>>(p);
    return cudaGetLastError();
  }
  switch (head_dim) {
    case 64: return launch<64>(p, st);
    case 128: return launch<128>(p, st);
    default: return cudaErrorNotSupported;
  }
}
