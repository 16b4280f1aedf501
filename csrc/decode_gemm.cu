// Decode GEMMs on the 5th-generation tensor cores, with the row-parallel all-reduce fused in.
//
// Decode multiplies few token rows (M <= 64) by large weights, so the weight stream is the
// whole cost.  Each CTA owns 128 output features (one weight slab) and, with split-K, a range
// of the reduction; the MMA is "swapped": A = the weight tile (128 features x 64 K, K-major),
// B = the token rows (M x 64 K, K-major), so the fp32 accumulator in TMEM is D^T[feature][token]
// with one TMEM lane per output feature.  Both operands stream through a ring of 2-D TMA tiles
// in the 128-byte swizzle layout (64 K elements per row; 4 stages at two CTAs per SM, 6 at one,
// 2 for the small-footprint fp32-score launches): one thread issues the copies against "full"
// mbarriers, one thread issues the MMAs and releases each stage through its "empty" mbarrier
// (tcgen05.commit).  Under programmatic dependent launch the weight tiles of the first stages
// are requested before griddepcontrol.wait, while the previous kernel drains.
//
// Epilogues (the accumulator is staged through shared memory as fp32 [token][feature] so every
// global access is a 16-byte row chunk):
//  * plain: + bias, + residual, bf16 store; columns >= split_col go to a second output (the
//    routing query rows appended to a QKV weight land in their own buffer);
//  * rotary QKV: q / k rotated and scattered into the query buffer and the cache rows, v into
//    its cache rows, the routing-query columns into their own buffer;
//  * SwiGLU: a [64 gate | 64 up]-interleaved weight tile yields 64 silu(gate) * up outputs;
//  * fp32 scores (routing);
//  * folded RMSNorm: a consumer scales its rows by rsqrt(mean square + eps) from the per-tile
//    sums of squares its producer (a residual-adding epilogue) wrote;
//  * split-K: the splits of a tile run as one thread-block cluster; each stages its fp32
//    partial in shared memory, and after a cluster barrier each CTA sums a slice of the token
//    rows over all splits' partials through distributed shared memory and finishes those rows
//    (no global workspace, no atomics, the epilogue spread over the splits);
//  * fused all-reduce (tensor-parallel row-parallel projection, world > 1): each CTA pushes
//    its rows of the bf16 partial tile into every rank's receive buffer (plain NVLink peer
//    stores), raises the (tile, row slice) flag on every rank with a release store, waits
//    (bounded) for every rank's flag of the same slice, then adds the residual to the sum of
//    all ranks' partials.  Slice (j, r) of every rank meets slice (j, r) of every peer, so no
//    grid-wide barrier is needed, and the per-slice call counters live in device memory
//    (graph capture replays stay in step).
//    Callers alternate two receive/flag halves between calls, so a rank that runs ahead
//    never writes a half its peers may still be reading.
#include <cuda.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace pra {
namespace dg {

constexpr int NT = 128;   // 4 warps: TMEM lanes 0..127 are the tile's 128 output features
constexpr int BF = 128;   // output features per tile
constexpr int BK = 64;    // reduction depth per stage: one 128-byte swizzle atom of bf16
constexpr int MT = 64;    // token rows per tile (MMA N)
// pipeline depth: a template parameter of the kernel (6: one CTA per SM; 4: two CTAs per SM)
constexpr int A_BYTES = BF * BK * 2;  // 16 KB
constexpr int B_BYTES = MT * BK * 2;  // 8 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
template <int STAGES>
struct Ring {
  static_assert(STAGES * STAGE_BYTES >= (MT * BF + MT + MT * (BF / 8)) * 4,
                "the epilogue stages the fp32 tile, the row scales and the chunk sums in the ring");
  static constexpr int OFF_BAR = STAGES * STAGE_BYTES;
  static constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;  // + barriers, + alignment slack for the 1024-byte atoms
  };
constexpr int TMEM_COLS = MT;
constexpr long long WAIT_CYCLES = 4000000000LL;  // about two seconds at the boost clock

__device__ __forceinline__ void signal_store(uint32_t* addr, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(addr), "r"(v) : "memory");
}

// ---- thread-block cluster: the split-K CTAs of one output tile
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
  return r;
}

// Address of the same shared-memory location in cluster CTA `rank`.
__device__ __forceinline__ uint32_t dsmem_map(uint32_t local, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(out) : "r"(local), "r"(rank));
  return out;
}

__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];\n"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// Shared-memory descriptor of a K-major bf16 tile in the 128-byte swizzle layout TMA writes:
// rows of 128 bytes (64 K elements) in 1024-byte atoms of 8 rows (SBO = 1024); the K offset
// within the atom moves the start address by 32 bytes per 16 elements.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
  uint64_t d = (uint64_t)((addr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;            // leading byte offset (unused by swizzled K-major layouts)
  d |= (uint64_t)(1024 >> 4) << 32;  // stride byte offset: 8 rows x 128 bytes
  d |= (uint64_t)1 << 46;            // descriptor version
  d |= (uint64_t)2 << 61;            // 128-byte swizzle
  return d;
}

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 raw = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

__device__ __forceinline__ void staged8(const float* p, float (&v)[8]) {
  const float4 lo = reinterpret_cast<const float4*>(p)[0], hi = reinterpret_cast<const float4*>(p)[1];
  v[0] = lo.x, v[1] = lo.y, v[2] = lo.z, v[3] = lo.w, v[4] = hi.x, v[5] = hi.y, v[6] = hi.z, v[7] = hi.w;
}

__device__ __forceinline__ uint4 pack8(const float (&v)[8]) {
  uint4 out;
  uint32_t* o = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i] = pack_bf16(v[2 * i], v[2 * i + 1]);
  return out;
}

template <int STAGES>
__global__ void __launch_bounds__(NT) decode_gemm_kernel(const __grid_constant__ CUtensorMap map_w,
                                                          const __grid_constant__ CUtensorMap map_x, DecodeGemmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  // the swizzle atoms need 1024-byte alignment
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Ring<STAGES>::OFF_BAR);
  uint64_t* empty = full + STAGES;
  uint64_t* done = empty + STAGES;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(done + 1);
  uint32_t* s_epoch = s_tmem + 1;
  int* s_flag = reinterpret_cast<int*>(s_tmem + 2);  // [0] a wait gave up, [1] last split, [2] peer wait gave up
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int n0 = tile * BF;
  const int nkb = a.K / BK;
  const int per = (nkb + a.splits - 1) / a.splits;
  const int kb0 = split * per, kb1 = min(nkb, kb0 + per);
  const int nk = kb1 - kb0;  // >= 1: the host sizes splits so every split has work

  if (warp == 0) {
    tc::alloc(s_tmem, TMEM_COLS);
    tc::relinquish();
  }
  if (tid == 32) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    mbar_init(done, 1);
    s_flag[0] = s_flag[1] = s_flag[2] = 0;
    tc::fence_mbarrier_init();
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *s_tmem;

  pdl_launch_dependents();
  if (warp == 0 && lane == 0) {  // TMA producer
    asm volatile("prefetch.tensormap [%0];\n" ::"l"(&map_w) : "memory");
    asm volatile("prefetch.tensormap [%0];\n" ::"l"(&map_x) : "memory");
    // the weight tiles of the first stages do not depend on the kernels before: under a
    // programmatic dependent launch they stream in while those kernels drain
    const int pre = min(nk, STAGES);
    for (int kb = 0; kb < pre; ++kb) {
      expect_tx(full + kb, STAGE_BYTES);
      tma_load(smem + kb * STAGE_BYTES, &map_w, (kb0 + kb) * BK, n0, full + kb);
    }
    pdl_wait();  // the token rows are the previous kernel's output
    for (int kb = 0; kb < pre; ++kb) tma_load(smem + kb * STAGE_BYTES + A_BYTES, &map_x, (kb0 + kb) * BK, 0, full + kb);
    for (int kb = pre; kb < nk; ++kb) {
      const int slot = kb % STAGES;
      if (kb >= STAGES && !tc::mbar_wait_cycles(empty + slot, (uint32_t)((kb / STAGES - 1) & 1), WAIT_CYCLES)) {
        s_flag[0] = 1;
        break;
      }
      uint8_t* st = smem + slot * STAGE_BYTES;
      expect_tx(full + slot, STAGE_BYTES);
      tma_load(st, &map_w, (kb0 + kb) * BK, n0, full + slot);
      tma_load(st + A_BYTES, &map_x, (kb0 + kb) * BK, 0, full + slot);
    }
  } else if (warp == 1 && lane == 0) {  // MMA issuer
    constexpr uint32_t IDESC = tc::idesc_bf16(BF, MT, false);
    for (int kb = 0; kb < nk; ++kb) {
      const int slot = kb % STAGES;
      if (!tc::mbar_wait_cycles(full + slot, (uint32_t)((kb / STAGES) & 1), WAIT_CYCLES)) {
        s_flag[0] = 1;
        break;
      }
      tc::fence_after();
      const uint32_t a_addr = smem_u32(smem + slot * STAGE_BYTES), b_addr = a_addr + A_BYTES;
#pragma unroll
      for (int kk = 0; kk < BK / 16; ++kk)
        tc::mma_bf16(tmem, sw128_desc(a_addr + kk * 32), sw128_desc(b_addr + kk * 32), IDESC,
                     (kb > 0 || kk > 0) ? 1u : 0u);
      tc::commit(empty + slot);
    }
    tc::commit(done);
  }
  // everyone: the accumulator is complete once `done` fires
  if (!tc::mbar_wait_cycles(done, 0, WAIT_CYCLES)) s_flag[0] = 1;
  pdl_wait();  // before the epilogue's reads (residual, workspace) and every global write
  tc::fence_after();
  __syncthreads();
  const bool timed_out = s_flag[0] != 0;
  float acc[MT];
  if (!timed_out) {
    uint32_t r[MT];
    tc::ld64(tmem + ((uint32_t)(warp * 32) << 16), r);
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m] = __uint_as_float(r[m]);
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) tc::dealloc(tmem, TMEM_COLS);
  if (timed_out) {
    if (tid == 0 && a.error) atomicExch(a.error, 1);
    if (a.splits > 1) {  // the cluster's other CTAs still meet this one at both cluster barriers
      cluster_sync();
      cluster_sync();
    }
    return;
  }
  const int feat = tid;  // this thread's output feature within the tile (TMEM lane)

  // ---- stage the fp32 tile as [token][feature] so every global access is a 16-byte row chunk
  float* tile_s = reinterpret_cast<float*>(smem);
#pragma unroll
  for (int m = 0; m < MT; ++m) tile_s[m * BF + feat] = acc[m];
  // ---- split-K: the splits of a tile are one thread-block cluster.  Each CTA sums a slice of
  // the token rows over every split's staged partial through distributed shared memory (split
  // order, so every rank and every call sums identically) and finishes those rows itself.
  const int S = a.splits;
  const int r = S > 1 ? (int)cluster_rank() : 0;
  const int m_lo = r * a.M / S, m_hi = (r + 1) * a.M / S;
  if (S > 1) {
    cluster_sync();  // every split's partial is staged
    for (int i = tid; i < (m_hi - m_lo) * (BF / 4); i += NT) {
      float* at = tile_s + (m_lo + i / (BF / 4)) * BF + (i % (BF / 4)) * 4;
      const uint32_t local = smem_u32(at);
      float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int q = 0; q < S; ++q) {
        const float4 v = ld_dsmem_f4(dsmem_map(local, (uint32_t)q));
        sum.x += v.x, sum.y += v.y, sum.z += v.z, sum.w += v.w;
      }
      *reinterpret_cast<float4*>(at) = sum;  // rows [m_lo, m_hi) are read remotely by nobody
    }
    cluster_sync();  // no CTA leaves (or reuses its shared memory) while another reads it
  } else {
    __syncthreads();
  }
  const int c_lo = m_lo * (BF / 8), c_hi = m_hi * (BF / 8);  // this CTA's 8-feature row chunks
  float* s_rstd = tile_s + MT * BF;  // [MT] folded-norm row scales
  float* s_part = s_rstd + MT;       // [MT][BF / 8] per-chunk sums of squares (producer)
  if (a.ss_in != nullptr) {  // folded RMSNorm: scale this CTA's rows by their rsqrt(mean square)
    for (int m = m_lo + tid; m < m_hi; m += NT) {
      float t = 0.f;
      for (int k = 0; k < a.ss_tiles; ++k) t += a.ss_in[k * MT + m];
      s_rstd[m] = rsqrtf(t / (float)a.ss_dim + a.ss_eps);
    }
    __syncthreads();
    for (int i = m_lo * BF + tid; i < m_hi * BF; i += NT) tile_s[i] *= s_rstd[i / BF];
    __syncthreads();
  }
  // producer side: sum of squares of the bf16 values stored, per (row, chunk), then per row in order
  auto ss_chunk = [&](int m, int c, const uint4& packed) {
    if (a.ss_out == nullptr) return;
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&packed);
    float t = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      t += f.x * f.x + f.y * f.y;
    }
    s_part[m * (BF / 8) + c] = t;
  };
  auto ss_finish = [&]() {
    if (a.ss_out == nullptr) return;
    __syncthreads();
    for (int m = m_lo + tid; m < m_hi; m += NT) {
      float t = 0.f;
      for (int c = 0; c < BF / 8; ++c) t += s_part[m * (BF / 8) + c];
      a.ss_out[tile * MT + m] = t;
    }
  };

  if (a.world <= 1 && a.pos != nullptr) {  // decode QKV: bias, rotary, scatter into q / caches / routing query
    const int half = a.head_dim / 2;
    for (int i = c_lo + tid; i < c_hi; i += NT) {
      const int m = i / (BF / 8), c = i % (BF / 8), n = n0 + c * 8;
      if (n >= a.N) continue;
      float v[8];
      staged8(tile_s + m * BF + c * 8, v);
      float b[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (a.bias) load8(a.bias + n, b);
      if (n < a.k_end) {  // query or key head: rotate pairs (i, i + half) of each head
        const int p = a.pos[m];
        float rr[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int f = c * 8 + j, hi = (n + j) % a.head_dim;  // tile-local feature, index within its head
          const bool first = hi < half;
          const int partner = first ? f + half : f - half;
          const float x = v[j] + b[j];
          const float xp = tile_s[m * BF + partner] + (a.bias ? __bfloat162float(a.bias[n0 + partner]) : 0.f);
          const int ii = first ? hi : hi - half;
          const float cs = a.cos_t[(int64_t)p * half + ii], sn = a.sin_t[(int64_t)p * half + ii];
          rr[j] = first ? x * cs - xp * sn : x * cs + xp * sn;
        }
        __nv_bfloat16* dst = n < a.q_end ? a.q_out + (int64_t)m * a.ldq + n
                                         : a.k_cache + (int64_t)a.cache_rows[m] * a.ld_cache + (n - a.q_end);
        *reinterpret_cast<uint4*>(dst) = pack8(rr);
        continue;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] += b[j];
      __nv_bfloat16* dst = n < a.split_col ? a.v_cache + (int64_t)a.cache_rows[m] * a.ld_cache + (n - a.k_end)
                                           : a.out2 + (int64_t)m * a.ldo2 + (n - a.split_col);
      *reinterpret_cast<uint4*>(dst) = pack8(v);
    }
    return;
  }

  if (a.swiglu) {  // [64 gate | 64 up] features -> 64 SwiGLU outputs per row
    for (int i = m_lo * 8 + tid; i < m_hi * 8; i += NT) {
      const int m = i / 8, c = i % 8, n = tile * (BF / 2) + c * 8;
      float g[8], u[8], v[8];
      staged8(tile_s + m * BF + c * 8, g);
      staged8(tile_s + m * BF + BF / 2 + c * 8, u);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = g[j] / (1.f + __expf(-g[j])) * u[j];
      *reinterpret_cast<uint4*>(a.out + (int64_t)m * a.ldo + n) = pack8(v);
    }
    return;
  }

  if (a.out_f32 != nullptr) {  // fp32 results (routing scores): 2 x 16-byte stores per chunk
    for (int i = c_lo + tid; i < c_hi; i += NT) {
      const int m = i / (BF / 8), c = i % (BF / 8), n = n0 + c * 8;
      if (n >= a.N) continue;
      const float4* src = reinterpret_cast<const float4*>(tile_s + m * BF + c * 8);
      float4* dst = reinterpret_cast<float4*>(a.out_f32 + (int64_t)m * a.ldo + n);
      dst[0] = src[0];
      dst[1] = src[1];
    }
    return;
  }

  if (a.world <= 1) {
    for (int i = c_lo + tid; i < c_hi; i += NT) {
      const int m = i / (BF / 8), c = i % (BF / 8), n = n0 + c * 8;
      if (n >= a.N) continue;
      float v[8];
      staged8(tile_s + m * BF + c * 8, v);
      if (a.bias) {
        float b[8];
        load8(a.bias + n, b);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] += b[j];
      }
      if (a.residual) {
        float rr[8];
        load8(a.residual + (int64_t)m * a.ldo + n, rr);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] += rr[j];
      }
      const bool second = a.out2 != nullptr && n >= a.split_col;
      __nv_bfloat16* dst = second ? a.out2 + (int64_t)m * a.ldo2 + (n - a.split_col) : a.out + (int64_t)m * a.ldo + n;
      const uint4 packed = pack8(v);
      *reinterpret_cast<uint4*>(dst) = packed;
      ss_chunk(m, c, packed);
    }
    ss_finish();
    return;
  }

  // ---- fused all-reduce: push this CTA's rows of the bf16 partial tile to every rank, raise
  // this (tile, row slice)'s flag on every rank, wait for every rank's flag of the same slice,
  // then sum the ranks' partials of those rows.  Row slices are the same on every rank (same
  // split count), so slice (j, r) of every rank meets slice (j, r) of every peer.
  const int slot = tile * DG_MAX_SPLITS + r;
  if (tid == 0) {
    const uint32_t e = a.epochs[slot] + 1;
    a.epochs[slot] = e;
    *s_epoch = e;
  }
  for (int i = c_lo + tid; i < c_hi; i += NT) {
    const int m = i / (BF / 8), c = i % (BF / 8), n = n0 + c * 8;
    if (n >= a.N) continue;
    float v[8];
    staged8(tile_s + m * BF + c * 8, v);
    const uint4 packed = pack8(v);
    const int64_t at = ((int64_t)a.rank * a.M + m) * a.N + n;
    for (int p = 0; p < a.world; ++p) *reinterpret_cast<uint4*>(a.recv[p] + at) = packed;
  }
  __syncthreads();
  const uint32_t epoch = *s_epoch;
  if (tid < a.world) {
    __threadfence_system();
    signal_store(a.flags[tid] + (int64_t)slot * a.world + a.rank, epoch);
  }
  if (tid < a.world) {
    if (!bounded_wait_geq(a.flags[a.rank] + (int64_t)slot * a.world + tid, epoch, a.max_spins)) {
      s_flag[2] = 1;
      atomicExch(a.error, 2);
    }
  }
  __syncthreads();
  if (s_flag[2]) return;
  for (int i = c_lo + tid; i < c_hi; i += NT) {
    const int m = i / (BF / 8), c = i % (BF / 8), n = n0 + c * 8;
    if (n >= a.N) continue;
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (a.residual) load8(a.residual + (int64_t)m * a.ldo + n, v);
    if (a.bias) {
      float b[8];
      load8(a.bias + n, b);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] += b[j];
    }
    for (int p = 0; p < a.world; ++p) {  // rank order: every rank sums identically
      float part[8];
      load8(a.recv[a.rank] + ((int64_t)p * a.M + m) * a.N + n, part);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] += part[j];
    }
    const uint4 packed = pack8(v);
    *reinterpret_cast<uint4*>(a.out + (int64_t)m * a.ldo + n) = packed;
    ss_chunk(m, c, packed);
  }
  ss_finish();
}

}  // namespace dg
}  // namespace pra

namespace {

// Tensor maps of [rows, cols] bf16 matrices (row stride ld elements) cut into 64-column x
// `box_rows` boxes in the 128-byte swizzle layout; cached by (address, shape) because weights
// are static and activation buffers repeat, and encoding costs microseconds of host time.
struct MapKey {
  const void* ptr;
  int64_t cols, rows, ld, box_rows;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && cols == o.cols && rows == o.rows && ld == o.ld && box_rows == o.box_rows;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<const void*>()(k.ptr) ^ (size_t)(k.cols * 1000003 + k.rows * 7919 + k.ld * 31 + k.box_rows);
  }
};

}  // namespace

const CUtensorMap* pra_tile_map_bf16(const void* ptr, int64_t cols, int64_t rows, int64_t ld, int box_rows) {
  static std::mutex mutex;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  const MapKey key{ptr, cols, rows, ld, box_rows};
  std::lock_guard<std::mutex> lock(mutex);
  auto it = cache.find(key);
  if (it != cache.end()) return &it->second;
  if (cache.size() > 4096) cache.clear();  // bounded: stale entries of freed buffers
  CUtensorMap map;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  const cuuint32_t box[2] = {(cuuint32_t)pra::dg::BK, (cuuint32_t)box_rows};
  const cuuint32_t elem[2] = {1, 1};
  if (cuTensorMapEncodeTiled(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, elem,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return nullptr;
  return &cache.emplace(key, map).first->second;
}

static int g_dg_ctas_per_sm = 2;
static int g_dg_min_kb = 8;
static int g_dg_max_splits = DG_MAX_SPLITS;
void pra_decode_gemm_configure(int ctas_per_sm, int min_blocks_per_split, int max_splits) {
  if (ctas_per_sm == 1 || ctas_per_sm == 2) g_dg_ctas_per_sm = ctas_per_sm;
  if (min_blocks_per_split >= 1) g_dg_min_kb = min_blocks_per_split;
  if (max_splits >= 1 && max_splits <= DG_MAX_SPLITS) g_dg_max_splits = max_splits;
}
int pra_decode_gemm_ctas_per_sm() { return g_dg_ctas_per_sm; }

int pra_decode_gemm_splits(int tiles, int nkb, int sms) {
  const int slots = sms * g_dg_ctas_per_sm;
  return std::max(1, std::min(std::min(nkb / g_dg_min_kb, slots / std::max(tiles, 1)), g_dg_max_splits));
}

// Whether `tiles` clusters of `splits` CTAs can all be resident at once (the fused all-reduce
// waits for its peers inside the kernel, so its whole grid must run concurrently).  Queried with
// the cluster shape alone; cached per (device, shape).
template <int STAGES>
static bool grid_fits(int tiles, int splits) {
  using namespace pra::dg;
  static std::mutex mu;
  static std::map<std::pair<int, int>, int> cache;  // (device, splits) -> resident clusters
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find({dev, splits});
  if (it == cache.end()) {
    cudaLaunchConfig_t q = {};
    q.gridDim = dim3(tiles, splits);
    q.blockDim = dim3(NT);
    q.dynamicSmemBytes = Ring<STAGES>::SMEM_BYTES;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = splits;
    attr[0].val.clusterDim.z = 1;
    q.attrs = attr;
    q.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, decode_gemm_kernel<STAGES>, &q) != cudaSuccess) {
      cudaGetLastError();  // clear; fall back to per-SM residency
      int per_sm = 0, sms = 0;
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_gemm_kernel<STAGES>, NT, Ring<STAGES>::SMEM_BYTES);
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      clusters = per_sm * sms / splits;
    }
    it = cache.emplace(std::make_pair(dev, splits), clusters).first;
  }
  return it->second >= tiles;
}

int pra_decode_gemm_resident_clusters(int splits) {
  const bool two = pra_decode_gemm_ctas_per_sm() == 2;
  for (int t = 1;; t *= 2) {  // the largest power-of-two tile count that fits (cached per shape)
    if (!(two ? grid_fits<4>(t, splits) : grid_fits<6>(t, splits))) return t / 2;
    if (t > 4096) return t;
  }
}

// Launch with the split-K cluster (1 x splits CTAs) and programmatic dependent launch.
template <int STAGES>
static cudaError_t launch_dg(const CUtensorMap& map_w, const CUtensorMap& map_x, const DecodeGemmArgs& b, int tiles,
                             cudaStream_t st) {
  using namespace pra::dg;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles, b.splits);
  cfg.blockDim = dim3(NT);
  cfg.dynamicSmemBytes = Ring<STAGES>::SMEM_BYTES;
  cfg.stream = st;
  cudaLaunchAttribute attr[3];
  int n = 0;
  if (b.splits > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = 1;
    attr[n].val.clusterDim.y = b.splits;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  n += pra_launch_attrs(attr + n);
  cfg.attrs = attr;
  cfg.numAttrs = n;
  if (b.world > 1 && !grid_fits<STAGES>(tiles, b.splits)) return cudaErrorInvalidConfiguration;
  return cudaLaunchKernelEx(&cfg, decode_gemm_kernel<STAGES>, map_w, map_x, b);
}

cudaError_t pra_decode_gemm(const DecodeGemmArgs& a, cudaStream_t st) {
  using namespace pra::dg;
  if (a.M <= 0 || a.N <= 0) return cudaSuccess;
  if (a.M > MT || a.K % BK || a.N % 8 || a.ldo % 8 || a.ldx % 8 || a.world > TP_MAX_RANKS) return cudaErrorInvalidValue;
  if (a.out2 && (a.split_col % 8 || a.ldo2 % 8)) return cudaErrorInvalidValue;
  if (a.pos && (a.world > 1 || a.head_dim <= 0 || BF % a.head_dim || a.q_end % a.head_dim || a.k_end % a.head_dim ||
                a.ldq % 8 || a.ld_cache % 8 || (a.split_col < a.N && a.out2 == nullptr) || !a.q_out || !a.k_cache ||
                !a.v_cache || !a.cache_rows || !a.cos_t || !a.sin_t))
    return cudaErrorInvalidValue;
  const int tiles = (a.N + BF - 1) / BF;
  if (tiles > DG_MAX_TILES) return cudaErrorInvalidValue;
  const int nkb = a.K / BK;
  int splits = std::min(std::max(a.splits, 1), std::min(nkb, DG_MAX_SPLITS));
  const int per = (nkb + splits - 1) / splits;
  splits = (nkb + per - 1) / per;  // no empty split
  if (a.world > 1 && (a.epochs == nullptr || a.error == nullptr)) return cudaErrorInvalidValue;
  if (a.out_f32 && (a.bias || a.residual || a.out2 || a.pos || a.world > 1 || a.ldo % 4)) return cudaErrorInvalidValue;
  if (a.swiglu && (a.N % BF || a.bias || a.residual || a.out2 || a.pos || a.out_f32 || a.world > 1))
    return cudaErrorInvalidValue;
  if (a.ss_out && (a.N % BF || a.out2 || a.pos || a.out_f32 || a.swiglu)) return cudaErrorInvalidValue;
  if (a.ss_in && (a.ss_tiles <= 0 || a.ss_dim <= 0 || a.out_f32)) return cudaErrorInvalidValue;
  static int configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    PRA_RETURN_IF_ERROR(cudaFuncSetAttribute(decode_gemm_kernel<6>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             Ring<6>::SMEM_BYTES));
    PRA_RETURN_IF_ERROR(cudaFuncSetAttribute(decode_gemm_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             Ring<4>::SMEM_BYTES));
    PRA_RETURN_IF_ERROR(cudaFuncSetAttribute(decode_gemm_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             Ring<2>::SMEM_BYTES));
    configured[dev] = 1;
  }
  if ((reinterpret_cast<uintptr_t>(a.w) | reinterpret_cast<uintptr_t>(a.x)) & 15) return cudaErrorInvalidValue;
  const CUtensorMap* map_w = pra_tile_map_bf16(a.w, a.K, a.N, a.K, BF);
  const CUtensorMap* map_x = pra_tile_map_bf16(a.x, a.K, a.M, a.ldx, MT);
  if (map_w == nullptr || map_x == nullptr) return cudaErrorInvalidValue;
  DecodeGemmArgs b = a;
  b.splits = splits;
  if (a.world > 1) {  // the fused all-reduce's grid must be resident at once: fewer splits until it is
    const bool two = pra_decode_gemm_ctas_per_sm() == 2;
    while (b.splits > 1 && !(two ? grid_fits<4>(tiles, b.splits) : grid_fits<6>(tiles, b.splits))) {
      const int per2 = (nkb + b.splits - 2) / (b.splits - 1);
      b.splits = (nkb + per2 - 1) / per2;
    }
    if (!(two ? grid_fits<4>(tiles, b.splits) : grid_fits<6>(tiles, b.splits))) return cudaErrorInvalidConfiguration;
  }
  if (a.out_f32 != nullptr) return launch_dg<2>(*map_w, *map_x, b, tiles, st);
  if (pra_decode_gemm_ctas_per_sm() == 2) return launch_dg<4>(*map_w, *map_x, b, tiles, st);
  return launch_dg<6>(*map_w, *map_x, b, tiles, st);
}
