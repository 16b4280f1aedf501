// Data-parallel gradient all-reduce fused with the bf16 -> fp32 cast and the 1/world scale,
// done with peer loads and stores over NVLink (no NCCL, no staging copy).
//
// Every rank's flat bf16 gradient buffer and fp32 output buffer live in symmetric
// memory, so each rank holds device pointers to all of them.  One launch handles an
// element range [offset, offset + count) (the whole buffer, or one bucket):
//   1. entry barrier: CTA b of every rank signals CTA b of every peer, then waits for
//      all peers' signals (the peers' backward kernels have completed, their gradient
//      writes are visible system wide);
//   2. reduce-scatter + all-gather in one pass: rank r owns the r-th slice of the
//      range; for each 16-byte vector of its slice it loads the 8 bf16 values of every
//      rank (ranks summed in a fixed order, so the result does not depend on the
//      reducing rank), scales, and stores the vector into EVERY rank's output: fp32 into
//      dst, or (in_place_bf16) bf16 back into the gradient buffers themselves.  In place
//      is race free: only the owner of a vector reads or writes it during the pass, and it
//      loads every rank's value before it stores.  bf16 stores move 2 bytes per element
//      and peer instead of 4;
//   3. exit barrier: the same handshake again, so a rank's output is complete (and its
//      gradient buffer no longer read) once its own launch has finished.
// Each wait polls at most `max_spins` times; on a timeout the CTA records
// `error = 1 + phase`, skips the rest and returns, leaving the context usable.
#include "common.cuh"

namespace pra {
namespace dp {

constexpr int NT = 512;

__device__ __forceinline__ void signal_store(uint32_t* addr, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(addr), "r"(v) : "memory");
}

// Barrier among CTA `blockIdx.x` of every rank; returns false on a timeout.
__device__ bool cta_barrier(const DpArgs& a, int phase) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  const int slot = (phase * gridDim.x + blockIdx.x) * a.world;
  if (threadIdx.x < a.world) {
    __threadfence_system();
    signal_store(a.sig[threadIdx.x] + slot + a.rank, a.epoch);
    if (!bounded_wait_geq(a.sig[a.rank] + slot + threadIdx.x, a.epoch, a.max_spins)) {
      ok = 0;
      atomicExch(a.error, 1 + phase);
    }
  }
  __syncthreads();
  return ok != 0;
}

__global__ void __launch_bounds__(NT) allreduce_kernel(DpArgs a) {
  if (!cta_barrier(a, 0)) return;
  // this rank's slice of the range, in 8-element vectors
  const int64_t vecs = a.count / 8;
  const int64_t per = (vecs + a.world - 1) / a.world;
  const int64_t v0 = a.rank * per, v1 = min(vecs, v0 + per);
  const int64_t base = a.offset / 8;
  for (int64_t v = v0 + (int64_t)blockIdx.x * NT + threadIdx.x; v < v1; v += (int64_t)gridDim.x * NT) {
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    for (int p = 0; p < a.world; ++p) {
      const uint4 raw = reinterpret_cast<const uint4*>(a.src[p])[base + v];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h[i]);
        acc[2 * i] += f.x;
        acc[2 * i + 1] += f.y;
      }
    }
    if (a.in_place_bf16) {
      uint4 packed;
      packed.x = pack_bf16(acc[0] * a.scale, acc[1] * a.scale);
      packed.y = pack_bf16(acc[2] * a.scale, acc[3] * a.scale);
      packed.z = pack_bf16(acc[4] * a.scale, acc[5] * a.scale);
      packed.w = pack_bf16(acc[6] * a.scale, acc[7] * a.scale);
      for (int p = 0; p < a.world; ++p)
        reinterpret_cast<uint4*>(const_cast<__nv_bfloat16*>(a.src[p]))[base + v] = packed;
      continue;
    }
    const float4 lo = make_float4(acc[0] * a.scale, acc[1] * a.scale, acc[2] * a.scale, acc[3] * a.scale);
    const float4 hi = make_float4(acc[4] * a.scale, acc[5] * a.scale, acc[6] * a.scale, acc[7] * a.scale);
    for (int p = 0; p < a.world; ++p) {
      float4* out = reinterpret_cast<float4*>(a.dst[p]) + 2 * (base + v);
      out[0] = lo;
      out[1] = hi;
    }
  }
  cta_barrier(a, 1);
}

}  // namespace dp
}  // namespace pra

int pra_dp_allreduce_blocks() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
    sms = 148;
  return 2 * sms;
}

cudaError_t pra_dp_allreduce(const DpArgs& a, cudaStream_t st) {
  if (a.world < 1 || a.world > DP_MAX_RANKS || a.rank < 0 || a.rank >= a.world) return cudaErrorInvalidValue;
  if (a.offset % 8 != 0 || a.count % 8 != 0 || a.count < 0) return cudaErrorInvalidValue;
  for (int p = 0; p < a.world; ++p) {
    if ((reinterpret_cast<uintptr_t>(a.src[p]) & 15) || a.sig[p] == nullptr ||
        (!a.in_place_bf16 && (a.dst[p] == nullptr || (reinterpret_cast<uintptr_t>(a.dst[p]) & 15))))
      return cudaErrorInvalidValue;
  }
  const int blocks = a.blocks > 0 && a.blocks < pra_dp_allreduce_blocks() ? a.blocks : pra_dp_allreduce_blocks();
  pra::dp::allreduce_kernel<<<blocks, pra::dp::NT, 0, st>>>(a);
  return cudaGetLastError();
}
