// Tensor-parallel collectives over peer memory (one process per GPU, plain peer loads/stores).
//
//  * allreduce_oneshot: out = residual + sum over ranks of every rank's bf16 partial (the
//    row-parallel GEMM outputs), read straight from the peers' buffers in one pass; the
//    residual add and the bf16 rounding are fused.  Callers alternate two partial buffers,
//    so the entry barrier of call n+1 also proves every peer finished reading call n.
//  * allgather_cols: every rank stores its [rows, cols] fp32 slice into column block
//    `rank` of every rank's [rows, world * cols] buffer, then all ranks handshake, so the
//    full matrix is readable locally once the launch has finished.
// Barriers are per CTA (CTA b of every rank meets CTA b of every peer); every wait polls at
// most max_spins times and records `error = 1 + phase` on a timeout.
#include "common.cuh"

namespace pra {
namespace tp {

constexpr int NT = 512;

__device__ __forceinline__ void signal_store(uint32_t* addr, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(addr), "r"(v) : "memory");
}

// The epoch of each call comes from this CTA's own counter in local device memory (read,
// incremented and written back by the CTA itself), so the collectives can be captured in a
// CUDA graph and replayed: every rank launches identical grids, so CTA b's counters of all
// ranks advance in lockstep.
__device__ bool cta_barrier(uint32_t* const* sig, uint32_t* epochs, int rank, int world, long long max_spins,
                            int* error, int phase) {
  __shared__ int ok;
  __shared__ uint32_t epoch;
  if (threadIdx.x == 0) {
    ok = 1;
    epoch = epochs[blockIdx.x] + 1;
    epochs[blockIdx.x] = epoch;
  }
  __syncthreads();
  const int slot = blockIdx.x * world;
  if (threadIdx.x < world) {
    __threadfence_system();
    signal_store(sig[threadIdx.x] + slot + rank, epoch);
    if (!bounded_wait_geq(sig[rank] + slot + threadIdx.x, epoch, max_spins)) {
      ok = 0;
      atomicExch(error, 1 + phase);
    }
  }
  __syncthreads();
  return ok != 0;
}

__global__ void __launch_bounds__(NT) allreduce_oneshot_kernel(TpAllreduceArgs a) {
  if (!cta_barrier(a.sig, a.epochs, a.rank, a.world, a.max_spins, a.error, 0)) return;
  const int64_t vecs = a.n / 8;
  for (int64_t v = (int64_t)blockIdx.x * NT + threadIdx.x; v < vecs; v += (int64_t)gridDim.x * NT) {
    float acc[8];
    if (a.residual) {
      const uint4 r = reinterpret_cast<const uint4*>(a.residual)[v];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&r);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h[i]);
        acc[2 * i] = f.x;
        acc[2 * i + 1] = f.y;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    }
    for (int p = 0; p < a.world; ++p) {
      const uint4 raw = reinterpret_cast<const uint4*>(a.part[p])[v];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h[i]);
        acc[2 * i] += f.x;
        acc[2 * i + 1] += f.y;
      }
    }
    uint4 out;
    uint32_t* o = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = pack_bf16(acc[2 * i], acc[2 * i + 1]);
    reinterpret_cast<uint4*>(a.out)[v] = out;
  }
}

__global__ void __launch_bounds__(NT) allgather_cols_kernel(TpAllgatherArgs a) {
  const int64_t total = (int64_t)a.rows * a.cols;
  for (int64_t e = (int64_t)blockIdx.x * NT + threadIdx.x; e < total; e += (int64_t)gridDim.x * NT) {
    const int64_t r = e / a.cols, c = e % a.cols;
    const float v = a.src[r * a.src_stride + c];
    const int64_t at = r * (int64_t)a.cols * a.world + (int64_t)a.rank * a.cols + c;
    for (int p = 0; p < a.world; ++p) a.dst[p][at] = v;
  }
  cta_barrier(a.sig, a.epochs, a.rank, a.world, a.max_spins, a.error, 1);
}

}  // namespace tp
}  // namespace pra

static int tp_blocks(int64_t work_items) {
  const int64_t want = (work_items + pra::tp::NT - 1) / pra::tp::NT;
  return (int)(want < 1 ? 1 : (want > TP_MAX_BLOCKS ? TP_MAX_BLOCKS : want));
}

cudaError_t pra_tp_allreduce(const TpAllreduceArgs& a, cudaStream_t st) {
  if (a.world < 1 || a.world > TP_MAX_RANKS || a.n % 8) return cudaErrorInvalidValue;
  for (int p = 0; p < a.world; ++p)
    if (reinterpret_cast<uintptr_t>(a.part[p]) & 15) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(a.out) | reinterpret_cast<uintptr_t>(a.residual)) & 15) return cudaErrorInvalidValue;
  pra::tp::allreduce_oneshot_kernel<<<tp_blocks(a.n / 8), pra::tp::NT, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t pra_tp_allgather(const TpAllgatherArgs& a, cudaStream_t st) {
  if (a.world < 1 || a.world > TP_MAX_RANKS) return cudaErrorInvalidValue;
  pra::tp::allgather_cols_kernel<<<tp_blocks((int64_t)a.rows * a.cols), pra::tp::NT, 0, st>>>(a);
  return cudaGetLastError();
}
