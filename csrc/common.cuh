// Shared device helpers for the PRA sm_100a kernels.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <map>
#include <mutex>
#include <utility>

#include "kernels.h"

// Launch helpers return the first CUDA error instead of throwing; the binding
// layer turns a non-success code into a Python exception.
#define PRA_RETURN_IF_ERROR(expr)          \
  do {                                     \
    cudaError_t err__ = (expr);            \
    if (err__ != cudaSuccess) return err__; \
  } while (0)

namespace pra {

inline int ceil_div(int a, int b) { return (a + b - 1) / b; }

// Raise a kernel's dynamic shared-memory limit to `bytes`, calling cudaFuncSetAttribute only
// when this (kernel, device) pair has not been given at least that much yet: the attribute
// lasts for the process, and setting it on every launch costs host time per launch.
inline cudaError_t set_max_dynamic_smem(const void* kernel, int bytes) {
  static std::mutex mu;
  static auto* granted = new std::map<std::pair<const void*, int>, int>();  // never freed
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  int& have = (*granted)[{kernel, dev}];
  if (have >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) have = bytes;
  return e;
}

// Explicit conversions (the build disables implicit bf16 <-> float conversions).
__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16(v); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum for blockDim.x <= 1024; `scratch` holds >= 32 floats.
__device__ __forceinline__ float block_sum(float v, float* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  const int nwarps = (blockDim.x + 31) >> 5;
  v = (threadIdx.x < nwarps) ? scratch[threadIdx.x] : 0.f;
  if (warp == 0) v = warp_sum(v);
  if (threadIdx.x == 0) scratch[0] = v;
  __syncthreads();
  float out = scratch[0];
  __syncthreads();
  return out;
}

__device__ __forceinline__ float block_max(float v, float* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  const int nwarps = (blockDim.x + 31) >> 5;
  v = (threadIdx.x < nwarps) ? scratch[threadIdx.x] : -INFINITY;
  if (warp == 0) v = warp_max(v);
  if (threadIdx.x == 0) scratch[0] = v;
  __syncthreads();
  float out = scratch[0];
  __syncthreads();
  return out;
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Tensor-core fragments (bf16 inputs, fp32 accumulate).
__device__ __forceinline__ void mma_bf16_16816(float* c, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t* r, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t* r, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
  const int bytes = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem), "r"(bytes));
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }

template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// TMA: arm `bar` for `bytes` of incoming copies (one arrival).
__device__ __forceinline__ void expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// 2-D tile copy of this GPU's global memory into this CTA's shared memory, completing on `bar`
// (no cluster, no multicast); x = the column element (16-byte aligned), y = the row.
__device__ __forceinline__ void tma_load(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Philox4x32-10 (Salmon, Moraes, Dror, Shaw: "Parallel Random Numbers: As Easy as 1, 2, 3",
// SC 2011): ten rounds of two 32x32->64-bit products mixed into the counter, the key bumped
// by the Weyl constants between rounds.
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(0xD2511F53u, c.x), lo0 = 0xD2511F53u * c.x;
    const uint32_t hi1 = __umulhi(0xCD9E8D57u, c.z), lo1 = 0xCD9E8D57u * c.z;
    c = make_uint4(hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0);
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c;
}

// The 4 Philox words of block `blk` of the dropout stream (seed, offset).
__device__ __forceinline__ uint4 dropout_block(uint64_t seed, uint64_t offset, uint64_t blk) {
  return philox4x32_10(make_uint4((uint32_t)blk, (uint32_t)(blk >> 32), (uint32_t)offset, (uint32_t)(offset >> 32)),
                       (uint32_t)seed, (uint32_t)(seed >> 32));
}

// Keep decision of element e of the stream (seed, offset).
__device__ __forceinline__ bool dropout_keep(uint64_t seed, uint64_t offset, uint64_t e, uint32_t thresh) {
  const uint4 r = dropout_block(seed, offset, e >> 2);
  const uint32_t w = (e & 3) == 0 ? r.x : (e & 3) == 1 ? r.y : (e & 3) == 2 ? r.z : r.w;
  return (w >> 8) >= thresh;
}

// Records the first bounds violation of a checked kernel (later ones keep the first record).
__device__ __forceinline__ void bounds_fail(BoundsStatus* s, int kernel, long long index, long long limit) {
  if (atomicCAS(&s->code, 0, 1) == 0) {
    s->kernel = kernel;
    s->index = index;
    s->limit = limit;
    __threadfence();
  }
}

// Bounded spin on a 32-bit flag in global (or peer) memory.  Returns true when
// `*flag >= expected` was observed before `max_spins` polls; the caller records
// a timeout status otherwise.  Every cross-agent wait in this library uses it.
__device__ __forceinline__ bool bounded_wait_geq(const volatile uint32_t* flag, uint32_t expected,
                                                 long long max_spins) {
  for (long long i = 0; i < max_spins; ++i) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(flag) : "memory");
    if (v >= expected) return true;
    __nanosleep(64);
  }
  return false;
}

}  // namespace pra

namespace pra {

// ---- mbarriers (CTA scope) and the generic -> async proxy fence ------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Makes earlier generic-proxy shared-memory writes (cp.async data, register stores) visible
// to the async proxy (the tensor cores' operand reads).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

__device__ __forceinline__ bool mbar_try_wait_parity(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

}  // namespace pra

// Tensor map of a [rows, cols] bf16 matrix (row stride ld elements, 16-byte aligned) cut into
// 64-column x box_rows boxes in the 128-byte swizzle layout; cached per (address, shape);
// nullptr when the driver rejects it.  Defined in decode_gemm.cu.
const CUtensorMap* pra_tile_map_bf16(const void* ptr, int64_t cols, int64_t rows, int64_t ld, int box_rows);

namespace pra {

// ---- programmatic dependent launch (the decode chain) ----------------------------------
// A decode step is a chain of short kernels (norm -> QKV GEMM -> routing -> attention ->
// merge -> O GEMM -> norm -> gate/up GEMM -> SwiGLU -> down GEMM, per layer).  Launched with
// the programmatic-serialization attribute, kernel N+1 is scheduled as soon as every CTA of
// kernel N has executed `pdl_launch_dependents`, and runs the part of its prologue that reads
// nothing kernel N writes (barrier set-up, TMEM allocation, tensor-map prefetch, the weight
// tiles of its first pipeline stages) while kernel N drains.  `pdl_wait` then blocks until
// kernel N has completed and its writes are visible.  Rules every instrumented kernel keeps:
// every thread calls `pdl_wait` before its first read of data an earlier kernel produces and
// before its first global write (so no write races a predecessor's read), and no thread exits
// without having called it (kernel N+1 completing then implies kernel N completed, which keeps
// the chain transitive).  Without the attribute both instructions are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

}  // namespace pra

// The launch attributes every instrumented decode kernel gets: programmatic stream
// serialization (when enabled) and the current launch priority (when set); returns how many
// of `attr[0..1]` it filled.
inline int pra_launch_attrs(cudaLaunchAttribute* attr) {
  int n = 0;
  if (pra_pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  const int prio = pra_launch_priority();
  if (prio != 0) {
    attr[n].id = cudaLaunchAttributePriority;
    attr[n].val.priority = prio;
    ++n;
  }
  return n;
}

// Launch `kernel` on `st`, with programmatic stream serialization when PDL is enabled.  Only
// for kernels that follow the `pdl_wait` rules above.
template <typename... Params, typename... Args>
inline cudaError_t pra_launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                  Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  cfg.attrs = attr;
  cfg.numAttrs = pra_launch_attrs(attr);
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}
