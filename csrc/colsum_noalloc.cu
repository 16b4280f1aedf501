// No-allocation entry point: column sums of a bf16 matrix (the bias-gradient reduction).
//
// This entry point has no counterpart in the reference implementation.
//
// pra_colsum_noalloc(g, M, N, out, stream) computes out[n] = sum_m g[m, n] for a
// row-major bf16 matrix g[M, N] and writes bf16 out[N].  It runs the library's
// ordinary column-sum op (pra_colsum, norm.cu) with one difference: it never
// allocates device memory.  The per-block partial sums that op needs live in a
// fixed scratch array that is part of the library image (`g_colsum_scratch`,
// 4 MiB of fp32), instead of a buffer the caller or torch would allocate.
//
// Who should call it: code that cannot allocate at the point of use.  Two common
// cases are (a) hosts that reserve all device memory up front and forbid any
// later cudaMalloc (a late allocation would fail, or fragment a pool another
// component owns), and (b) code running where its host forbids calls that can
// synchronise the device, which cudaMalloc and cudaFree may do.  Such callers
// pass their own input and output buffers and nothing else.
//
// Rules for callers:
//   * Capacity: the scratch holds at most 1,048,576 floats.  A call needs
//     pra_colsum_partials(M) * N floats (min(256, ceil(M / 64)) partial rows);
//     a call that needs more is rejected with cudaErrorInvalidValue (and a
//     message on stderr) before anything is launched.
//   * Arguments: N must be positive and even, g 4-byte aligned (the kernel reads
//     bf16 pairs) and out 2-byte aligned; anything else is rejected the same way.
//   * One-time set-up: the first call on each device looks up the device address
//     of the scratch array (cudaGetSymbolAddress, with that device current) and
//     caches it per device index.  Make that first call before any stream capture
//     begins.  The cached address belongs to the device's current context: after
//     cudaDeviceReset (or anything else that destroys the primary context) it is
//     stale, so call pra_colsum_noalloc_reset() once, before the next call.
//   * Sharing: every call on a device uses the same scratch array, and the array
//     keeps whatever the last call left in it.  Each call writes every scratch
//     slot it reads, so nothing needs to start at zero.  Calls that overlap on
//     the GPU (different streams, no ordering between them) race on the scratch
//     and give wrong sums: serialise them.
//   * Lifetime: every GPU that loads this library holds the 4 MiB array until
//     the process exits.
#include <cstdint>
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace {

constexpr size_t kScratchFloats = size_t(1) << 20;  // 4 MiB of fp32 partial sums
constexpr int kMaxDevices = 64;

__device__ __align__(256) float g_colsum_scratch[kScratchFloats];

float* g_scratch_address[kMaxDevices] = {};
std::mutex g_setup_mutex;

cudaError_t scratch_address(float** out) {
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return err;
  if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_address[device] == nullptr) {
    float* ptr = nullptr;
    err = cudaGetSymbolAddress(reinterpret_cast<void**>(&ptr), g_colsum_scratch);
    if (err != cudaSuccess) return err;
    g_scratch_address[device] = ptr;
  }
  *out = g_scratch_address[device];
  return cudaSuccess;
}

int reject(const char* why, int M, int N) {
  std::fprintf(stderr, "pra_colsum_noalloc: %s (M=%d, N=%d)\n", why, M, N);
  return static_cast<int>(cudaErrorInvalidValue);
}

}  // namespace

long long pra_colsum_noalloc_capacity() { return static_cast<long long>(kScratchFloats); }

void pra_colsum_noalloc_reset() {
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  for (float*& p : g_scratch_address) p = nullptr;
}

int pra_colsum_noalloc(const void* g, int M, int N, void* out, cudaStream_t stream) {
  if (g == nullptr || out == nullptr) return reject("null pointer", M, N);
  if (M < 0 || N <= 0 || N % 2 != 0) return reject("M must be >= 0 and N positive and even", M, N);
  if ((reinterpret_cast<uintptr_t>(g) & 3) != 0) return reject("g must be 4-byte aligned", M, N);
  if ((reinterpret_cast<uintptr_t>(out) & 1) != 0) return reject("out must be 2-byte aligned", M, N);
  const size_t need = static_cast<size_t>(pra_colsum_partials(M)) * static_cast<size_t>(N);
  if (need > kScratchFloats) {
    std::fprintf(stderr, "pra_colsum_noalloc: M=%d, N=%d needs %zu scratch floats, above the fixed capacity of %zu\n",
                 M, N, need, kScratchFloats);
    return static_cast<int>(cudaErrorInvalidValue);
  }
  float* scratch = nullptr;
  const cudaError_t err = scratch_address(&scratch);
  if (err != cudaSuccess) return static_cast<int>(err);
  return static_cast<int>(pra_colsum(static_cast<const __nv_bfloat16*>(g), M, N, scratch,
                                     static_cast<__nv_bfloat16*>(out), stream));
}
