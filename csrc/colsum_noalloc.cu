// No-allocation entry point: column sums of a bf16 matrix (the bias-gradient reduction).
//
// This entry point has no counterpart in the reference implementation.
//
// pra_colsum_noalloc(g, M, N, out, stream) computes out[n] = sum_m g[m, n] for a
// row-major bf16 matrix g[M, N] and writes bf16 out[N].  It does exactly what the
// library's ordinary column-sum op does, but it never allocates device memory:
// the per-block partial sums it needs live in a fixed scratch array that is part
// of the library image (`g_colsum_scratch`, 4 MiB of fp32).
//
// Who should call it: code that cannot allocate at the point of use.  Two common
// cases are (a) hosts that reserve all device memory up front and forbid any
// later cudaMalloc (a late allocation would fail, or fragment a pool another
// component owns), and (b) code issued while a stream is being captured into a
// CUDA graph in a capture mode where cudaMalloc is not a legal call.  Such
// callers pass their own input and output buffers and nothing else.
//
// Rules for callers:
//   * Capacity: the scratch holds at most 1,048,576 floats.  A call needs
//     partials(M) * N floats, where partials(M) = min(256, ceil(M / 64)); a call
//     that needs more is rejected with cudaErrorInvalidValue (and a message on
//     stderr) before anything is launched.  N must be even.
//   * One-time set-up: the first call on each device looks up the device address
//     of the scratch array (cudaGetSymbolAddress, with that device current) and
//     caches it.  Make that first call before any stream capture begins.
//   * Sharing: every call on a device uses the same scratch array, and the array
//     keeps whatever the last call left in it.  Each call writes every scratch
//     slot before it reads it, so nothing needs to start at zero.  Calls that
//     overlap on the GPU (different streams, no ordering between them) race on
//     the scratch and give wrong sums: serialise them.
//   * Lifetime: every GPU that loads this library holds the 4 MiB array until
//     the process exits.
#include <cstdio>
#include <mutex>

#include "common.cuh"

namespace {

constexpr size_t kScratchFloats = size_t(1) << 20;  // 4 MiB of fp32 partial sums
constexpr int kMaxDevices = 64;

__device__ __align__(256) float g_colsum_scratch[kScratchFloats];

float* g_scratch_address[kMaxDevices] = {};
std::mutex g_setup_mutex;

__global__ void noalloc_partial_kernel(const __nv_bfloat16* __restrict__ g, int M, int N, int rows_per_block,
                                       float* __restrict__ part) {
  const int pair = blockIdx.y * blockDim.x + threadIdx.x;  // column pair index
  if (2 * pair >= N) return;
  const int r0 = blockIdx.x * rows_per_block, r1 = min(r0 + rows_per_block, M);
  float sx = 0.f, sy = 0.f;
  for (int r = r0; r < r1; ++r) {
    const float2 v = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(g + (int64_t)r * N)[pair]);
    sx += v.x;
    sy += v.y;
  }
  part[(int64_t)blockIdx.x * N + 2 * pair] = sx;
  part[(int64_t)blockIdx.x * N + 2 * pair + 1] = sy;
}

__global__ void noalloc_reduce_kernel(const float* __restrict__ part, int parts, int N, __nv_bfloat16* __restrict__ out) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= N) return;
  float acc = 0.f;
  for (int p = 0; p < parts; ++p) acc += part[(int64_t)p * N + col];
  out[col] = __float2bfloat16(acc);
}

int partials_for(int M) { return M <= 0 ? 1 : ((M + 63) / 64 > 256 ? 256 : (M + 63) / 64); }

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

}  // namespace

// Scratch capacity in floats (so callers can check a shape before calling).
extern "C" __attribute__((visibility("default"))) long long pra_colsum_noalloc_capacity() {
  return static_cast<long long>(kScratchFloats);
}

// Returns a cudaError_t value (0 on success).  `g` and `out` are device pointers;
// `stream` is the cudaStream_t to launch on (0 for the legacy default stream).
extern "C" __attribute__((visibility("default"))) int pra_colsum_noalloc(const void* g, int M, int N, void* out,
                                                                         cudaStream_t stream) {
  if (g == nullptr || out == nullptr || M < 0 || N <= 0 || N % 2 != 0) {
    std::fprintf(stderr, "pra_colsum_noalloc: invalid arguments (M=%d, N=%d; N must be positive and even)\n", M, N);
    return static_cast<int>(cudaErrorInvalidValue);
  }
  const int parts = partials_for(M);
  if (static_cast<size_t>(parts) * static_cast<size_t>(N) > kScratchFloats) {
    std::fprintf(stderr,
                 "pra_colsum_noalloc: M=%d, N=%d needs %zu scratch floats, above the fixed capacity of %zu\n", M, N,
                 static_cast<size_t>(parts) * static_cast<size_t>(N), kScratchFloats);
    return static_cast<int>(cudaErrorInvalidValue);
  }
  float* scratch = nullptr;
  cudaError_t err = scratch_address(&scratch);
  if (err != cudaSuccess) return static_cast<int>(err);
  const int rows = M == 0 ? 0 : (M + parts - 1) / parts;
  dim3 grid(parts, (N / 2 + 255) / 256);
  noalloc_partial_kernel<<<grid, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(g), M, N, rows, scratch);
  err = cudaGetLastError();
  if (err != cudaSuccess) return static_cast<int>(err);
  noalloc_reduce_kernel<<<(N + 255) / 256, 256, 0, stream>>>(scratch, parts, N, static_cast<__nv_bfloat16*>(out));
  return static_cast<int>(cudaGetLastError());
}
