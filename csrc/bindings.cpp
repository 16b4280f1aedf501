// Python bindings of the PRA sm_100a kernels (torch tensors <-> raw launch blocks).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <nvtx3/nvToolsExt.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <vector>

#include "kernels.h"

// Native cache-build planner (planner.cpp).
pybind11::object pra_plan_batch(const pybind11::list& rows, const pybind11::object& tokenizer,
                                const pybind11::dict& cfg);

namespace {

inline cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void check(cudaError_t e, const char* what) {
  TORCH_CHECK(e == cudaSuccess, "pra_ops.", what, " failed: ", cudaGetErrorString(e));
}

void expect(const torch::Tensor& t, at::ScalarType dt, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == dt, name, " has dtype ", t.scalar_type(), ", expected ", dt);
}

template <typename T>
T* ptr(const torch::Tensor& t) {
  return reinterpret_cast<T*>(t.data_ptr());
}

// Memory pools may be device tensors or pinned host tensors (the CPU-resident K/V tier): a
// kernel then gathers only the selected rows over the host link, through the address under
// which the current device sees the pinned allocation.
void expect_pool(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() || t.is_pinned(), name, " must be a CUDA tensor or pinned host memory");
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, name, " must be bf16");
}

template <typename T>
T* pool_ptr(const torch::Tensor& t) {
  if (t.is_cuda()) return ptr<T>(t);
  cudaPointerAttributes attr{};
  const cudaError_t e = cudaPointerGetAttributes(&attr, t.data_ptr());
  TORCH_CHECK(e == cudaSuccess && attr.devicePointer != nullptr,
              "pinned host pool is not mapped into the device address space: ", cudaGetErrorString(e));
  return reinterpret_cast<T*>(attr.devicePointer);
}

template <typename T>
const T* optr(const c10::optional<torch::Tensor>& t) {
  return (t.has_value() && t->defined() && t->numel() > 0) ? reinterpret_cast<const T*>(t->data_ptr()) : nullptr;
}

// ---------------------------------------------------------------- attention
// Per-device status word of the attention kernels (1 after a kernel gave up on a bounded
// wait); allocated on first use and never freed (it outlives the interpreter's tensors).
torch::Tensor& attention_status_buffer(const torch::Device& dev) {
  static auto* bufs = new std::map<int, torch::Tensor>();
  auto& t = (*bufs)[dev.index()];
  if (!t.defined()) t = torch::zeros({1}, torch::TensorOptions().dtype(at::kInt).device(dev));
  return t;
}

AttnParams attn_params(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v, int64_t heads,
                       int64_t kv_heads, const c10::optional<torch::Tensor>& mem_k,
                       const c10::optional<torch::Tensor>& mem_v, const c10::optional<torch::Tensor>& mem_idx,
                       const c10::optional<torch::Tensor>& mem_len, const c10::optional<torch::Tensor>& key_valid,
                       double scale) {
  TORCH_CHECK(q.dim() == 3 && k.dim() == 3 && v.dim() == 3, "q/k/v must be [B, T, width] views");
  TORCH_CHECK(q.stride(2) == 1 && k.stride(2) == 1 && v.stride(2) == 1, "q/k/v feature dim must be contiguous");
  expect(q, at::kBFloat16, "q");
  expect(k, at::kBFloat16, "k");
  expect(v, at::kBFloat16, "v");
  TORCH_CHECK(heads % kv_heads == 0, "heads must be a multiple of kv heads");
  AttnParams p{};
  p.status = ptr<int>(attention_status_buffer(q.device()));
  p.B = q.size(0);
  p.T = q.size(1);
  p.H = heads;
  p.Hkv = kv_heads;
  p.q = ptr<const __nv_bfloat16>(q);
  p.k = ptr<const __nv_bfloat16>(k);
  p.v = ptr<const __nv_bfloat16>(v);
  p.q_row = q.stride(1);
  p.q_batch = q.stride(0);
  p.k_row = k.stride(1);
  p.k_batch = k.stride(0);
  p.v_row = v.stride(1);
  p.v_batch = v.stride(0);
  p.scale = static_cast<float>(scale);
  if (mem_idx.has_value() && mem_idx->numel() > 0) {
    TORCH_CHECK(mem_k.has_value() && mem_v.has_value() && mem_len.has_value(), "memory needs k, v, idx and len");
    expect_pool(*mem_k, "mem_k");
    expect_pool(*mem_v, "mem_v");
    expect(*mem_idx, at::kInt, "mem_idx");
    expect(*mem_len, at::kInt, "mem_len");
    TORCH_CHECK(mem_k->dim() == 2 && mem_k->stride(1) == 1 && mem_v->stride(1) == 1 &&
                    mem_k->stride(0) == mem_v->stride(0),
                "memory pools must be row-major [rows, width] with equal strides");
    TORCH_CHECK(mem_idx->is_contiguous() && mem_idx->size(0) == p.B, "mem_idx must be [B, max]");
    p.mem_k = pool_ptr<const __nv_bfloat16>(*mem_k);
    p.mem_v = pool_ptr<const __nv_bfloat16>(*mem_v);
    p.mem_row = mem_k->stride(0);
    p.mem_idx = ptr<const int>(*mem_idx);
    p.mem_len = ptr<const int>(*mem_len);
    p.mem_max = mem_idx->size(1);
  }
  if (key_valid.has_value() && key_valid->numel() > 0) {
    expect(*key_valid, at::kByte, "key_valid");
    TORCH_CHECK(key_valid->is_contiguous() && key_valid->size(0) == p.B && key_valid->size(1) == p.T,
                "key_valid must be [B, T]");
    p.key_valid = ptr<const uint8_t>(*key_valid);
  }
  return p;
}

// Attention-probability dropout (p > 0): element (b, h, q, t) of the stream (seed, offset).
static void set_attention_dropout(AttnParams& p, double drop_p, int64_t seed, int64_t offset) {
  p.drop_thresh = pra_dropout_threshold(drop_p);
  p.drop_scale = drop_p > 0.0 ? (float)(1.0 / (1.0 - drop_p)) : 1.f;
  p.drop_seed = (uint64_t)seed;
  p.drop_offset = (uint64_t)offset;
  TORCH_CHECK(p.drop_thresh == 0 || (p.mem_len == nullptr && p.H == p.Hkv),
              "attention dropout applies to local multi-head attention only (no memory, no GQA)");
}

std::vector<torch::Tensor> attention_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, int64_t heads,
                                         int64_t kv_heads, int64_t head_dim, c10::optional<torch::Tensor> mem_k,
                                         c10::optional<torch::Tensor> mem_v, c10::optional<torch::Tensor> mem_idx,
                                         c10::optional<torch::Tensor> mem_len, c10::optional<torch::Tensor> key_valid,
                                         double scale, double drop_p = 0.0, int64_t drop_seed = 0,
                                         int64_t drop_offset = 0) {
  c10::cuda::CUDAGuard guard(q.device());
  auto p = attn_params(q, k, v, heads, kv_heads, mem_k, mem_v, mem_idx, mem_len, key_valid, scale);
  set_attention_dropout(p, drop_p, drop_seed, drop_offset);
  auto out = torch::empty({p.B, p.T, heads * head_dim}, q.options());
  auto lse = torch::empty({p.B, heads, p.T}, q.options().dtype(at::kFloat));
  p.o = ptr<__nv_bfloat16>(out);
  p.o_row = out.stride(1);
  p.o_batch = out.stride(0);
  p.lse = ptr<float>(lse);
  check(pra_attention_fwd(p, (int)head_dim, stream()), "attention_fwd");
  return {out, lse};
}

std::vector<torch::Tensor> attention_bwd(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                         torch::Tensor out, torch::Tensor lse, int64_t heads, int64_t head_dim,
                                         c10::optional<torch::Tensor> mem_k, c10::optional<torch::Tensor> mem_v,
                                         c10::optional<torch::Tensor> mem_idx, c10::optional<torch::Tensor> mem_len,
                                         c10::optional<torch::Tensor> key_valid, double scale, double drop_p = 0.0,
                                         int64_t drop_seed = 0, int64_t drop_offset = 0) {
  c10::cuda::CUDAGuard guard(q.device());
  auto p = attn_params(q, k, v, heads, heads, mem_k, mem_v, mem_idx, mem_len, key_valid, scale);
  set_attention_dropout(p, drop_p, drop_seed, drop_offset);
  expect(dout, at::kBFloat16, "dout");
  TORCH_CHECK(dout.stride(2) == 1 && out.stride(2) == 1, "dout/out feature dim must be contiguous");
  p.o = ptr<__nv_bfloat16>(out);
  p.o_row = out.stride(1);
  p.o_batch = out.stride(0);
  p.lse = ptr<float>(lse);
  p.dout = ptr<const __nv_bfloat16>(dout);
  p.do_row = dout.stride(1);
  p.do_batch = dout.stride(0);
  auto delta = torch::empty({p.B, heads, p.T}, q.options().dtype(at::kFloat));
  p.delta = ptr<float>(delta);
  // dq, dk, dv packed as one [B, T, 3, H*D] buffer so the QKV weight gradient is a single GEMM.
  auto dqkv = torch::empty({p.B, p.T, 3 * heads * head_dim}, q.options());
  const int64_t w = heads * head_dim;
  p.dq = ptr<__nv_bfloat16>(dqkv);
  p.dk = p.dq + w;
  p.dv = p.dq + 2 * w;
  p.dq_row = p.dk_row = p.dv_row = dqkv.stride(1);
  p.dq_batch = p.dk_batch = p.dv_batch = dqkv.stride(0);
  check(pra_attention_bwd(p, (int)head_dim, stream()), "attention_bwd");
  return {dqkv};
}

// ---------------------------------------------------------------- dropout
// out = keep ? x / (1 - p) : 0 over the flat element order of x (out may alias x).
void dropout(torch::Tensor x, torch::Tensor out, double drop_p, int64_t seed, int64_t offset) {
  c10::cuda::CUDAGuard guard(x.device());
  expect(x, at::kBFloat16, "x");
  expect(out, at::kBFloat16, "out");
  TORCH_CHECK(x.is_contiguous() && out.is_contiguous() && x.numel() == out.numel(), "dropout: contiguous, same size");
  TORCH_CHECK(drop_p >= 0.0 && drop_p < 1.0, "dropout probability must be in [0, 1)");
  check(pra_dropout(ptr<const __nv_bfloat16>(x), ptr<__nv_bfloat16>(out), x.numel(), pra_dropout_threshold(drop_p),
                    (float)(1.0 / (1.0 - drop_p)), (uint64_t)seed, (uint64_t)offset, stream()),
        "dropout");
}

// out = res + (keep ? x / (1 - p) : 0) (out may alias res or x).
void dropout_add(torch::Tensor res, torch::Tensor x, torch::Tensor out, double drop_p, int64_t seed, int64_t offset) {
  c10::cuda::CUDAGuard guard(x.device());
  expect(res, at::kBFloat16, "res");
  expect(x, at::kBFloat16, "x");
  expect(out, at::kBFloat16, "out");
  TORCH_CHECK(res.is_contiguous() && x.is_contiguous() && out.is_contiguous() && x.numel() == out.numel() &&
                  res.numel() == x.numel(),
              "dropout_add: contiguous, same size");
  TORCH_CHECK(drop_p >= 0.0 && drop_p < 1.0, "dropout probability must be in [0, 1)");
  check(pra_dropout_add(ptr<const __nv_bfloat16>(res), ptr<const __nv_bfloat16>(x), ptr<__nv_bfloat16>(out),
                        x.numel(), pra_dropout_threshold(drop_p), (float)(1.0 / (1.0 - drop_p)), (uint64_t)seed,
                        (uint64_t)offset, stream()),
        "dropout_add");
}

// ---------------------------------------------------------------- GEMM
torch::Tensor& workspace(const torch::Tensor& like) {
  static std::vector<torch::Tensor> per_device(16);
  const int dev = like.get_device();
  if (!per_device[dev].defined()) per_device[dev] = torch::empty({64 << 20}, like.options().dtype(at::kByte));
  return per_device[dev];
}

void gemm(const std::string& kind, torch::Tensor A, torch::Tensor B, c10::optional<torch::Tensor> C, torch::Tensor D,
          c10::optional<torch::Tensor> bias, c10::optional<torch::Tensor> aux, double alpha, double beta,
          c10::optional<torch::Tensor> alpha_ptr) {
  c10::cuda::CUDAGuard guard(A.device());
  expect(A, at::kBFloat16, "A");
  expect(B, at::kBFloat16, "B");
  expect(D, kind == "tn_f32" ? at::kFloat : at::kBFloat16, "D");
  TORCH_CHECK(A.is_contiguous() && B.is_contiguous() && D.is_contiguous(), "GEMM operands must be contiguous");
  GemmArgs g{};
  g.A = A.data_ptr();
  g.B = B.data_ptr();
  g.C = optr<void>(C);
  g.D = D.data_ptr();
  g.bias = optr<void>(bias);
  g.aux = aux.has_value() ? aux->data_ptr() : nullptr;
  g.alpha = (float)alpha;
  g.beta = (float)beta;
  g.alpha_ptr = optr<float>(alpha_ptr);
  auto& ws = workspace(A);
  g.workspace = ws.data_ptr();
  g.workspace_bytes = ws.numel();
  if (kind == "tn" || kind == "tn_gelu" || kind == "tn_f32") {  // D[M,N] = A[M,K] B[N,K]^T
    g.M = A.size(0); g.K = A.size(1); g.N = B.size(0);
    TORCH_CHECK(B.size(1) == g.K && D.size(0) == g.M && D.size(1) == g.N, "tn shape mismatch");
  } else if (kind == "nn" || kind == "nn_dgelu" || kind == "nn_sk") {  // D[M,N] = A[M,K] B[K,N]
    g.M = A.size(0); g.K = A.size(1); g.N = B.size(1);
    TORCH_CHECK(B.size(0) == g.K && D.size(0) == g.M && D.size(1) == g.N, "nn shape mismatch");
  } else if (kind == "wgrad" || kind == "wgrad_sk") {  // D[M,N] = A[K,M]^T B[K,N]
    g.K = A.size(0); g.M = A.size(1); g.N = B.size(1);
    TORCH_CHECK(B.size(0) == g.K && D.size(0) == g.M && D.size(1) == g.N, "wgrad shape mismatch");
  } else {
    TORCH_CHECK(false, "unknown gemm kind ", kind);
  }
  if (C.has_value()) TORCH_CHECK(C->is_contiguous() && C->sizes() == D.sizes(), "C must match D");
  if (g.beta != 0.f) TORCH_CHECK(g.C != nullptr, "beta != 0 needs C");
  cudaError_t e;
  if (kind == "tn") e = pra_gemm_tn_auto(g, stream());
  else if (kind == "tn_f32") e = pra_gemm_tn_f32(g, stream());
  else if (kind == "tn_gelu") e = pra_gemm_tn_bias_gelu(g, stream());
  else if (kind == "nn") e = pra_gemm_nn_auto(g, stream());
  else if (kind == "nn_dgelu") e = pra_gemm_nn_dgelu(g, stream());
  else if (kind == "nn_sk") e = pra_gemm_nn_sk(g, stream());
  else if (kind == "wgrad_sk") e = pra_gemm_wgrad_sk(g, stream());
  else e = pra_gemm_wgrad_auto(g, stream());
  check(e, kind.c_str());
}

std::vector<torch::Tensor> gelu_probe(torch::Tensor z) {
  c10::cuda::CUDAGuard guard(z.device());
  expect(z, at::kFloat, "z");
  TORCH_CHECK(z.is_contiguous(), "z must be contiguous");
  auto y = torch::empty_like(z), dy = torch::empty_like(z);
  check(pra_gelu_probe(ptr<const float>(z), ptr<float>(y), ptr<float>(dy), z.numel(), stream()), "gelu_probe");
  return {y, dy};
}

// ---------------------------------------------------------------- norms
std::vector<torch::Tensor> norm_fwd(torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> b, double eps,
                                    bool rms) {
  c10::cuda::CUDAGuard guard(x.device());
  expect(x, at::kBFloat16, "x");
  expect(w, at::kBFloat16, "w");
  TORCH_CHECK(x.is_contiguous(), "x must be contiguous");
  const int D = x.size(-1);
  const int M = x.numel() / D;
  auto y = torch::empty_like(x);
  auto mean = torch::empty({M}, x.options().dtype(at::kFloat));
  auto rstd = torch::empty({M}, x.options().dtype(at::kFloat));
  check(pra_norm_fwd(ptr<const __nv_bfloat16>(x), ptr<const __nv_bfloat16>(w), optr<__nv_bfloat16>(b),
                     ptr<__nv_bfloat16>(y), ptr<float>(mean), ptr<float>(rstd), M, D, (float)eps, rms, stream()),
        "norm_fwd");
  return {y, mean, rstd};
}

std::vector<torch::Tensor> norm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor mean,
                                    torch::Tensor rstd, c10::optional<torch::Tensor> dres, bool rms) {
  c10::cuda::CUDAGuard guard(x.device());
  expect(dy, at::kBFloat16, "dy");
  TORCH_CHECK(dy.is_contiguous() && x.is_contiguous(), "norm_bwd inputs must be contiguous");
  const int D = x.size(-1);
  const int M = x.numel() / D;
  auto dx = torch::empty_like(x);
  const int parts = pra_norm_bwd_partials(M);
  auto part = torch::empty({2, parts, D}, x.options().dtype(at::kFloat));
  auto dw = torch::empty({D}, x.options());
  auto db = torch::empty({D}, x.options());
  check(pra_norm_bwd(ptr<const __nv_bfloat16>(dy), ptr<const __nv_bfloat16>(x), ptr<const __nv_bfloat16>(w),
                     ptr<const float>(mean), ptr<const float>(rstd), optr<__nv_bfloat16>(dres), ptr<__nv_bfloat16>(dx),
                     ptr<float>(part), ptr<float>(part) + (int64_t)parts * D, ptr<__nv_bfloat16>(dw),
                     ptr<__nv_bfloat16>(db), M, D, rms, stream()),
        "norm_bwd");
  return {dx, dw, db};
}

torch::Tensor colsum(torch::Tensor g) {
  c10::cuda::CUDAGuard guard(g.device());
  expect(g, at::kBFloat16, "g");
  TORCH_CHECK(g.is_contiguous(), "g must be contiguous");
  const int N = g.size(-1);
  const int M = g.numel() / N;
  auto part = torch::empty({pra_colsum_partials(M), N}, g.options().dtype(at::kFloat));
  auto out = torch::empty({N}, g.options());
  check(pra_colsum(ptr<const __nv_bfloat16>(g), M, N, ptr<float>(part), ptr<__nv_bfloat16>(out), stream()), "colsum");
  return out;
}

// ---------------------------------------------------------------- loss / optimizer
std::vector<torch::Tensor> cross_entropy(torch::Tensor logits, torch::Tensor labels, int64_t vocab,
                                         int64_t ignore_index) {
  c10::cuda::CUDAGuard guard(logits.device());
  expect(logits, at::kBFloat16, "logits");
  expect(labels, at::kLong, "labels");
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "logits must be [M, ld] row-major");
  const int64_t M = logits.size(0);
  auto loss = torch::empty({M}, logits.options().dtype(at::kFloat));
  auto valid = torch::empty({M}, logits.options().dtype(at::kFloat));
  check(pra_cross_entropy(ptr<__nv_bfloat16>(logits), M, logits.stride(0), (int)vocab,
                          ptr<const int64_t>(labels.contiguous()), (int)ignore_index, ptr<float>(loss),
                          ptr<float>(valid), stream()),
        "cross_entropy");
  return {loss, valid};
}

std::vector<torch::Tensor> grad_norm(torch::Tensor grad, double max_norm) {
  c10::cuda::CUDAGuard guard(grad.device());
  TORCH_CHECK(grad.is_contiguous(), "grad must be contiguous");
  auto part = torch::empty({pra_grad_norm_parts()}, grad.options().dtype(at::kFloat));
  auto norm = torch::empty({1}, grad.options().dtype(at::kFloat));
  auto coef = torch::empty({1}, grad.options().dtype(at::kFloat));
  check(pra_grad_norm(grad.data_ptr(), grad.scalar_type() == at::kBFloat16, grad.numel(), (float)max_norm,
                      ptr<float>(part), ptr<float>(norm), ptr<float>(coef), stream()),
        "grad_norm");
  return {norm, coef};
}

void adamw(torch::Tensor param, c10::optional<torch::Tensor> shadow, torch::Tensor grad, torch::Tensor m,
           torch::Tensor v, double lr, double beta1, double beta2, double eps, double weight_decay, int64_t step,
           c10::optional<torch::Tensor> coef, double grad_scale) {
  c10::cuda::CUDAGuard guard(param.device());
  expect(param, at::kFloat, "param");
  TORCH_CHECK(param.is_contiguous() && grad.is_contiguous() && m.is_contiguous() && v.is_contiguous(),
              "optimizer buffers must be contiguous");
  TORCH_CHECK(grad.numel() == param.numel(), "grad size mismatch");
  __nv_bfloat16* sh = nullptr;
  if (shadow.has_value() && shadow->defined()) {
    expect(*shadow, at::kBFloat16, "shadow");
    TORCH_CHECK(shadow->numel() == param.numel() && shadow->is_contiguous(), "shadow size mismatch");
    sh = ptr<__nv_bfloat16>(*shadow);
  }
  check(pra_adamw(ptr<float>(param), sh, grad.data_ptr(), grad.scalar_type() == at::kBFloat16, ptr<float>(m),
                  ptr<float>(v), param.numel(), (float)lr, (float)beta1, (float)beta2, (float)eps,
                  (float)weight_decay, (int)step, optr<float>(coef), (float)grad_scale, stream()),
        "adamw");
}

// ---------------------------------------------------------------- gists
// pool_k / pool_v: [L, R, D] (or [R, D]) bf16 views with unit feature stride.
GistArgs gist_args(const torch::Tensor& pool_k, const torch::Tensor& pool_v, const torch::Tensor& start,
                   const torch::Tensor& len, const c10::optional<torch::Tensor>& dest, const torch::Tensor& gk,
                   const torch::Tensor& gv, const torch::Tensor& gn, const torch::Tensor& count, int64_t nmax) {
  expect(pool_k, at::kBFloat16, "pool_k");
  expect(pool_v, at::kBFloat16, "pool_v");
  expect(gk, at::kFloat, "gk");
  expect(count, at::kInt, "count");
  const bool layered = pool_k.dim() == 3;
  TORCH_CHECK(pool_k.dim() == pool_v.dim() && (layered || pool_k.dim() == 2), "pools must be [L, R, D] or [R, D]");
  const int r = layered ? 1 : 0;
  TORCH_CHECK(pool_k.stride(r + 1) == 1 && pool_v.stride(r + 1) == 1 && pool_k.stride(r) == pool_v.stride(r) &&
                  (!layered || pool_k.stride(0) == pool_v.stride(0)),
              "pools must share row and layer strides");
  TORCH_CHECK(gk.dim() == 4 && gk.is_contiguous() && gv.is_contiguous() && gn.is_contiguous() &&
                  gv.sizes() == gk.sizes() && gn.sizes() == gk.sizes(),
              "gist tables must be contiguous [L, S, G, D]");
  TORCH_CHECK(count.dim() == 2 && count.is_contiguous() && count.size(0) == gk.size(0) && count.size(1) == gk.size(1),
              "count must be [L, S]");
  TORCH_CHECK(start.scalar_type() == at::kInt && len.scalar_type() == at::kInt, "start/len must be int32");
  GistArgs a{};
  a.pk = ptr<const __nv_bfloat16>(pool_k);
  a.pv = ptr<const __nv_bfloat16>(pool_v);
  a.row_stride = pool_k.stride(r);
  a.layer_stride = layered ? pool_k.stride(0) : 0;
  a.start = ptr<const int>(start);
  a.len = ptr<const int>(len);
  a.dest = optr<int>(dest);
  a.C = start.numel();
  a.D = pool_k.size(r + 1);
  a.G = gk.size(2);
  a.nmax = (int)nmax;
  TORCH_CHECK(gk.size(3) == a.D, "gist width must equal the pool width");
  TORCH_CHECK(gk.size(0) == (layered ? pool_k.size(0) : 1), "gist tables need one entry per pool layer");
  a.gk = ptr<float>(gk);
  a.gv = ptr<float>(gv);
  a.gn = ptr<float>(gn);
  a.out_layer_stride = gk.stride(0);
  a.count = ptr<int>(count);
  a.count_layer_stride = count.stride(0);
  return a;
}

void gist_mean_into(torch::Tensor pool_k, torch::Tensor pool_v, torch::Tensor start, torch::Tensor len,
                    c10::optional<torch::Tensor> dest, torch::Tensor gk, torch::Tensor gv, torch::Tensor gn,
                    torch::Tensor count) {
  c10::cuda::CUDAGuard guard(pool_k.device());
  GistArgs a = gist_args(pool_k, pool_v, start, len, dest, gk, gv, gn, count, 1);
  check(pra_gist_mean(a, gk.size(0), stream()), "gist_mean_into");
}

// Returns (iterations [L, C], status [L, C]).
std::vector<torch::Tensor> gist_kmeans_into(torch::Tensor pool_k, torch::Tensor pool_v, torch::Tensor start,
                                            torch::Tensor len, c10::optional<torch::Tensor> dest, torch::Tensor gk,
                                            torch::Tensor gv, torch::Tensor gn, torch::Tensor count, int64_t nmax,
                                            int64_t max_iters, double tol, bool normalize, bool kmeanspp,
                                            bool farthest, torch::Tensor init_first, torch::Tensor init_idx,
                                            torch::Tensor exp_draws, torch::Tensor exp_off,
                                            c10::optional<torch::Tensor> occupancy) {
  c10::cuda::CUDAGuard guard(pool_k.device());
  GistArgs a = gist_args(pool_k, pool_v, start, len, dest, gk, gv, gn, count, nmax);
  const int64_t L = gk.size(0);
  auto io = pool_k.options().dtype(at::kInt);
  auto iters = torch::empty({L, (int64_t)a.C}, io), status = torch::empty({L, (int64_t)a.C}, io);
  a.max_iters = (int)max_iters;
  a.tol = (float)tol;
  a.normalize = normalize;
  a.kmeanspp = kmeanspp;
  a.farthest = farthest;
  a.init_first = ptr<const int>(init_first);
  a.init_idx = ptr<const int>(init_idx);
  a.exp_draws = ptr<const float>(exp_draws);
  TORCH_CHECK(exp_off.scalar_type() == at::kInt && init_first.scalar_type() == at::kInt, "k-means offsets must be int32");
  a.exp_off = ptr<const int>(exp_off);
  a.occupancy = occupancy.has_value() ? ptr<int>(*occupancy) : nullptr;
  a.iterations = ptr<int>(iters);
  a.status = ptr<int>(status);
  check(pra_gist_kmeans(a, L, stream()), "gist_kmeans_into");
  return {iters, status};
}

// Allocating single-layer forms: outputs are indexed by chunk.
std::vector<torch::Tensor> gist_mean(torch::Tensor pool_k, torch::Tensor pool_v, torch::Tensor start,
                                     torch::Tensor len) {
  const int64_t C = start.numel(), D = pool_k.size(-1);
  auto opts = pool_k.options().dtype(at::kFloat);
  auto gk = torch::empty({1, C, 1, D}, opts), gv = torch::empty({1, C, 1, D}, opts), gn = torch::empty({1, C, 1, D}, opts);
  auto count = torch::empty({1, C}, pool_k.options().dtype(at::kInt));
  gist_mean_into(pool_k, pool_v, start, len, c10::nullopt, gk, gv, gn, count);
  return {gk.view({C, D}), gv.view({C, D}), gn.view({C, D})};
}

std::vector<torch::Tensor> gist_kmeans(torch::Tensor pool_k, torch::Tensor pool_v, torch::Tensor start,
                                       torch::Tensor len, int64_t G, int64_t max_iters, double tol, bool normalize,
                                       bool kmeanspp, bool farthest, torch::Tensor init_first, torch::Tensor init_idx,
                                       torch::Tensor exp_draws, torch::Tensor exp_off) {
  const int64_t C = start.numel(), D = pool_k.size(-1);
  auto fo = pool_k.options().dtype(at::kFloat);
  auto io = pool_k.options().dtype(at::kInt);
  auto gk = torch::zeros({1, C, G, D}, fo), gv = torch::zeros({1, C, G, D}, fo), gn = torch::zeros({1, C, G, D}, fo);
  auto count = torch::empty({1, C}, io), occ = torch::zeros({1, C, G}, io);
  const int64_t nmax = C ? len.max().item<int>() : 1;
  auto out = gist_kmeans_into(pool_k, pool_v, start, len, c10::nullopt, gk, gv, gn, count, std::max<int64_t>(nmax, 1),
                              max_iters, tol, normalize, kmeanspp, farthest, init_first, init_idx, exp_draws, exp_off,
                              occ);
  return {gk[0], gv[0], count[0], occ[0], out[0][0], out[1][0]};
}

// ---------------------------------------------------------------- routing
std::vector<torch::Tensor> route(torch::Tensor query, torch::Tensor gists, torch::Tensor gist_count,
                                 torch::Tensor row_pos_off, torch::Tensor row_ref_off, torch::Tensor ref_pos_off,
                                 torch::Tensor pos_chunk, torch::Tensor pos_ref, torch::Tensor pos_rank,
                                 torch::Tensor chunk_start,
                                 torch::Tensor chunk_len, torch::Tensor chunk_pool_row, int64_t k_ref, int64_t k_chunk,
                                 int64_t gist_agg, int64_t ref_agg, double threshold, int64_t budget, bool gist_only,
                                 bool full_reference, bool deduplicate, int64_t max_sel, int64_t max_mem,
                                 c10::optional<torch::Tensor> budget_rows, c10::optional<torch::Tensor> query_rows,
                                 bool global_chunks = false) {
  c10::cuda::CUDAGuard guard(query.device());
  expect(query, at::kBFloat16, "query");
  expect(gists, at::kFloat, "gists");
  // query: [B, >=D] (one query per row) or [B, T, >=D] with query_rows [B] int32 picking the token
  TORCH_CHECK((query.dim() == 2 || query.dim() == 3) && query.stride(-1) == 1, "query must be [B, (T,) >=D]");
  TORCH_CHECK(gists.dim() == 3 && gists.is_contiguous(), "gists must be [C, G, D] contiguous");
  RouteParams p{};
  p.B = query.size(0);
  p.D = gists.size(2);
  p.G = gists.size(1);
  p.query = ptr<const __nv_bfloat16>(query);
  p.query_stride = query.stride(0);
  if (query.dim() == 3) {
    TORCH_CHECK(query_rows.has_value() && query_rows->scalar_type() == at::kInt && query_rows->numel() == p.B,
                "a [B, T, D] query needs int32 query_rows [B]");
    p.query_row = ptr<const int>(*query_rows);
    p.query_row_stride = query.stride(1);
  }
  p.gists = ptr<const float>(gists);
  p.gist_count = ptr<const int>(gist_count);
  p.row_pos_off = ptr<const int>(row_pos_off);
  p.row_ref_off = ptr<const int>(row_ref_off);
  p.ref_pos_off = ptr<const int>(ref_pos_off);
  p.pos_chunk = ptr<const int>(pos_chunk);
  p.pos_ref = ptr<const int>(pos_ref);
  p.pos_rank = ptr<const int>(pos_rank);
  p.chunk_start = ptr<const int>(chunk_start);
  p.chunk_len = ptr<const int>(chunk_len);
  p.chunk_pool_row = ptr<const int>(chunk_pool_row);
  p.k_ref = k_ref;
  p.k_chunk = k_chunk;
  p.gist_agg = gist_agg;
  p.ref_agg = ref_agg;
  p.threshold = (float)threshold;
  p.budget = budget;
  p.budget_rows = optr<int>(budget_rows);
  p.gist_only = gist_only;
  p.full_reference = full_reference;
  p.deduplicate = deduplicate;
  p.global_chunks = global_chunks;
  TORCH_CHECK(!(global_chunks && full_reference), "global_chunks search with full-reference expansion is not supported");
  p.max_sel = max_sel;
  p.max_mem = max_mem;
  auto io = query.options().dtype(at::kInt);
  auto fo = query.options().dtype(at::kFloat);
  // the kernel writes every slot of ints and the trace tables; mem_idx is valid up to mem_len
  auto mem_idx = torch::empty({p.B, std::max<int64_t>(max_mem, 1)}, io);
  auto ints = torch::empty({5, p.B}, io);  // mem_len, sel_count, candidates, duplicates, status
  auto sel_i = torch::empty({4, p.B, std::max<int64_t>(max_sel, 1)}, io);
  auto sel_f = torch::empty({3, p.B, std::max<int64_t>(max_sel, 1)}, fo);
  p.max_sel = std::max<int64_t>(max_sel, 1);
  p.max_mem = std::max<int64_t>(max_mem, 1);
  p.mem_idx = ptr<int>(mem_idx);
  p.mem_len = ptr<int>(ints);
  p.sel_count = p.mem_len + p.B;
  p.routing_candidates = p.mem_len + 2 * p.B;
  p.duplicate_tokens = p.mem_len + 3 * p.B;
  p.status = p.mem_len + 4 * p.B;
  const int64_t s = (int64_t)p.B * std::max<int64_t>(max_sel, 1);
  p.sel_chunk = ptr<int>(sel_i);
  p.sel_ref_rank = p.sel_chunk + s;
  p.sel_chunk_rank = p.sel_chunk + 2 * s;
  p.sel_win_index = p.sel_chunk + 3 * s;
  p.sel_ref_score = ptr<float>(sel_f);
  p.sel_chunk_score = p.sel_ref_score + s;
  p.sel_win_score = p.sel_ref_score + 2 * s;
  check(pra_route(p, stream()), "route");
  return {mem_idx, ints, sel_i, sel_f};
}

}  // namespace

// ---------------------------------------------------------------- tensor-parallel collectives
void tp_allreduce(std::vector<int64_t> parts, std::vector<int64_t> sigs, int64_t rank,
                  c10::optional<torch::Tensor> residual, torch::Tensor out, torch::Tensor epochs, int64_t max_spins,
                  torch::Tensor error) {
  c10::cuda::CUDAGuard guard(out.device());
  const int world = parts.size();
  TORCH_CHECK(world >= 1 && world <= TP_MAX_RANKS && (int)sigs.size() == world, "one part/signal per rank");
  expect(out, at::kBFloat16, "out");
  TORCH_CHECK(out.is_contiguous(), "out must be contiguous");
  TpAllreduceArgs a{};
  for (int p = 0; p < world; ++p) {
    a.part[p] = reinterpret_cast<const __nv_bfloat16*>(parts[p]);
    a.sig[p] = reinterpret_cast<uint32_t*>(sigs[p]);
  }
  if (residual.has_value()) {
    TORCH_CHECK(residual->is_contiguous() && residual->numel() == out.numel(), "residual must match out");
    a.residual = ptr<const __nv_bfloat16>(*residual);
  }
  a.out = ptr<__nv_bfloat16>(out);
  a.rank = rank;
  a.world = world;
  a.n = out.numel();
  TORCH_CHECK(epochs.scalar_type() == at::kInt && epochs.numel() >= TP_MAX_BLOCKS, "epochs: int32 [TP_MAX_BLOCKS]");
  a.epochs = reinterpret_cast<uint32_t*>(epochs.data_ptr());
  a.max_spins = max_spins;
  a.error = ptr<int>(error);
  check(pra_tp_allreduce(a, stream()), "tp_allreduce");
}

void tp_allgather(torch::Tensor src, std::vector<int64_t> dsts, std::vector<int64_t> sigs, int64_t rank,
                  torch::Tensor epochs, int64_t max_spins, torch::Tensor error) {
  c10::cuda::CUDAGuard guard(src.device());
  const int world = dsts.size();
  TORCH_CHECK(world >= 1 && world <= TP_MAX_RANKS && (int)sigs.size() == world, "one dst/signal per rank");
  expect(src, at::kFloat, "src");
  TORCH_CHECK(src.dim() == 2 && src.stride(1) == 1, "src must be [rows, cols] row-major");
  TpAllgatherArgs a{};
  a.src = ptr<const float>(src);
  a.src_stride = src.stride(0);
  for (int p = 0; p < world; ++p) {
    a.dst[p] = reinterpret_cast<float*>(dsts[p]);
    a.sig[p] = reinterpret_cast<uint32_t*>(sigs[p]);
  }
  a.rank = rank;
  a.world = world;
  a.rows = src.size(0);
  a.cols = src.size(1);
  TORCH_CHECK(epochs.scalar_type() == at::kInt && epochs.numel() >= TP_MAX_BLOCKS, "epochs: int32 [TP_MAX_BLOCKS]");
  a.epochs = reinterpret_cast<uint32_t*>(epochs.data_ptr());
  a.max_spins = max_spins;
  a.error = ptr<int>(error);
  check(pra_tp_allgather(a, stream()), "tp_allgather");
}

// ---------------------------------------------------------------- decode GEMM
// out[M, N] (+ out2 for columns >= split_col) = x[M, K] w[N, K]^T (+ bias, + residual); with peer
// addresses in recv / flags (one per rank) the result is summed over the ranks (row-parallel
// projection) inside the same kernel.  splits <= 0 picks the K split from the SM count.
static void set_folded_norm(DecodeGemmArgs& a, const c10::optional<torch::Tensor>& ss_out,
                            const c10::optional<torch::Tensor>& ss_in, int64_t ss_tiles, int64_t ss_dim,
                            double ss_eps);

void decode_gemm(torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> bias,
                 c10::optional<torch::Tensor> residual, torch::Tensor out, c10::optional<torch::Tensor> out2,
                 int64_t split_col, int64_t splits, std::vector<int64_t> recv, std::vector<int64_t> flags, int64_t rank,
                 c10::optional<torch::Tensor> epochs, int64_t max_spins, c10::optional<torch::Tensor> error,
                 bool swiglu, c10::optional<torch::Tensor> ss_out, c10::optional<torch::Tensor> ss_in, int64_t ss_tiles,
                 int64_t ss_dim, double ss_eps) {
  c10::cuda::CUDAGuard guard(x.device());
  expect(x, at::kBFloat16, "x");
  expect(w, at::kBFloat16, "w");
  const bool f32 = out.scalar_type() == at::kFloat;  // routing scores: fp32, no epilogue terms
  if (!f32) expect(out, at::kBFloat16, "out");
  TORCH_CHECK(!f32 || (out.is_cuda() && !bias.has_value() && !residual.has_value() && !out2.has_value() && recv.empty()),
              "decode_gemm: an fp32 output takes no bias, residual, second output or all-reduce");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && w.dim() == 2 && w.is_contiguous() && w.size(1) == x.size(1),
              "decode_gemm: x [M, K] (unit column stride) and w [N, K] contiguous");
  TORCH_CHECK(out.dim() == 2 && out.stride(1) == 1 && out.size(0) == x.size(0), "decode_gemm: out [M, >=cols]");
  DecodeGemmArgs a{};
  a.x = ptr<const __nv_bfloat16>(x);
  a.ldx = x.stride(0);
  a.w = ptr<const __nv_bfloat16>(w);
  a.M = x.size(0);
  a.N = w.size(0);
  a.K = w.size(1);
  if (f32) a.out_f32 = ptr<float>(out);
  else a.out = ptr<__nv_bfloat16>(out);
  a.ldo = out.stride(0);
  a.bias = optr<__nv_bfloat16>(bias);
  if (bias.has_value()) TORCH_CHECK(bias->numel() == a.N && bias->scalar_type() == at::kBFloat16, "bias [N] bf16");
  if (residual.has_value()) {
    expect(*residual, at::kBFloat16, "residual");
    TORCH_CHECK(residual->dim() == 2 && residual->stride(0) == a.ldo && residual->stride(1) == 1 &&
                    residual->size(0) == a.M, "residual must share out's row stride");
    a.residual = ptr<const __nv_bfloat16>(*residual);
  }
  a.split_col = out2.has_value() ? (int)split_col : a.N;
  if (out2.has_value()) {
    expect(*out2, at::kBFloat16, "out2");
    TORCH_CHECK(out2->dim() == 2 && out2->stride(1) == 1 && out2->size(0) == a.M && out2->size(1) >= a.N - split_col,
                "out2 [M, >= N - split_col]");
    a.out2 = ptr<__nv_bfloat16>(*out2);
    a.ldo2 = out2->stride(0);
  }
  a.swiglu = swiglu ? 1 : 0;
  set_folded_norm(a, ss_out, ss_in, ss_tiles, ss_dim, ss_eps);
  TORCH_CHECK(swiglu ? out.size(1) >= a.N / 2 : out.size(1) >= a.split_col, "out narrower than its columns");
  const int tiles = (a.N + 127) / 128, nkb = a.K / 64;
  static int sm_cache[64] = {};
  int& sms = sm_cache[x.device().index() & 63];
  if (sms == 0) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, x.device().index());
  if (splits <= 0) splits = pra_decode_gemm_splits(tiles, nkb, sms);
  a.splits = (int)splits;
  a.world = 1;
  if (!recv.empty()) {
    const int world = recv.size();
    TORCH_CHECK(world <= TP_MAX_RANKS && (int)flags.size() == world && epochs.has_value() && error.has_value(),
                "fused all-reduce needs one receive buffer and one flag area per rank, epochs and an error word");
    TORCH_CHECK(!out2.has_value(), "the fused all-reduce writes one output");
    TORCH_CHECK(out.is_contiguous() && out.size(1) == a.N, "fused all-reduce: out [M, N] contiguous");
    a.world = world;
    a.rank = rank;
    for (int p = 0; p < world; ++p) {
      a.recv[p] = reinterpret_cast<__nv_bfloat16*>(recv[p]);
      a.flags[p] = reinterpret_cast<uint32_t*>(flags[p]);
    }
    TORCH_CHECK(epochs->scalar_type() == at::kInt && epochs->numel() >= DG_MAX_TILES * DG_MAX_SPLITS,
                "epochs: int32 [decode_gemm_flag_slots()]");
    a.epochs = reinterpret_cast<uint32_t*>(epochs->data_ptr());
    a.max_spins = max_spins;
    a.error = ptr<int>(*error);
  }
  check(pra_decode_gemm(a, stream()), "decode_gemm");
}

// Decode QKV projection with the rotary epilogue: one GEMM writes the rotated query rows, the
// rotated keys and the values straight into their cache rows, and (columns >= v_end) the
// routing query.
void decode_qkv_rope(torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> bias, torch::Tensor q_out,
                     torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor cache_rows, torch::Tensor pos,
                     torch::Tensor cos_t, torch::Tensor sin_t, int64_t head_dim, int64_t q_end, int64_t k_end,
                     int64_t v_end, c10::optional<torch::Tensor> route_out, c10::optional<torch::Tensor> ss_in,
                     int64_t ss_tiles, int64_t ss_dim, double ss_eps) {
  c10::cuda::CUDAGuard guard(x.device());
  expect(x, at::kBFloat16, "x");
  expect(w, at::kBFloat16, "w");
  expect(q_out, at::kBFloat16, "q_out");
  expect(k_cache, at::kBFloat16, "k_cache");
  expect(v_cache, at::kBFloat16, "v_cache");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && w.is_contiguous() && w.size(1) == x.size(1), "x [M, K], w [N, K]");
  TORCH_CHECK(cache_rows.scalar_type() == at::kInt && pos.scalar_type() == at::kInt &&
                  cache_rows.numel() == x.size(0) && pos.numel() == x.size(0), "cache_rows / pos: int32 [M]");
  TORCH_CHECK(cos_t.scalar_type() == at::kFloat && sin_t.scalar_type() == at::kFloat, "cos / sin tables: fp32");
  TORCH_CHECK(k_cache.stride(-1) == 1 && v_cache.stride(-1) == 1 && k_cache.stride(0) == v_cache.stride(0),
              "caches: row-major rows with one stride");
  DecodeGemmArgs a{};
  a.x = ptr<const __nv_bfloat16>(x);
  a.ldx = x.stride(0);
  a.w = ptr<const __nv_bfloat16>(w);
  a.M = x.size(0);
  a.N = w.size(0);
  a.K = w.size(1);
  a.bias = optr<__nv_bfloat16>(bias);
  a.split_col = (int)v_end;
  if (route_out.has_value()) {
    expect(*route_out, at::kBFloat16, "route_out");
    a.out2 = ptr<__nv_bfloat16>(*route_out);
    a.ldo2 = route_out->stride(0);
  }
  a.pos = ptr<const int>(pos);
  a.cos_t = ptr<const float>(cos_t);
  a.sin_t = ptr<const float>(sin_t);
  a.head_dim = (int)head_dim;
  a.q_end = (int)q_end;
  a.k_end = (int)k_end;
  a.q_out = ptr<__nv_bfloat16>(q_out);
  a.ldq = q_out.stride(0);
  a.k_cache = ptr<__nv_bfloat16>(k_cache);
  a.v_cache = ptr<__nv_bfloat16>(v_cache);
  a.ld_cache = k_cache.stride(0);
  a.cache_rows = ptr<const int>(cache_rows);
  a.out = a.q_out;
  a.ldo = a.ldq;
  static int sm_cache[64] = {};
  int& sms = sm_cache[x.device().index() & 63];
  if (sms == 0) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, x.device().index());
  const int tiles = (a.N + 127) / 128, nkb = a.K / 64;
  a.splits = pra_decode_gemm_splits(tiles, nkb, sms);
  a.world = 1;
  set_folded_norm(a, c10::nullopt, ss_in, ss_tiles, ss_dim, ss_eps);
  check(pra_decode_gemm(a, stream()), "decode_qkv_rope");
}

// ---------------------------------------------------------------- Llama-family ops
// Rotary copy: rows of src (heads * head_dim, unit stride) to dst rows (dst_rows or identity).
void rope_copy(torch::Tensor src, torch::Tensor dst, c10::optional<torch::Tensor> dst_rows,
               c10::optional<torch::Tensor> pos, c10::optional<torch::Tensor> cos_t,
               c10::optional<torch::Tensor> sin_t, int64_t heads, int64_t head_dim) {
  c10::cuda::CUDAGuard guard(src.device());
  expect(src, at::kBFloat16, "src");
  expect(dst, at::kBFloat16, "dst");
  TORCH_CHECK(src.dim() == 2 && dst.dim() == 2 && src.stride(1) == 1 && dst.stride(1) == 1, "rows must be 2-D");
  TORCH_CHECK(src.size(1) >= heads * head_dim && dst.size(1) >= heads * head_dim, "row too short");
  TORCH_CHECK(pos.has_value() == cos_t.has_value(), "positions need the cos/sin tables");
  RopeCopyArgs a{};
  a.src = ptr<const __nv_bfloat16>(src);
  a.src_stride = src.stride(0);
  a.dst = ptr<__nv_bfloat16>(dst);
  a.dst_stride = dst.stride(0);
  a.dst_rows = optr<int>(dst_rows);
  a.pos = optr<int>(pos);
  a.cos_t = optr<float>(cos_t);
  a.sin_t = optr<float>(sin_t);
  a.M = src.size(0);
  a.heads = heads;
  a.head_dim = head_dim;
  check(pra_rope_copy(a, stream()), "rope_copy");
}

static BoundsStatus* bounds_word(const torch::Device& dev);

// Folded-RMSNorm arguments of a decode GEMM (see DecodeGemmArgs::ss_out / ss_in).
static void set_folded_norm(DecodeGemmArgs& a, const c10::optional<torch::Tensor>& ss_out,
                            const c10::optional<torch::Tensor>& ss_in, int64_t ss_tiles, int64_t ss_dim,
                            double ss_eps) {
  if (ss_out.has_value()) {
    TORCH_CHECK(ss_out->scalar_type() == at::kFloat && ss_out->is_cuda() && ss_out->is_contiguous() &&
                    ss_out->numel() >= (int64_t)((a.N + 127) / 128) * 64,
                "ss_out: fp32 [tiles, 64]");
    a.ss_out = ptr<float>(*ss_out);
  }
  if (ss_in.has_value()) {
    TORCH_CHECK(ss_in->scalar_type() == at::kFloat && ss_in->is_cuda() && ss_in->is_contiguous() &&
                    ss_tiles > 0 && ss_in->numel() >= ss_tiles * 64 && ss_dim > 0,
                "ss_in: fp32 [ss_tiles, 64] with ss_dim > 0");
    a.ss_in = ptr<const float>(*ss_in);
    a.ss_tiles = (int)ss_tiles;
    a.ss_dim = (int)ss_dim;
    a.ss_eps = (float)ss_eps;
  }
}

// x [B, d], pos / rows / new_len [B] int32 for one decode step (see pra_decode_prologue).
std::vector<torch::Tensor> decode_prologue(torch::Tensor ids, torch::Tensor cache_len,
                                           c10::optional<torch::Tensor> pos_offset, torch::Tensor embed,
                                           int64_t max_len, c10::optional<torch::Tensor> ss_out) {
  c10::cuda::CUDAGuard guard(embed.device());
  expect(embed, at::kBFloat16, "embed");
  TORCH_CHECK(ids.scalar_type() == at::kLong && ids.is_cuda() && ids.is_contiguous(), "ids: int64 CUDA [B]");
  TORCH_CHECK(cache_len.scalar_type() == at::kInt && cache_len.is_contiguous() && cache_len.numel() == ids.numel(),
              "cache_len: int32 [B]");
  TORCH_CHECK(embed.is_contiguous() && embed.dim() == 2, "embed: [vocab, d] contiguous");
  const int64_t B = ids.numel();
  DecodePrologueArgs a{};
  a.ids = ids.data_ptr<int64_t>();
  a.cache_len = ptr<const int>(cache_len);
  if (pos_offset.has_value()) {
    TORCH_CHECK(pos_offset->scalar_type() == at::kInt && pos_offset->numel() == B && pos_offset->is_contiguous(),
                "pos_offset: int32 [B]");
    a.pos_offset = ptr<const int>(*pos_offset);
  }
  a.embed = ptr<const __nv_bfloat16>(embed);
  a.vocab = embed.size(0);
  a.d = embed.size(1);
  a.B = (int)B;
  a.max_len = (int)max_len;
  auto x = torch::empty({B, a.d}, embed.options());
  auto io = torch::empty({3, B}, cache_len.options());
  a.x = ptr<__nv_bfloat16>(x);
  a.pos = ptr<int>(io[0]);
  a.rows = ptr<int>(io[1]);
  a.new_len = ptr<int>(io[2]);
  a.bounds = bounds_word(embed.device());
  if (ss_out.has_value()) {
    TORCH_CHECK(ss_out->scalar_type() == at::kFloat && ss_out->is_contiguous() && ss_out->numel() >= B,
                "ss_out: fp32 [>= B]");
    a.ss_out = ptr<float>(*ss_out);
  }
  check(pra_decode_prologue(a, stream()), "decode_prologue");
  return {x, io[0], io[1], io[2]};
}

void silu_mul(torch::Tensor gate_up, torch::Tensor out, int64_t block) {
  c10::cuda::CUDAGuard guard(gate_up.device());
  expect(gate_up, at::kBFloat16, "gate_up");
  TORCH_CHECK(gate_up.is_contiguous() && out.is_contiguous() && gate_up.size(1) == 2 * out.size(1),
              "gate_up must be [M, 2F] and out [M, F]");
  check(pra_silu_mul(ptr<const __nv_bfloat16>(gate_up), gate_up.size(0), out.size(1), (int)block,
                     ptr<__nv_bfloat16>(out), stream()),
        "silu_mul");
}

// Split-K decode attention.  q [B, H*Dh]; memory pool k/v views [rows, >= Hkv*Dh] (row stride
// shared); local caches [B, max_len, Hkv*Dh] views.  Returns {out [B, H*Dh]} and, with
// export_partials, also the merged unnormalised (out, (max, sum)) fp32 partials.
// ---------------------------------------------------------------- bounds-checked variants
// set_bounds_check(true) makes the gather and routing launches below run their checked
// variants: the first out-of-range index is recorded in a per-device BoundsStatus and the
// access is skipped.  Enable it before capturing a CUDA graph (the status word is allocated on
// the first checked launch of each device).
static bool g_bounds_check = false;
static std::map<int, torch::Tensor> g_bounds_words;

static BoundsStatus* bounds_word(const torch::Device& dev) {
  if (!g_bounds_check) return nullptr;
  auto it = g_bounds_words.find(dev.index());
  if (it == g_bounds_words.end()) {
    auto t = torch::zeros({(int64_t)sizeof(BoundsStatus)}, torch::dtype(torch::kUInt8).device(dev));
    it = g_bounds_words.emplace(dev.index(), t).first;
  }
  return reinterpret_cast<BoundsStatus*>(it->second.data_ptr());
}

void set_bounds_check(bool on) { g_bounds_check = on; }
bool bounds_check_enabled() { return g_bounds_check; }

// {code, kernel check id, offending value, bound} of the first violation on `device` (zeros: clean).
std::vector<int64_t> bounds_status(int64_t device) {
  auto it = g_bounds_words.find((int)device);
  if (it == g_bounds_words.end()) return {0, 0, 0, 0};
  BoundsStatus h{};
  auto host = it->second.cpu();
  std::memcpy(&h, host.data_ptr(), sizeof h);
  return {h.code, h.kernel, h.index, h.limit};
}

void bounds_reset(int64_t device) {
  auto it = g_bounds_words.find((int)device);
  if (it != g_bounds_words.end()) it->second.zero_();
}

std::vector<torch::Tensor> decode_attention(torch::Tensor q, int64_t heads, int64_t kv_heads, int64_t head_dim,
                                            c10::optional<torch::Tensor> mem_k, c10::optional<torch::Tensor> mem_v,
                                            c10::optional<torch::Tensor> mem_idx,
                                            c10::optional<torch::Tensor> mem_len,
                                            c10::optional<torch::Tensor> loc_k, c10::optional<torch::Tensor> loc_v,
                                            c10::optional<torch::Tensor> loc_len, int64_t max_keys,
                                            int64_t split_keys, bool export_partials, int64_t mem_splits,
                                            int64_t mem_split_keys,
                                            int64_t split_lo, int64_t split_count, int64_t phase,
                                            c10::optional<torch::Tensor> part_o_in,
                                            c10::optional<torch::Tensor> part_ml_in, int64_t max_ctas) {
  c10::cuda::CUDAGuard guard(q.device());
  expect(q, at::kBFloat16, "q");
  TORCH_CHECK(q.dim() == 2 && q.stride(1) == 1 && q.size(1) == heads * head_dim, "q must be [B, H*Dh]");
  DecodeAttnParams p{};
  p.q = ptr<const __nv_bfloat16>(q);
  p.q_row = q.stride(0);
  p.B = q.size(0);
  p.H = heads;
  p.Hkv = kv_heads;
  if (mem_idx.has_value() && mem_idx->numel() > 0) {
    TORCH_CHECK(mem_k.has_value() && mem_v.has_value() && mem_len.has_value(), "memory needs k, v, idx and len");
    TORCH_CHECK(mem_k->stride(-1) == 1 && mem_v->stride(0) == mem_k->stride(0), "memory pools share a row stride");
    expect_pool(*mem_k, "mem_k");
    expect_pool(*mem_v, "mem_v");
    p.mem_k = pool_ptr<const __nv_bfloat16>(*mem_k);
    p.mem_v = pool_ptr<const __nv_bfloat16>(*mem_v);
    p.mem_row = mem_k->stride(0);
    p.mem_idx = ptr<const int>(*mem_idx);
    p.mem_max = mem_idx->size(1);
    p.mem_len = ptr<const int>(*mem_len);
    p.mem_rows = mem_k->size(0);
    p.mem_on_device = mem_k->is_cuda() ? 1 : 0;
  }
  if (loc_k.has_value() && loc_k->numel() > 0) {
    TORCH_CHECK(loc_k->dim() == 3 && loc_k->stride(2) == 1 && loc_v->strides() == loc_k->strides(),
                "local caches must be [B, max_len, width] views with equal strides");
    TORCH_CHECK(loc_len.has_value(), "local cache needs lengths");
    p.loc_k = ptr<const __nv_bfloat16>(*loc_k);
    p.loc_v = ptr<const __nv_bfloat16>(*loc_v);
    p.loc_batch = loc_k->stride(0);
    p.loc_row = loc_k->stride(1);
    p.loc_len = ptr<const int>(*loc_len);
    p.loc_cap = loc_k->size(1);
  }
  p.bounds = bounds_word(q.device());
  p.scale = 1.0f / std::sqrt((float)head_dim);
  p.split_keys = split_keys;
  p.n_split = std::max<int64_t>(1, (max_keys + split_keys - 1) / split_keys);
  if (mem_splits > 0) {  // separate memory and local splits: the local ones tile the cache capacity
    TORCH_CHECK(loc_k.has_value() && loc_k->numel() > 0, "separate memory / local splits need the local cache");
    p.mem_splits = mem_splits;
    p.mem_split_keys = mem_split_keys;
    p.n_split = mem_splits + (loc_k->size(1) + split_keys - 1) / split_keys;
  }
  p.split_lo = split_lo;
  p.split_count = split_count;
  p.phase = phase;
  p.max_ctas = (int)max_ctas;
  auto fo = q.options().dtype(at::kFloat);
  torch::Tensor part_o, part_ml;
  if (part_o_in.has_value()) {  // caller-owned partials (a launch split across streams shares them)
    TORCH_CHECK(part_ml_in.has_value(), "part_o and part_ml go together");
    part_o = *part_o_in;
    part_ml = *part_ml_in;
    expect(part_o, at::kFloat, "part_o");
    expect(part_ml, at::kFloat, "part_ml");
    TORCH_CHECK(part_o.is_contiguous() && part_ml.is_contiguous() &&
                    part_o.numel() >= (int64_t)p.B * heads * p.n_split * head_dim &&
                    part_ml.numel() >= (int64_t)p.B * heads * p.n_split * 2,
                "partials too small for [B, H, n_split, Dh]");
  } else {
    TORCH_CHECK(phase == 0, "a phase-split decode attention needs caller-owned partials");
    part_o = torch::empty({p.B, heads, p.n_split, head_dim}, fo);
    part_ml = torch::empty({p.B, heads, p.n_split, 2}, fo);
  }
  auto out = torch::empty({p.B, heads * head_dim}, q.options());
  p.part_o = ptr<float>(part_o);
  p.part_ml = ptr<float>(part_ml);
  p.out = ptr<__nv_bfloat16>(out);
  p.out_row = out.stride(0);
  std::vector<torch::Tensor> result{out};
  if (export_partials) {
    auto eo = torch::empty({p.B, heads, head_dim}, fo), eml = torch::empty({p.B, heads, 2}, fo);
    p.export_o = ptr<float>(eo);
    p.export_ml = ptr<float>(eml);
    result.push_back(eo);
    result.push_back(eml);
  }
  check(pra_decode_attention(p, head_dim, stream()), "decode_attention");
  return result;
}

// Exact top-k routing from approximate scores.  Returns {mem_idx [B, mem_max], mem_len [B],
// selected chunk ids [B, k]}.
std::vector<torch::Tensor> route_topk(torch::Tensor scores, torch::Tensor query, torch::Tensor gists,
                                      torch::Tensor ns_start, torch::Tensor ns_end, torch::Tensor chunk_len,
                                      torch::Tensor chunk_row0, int64_t k, int64_t k_cand, int64_t budget,
                                      int64_t mem_max, bool local, int64_t id_offset, int64_t gists_per_chunk,
                                      int64_t segments, int64_t pool_rows, c10::optional<torch::Tensor> page_table,
                                      c10::optional<torch::Tensor> trace) {
  c10::cuda::CUDAGuard guard(scores.device());
  expect(scores, at::kFloat, "scores");
  TORCH_CHECK(query.is_cuda() && (query.scalar_type() == at::kFloat || query.scalar_type() == at::kBFloat16),
              "query must be a CUDA fp32 or bf16 tensor");
  expect(gists, at::kFloat, "gists");
  TORCH_CHECK(scores.dim() == 2 && scores.stride(1) == 1 && query.stride(-1) == 1 && gists.is_contiguous(),
              "route_topk layouts");
  RouteTopkArgs a{};
  a.B = scores.size(0);
  a.D = gists.size(-1);
  a.G = gists_per_chunk;
  a.segments = std::max<int64_t>(segments, 1);
  TORCH_CHECK(a.segments == 1 || local, "segmented selection writes local candidates (merge them afterwards)");
  a.scores = ptr<const float>(scores);
  a.score_stride = scores.stride(0);
  if (query.scalar_type() == at::kBFloat16) a.query_bf16 = ptr<const __nv_bfloat16>(query);
  else a.query = ptr<const float>(query);
  a.query_stride = query.stride(0);
  a.gists = ptr<const float>(gists);
  a.ns_start = ptr<const int>(ns_start);
  a.ns_end = ptr<const int>(ns_end);
  a.chunk_len = ptr<const int>(chunk_len);
  a.chunk_row0 = ptr<const int>(chunk_row0);
  a.k = k;
  a.k_cand = k_cand;
  a.budget = budget;
  a.n_chunks = scores.size(1) / std::max<int64_t>(gists_per_chunk, 1);
  a.pool_rows = pool_rows;
  a.bounds = bounds_word(scores.device());
  if (page_table.has_value() && page_table->numel() > 0) {
    TORCH_CHECK(page_table->scalar_type() == at::kInt && page_table->dim() == 2 && page_table->stride(1) == 1 &&
                    page_table->size(0) == a.B && a.segments == 1,
                "page_table must be int32 [B, pages] (one segment per row)");
    a.page_table = ptr<const int>(*page_table);
    a.page_stride = page_table->stride(0);
  }
  if (trace.has_value()) {
    TORCH_CHECK(trace->scalar_type() == at::kLong && trace->numel() >= 8 && trace->is_cuda(), "trace: int64 [8]");
    a.trace = reinterpret_cast<long long*>(trace->data_ptr());
  }
  auto io = scores.options().dtype(at::kInt);
  if (local) {  // best k per (row, segment) (exact scores, global ids) for a merge
    if (a.segments > 1) {
      const int64_t width = scores.size(1) / std::max<int64_t>(gists_per_chunk, 1);
      a.seg_len = (width + a.segments - 1) / a.segments;
    }
    auto cs = torch::empty({a.B * a.segments, std::max<int64_t>(k, 1)}, scores.options());
    auto ci = torch::empty({a.B * a.segments, std::max<int64_t>(k, 1)}, io);
    a.cand_score = ptr<float>(cs);
    a.cand_id = ptr<int>(ci);
    a.id_offset = id_offset;
    check(pra_route_topk(a, stream()), "route_topk");
    return {cs, ci};
  }
  auto mem_idx = torch::empty({a.B, std::max<int64_t>(mem_max, 1)}, io);
  auto mem_len = torch::empty({a.B}, io);
  auto sel = torch::empty({a.B, std::max<int64_t>(k, 1)}, io);
  a.mem_idx = ptr<int>(mem_idx);
  a.mem_max = std::max<int64_t>(mem_max, 1);
  a.mem_len = ptr<int>(mem_len);
  a.sel_out = ptr<int>(sel);
  check(pra_route_topk(a, stream()), "route_topk");
  return {mem_idx, mem_len, sel};
}

// Local exact top-k with the cross-GPU candidate exchange and merge fused in (one kernel, one
// segment per row).  Returns {mem_idx [B, mem_max], mem_len [B], selected chunk ids [B, k]}.
std::vector<torch::Tensor> route_topk_exchange(torch::Tensor scores, torch::Tensor query, torch::Tensor gists,
                                               torch::Tensor ns_start, torch::Tensor ns_end, int64_t k, int64_t k_cand,
                                               int64_t budget, int64_t mem_max, int64_t id_offset,
                                               int64_t gists_per_chunk, std::vector<int64_t> recv,
                                               std::vector<int64_t> flags, torch::Tensor epochs, int64_t rank,
                                               int64_t B_max, torch::Tensor global_len, torch::Tensor global_row0,
                                               int64_t max_spins, torch::Tensor error, int64_t pool_rows) {
  c10::cuda::CUDAGuard guard(scores.device());
  expect(scores, at::kFloat, "scores");
  TORCH_CHECK(query.is_cuda() && (query.scalar_type() == at::kFloat || query.scalar_type() == at::kBFloat16),
              "query must be a CUDA fp32 or bf16 tensor");
  expect(gists, at::kFloat, "gists");
  TORCH_CHECK(scores.dim() == 2 && scores.stride(1) == 1 && query.stride(-1) == 1 && gists.is_contiguous(),
              "route_topk_exchange layouts");
  TORCH_CHECK(recv.size() == flags.size() && recv.size() >= 2 && recv.size() <= (size_t)TP_MAX_RANKS,
              "one receive buffer and one flag array per rank");
  TORCH_CHECK(epochs.scalar_type() == at::kInt && error.scalar_type() == at::kInt, "int32 epochs / error");
  RouteTopkArgs a{};
  a.B = scores.size(0);
  a.D = gists.size(-1);
  a.G = gists_per_chunk;
  a.segments = 1;
  a.scores = ptr<const float>(scores);
  a.score_stride = scores.stride(0);
  if (query.scalar_type() == at::kBFloat16) a.query_bf16 = ptr<const __nv_bfloat16>(query);
  else a.query = ptr<const float>(query);
  a.query_stride = query.stride(0);
  a.gists = ptr<const float>(gists);
  a.ns_start = ptr<const int>(ns_start);
  a.ns_end = ptr<const int>(ns_end);
  a.chunk_len = ptr<const int>(global_len);
  a.chunk_row0 = ptr<const int>(global_row0);
  a.k = k;
  a.k_cand = k_cand;
  a.budget = budget;
  a.id_offset = id_offset;
  a.n_chunks = scores.size(1) / std::max<int64_t>(gists_per_chunk, 1);
  a.pool_rows = pool_rows;
  a.bounds = bounds_word(scores.device());
  auto io = scores.options().dtype(at::kInt);
  auto mem_idx = torch::empty({a.B, std::max<int64_t>(mem_max, 1)}, io);
  auto mem_len = torch::empty({a.B}, io);
  auto sel = torch::empty({a.B, std::max<int64_t>(k, 1)}, io);
  a.mem_idx = ptr<int>(mem_idx);
  a.mem_max = std::max<int64_t>(mem_max, 1);
  a.mem_len = ptr<int>(mem_len);
  a.sel_out = ptr<int>(sel);
  RouteExchangeArgs x{};
  x.world = recv.size();
  for (int p = 0; p < x.world; ++p) {
    x.recv[p] = reinterpret_cast<float*>(recv[p]);
    x.flags[p] = reinterpret_cast<uint32_t*>(flags[p]);
  }
  x.epochs = reinterpret_cast<uint32_t*>(epochs.data_ptr());
  x.rank = rank;
  x.B_max = B_max;
  x.global_len = ptr<const int>(global_len);
  x.global_row0 = ptr<const int>(global_row0);
  x.max_spins = max_spins;
  x.error = ptr<int>(error);
  check(pra_route_topk_exchange(a, x, stream()), "route_topk_exchange");
  return {mem_idx, mem_len, sel};
}

// Merge per-rank candidates ([B, world * 2k]: per rank k scores then k ids as int bits).
std::vector<torch::Tensor> route_merge(torch::Tensor cands, int64_t world, int64_t k, int64_t budget,
                                       torch::Tensor chunk_len, torch::Tensor chunk_row0, int64_t mem_max,
                                       bool local, int64_t pool_rows) {
  c10::cuda::CUDAGuard guard(cands.device());
  expect(cands, at::kFloat, "cands");
  TORCH_CHECK(cands.dim() == 2 && cands.stride(1) == 1 && cands.size(1) == world * 2 * k, "cands [B, world*2k]");
  RouteMergeArgs a{};
  a.B = cands.size(0);
  a.world = world;
  a.k = k;
  a.cands = ptr<const float>(cands);
  a.row_stride = cands.stride(0);
  a.budget = budget;
  a.chunk_len = ptr<const int>(chunk_len);
  a.chunk_row0 = ptr<const int>(chunk_row0);
  a.n_chunks = chunk_len.numel();
  a.pool_rows = pool_rows;
  a.bounds = bounds_word(cands.device());
  auto io = cands.options().dtype(at::kInt);
  if (local) {  // merged best k as candidates (for a further merge across GPUs)
    auto cs = torch::empty({a.B, std::max<int64_t>(k, 1)}, cands.options());
    auto ci = torch::empty({a.B, std::max<int64_t>(k, 1)}, io);
    a.cand_score = ptr<float>(cs);
    a.cand_id = ptr<int>(ci);
    check(pra_route_merge(a, stream()), "route_merge");
    return {cs, ci};
  }
  auto mem_idx = torch::empty({a.B, std::max<int64_t>(mem_max, 1)}, io);
  auto mem_len = torch::empty({a.B}, io);
  auto sel = torch::empty({a.B, std::max<int64_t>(k, 1)}, io);
  a.mem_idx = ptr<int>(mem_idx);
  a.mem_max = std::max<int64_t>(mem_max, 1);
  a.mem_len = ptr<int>(mem_len);
  a.sel_out = ptr<int>(sel);
  check(pra_route_merge(a, stream()), "route_merge");
  return {mem_idx, mem_len, sel};
}

// Combine gathered attention partials [B, world * H * (D + 2)] -> [B, H * D] bf16.
torch::Tensor combine_partials(torch::Tensor parts, int64_t world, int64_t heads, int64_t head_dim) {
  c10::cuda::CUDAGuard guard(parts.device());
  expect(parts, at::kFloat, "parts");
  TORCH_CHECK(parts.is_contiguous() && parts.size(-1) == world * heads * (head_dim + 2), "parts layout");
  const int64_t B = parts.size(0);
  auto out = torch::empty({B, heads * head_dim}, parts.options().dtype(at::kBFloat16));
  check(pra_combine_partials(ptr<const float>(parts), B, world, heads, head_dim, ptr<__nv_bfloat16>(out), stream()),
        "combine_partials");
  return out;
}

// ---------------------------------------------------------------- embeddings
// ids int32 [M]; positions int32 [M] or null (position = m % period); tables bf16 [*, D].
torch::Tensor embed_add(torch::Tensor ids, c10::optional<torch::Tensor> positions, int64_t period, torch::Tensor tok,
                        torch::Tensor pos) {
  c10::cuda::CUDAGuard guard(ids.device());
  TORCH_CHECK(ids.scalar_type() == at::kInt && ids.is_contiguous(), "ids must be contiguous int32");
  expect(tok, at::kBFloat16, "tok");
  expect(pos, at::kBFloat16, "pos");
  TORCH_CHECK(tok.is_contiguous() && pos.is_contiguous() && tok.size(1) == pos.size(1), "embedding tables");
  if (positions.has_value()) {
    TORCH_CHECK(positions->scalar_type() == at::kInt && positions->is_contiguous() &&
                    positions->numel() == ids.numel(),
                "positions must be int32 like ids");
  }
  const int64_t M = ids.numel(), D = tok.size(1);
  auto out = torch::empty({M, D}, tok.options());
  check(pra_embed_add(ptr<const int>(ids), optr<int>(positions), (int)period, ptr<const __nv_bfloat16>(tok),
                      ptr<const __nv_bfloat16>(pos), M, D, ptr<__nv_bfloat16>(out), stream()),
        "embed_add");
  return out;
}

// ---------------------------------------------------------------- peer buffers (CUDA IPC)
// A dedicated cudaMalloc allocation (zeroed) that other processes on the node can map;
// plain peer loads and stores only (no multicast object is ever created).
py::tuple ipc_alloc(int64_t nbytes, int64_t device) {
  c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  void* p = nullptr;
  check(cudaMalloc(&p, (size_t)nbytes), "ipc_alloc (cudaMalloc)");
  check(cudaMemset(p, 0, (size_t)nbytes), "ipc_alloc (cudaMemset)");
  cudaIpcMemHandle_t h;
  check(cudaIpcGetMemHandle(&h, p), "ipc_alloc (cudaIpcGetMemHandle)");
  auto t = torch::from_blob(p, {nbytes}, [](void* q) { cudaFree(q); },
                            torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, device));
  return py::make_tuple(t, py::bytes(reinterpret_cast<const char*>(&h), sizeof(h)));
}

int64_t ipc_open(py::bytes handle, int64_t device) {
  c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  const std::string raw = handle;
  TORCH_CHECK(raw.size() == sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, raw.data(), sizeof(h));
  void* p = nullptr;
  check(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "ipc_open");
  return reinterpret_cast<int64_t>(p);
}

void ipc_close(int64_t address, int64_t device) {
  c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  check(cudaIpcCloseMemHandle(reinterpret_cast<void*>(address)), "ipc_close");
}

// ---------------------------------------------------------------- data-parallel reduction
// src/dst/sig: device addresses (ints) of every rank's gradient, output and signal buffers.
// dst empty: the bf16 result goes back into every rank's src buffer (in place).
void dp_allreduce(std::vector<int64_t> src, std::vector<int64_t> dst, std::vector<int64_t> sig, int64_t rank,
                  int64_t offset, int64_t count, double scale, int64_t epoch, int64_t max_spins,
                  torch::Tensor error, int64_t blocks) {
  const int world = src.size();
  const bool in_place = dst.empty();
  TORCH_CHECK(world >= 1 && world <= DP_MAX_RANKS && (in_place || dst.size() == src.size()) && sig.size() == src.size(),
              "dp_allreduce needs one src/dst/sig address per rank (at most ", DP_MAX_RANKS, ")");
  TORCH_CHECK(error.scalar_type() == at::kInt && error.is_cuda(), "error must be an int32 CUDA tensor");
  c10::cuda::CUDAGuard guard(error.device());
  DpArgs a{};
  for (int p = 0; p < world; ++p) {
    a.src[p] = reinterpret_cast<const __nv_bfloat16*>(src[p]);
    a.dst[p] = in_place ? nullptr : reinterpret_cast<float*>(dst[p]);
    a.sig[p] = reinterpret_cast<uint32_t*>(sig[p]);
  }
  a.rank = rank;
  a.world = world;
  a.offset = offset;
  a.count = count;
  a.scale = (float)scale;
  a.epoch = (uint32_t)epoch;
  a.max_spins = max_spins;
  a.error = ptr<int>(error);
  a.blocks = (int)blocks;
  a.in_place_bf16 = in_place ? 1 : 0;
  check(pra_dp_allreduce(a, stream()), "dp_allreduce");
}

int64_t dp_signal_words(int64_t world) { return 2LL * pra_dp_allreduce_blocks() * world; }

// One NVTX range per layer of the block-stack executors ("pra.layer 3 fwd"): a profiler's
// timeline shows which layer each kernel belongs to.  Without an attached tool NVTX calls are
// no-op stubs.
struct LayerRange {
  LayerRange(int64_t layer, const char* what) {
    char name[48];
    std::snprintf(name, sizeof name, "pra.layer %lld %s", (long long)layer, what);
    nvtxRangePushA(name);
  }
  ~LayerRange() { nvtxRangePop(); }
  LayerRange(const LayerRange&) = delete;
  LayerRange& operator=(const LayerRange&) = delete;
};


// ---------------------------------------------------------------- native block-stack executor
// Forward of a stack of pre-LN GPT blocks (LN -> QKV -> [route] -> attention -> O-proj + residual ->
// LN -> up-GELU -> down + residual) driven entirely from C++: no Python, no autograd records,
// one stream.  Used by the cache build (every layer's QKV lands in the K/V pool) and by
// no-grad forwards.  weights holds 12 tensors per layer: ln1 w/b, qkv w/b, o w/b, ln2 w/b,
// up w/b, down w/b (bf16).  ns (empty = no memory) holds the routing namespace: row_pos_off,
// row_ref_off, ref_pos_off, pos_chunk, pos_ref, pos_rank, chunk_start, chunk_len,
// chunk_pool_row; route_cfg = {k_ref, k_chunk, gist_agg, ref_agg, threshold, budget,
// gist_only, full_reference, deduplicate, max_sel, max_mem}.
// pool (optional) receives every layer's QKV rows; mem_pool is the [L, rows, 3D] pool the
// routed memory keys are read from.  after_qkv (a callable or None) runs after every layer's QKV
// GEMM with the layer index: the cache build computes that layer's gists of every chunk there,
// so one layer-synchronous pass serves chunks that route over each other's memory.
// Returns {x, then per routed layer: mem_idx, ints, sel_i, sel_f}.
std::vector<torch::Tensor> stack_forward(torch::Tensor x, int64_t B, int64_t T, std::vector<torch::Tensor> weights,
                                         int64_t heads, int64_t head_dim, double eps,
                                         c10::optional<torch::Tensor> key_valid, c10::optional<torch::Tensor> pool,
                                         int64_t pool_row0, bool stop_after_kv, c10::optional<torch::Tensor> mem_pool,
                                         std::vector<torch::Tensor> ns,
                                         c10::optional<torch::Tensor> gists, c10::optional<torch::Tensor> gist_count,
                                         c10::optional<torch::Tensor> gist_kv, c10::optional<torch::Tensor> budget_rows,
                                         c10::optional<torch::Tensor> query_rows, std::vector<double> route_cfg,
                                         pybind11::object after_qkv) {
  c10::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(weights.size() % 12 == 0, "stack_forward needs 12 weight tensors per layer");
  const bool hooked = !after_qkv.is_none();
  const int64_t L = weights.size() / 12;
  const int64_t D = heads * head_dim;
  const int64_t M = B * T;
  TORCH_CHECK(x.dim() == 2 && x.size(0) == M && x.size(1) == D && x.is_contiguous(), "x must be [B*T, D]");
  const bool routed = !ns.empty();
  if (routed) {
    TORCH_CHECK(ns.size() == 9 && gists.has_value() && gist_count.has_value() && route_cfg.size() >= 11,
                "routing needs 9 namespace tensors, gists, gist_count and 11 settings");
    TORCH_CHECK(mem_pool.has_value() || gist_kv.has_value(), "routing needs the memory K/V pool");
  }
  const bool gist_only = routed && route_cfg[6] != 0.0;
  const double scale = 1.0 / std::sqrt((double)head_dim);
  std::vector<torch::Tensor> out{x};
  for (int64_t l = 0; l < L; ++l) {
    LayerRange range(l, "fwd");
    const torch::Tensor* w = weights.data() + 12 * l;
    auto h = norm_fwd(x, w[0], w[1], eps, false)[0];
    torch::Tensor qkv = pool.has_value() ? pool->select(0, l).narrow(0, pool_row0, M)
                                         : torch::empty({M, 3 * D}, x.options());
    gemm("tn", h, w[2], c10::nullopt, qkv, w[3], c10::nullopt, 1.0, 0.0, c10::nullopt);
    if (hooked) after_qkv(l);  // e.g. this layer's gists of every chunk, before any routing reads them
    if (stop_after_kv && l == L - 1) break;
    auto qkv3 = qkv.view({B, T, 3 * D});
    c10::optional<torch::Tensor> mk, mv, mi, ml;
    if (routed) {
      auto r = route(qkv3.narrow(2, 0, D), gists->select(0, l), gist_count->select(0, l), ns[0], ns[1], ns[2], ns[3],
                     ns[4], ns[5], ns[6], ns[7], ns[8], (int64_t)route_cfg[0], (int64_t)route_cfg[1],
                     (int64_t)route_cfg[2], (int64_t)route_cfg[3], route_cfg[4], (int64_t)route_cfg[5], gist_only,
                     route_cfg[7] != 0.0, route_cfg[8] != 0.0, (int64_t)route_cfg[9], (int64_t)route_cfg[10],
                     budget_rows, query_rows.has_value() ? query_rows : c10::optional<torch::Tensor>(
                                                               torch::full({B}, (int)(T - 1), x.options().dtype(at::kInt))),
                     route_cfg.size() > 11 && route_cfg[11] != 0.0);
      if (gist_only) {
        mk = gist_kv->select(0, 0).select(0, l);
        mv = gist_kv->select(0, 1).select(0, l);
      } else {
        auto layer_pool = mem_pool->select(0, l);
        mk = layer_pool.narrow(1, D, D);
        mv = layer_pool.narrow(1, 2 * D, D);
      }
      mi = r[0];
      ml = r[1].select(0, 0);
      out.insert(out.end(), r.begin(), r.end());
    }
    auto a = attention_fwd(qkv3.narrow(2, 0, D), qkv3.narrow(2, D, D), qkv3.narrow(2, 2 * D, D), heads, heads,
                           head_dim, mk, mv, mi, ml, key_valid, scale)[0];
    auto x1 = torch::empty_like(x);
    gemm("tn", a.view({M, D}), w[4], x, x1, w[5], c10::nullopt, 1.0, 1.0, c10::nullopt);
    auto h2 = norm_fwd(x1, w[6], w[7], eps, false)[0];
    const int64_t F = w[8].size(0);
    auto z = torch::empty({M, F}, x.options()), u = torch::empty({M, F}, x.options());
    gemm("tn_gelu", h2, w[8], c10::nullopt, u, w[9], z, 1.0, 0.0, c10::nullopt);
    auto x2 = torch::empty_like(x);
    gemm("tn", u, w[10], x1, x2, w[11], c10::nullopt, 1.0, 1.0, c10::nullopt);
    x = x2;
  }
  out[0] = x;
  return out;
}

// ---------------------------------------------------------------- block stack with gradients
// The same per-layer math as stack_forward (pre-norm blocks: LN -> QKV -> [route] -> attention
// -> O + residual -> LN -> GELU MLP + residual), keeping what the backward needs, so one
// autograd node covers the whole stack instead of six per layer.
constexpr int kSavedPerLayer = 15;  // x, mean1, rstd1, h, qkv, a, lse, x1, mean2, rstd2, h2, z, u, mem_idx, mem_len

// Returns {x_out, [4 routing tensors per layer when routed], kSavedPerLayer tensors per layer}.
std::vector<torch::Tensor> stack_train_forward(torch::Tensor x, int64_t B, int64_t T, std::vector<torch::Tensor> weights,
                                               int64_t heads, int64_t head_dim, double eps,
                                               c10::optional<torch::Tensor> key_valid,
                                               c10::optional<torch::Tensor> mem_pool, std::vector<torch::Tensor> ns,
                                               c10::optional<torch::Tensor> gists,
                                               c10::optional<torch::Tensor> gist_count,
                                               c10::optional<torch::Tensor> gist_kv,
                                               c10::optional<torch::Tensor> budget_rows,
                                               c10::optional<torch::Tensor> query_rows, std::vector<double> route_cfg) {
  c10::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(weights.size() % 12 == 0, "stack_train_forward needs 12 weight tensors per layer");
  const int64_t L = weights.size() / 12;
  const int64_t D = heads * head_dim;
  const int64_t M = B * T;
  TORCH_CHECK(x.dim() == 2 && x.size(0) == M && x.size(1) == D && x.is_contiguous(), "x must be [B*T, D]");
  const bool routed = !ns.empty();
  if (routed) {
    TORCH_CHECK(ns.size() == 9 && gists.has_value() && gist_count.has_value() && route_cfg.size() >= 11,
                "routing needs 9 namespace tensors, gists, gist_count and 11 settings");
    TORCH_CHECK(mem_pool.has_value() || gist_kv.has_value(), "routing needs the memory K/V pool");
  }
  const bool gist_only = routed && route_cfg[6] != 0.0;
  const double scale = 1.0 / std::sqrt((double)head_dim);
  auto none = torch::empty({0}, x.options().dtype(at::kInt));
  auto last_rows = query_rows.has_value()
                       ? *query_rows
                       : torch::full({B}, (int)(T - 1), x.options().dtype(at::kInt));
  std::vector<torch::Tensor> routing, saved;
  saved.reserve(L * kSavedPerLayer);
  for (int64_t l = 0; l < L; ++l) {
    LayerRange range(l, "train fwd");
    const torch::Tensor* w = weights.data() + 12 * l;
    auto n1 = norm_fwd(x, w[0], w[1], eps, false);
    auto qkv = torch::empty({M, 3 * D}, x.options());
    gemm("tn", n1[0], w[2], c10::nullopt, qkv, w[3], c10::nullopt, 1.0, 0.0, c10::nullopt);
    auto qkv3 = qkv.view({B, T, 3 * D});
    c10::optional<torch::Tensor> mk, mv, mi, ml;
    torch::Tensor mi_s = none, ml_s = none;
    if (routed) {
      auto r = route(qkv3.narrow(2, 0, D), gists->select(0, l), gist_count->select(0, l), ns[0], ns[1], ns[2], ns[3],
                     ns[4], ns[5], ns[6], ns[7], ns[8], (int64_t)route_cfg[0], (int64_t)route_cfg[1],
                     (int64_t)route_cfg[2], (int64_t)route_cfg[3], route_cfg[4], (int64_t)route_cfg[5], gist_only,
                     route_cfg[7] != 0.0, route_cfg[8] != 0.0, (int64_t)route_cfg[9], (int64_t)route_cfg[10],
                     budget_rows, last_rows, route_cfg.size() > 11 && route_cfg[11] != 0.0);
      if (gist_only) {
        mk = gist_kv->select(0, 0).select(0, l);
        mv = gist_kv->select(0, 1).select(0, l);
      } else {
        auto layer_pool = mem_pool->select(0, l);
        mk = layer_pool.narrow(1, D, D);
        mv = layer_pool.narrow(1, 2 * D, D);
      }
      mi = r[0];
      ml = r[1].select(0, 0);
      mi_s = r[0];
      ml_s = r[1].select(0, 0);
      routing.insert(routing.end(), r.begin(), r.end());
    }
    auto att = attention_fwd(qkv3.narrow(2, 0, D), qkv3.narrow(2, D, D), qkv3.narrow(2, 2 * D, D), heads, heads,
                             head_dim, mk, mv, mi, ml, key_valid, scale);
    auto a = att[0];
    auto x1 = torch::empty_like(x);
    gemm("tn", a.view({M, D}), w[4], x, x1, w[5], c10::nullopt, 1.0, 1.0, c10::nullopt);
    auto n2 = norm_fwd(x1, w[6], w[7], eps, false);
    const int64_t F = w[8].size(0);
    auto z = torch::empty({M, F}, x.options()), u = torch::empty({M, F}, x.options());
    gemm("tn_gelu", n2[0], w[8], c10::nullopt, u, w[9], z, 1.0, 0.0, c10::nullopt);
    auto x2 = torch::empty_like(x);
    gemm("tn", u, w[10], x1, x2, w[11], c10::nullopt, 1.0, 1.0, c10::nullopt);
    for (auto& t : {x, n1[1], n1[2], n1[0], qkv, a, att[1], x1, n2[1], n2[2], n2[0], z, u, mi_s, ml_s})
      saved.push_back(t);
    x = x2;
  }
  std::vector<torch::Tensor> out{x};
  out.insert(out.end(), routing.begin(), routing.end());
  out.insert(out.end(), saved.begin(), saved.end());
  return out;
}

// g (+)= colsum(dy) into a bias-gradient view (written in place when not accumulating).
static void bias_grad(const torch::Tensor& dy, torch::Tensor& gb, double beta) {
  if (!gb.defined() || gb.numel() == 0) return;
  if (beta == 0.0 && gb.is_contiguous() && gb.scalar_type() == at::kBFloat16 && dy.is_contiguous()) {
    const int N = dy.size(-1);
    const int M = dy.numel() / N;
    auto part = torch::empty({pra_colsum_partials(M), N}, dy.options().dtype(at::kFloat));
    check(pra_colsum(ptr<const __nv_bfloat16>(dy), M, N, ptr<float>(part), ptr<__nv_bfloat16>(gb), stream()),
          "colsum");
    return;
  }
  auto s = colsum(dy);
  if (beta == 0.0) gb.copy_(s);
  else gb.add_(s);
}

// gw (+)= dy^T x, gb (+)= colsum(dy).
static void weight_grad(const torch::Tensor& dy, const torch::Tensor& x, torch::Tensor& gw, torch::Tensor& gb,
                        double beta) {
  if (gw.defined() && gw.numel() > 0)
    gemm("wgrad", dy, x, beta != 0.0 ? c10::optional<torch::Tensor>(gw) : c10::nullopt, gw, c10::nullopt,
         c10::nullopt, 1.0, beta, c10::nullopt);
  bias_grad(dy, gb, beta);
}

// LayerNorm backward with the residual gradient added (dx = LN'(dh) + dres); norm weight and
// bias gradients written (beta = 0) or added (beta = 1) into their views.
static torch::Tensor norm_grad(const torch::Tensor& dh, const torch::Tensor& x, const torch::Tensor& w,
                               const torch::Tensor& mean, const torch::Tensor& rstd, const torch::Tensor& dres,
                               torch::Tensor& gw, torch::Tensor& gb, double beta) {
  const bool direct = beta == 0.0 && gw.defined() && gw.numel() > 0 && gw.is_contiguous() && gb.defined() &&
                      gb.numel() > 0 && gb.is_contiguous() && dh.is_contiguous() && x.is_contiguous() &&
                      dres.is_contiguous();
  if (direct) {  // weight and bias gradients written straight into their views
    const int D = x.size(-1);
    const int M = x.numel() / D;
    auto dx = torch::empty_like(x);
    const int parts = pra_norm_bwd_partials(M);
    auto part = torch::empty({2, parts, D}, x.options().dtype(at::kFloat));
    check(pra_norm_bwd(ptr<const __nv_bfloat16>(dh), ptr<const __nv_bfloat16>(x), ptr<const __nv_bfloat16>(w),
                       ptr<const float>(mean), ptr<const float>(rstd), ptr<const __nv_bfloat16>(dres),
                       ptr<__nv_bfloat16>(dx), ptr<float>(part), ptr<float>(part) + (int64_t)parts * D,
                       ptr<__nv_bfloat16>(gw), ptr<__nv_bfloat16>(gb), M, D, false, stream()),
          "norm_bwd");
    return dx;
  }
  auto r = norm_bwd(dh, x, w, mean, rstd, dres, false);
  if (gw.defined() && gw.numel() > 0) {
    if (beta == 0.0) gw.copy_(r[1]);
    else gw.add_(r[1]);
  }
  if (gb.defined() && gb.numel() > 0) {
    if (beta == 0.0) gb.copy_(r[2]);
    else gb.add_(r[2]);
  }
  return r[0];
}

// Backward of stack_train_forward: dy of the stack output -> dx of its input; weight
// gradients into `grads` (12 per layer, aligned with `weights`; undefined/empty = none).
// The lists may hold a contiguous run of layers starting at stack layer `layer0` (the
// memory pool is indexed by stack layer), so a caller can act between layers.
torch::Tensor stack_train_backward(torch::Tensor dy, int64_t B, int64_t T, std::vector<torch::Tensor> weights,
                                   std::vector<torch::Tensor> grads, double beta, int64_t heads, int64_t head_dim,
                                   c10::optional<torch::Tensor> key_valid, std::vector<torch::Tensor> saved,
                                   c10::optional<torch::Tensor> mem_pool, c10::optional<torch::Tensor> gist_kv,
                                   bool gist_only, int64_t layer0) {
  c10::cuda::CUDAGuard guard(dy.device());
  const int64_t L = weights.size() / 12;
  TORCH_CHECK(grads.size() == weights.size() && (int64_t)saved.size() == L * kSavedPerLayer,
              "stack_train_backward: grads / saved tensors do not match the stack");
  const int64_t D = heads * head_dim;
  const int64_t M = B * T;
  const double scale = 1.0 / std::sqrt((double)head_dim);
  dy = dy.contiguous();
  for (int64_t l = L - 1; l >= 0; --l) {
    LayerRange range(l, "bwd");
    const torch::Tensor* w = weights.data() + 12 * l;
    torch::Tensor* g = grads.data() + 12 * l;
    const torch::Tensor* s = saved.data() + kSavedPerLayer * l;
    const auto &x = s[0], &mean1 = s[1], &rstd1 = s[2], &h = s[3], &qkv = s[4], &a = s[5], &lse = s[6], &x1 = s[7],
               &mean2 = s[8], &rstd2 = s[9], &h2 = s[10], &z = s[11], &u = s[12], &mi = s[13], &ml = s[14];
    // MLP: y = x1 + gelu(h2 W1^T + b1) W2^T + b2
    auto dz = torch::empty_like(z);
    gemm("nn_dgelu", dy, w[10], c10::nullopt, dz, c10::nullopt, z, 1.0, 0.0, c10::nullopt);
    weight_grad(dy, u, g[10], g[11], beta);
    auto dh2 = torch::empty_like(h2);
    gemm("nn", dz, w[8], c10::nullopt, dh2, c10::nullopt, c10::nullopt, 1.0, 0.0, c10::nullopt);
    weight_grad(dz, h2, g[8], g[9], beta);
    auto dx1 = norm_grad(dh2, x1, w[6], mean2, rstd2, dy, g[6], g[7], beta);
    // O projection: x1 = x + a W_o^T + b_o
    auto da = torch::empty({M, D}, dy.options());
    gemm("nn", dx1, w[4], c10::nullopt, da, c10::nullopt, c10::nullopt, 1.0, 0.0, c10::nullopt);
    weight_grad(dx1, a.view({M, D}), g[4], g[5], beta);
    // attention
    auto qkv3 = qkv.view({B, T, 3 * D});
    c10::optional<torch::Tensor> mk, mv, mio, mlo;
    if (mi.numel() > 0) {
      if (gist_only) {
        mk = gist_kv->select(0, 0).select(0, layer0 + l);
        mv = gist_kv->select(0, 1).select(0, layer0 + l);
      } else {
        auto layer_pool = mem_pool->select(0, layer0 + l);
        mk = layer_pool.narrow(1, D, D);
        mv = layer_pool.narrow(1, 2 * D, D);
      }
      mio = mi;
      mlo = ml;
    }
    auto dqkv = attention_bwd(da.view({B, T, D}), qkv3.narrow(2, 0, D), qkv3.narrow(2, D, D),
                              qkv3.narrow(2, 2 * D, D), a, lse, heads, head_dim, mk, mv, mio, mlo, key_valid,
                              scale)[0].view({M, 3 * D});
    auto dh = torch::empty_like(h);
    gemm("nn", dqkv, w[2], c10::nullopt, dh, c10::nullopt, c10::nullopt, 1.0, 0.0, c10::nullopt);
    weight_grad(dqkv, h, g[2], g[3], beta);
    dy = norm_grad(dh, x, w[0], mean1, rstd1, dx1, g[0], g[1], beta);
  }
  return dy;
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "PRA sm_100a kernels";
  m.def("attention_fwd", &attention_fwd, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("heads"),
        py::arg("kv_heads"), py::arg("head_dim"), py::arg("mem_k"), py::arg("mem_v"), py::arg("mem_idx"),
        py::arg("mem_len"), py::arg("key_valid"), py::arg("scale"), py::arg("drop_p") = 0.0,
        py::arg("drop_seed") = 0, py::arg("drop_offset") = 0);
  m.def("dropout", &dropout);
  m.def("dropout_add", &dropout_add);
  m.def("attention_status", [](int64_t device) { return attention_status_buffer(torch::Device(torch::kCUDA, device)); });
  m.def("set_attention_impl", [](const std::string& impl) {
    TORCH_CHECK(impl == "tcgen05" || impl == "mma", "attention impl must be 'tcgen05' or 'mma'");
    pra_attention_set_impl(impl == "tcgen05" ? 1 : 0);
  });
  m.def("attention_impl", []() { return std::string(pra_attention_get_impl() ? "tcgen05" : "mma"); });
  m.def("attention_bwd", &attention_bwd, py::arg("dout"), py::arg("q"), py::arg("k"), py::arg("v"),
        py::arg("out"), py::arg("lse"), py::arg("heads"), py::arg("head_dim"), py::arg("mem_k"), py::arg("mem_v"),
        py::arg("mem_idx"), py::arg("mem_len"), py::arg("key_valid"), py::arg("scale"), py::arg("drop_p") = 0.0,
        py::arg("drop_seed") = 0, py::arg("drop_offset") = 0);
  m.def("gemm", &gemm);
  m.def("norm_fwd", &norm_fwd);
  m.def("norm_bwd", &norm_bwd);
  m.def("colsum", &colsum);
  m.def("cross_entropy", &cross_entropy);
  m.def("grad_norm", &grad_norm);
  m.def("adamw", &adamw);
  m.def("gist_mean", &gist_mean);
  m.def("gist_kmeans", &gist_kmeans);
  m.def("gist_mean_into", &gist_mean_into);
  m.def("gist_kmeans_into", &gist_kmeans_into);
  m.def("route", &route, py::arg("query"), py::arg("gists"), py::arg("gist_count"), py::arg("row_pos_off"),
        py::arg("row_ref_off"), py::arg("ref_pos_off"), py::arg("pos_chunk"), py::arg("pos_ref"), py::arg("pos_rank"),
        py::arg("chunk_start"), py::arg("chunk_len"), py::arg("chunk_pool_row"), py::arg("k_ref"), py::arg("k_chunk"),
        py::arg("gist_agg"), py::arg("ref_agg"), py::arg("threshold"), py::arg("budget"), py::arg("gist_only"),
        py::arg("full_reference"), py::arg("deduplicate"), py::arg("max_sel"), py::arg("max_mem"),
        py::arg("budget_rows"), py::arg("query_rows"), py::arg("global_chunks") = false);
  m.def("stack_forward", &stack_forward);
  m.def("stack_train_forward", &stack_train_forward);
  m.def("stack_train_backward", &stack_train_backward);
  m.def("dp_allreduce", &dp_allreduce);
  m.def("rope_copy", &rope_copy);
  m.def("tp_allreduce", &tp_allreduce);
  m.def("tp_allgather", &tp_allgather);
  m.def("tp_signal_words", [](int64_t world) { return (int64_t)TP_MAX_BLOCKS * world; });
  m.def("silu_mul", &silu_mul, py::arg("gate_up"), py::arg("out"), py::arg("block") = 0);
  m.def("decode_prologue", &decode_prologue, py::arg("ids"), py::arg("cache_len"), py::arg("pos_offset"),
        py::arg("embed"), py::arg("max_len"), py::arg("ss_out") = py::none());
  m.def("decode_attention", &decode_attention, py::arg("q"), py::arg("heads"), py::arg("kv_heads"),
        py::arg("head_dim"), py::arg("mem_k"), py::arg("mem_v"), py::arg("mem_idx"), py::arg("mem_len"),
        py::arg("loc_k"), py::arg("loc_v"), py::arg("loc_len"), py::arg("max_keys"), py::arg("split_keys"),
        py::arg("export_partials"), py::arg("mem_splits") = 0, py::arg("mem_split_keys") = 0, py::arg("split_lo") = 0, py::arg("split_count") = 0,
        py::arg("phase") = 0, py::arg("part_o") = py::none(), py::arg("part_ml") = py::none(),
        py::arg("max_ctas") = 0);
  m.def("route_topk", &route_topk, py::arg("scores"), py::arg("query"), py::arg("gists"), py::arg("ns_start"),
        py::arg("ns_end"), py::arg("chunk_len"), py::arg("chunk_row0"), py::arg("k"), py::arg("k_cand"),
        py::arg("budget"), py::arg("mem_max"), py::arg("local"), py::arg("id_offset"), py::arg("gists_per_chunk"),
        py::arg("segments"), py::arg("pool_rows") = -1, py::arg("page_table") = py::none(),
        py::arg("trace") = py::none());
  m.def("route_merge", &route_merge, py::arg("cands"), py::arg("world"), py::arg("k"), py::arg("budget"),
        py::arg("chunk_len"), py::arg("chunk_row0"), py::arg("mem_max"), py::arg("local"),
        py::arg("pool_rows") = -1);
  m.def("route_topk_exchange", &route_topk_exchange);
  m.def("set_bounds_check", &set_bounds_check);
  m.def("decode_set_tma", [](bool on) { pra_decode_set_tma(on ? 1 : 0); });
  m.def("set_pdl", [](bool on) { pra_set_pdl(on ? 1 : 0); });
  m.def("gelu_probe", &gelu_probe);
  m.def("set_launch_priority", [](bool high) { pra_set_launch_priority(high ? 1 : 0); });
  m.def("pdl_enabled", []() { return pra_pdl_enabled() != 0; });
  m.def("decode_gemm_configure", [](int64_t ctas, int64_t min_kb, int64_t max_splits) {
    pra_decode_gemm_configure((int)ctas, (int)min_kb, (int)max_splits);
  }, py::arg("ctas"), py::arg("min_kb"), py::arg("max_splits") = 0);
  m.def("decode_set_stages", [](int64_t stages) { pra_decode_set_stages((int)stages); });
  m.def("bounds_check_enabled", &bounds_check_enabled);
  m.def("bounds_status", &bounds_status);
  m.def("bounds_reset", &bounds_reset);
  m.def("embed_add", &embed_add);
  m.def("combine_partials", &combine_partials);
  m.def("decode_gemm", &decode_gemm, py::arg("x"), py::arg("w"), py::arg("bias"), py::arg("residual"), py::arg("out"),
        py::arg("out2"), py::arg("split_col"), py::arg("splits"), py::arg("recv"), py::arg("flags"), py::arg("rank"),
        py::arg("epochs"), py::arg("max_spins"), py::arg("error"), py::arg("swiglu") = false,
        py::arg("ss_out") = py::none(), py::arg("ss_in") = py::none(), py::arg("ss_tiles") = 0, py::arg("ss_dim") = 0,
        py::arg("ss_eps") = 0.0);
  m.def("decode_qkv_rope", &decode_qkv_rope, py::arg("x"), py::arg("w"), py::arg("bias"), py::arg("q_out"),
        py::arg("k_cache"), py::arg("v_cache"), py::arg("cache_rows"), py::arg("pos"), py::arg("cos_t"),
        py::arg("sin_t"), py::arg("head_dim"), py::arg("q_end"), py::arg("k_end"), py::arg("v_end"),
        py::arg("route_out"), py::arg("ss_in") = py::none(), py::arg("ss_tiles") = 0, py::arg("ss_dim") = 0,
        py::arg("ss_eps") = 0.0);
  m.def("decode_gemm_max_tiles", []() { return (int64_t)DG_MAX_TILES; });
  m.def("decode_gemm_flag_slots", []() { return (int64_t)DG_MAX_TILES * DG_MAX_SPLITS; });
  m.def("decode_gemm_resident_clusters", [](int64_t splits) { return (int64_t)pra_decode_gemm_resident_clusters((int)splits); });
  m.def("plan_batch", &pra_plan_batch, "native cache-build planner (returns None when a batch needs the Python planner)");
  m.def("ipc_alloc", &ipc_alloc);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close", &ipc_close);
  m.def("dp_signal_words", &dp_signal_words);
}
