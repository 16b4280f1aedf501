// Host-visible parameter blocks and launch entry points of the PRA kernels.
// Pure C++ (no torch): shared by the .cu kernel files and the binding layer.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

// ---- ragged native-K/V attention (attention.cu) ---------------------------------
struct AttnParams {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  __nv_bfloat16* o;
  float* lse;                  // [B, H, T] natural-log LSE of the scaled scores
  const __nv_bfloat16* mem_k;  // pool rows [tokens, Hkv * D]
  const __nv_bfloat16* mem_v;
  const int* mem_idx;          // [B, mem_max] pool row of each memory key
  const int* mem_len;          // [B]
  const uint8_t* key_valid;    // [B, T] or nullptr
  int64_t q_row, q_batch, k_row, k_batch, v_row, v_batch, o_row, o_batch, mem_row;
  int B, T, H, Hkv, mem_max;
  float scale;
  const __nv_bfloat16* dout;
  int64_t do_row, do_batch;
  float* delta;                // [B, H, T] workspace
  __nv_bfloat16* dq;
  __nv_bfloat16* dk;
  __nv_bfloat16* dv;
  int64_t dq_row, dq_batch, dk_row, dk_batch, dv_row, dv_batch;
  int* status;                 // optional: set to 1 by a kernel that gave up on a bounded wait
  // Dropout on the attention probabilities (local keys only, no memory): element (b, h, q, t)
  // is kept when its Philox word passes drop_thresh (see pra_dropout); kept values are scaled
  // by drop_scale.  drop_thresh == 0: no dropout.
  uint32_t drop_thresh;
  float drop_scale;
  uint64_t drop_seed, drop_offset;
};

cudaError_t pra_attention_fwd(const AttnParams& p, int head_dim, cudaStream_t stream);

// ---- dropout (dropout.cu) --------------------------------------------------------------
// Counter-based dropout: element e of the stream (seed, offset) draws word e % 4 of the
// Philox4x32-10 block (e / 4, offset) under key seed; it is kept when (word >> 8) >= thresh
// (thresh = round(p * 2^24)) and then scaled by 1 / (1 - p).  The backward regenerates the
// same mask from (seed, offset), so nothing is stored.
uint32_t pra_dropout_threshold(double p);
// y = keep ? x * scale : 0 (y may alias x).
cudaError_t pra_dropout(const __nv_bfloat16* x, __nv_bfloat16* y, int64_t n, uint32_t thresh, float scale,
                        uint64_t seed, uint64_t offset, cudaStream_t stream);
// y = res + (keep ? x * scale : 0) (y may alias res or x).
cudaError_t pra_dropout_add(const __nv_bfloat16* res, const __nv_bfloat16* x, __nv_bfloat16* y, int64_t n,
                            uint32_t thresh, float scale, uint64_t seed, uint64_t offset, cudaStream_t stream);
// tcgen05 forward (head dims 64/128, 16-byte aligned rows); cudaErrorNotSupported otherwise.
cudaError_t pra_attention_fwd_tc(const AttnParams& p, int head_dim, cudaStream_t stream);
// dQ of the backward on tcgen05 (head dim 64); cudaErrorNotSupported otherwise.
cudaError_t pra_attention_bwd_dq_tc(const AttnParams& p, int head_dim, cudaStream_t stream);
// dK / dV of the local keys on tcgen05 (head dim 64, MHA); cudaErrorNotSupported otherwise.
cudaError_t pra_attention_bwd_dkdv_tc(const AttnParams& p, int head_dim, cudaStream_t stream);
// Forward implementation: 1 = tcgen05 where supported (default), 0 = mma.sync everywhere.
void pra_attention_set_impl(int tcgen05);
int pra_attention_get_impl();
cudaError_t pra_attention_bwd(const AttnParams& p, int head_dim, cudaStream_t stream);

// ---- GEMMs (gemm/*.cu, CUTLASS sm100 collectives) -------------------------------
struct GemmArgs {
  const void* A;
  const void* B;
  const void* C;      // beta * C source (may be null when beta == 0)
  void* D;
  const void* bias;   // per-column bias [N] (tn variants) or null
  void* aux;          // pre-activation output (gelu fwd) / input (gelu bwd)
  int M, N, K;
  float alpha, beta;
  const float* alpha_ptr;  // device scalar overriding alpha when non-null
  void* workspace;
  size_t workspace_bytes;
};
cudaError_t pra_gemm_tn_bias(const GemmArgs& g, cudaStream_t stream);
cudaError_t pra_gemm_tn_f32(const GemmArgs& g, cudaStream_t stream);  // fp32 D, no bias / C
cudaError_t pra_gemm_tn_bias_small(const GemmArgs& g, cudaStream_t stream);  // M <= 128, stream-K
cudaError_t pra_gemm_tn_bias_narrow(const GemmArgs& g, cudaStream_t stream);  // N <= 1024, 128x128 tiles
// The GELU / GELU-derivative of the GEMM epilogues on fp32 values (numerics probe).
cudaError_t pra_gelu_probe(const float* z, float* y, float* dy, int64_t n, cudaStream_t stream);
cudaError_t pra_gemm_tn_bias_gelu(const GemmArgs& g, cudaStream_t stream);
cudaError_t pra_gemm_nn(const GemmArgs& g, cudaStream_t stream);
// Stream-K variants (128 x 256 tiles) for long reductions into few output tiles.
cudaError_t pra_gemm_nn_sk(const GemmArgs& g, cudaStream_t stream);
cudaError_t pra_gemm_wgrad_sk(const GemmArgs& g, cudaStream_t stream);
// Shape-based choice among the instantiations (gemm/dispatch.cu): what ext.gemm runs.
cudaError_t pra_gemm_tn_auto(const GemmArgs& g, cudaStream_t stream);
cudaError_t pra_gemm_nn_auto(const GemmArgs& g, cudaStream_t stream);
cudaError_t pra_gemm_wgrad_auto(const GemmArgs& g, cudaStream_t stream);
cudaError_t pra_gemm_nn_dgelu(const GemmArgs& g, cudaStream_t stream);
cudaError_t pra_gemm_wgrad(const GemmArgs& g, cudaStream_t stream);

// ---- norms (norm.cu) --------------------------------------------------------------
cudaError_t pra_norm_fwd(const __nv_bfloat16* x, const __nv_bfloat16* w, const __nv_bfloat16* b, __nv_bfloat16* y,
                         float* mean, float* rstd, int M, int D, float eps, bool rms, cudaStream_t stream);
int pra_norm_bwd_partials(int M);
cudaError_t pra_norm_bwd(const __nv_bfloat16* dy, const __nv_bfloat16* x, const __nv_bfloat16* w, const float* mean,
                         const float* rstd, const __nv_bfloat16* dres, __nv_bfloat16* dx, float* dw_part,
                         float* db_part, __nv_bfloat16* dw, __nv_bfloat16* db, int M, int D, bool rms,
                         cudaStream_t stream);
int pra_colsum_partials(int M);
cudaError_t pra_colsum(const __nv_bfloat16* g, int M, int N, float* part, __nv_bfloat16* out, cudaStream_t stream);

// ---- allocation-free column sums (colsum_noalloc.cu) ---------------------------------
// Exported C symbols for callers that cannot allocate device memory where they call
// (the contract, capacity and sharing rules are in colsum_noalloc.cu).  Return values
// are cudaError_t codes.
extern "C" {
__attribute__((visibility("default"))) long long pra_colsum_noalloc_capacity();
__attribute__((visibility("default"))) void pra_colsum_noalloc_reset();
__attribute__((visibility("default"))) int pra_colsum_noalloc(const void* g, int M, int N, void* out,
                                                              cudaStream_t stream);
}

// ---- loss / optimizer (loss_optim.cu) -----------------------------------------------
cudaError_t pra_cross_entropy(__nv_bfloat16* logits, int64_t M, int64_t ld, int V, const int64_t* labels,
                              int ignore_index, float* row_loss, float* row_valid, cudaStream_t stream);
int pra_grad_norm_parts();
cudaError_t pra_grad_norm(const void* grad, bool grad_bf16, int64_t n, float max_norm, float* part, float* norm_out,
                          float* coef_out, cudaStream_t stream);
cudaError_t pra_adamw(float* param, __nv_bfloat16* shadow, const void* grad, bool grad_bf16, float* m, float* v,
                      int64_t n, float lr, float beta1, float beta2, float eps, float weight_decay, int step,
                      const float* coef, float grad_scale, cudaStream_t stream);
cudaError_t pra_cast_f32_bf16(const float* src, __nv_bfloat16* dst, int64_t n, cudaStream_t stream);

// ---- gists (gist.cu) ------------------------------------------------------------------
// One CTA per (chunk, layer).  Inputs: layer l's K/V rows at pk/pv + l * layer_stride
// (bf16, row stride row_stride); chunk c owns rows [start[c], start[c] + len[c]).
// Outputs land at chunk slot dest[c] (identity when null) of [L, S, G, D] fp32 tables
// (out_layer_stride = S * G * D) and of count [L, S] (count_layer_stride = S).
struct GistArgs {
  const __nv_bfloat16* pk;
  const __nv_bfloat16* pv;
  int64_t row_stride, layer_stride;
  const int* start;
  const int* len;
  const int* dest;
  int C, D, G;
  int nmax;                    // max chunk length in the launch (k-means scratch size)
  float* gk;
  float* gv;
  float* gn;
  int64_t out_layer_stride;
  int* count;
  int64_t count_layer_stride;
  // k-means only
  int max_iters;
  float tol;
  bool normalize, kmeanspp, farthest;
  const int* init_first;       // [C] kmeans++ first index, or offset into init_idx for sampled init
  const int* init_idx;         // flat sampled indices
  const float* exp_draws;      // flat Exp(1) draws
  const int* exp_off;          // [C] offset of this chunk's [G-1, len] draws
  int* occupancy;              // [L, C, G] members per occupied slot (nullable)
  int* iterations;             // [L, C] Lloyd iterations run (nullable)
  int* status;                 // [L, C] 0 ok, 1 empty cluster under the error policy, 2 chunk too long (nullable)
};
cudaError_t pra_gist_mean(const GistArgs& args, int layers, cudaStream_t stream);
cudaError_t pra_gist_kmeans(const GistArgs& args, int layers, cudaStream_t stream);

// ---- row-local routing + selection + materialisation plan (routing.cu) ----------------
struct RouteParams {
  int B, D, G;
  const __nv_bfloat16* query;  // row b's query: query + b * query_stride (+ query_row[b] * query_row_stride)
  int64_t query_stride;
  const int* query_row;        // [B] token row of each query inside its sequence, or null
  int64_t query_row_stride;
  const float* gists;          // [C, G, D] L2-normalised
  const int* gist_count;       // [C]
  // Namespace of row b: positions [row_pos_off[b], row_pos_off[b+1]); position q names the
  // global chunk pos_chunk[q], its URI pos_ref[q] (index among the row's URIs, which are
  // sorted by URI string) and its lexical chunk-id rank pos_rank[q] within that URI.
  // URI r (global slot, row_ref_off[b] <= r < row_ref_off[b+1]) owns positions
  // [ref_pos_off[r], ref_pos_off[r+1]).
  const int* row_pos_off;      // [B + 1]
  const int* row_ref_off;      // [B + 1]
  const int* ref_pos_off;      // [R + 1]
  const int* pos_chunk;        // [P]
  const int* pos_ref;          // [P]
  const int* pos_rank;         // [P]
  const int* chunk_start;      // [C] source token start
  const int* chunk_len;        // [C] materialisable tokens
  const int* chunk_pool_row;   // [C] first pool row of the chunk's K/V
  int k_ref, k_chunk, gist_agg, ref_agg;  // aggregations: 0 max, 1 mean, 2 logsumexp
  float threshold;
  int budget;
  const int* budget_rows;      // [B] per-row budgets, or null (scalar budget)
  bool gist_only, full_reference, deduplicate;
  bool global_chunks;          // search_strategy "global_chunks": one global chunk ranking under
                               // the distinct-URI and per-URI limits (else hierarchical)
  int max_sel, max_mem;
  int* mem_idx;                // [B, max_mem]
  int* mem_len;                // [B]
  int* sel_chunk;              // [B, max_sel] retained selections, selection order
  int* sel_ref_rank;
  int* sel_chunk_rank;
  float* sel_ref_score;
  float* sel_chunk_score;
  int* sel_win_index;
  float* sel_win_score;
  int* sel_count;              // [B]
  int* routing_candidates;     // [B]
  int* duplicate_tokens;       // [B]
  int* status;                 // [B] 0 ok, 1 namespace too large, 2 memory list truncated
};
cudaError_t pra_route(const RouteParams& p, cudaStream_t stream);

// ---- data-parallel gradient all-reduce over peer memory (dp_reduce.cu) -----------------
constexpr int DP_MAX_RANKS = 8;
struct DpArgs {
  const __nv_bfloat16* src[DP_MAX_RANKS];  // every rank's bf16 gradient buffer (symmetric memory)
  float* dst[DP_MAX_RANKS];                // every rank's fp32 reduced buffer (symmetric memory)
  uint32_t* sig[DP_MAX_RANKS];             // every rank's signal area: [2][blocks][world] uint32, zeroed once
  int rank, world;
  int64_t offset, count;                   // element range reduced by this launch (multiples of 8)
  float scale;                             // applied to the sum (1/world gives the average)
  uint32_t epoch;                          // strictly increasing per launch (signals compare >=)
  long long max_spins;                     // poll limit of every wait
  int* error;                              // local flag: 1 + phase of a timed-out wait
  int blocks;                              // CTAs of the launch (0: pra_dp_allreduce_blocks()); fewer
                                           // leave SMs to kernels that run concurrently (backward)
  int in_place_bf16;                       // 1: store the bf16 result back into every rank's src buffer
                                           // (dst unused): half the NVLink bytes of fp32 stores
};
int pra_dp_allreduce_blocks();  // 2 CTAs per SM of the current device
cudaError_t pra_dp_allreduce(const DpArgs& args, cudaStream_t stream);

// ---- Llama-family engine (llama.cu) ------------------------------------------------------
struct RopeCopyArgs {
  const __nv_bfloat16* src;    // row m at src + m * src_stride (heads * head_dim values)
  int64_t src_stride;
  __nv_bfloat16* dst;          // row dst_rows[m] (or m) at dst + row * dst_stride; may alias src
  int64_t dst_stride;
  const int* dst_rows;         // [M] or null
  const int* pos;              // [M] rotary positions, or null (plain copy)
  const float* cos_t;          // [max_pos, head_dim / 2] (null: plain copy)
  const float* sin_t;
  int M, heads, head_dim;
};
cudaError_t pra_rope_copy(const RopeCopyArgs& args, cudaStream_t stream);
// act = silu(gate) * up.  block == 0: gate_up rows are [gate (F) | up (F)]; block > 0: they
// alternate in runs of `block` features ([gate block j | up block j] ...), the layout the fused
// decode GEMM epilogue reads.
cudaError_t pra_silu_mul(const __nv_bfloat16* gate_up, int64_t M, int F, int block, __nv_bfloat16* out,
                         cudaStream_t stream);

// Bounds-checked kernel variants (``set_bounds_check(true)``): a checked kernel records the
// first out-of-range index it meets here and skips that access (the key is masked, the row is
// not written); it never traps.  Checks cost a compare per index, so they are opt-in.
struct BoundsStatus {
  int code;         // 0: clean, 1: a violation was recorded
  int kernel;       // which check (PRA_BOUNDS_* below)
  long long index;  // the offending value
  long long limit;  // the bound it broke
};
enum : int {
  PRA_BOUNDS_DECODE_MEM_LEN = 1,   // decode: memory length > the row list's capacity
  PRA_BOUNDS_DECODE_LOC_LEN = 2,   // decode: local length > the cache's capacity
  PRA_BOUNDS_DECODE_MEM_ROW = 3,   // decode: memory row id outside the pool
  PRA_BOUNDS_ROUTE_NAMESPACE = 4,  // routing: namespace range outside the chunk table
  PRA_BOUNDS_ROUTE_POOL_ROW = 5,   // routing: a selected chunk's rows run past the pool
  PRA_BOUNDS_ROUTE_CHUNK = 6,      // routing merge: candidate chunk id outside the chunk table
  PRA_BOUNDS_DECODE_TOKEN = 7,     // decode prologue: token id outside the vocabulary (row 0 read)
};

// Decode step prologue (one launch): token embeddings, rotary positions, cache rows, new lengths.
struct DecodePrologueArgs {
  const int64_t* ids;          // [B] token ids
  const int* cache_len;        // [B]
  const int* pos_offset;       // [B] or null
  const __nv_bfloat16* embed;  // [vocab, d]
  int64_t vocab, d;
  int B, max_len;
  __nv_bfloat16* x;            // [B, d]
  int* pos;                    // [B] cache_len + pos_offset
  int* rows;                   // [B] b * max_len + cache_len
  int* new_len;                // [B] cache_len + 1
  BoundsStatus* bounds;        // non-null: report out-of-vocabulary ids
  float* ss_out;               // [B] or null: sum of squares of each embedding row (first RMSNorm)
};
cudaError_t pra_decode_prologue(const DecodePrologueArgs& a, cudaStream_t stream);

struct DecodeAttnParams {
  const __nv_bfloat16* q;      // [B, H * Dh] post-rotary queries of the decoded tokens
  int64_t q_row;
  int B, H, Hkv;
  const __nv_bfloat16* mem_k;  // memory pool rows (kv head h at column h * Dh)
  const __nv_bfloat16* mem_v;
  int64_t mem_row;
  const int* mem_idx;          // [B, mem_max]
  int mem_max;
  const int* mem_len;          // [B] or null
  const __nv_bfloat16* loc_k;  // local cache: row t of batch b at b * loc_batch + t * loc_row
  const __nv_bfloat16* loc_v;
  int64_t loc_row, loc_batch;
  const int* loc_len;          // [B] or null
  float scale;
  int split_keys, n_split;     // keys per split (multiple of 64), number of splits
  float* part_o;               // [B, H, n_split, Dh] workspace
  float* part_ml;              // [B, H, n_split, 2] workspace
  __nv_bfloat16* out;          // [B, H * Dh] normalised output, or null
  int64_t out_row;
  float* export_o;             // [B, H, Dh] merged unnormalised output, or null
  float* export_ml;            // [B, H, 2] merged (max, sum), or null
  int64_t mem_rows;            // rows of the memory pool (bounds-checked variant, TMA maps)
  int loc_cap;                 // local cache capacity per row (bounds-checked variant, TMA maps)
  BoundsStatus* bounds;        // non-null: run the bounds-checked variant
  int mem_on_device;           // the memory pool is device memory (TMA-fed kernel allowed)
  int* status;                 // optional: set to 1 by a CTA that gave up on a bounded wait
  // Split layout.  mem_splits == 0: the splits tile each row's [memory ; local] key sequence.
  // mem_splits > 0: splits [0, mem_splits) tile the memory keys and splits [mem_splits,
  // n_split) tile the local cache on their own, so the local splits never read mem_len / mem_idx
  // and can run while the routing that produces them is still in flight.
  int mem_splits;
  int mem_split_keys;          // keys per memory split when mem_splits > 0 (0: split_keys; <= split_keys)
  int split_lo, split_count;   // the splits this launch runs (split_count 0: all n_split)
  int phase;                   // 0: attention then merge; 1: attention only; 2: merge only
  int max_ctas;                // > 0: a persistent grid of at most this many CTAs walks the work items
};
cudaError_t pra_decode_attention(const DecodeAttnParams& p, int head_dim, cudaStream_t stream);
// 1 (default): eligible decode attention calls run the TMA-fed kernel; 0: the cp.async kernel.
void pra_decode_set_tma(int on);
// Whether the instrumented decode kernels (decode GEMM, RMSNorm, SwiGLU, routing, decode
// attention and its merge) are launched with programmatic stream serialization (default on).
void pra_set_pdl(int on);
int pra_pdl_enabled();
// Scheduling priority given to the instrumented decode kernels launched from now on (0: none,
// else the device's highest stream priority): the routing chain that overlaps the decode
// attention sets it so its CTAs are dispatched ahead of the attention's pending CTAs, also
// inside a captured graph (the attribute is kept per kernel node).
void pra_set_launch_priority(int high);
int pra_launch_priority();
// Pipeline stages of the TMA-fed decode kernel (2, 3 or 4; 2 by default).
void pra_decode_set_stages(int stages);

struct RouteTopkArgs {
  int B, D;
  int G;                       // gists per chunk: scores / gists hold C * G rows, chunk score = max over G
  const float* scores;         // [B, score_stride] approximate cosine scores (tensor-core GEMM)
  int64_t score_stride;
  const float* query;          // [B, query_stride] routing queries (fp32, unnormalised), or
  const __nv_bfloat16* query_bf16;  // the same in bf16 (set instead of query: read and widened in the kernel)
  int64_t query_stride;
  const float* gists;          // [C, D] L2-normalised fp32 gists (exact rescoring)
  const int* ns_start;         // [B] namespace of row b: chunks [ns_start, ns_end)
  const int* ns_end;
  const int* chunk_len;        // [C]
  const int* chunk_row0;       // [C] memory pool row of the chunk's first token
  int k, k_cand;               // selected chunks (<= 64), approximate candidates (<= 512)
  int budget;                  // token budget per row (< 0: none)
  int* mem_idx;                // [B, mem_max]
  int mem_max;
  int* mem_len;                // [B]
  int* sel_out;                // [B, k] selected chunk ids in chunk order (-1 pad), or null
  float* cand_score;           // local mode: [B * segments, k] best exact scores in rank order (no budget / rows)
  int* cand_id;                // local mode: their chunk ids + id_offset (-1 pad)
  int id_offset;
  int segments, seg_len;       // > 1: each row's chunks are cut into slices of seg_len, one CTA each (local mode)
  int n_chunks;                // chunks in the table (bounds-checked variant)
  int64_t pool_rows;           // rows of the memory pool (bounds-checked variant)
  BoundsStatus* bounds;        // non-null: run the bounds-checked variant
  const int* page_table;       // [B, page_stride] or null: namespace position j of row b is chunk
  int64_t page_stride;         // page_table[b * page_stride + j] (scores / gists / tables by chunk id)
  long long* trace;            // optional [8]: clock64 at the phase boundaries of CTA 0 (profiling)
};
cudaError_t pra_route_topk(const RouteTopkArgs& args, cudaStream_t stream);

// Merge of the per-rank local top-k candidates (chunk-sharded routing across GPUs).
struct RouteMergeArgs {
  int B, world, k;
  const float* cands;          // [B, row_stride]: per rank [k scores | k ids as int bits]
  int64_t row_stride;
  int budget;
  const int* chunk_len;        // [C] (global chunk ids)
  const int* chunk_row0;       // [C]
  int* mem_idx;                // [B, mem_max]
  int mem_max;
  int* mem_len;                // [B]
  int* sel_out;                // [B, k] or null
  float* cand_score;           // local mode: [B, k] merged best candidates instead of rows (or null)
  int* cand_id;
  int n_chunks;                // chunks in the table (bounds-checked variant)
  int64_t pool_rows;           // rows of the memory pool (bounds-checked variant)
  BoundsStatus* bounds;        // non-null: run the bounds-checked variant
};
cudaError_t pra_route_merge(const RouteMergeArgs& args, cudaStream_t stream);
cudaError_t pra_combine_partials(const float* parts, int B, int world, int H, int D, __nv_bfloat16* out,
                                 cudaStream_t stream);

// ---- tensor-parallel collectives over peer memory (tp_comm.cu) -------------------------
constexpr int TP_MAX_RANKS = 8;
constexpr int TP_MAX_BLOCKS = 296;  // signal slots per rank: TP_MAX_BLOCKS * world
// Cross-GPU candidate exchange fused into the routing kernel (chunk-sharded memory, one
// segment per row): each row's local exact top-k goes into every rank's receive buffer over
// NVLink (plain peer stores), a per-row flag carrying the call epoch is raised on every rank,
// and once every rank's candidates of that row have landed (bounded wait) the same CTA merges
// them into the selection and the memory row list.  Receive halves alternate with the call
// parity, so a rank one call ahead never overwrites candidates a peer is still reading.
struct RouteExchangeArgs {
  float* recv[TP_MAX_RANKS];      // every rank's [2][B_max][world][2k] receive buffer
  uint32_t* flags[TP_MAX_RANKS];  // every rank's [B_max][world] flags
  uint32_t* epochs;               // local [B_max] per-row call counters (start at 0)
  int rank, world, B_max;
  const int* global_len;          // [C] every chunk's length (global ids)
  const int* global_row0;         // [C] first pool row of every chunk
  long long max_spins;
  int* error;                     // local flag: 1 when a wait gave up
};
cudaError_t pra_route_topk_exchange(const RouteTopkArgs& args, const RouteExchangeArgs& x, cudaStream_t stream);

struct TpAllreduceArgs {
  const __nv_bfloat16* part[TP_MAX_RANKS];  // every rank's partial (peer addresses)
  const __nv_bfloat16* residual;            // local [n] or null
  __nv_bfloat16* out;                       // local [n]
  uint32_t* sig[TP_MAX_RANKS];              // every rank's signal area
  int rank, world;
  int64_t n;                                // elements (multiple of 8)
  uint32_t* epochs;                         // local [TP_MAX_BLOCKS] per-CTA call counters (start at 0)
  long long max_spins;
  int* error;
};
struct TpAllgatherArgs {
  const float* src;                         // local [rows, src_stride]
  int64_t src_stride;
  float* dst[TP_MAX_RANKS];                 // every rank's [rows, world * cols] buffer
  uint32_t* sig[TP_MAX_RANKS];
  int rank, world, rows, cols;
  uint32_t* epochs;                         // local [TP_MAX_BLOCKS] per-CTA call counters (start at 0)
  long long max_spins;
  int* error;
};
cudaError_t pra_tp_allreduce(const TpAllreduceArgs& args, cudaStream_t stream);
cudaError_t pra_tp_allgather(const TpAllgatherArgs& args, cudaStream_t stream);

// ---- embeddings (embed.cu) ---------------------------------------------------------------
cudaError_t pra_embed_add(const int* ids, const int* positions, int period, const __nv_bfloat16* tok,
                          const __nv_bfloat16* pos, int64_t M, int D, __nv_bfloat16* out, cudaStream_t stream);

// ---- decode GEMM (decode_gemm.cu) ---------------------------------------------------------
// out[M, N] = x[M, K] . w[N, K]^T for few token rows (M <= 64): one CTA per 128 output features
// (and K split), tcgen05 MMA with the weight tile as A (M = 128 features) and the token rows as
// B, fp32 accumulator in TMEM.  Epilogue: bias, residual, bf16 store split over two outputs
// (columns >= split_col go to out2), or, with world > 1, the fused all-reduce of a row-parallel
// projection (every rank's bf16 partial tile pushed to every rank, per-tile flags, residual + sum).
constexpr int DG_MAX_TILES = 1024;
constexpr int DG_MAX_SPLITS = 8;  // split-K CTAs of one tile: one portable thread-block cluster
struct DecodeGemmArgs {
  const __nv_bfloat16* x;  // [M, K] rows at stride ldx
  int64_t ldx;
  const __nv_bfloat16* w;  // [N, K] row-major
  int M, N, K, splits;
  const __nv_bfloat16* bias;      // [N] or null
  const __nv_bfloat16* residual;  // [M, N] (row stride ldo) or null
  __nv_bfloat16* out;             // columns [0, split_col): out[m * ldo + n]
  float* out_f32;                 // instead of out: fp32 results (no bias / residual / out2; one GPU)
  int swiglu;                     // each 128-row weight tile is [64 gate | 64 up] rows: out[m, tile * 64 + j] =
                                  // silu(gate_j) * up_j (N / 2 output columns; no bias / residual; one GPU)
  // RMSNorm folded into the GEMMs around it (the norm weight multiplied into this GEMM's weight
  // columns): a producer writes, per 128-feature tile and token row, the sum of squares of its
  // bf16 output (ss_out[tile * 64 + m]); a consumer scales its accumulator row m by
  // rsqrt(sum_t ss_in[t * 64 + m] / ss_dim + ss_eps), the tiles summed in order.
  float* ss_out;
  const float* ss_in;
  int ss_tiles, ss_dim;
  float ss_eps;
  int64_t ldo;
  __nv_bfloat16* out2;            // columns [split_col, N): out2[m * ldo2 + n - split_col] (null: none)
  int64_t ldo2;
  int split_col;
  // fused all-reduce (world > 1)
  int world, rank;
  __nv_bfloat16* recv[TP_MAX_RANKS];  // every rank's receive half: [world][M][N]
  uint32_t* flags[TP_MAX_RANKS];      // every rank's flag half: [DG_MAX_TILES * DG_MAX_SPLITS][world]
  uint32_t* epochs;                   // local per-(tile, row slice) call counters [DG_MAX_TILES * DG_MAX_SPLITS]
  long long max_spins;
  int* error;                         // 1 + phase after a bounded wait gave up
  // rotary decode-QKV epilogue (pos != null, world == 1): columns [0, q_end) are query heads
  // (rotated into q_out), [q_end, k_end) key heads (rotated into k_cache row cache_rows[m]),
  // [k_end, split_col) value heads (into v_cache row cache_rows[m]); columns >= split_col
  // still go to out2.  Head boundaries are multiples of head_dim, which divides 128.
  const int* pos;                     // [M] rotary position per row
  const float* cos_t;                 // [max_pos, head_dim / 2]
  const float* sin_t;
  int head_dim, q_end, k_end;
  __nv_bfloat16* q_out;
  int64_t ldq;
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  int64_t ld_cache;
  const int* cache_rows;              // [M]
};
// Launch shape of the decode GEMM: 1 (6-stage ring) or 2 (4-stage ring) CTAs per SM (fp32-output
// launches, the routing scores, use a 2-stage ring: a small footprint that fits beside the
// decode-attention CTAs it runs concurrently with), and the
// fewest 64-deep K blocks a split keeps; defaults 2 and 8.  pra_decode_gemm_splits picks the
// K split of a launch from them (the grid fills the CTA slots once).
void pra_decode_gemm_configure(int ctas_per_sm, int min_blocks_per_split, int max_splits);
int pra_decode_gemm_ctas_per_sm();
int pra_decode_gemm_splits(int tiles, int nkb, int sms);
cudaError_t pra_decode_gemm(const DecodeGemmArgs& a, cudaStream_t stream);
// Clusters of `splits` decode-GEMM CTAs that can be resident at once (rounded down to a power of
// two): the fused all-reduce needs tiles <= this.
int pra_decode_gemm_resident_clusters(int splits);
