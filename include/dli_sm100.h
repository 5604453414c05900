/*
 * dli_sm100.h — C ABI of the B200 (sm_100a) kernel library libdli_sm100.so.
 *
 * Every entry point takes plain device pointers, element counts and a CUDA
 * stream (as `void*`, NULL = legacy default stream), launches asynchronously,
 * and returns a dli_status. A non-zero status leaves a message retrievable with
 * dli_sm100_last_error() on the calling thread. Nothing here allocates device
 * memory: kernels that need scratch take a caller-provided workspace whose size
 * the matching *_workspace_size() query returns.
 *
 * Each function names the reference operator it replaces. Paths are relative to
 * the dl-inference project root (yncxcw/dl-inference). The argument meaning follows
 * the reference kernel; where the reference is specialised on a fixed table
 * (python/dli_ops/aot/<op>/template.cc), these entry points accept any size.
 *
 * Tensor layouts are dense row-major unless stated. `dtype` selects the element
 * type of the floating-point tensors of the call; arithmetic is fp32 inside.
 */
#ifndef DLI_SM100_H_
#define DLI_SM100_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DLI_SM100_ABI_VERSION 1

/* Element types. F32 and I64 are the reference's DType {Float32, Int64}
 * (include/dli/tensor.h:15); BF16/F16/I32 are additive. */
typedef enum dli_dtype {
  DLI_DTYPE_F32 = 0,
  DLI_DTYPE_I64 = 1,
  DLI_DTYPE_BF16 = 2,
  DLI_DTYPE_F16 = 3,
  DLI_DTYPE_I32 = 4
} dli_dtype;

typedef enum dli_status {
  DLI_OK = 0,
  DLI_ERR_INVALID_ARGUMENT = 1, /* reference: std::invalid_argument */
  DLI_ERR_UNSUPPORTED = 2,      /* shape/dtype combination this build does not serve */
  DLI_ERR_CUDA = 3,             /* a CUDA runtime/driver call failed (reference: std::runtime_error) */
  DLI_ERR_WORKSPACE = 4,        /* workspace missing or smaller than *_workspace_size() */
  DLI_ERR_DEVICE = 5            /* a kernel reported an error through the device error word */
} dli_status;

/* ---- library ---------------------------------------------------------- */

int dli_sm100_abi_version(void);
/* Number of kernels this library has launched (or recorded into a CUDA graph
 * under capture) since load; the reference has no counterpart (bookkeeping). */
uint64_t dli_sm100_launch_count(void);
/* Message of the last failing call on this thread ("" if none). */
const char* dli_sm100_last_error(void);
/* Reads and clears the device error word of the current device (synchronises
 * the stream). Kernels with bounded spin-waits set it instead of hanging.
 * Returns DLI_OK or DLI_ERR_DEVICE with a message naming the failing kernel. */
dli_status dli_sm100_check_device_error(void* stream);

/* ---- contractions ----------------------------------------------------- */

/* linear: y[M,N] = x[M,K] · w[N,K]^T (+ bias[N]); bias may be NULL.
 * Replaces the `linear` operator: python/dli_ops/aot/linear/kernel.py:5-44 and
 * its launcher python/dli_ops/aot/linear/template.cc:14-34 (M = product of the
 * leading dims of x, template.cc:23). BF16/F16 run on tcgen05 tensor cores
 * (TMA-fed, TMEM accumulators, fp32 accumulate); F32 runs an exact-fp32 FFMA
 * kernel (the reference's tl.dot runs fp32 as TF32).
 * Decode-sized problems (few rows) stream the weight matrix once with the
 * weights on the MMA M side. When their tiles do not fill whole waves of the
 * GPU, the (tile, K block) work is split evenly over every resident CTA
 * (stream-K): partial tiles go through the workspace and the last contributor
 * of a tile sums them in a fixed order (deterministic). The workspace of
 * dli_sm100_linear_workspace_size() bytes must be zero-filled before its first
 * use and is left zeroed by every call (so it can be reused, and replayed in a
 * CUDA graph); calls sharing one workspace must not overlap on the GPU. Without
 * a workspace (NULL / too small) K is split over thread-block clusters reduced
 * through distributed shared memory instead. F32 needs no workspace. */
size_t dli_sm100_linear_workspace_size(int64_t m, int64_t n, int64_t k, dli_dtype dtype);
dli_status dli_sm100_linear(const void* x, const void* w, const void* bias, void* y, int64_t m,
                            int64_t n, int64_t k, dli_dtype dtype, void* workspace,
                            size_t workspace_bytes, void* stream);

/* linear with a wider output type: y[M,N] (out_dtype) = x[M,K] · w[N,K]^T (+ bias[N]),
 * x, w and bias in `dtype`. Serves BF16/F16 operands with an F32 output (the
 * fp32 accumulator stored without rounding to bf16), used for the LM-head logits
 * that greedy decoding takes the argmax of; out_dtype == dtype is
 * dli_sm100_linear. The workspace is dli_sm100_linear's (same size query). Additive: the reference's linear (python/dli_ops/aot/linear/
 * template.cc:14-34) always writes its input dtype, fp32. */
dli_status dli_sm100_linear_ex(const void* x, const void* w, const void* bias, void* y, int64_t m,
                               int64_t n, int64_t k, dli_dtype dtype, dli_dtype out_dtype, void* workspace,
                               size_t workspace_bytes, void* stream);

/* Fused gate/up projection + SwiGLU (additive; the reference graph runs
 * linear -> silu -> mul): y[M, inter] = silu(x · Wg^T) * (x · Wu^T), computed in
 * fp32 from the two fp32 accumulators and rounded to dtype once (the unfused
 * nodes round each linear output, the silu output and the product). w_glu holds Wg and Wu interleaved in 64-row blocks: rows
 * [128b, 128b+64) are gate rows [64b, 64b+64) and rows [128b+64, 128b+128) the
 * matching up rows, 2*ceil(inter/64)*64 rows of K in all, the rows past `inter`
 * zero. BF16/F16 only (DLI_ERR_UNSUPPORTED otherwise): one tcgen05 GEMM whose
 * epilogue pairs the gate and up accumulators, so the [M, 2*inter] gate/up
 * tensor is never written. */
dli_status dli_sm100_linear_silu_mul(const void* x, const void* w_glu, void* y, int64_t m, int64_t inter,
                                     int64_t k, dli_dtype dtype, void* stream);

/* matmul: out[M,N] = a[M,K] · b[K,N] (both row-major, 2-D).
 * Replaces python/dli_ops/aot/matmul/kernel.py:5-40, template.cc:14-30. */
dli_status dli_sm100_matmul(const void* a, const void* b, void* out, int64_t m, int64_t n,
                            int64_t k, dli_dtype dtype, void* stream);

/* conv2d (NCHW): out[N,OC,OH,OW] = conv(x[N,C,H,W], w[OC,C,KH,KW]) + bias[OC].
 * OH = (H + 2*pad_h - KH)/stride_h + 1 (python/dli_ops/aot/conv2d/template.cc:13-14).
 * Replaces python/dli_ops/aot/conv2d/kernel.py:5-49. BF16/F16 run as an implicit
 * GEMM on tcgen05: patch tiles are gathered into shared memory inside the GEMM,
 * no patch matrix is written; the workspace holds only a copy of the weight
 * padded to a multiple of 8 columns when C*KH*KW is not one (else 0 bytes).
 * F32 3x3 runs a tiled CUDA-core kernel, other F32 shapes a direct one. */
size_t dli_sm100_conv2d_workspace_size(int64_t n, int64_t c, int64_t h, int64_t w, int64_t oc,
                                       int64_t kh, int64_t kw, int64_t stride_h, int64_t stride_w,
                                       int64_t pad_h, int64_t pad_w, dli_dtype dtype);
dli_status dli_sm100_conv2d(const void* x, const void* weight, const void* bias, void* out,
                            int64_t n, int64_t c, int64_t h, int64_t w, int64_t oc, int64_t kh,
                            int64_t kw, int64_t stride_h, int64_t stride_w, int64_t pad_h,
                            int64_t pad_w, dli_dtype dtype, void* workspace,
                            size_t workspace_bytes, void* stream);

/* ---- normalisation ---------------------------------------------------- */

/* rms_norm over the last dim: out = x * rsqrt(mean(x^2) + eps) * w.
 * Replaces python/dli_ops/aot/rms_norm/kernel.py:5-14, template.cc:12-28. */
dli_status dli_sm100_rms_norm(const void* x, const void* w, void* out, int64_t rows,
                              int64_t hidden, float eps, dli_dtype dtype, void* stream);

/* Fused residual add + rms_norm: residual_out = residual + delta;
 * normed = rms_norm(residual_out, w). Replaces the `add` -> `rms_norm` node pair
 * the reference exporter emits per layer (python/dli_export/export.py:385-396).
 * residual_out may alias residual. */
dli_status dli_sm100_add_rms_norm(const void* residual, const void* delta, const void* w,
                                  void* normed, void* residual_out, int64_t rows, int64_t hidden,
                                  float eps, dli_dtype dtype, void* stream);

/* add_rms_norm with the residual stream in a wider type: residual and
 * residual_out are `residual_dtype` (F32), delta, w and normed are `dtype`
 * (BF16/F16). residual_out = residual + delta in fp32, unrounded; normed as
 * dli_sm100_add_rms_norm. residual_out may alias residual. Additive (the
 * reference's graphs run add then rms_norm in fp32, export.py:385,428): keeping
 * the running sum of a 16-bit model in fp32 removes a rounding per layer from
 * the logits. residual_dtype == dtype is dli_sm100_add_rms_norm. */
dli_status dli_sm100_add_rms_norm_ex(const void* residual, const void* delta, const void* w,
                                     void* normed, void* residual_out, int64_t rows, int64_t hidden,
                                     float eps, dli_dtype dtype, dli_dtype residual_dtype, void* stream);

/* batch_norm2d (inference): out = (x - mean[c]) * rsqrt(var[c] + eps) * weight[c] + bias[c].
 * Replaces python/dli_ops/aot/batch_norm2d/kernel.py:5-28, template.cc:1-33. */
dli_status dli_sm100_batch_norm2d(const void* x, const void* weight, const void* bias,
                                  const void* running_mean, const void* running_var, void* out,
                                  int64_t total, int64_t channels, int64_t spatial, float eps,
                                  dli_dtype dtype, void* stream);

/* softmax over the last dim. Replaces python/dli_ops/aot/softmax/kernel.py:5-14. */
dli_status dli_sm100_softmax(const void* x, void* out, int64_t rows, int64_t width,
                             dli_dtype dtype, void* stream);

/* ---- positional / attention ------------------------------------------- */

/* rotary_embedding on interleaved pairs (2i, 2i+1), the reference convention
 * (python/dli_ops/aot/rotary/kernel.py:22-35): q[B,Hq,S,D], k[B,Hk,S,D] (Hk may
 * differ from Hq), cos/sin fp32 [table_rows, pairs]. Pair i < pairs of token s
 * uses table row p = start_pos + s, or positions[b] + s when `positions` (int64,
 * numel == B) is given, or positions[b*S + s] when numel == B*S
 * (`positions_numel`). Pairs >= `pairs` are copied unchanged
 * (python/dli_ops/aot/rotary/template.cc:11-12). Rows beyond the table are an
 * error reported through the device error word and leave the pair unrotated.
 * Replaces python/dli_ops/aot/rotary/template.cc:1-28. */
dli_status dli_sm100_rotary_embedding(const void* q, const void* k, const float* cos_table,
                                      const float* sin_table, void* out_q, void* out_k,
                                      int64_t batch, int64_t q_heads, int64_t k_heads,
                                      int64_t seq, int64_t head_dim, int64_t pairs,
                                      int64_t table_rows, int64_t start_pos,
                                      const int64_t* positions, int64_t positions_numel,
                                      dli_dtype dtype, void* stream);

/* attention: out[B,Hq,Sq,D] = softmax(q k^T * scale (+ bottom-right causal mask)) v
 * with q[B,Hq,Sq,D], k/v[B,Hkv,Sk,D] read at row stride D inside a per-(b,h)
 * block of `kv_capacity` rows (kv_capacity >= Sk; == Sk for dense inputs).
 * Query row i may see key j iff j <= i + (Sk - Sq) (python/dli_ops/aot/attention/
 * kernel.py:35,49-50). Hq must be a multiple of Hkv (GQA; the reference requires
 * Hq == Hkv). scale <= 0 selects 1/sqrt(D) (build_triton_aot_ops.py:283).
 * Replaces python/dli_ops/aot/attention/kernel.py:5-62 and template.cc:1-49. */
size_t dli_sm100_attention_workspace_size(int64_t batch, int64_t q_heads, int64_t kv_heads,
                                          int64_t seq_q, int64_t seq_k, int64_t head_dim,
                                          dli_dtype dtype);
dli_status dli_sm100_attention(const void* q, const void* k, const void* v, void* out,
                               int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t seq_q,
                               int64_t seq_k, int64_t kv_capacity, int64_t head_dim, int causal,
                               float scale, dli_dtype dtype, void* workspace,
                               size_t workspace_bytes, void* stream);

/* KV-cache append: copies k/v[B,H,S_new,D] into rows [old_len, old_len+S_new) of
 * a preallocated cache_k/cache_v[B,H,capacity,D]. Replaces the realloc + flat
 * memcpy of src/kv_cache.cc:9-44, whose flat concatenation is wrong when B*H > 1. */
dli_status dli_sm100_kv_append(void* cache_k, void* cache_v, const void* k, const void* v,
                               int64_t batch, int64_t heads, int64_t capacity, int64_t old_len,
                               int64_t new_len, int64_t head_dim, dli_dtype dtype, void* stream);

/* Fused rotary + KV-cache write for a fused QKV projection (additive; used by the
 * batched Qwen2 graphs). qkv[B*S, (Hq + 2*Hkv)*D] holds q heads, then k heads,
 * then v heads per token. Token s of sequence b sits at position
 * p = positions[b] + s (int64). Writes rotated q to q_out[B,S,Hq,D], rotated k
 * and raw v to cache rows p of cache_k/cache_v[B,Hkv,capacity,D]. */
dli_status dli_sm100_qkv_rotary_cache(const void* qkv, const float* cos_table,
                                      const float* sin_table, const int64_t* positions,
                                      void* q_out, void* cache_k, void* cache_v, int64_t batch,
                                      int64_t seq, int64_t q_heads, int64_t kv_heads,
                                      int64_t head_dim, int64_t pairs, int64_t table_rows,
                                      int64_t capacity, dli_dtype dtype, void* stream);

/* The q|k|v projection and dli_sm100_qkv_rotary_cache in one kernel (additive):
 * qkv = x[B*S, k] . wqkv[(Hq+2Hkv)*D, k]^T + bqkv, rounded to dtype, then q
 * rotated into q_out [B,S,Hq,D] and rotated k / raw v written into the cache
 * rows positions[b] + s, bit-identical to linear followed by
 * dli_sm100_qkv_rotary_cache (same tables, same error words for positions
 * outside the table or the capacity). The qkv tensor is never written: the
 * GEMM's split-K epilogue rotates and scatters. Serves decode-sized calls
 * (B*S <= 128 on a split-K plan); other shapes return DLI_ERR_UNSUPPORTED
 * without launching, and callers run the two-step form. */
dli_status dli_sm100_linear_qkv_rotary_cache(const void* x, const void* wqkv, const void* bqkv, const float* cos_table,
                                             const float* sin_table, const int64_t* positions, void* q_out,
                                             void* cache_k, void* cache_v, int64_t batch, int64_t seq, int64_t k,
                                             int64_t q_heads, int64_t kv_heads, int64_t head_dim, int64_t pairs,
                                             int64_t table_rows, int64_t capacity, dli_dtype dtype, void* stream);

/* Attention over a KV cache with per-sequence lengths (additive). q/out are
 * [B,S,Hq,D] (token-major, the layout a linear emits); cache_k/v are
 * [B,Hkv,capacity,D]; sequence b sees keys [0, positions[b] + S) with the
 * bottom-right causal mask. */
size_t dli_sm100_attention_kvcache_workspace_size(int64_t batch, int64_t seq, int64_t q_heads,
                                                  int64_t kv_heads, int64_t capacity,
                                                  int64_t head_dim, dli_dtype dtype);
dli_status dli_sm100_attention_kvcache(const void* q, const void* cache_k, const void* cache_v,
                                       const int64_t* positions, void* out, int64_t batch,
                                       int64_t seq, int64_t q_heads, int64_t kv_heads,
                                       int64_t capacity, int64_t head_dim, float scale,
                                       dli_dtype dtype, void* workspace, size_t workspace_bytes,
                                       void* stream);

/* Same as dli_sm100_attention_kvcache, for callers that cannot allocate device
 * memory (a fixed memory budget set up front, an allocator owned by another
 * runtime, or a hot path that must not take allocator locks). No counterpart in
 * the reference: it is an additive entry point of this library. The split-KV
 * scratch comes from one fixed device array inside the library, sized
 * dli_sm100_attention_kvcache_noalloc_max_scratch() bytes (4 MiB) and held by
 * every GPU that loads the library until the process exits; shapes needing more
 * fail with DLI_ERR_WORKSPACE. The first call on a device resolves the array's
 * device address (cudaGetSymbolAddress) with that device current, so make that
 * first call before any stream capture. Every call shares the one array, so calls
 * that overlap on the GPU (other streams, other threads) race; serialize them.
 * Nothing in it has to start at zero. The call allocates nothing. */
size_t dli_sm100_attention_kvcache_noalloc_max_scratch(void);
dli_status dli_sm100_attention_kvcache_noalloc(const void* q, const void* cache_k,
                                               const void* cache_v, const int64_t* positions,
                                               void* out, int64_t batch, int64_t seq,
                                               int64_t q_heads, int64_t kv_heads, int64_t capacity,
                                               int64_t head_dim, float scale, dli_dtype dtype,
                                               void* stream);

/* ---- elementwise / data movement -------------------------------------- */

/* out[i] = a[i] + b[i mod width] (python/dli_ops/aot/add/kernel.py:5-11). */
dli_status dli_sm100_add(const void* a, const void* b, void* out, int64_t total, int64_t width,
                         dli_dtype dtype, void* stream);
/* out[i] = a[i] * b[i mod width] (python/dli_ops/aot/mul/kernel.py:5-11). */
dli_status dli_sm100_mul(const void* a, const void* b, void* out, int64_t total, int64_t width,
                         dli_dtype dtype, void* stream);
/* out = x / (1 + exp(-x)) (python/dli_ops/aot/silu/kernel.py:5-10). */
dli_status dli_sm100_silu(const void* x, void* out, int64_t total, dli_dtype dtype, void* stream);
/* out = max(x, 0) (python/dli_ops/aot/relu/kernel.py:5-10). */
dli_status dli_sm100_relu(const void* x, void* out, int64_t total, dli_dtype dtype, void* stream);
/* Fused SwiGLU (additive): gate_up[rows, 2*width] holds gate then up;
 * out[rows, width] = silu(gate) * up. Replaces the silu -> mul node pair of
 * python/dli_export/export.py:414-415. */
dli_status dli_sm100_silu_mul(const void* gate_up, void* out, int64_t rows, int64_t width,
                              dli_dtype dtype, void* stream);
/* out[t, :] = table[ids[t], :]; ids int64 (ids_dtype I64) or int32. Ids outside
 * [0, vocab) produce zero rows and set the device error word.
 * Replaces python/dli_ops/aot/embedding/kernel.py:5-23. */
dli_status dli_sm100_embedding(const void* ids, dli_dtype ids_dtype, const void* table, void* out,
                               int64_t total, int64_t hidden, int64_t vocab, dli_dtype dtype,
                               void* stream);
/* 2-D transpose out[C,R] = x[R,C]^T (python/dli_ops/aot/transpose/kernel.py:5-20). */
dli_status dli_sm100_transpose2d(const void* x, void* out, int64_t rows, int64_t cols,
                                 dli_dtype dtype, void* stream);
/* max_pool2d (NCHW), padding reads -inf (python/dli_ops/aot/max_pool2d/kernel.py:5-41). */
dli_status dli_sm100_max_pool2d(const void* x, void* out, int64_t n, int64_t c, int64_t h,
                                int64_t w, int64_t kh, int64_t kw, int64_t stride_h,
                                int64_t stride_w, int64_t pad_h, int64_t pad_w, dli_dtype dtype,
                                void* stream);
/* Row argmax (additive, greedy decoding): out_ids[r] = argmax_j x[r, j] (int64,
 * lowest index on ties). */
dli_status dli_sm100_argmax(const void* x, int64_t* out_ids, int64_t rows, int64_t width,
                            dli_dtype dtype, void* stream);
/* Gathers row `index` of every [seq, width] block (additive; last-token LM head):
 * out[b, :] = x[b, index, :]. */
dli_status dli_sm100_select_token(const void* x, void* out, int64_t batch, int64_t seq,
                                  int64_t width, int64_t index, dli_dtype dtype, void* stream);
/* Copies `n` elements converting between F32/BF16/F16 (additive, graph casts). */
dli_status dli_sm100_cast(const void* x, dli_dtype x_dtype, void* out, dli_dtype out_dtype,
                          int64_t n, void* stream);

/* ---- tensor-parallel exchange ---------------------------------------------
 * No counterpart in the reference, which runs every graph on one device. Used
 * by the Qwen2 tensor-parallel graphs (all_reduce after o_proj and down_proj).
 *
 * Each rank of a tensor-parallel group owns one exchange buffer of
 * dli_sm100_tp_exchange_bytes(tp, max_rows, row_elems, dtype) bytes, 256-byte
 * aligned, mapped into every other rank's process (CUDA IPC). Before first use
 * every rank zeroes its whole buffer with dli_sm100_tp_exchange_reset and the
 * group synchronises; afterwards the buffers are never reset (epochs advance on
 * the device, so CUDA-graph replays need no host work). A buffer whose call
 * timed out is out of step with its peers: reset the group before reusing it.
 * dli_sm100_tp_exchange_bytes returns 0 for unsupported arguments (tp outside
 * 1..8). */
size_t dli_sm100_tp_exchange_bytes(int tp, int64_t max_rows, int64_t row_elems, dli_dtype dtype);
dli_status dli_sm100_tp_exchange_reset(void* buffer, size_t bytes, void* stream);

/* All-reduce of `delta` over the group fused with add_rms_norm:
 * residual_out = residual + sum_ranks(delta) (the sum rounded to dtype, as an
 * all_reduce returns it); normed = rms_norm(residual_out, w) exactly as
 * dli_sm100_add_rms_norm. One CTA per row pushes its row of delta into every
 * peer's buffer over NVLink as 8-byte words carrying the call's epoch, and
 * polls its own buffer (bounded by timeout_ns, 0 = 2 s) for the peers' words of
 * that epoch; the sum runs in rank order, so every rank gets identical bits.
 * A wait that runs out sets the device error word (dli_sm100_check_device_error)
 * instead of hanging. Every rank of the group must make the same calls with
 * the same rows, in the same order.
 *   buffers[i]      rank i's exchange buffer as mapped in this process (tp entries)
 *   rank            this process's rank; ranks_in_launch = 1 for one process per GPU.
 *                   ranks_in_launch = tp (with rank = 0) runs the whole group in one
 *                   cooperative launch on one device, all buffers on that device,
 *                   per-rank tensors rank_stride elements apart (a test harness mode)
 *   rows <= max_rows, hidden <= row_elems, hidden * element size a multiple of 16
 * residual_out may alias residual. DLI_ERR_UNSUPPORTED when the shape does not
 * fit the exchange buffer or the launch cannot be resident at once (callers
 * then fall back to a library all-reduce + dli_sm100_add_rms_norm); these depend
 * on shapes only, so every rank reaches the same answer. A tensor that is not
 * 16-byte aligned is DLI_ERR_INVALID_ARGUMENT (a per-rank property: falling back
 * on it would leave this rank in a library collective its peers never join).
 * After a wait ran out (DLI_ERR_DEVICE from dli_sm100_check_device_error) the
 * buffers hold words of an abandoned exchange: every rank must zero its buffer
 * with dli_sm100_tp_exchange_reset, and the group must synchronise, before the
 * next exchange call. */
/* Greedy pick over a vocabulary split across the group (vocab-parallel LM head):
 * rank i holds logits[rows, width] for ids [i*width, (i+1)*width). out_ids[r] =
 * the id of the largest logit of row r over all ranks, lowest id on ties (the
 * result dli_sm100_argmax gives over the whole row; 0 for a row without a
 * candidate). Each CTA pushes its row's (value, id) to every peer as two
 * epoch-tagged words and polls for theirs (bounded by timeout_ns, 0 = 2 s).
 * Same buffers, rank arguments and call-order rule as
 * dli_sm100_allreduce_add_rms_norm; exchange_dtype and row_elems are the
 * buffers' (they place the candidate words). With ranks_in_launch = tp the
 * ranks' logits are rank_stride elements apart and out_ids holds tp x rows ids. */
dli_status dli_sm100_allgather_argmax(void* const* buffers, int tp, int rank, int ranks_in_launch, int64_t max_rows,
                                      int64_t row_elems, dli_dtype exchange_dtype, const void* logits, int64_t rows,
                                      int64_t width, int64_t rank_stride, int64_t* out_ids, int64_t timeout_ns,
                                      dli_dtype dtype, void* stream);

/* A row-split projection and its all-reduce in fewer steps (additive; the
 * reference has no tensor parallelism): dli_sm100_linear_exchange_push computes
 * y = x[m,k] . w[n,k]^T (+ bias[n]) for m <= 128 tokens on tcgen05 and, instead
 * of writing y, stores this rank's partial rows (rounded to dtype) as
 * epoch-tagged words into every rank's exchange buffer, from the GEMM's own
 * split-K epilogue; dli_sm100_exchange_add_rms_norm_ex then waits for all
 * ranks' rows in this rank's buffer, sums them in rank order and applies the
 * residual add and RMSNorm exactly as dli_sm100_allreduce_add_rms_norm_ex does
 * with the partial y as delta (bit-identical results). The two calls go
 * back to back on the stream, once per projection, on every rank of the group.
 * dli_sm100_linear_exchange_push returns DLI_ERR_UNSUPPORTED, launching
 * nothing, for shapes it does not serve (m > 128, a plan without split-K); the
 * decision depends on (m, n, k, dtype) only, so every rank makes the same one
 * and can fall back to linear + dli_sm100_allreduce_add_rms_norm_ex together.
 * Misaligned operands are DLI_ERR_INVALID_ARGUMENT. row_elems >= n, a multiple
 * of 8; max_rows >= m. */
dli_status dli_sm100_linear_exchange_push(const void* x, const void* w, const void* bias, int64_t m, int64_t n,
                                          int64_t k, dli_dtype dtype, void* const* buffers, int tp, int rank,
                                          int64_t max_rows, int64_t row_elems, void* stream);
dli_status dli_sm100_exchange_add_rms_norm_ex(void* const* buffers, int tp, int rank, int ranks_in_launch,
                                              int64_t max_rows, int64_t row_elems, const void* residual,
                                              const void* w, void* normed, void* residual_out, int64_t rank_stride,
                                              int64_t rows, int64_t hidden, float eps, int64_t timeout_ns,
                                              dli_dtype dtype, dli_dtype residual_dtype, void* stream);

dli_status dli_sm100_allreduce_add_rms_norm(void* const* buffers, int tp, int rank, int ranks_in_launch,
                                            int64_t max_rows, int64_t row_elems, const void* delta,
                                            const void* residual, const void* w, void* normed,
                                            void* residual_out, int64_t rank_stride, int64_t rows,
                                            int64_t hidden, float eps, int64_t timeout_ns, dli_dtype dtype,
                                            void* stream);
/* dli_sm100_allreduce_add_rms_norm with the residual stream in float32:
 * residual and residual_out are `residual_dtype` (F32) while delta, w and
 * normed are `dtype` (BF16/F16); the all-reduced delta is rounded to dtype (the
 * value an all-reduce returns) and added to the fp32 residual without rounding,
 * as dli_sm100_add_rms_norm_ex does. residual_dtype == dtype is the call above. */
dli_status dli_sm100_allreduce_add_rms_norm_ex(void* const* buffers, int tp, int rank, int ranks_in_launch,
                                               int64_t max_rows, int64_t row_elems, const void* delta,
                                               const void* residual, const void* w, void* normed,
                                               void* residual_out, int64_t rank_stride, int64_t rows,
                                               int64_t hidden, float eps, int64_t timeout_ns, dli_dtype dtype,
                                               dli_dtype residual_dtype, void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* DLI_SM100_H_ */
