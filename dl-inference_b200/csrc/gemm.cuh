// Internal GEMM interface shared by linear, matmul and conv2d.
#pragma once

#include "common.cuh"

namespace dli_sm100 {

// Output mapping of the TN GEMM D[i, j] = sum_k A[i, k] * B[j, k].
enum GemmEpilogue : int {
  kEpiRowMajor = 0,   // out[i * ldo + j], bias[j]           (A = activations, B = weights)
  kEpiTransposed = 1, // out[j * ldo + i], bias[i]           (swap-AB: A = weights, B = activations)
  kEpiNchw = 2,       // i = img * ohw + pix, j = channel -> out[(img * OC + j) * ohw + pix], bias[j]
  // SwiGLU over weights in 64-row gate/up blocks (rows 128b..128b+63 = gate rows
  // 64b.., rows 128b+64.. = the matching up rows): out = silu(gate) * up, I cols
  kEpiGluT = 3,       // swap-AB: D row i = weight row -> out[j * ldo + (i/128)*64 + i%64]
  kEpiGlu = 4,        // D column j = weight row -> out[i * ldo + (j/128)*64 + j%64]
  // swap-AB, split-K push plans only: D row i = output feature, column j = token;
  // the rows, rounded to T, go as epoch-tagged words into every tensor-parallel
  // rank's exchange buffer (row j, feature pairs i, i+1 per word), not to `out`
  kEpiExchange = 5,
  // swap-AB, split-K push plans only: D row i = feature of the fused q|k|v
  // projection, column j = token; rounded to T, the q and k rows rotated
  // (interleaved pairs i, i+1) and written to q_out [tokens, Hq, D] and into
  // the KV cache rows of each token's position, as dli_sm100_qkv_rotary_cache
  // does with the projection's output
  kEpiQkvRotary = 6,
};

struct GemmPlan {
  int bn = 0;             // tile width along j (tcgen05 N)
  int stages = 0;
  int tiles_i = 0, tiles_j = 0;
  int splits = 1;
  int kblocks = 0;
  bool tcgen05 = false;   // false -> SIMT fallback
  size_t workspace = 0;   // bytes of split-K scratch (partials + tile counters)
  int streamk_ctas = 0;   // > 0: stream-K over this many CTAs (tcgen05_gemm_streamk_kernel)
};

// Turns a swap-AB decode plan (tile width <= 64) whose tiles do not fill whole
// waves into a stream-K plan over every resident slot; sets streamk_ctas and
// workspace (partial tiles + per-tile counters, zero-filled by the caller once
// and left zeroed). Leaves other plans unchanged.
GemmPlan plan_streamk(GemmPlan plan);

// Occupancy of the tcgen05 GEMM with tile width bn and `stages` pipeline stages:
// CTAs per SM for cluster <= 1, else resident clusters of `cluster` CTAs
// (cached per device; 0 when no device answers).
int gemm_occupancy(int bn, int stages, int cluster);

// Plans a TN GEMM with rows_a x K and rows_b x K operands.
GemmPlan plan_tn_gemm(int64_t rows_a, int64_t rows_b, int64_t k, dli_dtype dtype, bool allow_split);

// Runs D = A * B^T on tcgen05 (bf16/f16 only; K % 8 == 0; A/B 16-byte aligned).
// `b_mn`: B is given MN-major as [K, rows_b] with row stride ldb (matmul's right
// operand); needs a row-major epilogue and a plan of tile width >= 64.
// `ldo` is the output row stride (elements); `ohw` is used by kEpiNchw.
// `const_a` / `const_b` mark an operand that no kernel writes (weights): its
// first tiles are fetched before the kernel waits on the previous kernel.
// Split-K plans reduce inside a thread-block cluster and need no workspace
// (the arguments are kept for plans that would).
dli_status run_tn_gemm_tcgen05(const void* a, const void* b, const void* bias, void* out,
                               int64_t rows_a, int64_t rows_b, int64_t k, int64_t lda,
                               int64_t ldb, int64_t ldo, int epilogue, int64_t ohw,
                               dli_dtype dtype, const GemmPlan& plan, void* workspace,
                               size_t workspace_bytes, cudaStream_t stream, bool const_a,
                               bool const_b, int64_t glu_cols = 0, bool out_f32 = false,
                               bool b_mn = false);

// NCHW convolution geometry (every extent, and N*C*H*W and N*OC*OH*OW, below 2^31).
struct ConvGeom {
  int n, c, h, w, oc, kh, kw, sh, sw, ph, pw, oh, ow;
};

// Implicit-GEMM convolution on tcgen05 (bf16/f16): patch tiles gathered in shared
// memory from the NCHW input, the weight as a K-major [OC, kp] operand (kp =
// C*KH*KW rounded up to 8, zero columns past K), bias, NCHW output.
dli_status run_conv_implicit_tcgen05(const void* x, const void* w_kmajor, int64_t kp, const void* bias, void* out,
                                     const ConvGeom& g, dli_dtype dtype, cudaStream_t stream, bool const_w);

// SIMT fallback (any float dtype, any alignment): out[M,N] = A[M,K] . B + bias,
// with B given as [N,K] (b_kmajor) or [K,N].
dli_status run_gemm_simt(const void* a, const void* b, const void* bias, void* out, int64_t m,
                         int64_t n, int64_t k, bool b_kmajor, dli_dtype dtype,
                         cudaStream_t stream);

}  // namespace dli_sm100
