// Internal interface of the tcgen05 prefill attention kernel (k_fmha.cu).
#pragma once

#include "common.cuh"

namespace dli_sm100 {

// softmax(q k^T * scale + bottom-right causal mask) v over strided q/out
// ([.., S, .., D] with element (b, h, s, d) at b*sb + h*sh + s*ss + d) and K/V
// rows of D elements, head (b, kvh) starting at b*k_sb + kvh*k_sh, key j at
// + j*D. Key count of sequence b: positions[b] + seq_q when positions is
// non-null (a KV cache addressed by position), else dense_kv.
struct FmhaArgs {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  int64_t q_sb, q_sh, q_ss;
  int64_t o_sb, o_sh, o_ss;
  int64_t k_sb, k_sh;
  int batch, hq, hkv, seq_q, dense_kv, head_dim;
  const int64_t* positions;
  float scale_log2;  // scale * log2(e)
  int causal;
};

// True when the tcgen05 kernel serves these arguments: bf16/f16, head_dim 64
// or 128, 16-byte aligned tensors and strides (TMA), batch-outermost layouts.
bool fmha_supported(const FmhaArgs& a, dli_dtype dtype);

// True when DLI_SM100_ATTN_FMHA=2: a bf16/f16 prefill this kernel cannot serve
// is an error instead of a launch of the mma.sync kernel.
bool fmha_required();

// 4-D bf16/f16 tensor map: dims[0] innermost (contiguous), byte strides of
// dims 1..3, 128-byte swizzle, elements outside the dims read as zero. Returns
// DLI_ERR_UNSUPPORTED when the encoder rejects the layout.
dli_status make_map_4d(CUtensorMap* map, const void* base, bool bf16, const uint64_t (&dims)[4],
                       const uint64_t (&strides)[3], const uint32_t (&box)[4]);

// Launches the kernel on `stream` (fmha_supported() must hold). Returns
// DLI_ERR_UNSUPPORTED, launching nothing, when a tensor map cannot be encoded.
dli_status run_fmha_prefill(const FmhaArgs& a, dli_dtype dtype, cudaStream_t stream);

}  // namespace dli_sm100
