// Layout of a tensor-parallel exchange buffer, shared by the fused all-reduce
// kernels (k_allreduce.cu) and the GEMM epilogue that pushes a row-split
// projection's partial rows straight into the group's buffers (k_gemm.cu).
//
//   epochs u32 [max_rows]                         local: last epoch of each row
//   epochs u32 [max_rows]                         local: same for the argmax exchange
//   words  u64 [2 slots][tp][max_rows][row_words] written by the ranks (row_words =
//                                                 row_elems * sizeof(T) / 4)
//   words  u64 [2 slots][tp][max_rows][2]         argmax candidates (value, id)
//
// A word carries 4 payload bytes in its low half and the epoch of the call that
// wrote it in its high half, stored and loaded as one single-copy-atomic 64-bit
// access: a reader that sees the current epoch sees that call's payload.
#pragma once

#include "common.cuh"

namespace dli_sm100 {

constexpr int kExchangeMaxRanks = 8;
constexpr int64_t kExchangeHeaderAlign = 4096;

__host__ __device__ inline int64_t exchange_header_bytes(int64_t max_rows) {
  return (2 * max_rows * 4 + kExchangeHeaderAlign - 1) / kExchangeHeaderAlign * kExchangeHeaderAlign;
}

// The words of row `row` from source rank `src` in slot `slot` of buffer `base`.
__device__ __forceinline__ uint64_t* exchange_row_words(char* base, int64_t max_rows, int64_t row_words, int tp,
                                                        int slot, int src, int64_t row) {
  uint64_t* w = reinterpret_cast<uint64_t*>(base + exchange_header_bytes(max_rows));
  return w + ((static_cast<int64_t>(slot) * tp + src) * max_rows + row) * row_words;
}

// One low-latency word (payload, epoch) as a single 64-bit store.
__device__ __forceinline__ void exchange_store_word(uint64_t* p, uint32_t payload, uint32_t epoch) {
  const uint64_t w = (static_cast<uint64_t>(epoch) << 32) | payload;
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

}  // namespace dli_sm100
