// Tensor-parallel all-reduce fused with the residual add and RMSNorm that
// follow it in a Megatron block (o_proj -> all_reduce -> add_rms_norm and
// down_proj -> all_reduce -> add_rms_norm).
//
// One-shot push over NVLink peer memory with a low-latency word format: every
// 8-byte word carries 4 payload bytes and the 4-byte epoch of the call that
// wrote it, stored and loaded as one single-copy-atomic 64-bit access. A reader
// that sees the current epoch in a word therefore sees that call's payload, so
// the protocol needs no memory fence and no separate flag: the only latency is
// one NVLink store. Every rank owns an exchange buffer of the same size, mapped
// into every other rank's address space (CUDA IPC):
//
//   epochs u32 [max_rows]                        local: last epoch of each row's CTA
//   epochs u32 [max_rows]                        local: same for the argmax exchange
//   words  u64 [2 slots][tp][max_rows][row_words] written by peers (row_words =
//                                                row_elems * sizeof(T) / 4)
//   words  u64 [2 slots][tp][max_rows][2]        argmax candidates (value, id)
//
// CTA r (one per row) of rank k takes epoch e = epochs[r] + 1 and stores its row
// of the partial sum into slot e&1, source k, row r of every peer's buffer. It
// then polls its own buffer's words of every peer j until they carry epoch e (a
// bounded wait), sums the tp partial rows in rank order 0..tp-1 (so every rank
// computes bit-identical results), rounds to T (the value an all_reduce would
// return), adds the residual and applies RMSNorm as dli_sm100_add_rms_norm does.
//
// Why two slots suffice: CTA r of rank k writes slot e&1 of a peer j only after
// its own call at epoch e-1 read peer j's epoch e-1 words. j stored those after
// its kernel passed griddepcontrol.wait, i.e. after every earlier kernel of j's
// stream, including the one that read slot e&1 at epoch e-2, completed. Rows
// live at fixed offsets, so calls with different row counts never overlap, and
// a word left from epoch e-2 never matches epoch e.
#include <algorithm>
#include <type_traits>

#include "exchange.cuh"

namespace dli_sm100 {
namespace {

constexpr int kMaxRanks = kExchangeMaxRanks;
constexpr uint64_t kDefaultTimeoutNs = 2000000000ull;

struct ExchangeParams {
  char* buf[kMaxRanks];      // exchange buffer of each rank, as mapped in this process
  int tp;
  int rank0;                 // rank of blockIdx.y == 0
  int64_t max_rows, row_words;
  int64_t rank_stride;       // elements between ranks' tensors when one launch runs several ranks
  int64_t rows, hidden;
  float eps;
  uint64_t timeout_ns;
  unsigned* err;
};

__host__ __device__ inline int64_t header_bytes(int64_t max_rows) { return exchange_header_bytes(max_rows); }

__device__ __forceinline__ uint64_t timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// two low-latency words: payload in the low half, epoch in the high half
__device__ __forceinline__ void st_ll2(uint64_t* p, uint32_t a, uint32_t b, uint32_t e) {
  const uint64_t wa = (static_cast<uint64_t>(e) << 32) | a;
  const uint64_t wb = (static_cast<uint64_t>(e) << 32) | b;
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(wa), "l"(wb) : "memory");
}
__device__ __forceinline__ void ld_ll2(const uint64_t* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

__device__ __forceinline__ uint64_t* row_words(char* base, const ExchangeParams& p, int slot, int src, int64_t row) {
  return exchange_row_words(base, p.max_rows, p.row_words, p.tp, slot, src, row);
}

// (value, id) candidate words of the argmax exchange, after the row words.
__device__ __forceinline__ uint64_t* argmax_words(char* base, const ExchangeParams& p, int slot, int src, int64_t row) {
  uint64_t* w = reinterpret_cast<uint64_t*>(base + header_bytes(p.max_rows)) + 2 * p.tp * p.max_rows * p.row_words;
  return w + ((static_cast<int64_t>(slot) * p.tp + src) * p.max_rows + row) * 2;
}

// Waits until the 4 words at `p` carry epoch e; returns their payload. On
// timeout records the error in `failed` (and the device word) and returns what
// is there.
__device__ __forceinline__ uint4 wait_ll4(const uint64_t* p, uint32_t e, uint64_t timeout_ns, unsigned* err,
                                          bool& failed) {
  uint64_t w0, w1, w2, w3;
  ld_ll2(p, w0, w1);
  ld_ll2(p + 2, w2, w3);
  auto ready = [&] {
    return static_cast<uint32_t>(w0 >> 32) == e && static_cast<uint32_t>(w1 >> 32) == e &&
           static_cast<uint32_t>(w2 >> 32) == e && static_cast<uint32_t>(w3 >> 32) == e;
  };
  if (!ready() && !failed) {
    const uint64_t start = timer_ns();
    while (true) {
      ld_ll2(p, w0, w1);
      ld_ll2(p + 2, w2, w3);
      if (ready()) break;
      if (timer_ns() - start > timeout_ns) {
        set_device_error(err, kDevErrExchangeTimeout);
        failed = true;
        break;
      }
    }
  }
  return make_uint4(static_cast<uint32_t>(w0), static_cast<uint32_t>(w1), static_cast<uint32_t>(w2),
                    static_cast<uint32_t>(w3));
}

// VPT 16-byte vectors per thread: the host picks the smallest VPT that fits the
// row in 512 threads, so as many threads as possible issue the peer stores (one
// thread's remote stores drain slowly; the push is throughput-bound per thread).
// Residual vectors: R = T (the residual stream in the model's type, rounded
// after the add) or R = float with a 16-bit T (the residual stream kept in fp32).
template <typename T, typename R>
__device__ __forceinline__ void load_res(const R* ptr, float (&f)[Vec16<T>::N]) {
  constexpr int V = Vec16<T>::N;
  if constexpr (std::is_same<T, R>::value) {
    const Vec16<T> v = load16(ptr);
#pragma unroll
    for (int j = 0; j < V; ++j) f[j] = to_f32(v.e[j]);
  } else {
#pragma unroll
    for (int q = 0; q < V / 4; ++q) {
      const float4 x = reinterpret_cast<const float4*>(ptr)[q];
      f[4 * q] = x.x;
      f[4 * q + 1] = x.y;
      f[4 * q + 2] = x.z;
      f[4 * q + 3] = x.w;
    }
  }
}
template <typename T, typename R>
__device__ __forceinline__ void store_res(R* ptr, const float (&f)[Vec16<T>::N]) {
  constexpr int V = Vec16<T>::N;
  if constexpr (std::is_same<T, R>::value) {
    Vec16<T> v;
#pragma unroll
    for (int j = 0; j < V; ++j) v.e[j] = from_f32<T>(f[j]);
    store16(ptr, v);
  } else {
#pragma unroll
    for (int q = 0; q < V / 4; ++q)
      reinterpret_cast<float4*>(ptr)[q] = make_float4(f[4 * q], f[4 * q + 1], f[4 * q + 2], f[4 * q + 3]);
  }
}

// kPushed: the row-split GEMM already stored every rank's partial rows (its own
// included) into the group's buffers at this call's epoch (dli_sm100_linear_
// exchange_push); `delta` is unused and every source is read from this rank's
// buffer.
template <typename T, typename R, int kVpt, bool kPushed = false>
__global__ void __launch_bounds__(512) allreduce_add_rms_norm_kernel(
    ExchangeParams p, const T* __restrict__ delta, const R* residual /* may alias residual_out */,
    const T* __restrict__ w, T* __restrict__ normed, R* residual_out) {
  constexpr int V = Vec16<T>::N;
  __shared__ float scratch[32];
  __shared__ uint32_t s_epoch;
  pdl_wait();  // the partial (or, pushed, the GEMM that stored it) comes from the previous kernel
  pdl_trigger();
  const int rank = p.rank0 + static_cast<int>(blockIdx.y);
  const int64_t r = blockIdx.x;
  const int64_t off = static_cast<int64_t>(blockIdx.y) * p.rank_stride + r * p.hidden;
  char* mine = p.buf[rank];
  uint32_t* epochs = reinterpret_cast<uint32_t*>(mine);
  if (threadIdx.x == 0) s_epoch = epochs[r] + 1u;
  __syncthreads();
  const uint32_t e = s_epoch;
  const int slot = static_cast<int>(e & 1u);
  const int64_t lanes = p.hidden / V;

  // 1. own partial row into registers, pushed to every peer (4 words per 16 bytes)
  Vec16<T> own[kVpt];
#pragma unroll
  for (int i = 0; i < kVpt; ++i) {
    const int64_t c = threadIdx.x + static_cast<int64_t>(i) * blockDim.x;
    if (!kPushed && c < lanes) own[i] = load16(delta + off + c * V);
  }
  for (int q = 0; q < (kPushed ? 0 : p.tp); ++q) {
    if (q == rank) continue;
    uint64_t* dst = row_words(p.buf[q], p, slot, rank, r);
#pragma unroll
    for (int i = 0; i < kVpt; ++i) {
      const int64_t c = threadIdx.x + static_cast<int64_t>(i) * blockDim.x;
      if (c < lanes) {
        st_ll2(dst + c * 4, own[i].raw.x, own[i].raw.y, e);
        st_ll2(dst + c * 4 + 2, own[i].raw.z, own[i].raw.w, e);
      }
    }
  }

  // 2. rank-ordered sum; each peer's words are awaited where they are consumed
  float acc[kVpt][V];
#pragma unroll
  for (int i = 0; i < kVpt; ++i)
#pragma unroll
    for (int j = 0; j < V; ++j) acc[i][j] = 0.f;
  bool failed = false;
  for (int src = 0; src < p.tp; ++src) {
    if (src == rank && !kPushed) {
#pragma unroll
      for (int i = 0; i < kVpt; ++i)
#pragma unroll
        for (int j = 0; j < V; ++j) acc[i][j] += to_f32(own[i].e[j]);
      continue;
    }
    const uint64_t* s = row_words(mine, p, slot, src, r);
#pragma unroll
    for (int i = 0; i < kVpt; ++i) {
      const int64_t c = threadIdx.x + static_cast<int64_t>(i) * blockDim.x;
      if (c < lanes) {
        Vec16<T> v;
        v.raw = wait_ll4(s + c * 4, e, p.timeout_ns, p.err, failed);
#pragma unroll
        for (int j = 0; j < V; ++j) acc[i][j] += to_f32(v.e[j]);
      }
    }
  }

  // 3. residual add and RMSNorm
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kVpt; ++i) {
    const int64_t c = threadIdx.x + static_cast<int64_t>(i) * blockDim.x;
    if (c < lanes) {
      float res[V];
      load_res<T, R>(residual + off + c * V, res);
#pragma unroll
      for (int j = 0; j < V; ++j) {
        const float sum = round_through<T>(acc[i][j]);  // the all-reduced value in T
        const float h = res[j] + sum;
        acc[i][j] = std::is_same<T, R>::value ? round_through<T>(h) : h;
        ss += acc[i][j] * acc[i][j];
      }
      store_res<T, R>(residual_out + off + c * V, acc[i]);
    }
  }
  const float total = block_sum(ss, scratch);
  const float inv = rsqrtf(total / static_cast<float>(p.hidden) + p.eps);
#pragma unroll
  for (int i = 0; i < kVpt; ++i) {
    const int64_t c = threadIdx.x + static_cast<int64_t>(i) * blockDim.x;
    if (c < lanes) {
      Vec16<T> g = load16(w + c * V), o;
#pragma unroll
      for (int j = 0; j < V; ++j) o.e[j] = from_f32<T>(round_through<T>(acc[i][j] * inv) * to_f32(g.e[j]));
      store16(normed + off + c * V, o);
    }
  }
  if (threadIdx.x == 0) epochs[r] = e;
}

// Vocabulary-parallel greedy pick: rank i holds the logits of ids
// [i*width, (i+1)*width). CTA r finds its row's local argmax (largest value,
// lowest id), pushes (value, global id) to every peer as two epoch-tagged words
// and picks the winner over the ranks in rank order, so ties go to the lowest
// id exactly as one argmax over the whole row would.
__device__ __forceinline__ void better(float v, int64_t i, float& bv, int64_t& bi) {
  if (v > bv || (v == bv && i < bi)) {
    bv = v;
    bi = i;
  }
}

template <typename T>
__global__ void __launch_bounds__(256) allgather_argmax_kernel(ExchangeParams p, const T* __restrict__ x,
                                                               int64_t width, int64_t* __restrict__ out) {
  constexpr int V = Vec16<T>::N;
  constexpr int64_t kNone = INT64_MAX;
  constexpr uint32_t kNoId = 0x7fffffffu;
  __shared__ float sval[8];
  __shared__ int64_t sidx[8];
  pdl_wait();  // the logits come from the previous kernel
  pdl_trigger();
  const int rank = p.rank0 + static_cast<int>(blockIdx.y);
  const int64_t r = blockIdx.x;
  const T* row = x + static_cast<int64_t>(blockIdx.y) * p.rank_stride + r * width;
  float best = -INFINITY;
  int64_t bi = kNone;
  const bool vec = (reinterpret_cast<uintptr_t>(row) & 15) == 0;
  const int64_t nvec = vec ? width / V : 0;
  for (int64_t v0 = threadIdx.x; v0 < nvec; v0 += blockDim.x) {
    const Vec16<T> pk = load16(row + v0 * V);
#pragma unroll
    for (int j = 0; j < V; ++j) better(to_f32(pk.e[j]), v0 * V + j, best, bi);
  }
  for (int64_t c = nvec * V + threadIdx.x; c < width; c += blockDim.x) better(to_f32(row[c]), c, best, bi);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    better(ov, oi, best, bi);
  }
  if ((threadIdx.x & 31) == 0) {
    sval[threadIdx.x >> 5] = best;
    sidx[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) better(sval[w], sidx[w], best, bi);
  const uint32_t gid = bi == kNone ? kNoId : static_cast<uint32_t>(rank * width + bi);
  char* mine = p.buf[rank];
  uint32_t* epochs = reinterpret_cast<uint32_t*>(mine) + p.max_rows;
  const uint32_t e = epochs[r] + 1u;
  const int slot = static_cast<int>(e & 1u);
  for (int q = 0; q < p.tp; ++q)
    if (q != rank) st_ll2(argmax_words(p.buf[q], p, slot, rank, r), __float_as_uint(best), gid, e);
  float wv = -INFINITY;
  int64_t wi = kNone;
  bool failed = false;
  for (int src = 0; src < p.tp; ++src) {
    float v = best;
    uint32_t id = gid;
    if (src != rank) {
      const uint64_t* w = argmax_words(mine, p, slot, src, r);
      uint64_t a, b;
      ld_ll2(w, a, b);
      if (!failed && (static_cast<uint32_t>(a >> 32) != e || static_cast<uint32_t>(b >> 32) != e)) {
        const uint64_t start = timer_ns();
        while (true) {
          ld_ll2(w, a, b);
          if (static_cast<uint32_t>(a >> 32) == e && static_cast<uint32_t>(b >> 32) == e) break;
          if (timer_ns() - start > p.timeout_ns) {
            set_device_error(p.err, kDevErrExchangeTimeout);
            failed = true;
            break;
          }
        }
      }
      v = __uint_as_float(static_cast<uint32_t>(a));
      id = static_cast<uint32_t>(b);
    }
    if (id != kNoId) better(v, id, wv, wi);
  }
  out[static_cast<int64_t>(blockIdx.y) * p.rows + r] = wi == kNone ? 0 : wi;
  epochs[r] = e;
}

}  // namespace
}  // namespace dli_sm100

using namespace dli_sm100;

extern "C" size_t dli_sm100_tp_exchange_bytes(int tp, int64_t max_rows, int64_t row_elems, dli_dtype dtype) {
  if (tp < 1 || tp > kMaxRanks || max_rows <= 0 || row_elems <= 0 || !is_float_dtype(dtype)) return 0;
  // 8-byte words carrying 4 payload bytes each, then two argmax words per row
  return static_cast<size_t>(header_bytes(max_rows)) +
         static_cast<size_t>(2) * tp * max_rows * (row_elems * dtype_bytes(dtype) / 4) * 8 +
         static_cast<size_t>(2) * tp * max_rows * 2 * 8;
}

extern "C" dli_status dli_sm100_tp_exchange_reset(void* buffer, size_t bytes, void* stream) {
  // zero epochs and words: a word matches an epoch only once a peer stored it
  if (buffer == nullptr || bytes == 0) return fail(DLI_ERR_INVALID_ARGUMENT, "tp_exchange_reset: bad arguments");
  if (cudaMemsetAsync(buffer, 0, bytes, as_stream(stream)) != cudaSuccess)
    return fail(DLI_ERR_CUDA, std::string("tp_exchange_reset: ") + cudaGetErrorString(cudaGetLastError()));
  return ok();
}

extern "C" dli_status dli_sm100_allreduce_add_rms_norm(
    void* const* buffers, int tp, int rank, int ranks_in_launch, int64_t max_rows, int64_t row_elems,
    const void* delta, const void* residual, const void* w, void* normed, void* residual_out,
    int64_t rank_stride, int64_t rows, int64_t hidden, float eps, int64_t timeout_ns, dli_dtype dtype,
    void* stream) {
  return dli_sm100_allreduce_add_rms_norm_ex(buffers, tp, rank, ranks_in_launch, max_rows, row_elems, delta,
                                             residual, w, normed, residual_out, rank_stride, rows, hidden, eps,
                                             timeout_ns, dtype, dtype, stream);
}

namespace {
// The all-reduce + residual add + RMSNorm launch; `pushed`: the partial rows are
// already in the buffers (delta unused).
dli_status run_allreduce_norm(void* const* buffers, int tp, int rank, int ranks_in_launch, int64_t max_rows,
                              int64_t row_elems, const void* delta, const void* residual, const void* w, void* normed,
                              void* residual_out, int64_t rank_stride, int64_t rows, int64_t hidden, float eps,
                              int64_t timeout_ns, dli_dtype dtype, dli_dtype residual_dtype, bool pushed,
                              void* stream) {
  const char* name = pushed ? "exchange_add_rms_norm" : "allreduce_add_rms_norm";
  if (pushed) delta = residual;  // unused: keeps the null-pointer check below meaningful
  const bool res32 = residual_dtype != dtype;
  if (res32 && (residual_dtype != DLI_DTYPE_F32 || (dtype != DLI_DTYPE_BF16 && dtype != DLI_DTYPE_F16)))
    return fail(DLI_ERR_INVALID_ARGUMENT, std::string(name) + ": a float32 residual needs bfloat16/float16 tensors");
  if (buffers == nullptr || tp < 1 || tp > kMaxRanks || rank < 0 || ranks_in_launch < 1 ||
      rank + ranks_in_launch > tp || (ranks_in_launch > 1 && rank != 0))
    return fail(DLI_ERR_INVALID_ARGUMENT, std::string(name) + ": bad rank arguments");
  if (rows < 0 || hidden <= 0 || max_rows <= 0 || row_elems <= 0)
    return fail(DLI_ERR_INVALID_ARGUMENT, std::string(name) + ": bad sizes");
  if (rows == 0) return ok();
  if (!delta || !residual || !w || !normed || !residual_out)
    return fail(DLI_ERR_INVALID_ARGUMENT, std::string(name) + ": null pointer");
  if (rows > max_rows || hidden > row_elems)
    return fail(DLI_ERR_UNSUPPORTED, std::string(name) + ": rows or hidden exceed the exchange buffer");
  if (!is_float_dtype(dtype)) return fail(DLI_ERR_INVALID_ARGUMENT, std::string(name) + ": float dtype expected");
  const int V = static_cast<int>(16 / dtype_bytes(dtype));
  if (hidden % V != 0 || row_elems % V != 0)
    return fail(DLI_ERR_UNSUPPORTED, std::string(name) + ": hidden must be a multiple of 16 bytes");
  if (ranks_in_launch > 1 && rank_stride % V != 0)
    return fail(DLI_ERR_UNSUPPORTED, std::string(name) + ": rank_stride must be a multiple of 16 bytes");
  const int64_t lanes = hidden / V;
  if (ceil_div(lanes, 4) > 512) return fail(DLI_ERR_UNSUPPORTED, std::string(name) + ": hidden too large");
  for (const void* ptr : {delta, residual, w, static_cast<const void*>(normed), static_cast<const void*>(residual_out)})
    // A per-rank property, so a hard error: DLI_ERR_UNSUPPORTED is reserved for
    // shape checks, which give the same answer on every rank of the group (a
    // caller that falls back to a library all-reduce on it stays in step).
    if (!aligned(ptr, 16)) return fail(DLI_ERR_INVALID_ARGUMENT, std::string(name) + ": 16-byte aligned tensors expected");

  ExchangeParams p{};
  for (int i = 0; i < tp; ++i) {
    if (buffers[i] == nullptr || !aligned(buffers[i], 256))
      return fail(DLI_ERR_INVALID_ARGUMENT, std::string(name) + ": exchange buffers must be 256-byte aligned");
    p.buf[i] = static_cast<char*>(buffers[i]);
  }
  p.tp = tp;
  p.rank0 = rank;
  p.max_rows = max_rows;
  p.row_words = row_elems * static_cast<int64_t>(dtype_bytes(dtype)) / 4;
  p.rank_stride = rank_stride;
  p.rows = rows;
  p.hidden = hidden;
  p.eps = eps;
  p.timeout_ns = timeout_ns > 0 ? static_cast<uint64_t>(timeout_ns) : kDefaultTimeoutNs;
  p.err = device_error_word();

  // Every CTA of the launch must be resident at once: rank 0's CTA r may wait
  // for rank 1's CTA r, in this launch (several ranks on one device) or on a
  // peer. Fewest vectors per thread (most threads storing to the peers) first;
  // more per thread when that many CTAs would not all be resident.
  int vpt = 0;
  int64_t threads = 0;
  dli_status st = DLI_OK;
  for (const int cand : {1, 2, 4}) {
    const int64_t th = std::max<int64_t>(64, ceil_div(ceil_div(lanes, cand), 32) * 32);
    if (th > 512) continue;
    int per_sm = 0;
    st = dispatch_float(dtype, name, [&](auto tag) {
      using T = decltype(tag);
      auto kern = cand == 1 ? allreduce_add_rms_norm_kernel<T, T, 1>
                            : (cand == 2 ? allreduce_add_rms_norm_kernel<T, T, 2> : allreduce_add_rms_norm_kernel<T, T, 4>);
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, static_cast<int>(th), 0);
    });
    if (st != DLI_OK) return st;
    if (static_cast<int64_t>(per_sm) * sm_count() >= rows * ranks_in_launch) {
      vpt = cand;
      threads = th;
      break;
    }
  }
  if (vpt == 0) return fail(DLI_ERR_UNSUPPORTED, std::string(name) + ": more rows than resident CTAs");
  const dim3 grid(static_cast<unsigned>(rows), static_cast<unsigned>(ranks_in_launch));
  auto go = [&](auto ttag, auto rtag) {
    using T = decltype(ttag);
    using R = decltype(rtag);
    auto kern = pushed ? (vpt == 1 ? allreduce_add_rms_norm_kernel<T, R, 1, true>
                                   : (vpt == 2 ? allreduce_add_rms_norm_kernel<T, R, 2, true>
                                               : allreduce_add_rms_norm_kernel<T, R, 4, true>))
                       : (vpt == 1 ? allreduce_add_rms_norm_kernel<T, R, 1>
                                   : (vpt == 2 ? allreduce_add_rms_norm_kernel<T, R, 2>
                                               : allreduce_add_rms_norm_kernel<T, R, 4>));
    const T* d = static_cast<const T*>(delta);
    const R* res = static_cast<const R*>(residual);
    const T* wt = static_cast<const T*>(w);
    T* nm = static_cast<T*>(normed);
    R* ro = static_cast<R*>(residual_out);
    if (ranks_in_launch == 1) {
      launch_pdl(kern, grid, dim3(static_cast<unsigned>(threads)), 0, as_stream(stream), p, d, res, wt, nm, ro);
    } else {
      // one cooperative launch over all ranks of the group: co-resident CTAs
      void* args[] = {&p, &d, &res, &wt, &nm, &ro};
      cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(kern), grid, dim3(static_cast<unsigned>(threads)),
                                  args, 0, as_stream(stream));
    }
  };
  st = dispatch_float(dtype, name, [&](auto tag) {
    using T = decltype(tag);
    if (res32) go(T{}, float{});
    else go(T{}, T{});
  });
  if (st != DLI_OK) return st;
  return check_launch(name);
}
}  // namespace

extern "C" dli_status dli_sm100_allreduce_add_rms_norm_ex(
    void* const* buffers, int tp, int rank, int ranks_in_launch, int64_t max_rows, int64_t row_elems,
    const void* delta, const void* residual, const void* w, void* normed, void* residual_out,
    int64_t rank_stride, int64_t rows, int64_t hidden, float eps, int64_t timeout_ns, dli_dtype dtype,
    dli_dtype residual_dtype, void* stream) {
  return run_allreduce_norm(buffers, tp, rank, ranks_in_launch, max_rows, row_elems, delta, residual, w, normed,
                            residual_out, rank_stride, rows, hidden, eps, timeout_ns, dtype, residual_dtype, false,
                            stream);
}

extern "C" dli_status dli_sm100_exchange_add_rms_norm_ex(
    void* const* buffers, int tp, int rank, int ranks_in_launch, int64_t max_rows, int64_t row_elems,
    const void* residual, const void* w, void* normed, void* residual_out, int64_t rank_stride, int64_t rows,
    int64_t hidden, float eps, int64_t timeout_ns, dli_dtype dtype, dli_dtype residual_dtype, void* stream) {
  return run_allreduce_norm(buffers, tp, rank, ranks_in_launch, max_rows, row_elems, nullptr, residual, w, normed,
                            residual_out, rank_stride, rows, hidden, eps, timeout_ns, dtype, residual_dtype, true,
                            stream);
}

extern "C" dli_status dli_sm100_allgather_argmax(void* const* buffers, int tp, int rank, int ranks_in_launch,
                                                int64_t max_rows, int64_t row_elems, dli_dtype exchange_dtype,
                                                const void* logits, int64_t rows, int64_t width,
                                                int64_t rank_stride, int64_t* out_ids, int64_t timeout_ns,
                                                dli_dtype dtype, void* stream) {
  const char* name = "allgather_argmax";
  if (buffers == nullptr || tp < 1 || tp > kMaxRanks || rank < 0 || ranks_in_launch < 1 ||
      rank + ranks_in_launch > tp || (ranks_in_launch > 1 && rank != 0))
    return fail(DLI_ERR_INVALID_ARGUMENT, std::string(name) + ": bad rank arguments");
  if (rows < 0 || width <= 0 || max_rows <= 0 || row_elems <= 0 || !is_float_dtype(exchange_dtype))
    return fail(DLI_ERR_INVALID_ARGUMENT, std::string(name) + ": bad sizes");
  if (static_cast<int64_t>(tp) * width >= 0x7fffffffll)
    return fail(DLI_ERR_UNSUPPORTED, std::string(name) + ": vocabulary beyond 2^31 ids");
  if (rows == 0) return ok();
  if (!logits || !out_ids) return fail(DLI_ERR_INVALID_ARGUMENT, std::string(name) + ": null pointer");
  if (rows > max_rows) return fail(DLI_ERR_UNSUPPORTED, std::string(name) + ": rows exceed the exchange buffer");
  if (!is_float_dtype(dtype)) return fail(DLI_ERR_INVALID_ARGUMENT, std::string(name) + ": float dtype expected");
  ExchangeParams p{};
  for (int i = 0; i < tp; ++i) {
    if (buffers[i] == nullptr || !aligned(buffers[i], 256))
      return fail(DLI_ERR_INVALID_ARGUMENT, std::string(name) + ": exchange buffers must be 256-byte aligned");
    p.buf[i] = static_cast<char*>(buffers[i]);
  }
  p.tp = tp;
  p.rank0 = rank;
  p.max_rows = max_rows;
  p.row_words = row_elems * static_cast<int64_t>(dtype_bytes(exchange_dtype)) / 4;
  p.rank_stride = rank_stride;
  p.rows = rows;
  p.timeout_ns = timeout_ns > 0 ? static_cast<uint64_t>(timeout_ns) : kDefaultTimeoutNs;
  p.err = device_error_word();
  constexpr int kThreadsAm = 256;
  // every CTA of the launch must be resident at once (rank 0's CTA r may wait for rank 1's)
  int per_sm = 0;
  dli_status st = dispatch_float(dtype, name, [&](auto tag) {
    using T = decltype(tag);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, allgather_argmax_kernel<T>, kThreadsAm, 0);
  });
  if (st != DLI_OK) return st;
  if (static_cast<int64_t>(per_sm) * sm_count() < rows * ranks_in_launch)
    return fail(DLI_ERR_UNSUPPORTED, std::string(name) + ": more rows than resident CTAs");
  const dim3 grid(static_cast<unsigned>(rows), static_cast<unsigned>(ranks_in_launch));
  st = dispatch_float(dtype, name, [&](auto tag) {
    using T = decltype(tag);
    const T* x = static_cast<const T*>(logits);
    if (ranks_in_launch == 1) {
      launch_pdl(allgather_argmax_kernel<T>, grid, dim3(kThreadsAm), 0, as_stream(stream), p, x, width, out_ids);
    } else {
      // one cooperative launch over all ranks of the group: co-resident CTAs
      void* args[] = {&p, &x, &width, &out_ids};
      cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(allgather_argmax_kernel<T>), grid, dim3(kThreadsAm),
                                  args, 0, as_stream(stream));
    }
  });
  if (st != DLI_OK) return st;
  return check_launch(name);
}
