// Rotary position embedding on interleaved pairs (2i, 2i+1) — the reference
// convention of python/dli_ops/aot/rotary/kernel.py:22-35:
//   out[2i]   = x[2i] * cos[p, i] - x[2i+1] * sin[p, i]
//   out[2i+1] = x[2i] * sin[p, i] + x[2i+1] * cos[p, i]
// with p the table row of the token. Two entry points:
//  * dli_sm100_rotary_embedding: q[B,Hq,S,D] and k[B,Hk,S,D] as separate
//    tensors (the reference operator; Hk may differ from Hq, which the reference
//    kernel gets wrong because it sizes k's loop from q, template.cc:14);
//  * dli_sm100_qkv_rotary_cache: one pass over a fused QKV projection that
//    rotates q into a [B,S,Hq,D] buffer and writes rotated k and raw v straight
//    into the KV cache rows of each token (no separate append pass).
// The reference-shaped kernel moves one pair per thread step; the fused QKV form
// moves one 16-byte vector per step when the layout allows.
#include <algorithm>

#include "common.cuh"

namespace dli_sm100 {
namespace {

template <typename T> struct Pair;
template <> struct Pair<float> { using type = float2; };
template <> struct Pair<__nv_bfloat16> { using type = __nv_bfloat162; };
template <> struct Pair<__half> { using type = __half2; };

template <typename T>
__device__ __forceinline__ float2 load_pair(const T* p) {
  if constexpr (sizeof(T) == 4) {
    return *reinterpret_cast<const float2*>(p);
  } else {
    const typename Pair<T>::type v = *reinterpret_cast<const typename Pair<T>::type*>(p);
    return make_float2(to_f32(v.x), to_f32(v.y));
  }
}
template <typename T>
__device__ __forceinline__ void store_pair(T* p, float a, float b) {
  if constexpr (sizeof(T) == 4) {
    *reinterpret_cast<float2*>(p) = make_float2(a, b);
  } else {
    typename Pair<T>::type v;
    v.x = from_f32<T>(a);
    v.y = from_f32<T>(b);
    *reinterpret_cast<typename Pair<T>::type*>(p) = v;
  }
}

__device__ __forceinline__ float2 rotate(float2 x, float c, float s) {
  return make_float2(x.x * c - x.y * s, x.x * s + x.y * c);
}

// q/k [B,H,S,D]; `half_d` = D/2 pairs per vector, `pairs` rotated (rest copied).
template <typename T>
__global__ void rotary_kernel(const T* __restrict__ q, const T* __restrict__ k,
                              const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                              T* __restrict__ out_q, T* __restrict__ out_k, int64_t batch,
                              int64_t hq, int64_t hk, int64_t seq, int64_t half_d, int64_t pairs,
                              int64_t table_rows, int64_t start_pos,
                              const int64_t* __restrict__ positions, int64_t positions_numel,
                              unsigned* err) {
  DLI_PDL_ENTRY();
  const int64_t q_pairs = batch * hq * seq * half_d;
  const int64_t total = q_pairs + batch * hk * seq * half_d;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const bool is_q = i < q_pairs;
    const int64_t j = is_q ? i : i - q_pairs;
    const int64_t heads = is_q ? hq : hk;
    const int64_t pair = j % half_d;
    const int64_t vec = j / half_d;           // (b, h, s) flattened
    const int64_t s = vec % seq;
    const int64_t b = vec / (seq * heads);
    const T* src = (is_q ? q : k) + vec * 2 * half_d + 2 * pair;
    T* dst = (is_q ? out_q : out_k) + vec * 2 * half_d + 2 * pair;
    float2 x = load_pair(src);
    if (pair < pairs) {
      int64_t p;
      if (positions == nullptr) p = start_pos + s;
      else if (positions_numel == batch) p = positions[b] + s;
      else p = positions[b * seq + s];
      if (p >= 0 && p < table_rows) {
        x = rotate(x, cos_t[p * pairs + pair], sin_t[p * pairs + pair]);
      } else {
        set_device_error(err, kDevErrRotaryPosition);
      }
    }
    store_pair(dst, x.x, x.y);
  }
}

// qkv [B*S, (Hq + 2Hkv) * D]; q_out [B,S,Hq,D]; caches [B,Hkv,cap,D].
template <typename T>
__global__ void qkv_rotary_cache_kernel(const T* __restrict__ qkv, const float* __restrict__ cos_t,
                                        const float* __restrict__ sin_t,
                                        const int64_t* __restrict__ positions,
                                        T* __restrict__ q_out, T* __restrict__ cache_k,
                                        T* __restrict__ cache_v, int64_t batch, int64_t seq,
                                        int64_t hq, int64_t hkv, int64_t half_d, int64_t pairs,
                                        int64_t table_rows, int64_t cap, unsigned* err) {
  DLI_PDL_ENTRY();
  const int64_t heads = hq + 2 * hkv;
  const int64_t total = batch * seq * heads * half_d;
  const int64_t d = 2 * half_d;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t pair = i % half_d;
    const int64_t h = (i / half_d) % heads;
    const int64_t t = i / (half_d * heads);  // token b*S + s
    const int64_t b = t / seq, s = t - b * seq;
    const int64_t p = positions[b] + s;
    float2 x = load_pair(qkv + t * heads * d + h * d + 2 * pair);
    const bool in_table = p >= 0 && p < table_rows;
    if (h < hq + hkv && pair < pairs) {
      if (in_table) x = rotate(x, cos_t[p * pairs + pair], sin_t[p * pairs + pair]);
      else set_device_error(err, kDevErrRotaryPosition);
    }
    if (h < hq) {
      store_pair(q_out + (t * hq + h) * d + 2 * pair, x.x, x.y);
    } else if (p >= 0 && p < cap) {
      const bool is_k = h < hq + hkv;
      const int64_t kvh = is_k ? h - hq : h - hq - hkv;
      T* cache = is_k ? cache_k : cache_v;
      store_pair(cache + ((b * hkv + kvh) * cap + p) * d + 2 * pair, x.x, x.y);
    } else {
      set_device_error(err, kDevErrKvCapacity);
    }
  }
}

// Vectorised form of qkv_rotary_cache_kernel: one thread moves one 16-byte
// vector (V/2 pairs) per step, so index arithmetic and memory transactions are
// paid once per 16 bytes instead of once per pair. Needs D % V == 0 and
// 16-byte aligned qkv / q_out / caches (the host checks).
template <typename T>
__global__ void qkv_rotary_cache_vec_kernel(const T* __restrict__ qkv, const float* __restrict__ cos_t,
                                            const float* __restrict__ sin_t, const int64_t* __restrict__ positions,
                                            T* __restrict__ q_out, T* __restrict__ cache_k, T* __restrict__ cache_v,
                                            int64_t batch, int64_t seq, int64_t hq, int64_t hkv, int64_t d,
                                            int64_t pairs, int64_t table_rows, int64_t cap, unsigned* err) {
  DLI_PDL_ENTRY();
  constexpr int V = Vec16<T>::N;
  const int64_t heads = hq + 2 * hkv;
  const int64_t vpr = d / V;  // vectors per head row
  const int64_t total = batch * seq * heads * vpr;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t vi = i % vpr;
    const int64_t th = i / vpr;  // token * heads + head
    const int64_t h = th % heads;
    const int64_t t = th / heads;  // token b*S + s
    const int64_t b = t / seq, s = t - b * seq;
    const int64_t p = positions[b] + s;
    Vec16<T> x = load16(qkv + th * d + vi * V);
    if (h < hq + hkv) {
      const bool in_table = p >= 0 && p < table_rows;
#pragma unroll
      for (int j = 0; j < V / 2; ++j) {
        const int64_t pair = vi * (V / 2) + j;
        if (pair < pairs) {
          if (in_table) {
            const float c = cos_t[p * pairs + pair], sn = sin_t[p * pairs + pair];
            const float a = to_f32(x.e[2 * j]), bb = to_f32(x.e[2 * j + 1]);
            x.e[2 * j] = from_f32<T>(a * c - bb * sn);
            x.e[2 * j + 1] = from_f32<T>(a * sn + bb * c);
          } else {
            set_device_error(err, kDevErrRotaryPosition);
          }
        }
      }
    }
    if (h < hq) {
      store16(q_out + (t * hq + h) * d + vi * V, x);
    } else if (p >= 0 && p < cap) {
      const bool is_k = h < hq + hkv;
      const int64_t kvh = is_k ? h - hq : h - hq - hkv;
      store16((is_k ? cache_k : cache_v) + ((b * hkv + kvh) * cap + p) * d + vi * V, x);
    } else {
      set_device_error(err, kDevErrKvCapacity);
    }
  }
}

inline unsigned grid_for(int64_t n) {
  return static_cast<unsigned>(std::min<int64_t>(ceil_div(std::max<int64_t>(n, 1), 256), sm_count() * 16));
}

}  // namespace
}  // namespace dli_sm100

using namespace dli_sm100;

extern "C" dli_status dli_sm100_rotary_embedding(const void* q, const void* k, const float* cos_table,
                                                 const float* sin_table, void* out_q, void* out_k,
                                                 int64_t batch, int64_t q_heads, int64_t k_heads,
                                                 int64_t seq, int64_t head_dim, int64_t pairs,
                                                 int64_t table_rows, int64_t start_pos,
                                                 const int64_t* positions, int64_t positions_numel,
                                                 dli_dtype dtype, void* stream) {
  if (batch < 0 || q_heads < 0 || k_heads < 0 || seq < 0 || head_dim <= 0 || pairs < 0 ||
      table_rows < 0)
    return fail(DLI_ERR_INVALID_ARGUMENT, "rotary_embedding: bad sizes");
  if (head_dim % 2 != 0) return fail(DLI_ERR_INVALID_ARGUMENT, "rotary_embedding: odd head_dim");
  if (2 * pairs > head_dim)
    return fail(DLI_ERR_INVALID_ARGUMENT, "rotary_embedding: cos/sin width exceeds head_dim/2");
  if (positions != nullptr && positions_numel != batch && positions_numel != batch * seq)
    return fail(DLI_ERR_INVALID_ARGUMENT, "rotary_embedding: positions must have B or B*S entries");
  const int64_t total = batch * (q_heads + k_heads) * seq * (head_dim / 2);
  if (total == 0) return ok();
  unsigned* err = device_error_word();
  dli_status st = dispatch_float(dtype, "rotary_embedding", [&](auto tag) {
    using T = decltype(tag);
    launch_pdl(rotary_kernel<T>, grid_for(total), 256, 0, as_stream(stream), (const T*)q,
               (const T*)k, cos_table, sin_table, (T*)out_q, (T*)out_k, batch, q_heads, k_heads, seq,
               head_dim / 2, pairs, table_rows, start_pos, positions, positions_numel, err);
  });
  if (st != DLI_OK) return st;
  return check_launch("rotary_embedding");
}

extern "C" dli_status dli_sm100_qkv_rotary_cache(const void* qkv, const float* cos_table,
                                                 const float* sin_table, const int64_t* positions,
                                                 void* q_out, void* cache_k, void* cache_v,
                                                 int64_t batch, int64_t seq, int64_t q_heads,
                                                 int64_t kv_heads, int64_t head_dim, int64_t pairs,
                                                 int64_t table_rows, int64_t capacity,
                                                 dli_dtype dtype, void* stream) {
  if (batch < 0 || seq < 0 || q_heads <= 0 || kv_heads <= 0 || head_dim <= 0 || pairs < 0 ||
      table_rows < 0 || capacity <= 0)
    return fail(DLI_ERR_INVALID_ARGUMENT, "qkv_rotary_cache: bad sizes");
  if (head_dim % 2 != 0 || 2 * pairs > head_dim)
    return fail(DLI_ERR_INVALID_ARGUMENT, "qkv_rotary_cache: bad head_dim/pairs");
  if (positions == nullptr) return fail(DLI_ERR_INVALID_ARGUMENT, "qkv_rotary_cache: positions required");
  const int64_t total = batch * seq * (q_heads + 2 * kv_heads) * (head_dim / 2);
  if (total == 0) return ok();
  unsigned* err = device_error_word();
  dli_status st = dispatch_float(dtype, "qkv_rotary_cache", [&](auto tag) {
    using T = decltype(tag);
    constexpr int V = Vec16<T>::N;
    const bool vec = head_dim % V == 0 && aligned(qkv, 16) && aligned(q_out, 16) && aligned(cache_k, 16) &&
                     aligned(cache_v, 16);
    if (vec)
      launch_pdl(qkv_rotary_cache_vec_kernel<T>, grid_for(total / (V / 2)), 256, 0, as_stream(stream),
                 (const T*)qkv, cos_table, sin_table, positions, (T*)q_out, (T*)cache_k, (T*)cache_v, batch, seq,
                 q_heads, kv_heads, head_dim, pairs, table_rows, capacity, err);
    else
      launch_pdl(qkv_rotary_cache_kernel<T>, grid_for(total), 256, 0, as_stream(stream),
                 (const T*)qkv, cos_table, sin_table, positions, (T*)q_out, (T*)cache_k, (T*)cache_v,
                 batch, seq, q_heads, kv_heads, head_dim / 2, pairs, table_rows, capacity, err);
  });
  if (st != DLI_OK) return st;
  return check_launch("qkv_rotary_cache");
}
