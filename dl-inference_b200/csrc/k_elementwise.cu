// Bandwidth kernels: broadcast add/mul, activations, SwiGLU, embedding gather,
// transpose, pooling, batch norm, softmax, argmax, token select, casts and the
// KV-cache append. All use 16-byte vector accesses where shape and alignment
// allow, fp32 arithmetic, grid-stride loops sized to the SM count, and
// programmatic dependent launch (pdl_wait before the first global access).
#include <algorithm>
#include <cfloat>

#include "common.cuh"
#include "tcgen05.cuh"

namespace dli_sm100 {
namespace {

constexpr int kThreads = 256;

inline unsigned grid_for(int64_t work_items, int threads = kThreads) {
  const int64_t blocks = ceil_div(std::max<int64_t>(work_items, 1), threads);
  const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
  return static_cast<unsigned>(std::min(blocks, cap));
}

// ---- broadcast binary ------------------------------------------------------
// out[i] = op(a[i], b[i mod width])  (python/dli_ops/aot/add/kernel.py:8-11)
template <int OP>
__device__ __forceinline__ float binop(float x, float y) {
  return OP == 0 ? x + y : x * y;
}

template <typename T, int OP>
__global__ void broadcast_vec_kernel(const T* __restrict__ a, const T* __restrict__ b,
                                     T* __restrict__ out, int64_t nvec, int64_t width) {
  DLI_PDL_ENTRY();
  constexpr int V = Vec16<T>::N;
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < nvec;
       v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = v * V;
    Vec16<T> x = load16(a + i);
    Vec16<T> y = load16(b + (i % width));
    Vec16<T> r;
#pragma unroll
    for (int j = 0; j < V; ++j) r.e[j] = from_f32<T>(binop<OP>(to_f32(x.e[j]), to_f32(y.e[j])));
    store16(out + i, r);
  }
}

template <typename T, int OP>
__global__ void broadcast_scalar_kernel(const T* __restrict__ a, const T* __restrict__ b,
                                        T* __restrict__ out, int64_t total, int64_t width) {
  DLI_PDL_ENTRY();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    out[i] = from_f32<T>(binop<OP>(to_f32(a[i]), to_f32(b[i % width])));
  }
}

template <int OP>
dli_status broadcast(const void* a, const void* b, void* out, int64_t total, int64_t width,
                     dli_dtype dtype, void* stream, const char* name) {
  if (total < 0 || width <= 0) return fail(DLI_ERR_INVALID_ARGUMENT, std::string(name) + ": bad sizes");
  if (total == 0) return ok();
  if (!a || !b || !out) return fail(DLI_ERR_INVALID_ARGUMENT, std::string(name) + ": null pointer");
  dli_status st = dispatch_float(dtype, name, [&](auto tag) {
    using T = decltype(tag);
    constexpr int V = Vec16<T>::N;
    const bool vec = total % V == 0 && width % V == 0 && aligned(a, 16) && aligned(b, 16) && aligned(out, 16);
    if (vec) {
      const int64_t nvec = total / V;
      launch_pdl(broadcast_vec_kernel<T, OP>, grid_for(nvec), kThreads, 0, as_stream(stream),
                 (const T*)a, (const T*)b, (T*)out, nvec, width);
    } else {
      launch_pdl(broadcast_scalar_kernel<T, OP>, grid_for(total), kThreads, 0, as_stream(stream),
                 (const T*)a, (const T*)b, (T*)out, total, width);
    }
  });
  if (st != DLI_OK) return st;
  return check_launch(name);
}

// ---- unary activations -------------------------------------------------------
// silu: x / (1 + exp(-x)) (python/dli_ops/aot/silu/kernel.py:10); relu: max(x, 0).
template <int ACT>
__device__ __forceinline__ float act(float x) {
  return ACT == 0 ? x / (1.0f + expf(-x)) : fmaxf(x, 0.0f);
}

template <typename T, int ACT>
__global__ void unary_kernel(const T* __restrict__ x, T* __restrict__ out, int64_t total) {
  DLI_PDL_ENTRY();
  constexpr int V = Vec16<T>::N;
  const int64_t nvec = total / V;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  for (int64_t v = tid; v < nvec; v += stride) {
    Vec16<T> a = load16(x + v * V), r;
#pragma unroll
    for (int j = 0; j < V; ++j) r.e[j] = from_f32<T>(act<ACT>(to_f32(a.e[j])));
    store16(out + v * V, r);
  }
  for (int64_t i = nvec * V + tid; i < total; i += stride) out[i] = from_f32<T>(act<ACT>(to_f32(x[i])));
}

template <typename T, int ACT>
__global__ void unary_scalar_kernel(const T* __restrict__ x, T* __restrict__ out, int64_t total) {
  DLI_PDL_ENTRY();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = from_f32<T>(act<ACT>(to_f32(x[i])));
}

template <int ACT>
dli_status unary(const void* x, void* out, int64_t total, dli_dtype dtype, void* stream,
                 const char* name) {
  if (total < 0) return fail(DLI_ERR_INVALID_ARGUMENT, std::string(name) + ": bad sizes");
  if (total == 0) return ok();
  if (!x || !out) return fail(DLI_ERR_INVALID_ARGUMENT, std::string(name) + ": null pointer");
  dli_status st = dispatch_float(dtype, name, [&](auto tag) {
    using T = decltype(tag);
    if (aligned(x, 16) && aligned(out, 16))
      launch_pdl(unary_kernel<T, ACT>, grid_for(ceil_div(total, Vec16<T>::N)), kThreads, 0,
                 as_stream(stream), (const T*)x, (T*)out, total);
    else
      launch_pdl(unary_scalar_kernel<T, ACT>, grid_for(total), kThreads, 0, as_stream(stream),
                 (const T*)x, (T*)out, total);
  });
  if (st != DLI_OK) return st;
  return check_launch(name);
}

// ---- SwiGLU ----------------------------------------------------------------
// out[r, j] = silu(g[r, j]) * u[r, j] with g = gate_up[r, 0:W], u = gate_up[r, W:2W].
// The product is rounded like two separate graph nodes would: silu output is
// rounded to T before the multiply (python/dli_export/export.py:414-415).
template <typename T>
__global__ void silu_mul_vec_kernel(const T* __restrict__ gu, T* __restrict__ out, int64_t rows,
                                    int64_t width) {
  DLI_PDL_ENTRY();
  constexpr int V = Vec16<T>::N;
  const int64_t per_row = width / V;
  const int64_t total = rows * per_row;
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < total;
       v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = v / per_row, c = (v - r * per_row) * V;
    Vec16<T> g = load16(gu + r * 2 * width + c);
    Vec16<T> u = load16(gu + r * 2 * width + width + c);
    Vec16<T> o;
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const float s = round_through<T>(act<0>(to_f32(g.e[j])));
      o.e[j] = from_f32<T>(s * to_f32(u.e[j]));
    }
    store16(out + r * width + c, o);
  }
}

template <typename T>
__global__ void silu_mul_scalar_kernel(const T* __restrict__ gu, T* __restrict__ out, int64_t rows,
                                       int64_t width) {
  DLI_PDL_ENTRY();
  const int64_t total = rows * width;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / width, c = i - r * width;
    const float s = round_through<T>(act<0>(to_f32(gu[r * 2 * width + c])));
    out[i] = from_f32<T>(s * to_f32(gu[r * 2 * width + width + c]));
  }
}

// ---- embedding ---------------------------------------------------------------
// out[t, :] = table[ids[t], :] (python/dli_ops/aot/embedding/kernel.py:13-23).
template <typename T, typename I>
__global__ void embedding_kernel(const I* __restrict__ ids, const T* __restrict__ table,
                                 T* __restrict__ out, int64_t total, int64_t hidden, int64_t vocab,
                                 bool vec, unsigned* err) {
  DLI_PDL_ENTRY();
  constexpr int V = Vec16<T>::N;
  for (int64_t t = blockIdx.x; t < total; t += gridDim.x) {
    const int64_t id = static_cast<int64_t>(ids[t]);
    const bool valid = id >= 0 && id < vocab;
    if (!valid && threadIdx.x == 0) set_device_error(err, kDevErrEmbeddingIndex);
    T* dst = out + t * hidden;
    const T* src = table + (valid ? id : 0) * hidden;
    if (vec) {
      for (int64_t c = threadIdx.x * V; c < hidden; c += blockDim.x * V) {
        Vec16<T> v;
        if (valid) v = load16(src + c); else v.raw = make_uint4(0, 0, 0, 0);
        store16(dst + c, v);
      }
    } else {
      for (int64_t c = threadIdx.x; c < hidden; c += blockDim.x)
        dst[c] = valid ? src[c] : from_f32<T>(0.f);
    }
  }
}

// ---- transpose ----------------------------------------------------------------
// out[c, r] = x[r, c] (python/dli_ops/aot/transpose/kernel.py:5-20), 32x32 smem tiles.
template <typename T>
__global__ void transpose_kernel(const T* __restrict__ x, T* __restrict__ out, int64_t rows,
                                 int64_t cols) {
  DLI_PDL_ENTRY();
  __shared__ T tile[32][33];
  const int64_t r0 = (int64_t)blockIdx.y * 32, c0 = (int64_t)blockIdx.x * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t r = r0 + i, c = c0 + threadIdx.x;
    if (r < rows && c < cols) tile[i][threadIdx.x] = x[r * cols + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t c = c0 + i, r = r0 + threadIdx.x;
    if (r < rows && c < cols) out[c * rows + r] = tile[threadIdx.x][i];
  }
}

// ---- max pool -------------------------------------------------------------------
// python/dli_ops/aot/max_pool2d/kernel.py:24-41: out-of-range taps read -inf.
template <typename T>
__global__ void max_pool2d_kernel(const T* __restrict__ x, T* __restrict__ out, int64_t total,
                                  int h, int w, int oh, int ow, int kh, int kw, int sh, int sw,
                                  int ph, int pw) {
  DLI_PDL_ENTRY();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int ox = static_cast<int>(i % ow);
    const int oy = static_cast<int>((i / ow) % oh);
    const int64_t nc = i / ((int64_t)ow * oh);
    const T* plane = x + nc * h * w;
    float acc = -INFINITY;
    for (int dy = 0; dy < kh; ++dy) {
      const int iy = oy * sh + dy - ph;
      if (iy < 0 || iy >= h) continue;
      for (int dx = 0; dx < kw; ++dx) {
        const int ix = ox * sw + dx - pw;
        if (ix < 0 || ix >= w) continue;
        acc = fmaxf(acc, to_f32(plane[(int64_t)iy * w + ix]));
      }
    }
    out[i] = from_f32<T>(acc);
  }
}

// ---- batch norm (inference) -----------------------------------------------------
// python/dli_ops/aot/batch_norm2d/kernel.py:19-28.
template <typename T>
__global__ void batch_norm2d_kernel(const T* __restrict__ x, const T* __restrict__ weight,
                                    const T* __restrict__ bias, const T* __restrict__ mean,
                                    const T* __restrict__ var, T* __restrict__ out, int64_t total,
                                    int64_t channels, int64_t spatial, float eps) {
  DLI_PDL_ENTRY();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t ch = (i / spatial) % channels;
    const float normalized = (to_f32(x[i]) - to_f32(mean[ch])) * rsqrtf(to_f32(var[ch]) + eps);
    out[i] = from_f32<T>(normalized * to_f32(weight[ch]) + to_f32(bias[ch]));
  }
}

// ---- softmax ----------------------------------------------------------------------
// python/dli_ops/aot/softmax/kernel.py:8-14: subtract the row max, exp, normalise.
// One block per row; the row is read twice (max+sum pass, then write pass).
template <typename T>
__global__ void softmax_kernel(const T* __restrict__ x, T* __restrict__ out, int64_t rows,
                               int64_t width) {
  DLI_PDL_ENTRY();
  __shared__ float scratch[32];
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const T* row = x + r * width;
    float m = -INFINITY;
    for (int64_t c = threadIdx.x; c < width; c += blockDim.x) m = fmaxf(m, to_f32(row[c]));
    m = block_max(m, scratch);
    float s = 0.f;
    for (int64_t c = threadIdx.x; c < width; c += blockDim.x) s += expf(to_f32(row[c]) - m);
    s = block_sum(s, scratch);
    const float inv = 1.0f / s;
    for (int64_t c = threadIdx.x; c < width; c += blockDim.x)
      out[r * width + c] = from_f32<T>(expf(to_f32(row[c]) - m) * inv);
  }
}

// ---- argmax -------------------------------------------------------------------------
// (best, best_i) over columns [begin, end) of a row, indices absolute; ties keep
// the lowest index. 16-byte loads, 4 in flight per thread, when the range
// starts 16-byte aligned; the scalar loop takes the tail.
template <typename T>
__device__ __forceinline__ void argmax_scan(const T* row, int64_t begin, int64_t end, float& best,
                                            int64_t& best_i) {
  constexpr int V = Vec16<T>::N;
  const T* base = row + begin;
  const int64_t len = end - begin;
  const bool vec = (reinterpret_cast<uintptr_t>(base) & 15) == 0;
  const int64_t nvec = vec ? len / V : 0;
  int64_t v0 = threadIdx.x;
  for (; v0 + 3 * (int64_t)blockDim.x < nvec; v0 += 4 * (int64_t)blockDim.x) {
    Vec16<T> pk[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) pk[u] = load16(base + (v0 + u * (int64_t)blockDim.x) * V);
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int j = 0; j < V; ++j) {
        const float v = to_f32(pk[u].e[j]);
        const int64_t c = begin + (v0 + u * (int64_t)blockDim.x) * V + j;
        if (v > best || (v == best && c < best_i)) { best = v; best_i = c; }
      }
  }
  for (; v0 < nvec; v0 += blockDim.x) {
    const Vec16<T> pk = load16(base + v0 * V);
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const float v = to_f32(pk.e[j]);
      const int64_t c = begin + v0 * V + j;
      if (v > best || (v == best && c < best_i)) { best = v; best_i = c; }
    }
  }
  for (int64_t c = begin + nvec * V + threadIdx.x; c < end; c += blockDim.x) {
    const float v = to_f32(row[c]);
    if (v > best || (v == best && c < best_i)) { best = v; best_i = c; }
  }
}

// Block-wide (max, lowest index); the result is valid in thread 0.
__device__ __forceinline__ void block_argmax(float& best, int64_t& best_i, float* sval, int64_t* sidx,
                                             int64_t sentinel) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, best_i, o);
    if (ov > best || (ov == best && oi < best_i)) { best = ov; best_i = oi; }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) { sval[warp] = best; sidx[warp] = best_i; }
  __syncthreads();
  if (warp == 0) {
    best = lane < nw ? sval[lane] : -INFINITY;
    best_i = lane < nw ? sidx[lane] : sentinel;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int64_t oi = __shfl_xor_sync(0xffffffffu, best_i, o);
      if (ov > best || (ov == best && oi < best_i)) { best = ov; best_i = oi; }
    }
  }
}

template <typename T>
__global__ void argmax_kernel(const T* __restrict__ x, int64_t* __restrict__ out, int64_t rows,
                              int64_t width) {
  DLI_PDL_ENTRY();
  __shared__ float sval[32];
  __shared__ int64_t sidx[32];
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    float best = -INFINITY;
    int64_t best_i = width;  // sentinel larger than any index
    argmax_scan(x + r * width, 0, width, best, best_i);
    block_argmax(best, best_i, sval, sidx, width);
    if (threadIdx.x == 0) out[r] = best_i < width ? best_i : 0;
  }
}

// Few long rows (greedy decoding over a vocabulary): the kArgmaxSplit CTAs of a
// cluster scan consecutive chunks of one row (chunk lengths a multiple of 8
// elements, so every chunk of an aligned row starts 16-byte aligned), then rank
// 0 combines the chunks' (max, index) in rank order through distributed shared
// memory. Chunks are in index order, so ties keep the lowest index, as above.
constexpr int kArgmaxSplit = 8;

template <typename T>
__global__ void __launch_bounds__(512) argmax_cluster_kernel(const T* __restrict__ x, int64_t* __restrict__ out,
                                                             int64_t width, int64_t chunk) {
  DLI_PDL_ENTRY();
  __shared__ float sval[32];
  __shared__ int64_t sidx[32];
  __shared__ float cand_v;
  __shared__ int64_t cand_i;
  const int64_t r = blockIdx.x;
  const int rank = static_cast<int>(blockIdx.y);  // cluster rank (clusters span y)
  const int64_t begin = min(width, rank * chunk), end = min(width, begin + chunk);
  float best = -INFINITY;
  int64_t best_i = width;
  argmax_scan(x + r * width, begin, end, best, best_i);
  block_argmax(best, best_i, sval, sidx, width);
  if (threadIdx.x == 0) {
    cand_v = best;
    cand_i = best_i;
  }
  cluster_sync();
  if (rank == 0 && threadIdx.x == 0) {
    const uint32_t va = smem_u32(&cand_v), ia = smem_u32(&cand_i);
    for (int s2 = 1; s2 < kArgmaxSplit; ++s2) {
      float v;
      uint64_t i;
      asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(mapa_shared(va, s2)) : "memory");
      asm volatile("ld.shared::cluster.u64 %0, [%1];" : "=l"(i) : "r"(mapa_shared(ia, s2)) : "memory");
      const int64_t ii = static_cast<int64_t>(i);
      if (v > best || (v == best && ii < best_i)) { best = v; best_i = ii; }
    }
    out[r] = best_i < width ? best_i : 0;
  }
  cluster_sync();  // every rank's candidate stays readable until rank 0 is done
}

// ---- token select ---------------------------------------------------------------------
template <typename T>
__global__ void select_token_kernel(const T* __restrict__ x, T* __restrict__ out, int64_t batch,
                                    int64_t seq, int64_t width, int64_t index) {
  DLI_PDL_ENTRY();
  for (int64_t b = blockIdx.x; b < batch; b += gridDim.x) {
    const T* src = x + (b * seq + index) * width;
    for (int64_t c = threadIdx.x; c < width; c += blockDim.x) out[b * width + c] = src[c];
  }
}

// ---- cast -------------------------------------------------------------------------------
template <typename S, typename D>
__global__ void cast_kernel(const S* __restrict__ x, D* __restrict__ out, int64_t n) {
  DLI_PDL_ENTRY();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = from_f32<D>(to_f32(x[i]));
}

// ---- KV append ---------------------------------------------------------------------------
// Row-strided copy of k/v[B,H,S_new,D] into cache[B,H,cap,D] at rows old_len...
template <typename T>
__global__ void kv_append_kernel(T* __restrict__ ck, T* __restrict__ cv, const T* __restrict__ k,
                                 const T* __restrict__ v, int64_t bh, int64_t cap, int64_t old_len,
                                 int64_t new_len, int64_t d) {
  DLI_PDL_ENTRY();
  const int64_t total = bh * new_len * d;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = i % d;
    const int64_t s = (i / d) % new_len;
    const int64_t g = i / (d * new_len);
    const int64_t dst = (g * cap + old_len + s) * d + e;
    ck[dst] = k[i];
    cv[dst] = v[i];
  }
}

}  // namespace
}  // namespace dli_sm100

using namespace dli_sm100;

extern "C" dli_status dli_sm100_add(const void* a, const void* b, void* out, int64_t total,
                                    int64_t width, dli_dtype dtype, void* stream) {
  return broadcast<0>(a, b, out, total, width, dtype, stream, "add");
}

extern "C" dli_status dli_sm100_mul(const void* a, const void* b, void* out, int64_t total,
                                    int64_t width, dli_dtype dtype, void* stream) {
  return broadcast<1>(a, b, out, total, width, dtype, stream, "mul");
}

extern "C" dli_status dli_sm100_silu(const void* x, void* out, int64_t total, dli_dtype dtype,
                                     void* stream) {
  return unary<0>(x, out, total, dtype, stream, "silu");
}

extern "C" dli_status dli_sm100_relu(const void* x, void* out, int64_t total, dli_dtype dtype,
                                     void* stream) {
  return unary<1>(x, out, total, dtype, stream, "relu");
}

extern "C" dli_status dli_sm100_silu_mul(const void* gate_up, void* out, int64_t rows,
                                         int64_t width, dli_dtype dtype, void* stream) {
  if (rows < 0 || width <= 0) return fail(DLI_ERR_INVALID_ARGUMENT, "silu_mul: bad sizes");
  if (rows == 0) return ok();
  if (!gate_up || !out) return fail(DLI_ERR_INVALID_ARGUMENT, "silu_mul: null pointer");
  dli_status st = dispatch_float(dtype, "silu_mul", [&](auto tag) {
    using T = decltype(tag);
    constexpr int V = Vec16<T>::N;
    if (width % V == 0 && aligned(gate_up, 16) && aligned(out, 16))
      launch_pdl(silu_mul_vec_kernel<T>, grid_for(rows * width / V), kThreads, 0, as_stream(stream),
                 (const T*)gate_up, (T*)out, rows, width);
    else
      launch_pdl(silu_mul_scalar_kernel<T>, grid_for(rows * width), kThreads, 0, as_stream(stream),
                 (const T*)gate_up, (T*)out, rows, width);
  });
  if (st != DLI_OK) return st;
  return check_launch("silu_mul");
}

extern "C" dli_status dli_sm100_embedding(const void* ids, dli_dtype ids_dtype, const void* table,
                                          void* out, int64_t total, int64_t hidden, int64_t vocab,
                                          dli_dtype dtype, void* stream) {
  if (total < 0 || hidden <= 0 || vocab <= 0)
    return fail(DLI_ERR_INVALID_ARGUMENT, "embedding: bad sizes");
  if (ids_dtype != DLI_DTYPE_I64 && ids_dtype != DLI_DTYPE_I32)
    return fail(DLI_ERR_INVALID_ARGUMENT, "embedding ids must be int64 or int32");
  if (total == 0) return ok();
  if (!ids || !table || !out) return fail(DLI_ERR_INVALID_ARGUMENT, "embedding: null pointer");
  unsigned* err = device_error_word();
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(total, sm_count() * 32));
  dli_status st = dispatch_float(dtype, "embedding", [&](auto tag) {
    using T = decltype(tag);
    const bool vec = hidden % Vec16<T>::N == 0 && aligned(table, 16) && aligned(out, 16);
    const int threads = hidden >= 1024 ? 256 : 128;
    if (ids_dtype == DLI_DTYPE_I64)
      launch_pdl(embedding_kernel<T, int64_t>, grid, threads, 0, as_stream(stream),
                 (const int64_t*)ids, (const T*)table, (T*)out, total, hidden, vocab, vec, err);
    else
      launch_pdl(embedding_kernel<T, int32_t>, grid, threads, 0, as_stream(stream),
                 (const int32_t*)ids, (const T*)table, (T*)out, total, hidden, vocab, vec, err);
  });
  if (st != DLI_OK) return st;
  return check_launch("embedding");
}

extern "C" dli_status dli_sm100_transpose2d(const void* x, void* out, int64_t rows, int64_t cols,
                                            dli_dtype dtype, void* stream) {
  if (rows < 0 || cols < 0) return fail(DLI_ERR_INVALID_ARGUMENT, "transpose: bad sizes");
  if (rows == 0 || cols == 0) return ok();
  if (ceil_div(rows, 32) > 65535) return fail(DLI_ERR_UNSUPPORTED, "transpose: too many rows");
  dim3 grid(static_cast<unsigned>(ceil_div(cols, 32)), static_cast<unsigned>(ceil_div(rows, 32)));
  dim3 block(32, 8);
  dli_status st = dispatch_float(dtype, "transpose", [&](auto tag) {
    using T = decltype(tag);
    launch_pdl(transpose_kernel<T>, grid, block, 0, as_stream(stream), (const T*)x, (T*)out, rows, cols);
  });
  if (st != DLI_OK) return st;
  return check_launch("transpose");
}

extern "C" dli_status dli_sm100_max_pool2d(const void* x, void* out, int64_t n, int64_t c,
                                           int64_t h, int64_t w, int64_t kh, int64_t kw,
                                           int64_t stride_h, int64_t stride_w, int64_t pad_h,
                                           int64_t pad_w, dli_dtype dtype, void* stream) {
  if (n < 0 || c < 0 || h <= 0 || w <= 0 || kh <= 0 || kw <= 0 || stride_h <= 0 || stride_w <= 0 ||
      pad_h < 0 || pad_w < 0)
    return fail(DLI_ERR_INVALID_ARGUMENT, "max_pool2d: bad sizes");
  const int64_t oh = (h + 2 * pad_h - kh) / stride_h + 1;
  const int64_t ow = (w + 2 * pad_w - kw) / stride_w + 1;
  if (oh <= 0 || ow <= 0) return fail(DLI_ERR_INVALID_ARGUMENT, "max_pool2d: empty output");
  const int64_t total = n * c * oh * ow;
  if (total == 0) return ok();
  dli_status st = dispatch_float(dtype, "max_pool2d", [&](auto tag) {
    using T = decltype(tag);
    launch_pdl(max_pool2d_kernel<T>, grid_for(total), kThreads, 0, as_stream(stream), (const T*)x,
               (T*)out, total, (int)h, (int)w, (int)oh, (int)ow, (int)kh, (int)kw, (int)stride_h,
               (int)stride_w, (int)pad_h, (int)pad_w);
  });
  if (st != DLI_OK) return st;
  return check_launch("max_pool2d");
}

extern "C" dli_status dli_sm100_batch_norm2d(const void* x, const void* weight, const void* bias,
                                             const void* running_mean, const void* running_var,
                                             void* out, int64_t total, int64_t channels,
                                             int64_t spatial, float eps, dli_dtype dtype,
                                             void* stream) {
  if (total < 0 || channels <= 0 || spatial <= 0)
    return fail(DLI_ERR_INVALID_ARGUMENT, "batch_norm2d: bad sizes");
  if (total == 0) return ok();
  dli_status st = dispatch_float(dtype, "batch_norm2d", [&](auto tag) {
    using T = decltype(tag);
    launch_pdl(batch_norm2d_kernel<T>, grid_for(total), kThreads, 0, as_stream(stream), (const T*)x,
               (const T*)weight, (const T*)bias, (const T*)running_mean, (const T*)running_var,
               (T*)out, total, channels, spatial, eps);
  });
  if (st != DLI_OK) return st;
  return check_launch("batch_norm2d");
}

extern "C" dli_status dli_sm100_softmax(const void* x, void* out, int64_t rows, int64_t width,
                                        dli_dtype dtype, void* stream) {
  if (rows < 0 || width <= 0) return fail(DLI_ERR_INVALID_ARGUMENT, "softmax: bad sizes");
  if (rows == 0) return ok();
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(rows, sm_count() * 16));
  const int threads = width >= 1024 ? 256 : (width >= 128 ? 128 : 32);
  dli_status st = dispatch_float(dtype, "softmax", [&](auto tag) {
    using T = decltype(tag);
    launch_pdl(softmax_kernel<T>, grid, threads, 0, as_stream(stream), (const T*)x, (T*)out, rows, width);
  });
  if (st != DLI_OK) return st;
  return check_launch("softmax");
}

extern "C" dli_status dli_sm100_argmax(const void* x, int64_t* out_ids, int64_t rows, int64_t width,
                                       dli_dtype dtype, void* stream) {
  if (rows < 0 || width <= 0) return fail(DLI_ERR_INVALID_ARGUMENT, "argmax: bad sizes");
  if (rows == 0) return ok();
  // few long rows: a cluster of CTAs per row while the clusters fit one wave
  if (width >= 16 * 1024 && rows * kArgmaxSplit <= 2ll * sm_count() && rows <= 65535) {
    const int64_t chunk = ceil_div(ceil_div(width, kArgmaxSplit), 8) * 8;
    dli_status st = dispatch_float(dtype, "argmax", [&](auto tag) {
      using T = decltype(tag);
      launch_pdl_cluster(argmax_cluster_kernel<T>, dim3(static_cast<unsigned>(rows), kArgmaxSplit), dim3(512), 0,
                         as_stream(stream), kArgmaxSplit, (const T*)x, out_ids, width, chunk);
    });
    if (st != DLI_OK) return st;
    return check_launch("argmax");
  }
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(rows, sm_count() * 16));
  dli_status st = dispatch_float(dtype, "argmax", [&](auto tag) {
    using T = decltype(tag);
    launch_pdl(argmax_kernel<T>, grid, 1024, 0, as_stream(stream), (const T*)x, out_ids, rows, width);
  });
  if (st != DLI_OK) return st;
  return check_launch("argmax");
}

extern "C" dli_status dli_sm100_select_token(const void* x, void* out, int64_t batch, int64_t seq,
                                             int64_t width, int64_t index, dli_dtype dtype,
                                             void* stream) {
  if (batch < 0 || seq <= 0 || width <= 0 || index < 0 || index >= seq)
    return fail(DLI_ERR_INVALID_ARGUMENT, "select_token: bad sizes");
  if (batch == 0) return ok();
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(batch, 65535));
  dli_status st = dispatch_float(dtype, "select_token", [&](auto tag) {
    using T = decltype(tag);
    launch_pdl(select_token_kernel<T>, grid, 256, 0, as_stream(stream), (const T*)x, (T*)out, batch,
               seq, width, index);
  });
  if (st != DLI_OK) return st;
  return check_launch("select_token");
}

extern "C" dli_status dli_sm100_cast(const void* x, dli_dtype x_dtype, void* out,
                                     dli_dtype out_dtype, int64_t n, void* stream) {
  if (n < 0) return fail(DLI_ERR_INVALID_ARGUMENT, "cast: bad size");
  if (n == 0) return ok();
  dli_status inner = DLI_OK;
  dli_status st = dispatch_float(x_dtype, "cast", [&](auto stag) {
    using S = decltype(stag);
    inner = dispatch_float(out_dtype, "cast", [&](auto dtag) {
      using D = decltype(dtag);
      launch_pdl(cast_kernel<S, D>, grid_for(n), kThreads, 0, as_stream(stream), (const S*)x, (D*)out, n);
    });
  });
  if (st != DLI_OK) return st;
  if (inner != DLI_OK) return inner;
  return check_launch("cast");
}

extern "C" dli_status dli_sm100_kv_append(void* cache_k, void* cache_v, const void* k,
                                          const void* v, int64_t batch, int64_t heads,
                                          int64_t capacity, int64_t old_len, int64_t new_len,
                                          int64_t head_dim, dli_dtype dtype, void* stream) {
  if (batch < 0 || heads < 0 || capacity <= 0 || old_len < 0 || new_len < 0 || head_dim <= 0)
    return fail(DLI_ERR_INVALID_ARGUMENT, "kv_append: bad sizes");
  if (old_len + new_len > capacity)
    return fail(DLI_ERR_INVALID_ARGUMENT, "kv_append: cache capacity exceeded");
  const int64_t total = batch * heads * new_len * head_dim;
  if (total == 0) return ok();
  dli_status st = dispatch_float(dtype, "kv_append", [&](auto tag) {
    using T = decltype(tag);
    launch_pdl(kv_append_kernel<T>, grid_for(total), kThreads, 0, as_stream(stream), (T*)cache_k,
               (T*)cache_v, (const T*)k, (const T*)v, batch * heads, capacity, old_len, new_len,
               head_dim);
  });
  if (st != DLI_OK) return st;
  return check_launch("kv_append");
}
