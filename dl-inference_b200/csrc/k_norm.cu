// RMSNorm and fused residual-add + RMSNorm.
//
// One CTA per row (grid-stride over rows). Pass 1 streams the row with 16-byte
// loads and reduces sum(x^2) with warp shuffles + one smem exchange; pass 2
// re-reads the row (an L1/L2 hit: a row is at most a few tens of KB) and writes
// the normalised values. HBM traffic is therefore one read of x (plus delta for
// the fused form) and one write per output, the algorithmic minimum. The
// fp32-residual form keeps the row in registers instead (one 8-element vector
// per thread, rows up to 8192 wide), so nothing is read twice.
//
// Rounding follows the reference formula (python/dli_ops/aot/rms_norm/kernel.py:11-13)
// for fp32; for 16-bit types the normalised value is rounded to T before the
// weight multiply, as the source model's RMSNorm does (weight * x_hat.to(dtype)).
#include <algorithm>

#include "common.cuh"

namespace dli_sm100 {
namespace {

template <typename T, bool kFused>
__global__ void rms_norm_kernel(const T* x /* may alias residual_out */,
                                const T* __restrict__ delta, const T* __restrict__ w,
                                T* __restrict__ out, T* residual_out, int64_t rows, int64_t hidden,
                                float eps, bool vec) {
  DLI_PDL_ENTRY();
  __shared__ float scratch[32];
  constexpr int V = Vec16<T>::N;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const T* xr = x + r * hidden;
    const T* dr = kFused ? delta + r * hidden : nullptr;
    T* rr = kFused ? residual_out + r * hidden : nullptr;
    float ss = 0.f;
    if (vec) {
      for (int64_t c = threadIdx.x * V; c < hidden; c += blockDim.x * V) {
        Vec16<T> a = load16(xr + c);
        if constexpr (kFused) {
          Vec16<T> d = load16(dr + c);
#pragma unroll
          for (int j = 0; j < V; ++j) a.e[j] = from_f32<T>(to_f32(a.e[j]) + to_f32(d.e[j]));
          store16(rr + c, a);
        }
#pragma unroll
        for (int j = 0; j < V; ++j) {
          const float f = to_f32(a.e[j]);
          ss += f * f;
        }
      }
    } else {
      for (int64_t c = threadIdx.x; c < hidden; c += blockDim.x) {
        float f = to_f32(xr[c]);
        if constexpr (kFused) {
          const T s = from_f32<T>(f + to_f32(dr[c]));
          rr[c] = s;
          f = to_f32(s);
        }
        ss += f * f;
      }
    }
    const float total = block_sum(ss, scratch);
    const float inv = rsqrtf(total / static_cast<float>(hidden) + eps);
    const T* src = kFused ? rr : xr;
    T* dst = out + r * hidden;
    if (vec) {
      for (int64_t c = threadIdx.x * V; c < hidden; c += blockDim.x * V) {
        Vec16<T> a = load16(src + c), g = load16(w + c), o;
#pragma unroll
        for (int j = 0; j < V; ++j)
          o.e[j] = from_f32<T>(round_through<T>(to_f32(a.e[j]) * inv) * to_f32(g.e[j]));
        store16(dst + c, o);
      }
    } else {
      for (int64_t c = threadIdx.x; c < hidden; c += blockDim.x)
        dst[c] = from_f32<T>(round_through<T>(to_f32(src[c]) * inv) * to_f32(w[c]));
    }
    __syncthreads();  // scratch reuse by the next row
  }
}

// Residual add + RMSNorm with the residual stream kept in float32 while the
// delta, the weight and the normalised output are T (bf16/f16): the running
// sum of a deep model then carries no 16-bit rounding from layer to layer.
// s = residual + delta in fp32 (stored unrounded), normed = T(T(s * inv) * w).
template <typename T>
__global__ void add_rms_norm_res32_kernel(const float* residual /* may alias residual_out */,
                                          const T* __restrict__ delta, const T* __restrict__ w,
                                          T* __restrict__ out, float* residual_out, int64_t rows,
                                          int64_t hidden, float eps, bool vec) {
  DLI_PDL_ENTRY();
  __shared__ float scratch[32];
  constexpr int V = Vec16<T>::N;  // 8 elements: 16 bytes of T, 32 bytes of residual
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* xr = residual + r * hidden;
    const T* dr = delta + r * hidden;
    float* rr = residual_out + r * hidden;
    float ss = 0.f;
    if (vec) {
      for (int64_t c = threadIdx.x * V; c < hidden; c += blockDim.x * V) {
        const Vec16<T> d = load16(dr + c);
        float4 a0 = *reinterpret_cast<const float4*>(xr + c);
        float4 a1 = *reinterpret_cast<const float4*>(xr + c + 4);
        a0.x += to_f32(d.e[0]); a0.y += to_f32(d.e[1]); a0.z += to_f32(d.e[2]); a0.w += to_f32(d.e[3]);
        a1.x += to_f32(d.e[4]); a1.y += to_f32(d.e[5]); a1.z += to_f32(d.e[6]); a1.w += to_f32(d.e[7]);
        *reinterpret_cast<float4*>(rr + c) = a0;
        *reinterpret_cast<float4*>(rr + c + 4) = a1;
        ss += a0.x * a0.x + a0.y * a0.y + a0.z * a0.z + a0.w * a0.w;
        ss += a1.x * a1.x + a1.y * a1.y + a1.z * a1.z + a1.w * a1.w;
      }
    } else {
      for (int64_t c = threadIdx.x; c < hidden; c += blockDim.x) {
        const float f = xr[c] + to_f32(dr[c]);
        rr[c] = f;
        ss += f * f;
      }
    }
    const float total = block_sum(ss, scratch);
    const float inv = rsqrtf(total / static_cast<float>(hidden) + eps);
    T* dst = out + r * hidden;
    if (vec) {
      for (int64_t c = threadIdx.x * V; c < hidden; c += blockDim.x * V) {
        const float4 a0 = *reinterpret_cast<const float4*>(rr + c);
        const float4 a1 = *reinterpret_cast<const float4*>(rr + c + 4);
        const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const Vec16<T> g = load16(w + c);
        Vec16<T> o;
#pragma unroll
        for (int j = 0; j < V; ++j) o.e[j] = from_f32<T>(round_through<T>(a[j] * inv) * to_f32(g.e[j]));
        store16(dst + c, o);
      }
    } else {
      for (int64_t c = threadIdx.x; c < hidden; c += blockDim.x)
        dst[c] = from_f32<T>(round_through<T>(rr[c] * inv) * to_f32(w[c]));
    }
    __syncthreads();  // scratch reuse by the next row
  }
}

// The same with one 8-element vector per thread (blockDim >= hidden / 8): the
// row stays in registers between the sum of squares and the normalisation, so
// residual, delta and weight are read once, in a single round trip, and the
// second pass over the stored residual is gone. Same formula as above; the
// squares are summed over another thread partition.
template <typename T>
__global__ void add_rms_norm_res32_reg_kernel(const float* residual /* may alias residual_out */,
                                              const T* __restrict__ delta, const T* __restrict__ w,
                                              T* __restrict__ out, float* residual_out, int64_t rows,
                                              int64_t hidden, float eps) {
  DLI_PDL_ENTRY();
  __shared__ float scratch[32];
  const int64_t c = static_cast<int64_t>(threadIdx.x) * 8;
  const bool act = c < hidden;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    Vec16<T> g;
    float ss = 0.f;
    if (act) {
      const Vec16<T> d = load16(delta + r * hidden + c);
      const float4 a0 = *reinterpret_cast<const float4*>(residual + r * hidden + c);
      const float4 a1 = *reinterpret_cast<const float4*>(residual + r * hidden + c + 4);
      g = load16(w + c);
      a[0] = a0.x + to_f32(d.e[0]); a[1] = a0.y + to_f32(d.e[1]); a[2] = a0.z + to_f32(d.e[2]);
      a[3] = a0.w + to_f32(d.e[3]); a[4] = a1.x + to_f32(d.e[4]); a[5] = a1.y + to_f32(d.e[5]);
      a[6] = a1.z + to_f32(d.e[6]); a[7] = a1.w + to_f32(d.e[7]);
      *reinterpret_cast<float4*>(residual_out + r * hidden + c) = make_float4(a[0], a[1], a[2], a[3]);
      *reinterpret_cast<float4*>(residual_out + r * hidden + c + 4) = make_float4(a[4], a[5], a[6], a[7]);
      ss = a[0] * a[0] + a[1] * a[1] + a[2] * a[2] + a[3] * a[3];
      ss += a[4] * a[4] + a[5] * a[5] + a[6] * a[6] + a[7] * a[7];
    }
    const float total = block_sum(ss, scratch);
    const float inv = rsqrtf(total / static_cast<float>(hidden) + eps);
    if (act) {
      Vec16<T> o;
#pragma unroll
      for (int j = 0; j < 8; ++j) o.e[j] = from_f32<T>(round_through<T>(a[j] * inv) * to_f32(g.e[j]));
      store16(out + r * hidden + c, o);
    }
    __syncthreads();  // scratch reuse by the next row
  }
}

template <bool kFused>
dli_status launch(const void* x, const void* delta, const void* w, void* out, void* residual_out,
                  int64_t rows, int64_t hidden, float eps, dli_dtype dtype, void* stream,
                  const char* name) {
  if (rows < 0 || hidden <= 0) return fail(DLI_ERR_INVALID_ARGUMENT, std::string(name) + ": bad sizes");
  if (rows == 0) return ok();
  if (!x || !w || !out || (kFused && (!delta || !residual_out)))
    return fail(DLI_ERR_INVALID_ARGUMENT, std::string(name) + ": null pointer");
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(rows, sm_count() * 16));
  dli_status st = dispatch_float(dtype, name, [&](auto tag) {
    using T = decltype(tag);
    constexpr int V = Vec16<T>::N;
    bool vec = hidden % V == 0 && aligned(x, 16) && aligned(w, 16) && aligned(out, 16);
    if (kFused) vec = vec && aligned(delta, 16) && aligned(residual_out, 16);
    const int64_t lanes = vec ? hidden / V : hidden;
    const int threads = lanes >= 512 ? 512 : (lanes >= 256 ? 256 : (lanes >= 128 ? 128 : 32));
    launch_pdl(rms_norm_kernel<T, kFused>, grid, threads, 0, as_stream(stream), (const T*)x,
               (const T*)delta, (const T*)w, (T*)out, (T*)residual_out, rows, hidden, eps, vec);
  });
  if (st != DLI_OK) return st;
  return check_launch(name);
}

}  // namespace
}  // namespace dli_sm100

using namespace dli_sm100;

extern "C" dli_status dli_sm100_rms_norm(const void* x, const void* w, void* out, int64_t rows,
                                         int64_t hidden, float eps, dli_dtype dtype, void* stream) {
  return launch<false>(x, nullptr, w, out, nullptr, rows, hidden, eps, dtype, stream, "rms_norm");
}

extern "C" dli_status dli_sm100_add_rms_norm(const void* residual, const void* delta, const void* w,
                                             void* normed, void* residual_out, int64_t rows,
                                             int64_t hidden, float eps, dli_dtype dtype,
                                             void* stream) {
  return launch<true>(residual, delta, w, normed, residual_out, rows, hidden, eps, dtype, stream,
                      "add_rms_norm");
}

extern "C" dli_status dli_sm100_add_rms_norm_ex(const void* residual, const void* delta, const void* w,
                                                void* normed, void* residual_out, int64_t rows,
                                                int64_t hidden, float eps, dli_dtype dtype,
                                                dli_dtype residual_dtype, void* stream) {
  const char* name = "add_rms_norm_ex";
  if (residual_dtype == dtype)
    return dli_sm100_add_rms_norm(residual, delta, w, normed, residual_out, rows, hidden, eps, dtype, stream);
  if (residual_dtype != DLI_DTYPE_F32 || (dtype != DLI_DTYPE_BF16 && dtype != DLI_DTYPE_F16))
    return fail(DLI_ERR_UNSUPPORTED, std::string(name) + ": a float32 residual with bfloat16/float16 tensors");
  if (rows < 0 || hidden <= 0) return fail(DLI_ERR_INVALID_ARGUMENT, std::string(name) + ": bad sizes");
  if (rows == 0) return ok();
  if (!residual || !delta || !w || !normed || !residual_out)
    return fail(DLI_ERR_INVALID_ARGUMENT, std::string(name) + ": null pointer");
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(rows, sm_count() * 16));
  const bool vec = hidden % 8 == 0 && aligned(residual, 32) && aligned(residual_out, 32) && aligned(delta, 16) &&
                   aligned(w, 16) && aligned(normed, 16);
  const int64_t lanes = vec ? hidden / 8 : hidden;
  if (vec && lanes <= 1024) {  // the whole row in registers, one vector per thread
    const int threads = static_cast<int>((lanes + 31) / 32 * 32);
    if (dtype == DLI_DTYPE_BF16)
      launch_pdl(add_rms_norm_res32_reg_kernel<__nv_bfloat16>, grid, threads, 0, as_stream(stream),
                 static_cast<const float*>(residual), static_cast<const __nv_bfloat16*>(delta),
                 static_cast<const __nv_bfloat16*>(w), static_cast<__nv_bfloat16*>(normed),
                 static_cast<float*>(residual_out), rows, hidden, eps);
    else
      launch_pdl(add_rms_norm_res32_reg_kernel<__half>, grid, threads, 0, as_stream(stream),
                 static_cast<const float*>(residual), static_cast<const __half*>(delta),
                 static_cast<const __half*>(w), static_cast<__half*>(normed), static_cast<float*>(residual_out),
                 rows, hidden, eps);
    return check_launch(name);
  }
  const int threads = lanes >= 512 ? 512 : (lanes >= 256 ? 256 : (lanes >= 128 ? 128 : 32));
  if (dtype == DLI_DTYPE_BF16)
    launch_pdl(add_rms_norm_res32_kernel<__nv_bfloat16>, grid, threads, 0, as_stream(stream),
               static_cast<const float*>(residual), static_cast<const __nv_bfloat16*>(delta),
               static_cast<const __nv_bfloat16*>(w), static_cast<__nv_bfloat16*>(normed),
               static_cast<float*>(residual_out), rows, hidden, eps, vec);
  else
    launch_pdl(add_rms_norm_res32_kernel<__half>, grid, threads, 0, as_stream(stream),
               static_cast<const float*>(residual), static_cast<const __half*>(delta), static_cast<const __half*>(w),
               static_cast<__half*>(normed), static_cast<float*>(residual_out), rows, hidden, eps, vec);
  return check_launch(name);
}
