// RMSNorm and fused residual-add + RMSNorm.
//
// One CTA per row (grid-stride over rows). Pass 1 streams the row with 16-byte
// loads and reduces sum(x^2) with warp shuffles + one smem exchange; pass 2
// re-reads the row (an L1/L2 hit: a row is at most a few tens of KB) and writes
// the normalised values. HBM traffic is therefore one read of x (plus delta for
// the fused form) and one write per output, the algorithmic minimum.
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
