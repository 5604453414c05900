// conv2d (NCHW, python/dli_ops/aot/conv2d/kernel.py:5-49 semantics: zero padding,
// stride, optional bias).
//
// bf16/f16: implicit GEMM on tcgen05 (run_conv_implicit_tcgen05): the patch
// tiles are gathered into shared memory inside the GEMM, no patch matrix is
// written. The weight [OC, C, KH, KW] is already a K-major [OC, K] operand,
// repacked into the workspace with K rounded up to Kp, a multiple of 8 (TMA row
// strides are 16-byte aligned), when K % 8 != 0. The epilogue scatters
// D[m, oc] straight to NCHW. DLI_SM100_CONV_IMPLICIT=0 selects the older form:
// an im2col kernel writes cols[M = N*OH*OW, Kp] and the plain GEMM reads it.
// f32: 3x3 kernels run the tiled kernel below (shared-memory input patches and
// weights, 16 output channels per thread); other sizes a direct convolution,
// one output per thread. Both exact fp32 FMA.
#include <algorithm>

#include "gemm.cuh"

namespace dli_sm100 {
namespace {

struct ConvShape {
  int64_t n, c, h, w, oc, kh, kw, sh, sw, ph, pw, oh, ow;
  __host__ __device__ int64_t k() const { return c * kh * kw; }
  __host__ __device__ int64_t kp() const { return (k() + 7) / 8 * 8; }
  __host__ __device__ int64_t m() const { return n * oh * ow; }
};

template <typename T>
__global__ void im2col_kernel(const T* __restrict__ x, T* __restrict__ cols, ConvShape s) {
  DLI_PDL_ENTRY();
  const int64_t kp = s.kp(), k = s.k();
  const int64_t total = s.m() * kp;
  const int64_t ohw = s.oh * s.ow;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t kk = i % kp, m = i / kp;
    T v = from_f32<T>(0.f);
    if (kk < k) {
      const int64_t img = m / ohw, pix = m - img * ohw;
      const int64_t oy = pix / s.ow, ox = pix - oy * s.ow;
      const int64_t ch = kk / (s.kh * s.kw), r = kk - ch * s.kh * s.kw;
      const int64_t ky = r / s.kw, kx = r - ky * s.kw;
      const int64_t iy = oy * s.sh + ky - s.ph, ix = ox * s.sw + kx - s.pw;
      if (iy >= 0 && iy < s.h && ix >= 0 && ix < s.w) v = x[((img * s.c + ch) * s.h + iy) * s.w + ix];
    }
    cols[i] = v;
  }
}

template <typename T>
__global__ void pad_weight_kernel(const T* __restrict__ w, T* __restrict__ wp, int64_t oc, int64_t k,
                                  int64_t kp) {
  DLI_PDL_ENTRY();
  const int64_t total = oc * kp;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t kk = i % kp, o = i / kp;
    wp[i] = kk < k ? w[o * k + kk] : from_f32<T>(0.f);
  }
}

template <typename T>
__global__ void conv_direct_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                   const T* __restrict__ bias, T* __restrict__ out, ConvShape s) {
  DLI_PDL_ENTRY();
  const int64_t total = s.n * s.oc * s.oh * s.ow;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t ox = i % s.ow, oy = (i / s.ow) % s.oh;
    const int64_t o = (i / (s.ow * s.oh)) % s.oc, img = i / (s.ow * s.oh * s.oc);
    float acc = bias ? to_f32(bias[o]) : 0.f;
    for (int64_t ch = 0; ch < s.c; ++ch) {
      const T* plane = x + (img * s.c + ch) * s.h * s.w;
      const T* wk = w + (o * s.c + ch) * s.kh * s.kw;
      for (int64_t ky = 0; ky < s.kh; ++ky) {
        const int64_t iy = oy * s.sh + ky - s.ph;
        if (iy < 0 || iy >= s.h) continue;
        for (int64_t kx = 0; kx < s.kw; ++kx) {
          const int64_t ix = ox * s.sw + kx - s.pw;
          if (ix < 0 || ix >= s.w) continue;
          acc = fmaf(to_f32(plane[iy * s.w + ix]), to_f32(wk[ky * s.kw + kx]), acc);
        }
      }
    }
    out[i] = from_f32<T>(acc);
  }
}

// fp32 3x3 convolution on CUDA cores, tiled: CTA = a 16x16 block of output
// pixels of one image x 16 output channels, 256 threads of one pixel and 16
// channel accumulators each. Input channels go through shared memory 8 at a
// time: the (15*stride + 3)^2 input patch (zero-padded at the borders) and the
// matching 8 x 9 x 16 weights, stored channel-fastest so one 16-byte shared
// load serves four accumulators. Exact fp32 FMA in (c, ky, kx) order.
constexpr int kConvTile = 16, kConvOcb = 16, kConvCb = 8;

__host__ __device__ inline int conv_patch(int64_t stride) { return static_cast<int>((kConvTile - 1) * stride + 3); }

__global__ void __launch_bounds__(256)
    conv3x3_f32_kernel(const float* __restrict__ x, const float* __restrict__ w, const float* __restrict__ bias,
                       float* __restrict__ out, ConvShape s, int tiles_x) {
  DLI_PDL_ENTRY();
  extern __shared__ __align__(16) float conv_smem[];
  const int ih = conv_patch(s.sh), iw = conv_patch(s.sw);
  float* wsm = conv_smem;                             // [kConvCb * 9][kConvOcb]
  float* patch = conv_smem + kConvCb * 9 * kConvOcb;  // [kConvCb][ih][iw]
  const int tid = threadIdx.x;
  const int py = tid / kConvTile, px = tid % kConvTile;
  const int ty = blockIdx.x / tiles_x, tx = blockIdx.x % tiles_x;
  const int oc0 = blockIdx.y * kConvOcb;
  const int64_t img = blockIdx.z;
  const int64_t oy = static_cast<int64_t>(ty) * kConvTile + py, ox = static_cast<int64_t>(tx) * kConvTile + px;
  const int64_t iy0 = static_cast<int64_t>(ty) * kConvTile * s.sh - s.ph;
  const int64_t ix0 = static_cast<int64_t>(tx) * kConvTile * s.sw - s.pw;
  float acc[kConvOcb];
#pragma unroll
  for (int o = 0; o < kConvOcb; ++o) acc[o] = (bias && oc0 + o < s.oc) ? bias[oc0 + o] : 0.f;
  const int plane = ih * iw;
  for (int64_t c0 = 0; c0 < s.c; c0 += kConvCb) {
    const int cb = static_cast<int>(s.c - c0 < kConvCb ? s.c - c0 : kConvCb);
    for (int i = tid; i < kConvCb * plane; i += 256) {
      const int cc = i / plane, rem = i - cc * plane;
      const int r = rem / iw, q = rem - r * iw;
      const int64_t iy = iy0 + r, ix = ix0 + q;
      float v = 0.f;
      if (cc < cb && iy >= 0 && iy < s.h && ix >= 0 && ix < s.w) v = x[((img * s.c + c0 + cc) * s.h + iy) * s.w + ix];
      patch[i] = v;
    }
    for (int i = tid; i < kConvCb * 9 * kConvOcb; i += 256) {
      const int o = i % kConvOcb, t = i / kConvOcb;
      const int cc = t / 9, kk = t - cc * 9;
      wsm[i] = (cc < cb && oc0 + o < s.oc) ? w[((static_cast<int64_t>(oc0) + o) * s.c + c0 + cc) * 9 + kk] : 0.f;
    }
    __syncthreads();
    for (int cc = 0; cc < cb; ++cc) {
#pragma unroll
      for (int ky = 0; ky < 3; ++ky) {
#pragma unroll
        for (int kx = 0; kx < 3; ++kx) {
          const float xv = patch[cc * plane + (py * static_cast<int>(s.sh) + ky) * iw + px * static_cast<int>(s.sw) + kx];
          const float4* wr = reinterpret_cast<const float4*>(wsm + (cc * 9 + ky * 3 + kx) * kConvOcb);
#pragma unroll
          for (int q = 0; q < kConvOcb / 4; ++q) {
            const float4 wv = wr[q];
            acc[4 * q] = fmaf(xv, wv.x, acc[4 * q]);
            acc[4 * q + 1] = fmaf(xv, wv.y, acc[4 * q + 1]);
            acc[4 * q + 2] = fmaf(xv, wv.z, acc[4 * q + 2]);
            acc[4 * q + 3] = fmaf(xv, wv.w, acc[4 * q + 3]);
          }
        }
      }
    }
    __syncthreads();
  }
  if (oy >= s.oh || ox >= s.ow) return;
#pragma unroll
  for (int o = 0; o < kConvOcb; ++o)
    if (oc0 + o < s.oc) out[((img * s.oc + oc0 + o) * s.oh + oy) * s.ow + ox] = acc[o];
}

inline unsigned grid_for(int64_t n) {
  return static_cast<unsigned>(std::min<int64_t>(ceil_div(std::max<int64_t>(n, 1), 256), sm_count() * 16));
}

inline size_t align256(size_t x) { return (x + 255) / 256 * 256; }

struct ConvWorkspace {
  size_t cols = 0, weight = 0, gemm = 0, total = 0;
  GemmPlan plan;
  bool tensor = false;  // a tcgen05 path serves the shape
  bool gather = false;  // the implicit (gathering) kernel; else im2col + GEMM
};

bool conv_implicit_enabled() {
  static const bool on = tuning_knob("CONV_IMPLICIT", 1) != 0;
  return on;
}

ConvWorkspace conv_workspace(const ConvShape& s, dli_dtype dtype) {
  ConvWorkspace ws;
  if (dtype != DLI_DTYPE_BF16 && dtype != DLI_DTYPE_F16) return ws;
  ws.plan = plan_tn_gemm(s.m(), s.oc, s.kp(), dtype, true);
  if (!ws.plan.tcgen05) return ws;
  ws.tensor = true;
  constexpr int64_t kIntMax = 0x7fffffff;
  ws.gather = conv_implicit_enabled() && s.n * s.c * s.h * s.w <= kIntMax && s.m() * s.oc <= kIntMax &&
              s.c * s.kh * s.kw <= kIntMax;
  ws.cols = ws.gather ? 0 : align256(static_cast<size_t>(s.m() * s.kp()) * 2);
  ws.weight = s.kp() != s.k() ? align256(static_cast<size_t>(s.oc * s.kp()) * 2) : 0;
  ws.gemm = align256(ws.plan.workspace);
  ws.total = ws.cols + ws.weight + ws.gemm;
  return ws;
}

dli_status make_shape(ConvShape& s, int64_t n, int64_t c, int64_t h, int64_t w, int64_t oc,
                      int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw) {
  if (n < 0 || c <= 0 || h <= 0 || w <= 0 || oc <= 0 || kh <= 0 || kw <= 0 || sh <= 0 || sw <= 0 ||
      ph < 0 || pw < 0)
    return fail(DLI_ERR_INVALID_ARGUMENT, "conv2d: bad sizes");
  s = ConvShape{n, c, h, w, oc, kh, kw, sh, sw, ph, pw, 0, 0};
  s.oh = (h + 2 * ph - kh) / sh + 1;
  s.ow = (w + 2 * pw - kw) / sw + 1;
  if (s.oh <= 0 || s.ow <= 0) return fail(DLI_ERR_INVALID_ARGUMENT, "conv2d: empty output");
  return DLI_OK;
}

}  // namespace
}  // namespace dli_sm100

using namespace dli_sm100;

extern "C" size_t dli_sm100_conv2d_workspace_size(int64_t n, int64_t c, int64_t h, int64_t w,
                                                  int64_t oc, int64_t kh, int64_t kw,
                                                  int64_t stride_h, int64_t stride_w,
                                                  int64_t pad_h, int64_t pad_w, dli_dtype dtype) {
  ConvShape s;
  if (make_shape(s, n, c, h, w, oc, kh, kw, stride_h, stride_w, pad_h, pad_w) != DLI_OK) return 0;
  if (s.m() == 0) return 0;
  return conv_workspace(s, dtype).total;
}

extern "C" dli_status dli_sm100_conv2d(const void* x, const void* weight, const void* bias,
                                       void* out, int64_t n, int64_t c, int64_t h, int64_t w,
                                       int64_t oc, int64_t kh, int64_t kw, int64_t stride_h,
                                       int64_t stride_w, int64_t pad_h, int64_t pad_w,
                                       dli_dtype dtype, void* workspace, size_t workspace_bytes,
                                       void* stream) {
  ConvShape s;
  dli_status st = make_shape(s, n, c, h, w, oc, kh, kw, stride_h, stride_w, pad_h, pad_w);
  if (st != DLI_OK) return st;
  if (!is_float_dtype(dtype)) return fail(DLI_ERR_INVALID_ARGUMENT, "conv2d expects a float dtype");
  if (s.m() == 0) return ok();
  if (!x || !weight || !out) return fail(DLI_ERR_INVALID_ARGUMENT, "conv2d: null pointer");
  cudaStream_t cs = as_stream(stream);
  const ConvWorkspace ws = conv_workspace(s, dtype);
  if (ws.tensor && ws.gather) {
    if (ws.total > 0 && (workspace == nullptr || workspace_bytes < ws.total))
      return fail(DLI_ERR_WORKSPACE, "conv2d: workspace too small (need " + std::to_string(ws.total) + " bytes)");
    const void* wk = weight;
    if (ws.weight) {
      st = dispatch_float(dtype, "conv2d", [&](auto tag) {
        using T = decltype(tag);
        launch_pdl(pad_weight_kernel<T>, grid_for(s.oc * s.kp()), 256, 0, cs, (const T*)weight, (T*)workspace,
                   s.oc, s.k(), s.kp());
      });
      if (st != DLI_OK) return st;
      st = check_launch("conv2d weight repack");
      if (st != DLI_OK) return st;
      wk = workspace;
    }
    const ConvGeom g{static_cast<int>(s.n), static_cast<int>(s.c), static_cast<int>(s.h), static_cast<int>(s.w),
                     static_cast<int>(s.oc), static_cast<int>(s.kh), static_cast<int>(s.kw), static_cast<int>(s.sh),
                     static_cast<int>(s.sw), static_cast<int>(s.ph), static_cast<int>(s.pw), static_cast<int>(s.oh),
                     static_cast<int>(s.ow)};
    return run_conv_implicit_tcgen05(x, wk, s.kp(), bias, out, g, dtype, cs, ws.weight == 0);
  }
  if (ws.tensor && s.m() * s.oc < (1ll << 31)) {
    if (workspace == nullptr || workspace_bytes < ws.total)
      return fail(DLI_ERR_WORKSPACE, "conv2d: workspace too small (need " + std::to_string(ws.total) + " bytes)");
    uint8_t* base = static_cast<uint8_t*>(workspace);
    void* cols = base;
    const void* wk = weight;
    st = dispatch_float(dtype, "conv2d", [&](auto tag) {
      using T = decltype(tag);
      launch_pdl(im2col_kernel<T>, grid_for(s.m() * s.kp()), 256, 0, cs, (const T*)x, (T*)cols, s);
      if (ws.weight) {
        launch_pdl(pad_weight_kernel<T>, grid_for(s.oc * s.kp()), 256, 0, cs, (const T*)weight,
                   (T*)(base + ws.cols), s.oc, s.k(), s.kp());
        wk = base + ws.cols;
      }
    });
    if (st != DLI_OK) return st;
    st = check_launch("conv2d im2col", ws.weight ? 2 : 1);
    if (st != DLI_OK) return st;
    return run_tn_gemm_tcgen05(cols, wk, bias, out, s.m(), s.oc, s.kp(), s.kp(), s.kp(), 0,
                               kEpiNchw, s.oh * s.ow, dtype, ws.plan, base + ws.cols + ws.weight,
                               ws.gemm, cs, false, ws.weight == 0);
  }
  static const bool tiled = tuning_knob("CONV_F32_TILED", 1) != 0;
  if (tiled && dtype == DLI_DTYPE_F32 && s.kh == 3 && s.kw == 3 && s.sh <= 2 && s.sw <= 2 && s.n <= 65535 &&
      ceil_div(s.oc, kConvOcb) <= 65535) {
    const int64_t tiles_x = ceil_div(s.ow, kConvTile), tiles_y = ceil_div(s.oh, kConvTile);
    if (tiles_x * tiles_y <= 0x7fffffff) {
      const int smem = (kConvCb * 9 * kConvOcb + kConvCb * conv_patch(s.sh) * conv_patch(s.sw)) * 4;
      // the limit is set once per device: at the largest patch (stride 2) so every launch fits
      constexpr int kMaxSmem = (kConvCb * 9 * kConvOcb + kConvCb * (15 * 2 + 3) * (15 * 2 + 3)) * 4;
      st = ensure_smem(reinterpret_cast<const void*>(conv3x3_f32_kernel), kMaxSmem, "conv2d fp32");
      if (st != DLI_OK) return st;
      launch_pdl(conv3x3_f32_kernel, dim3(static_cast<unsigned>(tiles_x * tiles_y),
                                          static_cast<unsigned>(ceil_div(s.oc, kConvOcb)), static_cast<unsigned>(s.n)),
                 dim3(256), smem, cs, static_cast<const float*>(x), static_cast<const float*>(weight),
                 static_cast<const float*>(bias), static_cast<float*>(out), s, static_cast<int>(tiles_x));
      return check_launch("conv2d fp32 3x3");
    }
  }
  st = dispatch_float(dtype, "conv2d", [&](auto tag) {
    using T = decltype(tag);
    launch_pdl(conv_direct_kernel<T>, grid_for(s.n * s.oc * s.oh * s.ow), 256, 0, cs, (const T*)x,
               (const T*)weight, (const T*)bias, (T*)out, s);
  });
  if (st != DLI_OK) return st;
  return check_launch("conv2d direct");
}
