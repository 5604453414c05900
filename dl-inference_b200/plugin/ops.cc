// libdli_sm100_ops.so — the operator plugin.
//
// Exports `extern "C" bool dli_register_operators(dli::OperatorRegistry*)`, the
// entry point the runtime resolves after dlopen (src/operator_registry.cc:23-41
// of yncxcw/dl-inference), and registers the reference's 16 operator strings
// (linear, matmul, conv2d, rms_norm, rotary_embedding, attention, embedding,
// add, mul, silu, relu, softmax, max_pool2d, batch_norm2d, reshape, transpose)
// plus additive fused operators for the batched Qwen2 graphs (add_rms_norm,
// silu_mul, qkv_rotary_cache, attention_kvcache, last_token, argmax, cast,
// all_reduce, all_reduce_add_rms_norm, tp_argmax, linear_silu_mul).
//
// Every operator validates arity/dtype/shape on the host and throws
// std::invalid_argument like the reference templates
// (python/dli_ops/aot/<op>/template.cc), allocates outputs and workspace from
// the ATen caching allocator, and launches through the C ABI of libdli_sm100.so
// on the run's stream (ExecutionContext::cuda_stream). There is no fallback:
// every tensor op runs a kernel of this project.
#include <ATen/ATen.h>
#include <cuda_runtime.h>

#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "dli/operator.h"
#include "dli/utils.h"
#include "dli_sm100.h"

#ifdef DLI_WITH_NCCL
#include <nccl.h>
#endif

namespace {

using dli::Attributes;
using dli::DType;
using dli::ExecutionContext;
using dli::Tensor;
using Inputs = std::vector<const Tensor*>;
using Outputs = std::vector<Tensor*>;

dli_dtype cdt(DType d) {
  switch (d) {
    case DType::Float32: return DLI_DTYPE_F32;
    case DType::Int64: return DLI_DTYPE_I64;
    case DType::BFloat16: return DLI_DTYPE_BF16;
    case DType::Float16: return DLI_DTYPE_F16;
    case DType::Int32: return DLI_DTYPE_I32;
  }
  throw std::invalid_argument("unknown dtype");
}

void check(dli_status st, const std::string& op) {
  if (st == DLI_OK) return;
  const std::string msg = op + ": " + dli_sm100_last_error();
  if (st == DLI_ERR_INVALID_ARGUMENT) throw std::invalid_argument(msg);
  throw std::runtime_error(msg);
}

void arity(const Inputs& in, const Outputs& out, std::size_t min_in, std::size_t max_in,
           std::size_t n_out, const std::string& op) {
  if (in.size() < min_in || in.size() > max_in || out.size() != n_out)
    throw std::invalid_argument(op + " arity");
}

at::Tensor workspace(std::size_t bytes, int device) {
  if (bytes == 0) return at::Tensor();
  return at::empty({static_cast<std::int64_t>(bytes)},
                   at::TensorOptions().dtype(at::kByte).device(at::kCUDA, device));
}
void* wsPtr(const at::Tensor& t) { return t.defined() ? t.data_ptr() : nullptr; }
std::size_t wsBytes(const at::Tensor& t) { return t.defined() ? static_cast<std::size_t>(t.numel()) : 0; }

void floatInputs(const Inputs& in, std::size_t n, const std::string& op) {
  dli::requireCudaInputs(in, op);
  for (std::size_t i = 0; i < n && i < in.size(); ++i) {
    dli::requireFloat(*in[i], op);
    if (i) dli::requireSameDtype(*in[0], *in[i], op);
  }
}

// (residual, delta, weight) of the add + RMSNorm operators: delta and weight
// share one float dtype; the residual has that dtype too, or is float32 (a
// residual stream kept in fp32 around a bfloat16/float16 model).
void residualInputs(const Inputs& in, const std::string& op) {
  dli::requireCudaInputs(in, op);
  for (const Tensor* t : in) dli::requireFloat(*t, op);
  dli::requireSameDtype(*in[1], *in[2], op);
  if (in[0]->dtype() != in[1]->dtype() &&
      !(in[0]->dtype() == DType::Float32 && (in[1]->dtype() == DType::BFloat16 || in[1]->dtype() == DType::Float16)))
    throw std::invalid_argument(op + ": residual must match delta or be float32 around a 16-bit delta");
}

template <typename Op>
void reg(dli::OperatorRegistry* r, const char* name) {
  r->registerFactory(name, [] { return std::make_unique<Op>(); });
}

// ---------------------------------------------------------------------------
// Reference operators
// ---------------------------------------------------------------------------

// linear: y = x . W^T (+ b); python/dli_ops/aot/linear/template.cc:14-34.
// Stream-K decode plans need a zero-initialised workspace that the kernel
// leaves zeroed; the operator (one instance per graph node in the engine's
// plan) keeps one such buffer and grows it when a larger plan needs more, so a
// decode step replayed from a CUDA graph allocates nothing.
class LinearOp final : public dli::Operator {
  mutable at::Tensor ws_;

 public:
  std::string type() const override { return "linear"; }
  void compute(const Inputs& in, const Outputs& out, const Attributes& attrs, ExecutionContext& ctx) const override {
    arity(in, out, 2, 3, 1, type());
    floatInputs(in, in.size(), type());
    const Tensor& x = *in[0];
    const Tensor& w = *in[1];
    if (w.rank() != 2) throw std::invalid_argument("linear weight must be 2-D");
    const std::int64_t k = x.shape().back(), n = w.dim(0);
    if (w.dim(1) != k) throw std::invalid_argument("linear weight K mismatch: " + dli::formatShape(w.shape()));
    if (in.size() == 3 && static_cast<std::int64_t>(in[2]->numel()) != n)
      throw std::invalid_argument("linear bias size mismatch");
    const std::int64_t m = dli::product(x.shape(), 0, x.rank() - 1);
    auto shape = x.shape();
    shape.back() = n;
    // Additive attribute: out_dtype = "float32" keeps the fp32 accumulator of a
    // bfloat16/float16 linear (LM-head logits ranked by argmax).
    const DType out_dt = attrs.contains("out_dtype")
                             ? dli::dtypeFromString(attrs.require<std::string>("out_dtype"))
                             : x.dtype();
    *out[0] = Tensor::cuda(out_dt, shape, x.deviceId());
    const dli_dtype dt = cdt(x.dtype());
    const std::size_t need = dli_sm100_linear_workspace_size(m, n, k, dt);
    if (need > wsBytes(ws_) || (ws_.defined() && ws_.device().index() != x.deviceId()))
      ws_ = at::zeros({static_cast<std::int64_t>(need)},
                      at::TensorOptions().dtype(at::kByte).device(at::kCUDA, x.deviceId()));
    if (out_dt != x.dtype()) {
      check(dli_sm100_linear_ex(dli::ptr(x), dli::ptr(w), in.size() == 3 ? dli::ptr(*in[2]) : nullptr,
                                out[0]->deviceData(), m, n, k, dt, cdt(out_dt), need ? wsPtr(ws_) : nullptr,
                                need ? wsBytes(ws_) : 0, ctx.cuda_stream),
            type());
      return;
    }
    check(dli_sm100_linear(dli::ptr(x), dli::ptr(w), in.size() == 3 ? dli::ptr(*in[2]) : nullptr,
                           out[0]->deviceData(), m, n, k, dt, need ? wsPtr(ws_) : nullptr,
                           need ? wsBytes(ws_) : 0, ctx.cuda_stream),
          type());
  }
};

// matmul: out[M,N] = a[M,K] . b[K,N]; python/dli_ops/aot/matmul/template.cc:14-30.
class MatmulOp final : public dli::Operator {
 public:
  std::string type() const override { return "matmul"; }
  void compute(const Inputs& in, const Outputs& out, const Attributes&, ExecutionContext& ctx) const override {
    arity(in, out, 2, 2, 1, type());
    floatInputs(in, 2, type());
    const Tensor& a = *in[0];
    const Tensor& b = *in[1];
    if (a.rank() != 2 || b.rank() != 2 || a.dim(1) != b.dim(0))
      throw std::invalid_argument("matmul expects [M,K] x [K,N]");
    *out[0] = Tensor::cuda(a.dtype(), {a.dim(0), b.dim(1)}, a.deviceId());
    check(dli_sm100_matmul(dli::ptr(a), dli::ptr(b), out[0]->deviceData(), a.dim(0), b.dim(1), a.dim(1),
                           cdt(a.dtype()), ctx.cuda_stream),
          type());
  }
};

// conv2d (NCHW); python/dli_ops/aot/conv2d/template.cc:1-37.
class Conv2dOp final : public dli::Operator {
 public:
  std::string type() const override { return "conv2d"; }
  void compute(const Inputs& in, const Outputs& out, const Attributes& attrs, ExecutionContext& ctx) const override {
    arity(in, out, 2, 3, 1, type());
    floatInputs(in, in.size(), type());
    const Tensor& x = *in[0];
    const Tensor& w = *in[1];
    if (x.rank() != 4 || w.rank() != 4 || w.dim(1) != x.dim(1))
      throw std::invalid_argument("conv2d expects NCHW input and [OC,C,KH,KW] weight");
    const auto stride = dli::attrInts(attrs, "stride", {1, 1});
    const auto pad = dli::attrInts(attrs, "padding", {0, 0});
    if (stride.size() != 2 || pad.size() != 2) throw std::invalid_argument("conv2d stride/padding must have 2 entries");
    const std::int64_t n = x.dim(0), c = x.dim(1), h = x.dim(2), wd = x.dim(3);
    const std::int64_t oc = w.dim(0), kh = w.dim(2), kw = w.dim(3);
    const std::int64_t oh = (h + 2 * pad[0] - kh) / stride[0] + 1;
    const std::int64_t ow = (wd + 2 * pad[1] - kw) / stride[1] + 1;
    *out[0] = Tensor::cuda(x.dtype(), {n, oc, oh, ow}, x.deviceId());
    const dli_dtype dt = cdt(x.dtype());
    at::Tensor ws = workspace(
        dli_sm100_conv2d_workspace_size(n, c, h, wd, oc, kh, kw, stride[0], stride[1], pad[0], pad[1], dt),
        x.deviceId());
    check(dli_sm100_conv2d(dli::ptr(x), dli::ptr(w), in.size() == 3 ? dli::ptr(*in[2]) : nullptr,
                           out[0]->deviceData(), n, c, h, wd, oc, kh, kw, stride[0], stride[1], pad[0],
                           pad[1], dt, wsPtr(ws), wsBytes(ws), ctx.cuda_stream),
          type());
  }
};

// rms_norm; python/dli_ops/aot/rms_norm/template.cc:12-28 (eps default 1e-6).
class RmsNormOp final : public dli::Operator {
 public:
  std::string type() const override { return "rms_norm"; }
  void compute(const Inputs& in, const Outputs& out, const Attributes& attrs, ExecutionContext& ctx) const override {
    arity(in, out, 2, 2, 1, type());
    floatInputs(in, 2, type());
    const Tensor& x = *in[0];
    const std::int64_t hidden = x.shape().back();
    if (static_cast<std::int64_t>(in[1]->numel()) != hidden) throw std::invalid_argument("rms_norm weight size mismatch");
    const float eps = static_cast<float>(dli::attrDouble(attrs, "eps", 1e-6));
    *out[0] = Tensor::cuda(x.dtype(), x.shape(), x.deviceId());
    check(dli_sm100_rms_norm(dli::ptr(x), dli::ptr(*in[1]), out[0]->deviceData(),
                             static_cast<std::int64_t>(x.numel()) / hidden, hidden, eps, cdt(x.dtype()),
                             ctx.cuda_stream),
          type());
  }
};

// rotary_embedding: (q, k, cos, sin[, positions]) -> (q', k'); interleaved pairs;
// python/dli_ops/aot/rotary/template.cc:1-28 (the reserved 5th input carries
// int64 positions: [B] start per sequence or [B,S] per token).
class RotaryOp final : public dli::Operator {
 public:
  std::string type() const override { return "rotary_embedding"; }
  void compute(const Inputs& in, const Outputs& out, const Attributes& attrs, ExecutionContext& ctx) const override {
    arity(in, out, 4, 5, 2, type());
    dli::requireCudaInputs(in, type());
    const Tensor& q = *in[0];
    const Tensor& k = *in[1];
    dli::requireFloat(q, type());
    dli::requireSameDtype(q, k, type());
    if (q.rank() != 4 || k.rank() != 4) throw std::invalid_argument("rotary_embedding expects [B,H,S,D] q and k");
    if (q.dim(0) != k.dim(0) || q.dim(2) != k.dim(2) || q.dim(3) != k.dim(3))
      throw std::invalid_argument("rotary_embedding q/k shape mismatch");
    const Tensor& cos = *in[2];
    const Tensor& sin = *in[3];
    if (cos.dtype() != DType::Float32 || sin.dtype() != DType::Float32 || cos.rank() != 2 ||
        cos.shape() != sin.shape())
      throw std::invalid_argument("rotary_embedding expects float32 cos/sin tables [max_pos, pairs]");
    const Tensor* pos = in.size() == 5 ? in[4] : nullptr;
    if (pos && pos->dtype() != DType::Int64) throw std::invalid_argument("rotary_embedding positions must be int64");
    const std::int64_t start = attrs.value_or<std::int64_t>("start_pos", 0);
    *out[0] = Tensor::cuda(q.dtype(), q.shape(), q.deviceId());
    *out[1] = Tensor::cuda(k.dtype(), k.shape(), k.deviceId());
    check(dli_sm100_rotary_embedding(dli::ptr(q), dli::ptr(k), static_cast<const float*>(dli::ptr(cos)),
                                     static_cast<const float*>(dli::ptr(sin)), out[0]->deviceData(),
                                     out[1]->deviceData(), q.dim(0), q.dim(1), k.dim(1), q.dim(2), q.dim(3),
                                     cos.dim(1), cos.dim(0), start,
                                     pos ? static_cast<const std::int64_t*>(dli::ptr(*pos)) : nullptr,
                                     pos ? static_cast<std::int64_t>(pos->numel()) : 0, cdt(q.dtype()),
                                     ctx.cuda_stream),
          type());
  }
};

// attention: (q[B,Hq,Sq,D], k[B,Hkv,Sk,D], v) -> out; attrs causal, kv_cache, scale.
// python/dli_ops/aot/attention/template.cc:1-49: with a non-empty kv_cache name
// the new k/v are appended to the named cache entry first and q attends to all
// cached rows.
class AttentionOp final : public dli::Operator {
 public:
  std::string type() const override { return "attention"; }
  void compute(const Inputs& in, const Outputs& out, const Attributes& attrs, ExecutionContext& ctx) const override {
    arity(in, out, 3, 3, 1, type());
    floatInputs(in, 3, type());
    const Tensor& q = *in[0];
    const Tensor* k = in[1];
    const Tensor* v = in[2];
    if (q.rank() != 4 || k->rank() != 4 || v->rank() != 4 || k->shape() != v->shape())
      throw std::invalid_argument("attention expects [B,H,S,D] q/k/v");
    std::int64_t seq_k = k->dim(2), capacity = k->dim(2);
    if (attrs.contains("kv_cache")) {
      const auto& name = attrs.require<std::string>("kv_cache");
      if (!name.empty()) {
        if (ctx.kv_cache == nullptr) throw std::invalid_argument("attention missing KV cache");
        ctx.kv_cache->append(name, *in[1], *in[2], ctx.cuda_stream);
        const dli::KVCacheEntry* e = ctx.kv_cache->get(name);
        k = &e->key;
        v = &e->value;
        seq_k = e->length;
        capacity = e->capacity();
      }
    }
    if (q.dim(0) != k->dim(0) || q.dim(3) != k->dim(3) || q.dim(1) % k->dim(1) != 0)
      throw std::invalid_argument("attention q/k shape mismatch");
    const bool causal = attrs.value_or<bool>("causal", false);
    const float scale = static_cast<float>(dli::attrDouble(attrs, "scale", 0.0));
    *out[0] = Tensor::cuda(q.dtype(), q.shape(), q.deviceId());
    const dli_dtype dt = cdt(q.dtype());
    at::Tensor ws = workspace(
        dli_sm100_attention_workspace_size(q.dim(0), q.dim(1), k->dim(1), q.dim(2), seq_k, q.dim(3), dt),
        q.deviceId());
    check(dli_sm100_attention(dli::ptr(q), dli::ptr(*k), dli::ptr(*v), out[0]->deviceData(), q.dim(0), q.dim(1),
                              k->dim(1), q.dim(2), seq_k, capacity, q.dim(3), causal ? 1 : 0, scale, dt,
                              wsPtr(ws), wsBytes(ws), ctx.cuda_stream),
          type());
  }
};

// embedding: out[..., :] = table[ids[...]]; python/dli_ops/aot/embedding/template.cc:12-31.
class EmbeddingOp final : public dli::Operator {
 public:
  std::string type() const override { return "embedding"; }
  void compute(const Inputs& in, const Outputs& out, const Attributes&, ExecutionContext& ctx) const override {
    arity(in, out, 2, 2, 1, type());
    dli::requireCudaInputs(in, type());
    const Tensor& ids = *in[0];
    const Tensor& table = *in[1];
    if (ids.dtype() != DType::Int64 && ids.dtype() != DType::Int32)
      throw std::invalid_argument("embedding ids must be int64");
    dli::requireFloat(table, type());
    if (table.rank() != 2) throw std::invalid_argument("embedding table must be 2-D");
    auto shape = ids.shape();
    shape.push_back(table.dim(1));
    *out[0] = Tensor::cuda(table.dtype(), shape, ids.deviceId());
    check(dli_sm100_embedding(dli::ptr(ids), cdt(ids.dtype()), dli::ptr(table), out[0]->deviceData(),
                              static_cast<std::int64_t>(ids.numel()), table.dim(1), table.dim(0),
                              cdt(table.dtype()), ctx.cuda_stream),
          type());
  }
};

// add / mul: out[i] = a[i] op b[i mod numel(b)]; python/dli_ops/aot/{add,mul}/template.cc.
template <int kMul>
class BinaryOp final : public dli::Operator {
 public:
  std::string type() const override { return kMul ? "mul" : "add"; }
  void compute(const Inputs& in, const Outputs& out, const Attributes&, ExecutionContext& ctx) const override {
    arity(in, out, 2, 2, 1, type());
    floatInputs(in, 2, type());
    const Tensor& a = *in[0];
    const Tensor& b = *in[1];
    if (b.numel() == 0 || a.numel() % b.numel() != 0)
      throw std::invalid_argument(type() + " broadcast requires numel(a) to be a multiple of numel(b)");
    *out[0] = Tensor::cuda(a.dtype(), a.shape(), a.deviceId());
    const auto fn = kMul ? dli_sm100_mul : dli_sm100_add;
    check(fn(dli::ptr(a), dli::ptr(b), out[0]->deviceData(), static_cast<std::int64_t>(a.numel()),
             static_cast<std::int64_t>(b.numel()), cdt(a.dtype()), ctx.cuda_stream),
          type());
  }
};

// silu / relu; python/dli_ops/aot/{silu,relu}/template.cc.
template <int kRelu>
class UnaryOp final : public dli::Operator {
 public:
  std::string type() const override { return kRelu ? "relu" : "silu"; }
  void compute(const Inputs& in, const Outputs& out, const Attributes&, ExecutionContext& ctx) const override {
    arity(in, out, 1, 1, 1, type());
    floatInputs(in, 1, type());
    const Tensor& x = *in[0];
    *out[0] = Tensor::cuda(x.dtype(), x.shape(), x.deviceId());
    const auto fn = kRelu ? dli_sm100_relu : dli_sm100_silu;
    check(fn(dli::ptr(x), out[0]->deviceData(), static_cast<std::int64_t>(x.numel()), cdt(x.dtype()),
             ctx.cuda_stream),
          type());
  }
};

// softmax over the last dim; python/dli_ops/aot/softmax/template.cc:20-37 (any width here).
class SoftmaxOp final : public dli::Operator {
 public:
  std::string type() const override { return "softmax"; }
  void compute(const Inputs& in, const Outputs& out, const Attributes&, ExecutionContext& ctx) const override {
    arity(in, out, 1, 1, 1, type());
    floatInputs(in, 1, type());
    const Tensor& x = *in[0];
    const std::int64_t width = x.shape().back();
    *out[0] = Tensor::cuda(x.dtype(), x.shape(), x.deviceId());
    check(dli_sm100_softmax(dli::ptr(x), out[0]->deviceData(), static_cast<std::int64_t>(x.numel()) / width,
                            width, cdt(x.dtype()), ctx.cuda_stream),
          type());
  }
};

// max_pool2d; python/dli_ops/aot/max_pool2d/template.cc:1-30 (stride defaults to kernel_size).
class MaxPool2dOp final : public dli::Operator {
 public:
  std::string type() const override { return "max_pool2d"; }
  void compute(const Inputs& in, const Outputs& out, const Attributes& attrs, ExecutionContext& ctx) const override {
    arity(in, out, 1, 1, 1, type());
    floatInputs(in, 1, type());
    const Tensor& x = *in[0];
    if (x.rank() != 4) throw std::invalid_argument("max_pool2d expects NCHW input");
    const auto ks = dli::attrInts(attrs, "kernel_size", {2, 2});
    const auto st = dli::attrInts(attrs, "stride", ks);
    const auto pad = dli::attrInts(attrs, "padding", {0, 0});
    if (ks.size() != 2 || st.size() != 2 || pad.size() != 2)
      throw std::invalid_argument("max_pool2d kernel_size/stride/padding must have 2 entries");
    const std::int64_t oh = (x.dim(2) + 2 * pad[0] - ks[0]) / st[0] + 1;
    const std::int64_t ow = (x.dim(3) + 2 * pad[1] - ks[1]) / st[1] + 1;
    *out[0] = Tensor::cuda(x.dtype(), {x.dim(0), x.dim(1), oh, ow}, x.deviceId());
    check(dli_sm100_max_pool2d(dli::ptr(x), out[0]->deviceData(), x.dim(0), x.dim(1), x.dim(2), x.dim(3), ks[0],
                               ks[1], st[0], st[1], pad[0], pad[1], cdt(x.dtype()), ctx.cuda_stream),
          type());
  }
};

// batch_norm2d (inference); python/dli_ops/aot/batch_norm2d/template.cc:1-33 (eps default 1e-5).
class BatchNorm2dOp final : public dli::Operator {
 public:
  std::string type() const override { return "batch_norm2d"; }
  void compute(const Inputs& in, const Outputs& out, const Attributes& attrs, ExecutionContext& ctx) const override {
    arity(in, out, 5, 5, 1, type());
    floatInputs(in, 5, type());
    const Tensor& x = *in[0];
    if (x.rank() != 4) throw std::invalid_argument("batch_norm2d expects NCHW input");
    for (std::size_t i = 1; i < 5; ++i)
      if (static_cast<std::int64_t>(in[i]->numel()) != x.dim(1))
        throw std::invalid_argument("batch_norm2d parameter size must match input channels");
    const float eps = static_cast<float>(dli::attrDouble(attrs, "eps", 1e-5));
    *out[0] = Tensor::cuda(x.dtype(), x.shape(), x.deviceId());
    check(dli_sm100_batch_norm2d(dli::ptr(x), dli::ptr(*in[1]), dli::ptr(*in[2]), dli::ptr(*in[3]),
                                 dli::ptr(*in[4]), out[0]->deviceData(), static_cast<std::int64_t>(x.numel()),
                                 x.dim(1), x.dim(2) * x.dim(3), eps, cdt(x.dtype()), ctx.cuda_stream),
          type());
  }
};

// reshape: a view; python/dli_ops/aot/reshape/template.cc:1-11.
class ReshapeOp final : public dli::Operator {
 public:
  std::string type() const override { return "reshape"; }
  void compute(const Inputs& in, const Outputs& out, const Attributes& attrs, ExecutionContext&) const override {
    arity(in, out, 1, 1, 1, type());
    dli::requireCudaInputs(in, type());
    *out[0] = in[0]->withShape(dli::reshapeShape(in[0]->shape(), attrs.require<std::vector<std::int64_t>>("shape")));
  }
};

// transpose: 2-D, perm [1,0]; python/dli_ops/aot/transpose/template.cc:1-20.
class TransposeOp final : public dli::Operator {
 public:
  std::string type() const override { return "transpose"; }
  void compute(const Inputs& in, const Outputs& out, const Attributes& attrs, ExecutionContext& ctx) const override {
    arity(in, out, 1, 1, 1, type());
    floatInputs(in, 1, type());
    const auto perm = attrs.require<std::vector<std::int64_t>>("perm");
    const Tensor& x = *in[0];
    if (x.rank() != 2 || perm != std::vector<std::int64_t>({1, 0}))
      throw std::invalid_argument("transpose supports 2D perm [1,0]");
    *out[0] = Tensor::cuda(x.dtype(), {x.dim(1), x.dim(0)}, x.deviceId());
    check(dli_sm100_transpose2d(dli::ptr(x), out[0]->deviceData(), x.dim(0), x.dim(1), cdt(x.dtype()),
                                ctx.cuda_stream),
          type());
  }
};

// ---------------------------------------------------------------------------
// Additive fused operators (batched Qwen2 graphs)
// ---------------------------------------------------------------------------

// add_rms_norm: (residual, delta, weight) -> (normed, residual + delta). normed
// has delta's dtype, the new residual the residual's (float32 when the graph
// keeps its residual stream in fp32).
class AddRmsNormOp final : public dli::Operator {
 public:
  std::string type() const override { return "add_rms_norm"; }
  void compute(const Inputs& in, const Outputs& out, const Attributes& attrs, ExecutionContext& ctx) const override {
    arity(in, out, 3, 3, 2, type());
    residualInputs(in, type());
    const Tensor& r = *in[0];
    const Tensor& d = *in[1];
    if (d.shape() != r.shape()) throw std::invalid_argument("add_rms_norm residual/delta shape mismatch");
    const std::int64_t hidden = r.shape().back();
    if (static_cast<std::int64_t>(in[2]->numel()) != hidden) throw std::invalid_argument("add_rms_norm weight size mismatch");
    const float eps = static_cast<float>(dli::attrDouble(attrs, "eps", 1e-6));
    *out[0] = Tensor::cuda(d.dtype(), r.shape(), r.deviceId());
    *out[1] = Tensor::cuda(r.dtype(), r.shape(), r.deviceId());
    check(dli_sm100_add_rms_norm_ex(dli::ptr(r), dli::ptr(d), dli::ptr(*in[2]), out[0]->deviceData(),
                                    out[1]->deviceData(), static_cast<std::int64_t>(r.numel()) / hidden, hidden, eps,
                                    cdt(d.dtype()), cdt(r.dtype()), ctx.cuda_stream),
          type());
  }
};

// silu_mul: gate_up [.., 2I] -> silu(gate) * up [.., I].
class SiluMulOp final : public dli::Operator {
 public:
  std::string type() const override { return "silu_mul"; }
  void compute(const Inputs& in, const Outputs& out, const Attributes&, ExecutionContext& ctx) const override {
    arity(in, out, 1, 1, 1, type());
    floatInputs(in, 1, type());
    const Tensor& x = *in[0];
    const std::int64_t w2 = x.shape().back();
    if (w2 % 2) throw std::invalid_argument("silu_mul expects an even last dimension");
    auto shape = x.shape();
    shape.back() = w2 / 2;
    *out[0] = Tensor::cuda(x.dtype(), shape, x.deviceId());
    check(dli_sm100_silu_mul(dli::ptr(x), out[0]->deviceData(), static_cast<std::int64_t>(x.numel()) / w2, w2 / 2,
                             cdt(x.dtype()), ctx.cuda_stream),
          type());
  }
};

int64_t requireIntAttr(const Attributes& attrs, const std::string& name, const std::string& op) {
  if (!attrs.contains(name)) throw std::invalid_argument(op + " missing attribute " + name);
  return attrs.require<std::int64_t>(name);
}

// linear_silu_mul: (x [.., K], w_glu [2*ceil(I/64)*64, K]) -> silu(x.Wg^T) * (x.Wu^T) [.., I],
// attr `intermediate` = I; w_glu holds gate/up rows in 64-row blocks. One
// tcgen05 GEMM with a SwiGLU epilogue (bfloat16/float16).
class LinearSiluMulOp final : public dli::Operator {
 public:
  std::string type() const override { return "linear_silu_mul"; }
  void compute(const Inputs& in, const Outputs& out, const Attributes& attrs, ExecutionContext& ctx) const override {
    arity(in, out, 2, 2, 1, type());
    floatInputs(in, 2, type());
    const Tensor& x = *in[0];
    const Tensor& w = *in[1];
    const std::int64_t inter = requireIntAttr(attrs, "intermediate", type());
    if (w.rank() != 2 || inter <= 0) throw std::invalid_argument("linear_silu_mul: bad weight or intermediate");
    const std::int64_t k = x.shape().back();
    if (w.dim(1) != k || w.dim(0) != 2 * ((inter + 63) / 64) * 64)
      throw std::invalid_argument("linear_silu_mul weight shape " + dli::formatShape(w.shape()) +
                                  " does not match the 64-row gate/up blocks of intermediate " + std::to_string(inter));
    const std::int64_t m = dli::product(x.shape(), 0, x.rank() - 1);
    auto shape = x.shape();
    shape.back() = inter;
    *out[0] = Tensor::cuda(x.dtype(), shape, x.deviceId());
    check(dli_sm100_linear_silu_mul(dli::ptr(x), dli::ptr(w), out[0]->deviceData(), m, inter, k, cdt(x.dtype()),
                                    ctx.cuda_stream),
          type());
  }
};

// qkv_rotary_cache: (qkv [B,S,(Hq+2Hkv)D], cos, sin, positions[B] int64) -> q [B,S,Hq,D].
// Rotated k and raw v go to rows positions[b]+s of the kv_cache entry (reserved
// with `capacity` rows on first use).
class QkvRotaryCacheOp final : public dli::Operator {
 public:
  std::string type() const override { return "qkv_rotary_cache"; }
  void compute(const Inputs& in, const Outputs& out, const Attributes& attrs, ExecutionContext& ctx) const override {
    arity(in, out, 4, 4, 1, type());
    dli::requireCudaInputs(in, type());
    const Tensor& qkv = *in[0];
    dli::requireFloat(qkv, type());
    const Tensor& cos = *in[1];
    const Tensor& sin = *in[2];
    const Tensor& pos = *in[3];
    if (cos.dtype() != DType::Float32 || sin.dtype() != DType::Float32 || cos.shape() != sin.shape() || cos.rank() != 2)
      throw std::invalid_argument("qkv_rotary_cache expects float32 cos/sin [max_pos, pairs]");
    if (pos.dtype() != DType::Int64) throw std::invalid_argument("qkv_rotary_cache positions must be int64");
    const std::int64_t hq = requireIntAttr(attrs, "q_heads", type());
    const std::int64_t hkv = requireIntAttr(attrs, "kv_heads", type());
    const std::int64_t d = requireIntAttr(attrs, "head_dim", type());
    const std::int64_t cap = requireIntAttr(attrs, "capacity", type());
    const std::string& name = attrs.require<std::string>("kv_cache");
    if (qkv.rank() != 3 || qkv.shape().back() != (hq + 2 * hkv) * d)
      throw std::invalid_argument("qkv_rotary_cache expects qkv [B,S,(Hq+2Hkv)*D]");
    const std::int64_t b = qkv.dim(0), s = qkv.dim(1);
    if (static_cast<std::int64_t>(pos.numel()) != b) throw std::invalid_argument("qkv_rotary_cache positions must be [B]");
    if (ctx.kv_cache == nullptr) throw std::invalid_argument("qkv_rotary_cache missing KV cache");
    dli::KVCacheEntry& e = ctx.kv_cache->reserve(name, b, hkv, cap, d, qkv.dtype(), qkv.deviceId());
    *out[0] = Tensor::cuda(qkv.dtype(), {b, s, hq, d}, qkv.deviceId());
    check(dli_sm100_qkv_rotary_cache(dli::ptr(qkv), static_cast<const float*>(dli::ptr(cos)),
                                     static_cast<const float*>(dli::ptr(sin)),
                                     static_cast<const std::int64_t*>(dli::ptr(pos)), out[0]->deviceData(),
                                     e.key.deviceData(), e.value.deviceData(), b, s, hq, hkv, d, cos.dim(1),
                                     cos.dim(0), e.capacity(), cdt(qkv.dtype()), ctx.cuda_stream),
          type());
  }
};

// linear_qkv_rotary_cache: (x [B,S,H], wqkv, bqkv, cos, sin, positions) -> q
// [B,S,Hq,D]: the fused q|k|v projection followed by qkv_rotary_cache, as one
// node. Decode-sized calls run one GEMM whose split-K epilogue rotates and
// scatters (the qkv tensor is never written); others run linear, then
// qkv_rotary_cache. Both forms give the same bits. Attributes as qkv_rotary_cache.
class LinearQkvRotaryCacheOp final : public dli::Operator {
 public:
  std::string type() const override { return "linear_qkv_rotary_cache"; }
  void compute(const Inputs& in, const Outputs& out, const Attributes& attrs, ExecutionContext& ctx) const override {
    arity(in, out, 6, 6, 1, type());
    dli::requireCudaInputs(in, type());
    const Tensor& x = *in[0];
    const Tensor& w = *in[1];
    const Tensor& bias = *in[2];
    const Tensor& cos = *in[3];
    const Tensor& sin = *in[4];
    const Tensor& pos = *in[5];
    dli::requireFloat(x, type());
    dli::requireSameDtype(x, w, type());
    dli::requireSameDtype(x, bias, type());
    if (cos.dtype() != DType::Float32 || sin.dtype() != DType::Float32 || cos.shape() != sin.shape() || cos.rank() != 2)
      throw std::invalid_argument(type() + " expects float32 cos/sin [max_pos, pairs]");
    if (pos.dtype() != DType::Int64) throw std::invalid_argument(type() + " positions must be int64");
    const std::int64_t hq = requireIntAttr(attrs, "q_heads", type());
    const std::int64_t hkv = requireIntAttr(attrs, "kv_heads", type());
    const std::int64_t d = requireIntAttr(attrs, "head_dim", type());
    const std::int64_t cap = requireIntAttr(attrs, "capacity", type());
    const std::string& name = attrs.require<std::string>("kv_cache");
    if (x.rank() != 3 || w.rank() != 2 || w.dim(0) != (hq + 2 * hkv) * d || w.dim(1) != x.dim(2) ||
        static_cast<std::int64_t>(bias.numel()) != w.dim(0))
      throw std::invalid_argument(type() + " expects x [B,S,H], wqkv [(Hq+2Hkv)*D, H], bqkv [(Hq+2Hkv)*D]");
    const std::int64_t b = x.dim(0), s = x.dim(1), k = x.dim(2);
    if (static_cast<std::int64_t>(pos.numel()) != b) throw std::invalid_argument(type() + " positions must be [B]");
    if (ctx.kv_cache == nullptr) throw std::invalid_argument(type() + " missing KV cache");
    if (x.dtype() == DType::BFloat16 || x.dtype() == DType::Float16) {
      dli::KVCacheEntry& e = ctx.kv_cache->reserve(name, b, hkv, cap, d, x.dtype(), x.deviceId());
      *out[0] = Tensor::cuda(x.dtype(), {b, s, hq, d}, x.deviceId());
      const dli_status st = dli_sm100_linear_qkv_rotary_cache(
          dli::ptr(x), dli::ptr(w), dli::ptr(bias), static_cast<const float*>(dli::ptr(cos)),
          static_cast<const float*>(dli::ptr(sin)), static_cast<const std::int64_t*>(dli::ptr(pos)),
          out[0]->deviceData(), e.key.deviceData(), e.value.deviceData(), b, s, k, hq, hkv, d, cos.dim(1),
          cos.dim(0), e.capacity(), cdt(x.dtype()), ctx.cuda_stream);
      if (st == DLI_OK) return;
      if (st != DLI_ERR_UNSUPPORTED) check(st, type());
    }
    // two-step form: the projection, then rotary + cache write
    Tensor qkv;
    const Tensor* lin_in[3] = {&x, &w, &bias};
    Tensor* lin_out[1] = {&qkv};
    LinearOp().compute(Inputs(lin_in, lin_in + 3), Outputs(lin_out, lin_out + 1), Attributes{}, ctx);
    const Tensor* rc_in[4] = {&qkv, &cos, &sin, &pos};
    QkvRotaryCacheOp().compute(Inputs(rc_in, rc_in + 4), out, attrs, ctx);
  }
};

// attention_kvcache: (q [B,S,Hq,D], positions[B]) -> out [B,S,Hq*D] over the
// kv_cache entry's rows [0, positions[b] + S), bottom-right causal.
class AttentionKvCacheOp final : public dli::Operator {
 public:
  std::string type() const override { return "attention_kvcache"; }
  void compute(const Inputs& in, const Outputs& out, const Attributes& attrs, ExecutionContext& ctx) const override {
    arity(in, out, 2, 2, 1, type());
    dli::requireCudaInputs(in, type());
    const Tensor& q = *in[0];
    const Tensor& pos = *in[1];
    dli::requireFloat(q, type());
    if (pos.dtype() != DType::Int64) throw std::invalid_argument("attention_kvcache positions must be int64");
    if (q.rank() != 4) throw std::invalid_argument("attention_kvcache expects q [B,S,Hq,D]");
    if (ctx.kv_cache == nullptr) throw std::invalid_argument("attention_kvcache missing KV cache");
    const dli::KVCacheEntry* e = ctx.kv_cache->get(attrs.require<std::string>("kv_cache"));
    if (e == nullptr) throw std::invalid_argument("attention_kvcache: unknown cache entry");
    const std::int64_t b = q.dim(0), s = q.dim(1), hq = q.dim(2), d = q.dim(3);
    const std::int64_t hkv = e->key.dim(1), cap = e->capacity();
    if (e->key.dim(0) != b || e->key.dim(3) != d || hq % hkv != 0)
      throw std::invalid_argument("attention_kvcache q/cache shape mismatch");
    const float scale = static_cast<float>(dli::attrDouble(attrs, "scale", 0.0));
    *out[0] = Tensor::cuda(q.dtype(), {b, s, hq * d}, q.deviceId());
    const dli_dtype dt = cdt(q.dtype());
    at::Tensor ws = workspace(dli_sm100_attention_kvcache_workspace_size(b, s, hq, hkv, cap, d, dt), q.deviceId());
    check(dli_sm100_attention_kvcache(dli::ptr(q), e->key.deviceData(), e->value.deviceData(),
                                      static_cast<const std::int64_t*>(dli::ptr(pos)), out[0]->deviceData(), b, s,
                                      hq, hkv, cap, d, scale, dt, wsPtr(ws), wsBytes(ws), ctx.cuda_stream),
          type());
  }
};

// last_token: x [B,S,W] -> x[:, index] (default S-1) as [B,W].
class LastTokenOp final : public dli::Operator {
 public:
  std::string type() const override { return "last_token"; }
  void compute(const Inputs& in, const Outputs& out, const Attributes& attrs, ExecutionContext& ctx) const override {
    arity(in, out, 1, 1, 1, type());
    floatInputs(in, 1, type());
    const Tensor& x = *in[0];
    if (x.rank() != 3) throw std::invalid_argument("last_token expects [B,S,W]");
    const std::int64_t index = attrs.value_or<std::int64_t>("index", x.dim(1) - 1);
    if (x.dim(1) == 1 && index == 0) {  // one token per sequence (decode): a view, no copy
      *out[0] = x.withShape({x.dim(0), x.dim(2)});
      return;
    }
    *out[0] = Tensor::cuda(x.dtype(), {x.dim(0), x.dim(2)}, x.deviceId());
    check(dli_sm100_select_token(dli::ptr(x), out[0]->deviceData(), x.dim(0), x.dim(1), x.dim(2), index,
                                 cdt(x.dtype()), ctx.cuda_stream),
          type());
  }
};

// argmax over the last dim -> int64 ids (greedy decoding).
class ArgmaxOp final : public dli::Operator {
 public:
  std::string type() const override { return "argmax"; }
  void compute(const Inputs& in, const Outputs& out, const Attributes&, ExecutionContext& ctx) const override {
    arity(in, out, 1, 1, 1, type());
    floatInputs(in, 1, type());
    const Tensor& x = *in[0];
    const std::int64_t width = x.shape().back();
    auto shape = x.shape();
    shape.pop_back();
    if (shape.empty()) shape.push_back(1);
    *out[0] = Tensor::cuda(DType::Int64, shape, x.deviceId());
    check(dli_sm100_argmax(dli::ptr(x), static_cast<std::int64_t*>(out[0]->deviceData()),
                           static_cast<std::int64_t>(x.numel()) / width, width, cdt(x.dtype()), ctx.cuda_stream),
          type());
  }
};

// cast: float dtype conversion, attr dtype = "float32" | "bfloat16" | "float16".
class CastOp final : public dli::Operator {
 public:
  std::string type() const override { return "cast"; }
  void compute(const Inputs& in, const Outputs& out, const Attributes& attrs, ExecutionContext& ctx) const override {
    arity(in, out, 1, 1, 1, type());
    floatInputs(in, 1, type());
    const Tensor& x = *in[0];
    const DType to = dli::dtypeFromString(attrs.require<std::string>("dtype"));
    if (!dli::isFloating(to)) throw std::invalid_argument("cast target must be a float dtype");
    if (to == x.dtype()) {  // nothing to convert: the output is the input
      *out[0] = x;
      return;
    }
    *out[0] = Tensor::cuda(to, x.shape(), x.deviceId());
    check(dli_sm100_cast(dli::ptr(x), cdt(x.dtype()), out[0]->deviceData(), cdt(to),
                         static_cast<std::int64_t>(x.numel()), ctx.cuda_stream),
          type());
  }
};

// all_reduce: sum over the tensor-parallel group (identity when tp_size == 1).
class AllReduceOp final : public dli::Operator {
 public:
  std::string type() const override { return "all_reduce"; }
  void compute(const Inputs& in, const Outputs& out, const Attributes&, ExecutionContext& ctx) const override {
    arity(in, out, 1, 1, 1, type());
    floatInputs(in, 1, type());
    const Tensor& x = *in[0];
    if (ctx.tp_size <= 1 || ctx.communicator == nullptr) {
      if (ctx.tp_size > 1) throw std::invalid_argument("all_reduce: no communicator for tp_size > 1");
      *out[0] = x;  // single rank: the sum is the input
      return;
    }
#ifdef DLI_WITH_NCCL
    *out[0] = Tensor::cuda(x.dtype(), x.shape(), x.deviceId());
    ncclDataType_t t = x.dtype() == DType::Float32 ? ncclFloat32
                       : x.dtype() == DType::BFloat16 ? ncclBfloat16 : ncclFloat16;
    const ncclResult_t r = ncclAllReduce(dli::ptr(x), out[0]->deviceData(), x.numel(), t, ncclSum,
                                         static_cast<ncclComm_t>(ctx.communicator),
                                         static_cast<cudaStream_t>(ctx.cuda_stream));
    if (r != ncclSuccess) throw std::runtime_error(std::string("all_reduce: ") + ncclGetErrorString(r));
#else
    throw std::runtime_error("all_reduce: plugin built without NCCL");
#endif
  }
};

// ---------------------------------------------------------------------------
// Tensor-parallel exchange buffers (one per communicator), created collectively
// by dli_sm100_tp_exchange_create: a cudaMalloc'ed buffer per rank whose CUDA IPC
// handle is all-gathered over the communicator and opened by every peer, so the
// fused all-reduce kernel can store into every peer's buffer over NVLink.
// ---------------------------------------------------------------------------
struct Exchange {
  int tp = 1, rank = 0, device = 0;
  std::int64_t max_rows = 0, row_elems = 0;
  dli_dtype dtype = DLI_DTYPE_BF16;
  void* local = nullptr;
  std::vector<void*> ptrs;  // rank i's buffer as mapped in this process
};

std::mutex g_exchange_mu;
std::map<void*, std::unique_ptr<Exchange>>& exchanges() {
  static std::map<void*, std::unique_ptr<Exchange>> m;
  return m;
}

const Exchange* findExchange(void* comm) {
  std::lock_guard<std::mutex> lock(g_exchange_mu);
  auto it = exchanges().find(comm);
  return it == exchanges().end() ? nullptr : it->second.get();
}

// all_reduce_add_rms_norm: (residual, delta, weight) -> (normed, residual + all_reduce(delta)).
// The tensor-parallel form of add_rms_norm. With an exchange buffer registered
// for the run's communicator and rows that fit it, one fused kernel does the
// all-reduce over NVLink peer memory and the norm; otherwise (prefill-sized
// rows, no buffer) an NCCL all_reduce followed by add_rms_norm. The kernel
// answers DLI_ERR_UNSUPPORTED for shape reasons only, so every rank of the group
// takes the same branch; a per-rank problem (alignment) is a thrown error.
class AllReduceAddRmsNormOp final : public dli::Operator {
 public:
  std::string type() const override { return "all_reduce_add_rms_norm"; }
  void compute(const Inputs& in, const Outputs& out, const Attributes& attrs, ExecutionContext& ctx) const override {
    arity(in, out, 3, 3, 2, type());
    residualInputs(in, type());
    const Tensor& r = *in[0];
    const Tensor& d = *in[1];
    if (d.shape() != r.shape()) throw std::invalid_argument("all_reduce_add_rms_norm residual/delta shape mismatch");
    const std::int64_t hidden = r.shape().back();
    if (static_cast<std::int64_t>(in[2]->numel()) != hidden)
      throw std::invalid_argument("all_reduce_add_rms_norm weight size mismatch");
    const std::int64_t rows = static_cast<std::int64_t>(r.numel()) / hidden;
    const float eps = static_cast<float>(dli::attrDouble(attrs, "eps", 1e-6));
    *out[0] = Tensor::cuda(d.dtype(), r.shape(), r.deviceId());
    *out[1] = Tensor::cuda(r.dtype(), r.shape(), r.deviceId());
    const void* delta = dli::ptr(d);
    Tensor summed;
    if (ctx.tp_size > 1) {
      if (ctx.communicator == nullptr) throw std::invalid_argument(type() + ": no communicator for tp_size > 1");
      const Exchange* ex = findExchange(ctx.communicator);
      if (ex != nullptr && ex->tp == ctx.tp_size && ex->rank == ctx.tp_rank && ex->dtype == cdt(d.dtype()) &&
          rows <= ex->max_rows && hidden <= ex->row_elems) {
        const dli_status st = dli_sm100_allreduce_add_rms_norm_ex(
            ex->ptrs.data(), ex->tp, ex->rank, 1, ex->max_rows, ex->row_elems, delta, dli::ptr(r),
            dli::ptr(*in[2]), out[0]->deviceData(), out[1]->deviceData(), 0, rows, hidden, eps, 0,
            cdt(d.dtype()), cdt(r.dtype()), ctx.cuda_stream);
        if (st == DLI_OK) return;
        if (st != DLI_ERR_UNSUPPORTED) check(st, type());
      }
#ifdef DLI_WITH_NCCL
      summed = Tensor::cuda(d.dtype(), d.shape(), d.deviceId());
      ncclDataType_t t = d.dtype() == DType::Float32 ? ncclFloat32
                         : d.dtype() == DType::BFloat16 ? ncclBfloat16 : ncclFloat16;
      const ncclResult_t res = ncclAllReduce(delta, summed.deviceData(), d.numel(), t, ncclSum,
                                             static_cast<ncclComm_t>(ctx.communicator),
                                             static_cast<cudaStream_t>(ctx.cuda_stream));
      if (res != ncclSuccess) throw std::runtime_error(type() + ": " + ncclGetErrorString(res));
      delta = summed.deviceData();
#else
      throw std::runtime_error(type() + ": plugin built without NCCL");
#endif
    }
    check(dli_sm100_add_rms_norm_ex(dli::ptr(r), delta, dli::ptr(*in[2]), out[0]->deviceData(),
                                    out[1]->deviceData(), rows, hidden, eps, cdt(d.dtype()), cdt(r.dtype()),
                                    ctx.cuda_stream),
          type());
  }
};

// linear_all_reduce_add_rms_norm: (residual, x, w, weight) -> (normed, residual +
// all_reduce(x . w^T)). A row-split projection and the all-reduce + residual add +
// RMSNorm after it as one node. With an exchange buffer for the run's
// communicator and a decode-sized call, the projection's GEMM pushes its
// partial rows into every rank's exchange buffer from its own split-K epilogue
// (dli_sm100_linear_exchange_push) and one kernel sums, adds and normalises
// (dli_sm100_exchange_add_rms_norm_ex), bit-identical to the two-node form.
// Other calls (prefill rows, tp == 1, no buffer) run linear, then the
// all_reduce_add_rms_norm operator. The fused path is declined
// (DLI_ERR_UNSUPPORTED) for shape reasons only, the same on every rank.
class LinearAllReduceAddRmsNormOp final : public dli::Operator {
 public:
  std::string type() const override { return "linear_all_reduce_add_rms_norm"; }
  void compute(const Inputs& in, const Outputs& out, const Attributes& attrs, ExecutionContext& ctx) const override {
    arity(in, out, 4, 4, 2, type());
    dli::requireCudaInputs(in, type());
    for (const Tensor* t : in) dli::requireFloat(*t, type());
    const Tensor& r = *in[0];
    const Tensor& x = *in[1];
    const Tensor& w = *in[2];
    const Tensor& g = *in[3];
    dli::requireSameDtype(x, w, type());
    dli::requireSameDtype(x, g, type());
    if (r.dtype() != x.dtype() &&
        !(r.dtype() == DType::Float32 && (x.dtype() == DType::BFloat16 || x.dtype() == DType::Float16)))
      throw std::invalid_argument(type() + ": residual must match x or be float32 around a 16-bit x");
    if (w.rank() != 2) throw std::invalid_argument(type() + ": weight must be 2-D");
    const std::int64_t k = x.shape().back(), n = w.dim(0);
    if (w.dim(1) != k) throw std::invalid_argument(type() + ": weight K mismatch");
    const std::int64_t m = dli::product(x.shape(), 0, x.rank() - 1);
    if (r.shape().back() != n || static_cast<std::int64_t>(r.numel()) != m * n)
      throw std::invalid_argument(type() + ": residual must be [.., " + std::to_string(n) + "] with x's rows");
    if (static_cast<std::int64_t>(g.numel()) != n) throw std::invalid_argument(type() + ": norm weight size");
    const float eps = static_cast<float>(dli::attrDouble(attrs, "eps", 1e-6));
    if (ctx.tp_size > 1 && ctx.communicator != nullptr) {
      const Exchange* ex = findExchange(ctx.communicator);
      if (ex != nullptr && ex->tp == ctx.tp_size && ex->rank == ctx.tp_rank && ex->dtype == cdt(x.dtype()) &&
          m <= ex->max_rows && n <= ex->row_elems) {
        const dli_status st = dli_sm100_linear_exchange_push(dli::ptr(x), dli::ptr(w), nullptr, m, n, k,
                                                             cdt(x.dtype()), ex->ptrs.data(), ex->tp, ex->rank,
                                                             ex->max_rows, ex->row_elems, ctx.cuda_stream);
        if (st == DLI_OK) {
          *out[0] = Tensor::cuda(x.dtype(), r.shape(), r.deviceId());
          *out[1] = Tensor::cuda(r.dtype(), r.shape(), r.deviceId());
          check(dli_sm100_exchange_add_rms_norm_ex(ex->ptrs.data(), ex->tp, ex->rank, 1, ex->max_rows,
                                                   ex->row_elems, dli::ptr(r), dli::ptr(g), out[0]->deviceData(),
                                                   out[1]->deviceData(), 0, m, n, eps, 0, cdt(x.dtype()),
                                                   cdt(r.dtype()), ctx.cuda_stream),
                type());
          return;
        }
        if (st != DLI_ERR_UNSUPPORTED) check(st, type());
      }
    }
    // two-node form: the partial projection, then the all-reduce + add + norm
    Tensor part;
    const Tensor* lin_in[2] = {&x, &w};
    Tensor* lin_out[1] = {&part};
    LinearOp().compute(Inputs(lin_in, lin_in + 2), Outputs(lin_out, lin_out + 1), Attributes{}, ctx);
    const Tensor* ar_in[3] = {&r, &part, &g};
    AllReduceAddRmsNormOp().compute(Inputs(ar_in, ar_in + 3), out, attrs, ctx);
  }
};

// tp_argmax: logits [.., width] holding ids [tp_rank*width, (tp_rank+1)*width) of a
// vocabulary split over the tensor-parallel group -> int64 ids of the row maxima
// over the whole vocabulary (lowest id on ties). One kernel: local argmax and an
// exchange of (value, id) candidates through the group's NVLink exchange
// buffers. With tp_size == 1 it is argmax.
class TpArgmaxOp final : public dli::Operator {
 public:
  std::string type() const override { return "tp_argmax"; }
  void compute(const Inputs& in, const Outputs& out, const Attributes&, ExecutionContext& ctx) const override {
    arity(in, out, 1, 1, 1, type());
    floatInputs(in, 1, type());
    const Tensor& x = *in[0];
    const std::int64_t width = x.shape().back();
    const std::int64_t rows = static_cast<std::int64_t>(x.numel()) / width;
    auto shape = x.shape();
    shape.pop_back();
    if (shape.empty()) shape.push_back(1);
    *out[0] = Tensor::cuda(DType::Int64, shape, x.deviceId());
    auto* ids = static_cast<std::int64_t*>(out[0]->deviceData());
    if (ctx.tp_size <= 1) {
      check(dli_sm100_argmax(dli::ptr(x), ids, rows, width, cdt(x.dtype()), ctx.cuda_stream), type());
      return;
    }
    const Exchange* ex = ctx.communicator ? findExchange(ctx.communicator) : nullptr;
    if (ex == nullptr || ex->tp != ctx.tp_size || ex->rank != ctx.tp_rank || rows > ex->max_rows)
      throw std::invalid_argument(type() + ": needs the group's exchange buffers with max_rows >= " +
                                  std::to_string(rows) + " (dli_sm100_tp_exchange_create)");
    check(dli_sm100_allgather_argmax(ex->ptrs.data(), ex->tp, ex->rank, 1, ex->max_rows, ex->row_elems, ex->dtype,
                                     dli::ptr(x), rows, width, 0, ids, 0, cdt(x.dtype()), ctx.cuda_stream),
          type());
  }
};

}  // namespace

extern "C" bool dli_register_operators(dli::OperatorRegistry* registry) {
  if (registry == nullptr) return false;
  if (dli_sm100_abi_version() != DLI_SM100_ABI_VERSION) return false;
  reg<LinearOp>(registry, "linear");
  reg<MatmulOp>(registry, "matmul");
  reg<Conv2dOp>(registry, "conv2d");
  reg<RmsNormOp>(registry, "rms_norm");
  reg<RotaryOp>(registry, "rotary_embedding");
  reg<AttentionOp>(registry, "attention");
  reg<EmbeddingOp>(registry, "embedding");
  reg<BinaryOp<0>>(registry, "add");
  reg<BinaryOp<1>>(registry, "mul");
  reg<UnaryOp<0>>(registry, "silu");
  reg<UnaryOp<1>>(registry, "relu");
  reg<SoftmaxOp>(registry, "softmax");
  reg<MaxPool2dOp>(registry, "max_pool2d");
  reg<BatchNorm2dOp>(registry, "batch_norm2d");
  reg<ReshapeOp>(registry, "reshape");
  reg<TransposeOp>(registry, "transpose");
  reg<AddRmsNormOp>(registry, "add_rms_norm");
  reg<SiluMulOp>(registry, "silu_mul");
  reg<LinearSiluMulOp>(registry, "linear_silu_mul");
  reg<QkvRotaryCacheOp>(registry, "qkv_rotary_cache");
  reg<AttentionKvCacheOp>(registry, "attention_kvcache");
  reg<LastTokenOp>(registry, "last_token");
  reg<ArgmaxOp>(registry, "argmax");
  reg<CastOp>(registry, "cast");
  reg<AllReduceOp>(registry, "all_reduce");
  reg<AllReduceAddRmsNormOp>(registry, "all_reduce_add_rms_norm");
  reg<LinearAllReduceAddRmsNormOp>(registry, "linear_all_reduce_add_rms_norm");
  reg<LinearQkvRotaryCacheOp>(registry, "linear_qkv_rotary_cache");
  reg<TpArgmaxOp>(registry, "tp_argmax");
  return true;
}

// ---- tensor-parallel communicator helpers (called from Python via ctypes) ----
extern "C" int dli_sm100_plugin_has_nccl(void) {
#ifdef DLI_WITH_NCCL
  return 1;
#else
  return 0;
#endif
}

extern "C" int dli_sm100_nccl_unique_id(void* out, int out_bytes) {
#ifdef DLI_WITH_NCCL
  if (out == nullptr || out_bytes < static_cast<int>(sizeof(ncclUniqueId))) return -1;
  ncclUniqueId id;
  if (ncclGetUniqueId(&id) != ncclSuccess) return -2;
  std::memcpy(out, &id, sizeof(id));
  return static_cast<int>(sizeof(id));
#else
  (void)out;
  (void)out_bytes;
  return -3;
#endif
}

extern "C" void* dli_sm100_nccl_comm_init(const void* id_bytes, int world, int rank, int device) {
#ifdef DLI_WITH_NCCL
  if (id_bytes == nullptr) return nullptr;
  if (cudaSetDevice(device) != cudaSuccess) return nullptr;
  ncclUniqueId id;
  std::memcpy(&id, id_bytes, sizeof(id));
  ncclComm_t comm = nullptr;
  if (ncclCommInitRank(&comm, world, id, rank) != ncclSuccess) return nullptr;
  return comm;
#else
  (void)id_bytes;
  (void)world;
  (void)rank;
  (void)device;
  return nullptr;
#endif
}

extern "C" void dli_sm100_nccl_comm_destroy(void* comm) {
#ifdef DLI_WITH_NCCL
  if (comm) ncclCommDestroy(static_cast<ncclComm_t>(comm));
#else
  (void)comm;
#endif
}

// Creates this rank's exchange buffer for `comm` and maps every peer's (a
// collective: every rank of the communicator calls it at the same point).
// Returns 0, or a negative code: -1 no NCCL, -2 bad arguments, -3 CUDA error,
// -4 NCCL error.
extern "C" int dli_sm100_tp_exchange_create(void* comm, int device, std::int64_t max_rows,
                                            std::int64_t row_elems, int dtype) {
#ifdef DLI_WITH_NCCL
  if (comm == nullptr) return -2;
  int tp = 0, rank = 0;
  if (ncclCommCount(static_cast<ncclComm_t>(comm), &tp) != ncclSuccess ||
      ncclCommUserRank(static_cast<ncclComm_t>(comm), &rank) != ncclSuccess)
    return -4;
  const std::size_t bytes = dli_sm100_tp_exchange_bytes(tp, max_rows, row_elems, static_cast<dli_dtype>(dtype));
  if (bytes == 0) return -2;
  if (cudaSetDevice(device) != cudaSuccess) return -3;
  auto ex = std::make_unique<Exchange>();
  ex->tp = tp;
  ex->rank = rank;
  ex->device = device;
  ex->max_rows = max_rows;
  ex->row_elems = row_elems;
  ex->dtype = static_cast<dli_dtype>(dtype);
  ex->ptrs.assign(tp, nullptr);
  cudaStream_t s = nullptr;
  void* handles_dev = nullptr;
  std::vector<cudaIpcMemHandle_t> handles(tp);
  int rc = 0;
  if (cudaMalloc(&ex->local, bytes) != cudaSuccess || cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMalloc(&handles_dev, sizeof(cudaIpcMemHandle_t) * tp) != cudaSuccess) {
    rc = -3;
  } else if (dli_sm100_tp_exchange_reset(ex->local, bytes, s) != DLI_OK ||
             cudaIpcGetMemHandle(&handles[rank], ex->local) != cudaSuccess ||
             cudaMemcpyAsync(static_cast<char*>(handles_dev) + rank * sizeof(cudaIpcMemHandle_t), &handles[rank],
                             sizeof(cudaIpcMemHandle_t), cudaMemcpyHostToDevice, s) != cudaSuccess) {
    rc = -3;
  } else if (ncclAllGather(static_cast<char*>(handles_dev) + rank * sizeof(cudaIpcMemHandle_t), handles_dev,
                           sizeof(cudaIpcMemHandle_t), ncclChar, static_cast<ncclComm_t>(comm), s) != ncclSuccess) {
    rc = -4;
  } else if (cudaMemcpyAsync(handles.data(), handles_dev, sizeof(cudaIpcMemHandle_t) * tp, cudaMemcpyDeviceToHost, s) !=
                 cudaSuccess ||
             cudaStreamSynchronize(s) != cudaSuccess) {
    rc = -3;
  }
  // After the all-gather completed here, every rank's buffer reset (ordered
  // before its all-gather on its stream) has completed too.
  for (int i = 0; rc == 0 && i < tp; ++i) {
    if (i == rank) {
      ex->ptrs[i] = ex->local;
    } else if (cudaIpcOpenMemHandle(&ex->ptrs[i], handles[i], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      rc = -3;
    }
  }
  if (handles_dev) cudaFree(handles_dev);
  if (s) cudaStreamDestroy(s);
  if (rc != 0) {
    for (int i = 0; i < tp; ++i)
      if (i != rank && ex->ptrs[i]) cudaIpcCloseMemHandle(ex->ptrs[i]);
    if (ex->local) cudaFree(ex->local);
    cudaGetLastError();
    return rc;
  }
  std::lock_guard<std::mutex> lock(g_exchange_mu);
  exchanges()[comm] = std::move(ex);
  return 0;
#else
  (void)comm;
  (void)device;
  (void)max_rows;
  (void)row_elems;
  (void)dtype;
  return -1;
#endif
}

// Unmaps the peers' buffers and frees this rank's. Call when no kernel of the
// group is in flight on any rank (after a device synchronisation and a barrier),
// before the communicator is destroyed.
extern "C" void dli_sm100_tp_exchange_destroy(void* comm) {
  std::unique_ptr<Exchange> ex;
  {
    std::lock_guard<std::mutex> lock(g_exchange_mu);
    auto it = exchanges().find(comm);
    if (it == exchanges().end()) return;
    ex = std::move(it->second);
    exchanges().erase(it);
  }
  cudaSetDevice(ex->device);
  for (int i = 0; i < ex->tp; ++i)
    if (i != ex->rank && ex->ptrs[i]) cudaIpcCloseMemHandle(ex->ptrs[i]);
  if (ex->local) cudaFree(ex->local);
}
