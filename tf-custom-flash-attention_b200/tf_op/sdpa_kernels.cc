// TensorFlow OpKernels of `Sdpa` / `SdpaGrad` on the GPU, calling the sm_100a
// kernels through the C ABI of include/sdpa_b200.h.
//
// Replaces SdpaFwdOp / SdpaBwdOp (sdpa/sdpa_cpu.cc:14-193): same attrs, same
// checks in the same order with the same InvalidArgument messages
// (sdpa/sdpa_cpu.cc:37-69 and :116-168), outputs allocated with
// allocate_output, seed / offset read on the host (registered HostMemory as in
// sdpa/sdpa_cpu.cc:470-487), launched on TF's compute stream.  Deliberate
// differences: only GPU kernels are registered (no CPU fallback), and a
// failing launch returns errors::Internal instead of aborting the process.
// The backward's per-row scratch comes from allocate_temp.
#include <algorithm>
#include <cstdint>

#include "tensorflow/core/framework/op_kernel.h"
#include "../../include/sdpa_b200.h"

namespace tensorflow {
namespace sdpa_b200_tf {

template <typename T> struct DType;
template <> struct DType<float> { static constexpr int v = SDPA_B200_F32; };
template <> struct DType<Eigen::half> { static constexpr int v = SDPA_B200_F16; };

struct OpAttrs {
  float scale = 1.0f;
  float dropout = 0.0f;
  bool causal = false;
};

Status ReadAttrs(OpKernelConstruction* c, OpAttrs* a) {
  TF_RETURN_IF_ERROR(c->GetAttr("dropout", &a->dropout));
  TF_RETURN_IF_ERROR(c->GetAttr("scale", &a->scale));
  TF_RETURN_IF_ERROR(c->GetAttr("causal_mask", &a->causal));
  return OkStatus();
}

// seed / offset scalars (host memory)
Status ReadRng(const Tensor& seed, const Tensor& offset, uint64* s, uint64* o) {
  if (!TensorShapeUtils::IsScalar(seed.shape())) return errors::InvalidArgument("seed must be scalar");
  if (!TensorShapeUtils::IsScalar(offset.shape())) return errors::InvalidArgument("offset must be scalar");
  *s = seed.scalar<uint64>()();
  *o = offset.scalar<uint64>()();
  return OkStatus();
}

struct Dims {
  int64_t B, S_q, D_qk, S_kv, D_v;
};

// Shape checks shared by both ops, in the reference's order.
Status CheckQKV(const Tensor& q, const Tensor& k, const Tensor& v, Dims* d) {
  d->B = q.dim_size(0);
  d->S_q = q.dim_size(1);
  d->D_qk = q.dim_size(2);
  d->S_kv = k.dim_size(1);
  d->D_v = v.dim_size(2);
  if (k.dim_size(0) != d->B) return errors::InvalidArgument("K batch size mismatch");
  if (k.dim_size(2) != d->D_qk) return errors::InvalidArgument("K feature size mismatch");
  if (v.dim_size(0) != d->B) return errors::InvalidArgument("V batch size mismatch");
  if (v.dim_size(1) != d->S_kv) return errors::InvalidArgument("V seq size mismatch");
  return OkStatus();
}

Status CheckTail(const Dims& d, bool causal) {
  if (causal && d.S_q != d.S_kv) return errors::InvalidArgument("seq size Q != K while causal_mask = True");
  if (std::max(d.D_qk, d.D_v) > 128)
    return errors::InvalidArgument(
        "CUDA kernel does not support feature size over 128. Set smaller feature size or use more heads");
  return OkStatus();
}

Status FromCode(int rc) {
  if (rc == SDPA_B200_OK) return OkStatus();
  return errors::Internal(sdpa_b200_strerror(rc));
}

template <typename T>
class SdpaOp : public OpKernel {
 public:
  explicit SdpaOp(OpKernelConstruction* c) : OpKernel(c) { OP_REQUIRES_OK(c, ReadAttrs(c, &a_)); }

  void Compute(OpKernelContext* ctx) override {
    const Tensor& q = ctx->input(0);
    const Tensor& k = ctx->input(1);
    const Tensor& v = ctx->input(2);
    uint64 seed = 0, offset = 0;
    OP_REQUIRES_OK(ctx, ReadRng(ctx->input(3), ctx->input(4), &seed, &offset));
    Dims d;
    OP_REQUIRES_OK(ctx, CheckQKV(q, k, v, &d));
    OP_REQUIRES_OK(ctx, CheckTail(d, a_.causal));
    Tensor* out = nullptr;
    Tensor* stats = nullptr;
    OP_REQUIRES_OK(ctx, ctx->allocate_output(0, TensorShape({d.B, d.S_q, d.D_v}), &out));
    OP_REQUIRES_OK(ctx, ctx->allocate_output(1, TensorShape({d.B, d.S_q}), &stats));
    void* stream = reinterpret_cast<void*>(ctx->template eigen_device<Eigen::GpuDevice>().stream());
    OP_REQUIRES_OK(ctx, FromCode(sdpa_b200_fwd(DType<T>::v, q.flat<T>().data(), k.flat<T>().data(), v.flat<T>().data(), out->flat<T>().data(),
                                               stats->flat<float>().data(), d.B, d.S_q, d.S_kv, d.D_qk,
                                               d.D_v, a_.scale, a_.dropout, a_.causal ? 1 : 0, seed, offset,
                                               stream)));
  }

 private:
  OpAttrs a_;
};

template <typename T>
class SdpaGradOp : public OpKernel {
 public:
  explicit SdpaGradOp(OpKernelConstruction* c) : OpKernel(c) { OP_REQUIRES_OK(c, ReadAttrs(c, &a_)); }

  void Compute(OpKernelContext* ctx) override {
    const Tensor& q = ctx->input(0);
    const Tensor& k = ctx->input(1);
    const Tensor& v = ctx->input(2);
    const Tensor& out = ctx->input(3);
    const Tensor& stats = ctx->input(4);
    const Tensor& d_out = ctx->input(5);
    uint64 seed = 0, offset = 0;
    OP_REQUIRES_OK(ctx, ReadRng(ctx->input(6), ctx->input(7), &seed, &offset));
    Dims d;
    OP_REQUIRES_OK(ctx, CheckQKV(q, k, v, &d));
    OP_REQUIRES(ctx, out.dim_size(0) == d.B, errors::InvalidArgument("O batch size mismatch"));
    OP_REQUIRES(ctx, out.dim_size(1) == d.S_q, errors::InvalidArgument("O seq size mismatch"));
    OP_REQUIRES(ctx, out.dim_size(2) == d.D_v, errors::InvalidArgument("O feature size mismatch"));
    OP_REQUIRES(ctx, d_out.dim_size(0) == d.B, errors::InvalidArgument("dO batch size mismatch"));
    OP_REQUIRES(ctx, d_out.dim_size(1) == d.S_q, errors::InvalidArgument("dO seq size mismatch"));
    OP_REQUIRES(ctx, d_out.dim_size(2) == d.D_v, errors::InvalidArgument("dO feature size mismatch"));
    OP_REQUIRES(ctx, stats.dim_size(0) == d.B, errors::InvalidArgument("S batch size mismatch"));
    OP_REQUIRES(ctx, stats.dim_size(1) == d.S_q, errors::InvalidArgument("S seq size mismatch"));
    OP_REQUIRES_OK(ctx, CheckTail(d, a_.causal));
    Tensor* dq = nullptr;
    Tensor* dk = nullptr;
    Tensor* dv = nullptr;
    OP_REQUIRES_OK(ctx, ctx->allocate_output(0, q.shape(), &dq));
    OP_REQUIRES_OK(ctx, ctx->allocate_output(1, k.shape(), &dk));
    OP_REQUIRES_OK(ctx, ctx->allocate_output(2, v.shape(), &dv));
    const size_t ws_bytes = sdpa_b200_bwd_workspace_bytes(DType<T>::v, d.B, d.S_q, d.S_kv, d.D_qk, d.D_v);
    Tensor ws;
    OP_REQUIRES_OK(ctx, ctx->allocate_temp(DT_FLOAT, TensorShape({static_cast<long>((ws_bytes + 3) / 4)}), &ws));
    void* stream = reinterpret_cast<void*>(ctx->template eigen_device<Eigen::GpuDevice>().stream());
    OP_REQUIRES_OK(ctx, FromCode(sdpa_b200_bwd(DType<T>::v, q.flat<T>().data(), k.flat<T>().data(), v.flat<T>().data(), out.flat<T>().data(),
                                               stats.flat<float>().data(), d_out.flat<T>().data(), dq->flat<T>().data(),
                                               dk->flat<T>().data(), dv->flat<T>().data(), d.B, d.S_q, d.S_kv, d.D_qk, d.D_v, a_.scale,
                                               a_.dropout, a_.causal ? 1 : 0, seed, offset, ws.flat<float>().data(), ws_bytes,
                                               stream)));
  }

 private:
  OpAttrs a_;
};

#define SDPA_B200_REGISTER(T)                                                                                   \
  REGISTER_KERNEL_BUILDER(                                                                                     \
      Name("Sdpa").Device(DEVICE_GPU).TypeConstraint<T>("T").HostMemory("seed").HostMemory("offset"),          \
      SdpaOp<T>);                                                                                              \
  REGISTER_KERNEL_BUILDER(                                                                                     \
      Name("SdpaGrad").Device(DEVICE_GPU).TypeConstraint<T>("T").HostMemory("seed").HostMemory("offset"),      \
      SdpaGradOp<T>)

SDPA_B200_REGISTER(float);
SDPA_B200_REGISTER(Eigen::half);
#undef SDPA_B200_REGISTER

}  // namespace sdpa_b200_tf
}  // namespace tensorflow
