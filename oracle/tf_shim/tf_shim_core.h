// Minimal stand-ins for the handful of TensorFlow / Eigen types that the
// reference op sources touch, so those sources compile UNMODIFIED with plain
// g++ / nvcc and can be run as a parity oracle and CPU baseline.
//
// TEST INFRASTRUCTURE ONLY.  Nothing in the product library includes this.
// It is also used to compile-check the product's own TensorFlow op surface
// (tf_op/) on a machine without TensorFlow.
//
// What is modelled (and nothing more):
//   * Eigen::half            -- binary16 with "multiply, then round to half"
//                               semantics (device: __hmul; host: exact fp32
//                               product rounded to nearest-even half).  The
//                               product of two halves is exact in fp32, so the
//                               two agree bit for bit.
//   * Eigen::numext::exp/log -- expf/logf on device, std::exp/std::log on host.
//   * TTypes<T,N>::Tensor    -- row-major N-d views with operator(), dimension,
//                               data, setZero.
//   * Eigen::ThreadPoolDevice::parallelFor -- contiguous blocks over std::thread.
//   * Eigen::GpuDevice::stream, GpuLaunchKernel, TF_CHECK_OK.
//   * OpKernel / OpKernelConstruction / OpKernelContext / Tensor /
//     TensorShape / Status / errors::InvalidArgument / OP_REQUIRES(_OK) /
//     REGISTER_KERNEL_BUILDER / REGISTER_OP -- enough to run Compute().
#pragma once

#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <cstdio>
#include <cmath>
#include <string>
#include <vector>
#include <map>
#include <functional>
#include <thread>
#include <initializer_list>
#include <utility>
#include <type_traits>

#if defined(__CUDACC__)
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#define TFS_HD __host__ __device__
#else
#define TFS_HD
#endif
#if defined(__CUDACC__) || defined(TFS_WITH_CUDA_RUNTIME)
#include <cuda_runtime_api.h>
#define TFS_HAVE_CUDA_RT 1
#endif

// ---------------------------------------------------------------- Eigen part
namespace Eigen {

typedef long DenseIndex;
enum { RowMajor = 1 };

namespace tfs_detail {
// IEEE binary16 <-> binary32, round to nearest even (host side).
inline uint16_t f32_to_f16_bits(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t absx = x & 0x7fffffffu;
  if (absx >= 0x7f800000u) {  // inf / nan
    return (uint16_t)(sign | 0x7c00u | (absx > 0x7f800000u ? 0x200u : 0u));
  }
  if (absx >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);  // overflow -> inf
  if (absx < 0x38800000u) {  // subnormal half (or zero)
    // value = absx as float; half subnormal unit = 2^-24
    float af;
    std::memcpy(&af, &absx, 4);
    float scaled = af * 16777216.0f;  // exact (power of two)
    // round to nearest even integer
    float r = std::nearbyint(scaled);
    return (uint16_t)(sign | (uint32_t)r);
  }
  uint32_t mant = absx & 0x7fffffu;
  int32_t exp = (int32_t)(absx >> 23) - 127 + 15;
  uint32_t h = ((uint32_t)exp << 10) | (mant >> 13);
  uint32_t rem = mant & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1;  // may carry into exponent: fine
  return (uint16_t)(sign | h);
}
inline float f16_bits_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1fu;
  uint32_t m = h & 0x3ffu;
  uint32_t x;
  if (e == 0) {
    if (m == 0) {
      x = sign;
    } else {
      float f = (float)m / 16777216.0f;
      std::memcpy(&x, &f, 4);
      x |= sign;
    }
  } else if (e == 31) {
    x = sign | 0x7f800000u | (m << 13);
  } else {
    x = sign | ((e - 15 + 127) << 23) | (m << 13);
  }
  float f;
  std::memcpy(&f, &x, 4);
  return f;
}
}  // namespace tfs_detail

struct half {
  uint16_t x;
  TFS_HD half() : x(0) {}
  TFS_HD explicit half(float f) {
#if defined(__CUDA_ARCH__)
    __half h = __float2half_rn(f);
    x = *reinterpret_cast<uint16_t*>(&h);
#else
    x = tfs_detail::f32_to_f16_bits(f);
#endif
  }
  TFS_HD explicit operator float() const {
#if defined(__CUDA_ARCH__)
    __half h;
    *reinterpret_cast<uint16_t*>(&h) = x;
    return __half2float(h);
#else
    return tfs_detail::f16_bits_to_f32(x);
#endif
  }
};

TFS_HD inline half operator*(const half& a, const half& b) {
#if defined(__CUDA_ARCH__)
  __half ha, hb;
  *reinterpret_cast<uint16_t*>(&ha) = a.x;
  *reinterpret_cast<uint16_t*>(&hb) = b.x;
  __half r = __hmul(ha, hb);
  half out;
  out.x = *reinterpret_cast<uint16_t*>(&r);
  return out;
#else
  return half(static_cast<float>(a) * static_cast<float>(b));
#endif
}

namespace numext {
TFS_HD inline float exp(float v) {
#if defined(__CUDA_ARCH__)
  return ::expf(v);
#else
  return std::exp(v);
#endif
}
TFS_HD inline float log(float v) {
#if defined(__CUDA_ARCH__)
  return ::logf(v);
#else
  return std::log(v);
#endif
}
}  // namespace numext

struct TensorOpCost {
  TensorOpCost(double, double, double) {}
};

int tfs_num_threads();  // defined by the wrapper; number of host threads

struct ThreadPoolDevice {
  // Contiguous blocks of [0, n) across tfs_num_threads() std::threads.
  template <typename F>
  void parallelFor(long n, const TensorOpCost&, F f) const {
    if (n <= 0) return;
    long nt = tfs_num_threads();
    if (nt < 1) nt = 1;
    if (nt > n) nt = n;
    if (nt == 1) {
      f(0, n);
      return;
    }
    std::vector<std::thread> ts;
    for (long t = 0; t < nt; ++t) {
      long s = n * t / nt, e = n * (t + 1) / nt;
      ts.emplace_back([&f, s, e]() { f(s, e); });
    }
    for (auto& th : ts) th.join();
  }
};

struct GpuDevice {
  void* stream_ = nullptr;
#if defined(TFS_HAVE_CUDA_RT)
  cudaStream_t stream() const { return (cudaStream_t)stream_; }
#else
  void* stream() const { return stream_; }
#endif
};

}  // namespace Eigen

// ----------------------------------------------------------- TensorFlow part
namespace tensorflow {

typedef uint64_t uint64;
typedef int64_t int64;
typedef uint32_t uint32;
typedef int32_t int32;

// Row-major N-d view over caller memory (models Eigen::TensorMap).
template <typename T, int N>
struct TfsTensorMap {
  T* ptr = nullptr;
  long dims[N] = {};
  TFS_HD long dimension(int i) const { return dims[i]; }
  TFS_HD T* data() const { return ptr; }
  template <typename... I>
  TFS_HD T& operator()(I... idx) const {
    static_assert(sizeof...(I) == N, "rank mismatch");
    long ii[N] = {static_cast<long>(idx)...};
    long off = 0;
    for (int d = 0; d < N; ++d) off = off * dims[d] + ii[d];
    return ptr[off];
  }
  void setZero() const {
    long n = 1;
    for (int d = 0; d < N; ++d) n *= dims[d];
    for (long i = 0; i < n; ++i) ptr[i] = typename std::remove_const<T>::type(0.0f);
  }
};

template <typename T, int NDIMS = 1, typename IndexType = Eigen::DenseIndex>
struct TTypes {
  typedef TfsTensorMap<T, NDIMS> Tensor;
  typedef TfsTensorMap<const T, NDIMS> ConstTensor;
};

class Status {
 public:
  Status() = default;
  explicit Status(std::string m) : ok_(false), msg_(std::move(m)) {}
  bool ok() const { return ok_; }
  const std::string& message() const { return msg_; }
  std::string ToString() const { return ok_ ? "OK" : "INVALID_ARGUMENT: " + msg_; }

 private:
  bool ok_ = true;
  std::string msg_;
};
inline Status OkStatus() { return Status(); }

namespace errors {
inline Status InvalidArgument(const std::string& m) { return Status(m); }
inline Status Internal(const std::string& m) { return Status(m); }
}  // namespace errors

class TensorShape {
 public:
  TensorShape() = default;
  TensorShape(std::initializer_list<long> d) : dims_(d) {}
  explicit TensorShape(const std::vector<long>& d) : dims_(d) {}
  int dims() const { return (int)dims_.size(); }
  long dim_size(int i) const { return dims_[i]; }
  long num_elements() const {
    long n = 1;
    for (long d : dims_) n *= d;
    return n;
  }
  const std::vector<long>& dim_sizes() const { return dims_; }

 private:
  std::vector<long> dims_;
};

struct TensorShapeUtils {
  static bool IsScalar(const TensorShape& s) { return s.dims() == 0; }
};

class Tensor {
 public:
  Tensor() = default;
  Tensor(void* p, TensorShape s) : ptr_(p), shape_(std::move(s)) {}
  const TensorShape& shape() const { return shape_; }
  long dim_size(int i) const { return shape_.dim_size(i); }
  int dims() const { return shape_.dims(); }
  template <typename T>
  struct ScalarRef {
    const T* p;
    T operator()() const { return *p; }
  };
  template <typename T>
  ScalarRef<T> scalar() const { return ScalarRef<T>{static_cast<const T*>(ptr_)}; }
  template <typename T, int N>
  typename TTypes<T, N>::ConstTensor tensor() const {
    typename TTypes<T, N>::ConstTensor m;
    m.ptr = static_cast<const T*>(ptr_);
    for (int i = 0; i < N; ++i) m.dims[i] = shape_.dim_size(i);
    return m;
  }
  template <typename T, int N>
  typename TTypes<T, N>::Tensor tensor() {
    typename TTypes<T, N>::Tensor m;
    m.ptr = static_cast<T*>(ptr_);
    for (int i = 0; i < N; ++i) m.dims[i] = shape_.dim_size(i);
    return m;
  }
  void* raw() const { return ptr_; }
  long NumElements() const { return shape_.num_elements(); }
  template <typename T>
  typename TTypes<T, 1>::ConstTensor flat() const {
    typename TTypes<T, 1>::ConstTensor m;
    m.ptr = static_cast<const T*>(ptr_);
    m.dims[0] = shape_.num_elements();
    return m;
  }
  template <typename T>
  typename TTypes<T, 1>::Tensor flat() {
    typename TTypes<T, 1>::Tensor m;
    m.ptr = static_cast<T*>(ptr_);
    m.dims[0] = shape_.num_elements();
    return m;
  }

 private:
  void* ptr_ = nullptr;
  TensorShape shape_;
};

// Attribute values handed to the kernel constructor.
struct TfsAttrs {
  std::map<std::string, float> f;
  std::map<std::string, bool> b;
};

class OpKernelConstruction {
 public:
  explicit OpKernelConstruction(const TfsAttrs* a) : attrs_(a) {}
  Status GetAttr(const std::string& name, float* v) const {
    auto it = attrs_->f.find(name);
    if (it == attrs_->f.end()) return errors::InvalidArgument("missing attr " + name);
    *v = it->second;
    return OkStatus();
  }
  Status GetAttr(const std::string& name, bool* v) const {
    auto it = attrs_->b.find(name);
    if (it == attrs_->b.end()) return errors::InvalidArgument("missing attr " + name);
    *v = it->second;
    return OkStatus();
  }
  void CtxFailure(const Status& s) { status_ = s; }
  const Status& status() const { return status_; }

 private:
  const TfsAttrs* attrs_;
  Status status_;
};

enum DataType { DT_FLOAT = 1, DT_HALF = 19 };

class OpKernelContext {
 public:
  // Scratch handed out by allocate_temp: device memory when a CUDA runtime is
  // available and gpu_temp is set (a GPU kernel runs), host memory otherwise.
  bool gpu_temp = false;
  std::vector<void*> temps;
  ~OpKernelContext() {
    for (void* t : temps) {
#if defined(TFS_HAVE_CUDA_RT)
      if (gpu_temp) {
        cudaFree(t);
        continue;
      }
#endif
      std::free(t);
    }
  }
  Status allocate_temp(DataType dt, const TensorShape& s, Tensor* out) {
    size_t bytes = static_cast<size_t>(s.num_elements()) * (dt == DT_HALF ? 2 : 4);
    if (bytes == 0) bytes = 4;
    void* p = nullptr;
#if defined(TFS_HAVE_CUDA_RT)
    if (gpu_temp) {
      if (cudaMalloc(&p, bytes) != cudaSuccess) return errors::Internal("allocate_temp failed");
    } else
#endif
      p = std::malloc(bytes);
    temps.push_back(p);
    *out = Tensor(p, s);
    return OkStatus();
  }
  std::vector<Tensor> inputs;
  std::vector<void*> output_buffers;  // caller-owned memory for each output
  std::vector<Tensor> outputs;
  Eigen::ThreadPoolDevice cpu_device;
  Eigen::GpuDevice gpu_device;

  const Tensor& input(int i) const { return inputs[i]; }
  Status allocate_output(int i, const TensorShape& s, Tensor** out) {
    if (i >= (int)outputs.size()) return errors::Internal("output index out of range");
    outputs[i] = Tensor(output_buffers[i], s);
    *out = &outputs[i];
    return OkStatus();
  }
  template <typename D>
  const D& eigen_device() const;
  void CtxFailure(const Status& s) { status_ = s; }
  const Status& status() const { return status_; }

 private:
  Status status_;
};
template <>
inline const Eigen::ThreadPoolDevice& OpKernelContext::eigen_device<Eigen::ThreadPoolDevice>() const {
  return cpu_device;
}
template <>
inline const Eigen::GpuDevice& OpKernelContext::eigen_device<Eigen::GpuDevice>() const {
  return gpu_device;
}

class OpKernel {
 public:
  explicit OpKernel(OpKernelConstruction*) {}
  virtual ~OpKernel() = default;
  virtual void Compute(OpKernelContext* ctx) = 0;
};

#define OP_REQUIRES(CTX, EXP, STATUS) \
  do {                                \
    if (!(EXP)) {                     \
      (CTX)->CtxFailure(STATUS);      \
      return;                         \
    }                                 \
  } while (0)

#define OP_REQUIRES_OK(CTX, ...)       \
  do {                                 \
    ::tensorflow::Status _s(__VA_ARGS__); \
    if (!_s.ok()) {                    \
      (CTX)->CtxFailure(_s);           \
      return;                          \
    }                                  \
  } while (0)

#define TF_RETURN_IF_ERROR(...)           \
  do {                                    \
    ::tensorflow::Status _s(__VA_ARGS__); \
    if (!_s.ok()) return _s;              \
  } while (0)

// ---- kernel registry
enum TfsDType { TFS_FLOAT = 1, TFS_HALF = 19 };
template <typename T> struct TfsDTypeOf;
template <> struct TfsDTypeOf<float> { static constexpr int v = TFS_FLOAT; };
template <> struct TfsDTypeOf<Eigen::half> { static constexpr int v = TFS_HALF; };

static const char* const DEVICE_CPU = "CPU";
static const char* const DEVICE_GPU = "GPU";

struct TfsKernelDef {
  std::string op, device;
  int dtype = 0;
  std::vector<std::string> host_memory;
};

class Name {
 public:
  explicit Name(const char* op) { def_.op = op; }
  Name& Device(const char* d) {
    def_.device = d;
    return *this;
  }
  template <typename T>
  Name& TypeConstraint(const char*) {
    def_.dtype = TfsDTypeOf<T>::v;
    return *this;
  }
  Name& HostMemory(const char* n) {
    def_.host_memory.push_back(n);
    return *this;
  }
  const TfsKernelDef& def() const { return def_; }

 private:
  TfsKernelDef def_;
};

typedef std::function<OpKernel*(OpKernelConstruction*)> TfsFactory;
struct TfsRegistryEntry {
  TfsKernelDef def;
  TfsFactory factory;
};
std::vector<TfsRegistryEntry>& tfs_kernel_registry();  // defined by the wrapper

struct TfsKernelRegistrar {
  TfsKernelRegistrar(const Name& n, TfsFactory f) { tfs_kernel_registry().push_back({n.def(), std::move(f)}); }
};

#define TFS_CONCAT_INNER(a, b) a##b
#define TFS_CONCAT(a, b) TFS_CONCAT_INNER(a, b)
#define REGISTER_KERNEL_BUILDER(builder, ...)                                            \
  static ::tensorflow::TfsKernelRegistrar TFS_CONCAT(tfs_kernel_registrar_, __COUNTER__)( \
      ::tensorflow::builder,                                                             \
      [](::tensorflow::OpKernelConstruction* c) -> ::tensorflow::OpKernel* { return new __VA_ARGS__(c); })

// ---- GPU launch helper (models tensorflow::GpuLaunchKernel)
void tfs_record_launch_error(const char* what);  // defined by the wrapper
#define TF_CHECK_OK(...)                                  \
  do {                                                    \
    ::tensorflow::Status _s(__VA_ARGS__);                 \
    if (!_s.ok()) ::tensorflow::tfs_record_launch_error(_s.message().c_str()); \
  } while (0)

#if defined(__CUDACC__)
template <typename... KArgs, typename... Args>
Status GpuLaunchKernel(void (*kernel)(KArgs...), int grid, int block, int smem, cudaStream_t stream,
                       Args... args) {
  if (grid <= 0) return OkStatus();
  kernel<<<grid, block, smem, stream>>>(static_cast<KArgs>(args)...);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return errors::Internal(cudaGetErrorString(e));
  return OkStatus();
}
#endif

// ---- op registration (REGISTER_OP) -- recorded, not executed
namespace shape_inference {
struct ShapeHandle {
  int rank = -1;
};
struct DimensionHandle {
  long v = -1;
};
class InferenceContext {
 public:
  std::vector<std::vector<long>> in_shapes;
  std::vector<std::vector<long>> out_shapes;
  ShapeHandle input(int i) const {
    ShapeHandle h;
    h.rank = i;
    return h;
  }
  Status WithRank(ShapeHandle in, int rank, ShapeHandle* out) {
    if ((int)in_shapes[in.rank].size() != rank)
      return errors::InvalidArgument("Shape must be rank " + std::to_string(rank));
    *out = in;
    return OkStatus();
  }
  DimensionHandle Dim(ShapeHandle h, int d) const {
    DimensionHandle r;
    r.v = in_shapes[h.rank][d];
    return r;
  }
  ShapeHandle MakeShape(std::initializer_list<DimensionHandle> dims) {
    std::vector<long> s;
    for (auto& d : dims) s.push_back(d.v);
    pending_.push_back(s);
    ShapeHandle h;
    h.rank = -1 - (int)(pending_.size() - 1);
    return h;
  }
  void set_output(int i, ShapeHandle h) {
    if ((int)out_shapes.size() <= i) out_shapes.resize(i + 1);
    out_shapes[i] = h.rank >= 0 ? in_shapes[h.rank] : pending_[-1 - h.rank];
  }

 private:
  std::vector<std::vector<long>> pending_;
};
}  // namespace shape_inference

struct TfsOpDef {
  std::string name;
  std::vector<std::string> inputs, outputs, attrs;
  std::function<Status(shape_inference::InferenceContext*)> shape_fn;
};
std::vector<TfsOpDef>& tfs_op_registry();  // defined by the wrapper

class TfsOpDefBuilder {
 public:
  explicit TfsOpDefBuilder(const char* n) { d_.name = n; }
  TfsOpDefBuilder& Input(const char* s) {
    d_.inputs.push_back(s);
    return *this;
  }
  TfsOpDefBuilder& Output(const char* s) {
    d_.outputs.push_back(s);
    return *this;
  }
  TfsOpDefBuilder& Attr(const char* s) {
    d_.attrs.push_back(s);
    return *this;
  }
  template <typename F>
  TfsOpDefBuilder& SetShapeFn(F f) {
    d_.shape_fn = f;
    return *this;
  }
  const TfsOpDef& def() const { return d_; }

 private:
  TfsOpDef d_;
};
struct TfsOpRegistrar {
  TfsOpRegistrar(const TfsOpDefBuilder& b) { tfs_op_registry().push_back(b.def()); }
};
#define REGISTER_OP(name) \
  static ::tensorflow::TfsOpRegistrar TFS_CONCAT(tfs_op_registrar_, __COUNTER__) = ::tensorflow::TfsOpDefBuilder(name)

}  // namespace tensorflow
