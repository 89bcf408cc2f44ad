// Drives the reference's OWN registered OpKernels (SdpaFwdOp / SdpaBwdOp from
// sdpa/sdpa_cpu.cc, and on a GPU build the functors of sdpa/sdpa_fwd.cu.cc and
// sdpa/sdpa_bwd.cu.cc) through the mock TF types of tf_shim/, so the reference
// runs unmodified as a parity oracle and as the timed CPU baseline.
//
// TEST INFRASTRUCTURE ONLY: built into oracle/_ref/ by oracle/build_ref.sh and
// loaded by tests/, bench.py's reference arm and cpu_baseline leg.
#include "tf_shim/tf_shim_core.h"

#include <atomic>
#include <cstdlib>
#include <mutex>
#include <string>

namespace Eigen {
static std::atomic<int> g_threads{0};
int tfs_num_threads() {
  int n = g_threads.load();
  if (n > 0) return n;
  unsigned h = std::thread::hardware_concurrency();
  return h ? (int)h : 1;
}
}  // namespace Eigen

namespace tensorflow {
std::vector<TfsRegistryEntry>& tfs_kernel_registry() {
  static std::vector<TfsRegistryEntry> r;
  return r;
}
std::vector<TfsOpDef>& tfs_op_registry() {
  static std::vector<TfsOpDef> r;
  return r;
}
static std::mutex g_err_mu;
static std::string g_launch_err;
void tfs_record_launch_error(const char* what) {
  std::lock_guard<std::mutex> lk(g_err_mu);
  g_launch_err = what ? what : "launch error";
}
}  // namespace tensorflow

using namespace tensorflow;

extern "C" {

// Number of kernels the reference registered in this build (CPU: 4, GPU build: 8).
int ref_num_kernels() { return (int)tfs_kernel_registry().size(); }

// Describes registered kernel i: op name, device, dtype (1 float, 19 half).
int ref_kernel_info(int i, char* op, int oplen, char* dev, int devlen, int* dtype) {
  auto& r = tfs_kernel_registry();
  if (i < 0 || i >= (int)r.size()) return -1;
  std::snprintf(op, oplen, "%s", r[i].def.op.c_str());
  std::snprintf(dev, devlen, "%s", r[i].def.device.c_str());
  *dtype = r[i].def.dtype;
  return 0;
}

// Host threads used by the reference's CPU parallelFor (0 = all cores).
void ref_set_num_threads(int n) { Eigen::g_threads.store(n); }
int ref_get_num_threads() { return Eigen::tfs_num_threads(); }

// Runs one registered kernel.
//   op      "Sdpa" or "SdpaGrad";   device "CPU" or "GPU";   dtype 1 (float) / 19 (half)
//   in_ptrs/in_ranks/in_dims   every input tensor (dims flattened, rank-0 scalars take none)
//   out_ptrs                    caller-owned memory for every output
//   out_dims                    receives the output shapes (rank 3 or 2, padded to 3 with -1)
// Returns 0 on success, 1 when the kernel rejected its inputs (message in err),
// 2 when no kernel is registered for (op, device, dtype), 3 on a GPU launch error.
int ref_run(const char* op, const char* device, int dtype, int n_in, void** in_ptrs, const long* in_ranks,
            const long* in_dims, int n_out, void** out_ptrs, long* out_dims, float scale, float dropout,
            int causal, void* stream, char* err, int errlen) {
  const TfsRegistryEntry* entry = nullptr;
  for (auto& e : tfs_kernel_registry())
    if (e.def.op == op && e.def.device == device && e.def.dtype == dtype) entry = &e;
  if (!entry) {
    std::snprintf(err, errlen, "no kernel registered for %s/%s/%d", op, device, dtype);
    return 2;
  }
  TfsAttrs attrs;
  attrs.f["scale"] = scale;
  attrs.f["dropout"] = dropout;
  attrs.b["causal_mask"] = causal != 0;
  OpKernelConstruction cons(&attrs);
  OpKernel* k = entry->factory(&cons);
  if (!cons.status().ok()) {
    std::snprintf(err, errlen, "%s", cons.status().message().c_str());
    delete k;
    return 1;
  }
  OpKernelContext ctx;
  long off = 0;
  for (int i = 0; i < n_in; ++i) {
    std::vector<long> d(in_dims + off, in_dims + off + in_ranks[i]);
    off += in_ranks[i];
    ctx.inputs.emplace_back(in_ptrs[i], TensorShape(d));
  }
  ctx.output_buffers.assign(out_ptrs, out_ptrs + n_out);
  ctx.outputs.resize(n_out);  // allocate_output hands out pointers into this vector
  ctx.gpu_device.stream_ = stream;
  ctx.gpu_temp = std::string(device) == "GPU";
  {
    std::lock_guard<std::mutex> lk(g_err_mu);
    g_launch_err.clear();
  }
  k->Compute(&ctx);
  delete k;
  if (!ctx.status().ok()) {
    std::snprintf(err, errlen, "%s", ctx.status().message().c_str());
    return 1;
  }
  for (int i = 0; i < n_out; ++i) {
    for (int d = 0; d < 3; ++d) out_dims[i * 3 + d] = -1;
    if (i < (int)ctx.outputs.size())
      for (int d = 0; d < ctx.outputs[i].dims() && d < 3; ++d) out_dims[i * 3 + d] = ctx.outputs[i].dim_size(d);
  }
  std::lock_guard<std::mutex> lk(g_err_mu);
  if (!g_launch_err.empty()) {
    std::snprintf(err, errlen, "%s", g_launch_err.c_str());
    return 3;
  }
  return 0;
}

}  // extern "C"
