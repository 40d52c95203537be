// oracle/_ref harness: one ONNX node through onnx-light's own RunNode on a GPU
// device -- test infrastructure only.
//
// The GPU tests call h_run_node to check the drop-in end to end: the node is
// built as a NodeProto, its inputs (device buffers) are placed in a
// RuntimeContext whose options name Device::kGPU0 + device, and
// RunNode (onnx_light/onnx_core/runtime/kernels/run_nodes.cc:1641) resolves the
// kernel through the device-keyed dispatch table (:1544-1604), where
// onnxl_b200::binding::RegisterB200KernelFunctions put the GPU kernels.  The
// outputs are copied into caller buffers.  Reference exceptions come back as
// status -1 with the message.
#include <cuda_runtime.h>

#include <cstring>
#include <exception>
#include <string>

#include "../include/onnxl_b200.h"
#include "../onnx-light_b200/binding/b200_kernels.h"
#include "onnx_core/runtime/kernels/run_nodes.h"
#include "onnx_core/runtime/runtime_context.h"
#include "onnx_core/symbolic/sym_tensor.h"
#include "onnx_extensions/kernels/kernels/math/include_math_kernels.h"

using namespace onnx_light;
using namespace onnx_light::core::runtime;
namespace sym = onnx_light::core::symbolic;

namespace {
void Fail(const std::exception &e, char *err, size_t errlen) {
  if (err && errlen) {
    std::strncpy(err, e.what(), errlen - 1);
    err[errlen - 1] = 0;
  }
}
} // namespace

extern "C" {

// Registers the GPU kernels for devices 0 .. ndev-1; returns the entries stored.
int h_register(int ndev) { return onnxl_b200::binding::RegisterB200KernelFunctions(ndev, false); }

// Runs one node.  Inputs: n_in descriptors of device buffers (a descriptor
// with ndim < 0 is an omitted optional input, named "").  Attributes: n_attr
// (name, kind 0 = INT / 1 = FLOAT, value).  Outputs: n_out slots; slot i is
// copied into out[i].data (capacity out_cap[i] bytes) and its dtype, rank and
// shape (up to 8 dims, out_shapes[8 i ..]) are written back; an output with
// out[i].data == NULL is not requested (empty name).
int h_run_node(const char *domain, const char *op_type, int device, int n_in, const b2_tensor *in,
               int n_attr, const char *const *attr_names, const int *attr_kinds,
               const int64_t *attr_i, const float *attr_f, int n_out, b2_tensor *out,
               const size_t *out_cap, int64_t *out_shapes, char *err, size_t errlen) {
  try {
    NodeProto node;
    node.set_op_type(op_type);
    node.set_domain(domain);
    RuntimeContextOptions opts;
    opts.device = sym::MakeGPUDevice(device);
    RuntimeContext rt(KernelContext(onnx_kernels::kernel::DefaultOpset(23)), opts);
    for (int i = 0; i < n_in; ++i) {
      if (in[i].ndim < 0) {
        node.add_input("");
        continue;
      }
      const std::string name = "in" + std::to_string(i);
      node.add_input(name);
      Shape shape(std::vector<int64_t>(in[i].shape, in[i].shape + in[i].ndim));
      int64_t n = 1;
      for (int d = 0; d < in[i].ndim; ++d) n *= in[i].shape[d];
      rt.tensors()[name] = Tensor::Borrow(name, in[i].dtype, shape,
                                          static_cast<const uint8_t *>(in[i].data),
                                          PackedByteSize(in[i].dtype, n));
    }
    for (int i = 0; i < n_out; ++i) node.add_output(out[i].data ? "out" + std::to_string(i) : "");
    for (int a = 0; a < n_attr; ++a) {
      AttributeProto attr;
      attr.set_name(attr_names[a]);
      if (attr_kinds[a] == 0) {
        attr.set_type(AttributeProto::INT);
        attr.set_i(attr_i[a]);
      } else {
        attr.set_type(AttributeProto::FLOAT);
        attr.set_f(attr_f[a]);
      }
      node.set_attribute(attr);
    }
    RunNode(node, rt);
    cudaStream_t st = onnxl_b200::binding::DeviceStream(device);
    for (int i = 0; i < n_out; ++i) {
      if (!out[i].data) continue;
      const Tensor &t = rt.tensors().at("out" + std::to_string(i));
      if (t.size_bytes() > out_cap[i]) throw std::runtime_error("h_run_node: output buffer too small");
      out[i].dtype = t.data_type;
      out[i].ndim = static_cast<int32_t>(t.shape.size());
      for (size_t d = 0; d < t.shape.size() && d < 8; ++d) out_shapes[8 * i + d] = t.shape[d];
      if (t.size_bytes() &&
          cudaMemcpyAsync(out[i].data, t.bytes(), t.size_bytes(), cudaMemcpyDeviceToDevice, st) !=
              cudaSuccess)
        throw std::runtime_error("h_run_node: output copy failed");
    }
    if (cudaStreamSynchronize(st) != cudaSuccess) throw std::runtime_error("h_run_node: stream failed");
    return 0;
  } catch (const std::exception &e) {
    Fail(e, err, errlen);
    return -1;
  }
}

// The dispatch key RunNode looks up for (domain, op_type) on GPU `device`.
int h_dispatch_key(const char *domain, const char *op_type, int device, char *buf, size_t len) {
  const std::string dom = (domain == nullptr || !*domain) ? "ai.onnx" : domain;
  const std::string key = dom + ":" + op_type + sym::DeviceKeySuffix(sym::MakeGPUDevice(device));
  std::strncpy(buf, key.c_str(), len - 1);
  buf[len - 1] = 0;
  return KernelDispatchTable().count(key) ? 1 : 0;
}

} // extern "C"
