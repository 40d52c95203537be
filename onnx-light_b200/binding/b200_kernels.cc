// onnx-light KernelBase subclasses over the onnxl_b200 C ABI (see
// b200_kernels.h).  Each Run() mirrors the reference kernel's Run() -- the
// same input and output counts, attribute names and defaults -- then hands
// device pointers to the C entry point and stores device tensors as outputs:
//   DequantizeLinear  kernel_dequantizelinear.cc:695-712 -> b2_dequantize_linear
//   MatMulInteger     kernel_matmul_integer.cc:236-250   -> b2_matmul_integer
//   QLinearMatMul     kernel_qlinearmatmul.cc:269-284    -> b2_qlinear_matmul
//   Attention         kernel_attention.cc:855-902        -> b2_attention_ex
//   RMSNormalization  kernel_rmsnormalization.cc:216-223 -> b2_rms_normalization
//   RotaryEmbedding   kernel_rotary_embedding.cc:220-240 -> b2_rotary_embedding
//   SwiGLU            kernel_swiglu.cc:119-127           -> b2_swiglu
//   b200:DequantizeMatMul (DequantizeLinear -> [Cast] -> MatMul) -> b2_dequantize_matmul
// A negative status becomes std::invalid_argument (the reference's
// EXT_ENFORCE_INVALID) for invalid arguments and dtypes, std::runtime_error
// otherwise, with the library's "kernel::<Op>:" message.
#include "b200_kernels.h"

#include <cstring>
#include <deque>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/onnxl_b200.h"
#include "onnx_core/runtime/kernels/node_helpers.h"
#include "onnx_core/runtime/runtime_context.h"
#include "onnx_core/symbolic/sym_tensor.h"

namespace onnxl_b200::binding {

namespace sym = onnx_light::core::symbolic;
using ort::KernelBase;
using ort::KernelContext;
using onnx_light::NodeProto;
using ort::RuntimeContext;
using ort::Shape;
using ort::Tensor;

namespace {

constexpr int kMaxDevices = 64;

void CudaCheck(cudaError_t e, const char *what) {
  if (e != cudaSuccess)
    throw std::runtime_error(std::string("onnxl_b200 binding: ") + what + ": " + cudaGetErrorString(e));
}

// Raises the C ABI's error as the reference would raise it.
void Check(int rc) {
  if (rc == B2_OK) return;
  char msg[1024];
  b2_last_error(msg, sizeof(msg));
  if (rc == B2_ERR_INVALID_ARGUMENT || rc == B2_ERR_UNSUPPORTED_DTYPE) throw std::invalid_argument(msg);
  throw std::runtime_error(msg);
}

int64_t Numel(const Shape &s) {
  int64_t n = 1;
  for (auto d : s) n *= static_cast<int64_t>(d);
  return n;
}

// Makes `device` current for the lifetime of the guard.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int device) {
    CudaCheck(cudaGetDevice(&prev), "cudaGetDevice");
    if (prev != device) CudaCheck(cudaSetDevice(device), "cudaSetDevice");
  }
  ~DeviceGuard() {
    int cur = -1;
    if (cudaGetDevice(&cur) == cudaSuccess && cur != prev && prev >= 0) cudaSetDevice(prev);
  }
};

bool IsDevicePointer(const void *p) {
  if (p == nullptr) return false;
  cudaPointerAttributes attr{};
  if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged;
}

// A b2_tensor view of a Tensor (shape storage kept alongside).
struct Desc {
  std::vector<int64_t> shape;
  b2_tensor t{};
  explicit Desc(const Tensor &x) {
    shape.assign(x.shape.begin(), x.shape.end());
    t.data = const_cast<uint8_t *>(x.bytes());
    t.dtype = x.data_type;
    t.ndim = static_cast<int32_t>(shape.size());
    t.shape = shape.data();
  }
  b2_tensor *ptr() { return &t; }
};

// NumPy MatMul output shape with a rank >= 1 left operand
// (onnx_light/onnx_core/runtime/kernels/matmul_shape_utils.h:24-108).
Shape MatMulShape(const Shape &a, const Shape &b) {
  std::vector<int64_t> a2(a.begin(), a.end()), b2(b.begin(), b.end());
  if (a2.size() == 1) a2.insert(a2.begin(), 1);
  if (b2.size() == 1) b2.push_back(1);
  std::vector<int64_t> ap(a2.begin(), a2.end() - 2), bp(b2.begin(), b2.end() - 2);
  const size_t r = std::max(ap.size(), bp.size());
  ap.insert(ap.begin(), r - ap.size(), 1);
  bp.insert(bp.begin(), r - bp.size(), 1);
  Shape out;
  for (size_t i = 0; i < r; ++i) out.push_back((ap[i] == 1) ? bp[i] : ap[i]);
  if (a.size() != 1) out.push_back(a2[a2.size() - 2]);
  if (b.size() != 1) out.push_back(b2.back());
  return out;
}

bool HasOutput(const NodeProto &node, int slot) {
  return slot < node.output_size() && !std::string(node.output(slot)).empty();
}

// Base of the GPU kernels: the device of the resolving context, inputs made
// device-resident, a kernel-owned workspace (zero-filled once, as the C ABI
// requires, and grown stream-ordered).
class GpuKernel : public KernelBase {
public:
  using KernelBase::KernelBase;

protected:
  int device_ = -1;
  std::shared_ptr<void> workspace_;
  size_t workspace_bytes_ = 0;
  std::deque<Tensor> staged_; // host inputs copied for the current call (stable references)

  void Bind(RuntimeContext &rt) {
    const int idx = sym::GPUIndex(rt.device());
    if (idx < 0) throw std::invalid_argument("onnxl_b200 binding: the context's device is not a GPU");
    device_ = idx;
    staged_.clear();
  }
  cudaStream_t stream() const { return DeviceStream(device_); }

  // The tensor itself when its bytes are device memory, else a device copy.
  const Tensor &OnDevice(const Tensor &t) {
    if (t.size_bytes() == 0 || IsDevicePointer(t.bytes())) return t;
    staged_.push_back(UploadTensor(t, device_));
    return staged_.back();
  }
  const Tensor *OnDevice(const Tensor *t) { return t ? &OnDevice(*t) : nullptr; }

  // Runs `call(workspace, &bytes)` once as a size query and once for real
  // (with no workspace at all when the plan needs none: a NULL workspace with
  // a size pointer is a size query, header of onnxl_b200.h).
  template <class F> void WithWorkspace(F call) {
    size_t need = 0;
    Check(call(nullptr, &need));
    if (need == 0) {
      Check(call(nullptr, nullptr));
      return;
    }
    if (need > workspace_bytes_) {
      DeviceGuard g(device_);
      if (workspace_) workspace_.reset();
      void *p = nullptr;
      CudaCheck(cudaMallocAsync(&p, need, stream()), "cudaMallocAsync (workspace)");
      CudaCheck(cudaMemsetAsync(p, 0, need, stream()), "cudaMemsetAsync (workspace)");
      const int dev = device_;
      cudaStream_t st = stream();
      workspace_ = std::shared_ptr<void>(p, [dev, st](void *q) {
        DeviceGuard gg(dev);
        cudaFreeAsync(q, st);
      });
      workspace_bytes_ = need;
    }
    size_t cap = workspace_bytes_;
    Check(call(workspace_.get(), &cap));
  }
};

class CudaDequantizeLinear final : public GpuKernel {
public:
  using GpuKernel::GpuKernel;
  void Run(RuntimeContext &rt) override {
    const NodeProto &node = *node_;
    ort::RequireMinInputCount(node, 2);
    if (node.input_size() > 3)
      throw std::invalid_argument("RunNode: op 'DequantizeLinear' expects 2 or 3 inputs, got " +
                                  std::to_string(node.input_size()) + ".");
    ort::RequireOutputCount(node, 1);
    Bind(rt);
    const Tensor &x = OnDevice(ort::GetInput(node, 0, rt));
    const Tensor &s = OnDevice(ort::GetInput(node, 1, rt));
    const Tensor *zp = OnDevice(ort::GetOptionalInput(node, 2, rt));
    const int64_t axis = ort::GetAttributeIntOrDefault(node, "axis", 1);
    Tensor y = MakeDeviceTensor(s.data_type, x.shape, device_);
    Desc dx(x), ds(s), dy(y);
    std::unique_ptr<Desc> dz(zp ? new Desc(*zp) : nullptr);
    Check(b2_dequantize_linear(dx.ptr(), ds.ptr(), dz ? dz->ptr() : nullptr, axis, dy.ptr(),
                               stream()));
    ort::SetOutput(node, 0, std::move(y), rt);
  }
};

class CudaMatMulInteger final : public GpuKernel {
public:
  using GpuKernel::GpuKernel;
  void Run(RuntimeContext &rt) override {
    const NodeProto &node = *node_;
    ort::RequireMinInputCount(node, 2);
    if (node.input_size() > 4)
      throw std::invalid_argument("RunNode: op 'MatMulInteger' expects at most 4 inputs, got " +
                                  std::to_string(node.input_size()) + ".");
    ort::RequireOutputCount(node, 1);
    Bind(rt);
    const Tensor &a = OnDevice(ort::GetInput(node, 0, rt));
    const Tensor &b = OnDevice(ort::GetInput(node, 1, rt));
    const Tensor *az = OnDevice(ort::GetOptionalInput(node, 2, rt));
    const Tensor *bz = OnDevice(ort::GetOptionalInput(node, 3, rt));
    Tensor y = MakeDeviceTensor(6 /* INT32 */, MatMulShape(a.shape, b.shape), device_);
    Desc da(a), db(b), dy(y);
    std::unique_ptr<Desc> daz(az ? new Desc(*az) : nullptr), dbz(bz ? new Desc(*bz) : nullptr);
    WithWorkspace([&](void *ws, size_t *bytes) {
      return b2_matmul_integer(da.ptr(), db.ptr(), daz ? daz->ptr() : nullptr,
                               dbz ? dbz->ptr() : nullptr, dy.ptr(), ws, bytes, stream());
    });
    ort::SetOutput(node, 0, std::move(y), rt);
  }
};

class CudaQLinearMatMul final : public GpuKernel {
public:
  using GpuKernel::GpuKernel;
  void Run(RuntimeContext &rt) override {
    const NodeProto &node = *node_;
    ort::RequireInputCount(node, 8);
    ort::RequireOutputCount(node, 1);
    Bind(rt);
    std::vector<const Tensor *> in(8);
    for (int i = 0; i < 8; ++i) in[i] = &OnDevice(ort::GetInput(node, i, rt));
    Tensor y = MakeDeviceTensor(in[7]->data_type, MatMulShape(in[0]->shape, in[3]->shape), device_);
    std::vector<std::unique_ptr<Desc>> d;
    for (int i = 0; i < 8; ++i) d.emplace_back(new Desc(*in[i]));
    Desc dy(y);
    WithWorkspace([&](void *ws, size_t *bytes) {
      return b2_qlinear_matmul(d[0]->ptr(), d[1]->ptr(), d[2]->ptr(), d[3]->ptr(), d[4]->ptr(),
                               d[5]->ptr(), d[6]->ptr(), d[7]->ptr(), dy.ptr(), ws, bytes,
                               stream());
    });
    ort::SetOutput(node, 0, std::move(y), rt);
  }
};

class CudaAttention final : public GpuKernel {
public:
  using GpuKernel::GpuKernel;
  void Run(RuntimeContext &rt) override {
    const NodeProto &node = *node_;
    if (node.input_size() < 3 || node.input_size() > 7)
      throw std::invalid_argument("RunNode: op '" + std::string(node.op_type()) +
                                  "' expects between 3 and 7 input(s), got " +
                                  std::to_string(node.input_size()) + ".");
    if (node.output_size() < 1 || node.output_size() > 4)
      throw std::invalid_argument("RunNode: op '" + std::string(node.op_type()) +
                                  "' expects between 1 and 4 output(s), got " +
                                  std::to_string(node.output_size()) + ".");
    Bind(rt);
    const Tensor &q = OnDevice(ort::GetInput(node, 0, rt));
    const Tensor &k = OnDevice(ort::GetInput(node, 1, rt));
    const Tensor &v = OnDevice(ort::GetInput(node, 2, rt));
    const Tensor *mask = OnDevice(ort::GetOptionalInput(node, 3, rt));
    const Tensor *pk = OnDevice(ort::GetOptionalInput(node, 4, rt));
    const Tensor *pv = OnDevice(ort::GetOptionalInput(node, 5, rt));
    const Tensor *nonpad = OnDevice(ort::GetOptionalInput(node, 6, rt));
    b2_attention_attrs at{};
    at.has_scale = ort::FindAttribute(node, "scale") != nullptr;
    at.scale = ort::GetAttributeFloatOrDefault(node, "scale", 0.0f);
    at.is_causal = ort::GetAttributeIntOrDefault(node, "is_causal", 0) != 0;
    at.softcap = ort::GetAttributeFloatOrDefault(node, "softcap", 0.0f);
    at.qk_matmul_output_mode =
        static_cast<int32_t>(ort::GetAttributeIntOrDefault(node, "qk_matmul_output_mode", 0));
    at.q_num_heads = ort::GetAttributeIntOrDefault(node, "q_num_heads", 0);
    at.kv_num_heads = ort::GetAttributeIntOrDefault(node, "kv_num_heads", 0);
    at.left_window_size = ort::GetAttributeIntOrDefault(node, "left_window_size", -1);
    at.right_window_size = ort::GetAttributeIntOrDefault(node, "right_window_size", -1);
    at.kv_capacity = 0;
    // Output shapes (kernel_attention.cc:179-214, 462-476, 520-527).
    const bool rank3 = q.shape.size() == 3;
    if (!rank3 && q.shape.size() != 4)
      throw std::invalid_argument("kernel::Attention: Q, K, V must be rank-3 or rank-4.");
    int64_t B = q.shape[0], Hq, Sq, Hkv, D, Dv, Sk;
    if (rank3) {
      Hq = at.q_num_heads;
      Hkv = at.kv_num_heads;
      if (Hq <= 0 || Hkv <= 0)
        throw std::invalid_argument("kernel::Attention: 'Q' needs a positive ``num_heads`` to promote rank-3.");
      Sq = q.shape[1];
      D = q.shape[2] / Hq;
      Dv = v.shape[2] / Hkv;
      Sk = k.shape[1];
    } else {
      Hq = q.shape[1];
      Sq = q.shape[2];
      Hkv = k.shape[1];
      D = q.shape[3];
      Dv = v.shape[3];
      Sk = k.shape[2];
    }
    const int64_t P = pk ? static_cast<int64_t>(pk->shape.size() == 4 ? pk->shape[2] : 0) : 0;
    const int64_t L = P + Sk;
    Shape yshape = rank3 ? Shape{B, Sq, Hq * Dv} : Shape{B, Hq, Sq, Dv};
    Tensor y = MakeDeviceTensor(q.data_type, yshape, device_);
    const bool want_pk = HasOutput(node, 1) || pk != nullptr;
    const bool want_pv = HasOutput(node, 2) || pv != nullptr;
    Tensor prk, prv, qk;
    if (want_pk && want_pv) {
      prk = MakeDeviceTensor(q.data_type, Shape{B, Hkv, L, D}, device_);
      prv = MakeDeviceTensor(q.data_type, Shape{B, Hkv, L, Dv}, device_);
    }
    if (HasOutput(node, 3)) qk = MakeDeviceTensor(q.data_type, Shape{B, Hq, Sq, L}, device_);
    Desc dq(q), dk(k), dv(v), dy(y);
    std::unique_ptr<Desc> dm(mask ? new Desc(*mask) : nullptr), dpk(pk ? new Desc(*pk) : nullptr),
        dpv(pv ? new Desc(*pv) : nullptr), dnp(nonpad ? new Desc(*nonpad) : nullptr);
    std::unique_ptr<Desc> dprk(want_pk && want_pv ? new Desc(prk) : nullptr),
        dprv(want_pk && want_pv ? new Desc(prv) : nullptr), dqk(HasOutput(node, 3) ? new Desc(qk) : nullptr);
    WithWorkspace([&](void *ws, size_t *bytes) {
      return b2_attention_ex(dq.ptr(), dk.ptr(), dv.ptr(), dm ? dm->ptr() : nullptr,
                             dpk ? dpk->ptr() : nullptr, dpv ? dpv->ptr() : nullptr,
                             dnp ? dnp->ptr() : nullptr, &at, dy.ptr(),
                             dprk ? dprk->ptr() : nullptr, dprv ? dprv->ptr() : nullptr,
                             dqk ? dqk->ptr() : nullptr, ws, bytes, stream());
    });
    ort::SetOutput(node, 0, std::move(y), rt);
    if (HasOutput(node, 1)) ort::SetOutput(node, 1, std::move(prk), rt);
    if (HasOutput(node, 2)) ort::SetOutput(node, 2, std::move(prv), rt);
    if (HasOutput(node, 3)) ort::SetOutput(node, 3, std::move(qk), rt);
  }
};

// RMSNormalization (kernel_rmsnormalization.cc:216-223): X, scale; axis
// (default -1), epsilon (default 1e-5).
class CudaRMSNormalization final : public GpuKernel {
public:
  using GpuKernel::GpuKernel;
  void Run(RuntimeContext &rt) override {
    const NodeProto &node = *node_;
    ort::RequireInputCount(node, 2);
    ort::RequireOutputCount(node, 1);
    Bind(rt);
    const Tensor &x = OnDevice(ort::GetInput(node, 0, rt));
    const Tensor &s = OnDevice(ort::GetInput(node, 1, rt));
    Tensor y = MakeDeviceTensor(x.data_type, x.shape, device_);
    Desc dx(x), ds(s), dy(y);
    Check(b2_rms_normalization(dx.ptr(), ds.ptr(), ort::GetAttributeIntOrDefault(node, "axis", -1),
                               ort::GetAttributeFloatOrDefault(node, "epsilon", 1e-5f), dy.ptr(),
                               stream()));
    ort::SetOutput(node, 0, std::move(y), rt);
  }
};

// RotaryEmbedding (kernel_rotary_embedding.cc:220-240): X, cos_cache,
// sin_cache [, position_ids]; interleaved, rotary_embedding_dim, num_heads.
class CudaRotaryEmbedding final : public GpuKernel {
public:
  using GpuKernel::GpuKernel;
  void Run(RuntimeContext &rt) override {
    const NodeProto &node = *node_;
    if (node.input_size() < 3 || node.input_size() > 4)
      throw std::invalid_argument("RunNode: op '" + std::string(node.op_type()) +
                                  "' expects between 3 and 4 input(s), got " +
                                  std::to_string(node.input_size()) + ".");
    ort::RequireOutputCount(node, 1);
    Bind(rt);
    const Tensor &x = OnDevice(ort::GetInput(node, 0, rt));
    const Tensor &c = OnDevice(ort::GetInput(node, 1, rt));
    const Tensor &s = OnDevice(ort::GetInput(node, 2, rt));
    const Tensor *pos = OnDevice(ort::GetOptionalInput(node, 3, rt));
    Tensor y = MakeDeviceTensor(x.data_type, x.shape, device_);
    Desc dx(x), dc(c), ds(s), dy(y);
    std::unique_ptr<Desc> dp(pos ? new Desc(*pos) : nullptr);
    Check(b2_rotary_embedding(
        dx.ptr(), dc.ptr(), ds.ptr(), dp ? dp->ptr() : nullptr,
        ort::GetAttributeIntOrDefault(node, "interleaved", 0) != 0,
        ort::GetAttributeIntOrDefault(node, "rotary_embedding_dim", 0),
        ort::GetAttributeIntOrDefault(node, "num_heads", 0), dy.ptr(), stream()));
    ort::SetOutput(node, 0, std::move(y), rt);
  }
};

// SwiGLU (kernel_swiglu.cc:119-127): A, B; alpha (default 1).
class CudaSwiGLU final : public GpuKernel {
public:
  using GpuKernel::GpuKernel;
  void Run(RuntimeContext &rt) override {
    const NodeProto &node = *node_;
    ort::RequireInputCount(node, 2);
    ort::RequireOutputCount(node, 1);
    Bind(rt);
    const Tensor &a = OnDevice(ort::GetInput(node, 0, rt));
    const Tensor &b = OnDevice(ort::GetInput(node, 1, rt));
    Tensor y = MakeDeviceTensor(a.data_type, a.shape, device_);
    Desc da(a), db(b), dy(y);
    Check(b2_swiglu(da.ptr(), db.ptr(), ort::GetAttributeFloatOrDefault(node, "alpha", 1.0f),
                    dy.ptr(), stream()));
    ort::SetOutput(node, 0, std::move(y), rt);
  }
};

// b200:DequantizeMatMul(A, W, W_scale [, W_zero_point]) with attributes axis
// (of the DequantizeLinear, default 0 for a [K, N] weight) and cast_to (the
// ONNX dtype of a Cast between the two nodes, 0 for none).
class CudaDequantizeMatMul final : public GpuKernel {
public:
  using GpuKernel::GpuKernel;
  void Run(RuntimeContext &rt) override {
    const NodeProto &node = *node_;
    ort::RequireMinInputCount(node, 3);
    if (node.input_size() > 4)
      throw std::invalid_argument("RunNode: op 'DequantizeMatMul' expects 3 or 4 inputs, got " +
                                  std::to_string(node.input_size()) + ".");
    ort::RequireOutputCount(node, 1);
    Bind(rt);
    const Tensor &a = OnDevice(ort::GetInput(node, 0, rt));
    const Tensor &w = OnDevice(ort::GetInput(node, 1, rt));
    const Tensor &s = OnDevice(ort::GetInput(node, 2, rt));
    const Tensor *zp = OnDevice(ort::GetOptionalInput(node, 3, rt));
    const int64_t axis = ort::GetAttributeIntOrDefault(node, "axis", 0);
    const int32_t cast_to = static_cast<int32_t>(ort::GetAttributeIntOrDefault(node, "cast_to", 0));
    Tensor y = MakeDeviceTensor(a.data_type, MatMulShape(a.shape, w.shape), device_);
    Desc da(a), dw(w), ds(s), dy(y);
    std::unique_ptr<Desc> dz(zp ? new Desc(*zp) : nullptr);
    WithWorkspace([&](void *ws, size_t *bytes) {
      return b2_dequantize_matmul(da.ptr(), dw.ptr(), ds.ptr(), dz ? dz->ptr() : nullptr, axis,
                                  cast_to, dy.ptr(), ws, bytes, stream());
    });
    ort::SetOutput(node, 0, std::move(y), rt);
  }
};

// The factory the dispatch table stores: constructs the kernel from the
// node's KernelContext and attaches the node (MakeKernel,
// onnx_light/onnx_extensions/kernels/kernel_dispatch_table.cc:83-90).
template <class K> ort::NodeKernelFn Factory() {
  return [](const NodeProto &node, RuntimeContext &,
            const KernelContext &kernel_context) -> std::unique_ptr<KernelBase> {
    auto kernel = std::make_unique<K>(kernel_context);
    kernel->set_node(node);
    return kernel;
  };
}

std::mutex g_stream_mu;
cudaStream_t g_streams[kMaxDevices] = {};

} // namespace

cudaStream_t DeviceStream(int device) {
  if (device < 0 || device >= kMaxDevices) throw std::out_of_range("onnxl_b200 binding: device index");
  std::lock_guard<std::mutex> lock(g_stream_mu);
  if (g_streams[device] == nullptr) {
    DeviceGuard g(device);
    CudaCheck(cudaStreamCreateWithFlags(&g_streams[device], cudaStreamNonBlocking),
              "cudaStreamCreateWithFlags");
  }
  return g_streams[device];
}

Tensor MakeDeviceTensor(int32_t dtype, const Shape &shape, int device) {
  const size_t bytes = ort::PackedByteSize(dtype, Numel(shape));
  cudaStream_t st = DeviceStream(device);
  DeviceGuard g(device);
  void *p = nullptr;
  if (bytes) CudaCheck(cudaMallocAsync(&p, bytes, st), "cudaMallocAsync");
  std::shared_ptr<void> owner(p, [device, st](void *q) {
    if (q == nullptr) return;
    DeviceGuard gg(device);
    cudaFreeAsync(q, st);
  });
  return Tensor::Borrow("", dtype, shape, static_cast<const uint8_t *>(p), bytes, owner);
}

Tensor UploadTensor(const Tensor &host, int device) {
  Tensor t = MakeDeviceTensor(host.data_type, host.shape, device);
  if (host.size_bytes()) {
    DeviceGuard g(device);
    CudaCheck(cudaMemcpyAsync(const_cast<uint8_t *>(t.bytes()), host.bytes(), host.size_bytes(),
                              cudaMemcpyHostToDevice, DeviceStream(device)),
              "cudaMemcpyAsync (upload)");
    // the host tensor may go away once the call returns
    CudaCheck(cudaStreamSynchronize(DeviceStream(device)), "cudaStreamSynchronize (upload)");
  }
  return t;
}

int RegisterB200KernelFunctions(int device_count, bool overwrite) {
  struct Entry {
    const char *domain, *op;
    ort::NodeKernelFn fn;
  };
  const Entry entries[] = {
      {"", "DequantizeLinear", Factory<CudaDequantizeLinear>()},
      {"", "MatMulInteger", Factory<CudaMatMulInteger>()},
      {"", "QLinearMatMul", Factory<CudaQLinearMatMul>()},
      {"", "Attention", Factory<CudaAttention>()},
      {"", "RMSNormalization", Factory<CudaRMSNormalization>()},
      {"", "RotaryEmbedding", Factory<CudaRotaryEmbedding>()},
      {"", "SwiGLU", Factory<CudaSwiGLU>()},
      {"b200", "DequantizeMatMul", Factory<CudaDequantizeMatMul>()},
  };
  int stored = 0;
  for (int i = 0; i < device_count; ++i)
    for (const Entry &e : entries)
      stored += ort::RegisterKernelFn(e.domain, e.op, sym::MakeGPUDevice(i), e.fn, overwrite) ? 1 : 0;
  return stored;
}

} // namespace onnxl_b200::binding
