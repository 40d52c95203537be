// onnx-light drop-in for the B200 kernels: KernelBase subclasses that the
// reference runtime resolves for Device::kGPU0 + i, each a thin C++ layer over
// the C ABI of include/onnxl_b200.h.
//
// Registration follows onnx_kernels::RegisterKernelFunctions
// (onnx_light/onnx_extensions/kernels/kernel_dispatch_table.cc:83-90, 477):
// one NodeKernelFn factory per (domain, op_type, device), registered through
// RegisterKernelFn (onnx_light/onnx_core/runtime/kernels/kernel_dispatch_table.h:148-164),
// so a RuntimeContext whose options name a GPU device resolves these kernels in
// RunNode (onnx_light/onnx_core/runtime/kernels/run_nodes.cc:1544-1604) and an
// operator without a GPU kernel still fails there with the device named.
//
// Device tensors.  The reference's RawBuffer owns a host std::vector
// (onnx_light/onnx_core/runtime/memory/simple_tensor.h:354-434), so device
// memory cannot come from a RawBufferAllocator.  It enters the runtime as
// Tensor::Borrow views (simple_tensor.h:612) whose owner releases the device
// allocation (stream-ordered cudaFreeAsync) when the last Tensor copy is
// dropped: outputs are owned by whoever holds them, as the reference's
// allocator-backed outputs are.  Inputs may be device tensors (used in place)
// or host tensors (copied to the device before the call; an initializer is
// better uploaded once with MakeDeviceTensor).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "onnx_core/runtime/kernels/kernel_dispatch_table.h"

namespace onnxl_b200::binding {

namespace ort = onnx_light::core::runtime;

/// Registers the GPU kernels for Device::kGPU0 .. kGPU0 + device_count - 1:
/// ai.onnx DequantizeLinear, MatMulInteger, QLinearMatMul, Attention,
/// RMSNormalization, RotaryEmbedding, SwiGLU and the fused node
/// b200:DequantizeMatMul (DequantizeLinear -> [Cast] -> MatMul; a pattern pass
/// rewrites the node pair into it).  With overwrite == false an
/// existing entry is kept, like the reference's built-in registration.
/// Returns the number of entries stored.
int RegisterB200KernelFunctions(int device_count, bool overwrite = false);

/// The stream every kernel of this binding runs on for GPU `device` (created
/// on first use, non-blocking).  Outputs are complete once it has drained.
cudaStream_t DeviceStream(int device);

/// A device tensor of the given type and shape on GPU `device`: a borrowed
/// view of a stream-ordered allocation that is released when the last copy
/// of the returned Tensor goes away.
ort::Tensor MakeDeviceTensor(int32_t dtype, const ort::Shape &shape, int device);

/// Copies a host tensor to a new device tensor (stream-ordered on
/// DeviceStream(device)).
ort::Tensor UploadTensor(const ort::Tensor &host, int device);

} // namespace onnxl_b200::binding
