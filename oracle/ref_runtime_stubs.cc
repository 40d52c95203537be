// oracle/_ref runtime stubs -- test infrastructure only.
//
// oracle/_ref/libref_runtime.so hosts the GPU drop-in (onnx-light_b200/binding)
// in onnx-light's own node runtime, compiled from the reference sources by
// oracle/Makefile (target `runtime`): RuntimeContext, the kernel dispatch
// table, RunNode's kernel resolution, the value store and the node helpers run
// as the reference wrote them.  These definitions stand in for the few
// symbols those sources reference but that a single-node run never reaches:
// packed-weight reconstruction codecs, BLAKE3 hashing (its vendored build
// wants TBB) and one shape-inference event logger.  Each throws if called.
#include "onnx_core/runtime/gguf.h"
#include "onnx_core/runtime/quantization.h"
#include "onnx_core/shapes/shapes_context.h"
#include "onnx_proto/blake3/blake3_hash.h"

#include <stdexcept>
#include <string>

namespace {
[[noreturn]] void NotOnNodePath(const char *what) {
  throw std::logic_error(std::string("oracle/_ref runtime: symbol outside the node path called: ") + what);
}
} // namespace

namespace onnx_light::core::runtime {
Tensor DequantizeGgufTensorPayload(const EncodedValueProto &, size_t, const StructTypeCatalogue &,
                                   RawBufferAllocator *) {
  NotOnNodePath("DequantizeGgufTensorPayload");
}
Tensor ReconstructGptqModelFp8Weights(const EncodedValueProto &, size_t, const StructTypeCatalogue &) {
  NotOnNodePath("ReconstructGptqModelFp8Weights");
}
Tensor ReconstructGptqWeights(const EncodedValueProto &, size_t, const StructTypeCatalogue &) {
  NotOnNodePath("ReconstructGptqWeights");
}
Tensor ReconstructBitblasWeights(const EncodedValueProto &, size_t, const StructTypeCatalogue &) {
  NotOnNodePath("ReconstructBitblasWeights");
}
Tensor ReconstructQqqWeights(const EncodedValueProto &, size_t, const StructTypeCatalogue &) {
  NotOnNodePath("ReconstructQqqWeights");
}
Tensor ReconstructAwqWeights(const EncodedValueProto &, size_t, const StructTypeCatalogue &) {
  NotOnNodePath("ReconstructAwqWeights");
}
Tensor ReconstructBitsAndBytesWeights(const EncodedValueProto &, size_t, const StructTypeCatalogue &,
                                      int) {
  NotOnNodePath("ReconstructBitsAndBytesWeights");
}
Tensor ReconstructExl3Weights(const EncodedValueProto &, size_t, const StructTypeCatalogue &, int) {
  NotOnNodePath("ReconstructExl3Weights");
}
Tensor ReconstructVptqWeights(const EncodedValueProto &, size_t, const StructTypeCatalogue &) {
  NotOnNodePath("ReconstructVptqWeights");
}
} // namespace onnx_light::core::runtime

namespace onnx_light::core::shapes {
void ShapesContext::LogSetEvent(const std::string &, const SymTensor &) {
  NotOnNodePath("ShapesContext::LogSetEvent");
}
} // namespace onnx_light::core::shapes

namespace onnx_light::utils {
Blake3Hasher::Blake3Hasher() { NotOnNodePath("Blake3Hasher"); }
void Blake3Hasher::Update(const void *, std::size_t) { NotOnNodePath("Blake3Hasher::Update"); }
int64_t Blake3Hasher::Finalize64() const { NotOnNodePath("Blake3Hasher::Finalize64"); }
} // namespace onnx_light::utils
