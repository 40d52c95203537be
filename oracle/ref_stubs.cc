// Link stubs for oracle/_ref — test infrastructure only.
//
// oracle/_ref links five onnx-light kernel sources (DequantizeLinear,
// MatMulInteger, QLinearMatMul, MatMul, Attention) with the handful of
// runtime sources their direct operator() calls need.  The symbols below are
// reachable only from the session path (KernelBase::Run, peak-memory
// estimators, tuning-schema registration, persistent KV storage), which
// ref_shim.cc never calls.  Each stub throws so that an unexpected call fails
// loudly instead of returning a made-up value.
#include "onnx_core/compute/execution_plan.h"
#include "onnx_core/expressions/expressions.h"
#include "onnx_core/runtime/kernels/node_helpers.h"
#include "onnx_core/runtime/persistent_value.h"
#include "onnx_core/runtime/runtime_context.h"
#include "onnx_core/runtime/tuning/kernel_tuning.h"
#include "onnx_core/shapes/dispatch_table.h"
#include "onnx_core/shapes/shape_broadcast.h"
#include "onnx_core/shapes/shape_check.h"
#include "onnx_core/symbolic/sym_tensor.h"

#include <stdexcept>

namespace {
[[noreturn]] void NotOnOraclePath(const char *what) {
  throw std::logic_error(std::string("oracle/_ref: session-path symbol called: ") + what);
}
} // namespace

namespace onnx_light::core::expressions {
DimType dim_add(const DimType &, const DimType &, SimplifiedExpressionCache *) { NotOnOraclePath("dim_add"); }
DimType dim_mul(const DimType &, const DimType &, SimplifiedExpressionCache *) { NotOnOraclePath("dim_mul"); }
DimType dim_max(const DimType &, const DimType &, SimplifiedExpressionCache *) { NotOnOraclePath("dim_max"); }
DimType dim_exact_div(const DimType &, const DimType &, SimplifiedExpressionCache *) {
  NotOnOraclePath("dim_exact_div");
}
DimType dim_multi_mul(const std::vector<DimType> &, SimplifiedExpressionCache *) {
  NotOnOraclePath("dim_multi_mul");
}
} // namespace onnx_light::core::expressions

namespace onnx_light::core::runtime {
const Tensor &GetInput(const NodeProto &, int, const RuntimeContext &) { NotOnOraclePath("GetInput"); }
const Tensor *GetOptionalInput(const NodeProto &, int, const RuntimeContext &) {
  NotOnOraclePath("GetOptionalInput");
}
void SetOutput(const NodeProto &, int, Tensor, RuntimeContext &) { NotOnOraclePath("SetOutput"); }
void RequireInputCount(const NodeProto &, int) { NotOnOraclePath("RequireInputCount"); }
void RequireMinInputCount(const NodeProto &, int) { NotOnOraclePath("RequireMinInputCount"); }
void RequireOutputCount(const NodeProto &, int) { NotOnOraclePath("RequireOutputCount"); }
int64_t GetAttributeIntOrDefault(const NodeProto &, const std::string &, int64_t) {
  NotOnOraclePath("GetAttributeIntOrDefault");
}
float GetAttributeFloatOrDefault(const NodeProto &, const std::string &, float) {
  NotOnOraclePath("GetAttributeFloatOrDefault");
}
KernelTuningSchema KernelTuningSchema::WithQueryValidation(KernelTuningParameters,
                                                           KernelTuningQueryValidationHook) {
  NotOnOraclePath("KernelTuningSchema::WithQueryValidation");
}
void RegisterKernelTuningSchema(KernelTuningSchema) { NotOnOraclePath("RegisterKernelTuningSchema"); }
std::span<uint8_t> PersistentTensor::AppendReservation::writable_bytes() {
  NotOnOraclePath("AppendReservation::writable_bytes");
}
RuntimeContext::RuntimeContext(KernelContext, RuntimeContextOptions) {
  NotOnOraclePath("RuntimeContext::RuntimeContext");
}
RuntimeContext::~RuntimeContext() {}
RuntimeContext RuntimeContext::MakeFunctionContext() const {
  NotOnOraclePath("RuntimeContext::MakeFunctionContext");
}
void RuntimeContext::Put(const std::string &, Tensor, RuntimeEventKind) {
  NotOnOraclePath("RuntimeContext::Put");
}
void RuntimeContext::RecordEvent(RuntimeEvent) { NotOnOraclePath("RuntimeContext::RecordEvent"); }
std::optional<PersistentTensor::AppendReservation>
RuntimeContext::ReservePersistentAppend(const Tensor &, const Shape &, size_t, int, int) {
  NotOnOraclePath("RuntimeContext::ReservePersistentAppend");
}
Tensor RuntimeContext::CommitPersistentAppend(int, PersistentTensor::AppendReservation, size_t) {
  NotOnOraclePath("RuntimeContext::CommitPersistentAppend");
}
} // namespace onnx_light::core::runtime

namespace onnx_light::core::runtime {
// Key function of ExecutionPlan: defining it emits the class vtable, which the
// RuntimeContext header references inline.
void ExecutionPlan::BuildActions() { NotOnOraclePath("ExecutionPlan::BuildActions"); }
} // namespace onnx_light::core::runtime

namespace onnx_light::core::shapes {
SymShape BroadcastShapes(const SymShape &, const SymShape &) { NotOnOraclePath("BroadcastShapes"); }
int64_t CheckedDimensionAdd(int64_t, int64_t) { NotOnOraclePath("CheckedDimensionAdd"); }
int64_t CheckedDimensionMultiply(int64_t, int64_t) { NotOnOraclePath("CheckedDimensionMultiply"); }
PeakMemoryEstimate UnknownPeakMemory(const std::string &, const std::string &) {
  NotOnOraclePath("UnknownPeakMemory");
}
PeakMemoryEstimate ComputePeakMemory(const ComputePeakMemoryNodeFn &, Device, const NodeProto &,
                                     const std::vector<SymShape> &) {
  NotOnOraclePath("ComputePeakMemory");
}
} // namespace onnx_light::core::shapes

namespace onnx_light::core::symbolic {
void SymShape::PushBack(SymDim) { NotOnOraclePath("SymShape::PushBack"); }
} // namespace onnx_light::core::symbolic

namespace onnx_light::utils {
std::shared_ptr<void> ByteSpan::acquire_export_guard() const {
  NotOnOraclePath("ByteSpan::acquire_export_guard");
}
} // namespace onnx_light::utils
