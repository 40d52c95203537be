// Fixed-scratch variant of the fused DequantizeLinear -> [Cast] -> MatMul.
//
// Some callers cannot hand the library a workspace: a runtime whose device
// memory plan is fixed before the run and has no scratch entry for this node,
// real-time or embedded loops that forbid allocation after start-up, and host
// plugins that receive only their input and output buffers.  For them this entry
// point runs the same kernels as b2_dequantize_matmul but takes its split-K
// scratch from one statically sized device array owned by this library.
//
// Rules of the fixed scratch:
//  * size: kStaticScratchBytes (8 MiB) per device, held by every GPU that
//    loads the library until the process exits;
//  * calls whose plan needs more are rejected with B2_ERR_WORKSPACE and a
//    message naming both sizes;
//  * every call shares the array: the arrival counters at its start are
//    cleared on each call, partial sums from the previous call are simply
//    overwritten, and two calls that overlap on the GPU (different streams,
//    or different host threads on one device) race on it;
//  * each call looks the array's device address up with cudaGetSymbolAddress
//    on the current device (the host-side name of a __device__ array is not a
//    device address); the first lookup on a device loads the module there, so
//    make the first call on each device before any stream capture;
//  * a kernel whose bounded wait gave up reports it through
//    b2_kernel_status() (device words of the library, outside this array), so
//    the per-call clearing of the counters never hides a time-out;
//  * nothing here allocates: no cudaMalloc, no cudaFree, no library allocator.
#include "dq_matmul.cuh"

namespace b2 {

constexpr size_t kStaticScratchBytes = size_t(8) << 20;

static __device__ __align__(256) uint8_t g_static_scratch[kStaticScratchBytes];

// Device address of g_static_scratch on the current device, looked up on
// every call with that device current: the lookup is cheap, and an address
// cached across calls would go stale after cudaDeviceReset or with a new
// primary context.
static int static_scratch(void **out) {
  void *p = nullptr;
  B2_CUDA(cudaGetSymbolAddress(&p, g_static_scratch));
  if (p == nullptr) B2_FAIL(B2_ERR_CUDA, "cudaGetSymbolAddress returned a null address");
  *out = p;
  return B2_OK;
}

} // namespace b2

using namespace b2;

extern "C" int b2_dequantize_matmul_noalloc(const b2_tensor *a, const b2_tensor *w,
                                            const b2_tensor *w_scale,
                                            const b2_tensor *w_zero_point, int64_t axis,
                                            int32_t cast_dtype, b2_tensor *y, void *stream) {
  // Size query: validates the call and plans it without launching anything.
  size_t need = 0;
  int rc = b2_dequantize_matmul(a, w, w_scale, w_zero_point, axis, cast_dtype, y, nullptr, &need,
                                stream);
  if (rc < 0) return rc;
  if (need > kStaticScratchBytes)
    B2_FAIL(B2_ERR_WORKSPACE,
            "b2_dequantize_matmul_noalloc: this call needs %zu bytes of scratch, more than the "
            "%zu-byte fixed scratch; use b2_dequantize_matmul with a workspace",
            need, kStaticScratchBytes);
  if (need == 0) return b2_dequantize_matmul(a, w, w_scale, w_zero_point, axis, cast_dtype, y,
                                             nullptr, nullptr, stream);
  void *scratch = nullptr;
  rc = static_scratch(&scratch);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // The split-K arrival counters must start at zero.
  B2_CUDA(cudaMemsetAsync(scratch, 0, kCounterBytes, st));
  size_t cap = kStaticScratchBytes;
  return b2_dequantize_matmul(a, w, w_scale, w_zero_point, axis, cast_dtype, y, scratch, &cap,
                              stream);
}
