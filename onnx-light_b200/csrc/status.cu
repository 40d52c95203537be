// Surfacing of the kernels' bounded-wait time-outs to the host.
//
// Every spin-wait in the device code (mbarrier waits on TMA loads, on MMA
// commits, on other warps) gives up after a wall-clock limit; the kernel then
// records a code (1 data never arrived, 2 a ring slot never freed, 3 an MMA
// never completed) in a device word of its own, skips the rest of its work,
// lets its own copies in flight land, frees its TMEM and returns, so the
// context stays usable.  A split-K contributor that gave up still arrives on
// its tile's counter (with a give-up mark), so the counters return to zero
// and the last contributor does not merge invalid partial sums.
// b2_kernel_status() reads every kernel's word; b2_selftest_bounded_wait()
// and b2_selftest_gemm_timeout() make a wait run out on purpose to check the
// whole path.
#include "b2_common.cuh"
#include "tc_common.cuh"

namespace b2 {

int status_read_gemv_mma(int reset);
int status_read_attn_decode(int reset);
int status_read_attn_prefill(int reset);
int status_read_attn_prefill_tc(int reset);
int status_read_dq_gemm_tc(int reset);
int status_read_imma_tc(int reset);
int status_read_dq_gemv(int reset);
int status_read_rotary(int reset);
int status_read_allgather(int reset);
int status_read_dq_gemm_f32(int reset);
int status_read_gemv_x(int reset);
int status_read_gemv_n(int reset);
int status_read_gemv_c(int reset);

__device__ int g_selftest_status;

namespace {

// One thread waits on a barrier that nothing completes, gives up after
// limit_ns and records code 1 (data never arrived).
__global__ void selftest_bounded_wait(uint64_t limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x != 0) return;
  tc::mbar_init(&bar, 1);
  tc::fence_barrier_init();
  if (!tc::mbar_wait(&bar, 0, limit_ns)) atomicExch(&g_selftest_status, tc::kTimeoutFull);
}

} // namespace

} // namespace b2

using namespace b2;

extern "C" B2_API int b2_kernel_status(int reset) {
  B2_CUDA(cudaDeviceSynchronize());
  // code: the kernels' time-out codes (1..3), or kOutOfRange for an input
  // value a device kernel could not reject on the host
  constexpr int kOutOfRange = 4;
  struct Src { const char *name; int (*read)(int); int code; };
  const Src srcs[] = {{"dq_gemv_mma", status_read_gemv_mma, 0},
                      {"dq_gemv_x", status_read_gemv_x, 0},
                      {"dq_gemv_n", status_read_gemv_n, 0},
                      {"dq_gemv_c", status_read_gemv_c, 0},
                      {"attn_decode_mma", status_read_attn_decode, 0},
                      {"attn_prefill_mma", status_read_attn_prefill, 0},
                      {"attn_prefill_tc", status_read_attn_prefill_tc, 0},
                      {"dq_gemm_tc", status_read_dq_gemm_tc, 0},
                      {"imma_tc", status_read_imma_tc, 0},
                      {"dq_gemv_i4h", status_read_dq_gemv, 0},
                      {"dq_gemm_f32", status_read_dq_gemm_f32, 0},
                      {"allgather_cols", status_read_allgather, 0},
                      {"kernel::RotaryEmbedding", status_read_rotary, kOutOfRange}};
  int first = 0;
  for (const Src &s : srcs) {
    const int v = s.read(reset);
    if (v < 0) B2_FAIL(B2_ERR_CUDA, "b2_kernel_status: reading the status of %s failed", s.name);
    if (v && !first) {
      first = s.code ? s.code : v;
      if (s.code == kOutOfRange)
        set_error(B2_OK, "%s: position_ids value out of range (those outputs were written as 0)",
                  s.name);
      else
        set_error(B2_OK, "%s: a bounded wait timed out (code %d: %s)", s.name, v,
                  v == tc::kTimeoutFull ? "data never arrived"
                  : v == tc::kTimeoutEmpty ? "a ring slot never freed" : "an MMA never completed");
    }
  }
  return first;
}

extern "C" B2_API int b2_selftest_bounded_wait(int64_t limit_ns, void *stream) {
  if (limit_ns <= 0 || limit_ns > 2000000000ll)
    B2_FAIL(B2_ERR_INVALID_ARGUMENT, "b2_selftest_bounded_wait: limit must be in (0, 2 s]");
  const int z = 0;
  B2_CUDA(cudaMemcpyToSymbol(g_selftest_status, &z, sizeof(int)));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  selftest_bounded_wait<<<1, 32, 0, st>>>((uint64_t)limit_ns);
  B2_LAUNCH_CHECK();
  B2_CUDA(cudaStreamSynchronize(st));
  int v = 0;
  B2_CUDA(cudaMemcpyFromSymbol(&v, g_selftest_status, sizeof(int)));
  return v;
}
