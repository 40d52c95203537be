// All-gather of column slices over NVLink peer memory, for the column-sharded
// projections and the KV-head-sharded attention of a multi-GPU group (one
// process per GPU).
//
// Rank r computes the slice y[:, r*n : (r+1)*n] of every sharded output.  The
// gather kernel stores that slice straight into the full [M, N] output buffer
// of every rank (its own included) through peer pointers (plain 16-byte global
// stores over NVLink; no TMA, no multicast), then publishes one arrival flag
// in every rank's flag array and waits -- bounded -- until every rank's flag
// for this call has arrived in its own array.  When the kernel ends, the full
// output is in place on this GPU, so the next kernel on the stream reads it.
// This replaces an NCCL all-gather into a rank-major staging buffer plus the
// transposing copy to [M, N].
//
// Ordering: each CTA's stores are made visible system-wide (fence.sc.sys)
// before it counts itself done; the last CTA bumps the call generation and
// writes it to each rank's flag word with a system-scope release store; the
// waiting side reads its own flags with system-scope acquire loads.  The
// generation lives in device memory and advances on the device, so the same
// launch can be captured in a CUDA graph and replayed.
//
// The peer buffers and flag arrays are cudaMalloc allocations shared between
// the processes with CUDA IPC handles (b2_ipc_*), exchanged by the host.
#include "b2_common.cuh"
#include "tc_common.cuh"

namespace b2 {

// Time-out of the last gather whose peers never all arrived (0 = none).
__device__ int g_allgather_status;

namespace {

constexpr int AG_MAX_WORLD = 8;
constexpr int AG_THREADS = 256;

struct AgArgs {
  const uint8_t *src;             // local slice [M, n_local] (row bytes slice_row)
  uint8_t *dst[AG_MAX_WORLD];     // every rank's full output [M, N] (row bytes full_row)
  uint32_t *flags[AG_MAX_WORLD];  // every rank's flag array [AG_MAX_WORLD]
  uint32_t *counters;             // this rank's [0] CTA arrivals, [1] generation
  int64_t M, slice_row, full_row, col_off; // bytes
  int world, rank;
  uint64_t wait_ns;
};

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(AG_THREADS) allgather_cols_kernel(const AgArgs a) {
  // 16-byte chunks of the slice (the host checks 16-byte row sizes and offsets)
  const int64_t chunks_row = a.slice_row / 16;
  const int64_t total = a.M * chunks_row;
  for (int64_t e = blockIdx.x * (int64_t)AG_THREADS + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * AG_THREADS) {
    const int64_t m = e / chunks_row, c = e % chunks_row;
    const uint4 v = *reinterpret_cast<const uint4 *>(a.src + m * a.slice_row + c * 16);
    const int64_t off = m * a.full_row + a.col_off + c * 16;
#pragma unroll
    for (int r = 0; r < AG_MAX_WORLD; ++r)
      if (r < a.world) *reinterpret_cast<uint4 *>(a.dst[r] + off) = v;
  }
  __syncthreads();
  __shared__ bool last;
  if (gridDim.x == 1) {
    // one CTA (a decode-sized slice): its stores are ordered before the flag
    // stores below by the barrier and the release fence
    if (threadIdx.x != 0) return;
    asm volatile("fence.acq_rel.sys;" ::: "memory");
  } else {
    if (threadIdx.x == 0) {
      asm volatile("fence.acq_rel.sys;" ::: "memory"); // this CTA's peer stores, system-wide
      const uint32_t prev = atomicAdd(&a.counters[0], 1u);
      last = prev + 1 == gridDim.x;
    }
    __syncthreads();
    if (!last || threadIdx.x != 0) return;
    a.counters[0] = 0u;
    asm volatile("fence.acq_rel.sys;" ::: "memory");
  }
  const uint32_t gen = a.counters[1] + 1u;
  a.counters[1] = gen;
  for (int r = 0; r < a.world; ++r) st_release_sys(a.flags[r] + a.rank, gen);
  // wait until every rank's slice of this call has landed here
  const uint32_t *mine = a.flags[a.rank];
  const uint64_t t0 = tc::globaltimer();
  for (int r = 0; r < a.world; ++r) {
    // a rank can be at most one call ahead (its next call waits for ours),
    // so "at least this generation" is the arrival test
    while ((int32_t)(ld_acquire_sys(mine + r) - gen) < 0) {
      if (tc::globaltimer() - t0 > a.wait_ns) {
        atomicExch(&g_allgather_status, tc::kTimeoutFull);
        return;
      }
      __nanosleep(32);
    }
  }
}

// One thread: wait until every rank has published the generation this rank
// last published (its last sharded call or all-gather).
__global__ void peer_wait_kernel(const uint32_t *mine, const uint32_t *counters, int world,
                                 uint64_t wait_ns) {
  const uint32_t gen = *(volatile const uint32_t *)(counters + 1);
  const uint64_t t0 = tc::globaltimer();
  for (int r = 0; r < world; ++r)
    while ((int32_t)(ld_acquire_sys(mine + r) - gen) < 0) {
      if (tc::globaltimer() - t0 > wait_ns) {
        atomicExch(&g_allgather_status, tc::kTimeoutFull);
        return;
      }
      __nanosleep(32);
    }
}

} // namespace

int status_read_allgather(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_allgather_status, sizeof(int)) != cudaSuccess) return -1;
  if (reset && v) {
    const int z = 0;
    if (cudaMemcpyToSymbol(g_allgather_status, &z, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}

} // namespace b2

using namespace b2;

extern "C" int b2_ipc_alloc(size_t bytes, void **ptr, void *handle) {
  if (!ptr || !handle) B2_FAIL(B2_ERR_INVALID_ARGUMENT, "b2_ipc_alloc: null argument");
  void *p = nullptr;
  B2_CUDA(cudaMalloc(&p, bytes ? bytes : 1));
  B2_CUDA(cudaMemset(p, 0, bytes ? bytes : 1));
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    B2_FAIL(B2_ERR_CUDA, "b2_ipc_alloc: cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  }
  memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return B2_OK;
}

extern "C" int b2_ipc_free(void *ptr) {
  B2_CUDA(cudaFree(ptr));
  return B2_OK;
}

extern "C" int b2_ipc_open(const void *handle, void **ptr) {
  if (!ptr || !handle) B2_FAIL(B2_ERR_INVALID_ARGUMENT, "b2_ipc_open: null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  B2_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return B2_OK;
}

extern "C" int b2_ipc_close(void *ptr) {
  B2_CUDA(cudaIpcCloseMemHandle(ptr));
  return B2_OK;
}

extern "C" int b2_allgather_cols(const b2_tensor *local, void *const *peer_full,
                                 uint32_t *const *peer_flags, uint32_t *counters, int world,
                                 int rank, int64_t n_total, void *stream) {
  if (!local || !peer_full || !peer_flags || !counters)
    B2_FAIL(B2_ERR_INVALID_ARGUMENT, "b2_allgather_cols: null argument");
  B2_ENFORCE(world >= 1 && world <= AG_MAX_WORLD, "b2_allgather_cols: world must be 1..%d", AG_MAX_WORLD);
  B2_ENFORCE(rank >= 0 && rank < world, "b2_allgather_cols: rank out of range");
  B2_ENFORCE(local->ndim >= 1, "b2_allgather_cols: the local slice must have rank >= 1");
  const int64_t esz = packed_bytes(local->dtype, 1);
  B2_ENFORCE(esz >= 1, "b2_allgather_cols: unsupported dtype %d", local->dtype);
  const int64_t n_local = local->shape[local->ndim - 1];
  B2_ENFORCE(n_local * world == n_total, "b2_allgather_cols: world x slice columns must equal N");
  const int64_t M = n_local ? numel(local) / n_local : 0;
  AgArgs a{};
  a.src = static_cast<const uint8_t *>(local->data);
  a.M = M;
  a.slice_row = n_local * esz;
  a.full_row = n_total * esz;
  a.col_off = (int64_t)rank * n_local * esz;
  B2_ENFORCE(a.slice_row % 16 == 0 && reinterpret_cast<uintptr_t>(a.src) % 16 == 0,
             "b2_allgather_cols: slice rows must be 16-byte multiples on 16-byte boundaries");
  for (int r = 0; r < world; ++r) {
    a.dst[r] = static_cast<uint8_t *>(peer_full[r]);
    a.flags[r] = peer_flags[r];
    B2_ENFORCE(a.dst[r] && a.flags[r] && reinterpret_cast<uintptr_t>(a.dst[r]) % 16 == 0,
               "b2_allgather_cols: peer buffers must be non-null and 16-byte aligned");
  }
  a.counters = counters;
  a.world = world;
  a.rank = rank;
  a.wait_ns = 5000000000ull; // a peer that has not arrived in 5 s is gone
  const int64_t chunks = M * (a.slice_row / 16);
  int64_t blocks = (chunks + AG_THREADS - 1) / AG_THREADS;
  const int64_t cap = (int64_t)sm_count() * 2;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  allgather_cols_kernel<<<(unsigned)blocks, AG_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(a);
  B2_LAUNCH_CHECK();
  return B2_OK;
}

extern "C" int b2_peer_wait(const b2_peer_out *out, void *stream) {
  if (!out || !out->counters) B2_FAIL(B2_ERR_INVALID_ARGUMENT, "b2_peer_wait: null argument");
  B2_ENFORCE(out->world >= 1 && out->world <= AG_MAX_WORLD, "b2_peer_wait: world must be 1..%d", AG_MAX_WORLD);
  B2_ENFORCE(out->rank >= 0 && out->rank < out->world && out->flags[out->rank],
             "b2_peer_wait: rank out of range or null flags");
  peer_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(out->flags[out->rank], out->counters,
                                                                    out->world, 5000000000ull);
  B2_LAUNCH_CHECK();
  return B2_OK;
}
