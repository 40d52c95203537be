/*
 * onnxl_b200 — C ABI of the B200 (sm_100a) kernels for onnx-light's
 * quantized-inference path.
 *
 * Every entry point replaces one onnx-light CPU kernel's operator() (cited
 * beside it, paths relative to the onnx-light source tree) and keeps its
 * argument meaning, accepted dtypes and validation.  Where the reference
 * throws std::invalid_argument (EXT_ENFORCE_INVALID), these return a negative
 * status and b2_last_error() holds a message with the same "kernel::<Op>:"
 * prefix.
 *
 * Conventions
 *  - Tensors are contiguous row-major device buffers (b2_tensor.data is a
 *    device address).  Sub-byte types (INT4, UINT4, FLOAT4E2M1, INT2, UINT2)
 *    are packed low-order-first, as in onnx-light's Tensor storage
 *    (onnx_light/onnx_core/runtime/kernels/cast_sub_byte.h:48-60).
 *  - dtype is the ONNX TensorProto.DataType code.
 *  - `stream` is a cudaStream_t (NULL = legacy default stream).  Calls are
 *    stream-ordered and never synchronize the host.
 *  - Nothing is allocated inside.  Entry points that need scratch take
 *    (workspace, workspace_bytes): with workspace == NULL the required size is
 *    written to *workspace_bytes and nothing runs; otherwise *workspace_bytes is
 *    the capacity offered.  A workspace must be zero-filled once before its
 *    first use; every call leaves the arrival counters it used at zero again,
 *    so the same buffer serves any later call on the same stream.  Calls that
 *    share one workspace must not overlap on the GPU.
 *  - No CPU fallback: every accepted call runs on the GPU or fails.
 */
#ifndef ONNXL_B200_H
#define ONNXL_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define B2_API __attribute__((visibility("default")))
#else
#define B2_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define B2_OK 0
#define B2_ERR_INVALID_ARGUMENT -1  /* reference: std::invalid_argument */
#define B2_ERR_UNSUPPORTED_DTYPE -2 /* reference: "unsupported data type" invalid_argument */
#define B2_ERR_CUDA -3              /* a CUDA runtime call failed */
#define B2_ERR_WORKSPACE -4         /* workspace smaller than required */
#define B2_ERR_TIMEOUT -5           /* a bounded device-side wait gave up */
#define B2_ERR_UNSUPPORTED -6       /* valid for the reference, not handled on the GPU */

typedef struct b2_tensor {
  void *data;           /* device address (NULL allowed when the tensor has no elements) */
  int32_t dtype;        /* ONNX TensorProto.DataType */
  int32_t ndim;         /* 0 for a scalar */
  const int64_t *shape; /* ndim entries (may be NULL when ndim == 0) */
} b2_tensor;

/* A column-sharded output over a multi-GPU group (one process per GPU): every
 * rank's full [M, n_full] output buffer and flag array (uint32[8], zeroed
 * once), mapped into this process (b2_ipc_open), and this rank's two-word
 * counter (zeroed once).  Rank r owns columns [r n_full / world, (r + 1)
 * n_full / world). */
typedef struct b2_peer_out {
  void *full[8];
  uint32_t *flags[8];
  uint32_t *counters;
  int32_t world, rank;
  int64_t n_full;
  /* b2_dequantize_matmul_peer: nonzero when the input `a` is (or may be) the
   * output of a sharded call not yet waited for, so the kernel first waits
   * for every rank to finish the group's previous call; zero skips the wait
   * (an input no sharded call wrote since the last wait). */
  int32_t wait_input;
} b2_peer_out;

/* Library identification, e.g. "onnxl_b200 0.1 sm_100a". */
B2_API const char *b2_version(void);

/* Copies the calling thread's last error message into buf (NUL-terminated,
 * truncated to len) and returns the status it belonged to. */
B2_API int b2_last_error(char *buf, size_t len);

/*
 * DequantizeLinear: y = (x - x_zero_point) * x_scale, bit-exact with the
 * reference.
 * Replaces kernel::DequantizeLinear::operator()(x, x_scale, x_zero_point,
 * axis, output, rt) (kernel_dequantizelinear.cc:522-651) and, with
 * x_zero_point == NULL, operator()(x, x_scale, axis, output, rt) (:670-693).
 *  x: UINT8, INT8, UINT16, INT16, INT32, FLOAT8E4M3FN, FLOAT8E4M3FNUZ,
 *     FLOAT8E5M2, FLOAT8E5M2FNUZ, UINT4, INT4, UINT2, INT2, FLOAT4E2M1,
 *     FLOAT6E2M3, FLOAT6E3M2.
 *  x_scale: FLOAT or FLOAT16; one element -> per-tensor; rank(x) -> blocked
 *     along `axis` (block = x.shape[axis] / x_scale.shape[axis]); otherwise
 *     per-axis with x.shape[axis] elements.
 *  y: dtype == x_scale dtype, shape == x shape.
 *  axis: must already be non-negative, as the reference requires (:539-540).
 */
B2_API int b2_dequantize_linear(const b2_tensor *x, const b2_tensor *x_scale,
                         const b2_tensor *x_zero_point, int64_t axis, b2_tensor *y,
                         void *stream);

/*
 * Fused DequantizeLinear -> [Cast] -> MatMul with the quantized operand on the
 * right: y = a @ cast(dequantize(w, w_scale, w_zero_point, axis)).
 * Replaces the node pair kernel::DequantizeLinear (as above) feeding
 * kernel::MatMul::operator()(a, b) (kernel_matmul.cc:181-223), optionally with
 * an ONNX Cast between them.
 *  a: FLOAT, FLOAT16 or BFLOAT16, rank >= 1 (NumPy MatMul broadcasting of the
 *     leading dimensions against a rank-2 w).
 *  w: rank-2 [K, N] quantized weight, any dtype b2_dequantize_linear takes.
 *  cast_dtype: 0 when the dequantized weight feeds MatMul directly (its dtype
 *     is then the scale dtype and must equal a's dtype, kernel_matmul.cc:182);
 *     otherwise FLOAT, FLOAT16 or BFLOAT16 (RNE cast of the dequantized value,
 *     onnx_light/onnx_core/runtime/kernels/cast_helper.cc:51-135), equal to a's dtype.
 *  y: dtype of a; shape = MatMul output shape.
 * Arithmetic: the dequantized weight is formed exactly as the reference does
 * (fp32 (q-zp)*s, rounded to the node's output type), then multiplied with fp32
 * accumulation; results agree with the reference within rel-L2 1e-3 for
 * FLOAT16/BFLOAT16 and 1e-5 for FLOAT.
 */
B2_API int b2_dequantize_matmul(const b2_tensor *a, const b2_tensor *w, const b2_tensor *w_scale,
                         const b2_tensor *w_zero_point, int64_t axis, int32_t cast_dtype,
                         b2_tensor *y, void *workspace, size_t *workspace_bytes, void *stream);


/*
 * Fused DequantizeLinear -> [Cast] -> MatMul without a caller-provided
 * workspace, for callers that cannot allocate device memory: sessions whose
 * memory plan is sealed before the run, real-time loops that forbid
 * allocation after start-up, and host plugins that only receive their input
 * and output buffers.  Same arguments, kernels and results as
 * b2_dequantize_matmul (no counterpart in onnx-light: the reference CPU kernel
 * allocates its temporaries itself).
 * Scratch: a fixed 8 MiB device array inside this library, held by every GPU
 * that loads it until the process exits.  Calls whose plan needs more are
 * rejected with B2_ERR_WORKSPACE.  All calls on a device share that array, so
 * calls that overlap on the GPU (other streams or host threads) race; calls
 * on one stream are safe.  Every call resolves the array's device address on
 * the current device; the first call on each device also loads the module
 * there and should come before any stream capture.  Time-outs of its kernels
 * are reported by b2_kernel_status().  Nothing is allocated.
 */
B2_API int b2_dequantize_matmul_noalloc(const b2_tensor *a, const b2_tensor *w,
                                        const b2_tensor *w_scale, const b2_tensor *w_zero_point,
                                        int64_t axis, int32_t cast_dtype, b2_tensor *y,
                                        void *stream);

/*
 * Bounded-wait time-outs recorded by any kernel of this library since the
 * last reset (decode GEMVs, tensor-core GEMMs, MatMulInteger, attention): 0
 * when none, else the first code found (1: data never arrived, 2: a ring slot
 * never freed, 3: an MMA never completed), with the kernel named in
 * b2_last_error(); 4 when b2_rotary_embedding met a position_ids value
 * outside its cos/sin cache (the reference throws there; those outputs are 0).
 * A call whose kernel gave up leaves its output unwritten (or partly written)
 * and is reported only here.  The codes live in device
 * words of the library, never in a caller's workspace.  Synchronizes the
 * device first; reset != 0 clears the codes.  No counterpart in onnx-light:
 * its CPU kernels do not wait on other units of work.
 */
B2_API int b2_kernel_status(int reset);

/*
 * Self-test of the time-out path: one kernel thread waits on a barrier that
 * nothing completes, gives up after limit_ns (at most 2 s) and records code 1;
 * returns the code read back (1 when the path works).  Nothing faults or
 * hangs; the context stays usable.  No counterpart in onnx-light.
 */
B2_API int b2_selftest_bounded_wait(int64_t limit_ns, void *stream);

/*
 * Self-test of the tensor-core dequant GEMM's time-out path, on a real call:
 * b2_dequantize_matmul's tcgen05 plan for (a, w, w_scale, y) is launched with
 * no data loads issued, so the first data wait of every CTA runs out after
 * limit_ns (at most 2 s).  Each CTA records code 1, arrives on its split-K
 * counter with a give-up mark (the last one resets the counter and skips the
 * merge) and returns; y is left unwritten.  The workspace (capacity
 * workspace_bytes) must satisfy b2_dequantize_matmul's size query for the same
 * tensors; its counters are zero again afterwards, so a following
 * b2_dequantize_matmul on it computes the right result.  Returns the code read
 * back (1 when the path works), which b2_kernel_status() then also reports.
 * Nothing faults or hangs.  No counterpart in onnx-light.
 */
B2_API int b2_selftest_gemm_timeout(const b2_tensor *a, const b2_tensor *w,
                                    const b2_tensor *w_scale, b2_tensor *y, void *workspace,
                                    size_t workspace_bytes, int64_t limit_ns, void *stream);

/*
 * MatMulInteger: y[i,j] = sum_k (a[i,k] - a_zp[i]) * (b[k,j] - b_zp[j]) in
 * int32, bit-exact.
 * Replaces kernel::MatMulInteger::operator()(a, b, a_zero_point, b_zero_point,
 * output) (kernel_matmul_integer.cc:178-234).
 *  a, b: INT8 or UINT8; zero points NULL (= 0), scalar, per-row [M] (a) or
 *  per-column [N] (b); y: INT32.
 */
B2_API int b2_matmul_integer(const b2_tensor *a, const b2_tensor *b, const b2_tensor *a_zero_point,
                      const b2_tensor *b_zero_point, b2_tensor *y, void *workspace,
                      size_t *workspace_bytes, void *stream);

/*
 * QLinearMatMul: y = saturate(nearbyint(float(acc) * (a_s * b_s / y_s)) + y_zp),
 * acc the exact integer dot product, bit-exact.
 * Replaces kernel::QLinearMatMul::operator() (kernel_qlinearmatmul.cc:221-267).
 * Scales: FLOAT or FLOAT16 scalars; zero points: scalars of a/b/y's dtype;
 * y: INT8 or UINT8 (y_zero_point's dtype).
 */
B2_API int b2_qlinear_matmul(const b2_tensor *a, const b2_tensor *a_scale, const b2_tensor *a_zero_point,
                      const b2_tensor *b, const b2_tensor *b_scale, const b2_tensor *b_zero_point,
                      const b2_tensor *y_scale, const b2_tensor *y_zero_point, b2_tensor *y,
                      void *workspace, size_t *workspace_bytes, void *stream);

/* Attributes of the opset-23 Attention node (kernel_attention.cc:867-878). */
typedef struct b2_attention_attrs {
  int32_t has_scale;        /* 0: scale = 1/sqrt(head_size) */
  float scale;
  int32_t is_causal;
  float softcap;            /* > 0: softcap * tanh(s / softcap) before the mask */
  int32_t qk_matmul_output_mode; /* 0..3, used when a qk_matmul_output is requested */
  int64_t q_num_heads;      /* rank-3 inputs only */
  int64_t kv_num_heads;     /* rank-3 inputs only */
  int64_t left_window_size; /* -1 = unbounded */
  int64_t right_window_size;
  /* Contiguous KV cache.  0: present_key/value are fresh [B,Hkv,past+new,D]
   * buffers (the reference's ConcatAxis2 repack, kernel_attention.cc:313-339).
   * > 0: past and present alias one capacity-reserved buffer
   * [B, Hkv, kv_capacity, D]; past occupies positions [0, past_len) and the new
   * keys/values are appended in place (ReservePersistentAppend,
   * kernel_attention.cc:297-310). */
  int64_t kv_capacity;
} b2_attention_attrs;

/*
 * Attention (opset 23) with GQA and a contiguous KV cache.
 * Replaces kernel::Attention::operator()(Q, K, V, attrs, attn_mask, past_key,
 * past_value, nonpad_kv_seqlen = nullptr) (kernel_attention.cc:767-852).
 *  q, k, v: FLOAT, FLOAT16 or BFLOAT16, rank 4 [B, H, S, D] (v: [B, Hkv, S,
 *    Dv], Dv may differ from D) or rank 3 [B, S, H*D].
 *  attn_mask: NULL, FLOAT or BOOL (true keeps a position, false masks it),
 *    or FLOAT16 / BFLOAT16 when q is half precision; rank 1-4, broadcast to
 *    [B, Hq, Sq, L]; positions past its last axis are masked.
 *  past_key/past_value: NULL or rank-4 [B, Hkv, past_len, D] (shape), with
 *    data pointing at the cache buffer (see kv_capacity).
 *  present_key/present_value: rank-4 outputs [B, Hkv, past_len+S, D]; may be
 *    NULL when no past is given and the caller does not want them.
 *  y: same dtype as q; rank and layout of q, head size Dv.
 * Equivalent to b2_attention_ex with no nonpad_kv_seqlen and no
 * qk_matmul_output.
 */
B2_API int b2_attention(const b2_tensor *q, const b2_tensor *k, const b2_tensor *v,
                 const b2_tensor *attn_mask, const b2_tensor *past_key,
                 const b2_tensor *past_value, const b2_attention_attrs *attrs, b2_tensor *y,
                 b2_tensor *present_key, b2_tensor *present_value, void *workspace,
                 size_t *workspace_bytes, void *stream);

/*
 * Attention with every input and output of the opset-23 node
 * (kernel::Attention::Run, kernel_attention.cc:855-902): b2_attention plus
 *  nonpad_kv_seqlen: NULL or INT64 [B]; keys j >= nonpad_kv_seqlen[b] are
 *    padding, and without a past the causal frontier is offset by
 *    nonpad_kv_seqlen[b] - Sq (:484-496, 572-582); not with a past cache.
 *  qk_matmul_output: NULL or [B, Hq, Sq, L] of q's dtype (FLOAT, or the half
 *    type the reference demotes to): the scores of qk_matmul_output_mode
 *    0 (scaled Q.K^T), 1 (after softcap), 2 (after the mask) or 3 (softmax).
 */
B2_API int b2_attention_ex(const b2_tensor *q, const b2_tensor *k, const b2_tensor *v,
                    const b2_tensor *attn_mask, const b2_tensor *past_key,
                    const b2_tensor *past_value, const b2_tensor *nonpad_kv_seqlen,
                    const b2_attention_attrs *attrs, b2_tensor *y, b2_tensor *present_key,
                    b2_tensor *present_value, b2_tensor *qk_matmul_output, void *workspace,
                    size_t *workspace_bytes, void *stream);

/*
 * RMSNormalization (opset 23): y = x / sqrt(mean(x^2 over axes [axis, rank)) +
 * epsilon) * scale, scale broadcast against the trailing axes.
 * Replaces kernel::RMSNormalization::operator()(x, scale, axis, epsilon)
 * (kernel_rmsnormalization.cc:83-214): sum of squares in double, rms in float,
 * x / rms in float; FLOAT16 / BFLOAT16 round the normalized value to their type
 * before the scale multiplies it.  x, scale, y: FLOAT, FLOAT16 or BFLOAT16 (one
 * dtype); axis may be negative.
 */
B2_API int b2_rms_normalization(const b2_tensor *x, const b2_tensor *scale, int64_t axis,
                                float epsilon, b2_tensor *y, void *stream);

/*
 * RotaryEmbedding (opset 23).
 * Replaces kernel::RotaryEmbedding::operator()(X, cos_cache, sin_cache,
 * position_ids, attrs) (kernel_rotary_embedding.cc:47-218).
 *  x: FLOAT / FLOAT16 / BFLOAT16, rank 4 [B, H, S, D] or rank 3 [B, S, H*D]
 *     (num_heads required); cos/sin: x's dtype, [max_pos, rot/2] with
 *     position_ids (INT64 [B, S]) or [B, S, rot/2] without (position_ids NULL);
 *  rotary_embedding_dim: 0 = D; interleaved: pairs (2i, 2i+1) instead of
 *     (i, i + rot/2).  Channels past rot/2 pairs are copied.  Bit-exact.
 *  A position outside the cache writes 0 and is reported by b2_kernel_status.
 */
B2_API int b2_rotary_embedding(const b2_tensor *x, const b2_tensor *cos_cache,
                               const b2_tensor *sin_cache, const b2_tensor *position_ids,
                               int32_t interleaved, int64_t rotary_embedding_dim,
                               int64_t num_heads, b2_tensor *y, void *stream);

/*
 * SwiGLU: y = a * sigmoid(alpha * a) * b, a and b of one shape.
 * Replaces kernel::SwiGLU::operator()(a, b, alpha) (kernel_swiglu.cc:13-20,
 * 58-112).  FLOAT, DOUBLE, FLOAT16 or BFLOAT16.  The exponential is CUDA's
 * expf / exp (within 2 ulps of the host library's).
 */
B2_API int b2_swiglu(const b2_tensor *a, const b2_tensor *b, float alpha, b2_tensor *y,
                     void *stream);

/*
 * Multi-GPU support: device buffers shared between the processes of a group
 * (one process per GPU) through CUDA IPC, for b2_allgather_cols.
 *  b2_ipc_alloc: cudaMalloc of `bytes` (zero-filled) and its 64-byte IPC handle
 *    (handle: caller buffer of 64 bytes).  Set-up only: this allocates.
 *  b2_ipc_open / b2_ipc_close: map / unmap another process's buffer by handle.
 *  b2_ipc_free: frees a b2_ipc_alloc buffer.
 * No counterpart in onnx-light (its runtime is single-process, CPU-only).
 */
B2_API int b2_ipc_alloc(size_t bytes, void **ptr, void *handle);
B2_API int b2_ipc_free(void *ptr);
B2_API int b2_ipc_open(const void *handle, void **ptr);
B2_API int b2_ipc_close(void *ptr);

/*
 * All-gather of column slices for column-sharded outputs (weights sharded
 * along N, attention sharded by KV head): this rank's slice `local` [..., n]
 * is stored into columns [rank n, (rank + 1) n) of every rank's full output
 * peer_full[r] ([..., n_total], same dtype, rows contiguous), over NVLink; the
 * call then waits (bounded, 5 s) until every rank's slice has arrived in its
 * own full output.  peer_flags[r]: rank r's flag array (8 uint32, zeroed);
 * counters: this rank's 2 uint32 (zeroed), kept by the kernel.  Every rank
 * must issue the same sequence of gathers; a rank must not read its previous
 * contents of a buffer after a later gather into that buffer has started.
 * Stream-ordered and graph-capturable (no host synchronisation).  A peer that
 * never arrives is reported by b2_kernel_status ("allgather_cols", code 1).
 * Replaces the NCCL all-gather of output slices of the sharded configurations
 * (no counterpart in onnx-light).
 */
B2_API int b2_allgather_cols(const b2_tensor *local, void *const *peer_full,
                             uint32_t *const *peer_flags, uint32_t *counters, int world, int rank,
                             int64_t n_total, void *stream);

/* b2_dequantize_matmul with a column-sharded output, fused with its
 * all-gather: this rank computes y[:, rank N_local : (rank + 1) N_local] (the
 * weight w holds those N_local columns) and stores every output value
 * straight into each rank's full buffer over NVLink (peer stores).  With
 * out->wait_input set, before reading `a` the kernel waits (bounded) until
 * every rank has finished the group's previous sharded call, so `a` may be
 * such a call's full output; when it ends it publishes its own completion in
 * every rank's flag array.  y_local
 * describes the local slice [.., N_local] (its data is not used).  Every rank
 * makes the same sequence of calls.  Int4 / uint4 weights with FLOAT16 scales
 * and activations, up to 16 rows (the register-MMA decode kernel); other
 * shapes return B2_ERR_UNSUPPORTED (use b2_dequantize_matmul on the slice and
 * b2_allgather_cols). */
B2_API int b2_dequantize_matmul_peer(const b2_tensor *a, const b2_tensor *w, const b2_tensor *w_scale,
                                     const b2_tensor *w_zero_point, int64_t axis, int32_t cast_dtype,
                                     const b2_tensor *y_local, const b2_peer_out *out,
                                     void *workspace, size_t *workspace_bytes, void *stream);

/*
 * Several DequantizeLinear -> MatMul nodes that read the same activations `a`
 * (the q / k / v projections of an attention block, the gate / up
 * projections of an MLP) in one call: y[i] = a @ DequantizeLinear(w[i],
 * w_scale[i]) for i < count (1..4).  w, w_scale and y point to arrays of
 * `count` tensors; each member obeys b2_dequantize_matmul's contract with the
 * same a and axis, no zero point and no cast (replaces `count` calls of
 * DequantizeLinear::operator() + MatMul::operator(),
 * onnx_light/onnx_extensions/kernels/kernels/quantization/kernel_dequantizelinear.cc:504-712
 * and kernels/math/kernel_matmul.cc:60-267, on one shared input).  Members
 * with the same K, weight type and scale layout that the int4 / fp16 decode
 * kernel takes (up to 16 rows) run as ONE launch whose CTAs split all the
 * members' weight tiles; otherwise each member runs as b2_dequantize_matmul
 * would, in order.  Results equal b2_dequantize_matmul's for each member
 * within its tolerance.  Workspace as b2_dequantize_matmul (workspace NULL
 * with workspace_bytes non-NULL: size query).
 */
B2_API int b2_dequantize_matmul_group(int32_t count, const b2_tensor *a, const b2_tensor *w,
                                      const b2_tensor *w_scale, int64_t axis, b2_tensor *y,
                                      void *workspace, size_t *workspace_bytes, void *stream);

/* b2_dequantize_matmul_group with column-sharded outputs, each fused with its
 * all-gather as in b2_dequantize_matmul_peer: y_local[i] describes member i's
 * local slice and out[i] its full buffers (out is an array of `count`; every
 * member has the same world and rank).  The call waits for its input and
 * publishes its completion once, through out[0]'s flags and counters
 * (out[0].wait_input).  Members must fit one launch of the decode kernel
 * (same K, weight type and scale layout, int4 / fp16, up to 16 rows);
 * otherwise B2_ERR_UNSUPPORTED. */
B2_API int b2_dequantize_matmul_group_peer(int32_t count, const b2_tensor *a, const b2_tensor *w,
                                           const b2_tensor *w_scale, int64_t axis,
                                           const b2_tensor *y_local, const b2_peer_out *out,
                                           void *workspace, size_t *workspace_bytes, void *stream);

/* Waits (on the device, bounded) until every rank has finished the group's
 * last sharded call or all-gather, so that this rank's full buffers may be
 * read. */
B2_API int b2_peer_wait(const b2_peer_out *out, void *stream);

/*
 * Seeded synthetic inputs, identical to onnx-light's SplitMix64 generators
 * (onnx_light/onnx_core/runtime/kernels/random.cc:38-176), produced on the
 * device so that benchmark inputs never cross PCIe.  Not part of the hot path.
 *  kind 0: uniform  lo + u*(hi-lo)             -> out FLOAT
 *  kind 1: normal   lo + (sum12(u)-6)*hi        -> out FLOAT   (lo = mean, hi = scale)
 *  kind 2: integer  RandInt(lo, hi+1)           -> out INT64
 * Returns B2_ERR_UNSUPPORTED if integer rejection sampling would be needed
 * (never for spans that divide 2^64 or are small).
 */
B2_API int b2_synth_fill(int32_t kind, uint64_t seed, int64_t n, double lo, double hi, void *out,
                  void *stream);

/*
 * Converts a device array: FLOAT -> FLOAT16/BFLOAT16 (RNE, reference NaN
 * patterns), INT64 -> packed INT4/UINT4/INT2/UINT2/INT8/UINT8 (two's-complement
 * truncation), FLOAT -> FLOAT8E4M3FN (saturating RNE).  Input-preparation
 * helper for synthetic inputs; not part of the hot path.
 */
B2_API int b2_convert(const void *src, int32_t src_dtype, void *dst, int32_t dst_dtype, int64_t n,
               void *stream);

#ifdef __cplusplus
}
#endif

#endif /* ONNXL_B200_H */
