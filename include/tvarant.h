/*
 * tvarant.h — C ABI of the B200 runtime and kernels behind the `tvarant`
 * PyTorch device.
 *
 * This header replaces the reference's internal runtime boundary: the
 * `tvarant::TvarantRuntime` virtual interface and the `LaunchParams`
 * grab-bag that every ATen kernel fills before `runtime().launch(p)`
 * (csrc/runtime/TvarantRuntime.h:17-61 in samthakur587/Tvarant).  Where the
 * reference dispatches on a kernel-name string (csrc/runtime/CpuSimRuntime.cpp:109-218),
 * each kernel here is its own typed entry point.
 *
 * Conventions (all entry points):
 *   - return 0 (TVR_OK) on success, a TVR_ERR_* code otherwise; the message
 *     for the calling thread is available from tvr_last_error();
 *   - buffers are borrowed raw device pointers; no entry point keeps a
 *     pointer after it returns (the caching allocator owns what it hands out);
 *   - sizes, strides and element counts are int64_t, in elements;
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default
 *     stream); work is enqueued asynchronously on it;
 *   - all floating-point kernels compute in fp32.
 * Kernels that wait on a barrier inside the device give up after a bounded
 * number of polls and record TVR_DEV_* in a per-device status word, read with
 * tvr_get_status(); they never trap.
 */
#ifndef TVARANT_H_
#define TVARANT_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* ---- status codes ------------------------------------------------------ */
#define TVR_OK 0
#define TVR_ERR_INVALID 1     /* bad argument (shape, null pointer, op id)      */
#define TVR_ERR_CUDA 2        /* a CUDA runtime/driver call failed              */
#define TVR_ERR_UNSUPPORTED 3 /* valid request the library does not implement */
#define TVR_ERR_OOM 4         /* device or pinned allocation failed             */
#define TVR_ERR_TIMEOUT 5     /* a bounded wait expired (host or device side)   */
#define TVR_ERR_NCCL 6        /* NCCL missing or an NCCL call failed            */
#define TVR_ERR_JIT 7         /* NVRTC compilation or module load failed        */

/* device-side status word values (tvr_get_status) */
#define TVR_DEV_OK 0
#define TVR_DEV_TIMEOUT_PRODUCER 1 /* TMA producer gave up waiting for a free stage */
#define TVR_DEV_TIMEOUT_MMA 2      /* MMA issuer gave up waiting for data / TMEM    */
#define TVR_DEV_TIMEOUT_EPILOGUE 3 /* epilogue gave up waiting for an accumulator   */
#define TVR_DEV_TIMEOUT_DRAIN 4    /* exit-time drain of async copies gave up       */
#define TVR_DEV_TIMEOUT_CONVERT 5  /* 3xTF32 converter gave up waiting for a stage  */
#define TVR_DEV_TIMEOUT_PEER 6     /* a cross-rank barrier gave up waiting for a rank */
#define TVR_DEV_CACHE_FULL 7       /* a KV-cache append past the cache's capacity was dropped */

/* GEMM precision modes */
#define TVR_GEMM_AUTO 0    /* TVARANT_GEMM_MODE env, else 3xTF32               */
#define TVR_GEMM_TF32 1    /* tcgen05 kind::tf32, one pass                      */
#define TVR_GEMM_3XTF32 2  /* hi*hi + hi*lo + lo*hi split, fp32-faithful        */
#define TVR_GEMM_FP32 3    /* CUDA-core fp32 FMA (exact fp32 products)          */

/* activations; same numbering as the reference `jit::apply_act`
 * (csrc/jit/Jit.h:48-56): 0 none, 1 relu, 2 silu */
#define TVR_ACT_NONE 0
#define TVR_ACT_RELU 1
#define TVR_ACT_SILU 2

/* unary op ids for tvr_unary; each replaces one OpenCL kernel / host loop
 * (csrc/kernels/host/HostKernels.cpp:39-98, csrc/runtime/OpenCLRuntime.cpp:49-88) */
#define TVR_UNARY_RELU 0
#define TVR_UNARY_SILU 1
#define TVR_UNARY_NEG 2
#define TVR_UNARY_ABS 3
#define TVR_UNARY_EXP 4
#define TVR_UNARY_EXP2 5
#define TVR_UNARY_SQRT 6
#define TVR_UNARY_RSQRT 7      /* 1/sqrt(x), as HostKernels.cpp:94-98      */
#define TVR_UNARY_SCALE 8      /* x * scalar   (scale_kernel)              */
#define TVR_UNARY_ADD_SCALAR 9 /* x + scalar   (add_scalar_kernel)         */
#define TVR_UNARY_SIGMOID 10
#define TVR_UNARY_COPY 11

/* binary op ids for tvr_binary */
#define TVR_BINARY_ADD 0 /* a + alpha*b (add_kernel, HostKernels.cpp:27-31) */
#define TVR_BINARY_MUL 1 /* a * b       (mul_kernel, HostKernels.cpp:33-37) */

#define TVR_MAX_DIMS 8

/* ---- errors / init ----------------------------------------------------- */

/* Thread-local message of the last failing call on this thread ("" if none). */
const char* tvr_last_error(void);

/* Idempotent process-wide initialisation (device enumeration, driver entry
 * points).  Replaces tvarant::initialize_runtime (csrc/runtime/Runtime.cpp:39-47). */
int tvr_init(void);

/* Backend name, "cuda".  Replaces TvarantRuntime::name (TvarantRuntime.h:42). */
const char* tvr_backend_name(void);

/* ---- devices ----------------------------------------------------------- */

/* Number of visible GPUs.  Replaces kDeviceCount (TvarantRuntime.h:12). */
int tvr_device_count(int* count);
/* Current device of the calling thread.  Replaces current_device /
 * set_device (csrc/runtime/Runtime.cpp:55-71). */
int tvr_get_device(int* device);
int tvr_set_device(int device);
/* Number of SMs, for grid sizing in callers and tests. */
int tvr_device_sm_count(int device, int* sms);
/* Wait for all work on `device`.  Replaces TvarantRuntime::synchronize
 * (TvarantRuntime.h:60). */
int tvr_device_synchronize(int device);
/* Device-side status word (TVR_DEV_*), set by kernels whose bounded waits
 * expired.  tvr_clear_status resets it to TVR_DEV_OK. */
int tvr_get_status(int device, int* code);
int tvr_clear_status(int device);

/* ---- memory ------------------------------------------------------------ */

/* Stream-ordered caching allocation on `device` (a pool that keeps freed
 * blocks).  Replaces TvarantRuntime::alloc/free (TvarantRuntime.h:45-46) and
 * the posix_memalign sim allocator (csrc/runtime/CpuSimRuntime.cpp:63-81).
 * nbytes == 0 returns NULL.  Allocations are 256-byte aligned. */
int tvr_malloc(void** ptr, size_t nbytes, int device, void* stream);
int tvr_free(void* ptr);
/* Make the free of `ptr` wait for the work queued so far on `stream`
 * (a cross-stream use; c10 recordDataPtrOnStream). */
int tvr_record_stream(void* ptr, void* stream);
/* Device index of an allocation made by tvr_malloc, or -1.  Replaces
 * TvarantRuntime::owns (TvarantRuntime.h:47) used by getDeviceFromPtr. */
int tvr_pointer_device(const void* ptr, int* device);
/* Bytes held by the pool (reserved) and handed out (in use) on `device`. */
int tvr_memory_stats(int device, size_t* reserved, size_t* in_use);
/* Return cached, unused blocks of `device` to the driver. */
int tvr_empty_cache(int device);
/* Page-locked host memory for asynchronous copies. */
int tvr_host_alloc(void** ptr, size_t nbytes);
int tvr_host_free(void* ptr);
int tvr_is_pinned(const void* ptr, int* pinned);

/* Asynchronous copies on `stream`.  Replace TvarantRuntime::copy_h2d /
 * copy_d2h / copy_d2d (TvarantRuntime.h:49-51).  With pageable host memory
 * the copy is staged by the driver and returns after the host side is read. */
int tvr_memcpy_h2d(void* dst, const void* src, size_t nbytes, void* stream);
int tvr_memcpy_d2h(void* dst, const void* src, size_t nbytes, void* stream);
int tvr_memcpy_d2d(void* dst, const void* src, size_t nbytes, void* stream);

/* ---- streams and events (the reference has only the DEFAULT stream,
 * csrc/runtime/Guard.cpp:43-62) ------------------------------------------ */
int tvr_stream_create(void** stream, int device, int priority);
int tvr_stream_destroy(void* stream);
int tvr_stream_synchronize(void* stream);
int tvr_stream_query(void* stream, int* done);
int tvr_stream_wait_event(void* stream, void* event);
int tvr_event_create(void** event, int enable_timing);
int tvr_event_destroy(void* event);
int tvr_event_record(void* event, void* stream);
int tvr_event_synchronize(void* event);
int tvr_event_query(void* event, int* done);
int tvr_event_elapsed_ms(void* start, void* end, float* ms);

/* ---- graphs: capture the device work issued on a stream once, replay it
 * (the reference launches synchronously, one kernel at a time,
 * csrc/runtime/CpuSimRuntime.cpp:109-218).  Work on other streams joins the
 * capture through events recorded on the capturing stream and must join back
 * before tvr_graph_end.  Device memory allocated during the capture
 * (tvr_malloc is stream-ordered) belongs to the graph: allocations still live
 * at the end of the capture keep their addresses and are reused by every
 * replay, so tensors produced by the captured work are rewritten in place. */
int tvr_graph_begin(void* stream);
/* Ends the capture begun on `stream` and instantiates it into *graph. */
int tvr_graph_end(void* stream, void** graph);
int tvr_graph_launch(void* graph, void* stream);
int tvr_graph_destroy(void* graph);

/* ---- dense contractions (tensor cores) --------------------------------- */

/* C[m,n] = act(alpha * sum_k A[m,k]*B(k,n) + beta * P[m,n]) where
 * P[m,n] = bias[n] if bias != NULL, else C[m,n] if beta != 0, else 0.
 * A is row-major [m,k] with row stride lda.  B is [n,k] (row stride ldb) when
 * trans_b != 0 (nn.Linear weight), else [k,n] (row stride ldb).  C is
 * row-major [m,n] with row stride ldc.  `mode` is a TVR_GEMM_* value.
 * Replaces ops::gemm_bias_act (csrc/aten/AtenCommon.h:33-86) ->
 * LaunchParams{"gemm_bias_act_kernel"} -> host::gemm_bias_act_f32
 * (csrc/kernels/host/HostKernels.cpp:100-144) / gemm.cl:27-64. */
int tvr_gemm_bias_act(const float* a, const float* b, const float* bias, float* c,
                      int64_t m, int64_t n, int64_t k,
                      int64_t lda, int64_t ldb, int64_t ldc,
                      float alpha, float beta, int act, int trans_b, int mode,
                      void* stream);

/* tvr_gemm_bias_act in TF32 mode (same arguments, minus the mode) for
 * callers that cannot allocate device memory during the call: a host that
 * hands out all device memory itself from a budget fixed at start-up, or a
 * runtime that forbids the CUDA allocator once it is serving (an allocation
 * can synchronize the device and its latency is unbounded).  No counterpart
 * in the reference.  The only scratch it uses — split-K partial sums — is a fixed
 * 16 MiB __device__ array inside the library, which every GPU that loads the
 * library keeps until the process exits; the call makes no allocation.
 * Limit: m*n <= 4194304 output elements, else TVR_ERR_INVALID.  The first call
 * on a device looks the array up (cudaGetSymbolAddress); make that first
 * call before any stream capture.  All calls share the array: two calls that
 * may run at the same time on the GPU (different streams, different host
 * threads) race on it and must be ordered by the caller.  Nothing in the
 * array needs to start at zero: each call writes every element it reads.
 * The SM limit of tvr_set_gemm_sm_limit applies.  An expired bounded wait
 * inside the kernel is reported through tvr_get_status only on a device that
 * tvr_init (or any other call of this library) has set up; setting a device up
 * allocates its status word, which this entry point never does itself. */
int tvr_gemm_bias_act_noalloc(const float* a, const float* b, const float* bias, float* c,
                              int64_t m, int64_t n, int64_t k,
                              int64_t lda, int64_t ldb, int64_t ldc,
                              float alpha, float beta, int act, int trans_b, void* stream);

/* Upper bound on the SMs (CTAs) the persistent tensor-core GEMM of this
 * device occupies; 0 (the default) means all.  Tensor-parallel code keeps a
 * few SMs free with it so that NCCL kernels overlap the GEMMs instead of
 * waiting for them.  Applies to launches issued after the call. */
int tvr_set_gemm_sm_limit(int device, int max_sms);
int tvr_get_gemm_sm_limit(int device, int* max_sms);

/* Gated (SwiGLU) projection: out[m, n] = silu(x . Wg^T) * (x . Wu^T), with x
 * [m, k] (row stride ldx) and both weights in nn.Linear layout [n, k] (row
 * strides ldw_gate, ldw_up).  No reference counterpart as one call: the
 * reference computes it as linear_act(x, Wg, None, "silu") * linear(x, Wu)
 * (csrc/aten/CustomOps.cpp:14-39, csrc/aten/LlmOps.cpp:150-174, Ops.cpp:312-327),
 * three kernels and two [m, n] round trips.  TVR_GEMM_TF32 runs one tcgen05
 * pass whose epilogue forms the product; the other modes run that composition
 * on the device. */
int tvr_gemm_swiglu(const float* x, const float* w_gate, const float* w_up, float* out,
                    int64_t m, int64_t n, int64_t k, int64_t ldx, int64_t ldw_gate,
                    int64_t ldw_up, int64_t ldo, int mode, void* stream);

/* Fused attention forward: out = softmax(scale * Q K^T + causal mask) V for
 * Q [batch, heads, seq_q, head_dim], K and V [batch, heads, seq_k, head_dim],
 * each given by its element strides over (batch, head, position) with a
 * contiguous last dimension; out has its own strides; lse (optional, may be
 * NULL) receives the natural-log log-sum-exp per (batch, head, query) as
 * [batch, heads, seq_q].  causal != 0 hides key j from query i when j > i
 * (PyTorch's is_causal).  The kernel computes in TF32 with head_dim 64 and
 * scale > 0; other head dimensions, modes and scales return
 * TVR_ERR_UNSUPPORTED (the caller then composes bmm / softmax / bmm).  No reference counterpart: the
 * reference materialises the scores (csrc/aten/LlmOps.cpp:68-148). */
int tvr_attention_fwd(const float* q, const float* k, const float* v, float* out, float* lse,
                      int64_t batch, int64_t heads, int64_t seq_q, int64_t seq_k,
                      int64_t head_dim, const int64_t* q_strides, const int64_t* k_strides,
                      const int64_t* v_strides, const int64_t* o_strides, float scale,
                      int causal, int mode, void* stream);

/* The same attention (no mask, no lse) over K / V buffers of seq_k positions
 * of which only the first clamp(*key_len + key_len_add, 1, seq_k) are
 * attended: key_len is an int64 in device memory written by earlier work on
 * the stream, so a step captured in a CUDA graph attends to a growing KV
 * cache without being captured again.  TF32 mode only (TVR_ERR_UNSUPPORTED
 * otherwise, as for tvr_attention_fwd).  No reference counterpart. */
int tvr_attention_fwd_keylen(const float* q, const float* k, const float* v, float* out,
                             int64_t batch, int64_t heads, int64_t seq_q, int64_t seq_k,
                             int64_t head_dim, const int64_t* q_strides,
                             const int64_t* k_strides, const int64_t* v_strides,
                             const int64_t* o_strides, float scale, const int64_t* key_len,
                             int key_len_add, int mode, void* stream);

/* KV-cache append: src [batch, heads, seq_new, dim] (strides src_strides for
 * batch, head, position; dim contiguous) is written into cache positions
 * *pos .. *pos + seq_new - 1 (cache strides cache_strides, dim contiguous).
 * *pos is an int64 in device memory; positions at or past max_len are
 * dropped and TVR_DEV_CACHE_FULL is set in the device status word.  The
 * position does not advance (tvr_counter_add).  No reference counterpart. */
int tvr_kv_append(float* cache, const float* src, int64_t batch, int64_t heads, int64_t seq_new,
                  int64_t dim, int64_t max_len, const int64_t* cache_strides,
                  const int64_t* src_strides, const int64_t* pos, void* stream);

/* One decode step's attention with its KV-cache append, in one launch: for
 * p = *pos (an int64 in device memory), k_new / v_new [batch, heads, 1, dim]
 * are written into cache position p of k_cache / v_cache [batch, heads,
 * max_len, dim], and q [batch, heads, 1, dim] attends (no mask) to cache
 * positions 0..p, out [batch, heads, 1, dim] = softmax(scale q k^T) v.  The
 * result, the caches and the status word are exactly those of tvr_kv_append
 * (k), tvr_kv_append (v), then tvr_attention_fwd_keylen with key_len = pos,
 * key_len_add = 1; a position outside [0, max_len) appends nothing, sets
 * TVR_DEV_CACHE_FULL and attends to clamp(p + 1, 1, max_len) cached keys.
 * Strides are for (batch, head, position), dim contiguous; q, k_new, v_new
 * and the caches need 16-byte aligned bases and strides that are multiples
 * of 4 elements.  dim 64, scale > 0, TF32 or 3xTF32 mode (the kernel computes
 * in fp32); anything else returns TVR_ERR_UNSUPPORTED and the caller runs
 * the three calls.  *pos does not advance (tvr_counter_add).  No reference
 * counterpart. */
int tvr_attention_decode_append(const float* q, const float* k_new, const float* v_new,
                                float* k_cache, float* v_cache, float* out, int64_t batch,
                                int64_t heads, int64_t max_len, int64_t head_dim,
                                const int64_t* q_strides, const int64_t* kn_strides,
                                const int64_t* vn_strides, const int64_t* kc_strides,
                                const int64_t* vc_strides, const int64_t* o_strides, float scale,
                                const int64_t* pos, int mode, void* stream);

/* *counter += delta on the stream (an int64 in device memory). */
int tvr_counter_add(int64_t* counter, int64_t delta, void* stream);

/* Batched C[i] = A[i] * op(B[i]) for i < batch, each as tvr_gemm_bias_act
 * with alpha 1, beta 0, no activation; matrices are dense row-major with the
 * given element strides between batch entries (stride_b may be 0 to
 * broadcast one B).  Replaces LaunchParams{"bmm_kernel"} -> host::bmm_f32
 * (csrc/kernels/host/HostKernels.cpp:146-172) / gemm.cl:66-95. */
int tvr_bmm(const float* a, const float* b, float* c,
            int64_t batch, int64_t m, int64_t n, int64_t k,
            int64_t stride_a, int64_t stride_b, int64_t stride_c,
            int trans_b, int mode, void* stream);

/* ---- reductions and gathers (memory-bound) ----------------------------- */

/* Softmax over `dim` of a contiguous (outer, dim, inner) view:
 * y = exp(x - max) * (1 / sum exp(x - max)).  Replaces
 * LaunchParams{"softmax_kernel"} -> host::softmax_f32
 * (csrc/kernels/host/HostKernels.cpp:174-198) / reduce.cl:2-30. */
int tvr_softmax(const float* x, float* y, int64_t outer, int64_t dim, int64_t inner,
                void* stream);

/* y[r, :] = softmax(x[r, :] + mask[r % mask_rows, :]) over rows of `dim`
 * contiguous values: an additive attention mask ([L, S], shared by every
 * batch entry and head of x [B, H, L, S]) applied as the row is loaded.  The
 * add is the same fp32 rounding as tvr_binary's, so the result equals
 * tvr_binary(ADD) followed by tvr_softmax.  Returns TVR_ERR_UNSUPPORTED
 * (nothing launched) unless dim % 4 == 0, dim <= 2048 and the three pointers
 * are 16-byte aligned; TVR_ERR_INVALID unless rows is a whole number of
 * mask_rows.  No reference counterpart as one call: the reference
 * runs add(scores, mask) then softmax (csrc/aten/LlmOps.cpp:68-105). */
int tvr_softmax_add(const float* x, const float* mask, float* y, int64_t rows, int64_t dim,
                    int64_t mask_rows, void* stream);

/* Row layer norm of x[rows, n]: mean, biased variance (two-pass),
 * rstd = 1/sqrt(var + eps), y = (x - mean) * rstd [* gamma] [+ beta].
 * gamma, beta, mean, rstd may be NULL.  Replaces
 * LaunchParams{"layernorm_kernel"} -> host::layer_norm_f32
 * (csrc/kernels/host/HostKernels.cpp:200-242) / reduce.cl:32-74. */
int tvr_layer_norm(const float* x, const float* gamma, const float* beta, float* y,
                   float* mean, float* rstd, int64_t rows, int64_t n, float eps,
                   void* stream);

/* out[i, :] = weight[idx[i], :] for i < n_idx; an index outside [0, vocab)
 * gives a zero row.  `indices` are int64 (index_bits 64) or int32
 * (index_bits 32) read directly on the device.  Replaces
 * LaunchParams{"embedding_kernel"} -> host::embedding_f32
 * (csrc/kernels/host/HostKernels.cpp:244-260) / reduce.cl:76-95, and the
 * host round trip of the indices in ops::embedding (csrc/aten/LlmOps.cpp:238-246). */
int tvr_embedding(const float* weight, const void* indices, int index_bits, float* out,
                  int64_t n_idx, int64_t dim, int64_t vocab, void* stream);

/* ---- elementwise ------------------------------------------------------- */

/* y[i] = op(x[i]) (TVR_UNARY_*), scalar used by SCALE / ADD_SCALAR.  x and y
 * may alias.  Replaces relu/silu/neg/abs/exp/exp2/sqrt/rsqrt/scale/
 * add_scalar/copy kernels (HostKernels.cpp:23-98). */
int tvr_unary(int op, const float* x, float* y, int64_t n, float scalar, void* stream);

/* Fill n elements of `elem_size` bytes (1, 2, 4 or 8) with the bit pattern
 * at `value` (host pointer).  Replaces fill_kernel (HostKernels.cpp:17-21). */
int tvr_fill(void* dst, const void* value, int elem_size, int64_t n, void* stream);

/* out = a (op) b over an `ndim`-dimensional output of `sizes`, with
 * per-operand element strides (0 for a broadcast dimension); `out` is
 * contiguous.  ADD computes a + alpha*b, MUL a*b.  Replaces add_kernel /
 * mul_kernel and the expand().contiguous() materialisation in front of them
 * (csrc/aten/Ops.cpp:283-327). */
int tvr_binary(int op, const float* a, const float* b, float* out, int ndim,
               const int64_t* sizes, const int64_t* a_strides, const int64_t* b_strides,
               float alpha, void* stream);

/* Strided -> strided copy of elements of `elem_size` bytes (1, 2, 4, 8 or
 * 16) over an `ndim`-dimensional index space.  Replaces the CPU-view
 * strided copy of _copy_from / clone / contiguous (csrc/aten/Ops.cpp:185-212,
 * csrc/aten/ExtendedOps.cpp:100-143). */
int tvr_strided_copy(void* dst, const void* src, int64_t elem_size, int ndim,
                     const int64_t* sizes, const int64_t* dst_strides,
                     const int64_t* src_strides, void* stream);

/* Element type conversion between float32 (0), float64 (1), int32 (2),
 * int64 (3), bool/uint8 (4) on contiguous buffers of n elements. */
int tvr_convert(void* dst, int dst_type, const void* src, int src_type, int64_t n,
                void* stream);

/* out = cond ? a : b over a dense output of `ndim` dimensions; cond is bool
 * (1 byte), a / b / out have elements of elem_size bytes (1, 4 or 8); each
 * input is read through its own element strides (0 broadcasts).  No
 * reference kernel: the reference runs where / masked_fill on the CPU
 * through its boxed fallback (csrc/aten/Ops.cpp:499-501). */
int tvr_where(const void* cond, const void* a, const void* b, void* out, int elem_size, int ndim,
              const int64_t* sizes, const int64_t* cond_strides, const int64_t* a_strides,
              const int64_t* b_strides, void* stream);

/* out[r] = index of the largest of the n contiguous values of row r (int64):
 * the first on ties, a NaN counting as the largest (PyTorch's argmax rule).
 * No reference kernel: the reference runs argmax on the CPU through its
 * boxed fallback (csrc/aten/Ops.cpp:499-501). */
int tvr_argmax_rows(const float* x, int64_t* out, int64_t rows, int64_t n, void* stream);

/* Triangular mask of dense [batch, rows, cols]: out = x where
 * col - row >= diagonal (upper != 0, triu) or col - row <= diagonal (tril),
 * else 0.  elem_size 1, 4 or 8.  No reference kernel (CPU fallback there). */
int tvr_triangle(const void* x, void* out, int elem_size, int64_t batch, int64_t rows,
                 int64_t cols, int64_t diagonal, int upper, void* stream);

/* RMSNorm over rows of n contiguous values: y = x / sqrt(mean(x^2) + eps)
 * [* weight] (weight [n] or null); rstd[row] = 1 / sqrt(mean(x^2) + eps)
 * when rstd is not null.  y must not overlap x.  No reference counterpart
 * (the reference has no RMSNorm; F.rms_norm decomposes into pow / mean /
 * rsqrt / mul there). */
int tvr_rms_norm(const float* x, const float* weight, float* y, float* rstd, int64_t rows,
                 int64_t n, float eps, void* stream);

/* Rotary position embedding of [batch, seq, heads] vectors of `dim` values
 * (dim contiguous; x_strides / y_strides give the batch, position and head
 * strides in elements): for each rotation pair (a, b) — (i, i + dim/2), or
 * (2i, 2i + 1) when interleaved — with c = cos_table[p][i], s =
 * sin_table[p][i] at position p = pos_offset + position:
 *   a' = a*c - b*s,  b' = b*c + a*s   (products and sums rounded separately).
 * The tables have table_rows rows of table_stride >= dim/2 values.  x and y
 * may be the same buffer with the same strides.  No reference counterpart. */
int tvr_rope(const float* x, float* y, const float* cos_table, const float* sin_table,
             int64_t batch, int64_t seq, int64_t heads, int64_t dim, const int64_t* x_strides,
             const int64_t* y_strides, int64_t table_rows, int64_t table_stride,
             int64_t pos_offset, int interleaved, void* stream);

/* ---- pointwise JIT ----------------------------------------------------- */

/* One SSA node.  Opcodes 0-8 keep the reference numbering
 * (csrc/jit/Jit.h:11-21): Load, Const, Add (a + alpha*b), Mul, Relu, Silu,
 * Neg, Scale (alpha*a), Sigmoid; this library appends Sub (a - alpha*b) = 9,
 * Exp = 10, Abs = 11. */
typedef struct tvr_pw_node {
  int32_t op;
  int32_t a;
  int32_t b;
  int32_t input_id;
  float alpha;
  float c;
} tvr_pw_node;

#define TVR_PW_MAX_INPUTS 16

/* out[i] = value of the last node at element i, for i < n.  The program is
 * emitted as CUDA C, compiled by NVRTC for sm_100a and cached by its
 * structure.  Replaces TvarantRuntime::launch_pointwise
 * (TvarantRuntime.h:53-58) -> jit::run_pointwise_host (csrc/jit/Jit.cpp:34-87)
 * / codegen_opencl (csrc/jit/Jit.cpp:89-138). */
int tvr_pointwise(const tvr_pw_node* nodes, int n_nodes, int n_inputs,
                  const float* const* inputs, float* out, int64_t n, void* stream);

/* Writes the CUDA C source generated for a program into buf (NUL
 * terminated, truncated to cap) and its length into *len.  Host only. */
int tvr_pointwise_source(const tvr_pw_node* nodes, int n_nodes, int n_inputs, char* buf,
                         size_t cap, size_t* len);

/* GEMM with a pointwise program on its output:
 *   y = act(alpha * A . op(B) + beta * bias)      (as tvr_gemm_bias_act)
 *   c[r, j] = program(input gemm_input = y[r, j], input i = inputs[i][r * input_ld[i] + j])
 * The program is a tvr_pointwise SSA program of at most 12 nodes over at most
 * three inputs, one of them (gemm_input) the GEMM result; inputs[gemm_input]
 * is ignored.  The other inputs are [m, n] fp32 with row stride input_ld[i]
 * (>= n), or 0 for one row of n values broadcast over all rows; they must not
 * overlap c.  The tensor-core GEMM runs the program in its epilogue, so y is
 * never written to memory; other GEMM kernels are followed by one in-place
 * pass.  Either way the result equals tvr_gemm_bias_act followed by
 * tvr_pointwise on the same program.  No reference counterpart as one call:
 * the reference's compiler emits linear_act followed by a pointwise program
 * (torch_tvarant/compiler.py, csrc/aten/CustomOps.cpp:14-89). */
int tvr_gemm_pointwise(const float* a, const float* b, const float* bias, float* c, int64_t m,
                       int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldc, float alpha,
                       float beta, int act, int trans_b, int mode, const tvr_pw_node* nodes,
                       int n_nodes, int n_inputs, int gemm_input, const float* const* inputs,
                       const int64_t* input_ld, void* stream);

/* How tvr_gemm_pointwise runs a program (host only, no device): *n_ops
 * receives the length of the two-slot stack code the tensor-core GEMM's
 * epilogue evaluates, 0 when the program runs as a pass over the GEMM's
 * output instead (it needs more than two stack slots or reads two extra
 * inputs).  Up to cap operations are written to ops / rev / vals: the stack
 * opcode (0 push GEMM result, 1 push the extra input, 2 push constant vals[i],
 * 3 add a + vals[i]*b, 4 sub a - vals[i]*b, 5 mul, 6 relu, 7 silu, 8 neg,
 * 9 scale vals[i]*a, 10 sigmoid, 11 exp, 12 abs; binary operations take
 * a = slot 1, b = slot 0, or the reverse when rev[i] is 1).  The program is
 * checked as tvr_gemm_pointwise checks it. */
int tvr_gemm_pointwise_plan(const tvr_pw_node* nodes, int n_nodes, int n_inputs, int gemm_input,
                            int* n_ops, int8_t* ops, int8_t* rev, float* vals, int cap);

/* ---- NCCL (no counterpart in the reference, which has one device) ------ */

/* NCCL is loaded at run time; these return TVR_ERR_NCCL when it is absent.
 * The unique id is NCCL's 128-byte ncclUniqueId. */
int tvr_nccl_available(int* available);
int tvr_nccl_get_unique_id(void* id128);
int tvr_nccl_comm_init(void** comm, int nranks, const void* id128, int rank, int device);
/* The same, with NCCL's kernels limited to at most max_ctas CTAs per
 * collective (ncclConfig_t.maxCTAs) when the loaded NCCL supports it
 * (2.28 and later); max_ctas <= 0 leaves NCCL's choice.  Lets collectives
 * run beside the persistent GEMM when tvr_set_gemm_sm_limit keeps SMs free. */
int tvr_nccl_comm_init_ctas(void** comm, int nranks, const void* id128, int rank, int device,
                            int max_ctas);
/* dtype: 0 float32; op: 0 sum.  In place when send == recv. */
int tvr_nccl_all_reduce(const void* send, void* recv, int64_t count, int dtype, int op,
                        void* comm, void* stream);
int tvr_nccl_all_gather(const void* send, void* recv, int64_t send_count, int dtype,
                        void* comm, void* stream);
int tvr_nccl_comm_destroy(void* comm);
int tvr_nccl_comm_abort(void* comm);

/* ---- NVLink SHARP all-reduce (no counterpart in the reference) -------- */

#define TVR_NVLS_MAX_RANKS 8
#define TVR_NVLS_MAX_BLOCKS 64
/* output tiles of one tvr_gemm_nvls_all_reduce_f32 call (128 x 256 each) */
#define TVR_NVLS_MAX_TILES 4096
/* uint32 words of one rank's flag array: barrier words for three phases,
 * then one arrival counter per output tile */
#define TVR_NVLS_FLAG_WORDS (3 * TVR_NVLS_MAX_BLOCKS * TVR_NVLS_MAX_RANKS + TVR_NVLS_MAX_TILES)

/* In-place sum of `count` fp32 values over `world` ranks (one process per
 * GPU) of a buffer bound to an NVLink multicast object: `multicast` is the
 * buffer's multicast address on this rank, peer_flags[r] the address (on this
 * rank) of rank r's flag array of TVR_NVLS_FLAG_WORDS uint32 (zero when
 * first used; mapped peer memory, e.g. from a symmetric-memory rendezvous).
 * Rank r reduces slice r through the switch (multimem.ld_reduce) and stores
 * it to every rank (multimem.st); two barriers on the flags order the call
 * after every rank's writes of the input and before every rank's next use.
 * epoch_counter is one uint32 in this rank's device memory, zero before the
 * first call with these flag arrays; each call first advances it on the
 * stream (so a captured CUDA graph uses a fresh value on every replay) and
 * the barriers wait for that value.  Every rank makes the same sequence of
 * calls with the same count and blocks.  count must be a multiple of
 * 4 x world.  A barrier wait that expires (2 s; a rank that never arrives)
 * sets TVR_DEV_TIMEOUT_PEER in the device status word and the kernel
 * returns: check tvr_get_status after synchronizing. */
int tvr_nvls_all_reduce_f32(void* multicast, int64_t count, void* const* peer_flags, int rank,
                            int world, uint32_t* epoch_counter, int blocks, void* stream);

/* C = A . B^T (TF32; A [m, k] with row stride lda, B [n, k] with row stride
 * ldb: an nn.Linear weight) followed by the in-place sum of C over `world`
 * ranks, in one kernel: the row-parallel projection of a tensor-parallel
 * layer and its all-reduce.  c is this rank's copy of a buffer bound to an
 * NVLink multicast object and c_multicast its multicast address; peer_flags,
 * epoch_counter, rank and world as for tvr_nvls_all_reduce_f32 (the same
 * flag arrays may serve both calls).  GEMM CTAs store each 128 x 256 output
 * tile to c and count it in the flag array of the rank that owns the tile
 * (tile index mod world); reduce_ctas further CTAs of the same launch (a
 * cooperative one, so every CTA is resident) wait for their rank's tiles to
 * arrive from every rank, sum each through the switch (multimem.ld_reduce)
 * and store the sum to every rank (multimem.st), so the exchange runs while
 * the GEMM is still computing other tiles.  A closing barrier keeps every
 * rank in the call until all tiles are summed.  Requires n % 4 == 0, 16-byte
 * aligned rows, m, n >= 32 and at most TVR_NVLS_MAX_TILES tiles;
 * 1 <= reduce_ctas <= TVR_NVLS_MAX_BLOCKS.  Expired waits (2 s) set
 * TVR_DEV_TIMEOUT_PEER. */
int tvr_gemm_nvls_all_reduce_f32(const float* a, const float* b, float* c, void* c_multicast,
                                 int64_t m, int64_t n, int64_t k, int64_t lda, int64_t ldb,
                                 int64_t ldc, void* const* peer_flags, int rank, int world,
                                 uint32_t* epoch_counter, int reduce_ctas, void* stream);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* TVARANT_H_ */
