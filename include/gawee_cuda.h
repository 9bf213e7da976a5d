/*
 * libgawee_cuda — B200 (sm_100a) backend for compiled inference of a
 * gawee-dialect `forward` function.
 *
 * It replaces the CPU code generation of `gawee-opt --gawee-to-llvm`
 * (middle/mlir/tools/gawee-opt.cpp:120-184) and the AOT launcher/runtime
 * (back/gawee_aot.cpp:174-291, back/runtime_support.h) for the same graph:
 * the graph text that `gawee-onnx-translate` prints is planned into a static
 * sequence of CUDA kernels, weights stay resident on the GPU, and each
 * forward replays the sequence.
 *
 * Conventions
 *   - Arguments are the `forward` arguments in order: graph inputs, then the
 *     float initializers (middle/mlir/lib/Emit/ONNXMLIREmitter.cpp:2932-2975).
 *   - Host buffers are dense C-order arrays of the argument's static shape;
 *     the caller owns them.  Boolean (i1) tensors use one byte per element.
 *   - No exception crosses this interface; every call returns a gawee_status.
 *     gawee_last_error() returns the message of the last failure on a context.
 *   - One context per device.  Calls on one context must be serialised by
 *     the caller; contexts on different devices may be used from different
 *     host threads.
 *   - `stream` arguments are cudaStream_t values passed as void* (NULL means
 *     the context's own stream).
 */
#ifndef GAWEE_CUDA_H
#define GAWEE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int gawee_status;
enum {
  GAWEE_OK = 0,
  GAWEE_ERR_INVALID = 1,      /* bad argument, index, size or state */
  GAWEE_ERR_PARSE = 2,        /* the MLIR text could not be parsed */
  GAWEE_ERR_UNSUPPORTED = 3,  /* an op or shape the backend does not implement */
  GAWEE_ERR_CUDA = 4,         /* a CUDA runtime error */
  GAWEE_ERR_OOM = 5,          /* device allocation failed */
  GAWEE_ERR_DEVICE = 6,       /* a kernel reported an error (e.g. gather index out of range) */
  GAWEE_ERR_NCCL = 7          /* a NCCL call failed */
};

/* Element types (numbering shared with the planner). */
enum {
  GAWEE_F32 = 0,
  GAWEE_F64 = 1,
  GAWEE_F16 = 2,
  GAWEE_I64 = 3,
  GAWEE_I32 = 4,
  GAWEE_I1 = 5
};

typedef struct gawee_ctx gawee_ctx;

/* Plan the function `entry` (NULL = "forward") of MLIR module text for
 * `device`.  Replaces `gawee-opt --gawee-to-llvm` + `gawee-aot build`
 * (back/gawee_aot.cpp:325-366): parsing, fusion, memory planning and device
 * allocation happen here, once. */
gawee_status gawee_create(const char* mlir_text, const char* entry, int device, gawee_ctx** out);

/* Same, reading the MLIR text from a file. */
gawee_status gawee_create_from_file(const char* mlir_path, const char* entry, int device, gawee_ctx** out);

void gawee_destroy(gawee_ctx* ctx);

/* Copies the last error message (NUL-terminated, truncated to n). */
gawee_status gawee_last_error(const gawee_ctx* ctx, char* buf, size_t n);

/* Signature of `forward`: counts, dtypes and static shapes (shape needs room
 * for `rank` values; rank <= 8).  Mirrors parseFuncSignature
 * (back/gawee_aot.cpp:104-144). */
int gawee_num_args(const gawee_ctx* ctx);
int gawee_num_outputs(const gawee_ctx* ctx);
gawee_status gawee_arg_info(const gawee_ctx* ctx, int i, int* dtype, int* rank, int64_t* shape);
gawee_status gawee_output_info(const gawee_ctx* ctx, int i, int* dtype, int* rank, int64_t* shape);

/* Stage argument i from host memory (asynchronous on `stream`; pinned host
 * memory gives true overlap).  Replaces loadNpy + makeDescriptor per argument
 * (back/gawee_aot.cpp:241-249).  Weights that are re-staged are re-packed on
 * the next forward; otherwise packed weights stay resident. */
gawee_status gawee_set_arg(gawee_ctx* ctx, int i, const void* host, size_t bytes, void* stream);

/* Stage argument i from device memory on the context's device. */
gawee_status gawee_set_arg_device(gawee_ctx* ctx, int i, const void* dev, size_t bytes, void* stream);

/* Enqueue one forward on `stream`.  Replaces the call of
 * _mlir_ciface_forward (back/gawee_aot.cpp:263-274).  Asynchronous. */
gawee_status gawee_forward(gawee_ctx* ctx, void* stream);

/* Copy output i to host memory (asynchronous on `stream`).  Replaces
 * saveReturnedMemRef (back/runtime_support.h:272-277). */
gawee_status gawee_get_output(gawee_ctx* ctx, int i, void* host, size_t bytes, void* stream);

/* Device pointer of output i (valid until the next forward). */
gawee_status gawee_output_device_ptr(gawee_ctx* ctx, int i, void** ptr);

/* Wait for `stream` and check the device status word: returns
 * GAWEE_ERR_DEVICE if a kernel flagged an error since the last check.  With
 * ctx NULL it checks the status word of gawee_matmul_f32_noalloc on the
 * current device instead (message via gawee_last_error(NULL, ...)). */
gawee_status gawee_synchronize(gawee_ctx* ctx, void* stream);

/* Capture the forward sequence into a CUDA graph on the next forward
 * (enabled = 1, the default) or launch kernels one by one (0). */
gawee_status gawee_set_graph_mode(gawee_ctx* ctx, int enabled);

/* Arithmetic of the tensor-core contractions (convolutions, GEMMs, fused
 * attention).  The reference computes in fp32 on the CPU; there is no
 * reference counterpart to this call.
 *   GAWEE_PRECISION_FP32 (default): each product from three TF32 products of
 *     the operands' high parts and remainders (hi*hi + hi*lo + lo*hi), fp32
 *     accumulation with round-to-nearest promotion every 64 k: parity with
 *     the fp32 reference at its own tolerances.
 *   GAWEE_PRECISION_TF32: one TF32 product of the truncated operands (10
 *     explicit mantissa bits each), same accumulation: |error| <= 2^-9 *
 *     sum |a_k * b_k| per output plus the accumulation term; not a parity mode.
 *   GAWEE_PRECISION_BF16: contractions on the TMA kernel take one bf16
 *     product (both operands rounded to nearest bf16, 8 significant bits,
 *     relative error <= 2^-9 each), same fp32 accumulation: |error| <=
 *     2^-8 * sum |a_k * b_k| plus the accumulation term; the other
 *     tensor-core kernels (the gather kernel, fused attention) run single-pass
 *     TF32.  The first switch to it allocates a bf16 copy of those
 *     contractions' B operands (half the size of one packed plane).
 * GAWEE_PRECISION=tf32 or bf16 in the environment selects the mode at
 * gawee_create.  Changing the mode drops the captured CUDA graph (it is
 * captured again on the next forward); call it between forwards, with no
 * forward in flight. */
enum { GAWEE_PRECISION_FP32 = 0, GAWEE_PRECISION_TF32 = 1, GAWEE_PRECISION_BF16 = 2 };
gawee_status gawee_set_precision(gawee_ctx* ctx, int mode);
int gawee_precision(const gawee_ctx* ctx); /* the current mode, -1 for NULL */

/* Kernel i of the per-forward sequence: name (fused ops joined by '+'),
 * whether it is a tensor-core contraction, and its algorithmic FLOPs
 * (2*M*N*K with the unpadded K; 0 for other kernels). */
gawee_status gawee_op_info(const gawee_ctx* ctx, int i, char* name, size_t n, int* is_tc, double* flops);

/* Run one forward eagerly with a CUDA event between every kernel and write
 * each kernel's device time in milliseconds to ms[0..gawee_num_kernels-1].
 * Synchronous. */
gawee_status gawee_profile_forward(gawee_ctx* ctx, void* stream, float* ms, int n);

/* Plan without a device: parse and plan `entry` of MLIR text and write the
 * plan summary (or the error message) into buf.  No CUDA call is made. */
gawee_status gawee_plan_text(const char* mlir_text, const char* entry, char* buf, size_t n);

/* Planned main-sequence steps of one forward (the index space of
 * gawee_op_info / gawee_profile_forward) and a human-readable plan summary.
 * gawee_num_launches counts the kernel launches of one forward: a step whose
 * contraction is split along k adds a reduce kernel. */
int gawee_num_kernels(const gawee_ctx* ctx);
int gawee_num_launches(const gawee_ctx* ctx);
gawee_status gawee_plan_summary(const gawee_ctx* ctx, char* buf, size_t n);

/* ---------------------------------------------------------------------------
 * _mlir_ciface_forward compatibility.
 *
 * The reference launcher calls
 *   void _mlir_ciface_forward(MemRefDescriptor<T,R>* result, MemRefDescriptor<Ti,Ri>* arg0, ...)
 * (back/gawee_aot.cpp:174-195, struct at back/runtime_support.h:21-28).
 * gawee_ciface_forward takes the same descriptors as an array: it stages every
 * argument, runs one forward, waits, and writes the single result into a
 * malloc'ed buffer described by `result` (the callee allocates, as the
 * reference's lowered code does).  A memref descriptor is
 *   { T* allocated; T* aligned; int64_t offset; int64_t sizes[R]; int64_t strides[R]; }
 * and must describe a dense C-order array.
 * ------------------------------------------------------------------------- */
gawee_status gawee_ciface_forward(gawee_ctx* ctx, void* result_desc, void* const* arg_descs, int nargs);

/* Entry point for code produced by the `--gawee-to-cuda` pipeline: the
 * lowered module keeps the gawee-level `forward` text as a global string and
 * its `_mlir_ciface_forward` calls this.  The first call on a thread plans the
 * text for `device` and caches the context (keyed by the string's address);
 * later calls reuse it.  Semantics as gawee_ciface_forward; on failure the
 * message is read with gawee_last_error(NULL, ...). */
gawee_status gawee_embedded_forward(const char* mlir_text, int device, void* result_desc, void* const* arg_descs,
                                    int nargs);

/* ---------------------------------------------------------------------------
 * Allocation-free matrix product (no counterpart in the reference).
 *
 * C[m][n] = A[m][k] . B[k][n], fp32 row-major device arrays owned by the
 * caller, computed on the tensor-core kernel with split-precision TF32
 * (the same arithmetic as gawee.matmul in a planned graph), enqueued on
 * `stream`.  For callers that cannot allocate device memory when they need
 * the product: a host framework whose own caching allocator owns the device
 * memory (an allocation behind its back can fail or fragment its pool), a
 * caller working within a fixed memory budget, or an error-recovery path
 * after an allocation has already failed; cudaMalloc and cudaFree can also
 * wait for the whole device.  It calls no cudaMalloc/cudaFree and no
 * allocating library routine: the packed TF32 planes of B use a 16 MiB array
 * in the library's static device memory, which every GPU that loads the
 * library holds until the process exits.
 *   - Limits: k a multiple of 4, A 16-byte aligned, n * k <= 2,097,152
 *     (two planes of n x k floats in 16 MiB); larger shapes return
 *     GAWEE_ERR_INVALID with a message for gawee_last_error(NULL, ...).
 *   - The first call on a device looks up the device addresses of the array
 *     and of a status word (cudaGetSymbolAddress); make that first call
 *     before any stream capture.
 *   - Every call shares the one array: calls that overlap on the GPU (on
 *     different streams, or from several threads) race.  Each call rewrites
 *     all of the scratch it reads, so nothing needs clearing between calls.
 *   - Errors inside the kernel (a bounded wait that gave up, leaving C
 *     partly written) are recorded in the shared status word:
 *     gawee_synchronize(NULL, stream) waits for `stream`, then returns
 *     GAWEE_ERR_DEVICE and clears the word if any call since the last check
 *     reported one.
 * ------------------------------------------------------------------------- */
gawee_status gawee_matmul_f32_noalloc(const float* a, const float* b, float* c, int64_t m, int64_t n, int64_t k,
                                      void* stream);

/* Diagnostic: the tensor cores' TF32 rate on `device`, measured now (one CTA
 * per SM issuing back-to-back M = 128, N = 128, K = 8 tcgen05 TF32 MMAs with
 * both operands in shared memory, timed with CUDA events; about 5 ms).  The
 * fp32 mode issues three such products per multiply-add, so a third of
 * *tflops is its tensor ceiling.  No reference counterpart. */
gawee_status gawee_probe_tf32_mma(int device, double* tflops);

/* ---------------------------------------------------------------------------
 * Data parallelism: batch sharding with replicated weights (one process or
 * thread per GPU).  The only collective is the gather of each rank's output
 * rows to rank 0 over NCCL.
 * ------------------------------------------------------------------------- */
#define GAWEE_NCCL_ID_BYTES 128

/* Fill `id` (GAWEE_NCCL_ID_BYTES) on rank 0; share it with the other ranks. */
gawee_status gawee_dp_unique_id(void* id);

/* Join a communicator of `world` ranks on the context's device.  Collective:
 * the ranks also exchange their output sizes (shards may differ by a row,
 * e.g. 5 rows over 2 ranks as 3 + 2). */
gawee_status gawee_dp_init(gawee_ctx* ctx, int world, int rank, const void* id);

/* Bytes of output i summed over every rank: the size of rank 0's
 * destination buffer for gawee_dp_gather_output. */
gawee_status gawee_dp_output_bytes(gawee_ctx* ctx, int i, size_t* total);

/* Gather output i of every rank, in rank order, into `dst` on rank 0 (a
 * device buffer of gawee_dp_output_bytes bytes; ignored on other ranks).
 * Each rank contributes its own output size, as exchanged at init.
 * Collective: every rank calls it, in the same order. */
gawee_status gawee_dp_gather_output(gawee_ctx* ctx, int i, void* dst, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GAWEE_CUDA_H */
