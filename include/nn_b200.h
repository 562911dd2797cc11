/*
 * nn_b200.h -- C ABI of the B200 NeuroNet kernel library (libnn_b200.so).
 *
 * The library is a drop-in for the OpenCL device layer that the MQL5 layer
 * classes of EAPrognoz/NN_in_Trading drive through COpenCLMy / COpenCL
 * (Experts/NeuroNet_DNG/NeuroNet_Declarations.mqh:359-513,
 *  NeuroNet_Core.mqh:241-346 and 14623-15000, macros in
 *  NeuroNet_Definitions.mqh:56-96).  The same contract is kept:
 *
 *   - buffers are int handles owned by the context;
 *   - kernels are created by id and by their NeuroNet.cl name, and their
 *     positional arguments PERSIST across executions (callers rebind only
 *     what changes);
 *   - argument order is the NeuroNet.cl signature order (the def_k_* indices
 *     of NeuroNet_Definitions.mqh:560-2540), enum values are ENUM_ACTIVATION /
 *     ENUM_OPTIMIZATION (NeuroNet_Definitions.mqh:3650-3685);
 *   - nn_execute takes (dims, offset, global, local) and global/local carry
 *     the problem shape exactly as the reference kernels read it through
 *     get_global_size / get_local_size;
 *   - the queue is in order, nn_execute is asynchronous, nn_buffer_read
 *     blocks.
 *
 * Every entry point returns an int status (NN_OK == 0, negative on error);
 * nn_last_error gives the text of the last failure.  Types are restricted to
 * int / float / double / pointers so that MQL5 `#import` can bind them.
 *
 * Extensions beyond the reference (used by the batched and data-parallel
 * training configurations): per-kernel batch count, command lists, and NCCL
 * data parallelism.
 */
#ifndef NN_B200_H
#define NN_B200_H

#if defined(_WIN32)
#define NN_API __declspec(dllexport)
#else
#define NN_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define NN_OK 0
#define NN_ERR_STATE -1       /* no context / wrong call order */
#define NN_ERR_ARG -2         /* bad argument value */
#define NN_ERR_HANDLE -3      /* unknown buffer / kernel / list handle */
#define NN_ERR_KERNEL -4      /* kernel name not in the library */
#define NN_ERR_BOUNDS -5      /* a buffer is too small for the launch shape */
#define NN_ERR_CUDA -6        /* CUDA runtime error */
#define NN_ERR_NCCL -7        /* NCCL error */
#define NN_ERR_TIMEOUT -8     /* a bounded wait expired */
#define NN_ERR_UNSUPPORTED -9 /* valid reference call this library does not implement */

/* activation enum, NeuroNet_Definitions.mqh:3650-3669 / NeuroNet.cl:32-39 */
#define NN_ACT_NONE -1
#define NN_ACT_TANH 0
#define NN_ACT_SIGMOID 1
#define NN_ACT_LRELU 2
#define NN_ACT_SOFTPLUS 3
#define NN_ACT_GELU 4
#define NN_ACT_MINUS_SOFTPLUS 5
#define NN_ACT_ELU 6
/* optimization enum, NeuroNet_Definitions.mqh:3671-3685 */
#define NN_OPT_SGD 0
#define NN_OPT_ADAM 1
#define NN_OPT_LS 2
#define NN_OPT_ADAM_MINI 3

/* ---------------------------------------------------------------- context */
/* COpenCLMy::Initialize + ContextCreate (NeuroNet_Core.mqh:241-326).
 * device: CUDA ordinal; flags: 0, or NN_INIT_SIMT_GEMM to run the matrix
 * products of the dense / convolution / LSTM kernels as FP32 SIMT GEMMs
 * instead of 3xTF32 tensor-core GEMMs (both meet the 1e-4 parity bound). */
#define NN_INIT_SIMT_GEMM 1
NN_API int nn_init(int device, int flags);
/* COpenCL::Shutdown: frees every buffer, kernel and list of the context. */
NN_API int nn_shutdown(void);
/* Text of the last error (CL_ERROR_DESCRIPTION / GetLastError role). */
NN_API int nn_last_error(char *buf, int len);
/* COpenCLMy::GetMaxLocalSize (NeuroNet_Declarations.mqh:469). */
NN_API int nn_max_local_size(int dim);
/* Wait until every enqueued launch finished (CLExecutionStatus polling);
 * bounded by timeout_ms (<= 0: wait without bound). */
NN_API int nn_finish(int timeout_ms);
/* The context's CUDA stream (cudaStream_t) so that other CUDA code can order
 * work against it. */
NN_API void *nn_stream(void);

/* ---------------------------------------------------------------- buffers */
/* COpenCLMy::AddBuffer / CBufferFloat::BufferCreate
 * (NeuroNet_Core.mqh:14623-14720, 14881-14920): returns a handle >= 0. */
NN_API int nn_buffer_create(long long bytes);
/* COpenCL::BufferFree. */
NN_API int nn_buffer_free(int handle);
/* CBufferFloat::BufferWrite / COpenCL::BufferWrite: count floats from src to
 * element offset `offset`.  Enqueued in order; src is read before return. */
NN_API int nn_buffer_write(int handle, const float *src, long long offset, long long count);
/* CBufferFloat::BufferRead / COpenCL::BufferRead: blocking read. */
NN_API int nn_buffer_read(int handle, float *dst, long long offset, long long count);
/* COpenCLMy::BufferWrite(buffer, data, offset, start, count) and COpenCL::BufferRead with the same
 * arguments (NeuroNet_Declarations.mqh:425-430, over MetaQuotes' CLBufferWrite / CLBufferRead):
 * `byte_offset` is the position in the device buffer in BYTES (a multiple of 4), `start` the index
 * of the first element of the host array `data`, `count` the number of floats.  Copies
 * data[start .. start+count) to / from device floats byte_offset/4 .. byte_offset/4+count. */
NN_API int nn_buffer_write_ex(int handle, const float *data, long long byte_offset, long long start,
                              long long count);
NN_API int nn_buffer_read_ex(int handle, float *data, long long byte_offset, long long start, long long count);
/* Extension (no reference counterpart): overlapped transfers, for a host that feeds the next step
 * while the current one computes.
 * nn_buffer_write_async: host -> device copy on a transfer stream, concurrent with the executions
 *   already enqueued; every execution enqueued afterwards waits for it.  The caller guarantees that
 *   no earlier execution still reads or writes the range (write into the half of a double buffer
 *   the previous step has finished with) and keeps `src` unchanged until the copy has happened
 *   (pinned host memory keeps it asynchronous).
 * nn_buffer_read_async: device -> host copy of the range as the executions enqueued so far leave
 *   it, on a second transfer stream, concurrent with later executions; returns a ticket (>= 0) or a
 *   negative status.  The caller guarantees that later executions do not write the range before
 *   the read has landed.
 * nn_transfer_wait: blocks until the read named by a ticket (one of the last 64) has landed. */
NN_API int nn_buffer_write_async(int handle, const float *src, long long offset, long long count);
NN_API int nn_buffer_read_async(int handle, float *dst, long long offset, long long count);
NN_API int nn_transfer_wait(int ticket);
/* Fill count floats from offset with `value` (CBufferFloat::BufferInit). */
NN_API int nn_buffer_fill(int handle, float value, long long offset, long long count);
/* Device-to-device copy inside the context (CopyBufferRaw role). */
NN_API int nn_buffer_copy(int dst, long long dst_offset, int src, long long src_offset, long long count);
/* Size in bytes, or a negative status. */
NN_API long long nn_buffer_bytes(int handle);
/* Device address of a buffer (for interop with other CUDA code). */
NN_API void *nn_buffer_device_ptr(int handle);

/* ---------------------------------------------------------------- kernels */
/* COpenCL::KernelCreate(id, name) via the CreateKernel macro
 * (NeuroNet_Definitions.mqh:56-58, NeuroNet_Core.mqh:23192-23651).
 * name: a NeuroNet.cl kernel name.  id: any value in [0, 65535].
 * Beyond the NeuroNet.cl names, three kernels of this library (no reference counterpart) serve a
 * squashed-Gaussian soft actor-critic update; each covers global[0] * batch samples:
 *   "SACGaussianPolicy"  (outputs, noise, actions, log_probs, int action_dim)
 *       a = tanh(mu + exp(clamp(log_std, -20, 2)) eps), outputs [n][2A] = (mu, log_std)
 *   "SACTargetValue"     (q1, q2, reward, done, log_probs, target, float gamma, float alpha)
 *       y = r + gamma (1 - done) (min(q1, q2) - alpha log pi)
 *   "SACPolicyGradient"  (outputs, noise, actions, q1, q2, dq1, dq2, gradient, int action_dim,
 *                         float alpha)
 *       the ascent direction of min(q1, q2) - alpha log pi for (mu, log_std), each entry
 *       clamped to +-1e-2 like every output gradient of the reference. */
NN_API int nn_kernel_create(int id, const char *name);
/* Same, for callers whose strings are UTF-16 (MQL5 `string`). */
NN_API int nn_kernel_create_w(int id, const unsigned short *name_utf16);
NN_API int nn_kernel_free(int id);
/* COpenCL::SetArgumentBuffer / SetArgument (NeuroNet_Definitions.mqh:61-66). */
NN_API int nn_set_arg_buffer(int id, int arg_index, int buffer_handle);
NN_API int nn_set_arg_int(int id, int arg_index, int value);
NN_API int nn_set_arg_float(int id, int arg_index, float value);
/* Extension: number of independent samples processed by one execution
 * (default 1).  Per-sample buffers (inputs, outputs, gradients, activations)
 * hold `batch` consecutive copies of the per-sample layout the reference
 * kernel reads; parameter buffers (weights, moments, options) are shared.
 * Forward and input-gradient kernels produce the reference result for every
 * sample; weight-update kernels average the per-sample weight gradient over
 * the batch and then apply the reference update arithmetic once.  MatMult and MatMultGrad
 * take their batch in global[2] (variables; a shared second matrix with multvarsecond = 0,
 * whose gradient MatMultGrad sums over it) and refuse a batch above 1 with NN_ERR_UNSUPPORTED. */
NN_API int nn_set_batch(int id, int batch);
/* COpenCL::Execute (NeuroNet_Definitions.mqh:69-90): enqueue one execution.
 * offset may be NULL (must be zero); local may be NULL. */
NN_API int nn_execute(int id, int dims, const unsigned int *offset, const unsigned int *global,
               const unsigned int *local);
/* Number of CUDA kernels this library launched since nn_init. */
NN_API long long nn_launch_count(void);

/* ----------------------------------------------------------- command lists */
/* Extension: record the nn_execute calls between begin and end (they are not
 * run while recording) into a list that nn_cmdlist_run replays with one call.
 * A replay resolves buffer handles again and re-checks every bound. */
NN_API int nn_cmdlist_begin(void);
NN_API int nn_cmdlist_end(void); /* returns the list id (>= 0) */
NN_API int nn_cmdlist_run(int list);
/* Overwrite scalar argument arg_index of recorded execution `position`
 * (e.g. the bias-corrected Adam learning rate of each step). */
NN_API int nn_cmdlist_set_float(int list, int position, int arg_index, float value);
NN_API int nn_cmdlist_set_int(int list, int position, int arg_index, int value);
NN_API int nn_cmdlist_size(int list);
NN_API int nn_cmdlist_free(int list);

/* ------------------------------------------------------------ data parallel */
/* Extension: NCCL data parallelism over the GPUs of one node.
 * nn_dp_unique_id writes the 128-byte ncclUniqueId (rank 0 creates it, the
 * caller distributes it); nn_dp_init joins the communicator. */
NN_API int nn_dp_unique_id(unsigned char *id128);
NN_API int nn_dp_init(int rank, int world, const unsigned char *id128);
NN_API int nn_dp_shutdown(void);
/* Sum-allreduce `count` floats of a buffer in place on the context stream,
 * then scale by `scale` (1/world for a mean). */
NN_API int nn_dp_allreduce(int handle, long long offset, long long count, float scale);
/* Deferred-update region: between begin and end, weight-update kernels write
 * their batch-mean weight gradient into a gradient arena instead of applying
 * it, and their update (and any NormalizeWeights execution) is queued.  The
 * arena is averaged over the ranks in buckets: once 1 MB of new gradients has
 * gathered, an NCCL allreduce of that bucket starts on a communication stream
 * while the context stream goes on with the rest of backward.  At
 * nn_dp_update_end the last bucket is reduced, the context stream waits for
 * every bucket, and the queued updates run in their original order.  Every
 * rank must issue the same updates in the same order (the bucket boundaries,
 * and so the collectives, then agree). */
NN_API int nn_dp_update_begin(void);
NN_API int nn_dp_update_end(void);

/* ---- update without allocation -------------------------------------------
 * No counterpart in the reference (its OpenCL buffers are all created by the
 * host up front).  The batched dense UpdateWeightsAdam -- the same result as
 * nn_execute of "UpdateWeightsAdam" with global (outputs, inputs+1) and
 * nn_set_batch(batch) -- on plain device pointers (nn_buffer_device_ptr),
 * with the weight-gradient partials in a fixed 8 MiB device array inside the
 * library instead of context scratch, so the call never allocates device
 * memory (for hosts that give all free memory to their own pool, or that
 * cannot take an allocation's device-wide stall mid-session).
 *   matrix_w, matrix_m, matrix_v  [outputs][inputs+1]
 *   matrix_g [batch][outputs]   matrix_i [batch][inputs]
 * Runs on the context stream (nn_init first).  outputs*(inputs+1) above
 * 2,097,152 floats returns NN_ERR_BOUNDS.  nn_init looks up the array's
 * address on the context's device, which also loads the module that holds it
 * (under lazy module loading the array is reserved then, not at the first
 * call); if that look-up failed, the first call retries it and should come
 * before any stream capture starts and before the host takes the device's
 * free memory.  The array is shared by every call on a device: calls that
 * overlap in time race and must be ordered by the caller.  The update is
 * local to this process: inside nn_dp_update_begin .. end it returns
 * NN_ERR_STATE instead of applying one rank's gradient. */
NN_API int nn_update_weights_adam_fixed(float *matrix_w, const float *matrix_g, const float *matrix_i,
                                        float *matrix_m, float *matrix_v, int outputs, int inputs, int batch,
                                        float l, float b1, float b2);

#ifdef __cplusplus
}
#endif
#endif /* NN_B200_H */
