/*
 * nkb.h -- C ABI of libnkb.so, the B200 (sm_100a) runtime that replaces
 * NKIPy's Spike/libnrt layer.
 *
 * Every function returns an int status (NKB_OK == 0); on failure
 * nkb_last_error() gives a thread-local message.  Handles are opaque and
 * plain pointers/sizes cross the boundary: no torch or Python types.
 *
 * Reference interfaces replaced (paths inside shaojiex-aws/nkipy):
 *   spike/src/include/spike.h:28-86      Spike class (runtime, tensors, execute)
 *   spike/src/include/nrt_wrapper.h:13-33 NrtRuntime (init/close/core count)
 *   spike/src/include/tensor.h:14-53     NrtTensor (alloc, slice, read, write)
 *   spike/src/include/model.h:12-55      NrtModel (load NEFF, load_collectives, execute)
 *   spike/src/include/sys_trace.h:16-39  SystemTraceSession (device timing)
 *   spike/src/include/error.h:12-43      SpikeError / NrtError(status)
 *
 * A "plan" takes the place of a NEFF: a text launch plan produced by the
 * Python planner (kernel ids, launch parameters, buffer map); loading it
 * resolves every kernel and sizes the scratch arena, executing it launches
 * the kernels in order on one CUDA stream.
 */
#ifndef NKB_H
#define NKB_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define NKB_API __attribute__((visibility("default")))
#else
#define NKB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum nkb_status {
  NKB_OK = 0,
  NKB_ERR_INVALID = 1,     /* bad argument (size, index, handle)            */
  NKB_ERR_CUDA = 2,        /* a CUDA runtime call failed                     */
  NKB_ERR_PLAN = 3,        /* plan text malformed / unknown kernel           */
  NKB_ERR_UNSUPPORTED = 4, /* shape/dtype the kernel library does not cover  */
  NKB_ERR_NCCL = 5,        /* NCCL missing or a NCCL call failed             */
  NKB_ERR_STATE = 6,       /* runtime not initialised / handle freed         */
  NKB_ERR_DEVICE = 7       /* a kernel reported an error flag (bounded wait,
                              bad index); the CUDA context stays usable      */
};

typedef struct nkb_buf_s *nkb_buf;
typedef struct nkb_plan_s *nkb_plan;
typedef struct nkb_comm_s *nkb_comm;

/* ---- runtime (Spike::Spike / close / get_visible_neuron_core_count,
 *      spike.h:30-42; NrtRuntime nrt_wrapper.h:13-33) ----------------------- */
NKB_API int nkb_init(int device);
NKB_API int nkb_shutdown(void);
NKB_API int nkb_device_count(int *count);
NKB_API const char *nkb_last_error(void);
NKB_API const char *nkb_status_str(int status);
NKB_API int nkb_version(int *major, int *minor);

/* ---- device buffers (Spike::allocate_tensor / slice_from_tensor /
 *      free_tensor, spike.h:51-58; NrtTensor tensor.h:14-53) --------------- */
NKB_API int nkb_alloc(size_t bytes, int device, nkb_buf *out);
NKB_API int nkb_slice(nkb_buf src, size_t offset, size_t bytes, nkb_buf *out);
NKB_API int nkb_wrap(void *device_ptr, size_t bytes, int device, nkb_buf *out);
NKB_API int nkb_free(nkb_buf buf);
NKB_API int nkb_buf_info(nkb_buf buf, size_t *bytes, int *device, void **device_ptr);

/* ---- data movement, bounds-checked (Spike::tensor_write / tensor_read,
 *      spike.h:59-63; NrtTensor::write/read tensor.cpp:65-105) ------------- */
NKB_API int nkb_h2d(nkb_buf dst, const void *src, size_t bytes, size_t offset);
NKB_API int nkb_d2h(nkb_buf src, void *dst, size_t bytes, size_t offset);
NKB_API int nkb_memset(nkb_buf dst, int value, size_t bytes, size_t offset);
/* Streams, events and asynchronous (bounds-checked) copies, for callers that
 * overlap the copies of one step with the compute of another.  The
 * reference's tensor_write / tensor_read are synchronous and have no such
 * calls; these add the pipelined form.  Streams are non-blocking streams of
 * the runtime's device; NULL stream = the runtime's own stream.  Host memory
 * must be page-locked (pinned) for the copies to run asynchronously. */
NKB_API int nkb_stream_create(void **stream);
NKB_API int nkb_stream_destroy(void *stream);
NKB_API int nkb_stream_synchronize(void *stream);
NKB_API int nkb_event_create(void **event);
NKB_API int nkb_event_destroy(void *event);
NKB_API int nkb_event_record(void *event, void *stream);
NKB_API int nkb_stream_wait_event(void *stream, void *event);
NKB_API int nkb_h2d_async(nkb_buf dst, const void *src, size_t bytes, size_t offset, void *stream);
NKB_API int nkb_d2h_async(nkb_buf src, void *dst, size_t bytes, size_t offset, void *stream);
/* device-to-device copy between buffers (synchronous, bounds-checked) */
NKB_API int nkb_copy(nkb_buf dst, size_t dst_offset, nkb_buf src, size_t src_offset, size_t bytes);

/* ---- plans (Spike::load_model / unload_model / get_tensor_info,
 *      spike.h:46-48,69; NrtModel model.h:12-55) ---------------------------- */
/* `device` must be the device nkb_init was given (NKB_ERR_INVALID otherwise);
   it is made current on the calling thread, and the plan's fused elementwise
   steps are compiled and loaded there (nkb_ew_compiler_stats). */
NKB_API int nkb_plan_load(const char *text, size_t len, int device, nkb_plan *out);
NKB_API int nkb_plan_free(nkb_plan plan);
NKB_API int nkb_plan_num_io(nkb_plan plan, int *n_inputs, int *n_outputs);
NKB_API int nkb_plan_io_bytes(nkb_plan plan, int is_output, int index, size_t *bytes);
NKB_API int nkb_plan_num_consts(nkb_plan plan, int *n_consts);
NKB_API int nkb_plan_set_const(nkb_plan plan, int const_index, const void *host, size_t bytes);
NKB_API int nkb_plan_num_launches(nkb_plan plan, int *n_launches);
/* Kernels one graph-replayed execute of `plan` launches: the kernel nodes of
   the CUDA graph captured last (a step may launch none, one or two kernels);
   -1 before the first graph execute.  No counterpart in the reference (its
   NEFF is one program). */
NKB_API int nkb_plan_graph_kernels(nkb_plan plan, int *n_kernels);
/* One graph replay of `plan` with an event record node before the first step
   and after each step (graph captured once per io binding and cached):
   *total_ms = the execute, step_ms[i] (num_launches entries) = step i inside
   it.  Launches here do not use programmatic dependent launch.  No counterpart
   in the reference (its profile is per NEFF). */
NKB_API int nkb_time_execute_steps(nkb_plan plan, const nkb_buf *ins, int n_in, const nkb_buf *outs, int n_out,
                                   float *total_ms, float *step_ms);
NKB_API int nkb_plan_scratch_bytes(nkb_plan plan, size_t *bytes);
/* Counters of the elementwise chain compiler since the library was loaded:
   distinct "ew" steps compiled to a specialised kernel (NVRTC, at plan load),
   steps it could not compile (they run on the interpreter kernel) and launches
   of compiled kernels issued by nkb_execute (a graph replay re-runs captured
   launches without counting them).  Any pointer may be NULL.  No counterpart in the
   reference (neuronx-cc compiles the whole kernel ahead of time). */
NKB_API int nkb_ew_compiler_stats(int64_t *compiled, int64_t *failed, int64_t *launched);
/* Compiles the specialised kernel of one elementwise step from its integer
   parameters (the "ew" step of a plan), without a device: warms the compiler's
   cache before nkb_plan_load, and lets a host without a GPU check that a
   plan's chains compile.  *taken = 1 when the step will run on a compiled
   kernel.  No counterpart in the reference. */
NKB_API int nkb_ew_compile_step(const int64_t *ints, size_t n_ints, int *taken);

/* ---- execution (Spike::execute spike.h:65-68, nrt_execute model.cpp:90-110).
 * ins/outs are indexed as the plan's io table; stream may be NULL (the
 * runtime's stream).  use_graph != 0 captures the launch sequence into a
 * CUDA graph on first use and replays it while the buffers are unchanged. */
NKB_API int nkb_execute(nkb_plan plan, const nkb_buf *ins, int n_in, const nkb_buf *outs, int n_out,
                void *stream, int use_graph);

/* Device timing of `iters` back-to-back executes after `warmup` (CUDA events
 * on the execute stream), replacing SystemTraceSession + nc_exec_running
 * durations (sys_trace.h:16-39, spike_model.py:42-79).  Writes per-iteration
 * milliseconds into ms_out[0..iters-1]. */
NKB_API int nkb_time_execute(nkb_plan plan, const nkb_buf *ins, int n_in, const nkb_buf *outs, int n_out,
                     int warmup, int iters, int use_graph, float *ms_out);
NKB_API int nkb_synchronize(void);

/* Per-launch device time: runs the plan `iters` times with CUDA events
 * between consecutive kernel launches and writes the mean duration of each
 * launch (milliseconds) into step_ms[0..n_launches-1].  Each run is preceded
 * by an L2 flush (256 MiB written, then read back) in a temporary buffer. */
NKB_API int nkb_time_steps(nkb_plan plan, const nkb_buf *ins, int n_in, const nkb_buf *outs, int n_out, int iters,
                           float *step_ms);

/* One execute with CUDA events between its launches (no graph): writes each
 * launch's start (relative to the first) and duration in milliseconds into
 * start_ms / dur_ms[0..n_launches-1].  Every launch of the runtime is also an
 * NVTX range named after its kernel.  Replaces the per-execute profile of the
 * reference (Spike::execute with save_trace / ntff_name, spike/src/model.cpp:97-103). */
NKB_API int nkb_trace_execute(nkb_plan plan, const nkb_buf *ins, int n_in, const nkb_buf *outs, int n_out,
                              float *start_ms, float *dur_ms);

/* Reads and clears the device error flag that a kernel raises when one of
 * its bounded waits expires (the kernel then frees its resources and exits
 * instead of hanging; the CUDA context stays usable). */
NKB_API int nkb_device_error(int *flag);

/* Budget of every wait on a counter that another rank (or another CTA)
 * advances -- the fused GEMM + all-reduce's row-block arrivals, the in-switch
 * all-reduce's barrier -- in microseconds at the GPU's maximum SM clock
 * (default 1,000,000).  Read by each launch.  No counterpart in the reference,
 * whose collectives run inside NRT with its own timeouts. */
NKB_API int nkb_set_wait_limit_us(uint64_t us);
NKB_API int nkb_get_wait_limit_us(uint64_t *us);
/* Diagnostics of the bounded wait: one thread polls the device counter
 * `counter` until it reaches `target` or the wait limit passes; an expired
 * wait is reported by nkb_device_error() like a kernel's, and the CUDA
 * context stays usable.  Lets a test drive the expiry path on one GPU with a
 * counter that nothing advances.  No counterpart in the reference. */
NKB_API int nkb_wait_probe(const uint32_t *counter, uint32_t target, void *stream);

/* ---- collectives (NrtModel load with nrt_load_collectives(rank, world),
 *      model.cpp:38-52).  NCCL is resolved at run time (dlopen).  The unique
 *      id is NKB_COMM_ID_BYTES bytes, produced on rank 0 and broadcast by the
 *      caller's control plane (torch.distributed in the Python layer). ------ */
#define NKB_COMM_ID_BYTES 128
NKB_API int nkb_comm_unique_id(void *id_out);
NKB_API int nkb_comm_init(const void *id, int rank, int world, int device, nkb_comm *out);
NKB_API int nkb_comm_free(nkb_comm comm);
NKB_API int nkb_plan_bind_comm(nkb_plan plan, nkb_comm comm);
NKB_API int nkb_comm_all_reduce(nkb_comm comm, nkb_buf buf, size_t count, int dtype, void *stream);
/* Binds a symmetric region to the communicator: `bytes` at `local` on this
 * rank, the same region through an NVLink multicast object at `multicast`,
 * and every rank's region as mapped in this process (`peers`, one per rank).
 * Afterwards bf16/fp32 sum all-reduces whose slices are whole 16-byte
 * vectors and that fit the region run as one kernel reducing inside NVSwitch
 * (multimem); the others keep using NCCL.  The last nkb_comm_symm_flag_bytes()
 * bytes of the region hold barrier flags: this call zeroes this rank's, and
 * the caller synchronises the ranks before the next all-reduce.  No
 * counterpart in the reference, whose collectives run inside NRT; the
 * allocation itself is the caller's (PyTorch symmetric memory in the Python
 * layer). */
NKB_API int nkb_comm_bind_symm(nkb_comm comm, void *local, void *multicast, void *const *peers, int n_peers,
                               size_t bytes);
NKB_API size_t nkb_comm_symm_flag_bytes(void);

/* dtype codes used by plans and nkb_comm_all_reduce */
enum nkb_dtype {
  NKB_F32 = 0, NKB_BF16 = 1, NKB_F16 = 2, NKB_I32 = 3, NKB_U32 = 4,
  NKB_I8 = 5, NKB_U8 = 6, NKB_BOOL = 7, NKB_I16 = 8, NKB_U16 = 9,
  NKB_F8E4M3 = 10, NKB_F8E5M2 = 11
};

/* ---- direct kernel entry points (no plan): used by the Python layer's
 *      micro-benchmarks and by the parity tests.  All pointers are device
 *      pointers of the current device; stream may be NULL. ----------------- */

/* Row softmax over the last axis: out[r,:] = exp(x[r,:]-max)/sum.  The
 * composition traced from tests/kernels/softmax.py:7-10. */
NKB_API int nkb_softmax_rows(const void *x, int x_dtype, void *out, int out_dtype, int64_t rows, int64_t cols,
                     void *stream);

/* out = (x + r) / sqrt(mean((x + r)^2) + eps) * w, rows of `cols`; r and
 * sum_out may be NULL.  examples/models/qwen3_embedding/kernels/rmsnorm.py:4-16
 * with the residual add of examples/models/qwen3/kernels/transformer_layer.py:60. */
NKB_API int nkb_rmsnorm_rows(const void *x, const void *r, const void *w, void *out, void *sum_out, int dtype,
                     int w_dtype, int64_t rows, int64_t cols, float eps, void *stream);

/* C[b] = A[b] @ B[b], bf16 inputs, fp32 accumulation, bf16 or fp32 output
 * (core/ops/linalg.py:15-125, HLO dot).  A is (M,K) row-major with row
 * stride lda, B is (K,N) row-major with row stride ldb, C is (M,N) with row
 * stride ldc; batch strides in elements (0 = broadcast). */
NKB_API int nkb_gemm_bf16(const void *A, const void *B, void *C, int c_dtype, int64_t M, int64_t N, int64_t K,
                  int64_t lda, int64_t ldb, int64_t ldc, int64_t batch, int64_t sA, int64_t sB, int64_t sC,
                  void *stream);

/* Top-k along the last axis of dense (rows, cols) x: values (rows, k) in x's
 * dtype, largest first, and their column indices (rows, k) as uint32; ties
 * keep the lower column first.  The reference's topk op (core/ops/nn.py:65-152,
 * HLO TopK largest=true; is_ascend traces as negate -> topk -> negate), used
 * by greedy sampling (examples/models/qwen3/kernels/sampling.py:113-147). */
NKB_API int nkb_topk_rows(const void *x, int dtype, void *values, uint32_t *indices, int64_t rows, int64_t cols,
                          int64_t k, void *stream);

/* All-gather / reduce-scatter (sum) of `count` elements per rank on the
 * leading axis, rank-major (core/ops/collectives.py:34-53,148-178; HLO
 * all-gather / reduce-scatter run by NRT in the reference).  `send` holds
 * this rank's count elements (all-gather) or world * count (reduce-scatter),
 * `recv` the other size.  NCCL. */
NKB_API int nkb_comm_all_gather(nkb_comm comm, const void *send, void *recv, size_t count, int dtype, void *stream);
NKB_API int nkb_comm_reduce_scatter(nkb_comm comm, const void *send, void *recv, size_t count, int dtype,
                                    void *stream);
/* All-to-all (core/ops/collectives.py:217-233): send and recv hold world
 * blocks of `count` elements, rank-major; block j of send goes to rank j and
 * block i of recv comes from rank i.  NCCL grouped send/recv. */
NKB_API int nkb_comm_all_to_all(nkb_comm comm, const void *send, void *recv, size_t count, int dtype, void *stream);

/* Allocation-free chunked causal linear attention.  No counterpart in the
 * reference: it serves callers that cannot allocate device memory when they
 * run this kernel, such as a host that has reserved the whole GPU for its own
 * caching allocator, or a latency-critical loop where cudaMalloc/cudaFree
 * could block or synchronise the device.  Same computation as the planned
 * "linattn" kernel (feature map elu + 1, chunk 64, fp32 running state); q, k,
 * v and out are dense bf16 (B, H, T, 128) device arrays of the current device,
 * T a multiple of 64, 16-byte aligned.  The caller passes inputs and the
 * output; the kernel's segment-state workspace is a fixed device array of
 * NKB_LINATTN_SCRATCH_BYTES inside libnkb, held by every GPU that loads the
 * library until the process exits.  The workspace is B * H * ceil(T / 1024)
 * * 66,048 bytes (one fp32 128 x 128 state and key sum per 1024-token
 * segment) when B * H < 96 and T > 1024, and none otherwise (each head is
 * then one segment); sizes whose workspace would exceed the array are
 * rejected with NKB_ERR_INVALID.  The function itself calls no cudaMalloc,
 * cudaFree or allocating library routine; its first call on a device looks up
 * the array's device address (cudaGetSymbolAddress), so make that first call
 * before any stream capture (the lookup is repeated, once, on a device whose
 * CUDA context was reset since).  All calls share the one array: calls that
 * overlap on the GPU (different streams, or several host threads) race and
 * must be serialised by the caller.  Each call writes every workspace entry
 * it reads, so the array needs no clearing between calls.  The return status
 * covers argument checks and the launch only: the kernel's waits are
 * bounded, and one that expires is reported afterwards by nkb_device_error()
 * (read it after synchronising the stream; the output is then invalid). */
#define NKB_LINATTN_SCRATCH_BYTES (64u << 20)
NKB_API int nkb_linear_attention_noalloc(const void *q, const void *k, const void *v, void *out, int64_t B, int64_t H,
                                         int64_t T, int64_t D, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* NKB_H */
