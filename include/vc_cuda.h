/*
 * vc_cuda.h -- C ABI of VectorCore's B200 (sm_100a) CUDA device.
 *
 * This is the drop-in boundary: VectorCore's C++20 host (or any FFI) binds
 * these entry points to add a `cuda` device next to `cpu` and `metal`. Every
 * function is extern "C", takes plain pointers and sizes, never throws, and
 * returns a vc_status; the message of the last failure on the calling thread
 * is available from vc_cuda_last_error(). There is no CPU fallback: without a
 * usable GPU every compute entry point fails with VC_ERR_RUNTIME.
 *
 * Conventions
 *  - Tensors are contiguous row-major float32 in device memory unless a
 *    stride array is passed. Shapes and strides are size_t element counts
 *    (the reference's Shape / Strides = std::vector<std::size_t>,
 *    include/vectorcore/shape.hpp:9-10).
 *  - All work is enqueued on one CUDA stream per process (vc_cuda_stream());
 *    calls return before the GPU finishes. A call with two independent
 *    halves (the two gradients of vc_cuda_binary_backward) may run one half
 *    on an internal second stream, forked from and joined back to that
 *    stream with events before it returns, so work ordered on
 *    vc_cuda_stream() sees the whole result. Only vc_cuda_download() and
 *    vc_cuda_synchronize() block, as MetalBackend::download / synchronize do
 *    (src/metal/metal_backend.mm:205-211, 415-444).
 *  - Errors detected on the device (bounded waits that gave up, out-of-range
 *    class targets) are recorded in a device error word and reported by the
 *    next blocking call, like Metal's completion-handler errors
 *    (src/metal/metal_backend.mm:545-549).
 *  - Scratch memory needed by a kernel (per-CTA partials) comes from the
 *    device's stream-ordered pool and is returned to it before the call
 *    returns; callers never see it.
 *  - Results match the reference's CPU path: bit-exact for add, sub, mul,
 *    div, neg, relu, max and argmax (first index wins ties); within 2 ulp of
 *    glibc for exp, log and sigmoid (a table-driven float exponential of this
 *    library, CUDA's logf); sums accumulate in double and round once, like
 *    cpu::sum / cpu::reduce_axis.
 *
 * Status codes map onto the reference's exception types
 * (src/ops.cpp, src/shape.cpp): invalid_argument -> VC_ERR_INVALID,
 * out_of_range -> VC_ERR_OUT_OF_RANGE, overflow_error -> VC_ERR_OVERFLOW,
 * runtime_error -> VC_ERR_RUNTIME / VC_ERR_OOM / VC_ERR_TIMEOUT.
 */
#ifndef VC_CUDA_H
#define VC_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum vc_status {
    VC_OK = 0,
    VC_ERR_INVALID = 1,
    VC_ERR_OUT_OF_RANGE = 2,
    VC_ERR_OVERFLOW = 3,
    VC_ERR_RUNTIME = 4,
    VC_ERR_OOM = 5,
    VC_ERR_TIMEOUT = 6
} vc_status;

/* Same numbering as vectorcore::cpu::BinaryOp / UnaryOp / ReduceOp
 * (include/vectorcore/cpu_backend.hpp:9-11), extended with Mean. */
typedef enum vc_binary_op { VC_ADD = 0, VC_SUB = 1, VC_MUL = 2, VC_DIV = 3 } vc_binary_op;
typedef enum vc_unary_op {
    VC_NEG = 0, VC_RELU = 1, VC_SIGMOID = 2, VC_RELU_GRAD = 3, VC_EXP = 4, VC_LOG = 5
} vc_unary_op;
typedef enum vc_reduce_op {
    VC_REDUCE_SUM = 0, VC_REDUCE_MAX = 1, VC_REDUCE_ARGMAX = 2, VC_REDUCE_MEAN = 3
} vc_reduce_op;

/* ---- device, errors, synchronisation ------------------------------------ */

/* 1 when a CUDA device of compute capability 10.x is usable, else 0.
 * Replaces metal_available() (include/vectorcore/metal_backend.hpp:58). */
int vc_cuda_available(void);

/* Select `device`, create the stream and the buffer pool. Idempotent; every
 * other entry point calls it with device 0 if it was never called.
 * Replaces MetalBackendImpl's constructor (src/metal/metal_backend.mm:80-130). */
vc_status vc_cuda_init(int device);

/* Message of the last failure on this thread ("" if none).
 * Replaces MetalBackend::last_error() (metal_backend.hpp:17). */
const char* vc_cuda_last_error(void);

/* Device name, e.g. "NVIDIA B200" (MetalBackend::device_name(), :16). */
vc_status vc_cuda_device_name(char* buffer, size_t length);

/* Block until all enqueued work finished; report asynchronous device errors.
 * Replaces MetalBackend::synchronize() (metal_backend.hpp:52) and the free
 * function vectorcore::synchronize() (:63). */
vc_status vc_cuda_synchronize(void);

/* The stream all work is enqueued on (a cudaStream_t). vc_cuda_set_stream
 * replaces it (synchronising the old one first); NULL restores the device's
 * own stream. No reference counterpart (Metal has one command queue). */
void* vc_cuda_stream(void);
vc_status vc_cuda_set_stream(void* stream);

/* Streaming multiprocessors of the current device. */
int vc_cuda_sm_count(void);

/* ---- memory --------------------------------------------------------------- */

/* Device buffer of at least `bytes` from the stream-ordered size-class pool
 * (256 B minimum, powers of two up to 4 MiB, then 1 MiB steps), 256-byte
 * aligned. Replaces MetalBackend::allocate (metal_backend.hpp:22;
 * src/metal/metal_backend.mm:161-191, 487-510). */
vc_status vc_cuda_alloc(size_t bytes, void** pointer);

/* Return a buffer to the pool. Stream-ordered: work already enqueued that
 * reads or writes it completes first, because the next user of the block is
 * enqueued after it on the same stream. Replaces the deferred release of
 * MetalStorage (src/metal/metal_backend.mm:184-191, 531-554). */
vc_status vc_cuda_free(void* pointer);

/* Pool statistics and trimming (cached blocks back to the driver). */
vc_status vc_cuda_pool_stats(size_t* cached_bytes, size_t* in_use_bytes,
                             size_t* hits, size_t* misses);
vc_status vc_cuda_pool_trim(void);

/* Page-locked host staging memory for fast, asynchronous copies. */
vc_status vc_cuda_host_alloc(size_t bytes, void** pointer);
vc_status vc_cuda_host_free(void* pointer);

/* Host -> device copy of `bytes`. Returns once `src` may be reused.
 * Replaces MetalBackend::upload (metal_backend.hpp:23). */
vc_status vc_cuda_upload(void* dst, const void* src, size_t bytes);

/* Device -> host copy of `bytes`; waits for all enqueued work first.
 * Replaces MetalBackend::download (metal_backend.hpp:25). */
vc_status vc_cuda_download(void* dst, const void* src, size_t bytes);

/* Asynchronous host <-> device copies (no counterpart in the reference,
 * whose MetalBackend::upload / download are synchronous). The host buffer
 * must be page-locked (vc_cuda_host_alloc), else VC_ERR_INVALID. Each copy
 * runs on a copy stream of its direction, after the work enqueued before
 * the call, and returns a ticket; work enqueued later does NOT wait for it
 * until vc_cuda_transfer_wait(ticket) (which enqueues the dependency and
 * returns at once). vc_cuda_transfer_sync(ticket) blocks the host until the
 * copy completed: only then may the host buffer be reused (upload) or read
 * (download). Freeing a device buffer orders its reuse after the transfers
 * still touching it; writing it with later work before
 * vc_cuda_transfer_wait is the caller's race. vc_cuda_synchronize waits for
 * every transfer too. Not allowed during graph capture. */
vc_status vc_cuda_upload_async(void* dst, const void* src, size_t bytes, uint64_t* ticket);
vc_status vc_cuda_download_async(void* dst, const void* src, size_t bytes, uint64_t* ticket);
vc_status vc_cuda_transfer_wait(uint64_t ticket);
vc_status vc_cuda_transfer_sync(uint64_t ticket);

/* Device -> device copy and fill, enqueued. */
vc_status vc_cuda_copy(void* dst, const void* src, size_t bytes);
vc_status vc_cuda_fill(float* out, size_t count, float value);

/* ---- elementwise --------------------------------------------------------- */

/* out = a (op) b with NumPy broadcasting (shapes right-aligned).
 * Strides may be NULL for contiguous operands. Fast paths: same shape,
 * scalar operand, row / column broadcast (128-bit accesses); any other
 * layout resolves per-row operand offsets per tile in shared memory and
 * never materialises an expanded operand. 64-bit indexing throughout.
 * Replaces MetalBackend::binary (metal_backend.hpp:27-30) and
 * cpu::binary (src/cpu/cpu_backend.cpp:275-289). */
vc_status vc_cuda_binary(int op,
                         const float* a, const size_t* a_shape, const size_t* a_strides, int a_rank,
                         const float* b, const size_t* b_shape, const size_t* b_strides, int b_rank,
                         float* out, const size_t* out_shape, int out_rank);

/* out = a (op) scalar, or scalar (op) a when scalar_first != 0, with the
 * scalar passed by value (no one-element upload). Equivalent to
 * Tensor::operator+(Tensor, float) & co. (src/tensor.cpp:323-330). */
vc_status vc_cuda_binary_scalar(int op, const float* a, float scalar, int scalar_first,
                                float* out, size_t count);

/* out = op(in). Replaces MetalBackend::unary (metal_backend.hpp:31-32) and
 * cpu::unary (src/cpu/cpu_backend.cpp:291-316). */
vc_status vc_cuda_unary(int op, const float* in, float* out, size_t count);

/* Fused vector-Jacobian products of the unary ops, one pass each
 * (src/ops.cpp:158-164, 360-376, 395-413):
 *   VC_NEG -g;  VC_EXP g*y;  VC_LOG g/x;  VC_RELU g*relugrad(x);
 *   VC_SIGMOID (g*y)*(1-y).
 * x = forward input, y = forward output (either may be NULL when unused). */
vc_status vc_cuda_unary_backward(int op, const float* x, const float* y, const float* g,
                                 float* dx, size_t count);

/* out (t_shape) = value broadcast + 0.0f. Replaces detail::broadcast_to
 * (src/autograd.cpp:74-91). */
vc_status vc_cuda_broadcast_to(const float* value, const size_t* v_shape, int v_rank,
                               float* out, const size_t* t_shape, int t_rank);

/* target += alpha * source. Replaces MetalBackend::axpy_inplace
 * (metal_backend.hpp:49-50). */
vc_status vc_cuda_axpy(float* target, const float* source, size_t count, float alpha);

/* ---- broadcast-gradient reduction (autograd) ------------------------------ */

/* out (t_shape) = sum of g over every axis where t_shape (right-aligned) is
 * 1 and g is not: ONE fused strided reduce over all those axes, double
 * accumulation. Replaces detail::sum_to_shape (src/autograd.cpp:50-72). */
vc_status vc_cuda_sum_to_shape(const float* g, const size_t* g_shape, int g_rank,
                               float* out, const size_t* t_shape, int t_rank);

/* Gradients of out = a (op) b for the upstream g, each computed and reduced
 * to its operand's shape in one pass without materialising the broadcast
 * product (src/ops.cpp:98-156):
 *   add: da = S(g), db = S(g);  sub: da = S(g), db = S(-g);
 *   mul: da = S(g*b), db = S(g*a);  div: da = S(g/b), db = S(-(g*a)/(b*b)).
 * g has g_shape, which must broadcast to the output shape (a dense gradient
 * has the output shape; a 0-d g is the broadcast scalar of a sum()).
 * da / db may be NULL to skip. */
vc_status vc_cuda_binary_backward(int op,
                                  const float* a, const size_t* a_shape, int a_rank,
                                  const float* b, const size_t* b_shape, int b_rank,
                                  const float* g, const size_t* g_shape, int g_rank,
                                  float* da, float* db);

/* ---- reductions ------------------------------------------------------------ */

/* Reduce all `count` elements: SUM / MEAN into out_value[0]; MAX into
 * out_value[0] (and its index into out_index[0] if not NULL); ARGMAX writes
 * the index (as float, the reference's convention) to out_value[0] when not
 * NULL and as int64 to out_index[0] when not NULL. Deterministic: fixed
 * 65536-element chunks, double partials combined in chunk order.
 * Replaces MetalBackend::reduce_sum (metal_backend.hpp:40-41) and
 * cpu::sum (src/cpu/cpu_backend.cpp:392-418). */
vc_status vc_cuda_reduce_all(int op, const float* in, size_t count, float* out_value,
                             int64_t* out_index);

/* Reduce the middle axis of a contiguous [outer, length, inner] view into
 * [outer, inner] (same out_value / out_index convention as reduce_all).
 * Max/argmax: strict '>' scan semantics of the reference -- first index
 * wins ties, a NaN only wins at index 0. Replaces MetalBackend::reduce_axis
 * (metal_backend.hpp:42-44) and cpu::reduce_axis (cpu_backend.cpp:420-460). */
vc_status vc_cuda_reduce_axis(int op, const float* in, size_t outer, size_t length,
                              size_t inner, float* out_value, int64_t* out_index);

/* out [outer, length, inner] = 0 except out[o, idx[o,i], i] = values[o,i]
 * (indices as float or int64; pass exactly one). Replaces
 * MetalBackend::scatter_axis (metal_backend.hpp:45-47). */
vc_status vc_cuda_scatter_axis(const float* values, const float* indices_f32,
                               const int64_t* indices_i64, float* out,
                               size_t outer, size_t length, size_t inner);

/* Backward of a reduction along an axis, fused into one pass:
 * SUM: out = g + 0 broadcast;  MEAN: out = g / length + 0 broadcast;
 * MAX: scatter of g at the argmax indices (int64). src/ops.cpp:304-347. */
vc_status vc_cuda_reduce_axis_backward(int op, const float* g, const int64_t* indices,
                                       float* out, size_t outer, size_t length, size_t inner);

/* ---- softmax family (fused: HBM reads each input once) ---------------------- */
/* Rows of 8192-40960 floats (forward) stream through a ring of shared-memory
 * slots fed by bulk copies, one CTA per SM; shorter rows and the backward use
 * one CTA per row group with an L2 re-read; longer rows a CTA cluster per
 * row; other axes a column kernel. All give the same results contract. */

/* y = log_softmax / softmax of x along the middle axis of [outer, length,
 * inner], computed as the reference does (src/ops.cpp:378-388): m = row max,
 * s = float(double sum of expf(x - m)), log_softmax = (x - m) - logf(s),
 * softmax = expf(log_softmax). row_max / row_sum (optional, outer*inner
 * floats) receive m and s for the backward kernels. */
vc_status vc_cuda_log_softmax(const float* x, float* y, float* row_max, float* row_sum,
                              size_t outer, size_t length, size_t inner);
vc_status vc_cuda_softmax(const float* x, float* y, float* row_max, float* row_sum,
                          size_t outer, size_t length, size_t inner);

/* dx for upstream g, given x and the saved row_max / row_sum: the reference
 * autograd chain of log_softmax (and of softmax = exp(log_softmax)) in one
 * pass over x and g. */
vc_status vc_cuda_log_softmax_backward(const float* x, const float* row_max,
                                       const float* row_sum, const float* g, float* dx,
                                       size_t outer, size_t length, size_t inner);
vc_status vc_cuda_softmax_backward(const float* x, const float* row_max,
                                   const float* row_sum, const float* g, float* dx,
                                   size_t outer, size_t length, size_t inner);

/* Mean softmax cross-entropy of [batch, classes] logits and int64 class
 * targets (device memory), without a one-hot mask (src/nn.cpp:31-53).
 * loss[0] = -(float)(sum of log_softmax at the targets) / batch_total,
 * where batch_total = batch when 0 is passed (a sharded batch passes the
 * global row count). Optional outputs: row_max / row_sum for the backward,
 * partial[0] = the double sum of this call's row terms (for a cross-GPU
 * ordered combine). Out-of-range targets fail at the next blocking call. */
vc_status vc_cuda_cross_entropy(const float* logits, const int64_t* targets, size_t batch,
                                size_t classes, size_t batch_total, float* loss,
                                float* row_max, float* row_sum, double* partial);

/* dlogits for the upstream gradient upstream[0] (a device scalar, so the
 * call needs no host round trip): the reference chain
 * dx = dls + ((dl / s) + 0) * expf(x - m) with dls = -(u/B) at the target. */
vc_status vc_cuda_cross_entropy_backward(const float* logits, const int64_t* targets,
                                         const float* row_max, const float* row_sum,
                                         const float* upstream, size_t batch, size_t classes,
                                         size_t batch_total, float* dlogits);

/* ---- CUDA graphs ------------------------------------------------------------
 * No counterpart in the reference (Metal encodes one command buffer per op,
 * src/metal/metal_backend.mm). Capture the library stream's work between
 * begin and end into a replayable graph: launch-bound chains (config 1) then
 * cost one launch. Every pool block allocated during the capture belongs to
 * the graph: it may be reused within the capture, and once freed after it
 * stays reserved (replays still use it) until vc_cuda_graph_destroy returns
 * it to the pool. Tensors created during the capture hold the buffers each
 * replay rewrites. Anything that synchronises the stream (download,
 * vc_cuda_synchronize, matmul) cannot be captured: vc_cuda_graph_end then
 * fails and the capture is discarded. One capture at a time per process. */
vc_status vc_cuda_graph_begin(void);
vc_status vc_cuda_graph_end(void** graph);
vc_status vc_cuda_graph_launch(void* graph);          /* enqueue one replay */
vc_status vc_cuda_graph_nodes(void* graph, size_t* nodes);
vc_status vc_cuda_graph_destroy(void* graph);

/* ---- fused forward chains ---------------------------------------------------
 * relu(x + b).sum() for x [rows, cols] and a row-broadcast bias b [cols], as
 * ONE launch each way. Replaces the reference's op-by-op chain
 * binary_forward (src/ops.cpp:27-41) -> relu (:395-403) -> sum (:288-302)
 * and its backward broadcast_to -> relu backward -> sum_to_shape
 * (src/autograd.cpp:50-91) for this pattern. */

/* loss[0] = float(sum of relu(x + b)); loss_partial[0] (optional) = the
 * unrounded double sum (a shard's partial). Either output may be null, not
 * both. The forward's last-CTA ticket is a counter owned by the stream the
 * call is enqueued on, so calls in flight on different streams do not share
 * it; a CUDA graph keeps the counter of the stream it was captured on, so
 * replay one graph on one stream at a time. */
vc_status vc_cuda_bias_relu_sum(const float* x, const float* b, size_t rows, size_t cols, float* loss,
                                double* loss_partial);
/* Given the upstream gradient u (device scalar) of the sum:
 * dx = (u + 0) * (x + b > 0 ? 1 : 0) (bit-exact with the reference),
 * db[j] = float(sum over rows of dx[:, j]), or db_partial[j] unrounded when
 * db is null. */
vc_status vc_cuda_bias_relu_sum_backward(const float* x, const float* b, const float* upstream, size_t rows,
                                         size_t cols, float* dx, float* db, double* db_partial);

/* ---- multi-GPU: leading-axis shards, partials combined in rank order -----
 * No counterpart in the reference (it is single-device). One process per
 * GPU; each rank reduces its shard into an unrounded partial, the partials
 * are all-gathered ([nranks][count], rank-major), and every rank combines
 * them in rank order 0..R-1, so results are independent of the collective's
 * internal order. */

/* This shard's part of a reduction over the middle axis of [outer, length,
 * inner]: SUM/MEAN -> partial_sum (double, not rounded); MAX/ARGMAX ->
 * partial_value + partial_index (int64, with index_base -- the shard's first
 * row -- added). continuation != 0 for every shard but the first: the
 * "NaN at index 0 wins" rule belongs to the first shard, and a later shard
 * without a candidate reports index -1. */
vc_status vc_cuda_reduce_axis_partial(int op, const float* in, size_t outer, size_t length, size_t inner,
                                      int64_t index_base, int continuation, double* partial_sum,
                                      float* partial_value, int64_t* partial_index);

/* vc_cuda_binary_backward's reductions, written as unrounded double
 * partials (e.g. a bias gradient over a sharded batch axis). */
vc_status vc_cuda_binary_backward_partial(int op,
                                          const float* a, const size_t* a_shape, int a_rank,
                                          const float* b, const size_t* b_shape, int b_rank,
                                          const float* g, const size_t* g_shape, int g_rank,
                                          double* da_partial, double* db_partial);

/* Combine nranks partials in rank order. SUM/MEAN: out = float(sum) (negated
 * when negate != 0), divided by divisor when divisor != 0 -- the mean
 * cross-entropy of a sharded batch is (SUM, negate=1, divisor=B).
 * MAX/ARGMAX: the first maximal element (a lower rank wins ties); out_value
 * gets the value (MAX) or the index as float (ARGMAX), out_index the int64. */
vc_status vc_cuda_combine_partials(int op, const double* partial_sum, const float* partial_value,
                                   const int64_t* partial_index, int nranks, size_t count, float divisor,
                                   int negate, float* out_value, int64_t* out_index);

/* NCCL communicator (libnccl.so.2 loaded at run time). Rank 0 creates the
 * 128-byte id and every rank passes it to comm_init (the id travels through
 * any host channel, e.g. torch.distributed's store). Non-blocking; each wait
 * is bounded by timeout_ms, after which the communicator is aborted and the
 * call returns VC_ERR_TIMEOUT. */
vc_status vc_cuda_comm_unique_id(void* id, size_t bytes);
vc_status vc_cuda_comm_init(int nranks, int rank, const void* id, size_t bytes, int timeout_ms);
/* recv [nranks * bytes_per_rank] = every rank's send, in rank order; enqueued. */
vc_status vc_cuda_comm_allgather(const void* send, void* recv, size_t bytes_per_rank);
/* `count` all-gathers (recvs[i] [nranks * bytes_per_rank[i]] = every rank's
 * sends[i]) issued as ONE NCCL group: one launch and one enqueue wait for the
 * partials of several reductions. Enqueued. */
vc_status vc_cuda_comm_allgather_group(const void* const* sends, void* const* recvs, const size_t* bytes_per_rank,
                                       int count);
/* Wait for the stream with a deadline, watching the communicator for errors. */
vc_status vc_cuda_comm_synchronize(int timeout_ms);
vc_status vc_cuda_comm_destroy(void);
int vc_cuda_comm_size(void);
int vc_cuda_comm_rank(void);

/* ---- failure detection -------------------------------------------------------
 * No counterpart in the reference (its Metal errors arrive through command
 * buffer completion handlers, src/metal/metal_backend.mm:545-549). */

/* Enqueue a one-thread kernel that waits on an mbarrier nothing completes,
 * using the bounded wait of the pipelined kernels limited to `polls` polls
 * (each at most ~2 us): the wait gives up, records the timeout in the device
 * error word and the kernel exits. The next blocking call (vc_cuda_download,
 * vc_cuda_synchronize) then fails with VC_ERR_TIMEOUT and clears the error;
 * the device stays usable. For tests of the failure path. 1 <= polls <= 2^21. */
vc_status vc_cuda_selftest_wait_timeout(long long polls);

/* ---- existing ops (correct, not tuned: off the bandwidth-bound path) ---- */

/* Batched out[z] (m x n) = op(A)[a_offsets[z]..] @ op(B)[b_offsets[z]..];
 * with trans_a A is stored (k x m), with trans_b B is stored (n x k); offsets
 * in elements, host arrays of `batch` entries. Replaces MetalBackend::matmul
 * (metal_backend.hpp:33-37) and cpu::matmul (cpu_backend.cpp:318-366). */
vc_status vc_cuda_matmul(const float* a, const float* b, float* out, size_t m, size_t k, size_t n,
                         const size_t* a_offsets, const size_t* b_offsets, size_t batch,
                         int trans_a, int trans_b);

/* Swap the last two axes of a contiguous [batch, rows, cols] tensor.
 * Replaces MetalBackend::transpose_last2 (metal_backend.hpp:38-39). */
vc_status vc_cuda_transpose_last2(const float* in, float* out, size_t batch, size_t rows, size_t cols);

/* ---- allocation-free sum ---------------------------------------------------- */

/* out[0] = sum of the `count` floats at `in` (device memory): double
 * accumulation in 65536-element chunks, rounded once, so it agrees with
 * vc_cuda_reduce_all(VC_REDUCE_SUM, ...) within double-accumulation rounding
 * (the two split the input differently). For callers that must not allocate
 * device memory: hosts that reserved the device's memory up front under a
 * hard budget, or loops that cannot stall on cudaMalloc / cudaFree. No
 * counterpart in the reference.
 *  - Allocates nothing: its scratch (4096 doubles, 32 KiB) is an array
 *    compiled into this library, held by every GPU that loads it until the
 *    process exits. Call vc_cuda_init first (it creates the stream); any
 *    host thread may then call it -- the call binds the thread to the
 *    library's GPU, as every other entry point does.
 *  - count <= 268435456 (2^28, one partial per 65536 elements); larger
 *    counts fail with VC_ERR_OVERFLOW before anything is launched.
 *  - The first call on a device looks up the array's device address
 *    (cudaGetSymbolAddress, which may load this library's kernels onto the
 *    device); make that first call before any stream capture.
 *  - Every call uses the same array: calls that overlap on the GPU (other
 *    streams, other host threads with their own streams) race. Calls on the
 *    library's one stream are ordered and safe. */
vc_status vc_cuda_reduce_sum_noalloc(const float* in, size_t count, float* out);

#ifdef __cplusplus
}
#endif
#endif /* VC_CUDA_H */
