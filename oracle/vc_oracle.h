/*
 * vc_oracle.h -- CPU restatement of VectorCore's float32 hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This is the parity checker for the CUDA device,
 * never the thing measured or shipped: only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline / reference legs may load it.
 *
 * Parity is pinned: tests/test_oracle.py checks every function here against
 * the reference's own CPU code compiled from its sources (oracle/Makefile ->
 * oracle/_ref/libvcref.so) and against the golden vectors in tests/golden/.
 *
 * Every function is single-threaded and follows the reference's arithmetic
 * step by step (same float roundings, same double accumulators, same
 * accumulation order) so results are bit-identical to the reference except
 * where libm differs (none: both call glibc expf/logf).
 *
 * Shapes are arrays of size_t (the reference's Shape = vector<size_t>);
 * tensors are contiguous row-major float32.
 */
#ifndef VC_ORACLE_H
#define VC_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Operation codes: same order as vectorcore::cpu::BinaryOp / UnaryOp /
 * ReduceOp (include/vectorcore/cpu_backend.hpp:9-11). */
enum { VCO_ADD = 0, VCO_SUB = 1, VCO_MUL = 2, VCO_DIV = 3 };
enum { VCO_NEG = 0, VCO_RELU = 1, VCO_SIGMOID = 2, VCO_RELU_GRAD = 3, VCO_EXP = 4, VCO_LOG = 5 };
enum { VCO_SUM = 0, VCO_MAX = 1, VCO_ARGMAX = 2 };

/* 0 on success, -1 on an invalid argument (message in vco_last_error()). */
const char* vco_last_error(void);

/* src/shape.cpp:34-47 (broadcast_shape). Writes rank max(a_rank,b_rank). */
int vco_broadcast_shape(const size_t* a, int a_rank, const size_t* b, int b_rank,
                        size_t* out, int* out_rank);

/* src/cpu/cpu_backend.cpp:29-106 (binary_kernel), element for element. */
int vco_binary(int op, const float* a, const size_t* a_shape, int a_rank,
               const float* b, const size_t* b_shape, int b_rank,
               float* out, const size_t* out_shape, int out_rank);

/* src/cpu/cpu_backend.cpp:291-316 (unary). */
void vco_unary(int op, const float* in, float* out, size_t n);

/* src/cpu/cpu_backend.cpp:392-418 (sum): 65536-element chunks, four
 * interleaved double accumulators, chunks combined in order. */
float vco_sum(const float* in, size_t n);

/* src/cpu/cpu_backend.cpp:420-460 (reduce_axis). Argmax writes float
 * indices; idx64 (optional) also receives them as int64. */
int vco_reduce_axis(int op, const float* in, float* out, int64_t* idx64,
                    size_t outer, size_t length, size_t inner);

/* src/cpu/cpu_backend.cpp:462-471 (scatter_axis). */
void vco_scatter_axis(const float* values, const float* indices, float* out,
                      size_t outer, size_t length, size_t inner);

/* src/autograd.cpp:50-72 (sum_to_shape): one sum(axis, keepdim) pass per
 * broadcast axis in ascending order, each rounded to float. */
int vco_sum_to_shape(const float* g, const size_t* g_shape, int g_rank,
                     float* out, const size_t* t_shape, int t_rank);

/* src/autograd.cpp:74-91 (broadcast_to): value + scalar 0 into t_shape. */
int vco_broadcast_to(const float* v, const size_t* v_shape, int v_rank,
                     float* out, const size_t* t_shape, int t_rank);

/* Backward rules of src/ops.cpp:98-156 for out = a (op) b with upstream g
 * (out-shaped). da / db may be NULL to skip. */
int vco_binary_backward(int op, const float* a, const size_t* a_shape, int a_rank,
                        const float* b, const size_t* b_shape, int b_rank,
                        const float* g, float* da, float* db);

/* Backward rules of src/ops.cpp:158-164, 360-376, 395-413:
 * x = forward input, y = forward output. */
void vco_unary_backward(int op, const float* x, const float* y, const float* g,
                        float* dx, size_t n);

/* src/ops.cpp:378-388: log_softmax / softmax along the middle axis of a
 * contiguous [outer, length, inner] view. row_max / row_sum (optional,
 * [outer*inner]) receive the detached max and the float sum of exp. */
void vco_log_softmax(const float* x, float* out, float* row_max, float* row_sum,
                     size_t outer, size_t length, size_t inner);
void vco_softmax(const float* x, float* out, size_t outer, size_t length, size_t inner);

/* The reference's autograd chain for log_softmax / softmax with upstream g
 * (engine order of src/tensor.cpp:251-301). */
void vco_log_softmax_backward(const float* x, const float* g, float* dx,
                              size_t outer, size_t length, size_t inner);
void vco_softmax_backward(const float* x, const float* g, float* dx,
                          size_t outer, size_t length, size_t inner);

/* src/nn.cpp:31-53 cross_entropy forward (returns the loss) and, when dx is
 * not NULL, the backward for upstream gradient `upstream`. -1 on invalid
 * targets (loss written to *loss). */
int vco_cross_entropy(const float* logits, size_t batch, size_t classes,
                      const int64_t* targets, float upstream, float* loss, float* dx);

/* Reductions with their backward rules (src/ops.cpp:288-358, 390-393):
 * kind 0 sum, 1 mean, 2 max; axis < 0 with full != 0 reduces everything.
 * out has the reduced shape; dx (optional) receives the gradient for the
 * upstream g (same element count as out). */
int vco_reduce_op(int kind, const float* x, const size_t* shape, int rank, int full,
                  long axis, float* out, const float* g, float* dx);

#ifdef __cplusplus
}
#endif
#endif
