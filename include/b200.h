/*
 * b200.h - C ABI of libb200.so, the B200 (sm_100a) execution backend for
 * ml-switcheroo-compiler fwd+bwd LogicalGraphs.
 *
 * Plain pointers, sizes and a CUDA stream (passed as void*, NULL = legacy default
 * stream); no framework types. All tensors are device pointers into HBM, dense
 * row-major unless a stride argument says otherwise. Every entry point returns an
 * int status (B200_OK = 0); on failure b200_last_error() gives a message for the
 * calling host thread. Kernels are launched asynchronously on `stream`; argument
 * checks happen on the host before any launch.
 *
 * Each entry replaces one kernel of the reference numpy backend, cited as
 * path:line inside src/ml_switcheroo_compiler/ of the reference.
 */
#ifndef B200_H_
#define B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes (mapped to Python exceptions by the host shim) */
#define B200_OK 0
#define B200_ERR_ARG 1        /* bad pointer / size / stride / attribute   -> ValueError            */
#define B200_ERR_DTYPE 2      /* dtype combination without a kernel        -> BackendNotSupportedError */
#define B200_ERR_CUDA 3       /* CUDA launch or runtime error              -> RuntimeError          */
#define B200_ERR_TIMEOUT 4    /* a bounded device-side wait gave up        -> TimeoutError          */
#define B200_ERR_UNSUPPORTED 5 /* shape/layout this build has no kernel for -> UnimplementedMathError */

/* element types */
#define B200_F32 0
#define B200_BF16 1
#define B200_I64 2
#define B200_BOOL 3 /* one byte, 0/1 */
#define B200_I32 4
#define B200_F64 5

int b200_abi_version(void);
const char* b200_last_error(void);
/* number of kernel launches issued by this process so far (all entry points) */
uint64_t b200_launch_count(void);

/* ------------------------------------------------------------------------------
 * Fused elementwise program (subsystem 1).
 *
 * Replaces the numpy per-op elementwise kernels: Add/Subtract/Multiply/TrueDivide
 * (backends/numpy/eager/math_binary.py:9-66), Exp (numpy/eager/math_unary.py:11),
 * Greater/Where (numpy/eager/math_logical.py:26,146), Relu
 * (numpy/eager/activation_ops.py:12), Gelu tanh (eager/core_math_ops/math_nn.py:184-199),
 * Negative/Log/Tanh/Sqrt/Power (np.<name> fallback, numpy/eager/__init__.py:114-125),
 * BroadcastLike/BroadcastTo (eager/core_math_ops/math_reduction.py:227,
 * math_manipulation.py:423), ZerosLike, Transpose materialisation
 * (numpy/eager/array_manipulation.py:121), and a chain of them fused into one pass
 * (the FusedElementwise node of transforms/passes/operator_fusion.py:673-715).
 *
 * A program reads up to B200_EW_MAX_IN inputs, each with its own element strides over
 * the output index space (stride 0 = broadcast), runs up to B200_EW_MAX_INS register
 * instructions per element in fp32, and writes up to B200_EW_MAX_OUT outputs
 * (dense, row-major over `shape`).
 * ----------------------------------------------------------------------------*/
#define B200_EW_MAX_IN 8
#define B200_EW_MAX_OUT 4
#define B200_EW_MAX_DIM 6
#define B200_EW_MAX_INS 48
#define B200_EW_MAX_REG 16

enum b200_ew_op {
  B200_EW_LOAD = 0,   /* r[dst] = in[a][idx]            */
  B200_EW_STORE = 1,  /* out[dst][idx] = r[a]           */
  B200_EW_IMM = 2,    /* r[dst] = imm                   */
  B200_EW_ADD = 3,
  B200_EW_SUB = 4,
  B200_EW_MUL = 5,
  B200_EW_DIV = 6,
  B200_EW_NEG = 7,
  B200_EW_EXP = 8,
  B200_EW_LOG = 9,
  B200_EW_TANH = 10,
  B200_EW_SQRT = 11,
  B200_EW_POW = 12,
  B200_EW_MAX = 13,
  B200_EW_MIN = 14,
  B200_EW_GT = 15,    /* 1.0f / 0.0f                    */
  B200_EW_GE = 16,
  B200_EW_LT = 17,
  B200_EW_EQ = 18,
  B200_EW_WHERE = 19, /* r[dst] = r[a] != 0 ? r[b] : r[c] */
  B200_EW_RELU = 20,  /* max(x, 0)                      */
  B200_EW_GELU = 21,  /* tanh approximation             */
  B200_EW_ABS = 22,
  B200_EW_SIGMOID = 23,
  B200_EW_ERF = 24,
  B200_EW_MOV = 25,
  B200_EW_RECIP = 26,
  B200_EW_FMA = 27    /* r[dst] = r[a] * r[b] + r[c]     */
};

typedef struct b200_ew_ins {
  uint8_t op, dst, a, b, c, pad0, pad1, pad2;
  float imm;
} b200_ew_ins;

typedef struct b200_ew_program {
  int32_t ndim;                                   /* 0..B200_EW_MAX_DIM (0 = scalar)  */
  int32_t n_in, n_out, n_ins;
  int64_t shape[B200_EW_MAX_DIM];                 /* output index space              */
  int64_t in_strides[B200_EW_MAX_IN][B200_EW_MAX_DIM]; /* element strides, 0 = broadcast */
  int32_t in_dtype[B200_EW_MAX_IN];
  int32_t out_dtype[B200_EW_MAX_OUT];
  b200_ew_ins ins[B200_EW_MAX_INS];
} b200_ew_program;

int b200_ew_run(const b200_ew_program* prog, const void* const* inputs, void* const* outputs, void* stream);

/* ------------------------------------------------------------------------------
 * Row reductions (subsystem 2). A tensor is viewed as [outer, red, inner] (dense);
 * the reduced axis is the middle one.
 * ----------------------------------------------------------------------------*/
#define B200_RED_SUM 0
#define B200_RED_MEAN 1
#define B200_RED_MAX 2

/* ReduceSum/ReduceMean/ReduceMax (eager/core_math_ops/math_reduction.py:37,57,97) and
 * BroadcastReduce (math_reduction.py:192-224) as one or more middle-axis passes.
 * x: [outer, red, inner] of in_dtype (F32/BF16), y: [outer, inner] F32. */
int b200_reduce(int in_dtype, const void* x, float* y, int64_t outer, int64_t red, int64_t inner, int op, void* workspace,
                size_t workspace_bytes, void* stream);
/* Scratch for b200_reduce: partial sums when `red` is split across CTAs (combined in a
 * fixed order). With less workspace than this the reduction runs unsplit (same result). */
size_t b200_reduce_workspace_bytes(int64_t outer, int64_t red, int64_t inner);

/* Argmax (numpy/eager/math_reductions.py:129-140): first maximum wins, int64 out. */
int b200_argmax(int in_dtype, const void* x, int64_t* idx, int64_t outer, int64_t red, int64_t inner, void* stream);

/* LayerNorm forward (numpy/eager/nn_ops.py:219-241) and LayerNormInputGrad (nn_ops.py:244)
 * over the last axis, writing fp32 (y / dx) and/or bf16 (y_bf16 / dx_bf16; either may be
 * NULL, not both). Rows of up to 2048 columns are read from HBM once. gamma / beta may be
 * NULL (ones / zeros). */
int b200_layernorm_rows(const float* x, const float* gamma, const float* beta, float* y, void* y_bf16, int64_t rows,
                        int64_t cols, float eps, void* stream);
int b200_layernorm_input_grad_rows(const float* dy, const float* x, const float* gamma, float* dx, void* dx_bf16,
                                   int64_t rows, int64_t cols, float eps, void* stream);

/* The whole LayerNorm backward in one pass over dy and x: LayerNormInputGrad (dx, fp32
 * and/or bf16), LayerNormGammaGrad (dgamma = sum_rows dy * xhat) and LayerNormBetaGrad
 * (dbeta = sum_rows dy) of numpy/eager/nn_ops.py:244-318; any output may be NULL. Column
 * sums go through per-CTA partials reduced in a fixed order (deterministic).
 * workspace >= b200_layernorm_bwd_workspace_bytes(rows, cols). */
size_t b200_layernorm_bwd_workspace_bytes(int64_t rows, int64_t cols);
int b200_layernorm_bwd_rows(const float* dy, const float* x, const float* gamma, float* dx, void* dx_bf16, float* dgamma,
                            float* dbeta, int64_t rows, int64_t cols, float eps, void* workspace, size_t workspace_bytes,
                            void* stream);

/* Softmax / LogSoftmax over the last axis (numpy/eager/math_advanced/math_signal.py:450-467,
 * math_advanced/math_log_exp.py:87-104). x, y: [rows, cols] F32. log != 0 -> LogSoftmax. */
int b200_softmax(const float* x, float* y, int64_t rows, int64_t cols, int log, void* stream);

/* LayerNorm forward over the last axis, biased variance (numpy/eager/nn_ops.py:219-241).
 * gamma/beta may be NULL (ones / zeros). */
int b200_layernorm(const float* x, const float* gamma, const float* beta, float* y, int64_t rows, int64_t cols,
                   float eps, void* stream);

/* LayerNormInputGrad (numpy/eager/nn_ops.py:244-273). gamma may be NULL. */
int b200_layernorm_input_grad(const float* dy, const float* x, const float* gamma, float* dx, int64_t rows,
                              int64_t cols, float eps, void* stream);

/* LayerNormGammaGrad / LayerNormBetaGrad (numpy/eager/nn_ops.py:276-318): column sums of
 * dy * x_hat and of dy over all rows, through per-CTA partials added in a fixed order.
 * Either output may be NULL. workspace >= b200_layernorm_param_grad_workspace_bytes. */
size_t b200_layernorm_param_grad_workspace_bytes(int64_t rows, int64_t cols);
int b200_layernorm_param_grad(const float* dy, const float* x, float* dgamma, float* dbeta, int64_t rows,
                              int64_t cols, float eps, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------
 * Indexing
 * ----------------------------------------------------------------------------*/
/* TakeAlongAxis on the last axis (numpy/eager/advanced_indexing.py:163-177):
 * x [rows, cols] F32, idx [rows, k] I64 -> y [rows, k] F32. Out-of-range idx -> ERR_ARG
 * is reported through the device error flag (see b200_check_device_error). */
int b200_take_along_last(const float* x, const int64_t* idx, float* y, int64_t rows, int64_t cols, int64_t k,
                         void* stream);
/* ScatterAdd on the last axis (numpy/eager/advanced_indexing.py:309-326): y = copy(base);
 * y[r, idx[r,j]] = y[r, idx[r,j]] + src[r,j] in order j = 0..k-1 within a row (a repeated
 * index keeps the last write, as put_along_axis does). base may equal NULL (zeros). */
int b200_scatter_add_last(const float* base, const int64_t* idx, const float* src, float* y, int64_t rows,
                          int64_t cols, int64_t k, void* stream);
/* Take along axis 0 (np.take fallback): rows of table [V, D] gathered by ids [n] -> [n, D]. */
int b200_take_rows(int dtype, const void* table, const int64_t* ids, void* y, int64_t n, int64_t V, int64_t D,
                   void* stream);
/* TensorScatterAdd of rows (numpy/eager/math_scatter.py:39-60 with [n,1] indices):
 * y [V, D] (+)= src[n, D] at rows ids[n]; accumulate != 0 keeps y, else y starts at 0. */
int b200_scatter_add_rows(const float* src, const int64_t* ids, float* y, int64_t n, int64_t V, int64_t D,
                          int accumulate, void* workspace, size_t workspace_bytes, void* stream);
/* Scratch for b200_scatter_add_rows: a stable bucketing of the positions by row id, so
 * each output row adds its source rows in position order (deterministic). */
size_t b200_scatter_add_rows_workspace_bytes(int64_t n, int64_t V);

/* device-side error flag (out-of-range index, timed-out wait): returns B200_OK or the
 * recorded code after synchronising `stream`, and clears the flag. */
int b200_check_device_error(void* stream);

/* ------------------------------------------------------------------------------
 * Contractions (subsystem 3)
 * ----------------------------------------------------------------------------*/
#define B200_EPI_NONE 0
#define B200_EPI_RELU 1       /* C = relu(acc + bias)                                    */
#define B200_EPI_GELU 2       /* C = gelu_tanh(acc + bias)                               */

/* Matmul / BatchMatMul (eager/core_math_ops/math_matrix.py:21-64), strided batched:
 *   C[z] = epi(alpha * op(A[z]) @ op(B[z]) + bias)      z = 0..batch-1
 * op(A) is M x K: element (m,k) at A + z*sA + m*rsA + k*csA (element strides, so any
 * transpose is a stride swap); op(B) K x N likewise with rsB/csB. C is row-major with
 * leading dimension ldc (elements) and batch stride sC. bias (F32, length N) may be NULL.
 * aux (optional, same layout as C, BOOL) receives (acc + bias > 0) for a later ReLU-grad.
 * ab_dtype F32 -> exact fp32 CUDA-core path; BF16 -> tcgen05 tensor cores, fp32
 * accumulation in TMEM (requires csA == 1 or rsA == 1, same for B, and 16-byte aligned
 * rows). c_dtype F32 or BF16. */
int b200_gemm(int ab_dtype, int c_dtype, const void* A, const void* B, void* C, int64_t batch, int64_t M,
              int64_t N, int64_t K, int64_t sA, int64_t rsA, int64_t csA, int64_t sB, int64_t rsB, int64_t csB,
              int64_t sC, int64_t ldc, float alpha, const float* bias, int epilogue, void* aux, void* stream);

/* Matmul over a two-level batch on the tcgen05 tensor cores (bf16 operands): batch
 * entry (zo, zi), zo < b_out, zi < b_in, reads A at zo*sA_out + zi*sA_in and B, C likewise
 * (a stride 0 shares that operand along the level). Covers matmuls of permuted views
 * such as attention's [B, H, S, hd] head split (math_matrix.py:21-64) without copies.
 * C2 (optional, bf16, same element offsets as C): receives act(pre) while C receives
 * pre = alpha A.B + bias, for a bias-add whose activation input is also needed (the
 * GELU of a transformer FFN, whose VJP reads the pre-activation). */
int b200_gemm_batched2(int ab_dtype, int c_dtype, const void* A, const void* B, void* C, int64_t b_out, int64_t b_in,
                       int64_t M, int64_t N, int64_t K, int64_t sA_out, int64_t sA_in, int64_t rsA, int64_t csA,
                       int64_t sB_out, int64_t sB_in, int64_t rsB, int64_t csB, int64_t sC_out, int64_t sC_in, int64_t ldc,
                       float alpha, const float* bias, int epilogue, void* aux, void* C2, void* stream);

/* The same bf16 tensor-core matmul with fp32 C = (A.B + bias) + resid: the Add of a residual
 * connection that follows a bias Add (numpy/eager/math_binary.py:9-20 twice), fused into
 * the epilogue and rounded as the two Adds are (the bias sum first). resid (F32) has C's
 * layout (batch strides sC_out / sC_in, leading dimension ldc); bias may be NULL. */
int b200_gemm_batched2_residual(const void* A, const void* B, float* C, int64_t b_out, int64_t b_in, int64_t M, int64_t N,
                                int64_t K, int64_t sA_out, int64_t sA_in, int64_t rsA, int64_t csA, int64_t sB_out,
                                int64_t sB_in, int64_t rsB, int64_t csB, int64_t sC_out, int64_t sC_in, int64_t ldc,
                                const float* bias, const float* resid, void* stream);

/* Conv2D (numpy/eager/conv.py:462-489) and its VJPs Conv2DInputGrad (conv.py:634-697),
 * Conv2DWeightGrad (conv.py:699-764): NCHW activations (F32), OIHW weights (F32),
 * explicit zero padding (pt, pl; bottom/right implied by the output size), stride
 * (sh, sw), groups = dilation = 1. ab_dtype selects the math: F32 exact or BF16 tensor
 * cores (operands rounded to bf16 while staging, fp32 accumulation). */
int b200_conv2d_fwd(int ab_dtype, const float* x, const float* w, float* y, int64_t N, int64_t C, int64_t H,
                    int64_t W, int64_t O, int64_t KH, int64_t KW, int64_t OH, int64_t OW, int64_t sh, int64_t sw,
                    int64_t pt, int64_t pl, void* stream);
int b200_conv2d_dgrad(int ab_dtype, const float* dy, const float* w, float* dx, int64_t N, int64_t C, int64_t H,
                      int64_t W, int64_t O, int64_t KH, int64_t KW, int64_t OH, int64_t OW, int64_t sh, int64_t sw,
                      int64_t pt, int64_t pl, void* stream);
int b200_conv2d_wgrad(int ab_dtype, const float* x, const float* dy, float* dw, int64_t N, int64_t C, int64_t H,
                      int64_t W, int64_t O, int64_t KH, int64_t KW, int64_t OH, int64_t OW, int64_t sh, int64_t sw,
                      int64_t pt, int64_t pl, void* stream);

/* ------------------------------------------------------------------------------
 * Whole-row fused forward + backward (subsystems 1 + 2 in one pass over HBM):
 *   y = Softmax(LayerNorm(Gelu(x * a + b); gamma, beta, eps)), am = Argmax(y, -1)
 *   and, for the upstream gradient cot of y, the VJP graph of that chain:
 *   dx [rows, cols], da = sum_rows(dp * x), db = sum_rows(dp) [cols],
 *   optional dgamma / dbeta (LayerNormGammaGrad / BetaGrad) [cols].
 * Replaces the per-node chain Multiply/Add (numpy/eager/math_binary.py:9-51), Gelu
 * (eager/core_math_ops/math_nn.py:184-199), LayerNorm (numpy/eager/nn_ops.py:219-241),
 * Softmax (numpy/eager/math_advanced/math_signal.py:450-467), Argmax
 * (numpy/eager/math_reductions.py:129-140), LayerNormInputGrad/GammaGrad/BetaGrad
 * (nn_ops.py:244-318) and BroadcastReduce (eager/core_math_ops/math_reduction.py:192-224).
 * x, cot, y, dx: [rows, cols] fp32 dense; a, b, gamma, beta: [cols] fp32 (gamma/beta may
 * be NULL = ones/zeros); am (int64 [rows]), dgamma, dbeta may be NULL. cols <= 16384.
 * `workspace` holds per-CTA column partials (b200_rowfused_workspace_bytes); the column
 * sums are reduced in a fixed order, so results are deterministic. */
size_t b200_rowfused_workspace_bytes(int64_t rows, int64_t cols);
int b200_rowfused_fwd_bwd(const float* x, const float* a, const float* b, const float* gamma, const float* beta,
                          const float* cot, float* y, int64_t* am, float* dx, float* da, float* db, float* dgamma,
                          float* dbeta, int64_t rows, int64_t cols, float eps, void* workspace, size_t workspace_bytes,
                          void* stream);

/* b200_rowfused_fwd_bwd without a workspace argument, for callers that cannot allocate
 * device memory per call: a serving process that reserves its whole HBM budget at
 * start-up and forbids later allocations, or a C/C++ host that links only this library
 * and has no device allocator of its own. No counterpart in the reference: its numpy
 * path has no device memory to manage. The column-partial scratch lives in a static
 * 16 MiB device array inside libb200.so (held by every GPU that loads the library), so
 * sizes whose b200_rowfused_workspace_bytes exceeds 16 MiB are rejected with
 * B200_ERR_ARG (use b200_rowfused_fwd_bwd then). The first call on each device looks up
 * the array's device address (set-up, no allocation); make that first call before any
 * stream capture. Nothing must be zeroed beforehand. Calls that overlap on the GPU share
 * the array and race: serialise them. The cached address does not survive a
 * cudaDeviceReset of that device: do not call this entry point again after one in the
 * same process. Outputs as b200_rowfused_fwd_bwd. */
int b200_rowfused_fwd_bwd_noalloc(const float* x, const float* a, const float* b, const float* gamma, const float* beta,
                                  const float* cot, float* y, int64_t* am, float* dx, float* da, float* db, float* dgamma,
                                  float* dbeta, int64_t rows, int64_t cols, float eps, void* stream);

/* Gather (numpy/eager/indexing.py:312-332: np.take_along_axis(tensor, index, axis=dim))
 * and TakeAlongAxis on any axis (numpy/eager/advanced_indexing.py:163-177): over the
 * output index space `shape` (ndim <= B200_GATHER_MAX_DIM, the broadcast of the tensor's
 * and the indices' shapes outside `axis`), y[i] = x[i with i[axis] replaced by idx[i]].
 * x_strides / idx_strides are element strides per output axis (0 = broadcast); the x
 * entry at `axis` is the stride along the gathered axis of length axis_len. Elements are
 * copied as raw elem_bytes (1, 2, 4 or 8) values, so every dtype keeps its bits. Negative
 * indices count from the end; an index outside [-axis_len, axis_len) sets the device
 * error flag (b200_check_device_error) and writes zero. y is dense row-major. */
#define B200_GATHER_MAX_DIM 8
int b200_gather_axis(int elem_bytes, const void* x, const int64_t* x_strides, const int64_t* idx, const int64_t* idx_strides,
                     void* y, const int64_t* shape, int ndim, int axis, int64_t axis_len, void* stream);

/* Attention score rows with the softmax (or its VJP) in the GEMM epilogue, for rows of
 * N <= 512 columns and K <= 128 (the scores Q.K^T and dO.V^T of multi-head attention):
 *   b200_gemm_softmax_rows:     y  = softmax(scale * A.B) over the last axis
 *   b200_gemm_softmax_bwd_rows: dx = scale * y * (G - rowsum(G * y)),  G = A.B
 * replacing the Matmul (eager/core_math_ops/math_matrix.py:21-64), the Multiply by the
 * scale and the Softmax (numpy/eager/math_advanced/math_signal.py:450-467), or the Softmax
 * VJP chain the AD pass emits (numpy/eager/math_binary.py:9-51,
 * eager/core_math_ops/math_reduction.py:37), without writing G or the scores to HBM.
 * bf16 operands, both K-major (csA = 1, rsB = 1), two batch levels as b200_gemm_batched2;
 * scale a device fp32 scalar (NULL: 1). Outputs y / dx fp32 and / or bf16 (either may be
 * NULL, not both), [b_out, b_in, M, N] with element strides (s_out, s_in, ld); the backward
 * reads y (fp32 or bf16 per y_dtype) with the same strides. B200_ERR_UNSUPPORTED for other
 * layouts or sizes. */
int b200_gemm_softmax_rows(const void* A, const void* B, int64_t b_out, int64_t b_in, int64_t M, int64_t N, int64_t K,
                           int64_t sA_out, int64_t sA_in, int64_t rsA, int64_t csA, int64_t sB_out, int64_t sB_in, int64_t rsB,
                           int64_t csB, const float* scale, float* y, void* y_bf16, int64_t sY_out, int64_t sY_in, int64_t ldy,
                           void* stream);
int b200_gemm_softmax_bwd_rows(const void* A, const void* B, int64_t b_out, int64_t b_in, int64_t M, int64_t N, int64_t K,
                               int64_t sA_out, int64_t sA_in, int64_t rsA, int64_t csA, int64_t sB_out, int64_t sB_in, int64_t rsB,
                               int64_t csB, const float* scale, int y_dtype, const void* y, float* dx, void* dx_bf16,
                               int64_t s_out, int64_t s_in, int64_t ld, void* stream);

/* Element copy between two strided views of one index space `shape` (ndim <=
 * B200_GATHER_MAX_DIM; element strides, src strides may be 0 to broadcast): the value
 * write of the interpreter's IndexPut / SetItem node (interpreter/evaluator.py:488-508,
 * `arr[key] = val` after the Clone of the base), with dst a view of the cloned base.
 * Raw elem_bytes (1, 2, 4 or 8) values. The views must not overlap. */
int b200_copy_strided(int elem_bytes, const void* src, const int64_t* src_strides, void* dst, const int64_t* dst_strides,
                      const int64_t* shape, int ndim, void* stream);

/* OneHot (numpy/eager/math_advanced/math_general.py:710-736): y = eye(depth)[idx] *
 * (on - off) + off, cast to out_dtype (B200_F32, B200_F64, B200_I64, B200_I32, B200_BOOL),
 * laid out [outer, depth, inner] where idx is [outer, inner] (the class axis moved to
 * position `axis` of the indices' shape). The arithmetic matches numpy's: fp32 outputs
 * round (on - off) and off to fp32 and compute in fp32; the others compute in fp64 and
 * then convert (truncation for integers, != 0 for bool). Index rules as b200_gather_axis. */
int b200_one_hot(const int64_t* idx, void* y, int out_dtype, int64_t outer, int64_t depth, int64_t inner, double on_value,
                 double off_value, void* stream);

/* ReLU-with-bias backward in one pass: gp = g * mask (Multiply(cot, Greater(pre, 0)),
 * the Relu VJP of transforms/autodiff_rules/vjp_rules.yaml:25-27 evaluated by
 * numpy/eager/math_binary.py:39-51) and dbias = column sums of gp (BroadcastReduce,
 * eager/core_math_ops/math_reduction.py:192-224). g [rows, cols] fp32, mask [rows, cols]
 * bool bytes; outputs gp as bf16 and/or fp32 (either may be NULL) and colsum [cols] fp32
 * (may be NULL). workspace >= b200_mask_mul_colsum_workspace_bytes(rows, cols). */
size_t b200_mask_mul_colsum_workspace_bytes(int64_t rows, int64_t cols);
int b200_mask_mul_colsum(const float* g, const uint8_t* mask, void* y_bf16, float* y_f32, float* colsum, int64_t rows,
                         int64_t cols, void* workspace, size_t workspace_bytes, void* stream);

/* GELU (tanh approximation) backward with its bias gradient in one pass: the VJP chain
 * the AD pass emits for Gelu (eager/core_math_ops/math_nn.py:184-199 forward; elementwise
 * ops numpy/eager/math_binary.py:9-51 and np.tanh) times the cotangent, and the column
 * sums of the result (BroadcastReduce, eager/core_math_ops/math_reduction.py:192-224):
 *   dp = g * (0.5 (1 + t) + 0.5 p (1 - t^2) k (1 + 3 c p^2)),  t = tanh(k (p + c p^3)).
 * g, p [rows, cols] fp32; dp as bf16 and/or fp32 (either may be NULL), colsum [cols]
 * (may be NULL). workspace >= b200_gelu_bwd_colsum_workspace_bytes(rows, cols). */
size_t b200_gelu_bwd_colsum_workspace_bytes(int64_t rows, int64_t cols);
int b200_gelu_bwd_colsum(const float* g, const float* p, void* y_bf16, float* y_f32, float* colsum, int64_t rows,
                         int64_t cols, void* workspace, size_t workspace_bytes, void* stream);

/* Fused LogSoftmax (numpy/eager/math_advanced/math_log_exp.py:87-104) -> TakeAlongAxis of
 * one label per row (numpy/eager/advanced_indexing.py:163-177) and its VJP (ZerosLike +
 * ScatterAdd advanced_indexing.py:309-326, then the LogSoftmax rule g - exp(ls) sum(g)):
 *   picked[r] = ls[r, label[r]],  dx[r, j] = d[r] ([j == label[r]] - softmax(x)[r, j]).
 * x [rows, cols] (F32 or BF16), label [rows] int64, d [rows] fp32 (cotangent of picked).
 * picked, ls (the full log-softmax), dx and dx_bf16 (dx in bf16, for fp32 x with cols % 4 == 0)
 * may each be NULL. */
int b200_logsoftmax_pick(int x_dtype, const void* x, const int64_t* label, const float* d, float* picked, float* ls,
                         float* dx, void* dx_bf16, int64_t rows, int64_t cols, void* stream);

/* LayerNorm forward (numpy/eager/nn_ops.py:219-241) and LayerNormInputGrad (nn_ops.py:244)
 * over the last axis, writing fp32 (y / dx) and/or bf16 (y_bf16 / dx_bf16; either may be
 * NULL, not both). Rows of up to 2048 columns are read from HBM once. gamma / beta may be
 * NULL (ones / zeros). */
int b200_layernorm_rows(const float* x, const float* gamma, const float* beta, float* y, void* y_bf16, int64_t rows,
                        int64_t cols, float eps, void* stream);
int b200_layernorm_input_grad_rows(const float* dy, const float* x, const float* gamma, float* dx, void* dx_bf16,
                                   int64_t rows, int64_t cols, float eps, void* stream);

/* The whole LayerNorm backward in one pass over dy and x: LayerNormInputGrad (dx, fp32
 * and/or bf16), LayerNormGammaGrad (dgamma = sum_rows dy * xhat) and LayerNormBetaGrad
 * (dbeta = sum_rows dy) of numpy/eager/nn_ops.py:244-318; any output may be NULL. Column
 * sums go through per-CTA partials reduced in a fixed order (deterministic).
 * workspace >= b200_layernorm_bwd_workspace_bytes(rows, cols). */
size_t b200_layernorm_bwd_workspace_bytes(int64_t rows, int64_t cols);
int b200_layernorm_bwd_rows(const float* dy, const float* x, const float* gamma, float* dx, void* dx_bf16, float* dgamma,
                            float* dbeta, int64_t rows, int64_t cols, float eps, void* workspace, size_t workspace_bytes,
                            void* stream);

/* Softmax / LogSoftmax over the last axis (numpy/eager/math_advanced/math_signal.py:450-467,
 * math_advanced/math_log_exp.py:87-104) of t = x * scale[0], where `scale` is an optional
 * device scalar (NULL = 1): the Multiply node that scales attention scores folds in.
 * x [rows, cols] fp32 dense; writes y (fp32) and/or y_bf16 (either may be NULL, not both). */
int b200_softmax_rows(const float* x, const float* scale, float* y, void* y_bf16, int64_t rows, int64_t cols, int log,
                      void* stream);

/* Softmax VJP as the AD pass composes it (Multiply, ReduceSum keepdims, Subtract, Multiply
 * over numpy/eager/math_binary.py:9-51 and core_math_ops/math_reduction.py:37), times an
 * optional device scalar (the VJP of the scaling Multiply):
 *   dx = scale[0] * (y * (g - sum_j g * y)).
 * y, g [rows, cols] fp32 dense; writes dx (fp32) and/or dx_bf16 (either may be NULL). */
int b200_softmax_bwd_rows(const float* y, const float* g, const float* scale, float* dx, void* dx_bf16, int64_t rows,
                          int64_t cols, void* stream);

/* Conv2D / Conv2DInputGrad / Conv2DWeightGrad (numpy/eager/conv.py:462-489, 634-697,
 * 699-764) on the tcgen05 tensor cores: bf16 operands staged in `workspace` (im2col of
 * the activations, packed weights / gradients), fp32 accumulation, fp32 NCHW / OIHW
 * results. Same tensor arguments as the b200_conv2d_* entry points above; op = 0 fwd,
 * 1 dgrad, 2 wgrad for the workspace query. */
size_t b200_conv2d_tc_workspace_bytes(int op, int64_t N, int64_t C, int64_t H, int64_t W, int64_t O, int64_t KH, int64_t KW,
                                      int64_t OH, int64_t OW, int64_t sh, int64_t sw, int64_t pt, int64_t pl);
int b200_conv2d_fwd_tc(const float* x, const float* w, float* y, int64_t N, int64_t C, int64_t H, int64_t W, int64_t O,
                       int64_t KH, int64_t KW, int64_t OH, int64_t OW, int64_t sh, int64_t sw, int64_t pt, int64_t pl,
                       void* workspace, size_t workspace_bytes, void* stream);
int b200_conv2d_dgrad_tc(const float* dy, const float* w, float* dx, int64_t N, int64_t C, int64_t H, int64_t W, int64_t O,
                         int64_t KH, int64_t KW, int64_t OH, int64_t OW, int64_t sh, int64_t sw, int64_t pt, int64_t pl,
                         void* workspace, size_t workspace_bytes, void* stream);
int b200_conv2d_wgrad_tc(const float* x, const float* dy, float* dw, int64_t N, int64_t C, int64_t H, int64_t W, int64_t O,
                         int64_t KH, int64_t KW, int64_t OH, int64_t OW, int64_t sh, int64_t sw, int64_t pt, int64_t pl,
                         void* workspace, size_t workspace_bytes, void* stream);

/* The same three convolutions as implicit GEMMs on the tcgen05 tensor cores (no im2col
 * buffer): bf16 operand tiles built in shared memory, fp32 accumulation, fp32 results in
 * NCHW / OIHW.
 *   b200_conv2d_fwd_igemm:   y = Conv2D(x, w)   (numpy/eager/conv.py:462-489); relu != 0
 *                            writes relu(y) instead (the Relu node that follows, fused)
 *   b200_conv2d_dgrad_igemm: dx = Conv2DInputGrad(dy, w) (conv.py:634-697); a non-null
 *                            mask [N, C, H, W] writes dx * (mask > 0) instead (the Multiply
 *                            by the Greater(pre, 0) mask of the ReLU VJP, fused); a non-null
 *                            mask_cl [N, H, W, mask_cp] bf16 (the channels-last copy that a
 *                            relu != 0 forward wrote as y_cl) writes dx * (mask_cl != 0)
 *   b200_conv2d_wgrad_igemm: dw = Conv2DWeightGrad(x, dy) (conv.py:699-764)
 * `workspace` (256-byte aligned, b200_conv2d_igemm_workspace_bytes(op, ...) bytes, op 0
 * fwd, 1 dgrad, 2 wgrad) holds the bf16 channels-last copies the tiles are copied from
 * (x for fwd, dy for dgrad, both for wgrad) and the weight gradient's per-split partial
 * sums. A caller that already holds such a copy passes it as x_cl / dy_cl (NULL: the
 * call makes it): b200_conv2d_channels_last writes src [N, C, HW] fp32 as [N, HW, Cp]
 * bf16, channels >= C zero; Cp = C rounded up to 8 for x and for dgrad's dy, O rounded up
 * to 64 for wgrad's dy. A non-null y_cl / dx_cl receives the result's own copy in that
 * layout (channels rounded up to 8) from the same epilogue, for the next convolution; y /
 * dx may then be NULL (only the copy is written). With relu != 0 the copy keeps positive
 * values nonzero (values below 2^-133 become the smallest bf16 subnormal instead of +0), so
 * it is nonzero exactly where y > 0.
 * b200_conv2d_igemm_supported(op, ...) is 1 when the shape fits the kernel (tensors up to
 * 2^30 elements, at most 2048 reduction indices with channels padded to 8, the bf16
 * weights resident in shared memory); the entry points return B200_ERR_UNSUPPORTED
 * otherwise. */
int b200_conv2d_igemm_supported(int op, int64_t N, int64_t C, int64_t H, int64_t W, int64_t O, int64_t KH, int64_t KW,
                                int64_t OH, int64_t OW, int64_t sh, int64_t sw, int64_t pt, int64_t pl);
size_t b200_conv2d_igemm_workspace_bytes(int op, int64_t N, int64_t C, int64_t H, int64_t W, int64_t O, int64_t KH, int64_t KW,
                                         int64_t OH, int64_t OW, int64_t sh, int64_t sw, int64_t pt, int64_t pl);
int b200_conv2d_channels_last(const float* src, void* dst, int64_t N, int64_t C, int64_t HW, int64_t Cp, void* stream);
int b200_conv2d_fwd_igemm(const float* x, const void* x_cl, const float* w, float* y, void* y_cl, int64_t N, int64_t C,
                          int64_t H, int64_t W, int64_t O, int64_t KH, int64_t KW, int64_t OH, int64_t OW, int64_t sh,
                          int64_t sw, int64_t pt, int64_t pl, int relu, void* workspace, size_t workspace_bytes,
                          void* stream);
int b200_conv2d_dgrad_igemm(const float* dy, const void* dy_cl, const float* w, const float* mask, const void* mask_cl,
                            int64_t mask_cp, float* dx, void* dx_cl, int64_t N, int64_t C, int64_t H, int64_t W,
                            int64_t O, int64_t KH, int64_t KW, int64_t OH, int64_t OW, int64_t sh, int64_t sw, int64_t pt,
                            int64_t pl, void* workspace, size_t workspace_bytes, void* stream);
int b200_conv2d_wgrad_igemm(const float* x, const void* x_cl, const float* dy, const void* dy_cl, float* dw, int64_t N,
                            int64_t C, int64_t H, int64_t W, int64_t O, int64_t KH, int64_t KW, int64_t OH, int64_t OW,
                            int64_t sh, int64_t sw, int64_t pt, int64_t pl, void* workspace, size_t workspace_bytes,
                            void* stream);


/* All-reduce of n fp32 values across `world` ranks through peer-mapped memory, for the
 * buckets of small gradients that the reference exchanges with its AllReduce node
 * (numpy/eager/distributed.py:205-225, all_reduce_ring :105). One kernel: every value
 * travels with its call number in one 64-bit word (call << 32 | value bits), pushed into
 * every peer's receive area over NVLink; each rank polls its own area (at most spin_limit
 * polls per thread) and adds all ranks' values in rank order, times `scale` (1 for a sum,
 * 1/world for a mean). The result is identical on every rank.
 *   bufs_dev: device array of `world` pointers, rank q's receive area of
 *             2 * world * capacity 64-bit words, zero before the first call
 *   epoch:    this rank's per-block call counters (64 uint32, zero at start); every rank
 *             must make the same calls with the same n
 *   status:   device int, set to B200_ERR_TIMEOUT when a peer's words did not arrive. The
 *             values of that block are left unchanged on this rank, but peers that
 *             received this rank's words did complete the call, so the ranks no longer
 *             agree on call numbers. A timeout is therefore fatal: while status is non-zero
 *             every later call returns at once (no values sent, summed or updated), so the
 *             peers time out too and no rank ever adds a stale word. Re-opening the
 *             exchange needs a collective reset: receive areas cleared, epoch and status
 *             zeroed on every rank. With the optimizer epilogue, parameters may differ
 *             across ranks after a timeout.
 * Every call of one rank must be issued on one stream, in call order (CUDA graph replays
 * included): the double-buffer argument above relies on call e - 2 having finished before
 * call e starts on this rank.
 * n <= capacity and n <= 64 * 4096. b200_peer_allreduce_blocks gives the blocks for n. */
int b200_peer_allreduce_blocks(int64_t n);
int b200_peer_allreduce_f32(float* data, int64_t n, const void* bufs_dev, int64_t capacity, int rank, int world,
                            unsigned int* epoch, int* status, int64_t spin_limit, float scale, void* stream);
/* The same exchange over `count` (<= 64) fp32 tensors laid end to end, without packing
 * them into one buffer: tensors[j] holds values [offsets[j], offsets[j + 1]) and receives
 * their sums in place (offsets[0] = 0, offsets[count] = total <= capacity). kind >= 0 adds
 * the optimizer epilogue of b200_peer_allreduce_apply_f32 on param / s1 / s2; kind -1 is
 * the plain sum. Host arrays of device pointers. */
int b200_peer_allreduce_tensors_f32(int count, const int64_t* offsets, float* const* tensors, const void* bufs_dev,
                                    int64_t capacity, int rank, int world, unsigned int* epoch, int* status, int64_t spin_limit,
                                    float scale, int kind, float* const* param, float* const* s1, float* const* s2, float lr,
                                    void* stream);
/* cudaMemsetAsync of a device range (clears a signal pad before its first use). */
int b200_memset_async(void* p, int value, size_t bytes, void* stream);

/* Optimizer update steps ApplyAdam (kind 0), ApplyAdagrad (1), ApplyFtrl (2), ApplyRMSProp
 * (3), as the reference's numpy backend computes them (numpy/eager/optimizers_ops.py:11-103):
 * its fixed hyperparameters, fp32, one IEEE rounding per operation in the same order, so the
 * results are bit-identical to the reference's. `count` fp32 tensors in one launch per 128:
 * host arrays of device pointers param[i], s1[i], s2[i] (the state arrays: Adam m, v;
 * Adagrad accum, s2 unused and may be NULL; FTRL accum, linear; RMSProp ms, mom), grad[i],
 * and the outputs, which may be the inputs themselves (in-place step); n[i] elements each.
 * b200_optimizer_default_lr gives the numpy kernels' default lr of each kind. */
double b200_optimizer_default_lr(int kind);
int b200_apply_optimizer_f32(int kind, int count, const float* const* param, const float* const* s1, const float* const* s2,
                             const float* const* grad, float* const* param_out, float* const* s1_out, float* const* s2_out,
                             const int64_t* n, float lr, void* stream);

/* b200_peer_allreduce_f32 followed, in the same kernel, by an optimizer step on the summed
 * values (the reference's AllReduce node and then ApplyAdam / ApplyAdagrad / ApplyFtrl /
 * ApplyRMSProp, numpy/eager/distributed.py:205-225 and numpy/eager/optimizers_ops.py:11-103):
 * the n values are the gradients of `count` (<= 64) parameter tensors laid end to end,
 * tensor j covering [offsets[j], offsets[j + 1]) with offsets[0] = 0, offsets[count] = n.
 * Each summed element also updates param[j], s1[j] (and s2[j]; Adagrad has none) in
 * place, bit-identically to b200_apply_optimizer_f32; `data` receives the summed values.
 * offsets, param, s1, s2 are host arrays (device pointers). */
int b200_peer_allreduce_apply_f32(float* data, int64_t n, const void* bufs_dev, int64_t capacity, int rank, int world,
                                  unsigned int* epoch, int* status, int64_t spin_limit, float scale, int kind, int count,
                                  const int64_t* offsets, float* const* param, float* const* s1, float* const* s2, float lr,
                                  void* stream);

#ifdef __cplusplus
}
#endif
#endif /* B200_H_ */
