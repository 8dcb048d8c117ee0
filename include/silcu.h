/* silcu.h -- the C ABI of the B200 backend for silarray's sil:: arrays.
 *
 * This is the drop-in boundary: it replaces silarray's `class gpu` static
 * functions (include/gpu.h:266-1036 of the reference), which array.h calls
 * with `storage` handles ({buffer, off, len} in elements) and uint32 shapes.
 * Here a storage handle becomes a plain device pointer already advanced by
 * `off` plus its element count `len`.  Every entry point
 *   - takes an explicit CUDA stream (NULL = the legacy default stream),
 *   - returns a silcu_status and never throws or aborts,
 *   - launches asynchronously and allocates nothing: outputs are
 *     preallocated by the caller, and scratch for multi-pass kernels comes
 *     from a caller-provided workspace sized by the matching *_workspace_bytes.
 * All pointers are device pointers unless the parameter name ends in _host.
 * The library is not thread-safe per stream (neither is the reference).
 */
#ifndef SILCU_H_
#define SILCU_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum silcu_status {
  SILCU_OK = 0,
  SILCU_INVALID_ARGUMENT = 1, /* bad shape / null pointer / misaligned      */
  SILCU_CUDA_ERROR = 2,       /* a CUDA call or launch failed               */
  SILCU_TIMEOUT = 3,          /* a bounded device-side wait gave up         */
  SILCU_WORKSPACE_TOO_SMALL = 4,
  SILCU_UNSUPPORTED = 5
} silcu_status;

typedef struct CUstream_st *silcu_stream; /* == cudaStream_t */

/* Message for the last non-OK status returned on this host thread. */
const char *silcu_last_error(void);
/* ABI version, bumped on any signature change. */
int silcu_abi_version(void);
/* Number of kernels this library has launched in this process (all devices). */
unsigned long long silcu_kernel_launches(void);
/* Blocks until `stream` is idle; replaces synchronize() (include/gpu.h:1375-1377)
 * and gpu_context::flush() (include/gpu.h:107-123). */
silcu_status silcu_synchronize(silcu_stream stream);
/* Reads and clears the device-side error word that bounded waits set
 * (SILCU_TIMEOUT when a wait gave up since the last call). */
silcu_status silcu_device_status(silcu_stream stream);

/* No counterpart in the reference: exercises the failure path of the bounded
 * device waits.  One CTA waits on a barrier that nothing arrives at, through
 * the same wait as the tensor-core kernels but with a limit of `limit_us`
 * (1..1000000) microseconds; it then records code 77 in the device error
 * word and returns, so the next silcu_device_status() on the stream reports
 * SILCU_TIMEOUT (and clears it) while the context stays usable. */
silcu_status silcu_check_bounded_wait(uint32_t limit_us, silcu_stream stream);

/* ------------------------------------------------------------ elementwise
 * out[i] = a[i % len_a] (op) b[i % len_b] for i < n.  Replaces
 * gpu::add/sub/mul/div/pow<float|int> (include/gpu.h:289-312, kernels
 * gpu_kernels.metal:826-968) with the CPU semantics of include/cpu.h:76-237:
 * IEEE fp32 per operation; int arithmetic wraps mod 2^32, int division
 * truncates, int pow = (int)pow(double, double). */
silcu_status silcu_add_f32(const float *a, size_t len_a, const float *b, size_t len_b, float *out, size_t n, silcu_stream stream);
silcu_status silcu_sub_f32(const float *a, size_t len_a, const float *b, size_t len_b, float *out, size_t n, silcu_stream stream);
silcu_status silcu_mul_f32(const float *a, size_t len_a, const float *b, size_t len_b, float *out, size_t n, silcu_stream stream);
silcu_status silcu_div_f32(const float *a, size_t len_a, const float *b, size_t len_b, float *out, size_t n, silcu_stream stream);
silcu_status silcu_pow_f32(const float *a, size_t len_a, const float *b, size_t len_b, float *out, size_t n, silcu_stream stream);
silcu_status silcu_add_i32(const int32_t *a, size_t len_a, const int32_t *b, size_t len_b, int32_t *out, size_t n, silcu_stream stream);
silcu_status silcu_sub_i32(const int32_t *a, size_t len_a, const int32_t *b, size_t len_b, int32_t *out, size_t n, silcu_stream stream);
silcu_status silcu_mul_i32(const int32_t *a, size_t len_a, const int32_t *b, size_t len_b, int32_t *out, size_t n, silcu_stream stream);
silcu_status silcu_div_i32(const int32_t *a, size_t len_a, const int32_t *b, size_t len_b, int32_t *out, size_t n, silcu_stream stream);
silcu_status silcu_pow_i32(const int32_t *a, size_t len_a, const int32_t *b, size_t len_b, int32_t *out, size_t n, silcu_stream stream);

/* gpu::sigmoid / gpu::relu (include/gpu.h:314-320). */
silcu_status silcu_sigmoid_f32(const float *in, float *out, size_t n, silcu_stream stream);
silcu_status silcu_relu_f32(const float *in, float *out, size_t n, silcu_stream stream);
/* gpu::sigmoid_backward (include/gpu.h:945-962): out = dout * s * (1 - s), s = sigmoid(x). */
silcu_status silcu_sigmoid_backward_f32(const float *dout, const float *x, float *out, size_t n, silcu_stream stream);
/* gpu::bias_sigmoid (include/gpu.h:965-982): data[i] = sigmoid(data[i] + bias[i % cols]), in place. */
silcu_status silcu_bias_sigmoid_f32(float *data, const float *bias, size_t n, size_t cols, silcu_stream stream);
/* gpu::affine (include/gpu.h:985-1004): out = in * scale + offset.  `fused`
 * selects one rounding (fmaf, the reference's NEON path for n >= 5e6) or
 * two (multiply then add, its vDSP path), see include/array.h:2003-2015. */
silcu_status silcu_affine_f32(const float *in, float *out, size_t n, float scale, float offset, int fused, silcu_stream stream);

/* Fused elementwise program: one kernel evaluates a chain of lazy-graph
 * nodes (the reference launches one kernel per node, include/array.h:2036-2050).
 * Each instruction writes register `dst` (0..7); operands are registers.
 * Inputs are read with storage-length broadcasting: value i of input j is
 * inputs[j][i % lens[j]].  Every instruction rounds like the reference's
 * per-node evaluation, so results equal a node-by-node evaluation bit for
 * bit (except sigmoid/pow/exp, which round like CUDA's expf/powf). */
typedef enum silcu_opcode {
  SILCU_OP_LOAD = 0,    /* r[dst] = input[a][i % len]                     */
  SILCU_OP_ADD = 1,     /* r[dst] = r[a] + r[b]                           */
  SILCU_OP_SUB = 2,
  SILCU_OP_MUL = 3,
  SILCU_OP_DIV = 4,
  SILCU_OP_POW = 5,
  SILCU_OP_AFFINE = 6,  /* r[dst] = r[a] * imm0 + imm1, two roundings       */
  SILCU_OP_AFFINE_FMA = 7, /* r[dst] = fmaf(r[a], imm0, imm1)             */
  SILCU_OP_SIGMOID = 8,
  SILCU_OP_RELU = 9,
  SILCU_OP_SIGMOID_BWD = 10, /* r[dst] = r[a] * s * (1 - s), s = sigmoid(r[b]) */
  SILCU_OP_RDIV_IMM = 11,   /* r[dst] = imm0 / r[a]                         */
  SILCU_OP_STORE = 12       /* outputs[b][i] = r[a] (silcu_fused_multi_f32 only) */
} silcu_opcode;

typedef struct silcu_instr {
  int32_t op, dst, a, b;
  float imm0, imm1;
} silcu_instr;

#define SILCU_MAX_PROGRAM 32
#define SILCU_MAX_INPUTS 8
typedef struct silcu_program {
  int32_t n_instr;  /* <= SILCU_MAX_PROGRAM; the last instruction's dst is stored */
  int32_t n_inputs; /* <= SILCU_MAX_INPUTS */
  silcu_instr code[SILCU_MAX_PROGRAM];
} silcu_program;

/* `prog_host` is read on the host at call time (passed by value to the kernel). */
silcu_status silcu_fused_f32(const silcu_program *prog_host, const float *const *inputs_host,
                             const size_t *lens_host, float *out, size_t n, silcu_stream stream);
/* The same interpreter with several outputs of n elements each: STORE
 * instructions write a register to outputs[b], and nothing is stored
 * implicitly.  The host layer's chain fusion uses it to write only the nodes
 * of a chain whose storage is still referenced (include/array.h:1987-2061
 * writes every node). */
#define SILCU_MAX_OUTPUTS 4
silcu_status silcu_fused_multi_f32(const silcu_program *prog_host, const float *const *inputs_host,
                                   const size_t *lens_host, float *const *outputs_host, int n_outputs, size_t n,
                                   silcu_stream stream);

/* ------------------------------------------------------------ reductions
 * Whole-array reductions, single pass over HBM plus a one-block finish.
 * Replace gpu::sum_f32 / min_f32 / max_f32 (include/gpu.h:323-470, which
 * leave <= 256 partials for the host) with an on-device result: `out` is one
 * device scalar.  sum: up to 4096 elements it adds sequentially in fp32 in
 * index order (bit-identical to the reference's CPU sum); beyond, it
 * accumulates in fp64 and rounds once.
 * argmax_all writes the first index of the maximum as int64 with the CPU
 * quirk of include/array.h:1733-1740 (values <= FLT_MIN never win; 0 if none). */
size_t silcu_reduce_workspace_bytes(size_t n);
silcu_status silcu_sum_f32(const float *in, size_t n, float *out, void *workspace, size_t workspace_bytes, silcu_stream stream);
/* Same result as silcu_sum_f32, but takes no workspace and allocates nothing.
 * No counterpart in the reference: it is for callers that cannot allocate
 * device memory (code running inside an allocator or memory-pool callback, or
 * a plugin whose host forbids cudaMalloc after start-up).  Scratch is a fixed
 * 32 KiB array inside the library (4096 fp64 partials) on every GPU that
 * loads it; the first pass never uses more than 4096 CTAs, so every input
 * size fits.  The first call on a device looks up that array's address (make
 * it before any stream capture); the address is cached for the process and
 * does not survive a cudaDeviceReset.  All calls share the array: calls that
 * overlap on the GPU (different streams, no ordering between them) race. */
silcu_status silcu_sum_f32_noalloc(const float *in, size_t n, float *out, silcu_stream stream);
silcu_status silcu_min_f32(const float *in, size_t n, float *out, void *workspace, size_t workspace_bytes, silcu_stream stream);
silcu_status silcu_max_f32(const float *in, size_t n, float *out, void *workspace, size_t workspace_bytes, silcu_stream stream);
silcu_status silcu_sum_i32(const int32_t *in, size_t n, int32_t *out, void *workspace, size_t workspace_bytes, silcu_stream stream);
silcu_status silcu_argmax_all_f32(const float *in, size_t n, int64_t *out_index, float *out_value,
                                  void *workspace, size_t workspace_bytes, silcu_stream stream);

/* Row-wise ops on a contiguous [rows, cols] fp32 matrix, one CTA per row
 * with the row held on chip (one HBM read, one write).
 * gpu::softmax (include/gpu.h:916-942), gpu::layer_norm (473-501),
 * gpu::argmax_f32 (890-913; first-index ties and the FLT_MIN floor of the
 * CPU branch, include/array.h:1728-1746). */
silcu_status silcu_softmax_f32(const float *in, float *out, size_t rows, size_t cols, silcu_stream stream);
silcu_status silcu_layer_norm_f32(const float *in, float *out, const float *gamma, const float *beta,
                                  size_t rows, size_t cols, float eps, silcu_stream stream);
/* The same two ops writing the exact tf32 split of their result: out_hi =
 * tf32_rna(y), out_lo = y - out_hi (so out_hi + out_lo == y), the operand
 * format of the tensor-core GEMM (silcu_gemm_args.A_hi/A_lo).  No reference
 * counterpart: a fusion of gpu::layer_norm/softmax with the GEMM's split. */
silcu_status silcu_softmax_split_f32(const float *in, float *out_hi, float *out_lo, size_t rows, size_t cols,
                                     silcu_stream stream);
silcu_status silcu_layer_norm_split_f32(const float *in, float *out_hi, float *out_lo, const float *gamma,
                                        const float *beta, size_t rows, size_t cols, float eps, silcu_stream stream);
silcu_status silcu_argmax_f32(const float *in, int32_t *out, size_t rows, size_t cols,
                              void *workspace, size_t workspace_bytes, silcu_stream stream);
size_t silcu_argmax_workspace_bytes(size_t rows, size_t cols);
/* sum over one axis of a contiguous array viewed as [outer, len, inner]:
 * axis = 1 of [rows, cols] is (rows, cols, 1); axis 0 is (1, rows, cols).
 * Replaces gpu::sum_axis0_f32 (include/gpu.h:356-406) and the CPU-only
 * enumerate_position_ path every other axis takes (include/array.h:2303-2317). */
size_t silcu_sum_axis_workspace_bytes(size_t outer, size_t len, size_t inner);
silcu_status silcu_sum_axis_f32(const float *in, float *out, size_t outer, size_t len, size_t inner,
                                void *workspace, size_t workspace_bytes, silcu_stream stream);
/* The same sum in the reference CPU loop's order (include/array.h:2303-2317,
 * the branch silarray's evaluator runs on the host for every axis but 0 of a
 * 2-D array): each output adds its inputs sequentially in fp32 in index order,
 * so the result is bit-identical to the reference; one thread per output, no
 * workspace.  The drop-in host layer routes sum(axis) here. */
silcu_status silcu_sum_axis_seq_f32(const float *in, float *out, size_t outer, size_t len, size_t inner,
                                    silcu_stream stream);

/* ------------------------------------------------------------ GEMM family
 * C[M,N] = act(alpha * op(A) . op(B) + bias[col % bias_len]) (+ residual).
 * A is [M,K] with row stride lda, or when trans_a, stored [K,M] with row
 * stride lda; B is [K,N] (ldb) or, when trans_b, stored [N,K].  C is [M,N]
 * with row stride ldc.  Batched: operand b starts at X + b * stride_X; a
 * second (inner) batch level gives the per-(batch, head) views of attention
 * without copies.  The residual uses C's batch strides.
 * fp32 in, fp32 out; the tensor-core path is 3xTF32 (hi*hi + hi*lo + lo*hi,
 * Ootomo & Yokota 2022), fp32-faithful within sqrt(K) * (1e-6 + 1e-5|c|).
 * Replaces gpu::sgemm (include/gpu.h:509-514), sgemm_batched /
 * sgemm_steel_batched (518-535), sgemm_steel (577-581), sgemm_bias_steel
 * (584-590), sgemm_bias_sigmoid_steel (609-615) and the MPS transposed
 * dot_f32_ex (1296-1328). */
typedef enum silcu_act { SILCU_ACT_NONE = 0, SILCU_ACT_RELU = 1, SILCU_ACT_SIGMOID = 2 } silcu_act;
typedef enum silcu_gemm_algo {
  SILCU_GEMM_AUTO = 0,   /* tensor cores when the shape pays, else CUDA cores */
  SILCU_GEMM_FFMA = 1,   /* CUDA-core fp32 FFMA (the accuracy reference)       */
  SILCU_GEMM_TC3XTF32 = 2 /* tcgen05 3xTF32                                    */
} silcu_gemm_algo;

typedef struct silcu_gemm_args {
  const float *A, *B;
  float *C;
  int64_t M, N, K;
  int64_t lda, ldb, ldc;
  int32_t trans_a, trans_b;
  int64_t batch;          /* outer batch count (>= 1)                        */
  int64_t stride_a, stride_b, stride_c;
  int64_t batch_inner;    /* inner batch count, 0 or 1 = none: operand (i, j) */
  int64_t stride_a_inner, stride_b_inner, stride_c_inner; /* starts at X + i*stride_X + j*stride_X_inner */
  float alpha;            /* 1 for a plain dot */
  const float *bias;      /* NULL for none */
  int64_t bias_len;       /* bias[col % bias_len] */
  int32_t act;            /* silcu_act, applied after bias */
  const float *residual;  /* NULL, or C += residual[row * ldr + col] after act */
  int64_t ldr;
  int32_t algo;           /* silcu_gemm_algo */
  /* Optional operands held as an exact tf32 split (x = hi + lo, hi =
   * tf32_rna(x)), the format the tensor-core path consumes.  A_hi/A_lo: A in
   * its normal [M,K] layout (lda, A's batch strides; trans_a must be 0).
   * B_hi/B_lo: B with trans_b = 1 ([N,K], ldb) is read directly; with
   * trans_b = 0 it is re-split internally.  C_hi/C_lo: also (or only, if C
   * is NULL) write the split of the result, in C's layout (ldc, strides).
   * Split arrays need 16-byte aligned rows and batch strides; they select
   * the tensor-core path. */
  const float *A_hi, *A_lo, *B_hi, *B_lo;
  float *C_hi, *C_lo;
  /* Tensor-core path: k values accumulated in one TMEM chunk before the
   * epilogue adds the chunk into fp32 registers with round-to-nearest (the
   * tensor core truncates as it accumulates).  0 = 128, the default that
   * keeps general inputs (e.g. U[-1,1) at K = 8192) within the dot
   * tolerance; a caller whose operand scales leave a wide margin (weights of
   * ~0.02) may trade some of it for speed with longer chunks (a multiple of
   * 16; the epilogue then stalls the MMAs less often). */
  int32_t acc_chunk_k;
} silcu_gemm_args;

/* gpu::conv2d (include/gpu.h:815-833; array::conv2d, include/array.h:1508-1519,
 * 2259-2273): input NHWC [N, H, W, C_in], weight OHWI [C_out, K, K, C_in],
 * stride 1, zero padding K / 2, output NHWC [N, H, W, C_out], no bias.  An
 * implicit GEMM (M = N*H*W, N = C_out, K = K*K*C_in) on the 3xTF32 tensor-core
 * path: one pass writes the split patch matrix into the workspace. */
size_t silcu_conv2d_workspace_bytes(uint32_t N, uint32_t H, uint32_t W, uint32_t C_in, uint32_t K, uint32_t C_out);
silcu_status silcu_conv2d_f32(const float *input, const float *weight, float *output, uint32_t N, uint32_t H,
                              uint32_t W, uint32_t C_in, uint32_t K, uint32_t C_out, void *workspace,
                              size_t workspace_bytes, silcu_stream stream);

/* Exact tf32 split of a [rows, cols] fp32 matrix (row stride ld) into
 * contiguous hi/lo arrays, [rows, cols] or, when transpose, [cols, rows] --
 * how a constant weight W[K,N] is turned once into the K-major B_hi/B_lo
 * (trans_b = 1) operand of silcu_sgemm_ex.  No reference counterpart. */
silcu_status silcu_split_f32(const float *src, size_t rows, size_t cols, size_t ld, int transpose, float *hi,
                             float *lo, silcu_stream stream);

/* Batched transposing split: block (b, h) of the source, a [rows, cols]
 * matrix at src + b*s_b + h*s_h with row stride ld, becomes the contiguous
 * [cols, rows] block b*heads + h of hi/lo.  When src_lo is given the source is
 * itself a split pair (value = src + src_lo, exact).  Used to turn V [S, D]
 * into the K-major V^T operand of silcu_attention_f32.  No reference counterpart. */
silcu_status silcu_transpose_split_f32(const float *src, const float *src_lo, size_t rows, size_t cols, size_t ld,
                                       size_t batch, size_t heads, size_t s_b, size_t s_h, float *hi, float *lo,
                                       silcu_stream stream);

/* ------------------------------------------------------------ attention
 * O = softmax(fl(Q . K^T * scale)) . V per (batch, head), fused in one
 * kernel: the score matrix never reaches HBM.  The reference computes this
 * chain node by node (Q.dot(K.transpose()) * scale, softmax, .dot(V):
 * gpu::dot_f32_ex, gpu::affine, gpu::softmax, gpu::sgemm_steel of
 * include/gpu.h:1296-1328, 985-1004, 916-942, 577-581); both products here
 * are 3xTF32 and the softmax is the streaming form over key blocks, equal to
 * the node-by-node result within fp32 rounding.  Operands are exact tf32
 * splits (hi/lo): Q [Sq, D] rows, K [Sk, D] rows, V^T [D, Sk] rows, each at
 * X + b*s_b + h*s_h with its row stride.  D = 64.  Outputs: O [Sq, D] fp32
 * and/or its split.  16-byte aligned rows and strides. */
typedef struct silcu_attention_args {
  const float *Q_hi, *Q_lo, *K_hi, *K_lo, *Vt_hi, *Vt_lo;
  float *O, *O_hi, *O_lo;
  int64_t Sq, Sk, D, batch, heads;
  int64_t ldq, sq_b, sq_h;
  int64_t ldk, sk_b, sk_h;
  int64_t ldv, sv_b, sv_h;
  int64_t ldo, so_b, so_h;
  float scale;
  /* Alternatively V itself, [Sk, D] rows (split hi/lo), e.g. the V columns of
   * a fused QKV projection read in place: set V_hi/V_lo and leave Vt_hi/Vt_lo
   * NULL; ldv, sv_b, sv_h then describe V's rows.  (ABI version 2.) */
  const float *V_hi, *V_lo;
} silcu_attention_args;
silcu_status silcu_attention_f32(const silcu_attention_args *args_host, silcu_stream stream);

/* The same with a workspace: when the (batch, head, query tile) units leave
 * the last wave of SMs mostly idle and the key axis is long enough, each
 * unit's key blocks are split into up to 4 contiguous ranges computed by
 * separate CTAs and combined (m, l rescaling) in a second pass.  The
 * workspace size depends on the shape only (0 when no split is taken);
 * with a smaller workspace the call runs unsplit. */
size_t silcu_attention_workspace_bytes(const silcu_attention_args *args_host);
silcu_status silcu_attention_ex(const silcu_attention_args *args_host, void *workspace, size_t workspace_bytes,
                                silcu_stream stream);

/* The general GEMM of the reference's dot / linear / linear_sigmoid /
 * batched_dot nodes.  The workspace (size from silcu_sgemm_workspace_bytes,
 * 0 when none is needed) holds the tf32 splits of operands given plain and,
 * when output tiles that would leave SMs idle (few tiles, or a partial last
 * wave) are cut into K parts, those tiles' partial sums; results are
 * deterministic (fixed summation order for a given shape and GPU). */
size_t silcu_sgemm_workspace_bytes(const silcu_gemm_args *args_host);
/* How silcu_sgemm_ex runs these arguments (diagnostics and tests: no GPU
 * work, no allocation, no pointer is dereferenced).  path: 0 = CUDA-core FFMA
 * tiles, 1 = GEMV / small-M kernels, 2 = 3xTF32 tensor cores; for path 2 the
 * output-tile width, CTA pairs (256-row tiles), the number of output tiles,
 * how many of them run whole and in how many K parts the others run. */
typedef struct {
  int32_t path, pair, tile_n, ksplit;
  int64_t tiles, whole_tiles;
} silcu_gemm_plan;
silcu_status silcu_sgemm_plan(const silcu_gemm_args *args_host, silcu_gemm_plan *plan);
silcu_status silcu_sgemm_ex(const silcu_gemm_args *args_host, void *workspace, size_t workspace_bytes,
                            silcu_stream stream);
/* Thin forms with the reference's argument lists. */
silcu_status silcu_sgemm(const float *A, const float *B, float *C, uint32_t M, uint32_t N, uint32_t K,
                         uint32_t lda, uint32_t ldb, int trans_a, int trans_b,
                         void *workspace, size_t workspace_bytes, silcu_stream stream);
silcu_status silcu_sgemm_batched(const float *A, const float *B, float *C, uint32_t M, uint32_t N,
                                 uint32_t K, uint32_t lda, uint32_t ldb, uint32_t batch,
                                 uint64_t stride_a, uint64_t stride_b, uint64_t stride_c,
                                 void *workspace, size_t workspace_bytes, silcu_stream stream);
silcu_status silcu_sgemm_bias(const float *A, const float *B, float *C, const float *bias,
                              uint32_t bias_len, uint32_t M, uint32_t N, uint32_t K, uint32_t lda,
                              uint32_t ldb, void *workspace, size_t workspace_bytes, silcu_stream stream);
silcu_status silcu_sgemm_bias_sigmoid(const float *A, const float *B, float *C, const float *bias,
                                      uint32_t bias_len, uint32_t M, uint32_t N, uint32_t K, uint32_t lda,
                                      uint32_t ldb, void *workspace, size_t workspace_bytes,
                                      silcu_stream stream);
/* gpu::sgemv (include/gpu.h:549-574): y[N] = x[K] . W[K,N] (+ bias), K split
 * across the CTAs of a thread-block cluster and combined in a fixed order
 * (a second pass, using the workspace, only for K beyond 8-16 K rows). */
size_t silcu_sgemv_workspace_bytes(uint32_t N, uint32_t K);
silcu_status silcu_sgemv(const float *x, const float *W, float *y, const float *bias, uint32_t N,
                         uint32_t K, void *workspace, size_t workspace_bytes, silcu_stream stream);

#ifdef __cplusplus
}
#endif
#endif /* SILCU_H_ */
