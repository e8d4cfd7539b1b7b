/*
 * avey_b200.h -- C ABI of the B200 (sm_100a) contextualizer forward library.
 *
 * One call computes, for every batch row b,
 *
 *   out[b] = z_tl[b] * act( (S_b (.) V (.) M_b) z_tr[b] / den_b + bias )
 *
 * with S_b the cosine similarity of the rows of z_tr[b], M_b the causal and
 * padding mask and den_b the signed row sum (Avey-B) or 1 (Avey): the math of
 * the reference's avey_kernels/ops.py:61-91 (_reference).
 *
 * The library is plain C at this boundary: raw device pointers, element
 * strides and sizes, no framework types. It never throws; every entry point
 * returns an AveyStatus and avey_last_error() describes the last failure on
 * the calling thread. Calls only enqueue work on the given stream: they do not
 * synchronise and do not allocate (scratch memory, when a kernel needs it, is
 * passed in by the caller as `workspace`), so they can be captured in a CUDA
 * graph.
 */
#ifndef AVEY_B200_H
#define AVEY_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AVEY_ABI_VERSION 5

#if defined(__GNUC__)
#define AVEY_API __attribute__((visibility("default")))
#else
#define AVEY_API
#endif

/* Element types of z_tr, v, z_tl, bias and out (all share one type). */
typedef enum AveyDtype {
  AVEY_F32 = 0,
  AVEY_F16 = 1,
  AVEY_BF16 = 2,
  AVEY_F64 = 3,
} AveyDtype;

/* Activation ids; the numbering is that of the reference, _triton.py:169. */
typedef enum AveyActivation {
  AVEY_ACT_IDENTITY = 0,
  AVEY_ACT_RELU = 1,
  AVEY_ACT_RELU2 = 2,
  AVEY_ACT_SILU = 3,
  AVEY_ACT_GELU = 4, /* tanh approximation */
} AveyActivation;

/* Kernel selection. AUTO picks the tcgen05 kernels whenever the shape, dtype
 * and alignment allow it, except for small fp32 problems (contexts up to
 * 512, features a multiple of 32 up to 256, a few waves of 8-row query
 * tiles), which finish sooner on an 8-row CUDA-core kernel (AveyPlan.reason
 * 6); else the general CUDA-core kernel. AVEY_KERNEL_SIMT forces the general
 * CUDA-core kernel, AVEY_KERNEL_TCGEN05 the tcgen05 kernels. */
typedef enum AveyKernel {
  AVEY_KERNEL_AUTO = 0,
  AVEY_KERNEL_SIMT = 1,   /* general CUDA-core kernel: any dtype/stride/shape */
  AVEY_KERNEL_TCGEN05 = 2 /* TMA + tcgen05 + TMEM kernels (bf16 / f16): one fused
                             kernel up to 512 tokens, two kernels from 513 to 8192 */
} AveyKernel;

typedef enum AveyStatus {
  AVEY_OK = 0,
  AVEY_ERR_ARGUMENT = -1,    /* bad size, pointer, stride, flag or struct */
  AVEY_ERR_ARCH = -2,        /* current device is not sm_100 */
  AVEY_ERR_UNSUPPORTED = -3, /* a forced kernel cannot run these inputs */
  AVEY_ERR_LAUNCH = -4,      /* the CUDA launch itself failed */
  AVEY_ERR_DEVICE = -5,      /* a kernel reported a timeout or fault flag */
  AVEY_ERR_CUDA = -6,        /* another CUDA runtime / driver call failed */
} AveyStatus;

/*
 * Forward parameters. Strides are in ELEMENTS. The feature (last) dimension
 * of z_tr, z_tl and out must have stride 1; the other strides are free, so the
 * head and tail halves of one [B, C, 2d'] tensor are passed as two views
 * (row stride 2d') without a copy. Optional tensors are NULL when absent.
 * valid holds one byte per (batch, position): nonzero = valid.
 */
typedef struct AveyFwdParams {
  uint32_t struct_size; /* sizeof(AveyFwdParams); guards ABI drift */
  int32_t dtype;        /* AveyDtype */
  int64_t batch;        /* B  >= 1 */
  int64_t context;      /* C  >= 1 (tokens per batch row) */
  int64_t features;     /* d' >= 1 */

  const void* z_tr;     /* [B, C, d'] tail half (required) */
  int64_t z_tr_batch_stride, z_tr_row_stride;
  const void* v;        /* [C, C] indexed [query, key] (Avey) or NULL */
  int64_t v_row_stride;
  const void* z_tl;     /* [B, C, d'] head half, the gate, or NULL */
  int64_t z_tl_batch_stride, z_tl_row_stride;
  const void* bias;     /* [d'] contiguous, or NULL */
  const uint8_t* valid; /* [B, C] bytes, or NULL */
  int64_t valid_batch_stride, valid_row_stride;
  void* out;            /* [B, C, d'] output, same dtype as z_tr */
  int64_t out_batch_stride, out_row_stride;

  double eps;      /* Avey-B denominator epsilon (used when normalize != 0) */
  double norm_eps; /* L2-normalisation epsilon: x / max(||x||, norm_eps) */
  int32_t causal;     /* keep key j <= query i (diagonal kept) */
  int32_t normalize;  /* divide by the signed row sum + eps (Avey-B) */
  int32_t activation; /* AveyActivation */
  int32_t kernel;     /* AveyKernel */
  void* workspace;          /* device scratch, >= avey_fwd_workspace_size() bytes */
  uint64_t workspace_bytes; /* size of `workspace` in bytes */

  /* Prefix form of the padding mask, instead of `valid` (passing both is an
   * error): a device array of B int32 lengths, positions [0, lengths[b]) of
   * batch row b are valid and the rest is padding (values above the context
   * act as the context, values below 1 leave the row all padding). No mask
   * bytes are read. The reference takes only the byte mask (ops.py:23-46);
   * this is the C-ABI fast path for callers that hold lengths. */
  const int32_t* lengths;
} AveyFwdParams;

/* What avey_fwd_v1 would launch for these parameters. */
typedef struct AveyPlan {
  int32_t kernel;        /* AVEY_KERNEL_SIMT or AVEY_KERNEL_TCGEN05 */
  int32_t launches;      /* kernel launches per call: 1 on the tcgen05 path up to
                            512 tokens (the fused kernel), 3 above (row-sum pre-pass,
                            G/P kernel, O = P Z kernel), 2 for fp32 on the 3xTF32
                            pair, 1 on CUDA cores */
  int32_t grid;          /* CTAs of the main launch */
  int32_t block;         /* threads per CTA of the main launch */
  int32_t smem_bytes;    /* dynamic shared memory per CTA */
  int32_t reason;        /* 0, or why the tcgen05 kernel was not chosen: 1 dtype,
                            2 context, 3 alignment, 4 AVEY_KERNEL_SIMT asked for,
                            5 features, 6 small fp32 problem (AUTO runs the 8-row
                            CUDA-core kernel, which finishes first there) */
} AveyPlan;

/*
 * Run the contextualizer forward on `stream` (a cudaStream_t; NULL is the
 * legacy default stream). Replaces, in the reference, the normalisation
 * pre-pass plus the fused mixing launch: avey_kernels/ops.py:107-114
 * (F.normalize into a temporary fp32 buffer, then mix) and
 * avey_kernels/_triton.py:153-188 (the avey_kernels::mix custom op that
 * launches _mix_kernel). Normalisation is fused into the kernel here.
 * Returns AVEY_OK or a negative AveyStatus.
 */
AVEY_API int avey_fwd_v1(const AveyFwdParams* params, void* stream);

/* Fill *plan with the launch avey_fwd_v1 would make; launches nothing.
 * Has no reference counterpart (introspection for tests and benchmarks). */
AVEY_API int avey_fwd_plan(const AveyFwdParams* params, AveyPlan* plan);

/* Device workspace avey_fwd_v1 needs for these parameters, in bytes: 0 for the
 * CUDA-core kernels and for the fused tcgen05 kernel (up to 512 tokens: it
 * sums the rows' squares from the tiles it stages); above 512 tokens and for
 * fp32 on the 3xTF32 pair, in 256-byte aligned parts, the row sums of squares
 * (4 bytes per row of z_tr), 4 bytes per row per group of 256 keys (partial
 * row sums) and P itself (2 bytes per (query, key) pair, 4 for fp32, rows
 * padded to 64 keys): 134 MB for batch 16 x 2048 tokens. The workspace must
 * be 256-byte aligned. The reference allocates its normalisation buffer
 * itself (ops.py:108); this library leaves allocation to the caller.
 * Launches nothing. */
AVEY_API int avey_fwd_workspace_size(const AveyFwdParams* params, uint64_t* bytes);

/*
 * avey_fwd_v1 for callers that cannot allocate device memory: no counterpart
 * in the reference. Some callers hold no device allocator of their own -- an
 * FFI host (cgo, JNI, a plugin ABI) that only passes raw pointers in, or code
 * that runs while a stream is being captured into a CUDA graph, where
 * allocation is not allowed -- so they cannot provide `workspace`. This entry
 * point ignores params->workspace and uses a scratch array that lives inside
 * the library instead (file-scope device memory, present on every GPU that
 * loads the library until the process exits). It allocates nothing.
 *
 * Contexts above 512 tokens run the CUDA-core kernel here (the tcgen05 path
 * for them needs a P workspace); forcing AVEY_KERNEL_TCGEN05 for them fails
 * with AVEY_ERR_UNSUPPORTED.
 *
 * On the fused tensor-core path (bf16 / f16 up to 512 tokens) this entry point
 * runs the kernel's pre-pass variant: a row-norm pre-pass writes each row's
 * sum of squares into the array and the fused kernel reads them, where
 * avey_fwd_v1 has the fused kernel sum the rows itself; the two agree to
 * the rounding of those sums.
 *
 * Limit: on the fused tensor-core path (the only path that reads the
 * scratch) batch * context <= AVEY_NOALLOC_MAX_ROWS
 * (1,048,576 rows; the array holds one float per row, 4 MiB per GPU); larger
 * inputs are rejected with AVEY_ERR_ARGUMENT. Inputs that run a CUDA-core
 * kernel use no scratch and have no such limit. The first call on each device
 * looks up the array's
 * device address (with that device current); make that first call before
 * any stream capture. All calls share the one array, so calls whose kernels
 * overlap on the GPU (for example on two streams) race; each call rewrites
 * every row it reads, so nothing needs clearing between calls.
 */
#define AVEY_NOALLOC_MAX_ROWS (1u << 20)
AVEY_API int avey_fwd_noalloc_v1(const AveyFwdParams* params, void* stream);

/*
 * Backward pass. The reference has no fused backward: autograd runs through
 * its PyTorch path (avey_kernels/ops.py:94-106 send any input that requires
 * grad to _reference, ops.py:61-91). This library splits the gradient into
 * five batched GEMMs, which the caller runs with a library GEMM, and five
 * fused steps that run here between them:
 *
 *   AVEY_BWD_PREP      zm = z_tr (padded rows 0), norms = ||zm|| (-1: padding)
 *                                                          then  g = zm zm^T
 *   AVEY_BWD_SCORES    s = g r_i r_j (.) v (.) mask, den = rowsum(s) + eps,
 *                      r = 1 / max(norms, norm_eps)        then  num = s zm
 *   AVEY_BWD_EPILOGUE  grad_z_tl, grad_bias, dnum, dden from grad_out
 *                                        then  ds0 = dnum zm^T, dzd = s^T dnum
 *   AVEY_BWD_DSCORES   dgsym = (dG + dG^T) diag(r), dG = (ds0 + dden) (.)
 *                      mask (.) v; grad_v                  then  dzh = dgsym zm
 *   AVEY_BWD_FINAL     grad_z_tr = dzd + normalisation backward of dzh
 *
 * GEMM operands (zm, s, dnum, dgsym) are of gemm_dtype: AVEY_BF16 for
 * bf16 inputs, AVEY_F32 for f16 and f32 inputs, AVEY_F64 for f64 inputs.
 * Accumulator arrays (norms, g, den, num, dden, ds0, dzd, dzh, workspace) are
 * float, or double for f64 inputs; GEMM outputs are written in that type. All
 * scratch arrays are contiguous ([B, C, d'], [B, C, C] or [B, C]); the
 * gradients are of the input dtype, and an output pointer left NULL is not
 * computed (grad_v needs v, grad_z_tl needs z_tl). Reductions use
 * fixed orders: results are bitwise reproducible.
 */
typedef enum AveyBwdStep {
  AVEY_BWD_PREP = 0,
  AVEY_BWD_SCORES = 1,
  AVEY_BWD_EPILOGUE = 2,
  AVEY_BWD_DSCORES = 3,
  AVEY_BWD_FINAL = 4,
} AveyBwdStep;

typedef struct AveyBwdParams {
  uint32_t struct_size; /* sizeof(AveyBwdParams) */
  int32_t dtype;        /* AveyDtype of the inputs and gradients */
  int32_t gemm_dtype;   /* AveyDtype of the GEMM operand arrays (see above) */
  int32_t causal, normalize, activation;
  int64_t batch, context, features;
  double eps, norm_eps;

  /* Forward inputs, strided as in AveyFwdParams. */
  const void* z_tr;
  int64_t z_tr_batch_stride, z_tr_row_stride;
  const void* v;
  int64_t v_row_stride;
  const void* z_tl;
  int64_t z_tl_batch_stride, z_tl_row_stride;
  const void* bias;
  const uint8_t* valid;
  int64_t valid_batch_stride, valid_row_stride;
  const void* grad_out; /* [B, C, d'] gradient of the forward output */
  int64_t grad_out_batch_stride, grad_out_row_stride;

  /* Scratch written by one step and read by later ones or by the GEMMs. */
  void* zm;        /* [B, C, d'] gemm_dtype; may be NULL when valid is NULL and
                      gemm_dtype == dtype (zm would equal z_tr): PREP then writes
                      only the norms, FINAL reads z_tr, and the caller's GEMMs
                      take z_tr (strided) in place of zm */
  void* norms;     /* [B, C]     acc: ||zm||, -1 on padded positions */
  void* g;         /* [B, C, C]  acc (GEMM output) */
  void* s;         /* [B, C, C]  gemm_dtype */
  void* den;       /* [B, C]     acc */
  void* num;       /* [B, C, d'] acc (GEMM output) */
  void* dnum;      /* [B, C, d'] gemm_dtype */
  void* dden;      /* [B, C]     acc */
  void* ds0;       /* [B, C, C]  acc (GEMM output) */
  void* dgsym;     /* [B, C, C]  gemm_dtype */
  void* dzd;       /* [B, C, d'] acc (GEMM output) */
  void* dzh;       /* [B, C, d'] acc (GEMM output) */
  void* workspace; /* partial sums, >= avey_bwd_workspace_size() bytes */
  uint64_t workspace_bytes;

  /* Gradients (input dtype); NULL = not wanted. grad_v and grad_bias are
   * contiguous; grad_z_tr and grad_z_tl share the element strides below
   * (0 = contiguous [B, C, d']), so both can be the halves of one
   * [B, C, 2d'] gradient (row stride 2d'). */
  void* grad_z_tr;
  void* grad_v;
  void* grad_z_tl;
  void* grad_bias;
  int64_t grad_batch_stride, grad_row_stride;
} AveyBwdParams;

/* Enqueue one backward step on `stream`. Returns AVEY_OK or a negative
 * AveyStatus; the pointers a step reads or writes must be set. */
AVEY_API int avey_bwd_step_v1(const AveyBwdParams* params, int step, void* stream);

/*
 * Batched matrix product on the tcgen05 tensor cores (no counterpart in the
 * reference, which computes its products with torch.matmul / tl.dot): for
 * every batch entry b,
 *
 *   C[b] = A[b] B[b]                              out_dtype AVEY_F32, or
 *   C[b] = act(A[b] B[b] + bias) (.) gate[b]      out_dtype == dtype (16-bit)
 *
 * with A [m x k] and B [k x n] of `dtype` (AVEY_BF16 or AVEY_F16) and fp32
 * accumulation. It runs the contractions of the backward steps above
 * (avey_kernel_b200/backward.py), the enricher projection that feeds
 * avey_fwd_v1 (with the row sums of squares of its tail columns, see
 * avey_fwd_presummed_v1) and the static layers.
 *
 * Layouts (strides in elements, each operand's contiguous dimension has
 * stride 1):
 *   A: a_major AVEY_MAJOR_K:  A[b][i][k] at a + b*a_batch_stride + i*a_ld + k
 *      a_major AVEY_MAJOR_MN: A[b][i][k] at a + b*a_batch_stride + k*a_ld + i
 *   B: b_major AVEY_MAJOR_K:  B[b][k][j] at b + b*b_batch_stride + j*b_ld + k
 *      b_major AVEY_MAJOR_MN: B[b][k][j] at b + b*b_batch_stride + k*b_ld + j
 *   C: C[b][i][j] at c + b*c_batch_stride + i*c_ld + j
 * A batch stride of 0 shares the operand across the batch. Base addresses
 * must be 16-byte aligned and every ld / batch stride a whole number of 16
 * bytes (TMA); k, m and n are otherwise free (edges are zero-filled).
 *
 * mode skips work that the causal structure makes unnecessary:
 *   AVEY_GEMM_DENSE      every C[b][i][j];
 *   AVEY_GEMM_LOWER_OUT  only C[b][i][j] with j <= i is wanted: 128 x 256
 *                        output tiles wholly above the diagonal are not
 *                        computed and not written (their memory keeps
 *                        whatever it held);
 *   AVEY_GEMM_K_LOWER    A[b][i][k] == 0 for k > i (lower-triangular A): the
 *                        K loop of each 128-row tile stops after its last row;
 *   AVEY_GEMM_K_UPPER    A[b][i][k] == 0 for k < i: the K loop of each
 *                        128-row tile starts at its first row.
 * The K-range modes give the dense result bit for bit (the skipped terms are
 * exact zeros).
 *
 * 16-bit output only: bias [n] (or NULL), activation (AveyActivation), gate
 * (same shape as C, or NULL), and sumsq: NULL, or n_planes = ceil((n -
 * sumsq_col0) / 128) planes of batch*m floats, plane p holding for every row
 * the sum of squares of the stored (rounded) outputs of columns
 * [sumsq_col0 + 128p, sumsq_col0 + 128p + 128) (sumsq_col0 a multiple of 128;
 * sums in a fixed order, bitwise reproducible).
 */
typedef enum AveyMajor {
  AVEY_MAJOR_K = 0,
  AVEY_MAJOR_MN = 1,
} AveyMajor;

typedef enum AveyGemmMode {
  AVEY_GEMM_DENSE = 0,
  AVEY_GEMM_LOWER_OUT = 1,
  AVEY_GEMM_K_LOWER = 2,
  AVEY_GEMM_K_UPPER = 3,
} AveyGemmMode;

typedef struct AveyGemmParams {
  uint32_t struct_size; /* sizeof(AveyGemmParams) */
  int32_t dtype;        /* operands: AVEY_BF16 or AVEY_F16 */
  int32_t out_dtype;    /* AVEY_F32, or dtype */
  int32_t mode;         /* AveyGemmMode */
  int64_t batch, m, n, k;
  const void* a;
  int64_t a_batch_stride, a_ld;
  int32_t a_major; /* AveyMajor */
  const void* b;
  int64_t b_batch_stride, b_ld;
  int32_t b_major; /* AveyMajor */
  void* c;
  int64_t c_batch_stride, c_ld;
  const void* bias; /* [n] of dtype, or NULL (16-bit output only) */
  const void* gate; /* [batch][m][n] of dtype, or NULL (16-bit output only) */
  int64_t gate_batch_stride, gate_ld;
  int32_t activation; /* AveyActivation (16-bit output only) */
  int32_t sumsq_col0; /* first column of the row sums of squares */
  float* sumsq;       /* planes of row sums of squares, or NULL */
  int32_t kernel;     /* AVEY_GEMM_KERNEL_*: AUTO runs SINGLE (measured the
                         faster of the two on every shape tried) */
} AveyGemmParams;

/* GEMM kernels: one CTA per 128 x 256 output tile, or a pair of CTAs on
 * neighbouring SMs per 256 x 256 tile sharing each MMA (tcgen05 cta_group::2),
 * which halves the B bytes each SM loads per MMA cycle. Same results. */
#define AVEY_GEMM_KERNEL_AUTO 0
#define AVEY_GEMM_KERNEL_SINGLE 1
#define AVEY_GEMM_KERNEL_PAIR 2

AVEY_API int avey_gemm_v1(const AveyGemmParams* params, void* stream);

/*
 * avey_fwd_v1 with the row sums of squares of z_tr supplied by the caller
 * (no counterpart in the reference, whose normalisation pre-pass,
 * ops.py:107-108, is always a separate pass over z_tr): `sumsq` holds
 * `planes` planes of batch*context floats, summed in plane order, as written
 * by the enricher's avey_gemm_v1 epilogue (its tail columns). The norm
 * fused tcgen05 kernel and the long-context path read these sums instead of
 * summing z_tr's rows; other paths ignore them. Up to 512 tokens the planes
 * are combined into params->workspace, which must then hold batch * context
 * floats (4-byte aligned); above 512 tokens the workspace is the one
 * avey_fwd_workspace_size reports.
 */
AVEY_API int avey_fwd_presummed_v1(const AveyFwdParams* params, const float* sumsq, int planes,
                                   void* stream);

/* Bytes of `workspace` the backward steps need for these parameters. */
AVEY_API int avey_bwd_workspace_size(const AveyBwdParams* params, uint64_t* bytes);

/* Message for the last non-OK status returned on this thread ("" if none). */
AVEY_API const char* avey_last_error(void);

/* Device-side status word of the current device: 0, or the OR of the
 * AVEY_DEVFLAG_* bits raised by kernels since the last clear. Synchronises
 * the device. clear != 0 resets it. */
#define AVEY_DEVFLAG_TIMEOUT 1u /* a bounded wait on an mbarrier gave up */
AVEY_API int avey_device_status(uint32_t* flags, int clear);

/* Number of kernels this library has launched in this process. */
AVEY_API uint64_t avey_launch_count(void);

/* Test-only hooks of the failure path (no counterpart in the reference).
 * wait_limit_cycles: SM cycles after which a bounded wait on an mbarrier gives
 * up (<= 0 restores the default of about one second). stall != 0: later
 * launches of the fused tensor-core kernel start with their TMA and MMA warps
 * issuing nothing, so its compute warps' first wait runs out, the kernel
 * raises AVEY_DEVFLAG_TIMEOUT, unwinds and returns (no trap, the context stays
 * usable). The wait limit applies to the current device; the stall flag to
 * the process. Not for production use. */
AVEY_API int avey_test_hooks_v1(long long wait_limit_cycles, int stall);

/* AVEY_ABI_VERSION of the loaded library. */
AVEY_API int avey_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* AVEY_B200_H */
