/*
 * thorn_b200: C ABI of the B200 (sm_100a) kernels behind the THORN optimizer step.
 *
 * Every entry point takes device pointers, sizes and scalars plus a CUDA
 * stream (as `void*`, NULL = legacy default stream), enqueues its kernels on
 * that stream and returns a status code (THORN_OK == 0).  None of them
 * allocates device memory or synchronises the host; scratch space is passed in
 * by the caller.  Tensors are dense row-major.  A matrix tensor of any rank >= 2
 * is viewed as `batch x rows x cols` (batch = product of the leading dims),
 * which is how the reference treats conv kernels (thorn.py:628-633).
 *
 * File references are to thorn/thorn.py of pykeio/THORN v3.1.1.
 */
#ifndef THORN_B200_H
#define THORN_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define THORN_API __attribute__((visibility("default")))
#else
#define THORN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* element types */
#define THORN_F32 0
#define THORN_BF16 1
#define THORN_F16 2

/* status codes */
#define THORN_OK 0
#define THORN_ERR_ARG 1          /* bad size / dtype / null pointer */
#define THORN_ERR_ALIGN 2        /* pointer or leading dimension not aligned as required */
#define THORN_ERR_CUDA 3         /* a CUDA runtime call or kernel launch failed */
#define THORN_ERR_UNSUPPORTED 4  /* no device / wrong architecture / missing driver entry point */
#define THORN_ERR_TOO_LARGE 5    /* problem needs more than THORN_NS_STATIC_WORKSPACE_BYTES */

/* --------------------------------------------------------------------------
 * Library information
 * ------------------------------------------------------------------------ */
THORN_API int thorn_abi_version(void);
THORN_API const char* thorn_status_string(int status);
/* Number of kernels this library has launched in this process. */
THORN_API uint64_t thorn_launch_count(void);
/* cudaError_t of the last failing CUDA call inside the library (0 if none). */
THORN_API int thorn_last_cuda_error(void);
/* Tensor-core work issued by thorn_ns_batched / thorn_sym_addmm so far:
 * dense-equivalent FLOPs (2 M N K per product) and FLOPs of the tiles
 * actually executed (lower-triangle tiles only for symmetric products). */
THORN_API void thorn_gemm_flops(double* dense, double* executed);
/* GEMM tiling of the NS products: nonzero (default) uses 2-CTA 256x256 cluster
 * tiles (tcgen05.mma.cta_group::2) whenever both output dimensions are >= 256;
 * zero keeps every product on single-CTA 128x256 tiles.  Returns the previous
 * setting.  Process-wide; both settings give the same results up to
 * floating-point summation order. */
THORN_API int thorn_set_gemm_pair(int enable);
/* Epilogue of the 2-CTA tiles: nonzero (default) stages each 32x32 output block
 * in shared memory and writes it (and its mirror or transpose) with TMA bulk
 * stores, with C blocks TMA-loaded one block ahead; zero stores from registers.
 * Applies when D, D2 and C are 16-byte aligned with leading dimensions and batch
 * strides that are multiples of 8.  Returns the previous setting.  Both settings
 * give bit-identical results. */
THORN_API int thorn_set_gemm_staged_epilogue(int enable);
/* NS GEMM launches: nonzero uses programmatic dependent launch, so each GEMM's
 * set-up (barriers, TMEM, descriptor prefetch) overlaps the previous kernel's
 * tail and its CTAs wait for that kernel to finish before touching global
 * memory; zero (default) launches in plain stream order.  Returns the previous
 * setting.  Both settings give bit-identical results. */
THORN_API int thorn_set_gemm_pdl(int enable);
/* 2-CTA NS GEMM tiles: nonzero gives operand TMA loads an L2 evict_last policy
 * and output bulk stores an evict_first policy; zero (default) uses none.
 * Returns the previous setting.  Both settings give bit-identical results. */
THORN_API int thorn_set_gemm_l2_hints(int enable);
/* Limit, in nanoseconds of GPU global time, of every bounded wait inside the NS
 * GEMMs (default 10 s; 0 restores the default).  A wait that runs out sets the
 * call's err_flag, stops the CTA's other roles and frees its tensor memory, so
 * the kernel returns and the context stays usable.  Returns the previous limit. */
THORN_API uint64_t thorn_set_wait_limit_ns(uint64_t limit_ns);
/* Failure test of the bounded waits: nonzero makes the NS GEMMs' TMA producers
 * issue no loads (and the small-matrix NS kernel issue no MMA), so no copy or
 * MMA is ever in flight and the first wait for one runs out after the wait
 * limit.  Results are undefined while set; zero (default) is the normal path.
 * Returns the previous setting.  For tests of the error path only. */
THORN_API int thorn_set_gemm_test_stall(int enable);
/* Newton-Schulz of matrices whose smaller dimension is at most 128 and larger
 * at most 512: nonzero (default) runs the whole iteration of a batch in one
 * launch, one CTA per matrix with every operand resident in shared memory;
 * zero runs the same products as separate GEMM launches.  Returns the previous
 * setting. */
THORN_API int thorn_set_ns_small(int enable);

/* --------------------------------------------------------------------------
 * (R)Adam(-atan2)W over many tensors in one launch per dtype pair.
 * Replaces _adam_update (thorn.py:838-888) and its Triton kernel
 * _adam_update_kernel (thorn.py:147-185), which the reference launches once
 * per parameter (thorn.py:859-874).
 *   m <- m + (g - m)(1 - beta1);  v <- beta2 v + (1 - beta2) g^2
 *   u  = atan2(m bc1, sqrt(v bc2))          (eps == 0)
 *      = m bc1 / (sqrt(v bc2) + eps)        (eps > 0)
 *      = m                                   (degenerate: RAdam rect == 0)
 *   u <- u + wd p  where u p >= 0 (cautious weight decay);  p <- p - lr u
 * ------------------------------------------------------------------------ */
typedef struct {
  void* p;            /* param (p_dtype); NULL: update the moments only */
  const void* g;      /* grad (p_dtype) */
  void* m;            /* first moment (s_dtype) */
  void* v;            /* second moment (s_dtype) */
  int64_t numel;
  float lr;           /* group lr * rect * magma scale */
  float bc1;          /* 1 / (1 - beta1^step) */
  float bc2;          /* 1 / (1 - beta2^step) */
  int32_t degenerate; /* nonzero: u = m (rect == 0) */
} thorn_adam_tensor;

/* beta1 and beta2 are doubles: the kernel uses fp32 (1 - beta) formed in double,
 * as the reference passes 1.0 - float(beta) to its kernel (thorn.py:868). */
THORN_API int thorn_adamw_multi(const thorn_adam_tensor* tensors, int n, int p_dtype, int s_dtype,
                                double beta1, double beta2, float weight_decay, float eps, void* stream);

/* --------------------------------------------------------------------------
 * Deterministic reductions.  Kernels that reduce (sums of squares, gain
 * gradients, per-neuron-norm statistics) never accumulate floats with
 * atomics: each block writes its partial sum to a caller-provided scratch
 * buffer, and the last block of each segment (found with an integer counter)
 * adds the partials in a fixed order.  Results are therefore bitwise
 * reproducible run to run.  A scratch buffer must be all zero on entry; the
 * kernels zero every counter and partial they used before they finish, so it
 * is all zero again on return and may be reused by any later call on the
 * same stream without clearing.  Calls that overlap in time need disjoint
 * scratch.
 * ------------------------------------------------------------------------ */

/* --------------------------------------------------------------------------
 * Orthogonalized group, before Newton-Schulz: momentum + Nesterov, and the
 * per-matrix sum of squares needed to normalise the NS input.
 * Replaces _update_momentum (thorn.py:1376-1381):  m <- beta1 m + g;
 * u = g + beta1 m (rounded to u_dtype; u itself is not stored -- the NS
 * input pass recomputes it from g and the new m).  With md != 0 it also does
 * _recover_direction (thorn.py:890-908): gain = row_sp col_sp (or the scalar
 * gain); p <- p / gain; g <- g gain (stored back when write_grad != 0), and
 * the gain-gradient sums of _update_magnitude (thorn.py:910-932):
 *   row_gsum[i] = sum_j round(round(p_dir g_raw) col_sp[j])
 *   col_gsum[j] = sum_i round(round(p_dir g_raw) row_sp[i])
 * (or row_gsum[0] = sum of round(p_dir g_raw) for a scalar gain).  With
 * m == NULL only the md part runs (no momentum, normsq unused): the direction
 * recovery of the (R)AdamW group with decouple_md (thorn.py:1704-1705).
 * ------------------------------------------------------------------------ */
typedef struct {
  void* p;
  void* g;
  void* m;
  float* normsq;        /* out: per sub-matrix sum of u^2, [batch] */
  int64_t batch, rows, cols;
  const float* row_sp;  /* md: softplus(row_gain) rounded to p dtype, [batch*rows] (scalar gain: [1]) */
  const float* col_sp;  /* md: softplus(col_gain) rounded to p dtype, [batch*cols] (scalar gain: unused) */
  int32_t scalar_gain;  /* md: nonzero when the gain is one scalar, row_sp[0] */
  float* row_gsum;      /* md out: [batch*rows] (scalar gain: [1]) */
  float* col_gsum;      /* md out: [batch*cols] (unused for a scalar gain) */
  void* scratch;        /* thorn_ortho_pre_scratch_bytes(batch, rows, cols, md) bytes (see above) */
} thorn_ortho_pre_tensor;

THORN_API int64_t thorn_ortho_pre_scratch_bytes(int64_t batch, int64_t rows, int64_t cols, int md);
THORN_API int thorn_ortho_pre_multi(const thorn_ortho_pre_tensor* tensors, int n, int p_dtype, int s_dtype,
                                    int u_dtype, float beta1, int md, int write_grad, void* stream);

/* --------------------------------------------------------------------------
 * Newton-Schulz input: X = ns(u / (||u||_F + 1e-8)) in the matrix's own
 * orientation (the NS GEMMs read a tall input transposed, so no transpose
 * pass is needed).  Replaces thorn.py:629-635.  u = round_u(fma(beta1, m, g_eff)) is recomputed from the
 * gradient and the moment written by thorn_ortho_pre_multi, with
 * g_eff = round_p(g * gain) when md != 0 (g still holds the raw gradient,
 * i.e. the pre pass ran with write_grad == 0) and g_eff = g otherwise.
 * x is [batch, rows, ld] with ld = thorn_ns_ld(cols).
 * ------------------------------------------------------------------------ */
typedef struct {
  const void* g;
  const void* m;
  const float* normsq;  /* [batch] sums of squares from thorn_ortho_pre_multi */
  void* x;              /* out, ns_dtype */
  int64_t batch, rows, cols;
  const float* row_sp;  /* md gains as in thorn_ortho_pre_tensor */
  const float* col_sp;
  int32_t scalar_gain;
  int32_t md;
} thorn_ns_cast_tensor;

THORN_API int64_t thorn_ns_ld(int64_t n);
THORN_API int thorn_ns_cast_multi(const thorn_ns_cast_tensor* tensors, int n, int p_dtype, int s_dtype, int u_dtype,
                        int ns_dtype, float beta1, void* stream);

/* --------------------------------------------------------------------------
 * Newton-Schulz polar factor of a batch of same-shape matrices.
 * Replaces _polar_decomp_impl (thorn.py:626-662) with its custom op
 * thorn::sym_addmm (thorn.py:298-377) and torch.bmm/baddbmm (thorn.py:614-624,
 * 653).  x: normalised input from thorn_ns_cast_multi, [batch, rows,
 * thorn_ns_ld(cols)] (a tall matrix is not transposed; the GEMMs read it as
 * X = x^T).  out: [batch, rows, cols], ns_dtype.  Runs the standard quintic for square
 * matrices and Gram Newton-Schulz (restarts at the listed iterations) for
 * rectangular ones, with the reference's recurrences and coefficients.
 * err_flag: device int set nonzero if a bounded wait in a kernel gave up
 * (may be NULL).
 * ------------------------------------------------------------------------ */
THORN_API int64_t thorn_ns_workspace_bytes(int64_t batch, int64_t rows, int64_t cols);
THORN_API int thorn_ns_batched(const void* x, void* out, void* workspace, int64_t workspace_bytes,
                     int64_t batch, int64_t rows, int64_t cols, int ns_dtype,
                     const double* coeffs, int iters, const int32_t* restarts, int n_restarts,
                     int* err_flag, void* stream);

/* Same as thorn_ns_batched, but allocates nothing and takes no workspace: for
 * callers that cannot allocate device memory, such as a custom call inside a
 * host framework that passes only operands and offers no allocator, or code
 * that must not call cudaMalloc after start-up.  It has no counterpart in the
 * reference.  The workspace is a fixed 64 MiB device array built into the
 * library, held on every GPU that loads the library's kernels until the
 * process exits.  Problems whose thorn_ns_workspace_bytes(batch, rows, cols)
 * exceed THORN_NS_STATIC_WORKSPACE_BYTES are rejected with
 * THORN_ERR_TOO_LARGE (e.g. one 2896x2896 or 1024x8192 matrix fits).
 * The first call on a device looks up the array's device address (once per
 * device, with that device current); make that first call before any CUDA
 * stream capture.  The address is cached for the life of the process: after
 * cudaDeviceReset (or any other teardown of the device's primary context) it
 * is stale, so do not use this entry point on that device again.  All calls on
 * a device share the one array and nothing in it needs to start at zero, so
 * calls that overlap on the GPU (two streams, two host threads) race on it and
 * must be serialised by the caller. */
#define THORN_NS_STATIC_WORKSPACE_BYTES (64ll * 1024 * 1024)
THORN_API int thorn_ns_batched_static(const void* x, void* out, int64_t batch, int64_t rows, int64_t cols,
                                      int ns_dtype, const double* coeffs, int iters, const int32_t* restarts,
                                      int n_restarts, int* err_flag, void* stream);

/* O = alpha A@B + beta C for symmetric A@B and C: the thorn::sym_addmm
 * contract (thorn.py:298-363).  A [batch, M, K], B [batch, K, M],
 * C [batch, M, M] (c_batched) or [M, M] or NULL, O [batch, M, M]; all with
 * leading dimensions a multiple of 8 elements.  Only tiles on or below the
 * diagonal are computed.  O is split into 128 x 128 blocks: diagonal blocks
 * hold the computed values, each block below the diagonal is mirrored into
 * the block above it (the reference's Triton kernel likewise keeps its
 * diagonal tiles as computed and mirrors the others). */
THORN_API int thorn_sym_addmm(const void* A, const void* B, const void* C, void* O, int64_t batch, int64_t M,
                    int64_t K, int c_batched, float alpha, float beta, int dtype, int* err_flag,
                    void* stream);

/* --------------------------------------------------------------------------
 * Per-neuron (row) normalisation statistics for tall matrices.
 * Replaces _pnn_row_stats_kernel (thorn.py:205-228) and _pnn_reduce_kernel
 * (thorn.py:230-253) of _per_neuron_norm_update (thorn.py:709-757):
 *   sumsq_r = sum_j u_rj^2;  s_r = rsqrt(max(sumsq_r / N, eps))
 *   stats[b] = {sum_r sumsq_r, sum_r s_r^2 sumsq_r}
 *   (gscale_b = sqrt(stats[b][0]) / max(sqrt(stats[b][1]), eps))
 * u is the NS output rounded to p_dtype; eps = finfo(p_dtype).eps.
 * ------------------------------------------------------------------------ */
typedef struct {
  const void* U;        /* u_dtype [batch, rows, cols] */
  float* row_scale;     /* out: s_r, [batch*rows] (s_r * gscale_b when fold != 0) */
  float* mat_stats;     /* out: [batch][2] */
  int64_t batch, rows, cols;
  void* scratch;        /* thorn_pnn_scratch_bytes(batch, rows) bytes */
  int32_t fold;         /* nonzero: fold gscale_b into row_scale (one factor per row) */
} thorn_pnn_tensor;

THORN_API int64_t thorn_pnn_scratch_bytes(int64_t batch, int64_t rows);
THORN_API int thorn_pnn_stats_multi(const thorn_pnn_tensor* tensors, int n, int u_dtype, int p_dtype,
                                    void* stream);

/* --------------------------------------------------------------------------
 * Orthogonalized group, after Newton-Schulz: scale and apply.
 * Replaces _ortho_post (thorn.py:1399-1413), _weight_decay_update
 * (thorn.py:683-702, Triton _wd_update_kernel thorn.py:187-203) and
 * _pnn_apply_kernel (thorn.py:255-280):
 *   u = round_p(U) * s_r * gscale_b   (pnn; or * row_scale[r] when mat_stats is NULL)
 *   u <- u + wd p where u p >= 0;  p <- p - lr u
 * With p_normsq != NULL it also writes ||p_new||^2 per sub-matrix (for the
 * decouple_md renorm; needs scratch).  U may be ns_dtype (bf16/f16) or f32.
 * ------------------------------------------------------------------------ */
typedef struct {
  const void* U;
  void* p;
  const float* row_scale;  /* NULL: no row scaling */
  const float* mat_stats;  /* NULL: row_scale is the final factor */
  float* p_normsq;         /* NULL or out [batch] */
  int64_t batch, rows, cols;
  float lr;                /* lr * lr_scale (thorn.py:768-780) * magma scale */
  void* scratch;           /* with p_normsq: thorn_sumsq_scratch_bytes(batch, rows, cols) bytes */
  int32_t round_u;         /* nonzero: round U to the param dtype first (thorn.py:1404);
                              zero: use it as is (the sharded path's fp32 u, thorn.py:1079-1081, 1143) */
} thorn_ortho_post_tensor;

THORN_API int thorn_ortho_post_multi(const thorn_ortho_post_tensor* tensors, int n, int u_dtype, int p_dtype,
                                     float weight_decay, void* stream);

/* --------------------------------------------------------------------------
 * Magnitude-direction decoupling helpers (thorn.py:910-977, 1414-1421).
 * thorn_md_prep_multi: sp = round_p(softplus(gain)), sig = round_p(sigmoid(gain))
 *   as fp32 (sig may be NULL)
 * thorn_md_gain_grad_multi: grad = round_p(round_p(gsum) * sig)  (p_dtype output)
 * thorn_md_finalize_multi: renorm to the target norm, then multiply by the
 *   new gains:  p <- round(round(round(p * round(target / round(round(||p||) + 1e-8)))
 *                 * row_sp) * col_sp)   (scalar gain: one multiply)
 * ------------------------------------------------------------------------ */
typedef struct {
  const void* gain;  /* p_dtype [n] */
  float* sp;         /* out [n] */
  float* sig;        /* out [n] or NULL */
  int64_t n;
} thorn_md_prep_tensor;

typedef struct {
  const float* gsum;  /* [n] */
  const float* sig;   /* [n] */
  void* grad;         /* out, p_dtype [n] */
  int64_t n;
} thorn_md_grad_tensor;

THORN_API int thorn_md_prep_multi(const thorn_md_prep_tensor* tensors, int n, int p_dtype, void* stream);
THORN_API int thorn_md_gain_grad_multi(const thorn_md_grad_tensor* tensors, int n, int p_dtype, void* stream);

typedef struct {
  void* p;
  const float* normsq;   /* [batch] ||p||^2 (NULL: no renorm) */
  const float* target;   /* target norm per sub-matrix (stride target_stride) */
  int64_t target_stride; /* 0: one target for all sub-matrices */
  const float* row_sp;   /* [batch*rows] (scalar gain: [1]) */
  const float* col_sp;   /* [batch*cols] (scalar gain: unused) */
  int32_t scalar_gain;
  int64_t batch, rows, cols;
} thorn_md_final_tensor;

THORN_API int thorn_md_finalize_multi(const thorn_md_final_tensor* tensors, int n, int p_dtype, void* stream);

/* Sum of squares per sub-matrix: out[b] = sum of x^2 over sub-matrix b (the
 * renorm of the (R)AdamW group with decouple_md, thorn.py:1716-1717). */
typedef struct {
  const void* x;
  float* out;            /* [batch] */
  int64_t batch, rows, cols;
  void* scratch;         /* thorn_sumsq_scratch_bytes(batch, rows, cols) bytes */
} thorn_sumsq_tensor;

THORN_API int64_t thorn_sumsq_scratch_bytes(int64_t batch, int64_t rows, int64_t cols);
THORN_API int thorn_sumsq_multi(const thorn_sumsq_tensor* tensors, int n, int dtype, void* stream);

/* Magma momentum-aligned masking statistics (replaces the three sums of
 * _momentum_aligned_mask, thorn.py:806-829, and the direction recovery
 * g * gain of _recover_direction, thorn.py:896-905, that feeds it):
 *   out[0] = sum g'*m,  out[1] = sum g'^2,  out[2] = sum m^2
 * over every element of the tensor (viewed as batch x rows x cols), each an
 * fp64 sum of fp32 products in a fixed order (bitwise reproducible), where
 * g' = g, or under decouple_md with row_gain set
 *   split gain:  g' = rn_G(g * rn_G(rn_G(softplus(row_gain[b*rows+r])) * rn_G(softplus(col_gain[b*cols+c]))))
 *   scalar gain: g' = rn_G(g * rn_G(softplus(row_gain[0])))
 * (rn_G: rounding to the gradient dtype; the gains have the gradient dtype).
 * An empty tensor leaves its out[] untouched. */
typedef struct {
  const void* g;         /* gradient, g_dtype */
  const void* m;         /* moment before this step's update, m_dtype, same shape */
  const void* row_gain;  /* NULL: no direction recovery */
  const void* col_gain;  /* split gain only */
  int32_t scalar_gain;
  int64_t batch, rows, cols;
  double* out;           /* [3] */
  void* scratch;         /* thorn_magma_scratch_bytes(batch, rows, cols) bytes, zero (kernels leave it zero) */
} thorn_magma_tensor;

THORN_API int64_t thorn_magma_scratch_bytes(int64_t batch, int64_t rows, int64_t cols);
THORN_API int thorn_magma_stats_multi(const thorn_magma_tensor* tensors, int n, int g_dtype, int m_dtype,
                                      void* stream);

/* --------------------------------------------------------------------------
 * Peer-memory exchange of the FSDP2 Shard(0) path (THORN.exchange = "peer").
 * Replaces the reference's per-matrix dist.gather / dist.scatter of fp32 rows
 * (_DistributedTHORNState.gather / scatter, thorn.py:1023-1122) for ranks of one
 * node: every rank exports one device arena by CUDA IPC and maps its peers'.
 * The NS input pass (thorn_ns_cast_multi) then stores each rank's rows straight
 * into the owner's arena, and result rows return with thorn_copy_async (copy
 * engines; no SMs).  Ordering: after its stores or copies a rank calls
 * thorn_peer_signal on its slot in every destination's arena; a receiver calls
 * thorn_peer_wait on its own slots.  Slot values must grow from step to step.
 * A wait that exceeds limit_ns sets *err_flag to 3 and returns.
 *   thorn_peer_alloc     cudaMalloc + zero fill (the flag slots start at 0)
 *   thorn_ipc_handle     THORN_IPC_HANDLE_BYTES bytes that another process opens
 *   thorn_ipc_open       map a peer's arena into the current device's context
 *   thorn_copy_async     cudaMemcpyAsync (cudaMemcpyDefault) on `stream`
 *   thorn_peer_signal    slots[i] <- value (release, system scope), i < n <= 64
 *   thorn_peer_wait      wait until slots[0..n) >= value (acquire, system scope)
 * ------------------------------------------------------------------------ */
#define THORN_IPC_HANDLE_BYTES 64
THORN_API int thorn_peer_alloc(int64_t bytes, void** out);
THORN_API int thorn_peer_free(void* p);
THORN_API int thorn_ipc_handle(const void* p, void* handle);
THORN_API int thorn_ipc_open(const void* handle, void** out);
THORN_API int thorn_ipc_close(void* p);
THORN_API int thorn_copy_async(void* dst, const void* src, int64_t bytes, void* stream);
THORN_API int thorn_peer_signal(uint64_t* const* slots, int n, uint64_t value, void* stream);
THORN_API int thorn_peer_wait(const uint64_t* slots, int n, uint64_t value, uint64_t limit_ns, int* err_flag,
                              void* stream);

#ifdef __cplusplus
}
#endif

#endif /* THORN_B200_H */
