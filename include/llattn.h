/*
 * llattn.h — C ABI of libllattn.so, the sm_100a kernels of the fused
 * local + latent attention block (LocalLatentAttention of
 * Fenix46/local-latent-attention, models.py:61-462).
 *
 * Plain C: device pointers, sizes and a stream handle. No torch types.
 * The caller owns every buffer (outputs, saved tensors and the backward
 * workspace); the library never allocates or frees device memory on its
 * launch paths. Its only global state: the device fault word of the
 * tensor-core kernels and its host-mapped mirror (one pinned 64-byte host
 * allocation per process, made by the first launching call), and the fixed
 * scratch array of llattn_bwd_noalloc. Every entry point returns 0 on success and
 * a nonzero llattn_status otherwise; llattn_last_error() then describes the
 * failure (thread-local string). Argument errors are detected on the host
 * before any launch.
 *
 * Reference interfaces replaced (paths within the reference project):
 *   llattn_pool_fwd / llattn_pool_bwd
 *       LocalLatentAttention._pool_to_latents      models.py:159-214
 *       LocalLatentAttention._pool_query_blocks    models.py:216-230
 *   llattn_pool_proj_fwd / llattn_pool_proj_bwd
 *       the pooling with rkv_proj / rq_proj       models.py:159-230, 333-347
 *   llattn_fwd
 *       kernels/llattn_op.py:34-84   _call_fwd (launch of llattn_fwd_kernel)
 *       with the math of models.py:232-305 (local) and :355-438 (latent,
 *       r_out, gate, mix) — the PyTorch module is the semantic target.
 *   llattn_bwd
 *       kernels/llattn_op.py:87-181  _call_bwd (dq and dkv kernels), with
 *       exact autograd of the same math.
 *   llattn_bwd_workspace_bytes
 *       replaces the zero-initialised fp32 grad buffers allocated by
 *       kernels/llattn_op.py:102-110.
 */
#ifndef LLATTN_H_
#define LLATTN_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LLATTN_VERSION 3

#if defined(__GNUC__)
#define LLATTN_API __attribute__((visibility("default")))
#else
#define LLATTN_API
#endif

typedef enum llattn_dtype {
  LLATTN_F32 = 0,  /* activations fp32: exact SIMT path (fp32 FMA)        */
  LLATTN_BF16 = 1  /* activations bf16: tcgen05 tensor-core path, fp32 acc */
} llattn_dtype;

typedef enum llattn_status {
  LLATTN_OK = 0,
  LLATTN_ERR_ARG = 1,       /* bad shape, pointer, stride or dtype          */
  LLATTN_ERR_ALIGN = 2,     /* pointer not aligned as the kernel requires   */
  LLATTN_ERR_LAUNCH = 3,    /* cudaLaunch / cudaFuncSetAttribute failure    */
  LLATTN_ERR_WORKSPACE = 4, /* workspace too small                          */
  LLATTN_ERR_DEVICE = 5     /* a kernel recorded a device-side fault        */
} llattn_status;

/* Block hyper-parameters: the ModelConfig fields the block reads
 * (models.py:21-37) plus the batch geometry of one call. */
typedef struct llattn_dims {
  int32_t batch;           /* B                                            */
  int32_t seq_len;         /* T                                            */
  int32_t n_heads;         /* H;  d_model = H * head_dim                   */
  int32_t head_dim;        /* hd                                           */
  int32_t latent_heads;    /* Lh                                           */
  int32_t latent_head_dim; /* ldh; latent_d_model = Lh * ldh               */
  int32_t window;          /* local_window W (> 0)                         */
  int32_t local_block;     /* local_block_size (default 256)              */
  int32_t latent_tokens;   /* latent_tokens Nl (upper bound on chunks)    */
  int32_t query_block;     /* latent_query_block_size; <= 1 = token-wise  */
  int32_t dtype;           /* llattn_dtype of activations                 */
  float gate_bias;         /* added to the local gate logit (0 = reference) */
  /* Sequence shards (since LLATTN_VERSION 2; both 0 = a whole sequence): the
   * call's row 0 is global position seq_offset of a total_len-token
   * sequence. The local block span, latent chunking and query blocks follow
   * total_len; masks and chunk ids follow global positions; gkv holds every
   * chunk of the whole sequence. The buffers must hold every key the rows'
   * outputs need (a shard plus a left halo of at least window rows, the
   * halo rows' own outputs being unused); seq_offset is a multiple of the
   * query block for block-pooled queries. */
  int32_t seq_offset;
  int32_t total_len;
  /* Row strides in elements (since LLATTN_VERSION 3; 0 = 3 * d_model, a
   * contiguous [B, T, 3d]): the qkv rows read by llattn_fwd / llattn_bwd and
   * the dqkv rows written by llattn_bwd may sit in a wider row-major buffer
   * (the qkv_proj output beside other per-token projections of one GEMM).
   * >= 3 d; a multiple of 8 for bf16 when not 3 d (16-byte TMA strides). */
  int32_t qkv_row_stride;
  int32_t dqkv_row_stride;
} llattn_dims;

/* Quantities derived from llattn_dims exactly as models.py derives them
 * (chunk / local_span / qblock from total_len; n_qrows over this call's rows). */
typedef struct llattn_geom {
  int32_t chunk;        /* cs  = ceil(T / min(Nl, T))          models.py:175-183 */
  int32_t n_chunks;     /* Nc  = ceil(T / cs)                                  */
  int32_t local_span;   /* bsL = min(T, max(W, local_block))   models.py:249   */
  int32_t qblock;       /* bs  = min(T, QB) if QB > 1 else 1   models.py:218   */
  int32_t n_qrows;      /* Tq  = ceil(T / bs)                                  */
} llattn_geom;

/* Forward of the attention core (everything between the projections):
 *   local  = windowed causal softmax(q k^T / sqrt(hd)) v   (per head)
 *   lat    = causal-chunk softmax(rq gk^T / sqrt(ldh)) gv  (per latent head)
 *   remote = lat W_rout^T + b_rout (broadcast per query block)
 *   w      = sigmoid(local.g_l + gate_bias - remote.g_r)
 *   mixed  = w local + (1 - w) remote
 * Layouts (row-major, element strides implied):
 *   qkv      [B, T, 3, H, hd]  dtype   (the qkv_proj output, un-split)
 *   rq       [B, Tq, Lh, ldh]  dtype   (the rq_proj output)
 *   gkv      [B, Nc, 2, Lh, ldh] dtype (the rkv_proj output of pooled x)
 *   w_rout   [H*hd, Lh*ldh]    dtype;  b_rout [H*hd] fp32
 *   g_local, g_remote [hd] fp32
 * Outputs: mixed [B, T, H*hd] dtype. Saved for backward: local_out
 * [B, T, H*hd] dtype, lse [B, H, T] fp32, lat [B, Tq, Lh*ldh] dtype,
 * lat_lse [B, Lh, Tq] fp32. */
typedef struct llattn_fwd_args {
  llattn_dims dims;
  const void* qkv;
  const void* rq;
  const void* gkv;
  const void* w_rout;
  const float* b_rout;
  const float* g_local;
  const float* g_remote;
  void* mixed;
  void* local_out;
  float* lse;
  void* lat;
  float* lat_lse;
} llattn_fwd_args;

/* One decode step: row t = dims.seq_len - 1 of llattn_fwd's `mixed` for the
 * dims.seq_len-token prefix (every size derived from that length, as the
 * reference's generation loop recomputes the whole prefix each step,
 * generate.py:188-202), computed from cached rows instead of recomputing
 * the prefix:
 *   qkv_cache [B, cache_len, 3, H, hd] dtype: rows 0..t of the prefix's
 *             qkv_proj output (cache_len >= seq_len)
 *   rq_row    [B, Lh*ldh] dtype: the rq_proj row of t's latent query (the
 *             token's own row, or its query block's pooled row)
 *   gkv       [B, Nc, 2, Lh, ldh] dtype: rkv_proj of the prefix's chunk means
 *   w_rout, b_rout, g_local, g_remote as in llattn_fwd
 * Output: mixed_row [B, H*hd] dtype. */
typedef struct llattn_decode_args {
  llattn_dims dims;
  int64_t cache_len;
  const void* qkv_cache;
  const void* rq_row;
  const void* gkv;
  const void* w_rout;
  const float* b_rout;
  const float* g_local;
  const float* g_remote;
  void* mixed_row;
} llattn_decode_args;

/* Backward of llattn_fwd. Inputs are the forward inputs, the saved tensors
 * and dmixed [B, T, H*hd] dtype. Outputs (all fully overwritten):
 *   dqkv [B, T, 3, H, hd] dtype, drq [B, Tq, Lh, ldh] dtype,
 *   dgkv [B, Nc, 2, Lh, ldh] dtype, dw_rout [H*hd, Lh*ldh] fp32,
 *   db_rout [H*hd] fp32, dg_local [hd] fp32, dg_remote [hd] fp32, and
 *   (optional, NULL to skip) db_qkv [3*H*hd] fp32 = the column sums of dqkv,
 *   the bias gradient of qkv_proj (models.py:80), which the tensor-core
 *   kernels take from the tiles they already hold instead of re-reading dqkv
 *   (fp32 sums of the unrounded values, fixed order).
 * workspace: device buffer of at least llattn_bwd_workspace_bytes(&dims)
 * bytes, 256-byte aligned; its contents need no initialisation. */
typedef struct llattn_bwd_args {
  llattn_dims dims;
  const void* qkv;
  const void* rq;
  const void* gkv;
  const void* w_rout;
  const float* b_rout;
  const float* g_local;
  const float* g_remote;
  const void* local_out;
  const float* lse;
  const void* lat;
  const float* lat_lse;
  const void* dmixed;
  void* dqkv;
  void* drq;
  void* dgkv;
  float* dw_rout;
  float* db_rout;
  float* dg_local;
  float* dg_remote;
  void* workspace;
  size_t workspace_bytes;
  float* db_qkv; /* since LLATTN_VERSION 2 */
} llattn_bwd_args;

/* Pool modes of llattn_pool_fwd / llattn_pool_bwd. */
typedef enum llattn_pool_mode {
  LLATTN_POOL_CHUNKS = 0, /* chunk means of x over cs tokens, last partial
                             chunk over its true count   (models.py:159-214) */
  LLATTN_POOL_QBLOCKS = 1, /* query-block means over bs tokens, zero padding
                              counted                    (models.py:216-230) */
  LLATTN_POOL_ACCUMULATE = 16 /* or'd into llattn_pool_bwd's mode: dx += the
                                 spread gradient instead of dx = (autograd's
                                 sum of x's gradient contributions) */
} llattn_pool_mode;

LLATTN_API int llattn_version(void);
LLATTN_API const char* llattn_last_error(void);

/* Fault bits (0 = none): set by a tensor-core kernel whose bounded wait on
 * a barrier ran out, after which that kernel abandoned its work and returned
 * (and every kernel launched after it on the device exits at once). The
 * kernels also set a host-mapped copy of the word, which llattn_fwd,
 * llattn_bwd, llattn_bwd_noalloc and llattn_decode test before launching:
 * once it is set they return LLATTN_ERR_DEVICE (like an asynchronous CUDA
 * error, the fault shows at the next call) until it is cleared. This
 * function returns the device word of the current device or'd with the host
 * copy; it synchronises with the device, so it is for tests and
 * diagnostics, not for the hot path. reset != 0 clears both. No counterpart
 * in the reference (its Triton kernels have no waits). */
LLATTN_API unsigned llattn_fault_status(int reset);
/* Sets bits in the host-mapped fault word without touching the GPU: the
 * host-side fault injection with which tests check that a recorded fault
 * makes the launching entry points fail. No counterpart in the reference. */
LLATTN_API int llattn_fault_inject_host(unsigned bits);

/* Fills *out from *dims. Returns LLATTN_ERR_ARG for inconsistent dims. */
LLATTN_API int llattn_geometry(const llattn_dims* dims, llattn_geom* out);

/* Workspace needed by llattn_bwd for these dims (0 on bad dims). */
LLATTN_API size_t llattn_bwd_workspace_bytes(const llattn_dims* dims);

/* x [B, T, d] dtype -> pooled [B, rows, d] dtype, rows = Nc or Tq. */
LLATTN_API int llattn_pool_fwd(const llattn_dims* dims, int mode, const void* x,
                    void* pooled, int64_t d, void* stream);
/* dpooled [B, rows, d] -> dx [B, T, d] (overwritten, or added to with
 * LLATTN_POOL_ACCUMULATE). */
LLATTN_API int llattn_pool_bwd(const llattn_dims* dims, int mode, const void* dpooled,
                    void* dx, int64_t d, void* stream);

/* Pooling fused with the latent projections. The pooled means are linear,
 * so chunk_mean(x) W_rkv^T + b_rkv = chunk_mean(x W_rkv^T) + b_rkv and
 * qblock_mean(x) W_rq^T + b_rq = qblock_mean(x W_rq^T) + b_rq: the caller
 * projects every token once, z = x [W_rkv; W_rq]^T (one GEMM, no bias), and
 * this pools the 3 Ld-wide rows of z instead of the d-wide rows of x.
 *   z    [B*T, ldz] dtype: columns [0, 2Ld) = x W_rkv^T, [2Ld, 3Ld) = x W_rq^T
 *   gkv  [B, Nc, 2Ld] = chunk means of z[:, :2Ld] + b_rkv
 *   rq   [B, Tq, Ld]  = query-block means of z[:, 2Ld:] + b_rq (the token's
 *        own row when latent_query_block_size <= 1)
 * b_rkv [2Ld] / b_rq [Ld] (dtype) may be NULL. Whole sequences only
 * (seq_offset 0), latent_d_model <= 128 (past that, projecting every token
 * costs more than pooling x first). Replaces the pooling and the two latent Linears of
 * LocalLatentAttention.forward (models.py:159-230, :333-347). */
LLATTN_API int llattn_pool_proj_fwd(const llattn_dims* dims, const void* z, int64_t ldz,
                    const void* b_rkv, const void* b_rq, void* gkv, void* rq, void* stream);
/* Its gradient with respect to z: dz[:, :2Ld] = dgkv of the token's chunk /
 * the chunk's count, dz[:, 2Ld:3Ld] = drq of the token's query block / bs
 * (or the token's own drq). Columns of dz past 3 Ld are left alone. */
LLATTN_API int llattn_pool_proj_bwd(const llattn_dims* dims, const void* dgkv, const void* drq,
                    void* dz, int64_t ldz, void* stream);

/* Bias gradient of a linear layer: out[c] = sum_r g[r, c] over a row-major
 * [rows, cols] matrix of dtype (LLATTN_BF16 / LLATTN_F32), fp32
 * accumulation in a fixed order (deterministic), out in dtype. Replaces the
 * bias-gradient reduction of torch.nn.Linear's autograd for the block's
 * qkv_proj / rq_proj / rkv_proj / out layers (models.py:80-84). workspace:
 * llattn_colsum_workspace_bytes(rows, cols, dtype) bytes of device memory. */
LLATTN_API size_t llattn_colsum_workspace_bytes(int64_t rows, int64_t cols, int dtype);
LLATTN_API int llattn_colsum(const void* g, int64_t rows, int64_t cols, int dtype, void* out,
                  void* workspace, size_t workspace_bytes, void* stream);

LLATTN_API int llattn_fwd(const llattn_fwd_args* args, void* stream);
/* Replaces nothing in the reference (its generation loop re-runs the whole
 * forward per token, generate.py:188-202); the per-token path of that loop. */
LLATTN_API int llattn_decode(const llattn_decode_args* args, void* stream);
LLATTN_API int llattn_bwd(const llattn_bwd_args* args, void* stream);

/* Backward without a caller-provided workspace. For callers that cannot
 * allocate device memory themselves: hosts that hand the library only
 * preallocated tensors from their own pool and forbid cudaMalloc, or loops
 * where an allocation (and its possible synchronisation) is not allowed.
 * No counterpart in the reference (its Triton backward allocates its fp32
 * grad buffers with torch on every call).
 *
 * Same arguments and results as llattn_bwd; args->workspace and
 * workspace_bytes are ignored. The scratch is a fixed array of
 * LLATTN_BWD_NOALLOC_SCRATCH_BYTES (32 MiB) inside the library, reserved on
 * every GPU that loads the library until the process exits. Dims whose
 * llattn_bwd_workspace_bytes exceeds that are rejected with
 * LLATTN_ERR_WORKSPACE (one 8192-token sequence of d_model 256 in bf16 needs
 * 21 MiB and fits; a 16 x 2048-token batch of d_model 1536 needs 307 MiB and
 * does not). The first call on each device looks up the array's device
 * address (with that device current) and caches it, so make that first call
 * before any stream capture; the cached address does not survive
 * cudaDeviceReset. The stream must belong to the current device (else
 * LLATTN_ERR_ARG). The array is reserved when the library's device code
 * first loads on a device (at context creation under
 * CUDA_MODULE_LOADING=EAGER): a device without 32 MiB free then yields
 * LLATTN_ERR_WORKSPACE. All calls on a device share the one array: calls that
 * can overlap on the GPU (different streams, or other threads) race and
 * corrupt each other's results — serialise them. Nothing in it needs clearing
 * between calls; it allocates and frees nothing. */
#define LLATTN_BWD_NOALLOC_SCRATCH_BYTES (32u << 20)
LLATTN_API int llattn_bwd_noalloc(const llattn_bwd_args* args, void* stream);

/* Per-kernel timing with CUDA events on the launching stream, the native
 * side of the module's set_profile/get_profile_stats (models.py:131-157,
 * which times phases with host syncs instead). enable != 0 turns it on;
 * every call resets the totals and returns the number of kernel groups.
 * llattn_profile_read synchronises on the recorded events and fills, per
 * group id < n, the summed milliseconds and launch counts. */
LLATTN_API int llattn_profile_enable(int enable);
LLATTN_API int llattn_profile_read(double* ms, long long* launches, int n);
LLATTN_API const char* llattn_profile_name(int id);

#ifdef __cplusplus
}
#endif

#endif /* LLATTN_H_ */
