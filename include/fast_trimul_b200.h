/*
 * fast_trimul_b200 -- C ABI of the B200 (sm_100a) triangle multiplicative update.
 *
 * The drop-in boundary for the reference's operator path. The reference
 * (fast_trimul, pure Python) reaches its GPU code through
 *   functional.triangle_multiplication(z, params, mask)        functional.py:7-26
 *   -> TriangleMultiplicativeUpdateKernelFused._forward_kernels _kernels.py:519-530
 * and the backend plug-in `execute(inp, params)`               backends/cuda_cute.py:38-39
 * Each entry point below names the reference code it replaces. Plain pointers and
 * sizes only; no framework types. All calls are asynchronous on `stream`, allocate
 * no memory and do not synchronise; the caller owns every buffer.
 *
 * Semantics follow the reference exactly: z is multiplied by the pair mask BEFORE the
 * input LayerNorm (functional.py:21-22), the output is multiplied by the mask again
 * (:25-26), residual=1 returns z*mask + delta (_kernels.py:547). Internal arithmetic is
 * fp16 storage with fp32 accumulation and fp32 LayerNorm statistics, as in the
 * reference's fp16 kernels (ops/triangle.py:39).
 */
#ifndef FAST_TRIMUL_B200_H
#define FAST_TRIMUL_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* ftm_stream_t; /* == cudaStream_t */

typedef enum {
  FTM_OK = 0,
  FTM_BAD_SHAPE = 1,        /* unsupported B/N/c_z/c_h (reference guard: context.py:41-55) */
  FTM_BAD_DTYPE = 2,
  FTM_BAD_ALIGN = 3,        /* a pointer is not 16-byte aligned */
  FTM_UNSUPPORTED_ARCH = 4, /* device is not sm_100 */
  FTM_LAUNCH_FAILED = 5,
  FTM_TIMEOUT = 6,          /* a bounded device-side wait expired (see ftm_check_error) */
  FTM_BAD_WORKSPACE = 7,    /* workspace missing or smaller than ftm_workspace_bytes() */
  FTM_BAD_ARGUMENT = 8
} ftm_status;

typedef enum { FTM_F32 = 0, FTM_F16 = 1, FTM_BF16 = 2 } ftm_dtype;
typedef enum { FTM_OUTGOING = 0, FTM_INCOMING = 1 } ftm_mode;

/* One forward problem. z is (batch, rows, cols, c_z) row-major; a full problem has
 * rows == cols == N. A row shard of an outgoing problem (multi-GPU) has rows = N/P. */
typedef struct {
  int32_t batch;     /* B */
  int32_t rows;      /* R: rows of z in this call */
  int32_t cols;      /* S: N */
  int32_t c_z;       /* pair channels (128) */
  int32_t c_h;       /* hidden channels (128) */
  int32_t mode;      /* ftm_mode */
  int32_t residual;  /* 1: z*mask + delta, 0: delta only */
  int32_t z_dtype;   /* FTM_F16 or FTM_BF16 (fp32 callers convert to fp16 first, as
                        functional.py:23 does) */
  int32_t out_dtype; /* FTM_F16, FTM_BF16 or FTM_F32 */
  float eps_in;      /* norm_in eps (nn.LayerNorm default 1e-5) */
  float eps_out;     /* norm_out eps */
} ftm_problem;

/* ---- parameters --------------------------------------------------------------
 * Replaces the per-call weight handling of _kernels.py:202-223 (`torch.cat` of the
 * [proj; gate] weights on every call) and KernelLinear's prebinding (:165-199):
 * parameters are packed once into a device buffer that all calls read.
 *
 * `params` holds 16 device pointers in the reference's _params() order
 * (_kernels.py:512-517): norm_in.{weight,bias}, norm_out.{weight,bias},
 * proj_a, gate_a, proj_b, gate_b, proj_g, proj_out as {weight (out x in), bias}.
 * param_dtype is FTM_F16 (the reference module is .half(), ops/triangle.py:39) or
 * FTM_F32. The LayerNorm affine is folded into the weights:
 *   LN(x) W^T + b = rstd*(x (W diag(gamma))^T - mean*rowsum(W diag(gamma))) + W beta + b. */
size_t ftm_packed_params_bytes(int32_t c_z, int32_t c_h);
int ftm_pack_params(const void* const params[16], int32_t param_dtype, int32_t c_z, int32_t c_h,
                    void* packed, ftm_stream_t stream);

/* ---- whole forward ----------------------------------------------------------
 * Replaces functional.triangle_multiplication -> _forward_kernels
 * (functional.py:7-26, _kernels.py:519-530). mask is (batch, rows, cols) fp32 or
 * NULL. out has z's shape in out_dtype. workspace: >= ftm_workspace_bytes(p),
 * 256-byte aligned (holds a, b, x in fp16 channel-major and the error word). */
size_t ftm_workspace_bytes(const ftm_problem* p);
int ftm_trimul_fwd(const ftm_problem* p, const void* z, const float* mask, const void* packed,
                   void* out, void* workspace, size_t workspace_bytes, ftm_stream_t stream);

/* ---- the three stages (for callers that interleave communication) -----------
 * Input stage: LayerNorm(z*mask) -> [a_p|a_g|b_p|b_g] projection on the tensor cores
 * -> sigmoid gating, written fp16 channel-major: a_cm[b][c][u][v] with (u,v) = (i,k)
 * for outgoing and (k,i) transposed for incoming, so the contraction always reads
 * K-major operands. Replaces layer_norm + _proj_gate + gate + permute copies
 * (_kernels.py:520-524, :138-139, :155-156). It also writes the LayerNorm statistics of
 * z*mask, zstats[(b*rows + r)*cols + s] = {mean, mask * rstd} (2 floats per position),
 * which the output stage reuses for its gate projection (the reference normalises z once,
 * _kernels.py:520, and reuses z_norm at :527). */
int ftm_input_stage(const ftm_problem* p, const void* z, const float* mask, const void* packed,
                    void* a_cm, void* b_cm, float* zstats, int* err_word, ftm_stream_t stream);

/* Contraction: for l in [0, L): X[l][i][j] = sum_k A[l][i][k] * B[l][j][k]
 * (fp16 in, fp32 accumulate, fp16 out). A is (L, m, k) row-major; B is stored as
 * `b_blocks` blocks of (L, b_rows_per_block, k), block-major (what an all-gather of
 * per-rank row shards produces), so B row j lives in block j / b_rows_per_block.
 * X is (L, m, n) with n = b_blocks * b_rows_per_block. Replaces outgoing()/incoming()
 * (_kernels.py:131-162). Requires k % 8 == 0 and, when b_blocks > 1,
 * b_rows_per_block % 128 == 0. */
int ftm_contraction(const void* A, const void* B, void* X, int32_t L, int32_t m, int32_t k,
                    int32_t b_rows_per_block, int32_t b_blocks, int* err_word,
                    ftm_stream_t stream);

/* Contraction with A (and X) given as row blocks too: A is `a_blocks` blocks of
 * (L, a_rows_per_block, k), X is written as `a_blocks` blocks of
 * (L, a_rows_per_block, n) -- the layouts an NCCL all-to-all between row shards and
 * channel shards produces and consumes. m = a_blocks * a_rows_per_block. Replaces
 * the same reference code as ftm_contraction (_kernels.py:131-162); requires
 * a_rows_per_block % 128 == 0 when a_blocks > 1. ftm_contraction is the a_blocks = 1 case. */
int ftm_contraction_blocked(const void* A, const void* B, void* X, int32_t L,
                            int32_t a_rows_per_block, int32_t a_blocks, int32_t k,
                            int32_t b_rows_per_block, int32_t b_blocks, int* err_word,
                            ftm_stream_t stream);

/* Contraction with the reduction index split into blocks:
 * X[l][i][j] = sum_k A[l][i][k] * B[l][j][k] with A stored as k_blocks blocks of
 * (L, m, k_rows_per_block) and B as k_blocks blocks of (L, n, k_rows_per_block) --
 * block q holding k in [q*k_rows_per_block, (q+1)*k_rows_per_block) -- and X written as
 * m / x_rows_per_block blocks of (L, x_rows_per_block, n). This is incoming mode's
 * contraction (_kernels.py:148-162) on channel shards gathered from row-sharded z
 * (each rank's transposed planes carry its own rows k). Requires k_rows_per_block % 64 == 0
 * and, when X has more than one block, x_rows_per_block % 256 == 0. */
int ftm_contraction_kblocked(const void* A, const void* B, void* X, int32_t L, int32_t m,
                             int32_t n, int32_t k_rows_per_block, int32_t k_blocks,
                             int32_t x_rows_per_block, int* err_word, ftm_stream_t stream);

/* General strided contraction -- the form the sharded forward uses for its partial
 * problems (one row owner's block, one source's columns, received channel shards):
 *   X[l][i][j] = sum_kk A[l][i][kk] * B[l][j][kk],  l < L, i < m, j < n, kk < k,
 * fp16 operands, fp32 accumulation, fp16 X, on the CTA-pair tensor-core kernel. Every
 * operand is described by element strides:
 *   A[l][i][kk] = a[(i / a_rows_per_block) * a_block_stride + l * a_l_stride
 *                   + (i % a_rows_per_block) * a_row_stride
 *                   + (kk / k_per_block) * a_kblock_stride + kk % k_per_block]
 *   B[l][j][kk] likewise with j and the b_* fields,
 *   X[l][i][j]  = x[(i / x_rows_per_block) * x_block_stride + l * x_l_stride
 *                   + (i % x_rows_per_block) * x_row_stride + j].
 * A rows-per-block or k_per_block of 0 (or >= the extent) means one block. Rules: 16-byte
 * aligned pointers; strides multiples of 8 elements (block strides may be 0 when there is
 * one block); n % 8 == 0; several row blocks need rows_per_block % 128 == 0 and the extent
 * a multiple of it; several k blocks need k_per_block % 64 == 0 and k a multiple of it.
 * With a_mn_major = 1, A is stored with its rows contiguous instead:
 *   A[l][i][kk] = a[l * a_l_stride + kk * a_row_stride + i]
 * (one row block, one k block; a_row_stride >= m); b_mn_major likewise for B. The
 * backward's products dA = dX B and dB = dX^T A read their operands this way.
 * Same reference code as ftm_contraction (_kernels.py:131-162). */
typedef struct {
  int32_t L, m, n, k;
  int32_t k_per_block;
  const void* a;
  int32_t a_rows_per_block;
  int64_t a_block_stride, a_l_stride, a_row_stride, a_kblock_stride;
  const void* b;
  int32_t b_rows_per_block;
  int64_t b_block_stride, b_l_stride, b_row_stride, b_kblock_stride;
  void* x;
  int32_t x_rows_per_block;
  int64_t x_block_stride, x_l_stride, x_row_stride;
  int32_t a_mn_major, b_mn_major;
} ftm_contraction_layout;
int ftm_contraction_general(const ftm_contraction_layout* layout, int* err_word,
                            ftm_stream_t stream);

/* Output stage: LayerNorm over c_h of x (channel-major fp16), the c_h -> c_z projection,
 * sigmoid(z_n W_g + b_g) gate, residual and mask, stored in out_dtype. Replaces
 * layer_norm + KernelLinear.raw x2 + gated_residual/gate + the mask/cast glue
 * (_kernels.py:526-530, functional.py:24-26). zstats: as written by ftm_input_stage. */
int ftm_output_stage(const ftm_problem* p, const void* z, const float* mask, const void* x_cm,
                     const float* zstats, const void* packed, void* out, int* err_word,
                     ftm_stream_t stream);

/* ---- row-sharded multi-GPU forward, exchange fused into the kernels ----------
 * No single counterpart in the reference (it has no multi-GPU path); this replaces
 * the all-to-all that moves the projections a, b from row shards to channel shards
 * and x back (the exchange around outgoing(), _kernels.py:131-146). With P ranks each
 * owning `rows` consecutive rows of z, rank q owns channels [q*c_h/P, (q+1)*c_h/P).
 * `base[q]` is rank q's receive plane as addressable from THIS GPU (a CUDA IPC or
 * peer mapping; base[rank] is local). The kernels write into the peers' planes over
 * NVLink themselves (TMA stores / stores from the epilogues); the caller orders the
 * phases with a barrier across ranks (all writes into a plane complete -- every
 * rank's kernel finished -- before its owner reads it). */
#define FTM_MAX_RANKS 8
typedef struct ftm_peer_planes {
  int32_t world;                   /* P, 1..FTM_MAX_RANKS, c_h % P == 0 */
  int32_t rank;                    /* this rank */
  void* base[FTM_MAX_RANKS];       /* receive plane of rank q (16-byte aligned) */
} ftm_peer_planes;

/* Input stage (as ftm_input_stage, p->rows = this rank's rows) whose a and b go
 * straight to the channel owners: rank q = c / (c_h/P) receives this rank's planes of
 * its channels at  base[q] + ((rank*B + b)*(c_h/P) + c%(c_h/P))*rows*cols  (fp16
 * elements) -- the receive layout [source rank][batch][c_h/P][plane]. The plane is
 * (rows, cols) [i][j] in outgoing mode and the transposed (cols, rows) [i][k] in incoming
 * mode, as ftm_input_stage writes them. zstats stay local. Requires (c_h/P) % 16 == 0. */
int ftm_input_stage_scatter(const ftm_problem* p, const void* z, const float* mask,
                            const void* packed, const ftm_peer_planes* a_dst,
                            const ftm_peer_planes* b_dst, float* zstats, int* err_word,
                            ftm_stream_t stream);

/* Contraction of this rank's channel shard over all n = P*rows rows (mode outgoing:
 * A, B are the row blocks of the receive layout above; incoming: the transposed planes,
 * so k is split by source rank), with every x row written straight to its row owner:
 * x[b][c][i][j] for c in this rank's channels, row i of owner o = i / rows, lands at
 * base[o] + ((b*c_h + c)*rows + i%rows)*n + j -- the owner's local channel-major x
 * plane (batch, c_h, rows, n), ready for ftm_output_stage. rows % 256 == 0. */
int ftm_contraction_scatter(const void* A, const void* B, const ftm_peer_planes* x_dst,
                            int32_t batch, int32_t c_h, int32_t rows, int32_t n, int32_t mode,
                            int* err_word, ftm_stream_t stream);

/* ---- per-position kernels of the training backward ---------------------------
 * Replace the elementwise and per-row parts of the autograd of the reference's
 * training path (_TrainableTriMul, _kernels.py:468-488, differentiating _torch_forward,
 * :532-547). c_z = c_h = 128. Positions p = (b*N + u)*N + v as rows of 128 channels;
 * planes [b][c][u][v]. H / dPGZ rows hold 640 fp16 columns [p_a g_a p_b g_b | g_z]
 * (GEMM results without biases / their gradients). Grids are fixed: partial-sum buffers
 * have ftm_bwd_partial_blocks() rows (256 floats: dgamma then dbeta per channel, or the
 * column sums of the gradient rows a kernel writes -- the bias gradients).
 * g_scale / dscale point to one device float: the factor applied to the output gradient
 * (the caller pre-scales it to unit magnitude) / to the da, db planes; passing them in
 * device memory lets the caller compute them without a host synchronisation. */
int ftm_bwd_partial_blocks(void);
/* zn = LayerNorm(z * mask) (fp16 rows), stats = (mean, rstd) per position */
int ftm_bwd_ln_in(const void* z, int32_t z_dtype, const float* mask, const float* gamma,
                  const float* beta, float eps, void* zn, float* stats, int64_t positions,
                  ftm_stream_t stream);
/* xn = LayerNorm(x) rows (fp16) and stats from the fp16 x plane */
int ftm_bwd_x_ln(const void* xplane, const float* gamma, const float* beta, float eps, void* xn,
                 float* stats, int32_t batch, int32_t n, ftm_stream_t stream);
/* output gate: dO = dout*m*sigmoid(gz), dPGZ[:, 512:640] = dout*m*o*sigmoid'(gz);
 * partial rows of 256: column sums of dO then of dgz */
int ftm_bwd_gate(const void* O, const float* b_o, const void* H, const float* b_g, const void* gout,
                 int32_t g_dtype, const float* g_scale, const float* mask, void* dO, void* dPGZ,
                 float* partial, int64_t positions, ftm_stream_t stream);
/* output LayerNorm backward: dx (fp32 plane) from dxn rows, partial dgamma / dbeta */
int ftm_bwd_x_ln_bwd(const void* xplane, const float* stats, const void* dxn, const float* gamma,
                     float* dxplane, float* partial, int32_t batch, int32_t n, ftm_stream_t stream);
/* input gates: dPGZ[:, 0:512] from da, db (fp16 planes in position order, x dscale);
 * partial rows of 512: column sums of dPGZ[:, 0:512] */
int ftm_bwd_gates_in(const void* dA, const void* dB, const float* dscale, const void* H, const float* b_in,
                     void* dPGZ, float* partial, int32_t batch, int32_t n, ftm_stream_t stream);
/* input LayerNorm backward (+ the residual path): dz, partial dgamma / dbeta */
int ftm_bwd_ln_in_bwd(const void* z, int32_t z_dtype, const float* mask, const float* stats,
                      const void* dzn, const float* gamma, const void* gout, int32_t g_dtype,
                      const float* g_scale, int32_t residual, void* dz, int32_t dz_dtype, float* partial,
                      int64_t positions, ftm_stream_t stream);

/* ---- row-sharded multi-GPU forward, native exchange pipeline ----------------
 * No counterpart in the reference (it has no multi-GPU path). P ranks, one GPU each,
 * rank r owning R = N / P consecutive rows of z and of the output. One call runs the
 * whole sharded forward of this rank on `stream`: the input stage in row_chunks
 * launches; copy-engine pushes of each chunk's pieces into the peers' receive windows
 * (CUDA IPC mappings) as soon as it is done, each followed by a flag raised in the
 * receiver's memory; bounded device-side waits on those flags; the contraction
 * (alltoall: this rank's channels for one row owner at a time, each owner's x block
 * pushed back as soon as it is done; allgather: own rows against each arriving chunk of
 * b); the output stage. No NCCL call and no host synchronisation on the data path.
 * Every rank must call ftm_shard_forward the same number of times; an expired wait is
 * reported through err_word (ftm_check_error), never by hanging.
 * Buffer sizes come from ftm_shard_buffer_bytes; recv_*, x_plane and flags are per rank
 * as mapped in this process (this rank's own entry is its local buffer); flags must be
 * zeroed before the first forward. The plan owns one copy stream and a few events (no
 * device memory). Requirements: rows % row_chunks == 0, rows / row_chunks % 128 == 0,
 * (128 / P) % 16 == 0 (P <= 8), row_chunks == 1 when batch > 1. */
#define FTM_SHARD_ALLTOALL 0
#define FTM_SHARD_ALLGATHER 1
#define FTM_SHARD_MAX_ROW_CHUNKS 8
#define FTM_SHARD_FLAG_WORDS 256
enum {
  FTM_SHARD_BUF_LOCAL = 0,   /* a_local: this rank's projections (alltoall: a and b), chunk-major */
  FTM_SHARD_BUF_ZSTATS = 1,  /* zstats */
  FTM_SHARD_BUF_XBLOCKS = 2, /* x_blocks: alltoall -- x per row owner; allgather -- x plane */
  FTM_SHARD_BUF_RECV = 3,    /* each receive window (two slots; alltoall: a and b in recv_a) */
  FTM_SHARD_BUF_XPLANE = 4,  /* each x plane (alltoall) */
  FTM_SHARD_BUF_FLAGS = 5    /* each flag buffer */
};
typedef struct {
  int32_t world, rank;
  int32_t scheme;       /* FTM_SHARD_ALLTOALL (both modes) or FTM_SHARD_ALLGATHER (outgoing) */
  int32_t row_chunks;   /* 1..FTM_SHARD_MAX_ROW_CHUNKS */
  ftm_problem shard;    /* this rank's rows: rows = N / world, cols = N */
  const void* packed;
  void* a_local;
  float* zstats;
  void* x_blocks;
  int* err_word;
  void* recv_a[FTM_MAX_RANKS];   /* alltoall: a and b arrive here */
  void* recv_b[FTM_MAX_RANKS];   /* allgather: b of every rank arrives here */
  void* x_plane[FTM_MAX_RANKS];  /* alltoall only */
  int* flags[FTM_MAX_RANKS];
} ftm_shard_config;
typedef struct ftm_shard_plan ftm_shard_plan;
size_t ftm_shard_buffer_bytes(const ftm_shard_config* cfg, int which);
int ftm_shard_plan_create(const ftm_shard_config* cfg, ftm_shard_plan** plan);
/* out_dtype: FTM_F16, FTM_BF16 or FTM_F32 (shard.out_dtype is the default a caller
 * normally passes). */
int ftm_shard_forward(ftm_shard_plan* plan, const void* z, const float* mask, void* out,
                      int32_t out_dtype, ftm_stream_t stream);
void ftm_shard_plan_destroy(ftm_shard_plan* plan);
/* Optional timeline of the following forwards (for profiling): `trace` is a device buffer
 * of 2 * FTM_SHARD_TRACE_POINTS int64; each forward overwrites it with (device clock ns,
 * tag) pairs taken when the work queued before each point has finished -- tag =
 * (what << 8) | index, what: 1 start, 2 input chunk done, 3 chunk pushed to a peer,
 * 4 data ready, 5 contraction done, 6 x pushed, 7 x ready, 8 output done. The extra
 * one-thread kernels cost a few microseconds each. NULL turns it off. */
#define FTM_SHARD_TRACE_POINTS 128
int ftm_shard_set_trace(ftm_shard_plan* plan, long long* trace);

/* ---- whole forward with no allocation ---------------------------------------
 * No counterpart in the reference. For callers that cannot provide a workspace --
 * hosts with a fixed device-memory budget handed out at start-up, or hosts that may
 * not call cudaMalloc while running because it can synchronise the device. Same
 * arguments and results as ftm_trimul_fwd, but a, b, x and the error word live in a
 * device array built into the library (about 48.5 MiB, held by each GPU that loads the
 * library until exit). Problems with batch*rows*cols > FTM_STATIC_SCRATCH_MAX_POSITIONS
 * return FTM_BAD_WORKSPACE. All calls on a device share that array: calls that overlap
 * on the GPU race and must be serialised. The first call on each device looks up the
 * array's device address; make it before any stream capture. Allocates nothing. */
#define FTM_STATIC_SCRATCH_MAX_POSITIONS 65536
int ftm_trimul_fwd_static_scratch(const ftm_problem* p, const void* z, const float* mask,
                                  const void* packed, void* out, ftm_stream_t stream);
/* The current device's error word inside that array (NULL if its address cannot be
 * looked up), for ftm_check_error after ftm_trimul_fwd_static_scratch calls: the word
 * is cleared at the start of each call, so check it before the next call. No
 * counterpart in the reference. */
int* ftm_static_scratch_error_word(void);

/* ---- status -------------------------------------------------------------- */
/* Synchronise `stream`, read the device error word of a workspace (or any err_word
 * passed to a stage) and clear it: FTM_OK, or FTM_TIMEOUT when a bounded device wait
 * expired (the failing kernel/role/site is stored in *detail when non-NULL). */
int ftm_check_error(const int* err_word, int* detail, ftm_stream_t stream);
/* Address of the error word inside a workspace laid out for `p`. */
int* ftm_workspace_error_word(const ftm_problem* p, void* workspace);
const char* ftm_status_string(int status);
/* 1 if `device` is an sm_100 GPU these kernels run on, else 0. */
int ftm_device_supported(int device);
/* Number of kernels the last successful ftm_trimul_fwd / stage call launched. */
int ftm_last_launch_count(void);

#ifdef __cplusplus
}
#endif
#endif /* FAST_TRIMUL_B200_H */
