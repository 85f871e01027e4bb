/*
 * pdb.h -- C ABI of the pdum_dsl_b200 kernel library (sm_100a).
 *
 * The reference (pdum.dsl / pdum.tl) lowers the tile regions produced by its
 * fusion templates through one Python entry point,
 *     compile_tile(region, launch=(), prune=()) -> run(values)
 * (conformance/triton_tile.py:662-698), which JIT-generates Triton source per
 * region.  This library replaces that lowering for the templates on the hot
 * path with fixed, hand-written CUDA kernels.  Each entry point below stands
 * for one template row of the reference registry (packages/tensorlib/src/
 * pdum/tl/fusion.py:762-868) and is what a reference-side binding (ctypes, a
 * torch custom op, or a C caller) would call.
 *
 * Conventions shared by every entry point:
 *   - all pointers are DEVICE pointers owned by the caller; the library never
 *     allocates or frees caller memory (workspace, when needed, is sized by a
 *     *_workspace_size query and passed in);
 *   - sizes and strides are int64 element counts (not bytes);
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default);
 *   - launches are asynchronous; the return value reports argument / launch
 *     errors only.  Device-side bounded waits that expire set a flag that
 *     pdb_check_error() reads back (PDB_ERR_TIMEOUT);
 *   - calls are stateless and re-entrant; the only global state is a lazily
 *     built, mutex-guarded per-device attribute cache.
 */
#ifndef PDB_H_
#define PDB_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum pdb_status {
  PDB_OK = 0,
  PDB_ERR_SHAPE = 1,        /* sizes / strides the kernel family cannot take   */
  PDB_ERR_ALIGN = 2,        /* pointer or stride alignment (TMA: 16 B)         */
  PDB_ERR_TIMEOUT = 3,      /* a bounded device wait expired (see check_error)  */
  PDB_ERR_CUDA = 4,         /* a CUDA runtime / driver call failed              */
  PDB_ERR_UNSUPPORTED = 5,  /* dtype / head-dim combination not built           */
  PDB_ERR_ARG = 6           /* null descriptor or required pointer              */
};

enum pdb_dtype { PDB_F32 = 0, PDB_BF16 = 1 };

/* ---- row-normalization: softmax over the last dim --------------------------
 * Replaces the "row-normalization" template (fusion.py:371-400, :818-826) as
 * lowered by compile_tile (triton_tile.py:662).  y[r, c] = exp(x[r,c] - max_c
 * x[r,:]) / sum_c exp(...).  f32 in / f32 out. */
typedef struct {
  const float* x;
  float* y;
  int64_t rows, cols;
  int64_t x_row_stride, y_row_stride; /* elements; the column stride is 1 */
} pdb_rowsoftmax_desc;
int pdb_rowsoftmax_f32(const pdb_rowsoftmax_desc* d, void* stream);

/* ---- row-statistics: two-pass layernorm over the last dim -------------------
 * Replaces the "row-statistics" template (fusion.py:403-443, :827-843;
 * zoo_common.py:56-60): y = (x - mean) / sqrt(mean((x - mean)^2) + eps) *
 * gamma + beta.  gamma / beta may be NULL (identity scale / zero shift). */
typedef struct {
  const float* x;
  const float* gamma;
  const float* beta;
  float* y;
  int64_t rows, cols;
  int64_t x_row_stride, y_row_stride;
  double eps;
} pdb_layernorm_desc;
int pdb_layernorm_f32(const pdb_layernorm_desc* d, void* stream);

/* ---- flash attention ---------------------------------------------------------
 * Replaces the "flash" template (fusion.py:480-615) and its widened rows
 * (batch/head riders, score scale, no mask, GQA).  Logical shapes:
 *   q [batch, heads_q,  seqlen_q, head_dim]     o [batch, heads_q, seqlen_q, head_dim_v]
 *   k [batch, heads_kv, seqlen_k, head_dim]     v [batch, heads_kv, seqlen_k, head_dim_v]
 * with heads_q = heads_kv * group (GQA: query head h reads KV head h / group).
 * Strides are per (batch, head, row); the innermost (feature) stride is 1.
 * Scores are scale * q.k; with `causal`, key s is visible to query row t iff
 * s <= t + q_start (absolute coordinates: the reference's iota mask
 * `le(iota(s), iota(t))`, dialect.py:1382-1383).  Optional per-row outputs
 * (float32, [batch, heads_q, seqlen_q] contiguous):
 *   lse = log(sum_s exp(score)),   m = max_s score,   den = sum_s exp(score - m)
 * -- m / den are the template's artifact finals (fusion.py:611-613).
 * General closed masks (the reference plans any closed iota mask forest as
 * flash, fusion.py:468-477,521, and prunes it per program, :659-690): with
 * key_lo / key_hi set (device int32 arrays of seqlen_q entries, `causal`
 * must be 0), query row t sees exactly the keys s with key_lo[t] <= s <
 * key_hi[t] (absolute key indices; the host evaluates the mask and checks
 * each row's visible keys form one non-empty run).  When key_lo and key_hi
 * are both nondecreasing in t, set mask_monotone: the kernels then visit, per
 * block of query rows, only the key tiles between the block's first row's
 * key_lo and its last row's key_hi; otherwise every key tile is visited and
 * the per-row bounds alone mask.
 * dtype PDB_BF16: bf16 q/k/v/o, fp32 accumulate, tcgen05/TMEM tensor cores
 * (head_dim, head_dim_v multiples of 8 up to 256, possibly different: the
 * kernels are built for 64, 128 and 256 features and the tensor maps zero-fill
 * the columns past each dim).  dtype PDB_F32: f32 everything, ieee
 * FMA path (any head_dim, head_dim_v <= 256), the precision of the reference's
 * f32 column (triton_tile.py:684-690 refuses tf32). */
typedef struct {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  float* lse; /* nullable */
  float* m;   /* nullable */
  float* den; /* nullable */
  int64_t batch, heads_q, heads_kv, seqlen_q, seqlen_k, head_dim, head_dim_v;
  int64_t q_stride[3], k_stride[3], v_stride[3], o_stride[3]; /* (b, h, row) */
  int64_t q_start;
  double scale;
  int32_t causal;
  int32_t dtype; /* enum pdb_dtype */
  const int32_t* key_lo; /* nullable: per query row, first visible key */
  const int32_t* key_hi; /* per query row, one past the last visible key */
  int32_t mask_monotone;
  int32_t sm_margin; /* bf16 path: SMs the persistent grid leaves free (e.g. for a collective
                        that overlaps this launch); 0 = use every SM */
} pdb_flash_desc;
int pdb_flash_fwd(const pdb_flash_desc* d, void* stream);

/* ---- flash attention backward ----------------------------------------------
 * The joint forward+backward region that autodiff.grad builds from the naive
 * attention region (autodiff.py:102-150) and plan_model carves
 * (partition.py:586-607): given q, k, v, o, dO and the forward's lse,
 *   P = exp(scale*q.k - lse),  D = rowsum(dO * o)        ("held-back D")
 *   dV = P^T dO,  dS = P * (dO.V^T - D),  dQ = scale * dS K,  dK = scale * dS^T Q.
 * dq/dk/dv share the layouts of q/k/v (GQA: dk/dv are summed over the group).
 * Workspace (float32) holds D and, for head_dim 64, the dQ accumulator; its
 * size in bytes comes from pdb_flash_bwd_workspace_size.  If lse is NULL the
 * kernel recomputes it (the "recompute" variant of the template); otherwise it
 * is the forward's stored lse ("stored" variant).  head_dim and head_dim_v
 * are multiples of 8 up to 128 and may differ.  Both <= 64
 * runs one fused pass whose dQ sums per-key-block parts with fp32 reductions in
 * L2, so dq's last bits may differ run to run; every other shape runs the
 * 128-wide dK/dV and dQ passes, with tensor maps that zero-fill the features
 * past each dim (reproducible).  Other dims return PDB_ERR_SHAPE. */
typedef struct {
  const void* q;
  const void* k;
  const void* v;
  const void* o;
  const void* dout;
  const float* lse; /* nullable: recompute */
  void* dq;
  void* dk;
  void* dv;
  void* workspace;
  size_t workspace_bytes;
  int64_t batch, heads_q, heads_kv, seqlen_q, seqlen_k, head_dim, head_dim_v;
  int64_t q_stride[3], k_stride[3], v_stride[3], o_stride[3], do_stride[3];
  int64_t dq_stride[3], dk_stride[3], dv_stride[3];
  int64_t q_start;
  double scale;
  int32_t causal;
  int32_t dtype;
} pdb_flash_bwd_desc;
size_t pdb_flash_bwd_workspace_size(const pdb_flash_bwd_desc* d);
int pdb_flash_bwd(const pdb_flash_bwd_desc* d, void* stream);

/* ---- flash attention backward without caller workspace ----------------------
 * No counterpart in the reference.  For callers that cannot allocate device
 * memory when they call (a pool or arena owns the device, or a plain C
 * caller has no allocator): same descriptor and results as pdb_flash_bwd, but
 * `workspace` / `workspace_bytes` are ignored and the scratch comes from a
 * fixed 16 MiB array inside the library, held on every device that loads it.
 * Problems whose scratch (pdb_flash_bwd_workspace_size) exceeds
 * pdb_flash_bwd_noalloc_max_scratch() are refused with PDB_ERR_SHAPE.  The
 * first call on a device looks up the array's address (make it before any
 * stream capture) and keeps it for the life of the process, so a device reset
 * (cudaDeviceReset, or destroying the primary context) invalidates it: do not
 * call this entry point on a device after resetting it.  Calls that may
 * overlap on the GPU share the array and race, so the caller must order them.
 * Nothing is allocated or freed. */
int pdb_flash_bwd_noalloc(const pdb_flash_bwd_desc* d, void* stream);
size_t pdb_flash_bwd_noalloc_max_scratch(void);

/* ---- contraction-epilogue and map-chain templates ---------------------------
 * Replace the "contraction-epilogue" template (fusion.py:159-324: a sum over
 * one contracted dim of a product of two operands, with an absorbed pointwise
 * epilogue) and the "map-chain" template (a pure pointwise chain) as
 * compile_tile lowers them (triton_tile.py:471-546).  The epilogue is a short
 * program of pointwise steps applied to each accumulator element (or, for
 * pdb_pointwise_f32, to each input element):
 *   value = op(value)              (unary: exp, log, sqrt, tanh, neg)
 *   value = op(value, operand)     (binary; swap = 1 gives op(operand, value))
 * where the operand is a constant or a float32 tensor read at the element's
 * (batch, m, n) coordinate through three element strides (0 broadcasts). */
enum pdb_ew_opcode {
  PDB_EW_ADD = 1, PDB_EW_SUB, PDB_EW_MUL, PDB_EW_DIV, PDB_EW_MAX, PDB_EW_MIN,
  PDB_EW_EXP, PDB_EW_LOG, PDB_EW_SQRT, PDB_EW_TANH, PDB_EW_NEG
};
#define PDB_MAX_EW_OPS 8
typedef struct {
  int32_t op;       /* enum pdb_ew_opcode */
  int32_t operand;  /* 0 none (unary), 1 constant, 2 tensor */
  int32_t swap;
  int32_t reserved;
  double value;
  const float* ptr;
  int64_t stride[3]; /* (batch, m, n) */
} pdb_ew_op;

/* c[b, m, n] = epilogue(alpha * sum_k a[b, m, k] * b[b, n, k]).
 * dtype PDB_F32: f32 operands / output, IEEE FMA (the reference's f32 column);
 * dtype PDB_BF16: bf16 operands with k contiguous (TMA, 16-byte rows), fp32
 * accumulate in TMEM (tcgen05), f32 epilogue, bf16 output. */
typedef struct {
  const void* a;
  const void* b;
  void* c;
  int64_t batch, m, n, k;
  int64_t a_stride[3]; /* (batch, m, k) */
  int64_t b_stride[3]; /* (batch, n, k) */
  int64_t c_stride[3]; /* (batch, m, n) */
  double alpha;
  int32_t dtype;
  int32_t n_ops;
  pdb_ew_op ops[PDB_MAX_EW_OPS];
} pdb_contract_desc;
int pdb_contract(const pdb_contract_desc* d, void* stream);

/* y[b, m, n] = epilogue(x[b, m, n]), f32 (map-chain template; also the
 * materialised prologue of a computed contraction operand). */
typedef struct {
  const float* x;
  float* y;
  int64_t batch, m, n;
  int64_t x_stride[3], y_stride[3];
  int32_t n_ops;
  int32_t reserved;
  pdb_ew_op ops[PDB_MAX_EW_OPS];
} pdb_pointwise_desc;
int pdb_pointwise_f32(const pdb_pointwise_desc* d, void* stream);

/* ---- score-space programs (the carves of the attention backward) ------------
 * Replaces, for the carves of the autodiff joint of attention that plan_model
 * produces (partition.py:586-607) and that the reference serves with its
 * contraction-epilogue row (fusion.py:159-324) or with run_region (red
 * groups, fusion.py:855-868), the lowering compile_tile would give them: a
 * carve that re-derives the probabilities from q, k and the forward's row
 * statistics and evaluates a pointwise expression over the score space.
 *
 * Index space: rows t < rows, columns s < cols (either of the carve's two
 * score dims may be the row dim), times batch x batch_mid x batch_inner
 * independent instances (up to three rider dims, e.g. batch, KV head and the
 * query heads of a GQA group; an operand without a rider has stride 0 along it).  Per element (t, s) a program of SSA steps
 * runs over float registers (booleans are 1.0 / 0.0); its step kinds are
 *   SCORE   dst = sum_f A_a[t, f] * B_a[s, f]        (score contraction a)
 *   ROW     dst = rowvec[a][t],  COL  dst = colvec[a][s]
 *   TILE    dst = tile[a][t, s]
 *   IOTA_ROW / IOTA_COL  dst = absolute coordinate (t + row_start / s + col_start)
 *   CONST   dst = value
 *   binary  dst = op(R[a], R[b]);  unary dst = op(R[a]);  WHERE dst = R[a] ? R[b] : R[c]
 * and the value in register `result` is stored per out_mode:
 *   OUT_TILE          out[b, t, s]
 *   OUT_ROW_SUM/MAX/MIN  out[b, t] = reduce over s
 *   OUT_ROW_CONTRACT  out[b, t, x] = sum_s V[t, s] * w[b, s, x]   (x < xdim)
 * (b standing for the three rider indices).  f32 throughout (IEEE FMA, the
 * precision of the reference's f32 column).  Every stride is an element count
 * and the strides of each operand start with its three rider strides; no
 * contiguity is required.  Row sums and row contractions of jobs with few row
 * blocks split the columns over several CTAs and add the partial results
 * atomically, so their f32 summation order varies from run to run. */
enum pdb_sp_opcode {
  PDB_SP_SCORE = 1, PDB_SP_ROW, PDB_SP_COL, PDB_SP_TILE, PDB_SP_IOTA_ROW, PDB_SP_IOTA_COL, PDB_SP_CONST,
  PDB_SP_WHERE,
  /* binary */
  PDB_SP_ADD, PDB_SP_SUB, PDB_SP_MUL, PDB_SP_DIV, PDB_SP_MAX, PDB_SP_MIN, PDB_SP_LE, PDB_SP_LT, PDB_SP_GE,
  PDB_SP_GT, PDB_SP_EQ, PDB_SP_NE, PDB_SP_AND, PDB_SP_OR,
  /* unary */
  PDB_SP_EXP, PDB_SP_LOG, PDB_SP_NEG, PDB_SP_RECIP, PDB_SP_SQRT, PDB_SP_TANH, PDB_SP_NOT, PDB_SP_ABS,
  PDB_SP_FLOOR
};
enum pdb_sp_out_mode {
  PDB_SP_OUT_TILE = 0, PDB_SP_OUT_ROW_SUM, PDB_SP_OUT_ROW_MAX, PDB_SP_OUT_ROW_MIN, PDB_SP_OUT_ROW_CONTRACT
};
#define PDB_SP_MAX_OPS 64
#define PDB_SP_MAX_REGS 12
#define PDB_SP_MAX_SCORES 2
#define PDB_SP_MAX_VECS 6
#define PDB_SP_MAX_TILES 4
typedef struct {
  int32_t op; /* enum pdb_sp_opcode */
  int32_t dst, a, b, c;
  int32_t reserved;
  double value;
} pdb_sp_op;
typedef struct {
  int64_t batch, batch_mid, batch_inner, rows, cols;
  int64_t row_start, col_start;
  int32_t n_scores, n_ops, n_regs, result;
  const float* score_a[PDB_SP_MAX_SCORES];
  const float* score_b[PDB_SP_MAX_SCORES];
  int64_t score_feat[PDB_SP_MAX_SCORES];
  int64_t score_a_stride[PDB_SP_MAX_SCORES][5]; /* (3 riders, row, feature) */
  int64_t score_b_stride[PDB_SP_MAX_SCORES][5]; /* (3 riders, col, feature) */
  const float* rowvec[PDB_SP_MAX_VECS];
  int64_t rowvec_stride[PDB_SP_MAX_VECS][4]; /* (3 riders, row) */
  const float* colvec[PDB_SP_MAX_VECS];
  int64_t colvec_stride[PDB_SP_MAX_VECS][4]; /* (3 riders, col) */
  const float* tile[PDB_SP_MAX_TILES];
  int64_t tile_stride[PDB_SP_MAX_TILES][5]; /* (3 riders, row, col) */
  pdb_sp_op ops[PDB_SP_MAX_OPS];
  int32_t out_mode; /* enum pdb_sp_out_mode */
  int32_t reserved;
  float* out;
  int64_t out_stride[5]; /* (3 riders, row, col | x); ROW_*: the last is unused */
  const float* w;
  int64_t w_stride[5]; /* (3 riders, col, x) */
  int64_t xdim;
} pdb_score_program_desc;
int pdb_score_program_f32(const pdb_score_program_desc* d, void* stream);

/* ---- status --------------------------------------------------------------------
 * pdb_check_error synchronises `stream`, reads and clears the device error flag
 * of the current device (set by bounded waits that expired; its address is
 * looked up once per device and, like the no-alloc scratch, is invalidated by
 * a device reset) and returns
 * PDB_ERR_TIMEOUT if it was set, PDB_ERR_CUDA on a CUDA error, else PDB_OK.
 * pdb_last_error_string returns a thread-local description of the last non-OK
 * status returned on this thread.  pdb_version returns a constant string that
 * keys compiled kernels (the backend fingerprint, registry.py:56-70). */
int pdb_check_error(void* stream);
/* Exercises the failure path of the bounded device waits: launches one
 * thread that waits on a barrier phase that never completes, gives up after
 * limit_ns (<= 2 s) and sets the device error word, so that the next
 * pdb_check_error(stream) returns PDB_ERR_TIMEOUT and clears it.  No fault,
 * no trap; the context stays usable.  (Host-side check of the reference's
 * refusal discipline, fusion.py:855-868; there is no device counterpart.) */
int pdb_selftest_wait_timeout(int64_t limit_ns, void* stream);
const char* pdb_last_error_string(void);
const char* pdb_version(void);

#ifdef __cplusplus
}
#endif
#endif /* PDB_H_ */
