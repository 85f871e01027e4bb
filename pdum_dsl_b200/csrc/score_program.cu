// Score-space programs: the carves of the attention backward that re-derive
// the probabilities inside the carve.
//
// plan_model (packages/tensorlib/src/pdum/tl/partition.py:586-607) carves the
// joint region that autodiff.grad builds from the naive attention region into
// flash-with-artifacts plus contraction carves (fusion.py:159-324).  Several of
// those carves are not plain GEMMs: they recompute P = exp(where(mask, q.k, fill)
// - m) / den from q, k and the forward's row statistics, evaluate a pointwise
// expression over the (t, s) score space (the derivative markers of autodiff,
// e.g. div.d1, exp.d0, where.d1), and then either store the (t, s) tile, reduce
// it over s (the D-rowsum and den-grad statistics), or contract it with a
// matrix over s (dV^T = P^T dO read as a contraction over t of the transposed
// space).  The host compiles such a carve into one program of SSA steps; this
// kernel runs it.
//
// Layout: one CTA owns 64 rows of the program space and walks its columns in
// 32-column tiles (all of them, or -- for sum outputs of a job with few row
// blocks -- a contiguous share, the shares' partial sums added atomically).  The per-element values live in a shared-memory register
// file R[reg][64 * 32] (element e = row * 32 + col; thread tid owns elements
// tid + 256 i, i < 8, so each warp owns whole 32-column rows and every global
// tile access is a coalesced 128-byte row).  Score contractions C[t, s] =
// sum_f A[t, f] B[s, f] are computed cooperatively (f staged 32 at a time,
// 2 x 4 outputs per thread, IEEE FMA) straight into their register slot.
// Output stages: store the tile; reduce each row (sum / max / min, warp
// shuffles, kept in registers across column tiles); or accumulate
// out[t, x] += sum_s V[t, s] W[s, x] for x < 128 (4 x 8 outputs per thread).
#include <cfloat>
#include <cmath>

#include "common.cuh"

namespace pdb {
namespace {

constexpr int SP_ROWS = 64, SP_COLS = 32, SP_THREADS = 256, SP_EPT = SP_ROWS * SP_COLS / SP_THREADS;  // 8
constexpr int SP_FK = 32;   // feature chunk of a score contraction
constexpr int SP_XMAX = 128;  // contraction-output columns per launch

struct SpParams {
  pdb_score_program_desc d;
  int csplit;  // CTAs per row block along the columns (sum outputs then combine with atomicAdd)
};

__device__ __forceinline__ float sp_apply1(int op, float a) {
  switch (op) {
    case PDB_SP_EXP: return expf(a);
    case PDB_SP_LOG: return logf(a);
    case PDB_SP_NEG: return -a;
    case PDB_SP_RECIP: return 1.0f / a;
    case PDB_SP_SQRT: return sqrtf(a);
    case PDB_SP_TANH: return tanhf(a);
    case PDB_SP_NOT: return a != 0.f ? 0.f : 1.f;
    case PDB_SP_ABS: return fabsf(a);
    case PDB_SP_FLOOR: return floorf(a);
    default: return a;
  }
}

__device__ __forceinline__ float sp_apply2(int op, float a, float b) {
  switch (op) {
    case PDB_SP_ADD: return a + b;
    case PDB_SP_SUB: return a - b;
    case PDB_SP_MUL: return a * b;
    case PDB_SP_DIV: return a / b;
    case PDB_SP_MAX: return fmaxf(a, b);
    case PDB_SP_MIN: return fminf(a, b);
    case PDB_SP_LE: return a <= b ? 1.f : 0.f;
    case PDB_SP_LT: return a < b ? 1.f : 0.f;
    case PDB_SP_GE: return a >= b ? 1.f : 0.f;
    case PDB_SP_GT: return a > b ? 1.f : 0.f;
    case PDB_SP_EQ: return a == b ? 1.f : 0.f;
    case PDB_SP_NE: return a != b ? 1.f : 0.f;
    case PDB_SP_AND: return (a != 0.f && b != 0.f) ? 1.f : 0.f;
    case PDB_SP_OR: return (a != 0.f || b != 0.f) ? 1.f : 0.f;
    default: return a;
  }
}

__device__ __forceinline__ float reduce_identity(int mode) {
  return mode == PDB_SP_OUT_ROW_MAX ? -INFINITY : (mode == PDB_SP_OUT_ROW_MIN ? INFINITY : 0.f);
}
__device__ __forceinline__ float reduce_combine(int mode, float a, float b) {
  return mode == PDB_SP_OUT_ROW_MAX ? fmaxf(a, b) : (mode == PDB_SP_OUT_ROW_MIN ? fminf(a, b) : a + b);
}

// One score contraction C[t0 + r, s0 + c] = sum_f A[t, f] B[s, f] into R[dst].
// offset of the CTA's rider instance (r0, r1, r2) along an operand's first three strides
__device__ __forceinline__ int64_t rider_off(const int64_t* st, int64_t r0, int64_t r1, int64_t r2) {
  return r0 * st[0] + r1 * st[1] + r2 * st[2];
}

__device__ void sp_score(const pdb_score_program_desc& d, int c, int64_t r0, int64_t r1, int64_t r2, int64_t t0,
                         int64_t s0, float* Rd, float (*As)[SP_ROWS + 1], float (*Bs)[SP_COLS + 1]) {
  const int tid = threadIdx.x;
  const int tr = tid >> 3, tc = tid & 7;  // rows 2 tr, 2 tr + 1; cols tc + 8 j
  const float* A = d.score_a[c] + rider_off(d.score_a_stride[c], r0, r1, r2);
  const float* B = d.score_b[c] + rider_off(d.score_b_stride[c], r0, r1, r2);
  const int64_t F = d.score_feat[c];
  float acc[2][4] = {};
  for (int64_t f0 = 0; f0 < F; f0 += SP_FK) {
    for (int e = tid; e < SP_ROWS * SP_FK; e += SP_THREADS) {
      const int r = e / SP_FK, kk = e % SP_FK;
      const int64_t gt = t0 + r, gf = f0 + kk;
      As[kk][r] = (gt < d.rows && gf < F) ? A[gt * d.score_a_stride[c][3] + gf * d.score_a_stride[c][4]] : 0.f;
    }
    for (int e = tid; e < SP_COLS * SP_FK; e += SP_THREADS) {
      const int r = e / SP_FK, kk = e % SP_FK;
      const int64_t gs = s0 + r, gf = f0 + kk;
      Bs[kk][r] = (gs < d.cols && gf < F) ? B[gs * d.score_b_stride[c][3] + gf * d.score_b_stride[c][4]] : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < SP_FK; ++kk) {
      const float a0 = As[kk][2 * tr], a1 = As[kk][2 * tr + 1];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float b = Bs[kk][tc + 8 * j];
        acc[0][j] = fmaf(a0, b, acc[0][j]);
        acc[1][j] = fmaf(a1, b, acc[1][j]);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int u = 0; u < 2; ++u)
#pragma unroll
    for (int j = 0; j < 4; ++j) Rd[(2 * tr + u) * SP_COLS + tc + 8 * j] = acc[u][j];
  __syncthreads();
}

__global__ void __launch_bounds__(SP_THREADS) score_program_kernel(const __grid_constant__ SpParams P) {
  extern __shared__ float4 sp_smem4[];
  float* smem = reinterpret_cast<float*>(sp_smem4);
  const pdb_score_program_desc& d = P.d;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // the three rider indices of this CTA's instance
  const int64_t r2 = blockIdx.y % d.batch_inner, r1 = (blockIdx.y / d.batch_inner) % d.batch_mid,
                r0 = blockIdx.y / (d.batch_inner * d.batch_mid);
  const int64_t t0 = (int64_t)blockIdx.x * SP_ROWS;
  // this CTA's column tiles [c_lo, c_hi) of the row block
  const int64_t ntiles = (d.cols + SP_COLS - 1) / SP_COLS;
  const int64_t c_lo = ntiles * blockIdx.z / P.csplit, c_hi = ntiles * (blockIdx.z + 1) / P.csplit;
  const bool atomic_out = P.csplit > 1;
  // shared memory: register file, contraction staging, W staging
  float* R = smem;                                                   // n_regs x 2048
  float(*As)[SP_ROWS + 1] = reinterpret_cast<float(*)[SP_ROWS + 1]>(R + d.n_regs * SP_ROWS * SP_COLS);
  float(*Bs)[SP_COLS + 1] = reinterpret_cast<float(*)[SP_COLS + 1]>(&As[SP_FK][0]);
  float* Ws = &Bs[SP_FK][0];  // SP_COLS x SP_XMAX
  const int mode = d.out_mode;

  float red[SP_EPT];
#pragma unroll
  for (int i = 0; i < SP_EPT; ++i) red[i] = reduce_identity(mode);
  float acc[4][8];
#pragma unroll
  for (int u = 0; u < 4; ++u)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[u][j] = 0.f;

  for (int64_t s0 = c_lo * SP_COLS; s0 < c_hi * SP_COLS; s0 += SP_COLS) {
    for (int k = 0; k < d.n_ops; ++k) {
      const pdb_sp_op& o = d.ops[k];
      float* Rd = R + o.dst * (SP_ROWS * SP_COLS);
      if (o.op == PDB_SP_SCORE) {
        sp_score(d, o.a, r0, r1, r2, t0, s0, Rd, As, Bs);
        continue;
      }
      const float* Ra = R + o.a * (SP_ROWS * SP_COLS);
      const float* Rb = R + o.b * (SP_ROWS * SP_COLS);
      const float* Rc = R + o.c * (SP_ROWS * SP_COLS);
#pragma unroll
      for (int i = 0; i < SP_EPT; ++i) {
        const int e = tid + SP_THREADS * i;
        const int64_t t = t0 + e / SP_COLS, s = s0 + e % SP_COLS;
        const bool in = t < d.rows && s < d.cols;
        float v;
        switch (o.op) {
          case PDB_SP_CONST: v = (float)o.value; break;
          case PDB_SP_IOTA_ROW: v = (float)(t + d.row_start); break;
          case PDB_SP_IOTA_COL: v = (float)(s + d.col_start); break;
          case PDB_SP_ROW:
            v = in ? d.rowvec[o.a][rider_off(d.rowvec_stride[o.a], r0, r1, r2) + t * d.rowvec_stride[o.a][3]] : 0.f;
            break;
          case PDB_SP_COL:
            v = in ? d.colvec[o.a][rider_off(d.colvec_stride[o.a], r0, r1, r2) + s * d.colvec_stride[o.a][3]] : 0.f;
            break;
          case PDB_SP_TILE:
            v = in ? d.tile[o.a][rider_off(d.tile_stride[o.a], r0, r1, r2) + t * d.tile_stride[o.a][3] +
                                 s * d.tile_stride[o.a][4]]
                   : 0.f;
            break;
          case PDB_SP_WHERE: v = Ra[e] != 0.f ? Rb[e] : Rc[e]; break;
          default:
            v = o.op >= PDB_SP_EXP ? sp_apply1(o.op, Ra[e]) : sp_apply2(o.op, Ra[e], Rb[e]);
            break;
        }
        Rd[e] = v;
      }
    }
    const float* V = R + d.result * (SP_ROWS * SP_COLS);
    if (mode == PDB_SP_OUT_TILE) {
#pragma unroll
      for (int i = 0; i < SP_EPT; ++i) {
        const int e = tid + SP_THREADS * i;
        const int64_t t = t0 + e / SP_COLS, s = s0 + e % SP_COLS;
        if (t < d.rows && s < d.cols)
          d.out[rider_off(d.out_stride, r0, r1, r2) + t * d.out_stride[3] + s * d.out_stride[4]] = V[e];
      }
    } else if (mode == PDB_SP_OUT_ROW_CONTRACT) {
      __syncthreads();  // V complete for every thread
      const float* W = d.w + rider_off(d.w_stride, r0, r1, r2);
      for (int e = tid; e < SP_COLS * SP_XMAX; e += SP_THREADS) {
        const int r = e / SP_XMAX, x = e % SP_XMAX;
        const int64_t s = s0 + r;
        Ws[e] = (s < d.cols && x < d.xdim) ? W[s * d.w_stride[3] + x * d.w_stride[4]] : 0.f;
      }
      __syncthreads();
      const int tr = tid >> 4, tx = tid & 15;  // rows 4 tr + u, x = tx + 16 j
#pragma unroll 4
      for (int c = 0; c < SP_COLS; ++c) {
        const int64_t s = s0 + c;
        float v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) v[u] = (s < d.cols) ? V[(4 * tr + u) * SP_COLS + c] : 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float w = Ws[c * SP_XMAX + tx + 16 * j];
#pragma unroll
          for (int u = 0; u < 4; ++u) acc[u][j] = fmaf(v[u], w, acc[u][j]);
        }
      }
      __syncthreads();  // Ws and V are rewritten by the next column tile
    } else {  // row reductions: warp w owns rows w + 8 i, lane = column
#pragma unroll
      for (int i = 0; i < SP_EPT; ++i) {
        const int e = tid + SP_THREADS * i;
        const int64_t t = t0 + e / SP_COLS, s = s0 + e % SP_COLS;
        float v = (t < d.rows && s < d.cols) ? V[e] : reduce_identity(mode);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v = reduce_combine(mode, v, __shfl_xor_sync(0xffffffffu, v, off));
        red[i] = reduce_combine(mode, red[i], v);
      }
    }
    __syncthreads();  // the register file is rewritten by the next column tile
  }

  if (mode == PDB_SP_OUT_ROW_CONTRACT) {
    const int tr = tid >> 4, tx = tid & 15;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t t = t0 + 4 * tr + u;
      if (t >= d.rows) continue;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int x = tx + 16 * j;
        if (x >= d.xdim) continue;
        float* o = d.out + rider_off(d.out_stride, r0, r1, r2) + t * d.out_stride[3] + x * d.out_stride[4];
        if (atomic_out) atomicAdd(o, acc[u][j]);
        else *o = acc[u][j];
      }
    }
  } else if (mode != PDB_SP_OUT_TILE && lane == 0) {
#pragma unroll
    for (int i = 0; i < SP_EPT; ++i) {
      const int64_t t = t0 + warp + 8 * i;
      if (t >= d.rows) continue;
      float* o = d.out + rider_off(d.out_stride, r0, r1, r2) + t * d.out_stride[3];
      if (atomic_out) atomicAdd(o, red[i]);
      else *o = red[i];
    }
  }
}

// zeroes out[b, t (, x)] ahead of a column-split launch that accumulates into it
struct SpZero {
  float* out;
  int64_t riders, mid, inner, rows, xdim;
  int64_t st[5];
};
__global__ void sp_zero_kernel(const SpZero z) {
  const int64_t total = z.riders * z.rows * z.xdim;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t x = e % z.xdim, t = (e / z.xdim) % z.rows, y = e / (z.xdim * z.rows);
    const int64_t r2 = y % z.inner, r1 = (y / z.inner) % z.mid, r0 = y / (z.inner * z.mid);
    z.out[r0 * z.st[0] + r1 * z.st[1] + r2 * z.st[2] + t * z.st[3] + x * z.st[4]] = 0.f;
  }
}

size_t sp_smem_bytes(int n_regs) {
  return sizeof(float) * ((size_t)n_regs * SP_ROWS * SP_COLS + SP_FK * (SP_ROWS + 1) + SP_FK * (SP_COLS + 1) +
                          SP_COLS * SP_XMAX);
}

int check_program(const pdb_score_program_desc* d) {
  if (d->n_ops <= 0 || d->n_ops > PDB_SP_MAX_OPS) return set_error(PDB_ERR_ARG, "score program: 1..%d steps", PDB_SP_MAX_OPS);
  if (d->n_regs <= 0 || d->n_regs > PDB_SP_MAX_REGS)
    return set_error(PDB_ERR_ARG, "score program: 1..%d registers", PDB_SP_MAX_REGS);
  if (d->result < 0 || d->result >= d->n_regs) return set_error(PDB_ERR_ARG, "score program: bad result register");
  if (d->n_scores < 0 || d->n_scores > PDB_SP_MAX_SCORES) return set_error(PDB_ERR_ARG, "score program: bad n_scores");
  for (int c = 0; c < d->n_scores; ++c) {
    if (!d->score_a[c] || !d->score_b[c] || d->score_feat[c] <= 0)
      return set_error(PDB_ERR_ARG, "score program: contraction %d needs operands and a positive feature size", c);
  }
  for (int k = 0; k < d->n_ops; ++k) {
    const pdb_sp_op& o = d->ops[k];
    if (o.dst < 0 || o.dst >= d->n_regs) return set_error(PDB_ERR_ARG, "score program step %d: bad dst", k);
    switch (o.op) {
      case PDB_SP_SCORE:
        if (o.a < 0 || o.a >= d->n_scores) return set_error(PDB_ERR_ARG, "step %d: bad contraction slot", k);
        break;
      case PDB_SP_ROW:
        if (o.a < 0 || o.a >= PDB_SP_MAX_VECS || !d->rowvec[o.a]) return set_error(PDB_ERR_ARG, "step %d: bad row vector", k);
        break;
      case PDB_SP_COL:
        if (o.a < 0 || o.a >= PDB_SP_MAX_VECS || !d->colvec[o.a]) return set_error(PDB_ERR_ARG, "step %d: bad column vector", k);
        break;
      case PDB_SP_TILE:
        if (o.a < 0 || o.a >= PDB_SP_MAX_TILES || !d->tile[o.a]) return set_error(PDB_ERR_ARG, "step %d: bad tile", k);
        break;
      case PDB_SP_CONST:
      case PDB_SP_IOTA_ROW:
      case PDB_SP_IOTA_COL:
        break;
      case PDB_SP_WHERE:
        if (o.c < 0 || o.c >= d->n_regs) return set_error(PDB_ERR_ARG, "step %d: bad operand register", k);
        /* fallthrough */
      default:
        if (o.op < PDB_SP_SCORE || o.op > PDB_SP_FLOOR) return set_error(PDB_ERR_ARG, "step %d: unknown opcode %d", k, o.op);
        if (o.a < 0 || o.a >= d->n_regs || (o.op < PDB_SP_EXP && (o.b < 0 || o.b >= d->n_regs)))
          return set_error(PDB_ERR_ARG, "step %d: bad operand register", k);
    }
  }
  return PDB_OK;
}

}  // namespace
}  // namespace pdb

using namespace pdb;

extern "C" int pdb_score_program_f32(const pdb_score_program_desc* d, void* stream) {
  if (!d) return set_error(PDB_ERR_ARG, "null descriptor");
  if (d->batch <= 0 || d->batch_mid <= 0 || d->batch_inner <= 0 || d->rows <= 0 || d->cols <= 0)
    return set_error(PDB_ERR_SHAPE, "score program: sizes must be positive");
  const int64_t nriders = d->batch * d->batch_mid * d->batch_inner;
  if (nriders > 65535 || d->rows > (int64_t)0x7fffffff * SP_ROWS)
    return set_error(PDB_ERR_SHAPE, "score program: grid too large");
  if (!d->out) return set_error(PDB_ERR_ARG, "score program: null out");
  if (int st = check_program(d)) return st;
  const int mode = d->out_mode;
  if (mode < PDB_SP_OUT_TILE || mode > PDB_SP_OUT_ROW_CONTRACT)
    return set_error(PDB_ERR_ARG, "score program: unknown output mode %d", mode);
  if (mode == PDB_SP_OUT_ROW_CONTRACT && (!d->w || d->xdim <= 0))
    return set_error(PDB_ERR_ARG, "score program: the contraction output needs w and xdim > 0");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t smem = sp_smem_bytes(d->n_regs);
  cudaError_t e = cudaFuncSetAttribute(score_program_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return cuda_status(e, "score program smem attribute");
  const int64_t row_blocks = (d->rows + SP_ROWS - 1) / SP_ROWS;
  const int64_t col_tiles = (d->cols + SP_COLS - 1) / SP_COLS;
  SpParams P;
  P.d = *d;
  // Few row blocks leave most SMs idle: sum-type outputs split the columns over
  // more CTAs (about two waves, at least four column tiles each) and add their
  // partial results atomically (the f32 summation order then varies run to run).
  P.csplit = 1;
  if (mode == PDB_SP_OUT_ROW_SUM || mode == PDB_SP_OUT_ROW_CONTRACT) {
    int dev = 0;
    cudaGetDevice(&dev);
    const int64_t nb = row_blocks * nriders;
    const int64_t want = (2 * (int64_t)sm_count(dev) + nb - 1) / nb;
    const int64_t most = col_tiles / 4 > 1 ? col_tiles / 4 : 1;
    P.csplit = (int)(want < most ? (want > 1 ? want : 1) : most);
    if (P.csplit > 64) P.csplit = 64;
  }
  dim3 grid((unsigned)row_blocks, (unsigned)nriders, (unsigned)P.csplit);
  // contraction outputs wider than SP_XMAX: one launch per 128-column slab of w / out
  const int64_t xdim = mode == PDB_SP_OUT_ROW_CONTRACT ? d->xdim : 1;
  for (int64_t x0 = 0; x0 < xdim; x0 += SP_XMAX) {
    if (mode == PDB_SP_OUT_ROW_CONTRACT) {
      P.d.w = d->w + x0 * d->w_stride[4];
      P.d.out = d->out + x0 * d->out_stride[4];
      P.d.xdim = xdim - x0 < SP_XMAX ? xdim - x0 : SP_XMAX;
    }
    if (P.csplit > 1) {
      const int64_t xd = mode == PDB_SP_OUT_ROW_CONTRACT ? P.d.xdim : 1;
      SpZero z{P.d.out, nriders, d->batch_mid, d->batch_inner, d->rows, xd,
                {d->out_stride[0], d->out_stride[1], d->out_stride[2], d->out_stride[3],
                 mode == PDB_SP_OUT_ROW_CONTRACT ? d->out_stride[4] : 0}};
      sp_zero_kernel<<<256, 256, 0, s>>>(z);
    }
    score_program_kernel<<<grid, SP_THREADS, smem, s>>>(P);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_status(e, "score program launch");
  }
  return PDB_OK;
}
