// Contraction-epilogue and map-chain templates.
//
// Reference rows: _match_contraction_epilogue / _generate_contraction
// (fusion.py:159-324): a sum over one contracted dim of a two-operand
// product, the pointwise epilogue absorbed so the accumulator never touches
// memory; and the map-chain row (fusion.py:830-860).  The reference lowers
// both through compile_tile (triton_tile.py:471-546) as an f32 IEEE dot.
//
// Here the epilogue is a short step program (pdb_ew_op) interpreted per
// element by the kernel, so one prebuilt kernel serves every chain:
//   * contract_f32_kernel  -- f32 operands, IEEE FMA, 64 x 64 tiles staged
//                             through shared memory (the reference's column);
//   * contract_bf16_kernel -- persistent; bf16 operands by TMA (128B swizzle),
//                             tcgen05 M128 N256 MMAs into two fp32 TMEM
//                             accumulators (epilogue of one tile overlaps the
//                             next tile's K loop), stored as bf16;
//   * pointwise_f32_kernel -- the map-chain template over a strided tensor.
#include <cfloat>
#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "tma.h"

namespace pdb {
namespace {

struct EwOp {  // device copy of pdb_ew_op with the constant already in f32
  int32_t op, operand, swap;
  float value;
  const float* ptr;
  int64_t stride[3];
};
struct EwProgram {
  int32_t n;
  EwOp ops[PDB_MAX_EW_OPS];
};

EwProgram make_program(int n, const pdb_ew_op* ops) {
  EwProgram pg{};
  pg.n = n;
  for (int s = 0; s < n; ++s) {
    pg.ops[s].op = ops[s].op;
    pg.ops[s].operand = ops[s].operand;
    pg.ops[s].swap = ops[s].swap;
    pg.ops[s].value = (float)ops[s].value;
    pg.ops[s].ptr = ops[s].ptr;
    for (int i = 0; i < 3; ++i) pg.ops[s].stride[i] = ops[s].stride[i];
  }
  return pg;
}

__device__ __forceinline__ float ew_apply(const EwProgram& pg, float v, int64_t b, int64_t i, int64_t j) {
  for (int s = 0; s < pg.n; ++s) {
    const EwOp& o = pg.ops[s];
    float w = 0.f;
    if (o.operand == 1) w = o.value;
    else if (o.operand == 2) w = __ldg(o.ptr + b * o.stride[0] + i * o.stride[1] + j * o.stride[2]);
    float x = v, y = w;
    if (o.swap) {
      x = w;
      y = v;
    }
    switch (o.op) {
      case PDB_EW_ADD: v = x + y; break;
      case PDB_EW_SUB: v = x - y; break;
      case PDB_EW_MUL: v = x * y; break;
      case PDB_EW_DIV: v = x / y; break;
      case PDB_EW_MAX: v = fmaxf(x, y); break;
      case PDB_EW_MIN: v = fminf(x, y); break;
      case PDB_EW_EXP: v = expf(v); break;
      case PDB_EW_LOG: v = logf(v); break;
      case PDB_EW_SQRT: v = sqrtf(v); break;
      case PDB_EW_TANH: v = tanhf(v); break;
      case PDB_EW_NEG: v = -v; break;
      default: break;
    }
  }
  return v;
}

// The epilogue program over 32 consecutive columns of one output row, step by
// step: a tensor operand's 32 values are loaded together (independent loads,
// one memory latency per step instead of one per element), then the step's
// op runs over the row.  Same arithmetic as ew_apply, element for element.
#define PDB_EW_ROW(EXPR)                       \
  _Pragma("unroll") for (int c = 0; c < 32; ++c) { \
    const float x = sw ? w[c] : v[c];          \
    const float y = sw ? v[c] : w[c];          \
    (void)x; (void)y;                          \
    v[c] = (EXPR);                             \
  }
#define PDB_EW_ROW4(EXPR)                      \
  _Pragma("unroll") for (int c = 0; c < 4; ++c) { \
    const float x = sw ? w[c] : v[c];          \
    const float y = sw ? v[c] : w[c];          \
    (void)x; (void)y;                          \
    v[c] = (EXPR);                             \
  }
__device__ __forceinline__ void ew_apply_row32(const EwProgram& pg, float (&v)[32], int64_t b, int64_t i, int64_t j0,
                                               int nvalid) {
  for (int s = 0; s < pg.n; ++s) {
    const EwOp& o = pg.ops[s];
    float w[32];
    if (o.operand == 2) {
      const float* base = o.ptr + b * o.stride[0] + i * o.stride[1] + j0 * o.stride[2];
      const int64_t js = o.stride[2];
#pragma unroll
      for (int c = 0; c < 32; ++c) w[c] = c < nvalid ? __ldg(base + c * js) : 0.f;
    } else {
      const float cv = o.operand == 1 ? o.value : 0.f;
#pragma unroll
      for (int c = 0; c < 32; ++c) w[c] = cv;
    }
    const bool sw = o.swap != 0;
    switch (o.op) {
      case PDB_EW_ADD: PDB_EW_ROW(x + y) break;
      case PDB_EW_SUB: PDB_EW_ROW(x - y) break;
      case PDB_EW_MUL: PDB_EW_ROW(x * y) break;
      case PDB_EW_DIV: PDB_EW_ROW(x / y) break;
      case PDB_EW_MAX: PDB_EW_ROW(fmaxf(x, y)) break;
      case PDB_EW_MIN: PDB_EW_ROW(fminf(x, y)) break;
      case PDB_EW_EXP: PDB_EW_ROW(expf(v[c])) break;
      case PDB_EW_LOG: PDB_EW_ROW(logf(v[c])) break;
      case PDB_EW_SQRT: PDB_EW_ROW(sqrtf(v[c])) break;
      case PDB_EW_TANH: PDB_EW_ROW(tanhf(v[c])) break;
      case PDB_EW_NEG: PDB_EW_ROW(-v[c]) break;
      default: break;
    }
  }
}
#undef PDB_EW_ROW

struct ContractParams {
  const void* a;
  const void* b;
  void* c;
  int64_t batch, m, n, k;
  int64_t as[3], bs[3], cs[3];
  float alpha;
  int* err;
  int group;  // m-tile rows per raster group of the pair kernel
  int serp;   // odd groups walk the n tiles backwards (B panels reused across the group boundary)
  EwProgram pg;
};

// ------------------------------------------------------------------ f32 path
constexpr int FT = 64, FK = 16, FTHREADS = 256;

__global__ void __launch_bounds__(FTHREADS) contract_f32_kernel(const ContractParams p) {
  __shared__ float As[FK][FT + 1];
  __shared__ float Bs[FK][FT + 1];
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const int64_t bidx = blockIdx.z;
  const int64_t m0 = (int64_t)blockIdx.y * FT, n0 = (int64_t)blockIdx.x * FT;
  const float* A = static_cast<const float*>(p.a) + bidx * p.as[0];
  const float* B = static_cast<const float*>(p.b) + bidx * p.bs[0];
  float acc[4][4] = {};
  for (int64_t k0 = 0; k0 < p.k; k0 += FK) {
    for (int e = tid; e < FT * FK; e += FTHREADS) {
      const int r = e / FK, kk = e % FK;
      const int64_t gm = m0 + r, gn = n0 + r, gk = k0 + kk;
      As[kk][r] = (gm < p.m && gk < p.k) ? A[gm * p.as[1] + gk * p.as[2]] : 0.f;
      Bs[kk][r] = (gn < p.n && gk < p.k) ? B[gn * p.bs[1] + gk * p.bs[2]] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < FK; ++kk) {
      float a[4], bb[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        a[u] = As[kk][ty * 4 + u];
        bb[u] = Bs[kk][tx + 16 * u];
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int w = 0; w < 4; ++w) acc[u][w] = fmaf(a[u], bb[w], acc[u][w]);
    }
    __syncthreads();
  }
  float* C = static_cast<float*>(p.c);
#pragma unroll
  for (int u = 0; u < 4; ++u)
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const int64_t gm = m0 + ty * 4 + u, gn = n0 + tx + 16 * w;
      if (gm < p.m && gn < p.n)
        C[bidx * p.cs[0] + gm * p.cs[1] + gn * p.cs[2]] = ew_apply(p.pg, acc[u][w] * p.alpha, bidx, gm, gn);
    }
}

// ----------------------------------------------------------------- bf16 path
// Persistent: one CTA per SM walks 128 x 256 output tiles.  Warp 0 streams A
// (128 x 64) and B (256 x 64) k-blocks by TMA through a 4-stage ring, warp 1
// issues M128 N256 K16 tcgen05 MMAs into one of two TMEM accumulators
// (2 x 256 columns), warps 4..7 drain the other accumulator through the
// epilogue program while the next tile accumulates.
constexpr int GM = 128, GN = 256, GK = 64, GSTAGES = 4, GTHREADS = 256;
constexpr int kStageA = GM * GK * 2, kStageB = GN * GK * 2;

struct __align__(8) GemmBars {
  uint64_t full[GSTAGES], empty[GSTAGES];
  uint64_t acc_full[2], acc_empty[2];
  uint32_t tmem_base;
  int abort;
};

__global__ void __launch_bounds__(GTHREADS, 1)
    contract_bf16_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                         const ContractParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + GSTAGES * kStageA;
  GemmBars* bar = reinterpret_cast<GemmBars*>(sB + GSTAGES * kStageB);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = (int)((p.k + GK - 1) / GK);
  const int tm = (int)((p.m + GM - 1) / GM), tn = (int)((p.n + GN - 1) / GN);
  const int num_tiles = (int)p.batch * tm * tn;

  if (threadIdx.x == 0) {
    for (int i = 0; i < GSTAGES; ++i) {
      mbar_init(&bar->full[i], 1);
      mbar_init(&bar->empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar->acc_full[i], 1);
      mbar_init(&bar->acc_empty[i], 4);  // one arrival per epilogue warp
    }
    bar->abort = 0;
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc(&bar->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar->tmem_base;
  volatile int* abort = &bar->abort;
  // tile t -> (batch, m-tile, n-tile) in groups of 8 m-tile rows, m fastest inside a group, so
  // the tiles in flight at once touch ~8 A row-blocks and ~20 B column-blocks (fits in L2)
  auto coords = [&](int t, int& bi, int& m0, int& n0) {
    bi = t / (tm * tn);
    const int r = t % (tm * tn);
    const int gsz = 8 * tn;  // tiles per group of 8 m-tile rows
    const int grp = r / gsz, in = r % gsz;
    const int rows = (tm - grp * 8) < 8 ? (tm - grp * 8) : 8;
    m0 = (grp * 8 + in % rows) * GM;
    n0 = (in / rows) * GN;
  };

  if (warp == 0 && lane == 0) {
    uint32_t g = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < num_tiles; t += gridDim.x) {
      int bi, m0, n0;
      coords(t, bi, m0, n0);
      for (int kb = 0; kb < nk; ++kb, ++g) {
        const int st = g % GSTAGES;
        if (!(ok = mbar_wait(&bar->empty[st], ((g / GSTAGES) & 1) ^ 1, abort, p.err))) break;
        mbar_expect_tx(&bar->full[st], kStageA + kStageB);
        tma_load_4d(sA + st * kStageA, &tm_a, &bar->full[st], kb * GK, m0, bi, 0);
        tma_load_4d(sB + st * kStageB, &tm_b, &bar->full[st], kb * GK, n0, bi, 0);
      }
    }
  } else if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc = idesc_bf16(GM, GN, 0, 0);
    uint32_t g = 0, tt = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < num_tiles; t += gridDim.x, ++tt) {
      const int buf = tt & 1;
      if (!(ok = mbar_wait(&bar->acc_empty[buf], ((tt >> 1) & 1) ^ 1, abort, p.err))) break;
      tc_fence_after();
      const uint32_t acc = tmem + buf * GN;
      for (int kb = 0; kb < nk; ++kb, ++g) {
        const int st = g % GSTAGES;
        if (!(ok = mbar_wait(&bar->full[st], (g / GSTAGES) & 1, abort, p.err))) break;
        tc_fence_after();
        const uint32_t a0 = smem_u32(sA + st * kStageA), b0 = smem_u32(sB + st * kStageB);
#pragma unroll
        for (int kk = 0; kk < GK / 16; ++kk)
          mma_ss(acc, sdesc_sw128(a0 + kk * 32, 16, 1024), sdesc_sw128(b0 + kk * 32, 16, 1024), idesc,
                 (kb > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&bar->empty[st]);
      }
      if (ok) tc_commit(&bar->acc_full[buf]);
    }
  } else if (warp >= 4) {
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const bool vec = p.cs[2] == 1 && (p.cs[1] & 7) == 0 && (p.cs[0] & 7) == 0 &&
                     (reinterpret_cast<uintptr_t>(p.c) & 15) == 0;
    uint32_t tt = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++tt) {
      int bi, m0, n0;
      coords(t, bi, m0, n0);
      const int buf = tt & 1;
      if (!mbar_wait(&bar->acc_full[buf], (tt >> 1) & 1, abort, p.err)) break;
      tc_fence_after();
      const int64_t gm = m0 + row;
      __nv_bfloat16* C = static_cast<__nv_bfloat16*>(p.c) + (int64_t)bi * p.cs[0] + gm * p.cs[1];
#pragma unroll 1
      for (int ch = 0; ch < GN / 32; ++ch) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_off + buf * GN + ch * 32, r);
        tmem_wait_ld();
        const int64_t c0 = n0 + ch * 32;
        if (gm >= p.m || c0 >= p.n) continue;
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) * p.alpha;
        ew_apply_row32(p.pg, v, bi, gm, c0, (int)(p.n - c0 < 32 ? p.n - c0 : 32));
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) pk[i] = pack_bf16(v[2 * i], v[2 * i + 1]);
        if (vec && c0 + 32 <= p.n) {
          uint4* dst = reinterpret_cast<uint4*>(C + c0);
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
        } else {
          const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(pk);
          for (int i = 0; i < 32 && c0 + i < p.n; ++i) C[(c0 + i) * p.cs[2]] = h[i];
        }
      }
      warp_arrive_after_tc(&bar->acc_empty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------ bf16 path, CTA pair
// Same schedule on a cluster of two CTAs (one per SM) and 256 x 256 output
// tiles: each CTA stages 128 rows of A and 128 rows of B per k-block, the
// pair's rank-0 thread issues cta_group::2 M256 N256 K16 MMAs that read both
// CTAs' shared memory and write 128 accumulator rows into each CTA's TMEM.
// Per SM that halves the B bytes fetched per MMA cycle (64 instead of 96 B per
// cycle at the full tensor rate).  Barriers: full[] of rank 0 counts both
// CTAs' TMA bytes; empty[] and acc_full[] of each CTA receive the pair
// commits; acc_empty[] of rank 0 counts the 16 epilogue warps of the pair
// (warps 4..11 of each CTA: TMEM lane quarter warp % 4, column half (warp - 4) / 4).
constexpr int PM = 256, PN = 256, PSTAGES = 6, PTHREADS = 384;
constexpr int kPairStage = 128 * GK * 2;  // A or B half tile per CTA per k-block

struct __align__(8) PairBars {
  uint64_t full[PSTAGES], empty[PSTAGES];
  uint64_t acc_full[2], acc_empty[2];
  uint32_t tmem_base;
  int abort;
};

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PTHREADS, 1)
    contract_bf16_pair_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                              const ContractParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + PSTAGES * kPairStage;
  PairBars* bar = reinterpret_cast<PairBars*>(sB + PSTAGES * kPairStage);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int nk = (int)((p.k + GK - 1) / GK);
  const int tm = (int)((p.m + PM - 1) / PM), tn = (int)((p.n + PN - 1) / PN);
  const int num_tiles = (int)p.batch * tm * tn;

  if (threadIdx.x == 0) {
    for (int i = 0; i < PSTAGES; ++i) {
      mbar_init(&bar->full[i], 1);
      mbar_init(&bar->empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar->acc_full[i], 1);
      mbar_init(&bar->acc_empty[i], 16);  // one arrival per epilogue warp of the pair
    }
    bar->abort = 0;
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc_pair(&bar->tmem_base, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = bar->tmem_base;
  volatile int* abort = &bar->abort;
  auto coords = [&](int t, int& bi, int& m0, int& n0) {
    bi = t / (tm * tn);
    const int r = t % (tm * tn);
    const int G = p.group;
    const int gsz = G * tn;
    const int grp = r / gsz, in = r % gsz;
    const int rows = (tm - grp * G) < G ? (tm - grp * G) : G;
    m0 = (grp * G + in % rows) * PM;
    const int nt = in / rows;
    n0 = ((p.serp && (grp & 1)) ? tn - 1 - nt : nt) * PN;
  };

  if (warp == 0 && lane == 0) {
    uint32_t g = 0;
    bool ok = true;
    for (int t = pair; ok && t < num_tiles; t += npairs) {
      int bi, m0, n0;
      coords(t, bi, m0, n0);
      for (int kb = 0; kb < nk; ++kb, ++g) {
        const int st = g % PSTAGES;
        if (!(ok = mbar_wait_cluster(&bar->empty[st], ((g / PSTAGES) & 1) ^ 1, abort, p.err))) break;
        if (rank == 0) mbar_expect_tx(&bar->full[st], 4 * kPairStage);
        const uint32_t full0 = mapa_shared(smem_u32(&bar->full[st]), 0);
        tma_load_4d_pair(sA + st * kPairStage, &tm_a, full0, kb * GK, m0 + (int)rank * 128, bi, 0);
        tma_load_4d_pair(sB + st * kPairStage, &tm_b, full0, kb * GK, n0 + (int)rank * 128, bi, 0);
      }
    }
  } else if (warp == 1 && lane == 0 && rank == 0) {
    constexpr uint32_t idesc = idesc_bf16(PM, PN, 0, 0);
    uint32_t g = 0, tt = 0;
    bool ok = true;
    for (int t = pair; ok && t < num_tiles; t += npairs, ++tt) {
      const int buf = tt & 1;
      if (!(ok = mbar_wait_cluster(&bar->acc_empty[buf], ((tt >> 1) & 1) ^ 1, abort, p.err))) break;
      tc_fence_after();
      const uint32_t acc = tmem + buf * PN;
      for (int kb = 0; kb < nk; ++kb, ++g) {
        const int st = g % PSTAGES;
        if (!(ok = mbar_wait_cluster(&bar->full[st], (g / PSTAGES) & 1, abort, p.err))) break;
        tc_fence_after();
        const uint32_t a0 = smem_u32(sA + st * kPairStage), b0 = smem_u32(sB + st * kPairStage);
#pragma unroll
        for (int kk = 0; kk < GK / 16; ++kk)
          mma_ss_pair(acc, sdesc_sw128(a0 + kk * 32, 16, 1024), sdesc_sw128(b0 + kk * 32, 16, 1024), idesc,
                      (kb > 0 || kk > 0) ? 1u : 0u);
        const uint32_t e = smem_u32(&bar->empty[st]);
        tc_commit_pair(e);
        tc_commit_pair(mapa_shared(e, 1));
      }
      if (ok) {
        const uint32_t f = smem_u32(&bar->acc_full[buf]);
        tc_commit_pair(f);
        tc_commit_pair(mapa_shared(f, 1));
      }
    }
  } else if (warp >= 4) {
    const int q4 = warp & 3, half = (warp - 4) >> 2;  // TMEM lane quarter, column half
    const int row = (int)rank * 128 + q4 * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const bool vec = p.cs[2] == 1 && (p.cs[1] & 7) == 0 && (p.cs[0] & 7) == 0 &&
                     (reinterpret_cast<uintptr_t>(p.c) & 15) == 0;
    uint32_t tt = 0;
    for (int t = pair; t < num_tiles; t += npairs, ++tt) {
      int bi, m0, n0;
      coords(t, bi, m0, n0);
      const int buf = tt & 1;
      if (!mbar_wait_cluster(&bar->acc_full[buf], (tt >> 1) & 1, abort, p.err)) break;
      tc_fence_after();
      const int64_t gm = m0 + row;
      __nv_bfloat16* C = static_cast<__nv_bfloat16*>(p.c) + (int64_t)bi * p.cs[0] + gm * p.cs[1];
#pragma unroll 1
      for (int ch = half * (PN / 64); ch < (half + 1) * (PN / 64); ++ch) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_off + buf * PN + ch * 32, r);
        tmem_wait_ld();
        const int64_t c0 = n0 + ch * 32;
        if (gm >= p.m || c0 >= p.n) continue;
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) * p.alpha;
        ew_apply_row32(p.pg, v, bi, gm, c0, (int)(p.n - c0 < 32 ? p.n - c0 : 32));
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) pk[i] = pack_bf16(v[2 * i], v[2 * i + 1]);
        if (vec && c0 + 32 <= p.n) {
          uint4* dst = reinterpret_cast<uint4*>(C + c0);
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
        } else {
          const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(pk);
          for (int i = 0; i < 32 && c0 + i < p.n; ++i) C[(c0 + i) * p.cs[2]] = h[i];
        }
      }
      warp_arrive_cluster_after_tc(mapa_shared(smem_u32(&bar->acc_empty[buf]), 0));
    }
  }
  tc_fence_before();
  cluster_sync_all();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

// -------------------------------------------------------------- map-chain
struct PointwiseArgs {
  const float* x;
  float* y;
  int64_t batch, m, n;
  int64_t xs[3], ys[3];
};

// Work items are 1024-column segments of one (batch, row): a block of 256
// threads takes a segment, each thread four consecutive columns -- one 16-byte
// load and store when both tensors are unit-stride along n and 16-byte aligned
// (`vec`), else four scalar accesses.  The (batch, row) coordinates are derived
// once per segment, not per element.
constexpr int kPwThreads = 256, kPwSeg = 4 * kPwThreads;

__global__ void __launch_bounds__(kPwThreads) pointwise_f32_kernel(const PointwiseArgs d, const EwProgram pg,
                                                                   const int vec) {
  const int64_t rows = d.batch * d.m;
  const int64_t nseg = (d.n + kPwSeg - 1) / kPwSeg;
  for (int64_t w = blockIdx.x; w < rows * nseg; w += gridDim.x) {
    const int64_t r = w / nseg, sg = w - r * nseg;
    const int64_t b = r / d.m, i = r - b * d.m;
    const int64_t j0 = sg * kPwSeg + 4 * threadIdx.x;
    if (j0 >= d.n) continue;
    const float* xr = d.x + b * d.xs[0] + i * d.xs[1];
    float* yr = d.y + b * d.ys[0] + i * d.ys[1];
    if (vec && j0 + 4 <= d.n) {
      const float4 x4 = __ldcs(reinterpret_cast<const float4*>(xr + j0));
      float v[4] = {x4.x, x4.y, x4.z, x4.w};
      // one dispatch per step for the four values
      for (int st = 0; st < pg.n; ++st) {
        const EwOp& o = pg.ops[st];
        float w[4];
        if (o.operand == 2) {
          const float* base = o.ptr + b * o.stride[0] + i * o.stride[1] + j0 * o.stride[2];
#pragma unroll
          for (int c = 0; c < 4; ++c) w[c] = __ldg(base + c * o.stride[2]);
        } else {
#pragma unroll
          for (int c = 0; c < 4; ++c) w[c] = o.value;
        }
        const bool sw = o.swap != 0;
        switch (o.op) {
          case PDB_EW_ADD: PDB_EW_ROW4(x + y) break;
          case PDB_EW_SUB: PDB_EW_ROW4(x - y) break;
          case PDB_EW_MUL: PDB_EW_ROW4(x * y) break;
          case PDB_EW_DIV: PDB_EW_ROW4(x / y) break;
          case PDB_EW_MAX: PDB_EW_ROW4(fmaxf(x, y)) break;
          case PDB_EW_MIN: PDB_EW_ROW4(fminf(x, y)) break;
          case PDB_EW_EXP: PDB_EW_ROW4(expf(v[c])) break;
          case PDB_EW_LOG: PDB_EW_ROW4(logf(v[c])) break;
          case PDB_EW_SQRT: PDB_EW_ROW4(sqrtf(v[c])) break;
          case PDB_EW_TANH: PDB_EW_ROW4(tanhf(v[c])) break;
          case PDB_EW_NEG: PDB_EW_ROW4(-v[c]) break;
          default: break;
        }
      }
      __stcs(reinterpret_cast<float4*>(yr + j0), make_float4(v[0], v[1], v[2], v[3]));
    } else {
      for (int64_t j = j0; j < j0 + 4 && j < d.n; ++j) yr[j * d.ys[2]] = ew_apply(pg, xr[j * d.xs[2]], b, i, j);
    }
  }
}

int check_ops(int n, const pdb_ew_op* ops) {
  if (n < 0 || n > PDB_MAX_EW_OPS) return set_error(PDB_ERR_ARG, "n_ops must be in [0, %d]", PDB_MAX_EW_OPS);
  for (int s = 0; s < n; ++s) {
    const pdb_ew_op& o = ops[s];
    if (o.op < PDB_EW_ADD || o.op > PDB_EW_NEG) return set_error(PDB_ERR_ARG, "epilogue step %d: bad opcode", s);
    const bool unary = o.op >= PDB_EW_EXP;
    if (unary != (o.operand == 0)) return set_error(PDB_ERR_ARG, "epilogue step %d: operand kind mismatch", s);
    if (o.operand == 2 && o.ptr == nullptr) return set_error(PDB_ERR_ARG, "epilogue step %d: null tensor", s);
  }
  return PDB_OK;
}

}  // namespace
}  // namespace pdb

using namespace pdb;

extern "C" int pdb_contract(const pdb_contract_desc* d, void* stream) {
  if (!d) return set_error(PDB_ERR_ARG, "null descriptor");
  if (d->batch <= 0 || d->m <= 0 || d->n <= 0 || d->k <= 0)
    return set_error(PDB_ERR_SHAPE, "contract: sizes must be positive");
  if (!d->a || !d->b || !d->c) return set_error(PDB_ERR_ARG, "null a / b / c");
  if (int st = check_ops(d->n_ops, d->ops)) return st;
  if (d->batch > 65535 || d->m > (int64_t)65535 * GM || d->n > 0x7fffffffLL)
    return set_error(PDB_ERR_SHAPE, "contract: grid too large");
  ContractParams p{};
  p.a = d->a;
  p.b = d->b;
  p.c = d->c;
  p.batch = d->batch;
  p.m = d->m;
  p.n = d->n;
  p.k = d->k;
  for (int i = 0; i < 3; ++i) {
    p.as[i] = d->a_stride[i];
    p.bs[i] = d->b_stride[i];
    p.cs[i] = d->c_stride[i];
  }
  p.alpha = (float)d->alpha;
  // raster of the pair kernel: groups of 8 m-tile rows (2048 rows of A), odd groups
  // walking n backwards; measured at 8192^3: G = 8 1365-1370, G = 4 / 16 / 32 1350 / 1353 /
  // 1305 TFLOP/s, DRAM reads 1.08 GB (G = 8) vs 1.24 GB (G = 16) for 268 MB of A + B
  p.group = 8;
  p.serp = 1;
  p.err = device_error_flag();
  p.pg = make_program(d->n_ops, d->ops);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (d->dtype == PDB_F32) {
    dim3 grid((unsigned)((d->n + FT - 1) / FT), (unsigned)((d->m + FT - 1) / FT), (unsigned)d->batch);
    contract_f32_kernel<<<grid, FTHREADS, 0, s>>>(p);
    return cuda_status(cudaGetLastError(), "contract f32 launch");
  }
  if (d->dtype != PDB_BF16) return set_error(PDB_ERR_UNSUPPORTED, "contract: unknown dtype %d", d->dtype);
  if (d->a_stride[2] != 1 || d->b_stride[2] != 1)
    return set_error(PDB_ERR_ALIGN, "contract bf16: the contracted dim must be contiguous in a and b");
  // 256 x 256 tiles on CTA pairs when both output dims fill one; PDB_CONTRACT_PAIR=0 forces single CTAs
  const char* pair_env = getenv("PDB_CONTRACT_PAIR");
  const bool pair = d->m >= PM && d->n >= PN && !(pair_env && pair_env[0] == '0');
  const uint32_t rows_a = pair ? 128 : GM, rows_b = pair ? 128 : GN;
  CUtensorMap ta, tb;
  {
    const uint64_t dims[4] = {(uint64_t)d->k, (uint64_t)d->m, (uint64_t)d->batch, 1};
    const uint64_t str[3] = {(uint64_t)d->a_stride[1] * 2, (uint64_t)(d->batch > 1 ? d->a_stride[0] : d->m * d->a_stride[1]) * 2,
                             (uint64_t)(d->batch * (d->batch > 1 ? d->a_stride[0] : d->m * d->a_stride[1])) * 2};
    const uint32_t box[4] = {GK, rows_a, 1, 1};
    if (int st = encode_tma_4d(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, d->a, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return st;
  }
  {
    const uint64_t dims[4] = {(uint64_t)d->k, (uint64_t)d->n, (uint64_t)d->batch, 1};
    const uint64_t str[3] = {(uint64_t)d->b_stride[1] * 2, (uint64_t)(d->batch > 1 ? d->b_stride[0] : d->n * d->b_stride[1]) * 2,
                             (uint64_t)(d->batch * (d->batch > 1 ? d->b_stride[0] : d->n * d->b_stride[1])) * 2};
    const uint32_t box[4] = {GK, rows_b, 1, 1};
    if (int st = encode_tma_4d(&tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, d->b, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return st;
  }
  int dev = 0;
  cudaGetDevice(&dev);
  if (pair) {
    const int smem = PSTAGES * 2 * kPairStage + 256 + 1024;
    cudaError_t e = cudaFuncSetAttribute(contract_bf16_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return cuda_status(e, "contract bf16 pair: smem attribute");
    const int64_t tiles = d->batch * ((d->m + PM - 1) / PM) * ((d->n + PN - 1) / PN);
    if (tiles > 0x7fffffffLL) return set_error(PDB_ERR_SHAPE, "contract bf16: too many tiles");
    // clusters of two that fit at once, per device (queried once, under a lock)
    static std::mutex mu;
    static int max_pairs[64] = {};
    int cap = sm_count(dev) / 2;
    if (dev >= 0 && dev < 64) {
      std::lock_guard<std::mutex> lk(mu);
      if (max_pairs[dev] == 0) {
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(2 * (unsigned)(sm_count(dev) / 2));
        cfg.blockDim = dim3(PTHREADS);
        cfg.dynamicSmemBytes = smem;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, contract_bf16_pair_kernel, &cfg) != cudaSuccess || n <= 0) {
          cudaGetLastError();
          n = sm_count(dev) / 2;
        }
        max_pairs[dev] = n;
      }
      cap = max_pairs[dev];
    }
    const int64_t pairs = tiles < cap ? tiles : cap;
    contract_bf16_pair_kernel<<<(unsigned)(2 * pairs), PTHREADS, smem, s>>>(ta, tb, p);
    return cuda_status(cudaGetLastError(), "contract bf16 pair launch");
  }
  const int smem = GSTAGES * (kStageA + kStageB) + 256 + 1024;
  cudaError_t e = cudaFuncSetAttribute(contract_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return cuda_status(e, "contract bf16: smem attribute");
  const int64_t tiles = d->batch * ((d->m + GM - 1) / GM) * ((d->n + GN - 1) / GN);
  if (tiles > 0x7fffffffLL) return set_error(PDB_ERR_SHAPE, "contract bf16: too many tiles");
  const int64_t grid = tiles < sm_count(dev) ? tiles : sm_count(dev);
  contract_bf16_kernel<<<(unsigned)grid, GTHREADS, smem, s>>>(ta, tb, p);
  return cuda_status(cudaGetLastError(), "contract bf16 launch");
}

extern "C" int pdb_pointwise_f32(const pdb_pointwise_desc* d, void* stream) {
  if (!d) return set_error(PDB_ERR_ARG, "null descriptor");
  if (d->batch < 0 || d->m < 0 || d->n < 0) return set_error(PDB_ERR_SHAPE, "pointwise: negative size");
  const int64_t total = d->batch * d->m * d->n;
  if (total == 0) return PDB_OK;
  if (!d->x || !d->y) return set_error(PDB_ERR_ARG, "null x / y");
  if (int st = check_ops(d->n_ops, d->ops)) return st;
  const EwProgram pg = make_program(d->n_ops, d->ops);
  int dev = 0;
  cudaGetDevice(&dev);
  const int64_t blocks = d->batch * d->m * ((d->n + kPwSeg - 1) / kPwSeg);
  const int64_t cap = (int64_t)sm_count(dev) * 8;
  PointwiseArgs a{d->x, d->y, d->batch, d->m, d->n, {d->x_stride[0], d->x_stride[1], d->x_stride[2]},
                  {d->y_stride[0], d->y_stride[1], d->y_stride[2]}};
  const bool aligned = ((reinterpret_cast<uintptr_t>(d->x) | reinterpret_cast<uintptr_t>(d->y)) & 15u) == 0;
  const int vec = aligned && d->x_stride[2] == 1 && d->y_stride[2] == 1 && ((d->x_stride[0] | d->x_stride[1] |
                  d->y_stride[0] | d->y_stride[1]) & 3) == 0;
  pointwise_f32_kernel<<<(unsigned)(blocks < cap ? blocks : cap), kPwThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      a, pg, vec);
  return cuda_status(cudaGetLastError(), "pointwise launch");
}
