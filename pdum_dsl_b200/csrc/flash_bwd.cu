// bf16 flash-attention backward for sm_100a (tcgen05 / TMEM / TMA).
//
// The reference obtains the backward by autodiff of the naive attention
// region (autodiff.py:102-150) and carves the joint with plan_model
// (partition.py:586-607) into: the flash forward with its (m, den)
// artifacts, a held-back D = rowsum(dO * O) row statistic, and contraction
// carves that re-derive P inside their sweep (partition.py:354-455).  This
// file executes that plan as:
//
//   bwd_prep     D[t] = sum_o dO[t,o] O[t,o] and nlse2[t] = -lse[t] * log2 e
//                (rows padded to a multiple of 128 with nlse2 = -inf, D = 0,
//                so padded query rows carry P = 0 without masks)
//   D = 64: bwd_fused64 (dK, dV and dQ in one persistent pass; dQ parts are
//                added into an fp32 accumulator in L2 by TMA bulk reductions)
//                and bwd_dq_convert (dQ = scale * accumulator, to bf16)
//   D = 128: bwd_dkdv128 and bwd_dq128, two persistent passes with 128-wide
//                items, so every score MMA is M = N = 128:
//   bwd_dkdv128  per (batch, KV head, 128-key block): for every 128-row query
//                tile of every query head of the group it forms S^T = K Q^T
//                and dP^T = V dO^T in TMEM, P^T = exp2(S^T c + nlse2) (bf16,
//                back to TMEM), dS^T = P^T (dP^T - D) (bf16, beside P^T in
//                TMEM; one thread per key row) and accumulates dV += P^T dO,
//                dK += dS^T Q in TMEM; GQA sums over the group in place.
//   bwd_dq128    per (batch, head, 128-row block): S = Q K^T, dP = dO V^T,
//                dS = P (dP - D), dQ += dS K over 128-key tiles.
// dQ = scale dS K, dK = scale dS^T Q; everything accumulates in fp32 (TMEM,
// and for the fused pass's dQ, fp32 in L2) and is rounded to bf16 once.  The
// D = 128 passes use no atomics (bit-reproducible); the fused pass's dQ sums
// its per-key-block parts in whatever order the reductions land.
#include <cfloat>
#include <mutex>
#include <utility>

#include "common.cuh"
#include "tma.h"

namespace pdb {
int flash_fwd_bf16_sm100(const pdb_flash_desc& d, cudaStream_t stream);
int validate_common(int64_t batch, int64_t hq, int64_t hkv, int64_t T, int64_t S, int64_t E, int64_t O,
                    int64_t q_start, const void* q, const void* k, const void* v);

namespace {

constexpr int BT = 128;  // query rows per tile
constexpr int kThreads = 384;  // warp0 TMA, warp1 MMA, warp2 TMEM, warps 4..11 two compute warpgroups
constexpr float kLog2e = 1.4426950408889634f;

struct BwdParams {
  const float* nlse2;  // -lse * log2 e, [B*H*Tpad]
  const float* dsum;  // [B*H*Tpad]
  void* out0;         // dkdv: dk ; dq: dq
  void* out1;         // dkdv: dv
  int64_t s0[3], s1[3];
  int T, S, H, HKV, Tpad;
  int q_start, causal;
  float scale, scale_log2;
  int n_blocks;  // key blocks (dkdv) or query blocks (dq) per head
  int B;
  int* ctr;      // work-unit counter of a persistent kernel (zeroed by the prologue)
  int* err;
  int ncols0, ncols1;  // true feature columns of out0 / out1 (<= D; the TMA maps zero-fill the rest)
};


// ---- MMA helpers.  Operand tiles are TMA boxes of 64 features x `rows` rows
// (128-byte swizzle), so a feature-chunk of 64 sits `rows * 128` bytes after
// the previous one.
// D (M x N) (+)= A (M x K=D, K-major smem) * B (N x K=D, K-major smem)^T
template <int D>
__device__ __forceinline__ void mma_kmajor(uint32_t d_tmem, uint32_t a_saddr, uint32_t a_box, uint32_t b_saddr,
                                           uint32_t b_box, uint32_t idesc) {
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const uint32_t o = (kk & 3) * 32;
    mma_ss(d_tmem, sdesc_sw128(a_saddr + (kk >> 2) * a_box + o, 16, 1024),
           sdesc_sw128(b_saddr + (kk >> 2) * b_box + o, 16, 1024), idesc, kk > 0);
  }
}

// rows of a TMEM accumulator (columns [c0, c0 + NC)) -> bf16 global, scaled
template <int NC>
__device__ __forceinline__ void store_cols_bf16(uint32_t t_src, float mul, __nv_bfloat16* row, bool store,
                                                int ncols = NC) {
#pragma unroll
  for (int ch = 0; ch < NC / 32; ++ch) {
    uint32_t r[32];
    tmem_ld32(t_src + ch * 32, r);
    tmem_wait_ld();
    uint32_t pk[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) pk[i] = pack_bf16(__uint_as_float(r[2 * i]) * mul, __uint_as_float(r[2 * i + 1]) * mul);
    if (store) {
      uint4* dst = reinterpret_cast<uint4*>(row + ch * 32);
#pragma unroll
      for (int i = 0; i < 4; ++i)  // columns past ncols are zero padding of the head dim: not stored
        if (ch * 32 + i * 8 < ncols) dst[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
    }
  }
}

// P, dS for 64 score columns held by one thread: p = exp2(s c + nl2), ds = p (dp - dsum).
// `valid(col)` masks causal positions; nl2 / dsum per column (dK/dV) or per row (dQ).
template <class ColL2, class ColDs, class Valid>
__device__ __forceinline__ void p_ds_64(const uint32_t (&sr)[64], const uint32_t (&dr)[64], float c, ColL2 l2,
                                        ColDs ds_of, Valid valid, uint32_t (&pp)[32], uint32_t (&dd)[32]) {
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    float pv[2], dv[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int col = 2 * i + u;
      float pr = ex2(fmaf(__uint_as_float(sr[col]), c, l2(col)));
      pr = valid(col) ? pr : 0.f;
      pv[u] = pr;
      dv[u] = pr * (__uint_as_float(dr[col]) - ds_of(col));
    }
    pp[i] = pack_bf16(pv[0], pv[1]);
    dd[i] = pack_bf16(dv[0], dv[1]);
  }
}

// Persistent scheduling of the backward kernels.  The work units (a 128-key
// block for dK/dV, a 128-row query block for dQ) differ in size under the
// causal mask (1 to n items); one CTA per unit left SMs idle ~40 % of the time
// (CTA start / drain gaps and the uneven tail).  Here one CTA per SM takes units
// from a global counter in descending size order (the counter lives in the
// workspace and is zeroed by the prologue kernel), and the producer hands each
// unit to the MMA thread and the compute warps through a two-slot queue in
// shared memory.  K/V (or Q/dO) of the next unit load while the current one
// runs; barrier phases follow running counters across units.
struct __align__(8) UnitQueue {
  uint64_t full[2], empty[2];  // producer -> consumers (1 MMA thread + 8 compute warps)
  int unit[2];
};

__device__ __forceinline__ int fetch_unit(UnitQueue* uq, uint32_t n, int u, volatile int* abort, int* err) {
  const int slot = n & 1;
  if (!mbar_wait(&uq->empty[slot], ((n >> 1) & 1) ^ 1, abort, err)) return -2;
  uq->unit[slot] = u;
  mbar_arrive(&uq->full[slot]);
  return u;
}
// consumer side: every compute warp (lane 0 after the warp converged) or the MMA thread
__device__ __forceinline__ int take_unit(UnitQueue* uq, uint32_t n, volatile int* abort, int* err, bool warp_wide) {
  const int slot = n & 1;
  if (!mbar_wait(&uq->full[slot], (n >> 1) & 1, abort, err)) return -2;
  const int u = *reinterpret_cast<volatile int*>(&uq->unit[slot]);
  if (warp_wide) __syncwarp();
  if (!warp_wide || (threadIdx.x & 31) == 0) mbar_arrive(&uq->empty[slot]);
  return u;
}

// ------------------------------------------------------------------ dK / dV
// dK / dV with 128-query items.  Unit = 128 keys of one (batch, KV head);
// items = (query head of the group, 128-row query tile), so the score MMAs
// run at N = 128.  TMEM: two 128-column slots take turns -- S^T of item g in
// slot g & 1, dP^T of item g in the other -- and dV [256, 384), dK [384, 512).
// The compute warpgroups split an item's queries (warpgroup x: queries
// [64x, 64x+64)).  Phase 1 forms P^T = exp2(S^T c + nlse2) and writes it
// (bf16 pairs) into its own first 32 columns of the S^T slot, the A operand of
// dV += P^T dO; phase 2 reads dP^T, whose slot is then free for S^T of the
// next item, and writes dS^T = P^T (dP^T - D) (bf16 pairs) into its other 32
// columns of the S^T slot, the A operand of dK += dS^T Q (both gradient MMAs
// take A from TMEM; dS^T in shared memory instead measured 0.5-1 % slower).
// Per item the MMA issuer sends
//   dV(g) [after P^T(g)], S^T(g+1) [once dP^T(g) is in registers],
//   dK(g) [after dS^T(g)], dP^T(g+1) [into the slot dV(g) read, behind it]
// dV(g) keeps the tensor core busy while the compute warps take dP^T(g) into
// registers, the hand-off the next score MMA waits for, and the next item's
// scores are formed while this item's gradients are.
// Q / dO (and the per-query nlse2 / D) pass through two stages each; Q is
// released by dK, dO by dV.
struct __align__(8) BarsK {
  uint64_t fixed_full, fixed_empty;  // K / V of the unit
  uint64_t q_full[2], q_empty[2];    // Q + nlse2 / D of an item
  uint64_t do_full[2], do_empty[2];
  uint64_t st_full[2], dpt_full[2];  // S^T(g), dP^T(g) complete
  uint64_t dp_free[2];               // dP^T(g) in registers (its slot may take S^T(g+1))
  uint64_t pt_full[2];               // P^T(g) written to TMEM
  uint64_t ds_full[2];               // dS^T(g) written to TMEM
  uint64_t o_full, acc_free;
  UnitQueue uq;
  uint32_t tmem_base;
  int abort;
};

constexpr int kKv128Tiles = 32768 * 6;                    // K, V, Q x 2, dO x 2
constexpr int kKv128Smem = kKv128Tiles + 2 * 256 * 4 + (int)sizeof(BarsK);  // + nlse2 / D per stage + barriers
constexpr int kMaxDynSmem = 227 * 1024;

__global__ void __launch_bounds__(kThreads, 1)
    bwd_dkdv128_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                       const BwdParams p) {
  constexpr int D = 128;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // the tiles need 1024-byte alignment and the launch has little slack above the layout:
  // refuse (error word, no access) rather than overrun if the window starts badly aligned
  if ((smem - smem_raw) + kKv128Smem > kMaxDynSmem) {
    if (threadIdx.x == 0 && p.err) atomicOr(p.err, kErrSmemWindow);
    return;
  }
  constexpr int kT = 128 * D * 2;
  constexpr uint32_t kBox = 128 * 128;
  uint8_t* sK = smem;
  uint8_t* sV = smem + kT;
  uint8_t* sQ = smem + 2 * kT;   // 2 stages
  uint8_t* sDO = smem + 4 * kT;  // 2 stages
  float* sVec = reinterpret_cast<float*>(smem + kKv128Tiles);  // per stage: nlse2[128], dsum[128]
  BarsK* bar = reinterpret_cast<BarsK*>(smem + kKv128Tiles + 2 * 256 * 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int group = p.H / p.HKV;
  const int n_qt = p.Tpad / 128;
  const int n_bh = p.B * p.HKV;
  const int n_units = p.n_blocks * n_bh;
  auto unit_info = [&](int u, int& b, int& hk, int& s0, int& qt0, int& per_head) {
    const int nblk = u / n_bh, bhk = u % n_bh;  // ascending key block = descending work (causal)
    b = bhk / p.HKV;
    hk = bhk % p.HKV;
    s0 = nblk * 128;
    qt0 = 0;
    if (p.causal) {
      const int first = s0 - p.q_start;  // first query row that can see key s0
      qt0 = first > 0 ? first / 128 : 0;
    }
    per_head = n_qt - qt0 > 0 ? n_qt - qt0 : 0;
  };

  if (threadIdx.x == 0) {
    mbar_init(&bar->fixed_full, 1);
    mbar_init(&bar->fixed_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar->q_full[i], 1);
      mbar_init(&bar->q_empty[i], 1);
      mbar_init(&bar->do_full[i], 1);
      mbar_init(&bar->do_empty[i], 1);
      mbar_init(&bar->st_full[i], 1);
      mbar_init(&bar->dpt_full[i], 1);
      mbar_init(&bar->dp_free[i], 8);  // one arrival per compute warp
      mbar_init(&bar->pt_full[i], 8);
      mbar_init(&bar->ds_full[i], 8);
      mbar_init(&bar->uq.full[i], 1);
      mbar_init(&bar->uq.empty[i], 9);  // the MMA thread + 8 compute warps
    }
    mbar_init(&bar->o_full, 1);
    mbar_init(&bar->acc_free, 8);
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
  grid_dep_wait();    // the prologue (D, nlse2, zeroed counters) has completed
  grid_dep_launch();  // the dQ grid may take SMs as this grid's CTAs retire
  const uint32_t tmem = bar->tmem_base;
  volatile int* abort = &bar->abort;
  constexpr int kNB = D / 64;
  constexpr uint32_t idS = idesc_bf16(128, 128, 0, 0);  // S^T, dP^T: M = 128 keys, N = 128 queries
  constexpr uint32_t idG = idesc_bf16(128, D, 0, 1);    // dV, dK: M = 128 keys, N = D, B MN-major
  constexpr uint32_t kDV = 256, kDK = 384;

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 80;" ::: "memory");
    if (warp == 0 && lane == 0) {
      // ---------------------------------------------------------- producer
      uint32_t gi = 0, nu = 0, nkv = 0;
      for (;; ++nu) {
        int u = atomicAdd(p.ctr, 1);
        if (u >= n_units) u = -1;
        if (fetch_unit(&bar->uq, nu, u, abort, p.err) < 0) break;
        int b, hk, s0, qt0, per_head;
        unit_info(u, b, hk, s0, qt0, per_head);
        const int n_items = per_head * group;
        if (n_items == 0) continue;
        if (!mbar_wait(&bar->fixed_empty, (nkv & 1) ^ 1, abort, p.err)) break;
        mbar_expect_tx(&bar->fixed_full, 2 * kT);
        for (int i = 0; i < kNB; ++i) {
          tma_load_4d(sK + i * kBox, &tm_k, &bar->fixed_full, i * 64, s0, hk, b);
          tma_load_4d(sV + i * kBox, &tm_v, &bar->fixed_full, i * 64, s0, hk, b);
        }
        ++nkv;
        bool ok = true;
        for (int it = 0; it < n_items; ++it, ++gi) {
          const int st = gi & 1;
          const uint32_t ph = ((gi >> 1) & 1) ^ 1;
          const int h = hk * group + it / per_head;
          const int t0 = (qt0 + it % per_head) * 128;
          if (!(ok = mbar_wait(&bar->q_empty[st], ph, abort, p.err))) break;
          mbar_expect_tx(&bar->q_full[st], kT + 2 * 128 * 4);
          for (int i = 0; i < kNB; ++i)
            tma_load_4d(sQ + st * kT + i * kBox, &tm_q, &bar->q_full[st], i * 64, t0, h, b);
          const int64_t vrow = ((int64_t)b * p.H + h) * p.Tpad + t0;
          bulk_load(sVec + st * 256, p.nlse2 + vrow, 128 * 4, &bar->q_full[st]);
          bulk_load(sVec + st * 256 + 128, p.dsum + vrow, 128 * 4, &bar->q_full[st]);
          if (!(ok = mbar_wait(&bar->do_empty[st], ph, abort, p.err))) break;
          mbar_expect_tx(&bar->do_full[st], kT);
          for (int i = 0; i < kNB; ++i)
            tma_load_4d(sDO + st * kT + i * kBox, &tm_do, &bar->do_full[st], i * 64, t0, h, b);
        }
        if (!ok) break;
      }
    } else if (warp == 1 && lane == 0) {
      // -------------------------------------------------------- MMA issuer
      uint32_t gi = 0, nu = 0, nkv = 0;
      bool ok = true;
      for (;; ++nu) {
        const int u = take_unit(&bar->uq, nu, abort, p.err, false);
        if (u < 0) break;
        int b, hk, s0, qt0, per_head;
        unit_info(u, b, hk, s0, qt0, per_head);
        const int n_items = per_head * group;
        if (n_items == 0) continue;
        auto issue_st = [&](int it) -> bool {  // S^T(g) into slot g & 1, once dP^T(g-1) left it
          const uint32_t g = gi + it;
          if (!mbar_wait(&bar->q_full[g & 1], (g >> 1) & 1, abort, p.err)) return false;
          if (g > 0 && !mbar_wait(&bar->dp_free[(g - 1) & 1], ((g - 1) >> 1) & 1, abort, p.err)) return false;
          tc_fence_after();
          mma_kmajor<D>(tmem + (g & 1) * 128, smem_u32(sK), kBox, smem_u32(sQ + (g & 1) * kT), kBox, idS);
          tc_commit(&bar->st_full[g & 1]);
          return true;
        };
        auto issue_dpt = [&](int it) -> bool {  // dP^T(g) into slot (g + 1) & 1
          const uint32_t g = gi + it;
          if (!mbar_wait(&bar->do_full[g & 1], (g >> 1) & 1, abort, p.err)) return false;
          tc_fence_after();
          mma_kmajor<D>(tmem + ((g + 1) & 1) * 128, smem_u32(sV), kBox, smem_u32(sDO + (g & 1) * kT), kBox, idS);
          tc_commit(&bar->dpt_full[g & 1]);
          if (it == n_items - 1) tc_commit(&bar->fixed_empty);  // K/V no longer needed: load the next unit's
          return true;
        };
        if (!(ok = mbar_wait(&bar->fixed_full, nkv & 1, abort, p.err))) break;
        ok = issue_st(0) && issue_dpt(0);
        for (int it = 0; ok && it < n_items; ++it) {
          const uint32_t g = gi + it;
          const int st = g & 1;
          // dV(g) first: it needs only phase 1, so it runs while the compute warps take dP^T(g)
          // into registers and the next score MMA waits for that slot
          if (!(ok = mbar_wait(&bar->pt_full[st], (g >> 1) & 1, abort, p.err))) break;
          if (it == 0 && nkv > 0 && !(ok = mbar_wait(&bar->acc_free, (nkv - 1) & 1, abort, p.err))) break;
          tc_fence_after();
          const uint32_t bq = smem_u32(sQ + st * kT), bdo = smem_u32(sDO + st * kT);
          const uint32_t a = tmem + st * 128;  // P^T of queries [0, 64) in columns [0, 32), [64, 128) in [64, 96)
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)  // dV += P^T dO
            mma_ts(tmem + kDV, a + (kk >> 2) * 64 + (kk & 3) * 8, sdesc_sw128(bdo + kk * 2048, kBox, 1024), idG,
                   (it > 0 || kk > 0) ? 1u : 0u);
          tc_commit(&bar->do_empty[st]);
          if (it + 1 < n_items && !(ok = issue_st(it + 1))) break;
          if (!(ok = mbar_wait(&bar->ds_full[st], (g >> 1) & 1, abort, p.err))) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)  // dK += dS^T Q, dS^T beside P^T in the slot
            mma_ts(tmem + kDK, a + (kk >> 2) * 64 + 32 + (kk & 3) * 8, sdesc_sw128(bq + kk * 2048, kBox, 1024), idG,
                   (it > 0 || kk > 0) ? 1u : 0u);
          tc_commit(&bar->q_empty[st]);
          if (it + 1 < n_items && !(ok = issue_dpt(it + 1))) break;
        }
        if (!ok) break;
        tc_commit(&bar->o_full);
        gi += n_items;
        ++nkv;
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 208;" ::: "memory");
    const int x = warp >= 8 ? 1 : 0;  // queries [64x, 64x + 64) of every item
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;  // key row within the block (TMEM lane)
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const uint64_t c2 = f2_pack(p.scale_log2, p.scale_log2);
    uint32_t gi = 0, nu = 0, nkv = 0;
    bool ok = true;
    for (;; ++nu) {
      const int u = take_unit(&bar->uq, nu, abort, p.err, true);
      if (u < 0) break;
      int b, hk, s0, qt0, per_head;
      unit_info(u, b, hk, s0, qt0, per_head);
      const int n_items = per_head * group;
      const int s = s0 + row;
      for (int it = 0; it < n_items; ++it) {
        const uint32_t g = gi + it;
        const int st = g & 1;
        const uint32_t ph = (g >> 1) & 1;
        const int t0 = (qt0 + it % per_head) * 128;
        if (!(ok = mbar_wait(&bar->q_full[st], ph, abort, p.err))) break;
        if (!(ok = mbar_wait(&bar->st_full[st], ph, abort, p.err))) break;
        tc_fence_after();
        const int lo = p.causal ? s - p.q_start - t0 - x * 64 : -(1 << 30);  // query columns below lo are masked
        const bool need_mask = __any_sync(0xffffffffu, lo > 0);
        const uint32_t sl = smem_u32(sVec + st * 256 + x * 64), sd = smem_u32(sVec + st * 256 + 128 + x * 64);
        // phase 1: P^T = exp2(S^T c + nlse2), kept in registers as f32 and written to TMEM as bf16
        uint32_t pr[64];
        {
          const uint32_t ts = tmem + lane_off + st * 128 + x * 64;
          tmem_ld32(ts, *reinterpret_cast<uint32_t(*)[32]>(pr));
          tmem_ld32(ts + 32, *reinterpret_cast<uint32_t(*)[32]>(pr + 32));
          tmem_wait_ld();
          uint32_t pp[32];
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const float4 l4 = lds128(sl + 16 * q);
#pragma unroll
            for (int h2 = 0; h2 < 2; ++h2) {
              const int cc = 4 * q + 2 * h2;
              const uint64_t s2 = (uint64_t)pr[cc] | ((uint64_t)pr[cc + 1] << 32);
              const uint64_t l2 = h2 ? f2_pack(l4.z, l4.w) : f2_pack(l4.x, l4.y);
              float x0, x1;
              f2_unpack(f2_fma(s2, c2, l2), x0, x1);
              float p0 = ex2(x0), p1 = ex2(x1);
              if (need_mask) {
                p0 = cc >= lo ? p0 : 0.f;
                p1 = cc + 1 >= lo ? p1 : 0.f;
              }
              pr[cc] = __float_as_uint(p0);
              pr[cc + 1] = __float_as_uint(p1);
              pp[2 * q + h2] = pack_bf16(p0, p1);
            }
          }
          tmem_st32(ts, pp);
          tmem_wait_st();
          warp_arrive_after_tc(&bar->pt_full[st]);
        }
        // phase 2: dS^T = P^T (dP^T - D) to TMEM
        if (!(ok = mbar_wait(&bar->dpt_full[st], ph, abort, p.err))) break;
        tc_fence_after();
        uint32_t dr[64];
        {
          const uint32_t td = tmem + lane_off + ((g + 1) & 1) * 128 + x * 64;
          tmem_ld32(td, *reinterpret_cast<uint32_t(*)[32]>(dr));
          tmem_ld32(td + 32, *reinterpret_cast<uint32_t(*)[32]>(dr + 32));
          tmem_wait_ld();
          warp_arrive_after_tc(&bar->dp_free[st]);
        }
        uint32_t dd[32];
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const float4 d4 = lds128(sd + 16 * q);
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            const int cc = 4 * q + 2 * h2;
            const uint64_t p2 = (uint64_t)pr[cc] | ((uint64_t)pr[cc + 1] << 32);
            const uint64_t g2 = (uint64_t)dr[cc] | ((uint64_t)dr[cc + 1] << 32);
            const uint64_t dd2 = h2 ? f2_pack(d4.z, d4.w) : f2_pack(d4.x, d4.y);
            float g0, g1;
            f2_unpack(f2_mul(p2, f2_sub(g2, dd2)), g0, g1);
            dd[2 * q + h2] = pack_bf16(g0, g1);
          }
        }
        tmem_st32(tmem + lane_off + st * 128 + x * 64 + 32, dd);  // its other 32 columns of the S^T slot
        tmem_wait_st();
        warp_arrive_after_tc(&bar->ds_full[st]);
      }
      if (!ok) break;
      const bool store = s < p.S;
      // warpgroup 0 writes dV, warpgroup 1 writes dK
      __nv_bfloat16* dst = x == 0
          ? static_cast<__nv_bfloat16*>(p.out1) + (int64_t)b * p.s1[0] + (int64_t)hk * p.s1[1] + (int64_t)s * p.s1[2]
          : static_cast<__nv_bfloat16*>(p.out0) + (int64_t)b * p.s0[0] + (int64_t)hk * p.s0[1] + (int64_t)s * p.s0[2];
      if (n_items == 0) {  // a key block past every query row: dK = dV = 0
        if (store)
          for (int i = 0; i < (x == 0 ? p.ncols1 : p.ncols0); i += 8)
            *reinterpret_cast<uint4*>(dst + i) = make_uint4(0, 0, 0, 0);
        continue;
      }
      if (!(ok = mbar_wait(&bar->o_full, nkv & 1, abort, p.err))) break;
      tc_fence_after();
      store_cols_bf16<D>(tmem + lane_off + (x == 0 ? kDV : kDK), x == 0 ? 1.0f : p.scale, dst, store,
                         x == 0 ? p.ncols1 : p.ncols0);
      warp_arrive_after_tc(&bar->acc_free);
      gi += n_items;
      ++nkv;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// dQ with 128-key items.  Unit = 128 query rows of one (batch, head); items =
// 128-key tiles, so both score MMAs run at N = 128.  TMEM: S of item g in slot
// g & 1 ([0,128) or [128,256)), dP of every item in [256,384), dQ in
// [384,512).  The two compute warpgroups split an item's keys (warpgroup x:
// keys [64x, 64x+64)) and write their dS (bf16 pairs) into their own first 32
// columns of the item's S slot, where dQ += dS K reads it.  Because dP has a
// slot of its own that is free as soon as the compute warps hold dP in
// registers, the tensor core runs dQ(g-1), S(g+1) and dP(g+1) while item g's
// exponentials are formed: per item the MMA issuer sends
//   dP(g+1) [after item g's dP is in registers], dQ(g) [after dS(g)], S(g+2)
// and S(g+2) overwrites the slot dQ(g) read, issued behind it.
// K stays resident until its dQ completes (three stages), V until its dP (two).
struct __align__(8) BarsQ {
  uint64_t fixed_full, fixed_empty;  // Q / dO of the unit
  uint64_t k_full[3], k_empty[3];
  uint64_t v_full[2], v_empty[2];
  uint64_t s_full[2];   // S(g), dP(g) complete
  uint64_t dp_free[2];  // compute warps hold dP(g) (and S(g)) in registers
  uint64_t p_full[2];   // dS(g) written to TMEM
  uint64_t o_full, acc_free;
  UnitQueue uq;
  uint32_t tmem_base;
  int abort;
};

constexpr int kDq128KStages = 3, kDq128VStages = 2;
constexpr int kDq128Smem = 2 * 32768 + (kDq128KStages + kDq128VStages) * 32768;  // + barriers + alignment

__global__ void __launch_bounds__(kThreads, 1)
    bwd_dq128_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                     const BwdParams p) {
  constexpr int D = 128;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int kT = 128 * D * 2;  // one 128-row tile of Q, dO, K or V
  constexpr uint32_t kBox = 128 * 128;
  uint8_t* sQ = smem;
  uint8_t* sDO = smem + kT;
  uint8_t* sK = smem + 2 * kT;                    // kDq128KStages
  uint8_t* sV = sK + kDq128KStages * kT;          // kDq128VStages
  BarsQ* bar = reinterpret_cast<BarsQ*>(sV + kDq128VStages * kT);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_bh = p.B * p.H;
  const int n_units = p.n_blocks * n_bh;
  const int n_all = (p.S + 127) / 128;
  auto unit_info = [&](int u, int& b, int& h, int& t0, int& n_kv) {
    const int mblk = p.n_blocks - 1 - u / n_bh, bh = u % n_bh;  // heaviest first
    b = bh / p.H;
    h = bh % p.H;
    t0 = mblk * 128;
    n_kv = n_all;
    if (p.causal) {
      int last = t0 + 127;
      if (last > p.T - 1) last = p.T - 1;
      const int n = (last + p.q_start) / 128 + 1;
      n_kv = n < n_all ? (n > 0 ? n : 0) : n_all;
    }
  };

  if (threadIdx.x == 0) {
    mbar_init(&bar->fixed_full, 1);
    mbar_init(&bar->fixed_empty, 1);
    for (int i = 0; i < kDq128KStages; ++i) {
      mbar_init(&bar->k_full[i], 1);
      mbar_init(&bar->k_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar->v_full[i], 1);
      mbar_init(&bar->v_empty[i], 1);
      mbar_init(&bar->s_full[i], 1);
      mbar_init(&bar->dp_free[i], 8);  // one arrival per compute warp
      mbar_init(&bar->p_full[i], 8);
      mbar_init(&bar->uq.full[i], 1);
      mbar_init(&bar->uq.empty[i], 9);
    }
    mbar_init(&bar->o_full, 1);
    mbar_init(&bar->acc_free, 8);
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
  constexpr int kNB = D / 64;
  constexpr uint32_t idS = idesc_bf16(128, 128, 0, 0);  // S, dP: M = 128 rows, N = 128 keys
  constexpr uint32_t idG = idesc_bf16(128, D, 0, 1);    // dQ: N = D, B = K tile MN-major
  constexpr uint32_t kDP = 256, kDQ = 384;              // TMEM columns

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 80;" ::: "memory");
    if (warp == 0 && lane == 0) {
      // ---------------------------------------------------------- producer
      uint32_t gi = 0, nu = 0, nqd = 0;
      for (;; ++nu) {
        int u = atomicAdd(p.ctr + 1, 1);
        if (u >= n_units) u = -1;
        if (fetch_unit(&bar->uq, nu, u, abort, p.err) < 0) break;
        int b, h, t0, n_kv;
        unit_info(u, b, h, t0, n_kv);
        if (n_kv == 0) continue;
        const int hk = h / (p.H / p.HKV);
        if (!mbar_wait(&bar->fixed_empty, (nqd & 1) ^ 1, abort, p.err)) break;
        mbar_expect_tx(&bar->fixed_full, 2 * kT);
        for (int i = 0; i < kNB; ++i) {
          tma_load_4d(sQ + i * kBox, &tm_q, &bar->fixed_full, i * 64, t0, h, b);
          tma_load_4d(sDO + i * kBox, &tm_do, &bar->fixed_full, i * 64, t0, h, b);
        }
        ++nqd;
        bool ok = true;
        for (int j = 0; j < n_kv; ++j, ++gi) {
          const int ks = gi % kDq128KStages, vs = gi & 1;
          if (!(ok = mbar_wait(&bar->k_empty[ks], ((gi / kDq128KStages) & 1) ^ 1, abort, p.err))) break;
          mbar_expect_tx(&bar->k_full[ks], kT);
          for (int i = 0; i < kNB; ++i)
            tma_load_4d(sK + ks * kT + i * kBox, &tm_k, &bar->k_full[ks], i * 64, j * 128, hk, b);
          if (!(ok = mbar_wait(&bar->v_empty[vs], ((gi >> 1) & 1) ^ 1, abort, p.err))) break;
          mbar_expect_tx(&bar->v_full[vs], kT);
          for (int i = 0; i < kNB; ++i)
            tma_load_4d(sV + vs * kT + i * kBox, &tm_v, &bar->v_full[vs], i * 64, j * 128, hk, b);
        }
        if (!ok) break;
      }
    } else if (warp == 1 && lane == 0) {
      // -------------------------------------------------------- MMA issuer
      uint32_t gi = 0, nu = 0, nqd = 0;
      bool ok = true;
      for (;; ++nu) {
        const int u = take_unit(&bar->uq, nu, abort, p.err, false);
        if (u < 0) break;
        int b, h, t0, n_kv;
        unit_info(u, b, h, t0, n_kv);
        if (n_kv == 0) continue;
        auto issue_s = [&](int j) -> bool {  // S(g) into slot g & 1
          const uint32_t g = gi + j;
          const int ks = g % kDq128KStages;
          if (!mbar_wait(&bar->k_full[ks], (g / kDq128KStages) & 1, abort, p.err)) return false;
          tc_fence_after();
          mma_kmajor<D>(tmem + (g & 1) * 128, smem_u32(sQ), kBox, smem_u32(sK + ks * kT), kBox, idS);
          return true;
        };
        auto issue_dp = [&](int j) -> bool {  // dP(g) into [256, 384) once item g-1's dP is in registers
          const uint32_t g = gi + j;
          const int vs = g & 1;
          if (!mbar_wait(&bar->v_full[vs], (g >> 1) & 1, abort, p.err)) return false;
          if (g > 0 && !mbar_wait(&bar->dp_free[(g - 1) & 1], ((g - 1) >> 1) & 1, abort, p.err)) return false;
          tc_fence_after();
          mma_kmajor<D>(tmem + kDP, smem_u32(sDO), kBox, smem_u32(sV + vs * kT), kBox, idS);
          tc_commit(&bar->v_empty[vs]);
          tc_commit(&bar->s_full[g & 1]);
          if (j == n_kv - 1) tc_commit(&bar->fixed_empty);  // Q / dO no longer needed: load the next unit's
          return true;
        };
        if (!(ok = mbar_wait(&bar->fixed_full, nqd & 1, abort, p.err))) break;
        ok = issue_s(0) && issue_dp(0);
        if (ok && n_kv > 1) ok = issue_s(1);
        for (int j = 0; ok && j < n_kv; ++j) {
          const uint32_t g = gi + j;
          if (j + 1 < n_kv && !(ok = issue_dp(j + 1))) break;
          if (!(ok = mbar_wait(&bar->p_full[g & 1], (g >> 1) & 1, abort, p.err))) break;
          if (j == 0 && nqd > 0 && !(ok = mbar_wait(&bar->acc_free, (nqd - 1) & 1, abort, p.err))) break;
          tc_fence_after();
          // dQ += dS K: dS of keys [0, 64) in the slot's columns [0, 32), of keys [64, 128) in [64, 96)
          const uint32_t a = tmem + (g & 1) * 128;
          const uint32_t bk = smem_u32(sK + (g % kDq128KStages) * kT);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_ts(tmem + kDQ, a + (kk >> 2) * 64 + (kk & 3) * 8, sdesc_sw128(bk + kk * 2048, kBox, 1024), idG,
                   (j > 0 || kk > 0) ? 1u : 0u);
          tc_commit(&bar->k_empty[g % kDq128KStages]);
          if (j + 2 < n_kv) ok = issue_s(j + 2);
        }
        if (!ok) break;
        tc_commit(&bar->o_full);
        gi += n_kv;
        ++nqd;
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 208;" ::: "memory");
    const int x = warp >= 8 ? 1 : 0;  // keys [64x, 64x + 64) of every item
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const float c = p.scale_log2;
    uint32_t gi = 0, nu = 0, nqd = 0;
    bool ok = true;
    for (;; ++nu) {
      const int u = take_unit(&bar->uq, nu, abort, p.err, true);
      if (u < 0) break;
      int b, h, t0, n_kv;
      unit_info(u, b, h, t0, n_kv);
      const int t = t0 + row;
      __nv_bfloat16* dq = static_cast<__nv_bfloat16*>(p.out0) + (int64_t)b * p.s0[0] + (int64_t)h * p.s0[1] +
                          (int64_t)t * p.s0[2];
      if (n_kv == 0) {  // no key is visible to these rows: dQ = 0
        if (t < p.T)
          for (int i = 0; i < D / 2; i += 8) *reinterpret_cast<uint4*>(dq + x * (D / 2) + i) = make_uint4(0, 0, 0, 0);
        continue;
      }
      const int64_t vrow = ((int64_t)b * p.H + h) * p.Tpad + t;
      const float l2 = p.nlse2[vrow];  // -inf on padded rows -> P = 0
      const float dsum = p.dsum[vrow];
      for (int j = 0; j < n_kv; ++j) {
        const uint32_t g = gi + j;
        if (!(ok = mbar_wait(&bar->s_full[g & 1], (g >> 1) & 1, abort, p.err))) break;
        tc_fence_after();
        const uint32_t ts = tmem + lane_off + (g & 1) * 128 + x * 64;
        const uint32_t td = tmem + lane_off + kDP + x * 64;
        const int lim = p.causal ? t + p.q_start + 1 - j * 128 - x * 64 : (1 << 30);  // key columns >= lim masked
        uint32_t sr[64], dr[64];
        tmem_ld32(ts, *reinterpret_cast<uint32_t(*)[32]>(sr));
        tmem_ld32(ts + 32, *reinterpret_cast<uint32_t(*)[32]>(sr + 32));
        tmem_ld32(td, *reinterpret_cast<uint32_t(*)[32]>(dr));
        tmem_ld32(td + 32, *reinterpret_cast<uint32_t(*)[32]>(dr + 32));
        tmem_wait_ld();
        warp_arrive_after_tc(&bar->dp_free[g & 1]);
        uint32_t pp[32], dd[32];
        p_ds_64(sr, dr, c, [&](int) { return l2; }, [&](int) { return dsum; }, [&](int col) { return col < lim; }, pp,
                dd);
        tmem_st32(ts, dd);
        tmem_wait_st();
        warp_arrive_after_tc(&bar->p_full[g & 1]);
      }
      if (!ok) break;
      if (!(ok = mbar_wait(&bar->o_full, nqd & 1, abort, p.err))) break;
      tc_fence_after();
      // each warpgroup writes half of the dQ columns
      store_cols_bf16<D / 2>(tmem + lane_off + kDQ + x * (D / 2), p.scale, dq + x * (D / 2), t < p.T,
                             p.ncols0 - x * (D / 2));
      warp_arrive_after_tc(&bar->acc_free);
      gi += n_kv;
      ++nqd;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  grid_dep_wait();  // complete only after the dK/dV grid this one overlapped has completed
}

// ---------------------------------------------------------------------------
// Fused D = 64 backward: dK, dV and dQ in one persistent pass.
// Unit = 128 keys of one (batch, KV head), taken by one CTA per SM from a
// global counter, heaviest first; items = (query head of the group, 128-row
// query tile).  Per item the tensor core forms S^T = K Q^T and dP^T = V dO^T
// (N = 128) in TMEM; the compute warpgroups (one thread per key row, each
// warpgroup 64 of the 128 query columns) form P^T and dS^T = P^T (dP^T - D);
// P^T goes to a TMEM staging area (A operand of dV += P^T dO) and dS^T to
// shared memory (bf16, 128-byte swizzled rows of 64 queries per key), where it
// serves as the K-major A operand of dK += dS^T Q and, read the other way, as
// the MN-major A operand of dQ_part = dS K.  The scores and exponentials are
// thus formed once for all three gradients.  dQ_part lands in its own TMEM
// columns; four drain warps read it out, stage it in shared memory and add it
// into an fp32 dQ accumulator in the workspace with TMA bulk reductions
// (performed in L2; the accumulator of config-5-sized problems fits there),
// and at the end of each unit store dV and dK (bf16) with TMA stores.  The
// next item's scores are issued as soon as S / dP sit in registers, and the
// next unit's first scores at the current unit's last item.  A final kernel
// scales and rounds the accumulator to bf16.  dQ then depends on the order of
// the fp32 additions (not bit-reproducible run to run); dK and dV do not.
constexpr int kStagesF = 3;
constexpr int kFusedThreads = 512;  // warps 0..3 control, 4..11 compute, 12..15 dQ drain

struct __align__(8) BarsF {
  uint64_t fixed_full[2], fixed_empty[2];          // K/V per buffer
  uint64_t op_full[kStagesF], op_empty[kStagesF];  // Q/dO ring
  uint64_t s_full, s_free, p_full, stage_free, o_full, acc_free;
  uint64_t dq_full, dq_free;                       // dQ_part in TMEM -> drain warps
  UnitQueue uq;
  uint32_t tmem_base;
  int abort;
};

// TMEM: S^T [0,128)  dP^T [128,256)  staging P^T [256,320)  dQ_part [320,384)
// dV [384,448)  dK [448,512).  Shared memory: K/V x 2 buffers, Q/dO x
// kStagesF, dS^T (two 16 KB halves of 64 queries), dQ staging (four 4 KB
// boxes, one per drain warp), nlse2/dsum rows.
__global__ void __launch_bounds__(kFusedThreads, 1)
    bwd_fused64_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                       const __grid_constant__ CUtensorMap tm_dqacc, const __grid_constant__ CUtensorMap tm_dk,
                       const __grid_constant__ CUtensorMap tm_dv, const BwdParams p) {
  constexpr int D = 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int kT = 128 * D * 2;  // any 128-row bf16 tile (16 KB)
  constexpr uint32_t kBox = 128 * 128;
  uint8_t* sKV = smem;                       // 2 buffers x (K, V)
  uint8_t* sQ = smem + 4 * kT;               // kStagesF
  uint8_t* sDO = sQ + kStagesF * kT;         // kStagesF
  uint8_t* sDS = sDO + kStagesF * kT;        // dS^T, 2 x 16 KB
  uint8_t* sDQ = sDS + 2 * kT;               // dQ staging, one 16 KB box
  float* sVec = reinterpret_cast<float*>(sDQ + kT);  // kStagesF x (nlse2[128], dsum[128])
  BarsF* bar = reinterpret_cast<BarsF*>(reinterpret_cast<uint8_t*>(sVec) + kStagesF * 2 * 128 * 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int group = p.H / p.HKV;
  const int n_qt = p.Tpad / 128;
  const int n_bh = p.B * p.HKV;
  const int n_units = p.n_blocks * n_bh;
  auto unit_info = [&](int u, int& b, int& hk, int& s0, int& qt0, int& per_head) {
    const int nblk = u / n_bh, bhk = u % n_bh;
    b = bhk / p.HKV;
    hk = bhk % p.HKV;
    s0 = nblk * 128;
    qt0 = 0;
    if (p.causal) {
      const int first = s0 - p.q_start;
      qt0 = first > 0 ? first / 128 : 0;
    }
    per_head = n_qt - qt0 > 0 ? n_qt - qt0 : 0;
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar->fixed_full[i], 1);
      mbar_init(&bar->fixed_empty[i], 1);
      mbar_init(&bar->uq.full[i], 1);
      mbar_init(&bar->uq.empty[i], 13);  // the MMA thread + 8 compute warps + 4 drain warps
    }
    for (int i = 0; i < kStagesF; ++i) {
      mbar_init(&bar->op_full[i], 1);
      mbar_init(&bar->op_empty[i], 1);
    }
    mbar_init(&bar->s_full, 1);
    mbar_init(&bar->s_free, 8);
    mbar_init(&bar->p_full, 8);
    mbar_init(&bar->stage_free, 1);
    mbar_init(&bar->o_full, 1);
    mbar_init(&bar->acc_free, 4);  // drain warps: dV / dK read out of TMEM
    mbar_init(&bar->dq_full, 1);
    mbar_init(&bar->dq_free, 4);   // drain warps: dQ_part in registers
    bar->abort = 0;
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc(&bar->tmem_base, 512);
    tmem_relinquish();
  }
  if (warp == 3 && lane == 0) {
    prefetch_tensormap(&tm_q);
    prefetch_tensormap(&tm_do);
    prefetch_tensormap(&tm_k);
    prefetch_tensormap(&tm_v);
    prefetch_tensormap(&tm_dqacc);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  grid_dep_wait();  // the prologue (D, nlse2, zeroed counters and dQ accumulator) has completed
  const uint32_t tmem = bar->tmem_base;
  volatile int* abort = &bar->abort;
  constexpr uint32_t idS = idesc_bf16(128, 128, 0, 0);
  constexpr uint32_t idG = idesc_bf16(128, D, 0, 1);   // dV, dK: A K-major (TMEM / smem), B MN-major
  constexpr uint32_t idQ = idesc_bf16(128, D, 1, 1);   // dQ: A = dS MN-major (smem), B = K MN-major

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 80;" ::: "memory");  // 128 x 80 + 256 x 176 + 128 x 80 = 65536
    if (warp == 0 && lane == 0) {
      // ---------------------------------------------------------- producer
      uint32_t gi = 0, nu = 0, nkv = 0;
      for (;; ++nu) {
        int u = atomicAdd(p.ctr, 1);
        if (u >= n_units) u = -1;
        if (fetch_unit(&bar->uq, nu, u, abort, p.err) < 0) break;
        int b, hk, s0, qt0, per_head;
        unit_info(u, b, hk, s0, qt0, per_head);
        const int n_items = per_head * group;
        if (n_items == 0) continue;
        const int kb = nkv & 1;
        if (!mbar_wait(&bar->fixed_empty[kb], ((nkv >> 1) & 1) ^ 1, abort, p.err)) break;
        mbar_expect_tx(&bar->fixed_full[kb], 2 * kT);
        tma_load_4d(sKV + kb * 2 * kT, &tm_k, &bar->fixed_full[kb], 0, s0, hk, b);
        tma_load_4d(sKV + kb * 2 * kT + kT, &tm_v, &bar->fixed_full[kb], 0, s0, hk, b);
        ++nkv;
        bool ok = true;
        for (int it = 0; it < n_items; ++it, ++gi) {
          const int st = gi % kStagesF;
          const int h = hk * group + it / per_head;
          const int t0 = (qt0 + it % per_head) * 128;
          if (!(ok = mbar_wait(&bar->op_empty[st], ((gi / kStagesF) & 1) ^ 1, abort, p.err))) break;
          mbar_expect_tx(&bar->op_full[st], 2 * kT + 2 * 128 * 4);
          tma_load_4d(sQ + st * kT, &tm_q, &bar->op_full[st], 0, t0, h, b);
          tma_load_4d(sDO + st * kT, &tm_do, &bar->op_full[st], 0, t0, h, b);
          const int64_t vrow = ((int64_t)b * p.H + h) * p.Tpad + t0;
          bulk_load(sVec + st * 256, p.nlse2 + vrow, 512, &bar->op_full[st]);
          bulk_load(sVec + st * 256 + 128, p.dsum + vrow, 512, &bar->op_full[st]);
        }
        if (!ok) break;
      }
    } else if (warp == 1 && lane == 0) {
      // -------------------------------------------------------- MMA issuer
      // The scores of the next unit's first item are issued at the last item of
      // the current one (its K/V are already resident), so the compute warps
      // move from unit to unit without waiting for the tensor core to drain.
      uint32_t gi = 0, nu = 0, nkv = 0;
      bool ok = true;
      const uint32_t sDSa = smem_u32(sDS);
      int b, hk, s0, qt0, per_head, n_items = 0;
      // the next unit that has items (units without any are taken and skipped)
      auto next_unit = [&](int& ub, int& uhk, int& us0, int& uqt0, int& uper, int& un) -> int {
        for (;;) {
          const int u = take_unit(&bar->uq, nu++, abort, p.err, false);
          if (u < 0) return u;  // -1: no more units, -2: gave up waiting
          unit_info(u, ub, uhk, us0, uqt0, uper);
          un = uper * group;
          if (un > 0) return u;
        }
      };
      auto issue_s = [&](uint32_t g, uint32_t sK, uint32_t sV) -> bool {
        const int st = g % kStagesF;
        if (!mbar_wait(&bar->op_full[st], (g / kStagesF) & 1, abort, p.err)) return false;
        tc_fence_after();
        // shared-memory descriptors advance by (byte offset >> 4) in their address field
        const uint64_t dk = sdesc_sw128(sK, 16, 1024), dv = sdesc_sw128(sV, 16, 1024);
        const uint64_t dq = sdesc_sw128(smem_u32(sQ + st * kT), 16, 1024);
        const uint64_t ddo = sdesc_sw128(smem_u32(sDO + st * kT), 16, 1024);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)  // S^T = K Q^T
          mma_ss(tmem + 0, dk + 2 * kk, dq + 2 * kk, idS, kk > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)  // dP^T = V dO^T
          mma_ss(tmem + 128, dv + 2 * kk, ddo + 2 * kk, idS, kk > 0 ? 1u : 0u);
        tc_commit(&bar->s_full);
        return true;
      };
      int cur = next_unit(b, hk, s0, qt0, per_head, n_items);
      if (cur >= 0) {
        if ((ok = mbar_wait(&bar->fixed_full[0], 0, abort, p.err))) ok = issue_s(0, smem_u32(sKV), smem_u32(sKV) + kT);
      }
      while (ok && cur >= 0) {
        const int kb = nkv & 1;
        const uint32_t sK = smem_u32(sKV + kb * 2 * kT);
        int nb = 0, nhk = 0, ns0 = 0, nqt0 = 0, nper = 0, nn = 0, nxt = -1;
        for (int it = 0; ok && it < n_items; ++it) {
          const uint32_t g = gi + it;
          const int st = g % kStagesF;
          if (it + 1 < n_items) {  // the next item's scores once this item's S / dP sit in registers
            if (!(ok = mbar_wait(&bar->s_free, g & 1, abort, p.err))) break;
            tc_fence_after();
            if (!(ok = issue_s(g + 1, sK, sK + kT))) break;
          } else {  // last item: the next unit's first scores, on its (prefetched) K / V
            nxt = next_unit(nb, nhk, ns0, nqt0, nper, nn);
            if (nxt == -2) {
              ok = false;
              break;
            }
            if (nxt >= 0) {
              const int nkb = (nkv + 1) & 1;
              if (!(ok = mbar_wait(&bar->fixed_full[nkb], ((nkv + 1) >> 1) & 1, abort, p.err))) break;
              if (!(ok = mbar_wait(&bar->s_free, g & 1, abort, p.err))) break;
              tc_fence_after();
              const uint32_t nK = smem_u32(sKV + nkb * 2 * kT);
              if (!(ok = issue_s(g + 1, nK, nK + kT))) break;
            }
          }
          if (!(ok = mbar_wait(&bar->p_full, g & 1, abort, p.err))) break;
          // dV / dK of the previous unit must be read out before this unit's first accumulation
          if (it == 0 && nkv > 0 && !(ok = mbar_wait(&bar->acc_free, (nkv - 1) & 1, abort, p.err))) break;
          tc_fence_after();
          const uint32_t sQst = smem_u32(sQ + st * kT), sDOst = smem_u32(sDO + st * kT);
          const uint64_t bdo = sdesc_sw128(sDOst, kBox, 1024), bq = sdesc_sw128(sQst, kBox, 1024);
          const uint64_t ads = sdesc_sw128(sDSa, 16, 1024);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)  // dV += P^T dO  (A: P^T in TMEM, B: dO MN-major, 16 rows = 2048 B per step)
            mma_ts(tmem + 384, tmem + 256 + kk * 8, bdo + 128 * kk, idG, (it > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)  // dK += dS^T Q  (A: dS^T K-major, two 64-query halves)
            mma_ss(tmem + 448, ads + (kk >> 2) * (kT >> 4) + (kk & 3) * 2, bq + 128 * kk, idG,
                   (it > 0 || kk > 0) ? 1u : 0u);
          // dQ_part = dS K once the drain holds the previous item's part in registers
          if (g > 0 && !(ok = mbar_wait(&bar->dq_free, (g - 1) & 1, abort, p.err))) break;
          tc_fence_after();
          const uint64_t adq = sdesc_sw128(sDSa, kT, 1024), bk = sdesc_sw128(sK, kBox, 1024);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)  // A: dS MN-major (query halves 16 KB apart), B: K MN-major
            mma_ss(tmem + 320, adq + 128 * kk, bk + 128 * kk, idQ, kk > 0 ? 1u : 0u);
          tc_commit(&bar->op_empty[st]);
          tc_commit(&bar->stage_free);
          tc_commit(&bar->dq_full);
        }
        if (!ok) break;
        tc_commit(&bar->fixed_empty[kb]);  // every MMA reading this K/V buffer has been issued
        tc_commit(&bar->o_full);
        gi += n_items;
        ++nkv;
        cur = nxt;
        b = nb, hk = nhk, s0 = ns0, qt0 = nqt0, per_head = nper, n_items = nn;
      }
      // the last item's s_free arrivals are never waited on: nothing reads S^T after them
    }
  } else if (warp < 12) {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 176;" ::: "memory");
    const int w = warp >= 8 ? 1 : 0;  // query-column half
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const uint32_t tl = tmem + lane_off;
    const float c = p.scale_log2;
    const uint64_t c2 = f2_pack(c, c);
    const uint32_t ds_row = smem_u32(sDS) + w * kT + row * 128;
    uint32_t gi = 0, nu = 0;
    bool ok = true;
    for (;; ++nu) {
      const int u = take_unit(&bar->uq, nu, abort, p.err, true);
      if (u < 0) break;
      int b, hk, s0, qt0, per_head;
      unit_info(u, b, hk, s0, qt0, per_head);
      const int n_items = per_head * group;
      const int s = s0 + row;
      const bool store = s < p.S;
      __nv_bfloat16* dst = w == 0
          ? static_cast<__nv_bfloat16*>(p.out1) + (int64_t)b * p.s1[0] + (int64_t)hk * p.s1[1] + (int64_t)s * p.s1[2]
          : static_cast<__nv_bfloat16*>(p.out0) + (int64_t)b * p.s0[0] + (int64_t)hk * p.s0[1] + (int64_t)s * p.s0[2];
      if (n_items == 0) {  // no query sees these keys: dK = dV = 0
        if (store)
          for (int i = 0; i < D; i += 8) *reinterpret_cast<uint4*>(dst + i) = make_uint4(0, 0, 0, 0);
        continue;
      }
      for (int it = 0; it < n_items; ++it) {
        const uint32_t g = gi + it;
        const int st = g % kStagesF;
        const int t0 = (qt0 + it % per_head) * 128;
        if (!(ok = mbar_wait(&bar->op_full[st], (g / kStagesF) & 1, abort, p.err))) break;
        if (!(ok = mbar_wait(&bar->s_full, g & 1, abort, p.err))) break;
        tc_fence_after();
        const int lo = p.causal ? s - p.q_start - t0 - w * 64 : -(1 << 30);  // columns below lo are masked
        uint32_t pp[32], dd[32];
        const bool need_mask = __any_sync(0xffffffffu, lo > 0);
        const uint32_t sl = smem_u32(sVec + st * 256 + w * 64), sd = smem_u32(sVec + st * 256 + 128 + w * 64);
        uint32_t srr[64], drr[64];
        tmem_ld32(tl + w * 64, *reinterpret_cast<uint32_t(*)[32]>(srr));
        tmem_ld32(tl + w * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(srr + 32));
        tmem_ld32(tl + 128 + w * 64, *reinterpret_cast<uint32_t(*)[32]>(drr));
        tmem_ld32(tl + 128 + w * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(drr + 32));
        tmem_wait_ld();
        warp_arrive_after_tc(&bar->s_free);
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const uint32_t* sr = srr + 32 * hf;
          const uint32_t* dr = drr + 32 * hf;
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 l4 = lds128(sl + 128 * hf + 16 * q);
            const float4 d4 = lds128(sd + 128 * hf + 16 * q);
#pragma unroll
            for (int h2 = 0; h2 < 2; ++h2) {
              const int cc = 4 * q + 2 * h2, col = 32 * hf + cc;
              const uint64_t s2 = (uint64_t)sr[cc] | ((uint64_t)sr[cc + 1] << 32);
              const uint64_t g2 = (uint64_t)dr[cc] | ((uint64_t)dr[cc + 1] << 32);
              const uint64_t l2 = h2 ? f2_pack(l4.z, l4.w) : f2_pack(l4.x, l4.y);
              const uint64_t dd2 = h2 ? f2_pack(d4.z, d4.w) : f2_pack(d4.x, d4.y);
              float x0, x1;
              f2_unpack(f2_fma(s2, c2, l2), x0, x1);
              float p0 = ex2(x0), p1 = ex2(x1);
              if (need_mask) {
                p0 = col >= lo ? p0 : 0.f;
                p1 = col + 1 >= lo ? p1 : 0.f;
              }
              float g0, g1;
              f2_unpack(f2_mul(f2_pack(p0, p1), f2_sub(g2, dd2)), g0, g1);
              pp[16 * hf + 2 * q + h2] = pack_bf16(p0, p1);
              dd[16 * hf + 2 * q + h2] = pack_bf16(g0, g1);
            }
          }
        }
        // the P^T staging columns and the dS^T buffer must be free of the previous item's MMAs
        if (g > 0 && !(ok = mbar_wait(&bar->stage_free, (g - 1) & 1, abort, p.err))) break;
        tc_fence_after();
        tmem_st32(tl + 256 + w * 32, pp);
#pragma unroll
        for (int ch = 0; ch < 8; ++ch)  // 128-byte swizzled row of 64 queries for key `row`
          sts128(ds_row + ((ch ^ (row & 7)) << 4), dd[4 * ch], dd[4 * ch + 1], dd[4 * ch + 2], dd[4 * ch + 3]);
        fence_proxy_async_smem();
        tmem_wait_st();
        warp_arrive_after_tc(&bar->p_full);
      }
      if (!ok) break;
      gi += n_items;
    }
  } else {
    // ------------------------------------------------------- drain warps
    // Each drain warp owns 32 TMEM lanes and a 4 KB staging box (32 rows x 128
    // bytes, 128-byte swizzled).  Per item it stages the two 32-column halves of
    // its 32 query rows of dQ_part in turn and adds each into the accumulator with
    // a bulk reduction; per unit it stores its 32 key rows of dV and dK (bf16)
    // with TMA stores.  It waits only for its own previous bulk operation to have
    // read the box before refilling it.
    asm volatile("setmaxnreg.dec.sync.aligned.u32 80;" ::: "memory");
    const int q4 = warp & 3;
    const uint32_t tl = tmem + ((uint32_t)(q4 * 32) << 16);
    const uint32_t box = smem_u32(sDQ) + q4 * 4096;
    const uint32_t stg = box + lane * 128;
    uint32_t gi = 0, nu = 0, nkv = 0;
    bool ok = true;
    for (;; ++nu) {
      const int u = take_unit(&bar->uq, nu, abort, p.err, true);
      if (u < 0) break;
      int b, hk, s0, qt0, per_head;
      unit_info(u, b, hk, s0, qt0, per_head);
      const int n_items = per_head * group;
      for (int it = 0; it < n_items; ++it) {
        const uint32_t g = gi + it;
        const int h = hk * group + it / per_head;
        const int t0 = (qt0 + it % per_head) * 128 + q4 * 32;
        if (!(ok = mbar_wait(&bar->dq_full, g & 1, abort, p.err))) break;
        tc_fence_after();
#pragma unroll 1
        for (int bx = 0; bx < 2; ++bx) {
          uint32_t r[32];
          tmem_ld32(tl + 320 + 32 * bx, r);
          tmem_wait_ld();
          if (bx == 1) warp_arrive_after_tc(&bar->dq_free);  // dQ_part is out of TMEM
          if (lane == 0) bulk_wait_read_all();  // the previous reduction has read the box
          __syncwarp();
#pragma unroll
          for (int ch = 0; ch < 8; ++ch)
            sts128(stg + ((ch ^ (lane & 7)) << 4), r[4 * ch], r[4 * ch + 1], r[4 * ch + 2], r[4 * ch + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_reduce_add_4d(&tm_dqacc, box, 32 * bx, t0, h, b);
            bulk_commit();
          }
        }
      }
      if (!ok) break;
      if (n_items > 0) {
        // the unit's dV, then dK (scaled): this warp's 32 key rows, out of TMEM as
        // bf16 into the staging box (one 128-byte row of 64 features per key) and
        // to global memory by a TMA store, which also drops rows past the sequence
        if (!(ok = mbar_wait(&bar->o_full, nkv & 1, abort, p.err))) break;
        tc_fence_after();
#pragma unroll 1
        for (int t = 0; t < 2; ++t) {
          const float mul = t == 0 ? 1.0f : p.scale;
#pragma unroll 1
          for (int hc = 0; hc < 2; ++hc) {
            uint32_t r[32];
            tmem_ld32(tl + 384 + 64 * t + 32 * hc, r);
            tmem_wait_ld();
            if (t == 1 && hc == 1) warp_arrive_after_tc(&bar->acc_free);  // dV / dK are out of TMEM
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i)
              pk[i] = pack_bf16(__uint_as_float(r[2 * i]) * mul, __uint_as_float(r[2 * i + 1]) * mul);
            if (hc == 0 && lane == 0) bulk_wait_read_all();  // the box's previous bulk operation has read it
            __syncwarp();
#pragma unroll
            for (int ch = 0; ch < 4; ++ch)
              sts128(stg + (((4 * hc + ch) ^ (lane & 7)) << 4), pk[4 * ch], pk[4 * ch + 1], pk[4 * ch + 2],
                     pk[4 * ch + 3]);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_4d(t == 0 ? &tm_dv : &tm_dk, box, 0, s0 + q4 * 32, hk, b);
            bulk_commit();
          }
        }
        ++nkv;
      }
      gi += n_items;
    }
    if (lane == 0) bulk_wait_all();  // the reductions and stores are complete before the CTA retires
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// dQ (bf16) = scale * the fp32 accumulator of the fused pass, rows t < T, features < E.
// Eight features per thread (two 16-byte loads, one 16-byte store).
__global__ void bwd_dq_convert_kernel(const float* __restrict__ acc, __nv_bfloat16* __restrict__ dq, int64_t s0,
                                      int64_t s1, int64_t s2, int H, int T, int Tpad, int E, float scale,
                                      int64_t n) {
  grid_dep_wait();  // the fused pass (and its bulk reductions) has completed
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int ch = (int)(i & 7);
  if (ch * 8 >= E) return;  // features past the head dim are zero padding
  const int64_t r = i >> 3;
  const int t = (int)(r % T);
  const int64_t bh = r / T;
  const int b = (int)(bh / H), h = (int)(bh % H);
  const float4* src = reinterpret_cast<const float4*>(acc + (bh * Tpad + t) * 64 + ch * 8);
  const float4 a = src[0], c = src[1];
  *reinterpret_cast<uint4*>(dq + b * s0 + h * s1 + t * s2 + ch * 8) =
      make_uint4(pack_bf16(a.x * scale, a.y * scale), pack_bf16(a.z * scale, a.w * scale),
                 pack_bf16(c.x * scale, c.y * scale), pack_bf16(c.z * scale, c.w * scale));
}

// ---------------------------------------------------------------- prologue
// D = sum(dO * O) and nlse2 = -lse * log2(e) per (b, h, padded row).  `tpr`
// threads share a row, each reading 16-byte chunks (8 bf16) of O and dO.  Also
// zeroes the work-unit counters of the persistent kernels that follow and, for
// the fused D = 64 pass, its fp32 dQ accumulator.
__global__ void bwd_prep_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dout,
                                const float* __restrict__ lse, float* __restrict__ lse2, float* __restrict__ dsum,
                                int64_t so0, int64_t so1, int64_t so2, int64_t sd0, int64_t sd1, int64_t sd2, int H,
                                int T, int Tpad, int DV, int64_t rows, int tpr, int vec, int* ctr,
                                float* __restrict__ dqacc) {
  if (blockIdx.x == 0 && threadIdx.x < 2) ctr[threadIdx.x] = 0;
  const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / tpr;
  const int sub = threadIdx.x % tpr;
  if (r >= rows) return;
  if (dqacc)  // the fused D = 64 pass adds its dQ parts into this (rows of 64 fp32)
    for (int i = sub * 4; i < 64; i += tpr * 4)
      *reinterpret_cast<float4*>(dqacc + r * 64 + i) = make_float4(0.f, 0.f, 0.f, 0.f);
  const int t = (int)(r % Tpad);
  const int64_t bh = r / Tpad;
  const int b = (int)(bh / H), h = (int)(bh % H);
  float acc = 0.f;
  if (t < T) {
    const __nv_bfloat16* orow = o + b * so0 + h * so1 + t * so2;
    const __nv_bfloat16* drow = dout + b * sd0 + h * sd1 + t * sd2;
    if (vec) {
      for (int i = sub * 8; i < DV; i += tpr * 8) {
        const uint4 a = *reinterpret_cast<const uint4*>(orow + i);
        const uint4 g = *reinterpret_cast<const uint4*>(drow + i);
        const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&a);
        const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&g);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float2 fa = __bfloat1622float2(a2[u]), fg = __bfloat1622float2(g2[u]);
          acc = fmaf(fa.x, fg.x, fmaf(fa.y, fg.y, acc));
        }
      }
    } else {
      for (int i = sub; i < DV; i += tpr) acc += __bfloat162float(orow[i]) * __bfloat162float(drow[i]);
    }
  }
  for (int off = tpr / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (sub == 0) {
    dsum[r] = t < T ? acc : 0.f;
    lse2[r] = t < T ? -lse[bh * T + t] * kLog2e : -INFINITY;
  }
}

// The prologue for 64-wide rows (the fused D = 64 pass): each warp takes 8 rows
// per step (8 lanes per row, one 16-byte chunk of O and of dO each, two rows
// per lane in flight) over a grid-stride loop sized to the resident warps, and
// zeroes the rows' fp32 dQ accumulator.
__global__ void __launch_bounds__(256) bwd_prep64_kernel(
    const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dout, const float* __restrict__ lse,
    float* __restrict__ lse2, float* __restrict__ dsum, int64_t so0, int64_t so1, int64_t so2, int64_t sd0,
    int64_t sd1, int64_t sd2, int H, int T, int Tpad, int64_t rows, int* ctr, float* __restrict__ dqacc) {
  if (blockIdx.x == 0 && threadIdx.x < 2) ctr[threadIdx.x] = 0;
  const int lane = threadIdx.x & 31, sub = lane & 7;
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t base = ((int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * 8; base < rows;
       base += nwarps * 8) {
    int64_t r[2];
    int t[2];
    uint4 a[2], g[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      r[u] = base + 4 * u + (lane >> 3);
      t[u] = (int)(r[u] % Tpad);
      a[u] = g[u] = make_uint4(0, 0, 0, 0);
      if (r[u] < rows && t[u] < T) {
        const int64_t bh = r[u] / Tpad;
        const int b = (int)(bh / H), h = (int)(bh % H);
        a[u] = *reinterpret_cast<const uint4*>(o + b * so0 + h * so1 + t[u] * so2 + sub * 8);
        g[u] = *reinterpret_cast<const uint4*>(dout + b * sd0 + h * sd1 + t[u] * sd2 + sub * 8);
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      if (r[u] < rows) {
        float4* z = reinterpret_cast<float4*>(dqacc + r[u] * 64 + sub * 8);
        z[0] = z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&a[u]);
      const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&g[u]);
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 fa = __bfloat1622float2(a2[i]), fg = __bfloat1622float2(g2[i]);
        acc = fmaf(fa.x, fg.x, fmaf(fa.y, fg.y, acc));
      }
      acc += __shfl_xor_sync(0xffffffffu, acc, 4);
      acc += __shfl_xor_sync(0xffffffffu, acc, 2);
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      if (sub == 0 && r[u] < rows) {
        const bool live = t[u] < T;
        dsum[r[u]] = live ? acc : 0.f;
        lse2[r[u]] = live ? -lse[(r[u] / Tpad) * T + t[u]] * kLog2e : -INFINITY;
      }
    }
  }
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct WsLayout {
  size_t lse2, dsum, ctr, dqacc, lse, o_scratch, total;
};

WsLayout ws_layout(const pdb_flash_bwd_desc& d) {
  WsLayout w{};
  // Every size below is a product of descriptor fields; a descriptor whose
  // products would wrap gets total = SIZE_MAX, which no workspace (and no fixed
  // scratch) satisfies.
  size_t rows = 0, tmp = 0;
  const int64_t tpad = (d.seqlen_q + BT - 1) / BT * BT;
  if (d.batch <= 0 || d.heads_q <= 0 || tpad <= 0 || d.head_dim_v <= 0 ||
      __builtin_mul_overflow((size_t)d.batch, (size_t)d.heads_q, &tmp) ||
      __builtin_mul_overflow(tmp, (size_t)tpad, &rows) || __builtin_mul_overflow(rows, (size_t)(64 * 4 * 4), &tmp) ||
      __builtin_mul_overflow(rows, (size_t)d.head_dim_v * 2 + 64, &tmp)) {
    w.total = SIZE_MAX;
    return w;
  }
  size_t off = 0;
  w.lse2 = off;
  off = align256(off + rows * 4);
  w.dsum = off;
  off = align256(off + rows * 4);
  w.ctr = off;  // two work-unit counters
  off = align256(off + 8);
  if (d.head_dim <= 64 && d.head_dim_v <= 64) {  // fp32 dQ accumulator of the fused pass, rows padded like lse2
    w.dqacc = off;
    off = align256(off + rows * 64 * 4);
  }
  if (d.lse == nullptr) {  // recompute variant: the forward's lse and a scratch output
    w.lse = off;
    off = align256(off + (size_t)(d.batch * d.heads_q * d.seqlen_q) * 4);
    w.o_scratch = off;
    off = align256(off + (size_t)(d.batch * d.heads_q * d.seqlen_q * d.head_dim_v) * 2);
  }
  w.total = off;
  return w;
}

int map_bf16(CUtensorMap* m, const void* base, int D, int64_t rows, int64_t heads, int64_t batch,
             const int64_t st[3], uint32_t box_rows) {
  const uint64_t dims[4] = {(uint64_t)D, (uint64_t)rows, (uint64_t)heads, (uint64_t)batch};
  const uint64_t str[3] = {(uint64_t)st[2] * 2, (uint64_t)st[1] * 2, (uint64_t)st[0] * 2};
  const uint32_t box[4] = {64, box_rows, 1, 1};
  return encode_tma_4d(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, base, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

// Launch behind the previous kernel of the stream with programmatic stream
// serialization: the grid may start (set-up: barriers, TMEM, tensor maps) while
// the previous one drains; the kernel orders its reads with grid_dep_wait.
template <class... KArgs, class... Args>
cudaError_t launch_overlapped(void (*kernel)(KArgs...), int64_t grid, int threads, int smem, cudaStream_t stream,
                              Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <int D>
int launch_bwd(const pdb_flash_bwd_desc& d, const float* lse, const WsLayout& w, cudaStream_t stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  uint8_t* ws = static_cast<uint8_t*>(d.workspace);
  const int64_t tpad = (d.seqlen_q + BT - 1) / BT * BT;
  float* lse2 = reinterpret_cast<float*>(ws + w.lse2);
  float* dsum = reinterpret_cast<float*>(ws + w.dsum);
  int* ctr = reinterpret_cast<int*>(ws + w.ctr);
  {
    const int64_t rows = d.batch * d.heads_q * tpad;
    const bool vec = (d.head_dim_v % 8 == 0) && ((d.o_stride[0] | d.o_stride[1] | d.o_stride[2]) % 8 == 0) &&
                     ((d.do_stride[0] | d.do_stride[1] | d.do_stride[2]) % 8 == 0) &&
                     (reinterpret_cast<uintptr_t>(d.o) & 15) == 0 && (reinterpret_cast<uintptr_t>(d.dout) & 15) == 0;
    int tpr = 32;  // threads per row: a power of two dividing the warp
    if (vec) {
      tpr = 1;
      while (tpr < 32 && tpr * 8 < d.head_dim_v) tpr *= 2;
    }
    const int64_t threads = rows * tpr;
    if (D == 64 && vec && d.head_dim_v == 64) {
      int64_t blocks = (rows + 63) / 64;
      const int64_t resident = 8LL * sm_count(dev);
      if (blocks > resident) blocks = resident;
      bwd_prep64_kernel<<<(unsigned)blocks, 256, 0, stream>>>(
          static_cast<const __nv_bfloat16*>(d.o), static_cast<const __nv_bfloat16*>(d.dout), lse, lse2, dsum,
          d.o_stride[0], d.o_stride[1], d.o_stride[2], d.do_stride[0], d.do_stride[1], d.do_stride[2],
          (int)d.heads_q, (int)d.seqlen_q, (int)tpad, rows, ctr, reinterpret_cast<float*>(ws + w.dqacc));
    } else
    bwd_prep_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(d.o), static_cast<const __nv_bfloat16*>(d.dout), lse, lse2, dsum,
        d.o_stride[0], d.o_stride[1], d.o_stride[2], d.do_stride[0], d.do_stride[1], d.do_stride[2],
        (int)d.heads_q, (int)d.seqlen_q, (int)tpad, (int)d.head_dim_v, rows, tpr, vec ? 1 : 0, ctr,
        D == 64 ? reinterpret_cast<float*>(ws + w.dqacc) : nullptr);
    if (int st = cuda_status(cudaGetLastError(), "bwd prep launch")) return st;
  }
  // 128-row boxes for every operand: 128-key / 128-row units and 128-wide items in both D = 128 passes
  CUtensorMap tk128, tv128, tq128, tdo128;
  // the maps carry the true head dims (e for q / k, e_v for v / dO): features between
  // them and D are zero-filled, so they add nothing to the scores or the gradients
  const int E = (int)d.head_dim, EV = (int)d.head_dim_v;
  if (int st = map_bf16(&tk128, d.k, E, d.seqlen_k, d.heads_kv, d.batch, d.k_stride, 128)) return st;
  if (int st = map_bf16(&tv128, d.v, EV, d.seqlen_k, d.heads_kv, d.batch, d.v_stride, 128)) return st;
  if (int st = map_bf16(&tq128, d.q, E, d.seqlen_q, d.heads_q, d.batch, d.q_stride, 128)) return st;
  if (int st = map_bf16(&tdo128, d.dout, EV, d.seqlen_q, d.heads_q, d.batch, d.do_stride, 128)) return st;
  BwdParams p{};
  p.nlse2 = lse2;
  p.dsum = dsum;
  p.T = (int)d.seqlen_q;
  p.S = (int)d.seqlen_k;
  p.H = (int)d.heads_q;
  p.HKV = (int)d.heads_kv;
  p.Tpad = (int)tpad;
  p.q_start = (int)d.q_start;
  p.causal = d.causal ? 1 : 0;
  p.scale = (float)d.scale;
  p.scale_log2 = (float)(d.scale * 1.4426950408889634);
  p.B = (int)d.batch;
  p.err = device_error_flag();
  if constexpr (D == 64) {  // one fused pass for dK, dV and dQ, then dQ scaled and rounded
    float* dqacc = reinterpret_cast<float*>(ws + w.dqacc);
    CUtensorMap tdq;
    {
      const uint64_t dims[4] = {64, (uint64_t)tpad, (uint64_t)d.heads_q, (uint64_t)d.batch};
      const uint64_t str[3] = {64 * 4, (uint64_t)tpad * 64 * 4, (uint64_t)(tpad * d.heads_q) * 64 * 4};
      const uint32_t box[4] = {32, 32, 1, 1};
      if (int st = encode_tma_4d(&tdq, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, dqacc, dims, str, box,
                                 CU_TENSOR_MAP_SWIZZLE_128B))
        return st;
    }
    p.out0 = d.dk;
    p.out1 = d.dv;
    for (int i = 0; i < 3; ++i) {
      p.s0[i] = d.dk_stride[i];
      p.s1[i] = d.dv_stride[i];
    }
    p.n_blocks = (int)((d.seqlen_k + 127) / 128);
    p.ctr = ctr;
    const int64_t grid = (int64_t)p.n_blocks * d.heads_kv * d.batch;
    const int smem = (7 + 2 * kStagesF) * 16384 + kStagesF * 1024 + (int)sizeof(BarsF) + 1024;
    cudaError_t e = cudaFuncSetAttribute(bwd_fused64_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return cuda_status(e, "bwd fused64 smem attribute");
    const int64_t pgrid = grid < sm_count(dev) ? grid : sm_count(dev);
    CUtensorMap tdk32, tdv32;  // dK / dV stores: 32-row boxes, one per drain warp
    // the store maps carry the true dims: the TMA drops the zero columns past them
    if (int st = map_bf16(&tdk32, d.dk, E, d.seqlen_k, d.heads_kv, d.batch, d.dk_stride, 32)) return st;
    if (int st = map_bf16(&tdv32, d.dv, EV, d.seqlen_k, d.heads_kv, d.batch, d.dv_stride, 32)) return st;
    e = launch_overlapped(bwd_fused64_kernel, pgrid, kFusedThreads, smem, stream, tq128, tk128, tv128, tdo128, tdq,
                          tdk32, tdv32, p);
    if (e != cudaSuccess) return cuda_status(e, "bwd fused64 launch");
    const int64_t n = d.batch * d.heads_q * d.seqlen_q * 8;
    e = launch_overlapped(bwd_dq_convert_kernel, (n + 255) / 256, 256, 0, stream, (const float*)dqacc,
                          static_cast<__nv_bfloat16*>(d.dq), d.dq_stride[0], d.dq_stride[1], d.dq_stride[2],
                          (int)d.heads_q, (int)d.seqlen_q, (int)tpad, E, (float)d.scale, n);
    if (e != cudaSuccess) return cuda_status(e, "bwd dq convert launch");
    return PDB_OK;
  } else {
    {  // dK, dV
      p.out0 = d.dk;
      p.out1 = d.dv;
      p.ncols0 = E;
      p.ncols1 = EV;
      for (int i = 0; i < 3; ++i) {
        p.s0[i] = d.dk_stride[i];
        p.s1[i] = d.dv_stride[i];
      }
      p.n_blocks = (int)((d.seqlen_k + 127) / 128);
      const int64_t grid = (int64_t)p.n_blocks * d.heads_kv * d.batch;
      {
        p.ctr = ctr;
        const int64_t pgrid = grid < sm_count(dev) ? grid : sm_count(dev);
        cudaError_t e = cudaFuncSetAttribute(bwd_dkdv128_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kMaxDynSmem);
        if (e != cudaSuccess) return cuda_status(e, "bwd dkdv smem attribute");
        e = launch_overlapped(bwd_dkdv128_kernel, pgrid, kThreads, kMaxDynSmem, stream, tq128, tk128, tv128, tdo128, p);
        if (e != cudaSuccess) return cuda_status(e, "bwd dkdv launch");
      }
      if (int st = cuda_status(cudaGetLastError(), "bwd dkdv launch")) return st;
    }
    {  // dQ
      p.out0 = d.dq;
      p.out1 = nullptr;
      p.ncols0 = E;
      p.ncols1 = 0;
      for (int i = 0; i < 3; ++i) p.s0[i] = d.dq_stride[i];
      p.n_blocks = (int)(tpad / 128);
      const int64_t grid = (int64_t)p.n_blocks * d.heads_q * d.batch;
      {
        p.ctr = ctr;
        const int64_t pgrid = grid < sm_count(dev) ? grid : sm_count(dev);
        const int smem = kDq128Smem + (int)sizeof(BarsQ) + 1024;
        cudaError_t e = cudaFuncSetAttribute(bwd_dq128_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return cuda_status(e, "bwd dq smem attribute");
        e = launch_overlapped(bwd_dq128_kernel, pgrid, kThreads, smem, stream, tq128, tk128, tv128, tdo128, p);
        if (e != cudaSuccess) return cuda_status(e, "bwd dq launch");
      }
      if (int st = cuda_status(cudaGetLastError(), "bwd dq launch")) return st;
    }
    return PDB_OK;
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace pdb

using namespace pdb;


extern "C" size_t pdb_flash_bwd_workspace_size(const pdb_flash_bwd_desc* d) {
  if (!d || d->batch <= 0 || d->heads_q <= 0 || d->seqlen_q <= 0) return 0;
  return ws_layout(*d).total;
}

extern "C" int pdb_flash_bwd(const pdb_flash_bwd_desc* d, void* stream) {
  if (!d) return set_error(PDB_ERR_ARG, "null descriptor");
  if (int st = validate_common(d->batch, d->heads_q, d->heads_kv, d->seqlen_q, d->seqlen_k, d->head_dim,
                               d->head_dim_v, d->q_start, d->q, d->k, d->v))
    return st;
  if (!d->o || !d->dout || !d->dq || !d->dk || !d->dv) return set_error(PDB_ERR_ARG, "null o / dout / dq / dk / dv");
  if (d->dtype != PDB_BF16)
    return set_error(PDB_ERR_UNSUPPORTED, "flash backward: bf16 only (dtype %d)", d->dtype);
  // both head dims <= 64: the fused pass; otherwise (multiples of 8 up to 128) the
  // D = 128 passes; the tensor maps zero-fill the features between each dim and D
  const bool fused = d->head_dim <= 64 && d->head_dim_v <= 64;
  if (d->head_dim % 8 || d->head_dim_v % 8 || d->head_dim > 128 || d->head_dim_v > 128)
    return set_error(PDB_ERR_UNSUPPORTED, "flash backward: head dims must be multiples of 8 up to 128 (got %lld, %lld)",
                     (long long)d->head_dim, (long long)d->head_dim_v);
  if (d->seqlen_q > (1 << 30) || d->seqlen_k > (1 << 30)) return set_error(PDB_ERR_SHAPE, "sequence too long");
  const WsLayout w = ws_layout(*d);
  if (!d->workspace || d->workspace_bytes < w.total)
    return set_error(PDB_ERR_ARG, "workspace too small: need %zu bytes", w.total);
  if (!aligned16(d->workspace)) return set_error(PDB_ERR_ALIGN, "workspace must be 16-byte aligned");
  for (const void* ptr : {d->dq, d->dk, d->dv})
    if (!aligned16(ptr)) return set_error(PDB_ERR_ALIGN, "dq / dk / dv must be 16-byte aligned");
  for (const int64_t* s : {d->dq_stride, d->dk_stride, d->dv_stride})
    if ((s[0] | s[1] | s[2]) & 7) return set_error(PDB_ERR_ALIGN, "dq / dk / dv strides must be multiples of 8");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const float* lse = d->lse;
  if (lse == nullptr) {  // recompute the forward's logsumexp
    uint8_t* ws = static_cast<uint8_t*>(d->workspace);
    pdb_flash_desc f{};
    f.q = d->q;
    f.k = d->k;
    f.v = d->v;
    f.o = ws + w.o_scratch;
    f.lse = reinterpret_cast<float*>(ws + w.lse);
    f.batch = d->batch;
    f.heads_q = d->heads_q;
    f.heads_kv = d->heads_kv;
    f.seqlen_q = d->seqlen_q;
    f.seqlen_k = d->seqlen_k;
    f.head_dim = d->head_dim;
    f.head_dim_v = d->head_dim_v;
    for (int i = 0; i < 3; ++i) {
      f.q_stride[i] = d->q_stride[i];
      f.k_stride[i] = d->k_stride[i];
      f.v_stride[i] = d->v_stride[i];
    }
    f.o_stride[2] = d->head_dim_v;
    f.o_stride[1] = d->seqlen_q * d->head_dim_v;
    f.o_stride[0] = d->heads_q * f.o_stride[1];
    f.q_start = d->q_start;
    f.scale = d->scale;
    f.causal = d->causal;
    f.dtype = PDB_BF16;
    if (int st = flash_fwd_bf16_sm100(f, s)) return st;
    lse = f.lse;
  }
  return fused ? launch_bwd<64>(*d, lse, w, s) : launch_bwd<128>(*d, lse, w, s);
}

// ---------------------------------------------------------------------------
// pdb_flash_bwd_noalloc: the same backward with its scratch in a fixed,
// library-owned device array instead of a caller-supplied workspace.
//
// Who needs it: callers that may not allocate device memory at call time --
// code running inside a memory pool or arena that owns every byte of the
// device, hosts whose allocator is locked while a step is in flight, or C
// callers with no allocator binding at all.  They pass inputs and outputs
// only.  The scratch (D and lse2 rows, plus the recomputed lse and a scratch
// forward output when lse is NULL) lives in g_bwd_scratch below; its address
// is looked up once per device, on the first call made with that device
// current (so make that first call before any stream capture), and kept for
// the life of the process: a device reset (cudaDeviceReset, or anything that
// destroys the primary context) reloads the library's device code and
// invalidates it, so a process that resets a device must not call this entry
// point on that device afterwards.  The prologue
// kernel rewrites every scratch word it later reads on each call, so nothing
// has to be cleared between calls.  Every call on a device shares the one
// array: calls that can overlap on the GPU (different streams without
// ordering) race on it and must be serialised by the caller.
namespace pdb {
namespace {
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;  // 16 MiB per device
static __device__ __align__(256) uint8_t g_bwd_scratch[kNoAllocScratchBytes];
constexpr int kMaxDev = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDev];
}  // namespace
}  // namespace pdb

extern "C" size_t pdb_flash_bwd_noalloc_max_scratch(void) { return pdb::kNoAllocScratchBytes; }

extern "C" int pdb_flash_bwd_noalloc(const pdb_flash_bwd_desc* d, void* stream) {
  using namespace pdb;
  if (!d) return set_error(PDB_ERR_ARG, "null descriptor");
  if (d->batch <= 0 || d->heads_q <= 0 || d->seqlen_q <= 0)
    return set_error(PDB_ERR_SHAPE, "all sizes must be positive");
  const WsLayout w = ws_layout(*d);
  if (w.total > kNoAllocScratchBytes)
    return set_error(PDB_ERR_SHAPE,
                     "pdb_flash_bwd_noalloc: problem needs %zu scratch bytes, the fixed scratch holds %zu "
                     "(use pdb_flash_bwd with a caller workspace)",
                     w.total, kNoAllocScratchBytes);
  int dev = 0;
  if (cudaError_t e = cudaGetDevice(&dev)) return cuda_status(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDev) return set_error(PDB_ERR_CUDA, "device index out of range");
  void* ptr = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (g_scratch_ptr[dev] == nullptr) {
      void* p = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&p, g_bwd_scratch);
      if (e != cudaSuccess || p == nullptr) return cuda_status(e, "cudaGetSymbolAddress(g_bwd_scratch)");
      g_scratch_ptr[dev] = p;
    }
    ptr = g_scratch_ptr[dev];
  }
  pdb_flash_bwd_desc local = *d;
  local.workspace = ptr;
  local.workspace_bytes = kNoAllocScratchBytes;
  return pdb_flash_bwd(&local, stream);
}
