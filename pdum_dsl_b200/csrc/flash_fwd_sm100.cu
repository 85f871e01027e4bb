// bf16 flash-attention forward for sm_100a: TMA-staged tiles, tcgen05 MMAs
// with TMEM accumulators, warp-specialised online softmax.
//
// What it computes is the reference's flash template (fusion.py:480-615):
// the online-softmax fold over key tiles of the masked, scaled score
// contraction, with the flashsm recurrence of zoo/attention.py:40-46, and
// the causal tile bounds that _prune_flash derives (fusion.py:659-690,
// hi = 1 + pid for BT = SI): key tiles past the diagonal are never visited.
//
// Work tile = 256 query rows of one (batch, head), as two 128-row tiles A and
// B; a persistent grid of one CTA per SM walks the tiles.
//   warp 0        TMA producer (Q once; K/V tiles through 2-stage rings)
//   warp 1        MMA issuer (one thread): S = Q K^T into TMEM, O += P V
//                 with P read from TMEM (the "TS" form)
//   warp 2        TMEM allocator
//   warps 4..7    softmax for tile A, one thread per query row (TMEM lane)
//   warps 8..11   softmax for tile B
// TMEM (512 columns x 128 lanes x 32 bit): S_A [0,128) S_B [128,256)
// O_A [256, 256+D) O_B [256+D, 256+2D).  P (bf16, packed in pairs)
// overwrites the first 64 columns of its S tile.
// Ping-pong: while softmax A works on S_A(j+1) the tensor core runs
// PV_B(j) and S_B(j+1), and vice versa.
//
// Softmax is in the log2 domain (c = scale * log2 e) with lazy rescaling:
// the running max used for the exponent only moves when a tile's max exceeds
// it by more than 8 (a factor 256), so most tiles need no O correction; the
// true max is tracked on the side for the m / den / lse outputs.
#include <cfloat>

#include "common.cuh"
#include "tma.h"

namespace pdb {
namespace {

constexpr int BM = 128;          // rows per tile (TMEM lanes)
constexpr int BN = 128;          // keys per tile
constexpr int kThreads = 384;    // 3 warpgroups
constexpr int kBoxBytes = 64 * 128 * 2;  // one TMA box: 128 rows x 64 bf16 (128 B, swizzled)
constexpr float kRescaleThreshold = 8.0f;

struct __align__(8) Barriers {
  uint64_t q_full, q_empty;
  uint64_t k_full[2], k_empty[2];
  uint64_t v_full[2], v_empty[2];
  uint64_t s_full[2];  // MMA -> softmax (tile A, B)
  uint64_t p_full[2];  // softmax -> MMA
  uint64_t o_full[2];  // last PV done -> epilogue
  uint64_t o_empty[2];  // epilogue read O -> next tile may accumulate
  uint64_t stg_free[4];  // an O staging region has been read by its TMA stores (A, B take turns)
  uint32_t tmem_base;
  int abort;
};

struct FwdParams {
  void* o;
  float* lse;
  float* m;
  float* den;
  int64_t o_stride[3];
  int T, S, H, HKV, B;
  int q_start;
  int causal;
  const int32_t* key_lo;  // per-row key intervals (general closed masks) or null
  const int32_t* key_hi;
  int mask_monotone;
  int lpt;          // heaviest-first snake schedule (else head-major pairs)
  int DV;           // the value / output head dim (<= the kernel's D; the TMA maps zero-fill the rest)
  int num_mblocks;  // 256-row blocks per head
  float scale_log2;  // scale * log2(e)
  int* err;
};

template <int D>
struct Smem {
  static constexpr int kTileBytes = BM * D * 2;  // Q / K / V tile
  static constexpr int kQ0 = 0;
  static constexpr int kQ1 = kTileBytes;
  static constexpr int kK = 2 * kTileBytes;  // 2 stages
  static constexpr int kV = 4 * kTileBytes;  // 2 stages
  // O staging for the TMA-store epilogue: per TMEM lane quarter, D / 64 boxes of
  // 32 rows x 64 bf16 (4 KB, 128-byte swizzled), shared by tiles A and B in turn
  static constexpr int kStg = 6 * kTileBytes;
  static constexpr int kBar = 7 * kTileBytes;
  static constexpr int kTotal = kBar + 1024 /*barriers*/ + 1024 /*alignment slack*/;
};

template <int D>
__device__ __forceinline__ void mma_qk(uint32_t d_tmem, uint32_t q_saddr, uint32_t k_saddr) {
  constexpr uint32_t idesc = idesc_bf16(BM, BN, 0, 0);
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const uint32_t off = (kk >> 2) * kBoxBytes + (kk & 3) * 32;
    mma_ss(d_tmem, sdesc_sw128(q_saddr + off, 16, 1024), sdesc_sw128(k_saddr + off, 16, 1024), idesc, kk > 0);
  }
}

template <int D>
__device__ __forceinline__ void mma_pv(uint32_t o_tmem, uint32_t p_tmem, uint32_t v_saddr, bool acc) {
  constexpr uint32_t idesc = idesc_bf16(BM, D, 0, 1);
#pragma unroll
  for (int kk = 0; kk < BN / 16; ++kk) {
    mma_ts(o_tmem, p_tmem + kk * 8, sdesc_sw128(v_saddr + kk * 2048, kBoxBytes, 1024), idesc, (acc || kk > 0) ? 1u : 0u);
  }
}

// Key tiles j0 .. j0 + nA - 1 (tile A) and j0 .. j0 + nB - 1 (tile B, nB >= nA).
struct TileInfo {
  int b, h, hk, t0, j0, nA, nB;
};

// Registers written by tcgen05.ld are valid only after tcgen05.wait::ld; this
// empty asm makes every later use of r[0..N) depend on a point after the wait.
template <int N>
__device__ __forceinline__ void regs_after_wait(uint32_t* r) {
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i]));
}

// The exponential phase of one 32-score chunk: P = exp2(s c - m) as 16 bf16
// pairs (packed f32x2 FMA for the argument, MUFU ex2 per score, cvt.rn.bf16x2
// to pack) and the pairs' f32 row sums on two chains.
__device__ __forceinline__ void exp_chunk(const uint32_t* sr, uint64_t c2, uint64_t nm2, uint64_t& sum_a,
                                          uint64_t& sum_b, uint32_t (&pk)[16]) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const uint64_t sv = (uint64_t)sr[2 * i] | ((uint64_t)sr[2 * i + 1] << 32);
    float x0, x1;
    f2_unpack(f2_fma(sv, c2, nm2), x0, x1);
    const float p0 = ex2(x0), p1 = ex2(x1);
    const uint64_t pv = f2_pack(p0, p1);
    if (i & 1) sum_b = f2_add(sum_b, pv); else sum_a = f2_add(sum_a, pv);
    pk[i] = pack_bf16(p0, p1);
  }
}

// Two static schedules of the persistent grid over the work tiles (256 query
// rows of one head each).
// * Pairs (large jobs): ordinals run head-major (concurrent CTAs share the K/V
//   of a few heads in L2); within a head they alternate heavy and light row
//   blocks (last, first, second-to-last, second, ...).  A CTA takes ordinals in
//   pairs, so each pair costs about the same under the causal mask.
// * Heaviest-first snake (small jobs, e.g. one rank's shard of a job split over
//   several GPUs, where a few hundred equal pairs over 148 SMs leave the last
//   wave half empty): ordinals run from the last row block of every head down
//   to the first, and CTA c takes ordinals c, 2G-1-c, 2G+c, ... (G CTAs), the
//   longest-processing-time-first rule dealt in a boustrophedon.  The K/V of
//   all heads of such a job fit in L2, so the head-major order buys nothing.
__device__ __forceinline__ int kth_tile(int k, int num_tiles, int lpt) {
  int t;
  if (lpt) {
    const int G = gridDim.x;
    t = k * G + ((k & 1) ? G - 1 - (int)blockIdx.x : (int)blockIdx.x);
  } else {
    t = (blockIdx.x + (k >> 1) * gridDim.x) * 2 + (k & 1);
  }
  return t < num_tiles ? t : -1;
}

__device__ __forceinline__ TileInfo tile_info(int tile, const FwdParams& p) {
  TileInfo ti;
  int bh, mblk;
  if (p.lpt) {
    const int nbh = p.H * p.B;
    bh = tile % nbh;
    mblk = p.num_mblocks - 1 - tile / nbh;
  } else {
    bh = tile / p.num_mblocks;
    const int r = tile % p.num_mblocks;
    mblk = (r & 1) ? (r >> 1) : p.num_mblocks - 1 - (r >> 1);
  }
  ti.b = bh / p.H;
  ti.h = bh % p.H;
  ti.hk = ti.h / (p.H / p.HKV);
  ti.t0 = mblk * 2 * BM;
  const int n_kv = (p.S + BN - 1) / BN;
  int n[2];
  ti.j0 = 0;
  if (p.key_lo && p.mask_monotone) {
    // visible keys of the 256 rows: [key_lo[first row], key_hi[last row])
    const int first = ti.t0 < p.T ? ti.t0 : p.T - 1;
    ti.j0 = __ldg(p.key_lo + first) / BN;
  }
#pragma unroll
  for (int x = 0; x < 2; ++x) {
    int last_row = ti.t0 + x * BM + BM - 1;
    if (last_row > p.T - 1) last_row = p.T - 1;
    int c = n_kv;
    if (p.causal) c = (last_row + p.q_start) / BN + 1;
    else if (p.key_lo && p.mask_monotone) c = (__ldg(p.key_hi + last_row) + BN - 1) / BN;
    c = c < n_kv ? c : n_kv;
    n[x] = c - ti.j0 > 1 ? c - ti.j0 : 1;
  }
  ti.nA = n[0];
  ti.nB = n[1] < n[0] ? n[0] : n[1];
  return ti;
}

// Persistent: gridDim.x <= #SMs CTAs walk the tile list (pairs of ordinals with
// stride gridDim.x pairs).
// Barrier phases run on counters that continue across tiles, so the loads and
// score MMAs of tile n+1 overlap the epilogue of tile n; O_x is only
// overwritten after the epilogue of its previous tile released it (o_empty).
template <int D, bool kKeyMask>
__global__ void __launch_bounds__(kThreads, 1)
    flash_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                           const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                           const FwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  using L = Smem<D>;
  Barriers* bar = reinterpret_cast<Barriers*>(smem + L::kBar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_tiles = p.num_mblocks * p.H * p.B;

  if (threadIdx.x == 0) {
    mbar_init(&bar->q_full, 1);
    mbar_init(&bar->q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar->k_full[i], 1);
      mbar_init(&bar->k_empty[i], 1);
      mbar_init(&bar->v_full[i], 1);
      mbar_init(&bar->v_empty[i], 1);
      mbar_init(&bar->s_full[i], 1);
      mbar_init(&bar->p_full[i], BM / 32);  // one arrival per softmax warp
      mbar_init(&bar->o_full[i], 1);
      mbar_init(&bar->o_empty[i], BM / 32);
    }
    bar->abort = 0;
    for (int i = 0; i < 4; ++i) mbar_init(&bar->stg_free[i], 1);
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

  const uint32_t sQ0 = smem_u32(smem + L::kQ0), sQ1 = smem_u32(smem + L::kQ1);
  const uint32_t sK = smem_u32(smem + L::kK), sV = smem_u32(smem + L::kV);
  constexpr int kNB = D / 64;  // boxes per tile

  // Register split (per warpgroup): the control warpgroup hands registers to
  // the two softmax warpgroups.  Launch budget 384 x 168 = 64512
  // = 128 x 88 + 256 x 208.
  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 88;" ::: "memory");
    if (warp == 0 && lane == 0) {
      // ---------------------------------------------------------- producer
      prefetch_tensormap(&tm_q);
      prefetch_tensormap(&tm_k);
      prefetch_tensormap(&tm_v);
      uint32_t g = 0, tt = 0;  // K/V tiles loaded, tiles started
      for (int k = 0, tile = kth_tile(0, num_tiles, p.lpt); tile >= 0; tile = kth_tile(++k, num_tiles, p.lpt), ++tt) {
        const TileInfo ti = tile_info(tile, p);
        if (!mbar_wait(&bar->q_empty, (tt & 1) ^ 1, abort, p.err)) break;
        mbar_expect_tx(&bar->q_full, 2 * L::kTileBytes);
        for (int i = 0; i < kNB; ++i) {
          tma_load_4d(smem + L::kQ0 + i * kBoxBytes, &tm_q, &bar->q_full, i * 64, ti.t0, ti.h, ti.b);
          tma_load_4d(smem + L::kQ1 + i * kBoxBytes, &tm_q, &bar->q_full, i * 64, ti.t0 + BM, ti.h, ti.b);
        }
        bool ok = true;
        for (int j = 0; j < ti.nB; ++j, ++g) {
          const int st = g & 1;
          const uint32_t ph = (g >> 1) & 1;
          if (!(ok = mbar_wait(&bar->k_empty[st], ph ^ 1, abort, p.err))) break;
          mbar_expect_tx(&bar->k_full[st], L::kTileBytes);
          for (int i = 0; i < kNB; ++i)
            tma_load_4d(smem + L::kK + st * L::kTileBytes + i * kBoxBytes, &tm_k, &bar->k_full[st], i * 64,
                        (ti.j0 + j) * BN, ti.hk, ti.b);
          if (!(ok = mbar_wait(&bar->v_empty[st], ph ^ 1, abort, p.err))) break;
          mbar_expect_tx(&bar->v_full[st], L::kTileBytes);
          for (int i = 0; i < kNB; ++i)
            tma_load_4d(smem + L::kV + st * L::kTileBytes + i * kBoxBytes, &tm_v, &bar->v_full[st], i * 64,
                        (ti.j0 + j) * BN, ti.hk, ti.b);
        }
        if (!ok) break;
      }
    } else if (warp == 1 && lane == 0) {
      // -------------------------------------------------------- MMA issuer
      const uint32_t tS[2] = {tmem + 0, tmem + 128};
      const uint32_t tO[2] = {tmem + 256, tmem + 256 + D};
      uint32_t g = 0, tt = 0, cs[2] = {0, 0};  // K/V tiles consumed, tiles, P tiles consumed per x
      bool ok = true;
      for (int k = 0, tile = kth_tile(0, num_tiles, p.lpt); ok && tile >= 0; tile = kth_tile(++k, num_tiles, p.lpt), ++tt) {
        const TileInfo ti = tile_info(tile, p);
        if (!(ok = mbar_wait(&bar->q_full, tt & 1, abort, p.err))) break;
        if (!(ok = mbar_wait(&bar->k_full[g & 1], (g >> 1) & 1, abort, p.err))) break;
        tc_fence_after();
        mma_qk<D>(tS[0], sQ0, sK + (g & 1) * L::kTileBytes);
        tc_commit(&bar->s_full[0]);
        mma_qk<D>(tS[1], sQ1, sK + (g & 1) * L::kTileBytes);
        tc_commit(&bar->s_full[1]);
        tc_commit(&bar->k_empty[g & 1]);
        for (int j = 0; ok && j < ti.nB; ++j) {
          const uint32_t gj = g + j, gn = gj + 1;
          const int st = gj & 1, stn = gn & 1;
          const uint32_t ph = (gj >> 1) & 1, phn = (gn >> 1) & 1;
          if (!(ok = mbar_wait(&bar->v_full[st], ph, abort, p.err))) break;
          if (j < ti.nA) {
            if (!(ok = mbar_wait(&bar->p_full[0], cs[0] & 1, abort, p.err))) break;
            ++cs[0];
            if (j == 0 && !(ok = mbar_wait(&bar->o_empty[0], (tt & 1) ^ 1, abort, p.err))) break;
            tc_fence_after();
            mma_pv<D>(tO[0], tS[0], sV + st * L::kTileBytes, j > 0);
            if (j + 1 < ti.nA) {
              if (!(ok = mbar_wait(&bar->k_full[stn], phn, abort, p.err))) break;
              tc_fence_after();
              mma_qk<D>(tS[0], sQ0, sK + stn * L::kTileBytes);
              tc_commit(&bar->s_full[0]);
            } else {
              tc_commit(&bar->o_full[0]);
            }
          }
          if (!(ok = mbar_wait(&bar->p_full[1], cs[1] & 1, abort, p.err))) break;
          ++cs[1];
          if (j == 0 && !(ok = mbar_wait(&bar->o_empty[1], (tt & 1) ^ 1, abort, p.err))) break;
          tc_fence_after();
          mma_pv<D>(tO[1], tS[1], sV + st * L::kTileBytes, j > 0);
          tc_commit(&bar->v_empty[st]);
          if (j + 1 < ti.nB) {
            if (!(ok = mbar_wait(&bar->k_full[stn], phn, abort, p.err))) break;
            tc_fence_after();
            mma_qk<D>(tS[1], sQ1, sK + stn * L::kTileBytes);
            tc_commit(&bar->s_full[1]);
            tc_commit(&bar->k_empty[stn]);
          } else {
            tc_commit(&bar->o_full[1]);
            tc_commit(&bar->q_empty);  // every score MMA of this tile has been issued
          }
        }
        g += ti.nB;
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 208;" ::: "memory");
    // ------------------------------------------------------------- softmax
    const int x = (warp >= 8) ? 1 : 0;  // tile A / B
    const int q4 = warp & 3;            // TMEM lane quadrant of this warp
    const int row = q4 * 32 + lane;     // row within the tile (= TMEM lane)
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const uint32_t tS = tmem + lane_off + x * 128;
    const uint32_t tO = tmem + lane_off + 256 + x * D;
    const float c = p.scale_log2;
    uint32_t cs = 0, tt = 0;
    bool ok = true;
    for (int k = 0, tile = kth_tile(0, num_tiles, p.lpt); ok && tile >= 0; tile = kth_tile(++k, num_tiles, p.lpt), ++tt) {
      const TileInfo ti = tile_info(tile, p);
      const int t = ti.t0 + x * BM + row;  // query row
      const int n = x ? ti.nB : ti.nA;
      // this row's visible keys [row_lo, row_hi) under a key-interval mask
      int row_lo = 0, row_hi = p.S;
      if constexpr (kKeyMask) {
        const int tc = t < p.T ? t : p.T - 1;
        row_lo = __ldg(p.key_lo + tc);
        row_hi = __ldg(p.key_hi + tc);
      }
      float m_used = -INFINITY, m_true = -INFINITY, l = 0.f;
      for (int j = 0; j < n; ++j, ++cs) {
        if (!(ok = mbar_wait(&bar->s_full[x], cs & 1, abort, p.err))) break;
        tc_fence_after();
        // keys at or past `lim` (tile-relative) are masked for this row
        const int kb = (ti.j0 + j) * BN;  // first key of this tile
        int lim = p.S - kb;
        if (p.causal) {
          const int lc = t + p.q_start + 1 - kb;
          lim = lc < lim ? lc : lim;
        }
        int lo_rel = 0;
        if constexpr (kKeyMask) {
          lo_rel = row_lo - kb;
          lim = row_hi - kb < lim ? row_hi - kb : lim;
        }
        const bool need_mask = __any_sync(0xffffffffu, lim < BN || lo_rel > 0);
        // the 128 scores of the row in registers, in two halves: the second half's
        // TMEM loads are in flight while the first half is masked and maxed
        uint32_t sr[BN];
        float mxa = -INFINITY, mxb = -INFINITY, mxc = -INFINITY, mxd = -INFINITY;  // 4 independent chains
#pragma unroll
        for (int ch = 0; ch < 2; ++ch) tmem_ld32(tS + ch * 32, *reinterpret_cast<uint32_t(*)[32]>(sr + ch * 32));
        tmem_wait_ld();
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          if (hf == 0) {
#pragma unroll
            for (int ch = 2; ch < 4; ++ch)
              tmem_ld32(tS + ch * 32, *reinterpret_cast<uint32_t(*)[32]>(sr + ch * 32));
          } else {
            tmem_wait_ld();
            regs_after_wait<BN / 2>(sr + BN / 2);  // no use of the second half moves above its wait
          }
          uint32_t* h = sr + hf * (BN / 2);
          if (need_mask) {
#pragma unroll
            for (int i = 0; i < BN / 2; ++i)
              if (hf * (BN / 2) + i >= lim || hf * (BN / 2) + i < lo_rel) h[i] = __float_as_uint(-INFINITY);
          }
#pragma unroll
          for (int i = 0; i < BN / 2; i += 8) {
            mxa = max3(mxa, __uint_as_float(h[i]), __uint_as_float(h[i + 1]));
            mxb = max3(mxb, __uint_as_float(h[i + 2]), __uint_as_float(h[i + 3]));
            mxc = max3(mxc, __uint_as_float(h[i + 4]), __uint_as_float(h[i + 5]));
            mxd = max3(mxd, __uint_as_float(h[i + 6]), __uint_as_float(h[i + 7]));
          }
        }
        const float mt = fmaxf(max3(mxa, mxb, mxc), mxd) * c;
        m_true = fmaxf(m_true, mt);
        if (j == 0) {
          m_used = mt;
        } else if (__any_sync(0xffffffffu, mt > m_used + kRescaleThreshold)) {
          const float m_new = fmaxf(m_used, mt);
          // a row that has seen no visible key yet (m_used = -inf) has l = 0 and O = 0: alpha 0 keeps it so
          const float alpha = m_used == -INFINITY ? 0.f : ex2(m_used - m_new);
          m_used = m_new;
          l *= alpha;
          // O is quiescent here: the commit that released S(j) also covers PV(j-1)
          uint32_t r[32];
#pragma unroll
          for (int ch = 0; ch < D / 32; ++ch) {
            tmem_ld32(tO + ch * 32, r);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
            tmem_st32(tO + ch * 32, r);
          }
        }
        const float neg_m = (m_used == -INFINITY) ? 0.f : -m_used;
        // P = exp2(s c - m) as bf16 pairs over the first 64 columns of S (chunk ch
        // lands on columns already read): packed f32x2 FMA for the argument, MUFU
        // ex2 per element, packed f32x2 adds for the row sum (two chains)
        const uint64_t c2 = f2_pack(c, c), nm2 = f2_pack(neg_m, neg_m);
        uint64_t sum_a = 0, sum_b = 0;
#pragma unroll
        for (int ch = 0; ch < BN / 32; ++ch) {
          uint32_t pk[16];
          exp_chunk(sr + ch * 32, c2, nm2, sum_a, sum_b, pk);
          tmem_st16(tS + ch * 16, pk);
        }
        float sa0, sa1, sb0, sb1;
        f2_unpack(sum_a, sa0, sa1);
        f2_unpack(sum_b, sb0, sb1);
        l += (sa0 + sa1) + (sb0 + sb1);
        tmem_wait_st();
        warp_arrive_after_tc(&bar->p_full[x]);
      }
      if (!ok || !(ok = mbar_wait(&bar->o_full[x], tt & 1, abort, p.err))) break;
      tc_fence_after();
      const float inv_l = 1.0f / l;
      const bool store = t < p.T;
      const int64_t bhq = (int64_t)ti.b * p.H + ti.h;
      // O / l as bf16 through this lane quarter's staging region (tiles A and B
      // take turns: use n waits for use n - 1's stores to have read it) and TMA
      // stores, which drop rows past T
      const uint32_t stg = smem_u32(smem + L::kStg) + q4 * (D / 64) * 4096;
      const uint32_t use = 2 * tt + x;
      if (use > 0 && !(ok = mbar_wait(&bar->stg_free[q4], (use - 1) & 1, abort, p.err))) break;
#pragma unroll
      for (int ch = 0; ch < D / 32; ++ch) {
        uint32_t r[32];
        tmem_ld32(tO + ch * 32, r);
        tmem_wait_ld();
        if (ch == D / 32 - 1) warp_arrive_after_tc(&bar->o_empty[x]);  // O_x may now be overwritten by the next tile
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          pk[i] = pack_bf16(__uint_as_float(r[2 * i]) * inv_l, __uint_as_float(r[2 * i + 1]) * inv_l);
        const uint32_t rowb = stg + (ch >> 1) * 4096 + lane * 128;
#pragma unroll
        for (int i = 0; i < 4; ++i)
          sts128(rowb + ((((ch & 1) * 4 + i) ^ (lane & 7)) << 4), pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
#pragma unroll
        for (int bx = 0; bx < D / 64; ++bx)  // boxes wholly past the value head dim are not stored
          if (bx * 64 < p.DV) tma_store_4d(&tm_o, stg + bx * 4096, bx * 64, ti.t0 + x * BM + q4 * 32, ti.h, ti.b);
        bulk_commit();
        bulk_wait_read_all();
        mbar_arrive(&bar->stg_free[q4]);
      }
      if (store) {
        const int64_t idx = bhq * p.T + t;
        constexpr float kLn2 = 0.6931471805599453f;
        if (p.lse) p.lse[idx] = (m_used + __log2f(l)) * kLn2;
        if (p.m) p.m[idx] = m_true * kLn2;
        if (p.den) p.den[idx] = l * ex2(m_used - m_true);
      }
    }
    if (lane == 0) bulk_wait_all();  // the O stores are complete before the CTA retires
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// D = 64: P in its own TMEM columns.  With D = 128 the 512 TMEM columns hold
// S_A, S_B, O_A, O_B and P must alias S, so a tile's next score MMA waits for
// its PV (softmax, PV and QK form one chain per tile).  With D = 64 the O
// accumulators take 64 columns each, which leaves room for P_A, P_B:
//   S_A [0,128) S_B [128,256) O_A [256,320) O_B [320,384) P_A [384,448) P_B [448,512)
// so S_x(j+1) is issued as soon as softmax x holds S_x(j) in registers
// (s_free) and runs under the exponentials of step j; PV_x(j) releases P_x
// (p_free) for step j+1.  K and V have their own producer threads and the
// score and PV MMAs their own issuing threads, so no in-order wait of one
// stream holds up the other.
struct __align__(8) BarriersD64 {
  uint64_t q_full, q_empty;
  uint64_t k_full[2], k_empty[2];
  uint64_t v_full[2], v_empty[2];
  uint64_t s_full[2];   // score MMA done -> softmax x
  uint64_t s_free[2];   // softmax x holds S in registers -> next score MMA (4 warp arrivals)
  uint64_t p_full[2];   // P_x written -> PV (4 warp arrivals)
  uint64_t p_free[2];   // PV_x done: P_x may be rewritten, O_x is quiescent
  uint64_t o_full[2], o_empty[2];
  uint32_t tmem_base;
  int abort;
};

template <bool kKeyMask>
__global__ void __launch_bounds__(kThreads, 1)
    flash_fwd_d64_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, const FwdParams p) {
  constexpr int D = 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  using L = Smem<D>;  // Q_A, Q_B, K x 2, V x 2
  BarriersD64* bar = reinterpret_cast<BarriersD64*>(smem + L::kBar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_tiles = p.num_mblocks * p.H * p.B;

  if (threadIdx.x == 0) {
    mbar_init(&bar->q_full, 1);
    mbar_init(&bar->q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar->k_full[i], 1);
      mbar_init(&bar->k_empty[i], 1);
      mbar_init(&bar->v_full[i], 1);
      mbar_init(&bar->v_empty[i], 1);
      mbar_init(&bar->s_full[i], 1);
      mbar_init(&bar->s_free[i], BM / 32);
      mbar_init(&bar->p_full[i], BM / 32);
      mbar_init(&bar->p_free[i], 1);
      mbar_init(&bar->o_full[i], 1);
      mbar_init(&bar->o_empty[i], BM / 32);
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
  const uint32_t sQ[2] = {smem_u32(smem + L::kQ0), smem_u32(smem + L::kQ1)};
  const uint32_t sK = smem_u32(smem + L::kK), sV = smem_u32(smem + L::kV);

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 88;" ::: "memory");
    if (warp == 0 && lane == 0) {
      // -------------------------------------------------- Q and K producer
      prefetch_tensormap(&tm_q);
      prefetch_tensormap(&tm_k);
      uint32_t gk = 0, tt = 0;
      bool ok = true;
      for (int k = 0, tile = kth_tile(0, num_tiles, p.lpt); ok && tile >= 0; tile = kth_tile(++k, num_tiles, p.lpt), ++tt) {
        const TileInfo ti = tile_info(tile, p);
        if (!(ok = mbar_wait(&bar->q_empty, (tt & 1) ^ 1, abort, p.err))) break;
        mbar_expect_tx(&bar->q_full, 2 * L::kTileBytes);
        tma_load_4d(smem + L::kQ0, &tm_q, &bar->q_full, 0, ti.t0, ti.h, ti.b);
        tma_load_4d(smem + L::kQ1, &tm_q, &bar->q_full, 0, ti.t0 + BM, ti.h, ti.b);
        for (int j = 0; j < ti.nB; ++j, ++gk) {
          const int st = gk & 1;
          if (!(ok = mbar_wait(&bar->k_empty[st], ((gk >> 1) & 1) ^ 1, abort, p.err))) break;
          mbar_expect_tx(&bar->k_full[st], L::kTileBytes);
          tma_load_4d(smem + L::kK + st * L::kTileBytes, &tm_k, &bar->k_full[st], 0, (ti.j0 + j) * BN, ti.hk, ti.b);
        }
      }
    } else if (warp == 2 && lane == 0) {
      // -------------------------------------------------------- V producer
      prefetch_tensormap(&tm_v);
      uint32_t gv = 0;
      bool ok = true;
      for (int k = 0, tile = kth_tile(0, num_tiles, p.lpt); ok && tile >= 0; tile = kth_tile(++k, num_tiles, p.lpt)) {
        const TileInfo ti = tile_info(tile, p);
        for (int j = 0; j < ti.nB; ++j, ++gv) {
          const int st = gv & 1;
          if (!(ok = mbar_wait(&bar->v_empty[st], ((gv >> 1) & 1) ^ 1, abort, p.err))) break;
          mbar_expect_tx(&bar->v_full[st], L::kTileBytes);
          tma_load_4d(smem + L::kV + st * L::kTileBytes, &tm_v, &bar->v_full[st], 0, (ti.j0 + j) * BN, ti.hk, ti.b);
        }
      }
    } else if (warp == 1 && lane == 0) {
      // ------------------------------------------ score MMA issuer (QK)
      const uint32_t tS[2] = {tmem + 0, tmem + 128};
      uint32_t gk = 0, tt = 0, nqk[2] = {0, 0};
      bool ok = true;
      auto issue_qk = [&](int x) -> bool {
        // S_x may only be overwritten once softmax x holds the previous one in registers
        if (nqk[x] > 0 && !mbar_wait(&bar->s_free[x], (nqk[x] - 1) & 1, abort, p.err)) return false;
        tc_fence_after();
        mma_qk<D>(tS[x], sQ[x], sK + (gk & 1) * L::kTileBytes);
        tc_commit(&bar->s_full[x]);
        ++nqk[x];
        return true;
      };
      for (int k = 0, tile = kth_tile(0, num_tiles, p.lpt); ok && tile >= 0; tile = kth_tile(++k, num_tiles, p.lpt), ++tt) {
        const TileInfo ti = tile_info(tile, p);
        if (!(ok = mbar_wait(&bar->q_full, tt & 1, abort, p.err))) break;
        for (int j = 0; ok && j < ti.nB; ++j) {
          if (!(ok = mbar_wait(&bar->k_full[gk & 1], (gk >> 1) & 1, abort, p.err))) break;
          if (j < ti.nA && !(ok = issue_qk(0))) break;
          if (!(ok = issue_qk(1))) break;
          tc_commit(&bar->k_empty[gk & 1]);
          ++gk;
        }
        if (ok) tc_commit(&bar->q_empty);  // every score MMA of this tile has been issued
      }
    } else if (warp == 3 && lane == 0) {
      // ------------------------------------------------ PV MMA issuer
      const uint32_t tO[2] = {tmem + 256, tmem + 256 + D};
      const uint32_t tP[2] = {tmem + 384, tmem + 448};
      uint32_t gv = 0, tt = 0, npf[2] = {0, 0};
      bool ok = true;
      for (int k = 0, tile = kth_tile(0, num_tiles, p.lpt); ok && tile >= 0; tile = kth_tile(++k, num_tiles, p.lpt), ++tt) {
        const TileInfo ti = tile_info(tile, p);
        for (int j = 0; ok && j < ti.nB; ++j) {
          const int st = gv & 1;
          if (!(ok = mbar_wait(&bar->v_full[st], (gv >> 1) & 1, abort, p.err))) break;
          for (int x = 0; x < 2; ++x) {
            if (x == 0 && j >= ti.nA) continue;
            if (!(ok = mbar_wait(&bar->p_full[x], npf[x] & 1, abort, p.err))) break;
            ++npf[x];
            if (j == 0 && !(ok = mbar_wait(&bar->o_empty[x], (tt & 1) ^ 1, abort, p.err))) break;
            tc_fence_after();
            mma_pv<D>(tO[x], tP[x], sV + st * L::kTileBytes, j > 0);
            tc_commit(&bar->p_free[x]);
            if (j + 1 == (x ? ti.nB : ti.nA)) tc_commit(&bar->o_full[x]);
          }
          if (!ok) break;
          tc_commit(&bar->v_empty[st]);
          ++gv;
        }
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 208;" ::: "memory");
    // ------------------------------------------------------------- softmax
    const int x = (warp >= 8) ? 1 : 0;  // tile A / B
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const uint32_t tS = tmem + lane_off + x * 128;
    const uint32_t tO = tmem + lane_off + 256 + x * D;
    const uint32_t tP = tmem + lane_off + 384 + x * 64;
    const float c = p.scale_log2;
    uint32_t cs = 0, tt = 0, pw = 0;  // S tiles read, work tiles, P tiles written
    bool ok = true;
    for (int k = 0, tile = kth_tile(0, num_tiles, p.lpt); ok && tile >= 0; tile = kth_tile(++k, num_tiles, p.lpt), ++tt) {
      const TileInfo ti = tile_info(tile, p);
      const int t = ti.t0 + x * BM + row;
      const int n = x ? ti.nB : ti.nA;
      // this row's visible keys [row_lo, row_hi) under a key-interval mask
      int row_lo = 0, row_hi = p.S;
      if constexpr (kKeyMask) {
        const int tc = t < p.T ? t : p.T - 1;
        row_lo = __ldg(p.key_lo + tc);
        row_hi = __ldg(p.key_hi + tc);
      }
      float m_used = -INFINITY, m_true = -INFINITY, l = 0.f;
      for (int j = 0; j < n; ++j, ++cs) {
        if (!(ok = mbar_wait(&bar->s_full[x], cs & 1, abort, p.err))) break;
        tc_fence_after();
        const int kb = (ti.j0 + j) * BN;  // first key of this tile
        int lim = p.S - kb;
        if (p.causal) {
          const int lc = t + p.q_start + 1 - kb;
          lim = lc < lim ? lc : lim;
        }
        int lo_rel = 0;
        if constexpr (kKeyMask) {
          lo_rel = row_lo - kb;
          lim = row_hi - kb < lim ? row_hi - kb : lim;
        }
        const bool need_mask = __any_sync(0xffffffffu, lim < BN || lo_rel > 0);
        uint32_t sr[BN];
#pragma unroll
        for (int ch = 0; ch < BN / 32; ++ch) tmem_ld32(tS + ch * 32, *reinterpret_cast<uint32_t(*)[32]>(sr + ch * 32));
        tmem_wait_ld();
        warp_arrive_after_tc(&bar->s_free[x]);  // the next score MMA of this tile may overwrite S_x
        if (need_mask) {
#pragma unroll
          for (int i = 0; i < BN; ++i)
            if (i >= lim || i < lo_rel) sr[i] = __float_as_uint(-INFINITY);
        }
        float mxa = -INFINITY, mxb = -INFINITY, mxc = -INFINITY, mxd = -INFINITY;
#pragma unroll
        for (int i = 0; i < BN; i += 8) {
          mxa = max3(mxa, __uint_as_float(sr[i]), __uint_as_float(sr[i + 1]));
          mxb = max3(mxb, __uint_as_float(sr[i + 2]), __uint_as_float(sr[i + 3]));
          mxc = max3(mxc, __uint_as_float(sr[i + 4]), __uint_as_float(sr[i + 5]));
          mxd = max3(mxd, __uint_as_float(sr[i + 6]), __uint_as_float(sr[i + 7]));
        }
        const float mt = fmaxf(max3(mxa, mxb, mxc), mxd) * c;
        m_true = fmaxf(m_true, mt);
        // PV_x(j-1) must be done before P_x is rewritten or O_x rescaled
        if (pw > 0 && !(ok = mbar_wait(&bar->p_free[x], (pw - 1) & 1, abort, p.err))) break;
        tc_fence_after();
        if (j == 0) {
          m_used = mt;
        } else if (__any_sync(0xffffffffu, mt > m_used + kRescaleThreshold)) {
          const float m_new = fmaxf(m_used, mt);
          // a row that has seen no visible key yet (m_used = -inf) has l = 0 and O = 0: alpha 0 keeps it so
          const float alpha = m_used == -INFINITY ? 0.f : ex2(m_used - m_new);
          m_used = m_new;
          l *= alpha;
          uint32_t r[32];
#pragma unroll
          for (int ch = 0; ch < D / 32; ++ch) {
            tmem_ld32(tO + ch * 32, r);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
            tmem_st32(tO + ch * 32, r);
          }
        }
        const float neg_m = (m_used == -INFINITY) ? 0.f : -m_used;
        const uint64_t c2 = f2_pack(c, c), nm2 = f2_pack(neg_m, neg_m);
        uint64_t sum_a = 0, sum_b = 0;
#pragma unroll
        for (int ch = 0; ch < BN / 32; ++ch) {
          uint32_t pk[16];
          exp_chunk(sr + ch * 32, c2, nm2, sum_a, sum_b, pk);
          tmem_st16(tP + ch * 16, pk);
        }
        float sa0, sa1, sb0, sb1;
        f2_unpack(sum_a, sa0, sa1);
        f2_unpack(sum_b, sb0, sb1);
        l += (sa0 + sa1) + (sb0 + sb1);
        tmem_wait_st();
        warp_arrive_after_tc(&bar->p_full[x]);
        ++pw;
      }
      if (!ok || !(ok = mbar_wait(&bar->o_full[x], tt & 1, abort, p.err))) break;
      tc_fence_after();
      const float inv_l = 1.0f / l;
      const bool store = t < p.T;
      const int64_t bhq = (int64_t)ti.b * p.H + ti.h;
      __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(p.o) + (int64_t)ti.b * p.o_stride[0] +
                            (int64_t)ti.h * p.o_stride[1] + (int64_t)t * p.o_stride[2];
#pragma unroll
      for (int ch = 0; ch < D / 32; ++ch) {
        uint32_t r[32];
        tmem_ld32(tO + ch * 32, r);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          pk[i] = pack_bf16(__uint_as_float(r[2 * i]) * inv_l, __uint_as_float(r[2 * i + 1]) * inv_l);
        if (store) {
          uint4* dst = reinterpret_cast<uint4*>(orow + ch * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i)  // columns past the value head dim are padding (zero by construction)
            if (ch * 32 + i * 8 < p.DV) dst[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
        }
      }
      warp_arrive_after_tc(&bar->o_empty[x]);
      if (store) {
        const int64_t idx = bhq * p.T + t;
        constexpr float kLn2 = 0.6931471805599453f;
        if (p.lse) p.lse[idx] = (m_used + __log2f(l)) * kLn2;
        if (p.m) p.m[idx] = m_true * kLn2;
        if (p.den) p.den[idx] = l * ex2(m_used - m_true);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D>
int launch(const pdb_flash_desc& d, cudaStream_t stream) {
  CUtensorMap tq, tk, tv;
  const uint32_t box[4] = {64, 128, 1, 1};
  // The maps carry the true head dims: feature columns from head_dim (q, k) or
  // head_dim_v (v) up to D are zero-filled by the TMA, so they add nothing to the
  // scores and produce zero output columns, which the stores drop.
  {
    const uint64_t dims[4] = {(uint64_t)d.head_dim, (uint64_t)d.seqlen_q, (uint64_t)d.heads_q, (uint64_t)d.batch};
    const uint64_t str[3] = {(uint64_t)d.q_stride[2] * 2, (uint64_t)d.q_stride[1] * 2, (uint64_t)d.q_stride[0] * 2};
    if (int st = encode_tma_4d(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, d.q, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return st;
  }
  {
    const uint64_t dk[4] = {(uint64_t)d.head_dim, (uint64_t)d.seqlen_k, (uint64_t)d.heads_kv, (uint64_t)d.batch};
    const uint64_t dv[4] = {(uint64_t)d.head_dim_v, (uint64_t)d.seqlen_k, (uint64_t)d.heads_kv, (uint64_t)d.batch};
    const uint64_t sk[3] = {(uint64_t)d.k_stride[2] * 2, (uint64_t)d.k_stride[1] * 2, (uint64_t)d.k_stride[0] * 2};
    const uint64_t sv[3] = {(uint64_t)d.v_stride[2] * 2, (uint64_t)d.v_stride[1] * 2, (uint64_t)d.v_stride[0] * 2};
    if (int st = encode_tma_4d(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, d.k, dk, sk, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return st;
    if (int st = encode_tma_4d(&tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, d.v, dv, sv, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return st;
  }
  FwdParams p;
  p.o = d.o;
  p.lse = d.lse;
  p.m = d.m;
  p.den = d.den;
  for (int i = 0; i < 3; ++i) p.o_stride[i] = d.o_stride[i];
  p.T = (int)d.seqlen_q;
  p.S = (int)d.seqlen_k;
  p.DV = (int)d.head_dim_v;
  p.H = (int)d.heads_q;
  p.HKV = (int)d.heads_kv;
  p.B = (int)d.batch;
  p.q_start = (int)d.q_start;
  p.causal = d.causal ? 1 : 0;
  p.key_lo = d.key_lo;
  p.key_hi = d.key_hi;
  p.mask_monotone = d.mask_monotone ? 1 : 0;
  p.num_mblocks = (int)((d.seqlen_q + 2 * BM - 1) / (2 * BM));
  p.scale_log2 = (float)(d.scale * 1.4426950408889634);
  p.err = device_error_flag();
  const int64_t nblk = (int64_t)p.num_mblocks * d.heads_q * d.batch;
  if (nblk > 0x7fffffffLL) return set_error(PDB_ERR_SHAPE, "bf16 flash: grid too large");
  int dev = 0;
  cudaGetDevice(&dev);
  const int64_t pairs = (nblk + 1) / 2;
  int sms = sm_count(dev) - (d.sm_margin > 0 ? d.sm_margin : 0);
  if (sms < 1) sms = 1;
  // a job of fewer than 4 waves of pairs schedules single tiles heaviest first
  p.lpt = pairs < 4 * (int64_t)sms ? 1 : 0;
  const int64_t units = p.lpt ? nblk : pairs;
  const int64_t grid = units < sms ? units : sms;  // persistent: one CTA per SM
  const int smem = Smem<D>::kTotal;
  if constexpr (D == 64) {  // P in its own TMEM columns (656 vs 610 TFLOP/s at B8 H32 S4096 causal)
    auto kern = p.key_lo ? flash_fwd_d64_kernel<true> : flash_fwd_d64_kernel<false>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return cuda_status(e, "bf16 flash: set smem attribute");
    kern<<<(unsigned)grid, kThreads, smem, stream>>>(tq, tk, tv, p);
    return cuda_status(cudaGetLastError(), "bf16 flash launch");
  } else {
  CUtensorMap to;  // O stores: 32-row boxes, one per softmax warp
  {
    const uint64_t dims[4] = {(uint64_t)d.head_dim_v, (uint64_t)d.seqlen_q, (uint64_t)d.heads_q, (uint64_t)d.batch};
    const uint64_t so[3] = {(uint64_t)d.o_stride[2] * 2, (uint64_t)d.o_stride[1] * 2, (uint64_t)d.o_stride[0] * 2};
    const uint32_t obox[4] = {64, 32, 1, 1};
    if (int st = encode_tma_4d(&to, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, d.o, dims, so, obox, CU_TENSOR_MAP_SWIZZLE_128B))
      return st;
  }
  auto kern = p.key_lo ? flash_fwd_sm100_kernel<D, true> : flash_fwd_sm100_kernel<D, false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return cuda_status(e, "bf16 flash: set smem attribute");
  kern<<<(unsigned)grid, kThreads, smem, stream>>>(tq, tk, tv, to, p);
  return cuda_status(cudaGetLastError(), "bf16 flash launch");
  }
}


// ---------------------------------------------------------------------------
// Head dims up to 256 (e and e_v in (128, 256]): one 128-row query tile per
// work tile.  TMEM: S0 [0,128) S1 [128,256) O [256,512) -- the O accumulator
// takes 256 columns, so there is room for two score buffers but not for a
// second query tile.  The score MMA of key tile j+1 is issued into the other
// buffer before the PV of key tile j, so the softmax of tile j+1 finds its
// scores ready when it finishes tile j; P (bf16) overwrites the first 64
// columns of its own S buffer, and the score MMA of tile j+2 into that buffer
// is issued after the PV that reads it (tcgen05 ops of one thread run in
// order).  Shared memory: Q (128 x 256, 64 KB) and a ring of five 32 KB slots
// (128 keys x 128 features each), through which K and V halves stream in the
// order the MMAs consume them: K0, then per key tile j: K(j+1), V(j).
//   warp 0        TMA producer        warp 1   MMA issuer (one thread)
//   warp 2        TMEM allocator      warps 4..7  softmax + epilogue
constexpr int kThreads256 = 256;
constexpr int kSlots256 = 5;
constexpr int kSlotBytes256 = 2 * kBoxBytes;  // 128 rows x 128 bf16
constexpr int kQ256 = 0;
constexpr int kRing256 = 4 * kBoxBytes;
constexpr int kBar256 = kRing256 + kSlots256 * kSlotBytes256;
constexpr int kSmem256 = kBar256 + 1024 + 1024;

struct __align__(8) Barriers256 {
  uint64_t q_full, q_empty;
  uint64_t slot_full[kSlots256], slot_empty[kSlots256];
  uint64_t s_full[2];  // score MMA into buffer b done -> softmax
  uint64_t p_full[2];  // P in buffer b written -> PV (4 warp arrivals)
  uint64_t pv_done;    // one completion per key tile's PV: O is quiescent up to it
  uint64_t o_full, o_empty;
  uint32_t tmem_base;
  int abort;
};

// 128-row work tiles: ordinal -> (b, h, row block), key tiles j0 .. j0 + n - 1.
__device__ __forceinline__ TileInfo tile_info128(int tile, const FwdParams& p) {
  TileInfo ti;
  int bh, mblk;
  if (p.lpt) {
    const int nbh = p.H * p.B;
    bh = tile % nbh;
    mblk = p.num_mblocks - 1 - tile / nbh;
  } else {
    bh = tile / p.num_mblocks;
    const int r = tile % p.num_mblocks;
    mblk = (r & 1) ? (r >> 1) : p.num_mblocks - 1 - (r >> 1);
  }
  ti.b = bh / p.H;
  ti.h = bh % p.H;
  ti.hk = ti.h / (p.H / p.HKV);
  ti.t0 = mblk * BM;
  const int n_kv = (p.S + BN - 1) / BN;
  const int first = ti.t0 < p.T ? ti.t0 : p.T - 1;
  int last_row = ti.t0 + BM - 1;
  if (last_row > p.T - 1) last_row = p.T - 1;
  ti.j0 = 0;
  if (p.key_lo && p.mask_monotone) ti.j0 = __ldg(p.key_lo + first) / BN;
  int c = n_kv;
  if (p.causal) c = (last_row + p.q_start) / BN + 1;
  else if (p.key_lo && p.mask_monotone) c = (__ldg(p.key_hi + last_row) + BN - 1) / BN;
  c = c < n_kv ? c : n_kv;
  ti.nA = ti.nB = c - ti.j0 > 1 ? c - ti.j0 : 1;
  return ti;
}

template <bool kKeyMask>
__global__ void __launch_bounds__(kThreads256, 1)
    flash_fwd_d256_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                          const __grid_constant__ CUtensorMap tm_v, const FwdParams p) {
  constexpr int D = 256;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Barriers256* bar = reinterpret_cast<Barriers256*>(smem + kBar256);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_tiles = p.num_mblocks * p.H * p.B;

  if (threadIdx.x == 0) {
    mbar_init(&bar->q_full, 1);
    mbar_init(&bar->q_empty, 1);
    for (int i = 0; i < kSlots256; ++i) {
      mbar_init(&bar->slot_full[i], 1);
      mbar_init(&bar->slot_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar->s_full[i], 1);
      mbar_init(&bar->p_full[i], BM / 32);
    }
    mbar_init(&bar->pv_done, 1);
    mbar_init(&bar->o_full, 1);
    mbar_init(&bar->o_empty, BM / 32);
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
  const uint32_t sQ = smem_u32(smem + kQ256), sRing = smem_u32(smem + kRing256);

  if (warp < 4) {
    if (warp == 0 && lane == 0) {
      // ---------------------------------------------------------- producer
      prefetch_tensormap(&tm_q);
      prefetch_tensormap(&tm_k);
      prefetch_tensormap(&tm_v);
      uint32_t g = 0, tt = 0;  // slot loads issued, tiles started
      // one 32 KB slot: 128 keys x features [128 h, 128 h + 128) of K or V
      auto load_half = [&](const CUtensorMap* m, int h, int key0, int hk, int b) -> bool {
        const uint32_t slot = g % kSlots256, ph = (g / kSlots256) & 1;
        if (!mbar_wait(&bar->slot_empty[slot], ph ^ 1, abort, p.err)) return false;
        mbar_expect_tx(&bar->slot_full[slot], kSlotBytes256);
        uint8_t* dst = smem + kRing256 + slot * kSlotBytes256;
        tma_load_4d(dst, m, &bar->slot_full[slot], h * 128, key0, hk, b);
        tma_load_4d(dst + kBoxBytes, m, &bar->slot_full[slot], h * 128 + 64, key0, hk, b);
        ++g;
        return true;
      };
      bool ok = true;
      for (int k = 0, tile = kth_tile(0, num_tiles, p.lpt); ok && tile >= 0;
           tile = kth_tile(++k, num_tiles, p.lpt), ++tt) {
        const TileInfo ti = tile_info128(tile, p);
        if (!(ok = mbar_wait(&bar->q_empty, (tt & 1) ^ 1, abort, p.err))) break;
        mbar_expect_tx(&bar->q_full, 4 * kBoxBytes);
        for (int i = 0; i < 4; ++i)
          tma_load_4d(smem + kQ256 + i * kBoxBytes, &tm_q, &bar->q_full, i * 64, ti.t0, ti.h, ti.b);
        const int n = ti.nA;
        ok = load_half(&tm_k, 0, ti.j0 * BN, ti.hk, ti.b) && load_half(&tm_k, 1, ti.j0 * BN, ti.hk, ti.b);
        for (int j = 0; ok && j < n; ++j) {
          const int key0 = (ti.j0 + j) * BN;
          if (j + 1 < n)
            ok = load_half(&tm_k, 0, key0 + BN, ti.hk, ti.b) && load_half(&tm_k, 1, key0 + BN, ti.hk, ti.b);
          ok = ok && load_half(&tm_v, 0, key0, ti.hk, ti.b) && load_half(&tm_v, 1, key0, ti.hk, ti.b);
        }
      }
    } else if (warp == 1 && lane == 0) {
      // -------------------------------------------------------- MMA issuer
      const uint32_t tO = tmem + 256;
      uint32_t g = 0, tt = 0, sc = 0;  // slots consumed, tiles, score tiles issued
      constexpr uint32_t idesc_s = idesc_bf16(BM, BN, 0, 0);
      constexpr uint32_t idesc_o = idesc_bf16(BM, 128, 0, 1);
      auto take_slot = [&](uint32_t& saddr, uint32_t& slot) -> bool {
        slot = g % kSlots256;
        if (!mbar_wait(&bar->slot_full[slot], (g / kSlots256) & 1, abort, p.err)) return false;
        tc_fence_after();
        saddr = sRing + slot * kSlotBytes256;
        ++g;
        return true;
      };
      // S_b = Q K^T over 256 features (16 K16 steps, K in two slots)
      auto qk = [&](uint32_t b) -> bool {
        for (int h = 0; h < 2; ++h) {
          uint32_t ks, slot;
          if (!take_slot(ks, slot)) return false;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int kk = h * 8 + i;
            const uint32_t qoff = (kk >> 2) * kBoxBytes + (kk & 3) * 32;
            const uint32_t koff = (i >> 2) * kBoxBytes + (i & 3) * 32;
            mma_ss(tmem + b * 128, sdesc_sw128(sQ + qoff, 16, 1024), sdesc_sw128(ks + koff, 16, 1024), idesc_s,
                   kk > 0 ? 1u : 0u);
          }
          tc_commit(&bar->slot_empty[slot]);
        }
        tc_commit(&bar->s_full[b]);
        return true;
      };
      // O[:, 128 h .. 128 h + 128) += P_b V_h, P from TMEM (the first 64 columns of S_b)
      auto pv = [&](uint32_t b, bool acc) -> bool {
        for (int h = 0; h < 2; ++h) {
          uint32_t vs, slot;
          if (!take_slot(vs, slot)) return false;
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk)
            mma_ts(tO + h * 128, tmem + b * 128 + kk * 8, sdesc_sw128(vs + kk * 2048, kBoxBytes, 1024), idesc_o,
                   (acc || kk > 0) ? 1u : 0u);
          tc_commit(&bar->slot_empty[slot]);
        }
        tc_commit(&bar->pv_done);
        return true;
      };
      bool ok = true;
      for (int k = 0, tile = kth_tile(0, num_tiles, p.lpt); ok && tile >= 0;
           tile = kth_tile(++k, num_tiles, p.lpt), ++tt) {
        const TileInfo ti = tile_info128(tile, p);
        const int n = ti.nA;
        if (!(ok = mbar_wait(&bar->q_full, tt & 1, abort, p.err))) break;
        if (!(ok = qk(sc & 1))) break;
        if (n == 1) tc_commit(&bar->q_empty);
        for (int j = 0; ok && j < n; ++j) {
          const uint32_t s = sc + j;
          if (j + 1 < n) {
            if (!(ok = qk((s + 1) & 1))) break;
            if (j + 2 == n) tc_commit(&bar->q_empty);  // every score MMA of this tile has been issued
          }
          if (!(ok = mbar_wait(&bar->p_full[s & 1], (s >> 1) & 1, abort, p.err))) break;
          if (j == 0 && !(ok = mbar_wait(&bar->o_empty, (tt & 1) ^ 1, abort, p.err))) break;
          tc_fence_after();
          if (!(ok = pv(s & 1, j > 0))) break;
        }
        if (!ok) break;
        tc_commit(&bar->o_full);
        sc += n;
      }
    }
  } else {
    // ------------------------------------------------------------- softmax
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const uint32_t tO = tmem + lane_off + 256;
    const float c = p.scale_log2;
    uint32_t gs = 0, tt = 0;  // score tiles read, work tiles
    bool ok = true;
    for (int k = 0, tile = kth_tile(0, num_tiles, p.lpt); ok && tile >= 0;
         tile = kth_tile(++k, num_tiles, p.lpt), ++tt) {
      const TileInfo ti = tile_info128(tile, p);
      const int t = ti.t0 + row;
      const int n = ti.nA;
      int row_lo = 0, row_hi = p.S;
      if constexpr (kKeyMask) {
        const int tc = t < p.T ? t : p.T - 1;
        row_lo = __ldg(p.key_lo + tc);
        row_hi = __ldg(p.key_hi + tc);
      }
      float m_used = -INFINITY, m_true = -INFINITY, l = 0.f;
      for (int j = 0; j < n; ++j, ++gs) {
        const uint32_t b = gs & 1;
        const uint32_t tS = tmem + lane_off + b * 128;
        if (!(ok = mbar_wait(&bar->s_full[b], (gs >> 1) & 1, abort, p.err))) break;
        tc_fence_after();
        const int kb = (ti.j0 + j) * BN;
        int lim = p.S - kb;
        if (p.causal) {
          const int lc = t + p.q_start + 1 - kb;
          lim = lc < lim ? lc : lim;
        }
        int lo_rel = 0;
        if constexpr (kKeyMask) {
          lo_rel = row_lo - kb;
          lim = row_hi - kb < lim ? row_hi - kb : lim;
        }
        const bool need_mask = __any_sync(0xffffffffu, lim < BN || lo_rel > 0);
        uint32_t sr[BN];
        float mxa = -INFINITY, mxb = -INFINITY, mxc = -INFINITY, mxd = -INFINITY;
#pragma unroll
        for (int ch = 0; ch < 2; ++ch) tmem_ld32(tS + ch * 32, *reinterpret_cast<uint32_t(*)[32]>(sr + ch * 32));
        tmem_wait_ld();
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          if (hf == 0) {
#pragma unroll
            for (int ch = 2; ch < 4; ++ch)
              tmem_ld32(tS + ch * 32, *reinterpret_cast<uint32_t(*)[32]>(sr + ch * 32));
          } else {
            tmem_wait_ld();
            regs_after_wait<BN / 2>(sr + BN / 2);
          }
          uint32_t* hv = sr + hf * (BN / 2);
          if (need_mask) {
#pragma unroll
            for (int i = 0; i < BN / 2; ++i)
              if (hf * (BN / 2) + i >= lim || hf * (BN / 2) + i < lo_rel) hv[i] = __float_as_uint(-INFINITY);
          }
#pragma unroll
          for (int i = 0; i < BN / 2; i += 8) {
            mxa = max3(mxa, __uint_as_float(hv[i]), __uint_as_float(hv[i + 1]));
            mxb = max3(mxb, __uint_as_float(hv[i + 2]), __uint_as_float(hv[i + 3]));
            mxc = max3(mxc, __uint_as_float(hv[i + 4]), __uint_as_float(hv[i + 5]));
            mxd = max3(mxd, __uint_as_float(hv[i + 6]), __uint_as_float(hv[i + 7]));
          }
        }
        const float mt = fmaxf(max3(mxa, mxb, mxc), mxd) * c;
        m_true = fmaxf(m_true, mt);
        if (j == 0) {
          m_used = mt;
        } else if (__any_sync(0xffffffffu, mt > m_used + kRescaleThreshold)) {
          const float m_new = fmaxf(m_used, mt);
          const float alpha = m_used == -INFINITY ? 0.f : ex2(m_used - m_new);
          m_used = m_new;
          l *= alpha;
          // O holds the PVs up to key tile j - 1 once that PV has completed
          if (!(ok = mbar_wait(&bar->pv_done, (gs - 1) & 1, abort, p.err))) break;
          tc_fence_after();
          uint32_t r[32];
#pragma unroll 1
          for (int ch = 0; ch < D / 32; ++ch) {
            tmem_ld32(tO + ch * 32, r);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
            tmem_st32(tO + ch * 32, r);
          }
        }
        const float neg_m = (m_used == -INFINITY) ? 0.f : -m_used;
        const uint64_t c2 = f2_pack(c, c), nm2 = f2_pack(neg_m, neg_m);
        uint64_t sum_a = 0, sum_b = 0;
#pragma unroll
        for (int ch = 0; ch < BN / 32; ++ch) {
          uint32_t pk[16];
          exp_chunk(sr + ch * 32, c2, nm2, sum_a, sum_b, pk);
          tmem_st16(tS + ch * 16, pk);
        }
        float sa0, sa1, sb0, sb1;
        f2_unpack(sum_a, sa0, sa1);
        f2_unpack(sum_b, sb0, sb1);
        l += (sa0 + sa1) + (sb0 + sb1);
        tmem_wait_st();
        warp_arrive_after_tc(&bar->p_full[b]);
      }
      if (!ok || !(ok = mbar_wait(&bar->o_full, tt & 1, abort, p.err))) break;
      tc_fence_after();
      const float inv_l = 1.0f / l;
      const bool store = t < p.T;
      const int64_t bhq = (int64_t)ti.b * p.H + ti.h;
      __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(p.o) + (int64_t)ti.b * p.o_stride[0] +
                            (int64_t)ti.h * p.o_stride[1] + (int64_t)t * p.o_stride[2];
#pragma unroll 1
      for (int ch = 0; ch < D / 32; ++ch) {
        if (ch * 32 >= p.DV) break;  // columns past the value head dim are zero padding
        uint32_t r[32];
        tmem_ld32(tO + ch * 32, r);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          pk[i] = pack_bf16(__uint_as_float(r[2 * i]) * inv_l, __uint_as_float(r[2 * i + 1]) * inv_l);
        if (store) {
          uint4* dst = reinterpret_cast<uint4*>(orow + ch * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            if (ch * 32 + i * 8 < p.DV) dst[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
        }
      }
      warp_arrive_after_tc(&bar->o_empty);
      if (store) {
        const int64_t idx = bhq * p.T + t;
        constexpr float kLn2 = 0.6931471805599453f;
        if (p.lse) p.lse[idx] = (m_used + __log2f(l)) * kLn2;
        if (p.m) p.m[idx] = m_true * kLn2;
        if (p.den) p.den[idx] = l * ex2(m_used - m_true);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

int launch256(const pdb_flash_desc& d, cudaStream_t stream) {
  CUtensorMap tq, tk, tv;
  const uint32_t box[4] = {64, 128, 1, 1};
  {  // the maps carry the true head dims; features up to 256 are zero-filled
    const uint64_t dims[4] = {(uint64_t)d.head_dim, (uint64_t)d.seqlen_q, (uint64_t)d.heads_q, (uint64_t)d.batch};
    const uint64_t str[3] = {(uint64_t)d.q_stride[2] * 2, (uint64_t)d.q_stride[1] * 2, (uint64_t)d.q_stride[0] * 2};
    if (int st = encode_tma_4d(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, d.q, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return st;
    const uint64_t dk[4] = {(uint64_t)d.head_dim, (uint64_t)d.seqlen_k, (uint64_t)d.heads_kv, (uint64_t)d.batch};
    const uint64_t dv[4] = {(uint64_t)d.head_dim_v, (uint64_t)d.seqlen_k, (uint64_t)d.heads_kv, (uint64_t)d.batch};
    const uint64_t sk[3] = {(uint64_t)d.k_stride[2] * 2, (uint64_t)d.k_stride[1] * 2, (uint64_t)d.k_stride[0] * 2};
    const uint64_t sv[3] = {(uint64_t)d.v_stride[2] * 2, (uint64_t)d.v_stride[1] * 2, (uint64_t)d.v_stride[0] * 2};
    if (int st = encode_tma_4d(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, d.k, dk, sk, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return st;
    if (int st = encode_tma_4d(&tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, d.v, dv, sv, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return st;
  }
  FwdParams p;
  p.o = d.o;
  p.lse = d.lse;
  p.m = d.m;
  p.den = d.den;
  for (int i = 0; i < 3; ++i) p.o_stride[i] = d.o_stride[i];
  p.T = (int)d.seqlen_q;
  p.S = (int)d.seqlen_k;
  p.DV = (int)d.head_dim_v;
  p.H = (int)d.heads_q;
  p.HKV = (int)d.heads_kv;
  p.B = (int)d.batch;
  p.q_start = (int)d.q_start;
  p.causal = d.causal ? 1 : 0;
  p.key_lo = d.key_lo;
  p.key_hi = d.key_hi;
  p.mask_monotone = d.mask_monotone ? 1 : 0;
  p.num_mblocks = (int)((d.seqlen_q + BM - 1) / BM);
  p.scale_log2 = (float)(d.scale * 1.4426950408889634);
  p.err = device_error_flag();
  const int64_t ntile = (int64_t)p.num_mblocks * d.heads_q * d.batch;
  if (ntile > 0x7fffffffLL) return set_error(PDB_ERR_SHAPE, "bf16 flash: grid too large");
  int dev = 0;
  cudaGetDevice(&dev);
  int sms = sm_count(dev) - (d.sm_margin > 0 ? d.sm_margin : 0);
  if (sms < 1) sms = 1;
  // fewer than 4 waves of tile pairs: single tiles heaviest first (else head-major pairs)
  p.lpt = (ntile + 1) / 2 < 4 * (int64_t)sms ? 1 : 0;
  const int64_t units = p.lpt ? ntile : (ntile + 1) / 2;
  const int64_t grid = units < sms ? units : sms;
  auto kern = p.key_lo ? flash_fwd_d256_kernel<true> : flash_fwd_d256_kernel<false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem256);
  if (e != cudaSuccess) return cuda_status(e, "bf16 flash d256: set smem attribute");
  kern<<<(unsigned)grid, kThreads256, kSmem256, stream>>>(tq, tk, tv, p);
  return cuda_status(cudaGetLastError(), "bf16 flash d256 launch");
}

}  // namespace

int flash_fwd_bf16_sm100(const pdb_flash_desc& d, cudaStream_t stream) {
  // head dims up to 64 run the D = 64 kernel, up to 128 the D = 128 kernel, up to
  // 256 the single-query-tile D = 256 kernel (the
  // tensor maps zero-fill the feature columns between the true head dim and D,
  // including the part of a 64-wide box past a dim below 64); rows of q / k / v /
  // o must be 16-byte multiples (TMA), so both dims are multiples of 8
  const int64_t dmax = d.head_dim > d.head_dim_v ? d.head_dim : d.head_dim_v;
  if (d.head_dim % 8 || d.head_dim_v % 8 || dmax > 256)
    return set_error(PDB_ERR_UNSUPPORTED,
                     "bf16 flash: head dims must be multiples of 8 up to 256 (got %lld, %lld)",
                     (long long)d.head_dim, (long long)d.head_dim_v);
  if (d.seqlen_q > 0x7fffffffLL - 512 || d.seqlen_k > 0x7fffffffLL - 512 || d.q_start > 0x3fffffffLL)
    return set_error(PDB_ERR_SHAPE, "bf16 flash: sequence too long");
  if ((reinterpret_cast<uintptr_t>(d.o) & 15u) || (d.o_stride[0] & 7) || (d.o_stride[1] & 7) || (d.o_stride[2] & 7))
    return set_error(PDB_ERR_ALIGN, "bf16 flash: o must be 16-byte aligned with strides multiple of 8 elements");
  return dmax <= 64 ? launch<64>(d, stream) : dmax <= 128 ? launch<128>(d, stream) : launch256(d, stream);
}

}  // namespace pdb
