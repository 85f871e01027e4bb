// f32 flash-attention forward on the CUDA cores (IEEE FMA, no tf32).
//
// The reference's device column for the flash template is f32 with an
// IEEE dot (conformance/triton_tile.py:471-522, tf32 refused at :684-690),
// and the f32 parity bar is 1e-5 relative to the f64 evaluator, which tf32
// tensor-core products (10-bit mantissa) cannot meet.  This kernel is that
// column on B200: the online-softmax fold of fusion.py:542-615 (_generate_flash)
// over 64-key tiles, one CTA per (64 query rows, batch, head), with
// K/V tiles staged once in shared memory (the template's tl.stage of K/V).
//
// The recurrence is the flashsm monoid of pdum/tl/zoo/attention.py:40-46:
//   m' = max(m, max_s sc),  den' = den*exp(m - m') + sum exp(sc - m'),
//   o'  = o*exp(m - m') + sum exp(sc - m') v
// finishing with out = o / den.  Masked scores never contribute (their exp
// underflows to exactly 0 in the reference as well, fusion.py:659-666).
#include <cfloat>

#include "common.cuh"

namespace pdb {
namespace {

constexpr int BM = 64, BN = 64, NT = 256;

template <int D>  // padded head-dim bound (64, 128 or 256)
__global__ void __launch_bounds__(NT) flash_f32_kernel(pdb_flash_desc p) {
  extern __shared__ float sm[];
  const int E = (int)p.head_dim, O = (int)p.head_dim_v;
  float* Qs = sm;                    // [BM][D+1]
  float* Ks = Qs + BM * (D + 1);     // [BN][D+1]
  float* Vs = Ks + BN * (D + 1);     // [BN][D]
  float* Ss = Vs + BN * D;           // [BM][BN+1]
  float* alpha_s = Ss + BM * (BN + 1);  // [BM]
  int* row_lo = reinterpret_cast<int*>(alpha_s + BM);  // [BM] key-interval mask bounds
  int* row_hi = row_lo + BM;                            // [BM]

  const int tid = threadIdx.x;
  const int64_t mblk = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int64_t group = p.heads_q / p.heads_kv;
  const int64_t hk = h / group;
  const float* q = static_cast<const float*>(p.q) + b * p.q_stride[0] + h * p.q_stride[1];
  const float* k = static_cast<const float*>(p.k) + b * p.k_stride[0] + hk * p.k_stride[1];
  const float* v = static_cast<const float*>(p.v) + b * p.v_stride[0] + hk * p.v_stride[1];
  float* o = static_cast<float*>(p.o) + b * p.o_stride[0] + h * p.o_stride[1];
  const int64_t T = p.seqlen_q, S = p.seqlen_k;
  const int64_t r0 = mblk * BM;
  const float scale = (float)p.scale;

  for (int i = tid; i < BM * E; i += NT) {
    const int r = i / E, c = i % E;
    Qs[r * (D + 1) + c] = (r0 + r < T) ? q[(r0 + r) * p.q_stride[2] + c] : 0.f;
  }
  // per-thread softmax row / output ownership: row = tid / 4, lane-in-row = tid % 4
  const int my_row = tid >> 2, sub = tid & 3;
  float m_run = -FLT_MAX, l_run = 0.f;
  float acc[D / 4];
#pragma unroll
  for (int j = 0; j < D / 4; ++j) acc[j] = 0.f;

  const int64_t last = r0 + BM - 1 < T - 1 ? r0 + BM - 1 : T - 1;
  int64_t s_begin = 0, s_end = S;
  if (p.causal) {
    const int64_t last_row = last + p.q_start;
    s_end = last_row + 1 < S ? last_row + 1 : S;
  }
  if (p.key_lo) {
    for (int i = tid; i < BM; i += NT) {
      const int64_t t = r0 + i < T ? r0 + i : T - 1;
      row_lo[i] = p.key_lo[t];
      row_hi[i] = p.key_hi[t];
    }
    if (p.mask_monotone) {  // this block's visible keys: [key_lo[first row], key_hi[last row])
      s_begin = (p.key_lo[r0] / BN) * BN;
      const int64_t h_ = p.key_hi[last];
      s_end = h_ < S ? h_ : S;
    }
  }
  const int ty = tid >> 4, tx = tid & 15;
  for (int64_t s0 = s_begin; s0 < s_end; s0 += BN) {
    __syncthreads();
    for (int i = tid; i < BN * E; i += NT) {
      const int r = i / E, c = i % E;
      Ks[r * (D + 1) + c] = (s0 + r < S) ? k[(s0 + r) * p.k_stride[2] + c] : 0.f;
    }
    for (int i = tid; i < BN * O; i += NT) {
      const int r = i / O, c = i % O;
      Vs[r * D + c] = (s0 + r < S) ? v[(s0 + r) * p.v_stride[2] + c] : 0.f;
    }
    __syncthreads();
    // scores: thread (ty, tx) -> rows ty*4..+3, cols tx + 16*j
    float sc[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int j = 0; j < 4; ++j) sc[a][j] = 0.f;
    for (int e = 0; e < E; ++e) {
      float qa[4], kb[4];
#pragma unroll
      for (int a = 0; a < 4; ++a) qa[a] = Qs[(ty * 4 + a) * (D + 1) + e];
#pragma unroll
      for (int j = 0; j < 4; ++j) kb[j] = Ks[(tx + 16 * j) * (D + 1) + e];
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int j = 0; j < 4; ++j) sc[a][j] = fmaf(qa[a], kb[j], sc[a][j]);
    }
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t t = r0 + ty * 4 + a, s = s0 + tx + 16 * j;
        const int rr = ty * 4 + a;
        const bool ok = s < S && (!p.causal || s <= t + p.q_start) &&
                        (!p.key_lo || (s >= row_lo[rr] && s < row_hi[rr]));
        Ss[(ty * 4 + a) * (BN + 1) + tx + 16 * j] = ok ? sc[a][j] * scale : -FLT_MAX;
      }
    __syncthreads();
    // online softmax: 4 threads per row, columns sub + 4*j
    {
      float* srow = Ss + my_row * (BN + 1);
      float mx = -FLT_MAX;
#pragma unroll
      for (int j = 0; j < BN / 4; ++j) mx = fmaxf(mx, srow[sub + 4 * j]);
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m_run, mx);
      float ps = 0.f;
#pragma unroll
      for (int j = 0; j < BN / 4; ++j) {
        const float sv = srow[sub + 4 * j];
        const float pv = sv == -FLT_MAX ? 0.f : expf(sv - m_new);
        srow[sub + 4 * j] = pv;
        ps += pv;
      }
      ps += __shfl_xor_sync(0xffffffffu, ps, 1);
      ps += __shfl_xor_sync(0xffffffffu, ps, 2);
      const float al = m_run == -FLT_MAX ? 0.f : expf(m_run - m_new);
      l_run = l_run * al + ps;
      m_run = m_new;
      if (sub == 0) alpha_s[my_row] = al;
    }
    __syncthreads();
    {
      const float al = alpha_s[my_row];
      const float* prow = Ss + my_row * (BN + 1);
#pragma unroll
      for (int j = 0; j < D / 4; ++j) acc[j] *= al;
      for (int s = 0; s < BN; ++s) {
        const float pv = prow[s];
        const float* vr = Vs + s * D;
#pragma unroll
        for (int j = 0; j < D / 4; ++j) acc[j] = fmaf(pv, vr[sub + 4 * j], acc[j]);
      }
    }
  }
  const int64_t t = r0 + my_row;
  if (t < T) {
    const float inv_l = 1.0f / l_run;
    float* orow = o + t * p.o_stride[2];
#pragma unroll
    for (int j = 0; j < D / 4; ++j) {
      const int c = sub + 4 * j;
      if (c < O) orow[c] = acc[j] * inv_l;
    }
    if (sub == 0) {
      const int64_t idx = ((int64_t)b * p.heads_q + h) * T + t;
      if (p.lse) p.lse[idx] = m_run + logf(l_run);
      if (p.m) p.m[idx] = m_run;
      if (p.den) p.den[idx] = l_run;
    }
  }
}

template <int D>
cudaError_t launch_f32(const pdb_flash_desc& p, dim3 grid, cudaStream_t stream) {
  const size_t smem = sizeof(float) * (BM * (D + 1) + BN * (D + 1) + BN * D + BM * (BN + 1) + 3 * BM);
  cudaError_t e = cudaFuncSetAttribute(flash_f32_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e == cudaSuccess) flash_f32_kernel<D><<<grid, NT, smem, stream>>>(p);
  return e;
}

}  // namespace

int flash_fwd_f32(const pdb_flash_desc& p, cudaStream_t stream) {
  if (p.head_dim > 256 || p.head_dim_v > 256)
    return set_error(PDB_ERR_UNSUPPORTED, "f32 flash: head_dim and head_dim_v must be <= 256");
  const int64_t mblocks = (p.seqlen_q + BM - 1) / BM;
  if (mblocks > 0x7fffffff || p.heads_q > 65535 || p.batch > 65535)
    return set_error(PDB_ERR_SHAPE, "f32 flash: grid too large");
  dim3 grid((unsigned)mblocks, (unsigned)p.heads_q, (unsigned)p.batch);
  const int64_t dmax = p.head_dim > p.head_dim_v ? p.head_dim : p.head_dim_v;
  const cudaError_t e = dmax <= 64 ? launch_f32<64>(p, grid, stream)
                        : dmax <= 128 ? launch_f32<128>(p, grid, stream)
                                      : launch_f32<256>(p, grid, stream);
  if (e != cudaSuccess) return cuda_status(e, "f32 flash: set smem attribute");
  return cuda_status(cudaGetLastError(), "f32 flash launch");
}

}  // namespace pdb
