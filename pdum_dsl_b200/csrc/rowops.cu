// Row-normalization (softmax) and row-statistics (two-pass layernorm) kernels.
//
// Reference rows: fusion.py:371-400 (_match_softmax) and :403-443
// (_match_rowstat), staged once by _stage_params (:339-350) and lowered by
// compile_tile with mean = sum / N (conformance/triton_tile.py:442-469).
//
// Both are HBM-streaming kernels: one CTA owns one row, the row is read from
// HBM exactly once into registers with 128-bit streaming loads, reduced with
// warp shuffles + a shared-memory tree, and written once with streaming
// stores.  Algorithmic traffic per row = 8 * cols bytes (f32 read + write).
// Rows longer than the register-resident maximum (8192) take a looped path
// that re-reads the row (three passes for softmax, three for layernorm).
#include <cfloat>

#include "common.cuh"

namespace pdb {
namespace {

#ifndef PDB_ROW_THREADS
#define PDB_ROW_THREADS 256
#endif
constexpr int kThreads = PDB_ROW_THREADS;
constexpr int kMaxVec = 8 * 256 / kThreads;  // float4 per thread: 8192 columns resident

template <typename Op>
__device__ __forceinline__ float block_reduce(float v, float* red, Op op, float ident) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();  // red[] may still be read by a previous reduction
  if (lane == 0) red[warp] = v;
  __syncthreads();
  v = lane < nw ? red[lane] : ident;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
struct MaxOp {
  __device__ float operator()(float a, float b) const { return fmaxf(a, b); }
};
struct SumOp {
  __device__ float operator()(float a, float b) const { return a + b; }
};

// ---- register-resident, 128-bit vector path (cols % 4 == 0, aligned) -------
template <int VEC>
__global__ void __launch_bounds__(kThreads) softmax_vec_kernel(const float* __restrict__ x, float* __restrict__ y,
                                                               int64_t cols, int64_t xs, int64_t ys) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const float4* xr = reinterpret_cast<const float4*>(x + row * xs);
  float4* yr = reinterpret_cast<float4*>(y + row * ys);
  const int n4 = (int)(cols >> 2);
  float4 v[VEC];
  float mx = -FLT_MAX;
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    const int c = threadIdx.x + i * kThreads;
    if (c < n4) {
      v[i] = __ldcs(xr + c);
      mx = fmaxf(mx, fmaxf(fmaxf(v[i].x, v[i].y), fmaxf(v[i].z, v[i].w)));
    }
  }
  mx = block_reduce(mx, red, MaxOp{}, -FLT_MAX);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    const int c = threadIdx.x + i * kThreads;
    if (c < n4) {
      v[i].x = expf(v[i].x - mx);
      v[i].y = expf(v[i].y - mx);
      v[i].z = expf(v[i].z - mx);
      v[i].w = expf(v[i].w - mx);
      s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    }
  }
  s = block_reduce(s, red, SumOp{}, 0.f);
  const float inv = 1.0f / s;
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    const int c = threadIdx.x + i * kThreads;
    if (c < n4) {
      float4 o = make_float4(v[i].x * inv, v[i].y * inv, v[i].z * inv, v[i].w * inv);
      __stcs(yr + c, o);
    }
  }
}

template <int VEC>
__global__ void __launch_bounds__(kThreads) layernorm_vec_kernel(const float* __restrict__ x,
                                                                 const float* __restrict__ g,
                                                                 const float* __restrict__ b, float* __restrict__ y,
                                                                 int64_t cols, int64_t xs, int64_t ys, float eps) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const float4* xr = reinterpret_cast<const float4*>(x + row * xs);
  float4* yr = reinterpret_cast<float4*>(y + row * ys);
  const int n4 = (int)(cols >> 2);
  float4 v[VEC];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    const int c = threadIdx.x + i * kThreads;
    if (c < n4) {
      v[i] = __ldcs(xr + c);
      s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    }
  }
  const float mean = block_reduce(s, red, SumOp{}, 0.f) / (float)cols;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    const int c = threadIdx.x + i * kThreads;
    if (c < n4) {
      v[i].x -= mean;
      v[i].y -= mean;
      v[i].z -= mean;
      v[i].w -= mean;
      q += (v[i].x * v[i].x + v[i].y * v[i].y) + (v[i].z * v[i].z + v[i].w * v[i].w);
    }
  }
  const float var = block_reduce(q, red, SumOp{}, 0.f) / (float)cols;
  const float inv = 1.0f / sqrtf(var + eps);
  const float4* g4 = reinterpret_cast<const float4*>(g);
  const float4* b4 = reinterpret_cast<const float4*>(b);
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    const int c = threadIdx.x + i * kThreads;
    if (c < n4) {
      float4 gg = g ? __ldg(g4 + c) : make_float4(1.f, 1.f, 1.f, 1.f);
      float4 bb = b ? __ldg(b4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      float4 o = make_float4(v[i].x * inv * gg.x + bb.x, v[i].y * inv * gg.y + bb.y, v[i].z * inv * gg.z + bb.z,
                             v[i].w * inv * gg.w + bb.w);
      __stcs(yr + c, o);
    }
  }
}

// ---- generic looped path: any cols, any alignment --------------------------
__global__ void __launch_bounds__(kThreads) softmax_loop_kernel(const float* __restrict__ x, float* __restrict__ y,
                                                                int64_t cols, int64_t xs, int64_t ys) {
  __shared__ float red[32];
  const float* xr = x + (int64_t)blockIdx.x * xs;
  float* yr = y + (int64_t)blockIdx.x * ys;
  float mx = -FLT_MAX;
  for (int64_t c = threadIdx.x; c < cols; c += kThreads) mx = fmaxf(mx, xr[c]);
  mx = block_reduce(mx, red, MaxOp{}, -FLT_MAX);
  float s = 0.f;
  for (int64_t c = threadIdx.x; c < cols; c += kThreads) s += expf(xr[c] - mx);
  s = block_reduce(s, red, SumOp{}, 0.f);
  const float inv = 1.0f / s;
  for (int64_t c = threadIdx.x; c < cols; c += kThreads) yr[c] = expf(xr[c] - mx) * inv;
}

__global__ void __launch_bounds__(kThreads) layernorm_loop_kernel(const float* __restrict__ x,
                                                                  const float* __restrict__ g,
                                                                  const float* __restrict__ b, float* __restrict__ y,
                                                                  int64_t cols, int64_t xs, int64_t ys, float eps) {
  __shared__ float red[32];
  const float* xr = x + (int64_t)blockIdx.x * xs;
  float* yr = y + (int64_t)blockIdx.x * ys;
  float s = 0.f;
  for (int64_t c = threadIdx.x; c < cols; c += kThreads) s += xr[c];
  const float mean = block_reduce(s, red, SumOp{}, 0.f) / (float)cols;
  float q = 0.f;
  for (int64_t c = threadIdx.x; c < cols; c += kThreads) {
    const float d = xr[c] - mean;
    q += d * d;
  }
  const float sd = sqrtf(block_reduce(q, red, SumOp{}, 0.f) / (float)cols + eps);
  for (int64_t c = threadIdx.x; c < cols; c += kThreads) {
    const float gg = g ? g[c] : 1.f, bb = b ? b[c] : 0.f;
    yr[c] = (xr[c] - mean) / sd * gg + bb;
  }
}

bool vec_ok(const void* p, int64_t stride) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0 && (stride & 3) == 0;
}

int check_rows(int64_t rows, int64_t cols, int64_t xs, int64_t ys) {
  if (rows < 0 || cols < 0) return set_error(PDB_ERR_SHAPE, "negative size");
  if (rows > 0x7fffffffLL) return set_error(PDB_ERR_SHAPE, "rows > 2^31-1");
  if (xs < cols || ys < cols) return set_error(PDB_ERR_SHAPE, "row stride smaller than cols");
  return PDB_OK;
}

}  // namespace
}  // namespace pdb

using namespace pdb;

extern "C" int pdb_rowsoftmax_f32(const pdb_rowsoftmax_desc* d, void* stream) {
  if (!d) return set_error(PDB_ERR_ARG, "null descriptor");
  if (int st = check_rows(d->rows, d->cols, d->x_row_stride, d->y_row_stride)) return st;
  if (d->rows == 0 || d->cols == 0) return PDB_OK;
  if (!d->x || !d->y) return set_error(PDB_ERR_ARG, "null x / y");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)d->rows), block(kThreads);
  const bool vec = (d->cols & 3) == 0 && vec_ok(d->x, d->x_row_stride) && vec_ok(d->y, d->y_row_stride);
  const int64_t v4 = (d->cols / 4 + kThreads - 1) / kThreads;
  if (vec && v4 <= kMaxVec) {
#define PDB_SM(V) softmax_vec_kernel<V><<<grid, block, 0, s>>>(d->x, d->y, d->cols, d->x_row_stride, d->y_row_stride)
    if (v4 <= 1) PDB_SM(1);
    else if (v4 <= 2) PDB_SM(2);
    else if (v4 <= 4) PDB_SM(4);
    else if (v4 <= 8) PDB_SM(8);
    else PDB_SM(16);
#undef PDB_SM
  } else {
    softmax_loop_kernel<<<grid, block, 0, s>>>(d->x, d->y, d->cols, d->x_row_stride, d->y_row_stride);
  }
  return cuda_status(cudaGetLastError(), "rowsoftmax launch");
}

extern "C" int pdb_layernorm_f32(const pdb_layernorm_desc* d, void* stream) {
  if (!d) return set_error(PDB_ERR_ARG, "null descriptor");
  if (int st = check_rows(d->rows, d->cols, d->x_row_stride, d->y_row_stride)) return st;
  if (d->rows == 0 || d->cols == 0) return PDB_OK;
  if (!d->x || !d->y) return set_error(PDB_ERR_ARG, "null x / y");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)d->rows), block(kThreads);
  const float eps = (float)d->eps;
  const bool gb_ok = (!d->gamma || vec_ok(d->gamma, 0)) && (!d->beta || vec_ok(d->beta, 0));
  const bool vec = (d->cols & 3) == 0 && gb_ok && vec_ok(d->x, d->x_row_stride) && vec_ok(d->y, d->y_row_stride);
  const int64_t v4 = (d->cols / 4 + kThreads - 1) / kThreads;
#define PDB_LN(V)                                                                                         \
  layernorm_vec_kernel<V><<<grid, block, 0, s>>>(d->x, d->gamma, d->beta, d->y, d->cols, d->x_row_stride, \
                                                 d->y_row_stride, eps)
  if (vec && v4 <= kMaxVec) {
    if (v4 <= 1) PDB_LN(1);
    else if (v4 <= 2) PDB_LN(2);
    else if (v4 <= 4) PDB_LN(4);
    else if (v4 <= 8) PDB_LN(8);
    else PDB_LN(16);
  } else {
    layernorm_loop_kernel<<<grid, block, 0, s>>>(d->x, d->gamma, d->beta, d->y, d->cols, d->x_row_stride,
                                                 d->y_row_stride, eps);
  }
#undef PDB_LN
  return cuda_status(cudaGetLastError(), "layernorm launch");
}
