// Status plumbing of the C ABI: thread-local error text, the per-device
// error word that bounded device waits report into, the device attribute
// cache and the TMA tensor-map encoder (driver entry point, looked up once).
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "tma.h"

namespace pdb {

static thread_local char g_err_text[512] = "ok";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err_text, sizeof(g_err_text), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return PDB_OK;
  return set_error(PDB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// One error word per device, in device global memory.  Bounded waits OR
// kErrTimeout into it; pdb_check_error reads and clears it.
__device__ int g_device_error;

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mu;
int g_sm_count[kMaxDevices];
int* g_err_ptr[kMaxDevices];
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
}  // namespace

int sm_count(int device) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (device < 0 || device >= kMaxDevices) return 148;
  if (g_sm_count[device] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0) n = 148;
    g_sm_count[device] = n;
  }
  return g_sm_count[device];
}

int* device_error_flag() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_err_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    g_err_ptr[dev] = static_cast<int*>(p);
  }
  return g_err_ptr[dev];
}

int encode_tma_4d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, const uint64_t dims[4],
                  const uint64_t strides_bytes[3], const uint32_t box[4], CUtensorMapSwizzle swizzle) {
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_encode == nullptr) {
      cudaDriverEntryPointQueryResult q;
      void* fn = nullptr;
      cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q);
      if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr)
        return set_error(PDB_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  }
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    return set_error(PDB_ERR_ALIGN, "TMA base address must be 16-byte aligned");
  for (int i = 0; i < 3; ++i)
    if (strides_bytes[i] % 16 != 0) return set_error(PDB_ERR_ALIGN, "TMA strides must be multiples of 16 bytes");
  cuuint64_t gdim[4] = {dims[0], dims[1], dims[2], dims[3]};
  cuuint64_t gstr[3] = {strides_bytes[0], strides_bytes[1], strides_bytes[2]};
  cuuint32_t bdim[4] = {box[0], box[1], box[2], box[3]};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = g_encode(map, dtype, 4, const_cast<void*>(base), gdim, gstr, bdim, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(PDB_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
  return PDB_OK;
}

}  // namespace pdb

extern "C" int pdb_check_error(void* stream) {
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return pdb::cuda_status(e, "stream synchronize");
  int* flag = pdb::device_error_flag();
  if (flag == nullptr) return pdb::set_error(PDB_ERR_CUDA, "device error flag unavailable");
  int h = 0;
  e = cudaMemcpy(&h, flag, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return pdb::cuda_status(e, "read device error flag");
  if (h != 0) {
    int z = 0;
    cudaMemcpy(flag, &z, sizeof(int), cudaMemcpyHostToDevice);
    if ((h & pdb::kErrTimeout) == 0)
      return pdb::set_error(PDB_ERR_CUDA, "a kernel refused its shared-memory window (flag 0x%x)", h);
    return pdb::set_error(PDB_ERR_TIMEOUT, "a bounded device wait expired (flag 0x%x)", h);
  }
  return PDB_OK;
}

extern "C" const char* pdb_last_error_string(void) { return pdb::g_err_text; }

extern "C" const char* pdb_version(void) { return "pdb-sm100a-0.1.0"; }

// ---------------------------------------------------------------------------
// Self-test of the bounded-wait failure path: one thread waits on an mbarrier
// phase that nothing will complete, gives up after `limit_ns` and reports
// through the device error word, exactly as a stuck pipeline stage would.
namespace pdb {
namespace {
__global__ void selftest_wait_kernel(unsigned long long limit_ns, int* err) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(&bar, 0, &abort_flag, err, limit_ns);  // never arrives
  __syncthreads();
}
}  // namespace
}  // namespace pdb

extern "C" int pdb_selftest_wait_timeout(int64_t limit_ns, void* stream) {
  if (limit_ns <= 0 || limit_ns > 2000000000LL) return pdb::set_error(PDB_ERR_ARG, "limit_ns must be in (0, 2e9]");
  int* flag = pdb::device_error_flag();
  if (!flag) return pdb::set_error(PDB_ERR_CUDA, "device error flag unavailable");
  pdb::selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>((unsigned long long)limit_ns, flag);
  return pdb::cuda_status(cudaGetLastError(), "selftest launch");
}
