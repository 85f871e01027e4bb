// pdb_flash_fwd / pdb_flash_bwd: descriptor validation and dispatch to the
// dtype-specific kernels (bf16 -> tcgen05 path, f32 -> IEEE CUDA-core path).
#include "common.cuh"

namespace pdb {
int flash_fwd_f32(const pdb_flash_desc& p, cudaStream_t stream);
int flash_fwd_bf16_sm100(const pdb_flash_desc& p, cudaStream_t stream);

int validate_common(int64_t batch, int64_t hq, int64_t hkv, int64_t T, int64_t S, int64_t E, int64_t O,
                    int64_t q_start, const void* q, const void* k, const void* v) {
  if (!q || !k || !v) return set_error(PDB_ERR_ARG, "null q / k / v");
  if (batch <= 0 || hq <= 0 || hkv <= 0 || T <= 0 || S <= 0 || E <= 0 || O <= 0)
    return set_error(PDB_ERR_SHAPE, "all sizes must be positive (batch %lld heads %lld/%lld T %lld S %lld E %lld O %lld)",
                     (long long)batch, (long long)hq, (long long)hkv, (long long)T, (long long)S, (long long)E,
                     (long long)O);
  if (hq % hkv != 0) return set_error(PDB_ERR_SHAPE, "heads_q (%lld) must be a multiple of heads_kv (%lld)",
                                      (long long)hq, (long long)hkv);
  if (q_start < 0) return set_error(PDB_ERR_SHAPE, "q_start must be >= 0");
  if (batch * hq > 0x7fffffffLL) return set_error(PDB_ERR_SHAPE, "batch * heads too large");
  return PDB_OK;
}
}  // namespace pdb

using namespace pdb;

extern "C" int pdb_flash_fwd(const pdb_flash_desc* d, void* stream) {
  if (!d) return set_error(PDB_ERR_ARG, "null descriptor");
  if (int st = validate_common(d->batch, d->heads_q, d->heads_kv, d->seqlen_q, d->seqlen_k, d->head_dim,
                               d->head_dim_v, d->q_start, d->q, d->k, d->v))
    return st;
  if (!d->o) return set_error(PDB_ERR_ARG, "null o");
  if ((d->key_lo == nullptr) != (d->key_hi == nullptr))
    return set_error(PDB_ERR_ARG, "key_lo and key_hi are given together");
  if (d->key_lo && d->causal) return set_error(PDB_ERR_ARG, "a key-interval mask replaces the causal flag");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (d->dtype) {
    case PDB_F32: return flash_fwd_f32(*d, s);
    case PDB_BF16: return flash_fwd_bf16_sm100(*d, s);
    default: return set_error(PDB_ERR_UNSUPPORTED, "unknown dtype %d", d->dtype);
  }
}
