// Flash-attention backward (placeholder until the kernels land).
#include "common.cuh"

using namespace pdb;

extern "C" size_t pdb_flash_bwd_workspace_size(const pdb_flash_bwd_desc* d) { return d ? 0 : 0; }

extern "C" int pdb_flash_bwd(const pdb_flash_bwd_desc* d, void* stream) {
  (void)d;
  (void)stream;
  return set_error(PDB_ERR_UNSUPPORTED, "flash backward not built yet");
}
