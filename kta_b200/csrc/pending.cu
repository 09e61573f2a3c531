// Entries declared in kta_b200.h whose kernels are not in this build yet: they reject every
// call with KTA_ERR_UNSUPPORTED (never a CPU fallback).
#include "kta_host.h"

extern "C" {

int kta_gemm_fp8_blockscaled(const void*, const void*, const void*, const void*, void*, int64_t,
                             int64_t, int64_t, void*) {
  return KTA_ERR_UNSUPPORTED;
}

}  // extern "C"
