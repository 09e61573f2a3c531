// Host-side helpers shared by the entry points of libkta_b200 (runtime.cu implements them).
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "kta_b200.h"

namespace kta {

// Device status block of the current device (4 words, see kta_device_status), or nullptr
// when it cannot be resolved. Resolved once per device with that device current.
unsigned int* device_status_ptr();

// SM count of the current device (cached per device); 0 on error.
int current_sm_count();

// Compute capability major of the current device; -1 on error.
int current_cc_major();

// Encodes a tiled tensor map (rank 2 or 3) through the driver's cuTensorMapEncodeTiled,
// resolved with cudaGetDriverEntryPoint (the library does not link libcuda).
// dims/strides are innermost-first; strides_bytes holds rank-1 entries (dims 1..rank-1).
int encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                CUtensorMapSwizzle swizzle);

// Maps the pending CUDA error of the last launch to a status code.
int launch_status();

// True if `p` is 16-byte aligned.
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Common device precondition of every entry: a device of compute capability 10.x.
int require_sm100();

// Raises the dynamic shared-memory limit of `kernel` to `bytes` on the current device
// (once per kernel and device: pass the largest size any launch of `kernel` will use).
int set_kernel_smem(const void* kernel, int bytes);

// Status of the last kta_so_* call on this host thread (kta_last_error).
void set_last_error(int s);

// Operand bytes above which a kernel prefetches its first ring of tiles into L2 before
// griddepcontrol.wait: such operands cannot already sit in the 126 MB L2, so the prefetch
// overlaps the first HBM round trip with the previous grid's tail. Below it the operands may
// be L2-resident, and the prefetches only occupy the L2 while the real loads queue behind
// them (an f16 1024^3 GEMM ran 30 % slower with them).
constexpr int64_t kPrefetchMinBytes = int64_t{64} << 20;

// Launches `kernel` with programmatic stream serialisation: the next kernel in the stream (or
// graph) may be scheduled and run its set-up while this one finishes; its griddepcontrol.wait
// holds every memory access until this grid has completed and its writes are visible.
// cluster_x > 1 launches clusters of that many CTAs.
template <typename... KArgs, typename... Args>
int launch_ex(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
              unsigned cluster_x, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[n].val.programmaticStreamSerializationAllowed = 1;
  ++n;
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  if (cudaLaunchKernelEx(&cfg, kernel, args...) != cudaSuccess) {
    (void)cudaGetLastError();
    return KTA_ERR_LAUNCH;
  }
  return launch_status();
}

}  // namespace kta
