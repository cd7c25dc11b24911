// Cached device facts for the launch paths. Every op call runs a launch path,
// and each driver query it would otherwise make (device attributes, the
// dynamic shared-memory attribute of a kernel, an occupancy calculation) costs
// tens of microseconds of host time, several times a kernel's own duration at
// small token counts. Values are cached per device; the dynamic shared-memory
// attribute is raised only when a launch needs more than it was set to.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

namespace attnres {

cudaError_t cached_sm_count(int* n);       // SMs of the current device
cudaError_t cached_smem_optin(int* bytes);  // opt-in shared memory per block, current device
// cudaFuncSetAttribute(fn, MaxDynamicSharedMemorySize, >= bytes) on the current device
cudaError_t ensure_dynamic_smem(const void* fn, int bytes);
// cudaOccupancyMaxActiveBlocksPerMultiprocessor, cached per (device, fn, block, smem)
cudaError_t cached_occupancy(int* per_sm, const void* fn, int block, size_t smem);

}  // namespace attnres
