// Host-side plumbing shared by the library's translation units: status codes, the last-error message, tensor-map
// encoding through the driver entry point, and launch checking.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>
#include <utility>

#include "../../include/tempo_b200.h"

namespace tempo {

// Records `message` as the last error and returns `status`.
tempo_status fail(tempo_status status, const char* format, ...) __attribute__((format(printf, 2, 3)));

// Maps a CUDA runtime error to TEMPO_ERR_RUNTIME with a message naming `what`.
tempo_status cuda_fail(cudaError_t err, const char* what);

// Checks the most recent kernel launch; returns TEMPO_OK or a runtime error naming `kernel`.
tempo_status check_launch(const char* kernel);

// Encodes a tiled tensor map (cuTensorMapEncodeTiled, fetched through cudaGetDriverEntryPoint so the library does
// not link libcuda). dims/strides are innermost first; strides has rank-1 entries, in bytes.
tempo_status encode_tmap(CUtensorMap* map, CUtensorMapDataType type, uint32_t rank, const void* base,
                         const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                         CUtensorMapSwizzle swizzle);

// The number of SMs of the current device (cached).
int sm_count();

// Opts a kernel into more than 48 KB of dynamic shared memory, once per device.
tempo_status set_smem(const void* kernel, int bytes);

// The failure-detection probe (gemm.cu): one CTA waits on an mbarrier that completes only if `arrive` is non-zero,
// giving up after `limit_ns` with the watchdog code the runtime reports.
tempo_status launch_wait_probe(uint32_t arrive, uint64_t limit_ns, cudaStream_t stream);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Whether a grid of `ctas` fits on the GPU at once with `per_sm` resident per SM. A kernel whose grid does lets its
// dependents launch at entry (their prologue overlaps the whole kernel); one that needs several waves triggers them
// only after its own work, so their CTAs do not take SM resources its later waves still need.
inline uint32_t single_wave(uint64_t ctas, uint32_t per_sm) { return ctas <= uint64_t(sm_count()) * per_sm ? 1u : 0u; }

// Launches `kernel` with programmatic stream serialization (it may overlap the tail of the previous kernel in the
// stream; the kernel itself waits with griddepcontrol.wait before reading anything that kernel wrote) and, when
// cluster_x > 1, as clusters of cluster_x CTAs along x.
template <typename... KernelArgs, typename... Args>
tempo_status launch(void (*kernel)(KernelArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                    unsigned cluster_x, const char* name, Args&&... args) {
  cudaLaunchConfig_t config = {};
  config.gridDim = grid;
  config.blockDim = block;
  config.dynamicSmemBytes = smem;
  config.stream = stream;
  cudaLaunchAttribute attributes[2];
  unsigned count = 0;
  attributes[count].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attributes[count].val.programmaticStreamSerializationAllowed = 1;
  ++count;
  if (cluster_x > 1) {
    attributes[count].id = cudaLaunchAttributeClusterDimension;
    attributes[count].val.clusterDim.x = cluster_x;
    attributes[count].val.clusterDim.y = 1;
    attributes[count].val.clusterDim.z = 1;
    ++count;
  }
  config.attrs = attributes;
  config.numAttrs = count;
  const cudaError_t err = cudaLaunchKernelEx(&config, kernel, std::forward<Args>(args)...);
  if (err != cudaSuccess) return cuda_fail(err, name);
  return check_launch(name);
}

}  // namespace tempo
