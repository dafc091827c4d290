// Host-side plumbing shared by the library's translation units: status codes, the last-error message, tensor-map
// encoding through the driver entry point, and launch checking.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>

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

// Opts a kernel into more than 48 KB of dynamic shared memory, once per process.
tempo_status set_smem(const void* kernel, int bytes);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace tempo
