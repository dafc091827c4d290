// Calibration: the HBM read bandwidth a streaming kernel can reach on this GPU, the ceiling against which the
// bandwidth-bound kernels (decode attention above all) are measured. Not part of the reference's surface.
#include <cuda_runtime.h>

#include "common.cuh"
#include "host.hpp"

namespace tempo {
namespace {

// Grid-stride over `words` 16-byte words, eight L1-bypassing loads in flight per thread; each thread folds what it
// read into one word of `sink` so the loads stay live. Words past the last full group of eight strides are skipped.
__global__ void __launch_bounds__(256) stream_read_kernel(const uint4* __restrict__ src, uint64_t words,
                                                          uint4* __restrict__ sink) {
  const uint64_t tid = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
  uint4 acc = make_uint4(0, 0, 0, 0);
  for (uint64_t base = tid; base + 7 * stride < words; base += 8 * stride) {
    uint4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u)
      asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                   : "=r"(v[u].x), "=r"(v[u].y), "=r"(v[u].z), "=r"(v[u].w)
                   : "l"(src + base + u * stride));
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      acc.x ^= v[u].x;
      acc.y ^= v[u].y;
      acc.z ^= v[u].z;
      acc.w ^= v[u].w;
    }
  }
  sink[tid] = acc;
}

}  // namespace
}  // namespace tempo

using namespace tempo;

extern "C" tempo_status tempo_stream_read_threads(uint32_t* threads) {
  if (threads == nullptr) return fail(TEMPO_ERR_VALUE, "tempo_stream_read_threads: null output");
  *threads = uint32_t(sm_count()) * 4u * 256u;
  return TEMPO_OK;
}

extern "C" tempo_status tempo_stream_read(const void* src, uint64_t bytes, void* sink, void* stream) {
  if (src == nullptr || sink == nullptr || !aligned16(src) || !aligned16(sink) || bytes < 16)
    return fail(TEMPO_ERR_VALUE, "tempo_stream_read: 16-byte aligned source of at least 16 bytes and a sink needed");
  // Four 256-thread CTAs per SM measured fastest (eight per SM lose about 5 %).
  const uint32_t blocks = uint32_t(sm_count()) * 4u;
  stream_read_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<const uint4*>(src),
                                                                            bytes / 16, static_cast<uint4*>(sink));
  return check_launch("stream_read_kernel");
}
