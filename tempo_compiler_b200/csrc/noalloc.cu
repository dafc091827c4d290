// An allocation-free variant of the LM head's greedy pick (tempo_gemm in argmax mode + tempo_argmax_finish).
//
// Some callers may not allocate device memory at all: an inference server's plugin or custom-op hook that hands the
// op its input and output buffers and accounts for every device byte itself, so an allocation inside the op would
// slip past its memory budget; or a host loop with a hard latency bound, where cudaMalloc/cudaFree (and the device
// synchronisation cudaFree implies) cannot be afforded. The allocating path needs a caller-provided partials buffer
// between its two kernels; this variant keeps those partials in one fixed array compiled into the library instead.
//
// The array is a file-scope static __device__ array: every GPU that loads the library holds its 2 MiB until the
// process exits. Its device address is fetched once per device with cudaGetSymbolAddress, with that device current,
// on the first call made on the device (so that first call should come before any stream capture). All calls share
// the array and it keeps the last call's contents; nothing in it needs to start at zero, because the GEMM epilogue
// writes every partial the reduction later reads. Two calls whose work overlaps on the GPU (on different streams, or
// on different host threads without ordering) race on the array and corrupt each other's result.
#include <cuda_runtime.h>

#include <mutex>

#include "host.hpp"

namespace {

constexpr uint32_t kMaxRows = 1024;     // token rows per call
constexpr uint32_t kTileColumns = 256;  // columns one argmax partial covers (the GEMM's 256-wide tile)
constexpr uint32_t kMaxTiles = 256;     // so the vocabulary may be up to 65536 entries
constexpr size_t kValuesBytes = size_t(kMaxRows) * kMaxTiles * sizeof(float);
constexpr size_t kScratchBytes = kValuesBytes + size_t(kMaxRows) * kMaxTiles * sizeof(int32_t);  // 2 MiB

static __device__ __align__(256) unsigned char g_argmax_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
void* g_scratch_address[kMaxDevices] = {};

// The scratch array's device address on the current device; looked up on the device's first call.
tempo_status scratch_address(void** out) {
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return tempo::cuda_fail(err, "tempo_lm_head_argmax_noalloc: cudaGetDevice");
  if (device < 0 || device >= kMaxDevices)
    return tempo::fail(TEMPO_ERR_STATE, "tempo_lm_head_argmax_noalloc: device %d is beyond the %d this library tracks",
                       device, kMaxDevices);
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_address[device] == nullptr) {
    void* address = nullptr;
    err = cudaGetSymbolAddress(&address, g_argmax_scratch);
    if (err != cudaSuccess)
      return tempo::cuda_fail(err, "tempo_lm_head_argmax_noalloc: cudaGetSymbolAddress of the scratch array");
    g_scratch_address[device] = address;
  }
  *out = g_scratch_address[device];
  return TEMPO_OK;
}

}  // namespace

extern "C" tempo_status tempo_lm_head_argmax_noalloc(const void* hidden, uint32_t ld_hidden, const void* embedding,
                                                     uint32_t ld_embedding, uint32_t rows, uint32_t vocab,
                                                     uint32_t width, int32_t* ids, void* stream) {
  if (rows == 0 || rows > kMaxRows)
    return tempo::fail(TEMPO_ERR_VALUE,
                       "tempo_lm_head_argmax_noalloc: %u rows; this allocation-free entry point takes 1 to %u rows per "
                       "call (its scratch array is sized for that), so split the batch or use tempo_gemm with "
                       "caller-allocated partials", rows, kMaxRows);
  const uint32_t tiles = (vocab + kTileColumns - 1) / kTileColumns;
  if (vocab == 0 || tiles > kMaxTiles)
    return tempo::fail(TEMPO_ERR_VALUE,
                       "tempo_lm_head_argmax_noalloc: a vocabulary of %u; this entry point covers 1 to %u entries",
                       vocab, kMaxTiles * kTileColumns);
  if (ids == nullptr) return tempo::fail(TEMPO_ERR_VALUE, "tempo_lm_head_argmax_noalloc: ids must not be NULL");
  void* scratch = nullptr;
  tempo_status status = scratch_address(&scratch);
  if (status != TEMPO_OK) return status;
  // Partials laid out [rows][tiles], values then indices, as the allocating path's caller would allocate them.
  float* values = static_cast<float*>(scratch);
  int32_t* indices = reinterpret_cast<int32_t*>(static_cast<unsigned char*>(scratch) + kValuesBytes);
  status = tempo_gemm(hidden, ld_hidden, embedding, ld_embedding, nullptr, nullptr, vocab, nullptr, vocab, rows, vocab,
                      width, TEMPO_GEMM_ARGMAX, values, indices, stream);
  if (status != TEMPO_OK) return status;
  return tempo_argmax_finish(values, indices, rows, tiles, ids, nullptr, 0, nullptr, 0, 0, stream);
}
