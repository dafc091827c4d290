// The drop-in device runtime: one arena of device memory addressed by 32-bit kernel addresses, a first-fit
// allocator, synchronous copies, and the launch of staged image descriptors onto the packed tile-op kernels.
//
// It replaces the reference's board runtime (board_package/runtime): minitpuMalloc/minitpuFree
// (runtime/device.py:148-196), minitpuMemcpy (runtime/memcpy.py:93-161) and minitpuLaunchKernel
// (runtime/launch.py:44-141), keeping their argument checks and error classes. Unlike the NPU, every operand range a
// launch touches is checked against the arena before the kernel runs, so a bad pointer is a ValueError rather than a
// stray access.
#include <cuda.h>
#include <cuda_runtime.h>

#include <chrono>
#include <cstring>
#include <map>
#include <mutex>
#include <set>
#include <string>
#include <thread>
#include <unordered_map>
#include <utility>

#include "host.hpp"

namespace tempo {

int watchdog_gemm();
int watchdog_attention();
int watchdog_prefill();
int watchdog_decode_step();

// ---------------------------------------------------------------------------------------------------------------
// Errors and shared host helpers
// ---------------------------------------------------------------------------------------------------------------

namespace {
std::mutex g_error_mutex;
std::string g_last_error;
}  // namespace

tempo_status fail(tempo_status status, const char* format, ...) {
  char buffer[1024];
  va_list args;
  va_start(args, format);
  vsnprintf(buffer, sizeof(buffer), format, args);
  va_end(args);
  std::lock_guard<std::mutex> lock(g_error_mutex);
  g_last_error = buffer;
  return status;
}

tempo_status cuda_fail(cudaError_t err, const char* what) {
  return fail(TEMPO_ERR_RUNTIME, "%s: %s (%s)", what, cudaGetErrorName(err), cudaGetErrorString(err));
}

tempo_status check_launch(const char* kernel) {
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return cuda_fail(err, kernel);
  return TEMPO_OK;
}

namespace {
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;
std::once_flag g_encode_once;
}  // namespace

tempo_status encode_tmap(CUtensorMap* map, CUtensorMapDataType type, uint32_t rank, const void* base,
                         const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                         CUtensorMapSwizzle swizzle) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  });
  if (g_encode == nullptr) return fail(TEMPO_ERR_RUNTIME, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], e[5];
  for (uint32_t i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i + 1 < rank) s[i] = strides_bytes[i];
  }
  const CUresult r = g_encode(map, type, rank, const_cast<void*>(base), d, s, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(TEMPO_ERR_VALUE, "cuTensorMapEncodeTiled rejected a tensor map (CUresult %d)", int(r));
  return TEMPO_OK;
}

int sm_count() {
  static int count = [] {
    int device = 0, n = 148;
    if (cudaGetDevice(&device) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
    return n;
  }();
  return count;
}

// A function attribute belongs to the device's context, so it is set once per (device, kernel).
tempo_status set_smem(const void* kernel, int bytes) {
  static std::mutex mu;
  static std::set<std::pair<int, const void*>> done;
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return cuda_fail(err, "cudaGetDevice");
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({device, kernel})) return TEMPO_OK;
  err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (err != cudaSuccess) return cuda_fail(err, "cudaFuncSetAttribute(max dynamic shared memory)");
  done.insert({device, kernel});
  return TEMPO_OK;
}

// ---------------------------------------------------------------------------------------------------------------
// Arena
// ---------------------------------------------------------------------------------------------------------------

namespace {

constexpr uint64_t kKernelBase = 0x80000000ull;
constexpr uint64_t kReserved = 0x00100000ull;  // image staging prefix (runtime/address_space.py:26)
constexpr uint64_t kAlign = 32;                // CDMA_ALIGN (runtime/memcpy.py:27)
constexpr uint64_t kMaxArena = 0x80000000ull;  // the kernel aperture must end within 32-bit addresses
constexpr uint64_t kMaxImage = 65536;          // IRAM capacity (runtime/launch.py:16-33)

struct Arena {
  std::mutex mu;
  int device = -1;
  uint8_t* base = nullptr;
  uint64_t size = 0;
  cudaStream_t stream = nullptr;
  std::map<uint64_t, uint64_t> free_spans;        // offset -> bytes, sorted, coalesced
  std::unordered_map<uint64_t, uint64_t> allocs;  // offset -> bytes
  std::map<uint64_t, tempo_image> images;         // staged descriptors read back, by offset
  std::set<void*> host_buffers;
  uint64_t launches = 0;
  uint64_t used = 0;
};

Arena g_arena;

uint64_t round_up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

// Translates a kernel address range to a device pointer, or returns null if it is not inside the arena.
uint8_t* translate(uint64_t address, uint64_t nbytes) {
  if (address < kKernelBase) return nullptr;
  const uint64_t offset = address - kKernelBase;
  if (offset > g_arena.size || nbytes > g_arena.size - offset) return nullptr;
  return g_arena.base + offset;
}

void forget_images(uint64_t offset, uint64_t nbytes) {
  for (auto it = g_arena.images.begin(); it != g_arena.images.end();) {
    if (it->first < offset + nbytes && offset < it->first + TEMPO_IMAGE_BYTES) it = g_arena.images.erase(it);
    else ++it;
  }
}

// Reads and clears every translation unit's watchdog; the first non-zero code, 0, or -1 if one could not be read.
int read_watchdogs(int* gemm, int* decode, int* prefill) {
  *gemm = watchdog_gemm();
  *decode = watchdog_attention();
  *prefill = watchdog_prefill();
  const int step = watchdog_decode_step();
  if (*gemm < 0 || *decode < 0 || *prefill < 0 || step < 0) return -1;
  if (*decode == 0) *decode = step;
  return *gemm != 0 ? *gemm : (*decode != 0 ? *decode : *prefill);
}

tempo_status watchdog_status() {
  int a, b, c;
  const int code = read_watchdogs(&a, &b, &c);
  if (code < 0) return fail(TEMPO_ERR_RUNTIME, "could not read the device watchdog");
  if (code != 0)
    return fail(TEMPO_ERR_TIMEOUT, "a kernel gave up a bounded wait (watchdog codes gemm=%d decode=%d prefill=%d); "
                                   "its results are not valid", a, b, c);
  return TEMPO_OK;
}

tempo_status sync_stream(cudaStream_t stream, double timeout_s) {
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::duration<double>(timeout_s);
  for (;;) {
    const cudaError_t err = cudaStreamQuery(stream);
    if (err == cudaSuccess) break;
    if (err != cudaErrorNotReady) return cuda_fail(err, "device work failed");
    if (std::chrono::steady_clock::now() > deadline)
      return fail(TEMPO_ERR_TIMEOUT, "the device did not finish within %.3f s", timeout_s);
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
  return watchdog_status();
}

}  // namespace
}  // namespace tempo

using namespace tempo;

extern "C" tempo_status tempo_open(int device, uint64_t arena_bytes) {
  std::lock_guard<std::mutex> lock(g_arena.mu);
  if (g_arena.base != nullptr) {
    if (device == g_arena.device) return TEMPO_OK;
    return fail(TEMPO_ERR_STATE, "tempo_open: device %d already open; close it before opening device %d",
                g_arena.device, device);
  }
  if (arena_bytes <= kReserved || arena_bytes > kMaxArena)
    return fail(TEMPO_ERR_VALUE, "tempo_open: the arena must be larger than the %llu-byte reserved prefix and at most "
                                 "2 GiB, got %llu bytes", (unsigned long long)kReserved,
                (unsigned long long)arena_bytes);
  int count = 0;
  cudaError_t err = cudaGetDeviceCount(&count);
  if (err != cudaSuccess || count == 0) return fail(TEMPO_ERR_STATE, "tempo_open: no CUDA device is visible");
  if (device < 0 || device >= count) return fail(TEMPO_ERR_VALUE, "tempo_open: device %d of %d", device, count);
  if ((err = cudaSetDevice(device)) != cudaSuccess) return cuda_fail(err, "cudaSetDevice");
  arena_bytes = round_up(arena_bytes, kAlign);
  void* base = nullptr;
  if ((err = cudaMalloc(&base, arena_bytes)) != cudaSuccess) return cuda_fail(err, "cudaMalloc(arena)");
  if ((err = cudaStreamCreateWithFlags(&g_arena.stream, cudaStreamNonBlocking)) != cudaSuccess) {
    cudaFree(base);
    return cuda_fail(err, "cudaStreamCreate");
  }
  g_arena.device = device;
  g_arena.base = static_cast<uint8_t*>(base);
  g_arena.size = arena_bytes;
  g_arena.free_spans.clear();
  g_arena.free_spans[kReserved] = arena_bytes - kReserved;
  g_arena.allocs.clear();
  g_arena.images.clear();
  g_arena.launches = 0;
  g_arena.used = 0;
  return TEMPO_OK;
}

extern "C" tempo_status tempo_close(void) {
  std::lock_guard<std::mutex> lock(g_arena.mu);
  if (g_arena.base == nullptr) return TEMPO_OK;
  cudaStreamSynchronize(g_arena.stream);
  cudaStreamDestroy(g_arena.stream);
  cudaFree(g_arena.base);
  for (void* p : g_arena.host_buffers) cudaFreeHost(p);
  g_arena.host_buffers.clear();
  g_arena.base = nullptr;
  g_arena.stream = nullptr;
  g_arena.device = -1;
  g_arena.size = 0;
  return TEMPO_OK;
}

extern "C" tempo_status tempo_address_space(uint32_t* kernel_base, uint64_t* kernel_size, uint32_t* reserved) {
  std::lock_guard<std::mutex> lock(g_arena.mu);
  if (g_arena.base == nullptr) return fail(TEMPO_ERR_STATE, "tempo_address_space: no device is open");
  *kernel_base = uint32_t(kKernelBase);
  *kernel_size = g_arena.size;
  *reserved = uint32_t(kReserved);
  return TEMPO_OK;
}

extern "C" tempo_status tempo_malloc(uint32_t* address, uint64_t nbytes) {
  std::lock_guard<std::mutex> lock(g_arena.mu);
  if (g_arena.base == nullptr) return fail(TEMPO_ERR_STATE, "tempo_malloc: no device is open");
  if (nbytes == 0)
    return fail(TEMPO_ERR_VALUE, "Unable to allocate device memory. The requested size must be positive, but got 0.");
  const uint64_t want = round_up(nbytes, kAlign);
  uint64_t largest = 0;
  for (auto it = g_arena.free_spans.begin(); it != g_arena.free_spans.end(); ++it) {
    if (it->second >= want) {
      const uint64_t offset = it->first, span = it->second;
      g_arena.free_spans.erase(it);
      if (span > want) g_arena.free_spans[offset + want] = span - want;
      g_arena.allocs[offset] = want;
      g_arena.used += want;
      *address = uint32_t(kKernelBase + offset);
      return TEMPO_OK;
    }
    largest = largest > it->second ? largest : it->second;
  }
  return fail(TEMPO_ERR_MEMORY,
              "Unable to allocate device memory. The arena needs %llu free contiguous bytes, but the largest free span "
              "is %llu bytes.", (unsigned long long)want, (unsigned long long)largest);
}

extern "C" tempo_status tempo_free(uint32_t address) {
  std::lock_guard<std::mutex> lock(g_arena.mu);
  if (g_arena.base == nullptr) return fail(TEMPO_ERR_STATE, "tempo_free: no device is open");
  const uint64_t offset = uint64_t(address) - kKernelBase;
  auto it = address >= kKernelBase ? g_arena.allocs.find(offset) : g_arena.allocs.end();
  if (it == g_arena.allocs.end())
    return fail(TEMPO_ERR_KEY, "Unable to free device memory. The pointer 0x%x was not returned by minitpuMalloc.",
                address);
  const uint64_t bytes = it->second;
  g_arena.allocs.erase(it);
  g_arena.used -= bytes;
  forget_images(offset, bytes);
  auto next = g_arena.free_spans.emplace(offset, bytes).first;
  if (next != g_arena.free_spans.begin()) {
    auto prev = std::prev(next);
    if (prev->first + prev->second == next->first) {
      prev->second += next->second;
      g_arena.free_spans.erase(next);
      next = prev;
    }
  }
  auto after = std::next(next);
  if (after != g_arena.free_spans.end() && next->first + next->second == after->first) {
    next->second += after->second;
    g_arena.free_spans.erase(after);
  }
  return TEMPO_OK;
}

extern "C" tempo_status tempo_device_reset(void) {
  std::lock_guard<std::mutex> lock(g_arena.mu);
  if (g_arena.base == nullptr) return fail(TEMPO_ERR_STATE, "tempo_device_reset: no device is open");
  g_arena.free_spans.clear();
  g_arena.free_spans[kReserved] = g_arena.size - kReserved;
  g_arena.allocs.clear();
  g_arena.images.clear();
  g_arena.used = 0;
  return TEMPO_OK;
}

static tempo_status check_copy(uint64_t host, uint64_t device, uint64_t nbytes) {
  if (nbytes == 0) return fail(TEMPO_ERR_VALUE, "Unable to copy. The byte count must be positive, but got a zero-length request.");
  if ((host % kAlign) || (device % kAlign))
    return fail(TEMPO_ERR_VALUE, "Unable to copy. Both addresses must be %llu-byte aligned, but got host 0x%llx and "
                                 "device 0x%llx.", (unsigned long long)kAlign, (unsigned long long)host,
                (unsigned long long)device);
  if (translate(device, nbytes) == nullptr)
    return fail(TEMPO_ERR_VALUE, "Unable to copy. The device range [0x%llx, 0x%llx) must lie inside the arena.",
                (unsigned long long)device, (unsigned long long)(device + nbytes));
  return TEMPO_OK;
}

extern "C" tempo_status tempo_memcpy_h2d(uint32_t dst, const void* src, uint64_t nbytes) {
  std::lock_guard<std::mutex> lock(g_arena.mu);
  if (g_arena.base == nullptr) return fail(TEMPO_ERR_STATE, "tempo_memcpy_h2d: no device is open");
  tempo_status s = check_copy(reinterpret_cast<uint64_t>(src), dst, nbytes);
  if (s != TEMPO_OK) return s;
  forget_images(uint64_t(dst) - kKernelBase, nbytes);
  cudaError_t err = cudaMemcpyAsync(translate(dst, nbytes), src, nbytes, cudaMemcpyHostToDevice, g_arena.stream);
  if (err != cudaSuccess) return cuda_fail(err, "cudaMemcpyAsync(host to device)");
  return sync_stream(g_arena.stream, 10.0);
}

extern "C" tempo_status tempo_memcpy_d2h(void* dst, uint32_t src, uint64_t nbytes) {
  std::lock_guard<std::mutex> lock(g_arena.mu);
  if (g_arena.base == nullptr) return fail(TEMPO_ERR_STATE, "tempo_memcpy_d2h: no device is open");
  tempo_status s = check_copy(reinterpret_cast<uint64_t>(dst), src, nbytes);
  if (s != TEMPO_OK) return s;
  cudaError_t err = cudaMemcpyAsync(dst, translate(src, nbytes), nbytes, cudaMemcpyDeviceToHost, g_arena.stream);
  if (err != cudaSuccess) return cuda_fail(err, "cudaMemcpyAsync(device to host)");
  return sync_stream(g_arena.stream, 10.0);
}

extern "C" tempo_status tempo_sync(double timeout_s) {
  cudaStream_t stream;
  {
    std::lock_guard<std::mutex> lock(g_arena.mu);
    stream = g_arena.stream;
  }
  if (stream == nullptr) {
    const cudaError_t err = cudaDeviceSynchronize();
    if (err != cudaSuccess) return cuda_fail(err, "cudaDeviceSynchronize");
    return watchdog_status();
  }
  return sync_stream(stream, timeout_s);
}

extern "C" tempo_status tempo_wait_probe(uint32_t arrive, uint64_t limit_ns, void* stream) {
  if (limit_ns == 0 || limit_ns > 10000000000ull)
    return fail(TEMPO_ERR_VALUE, "tempo_wait_probe: the limit must be in (0, 10 s], got %llu ns",
                (unsigned long long)limit_ns);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (s == nullptr) {
    std::lock_guard<std::mutex> lock(g_arena.mu);
    if (g_arena.stream == nullptr) return fail(TEMPO_ERR_STATE, "tempo_wait_probe: no device is open");
    s = g_arena.stream;
  }
  return launch_wait_probe(arrive, limit_ns, s);
}

extern "C" tempo_status tempo_host_alloc(void** ptr, uint64_t nbytes) {
  if (nbytes == 0) return fail(TEMPO_ERR_VALUE, "tempo_host_alloc: zero bytes");
  void* p = nullptr;
  const cudaError_t err = cudaHostAlloc(&p, nbytes, cudaHostAllocPortable);
  if (err != cudaSuccess) return fail(TEMPO_ERR_MEMORY, "cudaHostAlloc(%llu): %s", (unsigned long long)nbytes,
                                      cudaGetErrorString(err));
  std::lock_guard<std::mutex> lock(g_arena.mu);
  g_arena.host_buffers.insert(p);
  *ptr = p;
  return TEMPO_OK;
}

extern "C" tempo_status tempo_host_free(void* ptr) {
  std::lock_guard<std::mutex> lock(g_arena.mu);
  if (!g_arena.host_buffers.erase(ptr)) return fail(TEMPO_ERR_KEY, "tempo_host_free: unknown pointer");
  cudaFreeHost(ptr);
  return TEMPO_OK;
}

extern "C" tempo_status tempo_last_error(char* buffer, uint64_t size) {
  if (buffer == nullptr || size == 0) return TEMPO_ERR_VALUE;
  std::lock_guard<std::mutex> lock(g_error_mutex);
  std::strncpy(buffer, g_last_error.c_str(), size - 1);
  buffer[size - 1] = '\0';
  return TEMPO_OK;
}

extern "C" tempo_status tempo_stats(uint64_t* launches, uint64_t* arena_used) {
  std::lock_guard<std::mutex> lock(g_arena.mu);
  *launches = g_arena.launches;
  *arena_used = g_arena.used;
  return TEMPO_OK;
}

extern "C" tempo_status tempo_watchdog(int32_t* code) {
  int a, b, c;
  const int value = read_watchdogs(&a, &b, &c);
  *code = value < 0 ? 0 : value;
  return value < 0 ? fail(TEMPO_ERR_RUNTIME, "could not read the device watchdog") : TEMPO_OK;
}

// ---------------------------------------------------------------------------------------------------------------
// Launch of a staged image descriptor
// ---------------------------------------------------------------------------------------------------------------

namespace {

uint32_t image_checksum(const tempo_image& image) {
  const uint32_t* words = reinterpret_cast<const uint32_t*>(&image);
  uint32_t sum = 0;
  for (int i = 0; i < 14; ++i) sum += words[i];
  return sum;
}

// Resolves `nbytes` at kernel address `address` inside the arena, or fails naming the operand.
tempo_status operand(const char* kind, const char* name, uint64_t address, uint64_t nbytes, uint8_t** out,
                     bool need16 = true) {
  uint8_t* p = translate(address, nbytes);
  if (p == nullptr)
    return fail(TEMPO_ERR_VALUE, "Unable to launch the %s image. Its %s range [0x%llx, 0x%llx) must lie inside the "
                                 "device arena.", kind, name, (unsigned long long)address,
                (unsigned long long)(address + nbytes));
  if (need16 && (address % 16))
    return fail(TEMPO_ERR_VALUE, "Unable to launch the %s image. Its %s pointer 0x%llx must be 16-byte aligned.", kind,
                name, (unsigned long long)address);
  *out = p;
  return TEMPO_OK;
}

tempo_status dispatch(const tempo_image& im, const int64_t* args, uint32_t nargs) {
  const uint64_t a0 = nargs > 0 ? uint64_t(args[0]) : 0, a1 = nargs > 1 ? uint64_t(args[1]) : 0;
  const uint64_t a2 = nargs > 2 ? uint64_t(args[2]) : 0, a3 = nargs > 3 ? uint64_t(args[3]) : 0;
  cudaStream_t stream = g_arena.stream;
  uint8_t *p0 = nullptr, *p1 = nullptr, *p2 = nullptr, *p3 = nullptr;
  tempo_status s;
  auto need = [&](uint32_t count, const char* kind) -> tempo_status {
    if (nargs < count)
      return fail(TEMPO_ERR_VALUE, "Unable to launch the %s image. It binds %u arguments, but got %u.", kind, count,
                  nargs);
    return TEMPO_OK;
  };
  switch (im.kind) {
    case TEMPO_KIND_HALT:
      return TEMPO_OK;
    case TEMPO_KIND_GEMM:
    case TEMPO_KIND_GEMM_BIAS: {
      const bool bias = im.kind == TEMPO_KIND_GEMM_BIAS;
      const char* kind = bias ? "gemm_bias" : "gemm";
      const uint64_t depth = im.f[0], columns = im.f[1];
      if ((s = need(bias ? 4 : 3, kind))) return s;
      if ((s = operand(kind, "activations", a0, 32 * depth * 2, &p0))) return s;
      if ((s = operand(kind, "weights", a1, depth * columns * 2, &p1))) return s;
      if ((s = operand(kind, "drain", a2, 512 + 32 * columns * 2, &p2))) return s;
      if (bias && (s = operand(kind, "bias", a3, columns * 8, &p3))) return s;
      return tempo_block_gemm(p0, p1, p2, bias ? p3 : nullptr, uint32_t(depth), uint32_t(columns), im.f[2], stream);
    }
    case TEMPO_KIND_ADD:
    case TEMPO_KIND_ADD_BIAS: {
      const bool broadcast = im.kind == TEMPO_KIND_ADD_BIAS;
      const char* kind = broadcast ? "add_bias" : "add";
      const uint64_t features = im.f[0], bytes = 32 * features * 2;
      if ((s = need(3, kind))) return s;
      if ((s = operand(kind, "left", a0, bytes, &p0))) return s;
      if ((s = operand(kind, "right", a1, broadcast ? features * 8 : bytes, &p1))) return s;
      if ((s = operand(kind, "output", a2, bytes, &p2))) return s;
      return tempo_block_add(p0, p1, p2, uint32_t(features), broadcast, stream);
    }
    case TEMPO_KIND_LAYERNORM: {
      const uint64_t features = im.f[0], bytes = 32 * features * 2;
      if ((s = need(3, "layernorm"))) return s;
      if ((s = operand("layernorm", "rows", a0, bytes, &p0))) return s;
      if ((s = operand("layernorm", "constants", a1, (2 * features + 128) * 2, &p1))) return s;
      if ((s = operand("layernorm", "output", a2, bytes, &p2))) return s;
      return tempo_block_layernorm(p0, p1, p2, uint32_t(features), stream);
    }
    case TEMPO_KIND_ATTENTION: {
      const uint64_t tokens = im.f[0], heads = im.f[1], head = im.f[2];
      const uint64_t row = 3 * heads * head * 2, block = 512 + 32 * row;
      if ((s = need(3, "attention"))) return s;
      if ((s = operand("attention", "constants", a0, 3 * 512, &p0))) return s;
      if ((s = operand("attention", "fused tensor", a2, (tokens / 32 - 1) * block + 32 * row, &p2))) return s;
      return tempo_block_attention(p0, p2, uint32_t(tokens), uint32_t(heads), uint32_t(head), stream);
    }
    case TEMPO_KIND_DECODE_ATTENTION: {
      const uint64_t keys = im.f[0], heads = im.f[1], head = im.f[2], stated = im.f[3];
      const uint64_t width = heads * head, cache_block = 512 + 32 * 2 * width * 2;
      if ((s = need(3, "decode_attention"))) return s;
      if ((s = operand("decode_attention", "constants", a0, (2 + stated + keys / 16) * 512, &p0))) return s;
      if ((s = operand("decode_attention", "cache", a1, (keys / 32 - 1) * cache_block + 32 * 2 * width * 2, &p1)))
        return s;
      if ((s = operand("decode_attention", "fused tensor", a2, 32 * 3 * width * 2, &p2))) return s;
      return tempo_block_decode_attention(p0, p1, p2, uint32_t(keys), uint32_t(heads), uint32_t(head),
                                          uint32_t(stated), stream);
    }
    case TEMPO_KIND_COPY: {
      const uint64_t rows = im.f[0], stride = im.f[1], span = (rows - 1) * stride + 32;
      if ((s = need(3, "copy"))) return s;
      if ((s = operand("copy", "source", a0, span, &p0, false))) return s;
      if ((s = operand("copy", "destination", a2, span, &p2, false))) return s;
      return tempo_block_copy(p0, p2, uint32_t(rows), uint32_t(stride), stream);
    }
    default:
      return fail(TEMPO_ERR_RUNTIME, "Unable to complete the launch. The image names unknown kind %u.", im.kind);
  }
}

bool image_shape_ok(const tempo_image& im) {
  switch (im.kind) {
    case TEMPO_KIND_HALT: return true;
    case TEMPO_KIND_GEMM:
    case TEMPO_KIND_GEMM_BIAS:
      return im.f[0] && im.f[1] && !(im.f[0] % 16) && !(im.f[1] % 16) && im.f[2] <= 1 &&
             im.f[3] == 256 + im.f[1] * 32;
    case TEMPO_KIND_ADD:
    case TEMPO_KIND_ADD_BIAS:
    case TEMPO_KIND_LAYERNORM: return im.f[0] && !(im.f[0] % 16);
    case TEMPO_KIND_ATTENTION: return im.f[0] && !(im.f[0] % 32) && im.f[1] && im.f[2] == 64 && im.f[0] <= 65536;
    case TEMPO_KIND_DECODE_ATTENTION:
      return im.f[0] && !(im.f[0] % 32) && im.f[1] && im.f[2] == 64 && im.f[0] <= 65536;
    case TEMPO_KIND_COPY: return im.f[0] && im.f[1] >= 32;
    default: return false;
  }
}

}  // namespace

extern "C" tempo_status tempo_launch(uint64_t kbin_addr, uint64_t kbin_size, const int64_t* args, uint32_t nargs,
                                     double timeout_s) {
  // Rejects a malformed launch before touching the device, as runtime/launch.py:67-120 does.
  if (kbin_size == 0)
    return fail(TEMPO_ERR_VALUE, "Unable to launch a kernel. The binary size must be positive, but got 0.");
  if (kbin_size % 16)
    return fail(TEMPO_ERR_VALUE, "Unable to launch a kernel. The binary size must be a multiple of 16 bytes, but got "
                                 "%llu.", (unsigned long long)kbin_size);
  if (kbin_size > kMaxImage)
    return fail(TEMPO_ERR_VALUE, "Unable to launch a kernel. The binary must fit %llu bytes, but got %llu bytes.",
                (unsigned long long)kMaxImage, (unsigned long long)kbin_size);
  if (kbin_addr + kbin_size > (1ull << 32))
    return fail(TEMPO_ERR_VALUE, "Unable to launch a kernel. The device address range must fit 32 bits, but got "
                                 "[0x%llx, 0x%llx).", (unsigned long long)kbin_addr,
                (unsigned long long)(kbin_addr + kbin_size));
  if (kbin_addr % 32)
    return fail(TEMPO_ERR_VALUE, "Unable to launch a kernel. The binary base must be 32-byte aligned, but got 0x%llx.",
                (unsigned long long)kbin_addr);
  if (nargs > 4)
    return fail(TEMPO_ERR_VALUE, "Unable to launch a kernel. At most 4 values fit the argument slots, but got %u.",
                nargs);
  for (uint32_t i = 0; i < nargs; ++i)
    if (args[i] < 0 || args[i] > 0xFFFFFFFFll)
      return fail(TEMPO_ERR_VALUE, "Unable to launch a kernel. Argument slot %u must hold an unsigned 32-bit value, "
                                   "but got %lld.", i, (long long)args[i]);
  tempo_image image;
  {
    std::lock_guard<std::mutex> lock(g_arena.mu);
    if (g_arena.base == nullptr) return fail(TEMPO_ERR_STATE, "tempo_launch: no device is open");
    uint8_t* where = translate(kbin_addr, kbin_size);
    if (where == nullptr)
      return fail(TEMPO_ERR_VALUE, "Unable to launch a kernel. The binary range [0x%llx, 0x%llx) must lie inside the "
                                   "device arena.", (unsigned long long)kbin_addr,
                  (unsigned long long)(kbin_addr + kbin_size));
    const uint64_t offset = kbin_addr - kKernelBase;
    auto cached = g_arena.images.find(offset);
    if (cached != g_arena.images.end()) {
      image = cached->second;
    } else {
      if (kbin_size < TEMPO_IMAGE_BYTES)
        return fail(TEMPO_ERR_RUNTIME, "Unable to complete the launch. The %llu-byte binary at 0x%llx is shorter than "
                                       "an image descriptor, so the device never started it.",
                    (unsigned long long)kbin_size, (unsigned long long)kbin_addr);
      cudaError_t err = cudaMemcpyAsync(&image, where, sizeof(image), cudaMemcpyDeviceToHost, g_arena.stream);
      if (err == cudaSuccess) err = cudaStreamSynchronize(g_arena.stream);
      if (err != cudaSuccess) return cuda_fail(err, "reading the staged image");
      if (image.magic != TEMPO_IMAGE_MAGIC || image.version != 1 || image.checksum != image_checksum(image) ||
          !image_shape_ok(image))
        return fail(TEMPO_ERR_RUNTIME, "Unable to complete the launch. The binary at 0x%llx is not a valid image "
                                       "descriptor (magic 0x%08x, kind %u), so the device never started it.",
                    (unsigned long long)kbin_addr, image.magic, image.kind);
      g_arena.images[offset] = image;
    }
    const tempo_status s = dispatch(image, args, nargs);
    if (s != TEMPO_OK) return s;
    ++g_arena.launches;
  }
  return tempo_sync(timeout_s);
}
