// Bandwidth-bound kernels: the residual add and bias add, LayerNorm, the KV-cache copies, the embedding gather,
// the KV store of the native engine and the argmax reduction. 128-bit vector loads and stores throughout; row
// reductions are warp shuffles.
#include <cuda_runtime.h>

#include "common.cuh"
#include "host.hpp"

namespace tempo {
namespace {

constexpr uint32_t kBlockTokens = 32;
constexpr uint32_t kTile = 16;

// ---- packed block add: out = round(left + right) or round(left + bias row t%4), 8 values per thread ----
__global__ void block_add_kernel(const uint4* __restrict__ left, const uint4* __restrict__ right,
                                 uint4* __restrict__ out, uint32_t vectors, uint32_t broadcast) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= vectors) return;
  float a[8], b[8];
  unpack8(left[i], a);
  if (broadcast) {
    // Vector i covers values 8i..8i+7 of [tiles][32][16]: tile i/64, token (i/2)%32, half i%2.
    const uint32_t tile = i >> 6, token = (i >> 1) & 31u, half = i & 1u;
    unpack8(right[(tile * 4 + (token & 3u)) * 2 + half], b);
  } else {
    unpack8(right[i], b);
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) a[j] += b[j];
  out[i] = pack8(a);
}

// ---- packed block LayerNorm: one warp per token; features strided 1 KB apart in 16-wide tiles ----
__global__ void block_layernorm_kernel(const uint16_t* __restrict__ rows, const uint16_t* __restrict__ constants,
                                       uint16_t* __restrict__ out, uint32_t features) {
  const uint32_t token = blockIdx.x * (blockDim.x / 32) + warp_id();
  if (token >= kBlockTokens) return;
  const uint32_t lane = lane_id();
  const uint32_t chunks = features / 8;  // 16-byte chunks per token
  auto chunk_offset = [&](uint32_t c) { return (c >> 1) * (kBlockTokens * kTile) + token * kTile + (c & 1u) * 8; };
  const float inverse = bf16_to_float(constants[2 * features]);
  const float epsilon = bf16_to_float(constants[2 * features + 64]);
  float sum = 0.f;
  for (uint32_t c = lane; c < chunks; c += 32) {
    float f[8];
    unpack8(*reinterpret_cast<const uint4*>(rows + chunk_offset(c)), f);
#pragma unroll
    for (int j = 0; j < 8; ++j) sum += f[j];
  }
  const float mean = warp_sum(sum) * inverse;
  float sq = 0.f;
  for (uint32_t c = lane; c < chunks; c += 32) {
    float f[8];
    unpack8(*reinterpret_cast<const uint4*>(rows + chunk_offset(c)), f);
#pragma unroll
    for (int j = 0; j < 8; ++j) sq += (f[j] - mean) * (f[j] - mean);
  }
  const float scale = rsqrtf(warp_sum(sq) * inverse + epsilon);
  for (uint32_t c = lane; c < chunks; c += 32) {
    float f[8], g[8], b[8];
    unpack8(*reinterpret_cast<const uint4*>(rows + chunk_offset(c)), f);
    unpack8(*reinterpret_cast<const uint4*>(constants + c * 8), g);
    unpack8(*reinterpret_cast<const uint4*>(constants + features + c * 8), b);
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = (f[j] - mean) * scale * g[j] + b[j];
    *reinterpret_cast<uint4*>(out + chunk_offset(c)) = pack8(f);
  }
}

// ---- packed row copy: `rows` 32-byte rows, `stride` bytes apart at both ends; 4-byte words ----
__global__ void block_copy_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, uint32_t rows,
                                  uint32_t stride) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;  // word index: 8 words per row
  if (i >= rows * 8) return;
  const size_t offset = size_t(i >> 3) * stride + (i & 7u) * 4;
  *reinterpret_cast<uint32_t*>(dst + offset) = *reinterpret_cast<const uint32_t*>(src + offset);
}

// ---- native LayerNorm: one warp per row, CPL 16-byte chunks per lane held in registers ----
template <int CPL>
__global__ void layernorm_kernel(const uint16_t* __restrict__ x, uint32_t x_stride,
                                 const uint16_t* __restrict__ gamma, const uint16_t* __restrict__ beta,
                                 uint16_t* __restrict__ out, uint32_t rows, uint32_t features, float epsilon,
                                 uint32_t early) {
  if (early) pdl_launch_dependents();
  pdl_wait();
  const uint32_t row = blockIdx.x * (blockDim.x / 32) + warp_id();
  if (row < rows)
    layernorm_row<CPL>(x + size_t(row) * x_stride, gamma, beta, features, epsilon, out + size_t(row) * features);
  if (!early) pdl_launch_dependents();
}

// ---- row statistics partials: (mean, M2) of each 16-column chunk of each row, for a folded LayerNorm ----
__global__ void row_stats_kernel(const uint16_t* __restrict__ x, uint32_t ldx, uint32_t rows, uint32_t width,
                                 float2* __restrict__ stats, uint32_t early) {
  if (early) pdl_launch_dependents();
  pdl_wait();
  const uint32_t chunks = width / 16;
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < rows * chunks) {
    const uint32_t r = i / chunks, c = i % chunks;
    const uint4* src = reinterpret_cast<const uint4*>(x + size_t(r) * ldx + c * 16);
    float lo[8], hi[8], w[16];
    unpack8(src[0], lo);
    unpack8(src[1], hi);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      w[j] = lo[j];
      w[8 + j] = hi[j];
    }
    stats[i] = chunk_stats16(w);
  }
  if (!early) pdl_launch_dependents();
}

// ---- embedding gather: x[r] = round(wte[ids[r]] + wpe[pos[r]]) ----
__global__ void embed_kernel(const int32_t* __restrict__ ids, const int32_t* __restrict__ positions,
                             const uint16_t* __restrict__ wte, const uint16_t* __restrict__ wpe,
                             uint16_t* __restrict__ x, uint32_t rows, uint32_t width, uint32_t vocab,
                             uint32_t max_positions, uint32_t early) {
  if (early) pdl_launch_dependents();
  pdl_wait();
  const uint32_t per_row = width / 8;
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * per_row) return;
  const uint32_t r = i / per_row, c = i % per_row;
  if (uint32_t(ids[r]) >= vocab || uint32_t(positions[r]) >= max_positions) {
    reinterpret_cast<uint4*>(x + size_t(r) * width)[c] = make_uint4(0, 0, 0, 0);
    return;
  }
  float a[8], b[8];
  unpack8(__ldg(reinterpret_cast<const uint4*>(wte + size_t(ids[r]) * width) + c), a);
  unpack8(__ldg(reinterpret_cast<const uint4*>(wpe + size_t(positions[r]) * width) + c), b);
#pragma unroll
  for (int j = 0; j < 8; ++j) a[j] += b[j];
  reinterpret_cast<uint4*>(x + size_t(r) * width)[c] = pack8(a);
  if (!early) pdl_launch_dependents();
}

// ---- KV store: keys and values of qkv rows into [seq][head][capacity][head_dim] caches ----
__global__ void kv_store_kernel(const uint16_t* __restrict__ qkv, uint16_t* __restrict__ k_cache,
                                uint16_t* __restrict__ v_cache, const int32_t* __restrict__ seq_of,
                                const int32_t* __restrict__ pos_of, uint32_t rows, uint32_t seqs, uint32_t heads,
                                uint32_t head, uint32_t capacity, uint32_t early) {
  if (early) pdl_launch_dependents();
  pdl_wait();
  const uint32_t width = heads * head;
  const uint32_t per_row = 2 * width / 8;  // 16-byte vectors of keys then values
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * per_row) return;
  const uint32_t r = i / per_row, c = i % per_row;
  if (uint32_t(seq_of[r]) >= seqs || uint32_t(pos_of[r]) >= capacity) return;
  const uint32_t which = (c * 8) / width;       // 0 keys, 1 values
  const uint32_t feature = (c * 8) % width;
  const uint32_t h = feature / head, d = feature % head;
  const uint4 w = reinterpret_cast<const uint4*>(qkv + size_t(r) * 3 * width + width + which * width + feature)[0];
  uint16_t* cache = which ? v_cache : k_cache;
  const size_t slot = ((size_t(seq_of[r]) * heads + h) * capacity + size_t(pos_of[r])) * head + d;
  *reinterpret_cast<uint4*>(cache + slot) = w;
  if (!early) pdl_launch_dependents();
}

// ---- argmax reduction over the LM head's per-tile partials; first index wins ties ----
__global__ void argmax_finish_kernel(const float* __restrict__ part_val, const int32_t* __restrict__ part_idx,
                                     uint32_t rows, uint32_t tiles, int32_t* __restrict__ ids,
                                     int32_t* __restrict__ tokens_out, uint32_t out_stride,
                                     int32_t* __restrict__ positions, int32_t index_offset, int32_t advance) {
  pdl_launch_dependents();
  pdl_wait();
  const uint32_t row = blockIdx.x * (blockDim.x / 32) + warp_id();
  if (row >= rows) return;
  const uint32_t lane = lane_id();
  float best = -INFINITY;
  int32_t idx = 0x7FFFFFFF;
  for (uint32_t t = lane; t < tiles; t += 32) {
    const float v = part_val[size_t(row) * tiles + t];
    const int32_t i = part_idx[size_t(row) * tiles + t];
    if (v > best || (v == best && i < idx)) { best = v; idx = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xFFFFFFFFu, best, o);
    const int32_t oi = __shfl_xor_sync(0xFFFFFFFFu, idx, o);
    if (ov > best || (ov == best && oi < idx)) { best = ov; idx = oi; }
  }
  if (lane == 0) {
    ids[row] = idx;
    if (tokens_out != nullptr) {
      const int32_t column = (positions != nullptr ? positions[row] : 0) + index_offset;
      if (column >= 0 && uint32_t(column) < out_stride) tokens_out[size_t(row) * out_stride + column] = idx;
    }
    if (positions != nullptr) positions[row] += advance;
  }
}

}  // namespace
}  // namespace tempo

using namespace tempo;

extern "C" tempo_status tempo_block_add(const void* left, const void* right, void* out, uint32_t features,
                                        uint32_t broadcast, void* stream) {
  if (features == 0 || features % 16) return fail(TEMPO_ERR_VALUE, "tempo_block_add: features %u", features);
  if (!aligned16(left) || !aligned16(right) || !aligned16(out))
    return fail(TEMPO_ERR_VALUE, "tempo_block_add: operands must be 16-byte aligned");
  const uint32_t vectors = kBlockTokens * features / 8;
  block_add_kernel<<<(vectors + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(left), static_cast<const uint4*>(right), static_cast<uint4*>(out), vectors,
      broadcast);
  return check_launch("block_add_kernel");
}

extern "C" tempo_status tempo_block_layernorm(const void* rows, const void* constants, void* out, uint32_t features,
                                              void* stream) {
  if (features == 0 || features % 16) return fail(TEMPO_ERR_VALUE, "tempo_block_layernorm: features %u", features);
  if (!aligned16(rows) || !aligned16(constants) || !aligned16(out))
    return fail(TEMPO_ERR_VALUE, "tempo_block_layernorm: operands must be 16-byte aligned");
  block_layernorm_kernel<<<4, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(rows), static_cast<const uint16_t*>(constants), static_cast<uint16_t*>(out),
      features);
  return check_launch("block_layernorm_kernel");
}

extern "C" tempo_status tempo_block_copy(const void* source, void* destination, uint32_t rows, uint32_t stride,
                                         void* stream) {
  if (rows == 0 || stride < 32) return fail(TEMPO_ERR_VALUE, "tempo_block_copy: rows %u stride %u", rows, stride);
  if ((reinterpret_cast<uintptr_t>(source) | reinterpret_cast<uintptr_t>(destination) | stride) & 3u)
    return fail(TEMPO_ERR_VALUE, "tempo_block_copy: addresses and stride must be 4-byte aligned");
  const uint32_t words = rows * 8;
  block_copy_kernel<<<(words + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(source), static_cast<uint8_t*>(destination), rows, stride);
  return check_launch("block_copy_kernel");
}

extern "C" tempo_status tempo_layernorm(const void* x, uint32_t x_stride, const void* gamma, const void* beta,
                                        void* out, uint32_t rows, uint32_t features, float epsilon, void* stream) {
  if (rows == 0 || features == 0 || features % 8 || features > 4096 || x_stride < features || x_stride % 8)
    return fail(TEMPO_ERR_VALUE, "tempo_layernorm: rows %u features %u stride %u", rows, features, x_stride);
  if (!aligned16(x) || !aligned16(gamma) || !aligned16(beta) || !aligned16(out))
    return fail(TEMPO_ERR_VALUE, "tempo_layernorm: operands must be 16-byte aligned");
  const uint32_t cpl = (features / 8 + 31) / 32;
  const dim3 grid((rows + 7) / 8), block(256);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto* xs = static_cast<const uint16_t*>(x);
  auto* gs = static_cast<const uint16_t*>(gamma);
  auto* bs = static_cast<const uint16_t*>(beta);
  auto* os = static_cast<uint16_t*>(out);
  auto kernel = cpl <= 1 ? layernorm_kernel<1>
              : cpl <= 2 ? layernorm_kernel<2>
              : cpl <= 3 ? layernorm_kernel<3>
              : cpl <= 4 ? layernorm_kernel<4>
              : cpl <= 8 ? layernorm_kernel<8>
                         : layernorm_kernel<16>;
  return launch(kernel, grid, block, 0, st, 1, "layernorm_kernel", xs, x_stride, gs, bs, os, rows, features, epsilon,
                single_wave(grid.x, 8));
}

extern "C" tempo_status tempo_row_stats(const void* x, uint32_t ldx, uint32_t rows, uint32_t width, float* stats,
                                        void* stream) {
  if (rows == 0 || width == 0 || width % 16 || ldx < width || ldx % 8 || !aligned16(x) || stats == nullptr ||
      (reinterpret_cast<uintptr_t>(stats) & 7u))
    return fail(TEMPO_ERR_VALUE, "tempo_row_stats: rows %u width %u (multiple of 16) stride %u, aligned operands", rows,
                width, ldx);
  const uint64_t threads = uint64_t(rows) * (width / 16);
  const dim3 grid(uint32_t((threads + 255) / 256)), block(256);
  return launch(row_stats_kernel, grid, block, 0, static_cast<cudaStream_t>(stream), 1, "row_stats_kernel",
                static_cast<const uint16_t*>(x), ldx, rows, width, reinterpret_cast<float2*>(stats),
                single_wave(grid.x, 8));
}

extern "C" tempo_status tempo_embed(const int32_t* ids, const int32_t* positions, const void* wte, const void* wpe,
                                    void* x, uint32_t rows, uint32_t width, uint32_t vocab, uint32_t max_positions,
                                    void* stream) {
  if (rows == 0 || width == 0 || width % 8) return fail(TEMPO_ERR_VALUE, "tempo_embed: rows %u width %u", rows, width);
  if (!aligned16(wte) || !aligned16(wpe) || !aligned16(x))
    return fail(TEMPO_ERR_VALUE, "tempo_embed: operands must be 16-byte aligned");
  const uint64_t threads = uint64_t(rows) * (width / 8);
  const uint32_t blocks = uint32_t((threads + 255) / 256);
  return launch(embed_kernel, dim3(blocks), dim3(256), 0, static_cast<cudaStream_t>(stream), 1, "embed_kernel", ids,
                positions, static_cast<const uint16_t*>(wte), static_cast<const uint16_t*>(wpe),
                static_cast<uint16_t*>(x), rows, width, vocab, max_positions, single_wave(blocks, 8));
}

extern "C" tempo_status tempo_kv_store(const void* qkv, void* k_cache, void* v_cache, const int32_t* seq_of,
                                       const int32_t* pos_of, uint32_t rows, uint32_t seqs, uint32_t heads,
                                       uint32_t head, uint32_t capacity, void* stream) {
  if (rows == 0 || heads == 0 || head == 0 || head % 8 || capacity == 0)
    return fail(TEMPO_ERR_VALUE, "tempo_kv_store: rows %u heads %u head %u capacity %u", rows, heads, head, capacity);
  if (!aligned16(qkv) || !aligned16(k_cache) || !aligned16(v_cache))
    return fail(TEMPO_ERR_VALUE, "tempo_kv_store: operands must be 16-byte aligned");
  const uint64_t threads = uint64_t(rows) * (2 * heads * head / 8);
  const uint32_t blocks = uint32_t((threads + 255) / 256);
  return launch(kv_store_kernel, dim3(blocks), dim3(256), 0, static_cast<cudaStream_t>(stream), 1, "kv_store_kernel",
                static_cast<const uint16_t*>(qkv), static_cast<uint16_t*>(k_cache), static_cast<uint16_t*>(v_cache),
                seq_of, pos_of, rows, seqs, heads, head, capacity, single_wave(blocks, 8));
}

extern "C" tempo_status tempo_argmax_finish(const float* part_val, const int32_t* part_idx, uint32_t rows,
                                            uint32_t tiles, int32_t* ids, int32_t* tokens_out, uint32_t out_stride,
                                            int32_t* positions, int32_t index_offset, int32_t advance,
                                            void* stream) {
  if (rows == 0 || tiles == 0) return fail(TEMPO_ERR_VALUE, "tempo_argmax_finish: rows %u tiles %u", rows, tiles);
  return launch(argmax_finish_kernel, dim3((rows + 7) / 8), dim3(256), 0, static_cast<cudaStream_t>(stream), 1,
                "argmax_finish_kernel", part_val, part_idx, rows, tiles, ids, tokens_out, out_stride, positions,
                index_offset, advance);
}
