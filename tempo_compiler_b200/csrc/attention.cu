// Decode attention: one new query per sequence and head over its resident KV cache, the bandwidth-bound step of
// generation. Each cached key and value is read once with 16-byte loads (8 lanes per key); every lane group keeps an
// online softmax (running maximum, sum and weighted values) over its keys, and the groups and warps merge at the end.
// Two layouts: the native engine's [seq][head][position][64] caches, and the drop-in packed cache
// (decode_attention, board_package/gpt2_inference.py:1006-1039) with the step's mask tiles added to the scores.
#include <cuda.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "decode_math.cuh"
#include "host.hpp"

namespace tempo {

TEMPO_WATCHDOG_READER(watchdog_attention)

namespace {

constexpr float kLog2e = kDecodeLog2e;

// A 16-byte load of streamed cache data that allocates no L1 line: each key and value is read exactly once, and the
// SM's L1 may be small when a kernel with a large shared-memory carveout shares the SM.
__device__ __forceinline__ uint4 ld_stream(const uint4* ptr) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(ptr));
  return v;
}

// Native decode over the [seq][head][capacity][64] caches. A cluster of `chunks` CTAs (4 warps each) serves one
// (head, sequence): CTA c takes a contiguous share of the keys (a multiple of 32), each warp 32 keys per iteration
// (8 per lane group, 16 independent 16-byte loads in flight per lane). Lane groups and warps merge their online
// softmax states on the CTA; with chunks > 1 every CTA then stores its (max, sum, 64 weighted values) into the
// cluster leader's shared memory, and the leader merges them and writes the output. Few sequences therefore still
// put every SM to work, with no workspace and no second kernel.
constexpr uint32_t kDecodeMaxChunks = 8;

__device__ __forceinline__ uint32_t decode_cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// KI keys per lane group per iteration (a warp covers 4 KI keys): 8 keeps 16 loads per lane in flight; 4 halves the
// registers (71) so up to seven CTAs per SM are resident at once. The host picks between them by grid size.
template <int KI>
__global__ void __launch_bounds__(128) decode_attention_kernel(const uint16_t* __restrict__ qkv,
                                                               const uint16_t* __restrict__ k_cache,
                                                               const uint16_t* __restrict__ v_cache,
                                                               const int32_t* __restrict__ lengths,
                                                               int32_t length_offset, uint16_t* __restrict__ out,
                                                               uint32_t heads, uint32_t capacity, uint32_t early) {
  if (early) pdl_launch_dependents();
  const uint32_t chunks = gridDim.x, h = blockIdx.y, s = blockIdx.z;
  // A CTA's shared memory may be addressed by the others of its cluster only once every CTA of the cluster has
  // started: each announces itself here and waits for the rest just before its first remote store.
  if (chunks > 1) asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  pdl_wait();
  const uint32_t chunk = chunks > 1 ? decode_cluster_rank() : 0u;
  const uint32_t warp = warp_id(), lane = lane_id();
  const uint32_t g = lane >> 3, li = lane & 7u;
  const uint32_t width = heads * 64;
  const int32_t len = max(0, min(lengths[s] + length_offset, int32_t(capacity)));
  int32_t k_begin, k_end;
  decode_chunk_range(len, chunks, chunk, k_begin, k_end);
  float q[8];
  load8(reinterpret_cast<const uint4*>(qkv + size_t(s) * 3 * width + h * 64)[li], q);
#pragma unroll
  for (int d = 0; d < 8; ++d) q[d] *= kLog2e;
  const uint4* kb4 = reinterpret_cast<const uint4*>(k_cache + (size_t(s) * heads + h) * capacity * 64);
  const uint4* vb4 = reinterpret_cast<const uint4*>(v_cache + (size_t(s) * heads + h) * capacity * 64);
  DecodeState st;
  decode_state_init(st);
  decode_stretch<KI>(st, q, kb4, vb4, k_begin, k_end, warp, g, li, [](const uint4* ptr) { return ld_stream(ptr); });
  // A grid of several waves lets the next kernel start its prologue only now: a trigger at entry would let that
  // kernel's CTAs take SM resources while later waves of this grid still wait to be scheduled.
  if (!early) pdl_launch_dependents();
  merge_shfl(st, 8);
  merge_shfl(st, 16);
  __shared__ float sm_m[4], sm_l[4], sm_acc[4][64];
  __shared__ float part[kDecodeMaxChunks][66];  // the leader's: per CTA of the cluster, (max, sum, 64 values)
  if (g == 0) {
#pragma unroll
    for (int d = 0; d < 8; ++d) sm_acc[warp][li * 8 + d] = st.acc[d];
    if (li == 0) { sm_m[warp] = st.m; sm_l[warp] = st.l; }
  }
  __syncthreads();
  const uint32_t d = threadIdx.x;
  float m = -INFINITY, l = 0.f, a = 0.f;
  if (d < 64) merge_warps(sm_m, sm_l, sm_acc, d, m, l, a);
  if (chunks == 1) {
    if (d < 64) out[size_t(s) * width + h * 64 + d] = float_to_bf16(l > 0.f ? a / l : 0.f);
    return;
  }
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
  if (d < 64) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(&part[chunk][0])), "r"(0u));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(remote + (2 + d) * 4), "f"(a) : "memory");
    if (d == 0) {
      asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(remote), "f"(m) : "memory");
      asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(remote + 4), "f"(l) : "memory");
    }
  }
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
  if (chunk == 0 && d < 64)
    out[size_t(s) * width + h * 64 + d] =
        float_to_bf16(merge_chunks(&part[0][0], 66, chunks, d, [](const float* f) { return *f; }));
}

// Packed drop-in decode: CTA per (head, group of 4 query rows); warp = one query row over all `keys` keys, scores
// plus the step's mask tile entry (keys x queries layout), running maximum entering at the constants' first value.
__global__ void __launch_bounds__(128) block_decode_kernel(const uint16_t* __restrict__ constants,
                                                           const uint8_t* __restrict__ cache,
                                                           uint8_t* __restrict__ fused, uint32_t keys,
                                                           uint32_t heads, uint32_t stated, uint64_t cache_block) {
  const uint32_t h = blockIdx.x;
  const uint32_t warp = warp_id(), lane = lane_id();
  const uint32_t q_row = blockIdx.y * 4 + warp;  // 0..15
  const uint32_t g = lane >> 3, li = lane & 7u;
  const uint32_t tile_off = (h * 4 + (li >> 1)) * 1024 + (li & 1u) * 16;  // this lane's 8 dims inside a block
  const uint32_t v_tile_off = heads * 4 * 1024;
  uint8_t* q_ptr = fused + tile_off + q_row * 32;
  float q[8];
  load8(*reinterpret_cast<const uint4*>(q_ptr), q);
#pragma unroll
  for (int d = 0; d < 8; ++d) q[d] *= kLog2e;
  const uint16_t* masks = constants + (2 + stated) * 256;
  DecodeState st;
  st.m = bf16_to_float(constants[0]) * kLog2e;  // entering maximum
  st.l = 0.f;
#pragma unroll
  for (int d = 0; d < 8; ++d) st.acc[d] = 0.f;
  for (uint32_t base = 0; base < keys; base += 16) {
    uint4 kk[4], vv[4];
    float mk[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t key = base + i * 4 + g;
      const uint8_t* row = cache + size_t(key >> 5) * cache_block + (key & 31u) * 32 + tile_off;
      kk[i] = __ldg(reinterpret_cast<const uint4*>(row));
      vv[i] = __ldg(reinterpret_cast<const uint4*>(row + v_tile_off));
      mk[i] = bf16_to_float(masks[(key >> 4) * 256 + (key & 15u) * 16 + q_row]);
    }
    float sc[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) sc[i] = group_dot(q, kk[i]) + mk[i] * kLog2e;
    fold<4>(st, sc, vv);
  }
  merge_shfl(st, 8);
  merge_shfl(st, 16);
  if (g == 0) {
    const float inv = st.l > 0.f ? 1.f / st.l : 0.f;
    float o[8];
#pragma unroll
    for (int d = 0; d < 8; ++d) o[d] = st.acc[d] * inv;
    uint4 w;
    w.x = pack_bf16x2(o[0], o[1]);
    w.y = pack_bf16x2(o[2], o[3]);
    w.z = pack_bf16x2(o[4], o[5]);
    w.w = pack_bf16x2(o[6], o[7]);
    *reinterpret_cast<uint4*>(q_ptr) = w;
  }
}

}  // namespace
}  // namespace tempo

using namespace tempo;

extern "C" tempo_status tempo_block_decode_attention(const void* constants, const void* cache, void* fused,
                                                     uint32_t keys, uint32_t heads, uint32_t head, uint32_t stated,
                                                     void* stream) {
  if (keys == 0 || keys % 32 || heads == 0 || head != 64)
    return fail(TEMPO_ERR_VALUE, "tempo_block_decode_attention: keys %u heads %u head %u", keys, heads, head);
  if (!aligned16(cache) || !aligned16(fused) || (reinterpret_cast<uintptr_t>(constants) & 1u))
    return fail(TEMPO_ERR_VALUE, "tempo_block_decode_attention: misaligned operand");
  const uint64_t cache_block = 512 + 32ull * 2 * heads * head * 2;
  block_decode_kernel<<<dim3(heads, 4), 128, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(constants), static_cast<const uint8_t*>(cache), static_cast<uint8_t*>(fused), keys,
      heads, stated, cache_block);
  return check_launch("block_decode_kernel");
}

extern "C" tempo_status tempo_decode_attention(const void* qkv, const void* k_cache, const void* v_cache,
                                               const int32_t* lengths, int32_t length_offset, void* out,
                                               uint32_t seqs, uint32_t heads, uint32_t head, uint32_t capacity,
                                               void* stream) {
  if (seqs == 0 || heads == 0 || head != 64 || capacity == 0 || seqs > 65535 || heads > 65535)
    return fail(TEMPO_ERR_VALUE, "tempo_decode_attention: seqs %u heads %u head %u capacity %u", seqs, heads, head,
                capacity);
  if (!aligned16(qkv) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(out))
    return fail(TEMPO_ERR_VALUE, "tempo_decode_attention: operands must be 16-byte aligned");
  // Fewer (sequence, head) pairs than SMs (a handful of sequences): split each over up to eight CTAs of a cluster,
  // each with at least 64 keys of the capacity (one iteration of the 4-key variant's four warps), until every SM has
  // one. Larger batches keep one CTA per pair: the cluster merge costs more than the parallelism it adds once every
  // SM is busy.
  const uint64_t pairs = uint64_t(seqs) * heads, target = uint64_t(sm_count());
  uint32_t chunks = 1;
  while (chunks < kDecodeMaxChunks && pairs * chunks < target && capacity >= 2 * 64 * chunks) chunks *= 2;
  // The bytes each SM keeps in flight bound this kernel until the grid is several waves deep: the 8-key variant has
  // 32 KB in flight per CTA at 4 CTAs per SM (126 registers), the 4-key one 16 KB at 7 (71 registers). Measured on a
  // B200 (1088 cached keys, 12 heads): the 8-key variant is faster up to 4 CTAs per SM (13-48 sequences: 12.6-24.7 us
  // against 16.4-30.8) and again from about 7 per SM, where the 4-key grid no longer fits one wave (88-112 sequences:
  // 44-60 us against 61-66); the 4-key one between (52-72 sequences: 31.2-37.7 us against 33.3-39.3). Fewer pairs than
  // SMs (a handful of sequences, split over clusters or not) keep the 4-key variant: the persistent decode step of up
  // to 8 sequences computes their stretches with its arithmetic, bit for bit.
  const uint64_t ctas = pairs * chunks;
  const bool four = pairs < target || (ctas > 4 * target && ctas <= 6 * target);
  auto kernel = four ? decode_attention_kernel<4> : decode_attention_kernel<8>;
  return launch(kernel, dim3(chunks, heads, seqs), dim3(128), 0, static_cast<cudaStream_t>(stream), chunks,
                "decode_attention_kernel", static_cast<const uint16_t*>(qkv), static_cast<const uint16_t*>(k_cache),
                static_cast<const uint16_t*>(v_cache), lengths, length_offset, static_cast<uint16_t*>(out), heads,
                capacity, single_wave(ctas, four ? 7 : 4));
}
