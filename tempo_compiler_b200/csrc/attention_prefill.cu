// Causal prefill attention on the 5th-generation tensor cores (flash-attention tile loop, one CTA per 128 queries of
// one head of one sequence, two CTAs per SM).
//
//   warp 0      TMA: Q once, then K and V 128 keys at a time into a two-stage ring.
//   warp 1      MMA issuer and TMEM owner: S = Q K^T into TMEM (128 columns, FP32); after the softmax has written P
//               over S, O += P V with P read straight from TMEM (A operand in tensor memory) and V from shared memory;
//               O stays in TMEM (64 columns) for the whole key loop.
//   warps 2-5   softmax, one query row per thread: read S, mask (diagonal tile only), exp2 on the special-function
//               unit, P as BF16 pairs into TMEM, the row sum in FP32. The exponent base only moves when the row
//               maximum grows by more than 2^8; only then are O and the sum rescaled (in TMEM), which keeps the math
//               exact while skipping almost every rescale. At the end O / sum is written out.
//
// Two source layouts share the kernel:
//   PACKED    the drop-in fused QKV tensor, per 32-token block a 512-byte zero tile then [3*heads*4][32][16]
//             (attention, board_package/gpt2_inference.py:981-1003; tempo_ops.td:292-314). A 4-D tensor map
//             (16, 32 tokens, blocks, 16-wide feature tiles) loads 4 blocks x 4 tiles, which lands as four 128-row
//             K-major 32-byte-swizzled tiles: exactly the MMA operand layout. The output overwrites the queries.
//   ROWMAJOR  the native engine's qkv [seqs*tokens, 3*heads*64], 128-byte swizzle, output to its own buffer.
// Queries arrive scaled by 1/sqrt(head) (folded into the QKV weights, gpt2_inference.py:1153-1168).
#include <cuda.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "host.hpp"

namespace tempo {

TEMPO_WATCHDOG_READER(watchdog_prefill)

namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale only when the maximum grows by more than 2^8
constexpr int kThreads = 192;
constexpr uint32_t kTileBytes = 128 * 64 * 2;  // one 128 x 64 BF16 operand tile

struct PrefillParams {
  uint16_t* out;         // ROWMAJOR: [seqs*tokens, heads*64]; PACKED: the fused tensor (queries overwritten)
  uint32_t seqs, tokens, heads;
  uint32_t q_tiles;      // ceil(tokens / 128)
  uint64_t block_bytes;  // PACKED: bytes per 32-token block of the fused tensor
};

// Shared memory: Q | K[2] | V[2] | barriers.
constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffK = kTileBytes;
constexpr uint32_t kOffV = 3 * kTileBytes;
constexpr uint32_t kOffBar = 5 * kTileBytes;
// q_full, kv_full[2], kv_empty[2], s_full, p_full, o_full, final
constexpr uint32_t kBarCount = 9;
constexpr uint32_t kSmem = kOffBar + kBarCount * 8 + 16 + 1024;

template <bool PACKED>
__device__ __forceinline__ void load_tile(void* dst, const CUtensorMap* map, uint64_t* bar, uint32_t feature_tile16,
                                          int32_t row_or_block) {
  if constexpr (PACKED) {
    tma_load_4d(dst, map, bar, 0, 0, row_or_block, int32_t(feature_tile16));
  } else {
    tma_load_2d(dst, map, bar, int32_t(feature_tile16 * 16), row_or_block);
  }
}

// Descriptor of the kk-th 16-deep K-major slice of a 128-row operand tile.
template <bool PACKED>
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t tile_addr, uint32_t kk) {
  if constexpr (PACKED) return make_smem_desc(tile_addr + kk * 4096, 16, 256, kLayoutSw32);
  else return make_smem_desc(tile_addr + kk * 32, 16, 1024, kLayoutSw128);
}

// Descriptor of the kk-th 16-key slice of V as the MN-major B operand (N = 64 head dims).
template <bool PACKED>
__device__ __forceinline__ uint64_t v_desc(uint32_t tile_addr, uint32_t kk) {
  if constexpr (PACKED) return make_smem_desc(tile_addr + kk * 512, 4096, 256, kLayoutSw32);
  else return make_smem_desc(tile_addr + kk * 2048, 8192, 1024, kLayoutSw128);
}

template <bool PACKED>
__global__ void __launch_bounds__(kThreads, 2)
    attention_prefill_kernel(const __grid_constant__ CUtensorMap tmap, PrefillParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = bars + 3;
  uint64_t* s_full = bars + 5;
  uint64_t* p_full = bars + 6;
  uint64_t* o_full = bars + 7;
  uint64_t* final_bar = bars + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kBarCount);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  // Heaviest query tiles first (causal: tile qt reads qt+1 key tiles).
  const uint32_t qt = p.q_tiles - 1 - (blockIdx.x % p.q_tiles);
  const uint32_t h = (blockIdx.x / p.q_tiles) % p.heads;
  const uint32_t s = blockIdx.x / (p.q_tiles * p.heads);
  const uint32_t kv_tiles = qt + 1;
  const uint32_t warp = warp_id(), lane = lane_id();
  const uint32_t heads4 = p.heads * 4;  // 16-wide feature tiles per third of the fused tensor

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(p_full, 128);
    mbar_init(o_full, 1);
    mbar_init(final_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmap);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t tmem_s = tmem_base;        // 128 columns: S (FP32), then P (BF16 pairs) in its first 64
  const uint32_t tmem_o = tmem_base + 128;  // 64 columns: O (FP32)
  pdl_launch_dependents();
  pdl_wait();  // Q, K and V are the previous kernel's output

  auto tile_coord = [&](uint32_t t) -> int32_t {
    if constexpr (PACKED) return int32_t(t * 4);
    else return int32_t(s * p.tokens + t * 128);
  };

  if (warp == 0) {
    if (elect_one()) {
      bool issued[2] = {false, false};
      uint32_t parity_of[2] = {0, 0};
      mbar_arrive_expect_tx(q_full, kTileBytes);
      load_tile<PACKED>(smem + kOffQ, &tmap, q_full, h * 4, tile_coord(qt));
      for (uint32_t j = 0; j < kv_tiles; ++j) {
        const uint32_t st = j & 1u, ph = (j >> 1) & 1u;
        if (!mbar_wait(&kv_empty[st], ph ^ 1u, kWatchEmpty, abort_flag)) break;
        mbar_arrive_expect_tx(&kv_full[st], 2 * kTileBytes);
        load_tile<PACKED>(smem + kOffK + st * kTileBytes, &tmap, &kv_full[st], heads4 + h * 4, tile_coord(j));
        load_tile<PACKED>(smem + kOffV + st * kTileBytes, &tmap, &kv_full[st], 2 * heads4 + h * 4, tile_coord(j));
        issued[st] = true;
        parity_of[st] = ph;
      }
      mbar_wait(q_full, 0, kWatchFull, nullptr);
      for (int i = 0; i < 2; ++i)
        if (issued[i]) mbar_wait(&kv_full[i], parity_of[i], kWatchFull, nullptr);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc_s = make_idesc_bf16(128, 128, 0, 0);
      constexpr uint32_t idesc_o = make_idesc_bf16(128, 64, 0, 1);
      const uint32_t q_addr = smem_u32(smem + kOffQ);
      bool ok = mbar_wait(q_full, 0, kWatchFull, abort_flag);
      for (uint32_t j = 0; j < kv_tiles && ok; ++j) {
        const uint32_t st = j & 1u, ph = (j >> 1) & 1u;
        if (!mbar_wait(&kv_full[st], ph, kWatchFull, abort_flag)) break;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + kOffK + st * kTileBytes);
        const uint32_t v_addr = smem_u32(smem + kOffV + st * kTileBytes);
        // S overwrites the P of the previous tile, which the P V issued just before has read (issue order).
#pragma unroll
        for (uint32_t kk = 0; kk < 4; ++kk)
          umma_bf16(tmem_s, kmajor_desc<PACKED>(q_addr, kk), kmajor_desc<PACKED>(k_addr, kk), idesc_s, kk != 0);
        umma_commit(s_full);
        if (!mbar_wait(p_full, j & 1u, kWatchOther, abort_flag)) break;
        tc_fence_after();
#pragma unroll
        for (uint32_t kk = 0; kk < 8; ++kk)
          umma_bf16_tmem_a(tmem_o, tmem_s + kk * 8, v_desc<PACKED>(v_addr, kk), idesc_o, (j | kk) != 0u);
        umma_commit(o_full);
        umma_commit(&kv_empty[st]);
      }
      umma_commit(final_bar);
      mbar_wait(final_bar, 0, kWatchOther, nullptr);
    }
  } else {
    const uint32_t lane_base = 32u * (warp & 3u);
    const uint32_t row = lane_base + lane;
    const uint32_t q_local = qt * 128 + row;  // query position in the sequence
    const uint32_t lane_addr = lane_base << 16;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (uint32_t j = 0; j < kv_tiles; ++j) {
      if (!mbar_wait(s_full, j & 1u, kWatchOther, abort_flag)) { ok = false; break; }
      tc_fence_after();
      uint32_t sr[128];
      tmem_ld_32x32b_x32(tmem_s + lane_addr + 0, *reinterpret_cast<uint32_t(*)[32]>(sr + 0));
      tmem_ld_32x32b_x32(tmem_s + lane_addr + 32, *reinterpret_cast<uint32_t(*)[32]>(sr + 32));
      tmem_ld_32x32b_x32(tmem_s + lane_addr + 64, *reinterpret_cast<uint32_t(*)[32]>(sr + 64));
      tmem_ld_32x32b_x32(tmem_s + lane_addr + 96, *reinterpret_cast<uint32_t(*)[32]>(sr + 96));
      tmem_wait_ld();
      float mx = -INFINITY;
      if (j == qt) {
        // Diagonal tile: keys past the query, and past the sequence end, are masked.
#pragma unroll
        for (int c = 0; c < 128; ++c) {
          const uint32_t key = j * 128 + c;
          float v = __uint_as_float(sr[c]) * kLog2e;
          if (key > q_local || key >= p.tokens) v = -INFINITY;
          sr[c] = __float_as_uint(v);
          mx = fmaxf(mx, v);
        }
      } else {
#pragma unroll
        for (int c = 0; c < 128; ++c) {
          const float v = __uint_as_float(sr[c]) * kLog2e;
          sr[c] = __float_as_uint(v);
          mx = fmaxf(mx, v);
        }
      }
      bool rescale = false;
      float factor = 1.f;
      if (j == 0) {
        m_used = mx;
      } else if (mx > m_used + kRescaleThreshold) {
        factor = fast_exp2(m_used - mx);
        m_used = mx;
        l *= factor;
        rescale = true;
      }
      const float base = m_used == -INFINITY ? 0.f : m_used;
      float sum = 0.f;
#pragma unroll
      for (int c16 = 0; c16 < 4; ++c16) {
        uint32_t packed[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float e0 = fast_exp2(__uint_as_float(sr[c16 * 32 + 2 * i]) - base);
          const float e1 = fast_exp2(__uint_as_float(sr[c16 * 32 + 2 * i + 1]) - base);
          sum += e0 + e1;
          packed[i] = pack_bf16x2(e0, e1);
        }
        tmem_st_32x32b_x16(tmem_s + lane_addr + c16 * 16, packed);
      }
      l += sum;
      // The rescale must wait for the previous P V (the only MMA writing O) to finish.
      const bool warp_rescale = __any_sync(0xFFFFFFFFu, rescale);
      if (warp_rescale) {
        if (!mbar_wait(o_full, (j - 1) & 1u, kWatchOther, abort_flag)) { ok = false; }
        if (ok) {
          tc_fence_after();
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            uint32_t orr[32];
            tmem_ld_32x32b_x32(tmem_o + lane_addr + half * 32, orr);
            tmem_wait_ld();
            uint32_t lo[16], hi[16];
#pragma unroll
            for (int d = 0; d < 16; ++d) {
              lo[d] = __float_as_uint(__uint_as_float(orr[d]) * factor);
              hi[d] = __float_as_uint(__uint_as_float(orr[16 + d]) * factor);
            }
            tmem_st_32x32b_x16(tmem_o + lane_addr + half * 32, lo);
            tmem_st_32x32b_x16(tmem_o + lane_addr + half * 32 + 16, hi);
          }
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(p_full);
      if (!ok) break;
    }
    if (ok && mbar_wait(o_full, (kv_tiles - 1) & 1u, kWatchOther, abort_flag)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t orr[32];
        tmem_ld_32x32b_x32(tmem_o + lane_addr + half * 32, orr);
        tmem_wait_ld();
        if (q_local < p.tokens) {
          uint32_t w[16];
#pragma unroll
          for (int d = 0; d < 16; ++d)
            w[d] = pack_bf16x2(__uint_as_float(orr[2 * d]) * inv, __uint_as_float(orr[2 * d + 1]) * inv);
          if constexpr (PACKED) {
            // dims half*32 .. +31 are feature tiles h*4 + 2*half and +1 of the query's block
            uint8_t* base_ptr = reinterpret_cast<uint8_t*>(p.out) + size_t(q_local >> 5) * p.block_bytes +
                                size_t(h * 4 + 2 * half) * 1024 + (q_local & 31u) * 32;
            uint4* t0 = reinterpret_cast<uint4*>(base_ptr);
            uint4* t1 = reinterpret_cast<uint4*>(base_ptr + 1024);
            t0[0] = make_uint4(w[0], w[1], w[2], w[3]);
            t0[1] = make_uint4(w[4], w[5], w[6], w[7]);
            t1[0] = make_uint4(w[8], w[9], w[10], w[11]);
            t1[1] = make_uint4(w[12], w[13], w[14], w[15]);
          } else {
            uint4* dst = reinterpret_cast<uint4*>(p.out + (size_t(s) * p.tokens + q_local) * (p.heads * 64) + h * 64 +
                                                  half * 32);
            dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
            dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
            dst[2] = make_uint4(w[8], w[9], w[10], w[11]);
            dst[3] = make_uint4(w[12], w[13], w[14], w[15]);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 256);
  }
}

}  // namespace
}  // namespace tempo

using namespace tempo;

extern "C" tempo_status tempo_block_attention(const void* constants, void* fused, uint32_t tokens, uint32_t heads,
                                              uint32_t head, void* stream) {
  (void)constants;  // the causal diagonal mask is computed in-kernel; the runtime validates the block's range
  if (tokens == 0 || tokens % 32 || heads == 0 || head != 64)
    return fail(TEMPO_ERR_VALUE, "tempo_block_attention: tokens %u (multiple of 32), heads %u, head %u (64)", tokens,
                heads, head);
  if (!aligned16(fused)) return fail(TEMPO_ERR_VALUE, "tempo_block_attention: fused tensor must be 16-byte aligned");
  const uint64_t block_bytes = 512 + 32ull * 3 * heads * head * 2;
  CUtensorMap map;
  // The queries pointer is past block 0's zero tile; the map addresses every block's tiles from there.
  const uint64_t dims[4] = {16, 32, tokens / 32, 3ull * heads * 4};
  const uint64_t strides[3] = {32, block_bytes, 1024};
  const uint32_t box[4] = {16, 32, 4, 4};
  tempo_status s = encode_tmap(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, fused, dims, strides, box,
                               CU_TENSOR_MAP_SWIZZLE_32B);
  if (s != TEMPO_OK) return s;
  PrefillParams p{};
  p.out = static_cast<uint16_t*>(fused);
  p.seqs = 1;
  p.tokens = tokens;
  p.heads = heads;
  p.q_tiles = (tokens + 127) / 128;
  p.block_bytes = block_bytes;
  if ((s = set_smem(reinterpret_cast<const void*>(attention_prefill_kernel<true>), kSmem))) return s;
  return launch(attention_prefill_kernel<true>, dim3(p.q_tiles * heads), dim3(kThreads), kSmem,
                static_cast<cudaStream_t>(stream), 1, "attention_prefill_kernel<packed>", map, p);
}

extern "C" tempo_status tempo_attention_prefill(const void* qkv, void* out, uint32_t seqs, uint32_t tokens,
                                                uint32_t heads, uint32_t head, void* stream) {
  if (seqs == 0 || tokens == 0 || heads == 0 || head != 64)
    return fail(TEMPO_ERR_VALUE, "tempo_attention_prefill: seqs %u tokens %u heads %u head %u (64)", seqs, tokens,
                heads, head);
  if (!aligned16(qkv) || !aligned16(out))
    return fail(TEMPO_ERR_VALUE, "tempo_attention_prefill: operands must be 16-byte aligned");
  CUtensorMap map;
  const uint64_t dims[2] = {3ull * heads * head, uint64_t(seqs) * tokens};
  const uint64_t strides[1] = {3ull * heads * head * 2};
  const uint32_t box[2] = {64, 128};
  tempo_status s = encode_tmap(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, qkv, dims, strides, box,
                               CU_TENSOR_MAP_SWIZZLE_128B);
  if (s != TEMPO_OK) return s;
  PrefillParams p{};
  p.out = static_cast<uint16_t*>(out);
  p.seqs = seqs;
  p.tokens = tokens;
  p.heads = heads;
  p.q_tiles = (tokens + 127) / 128;
  const uint64_t ctas = uint64_t(p.q_tiles) * heads * seqs;
  if (ctas > 0x7FFFFFFFull) return fail(TEMPO_ERR_VALUE, "tempo_attention_prefill: too many tiles");
  if ((s = set_smem(reinterpret_cast<const void*>(attention_prefill_kernel<false>), kSmem))) return s;
  return launch(attention_prefill_kernel<false>, dim3(uint32_t(ctas)), dim3(kThreads), kSmem,
                static_cast<cudaStream_t>(stream), 1, "attention_prefill_kernel<rowmajor>", map, p);
}
