// Attention: causal prefill on the 5th-generation tensor cores, and the bandwidth-bound decode step.
//
// Prefill (attention_prefill_kernel) is a flash-attention tile loop for 128 queries of one head: TMA brings Q once
// and K/V 128 keys at a time (double-buffered); S = Q K^T is a tcgen05.mma into TMEM; four warps (one query row
// per thread) read S back, apply the causal mask and an online softmax in FP32, write P (BF16) into shared memory in
// the 128B-swizzled K-major layout; O_tile = P V is a second tcgen05.mma into TMEM, folded into per-thread FP32
// accumulators with the softmax rescale. Two source layouts share the kernel:
//   * PACKED: the drop-in fused QKV tensor, per 32-token block a 512-byte zero tile then [3*heads*4][32][16]
//     (attention, board_package/gpt2_inference.py:981-1003; tempo_ops.td:292-314). A 4-D tensor map with dims
//     (16, 32 tokens, blocks, 16-wide feature tiles) loads 4 blocks x 4 tiles, which lands in shared memory as four
//     128-row K-major 32-byte-swizzled tiles: exactly the MMA operand layout. The output overwrites the queries.
//   * ROWMAJOR: the native engine's qkv [seqs*tokens, 3*heads*64], 128-byte swizzle, output to a separate buffer.
// The queries arrive scaled by 1/sqrt(head) (folded into the QKV weights, gpt2_inference.py:1153-1168).
//
// Decode kernels read each cached key and value once with 16-byte loads (8 lanes per key), keep an online softmax
// per lane group and merge groups and warps at the end.
#include <cuda.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "host.hpp"

namespace tempo {

TEMPO_WATCHDOG_READER(watchdog_attention)

namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr int kAttnThreads = 192;
constexpr uint32_t kTileBytes = 128 * 64 * 2;  // one 128 x 64 BF16 operand tile

struct PrefillParams {
  uint16_t* out;           // ROWMAJOR: [seqs*tokens, heads*64]; PACKED: the fused tensor (queries overwritten)
  uint32_t seqs, tokens, heads;
  uint32_t q_tiles;        // ceil(tokens / 128)
  uint64_t block_bytes;    // PACKED: bytes per 32-token block of the fused tensor
};

// Shared memory: Q | K[2] | V[2] | P (2 x 16 KB halves) | barriers.
constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffK = kTileBytes;
constexpr uint32_t kOffV = 3 * kTileBytes;
constexpr uint32_t kOffP = 5 * kTileBytes;
constexpr uint32_t kOffBar = 7 * kTileBytes;
// q_full, kv_full[2], kv_empty[2], s_full, s_free, p_full, o_full, o_free, final
constexpr uint32_t kBarCount = 11;
constexpr uint32_t kPrefillSmem = kOffBar + kBarCount * 8 + 16 + 1024;

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
__global__ void __launch_bounds__(kAttnThreads, 1)
    attention_prefill_kernel(const __grid_constant__ CUtensorMap tmap, PrefillParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = bars + 3;
  uint64_t* s_full = bars + 5;
  uint64_t* s_free = bars + 6;
  uint64_t* p_full = bars + 7;
  uint64_t* o_full = bars + 8;
  uint64_t* o_free = bars + 9;
  uint64_t* final_bar = bars + 10;
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
    mbar_init(s_free, 128);
    mbar_init(p_full, 128);
    mbar_init(o_full, 1);
    mbar_init(o_free, 128);
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
  const uint32_t tmem_s = tmem_base;        // 128 columns: S
  const uint32_t tmem_o = tmem_base + 128;  // 64 columns: O tile

  // Row (packed: block) coordinate of query/key tile `t` of this sequence.
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
      const uint32_t p_addr = smem_u32(smem + kOffP);
      bool ok = mbar_wait(q_full, 0, kWatchFull, abort_flag);
      for (uint32_t j = 0; j < kv_tiles && ok; ++j) {
        const uint32_t st = j & 1u, ph = (j >> 1) & 1u;
        if (!mbar_wait(&kv_full[st], ph, kWatchFull, abort_flag)) break;
        if (j > 0 && !mbar_wait(s_free, (j - 1) & 1u, kWatchOther, abort_flag)) break;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + kOffK + st * kTileBytes);
        const uint32_t v_addr = smem_u32(smem + kOffV + st * kTileBytes);
#pragma unroll
        for (uint32_t kk = 0; kk < 4; ++kk)
          umma_bf16(tmem_s, kmajor_desc<PACKED>(q_addr, kk), kmajor_desc<PACKED>(k_addr, kk), idesc_s, kk != 0);
        umma_commit(s_full);
        if (!mbar_wait(p_full, j & 1u, kWatchOther, abort_flag)) break;
        if (j > 0 && !mbar_wait(o_free, (j - 1) & 1u, kWatchOther, abort_flag)) break;
        tc_fence_after();
#pragma unroll
        for (uint32_t kk = 0; kk < 8; ++kk) {
          const uint64_t a = make_smem_desc(p_addr + (kk >> 2) * 16384 + (kk & 3u) * 32, 16, 1024, kLayoutSw128);
          umma_bf16(tmem_o, a, v_desc<PACKED>(v_addr, kk), idesc_o, kk != 0);
        }
        umma_commit(o_full);
        umma_commit(&kv_empty[st]);
      }
      umma_commit(final_bar);
      mbar_wait(final_bar, 0, kWatchOther, nullptr);
    }
  } else {
    // Softmax / correction / output: thread = query row (TMEM lane).
    const uint32_t lane_base = 32u * (warp & 3u);
    const uint32_t row = lane_base + lane;
    const uint32_t q_local = qt * 128 + row;  // query position in the sequence
    const uint32_t lane_addr = lane_base << 16;
    uint8_t* p_row = smem + kOffP + row * 128;
    float o[64];
#pragma unroll
    for (int d = 0; d < 64; ++d) o[d] = 0.f;
    float m = -INFINITY, l = 0.f, alpha_prev = 1.f;
    bool ok = true;
    for (uint32_t j = 0; j < kv_tiles && ok; ++j) {
      // Fold the previous tile's P V into the accumulators (in units of the previous maximum). PV(j-1) was issued
      // before S(j), so this wait costs nothing; it also frees P for this tile.
      if (j > 0) {
        if (!mbar_wait(o_full, (j - 1) & 1u, kWatchOther, abort_flag)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t orr[32];
          tmem_ld_32x32b_x32(tmem_o + lane_addr + half * 32, orr);
          tmem_wait_ld();
#pragma unroll
          for (int d = 0; d < 32; ++d) o[half * 32 + d] = o[half * 32 + d] * alpha_prev + __uint_as_float(orr[d]);
        }
        tc_fence_before();
        mbar_arrive(o_free);
      }
      if (!mbar_wait(s_full, j & 1u, kWatchOther, abort_flag)) { ok = false; break; }
      tc_fence_after();
      uint32_t sr[128];
      tmem_ld_32x32b_x32(tmem_s + lane_addr + 0, *reinterpret_cast<uint32_t(*)[32]>(sr + 0));
      tmem_ld_32x32b_x32(tmem_s + lane_addr + 32, *reinterpret_cast<uint32_t(*)[32]>(sr + 32));
      tmem_ld_32x32b_x32(tmem_s + lane_addr + 64, *reinterpret_cast<uint32_t(*)[32]>(sr + 64));
      tmem_ld_32x32b_x32(tmem_s + lane_addr + 96, *reinterpret_cast<uint32_t(*)[32]>(sr + 96));
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(s_free);
      // Causal and sequence-end mask, scores to the log2 domain, row maximum.
      const uint32_t key0 = j * 128;
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 128; ++c) {
        const uint32_t key = key0 + c;
        float v = __uint_as_float(sr[c]) * kLog2e;
        if (key > q_local || key >= p.tokens) v = -INFINITY;
        sr[c] = __float_as_uint(v);
        mx = fmaxf(mx, v);
      }
      const float m_new = fmaxf(m, mx);
      const float base = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = exp2f(m - base);
      float sum = 0.f;
      // P = exp2(S - m) in BF16, written 8 keys (16 bytes) at a time into the swizzled K-major layout.
#pragma unroll
      for (int c8 = 0; c8 < 16; ++c8) {
        float e[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          e[i] = exp2f(__uint_as_float(sr[c8 * 8 + i]) - base);
          sum += e[i];
        }
        uint4 w;
        w.x = pack_bf16x2(e[0], e[1]);
        w.y = pack_bf16x2(e[2], e[3]);
        w.z = pack_bf16x2(e[4], e[5]);
        w.w = pack_bf16x2(e[6], e[7]);
        const uint32_t half = c8 >> 3, chunk = c8 & 7u;
        *reinterpret_cast<uint4*>(p_row + half * 16384 + ((chunk ^ (row & 7u)) * 16)) = w;
      }
      fence_proxy_async_smem();
      mbar_arrive(p_full);
      l = l * alpha + sum;
      m = m_new;
      alpha_prev = alpha;
    }
    if (ok && mbar_wait(o_full, (kv_tiles - 1) & 1u, kWatchOther, abort_flag)) {
      tc_fence_after();
      uint32_t orr[64];
      tmem_ld_32x32b_x32(tmem_o + lane_addr + 0, *reinterpret_cast<uint32_t(*)[32]>(orr + 0));
      tmem_ld_32x32b_x32(tmem_o + lane_addr + 32, *reinterpret_cast<uint32_t(*)[32]>(orr + 32));
      tmem_wait_ld();
      const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
      for (int d = 0; d < 64; ++d) o[d] = (o[d] * alpha_prev + __uint_as_float(orr[d])) * inv;
      if (q_local < p.tokens) {
        if constexpr (PACKED) {
          uint8_t* base_ptr = reinterpret_cast<uint8_t*>(p.out) + size_t(q_local >> 5) * p.block_bytes +
                              size_t(h * 4) * 1024 + (q_local & 31u) * 32;
#pragma unroll
          for (int f = 0; f < 4; ++f) {
            uint4 w0, w1;
            w0.x = pack_bf16x2(o[f * 16 + 0], o[f * 16 + 1]);
            w0.y = pack_bf16x2(o[f * 16 + 2], o[f * 16 + 3]);
            w0.z = pack_bf16x2(o[f * 16 + 4], o[f * 16 + 5]);
            w0.w = pack_bf16x2(o[f * 16 + 6], o[f * 16 + 7]);
            w1.x = pack_bf16x2(o[f * 16 + 8], o[f * 16 + 9]);
            w1.y = pack_bf16x2(o[f * 16 + 10], o[f * 16 + 11]);
            w1.z = pack_bf16x2(o[f * 16 + 12], o[f * 16 + 13]);
            w1.w = pack_bf16x2(o[f * 16 + 14], o[f * 16 + 15]);
            uint4* dst = reinterpret_cast<uint4*>(base_ptr + f * 1024);
            dst[0] = w0;
            dst[1] = w1;
          }
        } else {
          uint4* dst = reinterpret_cast<uint4*>(p.out + (size_t(s) * p.tokens + q_local) * (p.heads * 64) + h * 64);
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            uint4 w;
            w.x = pack_bf16x2(o[c * 8 + 0], o[c * 8 + 1]);
            w.y = pack_bf16x2(o[c * 8 + 2], o[c * 8 + 3]);
            w.z = pack_bf16x2(o[c * 8 + 4], o[c * 8 + 5]);
            w.w = pack_bf16x2(o[c * 8 + 6], o[c * 8 + 7]);
            dst[c] = w;
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

// ---------------------------------------------------------------------------------------------------------------
// Decode
// ---------------------------------------------------------------------------------------------------------------

__device__ __forceinline__ void load8(const uint4& w, float (&f)[8]) {
  f[0] = bf16_lo(w.x); f[1] = bf16_hi(w.x); f[2] = bf16_lo(w.y); f[3] = bf16_hi(w.y);
  f[4] = bf16_lo(w.z); f[5] = bf16_hi(w.z); f[6] = bf16_lo(w.w); f[7] = bf16_hi(w.w);
}

// Online-softmax state of one lane group (8 lanes x 8 dims = one head).
struct DecodeState {
  float m, l, acc[8];
};

// Folds four keys (scores already in the log2 domain, -inf when absent) into the state.
__device__ __forceinline__ void fold4(DecodeState& st, const float (&sc)[4], const uint4 (&vv)[4]) {
  const float mb = fmaxf(fmaxf(sc[0], sc[1]), fmaxf(sc[2], sc[3]));
  const float m_new = fmaxf(st.m, mb);
  if (m_new == -INFINITY) return;
  const float corr = exp2f(st.m - m_new);
  float pr[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) pr[i] = exp2f(sc[i] - m_new);
  st.l = st.l * corr + (pr[0] + pr[1]) + (pr[2] + pr[3]);
#pragma unroll
  for (int d = 0; d < 8; ++d) st.acc[d] *= corr;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float v[8];
    load8(vv[i], v);
#pragma unroll
    for (int d = 0; d < 8; ++d) st.acc[d] = fmaf(pr[i], v[d], st.acc[d]);
  }
  st.m = m_new;
}

// Merges the state of lane groups `other` lanes apart (xor shuffle).
__device__ __forceinline__ void merge_shfl(DecodeState& st, int offset) {
  const float om = __shfl_xor_sync(0xFFFFFFFFu, st.m, offset);
  const float ol = __shfl_xor_sync(0xFFFFFFFFu, st.l, offset);
  float oa[8];
#pragma unroll
  for (int d = 0; d < 8; ++d) oa[d] = __shfl_xor_sync(0xFFFFFFFFu, st.acc[d], offset);
  const float m_new = fmaxf(st.m, om);
  if (m_new == -INFINITY) return;
  const float a = exp2f(st.m - m_new), b = exp2f(om - m_new);
  st.l = st.l * a + ol * b;
#pragma unroll
  for (int d = 0; d < 8; ++d) st.acc[d] = st.acc[d] * a + oa[d] * b;
  st.m = m_new;
}

__device__ __forceinline__ float group_dot(const float (&q)[8], const uint4& k) {
  float kf[8];
  load8(k, kf);
  float s = 0.f;
#pragma unroll
  for (int d = 0; d < 8; ++d) s = fmaf(q[d], kf[d], s);
  s += __shfl_xor_sync(0xFFFFFFFFu, s, 1);
  s += __shfl_xor_sync(0xFFFFFFFFu, s, 2);
  s += __shfl_xor_sync(0xFFFFFFFFu, s, 4);
  return s;
}

// Native decode: one CTA (4 warps) per (head, sequence); caches [seq][head][capacity][64].
__global__ void __launch_bounds__(128) decode_attention_kernel(const uint16_t* __restrict__ qkv,
                                                               const uint16_t* __restrict__ k_cache,
                                                               const uint16_t* __restrict__ v_cache,
                                                               const int32_t* __restrict__ lengths,
                                                               int32_t length_offset, uint16_t* __restrict__ out,
                                                               uint32_t heads, uint32_t capacity) {
  const uint32_t h = blockIdx.x, s = blockIdx.y;
  const uint32_t warp = warp_id(), lane = lane_id();
  const uint32_t g = lane >> 3, li = lane & 7u;
  const uint32_t width = heads * 64;
  const int32_t len = max(0, min(lengths[s] + length_offset, int32_t(capacity)));
  float q[8];
  load8(reinterpret_cast<const uint4*>(qkv + size_t(s) * 3 * width + h * 64)[li], q);
#pragma unroll
  for (int d = 0; d < 8; ++d) q[d] *= kLog2e;
  const uint4* kb4 = reinterpret_cast<const uint4*>(k_cache + (size_t(s) * heads + h) * capacity * 64);
  const uint4* vb4 = reinterpret_cast<const uint4*>(v_cache + (size_t(s) * heads + h) * capacity * 64);
  DecodeState st;
  st.m = -INFINITY;
  st.l = 0.f;
#pragma unroll
  for (int d = 0; d < 8; ++d) st.acc[d] = 0.f;
  for (int32_t base = int32_t(warp) * 16; base < len; base += 64) {
    uint4 kk[4], vv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int32_t key = base + i * 4 + int32_t(g);
      if (key < len) {
        kk[i] = __ldg(kb4 + size_t(key) * 8 + li);
        vv[i] = __ldg(vb4 + size_t(key) * 8 + li);
      } else {
        kk[i] = make_uint4(0, 0, 0, 0);
        vv[i] = make_uint4(0, 0, 0, 0);
      }
    }
    float sc[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float v = group_dot(q, kk[i]);
      sc[i] = (base + i * 4 + int32_t(g) < len) ? v : -INFINITY;
    }
    fold4(st, sc, vv);
  }
  merge_shfl(st, 8);
  merge_shfl(st, 16);
  __shared__ float sm_m[4], sm_l[4], sm_acc[4][64];
  if (g == 0) {
#pragma unroll
    for (int d = 0; d < 8; ++d) sm_acc[warp][li * 8 + d] = st.acc[d];
    if (li == 0) { sm_m[warp] = st.m; sm_l[warp] = st.l; }
  }
  __syncthreads();
  if (threadIdx.x < 64) {
    const uint32_t d = threadIdx.x;
    float m = -INFINITY;
    for (int w = 0; w < 4; ++w) m = fmaxf(m, sm_m[w]);
    float l = 0.f, a = 0.f;
    if (m != -INFINITY) {
      for (int w = 0; w < 4; ++w) {
        const float f = exp2f(sm_m[w] - m);
        l += sm_l[w] * f;
        a += sm_acc[w][d] * f;
      }
    }
    out[size_t(s) * width + h * 64 + d] = float_to_bf16(l > 0.f ? a / l : 0.f);
  }
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
    fold4(st, sc, vv);
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

extern "C" tempo_status tempo_block_attention(const void* constants, void* fused, uint32_t tokens, uint32_t heads,
                                              uint32_t head, void* stream) {
  (void)constants;  // the causal diagonal mask is computed in-kernel; the block is validated by the caller
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
  if ((s = set_smem(reinterpret_cast<const void*>(attention_prefill_kernel<true>), kPrefillSmem))) return s;
  attention_prefill_kernel<true><<<p.q_tiles * heads, kAttnThreads, kPrefillSmem, static_cast<cudaStream_t>(stream)>>>(
      map, p);
  return check_launch("attention_prefill_kernel<packed>");
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
  if ((s = set_smem(reinterpret_cast<const void*>(attention_prefill_kernel<false>), kPrefillSmem))) return s;
  attention_prefill_kernel<false><<<uint32_t(ctas), kAttnThreads, kPrefillSmem, static_cast<cudaStream_t>(stream)>>>(
      map, p);
  return check_launch("attention_prefill_kernel<rowmajor>");
}

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
  if (seqs == 0 || heads == 0 || head != 64 || capacity == 0)
    return fail(TEMPO_ERR_VALUE, "tempo_decode_attention: seqs %u heads %u head %u capacity %u", seqs, heads, head,
                capacity);
  if (!aligned16(qkv) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(out))
    return fail(TEMPO_ERR_VALUE, "tempo_decode_attention: operands must be 16-byte aligned");
  decode_attention_kernel<<<dim3(heads, seqs), 128, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(qkv), static_cast<const uint16_t*>(k_cache), static_cast<const uint16_t*>(v_cache),
      lengths, length_offset, static_cast<uint16_t*>(out), heads, capacity);
  return check_launch("decode_attention_kernel");
}
