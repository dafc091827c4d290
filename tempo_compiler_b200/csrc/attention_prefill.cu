// Causal prefill attention on the 5th-generation tensor cores (flash-attention tile loop over 128 queries of one head
// of one sequence at a time; persistent CTAs, two per SM, each walking a share of those items).
//
//   warp 0      TMA: Q once, then K and V 64 keys at a time into a four-stage ring.
//   warp 1      MMA issuer and TMEM owner. S = Q K^T goes into one of two 64-column TMEM buffers (FP32), so the
//               product of the next key tile runs while the softmax works on this one; after the softmax has written
//               P over its S, O += P V with P read straight from TMEM (A operand in tensor memory) and V from shared
//               memory. O stays in TMEM (64 columns) for the whole key loop.
//   warps 2-5   softmax, one query row per thread: read S, mask (tiles reaching past the tile's first query only),
//               the row maximum (three-input max instructions), exp2 on the special-function unit of scores scaled
//               and shifted two at a time (paired FP32), P as BF16 pairs into TMEM, the row sum in FP32 (paired
//               adds, in the same order as one key at a time). The exponent base
//               only moves when the row maximum grows by more than 2^8; only then are O and the sum rescaled (in
//               TMEM), which keeps the math exact while skipping almost every rescale. At the end O / sum is written.
//
// Two source layouts share the kernel:
//   PACKED    the drop-in fused QKV tensor, per 32-token block a 512-byte zero tile then [3*heads*4][32][16]
//             (attention, board_package/gpt2_inference.py:981-1003; tempo_ops.td:292-314). 4-D tensor maps
//             (16, 32 tokens, blocks, 16-wide feature tiles) load 4 (queries) or 2 (keys, values) blocks x 4 tiles,
//             which land as 128- or 64-row K-major 32-byte-swizzled tiles: exactly the MMA operand layout. The output
//             overwrites the queries.
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
constexpr uint32_t kKeys = 64;                        // keys per K/V tile (32 or 64)
constexpr int kCtasPerSm = kKeys == 32 ? 4 : 2;         // TMEM: 2 x kKeys (S, P) + 64 (O) columns per CTA
constexpr uint32_t kStages = 4;                       // K/V ring depth
constexpr uint32_t kQBytes = 128 * 64 * 2;            // one 128-query x 64-dim BF16 tile
constexpr uint32_t kKvTileBytes = kKeys * 64 * 2;     // one 64-key x 64-dim BF16 tile

struct PrefillParams {
  uint16_t* out;         // ROWMAJOR: [seqs*tokens, heads*64]; PACKED: the fused tensor (queries overwritten)
  uint32_t seqs, tokens, heads;
  uint32_t q_tiles;      // ceil(tokens / 128)
  uint64_t block_bytes;  // PACKED: bytes per 32-token block of the fused tensor
  uint32_t early;        // the grid fits in one wave: dependents may launch at entry
};

// Shared memory: Q[2] (the current and the next item's) | K[kStages] | V[kStages] | barriers.
constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffK = 2 * kQBytes;
constexpr uint32_t kOffV = kOffK + kStages * kKvTileBytes;
constexpr uint32_t kOffBar = kOffV + kStages * kKvTileBytes;
// q_full[2], kv_full[S], kv_empty[S], s_full[2], p_full[2], o_full, final, q_empty[2], o_done
constexpr uint32_t kBarCount = 2 + 2 * kStages + 2 + 2 + 1 + 1 + 2 + 1;
constexpr uint32_t kSmem = kOffBar + kBarCount * 8 + 16 + 1024;

// TMEM columns: S/P buffer 0 | S/P buffer 1 | O.
constexpr uint32_t kTmemS0 = 0, kTmemS1 = kKeys, kTmemO = 2 * kKeys, kTmemCols = kKeys == 32 ? 128 : 256;

template <bool PACKED>
__device__ __forceinline__ void load_tile(void* dst, const CUtensorMap* map, uint64_t* bar, uint32_t feature_tile16,
                                          int32_t row_or_block) {
  if constexpr (PACKED) {
    tma_load_4d(dst, map, bar, 0, 0, row_or_block, int32_t(feature_tile16));
  } else {
    tma_load_2d(dst, map, bar, int32_t(feature_tile16 * 16), row_or_block);
  }
}

// Descriptor of the kk-th 16-deep K-major slice of a `rows`-row operand tile.
template <bool PACKED>
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t tile_addr, uint32_t kk, uint32_t rows) {
  if constexpr (PACKED) return make_smem_desc(tile_addr + kk * rows * 32, 16, 256, kLayoutSw32);
  else return make_smem_desc(tile_addr + kk * 32, 16, 1024, kLayoutSw128);
}

// Descriptor of the kk-th 16-key slice of a 64-key V tile as the MN-major B operand (N = 64 head dims).
template <bool PACKED>
__device__ __forceinline__ uint64_t v_desc(uint32_t tile_addr, uint32_t kk) {
  if constexpr (PACKED) return make_smem_desc(tile_addr + kk * 512, kKeys * 32, 256, kLayoutSw32);
  else return make_smem_desc(tile_addr + kk * 2048, 8192, 1024, kLayoutSw128);
}

// One (query tile, head, sequence) of the grid's work. The CTAs are persistent (at most kCtasPerSm per SM, all
// resident at once): the items are ranked heaviest first (causal: query tile qt reads about 2(qt + 1) key tiles) and
// dealt to the CTAs in snake order (round k hands out ranks kG .. kG + G - 1, ascending in even rounds and
// descending in odd ones), which evens out the key tiles per CTA. A CTA's TMA, MMA and softmax roles walk the same
// sequence, so one item's Q and first keys load while the previous item's last tiles and output are finished.
struct PrefillItem {
  uint32_t qt, h, s, kv_tiles, first_masked;
};

__device__ __forceinline__ bool next_item(const PrefillParams& p, uint32_t k, PrefillItem& it) {
  const uint32_t grid = gridDim.x, cta = blockIdx.x;
  const uint64_t rank = uint64_t(k) * grid + ((k & 1u) ? grid - 1 - cta : cta);
  const uint32_t per_tile = p.heads * p.seqs;
  if (rank >= uint64_t(p.q_tiles) * per_tile) return false;
  const uint32_t r = uint32_t(rank), rem = r % per_tile;
  it.qt = p.q_tiles - 1 - r / per_tile;
  it.h = rem % p.heads;
  it.s = rem / p.heads;
  const uint32_t last_query = min(p.tokens, (it.qt + 1) * 128) - 1;
  it.kv_tiles = last_query / kKeys + 1;
  it.first_masked = (it.qt * 128) / kKeys;  // key tiles from here on reach past the tile's first query
  return true;
}

template <bool PACKED>
__global__ void __launch_bounds__(kThreads, kCtasPerSm)
    attention_prefill_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_kv,
                             PrefillParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 2;
  uint64_t* kv_empty = bars + 2 + kStages;
  uint64_t* s_full = bars + 2 + 2 * kStages;
  uint64_t* p_full = s_full + 2;
  uint64_t* o_full = p_full + 2;
  uint64_t* final_bar = o_full + 1;
  uint64_t* q_empty = final_bar + 1;  // [2]
  uint64_t* o_done = q_empty + 2;     // completes once per item, after its last P V
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kBarCount);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t warp = warp_id(), lane = lane_id();
  const uint32_t heads4 = p.heads * 4;  // 16-wide feature tiles per third of the fused tensor

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    for (uint32_t i = 0; i < kStages; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
    }
    mbar_init(o_full, 1);
    mbar_init(final_bar, 1);
    mbar_init(o_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmap_q);
    tma_prefetch_desc(&tmap_kv);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (p.early) pdl_launch_dependents();
  pdl_wait();  // Q, K and V are the previous kernel's output

  auto q_coord = [&](const PrefillItem& it) -> int32_t {
    if constexpr (PACKED) return int32_t(it.qt * 4);
    else return int32_t(it.s * p.tokens + it.qt * 128);
  };
  auto kv_coord = [&](const PrefillItem& it, uint32_t j) -> int32_t {
    if constexpr (PACKED) return int32_t(j * (kKeys / 32));
    else return int32_t(it.s * p.tokens + j * kKeys);
  };

  if (warp == 0) {
    if (elect_one()) {
      bool issued[kStages];
      uint32_t parity_of[kStages];
      for (uint32_t i = 0; i < kStages; ++i) { issued[i] = false; parity_of[i] = 0; }
      uint32_t g = 0, items = 0;  // key tiles and items this CTA has loaded
      bool ok = true;
      PrefillItem it;
      for (uint32_t k = 0; ok && next_item(p, k, it); ++k) {
        // Item k's Q buffer (k & 1) is free once every S of item k - 2 has completed.
        const uint32_t qb = k & 1u;
        if (!mbar_wait(&q_empty[qb], ((k >> 1) & 1u) ^ 1u, kWatchEmpty, abort_flag)) break;
        mbar_arrive_expect_tx(&q_full[qb], kQBytes);
        load_tile<PACKED>(smem + kOffQ + qb * kQBytes, &tmap_q, &q_full[qb], it.h * 4, q_coord(it));
        ++items;
        for (uint32_t j = 0; j < it.kv_tiles; ++j, ++g) {
          const uint32_t st = g % kStages, ph = (g / kStages) & 1u;
          if (!mbar_wait(&kv_empty[st], ph ^ 1u, kWatchEmpty, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&kv_full[st], 2 * kKvTileBytes);
          load_tile<PACKED>(smem + kOffK + st * kKvTileBytes, &tmap_kv, &kv_full[st], heads4 + it.h * 4,
                            kv_coord(it, j));
          load_tile<PACKED>(smem + kOffV + st * kKvTileBytes, &tmap_kv, &kv_full[st], 2 * heads4 + it.h * 4,
                            kv_coord(it, j));
          issued[st] = true;
          parity_of[st] = ph;
        }
      }
      // Every copy issued must have landed before the CTA may exit.
      for (uint32_t k = items > 2 ? items - 2 : 0; k < items; ++k)
        mbar_wait(&q_full[k & 1u], (k >> 1) & 1u, kWatchFull, nullptr);
      for (uint32_t i = 0; i < kStages; ++i)
        if (issued[i]) mbar_wait(&kv_full[i], parity_of[i], kWatchFull, nullptr);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc_s = make_idesc_bf16(128, kKeys, 0, 0);
      constexpr uint32_t idesc_o = make_idesc_bf16(128, 64, 0, 1);
      uint32_t q_addr = smem_u32(smem + kOffQ);
      // S_g = Q K_g^T (g counts this CTA's key tiles over all its items) into buffer g & 1. The buffer held
      // P_{g-2}, whose P V was issued before (the MMAs of one thread run in issue order).
      auto issue_s = [&](uint32_t g) -> bool {
        const uint32_t st = g % kStages;
        if (!mbar_wait(&kv_full[st], (g / kStages) & 1u, kWatchFull, abort_flag)) return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + kOffK + st * kKvTileBytes);
        const uint32_t d = tmem_base + ((g & 1u) ? kTmemS1 : kTmemS0);
#pragma unroll
        for (uint32_t kk = 0; kk < 4; ++kk)
          umma_bf16(d, kmajor_desc<PACKED>(q_addr, kk, 128), kmajor_desc<PACKED>(k_addr, kk, kKeys), idesc_s,
                    kk != 0);
        umma_commit(&s_full[g & 1u]);
        return true;
      };
      uint32_t g = 0;
      bool ok = true;
      PrefillItem it;
      for (uint32_t k = 0; ok && next_item(p, k, it); ++k) {
        q_addr = smem_u32(smem + kOffQ + (k & 1u) * kQBytes);
        ok = mbar_wait(&q_full[k & 1u], (k >> 1) & 1u, kWatchFull, abort_flag);
        if (ok) {
          tc_fence_after();
          ok = issue_s(g);
        }
        for (uint32_t j = 0; j < it.kv_tiles && ok; ++j, ++g) {
          if (j + 1 < it.kv_tiles) {
            if (!issue_s(g + 1)) { ok = false; break; }
          } else {
            umma_commit(&q_empty[k & 1u]);  // every S of this item is issued: its Q is free once they complete
          }
          // The item's first P V overwrites O: the softmax threads read the previous item's O before they
          // signalled this P.
          if (!mbar_wait(&p_full[g & 1u], (g >> 1) & 1u, kWatchOther, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t v_addr = smem_u32(smem + kOffV + (g % kStages) * kKvTileBytes);
          const uint32_t pa = tmem_base + ((g & 1u) ? kTmemS1 : kTmemS0);
#pragma unroll
          for (uint32_t kk = 0; kk < kKeys / 16; ++kk)
            umma_bf16_tmem_a(tmem_base + kTmemO, pa + kk * 8, v_desc<PACKED>(v_addr, kk), idesc_o, (j | kk) != 0u);
          umma_commit(o_full);
          if (j + 1 == it.kv_tiles) umma_commit(o_done);
          umma_commit(&kv_empty[g % kStages]);
        }
      }
      umma_commit(final_bar);
      mbar_wait(final_bar, 0, kWatchOther, nullptr);
    }
  } else {
    const uint32_t lane_base = 32u * (warp & 3u);
    const uint32_t row = lane_base + lane;
    const uint32_t lane_addr = lane_base << 16;
    const uint32_t tmem_o = tmem_base + kTmemO;
    uint32_t g = 0;  // this CTA's key tiles so far, over all its items
    bool ok = true;
    PrefillItem it;
    for (uint32_t k = 0; ok && next_item(p, k, it); ++k) {
      const uint32_t q_local = it.qt * 128 + row;  // query position in the sequence
      float m_used = -INFINITY, l = 0.f;  // m_used: raw-score units
      for (uint32_t j = 0; j < it.kv_tiles; ++j, ++g) {
        const uint32_t buf = tmem_base + ((g & 1u) ? kTmemS1 : kTmemS0);
        if (!mbar_wait(&s_full[g & 1u], (g >> 1) & 1u, kWatchOther, abort_flag)) { ok = false; break; }
        tc_fence_after();
        uint32_t sr[kKeys];
#pragma unroll
        for (uint32_t c32 = 0; c32 < kKeys / 32; ++c32)
          tmem_ld_32x32b_x32(buf + lane_addr + c32 * 32, *reinterpret_cast<uint32_t(*)[32]>(sr + c32 * 32));
        tmem_wait_ld();
        if (j >= it.first_masked) {
          // Keys past the query, and past the sequence end, are masked: key j * kKeys + c is kept while it is at
          // most min(query, tokens - 1), one compare with a constant per key.
          const int last = int(min(q_local, p.tokens - 1u)) - int(j * kKeys);
#pragma unroll
          for (uint32_t c = 0; c < kKeys; ++c)
            if (int(c) > last) sr[c] = __float_as_uint(-INFINITY);
        }
        // Eight independent partial maxima (short dependency chains) of three-input maxima, then combined: 32
        // instructions for 64 keys.
        static_assert(kKeys >= 24 && kKeys % 2 == 0, "the maximum tree takes 24 keys, then pairs");
        float mxs[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          mxs[i] = fmax3(__uint_as_float(sr[3 * i]), __uint_as_float(sr[3 * i + 1]), __uint_as_float(sr[3 * i + 2]));
#pragma unroll
        for (uint32_t c = 24; c < kKeys; c += 2)
          mxs[(c / 2) % 8] = fmax3(mxs[(c / 2) % 8], __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]));
        const float mx = fmax3(fmax3(mxs[0], mxs[1], mxs[2]), fmax3(mxs[3], mxs[4], mxs[5]), fmaxf(mxs[6], mxs[7]));
        bool rescale = false;
        float factor = 1.f;
        if (m_used == -INFINITY) {
          m_used = mx;
        } else if ((mx - m_used) * kLog2e > kRescaleThreshold) {
          factor = fast_exp2((m_used - mx) * kLog2e);
          m_used = mx;
          l *= factor;
          rescale = true;
        }
        const float base = m_used == -INFINITY ? 0.f : m_used * kLog2e;
        // Four independent partial sums, key pair i (keys 2i, 2i+1) into sum i % 4, held as two pairs (sums 0 and
        // 1, sums 2 and 3) so that paired FP32 instructions scale, shift and add two keys or two sums at once, each
        // half rounded as its scalar form: the same values as one key at a time, in half the FP32 issue slots.
        const uint64_t log2e2 = f2_splat(kLog2e), shift2 = f2_splat(-base);
        uint64_t sums[2] = {f2_splat(0.f), f2_splat(0.f)};
#pragma unroll
        for (int c16 = 0; c16 < int(kKeys / 32); ++c16) {
          uint32_t packed[16];
#pragma unroll
          for (int i = 0; i < 16; i += 2) {
            const uint32_t c = c16 * 32 + 2 * i;
            float a0, a1, b0, b1;
            f2_unpack(f2_fma(f2_pack(__uint_as_float(sr[c]), __uint_as_float(sr[c + 1])), log2e2, shift2), a0, a1);
            f2_unpack(f2_fma(f2_pack(__uint_as_float(sr[c + 2]), __uint_as_float(sr[c + 3])), log2e2, shift2), b0,
                      b1);
            const float ea0 = fast_exp2(a0), ea1 = fast_exp2(a1), eb0 = fast_exp2(b0), eb1 = fast_exp2(b1);
            packed[i] = pack_bf16x2(ea0, ea1);
            packed[i + 1] = pack_bf16x2(eb0, eb1);
            // (pair i's sum, pair i+1's sum) into (sum i % 4, sum (i+1) % 4)
            sums[(i / 2) % 2] = f2_add(sums[(i / 2) % 2], f2_add(f2_pack(ea0, eb0), f2_pack(ea1, eb1)));
          }
          tmem_st_32x32b_x16(buf + lane_addr + c16 * 16, packed);
        }
        float s0, s1, s2, s3;
        f2_unpack(sums[0], s0, s1);
        f2_unpack(sums[1], s2, s3);
        l += (s0 + s1) + (s2 + s3);
        // The rescale must wait for the previous P V (the only MMA writing O) to finish.
        const bool warp_rescale = __any_sync(0xFFFFFFFFu, rescale);
        if (warp_rescale) {
          if (!mbar_wait(o_full, (g - 1) & 1u, kWatchOther, abort_flag)) { ok = false; }
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
        mbar_arrive(&p_full[g & 1u]);
        if (!ok) break;
      }
      // The item's O is final once its last P V has completed. o_full cannot say so here: a softmax warp may finish
      // the last tile while another is still on the one before, so the next-to-last P V may not even be issued yet,
      // and a parity wait on o_full would then see the completed phase two steps back and return at once. o_done
      // completes once per item, after the MMA thread has issued the item's last P V (which needs every warp's P).
      if (ok && !mbar_wait(o_done, k & 1u, kWatchOther, abort_flag)) ok = false;
      if (ok) {
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
                                  size_t(it.h * 4 + 2 * half) * 1024 + (q_local & 31u) * 32;
              uint4* t0 = reinterpret_cast<uint4*>(base_ptr);
              uint4* t1 = reinterpret_cast<uint4*>(base_ptr + 1024);
              t0[0] = make_uint4(w[0], w[1], w[2], w[3]);
              t0[1] = make_uint4(w[4], w[5], w[6], w[7]);
              t1[0] = make_uint4(w[8], w[9], w[10], w[11]);
              t1[1] = make_uint4(w[12], w[13], w[14], w[15]);
            } else {
              uint4* dst = reinterpret_cast<uint4*>(p.out + (size_t(it.s) * p.tokens + q_local) * (p.heads * 64) +
                                                    it.h * 64 + half * 32);
              dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
              dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
              dst[2] = make_uint4(w[8], w[9], w[10], w[11]);
              dst[3] = make_uint4(w[12], w[13], w[14], w[15]);
            }
          }
        }
      }
    }
  }

  if (!p.early) pdl_launch_dependents();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace
}  // namespace tempo

using namespace tempo;

// Persistent CTAs: one per item up to kCtasPerSm per SM.
static uint32_t prefill_grid(uint64_t items) {
  const uint64_t slots = uint64_t(sm_count()) * kCtasPerSm;
  return uint32_t(items < slots ? items : slots);
}

extern "C" tempo_status tempo_block_attention(const void* constants, void* fused, uint32_t tokens, uint32_t heads,
                                              uint32_t head, void* stream) {
  (void)constants;  // the causal diagonal mask is computed in-kernel; the runtime validates the block's range
  if (tokens == 0 || tokens % 32 || heads == 0 || head != 64)
    return fail(TEMPO_ERR_VALUE, "tempo_block_attention: tokens %u (multiple of 32), heads %u, head %u (64)", tokens,
                heads, head);
  if (!aligned16(fused)) return fail(TEMPO_ERR_VALUE, "tempo_block_attention: fused tensor must be 16-byte aligned");
  const uint64_t block_bytes = 512 + 32ull * 3 * heads * head * 2;
  CUtensorMap map_q, map_kv;
  // The queries pointer is past block 0's zero tile; the maps address every block's tiles from there.
  const uint64_t dims[4] = {16, 32, tokens / 32, 3ull * heads * 4};
  const uint64_t strides[3] = {32, block_bytes, 1024};
  const uint32_t box_q[4] = {16, 32, 4, 4};
  const uint32_t box_kv[4] = {16, 32, kKeys / 32, 4};
  tempo_status s = encode_tmap(&map_q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, fused, dims, strides, box_q,
                               CU_TENSOR_MAP_SWIZZLE_32B);
  if (s != TEMPO_OK) return s;
  s = encode_tmap(&map_kv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, fused, dims, strides, box_kv,
                  CU_TENSOR_MAP_SWIZZLE_32B);
  if (s != TEMPO_OK) return s;
  PrefillParams p{};
  p.out = static_cast<uint16_t*>(fused);
  p.seqs = 1;
  p.tokens = tokens;
  p.heads = heads;
  p.q_tiles = (tokens + 127) / 128;
  p.block_bytes = block_bytes;
  p.early = 1;  // the persistent grid is resident at once
  if ((s = set_smem(reinterpret_cast<const void*>(attention_prefill_kernel<true>), kSmem))) return s;
  return launch(attention_prefill_kernel<true>, dim3(prefill_grid(uint64_t(p.q_tiles) * heads)), dim3(kThreads),
                kSmem, static_cast<cudaStream_t>(stream), 1, "attention_prefill_kernel<packed>", map_q, map_kv, p);
}

extern "C" tempo_status tempo_attention_prefill(const void* qkv, void* out, uint32_t seqs, uint32_t tokens,
                                                uint32_t heads, uint32_t head, void* stream) {
  if (seqs == 0 || tokens == 0 || heads == 0 || head != 64)
    return fail(TEMPO_ERR_VALUE, "tempo_attention_prefill: seqs %u tokens %u heads %u head %u (64)", seqs, tokens,
                heads, head);
  if (!aligned16(qkv) || !aligned16(out))
    return fail(TEMPO_ERR_VALUE, "tempo_attention_prefill: operands must be 16-byte aligned");
  CUtensorMap map_q, map_kv;
  const uint64_t dims[2] = {3ull * heads * head, uint64_t(seqs) * tokens};
  const uint64_t strides[1] = {3ull * heads * head * 2};
  const uint32_t box_q[2] = {64, 128};
  const uint32_t box_kv[2] = {64, kKeys};
  tempo_status s = encode_tmap(&map_q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, qkv, dims, strides, box_q,
                               CU_TENSOR_MAP_SWIZZLE_128B);
  if (s != TEMPO_OK) return s;
  s = encode_tmap(&map_kv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, qkv, dims, strides, box_kv,
                  CU_TENSOR_MAP_SWIZZLE_128B);
  if (s != TEMPO_OK) return s;
  PrefillParams p{};
  p.out = static_cast<uint16_t*>(out);
  p.seqs = seqs;
  p.tokens = tokens;
  p.heads = heads;
  p.q_tiles = (tokens + 127) / 128;
  const uint64_t items = uint64_t(p.q_tiles) * heads * seqs;
  if (items > 0x7FFFFFFFull) return fail(TEMPO_ERR_VALUE, "tempo_attention_prefill: too many tiles");
  p.early = 1;  // the persistent grid is resident at once
  if ((s = set_smem(reinterpret_cast<const void*>(attention_prefill_kernel<false>), kSmem))) return s;
  return launch(attention_prefill_kernel<false>, dim3(prefill_grid(items)), dim3(kThreads), kSmem,
                static_cast<cudaStream_t>(stream), 1, "attention_prefill_kernel<rowmajor>", map_q, map_kv, p);
}
