// BF16 GEMMs on the 5th-generation tensor cores: TMA-fed, tcgen05.mma into TMEM accumulators, FP32 accumulate.
//
// Two kernels share the same warp-specialised pipeline (warp 0: TMA producer, warp 1: MMA issuer and TMEM owner, the
// rest epilogue: warps 2-9 in the row-major kernel, two per TMEM lane quarter; warps 2-5 in the block kernel):
//
//  * gemm_rowmajor_kernel -- the native engine's GEMM, out[M,N] = A[M,K] x W^T[N,K]^T, 128 x BN tiles, 64-deep
//    stages in the 128-byte swizzled K-major layout, a persistent tile loop and a double-buffered accumulator so the
//    epilogue of one tile overlaps the MMAs of the next. Epilogue: + bias, exact-erf GELU, + residual, BF16 store;
//    or a fused argmax over the tile for the LM head.
//
//  * gemm_block_kernel -- one 32-token block on the packed drop-in layouts (gemm_resident,
//    board_package/gpt2_inference.py:574-640; tile op mlir/include/tempo/tempo/tempo_ops.td:228-252). The weights'
//    16-column tiles ([columns/16][depth][16]) are the MMA's M side in the MN-major 32-byte swizzled layout and the
//    block's 16-deep activation tiles ([depth/16][32][16]) its N side in the K-major 32-byte swizzled layout, so both
//    operands stream straight from the packed tensors by TMA with no repacking (UMMA 128 x 32 x 16). With
//    `activate`, the epilogue warps pass each staged activation tile through the exact-erf GELU in shared memory
//    before the MMA reads it (the reference applies its GELU while staging, tile_to_vector.cpp:239-256).
#include <cuda.h>
#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"
#include "host.hpp"

namespace tempo {

TEMPO_WATCHDOG_READER(watchdog_gemm)

// gemv.cu: the bandwidth-bound path for at most 8 rows (TEMPO_ERR_VALUE when it does not apply), optionally
// normalising its input rows first (LayerNorm with gamma, beta, epsilon; K <= 1024).
tempo_status gemv_dispatch(const void* a, uint32_t lda, const void* w_t, uint32_t ldw, const void* bias,
                           const void* residual, uint32_t ldr, void* out, uint32_t ldo, uint32_t m, uint32_t n,
                           uint32_t k, uint32_t flags, float* part_val, int32_t* part_idx, const KvStore& kv,
                           cudaStream_t stream, const uint16_t* ln_gamma = nullptr, const uint16_t* ln_beta = nullptr,
                           float ln_eps = 0.f);

namespace {

constexpr int kThreads = 192;  // 6 warps
constexpr int kBK = 64;        // 64 BF16 = 128 bytes: one 128B-swizzle atom row

struct RowMajorParams {
  const uint16_t* bias;
  const uint16_t* residual;
  uint16_t* out;
  float* part_val;
  int32_t* part_idx;
  uint32_t m, n, k;
  uint32_t ldo, ldr;
  uint32_t flags;
  uint32_t m_tiles, n_tiles;
  uint32_t stages;  // split-K: shared-memory ring depth actually used (<= the template's STAGES)
  uint32_t stage_tx;  // bytes one stage's TMA loads deliver: the A box rows (64 when M <= 64) plus the B tile
  // TEMPO_GEMM_LN: the A operand is the raw rows x; the preceding LayerNorm is folded into the weights (gamma x W),
  // out = rstd (acc - mean colsum[n]) + ln_bias[n] with FP32 colsum / ln_bias, row statistics computed in-kernel.
  const uint16_t* ln_x;
  uint32_t ln_ldx;
  const float* ln_colsum;
  const float* ln_bias;
  float ln_eps;
  // TEMPO_GEMM_LN with ln_stats: the rows' statistics come as partials from the kernel that wrote x (below) instead
  // of being computed from the A stages.
  const float2* ln_stats;
  // row_stats: the output rows' statistics partials, (mean, M2) of each 16-column chunk of the BF16-rounded outputs,
  // row_stats[row * n / 16 + chunk]: what a folded LayerNorm after this projection needs.
  float2* row_stats;
  KvStore kv;  // QKV projection: key and value columns also stored into the caches
};

template <int BN, int STAGES, bool STAGED = false>
struct RowMajorSmem {
  static constexpr uint32_t kABytes = 128 * kBK * 2;
  static constexpr uint32_t kBBytes = BN * kBK * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  // STAGED: one 32 x 32 BF16 staging tile (2 KB) per epilogue warp for TMA stores of the output.
  static constexpr uint32_t kStagingOffset = STAGES * kStageBytes;
  static constexpr uint32_t kStagingBytes = STAGED ? 16u * 2048u : 0u;
  static constexpr uint32_t kBarrierOffset = kStagingOffset + kStagingBytes;
  // full[S], empty[S], acc_full[2], acc_empty[2], final, epilogue-wide (row statistics)
  static constexpr uint32_t kBarriers = 2 * STAGES + 6;
  static constexpr uint32_t kExchangeOffset = kBarrierOffset + kBarriers * 8 + 16;  // after tmem slot and abort flag
  // argmax mode: one column group's best value and index per tile row, handed to the next lower group
  static constexpr uint32_t kBytes = kExchangeOffset + 128 * 8 + 1024;  // + alignment slack
  // At most 195 KB: the 196 KB carveout, leaving L1 to the kernels that overlap this one on the SM.
  static_assert(kBytes <= 195 * 1024, "row-major GEMM shared memory exceeds the 196 KB carveout");
};

// Warp roles of the row-major kernel: 0 TMA, 1 MMA, 2..17 epilogue. Epilogue warp w reads TMEM lane quarter w % 4
// (the quarter a warp may access) and column quarter (w - 2) / 4 of each tile, so four warps share every row and
// the bias / GELU / store work of a 128 x BN tile is spread over 512 threads.
constexpr uint32_t kRowEpiGroups = 4;
constexpr int kRowEpiThreads = 128 * kRowEpiGroups;
constexpr int kRowThreads = 64 + kRowEpiThreads;
// The split-K kernel keeps 0 TMA, 1 MMA, 2..9 epilogue (two CTAs may share an SM).
constexpr int kSplitThreads = 320;
constexpr int kEpilogueThreads = 256;

// A 2-D tile from this CTA's shared memory to global memory (bulk-group completion).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int32_t c0, int32_t c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
               ::"l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(src)), "r"(c0), "r"(c1)
               : "memory");
}

// One thread's kCW accumulator columns n0 .. n0 + kCW - 1 of output row `row`: the folded LayerNorm (mean / rstd of the
// row), bias, exact-erf GELU of the BF16-rounded sum, residual, BF16 stores into the output and, for the QKV
// projection, into the key / value caches.
// With kStaged the BF16 row segment goes into `stage_row` (16-byte words XOR-swizzled by `swizzle`) for a TMA store
// the caller issues; the key / value cache store stays direct.
template <uint32_t kCW, bool kStaged = false>
__device__ __forceinline__ void epilogue_chunk(const RowMajorParams& p, const uint32_t (&r)[kCW], uint32_t row,
                                               uint32_t n0, bool gelu, bool ln, float mu, float rs,
                                               uint8_t* stage_row = nullptr, uint32_t swizzle = 0) {
  if (kStaged && row >= p.m) {
    // A row past M in a staged block: the copy clips it; read nothing for it.
#pragma unroll
    for (uint32_t q = 0; q < kCW / 8; ++q) reinterpret_cast<uint4*>(stage_row)[q ^ swizzle] = make_uint4(0, 0, 0, 0);
    return;
  }
  float v[kCW];
#pragma unroll
  for (uint32_t j = 0; j < kCW; ++j) v[j] = __uint_as_float(r[j]);
  const bool full_chunk = n0 + kCW <= p.n;
  if (ln) {
    // LayerNorm folded into the weights: rstd (x (gamma W) - mean colsum) + (beta W + b).
    for (uint32_t j = 0; j < kCW; ++j) {
      const uint32_t col = n0 + j < p.n ? n0 + j : p.n - 1;
      v[j] = fmaf(rs, fmaf(-mu, __ldg(p.ln_colsum + col), v[j]), __ldg(p.ln_bias + col));
    }
  }
  if (p.bias != nullptr) {
    if (full_chunk) {
      const uint4* b4 = reinterpret_cast<const uint4*>(p.bias + n0);
#pragma unroll
      for (uint32_t q = 0; q < kCW / 8; ++q) {
        const uint4 w = __ldg(b4 + q);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          v[q * 8 + 2 * h] += bf16_lo(ws[h]);
          v[q * 8 + 2 * h + 1] += bf16_hi(ws[h]);
        }
      }
    } else {
      for (uint32_t j = 0; j < kCW; ++j)
        if (n0 + j < p.n) v[j] += bf16_to_float(p.bias[n0 + j]);
    }
  }
  if (gelu) {
#pragma unroll
    for (uint32_t j = 0; j < kCW; j += 2) {
      const uint32_t rounded = pack_bf16x2(v[j], v[j + 1]);  // one conversion rounds both
      v[j] = bf16_lo(rounded);
      v[j + 1] = bf16_hi(rounded);
      gelu_erf_pair(v[j], v[j + 1]);
    }
  }
  uint16_t* orow = p.out + size_t(row) * p.ldo;
  if (p.residual != nullptr) {
    const uint16_t* rrow = p.residual + size_t(row) * p.ldr;
    if (full_chunk) {
      const uint4* r4 = reinterpret_cast<const uint4*>(rrow + n0);
#pragma unroll
      for (uint32_t q = 0; q < kCW / 8; ++q) {
        const uint4 w = r4[q];
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          v[q * 8 + 2 * h] += bf16_lo(ws[h]);
          v[q * 8 + 2 * h + 1] += bf16_hi(ws[h]);
        }
      }
    } else {
      for (uint32_t j = 0; j < kCW; ++j)
        if (n0 + j < p.n) v[j] += bf16_to_float(rrow[n0 + j]);
    }
  }
  if (kStaged || full_chunk) {
    uint4 pk[kCW / 8];
#pragma unroll
    for (uint32_t q = 0; q < kCW / 8; ++q) {
      pk[q].x = pack_bf16x2(v[q * 8 + 0], v[q * 8 + 1]);
      pk[q].y = pack_bf16x2(v[q * 8 + 2], v[q * 8 + 3]);
      pk[q].z = pack_bf16x2(v[q * 8 + 4], v[q * 8 + 5]);
      pk[q].w = pack_bf16x2(v[q * 8 + 6], v[q * 8 + 7]);
    }
    uint4* cache4 = full_chunk ? reinterpret_cast<uint4*>(kv_destination(p.kv, row, n0)) : nullptr;
    uint4* o4 = reinterpret_cast<uint4*>(orow + n0);
#pragma unroll
    for (uint32_t q = 0; q < kCW / 8; ++q) {
      if (kStaged) {
        reinterpret_cast<uint4*>(stage_row)[q ^ swizzle] = pk[q];
      } else {
        o4[q] = pk[q];
      }
      if (cache4 != nullptr) cache4[q] = pk[q];
    }
    // The statistics of each whole 16-column chunk of what was stored (the host guarantees N % 16 == 0).
    if (p.row_stats != nullptr) {
#pragma unroll
      for (uint32_t c = 0; c < kCW / 16; ++c) {
        if (n0 + 16 * (c + 1) > p.n) break;
        float lo[8], hi[8], w[16];
        unpack8(pk[2 * c], lo);
        unpack8(pk[2 * c + 1], hi);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          w[j] = lo[j];
          w[8 + j] = hi[j];
        }
        p.row_stats[size_t(row) * (p.n / 16) + n0 / 16 + c] = chunk_stats16(w);
      }
    }
  } else {
    for (uint32_t j = 0; j < kCW; ++j)
      if (n0 + j < p.n) orow[n0 + j] = float_to_bf16(v[j]);
    // A 32-column chunk whose second half lies past N: the first half's statistics.
    if (p.row_stats != nullptr && kCW == 32 && n0 + 16 <= p.n) {
      float w[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) w[j] = bf16_to_float(float_to_bf16(v[j]));
      p.row_stats[size_t(row) * (p.n / 16) + n0 / 16] = chunk_stats16(w);
    }
  }
}

// The mean and 1 / sqrt(variance + eps) of rows row0 .. row0 + nrows - 1 (nrows <= 8) from their (mean, M2) partials
// of 16 columns each (`chunks` <= 64 per row, written by the kernel that produced the rows), by one warp: every
// partial is loaded first (lane l takes chunks l and l + 32 of each row), then per row the mean of the chunk means
// and M2 = sum M2_c + 16 sum (mean_c - mean)^2, each summed by a fixed shuffle tree, the eight rows' trees side by
// side. Lane i writes mean_out[i] and rstd_out[i] for row row0 + i. Inlined: measured 0.15-0.2 us faster per
// projection than out of line (whose call saves and restores the epilogue's live registers).
__device__ __forceinline__ void combine_row_stats_warp(const float2* stats, uint32_t chunks, uint32_t row0,
                                                    uint32_t nrows, float eps, float* mean_out, float* rstd_out,
                                                    uint32_t lane) {
  float2 lo[8], hi[8];
#pragma unroll
  for (uint32_t i = 0; i < 8; ++i) {
    const float2* row = stats + size_t(row0 + i) * chunks;
    lo[i] = i < nrows && lane < chunks ? __ldcg(row + lane) : make_float2(0.f, 0.f);
    hi[i] = i < nrows && lane + 32 < chunks ? __ldcg(row + lane + 32) : make_float2(0.f, 0.f);
  }
  const float inv_chunks = 1.f / float(chunks);
  float mean[8], m2[8];
#pragma unroll
  for (uint32_t i = 0; i < 8; ++i) mean[i] = lo[i].x + hi[i].x;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (uint32_t i = 0; i < 8; ++i) mean[i] += __shfl_xor_sync(0xFFFFFFFFu, mean[i], o);
#pragma unroll
  for (uint32_t i = 0; i < 8; ++i) {
    mean[i] *= inv_chunks;
    const float dl = lo[i].x - mean[i], dh = hi[i].x - mean[i];
    m2[i] = (lane < chunks ? fmaf(16.f * dl, dl, lo[i].y) : 0.f) +
            (lane + 32 < chunks ? fmaf(16.f * dh, dh, hi[i].y) : 0.f);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (uint32_t i = 0; i < 8; ++i) m2[i] += __shfl_xor_sync(0xFFFFFFFFu, m2[i], o);
  if (lane < nrows) {
    // lane i keeps row i's values (selects: an array indexed by the lane would go to local memory)
    float mu = mean[0], sq = m2[0];
#pragma unroll
    for (uint32_t i = 1; i < 8; ++i)
      if (lane == i) {
        mu = mean[i];
        sq = m2[i];
      }
    mean_out[lane] = mu;
    rstd_out[lane] = rsqrtf(sq / float(chunks * 16) + eps);
  }
}

// A folded LayerNorm's row statistics for the 128 rows of the A operand as its k-blocks stream through the operand
// ring (128-byte swizzled rows, 64 columns per stage): thread t (of 512) takes row t / 4 and 16 of each k-block's 64
// columns, merges 8-element chunks exactly (Chan's update), and the four threads of a row merge by shuffles. Each
// warp releases every stage it has read (the stage's empty barrier counts the MMA and the sixteen warps). Kept out
// of line so its registers do not add to the epilogue's.
__device__ __noinline__ bool ln_stats_from_stages(const uint8_t* smem, uint32_t stage_bytes, uint32_t stages,
                                                  uint64_t* full, uint64_t* empty, uint32_t kblocks, uint32_t rows,
                                                  uint32_t k, float eps, float* mean_out, float* rstd_out,
                                                  uint32_t t, uint32_t lane, volatile int* abort_flag) {
  const uint32_t srow = t >> 2, part = t & 3u;
  float n = 0.f, mean = 0.f, m2 = 0.f;
  uint32_t stage = 0, phase = 0;
  bool ok = true;
  for (uint32_t kb = 0; kb < kblocks; ++kb) {
    if (!mbar_wait(&full[stage], phase, kWatchFull, abort_flag)) { ok = false; break; }
    if (srow < rows) {
      const uint8_t* a_row = smem + stage * stage_bytes + srow * 128;
#pragma unroll
      for (uint32_t h = 0; h < 2; ++h) {
        const uint32_t c = 2 * part + h;  // 16-byte chunk of the row (128-byte swizzle)
        const uint4 w = *reinterpret_cast<const uint4*>(a_row + ((c ^ (srow & 7u)) * 16));
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
        float v[8], cm = 0.f;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          v[2 * q] = bf16_lo(ws[q]);
          v[2 * q + 1] = bf16_hi(ws[q]);
        }
#pragma unroll
        for (int q = 0; q < 8; ++q) cm += v[q];
        cm *= 0.125f;
        float cm2 = 0.f;
#pragma unroll
        for (int q = 0; q < 8; ++q) cm2 = fmaf(v[q] - cm, v[q] - cm, cm2);
        const float n_new = n + 8.f, delta = cm - mean;
        mean = fmaf(delta, 8.f / n_new, mean);
        m2 += cm2 + delta * delta * (n * 8.f / n_new);
        n = n_new;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
    if (++stage == stages) { stage = 0; phase ^= 1u; }
  }
  for (uint32_t off = 2; off >= 1; off /= 2) {
    const float on = __shfl_xor_sync(0xFFFFFFFFu, n, off);
    const float om = __shfl_xor_sync(0xFFFFFFFFu, mean, off);
    const float o2 = __shfl_xor_sync(0xFFFFFFFFu, m2, off);
    const float tot = n + on;
    if (tot > 0.f) {
      const float delta = om - mean;
      mean = fmaf(delta, on / tot, mean);
      m2 += o2 + delta * delta * (n * on / tot);
      n = tot;
    }
  }
  if (srow < rows && part == 0) {
    mean_out[srow] = mean;
    rstd_out[srow] = rsqrtf(m2 / float(k) + eps);
  }
  return ok;
}

// LN: the folded-LayerNorm variant (tempo_gemm_ln); a separate instantiation, so the statistics code adds no
// registers to the others.
template <int BN, int STAGES, bool STAGED, bool LN>
__global__ void __launch_bounds__(kRowThreads, 1)
    gemm_rowmajor_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                         const __grid_constant__ CUtensorMap tmap_out, RowMajorParams p) {
  using L = RowMajorSmem<BN, STAGES, STAGED>;
  static_assert(!STAGED || BN >= 128, "staged stores need 32-column chunks");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarrierOffset);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* acc_full = bars + 2 * STAGES;
  uint64_t* acc_empty = bars + 2 * STAGES + 2;
  uint64_t* final_bar = bars + 2 * STAGES + 4;
  uint64_t* epi_bar = bars + 2 * STAGES + 5;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::kBarriers);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();
  const uint32_t tiles = p.m_tiles * p.n_tiles;
  const uint32_t kblocks = (p.k + kBK - 1) / kBK;
  constexpr uint32_t kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;

  if (threadIdx.x == 0) {
    // With a folded LayerNorm whose statistics are computed here the epilogue warps also read each A stage of the
    // first tile: a stage is free once the MMA and those sixteen warps are done with it.
    const uint32_t empty_count = LN && p.ln_stats == nullptr ? 1u + kRowEpiThreads / 32 : 1u;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], empty_count);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], kRowEpiThreads);
    }
    mbar_init(final_bar, 1);
    mbar_init(epi_bar, kRowEpiThreads);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
    if (STAGED) tma_prefetch_desc(&tmap_out);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_launch_dependents();
  // The A operand, the residual and the output may belong to the previous kernel in the stream: the producer waits
  // for it after prefetching weights, the epilogue before its first access. The MMA warp reads only shared memory.

  if (warp == 0) {
    if (elect_one()) {
      uint32_t stage = 0, phase = 0;
      uint32_t last_parity[STAGES];
      bool used[STAGES];
      for (int s = 0; s < STAGES; ++s) used[s] = false;
      bool ok = true;
      // The weights are not the previous kernel's output: the first tile's first ring of B tiles streams in before
      // the wait.
      const uint32_t early = blockIdx.x < tiles ? (kblocks < uint32_t(STAGES) ? kblocks : uint32_t(STAGES)) : 0u;
      if (early > 0) {
        const int32_t n0 = int32_t((blockIdx.x % p.n_tiles) * BN);
        for (uint32_t kb = 0; kb < early; ++kb) {
          mbar_arrive_expect_tx(&full[kb], p.stage_tx);
          tma_load_2d(smem + kb * L::kStageBytes + L::kABytes, &tmap_b, &full[kb], int32_t(kb * kBK), n0);
          used[kb] = true;  // a copy is in flight on this stage from here on
          last_parity[kb] = 0;
        }
      }
      pdl_wait();
      bool first = true;
      for (uint32_t t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int32_t m0 = int32_t((t / p.n_tiles) * 128);
        const int32_t n0 = int32_t((t % p.n_tiles) * BN);
        for (uint32_t kb = 0; kb < kblocks; ++kb) {
          uint8_t* a_dst = smem + stage * L::kStageBytes;
          if (!(first && kb < early)) {
            if (!mbar_wait(&empty[stage], phase ^ 1u, kWatchEmpty, abort_flag)) { ok = false; break; }
            mbar_arrive_expect_tx(&full[stage], p.stage_tx);
            tma_load_2d(a_dst + L::kABytes, &tmap_b, &full[stage], int32_t(kb * kBK), n0);
          }
          tma_load_2d(a_dst, &tmap_a, &full[stage], int32_t(kb * kBK), m0);
          used[stage] = true;
          last_parity[stage] = phase;
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        first = false;
      }
      // Every copy this thread issued must have landed before the CTA may exit.
      for (int s = 0; s < STAGES; ++s)
        if (used[s]) mbar_wait(&full[s], last_parity[s], kWatchFull, nullptr);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc = make_idesc_bf16(128, BN, 0, 0);
      uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
      bool ok = true;
      for (uint32_t t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u, kWatchAccEmpty, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (uint32_t kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, kWatchFull, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * L::kStageBytes);
          const uint32_t b_addr = a_addr + L::kABytes;
#pragma unroll
          for (uint32_t kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t a_desc = make_smem_desc(a_addr + kk * 32, 16, 1024, kLayoutSw128);
            const uint64_t b_desc = make_smem_desc(b_addr + kk * 32, 16, 1024, kLayoutSw128);
            umma_bf16(d_tmem, a_desc, b_desc, idesc, (kb | kk) != 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit(&acc_full[acc]);
        acc ^= 1u;
        if (acc == 0) acc_phase ^= 1u;
      }
      // Drain every MMA this thread issued before the accumulator is freed.
      umma_commit(final_bar);
      mbar_wait(final_bar, 0, kWatchOther, nullptr);
    }
  } else {
    // Epilogue: warp owns TMEM lanes 32*(warp%4) .. +31 (tile rows) and one quarter of the tile's columns.
    const uint32_t lane_base = 32u * (warp & 3u);
    const uint32_t row_in_tile = lane_base + lane;
    const uint32_t group = (warp - 2) >> 2;
    // Narrow tiles (BN 16 or 32) leave the upper column groups idle: every group needs 16 columns or more.
    constexpr uint32_t kActiveGroups = BN / 16 < kRowEpiGroups ? BN / 16 : kRowEpiGroups;
    constexpr uint32_t kGroupCols = BN / kActiveGroups;
    constexpr uint32_t kCW = kGroupCols >= 32 ? 32 : 16;  // columns per TMEM load
    static_assert(kActiveGroups >= 1 && kGroupCols % kCW == 0, "row-major tile width");
    float* exchange_val = reinterpret_cast<float*>(smem + L::kExchangeOffset);
    int32_t* exchange_idx = reinterpret_cast<int32_t*>(exchange_val + 128);
    uint32_t acc = 0, acc_phase = 0;
    pdl_wait();
    constexpr bool ln = LN;
    float* ln_mean = exchange_val;  // the argmax hand-off slot: the two modes are exclusive
    float* ln_rstd = exchange_val + 128;
    uint32_t ln_block = 0xFFFFFFFFu, epi_phase = 0;  // the 128-row block whose statistics are in ln_mean / ln_rstd
    // Every epilogue thread arrives; the wait is bounded, so a thread that left the loop cannot stall the others.
    auto epi_sync = [&]() -> bool {
      mbar_arrive(epi_bar);
      const bool ok = mbar_wait(epi_bar, epi_phase, kWatchOther, abort_flag);
      epi_phase ^= 1u;
      return ok;
    };
    const bool gelu = (p.flags & TEMPO_GEMM_GELU) != 0;
    const bool argmax = (p.flags & TEMPO_GEMM_ARGMAX) != 0;
    if (ln && blockIdx.x < tiles) {
      // The first tile's row statistics from its A stages as they stream in for the MMA, ready with the accumulator.
      const uint32_t first_block = blockIdx.x / p.n_tiles;
      const uint32_t rows = p.m - first_block * 128 < 128u ? p.m - first_block * 128 : 128u;
      bool ok = true;
      if (p.ln_stats != nullptr) {
        // From the partials of the kernel that wrote the rows (it has finished: the wait above): epilogue warp w
        // takes rows 8 w .. 8 w + 7.
        const uint32_t r0 = 8 * ((threadIdx.x - 64) / 32);
        if (r0 < rows)
          combine_row_stats_warp(p.ln_stats, p.k / 16, first_block * 128 + r0, rows - r0 < 8 ? rows - r0 : 8u,
                                 p.ln_eps, ln_mean + r0, ln_rstd + r0, lane);
      } else {
        ok = ln_stats_from_stages(smem, L::kStageBytes, STAGES, full, empty, kblocks, rows, p.k, p.ln_eps, ln_mean,
                                  ln_rstd, threadIdx.x - 64, lane, abort_flag);
      }
      ln_block = first_block;
      if (!ok || !epi_sync()) ln_block = 0xFFFFFFFFu;  // (a timeout: the tile loop below gives up as well)
    }
    // (A folded LayerNorm runs with one tile per CTA: the host guarantees it.)
    for (uint32_t t = blockIdx.x; t < tiles && !(ln && ln_block == 0xFFFFFFFFu); t += gridDim.x) {
      if (!mbar_wait(&acc_full[acc], acc_phase, kWatchAccFull, abort_flag)) break;
      tc_fence_after();
      const uint32_t m_blk = t / p.n_tiles, n_blk = t % p.n_tiles;
      const uint32_t row = m_blk * 128 + row_in_tile;
      const bool row_ok = row < p.m;
      float best = -INFINITY;
      int32_t best_idx = 0;
#pragma unroll 1
      for (uint32_t c = group * kGroupCols; group < kActiveGroups && c < (group + 1) * kGroupCols; c += kCW) {
        uint32_t r[kCW];
        if constexpr (kCW == 32) {
          tmem_ld_32x32b_x32(tmem_base + (lane_base << 16) + acc * BN + c, r);
        } else {
          tmem_ld_32x32b_x16(tmem_base + (lane_base << 16) + acc * BN + c, r);
        }
        tmem_wait_ld();
        const uint32_t n0 = n_blk * BN + c;
        if constexpr (STAGED) {
          // The warp's 32 x 32 block through its staging tile and one TMA store (rows past M and columns past N are
          // clipped by the copy). Never in argmax mode.
          const uint32_t row0 = m_blk * 128 + lane_base;
          if (row0 >= p.m || n0 >= p.n) continue;  // warp-uniform
          uint8_t* staging = smem + L::kStagingOffset + (warp - 2) * 2048;
          if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
          __syncwarp();
          const float mu = ln ? ln_mean[row_in_tile] : 0.f, rs = ln ? ln_rstd[row_in_tile] : 0.f;
          epilogue_chunk<kCW, true>(p, r, row, n0, gelu, ln, mu, rs, staging + lane * 64, (lane >> 1) & 3u);
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmap_out, staging, int32_t(n0), int32_t(row0));
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
          }
          continue;
        }
        if (!row_ok || n0 >= p.n) continue;
        if (argmax) {
#pragma unroll
          for (uint32_t j = 0; j < kCW; ++j) {
            const float v = __uint_as_float(r[j]);
            if (n0 + j < p.n && v > best) { best = v; best_idx = int32_t(n0 + j); }
          }
          continue;
        }
        const float mu = ln ? ln_mean[row_in_tile] : 0.f, rs = ln ? ln_rstd[row_in_tile] : 0.f;
        epilogue_chunk<kCW>(p, r, row, n0, gelu, ln, mu, rs);
      }
      if (argmax) {
        // The best of each row passes down the column groups, highest first, each keeping its own (earlier) index
        // on a tie; group 0 writes the tile's partial. One 128-row slot (1 KB) carries it.
        const uint32_t quarter_barrier = 1 + (warp & 3u);
#pragma unroll 1
        for (uint32_t g = kRowEpiGroups - 1; g >= 1; --g) {
          if (group == g) {
            exchange_val[row_in_tile] = best;
            exchange_idx[row_in_tile] = best_idx;
          }
          asm volatile("bar.sync %0, %1;" ::"r"(quarter_barrier), "r"(32 * kRowEpiGroups) : "memory");
          if (group == g - 1) {
            const float other = exchange_val[row_in_tile];
            if (other > best) { best = other; best_idx = exchange_idx[row_in_tile]; }
          }
        }
        if (group == 0 && row_ok) {
          p.part_val[size_t(row) * p.n_tiles + n_blk] = best;
          p.part_idx[size_t(row) * p.n_tiles + n_blk] = best_idx;
        }
        // The slot is free again only once group 0 has read it.
        asm volatile("bar.sync %0, %1;" ::"r"(quarter_barrier), "r"(32 * kRowEpiGroups) : "memory");
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[acc]);
      acc ^= 1u;
      if (acc == 0) acc_phase ^= 1u;
    }
  }

  if (STAGED && warp >= 2 && lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Packed per-block GEMM (swap-AB: UMMA M = 128 output columns, N = 32 tokens)
// ---------------------------------------------------------------------------------------------------------------

struct BlockParams {
  const uint16_t* bias;  // [columns/16][4][16] or null
  uint16_t* drain;       // zero tile, then [columns/16][32][16]
  uint32_t depth, columns;
  uint32_t activate;
};

constexpr int kBlockStages = 4;
constexpr uint32_t kBlockW = 128 * kBK * 2;  // 8 column tiles x 64 deep x 16
constexpr uint32_t kBlockA = 32 * kBK * 2;   // 4 k tiles x 32 tokens x 16
constexpr uint32_t kBlockStage = kBlockW + kBlockA;
constexpr uint32_t kBlockOut = 128 * 32 * 2;  // the CTA's 8 output tiles
constexpr uint32_t kBlockBarrierOffset = kBlockStages * kBlockStage + kBlockOut;
constexpr uint32_t kBlockBarriers = 3 * kBlockStages + 2;  // full, ready, empty, acc_full, final
constexpr uint32_t kBlockSmem = kBlockBarrierOffset + kBlockBarriers * 8 + 16 + 1024;

__global__ void __launch_bounds__(kThreads, 1)
    gemm_block_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_a,
                      BlockParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint16_t* out_tile = reinterpret_cast<uint16_t*>(smem + kBlockStages * kBlockStage);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBlockBarrierOffset);
  uint64_t* full = bars;
  uint64_t* ready = bars + kBlockStages;
  uint64_t* empty = bars + 2 * kBlockStages;
  uint64_t* acc_full = bars + 3 * kBlockStages;
  uint64_t* final_bar = acc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kBlockBarriers);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();
  const uint32_t kblocks = (p.depth + kBK - 1) / kBK;
  const uint32_t col_tile0 = blockIdx.x * 8;  // first 16-column tile of this CTA
  const bool activate = p.activate != 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kBlockStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&ready[s], 128);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(final_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmap_w);
    tma_prefetch_desc(&tmap_a);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (elect_one()) {
      uint32_t stage = 0, phase = 0;
      uint32_t last_parity[kBlockStages];
      bool used[kBlockStages] = {false, false, false, false};
      for (uint32_t kb = 0; kb < kblocks; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, kWatchEmpty, abort_flag)) break;
        uint8_t* w_dst = smem + stage * kBlockStage;
        uint8_t* a_dst = w_dst + kBlockW;
        mbar_arrive_expect_tx(&full[stage], kBlockStage);
        tma_load_3d(w_dst, &tmap_w, &full[stage], 0, int32_t(kb * kBK), int32_t(col_tile0));
        tma_load_3d(a_dst, &tmap_a, &full[stage], 0, 0, int32_t(kb * (kBK / 16)));
        used[stage] = true;
        last_parity[stage] = phase;
        if (++stage == kBlockStages) { stage = 0; phase ^= 1u; }
      }
      for (int s = 0; s < kBlockStages; ++s)
        if (used[s]) mbar_wait(&full[s], last_parity[s], kWatchFull, nullptr);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc = make_idesc_bf16(128, 32, 1, 0);
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      for (uint32_t kb = 0; kb < kblocks; ++kb) {
        uint64_t* wait_on = activate ? &ready[stage] : &full[stage];
        if (!mbar_wait(wait_on, phase, kWatchFull, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t w_addr = smem_u32(smem + stage * kBlockStage);
        const uint32_t a_addr = w_addr + kBlockW;
#pragma unroll
        for (uint32_t kk = 0; kk < kBK / 16; ++kk) {
          // Weights: MN-major, 16-column groups 64 rows x 32 B apart (LBO), 8-row groups 256 B apart (SBO).
          const uint64_t w_desc = make_smem_desc(w_addr + kk * 512, kBK * 32, 256, kLayoutSw32);
          // Activations: K-major, one 16-deep tile (32 rows x 32 B) per MMA, 8-row groups 256 B apart.
          const uint64_t a_desc = make_smem_desc(a_addr + kk * 1024, 16, 256, kLayoutSw32);
          umma_bf16(tmem_base, w_desc, a_desc, idesc, (kb | kk) != 0u);
        }
        umma_commit(&empty[stage]);
        if (++stage == kBlockStages) { stage = 0; phase ^= 1u; }
      }
      if (ok) umma_commit(acc_full);
      umma_commit(final_bar);
      mbar_wait(final_bar, 0, kWatchOther, nullptr);
    }
  } else {
    const uint32_t t128 = threadIdx.x - 64;  // 0..127
    if (activate) {
      // GELU on each staged activation tile (4096 bytes = 2048 values: 16 per thread), then release it to the MMA.
      uint32_t stage = 0, phase = 0;
      for (uint32_t kb = 0; kb < kblocks; ++kb) {
        if (!mbar_wait(&full[stage], phase, kWatchFull, abort_flag)) break;
        uint4* a4 = reinterpret_cast<uint4*>(smem + stage * kBlockStage + kBlockW);
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          uint4 w = a4[t128 * 2 + q];
          uint32_t* ws = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            float lo = bf16_lo(ws[h]), hi = bf16_hi(ws[h]);
            gelu_erf_pair(lo, hi);
            ws[h] = pack_bf16x2(lo, hi);
          }
          a4[t128 * 2 + q] = w;
        }
        fence_proxy_async_smem();
        mbar_arrive(&ready[stage]);
        if (++stage == kBlockStages) { stage = 0; phase ^= 1u; }
      }
    }
    // Epilogue: thread = output column (TMEM lane), 32 accumulator columns = the block's 32 tokens.
    const uint32_t lane_base = 32u * (warp & 3u);
    const uint32_t col = lane_base + lane;  // 0..127 within the CTA
    const uint32_t col_global = col_tile0 * 16 + col;
    if (mbar_wait(acc_full, 0, kWatchAccFull, abort_flag)) {
      tc_fence_after();
      uint32_t r[32];
      tmem_ld_32x32b_x32(tmem_base + (lane_base << 16), r);
      tmem_wait_ld();
      const uint32_t ct = col >> 4, j = col & 15u;
#pragma unroll
      for (int t = 0; t < 32; ++t) {
        float v = __uint_as_float(r[t]);
        // Token t reads bias row t % 4 of its feature tile, as the broadcast read does (bf16.py:159-175).
        if (p.bias != nullptr && col_global < p.columns)
          v += bf16_to_float(p.bias[(size_t(col_tile0 + ct) * 4 + (t & 3)) * 16 + j]);
        out_tile[(ct * 32 + t) * 16 + j] = float_to_bf16(v);
      }
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");
    // The CTA's 8 tiles are contiguous in the drain: 8 x 1 KB past the zero tile and the tiles before them.
    const uint32_t tiles_valid = min(8u, p.columns / 16 - col_tile0);
    uint4* dst = reinterpret_cast<uint4*>(p.drain + 256 + size_t(col_tile0) * 512);
    const uint4* src = reinterpret_cast<const uint4*>(out_tile);
    for (uint32_t i = t128; i < tiles_valid * 64; i += 128) dst[i] = src[i];
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 32);
  }
}

template <int BN, int STAGES, bool STAGED = false, bool LN = false>
tempo_status launch_rowmajor(const void* a, uint32_t lda, const void* w_t, uint32_t ldw, const RowMajorParams& base,
                             cudaStream_t stream) {
  using L = RowMajorSmem<BN, STAGES, STAGED>;
  CUtensorMap ta, tb;
  const uint64_t a_dims[2] = {base.k, base.m};
  const uint64_t a_strides[1] = {uint64_t(lda) * 2};
  // At most 64 rows: a 64-row box, so the copy fills no out-of-range rows (the MMA's upper 64 rows are discarded).
  const uint32_t a_rows = base.m <= 64 ? 64 : 128;
  const uint32_t a_box[2] = {kBK, a_rows};
  tempo_status s = encode_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a, a_dims, a_strides, a_box,
                               CU_TENSOR_MAP_SWIZZLE_128B);
  if (s != TEMPO_OK) return s;
  const uint64_t b_dims[2] = {base.k, base.n};
  const uint64_t b_strides[1] = {uint64_t(ldw) * 2};
  const uint32_t b_box[2] = {kBK, uint32_t(BN)};
  s = encode_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w_t, b_dims, b_strides, b_box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (s != TEMPO_OK) return s;
  CUtensorMap to = ta;  // unused unless STAGED
  if (STAGED) {
    const uint64_t o_dims[2] = {base.n, base.m};
    const uint64_t o_strides[1] = {uint64_t(base.ldo) * 2};
    const uint32_t o_box[2] = {32, 32};
    s = encode_tmap(&to, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base.out, o_dims, o_strides, o_box,
                    CU_TENSOR_MAP_SWIZZLE_64B);
    if (s != TEMPO_OK) return s;
  }
  RowMajorParams p = base;
  p.stage_tx = a_rows * kBK * 2 + L::kBBytes;
  p.m_tiles = (p.m + 127) / 128;
  p.n_tiles = (p.n + BN - 1) / BN;
  const uint32_t tiles = p.m_tiles * p.n_tiles;
  const uint32_t grid = tiles < uint32_t(sm_count()) ? tiles : uint32_t(sm_count());
  auto kernel = gemm_rowmajor_kernel<BN, STAGES, STAGED, LN>;
  s = set_smem(reinterpret_cast<const void*>(kernel), L::kBytes);
  if (s != TEMPO_OK) return s;
  return launch(kernel, dim3(grid), dim3(kRowThreads), L::kBytes, stream, 1, "gemm_rowmajor_kernel", ta, tb, to, p);
}

// ---------------------------------------------------------------------------------------------------------------
// Split-K for small M (the decode projections): a cluster of SPLITS CTAs shares one 128 x BN output tile, each CTA
// running a contiguous share of the k-blocks into its own TMEM accumulator. The FP32 partial tiles are reduced
// through distributed shared memory: CTA r owns rows [r*128/SPLITS, (r+1)*128/SPLITS) of the tile. Each epilogue
// warp holds 32 rows (its TMEM lane quarter) x one half of the columns; it writes the rows it owns straight into its
// own reduction buffer and the others into a staging tile in the (by then idle) operand ring, and sends each staged
// piece to its owner with one bulk shared::cta -> shared::cluster copy that completes on the owner's mbarrier. The
// owner waits for the bytes of the other SPLITS - 1 CTAs, sums the partials in rank order and runs the epilogue with
// coalesced 16-byte stores, its bias and residual already loaded while the MMAs ran. No workspace and no atomics.
// The 16-byte chunks of each partial row are XOR-swizzled by row % 8, so the 32 lanes of a warp, one row each, store
// into different banks without padding (the shared memory stays within the 196 KB carveout, which leaves 60 KB of
// L1 to kernels sharing the SM). The ring holds only as many stages as a split has k-blocks (two or more).
// ---------------------------------------------------------------------------------------------------------------

template <int BN, int SPLITS, int STAGES>
struct SplitSmem {
  static constexpr uint32_t kABytes = 128 * kBK * 2;
  static constexpr uint32_t kBBytes = BN * kBK * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr uint32_t kRowsPer = 128 / SPLITS;
  static constexpr uint32_t kHalfCols = BN / 2;  // the columns one epilogue warp holds
  // [SPLITS source ranks][2 halves][kRowsPer rows][kHalfCols] FP32 partials: the piece one warp sends an owner is
  // contiguous.
  static constexpr uint32_t kRedBytes = 128 * BN * 4;
  static constexpr uint32_t kRemoteBytes = (SPLITS - 1) * kRowsPer * BN * 4;  // what an owner receives
  // A staging tile of 32 rows x kHalfCols per epilogue warp, in the operand ring (two stages or more).
  static constexpr uint32_t kStagingBytes = (kEpilogueThreads / 32) * 32 * kHalfCols * 4;
  static_assert(kStagingBytes <= 2 * kStageBytes, "split-K staging exceeds two ring stages");
  static constexpr uint32_t kBarriers = 2 * STAGES + 3;  // full, empty, acc_full, final, red_full
  // A folded LayerNorm's mean and rstd of the owned rows, then the tile's column sums and folded bias.
  static constexpr uint32_t kLnBytes = (2 * kRowsPer + 2 * BN) * 4;
  __host__ __device__ static constexpr uint32_t red_offset(uint32_t stages) { return stages * kStageBytes; }
  __host__ __device__ static constexpr uint32_t ln_offset(uint32_t stages) { return red_offset(stages) + kRedBytes; }
  __host__ __device__ static constexpr uint32_t barrier_offset(uint32_t stages) { return ln_offset(stages) + kLnBytes; }
  __host__ __device__ static constexpr uint32_t bytes(uint32_t stages) {
    return barrier_offset(stages) + kBarriers * 8 + 16 + 1024;
  }
  __host__ __device__ static constexpr uint32_t block(uint32_t src, uint32_t half) {
    return (src * 2 + half) * kRowsPer * kHalfCols;  // in floats
  }
  static_assert(barrier_offset(STAGES) + kBarriers * 8 + 16 + 1024 <= 195 * 1024,
                "split-K GEMM shared memory exceeds the 196 KB carveout");
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t map_to_rank(uint32_t local_smem_addr, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_smem_addr), "r"(rank));
  return remote;
}

// A bulk copy from this CTA's shared memory into another CTA's of the cluster (both addresses 16-byte aligned, the
// size a multiple of 16), completing `bytes` of transactions on the destination CTA's mbarrier.
__device__ __forceinline__ void bulk_copy_to_cluster(uint32_t dst_cluster, uint32_t src_cta, uint32_t bytes,
                                                     uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst_cluster),
      "r"(src_cta), "r"(bytes), "r"(bar_cluster)
      : "memory");
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// The split halves of a cluster barrier: every thread of the cluster arrives once (relaxed: it orders nothing) and
// later waits for all the others to have arrived.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }

template <int BN, int SPLITS, int STAGES>
__global__ void __launch_bounds__(kSplitThreads, 1)
    gemm_splitk_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                       RowMajorParams p) {
  using L = SplitSmem<BN, SPLITS, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t stages = p.stages;
  float* red = reinterpret_cast<float*>(smem + L::red_offset(stages));
  float* ln_mu = reinterpret_cast<float*>(smem + L::ln_offset(stages));
  float* ln_rs = ln_mu + L::kRowsPer;
  float* ln_cs = ln_rs + L::kRowsPer;
  float* ln_b = ln_cs + BN;
  float* staging = reinterpret_cast<float*>(smem);  // the operand ring, idle once the accumulator is final
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::barrier_offset(stages));
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* acc_full = bars + 2 * STAGES;
  uint64_t* final_bar = acc_full + 1;
  uint64_t* red_full = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::kBarriers);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  constexpr uint32_t kTmemCols = BN < 32 ? 32 : BN;
  constexpr uint32_t kHalfCols = L::kHalfCols;
  constexpr uint32_t kChunks = BN / 8;  // 8-column chunks per tile row
  constexpr uint32_t kItems = (L::kRowsPer * kChunks + kEpilogueThreads - 1) / kEpilogueThreads;

  const uint32_t warp = warp_id(), lane = lane_id();
  const uint32_t rank = cluster_rank();
  const uint32_t tile = blockIdx.x / SPLITS;
  const uint32_t m_blk = tile / p.n_tiles, n_blk = tile % p.n_tiles;
  const uint32_t kblocks = (p.k + kBK - 1) / kBK;
  const uint32_t kb0 = rank * kblocks / SPLITS, kb1 = (rank + 1) * kblocks / SPLITS;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(final_bar, 1);
    // Completes once the other CTAs' partial rows for this CTA have all landed.
    mbar_init(red_full, 1);
    mbar_arrive_expect_tx(red_full, L::kRemoteBytes);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_launch_dependents();
  // Another CTA's shared memory (and its mbarrier) may be written only once every CTA of the cluster has started and
  // initialised its barriers: each announces itself here, and the epilogue warps wait for the whole cluster before
  // their first copy.
  cluster_arrive_relaxed();

  if (warp == 0) {
    if (elect_one()) {
      uint32_t stage = 0, phase = 0;
      uint32_t last_parity[STAGES];
      bool used[STAGES];
      for (int s = 0; s < STAGES; ++s) used[s] = false;
      // The weights do not depend on the previous kernel: the first ring's worth streams in before the wait.
      const uint32_t early = (kb1 - kb0) < stages ? (kb1 - kb0) : stages;
      for (uint32_t i = 0; i < early; ++i) {
        mbar_arrive_expect_tx(&full[i], p.stage_tx);
        tma_load_2d(smem + i * L::kStageBytes + L::kABytes, &tmap_b, &full[i], int32_t((kb0 + i) * kBK),
                    int32_t(n_blk * BN));
        used[i] = true;  // a copy is in flight on this stage from here on
        last_parity[i] = 0;
      }
      pdl_wait();
      for (uint32_t kb = kb0; kb < kb1; ++kb) {
        uint8_t* a_dst = smem + stage * L::kStageBytes;
        if (kb - kb0 >= early) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, kWatchEmpty, abort_flag)) break;
          mbar_arrive_expect_tx(&full[stage], p.stage_tx);
          tma_load_2d(a_dst + L::kABytes, &tmap_b, &full[stage], int32_t(kb * kBK), int32_t(n_blk * BN));
        }
        tma_load_2d(a_dst, &tmap_a, &full[stage], int32_t(kb * kBK), int32_t(m_blk * 128));
        used[stage] = true;
        last_parity[stage] = phase;
        if (++stage == stages) { stage = 0; phase ^= 1u; }
      }
      for (int s = 0; s < STAGES; ++s)
        if (used[s]) mbar_wait(&full[s], last_parity[s], kWatchFull, nullptr);
    }
    __syncwarp();
    cluster_wait();
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc = make_idesc_bf16(128, BN, 0, 0);
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      for (uint32_t kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&full[stage], phase, kWatchFull, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t a_addr = smem_u32(smem + stage * L::kStageBytes);
        const uint32_t b_addr = a_addr + L::kABytes;
#pragma unroll
        for (uint32_t kk = 0; kk < kBK / 16; ++kk) {
          const uint64_t a_desc = make_smem_desc(a_addr + kk * 32, 16, 1024, kLayoutSw128);
          const uint64_t b_desc = make_smem_desc(b_addr + kk * 32, 16, 1024, kLayoutSw128);
          umma_bf16(tmem_base, a_desc, b_desc, idesc, (kb != kb0 || kk != 0) ? 1u : 0u);
        }
        umma_commit(&empty[stage]);
        if (++stage == stages) { stage = 0; phase ^= 1u; }
      }
      if (ok) umma_commit(acc_full);
      umma_commit(final_bar);
      mbar_wait(final_bar, 0, kWatchOther, nullptr);
    }
    __syncwarp();
    cluster_wait();
  } else {
    const uint32_t t = threadIdx.x - 64;
    const bool gelu = (p.flags & TEMPO_GEMM_GELU) != 0;
    cluster_wait();
    // The bias and the residual of this thread's output chunks, loaded while the MMAs run. The residual (and the
    // output) may be the previous kernel's: wait for it first (the A operand's producer has already waited).
    pdl_wait();
    uint4 pre_bias[kItems], pre_res[kItems];
#pragma unroll
    for (uint32_t i = 0; i < kItems; ++i) {
      const uint32_t item = t + i * kEpilogueThreads;
      const uint32_t lr = item / kChunks, c8 = item % kChunks;
      const uint32_t row = m_blk * 128 + rank * L::kRowsPer + lr;
      const uint32_t col = n_blk * BN + c8 * 8;
      const bool in = item < L::kRowsPer * kChunks && row < p.m && col < p.n;
      pre_bias[i] = in && p.bias != nullptr ? __ldg(reinterpret_cast<const uint4*>(p.bias + col)) : make_uint4(0, 0, 0, 0);
      pre_res[i] = in && p.residual != nullptr
                       ? *reinterpret_cast<const uint4*>(p.residual + size_t(row) * p.ldr + col)
                       : make_uint4(0, 0, 0, 0);
    }
    // A folded LayerNorm: the owned rows' mean and rstd from the partials of the kernel that wrote the rows (epilogue
    // warp w takes kRowsPer / 8 of them), and the tile's column sums and folded bias, in shared memory before phase 2.
    const bool ln = p.ln_stats != nullptr;
    if (ln) {
      constexpr uint32_t kPerWarp = L::kRowsPer / 8;
      const uint32_t r0 = (t / 32) * kPerWarp, row0 = m_blk * 128 + rank * L::kRowsPer + r0;
      const uint32_t nrows = row0 >= p.m ? 0u : (p.m - row0 < kPerWarp ? p.m - row0 : kPerWarp);
      if (nrows > 0)
        combine_row_stats_warp(p.ln_stats, p.k / 16, row0, nrows, p.ln_eps, ln_mu + r0, ln_rs + r0, lane);
      if (t < uint32_t(BN)) {
        const uint32_t col = n_blk * BN + t;
        ln_cs[t] = col < p.n ? __ldg(p.ln_colsum + col) : 0.f;
        ln_b[t] = col < p.n ? __ldg(p.ln_bias + col) : 0.f;
      }
    }

    // Phase 1: warp (quarter q, half h) holds tile rows 32q .. 32q + 31 x columns h * BN / 2 ...; each lane's
    // half-row goes to its owner's block [rank][h], directly if this CTA owns it, else through the warp's staging
    // tile and one bulk copy per owner.
    const uint32_t quarter = warp & 3u, half = (warp - 2) >> 2;
    const uint32_t row_in_tile = 32u * quarter + lane;
    const uint32_t owner = row_in_tile / L::kRowsPer, owned_row = row_in_tile % L::kRowsPer;
    float* stage_rows = staging + (warp - 2) * 32 * kHalfCols;
    float* dst_row = owner == rank ? red + L::block(rank, half) + owned_row * kHalfCols : stage_rows + lane * kHalfCols;
    const uint32_t key = lane & 7u;  // == owned_row % 8: kRowsPer and 32 q are multiples of 8
    const bool have_acc = mbar_wait(acc_full, 0, kWatchAccFull, abort_flag);
    if (have_acc) {
      tc_fence_after();
#pragma unroll
      for (uint32_t c = 0; c < kHalfCols; c += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + ((32u * quarter) << 16) + half * kHalfCols + c, r);
        tmem_wait_ld();
#pragma unroll
        for (uint32_t q = 0; q < 8; ++q) {
          float4* chunk = reinterpret_cast<float4*>(dst_row) + ((c / 4 + q) ^ key);
          *chunk = make_float4(__uint_as_float(r[q * 4]), __uint_as_float(r[q * 4 + 1]),
                               __uint_as_float(r[q * 4 + 2]), __uint_as_float(r[q * 4 + 3]));
        }
      }
      // The staged rows reach the copy engine (the async proxy) only after this fence.
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      // One piece per owner: 32 rows (SPLITS <= 4) or two pieces of 16 rows (SPLITS = 8).
      constexpr uint32_t kPieceRows = L::kRowsPer < 32 ? L::kRowsPer : 32u;
      if (lane % kPieceRows == 0 && owner != rank) {
        const uint32_t bytes = kPieceRows * kHalfCols * 4;
        const uint32_t dst = map_to_rank(smem_u32(red + L::block(rank, half) + owned_row * kHalfCols), owner);
        bulk_copy_to_cluster(dst, smem_u32(stage_rows + lane * kHalfCols), bytes, map_to_rank(smem_u32(red_full), owner));
      }
    }
    // This CTA's own rows are in place once every epilogue warp has passed here; the others' once red_full completes.
    asm volatile("bar.sync 1, %0;" ::"r"(kEpilogueThreads) : "memory");
    const bool have_all = have_acc && mbar_wait(red_full, 0, kWatchOther, abort_flag);

    if (have_all && !*abort_flag) {
      // Phase 2: sum the owned rows' partials in rank order, then the folded LayerNorm, bias / GELU / residual and
      // 16-byte BF16 stores (and the stored rows' statistics). A warp leaves the loop only as a whole (the item bound
      // is a multiple of 32), so the two lanes of a 16-column chunk always meet at the shuffle.
#pragma unroll
      for (uint32_t i = 0; i < kItems; ++i) {
        const uint32_t item = t + i * kEpilogueThreads;
        if (item >= L::kRowsPer * kChunks) continue;
        const uint32_t lr = item / kChunks, c8 = item % kChunks;
        const uint32_t row = m_blk * 128 + rank * L::kRowsPer + lr;
        const uint32_t col = n_blk * BN + c8 * 8;
        const bool valid = row < p.m && col < p.n;
        const uint32_t h = c8 / (kChunks / 2), cc = c8 % (kChunks / 2);
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = 0.f;
#pragma unroll
        for (uint32_t s = 0; s < uint32_t(SPLITS); ++s) {
          const float4* row_base = reinterpret_cast<const float4*>(red + L::block(s, h) + lr * kHalfCols);
          const float4 x = row_base[(2 * cc) ^ (lr & 7u)], y = row_base[(2 * cc + 1) ^ (lr & 7u)];
          v[0] += x.x; v[1] += x.y; v[2] += x.z; v[3] += x.w;
          v[4] += y.x; v[5] += y.y; v[6] += y.z; v[7] += y.w;
        }
        if (ln) {
          const float mu = ln_mu[lr], rs = ln_rs[lr];
#pragma unroll
          for (int j = 0; j < 8; ++j) v[j] = fmaf(rs, fmaf(-mu, ln_cs[c8 * 8 + j], v[j]), ln_b[c8 * 8 + j]);
        }
        if (p.bias != nullptr) {
          const uint32_t ws[4] = {pre_bias[i].x, pre_bias[i].y, pre_bias[i].z, pre_bias[i].w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            v[2 * q] += bf16_lo(ws[q]);
            v[2 * q + 1] += bf16_hi(ws[q]);
          }
        }
        if (gelu) {
#pragma unroll
          for (int j = 0; j < 8; j += 2) {
            const uint32_t rounded = pack_bf16x2(v[j], v[j + 1]);
            v[j] = bf16_lo(rounded);
            v[j + 1] = bf16_hi(rounded);
            gelu_erf_pair(v[j], v[j + 1]);
          }
        }
        if (p.residual != nullptr) {
          const uint32_t ws[4] = {pre_res[i].x, pre_res[i].y, pre_res[i].z, pre_res[i].w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            v[2 * q] += bf16_lo(ws[q]);
            v[2 * q + 1] += bf16_hi(ws[q]);
          }
        }
        uint4 o;
        o.x = pack_bf16x2(v[0], v[1]);
        o.y = pack_bf16x2(v[2], v[3]);
        o.z = pack_bf16x2(v[4], v[5]);
        o.w = pack_bf16x2(v[6], v[7]);
        if (p.row_stats != nullptr) {
          // Lanes 2j and 2j + 1 hold the two 8-column halves of one 16-column chunk of the row.
          float w[8];
          unpack8(o, w);
          float sum = 0.f;
#pragma unroll
          for (int j = 0; j < 8; ++j) sum += w[j];
          sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 1);
          const float mean = sum * (1.f / 16.f);
          float m2 = 0.f;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float d = w[j] - mean;
            m2 = fmaf(d, d, m2);
          }
          m2 += __shfl_xor_sync(0xFFFFFFFFu, m2, 1);
          if (valid && (c8 & 1u) == 0) p.row_stats[size_t(row) * (p.n / 16) + col / 16] = make_float2(mean, m2);
        }
        if (!valid) continue;
        *reinterpret_cast<uint4*>(p.out + size_t(row) * p.ldo + col) = o;
        uint4* cache4 = reinterpret_cast<uint4*>(kv_destination(p.kv, row, col));
        if (cache4 != nullptr) *cache4 = o;
      }
    }
  }
  // No CTA leaves (freeing the shared memory that copies read from or write into) before every CTA of the cluster
  // has received its partials.
  cluster_sync_all();

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

template <int BN, int SPLITS, int STAGES>
tempo_status launch_splitk(const void* a, uint32_t lda, const void* w_t, uint32_t ldw, const RowMajorParams& base,
                           cudaStream_t stream) {
  using L = SplitSmem<BN, SPLITS, STAGES>;
  CUtensorMap ta, tb;
  const uint64_t a_dims[2] = {base.k, base.m};
  const uint64_t a_strides[1] = {uint64_t(lda) * 2};
  // At most 64 rows: a 64-row box, so the copy fills no out-of-range rows (the MMA's upper 64 rows are discarded).
  const uint32_t a_rows = base.m <= 64 ? 64 : 128;
  const uint32_t a_box[2] = {kBK, a_rows};
  tempo_status s = encode_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a, a_dims, a_strides, a_box,
                               CU_TENSOR_MAP_SWIZZLE_128B);
  if (s != TEMPO_OK) return s;
  const uint64_t b_dims[2] = {base.k, base.n};
  const uint64_t b_strides[1] = {uint64_t(ldw) * 2};
  const uint32_t b_box[2] = {kBK, uint32_t(BN)};
  s = encode_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w_t, b_dims, b_strides, b_box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (s != TEMPO_OK) return s;
  RowMajorParams p = base;
  p.stage_tx = a_rows * kBK * 2 + L::kBBytes;
  p.m_tiles = (p.m + 127) / 128;
  p.n_tiles = (p.n + BN - 1) / BN;
  const uint32_t per_split = ((p.k + kBK - 1) / kBK + SPLITS - 1) / SPLITS;
  p.stages = per_split < uint32_t(STAGES) ? per_split : uint32_t(STAGES);
  // The epilogue stages its outgoing partial rows in the first two ring stages.
  if (p.stages < 2 || (p.k + kBK - 1) / kBK < 2 * SPLITS)
    return fail(TEMPO_ERR_VALUE, "split-K GEMM needs two k-blocks or more per split (k %u, %d splits)", p.k, SPLITS);
  auto kernel = gemm_splitk_kernel<BN, SPLITS, STAGES>;
  s = set_smem(reinterpret_cast<const void*>(kernel), L::bytes(STAGES));
  if (s != TEMPO_OK) return s;
  return launch(kernel, dim3(p.m_tiles * p.n_tiles * SPLITS), dim3(kSplitThreads), L::bytes(p.stages), stream, SPLITS,
                "gemm_splitk_kernel", ta, tb, p);
}

// ---------------------------------------------------------------------------------------------------------------
// CTA-pair GEMM for large M (the prefill projections): a cluster of two CTAs on two SMs computes 256 x 256 output
// tiles with tcgen05.mma.cta_group::2 (M = 256): CTA r of the pair stages rows [128 r, 128 r + 128) of the A tile
// and rows [128 r, 128 r + 128) of the tile's 256 weight rows, the leader's MMA reads both CTAs' shared memory, and
// each CTA's TMEM receives its own 128 output rows x 256 columns. Per SM and k-block that is 32 KB of operands for
// 128 x 256 x 64 MACs instead of 48 KB, which is what feeds the tensor cores from L2 at this size.
//   warp 0      TMA (both CTAs; .cta_group::2 copies complete on the leader's full barrier)
//   warp 1      the leader's MMA issuer; both CTAs' warp 1 allocate and free the pair's TMEM
//   warps 2-17  epilogue (both CTAs), each warp releasing the accumulator on the leader's barrier
// Every copy has a single destination: each CTA loads its own halves, and the leader signals the peer's barriers
// with separate commits addressed to the peer.
// ---------------------------------------------------------------------------------------------------------------

constexpr uint32_t kPairBN = 256;

template <int STAGES>
struct PairSmem {
  static constexpr uint32_t kABytes = 128 * kBK * 2;
  static constexpr uint32_t kBBytes = 128 * kBK * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  // One 32 x 32 BF16 staging tile (2 KB) per epilogue warp for the output's TMA stores.
  static constexpr uint32_t kStagingOffset = STAGES * kStageBytes;
  static constexpr uint32_t kStagingBytes = (kRowEpiThreads / 32) * 2048;
  static constexpr uint32_t kBarrierOffset = kStagingOffset + kStagingBytes;
  // full[S] (the leader's), empty[S], acc_full[2], acc_empty[2] (the leader's), final
  static constexpr uint32_t kBarriers = 2 * STAGES + 5;
  static constexpr uint32_t kBytes = kBarrierOffset + kBarriers * 8 + 16 + 1024;
  static_assert(kBytes <= 195 * 1024, "pair GEMM shared memory exceeds the 196 KB carveout");
};

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst, uint32_t columns) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(columns)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t base, uint32_t columns) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(columns) : "memory");
}

// D[tmem of both CTAs] (+)= A[both CTAs' smem] x B[both CTAs' smem]^T, issued by the leader.
__device__ __forceinline__ void umma_bf16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                               uint32_t accumulate) {
  const uint32_t zero = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(zero));
}

// Arrives on one mbarrier (this CTA's or the peer's, by shared::cluster address) when the pair MMAs this thread issued
// complete.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar_cluster) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster)
               : "memory");
}

// A 2-D tile into this CTA's shared memory, its bytes counted on the leader's barrier (shared::cluster address).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int32_t c0,
                                                 int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}

template <int STAGES>
__global__ void __launch_bounds__(kRowThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                     const __grid_constant__ CUtensorMap tmap_out, RowMajorParams p) {
  using L = PairSmem<STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarrierOffset);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* acc_full = bars + 2 * STAGES;
  uint64_t* acc_empty = bars + 2 * STAGES + 2;
  uint64_t* final_bar = bars + 2 * STAGES + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::kBarriers);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  constexpr uint32_t kTmemCols = 2 * kPairBN;  // two 256-column accumulators
  constexpr uint32_t kEpiWarps = kRowEpiThreads / 32;

  const uint32_t warp = warp_id(), lane = lane_id();
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const uint32_t pairs = gridDim.x / 2, pair = blockIdx.x / 2;
  const uint32_t tiles = p.m_tiles * p.n_tiles;  // 256 x 256 tiles
  const uint32_t kblocks = (p.k + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 2 * kEpiWarps);  // one arrival per epilogue warp of either CTA
    }
    mbar_init(final_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
    tma_prefetch_desc(&tmap_out);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Both CTAs' barriers are initialised and the pair's TMEM allocated before either signals the other.
  cluster_sync_all();
  pdl_launch_dependents();

  if (warp == 0) {
    if (elect_one()) {
      const uint32_t full_leader = map_to_rank(smem_u32(full), 0);
      uint32_t stage = 0, phase = 0;
      uint32_t last_parity[STAGES];
      bool used[STAGES];
      for (int s = 0; s < STAGES; ++s) used[s] = false;
      bool ok = true;
      pdl_wait();
      for (uint32_t t = pair; t < tiles && ok; t += pairs) {
        const int32_t m0 = int32_t((t / p.n_tiles) * 256 + rank * 128);
        const int32_t n0 = int32_t((t % p.n_tiles) * kPairBN + rank * 128);
        for (uint32_t kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, kWatchEmpty, abort_flag)) { ok = false; break; }
          uint8_t* a_dst = smem + stage * L::kStageBytes;
          // The leader expects both CTAs' bytes on its barrier.
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * L::kStageBytes);
          const uint32_t bar = full_leader + stage * 8;
          tma_load_2d_pair(a_dst, &tmap_a, bar, int32_t(kb * kBK), m0);
          tma_load_2d_pair(a_dst + L::kABytes, &tmap_b, bar, int32_t(kb * kBK), n0);
          used[stage] = true;
          last_parity[stage] = phase;
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      // The copies complete on the leader's barrier; a stage's last use is over once the MMA released it here.
      for (int s = 0; s < STAGES; ++s)
        if (used[s]) mbar_wait(&empty[s], last_parity[s], kWatchEmpty, nullptr);
    }
  } else if (warp == 1) {
    if (leader && elect_one()) {
      constexpr uint32_t idesc = make_idesc_bf16(256, kPairBN, 0, 0);
      const uint32_t peer_empty = map_to_rank(smem_u32(empty), 1);
      const uint32_t peer_acc_full = map_to_rank(smem_u32(acc_full), 1);
      uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
      bool ok = true;
      for (uint32_t t = pair; t < tiles && ok; t += pairs) {
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u, kWatchAccEmpty, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kPairBN;
        for (uint32_t kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, kWatchFull, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * L::kStageBytes);
          const uint32_t b_addr = a_addr + L::kABytes;
#pragma unroll
          for (uint32_t kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t a_desc = make_smem_desc(a_addr + kk * 32, 16, 1024, kLayoutSw128);
            const uint64_t b_desc = make_smem_desc(b_addr + kk * 32, 16, 1024, kLayoutSw128);
            umma_bf16_pair(d_tmem, a_desc, b_desc, idesc, (kb | kk) != 0u);
          }
          umma_commit_pair(smem_u32(&empty[stage]));
          umma_commit_pair(peer_empty + stage * 8);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit_pair(smem_u32(&acc_full[acc]));
        umma_commit_pair(peer_acc_full + acc * 8);
        acc ^= 1u;
        if (acc == 0) acc_phase ^= 1u;
      }
      // Drain every MMA this thread issued before the pair's TMEM is freed.
      umma_commit_pair(smem_u32(final_bar));
      mbar_wait(final_bar, 0, kWatchOther, nullptr);
    }
  } else {
    // Epilogue: this CTA's 128 rows of each 256 x 256 tile, sixteen warps as in the row-major kernel.
    const uint32_t lane_base = 32u * (warp & 3u);
    const uint32_t group = (warp - 2) >> 2;
    constexpr uint32_t kGroupCols = kPairBN / kRowEpiGroups;
    constexpr uint32_t kCW = 32;
    const uint32_t acc_empty_leader = map_to_rank(smem_u32(acc_empty), 0);
    const bool gelu = (p.flags & TEMPO_GEMM_GELU) != 0;
    // This warp's 32 x 32 staging tile: row `lane` at 64 bytes, its four 16-byte words swizzled by (lane / 2) % 4
    // (the TMA 64-byte swizzle, which also spreads the warp's writes over all banks).
    uint8_t* staging = smem + L::kStagingOffset + (warp - 2) * 2048;
    uint8_t* stage_row = staging + lane * 64;
    const uint32_t swizzle = (lane >> 1) & 3u;
    uint32_t acc = 0, acc_phase = 0;
    pdl_wait();
    for (uint32_t t = pair; t < tiles; t += pairs) {
      if (!mbar_wait(&acc_full[acc], acc_phase, kWatchAccFull, abort_flag)) break;
      tc_fence_after();
      const uint32_t row0 = (t / p.n_tiles) * 256 + rank * 128 + lane_base;  // this warp's first row
      const uint32_t row = row0 + lane;
      const uint32_t n_base = (t % p.n_tiles) * kPairBN;
#pragma unroll 1
      for (uint32_t c = group * kGroupCols; c < (group + 1) * kGroupCols; c += kCW) {
        uint32_t r[kCW];
        tmem_ld_32x32b_x32(tmem_base + (lane_base << 16) + acc * kPairBN + c, r);
        tmem_wait_ld();
        const uint32_t n0 = n_base + c;
        if (row0 >= p.m || n0 >= p.n) continue;  // warp-uniform: the whole 32 x 32 block lies outside
        // The staging tile is free once the previous store from it has been read.
        if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
        __syncwarp();
        epilogue_chunk<kCW, true>(p, r, row, n0, gelu, false, 0.f, 0.f, stage_row, swizzle);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        // Rows past M and columns past N are clipped by the copy.
        if (lane == 0) {
          tma_store_2d(&tmap_out, staging, int32_t(n0), int32_t(row0));
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty_leader + acc * 8);
      acc ^= 1u;
      if (acc == 0) acc_phase ^= 1u;
    }
  }

  // Every output store has completed; both CTAs are done with the pair's TMEM and shared memory before either frees
  // or leaves.
  if (warp >= 2 && lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  tc_fence_before();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

template <int STAGES>
tempo_status launch_pair(const void* a, uint32_t lda, const void* w_t, uint32_t ldw, const RowMajorParams& base,
                         cudaStream_t stream) {
  using L = PairSmem<STAGES>;
  CUtensorMap ta, tb;
  const uint64_t a_dims[2] = {base.k, base.m};
  const uint64_t a_strides[1] = {uint64_t(lda) * 2};
  const uint32_t a_box[2] = {kBK, 128};
  tempo_status s = encode_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a, a_dims, a_strides, a_box,
                               CU_TENSOR_MAP_SWIZZLE_128B);
  if (s != TEMPO_OK) return s;
  const uint64_t b_dims[2] = {base.k, base.n};
  const uint64_t b_strides[1] = {uint64_t(ldw) * 2};
  const uint32_t b_box[2] = {kBK, 128};
  s = encode_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w_t, b_dims, b_strides, b_box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (s != TEMPO_OK) return s;
  CUtensorMap to;
  const uint64_t o_dims[2] = {base.n, base.m};
  const uint64_t o_strides[1] = {uint64_t(base.ldo) * 2};
  const uint32_t o_box[2] = {32, 32};
  s = encode_tmap(&to, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base.out, o_dims, o_strides, o_box,
                  CU_TENSOR_MAP_SWIZZLE_64B);
  if (s != TEMPO_OK) return s;
  RowMajorParams p = base;
  p.m_tiles = (p.m + 255) / 256;
  p.n_tiles = (p.n + kPairBN - 1) / kPairBN;
  const uint32_t tiles = p.m_tiles * p.n_tiles;
  auto kernel = gemm_pair_kernel<STAGES>;
  s = set_smem(reinterpret_cast<const void*>(kernel), L::kBytes);
  if (s != TEMPO_OK) return s;
  // The tiles are dealt out statically, so every pair must be resident at once: as many pairs as the GPCs can hold.
  static int resident_pairs = 0;
  if (resident_pairs == 0) {
    cudaLaunchConfig_t config = {};
    config.gridDim = dim3(uint32_t(sm_count()) & ~1u);
    config.blockDim = dim3(kRowThreads);
    config.dynamicSmemBytes = L::kBytes;
    cudaLaunchAttribute attribute;
    attribute.id = cudaLaunchAttributeClusterDimension;
    attribute.val.clusterDim.x = 2;
    attribute.val.clusterDim.y = 1;
    attribute.val.clusterDim.z = 1;
    config.attrs = &attribute;
    config.numAttrs = 1;
    int clusters = 0;
    const cudaError_t err = cudaOccupancyMaxActiveClusters(&clusters, kernel, &config);
    if (err != cudaSuccess || clusters <= 0) return cuda_fail(err, "cudaOccupancyMaxActiveClusters(gemm_pair_kernel)");
    resident_pairs = clusters;
  }
  const uint32_t pairs = tiles < uint32_t(resident_pairs) ? tiles : uint32_t(resident_pairs);
  return launch(kernel, dim3(2 * pairs), dim3(kRowThreads), L::kBytes, stream, 2, "gemm_pair_kernel", ta, tb, to, p);
}

// Picks a split-K configuration for a GEMM whose 128-row tiles alone leave SMs idle: the most CTAs (tiles x splits,
// two or more splits) that still fit one wave, each split keeping at least two k-blocks. Returns false when the
// plain kernel is better (including when only an unsplit grid fits: the persistent kernel runs that without a
// reduction step).
// How many clusters of the split-K kernel <BN, SPLITS> the device holds at once (cudaOccupancyMaxActiveClusters at
// its largest shared-memory size), cached per device; 0 if the query fails. A cluster needs its CTAs' SMs inside one
// GPC, so a grid of clusters can need a second wave although its CTAs number fewer than the SMs: measured on a B200,
// 36 clusters of 4 (the QKV projection of 192-256 rows) took 11.4 us against 5.0-5.5 for one wave of full-K tiles.
template <int BN, int SPLITS, int STAGES>
uint32_t splitk_resident_clusters() {
  using L = SplitSmem<BN, SPLITS, STAGES>;
  static std::mutex mu;
  static std::map<int, uint32_t> known;
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return 0;
  std::lock_guard<std::mutex> lock(mu);
  const auto it = known.find(device);
  if (it != known.end()) return it->second;
  auto kernel = gemm_splitk_kernel<BN, SPLITS, STAGES>;
  uint32_t result = 0;
  if (set_smem(reinterpret_cast<const void*>(kernel), L::bytes(STAGES)) == TEMPO_OK) {
    cudaLaunchConfig_t config = {};
    config.gridDim = dim3(SPLITS);
    config.blockDim = dim3(kSplitThreads);
    config.dynamicSmemBytes = L::bytes(STAGES);
    cudaLaunchAttribute attribute;
    attribute.id = cudaLaunchAttributeClusterDimension;
    attribute.val.clusterDim.x = SPLITS;
    attribute.val.clusterDim.y = 1;
    attribute.val.clusterDim.z = 1;
    config.attrs = &attribute;
    config.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &config) == cudaSuccess && clusters > 0)
      result = uint32_t(clusters);
    else
      (void)cudaGetLastError();
  }
  known[device] = result;
  return result;
}

uint32_t splitk_resident_clusters(uint32_t bn, uint32_t splits) {
  if (bn == 128) return splits == 2 ? splitk_resident_clusters<128, 2, 4>()
                        : splits == 4 ? splitk_resident_clusters<128, 4, 4>() : splitk_resident_clusters<128, 8, 4>();
  return splits == 2 ? splitk_resident_clusters<64, 2, 6>()
         : splits == 4 ? splitk_resident_clusters<64, 4, 6>() : splitk_resident_clusters<64, 8, 6>();
}

// Full-K row-major tiles for a decode-sized product (one wave of tiles covers it): the tile width (16, 32, 64 or
// 128 columns) that minimises an estimate of the operand time, the slowest CTA's A rows and BN weight rows over K at
// the rate one SM draws from L2 (about 60 GB/s) plus the whole grid's bytes at the aggregate rate (about 20 TB/s).
// The constants are fitted to a sweep of the GPT-2 decode projections (64-512 rows, K = 768) on a B200, where the
// estimate picks a width within 3 % of the fastest in 17 of 18 cases. 0 when no width fits one wave.
uint32_t pick_full_k_width(uint32_t m, uint32_t n, uint32_t k) {
  const uint64_t sms = uint64_t(sm_count()), m_tiles = (m + 127) / 128;
  const double a_rows = m <= 64 ? 64.0 : 128.0;
  uint32_t best = 0;
  double best_cost = 0.0;
  for (uint32_t bn : {16u, 32u, 64u, 128u}) {
    const uint64_t tiles = m_tiles * ((n + bn - 1) / bn);
    if (tiles > sms) continue;
    const double per_cta = (a_rows + bn) * k * 2.0;                // bytes
    const double cost = per_cta / 60e3 + double(tiles) * per_cta / 20e6;  // microseconds
    if (best == 0 || cost < best_cost) {
      best = bn;
      best_cost = cost;
    }
  }
  return best;
}

bool pick_split(uint32_t m, uint32_t n, uint32_t k, uint32_t* bn, uint32_t* splits) {
  const uint32_t sms = uint32_t(sm_count());
  const uint32_t m_tiles = (m + 127) / 128, kblocks = (k + kBK - 1) / kBK;
  if (uint64_t(m_tiles) * ((n + 127) / 128) >= sms) return false;
  uint32_t best_ctas = 0;
  for (uint32_t cand_bn : {128u, 64u}) {
    const uint32_t tiles = m_tiles * ((n + cand_bn - 1) / cand_bn);
    for (uint32_t s : {2u, 4u, 8u}) {
      const uint64_t ctas = uint64_t(tiles) * s;
      if (ctas > sms || kblocks < 2 * s) continue;
      if (tiles > splitk_resident_clusters(cand_bn, s)) continue;  // the clusters must all be resident at once
      if (ctas > best_ctas) {
        best_ctas = uint32_t(ctas);
        *bn = cand_bn;
        *splits = s;
      }
    }
  }
  return best_ctas > 0;
}

}  // namespace

}  // namespace tempo

using namespace tempo;

// The LayerNorm folded into a projection (TEMPO_GEMM_LN): FP32 column sums of the folded weights, the folded bias
// and the epsilon.
struct LnFold {
  const float* colsum = nullptr;
  const float* bias = nullptr;
  float eps = 0.f;
  const float2* stats = nullptr;  // the rows' statistics partials from their producer (else computed in-kernel)
};

static tempo_status gemm_impl(const void* a, uint32_t lda, const void* w_t, uint32_t ldw, const void* bias,
                              const void* residual, uint32_t ldr, void* out, uint32_t ldo, uint32_t m, uint32_t n,
                              uint32_t k, uint32_t flags, float* part_val, int32_t* part_idx, const KvStore& kv,
                              const LnFold& ln, void* stream, float2* row_stats = nullptr);

extern "C" tempo_status tempo_gemm(const void* a, uint32_t lda, const void* w_t, uint32_t ldw, const void* bias,
                                   const void* residual, uint32_t ldr, void* out, uint32_t ldo, uint32_t m,
                                   uint32_t n, uint32_t k, uint32_t flags, float* part_val, int32_t* part_idx,
                                   void* stream) {
  if (flags & TEMPO_GEMM_LN) return fail(TEMPO_ERR_VALUE, "tempo_gemm: TEMPO_GEMM_LN is tempo_gemm_ln's mode");
  return gemm_impl(a, lda, w_t, ldw, bias, residual, ldr, out, ldo, m, n, k, flags, part_val, part_idx, KvStore{},
                   LnFold{}, stream);
}

extern "C" tempo_status tempo_gemm_qkv(const void* a, uint32_t lda, const void* w_t, uint32_t ldw, const void* bias,
                                       void* out, uint32_t ldo, uint32_t m, uint32_t k, void* k_cache, void* v_cache,
                                       uint32_t seqs, uint32_t heads, uint32_t head, uint32_t capacity,
                                       uint32_t tokens_per_seq, const int32_t* positions, void* stream) {
  const uint32_t width = heads * head;
  if (k_cache == nullptr || v_cache == nullptr || !aligned16(k_cache) || !aligned16(v_cache))
    return fail(TEMPO_ERR_VALUE, "tempo_gemm_qkv: both caches are needed, 16-byte aligned");
  if (heads == 0 || head == 0 || head % 32 || seqs == 0 || capacity == 0 ||
      (positions == nullptr && tokens_per_seq == 0))
    return fail(TEMPO_ERR_VALUE, "tempo_gemm_qkv: heads %u head %u (multiple of 32) seqs %u capacity %u tokens %u",
                heads, head, seqs, capacity, tokens_per_seq);
  KvStore kv{static_cast<uint16_t*>(k_cache), static_cast<uint16_t*>(v_cache), positions, tokens_per_seq, seqs,
             heads, head, capacity, width};
  return gemm_impl(a, lda, w_t, ldw, bias, nullptr, 0, out, ldo, m, 3 * width, k, 0, nullptr, nullptr, kv, LnFold{},
                   stream);
}

extern "C" tempo_status tempo_gemm_rowstats(const void* a, uint32_t lda, const void* w_t, uint32_t ldw,
                                            const void* bias, const void* residual, uint32_t ldr, void* out,
                                            uint32_t ldo, uint32_t m, uint32_t n, uint32_t k, uint32_t flags,
                                            float* row_stats, void* stream) {
  if (row_stats == nullptr || (reinterpret_cast<uintptr_t>(row_stats) & 7u) || n % 16 ||
      (flags & (TEMPO_GEMM_LN | TEMPO_GEMM_ARGMAX)))
    return fail(TEMPO_ERR_VALUE, "tempo_gemm_rowstats: 8-byte aligned statistics, N (%u) a multiple of 16, no argmax "
                "or folded LayerNorm", n);
  return gemm_impl(a, lda, w_t, ldw, bias, residual, ldr, out, ldo, m, n, k, flags, nullptr, nullptr, KvStore{},
                   LnFold{}, stream, reinterpret_cast<float2*>(row_stats));
}

static tempo_status gemm_ln_impl(const void* x, uint32_t ldx, const void* w_t_folded, uint32_t ldw,
                                 const float* colsum, const float* bias_folded, float epsilon, const float2* stats,
                                 void* out, uint32_t ldo, uint32_t m, uint32_t n, uint32_t k, uint32_t flags,
                                 void* k_cache, void* v_cache, uint32_t seqs, uint32_t heads, uint32_t head,
                                 uint32_t capacity, const int32_t* positions, void* stream);

extern "C" tempo_status tempo_gemm_ln(const void* x, uint32_t ldx, const void* w_t_folded, uint32_t ldw,
                                      const float* colsum, const float* bias_folded, float epsilon, void* out,
                                      uint32_t ldo, uint32_t m, uint32_t n, uint32_t k, uint32_t flags, void* k_cache,
                                      void* v_cache, uint32_t seqs, uint32_t heads, uint32_t head, uint32_t capacity,
                                      const int32_t* positions, void* stream) {
  return gemm_ln_impl(x, ldx, w_t_folded, ldw, colsum, bias_folded, epsilon, nullptr, out, ldo, m, n, k, flags,
                      k_cache, v_cache, seqs, heads, head, capacity, positions, stream);
}

extern "C" tempo_status tempo_gemm_ln_rowstats(const void* x, uint32_t ldx, const void* w_t_folded, uint32_t ldw,
                                               const float* colsum, const float* bias_folded, float epsilon,
                                               const float* row_stats, void* out, uint32_t ldo, uint32_t m, uint32_t n,
                                               uint32_t k, uint32_t flags, void* k_cache, void* v_cache, uint32_t seqs,
                                               uint32_t heads, uint32_t head, uint32_t capacity,
                                               const int32_t* positions, void* stream) {
  if (row_stats == nullptr || (reinterpret_cast<uintptr_t>(row_stats) & 7u) || k % 16 || k > 1024)
    return fail(TEMPO_ERR_VALUE, "tempo_gemm_ln_rowstats: 8-byte aligned statistics, K (%u) a multiple of 16, <= 1024",
                k);
  return gemm_ln_impl(x, ldx, w_t_folded, ldw, colsum, bias_folded, epsilon,
                      reinterpret_cast<const float2*>(row_stats), out, ldo, m, n, k, flags, k_cache, v_cache, seqs,
                      heads, head, capacity, positions, stream);
}

static tempo_status gemm_ln_impl(const void* x, uint32_t ldx, const void* w_t_folded, uint32_t ldw,
                                 const float* colsum, const float* bias_folded, float epsilon, const float2* stats,
                                 void* out, uint32_t ldo, uint32_t m, uint32_t n, uint32_t k, uint32_t flags,
                                 void* k_cache, void* v_cache, uint32_t seqs, uint32_t heads, uint32_t head,
                                 uint32_t capacity, const int32_t* positions, void* stream) {
  if (colsum == nullptr || bias_folded == nullptr || !aligned16(colsum) || !aligned16(bias_folded))
    return fail(TEMPO_ERR_VALUE, "tempo_gemm_ln: column sums and folded bias are needed, 16-byte aligned");
  if (flags & ~TEMPO_GEMM_GELU) return fail(TEMPO_ERR_VALUE, "tempo_gemm_ln: only TEMPO_GEMM_GELU may be set");
  KvStore kv{};
  if (k_cache != nullptr || v_cache != nullptr) {
    const uint32_t width = heads * head;
    if (k_cache == nullptr || v_cache == nullptr || !aligned16(k_cache) || !aligned16(v_cache) || positions == nullptr)
      return fail(TEMPO_ERR_VALUE, "tempo_gemm_ln: the cache store needs both caches (16-byte aligned) and positions");
    if (heads == 0 || head == 0 || head % 32 || seqs == 0 || capacity == 0 || n != 3 * width)
      return fail(TEMPO_ERR_VALUE, "tempo_gemm_ln: heads %u head %u (multiple of 32) seqs %u capacity %u, N %u", heads,
                  head, seqs, capacity, n);
    kv = KvStore{static_cast<uint16_t*>(k_cache), static_cast<uint16_t*>(v_cache), positions, 0, seqs, heads, head,
                 capacity, width};
  }
  return gemm_impl(x, ldx, w_t_folded, ldw, nullptr, nullptr, 0, out, ldo, m, n, k, flags | TEMPO_GEMM_LN, nullptr,
                   nullptr, kv, LnFold{colsum, bias_folded, epsilon, stats}, stream);
}

extern "C" tempo_status tempo_gemm_norm(const void* x, uint32_t ldx, const void* gamma, const void* beta,
                                        float epsilon, const void* w_t, uint32_t ldw, const void* bias, void* out,
                                        uint32_t ldo, uint32_t m, uint32_t n, uint32_t k, uint32_t flags,
                                        float* part_val, int32_t* part_idx, void* k_cache, void* v_cache,
                                        uint32_t heads, uint32_t head, uint32_t capacity, const int32_t* positions,
                                        void* stream) {
  if (m == 0 || m > 8 || n == 0 || k == 0 || k > 1024 || k % 8 || ldx % 8 || ldx < k || ldw % 8 || ldw < k)
    return fail(TEMPO_ERR_VALUE, "tempo_gemm_norm: M %u (1..8) N %u K %u (8..1024, multiple of 8) strides %u %u", m,
                n, k, ldx, ldw);
  if (!aligned16(x) || !aligned16(gamma) || !aligned16(beta) || !aligned16(w_t) ||
      (bias != nullptr && !aligned16(bias)))
    return fail(TEMPO_ERR_VALUE, "tempo_gemm_norm: operands must be 16-byte aligned");
  if (flags & ~(TEMPO_GEMM_GELU | TEMPO_GEMM_ARGMAX))
    return fail(TEMPO_ERR_VALUE, "tempo_gemm_norm: only TEMPO_GEMM_GELU or TEMPO_GEMM_ARGMAX may be set");
  const bool argmax = (flags & TEMPO_GEMM_ARGMAX) != 0;
  if (argmax && (part_val == nullptr || part_idx == nullptr))
    return fail(TEMPO_ERR_VALUE, "tempo_gemm_norm: argmax mode needs the partial buffers");
  if (!argmax && (out == nullptr || ldo < n || ldo % 8 || !aligned16(out)))
    return fail(TEMPO_ERR_VALUE, "tempo_gemm_norm: output must be 16-byte aligned with a row stride >= N, multiple of 8");
  KvStore kv{};
  if (k_cache != nullptr || v_cache != nullptr) {
    const uint32_t width = heads * head;
    if (k_cache == nullptr || v_cache == nullptr || !aligned16(k_cache) || !aligned16(v_cache) || positions == nullptr)
      return fail(TEMPO_ERR_VALUE, "tempo_gemm_norm: the cache store needs both caches (16-byte aligned) and positions");
    if (heads == 0 || head == 0 || head % 32 || capacity == 0 || n != 3 * width)
      return fail(TEMPO_ERR_VALUE, "tempo_gemm_norm: heads %u head %u (multiple of 32) capacity %u, N %u", heads, head,
                  capacity, n);
    kv = KvStore{static_cast<uint16_t*>(k_cache), static_cast<uint16_t*>(v_cache), positions, 0, m, heads, head,
                 capacity, width};
  }
  const tempo_status s = gemv_dispatch(x, ldx, w_t, ldw, bias, nullptr, 0, out, ldo, m, n, k, flags, part_val,
                                       part_idx, kv, static_cast<cudaStream_t>(stream),
                                       static_cast<const uint16_t*>(gamma), static_cast<const uint16_t*>(beta),
                                       epsilon);
  if (s == TEMPO_ERR_VALUE) return fail(TEMPO_ERR_VALUE, "tempo_gemm_norm: %u x %u x %u does not fit the kernel", m, n, k);
  return s;
}

static tempo_status gemm_impl(const void* a, uint32_t lda, const void* w_t, uint32_t ldw, const void* bias,
                              const void* residual, uint32_t ldr, void* out, uint32_t ldo, uint32_t m, uint32_t n,
                              uint32_t k, uint32_t flags, float* part_val, int32_t* part_idx, const KvStore& kv,
                              const LnFold& ln, void* stream, float2* row_stats) {
  if (m == 0 || n == 0 || k == 0) return fail(TEMPO_ERR_VALUE, "tempo_gemm: empty problem %ux%ux%u", m, n, k);
  if (k % 8 || lda % 8 || ldw % 8 || lda < k || ldw < k)
    return fail(TEMPO_ERR_VALUE, "tempo_gemm: K (%u) and the row strides (%u, %u) must be multiples of 8 and >= K", k,
                lda, ldw);
  if (!aligned16(a) || !aligned16(w_t)) return fail(TEMPO_ERR_VALUE, "tempo_gemm: operands must be 16-byte aligned");
  const bool argmax = (flags & TEMPO_GEMM_ARGMAX) != 0;
  if (argmax && (flags & TEMPO_GEMM_LN)) return fail(TEMPO_ERR_VALUE, "tempo_gemm: argmax with a folded LayerNorm");
  if (argmax && (part_val == nullptr || part_idx == nullptr))
    return fail(TEMPO_ERR_VALUE, "tempo_gemm: argmax mode needs the partial buffers");
  if (!argmax && (out == nullptr || ldo < n || (ldo % 8) || !aligned16(out)))
    return fail(TEMPO_ERR_VALUE, "tempo_gemm: output must be 16-byte aligned with a row stride >= N, multiple of 8");
  if (residual != nullptr && (ldr < n || (ldr % 8) || !aligned16(residual)))
    return fail(TEMPO_ERR_VALUE, "tempo_gemm: residual must be 16-byte aligned with a row stride >= N, multiple of 8");
  if (bias != nullptr && !aligned16(bias)) return fail(TEMPO_ERR_VALUE, "tempo_gemm: bias must be 16-byte aligned");
  RowMajorParams p{};
  p.bias = static_cast<const uint16_t*>(bias);
  p.residual = static_cast<const uint16_t*>(residual);
  p.out = static_cast<uint16_t*>(out);
  p.part_val = part_val;
  p.part_idx = part_idx;
  p.m = m;
  p.n = n;
  p.k = k;
  p.ldo = ldo;
  p.ldr = ldr;
  p.flags = flags;
  p.kv = kv;
  p.row_stats = row_stats;
  const bool ln_mode = (flags & TEMPO_GEMM_LN) != 0;
  if (ln_mode) {
    p.ln_x = static_cast<const uint16_t*>(a);
    p.ln_ldx = lda;
    p.ln_colsum = ln.colsum;
    p.ln_bias = ln.bias;
    p.ln_eps = ln.eps;
    p.ln_stats = ln.stats;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // A handful of rows (decode of a few sequences): stream the weights on the CUDA cores instead (no statistics).
  if (m <= 8 && !ln_mode && row_stats == nullptr) {
    const tempo_status gemv = gemv_dispatch(a, lda, w_t, ldw, bias, residual, ldr, out, ldo, m, n, k, flags, part_val,
                                            part_idx, kv, st);
    if (gemv != TEMPO_ERR_VALUE) return gemv;
  }
  if (argmax) return launch_rowmajor<256, 4>(a, lda, w_t, ldw, p, st);
  // With the statistics from their producer, the folded LayerNorm runs wherever the plain projection would: narrow
  // full-K tiles for one 128-row block, else split-K.
  const bool ln_partials = ln_mode && ln.stats != nullptr;
  if (ln_partials && k <= 1024) {
    switch (pick_full_k_width(m, n, k)) {
      case 16: return launch_rowmajor<16, 8, false, true>(a, lda, w_t, ldw, p, st);
      case 32: return launch_rowmajor<32, 8, false, true>(a, lda, w_t, ldw, p, st);
      case 64: return launch_rowmajor<64, 8, false, true>(a, lda, w_t, ldw, p, st);
      case 128: return launch_rowmajor<128, 5, true, true>(a, lda, w_t, ldw, p, st);
      default: break;
    }
  }
  uint32_t bn = 0, splits = 0;
  if (ln_partials && n % 8 == 0 && pick_split(m, n, k, &bn, &splits)) {
    if (bn == 128) {
      switch (splits) {
        case 2: return launch_splitk<128, 2, 4>(a, lda, w_t, ldw, p, st);
        case 4: return launch_splitk<128, 4, 4>(a, lda, w_t, ldw, p, st);
        default: return launch_splitk<128, 8, 4>(a, lda, w_t, ldw, p, st);
      }
    }
    switch (splits) {
      case 2: return launch_splitk<64, 2, 6>(a, lda, w_t, ldw, p, st);
      case 4: return launch_splitk<64, 4, 6>(a, lda, w_t, ldw, p, st);
      default: return launch_splitk<64, 8, 6>(a, lda, w_t, ldw, p, st);
    }
  }
  if (ln_mode) {
    // The folded LayerNorm takes each tile's row statistics from its own A stages, so every CTA gets one tile: the
    // narrowest tiles (the most CTAs) that need no more tiles than SMs.
    const uint64_t sms = uint64_t(sm_count()), m_tiles = (m + 127) / 128;
    if (m <= 128 && k <= 1024 && (n + 15) / 16 <= sms) return launch_rowmajor<16, 8, false, true>(a, lda, w_t, ldw, p, st);
    if (m <= 128 && k <= 1024 && (n + 31) / 32 <= sms) return launch_rowmajor<32, 8, false, true>(a, lda, w_t, ldw, p, st);
    if (m_tiles * ((n + 63) / 64) <= sms) return launch_rowmajor<64, 8, false, true>(a, lda, w_t, ldw, p, st);
    if (m_tiles * ((n + 127) / 128) <= sms) return launch_rowmajor<128, 5, true, true>(a, lda, w_t, ldw, p, st);
    if (m_tiles * ((n + 255) / 256) <= sms) return launch_rowmajor<256, 3, true, true>(a, lda, w_t, ldw, p, st);
    return fail(TEMPO_ERR_VALUE, "tempo_gemm_ln: %u x %u needs more than one 128-row tile per SM", m, n);
  }
  // A decode-sized product with a short contraction (the decode projections): full-K tiles, at most one per SM, no
  // cross-CTA reduction; measured faster than split-K at K = 768 from 64 to 512 rows, or level with it.
  if (k <= 1024 && uint64_t((m + 127) / 128) * ((n + 127) / 128) < uint64_t(sm_count())) {
    switch (pick_full_k_width(m, n, k)) {
      case 16: return launch_rowmajor<16, 8>(a, lda, w_t, ldw, p, st);
      case 32: return launch_rowmajor<32, 8>(a, lda, w_t, ldw, p, st);
      case 64: return launch_rowmajor<64, 8>(a, lda, w_t, ldw, p, st);
      case 128: return launch_rowmajor<128, 5, true>(a, lda, w_t, ldw, p, st);
      default: break;
    }
  }
  // Small M (decode): split the contraction over a cluster so every SM has work.
  if (n % 8 == 0 && pick_split(m, n, k, &bn, &splits)) {
    if (bn == 128) {
      switch (splits) {
        case 2: return launch_splitk<128, 2, 4>(a, lda, w_t, ldw, p, st);
        case 4: return launch_splitk<128, 4, 4>(a, lda, w_t, ldw, p, st);
        default: return launch_splitk<128, 8, 4>(a, lda, w_t, ldw, p, st);
      }
    }
    switch (splits) {
      case 2: return launch_splitk<64, 2, 6>(a, lda, w_t, ldw, p, st);
      case 4: return launch_splitk<64, 4, 6>(a, lda, w_t, ldw, p, st);
      default: return launch_splitk<64, 8, 6>(a, lda, w_t, ldw, p, st);
    }
  }
  // Large problems (prefill): 256 x 256 tiles on CTA pairs, when there are at least four tiles per pair.
  if (!ln_mode && !argmax && uint64_t((m + 255) / 256) * ((n + 255) / 256) >= 4ull * (uint64_t(sm_count()) / 2))
    return launch_pair<5>(a, lda, w_t, ldw, p, st);
  // Wide tiles when the grid still fills the GPU; narrower ones otherwise.
  const uint64_t tiles256 = uint64_t((m + 127) / 128) * ((n + 255) / 256);
  if (tiles256 >= uint64_t(sm_count())) return launch_rowmajor<256, 3, true>(a, lda, w_t, ldw, p, st);
  const uint64_t tiles128 = uint64_t((m + 127) / 128) * ((n + 127) / 128);
  if (tiles128 >= uint64_t(sm_count()) / 2) return launch_rowmajor<128, 5, true>(a, lda, w_t, ldw, p, st);
  return launch_rowmajor<64, 8>(a, lda, w_t, ldw, p, st);
}

// ---------------------------------------------------------------------------------------------------------------
// Failure-detection probe: one bounded mbarrier wait that nothing completes unless asked to. It exercises, on the
// device, the path every pipeline wait takes when a copy or an MMA never arrives: the wait gives up after its limit,
// records a watchdog code, and the kernel returns, leaving the context usable.
// ---------------------------------------------------------------------------------------------------------------

namespace tempo {

__global__ void wait_probe_kernel(uint32_t arrive, unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (arrive) mbar_arrive(&bar);
    mbar_wait_for(&bar, 0, kWatchProbe, nullptr, limit_ns);
  }
}

tempo_status launch_wait_probe(uint32_t arrive, uint64_t limit_ns, cudaStream_t stream) {
  wait_probe_kernel<<<1, 32, 0, stream>>>(arrive, limit_ns);
  return check_launch("wait_probe_kernel");
}

}  // namespace tempo

extern "C" tempo_status tempo_block_gemm(const void* activations, const void* weights, void* drain, const void* bias,
                                         uint32_t depth, uint32_t columns, uint32_t activate, void* stream) {
  if (depth == 0 || columns == 0 || depth % 16 || columns % 16)
    return fail(TEMPO_ERR_VALUE, "tempo_block_gemm: depth (%u) and columns (%u) must be positive multiples of 16",
                depth, columns);
  if (!aligned16(activations) || !aligned16(weights) || !aligned16(drain) || (bias && !aligned16(bias)))
    return fail(TEMPO_ERR_VALUE, "tempo_block_gemm: operands must be 16-byte aligned");
  CUtensorMap tw, ta;
  // Weights [columns/16][depth][16]: dims (16, depth, columns/16), box (16, 64, 8).
  const uint64_t w_dims[3] = {16, depth, columns / 16};
  const uint64_t w_strides[2] = {32, uint64_t(depth) * 32};
  const uint32_t w_box[3] = {16, kBK, 8};
  tempo_status s = encode_tmap(&tw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, weights, w_dims, w_strides, w_box,
                               CU_TENSOR_MAP_SWIZZLE_32B);
  if (s != TEMPO_OK) return s;
  // Activations [depth/16][32][16]: dims (16, 32, depth/16), box (16, 32, 4).
  const uint64_t a_dims[3] = {16, 32, depth / 16};
  const uint64_t a_strides[2] = {32, 1024};
  const uint32_t a_box[3] = {16, 32, kBK / 16};
  s = encode_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, activations, a_dims, a_strides, a_box,
                  CU_TENSOR_MAP_SWIZZLE_32B);
  if (s != TEMPO_OK) return s;
  BlockParams p{static_cast<const uint16_t*>(bias), static_cast<uint16_t*>(drain), depth, columns, activate};
  s = set_smem(reinterpret_cast<const void*>(gemm_block_kernel), kBlockSmem);
  if (s != TEMPO_OK) return s;
  const uint32_t grid = (columns / 16 + 7) / 8;
  gemm_block_kernel<<<grid, kThreads, kBlockSmem, static_cast<cudaStream_t>(stream)>>>(tw, ta, p);
  return check_launch("gemm_block_kernel");
}
