// One greedy decode step of up to 8 sequences as one persistent kernel: one CTA per SM, launched cooperatively (every
// CTA resident), the step's phases separated by grid-wide barriers instead of kernel boundaries.
//
//   embed -> per layer [LayerNorm 1 + QKV + cache store | attention | out-projection + residual |
//                       LayerNorm 2 + FC + GELU | second projection + residual] -> final LayerNorm + LM head argmax
//
// The kernel-per-op path runs these as 5 kernels per layer (tempo_gemm_norm, tempo_decode_attention, tempo_gemm,
// tempo_gemm_norm, tempo_gemm); a small decode step is bound by those boundaries, not by its bytes (a few MB per
// kernel). Every output element is computed with the same arithmetic as there (decode_math.cuh's dot products and
// online softmax, common.cuh's LayerNorm, the same chunking of each attention stretch, the same merge order, the same
// epilogue), so the tokens are bit-identical to the kernel-per-op path.
//
// Data written inside the kernel by other CTAs (the hidden rows, QKV, attention partials, the new cache row) is read
// with L2-coherent loads (ld.global.cg) or staged through shared memory, never through the read-only path. A grid
// barrier is an arrival counter and a generation word in the workspace (release/acquire at GPU scope); a wait gives up
// after a bounded time, records watchdog code 7 and makes every CTA leave at its next barrier.
#include <cuda_runtime.h>

#include "common.cuh"
#include "decode_math.cuh"
#include "host.hpp"

namespace tempo {

TEMPO_WATCHDOG_READER(watchdog_decode_step)

namespace {

constexpr int kStepWarps = 8;
constexpr uint32_t kStepThreads = kStepWarps * 32;
constexpr int kStepMaxLayers = 16;
constexpr uint32_t kStepMaxChunks = 8;
constexpr int kWatchGridBarrier = 7;

struct StepLayer {
  const uint16_t *ln1_g, *ln1_b, *w_qkv, *b_qkv, *w_proj, *b_proj, *ln2_g, *ln2_b, *w_fc, *b_fc, *w_out, *b_out;
  uint16_t *k_cache, *v_cache;
};

struct StepParams {
  StepLayer layer[kStepMaxLayers];
  const uint16_t *wte, *wpe, *lnf_g, *lnf_b;
  int32_t* ids;
  int32_t* positions;
  int32_t* tokens_out;
  uint32_t out_stride;
  int32_t index_offset;
  // workspace sections
  uint32_t* sync;  // [0, 1] the barrier's 64-bit arrival count, [2] abort, [3] LM-head arrivals
  uint16_t *x, *qkv, *attn, *h;
  float* part;
  uint32_t* pair_done;  // per (sequence, head): stretches finished this step
  float* head_val;
  int32_t* head_idx;
  uint32_t layers, rows, width, heads, vocab, max_positions, capacity, chunks, runs;
  float eps;
};

__device__ __forceinline__ uint64_t ld_relaxed_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t ld_relaxed_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint4 ld_cg4(const void* p) { return __ldcg(reinterpret_cast<const uint4*>(p)); }

// A 16-byte read-only load the compiler keeps where it is written (volatile): a value loaded ahead of a barrier is
// then held in registers across it instead of being reloaded after it.
__device__ __forceinline__ uint4 ld_pinned(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

// The grid barrier: a 64-bit arrival counter that only grows. Every launch starts with it at a multiple of the grid
// size (each launch's barriers all complete), so a CTA reading it at entry, before its first arrival, rounds down to
// that base even if faster CTAs have arrived already; barrier b of the launch opens when the counter reaches
// base + (b + 1) x grid. An arrival is a release add, the wait a relaxed poll followed by an acquire fence; a wait
// gives up after kWaitLimitNs, records watchdog code 7 and raises the abort flag, which every CTA checks on its way
// through each barrier.
struct GridBarrier {
  uint64_t* count;
  uint32_t* abort_flag;
  uint64_t base;
  uint32_t index;

  __device__ void init(uint32_t* sync) {
    count = reinterpret_cast<uint64_t*>(sync);
    abort_flag = sync + 2;
    __shared__ uint64_t base_s;
    if (threadIdx.x == 0) base_s = (ld_relaxed_u64(count) / gridDim.x) * gridDim.x;
    __syncthreads();
    base = base_s;
    index = 0;
  }

  // Returns false (for every thread of the CTA) if a wait gave up, here or in another CTA.
  __device__ bool sync() {
    __shared__ int pass;
    __syncthreads();
    ++index;
    if (threadIdx.x == 0) {
      int ok = 1;
      asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(count) : "memory");
      const uint64_t target = base + uint64_t(index) * gridDim.x;
      const unsigned long long start = global_ns();
      for (uint32_t spin = 0; ld_relaxed_u64(count) < target; ++spin) {
        if ((spin & 63u) == 63u) {
          if (ld_relaxed_u32(abort_flag) != 0u) { ok = 0; break; }
          if (global_ns() - start > kWaitLimitNs) {
            atomicExch(&g_tempo_watchdog, kWatchGridBarrier);
            atomicExch(abort_flag, 1u);
            ok = 0;
            break;
          }
        }
      }
      asm volatile("fence.acq_rel.gpu;" ::: "memory");
      if (ld_relaxed_u32(abort_flag) != 0u) ok = 0;
      pass = ok;
    }
    __syncthreads();
    return pass != 0;
  }
};

// rows x k BF16 from global memory (written in this kernel) into shared memory, row stride k.
__device__ __forceinline__ void stage_rows(const uint16_t* src, uint32_t rows, uint32_t k, uint16_t* dst) {
  const uint32_t per_row = k / 8;
  for (uint32_t i = threadIdx.x; i < rows * per_row; i += blockDim.x)
    reinterpret_cast<uint4*>(dst)[i] = ld_cg4(src + size_t(i) * 8);
}

struct SharedLoad {
  __device__ __forceinline__ uint4 operator()(const uint4* p) const { return *p; }
};

// Warp r < rows normalises staged row r into `out` (the standalone LayerNorm's arithmetic), gamma and beta staged in
// shared memory.
__device__ __forceinline__ void norm_rows(const uint16_t* x_s, uint32_t rows, uint32_t width, const uint16_t* gamma_s,
                                          const uint16_t* beta_s, float eps, uint16_t* out) {
  const uint32_t warp = warp_id();
  if (warp < rows) {
    uint16_t* orow = out + size_t(warp) * width;
    layernorm_row_to<4>(x_s + size_t(warp) * width, gamma_s, beta_s, width, eps,
                        [orow](uint32_t c, const uint4& w) { *reinterpret_cast<uint4*>(orow + c * 8) = w; },
                        SharedLoad());
  }
}

enum Epilogue : uint32_t { kBias = 0, kBiasGelu = 1, kBiasResidual = 2 };

// A warp's CP consecutive columns of one phase, their weights loaded (one pass covers the whole contraction) before
// the barrier that precedes the phase, so the phase itself only reads activations. Warp w of the grid takes columns
// [w CP, w CP + CP).
template <int KCH, int CP>
struct Group {
  uint4 wv[CP][KCH];
  uint16_t bias[CP];
  uint16_t residual;  // this lane's epilogue slot (column c = lane / M, row r = lane % M), when the phase adds one
  uint32_t n0;
};

// Loads the group's weights and bias words and, when `residual` is set, this lane's residual word: everything the
// phase needs except its activations, so all of it is in flight before the barrier that precedes the phase. The
// residual must already be final (written before the previous barrier).
template <int M, int KCH, int CP>
__device__ __forceinline__ void preload(Group<KCH, CP>& g, const uint16_t* w, const uint16_t* bias, uint32_t n,
                                        uint32_t k, const uint16_t* residual, uint32_t ldr, uint32_t rows) {
  g.n0 = (blockIdx.x * kStepWarps + warp_id()) * CP;
  if (g.n0 >= n) return;
  // Volatile loads: the compiler may neither drop them for a reload after the barrier nor move them past it.
  const uint32_t lane = lane_id();
#pragma unroll
  for (int c = 0; c < CP; ++c) {
    const uint4* row = reinterpret_cast<const uint4*>(w + size_t(g.n0 + c) * k);
#pragma unroll
    for (int i = 0; i < KCH; ++i) {
      const uint32_t ch = lane + 32u * i;
      g.wv[c][i] = make_uint4(0, 0, 0, 0);
      if (g.n0 + c < n && ch < k / 8) g.wv[c][i] = ld_pinned(row + ch);
    }
  }
#pragma unroll
  for (int c = 0; c < CP; ++c) g.bias[c] = g.n0 + c < n ? __ldg(bias + g.n0 + c) : uint16_t(0);
  const uint32_t c = lane / M, r = lane % M;
  g.residual = 0;
  if (residual != nullptr && c < uint32_t(CP) && r < rows && g.n0 + c < n) {
    uint16_t word;
    asm volatile("ld.global.cg.u16 %0, [%1];" : "=h"(word) : "l"(residual + size_t(r) * ldr + g.n0 + c));
    g.residual = word;
  }
}

// The group's columns of rows x (A in shared memory, stride k) @ W^T, then + bias, [GELU], [+ residual], rounded to
// BF16 into out[r * ldo + col], and into the caches when kv.k is set (the GEMV epilogue's arithmetic).
template <int M, int KCH, int CP>
__device__ __forceinline__ void finish(const Group<KCH, CP>& g, const uint16_t* a_s, uint32_t n, uint32_t k,
                                       uint32_t rows, Epilogue epilogue, uint16_t* out, uint32_t ldo,
                                       const KvStore& kv) {
  if (g.n0 >= n) return;
  float acc[CP][M];
#pragma unroll
  for (int c = 0; c < CP; ++c)
#pragma unroll
    for (int r = 0; r < M; ++r) acc[c][r] = 0.f;
  fma_columns<M, KCH, CP>(g.wv, a_s, k, rows, 0, acc);
  reduce_columns<M, CP>(acc);
  const uint32_t lane = lane_id();
#pragma unroll
  for (int c = 0; c < CP; ++c) {
#pragma unroll
    for (int r = 0; r < M; ++r) {
      const uint32_t col = g.n0 + c;
      if (lane != uint32_t(c * M + r) || uint32_t(r) >= rows || col >= n) continue;
      float v = acc[c][r];
      v += bf16_to_float(g.bias[c]);
      if (epilogue == kBiasGelu) v = gelu_erf(round_bf16(v));
      if (epilogue == kBiasResidual) v += bf16_to_float(g.residual);
      const uint16_t word = float_to_bf16(v);
      out[size_t(r) * ldo + col] = word;
      uint16_t* cache = kv_destination(kv, r, col);
      if (cache != nullptr) *cache = word;
    }
  }
}

// Columns per grid warp in the LM head's argmax (a contiguous range each, taken CP at a time).
__device__ __forceinline__ uint32_t head_span(uint32_t vocab) {
  const uint32_t warps = gridDim.x * kStepWarps;
  return (vocab + warps - 1) / warps;
}

template <int M>
__global__ void __launch_bounds__(kStepThreads, 1) decode_step_kernel(const __grid_constant__ StepParams p) {
  // Dynamic shared memory: A rows (rows x up to 4 x width: the second projection's input) | staged hidden rows
  // (rows x width) | the next LayerNorm's gamma and beta (2 x width).
  extern __shared__ __align__(16) uint16_t a_s[];
  uint16_t* x_s = a_s + size_t(M) * 4 * p.width;
  uint16_t* lnp_s = x_s + size_t(M) * p.width;
  __shared__ float sm_m[2][4], sm_l[2][4], sm_acc[2][4][64];  // attention: one set per half CTA
  __shared__ int merge_turn[2];
  const uint32_t warp = warp_id(), lane = lane_id();
  const uint32_t rows = p.rows, width = p.width, heads = p.heads;
  const uint32_t threads = gridDim.x * blockDim.x, tid = blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t gwarp = blockIdx.x * kStepWarps + warp;
  constexpr int kHeadCP = M <= 2 ? 4 : 2;

  Group<3, 2> gq;   // QKV: 2 columns per warp
  Group<3, 1> go;   // out-projection
  Group<3, 3> gf;   // FC: 3 columns per warp
  Group<12, 1> g2;  // second projection (K = 4 width)
  preload<M>(gq, p.layer[0].w_qkv, p.layer[0].b_qkv, 3 * width, width, nullptr, 0, rows);
  // Each row's position, read by the cache store and the attention of every layer.
  __shared__ int32_t pos_s[8];
  if (threadIdx.x < rows) pos_s[threadIdx.x] = p.positions[threadIdx.x];
  GridBarrier barrier;
  barrier.init(p.sync);

  // The next LayerNorm's gamma and beta: fetched into registers at the start of the phase before it and written to
  // shared memory (lnp_s: gamma then beta) at that phase's end, so the normalising phase finds them there.
  const uint32_t ln_words = 2 * width / 8;
  uint4 ln_next = make_uint4(0, 0, 0, 0);
  auto ln_fetch = [&](const uint16_t* gamma, const uint16_t* beta) {
    if (threadIdx.x < ln_words) {
      const uint32_t half_words = width / 8;
      ln_next = threadIdx.x < half_words ? __ldg(reinterpret_cast<const uint4*>(gamma) + threadIdx.x)
                                         : __ldg(reinterpret_cast<const uint4*>(beta) + threadIdx.x - half_words);
    }
  };
  auto ln_store = [&]() {
    if (threadIdx.x < ln_words) reinterpret_cast<uint4*>(lnp_s)[threadIdx.x] = ln_next;
  };
  ln_fetch(p.layer[0].ln1_g, p.layer[0].ln1_b);

  // Embedding of each row's token at its position (the embedding kernel's arithmetic).
  for (uint32_t i = tid; i < rows * (width / 8); i += threads) {
    const uint32_t r = i / (width / 8), c = i % (width / 8);
    const int32_t id = p.ids[r], pos = p.positions[r];
    uint4 word = make_uint4(0, 0, 0, 0);
    if (uint32_t(id) < p.vocab && uint32_t(pos) < p.max_positions) {
      float a[8], b[8];
      unpack8(__ldg(reinterpret_cast<const uint4*>(p.wte + size_t(id) * width) + c), a);
      unpack8(__ldg(reinterpret_cast<const uint4*>(p.wpe + size_t(pos) * width) + c), b);
#pragma unroll
      for (int j = 0; j < 8; ++j) a[j] += b[j];
      word = pack8(a);
    }
    reinterpret_cast<uint4*>(p.x + size_t(r) * width)[c] = word;
  }
  ln_store();
  if (!barrier.sync()) return;

  const uint32_t pairs = rows * heads, units = pairs * p.chunks;
  const KvStore none{nullptr, nullptr, nullptr, 0, 0, 0, 0, 0, 0};
  for (uint32_t li = 0; li < p.layers; ++li) {
    const StepLayer& L = p.layer[li];
    const KvStore kv{L.k_cache, L.v_cache, pos_s, 0, rows, heads, 64, p.capacity, width};

    // 1. LayerNorm 1, QKV + bias, and this step's keys and values into the caches.
    stage_rows(p.x, rows, width, x_s);
    __syncthreads();
    norm_rows(x_s, rows, width, lnp_s, lnp_s + width, p.eps, a_s);
    __syncthreads();
    finish<M>(gq, a_s, 3 * width, width, rows, kBias, p.qkv, 3 * width, kv);
    // The out-projection's residual is the hidden state, final since the previous layer.
    preload<M>(go, L.w_proj, L.b_proj, width, width, p.x, width, rows);
    if (!barrier.sync()) return;

    // 2. Attention: (pair, chunk) units, one per half CTA (4 warps), each a stretch of one sequence's cache for one
    //    head; a unit of a split pair leaves (max, sum, 64 values) for the next phase to merge.
    {
      const uint32_t half = warp >> 2, wl = warp & 3u, g = lane >> 3, lg = lane & 7u;
      const uint32_t d = (warp & 3u) * 32 + lane;
      for (uint32_t u = blockIdx.x * 2 + half; u < units; u += gridDim.x * 2) {
        const uint32_t pair = u / p.chunks, chunk = u % p.chunks;
        const uint32_t s = pair / heads, h = pair % heads;
        const int32_t len = max(0, min(pos_s[s] + 1, int32_t(p.capacity)));
        int32_t k_begin, k_end;
        decode_chunk_range(len, p.chunks, chunk, k_begin, k_end);
        float q[8];
        load8(ld_cg4(p.qkv + size_t(s) * 3 * width + h * 64 + lg * 8), q);
#pragma unroll
        for (int j = 0; j < 8; ++j) q[j] *= kDecodeLog2e;
        const uint4* kb4 = reinterpret_cast<const uint4*>(L.k_cache + (size_t(s) * heads + h) * p.capacity * 64);
        const uint4* vb4 = reinterpret_cast<const uint4*>(L.v_cache + (size_t(s) * heads + h) * p.capacity * 64);
        DecodeState st;
        decode_state_init(st);
        decode_stretch<4>(st, q, kb4, vb4, k_begin, k_end, wl, g, lg, [](const uint4* ptr) { return ld_cg4(ptr); });
        merge_shfl(st, 8);
        merge_shfl(st, 16);
        if (g == 0) {
#pragma unroll
          for (int j = 0; j < 8; ++j) sm_acc[half][wl][lg * 8 + j] = st.acc[j];
          if (lg == 0) { sm_m[half][wl] = st.m; sm_l[half][wl] = st.l; }
        }
        asm volatile("bar.sync %0, 128;" ::"r"(1 + half) : "memory");
        if (d < 64) {
          float m, l, a;
          merge_warps(sm_m[half], sm_l[half], sm_acc[half], d, m, l, a);
          if (p.chunks == 1) {
            p.attn[size_t(s) * width + h * 64 + d] = float_to_bf16(l > 0.f ? a / l : 0.f);
          } else {
            float* slot = p.part + (size_t(pair) * p.chunks + chunk) * 66;
            slot[2 + d] = a;
            if (d == 0) { slot[0] = m; slot[1] = l; }
          }
        }
        if (p.chunks > 1) {
          // The pair's last stretch to finish merges all of them, in chunk order (the cluster leader's merge).
          asm volatile("bar.sync %0, 128;" ::"r"(1 + half) : "memory");
          if (d == 0) {
            __threadfence();
            merge_turn[half] = atomicAdd(p.pair_done + pair, 1u) == p.chunks - 1;
            if (merge_turn[half]) {
              p.pair_done[pair] = 0u;
              __threadfence();
            }
          }
          asm volatile("bar.sync %0, 128;" ::"r"(1 + half) : "memory");
          if (merge_turn[half] && d < 64) {
            const float* part = p.part + size_t(pair) * p.chunks * 66;
            p.attn[size_t(s) * width + h * 64 + d] =
                float_to_bf16(merge_chunks(part, 66, p.chunks, d, [](const float* f) { return __ldcg(f); }));
          }
        }
        asm volatile("bar.sync %0, 128;" ::"r"(1 + half) : "memory");
      }
    }
    if (!barrier.sync()) return;

    // 3. Out-projection + bias + residual, its input the attention rows.
    ln_fetch(L.ln2_g, L.ln2_b);
    stage_rows(p.attn, rows, width, a_s);
    __syncthreads();
    finish<M>(go, a_s, width, width, rows, kBiasResidual, p.x, width, none);
    preload<M>(gf, L.w_fc, L.b_fc, 4 * width, width, nullptr, 0, rows);
    ln_store();
    if (!barrier.sync()) return;

    // 4. LayerNorm 2, FC + bias, exact-erf GELU.
    stage_rows(p.x, rows, width, x_s);
    __syncthreads();
    norm_rows(x_s, rows, width, lnp_s, lnp_s + width, p.eps, a_s);
    __syncthreads();
    finish<M>(gf, a_s, 4 * width, width, rows, kBiasGelu, p.h, 4 * width, none);
    // The second projection's residual is the out-projection's output, final since the previous barrier.
    preload<M>(g2, L.w_out, L.b_out, width, 4 * width, p.x, width, rows);
    if (!barrier.sync()) return;

    // 5. Second projection + bias + residual; then the next layer's QKV weights (or the LM head's lines into L2).
    if (li + 1 < p.layers) ln_fetch(p.layer[li + 1].ln1_g, p.layer[li + 1].ln1_b);
    else ln_fetch(p.lnf_g, p.lnf_b);
    stage_rows(p.h, rows, 4 * width, a_s);
    __syncthreads();
    finish<M>(g2, a_s, width, 4 * width, rows, kBiasResidual, p.x, width, none);
    if (li + 1 < p.layers)
      preload<M>(gq, p.layer[li + 1].w_qkv, p.layer[li + 1].b_qkv, 3 * width, width, nullptr, 0, rows);
    ln_store();
    if (!barrier.sync()) return;
  }

  // Final LayerNorm and the tied LM head's argmax: each warp of the grid takes a contiguous run of columns and keeps
  // the first maximum (strict comparison in ascending order); the runs are reduced first index first.
  stage_rows(p.x, rows, width, x_s);
  __syncthreads();
  norm_rows(x_s, rows, width, lnp_s, lnp_s + width, p.eps, a_s);
  __syncthreads();
  {
    const uint32_t span = head_span(p.vocab), first = gwarp * span;
    float best[M];
    int32_t idx[M];
#pragma unroll
    for (int r = 0; r < M; ++r) { best[r] = -INFINITY; idx[r] = 0; }
    for (uint32_t c0 = 0; c0 < span; c0 += kHeadCP) {
      const uint32_t n0 = first + c0;
      if (n0 >= p.vocab) break;
      float acc[kHeadCP][M];
      dot_columns<M, 3, kHeadCP>(p.wte, width, p.vocab, width, rows, a_s, n0, acc);
#pragma unroll
      for (int c = 0; c < kHeadCP; ++c)
#pragma unroll
        for (int r = 0; r < M; ++r)
          if (c0 + c < span && n0 + c < p.vocab && acc[c][r] > best[r]) {
            best[r] = acc[c][r];
            idx[r] = int32_t(n0 + c);
          }
    }
    if (lane == 0) {
#pragma unroll
      for (int r = 0; r < M; ++r) {
        if (uint32_t(r) >= rows) break;
        p.head_val[size_t(r) * p.runs + gwarp] = best[r];
        p.head_idx[size_t(r) * p.runs + gwarp] = first < p.vocab ? idx[r] : 0x7FFFFFFF;
      }
    }
  }

  // The last CTA to finish reduces the runs (first index on ties), records each row's token and advances its
  // position.
  __shared__ int last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    last = atomicAdd(p.sync + 3, 1u) == gridDim.x - 1;
    if (last) {
      atomicExch(p.sync + 3, 0u);
      __threadfence();
    }
  }
  __syncthreads();
  if (!last || warp >= rows) return;
  const uint32_t r = warp;
  float best = -INFINITY;
  int32_t idx = 0x7FFFFFFF;
  for (uint32_t t = lane; t < p.runs; t += 32) {
    const float v = __ldcg(p.head_val + size_t(r) * p.runs + t);
    const int32_t i = __ldcg(p.head_idx + size_t(r) * p.runs + t);
    if (v > best || (v == best && i < idx)) { best = v; idx = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xFFFFFFFFu, best, o);
    const int32_t oi = __shfl_xor_sync(0xFFFFFFFFu, idx, o);
    if (ov > best || (ov == best && oi < idx)) { best = ov; idx = oi; }
  }
  if (lane == 0) {
    p.ids[r] = idx;
    const int32_t column = p.positions[r] + p.index_offset;
    if (p.tokens_out != nullptr && column >= 0 && uint32_t(column) < p.out_stride)
      p.tokens_out[size_t(r) * p.out_stride + column] = idx;
    p.positions[r] += 1;
  }
}

// Workspace sections, each 256-byte aligned.
struct StepLayout {
  uint64_t sync, x, qkv, attn, h, part, pair_done, head_val, head_idx, bytes;
};

// LM-head partials: one per grid warp and row.
uint32_t head_runs() { return uint32_t(sm_count()) * kStepWarps; }

StepLayout step_layout(uint32_t rows, uint32_t width, uint32_t heads, uint32_t vocab) {
  auto up = [](uint64_t v) { return (v + 255) & ~uint64_t(255); };
  StepLayout l{};
  uint64_t at = 0;
  l.sync = at; at = up(at + 64);
  l.x = at; at = up(at + uint64_t(rows) * width * 2);
  l.qkv = at; at = up(at + uint64_t(rows) * 3 * width * 2);
  l.attn = at; at = up(at + uint64_t(rows) * width * 2);
  l.h = at; at = up(at + uint64_t(rows) * 4 * width * 2);
  l.part = at; at = up(at + uint64_t(rows) * heads * kStepMaxChunks * 66 * 4);
  l.pair_done = at; at = up(at + uint64_t(rows) * heads * 4);
  (void)vocab;
  const uint64_t runs = head_runs();
  l.head_val = at; at = up(at + uint64_t(rows) * runs * 4);
  l.head_idx = at; at = up(at + uint64_t(rows) * runs * 4);
  l.bytes = at;
  return l;
}

// The chunking the kernel-per-op decode attention picks for `pairs` (sequence, head) pairs (tempo_decode_attention):
// split until every SM has a CTA, each chunk keeping at least 64 keys of the capacity.
uint32_t attention_chunks(uint64_t pairs, uint32_t capacity) {
  const uint64_t target = uint64_t(sm_count());
  uint32_t chunks = 1;
  while (chunks < kStepMaxChunks && pairs * chunks < target && capacity >= 2 * 64 * chunks) chunks *= 2;
  return chunks;
}

}  // namespace
}  // namespace tempo

using namespace tempo;

extern "C" tempo_status tempo_decode_step_workspace(uint32_t rows, uint32_t width, uint32_t heads, uint32_t vocab,
                                                    uint64_t* bytes) {
  if (bytes == nullptr || rows == 0 || rows > 8 || width == 0 || heads == 0 || vocab == 0)
    return fail(TEMPO_ERR_VALUE, "tempo_decode_step_workspace: rows %u (1 to 8), width %u, heads %u, vocab %u", rows,
                width, heads, vocab);
  *bytes = step_layout(rows, width, heads, vocab).bytes;
  return TEMPO_OK;
}

extern "C" tempo_status tempo_decode_step(const tempo_decode_step_args* args, void* stream) {
  if (args == nullptr) return fail(TEMPO_ERR_VALUE, "tempo_decode_step: no arguments");
  const tempo_decode_step_args& a = *args;
  if (a.rows == 0 || a.rows > 8 || a.layers == 0 || a.layers > uint32_t(kStepMaxLayers) || a.layer == nullptr)
    return fail(TEMPO_ERR_VALUE, "tempo_decode_step: rows %u (1 to 8), layers %u (1 to %d)", a.rows, a.layers,
                kStepMaxLayers);
  if (a.heads == 0 || a.width != 768 || a.width != a.heads * 64 || a.capacity == 0 || a.vocab == 0 ||
      a.max_positions == 0)
    return fail(TEMPO_ERR_VALUE, "tempo_decode_step: width %u must be 768 (one pass of every contraction per warp) "
                                 "and heads (%u) x 64; capacity %u, vocabulary %u, positions %u", a.width, a.heads,
                a.capacity, a.vocab, a.max_positions);
  // Every warp of the grid holds one group of columns per phase: 1152 groups for the QKV projection (2 each).
  if (uint32_t(sm_count()) * kStepWarps < 3 * a.width / 2)
    return fail(TEMPO_ERR_VALUE, "tempo_decode_step: %d SMs are too few (one CTA per SM must cover %u column pairs)",
                sm_count(), 3 * a.width / 2);
  const StepLayout l = step_layout(a.rows, a.width, a.heads, a.vocab);
  if (a.workspace == nullptr || a.workspace_bytes < l.bytes || (reinterpret_cast<uintptr_t>(a.workspace) & 255u))
    return fail(TEMPO_ERR_VALUE, "tempo_decode_step: the workspace needs %llu bytes, 256-byte aligned, got %llu",
                (unsigned long long)l.bytes, (unsigned long long)a.workspace_bytes);
  if (a.ids == nullptr || a.positions == nullptr || !aligned16(a.wte) || !aligned16(a.wpe))
    return fail(TEMPO_ERR_VALUE, "tempo_decode_step: ids, positions and 16-byte aligned embeddings are required");
  StepParams p{};
  for (uint32_t i = 0; i < a.layers; ++i) {
    const tempo_decode_layer& s = a.layer[i];
    const void* ptrs[] = {s.ln1_gamma, s.ln1_beta, s.w_qkv, s.b_qkv, s.w_proj, s.b_proj, s.ln2_gamma, s.ln2_beta,
                          s.w_fc, s.b_fc, s.w_out, s.b_out, s.k_cache, s.v_cache};
    for (const void* ptr : ptrs)
      if (!aligned16(ptr) || ptr == nullptr)
        return fail(TEMPO_ERR_VALUE, "tempo_decode_step: layer %u has a missing or misaligned operand", i);
    p.layer[i] = StepLayer{static_cast<const uint16_t*>(s.ln1_gamma), static_cast<const uint16_t*>(s.ln1_beta),
                           static_cast<const uint16_t*>(s.w_qkv),     static_cast<const uint16_t*>(s.b_qkv),
                           static_cast<const uint16_t*>(s.w_proj),    static_cast<const uint16_t*>(s.b_proj),
                           static_cast<const uint16_t*>(s.ln2_gamma), static_cast<const uint16_t*>(s.ln2_beta),
                           static_cast<const uint16_t*>(s.w_fc),      static_cast<const uint16_t*>(s.b_fc),
                           static_cast<const uint16_t*>(s.w_out),     static_cast<const uint16_t*>(s.b_out),
                           static_cast<uint16_t*>(s.k_cache),         static_cast<uint16_t*>(s.v_cache)};
  }
  uint8_t* ws = static_cast<uint8_t*>(a.workspace);
  p.wte = static_cast<const uint16_t*>(a.wte);
  p.wpe = static_cast<const uint16_t*>(a.wpe);
  p.lnf_g = static_cast<const uint16_t*>(a.lnf_gamma);
  p.lnf_b = static_cast<const uint16_t*>(a.lnf_beta);
  p.ids = a.ids;
  p.positions = a.positions;
  p.tokens_out = a.tokens_out;
  p.out_stride = a.out_stride;
  p.index_offset = a.index_offset;
  p.sync = reinterpret_cast<uint32_t*>(ws + l.sync);
  p.x = reinterpret_cast<uint16_t*>(ws + l.x);
  p.qkv = reinterpret_cast<uint16_t*>(ws + l.qkv);
  p.attn = reinterpret_cast<uint16_t*>(ws + l.attn);
  p.h = reinterpret_cast<uint16_t*>(ws + l.h);
  p.part = reinterpret_cast<float*>(ws + l.part);
  p.pair_done = reinterpret_cast<uint32_t*>(ws + l.pair_done);
  p.head_val = reinterpret_cast<float*>(ws + l.head_val);
  p.head_idx = reinterpret_cast<int32_t*>(ws + l.head_idx);
  p.layers = a.layers;
  p.rows = a.rows;
  p.width = a.width;
  p.heads = a.heads;
  p.vocab = a.vocab;
  p.max_positions = a.max_positions;
  p.capacity = a.capacity;
  p.chunks = attention_chunks(uint64_t(a.rows) * a.heads, a.capacity);
  p.runs = head_runs();
  p.eps = a.epsilon;

  const uint32_t m = a.rows == 1 ? 1 : a.rows == 2 ? 2 : a.rows <= 4 ? 4 : 8;
  void (*kernel)(StepParams) = m == 1 ? decode_step_kernel<1> : m == 2 ? decode_step_kernel<2>
                               : m == 4 ? decode_step_kernel<4> : decode_step_kernel<8>;
  // A rows (up to 4 x width), the staged hidden rows, and one LayerNorm's gamma and beta
  const size_t smem = (size_t(m) * 5 + 2) * a.width * 2;
  tempo_status s = set_smem(reinterpret_cast<const void*>(kernel), int(smem));
  if (s != TEMPO_OK) return s;
  int per_sm = 0;
  cudaError_t err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kStepThreads, smem);
  if (err != cudaSuccess || per_sm < 1) return cuda_fail(err, "decode_step_kernel occupancy");
  cudaLaunchConfig_t config = {};
  config.gridDim = dim3(uint32_t(sm_count()));
  config.blockDim = dim3(kStepThreads);
  config.dynamicSmemBytes = smem;
  config.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attribute;
  attribute.id = cudaLaunchAttributeCooperative;
  attribute.val.cooperative = 1;
  config.attrs = &attribute;
  config.numAttrs = 1;
  err = cudaLaunchKernelEx(&config, kernel, p);
  if (err != cudaSuccess) return cuda_fail(err, "decode_step_kernel");
  return check_launch("decode_step_kernel");
}
