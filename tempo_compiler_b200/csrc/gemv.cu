// GEMV-shaped products for decode with a handful of sequences (M <= 8 rows): bandwidth-bound, so they stream the
// weight rows (W^T[n][:], contiguous) once with 16-byte loads on the CUDA cores, the lanes of a warp splitting the
// contraction and a warp-shuffle reduction closing each output. The activations (M x K, at most 48 KB) sit in shared
// memory. A weight row's first lines are prefetched into L2 before waiting on the previous kernel, so the stream
// starts while that kernel drains. Epilogues match the tensor-core GEMM: + bias, exact-erf GELU of the BF16-rounded
// sum, + residual, or a fused argmax over each 256-column tile (the LM head).
#include <cuda_runtime.h>

#include "common.cuh"
#include "decode_math.cuh"
#include "host.hpp"

namespace tempo {
namespace {

constexpr int kWarps = 8;
constexpr uint32_t kArgmaxTile = 256;  // columns one argmax partial covers (matches the tensor-core path)

struct GemvParams {
  const uint16_t* a;  // [m, lda]
  const uint16_t* w;  // [n, ldw] (W transposed, K contiguous)
  const uint16_t* bias;
  const uint16_t* residual;
  uint16_t* out;
  float* part_val;
  int32_t* part_idx;
  uint32_t m, n, k, lda, ldw, ldr, ldo, flags, tiles;
  KvStore kv;
  // Optional LayerNorm of the input rows (gamma non-null): every CTA normalises the M rows of `a` itself, exactly as
  // the standalone LayerNorm would, into its shared-memory copy of the activations.
  const uint16_t* ln_gamma;
  const uint16_t* ln_beta;
  float ln_eps;
};

constexpr uint32_t kNormMaxK = 1024;  // rows a warp normalises from registers: 4 chunks of 8 per lane

__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// One warp per output column (CP = 1), or, in argmax mode, 32 columns of the block's 256-column tile per warp taken
// CP at a time.
template <int M, int KCH, int CP>
__global__ void __launch_bounds__(kWarps * 32) gemv_kernel(GemvParams p) {
  extern __shared__ __align__(16) uint16_t a_smem[];
  __shared__ float best_val[kWarps][M];
  __shared__ int32_t best_idx[kWarps][M];
  const uint32_t warp = warp_id(), lane = lane_id();
  const bool argmax = (p.flags & TEMPO_GEMM_ARGMAX) != 0;
  const bool gelu = (p.flags & TEMPO_GEMM_GELU) != 0;
  const uint32_t warp_cols = argmax ? kArgmaxTile / kWarps : uint32_t(CP);
  const uint32_t first = (blockIdx.x * kWarps + warp) * warp_cols;

  // The weights are not the previous kernel's output: start pulling this warp's rows into L2 now.
  for (uint32_t c = 0; c < warp_cols; ++c)
    if (first + c < p.n)
      for (uint32_t line = lane; line < p.k * 2 / 128; line += 32)
        prefetch_l2(reinterpret_cast<const uint8_t*>(p.w + size_t(first + c) * p.ldw) + line * 128);
  pdl_launch_dependents();
  pdl_wait();

  if (p.ln_gamma != nullptr) {
    // warp r normalises row r (M <= 8 = warps)
    if (warp < p.m)
      layernorm_row<kNormMaxK / 256>(p.a + size_t(warp) * p.lda, p.ln_gamma, p.ln_beta, p.k, p.ln_eps,
                                     a_smem + size_t(warp) * p.k);
  } else {
    for (uint32_t i = threadIdx.x; i < p.m * (p.k / 8); i += blockDim.x) {
      const uint32_t r = i / (p.k / 8), ch = i % (p.k / 8);
      reinterpret_cast<uint4*>(a_smem)[i] = *reinterpret_cast<const uint4*>(p.a + size_t(r) * p.lda + ch * 8);
    }
  }
  __syncthreads();

  float best[M];
  int32_t idx[M];
#pragma unroll
  for (int r = 0; r < M; ++r) { best[r] = -INFINITY; idx[r] = 0; }

  for (uint32_t c0 = 0; c0 < warp_cols; c0 += CP) {
    const uint32_t n0 = first + c0;
    if (n0 >= p.n) break;
    float acc[CP][M];
    dot_columns<M, KCH, CP>(p.w, p.ldw, p.n, p.k, p.m, a_smem, n0, acc);
    if (argmax) {
#pragma unroll
      for (int c = 0; c < CP; ++c)
#pragma unroll
        for (int r = 0; r < M; ++r)
          if (n0 + c < p.n && acc[c][r] > best[r]) { best[r] = acc[c][r]; idx[r] = int32_t(n0 + c); }
      continue;
    }
    // Lane (c * M + r) finishes column n0 + c of row r.
#pragma unroll
    for (int c = 0; c < CP; ++c) {
#pragma unroll
      for (int r = 0; r < M; ++r) {
        if (lane != uint32_t(c * M + r) || r >= int(p.m) || n0 + c >= p.n) continue;
        const uint32_t col = n0 + c;
        float v = acc[c][r];
        if (p.bias != nullptr) v += bf16_to_float(p.bias[col]);
        if (gelu) v = gelu_erf(round_bf16(v));
        if (p.residual != nullptr) v += bf16_to_float(p.residual[size_t(r) * p.ldr + col]);
        const uint16_t word = float_to_bf16(v);
        p.out[size_t(r) * p.ldo + col] = word;
        uint16_t* cache = kv_destination(p.kv, r, col);
        if (cache != nullptr) *cache = word;
      }
    }
  }
  if (argmax) {
    if (lane == 0) {
#pragma unroll
      for (int r = 0; r < M; ++r) { best_val[warp][r] = best[r]; best_idx[warp][r] = idx[r]; }
    }
    __syncthreads();
    // Warps cover ascending column ranges, so a strict comparison keeps the first index on a tie.
    if (threadIdx.x < p.m) {
      const uint32_t r = threadIdx.x;
      float v = best_val[0][r];
      int32_t j = best_idx[0][r];
      for (int w = 1; w < kWarps; ++w)
        if (best_val[w][r] > v) { v = best_val[w][r]; j = best_idx[w][r]; }
      p.part_val[size_t(r) * p.tiles + blockIdx.x] = v;
      p.part_idx[size_t(r) * p.tiles + blockIdx.x] = j;
    }
  }
}

template <int M, int KCH, int CP>
tempo_status launch_gemv_shape(const GemvParams& p, cudaStream_t stream) {
  const bool argmax = (p.flags & TEMPO_GEMM_ARGMAX) != 0;
  const uint32_t cols_per_block = argmax ? kArgmaxTile : kWarps * CP;
  const uint32_t blocks = (p.n + cols_per_block - 1) / cols_per_block;
  const size_t smem = size_t(p.m) * p.k * 2;
  tempo_status s = set_smem(reinterpret_cast<const void*>(gemv_kernel<M, KCH, CP>), 96 * 1024);
  if (s != TEMPO_OK) return s;
  return launch(gemv_kernel<M, KCH, CP>, dim3(blocks), dim3(kWarps * 32), smem, stream, 1, "gemv_kernel", p);
}

// Chunks per lane and pass: the whole contraction for K <= 768 (3) and K <= 3072 (12, one column at a time), else
// passes of 4. The argmax tile's 32 columns per warp go several at a time.
template <int M>
tempo_status launch_gemv(const GemvParams& p, cudaStream_t stream) {
  const bool argmax = (p.flags & TEMPO_GEMM_ARGMAX) != 0;
  const uint32_t per_lane = (p.k / 8 + 31) / 32;
  if (argmax) {
    // four columns at a time for one or two rows; two for more, which keeps two CTAs resident per SM
    if (per_lane <= 3) return launch_gemv_shape<M, 3, (M <= 2 ? 4 : 2)>(p, stream);
    return launch_gemv_shape<M, 4, 2>(p, stream);
  }
  if (per_lane <= 3) return launch_gemv_shape<M, 3, 1>(p, stream);
  if (per_lane <= 12 && per_lane > 4) return launch_gemv_shape<M, 12, 1>(p, stream);
  return launch_gemv_shape<M, 4, 1>(p, stream);
}

}  // namespace

// Routes a small-M product to the GEMV kernels; returns TEMPO_ERR_VALUE (without launching) when it does not apply.
tempo_status gemv_dispatch(const void* a, uint32_t lda, const void* w_t, uint32_t ldw, const void* bias,
                           const void* residual, uint32_t ldr, void* out, uint32_t ldo, uint32_t m, uint32_t n,
                           uint32_t k, uint32_t flags, float* part_val, int32_t* part_idx, const KvStore& kv,
                           cudaStream_t stream, const uint16_t* ln_gamma, const uint16_t* ln_beta, float ln_eps) {
  if (m == 0 || m > 8 || k % 8 || size_t(m) * k * 2 > 96 * 1024) return TEMPO_ERR_VALUE;
  if (ln_gamma != nullptr && (k > kNormMaxK || ln_beta == nullptr || lda % 8)) return TEMPO_ERR_VALUE;
  GemvParams p{};
  p.a = static_cast<const uint16_t*>(a);
  p.w = static_cast<const uint16_t*>(w_t);
  p.bias = static_cast<const uint16_t*>(bias);
  p.residual = static_cast<const uint16_t*>(residual);
  p.out = static_cast<uint16_t*>(out);
  p.part_val = part_val;
  p.part_idx = part_idx;
  p.m = m;
  p.n = n;
  p.k = k;
  p.lda = lda;
  p.ldw = ldw;
  p.ldr = ldr;
  p.ldo = ldo;
  p.flags = flags;
  p.tiles = (n + kArgmaxTile - 1) / kArgmaxTile;
  p.kv = kv;
  p.ln_gamma = ln_gamma;
  p.ln_beta = ln_beta;
  p.ln_eps = ln_eps;
  if (m == 1) return launch_gemv<1>(p, stream);
  if (m == 2) return launch_gemv<2>(p, stream);
  if (m <= 4) return launch_gemv<4>(p, stream);
  return launch_gemv<8>(p, stream);
}

}  // namespace tempo
