// The per-element arithmetic of the decode step, shared by the kernel-per-op path (gemv.cu, attention.cu) and the
// persistent decode step (decode_step.cu), so both produce the same bits: the GEMV column dot products and the decode
// attention's online softmax over one (sequence, head) stretch of keys.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace tempo {

constexpr float kDecodeLog2e = 1.4426950408889634f;

// ---------------------------------------------------------------------------------------------------------------
// GEMV: dot products of weight rows (W^T[n][:], K contiguous) with M activation rows held in shared memory
// ---------------------------------------------------------------------------------------------------------------

// Dot products of CP weight rows (columns n0 .. n0 + CP - 1) with every activation row, summed over the warp into
// acc[c][r]. Lane l covers the 16-byte chunks l, l + 32, ... of the contraction; each pass first issues all of its
// CP x KCH weight loads (load_columns), then does the arithmetic (fma_columns), so a lane keeps up to CP x KCH loads
// in flight (the memory-level parallelism the HBM needs at a handful of rows), and passes repeat while chunks remain;
// reduce_columns closes each sum over the warp. Activation row r sits at a_smem + r * k.
template <int KCH, int CP>
__device__ __forceinline__ void load_columns(const uint16_t* __restrict__ w, uint32_t ldw, uint32_t n, uint32_t k,
                                             uint32_t n0, uint32_t base, uint4 (&wv)[CP][KCH]) {
  const uint32_t lane = lane_id();
  const uint32_t chunks = k / 8;
#pragma unroll
  for (int c = 0; c < CP; ++c) {
    const uint4* row = reinterpret_cast<const uint4*>(w + size_t(n0 + c) * ldw);
#pragma unroll
    for (int i = 0; i < KCH; ++i) {
      const uint32_t ch = base + lane + 32u * i;
      wv[c][i] = (n0 + c < n && ch < chunks) ? __ldg(row + ch) : make_uint4(0, 0, 0, 0);
    }
  }
}

template <int M, int KCH, int CP>
__device__ __forceinline__ void fma_columns(const uint4 (&wv)[CP][KCH], const uint16_t* a_smem, uint32_t k,
                                            uint32_t m, uint32_t base, float (&acc)[CP][M]) {
  const uint32_t lane = lane_id();
  const uint32_t chunks = k / 8;
#pragma unroll
  for (int i = 0; i < KCH; ++i) {
    const uint32_t ch = base + lane + 32u * i;
    if (ch >= chunks) break;
#pragma unroll
    for (int r = 0; r < M; ++r) {
      if (r >= int(m)) break;
      float av[8];
      unpack8(*reinterpret_cast<const uint4*>(a_smem + size_t(r) * k + ch * 8), av);
#pragma unroll
      for (int c = 0; c < CP; ++c) {
        float wf[8];
        unpack8(wv[c][i], wf);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[c][r] = fmaf(av[j], wf[j], acc[c][r]);
      }
    }
  }
}

template <int M, int CP>
__device__ __forceinline__ void reduce_columns(float (&acc)[CP][M]) {
#pragma unroll
  for (int c = 0; c < CP; ++c)
#pragma unroll
    for (int r = 0; r < M; ++r)
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[c][r] += __shfl_xor_sync(0xFFFFFFFFu, acc[c][r], o);
}

template <int M, int KCH, int CP>
__device__ __forceinline__ void dot_columns(const uint16_t* __restrict__ w, uint32_t ldw, uint32_t n, uint32_t k,
                                            uint32_t m, const uint16_t* a_smem, uint32_t n0, float (&acc)[CP][M]) {
#pragma unroll
  for (int c = 0; c < CP; ++c)
#pragma unroll
    for (int r = 0; r < M; ++r) acc[c][r] = 0.f;
  for (uint32_t base = 0; base < k / 8; base += 32 * KCH) {
    uint4 wv[CP][KCH];
    load_columns<KCH, CP>(w, ldw, n, k, n0, base, wv);
    fma_columns<M, KCH, CP>(wv, a_smem, k, m, base, acc);
  }
  reduce_columns<M, CP>(acc);
}

// ---------------------------------------------------------------------------------------------------------------
// Decode attention: online softmax of one lane group (8 lanes x 8 dims = one 64-wide head)
// ---------------------------------------------------------------------------------------------------------------

__device__ __forceinline__ void load8(const uint4& w, float (&f)[8]) {
  f[0] = bf16_lo(w.x); f[1] = bf16_hi(w.x); f[2] = bf16_lo(w.y); f[3] = bf16_hi(w.y);
  f[4] = bf16_lo(w.z); f[5] = bf16_hi(w.z); f[6] = bf16_lo(w.w); f[7] = bf16_hi(w.w);
}

struct DecodeState {
  float m, l, acc[8];
};

__device__ __forceinline__ void decode_state_init(DecodeState& st) {
  st.m = -INFINITY;
  st.l = 0.f;
#pragma unroll
  for (int d = 0; d < 8; ++d) st.acc[d] = 0.f;
}

// Folds KI keys (scores already in the log2 domain, -inf when absent) into the state.
template <int KI>
__device__ __forceinline__ void fold(DecodeState& st, const float (&sc)[KI], const uint4 (&vv)[KI]) {
  float mb = sc[0];
#pragma unroll
  for (int i = 1; i < KI; ++i) mb = fmaxf(mb, sc[i]);
  const float m_new = fmaxf(st.m, mb);
  if (m_new == -INFINITY) return;
  const float corr = fast_exp2(st.m - m_new);
  float pr[KI], psum = 0.f;
#pragma unroll
  for (int i = 0; i < KI; ++i) {
    pr[i] = fast_exp2(sc[i] - m_new);
    psum += pr[i];
  }
  st.l = st.l * corr + psum;
#pragma unroll
  for (int d = 0; d < 8; ++d) st.acc[d] *= corr;
#pragma unroll
  for (int i = 0; i < KI; ++i) {
    float v[8];
    load8(vv[i], v);
#pragma unroll
    for (int d = 0; d < 8; ++d) st.acc[d] = fmaf(pr[i], v[d], st.acc[d]);
  }
  st.m = m_new;
}

// Merges the state of lane groups `offset` lanes apart (xor shuffle).
__device__ __forceinline__ void merge_shfl(DecodeState& st, int offset) {
  const float om = __shfl_xor_sync(0xFFFFFFFFu, st.m, offset);
  const float ol = __shfl_xor_sync(0xFFFFFFFFu, st.l, offset);
  float oa[8];
#pragma unroll
  for (int d = 0; d < 8; ++d) oa[d] = __shfl_xor_sync(0xFFFFFFFFu, st.acc[d], offset);
  const float m_new = fmaxf(st.m, om);
  if (m_new == -INFINITY) return;
  const float a = fast_exp2(st.m - m_new), b = fast_exp2(om - m_new);
  st.l = st.l * a + ol * b;
#pragma unroll
  for (int d = 0; d < 8; ++d) st.acc[d] = st.acc[d] * a + oa[d] * b;
  st.m = m_new;
}

// The lane group's dot product of the (log2-scaled) query with one key, reduced over its 8 lanes.
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

// One warp's share of a decode stretch [k_begin, k_end): keys base, base + 16 KI, ... from k_begin + 4 KI warp, KI per
// lane group per iteration, each key's 64 dims split over the group's 8 lanes. LOAD(ptr) fetches a 16-byte chunk.
template <int KI, typename Load>
__device__ __forceinline__ void decode_stretch(DecodeState& st, const float (&q)[8], const uint4* kb4, const uint4* vb4,
                                               int32_t k_begin, int32_t k_end, uint32_t warp, uint32_t g, uint32_t li,
                                               Load load) {
  for (int32_t base = k_begin + int32_t(warp) * 4 * KI; base < k_end; base += 16 * KI) {
    uint4 kk[KI], vv[KI];
#pragma unroll
    for (int i = 0; i < KI; ++i) {
      const int32_t key = base + i * 4 + int32_t(g);
      if (key < k_end) {
        kk[i] = load(kb4 + size_t(key) * 8 + li);
        vv[i] = load(vb4 + size_t(key) * 8 + li);
      } else {
        kk[i] = make_uint4(0, 0, 0, 0);
        vv[i] = make_uint4(0, 0, 0, 0);
      }
    }
    float sc[KI];
#pragma unroll
    for (int i = 0; i < KI; ++i) {
      const float v = group_dot(q, kk[i]);
      sc[i] = (base + i * 4 + int32_t(g) < k_end) ? v : -INFINITY;
    }
    fold<KI>(st, sc, vv);
  }
}

// The keys of chunk `chunk` of `chunks` for a cache holding `len` keys: a multiple of 32 per chunk.
__device__ __forceinline__ void decode_chunk_range(int32_t len, uint32_t chunks, uint32_t chunk, int32_t& k_begin,
                                                   int32_t& k_end) {
  const int32_t per = ((len + int32_t(chunks) - 1) / int32_t(chunks) + 31) & ~31;
  k_begin = min(len, int32_t(chunk) * per);
  k_end = min(len, k_begin + per);
}

// Merges four warps' states (sm_m[4], sm_l[4], sm_acc[4][64], filled by each warp's lane group 0) for output
// dimension d: the (max, sum, weighted value) of the stretch.
__device__ __forceinline__ void merge_warps(const float* sm_m, const float* sm_l, const float (*sm_acc)[64], uint32_t d,
                                            float& m, float& l, float& a) {
  m = -INFINITY;
  l = 0.f;
  a = 0.f;
  for (int w = 0; w < 4; ++w) m = fmaxf(m, sm_m[w]);
  if (m != -INFINITY) {
    for (int w = 0; w < 4; ++w) {
      const float f = fast_exp2(sm_m[w] - m);
      l += sm_l[w] * f;
      a += sm_acc[w][d] * f;
    }
  }
}

// Merges `chunks` stretch partials (max, sum, 64 values; `stride` floats apart) for dimension d into the output value;
// load(ptr) reads one float of the partials.
template <typename Load>
__device__ __forceinline__ float merge_chunks(const float* part, uint32_t stride, uint32_t chunks, uint32_t d,
                                              Load load) {
  float mm = -INFINITY;
  for (uint32_t c = 0; c < chunks; ++c) mm = fmaxf(mm, load(part + c * stride));
  float ll = 0.f, aa = 0.f;
  if (mm != -INFINITY) {
    for (uint32_t c = 0; c < chunks; ++c) {
      const float f = fast_exp2(load(part + c * stride) - mm);
      ll += load(part + c * stride + 1) * f;
      aa += load(part + c * stride + 2 + d) * f;
    }
  }
  return ll > 0.f ? aa / ll : 0.f;
}

}  // namespace tempo
