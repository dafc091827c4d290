// Shared device helpers for the sm_100a kernels: BF16 conversion, mbarriers with bounded waits, TMA tensor loads,
// and the tcgen05 (5th-generation tensor core) instructions with their shared-memory and instruction descriptors.
//
// Every wait on an mbarrier is bounded: after kWaitLimitNs of global time the waiting thread records a watchdog
// error (g_tempo_watchdog) and returns false, so a pipeline bug ends the kernel with a status the host reads
// instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace tempo {

// ---------------------------------------------------------------------------------------------------------------
// Watchdog
// ---------------------------------------------------------------------------------------------------------------

// Set (to a code naming the wait that gave up) by any bounded wait that expires. One copy per translation unit;
// each unit that waits defines a host reader with TEMPO_WATCHDOG_READER, which the runtime polls and clears.
static __device__ int g_tempo_watchdog = 0;

#define TEMPO_WATCHDOG_READER(fn)                                            \
  int fn() {                                                                 \
    int value = 0, zero = 0;                                                 \
    if (cudaMemcpyFromSymbol(&value, g_tempo_watchdog, sizeof(int)) != cudaSuccess) return -1; \
    if (value != 0) cudaMemcpyToSymbol(g_tempo_watchdog, &zero, sizeof(int)); \
    return value;                                                            \
  }

constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s of global time per wait

enum WatchdogCode : int {
  kWatchFull = 1,      // consumer waiting for a TMA stage
  kWatchEmpty = 2,     // producer waiting for a free stage
  kWatchAccFull = 3,   // epilogue waiting for the accumulator
  kWatchAccEmpty = 4,  // MMA waiting for the epilogue to drain the accumulator
  kWatchOther = 5,
  kWatchProbe = 6,     // the failure-detection probe's wait, which nothing completes unless asked to
};

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------------------------------------------
// BF16
// ---------------------------------------------------------------------------------------------------------------

__device__ __forceinline__ float bf16_lo(uint32_t pair) { return __uint_as_float(pair << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t pair) { return __uint_as_float(pair & 0xFFFF0000u); }
__device__ __forceinline__ float bf16_to_float(uint16_t word) { return __uint_as_float(uint32_t(word) << 16); }

// Round-to-nearest-even float -> BF16 (cuda_bf16's conversion is RNE).
__device__ __forceinline__ uint16_t float_to_bf16(float v) {
  __nv_bfloat16 b = __float2bfloat16_rn(v);
  return *reinterpret_cast<uint16_t*>(&b);
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&p);
}
__device__ __forceinline__ float round_bf16(float v) { return bf16_to_float(float_to_bf16(v)); }

// 1/x on the special-function unit (PTX rcp.approx.ftz.f32).
__device__ __forceinline__ float fast_rcp(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x on the special-function unit (PTX ex2.approx.ftz.f32).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// GELU with the exact normal CDF, x Phi(x). With z = |x| / sqrt 2 and t = 1 / (1 + z / 2), the tail
// c = erfc(z) / 2 = t 2^(P(t) - z^2 log2 e), P a degree-8 polynomial fitted to log2(erfcx(z) / 2t) over z <= 9.5
// (fit_gelu.py beside this file derives the coefficients); Phi = 1 - c for x >= 0 and c for x < 0. Relative error
// below 1e-5 over every BF16 input whose Phi(x) is a normal float, x > -13 (c is computed directly, so there is no
// cancellation in 1 + erf for negative x); in 16 FP32 operations and two special-function ones.
__device__ __forceinline__ float gelu_erf(float x) {
  const float t = fast_rcp(fmaf(fabsf(x), 0.35355339059327373f, 1.0f));
  float p = 0.11508675664663315f;
  p = fmaf(p, t, -0.8110487461090088f);
  p = fmaf(p, t, 2.1534459590911865f);
  p = fmaf(p, t, -2.604888916015625f);
  p = fmaf(p, t, 1.2568824291229248f);
  p = fmaf(p, t, -0.3535706400871277f);
  p = fmaf(p, t, 0.6373199224472046f);
  p = fmaf(p, t, 1.4320268630981445f);
  p = fmaf(p, t, -2.825253963470459f);
  const float tail = t * fast_exp2(fmaf(x, x * -0.72134752044448170f, p));
  return x * (x < 0.f ? tail : 1.0f - tail);
}

// Two floats in one 64-bit register pair for Blackwell's paired FP32 instructions (PTX fma / mul / add .rn.f32x2):
// one instruction computes both halves, each rounded exactly as its scalar form.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t r, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(r));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_splat(float c) { return f2_pack(c, c); }

// The largest of three floats in one instruction (PTX max.f32 with three inputs, sm_100 and later); a NaN operand is
// ignored, as by fmaxf.
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// gelu_erf of two values with paired instructions: the same operations in the same order, so the same results, in
// about half the FP32 issue slots.
__device__ __forceinline__ void gelu_erf_pair(float& a, float& b) {
  const uint64_t x = f2_pack(a, b);
  const uint64_t t = f2_pack(fast_rcp(fmaf(fabsf(a), 0.35355339059327373f, 1.0f)),
                             fast_rcp(fmaf(fabsf(b), 0.35355339059327373f, 1.0f)));
  uint64_t p = f2_fma(f2_splat(0.11508675664663315f), t, f2_splat(-0.8110487461090088f));
  p = f2_fma(p, t, f2_splat(2.1534459590911865f));
  p = f2_fma(p, t, f2_splat(-2.604888916015625f));
  p = f2_fma(p, t, f2_splat(1.2568824291229248f));
  p = f2_fma(p, t, f2_splat(-0.3535706400871277f));
  p = f2_fma(p, t, f2_splat(0.6373199224472046f));
  p = f2_fma(p, t, f2_splat(1.4320268630981445f));
  p = f2_fma(p, t, f2_splat(-2.825253963470459f));
  float ea, eb;
  f2_unpack(f2_fma(x, f2_mul(x, f2_splat(-0.72134752044448170f)), p), ea, eb);
  float ta, tb;
  f2_unpack(f2_mul(t, f2_pack(fast_exp2(ea), fast_exp2(eb))), ta, tb);
  a = a * (a < 0.f ? ta : 1.0f - ta);
  b = b * (b < 0.f ? tb : 1.0f - tb);
}

// (mean, M2) of 16 values: the mean, then the sum of squared deviations from it. The row statistics partials a
// projection writes for the LayerNorm folded into the projection after it.
__device__ __forceinline__ float2 chunk_stats16(const float (&w)[16]) {
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < 16; ++j) s += w[j];
  const float mean = s * (1.f / 16.f);
  float m2 = 0.f;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float d = w[j] - mean;
    m2 = fmaf(d, d, m2);
  }
  return make_float2(mean, m2);
}

// ---------------------------------------------------------------------------------------------------------------
// Shared memory addressing and mbarriers
// ---------------------------------------------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar_addr, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar_addr), "r"(parity)
      : "memory");
  return done != 0;
}

// Waits for the phase with the given parity to complete. Returns false (and records `code`) if it has not after
// `limit_ns` of global time, or if `abort` (a shared flag another role sets when it gives up) becomes non-zero.
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, int code, volatile int* abort,
                                              unsigned long long limit_ns) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const unsigned long long start = global_ns();
  for (uint32_t spin = 1;; ++spin) {
    if (mbar_try_wait(addr, parity)) return true;
    if ((spin & 255u) == 0u) {
      if (abort != nullptr && *abort) return false;
      if (global_ns() - start > limit_ns) {
        atomicExch(&g_tempo_watchdog, code);
        if (abort != nullptr) *abort = 1;
        return false;
      }
    }
  }
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int code, volatile int* abort) {
  return mbar_wait_for(bar, parity, code, abort, kWaitLimitNs);
}

// ---------------------------------------------------------------------------------------------------------------
// TMA (tensor memory accelerator) loads into shared memory, completing on an mbarrier
// ---------------------------------------------------------------------------------------------------------------

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int32_t c0, int32_t c1,
                                            int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int32_t c0, int32_t c1,
                                            int32_t c2, int32_t c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], [%2];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2),
        "r"(c3)
      : "memory");
}

// Orders this thread's generic-proxy shared-memory writes before later async-proxy reads (tcgen05.mma operands).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------------------------------------------
// tcgen05: tensor memory allocation, MMA, commit, loads
// ---------------------------------------------------------------------------------------------------------------

// Allocates `columns` (a power of two >= 32) TMEM columns; the base address lands in *dst (shared memory). Must be
// executed by one whole warp.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t columns) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(columns)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t base, uint32_t columns) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(columns) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] x B[smem desc], kind::f16 (BF16 inputs, FP32 accumulate per the instruction descriptor).
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on `bar` when every tcgen05 operation this thread issued so far has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// D[tmem] (+)= A[tmem] x B[smem desc]: the A operand (M rows on TMEM lanes, K packed two BF16 per 32-bit column) is
// read from tensor memory.
__device__ __forceinline__ void umma_bf16_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 lanes x 32 bits, 16 consecutive columns: thread t writes lane (base lane + t), columns c..c+15.
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// 32 lanes x 32 bits, 32 consecutive columns: thread t of the warp receives lane (base lane + t), columns c..c+31.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// ---------------------------------------------------------------------------------------------------------------
// UMMA descriptors
// ---------------------------------------------------------------------------------------------------------------

// Shared-memory matrix descriptor layout types (sm_100).
enum : uint32_t { kLayoutNone = 0, kLayoutSw128 = 2, kLayoutSw64 = 4, kLayoutSw32 = 6 };

// Builds a shared-memory matrix descriptor: start address, leading/stride byte offsets (bytes, multiples of 16),
// version 1 (Blackwell), base offset 0 (the swizzle atom is aligned), and the layout type.
__device__ __forceinline__ uint64_t make_smem_desc(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                                   uint32_t layout) {
  uint64_t desc = 0;
  desc |= uint64_t((smem_addr >> 4) & 0x3FFFu);
  desc |= uint64_t((lbo_bytes >> 4) & 0x3FFFu) << 16;
  desc |= uint64_t((sbo_bytes >> 4) & 0x3FFFu) << 32;
  desc |= uint64_t(1) << 46;
  desc |= uint64_t(layout & 0x7u) << 61;
  return desc;
}

// Instruction descriptor for kind::f16 with BF16 A and B, FP32 D. a_mn/b_mn select MN-major operands.
__host__ __device__ constexpr uint32_t make_idesc_bf16(uint32_t m, uint32_t n, uint32_t a_mn, uint32_t b_mn) {
  return (1u << 4)          // D format: F32
         | (1u << 7)        // A format: BF16
         | (1u << 10)       // B format: BF16
         | (a_mn << 15)     // A major
         | (b_mn << 16)     // B major
         | ((n >> 3) << 17)  // N / 8
         | ((m >> 4) << 24);  // M / 16
}

// ---------------------------------------------------------------------------------------------------------------
// Programmatic dependent launch: a kernel launched with programmatic stream serialization may start while the
// kernel before it in the stream is still running. It does its independent set-up (barriers, TMEM, weight
// prefetch), then waits for that kernel's completion and memory before touching anything the kernel wrote.
// Without the launch attribute both instructions are no-ops.
// ---------------------------------------------------------------------------------------------------------------

// Blocks until every prerequisite grid has completed and its memory operations are visible.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Lets the next grid in the stream begin launching once every CTA of this grid has executed it (or exited). Called
// after this CTA holds its tensor memory, so a dependent CTA can never take TMEM this grid still needs.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// ---------------------------------------------------------------------------------------------------------------
// KV-cache store fused into the QKV projection's epilogue
// ---------------------------------------------------------------------------------------------------------------

// Where the QKV product's key and value columns also go: caches [seqs][heads][capacity][head]. Row r of the product
// is sequence r / tokens at position r % tokens (prefill), or sequence r at positions[r] (decode).
struct KvStore {
  uint16_t* k;  // null: no cache store
  uint16_t* v;
  const int32_t* positions;
  uint32_t tokens, seqs, heads, head, capacity, width;  // width = heads * head (the query columns)
};

// The cache address of columns [col, col + count) of row `row` when they are key or value columns (count stays
// inside one head), or null.
__device__ __forceinline__ uint16_t* kv_destination(const KvStore& kv, uint32_t row, uint32_t col) {
  if (kv.k == nullptr || col < kv.width) return nullptr;
  const uint32_t which = (col - kv.width) / kv.width;
  const uint32_t feature = (col - kv.width) % kv.width;
  const uint32_t seq = kv.positions != nullptr ? row : row / kv.tokens;
  const uint32_t pos = kv.positions != nullptr ? uint32_t(kv.positions[row]) : row % kv.tokens;
  if (which > 1 || seq >= kv.seqs || pos >= kv.capacity) return nullptr;
  return (which ? kv.v : kv.k) + ((size_t(seq) * kv.heads + feature / kv.head) * kv.capacity + pos) * kv.head +
         feature % kv.head;
}

__device__ __forceinline__ uint32_t warp_id() { return threadIdx.x >> 5; }
__device__ __forceinline__ uint32_t lane_id() { return threadIdx.x & 31u; }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

__device__ __forceinline__ void unpack8(const uint4& w, float (&f)[8]) {
  f[0] = bf16_lo(w.x); f[1] = bf16_hi(w.x); f[2] = bf16_lo(w.y); f[3] = bf16_hi(w.y);
  f[4] = bf16_lo(w.z); f[5] = bf16_hi(w.z); f[6] = bf16_lo(w.w); f[7] = bf16_hi(w.w);
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 w;
  w.x = pack_bf16x2(f[0], f[1]); w.y = pack_bf16x2(f[2], f[3]);
  w.z = pack_bf16x2(f[4], f[5]); w.w = pack_bf16x2(f[6], f[7]);
  return w;
}

// The LayerNorm's per-element steps, written out (explicit fused multiply-adds) so that every kernel normalising a
// row rounds exactly alike: the centred square accumulated, and (x - mean) rstd gamma + beta.
__device__ __forceinline__ float ln_square_add(float x, float mean, float acc) {
  const float d = x - mean;
  return fmaf(d, d, acc);
}
__device__ __forceinline__ float ln_apply(float x, float mean, float scale, float gamma, float beta) {
  return fmaf((x - mean) * scale, gamma, beta);
}

// One row's LayerNorm by one warp: lane l holds the row's 16-byte chunks l, l + 32, ... (up to CPL of them, `features`
// / 8 in all); mean, centred variance, rsqrt(var + epsilon), then (x - mean) rstd gamma + beta rounded to BF16, chunk
// c handed to store(c, word) (layernorm_row: into `orow`, global or shared memory); gamma and beta are read with
// load (default: the read-only path). The standalone LayerNorm and the small-M projections that normalise their own
// input share it, so both produce the same bits; a larger CPL than needed only skips chunks, in the same order.
// Reads 16 bytes of read-only data (the LayerNorm's gamma and beta) through the read-only path.
struct ReadOnlyLoad {
  __device__ __forceinline__ uint4 operator()(const uint4* p) const { return __ldg(p); }
};

template <int CPL, typename Store, typename Load = ReadOnlyLoad>
__device__ __forceinline__ void layernorm_row_to(const uint16_t* __restrict__ xr, const uint16_t* __restrict__ gamma,
                                                 const uint16_t* __restrict__ beta, uint32_t features, float epsilon,
                                                 Store store, Load load = Load()) {
  const uint32_t lane = lane_id();
  const uint32_t chunks = features / 8;
  float v[CPL][8];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    const uint32_t c = lane + 32u * i;
    if (c < chunks) {
      unpack8(*reinterpret_cast<const uint4*>(xr + c * 8), v[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) sum += v[i][j];
    }
  }
  const float inv_f = 1.0f / float(features);
  const float mean = warp_sum(sum) * inv_f;
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    if (lane + 32u * i < chunks) {
#pragma unroll
      for (int j = 0; j < 8; ++j) sq = ln_square_add(v[i][j], mean, sq);
    }
  }
  const float scale = rsqrtf(warp_sum(sq) * inv_f + epsilon);
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    const uint32_t c = lane + 32u * i;
    if (c < chunks) {
      float g[8], b[8];
      unpack8(load(reinterpret_cast<const uint4*>(gamma + c * 8)), g);
      unpack8(load(reinterpret_cast<const uint4*>(beta + c * 8)), b);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = ln_apply(v[i][j], mean, scale, g[j], b[j]);
      store(c, pack8(v[i]));
    }
  }
}

template <int CPL>
__device__ __forceinline__ void layernorm_row(const uint16_t* __restrict__ xr, const uint16_t* __restrict__ gamma,
                                              const uint16_t* __restrict__ beta, uint32_t features, float epsilon,
                                              uint16_t* orow) {
  layernorm_row_to<CPL>(xr, gamma, beta, features, epsilon,
                        [orow](uint32_t c, const uint4& w) { *reinterpret_cast<uint4*>(orow + c * 8) = w; });
}

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, 0xFFFFFFFF;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

}  // namespace tempo
