/*
 * tempo_b200.h -- C ABI of libtempo_b200.so, the B200 (sm_100a) backend for the tile ops GPT-2 small launches in
 * yeungn523/tempo-compiler.
 *
 * Plain C types only: device memory is either a 32-bit address inside the library's arena (the drop-in runtime,
 * section 1) or a raw device pointer owned by the caller (sections 2 and 3). Every entry point returns a
 * tempo_status and never aborts; tempo_last_error() returns the message of the last failure. Calls taking a
 * `stream` (a cudaStream_t, NULL for the legacy default stream) only enqueue work on it; they allocate nothing and
 * do not synchronise, so they may be captured in a CUDA graph.
 *
 * Reference interfaces each entry point replaces are cited as path:line inside the reference project.
 */
#ifndef TEMPO_B200_H
#define TEMPO_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int32_t tempo_status;

/* Status codes; the Python runtime maps each to the exception the reference raises in the same situation. */
#define TEMPO_OK 0
#define TEMPO_ERR_VALUE 1   /* malformed argument            -> ValueError   */
#define TEMPO_ERR_MEMORY 2  /* no room in the arena / host   -> MemoryError  */
#define TEMPO_ERR_KEY 3     /* pointer not handed out        -> KeyError     */
#define TEMPO_ERR_RUNTIME 4 /* launch refused or CUDA error  -> RuntimeError */
#define TEMPO_ERR_TIMEOUT 5 /* bounded wait expired          -> TimeoutError */
#define TEMPO_ERR_STATE 6   /* no device opened              -> RuntimeError */

/* Manifest kinds (board_package/images/manifest.json, mlir/lib/tempo/manifest.cpp:103-167). */
#define TEMPO_KIND_GEMM 1
#define TEMPO_KIND_GEMM_BIAS 2
#define TEMPO_KIND_ADD 3
#define TEMPO_KIND_ADD_BIAS 4
#define TEMPO_KIND_LAYERNORM 5
#define TEMPO_KIND_ATTENTION 6
#define TEMPO_KIND_DECODE_ATTENTION 7
#define TEMPO_KIND_COPY 8
#define TEMPO_KIND_HALT 9

/* Image descriptor: the bytes a drop-in "image" holds. 64 bytes, little-endian; fields by kind:
 *   gemm/gemm_bias: f[0]=depth f[1]=columns f[2]=activate f[3]=drain_words
 *   add/add_bias:   f[0]=features
 *   layernorm:      f[0]=features
 *   attention:      f[0]=tokens f[1]=heads f[2]=head width
 *   decode_attention: f[0]=keys f[1]=heads f[2]=head width f[3]=stated constants
 *   copy:           f[0]=rows f[1]=stride
 */
#define TEMPO_IMAGE_MAGIC 0x49324254u /* "TB2I" */
#define TEMPO_IMAGE_BYTES 64u
typedef struct tempo_image {
  uint32_t magic;
  uint32_t version;
  uint32_t kind;
  uint32_t reserved0;
  uint32_t f[8];
  float scalars[2];
  uint32_t checksum; /* sum of the 14 words before it, mod 2^32 */
  uint32_t reserved1;
} tempo_image;

/* ---------------------------------------------------------------------------------------------------------------
 * 1. Drop-in device runtime: replaces board_package/runtime (runtime/__init__.py:7-58). One arena of device memory
 *    per process; device addresses are 32-bit, as the reference's kernel arguments are (runtime/launch.py:112-119).
 * ------------------------------------------------------------------------------------------------------------- */

/* Opens `device` and reserves an arena of `arena_bytes` (<= 2 GiB) at kernel address 0x80000000, the first
 * 1 MiB reserved for staged images. Replaces open_device / minitpuSetDevice (runtime/device.py:38-81).
 * Calling it again with the same device is a no-op. */
tempo_status tempo_open(int device, uint64_t arena_bytes);

/* Frees the arena and every pinned host buffer. */
tempo_status tempo_close(void);

/* The arena's kernel-view map: base address, size and reserved prefix (runtime/address_space.py:8-30,180-192). */
tempo_status tempo_address_space(uint32_t* kernel_base, uint64_t* kernel_size, uint32_t* reserved);

/* First-fit allocation, 32-byte aligned, out of the arena past the reserved prefix (runtime/device.py:148-175).
 * TEMPO_ERR_VALUE for nbytes == 0, TEMPO_ERR_MEMORY when no span fits. */
tempo_status tempo_malloc(uint32_t* address, uint64_t nbytes);

/* Returns a span to the free list, coalescing neighbours (runtime/device.py:178-196). TEMPO_ERR_KEY for a pointer
 * tempo_malloc did not return. */
tempo_status tempo_free(uint32_t address);

/* Forgets every allocation (runtime/device.py:199-204). */
tempo_status tempo_device_reset(void);

/* Synchronous copies between host memory and the arena (runtime/memcpy.py:93-161). Both addresses 32-byte
 * aligned, nbytes > 0, the device range inside the arena; TEMPO_ERR_VALUE otherwise. */
tempo_status tempo_memcpy_h2d(uint32_t dst, const void* src, uint64_t nbytes);
tempo_status tempo_memcpy_d2h(void* dst, uint32_t src, uint64_t nbytes);

/* Launches the image staged at kbin_addr with up to four 32-bit arguments, and waits for it
 * (runtime/launch.py:44-141). TEMPO_ERR_VALUE for a malformed launch (size not a positive multiple of 16 or past
 * 65536 bytes, base not 32-byte aligned, range past 4 GiB, more than four arguments, an argument outside
 * [0, 0xFFFFFFFF], or an operand range outside the arena); TEMPO_ERR_RUNTIME when the image is not a descriptor of a
 * known kind (the reference's sticky launch error); TEMPO_ERR_TIMEOUT past `timeout_s`. */
tempo_status tempo_launch(uint64_t kbin_addr, uint64_t kbin_size, const int64_t* args, uint32_t nargs,
                          double timeout_s);

/* Waits for the library's stream with a deadline; reports a device watchdog expiry as TEMPO_ERR_TIMEOUT
 * (runtime/memcpy.py:289-312). */
tempo_status tempo_sync(double timeout_s);

/* Pinned host staging memory (runtime/device.py:84-125). */
tempo_status tempo_host_alloc(void** ptr, uint64_t nbytes);
tempo_status tempo_host_free(void* ptr);

/* Copies the last error message into `buffer` (NUL-terminated, truncated to `size`). */
tempo_status tempo_last_error(char* buffer, uint64_t size);

/* Launches done, and bytes allocated, since tempo_open (for tests and reports). */
tempo_status tempo_stats(uint64_t* launches, uint64_t* arena_used);

/* Reads and clears the device watchdog: non-zero names the bounded wait that expired in a kernel. */
tempo_status tempo_watchdog(int32_t* code);

/* Failure-detection probe, the device half of the reference's drain and timeout tests
 * (board_package/tests/test_drain.py:23-159, runtime/memcpy.py:289-312): one CTA waits on an mbarrier that
 * completes only when `arrive` is non-zero, giving up after `limit_ns` (at most 10 s) as every pipeline wait does,
 * with watchdog code 6. `stream` NULL means the runtime's stream, the one tempo_sync waits for. */
tempo_status tempo_wait_probe(uint32_t arrive, uint64_t limit_ns, void* stream);

/* ---------------------------------------------------------------------------------------------------------------
 * 2. Per-32-token-block tile ops on the packed layouts, with 64-bit device pointers. One call is one launch of the
 *    corresponding image (board_package/gpt2_inference.py:474-640,981-1039,1204-1209).
 * ------------------------------------------------------------------------------------------------------------- */

/* drain[512 B zero tile | [columns/16][32][16]] = [GELU](activations) x weights (+ bias), FP32 accumulate, BF16
 * out. activations: [depth/16][32][16]; weights: [columns/16][depth][16]; bias: [columns/16][4][16] or NULL
 * (gemm_resident, gpt2_inference.py:574-640; tile op tempo_ops.td:228-252). depth % 16 == 0, columns % 16 == 0. */
tempo_status tempo_block_gemm(const void* activations, const void* weights, void* drain, const void* bias,
                              uint32_t depth, uint32_t columns, uint32_t activate, void* stream);

/* out = left + right (or + the broadcast bias row), BF16 round-to-nearest-even; [features/16][32][16] each
 * (add_resident / add_bias_resident, gpt2_inference.py:506-571). */
tempo_status tempo_block_add(const void* left, const void* right, void* out, uint32_t features, uint32_t broadcast,
                             void* stream);

/* LayerNorm of 32 token rows with the constants block gamma | beta | 1/F x64 | eps x64 (layernorm_resident,
 * gpt2_inference.py:439-503). */
tempo_status tempo_block_layernorm(const void* rows, const void* constants, void* out, uint32_t features,
                                   void* stream);

/* Causal attention over every head of a fused QKV tensor of `tokens` (a multiple of 32) tokens, packed per block
 * as a 512-byte zero tile then [3*heads*head/16][32][16]; the output overwrites the queries (attention,
 * gpt2_inference.py:981-1003; tempo_ops.td:292-314). `fused` is the operand of block 0 (past its zero tile). */
tempo_status tempo_block_attention(const void* constants, void* fused, uint32_t tokens, uint32_t heads,
                                   uint32_t head, void* stream);

/* The first 16 query rows of `fused`'s block 0 attend over `keys` cached keys with the step's mask tiles (laid out
 * keys by queries) added to the scores, writing over the queries (decode_attention, gpt2_inference.py:1006-1039).
 * cache: operand of block 0 of a [keys, 2*heads*head] packed tensor (keys then values). */
tempo_status tempo_block_decode_attention(const void* constants, const void* cache, void* fused, uint32_t keys,
                                          uint32_t heads, uint32_t head, uint32_t stated, void* stream);

/* Copies `rows` 32-byte rows spaced `stride` bytes apart at both ends (_launch_copy, gpt2_inference.py:1204-1209;
 * tempo_ops.td:316-327). */
tempo_status tempo_block_copy(const void* source, void* destination, uint32_t rows, uint32_t stride, void* stream);

/* ---------------------------------------------------------------------------------------------------------------
 * 3. Native row-major ops for the batched B200 engine (the B200-first layout of the same math).
 * ------------------------------------------------------------------------------------------------------------- */

#define TEMPO_GEMM_GELU 1u   /* out = GELU(round_bf16(acc + bias)) */
#define TEMPO_GEMM_ARGMAX 2u /* no output: per-row (max, first argmax) over each N tile into the partials */
#define TEMPO_GEMM_LN 4u     /* internal: the LayerNorm-folded mode of tempo_gemm_ln (rejected by tempo_gemm) */

/* out[M, ldo] = epilogue(a[M, K] (row stride lda) x w_t[N, K]^T (row stride ldw)) with optional bias[N] and
 * residual[M, ldr] (added after GELU), FP32 accumulate, BF16 out; tcgen05 + TMA. K % 8 == 0; lda, ldw % 8 == 0.
 * In TEMPO_GEMM_ARGMAX mode `out` is unused and `part_val`/`part_idx` receive [M][ceil(N/256)] partials. */
tempo_status tempo_gemm(const void* a, uint32_t lda, const void* w_t, uint32_t ldw, const void* bias,
                        const void* residual, uint32_t ldr, void* out, uint32_t ldo, uint32_t m, uint32_t n,
                        uint32_t k, uint32_t flags, float* part_val, int32_t* part_idx, void* stream);

/* The QKV projection with the KV-cache write fused into its epilogue: out[M, 3*heads*head] = a x w_t^T + bias as
 * tempo_gemm computes it, and each row's key and value columns are also stored into k_cache / v_cache
 * ([seqs][heads][capacity][head] BF16) -- row r being sequence r / tokens_per_seq at position r % tokens_per_seq
 * (prefill), or, when positions is not NULL, sequence r at positions[r] (decode). Rows whose sequence or position is
 * out of range are not stored. Replaces the copy images that fill the reference's KV cache
 * (KVCache.extend/append, board_package/gpt2_inference.py:253-293). head % 32 == 0. */
tempo_status tempo_gemm_qkv(const void* a, uint32_t lda, const void* w_t, uint32_t ldw, const void* bias, void* out,
                            uint32_t ldo, uint32_t m, uint32_t k, void* k_cache, void* v_cache, uint32_t seqs,
                            uint32_t heads, uint32_t head, uint32_t capacity, uint32_t tokens_per_seq,
                            const int32_t* positions, void* stream);

/* LayerNorm then projection for at most 8 rows, in one launch: layernorm_resident followed by gemm_resident
 * (board_package/gpt2_inference.py:474-503 and :574-640). Every CTA normalises the M rows of x (gamma, beta, epsilon,
 * the arithmetic of tempo_layernorm) into its shared memory and streams its weight columns against them, so the
 * result has exactly the bits of tempo_layernorm followed by tempo_gemm (or tempo_gemm_qkv with positions) and no
 * normalised copy is written. For decode with a handful of sequences, where each launch costs more than its work.
 * 1 <= M <= 8, K (the features) a multiple of 8 up to 1024. flags: 0, TEMPO_GEMM_GELU, or TEMPO_GEMM_ARGMAX (the
 * final LayerNorm before the LM head; part_val / part_idx as tempo_gemm's). With k_cache / v_cache non-NULL the key
 * and value columns are stored into the caches as tempo_gemm_qkv stores them in decode (row r is sequence r at
 * positions[r]; N == 3 * heads * head). */
tempo_status tempo_gemm_norm(const void* x, uint32_t ldx, const void* gamma, const void* beta, float epsilon,
                             const void* w_t, uint32_t ldw, const void* bias, void* out, uint32_t ldo, uint32_t m,
                             uint32_t n, uint32_t k, uint32_t flags, float* part_val, int32_t* part_idx, void* k_cache,
                             void* v_cache, uint32_t heads, uint32_t head, uint32_t capacity,
                             const int32_t* positions, void* stream);

/* A projection with the LayerNorm before it folded in: layernorm_resident followed by gemm_resident
 * (board_package/gpt2_inference.py:474-503 and :574-640) as one kernel, for the decode step. With wg = gamma x W
 * (w_t_folded[N, K] is W^T with column k scaled by gamma[k], BF16), colsum[n] = sum_k wg[n, k] (FP32, of the BF16
 * wg) and bias_folded[n] = b[n] + sum_k beta[k] W[k, n] (FP32):
 *   out[r, n] = epilogue(rstd_r * (sum_k x[r, k] wg[n, k] - mean_r * colsum[n]) + bias_folded[n]),
 * mean_r and rstd_r = 1 / sqrt(var_r + epsilon) being row r's statistics, computed in the kernel while its MMAs run.
 * flags: 0 or TEMPO_GEMM_GELU. With k_cache / v_cache non-NULL the key and value columns are also stored into the
 * caches as tempo_gemm_qkv stores them in decode (positions required, N == 3 * heads * head). */
tempo_status tempo_gemm_ln(const void* x, uint32_t ldx, const void* w_t_folded, uint32_t ldw, const float* colsum,
                           const float* bias_folded, float epsilon, void* out, uint32_t ldo, uint32_t m, uint32_t n,
                           uint32_t k, uint32_t flags, void* k_cache, void* v_cache, uint32_t seqs, uint32_t heads,
                           uint32_t head, uint32_t capacity, const int32_t* positions, void* stream);

/* tempo_gemm whose epilogue also writes the statistics partials of the BF16 rows it stores: row_stats [m][n / 16]
 * float pairs (mean, M2) of each 16-column chunk (M2 = sum of squared deviations from the chunk mean). N % 16 == 0,
 * flags 0 or TEMPO_GEMM_GELU. The residual projections write them for the folded LayerNorm of the next projection. */
tempo_status tempo_gemm_rowstats(const void* a, uint32_t lda, const void* w_t, uint32_t ldw, const void* bias,
                                 const void* residual, uint32_t ldr, void* out, uint32_t ldo, uint32_t m, uint32_t n,
                                 uint32_t k, uint32_t flags, float* row_stats, void* stream);

/* tempo_gemm_ln with mean_r and rstd_r combined from row_stats [m][k / 16] (tempo_gemm_rowstats' or
 * tempo_row_stats' partials of x: the mean of the chunk means, M2 = sum M2_c + 16 sum (mean_c - mean)^2, each summed
 * in a fixed order) instead of computed from x in the kernel, so the projection may split K. K % 16 == 0, K <= 1024. */
tempo_status tempo_gemm_ln_rowstats(const void* x, uint32_t ldx, const void* w_t_folded, uint32_t ldw,
                                    const float* colsum, const float* bias_folded, float epsilon, const float* row_stats,
                                    void* out, uint32_t ldo, uint32_t m, uint32_t n, uint32_t k, uint32_t flags,
                                    void* k_cache, void* v_cache, uint32_t seqs, uint32_t heads, uint32_t head,
                                    uint32_t capacity, const int32_t* positions, void* stream);

/* The statistics partials of `rows` BF16 rows of `width` (width % 16 == 0, row stride ldx % 8 == 0), in
 * tempo_gemm_rowstats' layout: for rows no projection wrote (the embedding's). */
tempo_status tempo_row_stats(const void* x, uint32_t ldx, uint32_t rows, uint32_t width, float* row_stats,
                             void* stream);

/* Row-wise LayerNorm of `rows` BF16 rows of `features` (features % 8 == 0, <= 4096) read `x_stride` elements apart
 * (x_stride % 8 == 0), FP32 statistics, BF16 out [rows, features]. */
tempo_status tempo_layernorm(const void* x, uint32_t x_stride, const void* gamma, const void* beta, void* out,
                             uint32_t rows, uint32_t features, float epsilon, void* stream);

/* x[r] = round_bf16(wte[ids[r]] + wpe[positions[r]]) for r < rows; ids/positions int32 on the device. A row whose
 * id is outside [0, vocab) or position outside [0, max_positions) is written as zeros. */
tempo_status tempo_embed(const int32_t* ids, const int32_t* positions, const void* wte, const void* wpe, void* x,
                         uint32_t rows, uint32_t width, uint32_t vocab, uint32_t max_positions, void* stream);

/* Causal attention of `seqs` sequences of `tokens` tokens each. qkv: [seqs*tokens, 3*heads*head] BF16 (queries
 * already scaled by 1/sqrt(head)); out: [seqs*tokens, heads*head] BF16. tcgen05 for QK^T and PV. head == 64. */
tempo_status tempo_attention_prefill(const void* qkv, void* out, uint32_t seqs, uint32_t tokens, uint32_t heads,
                                     uint32_t head, void* stream);

/* Writes the keys and values of `rows` rows of qkv into the caches: row r belongs to sequence seq_of[r] at
 * position pos_of[r]. Caches are [seqs][heads][capacity][head] BF16, one for keys and one for values. Rows whose
 * sequence or position is out of range are skipped. */
tempo_status tempo_kv_store(const void* qkv, void* k_cache, void* v_cache, const int32_t* seq_of,
                            const int32_t* pos_of, uint32_t rows, uint32_t seqs, uint32_t heads, uint32_t head,
                            uint32_t capacity, void* stream);

/* One query per sequence (row s of qkv, scaled) over the first lengths[s] + length_offset cached keys of each head
 * (clamped to [0, capacity]); out: [seqs, heads*head] BF16. */
tempo_status tempo_decode_attention(const void* qkv, const void* k_cache, const void* v_cache,
                                    const int32_t* lengths, int32_t length_offset, void* out, uint32_t seqs,
                                    uint32_t heads, uint32_t head, uint32_t capacity, void* stream);

/* Reduces argmax partials [rows][tiles] to token ids: ids[r] = first index of the row maximum (ties go to the lower
 * index, as numpy's argmax). When tokens_out is not NULL the id is also written to tokens_out[r * out_stride + c] with
 * c = positions[r] + index_offset (c = index_offset without positions), skipped unless 0 <= c < out_stride; then
 * positions[r] advances by `advance`. Keeping the column on the device lets one captured decode step be replayed. */
tempo_status tempo_argmax_finish(const float* part_val, const int32_t* part_idx, uint32_t rows, uint32_t tiles,
                                 int32_t* ids, int32_t* tokens_out, uint32_t out_stride, int32_t* positions,
                                 int32_t index_offset, int32_t advance, void* stream);

/* The LM head's greedy pick with no device allocation: ids[r] = the first j maximising hidden[r] . embedding[j], for
 * hidden [rows, width] BF16 (row stride ld_hidden) and embedding [vocab, width] BF16 (row stride ld_embedding).
 * No counterpart in the reference (its LM head runs on the host). It exists for callers that may not allocate device
 * memory -- a plugin host that owns every device byte, or a loop that cannot pay for cudaMalloc/cudaFree -- and
 * differs from tempo_gemm(TEMPO_GEMM_ARGMAX) + tempo_argmax_finish only in keeping their partials in a 2 MiB array
 * inside the library, held on every GPU that loads it. Limits: 1 <= rows <= 1024 and 1 <= vocab <= 65536, else
 * TEMPO_ERR_VALUE. The first call on a device looks up the array's address, so make it before any stream capture.
 * Every call shares the array: calls whose work overlaps on the GPU race and must be ordered by the caller. */
tempo_status tempo_lm_head_argmax_noalloc(const void* hidden, uint32_t ld_hidden, const void* embedding,
                                          uint32_t ld_embedding, uint32_t rows, uint32_t vocab, uint32_t width,
                                          int32_t* ids, void* stream);

/* One greedy decode step of 1 to 8 sequences as a single persistent kernel (one CTA per SM, launched cooperatively,
 * grid-wide barriers between its phases), replacing the kernel-per-op step of the reference's decode loop
 * (board_package/gpt2_inference.py:865-889, decode_block :775-797, the host LM head :915-938): embedding, then per
 * layer LayerNorm 1 + QKV + cache store, attention over each sequence's cache, out-projection + residual,
 * LayerNorm 2 + FC + GELU, second projection + residual; then the final LayerNorm and the tied LM head's argmax.
 * Tokens equal the kernel-per-op path's bit for bit (same per-element arithmetic). Row r consumes ids[r] at
 * positions[r]; the step writes its pick to ids[r] and, when tokens_out is not NULL, to
 * tokens_out[r * out_stride + positions[r] + index_offset] (if inside the row), then advances positions[r].
 * Weights are [out, in] BF16 (K contiguous), the query rows and bias of w_qkv / b_qkv pre-scaled by 1/sqrt(64); caches
 * are [rows][heads][capacity][64] BF16. `workspace` (tempo_decode_step_workspace bytes, 256-byte aligned) must be
 * zero before the first step and is then left consistent by every step; one workspace serves one stream. A grid
 * barrier that waits past its bounded time ends the kernel with watchdog code 7 (reported by tempo_sync /
 * tempo_watchdog) and leaves the workspace unusable until it is zeroed again. */
typedef struct tempo_decode_layer {
  const void* ln1_gamma;
  const void* ln1_beta;
  const void* w_qkv;     /* [3 width, width] */
  const void* b_qkv;     /* [3 width] */
  const void* w_proj;    /* [width, width] */
  const void* b_proj;
  const void* ln2_gamma;
  const void* ln2_beta;
  const void* w_fc;      /* [4 width, width] */
  const void* b_fc;
  const void* w_out;     /* [width, 4 width] */
  const void* b_out;
  void* k_cache;         /* [rows][heads][capacity][64] */
  void* v_cache;
} tempo_decode_layer;

typedef struct tempo_decode_step_args {
  uint32_t layers, rows, width, heads, vocab, max_positions, capacity;
  float epsilon;
  const tempo_decode_layer* layer;  /* `layers` entries, read on the host at each call */
  const void* wte;                  /* [vocab, width], also the LM head */
  const void* wpe;                  /* [max_positions, width] */
  const void* lnf_gamma;
  const void* lnf_beta;
  int32_t* ids;
  int32_t* positions;
  int32_t* tokens_out;
  uint32_t out_stride;
  int32_t index_offset;
  void* workspace;
  uint64_t workspace_bytes;
} tempo_decode_step_args;

tempo_status tempo_decode_step_workspace(uint32_t rows, uint32_t width, uint32_t heads, uint32_t vocab,
                                         uint64_t* bytes);
tempo_status tempo_decode_step(const tempo_decode_step_args* args, void* stream);

/* Calibration (no counterpart in the reference): reads `bytes` (rounded down to whole groups of 16-byte words per
 * thread) from `src` with streaming loads and writes one 16-byte word per thread into `sink`, which holds
 * tempo_stream_read_threads() words. Its rate is the HBM read ceiling the bandwidth-bound kernels are measured against. */
tempo_status tempo_stream_read_threads(uint32_t* threads);
tempo_status tempo_stream_read(const void* src, uint64_t bytes, void* sink, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TEMPO_B200_H */
