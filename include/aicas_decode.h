/* C ABI of the B200 decode engine for the Qwen3-VL-2B text decoder.
 *
 * Every entry point takes raw device pointers (fp16 data unless stated),
 * plain integer sizes and a CUDA stream; none allocates memory, none
 * synchronises the stream, and all are safe to capture in a CUDA graph.
 * Return value: AICAS_OK (0) or an AICAS_ERR_* code for errors detected on the
 * host (bad argument, shape, alignment, failed launch).  Errors detected on the
 * device during a launch (bounded waits that gave up, out-of-range token or
 * cache position) are written to the `error` word at the start of the scratch
 * block (see AicasScratch in aicas_phase_program.h); read it after the stream
 * synchronises.  A launch whose scratch block still holds a device error does
 * nothing (no read, write or step-state change): zero the scratch block (and,
 * for the step programs, the flag-in-data activation vectors) to resume.
 *
 * Scratch: kernels that need workspace (grid barrier, split-KV partials, the
 * cross-CTA argmax) take a `scratch` pointer to aicas_scratch_bytes() bytes of
 * device memory that the caller zero-fills ONCE; every launch leaves it ready
 * for the next.  Launches that share a scratch block must be ordered on one
 * stream (never concurrent).
 *
 * Each function names the reference interface it replaces (paths and lines
 * are within the reference checkout, wangxiyu191/AICASGC-2026).
 */
#ifndef AICAS_DECODE_H
#define AICAS_DECODE_H

#include <stddef.h>
#include <stdint.h>

#include "aicas_phase_program.h"

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define AICAS_API __attribute__((visibility("default")))
#else
#define AICAS_API
#endif

#define AICAS_ABI_VERSION 1

/* Host-side error codes (device error codes 10..15 are listed by
 * aicas_error_string). */
#define AICAS_OK 0
#define AICAS_ERR_ARG 1
#define AICAS_ERR_SHAPE 2
#define AICAS_ERR_ALIGN 3
#define AICAS_ERR_CUDA 4
#define AICAS_ERR_CAPACITY 5

typedef struct CUstream_st* aicas_stream_t; /* == cudaStream_t */

AICAS_API int aicas_abi_version(void);
AICAS_API const char* aicas_error_string(int code);
/* cudaError_t of the last AICAS_ERR_CUDA returned on this host thread, and
 * its CUDA description. */
AICAS_API int aicas_last_cuda_error(void);
AICAS_API const char* aicas_cuda_error_string(int err);
/* Bytes of the scratch block (sizeof(AicasScratch)). */
AICAS_API size_t aicas_scratch_bytes(void);
/* Struct sizes/offsets for binding checks; returns the number of values. */
AICAS_API int aicas_layout_signature(int64_t* out, int n);
/* CTAs of one persistent launch on `device` (= its SM count, <= 256), or a
 * negative error code. */
AICAS_API int aicas_num_ctas(int device);
/* 1 (default): launch the persistent kernel as a cooperative launch, which
 * fails instead of running when the grid cannot be co-resident. */
AICAS_API int aicas_set_cooperative_launch(int enable);
/* Host-side check of a phase list before it is copied to the device. */
AICAS_API int aicas_validate_phases(const AicasPhase* phases, int n);

/* y[n] = W[n,k] x[k] (+ bias[n]); fp32 accumulation, fp16 output.
 * k % 8 == 0, k <= 6144, x/W 16-byte aligned.
 * Replaces `nosplit_matvec_half` (cuda_decode_gemv_ops/matvec.py:274-321;
 * kernels cuda_extensions/decode_gemv_kernel_matvec.cuh:209-343). */
AICAS_API int aicas_gemv_f16(const void* x, const void* w, const void* bias, void* y, int64_t n, int64_t k,
                             void* scratch, aicas_stream_t stream);

/* y = W_qkv * RMSNorm(x) (HF rounding: norm in fp32, rounded to fp16, times
 * the fp16 weight, rounded).  Replaces `fused_rmsnorm_qkv_half`
 * (cuda_decode_gemv_ops/fused.py:71-105; kernel
 * cuda_extensions/decode_gemv_kernel_fused.cuh:99-185). */
AICAS_API int aicas_rmsnorm_qkv_f16(const void* x, const void* norm_w, const void* w, const void* bias, void* y,
                                    int64_t n, int64_t k, float eps, void* scratch, aicas_stream_t stream);

/* h = residual + attn_out; act = SiLU(W_gate RMSNorm(h)) * (W_up RMSNorm(h));
 * out = h + W_down act (+ bias).  act_out [inter] receives the activation
 * (the reference's `hidden_out`).  gate_up_w is [2*inter, hidden] with the
 * gate rows first.  One persistent launch, two phases, one grid barrier.
 * Replaces `fused_post_attn_mlp_softsync_half`
 * (cuda_decode_gemv_ops/fused.py:261-337; kernel
 * cuda_extensions/decode_gemv_kernel_fused.cuh:850-1076). */
AICAS_API int aicas_post_attn_mlp_f16(const void* residual, const void* attn_out, const void* norm_w,
                                      const void* gate_up_w, const void* down_w, const void* bias, void* act_out,
                                      void* out, int64_t hidden, int64_t inter, float eps, void* scratch,
                                      aicas_stream_t stream);

/* Decode attention for one query token: out[q_heads,128] =
 * softmax(q K^T * scale) V over cache slots [0, *cache_position] (int64 on
 * the device).  K/V: [kv_heads, max_len, 128] (HF StaticLayer.keys/values of
 * batch 1); q_heads == 2 * kv_heads <= 16.  One ordinary launch: up to 16
 * chunks of cache slots per KV head, each CTA's partial merged by the last CTA
 * of its head in split order (deterministic).  `scratch` (aicas_scratch_bytes,
 * zeroed before its first use) holds the partials, one arrival counter per KV
 * head (back to zero after every call) and the error word: a cache position
 * outside [0, max_len) records device error 15 and writes nothing, and a
 * block that holds an error refuses the call.  Replaces
 * `decode_attn_v4_cta_qhead_splitkv_fused` (cuda_decode_attention.py:489-558;
 * kernel cuda_extensions/decode_attention_v4_kernel.cu:647-900). */
AICAS_API int aicas_decode_attn_splitkv_f16(const void* q, const void* k_cache, const void* v_cache,
                                            const void* cache_position, float scale, void* out, int64_t q_heads,
                                            int64_t kv_heads, int64_t max_len, void* scratch,
                                            aicas_stream_t stream);

/* Per-head RMSNorm + rotary embedding of q and k with the given cos/sin
 * [128], k and v written to cache slot *cache_position, rotated q to q_out.
 * q [q_heads,128], k/v [kv_heads,128], q_heads == 2 * kv_heads.  Replaces
 * `fused_q_rope_kv_cache_update` (cuda_decode_small_ops.py:136-225; kernel
 * cuda_extensions/decode_small_ops_kernel.cu:115-186). */
AICAS_API int aicas_qk_norm_mrope_kvwrite_f16(const void* q, const void* k, const void* v, const void* q_norm_w,
                                              const void* k_norm_w, const void* cos, const void* sin, void* q_out,
                                              void* k_cache, void* v_cache, const void* cache_position, float eps,
                                              int64_t q_heads, int64_t kv_heads, int64_t max_len,
                                              aicas_stream_t stream);

/* logits[vocab] = W x' where x' = RMSNorm(x) when norm_w is not null;
 * *token_out (int64) = first index of the maximum fp16 logit.  logits may
 * be null.  Replaces the tied lm_head GEMV `FastLmHead.forward`
 * (evaluation_wrapper.py:1227-1240) plus `torch.argmax`
 * (evaluation_wrapper.py:952). */
AICAS_API int aicas_lm_head_argmax_f16(const void* x, const void* norm_w, const void* w, void* logits,
                                       void* token_out, int64_t vocab, int64_t k, float eps, void* scratch,
                                       aicas_stream_t stream);

/* One whole decode step (all layers + final norm + lm_head + argmax) as one
 * persistent launch running the phase list `device_phases` (device memory,
 * built and validated on the host).  Reads its inputs from `state` and
 * advances it (device-side greedy loop).  Replaces the graph-captured step
 * `DecodeCudaGraphRunner._run_step` (evaluation_wrapper.py:941-952), i.e. HF's
 * layer loop over `OptimizedDecoderLayer.forward` (optimized_layer.py:108-469). */
AICAS_API int aicas_decode_program_f16(const AicasPhase* device_phases, int n_phases, AicasStepState* state,
                                       void* scratch, aicas_stream_t stream);

/* Whether the lean kernel can run a program: every GEMV-type phase streams
 * whole 2048-column chunks (k % 2048 == 0) and has either k == 2048, or
 * k == 6144 with at most 2 row groups of 8 rows per CTA on a grid of
 * `num_ctas` CTAs (aicas_num_ctas) and is not a GATEUP phase.  The engine's
 * 28-layer Qwen3-VL program qualifies.  Returns AICAS_OK or AICAS_ERR_SHAPE;
 * `phases` is the host copy of the program. */
AICAS_API int aicas_lean_program_ok(const AicasPhase* phases, int n_phases, int num_ctas);

/* aicas_decode_program_f16 with options: `trace` (may be null) as in
 * aicas_decode_program_trace_f16; `flags` AICAS_PROGRAM_LEAN runs the lean
 * instantiation of the kernel (no code for the tile paths such programs
 * never take: a smaller instruction footprint), for programs that passed
 * aicas_lean_program_ok.  A program that does not qualify is not run past
 * its first unsuitable phase: the launch aborts with device error 14 (bad
 * phase) in the scratch block's error word. */
#define AICAS_PROGRAM_LEAN 1
AICAS_API int aicas_decode_program_ex_f16(const AicasPhase* device_phases, int n_phases, AicasStepState* state,
                                          void* scratch, int64_t* trace, int flags, aicas_stream_t stream);

/* Allocation-free variant of aicas_decode_attn_splitkv_f16, for callers that
 * cannot allocate device memory themselves (for example code running inside
 * a framework that owns every allocation, or a plugin that is only handed the
 * tensors of one call): same arguments and result, but no `scratch`
 * argument.  Its scratch is a fixed array inside this library, one per
 * device, of aicas_scratch_bytes() bytes (about 4.2 MB), held until the
 * process exits; it fits at most 8 KV heads (q_heads == 2 * kv_heads, head
 * dim 128) and returns AICAS_ERR_CAPACITY for anything larger.  The first
 * call on a device looks up the array's address, so make that call before
 * any stream capture.  Every call on a device shares the one array: calls
 * that overlap on the GPU (different streams, no ordering) race and give
 * wrong results.  Each call zeroes the array's counters before its launch;
 * `status` (device int32, may be null) receives the call's device error
 * code.  Nothing is allocated or freed.  Host threads may call it
 * concurrently (the address lookup is thread-safe; the launches still race
 * on the GPU unless ordered).  After a device reset (cudaDeviceReset) the
 * cached address is stale: reload the library.  This entry point has no
 * counterpart in the reference. */
AICAS_API int aicas_decode_attn_splitkv_f16_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                                   const void* cache_position, float scale, void* out,
                                                   int64_t q_heads, int64_t kv_heads, int64_t max_len,
                                                   int32_t* status, aicas_stream_t stream);

/* Profiling variant of aicas_decode_program_f16: additionally writes, per
 * CTA and phase, trace[cta][phase][8] (int64, aicas_num_ctas() * n_phases * 8
 * entries): the %globaltimer (ns) when the phase started, when its inputs
 * were ready, when it finished; the ns one consumer warp spent waiting for
 * weight/KV tiles to land; the ns the producer spent waiting for free ring
 * slots while issuing the phase's tiles; the number of tiles consumed; and
 * (ns) when the CTA's own attention units were computed, and when its
 * results were issued (attention partial stored / splits merged; GEMV: tile
 * loops done).  The reference records the same kind of per-block timelines
 * in its `*_profile_*` kernel variants
 * (cuda_extensions/decode_gemv_kernel_common.cuh:174-188). */
AICAS_API int aicas_decode_program_trace_f16(const AicasPhase* device_phases, int n_phases,
                                             AicasStepState* state, void* scratch, int64_t* trace,
                                             aicas_stream_t stream);

/* ---- batched decode: up to AICAS_MAX_BATCH requests per launch ----------
 *
 * One decode step of `nb` independent requests ("streams", each with its own
 * token, ragged cache position, KV cache slice and step state) as one
 * persistent launch: the weights stream from HBM once per step for all
 * streams, and every projection runs on the tensor cores (tcgen05.mma, fp16
 * operands, fp32 accumulation in tensor memory).  The reference serves one
 * request per engine (`GreedyDecodeEngine` rejects batch > 1,
 * evaluation_wrapper.py:110-111, and its attention kernel reads only
 * cache_position[0], cuda_extensions/decode_attention_v4_kernel.cu:647-900);
 * this is the batch-8 request-parallel configuration built on the same phase
 * programs.
 *
 * Phase list: the kinds of aicas_phase_program.h with these batch rules
 * (checked by aicas_validate_batch_phases):
 *   - activations are LL vectors [nb][len] (stream b's row starts at word
 *     b * len), every GEMV-type phase has F_LL_OUT except the LM head, and
 *     inputs are F_LL_IN or F_X_EMBED (stream b's token row);
 *   - GEMV weights are in the tensor-core tile layout: n % 8 == 0,
 *     k in {2048, 4096, 6144} (k > 2048 also F_KBLOCKED), and each 8-row x
 *     2048-column block (32 KB, at the block address of the batch-1 layouts)
 *     stored as [256 column groups][8 rows][8 columns];
 *     aicas_tile_weight_f16 converts a row-major [n, k] matrix;
 *   - attention: x is [nb][q_heads*128 + 2*kv_heads*128] (q, k, v of each
 *     stream; phase field k = that row length), out is [nb][q_heads*128]
 *     (phase field n), K/V caches [nb][kv_heads][max_len * 128] fp16 with
 *     max_len % 8 == 0, each (stream, head) slice in the KV tile layout:
 *     slot p, dim d at element (p/8)*1024 + (d/8)*64 + (p%8)*8 + d%8 (the
 *     size of HF StaticLayer of batch nb, not its order), q/k norm + MRoPE +
 *     KV write always on (no F_Q_READY);
 *   - the LM head writes stream b's logits to states[b].logits (if set) and
 *     advances states[b] (out_tokens, script, EOS) like the batch-1 step.
 * A stream whose state has done_step != 0 is inactive: it is skipped (no KV
 * write, no state change); a launch with no active stream returns at once.
 * Activations may also be "counted" vectors (AICAS_F_CNT_*: plain fp16 in the
 * operand layout [len/8][8 stream slots][8], one completion counter per
 * phase).  Scratch: aicas_batch_scratch_bytes() bytes (sizeof(AicasBatchScratch)),
 * zero-filled once, ordered launches only (as for the batch-1 scratch); the
 * completion counters assume every launch on one scratch block runs the same
 * phase list (zero the block again before switching to another). */
AICAS_API size_t aicas_batch_scratch_bytes(void);
AICAS_API int aicas_validate_batch_phases(const AicasPhase* phases, int n);
AICAS_API int aicas_decode_batch_f16(const AicasPhase* device_phases, int n_phases, AicasStepState* states, int nb,
                                     void* scratch, aicas_stream_t stream);
/* Profiling variant of aicas_decode_batch_f16: also writes, per CTA and
 * phase, trace[cta][phase][8] (int64, aicas_num_ctas() * n_phases * 8
 * entries): the %globaltimer (ns) when the consumers started the phase, when
 * its inputs were ready (GEMV: the streams' operand built; attention: the
 * first segment's queries loaded), when the phase ended; when the MMA warp
 * saw the operand ready and when it issued the phase's last MMA (GEMV
 * phases; attention: when the CTA's units were done, before its merges, and
 * the ns spent loading the segments' queries); the CTA's row groups or attention units in the phase; the ns one
 * consumer warp waited for attention tiles to land; and the ns the producer
 * waited for free ring stages while issuing the phase's tiles. */
AICAS_API int aicas_decode_batch_trace_f16(const AicasPhase* device_phases, int n_phases, AicasStepState* states,
                                           int nb, void* scratch, int64_t* trace, aicas_stream_t stream);
/* dst = W [n, k] (row-major, device) in the tensor-core tile layout above
 * (dst must not overlap w; n % 8 == 0, k % 2048 == 0). */
AICAS_API int aicas_tile_weight_f16(const void* w, void* dst, int64_t n, int64_t k, aicas_stream_t stream);

/* ---- one-pass prompt prefill (the kernels between the prefill's GEMMs) ---
 *
 * The reference prefills a prompt with HF's forward over all prompt tokens
 * (evaluation_wrapper.py:1836-1958; OptimizedDecoderLayer.prefill_forward_no_mask,
 * optimized_layer.py:471-619).  The projections are dense fp16 GEMMs with fp32
 * accumulation, run by the caller's GEMM library; these four entry points are
 * the rest of a prefill layer, with HF's fp16 rounding points, writing K and V
 * into the decode engine's StaticLayer-layout cache.  Row-major fp16 tensors,
 * 16-byte aligned. */

/* h_out = r16(h + delta) (delta may be null: h_out = h; h_out may be null or
 * alias h); x_out = RMSNorm(h_out) * norm_w with HF's rounding points.
 * [rows, cols], cols % 8 == 0, cols <= 8192. */
AICAS_API int aicas_prefill_add_rmsnorm_f16(const void* h, const void* delta, const void* norm_w, void* h_out,
                                            void* x_out, int64_t rows, int64_t cols, float eps,
                                            aicas_stream_t stream);
/* qkv [rows, (q_heads + 2 kv_heads) * 128]: per-head RMSNorm of q and k
 * (q_norm_w / k_norm_w [128]) and interleaved MRoPE from pos3 [3, rows]
 * (int64 t, h, w positions; inv_freq [64] fp32; sections sec1 / sec2 of the
 * h and w axes); q to q_out [rows, q_heads, 128], k and v to cache slots
 * start .. start + rows - 1 of k_cache / v_cache [kv_heads, max_len, 128].
 * `tiles` (optional, start == 0 only): also q, k and v into the workspace
 * of aicas_prefill_attention_tiles_f16 (q_out may then be null). */
AICAS_API int aicas_prefill_qk_norm_rope_kv_f16(const void* qkv, const void* q_norm_w, const void* k_norm_w,
                                                const void* pos3, const void* inv_freq, int sec1, int sec2,
                                                void* q_out, void* k_cache, void* v_cache, int64_t rows,
                                                int64_t start, int64_t max_len, int64_t q_heads, int64_t kv_heads,
                                                float eps, void* tiles, aicas_stream_t stream);
/* act [rows, inter] = r16(r16(SiLU(gate)) * up) of gate_up [rows, 2 inter]
 * (gate columns first); rows <= 65535. */
AICAS_API int aicas_prefill_silu_mul_f16(const void* gate_up, void* act, int64_t rows, int64_t inter,
                                         aicas_stream_t stream);
/* Causal GQA attention of `rows` queries (q [rows, q_heads, 128], query t at
 * cache slot start + t) over cache slots [0, start + t] of k_cache /
 * v_cache [kv_heads, max_len, 128]: out [rows, q_heads, 128] fp16, query
 * head h on KV head h / (q_heads / kv_heads); softmax(q k^T scale) v in fp32
 * with P rounded to fp16 for its product with V.  On the tcgen05 tensor
 * cores (csrc/prefill_attn_tc.cu): S = Q K^T and O += P V as M = N = 128
 * MMAs with fp32 accumulators in tensor memory, one CTA per 128-query tile
 * and head.  `workspace` (16-byte aligned, aicas_prefill_attention_workspace_bytes
 * bytes, overwritten) first receives q and the slots in the KV tile layout
 * (per head, row p, dim d at element (p/8)*1024 + (d/8)*64 + (p%8)*8 + d%8;
 * rows padded to a multiple of 128): two launches on `stream`.
 * aicas_prefill_attention_tiles_f16 is the attention alone on a workspace
 * that aicas_prefill_qk_norm_rope_kv_f16 filled (start == 0; its padding
 * rows zero or finite).  aicas_prefill_attention_timeouts() returns how many
 * of the kernel's bounded waits gave up in this process (0 unless something
 * is wrong; synchronises the device). */
AICAS_API size_t aicas_prefill_attention_workspace_bytes(int64_t rows, int64_t start, int64_t q_heads,
                                                         int64_t kv_heads);
AICAS_API int aicas_prefill_attention_f16(const void* q, const void* k_cache, const void* v_cache, void* out,
                                          int64_t rows, int64_t start, int64_t q_heads, int64_t kv_heads,
                                          int64_t max_len, float scale, void* workspace, aicas_stream_t stream);
AICAS_API int aicas_prefill_attention_tiles_f16(const void* tiles, void* out, int64_t rows, int64_t start,
                                                int64_t q_heads, int64_t kv_heads, float scale,
                                                aicas_stream_t stream);
AICAS_API int aicas_prefill_attention_timeouts(void);

#ifdef __cplusplus
}
#endif

#endif /* AICAS_DECODE_H */
