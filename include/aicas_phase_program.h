// Layouts shared by the host-side program builder and the persistent
// decode-program kernel.  Plain C structs: they are also mirrored by ctypes in
// `aicasgc-2026_b200/_native.py` (field order and sizes must match; `aicas_layout_signature`
// exports the sizes so the Python side can check them at load time).
//
// A decode step is a list of PHASES executed by one persistent launch of
// `decode_program_kernel` (one CTA per SM).  Every phase is a memory-bound
// sweep over one weight matrix (or over the KV cache).  Phases are ordered by
// their inputs: a phase that reads the vector of an earlier phase polls its
// flag-in-data words (AICAS_F_LL_IN, below) or, in the batched kernel, a
// per-phase completion counter (AICAS_F_CNT_IN); only a phase marked
// AICAS_F_BARRIER waits at a bounded software grid barrier first (for
// programs whose vectors are plain fp16; the engines' programs use none).
// One warp per CTA streams the
// phase's tiles from HBM into a shared-memory ring with bulk async copies,
// independently of the activations, so weight streaming never waits on
// another CTA.
#pragma once
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum AicasPhaseKind {
  AICAS_PH_GEMV = 1,     // out = [resid +] W x [+ bias]          (QKV, o_proj, down, generic)
  AICAS_PH_GATEUP = 2,   // out = silu(Wg x) * (Wu x)            (fused gate_up + SiLU*up)
  AICAS_PH_ATTN = 3,     // q/k norm + MRoPE + KV write + split-KV GQA attention + LSE merge
  AICAS_PH_LMHEAD = 4,   // logits = E x, argmax, advance the step state
};

// Flags of a phase.
enum AicasPhaseFlags {
  AICAS_F_NORM = 1 << 0,         // x := RMSNorm(x) * norm_w before the sweep (HF rounding points)
  AICAS_F_X_EMBED = 1 << 1,      // x := embedding row of the step token (x points at the table)
  AICAS_F_RESID = 1 << 2,        // out := r16(resid + r16(acc))
  AICAS_F_RESID_EMBED = 1 << 3,  // resid := embedding row of the step token
  AICAS_F_BIAS = 1 << 4,         // acc += bias (fp32, before rounding)
  AICAS_F_X_ADD = 1 << 5,        // x := r16(x + x2)   (before the optional norm)
  AICAS_F_RESID_ADD = 1 << 6,    // resid := r16(resid + resid2)
  AICAS_F_Q_READY = 1 << 7,      // attention: q is final (no norm/rope); no KV write
  AICAS_F_STORE_X = 1 << 8,      // GEMV/GATEUP: CTA 0 stores the prologue vector to x_out
  AICAS_F_KBLOCKED = 1 << 9,     // W is stored K-blocked: [k/2048][n][2048] (k % 2048 == 0), so every
                                 // 8-row x 2048-column tile is one contiguous 32 KB block
  AICAS_F_BARRIER = 1 << 10,     // grid barrier before this phase (inputs written by the previous phase)
  AICAS_F_LL_IN = 1 << 11,       // x is an LL vector written by phase `x_src` of this launch (see below)
  AICAS_F_LL_OUT = 1 << 12,      // out is an LL vector
  AICAS_F_LL_RESID = 1 << 13,    // resid is an LL vector (complete before this phase starts)
  // Batched programs only (aicas_decode_batch_f16): "counted" vectors are plain
  // fp16 in the batched operand layout [len/8][8 stream slots][8] (16 bytes per
  // 8 values of one stream); the phase that writes one adds 1 to its
  // per-phase completion counter once per CTA (release), and a reader waits
  // until all CTAs have counted (acquire), then reads the whole vector once.
  AICAS_F_CNT_IN = 1 << 14,      // x is a counted vector written by phase x_src of this launch
  AICAS_F_CNT_OUT = 1 << 15,     // out is a counted vector
  AICAS_F_CNT_RESID = 1 << 16,   // resid is a counted vector (complete before this phase starts)
};

// LL ("flag in data") vectors carry inter-phase activations without grid
// barriers: value i of an fp16 vector lives in 32-bit word i as {fp16 value
// (low half), uint16 epoch (high half)}, written with one 4-byte store.  A
// consumer polls the words it needs until every epoch equals the producing
// phase's epoch ((launch epoch base + phase index + 1) mod 2^16), so the data,
// the completion flag and the memory ordering arrive together.  Epochs grow
// by n_phases + 1 per launch (AicasScratch::epoch) and every word is rewritten
// every launch, so a stale word never matches.

// One phase.  Pointers are device pointers (fp16 data is `__half`, passed as
// void* so this header stays free of CUDA types).
typedef struct AicasPhase {
  int32_t kind;
  int32_t flags;
  int32_t n;        // GEMV/LMHEAD: output rows; GATEUP: intermediate size (rows of gate)
  int32_t k;        // reduction length (multiple of 8, <= AICAS_MAX_K = 6144)
  int32_t rot;      // CTA rotation of the row-group assignment (load balance across phases)
  int32_t kv_heads; // attention
  int32_t q_heads;  // attention
  int32_t max_len;  // attention: cache slots per head
  int32_t embed_rows; // F_X_EMBED / F_RESID_EMBED: rows of the embedding table
  int32_t x_src;      // F_LL_IN: index of the phase (in this program) that writes x
  const void* w;      // weight [n, k] row-major (GATEUP: [2n, k], gate rows first), or K-blocked
  const void* norm_w; // RMSNorm weight [k] (attention: q_norm weight [128])
  const void* norm_w2;// attention: k_norm weight [128]
  const void* x;      // input vector [k] (attention: the fused qkv vector or final q)
  const void* x2;     // second input (F_X_ADD)
  const void* resid;  // residual [n]
  const void* resid2; // second residual (F_RESID_ADD)
  const void* bias;   // [n]
  void* out;          // output [n] fp16 (attention: [q_heads*128])
  void* x_out;        // F_STORE_X target [k]
  void* k_cache;      // attention: [kv_heads, max_len, 128] fp16
  void* v_cache;
  const void* pos_ptr;// attention: int64 cache position (null: the step state's)
  void* idx_out;      // LMHEAD: int64 argmax output (may be null)
  float eps;
  float scale;        // attention softmax scale
} AicasPhase;

// Decode-step state in device memory, read by every launch and advanced by
// the LM-head phase (device-side greedy loop: no host write between steps).
typedef struct AicasStepState {
  int64_t token;        // input token of the current step
  int64_t cache_pos;    // KV slot written by this step; attention covers [0, cache_pos]
  int64_t rope[3];      // MRoPE positions (t, h, w) of this step
  int64_t step;         // steps executed so far
  int64_t script_len;   // steps whose inputs come from `script` (teacher forcing / prefill)
  const int64_t* script;// [script_len][5] = token, cache_pos, t, h, w
  int64_t* out_tokens;  // [max_steps] argmax of every step
  int64_t max_steps;
  void* logits;         // optional fp16 [logits_ring][vocab]
  int64_t logits_ring;
  float inv_freq[64];   // rotary inverse frequencies (host computes them like HF)
  int32_t mrope_section[3];
  int32_t pad0;
  int64_t eos_token;    // end-of-sequence id, or -1: a generated step whose argmax is this id ends the request
  int64_t done_step;    // 0 while running; after the EOS step s, s + 1 -- every later launch returns at once
} AicasStepState;

#define AICAS_MAX_CTAS 256
#define AICAS_MAX_SPLITS 256
#define AICAS_MAX_KV_HEADS 8
#define AICAS_HEAD_DIM 128
#define AICAS_MAX_K 6144

// Scratch memory of the persistent kernel (caller allocates, zero-fills once;
// every launch leaves it ready for the next one).
typedef struct AicasScratch {
  uint64_t bar_count;   // grid barrier arrivals (monotonic across launches)
  uint32_t epoch;       // LL epoch base of the next launch (never reset: see part)
  uint32_t pad0;
  int32_t error;        // first error code raised on the device (0 = none)
  int32_t abort;        // set with `error`; every wait gives up when it is set
  uint32_t argmax_done;
  uint32_t exit_count;  // CTAs finished in the running launch
  float am_val[AICAS_MAX_CTAS];
  int32_t am_idx[AICAS_MAX_CTAS];
  // split-KV partials as 64-bit LL words {fp32 value (low), uint32 epoch
  // (high)}: [kv head][split][group 2][log-sum-exp, normalised acc[128]].
  // A word is accepted when its epoch equals the writing phase's full 32-bit
  // epoch, so `epoch` must keep counting across launches.
  uint64_t part[AICAS_MAX_KV_HEADS][AICAS_MAX_SPLITS][2][AICAS_HEAD_DIM + 1];
} AicasScratch;

// Batched decode (aicas_decode_batch_f16): up to AICAS_MAX_BATCH requests
// ("streams") per launch.  The first eight words are laid out exactly as in
// AicasScratch (the grid barrier, epoch, error and exit words are shared code).
#define AICAS_MAX_BATCH 8
#define AICAS_MAX_PHASES 256

typedef struct AicasBatchScratch {
  uint64_t bar_count;
  uint32_t epoch;
  uint32_t pad0;
  int32_t error;
  int32_t abort;
  uint32_t argmax_done;
  uint32_t exit_count;
  uint32_t launches;                  // launches completed (advanced by the last CTA to exit)
  uint32_t pad1;
  uint32_t done[AICAS_MAX_PHASES];    // per phase: CTAs that finished writing its counted vector,
                                      // (launches + 1) * grid once every CTA has (wraps modulo 2^32)
  float am_val[AICAS_MAX_CTAS][AICAS_MAX_BATCH];   // per-CTA best logit of each stream
  int32_t am_idx[AICAS_MAX_CTAS][AICAS_MAX_BATCH];
  // split-KV partials per (stream, KV head) merge group (64-bit LL words, as above)
  uint64_t part[AICAS_MAX_BATCH * AICAS_MAX_KV_HEADS][AICAS_MAX_SPLITS][2][AICAS_HEAD_DIM + 1];
} AicasBatchScratch;

#ifdef __cplusplus
}
#endif
