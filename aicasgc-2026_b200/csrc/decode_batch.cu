// Batched greedy decode step for B200 (sm_100a): up to 8 requests per launch.
//
// The same phase programs as the batch-1 kernel (decode_program.cu), run for
// nb independent requests ("streams") at once.  Each stream has its own step
// state (token, ragged cache position, 3-axis rope position, script, EOS),
// its own KV cache slice and its own rows of every activation vector.  The
// weights stream from HBM once per step for all streams, so each projection
// is an [nb, k] x [k, n] contraction, and it runs on the tensor cores:
//
//   warp 0      producer: the CTA's weight / KV tiles, phase after phase, into
//               a 3-stage shared-memory ring (cp.async.bulk, L2 evict_first).
//   warps 1..8  consumers.  GEMV phases: build the streams' operand in shared
//               memory (a counted input lands there by bulk copies; the
//               layer-0 embedding rows and LL inputs are loaded or polled),
//               with the RMSNorm prologue at HF's fp16 rounding points; then
//               two sets of 4 warps (one warp per TMEM lane quarter each) run
//               the epilogues of alternate row groups.  Attention: the
//               split-KV units of all streams, tiles taken in pairs, on
//               the tensor cores.
//   warp 9      L2 prefetch cursor, kL2Ahead tiles ahead of the ring.
//   warp 10     MMA issuer and TMEM owner (below).
//
// Weight tile layout (aicas_tile_weight_f16): an 8-row x 2048-column block
// (32 KB) is stored as [256 column groups][8 rows][8 columns], the K-major
// no-swizzle canonical layout of the tcgen05 shared-memory descriptor (8-row x
// 16-byte core matrices), so one bulk copy lands a tile ready for the tensor
// core.  The streams' operand has the same layout with the 8 streams as rows.
//
// Block-pair MMA: the tile is read as a 128 x 128 operand A whose row
// (block j, weight row r) is columns 128 j .. 128 j + 127 of row r (8-row
// core-matrix groups 2 KB apart), and the streams' chunk as B with rows
// (block j', stream s).  8 tcgen05.mma.kind::f16 (M = 128, N = 128, K = 16)
// per tile accumulate fp32 D[(j, r)][(j', s)] in TMEM; the epilogue keeps the
// 16 diagonal blocks j == j': the warp of lane quarter q reads its 4 blocks'
// 32 columns (one tcgen05.ld.32x32b.x32 per part), sums its blocks with
// shuffles, and the set's leader warp adds the 4 quarters in a fixed order
// and applies bias / residual / SiLU / rounding (gate_up: gate and up in the
// two halves of a 256-column slot; down_proj: its 3 K chunks accumulate in
// the same columns).  A tcgen05.commit frees the ring stage when a tile's
// MMAs are done, another marks the slot full.
//
// Activations: qkv is an LL vector (each attention CTA polls only its heads'
// columns); attn, h_mid, act and h are counted vectors (AICAS_F_CNT_*): plain
// fp16 in the operand layout, one release add per CTA and phase on a
// completion counter, one acquire wait and a bulk copy per reader.
//
// KV cache: per (stream, KV head) slice of max_len slots, in the KV tile
// layout: slot p, dim d at element (p / 8) * 1024 + (d / 8) * 64 + (p % 8) * 8
// + d % 8 (8-slot groups of 2 KB; within a group, 16 core matrices of 8 slots
// x 8 dims).  A 64-slot chunk is 16 contiguous KB, so one bulk copy per K / V
// lands it as a tcgen05 operand: K-major for S = K Q^T (LBO 128, SBO 2048)
// and MN-major for O = V^T P^T (LBO 2048, SBO 128).
//
// Attention: units (stream, KV head, 64-slot chunk) over all active streams,
// split contiguously over the CTAs.  A segment's tiles go in pairs (warps 0..3
// and 4..7, one warp per TMEM lane quarter each): per tile one elected thread
// issues S = K Q^T (M = 128, N = 16: the 2 query heads of the KV head, zero
// rows after them) into TMEM; the quarter-0/1 warps read the 64 scores, take
// the tile maximum, and write the fp16 probabilities as the B operand of
// O = V^T P^T (M = 128 head dims); each warp folds its 32 dims of O into the
// running (max, sum, acc).  Each CTA first stores the (log-sum-exp, acc)
// partials of all its segments, then merges its slice of every group it
// shares, in a fixed split order.  Every wait is bounded (aicas_device.cuh);
// after a failed wait the kernel keeps walking the same program without
// waiting and ends with the error recorded.
//
// Reference behaviour per stream (file:line in the reference checkout) is
// that of the batch-1 step: decode_gemv_kernel_fused.cuh:99-185 and
// :850-1076, decode_gemv_kernel_matvec.cuh:209-343,
// decode_attention_v4_kernel.cu:647-900, decode_small_ops_kernel.cu:115-186,
// evaluation_wrapper.py:952 (argmax, first max wins).
#include <atomic>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#include "aicas_decode.h"
#include "aicas_device.cuh"
#include "aicas_phase_program.h"

namespace aicas {

int record_cuda_error(cudaError_t e);  // decode_program.cu

namespace bat {

constexpr int kMaxB = AICAS_MAX_BATCH;
constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = 32 * kConsumerWarps;
constexpr int kL2Warp = 1 + kConsumerWarps;
constexpr int kMmaWarp = kL2Warp + 1;
constexpr int kThreads = 32 * (kMmaWarp + 1);
constexpr int kRows = 8;                        // weight rows per tile (MMA N)
constexpr int kChunk = 2048;                    // columns per tile
constexpr int kTileBytes = kRows * kChunk * 2;  // 32 KB
constexpr int kStages = 3;
constexpr int kMaxC = AICAS_MAX_K / kChunk;     // K chunks of the longest reduction
constexpr int kMmaK = 16;
// One tile (8 weight rows x 2048 columns) is read by the tensor core as a
// 128 x 128 operand: row (block j, weight row r) = columns 128 j .. 128 j + 127
// of weight row r.  The streams' operand is built the same way: row (block
// j', stream s).  So one tile is 8 MMAs of M = 128, N = 128, K = 16, and
// D[(j, r)][(j', s)] is the product of block j of row r with block j' of
// stream s; the epilogue adds the 16 diagonal blocks j == j'.
constexpr int kBlocks = 16;
constexpr int kBlockCols = kChunk / kBlocks;     // 128
constexpr int kKSteps = kBlockCols / kMmaK;      // 8 MMAs per tile
constexpr int kOpSbo = kBlockCols / 8 * 128;     // 2048 bytes between 8-row core-matrix groups
constexpr int kTmemCols = 512;
constexpr int kDCols = kBlocks * kRows;          // 128 accumulator columns per part
constexpr int kDSlots = 2;                       // one per epilogue warp set
constexpr int kDSlotCols = 2 * kDCols;           // gate and up parts
static_assert(kDSlots * kDSlotCols == kTmemCols, "two slots fill the allocation");
constexpr int kAttnChunk = 64;
constexpr int kHD = AICAS_HEAD_DIM;
constexpr int kMergePer = 4;
constexpr int kL2Ahead = 8;
// instruction descriptor: D fp32 (bits 4-5 = 1), A and B fp16 (0), both
// K-major (bits 15, 16 = 0), N >> 3 at bit 17, M >> 4 at bit 24
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(128 >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
// attention: S = K Q^T (M = 128, N = 16, both K-major) and O = V^T P^T (A
// MN-major: bit 15)
constexpr uint32_t kIdescQK = (1u << 4) | ((uint32_t)(16 >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
constexpr uint32_t kIdescPV = kIdescQK | (1u << 15);
// attention operands in the streams' operand buffer (idle during an attention
// phase): the queries [16 rows x 128 dims] at 0, each warp set's
// probabilities [16 rows x 64 slots] at kAttnPOff + set * 2048
constexpr int kAttnPOff = 4096;
constexpr int kAttnOpBytes = kAttnPOff + 2 * 2048;
// TMEM columns of warp set `set` during an attention phase (the GEMV
// accumulators are idle then): S at 64 set, O at 64 set + 32
constexpr int kAttnTmemStride = 64;

// Byte offset of slot r, 8-dim block blk of a tile in the KV tile layout.
__host__ __device__ __forceinline__ uint32_t kvt_off(int r, int blk) {
  return (uint32_t)((r >> 3) * 2048 + blk * 128 + (r & 7) * 16);
}

static_assert(kAttnChunk * kHD * 2 * 2 == kTileBytes, "attention tile must fill one stage");
static_assert(offsetof(AicasBatchScratch, bar_count) == offsetof(AicasScratch, bar_count) &&
                  offsetof(AicasBatchScratch, epoch) == offsetof(AicasScratch, epoch) &&
                  offsetof(AicasBatchScratch, error) == offsetof(AicasScratch, error) &&
                  offsetof(AicasBatchScratch, abort) == offsetof(AicasScratch, abort) &&
                  offsetof(AicasBatchScratch, argmax_done) == offsetof(AicasScratch, argmax_done) &&
                  offsetof(AicasBatchScratch, exit_count) == offsetof(AicasScratch, exit_count),
              "the batch scratch header must match AicasScratch's");

struct StreamIn {
  int64_t token, pos, rope[3], step;
  int32_t active;  // b < nb and the request has not ended
  int32_t pad;
};

struct AttnSmem {
  float kf[kHD], vf[kHD];
  float wm[2][2];  // per warp set: running max, sum (per query head); acc per head dim
  float wl[2][2];
  float wacc[2][2][kHD];
  float tmax[2][2][2];  // per warp set, TMEM lane quarter 0 / 1, head: the tile's maximum score
  float tsum[2][2][2];  // ... and its sum of fp16 probabilities
  __half nw[2 * kHD];   // q_norm, k_norm weights of the running phase
};

struct __align__(128) Smem {
  uint8_t ring[kStages][kTileBytes];
  uint8_t xa[kMaxC * kTileBytes];  // the streams' operand (MMA B): [k/8 column groups][8 streams][8] fp16
  AttnSmem at;
  float rope_c[kMaxB][kHD / 2], rope_s[kMaxB][kHD / 2];
  float ssq[kConsumerWarps][kMaxB];
  // epilogue: per warp set, double-buffered, per lane quarter: [part][row][stream] sums of 4 blocks
  float red[2][2][4][2][kRows][kMaxB];
  float best_v[2][kMaxB];
  int best_i[2][kMaxB];
  StreamIn sin[kMaxB];
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t cempty[kStages];
  uint64_t dfull[kDSlots];
  uint64_t dempty[kDSlots];
  uint64_t xready;  // the streams' operand of the next GEMV phase is in shared memory
  uint64_t cdone;   // all consumer warps are done with TMEM
  uint64_t mdone;   // every MMA the issuer launched has completed
  uint64_t xfull;   // a counted input has landed in the operand buffer (bulk copies)
  uint64_t amma[2];  // per warp set: its attention MMAs (S, then O) have completed
  uint32_t ring_it;
  uint32_t tmem_base;
  int32_t last_cta;
};

struct BatchArgs {
  const AicasPhase* phases;
  int n_phases;
  int nb;
  AicasStepState* states;
  AicasBatchScratch* scratch;
  int64_t* trace;  // traced variant: [grid][n_phases][kTraceFields]
};

// consumer: phase start, inputs ready, phase end; MMA warp: operand ready,
// last MMA of the phase issued; row groups (or attention units) of the CTA;
// ns consumer warp 0 waited for attention tiles; ns the producer waited for
// free ring stages while issuing the phase's tiles
constexpr int kTraceFields = 8;

__device__ __forceinline__ void trace_put(const BatchArgs& a, int ph, int field, int64_t v) {
  a.trace[((size_t)blockIdx.x * a.n_phases + ph) * kTraceFields + field] = v;
}

struct Range {
  int start, count;
};

__device__ __forceinline__ Range split_range(int total, int nct, int cta, int rot) {
  int c = (cta - rot) % nct;
  if (c < 0) c += nct;
  const int base = total / nct, extra = total % nct;
  return {c * base + min(c, extra), base + (c < extra ? 1 : 0)};
}

__device__ __forceinline__ int owner_of(int u, int total, int nct) {
  const int base = total / nct, extra = total % nct;
  const int big = extra * (base + 1);
  if (u < big) return u / (base + 1);
  return extra + (u - big) / base;
}

__device__ __forceinline__ int attn_ctas(int U, int nct) { return max(1, min(nct, U)); }

// Cache slots [0, valid) of stream b in an attention phase; 0 when the
// stream is inactive or its position is outside the cache.
__device__ __forceinline__ int stream_valid(const AicasPhase& d, const StreamIn& in) {
  if (!in.active || in.pos < 0 || in.pos >= d.max_len) return 0;
  return (int)in.pos + 1;
}

// The attention units of a phase: stream b owns units [pre[b], pre[b + 1]),
// KV head h of b units pre[b] + h * cph[b] + [0, cph[b]).
struct AttnUnits {
  int pre[kMaxB + 1];
  int cph[kMaxB];
  int valid[kMaxB];
  __device__ __forceinline__ void init(const AicasPhase& d, const StreamIn* sin, int nb) {
    int U = 0;
#pragma unroll
    for (int b = 0; b < kMaxB; ++b) {
      pre[b] = U;
      valid[b] = b < nb ? stream_valid(d, sin[b]) : 0;
      cph[b] = (valid[b] + kAttnChunk - 1) / kAttnChunk;
      U += d.kv_heads * cph[b];
    }
    pre[kMaxB] = U;
  }
  __device__ __forceinline__ int total() const { return pre[kMaxB]; }
  // stream of unit u: the last b with pre[b] <= u (streams without units are skipped)
  __device__ __forceinline__ int stream_of(int u) const {
    int s = 0;
#pragma unroll
    for (int b = 1; b < kMaxB; ++b)
      if (pre[b] <= u) s = b;
    return s;
  }
};

// a[i] for a small array without dynamic indexing (keeps it in registers)
template <int N>
__device__ __forceinline__ int select_i(const int (&a)[N], int i) {
  int v = a[0];
#pragma unroll
  for (int b = 1; b < N; ++b)
    if (b == i) v = a[b];
  return v;
}

struct TileDesc {
  const uint8_t* src;
  int64_t src_stride;
  uint32_t bytes;
  int pieces;
  bool mma;        // GEMV tile for the tensor core (else an attention tile read in place)
  int c;           // K chunk of the tile
  int part;        // gate_up: 0 gate, 1 up (accumulator columns 8..15)
  bool group_end;  // last tile of its row group: the accumulator slot is complete
};

// Walks this CTA's tiles of the program in the order the consumers take
// them; the producer, the L2 prefetch warp and the MMA issuer each run one.
struct Cursor {
  const AicasPhase* P;
  int n_phases, nct, cta, nb;
  const StreamIn* sin;
  int ph = -1, ti = 0, n = 0;
  int kind, C, T, rows_total;
  Range rg;
  AttnUnits au;

  __device__ __forceinline__ void enter(int phase) {
    ph = phase;
    ti = 0;
    n = 0;
    if (ph >= n_phases) return;
    const AicasPhase& d = P[ph];
    kind = d.kind;
    if (kind == AICAS_PH_ATTN) {
      au.init(d, sin, nb);
      const int U = au.total();
      const int na = attn_ctas(U, nct);
      rg = (U > 0 && cta < na) ? split_range(U, na, cta, 0) : Range{0, 0};
      n = rg.count;
    } else {
      C = d.k / kChunk;
      T = kind == AICAS_PH_GATEUP ? 2 : C;
      rows_total = kind == AICAS_PH_GATEUP ? 2 * d.n : d.n;
      rg = split_range(d.n / kRows, nct, cta, d.rot);
      n = rg.count * T;
    }
  }

  __device__ __forceinline__ bool next(TileDesc& td) {
    while (ti >= n) {
      if (ph >= n_phases) return false;
      enter(ph + 1);
      if (ph >= n_phases) return false;
    }
    const AicasPhase& d = P[ph];
    if (kind == AICAS_PH_ATTN) {
      const int u = rg.start + ti;
      const int b = au.stream_of(u);
      const int cph = select_i(au.cph, b), valid = select_i(au.valid, b);
      const int r = u - select_i(au.pre, b);
      const int h = r / cph, j = r % cph;
      const int p0 = j * kAttnChunk;
      const size_t off = (((size_t)b * d.kv_heads + h) * d.max_len + p0) * kHD * 2;
      td.src = reinterpret_cast<const uint8_t*>(d.k_cache) + off;
      td.src_stride = reinterpret_cast<const uint8_t*>(d.v_cache) - reinterpret_cast<const uint8_t*>(d.k_cache);
      td.bytes = ((min(kAttnChunk, valid - p0) + 7) & ~7) * kHD * 2;  // whole 8-slot groups
      td.pieces = 2;
      td.mma = false;
      td.c = td.part = 0;
      td.group_end = false;
    } else {
      const int g = rg.start + ti / T, t = ti % T;
      const bool gu = kind == AICAS_PH_GATEUP;
      const int c = gu ? 0 : t;
      const int row0 = g * kRows + (gu && t == 1 ? d.n : 0);
      td.src = reinterpret_cast<const uint8_t*>(d.w) + ((size_t)c * rows_total + row0) * kChunk * 2;
      td.src_stride = 0;
      td.bytes = kTileBytes;
      td.pieces = 1;
      td.mma = true;
      td.c = c;
      td.part = gu ? t : 0;
      td.group_end = t == T - 1;
    }
    ++ti;
    return true;
  }
};

// ---------------------------------------------------------------------------
// tcgen05 pieces of the batch kernel
// ---------------------------------------------------------------------------
// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16, issued by one thread.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 8 LL words {fp16 value, epoch} with two 16-byte stores (each word is
// written whole, which is all the LL protocol needs).
__device__ __forceinline__ void ll_store8(uint32_t* p, const float (&y)[8], uint32_t epoch16) {
  uint32_t w[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) w[j] = (epoch16 << 16) | (uint32_t)__half_as_ushort(__float2half_rn(y[j]));
  asm volatile("st.relaxed.gpu.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(w[0]), "r"(w[1]), "r"(w[2]),
               "r"(w[3])
               : "memory");
  asm volatile("st.relaxed.gpu.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p + 4), "r"(w[4]), "r"(w[5]),
               "r"(w[6]), "r"(w[7])
               : "memory");
}

// Completion counters of counted vectors (AICAS_F_CNT_*): one release add per
// CTA and phase; a reader polls with relaxed loads and takes one acquire
// fence once the count is complete (wrap-safe comparison).
__device__ __forceinline__ void red_release_add_u32(uint32_t* p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_relaxed_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ bool wait_count(const uint32_t* p, uint32_t target, AicasScratch* s) {
  if ((int32_t)(ld_relaxed_u32(p) - target) >= 0) {
    fence_acquire_gpu();
    return true;
  }
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if ((int32_t)(ld_relaxed_u32(p) - target) >= 0) {
      fence_acquire_gpu();
      return true;
    }
    if ((it & 31u) == 0) {
      if (ld_volatile_int(&s->abort)) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        raise_error(s, kErrInputTimeout);
        return false;
      }
    }
  }
}

// Byte offset of values [8 v, 8 v + 8) of stream b in a counted vector (the
// batched operand layout [len/8][8 stream slots][8]).
__device__ __forceinline__ size_t cnt_off(int v, int b) { return ((size_t)v * kMaxB + b) * 16; }

// ---------------------------------------------------------------------------
// Producer, L2 prefetch, MMA issuer
// ---------------------------------------------------------------------------
template <bool kTrace>
__device__ __forceinline__ void run_producer(const BatchArgs& a, Smem& sm, AicasScratch* s) {
  if ((threadIdx.x & 31) != 0) return;
  const uint64_t pol = l2_evict_first_policy();
  Cursor cur{a.phases, a.n_phases, (int)gridDim.x, (int)blockIdx.x, a.nb, sm.sin};
  TileDesc td;
  uint32_t it = 0;
  int tph = 0;
  uint64_t waited = 0;
  while (cur.next(td)) {
    const int st = it % kStages;
    if (kTrace && cur.ph != tph) {
      trace_put(a, tph, 7, (int64_t)waited);
      waited = 0;
      tph = cur.ph;
    }
    const uint64_t w0 = kTrace ? globaltimer_ns() : 0;
    if (it >= (uint32_t)kStages && !mbar_wait_bounded(&sm.empty[st], ((it / kStages) - 1) & 1u, s, kErrEmptyTimeout))
      break;
    if (kTrace) waited += globaltimer_ns() - w0;
    mbar_arrive_expect_tx(&sm.full[st], td.pieces * td.bytes);
    for (int i = 0; i < td.pieces; ++i)
      bulk_g2s(sm.ring[st] + i * (kTileBytes / 2), td.src + i * td.src_stride, td.bytes, &sm.full[st], pol);
    ++it;
    *reinterpret_cast<volatile uint32_t*>(&sm.ring_it) = it;
  }
  if (kTrace) trace_put(a, tph, 7, (int64_t)waited);
  // every issued copy lands before the CTA may exit
  const uint32_t first = it > (uint32_t)kStages ? it - kStages : 0;
  for (uint32_t k = first; k < it; ++k) {
    const int st = k % kStages;
    if (!mbar_wait_bounded(&sm.full[st], (k / kStages) & 1u, s, kErrDrainTimeout)) {
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&sm.full[st], (k / kStages) & 1u)) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) break;
      }
    }
  }
}

__device__ __forceinline__ void run_l2_prefetcher(const BatchArgs& a, Smem& sm, AicasScratch* s) {
  if ((threadIdx.x & 31) != 0) return;
  Cursor pf{a.phases, a.n_phases, (int)gridDim.x, (int)blockIdx.x, a.nb, sm.sin};
  TileDesc td;
  const uint64_t pol_last = l2_evict_last_policy();
  for (uint32_t k = 0; pf.next(td); ++k) {
    uint64_t t0 = 0;
    uint32_t ri = 0;
    for (uint32_t it = 0;; ++it) {
      ri = *reinterpret_cast<volatile uint32_t*>(&sm.ring_it);
      if (k < ri + (uint32_t)kL2Ahead) break;
      if (it == 0) t0 = globaltimer_ns();
      if ((it & 15u) == 15u && (ld_volatile_int(&s->abort) || globaltimer_ns() - t0 > kWaitLimitNs)) return;
      __nanosleep(128);
    }
    if (k < ri) continue;
    for (int i = 0; i < td.pieces; ++i) bulk_prefetch_l2_hint(td.src + i * td.src_stride, td.bytes, pol_last);
  }
}

// MMA issuer (lane 0 of the last warp; the whole warp owns the TMEM
// allocation).  GEMV tiles: wait for the phase's streams' operand (once per phase),
// a free accumulator slot (first tile of a row group) and the landed tile,
// issue the tile's 128 MMAs, commit the stage (and the slot at the group's
// last tile).  Attention tiles: pass the consumers' in-place release on to
// the producer.
template <bool kTrace>
__device__ __forceinline__ void run_mma(const BatchArgs& a, Smem& sm, AicasScratch* s, uint32_t tmem) {
  const int lane = threadIdx.x & 31;
  if (lane == 0) {
    Cursor cur{a.phases, a.n_phases, (int)gridDim.x, (int)blockIdx.x, a.nb, sm.sin};
    TileDesc td;
    uint32_t it = 0, gc = 0, xph = 0, cpar = 0;
    int x_phase = -1;
    const uint32_t xa0 = smem_addr(sm.xa);
    const uint32_t ring0 = smem_addr(sm.ring[0]);
    while (cur.next(td)) {
      const int st = it % kStages;
      const uint32_t par = (it / kStages) & 1u;
      if (td.mma) {
        if (cur.ph != x_phase) {
          if (!mbar_wait_bounded(&sm.xready, xph & 1u, s, kErrTmemTimeout)) break;
          ++xph;
          x_phase = cur.ph;
          if (kTrace) trace_put(a, cur.ph, 3, (int64_t)globaltimer_ns());
        }
        const uint32_t slot = gc % kDSlots;
        if (td.c == 0 && td.part == 0 && gc >= (uint32_t)kDSlots &&
            !mbar_wait_bounded(&sm.dempty[slot], ((gc / kDSlots) - 1) & 1u, s, kErrTmemTimeout))
          break;
        if (!mbar_wait_bounded(&sm.full[st], par, s, kErrFullTimeout)) break;
        tc_fence_after();
        // A = the weight tile, B = the streams' chunk c: 8-row core-matrix
        // groups (blocks) 2 KB apart, K-adjacent core matrices 128 B apart;
        // K step ks starts 256 bytes further (16 units of the address field)
        const uint64_t adesc = smem_desc_kmajor(ring0 + st * kTileBytes, 128, kOpSbo);
        const uint64_t bdesc = smem_desc_kmajor(xa0 + td.c * kTileBytes, 128, kOpSbo);
        const uint32_t d = tmem + slot * kDSlotCols + td.part * kDCols;
#pragma unroll
        for (int ks = 0; ks < kKSteps; ++ks)
          umma_f16(d, adesc + 16u * ks, bdesc + 16u * ks, kIdesc, (ks > 0 || td.c > 0) ? 1u : 0u);
        if (kTrace) trace_put(a, cur.ph, 4, (int64_t)globaltimer_ns());
        tcgen05_commit(&sm.empty[st]);
        if (td.group_end) {
          tcgen05_commit(&sm.dfull[slot]);
          ++gc;
        }
      } else {
        // the stage goes back to the producer only once its copy has landed
        // (after an abort a consumer may release it without having waited)
        if (!mbar_wait_bounded(&sm.full[st], par, s, kErrFullTimeout)) break;
        if (!mbar_wait_bounded(&sm.cempty[st], (cpar >> st) & 1u, s, kErrEmptyTimeout)) break;
        cpar ^= 1u << st;
        mbar_arrive(&sm.empty[st]);
      }
      ++it;
    }
    // every MMA launched so far has completed before TMEM may be freed
    tcgen05_commit(&sm.mdone);
    uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(&sm.mdone, 0)) {
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        raise_error(s, kErrTmemTimeout);
        break;
      }
    }
    t0 = globaltimer_ns();
    while (!mbar_try_wait(&sm.cdone, 0)) {
      if (globaltimer_ns() - t0 > 2 * kWaitLimitNs) {
        raise_error(s, kErrTmemTimeout);
        break;
      }
    }
  }
  __syncwarp();
  tc_fence_after();
  tmem_dealloc(tmem, kTmemCols);
}

// ---------------------------------------------------------------------------
// Consumers (warps 1..8)
// ---------------------------------------------------------------------------
template <bool kTrace>
struct Consumer {
  const BatchArgs& a;
  Smem& sm;
  AicasScratch* s;
  AicasBatchScratch* bs;
  int tid, w, lane, nct, cta, nb;
  uint32_t tmem;
  uint32_t epoch_base;
  uint32_t cnt_target = 0;  // completion count of a counted vector in this launch: (launches + 1) * grid
  uint32_t xfull_n = 0;     // completions of sm.xfull so far
  uint32_t gc = 0;   // accumulator groups consumed (epilogue warps)
  uint32_t rit = 0;  // ring tiles passed (GEMV tiles via the MMA warp, attention tiles read in place)
  uint32_t acnt = 0;  // completed attention MMA groups of this warp's set (sm.amma parity)
  int ph = 0;

  __device__ __forceinline__ bool active(int b) const { return b < nb && sm.sin[b].active; }

  __device__ __forceinline__ int64_t checked_token(int b, int rows) {
    const int64_t t = sm.sin[b].token;
    if (t >= 0 && t < rows) return t;
    raise_error(s, kErrBadInput);
    return 0;
  }

  // Interleaved-MRoPE cos/sin of every active stream's position, once per
  // launch (modeling_qwen3_vl.py:352-386): frequency i takes axis 1 (h) when
  // i % 3 == 1 and i < 3 section[1], axis 2 (w) when i % 3 == 2 and
  // i < 3 section[2], else axis 0 (t); fp32 math, rounded to fp16.
  __device__ __noinline__ void init_rope() {
    for (int e = tid; e < kMaxB * (kHD / 2); e += kConsumerThreads) {
      const int b = e / (kHD / 2), i = e % (kHD / 2);
      if (!active(b)) continue;
      const AicasStepState* stt = a.states + b;
      int axis = 0;
      if (i % 3 == 1 && i < 3 * stt->mrope_section[1]) axis = 1;
      else if (i % 3 == 2 && i < 3 * stt->mrope_section[2]) axis = 2;
      const float ang = stt->inv_freq[i] * (float)sm.sin[b].rope[axis];
      sm.rope_c[b][i] = r16(cosf(ang));
      sm.rope_s[b][i] = r16(sinf(ang));
    }
  }

  // The streams' operand of a GEMV phase: thread (b = tid % 8, g = tid / 8) takes
  // column groups v = g + 32 i of stream b (8 columns each), so the 8 lanes
  // of a lane octet write one contiguous 128-byte core-matrix row set.
  // RMSNorm (F_NORM, k == 2048) with HF's rounding points
  // (modeling_qwen3_vl.py:398-403).  Inactive streams read as zeros.
  __device__ __forceinline__ void build_x(const AicasPhase& d) {
    const int k = d.k, C = k / kChunk;
    const int b = tid & 7, g = tid >> 3;
    const bool act = active(b);
    if (d.flags & AICAS_F_CNT_IN) {
      build_x_counted(d);
      return;
    }
    const uint32_t ep = (epoch_base + (uint32_t)d.x_src + 1) & 0xffffu;
    const bool ll = d.flags & AICAS_F_LL_IN;
    const uint32_t* xw = reinterpret_cast<const uint32_t*>(d.x) + (size_t)b * k;
    const __half* xh = reinterpret_cast<const __half*>(d.x);
    if (d.flags & AICAS_F_X_EMBED) xh += (act ? (size_t)checked_token(b, d.embed_rows) : 0) * k;
    else xh += (size_t)b * k;
    for (int i0 = 0; i0 < 8 * C; i0 += 8) {
      int cols[8];
      uint4 raw[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) cols[i] = act ? 8 * (g + 32 * (i0 + i)) : -1;
      if (ll) {
        ll_poll8_n<8>(xw, cols, ep, s, raw);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) raw[i] = cols[i] >= 0 ? ldcg_u4(xh + cols[i]) : make_uint4(0, 0, 0, 0);
      }
      if (d.flags & AICAS_F_NORM) {  // k == 2048: this is the only round
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const __half2* hp = reinterpret_cast<const __half2*>(&raw[i]);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 f = __half22float2(hp[q]);
            ss += f.x * f.x + f.y * f.y;
          }
        }
        // lanes l, l ^ 8, l ^ 16, l ^ 24 hold the same stream
        ss += __shfl_xor_sync(0xffffffffu, ss, 8);
        ss += __shfl_xor_sync(0xffffffffu, ss, 16);
        if (lane < 8) sm.ssq[w][lane] = ss;
        consumer_sync(kConsumerThreads);
        float tot = 0.f;
#pragma unroll
        for (int i = 0; i < kConsumerWarps; ++i) tot += sm.ssq[i][b];
        const float inv = rsqrtf(tot / (float)k + d.eps);
        const __half* nw = reinterpret_cast<const __half*>(d.norm_w);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint4 wr = __ldg(reinterpret_cast<const uint4*>(nw + 8 * (g + 32 * i)));
          __half2* hp = reinterpret_cast<__half2*>(&raw[i]);
          const __half2* wp = reinterpret_cast<const __half2*>(&wr);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 f = __half22float2(hp[q]);
            const float2 wf = __half22float2(wp[q]);
            hp[q] = __floats2half2_rn(wf.x * r16(f.x * inv), wf.y * r16(f.y * inv));
          }
          if (!act) raw[i] = make_uint4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int v = g + 32 * (i0 + i);  // column group 0 .. k/8 - 1
        *reinterpret_cast<uint4*>(sm.xa + (v / 256) * kTileBytes + (v % 256) * 128 + b * 16) = raw[i];
      }
    }
    // the MMA reads the operand through the async proxy
    fence_proxy_async_smem();
    consumer_sync(kConsumerThreads);
    if (tid == 0) mbar_arrive(&sm.xready);
    if (kTrace && tid == 0) trace_put(a, ph, 1, (int64_t)globaltimer_ns());
  }

  // A counted input: wait until every CTA has written its part, then copy the
  // vector (already in the operand layout: piece i = 16 bytes of stream i % 8)
  // into the streams' operand, applying the RMSNorm prologue (k == 2048) on the way.
  // Thread tid copies pieces tid, tid + 256, ...: all of stream tid % 8.
  __device__ __forceinline__ void build_x_counted(const AicasPhase& d) {
    const int k = d.k;
    const int b = tid & 7;
    const bool act = active(b);
    // thread 0: wait for the count, then copy the whole vector (8 streams x k
    // values, k / 2048 pieces of 32 KB) with bulk async copies; the other
    // threads wait for the copies to land.  The fence orders the acquired
    // generic-proxy data before the copies' async-proxy reads.
    if (tid == 0) {
      wait_count(&bs->done[d.x_src], cnt_target, s);
      asm volatile("fence.proxy.async.global;" ::: "memory");
      const int pieces = k / kChunk;
      mbar_arrive_expect_tx(&sm.xfull, pieces * kTileBytes);
      for (int c = 0; c < pieces; ++c)
        bulk_g2s(sm.xa + c * kTileBytes, reinterpret_cast<const uint8_t*>(d.x) + (size_t)c * kTileBytes, kTileBytes,
                 &sm.xfull, l2_evict_last_policy());
    }
    mbar_wait_copy(&sm.xfull, xfull_n & 1u, s, kErrFullTimeout);
    ++xfull_n;
    const uint4* src = reinterpret_cast<const uint4*>(sm.xa);
    uint4* dst = reinterpret_cast<uint4*>(sm.xa);
    if (d.flags & AICAS_F_NORM) {  // k == 2048: 8 pieces per thread
      uint4 raw[8];
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        raw[i] = act ? src[tid + kConsumerThreads * i] : make_uint4(0, 0, 0, 0);
        const __half2* hp = reinterpret_cast<const __half2*>(&raw[i]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = __half22float2(hp[q]);
          ss += f.x * f.x + f.y * f.y;
        }
      }
      ss += __shfl_xor_sync(0xffffffffu, ss, 8);
      ss += __shfl_xor_sync(0xffffffffu, ss, 16);
      if (lane < 8) sm.ssq[w][lane] = ss;
      consumer_sync(kConsumerThreads);
      float tot = 0.f;
#pragma unroll
      for (int i = 0; i < kConsumerWarps; ++i) tot += sm.ssq[i][b];
      const float inv = rsqrtf(tot / (float)k + d.eps);
      const __half* nw = reinterpret_cast<const __half*>(d.norm_w);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int v = (tid + kConsumerThreads * i) >> 3;  // column group
        const uint4 wr = __ldg(reinterpret_cast<const uint4*>(nw + 8 * v));
        __half2* hp = reinterpret_cast<__half2*>(&raw[i]);
        const __half2* wp = reinterpret_cast<const __half2*>(&wr);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = __half22float2(hp[q]);
          const float2 wf = __half22float2(wp[q]);
          hp[q] = __floats2half2_rn(wf.x * r16(f.x * inv), wf.y * r16(f.y * inv));
        }
        dst[tid + kConsumerThreads * i] = act ? raw[i] : make_uint4(0, 0, 0, 0);
      }
    } else if (!act) {  // streams that are not running read as zeros
      const int pieces = k;  // 8 streams x k values x 2 bytes / 16
      for (int i = tid; i < pieces; i += kConsumerThreads) dst[i] = make_uint4(0, 0, 0, 0);
    }
    fence_proxy_async_smem();
    consumer_sync(kConsumerThreads);
    if (tid == 0) mbar_arrive(&sm.xready);
    if (kTrace && tid == 0) trace_put(a, ph, 1, (int64_t)globaltimer_ns());
  }

  __device__ __forceinline__ void run_gemv(const AicasPhase& d) {
    const int n = d.n, flags = d.flags, kind = d.kind;
    const Range rg = split_range(n / kRows, nct, cta, d.rot);
    const bool lm = kind == AICAS_PH_LMHEAD;
    if (kTrace && tid == 0) trace_put(a, ph, 5, rg.count);
    // the MMA warp consumes these tiles; the ring position moves past them
    rit += rg.count * (kind == AICAS_PH_GATEUP ? 2 : d.k / kChunk);
    if (rg.count > 0) build_x(d);
    float best_v = -INFINITY;
    int best_i = 0x7fffffff;
    if (rg.count > 0) {
      // Row groups alternate between two sets of 4 warps (consumer warps
      // 0..3 and 4..7: TMEM lane quarters 1, 2, 3, 0 each) and the two
      // accumulator slots.  Warp of quarter q reads the 32 columns of its
      // 4 blocks j = 4q .. 4q + 3 (lane l: block 4q + l / 8, weight row
      // l % 8), keeps its diagonal block, sums its 4 blocks by shuffles and
      // hands the row sums to the set's leader warp through shared memory.
      const bool gu = kind == AICAS_PH_GATEUP;
      const int set = w >> 2, q = (w + 1) & 3, sub = lane >> 3;
      const bool leader = (w & 3) == 0;
      const int b = lane;  // leader lanes: one stream each
      const bool act = leader && b < kMaxB && active(b);
      const uint32_t ep16 = (epoch_base + (uint32_t)ph + 1) & 0xffffu;
      uint32_t* const out = reinterpret_cast<uint32_t*>(d.out);
      const __half* const bias = reinterpret_cast<const __half*>(d.bias);
      __half* logits = nullptr;
      if (lm && act) {
        const AicasStepState* stt = a.states + b;
        if (stt->logits) {
          const int64_t ring = stt->logits_ring > 0 ? stt->logits_ring : 1;
          logits = reinterpret_cast<__half*>(stt->logits) + (size_t)(sm.sin[b].step % ring) * n;
        }
      }
      const __half* embed_row = nullptr;
      if ((flags & AICAS_F_RESID_EMBED) && act)
        embed_row = reinterpret_cast<const __half*>(d.resid) + (size_t)checked_token(b, d.embed_rows) * n;
      const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16) + 32 * q;  // lanes 32q.., columns of blocks 4q..
      for (int gi = 0; gi < rg.count; ++gi, ++gc) {
        if ((int)(gc & 1u) != set) continue;
        const uint32_t slot = gc & 1u;  // == set
        const int buf = (gc >> 1) & 1;
        mbar_wait_bounded(&sm.dfull[slot], (gc >> 1) & 1u, s, kErrTmemTimeout);
        tc_fence_after();
        // one part (gate, then up) at a time: 32 accumulator registers live
#pragma unroll 1
        for (int p2 = 0; p2 < (gu ? 2 : 1); ++p2) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tq + slot * kDSlotCols + p2 * kDCols, v);
          tmem_wait_ld();
          if (p2 == (gu ? 1 : 0)) {  // the slot's last read: release it
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.dempty[slot]);
          }
          float part[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {  // the diagonal block's column of stream j
            const uint32_t x0 = v[j], x1 = v[8 + j], x2 = v[16 + j], x3 = v[24 + j];
            part[j] = __uint_as_float(sub == 0 ? x0 : sub == 1 ? x1 : sub == 2 ? x2 : x3);
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) {  // blocks of the quarter: lanes l, l ^ 8, l ^ 16, l ^ 24
            part[j] += __shfl_xor_sync(0xffffffffu, part[j], 8);
            part[j] += __shfl_xor_sync(0xffffffffu, part[j], 16);
          }
          if (lane < kRows) {  // lane r: weight row r of the group
#pragma unroll
            for (int j = 0; j < 8; ++j) sm.red[set][buf][q][p2][lane][j] = part[j];
          }
        }
        asm volatile("bar.sync %0, 128;" ::"r"(2 + set) : "memory");
        if (!act) continue;
        float sum[2][8];
#pragma unroll
        for (int p2 = 0; p2 < 2; ++p2)
#pragma unroll
          for (int r = 0; r < 8; ++r) {
            float t = 0.f;
            if (p2 == 0 || gu) {
#pragma unroll
              for (int q2 = 0; q2 < 4; ++q2) t += sm.red[set][buf][q2][p2][r][b];
            }
            sum[p2][r] = t;
          }
        const int row0 = (rg.start + gi) * kRows;
        float y[8];
        if (gu) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float gq = r16(sum[0][j]), uq = r16(sum[1][j]);
            const float sl = r16(gq / (1.0f + expf(-gq)));
            y[j] = r16(sl * uq);
          }
        } else {
          float rv[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) rv[j] = 0.f;
          if (flags & AICAS_F_RESID) {
            if (flags & AICAS_F_CNT_RESID) {  // counted, complete before this phase
              const uint4 r = ldcg_u4(reinterpret_cast<const uint8_t*>(d.resid) + cnt_off(row0 / 8, b));
              const __half2* hp = reinterpret_cast<const __half2*>(&r);
#pragma unroll
              for (int h2 = 0; h2 < 4; ++h2) {
                rv[2 * h2] = __low2float(hp[h2]);
                rv[2 * h2 + 1] = __high2float(hp[h2]);
              }
            } else if (flags & AICAS_F_LL_RESID) {  // complete before this phase: data only
              const uint32_t* rw = reinterpret_cast<const uint32_t*>(d.resid) + (size_t)b * n + row0;
              const uint4 r0 = ll_load4w(rw), r1 = ll_load4w(rw + 4);
              const uint32_t rr[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
#pragma unroll
              for (int j = 0; j < 8; ++j) rv[j] = __half2float(__ushort_as_half((unsigned short)(rr[j] & 0xffffu)));
            } else {
              const __half* rp = embed_row ? embed_row : reinterpret_cast<const __half*>(d.resid) + (size_t)b * n;
              const uint4 r = ldcg_u4(rp + row0);
              const __half2* hp = reinterpret_cast<const __half2*>(&r);
#pragma unroll
              for (int h2 = 0; h2 < 4; ++h2) {
                rv[2 * h2] = __low2float(hp[h2]);
                rv[2 * h2 + 1] = __high2float(hp[h2]);
              }
            }
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            float acc = sum[0][j];
            if (flags & AICAS_F_BIAS) acc += __half2float(bias[row0 + j]);
            y[j] = r16(acc);
            if (flags & AICAS_F_RESID) y[j] = r16(rv[j] + y[j]);
          }
        }
        if (lm) {
          if (logits) {
            __half2 hv[4];
#pragma unroll
            for (int h2 = 0; h2 < 4; ++h2) hv[h2] = __floats2half2_rn(y[2 * h2], y[2 * h2 + 1]);
            *reinterpret_cast<uint4*>(logits + row0) = *reinterpret_cast<const uint4*>(hv);
          }
          // this lane's rows ascend: strict > keeps the first max
#pragma unroll
          for (int j = 0; j < 8; ++j)
            if (y[j] > best_v) {
              best_v = y[j];
              best_i = row0 + j;
            }
        } else if (flags & AICAS_F_CNT_OUT) {
          __half2 hv[4];
#pragma unroll
          for (int h2 = 0; h2 < 4; ++h2) hv[h2] = __floats2half2_rn(y[2 * h2], y[2 * h2 + 1]);
          *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(d.out) + cnt_off(row0 / 8, b)) =
              *reinterpret_cast<const uint4*>(hv);
        } else {
          ll_store8(out + (size_t)b * n + row0, y, ep16);
        }
      }
    }
    if (lm) finish_argmax(best_v, best_i);
  }

  // Per stream: the best (value, row) of the two sets' leader warps, then of all
  // CTAs (the last CTA to arrive reduces, one warp per stream, and advances
  // the stream's step state exactly like the batch-1 kernel).
  __device__ __forceinline__ void finish_argmax(float bv, int bi) {
    if ((w & 3) == 0 && lane < kMaxB) {  // the two sets' leader warps
      sm.best_v[w >> 2][lane] = bv;
      sm.best_i[w >> 2][lane] = bi;
    }
    consumer_sync(kConsumerThreads);
    if (tid < kMaxB) {
      float v = sm.best_v[0][tid];
      int i = sm.best_i[0][tid];
      if (sm.best_v[1][tid] > v || (sm.best_v[1][tid] == v && sm.best_i[1][tid] < i)) {
        v = sm.best_v[1][tid];
        i = sm.best_i[1][tid];
      }
      bs->am_val[cta][tid] = v;
      bs->am_idx[cta][tid] = i;
    }
    consumer_sync(kConsumerThreads);
    if (tid == 0) {
      __threadfence();
      const uint32_t prev = atomicAdd(&bs->argmax_done, 1u);
      sm.last_cta = prev == (uint32_t)nct - 1;
    }
    consumer_sync(kConsumerThreads);
    if (!sm.last_cta) return;
    __threadfence();
    const int b = w;  // one warp per stream
    if (active(b)) {
      float v = -INFINITY;
      int i = 0x7fffffff;
      for (int c = lane; c < nct; c += 32) {
        const float cv = __ldcg(&bs->am_val[c][b]);
        const int ci = __ldcg(&bs->am_idx[c][b]);
        if (cv > v || (cv == v && ci < i)) {
          v = cv;
          i = ci;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
        const int i2 = __shfl_xor_sync(0xffffffffu, i, o);
        if (v2 > v || (v2 == v && i2 < i)) {
          v = v2;
          i = i2;
        }
      }
      if (lane == 0) {
        AicasStepState* stt = a.states + b;
        const StreamIn& in = sm.sin[b];
        const int64_t step = in.step;
        if (stt->out_tokens && step < stt->max_steps) stt->out_tokens[step] = i;
        const int64_t nx = step + 1;
        if (stt->script && nx < stt->script_len) {
          const int64_t* e = stt->script + nx * 5;
          stt->token = e[0];
          stt->cache_pos = e[1];
          stt->rope[0] = e[2];
          stt->rope[1] = e[3];
          stt->rope[2] = e[4];
        } else {
          stt->token = i;
          stt->cache_pos = in.pos + 1;
          stt->rope[0] = in.rope[0] + 1;
          stt->rope[1] = in.rope[1] + 1;
          stt->rope[2] = in.rope[2] + 1;
        }
        stt->step = nx;
        if (stt->eos_token >= 0 && i == stt->eos_token && nx >= stt->script_len) stt->done_step = nx;
        __threadfence();
      }
    }
    if (tid == 0) bs->argmax_done = 0;
  }

  // One 128-dim head per warp (lane l holds dims 4l..4l+3): per-head RMSNorm
  // (modeling_qwen3_vl.py:398-403) and rotary embedding (:124-128, :427-431).
  __device__ __forceinline__ void norm_rope_head(float (&v)[4], const __half* nw, float eps, const float (&cs)[4],
                                                 const float (&sn)[4]) {
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) ss += v[e] * v[e];
    const float inv = rsqrtf(warp_sum(ss) / (float)kHD + eps);
    float xn[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) xn[e] = r16(__half2float(nw[lane * 4 + e]) * r16(v[e] * inv));
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float p = __shfl_xor_sync(0xffffffffu, xn[e], 16);
      const float rot = lane < 16 ? -p : p;
      v[e] = r16(r16(xn[e] * cs[e]) + r16(rot * sn[e]));
    }
  }

  // Named barrier of warp set `set` (consumer warps 4 set .. 4 set + 3).
  __device__ __forceinline__ static void set_sync(int set) {
    asm volatile("bar.sync %0, 128;" ::"r"(2 + set) : "memory");
  }

  // One 64-slot K/V tile (ring stage st, KV tile layout) for warp set `set`
  // on the tensor cores; q = this warp's TMEM lane quarter, n = valid slots
  // of the tile, prow = this step's slot in the tile (-1: none).
  //   1. This step's k / v row (it may have been written after the tile was
  //      copied) and zeros for V rows [n, 16 ceil(n / 16)) go into the
  //      staged tile, so the last O = V^T P^T step reads no stale slot.
  //   2. S = K Q^T: 8 MMAs of M = 128 (TMEM lanes 0..63: the tile's slots;
  //      lanes 64..127 read the V half behind the K tile and are ignored),
  //      N = 16 (query heads 2h, 2h + 1, then zero rows), fp32 in TMEM.
  //   3. Lane quarters 0 and 1 (slot = TMEM lane) mask slots >= n, scale,
  //      take the tile maximum per head, and write P = exp(s - m) as fp16 in
  //      the B operand of step 4 (the sum uses the rounded values).
  //   4. O = V^T P^T: ceil(n / 16) MMAs of M = 128 (head dims), K = 16 slots.
  //   5. Each warp reads its 32 dims of O and folds them into (m, l, acc).
  // The elected thread (lane 0 of the set's first warp) issues the MMAs; a
  // commit on sm.amma[set] marks each group done (waited by every thread
  // of the set, ignoring the abort word: no MMA is still reading the stage
  // or writing TMEM when the set moves on).
  __device__ __forceinline__ void attend_tile_tc(int set, int q, int st, int n, int prow, float scale,
                                                 float (&m)[2], float (&l)[2], float (&acc)[2]) {
    AttnSmem& at = sm.at;
    uint8_t* const tile = sm.ring[st];
    const int tl = (w & 3) * 32 + lane;  // thread of the set
    const int n16 = (n + 15) & ~15;
    if (prow >= 0 || n < n16) {
      if (prow >= 0 && tl < 32) {  // 16 lanes K, 16 lanes V: 8 dims each
        const int kv = tl >> 4, blk = tl & 15;
        const float* src = (kv == 0 ? at.kf : at.vf) + blk * 8;
        uint4 pk;
        __half2* ph = reinterpret_cast<__half2*>(&pk);
#pragma unroll
        for (int e = 0; e < 4; ++e) ph[e] = __floats2half2_rn(src[2 * e], src[2 * e + 1]);
        *reinterpret_cast<uint4*>(tile + kv * (kTileBytes / 2) + kvt_off(prow, blk)) = pk;
      }
      for (int i = tl; i < (n16 - n) * 16; i += 128)
        *reinterpret_cast<uint4*>(tile + kTileBytes / 2 + kvt_off(n + i / 16, i % 16)) = make_uint4(0, 0, 0, 0);
      fence_proxy_async_smem();
    }
    set_sync(set);
    const bool leader = tl == 0;
    const uint32_t t_s = smem_addr(tile), q_s = smem_addr(sm.xa), p_s = q_s + kAttnPOff + set * 2048;
    const uint32_t dS = tmem + set * kAttnTmemStride, dO = dS + 32;
    if (leader) {
      tc_fence_after();
#pragma unroll
      for (int ks = 0; ks < kHD / kMmaK; ++ks)
        umma_f16(dS, smem_desc_kmajor(t_s + 256 * ks, 128, 2048), smem_desc_kmajor(q_s + 256 * ks, 128, 2048),
                 kIdescQK, ks > 0 ? 1u : 0u);
      tcgen05_commit(&sm.amma[set]);
    }
    mbar_wait_copy(&sm.amma[set], acnt & 1u, s, kErrTmemTimeout);
    ++acnt;
    tc_fence_after();
    float x0 = -INFINITY, x1 = -INFINITY;
    const int r = 32 * q + lane;  // the slot of this lane (quarters 0, 1)
    if (q < 2) {
      uint32_t s0, s1;
      tmem_ld_32x32b_x2(dS + ((uint32_t)(32 * q) << 16), s0, s1);
      tmem_wait_ld();
      if (r < n) {
        x0 = __uint_as_float(s0) * scale;
        x1 = __uint_as_float(s1) * scale;
      }
      const float t0 = warp_max(x0), t1 = warp_max(x1);
      if (lane == 0) {
        at.tmax[set][q][0] = t0;
        at.tmax[set][q][1] = t1;
      }
    }
    set_sync(set);
    float mn[2];
#pragma unroll
    for (int g = 0; g < 2; ++g) mn[g] = fmaxf(m[g], fmaxf(at.tmax[set][0][g], at.tmax[set][1][g]));
    if (q < 2) {
      const __half p0 = __float2half_rn(x0 == -INFINITY ? 0.f : expf(x0 - mn[0]));
      const __half p1 = __float2half_rn(x1 == -INFINITY ? 0.f : expf(x1 - mn[1]));
      // B operand [16 rows x 64 slots], K-major: row g, slot r at (r / 8) 128 + g 16 + (r % 8) 2
      uint8_t* pb = sm.xa + kAttnPOff + set * 2048 + (r >> 3) * 128 + (r & 7) * 2;
      *reinterpret_cast<__half*>(pb) = p0;
      *reinterpret_cast<__half*>(pb + 16) = p1;
      const float s0 = warp_sum(__half2float(p0)), s1 = warp_sum(__half2float(p1));
      if (lane == 0) {
        at.tsum[set][q][0] = s0;
        at.tsum[set][q][1] = s1;
      }
      fence_proxy_async_smem();
    }
    tc_fence_before();
    set_sync(set);
    if (leader) {
      tc_fence_after();
      for (int ks = 0; ks < n16 / kMmaK; ++ks)
        umma_f16(dO, smem_desc_kmajor(t_s + kTileBytes / 2 + 4096 * ks, 2048, 128),
                 smem_desc_kmajor(p_s + 256 * ks, 128, 1024), kIdescPV, ks > 0 ? 1u : 0u);
      tcgen05_commit(&sm.amma[set]);
    }
    mbar_wait_copy(&sm.amma[set], acnt & 1u, s, kErrTmemTimeout);
    ++acnt;
    tc_fence_after();
    uint32_t o0, o1;
    tmem_ld_32x32b_x2(dO + ((uint32_t)(32 * q) << 16), o0, o1);
    tmem_wait_ld();
    const float ov[2] = {__uint_as_float(o0), __uint_as_float(o1)};
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      const float corr = m[g] == -INFINITY ? 0.f : expf(m[g] - mn[g]);
      l[g] = l[g] * corr + (at.tsum[set][0][g] + at.tsum[set][1][g]);
      acc[g] = acc[g] * corr + ov[g];
      m[g] = mn[g];
    }
    tc_fence_before();
  }

  __device__ __forceinline__ void run_attention(const AicasPhase& d) {
    AttnSmem& at = sm.at;
    AttnUnits au;
    au.init(d, sm.sin, nb);
    const int U = au.total();
    if (tid == 0 && cta == 0) {
      for (int b = 0; b < nb; ++b)
        if (active(b) && au.valid[b] == 0) raise_error(s, kErrBadInput);
    }
    if (U == 0) return;
    const int na = attn_ctas(U, nct);
    const Range rg = cta < na ? split_range(U, na, cta, 0) : Range{0, 0};
    if (kTrace && tid == 0) trace_put(a, ph, 5, rg.count);
    // the MMA operands' zero rows: queries and both sets' probabilities
    // (the streams' operand buffer is idle until the next GEMV phase)
    for (int i = tid; i < kAttnOpBytes / 16; i += kConsumerThreads)
      reinterpret_cast<uint4*>(sm.xa)[i] = make_uint4(0, 0, 0, 0);
    fence_proxy_async_smem();
    tc_fence_before();  // the previous phase's TMEM reads come before these MMAs
    consumer_sync(kConsumerThreads);
    uint64_t tile_wait = 0, seg_ns = 0;
    const uint32_t* qkv_w = reinterpret_cast<const uint32_t*>(d.x);
    const uint32_t x_epoch = (epoch_base + (uint32_t)d.x_src + 1) & 0xffffu;
    __half* kc = reinterpret_cast<__half*>(d.k_cache);
    __half* vc = reinterpret_cast<__half*>(d.v_cache);
    const int qsz = d.q_heads * kHD, kvsz = d.kv_heads * kHD;
    const float scale = d.scale;
    const uint32_t ep = epoch_base + (uint32_t)ph + 1;
    // Tiles of a segment go in pairs: warps 0..3 (set 0) take the first,
    // warps 4..7 (set 1) the second; a set's state is (m, l) per query head,
    // uniform over the set, and acc of head dim 32 q + lane per head.
    float m[2], l[2], acc[2];
    const int set = w >> 2, q = (w + 1) & 3;
    bool first_seg = true;
    for (int u0 = rg.start; u0 < rg.start + rg.count;) {
      const int b = au.stream_of(u0);
      const int cph = select_i(au.cph, b), valid = select_i(au.valid, b);
      const int r0 = u0 - select_i(au.pre, b);
      const int h = r0 / cph, j0 = r0 % cph;
      const int nseg = min(cph - j0, rg.start + rg.count - u0);  // this CTA's units of the (b, h) group
      const int pos = valid - 1, jpos = pos / kAttnChunk;
      const size_t head_off = ((size_t)b * d.kv_heads + h) * d.max_len;
      const uint64_t ss0 = kTrace ? globaltimer_ns() : 0;
      {  // segment start: queries, and this step's k / v when the segment holds its slot
        float cs[4], sn[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          cs[e] = sm.rope_c[b][(lane * 4 + e) % (kHD / 2)];
          sn[e] = sm.rope_s[b][(lane * 4 + e) % (kHD / 2)];
        }
        const bool has_pos = jpos >= j0 && jpos < j0 + nseg;
        const uint32_t* xw = qkv_w + (size_t)b * d.k;
        if (w < 2) {  // query heads 2h, 2h+1 of stream b
          const int col = (h * 2 + w) * kHD + lane * 4;
          const uint2 raw = ll_poll4(xw, col, x_epoch, s);
          const __half2* hp = reinterpret_cast<const __half2*>(&raw);
          float v[4] = {__low2float(hp[0]), __high2float(hp[0]), __low2float(hp[1]), __high2float(hp[1])};
          norm_rope_head(v, at.nw, d.eps, cs, sn);
          // row w of the queries operand [16 rows x 128 dims], K-major:
          // dims 4 lane .. 4 lane + 3 at (dim / 8) 128 + w 16 + (dim % 8) 2
          __half2 o[2] = {__floats2half2_rn(v[0], v[1]), __floats2half2_rn(v[2], v[3])};
          *reinterpret_cast<uint2*>(sm.xa + (lane >> 1) * 128 + w * 16 + (lane & 1) * 8) =
              *reinterpret_cast<uint2*>(o);
          fence_proxy_async_smem();
        } else if (has_pos && w < 4) {  // this step's k (warp 2) / v (warp 3) of head h
          const int off = qsz + (w == 2 ? 0 : kvsz) + h * kHD + lane * 4;
          const uint2 raw = ll_poll4(xw, off, x_epoch, s);
          const __half2* hp = reinterpret_cast<const __half2*>(&raw);
          float v[4] = {__low2float(hp[0]), __high2float(hp[0]), __low2float(hp[1]), __high2float(hp[1])};
          if (w == 2) norm_rope_head(v, at.nw + kHD, d.eps, cs, sn);
          float* dst = w == 2 ? at.kf : at.vf;
#pragma unroll
          for (int e = 0; e < 4; ++e) dst[lane * 4 + e] = v[e];
          __half2 o[2] = {__floats2half2_rn(v[0], v[1]), __floats2half2_rn(v[2], v[3])};
          __half* cache = w == 2 ? kc : vc;  // KV tile layout
          *reinterpret_cast<uint2*>(cache + head_off * kHD + (pos >> 3) * 1024 + (lane >> 1) * 64 + (pos & 7) * 8 +
                                    (lane & 1) * 4) = *reinterpret_cast<uint2*>(o);
        }
      }
      consumer_sync(kConsumerThreads);
      if (kTrace && tid == 0) {
        if (first_seg) trace_put(a, ph, 1, (int64_t)globaltimer_ns());
        seg_ns += globaltimer_ns() - ss0;
      }
      first_seg = false;
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
        acc[g] = 0.f;
      }
#pragma unroll 1
      for (int t = 0; t < nseg; t += 2) {
        if (t + set < nseg) {
          const uint32_t ri = rit + set;
          const int st = ri % kStages;
          if (kTrace && tid == 0) {
            const uint64_t w0 = globaltimer_ns();
            mbar_wait_bounded(&sm.full[st], (ri / kStages) & 1u, s, kErrFullTimeout);
            tile_wait += globaltimer_ns() - w0;
          } else {
            mbar_wait_bounded(&sm.full[st], (ri / kStages) & 1u, s, kErrFullTimeout);
          }
          const int p0 = (j0 + t + set) * kAttnChunk;
          attend_tile_tc(set, q, st, min(kAttnChunk, valid - p0), pos - p0 < kAttnChunk ? pos - p0 : -1, scale, m,
                         l, acc);
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm.cempty[st]);
        }
        rit += t + 1 < nseg ? 2 : 1;
      }
      // segment end: merge the 2 sets' states into this CTA's partial
      if ((w & 3) == 0 && lane == 0) {
        at.wm[set][0] = m[0];
        at.wm[set][1] = m[1];
        at.wl[set][0] = l[0];
        at.wl[set][1] = l[1];
      }
#pragma unroll
      for (int g = 0; g < 2; ++g) at.wacc[set][g][32 * q + lane] = acc[g];
      consumer_sync(kConsumerThreads);
      {
        const int gfirst = select_i(au.pre, b) + h * cph;
        const int first_owner = owner_of(gfirst, U, na);
        const int nsplit = owner_of(gfirst + cph - 1, U, na) - first_owner + 1;
        const int g = tid / kHD, t = tid % kHD;
        float M = -INFINITY;
#pragma unroll
        for (int i = 0; i < 2; ++i) M = fmaxf(M, at.wm[i][g]);
        float L = 0.f, A = 0.f;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const float mi = at.wm[i][g];
          if (mi != -INFINITY) {
            const float f = expf(mi - M);
            L += at.wl[i][g] * f;
            A += at.wacc[i][g][t] * f;
          }
        }
        const float lse = M + logf(L), o = A / L;
        if (nsplit == 1) {  // the whole group is this CTA's
          store_attn(d, b, (h * 2 + g) * kHD + t, o, ep);
        } else {  // this CTA's partial as 64-bit LL words; merged below
          uint64_t* const hp = &bs->part[b * d.kv_heads + h][cta - first_owner][0][0];
          if (t == 0) ll64_store(hp + g * (kHD + 1), lse, ep);
          ll64_store(hp + g * (kHD + 1) + 1 + t, o, ep);
        }
      }
      u0 += nseg;
    }
    if (kTrace && tid == 0) {
      trace_put(a, ph, 6, (int64_t)tile_wait);
      trace_put(a, ph, 3, (int64_t)globaltimer_ns());  // units done (merges follow)
      trace_put(a, ph, 4, (int64_t)seg_ns);             // ns in segment starts (query loads)
    }
    // Merges, after every partial of this CTA is stored: a CTA only waits for
    // partials that other CTAs store before they wait on anything, so the
    // merges of consecutive groups never queue behind one another.
    for (int u = rg.start; u < rg.start + rg.count;) {
      const int b = au.stream_of(u);
      const int cph = select_i(au.cph, b);
      const int r = u - select_i(au.pre, b);
      const int h = r / cph, j = r % cph;
      const int seg = min(cph - j, rg.start + rg.count - u);
      u += seg;
      const int gfirst = select_i(au.pre, b) + h * cph;
      const int first_owner = owner_of(gfirst, U, na);
      const int nsplit = owner_of(gfirst + cph - 1, U, na) - first_owner + 1;
      if (nsplit == 1) continue;
      merge_group(d, b, h, cta - first_owner, nsplit, ep);
    }
  }

  // Every CTA of a (stream, KV head) group merges a 1/nsplit slice of its 256
  // outputs over all splits in order (the same order whichever CTA merges):
  // each output by a group of tpo lanes (a power of two <= 16), lane `sub` of
  // the group polling splits sub, sub + tpo, ... kMergePer at a time, then a
  // fixed xor-shuffle tree combines the lanes' (max, sum, acc) triples.
  __device__ __forceinline__ void merge_group(const AicasPhase& d, int b, int h, int split, int nsplit, uint32_t ep) {
    uint64_t* const hp = &bs->part[b * d.kv_heads + h][0][0][0];
    constexpr int kSplitStride = 2 * (kHD + 1);
    const int q0 = split * 2 * kHD / nsplit, q1 = (split + 1) * 2 * kHD / nsplit;
    const int npairs = q1 - q0;
    int tpo = 16;
    while (tpo > 1 && tpo * npairs > kConsumerThreads) tpo >>= 1;
    const int nact = npairs * tpo;
    if ((tid & ~31) >= nact) return;  // warps without an active lane
    const bool actv = tid < nact;
    const int pl = tid / tpo, sub = tid % tpo;
    const int q = q0 + (actv ? pl : 0), gq = q / kHD, tq = q % kHD;
    const uint64_t* const base = hp + gq * (kHD + 1);
    float mx = -INFINITY, S = 0.f, ac = 0.f;
#pragma unroll 1
    for (int b0 = actv ? sub : nsplit; b0 < nsplit; b0 += tpo * kMergePer) {
      uint64_t lw[kMergePer], ow[kMergePer];
      uint32_t lpend = 0u;
#pragma unroll
      for (int i = 0; i < kMergePer; ++i)
        if (b0 + i * tpo < nsplit) lpend |= 1u << i;
      uint32_t opend = lpend;
      const uint32_t have = lpend;
      uint64_t t0 = 0;
#pragma unroll 1
      for (uint32_t it = 0;; ++it) {
        // predicates from the round's starting masks: one round trip per round
        const uint32_t lp = lpend, op = opend;
#pragma unroll
        for (int i = 0; i < kMergePer; ++i) {
          const uint64_t* sp = base + (b0 + i * tpo) * kSplitStride;
          if (lp & (1u << i)) lw[i] = ll64_load(sp);
          if (op & (1u << i)) ow[i] = ll64_load(sp + 1 + tq);
        }
        lpend = opend = 0u;
#pragma unroll
        for (int i = 0; i < kMergePer; ++i) {
          if ((lp & (1u << i)) && ll64_epoch(lw[i]) != ep) lpend |= 1u << i;
          if ((op & (1u << i)) && ll64_epoch(ow[i]) != ep) opend |= 1u << i;
        }
        if ((lpend | opend) == 0u) break;
        if (it == 0) t0 = globaltimer_ns();
        if ((it & 31u) == 31u) {
          if (ld_volatile_int(&s->abort)) break;
          if (globaltimer_ns() - t0 > kWaitLimitNs) {
            raise_error(s, kErrInputTimeout);
            break;
          }
        }
      }
#pragma unroll
      for (int i = 0; i < kMergePer; ++i) {
        if (have & (1u << i)) {
          const float li = ll64_value(lw[i]), oi = ll64_value(ow[i]);
          if (li > mx) {
            const float c = expf(mx - li);
            S = S * c + 1.f;
            ac = ac * c + oi;
            mx = li;
          } else {
            const float c = expf(li - mx);
            S += c;
            ac += c * oi;
          }
        }
      }
    }
    for (int o2 = 1; o2 < tpo; o2 <<= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, mx, o2);
      const float s2 = __shfl_xor_sync(0xffffffffu, S, o2);
      const float a2 = __shfl_xor_sync(0xffffffffu, ac, o2);
      const float mm = fmaxf(mx, m2);
      if (mm != -INFINITY) {
        const float f1 = mx == -INFINITY ? 0.f : expf(mx - mm);
        const float f2 = m2 == -INFINITY ? 0.f : expf(m2 - mm);
        S = S * f1 + s2 * f2;
        ac = ac * f1 + a2 * f2;
        mx = mm;
      }
    }
    if (actv && sub == 0) store_attn(d, b, (h * 2 + gq) * kHD + tq, ac / S, ep);
  }

  // Attention output value q of stream b: a counted vector (operand layout) or LL words.
  __device__ __forceinline__ void store_attn(const AicasPhase& d, int b, int q, float v, uint32_t ep) {
    if (d.flags & AICAS_F_CNT_OUT)
      *reinterpret_cast<__half*>(reinterpret_cast<uint8_t*>(d.out) + cnt_off(q / 8, b) + (q % 8) * 2) =
          __float2half_rn(v);
    else
      ll_store(reinterpret_cast<uint32_t*>(d.out) + (size_t)b * d.n + q, v, ep & 0xffffu);
  }

  __device__ __forceinline__ void run() {
    init_rope();
    for (ph = 0; ph < a.n_phases; ++ph) {
      const AicasPhase& d = a.phases[ph];
      consumer_sync(kConsumerThreads);  // every warp is done with the previous phase's shared buffers
      // every warp has written its part of the previous phase's counted vector
      if (ph > 0 && tid == 0 && (a.phases[ph - 1].flags & AICAS_F_CNT_OUT)) red_release_add_u32(&bs->done[ph - 1], 1u);
      if (kTrace && tid == 0) trace_put(a, ph, 0, (int64_t)globaltimer_ns());
      if (d.kind == AICAS_PH_ATTN) {
        if (tid < 2 * kHD / 8) {
          const __half* src = reinterpret_cast<const __half*>(tid < kHD / 8 ? d.norm_w : d.norm_w2);
          const int v = tid % (kHD / 8);
          *reinterpret_cast<uint4*>(&sm.at.nw[(tid / (kHD / 8)) * kHD + v * 8]) =
              __ldg(reinterpret_cast<const uint4*>(src) + v);
        }
        consumer_sync(kConsumerThreads);
        run_attention(d);
      } else {
        run_gemv(d);
      }
      if (kTrace && tid == 0) trace_put(a, ph, 2, (int64_t)globaltimer_ns());
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.cdone);
    consumer_sync(kConsumerThreads);
    if (tid == 0) {
      if (a.phases[a.n_phases - 1].flags & AICAS_F_CNT_OUT) red_release_add_u32(&bs->done[a.n_phases - 1], 1u);
      __threadfence();
      if (atomicAdd(&bs->exit_count, 1u) == (uint32_t)nct - 1) {
        bs->exit_count = 0;
        bs->epoch = epoch_base + (uint32_t)a.n_phases + 1;
        bs->launches = bs->launches + 1u;
        __threadfence();
      }
    }
  }
};

template <bool kTrace>
__global__ void __launch_bounds__(kThreads, 1) decode_batch_kernel(const __grid_constant__ BatchArgs a) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
  AicasScratch* s = reinterpret_cast<AicasScratch*>(a.scratch);
  // A scratch block that still holds a device error from an earlier launch
  // refuses the launch (nothing is read, written or advanced) until the
  // caller zeroes it.
  if (ld_volatile_int(&s->error) != 0) return;
  if (threadIdx.x < kMaxB) {
    const int b = threadIdx.x;
    StreamIn in{};
    if (b < a.nb) {
      const volatile AicasStepState* st = a.states + b;
      in.active = st->done_step == 0 ? 1 : 0;
      in.token = st->token;
      in.pos = st->cache_pos;
      in.rope[0] = st->rope[0];
      in.rope[1] = st->rope[1];
      in.rope[2] = st->rope[2];
      in.step = st->step;
    }
    sm.sin[b] = in;
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], 1);
      mbar_init(&sm.cempty[i], kConsumerWarps / 2);  // attention tiles: 4 warps each
    }
    for (int i = 0; i < kDSlots; ++i) {
      mbar_init(&sm.dfull[i], 1);
      mbar_init(&sm.dempty[i], 4);
    }
    mbar_init(&sm.xready, 1);
    mbar_init(&sm.cdone, kConsumerWarps);
    mbar_init(&sm.mdone, 1);
    mbar_init(&sm.xfull, 1);
    mbar_init(&sm.amma[0], 1);
    mbar_init(&sm.amma[1], 1);
    sm.ring_it = 0;
    sm.last_cta = 0;
    mbar_fence_init();
  }
  __syncthreads();
  int any = 0;
#pragma unroll
  for (int b = 0; b < kMaxB; ++b) any |= sm.sin[b].active;
  if (!any) return;  // every request has ended: the whole grid returns before any barrier or copy
  const int warp = threadIdx.x / 32;
  if (warp == kMmaWarp) tmem_alloc(&sm.tmem_base, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(&sm.tmem_base);
  if (warp == kMmaWarp) {
    run_mma<kTrace>(a, sm, s, tmem);
    return;
  }
  if (warp == kL2Warp) {
    run_l2_prefetcher(a, sm, s);
    return;
  }
  if (warp == 0) {
    run_producer<kTrace>(a, sm, s);
    return;
  }
  Consumer<kTrace> c{a, sm, s, a.scratch};
  c.tid = threadIdx.x - 32;
  c.w = warp - 1;
  c.lane = threadIdx.x & 31;
  c.nct = gridDim.x;
  c.cta = blockIdx.x;
  c.nb = a.nb;
  c.tmem = tmem;
  c.epoch_base = *reinterpret_cast<volatile uint32_t*>(&a.scratch->epoch);
  c.cnt_target = (*reinterpret_cast<volatile uint32_t*>(&a.scratch->launches) + 1u) * (uint32_t)gridDim.x;
  c.run();
}

// dst tile (c, g) = [256 column groups][8 rows][8] of rows 8g.. and columns
// 2048c.. of the row-major w[n, k]; one thread per 16-byte piece.
__global__ void tile_weight_kernel(const uint4* __restrict__ w, uint4* __restrict__ dst, int64_t n, int64_t k) {
  const int64_t total = n * k / 8;  // 16-byte pieces
  const int64_t kg = k / 8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    // destination order: tile (c, g), column group v, row r
    const int64_t r = i % 8, v = (i / 8) % 256, tile = i / 2048;
    const int64_t groups = n / 8, g = tile % groups, c = tile / groups;
    const int64_t row = 8 * g + r, colg = 256 * c + v;
    dst[i] = w[row * kg + colg];
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
static constexpr int kMaxDevices = 64;
// per-device setup, done once (idempotent; the flag is published after the
// values it guards)
static std::atomic<int> g_setup_done[kMaxDevices];
static std::atomic<int> g_ctas[kMaxDevices];

static int setup(int* dev_out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return AICAS_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return AICAS_ERR_CUDA;
  if (!g_setup_done[dev].load(std::memory_order_acquire)) {
    for (int v = 0; v < 2; ++v) {
      const void* fn = v ? reinterpret_cast<const void*>(decode_batch_kernel<true>)
                         : reinterpret_cast<const void*>(decode_batch_kernel<false>);
      cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(Smem));
      if (e != cudaSuccess) return record_cuda_error(e);
      int per_sm = 0;
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kThreads, sizeof(Smem));
      if (e != cudaSuccess) return record_cuda_error(e);
      if (per_sm < 1) return record_cuda_error(cudaErrorLaunchOutOfResources);
    }
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return AICAS_ERR_CUDA;
    g_ctas[dev].store(sms < AICAS_MAX_CTAS ? sms : AICAS_MAX_CTAS, std::memory_order_relaxed);
    g_setup_done[dev].store(1, std::memory_order_release);
  }
  *dev_out = dev;
  return AICAS_OK;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static int count_bits(int v) {
  int c = 0;
  for (; v; v &= v - 1) ++c;
  return c;
}

static int validate(const AicasPhase& d) {
  constexpr int kUnsupported = AICAS_F_X_ADD | AICAS_F_RESID_ADD | AICAS_F_STORE_X | AICAS_F_BARRIER;
  if (d.flags & kUnsupported) return AICAS_ERR_ARG;
  if (count_bits(d.flags & (AICAS_F_LL_IN | AICAS_F_CNT_IN | AICAS_F_X_EMBED)) > 1) return AICAS_ERR_ARG;
  if (count_bits(d.flags & (AICAS_F_LL_OUT | AICAS_F_CNT_OUT)) > 1) return AICAS_ERR_ARG;
  if (count_bits(d.flags & (AICAS_F_LL_RESID | AICAS_F_CNT_RESID | AICAS_F_RESID_EMBED)) > 1) return AICAS_ERR_ARG;
  if ((d.flags & (AICAS_F_LL_IN | AICAS_F_CNT_IN)) && d.x_src < 0) return AICAS_ERR_ARG;
  switch (d.kind) {
    case AICAS_PH_GEMV:
    case AICAS_PH_GATEUP:
    case AICAS_PH_LMHEAD:
      if (d.n < kRows || d.n % kRows != 0) return AICAS_ERR_SHAPE;
      if (d.k < kChunk || d.k % kChunk != 0 || d.k > AICAS_MAX_K) return AICAS_ERR_SHAPE;
      if (d.k > kChunk && !(d.flags & AICAS_F_KBLOCKED)) return AICAS_ERR_SHAPE;
      if (!d.w || !aligned16(d.w) || !d.x || !aligned16(d.x)) return AICAS_ERR_ALIGN;
      if ((d.flags & AICAS_F_NORM) && (d.k != kChunk || !d.norm_w || !aligned16(d.norm_w))) return AICAS_ERR_ARG;
      if ((d.flags & AICAS_F_LL_IN) && ((d.flags & AICAS_F_X_EMBED) || d.x_src < 0)) return AICAS_ERR_ARG;
      if ((d.flags & (AICAS_F_X_EMBED | AICAS_F_RESID_EMBED)) && d.embed_rows < 1) return AICAS_ERR_ARG;
      if (d.kind == AICAS_PH_GATEUP && (d.k != kChunk || (d.flags & (AICAS_F_RESID | AICAS_F_BIAS))))
        return AICAS_ERR_ARG;
      if ((d.flags & AICAS_F_RESID) && (!d.resid || !aligned16(d.resid))) return AICAS_ERR_ALIGN;
      if ((d.flags & AICAS_F_BIAS) && !d.bias) return AICAS_ERR_ARG;
      if (d.kind != AICAS_PH_LMHEAD) {
        if (!(d.flags & (AICAS_F_LL_OUT | AICAS_F_CNT_OUT)) || !d.out || !aligned16(d.out)) return AICAS_ERR_ARG;
      }
      return AICAS_OK;
    case AICAS_PH_ATTN:
      if (d.kv_heads < 1 || d.kv_heads > AICAS_MAX_KV_HEADS || d.q_heads != 2 * d.kv_heads) return AICAS_ERR_SHAPE;
      if (d.max_len < 8 || d.max_len % 8 != 0) return AICAS_ERR_SHAPE;  // whole 8-slot groups
      if (d.k != (d.q_heads + 2 * d.kv_heads) * kHD || d.n != d.q_heads * kHD) return AICAS_ERR_SHAPE;
      if ((d.flags & AICAS_F_Q_READY) || !(d.flags & AICAS_F_LL_IN) ||
          !(d.flags & (AICAS_F_LL_OUT | AICAS_F_CNT_OUT)) || d.x_src < 0)
        return AICAS_ERR_ARG;
      if (!d.k_cache || !d.v_cache || !aligned16(d.k_cache) || !aligned16(d.v_cache)) return AICAS_ERR_ALIGN;
      if (!d.x || !d.out || !aligned16(d.x) || !aligned16(d.out)) return AICAS_ERR_ALIGN;
      if (!d.norm_w || !d.norm_w2 || !aligned16(d.norm_w) || !aligned16(d.norm_w2)) return AICAS_ERR_ALIGN;
      return AICAS_OK;
    default:
      return AICAS_ERR_ARG;
  }
}

}  // namespace bat
}  // namespace aicas

using namespace aicas;

extern "C" {

AICAS_API size_t aicas_batch_scratch_bytes(void) { return sizeof(AicasBatchScratch); }

AICAS_API int aicas_validate_batch_phases(const AicasPhase* phases, int n) {
  if (!phases || n < 1 || n > AICAS_MAX_PHASES) return AICAS_ERR_ARG;
  for (int i = 0; i < n; ++i) {
    const int rc = bat::validate(phases[i]);
    if (rc) return rc;
    const int f = phases[i].flags;
    if ((f & (AICAS_F_LL_IN | AICAS_F_CNT_IN)) && phases[i].x_src >= i) return AICAS_ERR_ARG;
    // an input's kind must match its source's output kind
    if (f & AICAS_F_CNT_IN && !(phases[phases[i].x_src].flags & AICAS_F_CNT_OUT)) return AICAS_ERR_ARG;
    if (f & AICAS_F_LL_IN && !(phases[phases[i].x_src].flags & AICAS_F_LL_OUT)) return AICAS_ERR_ARG;
  }
  return AICAS_OK;
}

static int launch_batch(const AicasPhase* device_phases, int n_phases, AicasStepState* states, int nb,
                        void* scratch, int64_t* trace, cudaStream_t stream) {
  if (!device_phases || n_phases < 1 || n_phases > AICAS_MAX_PHASES || !states || !scratch) return AICAS_ERR_ARG;
  if (nb < 1 || nb > AICAS_MAX_BATCH) return AICAS_ERR_ARG;
  int dev = 0;
  const int rc = bat::setup(&dev);
  if (rc) return rc;
  bat::BatchArgs a;
  memset(&a, 0, sizeof(a));
  a.phases = device_phases;
  a.n_phases = n_phases;
  a.nb = nb;
  a.states = states;
  a.scratch = reinterpret_cast<AicasBatchScratch*>(scratch);
  a.trace = trace;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(bat::g_ctas[dev].load(std::memory_order_relaxed));
  cfg.blockDim = dim3(bat::kThreads);
  cfg.dynamicSmemBytes = sizeof(bat::Smem);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = trace ? cudaLaunchKernelEx(&cfg, bat::decode_batch_kernel<true>, a)
                              : cudaLaunchKernelEx(&cfg, bat::decode_batch_kernel<false>, a);
  return e == cudaSuccess ? AICAS_OK : record_cuda_error(e);
}

AICAS_API int aicas_decode_batch_f16(const AicasPhase* device_phases, int n_phases, AicasStepState* states, int nb,
                                     void* scratch, cudaStream_t stream) {
  return launch_batch(device_phases, n_phases, states, nb, scratch, nullptr, stream);
}

AICAS_API int aicas_decode_batch_trace_f16(const AicasPhase* device_phases, int n_phases, AicasStepState* states,
                                           int nb, void* scratch, int64_t* trace, cudaStream_t stream) {
  if (!trace) return AICAS_ERR_ARG;
  return launch_batch(device_phases, n_phases, states, nb, scratch, trace, stream);
}

AICAS_API int aicas_tile_weight_f16(const void* w, void* dst, int64_t n, int64_t k, cudaStream_t stream) {
  if (!w || !dst) return AICAS_ERR_ARG;
  if (n < 8 || n % 8 != 0 || k < 2048 || k % 2048 != 0 || n > (int64_t)1 << 30) return AICAS_ERR_SHAPE;
  if (!bat::aligned16(w) || !bat::aligned16(dst)) return AICAS_ERR_ALIGN;
  const int64_t pieces = n * k / 8;
  int64_t blocks = (pieces + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  bat::tile_weight_kernel<<<(unsigned)blocks, 256, 0, stream>>>(reinterpret_cast<const uint4*>(w),
                                                                 reinterpret_cast<uint4*>(dst), n, k);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? AICAS_OK : record_cuda_error(e);
}

}  // extern "C"
