// Persistent decode-program kernel for B200 (sm_100a).
//
// One launch runs a list of phases (aicas_phase_program.h) with one CTA per SM:
//   warp 0      producer: streams every tile this CTA will consume, phase after
//               phase, from HBM into a small shared-memory ring (kStages) with
//               bulk async copies (cp.async.bulk + mbarrier complete_tx, L2
//               evict_first).  It never waits for activations, so HBM keeps
//               streaming the next phases' weights while the consumers wait.
//   warps 1..8  consumers: per phase, wait for the phase's input vector (LL
//               flag-in-data words written by the previous phase; the warps
//               poll disjoint slices and meet at one barrier), apply the
//               RMSNorm prologue with HF's fp16 rounding points, then reduce
//               each tile row against it with exact fp16 products and fp32
//               accumulation (one row per warp, four accumulation chains).
//   (warp 9     optional L2 prefetch, AICAS_L2_WARP=1: walks the same tile
//               schedule up to kL2Ahead tiles ahead of the producer and
//               prefetches them into L2; off by default, see below.)
//   last warp   TMEM mover: copies every landed GEMV tile from its ring stage
//               into an 8-slot ring in tensor memory (tcgen05.cp) and frees
//               the stage; consumers read their tile row from TMEM
//               (tcgen05.ld), so up to kStages + 8 tiles wait ahead of them.
//
// GEMV tile: 8 weight rows x 2048 columns (32 KB), fetched with ONE bulk copy
// (rows are contiguous when k <= 2048; the engine stores down_proj K-blocked,
// [k/2048][n][2048], so its tiles are contiguous too: bulk copies of 8 KB and
// more are what reach full HBM bandwidth on B200, 2 KB copies top out near
// 4 TB/s).  Consumer warp w owns row w of every tile; lane l the columns
// j*256 + 8l (j = 0..7) of each 2048-column chunk, so a lane keeps its slice
// of the input vector in registers for the whole phase, every weight byte is
// read from shared memory exactly once (conflict-free 512-byte warp accesses)
// and a row needs one warp reduction.
//
// Attention tile: K and V rows of 64 cache positions of one KV head (32 KB).
// A CTA's tiles go in pairs: consumer warps 0..3 take one, 4..7 the next,
// each warp 16 positions (a lane scores two positions over a quarter of the
// head dims, so it runs four independent dot chains).  Work units (KV head, 64-position chunk) are
// split into contiguous ranges over the CTAs; each CTA's segment of a head
// yields one (log-sum-exp, normalised acc) partial, stored as 64-bit LL words;
// every CTA of the head then merges a slice of the head's outputs over all
// partials in a fixed split order, so the result does not depend on timing.
//
// Phases are ordered only through their LL inputs; the op-level programs
// that need it use a grid barrier (split arrive / wait on a monotonic 64-bit
// counter) instead.  Every wait is bounded (see aicas_device.cuh).
//
// Reference behaviour this replaces (file:line in the reference checkout):
//   fused RMSNorm+QKV      cuda_extensions/decode_gemv_kernel_fused.cuh:99-185
//   o_proj GEMV            cuda_extensions/decode_gemv_kernel_matvec.cuh:276-343
//   post-attn MLP          cuda_extensions/decode_gemv_kernel_fused.cuh:850-1076
//   split-KV attention     cuda_extensions/decode_attention_v4_kernel.cu:647-900
//   q/k norm+rope+KV write cuda_extensions/decode_small_ops_kernel.cu:115-186
//   lm_head GEMV           cuda_extensions/decode_gemv_kernel_matvec.cuh:209-274
//   argmax                 evaluation_wrapper.py:952 (torch.argmax, first max wins)
#include <atomic>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#include "aicas_device.cuh"
#include "aicas_phase_program.h"

namespace aicas {

constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = kConsumerWarps * 32;
// AICAS_L2_WARP: 1 an extra warp runs an L2 prefetch cursor ahead of the
// ring (one bulk prefetch per tile, lines marked evict_last; the ring loads
// mark weights and KV tiles evict_first); 2 the same with per-line
// prefetches; 0 (default) no prefetch warp.  Once the norm weights stopped
// blocking each phase's input poll, the run-ahead cost more than it gave:
// same-box A/B on the 28-layer step, 996 -> 989 and 990 -> 979 us per token
// without it.
#ifndef AICAS_L2_WARP
#define AICAS_L2_WARP 0
#endif
// AICAS_KV_STAGES: attention K/V tiles land in their own shared-memory
// stages (this many, >= 2: the consumers take tiles in pairs), filled by their
// own producer warp, so a KV tile that waits for its phase's queries never
// holds a stage of the weight ring; 0 sends them through the weight ring in
// schedule order (the weight stream then stalls behind every attention
// phase).
#ifndef AICAS_KV_STAGES
#define AICAS_KV_STAGES 2
#endif
constexpr int kKvStages = AICAS_KV_STAGES;
constexpr bool kKvSplit = kKvStages > 0;
constexpr int kKvRing = kKvSplit ? kKvStages : 1;  // divisor of the K/V stage index (1 when unused)
static_assert(kKvStages == 0 || kKvStages >= 2, "attention tiles are consumed in pairs");
// Warp roles: 0 weight producer, 1..8 consumers, then the L2 prefetch warp
// (if enabled), the TMEM mover, and the KV producer (with AICAS_KV_STAGES).
constexpr int kL2Warp = 1 + kConsumerWarps;
constexpr int kMoverWarp = 1 + kConsumerWarps + (AICAS_L2_WARP ? 1 : 0);
constexpr int kKvWarp = kMoverWarp + 1;
constexpr int kThreads = 32 * (kMoverWarp + 1 + (kKvSplit ? 1 : 0));
// Tensor memory: an 8-slot ring of GEMV tiles (64 columns x 128 lanes each).
constexpr int kTmemSlots = 8;
constexpr int kTmemCols = 512;
constexpr int kTmemTileCols = 64;
constexpr int kRowsPerWarp = 1;
constexpr int kRows = kConsumerWarps * kRowsPerWarp;  // weight rows per GEMV tile
constexpr int kChunk = 2048;           // columns per GEMV tile
constexpr int kRowBytes = kChunk * 2;
constexpr int kStageBytes = kRows * kRowBytes;  // 32 KB: one bulk copy per tile
// Ring stages in shared memory.  With the TMEM slot ring behind them a stage
// only holds a tile until the mover has copied it out; measured on B200
// (28 layers, 1024-slot prefix): 6 stages 1219 us/token, 5: 1238, 4: 1140,
// 3: 1114-1120, 2: 1095-1098 (no TMEM ring, 6 stages: 1156-1174).
#ifndef AICAS_STAGES
#define AICAS_STAGES 2
#endif
constexpr int kStages = AICAS_STAGES;
constexpr int kAttnChunk = 64;  // cache positions per attention tile
constexpr int kHD = AICAS_HEAD_DIM;
constexpr int kVec = kChunk / 256;                // uint4 per lane per chunk
#ifndef AICAS_EPI_BATCH
#define AICAS_EPI_BATCH 16
#endif
constexpr int kEpiBatch = AICAS_EPI_BATCH;  // row groups whose epilogues are done together (one lane each, <= 32)
static_assert(kEpiBatch <= 32, "one lane per row group");

static_assert(kAttnChunk * kHD * 2 * 2 == kStageBytes, "attention tile must fill one stage");
static_assert(AICAS_MAX_K % kChunk == 0, "max K must be whole chunks");

struct AttnSmem {
  float kf[kHD], vf[kHD];  // this step's k (normed+rotated) / v of the current KV head
  float wm[kConsumerWarps][2];
  float wl[kConsumerWarps][2];
  float wacc[kConsumerWarps][2][kHD];
  float rope_c[kHD / 2], rope_s[kHD / 2];  // this launch's MRoPE cos/sin (fp16-rounded)
  __align__(16) __half qh[2][kHD];   // the segment's queries as fp16 (their values are fp16)
  float2 sc[kConsumerWarps][16];     // per warp: probabilities (both heads) of its 16 positions
};

struct __align__(128) Smem {
  uint8_t ring[kStages][kStageBytes];
  uint8_t kv[kKvSplit ? kKvStages : 1][kKvSplit ? kStageBytes : 16];  // attention K/V stages
  __half nw[AICAS_MAX_K];  // norm weights of the running phase (prefetched before its barrier)
  AttnSmem at;
  __half xs[kChunk];            // C == 1 phases: the input vector, shared by the 8 warps
  // batched epilogue: lane partial sums, [warp][group slot * 2 + part][lane]
  // (rows padded to 33 floats: a lane summing a row reads a different bank
  // from every other lane)
  float epi[kConsumerWarps][2 * kEpiBatch][33];
  float ssq[kConsumerWarps];    // per-warp sums of squares for the RMSNorm prologue
  float best_v[kConsumerWarps];
  int best_i[kConsumerWarps];
  uint64_t full[kStages];    // stage landed (bulk copy complete_tx)
  uint64_t empty[kStages];   // stage free again (arrived by the mover)
  uint64_t cempty[kStages];  // consumers done with a stage they read directly (attention, partial chunks)
  uint64_t tfull[kTmemSlots];   // TMEM slot filled (tcgen05.commit of the mover)
  uint64_t tempty[kTmemSlots];  // TMEM slot read by all 8 consumer warps
  uint64_t kvfull[kKvSplit ? kKvStages : 1];   // K/V stage landed
  uint64_t kvempty[kKvSplit ? kKvStages : 1];  // K/V stage read by its 4 consumer warps (2 arrivals each)
  uint64_t cdone;               // all consumer warps finished the program (TMEM may be freed)
  uint32_t ring_it;  // tiles the producer has issued (read by the L2 prefetch warp)
  uint32_t tmem_base;  // TMEM address of the slot ring (written by tcgen05.alloc)
};

struct ProgramArgs {
  const AicasPhase* phases;  // device array, or null: use `inl`
  int n_phases;
  int pad;
  AicasStepState* state;  // may be null (op-level calls)
  AicasScratch* scratch;
  int64_t* trace;  // optional [grid][n_phases][kTraceFields] (see aicas_decode_program_trace_f16)
  AicasPhase inl[4];
};

// start, inputs ready, end, consumer tile-wait ns, producer slot-wait ns,
// tiles, compute done, results issued
constexpr int kTraceFields = 8;

struct StepIn {
  int64_t token;
  int64_t pos;
  int64_t rope[3];
  int64_t step;
};

struct Range {
  int start, count;
};

// Contiguous split of `total` items over `nct` CTAs, CTA order rotated by `rot`.
__device__ __forceinline__ Range split_range(int total, int nct, int cta, int rot) {
  int c = (cta - rot) % nct;
  if (c < 0) c += nct;
  const int base = total / nct, extra = total % nct;
  return {c * base + min(c, extra), base + (c < extra ? 1 : 0)};
}

// Inverse of split_range (rot 0): the CTA owning item u.
__device__ __forceinline__ int owner_of(int u, int total, int nct) {
  const int base = total / nct, extra = total % nct;
  const int big = extra * (base + 1);
  if (u < big) return u / (base + 1);
  return extra + (u - big) / base;
}

// CTAs taking part in an attention phase of U units (KV head x 64-slot
// chunk): each gets at least kAttnMinUnits units (fewer partials to merge,
// but more serial unit work per CTA).  CTAs [0, attn_ctas) take part.
// Measured on B200 (1024-slot prefix): 1 unit 1258 us/token, 2: 1281,
// 3: 1500, 4: 1641, so the default keeps one unit per CTA.
#ifndef AICAS_ATTN_MIN_UNITS
#define AICAS_ATTN_MIN_UNITS 1
#endif
constexpr int kAttnMinUnits = AICAS_ATTN_MIN_UNITS;
__device__ __forceinline__ int attn_ctas(int U, int nct) {
  return max(1, min(nct, (U + kAttnMinUnits - 1) / kAttnMinUnits));
}
__device__ __forceinline__ Range attn_range(int U, int nct, int cta) {
  const int na = attn_ctas(U, nct);
  return cta < na ? split_range(U, na, cta, 0) : Range{0, 0};
}

// Attention covers cache slots [0, valid); 0 when the position is outside
// the cache (the phase is then skipped by producer and consumers alike and
// kErrBadInput is raised).
__device__ __forceinline__ int phase_valid_len(const AicasPhase& d, const StepIn& in) {
  const int64_t pos = d.pos_ptr ? *reinterpret_cast<const int64_t*>(d.pos_ptr) : in.pos;
  if (pos < 0 || pos >= d.max_len) return 0;
  return (int)pos + 1;
}

__device__ __forceinline__ int n_chunks(const AicasPhase& d) { return (d.k + kChunk - 1) / kChunk; }

__device__ __forceinline__ int tiles_per_group(const AicasPhase& d) {
  return d.kind == AICAS_PH_GATEUP ? 2 * n_chunks(d) : n_chunks(d);
}

// Phases with k > 2048 and few row groups per CTA stream their tiles
// chunk-major (all groups' chunk 0, then chunk 1, ...), so only one chunk of
// the input vector is needed in fp32 registers at a time.  Producer and
// consumers both call this to agree on the tile order.
constexpr int kMaxCmajorGroups = 2;
// split-KV merge: splits whose partial words one merging lane polls per round
constexpr int kMergePer = 4;
__host__ __device__ __forceinline__ bool chunk_major(int C, int kind, int groups) {
  return C > 1 && kind != AICAS_PH_GATEUP && groups <= kMaxCmajorGroups;
}

// A GEMV-type phase the lean kernel runs: whole 2048-column chunks (TMEM
// path), and either one chunk (row-major tile order) or three in chunk-major
// order on every CTA of an `nct`-CTA grid.
__host__ __device__ __forceinline__ bool lean_phase(const AicasPhase& d, int nct) {
  if (d.kind == AICAS_PH_ATTN) return true;
  if (d.k % kChunk != 0) return false;
  const int C = d.k / kChunk;
  if (C == 1) return true;
  if (d.kind == AICAS_PH_LMHEAD) return false;
  const int groups = (d.n + kRows - 1) / kRows;
  return C == 3 && chunk_major(C, d.kind, (groups + nct - 1) / nct);
}

// ---------------------------------------------------------------------------
// Producer (warp 0, lane 0)
// ---------------------------------------------------------------------------
struct Ring {
  uint32_t it = 0;  // tiles issued/consumed so far in this launch
  __device__ __forceinline__ int stage() const { return it % kStages; }
  __device__ __forceinline__ uint32_t round() const { return it / kStages; }
};

// One tile of the CTA's schedule: `pieces` copies of `bytes` each, from src
// + i * src_stride to ring stage + i * dst_stride.
// GEMV-type phases whose reduction length is a multiple of 2048 stream their
// tiles through the TMEM slot ring (every tile row is a full 4096-byte chunk
// row); other tiles are read by the consumers straight from the ring stage.
__device__ __forceinline__ bool tmem_phase(int kind, int k) {
  return kind != AICAS_PH_ATTN && k % kChunk == 0;
}

struct TileDesc {
  const uint8_t* src;
  int64_t src_stride;
  uint32_t dst_stride;
  uint32_t bytes;
  int pieces;
  bool tmem;  // GEMV tile that goes through the TMEM slot ring (else consumers read the stage)
};

// Walks this CTA's tiles of a program in the exact order the consumers
// take them.  The producer, the TMEM mover, the L2 prefetch warp and the KV
// producer each run one cursor; `sel` picks the tiles it yields.
enum { kAllTiles = 0, kWeightTiles = 1, kKvTiles = 2 };
constexpr int kRingSel = kKvSplit ? kWeightTiles : kAllTiles;
struct TileCursor {
  const AicasPhase* P;
  int n_phases;
  int nct, cta;
  int sel;
  int ph = -1;
  int ti = 0, n = 0;
  // cached per-phase schedule
  int kind, flags, C, T, rows_total;
  Range rg;
  bool cmajor, tm;
  int valid, cph;

  __device__ __forceinline__ void enter(int phase, const StepIn& in) {
    ph = phase;
    ti = 0;
    n = 0;
    if (ph >= n_phases) return;
    const AicasPhase& d = P[ph];
    kind = d.kind;
    flags = d.flags;
    if (kind == AICAS_PH_ATTN) {
      valid = phase_valid_len(d, in);
      cph = (valid + kAttnChunk - 1) / kAttnChunk;
      rg = attn_range(d.kv_heads * cph, nct, cta);  // empty when valid == 0
      n = rg.count;
    } else if (kind == AICAS_PH_GEMV || kind == AICAS_PH_GATEUP || kind == AICAS_PH_LMHEAD) {
      C = n_chunks(d);
      T = tiles_per_group(d);
      rg = split_range((d.n + kRows - 1) / kRows, nct, cta, d.rot);
      cmajor = chunk_major(C, kind, rg.count);
      tm = tmem_phase(kind, d.k);
      rows_total = kind == AICAS_PH_GATEUP ? 2 * d.n : d.n;
      n = rg.count * T;
    }
    if (sel != kAllTiles && (sel == kKvTiles) != (kind == AICAS_PH_ATTN)) n = 0;
  }

  // Next tile; false when the program is exhausted.
  __device__ __forceinline__ bool next(const StepIn& in, TileDesc& td) {
    while (ti >= n) {
      if (ph >= n_phases) return false;
      enter(ph + 1, in);
      if (ph >= n_phases) return false;
    }
    const AicasPhase& d = P[ph];
    if (kind == AICAS_PH_ATTN) {
      const int u = rg.start + ti;
      const int h = u / cph, p0 = (u % cph) * kAttnChunk;
      const int rows = min(kAttnChunk, valid - p0);
      const size_t off = ((size_t)h * d.max_len + p0) * kHD * 2;
      td.src = reinterpret_cast<const uint8_t*>(d.k_cache) + off;
      td.src_stride = reinterpret_cast<const uint8_t*>(d.v_cache) - reinterpret_cast<const uint8_t*>(d.k_cache);
      td.dst_stride = kStageBytes / 2;
      td.bytes = rows * kHD * 2;
      td.pieces = 2;
      td.tmem = false;
    } else {
      int g, t;
      if (cmajor) {
        t = ti / rg.count;
        g = rg.start + ti % rg.count;
      } else {
        g = rg.start + ti / T;
        t = ti % T;
      }
      const int nrows = min(kRows, d.n - g * kRows);
      const int c = t % C;
      const int row0 = g * kRows + (t >= C ? d.n : 0);
      const int col0 = c * kChunk;
      const uint32_t bytes = min(kChunk, d.k - col0) * 2;
      const uint8_t* W = reinterpret_cast<const uint8_t*>(d.w);
      td.tmem = tm;
      if (C == 1) {  // whole rows: one contiguous block, rows packed at stride k
        td.src = W + (size_t)row0 * d.k * 2;
        td.bytes = nrows * bytes;
        td.pieces = 1;
      } else if (flags & AICAS_F_KBLOCKED) {  // block c of rows row0.. is contiguous
        td.src = W + ((size_t)c * rows_total + row0) * kChunk * 2;
        td.bytes = nrows * bytes;
        td.pieces = 1;
      } else {  // row-major with k > 2048: one copy per row piece
        td.src = W + ((size_t)row0 * d.k + col0) * 2;
        td.src_stride = (int64_t)d.k * 2;
        td.dst_stride = kRowBytes;
        td.bytes = bytes;
        td.pieces = nrows;
      }
    }
    ++ti;
    return true;
  }
};

// L2 prefetch warp: distance in tiles ahead of the producer's ring cursor.
// Measured on B200 (1024-slot prefix, 28 layers): no prefetch 1173-1189
// us/token; distance 6 1161-1164, 8 1154-1159, 12 1188-1205, 24 1526 (the
// run-ahead then evicts itself from L2).  A prefetch cursor walked by the
// producer warp itself was slower at every distance (its descriptor reads
// delay the ring loads).
#ifndef AICAS_L2_AHEAD
#define AICAS_L2_AHEAD 8
#endif
constexpr int kL2Ahead = AICAS_L2_AHEAD;

// L2 prefetch warp (AICAS_L2_WARP): walks the CTA's tile schedule at most
// kL2Ahead tiles ahead of the producer's ring cursor and prefetches each tile
// into L2, so HBM keeps streaming while the ring is full and the consumers
// wait for a phase's inputs.  Only a hint: on abort or after a bounded wait it
// stops without raising an error.
__device__ __forceinline__ void run_l2_prefetcher(const ProgramArgs& a, Smem& sm, const StepIn& in) {
  const int lane = threadIdx.x & 31;
  const AicasPhase* P = a.phases ? a.phases : a.inl;
  TileCursor pf{P, a.n_phases, (int)gridDim.x, (int)blockIdx.x, kRingSel};
  TileDesc td;
  const uint64_t pol_last = l2_evict_last_policy();
  for (uint32_t k = 0; pf.next(in, td); ++k) {
    uint64_t t0 = 0;
    uint32_t ri = 0;
    for (uint32_t it = 0;; ++it) {
      ri = *reinterpret_cast<volatile uint32_t*>(&sm.ring_it);
      if (k < ri + (uint32_t)kL2Ahead) break;
      if (it == 0) t0 = globaltimer_ns();
      if ((it & 15u) == 15u && (ld_volatile_int(&a.scratch->abort) || globaltimer_ns() - t0 > kWaitLimitNs)) return;
      __nanosleep(128);
    }
    if (k < ri) continue;  // the ring has already requested it
    if (AICAS_L2_WARP == 1) {
      if (lane == 0)
        for (int i = 0; i < td.pieces; ++i) {
          bulk_prefetch_l2_hint(td.src + i * td.src_stride, td.bytes, pol_last);
        }
    } else {
      for (int i = 0; i < td.pieces; ++i)
        for (uint32_t off = lane * 128u; off < td.bytes; off += 32u * 128u) prefetch_l2_line(td.src + i * td.src_stride + off);
    }
  }
}

// TMEM mover (last warp; lane 0 walks the tile schedule in order): every
// GEMV tile that has landed in a ring stage is copied into the next TMEM slot
// with 8 tcgen05.cp (128 lanes x 256 bits each) -- slot lanes 32q..32q+31
// then hold tile row q in columns 0..31 and row 4 + q in columns 32..63, each
// lane 64 fp16 values of the row -- and one tcgen05.commit each marks the
// slot full and the stage free once the copies are done.  For tiles the
// consumers read in place it passes their release on to the producer (the
// producer waits on one arrival per stage).  So the ring stages turn over as
// fast as tiles can be parked in TMEM, and up to kStages + 8 tiles are in flight
// ahead of the consumers.  The whole warp allocates the TMEM at launch and
// frees it after every consumer warp has signalled that it is done.
__device__ __forceinline__ void run_mover(const ProgramArgs& a, Smem& sm, const StepIn& in, uint32_t tmem) {
  const int lane = threadIdx.x & 31;
  AicasScratch* s = a.scratch;
  if (lane == 0) {
    const AicasPhase* P = a.phases ? a.phases : a.inl;
    TileCursor cur{P, a.n_phases, (int)gridDim.x, (int)blockIdx.x, kRingSel};
    TileDesc td;
    uint32_t it = 0, g = 0;
    // cempty[st] completes once per in-place use of stage st (not per use):
    // its expected parity is tracked per stage
    uint32_t cpar = 0;
    while (cur.next(in, td)) {
      const int st = it % kStages;
      const uint32_t par = (it / kStages) & 1u;
      if (td.tmem) {
        const uint32_t t = g % kTmemSlots;
        if (!mbar_wait_bounded(&sm.full[st], par, s, kErrFullTimeout)) break;
        if (g >= kTmemSlots && !mbar_wait_bounded(&sm.tempty[t], ((g / kTmemSlots) - 1) & 1u, s, kErrTmemTimeout))
          break;
        tc_fence_after();
        const uint32_t stage = smem_addr(sm.ring[st]);
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int c = 0; c < 4; ++c)
            tcgen05_cp_128x256b(tmem + t * kTmemTileCols + h * 32 + c * 8,
                                smem_desc_kmajor(stage + h * 16384 + c * 256, 128, 1024));
        tcgen05_commit(&sm.tfull[t]);
        tcgen05_commit(&sm.empty[st]);
        ++g;
      } else {
        if (!mbar_wait_bounded(&sm.cempty[st], (cpar >> st) & 1u, s, kErrEmptyTimeout)) break;
        cpar ^= 1u << st;
        mbar_arrive(&sm.empty[st]);
      }
      ++it;
    }
    // TMEM is freed only after the consumers are done with it.  This wait
    // ignores the abort word (consumers finish promptly after an abort: every
    // wait of theirs is bounded) and is bounded by twice the wait limit.
    const uint64_t t0 = globaltimer_ns();
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

// Run by all 32 lanes of warp 0: lane 0 owns the ring (waits, expect_tx,
// copies); every lane takes part in the L2 run-ahead prefetches.
template <bool kTrace>
__device__ __forceinline__ void run_producer(const ProgramArgs& a, Smem& sm, const StepIn& in) {
  const int lane = threadIdx.x & 31;
  AicasScratch* s = a.scratch;
  const uint64_t pol = l2_evict_first_policy();
  Ring r;
  const AicasPhase* P = a.phases ? a.phases : a.inl;
  TileCursor ld{P, a.n_phases, (int)gridDim.x, (int)blockIdx.x, kRingSel};
  uint64_t slot_wait = 0;  // trace only
  int traced_ph = 0;
  TileDesc td;
  while (ld.next(in, td)) {
    if (kTrace && lane == 0 && ld.ph != traced_ph) {
      a.trace[((size_t)blockIdx.x * a.n_phases + traced_ph) * kTraceFields + 4] = (int64_t)slot_wait;
      slot_wait = 0;
    }
    traced_ph = ld.ph;
    const int st = r.stage();
    int good = 1;
    if (lane == 0) {
      if (r.round() > 0) {
        const uint32_t prev = (r.round() - 1) & 1u;
        if (kTrace) {
          const uint64_t t0 = globaltimer_ns();
          good = mbar_wait_bounded(&sm.empty[st], prev, s, kErrEmptyTimeout);
          slot_wait += globaltimer_ns() - t0;
        } else {
          good = mbar_wait_bounded(&sm.empty[st], prev, s, kErrEmptyTimeout);
        }
        // The stage's previous copy has landed before the stage is armed
        // again.  In-place stages (attention, partial chunks) are released by
        // the consumers' arrivals alone, and after an abort a consumer may
        // arrive without having waited for the copy; this wait (which ignores
        // the abort word and normally succeeds at once) keeps a second copy
        // from being issued into a stage that is still being written, so
        // every phase of full[st] completes once per copy and the drain
        // below sees each of them.
        if (good) good = mbar_wait_copy(&sm.full[st], prev, s, kErrDrainTimeout);
      }
      if (good) {
        mbar_arrive_expect_tx(&sm.full[st], td.pieces * td.bytes);
        for (int i = 0; i < td.pieces; ++i) {
          uint8_t* dst = sm.ring[st] + i * td.dst_stride;
          bulk_g2s(dst, td.src + i * td.src_stride, td.bytes, &sm.full[st], pol);  // weights and KV: evict_first
        }
      }
    }
    if (!__shfl_sync(0xffffffffu, good, 0)) break;
    ++r.it;
    if (AICAS_L2_WARP && lane == 0) *reinterpret_cast<volatile uint32_t*>(&sm.ring_it) = r.it;
  }
  if (kTrace && lane == 0)
    a.trace[((size_t)blockIdx.x * a.n_phases + traced_ph) * kTraceFields + 4] = (int64_t)slot_wait;
  if (lane != 0) return;
  // Drain: every issued copy must land before this CTA may exit.  In the
  // normal path the consumers already waited for all of them.
  const uint32_t issued = r.it;
  const uint32_t first = issued > (uint32_t)kStages ? issued - kStages : 0;
  for (uint32_t it = first; it < issued; ++it) {
    const int st = it % kStages;
    if (!mbar_wait_bounded(&sm.full[st], (it / kStages) & 1u, s, kErrDrainTimeout)) {
      // abort raised by someone else: still give the copy its own bounded time
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&sm.full[st], (it / kStages) & 1u)) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) break;
      }
    }
  }
}

// KV producer (AICAS_KV_STAGES > 0; lane 0 of its own warp): walks the
// CTA's attention tiles only and lands each one (K half, V half: two bulk
// copies) in the next K/V stage.  The weight producer never waits for a
// KV stage, so HBM keeps streaming weights into the ring and TMEM while the
// consumers wait for an attention phase's queries; the K/V tiles of the next
// layer land as soon as this layer's are read.  A stage is armed again only
// after its 8 consumer arrivals AND its previous copy's completion (an
// aborted consumer may arrive early), and every issued copy lands before
// the warp exits.
__device__ __forceinline__ void run_kv_producer(const ProgramArgs& a, Smem& sm, const StepIn& in) {
  if (!kKvSplit || (threadIdx.x & 31) != 0) return;
  AicasScratch* s = a.scratch;
  const uint64_t pol = l2_evict_first_policy();
  const AicasPhase* P = a.phases ? a.phases : a.inl;
  TileCursor ld{P, a.n_phases, (int)gridDim.x, (int)blockIdx.x, kKvTiles};
  TileDesc td;
  uint32_t it = 0;
  while (ld.next(in, td)) {
    const int st = it % kKvRing;
    const uint32_t round = it / kKvRing;
    if (round > 0) {
      const uint32_t prev = (round - 1) & 1u;
      if (!mbar_wait_bounded(&sm.kvempty[st], prev, s, kErrEmptyTimeout)) break;
      if (!mbar_wait_copy(&sm.kvfull[st], prev, s, kErrDrainTimeout)) break;
    }
    mbar_arrive_expect_tx(&sm.kvfull[st], td.pieces * td.bytes);
    for (int i = 0; i < td.pieces; ++i)
      bulk_g2s(sm.kv[st] + i * td.dst_stride, td.src + i * td.src_stride, td.bytes, &sm.kvfull[st], pol);
    ++it;
  }
  const uint32_t first = it > (uint32_t)kKvRing ? it - kKvRing : 0;
  for (uint32_t k = first; k < it; ++k) {
    const int st = k % kKvRing;
    if (!mbar_wait_bounded(&sm.kvfull[st], (k / kKvRing) & 1u, s, kErrDrainTimeout)) {
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&sm.kvfull[st], (k / kKvRing) & 1u)) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) break;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Consumers (warps 1..8)
// ---------------------------------------------------------------------------
// kLean: the instantiation for programs whose every GEMV-type phase streams
// whole 2048-column chunks through TMEM with k = 2048 (row-major tile order)
// or k = 6144 (chunk-major, <= 2 row groups per CTA) -- the engine's 28-layer
// program.  It carries none of the other tile paths: the kernel's executed
// code is smaller, and on B200 the step is sensitive to instruction-cache
// misses (same-box A/B on the 28-layer step: 972 -> 955 us per token).
template <bool kTrace, bool kLean>
struct Consumer {
  const ProgramArgs& a;
  Smem& sm;
  const StepIn in;
  AicasScratch* s;
  int tid;  // 0..255
  int w;    // consumer warp 0..7
  int lane;
  int nct, cta;
  Ring r;
  uint64_t bar_base;
  uint32_t bar_k = 0;
  uint32_t epoch_base;  // LL epoch of phase p = epoch_base + p + 1
  int ph = 0;           // running phase index
  uint32_t tmem = 0;    // TMEM slot ring base address
  uint32_t tg = 0;      // TMEM-path tiles consumed so far
  int rwt = 0;          // tile row of this warp: the row its TMEM lane quarter holds

  // GEMV column (within a 2048-column chunk) of this lane's value v = 0..7:
  // 512 (lane / 8) + 64 v + 8 (lane % 8) + [0, 8), the layout of a tile row in
  // a TMEM lane (see run_mover); the shared-memory path reads the same columns.
  __device__ __forceinline__ int colv(int v) const { return 512 * (lane >> 3) + 64 * v + 8 * (lane & 7); }
  // residual rows of this warp's first groups of the coming phase
  float rv_lane = 0.f;  // residual of the row this lane finishes in the phase's first epilogue batch

  // Waits never end the consumer loop early: after a failed (timed-out or
  // aborted) wait the CTA keeps walking the same program without waiting, so
  // every named barrier is still reached by all 256 consumer threads and the
  // launch ends promptly with the error recorded in the scratch block.
  uint64_t wait_ns = 0;  // trace only: time consumer warp 0 spent waiting for tiles in this phase
  __device__ __forceinline__ void wait_full_at(int st, uint32_t round) {
    if (kTrace && tid == 0) {
      const uint64_t t0 = globaltimer_ns();
      mbar_wait_bounded(&sm.full[st], round & 1u, s, kErrFullTimeout);
      wait_ns += globaltimer_ns() - t0;
      return;
    }
    mbar_wait_bounded(&sm.full[st], round & 1u, s, kErrFullTimeout);
  }
  uint32_t kv_it = 0;  // K/V tiles consumed so far (AICAS_KV_STAGES)
  __device__ __forceinline__ void wait_kv(int st, uint32_t round) {
    if (kTrace && tid == 0) {
      const uint64_t t0 = globaltimer_ns();
      mbar_wait_bounded(&sm.kvfull[st], round & 1u, s, kErrFullTimeout);
      wait_ns += globaltimer_ns() - t0;
      return;
    }
    mbar_wait_bounded(&sm.kvfull[st], round & 1u, s, kErrFullTimeout);
  }
  __device__ __forceinline__ void wait_full(int st) {
    if (kTrace && tid == 0) {
      const uint64_t t0 = globaltimer_ns();
      mbar_wait_bounded(&sm.full[st], r.round() & 1u, s, kErrFullTimeout);
      wait_ns += globaltimer_ns() - t0;
      return;
    }
    mbar_wait_bounded(&sm.full[st], r.round() & 1u, s, kErrFullTimeout);
  }
  __device__ __forceinline__ void release(int st) {
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.cempty[st]);
    ++r.it;
  }

  uint32_t it_at_start = 0;
  // which: 0 = phase start, 1 = inputs ready, 2 = phase end (also records
  // the tile-wait time and the number of tiles consumed)
  __device__ __forceinline__ void stamp(int phase, int which) {
    if (kTrace && tid == 0) {
      int64_t* t = a.trace + ((size_t)cta * a.n_phases + phase) * kTraceFields;
      t[which] = (int64_t)globaltimer_ns();
      if (which == 0) it_at_start = r.it + kv_it;
      if (which == 2) {
        t[3] = (int64_t)wait_ns;
        t[5] = (int64_t)(r.it + kv_it - it_at_start);
        wait_ns = 0;
      }
    }
  }

  // Extra timestamps of the traced variant: field 6 = this CTA's own compute
  // done (last tile or attention unit), field 7 = results issued (attention:
  // partial stored, or all splits merged by the merging CTA).
  __device__ __forceinline__ void stamp_field(int field) {
    if (kTrace && tid == 0) a.trace[((size_t)cta * a.n_phases + ph) * kTraceFields + field] = (int64_t)globaltimer_ns();
  }

  // Token id of the step, checked against the embedding table (an
  // out-of-range id raises kErrBadInput and reads row 0 instead).
  __device__ __forceinline__ int64_t checked_token(const AicasPhase& d) {
    if (in.token >= 0 && in.token < d.embed_rows) return in.token;
    if (tid == 0) raise_error(s, kErrBadInput);
    return 0;
  }

  __device__ __forceinline__ float resid_value(const AicasPhase& d, int row) {
    if (d.flags & AICAS_F_LL_RESID) {  // complete before this phase: data only
      const uint32_t word = ll_load1w(reinterpret_cast<const uint32_t*>(d.resid) + row);
      return __half2float(__ushort_as_half((unsigned short)(word & 0xffffu)));
    }
    const __half* rp = reinterpret_cast<const __half*>(d.resid);
    if (d.flags & AICAS_F_RESID_EMBED) rp += (size_t)checked_token(d) * d.n;
    float rv = ldcg_half(rp + row);
    if (d.flags & AICAS_F_RESID_ADD) rv = r16(rv + ldcg_half(reinterpret_cast<const __half*>(d.resid2) + row));
    return rv;
  }

  // Work for phase `d` that depends on nothing the previous phase writes: the
  // residual rows of the first epilogue batch -> registers (loads issued here,
  // first used in the epilogue).  Runs between this CTA's barrier arrival and
  // its wait.  Nothing here blocks on a load: a synchronous load before the
  // input poll would sit on the critical path of the hand-off (the norm
  // weights of a phase are loaded into registers by build_x, before its poll;
  // measured on B200 with the 28-layer step: 1019 -> 983 us per token).
  __device__ __forceinline__ void prefetch(const AicasPhase& d) {
    if (d.kind == AICAS_PH_ATTN) return;  // q/k norm weights are loaded into registers by run_attention
    if (d.flags & AICAS_F_RESID) {  // lane l: the row of group l of this CTA (first epilogue batch)
      const Range rg = split_range((d.n + kRows - 1) / kRows, nct, cta, d.rot);
      const int row = (rg.start + lane) * kRows + rwt;
      rv_lane = (lane < rg.count && lane < kEpiBatch && row < d.n) ? resid_value(d, row) : 0.f;
    }
  }

  // The phase input vector:
  //   v = x (or the token's embedding row) [+ x2, rounded]; optionally
  //   RMSNorm with HF's rounding points (modeling_qwen3_vl.py:398-403).
  // The warps load (or poll) disjoint slices and meet at one consumer
  // barrier; the sum of squares is reduced per warp and then over the 8
  // warps.  C == 1: each lane ends with its 64 values in registers (x0).
  // C > 1: the vector stays in sm.nw -- the norm prologue is limited to
  // k <= 2048.  Columns at or beyond k read as zero.
  template <int C>
  __device__ __forceinline__ void build_x(const AicasPhase& d, uint4 (&x0)[kVec]) {
    const int k = d.k, flags = d.flags;
    const __half* x = reinterpret_cast<const __half*>(d.x);
    if (flags & AICAS_F_X_EMBED) x += (size_t)checked_token(d) * k;
    const __half* x2 = reinterpret_cast<const __half*>(d.x2);
    const bool ll = flags & AICAS_F_LL_IN;
    const uint32_t* xw = reinterpret_cast<const uint32_t*>(d.x);
    const uint32_t x_epoch = (epoch_base + (uint32_t)d.x_src + 1) & 0xffffu;
    // The 8 warps split the input: vector index v = c*kVec + j covers
    // columns c*2048 + j*256 + [lane*8, lane*8 + 8), and warp w takes
    // v = w, w + 8, ...  Each CTA so reads (polls) the vector once, not once
    // per warp.  C == 1: the vector goes to sm.xs and every warp reads its
    // lanes' 64 values back into registers (x0); C > 1: to sm.nw.
    constexpr int NV = (C * kVec + kConsumerWarps - 1) / kConsumerWarps;
    int cols[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int v = i * kConsumerWarps + w;
      const int col = (v / kVec) * kChunk + (v % kVec) * 256 + lane * 8;
      cols[i] = (v < C * kVec && col < k) ? col : -1;
    }
    uint4 raw[NV];
    uint4 nwr[NV];
    const bool norm1 = C == 1 && (flags & AICAS_F_NORM);
    if (norm1) {  // issued before the poll, used after it: the load latency hides behind the wait
#pragma unroll
      for (int i = 0; i < NV; ++i)
        nwr[i] = cols[i] >= 0 ? __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(d.norm_w) + cols[i]))
                              : make_uint4(0, 0, 0, 0);
    }
    if (ll) {
      ll_poll8_n<NV>(xw, cols, x_epoch, s, raw);
    } else {
#pragma unroll
      for (int i = 0; i < NV; ++i) raw[i] = cols[i] >= 0 ? ldcg_u4(x + cols[i]) : make_uint4(0, 0, 0, 0);
    }
    float ss = 0.f;
    __half* xbuf = C == 1 ? sm.xs : sm.nw;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      if (cols[i] < 0) continue;
      if (flags & AICAS_F_X_ADD) {
        const uint4 raw2 = ldcg_u4(x2 + cols[i]);
        __half2* hp = reinterpret_cast<__half2*>(&raw[i]);
        const __half2* hq = reinterpret_cast<const __half2*>(&raw2);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 fa = __half22float2(hp[q]), fb = __half22float2(hq[q]);
          hp[q] = __floats2half2_rn(fa.x + fb.x, fa.y + fb.y);
        }
      }
      if (C == 1) {
        const __half2* hp = reinterpret_cast<const __half2*>(&raw[i]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = __half22float2(hp[q]);
          ss += f.x * f.x + f.y * f.y;
        }
      }
      if (!norm1) *reinterpret_cast<uint4*>(&xbuf[cols[i]]) = raw[i];
    }
    if (norm1) {
      // RMSNorm of the thread's own slice (HF rounding points), then the
      // normalised vector goes to shared memory for every warp
      ss = warp_sum(ss);
      if (lane == 0) sm.ssq[w] = ss;
      consumer_sync(kConsumerThreads);
      ss = 0.f;
#pragma unroll
      for (int i = 0; i < kConsumerWarps; ++i) ss += sm.ssq[i];
      const float inv = rsqrtf(ss / (float)k + d.eps);
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        if (cols[i] < 0) continue;
        __half2* hp = reinterpret_cast<__half2*>(&raw[i]);
        const __half2* wp = reinterpret_cast<const __half2*>(&nwr[i]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = __half22float2(hp[q]);
          const float2 g = __half22float2(wp[q]);
          hp[q] = __floats2half2_rn(g.x * r16(f.x * inv), g.y * r16(f.y * inv));
        }
        *reinterpret_cast<uint4*>(&xbuf[cols[i]]) = raw[i];
      }
    }
    consumer_sync(kConsumerThreads);
    if constexpr (C == 1) {
#pragma unroll
      for (int j = 0; j < kVec; ++j) {
        const int col = colv(j);
        x0[j] = col < k ? *reinterpret_cast<const uint4*>(&sm.xs[col]) : make_uint4(0, 0, 0, 0);
      }
    }
    if ((flags & AICAS_F_STORE_X) && cta == 0 && w == 0 && d.x_out) {
      __half* xo = reinterpret_cast<__half*>(d.x_out);
#pragma unroll
      for (int c = 0; c < C; ++c)
#pragma unroll
        for (int j = 0; j < kVec; ++j) {
          const int col = c * kChunk + colv(j);
          if (col < k) *reinterpret_cast<uint4*>(xo + col) = C == 1 ? x0[j] : *reinterpret_cast<const uint4*>(&sm.nw[col]);
        }
    }
  }

  // This lane's 8 fp16 x vectors of chunk c (registers for C == 1, else
  // read back from sm.nw).
  template <int C>
  __device__ __forceinline__ void x_chunk(int c, int k, const uint4 (&x0)[kVec], uint4 (&xc)[kVec]) {
#pragma unroll
    for (int j = 0; j < kVec; ++j) {
      const int col = c * kChunk + colv(j);
      // C > 1: inline-asm shared loads, so they stay after the tile wait they follow
      xc[j] = C == 1 ? x0[j] : (col < k ? lds_u4(smem_addr(&sm.nw[col])) : make_uint4(0, 0, 0, 0));
    }
  }

  // This lane's 64 columns of one tile row into registers (`row_s`: shared
  // address of the row plus the lane's offset 1024 (lane / 8) + 16 (lane % 8);
  // value v sits 128 v bytes further); `jmask` skips columns beyond k.  Loading a tile completely
  // before the math lets the stage go back to the producer immediately, so
  // the FMAs overlap the next copies instead of lengthening the ring cycle.
  __device__ __forceinline__ static void row_load(uint32_t row_s, unsigned jmask, uint4 (&wv)[kVec]) {
#pragma unroll
    for (int j = 0; j < kVec; ++j) wv[j] = ((jmask >> j) & 1u) ? lds_u4(row_s + j * 128) : make_uint4(0, 0, 0, 0);
  }

  // acc[0..3] += row . x (both fp16): exact fp16 products, fp32 accumulation
  // in 4 independent chains (PTX mixed-precision fma.rn.f32.f16).
  __device__ __forceinline__ static void row_fma(const uint4 (&wv)[kVec], const uint4 (&xh)[kVec], float (&acc)[4]) {
#pragma unroll
    for (int j = 0; j < kVec; ++j) acc[j & 3] = dot8_f16(wv[j], xh[j], acc[j & 3]);
  }

  // The 4 accumulation chains of a lane folded into its partial sum.
  __device__ __forceinline__ static float fold4(const float (&a)[4]) { return (a[0] + a[1]) + (a[2] + a[3]); }

  // Batched epilogue: the warp has written the lane partial sums of `cnt`
  // row groups (group base `gbase` + slot, `parts` sums each) to sm.epi; lane
  // l < cnt finishes group gbase + l: sums its 32 partials (in a fixed order),
  // applies bias/residual/SiLU and rounding (row_value) and stores the row.
  // One pass replaces a 5-shuffle reduction plus a lane-0 epilogue per group.
  __device__ __forceinline__ void epi_flush(const AicasPhase& d, int kind, int flags, int n, int gbase, int cnt,
                                            int parts, bool first_batch, const __half* bias, __half* logits,
                                            __half* out, float& best_v, int& best_i) {
    __syncwarp();
    if (lane < cnt) {
      float s2[2] = {0.f, 0.f};
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        if (p < parts) {
          const float* e = &sm.epi[w][lane * parts + p][0];
          float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int j = 0; j < 32; ++j) c[j & 3] += e[j];
          s2[p] = fold4(c);
        }
      }
      const int row = (gbase + lane) * kRows + rwt;
      if (row < n) {
        const float rv = !(flags & AICAS_F_RESID) ? 0.f : (first_batch ? rv_lane : resid_value(d, row));
        float y[kRowsPerWarp];
        y[0] = row_value(kind, flags, row, s2[0], s2[1], rv, bias, logits, best_v, best_i);
        store_rows(flags, n, row, y, out);
      }
    }
    __syncwarp();
  }

  // Output value of one row with the rounding points of HF's fp16 path; the
  // LM head also stores the logit and updates the lane's running argmax.
  __device__ __forceinline__ static float row_value(int kind, int flags, int row, float sum0, float sum1, float rv,
                                                    const __half* bias, __half* logits, float& best_v, int& best_i) {
    if (kind == AICAS_PH_GATEUP) {
      const float gq = r16(sum0), uq = r16(sum1);
      const float sl = r16(gq / (1.0f + expf(-gq)));
      return r16(sl * uq);
    }
    if (flags & AICAS_F_BIAS) sum0 += __half2float(bias[row]);
    float y = r16(sum0);
    if (flags & AICAS_F_RESID) y = r16(rv + y);
    if (kind == AICAS_PH_LMHEAD) {
      if (logits) logits[row] = __float2half_rn(y);
      // a lane's rows ascend (its groups ascend): strict > keeps the first max
      if (y > best_v) {
        best_v = y;
        best_i = row;
      }
    }
    return y;
  }

  // Stores output rows row0.. (LL words or plain fp16).
  __device__ __forceinline__ void store_rows(int flags, int n, int row0, const float (&y)[kRowsPerWarp], __half* out) {
    if (!out) return;
#pragma unroll
    for (int rr = 0; rr < kRowsPerWarp; ++rr) {
      if (row0 + rr >= n) break;
      if (flags & AICAS_F_LL_OUT)
        ll_store(reinterpret_cast<uint32_t*>(out) + row0 + rr, y[rr], (epoch_base + (uint32_t)ph + 1) & 0xffffu);
      else
        out[row0 + rr] = __float2half_rn(y[rr]);
    }
  }

  // GEMV / GATEUP / LMHEAD phase, C = number of 2048-column chunks of k.
  template <int C>
  __device__ __forceinline__ void matvec(const AicasPhase& d) {
    uint4 x0[kVec];
    build_x<C>(d, x0);
    stamp(ph, 1);
    // descriptor fields in registers (the waits below clobber memory).  A
    // GATEUP phase always has k <= 2048 (host-checked), and the lean kernel
    // runs the LM head only with k == 2048: for C > 1 those kinds cannot occur,
    // so this instantiation carries no code for them.
    const int n = d.n, k = d.k, flags = d.flags;
    const int kind = C == 1 ? d.kind : (d.kind == AICAS_PH_GATEUP || (kLean && d.kind == AICAS_PH_LMHEAD))
                                           ? AICAS_PH_GEMV : d.kind;
    const bool gateup = C == 1 && kind == AICAS_PH_GATEUP;
    __half* const out = reinterpret_cast<__half*>(d.out);
    const __half* const bias = reinterpret_cast<const __half*>(d.bias);
    const Range rg = split_range((n + kRows - 1) / kRows, nct, cta, d.rot);
    const int row_stride = C == 1 ? k * 2 : kRowBytes;
    // lanes whose columns of the last chunk lie beyond k skip them
    const int last_len = k - (C - 1) * kChunk;
    unsigned jlast = 0;
#pragma unroll
    for (int j = 0; j < kVec; ++j) jlast |= (colv(j) < last_len ? 1u : 0u) << j;
    const bool use_tm = kLean || tmem_phase(kind, k);
    float best_v = -INFINITY;
    int best_i = 0x7fffffff;
    __half* logits = nullptr;
    if (kind == AICAS_PH_LMHEAD && a.state && a.state->logits) {
      const int64_t ring = a.state->logits_ring > 0 ? a.state->logits_ring : 1;
      logits = reinterpret_cast<__half*>(a.state->logits) + (size_t)(in.step % ring) * n;
    }
    // everything the tile loops touch lives in registers
    const uint32_t ring_s = smem_addr(&sm.ring[0][0]) + 1024 * (lane >> 3) + 16 * (lane & 7);
    const uint32_t full_s = smem_addr(&sm.full[0]);
    const uint32_t cempty_s = smem_addr(&sm.cempty[0]);
    const uint32_t tfull_s = smem_addr(&sm.tfull[0]);
    const uint32_t tempty_s = smem_addr(&sm.tempty[0]);
    // this warp's row in the TMEM slot: lanes of its quarter, column half
    const uint32_t tm_row = tmem + ((uint32_t)(32 * ((w + 1) & 3)) << 16) + 32 * (w >> 2);
    uint32_t tgl = tg;
    AicasScratch* const scr = s;
    const int ln = lane;
    static_assert(kRowsPerWarp == 1, "one tile row per warp (its TMEM lane quarter and column half)");
    const bool timing = kTrace && tid == 0;
    uint64_t waited = 0;
    uint32_t it = r.it;
#define AICAS_TAKE(st)                                                                          \
  do {                                                                                          \
    st = it % kStages;                                                                          \
    if (timing) {                                                                               \
      const uint64_t t0_ = globaltimer_ns();                                                    \
      mbar_wait_bounded_s(full_s + st * 8, (it / kStages) & 1u, scr, kErrFullTimeout);          \
      waited += globaltimer_ns() - t0_;                                                         \
    } else {                                                                                    \
      mbar_wait_bounded_s(full_s + st * 8, (it / kStages) & 1u, scr, kErrFullTimeout);          \
    }                                                                                           \
  } while (0)
#define AICAS_GIVE(st)                        \
  do {                                        \
    __syncwarp();                             \
    if (ln == 0) mbar_arrive_s(cempty_s + st * 8); \
    ++it;                                     \
  } while (0)
// One tile row from the next TMEM slot (the whole warp) and the slot
// released; after a failed wait the row reads as zeros.
#define AICAS_TLOAD(wv_, valid_)                                                                  \
  do {                                                                                            \
    const uint32_t t_ = tgl % kTmemSlots;                                                         \
    uint64_t t0_ = timing ? globaltimer_ns() : 0;                                                 \
    bool ok_ = mbar_wait_bounded_s(tfull_s + t_ * 8, (tgl / kTmemSlots) & 1u, scr, kErrTmemTimeout); \
    if (timing) waited += globaltimer_ns() - t0_;                                                 \
    ok_ = __all_sync(0xffffffffu, ok_);                                                           \
    tc_fence_after();                                                                             \
    /* always in bounds: TMEM stays allocated until every consumer warp is done */              \
    tmem_ld_32x32b_x32_u4(tm_row + t_ * kTmemTileCols, wv_);                                      \
    tmem_wait_ld();                                                                               \
    tc_fence_before();                                                                            \
    __syncwarp();                                                                                 \
    if (ln == 0) mbar_arrive_s(tempty_s + t_ * 8);                                                \
    ++tgl;                                                                                        \
    ++it;                                                                                         \
    if (!(ok_ && (valid_))) {                                                                     \
      _Pragma("unroll") for (int v_ = 0; v_ < kVec; ++v_) wv_[v_] = make_uint4(0, 0, 0, 0);      \
    }                                                                                             \
  } while (0)
    uint4 xh[kVec];  // fp16 input slice of the running chunk (C > 1; C == 1 uses x0)
    if (kLean ? C > 1 : chunk_major(C, kind, rg.count)) {
      float acc[kMaxCmajorGroups][kRowsPerWarp][4];
#pragma unroll
      for (int g = 0; g < kMaxCmajorGroups; ++g)
#pragma unroll
        for (int rr = 0; rr < kRowsPerWarp; ++rr)
#pragma unroll
          for (int q = 0; q < 4; ++q) acc[g][rr][q] = 0.f;
#pragma unroll 1
      for (int c = 0; c < C; ++c) {  // not unrolled: one copy of the tile code per group
        x_chunk<C>(c, k, x0, xh);
        const unsigned jmask = c < C - 1 ? 0xffu : jlast;
#pragma unroll
        for (int gi = 0; gi < kMaxCmajorGroups; ++gi) {
          if (gi < rg.count) {
            uint4 wv[kRowsPerWarp][kVec];
            const int row = (rg.start + gi) * kRows + rwt;
            if (use_tm) {
              AICAS_TLOAD(wv[0], row < n);
            } else {
              uint32_t st;
              AICAS_TAKE(st);
              row_load(ring_s + st * kStageBytes + rwt * row_stride, row < n ? jmask : 0u, wv[0]);
              AICAS_GIVE(st);
            }
#pragma unroll
            for (int rr = 0; rr < kRowsPerWarp; ++rr) if constexpr (C == 1) row_fma(wv[rr], x0, acc[gi][rr]); else row_fma(wv[rr], xh, acc[gi][rr]);
          }
        }
      }
#pragma unroll
      for (int gi = 0; gi < kMaxCmajorGroups; ++gi)
        if (gi < rg.count) sm.epi[w][gi][ln] = fold4(acc[gi][0]);
      epi_flush(d, kind, flags, n, rg.start, rg.count, 1, true, bias, logits, out, best_v, best_i);
    } else {
      const int parts = gateup ? 2 : 1;
      int gb = 0;  // first group of the running epilogue batch
      for (int gi = 0; gi < rg.count; ++gi) {
        float acc[2][kRowsPerWarp][4];
#pragma unroll
        for (int p = 0; p < 2; ++p)
#pragma unroll
          for (int rr = 0; rr < kRowsPerWarp; ++rr)
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[p][rr][q] = 0.f;
#pragma unroll
        for (int part = 0; part < (C == 1 ? 2 : 1); ++part) {  // gate_up: k <= 2048 (host-checked)
          if (part == 1 && !gateup) break;
#pragma unroll 1
          for (int c = 0; c < C; ++c) {
            if (C > 1) x_chunk<C>(c, k, x0, xh);
            const unsigned jmask = c < C - 1 ? 0xffu : jlast;
            uint4 wv[kRowsPerWarp][kVec];
            const int row = (rg.start + gi) * kRows + rwt;
            if (use_tm) {
              AICAS_TLOAD(wv[0], row < n);
            } else {
              uint32_t st;
              AICAS_TAKE(st);
              row_load(ring_s + st * kStageBytes + rwt * row_stride, row < n ? jmask : 0u, wv[0]);
              AICAS_GIVE(st);
            }
#pragma unroll
            for (int rr = 0; rr < kRowsPerWarp; ++rr) if constexpr (C == 1) row_fma(wv[rr], x0, acc[part][rr]); else row_fma(wv[rr], xh, acc[part][rr]);
          }
        }
        const int slot = gi - gb;
        sm.epi[w][slot * parts][ln] = fold4(acc[0][0]);
        if (gateup) sm.epi[w][slot * parts + 1][ln] = fold4(acc[1][0]);
        if (slot == kEpiBatch - 1 || gi == rg.count - 1) {
          epi_flush(d, kind, flags, n, rg.start + gb, slot + 1, parts, gb == 0, bias, logits, out, best_v, best_i);
          gb = gi + 1;
        }
      }
    }
#undef AICAS_TAKE
#undef AICAS_GIVE
#undef AICAS_TLOAD
    stamp_field(7);
    wait_ns += waited;
    r.it = it;
    tg = tgl;
    if (kind == AICAS_PH_LMHEAD) {
      // lanes -> warp: larger value, or the same value at a smaller row
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float v2 = __shfl_xor_sync(0xffffffffu, best_v, o);
        const int i2 = __shfl_xor_sync(0xffffffffu, best_i, o);
        if (v2 > best_v || (v2 == best_v && i2 < best_i)) {
          best_v = v2;
          best_i = i2;
        }
      }
      finish_argmax(d, best_v, best_i);
    }
  }

  __device__ __forceinline__ void run_matvec(const AicasPhase& d) {
    const int C = n_chunks(d);
    if (C == 1) matvec<1>(d);
    else if (!kLean && C == 2) matvec<2>(d);
    else matvec<3>(d);
  }

  __device__ __forceinline__ void finish_argmax(const AicasPhase& d, float bv, int bi) {
    if (lane == 0) {
      sm.best_v[w] = bv;
      sm.best_i[w] = bi;
    }
    consumer_sync(kConsumerThreads);
    if (tid == 0) {
      float v = sm.best_v[0];
      int i = sm.best_i[0];
      for (int t = 1; t < kConsumerWarps; ++t) {
        if (sm.best_v[t] > v || (sm.best_v[t] == v && sm.best_i[t] < i)) {
          v = sm.best_v[t];
          i = sm.best_i[t];
        }
      }
      s->am_val[cta] = v;
      s->am_idx[cta] = i;
      __threadfence();
      const uint32_t prev = atomicAdd(&s->argmax_done, 1u);
      if (prev == (uint32_t)nct - 1) {
        __threadfence();
        float bv2 = -INFINITY;
        int bi2 = 0x7fffffff;
        for (int c = 0; c < nct; ++c) {
          const float cv = __ldcg(&s->am_val[c]);
          const int ci = __ldcg(&s->am_idx[c]);
          if (cv > bv2 || (cv == bv2 && ci < bi2)) {
            bv2 = cv;
            bi2 = ci;
          }
        }
        s->argmax_done = 0;
        if (d.idx_out) *reinterpret_cast<int64_t*>(d.idx_out) = bi2;
        AicasStepState* stt = a.state;
        if (stt) {
          const int64_t step = in.step;
          if (stt->out_tokens && step < stt->max_steps) stt->out_tokens[step] = bi2;
          const int64_t nx = step + 1;
          if (stt->script && nx < stt->script_len) {
            const int64_t* e = stt->script + nx * 5;
            stt->token = e[0];
            stt->cache_pos = e[1];
            stt->rope[0] = e[2];
            stt->rope[1] = e[3];
            stt->rope[2] = e[4];
          } else {
            stt->token = bi2;
            stt->cache_pos = in.pos + 1;
            stt->rope[0] = in.rope[0] + 1;
            stt->rope[1] = in.rope[1] + 1;
            stt->rope[2] = in.rope[2] + 1;
          }
          stt->step = nx;
          // device-side end of sequence: a generated token (the script's
          // last step onward) equal to eos_token ends the request
          if (stt->eos_token >= 0 && bi2 == stt->eos_token && nx >= stt->script_len) stt->done_step = nx;
          __threadfence();
        }
      }
    }
  }

  // One 128-dim head per warp (lane l holds dims 4l..4l+3): per-head RMSNorm
  // (modeling_qwen3_vl.py:398-403) and rotary embedding (:124-128, :427-431).
  // rotate_half's partner of dim d is d +- 64, held by lane l ^ 16.
  __device__ __forceinline__ void norm_rope_head(float (&v)[4], uint2 nw, float eps, const float (&cs)[4],
                                 const float (&sn)[4]) {
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) ss += v[e] * v[e];
    const float inv = rsqrtf(warp_sum(ss) / (float)kHD + eps);
    float xn[4];
    const __half2* nh = reinterpret_cast<const __half2*>(&nw);
    const float nwf[4] = {__low2float(nh[0]), __high2float(nh[0]), __low2float(nh[1]), __high2float(nh[1])};
#pragma unroll
    for (int e = 0; e < 4; ++e) xn[e] = r16(nwf[e] * r16(v[e] * inv));
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float p = __shfl_xor_sync(0xffffffffu, xn[e], 16);
      const float rot = lane < 16 ? -p : p;
      v[e] = r16(r16(xn[e] * cs[e]) + r16(rot * sn[e]));
    }
  }

  // Every CTA of a KV head merges a 1/nsplit slice of the head's 256
  // outputs, one output per group of tpo lanes (a power of two <= 16, as
  // many as the CTA's threads allow): lane `sub` of the group takes splits
  // sub, sub + tpo, ... in order (the same order whichever CTA merges),
  // polling up to kMergePer of them per round, then the group combines its
  // (max, sum, acc) triples with a fixed xor-shuffle tree.
  __device__ __forceinline__ void merge_head(const AicasPhase& d, int h, int split, int nsplit, uint32_t ep) {
    uint64_t* const hp = &s->part[h][0][0][0];
    constexpr int kSplitStride = 2 * (kHD + 1);
    uint32_t* const out_w = reinterpret_cast<uint32_t*>(d.out);
    __half* const out_h = reinterpret_cast<__half*>(d.out);
    const bool ll_out = d.flags & AICAS_F_LL_OUT;
    const int q0 = split * 2 * kHD / nsplit, q1 = (split + 1) * 2 * kHD / nsplit;
    const int npairs = q1 - q0;
    int tpo = 16;
    while (tpo > 1 && tpo * npairs > kConsumerThreads) tpo >>= 1;
    const int nact = npairs * tpo;
    if ((tid & ~31) < nact) {  // warps holding at least one active lane
      const bool act = tid < nact;
      const int pl = tid / tpo, sub = tid % tpo;
      const int q = q0 + (act ? pl : 0), gq = q / kHD, tq = q % kHD;
      const uint64_t* const base = hp + gq * (kHD + 1);
      float mx = -INFINITY, S = 0.f, acc = 0.f;
#pragma unroll 1
      for (int b0 = act ? sub : nsplit; b0 < nsplit; b0 += tpo * kMergePer) {
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
          // predicates from the round's starting masks: no load waits
          // for another load's result, so a round is one round trip
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
              acc = acc * c + oi;
              mx = li;
            } else {
              const float c = expf(li - mx);
              S += c;
              acc += c * oi;
            }
          }
        }
      }
      for (int o = 1; o < tpo; o <<= 1) {  // tpo is the same in every lane
        const float m2 = __shfl_xor_sync(0xffffffffu, mx, o);
        const float s2 = __shfl_xor_sync(0xffffffffu, S, o);
        const float a2 = __shfl_xor_sync(0xffffffffu, acc, o);
        const float mm = fmaxf(mx, m2);
        if (mm != -INFINITY) {
          const float f1 = mx == -INFINITY ? 0.f : expf(mx - mm);
          const float f2 = m2 == -INFINITY ? 0.f : expf(m2 - mm);
          S = S * f1 + s2 * f2;
          acc = acc * f1 + a2 * f2;
          mx = mm;
        }
      }
      if (act && sub == 0) {
        const int oidx = (h * 2 + gq) * kHD + tq;
        if (ll_out) ll_store(out_w + oidx, acc / S, ep & 0xffffu);
        else out_h[oidx] = __float2half_rn(acc / S);
      }
    }
  }

  // One warp's 16 positions p0 .. p0 + 15 of a 64-slot K/V tile (shared
  // address `tile`): online-softmax update of (m, l, acc) for both query
  // heads.  Scores: lane (pi = lane / 4, dim quarter qc = lane % 4) dots
  // positions p0 + pi and p0 + 8 + pi over dims qc*32 .. qc*32+31 (exact fp16
  // products, fp32 sums; K rows read in an order rotated by pi, free of bank
  // conflicts); two shuffles finish each score.  P V: lane l accumulates dims
  // 4l .. 4l+3; the probabilities pass through the warp's shared-memory row.
  // Slot `pos` (this step's k / v; -1: none) comes from at.kf / at.vf: the tile
  // may have been loaded before it was written.
  __device__ __forceinline__ void attend_tile(const uint8_t* tile, int p0, int pos, int valid, float scale,
                                              float (&m)[2], float (&l)[2], float (&acc)[2][4]) {
    AttnSmem& at = sm.at;
    const int pi = lane >> 2, qc = lane & 3;
    const int row0 = p0 % kAttnChunk;
    float sg[2][2];
#pragma unroll
    for (int a2 = 0; a2 < 2; ++a2) {
      sg[a2][0] = sg[a2][1] = 0.f;
      const int prow = row0 + 8 * a2 + pi;
      if (p0 + 8 * a2 + pi == pos) {
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const int qo = qc * 32 + 8 * ((jj + pi) & 3);
          uint4 kv;
          __half2* kh = reinterpret_cast<__half2*>(&kv);
#pragma unroll
          for (int e = 0; e < 4; ++e) kh[e] = __floats2half2_rn(at.kf[qo + 2 * e], at.kf[qo + 2 * e + 1]);
          sg[a2][0] = dot8_f16(kv, *reinterpret_cast<const uint4*>(&at.qh[0][qo]), sg[a2][0]);
          sg[a2][1] = dot8_f16(kv, *reinterpret_cast<const uint4*>(&at.qh[1][qo]), sg[a2][1]);
        }
      } else {
        const uint8_t* krow = tile + prow * (kHD * 2) + qc * 64;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const int jr = (jj + pi) & 3;
          const uint4 kv = *reinterpret_cast<const uint4*>(krow + 16 * jr);
          const int qo = qc * 32 + 8 * jr;
          sg[a2][0] = dot8_f16(kv, *reinterpret_cast<const uint4*>(&at.qh[0][qo]), sg[a2][0]);
          sg[a2][1] = dot8_f16(kv, *reinterpret_cast<const uint4*>(&at.qh[1][qo]), sg[a2][1]);
        }
      }
    }
    float pr[2][2];
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      float x[2];
#pragma unroll
      for (int a2 = 0; a2 < 2; ++a2) {
        float v = sg[a2][g];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        x[a2] = p0 + 8 * a2 + pi < valid ? v * scale : -INFINITY;
      }
      float cm = fmaxf(x[0], x[1]);
      cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 4));
      cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 8));
      cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 16));
      const float mn = fmaxf(m[g], cm);
      pr[0][g] = pr[1][g] = 0.f;
      if (mn == -INFINITY) continue;  // (warp-uniform) no valid position yet
#pragma unroll
      for (int a2 = 0; a2 < 2; ++a2) pr[a2][g] = x[a2] == -INFINITY ? 0.f : expf(x[a2] - mn);
      float ps = pr[0][g] + pr[1][g];
      ps += __shfl_xor_sync(0xffffffffu, ps, 4);
      ps += __shfl_xor_sync(0xffffffffu, ps, 8);
      ps += __shfl_xor_sync(0xffffffffu, ps, 16);
      const float corr = expf(m[g] - mn);
      l[g] = l[g] * corr + ps;
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[g][e] *= corr;
      m[g] = mn;
    }
    if (qc == 0) {
      at.sc[w][pi] = make_float2(pr[0][0], pr[0][1]);
      at.sc[w][8 + pi] = make_float2(pr[1][0], pr[1][1]);
    }
    __syncwarp();
    const uint8_t* vt = tile + kStageBytes / 2;
#pragma unroll 4
    for (int i = 0; i < 16; ++i) {
      if (p0 + i >= valid) break;
      const float2 pp = at.sc[w][i];
      float vv[4];
      if (p0 + i == pos) {
#pragma unroll
        for (int e = 0; e < 4; ++e) vv[e] = at.vf[lane * 4 + e];
      } else {
        const uint2 vr = *reinterpret_cast<const uint2*>(vt + (row0 + i) * kHD * 2 + lane * 8);
        const __half2* vh = reinterpret_cast<const __half2*>(&vr);
        vv[0] = __low2float(vh[0]);
        vv[1] = __high2float(vh[0]);
        vv[2] = __low2float(vh[1]);
        vv[3] = __high2float(vh[1]);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        acc[0][e] += pp.x * vv[e];
        acc[1][e] += pp.y * vv[e];
      }
    }
  }

  // Attention phase: the CTA's units (KV head x 64-slot chunk) segment by
  // segment; the tiles of a segment go in pairs (warps 0..3 and 4..7, each
  // warp 16 positions of its tile), and each segment ends with this CTA's
  // partial for the head (or the head's output when the CTA has all of it)
  // and its slice of the head's merge.
  __device__ __forceinline__ void run_attention(const AicasPhase& d) {
    AttnSmem& at = sm.at;
    const bool q_ready = d.flags & AICAS_F_Q_READY;
    const int valid = phase_valid_len(d, in);
    if (valid == 0) {
      if (tid == 0 && cta == 0) raise_error(s, kErrBadInput);
      return;
    }
    const int pos = valid - 1;
    const int cph = (valid + kAttnChunk - 1) / kAttnChunk;
    const int U = d.kv_heads * cph;
    const Range rg = attn_range(U, nct, cta);
    const __half* qkv = reinterpret_cast<const __half*>(d.x);
    const bool ll_in = d.flags & AICAS_F_LL_IN;
    const uint32_t* qkv_w = reinterpret_cast<const uint32_t*>(d.x);
    const uint32_t x_epoch = (epoch_base + (uint32_t)d.x_src + 1) & 0xffffu;
    __half* kc = reinterpret_cast<__half*>(d.k_cache);
    __half* vc = reinterpret_cast<__half*>(d.v_cache);
    const int qsz = d.q_heads * kHD, kvsz = d.kv_heads * kHD;
    // interleaved MRoPE cos/sin of this lane's 4 dims (table built by init_rope)
    float cs[4] = {1.f, 1.f, 1.f, 1.f}, sn[4] = {0.f, 0.f, 0.f, 0.f};
    if (!q_ready) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        cs[e] = at.rope_c[(lane * 4 + e) % (kHD / 2)];
        sn[e] = at.rope_s[(lane * 4 + e) % (kHD / 2)];
      }
    }
    const float scale = d.scale;
    const int jpos = pos / kAttnChunk;
    const int kpos = q_ready ? -1 : pos;  // the slot whose k / v come from shared memory
    const int slot = w >> 2, wq = w & 3;
    // warps 0, 1: q_norm weights of their query head; warp 2: k_norm (dims 4 lane .. 4 lane + 3),
    // issued here and first used after the q/k/v poll
    uint2 nwv = make_uint2(0, 0);
    if (!q_ready && w < 3)
      nwv = __ldg(reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(w < 2 ? d.norm_w : d.norm_w2)) + lane);
    bool stamped = false;
    float m[2], l[2], acc[2][4];
    for (int u0 = rg.start; u0 < rg.start + rg.count;) {
      const int h = u0 / cph, j0 = u0 % cph;
      const int nseg = min(cph - j0, rg.start + rg.count - u0);
      const bool has_pos = !q_ready && jpos >= j0 && jpos < j0 + nseg;
      if (w < 2) {  // query heads 2h, 2h+1
        const int col = (h * 2 + w) * kHD + lane * 4;
        const uint2 raw = ll_in ? ll_poll4(qkv_w, col, x_epoch, s) : __ldcg(reinterpret_cast<const uint2*>(qkv + col));
        const __half2* hp = reinterpret_cast<const __half2*>(&raw);
        float v[4] = {__low2float(hp[0]), __high2float(hp[0]), __low2float(hp[1]), __high2float(hp[1])};
        if (!q_ready) norm_rope_head(v, nwv, d.eps, cs, sn);
        *reinterpret_cast<__half2*>(&at.qh[w][lane * 4]) = __floats2half2_rn(v[0], v[1]);
        *reinterpret_cast<__half2*>(&at.qh[w][lane * 4 + 2]) = __floats2half2_rn(v[2], v[3]);
      } else if (has_pos && w < 4) {  // this step's k (warp 2) / v (warp 3) of head h
        const int off = qsz + (w == 2 ? 0 : kvsz) + h * kHD + lane * 4;
        const uint2 raw = ll_in ? ll_poll4(qkv_w, off, x_epoch, s) : __ldcg(reinterpret_cast<const uint2*>(qkv + off));
        const __half2* hp = reinterpret_cast<const __half2*>(&raw);
        float v[4] = {__low2float(hp[0]), __high2float(hp[0]), __low2float(hp[1]), __high2float(hp[1])};
        if (w == 2) norm_rope_head(v, nwv, d.eps, cs, sn);
        float* dst = w == 2 ? at.kf : at.vf;
#pragma unroll
        for (int e = 0; e < 4; ++e) dst[lane * 4 + e] = v[e];
        __half2 o[2] = {__floats2half2_rn(v[0], v[1]), __floats2half2_rn(v[2], v[3])};
        __half* cache = w == 2 ? kc : vc;
        *reinterpret_cast<uint2*>(cache + ((size_t)h * d.max_len + pos) * kHD + lane * 4) =
            *reinterpret_cast<uint2*>(o);
      }
      consumer_sync(kConsumerThreads);
      if (!stamped) {
        stamp(ph, 1);
        stamped = true;
      }
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[g][e] = 0.f;
      }
#pragma unroll 1
      for (int t = 0; t < nseg; t += 2) {
        if (t + slot < nseg) {
          if (kKvSplit) {
            const uint32_t ri = kv_it + slot;
            const int st = ri % kKvRing;
            wait_kv(st, ri / kKvRing);
            attend_tile(sm.kv[st], (j0 + t + slot) * kAttnChunk + 16 * wq, kpos, valid, scale, m, l, acc);
            __syncwarp();
            if (lane == 0) mbar_arrive_cnt(&sm.kvempty[st], 2);  // 4 warps per tile, 8 arrivals per stage use
          } else {
            const uint32_t ri = r.it + slot;
            const int st = ri % kStages;
            wait_full_at(st, ri / kStages);
            attend_tile(sm.ring[st], (j0 + t + slot) * kAttnChunk + 16 * wq, kpos, valid, scale, m, l, acc);
            __syncwarp();
            if (lane == 0) mbar_arrive_cnt(&sm.cempty[st], 2);  // 4 warps per tile, 8 arrivals per stage use
          }
        }
        (kKvSplit ? kv_it : r.it) += t + 1 < nseg ? 2 : 1;
      }
      stamp_field(6);
      // merge the 8 warps' states of this segment into one partial
      if (lane == 0) {
        at.wm[w][0] = m[0];
        at.wm[w][1] = m[1];
        at.wl[w][0] = l[0];
        at.wl[w][1] = l[1];
      }
#pragma unroll
      for (int g = 0; g < 2; ++g)
#pragma unroll
        for (int e = 0; e < 4; ++e) at.wacc[w][g][lane * 4 + e] = acc[g][e];
      consumer_sync(kConsumerThreads);
      const int na = attn_ctas(U, nct);
      const int first_owner = owner_of(h * cph, U, na);
      const int split = cta - first_owner;
      const int nsplit = owner_of(h * cph + cph - 1, U, na) - first_owner + 1;
      const uint32_t ep = epoch_base + (uint32_t)ph + 1;
      // thread (g, t): query head 2h + g, head dim t: merge the 8 warps' states
      const int g = tid / kHD, t = tid % kHD;
      float M = -INFINITY;
#pragma unroll
      for (int i = 0; i < kConsumerWarps; ++i) M = fmaxf(M, at.wm[i][g]);
      float L = 0.f, A = 0.f;
#pragma unroll 1
      for (int i = 0; i < kConsumerWarps; ++i) {
        const float mi = at.wm[i][g];
        if (mi != -INFINITY) {
          const float f = expf(mi - M);
          L += at.wl[i][g] * f;
          A += at.wacc[i][g][t] * f;
        }
      }
      const float lse = M + logf(L), o = A / L;
      if (nsplit == 1) {  // the whole head is this CTA's: thread (g, t) has its output
        const int oidx = (h * 2 + g) * kHD + t;
        if (d.flags & AICAS_F_LL_OUT) ll_store(reinterpret_cast<uint32_t*>(d.out) + oidx, o, ep & 0xffffu);
        else reinterpret_cast<__half*>(d.out)[oidx] = __float2half_rn(o);
      } else {
        // this CTA's partial as 64-bit LL words (no fence, no counter)
        uint64_t* const hp = &s->part[h][0][0][0];
        constexpr int kSplitStride = 2 * (kHD + 1);
        if (t == 0) ll64_store(hp + split * kSplitStride + g * (kHD + 1), lse, ep);
        ll64_store(hp + split * kSplitStride + g * (kHD + 1) + 1 + t, o, ep);
      }
      u0 += nseg;
    }
    // Then this CTA's slice of the merge of every head it shares.  The
    // partials of ALL its segments are stored before it waits for any other
    // CTA's: merging head h first would hold back this CTA's partial of head
    // h + 1 until head h's slowest CTA had stored, and at long contexts those
    // waits chained across the heads (measured at 8192 slots: the slowest CTA
    // 75 us against a 14 us median).  With every partial stored up front, a
    // merge waits only for other CTAs' unit work.
    const int na = attn_ctas(U, nct);
    const uint32_t ep = epoch_base + (uint32_t)ph + 1;
    for (int u0 = rg.start; u0 < rg.start + rg.count;) {
      const int h = u0 / cph, j0 = u0 % cph;
      const int nseg = min(cph - j0, rg.start + rg.count - u0);
      const int first_owner = owner_of(h * cph, U, na);
      const int nsplit = owner_of(h * cph + cph - 1, U, na) - first_owner + 1;
      if (nsplit > 1) merge_head(d, h, cta - first_owner, nsplit, ep);
      u0 += nseg;
    }
    stamp_field(7);
  }
  // Interleaved-MRoPE cos/sin of the step's position, once per launch
  // (every attention phase of the step uses the same table):
  // frequency i takes axis 1 (h) when i % 3 == 1 and i < 3 * section[1],
  // axis 2 (w) when i % 3 == 2 and i < 3 * section[2], else axis 0 (t);
  // cos/sin in fp32, rounded to fp16 (modeling_qwen3_vl.py:352-386).
  __device__ __noinline__ void init_rope() {
    const AicasStepState* stt = a.state;
    if (stt && tid < kHD / 2) {
      const int i = tid;
      int axis = 0;
      if (i % 3 == 1 && i < 3 * stt->mrope_section[1]) axis = 1;
      else if (i % 3 == 2 && i < 3 * stt->mrope_section[2]) axis = 2;
      const float ang = stt->inv_freq[i] * (float)in.rope[axis];
      sm.at.rope_c[i] = r16(cosf(ang));
      sm.at.rope_s[i] = r16(sinf(ang));
    }
  }

  __device__ __forceinline__ void run(const AicasPhase* P, int n_phases) {
    init_rope();  // visible after the first phase's consumer barrier
    for (ph = 0; ph < n_phases; ++ph) {
      const AicasPhase& d = P[ph];
      // every warp is done with the previous phase's shared buffers
      consumer_sync(kConsumerThreads);
      const bool barrier = ph > 0 && (d.flags & AICAS_F_BARRIER);
      if (barrier && tid == 0) grid_arrive(s);
      prefetch(d);  // registers only: nothing to publish through shared memory
      if (barrier) {
        if (tid == 0) grid_wait(s, bar_base + (uint64_t)(++bar_k) * nct);
        consumer_sync(kConsumerThreads);  // every consumer thread is past the grid barrier
      }
      stamp(ph, 0);
      if (d.kind == AICAS_PH_ATTN) run_attention(d);
      else if (!kLean || lean_phase(d, nct)) run_matvec(d);
      else if (tid == 0) raise_error(s, kErrBadPhase);  // not a lean program: the launch aborts
      stamp(ph, 2);
    }
    // this warp is done with TMEM: the mover may free it
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.cdone);
    // the last CTA to finish moves the LL epoch base past this launch
    consumer_sync(kConsumerThreads);
    if (tid == 0) {
      __threadfence();
      if (atomicAdd(&s->exit_count, 1u) == (uint32_t)nct - 1) {
        s->exit_count = 0;
        s->epoch = epoch_base + (uint32_t)n_phases + 1;
        __threadfence();
      }
    }
  }
};

// kTrace: the traced variant records per-phase timestamps (a.trace); the
// plain one carries none of that code.  kLean: see Consumer.
template <bool kTrace, bool kLean>
__global__ void __launch_bounds__(kThreads, 1) decode_program_kernel(const __grid_constant__ ProgramArgs a) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
  // a request that produced its end-of-sequence token: nothing to do (every
  // thread reads the same word, so the whole grid returns before any barrier,
  // TMEM allocation or copy)
  if (a.state && *reinterpret_cast<const volatile int64_t*>(&a.state->done_step) != 0) return;
  // A scratch block that still holds a device error from an earlier launch
  // refuses the launch: nothing is read, written or advanced until the caller
  // zeroes the block (an aborted launch leaves its barriers, counters and
  // vectors in an unknown state).
  if (ld_volatile_int(&a.scratch->error) != 0) return;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], 1);
      mbar_init(&sm.cempty[i], kConsumerWarps);
    }
    for (int i = 0; i < kTmemSlots; ++i) {
      mbar_init(&sm.tfull[i], 1);
      mbar_init(&sm.tempty[i], kConsumerWarps);
    }
    for (int i = 0; i < (kKvSplit ? kKvStages : 0); ++i) {
      mbar_init(&sm.kvfull[i], 1);
      mbar_init(&sm.kvempty[i], kConsumerWarps);
    }
    mbar_init(&sm.cdone, kConsumerWarps);
    sm.ring_it = 0;
    mbar_fence_init();
  }
  if (threadIdx.x / 32 == kMoverWarp) tmem_alloc(&sm.tmem_base, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(&sm.tmem_base);
  StepIn in{};
  if (a.state) {
    const volatile AicasStepState* st = a.state;
    in.token = st->token;
    in.pos = st->cache_pos;
    in.rope[0] = st->rope[0];
    in.rope[1] = st->rope[1];
    in.rope[2] = st->rope[2];
    in.step = st->step;
  }
  const AicasPhase* P = a.phases ? a.phases : a.inl;
  const int warp = threadIdx.x / 32;
  if (warp == kMoverWarp) {
    run_mover(a, sm, in, tmem);
    return;
  }
  if (kKvSplit && warp == kKvWarp) {
    run_kv_producer(a, sm, in);
    return;
  }
  if (AICAS_L2_WARP && warp == kL2Warp) {
    run_l2_prefetcher(a, sm, in);
    return;
  }
  if (warp == 0) {
    run_producer<kTrace>(a, sm, in);
    return;
  }
  Consumer<kTrace, kLean> c{a, sm, in, a.scratch};
  c.tid = threadIdx.x - 32;
  c.w = warp - 1;
  c.lane = threadIdx.x & 31;
  c.tmem = tmem;
  c.rwt = ((c.w + 1) & 3) + 4 * (c.w >> 2);
  c.nct = gridDim.x;
  c.cta = blockIdx.x;
  const uint64_t now = ld_relaxed_u64(&a.scratch->bar_count);
  c.bar_base = now - now % (uint64_t)gridDim.x;
  c.epoch_base = *reinterpret_cast<volatile uint32_t*>(&a.scratch->epoch);
  c.run(P, a.n_phases);
}

}  // namespace aicas

// ===========================================================================
// Host side: launch + C ABI
// ===========================================================================
#include "aicas_decode.h"

namespace aicas {

static constexpr int kMaxDevices = 64;
static thread_local int g_last_cuda_error = 0;

static int cuda_fail(cudaError_t e) {
  g_last_cuda_error = (int)e;
  return AICAS_ERR_CUDA;
}
// Shared with the batched kernel's translation unit (hidden symbol).
int record_cuda_error(cudaError_t e) { return cuda_fail(e); }

// per-device setup, done once (idempotent: threads racing on a first call
// both do it; the flag is published after the values it guards)
static std::atomic<int> g_attr_done[kMaxDevices];
static std::atomic<int> g_num_sms[kMaxDevices];
static std::atomic<int> g_cooperative{1};  // aicas_set_cooperative_launch

static int device_setup(int* dev_out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return AICAS_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return AICAS_ERR_CUDA;
  if (!g_attr_done[dev].load(std::memory_order_acquire)) {
    const void* fns[4] = {reinterpret_cast<const void*>(decode_program_kernel<false, false>),
                          reinterpret_cast<const void*>(decode_program_kernel<true, false>),
                          reinterpret_cast<const void*>(decode_program_kernel<false, true>),
                          reinterpret_cast<const void*>(decode_program_kernel<true, true>)};
    for (const void* fn : fns) {
      cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(Smem));
      if (e != cudaSuccess) return cuda_fail(e);
      int per_sm = 0;
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kThreads, sizeof(Smem));
      if (e != cudaSuccess) return cuda_fail(e);
      if (per_sm < 1) return cuda_fail(cudaErrorLaunchOutOfResources);
    }
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return AICAS_ERR_CUDA;
    g_num_sms[dev].store(sms < AICAS_MAX_CTAS ? sms : AICAS_MAX_CTAS, std::memory_order_relaxed);
    g_attr_done[dev].store(1, std::memory_order_release);
  }
  *dev_out = dev;
  return AICAS_OK;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static int validate_phase(const AicasPhase& d) {
  switch (d.kind) {
    case AICAS_PH_GEMV:
    case AICAS_PH_GATEUP:
    case AICAS_PH_LMHEAD:
      if (d.n < 1 || d.k < 8 || d.k % 8 != 0 || d.k > AICAS_MAX_K) return AICAS_ERR_SHAPE;
      if (!d.w || !aligned16(d.w)) return AICAS_ERR_ALIGN;
      if (!d.x || !aligned16(d.x)) return AICAS_ERR_ALIGN;
      if ((d.flags & AICAS_F_X_ADD) && (!d.x2 || !aligned16(d.x2))) return AICAS_ERR_ALIGN;
      if ((d.flags & AICAS_F_NORM) && (!d.norm_w || !aligned16(d.norm_w))) return AICAS_ERR_ALIGN;
      if ((d.flags & AICAS_F_NORM) && d.k > 2048) return AICAS_ERR_SHAPE;  // norm prologue: k <= 2048
      if ((d.flags & (AICAS_F_X_EMBED | AICAS_F_RESID_EMBED)) && d.embed_rows < 1) return AICAS_ERR_ARG;
      if ((d.flags & AICAS_F_RESID) && !d.resid) return AICAS_ERR_ARG;
      if ((d.flags & AICAS_F_RESID_ADD) && !d.resid2) return AICAS_ERR_ARG;
      if ((d.flags & AICAS_F_BIAS) && !d.bias) return AICAS_ERR_ARG;
      if ((d.flags & AICAS_F_STORE_X) && (!d.x_out || !aligned16(d.x_out))) return AICAS_ERR_ALIGN;
      if (d.kind != AICAS_PH_LMHEAD && !d.out) return AICAS_ERR_ARG;
      if (d.kind == AICAS_PH_GATEUP && (d.flags & (AICAS_F_RESID | AICAS_F_BIAS))) return AICAS_ERR_ARG;
      if (d.kind == AICAS_PH_GATEUP && d.k > 2048) return AICAS_ERR_SHAPE;
      if ((d.flags & AICAS_F_KBLOCKED) && d.k % 2048 != 0) return AICAS_ERR_SHAPE;
      if ((d.flags & AICAS_F_LL_IN) && ((d.flags & (AICAS_F_X_ADD | AICAS_F_X_EMBED)) || d.x_src < 0))
        return AICAS_ERR_ARG;
      return AICAS_OK;
    case AICAS_PH_ATTN:
      if (d.kv_heads < 1 || d.kv_heads > AICAS_MAX_KV_HEADS || d.q_heads != 2 * d.kv_heads) return AICAS_ERR_SHAPE;
      if (d.max_len < 1) return AICAS_ERR_SHAPE;
      if (!d.k_cache || !d.v_cache || !aligned16(d.k_cache) || !aligned16(d.v_cache)) return AICAS_ERR_ALIGN;
      if (!d.x || !d.out) return AICAS_ERR_ARG;
      if (!(d.flags & AICAS_F_Q_READY) && (!d.norm_w || !d.norm_w2)) return AICAS_ERR_ARG;
      if (!(d.flags & AICAS_F_Q_READY) && (!aligned16(d.norm_w) || !aligned16(d.norm_w2))) return AICAS_ERR_ALIGN;
      if ((d.flags & AICAS_F_LL_IN) && ((d.flags & AICAS_F_Q_READY) || d.x_src < 0)) return AICAS_ERR_ARG;
      return AICAS_OK;
    default:
      return AICAS_ERR_ARG;
  }
}

static int launch_program(ProgramArgs& a, cudaStream_t stream, bool lean = false) {
  int dev;
  int rc = device_setup(&dev);
  if (rc) return rc;
  if (!a.scratch) return AICAS_ERR_ARG;
  if (a.n_phases < 1) return AICAS_ERR_ARG;
  // Attention needs the rotary table of a step state unless q is final.
  const AicasPhase* P = a.phases ? nullptr : a.inl;
  if (P) {
    for (int i = 0; i < a.n_phases; ++i) {
      if ((rc = validate_phase(P[i]))) return rc;
      if (P[i].kind == AICAS_PH_ATTN && !(P[i].flags & AICAS_F_Q_READY) && !a.state) return AICAS_ERR_ARG;
      if ((P[i].flags & (AICAS_F_X_EMBED | AICAS_F_RESID_EMBED)) && !a.state) return AICAS_ERR_ARG;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(g_num_sms[dev].load(std::memory_order_relaxed));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = sizeof(Smem);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = g_cooperative.load(std::memory_order_relaxed);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e;
  if (lean) e = a.trace ? cudaLaunchKernelEx(&cfg, decode_program_kernel<true, true>, a)
                        : cudaLaunchKernelEx(&cfg, decode_program_kernel<false, true>, a);
  else e = a.trace ? cudaLaunchKernelEx(&cfg, decode_program_kernel<true, false>, a)
                   : cudaLaunchKernelEx(&cfg, decode_program_kernel<false, false>, a);
  return e == cudaSuccess ? AICAS_OK : cuda_fail(e);
}


}  // namespace aicas

using namespace aicas;

extern "C" {

AICAS_API int aicas_abi_version(void) { return AICAS_ABI_VERSION; }

AICAS_API int aicas_last_cuda_error(void) { return g_last_cuda_error; }

AICAS_API const char* aicas_cuda_error_string(int err) { return cudaGetErrorString((cudaError_t)err); }

AICAS_API size_t aicas_scratch_bytes(void) { return sizeof(AicasScratch); }

AICAS_API int aicas_layout_signature(int64_t* out, int n) {
  const int64_t v[] = {(int64_t)sizeof(AicasPhase), (int64_t)sizeof(AicasStepState), (int64_t)sizeof(AicasScratch),
                       (int64_t)offsetof(AicasPhase, w), (int64_t)offsetof(AicasPhase, eps),
                       (int64_t)offsetof(AicasStepState, inv_freq), (int64_t)offsetof(AicasScratch, part),
                       (int64_t)offsetof(AicasScratch, error)};
  const int m = (int)(sizeof(v) / sizeof(v[0]));
  for (int i = 0; i < n && i < m; ++i) out[i] = v[i];
  return m;
}

AICAS_API int aicas_num_ctas(int device) {
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) return -AICAS_ERR_CUDA;
  if (device != prev && cudaSetDevice(device) != cudaSuccess) return -AICAS_ERR_CUDA;
  int dev = 0;
  const int rc = device_setup(&dev);
  if (device != prev) cudaSetDevice(prev);
  return rc ? -rc : g_num_sms[dev].load(std::memory_order_relaxed);
}

AICAS_API int aicas_set_cooperative_launch(int enable) {
  g_cooperative.store(enable ? 1 : 0, std::memory_order_relaxed);
  return AICAS_OK;
}

AICAS_API const char* aicas_error_string(int code) {
  switch (code) {
    case AICAS_OK: return "ok";
    case AICAS_ERR_ARG: return "invalid argument";
    case AICAS_ERR_SHAPE: return "unsupported shape";
    case AICAS_ERR_ALIGN: return "pointer or size not 16-byte aligned";
    case AICAS_ERR_CUDA: return "CUDA runtime error (launch or device query failed)";
    case AICAS_ERR_CAPACITY: return "request exceeds the fixed device scratch of the allocation-free entry point";
    case kErrBarrierTimeout: return "device: grid barrier timed out";
    case kErrFullTimeout: return "device: bulk copy did not complete in time";
    case kErrEmptyTimeout: return "device: ring stage was not released in time";
    case kErrDrainTimeout: return "device: in-flight copies did not drain in time";
    case kErrBadPhase: return "device: bad phase descriptor";
    case kErrBadInput: return "device: token id or cache position out of range";
    case kErrInputTimeout: return "device: an input vector did not arrive in time";
    case kErrTmemTimeout: return "device: a tensor-memory hand-off did not complete in time";
    default: return "unknown error";
  }
}

AICAS_API int aicas_validate_phases(const AicasPhase* phases, int n) {
  if (!phases || n < 1) return AICAS_ERR_ARG;
  for (int i = 0; i < n; ++i) {
    const int rc = validate_phase(phases[i]);
    if (rc) return rc;
  }
  return AICAS_OK;
}

AICAS_API int aicas_decode_program_f16(const AicasPhase* device_phases, int n_phases, AicasStepState* state,
                                       void* scratch, cudaStream_t stream) {
  if (!device_phases || n_phases < 1 || !state) return AICAS_ERR_ARG;
  ProgramArgs a;
  memset(&a, 0, sizeof(a));
  a.phases = device_phases;
  a.n_phases = n_phases;
  a.state = state;
  a.scratch = reinterpret_cast<AicasScratch*>(scratch);
  return launch_program(a, stream);
}

AICAS_API int aicas_decode_program_trace_f16(const AicasPhase* device_phases, int n_phases,
                                             AicasStepState* state, void* scratch, int64_t* trace,
                                             cudaStream_t stream) {
  if (!device_phases || n_phases < 1 || !state || !trace) return AICAS_ERR_ARG;
  ProgramArgs a;
  memset(&a, 0, sizeof(a));
  a.phases = device_phases;
  a.n_phases = n_phases;
  a.state = state;
  a.scratch = reinterpret_cast<AicasScratch*>(scratch);
  a.trace = trace;
  return launch_program(a, stream);
}

AICAS_API int aicas_lean_program_ok(const AicasPhase* phases, int n_phases, int num_ctas) {
  if (!phases || n_phases < 1 || num_ctas < 1) return AICAS_ERR_ARG;
  for (int i = 0; i < n_phases; ++i)
    if (!lean_phase(phases[i], num_ctas)) return AICAS_ERR_SHAPE;
  return AICAS_OK;
}

AICAS_API int aicas_decode_program_ex_f16(const AicasPhase* device_phases, int n_phases, AicasStepState* state,
                                          void* scratch, int64_t* trace, int flags, cudaStream_t stream) {
  if (!device_phases || n_phases < 1 || !state) return AICAS_ERR_ARG;
  if (flags & ~AICAS_PROGRAM_LEAN) return AICAS_ERR_ARG;
  ProgramArgs a;
  memset(&a, 0, sizeof(a));
  a.phases = device_phases;
  a.n_phases = n_phases;
  a.state = state;
  a.scratch = reinterpret_cast<AicasScratch*>(scratch);
  a.trace = trace;
  return launch_program(a, stream, (flags & AICAS_PROGRAM_LEAN) != 0);
}

}  // extern "C"
