// Causal GQA prefill attention on the 5th-generation tensor cores (B200,
// sm_100a): S = Q K^T and O += P V as tcgen05.mma (M = N = 128, K = 16, fp16
// operands, fp32 accumulators in tensor memory), flash-style online softmax.
//
// Input layouts.  The entry point first copies q [rows, q_heads, 128] and the
// cache slots [0, start + rows) of k / v [kv_heads, max_len, 128] (HF
// StaticLayer order) into a workspace in the KV tile layout: for each head,
// slot (or query) p, dim d at element (p / 8) * 1024 + (d / 8) * 64 + (p % 8) *
// 8 + d % 8, zero beyond the last row.  128 consecutive rows are then one
// contiguous 32 KB piece that a single bulk copy lands as a tcgen05 operand:
// K-major for Q (A) and K (B) (8-row x 16-byte core matrices, LBO 128 B to
// the next 8 dims, SBO 2 KB to the next 8 rows) and MN-major for V (B of
// O += P V: LBO 2 KB along the keys, SBO 128 B along the dims).
//
// One CTA per (128-query tile, query head), 6 warps:
//   warp 0     producer: the Q tile once, then K / V blocks of 128 keys into
//              a 2-stage ring (cp.async.bulk, mbarrier completion);
//   warp 1     TMEM owner and MMA issuer: S_j = Q K_j^T into one of two S
//              buffers (128 columns each), then O += P_{j-1} V_{j-1} once the
//              softmax has written P_{j-1} (two P buffers), so each S product
//              and each P V product overlaps a block of softmax;
//   warps 2-5  softmax, one query row per thread (TMEM lane = row): the row's
//              128 scores, causal mask, row maximum, P = exp2(s - m) as fp16
//              into shared memory (the A operand of O += P V), running fp32 sum.
//              O is rescaled in TMEM only when the row maximum grows by more
//              than 2^8 over the reference the running sums use, so P stays
//              <= 256 and most blocks skip the rescale; the last step divides
//              the O row by its sum and stores fp16.
// Every wait is bounded (2 s); a wait that gives up records a timeout and the
// warp carries on without it, so the kernel always ends.  TMEM is freed after
// every MMA the CTA issued has completed.
//
// Reference behaviour (file:line in the reference checkout): the prefill the
// reference runs through HF's eager attention (optimized_layer.py:471-619,
// prefill_forward_no_mask; modeling_qwen3_vl.py eager_attention_forward):
// softmax(Q K^T * scale + causal mask) V per query head, KV head = head / 2.
#include <atomic>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "aicas_decode.h"
#include "aicas_device.cuh"

namespace aicas {

int record_cuda_error(cudaError_t e);  // decode_program.cu

namespace pfa {

constexpr int kHD = AICAS_HEAD_DIM;           // 128
constexpr int kBM = 128;                      // queries per CTA
constexpr int kBN = 128;                      // keys per block
constexpr int kTile = kBM * kHD * 2;          // 32 KB: 128 rows of one head
constexpr int kThreads = 192;                 // producer, MMA issuer, 4 softmax warps
constexpr int kTmemCols = 512;                // S double buffer (2 x 128) + O (128)
constexpr uint32_t kOCol = 256;
// D fp32 (bits 4-5), A / B fp16, N >> 3 at bit 17, M >> 4 at bit 24; PV: B MN-major (bit 16)
constexpr uint32_t kIdescQK = (1u << 4) | ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
constexpr uint32_t kIdescPV = (1u << 4) | (1u << 16) | ((uint32_t)(kHD >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
constexpr float kLog2e = 1.4426950408889634f;  // log2(e): exp(x) = 2^(x log2 e)
constexpr float kRescaleLog2 = 8.f;

struct Smem {
  uint8_t q[kTile];
  uint8_t k[2][kTile];
  uint8_t v[2][kTile];
  uint8_t p[2][kTile];  // P [128 queries][128 keys] fp16, K-major A operand (blocks alternate)
  uint64_t q_full, kv_full[2], kv_empty[2], s_full[2], s_empty[2], p_full, pv_done[2], mma_done;
  uint32_t tmem_base;
  int abort;  // a wait of this CTA gave up: later waits return at once
};
constexpr int kSmemBytes = (int)sizeof(Smem);
static_assert(kSmemBytes <= 227 * 1024, "one CTA's shared memory");

__device__ int g_timeouts;  // waits that gave up (none expected)

// Bounded wait for phase `parity` of `bar`; false after 2 s (recorded) or
// once another wait of the CTA has given up.
__device__ __forceinline__ bool wait_b(Smem& sm, uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 0) {
      if (*reinterpret_cast<volatile int*>(&sm.abort)) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        atomicAdd(&g_timeouts, 1);
        *reinterpret_cast<volatile int*>(&sm.abort) = 1;
        return false;
      }
    }
  }
}

// The same without the abort word, for the copies and MMAs this CTA issued
// (they complete in microseconds either way): none is still writing shared
// or tensor memory when the CTA exits.
__device__ __forceinline__ void wait_done(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return;
    if ((it & 63u) == 63u && globaltimer_ns() - t0 > kWaitLimitNs) {
      atomicAdd(&g_timeouts, 1);
      return;
    }
  }
}

__device__ __forceinline__ void umma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                     uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 2^x with the hardware's approximate exponent (2^-inf = +0).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// {lo, hi} rounded to fp16 in one 32-bit word.
__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Element offset of row p, dims [8 blk, 8 blk + 8) in the KV tile layout.
__host__ __device__ __forceinline__ uint32_t tile_off(int p, int blk) {
  return (uint32_t)((p >> 3) * 1024 + blk * 64 + (p & 7) * 8);
}

// q rows and cache slots [0, start + rows) -> workspace tiles (zeros beyond
// them): piece i = 8 dims of one row of one head.
__global__ void __launch_bounds__(256) relayout_kernel(const __half* __restrict__ q, const __half* __restrict__ kc,
                                                       const __half* __restrict__ vc, __half* __restrict__ ws,
                                                       int rows, int start, int hq, int hkv, int max_len, int r128,
                                                       int l128) {
  const int nq = hq * r128 * 16, nk = hkv * l128 * 16;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < nq + 2 * nk; i += gridDim.x * blockDim.x) {
    uint4 val = make_uint4(0, 0, 0, 0);
    __half* dst;
    const int blk = i & 15;
    if (i < nq) {
      const int rr = i >> 4, t = rr % r128, hh = rr / r128;
      if (t < rows) val = *reinterpret_cast<const uint4*>(q + ((size_t)t * hq + hh) * kHD + blk * 8);
      dst = ws + (size_t)hh * r128 * kHD + tile_off(t, blk);
    } else {
      const bool isv = i - nq >= nk;
      const int rr = (i - nq - (isv ? nk : 0)) >> 4, p = rr % l128, kh = rr / l128;
      if (p < start + rows)
        val = *reinterpret_cast<const uint4*>((isv ? vc : kc) + ((size_t)kh * max_len + p) * kHD + blk * 8);
      dst = ws + (size_t)hq * r128 * kHD + (isv ? (size_t)hkv * l128 * kHD : 0) + (size_t)kh * l128 * kHD +
            tile_off(p, blk);
    }
    *reinterpret_cast<uint4*>(dst) = val;
  }
}

__global__ void __launch_bounds__(kThreads, 1) attn_tc_kernel(const uint8_t* __restrict__ ws, __half* __restrict__ out,
                                                             int rows, int start, int hq, int hkv, int r128, int l128,
                                                             float scale) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hh = blockIdx.y, kh = hh / (hq / hkv);
  const int q0 = blockIdx.x * kBM;
  const int kv_end = min(start + rows, start + q0 + kBM);  // keys any of this tile's queries sees
  const int nblk = (kv_end + kBN - 1) / kBN;
  const uint8_t* qsrc = ws + ((size_t)hh * r128 + q0) * kHD * 2;
  const uint8_t* kbase = ws + ((size_t)hq * r128 + (size_t)kh * l128) * kHD * 2;
  const uint8_t* vbase = kbase + (size_t)hkv * l128 * kHD * 2;
  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.kv_full[i], 1);
      mbar_init(&sm.kv_empty[i], 1);
      mbar_init(&sm.s_full[i], 1);
      mbar_init(&sm.s_empty[i], 4);
    }
    mbar_init(&sm.p_full, 4);
    mbar_init(&sm.pv_done[0], 1);
    mbar_init(&sm.pv_done[1], 1);
    mbar_init(&sm.mma_done, 1);
    sm.abort = 0;
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc(&sm.tmem_base, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(&sm.tmem_base);

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_q = l2_evict_first_policy(), pol_kv = l2_evict_last_policy();
      mbar_arrive_expect_tx(&sm.q_full, kTile);
      bulk_g2s(sm.q, qsrc, kTile, &sm.q_full, pol_q);
      int issued = 0;
      for (int j = 0; j < nblk; ++j) {
        const int st = j & 1;
        if (j >= 2 && !wait_b(sm, &sm.kv_empty[st], ((j >> 1) - 1) & 1)) break;
        mbar_arrive_expect_tx(&sm.kv_full[st], 2 * kTile);
        bulk_g2s(sm.k[st], kbase + (size_t)j * kBN * kHD * 2, kTile, &sm.kv_full[st], pol_kv);
        bulk_g2s(sm.v[st], vbase + (size_t)j * kBN * kHD * 2, kTile, &sm.kv_full[st], pol_kv);
        issued = j + 1;
      }
      // the last copies land before the CTA may exit
      for (int j = max(0, issued - 2); j < issued; ++j) wait_done(&sm.kv_full[j & 1], (j >> 1) & 1);
      wait_done(&sm.q_full, 0);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t q_s = smem_addr(sm.q);
      wait_b(sm, &sm.q_full, 0);
      auto issue_pv = [&](int i) {
        wait_b(sm, &sm.p_full, i & 1);
        tc_fence_after();
        const uint32_t v_s = smem_addr(sm.v[i & 1]), p_s = smem_addr(sm.p[i & 1]);
#pragma unroll
        for (int ks = 0; ks < kBN / 16; ++ks)
          umma(tmem + kOCol, smem_desc_kmajor(p_s + 256 * ks, 128, 2048), smem_desc_kmajor(v_s + 4096 * ks, 2048, 128),
               kIdescPV, (i > 0 || ks > 0) ? 1u : 0u);
        tcgen05_commit(&sm.pv_done[i & 1]);
        tcgen05_commit(&sm.kv_empty[i & 1]);
      };
      for (int j = 0; j < nblk; ++j) {
        const int st = j & 1;
        wait_b(sm, &sm.kv_full[st], (j >> 1) & 1);
        if (j >= 2) wait_b(sm, &sm.s_empty[st], ((j >> 1) - 1) & 1);
        tc_fence_after();
        const uint32_t k_s = smem_addr(sm.k[st]);
#pragma unroll
        for (int ks = 0; ks < kHD / 16; ++ks)
          umma(tmem + st * kBN, smem_desc_kmajor(q_s + 256 * ks, 128, 2048), smem_desc_kmajor(k_s + 256 * ks, 128, 2048),
               kIdescQK, ks > 0 ? 1u : 0u);
        tcgen05_commit(&sm.s_full[st]);
        if (j >= 1) issue_pv(j - 1);
      }
      issue_pv(nblk - 1);
      // every MMA of this CTA has completed before TMEM may be freed
      tcgen05_commit(&sm.mma_done);
      wait_done(&sm.mma_done, 0);
    }
    __syncwarp();
  } else {
    // softmax: warp 2..5 -> TMEM lane quarter 2, 3, 0, 1; thread = query row r.
    // Rows past `rows` see zero queries (finite scores) and are not stored.
    const int quarter = warp & 3, r = 32 * quarter + lane;
    const int qrow = q0 + r, qpos = start + qrow;
    const bool live = qrow < rows;
    const uint32_t lane_base = (uint32_t)(32 * quarter) << 16;
    const float sl2 = scale * kLog2e;  // scores -> log2 units
    float m_ref = -INFINITY;           // reference maximum (raw score units) of l and O
    float l = 0.f;
    const int prow = (r >> 3) * 2048 + (r & 7) * 16;  // row r's bytes in a P buffer
    for (int j = 0; j < nblk; ++j) {
      const int sb = j & 1;
      wait_b(sm, &sm.s_full[sb], (j >> 1) & 1);
      tc_fence_after();
      float x[kBN];
      {
        uint32_t v[4][32];
#pragma unroll
        for (int c = 0; c < kBN / 32; ++c) tmem_ld_32x32b_x32(tmem + lane_base + sb * kBN + c * 32, v[c]);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < kBN / 32; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e) x[c * 32 + e] = __uint_as_float(v[c][e]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.s_empty[sb]);
      // causal mask: keys kb + c > qpos (only blocks that reach past this row)
      const int lim = qpos - j * kBN;
      if (lim < kBN - 1) {
#pragma unroll
        for (int c = 0; c < kBN; ++c) x[c] = c <= lim ? x[c] : -INFINITY;
      }
      float mx = x[0];
#pragma unroll
      for (int c = 1; c < kBN; ++c) mx = fmaxf(mx, x[c]);
      // P buffer j % 2 is free once O += P_{j-2} V_{j-2} has completed (its
      // commit barrier has completed at most that phase: P_j is not written)
      if (j >= 2) wait_b(sm, &sm.pv_done[j & 1], ((j >> 1) - 1) & 1);
      tc_fence_after();
      if (mx != -INFINITY && (m_ref == -INFINITY || (mx - m_ref) * sl2 > kRescaleLog2)) {
        if (m_ref != -INFINITY) {  // O holds blocks 0..j-1 at reference m_ref: rescale once P_{j-1} V_{j-1} is in
          wait_b(sm, &sm.pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1);
          tc_fence_after();
          const float f = ex2_approx((m_ref - mx) * sl2);
          l *= f;
#pragma unroll
          for (int c = 0; c < kHD / 32; ++c) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(tmem + lane_base + kOCol + c * 32, v);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * f);
            tmem_st_32x32b_x32(tmem + lane_base + kOCol + c * 32, v);
          }
          tmem_wait_st();
        }
        m_ref = mx;
      }
      // P = 2^((s - m) sl2) (masked keys: 2^-inf = 0), fp16 into row r of the
      // A operand; the running sum takes the fp32 values
      const float mofs = m_ref == -INFINITY ? 0.f : -m_ref * sl2;
      float ls[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int cb = 0; cb < kBN / 8; ++cb) {
        uint32_t pk[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float a = ex2_approx(fmaf(x[cb * 8 + 2 * e], sl2, mofs));
          const float b = ex2_approx(fmaf(x[cb * 8 + 2 * e + 1], sl2, mofs));
          ls[e] += a + b;
          pk[e] = pack_half2(a, b);
        }
        *reinterpret_cast<uint4*>(sm.p[j & 1] + prow + cb * 128) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
      l += (ls[0] + ls[1]) + (ls[2] + ls[3]);
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.p_full);
    }
    wait_b(sm, &sm.pv_done[(nblk - 1) & 1], ((nblk - 1) >> 1) & 1);  // in order: every O += P V is in
    tc_fence_after();
    const float inv = live && l > 0.f ? 1.f / l : 0.f;
    __half* orow = out + ((size_t)(live ? qrow : 0) * hq + hh) * kHD;
#pragma unroll
    for (int c = 0; c < kHD / 32; ++c) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(tmem + lane_base + kOCol + c * 32, v);
      tmem_wait_ld();
      if (live) {
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
          uint4 pk;
          __half2* ph = reinterpret_cast<__half2*>(&pk);
#pragma unroll
          for (int u = 0; u < 4; ++u)
            ph[u] = __floats2half2_rn(__uint_as_float(v[e + 2 * u]) * inv, __uint_as_float(v[e + 2 * u + 1]) * inv);
          *reinterpret_cast<uint4*>(orow + c * 32 + e) = pk;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

__host__ __forceinline__ int64_t round128(int64_t x) { return (x + 127) / 128 * 128; }

}  // namespace pfa
}  // namespace aicas

using namespace aicas::pfa;

AICAS_API size_t aicas_prefill_attention_workspace_bytes(int64_t rows, int64_t start, int64_t q_heads,
                                                         int64_t kv_heads) {
  if (rows < 1 || start < 0 || q_heads < 1 || kv_heads < 1) return 0;
  return (size_t)(q_heads * round128(rows) + 2 * kv_heads * round128(start + rows)) * kHD * 2;
}

static int attn_launch(const uint8_t* tiles, void* out, int64_t rows, int64_t start, int64_t q_heads,
                       int64_t kv_heads, float scale, aicas_stream_t stream) {
  static std::atomic<bool> attr_done[64];  // per device, set once (idempotent)
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return aicas::record_cuda_error(e);
  if (dev < 0 || dev >= 64) return AICAS_ERR_CUDA;
  if (!attr_done[dev].load(std::memory_order_acquire)) {
    e = cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return aicas::record_cuda_error(e);
    attr_done[dev].store(true, std::memory_order_release);
  }
  const int64_t r128 = round128(rows), l128 = round128(start + rows);
  const dim3 grid((unsigned)(r128 / kBM), (unsigned)q_heads);
  attn_tc_kernel<<<grid, kThreads, kSmemBytes, stream>>>(tiles, (__half*)out, (int)rows, (int)start, (int)q_heads,
                                                         (int)kv_heads, (int)r128, (int)l128, scale);
  e = cudaGetLastError();
  return e == cudaSuccess ? AICAS_OK : aicas::record_cuda_error(e);
}

static int attn_shape_ok(int64_t rows, int64_t start, int64_t q_heads, int64_t kv_heads) {
  if (rows < 1 || start < 0 || rows + start > (1 << 30)) return AICAS_ERR_SHAPE;
  if (kv_heads < 1 || q_heads < kv_heads || q_heads % kv_heads != 0 || q_heads > 65535) return AICAS_ERR_SHAPE;
  if ((q_heads * round128(rows) + 2 * kv_heads * round128(start + rows)) * 16 > 0x7fffffffLL)
    return AICAS_ERR_SHAPE;  // piece indices in int32
  return AICAS_OK;
}

static bool al16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

AICAS_API int aicas_prefill_attention_f16(const void* q, const void* k_cache, const void* v_cache, void* out,
                                          int64_t rows, int64_t start, int64_t q_heads, int64_t kv_heads,
                                          int64_t max_len, float scale, void* workspace, aicas_stream_t stream) {
  int rc = attn_shape_ok(rows, start, q_heads, kv_heads);
  if (rc) return rc;
  if (start + rows > max_len || max_len > (1 << 30)) return AICAS_ERR_SHAPE;
  if (!q || !k_cache || !v_cache || !out || !workspace || !al16(q) || !al16(k_cache) || !al16(v_cache) ||
      !al16(out) || !al16(workspace))
    return AICAS_ERR_ALIGN;
  const int64_t r128 = round128(rows), l128 = round128(start + rows);
  const int64_t pieces = (q_heads * r128 + 2 * kv_heads * l128) * 16;
  const unsigned rgrid = (unsigned)((pieces + 255) / 256 < 148 * 16 ? (pieces + 255) / 256 : 148 * 16);
  relayout_kernel<<<rgrid, 256, 0, stream>>>((const __half*)q, (const __half*)k_cache, (const __half*)v_cache,
                                            (__half*)workspace, (int)rows, (int)start, (int)q_heads, (int)kv_heads,
                                            (int)max_len, (int)r128, (int)l128);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return aicas::record_cuda_error(e);
  return attn_launch((const uint8_t*)workspace, out, rows, start, q_heads, kv_heads, scale, stream);
}

AICAS_API int aicas_prefill_attention_tiles_f16(const void* tiles, void* out, int64_t rows, int64_t start,
                                                int64_t q_heads, int64_t kv_heads, float scale,
                                                aicas_stream_t stream) {
  int rc = attn_shape_ok(rows, start, q_heads, kv_heads);
  if (rc) return rc;
  if (!tiles || !out || !al16(tiles) || !al16(out)) return AICAS_ERR_ALIGN;
  return attn_launch((const uint8_t*)tiles, out, rows, start, q_heads, kv_heads, scale, stream);
}

AICAS_API int aicas_prefill_attention_timeouts(void) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_timeouts, sizeof(int)) != cudaSuccess) return -1;
  return v;
}
