// Decode attention as a single op for B200 (sm_100a): the kernel behind
// aicas_decode_attn_splitkv_f16 and its allocation-free variant, which replace
// the reference's `decode_attn_v4_cta_qhead_splitkv_fused`
// (cuda_decode_attention.py:489-558; kernel decode_attention_v4_kernel.cu).
//
// One query token, GQA 2:1 (two query heads per KV head), head dim 128, a
// static cache [kv_heads][max_len][128] fp16 whose valid length (cache
// position + 1) is read on the device, so the call can sit in a CUDA graph.
// The op moves 4 KB of K/V per cache slot; at 8192 slots that is 33.5 MB, ~5
// us of HBM time, so the launch must put the whole cache in flight at once:
//
//   * grid (16 splits, kv heads): each CTA takes one contiguous chunk of slots
//     of one KV head (chunk = the valid length over the splits, rounded up to
//     128 slots; CTAs past the last chunk return at once), so both query heads
//     of a KV head read its K/V once;
//   * 8 warps per CTA take 16 slots each in turn (all 16 slots' K and V loads
//     issued first), as two groups of 8: lane (slot pi = lane / 4, quarter
//     qc = lane % 4) dots its 32 dims of K (four 16-byte loads, evict-first)
//     with both queries held in registers (exact fp16 products, fp32 sums),
//     two shuffles finish each score; an online softmax in fp32 per warp and
//     head; P V with lane l owning dims 4l .. 4l + 3 (one 8-byte V load per
//     slot);
//   * the 8 warps' states merge in shared memory into the CTA's partial
//     (running max, sum, unnormalised acc); with one chunk the CTA writes the
//     output directly, otherwise it stores its partial in the scratch block
//     and the last CTA of the KV head (arrival counter, fences on both sides)
//     merges all partials in split order -- deterministic -- and resets the
//     counter.
//
// Scratch use (AicasScratch, zeroed by the caller before its first use): the
// error word (a launch on a block holding an error does nothing; a cache
// position outside [0, max_len) raises kErrBadInput and writes nothing), the
// `part` array reinterpreted as fp32 partials [kv head][split][2][130] and,
// after them, one arrival counter per KV head, which returns to zero at the
// end of every call.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stddef.h>
#include <stdint.h>

#include <atomic>

#include "aicas_decode.h"
#include "aicas_device.cuh"

namespace aicas {

int record_cuda_error(cudaError_t e);  // decode_program.cu

namespace attn {

constexpr int kHD = AICAS_HEAD_DIM;
constexpr int kWarps = 8;
constexpr int kThreads = 32 * kWarps;
#ifndef AICAS_ATTN_ALIGN
#define AICAS_ATTN_ALIGN 128
#endif
// Chunk granularity (cache slots; 128 = one pass of the 8 warps) and splits per
// KV head.  Measured on B200 (bench.py --op attention, us per call at L = 128 /
// 1024 / 4096 / 8192): 64 splits of 64-slot units 7.8 / 10.1 / 21.5 / 24.6;
// 32 of 64: 7.0 / 8.2 / 14.0 / 18.5; 16 of 128: 4.6 / 7.5 / 10.7 / 14.9;
// 8 of 128: 4.5 / 7.4 / 13.5 / 21.5.  Each further split adds a partial that
// the last CTA must read back, so fewer, longer chunks win until the grid
// stops covering the SMs.
constexpr int kSlotAlign = AICAS_ATTN_ALIGN;
#ifndef AICAS_ATTN_SPLITS
#define AICAS_ATTN_SPLITS 16
#endif
constexpr int kMaxSplits = AICAS_ATTN_SPLITS;
constexpr int kPartFloats = 2 + kHD;    // running max, sum, acc[128]
static_assert(kMaxSplits <= AICAS_MAX_SPLITS, "partials must fit the scratch block");
static_assert((size_t)AICAS_MAX_KV_HEADS * kMaxSplits * 2 * kPartFloats * 4 + AICAS_MAX_KV_HEADS * 4 <=
                  sizeof(((AicasScratch*)0)->part),
              "partials and counters must fit the scratch block's part array");

__device__ __forceinline__ float* partial(AicasScratch* s, int h, int split, int g) {
  return reinterpret_cast<float*>(&s->part[0][0][0][0]) + ((size_t)(h * kMaxSplits + split) * 2 + g) * kPartFloats;
}
__device__ __forceinline__ uint32_t* counter(AicasScratch* s, int h) {
  return reinterpret_cast<uint32_t*>(reinterpret_cast<float*>(&s->part[0][0][0][0]) +
                                     (size_t)AICAS_MAX_KV_HEADS * kMaxSplits * 2 * kPartFloats) + h;
}

__device__ __forceinline__ uint4 ld_stream_u4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ uint2 ld_stream_u2(const void* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}

struct Smem {
  float wm[kWarps][2], wl[kWarps][2];
  float wacc[kWarps][2][kHD];
  float pm[2][kMaxSplits], pl[2][kMaxSplits];  // the merging CTA's copy of every split's (max, sum)
  uint32_t last;
};

#ifndef AICAS_ATTN_MINB
#define AICAS_ATTN_MINB 1
#endif
__global__ void __launch_bounds__(kThreads, AICAS_ATTN_MINB) decode_attention_kernel(const __half* __restrict__ q,
                                                                    const __half* __restrict__ kc,
                                                                    const __half* __restrict__ vc,
                                                                    const int64_t* __restrict__ pos_ptr, float scale,
                                                                    __half* __restrict__ out, int max_len,
                                                                    AicasScratch* s) {
  __shared__ Smem sm;
  const int split = blockIdx.x, h = blockIdx.y, nsplit = gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // a scratch block that still holds an error refuses the launch (every CTA
  // reads the same words, so every CTA returns alike)
  if (ld_volatile_int(&s->error) != 0) return;
  const int64_t pos = *pos_ptr;
  if (pos < 0 || pos >= max_len) {
    if (split == 0 && h == 0 && threadIdx.x == 0) raise_error(s, kErrBadInput);
    return;
  }
  const int valid = (int)pos + 1;
  const int per = (valid + nsplit - 1) / nsplit;
  const int chunk = ((per + kSlotAlign - 1) / kSlotAlign) * kSlotAlign;
  const int n_used = (valid + chunk - 1) / chunk;
  if (split >= n_used) return;
  const int p_begin = split * chunk, p_end = min(valid, p_begin + chunk);

  const int pi = lane >> 2, qc = lane & 3;
  // lane (slot pi, quarter qc) owns dims 32 j + 8 qc .. + 7 for j = 0..3, so
  // one load instruction of the 4 lanes of a slot covers 64 contiguous bytes
  // of its K row (two whole sectors); both queries' same dims in registers
  uint4 qv[2][4];
#pragma unroll
  for (int g = 0; g < 2; ++g)
#pragma unroll
    for (int j = 0; j < 4; ++j)
      qv[g][j] = __ldg(reinterpret_cast<const uint4*>(q + (size_t)(2 * h + g) * kHD + 32 * j + 8 * qc));
  const __half* kh = kc + (size_t)h * max_len * kHD;
  const __half* vh = vc + (size_t)h * max_len * kHD;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f}, acc[2][4] = {};
  // each warp takes 16 slots (two groups of 8) per pass, all their K and V
  // loads issued before any is used
  for (int p0 = p_begin + 16 * warp; p0 < p_end; p0 += 16 * kWarps) {
    uint4 kv[2][4];
    uint2 vv[2][8];
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      const int p = p0 + 8 * b + pi;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        kv[b][j] = p < p_end ? ld_stream_u4(kh + (size_t)p * kHD + 32 * j + 8 * qc) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int pv = p0 + 8 * b + i;
        vv[b][i] = pv < p_end ? ld_stream_u2(vh + (size_t)pv * kHD + lane * 4) : make_uint2(0, 0);
      }
    }
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      const int pb = p0 + 8 * b;
      if (pb >= p_end) break;  // warp-uniform
      const bool ok = pb + pi < p_end;
      float sc[2] = {0.f, 0.f};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        sc[0] = dot8_f16(kv[b][j], qv[0][j], sc[0]);
        sc[1] = dot8_f16(kv[b][j], qv[1][j], sc[1]);
      }
      float pr[2];
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        float v = sc[g];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        v = ok ? v * scale : -INFINITY;
        float mx = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float mn = fmaxf(m[g], mx);  // finite: the group's first slot is valid
        pr[g] = ok ? expf(v - mn) : 0.f;
        float ps = pr[g];
        ps += __shfl_xor_sync(0xffffffffu, ps, 4);
        ps += __shfl_xor_sync(0xffffffffu, ps, 8);
        ps += __shfl_xor_sync(0xffffffffu, ps, 16);
        const float corr = expf(m[g] - mn);
        l[g] = l[g] * corr + ps;
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[g][e] *= corr;
        m[g] = mn;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float p0g = __shfl_sync(0xffffffffu, pr[0], 4 * i), p1g = __shfl_sync(0xffffffffu, pr[1], 4 * i);
        const __half2* v2 = reinterpret_cast<const __half2*>(&vv[b][i]);
        const float vf[4] = {__low2float(v2[0]), __high2float(v2[0]), __low2float(v2[1]), __high2float(v2[1])};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          acc[0][e] += p0g * vf[e];
          acc[1][e] += p1g * vf[e];
        }
      }
    }
  }
  // the 8 warps' states -> this CTA's partial
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      sm.wm[warp][g] = m[g];
      sm.wl[warp][g] = l[g];
    }
  }
#pragma unroll
  for (int g = 0; g < 2; ++g)
#pragma unroll
    for (int e = 0; e < 4; ++e) sm.wacc[warp][g][lane * 4 + e] = acc[g][e];
  __syncthreads();
  const int g = threadIdx.x / kHD, t = threadIdx.x % kHD;  // 256 threads: (query head, dim)
  float M = -INFINITY;
#pragma unroll
  for (int i = 0; i < kWarps; ++i) M = fmaxf(M, sm.wm[i][g]);
  float L = 0.f, A = 0.f;
#pragma unroll
  for (int i = 0; i < kWarps; ++i) {
    const float mi = sm.wm[i][g];
    if (mi != -INFINITY) {  // a warp with no slot of this chunk contributes nothing
      const float f = expf(mi - M);
      L += sm.wl[i][g] * f;
      A += sm.wacc[i][g][t] * f;
    }
  }
  if (n_used == 1) {
    out[(size_t)(2 * h + g) * kHD + t] = __float2half_rn(A / L);
    return;
  }
  float* pp = partial(s, h, split, g);
  if (t == 0) {
    pp[0] = M;
    pp[1] = L;
  }
  pp[2 + t] = A;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) sm.last = atomicAdd(counter(s, h), 1u) == (uint32_t)(n_used - 1);
  __syncthreads();
  if (!sm.last) return;
  __threadfence();  // every other CTA's partial (fenced before its arrival) is visible
  for (int j = threadIdx.x; j < 2 * n_used; j += kThreads) {
    const int gg = j / n_used, i = j % n_used;
    const float* pj = partial(s, h, i, gg);
    sm.pm[gg][i] = __ldcg(pj);
    sm.pl[gg][i] = __ldcg(pj + 1);
  }
  __syncthreads();
  float Mx = -INFINITY;
  for (int i = 0; i < n_used; ++i) Mx = fmaxf(Mx, sm.pm[g][i]);
  // splits in order (deterministic); eight accumulator loads in flight
  float Ls = 0.f, As = 0.f;
#pragma unroll 8
  for (int i = 0; i < n_used; ++i) {
    const float f = expf(sm.pm[g][i] - Mx);
    Ls += sm.pl[g][i] * f;
    As += __ldcg(partial(s, h, i, g) + 2 + t) * f;
  }
  out[(size_t)(2 * h + g) * kHD + t] = __float2half_rn(As / Ls);
  if (threadIdx.x == 0) *counter(s, h) = 0u;  // ready for the next call
}

static int check_shapes(const void* q, const void* k_cache, const void* v_cache, const void* cache_position,
                        const void* out, int64_t q_heads, int64_t kv_heads, int64_t max_len) {
  if (max_len < 1 || max_len > (1 << 30)) return AICAS_ERR_SHAPE;
  if (!q || !k_cache || !v_cache || !cache_position || !out) return AICAS_ERR_ARG;
  if (kv_heads < 1 || q_heads != 2 * kv_heads) return AICAS_ERR_SHAPE;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!al16(q) || !al16(k_cache) || !al16(v_cache) || (reinterpret_cast<uintptr_t>(out) & 1u)) return AICAS_ERR_ALIGN;
  return AICAS_OK;
}

static int launch(const void* q, const void* k_cache, const void* v_cache, const void* cache_position, float scale,
                  void* out, int64_t kv_heads, int64_t max_len, AicasScratch* s, cudaStream_t stream) {
  const int64_t want = (max_len + kSlotAlign - 1) / kSlotAlign;
  const int splits = (int)(want < kMaxSplits ? want : kMaxSplits);
  decode_attention_kernel<<<dim3(splits, (unsigned)kv_heads), kThreads, 0, stream>>>(
      (const __half*)q, (const __half*)k_cache, (const __half*)v_cache, (const int64_t*)cache_position, scale,
      (__half*)out, (int)max_len, s);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? AICAS_OK : record_cuda_error(e);
}

// The allocation-free variant's scratch: one file-scope __device__ block per
// device (zero at module load, held until the process exits).  Host code must
// not hand the array's name to a kernel: on the host it only stands for the
// device symbol, so its address is looked up once per device with
// cudaGetSymbolAddress.  Atomic: host threads may call concurrently (two that
// both look it up store the same address).  A device reset invalidates it;
// the library must then be reloaded.
static __device__ __align__(256) AicasScratch g_noalloc_scratch;
constexpr int kMaxDevices = 64;
static std::atomic<AicasScratch*> g_noalloc_scratch_ptr[kMaxDevices];

}  // namespace attn
}  // namespace aicas

using namespace aicas;
using namespace aicas::attn;

extern "C" {

AICAS_API int aicas_decode_attn_splitkv_f16(const void* q, const void* k_cache, const void* v_cache,
                                            const void* cache_position, float scale, void* out, int64_t q_heads,
                                            int64_t kv_heads, int64_t max_len, void* scratch, cudaStream_t stream) {
  int rc = check_shapes(q, k_cache, v_cache, cache_position, out, q_heads, kv_heads, max_len);
  if (rc) return rc;
  if (kv_heads > AICAS_MAX_KV_HEADS) return AICAS_ERR_SHAPE;
  if (!scratch) return AICAS_ERR_ARG;
  return launch(q, k_cache, v_cache, cache_position, scale, out, kv_heads, max_len,
                reinterpret_cast<AicasScratch*>(scratch), stream);
}

AICAS_API int aicas_decode_attn_splitkv_f16_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                                   const void* cache_position, float scale, void* out,
                                                   int64_t q_heads, int64_t kv_heads, int64_t max_len,
                                                   int32_t* status, cudaStream_t stream) {
  if (max_len < 1 || max_len > (1 << 30)) return AICAS_ERR_SHAPE;
  if (!q || !k_cache || !v_cache || !cache_position || !out) return AICAS_ERR_ARG;
  // the fixed block holds partials for at most AICAS_MAX_KV_HEADS KV heads (GQA 2:1)
  if (kv_heads < 1 || kv_heads > AICAS_MAX_KV_HEADS || q_heads != 2 * kv_heads) return AICAS_ERR_CAPACITY;
  int rc = check_shapes(q, k_cache, v_cache, cache_position, out, q_heads, kv_heads, max_len);
  if (rc) return rc;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return record_cuda_error(e);
  if (dev < 0 || dev >= kMaxDevices) return AICAS_ERR_CUDA;
  AicasScratch* scr = g_noalloc_scratch_ptr[dev].load(std::memory_order_acquire);
  if (!scr) {  // first call on this device: resolve the block's device address
    e = cudaGetSymbolAddress(reinterpret_cast<void**>(&scr), g_noalloc_scratch);
    if (e != cudaSuccess) return record_cuda_error(e);
    g_noalloc_scratch_ptr[dev].store(scr, std::memory_order_release);
  }
  // the block keeps the previous call's contents: clear its error and abort
  // words (the arrival counters return to zero at the end of every call)
  e = cudaMemsetAsync(&scr->error, 0, 2 * sizeof(int32_t), stream);
  if (e != cudaSuccess) return record_cuda_error(e);
  rc = launch(q, k_cache, v_cache, cache_position, scale, out, kv_heads, max_len, scr, stream);
  if (rc) return rc;
  if (status) {  // the call's device-side error code, for callers that cannot read the block
    e = cudaMemcpyAsync(status, &scr->error, sizeof(int32_t), cudaMemcpyDeviceToDevice, stream);
    if (e != cudaSuccess) return record_cuda_error(e);
  }
  return AICAS_OK;
}

}  // extern "C"
