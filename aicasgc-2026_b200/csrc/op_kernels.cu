// Single-op decode GEMVs for B200 (sm_100a): the kernels behind the
// reference-facing op entry points aicas_gemv_f16, aicas_rmsnorm_qkv_f16,
// aicas_post_attn_mlp_f16 and aicas_lm_head_argmax_f16.
//
// A single GEMV of the decode step moves 8-50 MB (the LM head 622 MB); at
// B200's bandwidth that is 1.3-8 us, so an op called on its own is bound by
// how fast one launch gets its weight bytes in flight, not by any on-chip
// pipeline.  These kernels are therefore ordinary launches (no cooperative
// grid, no tensor memory, no grid barrier): each CTA stages the input vector
// in shared memory (with the RMSNorm / residual-add prologue at HF's fp16
// rounding points, modeling_qwen3_vl.py:398-403), then every warp streams
// whole weight rows with 128-bit loads that bypass L1 and are marked
// evict-first in L2 (lane l takes columns 256 j + 8 l of each 2048-column
// chunk, so a warp's loads of one j are 512 contiguous bytes), issuing all
// loads of a row pass before its FMAs.  Products are exact fp16 x fp16 and the
// sums fp32 (PTX mixed-precision fma.rn.f32.f16), then one warp reduction per
// row.  The whole-step decode program keeps its persistent kernel
// (decode_program.cu); these serve callers that run one op at a time (the
// reference's per-layer chain of fused ops, optimized_layer.py:156-469).
//
// Reference interfaces replaced (file:line in the reference checkout):
//   nosplit_matvec_half        cuda_decode_gemv_ops/matvec.py:274-321
//   fused_rmsnorm_qkv_half     cuda_decode_gemv_ops/fused.py:71-105
//   fused_post_attn_mlp_softsync_half   cuda_decode_gemv_ops/fused.py:261-337
//   FastLmHead + torch.argmax  evaluation_wrapper.py:1227-1240, :952
#include <atomic>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "aicas_decode.h"
#include "aicas_device.cuh"

namespace aicas {

int record_cuda_error(cudaError_t e);  // decode_program.cu

namespace op {

constexpr int kWarps = 8;
constexpr int kThreads = 32 * kWarps;
constexpr int kChunk = 2048;             // columns per row pass chunk
constexpr int kVec = kChunk / 256;       // uint4 per lane per chunk
constexpr int kMaxGridArgmax = AICAS_MAX_CTAS;

enum Mode : int { kPlain = 0, kGateUp = 1, kArgmax = 2 };
enum Flag : int { kNorm = 1, kXAdd = 2, kResid = 4, kResidAdd = 8, kBias = 16 };

struct Args {
  const __half* x;       // input vector [k]
  const __half* x2;      // kXAdd: x := r16(x + x2)
  const __half* norm_w;  // kNorm: x := r16(w * r16(x * rsqrt(mean(x^2) + eps)))
  const __half* w;       // [n, k] row-major (kGateUp: [2n, k], gate rows first)
  const __half* bias;    // kBias: [n]
  const __half* resid;   // kResid: out := r16(resid + r16(acc))
  const __half* resid2;  // kResidAdd: resid := r16(resid + resid2)
  __half* out;           // [n] (kArgmax: the fp16 logits, may be null)
  int64_t* idx_out;      // kArgmax: first index of the maximum logit
  AicasScratch* scratch; // refusal word; kArgmax: per-CTA partials and the done counter
  int n, k, flags;
  float eps;
};

// 16 bytes of weights: read once, so no L1 allocation and first in line for
// L2 eviction.
__device__ __forceinline__ uint4 ld_stream(const __half* p, uint64_t policy) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p), "l"(policy));
  return v;
}

// The input vector into shared memory with the optional residual add and
// RMSNorm prologue (every CTA computes it; the vector is at most 12 KB).
__device__ __forceinline__ void stage_x(const Args& a, __half* xs, float* red) {
  const int k = a.k, tid = threadIdx.x;
  float ss = 0.f;
  for (int v = tid; v < k / 8; v += kThreads) {
    uint4 raw = __ldg(reinterpret_cast<const uint4*>(a.x) + v);
    __half2* hp = reinterpret_cast<__half2*>(&raw);
    if (a.flags & kXAdd) {
      const uint4 r2 = __ldg(reinterpret_cast<const uint4*>(a.x2) + v);
      const __half2* hq = reinterpret_cast<const __half2*>(&r2);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 fa = __half22float2(hp[q]), fb = __half22float2(hq[q]);
        hp[q] = __floats2half2_rn(fa.x + fb.x, fa.y + fb.y);
      }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = __half22float2(hp[q]);
      ss += f.x * f.x + f.y * f.y;
    }
    reinterpret_cast<uint4*>(xs)[v] = raw;
  }
  if (a.flags & kNorm) {
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < kWarps; ++i) tot += red[i];
    const float inv = rsqrtf(tot / (float)k + a.eps);
    for (int v = tid; v < k / 8; v += kThreads) {
      uint4 raw = reinterpret_cast<const uint4*>(xs)[v];
      const uint4 wr = __ldg(reinterpret_cast<const uint4*>(a.norm_w) + v);
      __half2* hp = reinterpret_cast<__half2*>(&raw);
      const __half2* wp = reinterpret_cast<const __half2*>(&wr);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __half22float2(hp[q]);
        const float2 g = __half22float2(wp[q]);
        hp[q] = __floats2half2_rn(g.x * r16(f.x * inv), g.y * r16(f.y * inv));
      }
      reinterpret_cast<uint4*>(xs)[v] = raw;
    }
  }
  __syncthreads();
}

// R rows (R = 2 when the reduction is one chunk, else 1) of C chunks each per
// warp pass.  kGateUp: the pair (gate row r, up row r + n).
template <int C, int kMode>
__global__ void __launch_bounds__(kThreads) gemv_op_kernel(const Args a) {
  extern __shared__ __align__(16) __half xs[];
  __shared__ float red[kWarps];
  __shared__ float bv_s[kWarps];
  __shared__ int bi_s[kWarps];
  // a scratch block that still holds a device error refuses the launch
  if (a.scratch && ld_volatile_int(&a.scratch->error) != 0) return;
  constexpr int R = (C == 1 || kMode == kGateUp) ? 2 : 1;
  constexpr int P = kMode == kGateUp ? 1 : R;  // output rows per pass
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = a.n, k = a.k;
  const uint64_t pol = l2_evict_first_policy();
  float best_v = -INFINITY;
  int best_i = 0x7fffffff;
  const int stride = gridDim.x * kWarps * P;
  int rows[R];
  bool ok[R];
  uint4 wv[R][C][kVec];
  // this warp's rows of a pass and their weight loads (no dependence on x)
  auto load_pass = [&](int base) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      rows[r] = kMode == kGateUp ? base + r * n : base + r;
      ok[r] = kMode == kGateUp ? true : rows[r] < n;
    }
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int c = 0; c < C; ++c)
#pragma unroll
        for (int j = 0; j < kVec; ++j) {
          const int col = c * kChunk + j * 256 + lane * 8;
          wv[r][c][j] = (ok[r] && col < k) ? ld_stream(a.w + (size_t)rows[r] * k + col, pol) : make_uint4(0, 0, 0, 0);
        }
  };
  // the lm_head pass loop is long: its first pass's weights are requested
  // before the input is staged, so the two round trips overlap (measured
  // slower for the short loops of the other projections, whose loads the
  // compiler then holds in registers all at once)
  constexpr bool kEarly = kMode == kArgmax;
  const int first = (blockIdx.x * kWarps + warp) * P;
  if (kEarly && first < n) load_pass(first);
  stage_x(a, xs, red);
  for (int base = first; base < n; base += stride) {
    if (!kEarly || base != first) load_pass(base);
    float s[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < C; ++c)
#pragma unroll
        for (int j = 0; j < kVec; ++j) {
          const int col = c * kChunk + j * 256 + lane * 8;
          const uint4 xv = col < k ? *reinterpret_cast<const uint4*>(xs + col) : make_uint4(0, 0, 0, 0);
          acc[j & 3] = dot8_f16(wv[r][c][j], xv, acc[j & 3]);
        }
      s[r] = warp_sum((acc[0] + acc[1]) + (acc[2] + acc[3]));
    }
    if (lane == 0) {
      if (kMode == kGateUp) {
        const float gq = r16(s[0]), uq = r16(s[1]);
        const float sl = r16(gq / (1.0f + expf(-gq)));
        a.out[base] = __float2half_rn(sl * uq);
      } else {
#pragma unroll
        for (int r = 0; r < R; ++r) {
          if (!ok[r]) continue;
          const int row = rows[r];
          float acc = s[r];
          if (a.flags & kBias) acc += __half2float(a.bias[row]);
          float y = r16(acc);
          if (a.flags & kResid) {
            float rv = __half2float(a.resid[row]);
            if (a.flags & kResidAdd) rv = r16(rv + __half2float(a.resid2[row]));
            y = r16(rv + y);
          }
          if (kMode == kArgmax) {
            if (a.out) a.out[row] = __float2half_rn(y);
            if (y > best_v) {  // this lane's rows ascend: strict > keeps the first maximum
              best_v = y;
              best_i = row;
            }
          } else {
            a.out[row] = __float2half_rn(y);
          }
        }
      }
    }
  }
  if (kMode != kArgmax) return;
  // warps -> CTA -> grid: larger value, or the same value at a smaller row
  if (lane == 0) {
    bv_s[warp] = best_v;
    bi_s[warp] = best_i;
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  float v = bv_s[0];
  int i = bi_s[0];
  for (int t = 1; t < kWarps; ++t)
    if (bv_s[t] > v || (bv_s[t] == v && bi_s[t] < i)) {
      v = bv_s[t];
      i = bi_s[t];
    }
  AicasScratch* s = a.scratch;
  s->am_val[blockIdx.x] = v;
  s->am_idx[blockIdx.x] = i;
  __threadfence();
  if (atomicAdd(&s->argmax_done, 1u) != gridDim.x - 1) return;
  __threadfence();
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int c = 0; c < (int)gridDim.x; ++c) {
    const float cv = __ldcg(&s->am_val[c]);
    const int ci = __ldcg(&s->am_idx[c]);
    if (cv > bv || (cv == bv && ci < bi)) {
      bv = cv;
      bi = ci;
    }
  }
  s->argmax_done = 0;
  *a.idx_out = bi;
}

// Plain GEMV with k > 2048 (C chunks): the chunks of a row go to C warps of
// the CTA (warp w: row slot w / C, chunk w % C; warps beyond (8 / C) C idle),
// so each warp has all 8 of its 16-byte loads per lane in flight at once
// (one warp holding all C chunks of a row keeps only part of them in flight:
// 10.9 us for down_proj [2048 x 6144]).  The C partial sums meet in shared
// memory and the row is finished in chunk order.
template <int C>
__global__ void __launch_bounds__(kThreads) gemv_ksplit_kernel(const Args a) {
  extern __shared__ __align__(16) __half xs[];
  __shared__ float red[kWarps];
  __shared__ float part[kWarps];
  if (a.scratch && ld_volatile_int(&a.scratch->error) != 0) return;
  constexpr int RS = kWarps / C;  // rows per CTA pass
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slot = warp / C, c = warp % C;
  const bool active = slot < RS;
  const int n = a.n, k = a.k;
  const uint64_t pol = l2_evict_first_policy();
  uint4 wv[kVec];
  auto load_row = [&](int row) {
#pragma unroll
    for (int j = 0; j < kVec; ++j) {
      const int col = c * kChunk + j * 256 + lane * 8;
      wv[j] = (active && row < n && col < k) ? ld_stream(a.w + (size_t)row * k + col, pol) : make_uint4(0, 0, 0, 0);
    }
  };
  // the first pass's weights are requested before the input is staged
  load_row(blockIdx.x * RS + slot);
  stage_x(a, xs, red);
  for (int base = blockIdx.x * RS; base < n; base += gridDim.x * RS) {  // the same trip count for the whole CTA
    const int row = base + slot;
    if (base != (int)blockIdx.x * RS) load_row(row);
    float sum = 0.f;
    if (active && row < n) {
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int j = 0; j < kVec; ++j) {
        const int col = c * kChunk + j * 256 + lane * 8;
        const uint4 xv = col < k ? *reinterpret_cast<const uint4*>(xs + col) : make_uint4(0, 0, 0, 0);
        acc[j & 3] = dot8_f16(wv[j], xv, acc[j & 3]);
      }
      sum = warp_sum((acc[0] + acc[1]) + (acc[2] + acc[3]));
    }
    if (lane == 0) part[warp] = sum;
    __syncthreads();
    if (active && c == 0 && lane == 0 && row < n) {
      float acc = part[warp];
#pragma unroll
      for (int cc = 1; cc < C; ++cc) acc += part[warp + cc];
      if (a.flags & kBias) acc += __half2float(a.bias[row]);
      float y = r16(acc);
      if (a.flags & kResid) {
        float rv = __half2float(a.resid[row]);
        if (a.flags & kResidAdd) rv = r16(rv + __half2float(a.resid2[row]));
        y = r16(rv + y);
      }
      a.out[row] = __float2half_rn(y);
    }
    __syncthreads();
  }
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static int sm_count() {
  static std::atomic<int> cached[64];  // 0: not read yet (a racing first read stores the same value)
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int v = cached[dev].load(std::memory_order_relaxed);
  if (!v) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v < 1) v = 148;
    cached[dev].store(v, std::memory_order_relaxed);
  }
  return v;
}

template <int C, int M>
static cudaError_t launch_c(const Args& a, int grid, cudaStream_t stream) {
  gemv_op_kernel<C, M><<<grid, kThreads, (size_t)a.k * 2, stream>>>(a);
  return cudaGetLastError();
}

template <int M>
static cudaError_t launch_m(const Args& a, int grid, int C, cudaStream_t stream) {
  if constexpr (M == kGateUp) {
    return launch_c<1, M>(a, grid, stream);  // gate_up: k <= 2048 (checked by run)
  } else {
    if (C == 1) return launch_c<1, M>(a, grid, stream);
    if (C == 2) return launch_c<2, M>(a, grid, stream);
    return launch_c<3, M>(a, grid, stream);
  }
}

// Checks the shapes and pointers of one launch and runs it.
static int run(Args a, int mode, cudaStream_t stream) {
  if (a.n < 1 || a.k < 8 || a.k % 8 != 0 || a.k > AICAS_MAX_K) return AICAS_ERR_SHAPE;
  if (!a.x || !a.w || !aligned16(a.x) || !aligned16(a.w)) return AICAS_ERR_ALIGN;
  if ((a.flags & kXAdd) && (!a.x2 || !aligned16(a.x2))) return AICAS_ERR_ALIGN;
  if ((a.flags & kNorm) && (!a.norm_w || !aligned16(a.norm_w))) return AICAS_ERR_ALIGN;
  if ((a.flags & kResid) && !a.resid) return AICAS_ERR_ARG;
  if ((a.flags & kResidAdd) && !a.resid2) return AICAS_ERR_ARG;
  if ((a.flags & kBias) && !a.bias) return AICAS_ERR_ARG;
  if (mode != kArgmax && !a.out) return AICAS_ERR_ARG;
  if (mode == kArgmax && (!a.idx_out || !a.scratch)) return AICAS_ERR_ARG;
  const int C = (a.k + kChunk - 1) / kChunk;
  if (mode == kGateUp && C != 1) return AICAS_ERR_SHAPE;
  if (mode == kPlain && C > 1) {  // k > 2048: chunks split over warps
    const int rs = kWarps / C;
    long grid = (a.n + rs - 1) / rs;
    const long cap = (long)sm_count() * 8;
    if (grid > cap) grid = cap;
    if (C == 2) gemv_ksplit_kernel<2><<<(int)grid, kThreads, (size_t)a.k * 2, stream>>>(a);
    else gemv_ksplit_kernel<3><<<(int)grid, kThreads, (size_t)a.k * 2, stream>>>(a);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? AICAS_OK : record_cuda_error(e);
  }
  const int per_pass = (mode == kGateUp) ? 1 : (C == 1 ? 2 : 1);
  const long passes = (a.n + per_pass - 1) / per_pass;
  long grid = (passes + kWarps - 1) / kWarps;
  // enough warps per SM to keep ~100 KB of weights in flight, never more
  // than the argmax partials hold
  const long cap = mode == kArgmax ? kMaxGridArgmax : (long)sm_count() * 8;
  if (grid > cap) grid = cap;
  cudaError_t e = mode == kPlain ? launch_m<kPlain>(a, (int)grid, C, stream)
                  : mode == kGateUp ? launch_m<kGateUp>(a, (int)grid, C, stream)
                                    : launch_m<kArgmax>(a, (int)grid, C, stream);
  return e == cudaSuccess ? AICAS_OK : record_cuda_error(e);
}

}  // namespace op
}  // namespace aicas

using aicas::op::Args;

extern "C" {

AICAS_API int aicas_gemv_f16(const void* x, const void* w, const void* bias, void* y, int64_t n, int64_t k,
                             void* scratch, aicas_stream_t stream) {
  if (n < 1 || n > (1 << 30) || k < 1 || k > AICAS_MAX_K) return AICAS_ERR_SHAPE;
  Args a = {};
  a.x = (const __half*)x;
  a.w = (const __half*)w;
  a.bias = (const __half*)bias;
  a.out = (__half*)y;
  a.scratch = (AicasScratch*)scratch;
  a.n = (int)n;
  a.k = (int)k;
  a.flags = bias ? aicas::op::kBias : 0;
  return aicas::op::run(a, aicas::op::kPlain, stream);
}

AICAS_API int aicas_rmsnorm_qkv_f16(const void* x, const void* norm_w, const void* w, const void* bias, void* y,
                                    int64_t n, int64_t k, float eps, void* scratch, aicas_stream_t stream) {
  if (n < 1 || n > (1 << 30) || k < 1 || k > AICAS_MAX_K) return AICAS_ERR_SHAPE;
  Args a = {};
  a.x = (const __half*)x;
  a.norm_w = (const __half*)norm_w;
  a.w = (const __half*)w;
  a.bias = (const __half*)bias;
  a.out = (__half*)y;
  a.scratch = (AicasScratch*)scratch;
  a.n = (int)n;
  a.k = (int)k;
  a.eps = eps;
  a.flags = aicas::op::kNorm | (bias ? aicas::op::kBias : 0);
  return aicas::op::run(a, aicas::op::kPlain, stream);
}

AICAS_API int aicas_post_attn_mlp_f16(const void* residual, const void* attn_out, const void* norm_w,
                                      const void* gate_up_w, const void* down_w, const void* bias, void* act_out,
                                      void* out, int64_t hidden, int64_t inter, float eps, void* scratch,
                                      aicas_stream_t stream) {
  if (hidden < 1 || inter < 1 || hidden > AICAS_MAX_K || inter > AICAS_MAX_K) return AICAS_ERR_SHAPE;
  using namespace aicas::op;
  // act = SiLU(W_gate x') * (W_up x') with x' = RMSNorm(r16(residual + attn_out))
  Args g = {};
  g.x = (const __half*)residual;
  g.x2 = (const __half*)attn_out;
  g.norm_w = (const __half*)norm_w;
  g.w = (const __half*)gate_up_w;
  g.out = (__half*)act_out;
  g.scratch = (AicasScratch*)scratch;
  g.n = (int)inter;
  g.k = (int)hidden;
  g.eps = eps;
  g.flags = kXAdd | kNorm;
  int rc = run(g, kGateUp, stream);
  if (rc) return rc;
  // out = r16(residual + attn_out) + W_down act (+ bias): a second launch on
  // the same stream, ordered after the first
  Args d = {};
  d.x = (const __half*)act_out;
  d.w = (const __half*)down_w;
  d.bias = (const __half*)bias;
  d.resid = (const __half*)residual;
  d.resid2 = (const __half*)attn_out;
  d.out = (__half*)out;
  d.scratch = (AicasScratch*)scratch;
  d.n = (int)hidden;
  d.k = (int)inter;
  d.flags = kResid | kResidAdd | (bias ? kBias : 0);
  return run(d, kPlain, stream);
}

AICAS_API int aicas_lm_head_argmax_f16(const void* x, const void* norm_w, const void* w, void* logits,
                                       void* token_out, int64_t vocab, int64_t k, float eps, void* scratch,
                                       aicas_stream_t stream) {
  if (vocab < 1 || vocab > (1 << 30) || k < 1 || k > AICAS_MAX_K) return AICAS_ERR_SHAPE;
  if (!token_out || !scratch) return AICAS_ERR_ARG;
  Args a = {};
  a.x = (const __half*)x;
  a.norm_w = (const __half*)norm_w;
  a.w = (const __half*)w;
  a.out = (__half*)logits;
  a.idx_out = (int64_t*)token_out;
  a.scratch = (AicasScratch*)scratch;
  a.n = (int)vocab;
  a.k = (int)k;
  a.eps = eps;
  a.flags = norm_w ? aicas::op::kNorm : 0;
  return aicas::op::run(a, aicas::op::kArgmax, stream);
}

}  // extern "C"
