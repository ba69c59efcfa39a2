// Prompt prefill kernels for B200 (sm_100a): everything of the one-pass
// prefill except the projection GEMMs (which are plain dense fp16 GEMMs with
// fp32 accumulation, run by the library).  The reference prefills with HF's
// forward (evaluation_wrapper.py:1836-1958, optimized_layer.py:471-619); the
// arithmetic here keeps HF's fp16 rounding points
// (transformers modeling_qwen3_vl.py: RMSNorm :398-403, interleaved MRoPE
// :352-386, rotary :124-128 / :427-431, SiLU-gated MLP :519-521, residual
// adds :553-563) so the prefilled cache continues seamlessly into the decode
// kernels.
//
//   add_rmsnorm      h := r16(h + delta); x := RMSNorm(h) (one CTA per row)
//   qk_norm_rope_kv  per-head q/k RMSNorm + interleaved MRoPE from the 3-axis
//                    positions; q to a [P, Hq, 128] buffer, k and v into the
//                    static cache at slots start .. start + P - 1, and (when
//                    given) q, k and v once more into the tensor-core
//                    attention's tile workspace (prefill_attn_tc.cu)
//   silu_mul         act := r16(r16(silu(gate)) * up) of the fused gate_up rows
// The causal attention is in prefill_attn_tc.cu.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "aicas_decode.h"
#include "aicas_device.cuh"

namespace aicas {

int record_cuda_error(cudaError_t e);  // decode_program.cu

namespace pf {

constexpr int kHD = AICAS_HEAD_DIM;

// ---------------------------------------------------------------- add + RMSNorm
// One CTA (256 threads) per row of `cols` (<= 8192, a multiple of 8) values.
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(const __half* __restrict__ h, const __half* __restrict__ delta,
                                                          const __half* __restrict__ norm_w, __half* __restrict__ h_out,
                                                          __half* __restrict__ x_out, int cols, float eps) {
  __shared__ float red[8];
  const size_t base = (size_t)blockIdx.x * cols;
  const int nv = cols / 8;
  constexpr int kMaxV = 4;  // uint4 per thread (cols <= 8192)
  uint4 v[kMaxV], wv[kMaxV];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxV; ++i) {  // the norm weights load while the sum of squares is reduced
    const int c = threadIdx.x + i * 256;
    if (c < nv) wv[i] = __ldg(reinterpret_cast<const uint4*>(norm_w) + c);
  }
#pragma unroll
  for (int i = 0; i < kMaxV; ++i) {
    const int c = threadIdx.x + i * 256;
    if (c < nv) {
      v[i] = __ldg(reinterpret_cast<const uint4*>(h + base) + c);
      __half2* hp = reinterpret_cast<__half2*>(&v[i]);
      if (delta) {
        const uint4 dv = __ldg(reinterpret_cast<const uint4*>(delta + base) + c);
        const __half2* dp = reinterpret_cast<const __half2*>(&dv);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 a = __half22float2(hp[q]), b = __half22float2(dp[q]);
          hp[q] = __floats2half2_rn(a.x + b.x, a.y + b.y);
        }
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __half22float2(hp[q]);
        ss += f.x * f.x + f.y * f.y;
      }
      if (h_out) reinterpret_cast<uint4*>(h_out + base)[c] = v[i];
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float inv = rsqrtf(tot / (float)cols + eps);
#pragma unroll
  for (int i = 0; i < kMaxV; ++i) {
    const int c = threadIdx.x + i * 256;
    if (c < nv) {
      __half2* hp = reinterpret_cast<__half2*>(&v[i]);
      const __half2* wp = reinterpret_cast<const __half2*>(&wv[i]);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __half22float2(hp[q]);
        const float2 g = __half22float2(wp[q]);
        hp[q] = __floats2half2_rn(g.x * r16(f.x * inv), g.y * r16(f.y * inv));
      }
      reinterpret_cast<uint4*>(x_out + base)[c] = v[i];
    }
  }
}

// ---------------------------------------------------------------- q/k norm + MRoPE + KV write
// One CTA (8 warps) per token; warp w takes head tasks w, w + 8, ...: tasks
// [0, Hq) the query heads, [Hq, Hq + Hkv) the key heads, then the value heads.
// Lane l holds dims 4l .. 4l + 3; rotate_half's partner (d +- 64) is lane l ^ 16.
__global__ void __launch_bounds__(256) qk_norm_rope_kv_kernel(
    const __half* __restrict__ qkv, const __half* __restrict__ qn_w, const __half* __restrict__ kn_w,
    const int64_t* __restrict__ pos3, const float* __restrict__ inv_freq, int sec1, int sec2, __half* __restrict__ q_out,
    __half* __restrict__ k_cache, __half* __restrict__ v_cache, int P, int start, int max_len, int hq, int hkv, float eps,
    __half* __restrict__ tiles, int r128, int l128) {
  __shared__ float tcos[kHD / 2], tsin[kHD / 2];
  const int t = blockIdx.x, w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = hq + 2 * hkv;  // qkv row length in heads
  const size_t slot = (size_t)start + t;
  constexpr int kTasks = 4;  // head tasks of a warp whose loads are in flight together
  uint2 raw[kTasks], nwr[kTasks];
  // the warp's tasks task0, task0 + 8, ..., task0 + 8 (kTasks - 1): every
  // load issued before any is used
  auto load_round = [&](int task0) {
#pragma unroll
    for (int j = 0; j < kTasks; ++j) {
      const int task = task0 + 8 * j;
      raw[j] = task < row ? *reinterpret_cast<const uint2*>(qkv + ((size_t)t * row + task) * kHD + lane * 4)
                          : make_uint2(0, 0);
      nwr[j] = task < hq + hkv ? __ldg(reinterpret_cast<const uint2*>(task < hq ? qn_w : kn_w) + lane)
                               : make_uint2(0, 0);
    }
  };
  load_round(w);  // in flight while the rotary table is built
  // the token's 64 rotary frequencies, once per CTA: frequency i takes axis 1
  // (h) when i % 3 == 1 and i < 3 sec1, axis 2 (w) when i % 3 == 2 and
  // i < 3 sec2, else axis 0 (t); cos / sin in fp32, rounded to fp16
  if (threadIdx.x < kHD / 2) {
    const int i = threadIdx.x;
    int axis = 0;
    if (i % 3 == 1 && i < 3 * sec1) axis = 1;
    else if (i % 3 == 2 && i < 3 * sec2) axis = 2;
    float sv, cv;
    sincosf(inv_freq[i] * (float)pos3[(size_t)axis * P + t], &sv, &cv);
    tcos[i] = r16(cv);
    tsin[i] = r16(sv);
  }
  __syncthreads();
  // this lane's 4 frequencies (dims 4 lane .. 4 lane + 3, frequency d mod 64)
  float cs[4], sn[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    cs[e] = tcos[(lane * 4 + e) & 63];
    sn[e] = tsin[(lane * 4 + e) & 63];
  }
  for (int task0 = w; task0 < row; task0 += 8 * kTasks) {
    if (task0 != w) load_round(task0);
#pragma unroll
    for (int j = 0; j < kTasks; ++j) {
      const int task = task0 + 8 * j;
      if (task >= row) break;
      const __half2* hp = reinterpret_cast<const __half2*>(&raw[j]);
      float v[4] = {__low2float(hp[0]), __high2float(hp[0]), __low2float(hp[1]), __high2float(hp[1])};
      if (task < hq + hkv) {
        const __half2* nh = reinterpret_cast<const __half2*>(&nwr[j]);
        const float nwf[4] = {__low2float(nh[0]), __high2float(nh[0]), __low2float(nh[1]), __high2float(nh[1])};
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e) ss += v[e] * v[e];
        const float inv = rsqrtf(warp_sum(ss) / (float)kHD + eps);
        float xn[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) xn[e] = r16(nwf[e] * r16(v[e] * inv));
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float p = __shfl_xor_sync(0xffffffffu, xn[e], 16);
          const float rot = lane < 16 ? -p : p;
          v[e] = r16(r16(xn[e] * cs[e]) + r16(rot * sn[e]));
        }
      }
      const __half2 o[2] = {__floats2half2_rn(v[0], v[1]), __floats2half2_rn(v[2], v[3])};
      const uint2 ov = *reinterpret_cast<const uint2*>(o);
      __half* dst;
      if (task < hq) dst = q_out ? q_out + ((size_t)t * hq + task) * kHD : nullptr;
      else if (task < hq + hkv) dst = k_cache + ((size_t)(task - hq) * max_len + slot) * kHD;
      else dst = v_cache + ((size_t)(task - hq - hkv) * max_len + slot) * kHD;
      if (dst) *reinterpret_cast<uint2*>(dst + lane * 4) = ov;
      if (tiles) {  // the attention's KV tile layout: row p, dims 8 blk .. at (p/8) 1024 + blk 64 + (p%8) 8
        const int p = task < hq ? t : (int)slot;
        const size_t base = task < hq ? (size_t)task * r128 * kHD
                                      : (size_t)hq * r128 * kHD + (size_t)(task - hq) * l128 * kHD;
        *reinterpret_cast<uint2*>(tiles + base + (p >> 3) * 1024 + (lane >> 1) * 64 + (p & 7) * 8 + (lane & 1) * 4) =
            ov;
      }
    }
  }
}

// ---------------------------------------------------------------- SiLU * up
__global__ void __launch_bounds__(256) silu_mul_kernel(const __half* __restrict__ gu, __half* __restrict__ act, int P,
                                                       int inter) {
  // CTA (x, y): row y, 8-column groups 256 x + thread
  const int n8 = inter / 8, c = blockIdx.x * blockDim.x + threadIdx.x;
  const size_t r = blockIdx.y;
  if (c >= n8) return;
  const uint4 g = __ldg(reinterpret_cast<const uint4*>(gu + r * 2 * inter) + c);
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(gu + r * 2 * inter + inter) + c);
  const __half2* gp = reinterpret_cast<const __half2*>(&g);
  const __half2* up = reinterpret_cast<const __half2*>(&u);
  uint4 o;
  __half2* op = reinterpret_cast<__half2*>(&o);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float2 gf = __half22float2(gp[q]), uf = __half22float2(up[q]);
    // SiLU in fp32 (the fast exp: its error is far below the fp16 rounding that follows)
    const float s0 = r16(gf.x / (1.0f + __expf(-gf.x))), s1 = r16(gf.y / (1.0f + __expf(-gf.y)));
    op[q] = __floats2half2_rn(s0 * uf.x, s1 * uf.y);
  }
  reinterpret_cast<uint4*>(act + r * inter)[c] = o;
}

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace pf
}  // namespace aicas

using namespace aicas::pf;

extern "C" {

AICAS_API int aicas_prefill_add_rmsnorm_f16(const void* h, const void* delta, const void* norm_w, void* h_out,
                                            void* x_out, int64_t rows, int64_t cols, float eps,
                                            aicas_stream_t stream) {
  if (rows < 1 || rows > (1 << 24) || cols < 8 || cols % 8 != 0 || cols > 8192) return AICAS_ERR_SHAPE;
  if (!h || !norm_w || !x_out || !al16(h) || !al16(norm_w) || !al16(x_out) || (delta && !al16(delta)) ||
      (h_out && !al16(h_out)))
    return AICAS_ERR_ALIGN;
  add_rmsnorm_kernel<<<(unsigned)rows, 256, 0, stream>>>((const __half*)h, (const __half*)delta,
                                                         (const __half*)norm_w, (__half*)h_out, (__half*)x_out,
                                                         (int)cols, eps);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? AICAS_OK : aicas::record_cuda_error(e);
}

AICAS_API int aicas_prefill_qk_norm_rope_kv_f16(const void* qkv, const void* q_norm_w, const void* k_norm_w,
                                                const void* pos3, const void* inv_freq, int sec1, int sec2,
                                                void* q_out, void* k_cache, void* v_cache, int64_t rows,
                                                int64_t start, int64_t max_len, int64_t q_heads, int64_t kv_heads,
                                                float eps, void* tiles, aicas_stream_t stream) {
  if (rows < 1 || start < 0 || start + rows > max_len || max_len > (1 << 30)) return AICAS_ERR_SHAPE;
  if (kv_heads < 1 || q_heads < kv_heads || q_heads % kv_heads != 0 || q_heads + 2 * kv_heads > 4096)
    return AICAS_ERR_SHAPE;
  if (!qkv || !q_norm_w || !k_norm_w || !pos3 || !inv_freq || (!q_out && !tiles) || !k_cache || !v_cache)
    return AICAS_ERR_ARG;
  if (tiles && (start != 0 || !al16(tiles))) return AICAS_ERR_ARG;  // the tiles cover slots [0, rows)
  const int64_t r128 = (rows + 127) / 128 * 128;
  qk_norm_rope_kv_kernel<<<(unsigned)rows, 256, 0, stream>>>(
      (const __half*)qkv, (const __half*)q_norm_w, (const __half*)k_norm_w, (const int64_t*)pos3,
      (const float*)inv_freq, sec1, sec2, (__half*)q_out, (__half*)k_cache, (__half*)v_cache, (int)rows, (int)start,
      (int)max_len, (int)q_heads, (int)kv_heads, eps, (__half*)tiles, (int)r128, (int)r128);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? AICAS_OK : aicas::record_cuda_error(e);
}

AICAS_API int aicas_prefill_silu_mul_f16(const void* gate_up, void* act, int64_t rows, int64_t inter,
                                         aicas_stream_t stream) {
  if (rows < 1 || inter < 8 || inter % 8 != 0) return AICAS_ERR_SHAPE;
  if (!gate_up || !act || !al16(gate_up) || !al16(act)) return AICAS_ERR_ALIGN;
  if (rows > 65535) return AICAS_ERR_SHAPE;  // one grid row per token
  const dim3 grid((unsigned)((inter / 8 + 255) / 256), (unsigned)rows);
  silu_mul_kernel<<<grid, 256, 0, stream>>>((const __half*)gate_up, (__half*)act, (int)rows, (int)inter);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? AICAS_OK : aicas::record_cuda_error(e);
}

}  // extern "C"
