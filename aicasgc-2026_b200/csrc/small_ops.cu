// Fused q/k RMSNorm + rotary embedding + static-KV write for one decode token
// (B200, sm_100a).  Drop-in for the reference's
// `fused_q_rope_kv_cache_update` (cuda_decode_small_ops.py:136-225, kernel
// cuda_extensions/decode_small_ops_kernel.cu:115-186).
//
// One CTA per KV head, three 128-thread groups: query heads 2h and 2h+1 and
// key head h (whose group also copies v).  Each group normalises its head
// with HF's rounding points (modeling_qwen3_vl.py:398-403), rotates it with
// the given fp16 cos/sin (modeling_qwen3_vl.py:124-128, 427-431) and stores
// it.  The whole op moves ~10 KB: it is launch-latency bound, so it is one
// small launch; the decode engine fuses the same math into its attention
// phase instead.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "aicas_decode.h"
#include "aicas_device.cuh"

namespace aicas {

constexpr int kHeadDim = 128;

__global__ void __launch_bounds__(3 * kHeadDim) qk_norm_rope_kvwrite_kernel(
    const __half* __restrict__ q, const __half* __restrict__ k, const __half* __restrict__ v,
    const __half* __restrict__ qw, const __half* __restrict__ kw, const __half* __restrict__ cosv,
    const __half* __restrict__ sinv, __half* __restrict__ q_out, __half* __restrict__ kc, __half* __restrict__ vc,
    const int64_t* __restrict__ cache_position, float eps, int max_len, int* __restrict__ status) {
  __shared__ float red[3][4];
  __shared__ float tmp[3][kHeadDim];
  const int h = blockIdx.x;
  const int grp = threadIdx.x / kHeadDim, t = threadIdx.x % kHeadDim;
  const int lane = threadIdx.x & 31, wig = (threadIdx.x / 32) % 4;
  const int64_t pos = *cache_position;
  const bool pos_ok = pos >= 0 && pos < max_len;
  const __half* src = grp < 2 ? q + (size_t)(2 * h + grp) * kHeadDim : k + (size_t)h * kHeadDim;
  const __half* nw = grp < 2 ? qw : kw;
  const float x = __half2float(src[t]);
  const float ss = warp_sum(x * x);
  if (lane == 0) red[grp][wig] = ss;
  __syncthreads();
  const float tot = red[grp][0] + red[grp][1] + red[grp][2] + red[grp][3];
  const float n = r16(x * rsqrtf(tot / (float)kHeadDim + eps));
  const float xn = r16(__half2float(nw[t]) * n);
  tmp[grp][t] = xn;
  __syncthreads();
  const float rot = t < kHeadDim / 2 ? -tmp[grp][t + kHeadDim / 2] : tmp[grp][t - kHeadDim / 2];
  const __half y = __float2half_rn(r16(r16(xn * __half2float(cosv[t])) + r16(rot * __half2float(sinv[t]))));
  if (grp < 2) {
    q_out[(size_t)(2 * h + grp) * kHeadDim + t] = y;
  } else if (pos_ok) {
    const size_t slot = ((size_t)h * max_len + pos) * kHeadDim + t;
    kc[slot] = y;
    vc[slot] = v[(size_t)h * kHeadDim + t];
  }
  if (!pos_ok && threadIdx.x == 0 && blockIdx.x == 0 && status) *status = kErrBadInput;
}

}  // namespace aicas

extern "C" AICAS_API int aicas_qk_norm_mrope_kvwrite_f16(const void* q, const void* k, const void* v,
                                                         const void* q_norm_w, const void* k_norm_w,
                                                         const void* cos, const void* sin, void* q_out,
                                                         void* k_cache, void* v_cache, const void* cache_position,
                                                         float eps, int64_t q_heads, int64_t kv_heads,
                                                         int64_t max_len, aicas_stream_t stream) {
  if (kv_heads < 1 || kv_heads > 64 || q_heads != 2 * kv_heads || max_len < 1 || max_len > (1 << 30))
    return AICAS_ERR_SHAPE;
  if (!q || !k || !v || !q_norm_w || !k_norm_w || !cos || !sin || !q_out || !k_cache || !v_cache ||
      !cache_position)
    return AICAS_ERR_ARG;
  aicas::qk_norm_rope_kvwrite_kernel<<<(unsigned)kv_heads, 3 * aicas::kHeadDim, 0, stream>>>(
      (const __half*)q, (const __half*)k, (const __half*)v, (const __half*)q_norm_w, (const __half*)k_norm_w,
      (const __half*)cos, (const __half*)sin, (__half*)q_out, (__half*)k_cache, (__half*)v_cache,
      (const int64_t*)cache_position, eps, (int)max_len, nullptr);
  return cudaGetLastError() == cudaSuccess ? AICAS_OK : AICAS_ERR_CUDA;
}
