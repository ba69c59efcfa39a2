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
//                    static cache at slots start .. start + P - 1
//   silu_mul         act := r16(r16(silu(gate)) * up) of the fused gate_up rows
//   attention        causal GQA attention over the cache (flash form: 64-query
//                    tiles, 64-key blocks, online softmax in fp32, Q K^T and
//                    P V on the tensor cores with mma.sync m16n8k16, fp16
//                    operands and fp32 accumulation; P is rounded to fp16 for
//                    its product with V, the one rounding point HF's fp32
//                    softmax does not have)
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
    __half* __restrict__ k_cache, __half* __restrict__ v_cache, int P, int start, int max_len, int hq, int hkv, float eps) {
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
      __half* dst;
      if (task < hq) dst = q_out + ((size_t)t * hq + task) * kHD;
      else if (task < hq + hkv) dst = k_cache + ((size_t)(task - hq) * max_len + slot) * kHD;
      else dst = v_cache + ((size_t)(task - hq - hkv) * max_len + slot) * kHD;
      *reinterpret_cast<uint2*>(dst + lane * 4) = *reinterpret_cast<const uint2*>(o);
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

// ---------------------------------------------------------------- causal flash attention
constexpr int kBQ = 64;   // queries per CTA (4 warps x 16)
constexpr int kBK = 64;   // keys per block
constexpr int kAttnThreads = 128;
constexpr int kAttnSmem = 5 * 64 * 256;  // Q + two K/V stages (80 KB)

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;  // 0: fill the 16 bytes with zeros
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Shared-memory tile of 64 rows x 128 halves (256 B per row, 16 chunks of 16
// B); chunk c of row r is stored at chunk c ^ (r & 7) so ldmatrix reads of 8
// rows hit 8 different bank groups.
__device__ __forceinline__ uint32_t sw_off(int r, int c) { return (uint32_t)(r * 256 + ((c ^ (r & 7)) << 4)); }

// 64 rows of a [rows][128] fp16 matrix (row stride `ld` halves) into a
// swizzled tile; rows at or beyond `rows_valid` read as zeros.
__device__ __forceinline__ void load_tile(uint32_t tile, const __half* src, size_t ld, int rows_valid) {
  for (int i = threadIdx.x; i < 64 * 16; i += kAttnThreads) {
    const int r = i >> 4, c = i & 15;
    const bool ok = r < rows_valid;
    cp_async16(tile + sw_off(r, c), ok ? (const void*)(src + (size_t)r * ld + c * 8) : (const void*)src, ok);
  }
}

// out[t][head][:] = softmax(q K^T * scale) V over cache slots [0, start + t]
// for query t (row-major q [P][Hq][128]); grid (ceil(P / 64), Hq).
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const __half* __restrict__ q, const __half* __restrict__ kc,
                                                               const __half* __restrict__ vc, __half* __restrict__ out,
                                                               int P, int start, int hq, int hkv, int max_len,
                                                               float scale) {
  // Q | K, V of key block 2i | K, V of key block 2i + 1: the next block's
  // copies are in flight while this one is computed
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sq = smem_addr(smem);
  // the tiles with the most key blocks first (causal: the last query tile)
  const int qb = gridDim.x - 1 - blockIdx.x, head = blockIdx.y, kvh = head / (hq / hkv);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = qb * kBQ;
  const int qrows = min(kBQ, P - q0);
  const __half* kbase = kc + (size_t)kvh * max_len * kHD;
  const __half* vbase = vc + (size_t)kvh * max_len * kHD;
  load_tile(sq, q + ((size_t)q0 * hq + head) * kHD, (size_t)hq * kHD, qrows);
  asm volatile("cp.async.commit_group;" ::: "memory");
  // the last key any query of this tile sees
  const int kend = start + q0 + qrows;  // exclusive
  const int nkb = (kend + kBK - 1) / kBK;
  // Q fragments of this warp's 16 rows, all 8 k-steps of 16 dims
  uint32_t qa[8][4];
  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  const float sl2 = scale * 1.4426950408889634f;  // scores in log2 units
  const int g = lane >> 2, tig = lane & 3;
  const int qi0 = start + q0 + warp * 16 + g;  // absolute slots of this thread's rows g, g + 8
  auto issue = [&](int kb) {
    const int k0 = kb * kBK;
    const uint32_t sk = sq + (1 + 2 * (kb & 1)) * 64 * 256, sv = sk + 64 * 256;
    load_tile(sk, kbase + (size_t)k0 * kHD, kHD, min(kBK, kend - k0));
    load_tile(sv, vbase + (size_t)k0 * kHD, kHD, min(kBK, kend - k0));
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  issue(0);
  for (int kb = 0; kb < nkb; ++kb) {
    const int k0 = kb * kBK;
    const uint32_t sk = sq + (1 + 2 * (kb & 1)) * 64 * 256, sv = sk + 64 * 256;
    if (kb + 1 < nkb) {
      issue(kb + 1);  // its buffer was last read in iteration kb - 1 (barrier at that iteration's end)
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      cp_async_wait_all();
    }
    __syncthreads();
    if (kb == 0) {
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        // A 16x16: matrices (rows 0-7, k 0-7), (rows 8-15, k 0-7), (rows 0-7, k 8-15), (rows 8-15, k 8-15)
        const int r = warp * 16 + (lane & 15), c = ks * 2 + (lane >> 4);
        ldsm_x4(sq + sw_off(r, c), qa[ks]);
      }
    }
    // S = Q K^T for 64 keys: 8 n-tiles of 8 keys
    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {  // two n-tiles per ldmatrix.x4
        // matrices: (keys 16np .. +7, k lo), (same keys, k hi), (keys 16np+8 .. +15, k lo), (.., k hi)
        const int key = np * 16 + (lane & 7) + ((lane >> 4) << 3), c = ks * 2 + ((lane >> 3) & 1);
        uint32_t b[4];
        ldsm_x4(sk + sw_off(key, c), b);
        mma16816(s[2 * np], qa[ks], b[0], b[1]);
        mma16816(s[2 * np + 1], qa[ks], b[2], b[3]);
      }
    }
    // causal mask, online softmax (rows g and g + 8 of this warp)
    float mx[2] = {mrow[0], mrow[1]};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = k0 + nt * 8 + tig * 2 + (e & 1);
        const int qi = qi0 + (e >> 1) * 8;
        const float v = (key <= qi && key < kend) ? s[nt][e] * sl2 : -INFINITY;
        s[nt][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
    }
    float corr[2], rs[2] = {0.f, 0.f};
#pragma unroll
    for (int h = 0; h < 2; ++h) corr[h] = mx[h] == -INFINITY ? 1.f : exp2f(mrow[h] - mx[h]);
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int h = e >> 1;
        const float p = mx[h] == -INFINITY ? 0.f : exp2f(s[nt][e] - mx[h]);
        s[nt][e] = p;
        rs[h] += p;
      }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 1);
      rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 2);
      lrow[h] = lrow[h] * corr[h] + rs[h];
      mrow[h] = mx[h];
    }
#pragma unroll
    for (int dt = 0; dt < 16; ++dt) {
      o[dt][0] *= corr[0];
      o[dt][1] *= corr[0];
      o[dt][2] *= corr[1];
      o[dt][3] *= corr[1];
    }
    // O += P V: k-steps of 16 keys (two score n-tiles), 16 n-tiles of 8 dims
#pragma unroll
    for (int kt = 0; kt < 4; ++kt) {
      uint32_t pa[4];
      pa[0] = pack_h2(s[2 * kt][0], s[2 * kt][1]);
      pa[1] = pack_h2(s[2 * kt][2], s[2 * kt][3]);
      pa[2] = pack_h2(s[2 * kt + 1][0], s[2 * kt + 1][1]);
      pa[3] = pack_h2(s[2 * kt + 1][2], s[2 * kt + 1][3]);
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {  // two dim n-tiles per ldmatrix.x4.trans
        // matrices: (keys 16kt .. +7, dims 16dp .. +7), (keys +8 .. +15, same dims),
        //           (keys 16kt .. +7, dims 16dp + 8 ..), (keys +8 .., dims +8 ..)
        const int key = kt * 16 + (lane & 7) + (((lane >> 3) & 1) << 3), c = dp * 2 + (lane >> 4);
        uint32_t b[4];
        ldsm_x4_t(sv + sw_off(key, c), b);
        mma16816(o[2 * dp], pa, b[0], b[1]);
        mma16816(o[2 * dp + 1], pa, b[2], b[3]);
      }
    }
    __syncthreads();  // every warp is done with this block's buffer before it is refilled
  }
  // normalise and store rows g, g + 8 of this warp
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int t = q0 + warp * 16 + g + h * 8;
    if (t >= P) continue;
    const float inv = lrow[h] > 0.f ? 1.f / lrow[h] : 0.f;
    __half* dst = out + ((size_t)t * hq + head) * kHD;
#pragma unroll
    for (int dt = 0; dt < 16; ++dt)
      *reinterpret_cast<uint32_t*>(dst + dt * 8 + tig * 2) = pack_h2(o[dt][2 * h] * inv, o[dt][2 * h + 1] * inv);
  }
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
                                                float eps, aicas_stream_t stream) {
  if (rows < 1 || start < 0 || start + rows > max_len || max_len > (1 << 30)) return AICAS_ERR_SHAPE;
  if (kv_heads < 1 || q_heads < kv_heads || q_heads % kv_heads != 0 || q_heads + 2 * kv_heads > 4096)
    return AICAS_ERR_SHAPE;
  if (!qkv || !q_norm_w || !k_norm_w || !pos3 || !inv_freq || !q_out || !k_cache || !v_cache) return AICAS_ERR_ARG;
  qk_norm_rope_kv_kernel<<<(unsigned)rows, 256, 0, stream>>>(
      (const __half*)qkv, (const __half*)q_norm_w, (const __half*)k_norm_w, (const int64_t*)pos3,
      (const float*)inv_freq, sec1, sec2, (__half*)q_out, (__half*)k_cache, (__half*)v_cache, (int)rows, (int)start,
      (int)max_len, (int)q_heads, (int)kv_heads, eps);
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

AICAS_API int aicas_prefill_attention_f16(const void* q, const void* k_cache, const void* v_cache, void* out,
                                          int64_t rows, int64_t start, int64_t q_heads, int64_t kv_heads,
                                          int64_t max_len, float scale, aicas_stream_t stream) {
  if (rows < 1 || start < 0 || start + rows > max_len || max_len > (1 << 30)) return AICAS_ERR_SHAPE;
  if (kv_heads < 1 || q_heads < kv_heads || q_heads % kv_heads != 0 || q_heads > 65535) return AICAS_ERR_SHAPE;
  if (!q || !k_cache || !v_cache || !out || !al16(q) || !al16(k_cache) || !al16(v_cache) || !al16(out))
    return AICAS_ERR_ALIGN;
  const dim3 grid((unsigned)((rows + kBQ - 1) / kBQ), (unsigned)q_heads);
  // dynamic shared memory above 48 KB needs an opt-in, once per device
  static bool attr_done[64] = {};
  int dev = 0;
  cudaError_t ea = cudaGetDevice(&dev);
  if (ea != cudaSuccess) return aicas::record_cuda_error(ea);
  if (dev < 0 || dev >= 64) return AICAS_ERR_CUDA;
  if (!attr_done[dev]) {
    ea = cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem);
    if (ea != cudaSuccess) return aicas::record_cuda_error(ea);
    attr_done[dev] = true;
  }
  attention_kernel<<<grid, kAttnThreads, kAttnSmem, stream>>>((const __half*)q, (const __half*)k_cache,
                                                      (const __half*)v_cache, (__half*)out, (int)rows, (int)start,
                                                      (int)q_heads, (int)kv_heads, (int)max_len, scale);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? AICAS_OK : aicas::record_cuda_error(e);
}

}  // extern "C"
