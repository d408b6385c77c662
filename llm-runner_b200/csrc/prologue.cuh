// The fused QK-RMSNorm + RoPE + cast prologue of the attention path and its
// small type helpers (included by every translation unit that launches it).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace llmr {

template <typename T> __device__ __forceinline__ float to_f32(T x);
template <> __device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// Strided view of one of Q/K/V: element (b, s, h, d) at
// base[b*bs + s*rs + h*hs + d].
template <typename T>
struct View {
  const T *base;
  long long bs, rs, hs;
};

struct ProParams {
  int B, S, H;
  int split_row;        // rows < split use gain[0:D), rows >= split gain[D:2D)
  int rope_row_offset;  // table row of token 0
  float eps;
  const float *q_gain, *k_gain;  // null = no norm for that tensor
  const float *cos_t, *sin_t;    // null = no RoPE
};

template <typename T, int N>
struct alignas(sizeof(T) * N) Pack {
  T v[N];
};

// Rows per CTA of the prologue: 8 warps x 4 rows in flight per warp.
constexpr int kProRowsPerWarp = 4;
constexpr int kProWarps = 8;
constexpr int kProRowsPerCta = kProRowsPerWarp * kProWarps;

// Grid (ceil(S / 32), B*H, 3): blockIdx.z selects Q, K or V, blockIdx.y the
// (b, h) unit, and each warp owns 4 consecutive tokens s of that unit (a
// row = D elements). Q and K rows get the per-head RMSNorm of
// batch_head_norm (dependencies/zimage.c3l/shaders/zimage.slang:623-659:
// x * (1/sqrt(mean(x^2) + eps)) * g) and the interleaved rotation of mrope
// (dependencies/zimage.c3l/shaders/mrope.slang:47-53), computed in fp32 with
// the same operation order; V is only converted. Output: dense
// [3][B][H][S][D] in OutT (fp16 RNE, the rounding flash_attn.slang applies on
// load, or fp32 for the exact path). VEC: inputs and tables allow one
// vector access per lane (checked on the host).
template <int D, typename InT, typename OutT, bool VEC>
__global__ void __launch_bounds__(256)
    prologue_kernel(View<InT> q, View<InT> k, View<InT> v, OutT *out,
                    ProParams p) {
  constexpr int E = D / 32;  // elements per lane: 4 (D=128) or 2 (D=64)
  constexpr int U = kProRowsPerWarp;
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.z;  // 0 = Q, 1 = K, 2 = V
  const int bh = blockIdx.y;
  const int b = bh / p.H, h = bh - b * p.H;
  const int s0 = blockIdx.x * kProRowsPerCta + (threadIdx.x >> 5) * U;
  // Select by value (a reference into the parameter block would force it
  // into local memory).
  const InT *base = t == 0 ? q.base : (t == 1 ? k.base : v.base);
  const long long bs = t == 0 ? q.bs : (t == 1 ? k.bs : v.bs);
  const long long rs = t == 0 ? q.rs : (t == 1 ? k.rs : v.rs);
  const long long hs = t == 0 ? q.hs : (t == 1 ? k.hs : v.hs);
  const InT *src0 = base + (long long)b * bs + (long long)h * hs + lane * E;
  float x[U][E];
#pragma unroll
  for (int u = 0; u < U; u++) {
    if (s0 + u >= p.S) break;
    const InT *src = src0 + (long long)(s0 + u) * rs;
    if (VEC) {
      const Pack<InT, E> pk = *reinterpret_cast<const Pack<InT, E> *>(src);
#pragma unroll
      for (int e = 0; e < E; e++) x[u][e] = to_f32<InT>(pk.v[e]);
    } else {
#pragma unroll
      for (int e = 0; e < E; e++) x[u][e] = to_f32<InT>(src[e]);
    }
  }
  const float *gain = t == 0 ? p.q_gain : (t == 1 ? p.k_gain : nullptr);
  OutT *dst0 = out + ((long long)t * p.B * p.H + bh) * (long long)p.S * D + lane * E;
#pragma unroll
  for (int u = 0; u < U; u++) {
    const int s = s0 + u;
    if (s >= p.S) break;
    const long long grow = (long long)p.rope_row_offset + s;  // global token index
    if (gain != nullptr) {
      float ss = 0.0f;
#pragma unroll
      for (int e = 0; e < E; e++) ss = __fmaf_rn(x[u][e], x[u][e], ss);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float rms = 1.0f / sqrtf(ss / (float)D + p.eps);
      const float *g = gain + ((p.split_row > 0 && grow >= p.split_row) ? D : 0) + lane * E;
#pragma unroll
      for (int e = 0; e < E; e++) x[u][e] = __fmul_rn(__fmul_rn(x[u][e], rms), g[e]);
    }
    if (t < 2 && p.cos_t != nullptr) {
      const long long trow = grow * (D / 2) + lane * (E / 2);
      float cv[E / 2], sv[E / 2];
      if (VEC) {
        const Pack<float, E / 2> pc = *reinterpret_cast<const Pack<float, E / 2> *>(p.cos_t + trow);
        const Pack<float, E / 2> ps = *reinterpret_cast<const Pack<float, E / 2> *>(p.sin_t + trow);
#pragma unroll
        for (int e = 0; e < E / 2; e++) {
          cv[e] = pc.v[e];
          sv[e] = ps.v[e];
        }
      } else {
#pragma unroll
        for (int e = 0; e < E / 2; e++) {
          cv[e] = p.cos_t[trow + e];
          sv[e] = p.sin_t[trow + e];
        }
      }
#pragma unroll
      for (int e = 0; e < E; e += 2) {
        const float x0 = x[u][e], x1 = x[u][e + 1];
        x[u][e] = __fsub_rn(__fmul_rn(x0, cv[e / 2]), __fmul_rn(x1, sv[e / 2]));
        x[u][e + 1] = __fadd_rn(__fmul_rn(x0, sv[e / 2]), __fmul_rn(x1, cv[e / 2]));
      }
    }
    Pack<OutT, E> po;
#pragma unroll
    for (int e = 0; e < E; e++) po.v[e] = from_f32<OutT>(x[u][e]);
    *reinterpret_cast<Pack<OutT, E> *>(dst0 + (long long)s * D) = po;
  }
}

}  // namespace llmr
