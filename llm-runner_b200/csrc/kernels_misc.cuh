// Memory-bound kernels of the attention path: the fused QK-RMSNorm + RoPE +
// cast prologue, the fp32 mirrors of the reference's small ops, the exact
// fp32 attention (spatial_attention math) and the LSE merge of the ring.
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

// One warp per (tensor, b, s, h) row of D elements, 4 rows in flight per
// warp. Q and K rows get the per-head RMSNorm of batch_head_norm
// (dependencies/zimage.c3l/shaders/zimage.slang:623-659:
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
  constexpr int U = 4;       // rows per warp per iteration
  const int lane = threadIdx.x & 31;
  const long long rows = (long long)p.B * p.S * p.H;
  const long long total = 3 * rows;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  const long long plane = rows * D;
  for (long long w0 = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
       w0 < total; w0 += U * warps) {
    float x[U][E];
    int tsel[U], s[U];
    long long r[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const long long w = w0 + u * warps;
      tsel[u] = w < total ? (int)(w / rows) : 0;
      r[u] = w - tsel[u] * rows;
      s[u] = (int)(r[u] % p.S);
      if (w >= total) continue;
      // r enumerates (b, h, s) with s fastest, matching the output order.
      const long long bh = r[u] / p.S;
      const int h = (int)(bh % p.H), b = (int)(bh / p.H);
      // Select by value (a reference into the parameter block would force it
      // into local memory).
      const int t = tsel[u];
      const InT *base = t == 0 ? q.base : (t == 1 ? k.base : v.base);
      const long long bs = t == 0 ? q.bs : (t == 1 ? k.bs : v.bs);
      const long long rs = t == 0 ? q.rs : (t == 1 ? k.rs : v.rs);
      const long long hs = t == 0 ? q.hs : (t == 1 ? k.hs : v.hs);
      const InT *src = base + b * bs + (long long)s[u] * rs + (long long)h * hs + lane * E;
      if (VEC) {
        const Pack<InT, E> pk = *reinterpret_cast<const Pack<InT, E> *>(src);
#pragma unroll
        for (int e = 0; e < E; e++) x[u][e] = to_f32<InT>(pk.v[e]);
      } else {
#pragma unroll
        for (int e = 0; e < E; e++) x[u][e] = to_f32<InT>(src[e]);
      }
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      if (w0 + u * warps >= total) break;
      const float *gain = tsel[u] == 0 ? p.q_gain : (tsel[u] == 1 ? p.k_gain : nullptr);
      const long long grow = (long long)p.rope_row_offset + s[u];  // global token index
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
      if (tsel[u] < 2 && p.cos_t != nullptr) {
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
      *reinterpret_cast<Pack<OutT, E> *>(out + tsel[u] * plane + r[u] * D + lane * E) = po;
    }
  }
}

// batch_head_norm / perhead_rmsnorm mirror: in place on fp32 [S, H*D].
__global__ void head_norm_f32_kernel(float *data, const float *gain, int H,
                                     int D, int S, float eps) {
  const int lane = threadIdx.x & 31;
  const long long rows = (long long)S * H;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long w = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
       w < rows; w += warps) {
    float *x = data + w * D;
    float ss = 0.0f;
    for (int i = lane; i < D; i += 32) ss = __fmaf_rn(x[i], x[i], ss);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float rms = 1.0f / sqrtf(ss / (float)D + eps);
    for (int i = lane; i < D; i += 32) x[i] = __fmul_rn(__fmul_rn(x[i], rms), gain[i]);
  }
}

// transpose_heads mirror (zimage.slang:575-601).
__global__ void transpose_heads_kernel(const float *in, float *out, int S,
                                       int H, int D, int direction) {
  const long long total = (long long)S * H * D;
  for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (long long)gridDim.x * blockDim.x) {
    const long long d = t % D, rem = t / D;
    if (direction == 0) {
      const long long seq = rem / H, h = rem % H;
      out[h * S * D + seq * D + d] = in[t];
    } else {
      const long long h = rem / S, seq = rem % S;
      out[seq * H * D + h * D + d] = in[t];
    }
  }
}

// mrope mirror (mrope.slang:33-54): data [H, S, 2*half], tables [S, half].
__global__ void mrope_f32_kernel(float *data, const float *cos_t,
                                 const float *sin_t, int S, int H, int half) {
  const long long total = (long long)H * S * half;
  for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (long long)gridDim.x * blockDim.x) {
    const long long pair = t % half, hs = t / half, pos = hs % S;
    const float cv = cos_t[pos * half + pair], sv = sin_t[pos * half + pair];
    float *x = data + hs * 2 * half + 2 * pair;
    const float x0 = x[0], x1 = x[1];
    x[0] = __fsub_rn(__fmul_rn(x0, cv), __fmul_rn(x1, sv));
    x[1] = __fadd_rn(__fmul_rn(x0, sv), __fmul_rn(x1, cv));
  }
}

// split_qkv mirror (depth.slang:40-58).
__global__ void split_qkv_kernel(const float *qkv, float *q, float *k,
                                 float *v, int dim, int n_rows) {
  const long long total = (long long)n_rows * dim;
  for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (long long)gridDim.x * blockDim.x) {
    const long long row = t / dim, d = t % dim, base = row * 3 * dim;
    q[t] = qkv[base + d];
    k[t] = qkv[base + dim + d];
    v[t] = qkv[base + 2 * dim + d];
  }
}

// Exact fp32 attention (spatial_attention math, lib/shaders/diffusion.slang:
// 478-569: fp32 dot products, exact softmax, no fp16 rounding), computed
// flash-style with an fp32 online softmax so no S x S buffer exists. Inputs
// dense fp32 [B][H][S][D]. CTA = 4 warps x RPW query rows of one (b, h); key
// tiles staged in shared memory.
struct ExactParams {
  int B, H, S;
  float scale;
  float *o;
  long long o_batch_stride, o_row_stride, o_head_stride;
  float *lse;  // optional [B][H][S]
};

template <int D>
__global__ void __launch_bounds__(128)
    attn_exact_f32_kernel(const float *Q, const float *K, const float *V,
                          ExactParams p) {
  // Static shared memory stays under 48 KB: D=128 uses 32-key tiles and 4
  // rows per warp, D=64 64-key tiles and 8 rows per warp.
  constexpr int KT = D == 128 ? 32 : 64, NC = KT / 32;
  constexpr int RPW = D == 128 ? 4 : 8, DL = D / 32;
  __shared__ float sK[KT][D + 1];
  __shared__ float sV[KT][D];
  __shared__ float sQ[4 * RPW][D];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const long long head_off = (long long)bh * p.S * D;
  const int row0 = blockIdx.x * 4 * RPW;
  for (int i = threadIdx.x; i < 4 * RPW * D; i += blockDim.x) {
    const int r = i / D, d = i % D, qr = row0 + r;
    sQ[r][d] = qr < p.S ? Q[head_off + (long long)qr * D + d] : 0.0f;
  }
  float m[RPW], l[RPW], acc[RPW][DL];
#pragma unroll
  for (int r = 0; r < RPW; r++) {
    m[r] = -INFINITY;
    l[r] = 0.0f;
#pragma unroll
    for (int e = 0; e < DL; e++) acc[r][e] = 0.0f;
  }
  for (int k0 = 0; k0 < p.S; k0 += KT) {
    __syncthreads();
    for (int i = threadIdx.x; i < KT * D; i += blockDim.x) {
      const int r = i / D, d = i % D, kr = k0 + r;
      sK[r][d] = kr < p.S ? K[head_off + (long long)kr * D + d] : 0.0f;
      sV[r][d] = kr < p.S ? V[head_off + (long long)kr * D + d] : 0.0f;
    }
    __syncthreads();
#pragma unroll 1
    for (int r = 0; r < RPW; r++) {
      const float *qrow = sQ[warp * RPW + r];
      float sc[NC];
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < NC; c++) {
        const int kk = lane + 32 * c;
        float dot = 0.0f;
        for (int d = 0; d < D; d++) dot = __fmaf_rn(qrow[d], sK[kk][d], dot);
        sc[c] = (k0 + kk < p.S) ? dot * p.scale : -INFINITY;
        mx = fmaxf(mx, sc[c]);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float m_new = fmaxf(m[r], mx);
      const float alpha = expf(m[r] - m_new);
      float pv[NC], ps = 0.0f;
#pragma unroll
      for (int c = 0; c < NC; c++) {
        pv[c] = expf(sc[c] - m_new);
        ps += pv[c];
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
      l[r] = l[r] * alpha + ps;
      m[r] = m_new;
#pragma unroll
      for (int e = 0; e < DL; e++) acc[r][e] *= alpha;
#pragma unroll
      for (int c = 0; c < NC; c++) {
        for (int kk = 0; kk < 32; kk++) {
          const float pk = __shfl_sync(0xffffffffu, pv[c], kk);
#pragma unroll
          for (int e = 0; e < DL; e++)
            acc[r][e] = __fmaf_rn(pk, sV[32 * c + kk][lane + 32 * e], acc[r][e]);
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < RPW; r++) {
    const int qr = row0 + warp * RPW + r;
    if (qr >= p.S) continue;
    float *dst = p.o + (long long)b * p.o_batch_stride + (long long)qr * p.o_row_stride +
                 (long long)h * p.o_head_stride;
#pragma unroll
    for (int e = 0; e < DL; e++) dst[lane + 32 * e] = acc[r][e] / l[r];
    if (p.lse != nullptr && lane == 0) p.lse[(long long)bh * p.S + qr] = m[r] + logf(l[r]);
  }
}

// Combine two normalised partial results over disjoint key sets:
// o = (e^{la-m} oa + e^{lb-m} ob) / (e^{la-m} + e^{lb-m}), lse = m + log(...).
__global__ void merge_kernel(float *oa, float *la, const float *ob,
                             const float *lb, int rows, int H, int D,
                             long long o_row_stride) {
  const long long total = (long long)rows * H * D;
  for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (long long)gridDim.x * blockDim.x) {
    const int d = (int)(t % D);
    const long long rh = t / D;
    const int h = (int)(rh % H);
    const long long r = rh / H;
    const float a = la[(long long)h * rows + r], c = lb[(long long)h * rows + r];
    const float mm = fmaxf(a, c);
    const float wa = expf(a - mm), wb = expf(c - mm);
    const long long idx = r * o_row_stride + (long long)h * D + d;
    oa[idx] = (wa * oa[idx] + wb * ob[idx]) / (wa + wb);
    // The LSE update is written after every d of this (r, h) has read it:
    // it is done by a separate pass (merge_lse_kernel).
  }
}

__global__ void merge_lse_kernel(float *la, const float *lb, long long n) {
  for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < n;
       t += (long long)gridDim.x * blockDim.x) {
    const float a = la[t], c = lb[t], mm = fmaxf(a, c);
    la[t] = mm + logf(expf(a - mm) + expf(c - mm));
  }
}

}  // namespace llmr
