// Memory-bound kernels of the attention path (the fused prologue is in
// prologue.cuh): the fp32 mirrors of the reference's small ops, the exact
// fp32 attention (spatial_attention math) and the LSE merge of the ring.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "prologue.cuh"
#include "ptx.cuh"

namespace llmr {

// Failure-detection probe: one thread waits on an mbarrier that nothing
// arrives at, through the same bounded wait the attention kernel uses, and
// raises the error word when the limit expires. The kernel then ends
// normally, so the context stays usable.
__global__ void wait_timeout_probe_kernel(int *err, unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && !mbar_wait_for(&bar, 0, &abort_flag, limit_ns)) atomicExch(err, 1);
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

// Body of the exact kernels: KT keys per shared-memory tile, RPW query rows
// per warp, sK [KT][D+1] (padded: lane = key reads are conflict-free),
// sV [KT][D], sQ [4*RPW][D].
template <int D, int KT, int RPW>
__device__ __forceinline__ void attn_exact_body(const float *Q, const float *K, const float *V,
                                                const ExactParams &p, float (*sK)[D + 1],
                                                float (*sV)[D], float (*sQ)[D]) {
  constexpr int NC = KT / 32, DL = D / 32;
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

template <int D>
__global__ void __launch_bounds__(128)
    attn_exact_f32_kernel(const float *Q, const float *K, const float *V,
                          ExactParams p) {
  // Static shared memory stays under 48 KB: D=128 uses 32-key tiles and 4
  // rows per warp, D=64 64-key tiles and 8 rows per warp.
  constexpr int KT = D == 128 ? 32 : 64;
  constexpr int RPW = D == 128 ? 4 : 8;
  __shared__ float sK[KT][D + 1];
  __shared__ float sV[KT][D];
  __shared__ float sQ[4 * RPW][D];
  attn_exact_body<D, KT, RPW>(Q, K, V, p, sK, sV, sQ);
}

// Wide heads (D = 384 or 512, the VAE attention): 32-key tiles and 4 rows
// per warp in dynamic shared memory (exact_wide_smem bytes).
constexpr int kExactWideRows = 4;
__host__ __device__ constexpr int exact_wide_smem(int D) {
  return (32 * (D + 1) + 32 * D + 4 * kExactWideRows * D) * (int)sizeof(float);
}

template <int D>
__global__ void __launch_bounds__(128)
    attn_exact_wide_kernel(const float *Q, const float *K, const float *V, ExactParams p) {
  extern __shared__ float xsm[];
  float(*sK)[D + 1] = reinterpret_cast<float(*)[D + 1]>(xsm);
  float(*sV)[D] = reinterpret_cast<float(*)[D]>(xsm + 32 * (D + 1));
  float(*sQ)[D] = reinterpret_cast<float(*)[D]>(xsm + 32 * (D + 1) + 32 * D);
  attn_exact_body<D, 32, kExactWideRows>(Q, K, V, p, sK, sV, sQ);
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

// dst[i] = OutT(src[i]) (RNE), 4 values per thread when aligned.
template <typename OutT>
__global__ void convert_f32_kernel(const float *src, OutT *dst, long long n, bool vec4) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (vec4) {
    for (; 4 * i + 3 < n; i += stride) {
      const float4 x = reinterpret_cast<const float4 *>(src)[i];
      Pack<OutT, 4> o;
      o.v[0] = from_f32<OutT>(x.x);
      o.v[1] = from_f32<OutT>(x.y);
      o.v[2] = from_f32<OutT>(x.z);
      o.v[3] = from_f32<OutT>(x.w);
      reinterpret_cast<Pack<OutT, 4> *>(dst)[i] = o;
    }
    // tail (n % 4 values) handled by thread 0 of block 0
    if (blockIdx.x == 0 && threadIdx.x == 0)
      for (long long t = n & ~3LL; t < n; t++) dst[t] = from_f32<OutT>(src[t]);
  } else {
    for (; i < n; i += stride) dst[i] = from_f32<OutT>(src[i]);
  }
}

}  // namespace llmr
