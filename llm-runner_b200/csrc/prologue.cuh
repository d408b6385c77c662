// The fused QK-RMSNorm + RoPE + cast prologue of the attention path and its
// small type helpers (included by every translation unit that launches it).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "ptx.cuh"

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

// Programmatic dependent launch: a kernel launched right after this one with
// the programmatic-serialization attribute may start (its CTAs become
// resident as this grid's CTAs retire) once every CTA here has executed
// launch_dependents; it must execute griddep_wait before reading what this
// grid writes (the wait returns when this grid has completed and its
// memory is visible). Both are no-ops for kernels launched normally.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Prologue geometry: a row (one token of one head) is D elements, handled by
// an 8-lane group with E = D/8 elements per lane, so a warp works on 4 rows
// at once and the RMSNorm sum needs a 3-step shuffle. A CTA of 8 warps walks
// kProRowsPerCta rows of one (tensor, b, h).
constexpr int kProLanesPerRow = 8;
constexpr int kProRowsPerWarpStep = 32 / kProLanesPerRow;  // 4
constexpr int kProWarps = 8;
// Two row groups per warp keep a lane at 56 registers, so 4 CTAs (32 warps)
// share an SM and hide the norm / table latency; 4 groups (80 registers,
// 3 CTAs) ran 5 % slower, 1 group (47 registers, 5 CTAs) no faster.
constexpr int kProSteps = 2;  // row groups per warp
constexpr int kProRowsPerCta = kProRowsPerWarpStep * kProWarps * kProSteps;  // 64

// Grid (ceil(S / kProRowsPerCta), 3, B*H): blockIdx.y selects Q, K or V, blockIdx.z the
// (b, h) unit, last unit first. CTAs start roughly in grid order, so the
// (b, h) units the attention kernel starts with (its first round of work
// units is ordered by (b, h)) are written last and are still in L2 when it
// loads them. Q and K rows get the per-head RMSNorm of batch_head_norm
// (dependencies/zimage.c3l/shaders/zimage.slang:623-659:
// x * (1/sqrt(mean(x^2) + eps)) * g) and the interleaved rotation of mrope
// (dependencies/zimage.c3l/shaders/mrope.slang:47-53) in fp32, with the
// shader's operation order for the products; V is only converted. Output:
// dense [3][B][H][S][D] in OutT (fp16 RNE, the rounding flash_attn.slang
// applies on load, or fp32 for the exact path). VEC: every lane's slice of
// the inputs and tables is 16-byte aligned (checked on the host).
// Grid of prologue_kernel: (ceil(S / kProRowsPerCta), 3, B*H).
inline dim3 prologue_grid(int S, int BH) {
  return dim3((S + kProRowsPerCta - 1) / kProRowsPerCta, 3, BH);
}
#ifndef LLMR_PRO_MIN_CTAS
#define LLMR_PRO_MIN_CTAS 4  // CTAs per SM the register budget must allow
#endif
template <int D, typename InT, typename OutT, bool VEC>
__global__ void __launch_bounds__(256, LLMR_PRO_MIN_CTAS)
    prologue_kernel(View<InT> q, View<InT> k, View<InT> v, OutT *out,
                    ProParams p) {
  constexpr int E = D / kProLanesPerRow;  // 16 (D=128) or 8 (D=64)
  constexpr int VIN = 16 / sizeof(InT);   // elements per 16-byte load
  // The attention kernel launched behind this one may take SMs as this
  // grid's last CTAs retire (it waits for this grid's results).
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int sub = lane & (kProLanesPerRow - 1);  // position inside the row
  const int t = blockIdx.y;                      // 0 = Q, 1 = K, 2 = V
  const int tblk = blockIdx.x;                   // 128-token block
  const int bh = gridDim.z - 1 - blockIdx.z;
  const int b = bh / p.H, h = bh - b * p.H;
  // Select by value (a reference into the parameter block would force it
  // into local memory).
  const InT *base = t == 0 ? q.base : (t == 1 ? k.base : v.base);
  const long long bs = t == 0 ? q.bs : (t == 1 ? k.bs : v.bs);
  const long long rs = t == 0 ? q.rs : (t == 1 ? k.rs : v.rs);
  const long long hs = t == 0 ? q.hs : (t == 1 ? k.hs : v.hs);
  const InT *src0 = base + (long long)b * bs + (long long)h * hs + sub * E;
  const float *gain = t == 0 ? p.q_gain : (t == 1 ? p.k_gain : nullptr);
  const bool rope = t < 2 && p.cos_t != nullptr;
  OutT *dst0 = out + ((long long)t * p.B * p.H + bh) * (long long)p.S * D + sub * E;
  const int row_in_warp = lane / kProLanesPerRow;
  const int s_base = tblk * kProRowsPerCta + (threadIdx.x >> 5) * kProRowsPerWarpStep +
                     row_in_warp;
  // All row groups' loads are issued before any is used, so a warp keeps
  // kProSteps * 16 * (E / VIN) bytes per lane in flight.
  Pack<InT, VIN> raw[kProSteps][E / VIN];
#pragma unroll
  for (int step = 0; step < kProSteps; step++) {
    const int s = s_base + step * kProRowsPerWarpStep * kProWarps;
    if (VEC && s < p.S) {
      const InT *src = src0 + (long long)s * rs;
#pragma unroll
      for (int c = 0; c < E / VIN; c++)
        raw[step][c] = *reinterpret_cast<const Pack<InT, VIN> *>(src + c * VIN);
    }
  }
#pragma unroll
  for (int step = 0; step < kProSteps; step++) {
    const int s = s_base + step * kProRowsPerWarpStep * kProWarps;
    // Lanes of a row group share the row, so the whole 8-lane group is in
    // or out together; shuffles stay inside the group.
    const bool in = s < p.S;
    float x[E];
    if (in) {
      if (VEC) {
#pragma unroll
        for (int c = 0; c < E / VIN; c++)
#pragma unroll
          for (int e = 0; e < VIN; e++) x[c * VIN + e] = to_f32<InT>(raw[step][c].v[e]);
      } else {
        const InT *src = src0 + (long long)s * rs;
#pragma unroll
        for (int e = 0; e < E; e++) x[e] = to_f32<InT>(src[e]);
      }
    } else {
#pragma unroll
      for (int e = 0; e < E; e++) x[e] = 0.0f;
    }
    const long long grow = (long long)p.rope_row_offset + s;  // global token index
    if (gain != nullptr) {
      float ss = 0.0f;
#pragma unroll
      for (int e = 0; e < E; e++) ss = __fmaf_rn(x[e], x[e], ss);
#pragma unroll
      for (int o = kProLanesPerRow / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float rms = rsqrtf(ss / (float)D + p.eps);
      const float *g = gain + ((p.split_row > 0 && grow >= p.split_row) ? D : 0) + sub * E;
#pragma unroll
      for (int e = 0; e < E; e++) x[e] = __fmul_rn(__fmul_rn(x[e], rms), g[e]);
    }
    if (rope && in) {
      const float *ct = p.cos_t + grow * (D / 2) + sub * (E / 2);
      const float *st = p.sin_t + grow * (D / 2) + sub * (E / 2);
      float cv[E / 2], sv[E / 2];
      if (VEC) {
#pragma unroll
        for (int c = 0; c < E / 2; c += 4) {
          const float4 a = *reinterpret_cast<const float4 *>(ct + c);
          const float4 bq = *reinterpret_cast<const float4 *>(st + c);
          cv[c] = a.x; cv[c + 1] = a.y; cv[c + 2] = a.z; cv[c + 3] = a.w;
          sv[c] = bq.x; sv[c + 1] = bq.y; sv[c + 2] = bq.z; sv[c + 3] = bq.w;
        }
      } else {
#pragma unroll
        for (int e = 0; e < E / 2; e++) {
          cv[e] = ct[e];
          sv[e] = st[e];
        }
      }
#pragma unroll
      for (int e = 0; e < E; e += 2) {
        const float x0 = x[e], x1 = x[e + 1];
        x[e] = __fsub_rn(__fmul_rn(x0, cv[e / 2]), __fmul_rn(x1, sv[e / 2]));
        x[e + 1] = __fadd_rn(__fmul_rn(x0, sv[e / 2]), __fmul_rn(x1, cv[e / 2]));
      }
    }
    if (in) {
      constexpr int VOUT = 16 / sizeof(OutT);
      OutT *dst = dst0 + (long long)s * D;
#pragma unroll
      for (int c = 0; c < E / VOUT; c++) {
        Pack<OutT, VOUT> po;
#pragma unroll
        for (int e = 0; e < VOUT; e++) po.v[e] = from_f32<OutT>(x[c * VOUT + e]);
        *reinterpret_cast<Pack<OutT, VOUT> *>(dst + c * VOUT) = po;
      }
    }
  }
}

// 16-byte global -> shared copy that bypasses L1 and completes
// asynchronously (commit / wait groups); src_bytes = 0 writes zeros.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// The prologue arithmetic of prologue_kernel for one lane's slice of one row
// (lane `sub` of the row's 8 lanes; token s of tensor t = 0 Q, 1 K, 2 V) with
// the input already widened to fp32 in x (zeros for s >= S): RMSNorm in fp32
// with the same operation order, the interleaved RoPE rotation, fp16 RNE
// store to dst (the row's fp16 workspace slice). Whole warps only (the norm's
// shuffles); `t` is warp-uniform. Gains and tables 16-byte aligned.
template <int D>
__device__ __forceinline__ void pro_row_finish(float (&x)[D / kProLanesPerRow],
                                               const ProParams &p, int t, int s, int sub,
                                               __half *dst) {
  constexpr int E = D / kProLanesPerRow;
  const bool in = s < p.S;
  const float *gain = t == 0 ? p.q_gain : (t == 1 ? p.k_gain : nullptr);
  const long long grow = (long long)p.rope_row_offset + s;  // global token index
  if (gain != nullptr) {
    float ss = 0.0f;
#pragma unroll
    for (int e = 0; e < E; e++) ss = __fmaf_rn(x[e], x[e], ss);
#pragma unroll
    for (int o = kProLanesPerRow / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float rms = rsqrtf(ss / (float)D + p.eps);
    const float *g = gain + ((p.split_row > 0 && grow >= p.split_row) ? D : 0) + sub * E;
#pragma unroll
    for (int e = 0; e < E; e += 4) {
      const float4 gv = __ldg(reinterpret_cast<const float4 *>(g + e));
      x[e] = __fmul_rn(__fmul_rn(x[e], rms), gv.x);
      x[e + 1] = __fmul_rn(__fmul_rn(x[e + 1], rms), gv.y);
      x[e + 2] = __fmul_rn(__fmul_rn(x[e + 2], rms), gv.z);
      x[e + 3] = __fmul_rn(__fmul_rn(x[e + 3], rms), gv.w);
    }
  }
  if (t < 2 && p.cos_t != nullptr && in) {
    const float *ct = p.cos_t + grow * (D / 2) + sub * (E / 2);
    const float *st = p.sin_t + grow * (D / 2) + sub * (E / 2);
#pragma unroll
    for (int e = 0; e < E / 2; e += 4) {
      const float4 cv = __ldg(reinterpret_cast<const float4 *>(ct + e));
      const float4 sv = __ldg(reinterpret_cast<const float4 *>(st + e));
      const float c4[4] = {cv.x, cv.y, cv.z, cv.w}, s4[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const float x0 = x[2 * (e + u)], x1 = x[2 * (e + u) + 1];
        x[2 * (e + u)] = __fsub_rn(__fmul_rn(x0, c4[u]), __fmul_rn(x1, s4[u]));
        x[2 * (e + u) + 1] = __fadd_rn(__fmul_rn(x0, s4[u]), __fmul_rn(x1, c4[u]));
      }
    }
  }
  if (in) {
#pragma unroll
    for (int c = 0; c < E / 8; c++) {
      Pack<__half, 8> po;
#pragma unroll
      for (int e = 0; e < 8; e++) po.v[e] = __float2half_rn(x[c * 8 + e]);
      *reinterpret_cast<Pack<__half, 8> *>(dst + c * 8) = po;
    }
  }
}

// Strided view selection by value (a reference into a parameter block would
// force it into local memory): base / strides of tensor t.
template <typename InT>
struct ViewSel {
  const InT *base;
  long long bs, rs, hs;
  __device__ __forceinline__ ViewSel(const View<InT> &vq, const View<InT> &vk,
                                     const View<InT> &vv, int t)
      : base(t == 0 ? vq.base : (t == 1 ? vk.base : vv.base)),
        bs(t == 0 ? vq.bs : (t == 1 ? vk.bs : vv.bs)),
        rs(t == 0 ? vq.rs : (t == 1 ? vk.rs : vv.rs)),
        hs(t == 0 ? vq.hs : (t == 1 ? vk.hs : vv.hs)) {}
};

// Address of the fp16 workspace [3][B][H][S][D] row (t, b, h, s), lane slice.
template <int D>
__device__ __forceinline__ __half *pro_dst(__half *ws, const ProParams &p, int t, int b, int h,
                                           int s, int sub) {
  return ws + (((long long)t * p.B + b) * p.H + h) * (long long)p.S * D + (long long)s * D +
         sub * (D / kProLanesPerRow);
}

// One prologue piece for the attention kernel's fused prologue: token rows
// [s0, s0 + 32) of tensor t of (b, h) into the fp16 workspace, by one whole
// warp (8 lanes per row, 4 rows per step), the loads of NB steps issued
// before any is used. Inputs 16-byte aligned with strides in whole 16-byte
// units (checked on the host).
template <int D, typename InT, int NB>
__device__ __forceinline__ void pro_piece(const View<InT> &vq, const View<InT> &vk,
                                          const View<InT> &vv, __half *ws,
                                          const ProParams &p, int t, int b, int h, int s0,
                                          int lane) {
  constexpr int E = D / kProLanesPerRow;
  constexpr int VIN = 16 / sizeof(InT);
  constexpr int CH = E / VIN;
  constexpr int STEPS = 32 / kProRowsPerWarpStep;  // 8
  static_assert(STEPS % NB == 0, "steps per batch");
  const int sub = lane & (kProLanesPerRow - 1);
  const int r = lane / kProLanesPerRow;
  const ViewSel<InT> v(vq, vk, vv, t);
  const InT *src0 = v.base + (long long)b * v.bs + (long long)h * v.hs + sub * E;
#pragma unroll 1
  for (int st0 = 0; st0 < STEPS; st0 += NB) {
    Pack<InT, VIN> raw[NB][CH];
#pragma unroll
    for (int i = 0; i < NB; i++) {
      const int s = s0 + (st0 + i) * kProRowsPerWarpStep + r;
      if (s < p.S) {
        const InT *src = src0 + (long long)s * v.rs;
#pragma unroll
        for (int c = 0; c < CH; c++)
          raw[i][c] = *reinterpret_cast<const Pack<InT, VIN> *>(src + c * VIN);
      }
    }
#pragma unroll
    for (int i = 0; i < NB; i++) {
      const int s = s0 + (st0 + i) * kProRowsPerWarpStep + r;
      const bool in = s < p.S;
      float x[E];
#pragma unroll
      for (int c = 0; c < CH; c++)
#pragma unroll
        for (int e = 0; e < VIN; e++) x[c * VIN + e] = in ? to_f32<InT>(raw[i][c].v[e]) : 0.0f;
      pro_row_finish<D>(x, p, t, s, sub, pro_dst<D>(ws, p, t, b, h, in ? s : 0, sub));
    }
  }
}

// Prologue of the wide-head path (D = 384 / 512, the VAE attention, which has
// no norm or RoPE): Q, K, V from strided views of any input type to dense
// [3][B][H][S][D] OutT (fp16 RNE for the tensor-core kernel, fp32 for the
// exact one). Grid (x, 3): blockIdx.y selects the tensor; a thread converts
// 8 consecutive elements of one row. VEC: bases and strides allow 16-byte
// loads (checked on the host).
template <typename InT, typename OutT, bool VEC>
__global__ void __launch_bounds__(256)
    wide_cast_kernel(View<InT> q, View<InT> k, View<InT> v, OutT *out, int B, int H, int S,
                     int D) {
  const int t = blockIdx.y;
  const InT *base = t == 0 ? q.base : (t == 1 ? k.base : v.base);
  const long long bs = t == 0 ? q.bs : (t == 1 ? k.bs : v.bs);
  const long long rs = t == 0 ? q.rs : (t == 1 ? k.rs : v.rs);
  const long long hs = t == 0 ? q.hs : (t == 1 ? k.hs : v.hs);
  const int gpr = D / 8;  // 8-element groups per row
  const long long groups = (long long)B * H * S * gpr;
  OutT *dst0 = out + (long long)t * B * H * S * D;
  constexpr int VIN = 16 / sizeof(InT), VOUT = 16 / sizeof(OutT);
  for (long long g = (long long)blockIdx.x * blockDim.x + threadIdx.x; g < groups;
       g += (long long)gridDim.x * blockDim.x) {
    const int d = (int)(g % gpr) * 8;
    const long long row = g / gpr;  // (b * H + h) * S + s
    const int s = (int)(row % S);
    const long long bh = row / S;
    const int h = (int)(bh % H), b = (int)(bh / H);
    const InT *src = base + (long long)b * bs + (long long)s * rs + (long long)h * hs + d;
    float x[8];
    if (VEC) {
#pragma unroll
      for (int c = 0; c < 8 / VIN; c++) {
        const Pack<InT, VIN> pk = *reinterpret_cast<const Pack<InT, VIN> *>(src + c * VIN);
#pragma unroll
        for (int e = 0; e < VIN; e++) x[c * VIN + e] = to_f32<InT>(pk.v[e]);
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; e++) x[e] = to_f32<InT>(src[e]);
    }
    OutT *dst = dst0 + row * D + d;
#pragma unroll
    for (int c = 0; c < 8 / VOUT; c++) {
      Pack<OutT, VOUT> po;
#pragma unroll
      for (int e = 0; e < VOUT; e++) po.v[e] = from_f32<OutT>(x[c * VOUT + e]);
      *reinterpret_cast<Pack<OutT, VOUT> *>(dst + c * VOUT) = po;
    }
  }
}

}  // namespace llmr
