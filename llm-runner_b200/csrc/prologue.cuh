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

// Prologue geometry: a row (one token of one head) is D elements, handled by
// an 8-lane group with E = D/8 elements per lane, so a warp works on 4 rows
// at once and the RMSNorm sum needs a 3-step shuffle. A CTA of 8 warps walks
// kProRowsPerCta rows of one (tensor, b, h).
constexpr int kProLanesPerRow = 8;
constexpr int kProRowsPerWarpStep = 32 / kProLanesPerRow;  // 4
constexpr int kProWarps = 8;
constexpr int kProSteps = 4;  // row groups per warp
constexpr int kProRowsPerCta = kProRowsPerWarpStep * kProWarps * kProSteps;  // 128

// Grid (ceil(S / 128), B*H, 3): blockIdx.z selects Q, K or V, blockIdx.y the
// (b, h) unit. Q and K rows get the per-head RMSNorm of batch_head_norm
// (dependencies/zimage.c3l/shaders/zimage.slang:623-659:
// x * (1/sqrt(mean(x^2) + eps)) * g) and the interleaved rotation of mrope
// (dependencies/zimage.c3l/shaders/mrope.slang:47-53) in fp32, with the
// shader's operation order for the products; V is only converted. Output:
// dense [3][B][H][S][D] in OutT (fp16 RNE, the rounding flash_attn.slang
// applies on load, or fp32 for the exact path). VEC: every lane's slice of
// the inputs and tables is 16-byte aligned (checked on the host).
template <int D, typename InT, typename OutT, bool VEC>
__global__ void __launch_bounds__(256)
    prologue_kernel(View<InT> q, View<InT> k, View<InT> v, OutT *out,
                    ProParams p) {
  constexpr int E = D / kProLanesPerRow;  // 16 (D=128) or 8 (D=64)
  constexpr int VIN = 16 / sizeof(InT);   // elements per 16-byte load
  const int lane = threadIdx.x & 31;
  const int sub = lane & (kProLanesPerRow - 1);  // position inside the row
  const int t = blockIdx.z;                      // 0 = Q, 1 = K, 2 = V
  const int bh = blockIdx.y;
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
  const int s_base = blockIdx.x * kProRowsPerCta + (threadIdx.x >> 5) * kProRowsPerWarpStep +
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

// ------------------------------------------------------------ streaming form
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

// Streaming prologue (the default for 16-byte aligned inputs): the same
// arithmetic as prologue_kernel, organised for bandwidth.
//  * A work item is (b, 32 consecutive tokens, a chunk of heads); warp w of
//    the CTA owns tokens 4w..4w+3 of the item (8 lanes per token row) and
//    walks every (tensor, head) of the chunk, so the token's RoPE table
//    slice and its txt/img gain selection are loaded once per item into
//    registers instead of once per (token, head).
//  * Each thread prefetches its own 16-byte pieces of the next steps through
//    a ring in shared memory (cp.async, kPsStages steps ahead), so a warp
//    keeps up to 8 KB of input in flight with few registers; it reads back
//    only the bytes it copied itself, so no barrier is needed.
//  * The grid is at most two CTAs per SM (one wave); the head chunk is
//    shrunk until there are enough items to fill it.
// Output: dense [3][B][H][S][D] OutT, exactly as prologue_kernel writes it.
constexpr int kPsWarps = 8;
constexpr int kPsTokens = 4 * kPsWarps;  // tokens per work item
constexpr int kPsRingBytes = 8192;       // prefetch ring per warp
constexpr int kPsSmemBytes = kPsWarps * kPsRingBytes;

template <int D, typename InT, typename OutT>
__global__ void __launch_bounds__(256, 2)
    prologue_stream_kernel(View<InT> q, View<InT> k, View<InT> v, OutT *out, ProParams p,
                           int hchunk, int nitems) {
  constexpr int E = D / kProLanesPerRow;   // elements per lane (16 or 8)
  constexpr int VIN = 16 / sizeof(InT);    // elements per 16-byte piece
  constexpr int CH = E / VIN;              // pieces per lane and row
  constexpr int STAGE = 32 * CH * 16;      // bytes of one warp step (4 rows)
  constexpr int NST0 = kPsRingBytes / STAGE;
  constexpr int NST = NST0 > 8 ? 8 : NST0;  // steps in flight per warp
  static_assert(NST >= 2, "prefetch ring too small");
  extern __shared__ __align__(16) uint8_t ps_smem[];
  // The attention kernel that follows may take SMs as this grid drains.
  pdl_launch_dependents();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane & (kProLanesPerRow - 1);  // position inside the row
  const int r = lane / kProLanesPerRow;           // token row of the step
  const uint32_t ring = smem_u32(ps_smem + warp * kPsRingBytes);
  const int tok_blocks = (p.S + kPsTokens - 1) / kPsTokens;
  const int nhc = (p.H + hchunk - 1) / hchunk;
  const int nth = 3 * hchunk;  // (tensor, head) steps per item
  const int my_items =
      nitems > (int)blockIdx.x ? (nitems - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
  const int nsteps = my_items * nth;

  // Geometry of step g of this warp: item, tensor, head, token.
  struct Step {
    int b, h, t, s;
    bool run;  // head inside H (warp-uniform)
  };
  auto step_of = [&](int g) {
    Step st;
    const int item = (int)blockIdx.x + (g / nth) * (int)gridDim.x;
    const int th = g - (g / nth) * nth;
    const int hc = item % nhc;
    const int bt = item / nhc;
    st.b = bt / tok_blocks;
    const int tb = bt - st.b * tok_blocks;
    st.t = th / hchunk;
    st.h = hc * hchunk + (th - st.t * hchunk);
    st.s = tb * kPsTokens + warp * 4 + r;
    st.run = st.h < p.H;
    return st;
  };
  auto issue = [&](int g) {
    const Step st = step_of(g);
    const uint32_t dst = ring + (uint32_t)((g % NST) * STAGE) + (uint32_t)lane * 16u;
    if (st.run) {
      const InT *base = st.t == 0 ? q.base : (st.t == 1 ? k.base : v.base);
      const long long bs = st.t == 0 ? q.bs : (st.t == 1 ? k.bs : v.bs);
      const long long rs = st.t == 0 ? q.rs : (st.t == 1 ? k.rs : v.rs);
      const long long hs = st.t == 0 ? q.hs : (st.t == 1 ? k.hs : v.hs);
      const bool in = st.s < p.S;
      const InT *src = base + (long long)st.b * bs + (long long)(in ? st.s : 0) * rs +
                       (long long)st.h * hs + sub * E;
#pragma unroll
      for (int c = 0; c < CH; c++) cp_async16(dst + c * 512u, src + c * VIN, in ? 16u : 0u);
    }
  };

  // Per-item registers of this thread's token row: RoPE slice, gains.
  float cv[E / 2], sv[E / 2], gq[E], gk[E];
  int cur_item = -1;

#pragma unroll 1
  for (int g = 0; g < NST - 1; g++) {
    if (g < nsteps) issue(g);
    cp_async_commit();
  }
#pragma unroll 1
  for (int g = 0; g < nsteps; g++) {
    if (g + NST - 1 < nsteps) issue(g + NST - 1);
    cp_async_commit();
    cp_async_wait<NST - 1>();  // this thread's pieces of step g have landed
    const Step st = step_of(g);
    if (!st.run) continue;  // warp-uniform
    const bool in = st.s < p.S;
    const long long grow = (long long)p.rope_row_offset + st.s;  // global token index
    const int item = g / nth;
    if (item != cur_item) {
      cur_item = item;
      const int sel = (p.split_row > 0 && grow >= p.split_row) ? D : 0;
#pragma unroll
      for (int e = 0; e < E; e += 4) {
        const float4 a = p.q_gain ? __ldg(reinterpret_cast<const float4 *>(p.q_gain + sel + sub * E + e))
                                  : make_float4(1.f, 1.f, 1.f, 1.f);
        const float4 c = p.k_gain ? __ldg(reinterpret_cast<const float4 *>(p.k_gain + sel + sub * E + e))
                                  : make_float4(1.f, 1.f, 1.f, 1.f);
        gq[e] = a.x; gq[e + 1] = a.y; gq[e + 2] = a.z; gq[e + 3] = a.w;
        gk[e] = c.x; gk[e + 1] = c.y; gk[e + 2] = c.z; gk[e + 3] = c.w;
      }
      if (p.cos_t != nullptr) {
        const long long trow = in ? grow : (long long)p.rope_row_offset;
        const float *ct = p.cos_t + trow * (D / 2) + sub * (E / 2);
        const float *stb = p.sin_t + trow * (D / 2) + sub * (E / 2);
#pragma unroll
        for (int e = 0; e < E / 2; e += 4) {
          const float4 a = __ldg(reinterpret_cast<const float4 *>(ct + e));
          const float4 c = __ldg(reinterpret_cast<const float4 *>(stb + e));
          cv[e] = a.x; cv[e + 1] = a.y; cv[e + 2] = a.z; cv[e + 3] = a.w;
          sv[e] = c.x; sv[e + 1] = c.y; sv[e + 2] = c.z; sv[e + 3] = c.w;
        }
      }
    }
    float x[E];
    const uint8_t *src = ps_smem + warp * kPsRingBytes + (g % NST) * STAGE + lane * 16;
#pragma unroll
    for (int c = 0; c < CH; c++) {
      const Pack<InT, VIN> pk = *reinterpret_cast<const Pack<InT, VIN> *>(src + c * 512);
#pragma unroll
      for (int e = 0; e < VIN; e++) x[c * VIN + e] = to_f32<InT>(pk.v[e]);
    }
    const float *gain = st.t == 0 ? p.q_gain : (st.t == 1 ? p.k_gain : nullptr);
    if (gain != nullptr) {  // warp-uniform
      float ss = 0.0f;
#pragma unroll
      for (int e = 0; e < E; e++) ss = __fmaf_rn(x[e], x[e], ss);
#pragma unroll
      for (int o = kProLanesPerRow / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float rms = rsqrtf(ss / (float)D + p.eps);
#pragma unroll
      for (int e = 0; e < E; e++)
        x[e] = __fmul_rn(__fmul_rn(x[e], rms), st.t == 0 ? gq[e] : gk[e]);
    }
    if (st.t < 2 && p.cos_t != nullptr) {
#pragma unroll
      for (int e = 0; e < E; e += 2) {
        const float x0 = x[e], x1 = x[e + 1];
        x[e] = __fsub_rn(__fmul_rn(x0, cv[e / 2]), __fmul_rn(x1, sv[e / 2]));
        x[e + 1] = __fadd_rn(__fmul_rn(x0, sv[e / 2]), __fmul_rn(x1, cv[e / 2]));
      }
    }
    if (in) {
      constexpr int VOUT = 16 / sizeof(OutT);
      OutT *dst = out + (((long long)st.t * p.B + st.b) * p.H + st.h) * (long long)p.S * D +
                  (long long)st.s * D + sub * E;
#pragma unroll
      for (int c = 0; c < E / VOUT; c++) {
        Pack<OutT, VOUT> po;
#pragma unroll
        for (int e = 0; e < VOUT; e++) po.v[e] = from_f32<OutT>(x[c * VOUT + e]);
        *reinterpret_cast<Pack<OutT, VOUT> *>(dst + c * VOUT) = po;
      }
    }
  }
  cp_async_wait<0>();
}

// Head chunk for the streaming prologue: the whole H unless that leaves
// fewer items than two per SM.
inline int prologue_stream_hchunk(int B, int S, int H, int num_sms) {
  const long long blocks = (long long)B * ((S + kPsTokens - 1) / kPsTokens);
  int hc = H;
  while (hc > 1 && blocks * ((H + hc - 1) / hc) < 2LL * num_sms) hc = (hc + 1) / 2;
  return hc;
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
