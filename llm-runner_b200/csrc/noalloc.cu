// llmr_attention_fused_noalloc: the fused QK-RMSNorm + RoPE + tensor-core
// attention for callers that cannot allocate device memory.
//
// Who needs it: callers whose device memory is owned by another allocator (a
// serving runtime or host engine that reserves HBM up front and accounts for
// every byte through its own pool), and latency-critical paths that must not
// call cudaMalloc/cudaFree, which can synchronise the whole device. Such a
// caller cannot create an llmr_ctx (creating one allocates the workspace and
// an error word), so this entry point takes a stream instead of a context and
// uses a fixed scratch array compiled into the library.
//
// The scratch is a file-scope __device__ array: every GPU that loads this
// library holds LLMR_NOALLOC_SCRATCH_BYTES of it until the process exits.
// Host code cannot use the array's name as a device address (on the host it
// is only a stand-in symbol), so the address is looked up once per device
// with cudaGetSymbolAddress and cached. That set-up happens inside the first
// call on each device, with that device current; make that first call before
// any stream capture.
//
// All calls share the one array and it keeps the previous call's contents.
// The prologue kernel overwrites every scratch element the attention kernel
// then reads, so nothing has to be cleared between calls. Calls that overlap
// on the GPU (on different streams, without ordering between them) race on
// the scratch and produce wrong results.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <mutex>

#include "../../include/llmr_attn.h"
#include "fa_tc.cuh"
#include "kattr.cuh"
#include "prologue.cuh"

using namespace llmr;

static __device__ __align__(256) unsigned char g_noalloc_scratch[LLMR_NOALLOC_SCRATCH_BYTES];
// Raised by a kernel of this entry point whose bounded wait expired; read
// and cleared by llmr_noalloc_status.
static __device__ int g_noalloc_err;

namespace {

constexpr int kMaxDevices = 64;

struct DeviceSetup {
  bool done = false;
  void *scratch = nullptr;
  int *err = nullptr;
  int num_sms = 0;
};

std::mutex g_setup_mu;
DeviceSetup g_setup[kMaxDevices];

// Once per device, with that device current: device addresses of the
// scratch array and error word, and the SM count for the prologue grid.
int setup_current_device(DeviceSetup **out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return LLMR_ENODEV;
  if (dev < 0 || dev >= kMaxDevices) return LLMR_ENODEV;
  std::lock_guard<std::mutex> lock(g_setup_mu);
  DeviceSetup &s = g_setup[dev];
  if (!s.done) {
    int major = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        major != 10)
      return LLMR_ENODEV;
    if (cudaDeviceGetAttribute(&s.num_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return LLMR_ECUDA;
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess) return LLMR_ECUDA;
    s.scratch = p;
    if (cudaGetSymbolAddress(&p, g_noalloc_err) != cudaSuccess) return LLMR_ECUDA;
    s.err = static_cast<int *>(p);
    s.done = true;
  }
  *out = &s;
  return LLMR_OK;
}

typedef CUresult (*EncodeFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                             const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                             const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                             CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  }
  return fn;
}

// fp16 (d, s, h, b) tensor map, 64 x 128 box, 128-byte swizzle: the operand
// layout fa_fwd_tc_kernel expects.
int map4(CUtensorMap *m, const void *base, int D, int S, int H, int B, long long rs,
         long long hs, long long bs) {
  EncodeFn enc = encode_fn();
  if (!enc) return LLMR_ECUDA;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((rs * 2) & 15) || ((hs * 2) & 15) ||
      ((bs * 2) & 15))
    return LLMR_EINVAL;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)rs * 2, (cuuint64_t)hs * 2, (cuuint64_t)bs * 2};
  cuuint32_t box[4] = {64, 128, 1, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void *>(base), dims, strides,
             box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
                 CUDA_SUCCESS
             ? LLMR_OK
             : LLMR_ECUDA;
}

template <int D, typename InT>
int prologue(cudaStream_t st, int num_sms, const void *q, const void *k, const void *v,
             const long long *qs, const long long *ks, const long long *vs, __half *out,
             const ProParams &pp) {
  constexpr int VIN = 16 / sizeof(InT);
  View<InT> vq{static_cast<const InT *>(q), qs[0], qs[1], qs[2]};
  View<InT> vk{static_cast<const InT *>(k), ks[0], ks[1], ks[2]};
  View<InT> vv{static_cast<const InT *>(v), vs[0], vs[1], vs[2]};
  (void)num_sms;
  const dim3 blocks = prologue_grid(pp.S, pp.B * pp.H);
  auto ok = [&](const void *ptr, const long long *s) {
    return ptr == nullptr || ((reinterpret_cast<uintptr_t>(ptr) & 15) == 0 &&
                              (s == nullptr || (s[0] % VIN == 0 && s[1] % VIN == 0 && s[2] % VIN == 0)));
  };
  const bool vec = ok(q, qs) && ok(k, ks) && ok(v, vs) && ok(pp.cos_t, nullptr) &&
                   ok(pp.sin_t, nullptr);
  if (vec)
    prologue_kernel<D, InT, __half, true><<<blocks, 256, 0, st>>>(vq, vk, vv, out, pp);
  else
    prologue_kernel<D, InT, __half, false><<<blocks, 256, 0, st>>>(vq, vk, vv, out, pp);
  return cudaGetLastError() == cudaSuccess ? LLMR_OK : LLMR_ECUDA;
}

template <int D, typename OutT>
int attention(cudaStream_t st, int num_sms, const CUtensorMap &mq, const CUtensorMap &mk,
              const CUtensorMap &mv, int B, int H, int S, float scale, void *o, long long o_rs,
              long long o_bs, float *lse, int *err) {
  using C = FaCfg<D>;
  // The shared-memory limit is a per-device attribute: raised once per
  // device (thread-safe), like the rest of the per-device set-up.
  if (set_smem_once(fa_fwd_tc_kernel<D, OutT>, C::SMEM_BYTES) != cudaSuccess) return LLMR_ECUDA;
  int regs = 0;  // the register split must fit the launch allocation
  if (launch_regs(fa_fwd_tc_kernel<D, OutT>, &regs) != cudaSuccess ||
      regs * C::THREADS < C::REG_NEED)
    return LLMR_ECUDA;
  FaParams p;
  p.S = S;
  p.S_kv = S;
  p.H = H;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.o = o;
  p.o_row_stride = o_rs;
  p.o_batch_stride = o_bs;
  p.lse = lse;
  p.merge = 0;
  p.err = err;
  p.nseq = 0;
  p.seq_off[0] = 0;
  const dim3 grid = fa_grid<D>(p, B, num_sms);
  FusedPro none;  // the prologue ran as its own kernel
  memset(&none, 0, sizeof none);
  fa_fwd_tc_kernel<D, OutT><<<grid, C::THREADS, C::SMEM_BYTES, st>>>(mq, mk, mv, p, none);
  return cudaGetLastError() == cudaSuccess ? LLMR_OK : LLMR_ECUDA;
}

template <int D>
int attention_any(cudaStream_t st, int num_sms, llmr_dtype od, const CUtensorMap &mq,
                  const CUtensorMap &mk, const CUtensorMap &mv, int B, int H, int S, float scale,
                  void *o, long long o_rs, long long o_bs, float *lse, int *err) {
  if (od == LLMR_F32)
    return attention<D, float>(st, num_sms, mq, mk, mv, B, H, S, scale, o, o_rs, o_bs, lse, err);
  if (od == LLMR_F16)
    return attention<D, __half>(st, num_sms, mq, mk, mv, B, H, S, scale, o, o_rs, o_bs, lse, err);
  return attention<D, __nv_bfloat16>(st, num_sms, mq, mk, mv, B, H, S, scale, o, o_rs, o_bs, lse,
                                     err);
}

void strides_for(const llmr_attn_desc *d, uint64_t rs_in, uint64_t bs_in, uint64_t hs_in,
                 long long *out) {
  const long long H = d->n_heads, S = d->seq_len, D = d->head_dim;
  const bool bshd = d->layout == LLMR_LAYOUT_BSHD;
  out[0] = bs_in ? (long long)bs_in : S * H * D;
  out[1] = rs_in ? (long long)rs_in : (bshd ? H * D : D);
  out[2] = hs_in ? (long long)hs_in : (bshd ? D : S * D);
}

}  // namespace

extern "C" int llmr_attention_fused_noalloc(const llmr_attn_desc *d, const void *q,
                                            const void *k, const void *v,
                                            const float *q_gain, const float *k_gain,
                                            const float *cos_t, const float *sin_t, void *o,
                                            float *lse, void *stream) {
  if (!d || !q || !k || !v || !o) return LLMR_EINVAL;
  const int B = d->batch, H = d->n_heads, S = d->seq_len, D = d->head_dim;
  if (B < 1 || H < 1 || S < 1 || (D != 64 && D != 128) || (long long)B * H > 65535)
    return LLMR_EINVAL;
  if (d->in_dtype > LLMR_BF16 || d->out_dtype > LLMR_BF16 || d->layout > LLMR_LAYOUT_BHSD)
    return LLMR_EINVAL;
  if (d->flags & (LLMR_EXACT | LLMR_MERGE)) return LLMR_EINVAL;  // plain tensor-core path only
  if (d->kv_seq_len != 0 && d->kv_seq_len != d->seq_len) return LLMR_EINVAL;
  if (((d->flags & LLMR_NORM_Q) && !q_gain) || ((d->flags & LLMR_NORM_K) && !k_gain) ||
      ((d->flags & LLMR_ROPE) && (!cos_t || !sin_t)) || ((d->flags & LLMR_LSE) && !lse))
    return LLMR_EINVAL;
  if (!(d->scale > 0.0f) || !isfinite(d->scale)) return LLMR_EINVAL;
  const bool direct =
      d->in_dtype == LLMR_F16 && !(d->flags & (LLMR_NORM_Q | LLMR_NORM_K | LLMR_ROPE));
  const long long plane = (long long)B * H * S * D;
  if (!direct && (unsigned long long)plane * 3 * 2 > LLMR_NOALLOC_SCRATCH_BYTES)
    return LLMR_ENOMEM;  // beyond the fixed scratch: use llmr_attention_fused

  long long qs[3], ks[3], vs[3];
  strides_for(d, d->q_row_stride, d->q_batch_stride, d->q_head_stride, qs);
  strides_for(d, d->k_row_stride, d->k_batch_stride, d->k_head_stride, ks);
  strides_for(d, d->v_row_stride, d->v_batch_stride, d->v_head_stride, vs);
  const long long o_rs = d->o_row_stride ? (long long)d->o_row_stride : (long long)H * D;
  const long long o_bs = d->o_batch_stride ? (long long)d->o_batch_stride : (long long)S * o_rs;
  const size_t oes = d->out_dtype == LLMR_F32 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(o) & 15) || ((o_rs * (long long)oes) & 15) ||
      ((o_bs * (long long)oes) & 15))
    return LLMR_EINVAL;

  DeviceSetup *dev = nullptr;
  int rc = setup_current_device(&dev);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  CUtensorMap mq, mk, mv;
  if (direct) {
    if ((rc = map4(&mq, q, D, S, H, B, qs[1], qs[2], qs[0]))) return rc;
    if ((rc = map4(&mk, k, D, S, H, B, ks[1], ks[2], ks[0]))) return rc;
    if ((rc = map4(&mv, v, D, S, H, B, vs[1], vs[2], vs[0]))) return rc;
  } else {
    ProParams pp;
    pp.B = B;
    pp.S = S;
    pp.H = H;
    pp.split_row = (int)d->split_row;
    pp.rope_row_offset = (int)d->rope_row_offset;
    pp.eps = d->eps;
    pp.q_gain = (d->flags & LLMR_NORM_Q) ? q_gain : nullptr;
    pp.k_gain = (d->flags & LLMR_NORM_K) ? k_gain : nullptr;
    pp.cos_t = (d->flags & LLMR_ROPE) ? cos_t : nullptr;
    pp.sin_t = (d->flags & LLMR_ROPE) ? sin_t : nullptr;
    __half *w = static_cast<__half *>(dev->scratch);
    const llmr_dtype in = d->in_dtype;
    if (D == 128)
      rc = in == LLMR_F32   ? prologue<128, float>(st, dev->num_sms, q, k, v, qs, ks, vs, w, pp)
           : in == LLMR_F16 ? prologue<128, __half>(st, dev->num_sms, q, k, v, qs, ks, vs, w, pp)
                            : prologue<128, __nv_bfloat16>(st, dev->num_sms, q, k, v, qs, ks, vs, w, pp);
    else
      rc = in == LLMR_F32   ? prologue<64, float>(st, dev->num_sms, q, k, v, qs, ks, vs, w, pp)
           : in == LLMR_F16 ? prologue<64, __half>(st, dev->num_sms, q, k, v, qs, ks, vs, w, pp)
                            : prologue<64, __nv_bfloat16>(st, dev->num_sms, q, k, v, qs, ks, vs, w, pp);
    if (rc) return rc;
    const long long rs = D, hs = (long long)S * D, bs = (long long)H * S * D;
    if ((rc = map4(&mq, w, D, S, H, B, rs, hs, bs))) return rc;
    if ((rc = map4(&mk, w + plane, D, S, H, B, rs, hs, bs))) return rc;
    if ((rc = map4(&mv, w + 2 * plane, D, S, H, B, rs, hs, bs))) return rc;
  }
  float *lse_out = (d->flags & LLMR_LSE) ? lse : nullptr;
  if (D == 128)
    return attention_any<128>(st, dev->num_sms, d->out_dtype, mq, mk, mv, B, H, S, d->scale, o,
                              o_rs, o_bs, lse_out, dev->err);
  return attention_any<64>(st, dev->num_sms, d->out_dtype, mq, mk, mv, B, H, S, d->scale, o,
                           o_rs, o_bs, lse_out, dev->err);
}

extern "C" int llmr_noalloc_status(void *stream) {
  DeviceSetup *dev = nullptr;
  int rc = setup_current_device(&dev);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int h = 0;
  if (cudaMemcpyAsync(&h, dev->err, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return LLMR_ECUDA;
  if (h == 0) return LLMR_OK;
  if (cudaMemsetAsync(dev->err, 0, sizeof(int), st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return LLMR_ECUDA;
  return LLMR_ETIMEOUT;
}
