// C-ABI implementation of include/llmr_attn.h for sm_100a.
//
// Host side of the drop-in boundary: context and workspace management, TMA
// tensor-map construction, argument validation and the kernel launches that
// replace the reference's Vulkan dispatches for this op
// (lib/vulkan/compute.c3:86-133 dispatch_kernel; the call sites are
// dependencies/flux.c3l/flux_dit.c3:812-872, dependencies/zimage.c3l/
// dit.c3:1445-1483, dependencies/qwen_edit.c3l/mmdit.c3:577-678,
// dependencies/depth_anything.c3l/depth_anything.c3:610-630).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <string>

#include "../../include/llmr_attn.h"
#include "exact_tc.cuh"
#include "fa_tc.cuh"
#include "fa_wide.cuh"
#include "kattr.cuh"
#include "kernels_misc.cuh"
#include "qkv_proj.cuh"

using namespace llmr;

constexpr size_t kSyncInts = 1 + 65536;

struct llmr_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  bool own_stream = false;
  void *ws = nullptr;
  size_t ws_bytes = 0;
  int *d_err = nullptr;
  int *d_sync = nullptr;  // fused-prologue piece counters (self-resetting)
  unsigned long long *timeline = nullptr;  // LLMR_TIMELINE builds: event buffer
  uint64_t launches = 0;
  int num_sms = 0;
  bool prof_on = false;
  bool prof_valid = false;
  cudaEvent_t prof_ev[3] = {nullptr, nullptr, nullptr};
  std::string err;
};

namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t,
                                  void *, const cuuint64_t *, const cuuint64_t *,
                                  const cuuint32_t *, const cuuint32_t *,
                                  CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);

int fail(llmr_ctx *ctx, int code, const char *fmt, ...) {
  if (ctx) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    ctx->err = buf;
  }
  return code;
}

#define CUDA_TRY(ctx, call)                                                   \
  do {                                                                        \
    cudaError_t e_ = (call);                                                  \
    if (e_ != cudaSuccess)                                                    \
      return fail(ctx, LLMR_ECUDA, "%s: %s", #call, cudaGetErrorString(e_));  \
  } while (0)

// Checks the launch that was just enqueued.
int after_launch(llmr_ctx *ctx, const char *what) {
  ctx->launches++;
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return fail(ctx, LLMR_ECUDA, "%s launch: %s", what, cudaGetErrorString(e));
  return LLMR_OK;
}

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 4-D fp16 tensor map over (d, s, h, b) with a 64 x box_rows x 1 x 1 box and
// 128-byte swizzle: one box is one SW128 K-major operand chunk.
int make_map(llmr_ctx *ctx, CUtensorMap *map, const void *base, int D, int S,
             int H, int B, long long rs, long long hs, long long bs, int box_rows = 128) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return fail(ctx, LLMR_ECUDA, "cuTensorMapEncodeTiled unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((rs * 2) & 15) || ((hs * 2) & 15) ||
      ((bs * 2) & 15))
    return fail(ctx, LLMR_EINVAL, "TMA operand base/strides must be 16-byte aligned");
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)rs * 2, (cuuint64_t)hs * 2, (cuuint64_t)bs * 2};
  cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void *>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ctx, LLMR_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return LLMR_OK;
}

// 2-D 16-bit tensor map over `rows` rows of `inner` elements (row stride
// `row_stride` elements) with a 64 x box_rows box and 128-byte swizzle.
int make_map2d(llmr_ctx *ctx, CUtensorMap *map, const void *base, long long inner,
               long long rows, long long row_stride, int box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return fail(ctx, LLMR_ECUDA, "cuTensorMapEncodeTiled unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((row_stride * 2) & 15))
    return fail(ctx, LLMR_EINVAL, "TMA operand base/row stride must be 16-byte aligned");
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_stride * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ctx, LLMR_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return LLMR_OK;
}

// 4-D fp32 tensor map over (inner, rows, h, b) with a 32 x box_rows x 1 x 1
// box and 128-byte swizzle (one SW128 K-major tf32 operand chunk).
int make_map_f32(llmr_ctx *ctx, CUtensorMap *map, const void *base, int D, int S, int H, int B,
                 long long rs, long long hs, long long bs, int box_rows = 128) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return fail(ctx, LLMR_ECUDA, "cuTensorMapEncodeTiled unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((rs * 4) & 15) || ((hs * 4) & 15) ||
      ((bs * 4) & 15))
    return fail(ctx, LLMR_EINVAL, "TMA operand base/strides must be 16-byte aligned");
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)rs * 4, (cuuint64_t)hs * 4, (cuuint64_t)bs * 4};
  cuuint32_t box[4] = {32, (cuuint32_t)box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<void *>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ctx, LLMR_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return LLMR_OK;
}

template <int D, int BN, bool BF16>
int launch_qkv(llmr_ctx *ctx, const void *x, long long x_rs, const void *w, QkvParams &p,
               long long hidden) {
  using C = QkvCfg<D, BN>;
  CUDA_TRY(ctx, set_smem_once(qkv_proj_kernel<D, BN, BF16>, C::SMEM_BYTES));
  CUtensorMap mx, mw;
  int rc;
  if ((rc = make_map2d(ctx, &mx, x, hidden, p.M, x_rs, C::BM))) return rc;
  if ((rc = make_map2d(ctx, &mw, w, hidden, 3LL * p.H * D, hidden, BN))) return rc;
  const int sms = ctx->num_sms > 0 ? ctx->num_sms : 148;
  const int grid = p.tiles < sms ? p.tiles : sms;
  qkv_proj_kernel<D, BN, BF16><<<grid, C::THREADS, C::SMEM_BYTES, ctx->stream>>>(mx, mw, p);
  return after_launch(ctx, "qkv_proj");
}

template <bool BF16>
int launch_out_proj(llmr_ctx *ctx, const CUtensorMap &mx, const CUtensorMap &mw0,
                    const CUtensorMap &mw1, const ProjParams &p) {
  using C = QkvCfg<128, 256>;
  CUDA_TRY(ctx, set_smem_once(out_proj_kernel<BF16>, kProjSmemBytes));
  const int sms = ctx->num_sms > 0 ? ctx->num_sms : 148;
  const int grid = p.tiles < sms ? p.tiles : sms;
  out_proj_kernel<BF16><<<grid, C::THREADS, kProjSmemBytes, ctx->stream>>>(mx, mw0, mw1, p);
  return after_launch(ctx, "out_proj");
}

template <int D, bool BF16>
int launch_qkv_pair(llmr_ctx *ctx, const void *x, long long x_rs, const void *w, QkvParams &p,
                    long long hidden) {
  using C = Qkv2Cfg<D>;
  CUDA_TRY(ctx, set_smem_once(qkv_proj_pair_kernel<D, BF16>, C::SMEM_BYTES));
  CUtensorMap mx, mw;
  int rc;
  if ((rc = make_map2d(ctx, &mx, x, hidden, p.M, x_rs, C::BM))) return rc;
  if ((rc = make_map2d(ctx, &mw, w, hidden, 3LL * p.H * D, hidden, C::BN / 2))) return rc;
  const int pair_tiles = (p.M + 2 * C::BM - 1) / (2 * C::BM) * p.n_tiles;
  const int pairs_max = (ctx->num_sms > 0 ? ctx->num_sms : 148) / 2;
  const int grid = 2 * (pair_tiles < pairs_max ? pair_tiles : pairs_max);
  qkv_proj_pair_kernel<D, BF16><<<grid, C::THREADS, C::SMEM_BYTES, ctx->stream>>>(mx, mw, p);
  return after_launch(ctx, "qkv_proj_pair");
}

// fused != nullptr: the prologue runs inside the attention kernel (InT is
// the raw input type); the launch is cooperative (all CTAs resident).
template <int D, typename OutT, typename InT = void>
int launch_fa_tc(llmr_ctx *ctx, const CUtensorMap &mq, const CUtensorMap &mk,
                 const CUtensorMap &mv, int B, int H, int S, int S_kv, float scale, void *o,
                 long long o_rs, long long o_bs, float *lse, int merge, int nseq,
                 const int *seq_off, bool pdl, const FusedPro *fused = nullptr) {
  using C = FaCfg<D>;
  auto kern = fa_fwd_tc_kernel<D, OutT, InT>;
  CUDA_TRY(ctx, set_smem_once(kern, C::SMEM_BYTES));
  // setmaxnreg.inc waits until the registers it asks for are free within
  // the block's launch allocation: never launch a split that cannot fit.
  int regs = 0;
  CUDA_TRY(ctx, launch_regs(kern, &regs));
  if (regs * C::THREADS < C::REG_NEED)
    return fail(ctx, LLMR_ECUDA, "fa_fwd_tc: %d launch registers per thread are too few "
                "for the register split", regs);
  FaParams p;
  p.S = S;
  p.S_kv = S_kv;
  p.H = H;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.o = o;
  p.o_row_stride = o_rs;
  p.o_batch_stride = o_bs;
  p.lse = lse;
  p.merge = merge;
  p.err = ctx->d_err;
  p.timeline = ctx->timeline;
  p.nseq = seq_off != nullptr ? nseq : 0;
  p.seq_off[0] = 0;
  for (int i = 0; i <= p.nseq && p.nseq > 0; i++) p.seq_off[i] = seq_off[i];
  const dim3 grid = fa_grid<D>(p, B, ctx->num_sms);
  FusedPro fp;
  memset(&fp, 0, sizeof fp);
  if (fused) {
    fp = *fused;
    // The start-up phase writes K'/V' of every (b, h) the first round of
    // units touches (units are ordered by (b, h)).
    const int first_round = (int)grid.x < p.units ? (int)grid.x : p.units;
    fp.startup_bh = (first_round - 1) / p.nqt + 1;
  }
  if (!pdl && !fused) {
    kern<<<grid, C::THREADS, C::SMEM_BYTES, ctx->stream>>>(mq, mk, mv, p, fp);
    return after_launch(ctx, "fa_fwd_tc");
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(C::THREADS);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[1];
  if (fused) {
    // CTAs wait for prologue pieces written by other CTAs: all must be
    // resident at once, which a cooperative launch guarantees (one CTA per
    // SM at most).
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
  } else {
    // Right behind the prologue on the same stream: programmatic dependent
    // launch lets this grid's CTAs start (barrier init, TMEM allocation) on
    // SMs the prologue has left; the kernel waits for the prologue's results.
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
  }
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  CUDA_TRY(ctx, cudaLaunchKernelEx(&cfg, kern, mq, mk, mv, p, fp));
  return after_launch(ctx, fused ? "fa_fwd_tc(fused prologue)" : "fa_fwd_tc");
}

template <int D, typename InT>
int launch_fa_fused_t(llmr_ctx *ctx, llmr_dtype od, const CUtensorMap &mq, const CUtensorMap &mk,
                      const CUtensorMap &mv, int B, int H, int S, float scale, void *o,
                      long long o_rs, long long o_bs, float *lse, const FusedPro &fp) {
#define LLMR_FU_ARGS ctx, mq, mk, mv, B, H, S, S, scale, o, o_rs, o_bs, lse, 0, 0, nullptr, false, &fp
  if (od == LLMR_F32) return launch_fa_tc<D, float, InT>(LLMR_FU_ARGS);
  if (od == LLMR_F16) return launch_fa_tc<D, __half, InT>(LLMR_FU_ARGS);
  return launch_fa_tc<D, __nv_bfloat16, InT>(LLMR_FU_ARGS);
#undef LLMR_FU_ARGS
}

int launch_fa_tc_any(llmr_ctx *ctx, int D, llmr_dtype od, const CUtensorMap &mq,
                     const CUtensorMap &mk, const CUtensorMap &mv, int B, int H, int S, int S_kv,
                     float scale, void *o, long long o_rs, long long o_bs, float *lse,
                     int merge, int nseq = 0, const int *seq_off = nullptr,
                     bool pdl = false) {
#define LLMR_FA_ARGS ctx, mq, mk, mv, B, H, S, S_kv, scale, o, o_rs, o_bs, lse
  if (D == 128) {
    if (od == LLMR_F32) return launch_fa_tc<128, float>(LLMR_FA_ARGS, merge, nseq, seq_off, pdl);
    if (od == LLMR_F16) return launch_fa_tc<128, __half>(LLMR_FA_ARGS, 0, nseq, seq_off, pdl);
    return launch_fa_tc<128, __nv_bfloat16>(LLMR_FA_ARGS, 0, nseq, seq_off, pdl);
  }
  if (od == LLMR_F32) return launch_fa_tc<64, float>(LLMR_FA_ARGS, merge, nseq, seq_off, pdl);
  if (od == LLMR_F16) return launch_fa_tc<64, __half>(LLMR_FA_ARGS, 0, nseq, seq_off, pdl);
  return launch_fa_tc<64, __nv_bfloat16>(LLMR_FA_ARGS, 0, nseq, seq_off, pdl);
#undef LLMR_FA_ARGS
}

// LLMR_FUSED_PROLOGUE=1 runs the prologue inside the attention kernel (one
// cooperative launch) instead of as its own kernel launched ahead of it.
// Measured slower on B200 (the start-up pieces and the background warps are
// latency-bound and slow the softmax warps), so it is not the default.
bool fused_prologue_enabled() {
  static const bool v = getenv("LLMR_FUSED_PROLOGUE") != nullptr;
  return v;
}

// LLMR_NO_PDL launches the attention kernel after the prologue without
// programmatic dependent launch (for comparisons).
bool pdl_disabled() {
  static const bool v = getenv("LLMR_NO_PDL") != nullptr;
  return v;
}

template <int D, typename InT, typename OutT>
int launch_prologue_t(llmr_ctx *ctx, const void *q, const void *k, const void *v,
                      const long long *qs, const long long *ks, const long long *vs,
                      OutT *out, const ProParams &pp) {
  View<InT> vq{static_cast<const InT *>(q), qs[0], qs[1], qs[2]};
  View<InT> vk{static_cast<const InT *>(k), ks[0], ks[1], ks[2]};
  View<InT> vv{static_cast<const InT *>(v), vs[0], vs[1], vs[2]};
  const dim3 blocks = prologue_grid(pp.S, pp.B * pp.H);
  // 16-byte vector accesses per lane need 16-byte aligned bases and strides
  // that are whole 16-byte multiples (the tables' rows always are).
  constexpr int VIN = 16 / sizeof(InT);
  auto ok = [&](const void *ptr, const long long *st) {
    return ptr == nullptr ||
           ((reinterpret_cast<uintptr_t>(ptr) & 15) == 0 &&
            (st == nullptr || (st[0] % VIN == 0 && st[1] % VIN == 0 && st[2] % VIN == 0)));
  };
  const bool vec = ok(q, qs) && ok(k, ks) && ok(v, vs) && ok(pp.cos_t, nullptr) &&
                   ok(pp.sin_t, nullptr);
  if (vec)
    prologue_kernel<D, InT, OutT, true><<<blocks, 256, 0, ctx->stream>>>(vq, vk, vv, out, pp);
  else
    prologue_kernel<D, InT, OutT, false><<<blocks, 256, 0, ctx->stream>>>(vq, vk, vv, out, pp);
  return after_launch(ctx, "prologue");
}

template <typename OutT>
int launch_prologue(llmr_ctx *ctx, int D, llmr_dtype in, const void *q, const void *k,
                    const void *v, const long long *qs, const long long *ks,
                    const long long *vs, OutT *out, const ProParams &pp) {
#define PRO_CASE(DD, T) return launch_prologue_t<DD, T, OutT>(ctx, q, k, v, qs, ks, vs, out, pp)
  if (D == 128) {
    if (in == LLMR_F32) PRO_CASE(128, float);
    if (in == LLMR_F16) PRO_CASE(128, __half);
    PRO_CASE(128, __nv_bfloat16);
  }
  if (in == LLMR_F32) PRO_CASE(64, float);
  if (in == LLMR_F16) PRO_CASE(64, __half);
  PRO_CASE(64, __nv_bfloat16);
#undef PRO_CASE
}

unsigned grid_for(llmr_ctx *ctx, long long n, int threads) {
  long long b = (n + threads - 1) / threads;
  const long long cap = (long long)ctx->num_sms * 16;
  if (b > cap) b = cap;
  if (b < 1) b = 1;
  return (unsigned)b;
}

// LLMR_EXACT_SIMT keeps the exact path on the SIMT kernel even where the
// tensor-core (3xTF32) kernel applies (for comparisons).
bool exact_simt_forced() {
  static const bool v = getenv("LLMR_EXACT_SIMT") != nullptr;
  return v;
}

// Workspace floats the tensor-core exact kernel needs besides its inputs:
// the TF32 big and residual parts of Q and K, and of V transposed (keys
// padded to a multiple of 4 per row).
long long exact_tc_extra_floats(long long B, long long H, long long S, long long D) {
  const long long Sp = (S + 3) / 4 * 4;
  return 4 * B * H * S * D + 2 * B * H * D * Sp;
}

// Exact attention on the tensor cores (D = 64): q, k, v dense fp32
// [B][H][S][D]; extra: exact_tc_extra_floats(...) floats of workspace.
int launch_exact_tc(llmr_ctx *ctx, const float *q, const float *k, const float *v, float *extra,
                    const ExactParams &ep) {
  using C = ExactTcCfg;
  const int D = C::D, B = ep.B, H = ep.H, S = ep.S;
  const int Sp = (S + 3) / 4 * 4;
  const long long n = (long long)B * H * S * D, nt = (long long)B * H * D * Sp;
  float *qg = extra, *qr = extra + n, *kg = extra + 2 * n, *kr = extra + 3 * n;
  float *vtg = extra + 4 * n, *vtr = vtg + nt;
  dim3 pgrid((S + 31) / 32, D / 32, B * H);
  tf32_prepare_kernel<<<pgrid, 256, 0, ctx->stream>>>(q, k, v, qg, qr, kg, kr, vtg, vtr, S, Sp, D);
  int rc = after_launch(ctx, "tf32_prepare");
  if (rc) return rc;
  const long long rs = D, hs = (long long)S * D, bs = (long long)H * S * D;
  const long long trs = Sp, ths = (long long)D * Sp, tbs = (long long)H * D * Sp;
  CUtensorMap mq, mk, mv, mqr, mkr, mvr;
  if ((rc = make_map_f32(ctx, &mq, qg, D, S, H, B, rs, hs, bs))) return rc;
  if ((rc = make_map_f32(ctx, &mk, kg, D, S, H, B, rs, hs, bs))) return rc;
  if ((rc = make_map_f32(ctx, &mqr, qr, D, S, H, B, rs, hs, bs))) return rc;
  if ((rc = make_map_f32(ctx, &mkr, kr, D, S, H, B, rs, hs, bs))) return rc;
  if ((rc = make_map_f32(ctx, &mv, vtg, S, D, H, B, trs, ths, tbs, 64))) return rc;
  if ((rc = make_map_f32(ctx, &mvr, vtr, S, D, H, B, trs, ths, tbs, 64))) return rc;
  CUDA_TRY(ctx, set_smem_once(attn_exact_tc_kernel, C::SMEM_BYTES));
  dim3 grid((S + C::BM - 1) / C::BM, B * H);
  attn_exact_tc_kernel<<<grid, C::THREADS, C::SMEM_BYTES, ctx->stream>>>(mq, mk, mv, mqr, mkr,
                                                                         mvr, ep, ctx->d_err);
  return after_launch(ctx, "attn_exact_tc");
}

bool exact_tc_applies(int D, const void *q, const void *k, const void *v) {
  auto al = [](const void *ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
  return D == 64 && al(q) && al(k) && al(v) && !exact_simt_forced();
}

int launch_exact(llmr_ctx *ctx, int D, const float *q, const float *k, const float *v,
                 const ExactParams &ep) {
  const int rows_per_cta = D == 128 ? 16 : 32;
  dim3 grid((ep.S + rows_per_cta - 1) / rows_per_cta, ep.B * ep.H);
  if (D == 128)
    attn_exact_f32_kernel<128><<<grid, 128, 0, ctx->stream>>>(q, k, v, ep);
  else
    attn_exact_f32_kernel<64><<<grid, 128, 0, ctx->stream>>>(q, k, v, ep);
  return after_launch(ctx, "attn_exact_f32");
}


size_t dtype_size(llmr_dtype t) { return t == LLMR_F32 ? 4 : 2; }

bool aligned16(const void *p, long long elems_a, long long elems_b, size_t es) {
  return (reinterpret_cast<uintptr_t>(p) & 15) == 0 && ((elems_a * (long long)es) & 15) == 0 &&
         ((elems_b * (long long)es) & 15) == 0;
}

int check_ctx(llmr_ctx *ctx) {
  if (!ctx) return LLMR_EINVAL;
  CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  return LLMR_OK;
}

// Fills default strides for a desc (elements). Order: {batch, row, head}.
void default_strides(const llmr_attn_desc *d, uint64_t rs_in, uint64_t bs_in, uint64_t hs_in,
                     long long *out, long long rows) {
  const long long H = d->n_heads, S = rows, D = d->head_dim;
  long long rs, hs, bs;
  if (d->layout == LLMR_LAYOUT_BSHD) {
    rs = H * D;
    hs = D;
    bs = S * H * D;
  } else {
    rs = D;
    hs = S * D;
    bs = H * S * D;
  }
  out[0] = bs_in ? (long long)bs_in : bs;
  out[1] = rs_in ? (long long)rs_in : rs;
  out[2] = hs_in ? (long long)hs_in : hs;
}

// ---------------------------------------------------------------- wide heads

// The largest dynamic shared memory a block of this device may opt into.
int smem_optin(llmr_ctx *ctx) {
  int v = 0;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, ctx->device) !=
      cudaSuccess)
    return 0;
  return v;
}

template <int D, typename OutT>
int launch_fa_wide(llmr_ctx *ctx, const CUtensorMap &mq, const CUtensorMap &mk,
                   const CUtensorMap &mv, int B, int H, int S, int S_kv, float scale, void *o,
                   long long o_rs, long long o_bs, float *lse) {
  using C = FaWideCfg<D>;
  if (smem_optin(ctx) < C::SMEM_BYTES)
    return fail(ctx, LLMR_ECUDA, "fa_wide_tc needs %d bytes of shared memory per block",
                C::SMEM_BYTES);
  CUDA_TRY(ctx, set_smem_once(fa_wide_tc_kernel<D, OutT>, C::SMEM_BYTES));
  FaParams p;
  memset(&p, 0, sizeof p);
  p.S = S;
  p.S_kv = S_kv;
  p.H = H;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.o = o;
  p.o_row_stride = o_rs;
  p.o_batch_stride = o_bs;
  p.lse = lse;
  p.err = ctx->d_err;
  const dim3 grid = fa_wide_grid<D>(p, B, ctx->num_sms);
  fa_wide_tc_kernel<D, OutT><<<grid, C::THREADS, C::SMEM_BYTES, ctx->stream>>>(mq, mk, mv, p);
  return after_launch(ctx, "fa_wide_tc");
}

template <int D, typename OutT>
int launch_fa_wide_pair(llmr_ctx *ctx, const CUtensorMap &mq, const CUtensorMap &mk,
                        const CUtensorMap &mv, int B, int H, int S, int S_kv, float scale,
                        void *o, long long o_rs, long long o_bs, float *lse) {
  using C = FaWide2Cfg<D>;
  if (smem_optin(ctx) < C::SMEM_BYTES)
    return fail(ctx, LLMR_ECUDA, "fa_wide_pair needs %d bytes of shared memory per block",
                C::SMEM_BYTES);
  CUDA_TRY(ctx, set_smem_once(fa_wide_pair_kernel<D, OutT>, C::SMEM_BYTES));
  FaParams p;
  memset(&p, 0, sizeof p);
  p.S = S;
  p.S_kv = S_kv;
  p.H = H;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.o = o;
  p.o_row_stride = o_rs;
  p.o_batch_stride = o_bs;
  p.lse = lse;
  p.err = ctx->d_err;
  const dim3 grid = fa_wide_pair_grid<D>(p, B, ctx->num_sms);
  fa_wide_pair_kernel<D, OutT><<<grid, C::THREADS, C::SMEM_BYTES, ctx->stream>>>(mq, mk, mv, p);
  return after_launch(ctx, "fa_wide_pair");
}

// The pair kernel is the default; LLMR_WIDE_SINGLE_CTA selects the
// single-CTA kernel.
bool wide_single_cta() { return getenv("LLMR_WIDE_SINGLE_CTA") != nullptr; }

// single: the single-CTA kernel (mk with 128-row boxes like mq and mv), else
// the pair kernel (mk with 64-row boxes: each CTA loads 64 keys per block).
int launch_fa_wide_any(llmr_ctx *ctx, bool single, int D, llmr_dtype od, const CUtensorMap &mq,
                       const CUtensorMap &mk, const CUtensorMap &mv, int B, int H, int S,
                       int S_kv, float scale, void *o, long long o_rs, long long o_bs,
                       float *lse) {
#define LLMR_WIDE_ARGS ctx, mq, mk, mv, B, H, S, S_kv, scale, o, o_rs, o_bs, lse
  if (single) {
    if (D == 512) {
      if (od == LLMR_F32) return launch_fa_wide<512, float>(LLMR_WIDE_ARGS);
      if (od == LLMR_F16) return launch_fa_wide<512, __half>(LLMR_WIDE_ARGS);
      return launch_fa_wide<512, __nv_bfloat16>(LLMR_WIDE_ARGS);
    }
    if (od == LLMR_F32) return launch_fa_wide<384, float>(LLMR_WIDE_ARGS);
    if (od == LLMR_F16) return launch_fa_wide<384, __half>(LLMR_WIDE_ARGS);
    return launch_fa_wide<384, __nv_bfloat16>(LLMR_WIDE_ARGS);
  }
  if (D == 512) {
    if (od == LLMR_F32) return launch_fa_wide_pair<512, float>(LLMR_WIDE_ARGS);
    if (od == LLMR_F16) return launch_fa_wide_pair<512, __half>(LLMR_WIDE_ARGS);
    return launch_fa_wide_pair<512, __nv_bfloat16>(LLMR_WIDE_ARGS);
  }
  if (od == LLMR_F32) return launch_fa_wide_pair<384, float>(LLMR_WIDE_ARGS);
  if (od == LLMR_F16) return launch_fa_wide_pair<384, __half>(LLMR_WIDE_ARGS);
  return launch_fa_wide_pair<384, __nv_bfloat16>(LLMR_WIDE_ARGS);
#undef LLMR_WIDE_ARGS
}

template <typename InT, typename OutT>
int launch_wide_cast_t(llmr_ctx *ctx, const void *q, const void *k, const void *v,
                       const long long *qs, const long long *ks, const long long *vs, OutT *out,
                       int B, int H, int S, int D) {
  View<InT> vq{static_cast<const InT *>(q), qs[0], qs[1], qs[2]};
  View<InT> vk{static_cast<const InT *>(k), ks[0], ks[1], ks[2]};
  View<InT> vv{static_cast<const InT *>(v), vs[0], vs[1], vs[2]};
  constexpr int VIN = 16 / sizeof(InT);
  auto ok = [&](const void *ptr, const long long *st) {
    return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0 && st[0] % VIN == 0 &&
           st[1] % VIN == 0 && st[2] % VIN == 0;
  };
  const bool vec = ok(q, qs) && ok(k, ks) && ok(v, vs);
  const long long groups = (long long)B * H * S * (D / 8);
  const dim3 grid(grid_for(ctx, groups, 256), 3);
  if (vec)
    wide_cast_kernel<InT, OutT, true><<<grid, 256, 0, ctx->stream>>>(vq, vk, vv, out, B, H, S, D);
  else
    wide_cast_kernel<InT, OutT, false><<<grid, 256, 0, ctx->stream>>>(vq, vk, vv, out, B, H, S, D);
  return after_launch(ctx, "wide_cast");
}

template <typename OutT>
int launch_wide_cast(llmr_ctx *ctx, llmr_dtype in, const void *q, const void *k, const void *v,
                     const long long *qs, const long long *ks, const long long *vs, OutT *out,
                     int B, int H, int S, int D) {
  if (in == LLMR_F32) return launch_wide_cast_t<float, OutT>(ctx, q, k, v, qs, ks, vs, out, B, H, S, D);
  if (in == LLMR_F16) return launch_wide_cast_t<__half, OutT>(ctx, q, k, v, qs, ks, vs, out, B, H, S, D);
  return launch_wide_cast_t<__nv_bfloat16, OutT>(ctx, q, k, v, qs, ks, vs, out, B, H, S, D);
}

template <int D>
int launch_exact_wide_t(llmr_ctx *ctx, const float *q, const float *k, const float *v,
                        const ExactParams &ep) {
  constexpr int smem = exact_wide_smem(D);
  if (smem_optin(ctx) < smem)
    return fail(ctx, LLMR_ECUDA, "attn_exact_wide needs %d bytes of shared memory", smem);
  CUDA_TRY(ctx, set_smem_once(attn_exact_wide_kernel<D>, smem));
  constexpr int rows_per_cta = 4 * kExactWideRows;
  dim3 grid((ep.S + rows_per_cta - 1) / rows_per_cta, ep.B * ep.H);
  attn_exact_wide_kernel<D><<<grid, 128, smem, ctx->stream>>>(q, k, v, ep);
  return after_launch(ctx, "attn_exact_wide");
}

bool is_wide(int D) { return D == 384 || D == 512; }

}  // namespace

extern "C" {

int llmr_ctx_create(int device, size_t workspace_bytes, void *stream, llmr_ctx **out) {
  if (!out) return LLMR_EINVAL;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return LLMR_ENODEV;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return LLMR_ENODEV;
  if (prop.major != 10) return LLMR_ENODEV;  // sm_100a code only
  llmr_ctx *c = new llmr_ctx();
  c->device = device;
  c->num_sms = prop.multiProcessorCount;
  if (cudaSetDevice(device) != cudaSuccess) { delete c; return LLMR_ECUDA; }
  if (stream) {
    c->stream = static_cast<cudaStream_t>(stream);
  } else {
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) {
      delete c;
      return LLMR_ECUDA;
    }
    c->own_stream = true;
  }
  if (cudaMalloc(&c->d_err, sizeof(int)) != cudaSuccess ||
      cudaMemset(c->d_err, 0, sizeof(int)) != cudaSuccess) {
    llmr_ctx_destroy(c);
    return LLMR_ENOMEM;
  }
  // One counter per (b, h) (batch * n_heads <= 65535) plus the CTA count.
  if (cudaMalloc(&c->d_sync, kSyncInts * sizeof(int)) != cudaSuccess ||
      cudaMemset(c->d_sync, 0, kSyncInts * sizeof(int)) != cudaSuccess) {
    llmr_ctx_destroy(c);
    return LLMR_ENOMEM;
  }
  if (workspace_bytes && cudaMalloc(&c->ws, workspace_bytes) != cudaSuccess) {
    llmr_ctx_destroy(c);
    return LLMR_ENOMEM;
  }
  c->ws_bytes = workspace_bytes;
  *out = c;
  return LLMR_OK;
}

int llmr_ctx_destroy(llmr_ctx *ctx) {
  if (!ctx) return LLMR_EINVAL;
  cudaSetDevice(ctx->device);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  if (ctx->ws) cudaFree(ctx->ws);
  if (ctx->d_err) cudaFree(ctx->d_err);
  if (ctx->d_sync) cudaFree(ctx->d_sync);
  for (cudaEvent_t &e : ctx->prof_ev)
    if (e) cudaEventDestroy(e);
  if (ctx->own_stream && ctx->stream) cudaStreamDestroy(ctx->stream);
  delete ctx;
  return LLMR_OK;
}

int llmr_ctx_reserve(llmr_ctx *ctx, size_t bytes) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if (bytes <= ctx->ws_bytes) return LLMR_OK;
  CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
  if (ctx->ws) cudaFree(ctx->ws);
  ctx->ws = nullptr;
  ctx->ws_bytes = 0;
  if (cudaMalloc(&ctx->ws, bytes) != cudaSuccess)
    return fail(ctx, LLMR_ENOMEM, "workspace of %zu bytes: cudaMalloc failed", bytes);
  ctx->ws_bytes = bytes;
  return LLMR_OK;
}

int llmr_set_stream(llmr_ctx *ctx, void *stream) {
  if (!ctx || !stream) return LLMR_EINVAL;
  if (ctx->own_stream) {
    cudaStreamSynchronize(ctx->stream);
    cudaStreamDestroy(ctx->stream);
    ctx->own_stream = false;
  }
  ctx->stream = static_cast<cudaStream_t>(stream);
  return LLMR_OK;
}

int llmr_timeline_set(llmr_ctx *ctx, void *device_buffer, size_t bytes) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
#ifdef LLMR_TIMELINE
  if (device_buffer && bytes < (size_t)ctx->num_sms * kTimelineSlots * 8)
    return fail(ctx, LLMR_EINVAL, "timeline buffer needs %zu bytes",
                (size_t)ctx->num_sms * kTimelineSlots * 8);
  ctx->timeline = static_cast<unsigned long long *>(device_buffer);
  return LLMR_OK;
#else
  (void)device_buffer;
  (void)bytes;
  return fail(ctx, LLMR_EINVAL, "built without LLMR_TIMELINE");
#endif
}

int llmr_ctx_set_sm_budget(llmr_ctx *ctx, int sms) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  int all = 0;
  CUDA_TRY(ctx, cudaDeviceGetAttribute(&all, cudaDevAttrMultiProcessorCount, ctx->device));
  if (sms < 0 || sms > all) return fail(ctx, LLMR_EINVAL, "sm budget %d outside [0, %d]", sms, all);
  ctx->num_sms = sms == 0 ? all : sms;
  return LLMR_OK;
}

void *llmr_get_stream(llmr_ctx *ctx) { return ctx ? ctx->stream : nullptr; }

const char *llmr_last_error(llmr_ctx *ctx) { return ctx ? ctx->err.c_str() : "null context"; }

uint64_t llmr_launch_count(llmr_ctx *ctx) { return ctx ? ctx->launches : 0; }

int llmr_sync(llmr_ctx *ctx) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
  int h = 0;
  CUDA_TRY(ctx, cudaMemcpy(&h, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (h) {
    CUDA_TRY(ctx, cudaMemset(ctx->d_err, 0, sizeof(int)));
    return fail(ctx, LLMR_ETIMEOUT, "a device-side wait exceeded its limit; results are invalid");
  }
  return LLMR_OK;
}

int llmr_selftest_wait_timeout(llmr_ctx *ctx, uint64_t limit_ns) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if (limit_ns == 0 || limit_ns > 1000000000ull)
    return fail(ctx, LLMR_EINVAL, "limit_ns must be in (0, 1e9]");
  wait_timeout_probe_kernel<<<1, 32, 0, ctx->stream>>>(ctx->d_err, limit_ns);
  return after_launch(ctx, "wait_timeout_probe");
}

int llmr_alloc(llmr_ctx *ctx, size_t bytes, void **out) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if (!out) return fail(ctx, LLMR_EINVAL, "null out pointer");
  if (cudaMalloc(out, bytes) != cudaSuccess)
    return fail(ctx, LLMR_ENOMEM, "cudaMalloc(%zu) failed", bytes);
  return LLMR_OK;
}

int llmr_free(llmr_ctx *ctx, void *ptr) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  CUDA_TRY(ctx, cudaFree(ptr));
  return LLMR_OK;
}

int llmr_upload(llmr_ctx *ctx, void *dst, const void *src, size_t bytes) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  CUDA_TRY(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream));
  CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
  return LLMR_OK;
}

int llmr_download(llmr_ctx *ctx, void *dst, const void *src, size_t bytes) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  CUDA_TRY(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream));
  CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
  return LLMR_OK;
}

static_assert(sizeof(llmr_ipc_handle) == sizeof(cudaIpcMemHandle_t), "ipc handle size");

int llmr_ipc_export(llmr_ctx *ctx, void *base, llmr_ipc_handle *out) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if (!base || !out) return fail(ctx, LLMR_EINVAL, "null pointer");
  cudaIpcMemHandle_t h;
  CUDA_TRY(ctx, cudaIpcGetMemHandle(&h, base));
  memcpy(out->bytes, &h, sizeof(h));
  return LLMR_OK;
}

int llmr_ipc_open(llmr_ctx *ctx, const llmr_ipc_handle *handle, void **out) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if (!handle || !out) return fail(ctx, LLMR_EINVAL, "null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle->bytes, sizeof(h));
  CUDA_TRY(ctx, cudaIpcOpenMemHandle(out, h, cudaIpcMemLazyEnablePeerAccess));
  return LLMR_OK;
}

int llmr_ipc_close(llmr_ctx *ctx, void *mapped) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if (!mapped) return fail(ctx, LLMR_EINVAL, "null pointer");
  CUDA_TRY(ctx, cudaIpcCloseMemHandle(mapped));
  return LLMR_OK;
}

int llmr_copy_async(llmr_ctx *ctx, void *dst, const void *src, size_t bytes, void *stream) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if (bytes == 0) return LLMR_OK;
  if (!dst || !src) return fail(ctx, LLMR_EINVAL, "null pointer");
  cudaStream_t s = stream ? (cudaStream_t)stream : ctx->stream;
  CUDA_TRY(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, s));
  return LLMR_OK;
}

int llmr_copy2d_async(llmr_ctx *ctx, void *dst, size_t dpitch, const void *src, size_t spitch,
                      size_t width, size_t height, void *stream) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if (width == 0 || height == 0) return LLMR_OK;
  if (!dst || !src || width > dpitch || width > spitch)
    return fail(ctx, LLMR_EINVAL, "bad 2-D copy geometry");
  cudaStream_t s = stream ? (cudaStream_t)stream : ctx->stream;
  CUDA_TRY(ctx, cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, height, cudaMemcpyDefault, s));
  return LLMR_OK;
}

int llmr_qkv_project(llmr_ctx *ctx, const llmr_qkv_desc *d, const void *x, const void *w,
                     const float *q_gain, const float *k_gain, const float *cos_t,
                     const float *sin_t, void *qkv_out) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if (!d || !x || !w || !qkv_out) return fail(ctx, LLMR_EINVAL, "null argument");
  const long long B = d->batch, S = d->seq_len, K = d->hidden, H = d->n_heads, D = d->head_dim;
  if (B < 1 || S < 1 || H < 1 || K < 64) return fail(ctx, LLMR_EINVAL, "empty problem");
  if (D != 64 && D != 128) return fail(ctx, LLMR_EINVAL, "head_dim %lld unsupported (64 or 128)", D);
  if (K % 64) return fail(ctx, LLMR_EINVAL, "hidden must be a multiple of 64");
  if ((H * D) % 128) return fail(ctx, LLMR_EINVAL, "n_heads*head_dim must be a multiple of 128");
  if (d->dtype != LLMR_F16 && d->dtype != LLMR_BF16)
    return fail(ctx, LLMR_EINVAL, "x and w must be fp16 or bf16");
  if (d->flags & ~(uint32_t)(LLMR_NORM_Q | LLMR_NORM_K | LLMR_ROPE))
    return fail(ctx, LLMR_EINVAL, "only NORM_Q, NORM_K and ROPE apply to the projection");
  if ((d->flags & LLMR_NORM_Q) && !q_gain) return fail(ctx, LLMR_EINVAL, "LLMR_NORM_Q needs q_gain");
  if ((d->flags & LLMR_NORM_K) && !k_gain) return fail(ctx, LLMR_EINVAL, "LLMR_NORM_K needs k_gain");
  if ((d->flags & LLMR_ROPE) && (!cos_t || !sin_t)) return fail(ctx, LLMR_EINVAL, "LLMR_ROPE needs cos/sin tables");
  auto a16 = [](const void *ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
  if (!a16(qkv_out) || (q_gain && !a16(q_gain)) || (k_gain && !a16(k_gain)) ||
      (cos_t && !a16(cos_t)) || (sin_t && !a16(sin_t)))
    return fail(ctx, LLMR_EINVAL, "qkv_out, gains and tables must be 16-byte aligned");
  if (B * S > 0x7fffffffLL || 3 * B * H * S * D > (1LL << 40))
    return fail(ctx, LLMR_EINVAL, "problem too large");
  const long long x_rs = d->x_row_stride ? (long long)d->x_row_stride : K;
  QkvParams p;
  p.M = (int)(B * S);
  p.S = (int)S;
  p.B = (int)B;
  p.H = (int)H;
  p.k_blocks = (int)(K / 64);
  p.split_row = (int)d->split_row;
  p.rope_row_offset = (int)d->rope_row_offset;
  p.eps = d->eps;
  p.q_gain = (d->flags & LLMR_NORM_Q) ? q_gain : nullptr;
  p.k_gain = (d->flags & LLMR_NORM_K) ? k_gain : nullptr;
  p.cos_t = (d->flags & LLMR_ROPE) ? cos_t : nullptr;
  p.sin_t = (d->flags & LLMR_ROPE) ? sin_t : nullptr;
  p.out = static_cast<__half *>(qkv_out);
  p.err = ctx->d_err;
  const bool bf = d->dtype == LLMR_BF16;
  const bool wide = (H * D) % 256 == 0;  // 256-column tiles (two or four heads)
  const int BN = wide ? 256 : 128;
  p.n_tiles = (int)(3 * H * D / BN);
  p.tiles = (int)((p.M + 127) / 128) * p.n_tiles;
  // 256-column tiles run on CTA pairs (tcgen05 cta_group::2) unless
  // LLMR_QKV_SINGLE_CTA is set (for comparisons).
  static const bool single = getenv("LLMR_QKV_SINGLE_CTA") != nullptr;
  if (wide && !single) {
    if (D == 128) return bf ? launch_qkv_pair<128, true>(ctx, x, x_rs, w, p, K)
                            : launch_qkv_pair<128, false>(ctx, x, x_rs, w, p, K);
    return bf ? launch_qkv_pair<64, true>(ctx, x, x_rs, w, p, K)
              : launch_qkv_pair<64, false>(ctx, x, x_rs, w, p, K);
  }
  if (D == 128) {
    if (wide) return bf ? launch_qkv<128, 256, true>(ctx, x, x_rs, w, p, K)
                        : launch_qkv<128, 256, false>(ctx, x, x_rs, w, p, K);
    return bf ? launch_qkv<128, 128, true>(ctx, x, x_rs, w, p, K)
              : launch_qkv<128, 128, false>(ctx, x, x_rs, w, p, K);
  }
  if (wide) return bf ? launch_qkv<64, 256, true>(ctx, x, x_rs, w, p, K)
                      : launch_qkv<64, 256, false>(ctx, x, x_rs, w, p, K);
  return bf ? launch_qkv<64, 128, true>(ctx, x, x_rs, w, p, K)
            : launch_qkv<64, 128, false>(ctx, x, x_rs, w, p, K);
}

int llmr_out_project(llmr_ctx *ctx, const llmr_proj_desc *d, const void *o, const void *w0,
                     const void *w1, const float *bias0, const float *bias1, const float *gate0,
                     const float *gate1, float *hidden) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if (!d || !o || !w0 || !hidden) return fail(ctx, LLMR_EINVAL, "null argument");
  const long long B = d->batch, S = d->seq_len, K = d->in_dim, N = d->out_dim;
  if (B < 1 || S < 1 || K < 64 || N < 256) return fail(ctx, LLMR_EINVAL, "empty problem");
  if (K % 64 || N % 256)
    return fail(ctx, LLMR_EINVAL, "in_dim must be a multiple of 64 and out_dim of 256");
  if (d->dtype != LLMR_F16 && d->dtype != LLMR_BF16)
    return fail(ctx, LLMR_EINVAL, "o and the weights must be fp16 or bf16");
  const bool split = d->split_row > 0 && d->split_row < d->seq_len;
  if (d->split_row >= d->seq_len && d->split_row > 0)
    return fail(ctx, LLMR_EINVAL, "split_row must be below seq_len");
  if (split && !w1) return fail(ctx, LLMR_EINVAL, "split_row > 0 needs w1");
  auto a16 = [](const void *ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
  const long long h_rs = d->hidden_row_stride ? (long long)d->hidden_row_stride : N;
  if (!a16(hidden) || (h_rs % 4) || (bias0 && !a16(bias0)) || (bias1 && !a16(bias1)) ||
      (gate0 && !a16(gate0)) || (gate1 && !a16(gate1)))
    return fail(ctx, LLMR_EINVAL, "hidden (and its row stride), biases and gates must be 16-byte aligned");
  if (B * S > 0x7fffffffLL) return fail(ctx, LLMR_EINVAL, "problem too large");
  const long long o_rs = d->o_row_stride ? (long long)d->o_row_stride : K;
  ProjParams p;
  p.M = (int)(B * S);
  p.S = (int)S;
  p.B = (int)B;
  p.split = split ? (int)d->split_row : (int)S;
  p.seg_tiles0 = (p.split + 127) / 128;
  p.seg_tiles1 = split ? (int)((S - p.split + 127) / 128) : 0;
  p.k_blocks = (int)(K / 64);
  p.n_tiles = (int)(N / 256);
  p.tiles = p.B * (p.seg_tiles0 + p.seg_tiles1) * p.n_tiles;
  p.out_dim = (int)N;
  p.h_stride = h_rs;
  p.bias[0] = bias0;
  p.bias[1] = split ? bias1 : bias0;
  p.gate[0] = gate0;
  p.gate[1] = split ? gate1 : gate0;
  p.hidden = hidden;
  p.err = ctx->d_err;
  CUtensorMap mx, mw0, mw1;
  if ((rc = make_map2d(ctx, &mx, o, K, B * S, o_rs, 128))) return rc;
  if ((rc = make_map2d(ctx, &mw0, w0, K, N, K, 256))) return rc;
  if ((rc = make_map2d(ctx, &mw1, split ? w1 : w0, K, N, K, 256))) return rc;
  return d->dtype == LLMR_BF16 ? launch_out_proj<true>(ctx, mx, mw0, mw1, p)
                               : launch_out_proj<false>(ctx, mx, mw0, mw1, p);
}

size_t llmr_attention_workspace_bytes(const llmr_attn_desc *d) {
  if (!d) return 0;
  const size_t n = (size_t)d->batch * d->n_heads * d->seq_len * d->head_dim;
  // fp32 Q, K, V; for D = 64 also the tensor-core path's residuals and V^T.
  if (d->flags & LLMR_EXACT)
    return 3 * n * 4 + (d->head_dim == 64 ? (size_t)exact_tc_extra_floats(d->batch, d->n_heads,
                                                                            d->seq_len, 64) * 4
                                           : 0);
  if (d->in_dtype == LLMR_F16 && !(d->flags & (LLMR_NORM_Q | LLMR_NORM_K | LLMR_ROPE))) return 0;
  return 3 * n * 2;
}

static int attention_core(llmr_ctx *ctx, const llmr_attn_desc *d, const void *q, const void *k,
                          const void *v, const float *q_gain, const float *k_gain,
                          const float *cos_t, const float *sin_t, void *o, float *lse,
                          int nseq, const int *seq_off);

int llmr_attention_fused(llmr_ctx *ctx, const llmr_attn_desc *d, const void *q, const void *k,
                         const void *v, const float *q_gain, const float *k_gain,
                         const float *cos_t, const float *sin_t, void *o, float *lse) {
  return attention_core(ctx, d, q, k, v, q_gain, k_gain, cos_t, sin_t, o, lse, 0, nullptr);
}

int llmr_attention_varlen(llmr_ctx *ctx, const llmr_attn_desc *d, const uint32_t *seq_lens,
                          uint32_t n_seqs, const void *q, const void *k, const void *v,
                          const float *q_gain, const float *k_gain, const float *cos_t,
                          const float *sin_t, void *o, float *lse) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if (!d || !seq_lens) return fail(ctx, LLMR_EINVAL, "null argument");
  if (n_seqs < 1 || n_seqs > (uint32_t)kMaxSeqs)
    return fail(ctx, LLMR_EINVAL, "n_seqs must be in [1, %d]", kMaxSeqs);
  if (d->batch != 1) return fail(ctx, LLMR_EINVAL, "packed sequences: batch must be 1");
  if (d->split_row != 0) return fail(ctx, LLMR_EINVAL, "varlen: split_row must be 0");
  if (d->flags & (LLMR_EXACT | LLMR_MERGE))
    return fail(ctx, LLMR_EINVAL, "varlen: LLMR_EXACT and LLMR_MERGE are not supported");
  if (d->kv_seq_len != 0 && d->kv_seq_len != d->seq_len)
    return fail(ctx, LLMR_EINVAL, "varlen: kv_seq_len must be 0");
  int off[kMaxSeqs + 1];
  off[0] = 0;
  for (uint32_t i = 0; i < n_seqs; i++) {
    if (seq_lens[i] < 1) return fail(ctx, LLMR_EINVAL, "sequence %u is empty", i);
    off[i + 1] = off[i] + (int)seq_lens[i];
  }
  if ((uint32_t)off[n_seqs] != d->seq_len)
    return fail(ctx, LLMR_EINVAL, "seq_lens sum to %d, seq_len is %u", off[n_seqs], d->seq_len);
  return attention_core(ctx, d, q, k, v, q_gain, k_gain, cos_t, sin_t, o, lse, (int)n_seqs, off);
}

static int attention_core(llmr_ctx *ctx, const llmr_attn_desc *d, const void *q, const void *k,
                          const void *v, const float *q_gain, const float *k_gain,
                          const float *cos_t, const float *sin_t, void *o, float *lse,
                          int nseq, const int *seq_off) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if (!d || !q || !k || !v || !o) return fail(ctx, LLMR_EINVAL, "null argument");
  const int B = d->batch, H = d->n_heads, S = d->seq_len, D = d->head_dim;
  if (B < 1 || H < 1 || S < 1) return fail(ctx, LLMR_EINVAL, "batch, n_heads, seq_len must be >= 1");
  const bool wide = is_wide(D);
  if (D != 64 && D != 128 && !wide)
    return fail(ctx, LLMR_EINVAL, "head_dim %d unsupported (64, 128, 384 or 512)", D);
  if ((long long)B * H > 65535) return fail(ctx, LLMR_EINVAL, "batch*n_heads exceeds 65535");
  if (d->in_dtype > LLMR_BF16 || d->out_dtype > LLMR_BF16 || d->layout > LLMR_LAYOUT_BHSD)
    return fail(ctx, LLMR_EINVAL, "bad dtype or layout");
  if (wide && (d->flags & (LLMR_NORM_Q | LLMR_NORM_K | LLMR_ROPE | LLMR_MERGE)))
    return fail(ctx, LLMR_EINVAL, "head_dim %d takes no norm, RoPE or merge", D);
  if (wide && nseq > 0)
    return fail(ctx, LLMR_EINVAL, "head_dim %d takes no variable-length batch", D);
  if ((d->flags & LLMR_NORM_Q) && !q_gain) return fail(ctx, LLMR_EINVAL, "LLMR_NORM_Q needs q_gain");
  if ((d->flags & LLMR_NORM_K) && !k_gain) return fail(ctx, LLMR_EINVAL, "LLMR_NORM_K needs k_gain");
  if ((d->flags & LLMR_ROPE) && (!cos_t || !sin_t)) return fail(ctx, LLMR_EINVAL, "LLMR_ROPE needs cos/sin tables");
  if ((d->flags & LLMR_LSE) && !lse) return fail(ctx, LLMR_EINVAL, "LLMR_LSE needs an lse buffer");
  if ((d->flags & LLMR_MERGE) &&
      (!(d->flags & LLMR_LSE) || d->out_dtype != LLMR_F32 || (d->flags & LLMR_EXACT)))
    return fail(ctx, LLMR_EINVAL, "LLMR_MERGE needs LLMR_LSE, an fp32 output and the tensor-core path");
  const bool exact = d->flags & LLMR_EXACT;
  if (exact && d->out_dtype != LLMR_F32) return fail(ctx, LLMR_EINVAL, "LLMR_EXACT writes fp32 output");
  const size_t need = llmr_attention_workspace_bytes(d);
  if (need > ctx->ws_bytes)
    return fail(ctx, LLMR_ENOMEM, "workspace %zu bytes < %zu needed (llmr_ctx_reserve)", ctx->ws_bytes, need);
  const int S_kv = d->kv_seq_len ? (int)d->kv_seq_len : S;
  if (S_kv != S && need != 0)
    return fail(ctx, LLMR_EINVAL, "kv_seq_len != seq_len needs fp16 q/k/v without norm, RoPE or "
                                  "LLMR_EXACT");

  long long qs[3], ks[3], vs[3];
  default_strides(d, d->q_row_stride, d->q_batch_stride, d->q_head_stride, qs, S);
  default_strides(d, d->k_row_stride, d->k_batch_stride, d->k_head_stride, ks, S_kv);
  default_strides(d, d->v_row_stride, d->v_batch_stride, d->v_head_stride, vs, S_kv);
  const long long o_rs = d->o_row_stride ? (long long)d->o_row_stride : (long long)H * D;
  const long long o_bs = d->o_batch_stride ? (long long)d->o_batch_stride : (long long)S * o_rs;
  float *lse_out = (d->flags & LLMR_LSE) ? lse : nullptr;
  if (!(d->scale > 0.0f) || !isfinite(d->scale))
    return fail(ctx, LLMR_EINVAL, "scale must be finite and > 0");
  if (!exact && !aligned16(o, o_rs, o_bs, dtype_size(d->out_dtype)))
    return fail(ctx, LLMR_EINVAL, "o base, o_row_stride and o_batch_stride must be 16-byte aligned");

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

  const long long plane = (long long)B * H * S * D;
  auto mark = [&](int i) {
    if (ctx->prof_on) cudaEventRecord(ctx->prof_ev[i], ctx->stream);
  };
  ctx->prof_valid = false;
  mark(0);
  if (exact) {
    float *w = static_cast<float *>(ctx->ws);
    rc = wide ? launch_wide_cast<float>(ctx, d->in_dtype, q, k, v, qs, ks, vs, w, B, H, S, D)
              : launch_prologue<float>(ctx, D, d->in_dtype, q, k, v, qs, ks, vs, w, pp);
    if (rc) return rc;
    mark(1);
    ExactParams ep;
    ep.B = B;
    ep.H = H;
    ep.S = S;
    ep.scale = d->scale;
    ep.o = static_cast<float *>(o);
    ep.o_batch_stride = o_bs;
    ep.o_row_stride = o_rs;
    ep.o_head_stride = D;
    ep.lse = lse_out;
    if (!wide && exact_tc_applies(D, w, w + plane, w + 2 * plane))
      rc = launch_exact_tc(ctx, w, w + plane, w + 2 * plane, w + 3 * plane, ep);
    else if (!wide)
      rc = launch_exact(ctx, D, w, w + plane, w + 2 * plane, ep);
    else if (D == 512)
      rc = launch_exact_wide_t<512>(ctx, w, w + plane, w + 2 * plane, ep);
    else
      rc = launch_exact_wide_t<384>(ctx, w, w + plane, w + 2 * plane, ep);
    mark(2);
    ctx->prof_valid = ctx->prof_on && rc == LLMR_OK;
    return rc;
  }

  CUtensorMap mq, mk, mv;
  const bool direct = need == 0;
  // The wide pair kernel loads 64 keys per CTA and block.
  const bool wide_single = wide && wide_single_cta();
  const int k_box = wide && !wide_single ? 64 : 128;
  if (direct) {
    if ((rc = make_map(ctx, &mq, q, D, S, H, B, qs[1], qs[2], qs[0]))) return rc;
    if ((rc = make_map(ctx, &mk, k, D, S_kv, H, B, ks[1], ks[2], ks[0], k_box))) return rc;
    if ((rc = make_map(ctx, &mv, v, D, S_kv, H, B, vs[1], vs[2], vs[0]))) return rc;
  } else {
    __half *w = static_cast<__half *>(ctx->ws);
    // With LLMR_FUSED_PROLOGUE, 16-bit inputs with 16-byte aligned rows run
    // the prologue inside the attention kernel (one launch).
    auto al = [](const void *ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
    auto st8 = [](const long long *st) { return st[0] % 8 == 0 && st[1] % 8 == 0 && st[2] % 8 == 0; };
    const bool fused = !wide && nseq == 0 && d->in_dtype != LLMR_F32 && al(q) && al(k) &&
                       al(v) && st8(qs) && st8(ks) && st8(vs) && al(pp.q_gain) &&
                       al(pp.k_gain) && al(pp.cos_t) && al(pp.sin_t) &&
                       !(d->flags & LLMR_MERGE) && (long long)B * H < (long long)kSyncInts &&
                       fused_prologue_enabled();
    if (fused) {
      const long long rs = D, hs = (long long)S * D, bs = (long long)H * S * D;
      if ((rc = make_map(ctx, &mq, w, D, S, H, B, rs, hs, bs))) return rc;
      if ((rc = make_map(ctx, &mk, w + plane, D, S, H, B, rs, hs, bs))) return rc;
      if ((rc = make_map(ctx, &mv, w + 2 * plane, D, S, H, B, rs, hs, bs))) return rc;
      FusedPro fp;
      memset(&fp, 0, sizeof fp);
      fp.q = q;
      fp.k = k;
      fp.v = v;
      for (int i = 0; i < 3; i++) {
        fp.qs[i] = qs[i];
        fp.ks[i] = ks[i];
        fp.vs[i] = vs[i];
      }
      fp.ws = w;
      fp.sync = ctx->d_sync;
      fp.pp = pp;
      fp.nrb = (S + 31) / 32;
      mark(1);
      const bool bf = d->in_dtype == LLMR_BF16;
      if (D == 128)
        rc = bf ? launch_fa_fused_t<128, __nv_bfloat16>(ctx, d->out_dtype, mq, mk, mv, B, H, S,
                                                        d->scale, o, o_rs, o_bs, lse_out, fp)
                : launch_fa_fused_t<128, __half>(ctx, d->out_dtype, mq, mk, mv, B, H, S,
                                                 d->scale, o, o_rs, o_bs, lse_out, fp);
      else
        rc = bf ? launch_fa_fused_t<64, __nv_bfloat16>(ctx, d->out_dtype, mq, mk, mv, B, H, S,
                                                       d->scale, o, o_rs, o_bs, lse_out, fp)
                : launch_fa_fused_t<64, __half>(ctx, d->out_dtype, mq, mk, mv, B, H, S,
                                                d->scale, o, o_rs, o_bs, lse_out, fp);
      mark(2);
      ctx->prof_valid = ctx->prof_on && rc == LLMR_OK;
      return rc;
    }
    rc = wide ? launch_wide_cast<__half>(ctx, d->in_dtype, q, k, v, qs, ks, vs, w, B, H, S, D)
              : launch_prologue<__half>(ctx, D, d->in_dtype, q, k, v, qs, ks, vs, w, pp);
    if (rc) return rc;
    // Workspace layout: dense [3][B][H][S][D] fp16.
    const long long rs = D, hs = (long long)S * D, bs = (long long)H * S * D;
    if ((rc = make_map(ctx, &mq, w, D, S, H, B, rs, hs, bs))) return rc;
    if ((rc = make_map(ctx, &mk, w + plane, D, S, H, B, rs, hs, bs, k_box))) return rc;
    if ((rc = make_map(ctx, &mv, w + 2 * plane, D, S, H, B, rs, hs, bs))) return rc;
  }
  mark(1);
  if (wide)
    rc = launch_fa_wide_any(ctx, wide_single, D, d->out_dtype, mq, mk, mv, B, H, S, S_kv,
                            d->scale, o, o_rs, o_bs, lse_out);
  else
    rc = launch_fa_tc_any(ctx, D, d->out_dtype, mq, mk, mv, B, H, S, S_kv, d->scale, o, o_rs,
                          o_bs, lse_out, (d->flags & LLMR_MERGE) ? 1 : 0, nseq, seq_off,
                          /*pdl=*/!direct && !ctx->prof_on && !pdl_disabled());
  mark(2);
  ctx->prof_valid = ctx->prof_on && rc == LLMR_OK;
  return rc;
}

int llmr_profile_enable(llmr_ctx *ctx, int on) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if (on) {
    for (cudaEvent_t &e : ctx->prof_ev)
      if (!e) CUDA_TRY(ctx, cudaEventCreate(&e));
  }
  ctx->prof_on = on != 0;
  ctx->prof_valid = false;
  return LLMR_OK;
}

int llmr_profile_read(llmr_ctx *ctx, float *ms2) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if (!ms2) return fail(ctx, LLMR_EINVAL, "null output");
  if (!ctx->prof_valid) return fail(ctx, LLMR_EINVAL, "no profiled call recorded");
  CUDA_TRY(ctx, cudaEventSynchronize(ctx->prof_ev[2]));
  CUDA_TRY(ctx, cudaEventElapsedTime(&ms2[0], ctx->prof_ev[0], ctx->prof_ev[1]));
  CUDA_TRY(ctx, cudaEventElapsedTime(&ms2[1], ctx->prof_ev[1], ctx->prof_ev[2]));
  return LLMR_OK;
}

int llmr_attention_prologue(llmr_ctx *ctx, const llmr_attn_desc *d, const void *q,
                            const void *k, const void *v, const float *q_gain,
                            const float *k_gain, const float *cos_t, const float *sin_t,
                            void *qkv_out) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if (!d || !q || !k || !v || !qkv_out) return fail(ctx, LLMR_EINVAL, "null argument");
  const int B = d->batch, H = d->n_heads, S = d->seq_len, D = d->head_dim;
  if (B < 1 || H < 1 || S < 1) return fail(ctx, LLMR_EINVAL, "batch, n_heads, seq_len must be >= 1");
  if (D != 64 && D != 128) return fail(ctx, LLMR_EINVAL, "head_dim %d unsupported (64 or 128)", D);
  if ((long long)B * H > 65535) return fail(ctx, LLMR_EINVAL, "batch*n_heads exceeds 65535");
  if (d->in_dtype > LLMR_BF16 || d->layout > LLMR_LAYOUT_BHSD)
    return fail(ctx, LLMR_EINVAL, "bad dtype or layout");
  if (d->flags & LLMR_EXACT) return fail(ctx, LLMR_EINVAL, "the prologue writes fp16 operands");
  if ((d->flags & LLMR_NORM_Q) && !q_gain) return fail(ctx, LLMR_EINVAL, "LLMR_NORM_Q needs q_gain");
  if ((d->flags & LLMR_NORM_K) && !k_gain) return fail(ctx, LLMR_EINVAL, "LLMR_NORM_K needs k_gain");
  if ((d->flags & LLMR_ROPE) && (!cos_t || !sin_t)) return fail(ctx, LLMR_EINVAL, "LLMR_ROPE needs cos/sin tables");
  if (reinterpret_cast<uintptr_t>(qkv_out) & 15)
    return fail(ctx, LLMR_EINVAL, "qkv_out must be 16-byte aligned");
  long long qs[3], ks[3], vs[3];
  default_strides(d, d->q_row_stride, d->q_batch_stride, d->q_head_stride, qs, d->seq_len);
  default_strides(d, d->k_row_stride, d->k_batch_stride, d->k_head_stride, ks, d->seq_len);
  default_strides(d, d->v_row_stride, d->v_batch_stride, d->v_head_stride, vs, d->seq_len);
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
  return launch_prologue<__half>(ctx, D, d->in_dtype, q, k, v, qs, ks, vs,
                                 static_cast<__half *>(qkv_out), pp);
}

int llmr_convert_f32(llmr_ctx *ctx, const float *src, void *dst, llmr_dtype dt, size_t n) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if (!src || !dst || dt > LLMR_BF16) return fail(ctx, LLMR_EINVAL, "bad argument");
  if (n == 0) return LLMR_OK;
  const bool vec4 = (reinterpret_cast<uintptr_t>(src) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(dst) & (dt == LLMR_F32 ? 15 : 7)) == 0;
  const unsigned grid = grid_for(ctx, (long long)(vec4 ? (n + 3) / 4 : n), 256);
  if (dt == LLMR_F32)
    convert_f32_kernel<float><<<grid, 256, 0, ctx->stream>>>(src, static_cast<float *>(dst), (long long)n, vec4);
  else if (dt == LLMR_F16)
    convert_f32_kernel<__half><<<grid, 256, 0, ctx->stream>>>(src, static_cast<__half *>(dst), (long long)n, vec4);
  else
    convert_f32_kernel<__nv_bfloat16><<<grid, 256, 0, ctx->stream>>>(src, static_cast<__nv_bfloat16 *>(dst), (long long)n, vec4);
  return after_launch(ctx, "convert_f32");
}

int llmr_flash_attention_v2(llmr_ctx *ctx, const float *q, const float *k, const float *v,
                            float *o, uint32_t head_dim, uint32_t n_heads, uint32_t seq_len,
                            float scale) {
  llmr_attn_desc d;
  memset(&d, 0, sizeof d);
  d.batch = 1;
  d.n_heads = n_heads;
  d.seq_len = seq_len;
  d.head_dim = head_dim;
  d.in_dtype = LLMR_F32;
  d.out_dtype = LLMR_F32;
  d.layout = LLMR_LAYOUT_BHSD;
  d.scale = scale;
  return llmr_attention_fused(ctx, &d, q, k, v, nullptr, nullptr, nullptr, nullptr, o, nullptr);
}

int llmr_spatial_attention(llmr_ctx *ctx, const float *q, const float *k, const float *v,
                           float *scores, float *o, uint32_t head_dim, uint32_t n_heads,
                           uint32_t seq_len, float scale) {
  (void)scores;
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if (!q || !k || !v || !o) return fail(ctx, LLMR_EINVAL, "null argument");
  if (head_dim != 64 && head_dim != 128)
    return fail(ctx, LLMR_EINVAL, "head_dim %u unsupported (64 or 128)", head_dim);
  if (n_heads < 1 || seq_len < 1 || n_heads > 65535) return fail(ctx, LLMR_EINVAL, "bad n_heads/seq_len");
  ExactParams ep;
  ep.B = 1;
  ep.H = (int)n_heads;
  ep.S = (int)seq_len;
  ep.scale = scale;
  ep.o = o;
  ep.o_batch_stride = 0;
  ep.o_row_stride = head_dim;                      // [H, S, D] output
  ep.o_head_stride = (long long)seq_len * head_dim;
  ep.lse = nullptr;
  // Tensor cores (3xTF32) when the context workspace holds the residuals.
  const size_t res_bytes = (size_t)exact_tc_extra_floats(1, n_heads, seq_len, head_dim) * 4;
  if (exact_tc_applies((int)head_dim, q, k, v) && ctx->ws_bytes >= res_bytes)
    return launch_exact_tc(ctx, q, k, v, static_cast<float *>(ctx->ws), ep);
  return launch_exact(ctx, (int)head_dim, q, k, v, ep);
}

int llmr_vae_attention(llmr_ctx *ctx, const float *q, const float *k, const float *v, float *o,
                       uint32_t head_dim, uint32_t n_heads, uint32_t seq_len, float scale,
                       uint32_t channels) {
  if ((uint64_t)channels < (uint64_t)n_heads * head_dim)
    return fail(ctx, LLMR_EINVAL, "channels %u < n_heads * head_dim", channels);
  llmr_attn_desc d;
  memset(&d, 0, sizeof d);
  d.batch = 1;
  d.n_heads = n_heads;
  d.seq_len = seq_len;
  d.head_dim = head_dim;
  d.in_dtype = LLMR_F32;
  d.out_dtype = LLMR_F32;
  d.layout = LLMR_LAYOUT_BSHD;
  d.scale = scale;
  d.q_row_stride = d.k_row_stride = d.v_row_stride = d.o_row_stride = channels;
  return llmr_attention_fused(ctx, &d, q, k, v, nullptr, nullptr, nullptr, nullptr, o, nullptr);
}

int llmr_batch_head_norm(llmr_ctx *ctx, float *data, const float *gain, uint32_t n_heads,
                         uint32_t head_dim, uint32_t seq_len, float eps) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if (!data || !gain || !head_dim) return fail(ctx, LLMR_EINVAL, "null argument or head_dim 0");
  const long long rows = (long long)seq_len * n_heads;
  if (rows == 0) return LLMR_OK;
  head_norm_f32_kernel<<<grid_for(ctx, rows * 32, 256), 256, 0, ctx->stream>>>(
      data, gain, (int)n_heads, (int)head_dim, (int)seq_len, eps);
  return after_launch(ctx, "head_norm_f32");
}

int llmr_perhead_rmsnorm(llmr_ctx *ctx, float *data, const float *weight, uint32_t seq_len,
                         uint32_t n_heads, uint32_t head_dim, float eps) {
  return llmr_batch_head_norm(ctx, data, weight, n_heads, head_dim, seq_len, eps);
}

int llmr_transpose_heads(llmr_ctx *ctx, const float *in, float *out, uint32_t seq_len,
                         uint32_t n_heads, uint32_t head_dim, uint32_t direction) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if (!in || !out || in == out) return fail(ctx, LLMR_EINVAL, "null or aliased buffers");
  if (direction > 1) return fail(ctx, LLMR_EINVAL, "direction must be 0 or 1");
  const long long n = (long long)seq_len * n_heads * head_dim;
  if (n == 0) return LLMR_OK;
  transpose_heads_kernel<<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>(
      in, out, (int)seq_len, (int)n_heads, (int)head_dim, (int)direction);
  return after_launch(ctx, "transpose_heads");
}

int llmr_mrope(llmr_ctx *ctx, float *data, const float *cos_t, const float *sin_t,
               uint32_t seq_len, uint32_t n_heads) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if (!data || !cos_t || !sin_t) return fail(ctx, LLMR_EINVAL, "null argument");
  const long long n = (long long)seq_len * n_heads * 64;
  if (n == 0) return LLMR_OK;
  mrope_f32_kernel<<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>(data, cos_t, sin_t,
                                                                  (int)seq_len, (int)n_heads, 64);
  return after_launch(ctx, "mrope_f32");
}

int llmr_split_qkv(llmr_ctx *ctx, const float *qkv, float *q, float *k, float *v, uint32_t dim,
                   uint32_t n_rows) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if (!qkv || !q || !k || !v) return fail(ctx, LLMR_EINVAL, "null argument");
  const long long n = (long long)n_rows * dim;
  if (n == 0) return LLMR_OK;
  split_qkv_kernel<<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>(qkv, q, k, v, (int)dim,
                                                                  (int)n_rows);
  return after_launch(ctx, "split_qkv");
}

int llmr_attention_merge(llmr_ctx *ctx, float *o_a, float *lse_a, const float *o_b,
                         const float *lse_b, uint32_t rows, uint32_t n_heads, uint32_t head_dim,
                         uint64_t o_row_stride) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if (!o_a || !lse_a || !o_b || !lse_b) return fail(ctx, LLMR_EINVAL, "null argument");
  const long long rs = o_row_stride ? (long long)o_row_stride : (long long)n_heads * head_dim;
  const long long n = (long long)rows * n_heads * head_dim;
  if (n == 0) return LLMR_OK;
  merge_kernel<<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>(o_a, lse_a, o_b, lse_b, (int)rows,
                                                              (int)n_heads, (int)head_dim, rs);
  if ((rc = after_launch(ctx, "merge"))) return rc;
  const long long nl = (long long)rows * n_heads;
  merge_lse_kernel<<<grid_for(ctx, nl, 256), 256, 0, ctx->stream>>>(lse_a, lse_b, nl);
  return after_launch(ctx, "merge_lse");
}

int llmr_rope_tables(const int32_t *pos, uint32_t seq_len, uint32_t n_axes,
                     const uint32_t *axes_dims, float theta, float *cos_out, float *sin_out) {
  if (!pos || !axes_dims || !cos_out || !sin_out || n_axes == 0) return LLMR_EINVAL;
  uint32_t half = 0;
  for (uint32_t a = 0; a < n_axes; a++) {
    if (axes_dims[a] % 2) return LLMR_EINVAL;
    half += axes_dims[a] / 2;
  }
  // freq = 1/theta^(2k/d_a), angle = pos * freq, in float, as the reference
  // host code computes them (dependencies/flux.c3l/flux_dit.c3:461-497).
  for (uint64_t t = 0; t < seq_len; t++) {
    uint32_t pair = 0;
    for (uint32_t a = 0; a < n_axes; a++) {
      const uint32_t ha = axes_dims[a] / 2;
      for (uint32_t kk = 0; kk < ha; kk++) {
        const float freq = 1.0f / powf(theta, (float)(2 * kk) / (float)axes_dims[a]);
        const float angle = (float)pos[t * n_axes + a] * freq;
        cos_out[t * half + pair] = cosf(angle);
        sin_out[t * half + pair] = sinf(angle);
        pair++;
      }
    }
  }
  return LLMR_OK;
}

}  // extern "C"
