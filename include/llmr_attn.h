/*
 * llmr_attn — B200 (sm_100a) drop-in for llm-runner's fused non-causal
 * attention path: per-head QK-RMSNorm, multi-axis RoPE and flash attention.
 *
 * This C ABI replaces, for this op only, the Vulkan dispatch and buffer layer
 * that the reference's model code records attention through
 * (lib/vulkan/graph.c3:47-72 RenderGraph.dispatch -> lib/vulkan/compute.c3:86
 * dispatch_kernel, buffers from lib/model/tensor.c3:8-120). Paths cited below
 * are relative to the reference project root.
 *
 * Conventions
 *  - Every call returns an int status (LLMR_OK = 0). llmr_last_error() gives a
 *    one-line message for the last failure on that context.
 *  - Device buffers are caller-owned (as llm::Tensor is). The mirrors of the
 *    reference ops take fp32 device buffers in the reference's layouts.
 *  - Calls are asynchronous on the context's CUDA stream; llmr_sync() is the
 *    equivalent of RenderGraph.checkpoint()/flush() (lib/vulkan/graph.c3:96-107)
 *    and is where device-side timeouts surface as LLMR_ETIMEOUT.
 *  - A context is bound to one device and is not thread-safe, as the
 *    reference's single command buffer per context is not
 *    (lib/vulkan/context.c3:328-334). Use one context per host thread / GPU.
 *  - The hot calls never allocate: scratch comes from the workspace sized at
 *    llmr_ctx_create() (or grown explicitly with llmr_ctx_reserve()).
 */
#ifndef LLMR_ATTN_H
#define LLMR_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. Replace the reference's faultdef set
 * (lib/vulkan/context.c3:10: NO_SUITABLE_DEVICE, COMPUTE_ERROR, ...). */
enum {
  LLMR_OK = 0,
  LLMR_EINVAL = 1,      /* bad argument / unsupported shape */
  LLMR_ENOMEM = 2,      /* allocation failed or workspace too small */
  LLMR_ECUDA = 3,       /* CUDA runtime / driver error */
  LLMR_ENCCL = 4,       /* NCCL error (ring variant) */
  LLMR_ETIMEOUT = 5,    /* a bounded device-side wait gave up */
  LLMR_ENODEV = 6       /* no usable sm_100 device */
};

typedef enum { LLMR_F32 = 0, LLMR_F16 = 1, LLMR_BF16 = 2 } llmr_dtype;

/* Q/K/V/O tensor layouts.
 * BSHD: [batch][seq][head][dim] — the reference's activation layout
 *       [S, H*D] per batch element (dependencies/zimage.c3l/dit.c3:1445-1449).
 * BHSD: [batch][head][seq][dim] — the reference's post-transpose_heads layout
 *       (dependencies/zimage.c3l/shaders/zimage.slang:563-601). */
typedef enum { LLMR_LAYOUT_BSHD = 0, LLMR_LAYOUT_BHSD = 1 } llmr_layout;

/* Flags for llmr_attn_desc.flags. */
enum {
  LLMR_NORM_Q = 1u << 0,  /* per-head RMSNorm on Q (batch_head_norm) */
  LLMR_NORM_K = 1u << 1,  /* per-head RMSNorm on K */
  LLMR_ROPE = 1u << 2,    /* multi-axis RoPE on Q and K (mrope) from tables */
  LLMR_EXACT = 1u << 3,   /* fp32 operands and exact softmax (spatial_attention
                             math, lib/shaders/diffusion.slang:478-569) instead
                             of fp16 operands (flash_attention_v2 math) */
  LLMR_LSE = 1u << 4,     /* also write log-sum-exp (natural log) per row */
  LLMR_MERGE = 1u << 5    /* o (fp32) and lse already hold the normalised
                             result over other keys: merge this call's result
                             into them by log-sum-exp, in place (the step of
                             the sequence-sharded ring). Needs LLMR_LSE. */
};

typedef struct llmr_ctx llmr_ctx;

/* Create a context on CUDA device `device`, using `stream` (a cudaStream_t;
 * NULL = a new non-blocking stream owned by the context; pass
 * cudaStreamLegacy to run on the legacy default stream) and a device
 * workspace of `workspace_bytes` (may be 0 and grown by llmr_ctx_reserve).
 * Replaces createContext() (lib/vulkan/context.c3:73). */
int llmr_ctx_create(int device, size_t workspace_bytes, void *stream,
                    llmr_ctx **out);
int llmr_ctx_destroy(llmr_ctx *ctx);
/* Grow the workspace to at least `bytes` (synchronous; not for the hot loop). */
int llmr_ctx_reserve(llmr_ctx *ctx, size_t bytes);
int llmr_set_stream(llmr_ctx *ctx, void *stream);
/* Limit the persistent kernels of this context to `sms` SMs (0 = all SMs of
 * the device), leaving the rest to work that runs beside them, e.g. the
 * NCCL send/receive kernels of the sequence-sharded ring. No reference
 * counterpart (the reference is single-GPU). */
int llmr_ctx_set_sm_budget(llmr_ctx *ctx, int sms);
/* Diagnostic builds only (compiled with -DLLMR_TIMELINE, `make TIMELINE=1`):
 * the D <= 128 attention kernel records per-CTA event timestamps
 * (128 slots per CTA, the slot meanings are listed in csrc/fa_tc.cuh) into
 * `device_buffer` (>= num_sms * 128 * 8 bytes; NULL
 * turns it off). Other builds return LLMR_EINVAL. No reference counterpart
 * (the reference's timer is per dispatch, dependencies/zimage.c3l/
 * dit.c3:17-26). */
int llmr_timeline_set(llmr_ctx *ctx, void *device_buffer, size_t bytes);
void *llmr_get_stream(llmr_ctx *ctx);
const char *llmr_last_error(llmr_ctx *ctx);
/* Wait for all work on the context stream; reports device-side timeouts.
 * Replaces RenderGraph.checkpoint/flush (lib/vulkan/graph.c3:96-107). */
int llmr_sync(llmr_ctx *ctx);
/* Number of kernels this context has launched (for launch accounting). */
uint64_t llmr_launch_count(llmr_ctx *ctx);

/* Per-phase GPU timing of llmr_attention_fused, the device-side counterpart
 * of the reference's @prof_checkpoint phase timer (dependencies/zimage.c3l/
 * dit.c3:17-26, "C:attn_all" at :1484). When enabled, each fused call
 * records CUDA events around its prologue and attention kernels.
 * llmr_profile_read waits for the last profiled call and writes
 * ms[0] = prologue (0 if none ran), ms[1] = attention kernel. */
int llmr_profile_enable(llmr_ctx *ctx, int on);
int llmr_profile_read(llmr_ctx *ctx, float *ms2);

/* Failure-detection self-test. Launches one small kernel whose bounded
 * mbarrier wait can never complete (nothing arrives on the barrier); after
 * limit_ns it gives up and raises the context's error word, exactly as an
 * expired wait inside the attention kernel does. The next llmr_sync returns
 * LLMR_ETIMEOUT and clears the word; the context stays usable. No
 * counterpart in the reference, whose fence waits are unbounded
 * (lib/vulkan/compute.c3:156-165). limit_ns must be in (0, 1e9]. */
int llmr_selftest_wait_timeout(llmr_ctx *ctx, uint64_t limit_ns);

/* Buffers. Replace create_tensor / upload_to_tensor / download_tensor
 * (lib/model/tensor.c3:27-46, :79, :99). upload/download are synchronous,
 * as the reference's staging copies are. */
int llmr_alloc(llmr_ctx *ctx, size_t bytes, void **out);
int llmr_free(llmr_ctx *ctx, void *ptr);
int llmr_upload(llmr_ctx *ctx, void *dst_device, const void *src_host,
                size_t bytes);
int llmr_download(llmr_ctx *ctx, void *dst_host, const void *src_device,
                  size_t bytes);

/* Peer buffers for the sequence-sharded attention across GPUs (one process
 * per GPU). No counterpart in the reference, which runs on one GPU
 * (docs/flux_server.md:84-88). A buffer from llmr_alloc (the allocation's
 * base address) is exported as an opaque handle, sent to the other
 * processes by the caller (any host channel), and mapped there with
 * llmr_ipc_open. llmr_copy_async moves bytes between the GPUs on the copy
 * engines over NVLink, using no SMs, so the transfer of the next K/V block
 * overlaps the attention kernel. The caller orders copies against the
 * owner's writes (e.g. a barrier after the owner's prologue). */
typedef struct {
  unsigned char bytes[64];
} llmr_ipc_handle;
int llmr_ipc_export(llmr_ctx *ctx, void *base, llmr_ipc_handle *out);
int llmr_ipc_open(llmr_ctx *ctx, const llmr_ipc_handle *handle, void **out);
int llmr_ipc_close(llmr_ctx *ctx, void *mapped);
/* cudaMemcpyAsync(dst, src, bytes, default kind) on `stream` (NULL = the
 * context's stream). */
int llmr_copy_async(llmr_ctx *ctx, void *dst, const void *src, size_t bytes,
                    void *stream);
/* cudaMemcpy2DAsync: `height` rows of `width` bytes, consecutive rows
 * `dpitch` bytes apart in dst and `spitch` bytes apart in src (e.g. a peer's
 * head-major K block into its slot of a buffer that keeps each head's keys
 * from several blocks contiguous). */
int llmr_copy2d_async(llmr_ctx *ctx, void *dst, size_t dpitch, const void *src,
                      size_t spitch, size_t width, size_t height, void *stream);

/* ---- Mirrors of the reference's attention ops (fp32 buffers) ---------- */

/* flash_attention_v2 (dependencies/zimage.c3l/shaders/flash_attn.slang:38-241;
 * push constants FlashAttentionPC {head_dim, n_heads, seq_len, scale},
 * dependencies/zimage.c3l/dit.c3:136-142). q,k,v: [n_heads, seq_len,
 * head_dim]; o: [seq_len, n_heads*head_dim]. Operands are rounded to fp16 as
 * the shader does. head_dim 64 or 128 (the shader itself is 128-only). */
int llmr_flash_attention_v2(llmr_ctx *ctx, const float *q, const float *k,
                            const float *v, float *o, uint32_t head_dim,
                            uint32_t n_heads, uint32_t seq_len, float scale);

/* batch_head_norm (dependencies/zimage.c3l/shaders/zimage.slang:623-659;
 * BatchHeadNormPC {n_heads, head_dim, seq_len, eps}, dit.c3:128-134).
 * In place on data[seq_len, n_heads*head_dim] with gain[head_dim]. */
int llmr_batch_head_norm(llmr_ctx *ctx, float *data, const float *gain,
                         uint32_t n_heads, uint32_t head_dim, uint32_t seq_len,
                         float eps);

/* perhead_rmsnorm (dependencies/qwen_edit.c3l/shaders/vit.slang:590-616;
 * PerHeadRMSNormPC {seq_len, n_heads, head_dim, eps}). Same math. */
int llmr_perhead_rmsnorm(llmr_ctx *ctx, float *data, const float *weight,
                         uint32_t seq_len, uint32_t n_heads, uint32_t head_dim,
                         float eps);

/* transpose_heads (dependencies/zimage.c3l/shaders/zimage.slang:575-601;
 * TransposeHeadsPC {seq_len, n_heads, head_dim, direction}, dit.c3:120-126).
 * direction 0: [S,H,D] -> [H,S,D]; 1: reverse. in and out must not alias. */
int llmr_transpose_heads(llmr_ctx *ctx, const float *in, float *out,
                         uint32_t seq_len, uint32_t n_heads, uint32_t head_dim,
                         uint32_t direction);

/* mrope (dependencies/zimage.c3l/shaders/mrope.slang:33-54; MRoPEPC
 * {seq_len, n_heads, pad, pad}, dit.c3:164-170). In place on
 * data[n_heads, seq_len, 128] with cos/sin[seq_len, 64]. */
int llmr_mrope(llmr_ctx *ctx, float *data, const float *cos_t,
               const float *sin_t, uint32_t seq_len, uint32_t n_heads);

/* spatial_attention (lib/shaders/diffusion.slang:478-569;
 * SpatialAttentionPC {head_dim, n_heads, seq_len, scale},
 * dependencies/depth_anything.c3l/depth_anything.c3:335-337). q,k,v,o:
 * [n_heads, seq_len, head_dim] fp32, exact softmax. `scores` is accepted for
 * signature compatibility and ignored (may be NULL): no S x S buffer is
 * materialised. head_dim 64 or 128. head_dim 64 runs on the tensor cores
 * (three TF32 products per fp32 product, fp32 accumulation) when the
 * context workspace holds 4*n_heads*64*(4*seq_len + 2*ceil4(seq_len)) bytes
 * (llmr_ctx_reserve; ceil4 rounds up to a multiple of 4) for the operands
 * split into TF32 parts (V transposed); otherwise, and for head_dim 128, on an
 * fp32 FMA kernel. Both stay within 1e-5 of the reference's arithmetic. */
int llmr_spatial_attention(llmr_ctx *ctx, const float *q, const float *k,
                           const float *v, float *scores, float *o,
                           uint32_t head_dim, uint32_t n_heads,
                           uint32_t seq_len, float scale);

/* vae_attention (lib/shaders/diffusion.slang:1828-1975; VaeAttentionParams
 * {head_dim, n_heads, seq_len, scale, channels}, dispatched by
 * dependencies/zimage.c3l/flux_vae.c3:526-538 with one head of 512 and
 * dependencies/qwen_edit.c3l/qwen_vae.c3:459-464 with one head of 384).
 * q,k,v,o: [seq_len, channels] fp32, head h at columns [h*head_dim,
 * (h+1)*head_dim). head_dim 64, 128, 384 or 512. Computed on the tensor
 * cores with fp16 operands and fp32 accumulation (workspace
 * 3*seq_len*n_heads*head_dim*2 bytes); LLMR_EXACT through
 * llmr_attention_fused gives the fp32 path. */
int llmr_vae_attention(llmr_ctx *ctx, const float *q, const float *k,
                       const float *v, float *o, uint32_t head_dim,
                       uint32_t n_heads, uint32_t seq_len, float scale,
                       uint32_t channels);

/* split_qkv (dependencies/depth_anything.c3l/shaders/depth.slang:40-58;
 * {dim, n_rows}): qkv[n_rows, 3*dim] -> q,k,v [n_rows, dim]. */
int llmr_split_qkv(llmr_ctx *ctx, const float *qkv, float *q, float *k,
                   float *v, uint32_t dim, uint32_t n_rows);

/* ---- Fused op ---------------------------------------------------------- */

/* One call for the reference's whole 8-dispatch attention sequence
 * (batch_head_norm x2, transpose_heads x3, mrope x2, flash_attention_v2:
 * dependencies/flux.c3l/flux_dit.c3:812-872, :1020-1047,
 * dependencies/zimage.c3l/dit.c3:1445-1483, dependencies/qwen_edit.c3l/
 * mmdit.c3:577-678, dependencies/depth_anything.c3l/depth_anything.c3:
 * 610-630). Strides are in elements; 0 selects the dense default for the
 * layout. A fused QKV buffer [S, 3*H*D] is addressed by passing q, k, v
 * pointers at column offsets 0, H*D, 2*H*D with row stride 3*H*D (replaces
 * split_qkv). O is always [B][S][H*D] (row stride o_row_stride). */
typedef struct {
  /* head_dim 64 or 128; 384 or 512 (the VAE attention) without
   * LLMR_NORM_Q/NORM_K/ROPE/MERGE and not in llmr_attention_varlen */
  uint32_t batch, n_heads, seq_len, head_dim;
  llmr_dtype in_dtype;                        /* dtype of q, k, v */
  llmr_dtype out_dtype;                       /* dtype of o */
  llmr_layout layout;                         /* layout of q, k, v */
  uint32_t flags;                             /* LLMR_NORM_Q | ... */
  float scale;                                /* softmax scale */
  float eps;                                  /* RMSNorm epsilon */
  /* Tokens with global index < split_row use gain set 0, the others gain
   * set 1 (txt/img gains, flux_dit.c3:812-845). q_gain/k_gain point to
   * 2*head_dim fp32 device values when split_row > 0, else head_dim values.
   * The global index of token s is rope_row_offset + s. */
  uint32_t split_row;
  /* Global index of token 0: the cos/sin table row it uses and its position
   * against split_row (0 for a whole sequence; the shard start for a
   * sequence shard). */
  uint32_t rope_row_offset;
  /* Element strides; 0 = dense default. */
  uint64_t q_row_stride, k_row_stride, v_row_stride, o_row_stride;
  uint64_t q_batch_stride, k_batch_stride, v_batch_stride, o_batch_stride;
  uint64_t q_head_stride, k_head_stride, v_head_stride;
  /* Keys (K/V rows) per (batch, head); 0 = seq_len. A value other than
   * seq_len needs fp16 q/k/v without LLMR_NORM_Q/NORM_K/ROPE/EXACT (no
   * prologue): attention of seq_len queries over one block of keys, as the
   * sequence-sharded ring computes it. Default K/V strides use it. */
  uint32_t kv_seq_len;
} llmr_attn_desc;

/* ---- QKV projection with the prologue in its epilogue --------------------
 * The step before the path (the reference's three batch matmuls of a block,
 * dependencies/zimage.c3l/dit.c3:1437-1442 / flux.c3l/flux_dit.c3:787-801,
 * with the fp16 coopmat GEMM of dependencies/llm_text.c3l/shaders/
 * llm.slang:2039-2105, followed by batch_head_norm and mrope) as one
 * tensor-core GEMM: qkv_out[t][b][h][s][d] = epilogue_t(x[b*S+s, :] .
 * w[t*H*D + h*D + d, :]) written as dense fp16 [3][B][H][S][D] — exactly the
 * input llmr_attention_fused takes with layout BHSD, in_dtype F16 and no
 * NORM/ROPE flags (q, k, v at element offsets 0, B*H*S*D, 2*B*H*S*D). For
 * Q and K the epilogue applies LLMR_NORM_Q / LLMR_NORM_K (gain sets split at
 * split_row) and LLMR_ROPE (table row rope_row_offset + s), in fp32. */
typedef struct {
  uint32_t batch, seq_len, hidden, n_heads, head_dim; /* hidden % 64 == 0 */
  llmr_dtype dtype;   /* of x and w: LLMR_F16 or LLMR_BF16 (the same for both) */
  uint32_t flags;     /* LLMR_NORM_Q | LLMR_NORM_K | LLMR_ROPE */
  float eps;
  uint32_t split_row, rope_row_offset;
  uint64_t x_row_stride; /* elements between token rows of x; 0 = hidden */
} llmr_qkv_desc;
/* x: [batch*seq_len rows][hidden]; w: [3*n_heads*head_dim][hidden] dense;
 * qkv_out: fp16, 16-byte aligned. n_heads*head_dim must be a multiple of
 * 128. */
int llmr_qkv_project(llmr_ctx *ctx, const llmr_qkv_desc *desc, const void *x,
                     const void *w, const float *q_gain, const float *k_gain,
                     const float *cos_t, const float *sin_t, void *qkv_out);

/* ---- Output projection with the gated residual in its epilogue ---------
 * The step after the path: hidden[b*S+s, n] += gate_g[n] *
 * (o[b*S+s, :] . w_g[n, :] + bias_g[n]) with weight set g = 1 for tokens
 * s >= split_row when split_row > 0, else g = 0 — the joint blocks' two
 * streams with their own projection, bias and gate
 * (dependencies/flux.c3l/flux_dit.c3:874-885, dependencies/qwen_edit.c3l/
 * mmdit.c3:694-720: matmul, broadcast_bias_add vit.slang:133-137,
 * gated_residual_add vit.slang:638-647), in one tensor-core GEMM. o is the
 * attention output [batch*seq_len][in_dim] (fp16 or bf16, e.g. the output of
 * llmr_attention_fused), w0 / w1 [out_dim][in_dim] dense of o's type (w1
 * only with split_row > 0), bias / gate fp32 [out_dim] or NULL (0 / 1),
 * hidden fp32 [batch*seq_len][out_dim] (row stride hidden_row_stride,
 * 0 = out_dim), updated in place. in_dim % 64 == 0, out_dim % 256 == 0. */
typedef struct {
  uint32_t batch, seq_len, in_dim, out_dim;
  llmr_dtype dtype;    /* of o and the weights: LLMR_F16 or LLMR_BF16 */
  uint32_t split_row;
  uint64_t o_row_stride;      /* elements; 0 = in_dim */
  uint64_t hidden_row_stride; /* elements; 0 = out_dim */
} llmr_proj_desc;
int llmr_out_project(llmr_ctx *ctx, const llmr_proj_desc *desc, const void *o,
                     const void *w0, const void *w1, const float *bias0,
                     const float *bias1, const float *gate0,
                     const float *gate1, float *hidden);

/* Workspace bytes llmr_attention_fused needs for `desc`. */
size_t llmr_attention_workspace_bytes(const llmr_attn_desc *desc);

/* Fused QK-RMSNorm + RoPE + attention. cos_t/sin_t: fp32 device tables
 * [rows, head_dim/2] (required with LLMR_ROPE). lse: fp32 [B][H][S] device
 * buffer, written when LLMR_LSE is set (else may be NULL). */
int llmr_attention_fused(llmr_ctx *ctx, const llmr_attn_desc *desc,
                         const void *q, const void *k, const void *v,
                         const float *q_gain, const float *k_gain,
                         const float *cos_t, const float *sin_t, void *o,
                         float *lse);

/* Variable-length batch: q/k/v hold n_seqs sequences back to back as one
 * batch element of desc->seq_len = sum(seq_lens) tokens (desc->batch must be
 * 1; any layout and strides of llmr_attention_fused), and each sequence
 * attends only within itself — e.g. the cond/uncond pair of a CFG step with
 * different text lengths, which the reference runs as two forwards
 * (dependencies/zimage.c3l/pipeline.c3:494-520), in one call. The RoPE row of
 * packed token t is rope_row_offset + t (concatenate the sequences' tables).
 * split_row must be 0; LLMR_EXACT, LLMR_MERGE and kv_seq_len are not
 * supported. seq_lens: host array, 1 <= n_seqs <= 64. */
int llmr_attention_varlen(llmr_ctx *ctx, const llmr_attn_desc *desc,
                          const uint32_t *seq_lens, uint32_t n_seqs,
                          const void *q, const void *k, const void *v,
                          const float *q_gain, const float *k_gain,
                          const float *cos_t, const float *sin_t, void *o,
                          float *lse);

/* Allocation-free variant of llmr_attention_fused (tensor-core path only).
 * It has no counterpart in the reference. It is for callers that cannot
 * allocate device memory: those whose HBM belongs to another allocator (a
 * serving runtime or host engine that reserves memory up front and accounts
 * for every byte) and latency-critical paths that must not call
 * cudaMalloc/cudaFree, which can synchronise the whole device. Such callers
 * cannot create an llmr_ctx, so this call takes a cudaStream_t (NULL = the
 * default stream) and runs on the current device.
 *  - Scratch: a fixed array inside the library, LLMR_NOALLOC_SCRATCH_BYTES
 *    per GPU that loads the library, held until the process exits. Calls
 *    needing more (3*B*H*S*D*2 bytes, when a prologue runs) return
 *    LLMR_ENOMEM; fp16 input without norm/RoPE needs none.
 *  - The first call on each device looks up the scratch address; make that
 *    first call before any stream capture.
 *  - All calls share the scratch: calls that overlap on the GPU race.
 *  - LLMR_EXACT is rejected (LLMR_EINVAL). The call does not synchronise;
 *    a device-side wait that timed out is reported by llmr_noalloc_status.
 * Returns a status code only (there is no context for a message). */
#define LLMR_NOALLOC_SCRATCH_BYTES ((size_t)64 << 20)
int llmr_attention_fused_noalloc(const llmr_attn_desc *desc, const void *q,
                                 const void *k, const void *v,
                                 const float *q_gain, const float *k_gain,
                                 const float *cos_t, const float *sin_t,
                                 void *o, float *lse, void *stream);

/* Synchronises `stream` (NULL = the default stream) and reports whether any
 * llmr_attention_fused_noalloc call on the current device since the last
 * status query had a bounded device-side wait expire: LLMR_ETIMEOUT (the
 * results of those calls are invalid; the flag is cleared) or LLMR_OK.
 * Allocates nothing. No counterpart in the reference (its fence waits are
 * unbounded). */
int llmr_noalloc_status(void *stream);

/* The prologue of llmr_attention_fused on its own: per-head RMSNorm and RoPE
 * of Q and K, cast of V, written as dense fp16 [3][B][H][S][D] to `qkv_out`
 * (Q at 0, K at B*H*S*D, V at 2*B*H*S*D elements; 16-byte aligned). The
 * sequence-sharded ring runs it once per shard (rope_row_offset = shard
 * start) and then moves the fp16 K/V block between GPUs. Replaces the
 * batch_head_norm / transpose_heads / mrope dispatches of a block
 * (dependencies/flux.c3l/flux_dit.c3:812-863). LLMR_EXACT is rejected. */
int llmr_attention_prologue(llmr_ctx *ctx, const llmr_attn_desc *desc,
                            const void *q, const void *k, const void *v,
                            const float *q_gain, const float *k_gain,
                            const float *cos_t, const float *sin_t,
                            void *qkv_out);

/* dst[i] = (dtype) src[i] for n fp32 values (RNE), e.g. the merged fp32
 * output of the ring into the model's bf16 activations. */
int llmr_convert_f32(llmr_ctx *ctx, const float *src, void *dst,
                     llmr_dtype dst_dtype, size_t n);

/* Merge two normalised partial attention results over disjoint key sets
 * (o_a, lse_a) and (o_b, lse_b) into (o_a, lse_a): the combine step of the
 * sequence-sharded ring. o_*: fp32 [rows][n_heads*head_dim] (row stride
 * o_row_stride elements), lse_*: fp32 [n_heads][rows]. No reference
 * counterpart: the reference is single-GPU. */
int llmr_attention_merge(llmr_ctx *ctx, float *o_a, float *lse_a,
                         const float *o_b, const float *lse_b, uint32_t rows,
                         uint32_t n_heads, uint32_t head_dim,
                         uint64_t o_row_stride);

/* Host-side multi-axis RoPE table builder (precompute_flux_mrope,
 * dependencies/flux.c3l/flux_dit.c3:396-525; precompute_mrope_tables,
 * dependencies/zimage.c3l/dit.c3:561-757): pos is [seq_len][n_axes] int32,
 * outputs cos/sin [seq_len][sum(axes_dims)/2] fp32 in HOST memory. */
int llmr_rope_tables(const int32_t *pos, uint32_t seq_len, uint32_t n_axes,
                     const uint32_t *axes_dims, float theta, float *cos_out,
                     float *sin_out);

#ifdef __cplusplus
}
#endif
#endif /* LLMR_ATTN_H */
