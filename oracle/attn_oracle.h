/*
 * CPU oracle for the fused non-causal attention path of tonis2/llm-runner.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker that the CUDA path is
 * compared against (tests/, __graft_entry__.smoke(), and bench.py's
 * cpu_baseline / --impl reference leg). The shipped library never links,
 * loads or calls it.
 *
 * PARITY UNPINNED: the reference ships no golden vectors, known-answer tests or
 * fixtures for this path, and it cannot be built or run in this environment
 * (it needs the C3 compiler, the Slang compiler and a Vulkan device). Each
 * function below is a line-by-line restatement of a reference shader or host
 * routine, cited by file:line inside the reference project, cross-checked
 * against an independent numpy restatement (tests/golden/make_golden.py) and,
 * for the attention math, against a restatement of the reference test
 * suite's own CPU attention (test/mesh_encoder_test.c3:95-135).
 *
 * All buffers are fp32, as the reference's RWStructuredBuffer<float> bindings.
 */
#pragma once
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Round an fp32 value to IEEE binary16 (round-to-nearest-even), widen back. */
float orc_round_f16(float x);
void orc_set_threads(int n);
/* Round an fp32 value to bfloat16 (round-to-nearest-even), widen back. */
float orc_round_bf16(float x);

/* batch_head_norm / perhead_rmsnorm: in place on data[S, H*D] with gain[D].
 * dependencies/zimage.c3l/shaders/zimage.slang:623-659,
 * dependencies/qwen_edit.c3l/shaders/vit.slang:590-616 (same math). */
void orc_batch_head_norm(float *data, const float *gain, uint32_t n_heads,
                         uint32_t head_dim, uint32_t seq_len, float eps);

/* transpose_heads: direction 0 [S,H,D]->[H,S,D], 1 the reverse.
 * dependencies/zimage.c3l/shaders/zimage.slang:575-601. */
void orc_transpose_heads(const float *in, float *out, uint32_t seq_len,
                         uint32_t n_heads, uint32_t head_dim,
                         uint32_t direction);

/* mrope: in place on data[H, S, 2*half] with cos/sin[S, half].
 * dependencies/zimage.c3l/shaders/mrope.slang:33-54 (half fixed at 64 there;
 * generalised to any half = head_dim/2). */
void orc_mrope(float *data, const float *cos_t, const float *sin_t,
               uint32_t seq_len, uint32_t n_heads, uint32_t head_dim);

/* flash_attention_v2: Q,K,V [H,S,D], O [S, H*D].
 * dependencies/zimage.c3l/shaders/flash_attn.slang:38-241 (D fixed at 128
 * there; DP = D/2 generalises it). Only query blocks of 16 rows in
 * [qb_begin, qb_end) are computed (pass 0, UINT32_MAX for all). */
void orc_flash_attention_v2(const float *q, const float *k, const float *v,
                            float *o, uint32_t head_dim, uint32_t n_heads,
                            uint32_t seq_len, float scale, uint32_t qb_begin,
                            uint32_t qb_end, int n_threads);

/* spatial_attention: exact-softmax attention, Q,K,V,O [H,S,D].
 * lib/shaders/diffusion.slang:478-569. The reference's global scores buffer
 * is a per-row scratch here. Rows [row_begin,row_end) of every head. */
void orc_spatial_attention(const float *q, const float *k, const float *v,
                           float *o, uint32_t head_dim, uint32_t n_heads,
                           uint32_t seq_len, float scale, uint32_t row_begin,
                           uint32_t row_end, int n_threads);

/* vae_attention: single- or multi-head attention on Q, K, V, O in [S, C]
 * (head h at columns [h*D, h*D+D)), exact fp32 softmax over 4096-key tiles.
 * lib/shaders/diffusion.slang:1846-1975 (VaeAttentionParams {head_dim,
 * n_heads, seq_len, scale, channels}). Rows [row_begin,row_end) only. */
void orc_vae_attention(const float *q, const float *k, const float *v,
                       float *o, uint32_t head_dim, uint32_t n_heads,
                       uint32_t seq_len, float scale, uint32_t channels,
                       uint32_t row_begin, uint32_t row_end, int n_threads);

/* split_qkv: [N, 3*dim] -> three [N, dim].
 * dependencies/depth_anything.c3l/shaders/depth.slang:40-58. */
void orc_split_qkv(const float *qkv, float *q, float *k, float *v,
                   uint32_t dim, uint32_t n_rows);

/* Multi-axis RoPE table builder: for token t, axis a (dim d_a), k < d_a/2:
 * freq = 1/theta^(2k/d_a), angle = pos[t][a]*freq; pairs concatenated axis by
 * axis. dependencies/flux.c3l/flux_dit.c3:461-497,
 * dependencies/zimage.c3l/dit.c3:685-715. pos is [S, n_axes] int32. */
void orc_rope_tables(const int32_t *pos, uint32_t seq_len, uint32_t n_axes,
                     const uint32_t *axes_dims, float theta, float *cos_out,
                     float *sin_out);

/* The reference's per-block attention sequence for one batch element
 * (dependencies/flux.c3l/flux_dit.c3:812-872 and dit.c3:1445-1483):
 * batch_head_norm on Q and K rows [0,split) with gain set 0 and rows
 * [split,S) with gain set 1, transpose_heads x3, mrope on Q and K,
 * flash_attention_v2. q,k,v are [S, H*D] and are NOT modified; o is
 * [S, H*D]. Pass NULL gains to skip the norm, NULL cos to skip RoPE.
 * use_exact selects spatial_attention math (fp32, exact softmax) instead of
 * flash_attention_v2 (fp16 operands); its output is transposed back to
 * [S, H*D] as the reference call sites do (depth_anything.c3:628-630). */
void orc_attention_block(const float *q, const float *k, const float *v,
                         float *o, uint32_t seq_len, uint32_t n_heads,
                         uint32_t head_dim, float scale, float eps,
                         const float *q_gain0, const float *q_gain1,
                         const float *k_gain0, const float *k_gain1,
                         uint32_t split_row, const float *cos_t,
                         const float *sin_t, int use_exact,
                         uint32_t row_begin, uint32_t row_end, int n_threads);

/* fp64 exact-softmax attention on fp32 inputs [H,S,D] -> O [H,S,D] for error
 * budgeting (not a reference restatement). */
void orc_attention_f64(const float *q, const float *k, const float *v,
                       double *o, uint32_t head_dim, uint32_t n_heads,
                       uint32_t seq_len, double scale, uint32_t row_begin,
                       uint32_t row_end, int n_threads);

#ifdef __cplusplus
}
#endif
