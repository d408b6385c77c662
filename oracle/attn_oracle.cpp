// CPU oracle for the fused non-causal attention path of tonis2/llm-runner.
//
// TEST INFRASTRUCTURE ONLY: the checker for the CUDA path and the timed CPU
// baseline. Nothing in the shipped library links or calls this file.
//
// PARITY UNPINNED: the reference has no golden vectors for this path and
// cannot be built here (C3 + Slang + Vulkan). Every routine restates the
// reference source line by line; file:line citations are relative to the
// reference project root. Built with -ffp-contract=off so that every a*b+c
// rounds twice, as the shader source is written, and without -ffast-math so
// that summation order is kept.
#include "attn_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

// ---------------------------------------------------------------------------
// Rounding helpers. The shader converts with float16_t(v)
// (dependencies/zimage.c3l/shaders/flash_attn.slang:64,101,200); SPIR-V
// OpFConvert rounds to nearest even, which is what this restates.
// ---------------------------------------------------------------------------
static inline uint32_t f2u(float x) { uint32_t u; memcpy(&u, &x, 4); return u; }
static inline float u2f(uint32_t u) { float x; memcpy(&x, &u, 4); return x; }

extern "C" float orc_round_f16(float x) {
  uint32_t u = f2u(x);
  uint32_t sign = u & 0x80000000u;
  uint32_t absu = u & 0x7fffffffu;
  if (absu >= 0x7f800000u) return x;  // inf / nan pass through
  float a = u2f(absu);
  // Largest finite half is 65504; values rounding above it become inf.
  if (a >= 65520.0f) return u2f(sign | 0x7f800000u);
  if (a < 6.103515625e-05f) {
    // Subnormal half range: quantum is 2^-24. Round a / 2^-24 to an integer
    // with ties to even, which is exact in fp32 arithmetic here.
    float scaled = a * 16777216.0f;  // a * 2^24, exact
    float r = nearbyintf(scaled);    // default rounding mode: ties to even
    return u2f(sign | f2u(r / 16777216.0f));
  }
  // Normal range: keep 10 explicit mantissa bits (drop 13), ties to even.
  uint32_t lsb = (absu >> 13) & 1u;
  uint32_t rounded = (absu + 0x0fffu + lsb) & ~0x1fffu;
  return u2f(sign | rounded);
}

extern "C" float orc_round_bf16(float x) {
  uint32_t u = f2u(x);
  if ((u & 0x7fffffffu) > 0x7f800000u) return x;  // nan
  uint32_t lsb = (u >> 16) & 1u;
  u = (u + 0x7fffu + lsb) & 0xffff0000u;
  return u2f(u);
}

// Thread count for every parallel loop of this library (0 keeps the OpenMP
// default). Launchers such as torchrun set OMP_NUM_THREADS=1 per process;
// the CPU baseline sets the host's core count explicitly instead.
extern "C" void orc_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

static int pick_threads(int n) {
#ifdef _OPENMP
  return n > 0 ? n : omp_get_max_threads();
#else
  (void)n;
  return 1;
#endif
}

// ---------------------------------------------------------------------------
// batch_head_norm: dependencies/zimage.c3l/shaders/zimage.slang:623-659.
// One 256-thread workgroup per (pos, head): thread gi accumulates x[i]^2 for
// i = gi, gi+256, ... (:640-644), tree reduction s = 128..1 (:649-654),
// rms = 1/sqrt(sum/D + eps) (:656), x * rms * w[i] (:658).
// ---------------------------------------------------------------------------
extern "C" void orc_batch_head_norm(float *data, const float *gain,
                                    uint32_t H, uint32_t D, uint32_t S,
                                    float eps) {
#pragma omp parallel for schedule(static)
  for (int64_t wg = 0; wg < (int64_t)S * H; wg++) {
    uint64_t pos = wg / H, h = wg % H;
    float *x = data + (pos * H + h) * D;
    float sh[256];
    for (uint32_t gi = 0; gi < 256; gi++) {
      float s = 0.0f;
      for (uint32_t i = gi; i < D; i += 256) s += x[i] * x[i];
      sh[gi] = s;
    }
    for (uint32_t s = 128; s > 0; s >>= 1)
      for (uint32_t gi = 0; gi < s; gi++) sh[gi] += sh[gi + s];
    float rms = 1.0f / sqrtf(sh[0] / (float)D + eps);
    for (uint32_t i = 0; i < D; i++) x[i] = x[i] * rms * gain[i];
  }
}

// transpose_heads: dependencies/zimage.c3l/shaders/zimage.slang:575-601.
extern "C" void orc_transpose_heads(const float *in, float *out, uint32_t S,
                                    uint32_t H, uint32_t D,
                                    uint32_t direction) {
  int64_t total = (int64_t)S * H * D;
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < total; t++) {
    uint64_t d = t % D, rem = t / D;
    if (direction == 0) {
      uint64_t seq = rem / H, h = rem % H;
      out[h * S * D + seq * D + d] = in[t];
    } else {
      uint64_t h = rem / S, seq = rem % S;
      out[seq * H * D + h * D + d] = in[t];
    }
  }
}

// mrope: dependencies/zimage.c3l/shaders/mrope.slang:33-54.
extern "C" void orc_mrope(float *data, const float *cos_t, const float *sin_t,
                          uint32_t S, uint32_t H, uint32_t D) {
  uint32_t half = D / 2;
#pragma omp parallel for schedule(static)
  for (int64_t hp = 0; hp < (int64_t)H * S; hp++) {
    uint64_t h = hp / S, pos = hp % S;
    float *x = data + h * S * D + pos * D;
    for (uint32_t pair = 0; pair < half; pair++) {
      float cv = cos_t[pos * half + pair], sv = sin_t[pos * half + pair];
      float x0 = x[2 * pair], x1 = x[2 * pair + 1];
      x[2 * pair] = x0 * cv - x1 * sv;
      x[2 * pair + 1] = x0 * sv + x1 * cv;
    }
  }
}

// ---------------------------------------------------------------------------
// flash_attention_v2: dependencies/zimage.c3l/shaders/flash_attn.slang:38-241.
// BR = 16 query rows per workgroup (:18), BC = 32 keys per tile (:19).
// ---------------------------------------------------------------------------
static void fa2_block(const float *Q, const float *K, const float *V, float *O,
                      uint32_t D, uint32_t H, uint32_t S, float scale,
                      uint32_t head, uint32_t qblk) {
  const uint32_t BR = 16, BC = 32, DP = D / 2;
  const uint32_t q_start = qblk * BR;
  const uint64_t head_offset = (uint64_t)head * S * D;  // :49
  std::vector<float> qt(BR * D), kt(BC * D), vt(BC * D);
  // Step 1 (:52-66): Q tile rounded to fp16, zero beyond S.
  for (uint32_t r = 0; r < BR; r++)
    for (uint32_t d = 0; d < D; d++) {
      uint32_t aq = q_start + r;
      qt[r * D + d] = aq < S ? orc_round_f16(Q[head_offset + (uint64_t)aq * D + d]) : 0.0f;
    }
  // Step 2 (:70-79).
  std::vector<float> acc_x(BR * DP, 0.0f), acc_y(BR * DP, 0.0f);
  float m[16], l[16], resc[16];
  for (uint32_t r = 0; r < BR; r++) { m[r] = -1.0e30f; l[r] = 0.0f; }
  float Sv[16 * 32], red[16 * 32], mnew[16 * 32];
  const uint32_t nkv = (S + BC - 1) / BC;  // :83
  for (uint32_t kb = 0; kb < nkv; kb++) {
    const uint32_t kv_start = kb * BC;
    // 3a (:88-103): K tile rounded to fp16.
    for (uint32_t r = 0; r < BC; r++)
      for (uint32_t d = 0; d < D; d++) {
        uint32_t ak = kv_start + r;
        kt[r * D + d] = ak < S ? orc_round_f16(K[head_offset + (uint64_t)ak * D + d]) : 0.0f;
      }
    // 3b (:108-122): scores; dot accumulates q.x*k.x + q.y*k.y per pair.
    for (uint32_t qr = 0; qr < BR; qr++) {
      float dot[32];
      for (uint32_t kc = 0; kc < BC; kc++) dot[kc] = 0.0f;
      const float *qrow = &qt[qr * D];
      for (uint32_t dp = 0; dp < DP; dp++) {
        float qx = qrow[2 * dp], qy = qrow[2 * dp + 1];
        for (uint32_t kc = 0; kc < BC; kc++) {
          float t = qx * kt[kc * D + 2 * dp] + qy * kt[kc * D + 2 * dp + 1];
          dot[kc] += t;
        }
      }
      for (uint32_t kc = 0; kc < BC; kc++) {
        float dv = dot[kc] * scale;
        bool valid = (kv_start + kc < S) && (q_start + qr < S);
        Sv[qr * BC + kc] = valid ? dv : -1.0e30f;
      }
    }
    // 3c (:126-138): row max by tree (max is order independent).
    for (uint32_t f = 0; f < BR * BC; f++) red[f] = Sv[f];
    for (uint32_t s = 16; s > 0; s >>= 1)
      for (uint32_t f = 0; f < BR * BC; f++)
        if ((f % BC) < s) red[f] = fmaxf(red[f], red[f + s]);
    // 3d (:142-153).
    float expv[16 * 32];
    for (uint32_t f = 0; f < BR * BC; f++) {
      uint32_t qr = f / BC, kc = f % BC;
      float tile_max = red[qr * BC];
      float m_old = m[qr];
      mnew[f] = fmaxf(m_old, tile_max);
      bool valid = (kv_start + kc < S) && (q_start + qr < S);
      expv[f] = valid ? expf(Sv[f] - mnew[f]) : 0.0f;
    }
    // Row sum by the same 5-step tree (:157-170).
    for (uint32_t f = 0; f < BR * BC; f++) { Sv[f] = expv[f]; red[f] = expv[f]; }
    for (uint32_t s = 16; s > 0; s >>= 1)
      for (uint32_t f = 0; f < BR * BC; f++)
        if ((f % BC) < s) red[f] += red[f + s];
    // Running state (:173-184).
    for (uint32_t qr = 0; qr < BR; qr++) {
      uint32_t f = qr * BC;
      float tile_sum = red[f];
      float rv = expf(m[qr] - mnew[f]);
      m[qr] = mnew[f];
      l[qr] = rv * l[qr] + tile_sum;
      resc[qr] = rv;
    }
    // 3e (:188-202): V tile rounded to fp16.
    for (uint32_t r = 0; r < BC; r++)
      for (uint32_t d = 0; d < D; d++) {
        uint32_t ak = kv_start + r;
        vt[r * D + d] = ak < S ? orc_round_f16(V[head_offset + (uint64_t)ak * D + d]) : 0.0f;
      }
    // 3f (:207-223).
    for (uint32_t qr = 0; qr < BR; qr++)
      for (uint32_t dp = 0; dp < DP; dp++) {
        float nx = 0.0f, ny = 0.0f;
        for (uint32_t kv = 0; kv < BC; kv++) {
          float sv = Sv[qr * BC + kv];
          nx += sv * vt[kv * D + 2 * dp];
          ny += sv * vt[kv * D + 2 * dp + 1];
        }
        float r = resc[qr];
        acc_x[qr * DP + dp] = acc_x[qr * DP + dp] * r + nx;
        acc_y[qr * DP + dp] = acc_y[qr * DP + dp] * r + ny;
      }
  }
  // Step 4 (:228-240): normalise and write O[S, H*D].
  const uint64_t dim = (uint64_t)H * D;
  for (uint32_t qr = 0; qr < BR; qr++) {
    uint32_t aq = q_start + qr;
    if (aq >= S) continue;
    float inv_l = 1.0f / l[qr];
    for (uint32_t dp = 0; dp < DP; dp++) {
      uint64_t ob = (uint64_t)aq * dim + (uint64_t)head * D + dp * 2;
      O[ob] = acc_x[qr * DP + dp] * inv_l;
      O[ob + 1] = acc_y[qr * DP + dp] * inv_l;
    }
  }
}

extern "C" void orc_flash_attention_v2(const float *q, const float *k,
                                       const float *v, float *o, uint32_t D,
                                       uint32_t H, uint32_t S, float scale,
                                       uint32_t qb_begin, uint32_t qb_end,
                                       int n_threads) {
  uint32_t nqb = (S + 15) / 16;
  if (qb_end > nqb) qb_end = nqb;
  if (qb_begin >= qb_end) return;
  int64_t nb = (int64_t)(qb_end - qb_begin);
  int64_t total = nb * H;
  int nt = pick_threads(n_threads);
#pragma omp parallel for schedule(dynamic, 1) num_threads(nt)
  for (int64_t t = 0; t < total; t++) {
    uint32_t head = (uint32_t)(t / nb);
    uint32_t qb = qb_begin + (uint32_t)(t % nb);
    fa2_block(q, k, v, o, D, H, S, scale, head, qb);
  }
}

// ---------------------------------------------------------------------------
// spatial_attention: lib/shaders/diffusion.slang:478-569. One workgroup of
// 256 threads per (head, query). Thread gi owns keys gi, gi+256, ... for the
// strided partial max/sum (:527-529, :543-547), then tree reductions over 256
// (:531-534, :549-552). p = score / sum (:557). O[d] = sum over pos in order
// (:561-567).
// ---------------------------------------------------------------------------
static void spatial_row(const float *Q, const float *K, const float *V,
                        float *O, uint32_t D, uint32_t S, float scale,
                        uint32_t head, uint32_t qpos, float *sc) {
  const uint64_t ho = (uint64_t)head * S * D;
  const float *qr = Q + ho + (uint64_t)qpos * D;
  for (uint32_t kv = 0; kv < S; kv++) {
    const float *kr = K + ho + (uint64_t)kv * D;
    float dot = 0.0f;
    for (uint32_t d = 0; d < D; d++) dot += qr[d] * kr[d];
    sc[kv] = dot * scale;
  }
  float sh[256];
  for (uint32_t gi = 0; gi < 256; gi++) {
    float mx = -1.0e30f;
    for (uint32_t i = gi; i < S; i += 256) mx = fmaxf(mx, sc[i]);
    sh[gi] = mx;
  }
  for (uint32_t s = 128; s > 0; s >>= 1)
    for (uint32_t gi = 0; gi < s; gi++) sh[gi] = fmaxf(sh[gi], sh[gi + s]);
  float gmax = sh[0];
  for (uint32_t gi = 0; gi < 256; gi++) {
    float sum = 0.0f;
    for (uint32_t i = gi; i < S; i += 256) {
      float val = expf(sc[i] - gmax);
      sc[i] = val;
      sum += val;
    }
    sh[gi] = sum;
  }
  for (uint32_t s = 128; s > 0; s >>= 1)
    for (uint32_t gi = 0; gi < s; gi++) sh[gi] += sh[gi + s];
  float gsum = sh[0];
  for (uint32_t i = 0; i < S; i++) sc[i] /= gsum;
  float *orow = O + ho + (uint64_t)qpos * D;
  for (uint32_t d = 0; d < D; d++) {
    float acc = 0.0f;
    for (uint32_t pos = 0; pos < S; pos++) acc += sc[pos] * V[ho + (uint64_t)pos * D + d];
    orow[d] = acc;
  }
}

extern "C" void orc_spatial_attention(const float *q, const float *k,
                                      const float *v, float *o, uint32_t D,
                                      uint32_t H, uint32_t S, float scale,
                                      uint32_t row_begin, uint32_t row_end,
                                      int n_threads) {
  if (row_end > S) row_end = S;
  if (row_begin >= row_end) return;
  int64_t nr = row_end - row_begin;
  int64_t total = nr * H;
  int nt = pick_threads(n_threads);
#pragma omp parallel num_threads(nt)
  {
    std::vector<float> sc(S);
#pragma omp for schedule(dynamic, 4)
    for (int64_t t = 0; t < total; t++) {
      uint32_t head = (uint32_t)(t / nr);
      uint32_t row = row_begin + (uint32_t)(t % nr);
      spatial_row(q, k, v, o, D, S, scale, head, row, sc.data());
    }
  }
}

// vae_attention: lib/shaders/diffusion.slang:1846-1975. One (head, query) per
// 256-lane workgroup over Q, K, V, O in [S, C] (head h at columns
// [h*D, h*D+D)); keys in tiles of 4096 (:1878-1881) with a running max and
// sum (:1921-1960). Per tile: scores = (q . k) * scale with d ascending
// (:1884-1889); the tile max and sum are 256 lane partials (lane gi takes
// keys gi, gi+256, ...) folded by the shader's tree (:1893-1922); the output
// is rescaled by alpha = exp(old_max - new_max) and gains sum_i p_i v_i with
// i ascending (:1940-1951); the end multiplies by 1/run_sum (:1964-1972).
static void vae_row(const float *Q, const float *K, const float *V, float *O,
                    uint32_t D, uint32_t S, uint32_t C, float scale,
                    uint32_t head, uint32_t qpos, float *sc, float *acc) {
  const uint32_t TILE = 4096;
  const uint64_t hd = (uint64_t)head * D;
  const float *qr = Q + (uint64_t)qpos * C + hd;
  for (uint32_t d = 0; d < D; d++) acc[d] = 0.0f;
  float run_max = -1.0e30f, run_sum = 0.0f;
  float sh[256];
  for (uint32_t t0 = 0; t0 < S; t0 += TILE) {
    const uint32_t len = (S - t0 < TILE) ? S - t0 : TILE;
    for (uint32_t i = 0; i < len; i++) {
      const float *kr = K + (uint64_t)(t0 + i) * C + hd;
      float dot = 0.0f;
      for (uint32_t d = 0; d < D; d++) dot += qr[d] * kr[d];
      sc[i] = dot * scale;
    }
    for (uint32_t gi = 0; gi < 256; gi++) {
      float mx = -1.0e30f;
      for (uint32_t i = gi; i < len; i += 256) mx = fmaxf(mx, sc[i]);
      sh[gi] = mx;
    }
    for (uint32_t s = 128; s > 0; s >>= 1)
      for (uint32_t gi = 0; gi < s; gi++) sh[gi] = fmaxf(sh[gi], sh[gi + s]);
    const float tile_max = sh[0];
    const float new_max = fmaxf(run_max, tile_max);
    const float alpha = expf(run_max - new_max);
    for (uint32_t gi = 0; gi < 256; gi++) {
      float sum = 0.0f;
      for (uint32_t i = gi; i < len; i += 256) {
        const float e = expf(sc[i] - new_max);
        sc[i] = e;
        sum += e;
      }
      sh[gi] = sum;
    }
    for (uint32_t s = 128; s > 0; s >>= 1)
      for (uint32_t gi = 0; gi < s; gi++) sh[gi] += sh[gi + s];
    const float tile_sum = sh[0];
    for (uint32_t d = 0; d < D; d++) {
      acc[d] *= alpha;
      float va = 0.0f;
      for (uint32_t i = 0; i < len; i++) va += sc[i] * V[(uint64_t)(t0 + i) * C + hd + d];
      acc[d] += va;
    }
    run_max = new_max;
    run_sum = run_sum * alpha + tile_sum;
  }
  const float inv = 1.0f / run_sum;
  float *orow = O + (uint64_t)qpos * C + hd;
  for (uint32_t d = 0; d < D; d++) orow[d] = acc[d] * inv;
}

extern "C" void orc_vae_attention(const float *q, const float *k, const float *v,
                                  float *o, uint32_t D, uint32_t H, uint32_t S,
                                  float scale, uint32_t C, uint32_t row_begin,
                                  uint32_t row_end, int n_threads) {
  if (row_end > S) row_end = S;
  if (row_begin >= row_end) return;
  const int64_t nr = row_end - row_begin, total = nr * H;
  const int nt = pick_threads(n_threads);
#pragma omp parallel num_threads(nt)
  {
    std::vector<float> sc(S < 4096 ? S : 4096), acc(D);
#pragma omp for schedule(dynamic, 4)
    for (int64_t t = 0; t < total; t++)
      vae_row(q, k, v, o, D, S, C, scale, (uint32_t)(t / nr), row_begin + (uint32_t)(t % nr),
              sc.data(), acc.data());
  }
}

// split_qkv: dependencies/depth_anything.c3l/shaders/depth.slang:40-58.
extern "C" void orc_split_qkv(const float *qkv, float *q, float *k, float *v,
                              uint32_t dim, uint32_t n_rows) {
  uint64_t total = (uint64_t)n_rows * dim;
  for (uint64_t t = 0; t < total; t++) {
    uint64_t row = t / dim, d = t % dim, base = row * 3 * dim;
    q[t] = qkv[base + d];
    k[t] = qkv[base + dim + d];
    v[t] = qkv[base + 2 * dim + d];
  }
}

// Host RoPE tables: dependencies/flux.c3l/flux_dit.c3:461-497 and
// dependencies/zimage.c3l/dit.c3:685-715. freq = 1/pow(theta, 2k/d_a) and
// angle = pos * freq, both in float; cos/sin in float.
extern "C" void orc_rope_tables(const int32_t *pos, uint32_t S,
                                uint32_t n_axes, const uint32_t *axes_dims,
                                float theta, float *cos_out, float *sin_out) {
  uint32_t half = 0;
  for (uint32_t a = 0; a < n_axes; a++) half += axes_dims[a] / 2;
  for (uint64_t t = 0; t < S; t++) {
    uint32_t pair = 0;
    for (uint32_t a = 0; a < n_axes; a++) {
      uint32_t ha = axes_dims[a] / 2;
      for (uint32_t kk = 0; kk < ha; kk++) {
        float freq = 1.0f / powf(theta, (float)(2 * kk) / (float)axes_dims[a]);
        float angle = (float)pos[t * n_axes + a] * freq;
        cos_out[t * half + pair] = cosf(angle);
        sin_out[t * half + pair] = sinf(angle);
        pair++;
      }
    }
  }
}

// The per-block call sequence: dependencies/flux.c3l/flux_dit.c3:812-872
// (norm txt/img rows with their own gains, transpose x3, mrope x2, FA) and
// dependencies/depth_anything.c3l/depth_anything.c3:614-630 (transpose,
// spatial_attention, transpose back).
extern "C" void orc_attention_block(
    const float *q, const float *k, const float *v, float *o, uint32_t S,
    uint32_t H, uint32_t D, float scale, float eps, const float *q_gain0,
    const float *q_gain1, const float *k_gain0, const float *k_gain1,
    uint32_t split_row, const float *cos_t, const float *sin_t, int use_exact,
    uint32_t row_begin, uint32_t row_end, int n_threads) {
  const uint64_t n = (uint64_t)S * H * D, rowlen = (uint64_t)H * D;
  std::vector<float> qn(q, q + n), kn(k, k + n);
  if (split_row > S) split_row = S;
  if (q_gain0) {
    const float *g1 = q_gain1 ? q_gain1 : q_gain0;
    orc_batch_head_norm(qn.data(), q_gain0, H, D, split_row, eps);
    orc_batch_head_norm(qn.data() + split_row * rowlen, g1, H, D, S - split_row, eps);
  }
  if (k_gain0) {
    const float *g1 = k_gain1 ? k_gain1 : k_gain0;
    orc_batch_head_norm(kn.data(), k_gain0, H, D, split_row, eps);
    orc_batch_head_norm(kn.data() + split_row * rowlen, g1, H, D, S - split_row, eps);
  }
  std::vector<float> qt(n), kt(n), vt(n);
  orc_transpose_heads(qn.data(), qt.data(), S, H, D, 0);
  orc_transpose_heads(kn.data(), kt.data(), S, H, D, 0);
  orc_transpose_heads(v, vt.data(), S, H, D, 0);
  if (cos_t) {
    orc_mrope(qt.data(), cos_t, sin_t, S, H, D);
    orc_mrope(kt.data(), cos_t, sin_t, S, H, D);
  }
  if (row_end > S) row_end = S;
  if (!use_exact) {
    orc_flash_attention_v2(qt.data(), kt.data(), vt.data(), o, D, H, S, scale,
                           row_begin / 16, (row_end + 15) / 16, n_threads);
  } else {
    std::vector<float> ot(n, 0.0f);
    orc_spatial_attention(qt.data(), kt.data(), vt.data(), ot.data(), D, H, S,
                          scale, row_begin, row_end, n_threads);
    for (uint64_t h = 0; h < H; h++)
      for (uint64_t s = row_begin; s < row_end; s++)
        memcpy(o + s * rowlen + h * D, ot.data() + (h * S + s) * D, D * 4);
  }
}

extern "C" void orc_attention_f64(const float *q, const float *k,
                                  const float *v, double *o, uint32_t D,
                                  uint32_t H, uint32_t S, double scale,
                                  uint32_t row_begin, uint32_t row_end,
                                  int n_threads) {
  if (row_end > S) row_end = S;
  if (row_begin >= row_end) return;
  int64_t nr = row_end - row_begin, total = nr * H;
  int nt = pick_threads(n_threads);
#pragma omp parallel num_threads(nt)
  {
    std::vector<double> sc(S);
#pragma omp for schedule(dynamic, 4)
    for (int64_t t = 0; t < total; t++) {
      uint64_t h = t / nr, r = row_begin + t % nr, ho = h * S * D;
      double mx = -1e300;
      for (uint64_t j = 0; j < S; j++) {
        double dot = 0;
        for (uint64_t d = 0; d < D; d++) dot += (double)q[ho + r * D + d] * k[ho + j * D + d];
        sc[j] = dot * scale;
        if (sc[j] > mx) mx = sc[j];
      }
      double sum = 0;
      for (uint64_t j = 0; j < S; j++) { sc[j] = exp(sc[j] - mx); sum += sc[j]; }
      for (uint64_t d = 0; d < D; d++) {
        double acc = 0;
        for (uint64_t j = 0; j < S; j++) acc += sc[j] * v[ho + j * D + d];
        o[ho + r * D + d] = acc / sum;
      }
    }
  }
}
