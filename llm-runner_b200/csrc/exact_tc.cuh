// Exact fp32 attention (the reference's spatial_attention math,
// lib/shaders/diffusion.slang:478-569: fp32 operands, fp32 dot products,
// exact softmax) on the 5th-generation tensor cores, D = 64.
//
// Three-pass TF32 ("3xTF32"): tcgen05.mma kind::tf32 reads fp32 operands as
// TF32 (the 13 low mantissa bits dropped). Each operand is split as
// x = g(x) + r(x), g(x) = x rounded to the nearest TF32 value, r(x) = x - g(x)
// (exact in fp32, |r| <= 2^-11 |x|), and each product as
//   a*b ~= g(a) g(b) + g(a) r(b) + r(a) g(b)
// whose error (the dropped r*r term and the truncation of r to TF32) is
// below 2^-20 relative, accumulated in fp32 in TMEM. A small kernel
// (tf32_prepare_kernel) writes g and r of Q and K, and of V transposed
// (kind::tf32 takes no MN-major shared-memory operand); the softmax threads
// split P themselves.
//
// CTA = 128 query rows of one (b, h); 192 threads:
//   warps 0-3  softmax (thread i owns query row i = TMEM lane i)
//   warp  4    TMA producer: g(Q) and r(Q) once, then per 128-key block
//              g(K), r(K), g(V)^T, r(V)^T into four 32 KB slots
//   warp  5    TMEM owner and MMA issuer (one elected lane)
// TMEM (512 columns): S0 [0,128) S1 [128,256) r(P) [256,384) O [384,448).
// S_j lands in buffer j&1 while the softmax works on the other one; the
// softmax writes g(P_j) over S_j and r(P_j) into its own columns; MMA order: S_0, then per block S_{j+1}, PV_j. P feeds the MMA
// from TMEM. The row max is lazy (P rescaled only when the max grows by more
// than 2^8), which is exact softmax up to fp32 rounding.
#pragma once
#include <math.h>

#include "kernels_misc.cuh"
#include "ptx.cuh"

namespace llmr {

// D[tmem] (+)= A[smem] * B[smem], kind::tf32 (fp32 data read as TF32).
__device__ __forceinline__ void mma_ss_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem], kind::tf32.
__device__ __forceinline__ void mma_ts_tf32(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Instruction descriptor for kind::tf32 with fp32 accumulation: c_format F32
// (bit 4), A and B format TF32 (2 in bits 7-9 and 10-12), A K-major, B
// major in bit 16, N >> 3 in bits 17-22, M >> 4 in bits 24-28.
__host__ __device__ constexpr uint32_t idesc_tf32(uint32_t M, uint32_t N, uint32_t b_mn_major) {
  return (1u << 4) | (2u << 7) | (2u << 10) | (b_mn_major << 16) | ((N >> 3) << 17) |
         ((M >> 4) << 24);
}

// x rounded to the nearest TF32 value (ties away from zero): the "big" part
// of the split; its 13 low mantissa bits are zero, so the tensor core reads
// it exactly.
__device__ __forceinline__ float tf32_big(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// Operand preparation for the tensor-core exact kernel, dense fp32
// [B*H][S][D] inputs: g (big) and r (residual) parts of Q and K in the same
// layout, and of V transposed to [B*H][D][Sp] (keys contiguous, Sp = S
// rounded up to a multiple of 4 so rows are 16-byte aligned). Grid
// (ceil(S/32), D/32, B*H), 256 threads: one 32 x 32 tile each, V transposed
// through shared memory.
__global__ void __launch_bounds__(256)
    tf32_prepare_kernel(const float *q, const float *k, const float *v, float *qg, float *qr,
                        float *kg, float *kr, float *vtg, float *vtr, int S, int Sp, int D) {
  __shared__ float tile[32][33];
  const long long bh = blockIdx.z;
  const int s0 = blockIdx.x * 32, d0 = blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const long long base = bh * S * D;
  for (int r = ty; r < 32; r += 8) {
    const int s = s0 + r;
    if (s < S) {
      const long long i = base + (long long)s * D + d0 + tx;
      const float xq = q[i], xk = k[i];
      const float gq = tf32_big(xq), gk = tf32_big(xk);
      qg[i] = gq;
      qr[i] = xq - gq;
      kg[i] = gk;
      kr[i] = xk - gk;
      tile[r][tx] = v[i];
    }
  }
  __syncthreads();
  const long long tbase = bh * D * Sp;
  for (int r = ty; r < 32; r += 8) {
    const int s = s0 + tx;
    if (s < S) {
      const float x = tile[tx][r];
      const float g = tf32_big(x);
      const long long o = tbase + (long long)(d0 + r) * Sp + s;
      vtg[o] = g;
      vtr[o] = x - g;
    }
  }
}

struct ExactTcCfg {
  static constexpr int D = 64;
  static constexpr int BM = 128;                   // query rows per CTA
  static constexpr int BN = 128;                   // keys per block
  static constexpr int CHUNK = 128 * 128;          // 32 fp32 columns x 128 rows, SW128
  static constexpr int TILE = BM * D * 4;          // one fp32 tile of 128 rows (32 KB)
  static constexpr int Q_OFF = 0;                  // g(Q), r(Q)
  static constexpr int KV_OFF = 2 * TILE;          // slots: g(K), r(K), g(V)^T, r(V)^T
  static constexpr int VCHUNK = 64 * 128;          // 32 keys x 64 d-rows of V^T, SW128
  static constexpr int BAR_OFF = KV_OFF + 4 * TILE;
  // barriers: q_full, kv_full[4], kv_empty[4], s_full[2], p_full, pv_done,
  // drain; then tmem base word and abort flag
  static constexpr int NBAR = 1 + 4 + 4 + 2 + 1 + 1 + 1;
  static constexpr int SMEM_BYTES = BAR_OFF + NBAR * 8 + 16 + 1024;
  static constexpr int THREADS = 192;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t PL_COL = 256;          // r(P)
  static constexpr uint32_t O_COL = 384;
  static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
};

// Lazy-max threshold (log2 units): P <= 2^8 between rescales.
constexpr float kExactMaxExp = 8.0f;

// Maps (fp32, SW128): tmQ/tmK (g parts) and tmQr/tmKr (r parts) over
// (d, s, h, b) with 32 x 128 boxes; tmV/tmVr over g(V)^T and r(V)^T,
// (s, d, h, b) with 32 x 64 boxes.
__global__ void __launch_bounds__(192, 1)
    attn_exact_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                         const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV,
                         const __grid_constant__ CUtensorMap tmQr,
                         const __grid_constant__ CUtensorMap tmKr,
                         const __grid_constant__ CUtensorMap tmVr, const ExactParams p,
                         int *err) {
  using C = ExactTcCfg;
  constexpr int D = C::D;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t *smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t *sQ = smem + C::Q_OFF;
  uint8_t *sKV = smem + C::KV_OFF;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
  uint64_t *q_full = bars;
  uint64_t *kv_full = bars + 1;     // [slot]: 0 g(K), 1 r(K), 2 g(V)^T, 3 r(V)^T
  uint64_t *kv_empty = kv_full + 4;
  uint64_t *s_full = kv_empty + 4;  // [buffer]
  uint64_t *p_full = s_full + 2;
  uint64_t *pv_done = p_full + 1;
  uint64_t *drain = pv_done + 1;
  uint32_t *tmem_base_slot = reinterpret_cast<uint32_t *>(drain + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_base_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const int q0 = blockIdx.x * C::BM;
  const int nblk = (p.S + C::BN - 1) / C::BN;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 4; i++) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    mbar_init(p_full, 4);  // one arrival per softmax warp
    mbar_init(pv_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_base_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_slot;

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const CUtensorMap *maps[4] = {&tmK, &tmKr, &tmV, &tmVr};
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmQr);
      for (int i = 0; i < 4; i++) tma_prefetch_desc(maps[i]);
      mbar_arrive_expect_tx(q_full, 2 * C::TILE);
      for (int c = 0; c < D / 32; c++) {
        tma_load_4d(sQ + c * C::CHUNK, &tmQ, q_full, c * 32, q0, h, b);
        tma_load_4d(sQ + C::TILE + c * C::CHUNK, &tmQr, q_full, c * 32, q0, h, b);
      }
      bool ok = true;
      int armed[4] = {0, 0, 0, 0};  // loads armed per slot
      for (int j = 0; j < nblk && ok; j++) {
        for (int s = 0; s < 4; s++) {
          if (j > 0 && !mbar_wait(&kv_empty[s], (j - 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&kv_full[s], C::TILE);
          if (s < 2) {  // K rows: 2 chunks of 32 d-columns
            for (int c = 0; c < D / 32; c++)
              tma_load_4d(sKV + s * C::TILE + c * C::CHUNK, maps[s], &kv_full[s], c * 32,
                          j * C::BN, h, b);
          } else {  // V^T rows (d): 4 chunks of 32 keys
            for (int c = 0; c < C::BN / 32; c++)
              tma_load_4d(sKV + s * C::TILE + c * C::VCHUNK, maps[s], &kv_full[s],
                          j * C::BN + c * 32, 0, h, b);
          }
          armed[s] = j + 1;
        }
      }
      // Every armed copy lands before the CTA exits (also on the abort path).
      mbar_wait_raw(q_full, 0, 100000000ull);
      for (int s = 0; s < 4; s++)
        if (armed[s] > 0) mbar_wait_raw(&kv_full[s], (armed[s] - 1) & 1, 100000000ull);
    }
  } else if (warp == 5) {
    // ------------------------------------------------------- MMA issuer
    constexpr uint32_t IDESC_S = idesc_tf32(128, C::BN, 0);
    constexpr uint32_t IDESC_O = idesc_tf32(128, D, 0);  // V^T: K-major
    const uint32_t sQa = smem_u32(sQ), sKVa = smem_u32(sKV);
    // S_buf = g(Q) g(K)^T + g(Q) r(K)^T + r(Q) g(K)^T over D (8 steps of 8).
    auto issue_s = [&](int buf) {
#pragma unroll
      for (int pass = 0; pass < 3; pass++) {
        const uint32_t qa = sQa + (pass == 2 ? C::TILE : 0);
        const uint32_t ka = sKVa + (pass == 1 ? C::TILE : 0);
#pragma unroll
        for (int kk = 0; kk < D / 8; kk++) {
          const uint32_t off = (kk >> 2) * C::CHUNK + (kk & 3) * 32;
          if (elect_one())
            mma_ss_tf32(tmem + buf * 128, sdesc_sw128(qa + off, 16, 1024),
                        sdesc_sw128(ka + off, 16, 1024), IDESC_S, (pass > 0 || kk > 0) ? 1u : 0u);
        }
      }
    };
    // O (+)= g(P) g(V) + g(P) r(V) + r(P) g(V) over the block's 128 keys
    // (16 steps of 8); V^T is the K-major B operand (rows d, keys contiguous).
    auto issue_pv = [&](int buf, bool acc) {
#pragma unroll
      for (int pass = 0; pass < 3; pass++) {
        const uint32_t pa = tmem + (pass == 2 ? C::PL_COL : (uint32_t)buf * 128u);
        const uint32_t va = sKVa + (pass == 1 ? 3 : 2) * C::TILE;
#pragma unroll
        for (int ks = 0; ks < C::BN / 8; ks++) {
          const uint32_t off = (ks >> 2) * C::VCHUNK + (ks & 3) * 32;
          if (elect_one())
            mma_ts_tf32(tmem + C::O_COL, pa + ks * 8, sdesc_sw128(va + off, 16, 1024), IDESC_O,
                        (acc || pass > 0 || ks > 0) ? 1u : 0u);
        }
      }
    };
    bool ok = mbar_wait(q_full, 0, abort_flag) && mbar_wait(&kv_full[0], 0, abort_flag) &&
              mbar_wait(&kv_full[1], 0, abort_flag);
    if (ok) {
      tc_fence_after();
      issue_s(0);
      if (elect_one()) mma_commit(&s_full[0]);
      if (elect_one()) mma_commit(&kv_empty[0]);
      if (elect_one()) mma_commit(&kv_empty[1]);
    }
    for (int j = 0; j < nblk && ok; j++) {
      if (j + 1 < nblk) {
        // S_{j+1} overwrites buffer (j+1)&1, whose P_{j-1} PV_{j-1} (issued
        // before, in order) has read.
        const uint32_t ph = (j + 1) & 1;
        if (!(ok = mbar_wait(&kv_full[0], ph, abort_flag) && mbar_wait(&kv_full[1], ph, abort_flag)))
          break;
        tc_fence_after();
        issue_s((j + 1) & 1);
        if (elect_one()) mma_commit(&s_full[(j + 1) & 1]);
        if (elect_one()) mma_commit(&kv_empty[0]);
        if (elect_one()) mma_commit(&kv_empty[1]);
      }
      if (!(ok = mbar_wait(p_full, j & 1, abort_flag) && mbar_wait(&kv_full[2], j & 1, abort_flag) &&
                 mbar_wait(&kv_full[3], j & 1, abort_flag)))
        break;
      tc_fence_after();
      issue_pv(j & 1, j > 0);
      if (elect_one()) mma_commit(pv_done);
      if (elect_one()) mma_commit(&kv_empty[2]);
      if (elect_one()) mma_commit(&kv_empty[3]);
    }
    if (elect_one()) mma_commit(drain);
    mbar_wait_raw(drain, 0, 100000000ull);
  } else {
    // ------------------------------------------------------------- softmax
    const int row = threadIdx.x;  // TMEM lane
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const float sl2 = p.scale * 1.4426950408889634f;
    float m_used = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int j = 0; j < nblk; j++) {
      const int buf = j & 1;
      const uint32_t tS = tmem + lane_off + buf * 128;
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[buf], (j >> 1) & 1, abort_flag));
      if (!ok) break;
      tc_fence_after();
      uint32_t sv[128];
#pragma unroll
      for (int c = 0; c < 4; c++) tmem_ld32(tS + c * 32, sv + c * 32);
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 4; c++) reg_fence32(sv + c * 32);
      const int valid = p.S - j * C::BN;
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < 128; i++) {
        float x = __uint_as_float(sv[i]) * sl2;
        if (i >= valid) x = -INFINITY;
        sv[i] = __float_as_uint(x);
        mx = fmaxf(mx, x);
      }
      const bool need = mx > m_used + kExactMaxExp;  // always on block 0
      const float m_tgt = need ? mx : m_used;
      // PV_{j-1} has read r(P_{j-1}) and no longer accumulates into O.
      if (j > 0) {
        ok = __all_sync(0xffffffffu, mbar_wait(pv_done, (j - 1) & 1, abort_flag));
        if (!ok) break;
        tc_fence_after();
      }
      if (__any_sync(0xffffffffu, need) && j > 0) {
        const float factor = ex2_approx(m_used - m_tgt);  // 1 where not needed
        l *= factor;
#pragma unroll 1
        for (int c = 0; c < D / 32; c++) {
          uint32_t o[32];
          tmem_ld32(tmem + lane_off + C::O_COL + c * 32, o);
          tmem_wait_ld();
          reg_fence32(o);
#pragma unroll
          for (int i = 0; i < 32; i++) o[i] = __float_as_uint(__uint_as_float(o[i]) * factor);
          tmem_st32(tmem + lane_off + C::O_COL + c * 32, o);
        }
      }
      m_used = m_tgt;
      // P_j in chunks of 32 keys: g(P) over S_j's own columns (already read;
      // S_{j+2} comes after PV_j), r(P) into the r(P) columns.
#pragma unroll
      for (int c = 0; c < 4; c++) {
        uint32_t pg[32], pr[32];
#pragma unroll
        for (int i = 0; i < 32; i++) {
          const float pv = ex2_approx(__uint_as_float(sv[c * 32 + i]) - m_tgt);
          const float g = tf32_big(pv);
          l += pv;
          pg[i] = __float_as_uint(g);
          pr[i] = __float_as_uint(pv - g);
        }
        tmem_st32(tS + c * 32, pg);
        tmem_st32(tmem + lane_off + C::PL_COL + c * 32, pr);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(pv_done, (nblk - 1) & 1, abort_flag));
    if (ok) {
      tc_fence_after();
      const int qr = q0 + row;
      float *dst = p.o + (long long)b * p.o_batch_stride + (long long)qr * p.o_row_stride +
                   (long long)h * p.o_head_stride;
      const float inv = 1.0f / l;
#pragma unroll
      for (int c = 0; c < D / 32; c++) {
        uint32_t o[32];
        tmem_ld32(tmem + lane_off + C::O_COL + c * 32, o);
        tmem_wait_ld();
        reg_fence32(o);
        if (qr < p.S) {
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            *reinterpret_cast<float4 *>(dst + c * 32 + i) =
                make_float4(__uint_as_float(o[i]) * inv, __uint_as_float(o[i + 1]) * inv,
                            __uint_as_float(o[i + 2]) * inv, __uint_as_float(o[i + 3]) * inv);
        }
      }
      if (p.lse != nullptr && qr < p.S)
        p.lse[(long long)bh * p.S + qr] = (m_used + log2f(l)) * 0.69314718055994531f;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicExch(err, 1);
}

}  // namespace llmr
