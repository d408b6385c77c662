// Non-causal attention for wide heads (D = 384 or 512) on the tcgen05 tensor
// cores: the VAE mid-block attention (lib/shaders/diffusion.slang:1828-1975
// vae_attention, dispatched with one head of D = 512 by
// dependencies/zimage.c3l/flux_vae.c3:493-538 and of D = 384 by
// dependencies/qwen_edit.c3l/qwen_vae.c3:430-464).
//
// fp16 operands, fp32 scores / softmax state / O accumulation, the same
// rounding points as the D <= 128 kernel (fa_tc.cuh).
//
// TMEM has 512 fp32 columns per SM; a 128-row O of D = 512 alone would fill
// it. A work unit therefore produces one half of the output columns
// (DV = D/2) of 128 query rows: it computes the whole S = Q K^T (reduction
// over all D) and the softmax, then O_half = P V[:, half]. The two halves of
// a query tile are separate units; both compute bit-identical S and P, so
// they use the same row max and row sum. QK^T is thereby done twice: the MMA
// work is 1.5x the algorithmic FLOPs.
//
// Two kernels: fa_wide_pair_kernel (further down; the default) runs the units
// on 2-CTA clusters with cta_group::2 MMAs, so that each CTA loads half of
// every shared operand; fa_wide_tc_kernel (here; LLMR_WIDE_SINGLE_CTA) is
// the single-CTA form of the same schedule:
//
// CTA = 128 query rows x one output half; 192 threads:
//   warps 0-3  softmax (thread i owns query row i = TMEM lane i)
//   warp  4    TMA producer: Q once per unit (resident, D/64 chunks), then
//              the K and V chunks (128 keys x 64 columns, 16 KB each) through
//              an NST-slot ring, in the order the MMA warp consumes them
//   warp  5    MMA issuer (one elected lane) + TMEM owner
// TMEM: S0 [0,128), S1 [128,256), O [256, 256+DV). P_j (fp16x2) overwrites
// the first 64 columns of S_{j%2} after the softmax has read it.
// MMA order per unit: S_0, S_1, PV_0, S_2, PV_1, S_3, ..., PV_{n-1}; the
// softmax of block j overlaps PV_{j-1} and S_{j+1}.
#pragma once

#include "fa_tc.cuh"

namespace llmr {

template <int D>
struct FaWideCfg {
  static_assert(D == 384 || D == 512, "wide attention kernel: D = 384 or 512");
  static constexpr int BM = 128;                 // query rows per unit
  static constexpr int BN = 128;                 // keys per block
  static constexpr int DV = D / 2;               // output columns per unit
  static constexpr int CHUNK_BYTES = 128 * 128;  // 64 columns x 128 rows, SW128
  static constexpr int QCH = D / 64;             // Q / K chunks per block
  static constexpr int VCH = DV / 64;            // V chunks per block and unit
  static constexpr int Q_BYTES = QCH * CHUNK_BYTES;
  static constexpr int NST = D == 512 ? 6 : 8;   // K/V ring slots (one chunk each)
  static constexpr int Q_OFF = 0;
  static constexpr int KV_OFF = Q_BYTES;
  static constexpr int BAR_OFF = KV_OFF + NST * CHUNK_BYTES;
  // barriers: q_full, q_empty, kv_full[NST], kv_empty[NST], s_full[2],
  // p_half[2][2], pv_done, o_full, o_empty, drain; then tmem base word and
  // abort flag
  static constexpr int NBAR = 2 + 2 * NST + 2 + 4 + 4;
  static constexpr int SMEM_BYTES = BAR_OFF + NBAR * 8 + 16 + 1024;  // +align slack
  static_assert(SMEM_BYTES <= 232448, "shared memory above the sm_100 per-block limit");
  static_assert(VCH <= NST, "a block's V chunks must fit in the ring together");
  static constexpr int THREADS = 192;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t O_COL = 256;
  static_assert(O_COL + DV <= TMEM_COLS, "O does not fit next to the S buffers");
};

// Units: (b, h, output half, 128-query tile), query tile fastest, so CTAs
// running together share one (b, h, half)'s K and V chunks in L2.
template <int D>
inline dim3 fa_wide_grid(FaParams &p, int B, int num_sms) {
  using C = FaWideCfg<D>;
  p.nqt = (p.S + C::BM - 1) / C::BM;
  p.nseq = 0;
  p.units = B * p.H * 2 * p.nqt;
  const int sms = num_sms > 0 ? num_sms : 148;
  return dim3(p.units < sms ? p.units : sms);
}

template <int D, typename OutT>
__global__ void __launch_bounds__(192, 1)
    fa_wide_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                      const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV,
                      const FaParams p) {
  using C = FaWideCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t *smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);

  uint8_t *sQ = smem + C::Q_OFF;
  uint8_t *sKV = smem + C::KV_OFF;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
  uint64_t *q_full = bars;
  uint64_t *q_empty = bars + 1;
  uint64_t *kv_full = bars + 2;
  uint64_t *kv_empty = kv_full + C::NST;
  // Every barrier below completes at most one phase ahead of the wait that
  // observes it. The softmax can run one key block ahead of the MMA warp
  // (S_{j+1} is issued before PV_j), so the S and P barriers are per S
  // buffer: buffer b's next phase needs S_{j+2}, which is issued after PV_j.
  uint64_t *s_full = kv_empty + C::NST;  // [jj % 2]
  uint64_t *p_half = s_full + 2;         // [(jj % 2) * 2 + half of the keys]
  uint64_t *pv_done = p_half + 4;
  uint64_t *o_full = pv_done + 1;
  uint64_t *o_empty = o_full + 1;
  uint64_t *drain = o_empty + 1;
  uint32_t *tmem_base_slot = reinterpret_cast<uint32_t *>(drain + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_base_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  struct Unit {
    int b, h, half, q0, nblk;
  };
  auto decode = [&](int unit) {
    Unit u;
    const int per_bh = 2 * p.nqt;
    const int bh = unit / per_bh;
    const int r = unit - bh * per_bh;
    u.half = r / p.nqt;
    u.q0 = (r - u.half * p.nqt) * C::BM;
    u.b = bh / p.H;
    u.h = bh - u.b * p.H;
    u.nblk = (p.S_kv + C::BN - 1) / C::BN;
    return u;
  };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < C::NST; i++) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_half[2 * b], 4);  // one arrival per softmax warp
      mbar_init(&p_half[2 * b + 1], 4);
    }
    mbar_init(pv_done, 1);
    mbar_init(o_full, 1);
    mbar_init(o_empty, 4);
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
    // Chunk order per unit (= the MMA warp's order): K_0, K_1, V_0, K_2,
    // V_1, ..., K_{n-1}, V_{n-2}, V_{n-1}; K_j is QCH chunks of all D
    // columns, V_j the VCH chunks of this unit's output half.
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      bool ok = true;
      int pos = 0;  // chunks armed so far (over all units): the ring position
      int kq = 0;   // Q loads armed so far
      auto load_chunk = [&](const CUtensorMap *m, int col, int key0, int h, int b) {
        const int slot = pos % C::NST, round = pos / C::NST;
        if (round > 0 && !mbar_wait(&kv_empty[slot], (round - 1) & 1, abort_flag)) return false;
        mbar_arrive_expect_tx(&kv_full[slot], C::CHUNK_BYTES);
        tma_load_4d(sKV + slot * C::CHUNK_BYTES, m, &kv_full[slot], col, key0, h, b);
        pos++;
        return true;
      };
      for (int unit = blockIdx.x, k = 0; unit < p.units && ok; unit += gridDim.x, k++) {
        const Unit un = decode(unit);
        // Q of this unit may replace the previous unit's once its last S
        // MMAs have completed.
        if (k > 0 && !mbar_wait(q_empty, (k - 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(q_full, C::Q_BYTES);
        for (int c = 0; c < C::QCH; c++)
          tma_load_4d(sQ + c * C::CHUNK_BYTES, &tmQ, q_full, c * 64, un.q0, un.h, un.b);
        kq = k + 1;
        for (int i = 0; i <= un.nblk && ok; i++) {
          if (i < un.nblk)
            for (int c = 0; c < C::QCH && ok; c++)
              ok = load_chunk(&tmK, c * 64, i * C::BN, un.h, un.b);
          if (i >= 1)
            for (int c = 0; c < C::VCH && ok; c++)
              ok = load_chunk(&tmV, (un.half * C::VCH + c) * 64, (i - 1) * C::BN, un.h, un.b);
        }
      }
      if (!ok) {
        // Abort path: let every armed copy land before the CTA exits.
        if (kq > 0) mbar_wait_raw(q_full, (kq - 1) & 1, 100000000ull);
        for (int u = pos - C::NST < 0 ? 0 : pos - C::NST; u < pos; u++)
          mbar_wait_raw(&kv_full[u % C::NST], (u / C::NST) & 1, 100000000ull);
      }
    }
  } else if (warp == 5) {
    // ---------------------------------------------------------- MMA issuer
    // The whole warp runs the loop (descriptors stay warp-uniform); one
    // elected lane issues each MMA and commit.
    constexpr uint32_t IDESC_S = idesc_f16_f32(128, C::BN, 0);
    constexpr uint32_t IDESC_O = idesc_f16_f32(128, 64, 1);
    const uint32_t sQa = smem_u32(sQ), sKVa = smem_u32(sKV);
    int pos = 0;  // ring position, mirrors the producer's
    // S_jj = Q K_jj^T into buffer jj % 2, one K chunk (64 of the D columns,
    // four K=16 steps) at a time; each chunk's slot is released when its
    // MMAs complete.
    auto issue_s = [&](int jj) {
      const uint32_t dS = tmem + (uint32_t)(jj & 1) * 128;
      for (int c = 0; c < C::QCH; c++) {
        const int slot = pos % C::NST;
        if (!mbar_wait(&kv_full[slot], (pos / C::NST) & 1, abort_flag)) return false;
        tc_fence_after();
        const uint32_t qa = sQa + c * C::CHUNK_BYTES;
        const uint32_t ka = sKVa + slot * C::CHUNK_BYTES;
#pragma unroll
        for (int kk = 0; kk < 4; kk++)
          if (elect_one())
            mma_ss(dS, sdesc_sw128(qa + kk * 32, 16, 1024), sdesc_sw128(ka + kk * 32, 16, 1024),
                   IDESC_S, (c > 0 || kk > 0) ? 1u : 0u);
        if (elect_one()) mma_commit(&kv_empty[slot]);
        pos++;
      }
      if (elect_one()) mma_commit(&s_full[jj & 1]);
      return true;
    };
    // O (+)= P_jj V_jj: per half of the block's keys (as soon as the
    // softmax has written that half of P), per 64-column V chunk one N=64
    // MMA for each of the four K=16 key steps.
    auto issue_pv = [&](int jj, bool acc) {
      const int base = pos;
      for (int c = 0; c < C::VCH; c++) {
        const int u = base + c;
        if (!mbar_wait(&kv_full[u % C::NST], (u / C::NST) & 1, abort_flag)) return false;
      }
      const uint32_t aP = tmem + (uint32_t)(jj & 1) * 128;
      for (int half = 0; half < 2; half++) {
        if (!mbar_wait(&p_half[2 * (jj & 1) + half], (jj >> 1) & 1, abort_flag)) return false;
        tc_fence_after();
        for (int c = 0; c < C::VCH; c++) {
          const uint32_t va = sKVa + ((base + c) % C::NST) * C::CHUNK_BYTES;
#pragma unroll
          for (int kk = 0; kk < 4; kk++) {
            const int ks = half * 4 + kk;
            if (elect_one())
              mma_ts(tmem + C::O_COL + c * 64, aP + ks * 8,
                     sdesc_sw128(va + ks * 2048, C::CHUNK_BYTES, 1024), IDESC_O,
                     (acc || ks > 0) ? 1u : 0u);
          }
        }
      }
      for (int c = 0; c < C::VCH; c++)
        if (elect_one()) mma_commit(&kv_empty[(base + c) % C::NST]);
      pos += C::VCH;
      return true;
    };
    bool ok = true;
    int jb = 0;  // key blocks of this CTA's earlier units
    for (int unit = blockIdx.x, k = 0; unit < p.units && ok; unit += gridDim.x, k++) {
      const int nblk = decode(unit).nblk;
      if (!(ok = mbar_wait(q_full, k & 1, abort_flag))) break;
      tc_fence_after();
      // S of this unit's first blocks overwrites P of the previous unit's
      // last blocks: the PV MMAs that read it were issued earlier and run
      // first.
      if (!(ok = issue_s(jb))) break;
      if (nblk > 1 && !(ok = issue_s(jb + 1))) break;
      if (nblk <= 2 && elect_one()) mma_commit(q_empty);
      for (int j = 0; j < nblk; j++) {
        const int jj = jb + j;
        // O is overwritten by this unit's first PV: the previous unit's
        // epilogue must have read it.
        if (j == 0 && k > 0 && !(ok = mbar_wait(o_empty, (k - 1) & 1, abort_flag))) break;
        if (!(ok = issue_pv(jj, j > 0))) break;
        if (elect_one()) mma_commit(pv_done);
        if (j + 2 < nblk) {
          if (!(ok = issue_s(jj + 2))) break;
          // The unit's last S MMAs are issued: Q may be replaced after them.
          if (j + 3 == nblk && elect_one()) mma_commit(q_empty);
        }
      }
      if (!ok) break;
      if (elect_one()) mma_commit(o_full);
      jb += nblk;
    }
    // Drain: every MMA this warp issued has completed before TMEM is
    // released at the end of the kernel.
    if (elect_one()) mma_commit(drain);
    mbar_wait_raw(drain, 0, 100000000ull);
  } else {
    // ------------------------------------------------------------- softmax
    const int row = threadIdx.x;  // 0..127 = TMEM lane
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const uint32_t tO = tmem + lane_off + C::O_COL;
    const float sl2 = p.scale_log2;
    bool ok = true;
    int jb = 0;
    for (int unit = blockIdx.x, k = 0; unit < p.units && ok; unit += gridDim.x, k++) {
      const Unit un = decode(unit);
      const int nblk = un.nblk;
      float m_used = -INFINITY;  // log2-domain max the P values are relative to
      float l = 0.0f;
      for (int j = 0; j < nblk; j++) {
        const int jj = jb + j;
        const uint32_t tS = tmem + lane_off + (uint32_t)(jj & 1) * 128;
        ok = __all_sync(0xffffffffu, mbar_wait(&s_full[jj & 1], (jj >> 1) & 1, abort_flag));
        if (!ok) break;
        tc_fence_after();
        const int valid = p.S_kv - j * C::BN;  // keys of this block inside the sequence
        uint32_t sbuf[128];
#pragma unroll
        for (int c = 0; c < 4; c++) tmem_ld32(tS + c * 32, sbuf + c * 32);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 4; c++) reg_fence32(sbuf + c * 32);
        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int c = 0; c < 4; c++) {
          float *v = reinterpret_cast<float *>(sbuf + c * 32);
          if (valid < C::BN) {
#pragma unroll
            for (int i = 0; i < 32; i++)
              if (c * 32 + i >= valid) v[i] = -INFINITY;
          }
#pragma unroll
          for (int i = 0; i < 32; i += 2) mx[(i >> 1) & 3] = max3f(mx[(i >> 1) & 3], v[i], v[i + 1]);
        }
        // Lazy max, as in the D <= 128 kernel: P is relative to m_used, which
        // moves only on the first block or when the block's row max passes
        // it by more than kMaxExp; O and l are rescaled then.
        const float m_new = max3f(mx[0], mx[1], fmaxf(mx[2], mx[3])) * sl2;
        const bool need = m_new > m_used + kMaxExp;  // always true on block 0
        // PV of the previous block has completed (observed at every block so
        // that each pv_done phase is seen in turn; it is also what lets the
        // rescale below touch O). PV_{jj-1} is issued right after P_{jj-1},
        // well before the MMA warp needs P_jj.
        if (jj > 0) {
          ok = __all_sync(0xffffffffu, mbar_wait(pv_done, (jj - 1) & 1, abort_flag));
          if (!ok) break;
        }
        if (__any_sync(0xffffffffu, need)) {
          const float m_tgt = need ? m_new : m_used;
          const float factor = ex2_approx(m_used - m_tgt);  // 0 on the first block
          l *= factor;
          if (j > 0) {
            tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < C::DV / 32; c++) {
              uint32_t o[32];
              tmem_ld32(tO + c * 32, o);
              tmem_wait_ld();
              reg_fence32(o);
#pragma unroll
              for (int i = 0; i < 32; i++) o[i] = __float_as_uint(__uint_as_float(o[i]) * factor);
              tmem_st32(tO + c * 32, o);
            }
          }
          m_used = m_tgt;
        }
        // P = 2^(s*scale*log2e - m_used) as fp16 into the buffer's first 64
        // columns; each half (keys 0-63, then 64-127) is handed to the MMA
        // warp as soon as it is in TMEM (the wait also covers the O stores).
        uint64_t part2[2] = {f2_pack(0.0f, 0.0f), f2_pack(0.0f, 0.0f)};
        const uint64_t sl2x2 = f2_pack(sl2, sl2);
        const uint64_t neg_mx2 = f2_pack(-m_used, -m_used);
#pragma unroll
        for (int c = 0; c < 4; c++) {
          const float *v = reinterpret_cast<const float *>(sbuf + c * 32);
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; i++) {
            const float2 x = f2_unpack(f2_fma(f2_pack(v[2 * i], v[2 * i + 1]), sl2x2, neg_mx2));
            uint64_t pp;
            if ((kExp2EmuMask >> i) & 1u)
              pp = exp2_poly_x2(f2_pack(fmaxf(x.x, -125.0f), fmaxf(x.y, -125.0f)));
            else
              pp = f2_pack(ex2_approx(x.x), ex2_approx(x.y));
            part2[i & 1] = f2_add(part2[i & 1], pp);
            const float2 pf = f2_unpack(pp);
            pk[i] = pack_f16x2(pf.x, pf.y);
          }
          tmem_st16(tS + c * 16, pk);
          if (c == 1 || c == 3) {
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_half[2 * (jj & 1) + (c >> 1)]);
          }
        }
        const float2 s0 = f2_unpack(part2[0]), s1 = f2_unpack(part2[1]);
        l += (s0.x + s0.y) + (s1.x + s1.y);
      }
      jb += nblk;
      if (!ok) break;
      // ------------------------------------------------------- epilogue
      ok = __all_sync(0xffffffffu, mbar_wait(o_full, k & 1, abort_flag));
      if (!ok) break;
      tc_fence_after();
      const int q = un.q0 + row;
      const bool qin = q < p.S;
      OutT *dst = reinterpret_cast<OutT *>(p.o) + (long long)un.b * p.o_batch_stride +
                  (long long)q * p.o_row_stride + (long long)un.h * D + un.half * C::DV;
      const float inv_l = 1.0f / l;
#pragma unroll 1
      for (int c = 0; c < C::DV / 32; c++) {
        uint32_t o[32];
        tmem_ld32(tO + c * 32, o);
        tmem_wait_ld();
        reg_fence32(o);
        if (c == C::DV / 32 - 1) {
          // O is read out: the next unit's first PV may overwrite it.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(o_empty);
        }
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; i++) v[i] = __uint_as_float(o[i]) * inv_l;
        if (qin) store_row_chunk<OutT>(dst + c * 32, v);
      }
      // Both halves hold the same m_used and l; the first writes the LSE.
      if (p.lse != nullptr && qin && un.half == 0)
        p.lse[((long long)un.b * p.H + un.h) * p.S + q] =
            (m_used + log2f(l)) * 0.69314718055994531f;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicExch(p.err, 1);
}

// ---------------------------------------------------------------------------
// The same attention on CTA pairs (2-CTA clusters, tcgen05 cta_group::2). The
// single-CTA kernel above keeps Q resident (128 KB at D = 512), which leaves
// a 96 KB K/V ring against ~190 KB of K and V per key block: it runs out of
// loads in flight (tensor pipe ~30 % busy at ~14 % of L2 throughput). Here a
// pair computes 256 query rows (each CTA holds its own 128 rows of Q) with
// M = 256 MMAs, so each CTA loads only half of every operand it shares:
//   S = Q K^T : N = 128 keys, each CTA loads 64 of them (8 KB per K chunk);
//   O = P V   : N = the output part's columns, each CTA loads half of them.
// Output parts: columns [256p, min(256p + 256, D)), p = 0, 1 (D = 512:
// 256 + 256; D = 384: 256 + 128); a unit is (b, h, part, 256-query tile).
// The even CTA issues every MMA and owns the barriers that count both CTAs'
// TMA bytes (q_full, k_full, v_full) or both CTAs' softmax warps (p_half,
// o_empty); every MMA commit is delivered to the matching barrier of both
// CTAs (no multicast). Roles, TMEM use and the barrier protocol otherwise
// follow fa_wide_tc_kernel.
template <int D>
struct FaWide2Cfg {
  static_assert(D == 384 || D == 512, "wide attention pair kernel: D = 384 or 512");
  static constexpr int BM = 128;                 // query rows per CTA
  static constexpr int BN = 128;                 // keys per block (per pair)
  static constexpr int ATOM = 128 * 128;         // 64 columns x 128 rows, SW128
  static constexpr int QCH = D / 64;             // Q / K column chunks
  static constexpr int Q_BYTES = QCH * ATOM;
  static constexpr int K_BYTES = 64 * 128;       // 64 keys x 64 columns (this CTA's half)
  static constexpr int V_SLOT = 2 * ATOM;        // up to 128 of a part's columns
  static constexpr int NSTK = 8;                 // K ring slots
  static constexpr int NSTV = D == 512 ? 1 : 2;  // V ring slots
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_BYTES;
  static constexpr int V_OFF = K_OFF + NSTK * K_BYTES;
  static constexpr int BAR_OFF = V_OFF + NSTV * V_SLOT;
  // q_full, q_empty, k_full[NSTK], k_empty[NSTK], v_full[NSTV], v_empty[NSTV],
  // s_full[2], p_half[2][2], pv_done, o_full, o_empty, drain; tmem word; abort
  static constexpr int NBAR = 2 + 2 * NSTK + 2 * NSTV + 2 + 4 + 4;
  static constexpr int SMEM_BYTES = BAR_OFF + NBAR * 8 + 16 + 1024;
  static_assert(SMEM_BYTES <= 232448, "shared memory above the sm_100 per-block limit");
  static constexpr int THREADS = 192;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t O_COL = 256;
  // Columns of output part `part`.
  __host__ __device__ static constexpr int part_cols(int part) {
    return D - 256 * part < 256 ? D - 256 * part : 256;
  }
};

// Units: (b, h, part, 256-query tile), tile fastest; one pair per unit.
template <int D>
inline dim3 fa_wide_pair_grid(FaParams &p, int B, int num_sms) {
  p.nqt = (p.S + 255) / 256;
  p.nseq = 0;
  p.units = B * p.H * 2 * p.nqt;
  const int pairs_max = (num_sms > 0 ? num_sms : 148) / 2;
  return dim3(2 * (p.units < pairs_max ? p.units : pairs_max));
}

template <int D, typename OutT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(192, 1)
    fa_wide_pair_kernel(const __grid_constant__ CUtensorMap tmQ,
                        const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const FaParams p) {
  using C = FaWide2Cfg<D>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t *smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);

  uint8_t *sQ = smem + C::Q_OFF;
  uint8_t *sK = smem + C::K_OFF;
  uint8_t *sV = smem + C::V_OFF;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
  uint64_t *q_full = bars;
  uint64_t *q_empty = bars + 1;
  uint64_t *k_full = bars + 2;
  uint64_t *k_empty = k_full + C::NSTK;
  uint64_t *v_full = k_empty + C::NSTK;
  uint64_t *v_empty = v_full + C::NSTV;
  uint64_t *s_full = v_empty + C::NSTV;  // [jj % 2]
  uint64_t *p_half = s_full + 2;         // [(jj % 2) * 2 + half of the keys]
  uint64_t *pv_done = p_half + 4;
  uint64_t *o_full = pv_done + 1;
  uint64_t *o_empty = o_full + 1;
  uint64_t *drain = o_empty + 1;
  uint32_t *tmem_base_slot = reinterpret_cast<uint32_t *>(drain + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_base_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0 = the pair's MMA issuer
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  struct Unit {
    int b, h, part, col0, ncols, q0, nblk;
  };
  auto decode = [&](int unit) {
    Unit u;
    const int per_bh = 2 * p.nqt;
    const int bh = unit / per_bh;
    const int r = unit - bh * per_bh;
    u.part = r / p.nqt;
    u.q0 = (r - u.part * p.nqt) * 2 * C::BM;
    u.b = bh / p.H;
    u.h = bh - u.b * p.H;
    u.col0 = 256 * u.part;
    u.ncols = C::part_cols(u.part);
    u.nblk = (p.S_kv + C::BN - 1) / C::BN;
    return u;
  };
  // Cluster address of barrier `bar` in CTA `r` (0 = the even CTA).
  auto at = [&](uint64_t *bar, uint32_t r) { return mapa_shared(smem_u32(bar), r); };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < C::NSTK; i++) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < C::NSTV; i++) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_half[2 * b], 8);  // four softmax warps of each CTA
      mbar_init(&p_half[2 * b + 1], 8);
    }
    mbar_init(pv_done, 1);
    mbar_init(o_full, 1);
    mbar_init(o_empty, 8);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc_pair(tmem_base_slot, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_slot;

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    // Order per unit (= the MMA warp's): K_0, K_1, V_0, K_2, V_1, ...,
    // K_{n-1}, V_{n-2}, V_{n-1}. Each CTA loads its own Q rows, its 64 keys
    // of every K chunk and its half of the part's V columns; the bytes of
    // both CTAs complete on the even CTA's barriers, which the even CTA arms.
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      bool ok = true;
      int kpos = 0, vpos = 0, kq = 0;
      for (int unit = pair, k = 0; unit < p.units && ok; unit += npairs, k++) {
        const Unit un = decode(unit);
        if (k > 0 && !mbar_wait(q_empty, (k - 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
        if (rank == 0) mbar_arrive_expect_tx(q_full, 2 * C::Q_BYTES);
        for (int c = 0; c < C::QCH; c++)
          tma_load_4d_pair(sQ + c * C::ATOM, &tmQ, at(q_full, 0), c * 64,
                           un.q0 + (int)rank * C::BM, un.h, un.b);
        kq = k + 1;
        const int vcols = un.ncols / 2;  // this CTA's V columns
        for (int i = 0; i <= un.nblk && ok; i++) {
          if (i < un.nblk) {
            for (int c = 0; c < C::QCH; c++) {
              const int slot = kpos % C::NSTK, round = kpos / C::NSTK;
              if (round > 0 && !mbar_wait(&k_empty[slot], (round - 1) & 1, abort_flag)) {
                ok = false;
                break;
              }
              if (rank == 0) mbar_arrive_expect_tx(&k_full[slot], 2 * C::K_BYTES);
              tma_load_4d_pair(sK + slot * C::K_BYTES, &tmK, at(&k_full[slot], 0), c * 64,
                               i * C::BN + (int)rank * (C::BN / 2), un.h, un.b);
              kpos++;
            }
          }
          if (i >= 1 && ok) {
            const int slot = vpos % C::NSTV, round = vpos / C::NSTV;
            if (round > 0 && !mbar_wait(&v_empty[slot], (round - 1) & 1, abort_flag)) {
              ok = false;
              break;
            }
            if (rank == 0) mbar_arrive_expect_tx(&v_full[slot], 2 * vcols * C::BN * 2);
            for (int a = 0; a < vcols / 64; a++)
              tma_load_4d_pair(sV + slot * C::V_SLOT + a * C::ATOM, &tmV, at(&v_full[slot], 0),
                               un.col0 + (int)rank * vcols + a * 64, (i - 1) * C::BN, un.h,
                               un.b);
            vpos++;
          }
        }
      }
      if (!ok && rank == 0) {
        // Abort path: every armed load (both CTAs' bytes) lands before exit.
        if (kq > 0) mbar_wait_raw(q_full, (kq - 1) & 1, 100000000ull);
        for (int u = kpos - C::NSTK < 0 ? 0 : kpos - C::NSTK; u < kpos; u++)
          mbar_wait_raw(&k_full[u % C::NSTK], (u / C::NSTK) & 1, 100000000ull);
        for (int u = vpos - C::NSTV < 0 ? 0 : vpos - C::NSTV; u < vpos; u++)
          mbar_wait_raw(&v_full[u % C::NSTV], (u / C::NSTV) & 1, 100000000ull);
      }
    }
  } else if (warp == 5) {
    // ---------------------------------------------------------- MMA issuer
    if (rank == 0) {
      constexpr uint32_t IDESC_S = idesc_f16_f32(2 * C::BM, C::BN, 0);
      const uint32_t sQa = smem_u32(sQ), sKa = smem_u32(sK), sVa = smem_u32(sV);
      int kpos = 0, vpos = 0;
      auto commit_both = [&](uint64_t *bar) {
        if (elect_one()) {
          mma_commit_pair(at(bar, 0));
          mma_commit_pair(at(bar, 1));
        }
      };
      auto issue_s = [&](int jj) {
        const uint32_t dS = tmem + (uint32_t)(jj & 1) * 128;
        for (int c = 0; c < C::QCH; c++) {
          const int slot = kpos % C::NSTK;
          if (!mbar_wait(&k_full[slot], (kpos / C::NSTK) & 1, abort_flag)) return false;
          tc_fence_after();
          const uint32_t qa = sQa + c * C::ATOM;
          const uint32_t ka = sKa + slot * C::K_BYTES;
#pragma unroll
          for (int kk = 0; kk < 4; kk++)
            if (elect_one())
              mma_ss_pair(dS, sdesc_sw128(qa + kk * 32, 16, 1024),
                          sdesc_sw128(ka + kk * 32, 16, 1024), IDESC_S,
                          (c > 0 || kk > 0) ? 1u : 0u);
          commit_both(&k_empty[slot]);
          kpos++;
        }
        commit_both(&s_full[jj & 1]);
        return true;
      };
      // O (+)= P_jj V_jj over the part's columns: one N = ncols MMA per K=16
      // key step (each CTA supplies ncols/2 columns as 64-column atoms).
      auto issue_pv = [&](int jj, bool acc, uint32_t idesc_o) {
        const int slot = vpos % C::NSTV;
        if (!mbar_wait(&v_full[slot], (vpos / C::NSTV) & 1, abort_flag)) return false;
        const uint32_t aP = tmem + (uint32_t)(jj & 1) * 128;
        const uint32_t va = sVa + slot * C::V_SLOT;
        for (int half = 0; half < 2; half++) {
          if (!mbar_wait_cluster(&p_half[2 * (jj & 1) + half], (jj >> 1) & 1, abort_flag))
            return false;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 4; kk++) {
            const int ks = half * 4 + kk;
            if (elect_one())
              mma_ts_pair(tmem + C::O_COL, aP + ks * 8, sdesc_sw128(va + ks * 2048, C::ATOM, 1024),
                          idesc_o, (acc || ks > 0) ? 1u : 0u);
          }
        }
        commit_both(&v_empty[slot]);
        vpos++;
        return true;
      };
      bool ok = true;
      int jb = 0;
      for (int unit = pair, k = 0; unit < p.units && ok; unit += npairs, k++) {
        const Unit un = decode(unit);
        const int nblk = un.nblk;
        const uint32_t idesc_o = idesc_f16_f32(2 * C::BM, (uint32_t)un.ncols, 1);
        if (!(ok = mbar_wait(q_full, k & 1, abort_flag))) break;
        tc_fence_after();
        if (!(ok = issue_s(jb))) break;
        if (nblk > 1 && !(ok = issue_s(jb + 1))) break;
        if (nblk <= 2) commit_both(q_empty);
        for (int j = 0; j < nblk; j++) {
          const int jj = jb + j;
          if (j == 0 && k > 0 && !(ok = mbar_wait_cluster(o_empty, (k - 1) & 1, abort_flag)))
            break;
          if (!(ok = issue_pv(jj, j > 0, idesc_o))) break;
          commit_both(pv_done);
          if (j + 2 < nblk) {
            if (!(ok = issue_s(jj + 2))) break;
            if (j + 3 == nblk) commit_both(q_empty);
          }
        }
        if (!ok) break;
        commit_both(o_full);
        jb += nblk;
      }
      if (elect_one()) mma_commit_pair(smem_u32(drain));
      mbar_wait_raw(drain, 0, 100000000ull);
    }
  } else {
    // ------------------------------------------------------------- softmax
    const int row = threadIdx.x;  // 0..127 = TMEM lane
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const uint32_t tO = tmem + lane_off + C::O_COL;
    const float sl2 = p.scale_log2;
    bool ok = true;
    int jb = 0;
    for (int unit = pair, k = 0; unit < p.units && ok; unit += npairs, k++) {
      const Unit un = decode(unit);
      const int nblk = un.nblk;
      float m_used = -INFINITY;
      float l = 0.0f;
      for (int j = 0; j < nblk; j++) {
        const int jj = jb + j;
        const uint32_t tS = tmem + lane_off + (uint32_t)(jj & 1) * 128;
        ok = __all_sync(0xffffffffu, mbar_wait(&s_full[jj & 1], (jj >> 1) & 1, abort_flag));
        if (!ok) break;
        tc_fence_after();
        const int valid = p.S_kv - j * C::BN;
        uint32_t sbuf[128];
#pragma unroll
        for (int c = 0; c < 4; c++) tmem_ld32(tS + c * 32, sbuf + c * 32);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 4; c++) reg_fence32(sbuf + c * 32);
        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int c = 0; c < 4; c++) {
          float *v = reinterpret_cast<float *>(sbuf + c * 32);
          if (valid < C::BN) {
#pragma unroll
            for (int i = 0; i < 32; i++)
              if (c * 32 + i >= valid) v[i] = -INFINITY;
          }
#pragma unroll
          for (int i = 0; i < 32; i += 2) mx[(i >> 1) & 3] = max3f(mx[(i >> 1) & 3], v[i], v[i + 1]);
        }
        const float m_new = max3f(mx[0], mx[1], fmaxf(mx[2], mx[3])) * sl2;
        const bool need = m_new > m_used + kMaxExp;
        if (jj > 0) {
          ok = __all_sync(0xffffffffu, mbar_wait(pv_done, (jj - 1) & 1, abort_flag));
          if (!ok) break;
        }
        if (__any_sync(0xffffffffu, need)) {
          const float m_tgt = need ? m_new : m_used;
          const float factor = ex2_approx(m_used - m_tgt);
          l *= factor;
          if (j > 0) {
            tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < un.ncols / 32; c++) {
              uint32_t o[32];
              tmem_ld32(tO + c * 32, o);
              tmem_wait_ld();
              reg_fence32(o);
#pragma unroll
              for (int i = 0; i < 32; i++) o[i] = __float_as_uint(__uint_as_float(o[i]) * factor);
              tmem_st32(tO + c * 32, o);
            }
          }
          m_used = m_tgt;
        }
        uint64_t part2[2] = {f2_pack(0.0f, 0.0f), f2_pack(0.0f, 0.0f)};
        const uint64_t sl2x2 = f2_pack(sl2, sl2);
        const uint64_t neg_mx2 = f2_pack(-m_used, -m_used);
#pragma unroll
        for (int c = 0; c < 4; c++) {
          const float *v = reinterpret_cast<const float *>(sbuf + c * 32);
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; i++) {
            const float2 x = f2_unpack(f2_fma(f2_pack(v[2 * i], v[2 * i + 1]), sl2x2, neg_mx2));
            uint64_t pp;
            if ((kExp2EmuMask >> i) & 1u)
              pp = exp2_poly_x2(f2_pack(fmaxf(x.x, -125.0f), fmaxf(x.y, -125.0f)));
            else
              pp = f2_pack(ex2_approx(x.x), ex2_approx(x.y));
            part2[i & 1] = f2_add(part2[i & 1], pp);
            const float2 pf = f2_unpack(pp);
            pk[i] = pack_f16x2(pf.x, pf.y);
          }
          tmem_st16(tS + c * 16, pk);
          if (c == 1 || c == 3) {
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(at(&p_half[2 * (jj & 1) + (c >> 1)], 0));
          }
        }
        const float2 s0 = f2_unpack(part2[0]), s1 = f2_unpack(part2[1]);
        l += (s0.x + s0.y) + (s1.x + s1.y);
      }
      jb += nblk;
      if (!ok) break;
      // ------------------------------------------------------- epilogue
      ok = __all_sync(0xffffffffu, mbar_wait(o_full, k & 1, abort_flag));
      if (!ok) break;
      tc_fence_after();
      const int q = un.q0 + (int)rank * C::BM + row;
      const bool qin = q < p.S;
      OutT *dst = reinterpret_cast<OutT *>(p.o) + (long long)un.b * p.o_batch_stride +
                  (long long)q * p.o_row_stride + (long long)un.h * D + un.col0;
      const float inv_l = 1.0f / l;
      const int nc = un.ncols / 32;
#pragma unroll 1
      for (int c = 0; c < nc; c++) {
        uint32_t o[32];
        tmem_ld32(tO + c * 32, o);
        tmem_wait_ld();
        reg_fence32(o);
        if (c == nc - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_remote(at(o_empty, 0));
        }
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; i++) v[i] = __uint_as_float(o[i]) * inv_l;
        if (qin) store_row_chunk<OutT>(dst + c * 32, v);
      }
      if (p.lse != nullptr && qin && un.part == 0)
        p.lse[((long long)un.b * p.H + un.h) * p.S + q] =
            (m_used + log2f(l)) * 0.69314718055994531f;
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no pair MMA, remote arrival or peer TMA write is left in flight
  if (warp == 5) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem, C::TMEM_COLS);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicExch(p.err, 1);
}

}  // namespace llmr
