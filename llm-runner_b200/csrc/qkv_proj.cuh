// QKV projection with the attention prologue in its epilogue, for sm_100a:
//
//   out[t][b][h][s][:] = epi_t( x[b, s, :] . W[t*H*D + h*D + d, :] )   d < D
//
// x [B*S, hidden] and W [3*H*D, hidden] (the reference's [out_dim, in_dim]
// row-major weight convention, dependencies/llm_text.c3l/shaders/
// llm.slang:1198-1232 batch_matmul_f16 and :2039-2105
// batch_matmul_f16_coopmat: fp16 operands, fp32 accumulation; rows
// Q = 0, K = dim, V = 2*dim via row_offset, dependencies/zimage.c3l/
// dit.c3:1437-1442) are both fp16 or both bf16. epi_t is, for Q and K, the
// per-head RMSNorm with the txt/img gain split (zimage.slang:623-659) and the
// interleaved RoPE rotation (mrope.slang:47-53), in fp32 with the same
// operation order as the standalone prologue; for V the identity. The
// result is written as fp16 in the dense [3][B][H][S][D] layout the
// attention kernel reads, so the attention call that follows needs no
// prologue.
//
// CTA (persistent, one per SM) = 192 threads:
//   warp 0     TMA producer: x (128 x 64) and W (BN x 64) tiles into a
//              4-stage ring of SW128 buffers
//   warp 1     TMEM owner and MMA issuer (tcgen05.mma M128 x BN x 16, fp32
//              accumulators, two BN-column buffers so one tile's epilogue
//              overlaps the next tile's main loop)
//   warps 2-5  epilogue: thread = accumulator row (TMEM lane); for each head
//              of the tile a first pass over its columns gives the RMS, a
//              second pass normalises, rotates, rounds to fp16 and stores 32
//              columns at a time (one contiguous 2*D-byte row per thread).
#pragma once
#include <cuda_fp16.h>

#include "ptx.cuh"

namespace llmr {

struct QkvParams {
  int M;                 // B * S token rows
  int S;                 // tokens per batch element
  int B, H;
  int k_blocks;          // hidden / 64
  int n_tiles;           // 3 * H * D / BN
  int tiles;             // ceil(M / 128) * n_tiles
  int split_row;         // global token index from which gain set 1 applies
  int rope_row_offset;   // global token index of token 0
  float eps;
  const float *q_gain, *k_gain;  // [D] or [2][D]; null = no norm
  const float *cos_t, *sin_t;    // [rows][D/2]; null = no RoPE
  __half *out;                   // [3][B][H][S][D]
  int *err;
};

template <int D, int BN>
struct QkvCfg {
  static constexpr int BM = 128, BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;  // 16 KB
  static constexpr int B_BYTES = BN * BK * 2;  // 16 or 32 KB
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int NST = BN == 256 ? 4 : 6;
  static constexpr int BAR_OFF = NST * STAGE_BYTES;
  // barriers: full[NST], empty[NST], acc_full[2], acc_empty[2], drain; then
  // the tmem base word and the abort flag
  static constexpr int NBAR = 2 * NST + 2 + 2 + 1;
  static constexpr int SMEM_BYTES = BAR_OFF + NBAR * 8 + 16 + 1024;
  static constexpr int THREADS = 192;
  static constexpr uint32_t TMEM_COLS = 2 * BN;
  static constexpr int HEADS_PER_TILE = BN / D;
};

// Epilogue of one accumulator tile for one thread (= accumulator row m):
// per head of the tile, the RMS over its columns (pass 1), then norm,
// rotation, fp16 and a contiguous row store, 32 columns at a time (pass 2).
// tacc: the thread's TMEM address of the tile's first column. release() is
// called once, right after the last TMEM load of the tile.
template <int D, int BN, typename Release>
__device__ __forceinline__ void qkv_tile_epilogue(const QkvParams &p, uint32_t tacc0, int m,
                                                  int n0, Release release) {
  constexpr int HEADS = BN / D;
  const long long plane = (long long)p.B * p.H * p.S * D;
  const int hd = p.H * D;
  const bool in = m < p.M;
  const int b = in ? m / p.S : 0;
  const int s = in ? m - b * p.S : 0;
  const long long grow = (long long)p.rope_row_offset + s;
  const int t = n0 / hd;  // 0 = Q, 1 = K, 2 = V (a tile never spans two)
  const float *gain = t == 0 ? p.q_gain : (t == 1 ? p.k_gain : nullptr);
  const bool rope = t < 2 && p.cos_t != nullptr;
#pragma unroll 1
  for (int hl = 0; hl < HEADS; hl++) {
    const int h = (n0 - t * hd) / D + hl;
    const uint32_t tacc = tacc0 + hl * D;
    // Pass 1 (Q/K with norm): the row's sum of squares, chunk by chunk.
    float rms = 1.0f;
    if (gain != nullptr) {
      float ss = 0.0f;
#pragma unroll 1
      for (int c = 0; c < D / 32; c++) {
        uint32_t r[32];
        tmem_ld32(tacc + c * 32, r);
        tmem_wait_ld();
        reg_fence32(r);
#pragma unroll
        for (int e = 0; e < 32; e++) ss = __fmaf_rn(__uint_as_float(r[e]), __uint_as_float(r[e]), ss);
      }
      rms = rsqrtf(ss / (float)D + p.eps);
    }
    const float *g = gain == nullptr ? nullptr
                                     : gain + ((p.split_row > 0 && grow >= p.split_row) ? D : 0);
    const float *ct = p.cos_t + grow * (D / 2);
    const float *stt = p.sin_t + grow * (D / 2);
    __half *dst = p.out + t * plane + (((long long)b * p.H + h) * p.S + s) * D;
    // Pass 2: 32 columns at a time: norm, rotation, fp16, store.
#pragma unroll 1
    for (int c = 0; c < D / 32; c++) {
      uint32_t r[32];
      tmem_ld32(tacc + c * 32, r);
      tmem_wait_ld();
      reg_fence32(r);
      if (hl == HEADS - 1 && c == D / 32 - 1) release();
      float y[32];
#pragma unroll
      for (int e = 0; e < 32; e++) y[e] = __uint_as_float(r[e]);
      if (g != nullptr) {
#pragma unroll
        for (int e = 0; e < 32; e += 4) {
          const float4 gv = *reinterpret_cast<const float4 *>(g + c * 32 + e);
          y[e] = __fmul_rn(__fmul_rn(y[e], rms), gv.x);
          y[e + 1] = __fmul_rn(__fmul_rn(y[e + 1], rms), gv.y);
          y[e + 2] = __fmul_rn(__fmul_rn(y[e + 2], rms), gv.z);
          y[e + 3] = __fmul_rn(__fmul_rn(y[e + 3], rms), gv.w);
        }
      }
      if (rope && in) {
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
          const float4 cv = *reinterpret_cast<const float4 *>(ct + (c * 32 + e) / 2);
          const float4 sv = *reinterpret_cast<const float4 *>(stt + (c * 32 + e) / 2);
          const float cc[4] = {cv.x, cv.y, cv.z, cv.w};
          const float sn[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
          for (int i = 0; i < 8; i += 2) {
            const float x0 = y[e + i], x1 = y[e + i + 1];
            y[e + i] = __fsub_rn(__fmul_rn(x0, cc[i / 2]), __fmul_rn(x1, sn[i / 2]));
            y[e + i + 1] = __fadd_rn(__fmul_rn(x0, sn[i / 2]), __fmul_rn(x1, cc[i / 2]));
          }
        }
      }
      if (in) {
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
          uint4 u;
          u.x = pack_f16x2(y[e], y[e + 1]);
          u.y = pack_f16x2(y[e + 2], y[e + 3]);
          u.z = pack_f16x2(y[e + 4], y[e + 5]);
          u.w = pack_f16x2(y[e + 6], y[e + 7]);
          *reinterpret_cast<uint4 *>(dst + c * 32 + e) = u;
        }
      }
    }
  }
}

template <int D, int BN, bool BF16>
__global__ void __launch_bounds__(192, 1)
    qkv_proj_kernel(const __grid_constant__ CUtensorMap tmX,
                    const __grid_constant__ CUtensorMap tmW, const QkvParams p) {
  using C = QkvCfg<D, BN>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t *smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
  uint64_t *full = bars;
  uint64_t *empty = full + C::NST;
  uint64_t *acc_full = empty + C::NST;
  uint64_t *acc_empty = acc_full + 2;
  uint64_t *drain = acc_empty + 2;
  uint32_t *tmem_base_slot = reinterpret_cast<uint32_t *>(drain + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_base_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m_tiles = (p.M + C::BM - 1) / C::BM;
  // Tile order: groups of kGroupM row blocks, each group walked m-fastest
  // over all column blocks, so the CTAs running together (about one per SM)
  // share a few x row blocks and W column blocks in L2 instead of streaming
  // all of x from DRAM once per column block.
  constexpr int kGroupM = 16;
  auto decode = [&](int tile, int &m0, int &n0) {
    const int per_group = kGroupM * p.n_tiles;
    const int grp = tile / per_group;
    const int first = grp * kGroupM;
    const int gm = m_tiles - first < kGroupM ? m_tiles - first : kGroupM;
    const int in = tile - grp * per_group;
    m0 = (first + in % gm) * C::BM;
    n0 = (in / gm) * BN;
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::NST; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);  // one arrival per epilogue warp
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_base_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmX);
      tma_prefetch_desc(&tmW);
      bool ok = true;
      int it = 0;  // stage loads armed so far (over all tiles)
      for (int tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x) {
        int m0, n0;
        decode(tile, m0, n0);
        for (int kb = 0; kb < p.k_blocks; kb++, it++) {
          const int st = it % C::NST, round = it / C::NST;
          if (round > 0 && !mbar_wait(&empty[st], (round - 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t *sa = smem + st * C::STAGE_BYTES;
          mbar_arrive_expect_tx(&full[st], C::STAGE_BYTES);
          tma_load_2d(sa, &tmX, &full[st], kb * C::BK, m0);
          tma_load_2d(sa + C::A_BYTES, &tmW, &full[st], kb * C::BK, n0);
        }
      }
      if (!ok) {
        for (int u = it - C::NST < 0 ? 0 : it - C::NST; u < it; u++)
          mbar_wait_raw(&full[u % C::NST], (u / C::NST) & 1, 100000000ull);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    constexpr uint32_t IDESC = idesc_mma_f32(C::BM, BN, BF16 ? 1u : 0u);
    const uint32_t sbase = smem_u32(smem);
    bool ok = true;
    int it = 0;
    int local = 0;  // tiles of this CTA so far
    for (int tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x, local++) {
      const int buf = local & 1;
      // The epilogue must have read this accumulator buffer (two tiles ago).
      if (local >= 2 && !(ok = mbar_wait(&acc_empty[buf], ((local >> 1) - 1) & 1, abort_flag)))
        break;
      tc_fence_after();
      for (int kb = 0; kb < p.k_blocks; kb++, it++) {
        const int st = it % C::NST;
        if (!(ok = mbar_wait(&full[st], (it / C::NST) & 1, abort_flag))) break;
        tc_fence_after();
        const uint32_t a = sbase + st * C::STAGE_BYTES;
        const uint32_t b = a + C::A_BYTES;
#pragma unroll
        for (int kk = 0; kk < C::BK / 16; kk++) {
          if (elect_one())
            mma_ss(tmem + buf * BN, sdesc_sw128(a + kk * 32, 16, 1024),
                   sdesc_sw128(b + kk * 32, 16, 1024), IDESC, (kb > 0 || kk > 0) ? 1u : 0u);
        }
        if (elect_one()) mma_commit(&empty[st]);
      }
      if (!ok) break;
      if (elect_one()) mma_commit(&acc_full[buf]);
    }
    if (elect_one()) mma_commit(drain);
    mbar_wait_raw(drain, 0, 100000000ull);
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // warps 2..5 -> TMEM lane quarters 2,3,0,1
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    bool ok = true;
    int local = 0;
    for (int tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x, local++) {
      const int buf = local & 1;
      int m0, n0;
      decode(tile, m0, n0);
      ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[buf], (local >> 1) & 1, abort_flag));
      if (!ok) break;
      tc_fence_after();
      qkv_tile_epilogue<D, BN>(p, tmem + lane_off + buf * BN, m0 + row, n0, [&]() {
        // The accumulator buffer is read out: the MMA warp may reuse it.
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
      });
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicExch(p.err, 1);
}

// ---------------------------------------------------------------------------
// The same projection on CTA pairs (2-CTA clusters, tcgen05 cta_group::2):
// a pair computes a 256 x 256 tile — each CTA holds 128 rows of x and 128 of
// the 256 W rows (columns of the tile) per K step, so each SM moves half the
// operand bytes of the single-CTA kernel per MMA, and six 32 KB stages fit.
// The even CTA issues the pair's MMAs (M = 256, N = 256) and owns the stage
// "full" barriers, which count both CTAs' TMA bytes; every MMA commit is
// delivered to the matching barrier of both CTAs; each CTA's epilogue reads
// its own 128 accumulator rows from its own TMEM and releases the buffer on
// the even CTA's barrier.
template <int D>
struct Qkv2Cfg {
  static constexpr int BM = 128, BN = 256, BK = 64;  // BM per CTA; BN per pair
  static constexpr int A_BYTES = BM * BK * 2;          // 16 KB
  static constexpr int B_BYTES = (BN / 2) * BK * 2;    // 16 KB (this CTA's half)
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int NST = 6;
  static constexpr int BAR_OFF = NST * STAGE_BYTES;
  // full[NST], empty[NST], acc_full[2], acc_empty[2], drain; tmem word; abort
  static constexpr int NBAR = 2 * NST + 2 + 2 + 1;
  static constexpr int SMEM_BYTES = BAR_OFF + NBAR * 8 + 16 + 1024;
  static constexpr int THREADS = 192;
  static constexpr uint32_t TMEM_COLS = 2 * BN;
};

template <int D, bool BF16>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(192, 1)
    qkv_proj_pair_kernel(const __grid_constant__ CUtensorMap tmX,
                         const __grid_constant__ CUtensorMap tmW, const QkvParams p) {
  using C = Qkv2Cfg<D>;
  constexpr int BN = C::BN;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t *smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
  uint64_t *full = bars;
  uint64_t *empty = full + C::NST;
  uint64_t *acc_full = empty + C::NST;
  uint64_t *acc_empty = acc_full + 2;
  uint64_t *drain = acc_empty + 2;
  uint32_t *tmem_base_slot = reinterpret_cast<uint32_t *>(drain + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_base_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0 = the pair's MMA issuer
  const uint32_t peer = rank ^ 1u;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int m_tiles = (p.M + 2 * C::BM - 1) / (2 * C::BM);  // 256-row tiles
  const int tiles = m_tiles * p.n_tiles;
  constexpr int kGroupM = 8;
  auto decode = [&](int tile, int &m0, int &n0) {
    const int per_group = kGroupM * p.n_tiles;
    const int grp = tile / per_group;
    const int first = grp * kGroupM;
    const int gm = m_tiles - first < kGroupM ? m_tiles - first : kGroupM;
    const int in = tile - grp * per_group;
    m0 = (first + in % gm) * 2 * C::BM;
    n0 = (in / gm) * BN;
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::NST; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 8);  // four epilogue warps of each CTA
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_base_slot, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmX);
      tma_prefetch_desc(&tmW);
      bool ok = true;
      int it = 0;
      for (int tile = pair; tile < tiles && ok; tile += npairs) {
        int m0, n0;
        decode(tile, m0, n0);
        for (int kb = 0; kb < p.k_blocks; kb++, it++) {
          const int st = it % C::NST, round = it / C::NST;
          if (round > 0 && !mbar_wait(&empty[st], (round - 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t *sa = smem + st * C::STAGE_BYTES;
          // Both CTAs' bytes complete on the even CTA's full[st].
          if (rank == 0) mbar_arrive_expect_tx(&full[st], 2 * C::STAGE_BYTES);
          const uint32_t fb = mapa_shared(smem_u32(&full[st]), 0);
          tma_load_2d_pair(sa, &tmX, fb, kb * C::BK, m0 + rank * C::BM);
          tma_load_2d_pair(sa + C::A_BYTES, &tmW, fb, kb * C::BK, n0 + rank * (BN / 2));
        }
      }
      if (!ok && rank == 0) {
        // Abort path: every armed stage (both CTAs' bytes) lands before exit.
        for (int u = it - C::NST < 0 ? 0 : it - C::NST; u < it; u++)
          mbar_wait_raw(&full[u % C::NST], (u / C::NST) & 1, 100000000ull);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (rank == 0) {
      constexpr uint32_t IDESC = idesc_mma_f32(2 * C::BM, BN, BF16 ? 1u : 0u);
      const uint32_t sbase = smem_u32(smem);
      bool ok = true;
      int it = 0;
      int local = 0;
      for (int tile = pair; tile < tiles && ok; tile += npairs, local++) {
        const int buf = local & 1;
        if (local >= 2 &&
            !(ok = mbar_wait_cluster(&acc_empty[buf], ((local >> 1) - 1) & 1, abort_flag)))
          break;
        tc_fence_after();
        for (int kb = 0; kb < p.k_blocks; kb++, it++) {
          const int st = it % C::NST;
          if (!(ok = mbar_wait(&full[st], (it / C::NST) & 1, abort_flag))) break;
          tc_fence_after();
          const uint32_t a = sbase + st * C::STAGE_BYTES;
          const uint32_t b = a + C::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < C::BK / 16; kk++) {
            if (elect_one())
              mma_ss_pair(tmem + buf * BN, sdesc_sw128(a + kk * 32, 16, 1024),
                          sdesc_sw128(b + kk * 32, 16, 1024), IDESC,
                          (kb > 0 || kk > 0) ? 1u : 0u);
          }
          if (elect_one()) {
            mma_commit_pair(smem_u32(&empty[st]));
            mma_commit_pair(mapa_shared(smem_u32(&empty[st]), peer));
          }
        }
        if (!ok) break;
        if (elect_one()) {
          mma_commit_pair(smem_u32(&acc_full[buf]));
          mma_commit_pair(mapa_shared(smem_u32(&acc_full[buf]), peer));
        }
      }
      if (elect_one()) mma_commit_pair(smem_u32(drain));
      mbar_wait_raw(drain, 0, 100000000ull);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    bool ok = true;
    int local = 0;
    for (int tile = pair; tile < tiles && ok; tile += npairs, local++) {
      const int buf = local & 1;
      int m0, n0;
      decode(tile, m0, n0);
      ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[buf], (local >> 1) & 1, abort_flag));
      if (!ok) break;
      tc_fence_after();
      qkv_tile_epilogue<D, BN>(p, tmem + lane_off + buf * BN, m0 + rank * C::BM + row, n0,
                               [&]() {
                                 tc_fence_before();
                                 __syncwarp();
                                 if (lane == 0)
                                   mbar_arrive_remote(mapa_shared(smem_u32(&acc_empty[buf]), 0));
                               });
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no pair MMA or remote arrival is left in flight
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem, C::TMEM_COLS);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicExch(p.err, 1);
}

}  // namespace llmr

namespace llmr {

// ---------------------------------------------------------------------------
// Output projection with the gated residual in its epilogue:
//
//   hidden[b*S + s, n] += gate_g[n] * ( O[b*S + s, :] . W_g[n, :] + bias_g[n] )
//
// g = 1 for tokens s >= split_row (when split_row > 0), else 0: the joint
// blocks' two streams (txt / img, or img / txt) with their own weights,
// biases and gates (dependencies/flux.c3l/flux_dit.c3:874-885,
// dependencies/qwen_edit.c3l/mmdit.c3:694-720: matmul, broadcast_bias_add
// vit.slang:133-137, gated_residual_add vit.slang:638-647). O is the
// attention output [B*S][in_dim] (fp16 / bf16), W_g [out_dim][in_dim] of the
// same type, hidden fp32 [B*S][out_dim] updated in place. Same CTA layout as
// qkv_proj_kernel; m-tiles never straddle a segment, so every tile uses one
// weight matrix (rows of a tile beyond its segment are computed and dropped).
struct ProjParams {
  int M, S, B;
  int split;             // token index where set 1 starts (S when no split)
  int seg_tiles0;        // m-tiles of segment 0 per batch element
  int seg_tiles1;        // m-tiles of segment 1 per batch element
  int k_blocks;          // in_dim / 64
  int n_tiles;           // out_dim / 256
  int tiles;             // B * (seg_tiles0 + seg_tiles1) * n_tiles
  int out_dim;
  long long h_stride;    // hidden row stride (elements)
  const float *bias[2], *gate[2];
  float *hidden;
  int *err;
};

// Epilogue staging: 4 warps x 32 rows x 33 floats after the pipeline's
// barriers (16-byte aligned).
constexpr int kProjStageOff =
    ((QkvCfg<128, 256>::BAR_OFF + QkvCfg<128, 256>::NBAR * 8 + 16 + 15) / 16) * 16;
constexpr int kProjSmemBytes = kProjStageOff + 4 * 32 * 33 * 4 + 1024;

template <bool BF16>
__global__ void __launch_bounds__(192, 1)
    out_proj_kernel(const __grid_constant__ CUtensorMap tmX,
                    const __grid_constant__ CUtensorMap tmW0,
                    const __grid_constant__ CUtensorMap tmW1, const ProjParams p) {
  constexpr int BN = 256;
  using C = QkvCfg<128, BN>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t *smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
  uint64_t *full = bars;
  uint64_t *empty = full + C::NST;
  uint64_t *acc_full = empty + C::NST;
  uint64_t *acc_empty = acc_full + 2;
  uint64_t *drain = acc_empty + 2;
  uint32_t *tmem_base_slot = reinterpret_cast<uint32_t *>(drain + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_base_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int mt_per_b = p.seg_tiles0 + p.seg_tiles1;
  const int m_tiles = p.B * mt_per_b;
  // Tile -> (first row, last row + 1 of its segment, weight set, column).
  // Groups of 16 m-tiles walked m-fastest over all column blocks (L2 reuse).
  constexpr int kGroupM = 16;
  auto decode = [&](int tile, int &m0, int &m_end, int &set, int &n0) {
    const int per_group = kGroupM * p.n_tiles;
    const int grp = tile / per_group;
    const int first = grp * kGroupM;
    const int gm = m_tiles - first < kGroupM ? m_tiles - first : kGroupM;
    const int in = tile - grp * per_group;
    const int mt = first + in % gm;
    n0 = (in / gm) * BN;
    const int b = mt / mt_per_b, r = mt - b * mt_per_b;
    set = r < p.seg_tiles0 ? 0 : 1;
    const int seg0 = set == 0 ? 0 : p.split;
    const int seg1 = set == 0 ? p.split : p.S;
    m0 = b * p.S + seg0 + (set == 0 ? r : r - p.seg_tiles0) * C::BM;
    m_end = b * p.S + seg1;
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::NST; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_base_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmX);
      tma_prefetch_desc(&tmW0);
      tma_prefetch_desc(&tmW1);
      bool ok = true;
      int it = 0;
      for (int tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x) {
        int m0, m_end, set, n0;
        decode(tile, m0, m_end, set, n0);
        const CUtensorMap *mw = set ? &tmW1 : &tmW0;
        for (int kb = 0; kb < p.k_blocks; kb++, it++) {
          const int st = it % C::NST, round = it / C::NST;
          if (round > 0 && !mbar_wait(&empty[st], (round - 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t *sa = smem + st * C::STAGE_BYTES;
          mbar_arrive_expect_tx(&full[st], C::STAGE_BYTES);
          tma_load_2d(sa, &tmX, &full[st], kb * C::BK, m0);
          tma_load_2d(sa + C::A_BYTES, mw, &full[st], kb * C::BK, n0);
        }
      }
      if (!ok) {
        for (int u = it - C::NST < 0 ? 0 : it - C::NST; u < it; u++)
          mbar_wait_raw(&full[u % C::NST], (u / C::NST) & 1, 100000000ull);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    constexpr uint32_t IDESC = idesc_mma_f32(C::BM, BN, BF16 ? 1u : 0u);
    const uint32_t sbase = smem_u32(smem);
    bool ok = true;
    int it = 0;
    int local = 0;
    for (int tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x, local++) {
      const int buf = local & 1;
      if (local >= 2 && !(ok = mbar_wait(&acc_empty[buf], ((local >> 1) - 1) & 1, abort_flag)))
        break;
      tc_fence_after();
      for (int kb = 0; kb < p.k_blocks; kb++, it++) {
        const int st = it % C::NST;
        if (!(ok = mbar_wait(&full[st], (it / C::NST) & 1, abort_flag))) break;
        tc_fence_after();
        const uint32_t a = sbase + st * C::STAGE_BYTES;
        const uint32_t b = a + C::A_BYTES;
#pragma unroll
        for (int kk = 0; kk < C::BK / 16; kk++) {
          if (elect_one())
            mma_ss(tmem + buf * BN, sdesc_sw128(a + kk * 32, 16, 1024),
                   sdesc_sw128(b + kk * 32, 16, 1024), IDESC, (kb > 0 || kk > 0) ? 1u : 0u);
        }
        if (elect_one()) mma_commit(&empty[st]);
      }
      if (!ok) break;
      if (elect_one()) mma_commit(&acc_full[buf]);
    }
    if (elect_one()) mma_commit(drain);
    mbar_wait_raw(drain, 0, 100000000ull);
  } else {
    // ------------------------------------------------------------ epilogue
    // Per 32-column chunk: each thread (one accumulator row) parks its 32
    // values in this warp's padded staging block; the warp then updates the
    // 32 rows one at a time with coalesced 128-byte accesses, all 32 rows'
    // loads of `hidden` issued before any store.
    const int quarter = warp & 3;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    float *stage = reinterpret_cast<float *>(smem + kProjStageOff) + (warp - 2) * 32 * 33;
    bool ok = true;
    int local = 0;
    for (int tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x, local++) {
      const int buf = local & 1;
      int m0, m_end, set, n0;
      decode(tile, m0, m_end, set, n0);
      ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[buf], (local >> 1) & 1, abort_flag));
      if (!ok) break;
      tc_fence_after();
      // select by value: indexing the parameter arrays would copy them to
      // local memory
      const float *bias = set ? p.bias[1] : p.bias[0];
      const float *gate = set ? p.gate[1] : p.gate[0];
      const int rbase = m0 + quarter * 32;      // first row of this warp
      const int rlim = m_end < p.M ? m_end : p.M;
#pragma unroll 1
      for (int c = 0; c < BN / 32; c++) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_off + buf * BN + c * 32, r);
        tmem_wait_ld();
        reg_fence32(r);
        if (c == BN / 32 - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[buf]);
        }
#pragma unroll
        for (int k = 0; k < 32; k++) stage[lane * 33 + k] = __uint_as_float(r[k]);
        __syncwarp();
        const int col = n0 + c * 32 + lane;
        const float bj = bias != nullptr ? bias[col] : 0.0f;
        const float gj = gate != nullptr ? gate[col] : 1.0f;
        float hv[32];
#pragma unroll
        for (int rr = 0; rr < 32; rr++)
          hv[rr] = rbase + rr < rlim ? p.hidden[(long long)(rbase + rr) * p.h_stride + col] : 0.0f;
#pragma unroll
        for (int rr = 0; rr < 32; rr++)
          if (rbase + rr < rlim)
            p.hidden[(long long)(rbase + rr) * p.h_stride + col] =
                hv[rr] + gj * (stage[rr * 33 + lane] + bj);
        __syncwarp();
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicExch(p.err, 1);
}

}  // namespace llmr
