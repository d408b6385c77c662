// Non-causal flash attention forward for sm_100a on the 5th-generation
// tensor cores (tcgen05), fp16 operands, fp32 accumulation in TMEM.
//
// Computes, per (batch, head), O = softmax(scale * Q K^T) V with the same
// operand rounding as the reference shader (Q, K, V and P held as fp16,
// scores / softmax state / O accumulated in fp32:
// dependencies/zimage.c3l/shaders/flash_attn.slang:61-64, :98-101, :197-201,
// :113-118). Rows and keys beyond seq_len are masked exactly as :120-121 do.
//
// CTA = 2 query tiles of 128 rows of one (b, h) = 256 queries; 384 threads:
//   warps 0-3  softmax warpgroup for tile 0 (thread i owns query row i)
//   warps 4-7  softmax warpgroup for tile 1
//   warp  8    TMA producer: Q once, then K_j, V_j into an NST-slot ring
//   warp  9    MMA issuer (one elected lane) + TMEM owner
//   warps 10-11 idle (they complete warpgroup 2 for the register split)
// setmaxnreg moves registers from warpgroup 2 to the softmax warpgroups,
// which hold a whole row of 128 scores each between the two passes.
// TMEM (512 columns): S0 [0,128) S1 [128,256) O0 [256,256+D) O1 [256+D,256+2D)
// P_t (fp16x2) overwrites the first 64 columns of S_t after it is read.
// MMA order per key block j (ping-pong, so one tile's softmax overlaps the
// other tile's GEMMs):
//   PV0_j, S0_{j+1}, PV1_j, S1_{j+1}
// The softmax rescales O lazily: only when a row max grows by more than
// 2^15 over the max used so far (so fp16 P stays <= 32768).
#pragma once
#include <type_traits>

#include "prologue.cuh"
#include "ptx.cuh"

namespace llmr {

constexpr int kMaxSeqs = 64;  // packed sequences of one variable-length call

struct FaParams {
  int S;                 // queries per (b, h) (packed: total tokens)
  int S_kv;              // keys per (b, h)
  int H;                 // heads
  int nqt;               // query-tile pairs (256 queries) per (b, h)
  int units;             // work units (B * H * nqt, or the packed total)
  // Variable-length mode (nseq > 0): the maps hold one packed batch element
  // of S tokens; sequence i is tokens [seq_off[i], seq_off[i+1]) and owns
  // units [unit_off[i], unit_off[i+1]) (H * its query-tile pairs).
  int nseq;
  int seq_off[kMaxSeqs + 1];
  int unit_off[kMaxSeqs + 1];
  float scale_log2;      // softmax scale * log2(e)
  void *o;               // output base (OutT)
  long long o_row_stride;    // elements between consecutive tokens
  long long o_batch_stride;  // elements between batch elements
  float *lse;            // optional [B][H][S] natural-log LSE
  int merge;             // o (fp32) and lse hold a partial result over other
                         // keys: merge into them by log-sum-exp
  int *err;              // device error word (nonzero on timeout)
  // Per-CTA event timestamps (globaltimer ns, kTimelineSlots per CTA) when
  // the library is built with -DLLMR_TIMELINE and a buffer is set; else null.
  unsigned long long *timeline;
};

// Timeline slots (LLMR_TIMELINE builds): 0 kernel start, 1 start-up phase
// done, 2 + 2k / 3 + 2k producer begins unit k / its K'/V' are ready (k < 4),
// 10 + 2k / 11 + 2k tile 0's first S of unit k ready / epilogue done,
// 18 background Q' of unit 1 done, 19 background K'/V' pieces done,
// 20 background done, 21 kernel end, 22 past griddepcontrol.wait, for unit
// k < 3 of tile 0: 23 + k its last P handed over, 26 + k its O complete
// (epilogue starts), 29 + k its block 1's S ready (all %globaltimer ns).
// Slots 32-127, SM clock cycles (clock64) in blocks 4-11 of the CTA's second
// unit (i = j - 4): the softmax of tile t, row 0, at 32 + 32t + 4i S_j ready,
// +1 row max done, +2 P keys 0-63 handed over, +3 P keys 64-127 handed over;
// the MMA warp at 96 + 4i + 2t + half, the issue of the PV MMAs of that half
// of P_t (after their wait).
constexpr int kTimelineSlots = 128;
#ifdef LLMR_TIMELINE
#define LLMR_TL(slot)                                                                    \
  do {                                                                                   \
    if (p.timeline)                                                                      \
      p.timeline[(size_t)blockIdx.x * kTimelineSlots + (slot)] = globaltimer_ns();       \
  } while (0)
#define LLMR_TLC(slot)                                                                   \
  do {                                                                                   \
    if (p.timeline)                                                                      \
      p.timeline[(size_t)blockIdx.x * kTimelineSlots + (slot)] = clock64();              \
  } while (0)
#else
#define LLMR_TL(slot) \
  do {                \
  } while (0)
#define LLMR_TLC(slot) \
  do {                 \
  } while (0)
#endif

// The prologue fused into the attention kernel (LLMR_FUSED_PROLOGUE, not the
// default): the kernel itself writes the fp16 Q', K', V' its TMA maps read.
// Work is cut into pieces of 32 token rows of one (tensor, b, h).
//  * Start-up: every warp of every CTA writes the K'/V' pieces of the (b, h)
//    pairs that the first round of units touches (spread round-robin over
//    all warps of the grid), and the CTA's own warps write the Q' of its
//    first unit.
//  * Background: warps 10-11 (otherwise idle) write the Q' of the CTA's next
//    unit, then the K'/V' pieces of the remaining (b, h) pairs in order, then
//    the Q' of the later units, while the other warps run attention.
//  * sync[1 + b*H + h] counts the K'/V' pieces of (b, h) written (released
//    after the pieces' stores); a unit's K/V loads wait until it reaches
//    2 * nrb. Q' of a later unit is handed to the producer through a
//    per-warp counter in shared memory. The last CTA to finish resets sync[] to zero, so the
//    buffer is ready for the next launch without a memset.
// All CTAs must be resident together (they wait for pieces written by
// others): the kernel is launched cooperatively with at most one CTA per SM.
struct FusedPro {
  const void *q, *k, *v;          // raw inputs (fp16 / bf16)
  long long qs[3], ks[3], vs[3];  // {batch, row, head} strides in elements
  __half *ws;                     // Q', K', V' fp16 [3][B][H][S][D]
  int *sync;                      // [0] CTAs finished, [1 + bh] pieces ready
  ProParams pp;
  int nrb;                        // 32-row pieces per (b, h) and tensor
  int startup_bh;                 // (b, h) pairs written in the start-up phase
};

// Bounded wait until the global counter reaches `target` (acquire).
__device__ __forceinline__ bool counter_wait(const int *ctr, int target,
                                             volatile int *abort_flag) {
  const uint64_t t0 = globaltimer_ns();
  uint32_t n = 0;
  while (true) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
    if (v >= target) return true;
    if ((++n & 15u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > LLMR_WAIT_LIMIT_NS) {
        *abort_flag = 1;
        return false;
      }
    }
    __nanosleep(64);
  }
}

// Bounded wait until a counter in shared memory, written by another warp of
// the CTA after a __threadfence, reaches `target`.
__device__ __forceinline__ bool smem_counter_wait(volatile int *ctr, int target,
                                                  volatile int *abort_flag) {
  const uint64_t t0 = globaltimer_ns();
  uint32_t n = 0;
  while (*ctr < target) {
    if ((++n & 15u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > LLMR_WAIT_LIMIT_NS) {
        *abort_flag = 1;
        return false;
      }
    }
    __nanosleep(32);
  }
  __threadfence();
  return true;
}

// Orders this thread's generic-proxy global writes before later async-proxy
// (TMA) reads of them, by any thread that synchronises with this one.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

template <int D>
struct FaCfg {
  static constexpr int BM = 128;                 // query rows per tile
  static constexpr int BN = 128;                 // keys per block
  static constexpr int CHUNK_BYTES = 128 * 128;  // one 64-col x 128-row SW128 box
  static constexpr int NCHUNK = D / 64;
  static constexpr int TILE_BYTES = BM * D * 2;  // one Q/K/V tile, fp16
  static constexpr int NST = D == 128 ? 4 : 8;   // K/V ring slots
  static constexpr int Q_OFF = 0;
  static constexpr int KV_OFF = 2 * TILE_BYTES;
  static constexpr int BAR_OFF = KV_OFF + NST * TILE_BYTES;
  // barriers: q_full, q_empty, kv_full[NST], kv_empty[NST], s_full[2],
  // p_half[2][2] (P of keys 0-63 / 64-127 of tile t written), o_full[2],
  // o_empty[2], drain; then tmem base word and abort flag
  static constexpr int NBAR = 2 + 2 * NST + 2 + 4 + 2 + 2 + 1 + 1;  // + q_done[2]
  // Fused prologue: a cp.async prefetch ring per background warp in the
  // shared memory left over (the non-fused kernel leaves it unused).
  static constexpr int BG_OFF = (BAR_OFF + NBAR * 8 + 16 + 127) / 128 * 128;
  static constexpr int BG_RING = 12 * 1024;  // bytes per background warp
  // Without the fused prologue the same region stages the epilogue's output
  // rows: 4 KB per softmax warp (32 rows x 128 bytes).
  static constexpr int EPI_OFF = BG_OFF;
  static constexpr int EPI_BYTES = 8 * 4096;
  static constexpr int REGION = EPI_BYTES > 2 * BG_RING ? EPI_BYTES : 2 * BG_RING;
  static constexpr int SMEM_BYTES = BG_OFF + REGION + 1024;  // +align slack
  static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
  static constexpr int THREADS = 384;
  // Register split (setmaxnreg): the two softmax warpgroups hold a whole
  // 128-score row per thread; the producer / MMA warpgroup needs few.
  static constexpr int REG_SOFTMAX = 200;
  static constexpr int REG_OTHER = 104;
  static constexpr int REG_LAUNCH = 168;  // 65536 / 384, rounded down to 8
  static constexpr int REG_NEED = 2 * 128 * REG_SOFTMAX + 128 * REG_OTHER;
  static_assert(REG_NEED <= THREADS * REG_LAUNCH, "register split exceeds the launch allocation");
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t O_COL = 256;
};

// Work decomposition of a launch: units of (b, h, 256 queries), one CTA per
// SM walking them (the kernel keeps a whole SM: shared memory and TMEM).
template <int D>
inline dim3 fa_grid(FaParams &p, int B, int num_sms) {
  using C = FaCfg<D>;
  p.nqt = (p.S + 2 * C::BM - 1) / (2 * C::BM);
  if (p.nseq > 0) {
    p.unit_off[0] = 0;
    for (int i = 0; i < p.nseq; i++) {
      const int len = p.seq_off[i + 1] - p.seq_off[i];
      p.unit_off[i + 1] = p.unit_off[i] + p.H * ((len + 2 * C::BM - 1) / (2 * C::BM));
    }
    p.units = p.unit_off[p.nseq];
  } else {
    p.units = B * p.H * p.nqt;
  }
  const int sms = num_sms > 0 ? num_sms : 148;
  return dim3(p.units < sms ? p.units : sms);
}


// Which of the 16 exponential pairs of a 32-column chunk are computed on the
// FMA pipe (exp2_poly_x2) instead of MUFU ex2: bit i set = pair i. Sharing
// the work between the two pipes keeps MUFU (which also packs P to fp16) from
// bounding the softmax.
#ifndef LLMR_EXP2_EMU_MASK
#define LLMR_EXP2_EMU_MASK 0x1111u  // 1 pair in 4: the measured optimum on B200
#endif
constexpr uint32_t kExp2EmuMask = LLMR_EXP2_EMU_MASK;

#ifndef LLMR_HALF0_AT
#define LLMR_HALF0_AT 1
#endif
constexpr int kHalf0At = LLMR_HALF0_AT;  // chunk after which P keys 0-63 are handed over

// Largest exponent argument x = s*scale*log2e - m the softmax lets through
// without rescaling: P = 2^x <= 2^15 stays finite in fp16 (max 65504) with
// the same 2^-11 relative rounding as any other value, and O / l accumulate
// in fp32. A row max growing past this triggers the (rare) rescale path.
constexpr float kMaxExp = 15.0f;

template <typename OutT>
__device__ __forceinline__ void store_row_chunk(OutT *dst, const float *v);

template <>
__device__ __forceinline__ void store_row_chunk<float>(float *dst,
                                                       const float *v) {
#pragma unroll
  for (int i = 0; i < 32; i += 4)
    *reinterpret_cast<float4 *>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
}
template <>
__device__ __forceinline__ void store_row_chunk<__half>(__half *dst,
                                                        const float *v) {
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
    uint4 u;
    u.x = pack_f16x2(v[i], v[i + 1]);
    u.y = pack_f16x2(v[i + 2], v[i + 3]);
    u.z = pack_f16x2(v[i + 4], v[i + 5]);
    u.w = pack_f16x2(v[i + 6], v[i + 7]);
    *reinterpret_cast<uint4 *>(dst + i) = u;
  }
}
template <>
__device__ __forceinline__ void store_row_chunk<__nv_bfloat16>(
    __nv_bfloat16 *dst, const float *v) {
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
    uint4 u;
    __nv_bfloat162 a = __floats2bfloat162_rn(v[i], v[i + 1]);
    __nv_bfloat162 b = __floats2bfloat162_rn(v[i + 2], v[i + 3]);
    __nv_bfloat162 c = __floats2bfloat162_rn(v[i + 4], v[i + 5]);
    __nv_bfloat162 d = __floats2bfloat162_rn(v[i + 6], v[i + 7]);
    u.x = *reinterpret_cast<uint32_t *>(&a);
    u.y = *reinterpret_cast<uint32_t *>(&b);
    u.z = *reinterpret_cast<uint32_t *>(&c);
    u.w = *reinterpret_cast<uint32_t *>(&d);
    *reinterpret_cast<uint4 *>(dst + i) = u;
  }
}

// InT = void: Q', K', V' are already in the maps' memory. InT = __half or
// __nv_bfloat16: the kernel writes them from the raw inputs (FusedPro).
template <int D, typename OutT, typename InT = void>
__global__ void __launch_bounds__(384, 1)
    fa_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                     const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV,
                     const FaParams p, const __grid_constant__ FusedPro fp) {
  using C = FaCfg<D>;
  constexpr bool FUSED = !std::is_void<InT>::value;
  using In = typename std::conditional<FUSED, InT, __half>::type;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment: SW128 atoms must start on 1024-byte boundaries so
  // that the descriptors' base offset is 0.
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t *smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);

  uint8_t *sQ = smem + C::Q_OFF;
  uint8_t *sKV = smem + C::KV_OFF;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
  uint64_t *q_full = bars;
  uint64_t *q_empty = bars + 1;
  uint64_t *kv_full = bars + 2;
  uint64_t *kv_empty = kv_full + C::NST;
  uint64_t *s_full = kv_empty + C::NST;
  uint64_t *p_half = s_full + 2;  // [t * 2 + half]
  uint64_t *o_full = p_half + 4;  // [t]
  uint64_t *o_empty = o_full + 2; // [t]
  uint64_t *drain = o_empty + 2;
  // Fused prologue: units whose Q' each background warp has written (a
  // warp may run several units ahead of the producer, so counters rather
  // than an mbarrier's phases).
  volatile int *q_done = reinterpret_cast<volatile int *>(drain + 1);
  uint32_t *tmem_base_slot = reinterpret_cast<uint32_t *>(drain + 2);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_base_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int S = p.S;
  // Work units (b, h, query-tile pair), persistent over the grid: this CTA
  // takes units blockIdx.x, blockIdx.x + gridDim.x, ... Consecutive units
  // share (b, h), so CTAs running together share K/V tiles in L2. A unit's
  // geometry: map batch coordinate b, head h, first query q0 (relative to
  // row0, the first token of its sequence in the maps), its query and key
  // counts, and its number of key blocks.
  struct Unit {
    int b, h, q0, row0, sq, sk, nblk;
  };
  auto decode = [&](int unit) {
    Unit u;
    if (p.nseq > 0) {
      int i = 0;
      while (i + 1 < p.nseq && unit >= p.unit_off[i + 1]) i++;
      const int len = p.seq_off[i + 1] - p.seq_off[i];
      const int nqt = (len + 2 * C::BM - 1) / (2 * C::BM);
      const int local = unit - p.unit_off[i];
      u.h = local / nqt;
      u.q0 = (local - u.h * nqt) * 2 * C::BM;
      u.b = 0;
      u.row0 = p.seq_off[i];
      u.sq = len;
      u.sk = len;
    } else {
      const int bh = unit / p.nqt;
      u.q0 = (unit - bh * p.nqt) * 2 * C::BM;
      u.b = bh / p.H;
      u.h = bh - u.b * p.H;
      u.row0 = 0;
      u.sq = p.S;
      u.sk = p.S_kv;
    }
    u.nblk = (u.sk + C::BN - 1) / C::BN;
    return u;
  };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < C::NST; i++) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int t = 0; t < 2; t++) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_half[2 * t], 4);  // one arrival per softmax warp
      mbar_init(&p_half[2 * t + 1], 4);
      mbar_init(&o_full[t], 1);
      mbar_init(&o_empty[t], 4);
    }
    mbar_init(drain, 1);
    q_done[0] = q_done[1] = 0;
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_base_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_slot;
  if (threadIdx.x == 0) LLMR_TL(0);
  // Launched right behind the prologue (programmatic dependent launch), the
  // set-up above overlaps its tail; its output is read only after this.
  griddep_wait();
  if (threadIdx.x == 0) LLMR_TL(22);

  const View<In> vq{static_cast<const In *>(fp.q), fp.qs[0], fp.qs[1], fp.qs[2]};
  const View<In> vk{static_cast<const In *>(fp.k), fp.ks[0], fp.ks[1], fp.ks[2]};
  const View<In> vv{static_cast<const In *>(fp.v), fp.vs[0], fp.vs[1], fp.vs[2]};
  // K'/V' piece i (ordered by (b, h)): tensor 1 + r / nrb, rows 32 * (r % nrb).
  auto kv_piece = [&](int i) {
    const int per = 2 * fp.nrb;
    const int bh = i / per, r = i - bh * per;
    const int t = 1 + r / fp.nrb, rb = r - (t - 1) * fp.nrb;
    return make_int4(bh, t, rb, 0);
  };
  // Publishes a finished K'/V' piece of (b, h): the pieces' stores, made
  // visible to the async proxy and at GPU scope, then the counter.
  auto publish = [&](int bh) {
    fence_proxy_async_global();
    __threadfence();
    __syncwarp();
    if (lane == 0) atomicAdd(fp.sync + 1 + bh, 1);
  };
  if constexpr (FUSED) {
    // ------------------------------------------------ fused prologue, start-up
    const int G = gridDim.x;
    const int nstart = fp.startup_bh * 2 * fp.nrb;
    for (int i = warp * G + blockIdx.x; i < nstart; i += (C::THREADS / 32) * G) {
      const int4 pc = kv_piece(i);
      const int b = pc.x / p.H, h = pc.x - b * p.H;
      pro_piece<D, In, 4>(vq, vk, vv, fp.ws, fp.pp, pc.y, b, h, pc.z * 32, lane);
      publish(pc.x);
    }
    // Q' of this CTA's first unit: its 8 pieces on warps 0-7.
    if ((int)blockIdx.x < p.units && warp < 8) {
      const Unit un = decode(blockIdx.x);
      const int s0 = un.q0 + warp * 32;
      if (s0 < un.sq) pro_piece<D, In, 4>(vq, vk, vv, fp.ws, fp.pp, 0, un.b, un.h, s0, lane);
      fence_proxy_async_global();
    }
    __syncthreads();
    if (threadIdx.x == 0) LLMR_TL(1);
  }

  if (warp >= 8) {
    reg_dealloc<C::REG_OTHER>();
    if (warp == 8) {
      // ---------------------------------------------------------- producer
      if (lane == 0) {
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
        bool ok = true;
        int issued = 0;  // K/V tile loads armed so far (over all units)
        int kq = 0;      // Q loads armed so far
        int jb = 0;      // key blocks of this CTA's earlier units
        for (int unit = blockIdx.x, k = 0; unit < p.units && ok; unit += gridDim.x, k++) {
          const Unit un = decode(unit);
          const int b = un.b, h = un.h, nblk = un.nblk;
          // Q of this unit may replace the previous unit's once its last
          // S MMAs have completed.
          if (k < 4) LLMR_TL(2 + 2 * k);
          if (k > 0 && !mbar_wait(q_empty, (k - 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
          if constexpr (FUSED) {
            // Q' of a later unit comes from the background warps; K'/V' of
            // this (b, h) from pieces written all over the grid.
            if (k > 0 && !(smem_counter_wait(&q_done[0], k, abort_flag) &&
                           smem_counter_wait(&q_done[1], k, abort_flag))) {
              ok = false;
              break;
            }
            if (!counter_wait(fp.sync + 1 + b * p.H + h, 2 * fp.nrb, abort_flag)) {
              ok = false;
              break;
            }
            fence_proxy_async_global();
          }
          if (k < 4) LLMR_TL(3 + 2 * k);
          mbar_arrive_expect_tx(q_full, 2 * C::TILE_BYTES);
          for (int t = 0; t < 2; t++)
            for (int c = 0; c < C::NCHUNK; c++)
              tma_load_4d(sQ + t * C::TILE_BYTES + c * C::CHUNK_BYTES, &tmQ, q_full,
                          c * 64, un.row0 + un.q0 + t * C::BM, h, b);
          kq = k + 1;
          for (int j = 0; j < nblk && ok; j++) {
            for (int kind = 0; kind < 2; kind++) {
              const int u = 2 * (jb + j) + kind;
              const int slot = u % C::NST, round = u / C::NST;
              if (round > 0 && !mbar_wait(&kv_empty[slot], (round - 1) & 1, abort_flag)) {
                ok = false;
                break;
              }
              mbar_arrive_expect_tx(&kv_full[slot], C::TILE_BYTES);
              const CUtensorMap *m = kind ? &tmV : &tmK;
              for (int c = 0; c < C::NCHUNK; c++)
                tma_load_4d(sKV + slot * C::TILE_BYTES + c * C::CHUNK_BYTES, m,
                            &kv_full[slot], c * 64, un.row0 + j * C::BN, h, b);
              issued = u + 1;
            }
            // Halfway through a unit, the next unit's Q tiles and its first
            // two K/V blocks are pulled into L2 (its first loads are HBM
            // misses otherwise: Q is read by this CTA alone, and the K/V of
            // a new (b, h) are not in L2 yet), so the unit boundary does not
            // wait on HBM latency.
            if (j == nblk / 2 && unit + (int)gridDim.x < p.units) {
              const Unit nx = decode(unit + gridDim.x);
              for (int t = 0; t < 2; t++)
                for (int c = 0; c < C::NCHUNK; c++) {
                  tma_prefetch_l2_4d(&tmQ, c * 64, nx.row0 + nx.q0 + t * C::BM, nx.h, nx.b);
                  if (t * C::BN < nx.sk) {
                    tma_prefetch_l2_4d(&tmK, c * 64, nx.row0 + t * C::BN, nx.h, nx.b);
                    tma_prefetch_l2_4d(&tmV, c * 64, nx.row0 + t * C::BN, nx.h, nx.b);
                  }
                }
            }
          }
          jb += nblk;
        }
        if (!ok) {
          // Abort path: let every armed copy land before the CTA exits.
          if (kq > 0) mbar_wait_raw(q_full, (kq - 1) & 1, 100000000ull);
          for (int u = issued - C::NST < 0 ? 0 : issued - C::NST; u < issued; u++)
            mbar_wait_raw(&kv_full[u % C::NST], (u / C::NST) & 1, 100000000ull);
        }
      }
    } else if (warp == 9) {
      // -------------------------------------------------------- MMA issuer
      // The whole warp runs the loop (so descriptors stay warp-uniform); one
      // elected lane issues each MMA and commit.
      constexpr uint32_t IDESC_S = idesc_f16_f32(128, C::BN, 0);
      constexpr uint32_t IDESC_O = idesc_f16_f32(128, D, 1);
      const uint32_t sQa = smem_u32(sQ), sKVa = smem_u32(sKV);
      auto issue_s = [&](int t, int slot) {
        const uint32_t qa = sQa + t * C::TILE_BYTES;
        const uint32_t ka = sKVa + slot * C::TILE_BYTES;
#pragma unroll
        for (int kk = 0; kk < D / 16; kk++) {
          const uint32_t off = (kk >> 2) * C::CHUNK_BYTES + (kk & 3) * 32;
          if (elect_one())
            mma_ss(tmem + t * 128, sdesc_sw128(qa + off, 16, 1024),
                   sdesc_sw128(ka + off, 16, 1024), IDESC_S, kk > 0);
        }
      };
      // O_t (+)= P_t V for the keys of one half of the block (64 keys, four
      // K=16 steps), as soon as the softmax has written that half of P.
      auto issue_o_half = [&](int t, int slot, int half, bool acc) {
        const uint32_t va = sKVa + slot * C::TILE_BYTES;
#pragma unroll
        for (int kk = 0; kk < C::BN / 32; kk++) {
          const int ks = half * (C::BN / 32) + kk;
          if (elect_one())
            mma_ts(tmem + C::O_COL + t * D, tmem + t * 128 + ks * 8,
                   sdesc_sw128(va + ks * 2048, C::CHUNK_BYTES, 1024), IDESC_O,
                   (acc || ks > 0) ? 1u : 0u);
        }
      };
      auto issue_o = [&](int t, int slot, bool acc, uint32_t parity, int tl) {
        for (int half = 0; half < 2; half++) {
          if (!mbar_wait(&p_half[2 * t + half], parity, abort_flag)) return false;
          tc_fence_after();
          if (tl >= 0 && lane == 0) LLMR_TLC(tl + 2 * t + half);
          issue_o_half(t, slot, half, acc);
        }
        return true;
      };
      bool ok = true;
      int jb = 0;  // key blocks of this CTA's earlier units
      for (int unit = blockIdx.x, k = 0; unit < p.units && ok; unit += gridDim.x, k++) {
        const int nblk = decode(unit).nblk;
        const int ub = 2 * jb;  // K/V ring position of this unit's K_0
        ok = mbar_wait(q_full, k & 1, abort_flag);
        if (ok) ok = mbar_wait(&kv_full[ub % C::NST], (ub / C::NST) & 1, abort_flag);
        if (!ok) break;
        // S_t of block 0 overwrites P_t of the previous unit's last block:
        // the PV MMAs that read it were issued earlier and run first.
        tc_fence_after();
        issue_s(0, ub % C::NST);
        if (elect_one()) mma_commit(&s_full[0]);
        issue_s(1, ub % C::NST);
        if (elect_one()) mma_commit(&s_full[1]);
        if (elect_one()) mma_commit(&kv_empty[ub % C::NST]);
        if (nblk == 1 && elect_one()) mma_commit(q_empty);
        for (int j = 0; j < nblk; j++) {
          const int jj = jb + j;
          const int uV = 2 * jj + 1, sV = uV % C::NST;
          const int uK = 2 * jj + 2, sK = uK % C::NST;
          const bool more = j + 1 < nblk;
          const int tl = (k == 1 && j >= 4 && j < 12) ? 96 + 4 * (j - 4) : -1;
          if (!(ok = mbar_wait(&kv_full[sV], (uV / C::NST) & 1, abort_flag))) break;
          // O_t is overwritten by this unit's first PV: the previous unit's
          // epilogue must have read it.
          if (j == 0 && k > 0 && !(ok = mbar_wait(&o_empty[0], (k - 1) & 1, abort_flag))) break;
          if (!(ok = issue_o(0, sV, j > 0, jj & 1, tl))) break;
          if (more) {
            if (!(ok = mbar_wait(&kv_full[sK], (uK / C::NST) & 1, abort_flag))) break;
            tc_fence_after();
            issue_s(0, sK);
            if (elect_one()) mma_commit(&s_full[0]);
          } else {
            if (elect_one()) mma_commit(&o_full[0]);
          }
          if (j == 0 && k > 0 && !(ok = mbar_wait(&o_empty[1], (k - 1) & 1, abort_flag))) break;
          if (!(ok = issue_o(1, sV, j > 0, jj & 1, tl))) break;
          if (elect_one()) mma_commit(&kv_empty[sV]);
          if (more) {
            issue_s(1, sK);
            if (elect_one()) mma_commit(&s_full[1]);
            if (elect_one()) mma_commit(&kv_empty[sK]);
            // The unit's last S MMAs are issued: Q may be replaced after them.
            if (j + 2 == nblk && elect_one()) mma_commit(q_empty);
          } else {
            if (elect_one()) mma_commit(&o_full[1]);
          }
        }
        jb += nblk;
      }
      // Drain: every MMA this warp issued has completed before TMEM is
      // released at the end of the kernel.
      if (elect_one()) mma_commit(drain);
      mbar_wait_raw(drain, 0, 100000000ull);
    } else if constexpr (FUSED) {
      // ------------------------------------------- fused prologue, background
      // The warp's pieces, in order: its 4 pieces of Q' of unit 1 of this
      // CTA, its share of the remaining K'/V' pieces (ordered by (b, h), so
      // the pairs the next rounds need come first), its 4 pieces of Q' of
      // each later unit. Every lane prefetches its own 16-byte parts of the
      // next steps (4 rows each) into the warp's shared-memory ring and reads
      // back only what it copied itself.
      constexpr int E = D / kProLanesPerRow;
      constexpr int VIN = 16 / sizeof(In);
      constexpr int CH = E / VIN;
      constexpr int STEP = 32 * CH * 16;  // bytes of one step (4 rows)
      constexpr int NSTG = C::BG_RING / STEP > 16 ? 16 : C::BG_RING / STEP;
      const int G = gridDim.x, wb = warp - 10;
      const int sub = lane & (kProLanesPerRow - 1), r = lane / kProLanesPerRow;
      uint8_t *ring_p = smem + C::BG_OFF + wb * C::BG_RING;
      const uint32_t ring = smem_u32(ring_p);
      const int my_units = ((int)blockIdx.x < p.units) ? (p.units - (int)blockIdx.x + G - 1) / G : 0;
      const int nq1 = my_units > 1 ? 4 : 0;
      const int pairs = p.units > 0 ? (p.units - 1) / p.nqt + 1 : 0;
      const int kv_all = pairs * 2 * fp.nrb;
      const int kv0 = fp.startup_bh * 2 * fp.nrb + wb * G + (int)blockIdx.x;
      const int nkv = kv0 < kv_all ? (kv_all - kv0 + 2 * G - 1) / (2 * G) : 0;
      const int nqk = my_units > 2 ? 4 * (my_units - 2) : 0;
      const int nsteps = 8 * (nq1 + nkv + nqk);
      // Piece pi -> (t, b, h, first row, unit k or -1 for K'/V', index j).
      struct Pc {
        int t, b, h, s0, k, j;  // j: the piece's index among the warp's 4 of unit k
      };
      auto piece = [&](int pi) {
        Pc c;
        int k = -1, j = 0;
        if (pi < nq1) {
          k = 1;
          j = pi;
        } else if (pi >= nq1 + nkv) {
          const int rest = pi - nq1 - nkv;
          k = 2 + rest / 4;
          j = rest - (rest / 4) * 4;
        }
        if (k >= 0) {
          const Unit un = decode(blockIdx.x + k * G);
          c.t = 0;
          c.b = un.b;
          c.h = un.h;
          c.s0 = un.q0 + (wb * 4 + j) * 32;
        } else {
          const int4 kp = kv_piece(kv0 + (pi - nq1) * 2 * G);
          c.b = kp.x / p.H;
          c.h = kp.x - c.b * p.H;
          c.t = kp.y;
          c.s0 = kp.z * 32;
        }
        c.k = k;
        c.j = j;
        return c;
      };
      auto issue = [&](int g) {
        const Pc c = piece(g >> 3);
        const int s = c.s0 + (g & 7) * kProRowsPerWarpStep + r;
        const ViewSel<In> v(vq, vk, vv, c.t);
        const bool in = s < p.S;
        const In *src = v.base + (long long)c.b * v.bs + (long long)(in ? s : 0) * v.rs +
                        (long long)c.h * v.hs + sub * E;
        const uint32_t dst = ring + (uint32_t)((g % NSTG) * STEP) + (uint32_t)lane * 16u;
#pragma unroll
        for (int cc = 0; cc < CH; cc++) cp_async16(dst + cc * 512u, src + cc * VIN, in ? 16u : 0u);
      };
#pragma unroll 1
      for (int g = 0; g < NSTG - 1; g++) {
        if (g < nsteps) issue(g);
        cp_async_commit();
      }
#pragma unroll 1
      for (int g = 0; g < nsteps; g++) {
        if ((g & 7) == 0 && *abort_flag) break;
        if (g + NSTG - 1 < nsteps) issue(g + NSTG - 1);
        cp_async_commit();
        cp_async_wait<NSTG - 1>();  // this lane's parts of step g have landed
        const Pc c = piece(g >> 3);
        const int s = c.s0 + (g & 7) * kProRowsPerWarpStep + r;
        const bool in = s < p.S;
        float x[E];
        const uint8_t *part = ring_p + (g % NSTG) * STEP + lane * 16;
#pragma unroll
        for (int cc = 0; cc < CH; cc++) {
          const Pack<In, VIN> pk = *reinterpret_cast<const Pack<In, VIN> *>(part + cc * 512);
#pragma unroll
          for (int e = 0; e < VIN; e++) x[cc * VIN + e] = in ? to_f32<In>(pk.v[e]) : 0.0f;
        }
        pro_row_finish<D>(x, fp.pp, c.t, s, sub, pro_dst<D>(fp.ws, fp.pp, c.t, c.b, c.h, in ? s : 0, sub));
        if ((g & 7) == 7) {  // piece complete
          if (c.k < 0) {
            publish(c.b * p.H + c.h);
            if ((g >> 3) == nq1 + nkv - 1 && warp == 10 && lane == 0) LLMR_TL(19);
          } else if (c.j == 3) {  // the warp's last Q' piece of unit k
            fence_proxy_async_global();
            __threadfence();
            __syncwarp();
            if (lane == 0) q_done[wb] = c.k;
            if (c.k == 1 && warp == 10 && lane == 0) LLMR_TL(18);
          }
        }
      }
      cp_async_wait<0>();
      if (warp == 10 && lane == 0) LLMR_TL(20);
    }
  } else {
    reg_alloc<C::REG_SOFTMAX>();
    // ------------------------------------------------------------- softmax
    const int t = warp >> 2;                  // query tile 0 or 1
    const int row = threadIdx.x & 127;        // row within the tile = TMEM lane
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + lane_off + t * 128;
    const uint32_t tO = tmem + lane_off + C::O_COL + t * D;
    const float sl2 = p.scale_log2;
    bool ok = true;
    int jb = 0;  // key blocks of this CTA's earlier units
    for (int unit = blockIdx.x, k = 0; unit < p.units && ok; unit += gridDim.x, k++) {
      const Unit un = decode(unit);
      const int b = un.b, h = un.h, nblk = un.nblk;
      const int bh = b * p.H + h;
      float m_used = -INFINITY;  // log2-domain max the P values are relative to
      float l = 0.0f;
      for (int j = 0; j < nblk; j++) {
        const int jj = jb + j;
        ok = __all_sync(0xffffffffu, mbar_wait(&s_full[t], jj & 1, abort_flag));
        if (!ok) break;
        if (j == 0 && k < 4 && threadIdx.x == 0) LLMR_TL(10 + 2 * k);
        if (j == 1 && k < 3 && threadIdx.x == 0) LLMR_TL(29 + k);
        const bool tl_blk = k == 1 && j >= 4 && j < 12 && row == 0;
        const int tl0 = 32 + 32 * t + 4 * (j - 4);
        (void)tl0;  // read by the timeline stamps only
        if (tl_blk) LLMR_TLC(tl0);
        tc_fence_after();
        const int valid = un.sk - j * C::BN;  // keys of this block inside the sequence
        // Applies the key mask (keys past the sequence -> -inf) to chunk c.
        auto mask_chunk = [&](int c, float *v) {
          if (valid < C::BN) {
#pragma unroll
            for (int i = 0; i < 32; i++)
              if (c * 32 + i >= valid) v[i] = -INFINITY;
          }
        };
        // The whole row of raw scores, loaded in one TMEM round trip and kept
        // in registers until P is written.
        uint32_t sbuf[128];
#pragma unroll
        for (int c = 0; c < 4; c++) tmem_ld32(tS + c * 32, sbuf + c * 32);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 4; c++) reg_fence32(sbuf + c * 32);
        // Pass 1: the row max of this block's raw scores.
        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int c = 0; c < 4; c++) {
          float *v = reinterpret_cast<float *>(sbuf + c * 32);
          mask_chunk(c, v);
#pragma unroll
          for (int i = 0; i < 32; i += 2) mx[(i >> 1) & 3] = max3f(mx[(i >> 1) & 3], v[i], v[i + 1]);
        }
        // Lazy max: the max the P values are relative to moves only when this
        // block's row max passes it by more than kMaxExp (P would overflow
        // fp16), and on the first block; O and l are rescaled then.
        const float m_new = max3f(mx[0], mx[1], fmaxf(mx[2], mx[3])) * sl2;
        if (tl_blk) LLMR_TLC(tl0 + 1);
        const bool need = m_new > m_used + kMaxExp;  // always true on block 0
        if (__any_sync(0xffffffffu, need)) {
          const float m_tgt = need ? m_new : m_used;
          const float factor = ex2_approx(m_used - m_tgt);  // 0 on the first block
          l *= factor;
          if (j > 0) {
#pragma unroll 1
            for (int c = 0; c < D / 32; c++) {
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
        // Pass 2: P = 2^(s*scale*log2e - m_used) as fp16 over each chunk's
        // first 16 columns (chunk c's P lands in columns [16c, 16c+16), whose
        // scores are already in registers). A share of the exponential pairs
        // runs on the FMA pipe. Each half of P (keys 0-63, then 64-127) is
        // handed to the MMA warp as soon as it is in TMEM.
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
            if ((kExp2EmuMask >> i) & 1u)  // this pair's exponentials on the FMA pipe
              pp = exp2_poly_x2(f2_pack(fmaxf(x.x, -125.0f), fmaxf(x.y, -125.0f)));
            else
              pp = f2_pack(ex2_approx(x.x), ex2_approx(x.y));
            part2[i & 1] = f2_add(part2[i & 1], pp);
            const float2 pf = f2_unpack(pp);
            pk[i] = pack_f16x2(pf.x, pf.y);
          }
          tmem_st16(tS + c * 16, pk);
          // Keys 0-63 are handed over after chunk kHalf0At's stores (1: as
          // soon as they are written; 2: one chunk later, so the warp does not
          // stall on the store round trip in mid-row), keys 64-127 at the end.
          if (c == kHalf0At || c == 3) {
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_half[2 * t + (c == 3 ? 1 : 0)]);
            if (tl_blk) LLMR_TLC(tl0 + 2 + (c == 3 ? 1 : 0));
          }
        }
        const float2 s0 = f2_unpack(part2[0]), s1 = f2_unpack(part2[1]);
        l += (s0.x + s0.y) + (s1.x + s1.y);
      }
      jb += nblk;
      if (!ok) break;
      // ------------------------------------------------------- epilogue
      if (k < 3 && threadIdx.x == 0) LLMR_TL(23 + k);
      ok = __all_sync(0xffffffffu, mbar_wait(&o_full[t], k & 1, abort_flag));
      if (k < 3 && threadIdx.x == 0) LLMR_TL(26 + k);
      if (!ok) break;
      tc_fence_after();
      const int qloc = un.q0 + t * C::BM + row;  // query within its sequence
      const bool qin = qloc < un.sq;
      const int qrow = un.row0 + qloc;            // row in the maps / output
      OutT *dst = reinterpret_cast<OutT *>(p.o) + (long long)b * p.o_batch_stride +
                  (long long)qrow * p.o_row_stride + (long long)h * D;
      const float lse_t = (m_used + log2f(l)) * 0.69314718055994531f;
      // o = a * prev + c * acc: a = 0, c = 1/l normally; with merge, the
      // log-sum-exp weights of the previous partial result (over other
      // keys, read from o and lse in place) and of this one.
      float ca = 0.0f, ct = 1.0f / l, lse_out = lse_t;
      constexpr bool kCanMerge = std::is_same<OutT, float>::value;
      const bool merge = kCanMerge && p.merge && qin;
      if (merge) {
        const float la = p.lse[(long long)bh * S + qrow];
        const float mx2 = fmaxf(la, lse_t);
        const float wa = expf(la - mx2), wt = expf(lse_t - mx2);
        const float inv = 1.0f / (wa + wt);
        ca = wa * inv;
        ct = wt * inv / l;
        lse_out = mx2 + logf(wa + wt);
      }
      // The choice must be warp-uniform (the staged path's TMEM loads and
      // shuffles are warp-collective): it depends on the launch, not the row.
      if (!FUSED && !(kCanMerge && p.merge)) {
        // Coalesced stores through shared memory: each round, every lane puts
        // 128 bytes of its row (64 columns of 16-bit output, 32 of fp32) into
        // the warp's staging block (16-byte pieces XOR-swizzled by row), then
        // the warp writes 4 whole 128-byte row segments per store instruction.
        constexpr int CPR = 128 / (int)sizeof(OutT);  // columns per round
        uint8_t *stg = smem + C::EPI_OFF + warp * 4096;
        const int rbase = un.q0 + t * C::BM + (warp & 3) * 32;  // the warp's first row
#pragma unroll
        for (int rnd = 0; rnd < D / CPR; rnd++) {
#pragma unroll
          for (int cc = 0; cc < CPR / 32; cc++) {
            const int c = rnd * (CPR / 32) + cc;
            uint32_t o[32];
            tmem_ld32(tO + c * 32, o);
            tmem_wait_ld();
            reg_fence32(o);
            if (c == D / 32 - 1) {
              // O_t is read out: the next unit's first PV may overwrite it.
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&o_empty[t]);
            }
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; i++) v[i] = __uint_as_float(o[i]) * ct;
            // 32 columns = 32 * sizeof(OutT) bytes = 2 or 8 pieces of 16 bytes
            constexpr int PIECES = 32 * (int)sizeof(OutT) / 16;
            alignas(16) OutT pk[32];
#pragma unroll
            for (int i = 0; i < 32; i++) pk[i] = from_f32<OutT>(v[i]);
#pragma unroll
            for (int pc = 0; pc < PIECES; pc++) {
              const int piece = cc * PIECES + pc;
              *reinterpret_cast<uint4 *>(stg + lane * 128 + ((piece ^ (lane & 7)) << 4)) =
                  reinterpret_cast<const uint4 *>(pk)[pc];
            }
          }
          __syncwarp();
#pragma unroll
          for (int it = 0; it < 8; it++) {
            const int pid = it * 32 + lane, r = pid >> 3, part = pid & 7;
            const uint4 val = *reinterpret_cast<const uint4 *>(stg + r * 128 + ((part ^ (r & 7)) << 4));
            const int rloc = rbase + r;  // query within its sequence
            if (rloc < un.sq) {
              OutT *d = reinterpret_cast<OutT *>(p.o) + (long long)b * p.o_batch_stride +
                        (long long)(un.row0 + rloc) * p.o_row_stride + (long long)h * D +
                        rnd * CPR + part * (16 / (int)sizeof(OutT));
              *reinterpret_cast<uint4 *>(d) = val;
            }
          }
          __syncwarp();
        }
      } else {
#pragma unroll
      for (int c = 0; c < D / 32; c++) {
        uint32_t o[32];
        tmem_ld32(tO + c * 32, o);
        tmem_wait_ld();
        reg_fence32(o);
        if (c == D / 32 - 1) {
          // O_t is read out: the next unit's first PV may overwrite it.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&o_empty[t]);
        }
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; i++) v[i] = __uint_as_float(o[i]) * ct;
        if constexpr (kCanMerge) {
          if (merge) {
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
              const float4 pv = *reinterpret_cast<const float4 *>(dst + c * 32 + i);
              v[i] = fmaf(pv.x, ca, v[i]);
              v[i + 1] = fmaf(pv.y, ca, v[i + 1]);
              v[i + 2] = fmaf(pv.z, ca, v[i + 2]);
              v[i + 3] = fmaf(pv.w, ca, v[i + 3]);
            }
          }
        }
        if (qin) store_row_chunk<OutT>(dst + c * 32, v);
      }
      }
      if (p.lse != nullptr && qin) p.lse[(long long)bh * S + qrow] = lse_out;
      if (k < 4 && threadIdx.x == 0) LLMR_TL(11 + 2 * k);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicExch(p.err, 1);
  if (threadIdx.x == 0) LLMR_TL(21);
  if constexpr (FUSED) {
    // Every wait of this CTA on the piece counters is over. The last CTA to
    // get here clears the counters for the next launch.
    __shared__ int last_cta;
    if (threadIdx.x == 0) {
      __threadfence();
      last_cta = atomicAdd(fp.sync, 1) == (int)gridDim.x - 1;
    }
    __syncthreads();
    if (last_cta) {
      const int pairs = p.units > 0 ? (p.units - 1) / p.nqt + 1 : 0;
      for (int i = threadIdx.x; i < pairs; i += blockDim.x) fp.sync[1 + i] = 0;
      __syncthreads();
      if (threadIdx.x == 0) {
        fp.sync[0] = 0;
        __threadfence();
      }
    }
  }
}

}  // namespace llmr
