// mma_rate: clock cycles of tcgen05.mma kind::f16 groups in the operand
// shapes the attention kernels issue, one CTA (or CTA pair) per SM, so the
// attention kernel's tensor-pipe time per key block can be set against what
// the hardware delivers for those shapes rather than against the dense peak
// of a large GEMM.
//
// A group is one M x N x 128 product issued as 8 K=16 instructions (K = the
// head dimension for S = Q K^T, 128 keys for O += P V). Operands are zero
// (the rate does not depend on the values); shared memory holds SW128 tiles
// laid out exactly as the attention kernel's TMA maps leave them.
//   SS N=128  S = Q K^T of one 128-query tile and a 128-key block (fa_fwd_tc)
//   SS N=64   half of that key block
//   SS N=256  a 256-wide B operand (the shape of a large-GEMM tile)
//   TS N=128  O += P V with P in TMEM and V MN-major in shared memory
//   pair ...  the same on a CTA pair (cta_group::2, M = 256, B split)
// For each shape: `groups` = 1 (issue, commit, wait: latency) and 16 groups
// back to back before the commit (throughput). Printed: median cycles per
// group over the SMs, and the cycles the dense peak (8192 flop per clock
// per SM) would take.
//
// Build and run: make -C llm-runner_b200/csrc mma_rate && llm-runner_b200/mma_rate
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <vector>

#include "ptx.cuh"

using namespace llmr;

namespace {

constexpr int kTileA = 32768;         // 128 rows x 128 fp16 columns
constexpr int kTileB = 65536;         // up to 256 rows x 128 columns
constexpr int kSmem = 120 * 1024;     // > half an SM's shared memory: one CTA per SM
constexpr int kReps = 50;

enum Mode { kSS128, kSS64, kSS256, kTS128, kPairSS128, kPairSS256, kPairTS128, kModes };

struct Shape {
  const char *name;
  int n;       // N of the instruction (per pair for the pair modes)
  bool ts;     // A from TMEM
  bool pair;   // cta_group::2, M = 256
};
constexpr Shape kShapes[kModes] = {
    {"SS M=128 N=128", 128, false, false}, {"SS M=128 N=64", 64, false, false},
    {"SS M=128 N=256", 256, false, false}, {"TS M=128 N=128", 128, true, false},
    {"pair SS M=256 N=128", 128, false, true}, {"pair SS M=256 N=256", 256, false, true},
    {"pair TS M=256 N=128", 128, true, true}};

template <bool PAIR>
__global__ void __launch_bounds__(128, 1)
    mma_rate_kernel(int n, int ts, int groups, unsigned long long *cycles) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t *smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_slot;
  for (int i = threadIdx.x; i < (kTileA + kTileB) / 16; i += blockDim.x)
    reinterpret_cast<uint4 *>(smem)[i] = make_uint4(0, 0, 0, 0);
  fence_proxy_async_smem();
  const int warp = threadIdx.x >> 5;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    if (PAIR) {
      tmem_alloc_pair(&tmem_slot, 512);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(&tmem_slot, 512);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  if (warp == 0 && rank == 0) {
    const uint32_t a = smem_u32(smem), b = smem_u32(smem + kTileA);
    // B rows held by this CTA (the pair splits N), 128 bytes each, per
    // 64-column SW128 chunk.
    const uint32_t chunk_b = (uint32_t)(PAIR ? n / 2 : n) * 128u;
    const uint32_t idesc = idesc_f16_f32(PAIR ? 256 : 128, n, ts ? 1 : 0);
    const uint32_t bar_addr = PAIR ? mapa_shared(smem_u32(&bar), 0) : smem_u32(&bar);
    uint32_t phase = 0;
    unsigned long long t0 = 0;
    for (int r = 0; r <= kReps; r++) {
      if (r == 1) t0 = clock64();  // repetition 0 warms up
      for (int g = 0; g < groups; g++) {
#pragma unroll
        for (int kk = 0; kk < 8; kk++) {
          const uint32_t acc = (kk > 0 || g > 0) ? 1u : 0u;
          if (ts) {
            // A = P from TMEM columns 256.. (fp16 pairs), B = V MN-major.
            const uint64_t bd = sdesc_sw128(b + kk * 2048, 16384, 1024);
            if (elect_one()) {
              if (PAIR) mma_ts_pair(tmem, tmem + 256 + kk * 8, bd, idesc, acc);
              else mma_ts(tmem, tmem + 256 + kk * 8, bd, idesc, acc);
            }
          } else {
            const uint64_t ad = sdesc_sw128(a + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
            const uint64_t bd = sdesc_sw128(b + (kk >> 2) * chunk_b + (kk & 3) * 32, 16, 1024);
            if (elect_one()) {
              if (PAIR) mma_ss_pair(tmem, ad, bd, idesc, acc);
              else mma_ss(tmem, ad, bd, idesc, acc);
            }
          }
        }
      }
      if (elect_one()) {
        if (PAIR) mma_commit_pair(bar_addr);
        else mma_commit(&bar);
      }
      __syncwarp();
      mbar_wait_raw(&bar, phase, 1000000000ull);  // bounded: 1 s
      phase ^= 1;
    }
    if (threadIdx.x == 0) cycles[blockIdx.x / (PAIR ? 2 : 1)] = (clock64() - t0) / kReps;
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync();
  if (warp == 0) {
    tc_fence_after();
    if (PAIR) tmem_dealloc_pair(tmem, 512);
    else tmem_dealloc(tmem, 512);
  }
}

bool check(cudaError_t e, const char *what) {
  if (e == cudaSuccess) return true;
  fprintf(stderr, "%s: %s\n", what, cudaGetErrorString(e));
  return false;
}

}  // namespace

int main() {
  int nsm = 0;
  if (!check(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, 0), "device")) return 1;
  unsigned long long *d_cycles = nullptr;
  if (!check(cudaMalloc(&d_cycles, nsm * sizeof(unsigned long long)), "malloc")) return 1;
  if (!check(cudaFuncSetAttribute(mma_rate_kernel<false>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem), "attr") ||
      !check(cudaFuncSetAttribute(mma_rate_kernel<true>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem), "attr"))
    return 1;
  std::vector<unsigned long long> h(nsm);
  printf("%-22s %6s %12s %12s %8s\n", "shape", "groups", "clk/group", "dense peak", "ratio");
  for (int mode = 0; mode < kModes; mode++) {
    const Shape sh = kShapes[mode];
    for (int groups : {1, 16}) {
      cudaLaunchConfig_t cfg = {};
      cfg.blockDim = dim3(128);
      cfg.dynamicSmemBytes = kSmem;
      cudaLaunchAttribute attr[1];
      int n = nsm;
      cudaError_t e;
      if (sh.pair) {
        n = nsm / 2;
        cfg.gridDim = dim3(2 * n);
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, mma_rate_kernel<true>, sh.n, (int)sh.ts, groups, d_cycles);
      } else {
        cfg.gridDim = dim3(n);
        e = cudaLaunchKernelEx(&cfg, mma_rate_kernel<false>, sh.n, (int)sh.ts, groups, d_cycles);
      }
      if (!check(e, "launch") || !check(cudaDeviceSynchronize(), sh.name)) return 1;
      if (!check(cudaMemcpy(h.data(), d_cycles, n * sizeof(unsigned long long),
                            cudaMemcpyDeviceToHost), "copy"))
        return 1;
      std::sort(h.begin(), h.begin() + n);
      // Per SM: 128 rows x N x 128 x 2 flop (the pair: N per SM as well).
      const double peak_clk = 128.0 * sh.n * 128 * 2 / 8192.0;
      const double med = (double)h[n / 2] / groups;
      printf("%-22s %6d %12.0f %12.0f %8.2f\n", sh.name, groups, med, peak_clk, peak_clk / med);
    }
  }
  cudaFree(d_cycles);
  return 0;
}
