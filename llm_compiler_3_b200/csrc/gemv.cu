// Decode GEMV for one or two tokens, sm_100a: y[b, n] = sum_k W[n, k] x[b, k]
// on CUDA cores with FP32 accumulation, plus the same fused epilogues as the
// tensor-core projection (proj.cu).
//
// At batch 1-2 a projection is a pure weight stream (2 bytes per FMA), so the
// tensor-core path's machinery -- TMEM accumulators, split-K partials, cluster
// reductions -- is overhead.  Here the weight rows are cut into 16-row groups:
// in every 16 KB panel (128 rows x 64 columns, the layout pack_weight writes) a
// group's rows are one contiguous 2 KB slice.  With enough groups the grid
// is one wave of persistent CTAs, each walking a balanced share of the groups
// (no split-K); with few, K is split over a thread-block cluster and the
// members' sums meet in member 0's shared memory.  In every CTA one
// producer warp streams the slices with bulk copies, four panels (8 KB) per
// ring stage, the ring as deep as shared memory allows (launch_gemv trades
// CTAs per SM against stages for the most bytes in flight).  Each of
// four consumer warps takes one panel of a stage: the group's 16 rows are
// exactly the M of mma.sync m16n8k16 (A fetched with ldmatrix from the
// swizzled slice, the one or two tokens in N = 8, FP32 accumulators), which
// costs ~10x fewer instructions per byte than FMA-ing converted halves.  At
// the end of a group the four warps' partial sums are added in a fixed order
// and eight threads per row run the epilogue; a row's RoPE / SwiGLU partner
// (the adjacent row in the packed order) is eight lanes away.
//
// Replaces, like proj.cu, the NPU matmul lowering
// (lib/Transforms/HardwareOps.cpp:105-155, lib/Transforms/Emit.cpp:348-378)
// with FP16 operands and FP32 accumulation (lib/Transforms/Normalize.cpp:123-192).
#include <math.h>

#include <algorithm>

#include "common.cuh"
#include "gemv.cuh"
#include "host.hpp"
#include "proj.cuh"

namespace npu_b200 {
namespace {

using namespace gemv;

template <int BT, int KIND>
__global__ void __launch_bounds__(kGemvThreads)
    gemv_kernel(const uint8_t* __restrict__ w_packed, const __half* __restrict__ x,
                const __grid_constant__ EpiParams ep, int k, int kblocks, int n_groups,
                int stages, int split) {
  // split == 1: persistent CTAs walking groups blockIdx.x, + gridDim.x, ...
  // split > 1: a cluster of `split` CTAs per group, member r taking the r-th
  // share of the K stages; the members' sums meet in member 0's shared memory.
  const int kstages_all = (kblocks + kPanelsPerStage - 1) / kPanelsPerStage;
  const int crank = split > 1 ? static_cast<int>(blockIdx.x % split) : 0;
  const int ks_begin = split > 1 ? crank * kstages_all / split : 0;
  const int ks_end = split > 1 ? (crank + 1) * kstages_all / split : kstages_all;
  const int kstages = ks_end - ks_begin;
  const int kx0 = ks_begin * kPanelsPerStage * 64;                   // first column staged
  const int kx = min(k, ks_end * kPanelsPerStage * 64) - kx0;        // columns staged
  // Row stride of the staged activations: the largest member's share, so the
  // shared-memory layout is the same in every member of a cluster (the
  // members address member 0's barrier and sums by their own offsets).
  const int kx_ld = split > 1
                        ? min(k, (kstages_all + split - 1) / split * kPanelsPerStage * 64)
                        : k;
  const int g_first = split > 1 ? static_cast<int>(blockIdx.x / split) : static_cast<int>(blockIdx.x);
  const int g_step = split > 1 ? n_groups : static_cast<int>(gridDim.x);

  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* ring = smem;
  __half* xs = reinterpret_cast<__half*>(ring + stages * kStageBytes);  // [BT][kx_ld]
  uint64_t* full = reinterpret_cast<uint64_t*>(xs + BT * kx_ld);
  uint64_t* empty = full + kMaxStages;
  uint64_t* cl_bar = empty + kMaxStages;                           // member 0: others' sums landed
  float* cl_part = reinterpret_cast<float*>(cl_bar + 1);           // [8 members][16 rows][2]
  float* part_sum = cl_part + 8 * kRows * 2;                       // [4 warps][16 rows][2]
  float* red = part_sum + 4 * kRows * 2;                           // [4 warps][BT]
  int* red_id = reinterpret_cast<int*>(red + 4 * BT);             // [4 warps][BT]
  float* rn = reinterpret_cast<float*>(red_id + 4 * BT);          // [BT] RMSNorm scale
  int* pos_s = reinterpret_cast<int*>(rn + BT);                   // [BT] positions
  volatile int* abort_flag = pos_s + BT;

  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;

  pdl_launch_dependents();
  if (t == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumers / 32);
    }
    mbar_init(cl_bar, split > 1 ? split - 1 : 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (split > 1) cluster_sync_all();  // member 0's barrier is initialised before anyone arrives

  if (warp == kConsumers / 32) {
    // Producer: the weights never depend on the previous kernel, so it streams
    // without waiting for it.
    if (lane != 0) return;
    const uint64_t pol = policy_evict_first();
    int it = 0, slot = 0;
    uint32_t phase = 0;  // phase of the current pass over the ring
    bool ok = true;
    for (int g = g_first; g < n_groups && ok; g += g_step) {
      const int row0 = g * kRows;
      const uint8_t* base =
          w_packed + static_cast<size_t>(row0 >> 7) * kblocks * 16384 + (row0 & 127) * 128;
      for (int ks = ks_begin; ks < ks_end; ++ks, ++it) {
        if (!wait_or_abort(&empty[slot], phase ^ 1, abort_flag) || *abort_flag) {
          ok = false;
          break;
        }
        const int kb0 = ks * kPanelsPerStage;
        const int nk = min(kPanelsPerStage, kblocks - kb0);
        mbar_arrive_expect_tx(&full[slot], nk * kSlice);
        for (int j = 0; j < nk; ++j)
          bulk_load_hint(ring + slot * kStageBytes + j * kSlice,
                         base + static_cast<size_t>(kb0 + j) * 16384, kSlice, &full[slot], pol);
        if (++slot == stages) {
          slot = 0;
          phase ^= 1;
        }
      }
    }
    if (!ok)  // the CTA may not exit with copies still landing in its ring
      for (int i = max(0, it - stages); i < it; ++i)
        mbar_wait(&full[i % stages], (i / stages) & 1, kDevErrTmaTimeout);
    return;
  }

  // Consumers: activations, RMSNorm scale and positions of this step.
  pdl_wait();
  for (int b = 0; b < BT; ++b) {
    const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<size_t>(b) * k + kx0);
    uint4* dst = reinterpret_cast<uint4*>(xs + b * kx_ld);
    for (int i = t; i < kx / 8; i += kConsumers) dst[i] = src[i];
  }
#pragma unroll
  for (int b = 0; b < BT; ++b) {
    float s = 0.f;
    if (ep.ssq_in != nullptr && b < ep.batch)
      for (int p = t; p < ep.ssq_parts; p += kConsumers)
        s += ep.ssq_in[static_cast<size_t>(p) * ep.ssq_ld + b];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) red[warp * BT + b] = s;
  }
  consumer_sync();
  if (t < BT) {
    const float s = red[t] + red[BT + t] + red[2 * BT + t] + red[3 * BT + t];
    rn[t] = (ep.ssq_in != nullptr && t < ep.batch) ? rsqrtf(s * ep.ssq_inv_hidden + ep.ssq_eps) : 1.f;
    pos_s[t] = (ep.positions != nullptr && t < ep.batch) ? ep.positions[t] : 0;
  }
  consumer_sync();

  const int row = t / kParts, part = t % kParts;
  const bool lead = part == 0;  // one thread per row writes
  int slot = 0;
  uint32_t phase = 0;
  for (int g = g_first; g < n_groups; g += g_step) {
    // One accumulator per k-step of a panel: four independent MMA chains.
    float c[4][4];
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) c[kk][0] = c[kk][1] = c[kk][2] = c[kk][3] = 0.f;
    bool bad = false;
    for (int ks = 0; ks < kstages; ++ks) {
      if (!bad && !wait_or_abort(&full[slot], phase, abort_flag)) {
        bad = true;
        *abort_flag = 1;
      }
      const int kb = (ks_begin + ks) * kPanelsPerStage + warp;  // this warp's panel
      if (!bad && kb < kblocks) {
        mma_panel<BT>(c, smem_u32(ring + slot * kStageBytes + warp * kSlice), xs + (kb * 64 - kx0),
                      kx_ld);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
      if (++slot == stages) {
        slot = 0;
        phase ^= 1;
      }
    }
    if (consumer_sync_or(bad)) {
      // Member 0 stays until every other member has arrived (they write into it).
      if (split > 1 && crank == 0 && t == 0)
        for (uint32_t i = 0; i < kMaxPolls && !mbar_try_wait_cluster(cl_bar, 0); ++i) {
        }
      return;
    }

    float acc[BT];
    reduce_warps<BT>(c, part_sum, acc);
    if (split > 1) {
      if (crank != 0) {
        // Hand this member's sums to member 0 and leave.
        if (lead) {
          const uint32_t dst = cluster_map(smem_u32(cl_part + (crank * kRows + row) * 2), 0);
#pragma unroll
          for (int b = 0; b < BT; ++b) st_cluster_f32(dst + 4 * b, acc[b]);
        }
        consumer_sync();
        if (t == 0) mbar_arrive_cluster(cluster_map(smem_u32(cl_bar), 0));
        return;
      }
      // Member 0: the other members' sums, added in member order.
      bool landed = false;
      for (uint32_t i = 0; i < kMaxPolls && !landed; ++i) landed = mbar_try_wait_cluster(cl_bar, 0);
      if (!landed) {
        report_error(kDevErrTmaTimeout);
        return;
      }
#pragma unroll
      for (int b = 0; b < BT; ++b)
        for (int m = 1; m < split; ++m) acc[b] += cl_part[(m * kRows + row) * 2 + b];
    }
#pragma unroll
    for (int b = 0; b < BT; ++b) acc[b] *= rn[b];
    gemv_epilogue<BT, KIND>(ep, g, acc, pos_s, red, red_id);
  }
}

template <int BT>
size_t gemv_smem(int kx, int stages) {
  // ring + staged activations + full/empty/cluster barriers + member sums +
  // reduction scratch
  return static_cast<size_t>(stages) * kStageBytes + static_cast<size_t>(BT) * kx * 2 +
         (2 * kMaxStages + 1) * 8 +
         (8 * kRows * 2 + 4 * kRows * 2 + 4 * BT + 4 * BT + BT + BT + 1) * 4 + 64;
}

struct GemvLaunch {
  int grid = 0, stages = 0, split = 1;
};

// Enough groups to fill every SM twice: one wave of persistent CTAs.  For 1-4
// CTAs per SM take the deepest ring that fits and spread the groups so every
// CTA walks the same number (+-1); keep the choice with the most bytes in
// flight up to 12 MB (about where bulk streams saturate HBM), then the most
// CTAs, then the deepest ring.  Fewer groups: split K over clusters of 2-8
// CTAs until there are two CTAs per SM or the K shares get short.
template <int BT>
GemvLaunch choose_launch(int n_rows, int k) {
  const int n_groups = n_rows / kRows;
  const int kstages = (k / 64 + kPanelsPerStage - 1) / kPanelsPerStage;
  const int sms = sm_count();
  GemvLaunch best;
  int split = 1;
  // Double while that leaves at least 2 stages per member (splitting short K
  // only adds the reduction).
  while (split < 8 && n_groups * split < 2 * sms && kstages >= 4 * split) split *= 2;
  if (split > 1) {
    const int grid = n_groups * split;
    const int kx = std::min(k, (kstages + split - 1) / split * kPanelsPerStage * 64);
    const int per_sm = std::min(4, (grid + sms - 1) / sms);
    const long long avail = kGemvSmemPerSm / per_sm - kGemvSmemReserved -
                            static_cast<long long>(gemv_smem<BT>(kx, 0));
    const int slice = (kstages + split - 1) / split;
    best.grid = grid;
    best.split = split;
    best.stages = static_cast<int>(std::min<long long>({kMaxStages, slice, avail / kStageBytes}));
    if (best.stages >= 1) return best;
    best = GemvLaunch();
  }
  const size_t fixed = gemv_smem<BT>(k, 0);
  long long best_score = -1;
  for (int per_sm = 1; per_sm <= 4; ++per_sm) {
    const long long avail = kGemvSmemPerSm / per_sm - kGemvSmemReserved - static_cast<long long>(fixed);
    int stages = static_cast<int>(std::min<long long>(kMaxStages, avail / kStageBytes));
    if (stages < 4) break;
    const int slots = per_sm * sms;
    const int rounds = (n_groups + slots - 1) / slots;
    const int grid = (n_groups + rounds - 1) / rounds;
    // No deeper than the stages a CTA streams in all: shared memory it would
    // not fill only keeps the next kernel's CTAs from becoming resident early.
    stages = std::min(stages, std::max(4, rounds * kstages));
    const long long score =
        std::min<long long>(static_cast<long long>(grid) * stages * kStageBytes, 12ll << 20);
    if (score > best_score || (score == best_score && (grid > best.grid ||
                                                       (grid == best.grid && stages > best.stages)))) {
      best_score = score;
      best.grid = grid;
      best.stages = stages;
    }
  }
  return best;
}

template <int BT, int KIND>
int launch_gemv_kind(const void* w, const void* x, int n_rows, int k, const EpiParams& ep,
                     cudaStream_t stream, bool pdl) {
  const GemvLaunch g = choose_launch<BT>(n_rows, k);
  NPU_REQUIRE(g.grid > 0, "gemv: activations of K=%d leave no room for the ring", k);
  const int kstages = (k / 64 + kPanelsPerStage - 1) / kPanelsPerStage;
  const int kx = g.split > 1 ? std::min(k, (kstages + g.split - 1) / g.split * kPanelsPerStage * 64) : k;
  const size_t smem = gemv_smem<BT>(kx, g.stages);
  auto kern = gemv_kernel<BT, KIND>;
  // The limit is the function's, shared by the launches of every shape (and
  // by graph nodes a profiler relaunches after the capture): set it to the
  // most any launch may use, never to this launch's size.
  constexpr int kSmemLimit = kGemvSmemPerSm - kGemvSmemReserved;
  NPU_REQUIRE(smem <= static_cast<size_t>(kSmemLimit), "gemv: %zu bytes of shared memory", smem);
  NPU_TRY_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit));
  if (g.split > 1)
    NPU_TRY_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  LaunchCfg cfg;
  cfg.grid = dim3(g.grid);
  cfg.block = dim3(kGemvThreads);
  cfg.smem = smem;
  cfg.stream = stream;
  cfg.pdl = pdl;
  cfg.cluster = g.split;
  return launch(cfg, kern, static_cast<const uint8_t*>(w), static_cast<const __half*>(x), ep, k,
                k / 64, n_rows / kRows, g.stages, g.split);
}

template <int BT>
int launch_gemv(const void* w, const void* x, int n_rows, int k, const EpiParams& ep,
                cudaStream_t stream, bool pdl) {
  const bool peer = ep.px.seq >= 0;
  switch (ep.kind) {
    case kEpiStore:
      return peer ? launch_gemv_kind<BT, kGemvStorePeer>(w, x, n_rows, k, ep, stream, pdl)
                  : launch_gemv_kind<BT, kEpiStore>(w, x, n_rows, k, ep, stream, pdl);
    case kEpiResid:
      return peer ? launch_gemv_kind<BT, kGemvResidPeer>(w, x, n_rows, k, ep, stream, pdl)
                  : launch_gemv_kind<BT, kEpiResid>(w, x, n_rows, k, ep, stream, pdl);
    case kEpiSwiGLU:
      return launch_gemv_kind<BT, kEpiSwiGLU>(w, x, n_rows, k, ep, stream, pdl);
    case kEpiQKV:
      return launch_gemv_kind<BT, kEpiQKV>(w, x, n_rows, k, ep, stream, pdl);
    case kEpiArgmax:
      return launch_gemv_kind<BT, kEpiArgmax>(w, x, n_rows, k, ep, stream, pdl);
    default:
      NPU_REQUIRE(false, "gemv: unknown epilogue kind %d", ep.kind);
  }
  return NPU_B200_E_INVALID;
}

}  // namespace

bool gemv_supported(int n_rows, int k, int batch, const EpiParams& ep) {
  if (batch < 1 || batch > 2 || n_rows < kRows || n_rows % kRows != 0 || k < 64 || k % 64 != 0)
    return false;
  if (static_cast<size_t>(batch) * k * 2 > 64 * 1024) return false;  // staged activations
  if (ep.kind == kEpiQKV && (ep.q_norm_w != nullptr || ep.k_norm_w != nullptr)) return false;
  if (ep.kind == kEpiResid && ep.ssq_out_rows != kRows) return false;
  if (ep.kind == kEpiArgmax && ep.am_rows != kRows) return false;
  return true;
}

int gemv_run(const void* w_packed, const void* x, int n_rows, int k, int batch, const EpiParams& ep,
             cudaStream_t stream, bool pdl) {
  NPU_REQUIRE(gemv_supported(n_rows, k, batch, ep), "gemv: unsupported shape or epilogue");
  NPU_REQUIRE((reinterpret_cast<uintptr_t>(x) & 15) == 0, "gemv: x must be 16-byte aligned");
  return batch == 1 ? launch_gemv<1>(w_packed, x, n_rows, k, ep, stream, pdl)
                    : launch_gemv<2>(w_packed, x, n_rows, k, ep, stream, pdl);
}

}  // namespace npu_b200
