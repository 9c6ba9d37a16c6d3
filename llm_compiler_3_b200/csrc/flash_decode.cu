// Split-KV flash-decoding attention for sm_100a.
//
// Semantics follow npu.attention as LLM_Compiler_3 defines it
// (include/npu/Dialect/NPUDialect.td:31-61, 147-189) and expands it
// (lib/Transforms/Attention.cpp:296-374): per query head, with the KV head the
// GQA group maps it to, t = scale * q.k, m = running max, p = exp(t - m),
// l = alpha*l + sum p, O = alpha*O + P.V, out = O / l.  Unlike the NPU (which
// rounds every VPU op to FP16, lib/Transforms/Emit.cpp:932-1024) the running
// max, sum and O stay in FP32 and the output is rounded once.
//
// Work decomposition (B200-first): one CTA per (key split, KV head, sequence).
// Each warp owns every WARPS-th 32-key tile of the CTA's key range and runs its
// own TMA ring of STAGES stages (K and V tiles, 128-byte swizzle), so warps
// never wait on each other while streaming.  Scores S^T = K Q^T and the update
// O^T += V^T P^T use m16n8k16 tensor-core MMAs with the grouped query heads as
// the N=8 columns: the whole GQA group shares one pass over K and V.  Warps
// merge in shared memory; splits merge in the last CTA to finish (counter per
// (sequence, KV head)), so one launch produces the final FP16 output.
#include <math.h>

#include <mutex>

#include "common.cuh"
#include "host.hpp"

namespace npu_b200 {
namespace {

constexpr int kKeysPerTile = 32;  // keys per warp stage
constexpr int kMaxGroup = 8;      // query heads per KV head (MMA N)
constexpr int kMaxSplits = 256;   // merge statistics of all splits fit in shared memory
// Split counters occupy a fixed region at the start of the workspace, whatever
// the batch, so one workspace serves every batch size.
constexpr int kMaxUnits = 16384;  // sequences x KV heads
constexpr size_t kCounterBytes = kMaxUnits * sizeof(uint32_t);

template <int D>
struct FdShape {
  static constexpr int kRegions = D / 64;                 // 128-byte swizzle regions per row
  static constexpr int kRegionBytes = kKeysPerTile * 128;  // one region of one tile
  static constexpr int kTileBytes = kKeysPerTile * D * 2;  // K (or V) of one tile
  static constexpr int kStageBytes = 2 * kTileBytes;       // K + V
  static constexpr int kPartFloats = kMaxGroup * D + 2 * kMaxGroup;  // O, m, l per split
};

__device__ __forceinline__ uint8_t* align_1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

template <int D, int WARPS, int STAGES>
__global__ void __launch_bounds__(WARPS * 32, 1)
    flash_decode_kernel(const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap, const __half* __restrict__ q,
                        const int32_t* __restrict__ seq_lens, __half* __restrict__ out,
                        float* __restrict__ part, uint32_t* __restrict__ counters, int q_heads,
                        int kv_heads, int max_seq, int keys_per_split, int num_splits,
                        float scale_log2, const int32_t* __restrict__ positions) {
  using S = FdShape<D>;
  constexpr int KSTEPS = D / 16;  // k-steps of the score MMA
  constexpr int DBLK = D / 16;    // 16-dim blocks of the PV MMA

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + WARPS * STAGES * S::kStageBytes);
  __shared__ int s_last;

  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int group = q_heads / kv_heads;

  uint8_t* my_stages = smem + warp * STAGES * S::kStageBytes;
  uint64_t* my_bars = bars + warp * STAGES;
  uint64_t* merge_bar = bars + WARPS * STAGES;  // bulk copy of the split partials
  if (lane == 0) {
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
    for (int s = 0; s < STAGES; ++s) mbar_init(&my_bars[s], 1);
    if (warp == 0) mbar_init(merge_bar, 1);
    fence_barrier_init();
  }
  __syncwarp();

  // The next kernel may be scheduled once every CTA of this grid is resident;
  // it waits for this grid's results itself.
  pdl_launch_dependents();
  // With `positions` (the step's own input, written before the step) the
  // attended length is positions[b] + 1 and is known before the previous
  // kernel (the KV append) finishes: key tiles that end before the new key
  // were written by earlier steps and are loaded before waiting for it.
  // Without, the length comes from seq_lens, which may be the previous
  // kernel's output.
  if (positions == nullptr) pdl_wait();
  int len = positions != nullptr ? positions[b] + 1 : seq_lens[b];
  len = len < 0 ? 0 : (len > max_seq ? max_seq : len);
  const int k_begin = split * keys_per_split;
  const int k_end = min(len, k_begin + keys_per_split);
  const int n_keys = max(0, k_end - k_begin);
  const int n_tiles = (n_keys + kKeysPerTile - 1) / kKeysPerTile;
  const int my_tiles = n_tiles > warp ? (n_tiles - warp + WARPS - 1) / WARPS : 0;
  const int row_base = (b * kv_heads + h) * max_seq;

  auto issue = [&](int i) {
    const int t = warp + i * WARPS;
    const int key0 = k_begin + t * kKeysPerTile;
    const int st = i % STAGES;
    uint8_t* kst = my_stages + st * S::kStageBytes;
    uint8_t* vst = kst + S::kTileBytes;
    mbar_arrive_expect_tx(&my_bars[st], S::kStageBytes);
#pragma unroll
    for (int r = 0; r < S::kRegions; ++r) {
      tma_load_2d(kst + r * S::kRegionBytes, &kmap, &my_bars[st], r * 64, row_base + key0);
      tma_load_2d(vst + r * S::kRegionBytes, &vmap, &my_bars[st], r * 64, row_base + key0);
    }
  };

  int issued = 0;
  if (positions != nullptr) {
    if (lane == 0)
      for (; issued < my_tiles && issued < STAGES; ++issued)
        if (k_begin + (warp + issued * WARPS + 1) * kKeysPerTile > len - 1) break;  // holds the new key
        else issue(issued);
    issued = __shfl_sync(0xffffffffu, issued, 0);
    pdl_wait();  // q and the new key come from the previous kernel
  }
  if (lane == 0) {
    for (int i = issued; i < my_tiles && i < STAGES; ++i) issue(i);
  }

  // Q^T fragments (B operand of the score MMA): column n = query head g of the
  // group, rows = head dims.  Columns past the group are zero.
  uint32_t qf[KSTEPS][2];
  {
    const __half* qh = q + (static_cast<size_t>(b) * q_heads + h * group + g) * D;
#pragma unroll
    for (int s = 0; s < KSTEPS; ++s) {
      if (g < group) {
        qf[s][0] = *reinterpret_cast<const uint32_t*>(qh + 16 * s + 2 * c);
        qf[s][1] = *reinterpret_cast<const uint32_t*>(qh + 16 * s + 2 * c + 8);
      } else {
        qf[s][0] = qf[s][1] = 0u;
      }
    }
  }

  float m_run[2] = {-INFINITY, -INFINITY};  // heads 2c, 2c+1 (log2 domain)
  float l_run[2] = {0.f, 0.f};              // this thread's share of the row sums
  float o[DBLK][4];
#pragma unroll
  for (int d = 0; d < DBLK; ++d) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.f;

  bool aborted = false;
  int consumed = 0;
  for (int i = 0; i < my_tiles; ++i) {
    const int st = i % STAGES;
    if (!mbar_wait(&my_bars[st], (i / STAGES) & 1, kDevErrTmaTimeout)) {
      aborted = true;
      break;
    }
    consumed = i + 1;
    const int t = warp + i * WARPS;
    const int key0 = k_begin + t * kKeysPerTile;
    const int valid = min(kKeysPerTile, k_end - key0);
    uint8_t* kst = my_stages + st * S::kStageBytes;
    uint8_t* vst = kst + S::kTileBytes;

    // Rows past the last valid key may hold anything (other sequences, or
    // uninitialised cache); p is 0 there, but 0 * NaN is NaN, so zero them.
    if (valid < kKeysPerTile) {
      const int nbytes = (kKeysPerTile - valid) * 128;
#pragma unroll
      for (int r = 0; r < S::kRegions; ++r) {
        uint8_t* base = vst + r * S::kRegionBytes + valid * 128;
        for (int off = lane * 16; off < nbytes; off += 32 * 16)
          *reinterpret_cast<uint4*>(base + off) = make_uint4(0, 0, 0, 0);
      }
      __syncwarp();
    }

    const uint32_t kbase = smem_u32(kst), vbase = smem_u32(vst);

    // ---- scores: S^T[key, head] for two 16-key m-tiles ----
    float sacc[2][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      sacc[mt][0] = sacc[mt][1] = sacc[mt][2] = sacc[mt][3] = 0.f;
      const int row = mt * 16 + (lane & 15);
#pragma unroll
      for (int s = 0; s < KSTEPS; ++s) {
        const int chunk = 2 * s + (lane >> 4);
        const uint32_t addr = kbase + (chunk >> 3) * S::kRegionBytes + row * 128 +
                              (((chunk & 7) ^ (row & 7)) << 4);
        uint32_t a0, a1, a2, a3;
        ldmatrix_x4(a0, a1, a2, a3, addr);
        mma_16816(sacc[mt], a0, a1, a2, a3, qf[s][0], qf[s][1]);
      }
    }

    // ---- online softmax (log2 domain) ----
    float sv[2][4];
    float tmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int key_local = mt * 16 + g + ((r & 2) ? 8 : 0);
        const float v = key_local < valid ? sacc[mt][r] * scale_log2 : -INFINITY;
        sv[mt][r] = v;
        tmax[r & 1] = fmaxf(tmax[r & 1], v);
      }
    }
    float alpha[2], m_use[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      tmax[j] = fmaxf(tmax[j], __shfl_xor_sync(0xffffffffu, tmax[j], 4));
      tmax[j] = fmaxf(tmax[j], __shfl_xor_sync(0xffffffffu, tmax[j], 8));
      tmax[j] = fmaxf(tmax[j], __shfl_xor_sync(0xffffffffu, tmax[j], 16));
      const float m_new = fmaxf(m_run[j], tmax[j]);
      m_use[j] = m_new == -INFINITY ? 0.f : m_new;
      alpha[j] = fast_exp2(m_run[j] - m_use[j]);
      m_run[j] = m_new;
      l_run[j] *= alpha[j];
    }
    uint32_t pb[2][2];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      float p[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        p[r] = fast_exp2(sv[mt][r] - m_use[r & 1]);
        l_run[r & 1] += p[r];
      }
      pb[mt][0] = movmatrix_trans(pack_half2(p[0], p[1]));  // keys 0-7 of the m-tile
      pb[mt][1] = movmatrix_trans(pack_half2(p[2], p[3]));  // keys 8-15
    }
#pragma unroll
    for (int d = 0; d < DBLK; ++d) {
      o[d][0] *= alpha[0];
      o[d][1] *= alpha[1];
      o[d][2] *= alpha[0];
      o[d][3] *= alpha[1];
    }

    // ---- O^T[dim, head] += V^T P^T ----
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      const int q4 = lane >> 3;
      const int key_row = mt * 16 + (lane & 7) + ((q4 >> 1) << 3);
#pragma unroll
      for (int d = 0; d < DBLK; ++d) {
        const int chunk = 2 * d + (q4 & 1);
        const uint32_t addr = vbase + (chunk >> 3) * S::kRegionBytes + key_row * 128 +
                              (((chunk & 7) ^ (key_row & 7)) << 4);
        uint32_t a0, a1, a2, a3;
        ldmatrix_x4_trans(a0, a1, a2, a3, addr);
        mma_16816(o[d], a0, a1, a2, a3, pb[mt][0], pb[mt][1]);
      }
    }

    __syncwarp();
    if (lane == 0 && i + STAGES < my_tiles) {
      fence_proxy_async_smem();  // the zero-fill above precedes the next TMA write
      issue(i + STAGES);
    }
  }

  if (aborted) {
    // Drain copies still in flight into this warp's stages before leaving.
    for (int i = consumed; i < my_tiles && i < consumed + STAGES; ++i)
      mbar_wait(&my_bars[i % STAGES], (i / STAGES) & 1, kDevErrTmaTimeout);
    m_run[0] = m_run[1] = -INFINITY;
    l_run[0] = l_run[1] = 0.f;
#pragma unroll
    for (int d = 0; d < DBLK; ++d) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.f;
  }

  // Full row sums: reduce this thread's share over the 8 lanes of its column.
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    l_run[j] += __shfl_xor_sync(0xffffffffu, l_run[j], 4);
    l_run[j] += __shfl_xor_sync(0xffffffffu, l_run[j], 8);
    l_run[j] += __shfl_xor_sync(0xffffffffu, l_run[j], 16);
  }

  __syncthreads();  // every warp is done with its stages: reuse them for the merge

  // Per-warp results: cm/cl [WARPS][8], co [WARPS][8][D].
  float* cm = reinterpret_cast<float*>(smem);
  float* cl = cm + WARPS * kMaxGroup;
  float* co = cl + WARPS * kMaxGroup;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int head = 2 * c + j;
    if (head < group) {
      if (g == 0) {
        cm[warp * kMaxGroup + head] = m_run[j];
        cl[warp * kMaxGroup + head] = l_run[j];
      }
      float* oh = co + (warp * kMaxGroup + head) * D;
#pragma unroll
      for (int d = 0; d < DBLK; ++d) {
        oh[16 * d + g] = o[d][j];
        oh[16 * d + g + 8] = o[d][2 + j];
      }
    }
  }
  __syncthreads();

  const size_t unit = static_cast<size_t>(b) * kv_heads + h;
  // Split partials of one unit are contiguous, `pitch` floats each: O
  // [group][D], m [group] (log2 domain), l [group], padded to 16 bytes (at
  // most kPartFloats).
  const int pitch = (group * D + 2 * group + 3) & ~3;
  float* my_part = part + (unit * num_splits + split) * pitch;
  // The warps' weights exp2(m_w - m) per head, the CTA's max m and row sum,
  // formed once per head; then each thread combines one 4-dim slice.
  float* cw = co + WARPS * kMaxGroup * D;  // [WARPS][8]
  float* cM = cw + WARPS * kMaxGroup;  // [8]
  float* cL = cM + kMaxGroup;          // [8]
  if (threadIdx.x < group) {
    const int head = threadIdx.x;
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) mx = fmaxf(mx, cm[w * kMaxGroup + head]);
    float L = 0.f;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) {
      const float mw = cm[w * kMaxGroup + head];
      const float wt = mw == -INFINITY ? 0.f : fast_exp2(mw - mx);
      cw[w * kMaxGroup + head] = wt;
      L += cl[w * kMaxGroup + head] * wt;
    }
    cM[head] = mx;
    cL[head] = L;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < group * D / 4; idx += WARPS * 32) {
    const int head = (idx * 4) / D, dim = idx * 4 - head * D;
    float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < WARPS; ++w) {
      const float wt = cw[w * kMaxGroup + head];
      const float4 v = *reinterpret_cast<const float4*>(co + (w * kMaxGroup + head) * D + dim);
      O.x += v.x * wt;
      O.y += v.y * wt;
      O.z += v.z * wt;
      O.w += v.w * wt;
    }
    if (num_splits == 1) {
      const float L = cL[head];
      const float inv = L > 0.f ? 1.f / L : 0.f;
      __half2* dst = reinterpret_cast<__half2*>(
          out + (static_cast<size_t>(b) * q_heads + h * group + head) * D + dim);
      dst[0] = __floats2half2_rn(O.x * inv, O.y * inv);
      dst[1] = __floats2half2_rn(O.z * inv, O.w * inv);
    } else {
      *reinterpret_cast<float4*>(my_part + head * D + dim) = O;
      if (dim == 0) {
        my_part[group * D + head] = cM[head];
        my_part[group * D + group + head] = cL[head];
      }
    }
  }
  if (num_splits == 1) return;

  // Last CTA of this (sequence, KV head) merges every split.  One thread
  // releases the CTA's partial (ordered before it by the barrier) with its
  // count; the CTA that completes the count acquires the others'.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t prev = atomicAdd(&counters[unit], 1u);
    s_last = (prev == static_cast<uint32_t>(num_splits - 1)) ? 1 : 0;
    if (s_last) __threadfence();
  }
  __syncthreads();
  if (!s_last) return;
  // Merge with one L2 round trip: the unit's partials (contiguous) come into
  // the idle stage buffers with one bulk copy when they fit (else they are read
  // from L2 directly); one warp per head forms the split weights with
  // lane-parallel reductions; then each thread sums one 4-dim slice over the
  // splits.
  const float* up = part + unit * num_splits * pitch;
  const int slab = group * D;  // floats of one split's outputs; m and l follow
  const uint32_t unit_bytes = static_cast<uint32_t>(num_splits) * pitch * 4u;
  const bool staged = unit_bytes + 2 * static_cast<size_t>(num_splits) * kMaxGroup * 4 + 64 <=
                      static_cast<size_t>(WARPS) * STAGES * S::kStageBytes;
  const float* src = staged ? reinterpret_cast<const float*>(smem) : up;
  float* sw = reinterpret_cast<float*>(smem) + (staged ? num_splits * pitch : 0);  // [splits][8] weights
  float* sL = sw + num_splits * kMaxGroup;  // [8] merged row sums
  bool ready = true;
  if (staged) {
    if (threadIdx.x == 0) {
      // The partials were written by other CTAs' generic stores, and the stage
      // buffers were last used by this CTA's generic accesses: order both
      // before this thread's bulk (async-proxy) copy.
      asm volatile("fence.proxy.async.global;" ::: "memory");
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(merge_bar, unit_bytes);
      bulk_load_hint(smem, up, unit_bytes, merge_bar, policy_evict_first());
    }
    ready = mbar_wait(merge_bar, 0, kDevErrTmaTimeout);
  }
  // Split statistics: m at slab + head, l at slab + group + head of each split.
  auto stat = [&](int sp, int at) {
    const float* ps = src + static_cast<size_t>(sp) * pitch + slab + at;
    return staged ? *ps : __ldcg(ps);
  };
  for (int head = warp; ready && head < group; head += WARPS) {
    float mx = -INFINITY;
    for (int sp = lane; sp < num_splits; sp += 32) mx = fmaxf(mx, stat(sp, head));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float L = 0.f;
    for (int sp = lane; sp < num_splits; sp += 32) {
      const float ms = stat(sp, head);
      const float wt = ms == -INFINITY ? 0.f : fast_exp2(ms - mx);
      sw[sp * kMaxGroup + head] = wt;
      L += stat(sp, group + head) * wt;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    if (lane == 0) sL[head] = L;
  }
  __syncthreads();
  for (int idx = threadIdx.x; ready && idx < group * D / 4; idx += WARPS * 32) {
    const int head = (idx * 4) / D, dim = idx * 4 - head * D;
    const float* col = src + head * D + dim;
    const float* wcol = sw + head;
    // Two independent chains (even and odd splits), added at the end.
    auto part_at = [&](int sp) {
      const float4* at = reinterpret_cast<const float4*>(col + static_cast<size_t>(sp) * pitch);
      return staged ? *at : __ldcg(at);
    };
    float4 e = make_float4(0.f, 0.f, 0.f, 0.f), o = e;
    int sp = 0;
#pragma unroll 4
    for (; sp + 1 < num_splits; sp += 2) {
      const float w0 = wcol[sp * kMaxGroup], w1 = wcol[(sp + 1) * kMaxGroup];
      const float4 p0 = part_at(sp), p1 = part_at(sp + 1);
      e.x += w0 * p0.x;
      e.y += w0 * p0.y;
      e.z += w0 * p0.z;
      e.w += w0 * p0.w;
      o.x += w1 * p1.x;
      o.y += w1 * p1.y;
      o.z += w1 * p1.z;
      o.w += w1 * p1.w;
    }
    if (sp < num_splits) {
      const float w0 = wcol[sp * kMaxGroup];
      const float4 p0 = part_at(sp);
      e.x += w0 * p0.x;
      e.y += w0 * p0.y;
      e.z += w0 * p0.z;
      e.w += w0 * p0.w;
    }
    const float4 o4 = make_float4(e.x + o.x, e.y + o.y, e.z + o.z, e.w + o.w);
    const float L = sL[head];
    const float inv = L > 0.f ? 1.f / L : 0.f;
    __half2* dst = reinterpret_cast<__half2*>(
        out + (static_cast<size_t>(b) * q_heads + h * group + head) * D + dim);
    dst[0] = __floats2half2_rn(o4.x * inv, o4.y * inv);
    dst[1] = __floats2half2_rn(o4.z * inv, o4.w * inv);
  }
  if (threadIdx.x == 0) counters[unit] = 0u;  // leave the workspace reusable
}

constexpr int kWarps = 4;
constexpr int kStages = 3;

template <int D>
constexpr size_t fd_smem_bytes() {
  return 1024 + static_cast<size_t>(kWarps) * kStages * FdShape<D>::kStageBytes +
         (kWarps * kStages + 1) * sizeof(uint64_t);
}

// Splits per (sequence, KV head): the count whose waves of CTAs (one per SM)
// finish first, charging each CTA a fixed start-up cost equivalent to ~96 keys
// and each split ~6 keys of the merge (measured on 1-8 units of 4096 keys:
// 32 splits for 1-2 units, 16 for 8).
int choose_splits(int units, int max_seq, int sms) {
  int best = 1;
  double best_cost = 1e300;
  for (int s = 1; s <= 64; ++s) {
    int kps = (max_seq + s - 1) / s;
    kps = (kps + 63) / 64 * 64;
    const int s_eff = (max_seq + kps - 1) / kps;
    if (s_eff != s) continue;
    const long ctas = static_cast<long>(units) * s_eff;
    const long waves = (ctas + sms - 1) / sms;
    const double cost = static_cast<double>(waves) * (kps + 96) + 6.0 * s_eff;
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = s_eff;
    }
  }
  return best;
}

int resolve_splits(int batch, int kv_heads, int max_seq, int num_splits, int* kps_out) {
  int s = num_splits > 0 ? num_splits : choose_splits(batch * kv_heads, max_seq, sm_count());
  if (s > max_seq) s = max_seq;
  int kps = (max_seq + s - 1) / s;
  kps = (kps + kKeysPerTile - 1) / kKeysPerTile * kKeysPerTile;
  s = (max_seq + kps - 1) / kps;
  if (kps_out) *kps_out = kps;
  return s;
}

// The launch shape of one call: key splits per (sequence, KV head) and keys
// per split.
struct FdLaunch {
  int splits = 1, kps = 0;
};

FdLaunch plan_fd(int batch, int kv_heads, int max_seq, int num_splits) {
  FdLaunch L;
  L.splits = resolve_splits(batch, kv_heads, max_seq, num_splits, &L.kps);
  return L;
}

size_t workspace_bytes_for(int batch, int kv_heads, int head_dim, int splits) {
  if (splits <= 1) return 0;
  const size_t units = static_cast<size_t>(batch) * kv_heads;
  const size_t counters = kCounterBytes;
  const size_t part_floats = static_cast<size_t>(kMaxGroup) * head_dim + 2 * kMaxGroup;
  return counters + units * splits * part_floats * sizeof(float);
}

template <int D>
int launch_fd(const CUtensorMap& km, const CUtensorMap& vm, const __half* q, const int32_t* lens,
              __half* out, float* part, uint32_t* counters, int batch, int q_heads, int kv_heads,
              int max_seq, int kps, int splits, float scale_log2, cudaStream_t stream, bool pdl,
              const int32_t* positions) {
  auto kern = flash_decode_kernel<D, kWarps, kStages>;
  constexpr size_t smem = fd_smem_bytes<D>();
  NPU_TRY_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(smem)));
  LaunchCfg cfg;
  cfg.grid = dim3(splits, kv_heads, batch);
  cfg.block = dim3(kWarps * 32);
  cfg.smem = smem;
  cfg.stream = stream;
  cfg.pdl = pdl;
  return launch(cfg, kern, km, vm, q, lens, out, part, counters, q_heads, kv_heads, max_seq, kps,
                splits, scale_log2, positions);
}

}  // namespace

// Internal entry used by the decode runtime as well as the C ABI.  With
// `positions` (the decode step's input, seq_lens[b] == positions[b] + 1) the
// kernel starts loading the keys cached by earlier steps before the previous
// kernel finishes.
int flash_decode_run(const void* q, const void* k, const void* v, const int32_t* seq_lens,
                     void* out, int batch, int q_heads, int kv_heads, int head_dim, int max_seq,
                     float scale, int num_splits, void* workspace, size_t workspace_bytes,
                     cudaStream_t stream, bool pdl, const int32_t* positions) {
  NPU_REQUIRE(q && k && v && (seq_lens || positions) && out, "flash_decode: null tensor pointer");
  NPU_REQUIRE(batch >= 1 && batch <= 65535, "flash_decode: batch %d out of range", batch);
  NPU_REQUIRE(kv_heads >= 1 && kv_heads <= 65535 && q_heads >= kv_heads && q_heads % kv_heads == 0,
              "flash_decode: q_heads %d is not a multiple of kv_heads %d", q_heads, kv_heads);
  NPU_REQUIRE(q_heads / kv_heads <= kMaxGroup, "flash_decode: group %d exceeds %d",
              q_heads / kv_heads, kMaxGroup);
  NPU_REQUIRE(head_dim == 64 || head_dim == 128, "flash_decode: head_dim %d not in {64,128}",
              head_dim);
  NPU_REQUIRE(max_seq >= 1, "flash_decode: max_seq %d", max_seq);
  NPU_REQUIRE(batch * kv_heads <= kMaxUnits, "flash_decode: batch x kv_heads exceeds %d",
              kMaxUnits);
  NPU_REQUIRE(static_cast<long long>(batch) * kv_heads * max_seq < (1ll << 31),
              "flash_decode: cache has too many rows for 32-bit TMA coordinates");
  NPU_REQUIRE(std::isfinite(scale), "flash_decode: scale is not finite");
  NPU_REQUIRE((reinterpret_cast<uintptr_t>(q) & 3) == 0 && (reinterpret_cast<uintptr_t>(out) & 3) == 0,
              "flash_decode: q and out must be 4-byte aligned");
  NPU_REQUIRE(num_splits >= 0 && num_splits <= kMaxSplits, "flash_decode: num_splits %d not in [0, %d]",
              num_splits, kMaxSplits);
  const FdLaunch L = plan_fd(batch, kv_heads, max_seq, num_splits);
  const int kps = L.kps, splits = L.splits;
  const size_t need = workspace_bytes_for(batch, kv_heads, head_dim, splits);
  NPU_REQUIRE(need == 0 || (workspace && workspace_bytes >= need),
              "flash_decode: workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  NPU_REQUIRE(need == 0 || (reinterpret_cast<uintptr_t>(workspace) & 255) == 0,
              "flash_decode: workspace is not 256-byte aligned");

  const uint64_t rows = static_cast<uint64_t>(batch) * kv_heads * max_seq;
  CUtensorMap km, vm;
  int rc = make_tensor_map_2d(&km, k, rows, head_dim, kKeysPerTile, 64);
  if (rc) return rc;
  rc = make_tensor_map_2d(&vm, v, rows, head_dim, kKeysPerTile, 64);
  if (rc) return rc;

  uint32_t* counters = reinterpret_cast<uint32_t*>(workspace);
  float* part =
      need ? reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(workspace) + kCounterBytes)
           : nullptr;
  const float scale_log2 = scale * 1.4426950408889634f;
  const __half* qh = static_cast<const __half*>(q);
  __half* oh = static_cast<__half*>(out);
  if (head_dim == 128)
    return launch_fd<128>(km, vm, qh, seq_lens, oh, part, counters, batch, q_heads, kv_heads,
                          max_seq, kps, splits, scale_log2, stream, pdl, positions);
  return launch_fd<64>(km, vm, qh, seq_lens, oh, part, counters, batch, q_heads, kv_heads,
                       max_seq, kps, splits, scale_log2, stream, pdl, positions);
}

size_t flash_decode_workspace(int batch, int kv_heads, int head_dim, int max_seq, int num_splits) {
  if (batch < 1 || kv_heads < 1 || max_seq < 1) return 0;
  const FdLaunch L = plan_fd(batch, kv_heads, max_seq, num_splits);
  return workspace_bytes_for(batch, kv_heads, head_dim, L.splits);
}

}  // namespace npu_b200

extern "C" size_t npu_b200_flash_decode_workspace_size(int batch, int kv_heads, int head_dim,
                                                       int max_seq, int num_splits) {
  return npu_b200::flash_decode_workspace(batch, kv_heads, head_dim, max_seq, num_splits);
}

extern "C" int npu_b200_flash_decode(const void* d_q, const void* d_k, const void* d_v,
                                     const int32_t* d_seq_lens, void* d_out, int batch,
                                     int q_heads, int kv_heads, int head_dim, int max_seq,
                                     float scale, int num_splits, void* d_workspace,
                                     size_t workspace_bytes, void* stream) {
  npu_b200::clear_error();
  // Launched as a programmatic dependent of the stream's previous work: the
  // kernel reads no input and writes no output before griddepcontrol.wait
  // (which returns once that work has completed), so only the launch and the
  // barrier set-up overlap its tail.
  return npu_b200::flash_decode_run(d_q, d_k, d_v, d_seq_lens, d_out, batch, q_heads, kv_heads,
                                    head_dim, max_seq, scale, num_splits, d_workspace,
                                    workspace_bytes, static_cast<cudaStream_t>(stream), true,
                                    nullptr);
}

// ---------------------------------------------------------------------------
// Allocation-free variant: the split-merge scratch (counters + partial O, m, l)
// lives in a fixed array in the module's device memory instead of a caller
// buffer.  Every GPU that loads this library keeps this array until the
// process exits.
// ---------------------------------------------------------------------------
namespace npu_b200 {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;  // 4 MiB per device
static __device__ __align__(256) uint8_t g_flash_decode_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// The array's name is only a host-side stand-in for the symbol; the device
// address differs per device.  It is looked up with that device current on
// every call made outside stream capture (so a module reloaded after
// cudaDeviceReset is found again) and remembered for calls made while `s`
// is being captured, which must not be the first call on the device.
int scratch_address(cudaStream_t s, void** out) {
  int dev = 0;
  NPU_TRY_CUDA(cudaGetDevice(&dev));
  NPU_REQUIRE(dev >= 0 && dev < kMaxDevices, "device %d out of range", dev);
  cudaStreamCaptureStatus capturing = cudaStreamCaptureStatusNone;
  NPU_TRY_CUDA(cudaStreamIsCapturing(s, &capturing));
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (capturing == cudaStreamCaptureStatusNone) {
    void* p = nullptr;
    NPU_TRY_CUDA(cudaGetSymbolAddress(&p, g_flash_decode_scratch));
    g_scratch_ptr[dev] = p;
  }
  NPU_REQUIRE(g_scratch_ptr[dev] != nullptr,
              "flash_decode_noalloc: the first call on device %d was made during stream capture; "
              "make one call outside capture first",
              dev);
  *out = g_scratch_ptr[dev];
  return NPU_B200_OK;
}

}  // namespace
}  // namespace npu_b200

extern "C" int npu_b200_flash_decode_noalloc(const void* d_q, const void* d_k, const void* d_v,
                                             const int32_t* d_seq_lens, void* d_out, int batch,
                                             int q_heads, int kv_heads, int head_dim, int max_seq,
                                             float scale, int num_splits, void* stream) {
  using namespace npu_b200;
  clear_error();
  NPU_REQUIRE(batch >= 1 && kv_heads >= 1 && max_seq >= 1 && num_splits >= 0 &&
                  num_splits <= kMaxSplits && (head_dim == 64 || head_dim == 128),
              "flash_decode_noalloc: invalid shape");
  const size_t need = flash_decode_workspace(batch, kv_heads, head_dim, max_seq, num_splits);
  NPU_REQUIRE(need <= kNoAllocScratchBytes,
              "flash_decode_noalloc: this shape needs %zu bytes of split scratch, more than the "
              "%zu-byte static scratch; use fewer splits or npu_b200_flash_decode",
              need, kNoAllocScratchBytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  void* scratch = nullptr;
  int rc = scratch_address(s, &scratch);
  if (rc) return rc;
  if (need > 0) {  // a single split per unit merges nothing and uses no scratch
    // The array keeps whatever the previous call left: the split counters
    // must start at zero.
    const size_t units = static_cast<size_t>(batch) * kv_heads;
    NPU_TRY_CUDA(cudaMemsetAsync(scratch, 0, units * sizeof(uint32_t), s));
  }
  return flash_decode_run(d_q, d_k, d_v, d_seq_lens, d_out, batch, q_heads, kv_heads, head_dim,
                          max_seq, scale, num_splits, scratch, kNoAllocScratchBytes, s, true,
                          nullptr);
}
