// Device-side pieces of the batch 1-2 GEMV (gemv.cu): geometry, the consumer
// barrier, bounded waits, the per-panel MMA, and the fused epilogue of one
// 16-row group.
#pragma once

#include <math.h>

#include "common.cuh"
#include "peer.cuh"
#include "proj.cuh"

namespace npu_b200 {
namespace gemv {

constexpr int kRows = 16;                  // rows per group
constexpr int kParts = 8;                  // consumer threads per row
constexpr int kConsumers = kRows * kParts; // 128: warps 0-3
constexpr int kGemvThreads = kConsumers + 32;  // + producer warp 4
constexpr int kPanelsPerStage = 4;
constexpr int kSlice = kRows * 128;        // bytes of one group's slice of a panel
constexpr int kStageBytes = kPanelsPerStage * kSlice;
constexpr int kMaxStages = 16;
constexpr int kGemvSmemPerSm = 233472;     // usable shared memory per SM
constexpr int kGemvSmemReserved = 1024;    // per CTA, taken by the runtime

// Barrier of the four consumer warps (named barrier 1; the producer warp never
// takes part).
__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"r"(kConsumers) : "memory");
}
__device__ __forceinline__ bool consumer_sync_or(bool pred) {
  uint32_t any;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(any)
      : "r"(static_cast<uint32_t>(pred)), "r"(kConsumers)
      : "memory");
  return any != 0;
}

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

// One warp's share of a ring stage: the 16-row x 64-column panel slice at
// shared address `slice` (128-byte rows, 16-byte chunks swizzled by row % 8)
// times the staged activations `xk` (column 0 of the panel for token 0, token
// stride x_ld), into four independent accumulator chains (one per k-step).
template <int BT>
__device__ __forceinline__ void mma_panel(float (&c)[4][4], uint32_t slice, const __half* xk,
                                          int x_ld) {
  const int lane = threadIdx.x & 31;
  // ldmatrix source row / 16-byte chunk of this lane: matrix lane / 8 of the
  // A fragment is (rows 0-7 | 8-15) x (k 0-7 | 8-15).
  const int a_row = ((lane >> 3) & 1) * 8 + (lane & 7), a_chunk = lane >> 4;
  const int b_tok = lane >> 2, b_k = 2 * (lane & 3);  // B fragment: token, k pair
  slice += a_row * 128;
  xk += b_k;
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    uint32_t a0, a1, a2, a3, b0 = 0, b1 = 0;
    ldmatrix_x4(a0, a1, a2, a3, slice + (((2 * kk + a_chunk) ^ (a_row & 7)) << 4));
    if (b_tok < BT) {
      b0 = *reinterpret_cast<const uint32_t*>(xk + b_tok * x_ld + kk * 16);
      b1 = *reinterpret_cast<const uint32_t*>(xk + b_tok * x_ld + kk * 16 + 8);
    }
    mma_16816(c[kk], a0, a1, a2, a3, b0, b1);
  }
}

// The four consumer warps' chains of one group added in a fixed order through
// part_sum ([4 warps][16 rows][2]): acc[b] for row t / 8, token b (unscaled).
template <int BT>
__device__ __forceinline__ void reduce_warps(const float (&c)[4][4], float* part_sum,
                                             float (&acc)[BT]) {
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31, row = t / kParts;
  // Lanes 4i hold rows i and i + 8, tokens 0-1.
  if ((lane & 3) == 0) {
    float* ps = part_sum + warp * kRows * 2;
    float v[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) v[q] = (c[0][q] + c[1][q]) + (c[2][q] + c[3][q]);
    ps[(lane >> 2) * 2] = v[0];
    ps[(lane >> 2) * 2 + 1] = v[1];
    ps[((lane >> 2) + 8) * 2] = v[2];
    ps[((lane >> 2) + 8) * 2 + 1] = v[3];
  }
  consumer_sync();
#pragma unroll
  for (int b = 0; b < BT; ++b)
    acc[b] = ((part_sum[row * 2 + b] + part_sum[(kRows + row) * 2 + b]) +
              part_sum[(2 * kRows + row) * 2 + b]) +
             part_sum[(3 * kRows + row) * 2 + b];
}

// Epilogue kinds of the kernel's instantiations: EpiParams::kind, plus the
// STORE and RESID forms whose values go through the tensor-parallel exchange
// (px.seq >= 0).  Each instantiation carries only its own epilogue: code that
// is never taken still costs instruction fetch in a once-per-group path.
constexpr int kGemvStorePeer = 16;
constexpr int kGemvResidPeer = 17;

// The fused epilogue of row group g: acc[b] is row (g * 16 + t / 8)'s FP32
// value for token b (already RMSNorm-scaled), held by the 8 threads of the row;
// every consumer thread calls this (it contains consumer barriers).
template <int BT, int KIND>
__device__ __forceinline__ void gemv_epilogue(const EpiParams& ep, int g, float (&acc)[BT],
                                              const int* pos_s, float* red, int* red_id) {
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int row = t / kParts, part = t % kParts;
  const bool lead = part == 0;  // one thread per row writes
  const int n = g * kRows + row;         // row of W
  const int tile = n >> 7, p = n & 127;  // 128-row tile and row within it

  if constexpr (KIND == kEpiStore || KIND == kGemvStorePeer) {
    if (lead) {
      const float bias = ep.bias ? __half2float(ep.bias[n]) : 0.f;
#pragma unroll
      for (int b = 0; b < BT; ++b) {
        if (b < ep.batch) {
          float v = acc[b] + bias;
          if (ep.relu) v = fmaxf(v, 0.f);
          const size_t off = static_cast<size_t>(b) * ep.ld_out + n;
          if constexpr (KIND == kGemvStorePeer)
            px_store(ep.px, px_tag(ep.px, ep.px.seq), b, n, v);
          else if (ep.out_f32)
            static_cast<float*>(ep.out)[off] = v;
          else
            static_cast<__half*>(ep.out)[off] = __float2half_rn(v);
        }
      }
    }
  } else if constexpr (KIND == kEpiResid || KIND == kGemvResidPeer) {
    // Tensor parallel: all-reduce first.  The lead thread stores this rank's
    // partial as a tagged word, reads every rank's word for (b, n) over
    // NVLink (px_gather: all missing ranks' loads in flight together, round
    // after round) and adds them in rank order, as every rank does.
    if (KIND == kGemvResidPeer && lead) {
      const uint32_t tag = px_tag(ep.px, ep.px.seq);
#pragma unroll
      for (int b = 0; b < BT; ++b)
        if (b < ep.batch) px_store(ep.px, tag, b, n, acc[b]);
#pragma unroll
      for (int b = 0; b < BT; ++b) {
        if (b >= ep.batch) continue;
        uint32_t bits[kMaxRanks];
        px_gather(ep.px.part, ep.px.ranks, px_offset(ep.px, b, n), tag, bits);
        float sum = 0.f;
#pragma unroll
        for (int r = 0; r < kMaxRanks; ++r)
          if (r < ep.px.ranks) sum += __uint_as_float(bits[r]);
        acc[b] = sum;
      }
    }
    // Residual add, next norm's input, and the group's sum of squares.
    const float w = __half2float(ep.norm_w[n]);
#pragma unroll
    for (int b = 0; b < BT; ++b) {
      float h2 = 0.f;
      if (lead && b < ep.batch) {
        const size_t off = static_cast<size_t>(b) * ep.ld_resid + n;
        const float h = ep.resid[off] + acc[b];
        ep.resid[off] = h;
        ep.xw[static_cast<size_t>(b) * ep.ld_xw + n] = __float2half_rn(h * w);
        h2 = h * h;
      }
#pragma unroll
      for (int o = kParts; o < 32; o <<= 1) h2 += __shfl_xor_sync(0xffffffffu, h2, o);
      if (lane == 0) red[warp * BT + b] = h2;
    }
    consumer_sync();
    if (t < BT && t < ep.batch)
      ep.ssq_out[static_cast<size_t>(g) * ep.ssq_out_ld + t] =
          red[t] + red[BT + t] + red[2 * BT + t] + red[3 * BT + t];
  } else if constexpr (KIND == kEpiSwiGLU) {
    // (gate_j, up_j) are rows (2j, 2j + 1).
#pragma unroll
    for (int b = 0; b < BT; ++b) {
      const float up = __shfl_xor_sync(0xffffffffu, acc[b], kParts);
      if (lead && (n & 1) == 0 && b < ep.batch) {
        const float gt = acc[b];
        static_cast<__half*>(ep.out)[static_cast<size_t>(b) * ep.ld_out + (n >> 1)] =
            __float2half_rn(gt / (1.f + expf(-gt)) * up);
      }
    }
  } else if constexpr (KIND == kEpiQKV) {
    // Head rows in pair order: row p holds dim (p >> 1) + 64 * (p & 1).
    const bool is_q = tile < ep.q_heads;
    const bool is_k = !is_q && tile < ep.q_heads + ep.kv_heads;
    const int i = p >> 1, d = i + ((p & 1) << 6);
#pragma unroll
    for (int b = 0; b < BT; ++b) {
      const float partner = __shfl_xor_sync(0xffffffffu, acc[b], kParts);
      if ((is_q || is_k) && b < ep.batch) {
        float sn, cs;
        if (ep.rope_tab != nullptr) {
          const float2 cssn = reinterpret_cast<const float2*>(ep.rope_tab)[b * 64 + i];
          cs = cssn.x;
          sn = cssn.y;
        } else {
          sincosf(static_cast<float>(pos_s[b]) * ep.inv_freq[i], &sn, &cs);
        }
        acc[b] = (p & 1) == 0 ? acc[b] * cs - partner * sn : acc[b] * cs + partner * sn;
      }
    }
    if (lead) {
#pragma unroll
      for (int b = 0; b < BT; ++b) {
        if (b >= ep.batch) continue;
        if (is_q) {
          static_cast<__half*>(ep.out)[static_cast<size_t>(b) * ep.ld_out + tile * 128 + d] =
              __float2half_rn(acc[b]);
        } else {
          const int kh = is_k ? tile - ep.q_heads : tile - ep.q_heads - ep.kv_heads;
          const int pos = pos_s[b];
          if (pos < 0 || pos >= ep.max_seq) {
            report_error(kDevErrBounds);
          } else {
            __half* cache = is_k ? ep.k_cache : ep.v_cache;
            cache[static_cast<size_t>(b) * ep.cache_batch_stride +
                  (static_cast<size_t>(kh) * ep.max_seq + pos) * 128 + d] = __float2half_rn(acc[b]);
          }
        }
      }
    }
  } else if constexpr (KIND == kEpiArgmax) {
    // The group's (max, argmax) per token, lowest row on ties.
#pragma unroll
    for (int b = 0; b < BT; ++b) {
      float bv = lead ? acc[b] : -INFINITY;
      int bi = n;
#pragma unroll
      for (int o = kParts; o < 32; o <<= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (better(ov, oi, bv, bi)) {
          bv = ov;
          bi = oi;
        }
      }
      if (lane == 0) {
        red[warp * BT + b] = bv;
        red_id[warp * BT + b] = bi;
      }
    }
    consumer_sync();
    if (t < BT && t < ep.batch) {
      float bv = red[t];
      int bi = red_id[t];
      for (int w = 1; w < 4; ++w)
        if (better(red[w * BT + t], red_id[w * BT + t], bv, bi)) {
          bv = red[w * BT + t];
          bi = red_id[w * BT + t];
        }
      ep.am_val[static_cast<size_t>(g) * ep.am_ld + t] = bv;
      ep.am_idx[static_cast<size_t>(g) * ep.am_ld + t] = bi;
    }
  }
}

}  // namespace gemv
}  // namespace npu_b200
