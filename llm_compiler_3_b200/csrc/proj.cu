// Decode projections on 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
// Replaces the NPU matmul lowering (lib/Transforms/HardwareOps.cpp:105-155
// convertMatmul, lib/Transforms/Emit.cpp:348-378 matrix write-out): FP16
// operands, FP32 accumulation from zero, one rounding at the store
// (lib/Transforms/Normalize.cpp:123-192 foldAccumulateAndRound).
//
// Shape of the problem at decode: W [N, K] is large and read once, X [B, K]
// (B = tokens) is tiny.  So the weight is the M=128 operand ("swap AB"), the
// tokens are the N=BN columns (16..128), and the accumulator tile 128 x BN
// lives in tensor memory.  Weights stream through an S-stage TMA ring
// (128-byte swizzle, L2 evict-first); the k-loop is split "stream-K" over
// exactly one CTA per SM, so every SM pulls the same number of weight bytes
// whatever N and K are.  A tile whose k-range spans several CTAs is finished by
// the last of them to arrive, which adds the others' FP32 partials in CTA
// order (deterministic) before the fused epilogue runs.
//
// Warp roles (192 threads): warps 0-3 epilogue (TMEM lanes 0-127 = tile rows),
// warp 4 TMA producer, warp 5 MMA issuer.  Two TMEM accumulators let the MMA of
// the next tile overlap the epilogue of the previous one.
#include <math.h>
#include <string.h>

#include "common.cuh"
#include "host.hpp"
#include "proj.cuh"

namespace npu_b200 {
namespace {

constexpr int kEpiThreads = 128;
constexpr int kThreads = 192;
constexpr int kMaxStages = 8;
constexpr int kCtasPerSm = 2;        // one CTA streams while the other finishes its epilogue
constexpr int kSmemPerSm = 233472;   // 228 KB of shared memory per SM
constexpr int kSmemReserved = 1024;  // per-CTA system reservation
constexpr int kChunkCols = 16;       // tokens per epilogue chunk (one tcgen05.ld x16)
// Tile counters sit in a fixed-size region at the start of the workspace, so
// projections of different shapes can share one workspace: a counter is never
// overlapped by another shape's partial-sum slots.
constexpr int kMaxTiles = 16384;
constexpr size_t kCounterBytes = kMaxTiles * sizeof(uint32_t);

template <int BN>
struct ProjShape {
  static constexpr int kABytes = 128 * 64 * 2;  // one 128-row x 64-k weight block
  static constexpr int kBBytes = BN * 64 * 2;   // one BN-token x 64-k activation block
  static constexpr int kStageBytes = (kABytes + kBBytes + 1023) / 1024 * 1024;
  static constexpr int kPitch = 128 + 4;        // floats per token column of the epilogue tile
  static constexpr int kTileBytes = kPitch * kChunkCols * 4;
  static constexpr int kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;
  static constexpr int kMiscBytes = 640 + 8 * BN;  // barriers, TMEM slot, per-token scalars
};

__device__ __forceinline__ uint8_t* align_1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

__device__ __forceinline__ void epi_sync() {
  asm volatile("bar.sync 1, %0;" ::"r"(kEpiThreads) : "memory");
}

// Barrier over the epilogue warps that also ORs a predicate across them, so all
// 128 threads take the same branch afterwards.
__device__ __forceinline__ bool epi_sync_or(bool pred) {
  uint32_t any;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(any)
      : "r"(static_cast<uint32_t>(pred)), "r"(kEpiThreads)
      : "memory");
  return any != 0;
}

// CTA whose stream-K range contains iteration i.
__device__ __forceinline__ int owner_cta(long long i, long long total, int grid) {
  long long c = (i * grid) / total;
  while (c + 1 < grid && ((c + 1) * total) / grid <= i) ++c;
  while (c > 0 && (c * total) / grid > i) --c;
  return static_cast<int>(c);
}

// Column sums of a 16-token x 128-row chunk staged in tile_s ([q][r], pitch
// 132): warp w reduces columns 4w..4w+3, each lane summing 4 rows before a
// butterfly over the warp.  Lane 0 of each warp writes out[q].
__device__ __forceinline__ void column_sums(const float* tile_s, float* out) {
  constexpr int P = 128 + 4;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int q = warp * 4 + j;
    const float* col = tile_s + q * P;
    float s = col[lane] + col[lane + 32] + col[lane + 64] + col[lane + 96];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) out[q] = s;
  }
}

// Column max / argmax (lowest row on ties) of the same staging, rows first_row + r.
__device__ __forceinline__ void column_argmax(const float* tile_s, int first_row, float* out_val,
                                              int* out_idx) {
  constexpr int P = 128 + 4;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int q = warp * 4 + j;
    const float* col = tile_s + q * P;
    float bv = col[lane];
    int bi = lane;
#pragma unroll
    for (int k = 1; k < 4; ++k) {
      const float x = col[lane + 32 * k];
      if (x > bv) {
        bv = x;
        bi = lane + 32 * k;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      out_val[q] = bv;
      out_idx[q] = first_row + bi;
    }
  }
}

// Epilogue of one 16-token chunk of a finished 128-row tile, for the
// epilogue kind KIND (ep.kind): each instantiation of the kernel carries only
// its own epilogue's code.  Thread r holds
// row tile*128 + r for tokens b0 .. b0+15 in v[]; tokens at or past col_end
// are skipped.  All branches depend only on the tile and the chunk, so every
// epilogue thread reaches the same barriers.
// A STORE whose values go to this rank's peer-exchange buffer as tagged
// words (px.seq >= 0) is instantiated apart from the plain STORE: the
// exchange's system-scope store in the plain STORE's loop, even untaken, made
// every chunk ~1500 cycles slower.
constexpr int kEpiStorePeer = 16;

template <int KIND>
__device__ __forceinline__ void run_epilogue_chunk(const EpiParams& ep, int tile, int r, int b0,
                                                   float (&v)[kChunkCols], const float* rn,
                                                   float* tile_s, float* aux, const int* pos_s,
                                                   int col_end) {
  constexpr int P = 128 + 4;
  const int batch = col_end;  // tokens b0 + q < col_end of this chunk are written
#pragma unroll
  for (int q = 0; q < kChunkCols; ++q) v[q] *= rn[b0 + q];

  if constexpr (KIND == kEpiStore) {
    const int n = tile * 128 + r;
    if (n < ep.n_rows) {
      const float bias = ep.bias ? __half2float(ep.bias[n]) : 0.f;
#pragma unroll
      for (int q = 0; q < kChunkCols; ++q) {
        const int b = b0 + q;
        if (b < batch) {
          float val = v[q] + bias;
          if (ep.relu) val = fmaxf(val, 0.f);
          const size_t off = static_cast<size_t>(b) * ep.ld_out + n;
          if (ep.out_f32)
            static_cast<float*>(ep.out)[off] = val;
          else
            static_cast<__half*>(ep.out)[off] = __float2half_rn(val);
        }
      }
    }
  } else if constexpr (KIND == kEpiStorePeer) {
    const int n = tile * 128 + r;
    if (n < ep.n_rows) {
      const float bias = ep.bias ? __half2float(ep.bias[n]) : 0.f;
      const uint32_t tag = px_tag(ep.px, ep.px.seq);
#pragma unroll
      for (int q = 0; q < kChunkCols; ++q) {
        const int b = b0 + q;
        if (b < batch) {
          float val = v[q] + bias;
          if (ep.relu) val = fmaxf(val, 0.f);
          px_store(ep.px, tag, b, n, val);
        }
      }
    }
  } else if constexpr (KIND == kEpiResid) {
    const int n = tile * 128 + r;
    const bool valid = n < ep.n_rows;
    const float w = valid ? __half2float(ep.norm_w[n]) : 0.f;
    // Independent loads first: the chunk costs one memory round trip.
    float rv[kChunkCols];
#pragma unroll
    for (int q = 0; q < kChunkCols; ++q) {
      const int b = b0 + q;
      rv[q] = (valid && b < batch) ? __ldcg(ep.resid + static_cast<size_t>(b) * ep.ld_resid + n)
                                   : 0.f;
    }
#pragma unroll
    for (int q = 0; q < kChunkCols; ++q) {
      const int b = b0 + q;
      float h2 = 0.f;
      if (valid && b < batch) {
        const float h = rv[q] + v[q];
        ep.resid[static_cast<size_t>(b) * ep.ld_resid + n] = h;
        ep.xw[static_cast<size_t>(b) * ep.ld_xw + n] = __float2half_rn(h * w);
        h2 = h * h;
      }
      tile_s[q * P + r] = h2;
    }
    epi_sync();
    if (ep.ssq_out_rows == 16) {
      // One partial per 16 rows: warp w sums rows 16g..16g+15 (g = 2w, 2w+1)
      // for every token of the chunk, half a warp per group.
      const int warp = r >> 5, lane = r & 31;
      const int g = 2 * warp + (lane >> 4), row = lane & 15;
#pragma unroll
      for (int q = 0; q < kChunkCols; ++q) {
        float t = tile_s[q * P + 16 * g + row];
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        if (row == 0 && b0 + q < batch && tile * 128 + 16 * g < ep.n_rows)
          ep.ssq_out[static_cast<size_t>(tile * 8 + g) * ep.ssq_out_ld + b0 + q] = t;
      }
    } else {
      column_sums(tile_s, aux);
      epi_sync();
      if (r < kChunkCols && b0 + r < batch)
        ep.ssq_out[static_cast<size_t>(tile) * ep.ssq_out_ld + b0 + r] = aux[r];
    }
    epi_sync();
  } else if constexpr (KIND == kEpiSwiGLU) {
    // Rows come in (gate_j, up_j) pairs: even row r holds gate, r + 1 holds up,
    // j = tile * 64 + r / 2.  The partner is the neighbouring lane.
    const int j = tile * 64 + (r >> 1);
#pragma unroll
    for (int q = 0; q < kChunkCols; ++q) {
      const float other = __shfl_xor_sync(0xffffffffu, v[q], 1);
      if ((r & 1) == 0 && b0 + q < batch && j < ep.n_rows / 2) {
        const float g = v[q], u = other;
        static_cast<__half*>(ep.out)[static_cast<size_t>(b0 + q) * ep.ld_out + j] =
            __float2half_rn(g / (1.f + expf(-g)) * u);
      }
    }
  } else if constexpr (KIND == kEpiQKV) {
    // Head tiles store head dims in rotate_half pair order: row r holds dim
    // d = r / 2 + 64 * (r % 2), so RoPE partners (d, d + 64) are adjacent lanes.
    const bool is_q = tile < ep.q_heads;
    const bool is_k = !is_q && tile < ep.q_heads + ep.kv_heads;
    const int d = (r >> 1) + ((r & 1) << 6);
    const __half* nw = is_q ? ep.q_norm_w : (is_k ? ep.k_norm_w : nullptr);
    if (nw) {  // per-head RMSNorm over the 128 dims (Qwen3 q_norm / k_norm)
#pragma unroll
      for (int q = 0; q < kChunkCols; ++q) tile_s[q * P + r] = v[q] * v[q];
      epi_sync();
      column_sums(tile_s, aux);
      epi_sync();
      if (r < kChunkCols) aux[r] = rsqrtf(aux[r] * (1.f / 128.f) + ep.qk_eps);
      epi_sync();
      const float wr = __half2float(nw[d]);
#pragma unroll
      for (int q = 0; q < kChunkCols; ++q) v[q] = v[q] * aux[q] * wr;
      epi_sync();
    }
    if (is_q || is_k) {  // RoPE: out_d = x_d cos - x_{d+64} sin, out_{d+64} = x_{d+64} cos + x_d sin
      const int i = r >> 1;
      // The chunk's (cos, sin) first, as unconditional independent loads (tokens
      // past the end read the last token's row): one memory round trip per
      // chunk.  Loaded beside each token's shuffle, they cost one round trip
      // per token (~10 us per batch-64 launch).
      float2 cssn[kChunkCols];
      if (ep.rope_tab != nullptr) {  // cos / sin of this step's positions, precomputed
        const float2* tab = reinterpret_cast<const float2*>(ep.rope_tab) + i;
#pragma unroll
        for (int q = 0; q < kChunkCols; ++q) cssn[q] = __ldg(tab + min(b0 + q, batch - 1) * 64);
      } else {
        const float f = ep.inv_freq[i];
#pragma unroll
        for (int q = 0; q < kChunkCols; ++q) {
          float sn, cs;
          sincosf(static_cast<float>(pos_s[b0 + q]) * f, &sn, &cs);
          cssn[q] = make_float2(cs, sn);
        }
      }
#pragma unroll
      for (int q = 0; q < kChunkCols; ++q) {
        const float partner = __shfl_xor_sync(0xffffffffu, v[q], 1);
        const float cs = cssn[q].x, sn = cssn[q].y;
        if (b0 + q < batch)
          v[q] = (r & 1) == 0 ? v[q] * cs - partner * sn : v[q] * cs + partner * sn;
      }
    }
    if (is_q) {
      __half* qo = static_cast<__half*>(ep.out);
#pragma unroll
      for (int q = 0; q < kChunkCols; ++q)
        if (b0 + q < batch)
          qo[static_cast<size_t>(b0 + q) * ep.ld_out + tile * 128 + d] = __float2half_rn(v[q]);
    } else {
      const int kh = is_k ? tile - ep.q_heads : tile - ep.q_heads - ep.kv_heads;
      __half* cache = is_k ? ep.k_cache : ep.v_cache;
      bool out_of_cache = false;  // reported once, after the loop (an atomic in it slows it)
#pragma unroll
      for (int q = 0; q < kChunkCols; ++q) {
        const int b = b0 + q;
        if (b < batch) {
          const int pos = pos_s[b];
          if (pos < 0 || pos >= ep.max_seq) {
            out_of_cache = true;
          } else {
            cache[static_cast<size_t>(b) * ep.cache_batch_stride +
                  (static_cast<size_t>(kh) * ep.max_seq + pos) * 128 + d] = __float2half_rn(v[q]);
          }
        }
      }
      if (out_of_cache && r == 0) report_error(kDevErrBounds);
    }
  } else if constexpr (KIND == kEpiArgmax) {
    const int n = tile * 128 + r;
    const bool valid = n < ep.n_rows;
#pragma unroll
    for (int q = 0; q < kChunkCols; ++q) tile_s[q * P + r] = valid ? v[q] : -INFINITY;
    epi_sync();
    if (ep.am_rows == 16) {
      // One (max, argmax) per 16 rows, half a warp per group as for the sums.
      const int warp = r >> 5, lane = r & 31;
      const int g = 2 * warp + (lane >> 4), row = lane & 15;
#pragma unroll
      for (int q = 0; q < kChunkCols; ++q) {
        float bv = tile_s[q * P + 16 * g + row];
        int bi = row;
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
          }
        }
        if (row == 0 && b0 + q < batch && tile * 128 + 16 * g < ep.n_rows) {
          const size_t at = static_cast<size_t>(tile * 8 + g) * ep.am_ld + b0 + q;
          ep.am_val[at] = bv;
          ep.am_idx[at] = tile * 128 + 16 * g + bi;
        }
      }
    } else {
      int* aux_i = reinterpret_cast<int*>(aux) + kChunkCols;
      column_argmax(tile_s, tile * 128, aux, aux_i);
      epi_sync();
      if (r < kChunkCols && b0 + r < batch) {
        ep.am_val[static_cast<size_t>(tile) * ep.am_ld + b0 + r] = aux[r];
        ep.am_idx[static_cast<size_t>(tile) * ep.am_ld + b0 + r] = aux_i[r];
      }
    }
    epi_sync();
  }
}

template <int BN, int KIND>
__global__ void __launch_bounds__(kThreads, kCtasPerSm)
    proj_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                const __grid_constant__ EpiParams ep, const uint8_t* __restrict__ w_packed,
                int n_tiles, int kblocks, int stages, int clustered, float* __restrict__ slots,
                uint32_t* __restrict__ counters) {
  using S = ProjShape<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_1024(smem_raw);
  float* tile_s = reinterpret_cast<float*>(smem + stages * S::kStageBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(tile_s) + S::kTileBytes);
  uint64_t* empty = full + stages;
  uint64_t* tfull = empty + stages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* fixbar = drain + 1;  // stream-K owner: other contributors' partials landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(fixbar + 1);
  // Per-token scalars, padded by one chunk so a chunk starting anywhere below
  // BN may read 16 entries.
  float* rn = reinterpret_cast<float*>(tmem_slot + 4);          // [BN+16] RMSNorm scale
  int* pos_s = reinterpret_cast<int*>(rn + BN + kChunkCols);    // [BN+16] token positions
  float* aux = reinterpret_cast<float*>(pos_s + BN + kChunkCols);  // [32] chunk scratch
  volatile int* flags = reinterpret_cast<volatile int*>(aux + 2 * kChunkCols);  // abort, last

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long total = static_cast<long long>(n_tiles) * kblocks;
  const int grid = gridDim.x, cta = blockIdx.x;
  // Work split.  Stream-K: CTA c takes iterations [c*T/G, (c+1)*T/G) of the
  // (tile, k-block) space.  Clustered split-K: the s CTAs of a cluster share
  // one tile, member j taking k-blocks [j*KB/s, (j+1)*KB/s).
  long long it_begin, it_end;
  uint32_t crank = 0, csize = 1;
  if (clustered) {
    crank = cluster_ctarank();
    csize = cluster_nctarank();
    const long long tile = cta / static_cast<int>(csize);
    it_begin = tile * kblocks + static_cast<long long>(crank) * kblocks / csize;
    it_end = tile * kblocks + static_cast<long long>(crank + 1) * kblocks / csize;
  } else {
    it_begin = static_cast<long long>(cta) * total / grid;
    it_end = static_cast<long long>(cta + 1) * total / grid;
  }

  // The next kernel may be scheduled as soon as every CTA of this one is
  // resident; it waits for this grid's results itself (griddepcontrol.wait).
  pdl_launch_dependents();

  if (warp == 4 && lane == 0) {
    prefetch_tensormap(&wmap);
    prefetch_tensormap(&xmap);
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], kEpiThreads);
    }
    mbar_init(drain, 1);
    mbar_init(fixbar, 1);
    flags[0] = 0;
    flags[1] = 0;
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, S::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 4) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const int n_iter = static_cast<int>(it_end - it_begin);
      const int pre = min(stages, n_iter);
      // Packed weights: iteration `it` is the contiguous 16 KB panel `it`.
      auto load_w = [&](uint8_t* st, uint64_t* bar, long long it) {
        if (w_packed != nullptr) {
          bulk_load_hint(st, w_packed + static_cast<size_t>(it) * S::kABytes, S::kABytes, bar,
                         pol_w);
        } else {
          const int tile = static_cast<int>(it / kblocks), kb = static_cast<int>(it % kblocks);
          tma_load_2d_hint(st, &wmap, bar, kb * 64, tile * 128, pol_w);
        }
      };
      // Weights do not depend on the previous kernel: start streaming them
      // before waiting for it; the activations follow once it has finished.
      for (int i = 0; i < pre; ++i) {
        uint8_t* st = smem + i * S::kStageBytes;
        mbar_arrive_expect_tx(&full[i], S::kABytes + S::kBBytes);
        load_w(st, &full[i], it_begin + i);
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i) {
        const int kb = static_cast<int>((it_begin + i) % kblocks);
        tma_load_2d(smem + i * S::kStageBytes + S::kABytes, &xmap, &full[i], kb * 64, 0);
      }
      int issued = pre;
      for (int i = pre; i < n_iter; ++i) {
        const int s = i % stages;
        if (flags[0] || !mbar_wait(&empty[s], ((i / stages) - 1) & 1, kDevErrMmaTimeout)) {
          flags[0] = 1;
          break;
        }
        const long long it = it_begin + i;
        const int kb = static_cast<int>(it % kblocks);
        uint8_t* st = smem + s * S::kStageBytes;
        mbar_arrive_expect_tx(&full[s], S::kABytes + S::kBBytes);
        load_w(st, &full[s], it);
        tma_load_2d(st + S::kABytes, &xmap, &full[s], kb * 64, 0);
        issued = i + 1;
      }
      if (flags[0]) {  // leave no copy in flight into this CTA's shared memory
        for (int i = max(0, issued - stages); i < issued; ++i)
          mbar_wait(&full[i % stages], (i / stages) & 1, kDevErrTmaTimeout);
      }
    }
  } else if (warp == 5) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(128, BN);
      long long it = it_begin;
      int i = 0, seg = 0;
      while (it < it_end && !flags[0]) {
        const int tile = static_cast<int>(it / kblocks);
        const long long seg_end = min(it_end, static_cast<long long>(tile + 1) * kblocks);
        const int acc = seg & 1, use = seg >> 1;
        if (seg >= 2 && !mbar_wait(&tempty[acc], (use - 1) & 1, kDevErrEpilogueTimeout)) {
          flags[0] = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool first = true;
        for (; it < seg_end; ++it, ++i) {
          const int s = i % stages;
          if (flags[0] || !mbar_wait(&full[s], (i / stages) & 1, kDevErrTmaTimeout)) {
            flags[0] = 1;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(smem + s * S::kStageBytes);
          const uint32_t b = a + S::kABytes;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            tc_mma_f16(d_tmem, smem_desc_sw128(a + kk * 32), smem_desc_sw128(b + kk * 32), idesc,
                       (first && kk == 0) ? 0u : 1u);
          first = false;
          tc_commit(&empty[s]);  // the stage is free once these MMAs have read it
        }
        if (flags[0]) break;
        tc_commit(&tfull[acc]);
        ++seg;
      }
      if (flags[0]) {  // no MMA may still write TMEM when it is released
        tc_commit(drain);
        mbar_wait(drain, 0, kDevErrMmaTimeout);
      }
    }
  } else {
    // ---------------- epilogue (tile row r = TMEM lane r) ----------------
    const int r = threadIdx.x;
    pdl_wait();
    if (r < BN + kChunkCols) {
      float scale = 1.f;
      if (ep.ssq_in != nullptr && r < ep.batch) {
        // 16 independent loads per batch: one memory round trip per 16 parts.
        float s = 0.f;
        for (int p0 = 0; p0 < ep.ssq_parts; p0 += 16) {
          float t[16];
#pragma unroll
          for (int j = 0; j < 16; ++j)
            t[j] = p0 + j < ep.ssq_parts ? ep.ssq_in[static_cast<size_t>(p0 + j) * ep.ssq_ld + r] : 0.f;
#pragma unroll
          for (int j = 0; j < 16; ++j) s += t[j];
        }
        scale = rsqrtf(s * ep.ssq_inv_hidden + ep.ssq_eps);
      }
      rn[r] = scale;
      pos_s[r] = (ep.positions != nullptr && r < ep.batch) ? ep.positions[r] : 0;
    }
    epi_sync();
    long long it = it_begin;
    int seg = 0, fix_uses = 0;
    if (clustered) {
      // One segment: keep the FP32 partial in this CTA's own shared memory
      // (the pipeline stages are idle once every MMA has completed) and, when
      // the members reduce through L2 (mode 2), also in this CTA's workspace
      // slot, token by token (128 rows of a token are 512 contiguous bytes).
      const bool bad = flags[0] || !mbar_wait(&tfull[0], 0, kDevErrMmaTimeout);
      if (epi_sync_or(bad)) {
        flags[0] = 1;
      } else {
        tc_fence_after();
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(warp * 32) << 16);
        float* red = reinterpret_cast<float*>(smem);
        const int pitch = clustered == 2 ? 128 : S::kPitch;
        float* slot = clustered == 2 ? slots + static_cast<size_t>(cta) * 128 * BN : nullptr;
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += kChunkCols) {
          uint32_t rr[16];
          tmem_ld16(taddr + c0, rr);
          tmem_ld_wait();
#pragma unroll
          for (int q = 0; q < kChunkCols; ++q) {
            const float x = __uint_as_float(rr[q]);
            red[(c0 + q) * pitch + r] = x;
            if (slot != nullptr) __stcg(slot + (c0 + q) * 128 + r, x);
          }
        }
        tc_fence_before();
        if (slot != nullptr) __threadfence();
      }
      it = it_end;  // skip the stream-K loop
    }
    while (it < it_end) {
      const int tile = static_cast<int>(it / kblocks);
      const int kb0 = static_cast<int>(it % kblocks);
      const long long seg_end = min(it_end, static_cast<long long>(tile + 1) * kblocks);
      const int acc = seg & 1, use = seg >> 1;
      const bool bad = flags[0] || !mbar_wait(&tfull[acc], use & 1, kDevErrMmaTimeout);
      if (epi_sync_or(bad)) {
        flags[0] = 1;
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(warp * 32) << 16) + acc * BN;
      const bool whole = kb0 == 0 && seg_end == static_cast<long long>(tile + 1) * kblocks;
      if (whole) {
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += kChunkCols) {
          uint32_t rr[16];
          tmem_ld16(taddr + c0, rr);
          tmem_ld_wait();
          float v[kChunkCols];
#pragma unroll
          for (int q = 0; q < kChunkCols; ++q) v[q] = __uint_as_float(rr[q]);
          run_epilogue_chunk<KIND>(ep, tile, r, c0, v, rn, tile_s, aux, pos_s, ep.batch);
        }
        tc_fence_before();
        mbar_arrive(&tempty[acc]);
      } else if (kb0 != 0) {
        // Stream-K, a later part of a tile (the first segment of this CTA's
        // range, so it finishes early): publish this CTA's FP32 partial (slot
        // tile + cta is unique), release the accumulator and count the partial
        // for the tile's owner.
        float* slot = slots + static_cast<size_t>(tile + cta) * 128 * BN;
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += kChunkCols) {
          uint32_t rr[16];
          tmem_ld16(taddr + c0, rr);
          tmem_ld_wait();
#pragma unroll
          for (int q = 0; q < kChunkCols; ++q) __stcg(slot + (c0 + q) * 128 + r, __uint_as_float(rr[q]));
        }
        tc_fence_before();
        mbar_arrive(&tempty[acc]);
        __threadfence();
        epi_sync();
        if (r == 0) atomicAdd(&counters[tile], 1u);
      } else {
        // Stream-K, the head of a tile whose later k-blocks other CTAs hold
        // (always the last segment of this CTA's range, so the ring is idle):
        // wait until their partials are counted, bring them into the ring with
        // bulk copies (one round trip), add them to this CTA's accumulator in
        // CTA order -- the order of the k-blocks, so the sum is deterministic
        // -- and run the epilogue.  Partials that do not fit the ring are read
        // from L2 chunk by chunk instead.
        constexpr uint32_t kPartBytes = 128u * BN * 4u;
        const int cl = owner_cta(static_cast<long long>(tile + 1) * kblocks - 1, total, grid);
        const int n_other = cl - cta;
        const bool staged = n_other * kPartBytes <= static_cast<uint32_t>(stages) * S::kStageBytes;
        bool bad = false;
        if (r == 0) {
          bool ready = false;
          for (uint32_t i = 0; i < kMaxPolls && !ready; ++i) {
            ready = ld_acquire_gpu(counters + tile) >= static_cast<uint32_t>(n_other);
            if (!ready) __nanosleep(32);
          }
          if (!ready) report_error(kDevErrEpilogueTimeout);
          bad = !ready;
          if (ready && staged) {
            asm volatile("fence.proxy.async.global;" ::: "memory");
            mbar_arrive_expect_tx(fixbar, n_other * kPartBytes);
            for (int u = 0; u < n_other; ++u)
              bulk_load(smem + u * kPartBytes, slots + static_cast<size_t>(tile + cta + 1 + u) * 128 * BN,
                        kPartBytes, fixbar);
          }
        }
        bad = epi_sync_or(bad);
        if (!bad && staged) bad = epi_sync_or(!mbar_wait(fixbar, fix_uses & 1, kDevErrTmaTimeout));
        ++fix_uses;
        if (bad) {
          flags[0] = 1;
          tc_fence_before();
          mbar_arrive(&tempty[acc]);
          break;
        }
        __threadfence();
        const float* parts = reinterpret_cast<const float*>(smem);
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += kChunkCols) {
          uint32_t rr[16];
          tmem_ld16(taddr + c0, rr);
          tmem_ld_wait();
          float v[kChunkCols];
#pragma unroll
          for (int q = 0; q < kChunkCols; ++q) v[q] = __uint_as_float(rr[q]);
          for (int u = 0; u < n_other; ++u) {
            float t[kChunkCols];
            if (staged) {
              const float* src = parts + static_cast<size_t>(u) * 128 * BN + c0 * 128 + r;
#pragma unroll
              for (int q = 0; q < kChunkCols; ++q) t[q] = src[q * 128];
            } else {
              const float* src = slots + static_cast<size_t>(tile + cta + 1 + u) * 128 * BN + c0 * 128 + r;
#pragma unroll
              for (int q = 0; q < kChunkCols; ++q) t[q] = __ldcg(src + q * 128);
            }
#pragma unroll
            for (int q = 0; q < kChunkCols; ++q) v[q] += t[q];
          }
          run_epilogue_chunk<KIND>(ep, tile, r, c0, v, rn, tile_s, aux, pos_s, ep.batch);
        }
        tc_fence_before();
        mbar_arrive(&tempty[acc]);
        if (r == 0) counters[tile] = 0u;  // leave the workspace reusable
      }
      it = seg_end;
      ++seg;
    }
  }

  if (clustered) {
    // Cross-CTA reduction: member j sums the partials of every member, in rank
    // order, for its share of the tokens and runs the epilogue on them.  Mode
    // 2: the partials are in L2 (each member's workspace slot, published before
    // the cluster barrier); member j brings its tokens of every other member's
    // partial into its idle ring with one bulk copy each -- one round trip.
    // Mode 1 (when those do not fit the ring): member j reads them from the
    // peers' shared memory.
    cluster_sync_all();
    if (warp < 4) {
      const int r = threadIdx.x;
      const int tile = cta / static_cast<int>(csize);
      const int c_begin = static_cast<int>(static_cast<long long>(crank) * ep.batch / csize);
      const int c_end = static_cast<int>(static_cast<long long>(crank + 1) * ep.batch / csize);
      const uint32_t red0 = smem_u32(smem);
      bool ok = !epi_sync_or(flags[0] != 0);
      if (clustered == 2) {
        constexpr uint32_t kTokBytes = 128 * 4;
        const int n_tok = c_end - c_begin;
        uint8_t* recv = smem + BN * kTokBytes;  // [other member][n_tok][128] after the partial
        const bool fetch = ok && n_tok > 0 && csize > 1;
        if (fetch && r == 0) {
          asm volatile("fence.proxy.async.global;" ::: "memory");
          mbar_arrive_expect_tx(fixbar, (csize - 1) * n_tok * kTokBytes);
          int j = 0;
          for (uint32_t m = 0; m < csize; ++m) {
            if (m == crank) continue;
            const float* src = slots + static_cast<size_t>(cta - crank + m) * 128 * BN +
                               static_cast<size_t>(c_begin) * 128;
            bulk_load(recv + static_cast<size_t>(j) * n_tok * kTokBytes, src, n_tok * kTokBytes,
                      fixbar);
            ++j;
          }
        }
        const bool landed = !fetch || mbar_wait(fixbar, 0, kDevErrTmaTimeout);
        ok = !epi_sync_or(!ok || !landed);
        const float* own = reinterpret_cast<const float*>(smem);
        const float* got = reinterpret_cast<const float*>(recv);
        for (int b0 = c_begin; ok && b0 < c_end; b0 += kChunkCols) {
          float v[kChunkCols];
#pragma unroll
          for (int q = 0; q < kChunkCols; ++q) v[q] = 0.f;
          int j = 0;
          for (uint32_t m = 0; m < csize; ++m) {
            const float* src = m == crank
                                   ? own + static_cast<size_t>(b0) * 128 + r
                                   : got + (static_cast<size_t>(j) * n_tok + (b0 - c_begin)) * 128 + r;
#pragma unroll
            for (int q = 0; q < kChunkCols; ++q)
              if (b0 + q < c_end) v[q] += src[q * 128];
            if (m != crank) ++j;
          }
          run_epilogue_chunk<KIND>(ep, tile, r, b0, v, rn, tile_s, aux, pos_s, c_end);
        }
        ok = false;  // done: the shared-memory pull below is for mode 1
      }
      for (int b0 = c_begin; ok && b0 < c_end; b0 += kChunkCols) {
        float v[kChunkCols];
#pragma unroll
        for (int q = 0; q < kChunkCols; ++q) v[q] = 0.f;
        // Loads of up to 4 members in flight together; sums in rank order.
        for (uint32_t m = 0; m < csize; m += 4) {
          float t[4][kChunkCols];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const bool member = m + u < csize;
            const uint32_t base = cluster_map(red0, member ? m + u : 0);
#pragma unroll
            for (int q = 0; q < kChunkCols; ++q)
              t[u][q] = (member && b0 + q < c_end)
                            ? ld_cluster_f32(base + ((b0 + q) * S::kPitch + r) * 4)
                            : 0.f;
          }
#pragma unroll
          for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int q = 0; q < kChunkCols; ++q) v[q] += t[u][q];
        }
        run_epilogue_chunk<KIND>(ep, tile, r, b0, v, rn, tile_s, aux, pos_s, c_end);
      }
    }
    if (clustered == 1) cluster_sync_all();  // no CTA leaves while a peer may still read its partial
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem_base, S::kTmemCols);
  }
}

template <int BN>
int stages_for() {
  using S = ProjShape<BN>;
  const int budget = kSmemPerSm / kCtasPerSm - kSmemReserved;
  const int fixed = 1024 + S::kTileBytes + S::kMiscBytes;
  int st = (budget - fixed) / S::kStageBytes;
  return st > kMaxStages ? kMaxStages : st;
}

template <int BN>
size_t smem_for(int stages) {
  using S = ProjShape<BN>;
  return 1024 + static_cast<size_t>(stages) * S::kStageBytes + S::kTileBytes + S::kMiscBytes;
}

int bn_for(int batch) { return batch <= 16 ? 16 : batch <= 32 ? 32 : batch <= 64 ? 64 : 128; }

constexpr int kMaxCluster = 8;  // portable thread-block cluster size

template <int BN>
int stages_for();
template <int BN>
size_t smem_for(int stages);

// Stand-in with proj_kernel's launch shape (threads, CTAs per SM, dynamic
// shared memory) for cluster-occupancy queries.  For proj_kernel itself the
// occupancy API reports one CTA per SM, while the hardware co-schedules two
// (measured: 32 clusters of 8 start together); the stand-in's answer matches
// what is observed.
__global__ void __launch_bounds__(kThreads, kCtasPerSm) proj_shape_twin(int* never) {
  if (never) never[threadIdx.x] = 0;
}

// How many clusters of `s` CTAs (with proj_kernel<BN>'s shape) can be
// resident at once (cached; depends on how clusters pack into GPCs, not only
// on the SM count).  Falls back to a conservative estimate without a device.
template <int BN>
int max_active_clusters(int s) {
  static int cache[64][kMaxCluster + 1] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  if (cache[dev][s] != 0) return cache[dev][s];
  int n = 0;
  const size_t smem = smem_for<BN>(stages_for<BN>());
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(s * 64);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = s;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  if (cudaFuncSetAttribute(proj_shape_twin, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess ||
      cudaOccupancyMaxActiveClusters(&n, proj_shape_twin, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = (sm_count() * kCtasPerSm * 3 / 5) / s;  // no device: leave ~40% slack for packing
  }
  cache[dev][s] = n;
  return n;
}

int max_clusters(int bn, int s) {
  switch (bn) {
    case 16: return max_active_clusters<16>(s);
    case 32: return max_active_clusters<32>(s);
    case 64: return max_active_clusters<64>(s);
    default: return max_active_clusters<128>(s);
  }
}

struct Geometry {
  int bn, n_tiles, kblocks, grid;
  int split;       // > 0: clustered split-K with `split` CTAs per tile; 0: stream-K
  int mode;        // kernel's `clustered`: 0 stream-K, 1 reduce in shared memory, 2 through L2
  size_t counter_bytes, slot_bytes;
};

// Bytes of proj_kernel<bn>'s ring (idle once the k-loop is done).
size_t ring_bytes(int bn) {
  switch (bn) {
    case 16: return static_cast<size_t>(stages_for<16>()) * ProjShape<16>::kStageBytes;
    case 32: return static_cast<size_t>(stages_for<32>()) * ProjShape<32>::kStageBytes;
    case 64: return static_cast<size_t>(stages_for<64>()) * ProjShape<64>::kStageBytes;
    default: return static_cast<size_t>(stages_for<128>()) * ProjShape<128>::kStageBytes;
  }
}

// Few tiles (fewer than one per CTA slot): split each tile's K over a cluster
// and reduce through distributed shared memory -- no global scratch, no
// serialized fix-up.  The cluster size is the largest for which every cluster
// is resident at once, with slack: a second wave of clusters would double the
// time.
// Many tiles: stream-K over every CTA slot, where a tile has at most a couple
// of contributors.
Geometry geometry(int n_rows, int k, int batch) {
  Geometry g;
  g.bn = bn_for(batch);
  g.n_tiles = (n_rows + 127) / 128;
  g.kblocks = k / 64;
  const long long total = static_cast<long long>(g.n_tiles) * g.kblocks;
  const long long slots_total = static_cast<long long>(sm_count()) * kCtasPerSm;
  g.split = 0;
  if (2ll * g.n_tiles <= slots_total) {
    // Keep an eighth of the cluster slots free: with none spare, clusters
    // placed while the previous kernel's CTAs still hold SMs fragment the
    // GPCs, and the last clusters wait for a second wave (measured after the
    // attention: o_proj's last 5% of CTAs started ~15 us after it ended).
    int best = 1;
    for (int s = 2; s <= kMaxCluster && g.kblocks / s >= 2; ++s)
      if (8 * g.n_tiles <= 7 * max_clusters(g.bn, s)) best = s;
    g.split = best;
    g.grid = g.n_tiles * best;
    // Through L2 when the member's partial and its tokens of the others'
    // partials fit the ring; each member then needs a workspace slot.
    const size_t tok_max = (static_cast<size_t>(batch) + best - 1) / best;
    const size_t staged = static_cast<size_t>(g.bn) * 512 + (best - 1) * tok_max * 512;
    g.mode = best > 1 && staged <= ring_bytes(g.bn) ? 2 : 1;
    // The slots start after the stream-K counters, which a workspace shared
    // between projections must keep zero-filled.
    g.counter_bytes = g.mode == 2 ? kCounterBytes : 0;
    g.slot_bytes = g.mode == 2 ? static_cast<size_t>(g.grid) * 128 * g.bn * 4 : 0;
    return g;
  }
  g.grid = static_cast<int>(total < slots_total ? total : slots_total);
  g.mode = 0;
  g.counter_bytes = kCounterBytes;
  g.slot_bytes = static_cast<size_t>(g.n_tiles + g.grid - 1) * 128 * g.bn * 4;
  return g;
}

template <int BN, int KIND>
int launch_proj_kind(const CUtensorMap& wm, const CUtensorMap& xm, const EpiParams& ep,
                     const uint8_t* w_packed, const Geometry& g, float* slots, uint32_t* counters,
                     cudaStream_t stream, bool pdl) {
  const int stages = stages_for<BN>();
  const size_t smem = smem_for<BN>(stages);
  auto kern = proj_kernel<BN, KIND>;
  NPU_TRY_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(smem)));
  LaunchCfg cfg;
  cfg.grid = dim3(g.grid);
  cfg.block = dim3(kThreads);
  cfg.smem = smem;
  cfg.stream = stream;
  cfg.pdl = pdl;
  cfg.cluster = g.split > 1 ? g.split : 1;
  return launch(cfg, kern, wm, xm, ep, w_packed, g.n_tiles, g.kblocks, stages, g.mode, slots,
                counters);
}

template <int BN>
int launch_proj(const CUtensorMap& wm, const CUtensorMap& xm, const EpiParams& ep,
                const uint8_t* w_packed, const Geometry& g, float* slots, uint32_t* counters,
                cudaStream_t stream, bool pdl) {
  switch (ep.kind) {
    case kEpiStore:
      if (ep.px.seq >= 0)
        return launch_proj_kind<BN, kEpiStorePeer>(wm, xm, ep, w_packed, g, slots, counters, stream,
                                                   pdl);
      return launch_proj_kind<BN, kEpiStore>(wm, xm, ep, w_packed, g, slots, counters, stream, pdl);
    case kEpiResid:
      return launch_proj_kind<BN, kEpiResid>(wm, xm, ep, w_packed, g, slots, counters, stream, pdl);
    case kEpiSwiGLU:
      return launch_proj_kind<BN, kEpiSwiGLU>(wm, xm, ep, w_packed, g, slots, counters, stream,
                                              pdl);
    case kEpiQKV:
      return launch_proj_kind<BN, kEpiQKV>(wm, xm, ep, w_packed, g, slots, counters, stream, pdl);
    default:
      return launch_proj_kind<BN, kEpiArgmax>(wm, xm, ep, w_packed, g, slots, counters, stream,
                                              pdl);
  }
}

// One thread per 16-byte chunk of the source: row i, chunk c (elements 8c..8c+7)
// goes to panel (tile, kb) = (row / 128, c / 8), row r = row % 128, chunk slot
// (c % 8) ^ (r % 8): the layout TMA's 128-byte swizzle would leave in shared
// memory, so a plain bulk copy of the panel feeds the MMA directly.
__global__ void pack_panels_kernel(const __half* __restrict__ src, size_t src_pitch,
                                   int n_src_rows, int k, uint8_t* __restrict__ dst, int kblocks,
                                   int row_mode, int row_offset) {
  const int chunks = k / 8;
  const size_t total = static_cast<size_t>(n_src_rows) * chunks;
  for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int i = static_cast<int>(idx / chunks), c = static_cast<int>(idx % chunks);
    // 0: identity; 1: gate/up interleave (row 2i + offset); 2: head dims in
    // rotate_half pair order (dim d of a 128-row head -> row 2d or 2(d-64)+1).
    const int hd = i & 127;
    const int row = row_mode == 0   ? row_offset + i
                    : row_mode == 1 ? 2 * i + row_offset
                                    : row_offset + (i & ~127) + (hd < 64 ? 2 * hd : 2 * (hd - 64) + 1);
    const int t = row >> 7, r = row & 127, kb = c >> 3, j = c & 7;
    const size_t off = (static_cast<size_t>(t) * kblocks + kb) * 16384 + r * 128 + ((j ^ (r & 7)) << 4);
    *reinterpret_cast<uint4*>(dst + off) =
        *reinterpret_cast<const uint4*>(src + static_cast<size_t>(i) * src_pitch + 8 * c);
  }
}

}  // namespace

size_t proj_workspace_bytes(int n_rows, int k, int batch) {
  if (n_rows < 1 || k < 64 || batch < 1) return 0;
  const Geometry g = geometry(n_rows, k, batch);
  return g.counter_bytes + g.slot_bytes;
}

size_t packed_weight_bytes(int n_rows, int k) {
  if (n_rows < 1 || k < 64) return 0;
  return static_cast<size_t>((n_rows + 127) / 128) * 128 * k * 2;
}

int pack_weight(const void* src, size_t src_pitch, int n_src_rows, int k, void* dst,
                int dst_rows, int row_mode, int row_offset, cudaStream_t stream) {
  NPU_REQUIRE(src && dst, "pack: null pointer");
  NPU_REQUIRE(k >= 64 && k % 64 == 0 && n_src_rows >= 1 && src_pitch >= static_cast<size_t>(k),
              "pack: K must be a positive multiple of 64 (K=%d)", k);
  NPU_REQUIRE((reinterpret_cast<uintptr_t>(src) & 15) == 0 && (src_pitch * 2) % 16 == 0 &&
                  (reinterpret_cast<uintptr_t>(dst) & 15) == 0,
              "pack: source rows and destination must be 16-byte aligned");
  NPU_REQUIRE(row_mode >= 0 && row_mode <= 2, "pack: unknown row mode %d", row_mode);
  NPU_REQUIRE(row_mode != 2 || (n_src_rows % 128 == 0 && row_offset % 128 == 0),
              "pack: head-pair order needs whole 128-row heads");
  const int last = row_mode == 1 ? 2 * (n_src_rows - 1) + row_offset : row_offset + n_src_rows - 1;
  NPU_REQUIRE(row_offset >= 0 && last < ((dst_rows + 127) / 128) * 128,
              "pack: rows land outside the destination");
  LaunchCfg cfg;
  const size_t total = static_cast<size_t>(n_src_rows) * (k / 8);
  cfg.grid = dim3(static_cast<unsigned>(total / 256 + 1 < 4096 ? total / 256 + 1 : 4096));
  cfg.block = dim3(256);
  cfg.stream = stream;
  return launch(cfg, pack_panels_kernel, static_cast<const __half*>(src), src_pitch, n_src_rows, k,
                static_cast<uint8_t*>(dst), k / 64, row_mode, row_offset);
}

int proj_run(const void* w, bool w_packed, const void* x, int n_rows, int k, int batch,
             const EpiParams& ep, void* workspace, size_t workspace_bytes, cudaStream_t stream,
             bool pdl) {
  NPU_REQUIRE(w && x, "projection: null weight or activation pointer");
  NPU_REQUIRE(n_rows >= 1 && k >= 64 && k % 64 == 0,
              "projection: need rows >= 1 and K a positive multiple of 64 (rows=%d K=%d)", n_rows,
              k);
  NPU_REQUIRE(batch >= 1 && batch <= 128, "projection: batch %d not in [1, 128]", batch);
  NPU_REQUIRE((n_rows + 127) / 128 <= kMaxTiles, "projection: %d rows exceed %d tiles", n_rows,
              kMaxTiles);
  NPU_REQUIRE(ep.batch == batch && ep.n_rows == n_rows, "projection: epilogue shape mismatch");
  NPU_REQUIRE((reinterpret_cast<uintptr_t>(w) & 15) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0,
              "projection: W and X must be 16-byte aligned");
  if (ep.kind == kEpiQKV)
    NPU_REQUIRE(n_rows == (ep.q_heads + 2 * ep.kv_heads) * 128 && ep.positions && ep.inv_freq &&
                    ep.k_cache && ep.v_cache && ep.out && ep.max_seq > 0,
                "projection: QKV epilogue needs 128-dim heads, positions, RoPE table and caches");
  if (ep.kind == kEpiSwiGLU)
    NPU_REQUIRE(n_rows % 128 == 0 && ep.out, "projection: SwiGLU rows must be [gate64|up64] blocks");
  if (ep.kind == kEpiResid)
    NPU_REQUIRE(ep.resid && ep.norm_w && ep.xw && ep.ssq_out,
                "projection: residual epilogue needs resid, norm weight, xw and ssq outputs");
  if (ep.kind == kEpiArgmax)
    NPU_REQUIRE(ep.am_val && ep.am_idx && ep.am_ld >= batch && (ep.am_rows == 16 || ep.am_rows == 128),
                "projection: argmax outputs need am_ld >= batch and 16 or 128 rows per partial");
  if (ep.kind == kEpiResid)
    NPU_REQUIRE(ep.ssq_out_ld >= batch && (ep.ssq_out_rows == 16 || ep.ssq_out_rows == 128),
                "projection: sums of squares need ssq_out_ld >= batch and 16 or 128 rows per partial");
  if (ep.kind == kEpiStore)
    NPU_REQUIRE(ep.out != nullptr || ep.px.seq >= 0, "projection: null output");
  if (ep.px.seq >= 0)
    NPU_REQUIRE((ep.kind == kEpiStore || (ep.kind == kEpiResid && w_packed &&
                                          gemv_supported(n_rows, k, batch, ep))) &&
                    ep.px.ranks >= 1 && ep.px.ranks <= kMaxRanks && ep.px.seq < kArgmaxSeq &&
                    ep.n_rows == ep.px.hidden && batch <= ep.px.max_batch && ep.px.epoch,
                "projection: peer exchange needs a STORE of all hidden rows, or a residual "
                "epilogue on the GEMV path");
  NPU_REQUIRE(ep.kind >= kEpiStore && ep.kind <= kEpiArgmax, "projection: unknown epilogue %d",
              ep.kind);
  NPU_REQUIRE(ep.ssq_in == nullptr || (ep.ssq_parts >= 1 && ep.ssq_ld >= batch),
              "projection: RMSNorm input needs ssq_parts >= 1 and ssq_ld >= batch");

  if (w_packed && gemv_supported(n_rows, k, batch, ep))
    return gemv_run(w, x, n_rows, k, batch, ep, stream, pdl);

  if (w_packed && gemv_supported(n_rows, k, batch, ep))
    return gemv_run(w, x, n_rows, k, batch, ep, stream, pdl);

  const Geometry g = geometry(n_rows, k, batch);
  const size_t need = g.counter_bytes + g.slot_bytes;
  NPU_REQUIRE(need == 0 || (workspace && workspace_bytes >= need),
              "projection: workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  NPU_REQUIRE(need == 0 || (reinterpret_cast<uintptr_t>(workspace) & 255) == 0,
              "projection: workspace must be 256-byte aligned");
  CUtensorMap wm, xm;
  int rc = 0;
  if (w_packed)
    memset(&wm, 0, sizeof(wm));
  else if ((rc = make_tensor_map_2d(&wm, w, n_rows, k, 128, 64)))
    return rc;
  if ((rc = make_tensor_map_2d(&xm, x, batch, k, g.bn, 64))) return rc;
  uint32_t* counters = need ? static_cast<uint32_t*>(workspace) : nullptr;
  float* slots =
      need ? reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + g.counter_bytes) : nullptr;
  const uint8_t* wp = w_packed ? static_cast<const uint8_t*>(w) : nullptr;
  switch (g.bn) {
    case 16: return launch_proj<16>(wm, xm, ep, wp, g, slots, counters, stream, pdl);
    case 32: return launch_proj<32>(wm, xm, ep, wp, g, slots, counters, stream, pdl);
    case 64: return launch_proj<64>(wm, xm, ep, wp, g, slots, counters, stream, pdl);
    default: return launch_proj<128>(wm, xm, ep, wp, g, slots, counters, stream, pdl);
  }
}

}  // namespace npu_b200

using namespace npu_b200;

extern "C" size_t npu_b200_linear_workspace_size(int n_rows, int k, int batch) {
  return proj_workspace_bytes(n_rows, k, batch);
}

extern "C" size_t npu_b200_packed_weight_bytes(int n_rows, int k) {
  return packed_weight_bytes(n_rows, k);
}

extern "C" int npu_b200_pack_weight(const void* d_w, int n_rows, int k, void* d_packed,
                                    void* stream) {
  clear_error();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  NPU_REQUIRE(d_packed, "pack: null destination");
  NPU_TRY_CUDA(cudaMemsetAsync(d_packed, 0, packed_weight_bytes(n_rows, k), s));
  return pack_weight(d_w, static_cast<size_t>(k), n_rows, k, d_packed, n_rows, 0, 0, s);
}

extern "C" int npu_b200_pack_weight_rows(const void* d_w, int n_src_rows, int k, void* d_packed,
                                         int dst_rows, int order, int row_offset, void* stream) {
  clear_error();
  NPU_REQUIRE(order == NPU_B200_PACK_IDENTITY || order == NPU_B200_PACK_INTERLEAVE ||
                  order == NPU_B200_PACK_HEAD_PAIRS,
              "pack: unknown row order %d", order);
  return pack_weight(d_w, static_cast<size_t>(k), n_src_rows, k, d_packed, dst_rows, order,
                     row_offset, static_cast<cudaStream_t>(stream));
}

extern "C" int npu_b200_linear(const void* d_x, const void* d_w, const void* d_bias, void* d_out,
                               int batch, int n_rows, int k, int flags, void* d_workspace,
                               size_t workspace_bytes, void* stream) {
  clear_error();
  NPU_REQUIRE((flags & ~(NPU_B200_LINEAR_RELU | NPU_B200_LINEAR_OUT_F32 |
                         NPU_B200_LINEAR_PACKED_W)) == 0,
              "linear: unknown flags 0x%x", flags);
  EpiParams ep;
  ep.kind = kEpiStore;
  ep.n_rows = n_rows;
  ep.batch = batch;
  ep.out = d_out;
  ep.ld_out = n_rows;
  ep.out_f32 = (flags & NPU_B200_LINEAR_OUT_F32) ? 1 : 0;
  ep.relu = (flags & NPU_B200_LINEAR_RELU) ? 1 : 0;
  ep.bias = static_cast<const __half*>(d_bias);
  return proj_run(d_w, (flags & NPU_B200_LINEAR_PACKED_W) != 0, d_x, n_rows, k, batch, ep,
                  d_workspace, workspace_bytes, static_cast<cudaStream_t>(stream), false);
}

extern "C" int npu_b200_projection(const void* d_x, const void* d_w, int w_packed, int batch,
                                   int n_rows, int k, const npu_b200_epilogue* e, void* d_workspace,
                                   size_t workspace_bytes, void* stream) {
  clear_error();
  NPU_REQUIRE(e != nullptr, "projection: null epilogue");
  EpiParams ep;
  ep.kind = e->kind;
  ep.n_rows = n_rows;
  ep.batch = batch;
  ep.ssq_in = e->ssq_in;
  ep.ssq_parts = e->ssq_parts;
  ep.ssq_ld = e->ssq_ld;
  ep.ssq_inv_hidden = e->hidden > 0 ? 1.f / static_cast<float>(e->hidden) : 0.f;
  ep.ssq_eps = e->ssq_eps;
  ep.out = e->out;
  ep.ld_out = e->ld_out;
  ep.out_f32 = e->out_f32;
  ep.relu = e->relu;
  ep.bias = static_cast<const __half*>(e->bias);
  ep.resid = e->resid;
  ep.ld_resid = e->ld_resid;
  ep.norm_w = static_cast<const __half*>(e->norm_w);
  ep.xw = static_cast<__half*>(e->xw);
  ep.ld_xw = e->ld_xw;
  ep.ssq_out = e->ssq_out;
  ep.ssq_out_ld = e->ssq_out_ld;
  ep.q_heads = e->q_heads;
  ep.kv_heads = e->kv_heads;
  ep.positions = e->positions;
  ep.inv_freq = e->inv_freq;
  ep.k_cache = static_cast<__half*>(e->k_cache);
  ep.v_cache = static_cast<__half*>(e->v_cache);
  ep.max_seq = e->max_seq;
  ep.cache_batch_stride = e->kv_heads * e->max_seq * 128;
  ep.q_norm_w = static_cast<const __half*>(e->q_norm_w);
  ep.k_norm_w = static_cast<const __half*>(e->k_norm_w);
  ep.qk_eps = e->qk_eps;
  ep.am_val = e->am_val;
  ep.am_idx = e->am_idx;
  ep.am_ld = e->am_ld;
  ep.ssq_out_rows = e->ssq_out_rows == 0 ? 128 : e->ssq_out_rows;
  ep.am_rows = e->am_rows == 0 ? 128 : e->am_rows;
  NPU_REQUIRE(ep.ssq_in == nullptr || e->hidden > 0, "projection: RMSNorm input needs hidden");
  return proj_run(d_w, w_packed != 0, d_x, n_rows, k, batch, ep, d_workspace, workspace_bytes,
                  static_cast<cudaStream_t>(stream), false);
}
