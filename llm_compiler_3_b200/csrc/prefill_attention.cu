// Multi-query (prefill) attention for sm_100a on tcgen05 tensor cores.
//
// Semantics follow npu.attention with M >= 1 queries per head
// (include/npu/Dialect/NPUDialect.td:31-61, verifier lib/Dialect/NPUDialect.cpp:70-92)
// and its causal form: the frontend's is_causal mask shows key j to query i iff
// j <= i, torch's top-left alignment (lib/Transforms/Attention.cpp:70-92; the
// expansion masks the diagonal block and skips the blocks past it, 221-222).
// Generalised for a KV cache: query i of sequence b sits at position
// q_start[b] + i and sees keys [0, min(q_start[b] + i, keys - 1)]; q_start = 0 is
// the reference's mask.  Scores, the running max and sum and the output
// accumulator are FP32 (the NPU rounds each VPU op to FP16,
// lib/Transforms/Emit.cpp:932-1024); P is rounded to FP16 as the second MMA's
// operand, exactly as the NPU feeds its matrix unit; the output is rounded once.
//
// Work decomposition: one CTA of 128 threads per (query block, head subgroup,
// KV head, sequence).  Its 128 rows are `hp` query heads of one GQA group x `bm`
// queries, so the K/V tiles a group shares are read once for all of them (the
// reference stacks a group's heads the same way, Attention.cpp:213-215).
// Thread t owns row t, which is TMEM lane t of both accumulators.  Per 64-key
// tile:
//   S = Q K^T   one thread issues tcgen05.mma M=128 N=64 K=head_dim (Q and K
//               K-major, 128-byte swizzle) into TMEM columns [0, 64)
//   softmax     each thread reads its row of S from TMEM, updates its running
//               max and sum, and writes P = exp2(S * scale * log2 e - max) as
//               FP16 into shared memory (K-major, the A operand of the next MMA)
//   O_t = P V   tcgen05.mma M=128 N=head_dim K=64 into TMEM columns
//               [64, 64 + head_dim); V^T is written K-major by the threads that
//               load V, and acc = alpha * acc + O_t in registers.
// K of the next tile streams in by cp.async and V into registers while this
// tile's softmax runs; two CTAs share an SM, so one CTA's MMAs overlap the
// other's softmax.  Every wait is bounded and reports into the device error word.
#include <math.h>

#include <algorithm>

#include "common.cuh"
#include "host.hpp"

namespace npu_b200 {
namespace {

constexpr int kRows = 128;    // query rows per CTA: MMA M, TMEM lanes
constexpr int kKeys = 64;     // keys per tile: score MMA N, PV MMA K
constexpr int kThreads = 128; // one thread per row

template <int D>
struct PaShape {
  static constexpr int kAtoms = (D + 63) / 64;          // 128-byte K-major atoms per Q/K row
  static constexpr int kQBytes = kAtoms * kRows * 128;  // Q tile
  static constexpr int kKBytes = kAtoms * kKeys * 128;  // K tile
  static constexpr int kVBytes = D * 128;               // V^T tile: D rows x 64 keys
  static constexpr int kPBytes = kRows * 128;           // P tile: 128 rows x 64 keys
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + kQBytes;
  static constexpr int kV = kK + kKBytes;
  static constexpr int kP = kV + kVBytes;
  static constexpr int kBars = kP + kPBytes;            // 3 mbarriers + TMEM address
  static constexpr int kSmem = kBars + 64 + 1024;       // + slack to align the base to 1024
  static constexpr int kTmemCols = kKeys + D <= 128 ? 128 : 256;
  static constexpr int kVBlocks = D / 16;               // 16-dim blocks of a V row
  static constexpr int kVBlocksPerWarp = (kVBlocks + 3) / 4;
};

__device__ __forceinline__ uint8_t* align_1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// Byte offset of 16-byte chunk `chunk` (8 FP16 columns) of row `row` in a
// K-major tile of `rows` rows stored as 128-byte-swizzled atoms: atom
// chunk / 8 holds 64 columns of every row, rows 128 bytes apart, and chunk c of
// row r sits at position c ^ (r % 8) -- the layout a TMA load with the 128-byte
// swizzle writes and the tcgen05 descriptor (smem_desc_sw128) reads.
__device__ __forceinline__ uint32_t kmajor_offset(int rows, int row, int chunk) {
  return static_cast<uint32_t>((chunk >> 3) * rows * 128 + row * 128 + (((chunk & 7) ^ (row & 7)) << 4));
}

__device__ __forceinline__ void st_shared_u32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

template <int D>
__global__ void __launch_bounds__(kThreads, 2)
    prefill_attention_kernel(const __half* __restrict__ q, const __half* __restrict__ k,
                             const __half* __restrict__ v, const int32_t* __restrict__ q_start,
                             __half* __restrict__ out, int q_heads, int kv_heads, int queries,
                             int keys, int max_seq, int bm, int hp, int q_blocks,
                             float scale_log2, int causal) {
  using S = PaShape<D>;
  constexpr int kChunks = D / 8;  // 16-byte chunks of a Q/K/V row
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_1024(smem_raw);
  const uint32_t s_base = smem_u32(smem);
  const uint32_t sQ = s_base + S::kQ, sK = s_base + S::kK, sV = s_base + S::kV,
                 sP = s_base + S::kP;
  uint64_t* bar_s = reinterpret_cast<uint64_t*>(smem + S::kBars);
  uint64_t* bar_o = bar_s + 1;
  uint64_t* bar_drain = bar_s + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_s + 3);

  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int group = q_heads / kv_heads;
  const int subgroups = group / hp;
  // Last query blocks first: under the causal mask they see the most keys.  The
  // block index is the grid's slow dimension (y), so CTAs are dispatched
  // heaviest first across every head and sequence.
  const int qb = q_blocks - 1 - static_cast<int>(blockIdx.y) / subgroups;
  const int gs = static_cast<int>(blockIdx.y) % subgroups;
  const int hk = static_cast<int>(blockIdx.x) % kv_heads;
  const int b = static_cast<int>(blockIdx.x) / kv_heads;
  const int m0 = qb * bm;
  const long long qs = q_start != nullptr ? q_start[b] : 0;
  const size_t kv_base = (static_cast<size_t>(b) * kv_heads + hk) * max_seq;

  // This thread's row: head gs * hp + g of the group, query m0 + i.
  const int g = t / bm, i = t % bm;
  const int h = hk * group + gs * hp + g;
  const bool row_ok = g < hp && m0 + i < queries;
  long long last = keys - 1;  // last key the row sees (< 0: none)
  if (causal) last = min(last, qs + m0 + i);
  if (!row_ok) last = -1;
  // Tiles that any row of the CTA sees.
  long long cta_last = keys - 1;
  if (causal) cta_last = min(cta_last, qs + min(m0 + bm, queries) - 1);
  const int n_tiles = cta_last >= 0 ? static_cast<int>(cta_last / kKeys) + 1 : 0;

  if (t == 0) {
    mbar_init(bar_s, 1);
    mbar_init(bar_o, 1);
    mbar_init(bar_drain, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, S::kTmemCols);
    tmem_relinquish();
  }

  // Q tile; rows past the block or the subgroup are zero.
  for (int c = t; c < kRows * kChunks; c += kThreads) {
    const int r = c / kChunks, ch = c % kChunks;
    const int rg = r / bm, ri = r % bm;
    const bool ok = rg < hp && m0 + ri < queries;
    const size_t row =
        ok ? (static_cast<size_t>(b) * q_heads + hk * group + gs * hp + rg) * queries + m0 + ri : 0;
    cp_async_16(sQ + kmajor_offset(kRows, r, ch), q + row * D + ch * 8, ok);
  }
  // K tile `tile`; keys past `keys` are zero.
  auto load_k = [&](int tile) {
    const int key0 = tile * kKeys;
    for (int c = t; c < kKeys * kChunks; c += kThreads) {
      const int r = c / kChunks, ch = c % kChunks;
      const bool ok = key0 + r < keys;
      const size_t row = kv_base + (ok ? key0 + r : 0);
      cp_async_16(sK + kmajor_offset(kKeys, r, ch), k + row * D + ch * 8, ok);
    }
    cp_async_commit();
  };
  // V tile `tile` into registers: lane l holds keys 2l and 2l+1, warp w the
  // 16-dim blocks w, w + 4, ...; keys past `keys` are zero (P is 0 there, and
  // 0 x garbage could be NaN).
  uint4 vr[S::kVBlocksPerWarp][4];
  auto fetch_v = [&](int tile) {
    const int ka = tile * kKeys + 2 * lane, kb = ka + 1;
#pragma unroll
    for (int u = 0; u < S::kVBlocksPerWarp; ++u) {
      const int blk = warp + 4 * u;
      const uint4 z = make_uint4(0u, 0u, 0u, 0u);
      if (blk < S::kVBlocks) {
        const uint4* pa = reinterpret_cast<const uint4*>(v + (kv_base + ka) * D + blk * 16);
        const uint4* pb = reinterpret_cast<const uint4*>(v + (kv_base + kb) * D + blk * 16);
        vr[u][0] = ka < keys ? __ldg(pa) : z;
        vr[u][1] = ka < keys ? __ldg(pa + 1) : z;
        vr[u][2] = kb < keys ? __ldg(pb) : z;
        vr[u][3] = kb < keys ? __ldg(pb + 1) : z;
      }
    }
  };
  // The fetched tile as V^T (row d, keys 2l and 2l+1 in one 32-bit word), K-major:
  // a warp's 32 words for one d fill one 128-byte row, so the stores never conflict.
  auto store_v = [&]() {
#pragma unroll
    for (int u = 0; u < S::kVBlocksPerWarp; ++u) {
      const int blk = warp + 4 * u;
      if (blk < S::kVBlocks) {
        const uint32_t wa[8] = {vr[u][0].x, vr[u][0].y, vr[u][0].z, vr[u][0].w,
                                vr[u][1].x, vr[u][1].y, vr[u][1].z, vr[u][1].w};
        const uint32_t wb[8] = {vr[u][2].x, vr[u][2].y, vr[u][2].z, vr[u][2].w,
                                vr[u][3].x, vr[u][3].y, vr[u][3].z, vr[u][3].w};
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int d = blk * 16 + e;
          const uint32_t word = (e & 1) ? __byte_perm(wa[e >> 1], wb[e >> 1], 0x7632)
                                        : __byte_perm(wa[e >> 1], wb[e >> 1], 0x5410);
          st_shared_u32(sV + d * 128 + ((((lane >> 2) ^ (d & 7)) << 4) | ((lane & 3) << 2)), word);
        }
      }
    }
  };

  if (n_tiles > 0) {
    load_k(0);  // one cp.async group with the Q tile
    fetch_v(0);
  } else {
    cp_async_commit();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_row = tmem + (static_cast<uint32_t>(warp * 32) << 16);  // this warp's lanes

  float acc[D];
#pragma unroll
  for (int c = 0; c < D; ++c) acc[c] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;
  bool bad = false;
  for (int j = 0; j < n_tiles; ++j) {
    cp_async_wait_all();  // this thread's part of K_j (and Q)
    store_v();            // V_j^T: the previous P V has read the old one
    fence_proxy_async_smem();
    tc_fence_before();
    if (__syncthreads_or(bad)) {
      bad = true;
      break;
    }
    if (t == 0) {
      tc_fence_after();
      constexpr uint32_t idesc = idesc_f16_f32(kRows, kKeys);
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk)
        tc_mma_f16(tmem, smem_desc_sw128(sQ + (kk >> 2) * (kRows * 128) + (kk & 3) * 32),
                   smem_desc_sw128(sK + (kk >> 2) * (kKeys * 128) + (kk & 3) * 32), idesc,
                   kk > 0 ? 1u : 0u);
      tc_commit(bar_s);
    }
    if (j + 1 < n_tiles) fetch_v(j + 1);
    bad = !mbar_wait(bar_s, j & 1, kDevErrMmaTimeout) || bad;
    tc_fence_after();
    if (!bad && j + 1 < n_tiles) load_k(j + 1);  // the score MMA has read K_j

    // Online softmax of this row over tile j.
    const int key0 = j * kKeys;
    float mx = -INFINITY;
#pragma unroll
    for (int c = 0; c < kKeys; c += 16) {
      uint32_t rr[16];
      tmem_ld16(t_row + c, rr);
      tmem_ld_wait();
#pragma unroll
      for (int e = 0; e < 16; ++e)
        if (key0 + c + e <= last) mx = fmaxf(mx, __uint_as_float(rr[e]) * scale_log2);
    }
    const float m_new = fmaxf(m_run, mx);
    const float alpha = m_run == -INFINITY ? 0.f : fast_exp2(m_run - m_new);
    float sum = 0.f;
#pragma unroll
    for (int c = 0; c < kKeys; c += 16) {
      uint32_t rr[16];
      tmem_ld16(t_row + c, rr);
      tmem_ld_wait();
      uint32_t pk[8];
#pragma unroll
      for (int e = 0; e < 16; e += 2) {
        const float p0 =
            key0 + c + e <= last ? fast_exp2(__uint_as_float(rr[e]) * scale_log2 - m_new) : 0.f;
        const float p1 = key0 + c + e + 1 <= last
                             ? fast_exp2(__uint_as_float(rr[e + 1]) * scale_log2 - m_new)
                             : 0.f;
        pk[e >> 1] = pack_half2(p0, p1);
        // The sum takes the FP16 weights the MMA multiplies by.
        const float2 pr = __half22float2(*reinterpret_cast<const __half2*>(&pk[e >> 1]));
        sum += pr.x + pr.y;
      }
      const int ch = c >> 3;  // keys c..c+15: chunks ch, ch + 1 of row t
      st_shared_v4(sP + t * 128 + ((ch ^ (t & 7)) << 4), pk[0], pk[1], pk[2], pk[3]);
      st_shared_v4(sP + t * 128 + (((ch + 1) ^ (t & 7)) << 4), pk[4], pk[5], pk[6], pk[7]);
    }
    l_run = l_run * alpha + sum;
    m_run = m_new;

    fence_proxy_async_smem();
    tc_fence_before();
    if (__syncthreads_or(bad)) {
      bad = true;
      break;
    }
    if (t == 0) {
      tc_fence_after();
      constexpr uint32_t idesc = idesc_f16_f32(kRows, D);
#pragma unroll
      for (int kk = 0; kk < kKeys / 16; ++kk)
        tc_mma_f16(tmem + kKeys, smem_desc_sw128(sP + kk * 32), smem_desc_sw128(sV + kk * 32),
                   idesc, kk > 0 ? 1u : 0u);
      tc_commit(bar_o);
    }
    bad = !mbar_wait(bar_o, j & 1, kDevErrMmaTimeout) || bad;
    tc_fence_after();
#pragma unroll
    for (int c = 0; c < D; c += 16) {
      uint32_t rr[16];
      tmem_ld16(t_row + kKeys + c, rr);
      tmem_ld_wait();
#pragma unroll
      for (int e = 0; e < 16; ++e) acc[c + e] = acc[c + e] * alpha + __uint_as_float(rr[e]);
    }
  }

  cp_async_wait_all();  // no copy may land after the CTA exits
  const bool any_bad = __syncthreads_or(bad);
  if (any_bad && t == 0) {  // no MMA may write TMEM after it is released
    tc_commit(bar_drain);
    mbar_wait(bar_drain, 0, kDevErrMmaTimeout);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, S::kTmemCols);
  }
  if (row_ok && !any_bad) {
    const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
    uint4* o = reinterpret_cast<uint4*>(
        out + ((static_cast<size_t>(b) * q_heads + h) * queries + m0 + i) * D);
#pragma unroll
    for (int c = 0; c < D; c += 8)
      o[c / 8] = make_uint4(pack_half2(acc[c] * inv, acc[c + 1] * inv),
                            pack_half2(acc[c + 2] * inv, acc[c + 3] * inv),
                            pack_half2(acc[c + 4] * inv, acc[c + 5] * inv),
                            pack_half2(acc[c + 6] * inv, acc[c + 7] * inv));
  }
}

template <int D>
int launch_pa(const __half* q, const __half* k, const __half* v, const int32_t* q_start,
              __half* out, int batch, int q_heads, int kv_heads, int queries, int keys,
              int max_seq, int bm, int hp, int q_blocks, float scale_log2, int causal,
              cudaStream_t stream) {
  using S = PaShape<D>;
  auto kern = prefill_attention_kernel<D>;
  NPU_TRY_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmem));
  LaunchCfg cfg;
  cfg.grid = dim3(batch * kv_heads, q_blocks * (q_heads / kv_heads / hp));
  cfg.block = dim3(kThreads);
  cfg.smem = S::kSmem;
  cfg.stream = stream;
  return launch(cfg, kern, q, k, v, q_start, out, q_heads, kv_heads, queries, keys, max_seq, bm,
                hp, q_blocks, scale_log2, causal);
}

// ---------------------------------------------------------------------------
// Head size 128 (scale > 0): two query tiles per CTA on a warp-specialised
// pipeline.
//
//   warps 0-3  softmax of query tile 0 (thread r: row r, TMEM lane r)
//   warps 4-7  softmax of query tile 1
//   warp  8    TMA producer: both Q tiles once, then 64-key K and V tiles into
//              3-stage rings (3-D tensor maps whose row extent is `keys`, so
//              keys past it load as zero)
//   warp  9    MMA issuer (one thread) and TMEM owner
// Tensor-pipe order per key tile j: ... PV0(j-1) S0(j) PV1(j-1) S1(j) PV0(j)
// S0(j+1) PV1(j) S1(j+1) ..., so while one warpgroup turns its scores into P,
// the tensor pipe computes the other tile's P V and next scores.  Q, S, P and
// O live in TMEM (S0 cols [0,64), S1 [64,128), O0 [128,256), O1 [256,384),
// Q0 [384,448), Q1 [448,512); P_t over the first 32 columns of S_t, which the
// in-order tensor pipe reads for P V before the next S MMA overwrites them):
// the softmax threads copy their Q rows from the TMA tile into TMEM once and
// write P as FP16 pairs with tcgen05.st, and both MMAs take their A operand
// straight from TMEM, so the tensor pipe reads only K and V from shared
// memory.  O accumulates across tiles;
// a row's running max only moves -- and its O row is rescaled in TMEM -- when
// a tile's max exceeds it by more than 2^8, so P = exp2(s - max) <= 256 in
// FP16 and rescales are rare.  V enters the P V MMA as an MN-major operand
// straight from its TMA tile (keys x 128-byte rows of head dims): no transpose.
// ---------------------------------------------------------------------------
namespace pp {
constexpr int kTileKeys = 64;                      // keys per tile
constexpr int kStages = 3;                     // K and V ring depth
constexpr int kQBytes = 128 * 128 * 2;         // query tile: 128 rows x 128 dims
constexpr int kKVBytes = kTileKeys * 128 * 2;      // K or V tile: 64 keys x 128 dims
constexpr int kQ = 0;                          // Q0, Q1 (K-major, 2 atoms each)
constexpr int kK = kQ + 2 * kQBytes;           // K stages (K-major, 2 atoms each)
constexpr int kV = kK + kStages * kKVBytes;    // V stages (MN-major, 2 boxes each)
constexpr int kBars = kV + kStages * kKVBytes;
constexpr int kNumBars = 2 + 4 * kStages + 8 + 1;
constexpr int kSmem = kBars + kNumBars * 8 + 16 + 1024;
constexpr int kThreads = 320;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleLog2 = 8.f;
}  // namespace pp

__global__ void __launch_bounds__(pp::kThreads, 1)
    prefill_attention_pp_kernel(const __grid_constant__ CUtensorMap qmap,
                                const __grid_constant__ CUtensorMap kmap,
                                const __grid_constant__ CUtensorMap vmap,
                                const int32_t* __restrict__ q_start, __half* __restrict__ out,
                                int q_heads, int kv_heads, int queries, int keys, int bm, int hp,
                                int q_blocks, float scale_log2, int causal) {
  using namespace pp;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_1024(smem_raw);
  const uint32_t s_base = smem_u32(smem);
  const uint32_t sQ = s_base + kQ, sK = s_base + kK, sV = s_base + kV;
  uint64_t* q_full = reinterpret_cast<uint64_t*>(smem + kBars);
  uint64_t* k_full = q_full + 1;
  uint64_t* k_empty = k_full + kStages;
  uint64_t* v_full = k_empty + kStages;
  uint64_t* v_empty = v_full + kStages;
  uint64_t* s_full = v_empty + kStages;  // [2]
  uint64_t* p_full = s_full + 2;         // [2]
  uint64_t* o_done = p_full + 2;         // [2]
  uint64_t* turn = o_done + 2;           // [2] softmax turn of warpgroup t
  uint64_t* q_tmem = turn + 2;           // both Q tiles copied into TMEM
  uint64_t* drain = q_tmem + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int group = q_heads / kv_heads, subgroups = group / hp;
  const int n_units = q_blocks * subgroups;
  const int hk = static_cast<int>(blockIdx.x) % kv_heads;
  const int b = static_cast<int>(blockIdx.x) / kv_heads;
  const long long qs = q_start != nullptr ? q_start[b] : 0;
  // Units (query block, head subgroup), last query blocks first; this CTA
  // takes units u0 (tile 0) and u0 + 1 (tile 1, if it exists).
  const int u0 = 2 * static_cast<int>(blockIdx.y);  // slow grid dimension: heaviest first
  const bool has1 = u0 + 1 < n_units;
  auto unit_m0 = [&](int u) { return (q_blocks - 1 - u / subgroups) * bm; };
  long long cta_last = keys - 1;  // unit u0 has the later queries
  if (causal) cta_last = min(cta_last, qs + min(unit_m0(u0) + bm, queries) - 1);
  const int n_tiles = cta_last >= 0 ? static_cast<int>(cta_last / kTileKeys) + 1 : 0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 128);
      mbar_init(&o_done[t], 1);
      mbar_init(&turn[t], 128);
    }
    mbar_init(q_tmem, 256);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    // ---------------- TMA producer ----------------
    if (lane == 0 && n_tiles > 0) {
      prefetch_tensormap(&qmap);
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
      const int tiles_q = has1 ? 2 : 1;
      mbar_arrive_expect_tx(q_full, static_cast<uint32_t>(tiles_q * hp * 2 * bm * 128));
      for (int t = 0; t < tiles_q; ++t) {
        const int u = u0 + t, m0 = unit_m0(u), gs = u % subgroups;
        for (int g = 0; g < hp; ++g) {
          const int plane = b * q_heads + hk * group + gs * hp + g;
          for (int a = 0; a < 2; ++a)
            tma_load_3d(sQ + t * kQBytes + a * (kQBytes / 2) + g * bm * 128, &qmap, q_full, a * 64,
                        m0, plane);
        }
      }
      const int plane = b * kv_heads + hk;
      bool ok = true;
      int issued_k = 0, issued_v = 0;
      for (int j = 0; j < n_tiles && ok; ++j) {
        const int s = j % kStages;
        const uint32_t wait_phase = static_cast<uint32_t>((j / kStages) - 1) & 1u;
        if (j >= kStages && !wait_or_abort(&k_empty[s], wait_phase, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&k_full[s], kKVBytes);
        for (int a = 0; a < 2; ++a)
          tma_load_3d(sK + s * kKVBytes + a * (kKVBytes / 2), &kmap, &k_full[s], a * 64, j * kTileKeys,
                      plane);
        issued_k = j + 1;
        if (j >= kStages && !wait_or_abort(&v_empty[s], wait_phase, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&v_full[s], kKVBytes);
        for (int a = 0; a < 2; ++a)
          tma_load_3d(sV + s * kKVBytes + a * (kKVBytes / 2), &vmap, &v_full[s], a * 64, j * kTileKeys,
                      plane);
        issued_v = j + 1;
      }
      if (!ok) {  // leave no copy in flight into this CTA's shared memory
        *abort_flag = 1;
        mbar_wait(q_full, 0, kDevErrTmaTimeout);
        for (int j = max(0, issued_k - kStages); j < issued_k; ++j)
          mbar_wait(&k_full[j % kStages], (j / kStages) & 1, kDevErrTmaTimeout);
        for (int j = max(0, issued_v - kStages); j < issued_v; ++j)
          mbar_wait(&v_full[j % kStages], (j / kStages) & 1, kDevErrTmaTimeout);
      }
    }
  } else if (warp == 9) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && n_tiles > 0) {
      constexpr uint32_t idesc_s = idesc_f16_f32(128, kTileKeys);
      constexpr uint32_t idesc_pv = idesc_f16_f32(128, 128) | kIdescBMajorMN;
      // Descriptors of the tile bases; a byte offset moves the start-address
      // field by offset / 16 (no carry: shared addresses stay below 256 KB).
      const uint64_t dk = smem_desc_sw128(sK);
      const uint64_t dv = smem_desc_sw128_mn(sV, kKVBytes / 2, 1024);
      auto issue_s = [&](int t, int j) {
        const uint64_t k = dk + ((j % kStages) * kKVBytes >> 4);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          tc_mma_f16_tmem_a(tmem + t * kTileKeys, tmem + 384 + t * 64 + kk * 8,
                            k + (((kk >> 2) * (kKVBytes / 2) + (kk & 3) * 32) >> 4), idesc_s,
                            kk > 0 ? 1u : 0u);
        tc_commit(&s_full[t]);
      };
      auto issue_pv = [&](int t, int j) {
        const uint64_t v = dv + ((j % kStages) * kKVBytes >> 4);
#pragma unroll
        for (int kk = 0; kk < kTileKeys / 16; ++kk)
          tc_mma_f16_tmem_a(tmem + 128 + t * 128, tmem + t * kTileKeys + kk * 8,
                            v + (kk * 2048 >> 4), idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&o_done[t]);
      };
      bool ok = spin_or_abort(q_tmem, 0, abort_flag) && spin_or_abort(&k_full[0], 0, abort_flag);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        issue_s(1, 0);
        tc_commit(&k_empty[0]);
      }
      for (int j = 0; ok && j < n_tiles; ++j) {
        const int sj = j % kStages;
        for (int t = 0; t < 2; ++t) {
          ok = spin_or_abort(&p_full[t], j & 1, abort_flag) &&
               (t == 1 || spin_or_abort(&v_full[sj], (j / kStages) & 1, abort_flag));
          if (!ok) break;
          tc_fence_after();
          issue_pv(t, j);
          if (t == 1) tc_commit(&v_empty[sj]);
          if (j + 1 < n_tiles) {
            const int s1 = (j + 1) % kStages;
            if (t == 0) {
              ok = spin_or_abort(&k_full[s1], ((j + 1) / kStages) & 1, abort_flag);
              if (!ok) break;
              tc_fence_after();
            }
            issue_s(t, j + 1);
            if (t == 1) tc_commit(&k_empty[s1]);
          }
        }
      }
      if (!ok) {  // no MMA may write TMEM after it is released
        *abort_flag = 1;
        tc_commit(drain);
        mbar_wait(drain, 0, kDevErrMmaTimeout);
      }
    }
  } else {
    // ---------------- softmax warpgroups ----------------
    const int tt = warp >> 2, r = threadIdx.x & 127;
    const bool unit_ok = tt == 0 || has1;
    const int u = u0 + tt;
    const int m0 = unit_ok ? unit_m0(u) : 0, gs = u % subgroups;
    const int g = r / bm, i = r % bm;
    const bool row_ok = unit_ok && g < hp && m0 + i < queries;
    long long last = keys - 1;  // last key the row sees (< 0: none)
    if (causal) last = min(last, qs + m0 + i);
    if (!row_ok) last = -1;
    const uint32_t t_lane = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const uint32_t t_s = t_lane + tt * kTileKeys, t_o = t_lane + 128 + tt * 128;
    const uint32_t t_p = t_s;  // P_t over the first 32 columns of S_t
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    if (n_tiles > 0) {
      // This row of Q_t: from the swizzled TMA tile into TMEM columns
      // [384 + 64 t, 448 + 64 t), dims 2q and 2q + 1 in column q.
      ok = __all_sync(0xffffffffu, wait_or_abort(q_full, 0, abort_flag));
      if (ok) {
        const uint32_t q_row = sQ + tt * kQBytes + r * 128;
#pragma unroll
        for (int h = 0; h < 4; ++h) {  // dims 32h .. 32h + 31: chunks 4h .. 4h + 3
          uint32_t w[16];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const int ch = 4 * h + c;
            const uint32_t a = q_row + (ch >> 3) * (kQBytes / 2) + (((ch & 7) ^ (r & 7)) << 4);
            asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(w[4 * c]), "=r"(w[4 * c + 1]), "=r"(w[4 * c + 2]), "=r"(w[4 * c + 3])
                         : "r"(a));
          }
          tmem_st16(t_lane + 384 + tt * 64 + 16 * h, w);
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(q_tmem);
      }
    }
    for (int j = 0; ok && j < n_tiles; ++j) {
      ok = __all_sync(0xffffffffu, wait_or_abort(&s_full[tt], j & 1, abort_flag));
      if (!ok) break;
      // The two warpgroups take turns: warpgroup 0 runs tile j after warpgroup 1
      // finished tile j - 1, warpgroup 1 after warpgroup 0 finished tile j, so
      // each runs alone on the SM's issue slots and exp units while the tensor
      // pipe works on the other's tile.
      if (tt == 1 || j > 0) {
        ok = __all_sync(0xffffffffu, wait_or_abort(&turn[tt], (tt == 1 ? j : j - 1) & 1, abort_flag));
        if (!ok) break;
      }
      tc_fence_after();
      uint32_t sr[4][16];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld16(t_s + c * 16, sr[c]);
      tmem_ld_wait();
      const int key0 = j * kTileKeys;
      if (!__all_sync(0xffffffffu, key0 + kTileKeys - 1 <= last)) {  // mask keys past `last`
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int e = 0; e < 16; ++e)
            if (key0 + c * 16 + e > last) sr[c][e] = 0xff800000u;  // -inf
      }
      float part[8];
#pragma unroll
      for (int e = 0; e < 8; ++e)
        part[e] = fmaxf(fmaxf(__uint_as_float(sr[0][e]), __uint_as_float(sr[0][e + 8])),
                        fmaxf(__uint_as_float(sr[1][e]), __uint_as_float(sr[1][e + 8])));
#pragma unroll
      for (int e = 0; e < 8; ++e)
        part[e] = fmaxf(part[e], fmaxf(fmaxf(__uint_as_float(sr[2][e]), __uint_as_float(sr[2][e + 8])),
                                       fmaxf(__uint_as_float(sr[3][e]), __uint_as_float(sr[3][e + 8]))));
      const float mx = fmaxf(fmaxf(fmaxf(part[0], part[1]), fmaxf(part[2], part[3])),
                             fmaxf(fmaxf(part[4], part[5]), fmaxf(part[6], part[7])));
      const float m_tile = mx * scale_log2;  // scale_log2 > 0
      const bool grow = m_tile > m_run + kRescaleLog2;
      float alpha = 1.f;
      if (grow) {
        alpha = m_run == -INFINITY ? 0.f : fast_exp2(m_run - m_tile);
        l_run *= alpha;
        m_run = m_tile;
      }
      // P = exp2(s * scale * log2 e - max) as FP16 pairs (two exponentials per
      // exp-unit op), and this tile's row sum of exactly those FP16 weights.
      const float m_use = m_run == -INFINITY ? 0.f : m_run;  // no key seen: all s are -inf
      uint32_t pk[4][8];
      float psum[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int e = 0; e < 16; e += 2) {
          const uint32_t x = pack_half2(fmaf(__uint_as_float(sr[c][e]), scale_log2, -m_use),
                                        fmaf(__uint_as_float(sr[c][e + 1]), scale_log2, -m_use));
          const uint32_t h = ex2_f16x2(x);
          pk[c][e >> 1] = h;
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h));
          psum[(e >> 1) & 3] += f.x + f.y;
        }
      // P_t and O_t are free once this warpgroup's previous P V has completed.
      if (j > 0) {
        ok = __all_sync(0xffffffffu, wait_or_abort(&o_done[tt], (j - 1) & 1, abort_flag));
        if (!ok) break;
        tc_fence_after();
        if (__any_sync(0xffffffffu, grow)) {  // rescale this warp's O rows in TMEM
#pragma unroll 1
          for (int c = 0; c < 128; c += 16) {
            uint32_t o[16];
            tmem_ld16(t_o + c, o);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 16; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tmem_st16(t_o + c, o);
          }
          tmem_st_wait();
        }
      }
      // Keys 2q, 2q + 1 of the tile go to column q of this row of P_t.
      const uint32_t lo[16] = {pk[0][0], pk[0][1], pk[0][2], pk[0][3], pk[0][4], pk[0][5],
                               pk[0][6], pk[0][7], pk[1][0], pk[1][1], pk[1][2], pk[1][3],
                               pk[1][4], pk[1][5], pk[1][6], pk[1][7]};
      const uint32_t hi[16] = {pk[2][0], pk[2][1], pk[2][2], pk[2][3], pk[2][4], pk[2][5],
                               pk[2][6], pk[2][7], pk[3][0], pk[3][1], pk[3][2], pk[3][3],
                               pk[3][4], pk[3][5], pk[3][6], pk[3][7]};
      tmem_st16(t_p, lo);
      tmem_st16(t_p + 16, hi);
      tmem_st_wait();
      l_run += (psum[0] + psum[1]) + (psum[2] + psum[3]);
      tc_fence_before();
      mbar_arrive(&p_full[tt]);
      mbar_arrive(&turn[1 - tt]);
    }
    if (ok && n_tiles > 0)
      ok = __all_sync(0xffffffffu, wait_or_abort(&o_done[tt], (n_tiles - 1) & 1, abort_flag));
    if (!ok) {
      if (lane == 0) *abort_flag = 1;
    } else {
      tc_fence_after();
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      uint4* orow = reinterpret_cast<uint4*>(
          out + ((static_cast<size_t>(b) * q_heads + hk * group + gs * hp + g) * queries + m0 + i) *
                    128);
#pragma unroll 1
      for (int c = 0; c < 128; c += 16) {
        uint32_t o[16];
        if (n_tiles > 0) {
          tmem_ld16(t_o + c, o);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) o[e] = 0u;
        }
        if (row_ok) {
          float f[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) f[e] = __uint_as_float(o[e]) * inv;
          orow[c / 8] = make_uint4(pack_half2(f[0], f[1]), pack_half2(f[2], f[3]),
                                   pack_half2(f[4], f[5]), pack_half2(f[6], f[7]));
          orow[c / 8 + 1] = make_uint4(pack_half2(f[8], f[9]), pack_half2(f[10], f[11]),
                                       pack_half2(f[12], f[13]), pack_half2(f[14], f[15]));
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

int launch_pp(const void* q, const void* k, const void* v, const int32_t* q_start, __half* out,
              int batch, int q_heads, int kv_heads, int queries, int keys, int max_seq, int bm,
              int hp, int q_blocks, float scale_log2, int causal, cudaStream_t stream) {
  CUtensorMap qm, km, vm;
  int rc = make_tensor_map_3d(&qm, q, 128, queries, static_cast<uint64_t>(batch) * q_heads,
                              static_cast<uint64_t>(queries) * 256, bm, 64);
  if (rc) return rc;
  const uint64_t rows = keys > 0 ? keys : 1;
  rc = make_tensor_map_3d(&km, k, 128, rows, static_cast<uint64_t>(batch) * kv_heads,
                          static_cast<uint64_t>(max_seq) * 256, pp::kTileKeys, 64);
  if (rc) return rc;
  rc = make_tensor_map_3d(&vm, v, 128, rows, static_cast<uint64_t>(batch) * kv_heads,
                          static_cast<uint64_t>(max_seq) * 256, pp::kTileKeys, 64);
  if (rc) return rc;
  auto kern = prefill_attention_pp_kernel;
  NPU_TRY_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, pp::kSmem));
  const int n_units = q_blocks * (q_heads / kv_heads / hp);
  LaunchCfg cfg;
  cfg.grid = dim3(batch * kv_heads, (n_units + 1) / 2);
  cfg.block = dim3(pp::kThreads);
  cfg.smem = pp::kSmem;
  cfg.stream = stream;
  return launch(cfg, kern, qm, km, vm, q_start, out, q_heads, kv_heads, queries, keys, bm, hp,
                q_blocks, scale_log2, causal);
}

}  // namespace

// Rows of one head per CTA (a power of two, 16..128, covering `queries` when it
// is below 128) and heads of one GQA group stacked into the CTA's 128 rows.
void prefill_blocking(int queries, int group, int* bm, int* hp) {
  int m = kRows;
  while (m > 16 && m / 2 >= queries) m /= 2;
  int h = std::min(group, kRows / m);
  while (group % h != 0) --h;
  *bm = m;
  *hp = h;
}

int prefill_attention_run(const void* q, const void* k, const void* v, const int32_t* q_start,
                          void* out, int batch, int q_heads, int kv_heads, int head_dim,
                          int queries, int keys, int max_seq, float scale, int causal,
                          cudaStream_t stream) {
  NPU_REQUIRE(q && k && v && out, "prefill_attention: null tensor pointer");
  NPU_REQUIRE(batch >= 1 && kv_heads >= 1 && static_cast<long long>(batch) * kv_heads <= 65535,
              "prefill_attention: batch %d x kv_heads %d not in [1, 65535]", batch, kv_heads);
  NPU_REQUIRE(q_heads >= kv_heads && q_heads % kv_heads == 0,
              "prefill_attention: q_heads %d is not a multiple of kv_heads %d", q_heads, kv_heads);
  NPU_REQUIRE(head_dim == 32 || head_dim == 64 || head_dim == 128,
              "prefill_attention: head_dim %d not in {32,64,128}", head_dim);
  NPU_REQUIRE(queries >= 1, "prefill_attention: queries %d", queries);
  NPU_REQUIRE(max_seq >= 1 && keys >= 0 && keys <= max_seq,
              "prefill_attention: keys %d not in [0, max_seq %d]", keys, max_seq);
  NPU_REQUIRE(std::isfinite(scale), "prefill_attention: scale is not finite");
  const uintptr_t align = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                          reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(out);
  NPU_REQUIRE((align & 15) == 0, "prefill_attention: q, k, v and out must be 16-byte aligned");
  int bm = 0, hp = 0;
  prefill_blocking(queries, q_heads / kv_heads, &bm, &hp);
  const int q_blocks = (queries + bm - 1) / bm;
  NPU_REQUIRE(static_cast<long long>(q_blocks) * (q_heads / kv_heads / hp) <= 65535,
              "prefill_attention: %d queries make too many query blocks", queries);
  const float scale_log2 = scale * 1.4426950408889634f;
  const __half* qh = static_cast<const __half*>(q);
  const __half* kh = static_cast<const __half*>(k);
  const __half* vh = static_cast<const __half*>(v);
  __half* oh = static_cast<__half*>(out);
  if (head_dim == 128 && scale > 0.f)
    return launch_pp(q, k, v, q_start, oh, batch, q_heads, kv_heads, queries, keys, max_seq, bm,
                     hp, q_blocks, scale_log2, causal ? 1 : 0, stream);
  switch (head_dim) {
    case 32:
      return launch_pa<32>(qh, kh, vh, q_start, oh, batch, q_heads, kv_heads, queries, keys,
                           max_seq, bm, hp, q_blocks, scale_log2, causal ? 1 : 0, stream);
    case 64:
      return launch_pa<64>(qh, kh, vh, q_start, oh, batch, q_heads, kv_heads, queries, keys,
                           max_seq, bm, hp, q_blocks, scale_log2, causal ? 1 : 0, stream);
    default:
      return launch_pa<128>(qh, kh, vh, q_start, oh, batch, q_heads, kv_heads, queries, keys,
                            max_seq, bm, hp, q_blocks, scale_log2, causal ? 1 : 0, stream);
  }
}

}  // namespace npu_b200

extern "C" int npu_b200_prefill_attention(const void* d_q, const void* d_k, const void* d_v,
                                          const int32_t* d_q_start, void* d_out, int batch,
                                          int q_heads, int kv_heads, int head_dim, int queries,
                                          int keys, int max_seq, float scale, int causal,
                                          void* stream) {
  npu_b200::clear_error();
  return npu_b200::prefill_attention_run(d_q, d_k, d_v, d_q_start, d_out, batch, q_heads,
                                         kv_heads, head_dim, queries, keys, max_seq, scale, causal,
                                         static_cast<cudaStream_t>(stream));
}
