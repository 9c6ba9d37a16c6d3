// Small memory-bound kernels around the projections of a decode step.
//
//  * residual_update: the residual stream entering a layer stack or leaving an
//    all-reduce.  h = source (embedding row, FP16 hidden state, or resid +
//    all-reduced partial); resid = h (FP32); xw = fp16(h * norm_w); and one
//    partial sum of squares of h per 128-row chunk and token, which the next
//    projection turns into the RMSNorm scale in its epilogue
//    (lib/Transforms/Pipeline.cpp:149-185: row reductions in FP32).
//  * argmax_reduce / argmax_combine: greedy token choice over the per-tile
//    (max, index) pairs the LM-head epilogue leaves, ties to the lowest id;
//    with tensor parallelism the per-rank results go through NCCL or, over
//    peer memory, argmax_reduce_publish / argmax_combine_peers.
//  * store_hidden: FP32 residual -> FP16 hidden-state output.
#include <math.h>

#include "common.cuh"
#include "host.hpp"
#include "small.cuh"

namespace npu_b200 {
namespace {

constexpr int kChunk = 128;

// One CTA per (128-row chunk, token): every element is an independent load, so
// the whole update is one memory round trip wide.
__global__ void __launch_bounds__(kChunk)
    residual_update_kernel(ResidualUpdate p) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float red[kChunk / 32];
  const int n = blockIdx.x * kChunk + threadIdx.x;
  const int b = blockIdx.y;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (blockIdx.x == 0 && b == 0 && p.positions && p.seq_lens)
    for (int i = threadIdx.x; i < p.batch; i += blockDim.x) p.seq_lens[i] = p.positions[i] + 1;
  if (blockIdx.x == 0 && b == 0 && threadIdx.x == 0 && p.epoch) *p.epoch += 1;
  // This step's RoPE angles, once for every layer: theta = float(pos) * inv_freq
  // in FP32 (as transformers forms them), then an accurate sincos.
  if (blockIdx.x == 0 && p.rope_tab && p.positions && threadIdx.x < 64) {
    float sn, cs;
    sincosf(static_cast<float>(p.positions[b]) * p.inv_freq[threadIdx.x], &sn, &cs);
    reinterpret_cast<float2*>(p.rope_tab)[b * 64 + threadIdx.x] = make_float2(cs, sn);
  }
  float h;
  if (p.mode == kResidFromEmbedding) {
    const int tok = p.tokens[b];
    if (tok < 0 || tok >= p.vocab) {
      if (threadIdx.x == 0) report_error(kDevErrBounds);
      h = 0.f;
    } else {
      h = __half2float(p.embed[static_cast<size_t>(tok) * p.hidden + n]);
    }
  } else if (p.mode == kResidFromHidden) {
    h = __half2float(p.hidden_in[static_cast<size_t>(b) * p.hidden + n]);
  } else if (p.px.seq < 0) {
    h = p.resid[static_cast<size_t>(b) * p.hidden + n] +
        p.partial[static_cast<size_t>(b) * p.hidden + n];
  } else {
    // Every rank's partial (tagged words gathered with all missing ranks'
    // loads in flight together), added in rank order: the same bits on every
    // rank.  Two-shot: only for the rows this rank owns, whose sums it then
    // publishes; other rows' sums come from their owners (a warp's 32 rows
    // have one owner).
    const uint32_t tag = px_tag(p.px, p.px.seq);
    const int owner = p.two_shot ? n / (p.hidden / p.px.ranks) : p.px.rank;
    float sum = 0.f;
    if (owner == p.px.rank) {
      uint32_t bits[kMaxRanks];
      px_gather(p.px.part, p.px.ranks, px_offset(p.px, b, n), tag, bits);
#pragma unroll
      for (int r = 0; r < kMaxRanks; ++r)
        if (r < p.px.ranks) sum += __uint_as_float(bits[r]);
      if (p.two_shot)
        px_put(p.px.part[p.px.rank] + px_reduced_offset(p.px, b, n), tag, __float_as_uint(sum));
    } else {
      // The owner's warp publishes these 32 rows with one store instruction:
      // one lane waits for the last word (one 8-byte poll per warp, not 32
      // polls of NVLink while the owner is still adding), then all read.
      const uint64_t* src = p.px.part[owner] + px_reduced_offset(p.px, b, n);
      uint32_t bits = 0;
      if (lane == 31) px_get(src, tag, &bits);
      __syncwarp();
      px_get(src, tag, &bits);
      sum = __uint_as_float(bits);
    }
    h = p.resid[static_cast<size_t>(b) * p.hidden + n] + sum;
  }
  const float w = __half2float(p.norm_w[n]);
  p.resid[static_cast<size_t>(b) * p.hidden + n] = h;
  p.xw[static_cast<size_t>(b) * p.hidden + n] = __float2half_rn(h * w);
  float s = h * h;
  if (p.ssq_rows == 16) {  // one sum per half warp
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((lane & 15) == 0)
      p.ssq_out[static_cast<size_t>(blockIdx.x * 8 + warp * 2 + (lane >> 4)) * p.ssq_ld + b] = s;
    return;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) red[warp] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < kChunk / 32; ++i) t += red[i];
    p.ssq_out[static_cast<size_t>(blockIdx.x) * p.ssq_ld + b] = t;
  }
}

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

// Token blockIdx.x's (max, index) over n_tiles partials (part[t * ld + b]),
// lowest index on ties; thread 0's *bv_out / *bi_out hold the result.
__device__ __forceinline__ void block_argmax(const float* __restrict__ part_val,
                                             const int32_t* __restrict__ part_idx, int n_tiles,
                                             int ld, float* bv_out, int* bi_out) {
  const int b = blockIdx.x;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int t = threadIdx.x; t < n_tiles; t += blockDim.x) {
    const float v = part_val[static_cast<size_t>(t) * ld + b];
    const int i = part_idx[static_cast<size_t>(t) * ld + b];
    if (better(v, i, bv, bi)) {
      bv = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  __shared__ float sv[8];
  __shared__ int si[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = bv;
    si[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w)
      if (better(sv[w], si[w], bv, bi)) {
        bv = sv[w];
        bi = si[w];
      }
  }
  *bv_out = bv;
  *bi_out = bi;
}

__global__ void __launch_bounds__(256)
    argmax_reduce_kernel(const float* __restrict__ part_val, const int32_t* __restrict__ part_idx,
                         int n_tiles, int ld, int id_offset, float* __restrict__ out_val,
                         int32_t* __restrict__ out_idx) {
  pdl_launch_dependents();
  pdl_wait();
  float bv;
  int bi;
  block_argmax(part_val, part_idx, n_tiles, ld, &bv, &bi);
  if (threadIdx.x == 0) {
    out_val[blockIdx.x] = bv;
    out_idx[blockIdx.x] = bi + id_offset;
  }
}

// The same, published as tagged words in this rank's exchange buffer.
__global__ void __launch_bounds__(256)
    argmax_publish_kernel(const float* __restrict__ part_val, const int32_t* __restrict__ part_idx,
                          int n_tiles, int ld, int id_offset, const PeerExchange px) {
  pdl_launch_dependents();
  pdl_wait();
  float bv;
  int bi;
  block_argmax(part_val, part_idx, n_tiles, ld, &bv, &bi);
  if (threadIdx.x == 0) {
    const uint32_t tag = px_tag(px, kArgmaxSeq);
    uint64_t* w = px.part[px.rank] + px_argmax_offset(px, blockIdx.x);
    px_put(w, tag, __float_as_uint(bv));
    px_put(w + 1, tag, static_cast<uint32_t>(bi + id_offset));
  }
}

__global__ void argmax_combine_peers_kernel(const PeerExchange px, int batch,
                                            int32_t* __restrict__ out_ids) {
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < batch) {
    const uint32_t tag = px_tag(px, kArgmaxSeq);
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    uint32_t vb[kMaxRanks], ib[kMaxRanks];
    const size_t off = px_argmax_offset(px, b);
    const bool ok = px_gather(px.part, px.ranks, off, tag, vb) &&
                    px_gather(px.part, px.ranks, off + 1, tag, ib);
    for (int r = 0; r < px.ranks && ok; ++r) {
      const float v = __uint_as_float(vb[r]);
      const int i = static_cast<int>(ib[r]);
      if (better(v, i, bv, bi)) {
        bv = v;
        bi = i;
      }
    }
    out_ids[b] = ok ? bi : -1;
  }
}

// gathered: [ranks][2][ld] as {values; ids} per rank.
__global__ void argmax_combine_kernel(const float* __restrict__ gathered, int ranks, int ld,
                                      int batch, int32_t* __restrict__ out_ids) {
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < batch) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int r = 0; r < ranks; ++r) {
      const float v = gathered[static_cast<size_t>(r) * 2 * ld + b];
      const int i = __float_as_int(gathered[static_cast<size_t>(r) * 2 * ld + ld + b]);
      if (better(v, i, bv, bi)) {
        bv = v;
        bi = i;
      }
    }
    out_ids[b] = bi;
  }
}

__global__ void store_hidden_kernel(const float* __restrict__ resid, __half* __restrict__ out,
                                    size_t count) {
  pdl_launch_dependents();
  pdl_wait();
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < count;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    out[i] = __float2half_rn(resid[i]);
}

}  // namespace

int residual_update(const ResidualUpdate& p, cudaStream_t stream, bool pdl) {
  NPU_REQUIRE(p.hidden % kChunk == 0 && p.batch >= 1 && p.batch <= 1024,
              "residual update: hidden %d must be a multiple of 128", p.hidden);
  // Two-shot: every rank's slice of rows a whole number of warps, and every
  // CTA of the grid resident at once (128-thread CTAs, 16 per SM), so the
  // CTAs that reduce this rank's rows get an SM while the others poll.
  NPU_REQUIRE(!p.two_shot || (p.px.seq >= 0 && p.px.ranks >= 2 &&
                              p.hidden % (p.px.ranks * 32) == 0 &&
                              static_cast<long long>(p.hidden / kChunk) * p.batch <= 16ll * sm_count()),
              "residual update: two-shot exchange needs hidden %% (32 x ranks) == 0 and a "
              "co-resident grid");
  LaunchCfg cfg;
  cfg.grid = dim3(p.hidden / kChunk, p.batch);
  cfg.block = dim3(kChunk);
  cfg.stream = stream;
  cfg.pdl = pdl;
  return launch(cfg, residual_update_kernel, p);
}

int argmax_reduce(const float* part_val, const int32_t* part_idx, int n_tiles, int ld, int batch,
                  int id_offset, float* out_val, int32_t* out_idx, cudaStream_t stream, bool pdl) {
  LaunchCfg cfg;
  cfg.grid = dim3(batch);
  cfg.block = dim3(256);
  cfg.stream = stream;
  cfg.pdl = pdl;
  return launch(cfg, argmax_reduce_kernel, part_val, part_idx, n_tiles, ld, id_offset, out_val,
                out_idx);
}

int argmax_reduce_publish(const float* part_val, const int32_t* part_idx, int n_tiles, int ld,
                       int batch, int id_offset, const PeerExchange& px, cudaStream_t stream,
                       bool pdl) {
  NPU_REQUIRE(px.ranks >= 1 && px.ranks <= kMaxRanks && batch <= px.max_batch,
              "argmax: bad peer exchange");
  LaunchCfg cfg;
  cfg.grid = dim3(batch);
  cfg.block = dim3(256);
  cfg.stream = stream;
  cfg.pdl = pdl;
  return launch(cfg, argmax_publish_kernel, part_val, part_idx, n_tiles, ld, id_offset, px);
}

int argmax_combine_peers(const PeerExchange& px, int batch, int32_t* out_ids, cudaStream_t stream,
                         bool pdl) {
  LaunchCfg cfg;
  cfg.grid = dim3((batch + 127) / 128);
  cfg.block = dim3(128);
  cfg.stream = stream;
  cfg.pdl = pdl;
  return launch(cfg, argmax_combine_peers_kernel, px, batch, out_ids);
}

int argmax_combine(const float* gathered, int ranks, int ld, int batch, int32_t* out_ids,
                   cudaStream_t stream, bool pdl) {
  LaunchCfg cfg;
  cfg.grid = dim3((batch + 127) / 128);
  cfg.block = dim3(128);
  cfg.stream = stream;
  cfg.pdl = pdl;
  return launch(cfg, argmax_combine_kernel, gathered, ranks, ld, batch, out_ids);
}

int store_hidden(const float* resid, __half* out, size_t count, cudaStream_t stream, bool pdl) {
  LaunchCfg cfg;
  cfg.grid = dim3(static_cast<unsigned>((count + 255) / 256 < 1184 ? (count + 255) / 256 : 1184));
  cfg.block = dim3(256);
  cfg.stream = stream;
  cfg.pdl = pdl;
  return launch(cfg, store_hidden_kernel, resid, out, count);
}

}  // namespace npu_b200
