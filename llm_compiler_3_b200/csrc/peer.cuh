// Tensor-parallel exchange over NVLink peer memory (one process per GPU).
//
// Replaces the NCCL all-reduce after o_proj / down_proj (and the all-gather of
// the per-rank LM-head argmaxes) for the decode step.  The producing kernel's
// epilogue stores each FP32 partial into its OWN HBM as one 8-byte word
// {tag, value}; the consumer reads every rank's word over NVLink (peer
// pointers opened through CUDA IPC), re-reading until the tag is this
// exchange's (bounded), and adds the values in rank order, so every rank
// computes the same bits.  An aligned 8-byte store is seen whole or not at all,
// so no fence or flag is needed: a system-scope release after a projection
// costs tens of microseconds, the tagged words nothing.
//
// Buffer of each rank (zeroed once), uint64 words:
//   [2][max_batch][hidden] partials, double-buffered by the parity of the
//   exchange index (a rank can be at most one exchange ahead of a peer still
//   reading), then [max_batch][2] (value, index) of the rank's LM-head argmax,
//   then [2][max_batch][hidden] reduced sums of the rows this rank owns in a
//   two-shot exchange (same parity rule).
//
// One-shot (batch 1-2, and whenever the volume is small): every rank reads
// every rank's partials.  Two-shot (large batches over 3+ ranks): rank r owns
// rows [r H/R, (r+1) H/R); it reads every rank's partials of those rows only,
// adds them in rank order and publishes the sums; the other ranks read them
// from it.  Each rank then takes 2 (R-1)/R of the data over NVLink instead of
// R-1 times it, and every row is still added in rank order by one rank.
// tag = 0x80000000 | (epoch * 256 + seq): epoch counts steps on every rank
// alike, seq numbers the exchanges of a step, so a tag never repeats within
// 2^23 steps and is never 0 (the zeroed buffer).
#pragma once

#include <stdint.h>

#include "common.cuh"

namespace npu_b200 {

constexpr int kMaxRanks = 8;
constexpr int kArgmaxSeq = 255;  // sequence number of the argmax gather

struct PeerExchange {
  uint64_t* part[kMaxRanks] = {};   // every rank's exchange buffer
  const uint32_t* epoch = nullptr;  // this rank's step counter
  int rank = 0, ranks = 0, max_batch = 0, hidden = 0;
  int seq = -1;  // exchange index within the step (< 255); < 0: no exchange
};

__device__ __forceinline__ uint32_t px_tag(const PeerExchange& x, int seq) {
  return 0x80000000u | ((__ldcg(x.epoch) * 256u + static_cast<uint32_t>(seq)) & 0x7fffffffu);
}

__device__ __forceinline__ void st_relaxed_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void px_put(uint64_t* p, uint32_t tag, uint32_t bits) {
  st_relaxed_sys(p, (static_cast<uint64_t>(tag) << 32) | bits);
}

// Bounded wait for the word at p to carry `tag`; its low 32 bits to *bits.
__device__ __forceinline__ bool px_get(const uint64_t* p, uint32_t tag, uint32_t* bits) {
  for (uint32_t i = 0; i < kMaxPolls; ++i) {
    const uint64_t w = ld_relaxed_sys(p);
    if (static_cast<uint32_t>(w >> 32) == tag) {
      *bits = static_cast<uint32_t>(w);
      return true;
    }
    if (i >= 64) __nanosleep(64);
  }
  report_error(kDevErrPeerTimeout);
  return false;
}

// The word at offset `off` of every rank's buffer, once each carries `tag`:
// every round issues the loads of all ranks still missing at once and checks
// them together, so waiting for the slowest rank costs one NVLink round trip
// per round rather than one per rank.  v[r] gets rank r's low 32 bits (0 where
// a rank never arrived within the bound, which is reported).
__device__ __forceinline__ bool px_gather(uint64_t* const* part, int ranks, size_t off, uint32_t tag,
                                          uint32_t (&v)[kMaxRanks]) {
  uint32_t missing = (1u << ranks) - 1u;
#pragma unroll
  for (int r = 0; r < kMaxRanks; ++r) v[r] = 0;
  for (uint32_t i = 0; i < kMaxPolls && missing != 0; ++i) {
    uint64_t w[kMaxRanks];
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r) w[r] = (missing >> r) & 1u ? ld_relaxed_sys(part[r] + off) : 0;
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r) {
      if (((missing >> r) & 1u) && static_cast<uint32_t>(w[r] >> 32) == tag) {
        v[r] = static_cast<uint32_t>(w[r]);
        missing &= ~(1u << r);
      }
    }
    if (missing != 0 && i >= 64) __nanosleep(32);
  }
  if (missing != 0) report_error(kDevErrPeerTimeout);
  return missing == 0;
}

// Offset of (b, n) in a rank's partial buffer for exchange x.seq.
__device__ __forceinline__ size_t px_offset(const PeerExchange& x, int b, int n) {
  return (static_cast<size_t>(x.seq & 1) * x.max_batch + b) * x.hidden + n;
}

// This rank's partial for (b, n), into its own buffer.
__device__ __forceinline__ void px_store(const PeerExchange& x, uint32_t tag, int b, int n, float v) {
  px_put(x.part[x.rank] + px_offset(x, b, n), tag, __float_as_uint(v));
}

// Rank src's partial for (b, n), once it has landed.
__device__ __forceinline__ bool px_load(const PeerExchange& x, uint32_t tag, int src, int b, int n,
                                        float* v) {
  uint32_t bits = 0;
  const bool ok = px_get(x.part[src] + px_offset(x, b, n), tag, &bits);
  *v = ok ? __uint_as_float(bits) : 0.f;
  return ok;
}

// Offset of (b, n)'s reduced sum (two-shot) in its owner's buffer.
__device__ __forceinline__ size_t px_reduced_offset(const PeerExchange& x, int b, int n) {
  return static_cast<size_t>(2) * x.max_batch * x.hidden + static_cast<size_t>(2) * x.max_batch +
         (static_cast<size_t>(x.seq & 1) * x.max_batch + b) * x.hidden + n;
}

// Argmax words of a rank's buffer: (value, index) of token b.
__device__ __forceinline__ size_t px_argmax_offset(const PeerExchange& x, int b) {
  return static_cast<size_t>(2) * x.max_batch * x.hidden + static_cast<size_t>(b) * 2;
}

}  // namespace npu_b200
