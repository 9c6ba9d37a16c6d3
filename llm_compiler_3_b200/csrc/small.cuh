// Interfaces of the small kernels in small.cu.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "peer.cuh"

namespace npu_b200 {

enum ResidualSource : int {
  kResidFromEmbedding = 0,  // h = embed[tokens[b]]
  kResidFromHidden = 1,     // h = hidden_in[b] (FP16)
  kResidAddPartial = 2,     // h = resid[b] + partial[b] (after the all-reduce), or
                            // resid[b] + every rank's published partial in rank order (px)
};

struct ResidualUpdate {
  int mode = kResidFromEmbedding;
  int batch = 0;
  int hidden = 0;
  int vocab = 0;
  const int32_t* tokens = nullptr;
  const __half* embed = nullptr;      // [vocab, hidden]
  const __half* hidden_in = nullptr;  // [batch, hidden]
  const float* partial = nullptr;     // [batch, hidden]
  float* resid = nullptr;             // [batch, hidden]
  const __half* norm_w = nullptr;     // [hidden] weight of the RMSNorm that follows
  __half* xw = nullptr;               // [batch, hidden] fp16(h * norm_w)
  float* ssq_out = nullptr;           // [hidden / ssq_rows][ssq_ld]
  int ssq_ld = 0;
  int ssq_rows = 128;                 // rows per sum of squares: 128 or 16
  const int32_t* positions = nullptr; // optional: seq_lens[b] = positions[b] + 1
  int32_t* seq_lens = nullptr;
  const float* inv_freq = nullptr;    // optional with rope_tab: [64] RoPE inverse frequencies
  float* rope_tab = nullptr;          // [batch][64] (cos, sin) of positions[b] * inv_freq[i]
  uint32_t* epoch = nullptr;          // optional: step counter to advance (first kernel of a step)
  PeerExchange px;                    // kResidAddPartial with px.seq >= 0: the ranks' partials
  int two_shot = 0;                   // with px: reduce-scatter + all-gather (peer.cuh)
};

int residual_update(const ResidualUpdate& p, cudaStream_t stream, bool pdl);
int argmax_reduce(const float* part_val, const int32_t* part_idx, int n_tiles, int ld, int batch,
                  int id_offset, float* out_val, int32_t* out_idx, cudaStream_t stream, bool pdl);
int argmax_combine(const float* gathered, int ranks, int ld, int batch, int32_t* out_ids,
                   cudaStream_t stream, bool pdl);
// Tensor parallel over peer memory: each rank stores its (max, id) per token
// as tagged words in its exchange buffer (px; seq is ignored); the combine
// reads every rank's pair over NVLink once it has landed and keeps the largest
// value, lowest id on ties.
int argmax_reduce_publish(const float* part_val, const int32_t* part_idx, int n_tiles, int ld,
                       int batch, int id_offset, const PeerExchange& px, cudaStream_t stream,
                       bool pdl);
int argmax_combine_peers(const PeerExchange& px, int batch, int32_t* out_ids, cudaStream_t stream,
                         bool pdl);
int store_hidden(const float* resid, __half* out, size_t count, cudaStream_t stream, bool pdl);

}  // namespace npu_b200
