// Projection (linear layer) kernel interface: D[n, b] = sum_k W[n, k] X[b, k]
// on tcgen05 tensor cores, followed by one fused epilogue.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "peer.cuh"

namespace npu_b200 {

// What the epilogue does with the FP32 tile (128 weight rows x up to BN tokens).
enum EpiKind : int {
  kEpiStore = 0,   // out[b, n] = acc (+ bias[n]) (ReLU), FP16 or FP32
  kEpiResid = 1,   // h = resid + acc; resid = h; xw = fp16(h * norm_w); ssq partial of h
  kEpiSwiGLU = 2,  // rows (gate_j, up_j) interleaved: act[b, j] = silu(gate_j) * up_j
  kEpiQKV = 3,     // per-head tiles (dims in rotate_half pair order): [QK-norm], RoPE,
                   // write q / append k,v to the cache
  kEpiArgmax = 4,  // per-tile (max, argmax) over rows for every token
};

struct EpiParams {
  int kind = kEpiStore;
  int n_rows = 0;  // valid rows of W (N)
  int batch = 0;   // valid tokens (columns)

  // Optional RMSNorm scale of the input tokens: rn[b] = rsqrt(sum_p ssq_in[p][b] / hidden + eps),
  // sum over `ssq_parts` partial sums written by the producer of X.
  const float* ssq_in = nullptr;
  int ssq_parts = 0;
  int ssq_ld = 0;
  float ssq_inv_hidden = 0.f;
  float ssq_eps = 0.f;

  // kEpiStore
  void* out = nullptr;
  int ld_out = 0;
  int out_f32 = 0;
  int relu = 0;
  const __half* bias = nullptr;

  // kEpiResid
  float* resid = nullptr;
  int ld_resid = 0;
  const __half* norm_w = nullptr;
  __half* xw = nullptr;
  int ld_xw = 0;
  float* ssq_out = nullptr;  // [n / ssq_out_rows][ssq_out_ld]
  int ssq_out_ld = 0;
  int ssq_out_rows = 128;    // rows per partial sum: 128 or 16

  // kEpiQKV (head_dim 128: one tile is one head)
  int q_heads = 0, kv_heads = 0;
  const int32_t* positions = nullptr;
  const float* inv_freq = nullptr;  // [64]
  const float* rope_tab = nullptr;  // optional [batch][64] (cos, sin) of positions x inv_freq
  __half* k_cache = nullptr;        // [batch_cap][kv_heads][max_seq][128]
  __half* v_cache = nullptr;
  int max_seq = 0;
  int cache_batch_stride = 0;       // elements between sequences of the cache = kv_heads*max_seq*128
  const __half* q_norm_w = nullptr;
  const __half* k_norm_w = nullptr;
  float qk_eps = 0.f;

  // kEpiArgmax: part_val/part_idx [tile][batch]
  float* am_val = nullptr;    // [ceil(n / am_rows)][am_ld]
  int32_t* am_idx = nullptr;
  int am_ld = 0;
  int am_rows = 128;          // rows per partial (max, argmax): 128 or 16

  // px.seq >= 0, kEpiStore: instead of `out`, store the FP32 value as a tagged
  // word in this rank's exchange buffer (peer.cuh); kEpiResid (GEMV path only):
  // all-reduce the partial over the ranks before the residual add.
  PeerExchange px;
};

// Runs the projection.  w is [n_rows, k] FP16 row-major, or (w_packed) the
// panel layout pack_weight() writes; x [batch, k] FP16 row-major.
// Workspace: proj_workspace_bytes(); zero-filled once, left zero-filled.
int proj_run(const void* w, bool w_packed, const void* x, int n_rows, int k, int batch,
             const EpiParams& ep, void* workspace, size_t workspace_bytes, cudaStream_t stream,
             bool pdl);
size_t proj_workspace_bytes(int n_rows, int k, int batch);

// Batch 1-2 GEMV over packed panels (gemv.cu): no workspace.  Supported when
// n_rows % 16 == 0, the activations fit in shared memory, no QK-norm, and a
// residual epilogue writes 16-row sums of squares.
bool gemv_supported(int n_rows, int k, int batch, const EpiParams& ep);
int gemv_run(const void* w_packed, const void* x, int n_rows, int k, int batch, const EpiParams& ep,
             cudaStream_t stream, bool pdl);


// Weight panels: 16 KB blocks [ceil(n/128)][k/64] of 128 rows x 64 columns,
// each already in the 128-byte-swizzled K-major layout the tensor cores read,
// so one contiguous bulk copy moves a block from HBM to shared memory.
size_t packed_weight_bytes(int n_rows, int k);
// Packs n_src_rows source rows (row pitch src_pitch elements) into a panel
// buffer of dst_rows rows.  row_mode 0: destination row = row_offset + i;
// row_mode 1: gate/up interleave, destination row = 2 i + row_offset (0 or 1);
// row_mode 2: whole 128-row heads with dims in rotate_half pair order,
// dim d -> row 2d (d < 64) or 2(d - 64) + 1, after row_offset.
int pack_weight(const void* src, size_t src_pitch, int n_src_rows, int k, void* dst, int dst_rows,
                int row_mode, int row_offset, cudaStream_t stream);

}  // namespace npu_b200
