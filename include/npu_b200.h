/*
 * npu_b200.h -- C ABI of libnpu_b200, the B200 (sm_100a) execution backend for
 * the FP16 Llama/Qwen3 decode computation that LLM_Compiler_3 lowers.
 *
 * Reference interface this replaces (all paths inside LLM_Compiler_3):
 *   - the NPU back-end stages behind the pass registry: createTilePass,
 *     createPlacePass, createHardwareOpsPass, createPipelineAttentionPass,
 *     createAssignAddressesPass, createEmitPass, createEncodePass
 *     (include/npu/Transforms/Passes.h:24-31) and their stage functions
 *     (include/npu/Transforms/Pipeline.h:13-28);
 *   - the package they produce (program.bin / system.json / hbm.bin,
 *     tools/npu-compile/npu-compile.cpp:462-659) and the simulator that runs it
 *     (test/Integration/harness.py:19-33).
 * Instead of a package for a simulator, the B200 path hands a plan and the
 * captured weights (arg<N>.bin, python/npu/capture/export.py:30-40) to this
 * library, which runs them with hand-written sm_100a kernels.
 *
 * Conventions
 *   - Every function returns int: NPU_B200_OK (0) or a negative NPU_B200_E_*.
 *     On failure npu_b200_last_error() returns a thread-local message.  Nothing
 *     throws across this boundary and no kernel traps.
 *   - `stream` is a cudaStream_t passed as void*; 0 is the legacy default stream.
 *     Kernel-level calls are stream-ordered and asynchronous.
 *   - Pointers named d_* are device pointers; h_* are host pointers.
 *   - A context is thread-compatible, not thread-safe.  Device buffers the
 *     context allocates are owned by it; buffers passed in are borrowed.
 *   - Tensors are dense, row-major, FP16 unless stated; shapes are in elements.
 */
#ifndef NPU_B200_H
#define NPU_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(NPU_B200_BUILD)
#define NPU_B200_API __attribute__((visibility("default")))
#else
#define NPU_B200_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define NPU_B200_ABI_VERSION 1

enum {
  NPU_B200_OK = 0,
  NPU_B200_E_INVALID = -1,     /* bad argument, shape or layout */
  NPU_B200_E_CUDA = -2,        /* a CUDA runtime/driver call failed */
  NPU_B200_E_NCCL = -3,        /* a NCCL call failed or NCCL could not be loaded */
  NPU_B200_E_UNSUPPORTED = -4, /* valid request this build does not implement */
  NPU_B200_E_NOMEM = -5,       /* device or host allocation failed */
  NPU_B200_E_PLAN = -6,        /* plan file missing, malformed, or stamp mismatch */
  NPU_B200_E_DEVICE = -7,      /* a kernel reported a device-side error (timeout, bounds) */
  NPU_B200_E_STATE = -8        /* call out of order (e.g. decode before load) */
};

/* ---------------------------------------------------------------------------
 * Library-wide
 * ------------------------------------------------------------------------- */

/* ABI version this library implements (NPU_B200_ABI_VERSION). */
NPU_B200_API int npu_b200_abi_version(void);

/* Message for the last failing call on this thread ("" if none). */
NPU_B200_API const char* npu_b200_last_error(void);

/* Reads and clears the device error word on the current device.  *h_bits gets
 * the OR of every device-side error since the last call (0 = none).
 * Synchronizes the device.  Returns NPU_B200_E_DEVICE if any bit was set. */
NPU_B200_API int npu_b200_device_status(uint32_t* h_bits);

/* ---------------------------------------------------------------------------
 * Kernel-level entry points (borrowed device buffers, stream-ordered)
 * ------------------------------------------------------------------------- */

/* Split-KV flash-decoding attention for one decode query per sequence.
 *
 * Replaces the NPU lowering of npu.attention (lib/Transforms/Attention.cpp:187-375,
 * include/npu/Dialect/NPUDialect.td:147-189): per query head h with KV head
 * h / group, out = softmax(scale * q K^T) V over keys [0, seq_lens[b]).
 * Online softmax and every accumulator in FP32; output rounded once to FP16.
 *
 *   d_q        [batch, q_heads, head_dim]
 *   d_k, d_v   [batch, kv_heads, max_seq, head_dim]   (KV cache, one layer)
 *   d_seq_lens [batch] int32, each in [0, max_seq]; 0 keys gives a zero row
 *   d_out      [batch, q_heads, head_dim]
 *   head_dim in {64, 128}; group = q_heads / kv_heads in 1..8.
 *   num_splits: key-range splits per (sequence, KV head); 0 chooses one.
 *   d_workspace: npu_b200_flash_decode_workspace_size() bytes, zero-filled once
 *     before first use; the kernel returns it to zero-filled state itself, so
 *     calls on one stream may reuse it.  Calls that overlap on the GPU need
 *     separate workspaces.
 * The kernel is launched as a programmatic dependent of the stream's previous
 * work: it reads no input and writes no output before that work has completed,
 * so stream order is kept; only its launch overlaps that work's tail. */
NPU_B200_API size_t npu_b200_flash_decode_workspace_size(int batch, int kv_heads, int head_dim, int max_seq,
                                            int num_splits);
NPU_B200_API int npu_b200_flash_decode(const void* d_q, const void* d_k, const void* d_v,
                          const int32_t* d_seq_lens, void* d_out, int batch, int q_heads,
                          int kv_heads, int head_dim, int max_seq, float scale, int num_splits,
                          void* d_workspace, size_t workspace_bytes, void* stream);

/* npu_b200_flash_decode without any device allocation (no counterpart in the
 * reference: its compiled programs run on a simulator that owns all memory).
 *
 * For callers that cannot allocate device memory when they call attention:
 * code running inside a host application that has already handed all HBM to its
 * own pool allocator, code on a latency-critical path where the device-wide
 * synchronization of cudaMalloc/cudaFree is unacceptable, or plugins whose host
 * forbids device allocation after start-up.  The split-merge scratch is instead
 * a fixed 4 MiB array in this library's device memory, present on every GPU that
 * loads the library until the process exits.  A shape whose scratch would exceed
 * 4 MiB (batch x kv_heads x splits x (8 x head_dim + 16) x 4 bytes plus 64 KiB of
 * counters) is rejected with NPU_B200_E_INVALID.
 *
 * Each call made outside stream capture looks up the array's device address
 * (with the calling thread's current device, which must be the device of the
 * tensors); calls made while `stream` is being captured reuse the address the
 * last uncaptured call on that device found, so make the first call on each
 * device before any stream capture (also after cudaDeviceReset, which reloads
 * the module).  Every call uses the same array and clears the split counters it
 * needs before its kernel runs; a call with one split per unit touches no
 * scratch.
 * Calls that overlap on the GPU (different streams, or concurrent graphs) race
 * on the array.  Arguments and results are those of npu_b200_flash_decode. */
NPU_B200_API int npu_b200_flash_decode_noalloc(const void* d_q, const void* d_k, const void* d_v,
                                               const int32_t* d_seq_lens, void* d_out, int batch,
                                               int q_heads, int kv_heads, int head_dim,
                                               int max_seq, float scale, int num_splits,
                                               void* stream);

/* Multi-query (prefill) attention on tcgen05 tensor cores.
 *
 * Replaces the NPU lowering of npu.attention with M >= 1 queries per head and
 * of its causal form (lib/Transforms/Attention.cpp:187-375; the is_causal mask as
 * recognised at 70-92, blocks past the diagonal skipped at 221-222): per query
 * head h with KV head h / group,
 *   out[b,h,i] = sum_j softmax_j(scale * q[b,h,i] . k[b,h/group,j]) v[b,h/group,j]
 * over keys j < keys and, when causal != 0, j <= q_start[b] + i (d_q_start NULL:
 * 0, torch's top-left is_causal mask).  FP32 scores, online softmax and
 * accumulation; the softmax weights are rounded to FP16 as the second MMA's
 * operand; the output is rounded once.  A row that sees no key is zero.
 *
 *   d_q, d_out [batch, q_heads, queries, head_dim]
 *   d_k, d_v   [batch, kv_heads, max_seq, head_dim]   (the KV-cache layout)
 *   d_q_start  [batch] int32 or NULL
 *   head_dim in {32, 64, 128}; keys in [0, max_seq]; batch x kv_heads <= 65535;
 *   every pointer 16-byte aligned.  No workspace; calls may overlap. */
NPU_B200_API int npu_b200_prefill_attention(const void* d_q, const void* d_k, const void* d_v,
                                            const int32_t* d_q_start, void* d_out, int batch,
                                            int q_heads, int kv_heads, int head_dim, int queries,
                                            int keys, int max_seq, float scale, int causal,
                                            void* stream);

/* Linear layer on tcgen05 tensor cores:
 *   out[b, n] = act( sum_k x[b, k] * w[n, k] + bias[n] ),  FP32 accumulation.
 *
 * Replaces the NPU matmul lowering (lib/Transforms/HardwareOps.cpp:105-155,
 * lib/Transforms/Emit.cpp:348-378) of a legalized linalg.matmul with FP16
 * operands and a zero accumulator (lib/Transforms/Legalize.cpp:136-161), plus the
 * per-channel bias and the ReLU that normalizeGraph turns into maximumf
 * (lib/Transforms/Normalize.cpp:494-507).
 *
 *   d_x    [batch, k] FP16, batch in 1..128 (the decode tokens)
 *   d_w    [n_rows, k] FP16 (torch Linear layout, the capture's arg<N>.bin), k % 64 == 0
 *   d_bias [n_rows] FP16 or NULL
 *   d_out  [batch, n_rows] FP16, or FP32 with NPU_B200_LINEAR_OUT_F32
 *   d_workspace: npu_b200_linear_workspace_size() bytes, 256-byte aligned,
 *     zero-filled before first use and left zero-filled by every call. */
#define NPU_B200_LINEAR_RELU 1
#define NPU_B200_LINEAR_OUT_F32 2
#define NPU_B200_LINEAR_PACKED_W 4 /* d_w is in the panel layout of npu_b200_pack_weight */
NPU_B200_API size_t npu_b200_linear_workspace_size(int n_rows, int k, int batch);
NPU_B200_API int npu_b200_linear(const void* d_x, const void* d_w, const void* d_bias, void* d_out,
                                 int batch, int n_rows, int k, int flags, void* d_workspace,
                                 size_t workspace_bytes, void* stream);

/* Weight panels: the B200 counterpart of the reference image builder's packed
 * panels (lib/Transforms/Tile.cpp:351-395 packWeightPanels; hbm.bin layout
 * [N/p][K][p], tools/npu-compile/npu-compile.cpp:637-648).  W [n_rows, k] becomes
 * 16 KB blocks [ceil(n_rows/128)][k/64], each 128 rows x 64 columns in the
 * 128-byte-swizzled K-major order the tensor cores read, so a projection streams
 * every block with one contiguous bulk copy.  Rows past n_rows are zero. */
NPU_B200_API size_t npu_b200_packed_weight_bytes(int n_rows, int k);
NPU_B200_API int npu_b200_pack_weight(const void* d_w, int n_rows, int k, void* d_packed,
                                      void* stream);

/* Pack n_src_rows rows of d_w into rows of an existing panel buffer of dst_rows
 * rows (zero-filled by the caller), so several tensors can share one buffer in
 * the row orders the fused epilogues read:
 *   IDENTITY    source row i -> row row_offset + i
 *   INTERLEAVE  source row i -> row 2i + row_offset (gate with offset 0, up with 1)
 *   HEAD_PAIRS  whole 128-row heads; head dim d -> row 2d (d < 64) or 2(d - 64) + 1,
 *               after row_offset (a multiple of 128). */
#define NPU_B200_PACK_IDENTITY 0
#define NPU_B200_PACK_INTERLEAVE 1
#define NPU_B200_PACK_HEAD_PAIRS 2
NPU_B200_API int npu_b200_pack_weight_rows(const void* d_w, int n_src_rows, int k, void* d_packed,
                                           int dst_rows, int order, int row_offset, void* stream);

/* Projection with a fused epilogue (the decode runtime's building block,
 * exposed for kernel-level use and tests).  acc[b, n] = sum_k x[b, k] w[n, k]
 * in FP32, times rn[b] = rsqrt(sum_p ssq_in[p * ssq_ld + b] / hidden + ssq_eps) when
 * ssq_in is set (the RMSNorm of x, whose weight the producer of x applied), then:
 *   STORE   out[b * ld_out + n] = act(acc + bias[n])                (FP16 or FP32)
 *   RESID   h = resid[b * ld_resid + n] + acc; resid = h;
 *           xw[b * ld_xw + n] = fp16(h * norm_w[n]);
 *           ssq_out[(n / R) * ssq_out_ld + b] = sum of h^2 over R rows,
 *           R = ssq_out_rows (128 or 16; 0 means 128)
 *   SWIGLU  gate and up rows interleaved: row 2j holds gate_j, row 2j + 1 up_j
 *           (pack_weight of [gate; up] with NPU_B200_PACK_INTERLEAVE);
 *           out[b * ld_out + j] = silu(gate_j) * up_j
 *   QKV     rows = [q_heads | kv_heads | kv_heads] x 128, each head's rows in
 *           rotary pair order: dims d and d + 64 are rows 2d and 2d + 1
 *           (NPU_B200_PACK_HEAD_PAIRS); optional per-head RMSNorm (q_norm_w /
 *           k_norm_w, qk_eps), RoPE (rotate-half) at positions[b] (inv_freq[64]),
 *           q -> out[b * ld_out + head * 128 + d], k / v -> cache
 *           [b][head][positions[b]][d] of [batch][kv_heads][max_seq][128]
 *   ARGMAX  per R = am_rows rows (128 or 16; 0 means 128):
 *           am_val / am_idx[(n / R) * am_ld + b] = max / argmax of acc over those
 *           rows (lowest row on ties).
 * Batches of 1-2 with packed weights, 16-row partials and no QK-norm run a
 * CUDA-core GEMV (no workspace used); the rest run on the tensor cores. */
enum {
  NPU_B200_EPI_STORE = 0,
  NPU_B200_EPI_RESID = 1,
  NPU_B200_EPI_SWIGLU = 2,
  NPU_B200_EPI_QKV = 3,
  NPU_B200_EPI_ARGMAX = 4
};
typedef struct npu_b200_epilogue {
  int kind;
  const float* ssq_in;
  int ssq_parts, ssq_ld, hidden;
  float ssq_eps;
  void* out;
  int ld_out, out_f32, relu;
  const void* bias;
  float* resid;
  int ld_resid;
  const void* norm_w;
  void* xw;
  int ld_xw;
  float* ssq_out;
  int ssq_out_ld;
  int q_heads, kv_heads;
  const int32_t* positions;
  const float* inv_freq;
  void* k_cache;
  void* v_cache;
  int max_seq;
  const void* q_norm_w;
  const void* k_norm_w;
  float qk_eps;
  float* am_val;
  int32_t* am_idx;
  int am_ld;
  int ssq_out_rows;
  int am_rows;
} npu_b200_epilogue;
NPU_B200_API int npu_b200_projection(const void* d_x, const void* d_w, int w_packed, int batch,
                                     int n_rows, int k, const npu_b200_epilogue* epilogue,
                                     void* d_workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Decode runtime (context-level).
 *
 * Replaces, for the B200 path, everything the reference runs after its front
 * end: npu-tile / npu-place / npu-hw-ops / npu-pipeline-attention /
 * npu-assign-addresses / npu-emit / encode-npu (include/npu/Transforms/Passes.h:24-31,
 * run by tools/npu-compile/npu-compile.cpp:376-454), the hbm.bin image builder
 * (npu-compile.cpp:495-659) and the simulator run (test/Integration/harness.py:19-33).
 *
 * A plan is a strict "key = value" text file (stage = cuda-plan, schema = 1,
 * model shape, max_batch, max_seq), the counterpart of the reference's stamped
 * stage files (npu-compile.cpp:226-316).  Weights are given by their transformers
 * parameter names, whole (unsharded); each rank keeps its tensor-parallel shard.
 * Each decode step runs as one CUDA graph per (entry point, batch), captured on
 * first use; the first call for a batch size therefore must not happen inside
 * another stream capture.
 * ------------------------------------------------------------------------- */
typedef struct npu_b200_ctx npu_b200_ctx;

/* 128-byte NCCL unique id for tp_size > 1 (rank 0 makes it, every rank passes it
 * to npu_b200_create).  NCCL is loaded on first use (NPU_B200_NCCL_LIBRARY
 * overrides the library name). */
NPU_B200_API int npu_b200_nccl_unique_id(void* h_out128);

/* Context on `device` for rank tp_rank of tp_size (tensor parallel: q/k/v and
 * gate/up column-sharded by heads / FFN columns, o/down row-sharded with one
 * all-reduce each, LM head sharded by vocabulary).  nccl_unique_id may be NULL
 * when tp_size == 1. */
NPU_B200_API int npu_b200_create(int device, int tp_rank, int tp_size, const void* nccl_unique_id,
                                 npu_b200_ctx** out);
NPU_B200_API int npu_b200_destroy(npu_b200_ctx* ctx);

/* Parse a plan and allocate this rank's weights, KV cache and buffers. */
NPU_B200_API int npu_b200_load_plan(npu_b200_ctx* ctx, const char* plan_path);

/* Parse and validate a plan without a GPU (the stage / schema / shape checks
 * npu_b200_load_plan makes); out[] as npu_b200_plan_info with tp_size 1. */
NPU_B200_API int npu_b200_plan_check(const char* plan_path, int64_t* out, int n);

/* The share of tensor-parallel rank tp_rank of tp_size under the plan, as the
 * runtime shards the weights when they are set (no counterpart in the
 * reference, which runs one core array): out[0..4] = q heads, KV heads, FFN
 * columns, vocabulary rows and the first vocabulary row of this rank.  Rank r
 * holds q heads [r*out[0], (r+1)*out[0]) and KV heads [r*out[1], (r+1)*out[1])
 * (rows of q/k/v_proj, columns of o_proj), FFN columns [r*out[2], (r+1)*out[2])
 * (rows of gate/up_proj, columns of down_proj) and LM-head rows
 * [out[4], out[4] + out[3]).  Host only: no GPU is needed. */
NPU_B200_API int npu_b200_shard_info(const char* plan_path, int tp_rank, int tp_size, int64_t* out,
                                     int n);

/* out[0..11] = layers, hidden, local q heads, local kv heads, local ffn, local vocab,
 * vocab offset, max_batch, max_seq, head_dim, plan fingerprint (FNV-1a), tp_size;
 * out[12] (when n >= 13) = 1 if the tensor-parallel all-reduces run over NVLink
 * peer memory, 0 if through NCCL (NPU_B200_TP_EXCHANGE=nccl, or CUDA IPC unusable). */
NPU_B200_API int npu_b200_plan_info(const npu_b200_ctx* ctx, int64_t* out, int n);

/* Copy one whole FP16 parameter (host or device memory) into this rank's layout.
 * `name` is its transformers name, e.g. "model.layers.3.self_attn.q_proj.weight";
 * a one-layer plan also accepts a captured block's names ("block.mlp.up_proj.weight"). */
NPU_B200_API int npu_b200_set_weight(npu_b200_ctx* ctx, const char* name, const void* src,
                                     size_t bytes);

/* Read every weight of a capture directory written by CaptureResult.write
 * (python/npu/capture/export.py:30-40: arguments.txt + arg<N>.bin). */
NPU_B200_API int npu_b200_load_capture(npu_b200_ctx* ctx, const char* capture_dir);

/* Per-rank weight image: this rank's packed weight panels and norms (its
 * tensor-parallel shard, already in the kernels' layout) as files under
 * dir/rank<r>-of-<N>/ with a descriptor (image.txt: stage = cuda-image,
 * schema = 1, the plan fingerprint, the rank, and per tensor its size and FNV-1a
 * checksum).  Loading checks every stamp, size and checksum and copies the
 * bytes as they are: no sharding, no packing.  The B200 counterpart of the
 * reference's hbm.bin image (tools/npu-compile/npu-compile.cpp:495-659).  Saving
 * needs every weight set; loading sets them all. */
NPU_B200_API int npu_b200_save_image(npu_b200_ctx* ctx, const char* dir);
NPU_B200_API int npu_b200_load_image(npu_b200_ctx* ctx, const char* dir);

/* Device pointers of one layer's KV cache, each [max_batch][local kv heads][max_seq][head_dim]
 * FP16; sequence b's key at position p lives at [b][h][p][:]. */
NPU_B200_API int npu_b200_kv_cache(npu_b200_ctx* ctx, int layer, void** d_k, void** d_v);

/* Greedy decode step of the whole stack: embed h_tokens[b], write K/V at
 * h_positions[b] and attend positions [0, h_positions[b]] in every layer, final
 * norm, LM head, argmax -> h_out_ids[b] (ties to the lowest id).  Host buffers;
 * returns after the ids are copied back (synchronizes `stream`). */
NPU_B200_API int npu_b200_decode_step(npu_b200_ctx* ctx, const int32_t* h_tokens,
                                      const int32_t* h_positions, int batch, int32_t* h_out_ids,
                                      void* stream);
/* Same with device buffers; asynchronous on `stream`. */
NPU_B200_API int npu_b200_decode_step_device(npu_b200_ctx* ctx, const int32_t* d_tokens,
                                             const int32_t* d_positions, int batch,
                                             int32_t* d_out_ids, void* stream);

/* Graph plans: a captured module run as a sequence of this library's kernels.
 *
 * The B200 counterpart of compiling a capture and running the program on the
 * reference's simulator (tools/npu-compile/npu-compile.cpp; the run with the
 * captured arguments, examples/pytorch/mlp.py): `dir` is a capture directory
 * (arguments.txt, arg<N>.bin, python/npu/capture/export.py:30-40) plus the
 * graph.txt that llm_compiler_3_b200/graph.py writes from a torch.export of the
 * module -- FP16 linear layers (+ bias, + ReLU) and scaled-dot-product attention
 * (causal or not, GQA), the ops of the reference's MLP and SDPA integration
 * cases (examples/pytorch/mlp.py, test/Integration/attention.py).  Decoder
 * layers and stacks run through npu_b200_load_plan instead.
 *
 * npu_b200_graph_check: parses and checks dir/graph.txt on the host (shapes,
 *   kernel limits, parameter files); out[0..5] = inputs, outputs, ops, parameter
 *   bytes, temporary bytes, attention ops that run as flash-decoding.
 * npu_b200_load_graph: the same checks, then parameters and temporaries into
 *   device memory owned by the context (one graph per context; loading another
 *   replaces it).
 * npu_b200_run_graph: args[i] / outs[i] are device pointers to the i-th input /
 *   output of graph.txt (in their line order), FP16, contiguous, 16-byte
 *   aligned; stream-ordered on `stream`.  Calls on one context must not overlap
 *   on the GPU (they share the temporaries). */
NPU_B200_API int npu_b200_graph_check(const char* dir, int64_t* out, int n);
NPU_B200_API int npu_b200_load_graph(npu_b200_ctx* ctx, const char* dir);
NPU_B200_API int npu_b200_run_graph(npu_b200_ctx* ctx, void* const* args, void* const* outs,
                                    void* stream);

/* The layers only, on hidden states: x [batch, hidden] FP16 in, y [batch, hidden]
 * FP16 out (the captured decoder layer's function, examples/llama/capture.py:38-54,
 * as a decode step).  Host-buffer version synchronizes `stream`. */
NPU_B200_API int npu_b200_forward_hidden(npu_b200_ctx* ctx, const void* h_x,
                                         const int32_t* h_positions, int batch, void* h_y,
                                         void* stream);
NPU_B200_API int npu_b200_forward_hidden_device(npu_b200_ctx* ctx, const void* d_x,
                                                const int32_t* d_positions, int batch, void* d_y,
                                                void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NPU_B200_H */
