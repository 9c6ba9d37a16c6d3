// Decode runtime: plan, per-rank weights and KV cache, one CUDA graph per
// (mode, batch), tensor parallelism over NVLink peer memory (NCCL for setup,
// and as the fallback exchange).
//
// This is the B200 counterpart of what LLM_Compiler_3 does after its front
// end: where the reference tiles, places, lowers and encodes the legalized graph
// for the NPU (lib/Transforms/{Tile,Place,HardwareOps,Emit,Encode}.cpp) and
// writes hbm.bin (tools/npu-compile/npu-compile.cpp:495-659), this library takes
// a plan (the decoder's shape, stamped like the reference's stage files:
// stage / schema / fingerprint, npu-compile.cpp:226-316) and the captured
// weights, lays the weights out per tensor-parallel rank, and runs each decode
// step as one captured CUDA graph of fused kernels:
//
//   residual_update(embed)                      h, xw = h*w_in, ssq
//   per layer:  proj[QKV: rms scale, (QK-norm), RoPE, KV append]
//               flash_decode (split-KV, GQA group per CTA)
//               proj[O: + residual, xw = h*w_post, ssq]        (TP: all-reduce first)
//               proj[gate|up: rms scale, SwiGLU]
//               proj[down: + residual, xw = h*w_next, ssq]     (TP: all-reduce first)
//   proj[LM head: rms scale, per-tile argmax] -> argmax_reduce (TP: gather over ranks)
//
// At batch 1-2 every proj runs as the CUDA-core GEMV (gemv.cu) and the sums of
// squares and partial argmaxes are kept per 16 rows; above, on the tensor
// cores with per-128-row partials.  With tensor parallelism the all-reduce is
// the exchange of peer.cuh: at batch 1-2 inside the GEMV's residual epilogue,
// above it in residual_update after a STORE projection (NCCL all-reduce when
// peer memory is unavailable).
// Every kernel is launched with programmatic dependent launch, so the next
// projection starts streaming its weights while the previous kernel drains.
#include <dlfcn.h>
#include <math.h>
#include <nccl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <filesystem>
#include <fstream>
#include <map>
#include <sstream>
#include <string>
#include <utility>
#include <vector>

#include "common.cuh"
#include "host.hpp"
#include "proj.cuh"
#include "small.cuh"

namespace npu_b200 {

int flash_decode_run(const void* q, const void* k, const void* v, const int32_t* seq_lens,
                     void* out, int batch, int q_heads, int kv_heads, int head_dim, int max_seq,
                     float scale, int num_splits, void* workspace, size_t workspace_bytes,
                     cudaStream_t stream, bool pdl, const int32_t* positions);
size_t flash_decode_workspace(int batch, int kv_heads, int head_dim, int max_seq, int num_splits);

namespace {

// ---------------------------------------------------------------------------
// Plan: strict "key = value" text, stamped like the reference's stage files.
// ---------------------------------------------------------------------------
struct Plan {
  std::string arch;
  int hidden = 0, heads = 0, kv_heads = 0, head_dim = 0, ffn = 0, layers = 0, vocab = 0;
  float eps = 0.f, rope_theta = 0.f;
  int qk_norm = 0, max_batch = 0, max_seq = 0;
  std::vector<float> inv_freq;
  uint64_t fingerprint = 0;
};

uint64_t fnv1a(const std::string& s) {
  uint64_t h = 1469598103934665603ull;
  for (unsigned char c : s) {
    h ^= c;
    h *= 1099511628211ull;
  }
  return h;
}

std::string trim(const std::string& s) {
  const size_t a = s.find_first_not_of(" \t\r\n");
  if (a == std::string::npos) return "";
  return s.substr(a, s.find_last_not_of(" \t\r\n") - a + 1);
}

int parse_int(const std::string& key, const std::string& v, int* out) {
  char* end = nullptr;
  const long x = strtol(v.c_str(), &end, 10);
  if (end == v.c_str() || *end != 0 || x < 0 || x > (1l << 30))
    return set_error(NPU_B200_E_PLAN, "plan: %s = '%s' is not a non-negative integer", key.c_str(),
                     v.c_str());
  *out = static_cast<int>(x);
  return NPU_B200_OK;
}

int parse_float(const std::string& key, const std::string& v, float* out) {
  char* end = nullptr;
  const double x = strtod(v.c_str(), &end);
  if (end == v.c_str() || *end != 0 || !std::isfinite(x))
    return set_error(NPU_B200_E_PLAN, "plan: %s = '%s' is not a finite number", key.c_str(),
                     v.c_str());
  *out = static_cast<float>(x);
  return NPU_B200_OK;
}

int parse_plan(const std::string& text, Plan* plan) {
  Plan p;
  std::map<std::string, std::string> kv;
  std::istringstream in(text);
  std::string line;
  int lineno = 0;
  while (std::getline(in, line)) {
    ++lineno;
    line = trim(line.substr(0, line.find('#')));
    if (line.empty()) continue;
    const size_t eq = line.find('=');
    if (eq == std::string::npos)
      return set_error(NPU_B200_E_PLAN, "plan line %d: expected key = value", lineno);
    const std::string key = trim(line.substr(0, eq)), val = trim(line.substr(eq + 1));
    if (kv.count(key)) return set_error(NPU_B200_E_PLAN, "plan: duplicate key '%s'", key.c_str());
    kv[key] = val;
  }
  static const char* kKeys[] = {"stage", "schema", "arch", "hidden", "heads", "kv_heads",
                                "head_dim", "ffn", "layers", "vocab", "rms_eps", "rope_theta",
                                "qk_norm", "max_batch", "max_seq", "inv_freq"};
  for (auto& e : kv) {
    bool known = false;
    for (const char* k : kKeys) known |= e.first == k;
    if (!known) return set_error(NPU_B200_E_PLAN, "plan: unknown key '%s'", e.first.c_str());
  }
  for (const char* k : kKeys)
    if (std::string(k) != "inv_freq" && !kv.count(k))
      return set_error(NPU_B200_E_PLAN, "plan: missing key '%s'", k);
  if (kv["stage"] != "cuda-plan")
    return set_error(NPU_B200_E_PLAN, "plan: stage '%s' is not cuda-plan", kv["stage"].c_str());
  if (kv["schema"] != "1")
    return set_error(NPU_B200_E_PLAN, "plan: schema %s is not supported (want 1)",
                     kv["schema"].c_str());
  p.arch = kv["arch"];
  if (p.arch != "llama" && p.arch != "qwen3")
    return set_error(NPU_B200_E_PLAN, "plan: arch '%s' is not llama or qwen3", p.arch.c_str());
  int rc = 0;
  if ((rc = parse_int("hidden", kv["hidden"], &p.hidden)) ||
      (rc = parse_int("heads", kv["heads"], &p.heads)) ||
      (rc = parse_int("kv_heads", kv["kv_heads"], &p.kv_heads)) ||
      (rc = parse_int("head_dim", kv["head_dim"], &p.head_dim)) ||
      (rc = parse_int("ffn", kv["ffn"], &p.ffn)) ||
      (rc = parse_int("layers", kv["layers"], &p.layers)) ||
      (rc = parse_int("vocab", kv["vocab"], &p.vocab)) ||
      (rc = parse_int("qk_norm", kv["qk_norm"], &p.qk_norm)) ||
      (rc = parse_int("max_batch", kv["max_batch"], &p.max_batch)) ||
      (rc = parse_int("max_seq", kv["max_seq"], &p.max_seq)) ||
      (rc = parse_float("rms_eps", kv["rms_eps"], &p.eps)) ||
      (rc = parse_float("rope_theta", kv["rope_theta"], &p.rope_theta)))
    return rc;
  if (p.head_dim != 128)
    return set_error(NPU_B200_E_UNSUPPORTED, "plan: head_dim %d (this build fuses 128 only)",
                     p.head_dim);
  if (p.hidden % 128 || p.hidden < 128 || p.heads < 1 || p.kv_heads < 1 ||
      p.heads % p.kv_heads || p.heads / p.kv_heads > 8 || p.ffn % 64 || p.ffn < 64 ||
      p.layers < 1 || p.max_batch < 1 || p.max_batch > 128 || p.max_seq < 1 || p.eps <= 0.f ||
      p.rope_theta <= 0.f || p.qk_norm > 1)
    return set_error(NPU_B200_E_PLAN, "plan: inconsistent shape");
  if (p.qk_norm != (p.arch == "qwen3" ? 1 : 0))
    return set_error(NPU_B200_E_PLAN, "plan: qk_norm must be 1 for qwen3 and 0 for llama");
  const int half = p.head_dim / 2;
  if (kv.count("inv_freq")) {
    std::istringstream fs(kv["inv_freq"]);
    std::string tok;
    while (fs >> tok) {
      float f = 0.f;
      if ((rc = parse_float("inv_freq", tok, &f))) return rc;
      p.inv_freq.push_back(f);
    }
    if (static_cast<int>(p.inv_freq.size()) != half)
      return set_error(NPU_B200_E_PLAN, "plan: inv_freq has %zu entries, want %d",
                       p.inv_freq.size(), half);
  } else {
    for (int i = 0; i < half; ++i)
      p.inv_freq.push_back(1.0f / powf(p.rope_theta, static_cast<float>(2 * i) / p.head_dim));
  }
  p.fingerprint = fnv1a(text);
  *plan = p;
  return NPU_B200_OK;
}

// ---------------------------------------------------------------------------
// NCCL, loaded on demand so single-GPU use needs no NCCL at all.
// ---------------------------------------------------------------------------
struct NcclApi {
  void* handle = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

NcclApi g_nccl;

int load_nccl() {
  if (g_nccl.handle) return NPU_B200_OK;
  const char* env = getenv("NPU_B200_NCCL_LIBRARY");
  const char* name = env && *env ? env : "libnccl.so.2";
  void* h = dlopen(name, RTLD_NOW | RTLD_GLOBAL);
  if (!h) return set_error(NPU_B200_E_NCCL, "cannot load NCCL (%s): %s", name, dlerror());
  NcclApi api;
  api.handle = h;
#define NPU_SYM(field, sym)                                                         \
  api.field = reinterpret_cast<decltype(api.field)>(dlsym(h, sym));                 \
  if (!api.field) {                                                                 \
    dlclose(h);                                                                     \
    return set_error(NPU_B200_E_NCCL, "NCCL library %s lacks %s", name, sym);       \
  }
  NPU_SYM(GetUniqueId, "ncclGetUniqueId")
  NPU_SYM(CommInitRank, "ncclCommInitRank")
  NPU_SYM(CommDestroy, "ncclCommDestroy")
  NPU_SYM(AllReduce, "ncclAllReduce")
  NPU_SYM(AllGather, "ncclAllGather")
  NPU_SYM(GetErrorString, "ncclGetErrorString")
#undef NPU_SYM
  g_nccl = api;
  return NPU_B200_OK;
}

int check_nccl(ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return NPU_B200_OK;
  return set_error(NPU_B200_E_NCCL, "%s failed: %s", what,
                   g_nccl.GetErrorString ? g_nccl.GetErrorString(r) : "?");
}

// ---------------------------------------------------------------------------
// Weights: which tensor of the model a parameter name refers to.
// ---------------------------------------------------------------------------
enum TensorKind {
  kQ, kK, kV, kO, kGate, kUp, kDown, kInNorm, kPostNorm, kQNorm, kKNorm,  // per layer
  kEmbed, kFinalNorm, kLmHead, kNumKinds
};
constexpr int kPerLayerKinds = kEmbed;

struct NameRule {
  const char* suffix;
  int kind;
};
const NameRule kRules[] = {
    {"self_attn.q_proj.weight", kQ},          {"self_attn.k_proj.weight", kK},
    {"self_attn.v_proj.weight", kV},          {"self_attn.o_proj.weight", kO},
    {"mlp.gate_proj.weight", kGate},          {"mlp.up_proj.weight", kUp},
    {"mlp.down_proj.weight", kDown},          {"input_layernorm.weight", kInNorm},
    {"post_attention_layernorm.weight", kPostNorm}, {"self_attn.q_norm.weight", kQNorm},
    {"self_attn.k_norm.weight", kKNorm},      {"embed_tokens.weight", kEmbed},
    {"lm_head.weight", kLmHead},
};

bool ends_with(const std::string& s, const std::string& t) {
  return s.size() >= t.size() && s.compare(s.size() - t.size(), t.size(), t) == 0;
}

}  // namespace

struct LayerBuffers {
  __half *w_qkv = nullptr, *w_o = nullptr, *w_gu = nullptr, *w_down = nullptr;
  __half *in_norm = nullptr, *post_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
  __half *k_cache = nullptr, *v_cache = nullptr;
};

}  // namespace npu_b200

using namespace npu_b200;

struct npu_b200_ctx {
  int device = 0, tp_rank = 0, tp_size = 1;
  cudaStream_t stream = nullptr;      // capture stream
  ncclComm_t comm = nullptr;
  bool loaded = false;
  Plan plan;
  int q_loc = 0, kv_loc = 0, ffn_loc = 0, vocab_loc = 0, vocab_off = 0;
  std::vector<void*> device_allocs;
  std::vector<void*> host_allocs;
  std::vector<LayerBuffers> layers;
  __half *embed = nullptr, *final_norm = nullptr, *lm_head = nullptr;
  float *resid = nullptr, *ssq = nullptr, *partial = nullptr, *d_inv_freq = nullptr;
  float* rope_tab = nullptr;  // [max_batch][64] (cos, sin) of this step's positions
  __half *xw = nullptr, *q_buf = nullptr, *attn = nullptr, *act = nullptr, *hidden_io = nullptr;
  int32_t *d_tokens = nullptr, *d_positions = nullptr, *d_seq_lens = nullptr, *d_ids = nullptr;
  float *am_val = nullptr, *gather_send = nullptr, *gather_recv = nullptr;
  int32_t* am_idx = nullptr;
  void* proj_ws = nullptr;
  size_t proj_ws_bytes = 0;
  void* fd_ws = nullptr;
  size_t fd_ws_bytes = 0;
  int32_t *h_tokens = nullptr, *h_positions = nullptr, *h_ids = nullptr;
  __half* h_hidden = nullptr;
  std::map<std::pair<int, int>, cudaGraphExec_t> graphs;  // (mode, batch)
  std::vector<uint8_t> have;                              // [layers * kPerLayerKinds + 3]
  // Tensor parallel over NVLink peer memory (peer.cuh): this rank's exchange
  // buffer, the peers' opened through CUDA IPC, the step counter.
  uint32_t* epoch = nullptr;
  uint64_t* px_part = nullptr;
  std::vector<void*> px_opened;  // peers' IPC mappings, closed before the local buffers are freed
  bool px_ready = false;         // false: the all-reduces go through NCCL
  PeerExchange px;               // seq filled in per exchange
  GraphState* graph = nullptr;   // npu_b200_load_graph (graph.cu)
};

namespace npu_b200 {
namespace {

enum GraphMode { kModeTokens = 0, kModeHidden = 1 };

int dev_alloc(npu_b200_ctx* c, size_t bytes, void** out, bool zero) {
  void* p = nullptr;
  NPU_TRY_CUDA(cudaMalloc(&p, bytes < 256 ? 256 : bytes));
  c->device_allocs.push_back(p);
  if (zero) NPU_TRY_CUDA(cudaMemset(p, 0, bytes < 256 ? 256 : bytes));
  *out = p;
  return NPU_B200_OK;
}

template <typename T>
int dalloc(npu_b200_ctx* c, size_t count, T** out, bool zero = true) {
  void* p = nullptr;
  int rc = dev_alloc(c, count * sizeof(T), &p, zero);
  *out = static_cast<T*>(p);
  return rc;
}

template <typename T>
int halloc(npu_b200_ctx* c, size_t count, T** out) {
  void* p = nullptr;
  NPU_TRY_CUDA(cudaMallocHost(&p, count * sizeof(T) < 64 ? 64 : count * sizeof(T)));
  c->host_allocs.push_back(p);
  *out = static_cast<T*>(p);
  return NPU_B200_OK;
}

void release(npu_b200_ctx* c) {
  for (auto& g : c->graphs) cudaGraphExecDestroy(g.second);
  c->graphs.clear();
  for (void* p : c->px_opened) cudaIpcCloseMemHandle(p);
  c->px_opened.clear();
  c->px_ready = false;
  for (void* p : c->device_allocs) cudaFree(p);
  c->device_allocs.clear();
  for (void* p : c->host_allocs) cudaFreeHost(p);
  c->host_allocs.clear();
  c->layers.clear();
  c->loaded = false;
}

// Opens every rank's exchange buffers through CUDA IPC (handles all-gathered
// over NCCL, a collective of all ranks).  If this machine does not allow it, or
// NPU_B200_TP_EXCHANGE=nccl, the all-reduces stay on NCCL; every rank must take
// the same path, so the ranks agree on it with one more all-reduce.
int setup_peer_exchange(npu_b200_ctx* c) {
  const Plan& P = c->plan;
  const int T = c->tp_size;
  NPU_REQUIRE(T <= kMaxRanks, "tensor parallel: at most %d ranks", kMaxRanks);
  const size_t B = static_cast<size_t>(P.max_batch), H = static_cast<size_t>(P.hidden);
  const size_t part_words = 4 * B * H + B * 2;  // partials, argmax, reduced sums (peer.cuh)
  int rc = 0;
  if ((rc = dalloc(c, part_words, &c->px_part))) return rc;
  const char* env = getenv("NPU_B200_TP_EXCHANGE");
  int usable = !(env && strcmp(env, "nccl") == 0);
  cudaIpcMemHandle_t mine;
  memset(&mine, 0, sizeof(mine));
  if (usable && cudaIpcGetMemHandle(&mine, c->px_part) != cudaSuccess) {
    cudaGetLastError();
    usable = 0;
  }
  // Every rank's handle, and a vote (minimum over ranks) on whether to use them.
  const size_t hbytes = sizeof(cudaIpcMemHandle_t);
  uint8_t* d_all = nullptr;
  int32_t* d_vote = nullptr;
  if ((rc = dalloc(c, hbytes * T, &d_all)) || (rc = dalloc(c, 1, &d_vote))) return rc;
  NPU_TRY_CUDA(cudaMemcpy(d_all + hbytes * c->tp_rank, &mine, hbytes, cudaMemcpyHostToDevice));
  NPU_TRY_CUDA(cudaMemcpy(d_vote, &usable, sizeof(int32_t), cudaMemcpyHostToDevice));
  if ((rc = check_nccl(g_nccl.AllGather(d_all + hbytes * c->tp_rank, d_all, hbytes, ncclUint8,
                                        c->comm, c->stream),
                       "ncclAllGather(ipc handles)")) ||
      (rc = check_nccl(g_nccl.AllReduce(d_vote, d_vote, 1, ncclInt32, ncclMin, c->comm, c->stream),
                       "ncclAllReduce(peer exchange vote)")))
    return rc;
  NPU_TRY_CUDA(cudaStreamSynchronize(c->stream));
  std::vector<uint8_t> all(hbytes * T);
  int32_t agreed = 0;
  NPU_TRY_CUDA(cudaMemcpy(all.data(), d_all, all.size(), cudaMemcpyDeviceToHost));
  NPU_TRY_CUDA(cudaMemcpy(&agreed, d_vote, sizeof(int32_t), cudaMemcpyDeviceToHost));
  PeerExchange& x = c->px;
  x.rank = c->tp_rank;
  x.ranks = T;
  x.max_batch = P.max_batch;
  x.hidden = P.hidden;
  x.epoch = c->epoch;
  int opened_ok = agreed;
  for (int r = 0; r < T && opened_ok; ++r) {
    if (r == c->tp_rank) {
      x.part[r] = c->px_part;
      continue;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, all.data() + hbytes * r, sizeof(h));
    void* pr = nullptr;
    if (cudaIpcOpenMemHandle(&pr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      opened_ok = 0;
      break;
    }
    c->px_opened.push_back(pr);
    x.part[r] = static_cast<uint64_t*>(pr);
  }
  // Every rank must have opened every peer before anyone relies on it.
  NPU_TRY_CUDA(cudaMemcpy(d_vote, &opened_ok, sizeof(int32_t), cudaMemcpyHostToDevice));
  if ((rc = check_nccl(g_nccl.AllReduce(d_vote, d_vote, 1, ncclInt32, ncclMin, c->comm, c->stream),
                       "ncclAllReduce(peer exchange vote)")))
    return rc;
  NPU_TRY_CUDA(cudaStreamSynchronize(c->stream));
  NPU_TRY_CUDA(cudaMemcpy(&agreed, d_vote, sizeof(int32_t), cudaMemcpyDeviceToHost));
  c->px_ready = agreed != 0;
  return NPU_B200_OK;
}

// What tensor-parallel rank r of T holds (Megatron-style): q heads
// [r q_loc, (r+1) q_loc) and KV heads [r kv_loc, (r+1) kv_loc) of the q/k/v
// rows and of o_proj's columns, FFN columns [r ffn_loc, (r+1) ffn_loc) of
// gate/up rows and down_proj columns, vocabulary rows [vocab_off, vocab_off +
// vocab_loc) of the LM head.
struct Shard {
  int q_loc = 0, kv_loc = 0, ffn_loc = 0, vocab_loc = 0, vocab_off = 0;
};

int shard_layout(const Plan& P, int T, int r, Shard* s) {
  NPU_REQUIRE(T >= 1 && r >= 0 && r < T, "bad tp rank %d / size %d", r, T);
  NPU_REQUIRE(P.kv_heads % T == 0, "plan: kv_heads %d not divisible by tp_size %d", P.kv_heads, T);
  NPU_REQUIRE(P.ffn % (64 * T) == 0, "plan: ffn %d not divisible by 64 * tp_size", P.ffn);
  s->kv_loc = P.kv_heads / T;
  s->q_loc = P.heads / T;
  s->ffn_loc = P.ffn / T;
  s->vocab_loc = s->vocab_off = 0;
  if (P.vocab > 0) {
    s->vocab_loc = (P.vocab + T - 1) / T;
    s->vocab_off = r * s->vocab_loc;
    if (s->vocab_off + s->vocab_loc > P.vocab) s->vocab_loc = P.vocab - s->vocab_off;
    NPU_REQUIRE(s->vocab_loc >= 1, "plan: vocab %d too small for tp_size %d", P.vocab, T);
  }
  return NPU_B200_OK;
}

int allocate(npu_b200_ctx* c) {
  const Plan& P = c->plan;
  const int T = c->tp_size, r = c->tp_rank;
  Shard sh;
  if (int rc0 = shard_layout(P, T, r, &sh)) return rc0;
  c->kv_loc = sh.kv_loc;
  c->q_loc = sh.q_loc;
  c->ffn_loc = sh.ffn_loc;
  c->vocab_loc = sh.vocab_loc;
  c->vocab_off = sh.vocab_off;
  const size_t H = P.hidden, B = P.max_batch, D = P.head_dim;
  int rc = 0;
  c->layers.assign(P.layers, LayerBuffers());
  const size_t cache_elems = B * c->kv_loc * P.max_seq * D;
  for (int l = 0; l < P.layers; ++l) {
    LayerBuffers& L = c->layers[l];
    const int qkv_rows = (c->q_loc + 2 * c->kv_loc) * static_cast<int>(D);
    if ((rc = dalloc(c, packed_weight_bytes(qkv_rows, static_cast<int>(H)) / 2, &L.w_qkv)) ||
        (rc = dalloc(c, packed_weight_bytes(static_cast<int>(H), c->q_loc * static_cast<int>(D)) / 2,
                     &L.w_o)) ||
        (rc = dalloc(c, packed_weight_bytes(2 * c->ffn_loc, static_cast<int>(H)) / 2, &L.w_gu)) ||
        (rc = dalloc(c, packed_weight_bytes(static_cast<int>(H), c->ffn_loc) / 2, &L.w_down)) ||
        (rc = dalloc(c, H, &L.in_norm, false)) || (rc = dalloc(c, H, &L.post_norm, false)) ||
        (rc = dalloc(c, cache_elems, &L.k_cache)) || (rc = dalloc(c, cache_elems, &L.v_cache)))
      return rc;
    if (P.qk_norm &&
        ((rc = dalloc(c, D, &L.q_norm, false)) || (rc = dalloc(c, D, &L.k_norm, false))))
      return rc;
  }
  if (P.vocab > 0) {
    if ((rc = dalloc(c, static_cast<size_t>(P.vocab) * H, &c->embed, false)) ||
        (rc = dalloc(c, H, &c->final_norm, false)) ||
        (rc = dalloc(c, packed_weight_bytes(c->vocab_loc, static_cast<int>(H)) / 2, &c->lm_head)))
      return rc;
    // Partial argmaxes: one per 16 rows at batch 1-2, per 128 rows above.
    const int lm_parts = (c->vocab_loc + 15) / 16;
    if ((rc = dalloc(c, static_cast<size_t>(lm_parts) * B, &c->am_val)) ||
        (rc = dalloc(c, static_cast<size_t>(lm_parts) * B, &c->am_idx)) ||
        (rc = dalloc(c, 2 * B, &c->gather_send)) ||
        (rc = dalloc(c, 2 * B * static_cast<size_t>(T), &c->gather_recv)))
      return rc;
  }
  if ((rc = dalloc(c, B * H, &c->resid)) || (rc = dalloc(c, B * H, &c->xw)) ||
      (rc = dalloc(c, (H / 16) * B, &c->ssq)) || (rc = dalloc(c, B * H, &c->partial)) ||
      (rc = dalloc(c, B * c->q_loc * D, &c->q_buf)) || (rc = dalloc(c, B * c->q_loc * D, &c->attn)) ||
      (rc = dalloc(c, B * c->ffn_loc, &c->act)) || (rc = dalloc(c, B * H, &c->hidden_io)) ||
      (rc = dalloc(c, B, &c->d_tokens)) || (rc = dalloc(c, B, &c->d_positions)) ||
      (rc = dalloc(c, B, &c->d_seq_lens)) || (rc = dalloc(c, B, &c->d_ids)) ||
      (rc = dalloc(c, P.inv_freq.size(), &c->d_inv_freq)) ||
      (rc = dalloc(c, B * 128, &c->rope_tab)))
    return rc;
  NPU_TRY_CUDA(cudaMemcpy(c->d_inv_freq, P.inv_freq.data(), P.inv_freq.size() * sizeof(float),
                          cudaMemcpyHostToDevice));
  // Scratch shared by every kernel of a step: each leaves it zero-filled.
  size_t ws = 0;
  const int ks[] = {static_cast<int>(H), c->q_loc * static_cast<int>(D), c->ffn_loc};
  const int ns[] = {(c->q_loc + 2 * c->kv_loc) * static_cast<int>(D), static_cast<int>(H),
                    2 * c->ffn_loc, c->vocab_loc > 0 ? c->vocab_loc : 1};
  for (int batch = 1; batch <= static_cast<int>(B); ++batch)
    for (int n : ns)
      for (int k : ks) {
        const size_t w = proj_workspace_bytes(n, k, batch);
        ws = w > ws ? w : ws;
      }
  c->proj_ws_bytes = ws;
  if ((rc = dev_alloc(c, ws, &c->proj_ws, true))) return rc;
  size_t fws = 0;
  for (int batch = 1; batch <= static_cast<int>(B); ++batch) {
    const size_t w = flash_decode_workspace(batch, c->kv_loc, static_cast<int>(D), P.max_seq, 0);
    fws = w > fws ? w : fws;
  }
  c->fd_ws_bytes = fws;
  if ((rc = dev_alloc(c, fws, &c->fd_ws, true))) return rc;
  if ((rc = halloc(c, B, &c->h_tokens)) || (rc = halloc(c, B, &c->h_positions)) ||
      (rc = halloc(c, B, &c->h_ids)) || (rc = halloc(c, B * H, &c->h_hidden)))
    return rc;
  c->have.assign(static_cast<size_t>(P.layers) * kPerLayerKinds + 3, 0);
  if ((rc = dalloc(c, 1, &c->epoch))) return rc;
  if (T > 1 && (rc = setup_peer_exchange(c))) return rc;
  return NPU_B200_OK;
}

int required_missing(const npu_b200_ctx* c, bool tokens_mode, std::string* what) {
  const Plan& P = c->plan;
  static const char* kNames[] = {"q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj",
                                 "down_proj", "input_layernorm", "post_attention_layernorm",
                                 "q_norm", "k_norm"};
  for (int l = 0; l < P.layers; ++l)
    for (int k = 0; k < kPerLayerKinds; ++k) {
      if ((k == kQNorm || k == kKNorm) && !P.qk_norm) continue;
      if (!c->have[l * kPerLayerKinds + k]) {
        *what = "layer " + std::to_string(l) + " " + kNames[k];
        return 1;
      }
    }
  if (tokens_mode) {
    static const char* kTop[] = {"embed_tokens", "norm", "lm_head"};
    for (int i = 0; i < 3; ++i)
      if (!c->have[static_cast<size_t>(P.layers) * kPerLayerKinds + i]) {
        *what = kTop[i];
        return 1;
      }
  }
  return 0;
}

// Copy (a shard of) one full tensor into the context's layout.
int place_weight(npu_b200_ctx* c, int layer, int kind, const void* src, size_t bytes) {
  const Plan& P = c->plan;
  const size_t H = P.hidden, D = P.head_dim;
  const int r = c->tp_rank;
  auto expect = [&](size_t elems) -> int {
    if (bytes != elems * 2)
      return set_error(NPU_B200_E_INVALID, "weight: %zu bytes given, tensor has %zu", bytes,
                       elems * 2);
    return NPU_B200_OK;
  };
  int rc = 0;
  const uint8_t* s = static_cast<const uint8_t*>(src);
  cudaStream_t st = c->stream;
  // The source may still be being written by work on other streams (e.g. the
  // caller's generator kernels): the context stream does not order with them.
  NPU_TRY_CUDA(cudaDeviceSynchronize());
  // Matrices are packed into weight panels from a device copy of the source.
  void* tmp = nullptr;
  auto device_source = [&](const void** dsrc) -> int {
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, src) == cudaSuccess &&
        (attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged) &&
        attr.device == c->device) {
      *dsrc = src;
      return NPU_B200_OK;
    }
    cudaGetLastError();
    NPU_TRY_CUDA(cudaMalloc(&tmp, bytes));
    // Stream-ordered with the packing kernel that reads it (a synchronous copy
    // from pageable memory may return before its DMA has landed).
    NPU_TRY_CUDA(cudaMemcpyAsync(tmp, src, bytes, cudaMemcpyDefault, st));
    *dsrc = tmp;
    return NPU_B200_OK;
  };
  struct TmpGuard {
    void** p;
    ~TmpGuard() {
      if (*p) cudaFree(*p);
    }
  } guard{&tmp};
  const int Hi = static_cast<int>(H), Di = static_cast<int>(D);
  if (kind < kPerLayerKinds) {
    LayerBuffers& L = c->layers[layer];
    const void* d = nullptr;
    switch (kind) {
      case kQ:
      case kK:
      case kV: {
        const int heads = kind == kQ ? P.heads : P.kv_heads;
        const int loc = kind == kQ ? c->q_loc : c->kv_loc;
        if ((rc = expect(heads * D * H)) || (rc = device_source(&d))) return rc;
        const int row0 = kind == kQ ? 0 : (kind == kK ? c->q_loc : c->q_loc + c->kv_loc) * Di;
        const int rows = (c->q_loc + 2 * c->kv_loc) * Di;
        if ((rc = pack_weight(static_cast<const __half*>(d) + static_cast<size_t>(r) * loc * D * H,
                              H, loc * Di, Hi, L.w_qkv, rows, 2, row0, st)))
          return rc;
        break;
      }
      case kO: {  // [H, heads*D]: this rank's column block
        if ((rc = expect(H * P.heads * D)) || (rc = device_source(&d))) return rc;
        const int cols = c->q_loc * Di;
        if ((rc = pack_weight(static_cast<const __half*>(d) + static_cast<size_t>(r) * cols,
                              static_cast<size_t>(P.heads) * D, Hi, cols, L.w_o, Hi, 0, 0, st)))
          return rc;
        break;
      }
      case kGate:
      case kUp: {  // rows interleaved: gate_j at row 2j, up_j at row 2j + 1
        if ((rc = expect(static_cast<size_t>(P.ffn) * H)) || (rc = device_source(&d))) return rc;
        if ((rc = pack_weight(static_cast<const __half*>(d) + static_cast<size_t>(r) * c->ffn_loc * H,
                              H, c->ffn_loc, Hi, L.w_gu, 2 * c->ffn_loc, 1, kind == kUp ? 1 : 0,
                              st)))
          return rc;
        break;
      }
      case kDown: {  // [H, ffn]: this rank's column block
        if ((rc = expect(H * P.ffn)) || (rc = device_source(&d))) return rc;
        if ((rc = pack_weight(static_cast<const __half*>(d) + static_cast<size_t>(r) * c->ffn_loc,
                              static_cast<size_t>(P.ffn), Hi, c->ffn_loc, L.w_down, Hi, 0, 0, st)))
          return rc;
        break;
      }
      case kInNorm:
      case kPostNorm:
        if ((rc = expect(H))) return rc;
        NPU_TRY_CUDA(cudaMemcpyAsync(kind == kInNorm ? L.in_norm : L.post_norm, s, H * 2,
                                     cudaMemcpyDefault, st));
        break;
      case kQNorm:
      case kKNorm:
        NPU_REQUIRE(P.qk_norm, "weight: q_norm/k_norm given for a model without QK-norm");
        if ((rc = expect(D))) return rc;
        NPU_TRY_CUDA(cudaMemcpyAsync(kind == kQNorm ? L.q_norm : L.k_norm, s, D * 2,
                                     cudaMemcpyDefault, st));
        break;
    }
    c->have[static_cast<size_t>(layer) * kPerLayerKinds + kind] = 1;
  } else {
    NPU_REQUIRE(P.vocab > 0, "weight: plan has no vocabulary (hidden-state plan)");
    const size_t top = static_cast<size_t>(P.layers) * kPerLayerKinds;
    if (kind == kEmbed) {
      if ((rc = expect(static_cast<size_t>(P.vocab) * H))) return rc;
      NPU_TRY_CUDA(cudaMemcpyAsync(c->embed, s, bytes, cudaMemcpyDefault, st));
      c->have[top + 0] = 1;
    } else if (kind == kFinalNorm) {
      if ((rc = expect(H))) return rc;
      NPU_TRY_CUDA(cudaMemcpyAsync(c->final_norm, s, H * 2, cudaMemcpyDefault, st));
      c->have[top + 1] = 1;
    } else {
      const void* d = nullptr;
      if ((rc = expect(static_cast<size_t>(P.vocab) * H)) || (rc = device_source(&d))) return rc;
      if ((rc = pack_weight(static_cast<const __half*>(d) + static_cast<size_t>(c->vocab_off) * H, H,
                            c->vocab_loc, Hi, c->lm_head, c->vocab_loc, 0, 0, st)))
        return rc;
      c->have[top + 2] = 1;
    }
  }
  NPU_TRY_CUDA(cudaStreamSynchronize(st));
  return NPU_B200_OK;
}

int resolve_name(const npu_b200_ctx* c, const std::string& name, int* layer, int* kind) {
  const Plan& P = c->plan;
  *kind = -1;
  for (const NameRule& rule : kRules)
    if (ends_with(name, rule.suffix)) {
      *kind = rule.kind;
      break;
    }
  if (*kind < 0) {
    if (name == "norm.weight" || ends_with(name, ".norm.weight")) *kind = kFinalNorm;
    else return set_error(NPU_B200_E_INVALID, "weight: unknown parameter name '%s'", name.c_str());
  }
  *layer = -1;
  if (*kind < kPerLayerKinds) {
    const size_t at = name.find("layers.");
    if (at != std::string::npos) {
      *layer = atoi(name.c_str() + at + 7);
    } else if (P.layers == 1) {
      *layer = 0;  // a single captured block ("block.self_attn.q_proj.weight")
    }
    if (*layer < 0 || *layer >= P.layers)
      return set_error(NPU_B200_E_INVALID, "weight: '%s' names no layer of this plan", name.c_str());
  }
  return NPU_B200_OK;
}

// ---------------------------------------------------------------------------
// One decode step, enqueued on `s` (used under stream capture).
// ---------------------------------------------------------------------------
// Rows per partial sum of squares / partial argmax: 16 at batch 1-2 (the
// shapes the GEMV runs, one partial per 16-row CTA group), 128 above.
int part_rows(int batch) { return batch <= 2 ? 16 : 128; }

void norm_input(const npu_b200_ctx* c, int batch, EpiParams* e) {
  e->ssq_in = c->ssq;
  e->ssq_parts = c->plan.hidden / part_rows(batch);
  e->ssq_ld = c->plan.max_batch;
  e->ssq_inv_hidden = 1.f / static_cast<float>(c->plan.hidden);
  e->ssq_eps = c->plan.eps;
}

// The projection that closes a sub-block (o_proj / down_proj): residual add
// and the next RMSNorm's input; with tensor parallelism first the sum of the
// ranks' partials (exchange `seq` of the step: 2 per layer).
int residual_out(npu_b200_ctx* c, const __half* w, const void* x, int k, int batch,
                 const __half* next_norm, int seq, cudaStream_t s) {
  const Plan& P = c->plan;
  EpiParams e;
  e.n_rows = P.hidden;
  e.batch = batch;
  e.kind = kEpiResid;
  e.resid = c->resid;
  e.ld_resid = P.hidden;
  e.norm_w = next_norm;
  e.xw = c->xw;
  e.ld_xw = P.hidden;
  e.ssq_out = c->ssq;
  e.ssq_out_ld = P.max_batch;
  e.ssq_out_rows = part_rows(batch);
  if (c->tp_size == 1)
    return proj_run(w, true, x, P.hidden, k, batch, e, c->proj_ws, c->proj_ws_bytes, s, true);
  // Batch 1-2 with peer exchange: the GEMV's residual epilogue all-reduces
  // the partials itself (no separate kernel).
  if (c->px_ready && gemv_supported(P.hidden, k, batch, e)) {
    e.px = c->px;
    e.px.seq = seq;
    return proj_run(w, true, x, P.hidden, k, batch, e, c->proj_ws, c->proj_ws_bytes, s, true);
  }
  e = EpiParams();
  e.n_rows = P.hidden;
  e.batch = batch;
  e.kind = kEpiStore;
  e.out = c->partial;
  e.ld_out = P.hidden;
  e.out_f32 = 1;
  if (c->px_ready) {  // tagged partials into this rank's exchange buffer
    e.px = c->px;
    e.px.seq = seq;
  }
  int rc = proj_run(w, true, x, P.hidden, k, batch, e, c->proj_ws, c->proj_ws_bytes, s, true);
  if (rc) return rc;
  if (!c->px_ready &&
      (rc = check_nccl(g_nccl.AllReduce(c->partial, c->partial,
                                        static_cast<size_t>(batch) * P.hidden, ncclFloat32,
                                        ncclSum, c->comm, s),
                       "ncclAllReduce")))
    return rc;
  ResidualUpdate u;
  if (c->px_ready) {
    u.px = c->px;
    u.px.seq = seq;
    // Two-shot when the bytes it saves on each rank's NVLink, (R-1)(R-2)/R of
    // the tagged partials, outweigh its second hop and wait: measured at two
    // ranks, where both forms move the same bytes, 5.8 us per exchange more
    // (batch 64: 6.67 against 6.29 ms per step), ~4.5 MB at 770 GB/s.  At
    // batch 64 over 8 ranks it saves 11 MB (~14 us) per exchange; over 4
    // ranks 3 MB, less than its cost.
    // NPU_B200_TP_TWO_SHOT=1 / 0 forces it on (where the shape allows) / off;
    // every rank must see the same setting.
    const int R = c->tp_size;
    const double saved = static_cast<double>(R - 1) * (R - 2) / R * batch * P.hidden * 8.0;
    const bool possible = P.hidden % (32 * R) == 0 &&
                          static_cast<long long>(P.hidden / 128) * batch <= 16ll * sm_count();
    const char* force = getenv("NPU_B200_TP_TWO_SHOT");
    u.two_shot = possible && (force && force[0] == '1'   ? true
                              : force && force[0] == '0' ? false
                                                         : R >= 3 && saved > 4.5e6);
  }
  u.mode = kResidAddPartial;
  u.batch = batch;
  u.hidden = P.hidden;
  u.partial = c->partial;
  u.resid = c->resid;
  u.norm_w = next_norm;
  u.xw = c->xw;
  u.ssq_out = c->ssq;
  u.ssq_ld = P.max_batch;
  u.ssq_rows = part_rows(batch);
  return residual_update(u, s, c->px_ready);  // PDL only after our own kernel, not NCCL
}

EpiParams qkv_epi(const npu_b200_ctx* c, int l, int batch) {
  const Plan& P = c->plan;
  const LayerBuffers& L = c->layers[l];
  const int D = P.head_dim;
  EpiParams q;
  q.kind = kEpiQKV;
  q.n_rows = (c->q_loc + 2 * c->kv_loc) * D;
  q.batch = batch;
  norm_input(c, batch, &q);
  q.out = c->q_buf;
  q.ld_out = c->q_loc * D;
  q.q_heads = c->q_loc;
  q.kv_heads = c->kv_loc;
  q.positions = c->d_positions;
  q.inv_freq = c->d_inv_freq;
  q.rope_tab = c->rope_tab;
  q.k_cache = L.k_cache;
  q.v_cache = L.v_cache;
  q.max_seq = P.max_seq;
  q.cache_batch_stride = c->kv_loc * P.max_seq * D;
  q.q_norm_w = L.q_norm;
  q.k_norm_w = L.k_norm;
  q.qk_eps = P.eps;
  return q;
}

EpiParams swiglu_epi(const npu_b200_ctx* c, int batch) {
  EpiParams g;
  g.kind = kEpiSwiGLU;
  g.n_rows = 2 * c->ffn_loc;
  g.batch = batch;
  norm_input(c, batch, &g);
  g.out = c->act;
  g.ld_out = c->ffn_loc;
  return g;
}

EpiParams argmax_epi(const npu_b200_ctx* c, int batch) {
  EpiParams a;
  a.kind = kEpiArgmax;
  a.n_rows = c->vocab_loc;
  a.batch = batch;
  norm_input(c, batch, &a);
  a.am_val = c->am_val;
  a.am_idx = c->am_idx;
  a.am_ld = c->plan.max_batch;
  a.am_rows = part_rows(batch);
  return a;
}

const __half* norm_after(const npu_b200_ctx* c, int l) {
  const Plan& P = c->plan;
  return l + 1 < P.layers ? c->layers[l + 1].in_norm
                          : (c->final_norm ? c->final_norm : c->layers[l].in_norm);
}

// The greedy-id tail of a token step: reduce the LM head's partial argmaxes
// (and across ranks).
int finish_argmax(npu_b200_ctx* c, int batch, cudaStream_t s) {
  const Plan& P = c->plan;
  const int rows = part_rows(batch);
  const int lm_tiles = (c->vocab_loc + rows - 1) / rows;
  int rc = 0;
  if (c->tp_size == 1)
    return argmax_reduce(c->am_val, c->am_idx, lm_tiles, P.max_batch, batch, c->vocab_off,
                         c->gather_send, c->d_ids, s, true);
  if (c->px_ready) {
    PeerExchange x = c->px;
    x.seq = kArgmaxSeq;
    if ((rc = argmax_reduce_publish(c->am_val, c->am_idx, lm_tiles, P.max_batch, batch,
                                 c->vocab_off, x, s, true)))
      return rc;
    return argmax_combine_peers(x, batch, c->d_ids, s, true);
  }
  if ((rc = argmax_reduce(c->am_val, c->am_idx, lm_tiles, P.max_batch, batch, c->vocab_off,
                          c->gather_send, reinterpret_cast<int32_t*>(c->gather_send + P.max_batch),
                          s, true)))
    return rc;
  if ((rc = check_nccl(g_nccl.AllGather(c->gather_send, c->gather_recv, 2 * P.max_batch,
                                        ncclFloat32, c->comm, s),
                       "ncclAllGather")))
    return rc;
  return argmax_combine(c->gather_recv, c->tp_size, P.max_batch, batch, c->d_ids, s, false);
}

int enqueue_step(npu_b200_ctx* c, int mode, int batch, cudaStream_t s) {
  const Plan& P = c->plan;
  const int H = P.hidden, D = P.head_dim;
  int rc = 0;
  {
    ResidualUpdate u;
    u.mode = mode == kModeTokens ? kResidFromEmbedding : kResidFromHidden;
    u.batch = batch;
    u.hidden = H;
    u.vocab = P.vocab;
    u.tokens = c->d_tokens;
    u.embed = c->embed;
    u.hidden_in = c->hidden_io;
    u.resid = c->resid;
    u.norm_w = c->layers[0].in_norm;
    u.xw = c->xw;
    u.ssq_out = c->ssq;
    u.ssq_ld = P.max_batch;
    u.ssq_rows = part_rows(batch);
    u.positions = c->d_positions;
    u.seq_lens = c->d_seq_lens;
    u.inv_freq = c->d_inv_freq;
    u.rope_tab = c->rope_tab;
    u.epoch = c->epoch;
    if ((rc = residual_update(u, s, true))) return rc;
  }
  for (int l = 0; l < P.layers; ++l) {
    LayerBuffers& L = c->layers[l];
    const EpiParams q = qkv_epi(c, l, batch);
    if ((rc = proj_run(L.w_qkv, true, c->xw, q.n_rows, H, batch, q, c->proj_ws, c->proj_ws_bytes, s,
                       true)))
      return rc;
    if ((rc = flash_decode_run(c->q_buf, L.k_cache, L.v_cache, c->d_seq_lens, c->attn, batch,
                               c->q_loc, c->kv_loc, D, P.max_seq, 1.f / sqrtf(static_cast<float>(D)),
                               0, c->fd_ws, c->fd_ws_bytes, s, true, c->d_positions)))
      return rc;
    if ((rc = residual_out(c, L.w_o, c->attn, c->q_loc * D, batch, L.post_norm, 2 * l, s)))
      return rc;
    const EpiParams g = swiglu_epi(c, batch);
    if ((rc = proj_run(L.w_gu, true, c->xw, g.n_rows, H, batch, g, c->proj_ws, c->proj_ws_bytes, s,
                       true)))
      return rc;
    if ((rc = residual_out(c, L.w_down, c->act, c->ffn_loc, batch, norm_after(c, l), 2 * l + 1, s)))
      return rc;
  }
  if (mode == kModeHidden)
    return store_hidden(c->resid, c->hidden_io, static_cast<size_t>(batch) * H, s, true);
  const EpiParams a = argmax_epi(c, batch);
  if ((rc = proj_run(c->lm_head, true, c->xw, c->vocab_loc, H, batch, a, c->proj_ws, c->proj_ws_bytes,
                     s, true)))
    return rc;
  return finish_argmax(c, batch, s);
}

int graph_for(npu_b200_ctx* c, int mode, int batch, cudaGraphExec_t* out) {
  auto it = c->graphs.find({mode, batch});
  if (it != c->graphs.end()) {
    *out = it->second;
    return NPU_B200_OK;
  }
  std::string missing;
  if (required_missing(c, mode == kModeTokens, &missing))
    return set_error(NPU_B200_E_STATE, "weight '%s' was never set", missing.c_str());
  NPU_TRY_CUDA(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeRelaxed));
  const int rc = enqueue_step(c, mode, batch, c->stream);
  cudaGraph_t graph = nullptr;
  const cudaError_t end = cudaStreamEndCapture(c->stream, &graph);
  if (rc) {
    if (graph) cudaGraphDestroy(graph);
    return rc;
  }
  NPU_TRY_CUDA(end);
  cudaGraphExec_t exec = nullptr;
  const cudaError_t inst = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  NPU_TRY_CUDA(inst);
  c->graphs[{mode, batch}] = exec;
  *out = exec;
  return NPU_B200_OK;
}

int check_ready(npu_b200_ctx* c, int batch, bool tokens_mode) {
  NPU_REQUIRE(c != nullptr, "null context");
  if (!c->loaded) return set_error(NPU_B200_E_STATE, "no plan loaded");
  NPU_REQUIRE(batch >= 1 && batch <= c->plan.max_batch, "batch %d not in [1, %d]", batch,
              c->plan.max_batch);
  if (tokens_mode && c->plan.vocab == 0)
    return set_error(NPU_B200_E_STATE, "plan has no vocabulary: use the hidden-state entry points");
  NPU_TRY_CUDA(cudaSetDevice(c->device));
  return NPU_B200_OK;
}

int check_positions(const npu_b200_ctx* c, const int32_t* h_positions, int batch) {
  for (int b = 0; b < batch; ++b)
    NPU_REQUIRE(h_positions[b] >= 0 && h_positions[b] < c->plan.max_seq,
                "position %d of sequence %d is outside the cache [0, %d)", h_positions[b], b,
                c->plan.max_seq);
  return NPU_B200_OK;
}

}  // namespace
}  // namespace npu_b200

namespace npu_b200 {
int ctx_device(const npu_b200_ctx* c) { return c->device; }
GraphState*& ctx_graph(npu_b200_ctx* c) { return c->graph; }
}  // namespace npu_b200

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" int npu_b200_nccl_unique_id(void* out128) {
  clear_error();
  NPU_REQUIRE(out128, "null output");
  int rc = load_nccl();
  if (rc) return rc;
  ncclUniqueId id;
  if ((rc = check_nccl(g_nccl.GetUniqueId(&id), "ncclGetUniqueId"))) return rc;
  memcpy(out128, id.internal, sizeof(id.internal));
  return NPU_B200_OK;
}

extern "C" int npu_b200_create(int device, int tp_rank, int tp_size, const void* nccl_unique_id,
                               npu_b200_ctx** out) {
  clear_error();
  NPU_REQUIRE(out, "null output");
  *out = nullptr;
  NPU_REQUIRE(tp_size >= 1 && tp_rank >= 0 && tp_rank < tp_size, "bad tp rank %d / size %d",
              tp_rank, tp_size);
  NPU_REQUIRE(tp_size == 1 || nccl_unique_id, "tp_size > 1 needs an NCCL unique id");
  int rc = 0;
  if (tp_size > 1 && (rc = load_nccl())) return rc;
  NPU_TRY_CUDA(cudaSetDevice(device));
  npu_b200_ctx* c = new npu_b200_ctx();
  c->device = device;
  c->tp_rank = tp_rank;
  c->tp_size = tp_size;
  if ((rc = check_cuda(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking),
                       "cudaStreamCreate"))) {
    delete c;
    return rc;
  }
  if (tp_size > 1) {
    ncclUniqueId id;
    memcpy(id.internal, nccl_unique_id, sizeof(id.internal));
    if ((rc = check_nccl(g_nccl.CommInitRank(&c->comm, tp_size, id, tp_rank), "ncclCommInitRank"))) {
      cudaStreamDestroy(c->stream);
      delete c;
      return rc;
    }
  }
  *out = c;
  return NPU_B200_OK;
}

extern "C" int npu_b200_load_plan(npu_b200_ctx* c, const char* plan_path) {
  clear_error();
  NPU_REQUIRE(c && plan_path, "null argument");
  std::ifstream f(plan_path);
  if (!f) return set_error(NPU_B200_E_PLAN, "cannot read plan %s", plan_path);
  std::stringstream ss;
  ss << f.rdbuf();
  Plan p;
  int rc = parse_plan(ss.str(), &p);
  if (rc) return rc;
  NPU_TRY_CUDA(cudaSetDevice(c->device));
  NPU_TRY_CUDA(cudaDeviceSynchronize());
  release(c);
  c->plan = p;
  if ((rc = allocate(c))) {
    release(c);
    return rc;
  }
  c->loaded = true;
  return NPU_B200_OK;
}

extern "C" int npu_b200_plan_check(const char* plan_path, int64_t* out, int n) {
  clear_error();
  NPU_REQUIRE(plan_path && out && n >= 12, "plan_check needs a path and 12 slots");
  std::ifstream f(plan_path);
  if (!f) return set_error(NPU_B200_E_PLAN, "cannot read plan %s", plan_path);
  std::stringstream ss;
  ss << f.rdbuf();
  Plan p;
  const int rc = parse_plan(ss.str(), &p);
  if (rc) return rc;
  const int64_t v[12] = {p.layers, p.hidden, p.heads, p.kv_heads, p.ffn, p.vocab, 0, p.max_batch,
                         p.max_seq, p.head_dim,
                         static_cast<int64_t>(p.fingerprint & 0x7fffffffffffffffll), 1};
  for (int i = 0; i < 12; ++i) out[i] = v[i];
  return NPU_B200_OK;
}

extern "C" int npu_b200_shard_info(const char* plan_path, int tp_rank, int tp_size, int64_t* out,
                                   int n) {
  clear_error();
  NPU_REQUIRE(plan_path && out && n >= 5, "shard_info needs a path and 5 slots");
  std::ifstream f(plan_path);
  if (!f) return set_error(NPU_B200_E_PLAN, "cannot read plan %s", plan_path);
  std::stringstream ss;
  ss << f.rdbuf();
  Plan p;
  int rc = parse_plan(ss.str(), &p);
  if (rc) return rc;
  Shard sh;
  if ((rc = shard_layout(p, tp_size, tp_rank, &sh))) return rc;
  const int64_t v[5] = {sh.q_loc, sh.kv_loc, sh.ffn_loc, sh.vocab_loc, sh.vocab_off};
  for (int i = 0; i < 5; ++i) out[i] = v[i];
  return NPU_B200_OK;
}

extern "C" int npu_b200_plan_info(const npu_b200_ctx* c, int64_t* out, int n) {
  clear_error();
  NPU_REQUIRE(c && out && n >= 12, "plan_info needs a context and 12 slots");
  if (!c->loaded) return set_error(NPU_B200_E_STATE, "no plan loaded");
  const int64_t v[13] = {c->plan.layers, c->plan.hidden, c->q_loc, c->kv_loc, c->ffn_loc,
                         c->vocab_loc, c->vocab_off, c->plan.max_batch, c->plan.max_seq,
                         c->plan.head_dim, static_cast<int64_t>(c->plan.fingerprint & 0x7fffffffffffffffll),
                         c->tp_size, c->px_ready ? 1 : 0};
  for (int i = 0; i < (n < 13 ? n : 13); ++i) out[i] = v[i];
  return NPU_B200_OK;
}

extern "C" int npu_b200_set_weight(npu_b200_ctx* c, const char* name, const void* src,
                                   size_t bytes) {
  clear_error();
  NPU_REQUIRE(c && name && src, "null argument");
  if (!c->loaded) return set_error(NPU_B200_E_STATE, "no plan loaded");
  NPU_TRY_CUDA(cudaSetDevice(c->device));
  int layer = -1, kind = -1;
  int rc = resolve_name(c, name, &layer, &kind);
  if (rc) return rc;
  return place_weight(c, layer, kind, src, bytes);
}

extern "C" int npu_b200_load_capture(npu_b200_ctx* c, const char* dir) {
  clear_error();
  NPU_REQUIRE(c && dir, "null argument");
  if (!c->loaded) return set_error(NPU_B200_E_STATE, "no plan loaded");
  const std::string root(dir);
  std::ifstream args(root + "/arguments.txt");
  if (!args) return set_error(NPU_B200_E_PLAN, "cannot read %s/arguments.txt", dir);
  std::string line;
  int used = 0;
  while (std::getline(args, line)) {
    std::istringstream ls(line);
    int index = -1;
    std::string name, shape, dtype;
    if (!(ls >> index >> name >> shape >> dtype)) continue;
    int layer = -1, kind = -1;
    if (resolve_name(c, name, &layer, &kind) != NPU_B200_OK) {
      clear_error();
      continue;  // activations, RoPE tables, masks: not weights of this plan
    }
    NPU_REQUIRE(dtype == "float16", "capture argument %s is %s, expected float16", name.c_str(),
                dtype.c_str());
    const std::string path = root + "/arg" + std::to_string(index) + ".bin";
    std::ifstream bin(path, std::ios::binary | std::ios::ate);
    if (!bin) return set_error(NPU_B200_E_PLAN, "cannot read %s", path.c_str());
    const size_t bytes = static_cast<size_t>(bin.tellg());
    bin.seekg(0);
    std::vector<char> data(bytes);
    if (!bin.read(data.data(), static_cast<std::streamsize>(bytes)))
      return set_error(NPU_B200_E_PLAN, "short read of %s", path.c_str());
    int rc = npu_b200_set_weight(c, name.c_str(), data.data(), bytes);
    if (rc) return rc;
    ++used;
  }
  if (used == 0) return set_error(NPU_B200_E_PLAN, "%s names no weight of this plan", dir);
  return NPU_B200_OK;
}

// ---------------------------------------------------------------------------
// Per-rank weight image: this rank's packed panels and norms, saved as files
// with a descriptor and read back without sharding or packing -- the B200
// counterpart of the reference's hbm.bin image (tools/npu-compile/
// npu-compile.cpp:495-659), whose stage stamps it keeps (stage, schema, the
// plan fingerprint).
// ---------------------------------------------------------------------------
namespace npu_b200 {
namespace {

struct ImageEntry {
  std::string name;
  void* ptr = nullptr;
  size_t bytes = 0;
  std::vector<size_t> have;  // indices of c->have this tensor completes
};

std::vector<ImageEntry> image_entries(const npu_b200_ctx* c) {
  const Plan& P = c->plan;
  const int H = P.hidden, D = P.head_dim;
  std::vector<ImageEntry> e;
  for (int l = 0; l < P.layers; ++l) {
    const LayerBuffers& L = c->layers[l];
    const size_t base = static_cast<size_t>(l) * kPerLayerKinds;
    const std::string pre = "layers." + std::to_string(l) + ".";
    e.push_back({pre + "qkv", L.w_qkv, packed_weight_bytes((c->q_loc + 2 * c->kv_loc) * D, H),
                 {base + kQ, base + kK, base + kV}});
    e.push_back({pre + "o", L.w_o, packed_weight_bytes(H, c->q_loc * D), {base + kO}});
    e.push_back({pre + "gate_up", L.w_gu, packed_weight_bytes(2 * c->ffn_loc, H),
                 {base + kGate, base + kUp}});
    e.push_back({pre + "down", L.w_down, packed_weight_bytes(H, c->ffn_loc), {base + kDown}});
    e.push_back({pre + "input_layernorm", L.in_norm, static_cast<size_t>(H) * 2, {base + kInNorm}});
    e.push_back({pre + "post_attention_layernorm", L.post_norm, static_cast<size_t>(H) * 2,
                 {base + kPostNorm}});
    if (P.qk_norm) {
      e.push_back({pre + "q_norm", L.q_norm, static_cast<size_t>(D) * 2, {base + kQNorm}});
      e.push_back({pre + "k_norm", L.k_norm, static_cast<size_t>(D) * 2, {base + kKNorm}});
    }
  }
  if (P.vocab > 0) {
    const size_t top = static_cast<size_t>(P.layers) * kPerLayerKinds;
    e.push_back({"embed", c->embed, static_cast<size_t>(P.vocab) * H * 2, {top + 0}});
    e.push_back({"final_norm", c->final_norm, static_cast<size_t>(H) * 2, {top + 1}});
    e.push_back({"lm_head", c->lm_head, packed_weight_bytes(c->vocab_loc, H), {top + 2}});
  }
  return e;
}

uint64_t fnv1a_bytes(const uint8_t* p, size_t n) {
  uint64_t h = 1469598103934665603ull;
  for (size_t i = 0; i < n; ++i) h = (h ^ p[i]) * 1099511628211ull;
  return h;
}

std::string rank_dir(const npu_b200_ctx* c, const char* dir) {
  return std::string(dir) + "/rank" + std::to_string(c->tp_rank) + "-of-" +
         std::to_string(c->tp_size);
}

}  // namespace
}  // namespace npu_b200

extern "C" int npu_b200_save_image(npu_b200_ctx* c, const char* dir) {
  clear_error();
  NPU_REQUIRE(c && dir, "null argument");
  if (!c->loaded) return set_error(NPU_B200_E_STATE, "no plan loaded");
  std::string missing;
  if (required_missing(c, c->plan.vocab > 0, &missing))
    return set_error(NPU_B200_E_STATE, "image: weight %s was never set", missing.c_str());
  NPU_TRY_CUDA(cudaSetDevice(c->device));
  NPU_TRY_CUDA(cudaDeviceSynchronize());
  const std::string root = rank_dir(c, dir);
  std::error_code ec;
  std::filesystem::create_directories(root, ec);
  if (ec) return set_error(NPU_B200_E_INVALID, "image: cannot create %s", root.c_str());
  std::ostringstream desc;
  desc << "stage = cuda-image\nschema = 1\nfingerprint = " << c->plan.fingerprint
       << "\ntp_rank = " << c->tp_rank << "\ntp_size = " << c->tp_size << "\n";
  std::vector<uint8_t> host;
  for (const ImageEntry& t : image_entries(c)) {
    host.resize(t.bytes);
    NPU_TRY_CUDA(cudaMemcpy(host.data(), t.ptr, t.bytes, cudaMemcpyDeviceToHost));
    const std::string file = t.name + ".bin";
    std::ofstream out(root + "/" + file, std::ios::binary | std::ios::trunc);
    out.write(reinterpret_cast<const char*>(host.data()), static_cast<std::streamsize>(t.bytes));
    if (!out) return set_error(NPU_B200_E_INVALID, "image: cannot write %s/%s", root.c_str(), file.c_str());
    char sum[32];
    snprintf(sum, sizeof(sum), "%016llx", static_cast<unsigned long long>(fnv1a_bytes(host.data(), t.bytes)));
    desc << "tensor " << t.name << " " << t.bytes << " " << sum << " " << file << "\n";
  }
  std::ofstream d(root + "/image.txt", std::ios::trunc);
  d << desc.str();
  if (!d) return set_error(NPU_B200_E_INVALID, "image: cannot write %s/image.txt", root.c_str());
  return NPU_B200_OK;
}

extern "C" int npu_b200_load_image(npu_b200_ctx* c, const char* dir) {
  clear_error();
  NPU_REQUIRE(c && dir, "null argument");
  if (!c->loaded) return set_error(NPU_B200_E_STATE, "no plan loaded");
  NPU_TRY_CUDA(cudaSetDevice(c->device));
  const std::string root = rank_dir(c, dir);
  std::ifstream in(root + "/image.txt");
  if (!in) return set_error(NPU_B200_E_PLAN, "image: cannot read %s/image.txt", root.c_str());
  std::map<std::string, std::string> keys;
  std::map<std::string, std::vector<std::string>> tensors;
  std::string line;
  while (std::getline(in, line)) {
    std::istringstream ls(line);
    std::string first;
    if (!(ls >> first)) continue;
    if (first == "tensor") {
      std::string name, bytes, sum, file;
      if (!(ls >> name >> bytes >> sum >> file))
        return set_error(NPU_B200_E_PLAN, "image: malformed line '%s'", line.c_str());
      if (tensors.count(name)) return set_error(NPU_B200_E_PLAN, "image: duplicate tensor %s", name.c_str());
      tensors[name] = {bytes, sum, file};
    } else {
      std::string eq, value;
      if (!(ls >> eq >> value) || eq != "=")
        return set_error(NPU_B200_E_PLAN, "image: malformed line '%s'", line.c_str());
      keys[first] = value;
    }
  }
  if (keys["stage"] != "cuda-image" || keys["schema"] != "1")
    return set_error(NPU_B200_E_PLAN, "image: stage '%s' schema '%s', expected cuda-image 1",
                     keys["stage"].c_str(), keys["schema"].c_str());
  if (keys["fingerprint"] != std::to_string(c->plan.fingerprint))
    return set_error(NPU_B200_E_PLAN, "image: made for another plan (fingerprint %s, plan %llu)",
                     keys["fingerprint"].c_str(), static_cast<unsigned long long>(c->plan.fingerprint));
  if (keys["tp_rank"] != std::to_string(c->tp_rank) || keys["tp_size"] != std::to_string(c->tp_size))
    return set_error(NPU_B200_E_PLAN, "image: made for rank %s of %s", keys["tp_rank"].c_str(),
                     keys["tp_size"].c_str());
  const std::vector<ImageEntry> want = image_entries(c);
  if (tensors.size() != want.size())
    return set_error(NPU_B200_E_PLAN, "image: %zu tensors, the plan needs %zu", tensors.size(),
                     want.size());
  std::vector<uint8_t> host;
  for (const ImageEntry& t : want) {
    auto it = tensors.find(t.name);
    if (it == tensors.end()) return set_error(NPU_B200_E_PLAN, "image: no tensor %s", t.name.c_str());
    const std::vector<std::string>& f = it->second;
    if (f[0] != std::to_string(t.bytes))
      return set_error(NPU_B200_E_PLAN, "image: %s has %s bytes, the plan needs %zu", t.name.c_str(),
                       f[0].c_str(), t.bytes);
    if (f[2].find('/') != std::string::npos || f[2].find("..") != std::string::npos)
      return set_error(NPU_B200_E_PLAN, "image: file name '%s' leaves the image", f[2].c_str());
    std::ifstream bin(root + "/" + f[2], std::ios::binary | std::ios::ate);
    if (!bin || static_cast<size_t>(bin.tellg()) != t.bytes)
      return set_error(NPU_B200_E_PLAN, "image: %s/%s is missing or not %zu bytes", root.c_str(),
                       f[2].c_str(), t.bytes);
    bin.seekg(0);
    host.resize(t.bytes);
    if (!bin.read(reinterpret_cast<char*>(host.data()), static_cast<std::streamsize>(t.bytes)))
      return set_error(NPU_B200_E_PLAN, "image: short read of %s", f[2].c_str());
    char sum[32];
    snprintf(sum, sizeof(sum), "%016llx", static_cast<unsigned long long>(fnv1a_bytes(host.data(), t.bytes)));
    if (f[1] != sum)
      return set_error(NPU_B200_E_PLAN, "image: %s checksum %s, the descriptor says %s",
                       t.name.c_str(), sum, f[1].c_str());
    NPU_TRY_CUDA(cudaMemcpy(t.ptr, host.data(), t.bytes, cudaMemcpyHostToDevice));
    for (size_t h : t.have) c->have[h] = 1;
  }
  return NPU_B200_OK;
}

extern "C" int npu_b200_kv_cache(npu_b200_ctx* c, int layer, void** d_k, void** d_v) {
  clear_error();
  NPU_REQUIRE(c && d_k && d_v, "null argument");
  if (!c->loaded) return set_error(NPU_B200_E_STATE, "no plan loaded");
  NPU_REQUIRE(layer >= 0 && layer < c->plan.layers, "layer %d out of range", layer);
  *d_k = c->layers[layer].k_cache;
  *d_v = c->layers[layer].v_cache;
  return NPU_B200_OK;
}

extern "C" int npu_b200_decode_step_device(npu_b200_ctx* c, const int32_t* d_tokens,
                                           const int32_t* d_positions, int batch,
                                           int32_t* d_out_ids, void* stream) {
  clear_error();
  int rc = check_ready(c, batch, true);
  if (rc) return rc;
  NPU_REQUIRE(d_tokens && d_positions && d_out_ids, "null argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaGraphExec_t g = nullptr;
  if ((rc = graph_for(c, kModeTokens, batch, &g))) return rc;
  NPU_TRY_CUDA(cudaMemcpyAsync(c->d_tokens, d_tokens, batch * 4, cudaMemcpyDeviceToDevice, s));
  NPU_TRY_CUDA(cudaMemcpyAsync(c->d_positions, d_positions, batch * 4, cudaMemcpyDeviceToDevice, s));
  NPU_TRY_CUDA(cudaGraphLaunch(g, s));
  NPU_TRY_CUDA(cudaMemcpyAsync(d_out_ids, c->d_ids, batch * 4, cudaMemcpyDeviceToDevice, s));
  return NPU_B200_OK;
}

extern "C" int npu_b200_decode_step(npu_b200_ctx* c, const int32_t* h_tokens,
                                    const int32_t* h_positions, int batch, int32_t* h_out_ids,
                                    void* stream) {
  clear_error();
  int rc = check_ready(c, batch, true);
  if (rc) return rc;
  NPU_REQUIRE(h_tokens && h_positions && h_out_ids, "null argument");
  if ((rc = check_positions(c, h_positions, batch))) return rc;
  for (int b = 0; b < batch; ++b)
    NPU_REQUIRE(h_tokens[b] >= 0 && h_tokens[b] < c->plan.vocab, "token %d of sequence %d",
                h_tokens[b], b);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaGraphExec_t g = nullptr;
  if ((rc = graph_for(c, kModeTokens, batch, &g))) return rc;
  memcpy(c->h_tokens, h_tokens, batch * 4);
  memcpy(c->h_positions, h_positions, batch * 4);
  NPU_TRY_CUDA(cudaMemcpyAsync(c->d_tokens, c->h_tokens, batch * 4, cudaMemcpyHostToDevice, s));
  NPU_TRY_CUDA(cudaMemcpyAsync(c->d_positions, c->h_positions, batch * 4, cudaMemcpyHostToDevice, s));
  NPU_TRY_CUDA(cudaGraphLaunch(g, s));
  NPU_TRY_CUDA(cudaMemcpyAsync(c->h_ids, c->d_ids, batch * 4, cudaMemcpyDeviceToHost, s));
  NPU_TRY_CUDA(cudaStreamSynchronize(s));
  memcpy(h_out_ids, c->h_ids, batch * 4);
  return NPU_B200_OK;
}

extern "C" int npu_b200_forward_hidden_device(npu_b200_ctx* c, const void* d_x,
                                              const int32_t* d_positions, int batch, void* d_y,
                                              void* stream) {
  clear_error();
  int rc = check_ready(c, batch, false);
  if (rc) return rc;
  NPU_REQUIRE(d_x && d_positions && d_y, "null argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaGraphExec_t g = nullptr;
  if ((rc = graph_for(c, kModeHidden, batch, &g))) return rc;
  const size_t bytes = static_cast<size_t>(batch) * c->plan.hidden * 2;
  NPU_TRY_CUDA(cudaMemcpyAsync(c->hidden_io, d_x, bytes, cudaMemcpyDeviceToDevice, s));
  NPU_TRY_CUDA(cudaMemcpyAsync(c->d_positions, d_positions, batch * 4, cudaMemcpyDeviceToDevice, s));
  NPU_TRY_CUDA(cudaGraphLaunch(g, s));
  NPU_TRY_CUDA(cudaMemcpyAsync(d_y, c->hidden_io, bytes, cudaMemcpyDeviceToDevice, s));
  return NPU_B200_OK;
}

extern "C" int npu_b200_forward_hidden(npu_b200_ctx* c, const void* h_x,
                                       const int32_t* h_positions, int batch, void* h_y,
                                       void* stream) {
  clear_error();
  int rc = check_ready(c, batch, false);
  if (rc) return rc;
  NPU_REQUIRE(h_x && h_positions && h_y, "null argument");
  if ((rc = check_positions(c, h_positions, batch))) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaGraphExec_t g = nullptr;
  if ((rc = graph_for(c, kModeHidden, batch, &g))) return rc;
  const size_t bytes = static_cast<size_t>(batch) * c->plan.hidden * 2;
  memcpy(c->h_hidden, h_x, bytes);
  memcpy(c->h_positions, h_positions, batch * 4);
  NPU_TRY_CUDA(cudaMemcpyAsync(c->hidden_io, c->h_hidden, bytes, cudaMemcpyHostToDevice, s));
  NPU_TRY_CUDA(cudaMemcpyAsync(c->d_positions, c->h_positions, batch * 4, cudaMemcpyHostToDevice, s));
  NPU_TRY_CUDA(cudaGraphLaunch(g, s));
  NPU_TRY_CUDA(cudaMemcpyAsync(c->h_hidden, c->hidden_io, bytes, cudaMemcpyDeviceToHost, s));
  NPU_TRY_CUDA(cudaStreamSynchronize(s));
  memcpy(h_y, c->h_hidden, bytes);
  return NPU_B200_OK;
}

extern "C" int npu_b200_destroy(npu_b200_ctx* c) {
  clear_error();
  if (!c) return NPU_B200_OK;
  cudaSetDevice(c->device);
  cudaDeviceSynchronize();
  release(c);
  graph_free(c->graph);
  c->graph = nullptr;
  if (c->comm && g_nccl.CommDestroy) g_nccl.CommDestroy(c->comm);
  if (c->stream) cudaStreamDestroy(c->stream);
  delete c;
  return NPU_B200_OK;
}
