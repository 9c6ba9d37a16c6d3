// Graph plans: npu_b200_load_graph / npu_b200_run_graph.
//
// The reference compiles a captured module into a program for its simulator
// and runs it with the captured arguments (tools/npu-compile/npu-compile.cpp;
// python/npu/capture/export.py:108-139).  The B200 target executes a graph
// plan instead: a capture directory (arguments.txt, arg<N>.bin) plus graph.txt,
// written by llm_compiler_3_b200/graph.py from a torch.export of the module.
// Each op runs one of this library's kernels:
//
//   op linear y x w bias relu   the tcgen05 linear kernel (proj.cu), rows of x
//                               in launches of at most 128 (FP16 operands, FP32
//                               accumulation, bias and ReLU in the epilogue)
//   op sdpa o q k v scale causal
//                               npu.attention: flash-decoding (one query per
//                               head, no causal mask) or the prefill attention
//                               kernel (every other case)
//
// Tensors are inputs (the run call's argument pointers, in line order),
// outputs (its output pointers), parameters (loaded once from arg<N>.bin),
// temporaries (allocated once) and aliases (another tensor's bytes under other
// dimensions).  Everything is checked when the plan is read, on the host, so a
// bad plan fails at load with a message, never in a kernel.
#include <math.h>
#include <stdio.h>
#include <sys/stat.h>

#include <algorithm>
#include <fstream>
#include <map>
#include <sstream>
#include <string>
#include <vector>

#include "host.hpp"

namespace npu_b200 {

enum GraphRole { kRoleInput = 0, kRoleOutput = 1, kRoleParam = 2, kRoleTemp = 3, kRoleAlias = 4 };
enum GraphOpKind { kOpLinear = 0, kOpSdpa = 1 };

struct GraphTensor {
  std::string name;
  int role = kRoleTemp;
  std::vector<int64_t> dims;
  int64_t numel = 0;
  int arg = -1;   // parameter: arg<N>.bin
  int io = -1;    // input / output: index in the run call's pointer array
  int base = -1;  // alias: the tensor whose bytes it views
  void* dev = nullptr;
};

struct GraphOp {
  int kind = kOpLinear;
  int out = -1, a = -1, b = -1, c = -1, bias = -1;  // linear: x=a, w=b; sdpa: q=a, k=b, v=c
  int relu = 0, causal = 0;
  float scale = 0.f;
  int64_t rows = 0;
  int n = 0, k = 0;
  int batch = 0, heads = 0, kv_heads = 0, queries = 0, keys = 0, dim = 0;
  bool decode = false;
  int32_t* seq_lens = nullptr;  // flash-decoding: `keys` for every sequence
};

struct GraphState {
  std::string dir;
  std::vector<GraphTensor> t;
  std::map<std::string, int> index;
  std::vector<GraphOp> ops;
  std::vector<int> inputs, outputs;
  std::vector<void*> allocs;
  void* lin_ws = nullptr;
  size_t lin_ws_bytes = 0;
  void* fd_ws = nullptr;
  size_t fd_ws_bytes = 0;
  int64_t param_bytes = 0, temp_bytes = 0;
};

// Kernel limits mirrored at load time (proj.cu, prefill_attention.cu).
constexpr long long kLinearMaxTiles = 16384;
void prefill_blocking(int queries, int group, int* bm, int* hp);

namespace {

int plan_error(const std::string& dir, int line, const char* what) {
  return set_error(NPU_B200_E_PLAN, "%s/graph.txt:%d: %s", dir.c_str(), line, what);
}

bool parse_dims(const std::string& text, std::vector<int64_t>* dims, int64_t* numel) {
  dims->clear();
  std::stringstream ss(text);
  std::string part;
  int64_t n = 1;
  while (std::getline(ss, part, 'x')) {
    char* end = nullptr;
    const long long d = strtoll(part.c_str(), &end, 10);
    // Every dimension must fit the int arguments of the kernels' entry points.
    if (part.empty() || *end != '\0' || d <= 0 || d >= (1ll << 31)) return false;
    dims->push_back(d);
    n *= d;
    if (n > (1ll << 40)) return false;
  }
  *numel = n;
  return !dims->empty();
}

int64_t file_size(const std::string& path) {
  struct stat st;
  return stat(path.c_str(), &st) == 0 ? static_cast<int64_t>(st.st_size) : -1;
}

// Operand `name` of line `line`: must exist and, unless it is an input or a
// parameter, have been written by an earlier op.
int operand(GraphState* g, const std::vector<bool>& written, const std::string& name, int line,
            int* out) {
  auto it = g->index.find(name);
  if (it == g->index.end()) {
    std::string m = "unknown tensor " + name;
    return plan_error(g->dir, line, m.c_str());
  }
  const int i = it->second;
  const int base = g->t[i].role == kRoleAlias ? g->t[i].base : i;
  const int role = g->t[base].role;
  if ((role == kRoleTemp || role == kRoleOutput) && !written[base]) {
    std::string m = name + " is read before an op writes it";
    return plan_error(g->dir, line, m.c_str());
  }
  *out = i;
  return NPU_B200_OK;
}

int result(GraphState* g, std::vector<bool>* written, const std::string& name, int line, int* out) {
  auto it = g->index.find(name);
  if (it == g->index.end()) {
    std::string m = "unknown tensor " + name;
    return plan_error(g->dir, line, m.c_str());
  }
  const int i = it->second;
  if (g->t[i].role != kRoleTemp && g->t[i].role != kRoleOutput) {
    std::string m = name + ": an op may only write a temporary or an output";
    return plan_error(g->dir, line, m.c_str());
  }
  if ((*written)[i]) {
    std::string m = name + " is written twice";
    return plan_error(g->dir, line, m.c_str());
  }
  (*written)[i] = true;
  *out = i;
  return NPU_B200_OK;
}

int parse_graph(const std::string& dir, GraphState* g) {
  g->dir = dir;
  std::ifstream f(dir + "/graph.txt");
  if (!f) return set_error(NPU_B200_E_PLAN, "cannot read %s/graph.txt", dir.c_str());
  std::string raw;
  int line = 0;
  bool stage = false, schema = false;
  std::vector<bool> written;
  while (std::getline(f, raw)) {
    ++line;
    std::istringstream ls(raw);
    std::string kw;
    if (!(ls >> kw) || kw[0] == '#') continue;
    if (kw == "npu.stage") {
      std::string v;
      ls >> v;
      if (v != "cuda-graph") return plan_error(dir, line, "stage is not cuda-graph");
      stage = true;
    } else if (kw == "npu.schema") {
      int v = 0;
      ls >> v;
      if (v != 1) return plan_error(dir, line, "unsupported schema (this library reads 1)");
      schema = true;
    } else if (kw == "tensor" || kw == "alias") {
      if (!g->ops.empty()) return plan_error(dir, line, "tensors must precede the ops");
      GraphTensor t;
      std::string role_or_src, dtype, dims, argkw;
      if (kw == "tensor") {
        if (!(ls >> t.name >> role_or_src >> dtype >> dims))
          return plan_error(dir, line, "expected: tensor <name> <role> f16 <dims> [arg <N>]");
        static const std::map<std::string, int> roles = {
            {"input", kRoleInput}, {"output", kRoleOutput}, {"param", kRoleParam}, {"temp", kRoleTemp}};
        auto r = roles.find(role_or_src);
        if (r == roles.end()) return plan_error(dir, line, "role must be input, output, param or temp");
        t.role = r->second;
        if (dtype != "f16") return plan_error(dir, line, "graph tensors are f16");
        if (t.role == kRoleParam) {
          if (!(ls >> argkw >> t.arg) || argkw != "arg" || t.arg < 0)
            return plan_error(dir, line, "a parameter names its file: arg <N>");
        }
      } else {
        if (!(ls >> t.name >> role_or_src >> dims))
          return plan_error(dir, line, "expected: alias <name> <source> <dims>");
        t.role = kRoleAlias;
        auto src = g->index.find(role_or_src);
        if (src == g->index.end() || g->t[src->second].role == kRoleAlias)
          return plan_error(dir, line, "an alias views a tensor declared before it (not an alias)");
        t.base = src->second;
      }
      if (!parse_dims(dims, &t.dims, &t.numel)) return plan_error(dir, line, "bad dimensions");
      if (g->index.count(t.name)) return plan_error(dir, line, "tensor declared twice");
      if (t.role == kRoleAlias && t.numel != g->t[t.base].numel)
        return plan_error(dir, line, "an alias must have its source's element count");
      if (t.role == kRoleParam) {
        const std::string path = dir + "/arg" + std::to_string(t.arg) + ".bin";
        if (file_size(path) != t.numel * 2) {
          std::string m = path + " is missing or not " + std::to_string(t.numel * 2) + " bytes";
          return plan_error(dir, line, m.c_str());
        }
        g->param_bytes += t.numel * 2;
      }
      if (t.role == kRoleTemp) g->temp_bytes += t.numel * 2;
      if (t.role == kRoleInput) {
        t.io = static_cast<int>(g->inputs.size());
        g->inputs.push_back(static_cast<int>(g->t.size()));
      }
      if (t.role == kRoleOutput) {
        t.io = static_cast<int>(g->outputs.size());
        g->outputs.push_back(static_cast<int>(g->t.size()));
      }
      g->index[t.name] = static_cast<int>(g->t.size());
      g->t.push_back(t);
      written.push_back(false);
    } else if (kw == "op") {
      std::string kind;
      ls >> kind;
      GraphOp op;
      int rc = 0;
      if (kind == "linear") {
        std::string y, x, w, b;
        int relu = -1;
        if (!(ls >> y >> x >> w >> b >> relu) || (relu != 0 && relu != 1))
          return plan_error(dir, line, "expected: op linear <y> <x> <w> <bias|-> <relu 0|1>");
        op.kind = kOpLinear;
        op.relu = relu;
        if ((rc = operand(g, written, x, line, &op.a)) || (rc = operand(g, written, w, line, &op.b)))
          return rc;
        if (b != "-" && (rc = operand(g, written, b, line, &op.bias))) return rc;
        if ((rc = result(g, &written, y, line, &op.out))) return rc;
        const GraphTensor &tw = g->t[op.b], &tx = g->t[op.a], &ty = g->t[op.out];
        if (tw.dims.size() != 2) return plan_error(dir, line, "linear weight must be [N, K]");
        op.n = static_cast<int>(tw.dims[0]);
        op.k = static_cast<int>(tw.dims[1]);
        if (op.k % 64 != 0) return plan_error(dir, line, "linear K must be a multiple of 64");
        if ((static_cast<long long>(op.n) + 127) / 128 > kLinearMaxTiles)
          return plan_error(dir, line, "linear N exceeds the projection's 2097152 rows");
        if (tx.dims.back() != op.k || tx.numel % op.k != 0)
          return plan_error(dir, line, "linear input's last dimension is not the weight's K");
        op.rows = tx.numel / op.k;
        if (ty.numel != op.rows * op.n || ty.dims.back() != op.n)
          return plan_error(dir, line, "linear output is not [rows, N]");
        if (op.bias >= 0 && (g->t[op.bias].numel != op.n || g->t[op.bias].dims.size() != 1))
          return plan_error(dir, line, "linear bias is not [N]");
      } else if (kind == "sdpa") {
        std::string o, q, k, v;
        int causal = -1;
        if (!(ls >> o >> q >> k >> v >> op.scale >> causal) || (causal != 0 && causal != 1))
          return plan_error(dir, line, "expected: op sdpa <out> <q> <k> <v> <scale> <causal 0|1>");
        op.kind = kOpSdpa;
        op.causal = causal;
        if ((rc = operand(g, written, q, line, &op.a)) || (rc = operand(g, written, k, line, &op.b)) ||
            (rc = operand(g, written, v, line, &op.c)) || (rc = result(g, &written, o, line, &op.out)))
          return rc;
        const GraphTensor &tq = g->t[op.a], &tk = g->t[op.b], &tv = g->t[op.c], &to = g->t[op.out];
        if (tq.dims.size() != 4 || tk.dims.size() != 4 || tv.dims != tk.dims)
          return plan_error(dir, line, "sdpa needs q [B, H, L, D] and k, v [B, Hkv, S, D]");
        op.batch = static_cast<int>(tq.dims[0]);
        op.heads = static_cast<int>(tq.dims[1]);
        op.queries = static_cast<int>(tq.dims[2]);
        op.dim = static_cast<int>(tq.dims[3]);
        op.kv_heads = static_cast<int>(tk.dims[1]);
        op.keys = static_cast<int>(tk.dims[2]);
        if (tk.dims[0] != op.batch || tk.dims[3] != op.dim || op.heads % op.kv_heads != 0)
          return plan_error(dir, line, "sdpa k/v disagree with q (batch, head size or GQA group)");
        if (to.numel != tq.numel) return plan_error(dir, line, "sdpa output is not q's size");
        if (!std::isfinite(op.scale)) return plan_error(dir, line, "sdpa scale must be finite");
        op.decode = op.queries == 1 && !op.causal && (op.dim == 64 || op.dim == 128) &&
                    op.heads / op.kv_heads <= 8 &&
                    static_cast<long long>(op.batch) * op.kv_heads <= 16384 &&
                    static_cast<long long>(op.batch) * op.kv_heads * op.keys < (1ll << 31);
        if (!op.decode && op.dim != 32 && op.dim != 64 && op.dim != 128)
          return plan_error(dir, line, "sdpa head size must be 32, 64 or 128");
        if (static_cast<long long>(op.batch) * op.kv_heads > 65535)
          return plan_error(dir, line, "sdpa batch x kv_heads exceeds 65535");
        if (!op.decode) {  // the prefill grid: query blocks x head subgroups in grid.y
          int bm = 0, hp = 0;
          prefill_blocking(op.queries, op.heads / op.kv_heads, &bm, &hp);
          const long long q_blocks = (static_cast<long long>(op.queries) + bm - 1) / bm;
          if (q_blocks * (op.heads / op.kv_heads / hp) > 65535)
            return plan_error(dir, line, "sdpa query blocks x head subgroups exceed 65535");
        }
      } else {
        return plan_error(dir, line, "unknown op (this library runs linear and sdpa)");
      }
      g->ops.push_back(op);
    } else {
      return plan_error(dir, line, "unknown line");
    }
  }
  if (!stage || !schema) return plan_error(dir, line, "missing npu.stage / npu.schema stamp");
  if (g->ops.empty()) return plan_error(dir, line, "no ops");
  for (int o : g->outputs)
    if (!written[o]) {
      std::string m = "output " + g->t[o].name + " is never written";
      return plan_error(dir, line, m.c_str());
    }
  return NPU_B200_OK;
}

int alloc(GraphState* g, size_t bytes, void** out) {
  void* p = nullptr;
  NPU_TRY_CUDA(cudaMalloc(&p, bytes < 256 ? 256 : bytes));
  g->allocs.push_back(p);
  *out = p;
  return NPU_B200_OK;
}

int load_device(GraphState* g) {
  std::vector<char> buf;
  for (GraphTensor& t : g->t) {
    if (t.role == kRoleParam) {
      int rc = alloc(g, static_cast<size_t>(t.numel) * 2, &t.dev);
      if (rc) return rc;
      const std::string path = g->dir + "/arg" + std::to_string(t.arg) + ".bin";
      std::ifstream bin(path, std::ios::binary);
      buf.resize(static_cast<size_t>(t.numel) * 2);
      if (!bin.read(buf.data(), static_cast<std::streamsize>(buf.size())))
        return set_error(NPU_B200_E_PLAN, "short read of %s", path.c_str());
      NPU_TRY_CUDA(cudaMemcpy(t.dev, buf.data(), buf.size(), cudaMemcpyHostToDevice));
    } else if (t.role == kRoleTemp) {
      int rc = alloc(g, static_cast<size_t>(t.numel) * 2, &t.dev);
      if (rc) return rc;
    }
  }
  for (GraphOp& op : g->ops) {
    if (op.kind == kOpLinear) {
      // Launches of 128 rows and, if the rows do not divide, one shorter one.
      const int chunk = static_cast<int>(std::min<int64_t>(op.rows, 128));
      const int tail = static_cast<int>(op.rows % 128);
      g->lin_ws_bytes = std::max(g->lin_ws_bytes, npu_b200_linear_workspace_size(op.n, op.k, chunk));
      if (tail > 0)
        g->lin_ws_bytes = std::max(g->lin_ws_bytes, npu_b200_linear_workspace_size(op.n, op.k, tail));
    } else if (op.decode) {
      g->fd_ws_bytes = std::max(
          g->fd_ws_bytes, npu_b200_flash_decode_workspace_size(op.batch, op.kv_heads, op.dim, op.keys, 0));
      void* p = nullptr;
      int rc = alloc(g, sizeof(int32_t) * op.batch, &p);
      if (rc) return rc;
      op.seq_lens = static_cast<int32_t*>(p);
      std::vector<int32_t> lens(op.batch, op.keys);
      NPU_TRY_CUDA(cudaMemcpy(op.seq_lens, lens.data(), lens.size() * sizeof(int32_t),
                              cudaMemcpyHostToDevice));
    }
  }
  // Both workspaces start zero-filled; every kernel that uses one leaves it so.
  if (g->lin_ws_bytes) {
    int rc = alloc(g, g->lin_ws_bytes, &g->lin_ws);
    if (rc) return rc;
    NPU_TRY_CUDA(cudaMemset(g->lin_ws, 0, g->lin_ws_bytes));
  }
  if (g->fd_ws_bytes) {
    int rc = alloc(g, g->fd_ws_bytes, &g->fd_ws);
    if (rc) return rc;
    NPU_TRY_CUDA(cudaMemset(g->fd_ws, 0, g->fd_ws_bytes));
  }
  return NPU_B200_OK;
}

}  // namespace

void graph_free(GraphState* g) {
  if (!g) return;
  for (void* p : g->allocs) cudaFree(p);
  delete g;
}

}  // namespace npu_b200

using namespace npu_b200;

extern "C" int npu_b200_graph_check(const char* dir, int64_t* out, int n) {
  clear_error();
  NPU_REQUIRE(dir && out && n >= 6, "graph_check needs a directory and 6 slots");
  GraphState g;
  const int rc = parse_graph(dir, &g);
  if (rc) return rc;
  const int64_t v[6] = {static_cast<int64_t>(g.inputs.size()), static_cast<int64_t>(g.outputs.size()),
                        static_cast<int64_t>(g.ops.size()), g.param_bytes, g.temp_bytes,
                        static_cast<int64_t>(std::count_if(g.ops.begin(), g.ops.end(),
                                                           [](const GraphOp& o) { return o.decode; }))};
  for (int i = 0; i < 6; ++i) out[i] = v[i];
  return NPU_B200_OK;
}

extern "C" int npu_b200_load_graph(npu_b200_ctx* c, const char* dir) {
  clear_error();
  NPU_REQUIRE(c && dir, "null argument");
  GraphState* g = new GraphState();
  int rc = parse_graph(dir, g);
  if (!rc) rc = check_cuda(cudaSetDevice(ctx_device(c)), "cudaSetDevice");
  if (!rc) rc = load_device(g);
  if (rc) {
    graph_free(g);
    return rc;
  }
  GraphState*& slot = ctx_graph(c);
  if (slot) {
    cudaDeviceSynchronize();
    graph_free(slot);
  }
  slot = g;
  return NPU_B200_OK;
}

extern "C" int npu_b200_run_graph(npu_b200_ctx* c, void* const* args, void* const* outs,
                                  void* stream) {
  clear_error();
  NPU_REQUIRE(c, "null context");
  GraphState* g = ctx_graph(c);
  if (!g) return set_error(NPU_B200_E_STATE, "no graph loaded");
  NPU_REQUIRE(g->inputs.empty() || args, "graph has inputs but no argument array");
  NPU_REQUIRE(outs, "null output array");
  NPU_TRY_CUDA(cudaSetDevice(ctx_device(c)));
  std::vector<char*> ptr(g->t.size(), nullptr);
  for (size_t i = 0; i < g->t.size(); ++i) {
    const GraphTensor& t = g->t[i];
    if (t.role == kRoleInput) ptr[i] = static_cast<char*>(args[t.io]);
    if (t.role == kRoleOutput) ptr[i] = static_cast<char*>(outs[t.io]);
    if (t.role == kRoleParam || t.role == kRoleTemp) ptr[i] = static_cast<char*>(t.dev);
    if ((t.role == kRoleInput || t.role == kRoleOutput) &&
        (ptr[i] == nullptr || (reinterpret_cast<uintptr_t>(ptr[i]) & 15) != 0))
      return set_error(NPU_B200_E_INVALID, "graph %s %s: null or not 16-byte aligned",
                       t.role == kRoleInput ? "input" : "output", t.name.c_str());
  }
  for (size_t i = 0; i < g->t.size(); ++i)
    if (g->t[i].role == kRoleAlias) ptr[i] = ptr[g->t[i].base];
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (const GraphOp& op : g->ops) {
    int rc = 0;
    if (op.kind == kOpLinear) {
      for (int64_t r0 = 0; r0 < op.rows && !rc; r0 += 128) {
        const int rows = static_cast<int>(std::min<int64_t>(128, op.rows - r0));
        rc = npu_b200_linear(ptr[op.a] + r0 * op.k * 2, ptr[op.b],
                             op.bias >= 0 ? ptr[op.bias] : nullptr, ptr[op.out] + r0 * op.n * 2,
                             rows, op.n, op.k, op.relu ? NPU_B200_LINEAR_RELU : 0, g->lin_ws,
                             g->lin_ws_bytes, s);
      }
    } else if (op.decode) {
      rc = npu_b200_flash_decode(ptr[op.a], ptr[op.b], ptr[op.c], op.seq_lens, ptr[op.out],
                                 op.batch, op.heads, op.kv_heads, op.dim, op.keys, op.scale, 0,
                                 g->fd_ws, g->fd_ws_bytes, s);
    } else {
      rc = npu_b200_prefill_attention(ptr[op.a], ptr[op.b], ptr[op.c], nullptr, ptr[op.out],
                                      op.batch, op.heads, op.kv_heads, op.dim, op.queries,
                                      op.keys, op.keys, op.scale, op.causal, s);
    }
    if (rc) return rc;
  }
  return NPU_B200_OK;
}
