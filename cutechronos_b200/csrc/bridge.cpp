// Native implementation of the reference's C bridge (include/cutechronos_bridge.h)
// over the engine's C ABI: loads a Chronos-2 checkpoint directory (config.json +
// model.safetensors) without Python, keeps one session per handle and serves
// median forecasts of single series.
//
// Reference behaviour mirrored: cutechronos_bridge.c:96-406 (entry points,
// error buffer, -1 on failure) and foreign.py:85-186 / pipeline.py:327-474
// (device and dtype names, context truncation to context_length, horizon
// limit of max_output_patches * patch, N = ceil(H / patch), median = the 0.5
// quantile, interpolated between neighbours when it is not a trained level).
#include <cuda_runtime.h>

#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <mutex>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/cc2.h"
#include "../../include/cutechronos_bridge.h"

namespace {

// ---------------------------------------------------------------- errors ----
struct BridgeError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

std::string fmt(const char* f, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, f);
  vsnprintf(buf, sizeof(buf), f, ap);
  va_end(ap);
  return buf;
}

void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw BridgeError(fmt("%s: %s", what, cudaGetErrorString(e)));
}
void cc2_check(int s, const char* what) {
  if (s != CC2_OK) throw BridgeError(fmt("%s failed (%d): %s", what, s, cc2_last_error()));
}

void write_error(char* buf, size_t n, const std::string& msg) {
  if (!buf || n == 0) return;
  const size_t k = std::min(n - 1, msg.size());
  std::memcpy(buf, msg.data(), k);
  buf[k] = '\0';
}

// ------------------------------------------------------------------ JSON ----
struct Json {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  bool b = false;
  double num = 0.0;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;
  const Json* get(const std::string& k) const {
    for (const auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

struct JsonParser {
  const char* p;
  const char* end;
  void ws() {
    while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  [[noreturn]] void fail(const char* what) { throw BridgeError(fmt("JSON parse error: %s", what)); }
  char peek() {
    ws();
    if (p >= end) fail("unexpected end");
    return *p;
  }
  void expect(char c) {
    if (peek() != c) fail("unexpected character");
    ++p;
  }
  std::string string() {
    expect('"');
    std::string s;
    while (p < end && *p != '"') {
      if (*p == '\\') {
        ++p;
        if (p >= end) fail("bad escape");
        switch (*p) {
          case 'n': s += '\n'; break;
          case 't': s += '\t'; break;
          case 'r': s += '\r'; break;
          case 'b': s += '\b'; break;
          case 'f': s += '\f'; break;
          case 'u': {
            if (end - p < 5) fail("bad \\u escape");
            const unsigned cp = (unsigned)std::stoul(std::string(p + 1, p + 5), nullptr, 16);
            if (cp < 0x80) s += (char)cp; else s += '?';  // names and keys here are ASCII
            p += 4;
            break;
          }
          default: s += *p;
        }
        ++p;
      } else {
        s += *p++;
      }
    }
    if (p >= end) fail("unterminated string");
    ++p;
    return s;
  }
  Json value() {
    Json v;
    const char c = peek();
    if (c == '{') {
      ++p;
      v.kind = Json::Obj;
      if (peek() == '}') { ++p; return v; }
      while (true) {
        std::string k = string();
        expect(':');
        v.obj.emplace_back(std::move(k), value());
        if (peek() == ',') { ++p; continue; }
        expect('}');
        return v;
      }
    }
    if (c == '[') {
      ++p;
      v.kind = Json::Arr;
      if (peek() == ']') { ++p; return v; }
      while (true) {
        v.arr.push_back(value());
        if (peek() == ',') { ++p; continue; }
        expect(']');
        return v;
      }
    }
    if (c == '"') {
      v.kind = Json::Str;
      v.str = string();
      return v;
    }
    if (!std::strncmp(p, "true", 4)) { p += 4; v.kind = Json::Bool; v.b = true; return v; }
    if (!std::strncmp(p, "false", 5)) { p += 5; v.kind = Json::Bool; return v; }
    if (!std::strncmp(p, "null", 4)) { p += 4; return v; }
    char* e = nullptr;
    v.num = std::strtod(p, &e);
    if (e == p) fail("bad value");
    p = e;
    v.kind = Json::Num;
    return v;
  }
};

Json parse_json(const std::string& text) {
  JsonParser jp{text.data(), text.data() + text.size()};
  return jp.value();
}

std::string read_file(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw BridgeError("cannot open " + path);
  std::ostringstream ss;
  ss << f.rdbuf();
  return ss.str();
}

double num_or(const Json* o, const char* k, double dflt) {
  const Json* v = o ? o->get(k) : nullptr;
  return v && v->kind == Json::Num ? v->num : dflt;
}
bool bool_or(const Json* o, const char* k, bool dflt) {
  const Json* v = o ? o->get(k) : nullptr;
  return v && v->kind == Json::Bool ? v->b : dflt;
}

// --------------------------------------------------------------- weights ----
uint16_t f32_to_bf16(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);  // NaN stays NaN
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
float bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}
float f16_to_f32(uint16_t h) {
  const uint32_t s = (h >> 15) & 1u, e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
  float v;
  if (e == 0) v = std::ldexp((float)m, -24);
  else if (e == 31) v = m ? NAN : INFINITY;
  else v = std::ldexp((float)(m | 0x400u), (int)e - 25);
  return s ? -v : v;
}

struct SafeTensors {
  std::string blob;  // whole file
  size_t data0 = 0;  // start of the data section
  Json header;
  explicit SafeTensors(const std::string& path) {
    blob = read_file(path);
    if (blob.size() < 8) throw BridgeError("safetensors file too small: " + path);
    uint64_t n = 0;
    for (int i = 7; i >= 0; --i) n = (n << 8) | (uint8_t)blob[i];
    if (8 + n > blob.size()) throw BridgeError("safetensors header length out of range");
    header = parse_json(blob.substr(8, n));
    data0 = 8 + n;
  }
  // tensor `name` as `count` values converted to fp32
  std::vector<float> f32(const std::string& name, size_t count) const {
    const Json* t = header.get(name);
    if (!t) throw BridgeError("checkpoint is missing tensor " + name);
    const Json* dt = t->get("dtype");
    const Json* off = t->get("data_offsets");
    if (!dt || !off || off->arr.size() != 2) throw BridgeError("malformed entry for " + name);
    const size_t b = (size_t)off->arr[0].num, e = (size_t)off->arr[1].num;
    const std::string& d = dt->str;
    const size_t esz = d == "F32" ? 4 : (d == "BF16" || d == "F16") ? 2 : 0;
    if (!esz) throw BridgeError("unsupported dtype " + d + " for " + name);
    if ((e - b) != count * esz || data0 + e > blob.size())
      throw BridgeError(fmt("tensor %s has %zu bytes, expected %zu", name.c_str(), e - b, count * esz));
    const char* src = blob.data() + data0 + b;
    std::vector<float> out(count);
    for (size_t i = 0; i < count; ++i) {
      if (esz == 4) {
        std::memcpy(&out[i], src + 4 * i, 4);
      } else {
        uint16_t h;
        std::memcpy(&h, src + 2 * i, 2);
        out[i] = d == "BF16" ? bf16_to_f32(h) : f16_to_f32(h);
      }
    }
    return out;
  }
};

// ------------------------------------------------------------- sessions ----
struct Graph {
  cudaGraphExec_t exec = nullptr;
};

struct Session {
  int device = 0;
  int dtype = CC2_BF16;
  size_t esz = 2;
  cc2_config cfg{};
  std::vector<float> quantiles;
  bool use_graphs = false;
  cudaStream_t stream = nullptr;
  void* pack = nullptr;
  cc2_model* model = nullptr;
  void* ws = nullptr;
  size_t ws_bytes = 0;
  float* d_ctx = nullptr;
  size_t ctx_cap = 0;
  void* d_out = nullptr;
  size_t out_cap = 0;
  std::vector<uint8_t> h_out;
  std::map<std::pair<int, int>, Graph> graphs;
  std::mutex mu;

  void drop_graphs() {
    for (auto& kv : graphs)
      if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
    graphs.clear();
  }
  ~Session() {
    if (!stream) return;  // failed before the device was touched: nothing to free
    cudaSetDevice(device);
    drop_graphs();
    if (model) cc2_model_destroy(model);
    cudaFree(pack);
    cudaFree(ws);
    cudaFree(d_ctx);
    cudaFree(d_out);
    if (stream) cudaStreamDestroy(stream);
  }
};

std::mutex g_mu;
std::map<int, std::shared_ptr<Session>> g_sessions;
int g_next = 1;

int parse_device(const char* device) {
  if (!device || !*device || !std::strcmp(device, "cuda")) return 0;
  if (!std::strncmp(device, "cuda:", 5)) return std::atoi(device + 5);
  throw BridgeError(fmt("unsupported device '%s' (this engine runs on CUDA devices only)", device));
}

std::shared_ptr<Session> load_session(const char* model_id, const char* backend, const char* device,
                                      const char* dtype_name, const char* compile_mode) {
  if (!model_id || !*model_id) throw BridgeError("model_id is required");
  if (backend && *backend && std::strcmp(backend, "cute"))
    throw BridgeError(fmt("Unsupported backend '%s'. Expected 'cute'.", backend));
  auto s = std::make_shared<Session>();
  s->device = parse_device(device);
  const std::string dn = dtype_name && *dtype_name ? dtype_name : "bfloat16";
  if (dn == "bfloat16" || dn == "bf16") {
    s->dtype = CC2_BF16;
    s->esz = 2;
  } else if (dn == "float32" || dn == "fp32") {
    s->dtype = CC2_F32;
    s->esz = 4;
  } else {
    throw BridgeError("Unsupported dtype '" + dn + "'. Expected 'bfloat16' or 'float32'");
  }
  s->use_graphs = compile_mode && *compile_mode;

  const std::string dir = model_id;
  if (std::ifstream(dir + "/adapter_config.json"))
    throw BridgeError("LoRA adapter checkpoints are not loaded by the native bridge; merge the adapter first");
  if (!std::ifstream(dir + "/model.safetensors"))
    throw BridgeError("No model weights found in " + dir + ". The native bridge reads model.safetensors");
  const Json conf = parse_json(read_file(dir + "/config.json"));
  const Json* ch = conf.get("chronos_config");
  cc2_config& c = s->cfg;
  c.d_model = (int)num_or(&conf, "d_model", 768);
  c.d_kv = (int)num_or(&conf, "d_kv", 64);
  c.d_ff = (int)num_or(&conf, "d_ff", 3072);
  c.num_layers = (int)num_or(&conf, "num_layers", 12);
  c.num_heads = (int)num_or(&conf, "num_heads", 12);
  c.layer_norm_epsilon = (float)num_or(&conf, "layer_norm_epsilon", 1e-6);
  c.rope_theta = (float)num_or(&conf, "rope_theta", 10000.0);
  c.reg_token_id = (int)num_or(&conf, "reg_token_id", 1);
  c.context_length = (int)num_or(ch, "context_length", 8192);
  c.input_patch_size = (int)num_or(ch, "input_patch_size", 16);
  c.output_patch_size = (int)num_or(ch, "output_patch_size", 16);
  c.use_reg_token = bool_or(ch, "use_reg_token", true);
  c.use_arcsinh = bool_or(ch, "use_arcsinh", true);
  c.time_encoding_scale = (float)num_or(ch, "time_encoding_scale", c.context_length);
  c.max_output_patches = (int)num_or(ch, "max_output_patches", 64);
  const Json* act = conf.get("dense_act_fn");
  if (act && act->kind == Json::Str && act->str != "relu")
    throw BridgeError("dense_act_fn '" + act->str + "' is not supported (relu only)");
  const Json* q = ch ? ch->get("quantiles") : nullptr;
  if (q && q->kind == Json::Arr)
    for (const auto& v : q->arr) s->quantiles.push_back((float)v.num);
  if (s->quantiles.empty())
    s->quantiles = {0.01f, 0.05f, 0.1f, 0.15f, 0.2f, 0.25f, 0.3f, 0.35f, 0.4f, 0.45f, 0.5f,
                    0.55f, 0.6f, 0.65f, 0.7f, 0.75f, 0.8f, 0.85f, 0.9f, 0.95f, 0.99f};
  c.num_quantiles = (int)s->quantiles.size();

  // weights: HF names (model.py:833-900), converted to the model dtype and uploaded
  const SafeTensors st(dir + "/model.safetensors");
  const int d = c.d_model, dff = c.d_ff, in = 3 * c.input_patch_size, qps = c.num_quantiles * c.output_patch_size;
  const int inner = c.num_heads * c.d_kv;
  struct Item { std::string name; size_t count; };
  std::vector<Item> items = {
      {"shared.weight", (size_t)2 * d},
      {"input_patch_embedding.hidden_layer.weight", (size_t)dff * in},
      {"input_patch_embedding.hidden_layer.bias", (size_t)dff},
      {"input_patch_embedding.output_layer.weight", (size_t)d * dff},
      {"input_patch_embedding.output_layer.bias", (size_t)d},
      {"input_patch_embedding.residual_layer.weight", (size_t)d * in},
      {"input_patch_embedding.residual_layer.bias", (size_t)d},
      {"encoder.final_layer_norm.weight", (size_t)d},
      {"output_patch_embedding.hidden_layer.weight", (size_t)dff * d},
      {"output_patch_embedding.hidden_layer.bias", (size_t)dff},
      {"output_patch_embedding.output_layer.weight", (size_t)qps * dff},
      {"output_patch_embedding.output_layer.bias", (size_t)qps},
      {"output_patch_embedding.residual_layer.weight", (size_t)qps * d},
      {"output_patch_embedding.residual_layer.bias", (size_t)qps},
  };
  if (const Json* sh = st.header.get("shared.weight")) {
    const Json* shp = sh->get("shape");
    if (shp && shp->arr.size() == 2) items[0].count = (size_t)shp->arr[0].num * d;
  }
  for (int l = 0; l < c.num_layers; ++l) {
    const std::string p = "encoder.block." + std::to_string(l) + ".layer.";
    for (int j = 0; j < 2; ++j) {
      items.push_back({p + std::to_string(j) + ".layer_norm.weight", (size_t)d});
      for (const char* prj : {"q", "k", "v"})
        items.push_back({p + std::to_string(j) + ".self_attention." + prj + ".weight", (size_t)inner * d});
      items.push_back({p + std::to_string(j) + ".self_attention.o.weight", (size_t)d * inner});
    }
    items.push_back({p + "2.layer_norm.weight", (size_t)d});
    items.push_back({p + "2.mlp.wi.weight", (size_t)dff * d});
    items.push_back({p + "2.mlp.wo.weight", (size_t)d * dff});
  }
  // every tensor is checked and converted on the host before the device is touched
  std::vector<size_t> offs;
  size_t total = 0;
  for (const auto& it : items) {
    offs.push_back(total);
    total += (it.count * s->esz + 255) / 256 * 256;
  }
  std::vector<uint8_t> host(total);
  for (size_t i = 0; i < items.size(); ++i) {
    const std::vector<float> v = st.f32(items[i].name, items[i].count);
    uint8_t* dst = host.data() + offs[i];
    if (s->dtype == CC2_F32) {
      std::memcpy(dst, v.data(), v.size() * 4);
    } else {
      for (size_t k = 0; k < v.size(); ++k) {
        const uint16_t h = f32_to_bf16(v[k]);
        std::memcpy(dst + 2 * k, &h, 2);
      }
    }
  }
  cuda_check(cudaSetDevice(s->device), "cudaSetDevice");
  cuda_check(cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking), "cudaStreamCreate");
  void* raw = nullptr;
  cuda_check(cudaMalloc(&raw, total), "cudaMalloc(weights)");
  std::unique_ptr<void, decltype(&cudaFree)> raw_guard(raw, &cudaFree);
  cuda_check(cudaMemcpy(raw, host.data(), total, cudaMemcpyHostToDevice), "cudaMemcpy(weights)");
  std::map<std::string, const void*> ptr;
  for (size_t i = 0; i < items.size(); ++i) ptr[items[i].name] = static_cast<char*>(raw) + offs[i];
  auto P = [&](const std::string& n) { return ptr.at(n); };
  const int L = c.num_layers;
  std::vector<const void*> arrs[13];
  const char* names[13] = {"0.layer_norm.weight", "0.self_attention.q.weight", "0.self_attention.k.weight",
                           "0.self_attention.v.weight", "0.self_attention.o.weight", "1.layer_norm.weight",
                           "1.self_attention.q.weight", "1.self_attention.k.weight", "1.self_attention.v.weight",
                           "1.self_attention.o.weight", "2.layer_norm.weight", "2.mlp.wi.weight", "2.mlp.wo.weight"};
  for (int a = 0; a < 13; ++a)
    for (int l = 0; l < L; ++l) arrs[a].push_back(P("encoder.block." + std::to_string(l) + ".layer." + names[a]));
  cc2_weights w{};
  w.shared = P("shared.weight");
  w.in_hidden_w = P("input_patch_embedding.hidden_layer.weight");
  w.in_hidden_b = P("input_patch_embedding.hidden_layer.bias");
  w.in_output_w = P("input_patch_embedding.output_layer.weight");
  w.in_output_b = P("input_patch_embedding.output_layer.bias");
  w.in_residual_w = P("input_patch_embedding.residual_layer.weight");
  w.in_residual_b = P("input_patch_embedding.residual_layer.bias");
  w.time_ln = arrs[0].data(); w.time_q = arrs[1].data(); w.time_k = arrs[2].data();
  w.time_v = arrs[3].data(); w.time_o = arrs[4].data();
  w.group_ln = arrs[5].data(); w.group_q = arrs[6].data(); w.group_k = arrs[7].data();
  w.group_v = arrs[8].data(); w.group_o = arrs[9].data();
  w.ff_ln = arrs[10].data(); w.ff_wi = arrs[11].data(); w.ff_wo = arrs[12].data();
  w.final_ln = P("encoder.final_layer_norm.weight");
  w.out_hidden_w = P("output_patch_embedding.hidden_layer.weight");
  w.out_hidden_b = P("output_patch_embedding.hidden_layer.bias");
  w.out_output_w = P("output_patch_embedding.output_layer.weight");
  w.out_output_b = P("output_patch_embedding.output_layer.bias");
  w.out_residual_w = P("output_patch_embedding.residual_layer.weight");
  w.out_residual_b = P("output_patch_embedding.residual_layer.bias");
  size_t pack_bytes = 0;
  cc2_check(cc2_model_pack_bytes(&c, s->dtype, &pack_bytes), "cc2_model_pack_bytes");
  cuda_check(cudaMalloc(&s->pack, pack_bytes), "cudaMalloc(pack)");
  cc2_check(cc2_model_create(&c, s->dtype, &w, s->pack, pack_bytes, s->stream, &s->model), "cc2_model_create");
  cuda_check(cudaStreamSynchronize(s->stream), "cudaStreamSynchronize");
  return s;  // raw weights freed by raw_guard: the packed model no longer needs them
}

template <typename T>
void grow(T*& p, size_t& cap, size_t need, const char* what) {
  if (cap >= need) return;
  cudaFree(p);
  p = nullptr;
  cap = 0;
  cuda_check(cudaMalloc((void**)&p, need), what);
  cap = need;
}

void predict(Session& s, const float* context, int context_length, int H, float* out_values, int out_capacity,
             int* out_length, double* latency_ms) {
  const cc2_config& c = s.cfg;
  const int ps = c.output_patch_size;
  if (!context || context_length < 1) throw BridgeError("context must hold at least one value");
  if (H < 1) throw BridgeError("prediction_length must be positive");
  const int limit = c.max_output_patches * ps;
  if (H > limit)
    throw BridgeError(fmt("prediction_length (%d) exceeds model_prediction_length (%d). Quality may degrade. Set limit_prediction_length=False to allow this.", H,
                          limit));
  if (H > out_capacity) throw BridgeError("forecast buffer too small");
  cuda_check(cudaSetDevice(s.device), "cudaSetDevice");
  const int L = std::min(context_length, c.context_length);
  const float* src = context + (context_length - L);
  const int N = (H + ps - 1) / ps;
  const int Q = c.num_quantiles;
  size_t ws_need = 0;
  cc2_check(cc2_forward_workspace_bytes(s.model, 1, L, N, 1, &ws_need), "cc2_forward_workspace_bytes");
  const size_t out_bytes = (size_t)Q * N * ps * s.esz;
  if (s.ws_bytes < ws_need || s.ctx_cap < (size_t)L * 4 || s.out_cap < out_bytes) s.drop_graphs();
  {
    size_t cap = s.ws_bytes;
    void* p = s.ws;
    grow(p, cap, ws_need, "cudaMalloc(workspace)");
    s.ws = p;
    s.ws_bytes = cap;
  }
  grow(s.d_ctx, s.ctx_cap, (size_t)L * 4, "cudaMalloc(context)");
  grow(s.d_out, s.out_cap, out_bytes, "cudaMalloc(output)");
  s.h_out.resize(out_bytes);

  cuda_check(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  const auto t0 = std::chrono::steady_clock::now();
  cuda_check(cudaMemcpyAsync(s.d_ctx, src, (size_t)L * 4, cudaMemcpyHostToDevice, s.stream), "cudaMemcpyAsync(H2D)");
  auto run = [&]() {
    cc2_check(cc2_forward(s.model, s.d_ctx, nullptr, 1, L, N, nullptr, s.d_out, nullptr, nullptr, s.ws, s.ws_bytes,
                          s.stream),
              "cc2_forward");
  };
  if (s.use_graphs) {
    Graph& g = s.graphs[{L, N}];
    if (!g.exec) {
      run();  // first call of a shape runs eagerly, then the shape is captured
      cuda_check(cudaStreamSynchronize(s.stream), "cudaStreamSynchronize");
      cudaGraph_t graph = nullptr;
      cuda_check(cudaStreamBeginCapture(s.stream, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
      const int st = cc2_forward(s.model, s.d_ctx, nullptr, 1, L, N, nullptr, s.d_out, nullptr, nullptr, s.ws,
                                 s.ws_bytes, s.stream);
      const cudaError_t ce = cudaStreamEndCapture(s.stream, &graph);
      cc2_check(st, "cc2_forward (capture)");
      cuda_check(ce, "cudaStreamEndCapture");
      const cudaError_t ie = cudaGraphInstantiate(&g.exec, graph, 0);
      cudaGraphDestroy(graph);
      cuda_check(ie, "cudaGraphInstantiate");
    } else {
      cuda_check(cudaGraphLaunch(g.exec, s.stream), "cudaGraphLaunch");
    }
  } else {
    run();
  }
  cuda_check(cudaMemcpyAsync(s.h_out.data(), s.d_out, out_bytes, cudaMemcpyDeviceToHost, s.stream),
             "cudaMemcpyAsync(D2H)");
  cuda_check(cudaStreamSynchronize(s.stream), "cudaStreamSynchronize");
  const auto t1 = std::chrono::steady_clock::now();
  // a kernel whose bounded wait ran out returns early with incomplete outputs
  const int dev_status = cc2_device_status(1);
  if (dev_status < 0) cc2_check(dev_status, "cc2_device_status");
  if (dev_status != 0)
    throw BridgeError(fmt("a kernel of the forward gave up waiting (device status %d); no forecast returned",
                          dev_status));

  // the 0.5 quantile: the trained level, else linear between its neighbours (pipeline.py:24-58)
  const std::vector<float>& tq = s.quantiles;
  int lo = -1, hi = -1;
  float frac = 0.0f;
  for (int i = 0; i < Q; ++i)
    if (tq[i] == 0.5f) lo = hi = i;
  if (lo < 0) {
    int idx = 0;
    while (idx < Q && tq[idx] < 0.5f) ++idx;
    idx = std::max(1, std::min(Q - 1, idx));
    lo = idx - 1;
    hi = idx;
    frac = (0.5f - tq[lo]) / std::max(tq[hi] - tq[lo], 1e-9f);
  }
  const int Hfull = N * ps;
  auto value = [&](int qi, int t) -> float {
    const size_t k = (size_t)qi * Hfull + t;
    if (s.dtype == CC2_F32) {
      float f;
      std::memcpy(&f, s.h_out.data() + 4 * k, 4);
      return f;
    }
    uint16_t h;
    std::memcpy(&h, s.h_out.data() + 2 * k, 2);
    return bf16_to_f32(h);
  };
  for (int t = 0; t < H; ++t)
    out_values[t] = lo == hi ? value(lo, t) : value(lo, t) * (1.0f - frac) + value(hi, t) * frac;
  *out_length = H;
  *latency_ms = std::chrono::duration<double, std::milli>(t1 - t0).count();
}

std::shared_ptr<Session> find(int handle) {
  std::lock_guard<std::mutex> lock(g_mu);
  auto it = g_sessions.find(handle);
  if (it == g_sessions.end()) throw BridgeError(fmt("unknown pipeline handle %d", handle));
  return it->second;
}

}  // namespace

extern "C" {

int cutechronos_init_pipeline(const char* model_id, const char* backend, const char* device, const char* dtype_name,
                              const char* compile_mode, int* out_handle, char* error_buffer, size_t error_buffer_size) {
  try {
    if (!out_handle) throw BridgeError("out_handle is required");
    auto s = load_session(model_id, backend, device, dtype_name, compile_mode);
    std::lock_guard<std::mutex> lock(g_mu);
    const int h = g_next++;
    g_sessions[h] = std::move(s);
    *out_handle = h;
    write_error(error_buffer, error_buffer_size, "");
    return 0;
  } catch (const std::exception& e) {
    write_error(error_buffer, error_buffer_size, e.what());
    return -1;
  }
}

int cutechronos_predict_median(int handle, const float* context, int context_length, int prediction_length,
                               float* out_values, int out_capacity, int* out_length, double* out_latency_ms,
                               char* error_buffer, size_t error_buffer_size) {
  try {
    if (!out_values || !out_length || !out_latency_ms) throw BridgeError("output buffers are required");
    auto s = find(handle);
    std::lock_guard<std::mutex> lock(s->mu);
    predict(*s, context, context_length, prediction_length, out_values, out_capacity, out_length, out_latency_ms);
    write_error(error_buffer, error_buffer_size, "");
    return 0;
  } catch (const std::exception& e) {
    write_error(error_buffer, error_buffer_size, e.what());
    return -1;
  }
}

int cutechronos_destroy_pipeline(int handle, char* error_buffer, size_t error_buffer_size) {
  try {
    std::shared_ptr<Session> s;
    {
      std::lock_guard<std::mutex> lock(g_mu);
      auto it = g_sessions.find(handle);
      if (it == g_sessions.end()) throw BridgeError(fmt("unknown pipeline handle %d", handle));
      s = std::move(it->second);
      g_sessions.erase(it);
    }
    std::lock_guard<std::mutex> lock(s->mu);  // waits for a predict in flight on this handle
    write_error(error_buffer, error_buffer_size, "");
    return 0;  // the session's device memory is released when its last reference goes
  } catch (const std::exception& e) {
    write_error(error_buffer, error_buffer_size, e.what());
    return -1;
  }
}

}  // extern "C"
