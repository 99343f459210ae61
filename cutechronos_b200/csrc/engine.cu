// cc2 engine: weight packing, workspace layout, forward orchestration and the
// C ABI declared in include/cc2.h.
//
// Forward (CuteChronos2Model.forward, cutechronos/model.py:738-831) as launched
// here, for B series of S = P + 1 + N tokens, M = B*S rows, d = d_model:
//   preprocess           -> E[:, dff:dff+3ps] rows (context/REG/future), token mask, loc, scale
//   gemm  E[:,dff:] @ W1^T + b1, ReLU               -> E[:, :dff]      (input ResidualBlock hidden)
//   gemm  E @ [W2|W3]^T + (b2+b3), REG row := shared[1], ssq0 -> X    (hidden + skip in one GEMM)
//   per layer l:
//     gemm  X @ Wqkv_t^T * rs(ssq[3l]), RoPE on Q,K -> QKV            (RMSNorm folded; RoPE in the
//                                                                     epilogue in bf16 mode)
//     attention mode 0 (key mask)                   -> ATT
//     gemm  ATT @ Wo_t^T + X, ssq[3l+1]             -> X
//     group size 1: gemm X @ (Wo_g Wv_g)^T * rs + X, ssq[3l+2] -> Y; swap X, Y
//                   (softmax over one key = V, so the block is one projection)
//     else:         gemm X @ Wqkv_g^T * rs -> QKV; attention mode 1 -> ATT;
//                   gemm ATT @ Wo_g^T + X, ssq[3l+2] -> X
//     gemm  X @ Wi^T * rs(ssq[3l+2]), ReLU          -> E (as [M, dff])
//     gemm  E @ Wo^T + X, ssq[3l+3]                 -> X
//   rmsnorm_rows (final norm of the N future rows)  -> O[:, dff:]
//   gemm  O[:,dff:] @ W1o^T + b1o, ReLU             -> O[:, :dff]
//   gemm  O @ [W2o|W3o]^T + (b2o+b3o)               -> PRED [B*N, Q*ps]
//   output_transform (rearrange, sinh, unscale)     -> out [B, Q, N*ps]
#include <cmath>
#include <cstdarg>
#include <cstring>
#include <mutex>
#include <numeric>
#include <unordered_map>
#include <vector>

#include "common.cuh"

namespace cc2 {

// programmatic dependent launch of the forward's kernels (1 = on)
int g_launch_overlap = 1;
thread_local int t_launch_overlap = 1;

namespace {
// Sets t_launch_overlap for the duration of one forward.
struct LaunchOverlapScope {
  int saved;
  explicit LaunchOverlapScope(int on) : saved(t_launch_overlap) { t_launch_overlap = on; }
  ~LaunchOverlapScope() { t_launch_overlap = saved; }
};
}  // namespace

// ---- status -----------------------------------------------------------------
static thread_local std::string t_error;
void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_error = buf;
}
void clear_error() { t_error.clear(); }

int num_sms() {
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

// ---- kernels implemented in the other translation units ----------------------
int launch_preprocess(const float*, const float*, int, int, int, int, float, int, int, int, int, void*, int,
                      int, uint8_t*, float*, float*, float*, cudaStream_t);
int launch_output_transform(int, const void*, int, const float*, const float*, void*, int, int, int, int, int,
                            cudaStream_t);
int launch_rmsnorm_rows(int, const void*, int, const void*, void*, int, int, int, int, int, int, float,
                        cudaStream_t);
void set_gemm_weights_const(bool on);
int launch_gemm_tc(const void*, int, const void*, int, void*, int, int, int, int, const cc2_epilogue*,
                   cudaStream_t);
extern int g_gemm_variant;
extern int g_attn_variant;
int set_attn_trace(void* buf);
int set_attn_long_trace(void* buf);
int set_gemm_trace(void* buf);
int set_gemm_starve(int on);
int set_chain_starve(int on);
int set_chain_trace(void* buf);
size_t gemm_f32_splitk_floats();
int launch_kv_quant(int dtype, void* qkv, int ld, int rows, int q_col, int k_col, int v_col, int heads,
                    const cc2_kvq* key, const cc2_kvq* value, const float* rope_cs, int rope_period, float* stats,
                    cudaStream_t st);
bool attn_group_tc_supported(int g, int ld, int ldo, const void* qkv, const void* out);
int launch_attn_group_tc(const void* qkv, int ld, int qcol, int kcol, int vcol, void* out, int ldo,
                         const uint8_t* tok, int B, int S, int heads, int g, int* err, cudaStream_t st);
int attention_error_word(int** p);
int chain_max_stages();
int chain_max_set();
int chain_begin(int M);
void chain_abandon();
int chain_add_gemm(const void* A, int lda, const void* W, int ldw, void* out, int ldo, int M, int N, int K,
                   const cc2_epilogue* e);
int chain_add_attention(const void* qkv, int ld, int qcol, int kcol, int vcol, void* out, int ldo,
                        const uint8_t* tok, int sets, int S, int heads);
int chain_launch(void* scratch, size_t scratch_bytes, int exact, cudaStream_t st);
size_t chain_scratch_bytes();
// 1: the encoder layers of a bf16 forward with few token rows run as one
// layer-persistent kernel; 2: the same in its exact mode; 0 (default): kernel
// by kernel - the persistent launch measured no faster (cc2_set_layer_chain)
int g_layer_chain = 0;
constexpr int kChainMaxRows = 384;  // token rows (B x S) up to which the layers run as one launch
int launch_gemm_f32(const void*, int, const void*, int, void*, int, int, int, int, const cc2_epilogue*,
                    cudaStream_t, float* scratch = nullptr, size_t scratch_floats = 0);
int launch_attention(int, int, const void*, int, int, int, int, void*, int, const uint8_t*, int, int, int, int,
                     const int32_t*, const int32_t*, int, int, const float*, cudaStream_t);

// ---- packing kernels ------------------------------------------------------------
template <typename T>
__global__ void pack_matrix_kernel(T* dst, int ldd, const T* src, int rows, int cols, const T* colscale) {
  const size_t total = (size_t)rows * cols;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / cols), c = (int)(i % cols);
    float v = tof<T>(src[i]);
    if (colscale) v *= tof<T>(colscale[c]);
    dst[(size_t)r * ldd + c] = fromf<T>(v);
  }
}
// dst (fp32) = src * colscale[c], optionally transposed (dst[c][r]).
template <typename T>
__global__ void to_f32_kernel(float* dst, const T* src, int rows, int cols, const T* colscale, int transpose) {
  const size_t total = (size_t)rows * cols;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / cols), c = (int)(i % cols);
    float v = tof<T>(src[i]);
    if (colscale) v *= tof<T>(colscale[c]);
    dst[transpose ? (size_t)c * rows + r : i] = v;
  }
}
template <typename T>
__global__ void from_f32_kernel(T* dst, const float* src, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    dst[i] = fromf<T>(src[i]);
}

template <typename T>
__global__ void pack_bias_kernel(float* dst, const T* a, const T* b, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    dst[i] = tof<T>(a[i]) + (b ? tof<T>(b[i]) : 0.0f);
}

static int elem_size(int dtype) { return dtype == CC2_BF16 ? 2 : 4; }

template <typename T>
static int pack_matrix_t(void* dst, int ldd, const void* src, int rows, int cols, const void* colscale,
                         cudaStream_t st) {
  CC2_REQUIRE(src != nullptr, "pack: null weight pointer");
  pack_matrix_kernel<T><<<std::min(4096, (rows * cols + 255) / 256), 256, 0, st>>>(
      (T*)dst, ldd, (const T*)src, rows, cols, (const T*)colscale);
  CC2_CHECK_LAUNCH();
  return CC2_OK;
}
static int pack_matrix(int dtype, void* dst, int ldd, const void* src, int rows, int cols, const void* colscale,
                       cudaStream_t st) {
  return dtype == CC2_BF16 ? pack_matrix_t<__nv_bfloat16>(dst, ldd, src, rows, cols, colscale, st)
                           : pack_matrix_t<float>(dst, ldd, src, rows, cols, colscale, st);
}
// dst (dtype, d x d) = Wo . (Wv * ln)  -- the group block of a one-series group
// as a single projection; the product is formed in fp32 and rounded once.
static int pack_wov(int dtype, void* dst, const void* wo, const void* wv, const void* ln, int d, float* tmp,
                    cudaStream_t st) {
  CC2_REQUIRE(wo && wv && ln, "pack: null group weight");
  float* wo32 = tmp;
  float* wvt32 = tmp + (size_t)d * d;
  float* out32 = tmp + 2 * (size_t)d * d;
  const int blocks = std::min(4096, (d * d + 255) / 256);
  if (dtype == CC2_BF16) {
    to_f32_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(wo32, (const __nv_bfloat16*)wo, d, d, nullptr, 0);
    to_f32_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(wvt32, (const __nv_bfloat16*)wv, d, d,
                                                         (const __nv_bfloat16*)ln, 1);
  } else {
    to_f32_kernel<float><<<blocks, 256, 0, st>>>(wo32, (const float*)wo, d, d, nullptr, 0);
    to_f32_kernel<float><<<blocks, 256, 0, st>>>(wvt32, (const float*)wv, d, d, (const float*)ln, 1);
  }
  CC2_CHECK_LAUNCH();
  // out[n][k] = sum_j Wo[n][j] * WvT[k][j]
  CC2_TRY(launch_gemm_f32(wo32, d, wvt32, d, out32, d, d, d, d, nullptr, st));
  if (dtype == CC2_BF16)
    from_f32_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>((__nv_bfloat16*)dst, out32, (size_t)d * d);
  else
    from_f32_kernel<float><<<blocks, 256, 0, st>>>((float*)dst, out32, (size_t)d * d);
  CC2_CHECK_LAUNCH();
  return CC2_OK;
}

static int pack_bias(int dtype, float* dst, const void* a, const void* b, int n, cudaStream_t st) {
  CC2_REQUIRE(a != nullptr, "pack: null bias pointer");
  if (dtype == CC2_BF16)
    pack_bias_kernel<__nv_bfloat16><<<(n + 255) / 256, 256, 0, st>>>(dst, (const __nv_bfloat16*)a,
                                                                     (const __nv_bfloat16*)b, n);
  else
    pack_bias_kernel<float><<<(n + 255) / 256, 256, 0, st>>>(dst, (const float*)a, (const float*)b, n);
  CC2_CHECK_LAUNCH();
  return CC2_OK;
}

// ---- launch profiling ---------------------------------------------------------------
struct ProfRecord {
  int kind;
  double flops, bytes;
};
struct Profiler {
  bool on = false;
  int cap = 0;
  std::vector<cudaEvent_t> ev;
  std::vector<ProfRecord> rec;
};
static thread_local Profiler t_prof;

// Brackets one launch with events when profiling is on.
struct ProfScope {
  cudaStream_t st;
  bool active;
  ProfScope(int kind, double flops, double bytes, cudaStream_t s) : st(s), active(false) {
    Profiler& p = t_prof;
    if (!p.on || (int)p.rec.size() >= p.cap) return;
    const size_t i = p.rec.size();
    p.rec.push_back({kind, flops, bytes});
    cudaEventRecord(p.ev[2 * i], st);
    active = true;
  }
  ~ProfScope() {
    if (active) cudaEventRecord(t_prof.ev[2 * (t_prof.rec.size() - 1) + 1], st);
  }
};

}  // namespace cc2

using namespace cc2;

// ---- model handle ---------------------------------------------------------------
struct cc2_layer_pack {
  void* wqkv_t; void* wo_t; void* wqkv_g; void* wo_g; void* wi; void* wo_f;
  void* wov_g;  // Wo_g . diag-free (Wv_g * ln_g): the whole group block for groups of one series
};

struct cc2_model {
  cc2_config cfg;
  int dtype;
  int esz;
  int in_dim;    // 3 * patch
  int kin;       // dff + in_dim (input ResidualBlock fused K)
  int kin_pad;   // kin rounded up to 64
  int kout;      // dff + d (output ResidualBlock fused K)
  int qps;       // num_quantiles * patch
  int max_pos;   // RoPE table rows
  std::vector<cc2_layer_pack> layers;
  void* w1_in; float* b1_in; void* w23_in; float* b23_in; float* reg;
  void* final_ln; void* w1_out; float* b1_out; void* w23_out; float* b23_out;
  float* rope;
  float* pack_tmp;
  uint32_t* rope_bf;  // [pos][d_kv/2] packed (cos, sin) bf16 pairs for the QKV epilogue
  struct KvQuant {
    bool has_k = false, has_v = false;
    cc2_kvq key{}, value{};
    float* stats = nullptr;
  };
  std::vector<KvQuant> kvq;  // per layer: TurboQuant K/V hook of the time attention
};

namespace {

struct Planner {
  size_t off = 0;
  size_t take(size_t bytes) {
    size_t o = off;
    off = align_up(off + bytes, 256);
    return o;
  }
};

int validate_cfg(const cc2_config* c) {
  CC2_REQUIRE(c != nullptr, "config is null");
  CC2_REQUIRE(c->d_kv == 64, "d_kv must be 64 (got %d)", c->d_kv);
  CC2_REQUIRE(c->num_heads * c->d_kv == c->d_model, "num_heads * d_kv must equal d_model");
  CC2_REQUIRE(c->d_model % 64 == 0 && c->d_ff % 64 == 0, "d_model and d_ff must be multiples of 64");
  CC2_REQUIRE(c->input_patch_size == c->output_patch_size && c->input_patch_size > 0,
              "input and output patch sizes must match");
  CC2_REQUIRE(c->num_layers > 0 && c->num_quantiles > 0 && c->context_length > 0, "bad config sizes");
  CC2_REQUIRE((c->num_quantiles * c->output_patch_size) % 16 == 0,
              "num_quantiles * output_patch_size must be a multiple of 16");
  CC2_REQUIRE((3 * c->input_patch_size) % 8 == 0, "3 * patch size must be a multiple of 8");
  CC2_REQUIRE(c->max_output_patches > 0, "max_output_patches must be positive");
  CC2_REQUIRE(c->time_encoding_scale != 0.0f, "time_encoding_scale must be non-zero");
  return CC2_OK;
}

// Layout of the packed weight buffer (offsets in bytes); fills `m` pointers when base != null.
size_t plan_pack(const cc2_config& c, int dtype, cc2_model* m, char* base) {
  const size_t e = elem_size(dtype);
  const int d = c.d_model, dff = c.d_ff, in = 3 * c.input_patch_size;
  const int kin_pad = (int)align_up(dff + in, 64);
  const int qps = c.num_quantiles * c.output_patch_size;
  const int max_pos = (c.context_length + c.input_patch_size - 1) / c.input_patch_size + 1 + c.max_output_patches;
  Planner p;
  std::vector<size_t> lo;
  for (int l = 0; l < c.num_layers; ++l) {
    lo.push_back(p.take(e * 3 * d * d));
    lo.push_back(p.take(e * d * d));
    lo.push_back(p.take(e * 3 * d * d));
    lo.push_back(p.take(e * d * d));
    lo.push_back(p.take(e * (size_t)dff * d));
    lo.push_back(p.take(e * (size_t)d * dff));
    lo.push_back(p.take(e * (size_t)d * d));
  }
  size_t o_w1_in = p.take(e * (size_t)dff * in), o_b1_in = p.take(4 * dff);
  size_t o_w23_in = p.take(e * (size_t)d * kin_pad), o_b23_in = p.take(4 * d), o_reg = p.take(4 * d);
  size_t o_fln = p.take(e * d), o_w1_out = p.take(e * (size_t)dff * d), o_b1_out = p.take(4 * dff);
  size_t o_w23_out = p.take(e * (size_t)qps * (dff + d)), o_b23_out = p.take(4 * qps);
  size_t o_rope = p.take(sizeof(float) * 2 * (size_t)max_pos * (c.d_kv / 2));
  size_t o_tmp = p.take(sizeof(float) * 3 * (size_t)d * d);  // fp32 scratch used only while packing
  size_t o_rope_bf = p.take(sizeof(uint32_t) * (size_t)max_pos * (c.d_kv / 2));
  if (m && base) {
    m->layers.resize(c.num_layers);
    for (int l = 0; l < c.num_layers; ++l) {
      cc2_layer_pack& L = m->layers[l];
      L.wqkv_t = base + lo[7 * l + 0]; L.wo_t = base + lo[7 * l + 1];
      L.wqkv_g = base + lo[7 * l + 2]; L.wo_g = base + lo[7 * l + 3];
      L.wi = base + lo[7 * l + 4]; L.wo_f = base + lo[7 * l + 5]; L.wov_g = base + lo[7 * l + 6];
    }
    m->w1_in = base + o_w1_in; m->b1_in = (float*)(base + o_b1_in);
    m->w23_in = base + o_w23_in; m->b23_in = (float*)(base + o_b23_in); m->reg = (float*)(base + o_reg);
    m->final_ln = base + o_fln; m->w1_out = base + o_w1_out; m->b1_out = (float*)(base + o_b1_out);
    m->w23_out = base + o_w23_out; m->b23_out = (float*)(base + o_b23_out); m->rope = (float*)(base + o_rope);
    m->pack_tmp = (float*)(base + o_tmp);
    m->rope_bf = (uint32_t*)(base + o_rope_bf);
    m->in_dim = in; m->kin = dff + in; m->kin_pad = kin_pad; m->kout = dff + d; m->qps = qps; m->max_pos = max_pos;
  }
  return p.off;
}

struct Workspace {
  char* E; char* X; char* QKV; char* ATT; float* ssq; uint8_t* tok; float* loc; float* scale;
  char* XLO; char* ALO;  // bf16: low halves of the residual stream X and of its alternate buffer ATT
  int32_t* members; int32_t* offsets; char* O; char* PRED;
  float* splitk; size_t splitk_floats;  // fp32 mode: K-slice partial sums of the small-M GEMMs
  char* chain; size_t chain_bytes;      // layer-persistent forward: barrier, split-K counters and partials
};

size_t plan_ws(const cc2_model& m, int B, int L, int N, Workspace* w, char* base) {
  const cc2_config& c = m.cfg;
  const size_t e = m.esz;
  const int Leff = std::min(L, c.context_length);
  const int P = (Leff + c.input_patch_size - 1) / c.input_patch_size;
  const int S = P + (c.use_reg_token ? 1 : 0) + N;
  const size_t M = (size_t)B * S;
  const int d = c.d_model, dff = c.d_ff;
  const int KE = std::max(m.kin_pad, dff);
  Planner p;
  size_t oE = p.take(e * M * KE), oX = p.take(e * M * d), oQKV = p.take(e * M * 3 * d), oATT = p.take(e * M * d);
  const size_t groups = (size_t)(d + 63) / 64;  // 64-column partial sums of squares
  size_t oSSQ = p.take(4 * M * groups * 2), oTOK = p.take(M);
  size_t oLOC = p.take(4 * B), oSC = p.take(4 * B), oMEM = p.take(4 * B), oOFF = p.take(4 * (B + 1));
  size_t oO = p.take(e * (size_t)B * N * m.kout), oPRED = p.take(e * (size_t)B * N * m.qps);
  const size_t splitk_floats = m.dtype == CC2_F32 ? gemm_f32_splitk_floats() : 0;
  size_t oSPLIT = p.take(4 * splitk_floats);
  const size_t lo_bytes = m.dtype == CC2_BF16 ? e * align_up(M, 32) * d : 0;  // 32-row interleaved
  size_t oXLO = p.take(lo_bytes), oALO = p.take(lo_bytes);
  // the layer-persistent forward's scratch, for the forwards that may use it
  const size_t chain_bytes = (m.dtype == CC2_BF16 && M <= (size_t)kChainMaxRows) ? chain_scratch_bytes() : 0;
  size_t oCHAIN = p.take(chain_bytes);
  if (w && base) {
    w->E = base + oE; w->X = base + oX; w->QKV = base + oQKV; w->ATT = base + oATT;
    w->ssq = (float*)(base + oSSQ); w->tok = (uint8_t*)(base + oTOK);
    w->loc = (float*)(base + oLOC); w->scale = (float*)(base + oSC);
    w->members = (int32_t*)(base + oMEM); w->offsets = (int32_t*)(base + oOFF);
    w->O = base + oO; w->PRED = base + oPRED;
    w->splitk = (float*)(base + oSPLIT); w->splitk_floats = splitk_floats;
    w->XLO = lo_bytes ? base + oXLO : nullptr; w->ALO = lo_bytes ? base + oALO : nullptr;
    w->chain = chain_bytes ? base + oCHAIN : nullptr;
    w->chain_bytes = chain_bytes;
  }
  return p.off;
}

// fp32 split-K scratch of the forward being issued on this thread (null outside a forward)
thread_local int t_gemm_kind = CC2_K_GEMM;  // profiler kind of the next gemm() on this thread
thread_local float* t_splitk = nullptr;
thread_local size_t t_splitk_floats = 0;
thread_local bool t_chain_rec = false;  // gemm() records a stage of the layer-persistent forward

int gemm(int dtype, const void* A, int lda, const void* W, int ldw, void* out, int ldo, int M, int N, int K,
         const cc2_epilogue* e, cudaStream_t st) {
  if (t_chain_rec) {
    t_gemm_kind = CC2_K_GEMM;
    return chain_add_gemm(A, lda, W, ldw, out, ldo, M, N, K, e);
  }
  ProfScope ps_(t_gemm_kind, 2.0 * M * N * K, 0.0, st);
  t_gemm_kind = CC2_K_GEMM;
  if (dtype == CC2_BF16) return launch_gemm_tc(A, lda, W, ldw, out, ldo, M, N, K, e, st);
  return launch_gemm_f32(A, lda, W, ldw, out, ldo, M, N, K, e, st, t_splitk, t_splitk_floats);
}

// Records the layers' GEMMs and time attentions as stages of one
// layer-persistent launch for its lifetime.
struct ChainScope {
  bool on;
  explicit ChainScope(bool enable, int M) : on(enable && chain_begin(M) == CC2_OK) { t_chain_rec = on; }
  ~ChainScope() {
    if (on) chain_abandon();
    t_chain_rec = false;
  }
  int launch(void* scratch, size_t bytes, double flops, cudaStream_t st) {
    t_chain_rec = false;
    on = false;
    ProfScope ps_(CC2_K_LAYERS, flops, 0.0, st);
    return chain_launch(scratch, bytes, g_layer_chain == 2, st);
  }
};

struct SplitKScope {
  SplitKScope(float* p, size_t n) { t_splitk = p; t_splitk_floats = n; }
  ~SplitKScope() { t_splitk = nullptr; t_splitk_floats = 0; }
};

// The forward's GEMMs read only the packed model weights as W.
struct WeightsConstScope {
  WeightsConstScope() { set_gemm_weights_const(true); }
  ~WeightsConstScope() { set_gemm_weights_const(false); }
};

cc2_epilogue epi(int flags) {
  cc2_epilogue e;
  std::memset(&e, 0, sizeof(e));
  e.flags = flags;
  return e;
}

cc2_epilogue epi_m(int flags, int M) {
  cc2_epilogue e = epi(flags);
  e.ssq_ld = M;
  return e;
}

}  // namespace

extern "C" {

const char* cc2_last_error(void) { return t_error.c_str(); }
const char* cc2_version(void) { return "cc2-b200 0.1 (sm_100a)"; }

int cc2_device_status(int clear) {
  clear_error();
  CC2_CUDA(cudaDeviceSynchronize());
  int v = 0, a = 0;
  CC2_TRY(read_device_error(clear, &v));
  CC2_TRY(read_attention_error(clear, &a));
  return v | (a ? DEV_ERR_ATTN_TIMEOUT : 0);
}

int cc2_model_pack_bytes(const cc2_config* cfg, int dtype, size_t* bytes) {
  clear_error();
  CC2_TRY(validate_cfg(cfg));
  CC2_REQUIRE(dtype == CC2_BF16 || dtype == CC2_F32, "unsupported dtype %d", dtype);
  CC2_REQUIRE(bytes != nullptr, "bytes is null");
  *bytes = plan_pack(*cfg, dtype, nullptr, nullptr);
  return CC2_OK;
}

int cc2_model_create(const cc2_config* cfg, int dtype, const cc2_weights* w, void* pack_buf, size_t pack_bytes,
                     void* stream, cc2_model** out) {
  clear_error();
  CC2_TRY(validate_cfg(cfg));
  CC2_REQUIRE(dtype == CC2_BF16 || dtype == CC2_F32, "unsupported dtype %d", dtype);
  CC2_REQUIRE(w && pack_buf && out, "null argument");
  CC2_REQUIRE(((uintptr_t)pack_buf & 255u) == 0, "pack buffer must be 256-byte aligned");
  const size_t need = plan_pack(*cfg, dtype, nullptr, nullptr);
  if (pack_bytes < need) {
    set_error("pack buffer too small: %zu < %zu", pack_bytes, need);
    return CC2_E_WORKSPACE;
  }
  cudaStream_t st = (cudaStream_t)stream;
  cc2_model* m = new cc2_model();
  m->cfg = *cfg;
  m->dtype = dtype;
  m->esz = elem_size(dtype);
  plan_pack(*cfg, dtype, m, (char*)pack_buf);
  const cc2_config& c = *cfg;
  const int d = c.d_model, dff = c.d_ff, in = m->in_dim;
  const size_t e = m->esz;
  auto fail = [&](int s) { delete m; return s; };
  int s = CC2_OK;
#define PK(expr) do { s = (expr); if (s != CC2_OK) return fail(s); } while (0)
  for (int l = 0; l < c.num_layers; ++l) {
    cc2_layer_pack& L = m->layers[l];
    CC2_REQUIRE(w->time_q && w->time_k && w->time_v && w->time_o && w->time_ln && w->group_q && w->group_k &&
                    w->group_v && w->group_o && w->group_ln && w->ff_ln && w->ff_wi && w->ff_wo,
                "per-layer weight arrays must be non-null");
    PK(pack_matrix(dtype, L.wqkv_t, d, w->time_q[l], d, d, w->time_ln[l], st));
    PK(pack_matrix(dtype, (char*)L.wqkv_t + e * d * d, d, w->time_k[l], d, d, w->time_ln[l], st));
    PK(pack_matrix(dtype, (char*)L.wqkv_t + 2 * e * d * d, d, w->time_v[l], d, d, w->time_ln[l], st));
    PK(pack_matrix(dtype, L.wo_t, d, w->time_o[l], d, d, nullptr, st));
    PK(pack_matrix(dtype, L.wqkv_g, d, w->group_q[l], d, d, w->group_ln[l], st));
    PK(pack_matrix(dtype, (char*)L.wqkv_g + e * d * d, d, w->group_k[l], d, d, w->group_ln[l], st));
    PK(pack_matrix(dtype, (char*)L.wqkv_g + 2 * e * d * d, d, w->group_v[l], d, d, w->group_ln[l], st));
    PK(pack_matrix(dtype, L.wo_g, d, w->group_o[l], d, d, nullptr, st));
    PK(pack_wov(dtype, L.wov_g, w->group_o[l], w->group_v[l], w->group_ln[l], d, m->pack_tmp, st));
    PK(pack_matrix(dtype, L.wi, d, w->ff_wi[l], dff, d, w->ff_ln[l], st));
    PK(pack_matrix(dtype, L.wo_f, dff, w->ff_wo[l], d, dff, nullptr, st));
  }
  PK(pack_matrix(dtype, m->w1_in, in, w->in_hidden_w, dff, in, nullptr, st));
  PK(pack_bias(dtype, m->b1_in, w->in_hidden_b, nullptr, dff, st));
  if (cudaMemsetAsync(m->w23_in, 0, e * (size_t)d * m->kin_pad, st) != cudaSuccess) {
    set_error("memset failed");
    return fail(CC2_E_CUDA);
  }
  PK(pack_matrix(dtype, m->w23_in, m->kin_pad, w->in_output_w, d, dff, nullptr, st));
  PK(pack_matrix(dtype, (char*)m->w23_in + e * dff, m->kin_pad, w->in_residual_w, d, in, nullptr, st));
  PK(pack_bias(dtype, m->b23_in, w->in_output_b, w->in_residual_b, d, st));
  CC2_REQUIRE(w->shared != nullptr, "shared embedding is null");
  PK(pack_bias(dtype, m->reg, (const char*)w->shared + e * (size_t)c.reg_token_id * d, nullptr, d, st));
  PK(pack_matrix(dtype, m->final_ln, d, w->final_ln, 1, d, nullptr, st));
  PK(pack_matrix(dtype, m->w1_out, d, w->out_hidden_w, dff, d, nullptr, st));
  PK(pack_bias(dtype, m->b1_out, w->out_hidden_b, nullptr, dff, st));
  PK(pack_matrix(dtype, m->w23_out, m->kout, w->out_output_w, m->qps, dff, nullptr, st));
  PK(pack_matrix(dtype, (char*)m->w23_out + e * dff, m->kout, w->out_residual_w, m->qps, d, nullptr, st));
  PK(pack_bias(dtype, m->b23_out, w->out_output_b, w->out_residual_b, m->qps, st));
#undef PK
  // RoPE table: inv_freq = 1 / theta^(2i/d_kv) and freq = inv_freq * pos in fp32
  // as in model.py:200-203 / 94-109; cos/sin of the fp32 angle.
  const int half = c.d_kv / 2;
  std::vector<float> tab((size_t)m->max_pos * half * 2);
  for (int i = 0; i < half; ++i) {
    const float expo = (float)(2 * i) / (float)c.d_kv;
    const float inv = 1.0f / std::pow(c.rope_theta, expo);
    for (int pos = 0; pos < m->max_pos; ++pos) {
      const float f = inv * (float)pos;
      tab[((size_t)pos * half + i) * 2 + 0] = (float)std::cos((double)f);
      tab[((size_t)pos * half + i) * 2 + 1] = (float)std::sin((double)f);
    }
  }
  // bf16 copy (round to nearest even) packed as cos | sin << 16
  std::vector<uint32_t> tab_bf(tab.size() / 2);
  auto to_bf = [](float f) -> uint32_t {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return u >> 16;
  };
  for (size_t i = 0; i < tab_bf.size(); ++i) tab_bf[i] = to_bf(tab[2 * i]) | (to_bf(tab[2 * i + 1]) << 16);
  if (cudaMemcpyAsync(m->rope_bf, tab_bf.data(), tab_bf.size() * sizeof(uint32_t), cudaMemcpyHostToDevice, st) !=
          cudaSuccess ||
      cudaMemcpyAsync(m->rope, tab.data(), tab.size() * sizeof(float), cudaMemcpyHostToDevice, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess) {
    set_error("uploading the RoPE table failed");
    return fail(CC2_E_CUDA);
  }
  *out = m;
  return CC2_OK;
}

int cc2_model_destroy(cc2_model* m) {
  delete m;
  return CC2_OK;
}

int cc2_group_layout(const int64_t* gid, int B, int32_t* members, int32_t* offsets, int* num_groups,
                     int* max_group) {
  clear_error();
  CC2_REQUIRE(gid && members && offsets && num_groups && max_group && B > 0, "group_layout: bad args");
  std::unordered_map<int64_t, int> index;
  std::vector<std::vector<int>> groups;
  for (int b = 0; b < B; ++b) {
    auto it = index.find(gid[b]);
    if (it == index.end()) {
      index.emplace(gid[b], (int)groups.size());
      groups.push_back({b});
    } else {
      groups[it->second].push_back(b);
    }
  }
  int k = 0, mg = 0;
  offsets[0] = 0;
  for (size_t g = 0; g < groups.size(); ++g) {
    for (int b : groups[g]) members[k++] = b;
    offsets[g + 1] = k;
    mg = std::max(mg, (int)groups[g].size());
  }
  *num_groups = (int)groups.size();
  *max_group = mg;
  return CC2_OK;
}

int cc2_forward_workspace_bytes(const cc2_model* m, int B, int L, int N, int max_group, size_t* bytes) {
  clear_error();
  CC2_REQUIRE(m && bytes && B > 0 && L > 0 && N > 0 && max_group > 0, "workspace_bytes: bad args");
  *bytes = plan_ws(*m, B, L, N, nullptr, nullptr);
  return CC2_OK;
}

int cc2_forward(const cc2_model* m, const float* context, const float* context_mask, int B, int L, int N,
                const int64_t* group_ids, void* out, float* loc, float* scale, void* workspace, size_t ws_bytes,
                void* stream) {
  clear_error();
  CC2_REQUIRE(m && context && out && workspace, "forward: null argument");
  CC2_REQUIRE(B > 0 && L > 0, "forward: B and L must be positive");
  CC2_REQUIRE(N > 0 && N <= m->cfg.max_output_patches, "forward: N must be in [1, %d]", m->cfg.max_output_patches);
  CC2_REQUIRE(((uintptr_t)workspace & 255u) == 0, "workspace must be 256-byte aligned");
  const cc2_config& c = m->cfg;
  cudaStream_t st = (cudaStream_t)stream;
  const LaunchOverlapScope overlap(m->dtype == CC2_BF16 ? 1 : 0);
  const size_t need = plan_ws(*m, B, L, N, nullptr, nullptr);
  if (ws_bytes < need) {
    set_error("workspace too small: %zu < %zu", ws_bytes, need);
    return CC2_E_WORKSPACE;
  }
  Workspace w;
  plan_ws(*m, B, L, N, &w, (char*)workspace);
  SplitKScope splitk_scope(w.splitk, w.splitk_floats);
  const WeightsConstScope weights_const;
  const int dt = m->dtype;
  const size_t e = m->esz;
  const int d = c.d_model, dff = c.d_ff, ps = c.input_patch_size;
  const int Leff = std::min(L, c.context_length);
  const int P = (Leff + ps - 1) / ps;
  const int reg = c.use_reg_token ? 1 : 0;
  const int S = P + reg + N;
  CC2_REQUIRE(S <= m->max_pos, "forward: sequence of %d tokens exceeds the RoPE table (%d)", S, m->max_pos);
  const int M = B * S;
  const int KE = std::max(m->kin_pad, dff);
  const float eps = c.layer_norm_epsilon;
  // bf16: the residual stream is kept as bf16 high halves (what the GEMMs
  // read) plus bf16 low halves, so the twelve layers' residual additions do
  // not each round it to 8 significant bits
  const bool lo = dt == CC2_BF16;

  // group structure
  int num_groups = B, max_group = 1;
  int contig_g = 0;  // > 0: every group is a run of contig_g consecutive series (the tcgen05 group kernel)
  double gsq = (double)B;  // sum over groups of size^2 (attention FLOP count)
  if (group_ids) {
    std::vector<int32_t> mem(B), off(B + 1);
    CC2_TRY(cc2_group_layout(group_ids, B, mem.data(), off.data(), &num_groups, &max_group));
    gsq = 0.0;
    for (int g = 0; g < num_groups; ++g) gsq += (double)(off[g + 1] - off[g]) * (off[g + 1] - off[g]);
    contig_g = max_group;
    for (int g = 0; g < num_groups && contig_g; ++g)
      if (off[g + 1] - off[g] != max_group) contig_g = 0;
    for (int i = 0; i < B && contig_g; ++i)
      if (mem[i] != i) contig_g = 0;
    if (max_group > 1) {
      CC2_CUDA(cudaMemcpyAsync(w.members, mem.data(), sizeof(int32_t) * B, cudaMemcpyHostToDevice, st));
      CC2_CUDA(cudaMemcpyAsync(w.offsets, off.data(), sizeof(int32_t) * (num_groups + 1), cudaMemcpyHostToDevice, st));
    }
  }
  float* locp = loc ? loc : w.loc;
  float* scp = scale ? scale : w.scale;
  // RMS statistics: norm i's partial sums live in buffer i % 2 (its producer
  // runs after the consumer of norm i-2 in stream order).
  const size_t groups = (size_t)(d + 63) / 64;
  auto ssq = [&](int i) { return w.ssq + (size_t)(i & 1) * groups * M; };

  // preprocessing -> E[:, dff : dff + 3ps] (+ zero pad up to kin_pad)
  {
  ProfScope ps_(CC2_K_PREPROCESS, 0.0, (double)B * (4.0 * Leff + e * 3 * ps * P + P + 8), st);
  CC2_TRY(launch_preprocess(context, context_mask, B, L, ps, c.context_length, c.time_encoding_scale,
                            c.use_arcsinh, reg, N, dt, w.E + e * dff, m->kin_pad, m->kin_pad - dff, w.tok, nullptr,
                            locp, scp, st));
  }
  // input ResidualBlock
  {
    cc2_epilogue e1 = epi_m(CC2_EPI_BIAS | CC2_EPI_RELU, M);
    e1.bias = m->b1_in;
    t_gemm_kind = CC2_K_GEMM_IO;
    CC2_TRY(gemm(dt, w.E + e * dff, m->kin_pad, m->w1_in, m->in_dim, w.E, m->kin_pad, M, dff, m->in_dim, &e1, st));
    cc2_epilogue e2 = epi_m(CC2_EPI_BIAS | CC2_EPI_SSQ | (reg ? CC2_EPI_SPECIAL : 0), M);
    e2.bias = m->b23_in;
    e2.ssq_out = ssq(0);
    e2.special = m->reg;
    e2.special_period = S;
    e2.special_offset = P;
    if (lo) { e2.flags |= CC2_EPI_LO; e2.lo_out = w.XLO; e2.ld_lo = d; }
    t_gemm_kind = CC2_K_GEMM_IO;
    CC2_TRY(gemm(dt, w.E, m->kin_pad, m->w23_in, m->kin_pad, w.X, d, M, d, m->kin_pad, &e2, st));
  }
  // residual stream X and scratch Y swap roles after a one-GEMM group block
  // (with their low halves XL / YL in bf16 mode)
  char* X = w.X;
  char* Y = w.ATT;
  char* XL = w.XLO;
  char* YL = w.ALO;
  auto with_lo = [&](cc2_epilogue& ep, char* resid_lo, char* out_lo) {
    if (!lo) return;
    ep.flags |= CC2_EPI_LO; ep.resid_lo = resid_lo; ep.lo_out = out_lo; ep.ld_lo = d;
  };
  // Few token rows (batch-1 serving): the layers' GEMMs and time attentions
  // are recorded as stages and run as one layer-persistent launch.
  bool kvq_on = false;
  for (const auto& q : m->kvq) kvq_on = kvq_on || q.has_k || q.has_v;
  const bool chain = lo && g_layer_chain && g_gemm_variant == 0 && max_group == 1 && !kvq_on && c.d_kv == 64 &&
                     M <= kChainMaxRows && w.chain && S <= chain_max_set() &&
                     6 * c.num_layers <= chain_max_stages();
  ChainScope chain_scope(chain, M);
  for (int l = 0; l < c.num_layers; ++l) {
    const cc2_layer_pack& Lw = m->layers[l];
    // time attention
    // bf16: RoPE is applied to Q and K in the QKV epilogue (position = row % S);
    // fp32: inside the attention kernel
    const bool rope_in_gemm = dt == CC2_BF16;
    cc2_epilogue a = epi_m(CC2_EPI_ROWSCALE | (rope_in_gemm ? CC2_EPI_ROPE : 0), M);
    a.ssq_in = ssq(3 * l); a.norm_dim = d; a.eps = eps;
    a.rope_cs = m->rope_bf; a.rope_period = S; a.rope_cols = 2 * d;
    t_gemm_kind = CC2_K_GEMM_QKV;
    CC2_TRY(gemm(dt, X, d, Lw.wqkv_t, d, w.QKV, 3 * d, M, 3 * d, d, &a, st));
    // TurboQuant K/V hook: K and V replaced by their quantised reconstructions
    // after RoPE (applied here first in fp32, where the attention would)
    bool rope_done = rope_in_gemm;
    if (l < (int)m->kvq.size() && (m->kvq[l].has_k || m->kvq[l].has_v)) {
      const cc2_model::KvQuant& q = m->kvq[l];
      CC2_TRY(launch_kv_quant(dt, w.QKV, 3 * d, M, 0, d, 2 * d, c.num_heads, q.has_k ? &q.key : nullptr,
                              q.has_v ? &q.value : nullptr, rope_done ? nullptr : m->rope, S, q.stats, st));
      rope_done = true;
    }
    if (t_chain_rec) {
      CC2_TRY(chain_add_attention(w.QKV, 3 * d, 0, d, 2 * d, Y, d, w.tok, B, S, c.num_heads));
    } else {
      ProfScope ps_(CC2_K_ATTN_TIME, 4.0 * B * (double)S * S * d, 0.0, st);
      CC2_TRY(launch_attention(dt, 0, w.QKV, 3 * d, 0, d, 2 * d, Y, d, w.tok, B, S, c.num_heads, c.d_kv,
                               nullptr, nullptr, 0, 0, rope_done ? nullptr : m->rope, st));
    }
    cc2_epilogue o = epi_m(CC2_EPI_RESID | CC2_EPI_SSQ, M);
    o.resid = X; o.ld_resid = d; o.ssq_out = ssq(3 * l + 1);
    with_lo(o, XL, XL);
    t_gemm_kind = CC2_K_GEMM_O;
    CC2_TRY(gemm(dt, Y, d, Lw.wo_t, d, X, d, M, d, d, &o, st));
    // group attention
    cc2_epilogue g = epi_m(CC2_EPI_ROWSCALE, M);
    g.ssq_in = ssq(3 * l + 1); g.norm_dim = d; g.eps = eps;
    if (max_group == 1) {
      // softmax over a single unmasked key is exactly 1, so the block is
      // X + Wo (Wv norm(X)): one GEMM with the pre-multiplied Wo.Wv.  It
      // writes the other residual buffer (A and the output must differ).
      g.flags |= CC2_EPI_RESID | CC2_EPI_SSQ;
      g.resid = X; g.ld_resid = d; g.ssq_out = ssq(3 * l + 2);
      with_lo(g, XL, YL);
      t_gemm_kind = CC2_K_GEMM_GROUP;
      CC2_TRY(gemm(dt, X, d, Lw.wov_g, d, Y, d, M, d, d, &g, st));
      std::swap(X, Y);
      std::swap(XL, YL);
    } else {
      t_gemm_kind = CC2_K_GEMM_GROUP;
      CC2_TRY(gemm(dt, X, d, Lw.wqkv_g, d, w.QKV, 3 * d, M, 3 * d, d, &g, st));
      {
        ProfScope ps_(CC2_K_ATTN_GROUP, 4.0 * (double)S * gsq * d, 0.0, st);
        if (dt == CC2_BF16 && g_attn_variant == 0 && contig_g > 1 && c.d_kv == 64 &&
            attn_group_tc_supported(contig_g, 3 * d, d, w.QKV, Y)) {
          int* err = nullptr;
          CC2_TRY(attention_error_word(&err));
          CC2_TRY(launch_attn_group_tc(w.QKV, 3 * d, 0, d, 2 * d, Y, d, w.tok, B, S, c.num_heads, contig_g, err, st));
        } else {
          CC2_TRY(launch_attention(dt, 1, w.QKV, 3 * d, 0, d, 2 * d, Y, d, w.tok, S * num_groups, S, c.num_heads,
                                   c.d_kv, w.members, w.offsets, num_groups, max_group, nullptr, st));
        }
      }
      cc2_epilogue og = epi_m(CC2_EPI_RESID | CC2_EPI_SSQ, M);
      og.resid = X; og.ld_resid = d; og.ssq_out = ssq(3 * l + 2);
      with_lo(og, XL, XL);
      t_gemm_kind = CC2_K_GEMM_GROUP;
      CC2_TRY(gemm(dt, Y, d, Lw.wo_g, d, X, d, M, d, d, &og, st));
    }
    // feed-forward
    cc2_epilogue f1 = epi_m(CC2_EPI_ROWSCALE | CC2_EPI_RELU, M);
    f1.ssq_in = ssq(3 * l + 2); f1.norm_dim = d; f1.eps = eps;
    t_gemm_kind = CC2_K_GEMM_FFN_UP;
    CC2_TRY(gemm(dt, X, d, Lw.wi, d, w.E, dff, M, dff, d, &f1, st));
    cc2_epilogue f2 = epi_m(CC2_EPI_RESID | CC2_EPI_SSQ, M);
    f2.resid = X; f2.ld_resid = d; f2.ssq_out = ssq(3 * l + 3);
    with_lo(f2, XL, XL);
    t_gemm_kind = CC2_K_GEMM_FFN_DOWN;
    CC2_TRY(gemm(dt, w.E, dff, Lw.wo_f, dff, X, d, M, d, dff, &f2, st));
  }
  if (chain_scope.on) {
    const double per_layer = 2.0 * M * (5.0 * d * d + 2.0 * d * dff) + 4.0 * B * (double)S * S * d;
    CC2_TRY(chain_scope.launch(w.chain, w.chain_bytes, per_layer * c.num_layers, st));
  }
  (void)KE;
  // final RMSNorm of the N future rows -> O[:, dff:]
  const int BN_rows = B * N;
  {
    ProfScope ps_(CC2_K_RMSNORM, 0.0, 2.0 * e * BN_rows * d, st);
    CC2_TRY(launch_rmsnorm_rows(dt, X, d, m->final_ln, w.O + e * dff, m->kout, BN_rows, d, N, S, S - N, eps, st));
  }
  // output ResidualBlock
  {
    cc2_epilogue e1 = epi_m(CC2_EPI_BIAS | CC2_EPI_RELU, M);
    e1.bias = m->b1_out;
    t_gemm_kind = CC2_K_GEMM_IO;
    CC2_TRY(gemm(dt, w.O + e * dff, m->kout, m->w1_out, d, w.O, m->kout, BN_rows, dff, d, &e1, st));
    cc2_epilogue e2 = epi_m(CC2_EPI_BIAS, M);
    e2.bias = m->b23_out;
    t_gemm_kind = CC2_K_GEMM_IO;
    CC2_TRY(gemm(dt, w.O, m->kout, m->w23_out, m->kout, w.PRED, m->qps, BN_rows, m->qps, m->kout, &e2, st));
  }
  {
    ProfScope ps_(CC2_K_OUTPUT, 0.0, (double)B * (2.0 * e * m->qps * N + 8), st);
    CC2_TRY(launch_output_transform(dt, w.PRED, m->qps, locp, scp, out, B, N, c.num_quantiles, c.output_patch_size,
                                    c.use_arcsinh, st));
  }
  return CC2_OK;
}

int cc2_profile_begin(int capacity) {
  clear_error();
  CC2_REQUIRE(capacity > 0, "profile capacity must be positive");
  Profiler& p = t_prof;
  for (cudaEvent_t e : p.ev) cudaEventDestroy(e);
  p.ev.assign(2 * (size_t)capacity, nullptr);
  for (auto& e : p.ev) CC2_CUDA(cudaEventCreate(&e));
  p.rec.clear();
  p.rec.reserve(capacity);
  p.cap = capacity;
  p.on = true;
  return CC2_OK;
}

int cc2_profile_read(int* kinds, float* ms, double* flops, double* bytes, int capacity, int* count) {
  clear_error();
  Profiler& p = t_prof;
  p.on = false;
  const int n = (int)p.rec.size();
  if (count) *count = n;
  for (int i = 0; i < n && i < capacity; ++i) {
    CC2_CUDA(cudaEventSynchronize(p.ev[2 * i + 1]));
    float t = 0.0f;
    CC2_CUDA(cudaEventElapsedTime(&t, p.ev[2 * i], p.ev[2 * i + 1]));
    if (kinds) kinds[i] = p.rec[i].kind;
    if (ms) ms[i] = t;
    if (flops) flops[i] = p.rec[i].flops;
    if (bytes) bytes[i] = p.rec[i].bytes;
  }
  for (cudaEvent_t e : p.ev) cudaEventDestroy(e);
  p.ev.clear();
  p.rec.clear();
  return CC2_OK;
}

// ---- forward without a caller-provided workspace ------------------------------------
// Scratch for cc2_forward_noalloc: one static device array per GPU that loads
// the library.  Host code must not pass the symbol itself to a kernel (on the
// host it names a host-side stand-in); the device address comes from
// cudaGetSymbolAddress, looked up once per device with that device current.
static __device__ __align__(256) unsigned char g_noalloc_scratch[CC2_NOALLOC_SCRATCH_BYTES];

static int noalloc_scratch_ptr(void** out) {
  static std::mutex mu;
  static void* addr[64] = {nullptr};
  int dev = 0;
  CC2_CUDA(cudaGetDevice(&dev));
  CC2_REQUIRE(dev >= 0 && dev < 64, "noalloc: device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_error("cudaGetSymbolAddress(scratch) failed on device %d: %s", dev, cudaGetErrorString(e));
      return CC2_E_CUDA;
    }
    addr[dev] = p;
  }
  *out = addr[dev];
  return CC2_OK;
}

// ---- component entry points ---------------------------------------------------------
int cc2_forward_noalloc(const cc2_model* m, const float* context, const float* context_mask, int B, int L, int N,
                        const int64_t* group_ids, void* out, float* loc, float* scale, void* stream) {
  clear_error();
  CC2_REQUIRE(m && context && out, "forward_noalloc: null argument");
  CC2_REQUIRE(B > 0 && L > 0 && N > 0, "forward_noalloc: B, L and N must be positive");
  const size_t need = plan_ws(*m, B, L, N, nullptr, nullptr);
  if (need > CC2_NOALLOC_SCRATCH_BYTES) {
    set_error("forward_noalloc: B=%d L=%d N=%d needs %zu scratch bytes, the static scratch holds %zu; "
              "use cc2_forward with a workspace",
              B, L, N, need, (size_t)CC2_NOALLOC_SCRATCH_BYTES);
    return CC2_E_WORKSPACE;
  }
  void* ws = nullptr;
  CC2_TRY(noalloc_scratch_ptr(&ws));
  return cc2_forward(m, context, context_mask, B, L, N, group_ids, out, loc, scale, ws,
                     (size_t)CC2_NOALLOC_SCRATCH_BYTES, stream);
}

int cc2_preprocess(const float* context, const float* context_mask, int B, int L, int patch_size, int context_length,
                   float te_scale, int use_arcsinh, int use_reg, int N, int dtype, void* patched, int ld_patched,
                   int pad_cols, uint8_t* token_mask, float* attn_mask, float* loc, float* scale, void* stream) {
  clear_error();
  return launch_preprocess(context, context_mask, B, L, patch_size, context_length, te_scale, use_arcsinh, use_reg,
                           N, dtype, patched, ld_patched, pad_cols, token_mask, attn_mask, loc, scale,
                           (cudaStream_t)stream);
}

int cc2_set_gemm_variant(int variant) {
  const int old = g_gemm_variant;
  g_gemm_variant = (variant >= 1 && variant <= 3) ? variant : 0;
  return old;
}

int cc2_set_attention_variant(int variant) {
  const int old = g_attn_variant;
  g_attn_variant = (variant >= 1 && variant <= 3) ? variant : 0;
  return old;
}

int cc2_test_starve_gemm(int on) {
  clear_error();
  return set_gemm_starve(on);
}

int cc2_test_starve_layer_barrier(int on) {
  clear_error();
  return set_chain_starve(on);
}

int cc2_set_layer_chain(int enabled) {
  const int old = g_layer_chain;
  g_layer_chain = (enabled == 1 || enabled == 2) ? enabled : 0;
  return old;
}

int cc2_set_launch_overlap(int enabled) {
  const int old = g_launch_overlap;
  g_launch_overlap = enabled ? 1 : 0;
  return old;
}

int cc2_kv_quant(int dtype, void* qkv, int ld, int rows, int q_col, int k_col, int v_col, int heads,
                 const cc2_kvq* key, const cc2_kvq* value, const float* rope_cs, int rope_period, float* stats,
                 void* stream) {
  clear_error();
  return launch_kv_quant(dtype, qkv, ld, rows, q_col, k_col, v_col, heads, key, value, rope_cs, rope_period, stats,
                         (cudaStream_t)stream);
}

int cc2_model_set_kv_quant(cc2_model* m, int layer, const cc2_kvq* key, const cc2_kvq* value, float* stats) {
  clear_error();
  CC2_REQUIRE(m != nullptr, "cc2_model_set_kv_quant: null model");
  CC2_REQUIRE(layer >= 0 && layer < m->cfg.num_layers, "cc2_model_set_kv_quant: layer %d out of range", layer);
  CC2_REQUIRE(m->cfg.d_kv == 64, "cc2_model_set_kv_quant: the quantiser works on d_kv = 64");
  if (m->kvq.size() < (size_t)m->cfg.num_layers) m->kvq.resize(m->cfg.num_layers);
  cc2_model::KvQuant q;
  q.has_k = key != nullptr;
  q.has_v = value != nullptr;
  if (key) q.key = *key;
  if (value) q.value = *value;
  q.stats = stats;
  m->kvq[layer] = q;
  return CC2_OK;
}

int cc2_set_gemm_trace(void* device_buffer) {
  clear_error();
  return set_gemm_trace(device_buffer);
}

int cc2_set_layer_trace(void* device_buffer) {
  clear_error();
  return set_chain_trace(device_buffer);
}

int cc2_set_attention_trace(void* device_buffer) {
  clear_error();
  CC2_TRY(set_attn_trace(device_buffer));
  return set_attn_long_trace(device_buffer);
}

int cc2_gemm(int dtype, const void* A, int lda, const void* W, int ldw, void* out, int ldo, int M, int N, int K,
             const cc2_epilogue* epi_, void* stream) {
  clear_error();
  CC2_REQUIRE(dtype == CC2_BF16 || dtype == CC2_F32, "gemm: unsupported dtype %d", dtype);
  CC2_REQUIRE(A && W && out, "gemm: null operand");
  return gemm(dtype, A, lda, W, ldw, out, ldo, M, N, K, epi_, (cudaStream_t)stream);
}

int cc2_rmsnorm_rows(int dtype, const void* x, int ld_x, const void* w, void* y, int ld_y, int rows, int dim, int per,
                     int stride, int offset, float eps, void* stream) {
  clear_error();
  return launch_rmsnorm_rows(dtype, x, ld_x, w, y, ld_y, rows, dim, per, stride, offset, eps, (cudaStream_t)stream);
}

int cc2_attention(int dtype, int mode, const void* qkv, int ld_qkv, int q_col, int k_col, int v_col, void* out,
                  int ld_out, const uint8_t* token_mask, int num_sets, int S, int num_heads, int d_kv,
                  const int32_t* members, const int32_t* offsets, int num_groups, int max_group, const float* rope_cs,
                  void* stream) {
  clear_error();
  return launch_attention(dtype, mode, qkv, ld_qkv, q_col, k_col, v_col, out, ld_out, token_mask, num_sets, S,
                          num_heads, d_kv, members, offsets, num_groups, max_group, rope_cs, (cudaStream_t)stream);
}

int cc2_group_attention_tc(const void* qkv, int ld_qkv, int q_col, int k_col, int v_col, void* out, int ld_out,
                           const uint8_t* token_mask, int B, int S, int num_heads, int g, void* stream) {
  clear_error();
  CC2_REQUIRE(qkv && out && token_mask, "group_attention_tc: null pointer");
  CC2_REQUIRE(attn_group_tc_supported(g, ld_qkv, ld_out, qkv, out), "group_attention_tc: unsupported g=%d or alignment", g);
  int* err = nullptr;
  CC2_TRY(attention_error_word(&err));
  return launch_attn_group_tc(qkv, ld_qkv, q_col, k_col, v_col, out, ld_out, token_mask, B, S, num_heads, g, err,
                              (cudaStream_t)stream);
}

int cc2_output_transform(int dtype, const void* preds, int ld_preds, const float* loc, const float* scale, void* out,
                         int B, int N, int Q, int ps, int use_arcsinh, void* stream) {
  clear_error();
  return launch_output_transform(dtype, preds, ld_preds, loc, scale, out, B, N, Q, ps, use_arcsinh,
                                 (cudaStream_t)stream);
}

}  // extern "C"
