/*
 * cc2.h -- C ABI of the B200 (sm_100a) CuteChronos2 encoder engine.
 *
 * Every entry point takes plain pointers, sizes and a CUDA stream (as void*),
 * returns 0 on success or a negative CC2_E* code, and never allocates device
 * memory: the caller owns every buffer (weights pack, workspace, outputs).
 * On error, cc2_last_error() returns a message for the calling thread.
 * Device pointers are marked (dev), host pointers (host).
 *
 * Element types: CC2_F32 (float) or CC2_BF16 (bfloat16, fp32 accumulate).
 * "dtype" buffers hold elements of the model dtype.
 *
 * Reference interfaces these replace (paths inside lee101/cutedsl):
 *   cc2_preprocess        <- cutechronos/cpp/preprocessing.cpp:99-120 (pybind
 *                            fused_preprocess) and model.py:473-549
 *   cc2_output_transform  <- cutechronos/triton_kernels/fused_output.py:83-140
 *                            and model.py:816-829
 *   cc2_gemm              <- F.linear call sites model.py:178-181, 227-229,
 *                            271, 301-303, 308, 328-329; fused RMSNorm+QKV
 *                            kernel_backends.py:168-176; fused MLP
 *                            triton_kernels/fused_mlp.py:254-300
 *   cc2_rmsnorm_rows      <- kernel_backends.py:85-110 (rms_layernorm)
 *   cc2_attention         <- kernel_backends.py:113-153 (unscaled_attention)
 *                            + rope.py:126-180 (apply_rope) for time attention;
 *                            model.py:131-142 via model.py:305 for group attention
 *   cc2_model_* /
 *   cc2_forward           <- CuteChronos2Model.forward, model.py:738-831
 *                            (weights in the layout of load_chronos2_weights,
 *                            model.py:833-900)
 */
#ifndef CC2_H
#define CC2_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define CC2_API __attribute__((visibility("default")))
#else
#define CC2_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum { CC2_F32 = 0, CC2_BF16 = 1 };

enum {
  CC2_OK = 0,
  CC2_E_INVALID = -1,     /* bad argument (shape, null pointer, alignment) */
  CC2_E_CUDA = -2,        /* a CUDA runtime/driver call failed */
  CC2_E_UNSUPPORTED = -3, /* configuration not supported by this build */
  CC2_E_WORKSPACE = -4,   /* workspace or pack buffer too small */
  CC2_E_DEVICE = -5       /* a kernel reported a device-side error (timeout) */
};

/* Message for the last failing call on this thread (empty if none). */
CC2_API const char* cc2_last_error(void);
/* Library version string. */
CC2_API const char* cc2_version(void);
/* Device-side error word written by bounded waits inside kernels (0 = none,
 * else CC2_DEV_* bits); synchronises the current device.  clear != 0 resets
 * it.  A kernel whose wait ran out returns early and leaves its outputs
 * incomplete while the launching call has already returned CC2_OK, so callers
 * that need to know poll this after synchronising (the native bridge and
 * CuteChronos2Model.set_device_checks(True) do). */
enum { CC2_DEV_GEMM_TIMEOUT = 1, CC2_DEV_ATTN_TIMEOUT = 2, CC2_DEV_LAYER_TIMEOUT = 4 };
CC2_API int cc2_device_status(int clear);

/* ------------------------------------------------------------------------ */
/* Model configuration: mirror of CuteChronos2Config (model.py:59-91).       */
/* ------------------------------------------------------------------------ */
typedef struct {
  int d_model, d_kv, d_ff, num_layers, num_heads;
  float layer_norm_epsilon;
  float rope_theta;
  int reg_token_id;
  int context_length;        /* longer contexts keep their last context_length values */
  int input_patch_size;      /* must equal output_patch_size and input_patch_stride */
  int output_patch_size;
  int num_quantiles;
  int use_reg_token;
  int use_arcsinh;
  float time_encoding_scale;
  int max_output_patches;    /* largest N a forward may ask for (sizes the RoPE table) */
} cc2_config;

/* Weights in the reference layout (nn.Linear: out x in, row-major), device
 * pointers of the model dtype.  Per-layer fields point to HOST arrays of
 * num_layers device pointers.  Names follow model.py:833-900. */
typedef struct {
  const void* shared;                 /* (vocab, d) embedding */
  const void* in_hidden_w;  const void* in_hidden_b;   /* (d_ff, 3*ps), (d_ff) */
  const void* in_output_w;  const void* in_output_b;   /* (d, d_ff), (d) */
  const void* in_residual_w; const void* in_residual_b; /* (d, 3*ps), (d) */
  const void* const* time_ln;  const void* const* time_q;  const void* const* time_k;
  const void* const* time_v;   const void* const* time_o;
  const void* const* group_ln; const void* const* group_q; const void* const* group_k;
  const void* const* group_v;  const void* const* group_o;
  const void* const* ff_ln;    const void* const* ff_wi;   const void* const* ff_wo;
  const void* final_ln;                                 /* (d) */
  const void* out_hidden_w;  const void* out_hidden_b;  /* (d_ff, d), (d_ff) */
  const void* out_output_w;  const void* out_output_b;  /* (Q*ps, d_ff), (Q*ps) */
  const void* out_residual_w; const void* out_residual_b; /* (Q*ps, d), (Q*ps) */
} cc2_weights;

typedef struct cc2_model cc2_model;

/* Bytes of the device buffer that holds the packed (RMS-folded, fused)
 * weights of a model. */
CC2_API int cc2_model_pack_bytes(const cc2_config* cfg, int dtype, size_t* bytes);
/* Packs `w` into `pack_buf` (dev, >= cc2_model_pack_bytes, 256-byte aligned)
 * on `stream` and returns a handle that references pack_buf (not `w`).
 * The caller keeps pack_buf alive until cc2_model_destroy. */
CC2_API int cc2_model_create(const cc2_config* cfg, int dtype, const cc2_weights* w,
                     void* pack_buf, size_t pack_bytes, void* stream, cc2_model** out);
CC2_API int cc2_model_destroy(cc2_model* m);

/* Group layout helper (host): turns per-series group ids into the member
 * list / offsets cc2_forward uses.  members_out (B) and offsets_out (B+1)
 * are host arrays; *num_groups and *max_group are written.  Series keep
 * their order inside a group; groups are ordered by first appearance. */
CC2_API int cc2_group_layout(const int64_t* group_ids, int B, int32_t* members_out,
                     int32_t* offsets_out, int* num_groups, int* max_group);

/* Workspace bytes for one forward of B series of length L with N output
 * patches; max_group is the largest group size (1 = every series alone). */
CC2_API int cc2_forward_workspace_bytes(const cc2_model* m, int B, int L, int N, int max_group,
                                size_t* bytes);

/* CuteChronos2Model.forward (model.py:738-831).
 *   context      (dev) float32 (B, L), NaN = missing
 *   context_mask (dev) float32 (B, L) or NULL (NULL: mask = !isnan(context))
 *   group_ids    (host) int64 (B) or NULL (NULL: each series its own group)
 *   out          (dev) dtype (B, num_quantiles, N*output_patch_size)
 *   loc, scale   (dev) float32 (B) or NULL: the instance-norm statistics
 *   workspace    (dev) >= cc2_forward_workspace_bytes, 256-byte aligned
 * With group_ids == NULL the call issues only asynchronous work on `stream`
 * and may be captured into a CUDA graph. */
CC2_API int cc2_forward(const cc2_model* m, const float* context, const float* context_mask,
                int B, int L, int N, const int64_t* group_ids, void* out, float* loc,
                float* scale, void* workspace, size_t workspace_bytes, void* stream);

/* Launch profiling.  Between cc2_profile_begin and cc2_profile_read, every
 * kernel that cc2_forward launches on the calling thread is bracketed by a
 * pair of CUDA events (at most `capacity` launches are recorded).
 * cc2_profile_read synchronises those events, writes per launch its kind
 * (CC2_K_*), device time (ms), algorithmic FLOPs and algorithmic HBM bytes,
 * stores the number of launches in *count and stops profiling. */
enum {
  CC2_K_PREPROCESS = 1, CC2_K_GEMM = 2, CC2_K_ATTN_TIME = 3, CC2_K_ATTN_GROUP = 4,
  CC2_K_RMSNORM = 5, CC2_K_OUTPUT = 6,
  /* the forward's GEMMs by role (CC2_K_GEMM: any other GEMM) */
  CC2_K_GEMM_QKV = 7,       /* time-attention Q/K/V (RMSNorm + RoPE)          */
  CC2_K_GEMM_O = 8,         /* time-attention output projection + residual    */
  CC2_K_GEMM_GROUP = 9,     /* group block: Wo.Wv fold (g = 1) or group QKV/O */
  CC2_K_GEMM_FFN_UP = 10,   /* wi (RMSNorm + ReLU)                            */
  CC2_K_GEMM_FFN_DOWN = 11, /* wo + residual                                  */
  CC2_K_GEMM_IO = 12,       /* input / output ResidualBlocks                  */
  CC2_K_LAYERS = 13         /* all encoder layers as one layer-persistent launch (cc2_set_layer_chain) */
};
CC2_API int cc2_profile_begin(int capacity);
CC2_API int cc2_profile_read(int* kinds, float* ms, double* flops, double* bytes, int capacity,
                             int* count);

/* cc2_forward without a caller-provided workspace (no counterpart in the
 * reference).  For callers that cannot allocate device memory themselves:
 * foreign-language front ends with no device allocator of their own, and
 * latency-sensitive serving loops where a cudaMalloc would synchronise the
 * device.  The scratch lives in one static device array of
 * CC2_NOALLOC_SCRATCH_BYTES (32 MiB) that every GPU loading this library
 * holds until the process exits; it fits about 1,950 token rows of the
 * bf16 Chronos-2-base model (e.g. 14 series of context 2048 with N = 4) and
 * about 930 rows of the fp32 model (e.g. 7 series of context 2048).  Larger
 * requests fail with CC2_E_WORKSPACE and a message giving the bytes needed.
 * The first call on a device looks the array's device address up (once per
 * device, with that device current); make that first call before any stream
 * capture.  All calls share the array: calls that overlap on the GPU (other
 * streams, other host threads) race and corrupt each other.  The forward
 * writes every scratch byte it reads, so nothing needs clearing between
 * calls.  No allocation happens in this call. */
#define CC2_NOALLOC_SCRATCH_BYTES ((size_t)32 << 20)
CC2_API int cc2_forward_noalloc(const cc2_model* m, const float* context, const float* context_mask,
                                int B, int L, int N, const int64_t* group_ids, void* out, float* loc,
                                float* scale, void* stream);

/* ------------------------------------------------------------------------ */
/* Component kernels (each is one stage of cc2_forward).                     */
/* ------------------------------------------------------------------------ */

/* Fused preprocessing (model.py:473-519 + 521-549): NaN-aware instance norm,
 * arcsinh, left-pad + 16-wide patching, time encoding.  Writes, for each
 * series b, S = P + use_reg + N token rows at row b*S of `patched`
 * (row pitch ld_patched elements, dtype): the first 3*ps columns hold
 * [time_enc | value | mask] for the P context patches, zeros for the REG
 * row, and [future time_enc | 0 | 0] for the N future rows; columns
 * [3*ps, pad_cols) are zeroed.  token_mask (dev, uint8, B*S): 1 = attendable.
 * attn_mask (dev, float32 (B,P)) may be NULL.  loc/scale (dev, float32 B). */
CC2_API int cc2_preprocess(const float* context, const float* context_mask, int B, int L,
                   int patch_size, int context_length, float time_encoding_scale,
                   int use_arcsinh, int use_reg, int N, int dtype, void* patched,
                   int ld_patched, int pad_cols, uint8_t* token_mask, float* attn_mask,
                   float* loc, float* scale, void* stream);

/* Epilogue flags for cc2_gemm. */
enum {
  CC2_EPI_ROWSCALE = 1,  /* acc *= rsqrt(sum_g ssq_in[g*ssq_ld + row] / norm_dim + eps),
                            g < ceil(norm_dim / 64)                           */
  CC2_EPI_BIAS = 2,      /* acc += bias[col] (float32)                         */
  CC2_EPI_RELU = 4,      /* acc = max(acc, 0)                                  */
  CC2_EPI_RESID = 8,     /* out = resid[row, col] + acc (resid may == out)     */
  CC2_EPI_SSQ = 16,      /* ssq_out[g*ssq_ld + row] = sum over the 64 columns
                            64g..64g+63 of out[row, col]^2 (partial sums per
                            64-column group: deterministic, no atomics)        */
  CC2_EPI_SPECIAL = 32,  /* rows with row % period == offset get special[]     */
  CC2_EPI_ROPE = 64,     /* bf16 only: rotate-half RoPE on every 64-column head
                            with col < rope_cols at position row % rope_period,
                            rope_cs[pos*32 + i] = (cos | sin << 16) as bf16 */
  CC2_EPI_LO = 128       /* bf16 only: the result v (fp32) is stored as out =
                            bf16(v) plus lo_out = bf16(v - out), so out +
                            lo_out carries ~16 significant bits; with RESID
                            the residual is resid + resid_lo; SSQ sums v^2.
                            lo_out / resid_lo use a 32-row interleaved layout
                            (coalesced for the epilogue's row-per-lane
                            access): element (row, col) at
                            ((row/32 * ld_lo/8 + col/8) * 32 + row%32) * 8 +
                            col%8, ld_lo a multiple of 8, ceil(M/32)*32 rows
                            allocated.  The engine keeps the encoder's
                            residual stream this way */
};

typedef struct {
  int flags;
  const float* ssq_in; int norm_dim; float eps;
  const float* bias;
  const void* resid; int ld_resid;
  float* ssq_out;
  int ssq_ld;            /* row stride between 64-column groups of ssq_in / ssq_out */
  const float* special; int special_period; int special_offset;
  const uint32_t* rope_cs; int rope_period; int rope_cols;
  void* lo_out; const void* resid_lo; int ld_lo;  /* CC2_EPI_LO */
} cc2_epilogue;

/* Tile variant of the bf16 GEMM: 0 (default) = 1-SM 128 x 64 tiles when the
 * 2-SM grid would occupy at most half the SMs (few token rows, e.g. batch-1
 * serving), else 2-SM tcgen05 tiles of 256 x 256 per CTA pair when M > 128,
 * else 1-SM 128 x 256 / 128 x 128 tiles; 1 = 1-SM 128 x 256 / 128 x 128 tiles
 * only; 2 = as 0 without the 128 x 64 tiles; 3 = measurement only: the 2-SM
 * mainloop with the epilogue skipped (nothing is written).  All variants
 * except 3 give bit-identical results.  Process-wide; returns the previous
 * value. */
CC2_API int cc2_set_gemm_variant(int variant);

/* Time-attention kernel choice for bf16 sets (RoPE applied beforehand):
 * 0 (default) = tcgen05 (scores and outputs in TMEM) for 112..144 tokens,
 * the mma.sync kernels otherwise; 1 = the mma.sync kernels only; 2 = tcgen05
 * for every set of 17..144 tokens; 3 = the whole-set mma.sync kernel only (the
 * arithmetic of the layer-persistent forward, see cc2_set_layer_chain).
 * Process-wide; returns the previous value. */
CC2_API int cc2_set_attention_variant(int variant);

/* Event trace of the tcgen05 time-attention kernels: with a device buffer of
 * 16 x 44 uint64 (zeroed by the caller), CTA 0 of every later launch writes
 * %globaltimer stamps (ns) of its first 16 query tiles.  Sets of up to 144
 * tokens, 12 per tile: load issued, MMA saw the load, S MMAs issued, MMA saw
 * P, O MMAs issued, softmax saw S, P written, softmax saw O, O stored, scores
 * in registers, row max done (one slot unused).  Longer sets, 44 per tile: per
 * key block j at 8j + {0 softmax saw S, 1 block max exchanged, 2 P in
 * registers, 3 softmax saw P free, 4 P written, 5 S MMAs issued, 6 MMA saw P,
 * 7 O MMAs issued}, then 40 Q load issued, 41 softmax saw O, 42 O stored.
 * NULL turns it off. */
CC2_API int cc2_set_attention_trace(void* device_buffer);

/* Programmatic dependent launch of the forward's kernels (default 1): each
 * kernel may start - barrier set-up, TMEM allocation, descriptor prefetch -
 * while the previous one finishes, and waits for it before touching
 * activations.  0 launches them strictly one after another.  Process-wide;
 * returns the previous value. */
CC2_API int cc2_set_launch_overlap(int enabled);

/* Layer-persistent forward (default 0, off): with 1, a bf16 forward with at most 384 token
 * rows (B x S; batch-1 serving), no series groups and no K/V quantiser runs
 * its encoder layers as ONE cooperative launch of one CTA per SM instead of
 * six launches per layer: the QKV GEMM, time attention, O-projection, group
 * block, FFN up and FFN down of every layer are stages separated by a
 * grid-wide barrier.  Its GEMMs compute exactly what the 128 x 64-tile GEMMs
 * compute; its attention splits each 16-row query tile's keys over the CTA's
 * warps and merges their softmax states (results within bf16 rounding of the
 * per-kernel forward).  2 = the same launch with the attention of the
 * whole-set mma.sync kernel (cc2_set_attention_variant(3)), bit-identical to
 * the per-kernel forward with that variant (for tests).  0 launches the
 * layers kernel by kernel.  Measured at batch 1 the persistent launch is no
 * faster than the per-kernel forward (0.88 against 0.89 ms at context 2048,
 * 0.83 against 0.79 ms at 512, CUDA graphs): each stage is bound by its own
 * latency chain (first load, k-loop at one SM's TMA rate, epilogue, barrier),
 * which the launches it replaces already overlapped.  Process-wide; returns
 * the previous value. */
CC2_API int cc2_set_layer_chain(int enabled);
/* Test hook (no counterpart in the reference): on != 0 arms a one-shot
 * fault-free failure: the next single-SM bf16 GEMM CTA (cc2_gemm with
 * M <= 128) withholds the load of its first k-block (and disarms the hook),
 * so its bounded mbarrier wait runs out after 2 s; the
 * kernel then sets the device error word (cc2_device_status returns
 * CC2_DEV_GEMM_TIMEOUT), leaves its loops, frees its TMEM and returns.
 * Exists so that tests can exercise the failure path without a GPU fault;
 * keep it off (0) otherwise.  Applies to the current device. */
CC2_API int cc2_test_starve_gemm(int on);

/* Test hook, one-shot: CTA 0 of the next layer-persistent launch
 * (cc2_set_layer_chain) leaves at its first grid barrier without arriving, so
 * every other CTA's bounded wait there runs out (2 s); they raise
 * CC2_DEV_LAYER_TIMEOUT, leave their stage loops, free TMEM and return.  For
 * tests of the failure path without a GPU fault; keep it off (0) otherwise. */
CC2_API int cc2_test_starve_layer_barrier(int on);

/* Stage trace of the layer-persistent forward: with a device buffer of
 * 8 x 76 x 2 + 320 uint64 (zeroed by the caller), CTAs 0..7 of every later
 * launch write, for stage s, [cta][s][0] = %globaltimer (ns) when the CTA
 * finished the stage and [cta][s][1] when the grid barrier after it released
 * the CTA; CTA 0 then records its first tile of stages 2 and 5 (160 entries
 * each): [0..63] load of k-block issued, [64..127] k-block landed (MMA
 * issue), [128] accumulator full, [129] tile stored, [130] stores complete,
 * [131] stage start, [132] accumulator read, [133] residual box landed,
 * [134] epilogue computed, [135] epilogue tile start; and of stage 1 (time
 * attention, 8 entries from 320): [327] stage start, [320] Q/K/V staged,
 * [321..326] warp w done.  NULL turns it off.  Process-wide. */
CC2_API int cc2_set_layer_trace(void* device_buffer);

/* Event trace of the 2-SM GEMM: with a device buffer of 32 x 8 uint64
 * (zeroed by the caller), CTA 0 of every later launch writes, for its first
 * 32 tiles: %globaltimer stamps (ns) of accumulator free, first stage loaded,
 * last k-block issued (MMA thread), accumulator full, epilogue done (first
 * epilogue warp), first load issued (producer), and the nanoseconds the MMA
 * thread waited for loaded stages in the tile.  NULL turns it off. */
CC2_API int cc2_set_gemm_trace(void* device_buffer);

/* out[M, N] = epilogue(A[M, K] @ W[N, K]^T); A, W, out, resid of `dtype`,
 * row-major with the given row pitches (elements).  bf16 runs on tcgen05
 * tensor cores (TMEM accumulators, TMA-fed); f32 runs on CUDA cores. */
CC2_API int cc2_gemm(int dtype, const void* A, int lda, const void* W, int ldw, void* out, int ldo,
             int M, int N, int K, const cc2_epilogue* epi, void* stream);

/* y[r] = w * round(x[src_row(r)] * rsqrt(mean(x^2) + eps)) for r < rows, where
 * src_row(r) = (r / per) * stride + offset + r % per; y row pitch ld_y.
 * (T5 RMSNorm of the reference, applied to a strided subset of rows.) */
CC2_API int cc2_rmsnorm_rows(int dtype, const void* x, int ld_x, const void* w, void* y, int ld_y,
                     int rows, int dim, int per, int stride, int offset, float eps, void* stream);

/* Unscaled attention (no 1/sqrt(d)) over sets of token rows.
 *   mode 0 (time):  set b = rows b*S .. b*S+S-1, RoPE at positions 0..S-1
 *                   (rope_cs: float2 (cos, sin) table, [pos][d_kv/2]; NULL
 *                   = no RoPE).
 *   mode 1 (group): set (t, g) = rows members[offsets[g]+i]*S + t, no RoPE.
 * qkv rows hold Q at q_col, K at k_col, V at v_col (head h at +h*d_kv);
 * keys whose token_mask is 0 are masked; out gets head h at h*d_kv. */
CC2_API int cc2_attention(int dtype, int mode, const void* qkv, int ld_qkv, int q_col, int k_col,
                  int v_col, void* out, int ld_out, const uint8_t* token_mask, int num_sets,
                  int S, int num_heads, int d_kv, const int32_t* members,
                  const int32_t* offsets, int num_groups, int max_group,
                  const float* rope_cs, void* stream);

/* Group attention (mode 1 of cc2_attention) on the tensor cores for the common
 * layout of model.py:295-312's batches: B series in groups of g consecutive
 * series (g = 2, 4, 8, 16 or 32, B a multiple of g), bf16, d_kv = 64; S token
 * rows per series (row b*S + t), heads heads.  Same result as cc2_attention
 * mode 1 on that layout (P rounded to bf16 as the reference's softmax
 * .to(dtype)); the forward uses it whenever the group ids have this layout.
 * Returns CC2_E_INVALID for another g or misaligned operands. */
CC2_API int cc2_group_attention_tc(const void* qkv, int ld_qkv, int q_col, int k_col, int v_col, void* out,
                                   int ld_out, const uint8_t* token_mask, int B, int S, int num_heads, int g,
                                   void* stream);

/* Rearrange b n (q p) -> b q (n p), sinh (if use_arcsinh), * scale + loc
 * (model.py:816-829).  preds (B*N, Q*ps) dtype with row pitch ld_preds;
 * out (B, Q, N*ps) dtype. */
CC2_API int cc2_output_transform(int dtype, const void* preds, int ld_preds, const float* loc,
                         const float* scale, void* out, int B, int N, int Q, int ps,
                         int use_arcsinh, void* stream);

/* ------------------------------------------------------------------------ */
/* TurboQuant K/V hook of the time attention (model.py:615-667,              */
/* tubroquant/quantizer.py:41-178).                                           */
/* ------------------------------------------------------------------------ */
/* One quantiser of 64-value vectors; every pointer is device memory.        */
typedef struct {
  int mode;                 /* 0 = "mse", 1 = "prod" (centroids on bits - 1, plus a 1-bit QJL sketch) */
  int bits;                 /* bits per coordinate, 0..8 centroid bits */
  int rotation;             /* 0 = Hadamard (signs, perm, inv_perm), 1 = dense matrix */
  int norm_dtype;           /* storage of the norms: 0 float16, 1 bfloat16, 2 float32 */
  const float* signs;       /* (64) +-1 */
  const int32_t* perm;      /* (64): rotated[i] = fwht(x[perm[i]] * signs[i]) / 8 */
  const int32_t* inv_perm;  /* (64) */
  const float* matrix;      /* (64, 64) row-major: rotated = x @ matrix^T */
  const float* codebook;    /* (2^centroid bits), ascending */
  const float* boundaries;  /* (2^centroid bits - 1), ascending */
  const float* proj;        /* (64, 64) Gaussian projection (prod mode) */
} cc2_kvq;

/* In place on packed token rows (dtype, row pitch ld): RoPE on the Q and K
 * columns first when rope_cs (float32 [pos][32] (cos, sin) pairs, position =
 * row % rope_period) is given, then every 64-column K vector of each head
 * replaced by its quantised reconstruction with `key` and every V vector with
 * `value` (NULL = leave as is).  stats (dev float32[4] or NULL) accumulates K
 * squared error, K max |error|, V squared error, V max |error|. */
CC2_API int cc2_kv_quant(int dtype, void* qkv, int ld, int rows, int q_col, int k_col, int v_col, int heads,
                         const cc2_kvq* key, const cc2_kvq* value, const float* rope_cs, int rope_period,
                         float* stats, void* stream);

/* Enable (key and/or value non-NULL; the structs are copied, the tables they
 * point to stay the caller's) or disable (both NULL) the hook for one layer
 * of a model; cc2_forward then runs it between that layer's QKV GEMM and its
 * time attention, accumulating into stats (dev float32[4] or NULL). */
CC2_API int cc2_model_set_kv_quant(cc2_model* m, int layer, const cc2_kvq* key, const cc2_kvq* value,
                                   float* stats);

/* ------------------------------------------------------------------------ */
/* Pipeline steps on the device (pipeline.py:221-322, 24-58).                 */
/* ------------------------------------------------------------------------ */
/* Ragged series -> (B, L) batch: row b is values[offsets[b] .. offsets[b+1])
 * (dev float32, dev int64 offsets, B+1 entries), its last L values
 * right-aligned, NaN before them (_left_pad_and_stack_rows, pipeline.py:221-231;
 * truncation of _finalize_context_batch, :239-243).  out (dev) float32 (B, L). */
CC2_API int cc2_stack_series(const float* values, const int64_t* offsets, int B, int L, float* out,
                             void* stream);

/* Quantile levels of forecasts (_select_quantiles, pipeline.py:24-58).
 *   preds  (dev) dtype (B, Q, ld); the first H columns of each row are used
 *   level j (nq <= 64; host arrays): lo[j] == hi[j] gathers trained level
 *          lo[j]; otherwise fl(fl(a_lo * w_lo[j]) + fl(a_hi * w_hi[j]))
 *   layout 0: out (dev) float32 (B, nq, H); 1: out (B, H, nq)
 *   median (dev) float32 (B, H) or NULL: trained level median_q, gathered. */
CC2_API int cc2_select_quantiles(int dtype, const void* preds, int B, int Q, int ld, int H, int nq,
                                 const int* lo, const int* hi, const float* w_lo, const float* w_hi,
                                 int layout, float* out, int median_q, float* median, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CC2_H */
