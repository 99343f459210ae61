// Unscaled self-attention over "sets" of token rows (no 1/sqrt(d) factor).
//
//   time attention  (mode 0): set b = the S tokens of series b; RoPE (when a
//     cos/sin table is given) is applied to Q and K in the prologue at
//     positions 0..S-1; keys with token_mask 0
//     are masked.  Reference: TimeSelfAttentionFallback.forward
//     (cutechronos/model.py:209-275), RoPE model.py:94-128 / rope.py:126-180,
//     unscaled_attention kernel_backends.py:113-153 (SDPA with scale=1.0).
//   group attention (mode 1): set (t, g) = token t of every series in group g;
//     no RoPE; key (b, t) is masked when token_mask[b, t] is 0.  Reference:
//     GroupSelfAttentionFallback.forward (model.py:295-312) with the group-time
//     mask of model.py:561-569 - the reference materialises all B x B scores per
//     time step and masks the other groups; here only the group is visited.
//
// Masking: a masked key scores -1e30 (finite, like the reference's additive
// finfo.min), a key past the end of the set scores -inf.  A query whose keys
// are all masked therefore averages its set's values with equal weights
// (finite output); such queries are padding tokens whose state never reaches
// a forecast.
//
// Kernels:
//   attn_set_kernel   bf16, the default: one CTA per (head, set) with the
//                     set's Q, K and V resident in shared memory (sets up to
//                     ~590 keys); warps own 16-row query tiles; mma.sync
//                     m16n8k16, fp32 online softmax.
//   attn_mma_kernel   bf16, blocked flash kernel for larger sets: 64 queries per CTA (16 per warp),
//                     64-key blocks, mma.sync m16n8k16 with fp32 accumulation,
//                     online softmax in fp32 (exp2 domain), P re-used from
//                     registers as the A operand of P.V.  S x S never leaves
//                     registers.
//   attn_group_small_kernel  groups of <= 16 series: one CTA per (time step,
//                     group) over all heads, CUDA cores, fp32 math.
//   attn_simt_kernel  float or bf16 storage, fp32 math on CUDA cores: the fp32
//                     time attention and groups of 17..32 series.
#include <cuda.h>

#include "common.cuh"
#include "attn_set_tile.cuh"

namespace cc2 {

int encode_bf16_map(CUtensorMap* map, const void* ptr, int cols, int rows, int ld, int box_cols, int box_rows);
bool attn_tc_supported(int S, int ld, int ldo, const void* qkv);
bool attn_pack_tc_supported(int S, int ld, int ldo, const void* qkv, const void* out);
int launch_attn_pack_tc(const void* qkv, int ld, int qcol, int kcol, int vcol, void* out, int ldo, const uint8_t* tok,
                        int num_sets, int S, int heads, int* err, cudaStream_t st);
bool attn_tc_long_supported(int S, int ld, int ldo, const void* qkv, const void* out);
int launch_attn_tc_long(const void* qkv, int ld, int qcol, int kcol, int vcol, void* out, int ldo,
                        const uint8_t* tok, int num_sets, int S, int heads, int* err, cudaStream_t st);
int launch_attn_tc(const void* qkv, int ld, int qcol, int kcol, int vcol, void* out, int ldo, const uint8_t* tok,
                   int num_sets, int S, int heads, int* err, cudaStream_t st);

// 0 (default): tcgen05 time attention for sets of 112..144 tokens, where it
// is faster than the mma.sync kernels, and the long-set tcgen05 kernel for
// 145..640 tokens; 1: the mma.sync kernels only for time attention and the
// scalar kernel for small groups; 2: tcgen05 for every set it supports
// (17..640 tokens); 3: the whole-set mma.sync kernel (attn_set_kernel) for
// every time-attention set that fits its shared memory - the arithmetic of
// the layer-persistent forward's attention stage.  Set through
// cc2_set_attention_variant.
int g_attn_variant = 0;

// Error word of the attention kernels' bounded waits (1 = a wait ran out).
__device__ int g_attn_error = 0;

int attention_error_word(int** p) {
  CC2_CUDA(cudaGetSymbolAddress((void**)p, g_attn_error));
  return CC2_OK;
}

int read_attention_error(int clear, int* value) {
  CC2_CUDA(cudaMemcpyFromSymbol(value, g_attn_error, sizeof(int)));
  if (clear) {
    int z = 0;
    CC2_CUDA(cudaMemcpyToSymbol(g_attn_error, &z, sizeof(int)));
  }
  return CC2_OK;
}

namespace {

typedef __nv_bfloat16 bf16;
using namespace aset;

struct SetInfo {
  int mode;  // 0 time, 1 group
  int S;     // tokens per series
  const int32_t* members;
  const int32_t* offsets;
  int num_groups;
};

struct SetGeom {
  int n;
  int base;               // time: first row
  int t;                  // group: time index
  const int32_t* mem;     // group: member list
  __device__ __forceinline__ int row(int i, int S) const { return mem ? mem[i] * S + t : base + i; }
};

__device__ __forceinline__ SetGeom set_geom(const SetInfo& si, int set) {
  SetGeom g;
  if (si.mode == 0) {
    g.n = si.S; g.base = set * si.S; g.t = 0; g.mem = nullptr;
  } else {
    const int t = set / si.num_groups, grp = set % si.num_groups;
    const int o0 = si.offsets[grp];
    g.n = si.offsets[grp + 1] - o0; g.base = 0; g.t = t; g.mem = si.members + o0;
  }
  return g;
}


// ---------------------------------------------------------------------------
// tensor-core flash kernel (bf16)
// ---------------------------------------------------------------------------
constexpr int QT = 64, KT = 64, DH = 64, LDS = DH + 8;  // padded smem rows (144 B)


// Rotate-half RoPE on a [rows][LDS] bf16 tile in shared memory (fp32 math,
// one rounding), positions pos0 + r for rows r < valid.
__device__ __forceinline__ void rope_tile(bf16 (*T)[LDS], int valid, int pos0, const float2* __restrict__ cs) {
  for (int idx = threadIdx.x; idx < valid * (DH / 2); idx += blockDim.x) {
    const int r = idx / (DH / 2), i = idx % (DH / 2);
    const float2 c = cs[(size_t)(pos0 + r) * (DH / 2) + i];
    const float x1 = __bfloat162float(T[r][i]), x2 = __bfloat162float(T[r][i + DH / 2]);
    T[r][i] = __float2bfloat16_rn(x1 * c.x - x2 * c.y);
    T[r][i + DH / 2] = __float2bfloat16_rn(x2 * c.x + x1 * c.y);
  }
}

template <bool ROPE>
__global__ void __launch_bounds__(128)
attn_mma_kernel(const bf16* __restrict__ qkv, int ld, int qcol, int kcol, int vcol, bf16* __restrict__ out,
                int ldo, const uint8_t* __restrict__ tok, const float2* __restrict__ rope, SetInfo si) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ __align__(16) bf16 Qs[QT][LDS];
  __shared__ __align__(16) bf16 Ks[KT][LDS];
  __shared__ __align__(16) bf16 Vs[KT][LDS];
  __shared__ float kbias[KT];

  const SetGeom g = set_geom(si, blockIdx.z);
  const int h = blockIdx.y;
  const int q0 = blockIdx.x * QT;
  if (q0 >= g.n) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hq = qcol + h * DH, hk = kcol + h * DH, hv = vcol + h * DH;

  // ---- Q tile (+RoPE) -> registers ----
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = (tid >> 3) + 16 * i, c = (tid & 7) * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (q0 + r < g.n) v = *reinterpret_cast<const uint4*>(qkv + (size_t)g.row(q0 + r, si.S) * ld + hq + c);
    *reinterpret_cast<uint4*>(&Qs[r][c]) = v;
  }
  __syncthreads();
  if (ROPE) {
    rope_tile(Qs, min(QT, g.n - q0), q0, rope);
    __syncthreads();
  }
  uint32_t qf[4][4];
  {
    const uint32_t base = (uint32_t)__cvta_generic_to_shared(&Qs[16 * warp + (lane & 15)][(lane >> 4) * 8]);
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) ldsm_x4(base + ks * 32, qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3]);
  }

  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;

  for (int k0 = 0; k0 < g.n; k0 += KT) {
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = (tid >> 3) + 16 * i, c = (tid & 7) * 8;
      uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
      if (k0 + r < g.n) {
        const size_t rb = (size_t)g.row(k0 + r, si.S) * ld;
        kv = *reinterpret_cast<const uint4*>(qkv + rb + hk + c);
        vv = *reinterpret_cast<const uint4*>(qkv + rb + hv + c);
      }
      *reinterpret_cast<uint4*>(&Ks[r][c]) = kv;
      *reinterpret_cast<uint4*>(&Vs[r][c]) = vv;
    }
    if (tid < KT) {
      const int kj = k0 + tid;
      float b = -INFINITY;
      if (kj < g.n) b = tok[g.row(kj, si.S)] ? 0.0f : kMaskedScore;
      kbias[tid] = b;
    }
    __syncthreads();
    if (ROPE) {
      rope_tile(Ks, min(KT, g.n - k0), k0, rope);
      __syncthreads();
    }
    // ---- S = Q K^T (16 x 64 per warp) ----
    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.0f;
      const uint32_t kb = (uint32_t)__cvta_generic_to_shared(&Ks[nt * 8 + (lane & 7)][(lane >> 3) * 8]);
#pragma unroll
      for (int ks = 0; ks < 4; ks += 2) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kb + ks * 32, b0, b1, b2, b3);
        mma16816(s[nt], qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3], b0, b1);
        mma16816(s[nt], qf[ks + 1][0], qf[ks + 1][1], qf[ks + 1][2], qf[ks + 1][3], b2, b3);
      }
    }
    // ---- mask + online softmax (log2 domain) ----
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int c = nt * 8 + 2 * (lane & 3);
      const float b0 = kbias[c], b1 = kbias[c + 1];
      s[nt][0] = b0 == 0.0f ? s[nt][0] * kLog2e : b0;
      s[nt][1] = b1 == 0.0f ? s[nt][1] * kLog2e : b1;
      s[nt][2] = b0 == 0.0f ? s[nt][2] * kLog2e : b0;
      s[nt][3] = b1 == 0.0f ? s[nt][3] * kLog2e : b1;
      mx0 = fmaxf(mx0, fmaxf(s[nt][0], s[nt][1]));
      mx1 = fmaxf(mx1, fmaxf(s[nt][2], s[nt][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float c0 = exp2f(m0 - mn0), c1 = exp2f(m1 - mn1);
    m0 = mn0; m1 = mn1;
    l0 *= c0; l1 *= c1;
#pragma unroll
    for (int dt = 0; dt < 8; ++dt) { o[dt][0] *= c0; o[dt][1] *= c0; o[dt][2] *= c1; o[dt][3] *= c1; }
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      s[nt][0] = exp2f(s[nt][0] - mn0); s[nt][1] = exp2f(s[nt][1] - mn0);
      s[nt][2] = exp2f(s[nt][2] - mn1); s[nt][3] = exp2f(s[nt][3] - mn1);
      l0 += s[nt][0] + s[nt][1];
      l1 += s[nt][2] + s[nt][3];
    }
    // ---- O += P V ----
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t a0 = pack2(s[2 * j][0], s[2 * j][1]);
      const uint32_t a1 = pack2(s[2 * j][2], s[2 * j][3]);
      const uint32_t a2 = pack2(s[2 * j + 1][0], s[2 * j + 1][1]);
      const uint32_t a3 = pack2(s[2 * j + 1][2], s[2 * j + 1][3]);
      const uint32_t vb = (uint32_t)__cvta_generic_to_shared(&Vs[16 * j + (lane & 15)][(lane >> 4) * 8]);
#pragma unroll
      for (int dt = 0; dt < 8; dt += 2) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vb + dt * 16, b0, b1, b2, b3);
        mma16816(o[dt], a0, a1, a2, a3, b0, b1);
        mma16816(o[dt + 1], a0, a1, a2, a3, b2, b3);
      }
    }
  }
  // ---- normalise, stage through smem (own rows of Qs), coalesced store ----
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float i0 = 1.0f / l0, i1 = 1.0f / l1;
  const int r0 = 16 * warp + (lane >> 2);
#pragma unroll
  for (int dt = 0; dt < 8; ++dt) {
    const int c = dt * 8 + 2 * (lane & 3);
    *reinterpret_cast<uint32_t*>(&Qs[r0][c]) = pack2(o[dt][0] * i0, o[dt][1] * i0);
    *reinterpret_cast<uint32_t*>(&Qs[r0 + 8][c]) = pack2(o[dt][2] * i1, o[dt][3] * i1);
  }
  __syncwarp();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int rr = 16 * warp + (lane >> 3) + 4 * i, c = (lane & 7) * 8;
    if (q0 + rr < g.n)
      *reinterpret_cast<uint4*>(out + (size_t)g.row(q0 + rr, si.S) * ldo + h * DH + c) =
          *reinterpret_cast<const uint4*>(&Qs[rr][c]);
  }
}

// ---------------------------------------------------------------------------
// whole-set tensor-core kernel (bf16): one CTA per (head, set).  Q, K and V
// of the whole set are staged in shared memory with one wave of async copies,
// RoPE is applied there once, and each warp then owns 16-row query tiles and
// streams over the keys with no block-level barrier.  Key n-tiles past the end
// of the set are skipped, so a set of n keys costs ceil(n/8) score tiles per
// query tile.
// ---------------------------------------------------------------------------

constexpr int kSetMaxWarps = 8;
constexpr size_t kSetSmemLimit = 225 * 1024;  // larger sets use the blocked kernel


inline size_t set_kernel_smem(int npad) { return (size_t)npad * (3 * 128 + sizeof(float)); }

// RoPE (rotate half) on rows [0, n) of the swizzled Q and K tiles, position =
// row index.  Each (row, i) entry of the cos/sin table is read once for both
// tiles, and table loads are issued in batches of kRopeBatch per thread so
// their latency overlaps.
constexpr int kRopeBatch = 8;
__device__ __forceinline__ void rope_qk_swz(uint8_t* Qt, uint8_t* Kt, int n, const float2* __restrict__ cs) {
  const int total = n * (DH / 2);
  for (int base = threadIdx.x; base < total; base += blockDim.x * kRopeBatch) {
    float2 c[kRopeBatch];
#pragma unroll
    for (int j = 0; j < kRopeBatch; ++j) {
      const int idx = base + j * blockDim.x;
      c[j] = idx < total ? __ldg(cs + idx) : make_float2(1.0f, 0.0f);
    }
#pragma unroll
    for (int j = 0; j < kRopeBatch; ++j) {
      const int idx = base + j * blockDim.x;
      if (idx < total) {
        const int r = idx / (DH / 2), i = idx % (DH / 2);
        const int o1 = r * 128 + (((i >> 3) ^ (r & 7)) << 4) + (i & 7) * 2;
        const int o2 = r * 128 + ((((i >> 3) + 4) ^ (r & 7)) << 4) + (i & 7) * 2;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          uint8_t* T = t ? Kt : Qt;
          bf16* p1 = reinterpret_cast<bf16*>(T + o1);
          bf16* p2 = reinterpret_cast<bf16*>(T + o2);
          const float x1 = __bfloat162float(*p1), x2 = __bfloat162float(*p2);
          *p1 = __float2bfloat16_rn(x1 * c[j].x - x2 * c[j].y);
          *p2 = __float2bfloat16_rn(x2 * c[j].x + x1 * c[j].y);
        }
      }
    }
  }
}

// KTT: keys per inner tile (64; 48 for sets of at most 48 tokens, which then
// take one tile and fewer registers, so more CTAs share an SM)
template <bool ROPE, int KTT>
__global__ void __launch_bounds__(KTT == 64 ? kSetMaxWarps * 32 : 128, KTT == 64 ? 2 : 5)
attn_set_kernel(const bf16* __restrict__ qkv, int ld, int qcol, int kcol, int vcol, bf16* __restrict__ out,
                int ldo, const uint8_t* __restrict__ tok, const float2* __restrict__ rope, SetInfo si) {
  pdl_launch_dependents();
  pdl_wait();
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const SetGeom g = set_geom(si, blockIdx.y);
  const int h = blockIdx.x;
  const int n = g.n;
  if (n <= 0) return;
  const int npad = (n + 15) & ~15;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nwarps = blockDim.x >> 5;
  uint8_t* Qs = smem_raw;
  uint8_t* Ks = Qs + npad * 128;
  uint8_t* Vs = Ks + npad * 128;
  float* kbias = reinterpret_cast<float*>(Vs + npad * 128);
  const uint32_t qb = (uint32_t)__cvta_generic_to_shared(Qs);
  const uint32_t kb = (uint32_t)__cvta_generic_to_shared(Ks);
  const uint32_t vb = (uint32_t)__cvta_generic_to_shared(Vs);
  const int hq = qcol + h * DH, hk = kcol + h * DH, hv = vcol + h * DH;

  for (int idx = tid; idx < npad * 8; idx += blockDim.x) {
    const int r = idx >> 3, c = idx & 7;
    if (r < n) {
      const bf16* src = qkv + (size_t)g.row(r, si.S) * ld + c * 8;
      cp_async16(swz(qb, r, c), src + hq);
      cp_async16(swz(kb, r, c), src + hk);
      cp_async16(swz(vb, r, c), src + hv);
    } else {
      const uint4 z = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(Qs + (swz(qb, r, c) - qb)) = z;
      *reinterpret_cast<uint4*>(Ks + (swz(kb, r, c) - kb)) = z;
      *reinterpret_cast<uint4*>(Vs + (swz(vb, r, c) - vb)) = z;
    }
  }
  for (int r = tid; r < npad; r += blockDim.x)
    kbias[r] = r < n ? (tok[g.row(r, si.S)] ? 0.0f : kMaskedScore) : -INFINITY;
  cp_async_wait_all();
  __syncthreads();
  if (ROPE) {
    rope_qk_swz(Qs, Ks, n, rope);
    __syncthreads();
  }

  for (int q0 = warp * 16; q0 < n; q0 += nwarps * 16)
    set_tile<KTT>(qb, kb, vb, kbias, n, q0, lane, [&](int rr, int c, const uint4& v) {
      *reinterpret_cast<uint4*>(out + (size_t)g.row(rr, si.S) * ldo + h * DH + c * 8) = v;
    });
}

// ---------------------------------------------------------------------------
// SIMT kernel (fp32 mode, small groups)
// ---------------------------------------------------------------------------
constexpr int SQ = 16;  // queries per CTA (4 per warp)
constexpr int SK = 32;  // keys per block (one per lane)

template <typename T, bool ROPE>
__global__ void __launch_bounds__(128)
attn_simt_kernel(const T* __restrict__ qkv, int ld, int qcol, int kcol, int vcol, T* __restrict__ out, int ldo,
                 const uint8_t* __restrict__ tok, const float2* __restrict__ rope, SetInfo si) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float Qs[SQ][DH];
  __shared__ float Ks[SK][DH + 1];
  __shared__ float Vs[SK][DH];
  __shared__ float kbias[SK];
  const SetGeom g = set_geom(si, blockIdx.z);
  const int h = blockIdx.y;
  const int q0 = blockIdx.x * SQ;
  if (q0 >= g.n) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hq = qcol + h * DH, hk = kcol + h * DH, hv = vcol + h * DH;

  for (int idx = tid; idx < SQ * (DH / 2); idx += blockDim.x) {
    const int r = idx / (DH / 2), i = idx % (DH / 2);
    float x1 = 0.0f, x2 = 0.0f;
    if (q0 + r < g.n) {
      const T* src = qkv + (size_t)g.row(q0 + r, si.S) * ld + hq;
      x1 = tof<T>(src[i]);
      x2 = tof<T>(src[i + DH / 2]);
      if (ROPE) {
        const float2 c = rope[(size_t)(q0 + r) * (DH / 2) + i];
        const float y1 = x1 * c.x - x2 * c.y, y2 = x2 * c.x + x1 * c.y;
        x1 = roundT<T>(y1);
        x2 = roundT<T>(y2);
      }
    }
    Qs[r][i] = x1;
    Qs[r][i + DH / 2] = x2;
  }
  float m[4], l[4], o0[4], o1[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) { m[r] = -INFINITY; l[r] = 0.0f; o0[r] = 0.0f; o1[r] = 0.0f; }

  for (int k0 = 0; k0 < g.n; k0 += SK) {
    __syncthreads();
    for (int idx = tid; idx < SK * (DH / 2); idx += blockDim.x) {
      const int r = idx / (DH / 2), i = idx % (DH / 2);
      float k1 = 0.0f, k2 = 0.0f, v1 = 0.0f, v2 = 0.0f;
      if (k0 + r < g.n) {
        const size_t rb = (size_t)g.row(k0 + r, si.S) * ld;
        k1 = tof<T>(qkv[rb + hk + i]);
        k2 = tof<T>(qkv[rb + hk + i + DH / 2]);
        v1 = tof<T>(qkv[rb + hv + i]);
        v2 = tof<T>(qkv[rb + hv + i + DH / 2]);
        if (ROPE) {
          const float2 c = rope[(size_t)(k0 + r) * (DH / 2) + i];
          const float y1 = k1 * c.x - k2 * c.y, y2 = k2 * c.x + k1 * c.y;
          k1 = roundT<T>(y1);
          k2 = roundT<T>(y2);
        }
      }
      Ks[r][i] = k1; Ks[r][i + DH / 2] = k2;
      Vs[r][i] = v1; Vs[r][i + DH / 2] = v2;
    }
    if (tid < SK) {
      const int kj = k0 + tid;
      kbias[tid] = kj < g.n ? (tok[g.row(kj, si.S)] ? 0.0f : kMaskedScore) : -INFINITY;
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int qr = warp * 4 + r;
      float sc = 0.0f;
#pragma unroll 16
      for (int d = 0; d < DH; ++d) sc = fmaf(Qs[qr][d], Ks[lane][d], sc);
      const float b = kbias[lane];
      sc = b == 0.0f ? sc : b;
      float mx = sc;
      for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float mn = fmaxf(m[r], mx);
      const float corr = expf(m[r] - mn);
      const float p = expf(sc - mn);
      float ps = p;
      for (int off = 16; off > 0; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
      l[r] = l[r] * corr + ps;
      float a0 = o0[r] * corr, a1 = o1[r] * corr;
      for (int j = 0; j < SK; ++j) {
        const float pj = __shfl_sync(0xffffffffu, p, j);
        a0 = fmaf(pj, Vs[j][2 * lane], a0);
        a1 = fmaf(pj, Vs[j][2 * lane + 1], a1);
      }
      o0[r] = a0; o1[r] = a1;
      m[r] = mn;
    }
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int qi = q0 + warp * 4 + r;
    if (qi < g.n) {
      T* dst = out + (size_t)g.row(qi, si.S) * ldo + h * DH;
      const float inv = 1.0f / l[r];
      dst[2 * lane] = fromf<T>(o0[r] * inv);
      dst[2 * lane + 1] = fromf<T>(o1[r] * inv);
    }
  }
}

// ---------------------------------------------------------------------------
// small groups (<= 16 series): one CTA per (time step, group) covering every
// head.  The group's Q/K/V rows (contiguous, 3 x heads*64 elements each) are
// staged in shared memory once; scores, softmax and P.V run on CUDA cores in
// fp32.  Replaces a launch of (sets x heads) tiny CTAs.
// ---------------------------------------------------------------------------
constexpr int kSmallGroupMax = 16;

// 8 consecutive elements (16 bytes of bf16, 32 of float) <-> fp32 registers
__device__ __forceinline__ void load8(const bf16* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 f = __bfloat1622float2(h[e]);
    v[2 * e] = f.x;
    v[2 * e + 1] = f.y;
  }
}
__device__ __forceinline__ void load8(const float* p, float (&v)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void store8(bf16* p, const float (&v)[8]) {
  uint4 u;
  u.x = pack2(v[0], v[1]); u.y = pack2(v[2], v[3]); u.z = pack2(v[4], v[5]); u.w = pack2(v[6], v[7]);
  *reinterpret_cast<uint4*>(p) = u;
}
__device__ __forceinline__ void store8(float* p, const float (&v)[8]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}

template <typename T>
__global__ void __launch_bounds__(256)
attn_group_small_kernel(const T* __restrict__ qkv, int ld, int qcol, int kcol, int vcol, T* __restrict__ out,
                        int ldo, const uint8_t* __restrict__ tok, SetInfo si, int heads) {
  pdl_launch_dependents();
  pdl_wait();
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const SetGeom g = set_geom(si, blockIdx.x);
  const int n = g.n;
  if (n <= 0) return;
  const int HD = heads * DH;
  const int HP = HD + 16 / (int)sizeof(T);  // staged row pitch: +16 bytes keeps rows on distinct banks
  T* Qs = reinterpret_cast<T*>(smem_raw);
  T* Ks = Qs + (size_t)n * HP;
  T* Vs = Ks + (size_t)n * HP;
  float* P = reinterpret_cast<float*>(Vs + (size_t)n * HP);  // [heads][n][n]
  float* kb = P + (size_t)heads * n * n;                     // [n]
  const int tid = threadIdx.x;
  constexpr int V = 16 / sizeof(T);  // elements per 16-byte vector
  const int nvec = HD / V;
  for (int idx = tid; idx < n * nvec; idx += blockDim.x) {
    const int i = idx / nvec, c = (idx % nvec) * V;
    const T* src = qkv + (size_t)g.row(i, si.S) * ld;
    *reinterpret_cast<uint4*>(Qs + (size_t)i * HP + c) = *reinterpret_cast<const uint4*>(src + qcol + c);
    *reinterpret_cast<uint4*>(Ks + (size_t)i * HP + c) = *reinterpret_cast<const uint4*>(src + kcol + c);
    *reinterpret_cast<uint4*>(Vs + (size_t)i * HP + c) = *reinterpret_cast<const uint4*>(src + vcol + c);
  }
  for (int i = tid; i < n; i += blockDim.x) kb[i] = tok[g.row(i, si.S)] ? 0.0f : kMaskedScore;
  __syncthreads();
  // scores: one (head, query, key) dot product per thread iteration, 8 elements per 16-byte load
  for (int idx = tid; idx < heads * n * n; idx += blockDim.x) {
    const int h = idx / (n * n), qi = (idx / n) % n, kj = idx % n;
    const T* q = Qs + (size_t)qi * HP + h * DH;
    const T* k = Ks + (size_t)kj * HP + h * DH;
    float acc = 0.0f;
#pragma unroll
    for (int d = 0; d < DH; d += 8) {
      float qa[8], ka[8];
      load8(q + d, qa);
      load8(k + d, ka);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc = fmaf(qa[e], ka[e], acc);
    }
    P[idx] = kb[kj] == 0.0f ? acc : kb[kj];
  }
  __syncthreads();
  // softmax over the keys of each (head, query) row
  for (int idx = tid; idx < heads * n; idx += blockDim.x) {
    float* row = P + (size_t)idx * n;
    float m = -INFINITY;
    for (int j = 0; j < n; ++j) m = fmaxf(m, row[j]);
    float sum = 0.0f;
    for (int j = 0; j < n; ++j) {
      const float e = expf(row[j] - m);
      row[j] = e;
      sum += e;
    }
    const float inv = 1.0f / sum;
    for (int j = 0; j < n; ++j) row[j] *= inv;
  }
  __syncthreads();
  // out[qi][c..c+7] = sum_j P[h][qi][j] V[j][c..c+7]
  for (int idx = tid; idx < n * (HD / 8); idx += blockDim.x) {
    const int qi = idx / (HD / 8), c = (idx % (HD / 8)) * 8, h = c / DH;
    const float* prow = P + ((size_t)h * n + qi) * n;
    float acc[8] = {};
    for (int j = 0; j < n; ++j) {
      float va[8];
      load8(Vs + (size_t)j * HP + c, va);
      const float pj = prow[j];
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = fmaf(pj, va[e], acc[e]);
    }
    store8(out + (size_t)g.row(qi, si.S) * ldo + c, acc);
  }
}

// ---------------------------------------------------------------------------
// persistent time attention (bf16, Q/K already rotated): one CTA of 16 warps
// per SM walks its share of the (series, head) items.  Up to kPBufs items are
// resident in shared memory; each is loaded by three TMA boxes (Q, K, V: the
// item's rows x 64 columns, 128-byte swizzle) on an mbarrier.  Warps take
// (item, 16-row query tile) units from a shared counter in order, so no warp
// idles at an item boundary; the warp that finishes an item's last tile
// refills that buffer with the item kBufs ahead (TMA + key mask), so loads
// overlap compute.  A warp waiting for an item first waits until that item's
// load has been issued (warps may run more than one buffer generation ahead
// when an item has few tiles), then on the buffer's mbarrier.  All waits are
// bounded.
// ---------------------------------------------------------------------------
constexpr int kPWarps = 16;
constexpr int kPBufs = 4;
constexpr size_t kPSmemLimit = 220 * 1024;

__device__ __forceinline__ bool pmbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
               : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}
// Bounded wait (about 2 s); false when it ran out.
__device__ __noinline__ bool pmbar_wait_slow(uint32_t bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer_ns();
  for (uint32_t n = 1;; ++n) {
    if (pmbar_try(bar, parity)) return true;
    if ((n & 63u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) return false;
  }
}
__device__ __forceinline__ bool pmbar_wait(uint32_t bar, uint32_t parity) {
  return pmbar_try(bar, parity) || pmbar_wait_slow(bar, parity);
}

struct PersistArgs {
  int S;          // tokens per series (= set size)
  int npad;       // S rounded up to 16
  int heads;
  int items;      // B * heads
  int qcol, kcol, vcol;
  int box_rows;   // rows per TMA box (<= 256)
  int nboxes;     // boxes per operand
  int nbufs;
  size_t buf_bytes;
};

__global__ void __launch_bounds__(kPWarps * 32, 1)
attn_persist_kernel(const __grid_constant__ CUtensorMap tmQKV, bf16* __restrict__ out, int ldo,
                    const uint8_t* __restrict__ tok, PersistArgs a, int* __restrict__ err) {
  pdl_launch_dependents();
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  __shared__ __align__(8) uint64_t full_bar[kPBufs];
  __shared__ int done[kPBufs];
  __shared__ int next_unit;
  __shared__ int failed;
  // local item whose load was last issued into each buffer: a warp waits for
  // its item's load to be issued before it waits on the buffer's mbarrier, so
  // the parity it waits for always names that load's phase
  __shared__ volatile int buf_item[kPBufs];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n = a.S, npad = a.npad;
  const int nqt = (n + 15) / 16;
  const int my_items = a.items > (int)blockIdx.x ? (a.items - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int units = my_items * nqt;
  auto buf_base = [&](int b) { return smem + (size_t)b * a.buf_bytes; };
  auto kbias_of = [&](int b) { return reinterpret_cast<float*>(buf_base(b) + (size_t)3 * npad * 128); };
  auto full_addr = [&](int b) { return (uint32_t)__cvta_generic_to_shared(&full_bar[b]); };

  // issue the loads (and key mask) of local item li into its buffer; called by one full warp
  auto issue = [&](int li) {
    const int item = (int)blockIdx.x + li * (int)gridDim.x;
    const int b = li % a.nbufs;
    const int bser = item / a.heads, h = item % a.heads;
    float* kb = kbias_of(b);
    if (lane == 0) buf_item[b] = li;
    for (int r = lane; r < npad; r += 32)
      kb[r] = r < n ? (tok[(size_t)bser * n + r] ? 0.0f : kMaskedScore) : -INFINITY;
    __syncwarp();
    if (lane == 0) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      const uint32_t bar = full_addr(b);
      const uint32_t bytes = (uint32_t)(3 * a.nboxes * a.box_rows * 128);
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
      const uint32_t dst0 = (uint32_t)__cvta_generic_to_shared(buf_base(b));
      const int cols[3] = {a.qcol + h * DH, a.kcol + h * DH, a.vcol + h * DH};
      for (int t = 0; t < 3; ++t)
        for (int x = 0; x < a.nboxes; ++x) {
          const uint32_t dst = dst0 + (uint32_t)t * npad * 128 + (uint32_t)x * a.box_rows * 128;
          asm volatile(
              "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
              " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
              "l"((uint64_t)&tmQKV), "r"(bar), "r"(cols[t]), "r"(bser * n + x * a.box_rows)
              : "memory");
        }
    }
  };

  if (tid == 0) {
    for (int b = 0; b < kPBufs; ++b) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(full_addr(b)) : "memory");
      done[b] = 0;
      buf_item[b] = -1;
    }
    next_unit = 0;
    failed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  pdl_wait();  // the kernel before may still run until here; activations are read from now on
  if (warp < a.nbufs && warp < my_items) issue(warp);

  while (true) {
    int u = 0;
    if (lane == 0) u = atomicAdd(&next_unit, 1);
    u = __shfl_sync(0xffffffffu, u, 0);
    if (u >= units || failed) break;
    const int li = u / nqt, qt = u % nqt;
    const int b = li % a.nbufs;
    bool issued = buf_item[b] == li;
    if (!issued) {  // bounded spin until this item's load has been issued
      const unsigned long long t0 = globaltimer_ns();
      while (!(issued = buf_item[b] == li) && globaltimer_ns() - t0 < kWaitLimitNs) __nanosleep(64);
    }
    if (!issued || !pmbar_wait(full_addr(b), (uint32_t)(li / a.nbufs) & 1u)) {
      if (lane == 0) {
        failed = 1;
        atomicOr(err, 1);
      }
      break;
    }
    const int item = (int)blockIdx.x + li * (int)gridDim.x;
    const int bser = item / a.heads, h = item % a.heads;
    const uint32_t qb = (uint32_t)__cvta_generic_to_shared(buf_base(b));
    const uint32_t kb = qb + (uint32_t)npad * 128, vb = kb + (uint32_t)npad * 128;
    const float* kbias = kbias_of(b);
    const int q0 = qt * 16;

    uint32_t qf[4][4];
#pragma unroll
    for (int ks = 0; ks < 4; ++ks)
      ldsm_x4(swz(qb, q0 + (lane & 15), 2 * ks + (lane >> 4)), qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3]);
    float o[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
    for (int k0 = 0; k0 < n; k0 += KT) {
      const int kvalid = n - k0;
      float s[8][4];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.0f;
        if (nt * 8 < kvalid) {
          const int kr = k0 + nt * 8 + (lane & 7);
#pragma unroll
          for (int ks = 0; ks < 4; ks += 2) {
            uint32_t b0, b1, b2, b3;
            ldsm_x4(swz(kb, kr, 2 * ks + (lane >> 3)), b0, b1, b2, b3);
            mma16816(s[nt], qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3], b0, b1);
            mma16816(s[nt], qf[ks + 1][0], qf[ks + 1][1], qf[ks + 1][2], qf[ks + 1][3], b2, b3);
          }
        }
      }
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int c = nt * 8 + 2 * (lane & 3);
        const float b0 = c < kvalid ? kbias[k0 + c] : -INFINITY;
        const float b1 = c + 1 < kvalid ? kbias[k0 + c + 1] : -INFINITY;
        s[nt][0] = b0 == 0.0f ? s[nt][0] * kLog2e : b0;
        s[nt][1] = b1 == 0.0f ? s[nt][1] * kLog2e : b1;
        s[nt][2] = b0 == 0.0f ? s[nt][2] * kLog2e : b0;
        s[nt][3] = b1 == 0.0f ? s[nt][3] * kLog2e : b1;
        mx0 = fmaxf(mx0, fmaxf(s[nt][0], s[nt][1]));
        mx1 = fmaxf(mx1, fmaxf(s[nt][2], s[nt][3]));
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      const float c0 = exp2f(m0 - mn0), c1 = exp2f(m1 - mn1);
      m0 = mn0; m1 = mn1;
      l0 *= c0; l1 *= c1;
#pragma unroll
      for (int dt = 0; dt < 8; ++dt) { o[dt][0] *= c0; o[dt][1] *= c0; o[dt][2] *= c1; o[dt][3] *= c1; }
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        s[nt][0] = exp2f(s[nt][0] - mn0); s[nt][1] = exp2f(s[nt][1] - mn0);
        s[nt][2] = exp2f(s[nt][2] - mn1); s[nt][3] = exp2f(s[nt][3] - mn1);
        l0 += s[nt][0] + s[nt][1];
        l1 += s[nt][2] + s[nt][3];
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (j * 16 < kvalid) {
          const uint32_t a0 = pack2(s[2 * j][0], s[2 * j][1]);
          const uint32_t a1 = pack2(s[2 * j][2], s[2 * j][3]);
          const uint32_t a2 = pack2(s[2 * j + 1][0], s[2 * j + 1][1]);
          const uint32_t a3 = pack2(s[2 * j + 1][2], s[2 * j + 1][3]);
          const int vr = k0 + 16 * j + (lane & 15);
#pragma unroll
          for (int dt = 0; dt < 8; dt += 2) {
            uint32_t b0, b1, b2, b3;
            ldsm_x4_t(swz(vb, vr, dt + (lane >> 4)), b0, b1, b2, b3);
            mma16816(o[dt], a0, a1, a2, a3, b0, b1);
            mma16816(o[dt + 1], a0, a1, a2, a3, b2, b3);
          }
        }
      }
    }
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    const float i0 = 1.0f / l0, i1 = 1.0f / l1;
    // this warp's 16 rows of Q are no longer read by anyone: stage the output there
    const int r0 = q0 + (lane >> 2);
#pragma unroll
    for (int dt = 0; dt < 8; ++dt) {
      const uint32_t off = 4u * (lane & 3);
      asm volatile("st.shared.b32 [%0], %1;" ::"r"(swz(qb, r0, dt) + off), "r"(pack2(o[dt][0] * i0, o[dt][1] * i0)));
      asm volatile("st.shared.b32 [%0], %1;" ::"r"(swz(qb, r0 + 8, dt) + off), "r"(pack2(o[dt][2] * i1, o[dt][3] * i1)));
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int rr = q0 + (lane >> 3) + 4 * i, c = lane & 7;
      if (rr < n) {
        uint4 v;
        asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                     : "r"(swz(qb, rr, c)));
        *reinterpret_cast<uint4*>(out + ((size_t)bser * n + rr) * ldo + h * DH + c * 8) = v;
      }
    }
    __syncwarp();
    // the warp that completes an item's last tile refills its buffer
    int last = 0;
    if (lane == 0) {
      __threadfence_block();
      last = atomicAdd(&done[b], 1) == nqt - 1;
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (last) {
      if (lane == 0) done[b] = 0;
      if (li + a.nbufs < my_items) issue(li + a.nbufs);
    }
  }
}

// ---------------------------------------------------------------------------
// group attention for groups of <= 16 series on the tensor cores (bf16)
// ---------------------------------------------------------------------------
// One CTA per (time step, group), one warp per head.  The group's Q, K and V
// rows (all heads) are staged in shared memory with cp.async; rows past the
// group's size read a zero row.  Per head: S = Q K^T as mma.sync m16n8k16
// (M = 16 query rows, N = 8 or 16 keys, K = 64), the softmax on the
// accumulator fragments (quad shuffles), P re-packed from the accumulators
// as the A fragment, split into two bf16 parts (hi + lo) so that it keeps
// about 16 significant bits, and O = P V (K = 16 keys, N = 64 in blocks of
// 8, V read with ldmatrix.trans).  Masking as attn_group_small_kernel: a masked key
// scores -1e30, keys past the group -inf.  The scalar kernel unpacked each
// bf16 Q/K/V element once per use (the ALU bound it ran at).
constexpr int kGroupMmaMaxN = 16, kGroupMmaMaxHeads = 16;

__global__ void __launch_bounds__(32 * kGroupMmaMaxHeads)
attn_group_mma_kernel(const bf16* __restrict__ qkv, int ld, int qcol, int kcol, int vcol, bf16* __restrict__ out,
                      int ldo, const uint8_t* __restrict__ tok, SetInfo si, int heads) {
  pdl_launch_dependents();
  pdl_wait();
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const SetGeom g = set_geom(si, blockIdx.x);
  const int n = g.n;
  if (n <= 0) return;
  const int HD = heads * DH;
  const int pitch = HD * 2 + 16;  // bytes per staged row: +16 keeps ldmatrix rows on distinct banks
  const uint32_t sb = (uint32_t)__cvta_generic_to_shared(smem_raw);
  const uint32_t zero_row = sb + 3u * (uint32_t)n * (uint32_t)pitch;
  float* kb = reinterpret_cast<float*>(smem_raw + (size_t)(3 * n + 1) * pitch);
  const int tid = threadIdx.x;
  const int cpr = HD / 8;  // 16-byte chunks per row and matrix
  // a warp per (matrix, row), its lanes along the row
  for (int wr = tid >> 5; wr < 3 * n; wr += (int)(blockDim.x >> 5)) {
    const int mtx = wr >= 2 * n ? 2 : wr >= n ? 1 : 0, i = wr - mtx * n;
    const bf16* src = qkv + (size_t)g.row(i, si.S) * ld + (mtx == 0 ? qcol : mtx == 1 ? kcol : vcol);
    const uint32_t dst = sb + (uint32_t)(wr * pitch);
    for (int c = tid & 31; c < cpr; c += 32)
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst + 16u * c), "l"(src + 8 * c) : "memory");
  }
  for (int c = tid; c < cpr; c += blockDim.x)
    asm volatile("st.shared.v4.b32 [%0], {%1,%1,%1,%1};" ::"r"(zero_row + 16u * c), "r"(0u) : "memory");
  if (tid < kGroupMmaMaxN)
    kb[tid] = tid < n ? (tok[g.row(tid, si.S)] ? 0.0f : kMaskedScore) : -INFINITY;
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();

  const int h = tid >> 5, lane = tid & 31;
  if (h >= heads) return;
  const int gq = lane >> 2, tq = lane & 3;  // fragment row group and column pair
  const uint32_t qbase = sb, kbase = sb + (uint32_t)(n * pitch), vbase = sb + (uint32_t)(2 * n * pitch);
  auto row_addr = [&](uint32_t base, int r) -> uint32_t {
    return r < n ? base + (uint32_t)(r * pitch) : zero_row;
  };
  const bool two = n > 8;  // a second block of 8 keys
  // ---- S = Q K^T ----
  float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  {
    const int ar = lane & 15, ac = (lane >> 4) * 8;                  // A: rows 0-15, column halves
    const int bk = (lane & 7) + ((lane >> 4) << 3), bc = ((lane >> 3) & 1) * 8;  // B: key rows, dim halves
    const uint32_t a_row = row_addr(qbase, ar), b_row = row_addr(kbase, bk);
#pragma unroll
    for (int ks = 0; ks < DH / 16; ++ks) {
      const int d0 = h * DH + 16 * ks;
      uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
      ldsm_x4(a_row + 2u * (uint32_t)(d0 + ac), a0, a1, a2, a3);
      ldsm_x4(b_row + 2u * (uint32_t)(d0 + bc), b0, b1, b2, b3);
      mma16816(s[0], a0, a1, a2, a3, b0, b1);
      if (two) mma16816(s[1], a0, a1, a2, a3, b2, b3);
    }
  }
  // ---- softmax over the keys of rows gq and gq + 8 ----
  float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
  for (int nb = 0; nb < 2; ++nb) {
    const float k0 = kb[8 * nb + 2 * tq], k1 = kb[8 * nb + 2 * tq + 1];
    s[nb][0] = fmaf(s[nb][0], kLog2e, k0);
    s[nb][1] = fmaf(s[nb][1], kLog2e, k1);
    s[nb][2] = fmaf(s[nb][2], kLog2e, k0);
    s[nb][3] = fmaf(s[nb][3], kLog2e, k1);
    mx0 = fmaxf(mx0, fmaxf(s[nb][0], s[nb][1]));
    mx1 = fmaxf(mx1, fmaxf(s[nb][2], s[nb][3]));
  }
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
  // P as the sum of two bf16 fragments (P = hi + lo, about 16 significant
  // bits) so that P V keeps the precision of the fp32 weights
  float l0 = 0.f, l1 = 0.f;
  uint32_t pa[4], pl[4];
  auto split = [](float x, float y, uint32_t& hi, uint32_t& lo) {
    hi = pack2(x, y);
    const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&hi);
    lo = pack2(x - __bfloat162float(h.x), y - __bfloat162float(h.y));
  };
#pragma unroll
  for (int nb = 0; nb < 2; ++nb) {
    const float p0 = exp2f(s[nb][0] - mx0), p1 = exp2f(s[nb][1] - mx0);
    const float p2 = exp2f(s[nb][2] - mx1), p3 = exp2f(s[nb][3] - mx1);
    l0 += p0 + p1;
    l1 += p2 + p3;
    split(p0, p1, pa[2 * nb], pl[2 * nb]);          // row gq,     keys 8 nb + 2 tq ..
    split(p2, p3, pa[2 * nb + 1], pl[2 * nb + 1]);  // row gq + 8
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = 1.0f / l0, inv1 = 1.0f / l1;
  // ---- O = P V, 8 dims at a time ----
  const int vk = (lane & 7) + (((lane >> 3) & 1) << 3), vc = (lane >> 4) * 8;  // key rows, dim-block pair
  const uint32_t v_row = row_addr(vbase, vk);
  const int r0 = gq, r1 = gq + 8;
  bf16* o0 = r0 < n ? out + (size_t)g.row(r0, si.S) * ldo + h * DH : nullptr;
  bf16* o1 = r1 < n ? out + (size_t)g.row(r1, si.S) * ldo + h * DH : nullptr;
#pragma unroll
  for (int dn = 0; dn < DH / 8; dn += 2) {
    uint32_t b0, b1, b2, b3;
    ldsm_x4_t(v_row + 2u * (uint32_t)(h * DH + 8 * dn + vc), b0, b1, b2, b3);
    float o[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    mma16816(o[0], pl[0], pl[1], pl[2], pl[3], b0, b1);
    mma16816(o[1], pl[0], pl[1], pl[2], pl[3], b2, b3);
    mma16816(o[0], pa[0], pa[1], pa[2], pa[3], b0, b1);
    mma16816(o[1], pa[0], pa[1], pa[2], pa[3], b2, b3);
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int c = 8 * (dn + e) + 2 * tq;
      if (o0) *reinterpret_cast<uint32_t*>(o0 + c) = pack2(o[e][0] * inv0, o[e][1] * inv0);
      if (o1) *reinterpret_cast<uint32_t*>(o1 + c) = pack2(o[e][2] * inv1, o[e][3] * inv1);
    }
  }
}

inline size_t group_mma_smem(int n, int heads) {
  return (size_t)(3 * n + 1) * (heads * DH * 2 + 16) + kGroupMmaMaxN * sizeof(float);
}

inline size_t small_group_smem(int n, int heads, size_t esz) {
  return 3 * (size_t)n * (heads * DH * esz + 16) + ((size_t)heads * n * n + n) * sizeof(float);
}

template <typename T>
int set_small_group_attr(size_t bytes) {
  if (bytes <= 48 * 1024) return CC2_OK;
  CC2_CUDA(cudaFuncSetAttribute(attn_group_small_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
  return CC2_OK;
}

}  // namespace

int launch_attention(int dtype, int mode, const void* qkv, int ld, int qcol, int kcol, int vcol, void* out,
                     int ldo, const uint8_t* tok, int num_sets, int S, int heads, int dkv,
                     const int32_t* members, const int32_t* offsets, int num_groups, int max_group,
                     const float* rope_cs, cudaStream_t st) {
  CC2_REQUIRE(dkv == DH, "attention: d_kv must be %d (got %d)", DH, dkv);
  CC2_REQUIRE(mode == 0 || mode == 1, "attention: bad mode");
  CC2_REQUIRE(qkv && out && tok && num_sets > 0 && S > 0 && heads > 0, "attention: bad args");
  CC2_REQUIRE(mode == 0 || (members && offsets && num_groups > 0 && max_group > 0),
              "attention: group mode needs members/offsets");
  SetInfo si{mode, S, members, offsets, num_groups};
  const int nmax = mode == 0 ? S : max_group;
  const float2* cs = (const float2*)rope_cs;
  if (dtype == CC2_BF16) {
    CC2_REQUIRE(ld % 8 == 0 && ldo % 8 == 0 && qcol % 8 == 0 && kcol % 8 == 0 && vcol % 8 == 0,
                "attention(bf16): columns/pitches must be multiples of 8");
    const int npad = (nmax + 15) & ~15;
    const int nqt = (nmax + 15) / 16;
    const int rounds = (nqt + kSetMaxWarps - 1) / kSetMaxWarps;
    const int warps = (nqt + rounds - 1) / rounds;
    const size_t smem = set_kernel_smem(npad);
    // persistent TMA kernel: time mode with RoPE already applied (the forward's case)
    const int nbox = (S + 255) / 256;
    const int npad_t = (S + 16 * nbox - 1) / (16 * nbox) * (16 * nbox);
    const size_t pbuf = align_up((size_t)npad_t * (3 * 128 + sizeof(float)), 1024);
    const int pbufs = (int)std::min<size_t>(kPBufs, kPSmemLimit / pbuf);
    const bool aligned = ((uintptr_t)qkv & 15u) == 0 && (ld * 2) % 16 == 0;
    // (sets of fewer than 8 query tiles run faster in the whole-set kernel below)
    const bool tc_pick = g_attn_variant == 2 || (g_attn_variant == 0 && S >= 112);
    if (mode == 0 && !cs && g_attn_variant == 0 && attn_pack_tc_supported(S, ld, ldo, qkv, out)) {
      // short sets (16 < S <= 64): two per tcgen05 tile
      int* err = nullptr;
      CC2_CUDA(cudaGetSymbolAddress((void**)&err, g_attn_error));
      return launch_attn_pack_tc(qkv, ld, qcol, kcol, vcol, out, ldo, tok, num_sets, S, heads, err, st);
    } else if (mode == 0 && !cs && tc_pick && ((uintptr_t)out & 15u) == 0 && attn_tc_supported(S, ld, ldo, qkv)) {
      int* err = nullptr;
      CC2_CUDA(cudaGetSymbolAddress((void**)&err, g_attn_error));
      return launch_attn_tc(qkv, ld, qcol, kcol, vcol, out, ldo, tok, num_sets, S, heads, err, st);
    } else if (mode == 0 && !cs && (g_attn_variant == 0 || g_attn_variant == 2) &&
               attn_tc_long_supported(S, ld, ldo, qkv, out)) {
      int* err = nullptr;
      CC2_CUDA(cudaGetSymbolAddress((void**)&err, g_attn_error));
      return launch_attn_tc_long(qkv, ld, qcol, kcol, vcol, out, ldo, tok, num_sets, S, heads, err, st);
    } else if (mode == 0 && !cs && g_attn_variant != 3 && pbufs >= 1 && aligned && (S + 15) / 16 >= 8) {
      CUtensorMap map;
      CC2_TRY(encode_bf16_map(&map, qkv, ld, num_sets * S, ld, 64, npad_t / nbox));
      PersistArgs pa{S, npad_t, heads, num_sets * heads, qcol, kcol, vcol, npad_t / nbox, nbox, pbufs, pbuf};
      const size_t smem_p = (size_t)pbufs * pbuf + 1024;
      static unsigned long long attr_p = 0;  // one bit per device
      int dev = 0;
      CC2_CUDA(cudaGetDevice(&dev));
      if (dev >= 64 || !((attr_p >> dev) & 1ull)) {
        CC2_CUDA(cudaFuncSetAttribute(attn_persist_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)(kPSmemLimit + 1024)));
        if (dev < 64) attr_p |= 1ull << dev;
      }
      int* err = nullptr;
      CC2_CUDA(cudaGetSymbolAddress((void**)&err, g_attn_error));
      const int grid = std::min(num_sets * heads, num_sms());
      CC2_CUDA(launch_k(attn_persist_kernel, grid, kPWarps * 32, smem_p, st, map, (bf16*)out, ldo, tok, pa, err));
    } else if (mode == 1 && max_group <= kGroupMmaMaxN && heads <= kGroupMmaMaxHeads && g_attn_variant != 1 &&
               ((uintptr_t)qkv & 15u) == 0 && ((uintptr_t)out & 3u) == 0) {
      const size_t sm = group_mma_smem(max_group, heads);
      static unsigned long long attr_g = 0;  // one bit per device
      int dev = 0;
      CC2_CUDA(cudaGetDevice(&dev));
      if (dev >= 64 || !((attr_g >> dev) & 1ull)) {
        CC2_CUDA(cudaFuncSetAttribute(attn_group_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)group_mma_smem(kGroupMmaMaxN, kGroupMmaMaxHeads)));
        if (dev < 64) attr_g |= 1ull << dev;
      }
      CC2_CUDA(launch_k(attn_group_mma_kernel, num_sets, 32 * heads, sm, st, (const bf16*)qkv, ld, qcol, kcol, vcol,
                        (bf16*)out, ldo, tok, si, heads));
    } else if (mode == 1 && max_group <= kSmallGroupMax) {
      const size_t sm = small_group_smem(max_group, heads, sizeof(bf16));
      CC2_TRY(set_small_group_attr<bf16>(sm));
      CC2_CUDA(launch_k(attn_group_small_kernel<bf16>, num_sets, 256, sm, st, (const bf16*)qkv, ld, qcol, kcol, vcol, (bf16*)out,
                                                               ldo, tok, si, heads));
    } else if (mode == 1 && max_group <= SK) {
      dim3 grid((nmax + SQ - 1) / SQ, heads, num_sets);
      CC2_CUDA(launch_k(attn_simt_kernel<bf16, false>, grid, 128, 0, st, (const bf16*)qkv, ld, qcol, kcol, vcol, (bf16*)out,
                                                          ldo, tok, cs, si));
    } else if (smem <= kSetSmemLimit) {
      static unsigned long long attr_done = 0;  // one bit per device
      int dev = 0;
      CC2_CUDA(cudaGetDevice(&dev));
      if (dev >= 64 || !((attr_done >> dev) & 1ull)) {
        CC2_CUDA(cudaFuncSetAttribute(attn_set_kernel<true, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)kSetSmemLimit));
        CC2_CUDA(cudaFuncSetAttribute(attn_set_kernel<false, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)kSetSmemLimit));
        if (dev < 64) attr_done |= 1ull << dev;
      }
      dim3 grid(heads, num_sets);
      const bool rope_k = mode == 0 && cs;
      if (nmax <= 48 && warps * 32 <= 128) {  // one 48-key tile; smem < 48 KB needs no attribute
        if (rope_k)
          CC2_CUDA(launch_k(attn_set_kernel<true, 48>, grid, warps * 32, smem, st, (const bf16*)qkv, ld, qcol, kcol,
                            vcol, (bf16*)out, ldo, tok, cs, si));
        else
          CC2_CUDA(launch_k(attn_set_kernel<false, 48>, grid, warps * 32, smem, st, (const bf16*)qkv, ld, qcol, kcol,
                            vcol, (bf16*)out, ldo, tok, cs, si));
      } else if (rope_k) {
        CC2_CUDA(launch_k(attn_set_kernel<true, 64>, grid, warps * 32, smem, st, (const bf16*)qkv, ld, qcol, kcol, vcol,
                          (bf16*)out, ldo, tok, cs, si));
      } else {
        CC2_CUDA(launch_k(attn_set_kernel<false, 64>, grid, warps * 32, smem, st, (const bf16*)qkv, ld, qcol, kcol,
                          vcol, (bf16*)out, ldo, tok, cs, si));
      }
    } else {
      dim3 grid((nmax + QT - 1) / QT, heads, num_sets);
      if (mode == 0 && cs)
        CC2_CUDA(launch_k(attn_mma_kernel<true>, grid, 128, 0, st, (const bf16*)qkv, ld, qcol, kcol, vcol, (bf16*)out, ldo,
                                                    tok, cs, si));
      else
        CC2_CUDA(launch_k(attn_mma_kernel<false>, grid, 128, 0, st, (const bf16*)qkv, ld, qcol, kcol, vcol, (bf16*)out, ldo,
                                                     tok, cs, si));
    }
  } else if (dtype == CC2_F32 && mode == 1 && max_group <= kSmallGroupMax) {
    const size_t sm = small_group_smem(max_group, heads, sizeof(float));
    CC2_TRY(set_small_group_attr<float>(sm));
    CC2_CUDA(launch_k(attn_group_small_kernel<float>, num_sets, 256, sm, st, (const float*)qkv, ld, qcol, kcol, vcol, (float*)out,
                                                              ldo, tok, si, heads));
  } else if (dtype == CC2_F32) {
    dim3 grid((nmax + SQ - 1) / SQ, heads, num_sets);
    if (mode == 0 && cs)
      CC2_CUDA(launch_k(attn_simt_kernel<float, true>, grid, 128, 0, st, (const float*)qkv, ld, qcol, kcol, vcol, (float*)out,
                                                          ldo, tok, cs, si));
    else
      CC2_CUDA(launch_k(attn_simt_kernel<float, false>, grid, 128, 0, st, (const float*)qkv, ld, qcol, kcol, vcol, (float*)out,
                                                           ldo, tok, cs, si));
  } else {
    CC2_REQUIRE(false, "attention: unsupported dtype %d", dtype);
  }
  CC2_CHECK_LAUNCH();
  return CC2_OK;
}

}  // namespace cc2
