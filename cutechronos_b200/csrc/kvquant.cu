// TurboQuant-style fake quantisation of the time-attention K and V vectors
// (the reference's CuteChronos2Model.enable_turboquant_kv hook,
// cutechronos/model.py:615-667, quantiser tubroquant/quantizer.py:119-178),
// run in place on the packed [Q|K|V] token rows between the QKV GEMM and the
// time attention.
//
// One warp per (token row, head): lane i holds coordinates i and i + 32 of
// the 64-value vector.  Optionally RoPE is first applied to Q and K (the fp32
// forward, whose attention kernel otherwise rotates them itself), then each of
// K and V with a quantiser:
//   norm -> unit vector -> rotation (Hadamard: gather by the permutation,
//   random signs, butterflies of width 1..32 by lane shuffles, x 1/8; dense:
//   64x64 matrix from shared memory) -> bucket of each coordinate (binary
//   search of the sorted boundaries) -> centroid -> inverse rotation
//   [-> prod mode: residual, its norm, signs of the Gaussian projection,
//   back-projection scaled by sqrt(pi/2)/64 * residual norm] -> times the
//   norm as stored (float16 / bfloat16 / float32 round trip).
// Squared error and max |error| against the input are accumulated per tensor
// for the reference's statistics (atomics: the statistics' last bits depend
// on timing; the quantised values do not).
#include "common.cuh"

namespace cc2 {
namespace {

constexpr int kWarps = 8;

// Per-quantiser tables staged in shared memory.
struct QTab {
  float signs[64];
  int perm[64], inv_perm[64];
  float codebook[256];
  float bounds[256];
  float* mat;   // dense rotation, row-major [e][d] (y[e] = sum_d x[d] mat[e][d])
  float* matT;  // its transpose [d][e]
  float* proj;  // QJL projection [e][d]
  float* projT; // [d][e]
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// value of coordinate `src` (0..63) of a vector held as (lo = [lane], hi = [lane + 32])
__device__ __forceinline__ float gather(float lo, float hi, int src) {
  const float a = __shfl_sync(0xffffffffu, lo, src & 31);
  const float b = __shfl_sync(0xffffffffu, hi, src & 31);
  return src < 32 ? a : b;
}

// in-place Walsh-Hadamard butterflies of width 1, 2, ..., 32 (a + b | a - b)
__device__ __forceinline__ void fwht(float& lo, float& hi, int lane) {
#pragma unroll
  for (int h = 1; h < 32; h <<= 1) {
    const float plo = __shfl_xor_sync(0xffffffffu, lo, h);
    const float phi = __shfl_xor_sync(0xffffffffu, hi, h);
    const bool upper = (lane & h) != 0;
    lo = upper ? __fsub_rn(plo, lo) : __fadd_rn(lo, plo);
    hi = upper ? __fsub_rn(phi, hi) : __fadd_rn(hi, phi);
  }
  const float a = lo, b = hi;
  lo = __fadd_rn(a, b);
  hi = __fsub_rn(a, b);
}

// y = M-product of each of NV vectors (lo, hi): y[e] = sum_d v[d] * A[d][e]
// with A given transposed ([d][e]); the vectors are broadcast through
// `scratch` ([NV][64]) and every row of A read once serves all NV vectors.
template <int NV>
__device__ __forceinline__ void matvec(float (&lo)[NV], float (&hi)[NV], const float* AT, float (*scratch)[64],
                                       int lane) {
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    scratch[i][lane] = lo[i];
    scratch[i][lane + 32] = hi[i];
  }
  __syncwarp();
  // lane owns output columns 2*lane and 2*lane+1 (one 8-byte table load per d);
  // the inputs are read four d at a time; each column still sums d = 0..63 in order
  float a[NV], b[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) a[i] = b[i] = 0.0f;
  const float2* at2 = reinterpret_cast<const float2*>(AT) + lane;
#pragma unroll 2
  for (int d = 0; d < 64; d += 4) {
    float2 t[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) t[j] = at2[(d + j) * 32];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const float4 v = *reinterpret_cast<const float4*>(&scratch[i][d]);
      a[i] = fmaf(v.x, t[0].x, a[i]);
      b[i] = fmaf(v.x, t[0].y, b[i]);
      a[i] = fmaf(v.y, t[1].x, a[i]);
      b[i] = fmaf(v.y, t[1].y, b[i]);
      a[i] = fmaf(v.z, t[2].x, a[i]);
      b[i] = fmaf(v.z, t[2].y, b[i]);
      a[i] = fmaf(v.w, t[3].x, a[i]);
      b[i] = fmaf(v.w, t[3].y, b[i]);
    }
  }
  __syncwarp();
#pragma unroll
  for (int i = 0; i < NV; ++i) *reinterpret_cast<float2*>(&scratch[i][2 * lane]) = make_float2(a[i], b[i]);
  __syncwarp();
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    lo[i] = scratch[i][lane];
    hi[i] = scratch[i][lane + 32];
  }
  __syncwarp();
}

__device__ __forceinline__ float norm_storage(float v, int kind) {
  if (kind == 0) return __half2float(__float2half_rn(v));
  if (kind == 1) return __bfloat162float(__float2bfloat16_rn(v));
  return v;
}

__device__ __forceinline__ int bucket(const float* b, int nb, float y) {
  int lo = 0, hi = nb;  // number of boundaries strictly below y
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (b[mid] < y) lo = mid + 1; else hi = mid;
  }
  return lo;
}

// Quantise NV 64-value vectors in registers (lo, hi); returns the squared
// error and max |error| contributions of this lane.  Every vector goes through
// the same arithmetic as alone; NV only interleaves them.
template <int NV>
__device__ void quantise(float (&lo)[NV], float (&hi)[NV], const cc2_kvq& p, const QTab& t, float (*scratch)[64],
                         int lane, float& sse, float& mx) {
  const int mse_bits = p.mode == 0 ? p.bits : max(p.bits - 1, 0);
  float x0[NV], x1[NV], norm[NV], u0[NV], u1[NV], m0[NV], m1[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    x0[i] = lo[i];
    x1[i] = hi[i];
    norm[i] = sqrtf(warp_sum(x0[i] * x0[i] + x1[i] * x1[i]));
    const float safe = fmaxf(norm[i], 1e-12f);
    u0[i] = norm[i] > 0.0f ? x0[i] / safe : 0.0f;
    u1[i] = norm[i] > 0.0f ? x1[i] / safe : 0.0f;
    m0[i] = m1[i] = 0.0f;  // unit-vector reconstruction from the centroids
  }
  if (mse_bits > 0) {
    float y0[NV], y1[NV];
    if (p.rotation == 0) {
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        y0[i] = gather(u0[i], u1[i], t.perm[lane]) * t.signs[lane];
        y1[i] = gather(u0[i], u1[i], t.perm[lane + 32]) * t.signs[lane + 32];
        fwht(y0[i], y1[i], lane);
        y0[i] *= 0.125f;
        y1[i] *= 0.125f;
      }
    } else {
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        y0[i] = u0[i];
        y1[i] = u1[i];
      }
      matvec<NV>(y0, y1, t.matT, scratch, lane);
    }
    const int nb = (1 << mse_bits) - 1;
    float c0[NV], c1[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      c0[i] = t.codebook[bucket(t.bounds, nb, y0[i])];
      c1[i] = t.codebook[bucket(t.bounds, nb, y1[i])];
    }
    if (p.rotation == 0) {
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        fwht(c0[i], c1[i], lane);
        c0[i] = (c0[i] * 0.125f) * t.signs[lane];
        c1[i] = (c1[i] * 0.125f) * t.signs[lane + 32];
        m0[i] = gather(c0[i], c1[i], t.inv_perm[lane]);
        m1[i] = gather(c0[i], c1[i], t.inv_perm[lane + 32]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        m0[i] = c0[i];
        m1[i] = c1[i];
      }
      matvec<NV>(m0, m1, t.mat, scratch, lane);  // inverse: x[d] = sum_e y[e] mat[e][d]
    }
  }
  float r0[NV], r1[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    r0[i] = m0[i];
    r1[i] = m1[i];
  }
  if (p.mode == 1) {
    float e0[NV], e1[NV], rn[NV], s0[NV], s1[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      e0[i] = u0[i] - m0[i];
      e1[i] = u1[i] - m1[i];
      rn[i] = norm_storage(sqrtf(warp_sum(e0[i] * e0[i] + e1[i] * e1[i])), p.norm_dtype);
      s0[i] = s1[i] = 1.0f;
    }
    if (p.bits > 0) {
      float q0[NV], q1[NV];
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        q0[i] = e0[i];
        q1[i] = e1[i];
      }
      matvec<NV>(q0, q1, t.projT, scratch, lane);  // sr[e] = sum_d residual[d] proj[e][d]
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        s0[i] = q0[i] >= 0.0f ? 1.0f : -1.0f;
        s1[i] = q1[i] >= 0.0f ? 1.0f : -1.0f;
      }
    }
    matvec<NV>(s0, s1, t.proj, scratch, lane);  // direction[d] = sum_e sign[e] proj[e][d]
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const float coeff = (float)(1.2533141373155003 / 64.0) * rn[i];  // sqrt(pi / 2) / dim
      r0[i] = m0[i] + coeff * s0[i];
      r1[i] = m1[i] + coeff * s1[i];
    }
  }
  sse = 0.0f;
  mx = 0.0f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const float ns = norm_storage(norm[i], p.norm_dtype);
    lo[i] = r0[i] * ns;
    hi[i] = r1[i] * ns;
    const float d0 = lo[i] - x0[i], d1 = hi[i] - x1[i];
    sse += d0 * d0 + d1 * d1;
    mx = fmaxf(mx, fmaxf(fabsf(d0), fabsf(d1)));
  }
}

// floats of shared memory a quantiser's dense tables take (matrix and its
// transpose for the dense rotation, projection and its transpose in prod mode)
__host__ __device__ __forceinline__ int dense_floats(const cc2_kvq& p) {
  return (p.rotation == 1 ? 2 * 4096 : 0) + (p.mode == 1 ? 2 * 4096 : 0);
}

__device__ void load_tab(QTab& t, const cc2_kvq& p, float* dense, int tid, int nthreads) {
  const int mse_bits = p.mode == 0 ? p.bits : max(p.bits - 1, 0);
  const int ncb = 1 << mse_bits, nb = ncb - 1;
  for (int i = tid; i < 64; i += nthreads) {
    if (p.rotation == 0) {
      t.signs[i] = p.signs[i];
      t.perm[i] = p.perm[i];
      t.inv_perm[i] = p.inv_perm[i];
    }
  }
  for (int i = tid; i < ncb; i += nthreads) t.codebook[i] = mse_bits > 0 ? p.codebook[i] : 0.0f;
  for (int i = tid; i < nb; i += nthreads) t.bounds[i] = p.boundaries[i];
  // table addresses are computed by every thread in registers; only thread 0
  // publishes them in the shared struct (read after the caller's barrier)
  float* next = dense;
  float* mat = nullptr;
  float* matT = nullptr;
  float* proj = nullptr;
  float* projT = nullptr;
  if (p.rotation == 1) {
    mat = next;
    matT = next + 4096;
    next += 8192;
  }
  if (p.mode == 1) {
    proj = next;
    projT = next + 4096;
  }
  if (tid == 0) {
    t.mat = mat;
    t.matT = matT;
    t.proj = proj;
    t.projT = projT;
  }
  for (int i = tid; i < 4096; i += nthreads) {
    const int r = i >> 6, c = i & 63;
    if (p.rotation == 1) {
      mat[i] = p.matrix[i];
      matT[c * 64 + r] = p.matrix[i];
    }
    if (p.mode == 1) {
      proj[i] = p.proj[i];
      projT[c * 64 + r] = p.proj[i];
    }
  }
}

// NV: vectors per warp (consecutive heads of one token row)
template <typename T, int NV>
__global__ void __launch_bounds__(kWarps * 32, 4)  // 4 CTAs (32 warps) per SM: the kernel is latency-bound
kv_quant_kernel(T* __restrict__ qkv, int ld, int rows, int q_col, int k_col, int v_col, int heads, cc2_kvq kp,
                cc2_kvq vp, int has_k, int has_v, const float2* __restrict__ rope, int rope_period,
                float* __restrict__ stats) {
  pdl_launch_dependents();
  pdl_wait();
  extern __shared__ __align__(16) float dyn[];
  __shared__ QTab tab[2];
  __shared__ __align__(16) float scratch[kWarps][NV][64];
  __shared__ float part[kWarps][4];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (has_k) load_tab(tab[0], kp, dyn, tid, blockDim.x);
  if (has_v) load_tab(tab[1], vp, dyn + (has_k ? dense_floats(kp) : 0), tid, blockDim.x);
  __syncthreads();
  float ksse = 0.0f, kmx = 0.0f, vsse = 0.0f, vmx = 0.0f;
  const int groups = heads / NV;
  const long long total = (long long)rows * groups;
  for (long long v = (long long)blockIdx.x * kWarps + warp; v < total; v += (long long)gridDim.x * kWarps) {
    const int row = (int)(v / groups), h0 = (int)(v % groups) * NV;
    T* base = qkv + (size_t)row * ld + h0 * 64 + lane;
    float k0[NV], k1[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      T* kq = base + k_col + i * 64;
      k0[i] = Elem<T>::to_f(kq[0]);
      k1[i] = Elem<T>::to_f(kq[32]);
    }
    if (rope != nullptr) {  // rotate-half RoPE at position row % rope_period
      const float2 cs = rope[(size_t)(row % rope_period) * 32 + lane];
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        T* qq = base + q_col + i * 64;
        const float q0 = Elem<T>::to_f(qq[0]), q1 = Elem<T>::to_f(qq[32]);
        qq[0] = Elem<T>::from_f(q0 * cs.x - q1 * cs.y);
        qq[32] = Elem<T>::from_f(q1 * cs.x + q0 * cs.y);
        const float r0 = k0[i] * cs.x - k1[i] * cs.y, r1 = k1[i] * cs.x + k0[i] * cs.y;
        // the quantiser sees K as the attention would (rounded to the storage type)
        k0[i] = Elem<T>::to_f(Elem<T>::from_f(r0));
        k1[i] = Elem<T>::to_f(Elem<T>::from_f(r1));
      }
    }
    if (has_k) {
      float s, m;
      quantise<NV>(k0, k1, kp, tab[0], scratch[warp], lane, s, m);
      ksse += s;
      kmx = fmaxf(kmx, m);
    }
    if (has_k || rope != nullptr) {
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        T* kq = base + k_col + i * 64;
        kq[0] = Elem<T>::from_f(k0[i]);
        kq[32] = Elem<T>::from_f(k1[i]);
      }
    }
    if (has_v) {
      float v0[NV], v1[NV];
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        T* vq = base + v_col + i * 64;
        v0[i] = Elem<T>::to_f(vq[0]);
        v1[i] = Elem<T>::to_f(vq[32]);
      }
      float s, m;
      quantise<NV>(v0, v1, vp, tab[1], scratch[warp], lane, s, m);
      vsse += s;
      vmx = fmaxf(vmx, m);
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        T* vq = base + v_col + i * 64;
        vq[0] = Elem<T>::from_f(v0[i]);
        vq[32] = Elem<T>::from_f(v1[i]);
      }
    }
  }
  if (stats == nullptr) return;
  ksse = warp_sum(ksse);
  vsse = warp_sum(vsse);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    kmx = fmaxf(kmx, __shfl_xor_sync(0xffffffffu, kmx, o));
    vmx = fmaxf(vmx, __shfl_xor_sync(0xffffffffu, vmx, o));
  }
  if (lane == 0) {
    part[warp][0] = ksse;
    part[warp][1] = kmx;
    part[warp][2] = vsse;
    part[warp][3] = vmx;
  }
  __syncthreads();
  if (tid == 0) {
    float a = 0.0f, b = 0.0f, c = 0.0f, e = 0.0f;
    for (int w = 0; w < kWarps; ++w) {
      a += part[w][0];
      b = fmaxf(b, part[w][1]);
      c += part[w][2];
      e = fmaxf(e, part[w][3]);
    }
    atomicAdd(&stats[0], a);
    atomicMax(reinterpret_cast<int*>(&stats[1]), __float_as_int(b));  // non-negative floats order as ints
    atomicAdd(&stats[2], c);
    atomicMax(reinterpret_cast<int*>(&stats[3]), __float_as_int(e));
  }
}

int check_kvq(const cc2_kvq* p, const char* which) {
  if (p == nullptr) return CC2_OK;
  CC2_REQUIRE(p->mode == 0 || p->mode == 1, "kv_quant(%s): mode must be 0 (mse) or 1 (prod)", which);
  const int mse_bits = p->mode == 0 ? p->bits : std::max(p->bits - 1, 0);
  CC2_REQUIRE(p->bits >= 0 && mse_bits <= 8, "kv_quant(%s): bits %d out of range", which, p->bits);
  CC2_REQUIRE(p->rotation == 0 || p->rotation == 1, "kv_quant(%s): rotation must be 0 or 1", which);
  CC2_REQUIRE(p->norm_dtype >= 0 && p->norm_dtype <= 2, "kv_quant(%s): norm dtype must be 0, 1 or 2", which);
  CC2_REQUIRE(p->rotation != 0 || (p->signs && p->perm && p->inv_perm), "kv_quant(%s): Hadamard tables", which);
  CC2_REQUIRE(p->rotation != 1 || p->matrix, "kv_quant(%s): rotation matrix", which);
  CC2_REQUIRE(mse_bits == 0 || (p->codebook && p->boundaries), "kv_quant(%s): codebook", which);
  CC2_REQUIRE(p->mode != 1 || p->proj, "kv_quant(%s): projection", which);
  return CC2_OK;
}

}  // namespace

int launch_kv_quant(int dtype, void* qkv, int ld, int rows, int q_col, int k_col, int v_col, int heads,
                    const cc2_kvq* key, const cc2_kvq* value, const float* rope_cs, int rope_period, float* stats,
                    cudaStream_t st) {
  CC2_REQUIRE(qkv && rows > 0 && heads > 0 && ld > 0, "kv_quant: bad arguments");
  CC2_REQUIRE(!rope_cs || rope_period > 0, "kv_quant: rope_period must be positive");
  CC2_TRY(check_kvq(key, "key"));
  CC2_TRY(check_kvq(value, "value"));
  if (!key && !value && !rope_cs) return CC2_OK;
  cc2_kvq kp{}, vp{};
  if (key) kp = *key;
  if (value) vp = *value;
  const size_t smem = ((key ? dense_floats(kp) : 0) + (value ? dense_floats(vp) : 0)) * sizeof(float);
  static unsigned long long attr_done = 0;  // one bit per device
  int dev = 0;
  CC2_CUDA(cudaGetDevice(&dev));
  if (dev >= 64 || !((attr_done >> dev) & 1ull)) {
    const int most = 8 * 4096 * (int)sizeof(float);  // both quantisers dense and prod
    CC2_CUDA(cudaFuncSetAttribute(kv_quant_kernel<__nv_bfloat16, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, most));
    CC2_CUDA(cudaFuncSetAttribute(kv_quant_kernel<__nv_bfloat16, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, most));
    CC2_CUDA(cudaFuncSetAttribute(kv_quant_kernel<float, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, most));
    CC2_CUDA(cudaFuncSetAttribute(kv_quant_kernel<float, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, most));
    if (dev < 64) attr_done |= 1ull << dev;
  }
  const int nv = heads % 4 == 0 ? 4 : 1;  // four heads of a row per warp when the head count allows
  const long long units = (long long)rows * (heads / nv);
  const int grid = (int)std::min<long long>((units + kWarps - 1) / kWarps, 4LL * num_sms());
  const float2* cs = (const float2*)rope_cs;
#define CC2_KVQ(TT, NV_)                                                                                     \
  CC2_CUDA(launch_k(kv_quant_kernel<TT, NV_>, grid, kWarps * 32, smem, st, (TT*)qkv, ld, rows, q_col, k_col,  \
                    v_col, heads, kp, vp, key != nullptr, value != nullptr, cs, rope_period, stats))
  if (dtype == CC2_BF16) {
    if (nv == 4) CC2_KVQ(__nv_bfloat16, 4); else CC2_KVQ(__nv_bfloat16, 1);
  } else if (dtype == CC2_F32) {
    if (nv == 4) CC2_KVQ(float, 4); else CC2_KVQ(float, 1);
  } else {
    CC2_REQUIRE(false, "kv_quant: unsupported dtype %d", dtype);
  }
#undef CC2_KVQ
  CC2_CHECK_LAUNCH();
  return CC2_OK;
}

}  // namespace cc2
