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

// y = M-product of the vector v (lo, hi): y[e] = sum_d v[d] * A[d][e] with A
// given transposed ([d][e]); the vector is broadcast through `scratch`.
__device__ __forceinline__ void matvec(float& lo, float& hi, const float* AT, float* scratch, int lane) {
  scratch[lane] = lo;
  scratch[lane + 32] = hi;
  __syncwarp();
  float a = 0.0f, b = 0.0f;
  for (int d = 0; d < 64; ++d) {
    const float v = scratch[d];
    a = fmaf(v, AT[d * 64 + lane], a);
    b = fmaf(v, AT[d * 64 + lane + 32], b);
  }
  __syncwarp();
  lo = a;
  hi = b;
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

// Quantise one 64-value vector in registers (lo, hi); returns the squared
// error and max |error| contributions of this lane.
__device__ void quantise(float& lo, float& hi, const cc2_kvq& p, const QTab& t, float* scratch, int lane,
                         float& sse, float& mx) {
  const int mse_bits = p.mode == 0 ? p.bits : max(p.bits - 1, 0);
  const float x0 = lo, x1 = hi;
  const float norm = sqrtf(warp_sum(x0 * x0 + x1 * x1));
  const float safe = fmaxf(norm, 1e-12f);
  const float u0 = norm > 0.0f ? x0 / safe : 0.0f, u1 = norm > 0.0f ? x1 / safe : 0.0f;
  float m0 = 0.0f, m1 = 0.0f;  // unit-vector reconstruction from the centroids
  if (mse_bits > 0) {
    float y0, y1;
    if (p.rotation == 0) {
      y0 = gather(u0, u1, t.perm[lane]) * t.signs[lane];
      y1 = gather(u0, u1, t.perm[lane + 32]) * t.signs[lane + 32];
      fwht(y0, y1, lane);
      y0 *= 0.125f;
      y1 *= 0.125f;
    } else {
      y0 = u0;
      y1 = u1;
      matvec(y0, y1, t.matT, scratch, lane);
    }
    const int nb = (1 << mse_bits) - 1;
    float c0 = t.codebook[bucket(t.bounds, nb, y0)], c1 = t.codebook[bucket(t.bounds, nb, y1)];
    if (p.rotation == 0) {
      fwht(c0, c1, lane);
      c0 = (c0 * 0.125f) * t.signs[lane];
      c1 = (c1 * 0.125f) * t.signs[lane + 32];
      m0 = gather(c0, c1, t.inv_perm[lane]);
      m1 = gather(c0, c1, t.inv_perm[lane + 32]);
    } else {
      m0 = c0;
      m1 = c1;
      matvec(m0, m1, t.mat, scratch, lane);  // inverse: x[d] = sum_e y[e] mat[e][d]
    }
  }
  float r0 = m0, r1 = m1;
  if (p.mode == 1) {
    const float e0 = u0 - m0, e1 = u1 - m1;
    const float rn = norm_storage(sqrtf(warp_sum(e0 * e0 + e1 * e1)), p.norm_dtype);
    float s0 = 1.0f, s1 = 1.0f;
    if (p.bits > 0) {
      float q0 = e0, q1 = e1;
      matvec(q0, q1, t.projT, scratch, lane);  // sr[e] = sum_d residual[d] proj[e][d]
      s0 = q0 >= 0.0f ? 1.0f : -1.0f;
      s1 = q1 >= 0.0f ? 1.0f : -1.0f;
    }
    matvec(s0, s1, t.proj, scratch, lane);  // direction[d] = sum_e sign[e] proj[e][d]
    const float coeff = (float)(1.2533141373155003 / 64.0) * rn;  // sqrt(pi / 2) / dim
    r0 = m0 + coeff * s0;
    r1 = m1 + coeff * s1;
  }
  const float ns = norm_storage(norm, p.norm_dtype);
  lo = r0 * ns;
  hi = r1 * ns;
  const float d0 = lo - x0, d1 = hi - x1;
  sse = d0 * d0 + d1 * d1;
  mx = fmaxf(fabsf(d0), fabsf(d1));
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

template <typename T>
__global__ void __launch_bounds__(kWarps * 32)
kv_quant_kernel(T* __restrict__ qkv, int ld, int rows, int q_col, int k_col, int v_col, int heads, cc2_kvq kp,
                cc2_kvq vp, int has_k, int has_v, const float2* __restrict__ rope, int rope_period,
                float* __restrict__ stats) {
  pdl_launch_dependents();
  pdl_wait();
  extern __shared__ __align__(16) float dyn[];
  __shared__ QTab tab[2];
  __shared__ float scratch[kWarps][64];
  __shared__ float part[kWarps][4];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (has_k) load_tab(tab[0], kp, dyn, tid, blockDim.x);
  if (has_v) load_tab(tab[1], vp, dyn + (has_k ? dense_floats(kp) : 0), tid, blockDim.x);
  __syncthreads();
  float ksse = 0.0f, kmx = 0.0f, vsse = 0.0f, vmx = 0.0f;
  const long long total = (long long)rows * heads;
  for (long long v = (long long)blockIdx.x * kWarps + warp; v < total; v += (long long)gridDim.x * kWarps) {
    const int row = (int)(v / heads), h = (int)(v % heads);
    T* base = qkv + (size_t)row * ld + h * 64 + lane;
    T* kq = base + k_col;
    float k0 = Elem<T>::to_f(kq[0]), k1 = Elem<T>::to_f(kq[32]);
    if (rope != nullptr) {  // rotate-half RoPE at position row % rope_period
      const float2 cs = rope[(size_t)(row % rope_period) * 32 + lane];
      T* qq = base + q_col;
      const float q0 = Elem<T>::to_f(qq[0]), q1 = Elem<T>::to_f(qq[32]);
      qq[0] = Elem<T>::from_f(q0 * cs.x - q1 * cs.y);
      qq[32] = Elem<T>::from_f(q1 * cs.x + q0 * cs.y);
      const float r0 = k0 * cs.x - k1 * cs.y, r1 = k1 * cs.x + k0 * cs.y;
      // the quantiser sees K as the attention would (rounded to the storage type)
      k0 = Elem<T>::to_f(Elem<T>::from_f(r0));
      k1 = Elem<T>::to_f(Elem<T>::from_f(r1));
    }
    if (has_k) {
      float s, m;
      quantise(k0, k1, kp, tab[0], scratch[warp], lane, s, m);
      ksse += s;
      kmx = fmaxf(kmx, m);
    }
    if (has_k || rope != nullptr) {
      kq[0] = Elem<T>::from_f(k0);
      kq[32] = Elem<T>::from_f(k1);
    }
    if (has_v) {
      T* vq = base + v_col;
      float v0 = Elem<T>::to_f(vq[0]), v1 = Elem<T>::to_f(vq[32]);
      float s, m;
      quantise(v0, v1, vp, tab[1], scratch[warp], lane, s, m);
      vsse += s;
      vmx = fmaxf(vmx, m);
      vq[0] = Elem<T>::from_f(v0);
      vq[32] = Elem<T>::from_f(v1);
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
    CC2_CUDA(cudaFuncSetAttribute(kv_quant_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, most));
    CC2_CUDA(cudaFuncSetAttribute(kv_quant_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, most));
    if (dev < 64) attr_done |= 1ull << dev;
  }
  const long long vecs = (long long)rows * heads;
  const int grid = (int)std::min<long long>((vecs + kWarps - 1) / kWarps, 4LL * num_sms());
  const float2* cs = (const float2*)rope_cs;
  if (dtype == CC2_BF16)
    CC2_CUDA(launch_k(kv_quant_kernel<__nv_bfloat16>, grid, kWarps * 32, smem, st, (__nv_bfloat16*)qkv, ld, rows, q_col, k_col,
                                                                   v_col, heads, kp, vp, key != nullptr,
                                                                   value != nullptr, cs, rope_period, stats));
  else if (dtype == CC2_F32)
    CC2_CUDA(launch_k(kv_quant_kernel<float>, grid, kWarps * 32, smem, st, (float*)qkv, ld, rows, q_col, k_col, v_col, heads, kp, vp,
                                                            key != nullptr, value != nullptr, cs, rope_period, stats));
  else
    CC2_REQUIRE(false, "kv_quant: unsupported dtype %d", dtype);
  CC2_CHECK_LAUNCH();
  return CC2_OK;
}

}  // namespace cc2
