// Memory-bound stages of the forward: fused preprocessing (instance norm +
// arcsinh + patching + time encoding), the output transform (rearrange +
// sinh + unscale) and a strided-row T5 RMSNorm.
//
// Reference semantics:
//   preprocessing     cutechronos/model.py:361-385 (InstanceNorm.forward),
//                     406-414 (Patch), 473-519 (_prepare_patched_context),
//                     521-549 (_prepare_patched_future)
//   output transform  cutechronos/model.py:387-394, 816-829
//   rms norm          cutechronos/modules/_fallbacks.py:14-22
#include <cmath>

#include "common.cuh"

namespace cc2 {

namespace {

constexpr int kPreThreads = 256;

__device__ __forceinline__ uint32_t pack2bf(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// s + e += x with an error-free transformation (Knuth's two-sum), on two
// independent accumulators at once (packed fp32, each lane rounded as a
// scalar instruction would be; t - s is formed as fma(s, -1, t), the same
// single rounding as a subtraction): s + e keeps the exact sum of the values
// added so far, up to the rounding of e itself (below 2^-48 of the sum for
// the <= 32 values a thread adds).
__device__ __forceinline__ void two_sum_acc2(float2& s, float2& e, float2 x) {
  const float2 m1 = make_float2(-1.0f, -1.0f);
  const float2 t = __fadd2_rn(s, x);
  const float2 bp = __ffma2_rn(s, m1, t);
  const float2 err = __fadd2_rn(__ffma2_rn(__ffma2_rn(bp, m1, t), m1, s), __ffma2_rn(bp, m1, x));
  s = t;
  e = __fadd2_rn(e, err);
}

// Two sums in one pass over the block (one pair of barriers); red holds
// 2 * warps doubles.
__device__ __forceinline__ void block_sum2(double& a, double& b, double* red) {
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    b += __shfl_xor_sync(0xffffffffu, b, o);
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = (int)(blockDim.x >> 5);
  __syncthreads();
  if (l == 0) {
    red[w] = a;
    red[nw + w] = b;
  }
  __syncthreads();
  double ta = 0.0, tb = 0.0;
  for (int i = 0; i < nw; ++i) {
    ta += red[i];
    tb += red[nw + i];
  }
  a = ta;
  b = tb;
}

__device__ __forceinline__ double block_sum(double v, double* red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  double t = 0.0;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += red[i];
  return t;
}

// A NaN in a caller's context mask counts as 0 (the reference patches the mask
// and applies nan_to_num).
__device__ __forceinline__ float nan_to_zero(float v) { return isnan(v) ? 0.0f : v; }

// asinh for the vectorised preprocessing, from its definition
// ln(|x| + sqrt(x^2 + 1)) with the hardware log2 and square root: absolute
// error about 2e-7 near 0 and relative error about 1e-7 elsewhere; past 1e18
// the square would overflow and ln(2|x|) = ln2 (log2|x| + 1) is used.
__device__ __forceinline__ float asinh_fast(float x) {
  const float a = fabsf(x);
  const bool large = a > 1e18f;
  float r;
  asm("sqrt.approx.f32 %0, %1;" : "=f"(r) : "f"(fmaf(a, a, 1.0f)));
  float l;
  asm("lg2.approx.f32 %0, %1;" : "=f"(l) : "f"(large ? a : a + r));
  return copysignf((l + (large ? 1.0f : 0.0f)) * 0.6931471805599453f, x);
}

// asinh_fast for two values at once (packed fp32), without the overflow
// branch: the vectorised preprocessing applies it to (x - loc) / scale of a
// series, whose magnitude is at most sqrt(n - 1) <= 91 for n <= 8192 values
// (Samuelson's inequality; a sanitised 0 for missing values), far below the
// 1e18 where x^2 + 1 would overflow.
__device__ __forceinline__ float2 asinh_bounded2(float2 x) {
  const float2 a = make_float2(fabsf(x.x), fabsf(x.y));
  const float2 q = __ffma2_rn(a, a, make_float2(1.0f, 1.0f));
  float2 r, l;
  asm("sqrt.approx.f32 %0, %1;" : "=f"(r.x) : "f"(q.x));
  asm("sqrt.approx.f32 %0, %1;" : "=f"(r.y) : "f"(q.y));
  const float2 u = __fadd2_rn(a, r);
  asm("lg2.approx.f32 %0, %1;" : "=f"(l.x) : "f"(u.x));
  asm("lg2.approx.f32 %0, %1;" : "=f"(l.y) : "f"(u.y));
  l = __fmul2_rn(l, make_float2(0.6931471805599453f, 0.6931471805599453f));
  return make_float2(copysignf(l.x, x.x), copysignf(l.y, x.y));
}

// One CTA per series.  Sums are accumulated in double so that the loc/scale
// statistics are the correctly rounded fp32 values of the NaN-aware mean and
// (population) standard deviation, whatever the series length or offset.
template <typename T>
__global__ void __launch_bounds__(kPreThreads)
preprocess_kernel(const float* __restrict__ ctx, const float* __restrict__ cmask, int L, int Leff,
                  int P, int ps, float te_scale, int use_arcsinh, int use_reg, int N,
                  T* __restrict__ out, int ld, int pad_cols, uint8_t* __restrict__ tok_mask,
                  float* __restrict__ attn_out, float* __restrict__ loc_out,
                  float* __restrict__ scale_out) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ double red[kPreThreads / 32];
  __shared__ float s_loc, s_scale;
  const int b = blockIdx.x;
  const int S = P + use_reg + N;
  const float* x = ctx + (size_t)b * L + (L - Leff);
  const float* m = cmask ? cmask + (size_t)b * L + (L - Leff) : nullptr;

  // pass 1: NaN-aware mean
  double sum = 0.0, cnt = 0.0;
  for (int i = threadIdx.x; i < Leff; i += blockDim.x) {
    float v = x[i];
    if (!isnan(v)) { sum += v; cnt += 1.0; }
  }
  sum = block_sum(sum, red);
  cnt = block_sum(cnt, red);
  const float loc = cnt > 0.0 ? (float)(sum / cnt) : 0.0f;
  // pass 2: NaN-aware population variance around the fp32 loc
  double ss = 0.0;
  for (int i = threadIdx.x; i < Leff; i += blockDim.x) {
    float v = x[i];
    if (!isnan(v)) { float d = v - loc; ss += (double)(d * d); }
  }
  ss = block_sum(ss, red);
  if (threadIdx.x == 0) {
    float sc = cnt > 0.0 ? sqrtf((float)(ss / cnt)) : 1.0f;
    if (sc == 0.0f) sc = 1e-5f;
    s_loc = loc;
    s_scale = sc;
    loc_out[b] = loc;
    scale_out[b] = sc;
  }
  __syncthreads();
  const float lo = s_loc, sc = s_scale;
  const int total = P * ps;
  const int pad = total - Leff;  // left padding (NaN values, mask 0)
  const size_t row0 = (size_t)b * S;

  // pass 3: [time_enc | value | mask] per context position
  for (int j = threadIdx.x; j < total; j += blockDim.x) {
    const int src = j - pad;
    float v = __int_as_float(0x7fc00000);  // NaN
    float mk = 0.0f;
    if (src >= 0) {
      v = x[src];
      mk = m ? nan_to_zero(m[src]) : (isnan(v) ? 0.0f : 1.0f);
      float z = (v - lo) / sc;
      if (use_arcsinh) z = asinhf(z);
      v = z;
    }
    const float mkT = roundT<T>(mk);
    const float val = mkT > 0.0f ? roundT<T>(v) : 0.0f;
    const int p = j / ps, c = j % ps;
    T* r = out + (row0 + p) * ld;
    r[c] = fromf<T>((float)(j - total) / te_scale);
    r[ps + c] = fromf<T>(val);
    r[2 * ps + c] = fromf<T>(mkT);
  }
  // attention mask per patch: sum of the (rounded) patch mask > 0
  for (int p = threadIdx.x; p < P; p += blockDim.x) {
    float acc = 0.0f;
    for (int c = 0; c < ps; ++c) {
      const int src = p * ps + c - pad;
      if (src >= 0) {
        float mk = m ? nan_to_zero(m[src]) : (isnan(x[src]) ? 0.0f : 1.0f);
        acc += roundT<T>(mk);
      }
    }
    const bool on = acc > 0.0f;
    tok_mask[row0 + p] = on ? 1 : 0;
    if (attn_out) attn_out[(size_t)b * P + p] = on ? 1.0f : 0.0f;
  }
  // REG row (zeros) and future rows ([future time enc | 0 | 0])
  const int extra = use_reg + N;
  for (int idx = threadIdx.x; idx < extra * 3 * ps; idx += blockDim.x) {
    const int e = idx / (3 * ps), c = idx % (3 * ps);
    T* r = out + (row0 + P + e) * ld;
    float v = 0.0f;
    const int n = e - use_reg;
    if (n >= 0 && c < ps) v = (float)(n * ps + c) / te_scale;
    r[c] = fromf<T>(v);
  }
  for (int e = threadIdx.x; e < extra; e += blockDim.x) tok_mask[row0 + P + e] = 1;
  // zero the padding columns [3*ps, pad_cols) of every token row
  const int pc = pad_cols - 3 * ps;
  if (pc > 0) {
    for (int idx = threadIdx.x; idx < S * pc; idx += blockDim.x) {
      const int rr = idx / pc, c = idx % pc;
      out[(row0 + rr) * ld + 3 * ps + c] = fromf<T>(0.0f);
    }
  }
}

// Vectorised preprocessing: one CTA per series, each thread owns chunks of 8
// consecutive patch positions (CH per thread, kept in registers across the
// three passes), 16-byte loads when the series is 16-byte aligned, and the
// [time_enc | value | mask] chunks written as 16-byte (bf16) / 32-byte (fp32)
// stores.  Same arithmetic as preprocess_kernel.
// Vectorised preprocessing: one CTA per series of up to 4 x 8 x kPreThreads
// positions.  Each thread holds CH chunks of 8 consecutive positions in
// registers across the mean, variance and patching passes; 16-byte loads and
// stores.  (A warp per series, with up to 64 positions per lane, ran slower:
// fewer series fit on an SM and each warp's chain of work grew.)
template <typename T, int CH, int NTH>
__global__ void __launch_bounds__(NTH, NTH == 128 ? 8 : (CH == 1 ? 5 : 1))
preprocess_vec_kernel(const float* __restrict__ ctx, const float* __restrict__ cmask, int B, int L, int Leff, int P,
                      int ps, float te_scale, float te_inv, int use_arcsinh, int use_reg, int N,
                      T* __restrict__ out, int ld, int pad_cols, uint8_t* __restrict__ tok_mask,
                      float* __restrict__ attn_out, float* __restrict__ loc_out, float* __restrict__ scale_out,
                      int vec_loads) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ double red[2 * (NTH / 32)];
  const int b = (int)blockIdx.x;
  const int tid = (int)threadIdx.x;
  const int G = (int)blockDim.x;
  const int S = P + use_reg + N;
  const float* x = ctx + (size_t)b * L + (L - Leff);
  const float* m = cmask ? cmask + (size_t)b * L + (L - Leff) : nullptr;
  const int total = P * ps, pad = total - Leff;
  float v[CH][8];
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int j0 = 8 * (tid + c * G);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[c][i] = __int_as_float(0x7fc00000);
    if (j0 < total) {
      const int s0 = j0 - pad;
      if (vec_loads && s0 >= 0) {
        const float4 a = *reinterpret_cast<const float4*>(x + s0);
        const float4 e = *reinterpret_cast<const float4*>(x + s0 + 4);
        v[c][0] = a.x; v[c][1] = a.y; v[c][2] = a.z; v[c][3] = a.w;
        v[c][4] = e.x; v[c][5] = e.y; v[c][6] = e.z; v[c][7] = e.w;
      } else if (vec_loads && s0 + 4 >= 0 && s0 < 0) {  // pad is a multiple of 4: upper half present
        const float4 e = *reinterpret_cast<const float4*>(x + s0 + 4);
        v[c][4] = e.x; v[c][5] = e.y; v[c][6] = e.z; v[c][7] = e.w;
      } else if (!vec_loads) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (s0 + i >= 0) v[c][i] = x[s0 + i];
      }
    }
  }
  // per-thread sums as an unevaluated fp32 pair (error-free additions): the
  // same exact partial sums as accumulating in double, without a conversion
  // to double per value; the block then reduces them in double
  // (one pair per chunk: independent dependency chains)
  // (two chains per chunk, even and odd positions, as the lanes of packed
  // fp32 instructions)
  float2 s_hi[CH], s_lo[CH];
  int n_ok = 0;
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    s_hi[c] = s_lo[c] = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
      const bool ok0 = !isnan(v[c][i]), ok1 = !isnan(v[c][i + 1]);
      n_ok += (ok0 ? 1 : 0) + (ok1 ? 1 : 0);
      two_sum_acc2(s_hi[c], s_lo[c], make_float2(ok0 ? v[c][i] : 0.0f, ok1 ? v[c][i + 1] : 0.0f));
    }
  }
  double sum = 0.0, cnt = (double)n_ok;
#pragma unroll
  for (int c = 0; c < CH; ++c)
    sum += ((double)s_hi[c].x + (double)s_lo[c].x) + ((double)s_hi[c].y + (double)s_lo[c].y);
  block_sum2(sum, cnt, red);
  const float lo = cnt > 0.0 ? (float)(sum / cnt) : 0.0f;
  // squared deviations: non-negative terms, so the sum needs no
  // compensation: two plain fp32 sums (fused multiply-adds) of 4 terms per
  // chunk (at most 4 roundings each, 2.4e-7 relative, about 1e-7 on the
  // scale), then double across chunks and threads
  float2 q[CH];
  const float2 nlo = make_float2(-lo, -lo);
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    q[c] = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
      float2 d = __fadd2_rn(make_float2(v[c][i], v[c][i + 1]), nlo);
      d.x = isnan(d.x) ? 0.0f : d.x;
      d.y = isnan(d.y) ? 0.0f : d.y;
      q[c] = __ffma2_rn(d, d, q[c]);
    }
  }
  double ssp = 0.0;
#pragma unroll
  for (int c = 0; c < CH; ++c) ssp += (double)q[c].x + (double)q[c].y;
  double ss = block_sum(ssp, red);
  // the scale is computed once (thread 0) and shared
  __shared__ float sc_sh;
  if (tid == 0) {
    float sc0 = cnt > 0.0 ? sqrtf((float)(ss / cnt)) : 1.0f;
    if (sc0 == 0.0f) sc0 = 1e-5f;
    sc_sh = sc0;
    loc_out[b] = lo;
    scale_out[b] = sc0;
  }
  __syncthreads();
  const float sc = sc_sh;
  // (x - loc) / scale as a product with the reciprocal: within 1.5 ulp of the
  // quotient, one division per series instead of one per value
  const float rsc = 1.0f / sc;
  const size_t row0 = (size_t)b * S;
  const int cpp = ps / 8;  // chunks per patch: 1, 2 or 4 adjacent lanes
  const int ps_log = __ffs(ps) - 1;  // the patch width is 8, 16 or 32 here: shifts, not divisions
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int k = tid + c * G;
    const int j0 = 8 * k;
    float acc = 0.0f;
    if (j0 < total) {
      float te[8], val[8], mt[8];
      // time encoding (position - total) / te_scale; for a power-of-two scale the
      // product with its exact reciprocal is the same number (positions are
      // integers of magnitude < 2^24, so base + i is exact)
      const float tbase = (float)(j0 - total);
      // uniform conditions are tested once per chunk, outside the per-value
      // loops, so no value pays for the path it does not take
      if (te_inv != 0.0f) {
        // te_inv is a power of two here, so tbase * te_inv and i * te_inv are
        // exact and so is their sum (the value (tbase + i) * te_inv): one FMA
        const float2 tb = make_float2(tbase * te_inv, tbase * te_inv), ti = make_float2(te_inv, te_inv);
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          const float2 t2 = __ffma2_rn(make_float2((float)i, (float)(i + 1)), ti, tb);
          te[i] = t2.x; te[i + 1] = t2.y;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) te[i] = (float)(j0 + i - total) / te_scale;
      }
      if (sizeof(T) == 2 && m == nullptr && j0 - pad >= 0) {  // bf16, NaN mask, all 8 positions in the series
        if (use_arcsinh) {
          // branch-free, two positions per packed instruction: asinh of a
          // sanitised argument (0 for a NaN value, asinh(0) = 0), then times
          // the 0/1 mask
#pragma unroll
          for (int i = 0; i < 8; i += 2) {
            const bool ok0 = !isnan(v[c][i]), ok1 = !isnan(v[c][i + 1]);
            const float2 mk = make_float2(ok0 ? 1.0f : 0.0f, ok1 ? 1.0f : 0.0f);
            float2 z = __fmul2_rn(__fadd2_rn(make_float2(v[c][i], v[c][i + 1]), nlo), make_float2(rsc, rsc));
            z.x = ok0 ? z.x : 0.0f;
            z.y = ok1 ? z.y : 0.0f;
            z = __fmul2_rn(asinh_bounded2(z), mk);
            mt[i] = mk.x; mt[i + 1] = mk.y;
            val[i] = z.x; val[i + 1] = z.y;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const bool ok = !isnan(v[c][i]);
            mt[i] = ok ? 1.0f : 0.0f;
            val[i] = ok ? (v[c][i] - lo) * rsc : 0.0f;
          }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) acc += mt[i];
      } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int src = j0 + i - pad;
        float z = __int_as_float(0x7fc00000);
        float mk = 0.0f;
        if (src >= 0) {
          if constexpr (sizeof(T) == 4) {  // fp32 model: the reference's division and accurate asinh
            z = __fdiv_rn(v[c][i] - lo, sc);
            if (use_arcsinh) z = asinhf(z);
          } else {
            z = (v[c][i] - lo) * rsc;
            if (use_arcsinh) z = asinh_fast(z);
          }
          mk = m ? nan_to_zero(m[src]) : (isnan(v[c][i]) ? 0.0f : 1.0f);
        }
        mt[i] = roundT<T>(mk);  // the mask in the model dtype (fractional masks pass through)
        // bf16: rounded once when packed below
        val[i] = mt[i] > 0.0f ? (sizeof(T) == 2 ? z : roundT<T>(z)) : 0.0f;
        acc += mt[i];
      }
      }
      const int p = j0 >> ps_log, c0 = j0 & (ps - 1);
      T* r = out + (row0 + p) * ld + c0;
      if constexpr (sizeof(T) == 2) {
        uint4 w;
        w.x = pack2bf(te[0], te[1]); w.y = pack2bf(te[2], te[3]); w.z = pack2bf(te[4], te[5]); w.w = pack2bf(te[6], te[7]);
        *reinterpret_cast<uint4*>(r) = w;
        w.x = pack2bf(val[0], val[1]); w.y = pack2bf(val[2], val[3]); w.z = pack2bf(val[4], val[5]);
        w.w = pack2bf(val[6], val[7]);
        *reinterpret_cast<uint4*>(r + ps) = w;
        w.x = pack2bf(mt[0], mt[1]); w.y = pack2bf(mt[2], mt[3]); w.z = pack2bf(mt[4], mt[5]); w.w = pack2bf(mt[6], mt[7]);
        *reinterpret_cast<uint4*>(r + 2 * ps) = w;
      } else {
        float4* q4 = reinterpret_cast<float4*>(r);
        q4[0] = make_float4(te[0], te[1], te[2], te[3]);
        q4[1] = make_float4(te[4], te[5], te[6], te[7]);
        q4 = reinterpret_cast<float4*>(r + ps);
        q4[0] = make_float4(val[0], val[1], val[2], val[3]);
        q4[1] = make_float4(val[4], val[5], val[6], val[7]);
        q4 = reinterpret_cast<float4*>(r + 2 * ps);
        q4[0] = make_float4(mt[0], mt[1], mt[2], mt[3]);
        q4[1] = make_float4(mt[4], mt[5], mt[6], mt[7]);
      }
    }
    // attention mask per patch: sum of the (rounded) patch mask > 0, over the
    // patch's cpp adjacent lanes
    for (int o = 1; o < cpp; o <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (j0 < total && (k & (cpp - 1)) == 0) {
      const int p = j0 >> ps_log;
      const bool on = acc > 0.0f;
      tok_mask[row0 + p] = on ? 1 : 0;
      if (attn_out) attn_out[(size_t)b * P + p] = on ? 1.0f : 0.0f;
    }
  }
  // REG row (zeros) and future rows ([future time enc | 0 | 0]); no integer
  // division per element
  const int extra = use_reg + N;
  for (int c = tid; c < 3 * ps; c += G)
    for (int e = 0; e < extra; ++e) {
      const int n = e - use_reg;
      const float pos = (float)(n * ps + c);  // an integer below 2^24: exact
      const float fv = n >= 0 && c < ps ? (te_inv != 0.0f ? pos * te_inv : pos / te_scale) : 0.0f;
      out[(row0 + P + e) * ld + c] = fromf<T>(fv);
    }
  for (int e = tid; e < extra; e += G) tok_mask[row0 + P + e] = 1;
  // zero the padding columns [3*ps, pad_cols) of every token row: one row per thread
  const int pc = pad_cols - 3 * ps;
  if (pc > 0) {
    const bool vec16 = (pc * (int)sizeof(T)) % 16 == 0;  // 3*ps*sizeof(T) is a multiple of 16 here
    for (int rr = tid; rr < S; rr += G) {
      T* r = out + (row0 + rr) * ld + 3 * ps;
      if (vec16) {
        for (int q = 0; q < pc * (int)sizeof(T) / 16; ++q) reinterpret_cast<uint4*>(r)[q] = make_uint4(0u, 0u, 0u, 0u);
      } else {
        for (int c = 0; c < pc; ++c) r[c] = fromf<T>(0.0f);
      }
    }
  }
}

// sinh for the bf16 output transform, from its definition, for a pair of
// values with the Blackwell packed-fp32 instructions (one issue slot for both
// lanes, each lane rounded as a scalar instruction would be): |x| < 1/2 by
// the odd Taylor polynomial x + x^3/3! + x^5/5! (truncation below 1.6e-6
// relative, three orders below the final bf16 rounding's 2^-9), otherwise
// (e - 1/e) / 2 with e = 2^(|x| log2 e) from the hardware exp2 and
// reciprocal (relative error about 6e-8 |x|, below 1e-6 for the |x| <= 15 a
// forecast in arcsinh space reaches), sign restored.  Overflow gives inf,
// NaN stays NaN.  The kernel is bound by instruction issue (an FMA-only
// version, Cody-Waite reduction and a shared even/odd polynomial with no MUFU
// op, needed ~30 instructions per output and was slower).
__device__ __forceinline__ float2 f2(float v) { return make_float2(v, v); }
__device__ __forceinline__ float2 sinh_fast2(float2 x) {
  const float2 a = make_float2(fabsf(x.x), fabsf(x.y));
  const float2 a2 = __fmul2_rn(a, a);
  const float2 u = __fmul2_rn(__ffma2_rn(a2, f2(1.0f / 120.0f), f2(1.0f / 6.0f)), a2);
  const float2 poly = __ffma2_rn(u, a, a);
  float2 e, inv;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e.x) : "f"(fabsf(x.x) * 1.4426950408889634f));
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e.y) : "f"(fabsf(x.y) * 1.4426950408889634f));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(inv.x) : "f"(e.x));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(inv.y) : "f"(e.y));
  const float2 big = __fmul2_rn(__ffma2_rn(inv, f2(-1.0f), e), f2(0.5f));
  return make_float2(copysignf(fabsf(x.x) < 0.5f ? poly.x : big.x, x.x),
                     copysignf(fabsf(x.y) < 0.5f ? poly.y : big.y, x.y));
}

// Output transform: (B, N, ld) forecasts in the model's row layout ->
// (B, Q, N * ps) rows, sinh and unscale.  A thread owns one 8-output segment
// of the per-series layout (its source and destination offsets computed once)
// and walks the series of its block, UNR of them per step so that UNR
// 16-byte loads are in flight per thread.
template <typename T, int UNR>
__global__ void __launch_bounds__(256)
output_transform_seg_kernel(const T* __restrict__ preds, int ld, const float* __restrict__ loc,
                            const float* __restrict__ scale, T* __restrict__ out, int B, int N, int Q, int ps,
                            int use_arcsinh) {
  pdl_launch_dependents();
  pdl_wait();
  const int spp = ps / 8;  // segments per patch row
  const int per_series = Q * N * spp;
  constexpr int V = 8 * (int)sizeof(T) / 16;  // 16-byte vectors per segment
  using Vec = uint4;
  for (int seg = (int)threadIdx.x; seg < per_series; seg += (int)blockDim.x) {
    // output order: seg = (q * N + n) * spp + s8
    const int t = seg / spp, s8 = seg - t * spp;
    const int q = t / N, n = t - q * N;
    const size_t src0 = (size_t)n * ld + (size_t)q * ps + 8 * s8;
    const size_t dst0 = (size_t)seg * 8;
    const size_t src_step = (size_t)N * ld, dst_step = (size_t)per_series * 8;
    for (int b0 = (int)blockIdx.x * UNR; b0 < B; b0 += (int)gridDim.x * UNR) {
      Vec w[UNR][V];
      float sc[UNR], lo[UNR];
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        const int b = b0 + u;
        if (b < B) {
          const Vec* src = reinterpret_cast<const Vec*>(preds + (size_t)b * src_step + src0);
#pragma unroll
          for (int v = 0; v < V; ++v) w[u][v] = __ldcs(src + v);
          sc[u] = __ldg(scale + b);
          lo[u] = __ldg(loc + b);
        }
      }
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        const int b = b0 + u;
        if (b >= B) break;
        float f[8];
        if constexpr (sizeof(T) == 2) {
          const uint32_t uu[4] = {w[u][0].x, w[u][0].y, w[u][0].z, w[u][0].w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            f[2 * i] = __uint_as_float(uu[i] << 16);
            f[2 * i + 1] = __uint_as_float(uu[i] & 0xffff0000u);
          }
        } else {
#pragma unroll
          for (int v = 0; v < V; ++v) {
            f[4 * v] = __uint_as_float(w[u][v].x); f[4 * v + 1] = __uint_as_float(w[u][v].y);
            f[4 * v + 2] = __uint_as_float(w[u][v].z); f[4 * v + 3] = __uint_as_float(w[u][v].w);
          }
        }
        if constexpr (sizeof(T) == 2) {
          // bf16 model: pairs of outputs on the packed-fp32 path
#pragma unroll
          for (int i = 0; i < 8; i += 2) {
            float2 vv = make_float2(f[i], f[i + 1]);
            if (use_arcsinh) vv = sinh_fast2(vv);
            vv = __fadd2_rn(__fmul2_rn(vv, f2(sc[u])), f2(lo[u]));
            f[i] = vv.x;
            f[i + 1] = vv.y;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            float vv = f[i];
            if (use_arcsinh) vv = sinhf(vv);  // fp32 model: the error is not hidden by a bf16 rounding
            f[i] = __fadd_rn(__fmul_rn(vv, sc[u]), lo[u]);
          }
        }
        Vec* dst = reinterpret_cast<Vec*>(out + (size_t)b * dst_step + dst0);
        if constexpr (sizeof(T) == 2) {
          Vec o;
          o.x = pack2bf(f[0], f[1]); o.y = pack2bf(f[2], f[3]); o.z = pack2bf(f[4], f[5]); o.w = pack2bf(f[6], f[7]);
          __stcs(dst, o);
        } else {
          __stcs(dst, make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                                 __float_as_uint(f[3])));
          __stcs(dst + 1, make_uint4(__float_as_uint(f[4]), __float_as_uint(f[5]), __float_as_uint(f[6]),
                                     __float_as_uint(f[7])));
        }
      }
    }
  }
}

// Vectorised RMSNorm rows: one warp per row, each lane holds VPL = dim / 32
// values loaded 16 bytes at a time.
template <typename T, int VPL>
__global__ void __launch_bounds__(256)
rmsnorm_rows_vec_kernel(const T* __restrict__ x, int ldx, const T* __restrict__ w, T* __restrict__ y, int ldy,
                        int rows, int dim, int per, int stride, int offset, float eps) {
  pdl_launch_dependents();
  pdl_wait();
  constexpr int V = 16 / sizeof(T);  // elements per 16-byte access
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const size_t src = (size_t)(warp / per) * stride + offset + warp % per;
  const T* xr = x + src * ldx;
  float xv[VPL];
  float ss = 0.0f;
#pragma unroll
  for (int g = 0; g < VPL / V; ++g) {
    const int c = (g * 32 + lane) * V;
    const uint4 u = *reinterpret_cast<const uint4*>(xr + c);
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < V; ++i) {
      xv[g * V + i] = tof<T>(e[i]);
      ss += xv[g * V + i] * xv[g * V + i];
    }
  }
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float r = rsqrtf(ss / (float)dim + eps);
  T* yr = y + (size_t)warp * ldy;
#pragma unroll
  for (int g = 0; g < VPL / V; ++g) {
    const int c = (g * 32 + lane) * V;
    const uint4 wu = *reinterpret_cast<const uint4*>(w + c);
    const T* we = reinterpret_cast<const T*>(&wu);
    uint4 o;
    T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
    for (int i = 0; i < V; ++i) oe[i] = fromf<T>(tof<T>(we[i]) * roundT<T>(xv[g * V + i] * r));
    *reinterpret_cast<uint4*>(yr + c) = o;
  }
}

template <typename T>
__global__ void output_transform_kernel(const T* __restrict__ preds, int ld, const float* __restrict__ loc,
                                        const float* __restrict__ scale, T* __restrict__ out, int B,
                                        int N, int Q, int ps, int use_arcsinh) {
  pdl_launch_dependents();
  pdl_wait();
  const size_t H = (size_t)N * ps;
  const size_t total = (size_t)B * Q * H;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const int h = (int)(i % H);
    const int q = (int)((i / H) % Q);
    const int b = (int)(i / (H * Q));
    const int n = h / ps, j = h % ps;
    float v = tof<T>(preds[((size_t)b * N + n) * ld + q * ps + j]);
    if (use_arcsinh) v = sinhf(v);
    out[i] = fromf<T>(__fadd_rn(__fmul_rn(v, scale[b]), loc[b]));
  }
}

// One warp per output row.
template <typename T>
__global__ void rmsnorm_rows_kernel(const T* __restrict__ x, int ldx, const T* __restrict__ w,
                                    T* __restrict__ y, int ldy, int rows, int dim, int per,
                                    int stride, int offset, float eps) {
  pdl_launch_dependents();
  pdl_wait();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const size_t src = (size_t)(warp / per) * stride + offset + warp % per;
  const T* xr = x + src * ldx;
  float ss = 0.0f;
  for (int c = lane; c < dim; c += 32) {
    float v = tof<T>(xr[c]);
    ss += v * v;
  }
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float r = rsqrtf(ss / (float)dim + eps);
  T* yr = y + (size_t)warp * ldy;
  for (int c = lane; c < dim; c += 32) {
    float v = roundT<T>(tof<T>(xr[c]) * r);
    yr[c] = fromf<T>(tof<T>(w[c]) * v);
  }
}

}  // namespace

int launch_preprocess(const float* context, const float* cmask, int B, int L, int ps, int ctx_len,
                      float te_scale, int use_arcsinh, int use_reg, int N, int dtype, void* patched,
                      int ld, int pad_cols, uint8_t* tok, float* attn, float* loc, float* scale,
                      cudaStream_t st) {
  CC2_REQUIRE(B > 0 && L > 0 && ps > 0 && ctx_len > 0 && N >= 0, "preprocess: bad sizes");
  CC2_REQUIRE(context && patched && tok && loc && scale, "preprocess: null pointer");
  CC2_REQUIRE(pad_cols >= 3 * ps && ld >= pad_cols, "preprocess: ld/pad_cols too small");
  const int Leff = L < ctx_len ? L : ctx_len;
  const int P = (Leff + ps - 1) / ps;
  const int total = P * ps;
  const size_t esz = dtype == CC2_BF16 ? 2 : 4;
  // vectorised kernel: patch width 8/16/32, 16-byte aligned rows, <= 8192 positions
  const bool vec = (ps == 8 || ps == 16 || ps == 32) && ((uintptr_t)patched & 15u) == 0 && (ld * esz) % 16 == 0 &&
                   total <= 4 * 8 * kPreThreads;
  const int vec_loads = ((uintptr_t)context & 15u) == 0 && L % 4 == 0 && (L - Leff) % 4 == 0 && (total - Leff) % 4 == 0;
  // 128 threads per series up to 2048 positions (two chunks of 8 per thread:
  // the per-thread reductions and statistics are shared by 16 values), 256 above
  const int NTH = total <= 16 * 128 ? 128 : kPreThreads;
  const int CH = total <= 8 * NTH ? 1 : total <= 16 * NTH ? 2 : 4;
  // exact reciprocal of a power-of-two time-encoding scale (0: divide instead)
  int te_exp = 0;
  const float te_frac = std::frexp(te_scale, &te_exp);
  const float te_inv = te_frac == 0.5f && te_exp > -120 && te_exp < 120 ? std::ldexp(1.0f, 1 - te_exp) : 0.0f;
#define CC2_PRE_VEC(TT, C_)                                                                                       \
  CC2_CUDA(launch_k(NTH == 128 ? preprocess_vec_kernel<TT, C_, 128> : preprocess_vec_kernel<TT, C_, kPreThreads>, \
                    B, NTH, 0, st, context, cmask, B, L, Leff, P, ps,                                           \
                    te_scale, te_inv, use_arcsinh, use_reg ? 1 : 0, N, (TT*)patched, ld, pad_cols, tok, attn, loc, \
                    scale, vec_loads))
#define CC2_PRE_VEC_ALL(TT)       \
  if (CH == 1)                    \
    CC2_PRE_VEC(TT, 1);           \
  else if (CH == 2)               \
    CC2_PRE_VEC(TT, 2);           \
  else                            \
    CC2_PRE_VEC(TT, 4);
  if (vec && dtype == CC2_BF16) {
    CC2_PRE_VEC_ALL(__nv_bfloat16)
  } else if (vec && dtype == CC2_F32) {
    CC2_PRE_VEC_ALL(float)
  } else if (dtype == CC2_BF16) {
    CC2_CUDA(launch_k(preprocess_kernel<__nv_bfloat16>, B, kPreThreads, 0, st, 
        context, cmask, L, Leff, P, ps, te_scale, use_arcsinh, use_reg ? 1 : 0, N,
        (__nv_bfloat16*)patched, ld, pad_cols, tok, attn, loc, scale));
  } else if (dtype == CC2_F32) {
    CC2_CUDA(launch_k(preprocess_kernel<float>, B, kPreThreads, 0, st, context, cmask, L, Leff, P, ps, te_scale,
                                                        use_arcsinh, use_reg ? 1 : 0, N,
                                                        (float*)patched, ld, pad_cols, tok, attn,
                                                        loc, scale));
  } else {
    CC2_REQUIRE(false, "preprocess: unsupported dtype %d", dtype);
  }
  CC2_CHECK_LAUNCH();
  return CC2_OK;
}

int launch_output_transform(int dtype, const void* preds, int ld, const float* loc,
                            const float* scale, void* out, int B, int N, int Q, int ps,
                            int use_arcsinh, cudaStream_t st) {
  CC2_REQUIRE(B > 0 && N > 0 && Q > 0 && ps > 0 && ld >= Q * ps, "output_transform: bad sizes");
  CC2_REQUIRE(preds && loc && scale && out, "output_transform: null pointer");
  const size_t total = (size_t)B * Q * N * ps;
  const int threads = 256;
  const size_t esz = dtype == CC2_BF16 ? 2 : 4;
  if (ps % 8 == 0 && ((uintptr_t)preds & 15u) == 0 && ((uintptr_t)out & 15u) == 0 && (ld * esz) % 16 == 0 &&
      (ps * esz) % 16 == 0 && total / 8 < ((size_t)1 << 31)) {
    // one 8-output segment per thread of the per-series layout, whole series per block step
    const int per_series = Q * N * (ps / 8);
    const int vt = per_series >= 256 ? 256 : (per_series + 31) / 32 * 32;
    // a small batch (the forward's) takes one series per block and step, so
    // that every series has its own block; a streaming batch eight, so that
    // eight loads per thread are in flight
    int per_sm = 0;  // resident blocks per SM of the streaming kernel (registers bound it)
    if (dtype == CC2_BF16)
      CC2_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, output_transform_seg_kernel<__nv_bfloat16, 8>,
                                                             vt, 0));
    else
      CC2_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, output_transform_seg_kernel<float, 8>, vt, 0));
    const long resident = (long)num_sms() * std::max(per_sm, 1);
    const bool stream = B > resident;
    const int vb = (int)std::min<long>(stream ? (B + 7) / 8 : B, resident);
#define CC2_OT_SEG(TT, U)                                                                                    \
  CC2_CUDA(launch_k(output_transform_seg_kernel<TT, U>, vb, vt, 0, st, (const TT*)preds, ld, loc, scale, (TT*)out, \
                    B, N, Q, ps, use_arcsinh))
    if (dtype == CC2_BF16) {
      if (stream) CC2_OT_SEG(__nv_bfloat16, 8); else CC2_OT_SEG(__nv_bfloat16, 1);
    } else if (dtype == CC2_F32) {
      if (stream) CC2_OT_SEG(float, 8); else CC2_OT_SEG(float, 1);
    } else
#undef CC2_OT_SEG
      CC2_REQUIRE(false, "output_transform: unsupported dtype %d", dtype);
    CC2_CHECK_LAUNCH();
    return CC2_OK;
  }
  const int blocks = (int)std::min<size_t>((total + threads - 1) / threads, (size_t)num_sms() * 16);
  if (dtype == CC2_BF16)
    CC2_CUDA(launch_k(output_transform_kernel<__nv_bfloat16>, blocks, threads, 0, st, 
        (const __nv_bfloat16*)preds, ld, loc, scale, (__nv_bfloat16*)out, B, N, Q, ps, use_arcsinh));
  else if (dtype == CC2_F32)
    CC2_CUDA(launch_k(output_transform_kernel<float>, blocks, threads, 0, st, (const float*)preds, ld, loc, scale,
                                                                (float*)out, B, N, Q, ps, use_arcsinh));
  else
    CC2_REQUIRE(false, "output_transform: unsupported dtype %d", dtype);
  CC2_CHECK_LAUNCH();
  return CC2_OK;
}

int launch_rmsnorm_rows(int dtype, const void* x, int ldx, const void* w, void* y, int ldy, int rows,
                        int dim, int per, int stride, int offset, float eps, cudaStream_t st) {
  CC2_REQUIRE(rows > 0 && dim > 0 && per > 0, "rmsnorm_rows: bad sizes");
  CC2_REQUIRE(x && w && y, "rmsnorm_rows: null pointer");
  const int threads = 256;
  const int blocks = (rows * 32 + threads - 1) / threads;
  const int V = dtype == CC2_BF16 ? 8 : 4;
  const int vpl = dim / 32;
  const bool vec = dim % (32 * V) == 0 && (vpl == 8 || vpl == 16 || vpl == 24 || vpl == 32) && ldx % V == 0 &&
                   ldy % V == 0 && ((uintptr_t)x & 15u) == 0 && ((uintptr_t)w & 15u) == 0 && ((uintptr_t)y & 15u) == 0;
  if (vec) {
#define CC2_RMS_VEC(TT, VP)                                                                                     \
  CC2_CUDA(launch_k(rmsnorm_rows_vec_kernel<TT, VP>, blocks, threads, 0, st, (const TT*)x, ldx, (const TT*)w, (TT*)y, ldy, rows, dim, \
                                                              per, stride, offset, eps))
    if (dtype == CC2_BF16) {
      if (vpl == 8) CC2_RMS_VEC(__nv_bfloat16, 8); else if (vpl == 16) CC2_RMS_VEC(__nv_bfloat16, 16);
      else if (vpl == 24) CC2_RMS_VEC(__nv_bfloat16, 24); else CC2_RMS_VEC(__nv_bfloat16, 32);
    } else if (dtype == CC2_F32) {
      if (vpl == 8) CC2_RMS_VEC(float, 8); else if (vpl == 16) CC2_RMS_VEC(float, 16);
      else if (vpl == 24) CC2_RMS_VEC(float, 24); else CC2_RMS_VEC(float, 32);
    } else {
      CC2_REQUIRE(false, "rmsnorm_rows: unsupported dtype %d", dtype);
    }
    CC2_CHECK_LAUNCH();
    return CC2_OK;
  }
  if (dtype == CC2_BF16)
    CC2_CUDA(launch_k(rmsnorm_rows_kernel<__nv_bfloat16>, blocks, threads, 0, st, 
        (const __nv_bfloat16*)x, ldx, (const __nv_bfloat16*)w, (__nv_bfloat16*)y, ldy, rows, dim,
        per, stride, offset, eps));
  else if (dtype == CC2_F32)
    CC2_CUDA(launch_k(rmsnorm_rows_kernel<float>, blocks, threads, 0, st, (const float*)x, ldx, (const float*)w,
                                                            (float*)y, ldy, rows, dim, per, stride,
                                                            offset, eps));
  else
    CC2_REQUIRE(false, "rmsnorm_rows: unsupported dtype %d", dtype);
  CC2_CHECK_LAUNCH();
  return CC2_OK;
}

}  // namespace cc2
