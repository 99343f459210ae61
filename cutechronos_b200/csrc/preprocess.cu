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
#include "common.cuh"

namespace cc2 {

namespace {

constexpr int kPreThreads = 256;

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
      mk = m ? m[src] : (isnan(v) ? 0.0f : 1.0f);
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
        float mk = m ? m[src] : (isnan(x[src]) ? 0.0f : 1.0f);
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

template <typename T>
__global__ void output_transform_kernel(const T* __restrict__ preds, int ld, const float* __restrict__ loc,
                                        const float* __restrict__ scale, T* __restrict__ out, int B,
                                        int N, int Q, int ps, int use_arcsinh) {
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
  if (dtype == CC2_BF16) {
    preprocess_kernel<__nv_bfloat16><<<B, kPreThreads, 0, st>>>(
        context, cmask, L, Leff, P, ps, te_scale, use_arcsinh, use_reg ? 1 : 0, N,
        (__nv_bfloat16*)patched, ld, pad_cols, tok, attn, loc, scale);
  } else if (dtype == CC2_F32) {
    preprocess_kernel<float><<<B, kPreThreads, 0, st>>>(context, cmask, L, Leff, P, ps, te_scale,
                                                        use_arcsinh, use_reg ? 1 : 0, N,
                                                        (float*)patched, ld, pad_cols, tok, attn,
                                                        loc, scale);
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
  const int blocks = (int)std::min<size_t>((total + threads - 1) / threads, (size_t)num_sms() * 16);
  if (dtype == CC2_BF16)
    output_transform_kernel<__nv_bfloat16><<<blocks, threads, 0, st>>>(
        (const __nv_bfloat16*)preds, ld, loc, scale, (__nv_bfloat16*)out, B, N, Q, ps, use_arcsinh);
  else if (dtype == CC2_F32)
    output_transform_kernel<float><<<blocks, threads, 0, st>>>((const float*)preds, ld, loc, scale,
                                                                (float*)out, B, N, Q, ps, use_arcsinh);
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
  if (dtype == CC2_BF16)
    rmsnorm_rows_kernel<__nv_bfloat16><<<blocks, threads, 0, st>>>(
        (const __nv_bfloat16*)x, ldx, (const __nv_bfloat16*)w, (__nv_bfloat16*)y, ldy, rows, dim,
        per, stride, offset, eps);
  else if (dtype == CC2_F32)
    rmsnorm_rows_kernel<float><<<blocks, threads, 0, st>>>((const float*)x, ldx, (const float*)w,
                                                            (float*)y, ldy, rows, dim, per, stride,
                                                            offset, eps);
  else
    CC2_REQUIRE(false, "rmsnorm_rows: unsupported dtype %d", dtype);
  CC2_CHECK_LAUNCH();
  return CC2_OK;
}

}  // namespace cc2
