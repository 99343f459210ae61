// fp32 GEMM on CUDA cores for the fp32 model mode:
//   out[M,N] = epilogue(A[M,K] @ W[N,K]^T)
// tcgen05 has no full-precision fp32 kind (kind::tf32 rounds inputs to 10
// mantissa bits), so the fp32 mode, whose parity bar is max-abs 1e-4 against
// the reference's fp32 CPU path, runs this FFMA kernel.  It applies the same
// fused epilogue as the tensor-core kernel (row scale, bias, ReLU, residual,
// sum of squares, special rows).
#include "common.cuh"

namespace cc2 {
namespace {

constexpr int TM = 64, TN = 64, TK = 16, kThreads = 256;

__global__ void __launch_bounds__(kThreads)
gemm_f32_kernel(const float* __restrict__ A, int lda, const float* __restrict__ W, int ldw,
                float* out, int ldo, int M, int N, int K, cc2_epilogue ep) {
  __shared__ float As[TK][TM + 4];
  __shared__ float Ws[TK][TN + 4];
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += TK) {
    // each thread loads 4 elements of A and 4 of W (row = tid/4, k = (tid%4)*4 + i)
    const int lr = tid >> 2, lk = (tid & 3) * 4;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int k = k0 + lk + i;
      const int am = m0 + lr, wn = n0 + lr;
      As[lk + i][lr] = (am < M && k < K) ? A[(size_t)am * lda + k] : 0.0f;
      Ws[lk + i][lr] = (wn < N && k < K) ? W[(size_t)wn * ldw + k] : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < TK; ++k) {
      float a[4], w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[k][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) w[j] = Ws[k][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], w[j], acc[i][j]);
    }
    __syncthreads();
  }
  const float inv_dim = ep.norm_dim > 0 ? 1.0f / (float)ep.norm_dim : 0.0f;
  const float* resid = (const float*)ep.resid;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int row = m0 + ty + 16 * i;
    const bool row_ok = row < M;
    float rs = 1.0f;
    if ((ep.flags & CC2_EPI_ROWSCALE) && row_ok) {
      float t = 0.0f;
      const int parts = (ep.norm_dim + 63) / 64;
      for (int g = 0; g < parts; ++g) t += ep.ssq_in[(size_t)g * ep.ssq_ld + row];
      rs = rsqrtf(t * inv_dim + ep.eps);
    }
    const bool special = (ep.flags & CC2_EPI_SPECIAL) && row_ok && (row % ep.special_period) == ep.special_offset;
    float ssq = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int col = n0 + tx + 16 * j;
      if (!row_ok || col >= N) continue;
      float v = acc[i][j] * rs;
      if (ep.flags & CC2_EPI_BIAS) v += ep.bias[col];
      if (ep.flags & CC2_EPI_RELU) v = fmaxf(v, 0.0f);
      if (ep.flags & CC2_EPI_RESID) v += resid[(size_t)row * ep.ld_resid + col];
      if (special) v = ep.special[col];
      ssq = fmaf(v, v, ssq);
      out[(size_t)row * ldo + col] = v;
    }
    if (ep.flags & CC2_EPI_SSQ) {
      // the 16 threads sharing ty hold this CTA's 64 columns of the row (lanes tx 0..15)
      for (int o = 8; o > 0; o >>= 1) ssq += __shfl_xor_sync(0xffffffffu, ssq, o);
      if (tx == 0 && row_ok) ep.ssq_out[(size_t)blockIdx.x * ep.ssq_ld + row] = ssq;
    }
  }
}

}  // namespace

int launch_gemm_f32(const void* A, int lda, const void* W, int ldw, void* out, int ldo, int M, int N,
                    int K, const cc2_epilogue* e, cudaStream_t st) {
  CC2_REQUIRE(M > 0 && N > 0 && K > 0, "gemm: bad sizes M=%d N=%d K=%d", M, N, K);
  CC2_REQUIRE(A && W && out, "gemm: null pointer");
  cc2_epilogue ep{};
  if (e) ep = *e;
  CC2_REQUIRE(!(ep.flags & CC2_EPI_ROWSCALE) || (ep.ssq_in && ep.norm_dim > 0), "gemm: rowscale args");
  CC2_REQUIRE(!(ep.flags & CC2_EPI_BIAS) || ep.bias, "gemm: bias null");
  CC2_REQUIRE(!(ep.flags & CC2_EPI_RESID) || ep.resid, "gemm: resid null");
  CC2_REQUIRE(!(ep.flags & CC2_EPI_SSQ) || ep.ssq_out, "gemm: ssq_out null");
  CC2_REQUIRE(!(ep.flags & (CC2_EPI_SSQ | CC2_EPI_ROWSCALE)) || ep.ssq_ld >= M, "gemm: ssq_ld must be >= M");
  CC2_REQUIRE(!(ep.flags & CC2_EPI_SPECIAL) || (ep.special && ep.special_period > 0), "gemm: special args");
  dim3 grid((N + TN - 1) / TN, (M + TM - 1) / TM);
  gemm_f32_kernel<<<grid, kThreads, 0, st>>>((const float*)A, lda, (const float*)W, ldw, (float*)out,
                                             ldo, M, N, K, ep);
  CC2_CHECK_LAUNCH();
  return CC2_OK;
}

}  // namespace cc2
