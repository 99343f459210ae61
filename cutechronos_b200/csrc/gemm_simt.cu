// fp32 GEMM on CUDA cores for the fp32 model mode:
//   out[M,N] = epilogue(A[M,K] @ W[N,K]^T)
// tcgen05 has no full-precision fp32 kind (kind::tf32 rounds inputs to 10
// mantissa bits), so the fp32 mode, whose parity bar is max-abs 1e-4 against
// the reference's fp32 CPU path, runs these FFMA kernels.  They apply the same
// fused epilogue as the tensor-core kernel (row scale, bias, ReLU, residual,
// per-64-column sums of squares, special rows).
//
// Small M (batch-1 serving: 37 rows for a 512-step context) leaves a 64x64
// tiling with a handful of CTAs, so when a scratch buffer is available the
// K dimension is split: gemm_f32_kernel<true> writes fp32 partial sums per
// K-slice, and splitk_epilogue_kernel adds the slices in a fixed order (the
// result does not depend on timing) and applies the epilogue.
#include "common.cuh"

namespace cc2 {
namespace {

constexpr int TM = 64, TN = 64, TK = 16, kThreads = 256;

__device__ __forceinline__ float row_scale_f32(const cc2_epilogue& ep, int row, float inv_dim) {
  float t = 0.0f;
  const int parts = (ep.norm_dim + 63) / 64;
  for (int g = 0; g < parts; ++g) t += ep.ssq_in[(size_t)g * ep.ssq_ld + row];
  return rsqrtf(t * inv_dim + ep.eps);
}

// SPLIT = false: full K, epilogue applied.  SPLIT = true: K range
// [blockIdx.z * kchunk, +kchunk), raw partial sums to part[z][M][N].
template <bool SPLIT>
__global__ void __launch_bounds__(kThreads)
gemm_f32_kernel(const float* __restrict__ A, int lda, const float* __restrict__ W, int ldw, float* out, int ldo,
                int M, int N, int K, cc2_epilogue ep, int kchunk, float* __restrict__ part) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float As[2][TK][TM + 4];
  __shared__ float Ws[2][TK][TN + 4];
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN;
  const int kbeg = SPLIT ? blockIdx.z * kchunk : 0;
  const int kend = SPLIT ? min(K, kbeg + kchunk) : K;
  const int lr = tid >> 2, lk = (tid & 3) * 4;
  float acc[4][4] = {};
  float ra[4], rw[4];
  auto load = [&](int k0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int k = k0 + lk + i;
      const int am = m0 + lr, wn = n0 + lr;
      ra[i] = (am < M && k < kend) ? A[(size_t)am * lda + k] : 0.0f;
      rw[i] = (wn < N && k < kend) ? W[(size_t)wn * ldw + k] : 0.0f;
    }
  };
  auto stash = [&](int b) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      As[b][lk + i][lr] = ra[i];
      Ws[b][lk + i][lr] = rw[i];
    }
  };
  load(kbeg);
  stash(0);
  __syncthreads();
  int b = 0;
  for (int k0 = kbeg; k0 < kend; k0 += TK) {
    const bool more = k0 + TK < kend;
    if (more) load(k0 + TK);  // next tile in flight while this one is used
#pragma unroll
    for (int k = 0; k < TK; ++k) {
      float a[4], w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[b][k][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) w[j] = Ws[b][k][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], w[j], acc[i][j]);
    }
    if (more) stash(b ^ 1);
    __syncthreads();
    b ^= 1;
  }
  if (SPLIT) {
    float* dst = part + (size_t)blockIdx.z * M * N;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int row = m0 + ty + 16 * i;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int col = n0 + tx + 16 * j;
        if (row < M && col < N) dst[(size_t)row * N + col] = acc[i][j];
      }
    }
    return;
  }
  const float inv_dim = ep.norm_dim > 0 ? 1.0f / (float)ep.norm_dim : 0.0f;
  const float* resid = (const float*)ep.resid;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int row = m0 + ty + 16 * i;
    const bool row_ok = row < M;
    const float rs = ((ep.flags & CC2_EPI_ROWSCALE) && row_ok) ? row_scale_f32(ep, row, inv_dim) : 1.0f;
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

// One warp per (row, 64-column group): sums the K-slices in order, applies
// the epilogue and writes the group's sum of squares.
__global__ void __launch_bounds__(256)
splitk_epilogue_kernel(const float* __restrict__ part, int slices, float* out, int ldo, int M, int N,
                       cc2_epilogue ep) {
  pdl_launch_dependents();
  pdl_wait();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int groups = (N + 63) / 64;
  if (warp >= M * groups) return;
  const int row = warp / groups, g = warp % groups;
  const float inv_dim = ep.norm_dim > 0 ? 1.0f / (float)ep.norm_dim : 0.0f;
  const float rs = (ep.flags & CC2_EPI_ROWSCALE) ? row_scale_f32(ep, row, inv_dim) : 1.0f;
  const bool special = (ep.flags & CC2_EPI_SPECIAL) && (row % ep.special_period) == ep.special_offset;
  const float* resid = (const float*)ep.resid;
  float ssq = 0.0f;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int col = g * 64 + h * 32 + lane;
    if (col >= N) continue;
    float v = 0.0f;
    for (int z = 0; z < slices; ++z) v += part[((size_t)z * M + row) * N + col];
    v *= rs;
    if (ep.flags & CC2_EPI_BIAS) v += ep.bias[col];
    if (ep.flags & CC2_EPI_RELU) v = fmaxf(v, 0.0f);
    if (ep.flags & CC2_EPI_RESID) v += resid[(size_t)row * ep.ld_resid + col];
    if (special) v = ep.special[col];
    ssq = fmaf(v, v, ssq);
    out[(size_t)row * ldo + col] = v;
  }
  if (ep.flags & CC2_EPI_SSQ) {
    for (int o = 16; o > 0; o >>= 1) ssq += __shfl_xor_sync(0xffffffffu, ssq, o);
    if (lane == 0) ep.ssq_out[(size_t)g * ep.ssq_ld + row] = ssq;
  }
}

}  // namespace

size_t gemm_f32_splitk_floats() {
  // A split GEMM has tiles < num_sms() and at most ceil(2 num_sms / tiles)
  // slices of M x N <= tiles x TM x TN floats, so this bound never limits the
  // slice count chosen below.
  return (size_t)3 * num_sms() * TM * TN;
}

int launch_gemm_f32(const void* A, int lda, const void* W, int ldw, void* out, int ldo, int M, int N, int K,
                    const cc2_epilogue* e, cudaStream_t st, float* scratch, size_t scratch_floats) {
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
  CC2_REQUIRE(!(ep.flags & CC2_EPI_ROPE), "gemm(f32): CC2_EPI_ROPE is a bf16 epilogue");
  CC2_REQUIRE(!(ep.flags & CC2_EPI_LO), "gemm(f32): CC2_EPI_LO is a bf16 epilogue");
  const int tiles = ((N + TN - 1) / TN) * ((M + TM - 1) / TM);
  int slices = 1;
  if (scratch && tiles < num_sms() && K >= 8 * TK) {
    slices = std::min((2 * num_sms() + tiles - 1) / tiles, K / (4 * TK));
    slices = (int)std::min<size_t>((size_t)slices, scratch_floats / ((size_t)M * N));
  }
  if (slices >= 2) {
    const int kchunk = ((K + slices - 1) / slices + TK - 1) / TK * TK;
    slices = (K + kchunk - 1) / kchunk;
    dim3 grid((N + TN - 1) / TN, (M + TM - 1) / TM, slices);
    CC2_CUDA(launch_k(gemm_f32_kernel<true>, grid, kThreads, 0, st, (const float*)A, lda, (const float*)W, ldw, nullptr, 0, M, N,
                                                     K, ep, kchunk, scratch));
    CC2_CHECK_LAUNCH();
    const int warps = M * ((N + 63) / 64);
    CC2_CUDA(launch_k(splitk_epilogue_kernel, (warps * 32 + 255) / 256, 256, 0, st, scratch, slices, (float*)out, ldo, M, N, ep));
    CC2_CHECK_LAUNCH();
    return CC2_OK;
  }
  dim3 grid((N + TN - 1) / TN, (M + TM - 1) / TM);
  CC2_CUDA(launch_k(gemm_f32_kernel<false>, grid, kThreads, 0, st, (const float*)A, lda, (const float*)W, ldw, (float*)out, ldo, M,
                                                    N, K, ep, K, nullptr));
  CC2_CHECK_LAUNCH();
  return CC2_OK;
}

}  // namespace cc2
