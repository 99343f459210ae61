// Device side of the forecasting pipeline around the forward
// (pipeline.py:221-322 and 24-58 of the reference, which run these steps as
// Python loops and CPU tensor ops):
//
//  * stack_series: ragged series, concatenated in one buffer with int64
//    offsets, become the (B, L) NaN-left-padded batch the forward takes; a
//    series longer than L keeps its last L values (_left_pad_and_stack_rows +
//    _finalize_context_batch).
//  * select_quantiles: the (B, Q, ld) forecasts of the forward become fp32
//    requested levels, each either a trained level (gathered) or a linear
//    interpolation between two neighbours, computed as the reference's CPU
//    path does: fl(fl(a * w_lo) + fl(b * w_hi)) with fp32 weights and no
//    fused multiply-add, so results are bit-identical; the median row can be
//    written alongside.  Output layout (B, nq, H) (predict) or (B, H, nq)
//    (predict_quantiles, predict_df).
//
// Both kernels move a few bytes per element and are HBM- or launch-bound.
#include "common.cuh"

namespace cc2 {
namespace {

__global__ void __launch_bounds__(256)
stack_series_kernel(const float* __restrict__ values, const int64_t* __restrict__ offsets, int B, int L,
                    float* __restrict__ out) {
  const int b = blockIdx.y;
  const int64_t beg = offsets[b], end = offsets[b + 1];
  const int64_t len = end - beg, take = len < (int64_t)L ? len : (int64_t)L;
  const int pad = L - (int)take;
  const float* src = values + (end - take);  // the kept tail of the row
  for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < L; t += gridDim.x * blockDim.x)
    out[(size_t)b * L + t] = t < pad ? __int_as_float(0x7fc00000) : src[t - pad];
}

constexpr int kMaxLevels = 64;

struct LevelTable {
  int lo[kMaxLevels], hi[kMaxLevels];
  float w_lo[kMaxLevels], w_hi[kMaxLevels];
};

// One thread per (series, step): reads the Q trained values of that step once
// through the cache and writes every requested level.
template <typename T>
__global__ void __launch_bounds__(256)
select_quantiles_kernel(const T* __restrict__ preds, int B, int Q, int ld, int H, int nq, LevelTable lv,
                        int layout, float* __restrict__ out, int median_q, float* __restrict__ median) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)B * H) return;
  const int b = (int)(i / H), t = (int)(i % H);
  const T* p = preds + (size_t)b * Q * ld + t;
  for (int j = 0; j < nq; ++j) {
    const float a = Elem<T>::to_f(p[(size_t)lv.lo[j] * ld]);
    float v = a;
    if (lv.hi[j] != lv.lo[j]) {
      const float c = Elem<T>::to_f(p[(size_t)lv.hi[j] * ld]);
      v = __fadd_rn(__fmul_rn(a, lv.w_lo[j]), __fmul_rn(c, lv.w_hi[j]));
    }
    const size_t o = layout == 0 ? ((size_t)b * nq + j) * H + t : ((size_t)b * H + t) * nq + j;
    out[o] = v;
  }
  if (median) median[(size_t)b * H + t] = Elem<T>::to_f(p[(size_t)median_q * ld]);
}

}  // namespace

int launch_stack_series(const float* values, const int64_t* offsets, int B, int L, float* out, cudaStream_t st) {
  CC2_REQUIRE(B > 0 && L > 0, "stack_series: bad sizes B=%d L=%d", B, L);
  CC2_REQUIRE(values && offsets && out, "stack_series: null pointer");
  dim3 grid((L + 255) / 256 < 64 ? (L + 255) / 256 : 64, B);
  CC2_REQUIRE(B <= 65535, "stack_series: B=%d exceeds 65535", B);
  stack_series_kernel<<<grid, 256, 0, st>>>(values, offsets, B, L, out);
  CC2_CHECK_LAUNCH();
  return CC2_OK;
}

int launch_select_quantiles(int dtype, const void* preds, int B, int Q, int ld, int H, int nq, const int* lo,
                            const int* hi, const float* w_lo, const float* w_hi, int layout, float* out,
                            int median_q, float* median, cudaStream_t st) {
  CC2_REQUIRE(B > 0 && Q > 0 && H > 0 && ld >= H, "select_quantiles: bad sizes B=%d Q=%d ld=%d H=%d", B, Q, ld, H);
  CC2_REQUIRE(nq >= 0 && nq <= kMaxLevels, "select_quantiles: nq=%d outside [0, %d]", nq, kMaxLevels);
  CC2_REQUIRE(preds && (nq == 0 || (out && lo && hi && w_lo && w_hi)), "select_quantiles: null pointer");
  CC2_REQUIRE(layout == 0 || layout == 1, "select_quantiles: layout must be 0 or 1");
  CC2_REQUIRE(!median || (median_q >= 0 && median_q < Q), "select_quantiles: median_q=%d outside [0, Q)", median_q);
  CC2_REQUIRE(dtype == CC2_BF16 || dtype == CC2_F32, "select_quantiles: dtype %d", dtype);
  LevelTable lv{};
  for (int j = 0; j < nq; ++j) {
    CC2_REQUIRE(lo[j] >= 0 && lo[j] < Q && hi[j] >= 0 && hi[j] < Q, "select_quantiles: level %d index outside [0, Q)",
                j);
    lv.lo[j] = lo[j];
    lv.hi[j] = hi[j];
    lv.w_lo[j] = w_lo[j];
    lv.w_hi[j] = w_hi[j];
  }
  const int64_t n = (int64_t)B * H;
  const int blocks = (int)((n + 255) / 256);
  if (dtype == CC2_BF16)
    select_quantiles_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>((const __nv_bfloat16*)preds, B, Q, ld, H, nq, lv,
                                                                   layout, out, median_q, median);
  else
    select_quantiles_kernel<float><<<blocks, 256, 0, st>>>((const float*)preds, B, Q, ld, H, nq, lv, layout, out,
                                                           median_q, median);
  CC2_CHECK_LAUNCH();
  return CC2_OK;
}

}  // namespace cc2

extern "C" {

int cc2_stack_series(const float* values, const int64_t* offsets, int B, int L, float* out, void* stream) {
  cc2::clear_error();
  return cc2::launch_stack_series(values, offsets, B, L, out, (cudaStream_t)stream);
}

int cc2_select_quantiles(int dtype, const void* preds, int B, int Q, int ld, int H, int nq, const int* lo,
                         const int* hi, const float* w_lo, const float* w_hi, int layout, float* out, int median_q,
                         float* median, void* stream) {
  cc2::clear_error();
  return cc2::launch_select_quantiles(dtype, preds, B, Q, ld, H, nq, lo, hi, w_lo, w_hi, layout, out, median_q,
                                      median, (cudaStream_t)stream);
}

}  // extern "C"
