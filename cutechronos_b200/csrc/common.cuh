// Shared helpers of the cc2 engine: status handling, element conversions,
// the device-side error word used by bounded waits.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <cstdio>
#include <string>
#include <utility>

#include "../../include/cc2.h"

namespace cc2 {

// ---- host-side status -------------------------------------------------------
void set_error(const char* fmt, ...);
void clear_error();

#define CC2_REQUIRE(cond, ...)                 \
  do {                                         \
    if (!(cond)) {                             \
      ::cc2::set_error(__VA_ARGS__);           \
      return CC2_E_INVALID;                    \
    }                                          \
  } while (0)

#define CC2_CUDA(call)                                                        \
  do {                                                                        \
    cudaError_t e_ = (call);                                                  \
    if (e_ != cudaSuccess) {                                                  \
      ::cc2::set_error("%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                       __FILE__, __LINE__);                                   \
      return CC2_E_CUDA;                                                      \
    }                                                                         \
  } while (0)

#define CC2_CHECK_LAUNCH()                                                     \
  do {                                                                         \
    cudaError_t e_ = cudaGetLastError();                                       \
    if (e_ != cudaSuccess) {                                                   \
      ::cc2::set_error("kernel launch failed: %s (%s:%d)", cudaGetErrorString(e_), \
                       __FILE__, __LINE__);                                    \
      return CC2_E_CUDA;                                                       \
    }                                                                          \
  } while (0)

#define CC2_TRY(expr)          \
  do {                         \
    int s_ = (expr);           \
    if (s_ != CC2_OK) return s_; \
  } while (0)

int num_sms();

// ---- device-side error word -------------------------------------------------
// Bit flags written by kernels whose bounded waits gave up.
enum : int {
  DEV_ERR_GEMM_TIMEOUT = 1,
  DEV_ERR_ATTN_TIMEOUT = 2,
  DEV_ERR_LAYER_TIMEOUT = 4,  // grid barrier of the layer-persistent forward
};
// Read (and optionally clear) the device error words of the current device.
int read_device_error(int clear, int* value);
int read_attention_error(int clear, int* value);

// Wall-clock limit for any spin-wait inside a kernel (nanoseconds).
constexpr unsigned long long kWaitLimitNs = 2000ull * 1000ull * 1000ull;

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- element conversions ----------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float to_f(float x) { return x; }
  static __device__ __forceinline__ float from_f(float x) { return x; }
  static constexpr int code = CC2_F32;
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
  static constexpr int code = CC2_BF16;
};

template <typename T> __device__ __forceinline__ float tof(T x) { return Elem<T>::to_f(x); }
template <typename T> __device__ __forceinline__ T fromf(float x) { return Elem<T>::from_f(x); }
// Round-trip through T (models the reference's intermediate casts).
template <typename T> __device__ __forceinline__ float roundT(float x) { return tof<T>(fromf<T>(x)); }

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// ---- programmatic dependent launch ------------------------------------------
// Every kernel of the forward is launched with programmatic stream
// serialization (unless turned off by cc2_set_launch_overlap): it may start
// while the kernel before it on the stream is still running.  Each kernel
// therefore (1) signals at its start that the next one may be scheduled and
// (2) executes pdl_wait() - which returns once the previous kernel has
// completed and its writes are visible - before it reads or writes any
// activation memory; only its prologue (barrier set-up, TMEM allocation,
// descriptor prefetch, weight-only work) overlaps the previous kernel.
// Outside a programmatic launch both instructions are no-ops.
// The fp32 forward runs without it: its CUDA-core kernels span several waves,
// and there the early launches cost more than they hide (configs[0] batch-1
// latency 1.39 ms without, 2.02 ms with); the bf16 forward's kernels are
// persistent and gain (batch-1 1.49 -> 1.30 ms).  t_launch_overlap is cleared
// by the forward of an fp32 model for its duration.
extern int g_launch_overlap;
extern thread_local int t_launch_overlap;
inline bool launch_overlap() { return g_launch_overlap != 0 && t_launch_overlap != 0; }

__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                            Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = launch_overlap() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace cc2
