// bf16 GEMM on the 5th-generation tensor cores (sm_100a):
//   out[M,N] = epilogue(A[M,K] @ W[N,K]^T), fp32 accumulation in TMEM.
//
// Structure (one persistent CTA per SM, 192 threads, 6 warps):
//   warp 0      TMA producer: streams 128x64 A tiles and BNx64 W tiles into a
//               STAGES-deep shared-memory ring (128-byte swizzle).
//   warp 1      MMA issuer: one elected thread issues tcgen05.mma
//               (cta_group::1, kind::f16, M=128, N=BN, K=16) into one of two
//               TMEM accumulators; tcgen05.commit frees ring slots and hands a
//               finished accumulator to the epilogue.
//   warps 2..5  epilogue: tcgen05.ld the accumulator (warp w reads TMEM lanes
//               32*(w%4) ..+31 = tile rows), apply the fused epilogue (RMS row
//               scale, bias, ReLU, residual add, sum-of-squares for the next
//               RMSNorm, REG-row substitution) and store bf16.
// Two accumulators let the epilogue of tile i overlap the MMAs of tile i+1.
//
// This kernel replaces the reference's F.linear / cuBLAS calls and its
// Triton RMSNorm+QKV and MLP kernels (cutechronos/model.py:178-181, 227-229,
// 271, 301-303, 308, 328-329; triton_kernels/fused_layernorm_linear.py:142-212;
// triton_kernels/fused_mlp.py:33-108).  The T5 RMSNorm is folded in: its
// weight is pre-multiplied into W's columns and its 1/rms is a per-row scale
// computed from the sum of squares accumulated by the producing epilogue.
//
// Every mbarrier wait is bounded (kWaitLimitNs); on timeout the kernel raises
// DEV_ERR_GEMM_TIMEOUT, all roles leave their loops, TMEM is freed and the
// kernel returns.
#include <cuda.h>
#include <mutex>

#include "common.cuh"

namespace cc2 {

// Device error word (bit flags DEV_ERR_*), defined in this translation unit
// because the library is built without relocatable device code.
__device__ int g_dev_error = 0;

int read_device_error(int clear, int* value) {
  CC2_CUDA(cudaMemcpyFromSymbol(value, g_dev_error, sizeof(int)));
  if (clear) {
    int z = 0;
    CC2_CUDA(cudaMemcpyToSymbol(g_dev_error, &z, sizeof(int)));
  }
  return CC2_OK;
}

namespace tc {

typedef __nv_bfloat16 bf16;

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = 128 bytes = one swizzle row
constexpr int kThreads = 192;

template <int BN>
struct Cfg {
  static constexpr int STAGES = BN == 256 ? 4 : 6;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
};

struct Epi {
  int flags;
  const float* ssq_in;
  int ssq_parts;  // 64-column groups summed by ROWSCALE
  int ssq_ld;
  float inv_dim;
  float eps;
  const float* bias;
  const bf16* resid;
  int ld_resid;
  float* ssq_out;
  const float* special;
  int sp_period;
  int sp_offset;
};

// ---- PTX wrappers -------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: false when the CTA is aborting or the limit ran out.
__device__ __noinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  for (uint32_t n = 1;; ++n) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((n & 63u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        *abort_flag = 1;
        atomicOr(&g_dev_error, DEV_ERR_GEMM_TIMEOUT);
        return false;
      }
    }
  }
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"((uint64_t)map), "r"(bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)map) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, rows of
// 128 bytes, 8-row core groups 1024 bytes apart (SBO); LBO unused for this
// layout; bits 46-47 = descriptor version 1; bits 61-63 = 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor, kind::f16: D fp32 (bits 4-5 = 1), A bf16 (7-9 = 1),
// B bf16 (10-12 = 1), both K-major (bits 15/16 = 0), N>>3 at 17-22, M>>4 at 24-28.
template <int BN>
__device__ __forceinline__ constexpr uint32_t idesc_bf16() {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
         ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               bf16* __restrict__ out, int ldo, int M, int N, int K, Epi ep) {
  using C = Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = (uint64_t*)(smem + C::STAGES * C::STAGE_BYTES);
  // bars[0..S): full, [S..2S): empty, [2S..2S+2): tmem full, [2S+2..2S+4): tmem empty
  uint32_t* tmem_slot = (uint32_t*)(bars + 2 * C::STAGES + 4);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t bar0 = smem_u32(bars);
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (C::STAGES + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * C::STAGES + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * C::STAGES + 2 + a); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int m_tiles = (M + BM - 1) / BM;
  const int n_tiles = (N + BN - 1) / BN;
  const int num_tiles = m_tiles * n_tiles;
  const int kblocks = (K + BK - 1) / BK;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int mt = tile / n_tiles, nt = tile % n_tiles;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag)) { ok = false; break; }
          const uint32_t sa = smem_u32(smem + stage * C::STAGE_BYTES);
          mbar_arrive_expect_tx(full_bar(stage), C::STAGE_BYTES);
          tma_load_2d(sa, &tmA, full_bar(stage), kb * BK, mt * BM);
          tma_load_2d(sa + C::A_BYTES, &tmB, full_bar(stage), kb * BK, nt * BN);
          if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16<BN>();
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int it = 0;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++it) {
        const int acc = it & 1;
        const uint32_t acc_phase = (uint32_t)(it >> 1) & 1u;
        if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint32_t sb = sa + C::A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            mma_bf16(d_tmem, sw128_desc(sa + 32u * k), sw128_desc(sb + 32u * k), idesc,
                     (kb | k) != 0 ? 1u : 0u);
          }
          mma_commit(empty_bar(stage));
          if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
        }
        if (ok) mma_commit(tfull_bar(acc));
      }
    }
    __syncwarp();
  } else {
    // epilogue warps 2..5 -> TMEM lane quarter q = warp % 4
    const int q = warp & 3;
    int it = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++it) {
      const int acc = it & 1;
      const uint32_t acc_phase = (uint32_t)(it >> 1) & 1u;
      if (!mbar_wait(tfull_bar(acc), acc_phase, abort_flag)) break;
      tc_fence_after();
      const int mt = tile / n_tiles, nt = tile % n_tiles;
      const int row = mt * BM + q * 32 + lane;
      const bool row_ok = row < M;
      float rs = 1.0f;
      if ((ep.flags & CC2_EPI_ROWSCALE) && row_ok) {
        float t = 0.0f;
        for (int g = 0; g < ep.ssq_parts; ++g) t += ep.ssq_in[(size_t)g * ep.ssq_ld + row];
        rs = rsqrtf(t * ep.inv_dim + ep.eps);
      }
      const bool special = (ep.flags & CC2_EPI_SPECIAL) && row_ok && (row % ep.sp_period) == ep.sp_offset;
      float ssq = 0.0f;
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 16) {
        uint32_t r[16];
        tmem_ld16(taddr + (uint32_t)c0, r);
        tmem_ld_wait();
        const int col = nt * BN + c0;
        if (row_ok && col < N) {
          float v[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]) * rs;
          if (ep.flags & CC2_EPI_BIAS) {
            const float4* bp = reinterpret_cast<const float4*>(ep.bias + col);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              float4 b4 = __ldg(bp + j);
              v[4 * j] += b4.x; v[4 * j + 1] += b4.y; v[4 * j + 2] += b4.z; v[4 * j + 3] += b4.w;
            }
          }
          if (ep.flags & CC2_EPI_RELU) {
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = fmaxf(v[j], 0.0f);
          }
          if (ep.flags & CC2_EPI_RESID) {
            const uint4* rp = reinterpret_cast<const uint4*>(ep.resid + (size_t)row * ep.ld_resid + col);
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              uint4 u = rp[j];
              const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                float2 f = __bfloat1622float2(h[e]);
                v[8 * j + 2 * e] += f.x;
                v[8 * j + 2 * e + 1] += f.y;
              }
            }
          }
          if (special) {
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = ep.special[col + j];
          }
          uint4 o[2];
          uint32_t* ow = reinterpret_cast<uint32_t*>(o);
#pragma unroll
          for (int j = 0; j < 8; ++j) ow[j] = pack_bf16(v[2 * j], v[2 * j + 1]);
          if (ep.flags & CC2_EPI_SSQ) {
            const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(o);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              float2 f = __bfloat1622float2(h[e]);
              ssq = fmaf(f.x, f.x, ssq);
              ssq = fmaf(f.y, f.y, ssq);
            }
          }
          uint4* op = reinterpret_cast<uint4*>(out + (size_t)row * ldo + col);
          op[0] = o[0];
          op[1] = o[1];
        }
        if ((c0 & 63) == 48) {  // end of a 64-column group: store its partial sum of squares
          if ((ep.flags & CC2_EPI_SSQ) && row_ok && nt * BN + (c0 & ~63) < N)
            ep.ssq_out[(size_t)((nt * BN + c0) >> 6) * ep.ssq_ld + row] = ssq;
          ssq = 0.0f;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar(acc));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ---- host side ------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)p;
  });
  return fn;
}

// 2-D bf16 tensor map over a row-major [rows, cols] matrix with row pitch ld
// (elements); box = 64 columns x box_rows rows, 128-byte swizzle, zero fill
// outside the matrix.
static int make_map(CUtensorMap* map, const void* ptr, int cols, int rows, int ld, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  CC2_REQUIRE(fn != nullptr, "cuTensorMapEncodeTiled unavailable");
  CC2_REQUIRE(((uintptr_t)ptr & 15u) == 0, "gemm operand not 16-byte aligned");
  CC2_REQUIRE((ld * 2) % 16 == 0, "gemm row pitch must be a multiple of 8 elements");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d): cols=%d rows=%d ld=%d", (int)r, cols, rows, ld);
    return CC2_E_CUDA;
  }
  return CC2_OK;
}

template <int BN>
static int launch(const CUtensorMap& ma, const CUtensorMap& mb, bf16* out, int ldo, int M, int N,
                  int K, const Epi& ep, cudaStream_t st) {
  using C = Cfg<BN>;
  static unsigned long long attr_set = 0;  // one bit per device
  int dev = 0;
  CC2_CUDA(cudaGetDevice(&dev));
  if (dev >= 64 || !((attr_set >> dev) & 1ull)) {
    CC2_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  C::SMEM));
    if (dev < 64) attr_set |= 1ull << dev;
  }
  const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int grid = tiles < num_sms() ? tiles : num_sms();
  gemm_tc_kernel<BN><<<grid, kThreads, C::SMEM, st>>>(ma, mb, out, ldo, M, N, K, ep);
  CC2_CHECK_LAUNCH();
  return CC2_OK;
}

}  // namespace tc

int launch_gemm_tc(const void* A, int lda, const void* W, int ldw, void* out, int ldo, int M, int N,
                   int K, const cc2_epilogue* e, cudaStream_t st) {
  using namespace tc;
  CC2_REQUIRE(M > 0 && N > 0 && K > 0, "gemm: bad sizes M=%d N=%d K=%d", M, N, K);
  CC2_REQUIRE(N % 16 == 0, "gemm(bf16): N must be a multiple of 16 (got %d)", N);
  CC2_REQUIRE(((uintptr_t)out & 15u) == 0 && ldo % 8 == 0, "gemm(bf16): out alignment");
  Epi ep{};
  ep.flags = e ? e->flags : 0;
  if (e) {
    ep.ssq_in = e->ssq_in;
    ep.ssq_parts = (e->norm_dim + 63) / 64;
    ep.ssq_ld = e->ssq_ld;
    ep.inv_dim = e->norm_dim > 0 ? 1.0f / (float)e->norm_dim : 0.0f;
    ep.eps = e->eps;
    ep.bias = e->bias;
    ep.resid = (const bf16*)e->resid;
    ep.ld_resid = e->ld_resid;
    ep.ssq_out = e->ssq_out;
    ep.special = e->special;
    ep.sp_period = e->special_period;
    ep.sp_offset = e->special_offset;
  }
  CC2_REQUIRE(!(ep.flags & CC2_EPI_ROWSCALE) || (ep.ssq_in && e->norm_dim > 0), "gemm: rowscale args");
  CC2_REQUIRE(!(ep.flags & CC2_EPI_BIAS) || (ep.bias && ((uintptr_t)ep.bias & 15u) == 0),
              "gemm: bias must be non-null and 16-byte aligned");
  CC2_REQUIRE(!(ep.flags & CC2_EPI_RESID) ||
                  (ep.resid && ((uintptr_t)ep.resid & 15u) == 0 && ep.ld_resid % 8 == 0),
              "gemm: resid alignment");
  CC2_REQUIRE(!(ep.flags & CC2_EPI_SSQ) || ep.ssq_out, "gemm: ssq_out null");
  CC2_REQUIRE(!(ep.flags & (CC2_EPI_SSQ | CC2_EPI_ROWSCALE)) || ep.ssq_ld >= M, "gemm: ssq_ld must be >= M");
  CC2_REQUIRE(!(ep.flags & CC2_EPI_SPECIAL) || (ep.special && ep.sp_period > 0), "gemm: special args");
  const int tiles256 = ((M + BM - 1) / BM) * ((N + 255) / 256);
  const bool use256 = N >= 256 && tiles256 >= num_sms();
  CUtensorMap ma, mb;
  CC2_TRY(make_map(&ma, A, K, M, lda, BM));
  if (use256) {
    CC2_TRY(make_map(&mb, W, K, N, ldw, 256));
    return launch<256>(ma, mb, (bf16*)out, ldo, M, N, K, ep, st);
  }
  CC2_TRY(make_map(&mb, W, K, N, ldw, 128));
  return launch<128>(ma, mb, (bf16*)out, ldo, M, N, K, ep, st);
}

}  // namespace cc2
