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
//               RMSNorm, REG-row substitution) in 32x64 boxes staged in shared
//               memory: the residual box arrives by TMA, the bf16 result leaves
//               by a TMA bulk-tensor store.
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
#include <algorithm>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "attn_set_tile.cuh"

namespace cc2 {

// Device error word (bit flags DEV_ERR_*), defined in this translation unit
// because the library is built without relocatable device code.
__device__ int g_dev_error = 0;

// Test hook (cc2_test_starve_gemm), one-shot: the first single-SM GEMM CTA
// that finds it set clears it and skips the load of its first k-block, so the
// MMA warp's bounded wait on that stage runs out.  Only loads that were issued are in flight when the
// kernel leaves, and they land within microseconds of the 2 s limit.
__device__ int g_gemm_starve = 0;
// Test hook (cc2_test_starve_layer_barrier), one-shot: CTA 0 of the next
// layer-persistent launch leaves at its first grid barrier without arriving.
__device__ int g_chain_starve = 0;

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
  static constexpr int SMEM = STAGES * STAGE_BYTES + 8 * 32 * 64 * 2 + 1024 + 256;
};

// The single-SM kernel moves KPS = 2 k-blocks per ring stage (one mbarrier
// round trip per 2 k-blocks): a TMA probe on this pool streamed ~58 GB/s per
// SM with one 16 KB box per barrier and ~116 GB/s with two, whatever the
// number of barriers in flight - the per-barrier round trip, not the bytes,
// bounded the k-loop of few-row GEMMs (0.29 us per k-block).
// AR: rows of an A slot.  With at most 64 token rows (batch-1 serving at
// context <= 1024) the A box never holds more than 64 rows, so the ring uses
// 64-row A slots and 4 k-blocks per stage: twice the bytes per barrier round
// trip in the same shared memory.  The M = 128 MMA still reads 128 rows from
// the slot; rows past the box read the next slot's bytes and only produce
// accumulator rows that are never stored.
template <int BN, int AR = BM, int KPS_ = 2>
struct Cfg2 {
  static constexpr int KPS = KPS_;
  static constexpr int A_BYTES = AR * BK * 2;  // per k-block
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = KPS * (A_BYTES + B_BYTES);  // [A kb0][A kb1]..[B kb0][B kb1]..
  static constexpr int STAGES = (192 * 1024) / STAGE_BYTES;      // 256: 2, 128: 3, 64: 4 (64-row slots: 3)
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 8 * 32 * 64 * 2 + 1024 + 256;
  static_assert(STAGES >= 2 && SMEM <= 232448, "single-SM GEMM ring");
  // the last A slot of a stage, read as 128 rows, stays inside the stage
  static_assert((KPS - 1) * A_BYTES + BM * BK * 2 <= STAGE_BYTES, "A slot read past its stage");
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
  const uint32_t* rope_cs;  // [pos][32] packed (cos, sin) bf16 pairs
  int rope_period;
  int rope_cols;
  bf16* lo_out;          // LO: low halves of the result
  const bf16* resid_lo;  // LO + RESID: low halves of the residual
  int ld_lo;
  int wpre;  // W is constant (packed model weights): the single-SM kernel may load
             // it before the grid dependency wait, under the previous kernel's tail
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
__device__ __noinline__ bool mbar_wait_slow(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
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
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  return mbar_try_wait(bar, parity) || mbar_wait_slow(bar, parity, abort_flag);
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

// TMA bulk-tensor store of a staged smem box, bulk-group completion.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"((uint64_t)map),
               "r"(src), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// Epilogue staging box: 32 rows x 64 bf16 columns (4 KB) in 128-byte swizzle
// (16-byte chunk c of row r lives at chunk c ^ (r & 7)).  A box is filled by
// TMA with the residual tile (RESID), combined with the accumulator by its
// warp, and written back to global memory by a TMA bulk-tensor store.
constexpr int kEpiBox = 32 * 64 * 2;

// Loads the 32 packed (cos, sin) pairs of this row's token position.
__device__ __forceinline__ void load_rope_row(const Epi& ep, int row, bool row_ok, uint32_t (&cs)[32]) {
  const uint4* src = reinterpret_cast<const uint4*>(ep.rope_cs + (size_t)(row_ok ? row % ep.rope_period : 0) * 32);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint4 u = __ldg(src + j);
    cs[4 * j] = u.x; cs[4 * j + 1] = u.y; cs[4 * j + 2] = u.z; cs[4 * j + 3] = u.w;
  }
}
// Rotate-half RoPE on one 64-column head held in r (row-scaled first).
// Here and in the epilogue every product and sum is an explicit round-to-
// nearest intrinsic: the compiler may not contract them into FMAs one way in
// one tile kernel and another way in the next, so every tile path rounds the
// same (results do not depend on which kernel a batch size selects).
__device__ __forceinline__ void rope_group(uint32_t* r, const uint32_t (&cs)[32], float rs) {
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const float c = __uint_as_float(cs[i] << 16), sn = __uint_as_float(cs[i] & 0xffff0000u);
    const float x1 = __fmul_rn(__uint_as_float(r[i]), rs), x2 = __fmul_rn(__uint_as_float(r[i + 32]), rs);
    r[i] = __float_as_uint(__fmaf_rn(x1, c, -__fmul_rn(x2, sn)));
    r[i + 32] = __float_as_uint(__fmaf_rn(x2, c, __fmul_rn(x1, sn)));
  }
}

// Applies the fused epilogue to one 64-column group of one row (values r[64]
// from TMEM) and writes the bf16 result into the swizzled box.  Returns the
// group's sum of squares of the stored values (columns < N).
// Low halves (CC2_EPI_LO) live in a 32-row interleaved layout, so that the
// 32 lanes of an epilogue warp (one row each) touch 512 contiguous bytes per
// 16-byte access: element (row, col) at
// ((row / 32 * ld / 8 + col / 8) * 32 + row % 32) * 8 + col % 8.
__device__ __forceinline__ size_t lo_index(int row, int col, int ld) {
  return (((size_t)(row >> 5) * (size_t)(ld >> 3) + (size_t)(col >> 3)) * 32 + (size_t)(row & 31)) * 8;
}

// LO (CC2_EPI_LO): the residual's low halves are added after its bf16 high
// halves, and the result's low halves bf16(v - bf16(v)) go straight to global
// memory (interleaved layout above: coalesced across the warp's rows).
// Loads one 64-column group's residual low halves of this lane's row (zeros
// outside the matrix).
// CG: through L2 only - for data that other SMs wrote earlier in the same
// kernel (the layer-persistent forward); otherwise the read-only path.
template <bool CG = false>
__device__ __forceinline__ void load_lo_group(uint4 (&rl)[8], const Epi& ep, int row, bool row_ok, int col0, int N) {
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    rl[c] = make_uint4(0u, 0u, 0u, 0u);
    if (ep.resid_lo && row_ok && col0 + c * 8 < N) {
      if (CG)
        asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(rl[c].x), "=r"(rl[c].y), "=r"(rl[c].z), "=r"(rl[c].w)
                     : "l"(ep.resid_lo + lo_index(row, col0 + c * 8, ep.ld_lo)));
      else
        asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(rl[c].x), "=r"(rl[c].y), "=r"(rl[c].z), "=r"(rl[c].w)
                     : "l"(ep.resid_lo + lo_index(row, col0 + c * 8, ep.ld_lo)));
    }
  }
}

// rl: the group's residual low halves (LO with RESID), loaded by the caller
// ahead of time so that their latency overlaps the accumulator wait.
__device__ __forceinline__ float epilogue_group(const Epi& ep, const int flags, const uint32_t* r, float rs, bool special, int col0,
                                                int N, uint32_t box, int lane, bool resid, int row, bool row_ok,
                                                const uint4 (&rl)[8]) {
  const uint32_t rsw = (uint32_t)(lane & 7);
  float ssq = 0.0f;
  const bool lo = (flags & CC2_EPI_LO) != 0;
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const int col = col0 + c * 8;
    const uint32_t addr = box + (uint32_t)lane * 128u + (((uint32_t)c ^ rsw) << 4);
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = __fmul_rn(__uint_as_float(r[c * 8 + j]), rs);
    const bool col_ok = col < N;
    if ((flags & CC2_EPI_BIAS) && col_ok) {
      const float4 b0 = __ldg(reinterpret_cast<const float4*>(ep.bias + col));
      const float4 b1 = __ldg(reinterpret_cast<const float4*>(ep.bias + col) + 1);
      v[0] = __fadd_rn(v[0], b0.x); v[1] = __fadd_rn(v[1], b0.y); v[2] = __fadd_rn(v[2], b0.z);
      v[3] = __fadd_rn(v[3], b0.w); v[4] = __fadd_rn(v[4], b1.x); v[5] = __fadd_rn(v[5], b1.y);
      v[6] = __fadd_rn(v[6], b1.z); v[7] = __fadd_rn(v[7], b1.w);
    }
    if (flags & CC2_EPI_RELU) {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = fmaxf(v[j], 0.0f);
    }
    if (resid) {
      uint4 u;
      asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(u.x), "=r"(u.y), "=r"(u.z), "=r"(u.w) : "r"(addr));
      const __nv_bfloat162* hh = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(hh[e]);
        v[2 * e] = __fadd_rn(v[2 * e], f.x);
        v[2 * e + 1] = __fadd_rn(v[2 * e + 1], f.y);
      }
      if (lo) {
        const __nv_bfloat162* ll = reinterpret_cast<const __nv_bfloat162*>(&rl[c]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(ll[e]);
          v[2 * e] = __fadd_rn(v[2 * e], f.x);
          v[2 * e + 1] = __fadd_rn(v[2 * e + 1], f.y);
        }
      }
    }
    if (special && col_ok) {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = ep.special[col + j];
    }
    uint4 o;
    o.x = pack_bf16(v[0], v[1]); o.y = pack_bf16(v[2], v[3]);
    o.z = pack_bf16(v[4], v[5]); o.w = pack_bf16(v[6], v[7]);
    if (lo) {
      const __nv_bfloat162* hh = reinterpret_cast<const __nv_bfloat162*>(&o);
      float d[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(hh[e]);
        d[2 * e] = __fsub_rn(v[2 * e], f.x);
        d[2 * e + 1] = __fsub_rn(v[2 * e + 1], f.y);
      }
      if (ep.lo_out && row_ok && col_ok) {
        uint4 lw;
        lw.x = pack_bf16(d[0], d[1]); lw.y = pack_bf16(d[2], d[3]);
        lw.z = pack_bf16(d[4], d[5]); lw.w = pack_bf16(d[6], d[7]);
        asm volatile("st.global.L1::no_allocate.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(ep.lo_out + lo_index(row, col, ep.ld_lo)),
                     "r"(lw.x), "r"(lw.y), "r"(lw.z), "r"(lw.w)
                     : "memory");
      }
      if ((flags & CC2_EPI_SSQ) && col_ok) {
#pragma unroll
        for (int j = 0; j < 8; ++j) ssq = fmaf(v[j], v[j], ssq);
      }
    } else if ((flags & CC2_EPI_SSQ) && col_ok) {
      const __nv_bfloat162* hh = reinterpret_cast<const __nv_bfloat162*>(&o);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(hh[e]);
        ssq = fmaf(f.x, f.x, ssq);
        ssq = fmaf(f.y, f.y, ssq);
      }
    }
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(o.x), "r"(o.y), "r"(o.z), "r"(o.w)
                 : "memory");
  }
  return ssq;
}

template <bool CG = false>
__device__ __forceinline__ float row_scale(const Epi& ep, const int flags, int row, bool row_ok) {
  if (!(flags & CC2_EPI_ROWSCALE) || !row_ok) return 1.0f;
  float t = 0.0f;
  for (int g = 0; g < ep.ssq_parts; ++g) {
    const float* q = ep.ssq_in + (size_t)g * ep.ssq_ld + row;
    t = __fadd_rn(t, CG ? __ldcg(q) : *q);
  }
  return rsqrtf(__fmaf_rn(t, ep.inv_dim, ep.eps));
}

template <int BN, int AR = BM, int KPS = 2>
__global__ void __launch_bounds__(kThreads, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmR,
               const __grid_constant__ CUtensorMap tmAt, int tail_rows, int M, int N, int K, Epi ep) {
  pdl_launch_dependents();
  using C = Cfg2<BN, AR, KPS>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* epi_smem = smem + C::STAGES * C::STAGE_BYTES;  // 4 warps x 2 boxes
  uint64_t* bars = (uint64_t*)(epi_smem + 8 * kEpiBox);
  // bars: [0,S) full, [S,2S) empty, [2S,2S+2) tmem full, [2S+2,2S+4) tmem empty,
  //       [2S+4, 2S+12) residual box loaded (warp q, box b) at 2S+4+2q+b
  uint32_t* tmem_slot = (uint32_t*)(bars + 2 * C::STAGES + 12);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t bar0 = smem_u32(bars);
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (C::STAGES + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * C::STAGES + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * C::STAGES + 2 + a); };
  auto rbar = [&](int q, int b) { return bar0 + 8u * (2 * C::STAGES + 4 + 2 * q + b); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 4);
    }
    for (int i = 0; i < 8; ++i) mbar_init(bar0 + 8u * (2 * C::STAGES + 4 + i), 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
    tma_prefetch_desc(&tmR);
    tma_prefetch_desc(&tmAt);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // the producer warp waits below, after it has issued the weight loads it may issue early
  if (warp != 0 || !ep.wpre) pdl_wait();  // activations are read from now on
  const uint32_t tmem_base = *tmem_slot;

  const int m_tiles = (M + BM - 1) / BM;
  const int n_tiles = (N + BN - 1) / BN;
  const int num_tiles = m_tiles * n_tiles;
  const int kblocks = (K + BK - 1) / BK;

  if (warp == 0) {
    if (lane == 0) {
      // Weights do not depend on the previous kernel: with ep.wpre the first
      // tile's W boxes for the first `pre` (fresh) stages are issued before the
      // grid dependency wait, so their HBM latency overlaps the previous
      // kernel's tail; the stage's full barrier expects the A bytes too, which
      // are issued after the wait.
      int pre = 0;
      if (ep.wpre && (int)blockIdx.x < num_tiles) {
        const int mt = (int)blockIdx.x / n_tiles, nt = (int)blockIdx.x % n_tiles;
        const bool tail = mt == m_tiles - 1 && tail_rows < BM;
        const uint32_t a_bytes = tail ? (uint32_t)tail_rows * BK * 2 : (uint32_t)C::A_BYTES;
        for (int kb = 0; kb < kblocks && pre < C::STAGES; kb += C::KPS, ++pre) {
          const uint32_t sb = smem_u32(smem + pre * C::STAGE_BYTES) + C::KPS * C::A_BYTES;
          const int nk = min(C::KPS, kblocks - kb);
          mbar_arrive_expect_tx(full_bar(pre), (uint32_t)nk * (a_bytes + (uint32_t)C::B_BYTES));
          for (int j = 0; j < nk; ++j) tma_load_2d(sb + j * C::B_BYTES, &tmB, full_bar(pre), (kb + j) * BK, nt * BN);
        }
        pdl_wait();
      }
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int mt = tile / n_tiles, nt = tile % n_tiles;
        for (int kb = 0; kb < kblocks; kb += C::KPS) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag)) { ok = false; break; }
          if (kb == 0 && tile == (int)blockIdx.x && *(volatile int*)&g_gemm_starve &&
              atomicExch(&g_gemm_starve, 0)) {
            if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
            continue;  // test hook: this stage never fills
          }
          const uint32_t sa = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint32_t sb = sa + C::KPS * C::A_BYTES;
          const int nk = min(C::KPS, kblocks - kb);
          // the last row tile loads only its tail_rows rows (a smaller box); the MMA
          // rows past them only produce accumulator rows that are never stored
          const bool tail = mt == m_tiles - 1 && tail_rows < BM;
          const uint32_t a_bytes = tail ? (uint32_t)tail_rows * BK * 2 : (uint32_t)C::A_BYTES;
          // the first tile's first `pre` stages: W already in flight, A only
          const bool early = tile == (int)blockIdx.x && kb / C::KPS < pre;
          if (!early) mbar_arrive_expect_tx(full_bar(stage), (uint32_t)nk * (a_bytes + (uint32_t)C::B_BYTES));
          for (int j = 0; j < nk; ++j) {
            tma_load_2d(sa + j * C::A_BYTES, tail ? &tmAt : &tmA, full_bar(stage), (kb + j) * BK, mt * BM);
            if (!early) tma_load_2d(sb + j * C::B_BYTES, &tmB, full_bar(stage), (kb + j) * BK, nt * BN);
          }
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
        for (int kb = 0; kb < kblocks; kb += C::KPS) {
          if (!mbar_wait(full_bar(stage), phase, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint32_t sb = sa + C::KPS * C::A_BYTES;
          const int nk = min(C::KPS, kblocks - kb);
          for (int j = 0; j < nk; ++j) {
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
              mma_bf16(d_tmem, sw128_desc(sa + j * C::A_BYTES + 32u * k), sw128_desc(sb + j * C::B_BYTES + 32u * k),
                       idesc, ((kb + j) | k) != 0 ? 1u : 0u);
          }
          mma_commit(empty_bar(stage));
          if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
        }
        if (ok) mma_commit(tfull_bar(acc));
      }
    }
    __syncwarp();
  } else {
    // ---- epilogue warps 2..5: TMEM lane quarter q = warp % 4 = tile rows 32q..32q+31
    const int q = warp & 3;
    const bool resid = (ep.flags & CC2_EPI_RESID) != 0;
    const uint32_t box0 = smem_u32(epi_smem + (size_t)q * 2 * kEpiBox);
    uint32_t rphase = 0;  // bit b: parity of the next wait on rbar(q, b)
    uint32_t use = 0;     // running box counter (box = use & 1)
    int it = 0;
    constexpr int G = BN / 64;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++it) {
      const int mt = tile / n_tiles, nt = tile % n_tiles;
      const int row0 = mt * BM + q * 32;
      const int ng = min(G, (N - nt * BN + 63) / 64);
      if (resid && lane == 0) {  // prefetch group 0's residual box (overlaps the MMA wait)
        bulk_wait_read0();
        const int b = use & 1;
        mbar_arrive_expect_tx(rbar(q, b), kEpiBox);
        tma_load_2d(box0 + b * kEpiBox, &tmR, rbar(q, b), nt * BN, row0);
      }
      const int row = row0 + lane;
      const bool row_ok = row < M;
      const int acc = it & 1;
      const uint32_t acc_phase = (uint32_t)(it >> 1) & 1u;
      if (!mbar_wait(tfull_bar(acc), acc_phase, abort_flag)) break;
      tc_fence_after();
      const float rs = row_scale(ep, ep.flags, row, row_ok);
      const bool special = (ep.flags & CC2_EPI_SPECIAL) && row_ok && (row % ep.sp_period) == ep.sp_offset;
      const bool rope_tile = (ep.flags & CC2_EPI_ROPE) && nt * BN < ep.rope_cols;
      uint32_t cs[32];
      if (rope_tile) load_rope_row(ep, row, row_ok, cs);
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
      bool aborted = false;
      for (int g = 0; g < ng; ++g, ++use) {
        const int b = use & 1;
        const uint32_t box = box0 + b * kEpiBox;
        const int col0 = nt * BN + g * 64;
        uint32_t r[64];
        tmem_ld32(tbase + g * 64, r);
        tmem_ld32(tbase + g * 64 + 32, r + 32);
        tmem_ld_wait();
        if (resid) {
          if (!mbar_wait(rbar(q, b), (rphase >> b) & 1u, abort_flag)) { aborted = true; break; }
          rphase ^= 1u << b;
          if (lane == 0 && g + 1 < ng) {  // next group's residual into the other box
            bulk_wait_read0();
            mbar_arrive_expect_tx(rbar(q, b ^ 1), kEpiBox);
            tma_load_2d(box0 + (b ^ 1) * kEpiBox, &tmR, rbar(q, b ^ 1), col0 + 64, row0);
          }
        } else if (lane == 0) {
          bulk_wait_read1();  // the store that last used this box has finished reading it
        }
        __syncwarp();
        float rsg = rs;
        if (rope_tile && col0 < ep.rope_cols) {
          rope_group(r, cs, rs);
          rsg = 1.0f;
        }
        uint4 rl[8];
        if ((ep.flags & CC2_EPI_LO) && resid) load_lo_group(rl, ep, row, row_ok, col0, N);
        const float ssq = epilogue_group(ep, ep.flags, r, rsg, special, col0, N, box, lane, resid, row, row_ok, rl);
        if ((ep.flags & CC2_EPI_SSQ) && row_ok) ep.ssq_out[(size_t)(col0 >> 6) * ep.ssq_ld + row] = ssq;
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmC, box, col0, row0);
          bulk_commit();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar(acc));
      if (aborted) break;
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------
// 2-SM variant: a cluster of two CTAs computes a 256 x 256 output tile with
// tcgen05.mma.cta_group::2 (M = 256, N = 256).  CTA r of the pair loads rows
// [128 r, 128 r + 128) of the A tile and rows [128 r, 128 r + 128) of the W
// tile (half of N) into its own shared memory; the leader (rank 0) issues the
// MMAs, which read both CTAs' halves, and each CTA's TMEM receives its own 128
// rows x 256 columns.  Per SM this moves 32 KB per 128x256x64 step instead of
// 48 KB.  Barriers: the leader's full[s] collects both CTAs' TMA bytes; the
// leader's MMA commits release empty[s] and tmem_full[a] in both CTAs (one
// commit per CTA, addressed through the cluster window); both CTAs' epilogue
// warps release the leader's tmem_empty[a] (count 16).  Eight epilogue warps
// per CTA (two per TMEM lane quarter) split the 64-column groups; each
// prefetches its residual boxes and row scales while the MMAs of the tile run.
// ---------------------------------------------------------------------------------
namespace pair {

// Optional event trace (cc2_set_gemm_trace): CTA 0 records %globaltimer stamps
// of its first kTraceTiles tiles, kTraceEv per tile:
//   0 MMA: accumulator free   1 MMA: first stage loaded   2 MMA: last k-block
//   issued   3 epilogue warp 2: accumulator full   4 epilogue warp 2: done
//   5 producer: first load of the tile issued   6 MMA: ns spent waiting for
//   loaded stages during the tile
constexpr int kTraceTiles = 32, kTraceEv = 8;
__device__ unsigned long long* g_gemm_trace = nullptr;

__device__ __forceinline__ void gtrace(unsigned long long* tr, int tile_it, int ev, unsigned long long v) {
  if (tr != nullptr && tile_it < kTraceTiles) tr[tile_it * kTraceEv + ev] = v;
}

constexpr int A_BYTES = 128 * BK * 2;
constexpr int B_BYTES = 128 * BK * 2;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int BN = 256;
constexpr int TMEM_COLS = 2 * BN;
constexpr int EPI_WARPS = 8;               // two per TMEM lane quarter, each takes half the column groups
constexpr int GPW = 2;                      // 64-column groups per epilogue warp
constexpr int THREADS = 32 * (2 + EPI_WARPS);
// STAGES: depth of the TMA ring; BOXES: epilogue staging boxes per warp (2 =
// one per group, needed for the residual prefetch; 1 = boxes reused, which
// frees shared memory for a deeper ring).
template <int STAGES, int BOXES>
constexpr int smem_bytes() { return STAGES * STAGE_BYTES + EPI_WARPS * BOXES * kEpiBox + 1024 + 256; }

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(saddr), "r"(rank));
  return out;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void arrive_expect_tx_cluster(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cluster.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void arrive_cluster(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"((uint64_t)map), "r"(bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void mma_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive (once) on the mbarrier at cluster address `bar` when all prior
// tcgen05.mma of this thread have completed.
__device__ __forceinline__ void commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ constexpr uint32_t idesc_pair() {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
}

// F >= 0: the epilogue flags, fixed at compile time (only the work a GEMM
// needs is emitted); F = -1: flags read at run time (RoPE not supported).
template <int F, int STAGES, int BOXES, bool SKIP_EPI = false>
__global__ void __launch_bounds__(THREADS, 1)
gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmR, int M, int N,
                 int K, Epi ep) {
  pdl_launch_dependents();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* epi_smem = smem + STAGES * STAGE_BYTES;
  uint64_t* bars = (uint64_t*)(epi_smem + EPI_WARPS * BOXES * kEpiBox);
  // bars: [0,S) full, [S,2S) empty, [2S,2S+2) tmem full, [2S+2,2S+4) tmem empty,
  //       [2S+4, 2S+4+16) residual box loaded (epilogue warp e, box j) at 2S+4+2e+j
  uint32_t* tmem_slot = (uint32_t*)(bars + 2 * STAGES + 4 + EPI_WARPS * BOXES);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  constexpr bool ROPE = F >= 0 && (F & CC2_EPI_ROPE);
  const int flags = F >= 0 ? F : ep.flags;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const uint32_t bar0 = smem_u32(bars);
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + 2 + a); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 2 * EPI_WARPS);
    }
    for (int i = 0; i < EPI_WARPS * BOXES; ++i) mbar_init(bar0 + 8u * (2 * STAGES + 4 + i), 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
    tma_prefetch_desc(&tmR);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  // the producer warp waits below, after it has issued the weight loads it may issue early
  if (warp != 0 || !ep.wpre) pdl_wait();  // activations are read from now on
  const uint32_t tmem_base = *tmem_slot;

  const int m_tiles = (M + 255) / 256;
  const int n_tiles = (N + BN - 1) / BN;
  const int num_tiles = m_tiles * n_tiles;
  const int kblocks = (K + BK - 1) / BK;
  const int pair_id = blockIdx.x >> 1, num_pairs = gridDim.x >> 1;
  unsigned long long* const gtr = blockIdx.x == 0 ? g_gemm_trace : nullptr;

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t lead_full0 = map_to_rank(full_bar(0), 0);
      // constant weights (ep.wpre): this CTA's W half of the first tile's first
      // `pre` (fresh) stages is issued before the grid dependency wait; the
      // leader's full barrier expects both CTAs' A and W bytes as usual
      int pre = 0;
      if (ep.wpre && pair_id < num_tiles) {
        const int nt = pair_id % n_tiles;
        for (int kb = 0; kb < kblocks && pre < STAGES; ++kb, ++pre) {
          const uint32_t fb = lead_full0 + 8u * pre;
          if (leader) arrive_expect_tx_cluster(fb, 2 * STAGE_BYTES);
          tma_load_2d_pair(smem_u32(smem + pre * STAGE_BYTES) + A_BYTES, &tmB, fb, kb * BK, nt * BN + (int)rank * 128);
        }
        pdl_wait();
      }
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int pit = 0;
      for (int tile = pair_id; tile < num_tiles && ok; tile += num_pairs, ++pit) {
        const int mt = tile / n_tiles, nt = tile % n_tiles;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (kb == 1) gtrace(gtr, pit, 5, globaltimer_ns());
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag)) { ok = false; break; }
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t fb = lead_full0 + 8u * stage;
          const bool early = tile == pair_id && kb < pre;  // W already in flight: A only
          if (leader && !early) arrive_expect_tx_cluster(fb, 2 * STAGE_BYTES);
          tma_load_2d_pair(sa, &tmA, fb, kb * BK, mt * 256 + (int)rank * 128);
          if (!early) tma_load_2d_pair(sa + A_BYTES, &tmB, fb, kb * BK, nt * BN + (int)rank * 128);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = idesc_pair();
      const uint32_t peer_empty0 = map_to_rank(empty_bar(0), 1), own_empty0 = map_to_rank(empty_bar(0), 0);
      const uint32_t peer_tfull0 = map_to_rank(tfull_bar(0), 1), own_tfull0 = map_to_rank(tfull_bar(0), 0);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int it = 0;
      for (int tile = pair_id; tile < num_tiles && ok; tile += num_pairs, ++it) {
        const int acc = it & 1;
        const uint32_t acc_phase = (uint32_t)(it >> 1) & 1u;
        if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        if (gtr) gtrace(gtr, it, 0, globaltimer_ns());
        unsigned long long waited = 0;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (gtr && !mbar_try_wait(full_bar(stage), phase)) {
            const unsigned long long w0 = globaltimer_ns();
            if (!mbar_wait(full_bar(stage), phase, abort_flag)) { ok = false; break; }
            waited += globaltimer_ns() - w0;
          } else if (!mbar_wait(full_bar(stage), phase, abort_flag)) { ok = false; break; }
          tc_fence_after();
          if (gtr && kb == 0) gtrace(gtr, it, 1, globaltimer_ns());
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            mma_pair(d_tmem, sw128_desc(sa + 32u * k), sw128_desc(sb + 32u * k), idesc, (kb | k) != 0 ? 1u : 0u);
          commit_pair(own_empty0 + 8u * stage);
          commit_pair(peer_empty0 + 8u * stage);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (gtr) {
          gtrace(gtr, it, 2, globaltimer_ns());
          gtrace(gtr, it, 6, waited);
        }
        if (ok) {
          commit_pair(own_tfull0 + 8u * acc);
          commit_pair(peer_tfull0 + 8u * acc);
        }
      }
    }
    __syncwarp();
  } else {
    // ---- epilogue warps 2..9: TMEM lane quarter q = warp % 4 (rows 32q..32q+31 of
    // this CTA's half); warps 2..5 take column groups 0-1, warps 6..9 groups 2-3.
    const int ew = warp - 2;
    const int q = warp & 3;
    const int g0 = (ew >> 2) * GPW;
    const bool resid = (flags & CC2_EPI_RESID) != 0;
    const uint32_t box0 = smem_u32(epi_smem + (size_t)ew * BOXES * kEpiBox);
    const uint32_t lead_tempty0 = map_to_rank(tempty_bar(0), 0);
    auto rbar = [&](int j) { return bar0 + 8u * (2 * STAGES + 4 + BOXES * ew + j); };
    int it = 0;
    for (int tile = pair_id; tile < num_tiles; tile += num_pairs, ++it) {
      const int mt = tile / n_tiles, nt = tile % n_tiles;
      const int row0 = mt * 256 + (int)rank * 128 + q * 32;
      const int ng = min(GPW, max(0, (N - nt * BN + 63) / 64 - g0));  // groups of this warp inside N
      if (lane == 0) {
        bulk_wait_read0();  // the previous tile's stores have left the boxes
        if (resid) {        // prefetch this warp's residual boxes while the MMAs run
          for (int j = 0; j < ng; ++j) {
            mbar_arrive_expect_tx(rbar(j), kEpiBox);
            tma_load_2d(box0 + j * kEpiBox, &tmR, rbar(j), nt * BN + (g0 + j) * 64, row0);
          }
        }
      }
      __syncwarp();
      // per-row terms that do not depend on the accumulator, also before the wait
      const int row = row0 + lane;
      const bool row_ok = row < M;
      const float rs = row_scale(ep, flags, row, row_ok);
      const bool special = (flags & CC2_EPI_SPECIAL) && row_ok && (row % ep.sp_period) == ep.sp_offset;
      const bool rope_tile = ROPE && nt * BN + g0 * 64 < ep.rope_cols;
      uint32_t cs[ROPE ? 32 : 1];
      if constexpr (ROPE) {
        if (rope_tile) load_rope_row(ep, row, row_ok, cs);
      }
      constexpr bool LOR = F >= 0 && (F & CC2_EPI_LO) && (F & CC2_EPI_RESID);
      uint4 rl[8];
      if constexpr (LOR) {  // group 0's residual low halves, in flight during the accumulator wait
        if (ng > 0) load_lo_group(rl, ep, row, row_ok, nt * BN + g0 * 64, N);
      } else if (F < 0 && (flags & CC2_EPI_LO) && resid && ng > 0) {
        load_lo_group(rl, ep, row, row_ok, nt * BN + g0 * 64, N);
      }
      const int acc = it & 1;
      const uint32_t acc_phase = (uint32_t)(it >> 1) & 1u;
      if (!mbar_wait(tfull_bar(acc), acc_phase, abort_flag)) break;
      tc_fence_after();
      const bool tw = gtr != nullptr && warp == 2 && lane == 0;
      if (tw) gtrace(gtr, it, 3, globaltimer_ns());
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
      bool aborted = false;
      for (int j = 0; j < (SKIP_EPI ? 0 : ng); ++j) {
        const uint32_t box = box0 + (j % BOXES) * kEpiBox;
        const int col0 = nt * BN + (g0 + j) * 64;
        if (j >= BOXES) {  // reusing a box: its previous store must have read it
          if (lane == 0) bulk_wait_read0();
          __syncwarp();
        }
        uint32_t r[64];
        tmem_ld32(tbase + (g0 + j) * 64, r);
        tmem_ld32(tbase + (g0 + j) * 64 + 32, r + 32);
        tmem_ld_wait();
        if (resid && !mbar_wait(rbar(j), (uint32_t)it & 1u, abort_flag)) { aborted = true; break; }
        float rsg = rs;
        if constexpr (ROPE) {
          if (rope_tile && col0 < ep.rope_cols) {
            rope_group(r, cs, rs);
            rsg = 1.0f;
          }
        }
        const float ssq = epilogue_group(ep, flags, r, rsg, special, col0, N, box, lane, resid, row, row_ok, rl);
        if ((flags & CC2_EPI_LO) && resid && j + 1 < ng) load_lo_group(rl, ep, row, row_ok, col0 + 64, N);  // next group's
        if ((flags & CC2_EPI_SSQ) && row_ok) ep.ssq_out[(size_t)(col0 >> 6) * ep.ssq_ld + row] = ssq;
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmC, box, col0, row0);
          bulk_commit();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) arrive_cluster(lead_tempty0 + 8u * acc);
      if (tw) gtrace(gtr, it, 4, globaltimer_ns());
      if (aborted) break;
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its peer may still signal or read it
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                 : "memory");
  }
}

}  // namespace pair

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
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)p;
  });
  return fn;
}

// 2-D bf16 tensor map over a row-major [rows, cols] matrix with row pitch ld
// (elements); box = box_cols x box_rows, 128-byte swizzle, zero fill outside
// the matrix (loads) / clipping (stores).
static int make_map_box(CUtensorMap* map, const void* ptr, int cols, int rows, int ld, int box_cols, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  CC2_REQUIRE(fn != nullptr, "cuTensorMapEncodeTiled unavailable");
  CC2_REQUIRE(((uintptr_t)ptr & 15u) == 0, "gemm operand not 16-byte aligned");
  CC2_REQUIRE((ld * 2) % 16 == 0, "gemm row pitch must be a multiple of 8 elements");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d): cols=%d rows=%d ld=%d", (int)r, cols, rows, ld);
    return CC2_E_CUDA;
  }
  return CC2_OK;
}
static int make_map(CUtensorMap* map, const void* ptr, int cols, int rows, int ld, int box_rows) {
  return make_map_box(map, ptr, cols, rows, ld, BK, box_rows);
}

template <int BN, int AR = BM, int KPS = 2>
static int launch(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const CUtensorMap& mr, int M,
                  int N, int K, const Epi& ep, cudaStream_t st, const void* A, int lda) {
  using C = Cfg2<BN, AR, KPS>;
  static_assert(AR == BM || AR == 64, "A slot rows");
  // 64-row A slots hold only the tail box: one row tile of at most 64 rows
  CC2_REQUIRE(AR == BM || M <= AR, "gemm: %d rows do not fit the %d-row A slots", M, AR);
  // rows of the last row tile, rounded up to whole 8-row swizzle atoms
  const int rem = M % BM;
  const int tail_rows = rem == 0 ? BM : (rem + 7) / 8 * 8;
  CUtensorMap mat = ma;
  if (tail_rows < BM) CC2_TRY(make_map(&mat, A, K, M, lda, tail_rows));
  static unsigned long long attr_set = 0;  // one bit per device
  int dev = 0;
  CC2_CUDA(cudaGetDevice(&dev));
  if (dev >= 64 || !((attr_set >> dev) & 1ull)) {
    CC2_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<BN, AR, KPS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  C::SMEM));
    if (dev < 64) attr_set |= 1ull << dev;
  }
  const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int grid = tiles < num_sms() ? tiles : num_sms();
  CC2_CUDA(launch_k(gemm_tc_kernel<BN, AR, KPS>, grid, kThreads, C::SMEM, st, ma, mb, mc, mr, mat, tail_rows, M, N,
                    K, ep));
  CC2_CHECK_LAUNCH();
  return CC2_OK;
}

template <int F, int STAGES, int BOXES, bool SKIP_EPI = false>
static int launch_pair_t(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const CUtensorMap& mr,
                         int M, int N, int K, const Epi& ep, cudaStream_t st) {
  constexpr int SMEM = pair::smem_bytes<STAGES, BOXES>();
  static unsigned long long attr_set = 0;  // one bit per device
  int dev = 0;
  CC2_CUDA(cudaGetDevice(&dev));
  if (dev >= 64 || !((attr_set >> dev) & 1ull)) {
    CC2_CUDA(cudaFuncSetAttribute(pair::gemm_pair_kernel<F, STAGES, BOXES, SKIP_EPI>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
    if (dev < 64) attr_set |= 1ull << dev;
  }
  const int tiles = ((M + 255) / 256) * ((N + pair::BN - 1) / pair::BN);
  const int pairs = std::min(tiles, num_sms() / 2);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(pair::THREADS, 1, 1);
  cfg.dynamicSmemBytes = SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = launch_overlap() ? 2 : 1;
  CC2_CUDA(cudaLaunchKernelEx(&cfg, pair::gemm_pair_kernel<F, STAGES, BOXES, SKIP_EPI>, ma, mb, mc, mr, M, N, K,
                              ep));
  return CC2_OK;
}

static int launch_pair(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const CUtensorMap& mr,
                       int M, int N, int K, const Epi& ep, cudaStream_t st, int variant) {
  constexpr int RS = CC2_EPI_ROWSCALE, BI = CC2_EPI_BIAS, RL = CC2_EPI_RELU, RE = CC2_EPI_RESID,
                SQ = CC2_EPI_SSQ, SP = CC2_EPI_SPECIAL, RP = CC2_EPI_ROPE, LO = CC2_EPI_LO;
  if (variant == 3)  // measurement only: mainloop with the epilogue reduced to releasing TMEM (no output)
    return launch_pair_t<0, 5, 2, true>(ma, mb, mc, mr, M, N, K, ep, st);
#define CC2_PAIR(FL) \
  case (FL): return launch_pair_t<(FL), 5, 2>(ma, mb, mc, mr, M, N, K, ep, st);
  // an epilogue without a residual needs one staging box per warp, which
  // leaves room for a sixth ring stage (more loads in flight per SM): FFN up
  // 141-142 -> 139-140 us at configs[1]; QKV measured no better (114 -> 116).
  // Residual epilogues keep their boxes: reading the residual into registers
  // instead, to free the room, doubled the O-projection's time (61 -> 123 us).
#define CC2_PAIR6(FL) \
  case (FL): return launch_pair_t<(FL), 6, 1>(ma, mb, mc, mr, M, N, K, ep, st);
  switch (ep.flags) {  // the epilogues the forward uses, specialised at compile time
    CC2_PAIR(RS | RP)            // time-attention QKV (RMSNorm + RoPE)
    CC2_PAIR(RP)                 // RoPE alone (component use)
    CC2_PAIR(RS)                 // group QKV
    CC2_PAIR6(RS | RL)           // FFN up
    CC2_PAIR(RE | SQ)            // O-projections, FFN down (component use)
    CC2_PAIR(RE | SQ | LO)       // O-projections, FFN down (hi + lo residual stream)
    CC2_PAIR(RS | RE | SQ)       // one-series group block (component use)
    CC2_PAIR(RS | RE | SQ | LO)  // one-series group block (hi + lo residual stream)
    CC2_PAIR(BI | SQ | SP | LO)  // input ResidualBlock output (+REG row, hi + lo)
    CC2_PAIR(BI | RL)            // ResidualBlock hidden
    CC2_PAIR(BI | SQ | SP)       // input ResidualBlock output (+REG row)
    CC2_PAIR(BI)                 // output ResidualBlock output
    CC2_PAIR(0)                  // plain
    default:
      break;
  }
#undef CC2_PAIR
#undef CC2_PAIR6
  if (ep.flags & RP) {
    set_error("gemm: CC2_EPI_ROPE combines with CC2_EPI_ROWSCALE only");
    return CC2_E_UNSUPPORTED;
  }
  return launch_pair_t<-1, 5, 2>(ma, mb, mc, mr, M, N, K, ep, st);
}

// ---------------------------------------------------------------------------------
// Layer-persistent forward for few token rows (batch-1 serving).
//
// With a few hundred token rows every GEMM of an encoder layer is a handful of
// 128 x 64 tiles and the time attention a dozen (head, set) items; launched
// one kernel each, the forward is a chain of ~72 launches whose fixed costs
// (launch, prologue, first load, drain) exceed the work.  Here one
// cooperative launch of one CTA per SM runs the whole list of stages (QKV
// GEMM, time attention, O-projection, group block, FFN up, FFN down, per
// layer), with a grid-wide barrier between stages.  TMEM, the mbarriers and
// the shared-memory ring are set up once; the producer / MMA / epilogue roles
// keep their ring and accumulator phases across stages.
//
// Each GEMM stage is the 1-SM 128 x 64 tile GEMM above (same MMAs, same
// epilogue functions); stages with a long k-loop and few tiles split it over
// 2 or 4 CTAs whose fp32 partials are summed in split order.  The time
// attention gives each CTA one 16-row query tile and splits the keys over
// its warps (softmax states merged in warp order).  In exact mode (no split,
// attention by aset::set_tile, the body of the whole-set attention kernel)
// the results equal those of the per-kernel forward with gemm_tc_kernel<64>
// and attention variant 3, bit for bit.
//
// Measured at batch 1 (133 token rows) a stage costs ~10 us (K = 768) - the
// first load ~0.7 us, the k-loop at one SM's TMA rate (~0.3 us per 24 KB
// k-block), the epilogue ~2.3 us (one warp per 64 columns), the grid barrier
// ~1.5 us - so the launch is about as fast as the per-kernel forward, whose
// programmatic launches already overlapped the same latencies; it is off by
// default (cc2_set_layer_chain).
//
// Coherence inside the kernel: activations written by one stage are read by
// other SMs in the next, so loads that could hit a stale L1 line go through
// L2 (ld.global.cg / cp.async.cg / TMA), and every thread fences its generic
// and async proxies around the grid barrier.  The barrier (arrival counter,
// generation, abort word in caller-zeroed global memory) waits with the same
// wall-clock bound as the mbarrier waits; on expiry it raises
// DEV_ERR_LAYER_TIMEOUT and the abort word, every CTA leaves its stage loop,
// frees its TMEM and returns.
// ---------------------------------------------------------------------------------
namespace chain {

constexpr int BN = 64;
using C = Cfg<BN>;
constexpr int kMaxMaps = 72;
constexpr int kMaxStages = 76;
constexpr int kWarps = kThreads / 32;
constexpr int SMEM = C::SMEM + 512;  // + the current stage's descriptor

struct Stage {
  Epi ep;
  int kind;  // 0: GEMM, 1: time attention
  int N, K;
  int a, b, c, r;  // tensor-map indices (GEMM)
  const void* w;    // GEMM: the weight matrix (contiguous, prefetched into L2 one stage ahead)
  unsigned long long wbytes;
  int split;        // GEMM: k-ranges per tile (1, 2 or 4)
  int cnt_off;      // GEMM with split > 1: this stage's partial counters (tiles x 4) in cnt
  const bf16* qkv;  // attention: [sets * S, ld] rows with Q, K, V column blocks
  bf16* out;
  const uint8_t* tok;
  int ld, ldo, qcol, kcol, vcol, sets, S, heads;
};

struct Params {
  CUtensorMap maps[kMaxMaps];
  Stage st[kMaxStages];
  int nstages, M;
  int exact;          // 1: no split-K, attention as aset::set_tile (the per-kernel forward's arithmetic)
  unsigned int* bar;  // [0] arrivals (monotonic), [2] abort (zeroed before the launch)
  unsigned int* cnt;  // split-K partial counters (zeroed before the launch)
  float* part;        // split-K partials: [unit][4][16][32] float4 (grid x 32 KB)
};
static_assert(sizeof(Params) <= 32000, "kernel parameter block too large");
static_assert(sizeof(Stage) <= 448, "stage descriptor must fit its shared-memory slot");

__device__ __forceinline__ void fence_proxy_async_all() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Optional stage trace (cc2_set_layer_trace): CTAs < kTraceCtas record, per
// stage, the %globaltimer when all their roles finished the stage and when
// the grid barrier released them.
constexpr int kTraceCtas = 8;
__device__ unsigned long long* g_chain_trace = nullptr;

// Copies a stage descriptor from the parameter block into shared memory (all
// threads but 0 take part): the roles then read their arguments from shared
// memory instead of through the constant cache, which a 26 KB parameter block
// overflows.
__device__ __forceinline__ void copy_stage(Stage* dst, const Stage* src) {
  const uint32_t* a = reinterpret_cast<const uint32_t*>(src);
  uint32_t* b = reinterpret_cast<uint32_t*>(dst);
  for (int i = (int)threadIdx.x - 1; i >= 0 && i < (int)(sizeof(Stage) / 4); i += blockDim.x - 1) b[i] = a[i];
}

// Grid-wide barrier (all threads of every CTA call it).  False: abort.
// next: the following stage, copied into sst while thread 0 waits.
__device__ __noinline__ bool grid_sync(unsigned* bar, volatile int* abort_flag, int si, const Stage* next,
                                       Stage* sst) {
  fence_proxy_async_all();
  __syncthreads();  // then thread 0's fence makes the CTA's writes visible before its arrival
  copy_stage(sst, next);
  unsigned long long* tr = g_chain_trace;
  if (tr && threadIdx.x == 0 && blockIdx.x < kTraceCtas)
    tr[((size_t)blockIdx.x * kMaxStages + si) * 2] = globaltimer_ns();
  if (threadIdx.x == 0) {
    bool ok = *abort_flag == 0;
    if (ok && blockIdx.x == 0 && *(volatile int*)&g_chain_starve && atomicExch(&g_chain_starve, 0)) {
      *abort_flag = 1;  // test hook: this CTA never arrives, so the others' bounded waits run out
    } else if (ok) {
      // barrier k (after stage k) completes when (k + 1) x gridDim arrivals are counted
      const unsigned target = (unsigned)(si + 1) * gridDim.x;
      __threadfence();
      if (atomicAdd(bar, 1u) + 1u < target) {
        const unsigned long long t0 = globaltimer_ns();
        for (uint32_t n = 1;; ++n) {
          if (ld_acquire(bar) >= target) break;
          if ((n & 15u) == 0) {
            if (*(volatile unsigned*)(bar + 2)) { ok = false; break; }
            if (globaltimer_ns() - t0 > kWaitLimitNs) {
              atomicOr(&g_dev_error, DEV_ERR_LAYER_TIMEOUT);
              ok = false;
              break;
            }
          }
        }
      }
    }
    if (!ok) {
      atomicExch(bar + 2, 1u);
      *abort_flag = 1;
    }
    __threadfence();
    if (tr && blockIdx.x < kTraceCtas) tr[((size_t)blockIdx.x * kMaxStages + si) * 2 + 1] = globaltimer_ns();
  }
  __syncthreads();
  fence_proxy_async_all();
  return *abort_flag == 0;
}

__global__ void __launch_bounds__(kThreads, 1) chain_kernel(const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* epi_smem = smem + C::STAGES * C::STAGE_BYTES;
  uint64_t* bars = (uint64_t*)(epi_smem + 8 * kEpiBox);
  uint32_t* tmem_slot = (uint32_t*)(bars + 2 * C::STAGES + 12);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  Stage* sst = (Stage*)(((uintptr_t)(tmem_slot + 2) + 15) & ~(uintptr_t)15);  // the current stage

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t bar0 = smem_u32(bars);
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (C::STAGES + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * C::STAGES + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * C::STAGES + 2 + a); };
  auto rbar = [&](int q, int b) { return bar0 + 8u * (2 * C::STAGES + 4 + 2 * q + b); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 4);
    }
    for (int i = 0; i < 8; ++i) mbar_init(bar0 + 8u * (2 * C::STAGES + 4 + i), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  copy_stage(sst, &p.st[0]);
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int M = p.M;
  const int m_tiles = (M + BM - 1) / BM;

  // role state carried across stages
  int pstage = 0; uint32_t pphase = 0;             // producer ring position
  int mstage = 0; uint32_t mphase = 0; int mit = 0;  // MMA ring position, tiles issued
  int eit = 0; uint32_t use = 0, rphase = 0;        // epilogue tiles, residual boxes

  for (int si = 0; si < p.nstages; ++si) {
    const Stage& s = *sst;
    if (warp == 1 && lane == 1 && si + 1 < p.nstages && p.st[si + 1].kind == 0) {
      // the next GEMM's weights into L2 (each CTA a slice) and its tensor maps
      // into the descriptor cache, while this stage runs
      const Stage& nx = p.st[si + 1];
      const unsigned long long slice = ((nx.wbytes + gridDim.x - 1) / gridDim.x + 255) & ~255ull;
      const unsigned long long lo = slice * blockIdx.x;
      const unsigned long long hi = lo + slice < nx.wbytes ? lo + slice : nx.wbytes;
      for (unsigned long long o = lo; o < hi; o += 16384) {
        const unsigned n = (unsigned)(hi - o < 16384 ? hi - o : 16384);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"((const char*)nx.w + o), "r"(n) : "memory");
      }
      tma_prefetch_desc(&p.maps[nx.a]);
      tma_prefetch_desc(&p.maps[nx.b]);
      tma_prefetch_desc(&p.maps[nx.c]);
      tma_prefetch_desc(&p.maps[nx.r]);
    }
    if (s.kind == 0) {
      // Work units: tile x split.  With split S > 1 the tile's k-blocks are
      // divided into S ranges on S CTAs; each unit's epilogue warp q either
      // writes its fp32 partial of rows 32q..32q+31 to the scratch and counts
      // it (q % S != split), or (q % S == split) waits for the other S - 1
      // partials of those rows, sums all S in split order and runs the
      // epilogue.  Units never exceed the grid, so all of a tile's units are
      // resident at once.
      unsigned long long* ktr = nullptr;
      if (g_chain_trace && blockIdx.x == 0 && (si == 2 || si == 4))
        ktr = g_chain_trace + (size_t)kTraceCtas * kMaxStages * 2 + (si == 4 ? 160 : 0);
      if (ktr && threadIdx.x == 0) ktr[131] = globaltimer_ns();
      const int N = s.N;
      const int n_tiles = (N + BN - 1) / BN;
      const int S = s.split;
      const int num_units = m_tiles * n_tiles * S;
      const int kblocks = (s.K + BK - 1) / BK;
      const int kpb = (kblocks + S - 1) / S;  // k-blocks per split
      const CUtensorMap* tmA = &p.maps[s.a];
      const CUtensorMap* tmB = &p.maps[s.b];
      const CUtensorMap* tmC = &p.maps[s.c];
      const CUtensorMap* tmR = &p.maps[s.r];
      if (warp == 0) {
        if (lane == 0) {
          bool ok = true;
          for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
            const int tile = u / S, sp = u % S;
            const int mt = tile / n_tiles, nt = tile % n_tiles;
            const int kb1 = min(kblocks, (sp + 1) * kpb);
            for (int kb = sp * kpb; kb < kb1; ++kb) {
              if (!mbar_wait(empty_bar(pstage), pphase ^ 1u, abort_flag)) { ok = false; break; }
              if (ktr && u == (int)blockIdx.x && kb < 64) ktr[kb] = globaltimer_ns();
              const uint32_t sa = smem_u32(smem + pstage * C::STAGE_BYTES);
              mbar_arrive_expect_tx(full_bar(pstage), C::STAGE_BYTES);
              tma_load_2d(sa, tmA, full_bar(pstage), kb * BK, mt * BM);
              tma_load_2d(sa + C::A_BYTES, tmB, full_bar(pstage), kb * BK, nt * BN);
              if (++pstage == C::STAGES) { pstage = 0; pphase ^= 1u; }
            }
          }
        }
        __syncwarp();
      } else if (warp == 1) {
        if (lane == 0) {
          constexpr uint32_t idesc = idesc_bf16<BN>();
          bool ok = true;
          for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x, ++mit) {
            const int sp = u % S;
            const int kb0 = sp * kpb, kb1 = min(kblocks, (sp + 1) * kpb);
            const int acc = mit & 1;
            const uint32_t acc_phase = (uint32_t)(mit >> 1) & 1u;
            if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1u, abort_flag)) break;
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
            for (int kb = kb0; kb < kb1; ++kb) {
              if (!mbar_wait(full_bar(mstage), mphase, abort_flag)) { ok = false; break; }
              if (ktr && u == (int)blockIdx.x && kb < 64) ktr[64 + kb] = globaltimer_ns();
              tc_fence_after();
              const uint32_t sa = smem_u32(smem + mstage * C::STAGE_BYTES);
              const uint32_t sb = sa + C::A_BYTES;
#pragma unroll
              for (int k = 0; k < BK / 16; ++k)
                mma_bf16(d_tmem, sw128_desc(sa + 32u * k), sw128_desc(sb + 32u * k), idesc,
                         (kb != kb0 || k != 0) ? 1u : 0u);
              mma_commit(empty_bar(mstage));
              if (++mstage == C::STAGES) { mstage = 0; mphase ^= 1u; }
            }
            if (ok) mma_commit(tfull_bar(acc));
          }
        }
        __syncwarp();
      } else {
        // epilogue warps 2..5: TMEM lane quarter q = tile rows 32q..32q+31
        const Epi& ep = s.ep;
        const int q = warp & 3;
        const bool resid = (ep.flags & CC2_EPI_RESID) != 0;
        const uint32_t box0 = smem_u32(epi_smem + (size_t)q * 2 * kEpiBox);
        bool aborted = false;
        for (int u = blockIdx.x; u < num_units && !aborted; u += gridDim.x, ++eit) {
          const int tile = u / S, sp = u % S;
          const int mt = tile / n_tiles, nt = tile % n_tiles;
          const int row0 = mt * BM + q * 32;
          const int col0 = nt * BN;
          const bool mine = (q % S) == sp;  // this warp finishes rows 32q.. of the tile
          const int b = use & 1;
          const uint32_t box = box0 + b * kEpiBox;
          const int row = row0 + lane;
          const bool row_ok = row < M;
          float rs = 1.0f;
          bool special = false, rope_tile = false;
          uint32_t cs[32];
          uint4 rl[8];
          if (mine) {
            if (ktr && q == 2 && lane == 0 && u == (int)blockIdx.x) ktr[135] = globaltimer_ns();
            if (lane == 0) {
              bulk_wait_read0();  // the store that last used this box has read it
              if (resid) {
                mbar_arrive_expect_tx(rbar(q, b), kEpiBox);
                tma_load_2d(box, tmR, rbar(q, b), col0, row0);
              }
            }
            __syncwarp();
            rs = row_scale<true>(ep, ep.flags, row, row_ok);
            special = (ep.flags & CC2_EPI_SPECIAL) && row_ok && (row % ep.sp_period) == ep.sp_offset;
            rope_tile = (ep.flags & CC2_EPI_ROPE) && col0 < ep.rope_cols;
            if (rope_tile) load_rope_row(ep, row, row_ok, cs);
            if ((ep.flags & CC2_EPI_LO) && resid) load_lo_group<true>(rl, ep, row, row_ok, col0, N);
          }
          const int acc = eit & 1;
          const uint32_t acc_phase = (uint32_t)(eit >> 1) & 1u;
          if (!mbar_wait(tfull_bar(acc), acc_phase, abort_flag)) break;
          if (ktr && q == 2 && lane == 0 && u == (int)blockIdx.x) ktr[128] = globaltimer_ns();
          tc_fence_after();
          const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
          uint32_t r[64];
          tmem_ld32(tbase, r);
          tmem_ld32(tbase + 32, r + 32);
          tmem_ld_wait();
          if (ktr && q == 2 && lane == 0 && u == (int)blockIdx.x) ktr[132] = globaltimer_ns();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(tempty_bar(acc));  // accumulator is in registers
          if (S > 1) {
            // partial of rows 32q..32q+31: [unit][q][16 float4 columns][32 rows] (coalesced)
            unsigned* cnt = p.cnt + s.cnt_off + tile * 4 + q;
            if (!mine) {
              float4* dst = reinterpret_cast<float4*>(p.part) + ((size_t)u * 4 + q) * 16 * 32 + lane;
#pragma unroll
              for (int c4 = 0; c4 < 16; ++c4)
                __stcg(dst + c4 * 32, make_float4(__uint_as_float(r[4 * c4]), __uint_as_float(r[4 * c4 + 1]),
                                                  __uint_as_float(r[4 * c4 + 2]), __uint_as_float(r[4 * c4 + 3])));
              __syncwarp();
              if (lane == 0) {
                __threadfence();
                atomicAdd(cnt, 1u);
              }
              __syncwarp();
              continue;
            }
            // wait for the other S - 1 partials of these rows, then sum all S in split order
            if (lane == 0) {
              const unsigned long long t0 = globaltimer_ns();
              for (uint32_t n = 1;; ++n) {
                if (ld_acquire(cnt) >= (unsigned)(S - 1)) break;
                if ((n & 15u) == 0) {
                  if (*abort_flag || *(volatile unsigned*)(p.bar + 2)) { *abort_flag = 1; break; }
                  if (globaltimer_ns() - t0 > kWaitLimitNs) {
                    atomicOr(&g_dev_error, DEV_ERR_LAYER_TIMEOUT);
                    atomicExch(p.bar + 2, 1u);
                    *abort_flag = 1;
                    break;
                  }
                }
              }
            }
            __syncwarp();
            if (*abort_flag) { aborted = true; break; }
            float sum[64];
#pragma unroll
            for (int j = 0; j < 64; ++j) sum[j] = 0.0f;
            for (int o = 0; o < S; ++o) {
              if (o == sp) {
#pragma unroll
                for (int j = 0; j < 64; ++j) sum[j] = __fadd_rn(sum[j], __uint_as_float(r[j]));
              } else {
                const float4* src = reinterpret_cast<const float4*>(p.part) + ((size_t)(tile * S + o) * 4 + q) * 16 * 32 + lane;
#pragma unroll
                for (int c4 = 0; c4 < 16; ++c4) {
                  const float4 v = __ldcg(src + c4 * 32);
                  sum[4 * c4] = __fadd_rn(sum[4 * c4], v.x);
                  sum[4 * c4 + 1] = __fadd_rn(sum[4 * c4 + 1], v.y);
                  sum[4 * c4 + 2] = __fadd_rn(sum[4 * c4 + 2], v.z);
                  sum[4 * c4 + 3] = __fadd_rn(sum[4 * c4 + 3], v.w);
                }
              }
            }
#pragma unroll
            for (int j = 0; j < 64; ++j) r[j] = __float_as_uint(sum[j]);
          }
          if (resid) {
            if (!mbar_wait(rbar(q, b), (rphase >> b) & 1u, abort_flag)) break;
            rphase ^= 1u << b;
          }
          if (ktr && q == 2 && lane == 0 && u == (int)blockIdx.x) ktr[133] = globaltimer_ns();
          float rsg = rs;
          if (rope_tile) {
            rope_group(r, cs, rs);
            rsg = 1.0f;
          }
          const float ssq = epilogue_group(ep, ep.flags, r, rsg, special, col0, N, box, lane, resid, row, row_ok, rl);
          if ((ep.flags & CC2_EPI_SSQ) && row_ok) ep.ssq_out[(size_t)(col0 >> 6) * ep.ssq_ld + row] = ssq;
          if (ktr && q == 2 && lane == 0 && u == (int)blockIdx.x) ktr[134] = globaltimer_ns();
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(tmC, box, col0, row0);
            bulk_commit();
          }
          ++use;
          if (ktr && q == 2 && lane == 0 && u == (int)blockIdx.x) ktr[129] = globaltimer_ns();
        }
        if (lane == 0) bulk_wait_all();  // this stage's outputs are in global memory
        if (ktr && q == 2 && lane == 0) ktr[130] = globaltimer_ns();
        __syncwarp();
      }
    } else if (!p.exact) {
      // time attention: items (set, head, 16-row query tile); the CTA's warps
      // split the keys (chunks of kc, a multiple of 32) and their partial
      // softmax states are merged in a fixed order
      const int n = s.S;
      const int npad = (n + 15) & ~15;
      const int nqt = npad / 16;
      const int kc = (((n + kWarps - 1) / kWarps) + 31) & ~31;
      const int nkc = (n + kc - 1) / kc;
      const int items = s.sets * s.heads * nqt;
      const uint32_t qb = smem_u32(smem);
      const uint32_t kb = qb + 16u * 128u;
      const uint32_t vb = kb + (uint32_t)npad * 128u;
      float* kbias = reinterpret_cast<float*>(smem + 2048 + (size_t)npad * 256);
      float* mo = kbias + npad;                    // [kWarps][16][64] unnormalised outputs
      float2* mm = reinterpret_cast<float2*>(mo + kWarps * 16 * 64);  // [kWarps][16] (max, sum)
      for (int item = blockIdx.x; item < items; item += gridDim.x) {
        const int set = item / (s.heads * nqt);
        const int h = (item / nqt) % s.heads;
        const int qt = item % nqt;
        const size_t row0 = (size_t)set * n;
        for (int idx = threadIdx.x; idx < npad * 8; idx += blockDim.x) {
          const int rr = idx >> 3, c = idx & 7;
          const int qr = rr - qt * 16;  // row of the Q tile, if any
          if (rr < n) {
            const bf16* src = s.qkv + (row0 + rr) * s.ld + c * 8;
            if (qr >= 0 && qr < 16) aset::cp_async16(aset::swz(qb, qr, c), src + s.qcol + h * 64);
            aset::cp_async16(aset::swz(kb, rr, c), src + s.kcol + h * 64);
            aset::cp_async16(aset::swz(vb, rr, c), src + s.vcol + h * 64);
          } else {
            const uint4 z = make_uint4(0, 0, 0, 0);
            if (qr >= 0 && qr < 16) *reinterpret_cast<uint4*>(smem + (aset::swz(qb, qr, c) - qb)) = z;
            *reinterpret_cast<uint4*>(smem + (aset::swz(kb, rr, c) - qb)) = z;
            *reinterpret_cast<uint4*>(smem + (aset::swz(vb, rr, c) - qb)) = z;
          }
        }
        for (int rr = threadIdx.x; rr < npad; rr += blockDim.x)
          kbias[rr] = rr < n ? (s.tok[row0 + rr] ? 0.0f : aset::kMaskedScore) : -INFINITY;
        aset::cp_async_wait_all();
        __syncthreads();
        if (warp < nkc) {
          float o[8][4];
          float m0, m1, l0, l1;
          const int k_lo = warp * kc;
          aset::tile_range<32>(qb, kb, vb, kbias, k_lo, min(n, k_lo + kc), 0, lane, o, m0, m1, l0, l1);
          l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
          l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
          l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
          l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
          const int r0 = lane >> 2;
          float* mw = mo + warp * 16 * 64;
#pragma unroll
          for (int dt = 0; dt < 8; ++dt) {
            const int c = dt * 8 + 2 * (lane & 3);
            *reinterpret_cast<float2*>(mw + r0 * 64 + c) = make_float2(o[dt][0], o[dt][1]);
            *reinterpret_cast<float2*>(mw + (r0 + 8) * 64 + c) = make_float2(o[dt][2], o[dt][3]);
          }
          if ((lane & 3) == 0) {
            mm[warp * 16 + r0] = make_float2(m0, l0);
            mm[warp * 16 + r0 + 8] = make_float2(m1, l1);
          }
        }
        __syncthreads();
        if (threadIdx.x < 128) {
          const int row = threadIdx.x >> 3, c = threadIdx.x & 7;
          float mx = -INFINITY;
          for (int w = 0; w < nkc; ++w) mx = fmaxf(mx, mm[w * 16 + row].x);
          float l = 0.0f, acc[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
          for (int w = 0; w < nkc; ++w) {
            const float2 ml = mm[w * 16 + row];
            const float f = exp2f(ml.x - mx);
            l = __fmaf_rn(ml.y, f, l);
            const float4 a = *reinterpret_cast<const float4*>(mo + (w * 16 + row) * 64 + c * 8);
            const float4 b = *reinterpret_cast<const float4*>(mo + (w * 16 + row) * 64 + c * 8 + 4);
            acc[0] = __fmaf_rn(a.x, f, acc[0]); acc[1] = __fmaf_rn(a.y, f, acc[1]);
            acc[2] = __fmaf_rn(a.z, f, acc[2]); acc[3] = __fmaf_rn(a.w, f, acc[3]);
            acc[4] = __fmaf_rn(b.x, f, acc[4]); acc[5] = __fmaf_rn(b.y, f, acc[5]);
            acc[6] = __fmaf_rn(b.z, f, acc[6]); acc[7] = __fmaf_rn(b.w, f, acc[7]);
          }
          const float il = 1.0f / l;
          const int qrow = qt * 16 + row;
          if (qrow < n) {
            uint4 v;
            v.x = pack_bf16(acc[0] * il, acc[1] * il); v.y = pack_bf16(acc[2] * il, acc[3] * il);
            v.z = pack_bf16(acc[4] * il, acc[5] * il); v.w = pack_bf16(acc[6] * il, acc[7] * il);
            *reinterpret_cast<uint4*>(s.out + (row0 + qrow) * s.ldo + h * 64 + c * 8) = v;
          }
        }
        __syncthreads();
      }
    } else {
      // time attention: items (set, head, chunk of up to kWarps query tiles);
      // Q / K / V of the item's set and head staged in the ring's memory
      const int n = s.S;
      const int npad = (n + 15) & ~15;
      const int nqt = npad / 16;
      const int chunks = (nqt + kWarps - 1) / kWarps;
      const int items = s.sets * s.heads * chunks;
      const uint32_t qb = smem_u32(smem);
      const uint32_t kb = qb + (uint32_t)npad * 128u;
      const uint32_t vb = kb + (uint32_t)npad * 128u;
      float* kbias = reinterpret_cast<float*>(smem + (size_t)npad * 384);
      if (g_chain_trace && blockIdx.x == 0 && si == 1 && threadIdx.x == 0)
        g_chain_trace[(size_t)kTraceCtas * kMaxStages * 2 + 327] = globaltimer_ns();
      for (int item = blockIdx.x; item < items; item += gridDim.x) {
        const int set = item / (s.heads * chunks);
        const int h = (item / chunks) % s.heads;
        const int ch = item % chunks;
        const int q_lo = ch * kWarps * 16, q_hi = min(npad, q_lo + kWarps * 16);
        const size_t row0 = (size_t)set * n;
        for (int idx = threadIdx.x; idx < npad * 8; idx += blockDim.x) {
          const int rr = idx >> 3, c = idx & 7;
          const bool q_row = rr >= q_lo && rr < q_hi;
          if (rr < n) {
            const bf16* src = s.qkv + (row0 + rr) * s.ld + c * 8;
            if (q_row) aset::cp_async16(aset::swz(qb, rr, c), src + s.qcol + h * 64);
            aset::cp_async16(aset::swz(kb, rr, c), src + s.kcol + h * 64);
            aset::cp_async16(aset::swz(vb, rr, c), src + s.vcol + h * 64);
          } else {
            const uint4 z = make_uint4(0, 0, 0, 0);
            if (q_row) *reinterpret_cast<uint4*>(smem + (aset::swz(qb, rr, c) - qb)) = z;
            *reinterpret_cast<uint4*>(smem + (aset::swz(kb, rr, c) - qb)) = z;
            *reinterpret_cast<uint4*>(smem + (aset::swz(vb, rr, c) - qb)) = z;
          }
        }
        for (int rr = threadIdx.x; rr < npad; rr += blockDim.x)
          kbias[rr] = rr < n ? (s.tok[row0 + rr] ? 0.0f : aset::kMaskedScore) : -INFINITY;
        aset::cp_async_wait_all();
        __syncthreads();
        unsigned long long* atr = (g_chain_trace && blockIdx.x == 0 && si == 1 && item == (int)blockIdx.x)
                                      ? g_chain_trace + (size_t)kTraceCtas * kMaxStages * 2 + 320 : nullptr;
        if (atr && threadIdx.x == 0) atr[0] = globaltimer_ns();
        const int q0 = q_lo + warp * 16;
        if (q0 < n)
          aset::set_tile<64>(qb, kb, vb, kbias, n, q0, lane, [&](int rr, int c, const uint4& v) {
            *reinterpret_cast<uint4*>(s.out + (row0 + rr) * s.ldo + h * 64 + c * 8) = v;
          });
        if (atr && lane == 0) atr[1 + warp] = globaltimer_ns();
        __syncthreads();
      }
    }
    if (si + 1 < p.nstages && !grid_sync(p.bar, abort_flag, si, &p.st[si + 1], sst)) break;
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ---- host side: stages are recorded by the forward, then launched at once ----
struct Rec {
  Params p;
  int nmaps = 0;
  bool active = false;
};
static thread_local Rec t_rec;

static int map_index(const CUtensorMap& m) {
  Rec& r = t_rec;
  for (int i = 0; i < r.nmaps; ++i)
    if (std::memcmp(&r.p.maps[i], &m, sizeof(CUtensorMap)) == 0) return i;
  if (r.nmaps >= kMaxMaps) return -1;
  r.p.maps[r.nmaps] = m;
  return r.nmaps++;
}

}  // namespace chain

}  // namespace tc

// bf16 2-D tensor map with 128-byte swizzle (shared with the attention kernels).
int set_gemm_trace(void* buf) {
  unsigned long long* p = (unsigned long long*)buf;
  CC2_CUDA(cudaMemcpyToSymbol(tc::pair::g_gemm_trace, &p, sizeof(p)));
  return CC2_OK;
}

int encode_bf16_map(CUtensorMap* map, const void* ptr, int cols, int rows, int ld, int box_cols, int box_rows) {
  return tc::make_map_box(map, ptr, cols, rows, ld, box_cols, box_rows);
}

// 0 (default): 1-SM 128 x 64 tiles for few rows, else 2-SM tiles when
// M > 128; 1: single-SM 128 x 256 / 128 x 128 tiles only; 2: as 0 without the
// 128 x 64 tiles; 3: 2-SM mainloop with the epilogue skipped (measurement
// only, output not written).  Set through cc2_set_gemm_variant.
int g_gemm_variant = 0;

int set_chain_trace(void* buf) {
  unsigned long long* p = (unsigned long long*)buf;
  CC2_CUDA(cudaMemcpyToSymbol(tc::chain::g_chain_trace, &p, sizeof(p)));
  return CC2_OK;
}

int set_chain_starve(int on) {
  const int v = on ? 1 : 0;
  CC2_CUDA(cudaMemcpyToSymbol(g_chain_starve, &v, sizeof(int)));
  return CC2_OK;
}

int set_gemm_starve(int on) {
  const int v = on ? 1 : 0;
  CC2_CUDA(cudaMemcpyToSymbol(g_gemm_starve, &v, sizeof(int)));
  return CC2_OK;
}

// Device epilogue arguments from the public ones, validated.
static int build_epi(const cc2_epilogue* e, int M, int N, tc::Epi* ep) {
  using namespace tc;
  *ep = Epi{};
  ep->flags = e ? e->flags : 0;
  if (e) {
    ep->ssq_in = e->ssq_in;
    ep->ssq_parts = (e->norm_dim + 63) / 64;
    ep->ssq_ld = e->ssq_ld;
    ep->inv_dim = e->norm_dim > 0 ? 1.0f / (float)e->norm_dim : 0.0f;
    ep->eps = e->eps;
    ep->bias = e->bias;
    ep->resid = (const bf16*)e->resid;
    ep->ld_resid = e->ld_resid;
    ep->ssq_out = e->ssq_out;
    ep->special = e->special;
    ep->sp_period = e->special_period;
    ep->sp_offset = e->special_offset;
    ep->rope_cs = e->rope_cs;
    ep->rope_period = e->rope_period;
    ep->rope_cols = e->rope_cols;
    ep->lo_out = (bf16*)e->lo_out;
    ep->resid_lo = (const bf16*)e->resid_lo;
    ep->ld_lo = e->ld_lo;
  }
  CC2_REQUIRE(!(ep->flags & CC2_EPI_LO) ||
                  (ep->lo_out && ((uintptr_t)ep->lo_out & 15u) == 0 && ep->ld_lo % 8 == 0 && ep->ld_lo >= N &&
                   (!(ep->flags & CC2_EPI_RESID) || (ep->resid_lo && ((uintptr_t)ep->resid_lo & 15u) == 0))),
              "gemm: lo args (16-byte aligned lo_out and resid_lo, ld_lo >= N and a multiple of 8)");
  CC2_REQUIRE(!(ep->flags & CC2_EPI_ROPE) ||
                  (ep->rope_cs && ((uintptr_t)ep->rope_cs & 15u) == 0 && ep->rope_period > 0 && ep->rope_cols % 64 == 0),
              "gemm: rope args (16-byte aligned table, period > 0, cols multiple of 64)");
  CC2_REQUIRE(!(ep->flags & CC2_EPI_ROWSCALE) || (ep->ssq_in && e->norm_dim > 0), "gemm: rowscale args");
  CC2_REQUIRE(!(ep->flags & CC2_EPI_BIAS) || (ep->bias && ((uintptr_t)ep->bias & 15u) == 0),
              "gemm: bias must be non-null and 16-byte aligned");
  CC2_REQUIRE(!(ep->flags & CC2_EPI_RESID) || (ep->resid && ((uintptr_t)ep->resid & 15u) == 0 && ep->ld_resid % 8 == 0),
              "gemm: resid alignment");
  CC2_REQUIRE(!(ep->flags & CC2_EPI_SSQ) || ep->ssq_out, "gemm: ssq_out null");
  CC2_REQUIRE(!(ep->flags & (CC2_EPI_SSQ | CC2_EPI_ROWSCALE)) || ep->ssq_ld >= M, "gemm: ssq_ld must be >= M");
  CC2_REQUIRE(!(ep->flags & CC2_EPI_SPECIAL) || (ep->special && ep->sp_period > 0), "gemm: special args");
  return CC2_OK;
}

// Set by the forward for its lifetime: every GEMM it issues reads the packed
// (constant) model weights as W.
static thread_local bool t_weights_const = false;
void set_gemm_weights_const(bool on) { t_weights_const = on; }

int launch_gemm_tc(const void* A, int lda, const void* W, int ldw, void* out, int ldo, int M, int N, int K,
                   const cc2_epilogue* e, cudaStream_t st) {
  using namespace tc;
  CC2_REQUIRE(M > 0 && N > 0 && K > 0, "gemm: bad sizes M=%d N=%d K=%d", M, N, K);
  CC2_REQUIRE(N % 16 == 0, "gemm(bf16): N must be a multiple of 16 (got %d)", N);
  CC2_REQUIRE(((uintptr_t)out & 15u) == 0 && ldo % 8 == 0, "gemm(bf16): out alignment");
  Epi ep{};
  CC2_TRY(build_epi(e, M, N, &ep));
  ep.wpre = t_weights_const && launch_overlap() ? 1 : 0;
  CUtensorMap ma, mb, mc, mr;
  CC2_TRY(make_map(&ma, A, K, M, lda, BM));
  CC2_TRY(make_map_box(&mc, out, N, M, ldo, 64, 32));
  if (ep.flags & CC2_EPI_RESID) {
    CC2_TRY(make_map_box(&mr, ep.resid, N, M, ep.ld_resid, 64, 32));
  } else {
    mr = mc;
  }
  // Few token rows (batch-1 serving: 133 rows per series): the 256 x 256 pair
  // tiles would put the whole GEMM on a handful of SMs, each running a
  // K-long chain of 128 x 256 MMAs.  128 x 64 tiles on single SMs spread the
  // weight stream and the MMAs over 4-8x more SMs (same per-element
  // accumulation order, so the results do not change).
  const int pair_ctas = 2 * ((M + 255) / 256) * ((N + 255) / 256);
  if (g_gemm_variant == 0 && N >= 64 && 2 * pair_ctas <= num_sms()) {
    CC2_TRY(make_map(&mb, W, K, N, ldw, 64));
    if (M <= 64) return launch<64, 64, 4>(ma, mb, mc, mr, M, N, K, ep, st, A, lda);
    return launch<64>(ma, mb, mc, mr, M, N, K, ep, st, A, lda);
  }
  if (g_gemm_variant != 1 && M > BM) {  // 2-SM tiles (256 x 256 per CTA pair)
    CC2_TRY(make_map(&mb, W, K, N, ldw, 128));
    return launch_pair(ma, mb, mc, mr, M, N, K, ep, st, g_gemm_variant);
  }
  const int tiles256 = ((M + BM - 1) / BM) * ((N + 255) / 256);
  if (N >= 256 && tiles256 >= num_sms()) {
    CC2_TRY(make_map(&mb, W, K, N, ldw, 256));
    return launch<256>(ma, mb, mc, mr, M, N, K, ep, st, A, lda);
  }
  CC2_TRY(make_map(&mb, W, K, N, ldw, 128));
  return launch<128>(ma, mb, mc, mr, M, N, K, ep, st, A, lda);
}

// ---- layer-persistent forward (see tc::chain) ----------------------------------
int chain_max_stages() { return tc::chain::kMaxStages; }
int chain_max_set() {
  const int ring = tc::chain::C::STAGES * tc::chain::C::STAGE_BYTES;
  const int whole_set = ring / (3 * 128 + 4);  // exact mode: Q, K, V, bias of the whole set
  const int split = (ring - 2048 - tc::chain::kWarps * 16 * (64 * 4 + 8)) / (2 * 128 + 4);  // split-key mode
  return std::min(whole_set, split) / 16 * 16;
}

int chain_begin(int M) {
  tc::chain::Rec& r = tc::chain::t_rec;
  CC2_REQUIRE(M > 0, "layer chain: M must be positive");
  r.p.nstages = 0;
  r.p.M = M;
  r.p.bar = nullptr;
  r.nmaps = 0;
  r.active = true;
  return CC2_OK;
}

void chain_abandon() { tc::chain::t_rec.active = false; }

int chain_add_gemm(const void* A, int lda, const void* W, int ldw, void* out, int ldo, int M, int N, int K,
                   const cc2_epilogue* e) {
  using namespace tc;
  chain::Rec& r = chain::t_rec;
  CC2_REQUIRE(r.active && M == r.p.M, "layer chain: GEMM of %d rows in a chain of %d", M, r.p.M);
  CC2_REQUIRE(r.p.nstages < chain::kMaxStages, "layer chain: more than %d stages", chain::kMaxStages);
  CC2_REQUIRE(N > 0 && K > 0 && N % 16 == 0, "layer chain: bad GEMM sizes N=%d K=%d", N, K);
  CC2_REQUIRE(((uintptr_t)out & 15u) == 0 && ldo % 8 == 0, "gemm(bf16): out alignment");
  chain::Stage& s = r.p.st[r.p.nstages];
  s = chain::Stage{};
  CC2_TRY(build_epi(e, M, N, &s.ep));
  CUtensorMap ma, mb, mc, mr;
  CC2_TRY(make_map(&ma, A, K, M, lda, BM));
  CC2_TRY(make_map(&mb, W, K, N, ldw, chain::BN));
  CC2_TRY(make_map_box(&mc, out, N, M, ldo, 64, 32));
  if (s.ep.flags & CC2_EPI_RESID) {
    CC2_TRY(make_map_box(&mr, s.ep.resid, N, M, s.ep.ld_resid, 64, 32));
  } else {
    mr = mc;
  }
  s.a = chain::map_index(ma); s.b = chain::map_index(mb); s.c = chain::map_index(mc); s.r = chain::map_index(mr);
  CC2_REQUIRE(s.a >= 0 && s.b >= 0 && s.c >= 0 && s.r >= 0, "layer chain: more than %d tensor maps",
              chain::kMaxMaps);
  s.kind = 0;
  s.N = N;
  s.K = K;
  s.w = W;
  s.wbytes = (ldw == K && (K * 2) % 16 == 0) ? (unsigned long long)N * K * 2 : 0;  // contiguous only
  ++r.p.nstages;
  return CC2_OK;
}

int chain_add_attention(const void* qkv, int ld, int qcol, int kcol, int vcol, void* out, int ldo,
                        const uint8_t* tok, int sets, int S, int heads) {
  using namespace tc;
  chain::Rec& r = chain::t_rec;
  CC2_REQUIRE(r.active && sets * S == r.p.M, "layer chain: attention over %d x %d rows in a chain of %d", sets, S,
              r.p.M);
  CC2_REQUIRE(r.p.nstages < chain::kMaxStages, "layer chain: more than %d stages", chain::kMaxStages);
  CC2_REQUIRE(qkv && out && tok && sets > 0 && heads > 0 && S > 0 && S <= chain_max_set(),
              "layer chain: attention sets of 1..%d tokens", chain_max_set());
  CC2_REQUIRE(((uintptr_t)qkv & 15u) == 0 && ((uintptr_t)out & 15u) == 0 && ld % 8 == 0 && ldo % 8 == 0 &&
                  qcol % 8 == 0 && kcol % 8 == 0 && vcol % 8 == 0,
              "layer chain: attention operands must be 16-byte aligned");
  chain::Stage& s = r.p.st[r.p.nstages];
  s = chain::Stage{};
  s.kind = 1;
  s.qkv = (const bf16*)qkv; s.out = (bf16*)out; s.tok = tok;
  s.ld = ld; s.ldo = ldo; s.qcol = qcol; s.kcol = kcol; s.vcol = vcol;
  s.sets = sets; s.S = S; s.heads = heads;
  ++r.p.nstages;
  return CC2_OK;
}

// Device scratch of a layer-persistent launch over M token rows: barrier
// word, split-K counters, split-K partials.
size_t chain_scratch_bytes() {
  const size_t counters = (size_t)tc::chain::kMaxStages * 3 * (3072 / tc::chain::BN) * 4 * sizeof(unsigned);
  return 256 + align_up(counters, 256) + (size_t)num_sms() * 128 * tc::chain::BN * sizeof(float);
}

// Launches the recorded stages on scratch (chain_scratch_bytes(), 256-byte
// aligned; its barrier word and counters are zeroed here on the stream).
// exact: no split-K and the whole-set attention arithmetic.
int chain_launch(void* scratch, size_t scratch_bytes, int exact, cudaStream_t st) {
  using namespace tc;
  chain::Rec& r = chain::t_rec;
  CC2_REQUIRE(r.active, "layer chain: nothing recorded");
  r.active = false;
  if (r.p.nstages == 0) return CC2_OK;
  CC2_REQUIRE(scratch && ((uintptr_t)scratch & 255u) == 0 && scratch_bytes >= chain_scratch_bytes(),
              "layer chain: scratch must be 256-byte aligned and at least %zu bytes", chain_scratch_bytes());
  const int grid = num_sms();
  const size_t counters_max = (size_t)chain::kMaxStages * 3 * (3072 / chain::BN) * 4;
  size_t cnt_used = 0;
  const int m_tiles = (r.p.M + BM - 1) / BM;
  for (int i = 0; i < r.p.nstages; ++i) {
    chain::Stage& s = r.p.st[i];
    if (s.kind != 0) continue;
    const int tiles = m_tiles * ((s.N + chain::BN - 1) / chain::BN);
    const int kblocks = (s.K + BK - 1) / BK;
    // Split only long k-loops: the partial round trip (store, fence, count,
    // reload) costs ~3 us, which a 12-k-block loop (~3.6 us) does not repay
    // (K = 3072 at 24 tiles: 20.9 -> 16.3 us per stage; K = 768: 9.8 -> 13.2).
    int S = 1;
    if (!exact && kblocks >= 32) {
      if (tiles * 4 <= grid) S = 4;
      else if (tiles * 2 <= grid) S = 2;
    }
    if (S > 1 && cnt_used + (size_t)tiles * 4 > counters_max) S = 1;
    s.split = S;
    s.cnt_off = (int)cnt_used;
    if (S > 1) cnt_used += (size_t)tiles * 4;
  }
  char* base = (char*)scratch;
  r.p.bar = (unsigned int*)base;
  r.p.cnt = (unsigned int*)(base + 256);
  r.p.part = (float*)(base + 256 + align_up(counters_max * sizeof(unsigned), 256));
  r.p.exact = exact ? 1 : 0;
  static unsigned long long attr_set = 0;  // one bit per device
  int dev = 0;
  CC2_CUDA(cudaGetDevice(&dev));
  if (dev >= 64 || !((attr_set >> dev) & 1ull)) {
    CC2_CUDA(cudaFuncSetAttribute(chain::chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, chain::SMEM));
    if (dev < 64) attr_set |= 1ull << dev;
  }
  CC2_CUDA(cudaMemsetAsync(base, 0, 256 + cnt_used * sizeof(unsigned), st));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = chain::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  CC2_CUDA(cudaLaunchKernelEx(&cfg, chain::chain_kernel, r.p));
  CC2_CHECK_LAUNCH();
  return CC2_OK;
}

}  // namespace cc2
