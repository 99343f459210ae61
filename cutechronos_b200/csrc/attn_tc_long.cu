// Time attention on tcgen05 for long sets: 145..640 tokens (context 8192:
// S = 521), bf16, RoPE already applied by the QKV GEMM.  Same semantics as
// the other attention kernels of this library (unscaled softmax; a masked key
// scores -1e30, keys past the set -inf): TimeSelfAttentionFallback.forward,
// cutechronos/model.py:209-275, unscaled_attention kernel_backends.py:113-153.
//
// One persistent CTA per SM walks (series, head) items.  Per item the whole
// K and V (up to 640 rows each, 128-byte swizzled TMA boxes of 128 rows)
// stay in shared memory; the queries run as tiles of 128 rows, two at a time:
// even tiles belong to pipeline 0, odd tiles to pipeline 1.  Each pipeline
// has its own Q buffer, its own MMA-issuing warp, four softmax warps (one
// thread per query row) and TMEM columns for S (128), P (64) and O (64).
// Per query tile the keys are visited once, in blocks of 128, with an
// online softmax:
//   S_j = Q K_j^T -> row max -> P_j = exp2(S_j - m) (bf16, written to TMEM)
//   -> O += P_j V_j (P the TMEM operand, V read MN-major from its box)
// The running max m is only moved when a block's max exceeds it by more than
// 2^8 (then O and the row sum are rescaled in TMEM first); otherwise the
// exponents are taken against the stale max, which keeps P <= 256 and costs
// nothing in precision (the same lazy-rescale rule as FlashAttention-4).
// S_{j+1} is computed while the softmax threads turn S_j into P_j, and the
// tensor core alternates between the two pipelines' MMAs.  A share of the
// exponentials runs as a polynomial on the FMA pipe next to the MUFU unit.
//   warp 0        TMA producer (K, V and the key bias per item; Q per tile)
//   warps 1, 2    MMA issuers of pipelines 0 and 1 (one thread each);
//                 warp 1 owns the 512 TMEM columns
//   warp 3        idle (it completes the first warpgroup, which hands its
//                 registers to the softmax warpgroups)
//   warps 4-7     softmax and epilogue of pipeline 0 (TMEM lane quarter
//                 warp % 4), warps 8-11 of pipeline 1
// Every wait is bounded (about 2 s): on expiry the CTA sets the attention
// error word, all roles leave their loops, copies and MMAs in flight are
// waited for, TMEM is freed and the kernel returns.
#include <cuda.h>

#include "common.cuh"
#include "tc_attn.cuh"

namespace cc2 {

int encode_bf16_map(CUtensorMap* map, const void* ptr, int cols, int rows, int ld, int box_cols, int box_rows);

namespace {

using namespace tcx;

constexpr int kThreads = 384;
// Registers per thread after the split: the producer / MMA warpgroup gives
// registers to the two softmax warpgroups.  128 x 72 + 256 x 216 = 64512 is
// exactly the 384 x 168 = 64512 the block is launched with.
constexpr int kRegsControl = 72, kRegsSoftmax = 216;
constexpr int kQT = 128, kKB = 128;
constexpr int kMaxKeys = 640;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kSCol = 0, kPCol = 256, kOCol = 384;  // + 128 G, + 64 G, + 64 G for pipeline G
constexpr uint32_t kBlockBytes = 128 * 128;            // 128 rows x 128 bytes
constexpr float kMaskedScore = -1e30f;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleLog2 = 8.0f;  // move the running max only past 2^8
// Pairs (of each 16) whose exponentials run on the FMA pipe instead of the
// MUFU unit (6 of 16): the MUFU unit alone would bound the softmax.
constexpr uint32_t kPolyPairs = (1u << 2) | (1u << 5) | (1u << 7) | (1u << 10) | (1u << 13) | (1u << 15);

// Optional event trace (cc2_set_attention_trace): CTA 0 records %globaltimer
// stamps of the first 8 query tiles of each pipeline (unit 8 G + tile).  Per
// key block j (events 8j + e): 0 softmax saw S_j, 1 row max done, 2 P_j in
// registers, 3 softmax saw P free, 4 P_j written; 5 S_j MMAs issued, 6 MMA
// saw P_j, 7 O MMAs issued.  Per tile: 40 Q load issued, 41 softmax saw O,
// 42 O stored.
constexpr int kTraceUnits = 16, kTraceEvents = 44;
__device__ unsigned long long* g_attn_long_trace = nullptr;

__device__ __forceinline__ void trace(unsigned long long* tr, uint32_t G, uint32_t n, int ev) {
  if (tr != nullptr && n < 8u) tr[(8u * G + n) * kTraceEvents + ev] = globaltimer_ns();
}

struct LArgs {
  int S, heads, items, nkb, nqt;
  int qcol, kcol, vcol, ldo;
  uint32_t k_off, v_off, kv_bytes;
};

__global__ void __launch_bounds__(kThreads, 1)
attn_tc_long_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV,
                    bf16* __restrict__ out, const uint8_t* __restrict__ tok, LArgs a, int* __restrict__ err) {
  pdl_launch_dependents();
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  __shared__ __align__(8) uint64_t q_full[2], q_empty[2], kv_full, kv_empty, s_full[2], s_free[2], p_full[2],
      p_free[2], o_full[2], mma_done[2];
  __shared__ __align__(16) float kbias[kMaxKeys];
  __shared__ uint32_t blk_masked;  // bit j: key block j of the item holds a masked or padding key
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;
  // pipeline 0 has written its first P: pipeline 1 starts then, half a block
  // behind, so that the two pipelines' exponentials do not coincide
  __shared__ volatile int p0_started;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int my_items = a.items > (int)blockIdx.x ? (a.items - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const uint32_t sbase = smem_u32(smem);  // Q buffers of the two pipelines at 0 and kBlockBytes

  if (tid == 0) {
    for (int G = 0; G < 2; ++G) {
      mbar_init(smem_u32(&q_full[G]), 1);
      mbar_init(smem_u32(&q_empty[G]), 1);
      mbar_init(smem_u32(&s_full[G]), 1);
      mbar_init(smem_u32(&s_free[G]), 4);
      mbar_init(smem_u32(&p_full[G]), 4);
      mbar_init(smem_u32(&p_free[G]), 1);
      mbar_init(smem_u32(&o_full[G]), 1);
      mbar_init(smem_u32(&mma_done[G]), 1);
    }
    mbar_init(smem_u32(&kv_full), 32);
    mbar_init(smem_u32(&kv_empty), 2);
    abort_flag = 0;
    p0_started = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();  // the kernel before may still run until here; activations are read from now on
  const uint32_t tmem = tmem_slot;
  unsigned long long* const tr = blockIdx.x == 0 ? g_attn_long_trace : nullptr;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsControl));
    int kv_issued = -1;
    uint32_t nq[2] = {0, 0};  // Q tiles loaded per pipeline
    for (int li = 0; li < my_items && !abort_flag; ++li) {
      const int item = (int)blockIdx.x + li * (int)gridDim.x;
      const int b = item / a.heads, h = item % a.heads;
      const int row0 = b * a.S;
      // K, V and the key bias of the item once both pipelines finished the previous item
      if (li > 0 && !mbar_wait_inl(smem_u32(&kv_empty), (uint32_t)(li - 1) & 1u, &abort_flag, err)) break;
      const uint32_t bkv = smem_u32(&kv_full);
      if (lane == 0) {
        mbar_expect_tx(bkv, a.kv_bytes);
        for (int j = 0; j < a.nkb; ++j) {
          tma_load(sbase + a.k_off + (uint32_t)j * kBlockBytes, &tmKV, bkv, a.kcol + h * 64, row0 + j * kKB);
          tma_load(sbase + a.v_off + (uint32_t)j * kBlockBytes, &tmKV, bkv, a.vcol + h * 64, row0 + j * kKB);
        }
      }
      uint32_t masked = 0;
      for (int k = lane; k < a.nkb * kKB; k += 32) {
        const float kb = k < a.S ? (tok[(size_t)b * a.S + k] ? 0.0f : kMaskedScore) : -INFINITY;
        kbias[k] = kb;
        if (__any_sync(0xffffffffu, kb != 0.0f)) masked |= 1u << (k / kKB);
      }
      if (lane == 0) blk_masked = masked;
      mbar_arrive(bkv);
      kv_issued = li;
      bool ok = true;
      for (int qt = 0; qt < a.nqt; ++qt) {
        const int G = qt & 1;
        if (nq[G] > 0 && !mbar_wait_inl(smem_u32(&q_empty[G]), (nq[G] - 1) & 1u, &abort_flag, err)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          const uint32_t bq = smem_u32(&q_full[G]);
          mbar_arrive_expect_tx(bq, kBlockBytes);
          tma_load(sbase + (uint32_t)G * kBlockBytes, &tmQ, bq, a.qcol + h * 64, row0 + qt * kQT);
          trace(tr, (uint32_t)G, nq[G], 40);
        }
        ++nq[G];
      }
      if (!ok) break;
    }
    // no copy may still be landing in shared memory when the CTA exits
    if (lane == 0) {
      const unsigned long long t0 = globaltimer_ns();
      if (kv_issued >= 0)
        while (!mbar_try(smem_u32(&kv_full), (uint32_t)kv_issued & 1u) && globaltimer_ns() - t0 < kWaitLimitNs) {
        }
      for (int G = 0; G < 2; ++G)
        if (nq[G] > 0)
          while (!mbar_try(smem_u32(&q_full[G]), (nq[G] - 1) & 1u) && globaltimer_ns() - t0 < kWaitLimitNs) {
          }
    }
    __syncwarp();
  } else if (warp == 1 || warp == 2) {
    // ---------------- MMA issuer of pipeline G ----------------
    // Per query tile: S_0, S_1, PV_0, S_2, PV_1, ..., S_{n-1}, PV_{n-2}, PV_{n-1}.
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsControl));
    const uint32_t G = (uint32_t)warp - 1u;
    if (lane == 0) {
      if (G == 1) {  // bounded: on expiry pipeline 1 simply starts
        const unsigned long long t0 = globaltimer_ns();
        while (!p0_started && !abort_flag && globaltimer_ns() - t0 < kWaitLimitNs) __nanosleep(64);
      }
      const uint32_t id_s = idesc(128, kKB, false), id_o = idesc(128, 64, true);
      const uint64_t dq = sw128_desc(sbase + G * kBlockBytes), dk0 = sw128_desc(sbase + a.k_off),
                     dv0 = sw128_desc(sbase + a.v_off);
      const uint32_t t_s = tmem + kSCol + 128u * G, t_p = tmem + kPCol + 64u * G, t_o = tmem + kOCol + 64u * G;
      uint32_t ns = 0, np = 0, nt = 0;  // S blocks, P blocks, query tiles so far
      bool ok = true, any = false;
      // S_j = Q K_j^T, after the softmax threads read the previous S
      auto issue_s = [&](int j) -> bool {
        if (ns > 0 && !mbar_wait_inl(smem_u32(&s_free[G]), (ns - 1) & 1u, &abort_flag, err)) return false;
        tc_fence_after();
        const uint64_t dk = dk0 + (uint64_t)(j * (kBlockBytes >> 4));
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) mma_bf16(t_s, dq + 2u * ks, dk + 2u * ks, id_s, ks > 0);
        mma_commit(smem_u32(&s_full[G]));
        trace(tr, G, nt, 8 * j + 5);
        ++ns;
        any = true;
        return true;
      };
      for (int li = 0; li < my_items && ok; ++li) {
        if (!mbar_wait_inl(smem_u32(&kv_full), (uint32_t)li & 1u, &abort_flag, err)) break;
        for (int qt = (int)G; qt < a.nqt && ok; qt += 2, ++nt) {
          if (!mbar_wait_inl(smem_u32(&q_full[G]), nt & 1u, &abort_flag, err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          ok = issue_s(0);
          for (int j = 0; j < a.nkb && ok; ++j) {
            if (j + 1 < a.nkb) ok = issue_s(j + 1);
            if (!ok) break;
            if (j == a.nkb - 1) mma_commit(smem_u32(&q_empty[G]));  // the tile's last S MMA is issued
            if (!mbar_wait_inl(smem_u32(&p_full[G]), np & 1u, &abort_flag, err)) {
              ok = false;
              break;
            }
            trace(tr, G, nt, 8 * j + 6);
            tc_fence_after();
            const uint64_t dv = dv0 + (uint64_t)(j * (kBlockBytes >> 4));
#pragma unroll
            for (int ks = 0; ks < kKB / 16; ++ks)
              mma_bf16_ts(t_o, t_p + 8u * ks, dv + 128u * ks, id_o, (j > 0 || ks > 0) ? 1u : 0u);
            mma_commit(smem_u32(&p_free[G]));
            trace(tr, G, nt, 8 * j + 7);
            ++np;
          }
          if (ok) mma_commit(smem_u32(&o_full[G]));
        }
        if (ok) mma_commit(smem_u32(&kv_empty));  // this pipeline is done with the item's K and V
      }
      // every MMA issued above has completed before TMEM is released
      if (any) {
        mma_commit(smem_u32(&mma_done[G]));
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try(smem_u32(&mma_done[G]), 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
        }
      }
    }
    __syncwarp();
  } else if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsControl));
  } else {
    // ---------------- softmax + epilogue of pipeline G (warps 4-7: 0, 8-11: 1) ----------------
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
    const uint32_t G = warp >= 8 ? 1u : 0u;
    const int q = warp & 3;
    const int r = 32 * q + lane;
    const uint32_t t_lane = tmem + ((uint32_t)(32 * q) << 16);
    const uint32_t t_s = t_lane + kSCol + 128u * G, t_p = t_lane + kPCol + 64u * G, t_o = t_lane + kOCol + 64u * G;
    const bool tw = (warp == 4 || warp == 8) && lane == 0;
    uint32_t ns = 0, np = 0, nt = 0;
    bool ok = true;
    for (int li = 0; li < my_items && ok; ++li) {
      if (!mbar_wait_inl(smem_u32(&kv_full), (uint32_t)li & 1u, &abort_flag, err)) break;  // key bias
      const int item = (int)blockIdx.x + li * (int)gridDim.x;
      const int b = item / a.heads, h = item % a.heads;
      const uint32_t masked = blk_masked;
      for (int qt = (int)G; qt < a.nqt && ok; qt += 2, ++nt) {
        const int row = qt * kQT + r;
        const bool valid = row < a.S;
        const bool warp_rows = qt * kQT + 32 * q < a.S;  // warp-uniform
        float m = -INFINITY, l = 0.0f;
        for (int j = 0; j < a.nkb; ++j) {
          if (!mbar_wait_inl(smem_u32(&s_full[G]), ns & 1u, &abort_flag, err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (tw) trace(tr, G, nt, 8 * j);
          uint32_t v[128];
          if (warp_rows) {
#pragma unroll
            for (int c = 0; c < 4; ++c) tmem_ld32(t_s + 32u * c, v + 32 * c);
            tmem_ld_wait();
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&s_free[G]));  // S_j is in registers
          ++ns;
          float scale = 1.0f;
          bool rescale = false;
          if (warp_rows) {
            // x = S log2(e) + key bias; blocks without masked keys skip the bias and
            // fold the scale into the exponent's FMA
            const bool clean = !((masked >> j) & 1u);
            float bm;
            if (clean) {
              float bm0 = -INFINITY, bm1 = -INFINITY;
#pragma unroll
              for (int i = 0; i < 128; i += 4) {
                bm0 = max3(bm0, __uint_as_float(v[i]), __uint_as_float(v[i + 1]));
                bm1 = max3(bm1, __uint_as_float(v[i + 2]), __uint_as_float(v[i + 3]));
              }
              bm = fmaxf(bm0, bm1) * kLog2e;
            } else {
              const float* kb = kbias + j * kKB;
              float bm0 = -INFINITY, bm1 = -INFINITY;
#pragma unroll
              for (int i = 0; i < 128; i += 4) {
                float4 b4;
                asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
                             : "=f"(b4.x), "=f"(b4.y), "=f"(b4.z), "=f"(b4.w)
                             : "r"(smem_u32(kb + i)));
                const float x0 = fmaf(__uint_as_float(v[i]), kLog2e, b4.x);
                const float x1 = fmaf(__uint_as_float(v[i + 1]), kLog2e, b4.y);
                const float x2 = fmaf(__uint_as_float(v[i + 2]), kLog2e, b4.z);
                const float x3 = fmaf(__uint_as_float(v[i + 3]), kLog2e, b4.w);
                v[i] = __float_as_uint(x0);
                v[i + 1] = __float_as_uint(x1);
                v[i + 2] = __float_as_uint(x2);
                v[i + 3] = __float_as_uint(x3);
                bm0 = max3(bm0, x0, x1);
                bm1 = max3(bm1, x2, x3);
              }
              bm = fmaxf(bm0, bm1);
            }
            if (j == 0) {
              m = bm;
            } else if (bm > m + kRescaleLog2) {
              scale = ex2(m - bm);
              l *= scale;
              m = bm;
              rescale = true;
            }
            if (tw) trace(tr, G, nt, 8 * j + 1);
          }
          // the previous O MMA has finished reading P and writing O
          if (np > 0 && !mbar_wait_inl(smem_u32(&p_free[G]), (np - 1) & 1u, &abort_flag, err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (tw) trace(tr, G, nt, 8 * j + 3);
          if (warp_rows) {
            // P_j = exp2(x - m), stored to TMEM 32 keys at a time; exponent
            // fma(x, 1, -m) = x - m exactly on masked blocks
            const bool clean = !((masked >> j) & 1u);
            const float sc = clean ? kLog2e : 1.0f;
            const uint64_t sc2 = f2_pack(sc, sc), nm2 = f2_pack(-m, -m);
            uint64_t l2 = f2_pack(0.0f, 0.0f);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              uint32_t pk[16];
#pragma unroll
              for (int k = 0; k < 16; ++k) {
                const uint64_t x2 =
                    f2_fma(f2_pack(__uint_as_float(v[32 * c + 2 * k]), __uint_as_float(v[32 * c + 2 * k + 1])), sc2, nm2);
                uint64_t p2;
                if ((kPolyPairs >> k) & 1u) {
                  p2 = f2_exp2_poly(x2);
                } else {
                  float x0, x1;
                  f2_unpack(x2, x0, x1);
                  p2 = f2_pack(ex2(x0), ex2(x1));
                }
                l2 = f2_add(l2, p2);
                float p0, p1;
                f2_unpack(p2, p0, p1);
                pk[k] = pack_bf16(p0, p1);
              }
              tmem_st16(t_p + 16u * c, pk);
            }
            float l0, l1;
            f2_unpack(l2, l0, l1);
            l += l0 + l1;
            if (tw) trace(tr, G, nt, 8 * j + 2);
          }
          if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
            for (int c = 0; c < 2; ++c) {
              uint32_t o[32];
              tmem_ld32(t_o + 32u * c, o);
              tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * scale);
              tmem_st32(t_o + 32u * c, o);
            }
          }
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&p_full[G]));
          if (G == 0 && lane == 0 && np == 0) p0_started = 1;
          if (tw) trace(tr, G, nt, 8 * j + 4);
          ++np;
        }
        if (!ok) break;
        if (!mbar_wait_inl(smem_u32(&o_full[G]), nt & 1u, &abort_flag, err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (tw) trace(tr, G, nt, 41);
        if (warp_rows) {
          const float inv = 1.0f / l;
          uint4* dst = reinterpret_cast<uint4*>(out + ((size_t)b * a.S + row) * a.ldo + h * 64);
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            uint32_t o[32];
            tmem_ld32(t_o + 32u * c, o);
            tmem_ld_wait();
            if (valid) {
#pragma unroll
              for (int gq = 0; gq < 4; ++gq) {
                uint4 w4;
                w4.x = pack_bf16(__uint_as_float(o[8 * gq + 0]) * inv, __uint_as_float(o[8 * gq + 1]) * inv);
                w4.y = pack_bf16(__uint_as_float(o[8 * gq + 2]) * inv, __uint_as_float(o[8 * gq + 3]) * inv);
                w4.z = pack_bf16(__uint_as_float(o[8 * gq + 4]) * inv, __uint_as_float(o[8 * gq + 5]) * inv);
                w4.w = pack_bf16(__uint_as_float(o[8 * gq + 6]) * inv, __uint_as_float(o[8 * gq + 7]) * inv);
                dst[4 * c + gq] = w4;
              }
            }
          }
          if (tw) trace(tr, G, nt, 42);
        }
        tc_fence_before();
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

size_t plan_long(int S, int heads, int num_sets, LArgs& a) {
  a = LArgs{};
  a.S = S;
  a.heads = heads;
  a.items = num_sets * heads;
  a.nkb = (S + kKB - 1) / kKB;
  a.nqt = (S + kQT - 1) / kQT;
  a.k_off = 2 * kBlockBytes;  // after the two Q buffers
  a.v_off = a.k_off + (uint32_t)a.nkb * kBlockBytes;
  a.kv_bytes = 2u * (uint32_t)a.nkb * kBlockBytes;
  return 1024 + (size_t)a.v_off + (size_t)a.nkb * kBlockBytes;
}

}  // namespace

int set_attn_long_trace(void* buf) {
  unsigned long long* p = (unsigned long long*)buf;
  CC2_CUDA(cudaMemcpyToSymbol(g_attn_long_trace, &p, sizeof(p)));
  return CC2_OK;
}

// True when the long-set tcgen05 kernel takes this call: 144 < S <= 640, aligned operands.
bool attn_tc_long_supported(int S, int ld, int ldo, const void* qkv, const void* out) {
  return S > 144 && S <= kMaxKeys && ((uintptr_t)qkv & 15u) == 0 && ((uintptr_t)out & 15u) == 0 &&
         (ld * 2) % 16 == 0 && ldo % 8 == 0;
}

int launch_attn_tc_long(const void* qkv, int ld, int qcol, int kcol, int vcol, void* out, int ldo,
                        const uint8_t* tok, int num_sets, int S, int heads, int* err, cudaStream_t st) {
  CC2_REQUIRE(attn_tc_long_supported(S, ld, ldo, qkv, out), "attention(tcgen05 long): unsupported shape S=%d", S);
  CC2_REQUIRE(qcol % 8 == 0 && kcol % 8 == 0 && vcol % 8 == 0,
              "attention(tcgen05 long): columns must be multiples of 8");
  LArgs a;
  const size_t smem = plan_long(S, heads, num_sets, a);
  a.qcol = qcol;
  a.kcol = kcol;
  a.vcol = vcol;
  a.ldo = ldo;
  CC2_REQUIRE(smem <= 227 * 1024, "attention(tcgen05 long): %zu bytes of shared memory needed", smem);
  CUtensorMap mq, mkv;
  const int rows = num_sets * S;
  CC2_TRY(encode_bf16_map(&mq, qkv, ld, rows, ld, 64, kQT));
  CC2_TRY(encode_bf16_map(&mkv, qkv, ld, rows, ld, 64, kKB));
  static unsigned long long attr_done = 0;  // one bit per device
  int dev = 0;
  CC2_CUDA(cudaGetDevice(&dev));
  if (dev >= 64 || !((attr_done >> dev) & 1ull)) {
    LArgs big;
    CC2_CUDA(cudaFuncSetAttribute(attn_tc_long_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)plan_long(kMaxKeys, 1, 1, big)));
    if (dev < 64) attr_done |= 1ull << dev;
  }
  const int grid = std::min(a.items, num_sms());
  CC2_CUDA(launch_k(attn_tc_long_kernel, grid, kThreads, smem, st, mq, mkv, (bf16*)out, tok, a, err));
  CC2_CHECK_LAUNCH();
  return CC2_OK;
}

}  // namespace cc2
