// Time attention on tcgen05 for long sets: 145..640 tokens (context 8192:
// S = 521), bf16, RoPE already applied by the QKV GEMM.  Same semantics as
// the other attention kernels of this library (unscaled softmax; a masked key
// scores -1e30, keys past the set -inf): TimeSelfAttentionFallback.forward,
// cutechronos/model.py:209-275, unscaled_attention kernel_backends.py:113-153.
//
// One persistent CTA per SM walks (series, head) items.  Per item the whole
// K and V (up to 640 rows each, 128-byte swizzled TMA boxes of 128 rows)
// stay in shared memory; the queries run as tiles of 128 rows.  Per query
// tile the keys are visited once, in blocks of 128, with an online softmax:
//   S_j = Q K_j^T -> block row max -> P_j = exp2(S_j - m) (bf16, swizzled
//   K-major in shared memory) -> O += P_j V_j (V read MN-major from its box)
// The running max m is only moved when a block's max exceeds it by more than
// 2^8 (then O and the row sum are rescaled in TMEM first); otherwise the
// exponents are taken against the stale max, which keeps P <= 256 and costs
// nothing in precision (the same lazy-rescale rule as FlashAttention-4).
//   warp 0      TMA producer (K, V and the key bias per item; Q per tile)
//   warp 1      TMEM owner and MMA issuer (one thread); TMEM: S in two
//               ping-pong buffers of 128 columns, O in 64 columns
//   warps 2-9   softmax and epilogue: TMEM lane quarter q = warp % 4 (query
//               rows 32q..), warps 2-5 the first 64 keys of each block and
//               O columns 0-31, warps 6-9 the other half; the two warps of a
//               quarter exchange block maxima through shared memory
// The S MMA of block j + 1 runs while the softmax warps process block j.
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

constexpr int kThreads = 320;
constexpr int kQT = 128, kKB = 128;
constexpr int kMaxKeys = 640;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kOCol = 256;
constexpr uint32_t kBlockBytes = 128 * 128;  // 128 rows x 128 bytes
constexpr float kMaskedScore = -1e30f;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleLog2 = 8.0f;  // move the running max only past 2^8

// Optional event trace (cc2_set_attention_trace): CTA 0 records %globaltimer
// stamps of its first kTraceUnits query tiles.  Per key block j (events
// 8j + e): 0 softmax saw S_j, 1 block max exchanged, 2 P_j in registers,
// 3 softmax saw P free, 4 P_j written; 5 S_j MMAs issued, 6 MMA saw P_j,
// 7 O MMAs issued.  Per tile: 40 Q load issued, 41 softmax saw O, 42 O stored.
constexpr int kTraceUnits = 16, kTraceEvents = 44;
__device__ unsigned long long* g_attn_long_trace = nullptr;

__device__ __forceinline__ void trace(unsigned long long* tr, uint32_t unit, int ev) {
  if (tr != nullptr && unit < (uint32_t)kTraceUnits) tr[unit * kTraceEvents + ev] = globaltimer_ns();
}

struct LArgs {
  int S, heads, items, nkb, nqt;
  int qcol, kcol, vcol, ldo;
  uint32_t k_off, v_off, p_off, kv_bytes;
};

__global__ void __launch_bounds__(kThreads, 1)
attn_tc_long_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV,
                    bf16* __restrict__ out, const uint8_t* __restrict__ tok, LArgs a, int* __restrict__ err) {
  pdl_launch_dependents();
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  __shared__ __align__(8) uint64_t q_full, q_empty, kv_full, kv_empty, s_full[2], s_free[2], p_full, p_free, o_full,
      mma_done;
  __shared__ __align__(16) float kbias[kMaxKeys];
  __shared__ float red_max[2][2][128], red_sum[2][128];
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int my_items = a.items > (int)blockIdx.x ? (a.items - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const uint32_t sbase = smem_u32(smem);  // Q tile at offset 0

  if (tid == 0) {
    mbar_init(smem_u32(&q_full), 1);
    mbar_init(smem_u32(&q_empty), 1);
    mbar_init(smem_u32(&kv_full), 32);
    mbar_init(smem_u32(&kv_empty), 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&s_full[b]), 1);
      mbar_init(smem_u32(&s_free[b]), 8);
    }
    mbar_init(smem_u32(&p_full), 8);
    mbar_init(smem_u32(&p_free), 1);
    mbar_init(smem_u32(&o_full), 1);
    mbar_init(smem_u32(&mma_done), 1);
    abort_flag = 0;
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
    int kv_issued = -1, q_issued = -1;  // phases of the last loads (for the exit wait)
    int t = 0;                          // query tiles issued so far
    for (int li = 0; li < my_items && !abort_flag; ++li) {
      const int item = (int)blockIdx.x + li * (int)gridDim.x;
      const int b = item / a.heads, h = item % a.heads;
      const int row0 = b * a.S;
      // K, V and the key bias of the item once the previous item's MMAs are done
      if (li > 0 && !mbar_wait(smem_u32(&kv_empty), (uint32_t)(li - 1) & 1u, &abort_flag, err)) break;
      const uint32_t bkv = smem_u32(&kv_full);
      if (lane == 0) {
        mbar_expect_tx(bkv, a.kv_bytes);
        for (int j = 0; j < a.nkb; ++j) {
          tma_load(sbase + a.k_off + (uint32_t)j * kBlockBytes, &tmKV, bkv, a.kcol + h * 64, row0 + j * kKB);
          tma_load(sbase + a.v_off + (uint32_t)j * kBlockBytes, &tmKV, bkv, a.vcol + h * 64, row0 + j * kKB);
        }
      }
      for (int k = lane; k < a.nkb * kKB; k += 32)
        kbias[k] = k < a.S ? (tok[(size_t)b * a.S + k] ? 0.0f : kMaskedScore) : -INFINITY;
      mbar_arrive(bkv);
      kv_issued = li;
      bool ok = true;
      for (int qt = 0; qt < a.nqt; ++qt, ++t) {
        if (t > 0 && !mbar_wait(smem_u32(&q_empty), (uint32_t)(t - 1) & 1u, &abort_flag, err)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          const uint32_t bq = smem_u32(&q_full);
          mbar_arrive_expect_tx(bq, kBlockBytes);
          tma_load(sbase, &tmQ, bq, a.qcol + h * 64, row0 + qt * kQT);
          trace(tr, (uint32_t)t, 40);
        }
        q_issued = t;
      }
      if (!ok) break;
    }
    // no copy may still be landing in shared memory when the CTA exits
    if (lane == 0) {
      const unsigned long long t0 = globaltimer_ns();
      if (kv_issued >= 0)
        while (!mbar_try(smem_u32(&kv_full), (uint32_t)kv_issued & 1u) && globaltimer_ns() - t0 < kWaitLimitNs) {
        }
      if (q_issued >= 0)
        while (!mbar_try(smem_u32(&q_full), (uint32_t)q_issued & 1u) && globaltimer_ns() - t0 < kWaitLimitNs) {
        }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t id_s = idesc(128, kKB, false), id_o = idesc(128, 64, true);
      const uint64_t dq = sw128_desc(sbase), dk0 = sw128_desc(sbase + a.k_off), dv0 = sw128_desc(sbase + a.v_off);
      const uint64_t dp = sw128_desc(sbase + a.p_off);
      uint32_t g = 0, c = 0, t = 0;  // S blocks, P blocks, query tiles so far
      bool ok = true, any = false;
      // S_j = Q K_j^T into buffer g & 1 (after the softmax released it)
      auto issue_s = [&](int j) -> bool {
        const uint32_t b = g & 1u;
        if (g >= 2 && !mbar_wait(smem_u32(&s_free[b]), ((g >> 1) - 1) & 1u, &abort_flag, err)) return false;
        tc_fence_after();
        const uint64_t dk = dk0 + (uint64_t)(j * (kBlockBytes >> 4));
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) mma_bf16(tmem + b * 128u, dq + 2u * ks, dk + 2u * ks, id_s, ks > 0);
        mma_commit(smem_u32(&s_full[b]));
        trace(tr, t, 8 * j + 5);
        ++g;
        any = true;
        return true;
      };
      for (int li = 0; li < my_items && ok; ++li) {
        if (!mbar_wait(smem_u32(&kv_full), (uint32_t)li & 1u, &abort_flag, err)) break;
        for (int qt = 0; qt < a.nqt && ok; ++qt, ++t) {
          if (!mbar_wait(smem_u32(&q_full), t & 1u, &abort_flag, err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          ok = issue_s(0);
          for (int j = 0; j < a.nkb && ok; ++j) {
            if (j + 1 < a.nkb) ok = issue_s(j + 1);
            if (!ok) break;
            if (j == a.nkb - 1) mma_commit(smem_u32(&q_empty));  // the tile's last S MMA is issued
            if (!mbar_wait(smem_u32(&p_full), c & 1u, &abort_flag, err)) {
              ok = false;
              break;
            }
            trace(tr, t, 8 * j + 6);
            tc_fence_after();
            const uint64_t dv = dv0 + (uint64_t)(j * (kBlockBytes >> 4));
            for (int ks = 0; ks < kKB / 16; ++ks)
              mma_bf16(tmem + kOCol, dp + (uint64_t)((ks >> 2) * (kBlockBytes >> 4) + 2 * (ks & 3)), dv + 128u * ks,
                       id_o, (j > 0 || ks > 0) ? 1u : 0u);
            mma_commit(smem_u32(&p_free));
            trace(tr, t, 8 * j + 7);
            ++c;
          }
          if (ok) mma_commit(smem_u32(&o_full));
        }
        if (ok) mma_commit(smem_u32(&kv_empty));
      }
      // every MMA issued above has completed before TMEM is released
      if (any) {
        mma_commit(smem_u32(&mma_done));
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try(smem_u32(&mma_done), 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------- softmax + epilogue (warps 2-9) ----------------
    const int q = warp & 3, hf = (warp - 2) >> 2;
    const int r = 32 * q + lane;
    const uint32_t t_lane = tmem + ((uint32_t)(32 * q) << 16);
    const uint32_t prow = sbase + a.p_off + (uint32_t)hf * kBlockBytes + (uint32_t)r * 128u;
    const uint32_t sw = (uint32_t)(r & 7);
    const uint32_t pair_bar = 1u + (uint32_t)q;  // named barrier of the two warps on these lanes
    uint32_t g = 0, c = 0, t = 0;
    bool ok = true;
    for (int li = 0; li < my_items && ok; ++li) {
      if (!mbar_wait(smem_u32(&kv_full), (uint32_t)li & 1u, &abort_flag, err)) break;  // key bias
      const int item = (int)blockIdx.x + li * (int)gridDim.x;
      const int b = item / a.heads, h = item % a.heads;
      for (int qt = 0; qt < a.nqt && ok; ++qt, ++t) {
        const int row = qt * kQT + r;
        const bool valid = row < a.S;
        const bool warp_rows = qt * kQT + 32 * q < a.S;  // warp-uniform
        float m = -INFINITY, l = 0.0f;
        const bool tw = warp == 2 && lane == 0;
        for (int j = 0; j < a.nkb; ++j) {
          const uint32_t sb = g & 1u;
          if (!mbar_wait(smem_u32(&s_full[sb]), (g >> 1) & 1u, &abort_flag, err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (tw) trace(tr, t, 8 * j);
          float scale = 1.0f;
          bool rescale = false;
          uint32_t pk[32];
          if (warp_rows) {
            uint32_t v[64];
            tmem_ld32(t_lane + sb * 128u + 64u * hf, v);
            tmem_ld32(t_lane + sb * 128u + 64u * hf + 32u, v + 32);
            tmem_ld_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&s_free[sb]));  // S_j is in registers
            const float* kb = kbias + j * kKB + 64 * hf;
            float bm = -INFINITY;
#pragma unroll
            for (int i = 0; i < 64; i += 4) {
              const float4 b4 = *reinterpret_cast<const float4*>(kb + i);
              v[i] = __float_as_uint(fmaf(__uint_as_float(v[i]), kLog2e, b4.x));
              v[i + 1] = __float_as_uint(fmaf(__uint_as_float(v[i + 1]), kLog2e, b4.y));
              v[i + 2] = __float_as_uint(fmaf(__uint_as_float(v[i + 2]), kLog2e, b4.z));
              v[i + 3] = __float_as_uint(fmaf(__uint_as_float(v[i + 3]), kLog2e, b4.w));
              bm = fmaxf(bm, fmaxf(fmaxf(__uint_as_float(v[i]), __uint_as_float(v[i + 1])),
                                   fmaxf(__uint_as_float(v[i + 2]), __uint_as_float(v[i + 3]))));
            }
            red_max[j & 1][hf][r] = bm;
            named_sync(pair_bar, 64);
            bm = fmaxf(bm, red_max[j & 1][hf ^ 1][r]);
            if (tw) trace(tr, t, 8 * j + 1);
            if (j == 0) {
              m = bm;
            } else if (bm > m + kRescaleLog2) {
              scale = ex2(m - bm);
              l *= scale;
              m = bm;
              rescale = true;
            }
            // P_j while the previous O MMA still runs
#pragma unroll
            for (int i = 0; i < 64; i += 2) {
              const float p0 = ex2(__uint_as_float(v[i]) - m), p1 = ex2(__uint_as_float(v[i + 1]) - m);
              l += p0 + p1;
              pk[i >> 1] = pack_bf16(p0, p1);
            }
            if (tw) trace(tr, t, 8 * j + 2);
          } else {
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&s_free[sb]));
          }
          ++g;
          // the previous O MMA has finished reading P and writing O
          if (c > 0 && !mbar_wait(smem_u32(&p_free), (c - 1) & 1u, &abort_flag, err)) {
            ok = false;
            break;
          }
          if (tw) trace(tr, t, 8 * j + 3);
          if (__any_sync(0xffffffffu, rescale)) {
            tc_fence_after();
            uint32_t o[32];
            tmem_ld32(t_lane + kOCol + 32u * hf, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * scale);
            tmem_st32(t_lane + kOCol + 32u * hf, o);
            tmem_st_wait();
          }
          if (warp_rows && valid) {
#pragma unroll
            for (int ch = 0; ch < 8; ++ch)
              asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(prow + (((uint32_t)ch ^ sw) << 4)),
                           "r"(pk[4 * ch]), "r"(pk[4 * ch + 1]), "r"(pk[4 * ch + 2]), "r"(pk[4 * ch + 3])
                           : "memory");
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&p_full));
          if (tw) trace(tr, t, 8 * j + 4);
          ++c;
        }
        if (!ok) break;
        if (!mbar_wait(smem_u32(&o_full), t & 1u, &abort_flag, err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (tw) trace(tr, t, 41);
        if (warp_rows) {
          red_sum[hf][r] = l;
          named_sync(pair_bar, 64);
          const float inv = 1.0f / (l + red_sum[hf ^ 1][r]);
          uint32_t o[32];
          tmem_ld32(t_lane + kOCol + 32u * hf, o);
          tmem_ld_wait();
          if (valid) {
            uint4* dst = reinterpret_cast<uint4*>(out + ((size_t)b * a.S + row) * a.ldo + h * 64 + 32 * hf);
#pragma unroll
            for (int gq = 0; gq < 4; ++gq) {
              uint4 w4;
              w4.x = pack_bf16(__uint_as_float(o[8 * gq + 0]) * inv, __uint_as_float(o[8 * gq + 1]) * inv);
              w4.y = pack_bf16(__uint_as_float(o[8 * gq + 2]) * inv, __uint_as_float(o[8 * gq + 3]) * inv);
              w4.z = pack_bf16(__uint_as_float(o[8 * gq + 4]) * inv, __uint_as_float(o[8 * gq + 5]) * inv);
              w4.w = pack_bf16(__uint_as_float(o[8 * gq + 6]) * inv, __uint_as_float(o[8 * gq + 7]) * inv);
              dst[gq] = w4;
            }
          }
          named_sync(pair_bar, 64);  // red_sum is rewritten by the next tile
          if (tw) trace(tr, t, 42);
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
  a.k_off = kBlockBytes;  // after the Q tile
  a.v_off = a.k_off + (uint32_t)a.nkb * kBlockBytes;
  a.p_off = a.v_off + (uint32_t)a.nkb * kBlockBytes;
  a.kv_bytes = 2u * (uint32_t)a.nkb * kBlockBytes;
  return 1024 + (size_t)a.p_off + 2 * kBlockBytes;
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
