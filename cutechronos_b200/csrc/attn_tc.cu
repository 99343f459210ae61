// Time attention on the 5th-generation tensor cores (tcgen05), bf16, for
// sets of 17..144 tokens (context 2048: S = 133; context 512: S = 37).
//
// One item = (series b, head h): Q, K, V are the set's S rows x 64 columns of
// the packed [Q|K|V] activations (RoPE already applied by the QKV GEMM).
// Unscaled softmax(Q K^T + mask) V, as TimeSelfAttentionFallback.forward
// (cutechronos/model.py:209-275) with unscaled_attention
// (kernel_backends.py:113-153).  Masking as the other attention kernels of
// this library: a masked key scores -1e30 (finite), keys past the set -inf.
//
// Persistent CTAs (two per SM), each with
//   warp 0      TMA producer: Q rows 0..127 (box 1), Q rows 128..S-1 (box 2,
//               when S > 128), K and V (NK = 64, 128 or 144 rows), plus
//               the set's key bias in shared memory;
//   warp 1      TMEM owner and MMA issuer (one thread):
//                 S = Q_t K^T   (M 128, N NK, K 64; both operands K-major)
//                 O = P V       (M 128, N 64,  K NK; V read MN-major)
//               accumulators in TMEM: S in columns [0, NK), O in [192, 256);
//   warps 2-5   one query row per thread (TMEM lane = row): the row's scores
//               read from TMEM in one round trip (NKM = 64, 128 or 144
//               columns, a template parameter), row max and exp2,
//               P written to shared memory
//               in the 128-byte-swizzled K-major layout the second MMA reads,
//               then O / rowsum written to global memory.
// A set with S > 128 has two query tiles that share K and V; the second one
// reuses the S and O columns.  Every wait is bounded (about 2 s): on expiry
// the CTA sets the attention error word, all roles leave their loops, copies
// and MMAs in flight are waited for, TMEM is freed, and the kernel returns.
#include <cuda.h>

#include "common.cuh"
#include "tc_attn.cuh"

namespace cc2 {

int encode_bf16_map(CUtensorMap* map, const void* ptr, int cols, int rows, int ld, int box_cols, int box_rows);

namespace {

using namespace tcx;

constexpr int kThreads = 320;  // TMA warp, MMA warp, 8 softmax warps
constexpr int kMaxNK = 144;
constexpr int kMaxStages = 2;
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kOCol = 192;
constexpr uint32_t kPBlock = 128 * 128;  // one 64-key block of P: 128 rows x 128 bytes
constexpr float kMaskedScore = -1e30f;
constexpr float kLog2e = 1.4426950408889634f;

// Optional event trace (cc2_set_attention_trace): CTA 0 records %globaltimer
// stamps of its first kTraceUnits query tiles, kTraceEvents per tile:
//   0 load issued  1 MMA saw the load  2 S MMAs issued  3 MMA saw P
//   4 O MMAs issued  5 softmax saw S  6 P written  7 softmax saw O  8 O stored
//   9 scores in registers  10 row max done
constexpr int kTraceUnits = 16, kTraceEvents = 12;
__device__ unsigned long long* g_attn_trace = nullptr;

__device__ __forceinline__ void trace(unsigned long long* tr, uint32_t unit, int ev) {
  if (tr != nullptr && unit < (uint32_t)kTraceUnits) tr[unit * kTraceEvents + ev] = globaltimer_ns();
}

struct Args {
  int S, heads, items, NK, T, q1rows;
  int split;  // 1: an item is one query tile of a (series, head) set (few sets: twice the CTAs)
  int qcol, kcol, vcol, ldo;
  int stages;
  uint32_t stage_bytes, q1_off, k_off, v_off, p_off, qk_bytes, v_bytes;
};

template <int NKM>
__global__ void __launch_bounds__(kThreads, 2)
attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ0, const __grid_constant__ CUtensorMap tmQ1,
               const __grid_constant__ CUtensorMap tmKV, bf16* __restrict__ out, const uint8_t* __restrict__ tok,
               Args a, int* __restrict__ err) {
  pdl_launch_dependents();
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  __shared__ __align__(8) uint64_t full_qk[kMaxStages], full_v[kMaxStages], empty_qk[kMaxStages],
      empty_v[kMaxStages];
  __shared__ __align__(8) uint64_t s_full, p_full, o_full, mma_done;
  // key bias by item index mod 3: the producer refills a buffer once the S MMA
  // of the item two or three places later is done, which orders it after
  // every read of the item that used it before
  __shared__ __align__(16) float kbias[3][kMaxNK];
  __shared__ float red_max[2][128], red_sum[2][128];
  // key bias buffer li % 3 filled (32 producer lanes arrive; phase li / 3).  Its
  // parity cannot alias: the producer refills a buffer only after the S MMA of
  // a later item, which needs this item's P.  (full_qk, which the producer may
  // complete twice while the softmax warps finish an item, would alias.)
  __shared__ __align__(8) uint64_t kb_full[3];
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int my_items = a.items > (int)blockIdx.x ? (a.items - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t pbase = sbase + a.p_off;
  unsigned long long* const tr = blockIdx.x == 0 ? g_attn_trace : nullptr;

  if (tid == 0) {
    for (int s = 0; s < kMaxStages; ++s) {
      mbar_init(smem_u32(&full_qk[s]), 32);
      mbar_init(smem_u32(&full_v[s]), 1);
      mbar_init(smem_u32(&empty_qk[s]), 1);
      mbar_init(smem_u32(&empty_v[s]), 1);
    }
    mbar_init(smem_u32(&s_full), 1);
    mbar_init(smem_u32(&p_full), 8);
    mbar_init(smem_u32(&o_full), 1);
    mbar_init(smem_u32(&mma_done), 1);
    for (int i = 0; i < 3; ++i) mbar_init(smem_u32(&kb_full[i]), 32);
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

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    // per item: Q, K and the key bias on full_qk (freed once the item's last
    // S MMA is done), V on full_v (freed after its last O MMA), so the next
    // item's Q and K stream in while this item's last tile is still running
    int qk_phase[kMaxStages] = {-1, -1}, v_phase[kMaxStages] = {-1, -1};
    for (int li = 0; li < my_items && !abort_flag; ++li) {
      const int st = li % a.stages, n = li / a.stages;
      const int item = (int)blockIdx.x + li * (int)gridDim.x;
      const int set_item = a.split ? item / a.T : item, tile = a.split ? item % a.T : -1;
      const int b = set_item / a.heads, h = set_item % a.heads;
      const uint32_t dst = sbase + (uint32_t)st * a.stage_bytes;
      const int row0 = b * a.S;
      if (n > 0 && !mbar_wait(smem_u32(&empty_qk[st]), (uint32_t)(n - 1) & 1u, &abort_flag, err)) break;
      const uint32_t bqk = smem_u32(&full_qk[st]);
      if (lane == 0) {
        // a split item loads only its own query box (tile 1 reads the Q0 slot's
        // last 64 rows as the A operand's first rows: stale, and their score
        // and output rows are never used)
        mbar_expect_tx(bqk, tile < 0 ? a.qk_bytes
                                     : a.v_bytes + (tile == 0 ? 128u * 128u : (uint32_t)a.q1rows * 128u));
        if (tile <= 0) tma_load(dst, &tmQ0, bqk, a.qcol + h * 64, row0);
        if (a.T == 2 && tile != 0) tma_load(dst + a.q1_off, &tmQ1, bqk, a.qcol + h * 64, row0 + 128);
        tma_load(dst + a.k_off, &tmKV, bqk, a.kcol + h * 64, row0);
        trace(tr, (uint32_t)(li * a.T), 0);
      }
      // the key bias is written while the copies are in flight; every lane
      // arrives after its own writes
      float* kb = kbias[li % 3];
      for (int k = lane; k < NKM; k += 32)
        kb[k] = k < a.S ? (tok[(size_t)b * a.S + k] ? 0.0f : kMaskedScore) : -INFINITY;
      mbar_arrive(smem_u32(&kb_full[li % 3]));
      mbar_arrive(bqk);
      qk_phase[st] = n;
      if (n > 0 && !mbar_wait(smem_u32(&empty_v[st]), (uint32_t)(n - 1) & 1u, &abort_flag, err)) break;
      if (lane == 0) {
        const uint32_t bv = smem_u32(&full_v[st]);
        mbar_arrive_expect_tx(bv, a.v_bytes);
        tma_load(dst + a.v_off, &tmKV, bv, a.vcol + h * 64, row0);
      }
      v_phase[st] = n;
    }
    // no copy may still be landing in shared memory when the CTA exits
    if (lane == 0)
      for (int s = 0; s < kMaxStages; ++s)
        for (int w = 0; w < 2; ++w) {
          const int ph = w == 0 ? qk_phase[s] : v_phase[s];
          if (ph < 0) continue;
          const uint32_t bar = smem_u32(w == 0 ? &full_qk[s] : &full_v[s]), par = (uint32_t)ph & 1u;
          const unsigned long long t0 = globaltimer_ns();
          while (!mbar_try(bar, par) && globaltimer_ns() - t0 < kWaitLimitNs) {
          }
        }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t id_s = idesc(128, a.NK, false), id_o = idesc(128, 64, true);
      const int ksteps_o = a.NK / 16;
      const uint64_t dp = sw128_desc(pbase);
      uint32_t u = 0;
      bool any = false;
      for (int li = 0; li < my_items; ++li) {
        const int st = li % a.stages, n = li / a.stages;
        if (!mbar_wait(smem_u32(&full_qk[st]), (uint32_t)n & 1u, &abort_flag, err)) break;
        tc_fence_after();
        trace(tr, u, 1);
        const uint32_t stage = sbase + (uint32_t)st * a.stage_bytes;
        const uint64_t dk = sw128_desc(stage + a.k_off), dv = sw128_desc(stage + a.v_off);
        const int item = (int)blockIdx.x + li * (int)gridDim.x;
        const int t_begin = a.split ? item % a.T : 0, t_end = a.split ? t_begin + 1 : a.T;
        bool ok = true;
        for (int t = t_begin; t < t_end; ++t, ++u) {
          // tile 1: the A operand starts 64 rows before the Q1 box, so the
          // set's last rows land on TMEM lanes 64.. (warps 2 and 6, whose
          // SM sub-partition runs neither the producer nor the MMA warp)
          const uint64_t dq = sw128_desc(t == 0 ? stage : stage + a.q1_off - 64u * 128u);
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) mma_bf16(tmem, dq + 2u * ks, dk + 2u * ks, id_s, ks > 0);
          mma_commit(smem_u32(&s_full));
          if (t == t_end - 1) mma_commit(smem_u32(&empty_qk[st]));
          trace(tr, u, 2);
          any = true;
          if (!mbar_wait(smem_u32(&p_full), u & 1u, &abort_flag, err) ||
              (t == t_begin && !mbar_wait(smem_u32(&full_v[st]), (uint32_t)n & 1u, &abort_flag, err))) {
            ok = false;
            break;
          }
          tc_fence_after();
          trace(tr, u, 3);
          // descriptor start addresses advance in 16-byte units: P by 32 bytes per
          // 16 keys within a 64-key block, V by 16 rows (2048 bytes) per step
          for (int ks = 0; ks < ksteps_o; ++ks)
            mma_bf16(tmem + kOCol, dp + (uint64_t)((ks >> 2) * (kPBlock >> 4) + 2 * (ks & 3)), dv + 128u * ks, id_o,
                     ks > 0);
          mma_commit(smem_u32(&o_full));
          trace(tr, u, 4);
          if (t == t_end - 1) mma_commit(smem_u32(&empty_v[st]));
        }
        if (!ok) break;
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
    // warp w reads TMEM lanes 32 * (w % 4) ...; warps 2-5 take the first half
    // of each score row's NKM columns and of O's 64 columns, warps 6-9 the second
    const int q = warp & 3, hf = (warp - 2) >> 2;
    const int r = 32 * q + lane;
    constexpr int HW = NKM / 2;  // score columns per thread
    const int c0 = hf * HW;
    const uint32_t t_s = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0;
    const uint32_t t_o = tmem + ((uint32_t)(32 * q) << 16) + kOCol + 32u * hf;
    const uint32_t prow = pbase + (uint32_t)r * 128u;
    const uint32_t sw = (uint32_t)(r & 7);
    // Named barrier of the two warps on these lanes.  Both pass the same two
    // barriers per tile whether or not they hold rows of it; a failed bounded
    // wait is carried to the next barrier, whose AND tells both to stop, so
    // neither can be left waiting for the other.
    const uint32_t pair_bar = 1u + (uint32_t)q;
    uint32_t u = 0;
    bool ok = true;
    for (int li = 0; li < my_items && ok; ++li) {
      ok = mbar_wait(smem_u32(&kb_full[li % 3]), (uint32_t)(li / 3) & 1u, &abort_flag, err);  // key bias
      const int item = (int)blockIdx.x + li * (int)gridDim.x;
      const int set_item = a.split ? item / a.T : item;
      const int t_begin = a.split ? item % a.T : 0, t_end = a.split ? t_begin + 1 : a.T;
      const int b = set_item / a.heads, h = set_item % a.heads;
      const float* kb = kbias[li % 3] + c0;
      for (int t = t_begin; t < t_end; ++t, ++u) {
        // lane r holds query row t * 128 + r - lane0 (tile 1 starts at lane 64)
        const int lane0 = t == 0 ? 0 : 64;
        const int rows_t = t == 0 ? min(a.S, 128) : a.S - 128;
        const bool warp_rows = 32 * q + 31 >= lane0 && 32 * q < lane0 + rows_t;  // warp-uniform
        const bool valid = r >= lane0 && r < lane0 + rows_t;
        if (ok) ok = mbar_wait(smem_u32(&s_full), u & 1u, &abort_flag, err);
        tc_fence_after();
        const bool tw = tr != nullptr && warp == 2 && lane == 0;
        if (tw) trace(tr, u, 5);
        float l = 0.0f;
        if (warp_rows) {
          float v[HW];
          float mx = -INFINITY;
          {  // (after a failed wait the scores are garbage and unused)
#pragma unroll
            for (int c = 0; c + 32 <= HW; c += 32) tmem_ld32(t_s + (uint32_t)c, reinterpret_cast<uint32_t*>(v + c));
            if (HW % 32 == 8) tmem_ld8(t_s + (uint32_t)(HW - 8), reinterpret_cast<uint32_t*>(v + HW - 8));
            tmem_ld_wait();
            if (tw) trace(tr, u, 9);
            // score * log2(e) + bias: 0 for a key, -1e30 for a masked key (the
            // sum stays -1e30 in fp32), -inf past the set
#pragma unroll
            for (int j = 0; j < HW; j += 4) {
              const float4 b4 = *reinterpret_cast<const float4*>(kb + j);
              v[j] = fmaf(v[j], kLog2e, b4.x);
              v[j + 1] = fmaf(v[j + 1], kLog2e, b4.y);
              v[j + 2] = fmaf(v[j + 2], kLog2e, b4.z);
              v[j + 3] = fmaf(v[j + 3], kLog2e, b4.w);
              mx = fmaxf(fmaxf(mx, fmaxf(v[j], v[j + 1])), fmaxf(v[j + 2], v[j + 3]));
            }
          }
          red_max[hf][r] = mx;
          ok = barrier_and(pair_bar, 64, ok);
          if (ok) {
            mx = fmaxf(mx, red_max[hf ^ 1][r]);
            if (tw) trace(tr, u, 10);
#pragma unroll
            for (int j = 0; j < HW; j += 8) {
              uint32_t pk[4];
              float ls = 0.0f;
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const float p0 = ex2(v[j + 2 * i] - mx), p1 = ex2(v[j + 2 * i + 1] - mx);
                ls += p0 + p1;
                pk[i] = pack_bf16(p0, p1);
              }
              l += ls;
              if (valid) {
                const int k = c0 + j;
                const uint32_t addr = prow + (uint32_t)(k >> 6) * kPBlock + ((((uint32_t)(k & 63) >> 3) ^ sw) << 4);
                asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(pk[0]), "r"(pk[1]),
                             "r"(pk[2]), "r"(pk[3])
                             : "memory");
              }
            }
            red_sum[hf][r] = l;
          }
        } else {
          ok = barrier_and(pair_bar, 64, ok);
        }
        if (!ok) break;
        tc_fence_before();
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&p_full));
        if (tw) trace(tr, u, 6);
        ok = mbar_wait(smem_u32(&o_full), u & 1u, &abort_flag, err);
        tc_fence_after();
        if (tw) trace(tr, u, 7);
        if (warp_rows) {
          uint32_t o[32];
          tmem_ld32(t_o, o);
          ok = barrier_and(pair_bar, 64, ok);  // and the other half's row sum is in red_sum
          tmem_ld_wait();                      // nothing may be outstanding at an exit
          if (!ok) break;
          const float inv = 1.0f / (l + red_sum[hf ^ 1][r]);
          // normalised bf16 row (32 columns = 4 chunks of 16 bytes) into this
          // warp's own part of P (dead since the O MMAs completed) ...
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const int k = c0 + 8 * g;
            const uint32_t addr = prow + (uint32_t)(k >> 6) * kPBlock + ((((uint32_t)(k & 63) >> 3) ^ sw) << 4);
            asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr),
                         "r"(pack_bf16(__uint_as_float(o[8 * g + 0]) * inv, __uint_as_float(o[8 * g + 1]) * inv)),
                         "r"(pack_bf16(__uint_as_float(o[8 * g + 2]) * inv, __uint_as_float(o[8 * g + 3]) * inv)),
                         "r"(pack_bf16(__uint_as_float(o[8 * g + 4]) * inv, __uint_as_float(o[8 * g + 5]) * inv)),
                         "r"(pack_bf16(__uint_as_float(o[8 * g + 6]) * inv, __uint_as_float(o[8 * g + 7]) * inv))
                         : "memory");
          }
          __syncwarp();
          // ... then read back so that 4 lanes write one row's 64 contiguous bytes
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int rr = 32 * q + 8 * i + (lane >> 2), g = lane & 3;
            const int orow = t * 128 + rr - lane0;
            if (rr >= lane0 && rr < lane0 + rows_t) {
              const int k = c0 + 8 * g;
              const uint32_t addr = pbase + (uint32_t)rr * 128u + (uint32_t)(k >> 6) * kPBlock +
                                    ((((uint32_t)(k & 63) >> 3) ^ (uint32_t)(rr & 7)) << 4);
              uint4 w4;
              asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
                           : "=r"(w4.x), "=r"(w4.y), "=r"(w4.z), "=r"(w4.w)
                           : "r"(addr));
              *reinterpret_cast<uint4*>(out + ((size_t)b * a.S + orow) * a.ldo + h * 64 + 32 * hf + 8 * g) = w4;
            }
          }
          __syncwarp();
        } else {
          ok = barrier_and(pair_bar, 64, ok);
          if (!ok) break;
        }
        tc_fence_before();
        if (tw) trace(tr, u, 8);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

// Launch plan: shared-memory layout of one CTA.  Two CTAs share an SM, so a
// CTA takes at most half of the 227 KB, and at least a third of it so that no
// third CTA lands on an SM (TMEM holds two 256-column grants).
constexpr size_t kHalfSmem = 113 * 1024;

size_t plan(int S, int heads, int num_sets, Args& a) {
  a = Args{};
  a.S = S;
  a.heads = heads;
  a.items = num_sets * heads;
  // keys per set as the MMAs see them: 64, 128 or 144 rows of K and V (rows
  // past the set are the next set's, or zero past the tensor, and masked)
  a.NK = S <= 64 ? 64 : S <= 128 ? 128 : 144;
  a.T = S > 128 ? 2 : 1;
  a.q1rows = a.T == 2 ? ((S - 128 + 7) & ~7) : 8;
  const uint32_t kv_bytes = (uint32_t)a.NK * 128u;
  a.q1_off = 128u * 128u;
  const uint32_t q1_bytes = a.T == 2 ? ((uint32_t)a.q1rows * 128u + 1023u) & ~1023u : 0u;
  a.k_off = a.q1_off + q1_bytes;
  a.v_off = a.k_off + ((kv_bytes + 1023u) & ~1023u);
  a.stage_bytes = a.v_off + ((kv_bytes + 1023u) & ~1023u);
  a.qk_bytes = 128u * 128u + (a.T == 2 ? (uint32_t)a.q1rows * 128u : 0u) + kv_bytes;
  a.v_bytes = kv_bytes;
  const size_t p_bytes = (size_t)((a.NK + 63) / 64) * kPBlock;
  a.stages = 1024 + 2 * (size_t)a.stage_bytes + p_bytes <= kHalfSmem ? 2 : 1;
  a.p_off = (uint32_t)a.stages * a.stage_bytes;
  return 1024 + (size_t)a.p_off + p_bytes;
}

}  // namespace

// True when the tcgen05 kernel takes this call (bf16 time attention, RoPE
// already applied, 16 < S <= 144, aligned operands).
bool attn_tc_supported(int S, int ld, int ldo, const void* qkv) {
  if (S <= 16 || S > kMaxNK || ((uintptr_t)qkv & 15u) != 0 || (ld * 2) % 16 != 0 || ldo % 8 != 0) return false;
  Args a;
  return plan(S, 1, 1, a) <= kHalfSmem;
}

int set_attn_trace(void* buf) {
  unsigned long long* p = (unsigned long long*)buf;
  CC2_CUDA(cudaMemcpyToSymbol(g_attn_trace, &p, sizeof(p)));
  return CC2_OK;
}

int launch_attn_tc(const void* qkv, int ld, int qcol, int kcol, int vcol, void* out, int ldo, const uint8_t* tok,
                   int num_sets, int S, int heads, int* err, cudaStream_t st) {
  CC2_REQUIRE(attn_tc_supported(S, ld, ldo, qkv), "attention(tcgen05): unsupported shape S=%d", S);
  CC2_REQUIRE(qcol % 8 == 0 && kcol % 8 == 0 && vcol % 8 == 0, "attention(tcgen05): columns must be multiples of 8");
  Args a;
  size_t smem = plan(S, heads, num_sets, a);
  a.qcol = qcol;
  a.kcol = kcol;
  a.vcol = vcol;
  a.ldo = ldo;
  smem = std::max<size_t>(smem, 80 * 1024);
  const size_t half = kHalfSmem;

  CUtensorMap mq0, mq1, mkv;
  const int rows = num_sets * S;
  CC2_TRY(encode_bf16_map(&mq0, qkv, ld, rows, ld, 64, 128));
  CC2_TRY(encode_bf16_map(&mq1, qkv, ld, rows, ld, 64, a.q1rows));
  CC2_TRY(encode_bf16_map(&mkv, qkv, ld, rows, ld, 64, a.NK));
  static unsigned long long attr_done = 0;  // one bit per device
  int dev = 0;
  CC2_CUDA(cudaGetDevice(&dev));
  if (dev >= 64 || !((attr_done >> dev) & 1ull)) {
    CC2_CUDA(cudaFuncSetAttribute(attn_tc_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)half));
    CC2_CUDA(cudaFuncSetAttribute(attn_tc_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)half));
    CC2_CUDA(cudaFuncSetAttribute(attn_tc_kernel<144>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)half));
    if (dev < 64) attr_done |= 1ull << dev;
  }
  // few sets (batch-1 serving): each query tile of a two-tile set is an item
  // of its own, so the two tile chains run on two CTAs at once
  a.split = a.T == 2 && 2 * a.items <= 2 * num_sms() ? 1 : 0;
  if (a.split) a.items *= a.T;
  const int grid = std::min(a.items, 2 * num_sms());
  if (a.NK <= 64)
    CC2_CUDA(launch_k(attn_tc_kernel<64>, grid, kThreads, smem, st, mq0, mq1, mkv, (bf16*)out, tok, a, err));
  else if (a.NK <= 128)
    CC2_CUDA(launch_k(attn_tc_kernel<128>, grid, kThreads, smem, st, mq0, mq1, mkv, (bf16*)out, tok, a, err));
  else
    CC2_CUDA(launch_k(attn_tc_kernel<144>, grid, kThreads, smem, st, mq0, mq1, mkv, (bf16*)out, tok, a, err));
  CC2_CHECK_LAUNCH();
  return CC2_OK;
}

}  // namespace cc2
