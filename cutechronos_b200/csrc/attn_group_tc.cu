// Group self-attention on the 5th-generation tensor cores (tcgen05), bf16, for
// batches whose series groups are contiguous runs of g series (g = 2, 4, 8,
// 16 or 32; configs[2]: 64 groups of 8).
//
// GroupSelfAttentionFallback.forward (cutechronos/model.py:295-312) attends,
// at every time step t and for every head, across the series of a group:
// softmax(q_b . k_b' + mask) over the g series b' of b's group, unscaled, no
// RoPE.  One item here = (time step t, head h, block of 128 consecutive
// series = 128 / g whole groups):
//   Q, K, V   the block's 128 rows at token t (a 3-D TMA box over
//             [series, token, column]: 128 series x 1 token x 64 columns)
//   S = Q K^T M = 128, N = 128 keys, K = 64 on tcgen05, fp32 in TMEM; only
//             the g x g diagonal blocks are used
//   softmax   warps 2..5, one query row per thread: the thread's g scores are
//             picked from a 32-column TMEM load of its warp's diagonal window
//             (rows 32q..32q+31 are exactly the keys 32q..32q+31 when g <= 32),
//             masked keys (token mask) score -1e30; P rounded to bf16 (as the
//             reference's .to(q.dtype)) is written into the row's g slots of
//             a 128 x 128 P tile in shared memory that is zero elsewhere
//             (zeroed once: every item writes the same slots)
//   O = P V   M = 128, N = 64, K = 128 on tcgen05 (V read MN-major from its
//             box); O / rowsum written to the series' output row.
// Persistent CTAs (two per SM); Q/K and V on separate barriers so the next
// item's Q and K stream in while this item's softmax runs.  Every wait is
// bounded (about 2 s): on expiry the CTA sets the attention error word, the
// roles leave their loops, copies and MMAs in flight are waited for, TMEM is
// freed and the kernel returns.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "tc_attn.cuh"

namespace cc2 {

namespace {

using namespace tcx;

constexpr int kGThreads = 192;               // TMA warp, MMA warp, 4 softmax/epilogue warps
constexpr uint32_t kGBox = 128u * 128u;      // 128 rows x 128 bytes
constexpr uint32_t kGTmemCols = 256;
constexpr uint32_t kGOCol = 128;
constexpr float kGMasked = -1e30f;
constexpr float kGLog2e = 1.4426950408889634f;
// shared memory: Q | K | V boxes, then the P tile (two 64-key blocks)
constexpr uint32_t kGQOff = 0, kGKOff = kGBox, kGVOff = 2 * kGBox, kGPOff = 3 * kGBox;
constexpr size_t kGSmem = 1024 + 5 * (size_t)kGBox;
// the packed short-set kernel: P in its own two blocks after Q | K | V (same offsets)
constexpr uint32_t kGPOffPack = 3 * kGBox;

struct GArgs {
  int S, heads, B, g, nblk, items;
  int qcol, kcol, vcol, ldo;
};

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"((uint64_t)map), "r"(bar), "r"(x), "r"(y), "r"(z)
      : "memory");
}

template <int G>
__global__ void __launch_bounds__(kGThreads, 2)
attn_group_tc_kernel(const __grid_constant__ CUtensorMap tm, bf16* __restrict__ out, const uint8_t* __restrict__ tok,
                     GArgs a, int* __restrict__ err) {
  pdl_launch_dependents();
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  __shared__ __align__(8) uint64_t full_qk, full_v, empty_qk, empty_v, s_full, p_full, o_full, mma_done;
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int my_items = a.items > (int)blockIdx.x ? (a.items - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const uint32_t sbase = smem_u32(smem);

  if (tid == 0) {
    mbar_init(smem_u32(&full_qk), 1);
    mbar_init(smem_u32(&full_v), 1);
    mbar_init(smem_u32(&empty_qk), 1);
    mbar_init(smem_u32(&empty_v), 1);
    mbar_init(smem_u32(&s_full), 1);
    mbar_init(smem_u32(&p_full), 4);
    mbar_init(smem_u32(&o_full), 1);
    mbar_init(smem_u32(&mma_done), 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // the P tile is zero outside the diagonal blocks for the whole kernel
  for (int i = tid; i < (int)(2 * kGBox / 16); i += kGThreads)
    asm volatile("st.shared.v4.b32 [%0], {%1,%1,%1,%1};" ::"r"(sbase + kGPOff + 16u * i), "r"(0u) : "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                 "r"(kGTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();  // activations are read from here on
  const uint32_t tmem = tmem_slot;

  auto item_coords = [&](int li, int& t, int& h, int& blk) {
    const int item = (int)blockIdx.x + li * (int)gridDim.x;  // item = (t * nblk + blk) * heads + h
    h = item % a.heads;
    const int r = item / a.heads;
    blk = r % a.nblk;
    t = r / a.nblk;
  };

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    int qk_n = -1, v_n = -1;
    for (int li = 0; li < my_items && !abort_flag; ++li) {
      int t, h, blk;
      item_coords(li, t, h, blk);
      if (li > 0 && !mbar_wait(smem_u32(&empty_qk), (uint32_t)(li - 1) & 1u, &abort_flag, err)) break;
      if (lane == 0) {
        const uint32_t b = smem_u32(&full_qk);
        mbar_arrive_expect_tx(b, 2 * kGBox);
        tma_load_3d(sbase + kGQOff, &tm, b, a.qcol + h * 64, t, blk * 128);
        tma_load_3d(sbase + kGKOff, &tm, b, a.kcol + h * 64, t, blk * 128);
      }
      qk_n = li;
      if (li > 0 && !mbar_wait(smem_u32(&empty_v), (uint32_t)(li - 1) & 1u, &abort_flag, err)) break;
      if (lane == 0) {
        const uint32_t b = smem_u32(&full_v);
        mbar_arrive_expect_tx(b, kGBox);
        tma_load_3d(sbase + kGVOff, &tm, b, a.vcol + h * 64, t, blk * 128);
      }
      v_n = li;
    }
    // no copy may still be landing in shared memory when the CTA exits
    if (lane == 0) {
      const int ns[2] = {qk_n, v_n};
      const uint32_t bs[2] = {smem_u32(&full_qk), smem_u32(&full_v)};
      for (int w = 0; w < 2; ++w) {
        if (ns[w] < 0) continue;
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try(bs[w], (uint32_t)ns[w] & 1u) && globaltimer_ns() - t0 < kWaitLimitNs) {
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t id_s = idesc(128, 128, false), id_o = idesc(128, 64, true);
      const uint64_t dq = sw128_desc(sbase + kGQOff), dk = sw128_desc(sbase + kGKOff);
      const uint64_t dv = sw128_desc(sbase + kGVOff), dp = sw128_desc(sbase + kGPOff);
      bool any = false;
      for (int li = 0; li < my_items; ++li) {
        const uint32_t par = (uint32_t)li & 1u;
        if (!mbar_wait(smem_u32(&full_qk), par, &abort_flag, err)) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) mma_bf16(tmem, dq + 2u * ks, dk + 2u * ks, id_s, ks > 0);
        mma_commit(smem_u32(&s_full));
        mma_commit(smem_u32(&empty_qk));
        any = true;
        if (!mbar_wait(smem_u32(&p_full), par, &abort_flag, err) ||
            !mbar_wait(smem_u32(&full_v), par, &abort_flag, err))
          break;
        tc_fence_after();
        // P: 16 keys per step, 32 bytes within a 64-key block; V: 16 rows (2048 bytes) per step
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          mma_bf16(tmem + kGOCol, dp + (uint64_t)((ks >> 2) * (kGBox >> 4) + 2 * (ks & 3)), dv + 128u * ks, id_o,
                   ks > 0);
        mma_commit(smem_u32(&o_full));
        mma_commit(smem_u32(&empty_v));
      }
      if (any) {  // every MMA issued above has completed before TMEM is released
        mma_commit(smem_u32(&mma_done));
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try(smem_u32(&mma_done), 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------- softmax + epilogue (warps 2..5) ----------------
    const int q = warp & 3;          // TMEM lane quarter: rows 32q .. 32q + 31
    const int r = 32 * q + lane;     // query row of the block
    const int gl = lane & ~(G - 1);  // first key of this row's group, relative to the warp's window
    const uint32_t t_s = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(32 * q);
    const uint32_t t_o = tmem + ((uint32_t)(32 * q) << 16) + kGOCol;
    // this row's P slots: keys 32q + gl .. + G - 1 (a 64-key block, chunks of 8 keys)
    const int k0 = 32 * q + gl;
    const uint32_t prow = sbase + kGPOff + (uint32_t)(k0 >> 6) * kGBox + (uint32_t)r * 128u;
    bool ok = true;
    // token-mask bytes of the row's group keys, loaded one item ahead (their
    // latency would otherwise sit on every item's softmax; series past B: masked)
    auto load_tok = [&](int li, uint32_t (&tk)[G]) {
      if (li >= my_items) return;
      int t, h, blk;
      item_coords(li, t, h, blk);
#pragma unroll
      for (int j = 0; j < G; ++j) {
        const int kb = blk * 128 + k0 + j;
        tk[j] = kb < a.B ? (uint32_t)__ldg(tok + (size_t)kb * a.S + t) : 0u;
      }
    };
    uint32_t tk_next[G];
    load_tok(0, tk_next);
    for (int li = 0; li < my_items && ok; ++li) {
      int t, h, blk;
      item_coords(li, t, h, blk);
      const int b = blk * 128 + r;  // this row's series
      float bias[G];
#pragma unroll
      for (int j = 0; j < G; ++j) bias[j] = tk_next[j] ? 0.0f : kGMasked;
      load_tok(li + 1, tk_next);
      ok = mbar_wait(smem_u32(&s_full), (uint32_t)li & 1u, &abort_flag, err);
      tc_fence_after();
      uint32_t sv[32];
      tmem_ld32(t_s, sv);
      tmem_ld_wait();
      // pick the row's G scores out of the 32-column window (no dynamic register indexing)
      float x[G];
#pragma unroll
      for (int j = 0; j < G; ++j) x[j] = 0.0f;
#pragma unroll
      for (int grp = 0; grp < 32 / G; ++grp)
#pragma unroll
        for (int j = 0; j < G; ++j) x[j] = gl == grp * G ? __uint_as_float(sv[grp * G + j]) : x[j];
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < G; ++j) {
        x[j] = fmaf(x[j], kGLog2e, bias[j]);
        mx = fmaxf(mx, x[j]);
      }
      float l = 0.0f;
      uint32_t pk[(G + 1) / 2];
#pragma unroll
      for (int j = 0; j < G; j += 2) {
        const float p0 = ex2(x[j] - mx), p1 = G > 1 ? ex2(x[j + 1] - mx) : 0.0f;
        l += p0 + p1;
        pk[j / 2] = pack_bf16(p0, p1);
      }
      // P slots: 16-byte chunks of 8 keys, 128-byte swizzle (chunk c of row r at c ^ (r % 8))
      const uint32_t sw = (uint32_t)(r & 7);
      if constexpr (G >= 8) {
#pragma unroll
        for (int c = 0; c < G / 8; ++c) {
          const uint32_t chunk = (uint32_t)(((k0 & 63) >> 3) + c);
          asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(prow + ((chunk ^ sw) << 4)), "r"(pk[4 * c]),
                       "r"(pk[4 * c + 1]), "r"(pk[4 * c + 2]), "r"(pk[4 * c + 3])
                       : "memory");
        }
      } else {
        const uint32_t chunk = (uint32_t)((k0 & 63) >> 3), within = (uint32_t)(k0 & 7) * 2u;
#pragma unroll
        for (int j = 0; j < G / 2; ++j)
          asm volatile("st.shared.b32 [%0], %1;" ::"r"(prow + ((chunk ^ sw) << 4) + within + 4u * j), "r"(pk[j])
                       : "memory");
      }
      tc_fence_before();
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&p_full));
      ok = mbar_wait(smem_u32(&o_full), (uint32_t)li & 1u, &abort_flag, err) && ok;
      tc_fence_after();
      uint32_t o[64];
      tmem_ld32(t_o, o);
      tmem_ld32(t_o + 32, o + 32);
      tmem_ld_wait();
      if (!ok) break;
      if (b < a.B) {
        const float inv = 1.0f / l;
        uint4* dst = reinterpret_cast<uint4*>(out + ((size_t)b * a.S + t) * a.ldo + h * 64);
#pragma unroll
        for (int c = 0; c < 8; ++c)
          dst[c] = make_uint4(pack_bf16(__uint_as_float(o[8 * c + 0]) * inv, __uint_as_float(o[8 * c + 1]) * inv),
                              pack_bf16(__uint_as_float(o[8 * c + 2]) * inv, __uint_as_float(o[8 * c + 3]) * inv),
                              pack_bf16(__uint_as_float(o[8 * c + 4]) * inv, __uint_as_float(o[8 * c + 5]) * inv),
                              pack_bf16(__uint_as_float(o[8 * c + 6]) * inv, __uint_as_float(o[8 * c + 7]) * inv));
      }
      tc_fence_before();
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kGTmemCols) : "memory");
}

// ---------------------------------------------------------------------------------
// Time attention for short sets (16 < S <= 64 tokens; context 512 gives S = 37)
// on tcgen05: two sets per 128-row tile, each in its own 64-row slot, so that a
// warp's 32 query rows (one TMEM lane quarter) always belong to one set and its
// keys are the 64 columns of that slot.  One item = (pair of sets, head):
//   Q, K, V   each set's S rows by a 2-D TMA box (64 columns x BH rows, BH = S
//             rounded up to 8) into rows 64 i .. of the slot i (rows past BH
//             keep finite data from before: the boxes were zeroed at start)
//   S = Q K^T 128 x 128 x 64; only the two 64 x 64 diagonal blocks are used
//   softmax   warps 2..5, one row per thread, the slot's 64 scores in one TMEM
//             round trip; key bias from shared memory (0, -1e30 for a masked
//             token, -inf past the set), written by the producer per item
//   O = P V   P (bf16, as the reference's .to(dtype)) fills the row's own
//             64-key block; the other block stays zero (zeroed once)
// Same structure, barriers and bounded waits as the group kernel above.
struct PArgs {
  int S, heads, num_sets, BH, items;
  int qcol, kcol, vcol, ldo;
};

template <int NCH>  // 8-key chunks that hold a set's keys: ceil(S / 8)
__global__ void __launch_bounds__(kGThreads, 2)
attn_pack_tc_kernel(const __grid_constant__ CUtensorMap tm, bf16* __restrict__ out, const uint8_t* __restrict__ tok,
                    PArgs a, int* __restrict__ err) {
  pdl_launch_dependents();
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  __shared__ __align__(8) uint64_t full_qk, full_v, empty_qk, empty_v, s_full, p_full, o_full, mma_done, kb_full[2];
  __shared__ __align__(16) float kbias[2][128];
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int my_items = a.items > (int)blockIdx.x ? (a.items - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const uint32_t sbase = smem_u32(smem);

  if (tid == 0) {
    mbar_init(smem_u32(&full_qk), 1);
    mbar_init(smem_u32(&full_v), 1);
    mbar_init(smem_u32(&empty_qk), 1);
    mbar_init(smem_u32(&empty_v), 1);
    mbar_init(smem_u32(&s_full), 1);
    mbar_init(smem_u32(&p_full), 4);
    mbar_init(smem_u32(&o_full), 1);
    mbar_init(smem_u32(&mma_done), 1);
    mbar_init(smem_u32(&kb_full[0]), 32);
    mbar_init(smem_u32(&kb_full[1]), 32);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // Q | K | V | P all zero to begin with: rows of a slot past its box and the
  // off-diagonal P block are then finite zeros for the whole kernel
  for (int i = tid; i < (int)(5 * kGBox / 16); i += kGThreads)
    asm volatile("st.shared.v4.b32 [%0], {%1,%1,%1,%1};" ::"r"(sbase + 16u * i), "r"(0u) : "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                 "r"(kGTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();
  const uint32_t tmem = tmem_slot;

  auto item_coords = [&](int li, int& pair, int& h) {
    const int item = (int)blockIdx.x + li * (int)gridDim.x;  // item = pair * heads + h
    h = item % a.heads;
    pair = item / a.heads;
  };
  const uint32_t box_bytes = (uint32_t)a.BH * 128u;

  if (warp == 0) {
    // ---------------- TMA producer + key biases ----------------
    int qk_n = -1, v_n = -1;
    // token-mask bytes of the item's 128 key slots (4 per lane), loaded one item ahead
    auto load_tok = [&](int li, uint32_t (&tk)[4]) {
      if (li >= my_items) return;
      int pair, h;
      item_coords(li, pair, h);
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int k = lane + 32 * m, set = 2 * pair + (k >> 6), j = k & 63;
        tk[m] = j < a.S && set < a.num_sets ? (tok[(size_t)set * a.S + j] ? 1u : 0u) : 2u;
      }
    };
    uint32_t tk[4] = {2u, 2u, 2u, 2u};
    load_tok(0, tk);
    for (int li = 0; li < my_items && !abort_flag; ++li) {
      int pair, h;
      item_coords(li, pair, h);
      if (li > 0 && !mbar_wait(smem_u32(&empty_qk), (uint32_t)(li - 1) & 1u, &abort_flag, err)) break;
      if (lane == 0) {
        const uint32_t b = smem_u32(&full_qk);
        mbar_arrive_expect_tx(b, 4 * box_bytes);
        for (int i = 0; i < 2; ++i) {
          const int row0 = (2 * pair + i) * a.S;  // rows past the tensor are zero-filled
          tma_load(sbase + kGQOff + 64u * 128u * i, &tm, b, a.qcol + h * 64, row0);
          tma_load(sbase + kGKOff + 64u * 128u * i, &tm, b, a.kcol + h * 64, row0);
        }
      }
      // key biases of both slots (buffer li % 2: its previous item's softmax
      // finished before S(li - 1) was issued, which empty_qk(li - 1) follows)
      float* kb = kbias[li & 1];
#pragma unroll
      for (int m = 0; m < 4; ++m) kb[lane + 32 * m] = tk[m] == 1u ? 0.0f : tk[m] == 0u ? kGMasked : -INFINITY;
      mbar_arrive(smem_u32(&kb_full[li & 1]));
      load_tok(li + 1, tk);
      qk_n = li;
      if (li > 0 && !mbar_wait(smem_u32(&empty_v), (uint32_t)(li - 1) & 1u, &abort_flag, err)) break;
      if (lane == 0) {
        const uint32_t b = smem_u32(&full_v);
        mbar_arrive_expect_tx(b, 2 * box_bytes);
        for (int i = 0; i < 2; ++i)
          tma_load(sbase + kGVOff + 64u * 128u * i, &tm, b, a.vcol + h * 64, (2 * pair + i) * a.S);
      }
      v_n = li;
    }
    if (lane == 0) {
      const int ns[2] = {qk_n, v_n};
      const uint32_t bs[2] = {smem_u32(&full_qk), smem_u32(&full_v)};
      for (int w = 0; w < 2; ++w) {
        if (ns[w] < 0) continue;
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try(bs[w], (uint32_t)ns[w] & 1u) && globaltimer_ns() - t0 < kWaitLimitNs) {
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t id_s = idesc(128, 128, false), id_o = idesc(128, 64, true);
      const uint64_t dq = sw128_desc(sbase + kGQOff), dk = sw128_desc(sbase + kGKOff);
      const uint64_t dv = sw128_desc(sbase + kGVOff), dp = sw128_desc(sbase + kGPOffPack);
      bool any = false;
      for (int li = 0; li < my_items; ++li) {
        const uint32_t par = (uint32_t)li & 1u;
        if (!mbar_wait(smem_u32(&full_qk), par, &abort_flag, err)) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) mma_bf16(tmem, dq + 2u * ks, dk + 2u * ks, id_s, ks > 0);
        mma_commit(smem_u32(&s_full));
        mma_commit(smem_u32(&empty_qk));
        any = true;
        if (!mbar_wait(smem_u32(&p_full), par, &abort_flag, err) ||
            !mbar_wait(smem_u32(&full_v), par, &abort_flag, err))
          break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          mma_bf16(tmem + kGOCol, dp + (uint64_t)((ks >> 2) * (kGBox >> 4) + 2 * (ks & 3)), dv + 128u * ks, id_o,
                   ks > 0);
        mma_commit(smem_u32(&o_full));
        mma_commit(smem_u32(&empty_v));
      }
      if (any) {
        mma_commit(smem_u32(&mma_done));
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try(smem_u32(&mma_done), 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------- softmax + epilogue (warps 2..5) ----------------
    const int q = warp & 3;
    const int slot = q >> 1;                 // warps on lanes 0..63 hold slot 0, 64..127 slot 1
    const int i = 32 * (q & 1) + lane;       // query row within the set
    const int r = 32 * q + lane;             // tile row = TMEM lane
    const uint32_t t_s = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(64 * slot);
    const uint32_t t_o = tmem + ((uint32_t)(32 * q) << 16) + kGOCol;
    const uint32_t prow = sbase + kGPOffPack + (uint32_t)slot * kGBox + (uint32_t)r * 128u;
    const uint32_t sw = (uint32_t)(r & 7);
    bool ok = true;
    for (int li = 0; li < my_items && ok; ++li) {
      int pair, h;
      item_coords(li, pair, h);
      const int set = 2 * pair + slot;
      ok = mbar_wait(smem_u32(&kb_full[li & 1]), (uint32_t)(li >> 1) & 1u, &abort_flag, err);
      ok = mbar_wait(smem_u32(&s_full), (uint32_t)li & 1u, &abort_flag, err) && ok;
      tc_fence_after();
      uint32_t v[64];
      tmem_ld32(t_s, v);
      if constexpr (NCH > 4) tmem_ld32(t_s + 32, v + 32);
      tmem_ld_wait();
      const float* kb = kbias[li & 1] + 64 * slot;
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 8 * NCH; j += 4) {
        const float4 b4 = *reinterpret_cast<const float4*>(kb + j);
        float* f = reinterpret_cast<float*>(v + j);
        f[0] = fmaf(f[0], kGLog2e, b4.x);
        f[1] = fmaf(f[1], kGLog2e, b4.y);
        f[2] = fmaf(f[2], kGLog2e, b4.z);
        f[3] = fmaf(f[3], kGLog2e, b4.w);
        mx = fmaxf(fmaxf(mx, fmaxf(f[0], f[1])), fmaxf(f[2], f[3]));
      }
      float l = 0.0f;
      // chunks past the set's keys stay zero (written once at start)
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        uint32_t pk[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float p0 = ex2(__uint_as_float(v[8 * c + 2 * e]) - mx);
          const float p1 = ex2(__uint_as_float(v[8 * c + 2 * e + 1]) - mx);
          l += p0 + p1;
          pk[e] = pack_bf16(p0, p1);
        }
        asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(prow + (((uint32_t)c ^ sw) << 4)), "r"(pk[0]),
                     "r"(pk[1]), "r"(pk[2]), "r"(pk[3])
                     : "memory");
      }
      tc_fence_before();
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&p_full));
      ok = mbar_wait(smem_u32(&o_full), (uint32_t)li & 1u, &abort_flag, err) && ok;
      tc_fence_after();
      uint32_t o[64];
      tmem_ld32(t_o, o);
      tmem_ld32(t_o + 32, o + 32);
      tmem_ld_wait();
      if (!ok) break;
      if (i < a.S && set < a.num_sets) {
        const float inv = 1.0f / l;
        uint4* dst = reinterpret_cast<uint4*>(out + ((size_t)set * a.S + i) * a.ldo + h * 64);
#pragma unroll
        for (int c = 0; c < 8; ++c)
          dst[c] = make_uint4(pack_bf16(__uint_as_float(o[8 * c + 0]) * inv, __uint_as_float(o[8 * c + 1]) * inv),
                              pack_bf16(__uint_as_float(o[8 * c + 2]) * inv, __uint_as_float(o[8 * c + 3]) * inv),
                              pack_bf16(__uint_as_float(o[8 * c + 4]) * inv, __uint_as_float(o[8 * c + 5]) * inv),
                              pack_bf16(__uint_as_float(o[8 * c + 6]) * inv, __uint_as_float(o[8 * c + 7]) * inv));
      }
      tc_fence_before();
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kGTmemCols) : "memory");
}

typedef CUresult (*EncodeTiledFn3)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn3 encode3() {
  static EncodeTiledFn3 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn3)p;
  });
  return fn;
}

}  // namespace

// True when the tcgen05 group kernel takes this layer: bf16, groups of g
// consecutive series (g = 2..32, a power of two), 16-byte aligned rows.
bool attn_group_tc_supported(int g, int ld, int ldo, const void* qkv, const void* out) {
  return (g == 2 || g == 4 || g == 8 || g == 16 || g == 32) && ((uintptr_t)qkv & 15u) == 0 &&
         ((uintptr_t)out & 15u) == 0 && (ld * 2) % 16 == 0 && ldo % 8 == 0;
}

int launch_attn_group_tc(const void* qkv, int ld, int qcol, int kcol, int vcol, void* out, int ldo,
                         const uint8_t* tok, int B, int S, int heads, int g, int* err, cudaStream_t st) {
  CC2_REQUIRE(attn_group_tc_supported(g, ld, ldo, qkv, out), "group attention(tcgen05): unsupported g=%d", g);
  CC2_REQUIRE(B > 0 && S > 0 && heads > 0 && B % g == 0, "group attention(tcgen05): bad sizes");
  CC2_REQUIRE(qcol % 8 == 0 && kcol % 8 == 0 && vcol % 8 == 0, "group attention(tcgen05): column alignment");
  EncodeTiledFn3 fn = encode3();
  CC2_REQUIRE(fn != nullptr, "cuTensorMapEncodeTiled unavailable");
  // [series B][token S][column ld] bf16, box 64 columns x 1 token x 128 series
  CUtensorMap map;
  cuuint64_t dims[3] = {(cuuint64_t)ld, (cuuint64_t)S, (cuuint64_t)B};
  cuuint64_t strides[2] = {(cuuint64_t)ld * 2, (cuuint64_t)S * ld * 2};
  cuuint32_t box[3] = {64, 1, 128};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(qkv), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled (group attention) failed (%d)", (int)r);
    return CC2_E_CUDA;
  }
  GArgs a{};
  a.S = S;
  a.heads = heads;
  a.B = B;
  a.g = g;
  a.nblk = (B + 127) / 128;
  a.items = S * heads * a.nblk;
  a.qcol = qcol;
  a.kcol = kcol;
  a.vcol = vcol;
  a.ldo = ldo;
  static unsigned long long attr_done = 0;  // one bit per device
  int dev = 0;
  CC2_CUDA(cudaGetDevice(&dev));
  if (dev >= 64 || !((attr_done >> dev) & 1ull)) {
    CC2_CUDA(cudaFuncSetAttribute(attn_group_tc_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGSmem));
    CC2_CUDA(cudaFuncSetAttribute(attn_group_tc_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGSmem));
    CC2_CUDA(cudaFuncSetAttribute(attn_group_tc_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGSmem));
    CC2_CUDA(cudaFuncSetAttribute(attn_group_tc_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGSmem));
    CC2_CUDA(cudaFuncSetAttribute(attn_group_tc_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGSmem));
    if (dev < 64) attr_done |= 1ull << dev;
  }
  const int grid = std::min(a.items, 2 * num_sms());
  switch (g) {
    case 2: CC2_CUDA(launch_k(attn_group_tc_kernel<2>, grid, kGThreads, kGSmem, st, map, (bf16*)out, tok, a, err)); break;
    case 4: CC2_CUDA(launch_k(attn_group_tc_kernel<4>, grid, kGThreads, kGSmem, st, map, (bf16*)out, tok, a, err)); break;
    case 8: CC2_CUDA(launch_k(attn_group_tc_kernel<8>, grid, kGThreads, kGSmem, st, map, (bf16*)out, tok, a, err)); break;
    case 16: CC2_CUDA(launch_k(attn_group_tc_kernel<16>, grid, kGThreads, kGSmem, st, map, (bf16*)out, tok, a, err)); break;
    default: CC2_CUDA(launch_k(attn_group_tc_kernel<32>, grid, kGThreads, kGSmem, st, map, (bf16*)out, tok, a, err)); break;
  }
  CC2_CHECK_LAUNCH();
  return CC2_OK;
}


// True when the packed tcgen05 kernel takes a time-attention call (bf16, RoPE
// already applied, 16 < S <= 64, aligned operands).
bool attn_pack_tc_supported(int S, int ld, int ldo, const void* qkv, const void* out) {
  return S > 16 && S <= 64 && ((uintptr_t)qkv & 15u) == 0 && ((uintptr_t)out & 15u) == 0 && (ld * 2) % 16 == 0 &&
         ldo % 8 == 0;
}

int launch_attn_pack_tc(const void* qkv, int ld, int qcol, int kcol, int vcol, void* out, int ldo, const uint8_t* tok,
                        int num_sets, int S, int heads, int* err, cudaStream_t st) {
  CC2_REQUIRE(attn_pack_tc_supported(S, ld, ldo, qkv, out), "attention(tcgen05 packed): unsupported S=%d", S);
  CC2_REQUIRE(num_sets > 0 && heads > 0, "attention(tcgen05 packed): bad sizes");
  CC2_REQUIRE(qcol % 8 == 0 && kcol % 8 == 0 && vcol % 8 == 0, "attention(tcgen05 packed): column alignment");
  EncodeTiledFn3 fn = encode3();
  CC2_REQUIRE(fn != nullptr, "cuTensorMapEncodeTiled unavailable");
  PArgs a{};
  a.S = S;
  a.heads = heads;
  a.num_sets = num_sets;
  a.BH = (S + 7) & ~7;
  a.items = (num_sets + 1) / 2 * heads;
  a.qcol = qcol;
  a.kcol = kcol;
  a.vcol = vcol;
  a.ldo = ldo;
  // [row][column] bf16 over the sets' rows, box 64 columns x BH rows
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)ld, (cuuint64_t)num_sets * S};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)a.BH};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(qkv), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled (packed attention) failed (%d)", (int)r);
    return CC2_E_CUDA;
  }
  static unsigned long long attr_done = 0;  // one bit per device
  int dev = 0;
  CC2_CUDA(cudaGetDevice(&dev));
  if (dev >= 64 || !((attr_done >> dev) & 1ull)) {
    CC2_CUDA(cudaFuncSetAttribute(attn_pack_tc_kernel<3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGSmem));
    CC2_CUDA(cudaFuncSetAttribute(attn_pack_tc_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGSmem));
    CC2_CUDA(cudaFuncSetAttribute(attn_pack_tc_kernel<5>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGSmem));
    CC2_CUDA(cudaFuncSetAttribute(attn_pack_tc_kernel<6>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGSmem));
    CC2_CUDA(cudaFuncSetAttribute(attn_pack_tc_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGSmem));
    if (dev < 64) attr_done |= 1ull << dev;
  }
  const int grid = std::min(a.items, 2 * num_sms());
  const int nch = (S + 7) / 8;  // 3..8
  if (nch <= 3)
    CC2_CUDA(launch_k(attn_pack_tc_kernel<3>, grid, kGThreads, kGSmem, st, map, (bf16*)out, tok, a, err));
  else if (nch == 4)
    CC2_CUDA(launch_k(attn_pack_tc_kernel<4>, grid, kGThreads, kGSmem, st, map, (bf16*)out, tok, a, err));
  else if (nch == 5)
    CC2_CUDA(launch_k(attn_pack_tc_kernel<5>, grid, kGThreads, kGSmem, st, map, (bf16*)out, tok, a, err));
  else if (nch == 6)
    CC2_CUDA(launch_k(attn_pack_tc_kernel<6>, grid, kGThreads, kGSmem, st, map, (bf16*)out, tok, a, err));
  else
    CC2_CUDA(launch_k(attn_pack_tc_kernel<8>, grid, kGThreads, kGSmem, st, map, (bf16*)out, tok, a, err));
  CC2_CHECK_LAUNCH();
  return CC2_OK;
}

}  // namespace cc2
