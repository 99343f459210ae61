// One warp's share of the whole-set bf16 attention: a 16-row query tile of a
// set whose Q, K and V rows sit in swizzled shared memory, mma.sync m16n8k16
// with fp32 accumulation and an online softmax in the exp2 domain over key
// tiles of KTT.  Shared by the per-(head, set) attention kernel and the
// layer-persistent forward, so both compute the same values bit for bit.
// Attention is unscaled (no 1/sqrt(d)); a key bias of 0 keeps the score, any
// other value replaces it (masked keys -1e30, keys past the set -inf).
// Reference: unscaled_attention, cutechronos/kernel_backends.py:113-153.
#pragma once

#include <cuda_bf16.h>
#include <math.h>
#include <cstdint>

namespace cc2 {
namespace aset {

constexpr int kDH = 64;
constexpr float kMaskedScore = -1e30f;
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
// 16-byte async copy global -> shared through L2 only (coherent with writes
// of other SMs made earlier in the same kernel).
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Q, K, V tiles live in shared memory as [row][64] bf16 with 128-byte rows;
// 16-byte chunk c of row r is stored at chunk c ^ (r & 7), so ldmatrix on 8
// consecutive rows touches 8 distinct bank groups.
__device__ __forceinline__ uint32_t swz(uint32_t base, int r, int chunk) {
  return base + (uint32_t)r * 128u + ((uint32_t)(chunk ^ (r & 7)) << 4);
}

// Online softmax of query rows [q0, q0 + 16) over keys [k_lo, k_hi) in key
// tiles of KTT (qb / kb / vb: shared-memory bases of the swizzled tiles, rows
// up to the tile ends zero-filled; kbias: one bias per key row).  Leaves the
// unnormalised output o (m16n8 accumulator layout: rows lane / 4 and
// lane / 4 + 8, columns 8 dt + 2 (lane % 4) + {0, 1}), the running maxima
// m0 / m1 (log2 domain) and this lane's partial row sums l0 / l1.
template <int KTT>
__device__ __forceinline__ void tile_range(uint32_t qb, uint32_t kb, uint32_t vb, const float* kbias, int k_lo,
                                           int k_hi, int q0, int lane, float (&o)[8][4], float& m0, float& m1,
                                           float& l0, float& l1) {
  uint32_t qf[4][4];
#pragma unroll
  for (int ks = 0; ks < 4; ++ks)
    ldsm_x4(swz(qb, q0 + (lane & 15), 2 * ks + (lane >> 4)), qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3]);
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
  m0 = -INFINITY; m1 = -INFINITY; l0 = 0.0f; l1 = 0.0f;

  for (int k0 = k_lo; k0 < k_hi; k0 += KTT) {
    const int kvalid = k_hi - k0;
    float s[KTT / 8][4];
#pragma unroll
    for (int nt = 0; nt < KTT / 8; ++nt) {
      s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.0f;
      if (nt * 8 < kvalid) {
        const int kr = k0 + nt * 8 + (lane & 7);
#pragma unroll
        for (int ks = 0; ks < 4; ks += 2) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4(swz(kb, kr, 2 * ks + (lane >> 3)), b0, b1, b2, b3);
          mma16816(s[nt], qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3], b0, b1);
          mma16816(s[nt], qf[ks + 1][0], qf[ks + 1][1], qf[ks + 1][2], qf[ks + 1][3], b2, b3);
        }
      }
    }
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < KTT / 8; ++nt) {
      const int c = nt * 8 + 2 * (lane & 3);
      const float b0 = c < kvalid ? kbias[k0 + c] : -INFINITY;
      const float b1 = c + 1 < kvalid ? kbias[k0 + c + 1] : -INFINITY;
      s[nt][0] = b0 == 0.0f ? s[nt][0] * kLog2e : b0;
      s[nt][1] = b1 == 0.0f ? s[nt][1] * kLog2e : b1;
      s[nt][2] = b0 == 0.0f ? s[nt][2] * kLog2e : b0;
      s[nt][3] = b1 == 0.0f ? s[nt][3] * kLog2e : b1;
      mx0 = fmaxf(mx0, fmaxf(s[nt][0], s[nt][1]));
      mx1 = fmaxf(mx1, fmaxf(s[nt][2], s[nt][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float c0 = exp2f(m0 - mn0), c1 = exp2f(m1 - mn1);
    m0 = mn0; m1 = mn1;
    l0 *= c0; l1 *= c1;
#pragma unroll
    for (int dt = 0; dt < 8; ++dt) { o[dt][0] *= c0; o[dt][1] *= c0; o[dt][2] *= c1; o[dt][3] *= c1; }
#pragma unroll
    for (int nt = 0; nt < KTT / 8; ++nt) {
      s[nt][0] = exp2f(s[nt][0] - mn0); s[nt][1] = exp2f(s[nt][1] - mn0);
      s[nt][2] = exp2f(s[nt][2] - mn1); s[nt][3] = exp2f(s[nt][3] - mn1);
      l0 += s[nt][0] + s[nt][1];
      l1 += s[nt][2] + s[nt][3];
    }
#pragma unroll
    for (int j = 0; j < KTT / 16; ++j) {
      if (j * 16 < kvalid) {
        const uint32_t a0 = pack2(s[2 * j][0], s[2 * j][1]);
        const uint32_t a1 = pack2(s[2 * j][2], s[2 * j][3]);
        const uint32_t a2 = pack2(s[2 * j + 1][0], s[2 * j + 1][1]);
        const uint32_t a3 = pack2(s[2 * j + 1][2], s[2 * j + 1][3]);
        const int vr = k0 + 16 * j + (lane & 15);
#pragma unroll
        for (int dt = 0; dt < 8; dt += 2) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(swz(vb, vr, dt + (lane >> 4)), b0, b1, b2, b3);
          mma16816(o[dt], a0, a1, a2, a3, b0, b1);
          mma16816(o[dt + 1], a0, a1, a2, a3, b2, b3);
        }
      }
    }
  }
}

// Query rows [q0, q0 + 16) of a set of n tokens over all its keys (tiles of
// KTT), normalised; the bf16 output is staged in the tile's own Q rows and
// handed out as store(row, chunk, 16 bytes) for rows < n.
template <int KTT, typename Store>
__device__ __forceinline__ void set_tile(uint32_t qb, uint32_t kb, uint32_t vb, const float* kbias, int n, int q0,
                                         int lane, Store&& store) {
  float o[8][4];
  float m0, m1, l0, l1;
  tile_range<KTT>(qb, kb, vb, kbias, 0, n, q0, lane, o, m0, m1, l0, l1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float i0 = 1.0f / l0, i1 = 1.0f / l1;
  // stage the 16 x 64 output in this warp's own (already consumed) Q rows
  __syncwarp();
  const int r0 = q0 + (lane >> 2);
#pragma unroll
  for (int dt = 0; dt < 8; ++dt) {
    const uint32_t off = 4u * (lane & 3);
    asm volatile("st.shared.b32 [%0], %1;" ::"r"(swz(qb, r0, dt) + off), "r"(pack2(o[dt][0] * i0, o[dt][1] * i0)));
    asm volatile("st.shared.b32 [%0], %1;" ::"r"(swz(qb, r0 + 8, dt) + off), "r"(pack2(o[dt][2] * i1, o[dt][3] * i1)));
  }
  __syncwarp();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int rr = q0 + (lane >> 3) + 4 * i, c = lane & 7;
    if (rr < n) {
      uint4 v;
      asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                   : "r"(swz(qb, rr, c)));
      store(rr, c, v);
    }
  }
}

}  // namespace aset
}  // namespace cc2
