// Tensor-core INT4 group-wise GEMV building blocks shared by the decode GEMV
// kernel (gemv_mma.cu) and the persistent decode kernel (decode_persist.cu).
//
// Weight layout ("fragment tiles", built by qweight_to_mma_layout): per row
// tile t (16 rows) and group (kpg = group/16 k-steps of 16 columns):
//   codes [kpg/4][32 lanes][4] u32 - lane l's word for k-step s holds the 8
//         codes of its mma.m16n8k16 A fragment, nibbles
//         q(r0,k0) q(r1,k0) q(r0,k0+8) q(r1,k0+8) q(r0,k0+1) q(r1,k0+1)
//         q(r0,k0+9) q(r1,k0+9)   with r0 = l/4, r1 = r0+8, k0 = 16s + 2(l%4)
//   sz    [8] x {s_r0, s_r1, z_r0, z_r1} fp16 (64 B)
// so group u = t*G + g sits at byte offset u * (kpg*128 + 64): any run of
// groups is one contiguous bulk copy.
#pragma once
#include "common.cuh"

namespace n730 {

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
               "{%0,%1,%2,%3};"
               : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
               : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = gtimer();
  while (!mbar_try_wait(bar, parity))
    if (gtimer() - t0 > 2000000000ull) return false;
  return true;
}

// D = A B with C = 0 (the first k-step of a group: no accumulator zeroing)
__device__ __forceinline__ void mma16816_z(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                           uint32_t b0, uint32_t b1) {
  const float z = 0.f;
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
               "{%10,%10,%10,%10};"
               : "=f"(c[0]), "=f"(c[1]), "=f"(c[2]), "=f"(c[3])
               : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(z));
}

// Groups [0, NG) of one chunk in shared memory: straight-line code, so the NG
// groups' accumulator chains interleave.  xb[nn] points at the chunk's first
// k-step pair of x fragments (n-tile nn); sxg at the chunk's first group of Sx,
// SXS floats per group ([group][NT*8 columns] by default).  B1: only batch
// column 0 is live (acc[.][0] row g, acc[.][2] row g+8), so the other columns
// are not updated.
template <int KPG, int NT, int NG, bool B1 = false, int SXS = NT * 8>
__device__ __forceinline__ void mma_chunk(const uint8_t* buf, int lane, const uint4* const (&xb)[NT],
                                          const float* sxg, float (&acc)[NT][4]) {
  constexpr int GB = KPG * 128 + 64;
  constexpr uint32_t MAGIC = 0x64006400u;
  const int g = lane >> 2, tq = lane & 3;
#pragma unroll
  for (int gr = 0; gr < NG; ++gr) {
    const uint32_t* cw = reinterpret_cast<const uint32_t*>(buf + gr * GB) + lane * 4;
    float cg[NT][4];
#pragma unroll
    for (int kk = 0; kk < KPG; kk += 4) {
      const int kl = gr * KPG + kk;  // k-step within the chunk
      const uint4 w4 = *reinterpret_cast<const uint4*>(cw + (kk >> 2) * 128);
      const uint32_t wv[4] = {w4.x, w4.y, w4.z, w4.w};
      uint4 bx[NT][2];
#pragma unroll
      for (int nn = 0; nn < NT; ++nn) {
        bx[nn][0] = xb[nn][(kl >> 1) * 4];
        bx[nn][1] = xb[nn][((kl >> 1) + 1) * 4];
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t w = wv[j], ws = w >> 8;
        const uint32_t a0 = lop3_and_or(w, 0x000F000Fu, MAGIC);   // rows g,   k 2tq..+1:  1024 + q
        const uint32_t a1 = lop3_and_or(w, 0x00F000F0u, MAGIC);   // rows g+8, k 2tq..+1:  1024 + 16 q
        const uint32_t a2 = lop3_and_or(ws, 0x000F000Fu, MAGIC);  // rows g,   k 2tq+8..+9
        const uint32_t a3 = lop3_and_or(ws, 0x00F000F0u, MAGIC);  // rows g+8, k 2tq+8..+9
#pragma unroll
        for (int nn = 0; nn < NT; ++nn) {
          const uint4 v = bx[nn][j >> 1];
          const uint32_t b0 = (j & 1) ? v.z : v.x, b1 = (j & 1) ? v.w : v.y;
          if (kk == 0 && j == 0) mma16816_z(cg[nn], a0, a1, a2, a3, b0, b1);
          else                   mma16816(cg[nn], a0, a1, a2, a3, b0, b1);
        }
      }
    }
    // group epilogue: y += s C - s (1024 + z) Sx ; rows g+8: (s/16) C - s (64 + z) Sx
    const uint2 szv = *reinterpret_cast<const uint2*>(buf + gr * GB + KPG * 128 + g * 8);
    const float2 sf = __half22float2(u2h(szv.x)), zf = __half22float2(u2h(szv.y));
    const float m0 = sf.x, m1 = sf.y * 0.0625f;
    const float o0 = -sf.x * (1024.f + zf.x), o1 = -sf.y * (64.f + zf.y);
#pragma unroll
    for (int nn = 0; nn < NT; ++nn) {
      if (B1) {
        const float xs = sxg[gr * SXS];
        acc[nn][0] = fmaf(m0, cg[nn][0], fmaf(o0, xs, acc[nn][0]));
        acc[nn][2] = fmaf(m1, cg[nn][2], fmaf(o1, xs, acc[nn][2]));
      } else {
        const float2 xs = *reinterpret_cast<const float2*>(sxg + gr * SXS + nn * 8 + 2 * tq);
        acc[nn][0] = fmaf(m0, cg[nn][0], fmaf(o0, xs.x, acc[nn][0]));
        acc[nn][1] = fmaf(m0, cg[nn][1], fmaf(o0, xs.y, acc[nn][1]));
        acc[nn][2] = fmaf(m1, cg[nn][2], fmaf(o1, xs.x, acc[nn][2]));
        acc[nn][3] = fmaf(m1, cg[nn][3], fmaf(o1, xs.y, acc[nn][3]));
      }
    }
  }
}

// NU independent units (row tiles) of ONE group each, all against the same x
// group (xb, xs): unit i sits at buf + i * GB and accumulates into acc[i]
// (batch column 0 only: acc[i][0] row g, acc[i][2] row g+8).  The x
// fragments are loaded once per k-step pair and shared by the NU chains.
template <int KPG, int NU>
__device__ __forceinline__ void mma_units(const uint8_t* buf, int lane, const uint4* xb, float xs,
                                          float (&acc)[NU][4]) {
  constexpr int GB = KPG * 128 + 64;
  constexpr uint32_t MAGIC = 0x64006400u;
  const int g = lane >> 2;
  float cg[NU][4];
#pragma unroll
  for (int kk = 0; kk < KPG; kk += 4) {
    const uint4 bx0 = xb[(kk >> 1) * 4], bx1 = xb[((kk >> 1) + 1) * 4];
    uint4 w4[NU];
#pragma unroll
    for (int i = 0; i < NU; ++i)
      w4[i] = *reinterpret_cast<const uint4*>(buf + i * GB + lane * 16 + (kk >> 2) * 512);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 v = (j >> 1) ? bx1 : bx0;
      const uint32_t b0 = (j & 1) ? v.z : v.x, b1 = (j & 1) ? v.w : v.y;
#pragma unroll
      for (int i = 0; i < NU; ++i) {
        const uint32_t w = j == 0 ? w4[i].x : j == 1 ? w4[i].y : j == 2 ? w4[i].z : w4[i].w, ws = w >> 8;
        const uint32_t a0 = lop3_and_or(w, 0x000F000Fu, MAGIC);
        const uint32_t a1 = lop3_and_or(w, 0x00F000F0u, MAGIC);
        const uint32_t a2 = lop3_and_or(ws, 0x000F000Fu, MAGIC);
        const uint32_t a3 = lop3_and_or(ws, 0x00F000F0u, MAGIC);
        if (kk == 0 && j == 0) mma16816_z(cg[i], a0, a1, a2, a3, b0, b1);
        else                   mma16816(cg[i], a0, a1, a2, a3, b0, b1);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < NU; ++i) {
    const uint2 szv = *reinterpret_cast<const uint2*>(buf + i * GB + KPG * 128 + g * 8);
    const float2 sf = __half22float2(u2h(szv.x)), zf = __half22float2(u2h(szv.y));
    acc[i][0] = fmaf(sf.x, cg[i][0], fmaf(-sf.x * (1024.f + zf.x), xs, acc[i][0]));
    acc[i][2] = fmaf(sf.y * 0.0625f, cg[i][2], fmaf(-sf.y * (64.f + zf.y), xs, acc[i][2]));
  }
}

}  // namespace n730
