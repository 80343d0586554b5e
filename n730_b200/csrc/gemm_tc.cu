// Prefill / batched GEMM on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Y[T x N] = X[T x K] . dequant(W)[N x K]^T for INT4 group-wise weights held in
// the fragment-tiled layout of the decode GEMV (no second copy of the weights),
// with the decoder's epilogues: bias, residual add (in place), SwiGLU of
// interleaved gate/up rows, and RMSNorm folded into the A operand.
//
// A pre-pass packs x once per call (RMS-normalised, rounded to fp16) into
// 128-token x 64-column blocks already in the K-major, 128-byte-swizzled
// layout the UMMA shared-memory descriptors read (8-row x 128-byte atoms,
// 16-byte chunk c of row r at c ^ (r % 8)).  One CTA computes a 128-token x
// 128-row output tile over K in steps of 128 (one group) through a 3-stage
// pipeline of specialised warps, with no CTA-wide barrier inside the K loop:
//  * a producer warp issues, once a stage's previous MMAs have completed, one
//    bulk copy of the packed A tile and one bulk copy per 16-row tile of W
//    (the step's whole group blocks: codes and fp16 scale/zero);
//  * 8 dequant warps turn their row tile's codes into (q - z) * s fp16 values
//    in the swizzled B tile and arrive on the stage's conversion barrier;
//  * an MMA warp issues eight tcgen05.mma.kind::f16 (M 128, N 128, K 16,
//    fp32 accumulate in tensor memory) and a tcgen05.commit to the stage's
//    empty barrier, which gates that stage's next copies;
//  * after the last step the accumulator is read back with tcgen05.ld
//    (32 lanes x 32 columns per warp and instruction) and written with the
//    epilogue.
// Every mbarrier wait is bounded (%globaltimer, 2 s); a wait that runs out sets
// the device error word, stops issuing, waits (bounded) for the MMAs in
// flight, and still frees the tensor memory.
// Numerics: dequantised weights in fp16 ((q - z) s from an fp16 FMA with the
// zero-point term z s rounded to fp16), x rounded to fp16, fp32 accumulation.
#include <algorithm>

#include "mma_gemv.cuh"
#include "qweight.h"

namespace n730 {

constexpr int TC_BM = 128, TC_BN = 128, TC_BK = 128, TC_STAGES = 3;
constexpr int TC_SUB = 128 * 64 * 2;        // one 128-row x 64-column fp16 sub-tile (one 128-byte swizzle atom wide)
constexpr int TC_TILE = 2 * TC_SUB;         // A or B operand of one K-step (two sub-tiles)
constexpr int TC_RAWT = 1152;               // raw codes + scale/zero blocks of one 16-row tile per K-step
constexpr int TC_STAGE = 2 * TC_TILE + 9216;  // A | B | raw B (8 x TC_RAWT), a multiple of 1024
constexpr uint32_t TC_TMEM_COLS = 128;      // fp32 accumulator columns (N)

struct TcArgs {
  const uint8_t* blob;  // fragment tiles: group u = tile*G + g at u * (kpg*128 + 64)
  int rows, cols, G, kpg;
  const uint8_t* x16;   // packed A: [token tile][64-column block] sub-tiles of 128 x 64 fp16, 128B-swizzled
  int T;
  float* y; int ldy;
  const float* bias;
  const float* residual; int ldr;
  int swiglu;
  int* err;
};

// UMMA shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row x 128 B
// atoms stacked every 1024 B along M/N.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);  // start address, 16-byte units
  d |= (uint64_t)1 << 16;                            // leading byte offset (not used by swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;                  // stride byte offset: next 8-row atom
  d |= (uint64_t)1 << 46;                            // descriptor version
  d |= (uint64_t)2 << 61;                            // swizzle: 128 B
  return d;
}

// kind::f16 instruction descriptor: D fp32, A = B = fp16, both K-major, N = 128, M = 128.
constexpr uint32_t TC_IDESC = (1u << 4) | ((uint32_t)(TC_BN >> 3) << 17) | ((uint32_t)(TC_BM >> 4) << 24);

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
               " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}"
               :: "r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(TC_IDESC), "r"(accumulate) : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               :: "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tc_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
               "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                 "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                 "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
                 "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
                 "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// byte offset of element (row r, column k) in a K-major 128B-swizzled tile (64 fp16 per row)
__device__ __forceinline__ uint32_t sw128(int r, int k) {
  return (uint32_t)(r * 128 + ((((k >> 3) ^ (r & 7)) & 7) << 4) + ((k & 7) << 1));
}

// A operand packing: x [T][ldx] (RMS-normalised with inv_rms and norm_w when
// given) -> fp16 blocks of 128 tokens x 64 columns, each laid out exactly as
// the GEMM's shared-memory A tile (row r: 128 bytes, 16-byte chunk c at
// c ^ (r % 8)); tokens >= T are zero.  Grid (K / 64, token tiles).
__global__ void x16_pack_kernel(const float* x, int ldx, int T, const float* inv_rms, const float* norm_w,
                                uint8_t* out) {
  const int kb = blockIdx.x, tt = blockIdx.y;
  uint8_t* blk = out + ((size_t)tt * gridDim.x + kb) * TC_SUB;
  for (int i = threadIdx.x; i < TC_BM * 8; i += blockDim.x) {
    const int r = i >> 3, c8 = i & 7, tok = tt * TC_BM + r, k = kb * 64 + c8 * 8;
    uint4 pk = make_uint4(0u, 0u, 0u, 0u);
    if (tok < T) {
      const float4* src = reinterpret_cast<const float4*>(x + (int64_t)tok * ldx + k);
      float4 a = src[0], b = src[1];
      if (inv_rms) {
        const float iv = inv_rms[tok];
        const float4* nw = reinterpret_cast<const float4*>(norm_w + k);
        const float4 na = nw[0], nb = nw[1];
        a.x *= iv * na.x; a.y *= iv * na.y; a.z *= iv * na.z; a.w *= iv * na.w;
        b.x *= iv * nb.x; b.y *= iv * nb.y; b.z *= iv * nb.z; b.w *= iv * nb.w;
      }
      pk = make_uint4(h2u(__floats2half2_rn(a.x, a.y)), h2u(__floats2half2_rn(a.z, a.w)),
                      h2u(__floats2half2_rn(b.x, b.y)), h2u(__floats2half2_rn(b.z, b.w)));
    }
    *reinterpret_cast<uint4*>(blk + r * 128 + ((c8 ^ (r & 7)) << 4)) = pk;
  }
}

// Bounded mbarrier wait that also gives up when another role raised the
// CTA's abort flag; raises it itself after 2 s.
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, volatile int* abortf) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = gtimer();
  while (!mbar_try_wait(bar, parity)) {
    if (*abortf) return false;
    if (gtimer() - t0 > 2000000000ull) { *abortf = 1; return false; }
  }
  return true;
}
__device__ __forceinline__ void mbar_arrive1(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" :: "r"(smem_u32(bar)) : "memory");
}

// One CTA per 128-token x 128-row output tile; K in steps of 128 through a
// 3-stage pipeline with specialised warps and no CTA-wide barrier in the loop:
//  * warp 8 (producer): once a stage's MMAs are done (empty[s]) it issues the
//    next step's bulk copies into it (the packed A tile, 32 KB; per 16-row tile
//    of W the step's codes with their scale/zero blocks, one copy when the
//    step covers whole groups) -> full[s];
//  * warps 0-7 (dequant, then epilogue): warp w waits for full[s], turns row
//    tile w's codes into (q - z) * s fp16 in the swizzled B tile and arrives on
//    conv[s];
//  * warp 9 (MMA): waits for conv[s], issues four tcgen05.mma.kind::f16 and
//    commits them to empty[s]; after the last step, to `done`.
constexpr int TC_WARPS = 10;

__global__ void __launch_bounds__(TC_WARPS * 32, 1) gemm_tc_kernel(const TcArgs p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + TC_STAGES * TC_STAGE);  // [STAGES] copies landed
  uint64_t* conv = full + TC_STAGES;                                           // [STAGES] B tile converted
  uint64_t* empty = conv + TC_STAGES;                                          // [STAGES] MMAs done
  uint64_t* done = empty + TC_STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abortf = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* counts = const_cast<int*>(abortf) + 1;  // [0] steps produced, [1] steps issued, [2] result ok
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n0 = blockIdx.x * TC_BN, tt = blockIdx.y, m0 = tt * TC_BM;
  const int GB = p.kpg * 128 + 64;
  const int n_tiles = (p.rows + 15) >> 4, tile0 = n0 >> 4;
  const int nt_here = min(8, n_tiles - tile0);  // 16-row tiles of W in this CTA's B (>= 1)
  // per 16-row tile and K-step: whole groups (kpg <= 8: 8/kpg contiguous group
  // blocks) or, for kpg 16, half a group's codes plus its scale/zero block
  const int gps = p.kpg <= 8 ? 8 / p.kpg : 1;                  // groups touched per step
  const uint32_t raw_b = p.kpg <= 8 ? (uint32_t)(gps * GB) : 1088u;
  const uint32_t stage_tx = (uint32_t)TC_TILE + (uint32_t)nt_here * raw_b;
  const int KT = p.cols / TC_BK;

  if (tid == 0) {
    for (int s = 0; s < TC_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 8);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    fence_mbar_init();
    *abortf = 0;
    counts[0] = counts[1] = counts[2] = 0;
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(tmem_slot)), "r"(TC_TMEM_COLS) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    // ---------------- producer ----------------
    if (lane == 0) {
      int kt = 0;
      for (; kt < KT; ++kt) {
        const int s = kt % TC_STAGES;
        if (kt >= TC_STAGES && !tc_wait(&empty[s], (uint32_t)(((kt / TC_STAGES) - 1) & 1), abortf)) break;
        uint8_t* st = smem + s * TC_STAGE;
        mbar_arrive_expect_tx(&full[s], stage_tx);
        bulk_g2s(st, p.x16 + ((size_t)tt * KT + kt) * TC_TILE, TC_TILE, &full[s]);
        const int s0 = kt * 8, gi = s0 / p.kpg;  // first k-step and group of this step
        for (int w = 0; w < nt_here; ++w) {
          const uint8_t* grp = p.blob + ((int64_t)(tile0 + w) * p.G + gi) * GB;
          uint8_t* dst = st + 2 * TC_TILE + w * TC_RAWT;
          if (p.kpg <= 8) {
            bulk_g2s(dst, grp, raw_b, &full[s]);
          } else {  // half of a 16-k-step group: quads 2h, 2h+1, then the group's scale/zero block
            bulk_g2s(dst, grp + ((s0 % 16) >> 3) * 1024, 1024, &full[s]);
            bulk_g2s(dst + 1024, grp + 16 * 128, 64, &full[s]);
          }
        }
      }
      counts[0] = kt;
    }
  } else if (warp == 9) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int kt = 0;
      for (; kt < KT; ++kt) {
        const int s = kt % TC_STAGES;
        if (!tc_wait(&conv[s], (uint32_t)((kt / TC_STAGES) & 1), abortf)) break;
        tc_fence_after();
        const uint32_t a0 = smem_u32(smem + s * TC_STAGE), b0 = a0 + TC_TILE;
#pragma unroll
        for (int j = 0; j < TC_BK / 16; ++j) {  // K = 16 per MMA: 32 bytes along the swizzled row of a sub-tile
          const uint32_t off = (uint32_t)((j >> 2) * TC_SUB + (j & 3) * 32);
          tc_mma(tmem, umma_desc_sw128(a0 + off), umma_desc_sw128(b0 + off), (kt > 0 || j > 0) ? 1u : 0u);
        }
        tc_commit(&empty[s]);
      }
      counts[1] = kt;
      if (kt > 0) {
        tc_commit(done);
        // every MMA must be complete before the accumulator is read or freed (bounded, even on abort)
        const bool ok = wait_bar(done, 0);
        counts[2] = ok && kt == KT && !*abortf;
        if (!ok) *abortf = 1;
      }
    }
  } else {
    // ---------------- dequant warps 0-7: row tile `warp` of the B tile ----------------
    const int r0 = warp * 16 + (lane >> 2), r1 = r0 + 8;
    const int kb = 2 * (lane & 3);
    for (int kt = 0; kt < KT; ++kt) {
      const int s = kt % TC_STAGES;
      int ok = 1;
      if (lane == 0) ok = tc_wait(&full[s], (uint32_t)((kt / TC_STAGES) & 1), abortf);
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      uint8_t* st = smem + s * TC_STAGE;
      uint8_t* bs = st + TC_TILE;
#pragma unroll
      for (int h = 0; h < 2; ++h) {  // quad h: k-steps 4h..4h+3 of the step -> sub-tile h of B
        uint8_t* sb = bs + h * TC_SUB;
        if (warp < nt_here) {
          const uint8_t* raw = st + 2 * TC_TILE + warp * TC_RAWT;
          // kpg 4: [quad | sz] per group; kpg 8 and 16: [quad 0 | quad 1 | sz]
          const int qoff = p.kpg == 4 ? h * 576 : h * 512, zoff = p.kpg == 4 ? h * 576 + 512 : 1024;
          const uint4 w4 = *reinterpret_cast<const uint4*>(raw + qoff + lane * 16);
          const uint2 szv = *reinterpret_cast<const uint2*>(raw + zoff + (lane >> 2) * 8);
          const float2 sc = __half22float2(u2h(szv.x)), zp = __half22float2(u2h(szv.y));
          // (q - z) s in fp16: the code nibble ORed into fp16 1024 (low nibbles) or 64 (bits 4-7)
          // gives 1024 + q / 64 + q exactly, one subtraction gives q, one FMA q s - z s (z s
          // rounded to fp16 once: <= 2^-12 relative of z s per weight)
          const __half2 s0 = __float2half2_rn(sc.x), s1 = __float2half2_rn(sc.y);
          const __half2 c0 = __float2half2_rn(-zp.x * sc.x), c1 = __float2half2_rn(-zp.y * sc.y);
          const __half2 k1024 = u2h(0x64006400u), k64 = u2h(0x54005400u);
          const uint32_t wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t w = wv[j], ws = w >> 8;
            const int k0 = j * 16 + kb;
            const __half2 q0 = __hsub2(u2h(lop3_and_or(w, 0x000F000Fu, 0x64006400u)), k1024);   // r0, k0 / k0+1
            const __half2 q1 = __hsub2(u2h(lop3_and_or(w, 0x00F000F0u, 0x54005400u)), k64);     // r1, k0 / k0+1
            const __half2 q2 = __hsub2(u2h(lop3_and_or(ws, 0x000F000Fu, 0x64006400u)), k1024);  // r0, k0+8 / +9
            const __half2 q3 = __hsub2(u2h(lop3_and_or(ws, 0x00F000F0u, 0x54005400u)), k64);    // r1, k0+8 / +9
            *reinterpret_cast<uint32_t*>(sb + sw128(r0, k0)) = h2u(__hfma2(q0, s0, c0));
            *reinterpret_cast<uint32_t*>(sb + sw128(r1, k0)) = h2u(__hfma2(q1, s1, c1));
            *reinterpret_cast<uint32_t*>(sb + sw128(r0, k0 + 8)) = h2u(__hfma2(q2, s0, c0));
            *reinterpret_cast<uint32_t*>(sb + sw128(r1, k0 + 8)) = h2u(__hfma2(q3, s1, c1));
          }
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int k0 = j * 16 + kb;
            *reinterpret_cast<uint32_t*>(sb + sw128(r0, k0)) = 0u;
            *reinterpret_cast<uint32_t*>(sb + sw128(r1, k0)) = 0u;
            *reinterpret_cast<uint32_t*>(sb + sw128(r0, k0 + 8)) = 0u;
            *reinterpret_cast<uint32_t*>(sb + sw128(r1, k0 + 8)) = 0u;
          }
        }
      }
      // generic-proxy shared-memory writes -> visible to the tensor core's (async proxy) reads
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive1(&conv[s]);
    }
  }
  __syncthreads();
  // copies still in flight (abort path) land before the CTA exits
  if (tid == 8 * 32)
    for (int q = counts[1]; q < counts[0]; ++q)
      wait_bar(&full[q % TC_STAGES], (uint32_t)((q / TC_STAGES) & 1));
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (*abortf && tid == 0) atomicExch(p.err, DEV_ERR_TIMEOUT);
  if (counts[2] && warp < 8) {
    // ---- epilogue: warp w reads TMEM lanes 32*(w%4).. (tokens), columns 64*(w/4).. (rows) ----
    const int qd = warp & 3, half = warp >> 2;
    const int m = qd * 32 + lane, tok = m0 + m;
#pragma unroll 1
    for (int c = 0; c < 2; ++c) {
      const int col0 = half * 64 + c * 32;
      float v[32];
      tc_ld32(tmem + ((uint32_t)(qd * 32) << 16) + (uint32_t)col0, v);
      if (tok < p.T) {
        if (p.swiglu) {
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const int n = n0 + col0 + i;
            if (n + 1 < p.rows) {
              const float gt = v[i] + (p.bias ? p.bias[n] : 0.f);
              const float up = v[i + 1] + (p.bias ? p.bias[n + 1] : 0.f);
              p.y[(int64_t)tok * p.ldy + (n >> 1)] = (gt / (1.0f + expf(-gt))) * up;
            }
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int n = n0 + col0 + i;
            if (n < p.rows) {
              float o = v[i] + (p.bias ? p.bias[n] : 0.f);
              if (p.residual) o += p.residual[(int64_t)tok * p.ldr + n];
              p.y[(int64_t)tok * p.ldy + n] = o;
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(TC_TMEM_COLS) : "memory");
}

// per-token 1/rms of x [T][ldx] over K columns: one warp per token
__global__ void inv_rms_kernel(const float* x, int ldx, int T, int K, float eps, float* out) {
  const int tok = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (tok >= T) return;
  const float* r = x + (int64_t)tok * ldx;
  float ss = 0.f;
  for (int k = lane * 4; k < K; k += 128) {
    const float4 v = *reinterpret_cast<const float4*>(r + k);
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  ss = warp_sum(ss);
  if (lane == 0) out[tok] = rsqrtf(ss / K + eps);
}

int* gemv_err_word();

constexpr size_t TC_SMEM = 1024 + (size_t)TC_STAGES * TC_STAGE + (3 * TC_STAGES + 1) * 8 + 32;

// One-time kernel attribute set-up (call before any stream capture).
int gemm_tc_prepare() {
  return smem_attr_once<gemm_tc_kernel>((int)TC_SMEM);
}

bool gemm_tc_supported(const QWeight& w, int T) {
  const int kpg = w.group / 16;
  return w.layout == 1 && w.bits == 4 && w.cols % TC_BK == 0 && (kpg == 4 || kpg == 8 || kpg == 16) && T >= 1;
}

// Packed-A workspace of the current device, grown on demand (never inside a stream capture).
static int x16_workspace(size_t bytes, cudaStream_t st, uint8_t** out) {
  static uint8_t* buf[64] = {};
  static size_t cap[64] = {};
  int dev = 0;
  N730_CUDA(cudaGetDevice(&dev));
  N730_REQUIRE(dev >= 0 && dev < 64, N730_BAD_ARG, "gemm_tc: device %d", dev);
  if (cap[dev] < bytes) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    N730_CUDA(cudaStreamIsCapturing(st, &cs));
    N730_REQUIRE(cs == cudaStreamCaptureStatusNone, N730_STATE,
                 "gemm_tc: packed-A workspace must grow outside stream capture (%zu bytes)", bytes);
    N730_CUDA(cudaStreamSynchronize(st));  // a kernel in flight may still read the old buffer
    if (buf[dev]) N730_CUDA(cudaFree(buf[dev]));
    buf[dev] = nullptr;
    cap[dev] = 0;
    N730_CUDA(cudaMalloc(&buf[dev], bytes));
    cap[dev] = bytes;
  }
  *out = buf[dev];
  return N730_OK;
}

int gemm_tc_launch(const GemvArgs& a, float* inv_ws, cudaStream_t st) {
  const QWeight& w = *a.w;
  N730_REQUIRE(gemm_tc_supported(w, a.batch), N730_UNSUPPORTED, "gemm_tc: needs INT4 fragment tiles, K %% 64 == 0");
  N730_REQUIRE(!a.swiglu || w.rows % 2 == 0, N730_BAD_ARG, "gemm_tc: swiglu needs even rows");
  N730_REQUIRE(((uintptr_t)a.x & 15) == 0 && a.ldx % 4 == 0, N730_BAD_ARG, "gemm_tc: x must be 16-byte aligned");
  N730_REQUIRE(!a.norm_w || (inv_ws && ((uintptr_t)a.norm_w & 15) == 0), N730_BAD_ARG,
               "gemm_tc: RMSNorm needs a workspace of batch floats and 16-byte aligned weights");
  int* err = gemv_err_word();
  N730_REQUIRE(err, N730_OOM, "gemm_tc: error word allocation failed");
  if (int rc = gemm_tc_prepare()) return rc;
  const int TT = (a.batch + TC_BM - 1) / TC_BM, KB = w.cols / 64;
  uint8_t* x16 = nullptr;
  if (int rc = x16_workspace((size_t)TT * KB * TC_SUB, st, &x16)) return rc;
  if (a.norm_w) {
    inv_rms_kernel<<<(a.batch + 7) / 8, 256, 0, st>>>(a.x, a.ldx, a.batch, w.cols, a.eps, inv_ws);
    N730_CHECK_LAUNCH();
  }
  x16_pack_kernel<<<dim3(KB, TT), 256, 0, st>>>(a.x, a.ldx, a.batch, a.norm_w ? inv_ws : nullptr, a.norm_w, x16);
  N730_CHECK_LAUNCH();
  TcArgs p = {};
  p.blob = w.codes; p.rows = w.rows; p.cols = w.cols; p.G = w.n_groups; p.kpg = w.group / 16;
  p.x16 = x16; p.T = a.batch;
  p.y = a.y; p.ldy = a.ldy; p.bias = a.bias; p.residual = a.residual; p.ldr = a.ldr; p.swiglu = a.swiglu;
  p.err = err;
  const dim3 grid((w.rows + TC_BN - 1) / TC_BN, TT);
  gemm_tc_kernel<<<grid, TC_WARPS * 32, TC_SMEM, st>>>(p);
  N730_CHECK_LAUNCH();
  return N730_OK;
}

}  // namespace n730
