// Prefill / batched GEMM on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Y[T x N] = X[T x K] . dequant(W)[N x K]^T for INT4 group-wise weights held in
// the fragment-tiled layout of the decode GEMV (no second copy of the weights),
// with the decoder's epilogues: bias, residual add (in place), SwiGLU of
// interleaved gate/up rows, and RMSNorm folded into the x operand.
//
// A pre-pass packs x once per call (RMS-normalised, rounded to fp16) into
// 128-token x 64-column blocks already in the K-major, 128-byte-swizzled
// layout the UMMA shared-memory descriptors read (8-row x 128-byte atoms,
// 16-byte chunk c of row r at c ^ (r % 8)).  One CTA computes a 128-row x
// NTOK-token output tile (NTOK 256 for prefill, or 128 when 256-token tiles
// would leave SMs idle; 32 / 64 / 128 for decode batches, with K split over
// blockIdx.z and a fold kernel when the grid would leave SMs idle) over K in
// steps of 128 through a pipeline of specialised warps, with no CTA-wide
// barrier inside the K loop:
//  * a producer warp issues, once a stage's previous MMAs have completed, the
//    bulk copies of the step's x blocks (NTOK x 128 fp16) and one 2-D tensor
//    copy of the step's whole group blocks (codes and fp16 scale/zero) of all
//    8 row tiles (the per-copy cost of 8 small copies bounded the step rate);
//    the first stages' weight copies go out before the programmatic
//    dependent-launch wait, since weights do not depend on the previous kernel;
//  * 8 dequant warps turn the codes into (q - z) * s fp16 and store them
//    straight into tensor memory (tcgen05.st, one W row per TMEM lane, two
//    fp16 per 32-bit column): the weights are the MMA's A operand, read from
//    TMEM, so the converted tile never goes through shared memory, and each
//    dequantised weight serves NTOK tokens;
//  * an MMA warp issues eight tcgen05.mma.kind::f16 (A from TMEM, B = x from
//    shared memory; M 128, N NTOK, K 16; fp32 accumulator in TMEM) and a
//    tcgen05.commit to the stage's empty barrier, which gates that stage's
//    next copies and next conversion;
//  * after the last step the accumulator (TMEM lane = W row, column = token)
//    is read back with tcgen05.ld and written with the epilogue, each warp
//    instruction storing 32 consecutive rows of one token.
// Every mbarrier wait is bounded (%globaltimer, 2 s); a wait that runs out sets
// the device error word, stops issuing, waits (bounded) for the MMAs in
// flight, and still frees the tensor memory.
// Numerics: dequantised weights in fp16 ((q - z) s from an fp16 FMA with the
// zero-point term z s rounded to fp16), x rounded to fp16, fp32 accumulation.
#include <algorithm>
#include <cstring>
#include <mutex>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "mma_gemv.cuh"
#include "qweight.h"

namespace n730 {

constexpr int TC_BN = 128;                  // W rows per CTA: the MMA's M, one per TMEM lane
constexpr int TC_BK = 128;                  // K per pipeline step
constexpr int TC_XT = 128;                  // tokens per packed x sub-tile
constexpr int TC_SUB = TC_XT * 64 * 2;      // one 128-token x 64-column fp16 sub-tile (one swizzle atom wide)
constexpr int TC_RAWT = 1152;               // raw codes + scale/zero blocks of one 16-row tile per K-step
constexpr int TC_RAW = 8 * TC_RAWT;         // raw W of one step (8 row tiles), a multiple of 1024
constexpr int TC_ACOLS = TC_BK / 2;         // TMEM columns of one step's A (two fp16 per column)
// TMEM per CTA: the accumulator (NTOK columns) + one A block per stage, rounded to 256 or 512

template <int NTOK>
struct TcCfg {
  // pipeline depth within shared memory and TMEM; 32- and 64-token tiles (decode batches) take
  // 3 stages in 256 TMEM columns, so two CTAs (two pipelines) share an SM: measured at 32 tokens,
  // 7 stages in 512 columns (one CTA per SM) ran gate|up in 46 us, this 37 us
  static constexpr int STAGES = NTOK == 256 ? 3 : NTOK == 128 ? 4 : 3;
  static constexpr uint32_t TMEM = NTOK + STAGES * TC_ACOLS <= 256 ? 256u : 512u;  // columns allocated
  static constexpr int XB = NTOK * TC_BK * 2;  // x bytes per step: [64-column block][NTOK rows][128 B]
  static constexpr int XR = NTOK < TC_XT ? NTOK : TC_XT;  // token rows per x copy (one packed sub-tile at most)
  static constexpr int STAGE = XB + TC_RAW;    // a multiple of 1024 (swizzle atoms stay aligned)
  static constexpr size_t SMEM = 1024 + (size_t)STAGES * STAGE + (3 * STAGES + 1) * 8 + 32;
  // kind::f16 instruction descriptor: D fp32, A = B = fp16, both K-major, N = NTOK, M = 128
  static constexpr uint32_t IDESC = (1u << 4) | ((uint32_t)(NTOK >> 3) << 17) | ((uint32_t)(TC_BN >> 4) << 24);
  static_assert(NTOK + STAGES * TC_ACOLS <= (int)TMEM, "tensor memory budget");
  static_assert(STAGE % 1024 == 0, "stage alignment");
};

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
  int wtma;             // 1: the step's W blocks of all 8 row tiles come in one 2-D tensor copy (wmap)
  int kparts;           // K split over blockIdx.z (1: none); with part, raw sums go to part[z][token][row]
  float* part;
  int64_t part_stride;
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

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem_d] (+)= A[tmem_a] . B[bdesc]^T with A in tensor memory (lane = row,
// two fp16 per 32-bit column) and B in shared memory.
template <uint32_t IDESC>
__device__ __forceinline__ void tc_mma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t accumulate) {
  asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
               " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}"
               :: "r"(tmem_d), "r"(tmem_a), "l"(bdesc), "r"(IDESC), "r"(accumulate) : "memory");
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

// 32 consecutive 32-bit columns of this thread's TMEM lane (the warp's 32 lanes)
__device__ __forceinline__ void tc_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
               "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
               :: "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
                  "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
                  "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
                  "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
               : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 2-D tiled tensor copy (no multicast) of the box at element coordinates (c0, c1)
// into shared memory, completing on `bar`
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
               :: "r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
               : "memory");
}

// x operand packing: x [T][ldx] (RMS-normalised with norm_w when given, 1/rms
// from inv_rms or from ss: ss_parts sums of squares per token that the split-K
// fold which wrote x left behind, added in order) -> fp16 blocks of 128 tokens
// x 64 columns, each laid out exactly as a 128-token slice of the GEMM's
// shared-memory x block (row r: 128 bytes, 16-byte chunk c at c ^ (r % 8));
// tokens >= T are zero.  Grid (K / 64, token sub-tiles).
__global__ void x16_pack_kernel(const float* x, int ldx, int T, const float* inv_rms, const float* ss, int ss_parts,
                                int K, float eps, const float* norm_w, uint8_t* out) {
  __shared__ float siv[TC_XT];
  const int kb = blockIdx.x, tt = blockIdx.y;
  uint8_t* blk = out + ((size_t)tt * gridDim.x + kb) * TC_SUB;
  pdl_wait();  // x (and inv_rms / ss) come from the previous kernels
  pdl_launch_dependents();
  if (ss) {
    for (int r = threadIdx.x; r < TC_XT; r += blockDim.x) {
      const int tok = tt * TC_XT + r;
      float t = 0.f;
      if (tok < T)
        for (int j = 0; j < ss_parts; ++j) t += ss[(int64_t)tok * ss_parts + j];
      siv[r] = rsqrtf(t / K + eps);
    }
    __syncthreads();
  }
  for (int i = threadIdx.x; i < TC_XT * 8; i += blockDim.x) {
    const int r = i >> 3, c8 = i & 7, tok = tt * TC_XT + r, k = kb * 64 + c8 * 8;
    uint4 pk = make_uint4(0u, 0u, 0u, 0u);
    if (tok < T) {
      const float4* src = reinterpret_cast<const float4*>(x + (int64_t)tok * ldx + k);
      float4 a = src[0], b = src[1];
      if (norm_w) {
        const float iv = ss ? siv[r] : inv_rms[tok];
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

// One CTA per 128-row x NTOK-token output tile; K in steps of 128 through a
// pipeline of specialised warps with no CTA-wide barrier in the loop:
//  * warp 8 (producer): once a stage's MMAs are done (empty[s]) it issues the
//    next step's bulk copies into it (the x blocks of the step, NTOK x 128
//    fp16; per 16-row tile of W the step's codes with their scale/zero
//    blocks, one copy when the step covers whole groups) -> full[s];
//  * warps 0-7 (dequant, then epilogue): warp w owns TMEM lanes 32(w%4).. (W
//    rows) and K half w/4 of each step; it waits for full[s], writes its 32
//    rows x 64 dequantised fp16 into stage s's A columns with one tcgen05.st
//    and arrives on conv[s];
//  * warp 9 (MMA): waits for conv[s], issues eight tcgen05.mma.kind::f16 (A in
//    TMEM, B = x in shared memory) and commits them to empty[s]; after the last
//    step, to `done`.
// full[s] of a step is only raised after the producer saw empty[s] of the
// step that last used stage s, so the dequant warps never overwrite an A block
// the tensor core is still reading.
constexpr int TC_WARPS = 10;

template <int NTOK>
__global__ void __launch_bounds__(TC_WARPS * 32, NTOK <= 64 ? 2 : 1)
gemm_tc_kernel(const TcArgs p, const __grid_constant__ CUtensorMap wmap) {
  using Cfg = TcCfg<NTOK>;
  constexpr int S = Cfg::STAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * Cfg::STAGE);  // [S] copies landed
  uint64_t* conv = full + S;                                             // [S] A block in TMEM
  uint64_t* empty = conv + S;                                            // [S] MMAs done
  uint64_t* done = empty + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abortf = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* counts = const_cast<int*>(abortf) + 1;  // [0] steps produced, [1] steps issued, [2] result ok
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n0 = blockIdx.x * TC_BN, m0 = blockIdx.y * NTOK;
  const int KB = p.cols / 64;                   // packed 64-column blocks per sub-tile
  const int GB = p.kpg * 128 + 64;
  const int n_tiles = (p.rows + 15) >> 4, tile0 = n0 >> 4;
  const int nt_here = min(8, n_tiles - tile0);  // 16-row tiles of W in this CTA (>= 1)
  // per 16-row tile and K-step: whole groups (kpg <= 8: 8/kpg contiguous group
  // blocks) or, for kpg 16, half a group's codes plus its scale/zero block
  const int gps = p.kpg <= 8 ? 8 / p.kpg : 1;                  // groups touched per step
  const uint32_t raw_b = p.kpg <= 8 ? (uint32_t)(gps * GB) : 1088u;
  // the tensor copy always delivers its whole 8-row box (rows past the weight read as zeros)
  const uint32_t stage_tx = (uint32_t)Cfg::XB + (uint32_t)(p.wtma ? 8 : nt_here) * raw_b;
  const int rstride = p.wtma ? (int)raw_b : TC_RAWT;  // shared-memory bytes per row tile of raw W
  // this CTA's K-part: steps [k0, k0 + KT) of the row (kparts 1: all of them)
  const int kz = blockIdx.z, KT_all = p.cols / TC_BK;
  const int k0 = KT_all * kz / p.kparts, KT = KT_all * (kz + 1) / p.kparts - k0;

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
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
                 :: "r"(smem_u32(tmem_slot)), "r"(Cfg::TMEM) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;  // accumulator: columns [0, NTOK); A block of stage s at NTOK + s * TC_ACOLS

  if (warp == 8) {
    // ---------------- producer ----------------
    if (lane == 0) {
      // step kt's x blocks: 64-column block h holds NTOK rows, copied XR rows (<= one packed
      // sub-tile, row r of a sub-tile at byte 128 r) at a time
      auto issue_x = [&](int s, int kt) {
        uint8_t* st = smem + s * Cfg::STAGE;
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int i = 0; i < NTOK / Cfg::XR; ++i) {
            const int tok = m0 + i * Cfg::XR;
            bulk_g2s(st + h * (NTOK * 128) + i * Cfg::XR * 128,
                     p.x16 + ((size_t)(tok / TC_XT) * KB + 2 * (k0 + kt) + h) * TC_SUB + (size_t)(tok % TC_XT) * 128,
                     Cfg::XR * 128, &full[s]);
          }
      };
      // step kt's weight blocks of the CTA's row tiles
      auto issue_w = [&](int s, int kt) {
        uint8_t* st = smem + s * Cfg::STAGE;
        const int s0 = (k0 + kt) * 8, gi = s0 / p.kpg;  // first k-step and group of this step
        if (p.wtma) {  // one copy: row tiles [tile0, tile0 + 8) x the step's raw_b bytes from group gi
          tma_load_2d(st + Cfg::XB, &wmap, gi * GB / 8, tile0, &full[s]);
          return;
        }
        for (int w = 0; w < nt_here; ++w) {
          const uint8_t* grp = p.blob + ((int64_t)(tile0 + w) * p.G + gi) * GB;
          uint8_t* dst = st + Cfg::XB + w * TC_RAWT;
          if (p.kpg <= 8) {
            bulk_g2s(dst, grp, raw_b, &full[s]);
          } else {  // half of a 16-k-step group: quads 2h, 2h+1, then the group's scale/zero block
            bulk_g2s(dst, grp + ((s0 % 16) >> 3) * 1024, 1024, &full[s]);
            bulk_g2s(dst + 1024, grp + 16 * 128, 64, &full[s]);
          }
        }
      };
      // weights do not depend on the previous kernel (programmatic dependent launch): the first
      // stages' weight copies go out before the grid-dependency wait, their x copies after it
      const int pre = min(S, KT);
      for (int j = 0; j < pre; ++j) {
        mbar_arrive_expect_tx(&full[j], stage_tx);
        issue_w(j, j);
      }
      pdl_wait();
      int kt = 0;
      for (; kt < KT; ++kt) {
        const int s = kt % S;
        if (kt >= S) {
          if (!tc_wait(&empty[s], (uint32_t)(((kt / S) - 1) & 1), abortf)) break;
          mbar_arrive_expect_tx(&full[s], stage_tx);
          issue_w(s, kt);
        }
        issue_x(s, kt);
      }
      counts[0] = kt;
    }
  } else if (warp == 9) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int kt = 0;
      for (; kt < KT; ++kt) {
        const int s = kt % S;
        if (!tc_wait(&conv[s], (uint32_t)((kt / S) & 1), abortf)) break;
        tc_fence_after();
        const uint32_t b0 = smem_u32(smem + s * Cfg::STAGE);
        const uint32_t a0 = tmem + (uint32_t)(NTOK + s * TC_ACOLS);
#pragma unroll
        for (int j = 0; j < TC_BK / 16; ++j) {  // K = 16 per MMA: 8 TMEM columns of A, 32 bytes along x's swizzled rows
          const uint32_t boff = (uint32_t)((j >> 2) * (NTOK * 128) + (j & 3) * 32);
          tc_mma_ts<Cfg::IDESC>(tmem, a0 + (uint32_t)(j * 8), umma_desc_sw128(b0 + boff), (kt > 0 || j > 0) ? 1u : 0u);
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
    // ---------------- dequant warps 0-7: W row 32 (w % 4) + lane, K half w / 4 ----------------
    const int q = warp & 3, h = warp >> 2;
    const int r = 32 * q + lane, wt = r >> 4, g = r & 7, hi = (r >> 3) & 1;
    // row g of the 16-row tile sits in the low nibbles of its fragment words, row g + 8 in the high ones
    const uint32_t msk = hi ? 0x00F000F0u : 0x000F000Fu, mag = hi ? 0x54005400u : 0x64006400u;
    const __half2 kmag = u2h(mag);  // fp16 64 or 1024: the value the magic bits stand for
    const int qoff = p.kpg == 4 ? h * 576 : h * 512, zoff = p.kpg == 4 ? h * 576 + 512 : 1024;
    const uint32_t ta = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(NTOK + h * 32);
    for (int kt = 0; kt < KT; ++kt) {
      const int s = kt % S;
      int ok = 1;
      if (lane == 0) ok = tc_wait(&full[s], (uint32_t)((kt / S) & 1), abortf);
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      tc_fence_after();
      const uint8_t* raw = smem + s * Cfg::STAGE + Cfg::XB + wt * rstride;
      uint32_t out[32];
      if (wt < nt_here) {
        // column c of the half: K pair (16 j + 2 tq (+ 8), +1) for c = 8 j + tq (+ 4), from
        // word j of fragment lane 4 g + tq (8 nibbles: rows g / g + 8, K 2tq, 2tq+1, 2tq+8, 2tq+9)
        const uint2 szv = *reinterpret_cast<const uint2*>(raw + zoff + g * 8);
        const float2 sc = __half22float2(u2h(szv.x)), zp = __half22float2(u2h(szv.y));
        const float sv = hi ? sc.y : sc.x, zv = hi ? zp.y : zp.x;
        // (q - z) s in fp16: the nibble ORed into the magic gives magic + q exactly, one
        // subtraction gives q, one FMA q s - z s (z s rounded to fp16 once)
        const __half2 s2 = __float2half2_rn(sv), c2 = __float2half2_rn(-zv * sv);
        const uint4* src = reinterpret_cast<const uint4*>(raw + qoff + g * 64);
#pragma unroll
        for (int tq = 0; tq < 4; ++tq) {
          const uint4 w4 = src[tq];
          const uint32_t wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            out[8 * j + tq] = h2u(__hfma2(__hsub2(u2h(lop3_and_or(wv[j], msk, mag)), kmag), s2, c2));
            out[8 * j + 4 + tq] = h2u(__hfma2(__hsub2(u2h(lop3_and_or(wv[j] >> 8, msk, mag)), kmag), s2, c2));
          }
        }
      } else {
#pragma unroll
        for (int c = 0; c < 32; ++c) out[c] = 0u;
      }
      tc_st32(ta + (uint32_t)(s * TC_ACOLS), out);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive1(&conv[s]);
    }
  }
  pdl_launch_dependents();  // the next kernel may launch; it waits for this grid before reading y
  __syncthreads();
  // copies still in flight (abort path) land before the CTA exits
  if (tid == 8 * 32)
    for (int qq = counts[1]; qq < counts[0]; ++qq)
      wait_bar(&full[qq % S], (uint32_t)((qq / S) & 1));
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (*abortf && tid == 0) atomicExch(p.err, DEV_ERR_TIMEOUT);
  if (counts[2] && warp < 8) {
    pdl_wait();  // y / residual may be in use by the kernels before this one until they complete
    // ---- epilogue: warp w reads TMEM lanes 32 (w % 4).. (W rows), token columns 32 c.. for c = w / 4, + 2, ... ----
    const int q = warp & 3, hh = warp >> 2;
    const int n = n0 + 32 * q + lane;
    const bool nin = n < p.rows;
    const float bv = p.bias && nin ? p.bias[n] : 0.f;
#pragma unroll 1
    for (int c = hh; c < NTOK / 32; c += 2) {
      const int col0 = c * 32;
      float v[32];
      tc_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)col0, v);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int tok = m0 + col0 + i;
        if (tok >= p.T) break;  // warp-uniform
        if (p.part) {  // split K: this part's raw sums (the fold adds bias and residual in part order)
          if (nin) p.part[(size_t)kz * p.part_stride + (int64_t)tok * p.rows + n] = v[i];
          continue;
        }
        const float o = v[i] + bv;
        if (p.swiglu) {  // gate row n (even lane), up row n + 1 (the next lane)
          const float up = __shfl_down_sync(0xffffffffu, o, 1);
          if (nin && !(lane & 1) && n + 1 < p.rows) p.y[(int64_t)tok * p.ldy + (n >> 1)] = (o / (1.0f + expf(-o))) * up;
        } else if (nin) {
          p.y[(int64_t)tok * p.ldy + n] = p.residual ? o + p.residual[(int64_t)tok * p.ldr + n] : o;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(Cfg::TMEM) : "memory");
}

// per-token 1/rms of x [T][ldx] over K columns (K % 4 == 0): one CTA of RMS_THREADS per
// token, so a decode batch's rows are read by as many SMs as it has tokens, each thread's
// float4 loads independent of one another
constexpr int RMS_THREADS = 128;
__global__ void __launch_bounds__(RMS_THREADS) inv_rms_kernel(const float* x, int ldx, int T, int K, float eps,
                                                              float* out) {
  __shared__ float red[RMS_THREADS / 32];
  const int tok = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  pdl_wait();
  pdl_launch_dependents();
  if (tok >= T) return;
  const float4* r = reinterpret_cast<const float4*>(x + (int64_t)tok * ldx);
  float ss = 0.f;
#pragma unroll 4
  for (int i = threadIdx.x; i < K / 4; i += RMS_THREADS) {
    const float4 v = r[i];
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < RMS_THREADS / 32; ++w) t += red[w];
    out[tok] = rsqrtf(t / K + eps);
  }
}

int* gemv_err_word();

// One-time kernel attribute set-up (call before any stream capture).
int gemm_tc_prepare() {
  if (int rc = smem_attr_once<gemm_tc_kernel<256>>((int)TcCfg<256>::SMEM)) return rc;
  if (int rc = smem_attr_once<gemm_tc_kernel<128>>((int)TcCfg<128>::SMEM)) return rc;
  if (int rc = smem_attr_once<gemm_tc_kernel<64>>((int)TcCfg<64>::SMEM)) return rc;
  return smem_attr_once<gemm_tc_kernel<32>>((int)TcCfg<32>::SMEM);
}

bool gemm_tc_supported(const QWeight& w, int T) {
  const int kpg = w.group / 16;
  return w.layout == 1 && w.bits == 4 && w.cols % TC_BK == 0 && (kpg == 4 || kpg == 8 || kpg == 16) && T >= 1;
}

// Launch on `st`, with programmatic dependent launch when `pdl` (every kernel of the GEMM
// chain waits for its predecessor before reading what that one wrote).
template <typename... KArgs, typename... Args>
static cudaError_t tc_launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                             Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Token tile of a launch: decode batches (< 128 tokens) one tile of 32 / 64 / 128;
// prefill 256-token tiles (each dequantised weight serves 256 tokens) unless that
// leaves SMs idle, then 128.
int gemm_tc_tile(int row_tiles, int tokens) {
  if (tokens <= 32) return 32;
  if (tokens <= 64) return 64;
  if (tokens < 128) return 128;
  return (int64_t)row_tiles * ((tokens + 255) / 256) >= num_sms() ? 256 : 128;
}

// Packed-x workspace of the current device, grown on demand (never inside a stream capture).
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
                 "gemm_tc: packed-x workspace must grow outside stream capture (%zu bytes)", bytes);
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

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
static PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    else
      cudaGetLastError();
  });
  return fn;
}

// The fragment tiles as a 2-D tensor of 8-byte elements: one row per 16-row tile
// (n_groups x group-block bytes), box = one step's bytes x 8 row tiles.  Every
// coordinate the kernel passes is a whole number of group blocks (multiples of
// 16 bytes), the row pitch and the base are 16-byte aligned.
static bool encode_wmap(const QWeight& w, uint32_t step_bytes, CUtensorMap* out) {
  auto enc = tmap_encoder();
  const int GB = (w.group / 16) * 128 + 64;
  const uint64_t pitch = (uint64_t)w.n_groups * GB;
  if (!enc || step_bytes % 16 || step_bytes / 8 > 256 || pitch % 16 || ((uintptr_t)w.codes & 15)) return false;
  const cuuint64_t dims[2] = {pitch / 8, (cuuint64_t)((w.rows + 15) / 16)};
  const cuuint64_t strides[1] = {pitch};
  const cuuint32_t box[2] = {step_bytes / 8, 8};
  const cuuint32_t es[2] = {1, 1};
  return enc(out, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<uint8_t*>(w.codes), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// y[t][r] = residual[t][r] + bias[r] + the K-parts' sums part[z][t][r] added in part order
__global__ void tc_fold_kernel(const float* part, int kparts, int64_t stride, int T, int rows, float* y, int ldy,
                               const float* residual, int ldr, const float* bias) {
  const int64_t n = (int64_t)T * rows;
  pdl_wait();  // the GEMM's parts, and a residual an earlier kernel wrote
  pdl_launch_dependents();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / rows), r = (int)(i - (int64_t)t * rows);
    float v = 0.f;
    for (int z = 0; z < kparts; ++z) v += __ldcg(part + z * stride + i);
    if (bias) v += bias[r];
    if (residual) v += residual[(int64_t)t * ldr + r];
    y[(int64_t)t * ldy + r] = v;
  }
}

// tc_fold_kernel for one token per blockIdx.y and TC_SS_ROWS rows per blockIdx.x, which also
// writes the sum of squares of its outputs to ss[t][blockIdx.x] (fixed-order reductions): the
// next RMSNorm of y then needs no pass over y of its own
__global__ void __launch_bounds__(TC_SS_ROWS) tc_fold_ss_kernel(const float* part, int kparts, int64_t stride,
                                                                int rows, float* y, int ldy, const float* residual,
                                                                int ldr, const float* bias, float* ss) {
  __shared__ float red[TC_SS_ROWS / 32];
  const int t = blockIdx.y, r = blockIdx.x * TC_SS_ROWS + threadIdx.x;
  pdl_wait();  // the GEMM's parts, and a residual an earlier kernel wrote
  pdl_launch_dependents();
  float v = 0.f;
  if (r < rows) {
    const int64_t i = (int64_t)t * rows + r;
    for (int z = 0; z < kparts; ++z) v += __ldcg(part + z * stride + i);
    if (bias) v += bias[r];
    if (residual) v += residual[(int64_t)t * ldr + r];
    y[(int64_t)t * ldy + r] = v;
  }
  const float sq = warp_sum(v * v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sq;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < TC_SS_ROWS / 32; ++w) tot += red[w];
    ss[(int64_t)t * gridDim.x + blockIdx.x] = tot;
  }
}

constexpr int TC_MAX_KPARTS = 8;

// Split-K partial sums of the current device, grown on demand (never inside a stream capture).
static int part_workspace(size_t floats, cudaStream_t st, float** out) {
  static std::mutex mu;
  static float* buf[N730_MAX_DEVICES] = {};
  static size_t cap[N730_MAX_DEVICES] = {};
  int dev = 0;
  N730_CUDA(cudaGetDevice(&dev));
  N730_REQUIRE(dev >= 0 && dev < N730_MAX_DEVICES, N730_BAD_ARG, "gemm_tc: device %d", dev);
  std::lock_guard<std::mutex> lk(mu);
  if (cap[dev] < floats) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    N730_CUDA(cudaStreamIsCapturing(st, &cs));
    N730_REQUIRE(cs == cudaStreamCaptureStatusNone, N730_STATE,
                 "gemm_tc: split-K workspace must grow outside stream capture (%zu floats)", floats);
    N730_CUDA(cudaStreamSynchronize(st));
    if (buf[dev]) N730_CUDA(cudaFree(buf[dev]));
    buf[dev] = nullptr;
    cap[dev] = 0;
    N730_CUDA(cudaMalloc(&buf[dev], floats * sizeof(float)));
    cap[dev] = floats;
  }
  *out = buf[dev];
  return N730_OK;
}

// K-parts of a launch: decode-sized calls (< 128 tokens) whose grid of row and token tiles
// leaves SMs idle split K over blockIdx.z (each part >= 2 steps; SwiGLU outputs never split)
static int gemm_tc_kparts(int row_tiles, int token_tiles, int ksteps, int tokens, bool swiglu) {
  const int ctas = row_tiles * token_tiles;
  if (tokens >= 128 || swiglu || ctas >= num_sms()) return 1;
  return std::max(1, std::min({TC_MAX_KPARTS, (num_sms() + ctas - 1) / ctas, ksteps / 2}));
}

// CTAs of a launch (row tiles x token tiles x K-parts)
int gemm_tc_ctas(int rows, int cols, int tokens, bool swiglu) {
  const int rt = (rows + TC_BN - 1) / TC_BN, ntok = gemm_tc_tile(rt, tokens), tt = (tokens + ntok - 1) / ntok;
  return rt * tt * gemm_tc_kparts(rt, tt, cols / TC_BK, tokens, swiglu);
}

bool gemm_tc_folds(const QWeight& w, int tokens, bool swiglu) {
  if (!gemm_tc_supported(w, tokens)) return false;
  const int rt = (w.rows + TC_BN - 1) / TC_BN, ntok = gemm_tc_tile(rt, tokens), tt = (tokens + ntok - 1) / ntok;
  return gemm_tc_kparts(rt, tt, w.cols / TC_BK, tokens, swiglu) > 1;
}

// Grow the packed-x workspace for calls of up to `tokens` tokens and `cols` columns now,
// so that calls captured into a CUDA graph later never need to grow it.
int gemm_tc_reserve(int tokens, int cols, int rows, cudaStream_t st) {
  if (tokens < 1 || cols < 64) return N730_OK;
  const int KB = (cols + 63) / 64;
  const int XT = (tokens + 255) / 256 * 2;  // the most sub-tiles any token tile choice packs
  uint8_t* x16 = nullptr;
  if (int rc = x16_workspace((size_t)XT * KB * TC_SUB, st, &x16)) return rc;
  float* part = nullptr;
  return part_workspace((size_t)TC_MAX_KPARTS * std::min(tokens, 127) * std::max(rows, 1), st, &part);
}

int gemm_tc_launch(const GemvArgs& a, float* inv_ws, cudaStream_t st) {
  const QWeight& w = *a.w;
  N730_REQUIRE(gemm_tc_supported(w, a.batch), N730_UNSUPPORTED, "gemm_tc: needs INT4 fragment tiles, K %% 64 == 0");
  N730_REQUIRE(!a.swiglu || w.rows % 2 == 0, N730_BAD_ARG, "gemm_tc: swiglu needs even rows");
  N730_REQUIRE(((uintptr_t)a.x & 15) == 0 && a.ldx % 4 == 0, N730_BAD_ARG, "gemm_tc: x must be 16-byte aligned");
  N730_REQUIRE(!a.norm_w || ((inv_ws || a.ss_in) && ((uintptr_t)a.norm_w & 15) == 0), N730_BAD_ARG,
               "gemm_tc: RMSNorm needs a workspace of batch floats (or sums of squares) and 16-byte aligned weights");
  int* err = gemv_err_word();
  N730_REQUIRE(err, N730_OOM, "gemm_tc: error word allocation failed");
  if (int rc = gemm_tc_prepare()) return rc;
  // 256-token tiles dequantise each weight once per 256 tokens; 128-token tiles
  // when 256 would leave SMs idle (few row tiles, few tokens)
  const int RT = (w.rows + TC_BN - 1) / TC_BN, KB = w.cols / 64;
  const int ntok = gemm_tc_tile(RT, a.batch);
  const int TT = (a.batch + ntok - 1) / ntok;              // output token tiles
  const int XT = (TT * ntok + TC_XT - 1) / TC_XT;          // packed 128-token sub-tiles
  const int kparts = gemm_tc_kparts(RT, TT, w.cols / TC_BK, a.batch, a.swiglu != 0);
  N730_REQUIRE(!a.ss_out || kparts > 1, N730_BAD_ARG, "gemm_tc: sums of squares come from the split-K fold only");
  uint8_t* x16 = nullptr;
  if (int rc = x16_workspace((size_t)XT * KB * TC_SUB, st, &x16)) return rc;
  const bool pdl = a.pdl != 0;
  const float* ss_in = a.norm_w ? a.ss_in : nullptr;
  if (a.norm_w && !ss_in)
    N730_CUDA(tc_launch(inv_rms_kernel, dim3(a.batch), RMS_THREADS, 0, st, pdl, a.x, a.ldx, a.batch, w.cols, a.eps,
                        inv_ws));
  // every sub-tile a CTA copies is packed (tokens >= T as zeros)
  N730_CUDA(tc_launch(x16_pack_kernel, dim3(KB, XT), 256, 0, st, pdl, a.x, a.ldx, a.batch,
                      (const float*)(a.norm_w && !ss_in ? inv_ws : nullptr), ss_in,
                      (w.cols + TC_SS_ROWS - 1) / TC_SS_ROWS, w.cols, a.eps, a.norm_w, x16));
  TcArgs p = {};
  p.blob = w.codes; p.rows = w.rows; p.cols = w.cols; p.G = w.n_groups; p.kpg = w.group / 16;
  p.x16 = x16; p.T = a.batch;
  p.y = a.y; p.ldy = a.ldy; p.bias = a.bias; p.residual = a.residual; p.ldr = a.ldr; p.swiglu = a.swiglu;
  p.err = err;
  p.kparts = kparts;
  if (p.kparts > 1) {
    p.part_stride = (int64_t)a.batch * w.rows;
    if (int rc = part_workspace((size_t)p.kparts * p.part_stride, st, &p.part)) return rc;
  }
  const dim3 grid(RT, TT, p.kparts);
  CUtensorMap wmap;
  std::memset(&wmap, 0, sizeof(wmap));
  const int kpg = w.group / 16;
  p.wtma = (kpg == 4 || kpg == 8) && encode_wmap(w, (uint32_t)((8 / kpg) * (kpg * 128 + 64)), &wmap);
  if (ntok == 256) N730_CUDA(tc_launch(gemm_tc_kernel<256>, grid, TC_WARPS * 32, TcCfg<256>::SMEM, st, pdl, p, wmap));
  else if (ntok == 128) N730_CUDA(tc_launch(gemm_tc_kernel<128>, grid, TC_WARPS * 32, TcCfg<128>::SMEM, st, pdl, p, wmap));
  else if (ntok == 64) N730_CUDA(tc_launch(gemm_tc_kernel<64>, grid, TC_WARPS * 32, TcCfg<64>::SMEM, st, pdl, p, wmap));
  else N730_CUDA(tc_launch(gemm_tc_kernel<32>, grid, TC_WARPS * 32, TcCfg<32>::SMEM, st, pdl, p, wmap));
  N730_CHECK_LAUNCH();
  if (p.kparts > 1 && a.ss_out) {
    N730_CUDA(tc_launch(tc_fold_ss_kernel, dim3((w.rows + TC_SS_ROWS - 1) / TC_SS_ROWS, a.batch), TC_SS_ROWS, 0, st,
                        pdl, (const float*)p.part, p.kparts, p.part_stride, w.rows, a.y, a.ldy, a.residual, a.ldr,
                        a.bias, a.ss_out));
  } else if (p.kparts > 1) {
    const int64_t n = (int64_t)a.batch * w.rows;
    const int fg = (int)std::min<int64_t>((n + 255) / 256, (int64_t)num_sms() * 4);
    N730_CUDA(tc_launch(tc_fold_kernel, dim3(fg), 256, 0, st, pdl, (const float*)p.part, p.kparts, p.part_stride,
                        a.batch, w.rows, a.y, a.ldy, a.residual, a.ldr, a.bias));
  }
  return N730_OK;
}

}  // namespace n730
