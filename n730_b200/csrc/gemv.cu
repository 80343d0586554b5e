// Decode dequant-GEMV: y[b, n] = sum_k (q[n,k] - z) * s * x[b, k] for packed
// INT2/INT4/INT8 (group-wise fp16 scale/zero, or per-row fp32) and FP16 weights.
//
// Replaces the reference's per-token "dequant to fp32 d_weights, then
// cublasSgemm" pair (src-code/cpp/n730_cuda.cu:76-107,472-505,549-579,847-870)
// with one HBM-streaming kernel that never materialises fp32 weights.
//
// Design (B200, sm_100a):
//  * One 512-thread CTA per SM owns a contiguous run of weight rows.  Its rows
//    (codes) and their scale/zero rows are contiguous in HBM, so a single
//    thread streams them into a ring of shared-memory stages with 1-D bulk
//    copies (cp.async.bulk, the TMA engine) completing on mbarriers.  Up to
//    ~150 KB per SM is in flight independent of the compute warps, and the
//    first stages are issued before griddepcontrol.wait, overlapping the
//    previous kernel (programmatic dependent launch).
//  * Codes become exact fp32 values with one LOP3 each: the code is masked in
//    place into the mantissa of a power-of-two constant whose mantissa bit at
//    the code's position weighs 1; the constant is removed with a packed
//    f32x2 add (FADD2) and products accumulate with packed FFMA2.  fp32
//    products, fp32 accumulation.
//  * The zero point is applied per 16-byte chunk as s * (sum q*x - z * sum x),
//    the per-chunk sums of x precomputed once per CTA.
//  * x, optionally RMS-normalised in the prologue (fusing the reference's
//    separate rmsnorm launch), sits in shared memory in a chunk-transposed
//    layout so each LDS.128 of a warp reads 512 contiguous bytes.
//  * The inner loop is branch-free (invalid chunks are zero by selection);
//    warps reduce with shuffles, K-split warps through shared memory.
//  * Epilogues: bias, residual add (o_proj / down_proj), SwiGLU on
//    interleaved gate/up rows.
//  * Every mbarrier wait is bounded (globaltimer); on timeout the CTA records
//    DEV_ERR_TIMEOUT in the error word, drains its copies (bounded) and exits.
#include <algorithm>

#include "qweight.h"

namespace n730 {

template <int BITS> struct Fmt {
  static constexpr int E = BITS == 16 ? 8 : 128 / BITS;  // elements per 16-byte chunk
  static constexpr int F4 = E / 4;                       // float4 of x per chunk
  static constexpr int EW = BITS == 16 ? 2 : 32 / BITS;  // elements per 32-bit word
};

__device__ __forceinline__ float mag(int pos) { return __uint_as_float(magic_bits(pos)); }

// Exact fp32 code values of one 32-bit word, as consecutive pairs.
template <int BITS> struct Unpack;

template <> struct Unpack<4> {
  __device__ __forceinline__ static void run(uint32_t w, float2 (&t)[4]) {
    const uint32_t ws = w >> 20;  // nibbles 5..7 to bits 0..11
    t[0] = __fadd2_rn(make_float2(__uint_as_float(lop3_and_or(w, 0xFu, magic_bits(0))),
                                  __uint_as_float(lop3_and_or(w, 0xF0u, magic_bits(4)))),
                      make_float2(-mag(0), -mag(4)));
    t[1] = __fadd2_rn(make_float2(__uint_as_float(lop3_and_or(w, 0xF00u, magic_bits(8))),
                                  __uint_as_float(lop3_and_or(w, 0xF000u, magic_bits(12)))),
                      make_float2(-mag(8), -mag(12)));
    t[2] = __fadd2_rn(make_float2(__uint_as_float(lop3_and_or(w, 0xF0000u, magic_bits(16))),
                                  __uint_as_float(lop3_and_or(ws, 0xFu, magic_bits(0)))),
                      make_float2(-mag(16), -mag(0)));
    t[3] = __fadd2_rn(make_float2(__uint_as_float(lop3_and_or(ws, 0xF0u, magic_bits(4))),
                                  __uint_as_float(lop3_and_or(ws, 0xF00u, magic_bits(8)))),
                      make_float2(-mag(4), -mag(8)));
  }
};

template <> struct Unpack<8> {
  __device__ __forceinline__ static void run(uint32_t w, float2 (&t)[2]) {
    const uint32_t ws = w >> 16;
    t[0] = __fadd2_rn(make_float2(__uint_as_float(lop3_and_or(w, 0xFFu, magic_bits(0))),
                                  __uint_as_float(lop3_and_or(w, 0xFF00u, magic_bits(8)))),
                      make_float2(-mag(0), -mag(8)));
    t[1] = __fadd2_rn(make_float2(__uint_as_float(lop3_and_or(ws, 0xFFu, magic_bits(0))),
                                  __uint_as_float(lop3_and_or(ws, 0xFF00u, magic_bits(8)))),
                      make_float2(-mag(0), -mag(8)));
  }
};

template <> struct Unpack<2> {
  template <int P0, int P1>
  __device__ __forceinline__ static float2 pair(uint32_t a, uint32_t b) {
    return __fadd2_rn(make_float2(__uint_as_float(lop3_and_or(a, 3u << P0, magic_bits(P0))),
                                  __uint_as_float(lop3_and_or(b, 3u << P1, magic_bits(P1)))),
                      make_float2(-mag(P0), -mag(P1)));
  }
  __device__ __forceinline__ static void run(uint32_t w, float2 (&t)[8]) {
    const uint32_t ws = w >> 22;  // crumbs 11..15 to bits 0..9
    t[0] = pair<0, 2>(w, w);
    t[1] = pair<4, 6>(w, w);
    t[2] = pair<8, 10>(w, w);
    t[3] = pair<12, 14>(w, w);
    t[4] = pair<16, 18>(w, w);
    t[5] = pair<20, 0>(w, ws);
    t[6] = pair<2, 4>(ws, ws);
    t[7] = pair<6, 8>(ws, ws);
  }
};

template <> struct Unpack<16> {
  __device__ __forceinline__ static void run(uint32_t w, float2 (&t)[1]) {
    t[0] = __half22float2(*reinterpret_cast<const __half2*>(&w));
  }
};

constexpr int GEMV_THREADS = 512;
constexpr int GEMV_WARPS = GEMV_THREADS / 32;
constexpr int GEMV_MAX_STAGES = 6;

struct GemvParams {
  const uint8_t* codes;
  const uint8_t* sz;
  int64_t row_bytes, sz_pitch;
  int rows, cols;
  int C;              // 16-byte chunks per row
  int Cx;             // chunks of x staged (>= C + 31, multiple of 32)
  uint32_t gmagic;    // group index of chunk c = umulhi(c, gmagic) when gshift < 0
  int gshift;         // group index of chunk c = c >> gshift when >= 0
  int WK, Ck;         // K-split warps, chunks per K-split warp
  int rows_per_cta;
  int stage_rows, n_stages;
  int stage_off, stage_stride;  // bytes
  const float* x; int ldx;
  float* y; int ldy;
  const float* bias;
  const float* residual; int ldr;
  const float* norm_w; float eps;
  int swiglu;
  int* err;
};

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ bool wait_stage(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer() - t0 > 2000000000ull) return false;  // 2 s
  return true;
}

template <int BITS, int SZM, int NB, int R>
__global__ void __launch_bounds__(GEMV_THREADS, 1) gemv_kernel(const GemvParams p) {
  using F = Fmt<BITS>;
  constexpr int E = F::E, F4 = F::F4, EW = F::EW;
  constexpr int NP = EW / 2 > 0 ? EW / 2 : 1;
  constexpr int XF = EW >= 4 ? EW / 4 : 1;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);                 // [S] stage-full barriers
  int* done = reinterpret_cast<int*>(smem + 64);                      // [S] warps finished with stage
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + 96);
  float4* xs = reinterpret_cast<float4*>(smem + 128);                 // [NB][Cx/32][F4][32]
  float* xp = reinterpret_cast<float*>(xs + (size_t)NB * p.Cx * F4);  // [NB][Cx]
  float* red = xp + NB * p.Cx;                                        // [2][warps][R][NB]
  float* red32 = red + 2 * GEMV_WARPS * R * NB;
  uint8_t* stages = smem + p.stage_off;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row_begin = blockIdx.x * p.rows_per_cta;
  if (row_begin >= p.rows) return;
  const int row_end = min(p.rows, row_begin + p.rows_per_cta);
  const int npass = (row_end - row_begin + p.stage_rows - 1) / p.stage_rows;
  const int S = p.n_stages;

  auto issue = [&](int pass) {
    const int s = pass % S;
    const int r0 = row_begin + pass * p.stage_rows;
    const int nr = min(p.stage_rows, row_end - r0);
    uint8_t* dst = stages + (size_t)s * p.stage_stride;
    const uint32_t cb = (uint32_t)(nr * p.row_bytes);
    const uint32_t sb = BITS == 16 ? 0u : (uint32_t)(nr * p.sz_pitch);
    mbar_arrive_expect_tx(&full[s], cb + sb);
    bulk_g2s(dst, p.codes + (int64_t)r0 * p.row_bytes, cb, &full[s]);
    if (BITS != 16)
      bulk_g2s(dst + (size_t)p.stage_rows * p.row_bytes, p.sz + (int64_t)r0 * p.sz_pitch, sb, &full[s]);
  };

  if (tid == 0) {
    for (int s = 0; s < S; ++s) { mbar_init(&full[s], 1); done[s] = 0; }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0)
    for (int q = 0; q < min(S, npass); ++q) issue(q);  // weights do not depend on the previous kernel
  pdl_wait();

  // ---- stage x (optionally RMS-normalised) into the chunk-transposed layout ----
  const int K = p.cols;
  const int Kp4 = p.Cx * E / 4;
  const bool vec = (K % 4 == 0) && (p.ldx % 4 == 0);
  for (int b = 0; b < NB; ++b) {
    const float* xb = p.x + (int64_t)b * p.ldx;
    float inv = 1.f;
    if (p.norm_w) {
      float ss = 0.f;
      if (vec) {
        for (int k4 = tid; k4 < K / 4; k4 += GEMV_THREADS) {
          const float4 v = reinterpret_cast<const float4*>(xb)[k4];
          ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
      } else {
        for (int k = tid; k < K; k += GEMV_THREADS) ss += xb[k] * xb[k];
      }
      ss = block_sum(ss, red32);
      inv = rsqrtf(ss / K + p.eps);
    }
    for (int k4 = tid; k4 < Kp4; k4 += GEMV_THREADS) {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      const int k = k4 * 4;
      if (vec) {
        if (k < K) {
          v = reinterpret_cast<const float4*>(xb)[k4];
          if (p.norm_w) {
            const float4 w = reinterpret_cast<const float4*>(p.norm_w)[k4];
            v.x = v.x * inv * w.x; v.y = v.y * inv * w.y;
            v.z = v.z * inv * w.z; v.w = v.w * inv * w.w;
          }
        }
      } else {
        float e[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          e[j] = (k + j < K) ? xb[k + j] : 0.f;
          if (p.norm_w && k + j < K) e[j] = e[j] * inv * p.norm_w[k + j];
        }
        v = make_float4(e[0], e[1], e[2], e[3]);
      }
      const int c = k / E, f = (k % E) / 4;
      xs[(((size_t)b * (p.Cx / 32) + c / 32) * F4 + f) * 32 + (c & 31)] = v;
    }
    __syncthreads();
    if (BITS != 16) {
      for (int c = tid; c < p.Cx; c += GEMV_THREADS) {
        const float4* xc = xs + (((size_t)b * (p.Cx / 32) + c / 32) * F4) * 32 + (c & 31);
        float s = 0.f;
#pragma unroll
        for (int f = 0; f < F4; ++f) { const float4 v = xc[f * 32]; s += (v.x + v.y) + (v.z + v.w); }
        xp[b * p.Cx + c] = s;
      }
    }
  }
  __syncthreads();
  pdl_launch_dependents();

  const int WK = p.WK;
  const int wk = warp % WK, wr = warp / WK;
  const int cbeg = wk * p.Ck, cend = min(p.C, cbeg + p.Ck);
  const int nj = cend > cbeg ? (cend - cbeg + 31) >> 5 : 0;
  const size_t bstride = (size_t)(p.Cx / 32) * F4 * 32;

  for (int pass = 0; pass < npass; ++pass) {
    const int s = pass % S;
    int okl = 0;
    if (lane == 0) {
      okl = !*abort_flag && wait_stage(&full[s], (uint32_t)((pass / S) & 1));
      if (!okl && !*abort_flag) { *abort_flag = 1; atomicExch(p.err, DEV_ERR_TIMEOUT); }
    }
    const bool ok = __shfl_sync(0xffffffffu, okl, 0) != 0;
    const uint8_t* sc = stages + (size_t)s * p.stage_stride;
    const uint8_t* ss = sc + (size_t)p.stage_rows * p.row_bytes;
    const int prow0 = row_begin + pass * p.stage_rows;

    float part[R][NB];
#pragma unroll
    for (int i = 0; i < R; ++i)
#pragma unroll
      for (int b = 0; b < NB; ++b) part[i][b] = 0.f;

    const int njj = ok ? nj : 0;
    for (int j = 0; j < njj; ++j) {
      const int c = cbeg + j * 32 + lane;
      const bool valid = c < cend;
      const int gi = !valid ? 0 : p.gshift >= 0 ? (c >> p.gshift) : (int)__umulhi((uint32_t)c, p.gmagic);
      float xpv[NB];
#pragma unroll
      for (int b = 0; b < NB; ++b) xpv[b] = (valid && BITS != 16) ? xp[b * p.Cx + c] : 0.f;
      const float4* xc = xs + (size_t)(c >> 5) * F4 * 32 + (c & 31);

      uint4 q[R];
      float2 szv[R];
#pragma unroll
      for (int i = 0; i < R; ++i) {
        const int r = wr * R + i;
        q[i] = valid ? *reinterpret_cast<const uint4*>(sc + (size_t)r * p.row_bytes + (size_t)c * 16)
                     : make_uint4(0, 0, 0, 0);
        if (BITS != 16) {
          const uint8_t* srow = ss + (size_t)r * p.sz_pitch;
          szv[i] = SZM == 0 ? __half22float2(reinterpret_cast<const __half2*>(srow)[gi])
                            : *reinterpret_cast<const float2*>(srow);
        } else {
          szv[i] = make_float2(1.f, 0.f);
        }
      }
      float2 acc[R][NB];
#pragma unroll
      for (int i = 0; i < R; ++i)
#pragma unroll
        for (int b = 0; b < NB; ++b) acc[i][b] = make_float2(0.f, 0.f);
#pragma unroll
      for (int wi = 0; wi < 4; ++wi) {
        float4 xv[NB][XF];
#pragma unroll
        for (int b = 0; b < NB; ++b)
#pragma unroll
          for (int jj = 0; jj < XF; ++jj) xv[b][jj] = xc[b * bstride + (size_t)((wi * EW) / 4 + jj) * 32];
#pragma unroll
        for (int i = 0; i < R; ++i) {
          const uint32_t w = wi == 0 ? q[i].x : wi == 1 ? q[i].y : wi == 2 ? q[i].z : q[i].w;
          float2 t[NP];
          Unpack<BITS>::run(w, t);
#pragma unroll
          for (int b = 0; b < NB; ++b)
#pragma unroll
            for (int pi = 0; pi < NP; ++pi) {
              float2 xx;
              if (EW >= 4) {
                const float4 v = xv[b][pi / 2];
                xx = (pi & 1) ? make_float2(v.z, v.w) : make_float2(v.x, v.y);
              } else {
                const float4 v = xv[b][0];
                xx = (wi & 1) ? make_float2(v.z, v.w) : make_float2(v.x, v.y);
              }
              acc[i][b] = __ffma2_rn(t[pi], xx, acc[i][b]);
            }
        }
      }
#pragma unroll
      for (int i = 0; i < R; ++i)
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          const float dot = acc[i][b].x + acc[i][b].y;
          if (BITS == 16) part[i][b] += dot;
          else part[i][b] = fmaf(szv[i].x, fmaf(-szv[i].y, xpv[b], dot), part[i][b]);
        }
    }

    // release the stage: the last warp to finish refills it
    __syncwarp();
    if (lane == 0) {
      __threadfence_block();
      if (atomicAdd(&done[s], 1) == GEMV_WARPS - 1) {
        done[s] = 0;
        if (pass + S < npass && !*abort_flag) issue(pass + S);
      }
    }

#pragma unroll
    for (int i = 0; i < R; ++i)
#pragma unroll
      for (int b = 0; b < NB; ++b) part[i][b] = warp_sum(part[i][b]);

    if (WK > 1) {  // K-split warps of one row group meet at a named barrier
      float* rb = red + (pass & 1) * GEMV_WARPS * R * NB;
      if (lane == 0) {
#pragma unroll
        for (int i = 0; i < R; ++i)
#pragma unroll
          for (int b = 0; b < NB; ++b) rb[(warp * R + i) * NB + b] = part[i][b];
      }
      asm volatile("bar.sync %0, %1;" :: "r"(1 + wr), "r"(WK * 32) : "memory");
      if (wk == 0) {
#pragma unroll
        for (int i = 0; i < R; ++i)
#pragma unroll
          for (int b = 0; b < NB; ++b) {
            float t = 0.f;
            for (int j2 = 0; j2 < WK; ++j2) t += rb[((wr * WK + j2) * R + i) * NB + b];
            part[i][b] = t;
          }
      }
    }
    if (ok && wk == 0 && lane < NB) {
      const int b = lane;
#pragma unroll
      for (int i = 0; i < R; ++i) {
        const int row = prow0 + wr * R + i;
        if (row >= row_end) continue;
        float v = 0.f, u = 0.f;
#pragma unroll
        for (int bb = 0; bb < NB; ++bb)
          if (bb == b) { v = part[i][bb]; if (i + 1 < R) u = part[i + 1][bb]; }
        v += p.bias ? p.bias[row] : 0.f;
        if (p.swiglu) {
          if ((i & 1) == 0 && row + 1 < row_end) {
            u += p.bias ? p.bias[row + 1] : 0.f;
            p.y[(int64_t)b * p.ldy + row / 2] = (v / (1.0f + expf(-v))) * u;
          }
        } else {
          if (p.residual) v += p.residual[(int64_t)b * p.ldr + row];
          p.y[(int64_t)b * p.ldy + row] = v;
        }
      }
    }
  }
  // A timed-out CTA waits (bounded) for the copies it issued before exiting.
  __syncthreads();
  if (tid == 0 && *abort_flag)
    for (int q = 0; q < npass; ++q) wait_stage(&full[q % S], (uint32_t)((q / S) & 1));
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static int* device_err_word() {
  static int* w[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return nullptr;
  if (!w[dev]) {
    if (cudaMalloc(&w[dev], sizeof(int)) != cudaSuccess) { cudaGetLastError(); return nullptr; }
    cudaMemset(w[dev], 0, sizeof(int));
  }
  return w[dev];
}

template <int BITS, int SZM, int NB, int R>
static int launch_t(const GemvParams& p, int grid, size_t smem, cudaStream_t st, bool pdl) {
  auto fn = gemv_kernel<BITS, SZM, NB, R>;
  if (int rc = smem_attr_once<gemv_kernel<BITS, SZM, NB, R>>(227 * 1024)) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(GEMV_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  N730_CUDA(cudaLaunchKernelEx(&cfg, fn, p));
  return N730_OK;
}

template <int BITS, int SZM>
static int dispatch(int nb, int r, const GemvParams& p, int grid, size_t smem, cudaStream_t st, bool pdl) {
  if (nb == 1 && r == 4) return launch_t<BITS, SZM, 1, 4>(p, grid, smem, st, pdl);
  if (nb == 1 && r == 2) return launch_t<BITS, SZM, 1, 2>(p, grid, smem, st, pdl);
  if (nb == 1 && r == 1) return launch_t<BITS, SZM, 1, 1>(p, grid, smem, st, pdl);
  if (nb == 2 && r == 2) return launch_t<BITS, SZM, 2, 2>(p, grid, smem, st, pdl);
  if (nb == 2 && r == 1) return launch_t<BITS, SZM, 2, 1>(p, grid, smem, st, pdl);
  if (nb == 3 && r == 2) return launch_t<BITS, SZM, 3, 2>(p, grid, smem, st, pdl);
  if (nb == 3 && r == 1) return launch_t<BITS, SZM, 3, 1>(p, grid, smem, st, pdl);
  if (nb == 4 && r == 2) return launch_t<BITS, SZM, 4, 2>(p, grid, smem, st, pdl);
  if (nb == 4 && r == 1) return launch_t<BITS, SZM, 4, 1>(p, grid, smem, st, pdl);
  set_error("gemv: no kernel for batch chunk %d, rows/warp %d", nb, r);
  return N730_BAD_ARG;
}

constexpr int GEMV_MAX_NB = 4;
constexpr size_t SMEM_MAX = 227 * 1024;
constexpr size_t STAGE_MAX = 64 * 1024;

struct Plan {
  int R, WK, Ck, stage_rows, S, stage_off, stage_stride, Cx;
  size_t smem;
};

// SwiGLU pairs rows 2i (gate) and 2i+1 (up) inside one warp, so it needs an even R.
static bool plan_for(const QWeight& w, int nb, int rows_per_cta, int C, bool swiglu, Plan& out) {
  const int E = w.bits == 16 ? 8 : 128 / w.bits;
  const int Cx = (C + 31 + 31) / 32 * 32;
  const size_t fixed = 128 + (size_t)nb * Cx * E * 4 + (size_t)nb * Cx * 4;
  double best = -1;
  for (int R : {4, 2, 1}) {
    if (nb >= 2 && R == 4) continue;
    if (swiglu && (R & 1)) continue;
    for (int WK = 1; WK <= GEMV_WARPS; WK *= 2) {
      const int WR = GEMV_WARPS / WK;
      const int stage_rows = WR * R;
      const int64_t code_b = (int64_t)stage_rows * w.row_bytes;
      const int64_t sz_b = w.bits == 16 ? 0 : (int64_t)stage_rows * w.sz_pitch;
      const size_t stride = (size_t)((code_b + sz_b + 127) / 128 * 128);
      if (stride > STAGE_MAX && !(R == 1 && WK == GEMV_WARPS)) continue;
      const size_t off = (fixed + (size_t)2 * GEMV_WARPS * R * nb * 4 + 128 + 127) / 128 * 128;
      if (off + stride > SMEM_MAX) continue;
      const int S = (int)std::min<size_t>(GEMV_MAX_STAGES, (SMEM_MAX - off) / stride);
      const int Ck = (C + WK - 1) / WK;
      const double ceff = (double)C / ((double)WK * 32.0 * ((Ck + 31) / 32));
      const int passes = (rows_per_cta + stage_rows - 1) / stage_rows;
      const double reff = (double)rows_per_cta / ((double)passes * stage_rows);
      // bytes in flight per SM (capped at what the stages hold)
      const double inflight = (double)std::min(S, passes) * (double)stride;
      const double mem = std::min(1.0, inflight / (96.0 * 1024));
      // K-split warps pay a shuffle reduction + named barrier per pass; more rows
      // per warp amortise the shared x loads.
      const double wkpen = WK == 1 ? 1.0 : 1.0 / (1.0 + 0.12 * (WK > 4 ? 2 : 1));
      const double score = ceff * reff * mem * wkpen * (R == 4 ? 1.06 : R == 2 ? 1.03 : 1.0);
      if (score > best + 1e-9) {
        best = score;
        out = {R, WK, Ck, stage_rows, S, (int)off, (int)stride, Cx, off + (size_t)S * stride};
      }
    }
  }
  return best > 0;
}

int* gemv_err_word() { return device_err_word(); }

int gemv_launch(const GemvArgs& a, cudaStream_t stream) {
  const QWeight& w = *a.w;
  if (w.layout == 1) return gemv_mma_launch(a, stream);
  N730_REQUIRE(w.codes && a.x && a.y, N730_NULL, "gemv: null pointer");
  N730_REQUIRE(a.batch >= 1, N730_BAD_ARG, "gemv: batch %d", a.batch);
  const int bits = w.bits;
  N730_REQUIRE(bits == 2 || bits == 4 || bits == 8 || bits == 16, N730_BAD_ARG, "gemv: bits %d", bits);
  const int E = bits == 16 ? 8 : 128 / bits;
  N730_REQUIRE(w.row_bytes % 16 == 0 && w.row_bytes * 8 >= (int64_t)w.cols * bits, N730_BAD_ARG,
               "gemv: rows must be padded to 16 bytes");
  if (bits != 16) {
    N730_REQUIRE(w.sz && w.sz_pitch % 16 == 0, N730_BAD_ARG, "gemv: scale rows must be 16-byte aligned");
    N730_REQUIRE(w.sz_mode == 1 || (w.group % E == 0 && w.cols % w.group == 0), N730_BAD_ARG,
                 "gemv: group %d incompatible with %d-element chunks", w.group, E);
  }
  N730_REQUIRE(!a.swiglu || w.rows % 2 == 0, N730_BAD_ARG, "gemv: swiglu needs even rows");
  int* err = device_err_word();
  N730_REQUIRE(err, N730_OOM, "gemv: error word allocation failed");

  GemvParams p = {};
  p.codes = w.codes; p.sz = (const uint8_t*)w.sz; p.row_bytes = w.row_bytes; p.sz_pitch = w.sz_pitch;
  p.rows = w.rows; p.cols = w.cols;
  p.C = (w.cols + E - 1) / E;
  // chunk -> group: floor(c / (group / E)) via multiply-high (exact for c < 2^32 / d)
  const uint32_t d = (bits == 16 || w.sz_mode == 1 || w.n_groups <= 1) ? 0u : (uint32_t)(w.group / E);
  p.gshift = -1;
  p.gmagic = 0;
  if (d == 0) {
    p.gshift = 31;  // single group: c >> 31 == 0
  } else if ((d & (d - 1)) == 0) {
    p.gshift = __builtin_ctz(d);
  } else {
    p.gmagic = (uint32_t)(((1ull << 32) + d - 1) / d);
  }
  p.ldy = a.ldy; p.bias = a.bias; p.ldr = a.ldr;
  p.norm_w = a.norm_w; p.eps = a.eps; p.swiglu = a.swiglu; p.err = err;
  const int sms = num_sms();
  int rpc = (w.rows + sms - 1) / sms;
  rpc = (rpc + 1) / 2 * 2;  // even: swiglu pairs never straddle CTAs
  p.rows_per_cta = rpc;
  const int grid = (w.rows + rpc - 1) / rpc;

  int b0 = 0;
  while (b0 < a.batch) {
    int nb = std::min(GEMV_MAX_NB, a.batch - b0);
    Plan pl;
    while (nb >= 1 && !plan_for(w, nb, rpc, p.C, a.swiglu != 0, pl)) --nb;
    N730_REQUIRE(nb >= 1, N730_BAD_ARG, "gemv: K=%d too large for one CTA's shared memory", w.cols);
    p.WK = pl.WK; p.Ck = pl.Ck; p.Cx = pl.Cx; p.stage_rows = pl.stage_rows; p.n_stages = pl.S;
    p.stage_off = pl.stage_off; p.stage_stride = pl.stage_stride;
    p.x = a.x + (int64_t)b0 * a.ldx; p.ldx = a.ldx;
    p.y = a.y + (int64_t)b0 * a.ldy;
    p.residual = a.residual ? a.residual + (int64_t)b0 * a.ldr : nullptr;
    const bool pdl = a.pdl != 0;
    int rc;
    switch (bits) {
      case 4: rc = w.sz_mode == 0 ? dispatch<4, 0>(nb, pl.R, p, grid, pl.smem, stream, pdl)
                                  : dispatch<4, 1>(nb, pl.R, p, grid, pl.smem, stream, pdl); break;
      case 8: rc = w.sz_mode == 0 ? dispatch<8, 0>(nb, pl.R, p, grid, pl.smem, stream, pdl)
                                  : dispatch<8, 1>(nb, pl.R, p, grid, pl.smem, stream, pdl); break;
      case 2: rc = w.sz_mode == 0 ? dispatch<2, 0>(nb, pl.R, p, grid, pl.smem, stream, pdl)
                                  : dispatch<2, 1>(nb, pl.R, p, grid, pl.smem, stream, pdl); break;
      default: rc = dispatch<16, 1>(nb, pl.R, p, grid, pl.smem, stream, pdl); break;
    }
    if (rc) return rc;
    b0 += nb;
  }
  return N730_OK;
}

// Allocate the per-device error word outside any stream capture.
int gemv_prepare() {
  N730_REQUIRE(device_err_word(), N730_OOM, "gemv: error word allocation failed");
  return N730_OK;
}

int gemv_check_error(bool reset) {
  int* err = device_err_word();
  if (!err) return N730_OK;
  int h = 0;
  N730_CUDA(cudaMemcpy(&h, err, sizeof(int), cudaMemcpyDeviceToHost));
  if (h && reset) cudaMemset(err, 0, sizeof(int));
  if (h == DEV_ERR_TIMEOUT) {
    set_error("a GEMV stage wait timed out on the device");
    return N730_TIMEOUT;
  }
  return N730_OK;
}

}  // namespace n730
