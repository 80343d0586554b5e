// Tensor-core decode GEMV for INT4 group-wise weights (batch <= 16).
//
// The fp32 CUDA-core kernel (gemv.cu) needs ~2.4 issue slots per INT4 weight
// at best, which caps it well below the HBM roofline on B200.  This kernel
// moves the multiply-adds onto the tensor cores with mma.m16n8k16 (f16 in, f32
// accumulate) and leaves ~5 integer instructions per 8 codes per lane:
//  * Weights use a fragment-ordered layout built once at registration: for
//    row tile t (16 rows) and k-step s (16 columns), lane l's 32-bit word holds
//    exactly the 8 codes of its A fragment.  One LOP3 per two codes ORs them
//    into the mantissa of fp16 1024: A = 1024 + q (rows g) or 1024 + 16 q
//    (rows g+8, the high nibbles), both exact in fp16.
//  * x (RMS-normalised in the prologue) is the B operand, rounded to fp16;
//    batch rows are the n dimension (n-tiles of 8).  The prologue also forms
//    Sx = sum of the fp16 x over each group, in fp32.
//  * Each group accumulates C = sum (1024 + q) x in fresh fp32 fragments; the
//    group epilogue removes the offset and zero point and applies the scale in
//    fp32:  y += s C - s (1024 + z) Sx   (rows g+8: (s/16) C - s (64 + z) Sx),
//    which equals s sum (q - z) x.
//  * Every warp streams its own work units (row tile, K-part) through a private
//    ring of TMA bulk copies; a unit's groups are contiguous in the layout, so
//    each chunk (codes plus the groups' scale/zero blocks) is one copy.
// Numerics: exact codes, scales and zero points; x rounded to fp16 (relative
// 2^-11 per element); the offset cancellation costs ~7 of fp32's 24 bits - the
// decoder's 1e-2 logit bar holds with a wide margin.  The bit-exact fp32 path
// stays available (gemv.cu).
#include <algorithm>
#include <cstdlib>

#include "mma_gemv.cuh"
#include "qweight.h"

namespace n730 {


// ---------------------------------------------------------------------------
// layout, per row tile and group (kpg = group/16 k-steps):
//   codes [kpg/4][32 lanes][4] u32  (a lane's 4 consecutive k-step words are
//                                    contiguous: one LDS.128)
//   sz    [8] x {s_g, s_g8, z_g, z_g8} fp16 (64 B; g = lane/4, rows g and g+8)
// so any run of whole groups of a tile is one contiguous bulk copy.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int64_t mma_group_bytes(int kpg) { return (int64_t)kpg * 128 + 64; }

__global__ void to_mma_layout_kernel(const uint8_t* codes, int64_t row_bytes, const uint8_t* sz, int64_t sz_pitch,
                                     int rows, int cols, int group, uint8_t* out) {
  const int ks_n = cols / 16, tiles = (rows + 15) / 16, G = cols / group, kpg = group / 16;
  const int64_t gb = mma_group_bytes(kpg);
  const int64_t nwords = (int64_t)tiles * ks_n * 32;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nwords;
       i += (int64_t)gridDim.x * blockDim.x) {
    // i enumerates [t][s4][lane][j]
    const int j = (int)(i & 3), lane = (int)((i >> 2) & 31);
    const int64_t ts4 = i >> 7;
    const int s4 = (int)(ts4 % (ks_n / 4)), t = (int)(ts4 / (ks_n / 4));
    const int s = s4 * 4 + j;
    const int gi = s / kpg, sl = s % kpg;  // group, k-step within the group
    const int g = lane >> 2, tq = lane & 3;
    const int r0 = t * 16 + g, r1 = r0 + 8;
    const int k0 = s * 16 + 2 * tq;
    auto q = [&](int r, int k) -> uint32_t {
      if (r >= rows) return 0u;
      const uint8_t byte = codes[(int64_t)r * row_bytes + (k >> 1)];
      return (k & 1) ? (byte >> 4) : (byte & 15u);
    };
    const uint32_t w = q(r0, k0) | q(r1, k0) << 4 | q(r0, k0 + 8) << 8 | q(r1, k0 + 8) << 12 |
                       q(r0, k0 + 1) << 16 | q(r1, k0 + 1) << 20 | q(r0, k0 + 9) << 24 | q(r1, k0 + 9) << 28;
    uint32_t* dst = reinterpret_cast<uint32_t*>(out + ((int64_t)t * G + gi) * gb);
    dst[((sl >> 2) * 32 + lane) * 4 + (sl & 3)] = w;
  }
  const int64_t nsz = (int64_t)tiles * G * 8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nsz; i += (int64_t)gridDim.x * blockDim.x) {
    const int g = (int)(i & 7);
    const int64_t tg = i >> 3;
    const int gi = (int)(tg % G), t = (int)(tg / G);
    const int r0 = t * 16 + g, r1 = r0 + 8;
    auto get = [&](int r) -> __half2 {
      if (r >= rows) return __halves2half2(__float2half(0.f), __float2half(0.f));
      return reinterpret_cast<const __half2*>(sz + (int64_t)r * sz_pitch)[gi];
    };
    const __half2 a = get(r0), b = get(r1);  // (scale, zero)
    const __half s0 = __low2half(a), z0 = __high2half(a), s1 = __low2half(b), z1 = __high2half(b);
    const __half2 lo = __halves2half2(s0, s1);
    const __half2 hi = __halves2half2(z0, z1);
    uint2 v;
    v.x = *reinterpret_cast<const uint32_t*>(&lo);
    v.y = *reinterpret_cast<const uint32_t*>(&hi);
    reinterpret_cast<uint2*>(out + ((int64_t)t * G + gi) * gb + (int64_t)kpg * 128)[g] = v;
  }
}

int qweight_to_mma_layout(QWeight& w, cudaStream_t st) {
  if (w.layout == 1) return N730_OK;
  N730_REQUIRE(w.bits == 4 && w.sz_mode == 0 && w.group % 64 == 0 && w.cols % 64 == 0, N730_UNSUPPORTED,
               "mma layout: needs INT4 group-wise weights with group %% 64 == 0");
  const int tiles = (w.rows + 15) / 16, ks_n = w.cols / 16, G = w.n_groups, kpg = w.group / 16;
  uint8_t* blob = nullptr;
  if (cudaMalloc(&blob, (size_t)tiles * G * ((size_t)kpg * 128 + 64)) != cudaSuccess) {
    cudaGetLastError();
    set_error("mma layout: out of device memory");
    return N730_OOM;
  }
  const int64_t work = std::max<int64_t>((int64_t)tiles * ks_n * 32, (int64_t)tiles * G * 8);
  const int grid = (int)std::min<int64_t>((work + 255) / 256, num_sms() * 16);
  to_mma_layout_kernel<<<grid, 256, 0, st>>>(w.codes, w.row_bytes, (const uint8_t*)w.sz, w.sz_pitch, w.rows, w.cols,
                                             w.group, blob);
  if (int rc = cuda_rc(cudaGetLastError(), __FILE__, __LINE__)) { cudaFree(blob); return rc; }
  N730_CUDA(cudaStreamSynchronize(st));
  if (w.owns) { cudaFree(w.codes); cudaFree(w.sz); }
  w.codes = blob;
  w.sz = nullptr;
  w.owns = true;
  w.layout = 1;
  w.row_bytes = (int64_t)w.cols / 2;  // logical bytes per row (16 rows share a tile)
  w.sz_pitch = 0;
  return N730_OK;
}

// ---------------------------------------------------------------------------
// kernel
// ---------------------------------------------------------------------------
struct MmaParams {
  const uint8_t* blob;     // [tiles][G] x (codes kpg*128 B, sz 64 B)
  int rows, cols, ks_n, G;
  int tiles_per_cta;
  int parts;               // K-parts per row tile
  int xf_off, sx_off, acc_off, ring_off, ring_stride;  // smem byte offsets / per-buffer bytes
  int ring;                // chunks in flight per warp (<= MG2_RING)
  const float* x; int ldx; int batch;
  float* y; int ldy;
  const float* bias;
  const float* residual; int ldr;
  const float* norm_w; float eps;
  int swiglu;
  int* err;
  // split K (blockIdx.y = K-block of kb_n, whole groups each): the CTA writes its
  // raw partial sums to part[kb * part_stride + b * rows + row] and a fold kernel
  // adds the K-blocks in order plus bias and residual
  int kb_n;
  float* part;
  int64_t part_stride;
};

constexpr int MG2_RING = 3;   // chunks in flight per warp (fewer when shared memory is short)
constexpr int MG2_CHUNK = 32; // k-steps per chunk: a whole number of groups, ~4.3 KB with their scales

// Work of one warp: units u = warp, warp+WARPS, ... of the CTA; unit -> (row
// tile, K-part).  Each warp streams its units' chunks through its own bulk-copy
// ring, so warps never wait for one another; K-parts of a tile merge with
// shared-memory atomics and the warp that completes a tile writes it out.
// WARPS = 8 fits two CTAs per SM, so the next kernel of a PDL chain can start
// its weight copies while this one finishes.
template <int KPG, int NT, int WARPS>
__global__ void __launch_bounds__(WARPS * 32, 16 / WARPS) gemv_mma2_kernel(const MmaParams p) {
  constexpr int THREADS = WARPS * 32;
  constexpr int GPC = MG2_CHUNK / KPG;       // groups per chunk
  constexpr int GB = KPG * 128 + 64;         // bytes per group: codes + scale/zero block
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);                   // [WARPS][MG2_RING]
  int* tile_cnt = reinterpret_cast<int*>(smem + WARPS * MG2_RING * 8);  // [tiles_per_cta]
  uint4* xf = reinterpret_cast<uint4*>(smem + p.xf_off);                // [batch][ks_n/2][4 tq] x 2 k-steps
  float* sx = reinterpret_cast<float*>(smem + p.sx_off);                // [G][NT*8]
  // [slots][16][NT*8]: one slot per (tile, K-part), or per warp when there is one part
  float* accs = reinterpret_cast<float*>(smem + p.acc_off);
  const int acc_slots = p.parts == 1 ? WARPS : p.tiles_per_cta * p.parts;  // as laid out by the host
  float* red = accs + acc_slots * 16 * NT * 8;                          // [WARPS][16] + [16]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n_tiles = (p.rows + 15) / 16;
  const int tile0 = blockIdx.x * p.tiles_per_cta;
  // this CTA's K-block: groups [g0, g0 + Gk), k-steps [s0, s0 + ks_loc)
  const int kb = blockIdx.y;
  const int g0 = (int)((int64_t)p.G * kb / p.kb_n), Gk = (int)((int64_t)p.G * (kb + 1) / p.kb_n) - g0;
  const int s0 = g0 * KPG, ks_loc = Gk * KPG;
  if (tile0 >= n_tiles) return;
  const int ntc = min(p.tiles_per_cta, n_tiles - tile0);
  const int P = p.parts;
  const int n_units = ntc * P;
  uint64_t* wb = bars + warp * MG2_RING;
  uint8_t* ring = smem + p.ring_off + (size_t)warp * p.ring * p.ring_stride;

  for (int i = tid; i < ntc; i += THREADS) tile_cnt[i] = 0;
  if (lane == 0) {
    for (int r = 0; r < p.ring; ++r) mbar_init(&wb[r], 1);
    fence_mbar_init();
  }
  __syncwarp();

  // chunk cursor over this warp's units; unit u -> (row tile, K-part)
  struct Cursor { int u, t, ks, ks_end; };
  auto start_unit = [&](Cursor& c) {
    if (c.u >= n_units) return;
    c.t = tile0 + c.u / P;
    const int part = c.u % P;
    c.ks = (g0 + part * Gk / P) * KPG;
    c.ks_end = (g0 + (part + 1) * Gk / P) * KPG;
  };
  auto issue = [&](const Cursor& c, int slot) {
    const int ng = min(MG2_CHUNK, c.ks_end - c.ks) / KPG;
    const uint32_t bytes = (uint32_t)(ng * GB);
    mbar_arrive_expect_tx(&wb[slot], bytes);
    bulk_g2s(ring + (size_t)slot * p.ring_stride, p.blob + ((int64_t)c.t * p.G + c.ks / KPG) * GB, bytes, &wb[slot]);
  };
  auto advance = [&](Cursor& c) {
    c.ks += MG2_CHUNK;
    if (c.ks >= c.ks_end) { c.u += WARPS; start_unit(c); }
  };

  // weights do not depend on the previous kernel: start streaming before the
  // grid dependency wait
  Cursor prod{warp, 0, 0, 0};
  start_unit(prod);
  if (lane == 0)
    for (int r = 0; r < p.ring && prod.u < n_units; ++r) { issue(prod, r); advance(prod); }
  pdl_wait();

  // ---- prologue: per-row inverse RMS (all batch rows in one pass) ----
  const int K = p.cols, nb = p.batch;
  float* inv = red + WARPS * 16;
  if (p.norm_w) {
    float ss[16];
#pragma unroll
    for (int b = 0; b < 16; ++b) ss[b] = 0.f;
    for (int i = tid; i < (K >> 2); i += THREADS) {
#pragma unroll
      for (int b = 0; b < 16; ++b) {
        if (b < nb) {
          const float4 v = reinterpret_cast<const float4*>(p.x + (int64_t)b * p.ldx)[i];
          ss[b] += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
      }
    }
#pragma unroll
    for (int b = 0; b < 16; ++b) {
      if (b < nb) {
        const float v = warp_sum(ss[b]);
        if (lane == 0) red[warp * 16 + b] = v;
      }
    }
    __syncthreads();
    if (tid < nb) {
      float v = 0.f;
      for (int w = 0; w < WARPS; ++w) v += red[w * 16 + tid];
      inv[tid] = rsqrtf(v / K + p.eps);
    }
    __syncthreads();
  }
  // ---- x -> (RMS-normalised) fp16 B fragments of the K-block:
  //      xf[b][s - s0][tq] = {x[2tq], x[2tq+1], x[2tq+8], x[2tq+9]} of k-step s ----
  uint2* xf2 = reinterpret_cast<uint2*>(xf);
  const int per_row = ks_loc * 4;
#pragma unroll 4
  for (int i = tid; i < nb * per_row; i += THREADS) {
    const int b = i / per_row, r = i - b * per_row;
    const int s = r >> 2, tq = r & 3, k = (s0 + s) * 16 + 2 * tq;
    const float* xb = p.x + (int64_t)b * p.ldx;
    float2 v0 = *reinterpret_cast<const float2*>(xb + k), v1 = *reinterpret_cast<const float2*>(xb + k + 8);
    if (p.norm_w) {
      const float iv = inv[b];
      const float2 n0 = *reinterpret_cast<const float2*>(p.norm_w + k);
      const float2 n1 = *reinterpret_cast<const float2*>(p.norm_w + k + 8);
      v0.x = v0.x * iv * n0.x; v0.y = v0.y * iv * n0.y;
      v1.x = v1.x * iv * n1.x; v1.y = v1.y * iv * n1.y;
    }
    // element (b, s, tq) at uint2 index ((b * ks_loc/2 + s/2) * 4 + tq) * 2 + (s & 1)
    xf2[(((size_t)b * (ks_loc >> 1) + (s >> 1)) * 4 + tq) * 2 + (s & 1)] =
        make_uint2(h2u(__floats2half2_rn(v0.x, v0.y)), h2u(__floats2half2_rn(v1.x, v1.y)));
  }
  __syncthreads();
  // Sx[grp][col]: sum of the fp16 x of group grp, batch row col (0 beyond the
  // batch); one thread per (group, col), sequential order
  for (int pr = tid; pr < Gk * NT * 8; pr += THREADS) {
    const int grp = pr / (NT * 8), col = pr - grp * (NT * 8);
    float v = 0.f;
    if (col < nb) {
      const uint4* src = xf + ((size_t)col * (ks_loc >> 1) + grp * (KPG >> 1)) * 4;
#pragma unroll 4
      for (int e = 0; e < KPG * 2; ++e) {  // KPG/2 k-step pairs x 4 tq
        const uint4 u = src[e];
        const float2 f0 = __half22float2(u2h(u.x)), f1 = __half22float2(u2h(u.y));
        const float2 f2 = __half22float2(u2h(u.z)), f3 = __half22float2(u2h(u.w));
        v += ((f0.x + f0.y) + (f1.x + f1.y)) + ((f2.x + f2.y) + (f3.x + f3.y));
      }
    }
    sx[pr] = v;
  }
  __syncthreads();
  pdl_launch_dependents();

  const int g = lane >> 2, tq = lane & 3;
  const int ks_half = ks_loc >> 1;
  bool aborted = false;
  Cursor cons{warp, 0, 0, 0};
  start_unit(cons);
  int q = 0;  // chunks consumed by this warp
  while (cons.u < n_units) {
    const int t = cons.t, ks0 = cons.ks, nks = cons.ks_end - cons.ks;
    float acc[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
    for (int off = 0; off < nks; off += MG2_CHUNK, ++q) {
      const int slot = q % p.ring;
      int okl = 0;
      if (lane == 0) okl = !aborted && wait_bar(&wb[slot], (uint32_t)((q / p.ring) & 1));
      if (!__shfl_sync(0xffffffffu, okl, 0)) {
        if (lane == 0 && !aborted) atomicExch(p.err, DEV_ERR_TIMEOUT);
        aborted = true;
        break;
      }
      const uint8_t* buf = ring + (size_t)slot * p.ring_stride;
      const int ngr = min(MG2_CHUNK, nks - off) / KPG;
      const int grp0 = (ks0 + off) / KPG;
      // x fragments of this chunk: row min(g, batch-1) (columns >= batch are never read)
      const uint4* xb[NT];
#pragma unroll
      for (int nn = 0; nn < NT; ++nn)
        xb[nn] = xf + ((size_t)min(nn * 8 + g, nb - 1) * ks_half + ((ks0 + off - s0) >> 1)) * 4 + tq;
      const float* sxg = sx + (grp0 - g0) * (NT * 8);
      if (ngr == GPC) {
        mma_chunk<KPG, NT, GPC>(buf, lane, xb, sxg, acc);
      } else {
        for (int gr = 0; gr < ngr; ++gr) {
          const uint4* xg[NT];
#pragma unroll
          for (int nn = 0; nn < NT; ++nn) xg[nn] = xb[nn] + gr * (KPG >> 1) * 4;
          mma_chunk<KPG, NT, 1>(buf + gr * GB, lane, xg, sxg + gr * (NT * 8), acc);
        }
      }
      // this chunk's buffer is free: issue the chunk RING positions ahead
      __syncwarp();
      if (lane == 0 && prod.u < n_units) { issue(prod, slot); advance(prod); }
    }
    if (aborted) break;
    // this K-part's partial goes to its own slot; the warp completing the tile
    // sums the slots in part order (deterministic) and writes the tile out
    const int tl = t - tile0, part = (cons.u - (cons.u / P) * P);
    constexpr int TS = 16 * NT * 8;  // floats per slot
    // one slot per (tile, K-part); with a single part the warp's own slot serves
    const size_t slot0 = P == 1 ? (size_t)warp : (size_t)tl * P;
    float* ta = accs + (slot0 + part) * TS;
#pragma unroll
    for (int nn = 0; nn < NT; ++nn) {
      const int c = nn * 8 + 2 * tq;
      ta[g * NT * 8 + c] = acc[nn][0]; ta[(g + 8) * NT * 8 + c] = acc[nn][2];
      ta[g * NT * 8 + c + 1] = acc[nn][1]; ta[(g + 8) * NT * 8 + c + 1] = acc[nn][3];
    }
    __threadfence_block();
    __syncwarp();
    int last = 0;
    if (lane == 0) last = atomicAdd(&tile_cnt[tl], 1) == P - 1;
    if (__shfl_sync(0xffffffffu, last, 0)) {
      __threadfence_block();
      const volatile float* tb = accs + slot0 * TS;
      auto tile_sum = [&](int i) {
        float v = 0.f;
        for (int q2 = 0; q2 < P; ++q2) v += tb[q2 * TS + i];
        return v;
      };
      for (int i = lane; i < TS; i += 32) {
        const int r = i / (NT * 8), bc = i % (NT * 8);
        const int row = t * 16 + r;
        if (bc >= nb || row >= p.rows) continue;
        if (p.part) {  // split K: raw partial of this K-block
          p.part[(int64_t)kb * p.part_stride + (int64_t)bc * p.rows + row] = tile_sum(i);
          continue;
        }
        if (p.swiglu && (r & 1)) continue;
        float v = tile_sum(i) + (p.bias ? p.bias[row] : 0.f);
        if (p.swiglu) {
          const float u = tile_sum(i + NT * 8) + (p.bias ? p.bias[row + 1] : 0.f);
          p.y[(int64_t)bc * p.ldy + row / 2] = (v / (1.0f + expf(-v))) * u;
        } else {
          if (p.residual) v += p.residual[(int64_t)bc * p.ldr + row];
          p.y[(int64_t)bc * p.ldy + row] = v;
        }
      }
    }
    cons.u += WARPS;
    start_unit(cons);
  }
  // a timed-out warp waits (bounded) for the copies it issued before exiting
  if (aborted && lane == 0)
    for (int r = 0; r < p.ring; ++r) wait_bar(&wb[r], 0), wait_bar(&wb[r], 1);
}

int* gemv_err_word();

template <int KPG, int NT, int WARPS>
static int launch_mma2(const MmaParams& p, int grid, size_t smem, cudaStream_t st, bool pdl) {
  const dim3 g3(grid, p.kb_n);
  if (int rc = smem_attr_once<gemv_mma2_kernel<KPG, NT, WARPS>>(227 * 1024)) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = g3;
  cfg.blockDim = dim3(WARPS * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  N730_CUDA(cudaLaunchKernelEx(&cfg, gemv_mma2_kernel<KPG, NT, WARPS>, p));
  return N730_OK;
}

template <int WARPS>
static int launch_mma2_w(int kpg, int NT, const MmaParams& p, int grid, size_t smem, cudaStream_t st, bool pdl) {
  if (kpg == 8) return NT == 1 ? launch_mma2<8, 1, WARPS>(p, grid, smem, st, pdl) : launch_mma2<8, 2, WARPS>(p, grid, smem, st, pdl);
  if (kpg == 4) return NT == 1 ? launch_mma2<4, 1, WARPS>(p, grid, smem, st, pdl) : launch_mma2<4, 2, WARPS>(p, grid, smem, st, pdl);
  return NT == 1 ? launch_mma2<16, 1, WARPS>(p, grid, smem, st, pdl) : launch_mma2<16, 2, WARPS>(p, grid, smem, st, pdl);
}

// Warps per CTA: 16 (one CTA per SM, the most bytes in flight), except for a
// single-row GEMV too small to give every warp two chunks: 8, so that two CTAs
// fit on an SM and the next kernel of a PDL chain streams its weights while this
// one finishes (measured: batched decode is faster with 16 warps throughout).
// N730_GEMV_WARPS=8 or 16 forces one of them.
static int mma_warps(int64_t chunks, int batch) {
  static int forced = [] {
    const char* e = getenv("N730_GEMV_WARPS");
    return e ? atoi(e) : 0;
  }();
  if (forced == 8 || forced == 16) return forced;
  return batch > 1 || chunks >= (int64_t)num_sms() * 16 * 2 ? 16 : 8;
}

// y[b][r] = residual[b][r] + bias[r] + sum over K-blocks of part[kb][b][r], in K-block order
__global__ void split_fold_kernel(const float* part, int kb_n, int64_t stride, int nb, int rows, float* y, int ldy,
                                  const float* residual, int ldr, const float* bias) {
  const int64_t n = (int64_t)nb * rows;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int b = (int)(i / rows), r = (int)(i - (int64_t)b * rows);
    float v = 0.f;
    for (int kb = 0; kb < kb_n; ++kb) v += __ldcg(part + kb * stride + i);
    if (bias) v += bias[r];
    if (residual) v += residual[(int64_t)b * ldr + r];
    y[(int64_t)b * ldy + r] = v;
  }
}

int gemv_mma_launch(const GemvArgs& a, cudaStream_t st) {
  const QWeight& w = *a.w;
  N730_REQUIRE(w.layout == 1, N730_BAD_ARG, "gemv_mma: weight not in mma layout");
  N730_REQUIRE(!a.swiglu || w.rows % 2 == 0, N730_BAD_ARG, "gemv_mma: swiglu needs even rows");
  int* err = gemv_err_word();
  N730_REQUIRE(err, N730_OOM, "gemv_mma: error word allocation failed");
  const int kpg = w.group / 16;
  N730_REQUIRE(kpg == 4 || kpg == 8 || kpg == 16, N730_UNSUPPORTED, "gemv_mma: group %d", w.group);
  N730_REQUIRE(((uintptr_t)a.x & 15) == 0 && a.ldx % 4 == 0 && (!a.norm_w || ((uintptr_t)a.norm_w & 7) == 0),
               N730_BAD_ARG, "gemv_mma: x must be 16-byte aligned with ldx %% 4 == 0");
  const int n_tiles0 = (w.rows + 15) / 16;
  const int WARPS = mma_warps((int64_t)n_tiles0 * ((w.n_groups * kpg + MG2_CHUNK - 1) / MG2_CHUNK), a.batch);
  MmaParams p = {};
  p.blob = w.codes;
  p.rows = w.rows; p.cols = w.cols; p.ks_n = w.cols / 16; p.G = w.n_groups;
  p.ldy = a.ldy; p.bias = a.bias; p.ldr = a.ldr; p.norm_w = a.norm_w; p.eps = a.eps; p.swiglu = a.swiglu;
  p.err = err;
  const int n_tiles = (w.rows + 15) / 16;
  const int ctas = num_sms();
  p.ring_stride = ((MG2_CHUNK / kpg) * (kpg * 128 + 64) + 127) / 128 * 128;
  const size_t cap = WARPS == 16 ? 227 * 1024 : 113 * 1024;
  // grid for kb_n K-blocks: one CTA per SM in all, row tiles split over ceil(ctas / kb_n) CTAs
  int grid = 0;
  auto geometry = [&](int kb_n) {
    p.kb_n = kb_n;
    const int row_ctas = std::max(1, ctas / kb_n);
    p.tiles_per_cta = (n_tiles + row_ctas - 1) / row_ctas;
    grid = (n_tiles + p.tiles_per_cta - 1) / p.tiles_per_cta;
    const int Gk = p.G / kb_n;  // smallest K-block
    // K-parts so every warp has a unit; each part a whole number of groups
    p.parts = std::max(1, std::min(Gk, (WARPS + p.tiles_per_cta - 1) / p.tiles_per_cta));
  };
  auto layout = [&](int nb_) {
    const int NT = nb_ > 8 ? 2 : 1;
    const int gk_max = (p.G + p.kb_n - 1) / p.kb_n;
    size_t off = 128 + (size_t)WARPS * MG2_RING * 8 + (size_t)p.tiles_per_cta * 4;
    off = (off + 127) / 128 * 128;
    p.xf_off = (int)off;
    off += (size_t)nb_ * gk_max * kpg * 4 * sizeof(uint2);  // k-steps of the K-block (even)
    off = (off + 127) / 128 * 128;
    p.sx_off = (int)off;
    off += (size_t)gk_max * NT * 8 * 4;
    off = (off + 127) / 128 * 128;
    p.acc_off = (int)off;
    const size_t slots = p.parts == 1 ? (size_t)WARPS : (size_t)p.tiles_per_cta * p.parts;
    off += (slots * 16 * NT * 8 + (WARPS + 1) * 16) * 4;
    off = (off + 127) / 128 * 128;
    p.ring_off = (int)off;
    return off + (size_t)WARPS * p.ring * p.ring_stride;
  };
  int b0 = 0;
  while (b0 < a.batch) {
    int nb = std::min(16, a.batch - b0);
    p.ring = MG2_RING;
    geometry(1);
    // no more ring slots than the warp has chunks (a small GEMV then fits two CTAs per SM)
    auto fit_ring = [&]() {
      const int chunks_per_unit = ((p.G / p.kb_n + p.parts - 1) / p.parts * kpg + MG2_CHUNK - 1) / MG2_CHUNK;
      const int per_warp = (p.tiles_per_cta * p.parts + WARPS - 1) / WARPS * chunks_per_unit;
      p.ring = std::max(1, std::min(MG2_RING, per_warp));
    };
    fit_ring();
    while (p.ring > 2 && layout(nb) > cap) --p.ring;
    // the chunk's x fragments do not fit: split K over CTAs (partials + fold) when a workspace
    // is given, else fewer batch columns per pass
    if (layout(nb) > cap && a.split_ws && !a.swiglu) {
      int kb_n = 2;
      for (; kb_n <= std::min(p.G, 16); ++kb_n) {
        geometry(kb_n);
        fit_ring();
        while (p.ring > 2 && layout(nb) > cap) --p.ring;
        if (layout(nb) <= cap && (int64_t)kb_n * nb * w.rows <= a.split_ws_floats) break;
      }
      if (kb_n > std::min(p.G, 16)) geometry(1);
      fit_ring();
      while (p.ring > 2 && layout(nb) > cap) --p.ring;
    }
    while (nb > 1 && layout(nb) > cap) --nb;
    const size_t smem = layout(nb);
    N730_REQUIRE(smem <= cap, N730_BAD_ARG, "gemv_mma: K=%d too large for shared memory", w.cols);
    const int NT = nb > 8 ? 2 : 1;
    p.x = a.x + (int64_t)b0 * a.ldx; p.ldx = a.ldx; p.batch = nb;
    p.y = a.y + (int64_t)b0 * a.ldy;
    p.residual = a.residual ? a.residual + (int64_t)b0 * a.ldr : nullptr;
    p.part = p.kb_n > 1 ? a.split_ws : nullptr;
    p.part_stride = (int64_t)nb * w.rows;
    const bool pdl = a.pdl != 0;
    const int rc = WARPS == 16 ? launch_mma2_w<16>(kpg, NT, p, grid, smem, st, pdl)
                               : launch_mma2_w<8>(kpg, NT, p, grid, smem, st, pdl);
    if (rc) return rc;
    if (p.kb_n > 1) {
      const int64_t n = (int64_t)nb * w.rows;
      const int fg = (int)std::min<int64_t>((n + 255) / 256, ctas * 4);
      split_fold_kernel<<<fg, 256, 0, st>>>(a.split_ws, p.kb_n, p.part_stride, nb, w.rows, p.y, a.ldy, p.residual,
                                            a.ldr, a.bias);
      N730_CUDA(cudaGetLastError());
    }
    b0 += nb;
  }
  return N730_OK;
}

}  // namespace n730
